/*
 * Minimal stand-in for the ggml header, just large enough to compile the
 * reference's header-only custom-op kernels (src/b1_0_kernel.h and
 * src/diffuser_types.h) unmodified.  It is test infrastructure for the CPU
 * oracle: it provides the tensor struct fields those kernels read
 * (ne, nb, src, data), IEEE fp16 -> fp32 conversion, and a ggml_custom_4d
 * that only records the node (the bridge in ref_bridge.cpp runs the
 * callback itself on a thread pool, as ggml's CPU backend does).
 * The real ggml lives in the reference's empty llama.cpp submodule.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_N_TASKS_MAX (-1)

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_I8 = 24 };

struct ggml_context;  // opaque; never dereferenced by the kernels

struct ggml_tensor {
  enum ggml_type type;
  int64_t ne[GGML_MAX_DIMS];
  size_t nb[GGML_MAX_DIMS];
  struct ggml_tensor* src[GGML_MAX_SRC];
  void* data;
};

typedef void (*ggml_custom_op_t)(struct ggml_tensor* dst, int ith, int nth, void* userdata);

static inline int64_t ggml_nelements(const struct ggml_tensor* t) {
  return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
}
static inline size_t ggml_nbytes(const struct ggml_tensor* t) {
  return (size_t)ggml_nelements(t) * (t->type == GGML_TYPE_F32 ? 4 : t->type == GGML_TYPE_F16 ? 2 : 1);
}

/* IEEE-754 binary16 -> binary32, exact for every input (subnormals, inf, nan). */
static inline float ggml_fp16_to_fp32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Records nothing: the oracle bridge invokes the callback directly. */
static inline struct ggml_tensor* ggml_custom_4d(struct ggml_context* ctx, enum ggml_type type,
                                                 int64_t ne0, int64_t ne1, int64_t ne2,
                                                 int64_t ne3, struct ggml_tensor** args,
                                                 int n_args, ggml_custom_op_t fun, int n_tasks,
                                                 void* userdata) {
  (void)ctx; (void)type; (void)ne0; (void)ne1; (void)ne2; (void)ne3;
  (void)args; (void)n_args; (void)fun; (void)n_tasks; (void)userdata;
  return NULL;
}
