/*
 * Minimal stand-in for the ggml header, just large enough to compile the
 * reference's header-only custom-op kernels (src/b1_0_kernel.h and
 * src/diffuser_types.h) unmodified.  It is test infrastructure for the CPU
 * oracle: it provides the tensor struct fields those kernels read
 * (ne, nb, src, data), IEEE fp16 -> fp32 conversion, and a ggml_custom_4d
 * that builds the custom node in a small fixed arena of the context -- its
 * shape, sources, callback, task count and user-data pointer, which real
 * ggml keeps among the node's op parameters -- or returns NULL without a
 * context (the bridge in ref_bridge.cpp runs the callbacks itself on a
 * thread pool, as ggml's CPU backend does).
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

typedef void (*ggml_custom_op_t)(struct ggml_tensor* dst, int ith, int nth, void* userdata);

struct ggml_tensor {
  enum ggml_type type;
  int64_t ne[GGML_MAX_DIMS];
  size_t nb[GGML_MAX_DIMS];
  struct ggml_tensor* src[GGML_MAX_SRC];
  void* data;
  /* custom-op parameters of a node made by ggml_custom_4d */
  ggml_custom_op_t op_fun;
  int op_n_tasks;
  void* op_userdata;
};

#define GGML_SHIM_MAX_NODES 64
struct ggml_context {
  struct ggml_tensor nodes[GGML_SHIM_MAX_NODES];
  int n_nodes;
};

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

/* The custom node: f32/f16 output of shape {ne0..ne3} with sources args,
 * whose data the caller provides; NULL without a context or when the arena
 * is full or n_args exceeds GGML_MAX_SRC. */
static inline struct ggml_tensor* ggml_custom_4d(struct ggml_context* ctx, enum ggml_type type,
                                                 int64_t ne0, int64_t ne1, int64_t ne2,
                                                 int64_t ne3, struct ggml_tensor** args,
                                                 int n_args, ggml_custom_op_t fun, int n_tasks,
                                                 void* userdata) {
  if (!ctx || ctx->n_nodes >= GGML_SHIM_MAX_NODES || n_args > GGML_MAX_SRC) return NULL;
  struct ggml_tensor* t = &ctx->nodes[ctx->n_nodes++];
  memset(t, 0, sizeof(*t));
  t->type = type;
  t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = ne2; t->ne[3] = ne3;
  for (int i = 0; i < n_args; ++i) t->src[i] = args[i];
  t->op_fun = fun;
  t->op_n_tasks = n_tasks;
  t->op_userdata = userdata;
  return t;
}
