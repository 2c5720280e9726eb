// A compiled caller of the C ABI, written the way a ggml backend of the
// reference would use it (test infrastructure: built by oracle/Makefile from
// the reference's own headers, run by tests/test_dropin_caller_gpu.py).
//
// The reference builds its custom ops with b1_linear() and rope_2d_fwd()
// (src/b1_0_kernel.h:290-300, :363-371): ggml_custom_4d nodes whose user data
// starts with a magic number that GPU backends match on (:32, :303).  Here
// those factory functions -- the reference's code, through the ggml shim in
// oracle/shim -- build the nodes, and a miniature CUDA backend dispatches each
// node by its magic to bonsai_b1_linear_f32 / bonsai_rope_2d_f32, the way a
// backend that replaces the two custom ops binds them.  The same nodes are then run through
// their own CPU callbacks (the reference's kernels, every (ith, nth) slice)
// and the two results compared:
//   B1_0 linear: cos >= 0.9999 and max-abs <= 1e-2 * RMS (the device rounds
//     the activations to f16; tests/c_ops/test_webgpu_ops.cpp:125-130);
//   RoPE: max-abs <= 1e-5 (tests/ops/test_all_ops.py:300-341).
// Prints one line per case and exits 0 when every case passes.
#include "diffuser_types.h"
#include "b1_0_kernel.h"

#include "bonsai_cuda.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <random>
#include <vector>

namespace bonsai {
bool g_bonsai_debug = false;  // defined by the reference's drivers (src/diffuser.cpp:21-23)
}

namespace {

#define CK(x)                                                                      \
  do {                                                                             \
    cudaError_t e_ = (x);                                                          \
    if (e_ != cudaSuccess) {                                                       \
      std::fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e_));         \
      std::exit(2);                                                                \
    }                                                                              \
  } while (0)

// Device copies of the host tensors a node reads and writes, and the B1_0
// weights uploaded once per ggml weight tensor (as a backend would at load
// time, next to load_b1: src/diffuser.cpp:39-50).
struct Backend {
  std::map<const ggml_tensor*, void*> dev;
  std::map<const ggml_tensor*, bonsai_b1_t> b1;

  ~Backend() {
    for (auto& kv : dev) cudaFree(kv.second);
    for (auto& kv : b1) bonsai_b1_free(kv.second);
  }
  void* upload(const ggml_tensor* t, size_t bytes) {
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes));
    CK(cudaMemcpy(p, t->data, bytes, cudaMemcpyHostToDevice));
    dev[t] = p;
    return p;
  }
  void* alloc(const ggml_tensor* t, size_t bytes) {
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes));
    dev[t] = p;
    return p;
  }
  int add_b1(const ggml_tensor* w, int out_dim, int in_dim) {
    bonsai_b1_t h = nullptr;
    const int rc = bonsai_b1_upload(static_cast<const uint8_t*>(w->data), out_dim, in_dim, -1, &h);
    if (rc) return rc;
    b1[w] = h;
    return 0;
  }

  // The node loop of the backend: dispatch on the user data's magic.
  int compute(ggml_tensor* node, float* host_out) {
    const int magic = *static_cast<const int*>(node->op_userdata);
    void* stream = nullptr;  // the legacy stream
    if (magic == BONSAI_B1_MAGIC) {
      const auto* ud = static_cast<const bonsai::B1LinearUserData*>(node->op_userdata);
      const ggml_tensor* act = node->src[0];
      const int tokens = (int)act->ne[1];
      const float* x = static_cast<const float*>(upload(act, sizeof(float) * act->ne[0] * tokens));
      float* y = static_cast<float*>(alloc(node, sizeof(float) * (size_t)ud->out_dim * tokens));
      const int rc = bonsai_b1_linear_f32(x, tokens, b1.at(node->src[1]), y, stream);
      if (rc) return rc;
      CK(cudaMemcpy(host_out, y, sizeof(float) * (size_t)ud->out_dim * tokens, cudaMemcpyDeviceToHost));
      return 0;
    }
    if (magic == BONSAI_ROPE_MAGIC) {
      const auto* ud = static_cast<const bonsai::Rope2DUserData*>(node->op_userdata);
      const size_t n = (size_t)ud->head_dim * ud->n_heads * ud->seq;
      const size_t nt = (size_t)(ud->head_dim / 2) * ud->seq;
      const float* x = static_cast<const float*>(upload(node->src[0], n * sizeof(float)));
      const float* c = static_cast<const float*>(upload(node->src[1], nt * sizeof(float)));
      const float* s = static_cast<const float*>(upload(node->src[2], nt * sizeof(float)));
      float* y = static_cast<float*>(alloc(node, n * sizeof(float)));
      const int rc = bonsai_rope_2d_f32(x, c, s, ud->head_dim, ud->n_heads, ud->seq, y, stream);
      if (rc) return rc;
      CK(cudaMemcpy(host_out, y, n * sizeof(float), cudaMemcpyDeviceToHost));
      return 0;
    }
    return BONSAI_ERR_UNSUPPORTED;
  }
};

// The node's own CPU callback over every (ith, nth) slice, as ggml's CPU
// backend runs it.
void run_cpu(ggml_tensor* node, int nth) {
  for (int ith = 0; ith < nth; ++ith) node->op_fun(node, ith, nth, node->op_userdata);
}

ggml_tensor host_tensor(ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, void* data) {
  ggml_tensor t;
  std::memset(&t, 0, sizeof(t));
  t.type = type;
  t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = 1;
  t.data = data;
  return t;
}

bool b1_case(int tokens, int in_dim, int out_dim, unsigned seed) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> nd(0.f, 1.f);
  std::uniform_int_distribution<int> byte(0, 255);
  const int nb = in_dim / 32;
  std::vector<float> act((size_t)tokens * in_dim);
  for (auto& v : act) v = nd(gen);
  std::vector<uint8_t> packed((size_t)out_dim * nb * 6);
  for (size_t g = 0; g < (size_t)out_dim * nb; ++g) {
    const _Float16 sc = (_Float16)std::fabs(nd(gen) * 0.02f);
    std::memcpy(&packed[g * 6], &sc, 2);
    for (int b = 2; b < 6; ++b) packed[g * 6 + b] = (uint8_t)byte(gen);
  }
  ggml_context ctx;
  ctx.n_nodes = 0;
  ggml_tensor a = host_tensor(GGML_TYPE_F32, in_dim, tokens, 1, act.data());
  ggml_tensor w = host_tensor(GGML_TYPE_I8, (int64_t)packed.size(), 1, 1, packed.data());
  bonsai::B1Weights bw;
  bw.data = &w;
  bw.in_dim = in_dim;
  bw.out_dim = out_dim;
  bonsai::B1LinearUserData ud;
  ggml_tensor* node = bonsai::b1_linear(&ctx, &a, bw, 4, ud);  // the reference's factory
  if (!node) return false;
  std::vector<float> gpu((size_t)tokens * out_dim), cpu((size_t)tokens * out_dim);
  Backend be;
  if (be.add_b1(&w, out_dim, in_dim) || be.compute(node, gpu.data())) {
    std::printf("b1 %dx%d->%d: bonsai call failed: %s\n", tokens, in_dim, out_dim, bonsai_last_error());
    return false;
  }
  node->data = cpu.data();
  run_cpu(node, node->op_n_tasks);
  double dot = 0, ng = 0, nr = 0, maxabs = 0, ss = 0;
  for (size_t i = 0; i < cpu.size(); ++i) {
    dot += (double)gpu[i] * cpu[i];
    ng += (double)gpu[i] * gpu[i];
    nr += (double)cpu[i] * cpu[i];
    maxabs = std::fmax(maxabs, std::fabs((double)gpu[i] - cpu[i]));
    ss += (double)cpu[i] * cpu[i];
  }
  const double cos = dot / std::sqrt(ng * nr), rel = maxabs / std::sqrt(ss / cpu.size());
  const bool ok = ud.magic == BONSAI_B1_MAGIC && cos >= 0.9999 && rel <= 1e-2;
  std::printf("b1 %dx%d->%d: cos=%.7f maxabs/rms=%.3e %s\n", tokens, in_dim, out_dim, cos, rel,
              ok ? "ok" : "FAIL");
  return ok;
}

bool rope_case(int head_dim, int n_heads, int seq, unsigned seed) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> nd(0.f, 1.f);
  std::uniform_real_distribution<float> ang(-3.14159f, 3.14159f);
  std::vector<float> x((size_t)head_dim * n_heads * seq), c((size_t)head_dim / 2 * seq),
      s((size_t)head_dim / 2 * seq);
  for (auto& v : x) v = nd(gen);
  for (size_t i = 0; i < c.size(); ++i) {
    const float a = ang(gen);
    c[i] = std::cos(a);
    s[i] = std::sin(a);
  }
  ggml_context ctx;
  ctx.n_nodes = 0;
  ggml_tensor xt = host_tensor(GGML_TYPE_F32, head_dim, n_heads, seq, x.data());
  ggml_tensor ct = host_tensor(GGML_TYPE_F32, head_dim / 2, seq, 1, c.data());
  ggml_tensor st = host_tensor(GGML_TYPE_F32, head_dim / 2, seq, 1, s.data());
  bonsai::Rope2DUserData ud;
  ud.head_dim = head_dim;
  ud.n_heads = n_heads;
  ud.seq = seq;
  ggml_tensor* node = bonsai::rope_2d_fwd(&ctx, &xt, &ct, &st, ud);  // the reference's factory
  if (!node) return false;
  std::vector<float> gpu(x.size()), cpu(x.size());
  Backend be;
  if (be.compute(node, gpu.data())) {
    std::printf("rope: bonsai call failed: %s\n", bonsai_last_error());
    return false;
  }
  node->data = cpu.data();
  run_cpu(node, 7);  // GGML_N_TASKS_MAX: as many workers as the pool has
  double maxabs = 0;
  for (size_t i = 0; i < cpu.size(); ++i) maxabs = std::fmax(maxabs, std::fabs((double)gpu[i] - cpu[i]));
  const bool ok = ud.magic == BONSAI_ROPE_MAGIC && maxabs <= 1e-5;
  std::printf("rope %dx%dx%d: maxabs=%.3e %s\n", head_dim, n_heads, seq, maxabs, ok ? "ok" : "FAIL");
  return ok;
}

}  // namespace

int main() {
  if (bonsai_init(0) != 0) {
    std::printf("bonsai_init failed: %s\n", bonsai_last_error());
    return 1;
  }
  bool ok = true;
  ok &= b1_case(1, 64, 32, 1);        // the reference's own unit-test shape
  ok &= b1_case(300, 3072, 1000, 2);  // ragged rows and tokens
  ok &= b1_case(512, 3072, 9216, 3);  // the text stream's fused QKV
  ok &= rope_case(128, 3, 50, 4);
  ok &= rope_case(128, 24, 333, 5);
  std::printf(ok ? "ALL OK\n" : "FAILED\n");
  return ok ? 0 : 1;
}
