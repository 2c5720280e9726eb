// Bridge that exposes the reference's own CPU kernels, compiled from the
// reference sources where they lie (src/b1_0_kernel.h, src/diffuser_types.h,
// included through -I), as plain C functions for the oracle and the CPU
// baseline.  It plays the role of ggml's CPU backend for these two custom
// ops: the callback is run once per worker with (ith, nth), exactly as
// ggml_backend_graph_compute does for a custom node (src/diffuser.cpp:269).
// Test infrastructure only: never linked into the product library.
#include "diffuser_types.h"
#include "b1_0_kernel.h"

#include <thread>
#include <vector>

namespace bonsai {
bool g_bonsai_debug = false;  // defined by the reference's drivers (src/diffuser.cpp:21-23)
}

namespace {
void run_threads(ggml_custom_op_t fn, ggml_tensor* dst, int nth, void* ud) {
  if (nth <= 1) {
    fn(dst, 0, 1, ud);
    return;
  }
  std::vector<std::thread> ts;
  ts.reserve(nth);
  for (int i = 0; i < nth; ++i) ts.emplace_back(fn, dst, i, nth, ud);
  for (auto& t : ts) t.join();
}
}  // namespace

extern "C" {

// out[t][r] for act f32 [tokens][in_dim], w = packed [out_dim][in_dim/32][6].
// Calls bonsai::b1_linear_f32_f32 (src/b1_0_kernel.h:37-288) with the tensor
// shapes b1_linear() builds (src/b1_0_kernel.h:290-300).
void ref_b1_linear(const float* act, int tokens, int in_dim, const uint8_t* w, int out_dim,
                   float* out, int nthreads) {
  ggml_tensor a{}, wt{}, dst{};
  a.type = GGML_TYPE_F32;
  a.ne[0] = in_dim; a.ne[1] = tokens; a.ne[2] = 1; a.ne[3] = 1;
  a.data = const_cast<float*>(act);
  wt.type = GGML_TYPE_I8;
  wt.ne[0] = (int64_t)out_dim * (in_dim / 32) * 6; wt.ne[1] = 1; wt.ne[2] = 1; wt.ne[3] = 1;
  wt.data = const_cast<uint8_t*>(w);
  dst.type = GGML_TYPE_F32;
  dst.ne[0] = out_dim; dst.ne[1] = tokens; dst.ne[2] = 1; dst.ne[3] = 1;
  dst.src[0] = &a;
  dst.src[1] = &wt;
  dst.data = out;
  bonsai::B1LinearUserData ud;
  ud.in_dim = in_dim;
  ud.out_dim = out_dim;
  run_threads(bonsai::b1_linear_f32_f32, &dst, nthreads, &ud);
}

// rope_2d_fwd_f32 (src/b1_0_kernel.h:309-361): x/out f32 [seq][n_heads][head_dim],
// cos/sin f32 [seq][head_dim/2].
void ref_rope_2d(const float* x, const float* c, const float* s, int head_dim, int n_heads,
                 int seq, float* out, int nthreads) {
  ggml_tensor xt{}, ct{}, st{}, dst{};
  xt.type = ct.type = st.type = dst.type = GGML_TYPE_F32;
  xt.data = const_cast<float*>(x);
  ct.data = const_cast<float*>(c);
  st.data = const_cast<float*>(s);
  dst.ne[0] = head_dim; dst.ne[1] = n_heads; dst.ne[2] = seq; dst.ne[3] = 1;
  dst.src[0] = &xt; dst.src[1] = &ct; dst.src[2] = &st;
  dst.data = out;
  bonsai::Rope2DUserData ud;
  ud.head_dim = head_dim;
  ud.n_heads = n_heads;
  ud.seq = seq;
  run_threads(bonsai::rope_2d_fwd_f32, &dst, nthreads, &ud);
}

int ref_has_avx2(void) {
#ifdef __AVX2__
  return 1;
#else
  return 0;
#endif
}
}
