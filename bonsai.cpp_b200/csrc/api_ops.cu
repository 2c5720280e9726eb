// C ABI wrappers of the pointwise ops and of attention (include/bonsai_cuda.h).
#include "../../include/bonsai_cuda.h"
#include "internal.cuh"

#include <cmath>
#include <vector>

namespace bonsai {

void rope_pair_table(const int* axes_dim, int n_axes, float theta, int* pair_axis,
                     float* pair_freq) {
  int d = 0;
  for (int a = 0; a < n_axes; ++a)
    for (int j = 0; j < axes_dim[a] / 2; ++j, ++d) {
      const float scale = (float)(j * 2) / (float)axes_dim[a];
      pair_axis[d] = a;
      pair_freq[d] = 1.0f / powf(theta, scale);
    }
}

}  // namespace bonsai

using namespace bonsai;

static cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

int bonsai_count_nonfinite(const float* x, long long n, long long* count, void* stream) {
  if (!count || n < 0 || (n > 0 && !x)) return fail(BONSAI_ERR_ARG, "count_nonfinite: bad argument");
  *count = 0;
  if (n == 0) return 0;
  cudaStream_t st = S(stream);
  unsigned long long* d = nullptr;
  int rc = cuda_status(cudaMallocAsync(reinterpret_cast<void**>(&d), sizeof(*d), st),
                       "count_nonfinite: allocation");
  if (rc) return rc;
  unsigned long long h = 0;
  rc = cuda_status(cudaMemsetAsync(d, 0, sizeof(*d), st), "count_nonfinite: memset");
  if (!rc) rc = launch_count_nonfinite(x, n, d, st);
  if (!rc) rc = cuda_status(cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, st),
                            "count_nonfinite: copy");
  cudaFreeAsync(d, st);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(st), "count_nonfinite: synchronize");
  if (!rc) *count = (long long)h;
  return rc;
}

int bonsai_rope_2d_f32(const float* x, const float* cos_t, const float* sin_t, int head_dim,
                       int n_heads, int seq, float* out, void* stream) {
  if (seq == 0 || n_heads == 0) return 0;
  if (!x || !cos_t || !sin_t || !out) return fail(BONSAI_ERR_ARG, "rope_2d_f32: null tensor");
  if (head_dim <= 0 || (head_dim & 1) || n_heads < 0 || seq < 0)
    return fail(BONSAI_ERR_ARG, "rope_2d_f32: head_dim must be positive and even");
  return launch_rope_2d_f32(x, cos_t, sin_t, head_dim, n_heads, seq, out, S(stream));
}

int bonsai_rope_tables(const float* ids, int seq, int n_axes, const int* host_axes_dim,
                       float theta, float* cos_out, float* sin_out, void* stream) {
  if (seq == 0) return 0;
  if (!ids || !host_axes_dim || !cos_out || !sin_out || n_axes <= 0 || n_axes > 16 || seq < 0)
    return fail(BONSAI_ERR_ARG, "rope_tables: bad arguments");
  int half = 0;
  for (int a = 0; a < n_axes; ++a) {
    if (host_axes_dim[a] <= 0 || (host_axes_dim[a] & 1))
      return fail(BONSAI_ERR_ARG, "rope_tables: axes_dim entries must be positive and even");
    half += host_axes_dim[a] / 2;
  }
  std::vector<int> pa(half);
  std::vector<float> pf(half);
  rope_pair_table(host_axes_dim, n_axes, theta, pa.data(), pf.data());
  cudaStream_t st = S(stream);
  void* dev = nullptr;
  cudaError_t e = cudaMallocAsync(&dev, (size_t)half * 8, st);
  if (e != cudaSuccess) return fail(BONSAI_ERR_NOMEM, "rope_tables: table allocation failed");
  int* pa_d = static_cast<int*>(dev);
  float* pf_d = reinterpret_cast<float*>(pa_d + half);
  // Host vectors must outlive the async copy: copy synchronously w.r.t. the stream.
  e = cudaMemcpyAsync(pa_d, pa.data(), (size_t)half * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(pf_d, pf.data(), (size_t)half * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  int rc = (e == cudaSuccess) ? launch_rope_tables(ids, seq, n_axes, pa_d, pf_d, half, cos_out, sin_out, st)
                              : cuda_status(e, "rope_tables copy");
  cudaFreeAsync(dev, st);
  return rc;
}

int bonsai_linear_f32(const float* x, int tokens, int in_dim, const float* W, const float* bias,
                      int out_dim, float* y, void* stream) {
  if (tokens < 0 || in_dim <= 0 || out_dim < 0) return fail(BONSAI_ERR_ARG, "linear_f32: bad shape");
  if (tokens == 0 || out_dim == 0) return 0;
  if (!x || !W || !y) return fail(BONSAI_ERR_ARG, "linear_f32: null tensor");
  cudaStream_t st = S(stream);
  // Up to 8 partial sums of the output (the split-K limit of the kernel).
  const long long ws_elems = 8LL * tokens * out_dim;
  float* ws = nullptr;
  int rc = cuda_status(cudaMallocAsync(reinterpret_cast<void**>(&ws), (size_t)ws_elems * 4, st),
                       "linear_f32: workspace");
  if (rc) return rc;
  rc = launch_linear_f32(x, in_dim, tokens, in_dim, W, bias, out_dim, y, out_dim, false, st, ws,
                         ws_elems);
  cudaFreeAsync(ws, st);
  return rc;
}

int bonsai_rms_norm_f32(const float* x, const float* w, int rows, int head_dim, float eps,
                        float* out, void* stream) {
  if (rows == 0) return 0;
  if (!x || !w || !out || rows < 0 || head_dim <= 0) return fail(BONSAI_ERR_ARG, "rms_norm_f32: bad arguments");
  return launch_rms_norm_f32(x, w, rows, head_dim, eps, out, S(stream));
}

int bonsai_ln_modulate(const float* x, int rows, int dim, const float* shift, const float* scale,
                       float eps, uint16_t* y, long long ld_y, void* stream) {
  return launch_ln_modulate_f16(x, rows, dim, shift, scale, eps, reinterpret_cast<__half*>(y),
                                ld_y, S(stream));
}

int bonsai_ln_modulate_f32(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, float* y, void* stream) {
  return launch_ln_modulate_f32(x, rows, dim, shift, scale, eps, y, dim, S(stream));
}

int bonsai_joint_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int n_heads,
                           int seq, int head_dim, float scale, uint16_t* out, long long ld_out,
                           void* stream) {
  return launch_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                          reinterpret_cast<const __half*>(v), n_heads, seq, head_dim, scale,
                          reinterpret_cast<__half*>(out), ld_out, S(stream));
}

int bonsai_qk_norm_rope(uint16_t* qk, int n_heads, int seq, int head_dim, const float* w_lo,
                        const float* w_hi, int split, float eps, const float* cos_t,
                        const float* sin_t, void* stream) {
  if (head_dim != 128) return fail(BONSAI_ERR_UNSUPPORTED, "qk_norm_rope: head_dim must be 128");
  return launch_qk_norm_rope(reinterpret_cast<__half*>(qk), nullptr, n_heads, seq, w_lo, w_hi,
                             nullptr, nullptr, split, eps, cos_t, sin_t, S(stream));
}

}  // extern "C"
