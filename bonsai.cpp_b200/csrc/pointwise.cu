// HBM-bound pointwise / row kernels of the diffuser step.  Each is one pass
// over its tensors (read once, write once); rows are handled by one warp
// with 16-byte vector accesses.
#include "internal.cuh"
#include "ptx.cuh"

#include <algorithm>
#include <cmath>

namespace bonsai {
namespace pw {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------- LN-modulate
// y = LayerNorm(x; eps, no affine) * (1 + scale) + shift      (ggml_norm +
// mul/add chain, src/diffuser_graph.cpp:347-352).  Two-pass statistics on a
// register-resident row: mean, then variance of (x - mean).
template <int VPL, typename OutT>
__global__ void ln_modulate_kernel(const float* __restrict__ x, int rows, int dim,
                                   const float* __restrict__ shift,
                                   const float* __restrict__ scale, float eps, OutT* __restrict__ y,
                                   long long ld_y) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * dim);
  const int n4 = dim / 4;
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + i * 32;
    v[i] = idx < n4 ? xr[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(s) / dim;
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + i * 32;
    if (idx < n4) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      s2 += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float var = warp_sum(s2) / dim;
  const float rstd = 1.0f / sqrtf(var + eps);
  const float4* sh4 = reinterpret_cast<const float4*>(shift);
  const float4* sc4 = reinterpret_cast<const float4*>(scale);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + i * 32;
    if (idx >= n4) continue;
    const float4 sh = sh4[idx], sc = sc4[idx];
    float o0 = ((v[i].x - mean) * rstd) * (sc.x + 1.0f) + sh.x;
    float o1 = ((v[i].y - mean) * rstd) * (sc.y + 1.0f) + sh.y;
    float o2 = ((v[i].z - mean) * rstd) * (sc.z + 1.0f) + sh.z;
    float o3 = ((v[i].w - mean) * rstd) * (sc.w + 1.0f) + sh.w;
    if constexpr (sizeof(OutT) == 2) {
      __half2 a = __floats2half2_rn(o0, o1), b = __floats2half2_rn(o2, o3);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&a);
      pk.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(y + (size_t)row * ld_y + idx * 4) = pk;
    } else {
      *reinterpret_cast<float4*>(y + (size_t)row * ld_y + idx * 4) = make_float4(o0, o1, o2, o3);
    }
  }
}

// One 128-thread block per row: each thread keeps VPT float4 of the row in
// registers (dim <= 512 * VPT), block-wide two-pass statistics.  Small
// per-thread state lets 16 rows per SM be in flight, which the one-warp-
// per-row form above cannot reach for dim = 3072.
template <int VPT, typename OutT>
__global__ void __launch_bounds__(128) ln_modulate_block_kernel(
    const float* __restrict__ x, int rows, int dim, const float* __restrict__ shift,
    const float* __restrict__ scale, float eps, OutT* __restrict__ y, long long ld_y,
    const PeerCopies copies) {
  __shared__ float red[2][4];
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * dim);
  const int n4 = dim / 4;
  float4 v[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = tid + i * 128;
    v[i] = idx < n4 ? xr[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  if (lane == 0) red[0][wid] = s;
  __syncthreads();
  const float mean = ((red[0][0] + red[0][1]) + (red[0][2] + red[0][3])) / dim;
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = tid + i * 128;
    if (idx < n4) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      s2 += (a * a + b * b) + (c * c + d * d);
    }
  }
  s2 = warp_sum(s2);
  if (lane == 0) red[1][wid] = s2;
  __syncthreads();
  const float var = ((red[1][0] + red[1][1]) + (red[1][2] + red[1][3])) / dim;
  const float rstd = 1.0f / sqrtf(var + eps);
  const float4* sh4 = reinterpret_cast<const float4*>(shift);
  const float4* sc4 = reinterpret_cast<const float4*>(scale);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = tid + i * 128;
    if (idx >= n4) continue;
    const float4 sh = sh4[idx], sc = sc4[idx];
    const float o0 = ((v[i].x - mean) * rstd) * (sc.x + 1.0f) + sh.x;
    const float o1 = ((v[i].y - mean) * rstd) * (sc.y + 1.0f) + sh.y;
    const float o2 = ((v[i].z - mean) * rstd) * (sc.z + 1.0f) + sh.z;
    const float o3 = ((v[i].w - mean) * rstd) * (sc.w + 1.0f) + sh.w;
    if constexpr (sizeof(OutT) == 2) {
      __half2 a = __floats2half2_rn(o0, o1), b = __floats2half2_rn(o2, o3);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&a);
      pk.y = *reinterpret_cast<uint32_t*>(&b);
      const size_t off = (size_t)row * ld_y + idx * 4;
      *reinterpret_cast<uint2*>(y + off) = pk;
#pragma unroll
      for (int k = 0; k < kMaxPeers - 1; ++k)  // static indices: the copies stay in parameter space
        if (k < copies.n) *reinterpret_cast<uint2*>(copies.y[k] + off) = pk;
    } else {
      *reinterpret_cast<float4*>(y + (size_t)row * ld_y + idx * 4) = make_float4(o0, o1, o2, o3);
    }
  }
  if (copies.n > 0) __threadfence_system();  // peer stores ordered before the kernel's end
}

// Generic (any dim) three-pass version for rows that do not fit registers.
template <typename OutT>
__global__ void ln_modulate_generic_kernel(const float* __restrict__ x, int rows, int dim,
                                           const float* __restrict__ shift,
                                           const float* __restrict__ scale, float eps,
                                           OutT* __restrict__ y, long long ld_y) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * dim;
  float s = 0.f;
  for (int i = lane; i < dim; i += 32) s += xr[i];
  const float mean = warp_sum(s) / dim;
  float s2 = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float a = xr[i] - mean;
    s2 += a * a;
  }
  const float rstd = 1.0f / sqrtf(warp_sum(s2) / dim + eps);
  for (int i = lane; i < dim; i += 32) {
    const float o = ((xr[i] - mean) * rstd) * (scale[i] + 1.0f) + shift[i];
    if constexpr (sizeof(OutT) == 2)
      y[(size_t)row * ld_y + i] = __float2half_rn(o);
    else
      y[(size_t)row * ld_y + i] = o;
  }
}

// ------------------------------------------------ Q/K RMSNorm + RoPE (f16)
// In place on head-major [n_heads][seq][128] f16 q and k: per (head, token)
// row, x / sqrt(mean(x^2) + eps) * w (rms_norm_qk, src/diffuser_graph.cpp:71-79)
// followed by the pair rotation of rope_2d_fwd_f32 (src/b1_0_kernel.h:339-352).
// Tokens < split use the *_lo weights (text stream of a double block).
// One warp per (tensor, token, group of 8 heads): half-warp h takes heads
// h0 + h, h0 + h + 2, ..., 16 lanes per row with 8 elements (16 bytes) each,
// all four rows' loads in flight before the first reduction.
constexpr int QK_HEADS_PER_WARP = 8;
__global__ void qk_norm_rope_kernel(__half* __restrict__ q, __half* __restrict__ k, int n_heads,
                                    int seq, const float* __restrict__ wq_lo,
                                    const float* __restrict__ wq_hi,
                                    const float* __restrict__ wk_lo,
                                    const float* __restrict__ wk_hi, int split, float eps,
                                    const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t) {
  // work item = (tensor, head group, token); token fastest so neighbouring
  // warps share cos/sin rows in L1/L2.
  const int warps = blockDim.x / 32;
  const long long gw = (long long)blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int groups = (n_heads + QK_HEADS_PER_WARP - 1) / QK_HEADS_PER_WARP;
  const long long per_tensor = (long long)groups * seq;
  const long long total = k ? 2 * per_tensor : per_tensor;
  if (gw >= total) return;
  const bool is_k = gw >= per_tensor;
  const long long r = is_k ? gw - per_tensor : gw;
  const int t = (int)(r % seq);
  const int h0 = (int)(r / seq) * QK_HEADS_PER_WARP + half;
  __half* base = (is_k ? k : q) + ((size_t)h0 * seq + t) * 128 + hl * 8;
  const size_t hstride = (size_t)2 * seq * 128;
  const float* w = is_k ? (t < split ? wk_lo : wk_hi) : (t < split ? wq_lo : wq_hi);
  constexpr int R = QK_HEADS_PER_WARP / 2;
  uint4 raw[R];
#pragma unroll
  for (int i = 0; i < R; ++i)
    raw[i] = h0 + 2 * i < n_heads ? *reinterpret_cast<const uint4*>(base + i * hstride)
                                  : make_uint4(0u, 0u, 0u, 0u);
  const float4 wa = *reinterpret_cast<const float4*>(w + hl * 8);
  const float4 wb = *reinterpret_cast<const float4*>(w + hl * 8 + 4);
  const float4 c4 = *reinterpret_cast<const float4*>(cos_t + (size_t)t * 64 + hl * 4);
  const float4 s4 = *reinterpret_cast<const float4*>(sin_t + (size_t)t * 64 + hl * 4);
  const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
  const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
  const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const uint32_t u[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    float x[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[e]));
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
    float ss = ((x[0] * x[0] + x[1] * x[1]) + (x[2] * x[2] + x[3] * x[3])) +
               ((x[4] * x[4] + x[5] * x[5]) + (x[6] * x[6] + x[7] * x[7]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);  // within the half-warp
    const float sc = 1.0f / sqrtf(ss / 128.0f + eps);
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x0 = (x[2 * e] * sc) * wv[2 * e], x1 = (x[2 * e + 1] * sc) * wv[2 * e + 1];
      const __half2 h = __floats2half2_rn(x0 * cv[e] - x1 * sv[e], x0 * sv[e] + x1 * cv[e]);
      o4[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (h0 + 2 * i < n_heads)
      *reinterpret_cast<uint4*>(base + i * hstride) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// --------------------------------------------------------- f32 drop-ins
// rope_2d_fwd_f32 (src/b1_0_kernel.h:309-361).
__global__ void rope_2d_f32_kernel(const float* __restrict__ x, const float* __restrict__ c,
                                   const float* __restrict__ s, int head_dim, int n_heads,
                                   int seq, float* __restrict__ out) {
  const int half = head_dim / 2;
  const long long total = (long long)seq * n_heads * half;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % half);
    const long long sh = i / half;
    const int t = (int)(sh / n_heads);
    const size_t e = (size_t)sh * head_dim + 2 * d;
    const float cv = c[(size_t)t * half + d], sv = s[(size_t)t * half + d];
    const float a = x[e], b = x[e + 1];
    out[e] = a * cv - b * sv;
    out[e + 1] = a * sv + b * cv;
  }
}

// ggml_rms_norm(eps) * w over rows (rms_norm_qk, src/diffuser_graph.cpp:71-79).
__global__ void rms_norm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    int rows, int dim, float eps, float* __restrict__ y) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * dim;
  float s = 0.f;
  for (int i = lane; i < dim; i += 32) s += xr[i] * xr[i];
  const float sc = 1.0f / sqrtf(warp_sum(s) / dim + eps);
  for (int i = lane; i < dim; i += 32) y[(size_t)row * dim + i] = (xr[i] * sc) * w[i];
}

// RoPE angle tables (build_rope_cos_sin, src/diffuser_graph.cpp:142-182):
// pair d -> (axis, freq) precomputed on the host; angle = ids[t][axis] * freq.
__global__ void rope_tables_kernel(const float* __restrict__ ids, int seq, int n_axes,
                                   const int* __restrict__ pair_axis,
                                   const float* __restrict__ pair_freq, int half,
                                   float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const long long total = (long long)seq * half;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % half);
    const int t = (int)(i / half);
    const float ang = pair_freq[d] * ids[(size_t)t * n_axes + pair_axis[d]];
    cos_out[i] = cosf(ang);
    sin_out[i] = sinf(ang);
  }
}

}  // namespace pw

static int row_grid(long long rows, int warps_per_block) {
  return (int)((rows + warps_per_block - 1) / warps_per_block);
}

template <typename OutT>
static int ln_mod_impl(const float* x, int rows, int dim, const float* shift, const float* scale,
                       float eps, OutT* y, long long ld_y, cudaStream_t st,
                       const PeerCopies& copies = PeerCopies()) {
  if (rows == 0) return 0;
  if (!x || !shift || !scale || !y || rows < 0 || dim <= 0 || ld_y < dim)
    return fail(-1, "ln_modulate: bad arguments");
  const int wpb = 8;
  const bool vec = (dim % 4 == 0) && (ld_y % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) |
                     reinterpret_cast<uintptr_t>(scale)) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & (sizeof(OutT) == 2 ? 7 : 15)) == 0;
  const int n4 = dim / 4;
  if (copies.n > 0) {
    bool ok = vec && n4 <= 6 * 128 && copies.n < kMaxPeers;
    for (int k = 0; k < copies.n && ok; ++k)
      ok = copies.y[k] && (reinterpret_cast<uintptr_t>(copies.y[k]) & 7) == 0;
    if (!ok) return fail(-1, "ln_modulate: peer copies need the vectorised row kernel (dim <= 3072)");
  }
  ProfScope prof("ln_modulate", 0.0, (double)rows * dim * (4 + sizeof(OutT) * (1 + copies.n)), st);
  if (vec && n4 <= 6 * 128)
    pw::ln_modulate_block_kernel<6, OutT><<<rows, 128, 0, st>>>(x, rows, dim, shift, scale, eps, y,
                                                                 ld_y, copies);
  else if (vec && n4 <= 24 * 32)
    pw::ln_modulate_kernel<24, OutT><<<row_grid(rows, wpb), wpb * 32, 0, st>>>(x, rows, dim, shift, scale, eps, y, ld_y);
  else if (vec && n4 <= 48 * 32)
    pw::ln_modulate_kernel<48, OutT><<<row_grid(rows, wpb), wpb * 32, 0, st>>>(x, rows, dim, shift, scale, eps, y, ld_y);
  else
    pw::ln_modulate_generic_kernel<OutT><<<row_grid(rows, wpb), wpb * 32, 0, st>>>(x, rows, dim, shift, scale, eps, y, ld_y);
  return launch_status("ln_modulate launch");
}

int launch_ln_modulate_f16(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, __half* y, long long ld_y,
                           cudaStream_t st) {
  return ln_mod_impl<__half>(x, rows, dim, shift, scale, eps, y, ld_y, st);
}
int launch_ln_modulate_f16_peers(const float* x, int rows, int dim, const float* shift,
                                 const float* scale, float eps, __half* y, long long ld_y,
                                 const PeerCopies& copies, cudaStream_t st) {
  return ln_mod_impl<__half>(x, rows, dim, shift, scale, eps, y, ld_y, st, copies);
}
int launch_ln_modulate_f32(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, float* y, long long ld_y,
                           cudaStream_t st) {
  return ln_mod_impl<float>(x, rows, dim, shift, scale, eps, y, ld_y, st);
}

int launch_qk_norm_rope(__half* q, __half* k, int n_heads, int seq, const float* wq_lo,
                        const float* wq_hi, const float* wk_lo, const float* wk_hi, int split,
                        float eps, const float* cos_t, const float* sin_t, cudaStream_t st) {
  if (seq == 0 || n_heads == 0) return 0;
  if (!q || !wq_lo || !wq_hi || !cos_t || !sin_t || (k && (!wk_lo || !wk_hi)))
    return fail(-1, "qk_norm_rope: null argument");
  const long long rows = (long long)n_heads * seq * (k ? 2 : 1);
  const long long items = (long long)((n_heads + pw::QK_HEADS_PER_WARP - 1) / pw::QK_HEADS_PER_WARP) *
                          seq * (k ? 2 : 1);
  const int wpb = 8;
  ProfScope prof("qk_norm_rope", 0.0, (double)rows * 128 * 4, st);
  pw::qk_norm_rope_kernel<<<row_grid(items, wpb), wpb * 32, 0, st>>>(
      q, k, n_heads, seq, wq_lo, wq_hi, wk_lo, wk_hi, split, eps, cos_t, sin_t);
  return launch_status("qk_norm_rope launch");
}

int launch_rope_2d_f32(const float* x, const float* c, const float* s, int head_dim, int n_heads,
                       int seq, float* out, cudaStream_t st) {
  const long long total = (long long)seq * n_heads * (head_dim / 2);
  if (total == 0) return 0;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 65535LL * 4);
  pw::rope_2d_f32_kernel<<<(unsigned)blocks, threads, 0, st>>>(x, c, s, head_dim, n_heads, seq, out);
  return launch_status("rope_2d_f32 launch");
}

int launch_rms_norm_f32(const float* x, const float* w, int rows, int dim, float eps, float* y,
                        cudaStream_t st) {
  if (rows == 0) return 0;
  const int wpb = 8;
  pw::rms_norm_f32_kernel<<<row_grid(rows, wpb), wpb * 32, 0, st>>>(x, w, rows, dim, eps, y);
  return launch_status("rms_norm_f32 launch");
}

int launch_rope_tables(const float* ids, int seq, int n_axes, const int* pair_axis_dev,
                       const float* pair_freq_dev, int half, float* cos_out, float* sin_out,
                       cudaStream_t st) {
  const long long total = (long long)seq * half;
  if (total == 0) return 0;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 65535LL * 4);
  pw::rope_tables_kernel<<<(unsigned)blocks, threads, 0, st>>>(ids, seq, n_axes, pair_axis_dev,
                                                               pair_freq_dev, half, cos_out, sin_out);
  return launch_status("rope_tables launch");
}

}  // namespace bonsai
