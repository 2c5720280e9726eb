// Edge ops of the step that sit outside the B1_0 path: the f32 dense
// linears of the embedders, time / vector MLPs, shared modulation and the
// output head (ggml_mul_mat with f32 weights, src/diffuser_graph.cpp:283-320,
// :544-556), plus small elementwise helpers.  They are < 1% of the step's
// FLOPs; the dense linear is a plain SIMT tiled kernel (f32 accumulate).
#include "internal.cuh"
#include "vae.cuh"
#include "bonsai_cuda.h"

#define RC_EDGE(x)       \
  do {                   \
    int _rc = (x);       \
    if (_rc) return _rc; \
  } while (0)

#include <algorithm>

namespace bonsai {
namespace edge {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// y[o] = sum_i W[o][i] x[i] (+ b[o]); one warp per output row (coalesced W).
__global__ void gemv_kernel(const float* __restrict__ x, const float* __restrict__ W,
                            const float* __restrict__ b, int K, int N, float* __restrict__ y,
                            int act_silu_in) {
  const int warps = blockDim.x / 32;
  const int o = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (o >= N) return;
  const float* wr = W + (size_t)o * K;
  float s = 0.f;
  if ((K & 3) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(wr);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = lane; i < K / 4; i += 32) {
      const float4 a = w4[i];
      float4 v = x4[i];
      if (act_silu_in) {
        v.x = v.x / (1.f + expf(-v.x)); v.y = v.y / (1.f + expf(-v.y));
        v.z = v.z / (1.f + expf(-v.z)); v.w = v.w / (1.f + expf(-v.w));
      }
      s += (a.x * v.x + a.y * v.y) + (a.z * v.z + a.w * v.w);
    }
  } else {
    for (int i = lane; i < K; i += 32) {
      float v = x[i];
      if (act_silu_in) v = v / (1.f + expf(-v));
      s += wr[i] * v;
    }
  }
  s = warp_sum(s);
  if (lane == 0) y[o] = s + (b ? b[o] : 0.f);
}

// Tiled y[t][o] = sum_i W[o][i] x[t][i] (+ b[o]); 64 x 64 tile, 4 x 4 per thread.
constexpr int TB = 64, TK = 16;
__global__ void __launch_bounds__(256) linear_kernel(const float* __restrict__ x, long long ldx,
                                                     int T, int K, const float* __restrict__ W,
                                                     const float* __restrict__ b, int N,
                                                     float* __restrict__ y, long long ldy) {
  __shared__ float xs[TK][TB + 4];
  __shared__ float ws[TK][TB + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int t0 = blockIdx.y * TB, o0 = blockIdx.x * TB;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TB * TK; i += 256) {
      const int r = i / TK, c = i % TK;
      const int t = t0 + r, o = o0 + r, kk = k0 + c;
      xs[c][r] = (t < T && kk < K) ? x[(size_t)t * ldx + kk] : 0.f;
      ws[c][r] = (o < N && kk < K) ? W[(size_t)o * K + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < TK; ++c) {
      float xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xv[i] = xs[c][ty * 4 + i];
        wv[i] = ws[c][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += xv[i] * wv[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int o = o0 + tx * 4 + j;
      if (o < N) y[(size_t)t * ldy + o] = acc[i][j] + (b ? b[o] : 0.f);
    }
  }
}

// Larger tiled f32 linear for the big edge GEMMs: 128 x 128 outputs per
// 256-thread block, 8 x 8 per thread, k-slices of 8 double-buffered in SMEM.
constexpr int LB = 128, LK = 8;
// blockIdx.z selects a K slice [z*kspan, (z+1)*kspan) whose partial sum goes to
// y + z * zstride (bias only from slice 0 when it writes the final output).
__global__ void __launch_bounds__(256) linear128_kernel(const float* __restrict__ x,
                                                        long long ldx, int T, int K,
                                                        const float* __restrict__ W,
                                                        const float* __restrict__ b, int N,
                                                        float* __restrict__ y, long long ldy,
                                                        int kspan, long long zstride) {
  __shared__ __align__(16) float xs[2][LK][LB];
  __shared__ __align__(16) float ws[2][LK][LB];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int t0 = blockIdx.y * LB, o0 = blockIdx.x * LB;
  // loader mapping: thread -> (row = tid / 2, k4 = (tid % 2) * 4)
  const int lr = tid >> 1, lk = (tid & 1) * 4;
  const int Kfull = K;  // row stride of W
  const int kb = blockIdx.z * kspan;
  K = min(K, kb + kspan);  // this block's slice is [kb, K)
  y += blockIdx.z * zstride;
  // The next k-tile is fetched into registers before the current one is
  // multiplied and stored to shared memory after it, so the global-load
  // latency overlaps the FMAs.
  float rx[4], rw[4];
  auto fetch = [&](int k0) {
    const int t = t0 + lr, o = o0 + lr;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = k0 + lk + u;
      rx[u] = (t < T && kk < K) ? x[(size_t)t * ldx + kk] : 0.f;
      rw[u] = (o < N && kk < K) ? W[(size_t)o * Kfull + kk] : 0.f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      xs[buf][lk + u][lr] = rx[u];
      ws[buf][lk + u][lr] = rw[u];
    }
  };
  float acc[8][8] = {};
  fetch(kb);
  stash(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = kb; k0 < K; k0 += LK) {
    const bool more = k0 + LK < K;
    if (more) fetch(k0 + LK);
#pragma unroll
    for (int c = 0; c < LK; ++c) {
      const float4 a0 = *reinterpret_cast<const float4*>(&xs[buf][c][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&xs[buf][c][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&ws[buf][c][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&ws[buf][c][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) stash(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + ty * 8 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int o = o0 + tx * 8 + j;
      if (o < N) y[(size_t)t * ldy + o] = acc[i][j] + (b ? b[o] : 0.f);
    }
  }
}

// y[t][o] = sum_z part[z][t][o] + b[o] (fixed order: deterministic).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int T, int N,
                                     const float* __restrict__ b, float* __restrict__ y,
                                     long long ldy) {
  const long long n = (long long)T * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int z = 0; z < splits; ++z) acc += part[z * n + i];
    const int t = (int)(i / N), o = (int)(i % N);
    y[(size_t)t * ldy + o] = acc + (b ? b[o] : 0.f);
  }
}

__global__ void silu_kernel(const float* __restrict__ x, long long n, float* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = x[i] / (1.f + expf(-x[i]));
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, long long n,
                           float* __restrict__ y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = a[i] + b[i];
}

// Non-finite values (NaN or +-Inf) in x, one atomic per warp.
__global__ void count_nonfinite_kernel(const float* __restrict__ x, long long n,
                                       unsigned long long* __restrict__ count) {
  unsigned int mine = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    mine += isfinite(x[i]) ? 0u : 1u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((threadIdx.x & 31) == 0 && mine) atomicAdd(count, (unsigned long long)mine);
}

// One Euler step of the reference's sampler (src/diffuser.cpp:290-291):
// lat += dt * pred, plus the per-step diagnostics it prints (:276-288):
// stats = {NaN count, Inf count, min, max, mean} of pred, min/max over the
// non-NaN values.  One CTA of kEulerThreads; deterministic reduction order.
constexpr int kEulerThreads = 1024;
__global__ void __launch_bounds__(kEulerThreads)
    euler_stats_kernel(float* __restrict__ lat, const float* __restrict__ pred, long long n,
                       float dt, float* __restrict__ stats) {
  __shared__ float s_min[kEulerThreads / 32], s_max[kEulerThreads / 32], s_sum[kEulerThreads / 32];
  __shared__ unsigned int s_nan[kEulerThreads / 32], s_inf[kEulerThreads / 32];
  unsigned int nan_c = 0, inf_c = 0;
  float mn = INFINITY, mx = -INFINITY, sum = 0.0f;
  for (long long i = threadIdx.x; i < n; i += kEulerThreads) {
    const float v = pred[i];
    if (isnan(v)) ++nan_c;
    else if (isinf(v)) ++inf_c;
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
    sum += v;
    lat[i] = __fadd_rn(lat[i], __fmul_rn(dt, v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nan_c += __shfl_xor_sync(0xffffffffu, nan_c, o);
    inf_c += __shfl_xor_sync(0xffffffffu, inf_c, o);
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    s_nan[w] = nan_c;
    s_inf[w] = inf_c;
    s_min[w] = mn;
    s_max[w] = mx;
    s_sum[w] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kEulerThreads / 32; ++k) {
      nan_c += s_nan[k];
      inf_c += s_inf[k];
      mn = fminf(mn, s_min[k]);
      mx = fmaxf(mx, s_max[k]);
      sum += s_sum[k];
    }
    stats[0] = (float)nan_c;
    stats[1] = (float)inf_c;
    stats[2] = mn;
    stats[3] = mx;
    stats[4] = n > 0 ? sum / (float)n : 0.0f;
  }
}

// x [M][K] (leading dimension ldx) -> out [M][3K] bf16: with hi = bf16(x),
// lo = bf16(x - hi), activations as [hi | hi | lo] (weights = false) and
// weights as [hi | lo | hi] (weights = true), so that one GEMM over 3K
// accumulates x_hi w_hi + x_hi w_lo + x_lo w_hi.
__global__ void split_bf16x3_kernel(const float* __restrict__ x, long long ldx, int M, int K,
                                    int weights, __nv_bfloat16* __restrict__ out) {
  const int k4n = K / 4;
  const long long total = (long long)M * k4n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / k4n;
    const int k = (int)(i - m * k4n) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + m * ldx + k);
    const float f[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hi[j] = __float2bfloat16_rn(f[j]);
      lo[j] = __float2bfloat16_rn(f[j] - __bfloat162float(hi[j]));
    }
    __nv_bfloat16* o = out + m * 3LL * K + k;
    const uint2 h2 = *reinterpret_cast<const uint2*>(hi);
    const uint2 l2 = *reinterpret_cast<const uint2*>(lo);
    *reinterpret_cast<uint2*>(o) = h2;
    *reinterpret_cast<uint2*>(o + K) = weights ? l2 : h2;
    *reinterpret_cast<uint2*>(o + 2 * K) = weights ? h2 : l2;
  }
}

}  // namespace edge

int launch_split_bf16x3(const float* x, long long ldx, int M, int K, bool weights,
                        __nv_bfloat16* out, cudaStream_t st) {
  if (M <= 0) return 0;
  if (K % 8 != 0 || ldx % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return fail(BONSAI_ERR_ARG, "split_bf16x3: K % 8, ldx % 4 and 16-byte rows required");
  const long long work = (long long)M * (K / 4);
  const int blocks = (int)std::max<long long>(1, std::min<long long>((work + 255) / 256, (long long)num_sms() * 8));
  edge::split_bf16x3_kernel<<<blocks, 256, 0, st>>>(x, ldx, M, K, weights ? 1 : 0, out);
  return launch_status("split_bf16x3_kernel launch");
}

int launch_linear_bf16x3(const float* x, long long ldx, int M, int K, const __nv_bfloat16* w3,
                         const float* bias, int N, float* y, long long ldy, __nv_bfloat16* a3,
                         cudaStream_t st) {
  if (M <= 0) return 0;
  RC_EDGE(launch_split_bf16x3(x, ldx, M, K, false, a3, st));
  VaeConvArgs a;
  a.in = a3;
  a.ld_in = 3LL * K;
  a.H = 1;
  a.W = M;
  a.cin = 3 * K;
  a.bf16 = true;
  a.taps = 1;
  a.w = w3;
  a.w_ld = 3LL * K;
  a.N = N;
  a.bias = bias;
  a.out = y;
  a.ld_out = ldy;
  a.out_mode = VOUT_F32;
  a.prof_name = "edge_linear_bf16x3";
  return launch_vae_conv(a, st);
}

int launch_linear_f32(const float* x, long long ldx, int T, int K, const float* W, const float* b,
                      int N, float* y, long long ldy, bool silu_in, cudaStream_t st,
                      float* workspace, long long workspace_elems) {
  if (T == 0 || N == 0) return 0;
  if (T == 1) {
    const int wpb = 8;
    edge::gemv_kernel<<<(N + wpb - 1) / wpb, wpb * 32, 0, st>>>(x, W, b, K, N, y, silu_in ? 1 : 0);
    return launch_status("gemv launch");
  }
  if (silu_in) return fail(-2, "linear_f32: silu input only supported for T == 1");
  ProfScope prof("linear_f32", 2.0 * T * N * (double)K, 4.0 * ((double)T * K + (double)N * K + (double)T * N), st);
  // 128x128 tiles for large outputs, and for small ones whenever a split-K
  // workspace lets the grid grow (e.g. the 64-wide output projection).
  if ((long long)T * N >= 64LL * 128 * 128 || workspace) {
    dim3 grid((N + edge::LB - 1) / edge::LB, (T + edge::LB - 1) / edge::LB);
    // Split K so that the grid covers the GPU twice, when a workspace for the
    // partial sums is available (deterministic reduction afterwards).
    int splits = 1;
    const long long blocks = (long long)grid.x * grid.y;
    while (splits < 8 && blocks * splits < 2LL * num_sms() && K / (splits * 2) >= 256 &&
           workspace && (long long)(splits * 2) * T * N <= workspace_elems)
      splits *= 2;
    if (splits > 1) {
      const int kspan = (((K + splits - 1) / splits) + edge::LK - 1) / edge::LK * edge::LK;
      grid.z = splits;
      edge::linear128_kernel<<<grid, 256, 0, st>>>(x, ldx, T, K, W, nullptr, N, workspace, N,
                                                   kspan, (long long)T * N);
      int rc = launch_status("linear_f32 split-K launch");
      if (rc) return rc;
      const long long n = (long long)T * N;
      edge::splitk_reduce_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 4096), 256, 0, st>>>(
          workspace, splits, T, N, b, y, ldy);
      return launch_status("linear_f32 split-K reduce");
    }
    edge::linear128_kernel<<<grid, 256, 0, st>>>(x, ldx, T, K, W, b, N, y, ldy, K, 0);
  } else {
    dim3 grid((N + edge::TB - 1) / edge::TB, (T + edge::TB - 1) / edge::TB);
    edge::linear_kernel<<<grid, 256, 0, st>>>(x, ldx, T, K, W, b, N, y, ldy);
  }
  return launch_status("linear_f32 launch");
}

int launch_silu_f32(const float* x, long long n, float* y, cudaStream_t st) {
  if (n == 0) return 0;
  const long long blocks = std::min<long long>((n + 255) / 256, 4096);
  edge::silu_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, y);
  return launch_status("silu launch");
}

int launch_add_f32(const float* a, const float* b, long long n, float* y, cudaStream_t st) {
  if (n == 0) return 0;
  const long long blocks = std::min<long long>((n + 255) / 256, 4096);
  edge::add_kernel<<<(unsigned)blocks, 256, 0, st>>>(a, b, n, y);
  return launch_status("add launch");
}

int launch_count_nonfinite(const float* x, long long n, unsigned long long* dev_count,
                           cudaStream_t st) {
  if (n <= 0) return 0;
  const long long blocks = std::min<long long>((n + 255) / 256, (long long)num_sms() * 8);
  edge::count_nonfinite_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, dev_count);
  return launch_status("count_nonfinite launch");
}

int launch_euler_stats(float* lat, const float* pred, long long n, float dt, float* stats,
                       cudaStream_t st) {
  edge::euler_stats_kernel<<<1, edge::kEulerThreads, 0, st>>>(lat, pred, n, dt, stats);
  return launch_status("euler_stats launch");
}

}  // namespace bonsai
