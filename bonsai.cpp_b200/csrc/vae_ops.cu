// Memory-bound kernels of the Flux VAE decoder (src/vae_graph.cpp,
// src/vae_decoder.cpp): GroupNorm statistics and GroupNorm + SiLU
// application, nearest 2x upsampling, the latent preprocessing, the
// attention softmax, weight packing and seeded synthetic weights.  All work
// on NHWC tensors with vectorised 16-byte loads and grid-stride loops sized
// to the SM count.
#include "internal.cuh"
#include "vae.cuh"
#include "bonsai_cuda.h"

#include <algorithm>

namespace bonsai {
namespace vops {

__device__ __forceinline__ uint16_t to16(float v, bool bf) {
  return bf ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d, bool bf) {
  uint2 o;
  o.x = (uint32_t)to16(a, bf) | ((uint32_t)to16(b, bf) << 16);
  o.y = (uint32_t)to16(c, bf) | ((uint32_t)to16(d, bf) << 16);
  return o;
}

// Block b sums rows [b*rows_per_blk, ...) of x[pixels][C]: thread t owns the
// 4 channels (t % (C/4))*4.. of every (256 / (C/4))-th row; the 8 threads of
// a group (C/128 float4 columns x 1024/C row phases) are combined in f64.
__global__ void gn_stats_kernel(const float* __restrict__ x, long long pixels, int C,
                                long long rows_per_blk, double* __restrict__ part) {
  const int c4n = C / 4;
  const int rpp = 256 / c4n;
  const int col4 = threadIdx.x % c4n;
  const int r0 = threadIdx.x / c4n;
  const long long row_begin = (long long)blockIdx.x * rows_per_blk;
  const long long row_end = min(pixels, row_begin + rows_per_blk);
  double s = 0.0, ss = 0.0;
  for (long long r = row_begin + r0; r < row_end; r += rpp) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x + r * C) + col4);
    const float a = (v.x + v.y) + (v.z + v.w);
    const float b = fmaf(v.x, v.x, v.y * v.y) + fmaf(v.z, v.z, v.w * v.w);
    s += (double)a;
    ss += (double)b;
  }
  __shared__ double sh[2][256];
  sh[0][threadIdx.x] = s;
  sh[1][threadIdx.x] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    const int g = threadIdx.x;
    const int cpg4 = c4n / 32;
    double a = 0.0, b = 0.0;
    for (int r = 0; r < rpp; ++r)
      for (int k = 0; k < cpg4; ++k) {
        const int idx = r * c4n + g * cpg4 + k;
        a += sh[0][idx];
        b += sh[1][idx];
      }
    part[((long long)blockIdx.x * 32 + g) * 2] = a;
    part[((long long)blockIdx.x * 32 + g) * 2 + 1] = b;
  }
}

// Warp g folds group g's partials in a fixed order (deterministic).
__global__ void gn_finalize_kernel(const double* __restrict__ part, int nblk, double count,
                                   float eps, float* __restrict__ mean_rstd) {
  const int g = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  double a = 0.0, b = 0.0;
  for (int i = lane; i < nblk; i += 32) {
    a += part[((long long)i * 32 + g) * 2];
    b += part[((long long)i * 32 + g) * 2 + 1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (lane == 0) {
    const double mean = a / count;
    const double var = fmax(b / count - mean * mean, 0.0);
    mean_rstd[2 * g] = (float)mean;
    mean_rstd[2 * g + 1] = (float)(1.0 / sqrt(var + (double)eps));
  }
}

__global__ void gn_apply_kernel(const float* __restrict__ x, long long n4, int C,
                                const float* __restrict__ mean_rstd,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                int silu, uint2* __restrict__ y, int bf) {
  __shared__ float st[64];
  if (threadIdx.x < 64) st[threadIdx.x] = mean_rstd[threadIdx.x];
  __syncthreads();
  const int c4n = C / 4;
  const int cpg = C / 32;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % c4n) * 4;
    const int g = c / cpg;
    const float mean = st[2 * g], rstd = st[2 * g + 1];
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma + c));
    const float4 be = __ldg(reinterpret_cast<const float4*>(beta + c));
    float o[4] = {(v.x - mean) * rstd * ga.x + be.x, (v.y - mean) * rstd * ga.y + be.y,
                  (v.z - mean) * rstd * ga.z + be.z, (v.w - mean) * rstd * ga.w + be.w};
    if (silu) {
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = o[k] / (1.0f + __expf(-o[k]));
    }
    y[i] = pack4(o[0], o[1], o[2], o[3], bf != 0);
  }
}

__global__ void upsample2_kernel(const float* __restrict__ x, int H, int W, int C,
                                 uint2* __restrict__ y, int bf) {
  const int c4n = C / 4;
  const long long n4 = (long long)H * W * c4n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const int c4 = (int)(i % c4n);
    const long long pix = i / c4n;
    const int yy = (int)(pix / W), xx = (int)(pix % W);
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    const uint2 o = pack4(v.x, v.y, v.z, v.w, bf != 0);
    const long long W2 = 2LL * W;
    const long long base = ((2LL * yy) * W2 + 2LL * xx) * c4n + c4;
    y[base] = o;
    y[base + c4n] = o;
    y[base + W2 * c4n] = o;
    y[base + W2 * c4n + c4n] = o;
  }
}

__global__ void cast_kernel(const float* __restrict__ x, long long n4, uint2* __restrict__ y,
                            int bf) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    y[i] = pack4(v.x, v.y, v.z, v.w, bf != 0);
  }
}

__global__ void preprocess_kernel(const float* __restrict__ lat, int h, int w,
                                  const float* __restrict__ mean, const float* __restrict__ stdv,
                                  __half* __restrict__ y) {
  const long long total = 4LL * h * w * 64;
  const int W2 = 2 * w;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % 64);
    const long long pix = i / 64;
    float v = 0.0f;
    if (c < 32) {
      const int Y = (int)(pix / W2), X = (int)(pix % W2);
      const int sc = c * 4 + (Y & 1) * 2 + (X & 1);
      const float l = lat[((long long)sc * h + (Y >> 1)) * w + (X >> 1)];
      v = __fadd_rn(__fmul_rn(l, stdv[sc]), mean[sc]);
    }
    y[i] = __float2half_rn(v);
  }
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  const int nw = blockDim.x / 32;
  v = lane < nw ? sh[lane] : (is_max ? -INFINITY : 0.0f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  return v;
}

constexpr int kSoftmaxThreads = 256;
constexpr int kSoftmaxRegs4 = 16;  // float4 per thread held in registers (cols <= 16384)

__global__ void __launch_bounds__(kSoftmaxThreads)
    softmax_kernel(const float* __restrict__ S, long long ld_s, int cols, float scale,
                   __half* __restrict__ P, long long ld_p, float* __restrict__ rowinv, int fast) {
  __shared__ float sh[32];
  const long long r = blockIdx.x;
  const float* s = S + r * ld_s;
  __half* p = P + r * ld_p;
  const int tid = threadIdx.x;
  if (fast) {
    float4 v[kSoftmaxRegs4];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kSoftmaxRegs4; ++k) {
      const int c4 = tid + k * kSoftmaxThreads;
      if (c4 * 4 < cols) {
        v[k] = __ldg(reinterpret_cast<const float4*>(s) + c4);
        m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
      }
    }
    m = block_reduce(m, true, sh);
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kSoftmaxRegs4; ++k) {
      const int c4 = tid + k * kSoftmaxThreads;
      if (c4 * 4 < cols) {
        const float e0 = __expf(scale * (v[k].x - m)), e1 = __expf(scale * (v[k].y - m));
        const float e2 = __expf(scale * (v[k].z - m)), e3 = __expf(scale * (v[k].w - m));
        sum += (e0 + e1) + (e2 + e3);
        reinterpret_cast<uint2*>(p)[c4] = pack4(e0, e1, e2, e3, false);
      }
    }
    sum = block_reduce(sum, false, sh);
    if (tid == 0) rowinv[r] = 1.0f / sum;
    return;
  }
  float m = -INFINITY;
  for (int c = tid; c < cols; c += kSoftmaxThreads) m = fmaxf(m, s[c]);
  m = block_reduce(m, true, sh);
  float sum = 0.0f;
  for (int c = tid; c < cols; c += kSoftmaxThreads) {
    const float e = __expf(scale * (s[c] - m));
    sum += e;
    p[c] = __float2half_rn(e);
  }
  sum = block_reduce(sum, false, sh);
  if (tid == 0) rowinv[r] = 1.0f / sum;
}

__global__ void pack_weight_kernel(const float* __restrict__ src, int cout, int cin, int taps,
                                   long long total, int cin_pad, uint16_t* __restrict__ dst,
                                   int bf) {
  const long long per_row = (long long)taps * cin_pad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / per_row;
    const int rem = (int)(i - n * per_row);
    const int t = rem / cin_pad, c = rem % cin_pad;
    const float v = (n < cout && c < cin) ? src[(n * cin + c) * taps + t] : 0.0f;
    dst[i] = to16(v, bf != 0);
  }
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fill_kernel(float* __restrict__ dst, long long n, unsigned long long seed,
                            float mean, float stdv, int uniform) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const unsigned long long z = splitmix64(seed * 0x100000001B3ull + (unsigned long long)i);
    const float u2 = (float)(uint32_t)z * 2.3283064365386963e-10f;            // [0, 1)
    if (uniform) {
      dst[i] = mean + stdv * u2;
    } else {
      const float u1 = ((float)(uint32_t)(z >> 32) + 0.5f) * 2.3283064365386963e-10f;  // (0, 1)
      // Box-Muller transform.
      dst[i] = mean + stdv * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
  }
}

int grid_for(long long work, int threads) {
  const long long want = (work + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(want, (long long)num_sms() * 8));
}

}  // namespace vops

int launch_vae_gn_stats(const float* x, long long pixels, int C, double* partials,
                        float* mean_rstd, float eps, cudaStream_t st) {
  if (C < 128 || C > 1024 || (256 % (C / 4)) != 0 || pixels <= 0)
    return fail(BONSAI_ERR_ARG, "vae group norm: C must be 128, 256, 512 or 1024");
  const int rpp = 256 / (C / 4);
  const long long passes = (pixels + rpp - 1) / rpp;
  const int nblk = (int)std::min<long long>(passes, kGnMaxBlocks);
  const long long rows_per_blk = ((pixels + nblk - 1) / nblk + rpp - 1) / rpp * rpp;
  const int used = (int)((pixels + rows_per_blk - 1) / rows_per_blk);
  {
    ProfScope prof("vae_gn_stats", 0.0, (double)pixels * C * 4, st);
    vops::gn_stats_kernel<<<used, 256, 0, st>>>(x, pixels, C, rows_per_blk, partials);
  }
  if (int rc = launch_status("vae gn_stats_kernel launch")) return rc;
  vops::gn_finalize_kernel<<<1, 1024, 0, st>>>(partials, used, (double)pixels * (C / 32), eps,
                                               mean_rstd);
  return launch_status("vae gn_finalize_kernel launch");
}

int launch_vae_gn_apply(const float* x, long long pixels, int C, const float* mean_rstd,
                        const float* gamma, const float* beta, bool silu, void* y, bool y_bf16,
                        cudaStream_t st) {
  if (C % 32 != 0 || (C / 32) % 4 != 0) return fail(BONSAI_ERR_ARG, "vae group norm: C % 128");
  const long long n4 = pixels * C / 4;
  ProfScope prof("vae_gn_apply", 0.0, (double)pixels * C * 6, st);
  vops::gn_apply_kernel<<<vops::grid_for(n4, 256), 256, 0, st>>>(
      x, n4, C, mean_rstd, gamma, beta, silu ? 1 : 0, reinterpret_cast<uint2*>(y), y_bf16 ? 1 : 0);
  return launch_status("vae gn_apply_kernel launch");
}

int launch_vae_upsample2(const float* x, int H, int W, int C, void* y, bool y_bf16,
                         cudaStream_t st) {
  if (C % 4 != 0) return fail(BONSAI_ERR_ARG, "vae upsample: C % 4");
  const long long n4 = (long long)H * W * C / 4;
  ProfScope prof("vae_upsample2", 0.0, (double)H * W * C * 12, st);
  vops::upsample2_kernel<<<vops::grid_for(n4, 256), 256, 0, st>>>(
      x, H, W, C, reinterpret_cast<uint2*>(y), y_bf16 ? 1 : 0);
  return launch_status("vae upsample2_kernel launch");
}

int launch_vae_cast(const float* x, long long n, void* y, bool y_bf16, cudaStream_t st) {
  if (n % 4 != 0) return fail(BONSAI_ERR_ARG, "vae cast: n % 4");
  ProfScope prof("vae_cast", 0.0, (double)n * 6, st);
  vops::cast_kernel<<<vops::grid_for(n / 4, 256), 256, 0, st>>>(
      x, n / 4, reinterpret_cast<uint2*>(y), y_bf16 ? 1 : 0);
  return launch_status("vae cast_kernel launch");
}

int launch_vae_preprocess(const float* latent, int h, int w, const float* bn_mean,
                          const float* bn_std, __half* y, cudaStream_t st) {
  const long long total = 4LL * h * w * 64;
  vops::preprocess_kernel<<<vops::grid_for(total, 256), 256, 0, st>>>(latent, h, w, bn_mean,
                                                                      bn_std, y);
  return launch_status("vae preprocess_kernel launch");
}

int launch_vae_softmax(const float* S, long long ld_s, int rows, int cols, float scale,
                       __half* P, long long ld_p, float* rowinv, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return fail(BONSAI_ERR_ARG, "vae softmax: empty");
  const bool fast = cols % 4 == 0 && ld_s % 4 == 0 && ld_p % 4 == 0 &&
                    cols <= vops::kSoftmaxThreads * vops::kSoftmaxRegs4 * 4;
  ProfScope prof("vae_softmax", 0.0, (double)rows * cols * 6, st);
  vops::softmax_kernel<<<rows, vops::kSoftmaxThreads, 0, st>>>(S, ld_s, cols, scale, P, ld_p,
                                                              rowinv, fast ? 1 : 0);
  return launch_status("vae softmax_kernel launch");
}

int launch_vae_pack_weight(const float* src, int cout, int cin, int taps, int rows, int cin_pad,
                           void* dst, bool bf16, cudaStream_t st) {
  const long long total = (long long)rows * taps * cin_pad;
  vops::pack_weight_kernel<<<vops::grid_for(total, 256), 256, 0, st>>>(
      src, cout, cin, taps, total, cin_pad, reinterpret_cast<uint16_t*>(dst), bf16 ? 1 : 0);
  return launch_status("vae pack_weight_kernel launch");
}

int launch_vae_fill(float* dst, long long n, unsigned long long seed, float mean, float std,
                    bool uniform, cudaStream_t st) {
  vops::fill_kernel<<<vops::grid_for(n, 256), 256, 0, st>>>(dst, n, seed, mean, std,
                                                            uniform ? 1 : 0);
  return launch_status("vae fill_kernel launch");
}

}  // namespace bonsai
