// Memory-bound kernels of the Flux VAE decoder (src/vae_graph.cpp,
// src/vae_decoder.cpp): the GroupNorm statistics finalize (the partial sums
// come from the convolution epilogue) and GroupNorm + SiLU application, the
// latent preprocessing, the attention softmax, weight packing (including the
// 3x3 kernels folded for the upsampling convolutions) and seeded synthetic
// weights.  All work
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

constexpr int kGnMergeWarps = 8;

// Stage 1: block b reduces slots b*8 + w + k*(gridDim.x*8) (warp w, lane =
// group; one coalesced 512-byte row per slot) into f64 sums of
// {count, sum, M2, sum^2 / count}, combined over its warps in warp order.
__global__ void __launch_bounds__(32 * kGnMergeWarps)
    gn_merge_kernel(const float4* __restrict__ part, long long slots, double* __restrict__ out) {
  const int g = threadIdx.x % 32;
  const int w = threadIdx.x / 32;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (long long i = (long long)blockIdx.x * kGnMergeWarps + w; i < slots;
       i += (long long)gridDim.x * kGnMergeWarps) {
    const float4 v = part[i * kStatGroups + g];
    if (v.z > 0.0f) {
      acc[0] += v.z;
      acc[1] += v.x;
      acc[2] += v.y;
      acc[3] += (double)v.x * ((double)v.x / v.z);
    }
  }
  __shared__ double sh[kGnMergeWarps][32][4];
#pragma unroll
  for (int k = 0; k < 4; ++k) sh[w][g][k] = acc[k];
  __syncthreads();
  if (w == 0) {
    for (int j = 1; j < kGnMergeWarps; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] += sh[j][g][k];
    double* o = out + ((long long)blockIdx.x * 32 + g) * 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = acc[k];
  }
}

// Stage 2: warp g sums group g's block results (lane-strided, then a fixed
// shuffle tree).  With N = count, S = sum: mean = S / N and
// M2 = sum_k M2_k + sum_k n_k mean_k^2 - N mean^2 (the scatter of the slot
// means about the mean; f64 keeps the cancellation harmless).
__global__ void gn_merge_final_kernel(const double* __restrict__ in, int nblk, float eps,
                                      float* __restrict__ mean_rstd) {
  const int g = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int b = lane; b < nblk; b += 32) {
    const double* r = in + ((long long)b * 32 + g) * 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += r[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  if (lane == 0) {
    const double n = acc[0];
    const double mean = n > 0.0 ? acc[1] / n : 0.0;
    const double m2 = acc[2] + acc[3] - (n > 0.0 ? acc[1] * mean : 0.0);
    const double var = n > 0.0 ? fmax(m2 / n, 0.0) : 0.0;
    mean_rstd[2 * g] = (float)mean;
    mean_rstd[2 * g + 1] = (float)(1.0 / sqrt(var + (double)eps));
  }
}

// Thread t owns the 4 channels (t % (C/4))*4.. for every (256/(C/4))-th row
// of its block's row range, so its group statistics and affine terms are
// loaded once; four rows are in flight per iteration.
__global__ void __launch_bounds__(256, 4)
    gn_apply_kernel(const float* __restrict__ x, long long pixels, int C,
                    long long rows_per_blk, const float* __restrict__ mean_rstd,
                    const float* __restrict__ gamma, const float* __restrict__ beta, int silu,
                    uint2* __restrict__ y, int bf) {
  const int c4n = C / 4;
  const int rpp = 256 / c4n;
  const int col4 = threadIdx.x % c4n;
  const int r0 = threadIdx.x / c4n;
  const int c = col4 * 4;
  const int g = c / (C / 32);
  const float mean = mean_rstd[2 * g], rstd = mean_rstd[2 * g + 1];
  const float4 ga = __ldg(reinterpret_cast<const float4*>(gamma + c));
  const float4 be = __ldg(reinterpret_cast<const float4*>(beta + c));
  const float sc[4] = {rstd * ga.x, rstd * ga.y, rstd * ga.z, rstd * ga.w};
  const float sh[4] = {be.x, be.y, be.z, be.w};
  const long long row_begin = (long long)blockIdx.x * rows_per_blk;
  const long long row_end = min(pixels, row_begin + rows_per_blk);
  const float4* xin = reinterpret_cast<const float4*>(x);
  auto emit = [&](long long r, float4 v) {
    float o[4] = {(v.x - mean) * sc[0] + sh[0], (v.y - mean) * sc[1] + sh[1],
                  (v.z - mean) * sc[2] + sh[2], (v.w - mean) * sc[3] + sh[3]};
    if (silu) {
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = __fdividef(o[k], 1.0f + __expf(-o[k]));
    }
    y[r * c4n + col4] = pack4(o[0], o[1], o[2], o[3], bf != 0);
  };
  long long r = row_begin + r0;
  for (; r + 3 * rpp < row_end; r += 4 * rpp) {
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = __ldg(xin + (r + k * rpp) * c4n + col4);
#pragma unroll
    for (int k = 0; k < 4; ++k) emit(r + k * rpp, v[k]);
  }
  for (; r < row_end; r += rpp) emit(r, __ldg(xin + r * c4n + col4));
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

// Rows of 3x3 taps feeding 2x2 tap r of phase a: a = 0: {0}, {1, 2};
// a = 1: {0, 1}, {2} (nearest upsampling repeats each input row twice).
__device__ __forceinline__ void fold_range(int a, int r, int& lo, int& hi) {
  lo = (a == 0) ? (r == 0 ? 0 : 1) : (r == 0 ? 0 : 2);
  hi = (a == 0) ? (r == 0 ? 0 : 2) : (r == 0 ? 1 : 2);
}

__global__ void pack_subpixel_kernel(const float* __restrict__ src, int cout, int cin,
                                     int cin_pad, long long total, uint16_t* __restrict__ dst,
                                     int bf) {
  const long long per_phase = (long long)cout * 4 * cin_pad;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int phase = (int)(i / per_phase);
    const long long rem = i - phase * per_phase;
    const int n = (int)(rem / (4 * cin_pad));
    const int rem2 = (int)(rem - (long long)n * 4 * cin_pad);
    const int t = rem2 / cin_pad, c = rem2 % cin_pad;
    float v = 0.0f;
    if (c < cin) {
      int ylo, yhi, xlo, xhi;
      fold_range(phase >> 1, t >> 1, ylo, yhi);
      fold_range(phase & 1, t & 1, xlo, xhi);
      const float* w = src + ((long long)n * cin + c) * 9;
      for (int ky = ylo; ky <= yhi; ++ky)
        for (int kx = xlo; kx <= xhi; ++kx) v += w[ky * 3 + kx];
    }
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

int launch_vae_gn_finalize(const float* partials, long long slots, float eps, float* mean_rstd,
                           double* scratch, cudaStream_t st) {
  const long long want = (slots + 4 * vops::kGnMergeWarps - 1) / (4 * vops::kGnMergeWarps);
  const int nblk = (int)std::max<long long>(1, std::min<long long>(want, kGnMergeBlocks));
  ProfScope prof("vae_gn_stats", 0.0, (double)slots * kStatGroups * 16, st);
  vops::gn_merge_kernel<<<nblk, 32 * vops::kGnMergeWarps, 0, st>>>(
      reinterpret_cast<const float4*>(partials), slots, scratch);
  if (int rc = launch_status("vae gn_merge_kernel launch")) return rc;
  vops::gn_merge_final_kernel<<<1, 32 * kStatGroups, 0, st>>>(scratch, nblk, eps, mean_rstd);
  return launch_status("vae gn_merge_final_kernel launch");
}

int launch_vae_gn_apply(const float* x, long long pixels, int C, const float* mean_rstd,
                        const float* gamma, const float* beta, bool silu, void* y, bool y_bf16,
                        cudaStream_t st) {
  if (C < 128 || C > 1024 || 256 % (C / 4) != 0 || C % 4 != 0 || pixels <= 0)
    return fail(BONSAI_ERR_ARG, "vae group norm: C must be 128, 256, 512 or 1024");
  const int rpp = 256 / (C / 4);
  const long long want_blocks = (long long)num_sms() * 8;
  long long rows_per_blk = (pixels + want_blocks - 1) / want_blocks;
  rows_per_blk = std::max<long long>(rpp, (rows_per_blk + rpp - 1) / rpp * rpp);
  const long long blocks = (pixels + rows_per_blk - 1) / rows_per_blk;
  ProfScope prof("vae_gn_apply", 0.0, (double)pixels * C * 6, st);
  vops::gn_apply_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, pixels, C, rows_per_blk, mean_rstd,
                                                         gamma, beta, silu ? 1 : 0,
                                                         reinterpret_cast<uint2*>(y), y_bf16 ? 1 : 0);
  return launch_status("vae gn_apply_kernel launch");
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

int launch_vae_pack_subpixel_weight(const float* src, int cout, int cin, int cin_pad, void* dst,
                                    bool bf16, cudaStream_t st) {
  const long long total = 4LL * cout * 4 * cin_pad;
  vops::pack_subpixel_kernel<<<vops::grid_for(total, 256), 256, 0, st>>>(
      src, cout, cin, cin_pad, total, reinterpret_cast<uint16_t*>(dst), bf16 ? 1 : 0);
  return launch_status("vae pack_subpixel_kernel launch");
}

int launch_vae_fill(float* dst, long long n, unsigned long long seed, float mean, float std,
                    bool uniform, cudaStream_t st) {
  vops::fill_kernel<<<vops::grid_for(n, 256), 256, 0, st>>>(dst, n, seed, mean, std,
                                                            uniform ? 1 : 0);
  return launch_status("vae fill_kernel launch");
}

}  // namespace bonsai
