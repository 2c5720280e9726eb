// Implicit-GEMM convolution / dense GEMM on tcgen05 for the Flux VAE decoder.
//
// Replaces the ggml_conv_2d_direct and ggml_mul_mat nodes of the reference's
// decoder graph (src/vae_graph.cpp:44-212).  Activations are NHWC (channels
// innermost) f16 or bf16; a stride-1 convolution with 'same' zero padding
// (3x3 or 1x1) is a GEMM with M = pixels, N = output channels and
// K = taps x input channels:
//
//   out[pix][n] = sum_tap sum_c in[pix + offset(tap)][c] * w[n][tap][c]
//
// Two forms share the code (template parameter kPair):
//  * the CTA-pair kernel (default): a cluster of two CTAs on the two SMs of a
//    TPC computes 256 pixels x BN output channels per tile with
//    tcgen05.mma.cta_group::2 (M = 256).  Each CTA loads its own 128-pixel
//    unit and half of the weight tile (BN/2 rows) into its shared memory;
//    the even CTA issues the MMAs and each CTA's TMEM receives its 128
//    pixels x BN.  Per SM and k-step that reads 16 KB of activations + BN/2
//    x 128 B of weights, against 16 KB + BN x 128 B for one CTA alone -- the
//    shared-memory bandwidth that bounds a 128 x 128 tile.
//  * the single-CTA kernel: 128 pixels x BN per tile (cta_group::1).
// Both are persistent with f32 accumulators in TMEM (two of them, so the
// epilogue of one tile overlaps the next tile's MMAs).  The 128 pixels of a
// unit are a bw x bh rectangle of the image; for each tap the TMA warp loads
// the rectangle shifted by the tap's offset as one 3-D box {64 channels, bw,
// bh} of the NHWC tensor.  Pixels outside the image come back as zeros from
// the TMA's out-of-bounds fill, which is exactly the convolution's zero
// padding; the box lands in shared memory as 128 rows of 128 bytes in the
// 128-byte-swizzled K-major layout the MMA reads.  The weight tile {64, rows}
// of w[n][tap*Cin + c] comes by a 2-D TMA load.  A plain GEMM is the 1x1
// case over a 1-row "image".  No load uses cluster multicast.
//
// The epilogue (8 warps per CTA) reads the accumulators with tcgen05.ld (one
// pixel per thread), optionally scales by a per-pixel factor, adds the bias
// and an f32 residual, writes f32 / f16 / bf16 NHWC, an f16 transposed
// [n][pixel] tensor or f32 NCHW (the decoder's final image), and optionally
// a bf16 copy of the output and GroupNorm partial statistics.
#include "internal.cuh"
#include "ptx.cuh"
#include "vae.cuh"
#include "bonsai_cuda.h"

#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace bonsai {
namespace gemm {
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn();
}

namespace vconv {

constexpr int BM = 128;       // pixels per CTA (MMA M per CTA)
constexpr int BN_MAX = 256;   // output channels per tile (MMA N)
constexpr int BK = 64;        // input channels per pipeline stage
constexpr int A_BYTES = BM * BK * 2;  // one 128-pixel A box: 16 KB
constexpr int TMEM_COLS = 2 * BN_MAX;
constexpr int WARP_TMA = 0;
constexpr int WARP_MMA = 1;
constexpr int WARP_EPI0 = 2;
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = (WARP_EPI0 + EPI_WARPS) * 32;

// Shared memory: barriers in the first 1 KB, then the pipeline stages (each
// the 16 KB pixel box + this CTA's weight rows), as many as fit in
// kStageBudget: a stage lasts BN/2 x 4 clocks of MMA (pair) or BN x 4
// (single), so the narrow-N tiles get more stages in flight.
constexpr int kMaxStages = 8;
constexpr int kStageBudget = 224 * 1024;
// Horizontal-tap sharing: when a tile is one 128-pixel image row, the taps of
// one kernel row (dx = -1, 0, 1; or the two of an upsampling phase) read the
// same pixels shifted by one: one box of kHaloPix pixels serves all of them,
// the MMA reading it from row j (descriptor base offset j).
constexpr int kHaloPix = 136;  // 128 + 2, rounded up to the 8-row swizzle atom
constexpr int SMEM_BYTES = 1024 /*align slack*/ + 1024 /*barriers*/ + kStageBudget;

struct Params {
  int H, W;                // input grid (the output is H*S x W*S, S = 2 when phases = 4)
  int bw, bh, tiles_x;     // 128-pixel unit bw x bh
  int units;               // units of the input grid
  int n_mtiles, n_ntiles, num_tiles;  // m-tiles: units (single) or unit pairs (pair)
  int phases;              // 1, or 4: nearest 2x upsample folded into per-phase 2x2 weights
  int BN;                  // output channels per tile (multiple of 16, <= 256)
  int taps;                // taps per phase
  int8_t tap_dy[9], tap_dx[9];
  int stages, stage_bytes; // pipeline depth and stage size (shared memory layout)
  int group;               // taps sharing one pixel box (1, or 3 / 2 with a halo box)
  int a_bytes;             // pixel box bytes per stage (16 KB, or the halo box)
  int cin_blocks;          // 64-channel blocks per tap
  int k_per_tap;           // weight K offset between taps
  int w_rows_phase;        // weight rows per phase
  int N;                   // output channels
  const float* bias;
  const float* row_scale;
  const float* resid;
  long long ld_resid;
  void* out;
  long long ld_out;
  int out_mode;
  uint16_t* out2;          // optional bf16 copy of the output (NHWC, ld_out2)
  long long ld_out2;
  float4* stats;           // optional GroupNorm partials [slot][32] {sum, M2, count, 0}
  int gw;                  // channels per group (N / 32) when stats
  int* err;
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// GroupNorm partials of one 32-column chunk over the warp's 32 pixels, one
// pass: per group of GW columns each lane forms the sum and the sum of
// squares of its values centred on the group's mean bias (a uniform shift,
// so the variance is unchanged and the f32 cancellation of q - s^2/n only
// depends on how far the data's mean sits from it), then the warp reduces
// all 2 * (32/GW) values at once by a transpose reduce-scatter (each level
// exchanges half of the remaining values: 16 / 9 / 6 shuffles for GW = 4 / 8
// / 16 instead of a butterfly per value).  Writes {sum, M2 about the chunk
// mean, count} per group (combined by launch_vae_gn_finalize).
template <int GW>
__device__ __forceinline__ void chunk_stats(const float (&f)[32], const float* bias, int nb,
                                            bool valid, float nvalid, float4* dst, uint32_t lane) {
  constexpr int NG = 32 / GW;
  constexpr int V = 2 * NG;  // s and q of every group
  float shift[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float b = 0.0f;
    if (bias) {
#pragma unroll
      for (int k = 0; k < GW; ++k) b += bias[nb + g * GW + k];
    }
    shift[g] = b * (1.0f / GW);
  }
  float v[V];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float a = 0.0f, q = 0.0f;
#pragma unroll
    for (int k = 0; k < GW; ++k) {
      const float e = f[g * GW + k] - shift[g];
      a += e;
      q = fmaf(e, e, q);
    }
    v[2 * g] = valid ? a : 0.0f;
    v[2 * g + 1] = valid ? q : 0.0f;
  }
  // Reduce-scatter: at offset o the lane keeps the upper half of its values
  // if bit o of its lane id is set, else the lower half, and adds the
  // partner's copy of the half it keeps.
#pragma unroll
  for (int h = V / 2, o = 16; h >= 1; h >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  // Lanes now hold value index (lane / (32 / V)) % V summed over the lanes
  // that differ in the used bits; the rest of the lanes sum by butterfly.
  constexpr int REP = 32 / V;
#pragma unroll
  for (int o = REP / 2; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  const int idx = (int)(lane / REP) % V;
  const float other = __shfl_xor_sync(0xffffffffu, v[0], REP);  // the q next to this s
  if ((idx & 1) == 0 && (lane % REP) == 0) {
    const int g = idx >> 1;
    const float cnt = nvalid * GW;
    const float sc = v[0], qc = other;
    const float m2 = cnt > 0.0f ? fmaxf(qc - sc * (sc / cnt), 0.0f) : 0.0f;
    float sh = 0.0f;
#pragma unroll
    for (int gg = 0; gg < NG; ++gg)  // static indices keep shift[] in registers
      if (gg == g) sh = shift[gg];
    dst[g] = make_float4(sc + cnt * sh, m2, cnt, 0.0f);
  }
}

struct TileCoord {
  int phase, n0, mt;
};
__device__ __forceinline__ TileCoord tile_coord(const Params& p, int tile) {
  TileCoord t;
  const int nt = tile % p.n_ntiles;
  const int r = tile / p.n_ntiles;
  t.phase = r % p.phases;
  t.mt = r / p.phases;
  t.n0 = nt * p.BN;
  return t;
}
__device__ __forceinline__ void unit_origin(const Params& p, int u, int& x0, int& y0) {
  const int ty = u / p.tiles_x;
  x0 = (u - ty * p.tiles_x) * p.bw;
  y0 = ty * p.bh;
}

// One 32-column chunk of the epilogue: scale, bias, residual, statistics,
// stores.  Warp-collective (the statistics shuffle); `valid` is per lane.
// The residual of one chunk (zeros when there is none or the pixel is
// invalid); loaded ahead of the accumulator so the DRAM latency overlaps.
__device__ __forceinline__ void load_resid(const Params& p, int nb, int nn, bool valid,
                                           long long pix, float (&r)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) r[j] = 0.0f;
  if (!p.resid || !valid || nn <= 0) return;
  const float* src = p.resid + pix * p.ld_resid + nb;
  if (nn == 32 && (p.ld_resid & 3) == 0) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 o = __ldg(reinterpret_cast<const float4*>(src + j));
      r[j] = o.x;
      r[j + 1] = o.y;
      r[j + 2] = o.z;
      r[j + 3] = o.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nn) r[j] = src[j];
  }
}

__device__ __forceinline__ void epilogue_chunk(const Params& p, const uint32_t (&v)[32],
                                               const float (&res)[32], int nb, int nn, bool valid,
                                               long long pix, float rs, float nvalid, float4* srow,
                                               long long plane, uint32_t lane) {
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) * rs;
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nn) f[j] += p.bias[nb + j];
  }
  const bool vec = nn == 32;
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] += res[j];
  if (srow) {  // warp-uniform; N == 32 * gw so every chunk is full
    float4* dst = srow + nb / p.gw;
    if (p.gw == 16) chunk_stats<16>(f, p.bias, nb, valid, nvalid, dst, lane);
    else if (p.gw == 8) chunk_stats<8>(f, p.bias, nb, valid, nvalid, dst, lane);
    else chunk_stats<4>(f, p.bias, nb, valid, nvalid, dst, lane);
  }
  if (!valid) return;
  if (p.out2) {
    uint16_t* d = p.out2 + pix * p.ld_out2 + nb;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 o;
      o.x = pack_bf2(f[j], f[j + 1]);
      o.y = pack_bf2(f[j + 2], f[j + 3]);
      o.z = pack_bf2(f[j + 4], f[j + 5]);
      o.w = pack_bf2(f[j + 6], f[j + 7]);
      *reinterpret_cast<uint4*>(d + j) = o;
    }
  }
  switch (p.out_mode) {
    case VOUT_F32: {
      float* d = reinterpret_cast<float*>(p.out) + pix * p.ld_out + nb;
      if (vec && (p.ld_out & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(d + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nn) d[j] = f[j];
      }
      break;
    }
    case VOUT_F16:
    case VOUT_BF16: {
      const bool bf = p.out_mode == VOUT_BF16;
      uint16_t* d = reinterpret_cast<uint16_t*>(p.out) + pix * p.ld_out + nb;
      if (vec && (p.ld_out & 7) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 o;
          o.x = bf ? pack_bf2(f[j], f[j + 1]) : pack_h2(f[j], f[j + 1]);
          o.y = bf ? pack_bf2(f[j + 2], f[j + 3]) : pack_h2(f[j + 2], f[j + 3]);
          o.z = bf ? pack_bf2(f[j + 4], f[j + 5]) : pack_h2(f[j + 4], f[j + 5]);
          o.w = bf ? pack_bf2(f[j + 6], f[j + 7]) : pack_h2(f[j + 6], f[j + 7]);
          *reinterpret_cast<uint4*>(d + j) = o;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nn)
            d[j] = bf ? __bfloat16_as_ushort(__float2bfloat16_rn(f[j]))
                      : __half_as_ushort(__float2half_rn(f[j]));
      }
      break;
    }
    case VOUT_F16_T: {
      __half* d = reinterpret_cast<__half*>(p.out) + pix;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nn) d[(long long)(nb + j) * p.ld_out] = __float2half_rn(f[j]);
      break;
    }
    default: {  // VOUT_F32_NCHW
      float* d = reinterpret_cast<float*>(p.out) + pix;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nn) d[(long long)(nb + j) * plane] = f[j];
      break;
    }
  }
}

template <bool kPair>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    conv_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                const Params p, const uint32_t idesc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smem = base + 1024;  // stages (1024-aligned)
  const int STAGES = p.stages;
  const int STAGE_BYTES = p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(base);
  uint64_t* empty = full + kMaxStages;
  uint64_t* dfull = empty + kMaxStages;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  // Pair: rank 0 issues the MMAs; the cluster walks the tiles.  Single: the CTA.
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int first = kPair ? (int)cluster_id_x() : (int)blockIdx.x;
  const int stride = kPair ? (int)cluster_count_x() : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&dfull[b], 1);
      bar_init(&dempty[b], (kPair ? 2 : 1) * EPI_WARPS);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // barrier inits and TMEM of both CTAs visible
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ksteps = (p.taps / p.group) * p.cin_blocks;
  const int rows_per_cta = kPair ? p.BN / 2 : p.BN;
  const int b_tap_bytes = rows_per_cta * BK * 2;

  if (warp == WARP_TMA) {
    if (elect_one()) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      const uint32_t cta_bytes = (uint32_t)(p.a_bytes + p.group * b_tap_bytes);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = first; tile < p.num_tiles && ok; tile += stride) {
        const TileCoord tc = tile_coord(p, tile);
        const int a = tc.phase >> 1, bph = tc.phase & 1;
        int x0, y0;
        unit_origin(p, kPair ? 2 * tc.mt + (int)rank : tc.mt, x0, y0);
        const int brow = tc.phase * p.w_rows_phase + tc.n0 + (int)rank * rows_per_cta;
        for (int t0 = 0; t0 < p.taps && ok; t0 += p.group) {
          // the group's taps share dy; its box starts at the first tap's dx
          const int dy = p.tap_dy[t0] + a, dx = p.tap_dx[t0] + bph;
          for (int cb = 0; cb < p.cin_blocks; ++cb, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!wait_bar(&empty[s], ph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * STAGE_BYTES;
            if constexpr (kPair) {
              // Both CTAs' loads count on the even CTA's barrier.
              if (rank == 0) bar_arrive_expect_tx(&full[s], 2 * cta_bytes);
              const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
              tma_load_3d_pair(st, &amap, fb, cb * BK, x0 + dx, y0 + dy);
              for (int j = 0; j < p.group; ++j)
                tma_load_2d_pair(st + p.a_bytes + j * b_tap_bytes, &bmap, fb,
                                 (t0 + j) * p.k_per_tap + cb * BK, brow);
            } else {
              bar_arrive_expect_tx(&full[s], cta_bytes);
              tma_load_3d(st, &amap, &full[s], cb * BK, x0 + dx, y0 + dy);
              for (int j = 0; j < p.group; ++j)
                tma_load_2d(st + p.a_bytes + j * b_tap_bytes, &bmap, &full[s],
                            (t0 + j) * p.k_per_tap + cb * BK, brow);
            }
          }
        }
      }
      if (!ok) {
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == WARP_MMA) {
    if (elect_one()) {
      if (rank == 0) {
        uint32_t it = 0, lt = 0;
        bool ok = true;
        for (int tile = first; tile < p.num_tiles && ok; tile += stride, ++lt) {
          const uint32_t b = lt & 1;
          const uint32_t dph = (lt >> 1) & 1;
          if (!wait_bar(&dempty[b], dph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + b * BN_MAX;
          for (int ks = 0; ks < ksteps; ++ks, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!wait_bar(&full[s], ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t saddr = smem_u32(smem + s * STAGE_BYTES);
            for (int j = 0; j < p.group; ++j) {
              // tap j of the group reads the pixel box from row j
              const uint32_t arow = saddr + (uint32_t)j * 128u;
              const uint32_t bbase = saddr + (uint32_t)(p.a_bytes + j * b_tap_bytes);
#pragma unroll
              for (int k16 = 0; k16 < BK / 16; ++k16) {
                // the 128-byte swizzle follows the address bits, so a start j rows
                // into the 1024-byte-aligned box needs no base offset (as the
                // +32-byte k16 steps within a row need none)
                const uint64_t adesc = make_smem_desc(arow + k16 * 32, 16, 1024);
                const uint64_t bdesc = make_smem_desc(bbase + k16 * 32, 16, 1024);
                const uint32_t acc = (ks | j | k16) != 0 ? 1u : 0u;
                if constexpr (kPair)
                  mma_ss_pair(d_tmem, adesc, bdesc, idesc, acc);
                else
                  mma_ss(d_tmem, adesc, bdesc, idesc, acc);
              }
            }
            if constexpr (kPair) tc_commit_pair(&empty[s], 0x3);
            else tc_commit(&empty[s]);
          }
          if (!ok) break;
          if constexpr (kPair) tc_commit_pair(&dfull[b], 0x3);
          else tc_commit(&dfull[b]);
        }
        if constexpr (kPair) tc_commit_pair(drain, 0x3);
        else tc_commit(drain);
      }
      // Wait until every MMA has completed (the pair's commit arrives on the
      // drain barrier of both CTAs).
      const uint32_t da = smem_u32(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!bar_try_wait(da, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          if (p.err) atomicCAS(p.err, 0, DEV_ERR_TIMEOUT_MMA);
          break;
        }
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (its pixels); the two
    // warps of a lane quarter take alternate 32-column chunks.
    const int q = warp & 3;
    const int eh = (warp - WARP_EPI0) >> 2;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int nch = (p.BN + 31) / 32;
    const int S = p.phases == 4 ? 2 : 1;
    const long long Wout = (long long)p.W * S;
    const long long plane = (long long)p.H * S * Wout;
    const uint32_t dempty_lead = kPair ? mapa_shared(smem_u32(&dempty[0]), 0) : 0u;
    uint32_t lt = 0;
    for (int tile = first; tile < p.num_tiles; tile += stride, ++lt) {
      const TileCoord tc = tile_coord(p, tile);
      const uint32_t b = lt & 1;
      const uint32_t dph = (lt >> 1) & 1;
      const int unit = kPair ? 2 * tc.mt + (int)rank : tc.mt;
      int x0, y0;
      unit_origin(p, unit, x0, y0);
      const int ml = q * 32 + (int)lane;
      const int px = x0 + ml % p.bw;
      const int py = y0 + ml / p.bw;
      const bool valid = unit < p.units && px < p.W && py < p.H;
      const long long pix =
          (long long)(py * S + (tc.phase >> 1)) * Wout + (long long)px * S + (tc.phase & 1);
      // The first chunk's residual is in flight while the tile's MMAs finish.
      float res[32];
      load_resid(p, tc.n0 + eh * 32, min(min(32, p.BN - eh * 32), p.N - tc.n0 - eh * 32), valid,
                 pix, res);
      const bool good = wait_bar(&dfull[b], dph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, good)) break;  // tcgen05.ld is warp-collective
      tc_fence_after();

      const float rs = (p.row_scale && valid) ? p.row_scale[pix] : 1.0f;
      const float nvalid = (float)__popc(__ballot_sync(0xffffffffu, valid));
      const int slot = (tc.mt * p.phases + tc.phase) * (kPair ? 2 : 1) + (int)rank;
      float4* srow = p.stats ? p.stats + ((size_t)slot * 4 + q) * kStatGroups : nullptr;
      for (int c = eh; c < nch; c += 2) {
        const int nb = tc.n0 + c * 32;
        const int nn = min(min(32, p.BN - c * 32), p.N - nb);
        if (c != eh) load_resid(p, nb, nn, valid, pix, res);
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + b * BN_MAX + c * 32, v);
        tmem_wait_ld();
        if (nn <= 0) continue;
        epilogue_chunk(p, v, res, nb, nn, valid, pix, rs, nvalid, srow, plane, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) bar_arrive_remote(dempty_lead + b * 8u);
        else bar_arrive(&dempty[b]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // no pair MMA, remote arrive or TMEM access left
  if (warp == WARP_MMA) {
    __syncwarp();
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem, TMEM_COLS);
    else tmem_dealloc(tmem, TMEM_COLS);
  }
}

// 128-pixel unit tile bw x bh (bw a power of two in [8, 128]) with the least
// padded area for a W x H image (ties go to the wider tile).
void pick_pixel_tile(int H, int W, int& bw, int& bh) {
  long long best = -1;
  for (int cand = 128; cand >= 8; cand /= 2) {
    const int ch = 128 / cand;
    const long long area = (long long)((W + cand - 1) / cand) * cand * ((H + ch - 1) / ch) * ch;
    if (best < 0 || area < best) {
      best = area;
      bw = cand;
      bh = ch;
    }
  }
}

// Output-channel tile: the smallest power of two >= N up to 128; for wider
// N, 256 unless 128 fills the SMs in fewer equivalent waves.
int pick_bn(int N, long long units, int sms) {
  if (N <= 16) return 16;
  if (N <= 32) return 32;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  auto cost = [&](int bn) {
    const long long tiles = units * ((N + bn - 1) / bn);
    const long long waves = (tiles + sms - 1) / sms;
    return (double)waves * (bn + 32);
  };
  return cost(128) < cost(256) ? 128 : 256;
}

}  // namespace vconv

long long vae_conv_stat_slots(int H, int W, int phases) {
  int bw = 128, bh = 1;
  vconv::pick_pixel_tile(H, W, bw, bh);
  const long long units = (long long)((W + bw - 1) / bw) * ((H + bh - 1) / bh);
  return (units + 1) * 4 * (phases == 4 ? 4 : 1);  // + 1: the pair kernel rounds units up to even
}

namespace {

enum class ConvKernel { Pair, Single };

// BONSAI_VAE_CONV=single selects the one-CTA form (used by the tests to
// check both); the CTA-pair form is the default.
ConvKernel conv_kernel_choice() {
  const char* e = getenv("BONSAI_VAE_CONV");
  return (e && std::strcmp(e, "single") == 0) ? ConvKernel::Single : ConvKernel::Pair;
}

template <bool kPair>
int ensure_smem_attr() {
  static bool done_dev[64] = {};
  bool& done = done_dev[device_slot()];
  if (!done) {
    cudaError_t e = cudaFuncSetAttribute(vconv::conv_kernel<kPair>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         vconv::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_status(e, "vae conv: smem attribute");
    done = true;
  }
  return 0;
}

// Clusters of two conv CTAs that can be resident at once (0 if none).
int conv_pair_slots() {
  struct Slots {
    int n = -1;
  };
  static Slots slots[64];
  int& n = slots[device_slot()].n;
  if (n >= 0) return n;
  n = 0;
  if (ensure_smem_attr<true>()) return n;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * std::max(1, num_sms() / 2));
  cfg.blockDim = dim3(vconv::NUM_THREADS);
  cfg.dynamicSmemBytes = vconv::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int c = 0;
  if (cudaOccupancyMaxActiveClusters(&c, vconv::conv_kernel<true>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return n;
  }
  n = c;
  return n;
}

}  // namespace

int launch_vae_conv(const VaeConvArgs& a, cudaStream_t st) {
  using namespace vconv;
  const int phases = a.phases == 4 ? 4 : 1;
  if (a.phases != 1 && a.phases != 4) return fail(BONSAI_ERR_ARG, "vae conv: phases must be 1 or 4");
  if (phases == 1 && a.taps != 1 && a.taps != 9)
    return fail(BONSAI_ERR_ARG, "vae conv: taps must be 1 or 9");
  if (phases == 4 && a.taps != 4) return fail(BONSAI_ERR_ARG, "vae conv: the upsampling form has 4 taps");
  if (a.H <= 0 || a.W <= 0 || a.cin <= 0 || a.N <= 0)
    return fail(BONSAI_ERR_ARG, "vae conv: empty shape");
  if ((a.ld_in & 7) != 0 || (a.w_ld & 7) != 0 || a.ld_in < a.cin)
    return fail(BONSAI_ERR_ARG, "vae conv: leading dimensions must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(a.in) & 15) != 0 || (reinterpret_cast<uintptr_t>(a.w) & 15) != 0)
    return fail(BONSAI_ERR_ARG, "vae conv: operands must be 16-byte aligned");
  const int cin_blocks = (a.cin + BK - 1) / BK;
  const int k_per_tap = a.taps == 1 ? 0 : a.k_per_tap;
  if (a.taps > 1 && k_per_tap < cin_blocks * BK)
    return fail(BONSAI_ERR_ARG, "vae conv: weight taps must be padded to 64 channels");
  const long long k_total = a.taps == 1 ? a.cin : (long long)a.taps * k_per_tap;
  if (k_total > a.w_ld) return fail(BONSAI_ERR_ARG, "vae conv: weight row shorter than K");
  if (a.stats && (a.N % 32 != 0 || (a.N / 32 != 4 && a.N / 32 != 8 && a.N / 32 != 16)))
    return fail(BONSAI_ERR_ARG, "vae conv: GroupNorm statistics need N in {128, 256, 512}");
  if ((a.out_mode == VOUT_F16_T || a.out_mode == VOUT_F32_NCHW) && (a.resid || a.stats || a.out2))
    return fail(BONSAI_ERR_ARG, "vae conv: transposed / planar outputs take no residual, statistics or copy");
  if (a.out2 && (a.N % 32 != 0 || (a.ld_out2 & 7) != 0 ||
                 (reinterpret_cast<uintptr_t>(a.out2) & 15) != 0))
    return fail(BONSAI_ERR_ARG, "vae conv: the bf16 copy needs N % 32 == 0 and 16-byte rows");

  auto fn = gemm::get_encode_fn();
  if (!fn) return fail(-5, "cuTensorMapEncodeTiled entry point unavailable");
  int bw = 128, bh = 1;
  pick_pixel_tile(a.H, a.W, bw, bh);
  const int tiles_x = (a.W + bw - 1) / bw;
  const long long units = (long long)tiles_x * ((a.H + bh - 1) / bh);
  const int sms = num_sms();
  const int slots = conv_pair_slots();
  const bool pair = conv_kernel_choice() == ConvKernel::Pair && slots > 0;
  const int BN = a.bn > 0 ? a.bn : pick_bn(a.N, units * phases, sms);
  if (BN % 16 != 0 || BN < 16 || BN > BN_MAX) return fail(BONSAI_ERR_ARG, "vae conv: bad BN");
  const int rows_per_cta = pair ? BN / 2 : BN;
  const long long n_mtiles = pair ? (units + 1) / 2 : units;
  const long long n_ntiles = (a.N + BN - 1) / BN;
  const long long num_tiles = n_mtiles * phases * n_ntiles;
  const long long stat_slots = n_mtiles * phases * (pair ? 2 : 1) * 4;
  if (num_tiles > 0x7FFFFFFFLL) return fail(BONSAI_ERR_ARG, "vae conv: too many tiles");
  if (a.stats && stat_slots > a.stats_slots)
    return fail(BONSAI_ERR_ARG, "vae conv: GroupNorm partial buffer too small");
  const int w_rows_phase = std::max(a.N, a.w_rows);

  // Halo boxes when a tile is one 128-pixel row and at least three stages fit.
  bool halo = bw == 128 && bh == 1 && (a.taps == 9 || a.taps == 4);
  if (halo) {
    const int group = a.taps == 9 ? 3 : 2;
    halo = kStageBudget / (kHaloPix * BK * 2 + group * rows_per_cta * BK * 2) >= 3;
  }
  const CUtensorMapDataType dt =
      a.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap amap, bmap;
  {
    cuuint64_t dims[3] = {(cuuint64_t)a.cin, (cuuint64_t)a.W, (cuuint64_t)a.H};
    cuuint64_t strides[2] = {(cuuint64_t)a.ld_in * 2, (cuuint64_t)a.ld_in * 2 * a.W};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)(halo ? kHaloPix : bw), (cuuint32_t)bh};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&amap, dt, 3, const_cast<void*>(a.in), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(-5, "vae conv: activation tensor map (code " + std::to_string((int)r) + ")");
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)k_total, (cuuint64_t)w_rows_phase * phases};
    cuuint64_t strides[1] = {(cuuint64_t)a.w_ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)rows_per_cta};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&bmap, dt, 2, const_cast<void*>(a.w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(-5, "vae conv: weight tensor map (code " + std::to_string((int)r) + ")");
  }

  Params p{};
  p.H = a.H;
  p.W = a.W;
  p.bw = bw;
  p.bh = bh;
  p.tiles_x = tiles_x;
  p.units = (int)units;
  p.n_mtiles = (int)n_mtiles;
  p.n_ntiles = (int)n_ntiles;
  p.num_tiles = (int)num_tiles;
  p.phases = phases;
  p.BN = BN;
  p.taps = a.taps;
  for (int t = 0; t < 9; ++t) {
    // 3x3: offsets -1..1; 2x2 upsampling phases: base offsets -1..0 (+ the
    // phase bit in the kernel); 1x1: 0.
    if (a.taps == 9) {
      p.tap_dy[t] = (int8_t)(t / 3 - 1);
      p.tap_dx[t] = (int8_t)(t % 3 - 1);
    } else if (a.taps == 4) {
      p.tap_dy[t] = (int8_t)((t >> 1) - 1);
      p.tap_dx[t] = (int8_t)((t & 1) - 1);
    } else {
      p.tap_dy[t] = 0;
      p.tap_dx[t] = 0;
    }
  }
  p.group = 1;
  p.a_bytes = A_BYTES;
  p.stage_bytes = A_BYTES + rows_per_cta * BK * 2;
  if (halo) {
    p.group = a.taps == 9 ? 3 : 2;
    p.a_bytes = kHaloPix * BK * 2;
    p.stage_bytes = p.a_bytes + p.group * rows_per_cta * BK * 2;
  }
  p.stages = std::min(kMaxStages, kStageBudget / p.stage_bytes);
  p.cin_blocks = cin_blocks;
  p.k_per_tap = k_per_tap;
  p.w_rows_phase = w_rows_phase;
  p.N = a.N;
  p.bias = a.bias;
  p.row_scale = a.row_scale;
  p.resid = a.resid;
  p.ld_resid = a.ld_resid;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.out_mode = a.out_mode;
  p.out2 = static_cast<uint16_t*>(a.out2);
  p.ld_out2 = a.ld_out2;
  p.stats = reinterpret_cast<float4*>(a.stats);
  p.gw = a.N / 32;
  p.err = device_error_word();
  const uint32_t idesc = make_idesc_f16(pair ? 2 * BM : BM, BN, a.bf16 ? 1 : 0, 0, 0);

  const double flop = 2.0 * a.H * a.W * phases * (double)a.N * a.cin * a.taps;
  const char* kind = a.prof_name ? a.prof_name
                     : phases == 4 ? "vae_conv_up2x"
                     : a.taps == 9 ? (BN == 128 ? "vae_conv3x3_n128" : "vae_conv3x3")
                     : a.H == 1     ? "vae_attn_gemm"
                                    : "vae_conv1x1";
  if (pair) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (unsigned)std::min<long long>(num_tiles, slots));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfScope prof(kind, flop, 0.0, st);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, conv_kernel<true>, amap, bmap, p, idesc);
    if (e != cudaSuccess) return cuda_status(e, "vae conv_kernel (pair) launch");
    if (int rc = launch_status("vae conv_kernel (pair) launch")) return rc;
  } else {
    if (int rc = ensure_smem_attr<false>()) return rc;
    const int grid = (int)std::min<long long>(num_tiles, sms);
    ProfScope prof(kind, flop, 0.0, st);
    conv_kernel<false><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(amap, bmap, p, idesc);
    if (int rc = launch_status("vae conv_kernel launch")) return rc;
  }
  if (a.stats_slots_used) *a.stats_slots_used = stat_slots;
  return 0;
}

}  // namespace bonsai
