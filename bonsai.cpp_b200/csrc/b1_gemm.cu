// B1_0 1-bit-weight GEMM for sm_100a (tcgen05 / TMEM / TMA).
//
// Replaces the reference's b1_linear_f32_f32 (src/b1_0_kernel.h:37-288),
// which computes out[t][r] = sum_blk scale[r][blk] * sum_i (bit ? +x : -x)
// over the packed layout of src/diffuser_types.h:10-11 /
// convert_to_b1_0_packed.py:21-43.
//
// Two kernels share the retiled weight layout, the epilogues and the
// warp-specialised structure (TMA warp, MMA warp, expansion warps, epilogue
// warps, persistent tile loop, mbarrier rings with bounded waits):
//
// b1_gemm_pair_kernel (the main path): a cluster of two CTAs on the two SMs
//   of a TPC computes a 256-weight-row x 256-token tile with
//   tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16 per instruction).
//   Each CTA's expansion warps turn the sign words + fp16 scales of its 128
//   weight rows into exact f16 +-scale values and store them into its own
//   shared memory in the 128-byte-swizzled K-major layout; its TMA warp loads
//   its 128-token half of the activation tile.  The even CTA issues the MMAs;
//   each CTA's TMEM receives its 128 rows x 256 tokens (two 256-column
//   accumulators, so the epilogue of one tile overlaps the next tile's MMAs).
//   Per SM and k-block of 64 this expands 8 K weights per 128x256x64 MMA
//   block, half of what a 128x128 tile needs.
//
// b1_gemm_kernel (small grids): one CTA per 128x128 tile; the expanded
//   weights go straight into TMEM with tcgen05.st (A from TMEM, B from SMEM).
//   It has twice as many tiles as the pair kernel for the same problem, so it
//   keeps more SMs busy when the pair kernel would run a single short wave
//   (e.g. the 512-token text stream).
//
// launch_b1_gemm picks the kernel with the smaller estimated time (waves x
// tile time); BONSAI_B1_KERNEL=pair|single forces one (used by the tests).
#include "internal.cuh"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace bonsai {
namespace gemm {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BN = 128;  // tokens per tile (MMA N)
constexpr int BK = 64;   // inputs per pipeline stage
constexpr int STAGES = 8;
constexpr int X_STAGE_BYTES = BN * BK * 2;       // 16 KB
constexpr int RAW_STAGE_BYTES = kChunkWords * 4;  // 1.5 KB
constexpr int TMEM_COLS = 512;
constexpr int D_COL0 = 0;      // accumulators at columns [0,128) and [128,256)
constexpr int A_COL0 = 256;    // A stages at 256 + s*32 (64 f16 = 32 columns)

constexpr int WARP_TMA = 0;
constexpr int WARP_MMA = 1;
constexpr int EXP_PER_Q = 2;   // expansion warps per TMEM lane quarter (round-robin k-blocks)
constexpr int EXP_WARPS = 4 * EXP_PER_Q;
constexpr int WARP_EXP0 = 2;
constexpr int EPI_PER_Q = 2;   // epilogue warps per lane quarter (split the token columns)
constexpr int EPI_WARPS = 4 * EPI_PER_Q;
constexpr int WARP_EPI0 = WARP_EXP0 + EXP_WARPS;
constexpr int NUM_THREADS = (WARP_EPI0 + EPI_WARPS) * 32;

constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * X_STAGE_BYTES +
                           STAGES * RAW_STAGE_BYTES + 256 /*barriers etc*/;

__device__ __forceinline__ int sel_ftile(int fidx, int fcount, const int* fbase) {
  const int g = fidx / fcount;
  return fbase[g] + (fidx - g * fcount);
}

struct Params {
  int tokens;
  int n_rows;
  int n_ftiles, n_ttiles, k_blocks;
  int num_tiles;
  // Weight-tile selection: the nf = fgroups * fcount selected feature tiles
  // are fbase[g] + i (g < fgroups, i < fcount).
  int nf, fcount, fgroups;
  int fbase[kMaxTileGroups];
  const uint32_t* chunks;
  int nseg;
  EpiSeg seg[kMaxSegs];
  int* err;
  int fence_sys;  // a segment stores to other GPUs: fence.sys after the epilogue's stores
  // Test hook (bonsai_debug_stall_next_gemm): the load warp issues nothing,
  // so every other role's first bounded wait expires and the kernel unwinds
  // through its abort path with no copy or MMA in flight.  0 in normal use.
  int idle_loads;
};

__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))); hardware tanh (the
  // result is rounded to f16 right after, well below tanh.approx's error).
  const float k0 = 0.7978845608028654f;
  const float u = k0 * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanh_hw(u));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Expand one 32-input group: pair-split sign word p, f16 scale bits s.
// Output word j holds inputs (2j, 2j+1) as f16 +-s (low half = input 2j).
__device__ __forceinline__ void expand_group(uint32_t p, uint32_t s, uint32_t* out) {
  const uint32_t s2 = s | (s << 16);
  const uint32_t inv = ~p;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    out[j] = s2 ^ ((inv << (15 - j)) & 0x80008000u);
  }
}

template <bool kBF16>
__device__ __forceinline__ uint32_t bf16_from_f16_scale(uint32_t s16) {
  // bf16 operand mode: convert the f16 scale to bf16 bits (round-to-nearest).
  if constexpr (kBF16) {
    const float f = __half2float(__ushort_as_half((unsigned short)s16));
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
  } else {
    return s16;
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    b1_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint32_t* raw = reinterpret_cast<uint32_t*>(smem + STAGES * X_STAGE_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(raw + STAGES * kChunkWords);
  uint64_t* rawfull = full + STAGES;
  uint64_t* empty = rawfull + STAGES;
  uint64_t* dfull = empty + STAGES;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(&full[s], 1 + 4);  // TMA expect_tx arrival + 4 expansion warps
      bar_init(&rawfull[s], 1);
      bar_init(&empty[s], 1);     // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&dfull[b], 1);
      bar_init(&dempty[b], EPI_WARPS);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int k_blocks = p.k_blocks;

  if (warp == WARP_TMA) {
    if (elect_one() && !p.idle_loads) {
      tma_prefetch_desc(&xmap);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int ttile = tile / p.nf;
        const int ftile = sel_ftile(tile - ttile * p.nf, p.fcount, p.fbase);
        const uint32_t* wsrc = p.chunks + (size_t)ftile * k_blocks * kChunkWords;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_bar(&empty[s], ph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          bar_arrive_expect_tx(&rawfull[s], RAW_STAGE_BYTES);
          bulk_load(raw + s * kChunkWords, wsrc + (size_t)kb * kChunkWords, RAW_STAGE_BYTES,
                    &rawfull[s]);
          bar_arrive_expect_tx(&full[s], X_STAGE_BYTES);
          tma_load_2d(xs + s * X_STAGE_BYTES, &xmap, &full[s], kb * BK, ttile * BN);
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA's SMEM is released.
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == WARP_MMA) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(BM, BN, kBF16 ? 1 : 0, 0, 0);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++lt) {
        const uint32_t b = lt & 1;
        const uint32_t dph = (lt >> 1) & 1;
        if (!wait_bar(&dempty[b], dph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + D_COL0 + b * BN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_bar(&full[s], ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(xs + s * X_STAGE_BYTES);
#pragma unroll
          for (int k16 = 0; k16 < BK / 16; ++k16) {
            const uint32_t a_tmem = tmem + A_COL0 + s * 32 + k16 * 8;
            const uint64_t bdesc = make_smem_desc(xaddr + k16 * 32, 16, 1024);
            mma_ts(d_tmem, a_tmem, bdesc, idesc, (kb | k16) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&dfull[b]);
      }
      // Drain: wait until every MMA this thread issued has completed.
      tc_commit(drain);
      const uint32_t da = smem_u32(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!bar_try_wait(da, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          if (p.err) atomicCAS(p.err, 0, DEV_ERR_TIMEOUT_MMA);
          break;
        }
      }
    }
  } else if (warp >= WARP_EXP0 && warp < WARP_EXP0 + EXP_WARPS) {
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int r = q * 32 + (int)lane;   // weight row within the tile
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // The EXP_PER_Q warps of a quarter take pipeline iterations round-robin.
    // Each warp overlaps the tcgen05.st of one k-block with the expansion of
    // its next one: the stage is published (wait::st, arrive) only after the
    // following k-block's values are in registers.
    const uint32_t slot = (uint32_t)((warp - WARP_EXP0) >> 2);
    uint32_t it = 0;
    int pending = -1;  // stage whose tcgen05.st is in flight
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < k_blocks; ++kb, ++it) {
        if (it % EXP_PER_Q != slot) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        bool good = wait_bar(&rawfull[s], ph, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER) &&
                    wait_bar(&empty[s], ph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER);
        // tcgen05.st below is warp-collective: every lane must take the same path.
        if (!__all_sync(0xffffffffu, good)) {
          ok = false;
          break;
        }
        const uint32_t* rs = raw + s * kChunkWords;
        const uint32_t p0 = rs[r];
        const uint32_t p1 = rs[128 + r];
        const uint32_t sc = rs[256 + r];
        uint32_t v[32];
        expand_group(p0, bf16_from_f16_scale<kBF16>(sc & 0xFFFFu), v);
        expand_group(p1, bf16_from_f16_scale<kBF16>(sc >> 16), v + 16);
        if (pending >= 0) {
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) bar_arrive(&full[pending]);
        }
        tmem_st32(tmem + lane_base + A_COL0 + s * 32, v);
        pending = s;
      }
    }
    if (pending >= 0) {
      // Publish the last stage (also on the abort path: the MMA side is
      // bounded and ignores it).
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&full[pending]);
    }
  } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + EPI_WARPS) {
    const int q = warp & 3;
    const int eh = (warp - WARP_EPI0) >> 2;  // which half of the token columns
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
      const int ttile = tile / p.nf;
      const int ftile = sel_ftile(tile - ttile * p.nf, p.fcount, p.fbase);
      const uint32_t b = lt & 1;
      const uint32_t dph = (lt >> 1) & 1;
      const bool good = wait_bar(&dfull[b], dph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, good)) break;  // tcgen05.ld is warp-collective
      tc_fence_after();

      const int row = ftile * BM + q * 32 + (int)lane;
      int si = -1;
#pragma unroll
      for (int i = 0; i < kMaxSegs; ++i)
        if (i < p.nseg && row >= p.seg[i].row_begin && row < p.seg[i].row_end) si = i;
      // Segments are tile-aligned in every caller, but stay correct per row.
      EpiSeg sg;
      if (si >= 0) sg = p.seg[si];
      const int mode = si >= 0 ? sg.mode : -1;
      const int rr = row - sg.row_begin;
      float gate = 1.0f;
      if (mode == EPI_RESID_F32 && sg.gate) gate = sg.gate[rr];
      // Per-thread destination of token t: base + t * stride (elements).
      size_t base = 0;
      uint32_t stride = (uint32_t)sg.ld;
      if (mode == EPI_QKV_F16) {
        const int hd = sg.head_dim;
        const int which = rr / (sg.heads * hd);
        const int rem = rr - which * sg.heads * hd;
        const int h = rem / hd;
        const int d = rem - h * hd;
        base = ((size_t)(which * sg.heads + h) * sg.seq_total + sg.tok_off) * hd + d;
        stride = (uint32_t)hd;
        if (sg.route_heads > 0) {  // the head's owner (unrolled select: no dynamic indexing)
          const int owner = h / sg.route_heads;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r)
            if (r == owner) sg.dst = sg.route[r];
        }
      } else if (mode == EPI_SWIGLU_F16) {
        base = (size_t)sg.col_off + (rr >> 1);
      } else if (mode >= 0) {
        base = (size_t)sg.col_off + rr;
      }
      const bool warp_swiglu = __any_sync(0xffffffffu, mode == EPI_SWIGLU_F16);

#pragma unroll 1
      for (int cc = 0; cc < BN / 32 / EPI_PER_Q; ++cc) {
        const int c = eh * (BN / 32 / EPI_PER_Q) + cc;
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + D_COL0 + b * BN + c * 32, v);
        tmem_wait_ld();
        const int t0 = ttile * BN + c * 32;
        const int nt = min(32, p.tokens - t0);
        if (warp_swiglu) {
          // Rows are stored gate/value interleaved; the even lane owns the pair.
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
          const bool own = mode == EPI_SWIGLU_F16 && (rr & 1) == 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float a = __uint_as_float(v[j]);
            const float o = __shfl_xor_sync(0xffffffffu, a, 1);
            if (own && j < nt) dst[j * stride] = __float2half_rn(silu(a) * o);
          }
          continue;
        }
        if (mode < 0 || nt <= 0) continue;
        if (mode == EPI_F16 || mode == EPI_QKV_F16) {
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __float2half_rn(__uint_as_float(v[j]));
        } else if (mode == EPI_GELU_F16) {
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __float2half_rn(gelu_tanh(__uint_as_float(v[j])));
        } else if (mode == EPI_RESID_F32) {
          float* dst = reinterpret_cast<float*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int h16 = 0; h16 < 32; h16 += 16) {
            float old[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) old[j] = h16 + j < nt ? dst[(h16 + j) * stride] : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (h16 + j < nt) dst[(h16 + j) * stride] = fmaf(gate, __uint_as_float(v[h16 + j]), old[j]);
          }
        } else if (mode == EPI_F32) {
          float* dst = reinterpret_cast<float*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __uint_as_float(v[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&dempty[b]);
    }
    if (p.fence_sys) __threadfence_system();  // peer stores ordered before the kernel's end
  }

  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------- CTA-pair kernel (2 SMs)
// A cluster of two CTAs computes a 256-row x 256-token tile with
// tcgen05.mma.cta_group::2: each CTA expands its 128 weight rows into its
// own shared memory (128-byte-swizzled K-major, the layout TMA writes) and
// loads its 128-token half of the activation tile; the even CTA issues the
// MMAs and each CTA's TMEM receives its 128 rows x 256 tokens.
namespace pair {
constexpr int BM = 128;                  // weight rows per CTA (MMA M = 256 per pair)
constexpr int BN = 256;                  // tokens per pair tile (MMA N)
constexpr int BNH = BN / 2;              // tokens loaded by each CTA
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_STAGE_BYTES = BM * BK * 2;    // 16 KB
constexpr int X_STAGE_BYTES = BNH * BK * 2;   // 16 KB
constexpr int RAW_STAGE_BYTES = kChunkWords * 4;
constexpr int TMEM_COLS = 512;               // two 256-column accumulators
constexpr int WARP_TMA = 0;
constexpr int WARP_MMA = 1;
constexpr int EXP_PER_G = 2;                 // expansion warps per 32-row group
constexpr int EXP_WARPS = 4 * EXP_PER_G;
constexpr int WARP_EXP0 = 2;
constexpr int EPI_PER_Q = 2;
constexpr int EPI_WARPS = 4 * EPI_PER_Q;
constexpr int WARP_EPI0 = WARP_EXP0 + EXP_WARPS;
constexpr int NUM_THREADS = (WARP_EPI0 + EPI_WARPS) * 32;
constexpr int SMEM_BYTES = 1024 + STAGES * (A_STAGE_BYTES + X_STAGE_BYTES + RAW_STAGE_BYTES) + 256;

struct Params {
  int tokens;
  int n_ttiles, k_blocks;
  int npf;          // weight-tile pairs: selected tiles 2i and 2i+1
  int num_tiles;    // npf * n_ttiles * ksplit
  // K split: tile index = (ttile * npf + pf) * ksplit + ks; part ks covers
  // k-blocks [ks * kchunk, min(k_blocks, (ks + 1) * kchunk)).  ksplit > 1
  // only with gate-residual segments, whose epilogues then add atomically.
  int ksplit, kchunk;
  int nf, fcount, fgroups;
  int fbase[kMaxTileGroups];
  const uint32_t* chunks;
  int nseg;
  EpiSeg seg[kMaxSegs];
  int* err;
  int fence_sys;  // a segment stores to other GPUs: fence.sys after the epilogue's stores
};

template <bool kBF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    b1_gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* as = smem;
  uint8_t* xs = as + STAGES * A_STAGE_BYTES;
  uint32_t* raw = reinterpret_cast<uint32_t*>(xs + STAGES * X_STAGE_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(raw + STAGES * kChunkWords);
  uint64_t* rawfull = full + STAGES;
  uint64_t* empty = rawfull + STAGES;
  uint64_t* dfull = empty + STAGES;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();      // 0 = the CTA that issues the MMAs
  const int cid = (int)cluster_id_x();
  const int ncl = (int)cluster_count_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // even CTA: its producer's expect_tx arrival + 4 expansion warps per CTA
      bar_init(&full[s], 1 + 2 * 4);
      bar_init(&rawfull[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&dfull[b], 1);
      bar_init(&dempty[b], 2 * EPI_WARPS);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits and TMEM of both CTAs visible to the pair
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int k_blocks = p.k_blocks;

  if (warp == WARP_TMA) {
    if (elect_one()) {
      tma_prefetch_desc(&xmap);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cid; tile < p.num_tiles && ok; tile += ncl) {
        const int t2 = tile / p.ksplit;
        const int kb0 = (tile - t2 * p.ksplit) * p.kchunk;
        const int kb1 = min(k_blocks, kb0 + p.kchunk);
        const int ttile = t2 / p.npf;
        const int pf = t2 - ttile * p.npf;
        const int fidx = min(2 * pf + (int)rank, p.nf - 1);
        const int ftile = sel_ftile(fidx, p.fcount, p.fbase);
        const uint32_t* wsrc = p.chunks + (size_t)ftile * k_blocks * kChunkWords;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_bar(&empty[s], ph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          bar_arrive_expect_tx(&rawfull[s], RAW_STAGE_BYTES);
          bulk_load(raw + s * kChunkWords, wsrc + (size_t)kb * kChunkWords, RAW_STAGE_BYTES,
                    &rawfull[s]);
          if (rank == 0) bar_arrive_expect_tx(&full[s], 2 * X_STAGE_BYTES);
          tma_load_2d_pair(xs + s * X_STAGE_BYTES, &xmap, mapa_shared(smem_u32(&full[s]), 0),
                           kb * BK, ttile * BN + (int)rank * BNH);
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
        constexpr uint32_t idesc = make_idesc_f16(2 * BM, BN, kBF16 ? 1 : 0, 0, 0);
        uint32_t it = 0, lt = 0;
        bool ok = true;
        for (int tile = cid; tile < p.num_tiles && ok; tile += ncl, ++lt) {
          const uint32_t b = lt & 1;
          const uint32_t dph = (lt >> 1) & 1;
          if (!wait_bar(&dempty[b], dph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + b * BN;
          const int kb0 = (tile % p.ksplit) * p.kchunk;
          const int kb1 = min(k_blocks, kb0 + p.kchunk);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!wait_bar(&full[s], ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t aaddr = smem_u32(as + s * A_STAGE_BYTES);
            const uint32_t xaddr = smem_u32(xs + s * X_STAGE_BYTES);
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16) {
              const uint64_t adesc = make_smem_desc(aaddr + k16 * 32, 16, 1024);
              const uint64_t bdesc = make_smem_desc(xaddr + k16 * 32, 16, 1024);
              mma_ss_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k16 != 0) ? 1u : 0u);
            }
            tc_commit_pair(&empty[s], 0x3);
          }
          if (!ok) break;
          tc_commit_pair(&dfull[b], 0x3);
        }
        tc_commit_pair(drain, 0x3);
      }
      // Both CTAs: wait until every pair MMA has completed (the commit above
      // arrives on the drain barrier of each CTA).
      const uint32_t da = smem_u32(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!bar_try_wait(da, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          if (p.err) atomicCAS(p.err, 0, DEV_ERR_TIMEOUT_MMA);
          break;
        }
      }
    }
  } else if (warp >= WARP_EXP0 && warp < WARP_EXP0 + EXP_WARPS) {
    const int g = (warp - WARP_EXP0) & 3;   // 32-row group
    const uint32_t slot = (uint32_t)((warp - WARP_EXP0) >> 2);
    const int r = g * 32 + (int)lane;        // weight row within this CTA's 128
    const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);
    const uint32_t row_off = (uint32_t)r * 128u;
    const uint32_t sw = (uint32_t)(r & 7);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = cid; tile < p.num_tiles && ok; tile += ncl) {
      const int kb0 = (tile % p.ksplit) * p.kchunk;
      const int kb1 = min(k_blocks, kb0 + p.kchunk);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        if (it % EXP_PER_G != slot) continue;
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        const bool good =
            wait_bar(&rawfull[s], ph, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER) &&
            wait_bar(&empty[s], ph ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER);
        if (!__all_sync(0xffffffffu, good)) {
          ok = false;
          break;
        }
        const uint32_t* rs = raw + s * kChunkWords;
        const uint32_t p0 = rs[r];
        const uint32_t p1 = rs[128 + r];
        const uint32_t sc = rs[256 + r];
        uint32_t v[32];
        expand_group(p0, bf16_from_f16_scale<kBF16>(sc & 0xFFFFu), v);
        expand_group(p1, bf16_from_f16_scale<kBF16>(sc >> 16), v + 16);
        const uint32_t abase = smem_u32(as + s * A_STAGE_BYTES) + row_off;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(abase + (((uint32_t)c ^ sw) << 4), v[4 * c], v[4 * c + 1], v[4 * c + 2],
                       v[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) bar_arrive_remote(full0 + (uint32_t)s * 8u);
      }
    }
  } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + EPI_WARPS) {
    const int q = warp & 3;
    const int eh = (warp - WARP_EPI0) >> 2;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t dempty0 = mapa_shared(smem_u32(&dempty[0]), 0);
    uint32_t lt = 0;
    for (int tile = cid; tile < p.num_tiles; tile += ncl, ++lt) {
      const int t2 = tile / p.ksplit;
      const int ttile = t2 / p.npf;
      const int pf = t2 - ttile * p.npf;
      const int fidx = 2 * pf + (int)rank;
      const uint32_t b = lt & 1;
      const uint32_t dph = (lt >> 1) & 1;
      const bool good = wait_bar(&dfull[b], dph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, good)) break;
      tc_fence_after();

      int si = -1;
      int row = 0;
      if (fidx < p.nf) {
        row = sel_ftile(fidx, p.fcount, p.fbase) * BM + q * 32 + (int)lane;
#pragma unroll
        for (int i = 0; i < kMaxSegs; ++i)
          if (i < p.nseg && row >= p.seg[i].row_begin && row < p.seg[i].row_end) si = i;
      }
      EpiSeg sg;
      if (si >= 0) sg = p.seg[si];
      const int mode = si >= 0 ? sg.mode : -1;
      const int rr = row - sg.row_begin;
      float gate = 1.0f;
      if (mode == EPI_RESID_F32 && sg.gate) gate = sg.gate[rr];
      size_t base = 0;
      uint32_t stride = (uint32_t)sg.ld;
      if (mode == EPI_QKV_F16) {
        const int hd = sg.head_dim;
        const int which = rr / (sg.heads * hd);
        const int rem = rr - which * sg.heads * hd;
        const int h = rem / hd;
        const int d = rem - h * hd;
        base = ((size_t)(which * sg.heads + h) * sg.seq_total + sg.tok_off) * hd + d;
        stride = (uint32_t)hd;
        if (sg.route_heads > 0) {  // the head's owner (unrolled select: no dynamic indexing)
          const int owner = h / sg.route_heads;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r)
            if (r == owner) sg.dst = sg.route[r];
        }
      } else if (mode == EPI_SWIGLU_F16) {
        base = (size_t)sg.col_off + (rr >> 1);
      } else if (mode >= 0) {
        base = (size_t)sg.col_off + rr;
      }
      const bool warp_swiglu = __any_sync(0xffffffffu, mode == EPI_SWIGLU_F16);

#pragma unroll 1
      for (int cc = 0; cc < BN / 32 / EPI_PER_Q; ++cc) {
        const int c = eh * (BN / 32 / EPI_PER_Q) + cc;
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + b * BN + c * 32, v);
        tmem_wait_ld();
        const int t0 = ttile * BN + c * 32;
        const int nt = min(32, p.tokens - t0);
        if (warp_swiglu) {
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
          const bool own = mode == EPI_SWIGLU_F16 && (rr & 1) == 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float a = __uint_as_float(v[j]);
            const float o = __shfl_xor_sync(0xffffffffu, a, 1);
            if (own && j < nt) dst[j * stride] = __float2half_rn(silu(a) * o);
          }
          continue;
        }
        if (mode < 0 || nt <= 0) continue;
        if (mode == EPI_F16 || mode == EPI_QKV_F16) {
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __float2half_rn(__uint_as_float(v[j]));
        } else if (mode == EPI_GELU_F16) {
          __half* dst = reinterpret_cast<__half*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __float2half_rn(gelu_tanh(__uint_as_float(v[j])));
        } else if (mode == EPI_RESID_F32 && p.ksplit > 1) {
          // this K part's share of h += gate * acc; the other part adds its own
          float* dst = reinterpret_cast<float*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) atomicAdd(dst + (size_t)j * stride, gate * __uint_as_float(v[j]));
        } else if (mode == EPI_RESID_F32) {
          float* dst = reinterpret_cast<float*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int h16 = 0; h16 < 32; h16 += 16) {
            float old[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) old[j] = h16 + j < nt ? dst[(h16 + j) * stride] : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (h16 + j < nt) dst[(h16 + j) * stride] = fmaf(gate, __uint_as_float(v[h16 + j]), old[j]);
          }
        } else if (mode == EPI_F32) {
          float* dst = reinterpret_cast<float*>(sg.dst) + base + (size_t)t0 * stride;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nt) dst[j * stride] = __uint_as_float(v[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive_remote(dempty0 + b * 8u);
    }
    if (p.fence_sys) __threadfence_system();  // peer stores ordered before the kernel's end
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no pair MMA, remote arrive or TMEM access is left in either CTA
  if (warp == WARP_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}
}  // namespace pair

// ------------------------------------------------------------ retile kernel
__device__ __forceinline__ uint32_t compress_even_bits(uint32_t x) {
  x &= 0x55555555u;
  x = (x | (x >> 1)) & 0x33333333u;
  x = (x | (x >> 2)) & 0x0F0F0F0Fu;
  x = (x | (x >> 4)) & 0x00FF00FFu;
  x = (x | (x >> 8)) & 0x0000FFFFu;
  return x;
}

// Device row n of the retiled weight reads source row src_row(n): rows in
// [swiglu_from, N) are interleaved so that device row swiglu_from + 2j is
// source row swiglu_from + j (gate) and device row swiglu_from + 2j + 1 is
// source row swiglu_from + half + j (value).
__global__ void b1_retile_kernel(const uint8_t* __restrict__ src, uint32_t* __restrict__ dst,
                                 int N, int K, int n_ftiles, int k_blocks, int swiglu_from) {
  const long long total = (long long)n_ftiles * 128 * k_blocks;
  const int groups = K / 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i % 128);
    const long long rest = i / 128;
    const int kb = (int)(rest % k_blocks);
    const int ftile = (int)(rest / k_blocks);
    const int n = ftile * 128 + r;
    uint32_t words[2] = {0u, 0u};
    uint32_t scales[2] = {0u, 0u};
    if (n < N) {
      int srow = n;
      if (swiglu_from >= 0 && n >= swiglu_from) {
        const int half = (N - swiglu_from) / 2;
        const int j = n - swiglu_from;
        srow = swiglu_from + ((j & 1) ? half + (j >> 1) : (j >> 1));
      }
      for (int g = 0; g < 2; ++g) {
        const int grp = kb * 2 + g;
        if (grp < groups) {
          const uint8_t* b = src + ((size_t)srow * groups + grp) * 6;
          const uint32_t s = (uint32_t)b[0] | ((uint32_t)b[1] << 8);
          const uint32_t bits = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) |
                                ((uint32_t)b[5] << 24);
          words[g] = compress_even_bits(bits) | (compress_even_bits(bits >> 1) << 16);
          scales[g] = s;
        }
      }
    }
    uint32_t* c = dst + ((size_t)ftile * k_blocks + kb) * kChunkWords;
    c[r] = words[0];
    c[128 + r] = words[1];
    c[256 + r] = scales[0] | (scales[1] << 16);
  }
}

// Inverse of compress_even_bits: bit j of x (j < 16) -> bit 2j.
__device__ __forceinline__ uint32_t spread_even_bits(uint32_t x) {
  x &= 0x0000FFFFu;
  x = (x | (x << 8)) & 0x00FF00FFu;
  x = (x | (x << 4)) & 0x0F0F0F0Fu;
  x = (x | (x << 2)) & 0x33333333u;
  x = (x | (x << 1)) & 0x55555555u;
  return x;
}

// Packed row srow, group grp <- device chunks (the exact inverse of
// b1_retile_kernel, including the SwiGLU row interleave).
__global__ void b1_unretile_kernel(const uint32_t* __restrict__ chunks, uint8_t* __restrict__ dst,
                                   int N, int K, int k_blocks, int swiglu_from) {
  const int groups = K / 32;
  const long long total = (long long)N * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int srow = (int)(i / groups);
    const int grp = (int)(i - (long long)srow * groups);
    int n = srow;
    if (swiglu_from >= 0 && srow >= swiglu_from) {
      const int half = (N - swiglu_from) / 2;
      const int j = srow - swiglu_from;
      n = swiglu_from + (j < half ? 2 * j : 2 * (j - half) + 1);
    }
    const int ftile = n / 128, r = n % 128, kb = grp / 2, g = grp & 1;
    const uint32_t* c = chunks + ((size_t)ftile * k_blocks + kb) * kChunkWords;
    const uint32_t word = c[g * 128 + r];
    const uint32_t sc = (c[256 + r] >> (16 * g)) & 0xFFFFu;
    const uint32_t bits = spread_even_bits(word) | (spread_even_bits(word >> 16) << 1);
    uint8_t* o = dst + ((size_t)srow * groups + grp) * 6;
    o[0] = (uint8_t)(sc & 0xFF);
    o[1] = (uint8_t)(sc >> 8);
    o[2] = (uint8_t)(bits & 0xFF);
    o[3] = (uint8_t)((bits >> 8) & 0xFF);
    o[4] = (uint8_t)((bits >> 16) & 0xFF);
    o[5] = (uint8_t)(bits >> 24);
  }
}

// -------------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// ------------------------------------------------------------------------
// B1_0 GEMV: y[n] = sum_k W[n][k] x[k] for ONE activation row, on the
// chunked device layout.  A matrix-vector product has no reuse for the
// tensor cores (a 128-token GEMM tile would be 127/128 padding); it is bound
// by streaming the 6 bytes per 32 weights from HBM.  Each CTA first builds,
// in shared memory, a table of signed partial sums of x: for every 32-input
// group, every 4-bit nibble of its sign word (pair-split order: bit j is
// input 2j, bit j + 16 input 2j + 1) and every value v of that nibble, the
// sum over the nibble's four inputs of (bit ? +x : -x).  A row's group sum
// is then eight table lookups, scaled by the group's f16 scale, which is
// the reference's sum_i (bit ? +x_i : -x_i) * scale (src/b1_0_kernel.h:
// 240-287) with x in f32.  Thread r of each 128-thread half handles row r of
// one 128-row tile; a tile's sign words and scales are read coalesced
// (128 consecutive u32 per array).  The 16 entries of one nibble's table are
// consecutive floats, so a warp's lookups into one table hit 16 distinct
// banks: no conflicts.
constexpr int kGemvThreads = 256;
constexpr int kGemvMaxKBlocks = 128;  // table = k_blocks KB of shared memory (K <= 8192)
constexpr int kGemvBatch = 8;         // k-blocks whose weight words are loaded together

__global__ void __launch_bounds__(kGemvThreads) b1_gemv_kernel(
    const float* __restrict__ x, const uint32_t* __restrict__ chunks, int n_rows, int k_in,
    int n_ftiles, int k_blocks, float* __restrict__ y) {
  extern __shared__ float lut[];  // [k_blocks][2 groups][8 nibbles][16 values]
  const int entries = k_blocks * 256;
  for (int e = threadIdx.x; e < entries; e += blockDim.x) {
    const int v = e & 15, nib = (e >> 4) & 7, g = (e >> 7) & 1, kb = e >> 8;
    const int base = kb * 64 + g * 32 + (nib < 4 ? 8 * nib : 8 * (nib - 4) + 1);
    float sum = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int k = base + 2 * t;
      const float xv = k < k_in ? x[k] : 0.f;
      sum += ((v >> t) & 1) ? xv : -xv;
    }
    lut[e] = sum;
  }
  __syncthreads();
  const int r = threadIdx.x & 127;
  for (int ft = blockIdx.x * 2 + (threadIdx.x >> 7); ft < n_ftiles; ft += gridDim.x * 2) {
    const uint32_t* c = chunks + (size_t)ft * k_blocks * kChunkWords;
    float acc = 0.f;
    // kGemvBatch k-blocks' words are loaded before any is used, so that
    // 3 * kGemvBatch loads per thread are in flight (the kernel is bound by
    // the latency of this weight stream, not by its bandwidth, otherwise).
    for (int kb0 = 0; kb0 < k_blocks; kb0 += kGemvBatch) {
      uint32_t w0[kGemvBatch], w1[kGemvBatch], sc[kGemvBatch];
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) {
        const uint32_t* ck = c + (size_t)(kb0 + u) * kChunkWords;
        const bool in = kb0 + u < k_blocks;
        w0[u] = in ? __ldcs(ck + r) : 0u;
        w1[u] = in ? __ldcs(ck + 128 + r) : 0u;
        sc[u] = in ? __ldcs(ck + 256 + r) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kGemvBatch; ++u) {
        if (kb0 + u >= k_blocks) break;
        const float* l0 = lut + (kb0 + u) * 256;
        const float* l1 = l0 + 128;
        float p0 = 0.f, p1 = 0.f;
#pragma unroll
        for (int nib = 0; nib < 8; ++nib) {
          p0 += l0[nib * 16 + ((w0[u] >> (4 * nib)) & 15)];
          p1 += l1[nib * 16 + ((w1[u] >> (4 * nib)) & 15)];
        }
        acc = fmaf(__half2float(__ushort_as_half((unsigned short)(sc[u] & 0xffffu))), p0, acc);
        acc = fmaf(__half2float(__ushort_as_half((unsigned short)(sc[u] >> 16))), p1, acc);
      }
    }
    const int n = ft * 128 + r;
    if (n < n_rows) y[n] = acc;
  }
}

}  // namespace gemm

// 2-D row-major [rows][cols] 16-bit tensor, box {box_cols, box_rows}, 128B swizzle.
int encode_tmap_2d_16b(CUtensorMap* map, const void* base, long long rows, long long cols,
                       long long ld, int box_cols, int box_rows, bool bf16) {
  auto fn = gemm::get_encode_fn();
  if (!fn) return fail(-5, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(-5, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return 0;
}

// 3-D head-major [n_heads][seq][head_dim] f16 tensor, box {64, box_rows, 1}, 128B swizzle.
int encode_tmap_heads(CUtensorMap* map, const void* base, int n_heads, int seq, int head_dim,
                      int box_rows) {
  auto fn = gemm::get_encode_fn();
  if (!fn) return fail(-5, "cuTensorMapEncodeTiled entry point unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(-1, "attention: q/k/v must be 16-byte aligned");
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)seq, (cuuint64_t)n_heads};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)seq * head_dim * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(-5, "cuTensorMapEncodeTiled (heads) failed (code " + std::to_string((int)r) + ")");
  return 0;
}

int launch_b1_retile(const uint8_t* dev_packed, B1Weight& w, cudaStream_t st) {
  const long long total = (long long)w.n_ftiles * 128 * w.k_blocks;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 65535LL * 8);
  gemm::b1_retile_kernel<<<(unsigned)blocks, threads, 0, st>>>(dev_packed, w.chunks, w.n_rows,
                                                               w.k_in, w.n_ftiles, w.k_blocks,
                                                               w.swiglu_from);
  return launch_status("b1_retile_kernel launch");
}

namespace {

enum class B1Kernel { Auto, Single, Pair };

B1Kernel forced_kernel() {
  const char* e = getenv("BONSAI_B1_KERNEL");
  if (!e) return B1Kernel::Auto;
  if (strcmp(e, "pair") == 0) return B1Kernel::Pair;
  if (strcmp(e, "single") == 0) return B1Kernel::Single;
  return B1Kernel::Auto;
}

// Largest number of co-resident pair clusters (one per TPC when every SM
// takes one CTA of the pair kernel); 0 if the query fails.
int pair_cluster_slots(bool bf16) {
  struct Slots {
    int n[2] = {-1, -1};
  };
  static Slots slots[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int& n = slots[device_slot()].n[bf16 ? 1 : 0];
  if (n >= 0) return n;
  auto k2 = bf16 ? gemm::pair::b1_gemm_pair_kernel<true> : gemm::pair::b1_gemm_pair_kernel<false>;
  n = 0;
  if (cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           gemm::pair::SMEM_BYTES) != cudaSuccess)
    return n;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * std::max(1, num_sms() / 2));
  cfg.blockDim = dim3(gemm::pair::NUM_THREADS);
  cfg.dynamicSmemBytes = gemm::pair::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int c = 0;
  if (cudaOccupancyMaxActiveClusters(&c, k2, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return n;
  }
  n = c;
  return n;
}

}  // namespace

int launch_b1_unretile(const B1Weight& w, uint8_t* dev_packed, cudaStream_t st) {
  const long long total = (long long)w.n_rows * (w.k_in / 32);
  if (total <= 0) return 0;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 65535LL * 8);
  gemm::b1_unretile_kernel<<<(unsigned)blocks, threads, 0, st>>>(w.chunks, dev_packed, w.n_rows,
                                                                 w.k_in, w.k_blocks,
                                                                 w.swiglu_from);
  return launch_status("b1_unretile_kernel launch");
}

// Set by bonsai_debug_stall_next_gemm, consumed by the next launch on the thread.
thread_local bool g_stall_next_gemm = false;

bool b1_gemv_supported(const B1Weight& w) {
  return w.swiglu_from < 0 && w.k_blocks >= 1 && w.k_blocks <= gemm::kGemvMaxKBlocks;
}

int launch_b1_gemv_f32(const float* x, const B1Weight& w, float* y, cudaStream_t st) {
  if (!x || !y || !w.chunks) return fail(-1, "b1_gemv: null argument");
  if (!b1_gemv_supported(w))
    return fail(-2, "b1_gemv: needs in_dim <= 8192 and a weight without the SwiGLU interleave");
  const int smem = w.k_blocks * 256 * (int)sizeof(float);
  static bool attr_dev[64] = {};
  bool& attr = attr_dev[device_slot()];
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(gemm::b1_gemv_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               gemm::kGemvMaxKBlocks * 256 * (int)sizeof(float));
    if (e != cudaSuccess) return cuda_status(e, "b1_gemv set smem attribute");
    attr = true;
  }
  // enough CTAs to keep the weight stream in flight on every SM; each builds
  // its own table once and then walks tiles
  const int tile_pairs = (w.n_ftiles + 1) / 2;
  const int grid = std::max(1, std::min(tile_pairs, num_sms() * 4));
  ProfScope prof("b1_gemv", 2.0 * w.n_rows * (double)w.k_in,
                 (double)w.k_in * 4 + (double)w.n_rows * w.k_in * 6 / 32 + w.n_rows * 4.0, st);
  gemm::b1_gemv_kernel<<<grid, gemm::kGemvThreads, smem, st>>>(x, w.chunks, w.n_rows, w.k_in,
                                                                w.n_ftiles, w.k_blocks, y);
  return launch_status("b1_gemv_kernel launch");
}

int launch_b1_gemm(const void* x, long long ldx, int tokens, const B1Weight& w, const EpiSeg* segs,
                   int nseg, bool x_bf16, cudaStream_t st, const TileSel* sel) {
  if (tokens < 0) return fail(-1, "b1_gemm: negative token count");
  if (tokens == 0) return 0;
  if (!x || !w.chunks) return fail(-1, "b1_gemm: null activation or weight");
  if (nseg < 1 || nseg > kMaxSegs) return fail(-1, "b1_gemm: bad segment count");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0 || ldx < w.k_in)
    return fail(-1, "b1_gemm: activation must be 16-byte aligned with ld % 8 == 0 and ld >= K");

  // Weight-tile selection: the nf = groups * count selected 128-row tiles
  // are base[g] + i (g < groups, i < count).
  int fgroups = 1, fcount = w.n_ftiles;
  int fbase[kMaxTileGroups] = {0, 0, 0};
  if (sel) {
    if (sel->groups < 1 || sel->groups > kMaxTileGroups || sel->count < 1)
      return fail(-1, "b1_gemm: bad tile selection");
    for (int g = 0; g < sel->groups; ++g)
      if (sel->base[g] < 0 || sel->base[g] + sel->count > w.n_ftiles)
        return fail(-1, "b1_gemm: tile selection outside the weight");
    fgroups = sel->groups;
    fcount = sel->count;
    for (int g = 0; g < sel->groups; ++g) fbase[g] = sel->base[g];
  }
  const int nf = fgroups * fcount;
  bool routed = false;
  for (int i = 0; i < nseg; ++i) {
    if (segs[i].route_heads <= 0) continue;
    if (segs[i].mode != EPI_QKV_F16 || segs[i].heads % segs[i].route_heads != 0)
      return fail(-1, "b1_gemm: head routing needs a QKV segment whose heads divide by route_heads");
    for (int r = 0; r < segs[i].heads / segs[i].route_heads; ++r)
      if (!segs[i].route[r]) return fail(-1, "b1_gemm: null head route");
    routed = true;
  }

  // Kernel choice: estimated time = waves x tile time, with a 256x256 pair
  // tile (two SMs) taking kPairTileCost 128x128-tile times of one SM (about
  // 2 x 1255 / 1536 from isolated measurements of the two kernels).
  const int slots = pair_cluster_slots(x_bf16);
  const int n_tt1 = (tokens + gemm::BN - 1) / gemm::BN;
  const int n_tt2 = (tokens + gemm::pair::BN - 1) / gemm::pair::BN;
  const long long tiles1 = (long long)nf * n_tt1;
  const long long tiles2 = (long long)((nf + 1) / 2) * n_tt2;
  constexpr double kPairTileCost = 1.63;
  // K split of the pair kernel: only for launches whose every segment is a
  // gate-residual that allows it (split_ok: the partitioned multi-GPU step),
  // where doubling the work units fills the last wave of clusters better
  // (e.g. 108 tiles on 74 clusters: 2 waves of whole tiles, 3 of half
  // tiles); BONSAI_B1_SPLITK=n forces n parts on any gate-residual launch
  // (tests).
  bool all_resid = true, all_split_ok = true;
  for (int i = 0; i < nseg; ++i) {
    all_resid = all_resid && segs[i].mode == EPI_RESID_F32;
    all_split_ok = all_split_ok && segs[i].mode == EPI_RESID_F32 && segs[i].split_ok;
  }
  int ksplit = 1;
  if (const char* e = getenv("BONSAI_B1_SPLITK")) {
    if (all_resid) ksplit = std::max(1, std::min(atoi(e), std::max(1, w.k_blocks / 2)));
  } else if (all_split_ok && w.k_blocks >= 16 && slots >= 1 && tiles2 >= slots) {
    // (a launch below one wave -- the 512-token text stream -- keeps whole
    // tiles: its result then stays bit-identical to the unpartitioned step)
    const double whole = (double)((tiles2 + slots - 1) / slots);
    const double half = 0.5 * (double)((2 * tiles2 + slots - 1) / slots);
    // >= 20% fewer waves (8 GPUs: 2 -> 1.5); a smaller modelled gain (rank
    // 0's image rows at 4 GPUs: 3 -> 2.5 waves) measured nothing, and whole
    // tiles keep the result bit-identical to the unpartitioned forward
    if (half < 0.8 * whole) ksplit = 2;
  }
  bool use_pair = false;
  const B1Kernel force = forced_kernel();
  const bool stall = g_stall_next_gemm;  // test hook: this launch runs the one-CTA kernel idle
  g_stall_next_gemm = false;
  if (stall) {
    use_pair = false;
  } else if (force == B1Kernel::Pair) {
    if (slots < 1) return fail(-3, "b1_gemm: the pair kernel cannot be scheduled on this device");
    use_pair = true;
  } else if (force == B1Kernel::Auto && slots >= 1) {
    const double t1 = (double)((tiles1 + num_sms() - 1) / num_sms());
    const double t2 = kPairTileCost * (double)((tiles2 * ksplit + slots - 1) / slots) / ksplit;
    use_pair = t2 < t1;
  }

  double out_bytes = 0;
  for (int i = 0; i < nseg; ++i) {
    const double rows = segs[i].row_end - segs[i].row_begin;
    const int m = segs[i].mode;
    const double per = (m == EPI_F32) ? 4 : (m == EPI_RESID_F32) ? 8 : (m == EPI_SWIGLU_F16) ? 1 : 2;
    out_bytes += rows * tokens * per;
  }
  const double rows_done = sel ? std::min<double>(w.n_rows, 128.0 * nf) : (double)w.n_rows;
  if (sel) out_bytes *= rows_done / std::max(1, w.n_rows);

  if (use_pair) {
    CUtensorMap xmap;
    int rc = encode_tmap_2d_16b(&xmap, x, tokens, w.k_in, ldx, gemm::pair::BK, gemm::pair::BNH,
                                x_bf16);
    if (rc) return rc;
    gemm::pair::Params q{};
    q.tokens = tokens;
    q.n_ttiles = n_tt2;
    q.k_blocks = w.k_blocks;
    q.nf = nf;
    q.fcount = fcount;
    q.fgroups = fgroups;
    for (int g = 0; g < kMaxTileGroups; ++g) q.fbase[g] = fbase[g];
    q.npf = (nf + 1) / 2;
    q.kchunk = (w.k_blocks + ksplit - 1) / ksplit;
    q.ksplit = (w.k_blocks + q.kchunk - 1) / q.kchunk;  // every part gets >= 1 k-block
    q.num_tiles = (int)(tiles2 * q.ksplit);
    q.chunks = w.chunks;
    q.nseg = nseg;
    for (int i = 0; i < nseg; ++i) q.seg[i] = segs[i];
    q.err = device_error_word();
    q.fence_sys = routed ? 1 : 0;
    auto k2 = x_bf16 ? gemm::pair::b1_gemm_pair_kernel<true> : gemm::pair::b1_gemm_pair_kernel<false>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (unsigned)std::min<long long>(tiles2, slots));
    cfg.blockDim = dim3(gemm::pair::NUM_THREADS);
    cfg.dynamicSmemBytes = gemm::pair::SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfScope prof("b1_gemm", 2.0 * tokens * rows_done * (double)w.k_in,
                   (double)tokens * w.k_in * 2 + rows_done * w.k_in * 6 / 32 + out_bytes, st);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k2, xmap, q);
    if (e != cudaSuccess) return cuda_status(e, "b1_gemm_pair_kernel launch");
    return launch_status("b1_gemm_pair_kernel launch");
  }

  CUtensorMap xmap;
  int rc = encode_tmap_2d_16b(&xmap, x, tokens, w.k_in, ldx, gemm::BK, gemm::BN, x_bf16);
  if (rc) return rc;
  gemm::Params p{};
  p.tokens = tokens;
  p.n_rows = w.n_rows;
  p.n_ftiles = w.n_ftiles;
  p.n_ttiles = n_tt1;
  p.k_blocks = w.k_blocks;
  p.fgroups = fgroups;
  p.fcount = fcount;
  for (int g = 0; g < kMaxTileGroups; ++g) p.fbase[g] = fbase[g];
  p.nf = nf;
  p.num_tiles = (int)tiles1;
  p.chunks = w.chunks;
  p.nseg = nseg;
  for (int i = 0; i < nseg; ++i) p.seg[i] = segs[i];
  p.err = device_error_word();
  p.fence_sys = routed ? 1 : 0;
  p.idle_loads = stall ? 1 : 0;

  const int grid = (int)std::min<long long>(tiles1, num_sms());
  auto kern = x_bf16 ? gemm::b1_gemm_kernel<true> : gemm::b1_gemm_kernel<false>;
  static bool attr_set[64][2] = {};
  bool& attr_done = attr_set[device_slot()][x_bf16 ? 1 : 0];
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_status(e, "b1_gemm set smem attribute");
    attr_done = true;
  }
  ProfScope prof("b1_gemm", 2.0 * tokens * rows_done * (double)w.k_in,
                 (double)tokens * w.k_in * 2 + rows_done * w.k_in * 6 / 32 + out_bytes, st);
  kern<<<grid, gemm::NUM_THREADS, gemm::SMEM_BYTES, st>>>(xmap, p);
  return launch_status("b1_gemm_kernel launch");
}

}  // namespace bonsai

extern "C" int bonsai_debug_stall_next_gemm(void) {
  bonsai::g_stall_next_gemm = true;
  return 0;
}
