// B1_0 1-bit-weight GEMM for sm_100a (tcgen05 / TMEM / TMA).
//
// Replaces the reference's b1_linear_f32_f32 (src/b1_0_kernel.h:37-288),
// which computes out[t][r] = sum_blk scale[r][blk] * sum_i (bit ? +x : -x)
// over the packed layout of src/diffuser_types.h:10-11 /
// convert_to_b1_0_packed.py:21-43.
//
// Design (weights-as-A, tokens-as-B):
//   * The MMA computes D[128 weight rows][128 tokens] += A * B^T with
//     A = expanded weights held in TMEM and B = activation tile in SMEM.
//   * Four expansion warps turn the retiled sign words + fp16 scales into
//     exact f16 +-scale values in registers and write them straight into
//     TMEM with tcgen05.st: the expanded weights never touch shared memory,
//     so SMEM bandwidth is spent only on the activations.
//   * A TMA warp streams activation tiles (128 tokens x 64 k, 128-byte
//     swizzle) and the 1.5 KB weight chunk of each k-block.
//   * One thread issues tcgen05.mma (A from TMEM, B from SMEM descriptor).
//   * Four epilogue warps drain the double-buffered accumulator with
//     tcgen05.ld and apply the fused epilogue (store, GELU, SwiGLU,
//     gate-residual, head-major QKV scatter).
//   * Persistent grid: one CTA per SM walks the tile list.
#include "internal.cuh"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <cstdio>
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
    if (elect_one()) {
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
  }

  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

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

// 3-D head-major [n_heads][seq][head_dim] f16 tensor, box {64, 128, 1}, 128B swizzle.
int encode_tmap_heads(CUtensorMap* map, const void* base, int n_heads, int seq, int head_dim) {
  auto fn = gemm::get_encode_fn();
  if (!fn) return fail(-5, "cuTensorMapEncodeTiled entry point unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(-1, "attention: q/k/v must be 16-byte aligned");
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)seq, (cuuint64_t)n_heads};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)seq * head_dim * 2};
  cuuint32_t box[3] = {64, 128, 1};
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

int launch_b1_gemm(const void* x, long long ldx, int tokens, const B1Weight& w, const EpiSeg* segs,
                   int nseg, bool x_bf16, cudaStream_t st, const TileSel* sel) {
  if (tokens < 0) return fail(-1, "b1_gemm: negative token count");
  if (tokens == 0) return 0;
  if (!x || !w.chunks) return fail(-1, "b1_gemm: null activation or weight");
  if (nseg < 1 || nseg > kMaxSegs) return fail(-1, "b1_gemm: bad segment count");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (ldx % 8) != 0 || ldx < w.k_in)
    return fail(-1, "b1_gemm: activation must be 16-byte aligned with ld % 8 == 0 and ld >= K");
  CUtensorMap xmap;
  int rc = encode_tmap_2d_16b(&xmap, x, tokens, w.k_in, ldx, gemm::BK, gemm::BN, x_bf16);
  if (rc) return rc;

  gemm::Params p{};
  p.tokens = tokens;
  p.n_rows = w.n_rows;
  p.n_ftiles = w.n_ftiles;
  p.n_ttiles = (tokens + gemm::BN - 1) / gemm::BN;
  p.k_blocks = w.k_blocks;
  if (sel) {
    if (sel->groups < 1 || sel->groups > kMaxTileGroups || sel->count < 1)
      return fail(-1, "b1_gemm: bad tile selection");
    for (int g = 0; g < sel->groups; ++g)
      if (sel->base[g] < 0 || sel->base[g] + sel->count > w.n_ftiles)
        return fail(-1, "b1_gemm: tile selection outside the weight");
    p.fgroups = sel->groups;
    p.fcount = sel->count;
    for (int g = 0; g < sel->groups; ++g) p.fbase[g] = sel->base[g];
  } else {
    p.fgroups = 1;
    p.fcount = w.n_ftiles;
    p.fbase[0] = 0;
  }
  p.nf = p.fgroups * p.fcount;
  p.num_tiles = p.nf * p.n_ttiles;
  p.chunks = w.chunks;
  p.nseg = nseg;
  for (int i = 0; i < nseg; ++i) p.seg[i] = segs[i];
  p.err = device_error_word();

  const int grid = std::min(p.num_tiles, num_sms());
  auto kern = x_bf16 ? gemm::b1_gemm_kernel<true> : gemm::b1_gemm_kernel<false>;
  static bool attr_set[2] = {false, false};
  if (!attr_set[x_bf16 ? 1 : 0]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_status(e, "b1_gemm set smem attribute");
    attr_set[x_bf16 ? 1 : 0] = true;
  }
  double out_bytes = 0;
  for (int i = 0; i < nseg; ++i) {
    const double rows = segs[i].row_end - segs[i].row_begin;
    const int m = segs[i].mode;
    const double per = (m == EPI_F32) ? 4 : (m == EPI_RESID_F32) ? 8 : (m == EPI_SWIGLU_F16) ? 1 : 2;
    out_bytes += rows * tokens * per;
  }
  const double rows_done = sel ? std::min<double>(w.n_rows, 128.0 * p.nf) : (double)w.n_rows;
  if (sel) out_bytes *= rows_done / std::max(1, w.n_rows);
  ProfScope prof("b1_gemm", 2.0 * tokens * rows_done * (double)w.k_in,
                 (double)tokens * w.k_in * 2 + rows_done * w.k_in * 6 / 32 + out_bytes, st);
  kern<<<grid, gemm::NUM_THREADS, gemm::SMEM_BYTES, st>>>(xmap, p);
  return launch_status("b1_gemm_kernel launch");
}

}  // namespace bonsai
