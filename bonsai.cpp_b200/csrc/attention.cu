// Joint (text + image) non-causal attention for sm_100a.
//
// Replaces ggml_flash_attn_ext as the reference calls it
// (src/diffuser_graph.cpp:403-416 double blocks, :506-519 single blocks):
// softmax(Q K^T * scale) V per head, no mask, K and V in f16, f32 softmax.
//
// One CTA = one head x 256 queries, processed as two 128-query tiles that
// ping-pong on the tensor core: while the softmax warps of one tile work,
// the MMA thread runs the other tile's P*V and its next Q*K^T.
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1: thread i
//               owns query row i (TMEM lane i).  Online softmax in the log2
//               domain with lazy rescaling: the running max only moves (and
//               O_g in TMEM is rescaled) when a tile's max exceeds it by more
//               than 8 (p <= 2^8 stays accurate in f16); the final 1/l is
//               exact.  Scale/subtract and the row sum use packed f32x2 ops.
//   warp 8      TMA: Q0/Q1 once, then K_j / V_j tiles (128 keys x 128 dims,
//               two 64-dim halves, 128-byte swizzle) through 2-deep rings.
//   warp 9      one thread issues tcgen05.mma:
//                 S_g  = Q_g K_j^T   (A, B from SMEM)          g = 0, 1
//                 O_g += P_g V_j     (A = P_g from TMEM, B = V MN-major)
//   warps 10-11 idle (they complete the third warpgroup).
// setmaxnreg gives the softmax warpgroups 224 registers per thread (the whole
// S row stays in registers) and the TMA/MMA warpgroup 56; the three
// warpgroups' code paths never rejoin, so each keeps its own budget, and the
// MMA warp frees TMEM after every softmax warp has signalled it is done.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// P_g (f16 pairs, 64 columns) overwrites the first half of S_g once the
// softmax has read S_g; the next S_g is issued after P_g V_j in the same
// in-order MMA stream.
#include "internal.cuh"
#include "ptx.cuh"

#include <cudaTypedefs.h>

namespace bonsai {
namespace attn {

constexpr int BQ = 128;   // queries per tile (two tiles per CTA)
constexpr int BKV = 128;
constexpr int HD = 128;
constexpr int KS = 2;  // K ring depth
constexpr int VS = 2;  // V ring depth
constexpr int TILE_BYTES = BKV * HD * 2;  // 32 KB (two 16 KB halves)
constexpr int HALF_BYTES = TILE_BYTES / 2;
// Warpgroup 0: softmax of query tile 0, warpgroup 1: tile 1 (one thread per
// query row); warpgroup 2: TMA warp, MMA warp and two idle warps.  setmaxnreg
// moves registers from warpgroup 2 to the softmax warpgroups.
constexpr int NUM_THREADS = 384;
constexpr int WARP_TMA = 8;
constexpr int WARP_MMA = 9;
constexpr int kLaunchRegs = 168;   // 65536 / 384, rounded down to 8
constexpr int kSoftmaxRegs = 224;
constexpr int kAuxRegs = 56;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kAuxRegs <= NUM_THREADS * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0, O_COL = 256;
constexpr int SMEM_BYTES = 1024 + TILE_BYTES * (2 + KS + VS) + 256;
constexpr float kRescaleThreshold = 8.0f;

struct Params {
  int seq;
  int n_heads;
  float scale_log2;  // softmax scale * log2(e)
  __half* out;
  long long ld_out;
  RowRoutes routes;  // routes.n == 0: every row through out
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed pairs of f32 in one 64-bit register (Blackwell f32x2 FMA pipe).
__device__ __forceinline__ unsigned long long pack2(float a, float b) {
  unsigned long long d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t cvt_h2(float lo, float hi) {
  uint32_t y;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(y) : "f"(hi), "f"(lo));
  return y;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* qs = smem;  // Q0 then Q1
  uint8_t* ks = qs + 2 * TILE_BYTES;
  uint8_t* vs = ks + KS * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + VS * TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;   // [2] one per query tile
  uint64_t* p_ready = s_full + 2;    // [2]
  uint64_t* pv_done = p_ready + 2;   // [2]
  uint64_t* drain = pv_done + 2;
  uint64_t* sm_done = drain + 1;     // softmax warps finished with TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * 2 * BQ;
  const int nkv = (p.seq + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      bar_init(&v_full[s], 1);
      bar_init(&v_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      bar_init(&s_full[g], 1);
      bar_init(&p_ready[g], 4);
      bar_init(&pv_done[g], 1);
    }
    bar_init(drain, 1);
    bar_init(sm_done, 8);
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

  if (warp >= 8) {
  regs_dec<kAuxRegs>();
  if (warp == WARP_TMA) {
    if (elect_one()) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      bar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
      for (int g = 0; g < 2; ++g) {
        tma_load_3d(qs + g * TILE_BYTES, &qmap, q_full, 0, q0 + g * BQ, head);
        tma_load_3d(qs + g * TILE_BYTES + HALF_BYTES, &qmap, q_full, 64, q0 + g * BQ, head);
      }
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int sk = j % KS;
        if (!wait_bar(&k_empty[sk], ((j / KS) & 1) ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        bar_arrive_expect_tx(&k_full[sk], TILE_BYTES);
        tma_load_3d(ks + sk * TILE_BYTES, &kmap, &k_full[sk], 0, j * BKV, head);
        tma_load_3d(ks + sk * TILE_BYTES + HALF_BYTES, &kmap, &k_full[sk], 64, j * BKV, head);
        const int sv = j % VS;
        if (!wait_bar(&v_empty[sv], ((j / VS) & 1) ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        bar_arrive_expect_tx(&v_full[sv], TILE_BYTES);
        tma_load_3d(vs + sv * TILE_BYTES, &vmap, &v_full[sv], 0, j * BKV, head);
        tma_load_3d(vs + sv * TILE_BYTES + HALF_BYTES, &vmap, &v_full[sv], 64, j * BKV, head);
      }
      if (!ok) {
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == WARP_MMA) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_f16(BQ, BKV, 0, 0, 0);   // K-major A and B
      constexpr uint32_t idesc_o = make_idesc_f16(BQ, HD, 0, 0, 1);    // B (V) MN-major
      bool ok = wait_bar(q_full, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA);
      // S_g = Q_g K_j^T into S_g (g = query tile); the K stage is released
      // after the second tile's product.
      auto issue_s = [&](int j, int g) -> bool {
        const int sk = j % KS;
        if (g == 0 &&
            !wait_bar(&k_full[sk], (j / KS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(qs + g * TILE_BYTES);
        const uint32_t k_addr = smem_u32(ks + sk * TILE_BYTES);
        const uint32_t d = tmem + S_COL + g * BKV;
#pragma unroll
        for (int k16 = 0; k16 < HD / 16; ++k16) {
          const uint32_t off = (k16 >> 2) * HALF_BYTES + (k16 & 3) * 32;
          mma_ss(d, make_smem_desc(q_addr + off, 16, 1024), make_smem_desc(k_addr + off, 16, 1024),
                 idesc_s, k16 > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[g]);
        if (g == 1) tc_commit(&k_empty[sk]);
        return true;
      };
      // O_g += P_g V_j; the V stage is released after the second tile's product.
      auto issue_pv = [&](int j, int g) -> bool {
        if (!wait_bar(&p_ready[g], j & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA)) return false;
        const int sv = j % VS;
        if (g == 0 &&
            !wait_bar(&v_full[sv], (j / VS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(vs + sv * TILE_BYTES);
#pragma unroll
        for (int k16 = 0; k16 < BKV / 16; ++k16) {
          // 16 keys per step: rows k16*16.. of both 64-dim halves (LBO = half stride).
          mma_ts(tmem + O_COL + g * HD, tmem + S_COL + g * BKV + k16 * 8,
                 make_smem_desc(v_addr + k16 * 16 * 128, HALF_BYTES, 1024), idesc_o,
                 (j > 0 || k16 > 0) ? 1u : 0u);
        }
        tc_commit(&pv_done[g]);
        if (g == 1) tc_commit(&v_empty[sv]);
        return true;
      };
      if (ok) ok = issue_s(0, 0) && issue_s(0, 1);
      for (int j = 0; j < nkv && ok; ++j) {
        ok = issue_pv(j, 0);
        if (ok && j + 1 < nkv) ok = issue_s(j + 1, 0);
        if (ok) ok = issue_pv(j, 1);
        if (ok && j + 1 < nkv) ok = issue_s(j + 1, 1);
      }
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
    __syncwarp();
    // Free TMEM once every softmax warp has finished reading it (the roles
    // never rejoin, so that each keeps its own register budget).
    const uint32_t sd = smem_u32(sm_done);
    const unsigned long long t1 = globaltimer_ns();
    bool done = bar_try_wait(sd, 0);
    while (!__all_sync(0xffffffffu, done)) {
      if (globaltimer_ns() - t1 > kWaitLimitNs) {
        if (p.err && lane == 0) atomicCAS(p.err, 0, DEV_ERR_TIMEOUT_MMA);
        break;
      }
      done = bar_try_wait(sd, 0);
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  } else {
    regs_inc<kSoftmaxRegs>();
    // softmax warps: 0..3 -> query tile 0, 4..7 -> query tile 1
    const int g = warp >> 2;
    const int qd = warp & 3;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + S_COL + g * BKV;
    const uint32_t o_addr = tmem + lane_base + O_COL + g * HD;
    const int row = qd * 32 + (int)lane;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      bool good = wait_bar(&s_full[g], j & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX);
      if (!__all_sync(0xffffffffu, good)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BKV];
      {
        // All four 32-column loads in flight before the one wait.
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(s_addr, r0);
        tmem_ld32(s_addr + 32, r1);
        tmem_ld32(s_addr + 64, r2);
        tmem_ld32(s_addr + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
          s[64 + i] = __uint_as_float(r2[i]);
          s[96 + i] = __uint_as_float(r3[i]);
        }
      }
      const int kbase = j * BKV;
      if (kbase + BKV > p.seq) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (kbase + c >= p.seq) s[c] = -INFINITY;
      }
      // Row max as 8 independent chains, then a tree.
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = fmaxf(s[i], s[8 + i]);
#pragma unroll
      for (int c = 16; c < BKV; c += 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = max3f(m8[i], s[c + i], s[c + 8 + i]);
      }
      float mx = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      mx *= p.scale_log2;
      float alpha = 1.0f;
      if (j == 0) {
        m = mx;
      } else if (mx > m + kRescaleThreshold) {
        alpha = ex2(m - mx);
        m = mx;
      }
      if (j > 0) {
        // P_g and O_g are free once the previous P_g V has completed (it
        // precedes S_g of this step in the MMA stream, so this is immediate).
        bool good2 = wait_bar(&pv_done[g], (j - 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX);
        if (!__all_sync(0xffffffffu, good2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(o_addr + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(o_addr + c * 32, r);
          }
        }
      }
      unsigned long long rs2[4] = {0ull, 0ull, 0ull, 0ull};
      const unsigned long long sc2 = pack2(p.scale_log2, p.scale_log2);
      const unsigned long long nm2 = pack2(-m, -m);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = ch * 16 + i;
          const unsigned long long x2 = fma2(pack2(s[2 * c], s[2 * c + 1]), sc2, nm2);
          float x0, x1;
          unpack2(x2, x0, x1);
          const float a = ex2(x0);
          const float b = ex2(x1);
          rs2[c & 3] = add2(rs2[c & 3], pack2(a, b));
          pk[i] = cvt_h2(a, b);
        }
        tmem_st16(s_addr + ch * 16, pk);
      }
      float rsv[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack2(rs2[i], rsv[2 * i], rsv[2 * i + 1]);
      const float rs = ((rsv[0] + rsv[1]) + (rsv[2] + rsv[3])) + ((rsv[4] + rsv[5]) + (rsv[6] + rsv[7]));
      l = l * alpha + rs;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&p_ready[g]);
    }
    if (ok) {
      const bool good =
          wait_bar(&pv_done[g], (nkv - 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX);
      if (__all_sync(0xffffffffu, good)) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        const int q = q0 + g * BQ + row;
        __half* base = p.out;
        if (p.routes.n > 0) {
          int r = 0;
          while (r + 1 < p.routes.n && q >= p.routes.row_bound[r + 1]) ++r;
          base = p.routes.outs[r];
        }
        __half* dst = base + (size_t)q * p.ld_out + (size_t)head * HD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(o_addr + c * 32, r);
          tmem_wait_ld();
          if (q < p.seq) {
            uint32_t hv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const __half2 h2 = __floats2half2_rn(__uint_as_float(r[2 * i]) * inv_l,
                                                   __uint_as_float(r[2 * i + 1]) * inv_l);
              hv[i] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              d4[i] = make_uint4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
          }
        }
        if (p.routes.n > 0) __threadfence_system();  // peer stores ordered before the kernel's end
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) bar_arrive(sm_done);
  }
}

}  // namespace attn

int encode_tmap_heads(CUtensorMap* map, const void* base, int n_heads, int seq, int head_dim);

int launch_attention(const __half* q, const __half* k, const __half* v, int n_heads, int seq,
                     int head_dim, float scale, __half* out, long long ld_out, cudaStream_t st,
                     const RowRoutes* routes) {
  if (seq == 0 || n_heads == 0) return 0;
  if (routes && routes->n > 0) {
    if (routes->n > kMaxPeers || routes->row_bound[0] != 0 || routes->row_bound[routes->n] != seq)
      return fail(-1, "attention: row routes must cover [0, seq) with at most 8 destinations");
    for (int r = 0; r < routes->n; ++r)
      if (!routes->outs[r] || (reinterpret_cast<uintptr_t>(routes->outs[r]) & 15) != 0 ||
          routes->row_bound[r + 1] < routes->row_bound[r])
        return fail(-1, "attention: bad row route");
  }
  if (head_dim != attn::HD) return fail(-2, "attention: head_dim must be 128");
  if (!q || !k || !v || !out) return fail(-1, "attention: null tensor");
  if (seq < 0 || n_heads < 0) return fail(-1, "attention: negative shape");
  if (ld_out < (long long)n_heads * head_dim || (ld_out % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15) != 0)
    return fail(-1, "attention: out must be 16-byte aligned with ld_out % 8 == 0 and >= heads*128");
  CUtensorMap qm, km, vm;
  int rc = encode_tmap_heads(&qm, q, n_heads, seq, head_dim);
  if (!rc) rc = encode_tmap_heads(&km, k, n_heads, seq, head_dim);
  if (!rc) rc = encode_tmap_heads(&vm, v, n_heads, seq, head_dim);
  if (rc) return rc;
  attn::Params p{};
  p.seq = seq;
  p.n_heads = n_heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.ld_out = ld_out;
  if (routes) p.routes = *routes;
  p.err = device_error_word();
  static bool attr = false;
  if (!attr) {
    // setmaxnreg.inc waits until the block's launch allocation can supply
    // the registers: refuse to launch unless the kernel was built with the
    // per-thread count the split above assumes.
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, attn::attention_kernel);
    if (e != cudaSuccess) return cuda_status(e, "attention function attributes");
    if (fa.numRegs != attn::kLaunchRegs)
      return fail(-2, "attention: kernel built with " + std::to_string(fa.numRegs) +
                          " registers per thread, the register split needs " +
                          std::to_string(attn::kLaunchRegs));
    e = cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_status(e, "attention set smem attribute");
    attr = true;
  }
  dim3 grid((seq + 2 * attn::BQ - 1) / (2 * attn::BQ), n_heads);
  ProfScope prof("attention", 4.0 * (double)seq * seq * head_dim * n_heads,
                 4.0 * (double)seq * n_heads * head_dim * 2, st);
  attn::attention_kernel<<<grid, attn::NUM_THREADS, attn::SMEM_BYTES, st>>>(qm, km, vm, p);
  return launch_status("attention_kernel launch");
}

}  // namespace bonsai
