// Joint (text + image) non-causal attention for sm_100a.
//
// Replaces ggml_flash_attn_ext as the reference calls it
// (src/diffuser_graph.cpp:403-416 double blocks, :506-519 single blocks):
// softmax(Q K^T * scale) V per head, no mask, K and V in f16, f32 softmax.
//
// One CTA = one head x 256 queries, processed as two 128-query tiles that
// ping-pong on the tensor core: while the softmax warps of one tile work,
// the MMA thread runs the other tile's P*V and its next Q*K^T.  The default
// launch pairs two such CTAs into a cluster that runs each product as one
// cta_group::2 MMA (see attention_kernel<true> below).
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1: thread i
//               owns query row i (TMEM lane i).  Online softmax in the log2
//               domain with lazy rescaling: the running max only moves (and
//               O_g in TMEM is rescaled) when a tile's max exceeds it by more
//               than 8 (p <= 2^8 stays accurate in f16); the final 1/l is
//               exact.  Scale/subtract and the row sum use packed f32x2 ops.
//   warp 8      TMA: Q0/Q1 once, then K_j / V_j blocks (64 keys x 128 dims,
//               two 64-dim halves, 128-byte swizzle) through 4-deep rings.
//   warp 9      one thread issues tcgen05.mma:
//                 S_g(j) = Q_g K_j^T   (A, B from SMEM)          g = 0, 1
//                 O_g   += P_g(j) V_j  (A = P_g from TMEM, B = V MN-major)
//               S runs two blocks ahead of P V (S double-buffered per tile),
//               so a tile's softmax goes from block to block without waiting
//               for that tile's products.
//   warps 10-11 idle (they complete the third warpgroup).
// setmaxnreg gives the softmax warpgroups 224 registers per thread (the whole
// S row stays in registers) and the TMA/MMA warpgroup 56; the three
// warpgroups' code paths never rejoin, so each keeps its own budget, and the
// MMA warp frees TMEM after every softmax warp has signalled it is done.
// TMEM (512 columns): S_{0,0} [0,64) S_{0,1} [64,128) S_{1,0} [128,192)
// S_{1,1} [192,256) O0 [256,384) O1 [384,512); block j of tile g uses
// S_{g, j&1}.  P_g(j) (f16 pairs, 32 columns) overwrites the first half of
// that buffer once the softmax has read S_g(j); S_g(j + 2) is issued after
// P_g(j) V_j in the same in-order MMA stream.
#include "internal.cuh"
#include "ptx.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace bonsai {
namespace attn {

constexpr int BQ = 128;   // queries per tile (two tiles per CTA)
constexpr int BKV = 64;   // keys per block
constexpr int HD = 128;
constexpr int KS = 4;  // K ring depth
constexpr int VS = 4;  // V ring depth
constexpr int Q_BYTES = BQ * HD * 2;      // 32 KB per query tile (two 16 KB halves of 64 dims)
constexpr int Q_HALF = Q_BYTES / 2;
constexpr int KV_BYTES = BKV * HD * 2;    // 16 KB per K or V block (two 8 KB halves)
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
// S_{g,b} (query tile g, buffer b = block parity): 64 columns at g*128 + b*64;
// O_g: 128 columns at 256 + g*128.
constexpr int S_COL = 0, O_COL = 256;
constexpr int SMEM_BYTES = 1024 + 2 * Q_BYTES + (KS + VS) * KV_BYTES + 512;
constexpr float kRescaleThreshold = 8.0f;
// Row-sum bound of a block computed against the running max: above it the
// block is redone with its own max (2^15: every P then fits f16).
constexpr float kSpeculativeSumLimit = 32768.0f;
// Pairs of a row whose exponentials take the polynomial (bit k: pair
// positions k mod 16); the rest go to the MUFU.  Measured best: 2 of 16 for
// the one-CTA kernel, 4 of 16 for the CTA pair (whose tensor-core side is
// faster, so the softmax carries more of the block time).
constexpr unsigned kPolyPairsSingle = 0x8080;
constexpr unsigned kPolyPairsPair = 0x8888;

struct Params {
  int seq;
  int n_heads;
  float scale_log2;  // softmax scale * log2(e)
  __half* out;
  long long ld_out;
  RowRoutes routes;  // routes.n == 0: every row through out
  int* err;
  // Key split: the keys of a head are cut into kv_split ranges of
  // kv_chunk blocks of 64 (the last one shorter), each taken by its own
  // CTA (pair); kv_split > 1 writes each range's normalised partial output
  // and the log2 of its exponential sum instead of `out`, and
  // combine_kernel merges them.
  int kv_split, kv_chunk;
  float* part_o;    // [kv_split][seq][n_heads * 128]
  float* part_lse;  // [kv_split][n_heads][seq]
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

// 2^x for a pair on the FMA and ALU pipes, to take part of the exponentials
// off the MUFU (16 ex2 per clock per SM, the softmax's narrowest pipe).
// x = n + f with n = round(x) (the 1.5 * 2^23 shift leaves n in the low
// mantissa bits of t) and f in [-0.5, 0.5]; 2^f by a degree-3 polynomial
// (coefficients from a Remez exchange on the relative error, max 7.5e-5,
// below the f16 rounding of P); 2^n added to the exponent field.  x is
// clamped to [-126, 126] so that n + the exponent of 2^f stays a valid
// exponent: results below 2^-126 are not needed (P is rounded to f16), and a
// large x (a block computed against a stale running max) still gives a large
// finite P, which the row-sum check catches.
constexpr float kRoundShift = 12582912.0f;  // 1.5 * 2^23
__device__ __forceinline__ void ex2_poly2(unsigned long long x2, float& a, float& b) {
  float x0, x1;
  unpack2(x2, x0, x1);
  const unsigned long long xc =
      pack2(fminf(fmaxf(x0, -126.0f), 126.0f), fminf(fmaxf(x1, -126.0f), 126.0f));
  const unsigned long long t = add2(xc, pack2(kRoundShift, kRoundShift));
  const unsigned long long r = add2(t, pack2(-kRoundShift, -kRoundShift));
  const unsigned long long f = fma2(r, pack2(-1.0f, -1.0f), xc);
  unsigned long long p = fma2(f, pack2(0.0551716685f, 0.0551716685f), pack2(0.2426111251f, 0.2426111251f));
  p = fma2(p, f, pack2(0.6932609677f, 0.6932609677f));
  p = fma2(p, f, pack2(0.9999280572f, 0.9999280572f));
  float p0, p1, t0, t1;
  unpack2(p, p0, p1);
  unpack2(t, t0, t1);
  a = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  b = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ uint32_t cvt_h2(float lo, float hi) {
  uint32_t y;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(y) : "f"(hi), "f"(lo));
  return y;
}

// kPair: a cluster of two CTAs (two SMs) runs every product as one
// cta_group::2 MMA of M = 256 (each CTA's query tile g is one half).  The B
// operands are split between the pair, so each CTA stages half of every K
// block (32 keys) and half of every V block (64 of the 128 dims): per SM, a
// Q K^T reads 5 KB of shared memory per 32 clocks instead of 6 KB.  The even
// CTA issues the MMAs; both CTAs' TMA loads complete on its barriers, its
// commits arrive on both CTAs' barriers, and both CTAs' softmax warps arrive
// on its p_ready.  CTA r of pair c holds query tiles c*512 + g*256 + r*128.
//
// kSplit: the CTA (pair) takes one range of the head's keys and writes
// partials (Params::kv_split > 1); the unsplit instantiation keeps the key
// offset a compile-time zero.
template <bool kPair, bool kSplit>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const Params p) {
  constexpr int K_SLOT = kPair ? KV_BYTES / 2 : KV_BYTES;  // two 64-dim halves of 32 or 64 keys
  constexpr int K_SLOT_HALF = K_SLOT / 2;
  constexpr int V_SLOT = kPair ? KV_BYTES / 2 : KV_BYTES;  // pair: this CTA's 64 dims of 64 keys
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* qs = smem;  // Q0 then Q1
  uint8_t* ks = qs + 2 * Q_BYTES;
  uint8_t* vs = ks + KS * K_SLOT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + VS * V_SLOT);
  uint64_t* q_full = bars;           // [2] per query tile
  uint64_t* k_full = q_full + 2;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;   // [4] per query tile g and buffer b: g * 2 + b
  uint64_t* p_ready = s_full + 4;    // [4]
  uint64_t* pv_done = p_ready + 4;   // [4]
  uint64_t* drain = pv_done + 4;
  uint64_t* sm_done = drain + 1;     // softmax warps finished with TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const int head = blockIdx.y;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  // Unit = (query block, key range): query block qb, key range ksplit.
  const int unit = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ksplit = kSplit ? unit % p.kv_split : 0;
  const int qb = kSplit ? unit / p.kv_split : unit;
  // first query of tile g: q0 + g * tstride
  const int q0 = kPair ? qb * 4 * BQ + (int)rank * BQ : qb * 2 * BQ;
  constexpr int tstride = kPair ? 2 * BQ : BQ;
  const bool leader = !kPair || rank == 0;
  // key blocks [j0, j0 + nkv) of 64 keys (the host guarantees nkv >= 1)
  const int j0 = kSplit ? ksplit * p.kv_chunk : 0;
  const int nkv = kSplit ? min((p.seq + BKV - 1) / BKV - j0, p.kv_chunk) : (p.seq + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    bar_init(&q_full[0], 1);
    bar_init(&q_full[1], 1);
    for (int s = 0; s < KS; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      bar_init(&v_full[s], 1);
      bar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 4; ++i) {
      bar_init(&s_full[i], 1);
      bar_init(&p_ready[i], kPair ? 8 : 4);
      bar_init(&pv_done[i], 1);
    }
    bar_init(drain, 1);
    bar_init(sm_done, 8);
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
  if constexpr (kPair) cluster_sync_all();  // barrier inits and TMEM of both CTAs visible to the pair
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Cluster addresses of the even CTA's barriers (pair loads and remote arrives).
  auto lead_bar = [&](uint64_t* b) -> uint32_t { return mapa_shared(smem_u32(b), 0); };

  if (warp >= 8) {
  regs_dec<kAuxRegs>();
  if (warp == WARP_TMA) {
    if (elect_one()) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      constexpr int ncta = kPair ? 2 : 1;
      // Query tile g on its own barrier: Q0 first, Q1 after the first key
      // block, so that S_0(0) can start before Q1 has landed.
      auto load_q = [&](int g) {
        if (leader) bar_arrive_expect_tx(&q_full[g], ncta * Q_BYTES);
        for (int h = 0; h < 2; ++h) {
          if constexpr (kPair)
            tma_load_3d_pair(qs + g * Q_BYTES + h * Q_HALF, &qmap, lead_bar(&q_full[g]), h * 64,
                             q0 + g * tstride, head);
          else
            tma_load_3d(qs + g * Q_BYTES + h * Q_HALF, &qmap, &q_full[g], h * 64,
                        q0 + g * tstride, head);
        }
      };
      load_q(0);
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int sk = j % KS;
        if (!wait_bar(&k_empty[sk], ((j / KS) & 1) ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        if (leader) bar_arrive_expect_tx(&k_full[sk], ncta * K_SLOT);
        for (int h = 0; h < 2; ++h) {
          if constexpr (kPair)  // this CTA's 32 keys of the block
            tma_load_3d_pair(ks + sk * K_SLOT + h * K_SLOT_HALF, &kmap, lead_bar(&k_full[sk]), h * 64,
                             (j0 + j) * BKV + (int)rank * (BKV / 2), head);
          else
            tma_load_3d(ks + sk * K_SLOT + h * K_SLOT_HALF, &kmap, &k_full[sk], h * 64,
                        (j0 + j) * BKV, head);
        }
        if (j == 0) load_q(1);
        const int sv = j % VS;
        if (!wait_bar(&v_empty[sv], ((j / VS) & 1) ^ 1, abort_flag, p.err, DEV_ERR_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        if (leader) bar_arrive_expect_tx(&v_full[sv], ncta * V_SLOT);
        if constexpr (kPair) {  // this CTA's 64 dims of the block
          tma_load_3d_pair(vs + sv * V_SLOT, &vmap, lead_bar(&v_full[sv]), (int)rank * 64,
                           (j0 + j) * BKV, head);
        } else {
          tma_load_3d(vs + sv * V_SLOT, &vmap, &v_full[sv], 0, (j0 + j) * BKV, head);
          tma_load_3d(vs + sv * V_SLOT + V_SLOT / 2, &vmap, &v_full[sv], 64, (j0 + j) * BKV, head);
        }
      }
      if (!ok) {
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) {
        }
      }
    }
    __syncwarp();
    if constexpr (kPair) cluster_sync_all();
  } else if (warp == WARP_MMA) {
    if (elect_one()) {
    if (leader) {
      constexpr int MM = kPair ? 2 * BQ : BQ;
      constexpr uint32_t idesc_s = make_idesc_f16(MM, BKV, 0, 0, 0);   // K-major A and B
      constexpr uint32_t idesc_o = make_idesc_f16(MM, HD, 0, 0, 1);    // B (V) MN-major
      auto commit = [&](uint64_t* b) {
        if constexpr (kPair)
          tc_commit_pair(b, 0x3);
        else
          tc_commit(b);
      };
      bool ok = true;
      // S_g(j) = Q_g K_j^T into S_{g, j&1}; the K stage is released after the
      // second tile's product.
      auto issue_s = [&](int j, int g) -> bool {
        const int sk = j % KS;
        if (j == 0 && !wait_bar(&q_full[g], 0, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        if (g == 0 &&
            !wait_bar(&k_full[sk], (j / KS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(qs + g * Q_BYTES);
        const uint32_t k_addr = smem_u32(ks + sk * K_SLOT);
        const uint32_t d = tmem + S_COL + g * 128 + (j & 1) * BKV;
#pragma unroll
        for (int k16 = 0; k16 < HD / 16; ++k16) {
          const uint32_t qo = (k16 >> 2) * Q_HALF + (k16 & 3) * 32;
          const uint32_t ko = (k16 >> 2) * K_SLOT_HALF + (k16 & 3) * 32;
          const uint64_t qd = make_smem_desc(q_addr + qo, 16, 1024);
          const uint64_t kd = make_smem_desc(k_addr + ko, 16, 1024);
          if constexpr (kPair)
            mma_ss_pair(d, qd, kd, idesc_s, k16 > 0 ? 1u : 0u);
          else
            mma_ss(d, qd, kd, idesc_s, k16 > 0 ? 1u : 0u);
        }
        commit(&s_full[g * 2 + (j & 1)]);
        if (g == 1) commit(&k_empty[sk]);
        return true;
      };
      // O_g += P_g(j) V_j with P_g(j) over the first 32 columns of S_{g, j&1};
      // the V stage is released after the second tile's product.
      auto issue_pv = [&](int j, int g) -> bool {
        const int b = j & 1;
        if (!wait_bar(&p_ready[g * 2 + b], (j >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        const int sv = j % VS;
        if (g == 0 &&
            !wait_bar(&v_full[sv], (j / VS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(vs + sv * V_SLOT);
#pragma unroll
        for (int k16 = 0; k16 < BKV / 16; ++k16) {
          // 16 keys per step: rows k16*16.. of the 64-dim halves (LBO = half
          // stride; the pair's CTAs hold one half each).
          const uint32_t a = tmem + S_COL + g * 128 + b * BKV + k16 * 8;
          const uint64_t vd = make_smem_desc(v_addr + k16 * 16 * 128, V_SLOT / 2, 1024);
          if constexpr (kPair)
            mma_ts_pair(tmem + O_COL + g * HD, a, vd, idesc_o, (j > 0 || k16 > 0) ? 1u : 0u);
          else
            mma_ts(tmem + O_COL + g * HD, a, vd, idesc_o, (j > 0 || k16 > 0) ? 1u : 0u);
        }
        commit(&pv_done[g * 2 + b]);
        if (g == 1) commit(&v_empty[sv]);
        return true;
      };
      // S runs two blocks ahead of P V: S_g(j + 2) reuses the buffer of
      // P_g(j) and follows P_g(j) V_j in the in-order MMA stream, so the
      // softmax of block j + 1 never waits for the products of block j.
      if (ok) ok = issue_s(0, 0) && issue_s(0, 1);
      if (ok && nkv > 1) ok = issue_s(1, 0) && issue_s(1, 1);
      for (int j = 0; j < nkv && ok; ++j) {
        ok = issue_pv(j, 0);
        if (ok && j + 2 < nkv) ok = issue_s(j + 2, 0);
        if (ok) ok = issue_pv(j, 1);
        if (ok && j + 2 < nkv) ok = issue_s(j + 2, 1);
      }
      commit(drain);
    }
      // Both CTAs of a pair: wait until every MMA has completed (the commit
      // above arrives on the drain barrier of each CTA).
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
    if constexpr (kPair) {
      // Every warp of both CTAs ends at this cluster barrier, after its last
      // MMA, remote arrive and TMEM access.
      cluster_sync_all();
      tc_fence_after();
      tmem_dealloc_pair(tmem, TMEM_COLS);
    } else {
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
    if constexpr (kPair) cluster_sync_all();  // warps 10-11
  }
  } else {
    regs_inc<kSoftmaxRegs>();
    // softmax warps: 0..3 -> query tile 0, 4..7 -> query tile 1
    const int g = warp >> 2;
    const int qd = warp & 3;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + O_COL + g * HD;
    const int row = qd * 32 + (int)lane;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int buf = j & 1;
      const uint32_t s_addr = tmem + lane_base + S_COL + g * 128 + buf * BKV;
      bool good = wait_bar(&s_full[g * 2 + buf], (j >> 1) & 1, abort_flag, p.err,
                           DEV_ERR_TIMEOUT_SOFTMAX);
      if (!__all_sync(0xffffffffu, good)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BKV];
      {
        // Both 32-column loads in flight before the one wait.
        uint32_t r0[32], r1[32];
        tmem_ld32(s_addr, r0);
        tmem_ld32(s_addr + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
        }
      }
      const int kbase = (j0 + j) * BKV;
      if (kbase + BKV > p.seq) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (kbase + c >= p.seq) s[c] = -INFINITY;
      }
      // Row max as 8 independent chains, then a tree (log2 domain).
      auto row_max = [&]() -> float {
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(s[i], s[8 + i]);
#pragma unroll
        for (int c = 16; c < BKV; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = max3f(m8[i], s[c + i], s[c + 8 + i]);
        }
        return max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]),
                     fmaxf(m8[6], m8[7])) * p.scale_log2;
      };
      // P = 2^(s * scale - mref) into the first half of this S buffer; returns
      // the row sum of P (f32, before the f16 rounding).
      auto exps = [&](float mref) -> float {
        unsigned long long rs2[4] = {0ull, 0ull, 0ull, 0ull};
        const unsigned long long sc2 = pack2(p.scale_log2, p.scale_log2);
        const unsigned long long nm2 = pack2(-mref, -mref);
#pragma unroll
        for (int ch = 0; ch < BKV / 32; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = ch * 16 + i;
            const unsigned long long x2 = fma2(pack2(s[2 * c], s[2 * c + 1]), sc2, nm2);
            float a, b;
            if (((kPair ? kPolyPairsPair : kPolyPairsSingle) >> i) & 1) {
              ex2_poly2(x2, a, b);
            } else {
              float x0, x1;
              unpack2(x2, x0, x1);
              a = ex2(x0);
              b = ex2(x1);
            }
            rs2[c & 3] = add2(rs2[c & 3], pack2(a, b));
            pk[i] = cvt_h2(a, b);
          }
          tmem_st16(s_addr + ch * 16, pk);
        }
        float rsv[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) unpack2(rs2[i], rsv[2 * i], rsv[2 * i + 1]);
        return ((rsv[0] + rsv[1]) + (rsv[2] + rsv[3])) + ((rsv[4] + rsv[5]) + (rsv[6] + rsv[7]));
      };
      float alpha = 1.0f;
      float rs = 0.0f;
      // This block's max; the running max moves (and O_g is rescaled) only
      // when it exceeds it by more than kRescaleThreshold.  False on timeout.
      auto rescale_step = [&]() -> bool {
        const float mx = row_max();
        if (mx > m + kRescaleThreshold) {
          alpha = ex2(m - mx);
          m = mx;
        }
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
          // O_g is rescaled once P_g(j - 1) V_{j-1} has completed (it may
          // still be in flight: S runs ahead of P V).  P_g(j) V_j waits for
          // this block's p_ready, so nothing else writes O_g meanwhile.
          const int pb = (j - 1) & 1;
          bool good2 = wait_bar(&pv_done[g * 2 + pb], ((j - 1) >> 1) & 1, abort_flag, p.err,
                                DEV_ERR_TIMEOUT_SOFTMAX);
          if (!__all_sync(0xffffffffu, good2)) return false;
          tc_fence_after();
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
        return true;
      };
      // CTA pair: from the second block on, the exponentials are first taken
      // against the running max, without this block's max.  Every P is <=
      // the row sum, so a row sum <= 2^15 means every P fits f16 (and is as
      // precise there as any other value); only when some row's sum exceeds
      // it (a block max more than ~9 above the running max, rare after the
      // first blocks) is the block redone the usual way.  One copy of the
      // exponential code serves both passes.  (The one-CTA form measured
      // slower this way and keeps the max first.)
      constexpr bool kSpeculative = kPair;
      if (j == 0) {
        m = row_max();
      } else if (!kSpeculative && !rescale_step()) {
        ok = false;
        break;
      }
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        rs = exps(m);
        if (!kSpeculative || j == 0 || pass == 1 ||
            !__any_sync(0xffffffffu, !(rs <= kSpeculativeSumLimit)))
          break;
        if (!rescale_step()) {
          ok = false;
          break;
        }
        tmem_wait_st();  // the first pass's P stores land before they are overwritten
      }
      if (!ok) break;
      l = l * alpha + rs;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair)
          bar_arrive_remote(lead_bar(&p_ready[g * 2 + buf]));
        else
          bar_arrive(&p_ready[g * 2 + buf]);
      }
    }
    if (ok) {
      const bool good =
          wait_bar(&pv_done[g * 2 + ((nkv - 1) & 1)], ((nkv - 1) >> 1) & 1, abort_flag, p.err,
                   DEV_ERR_TIMEOUT_SOFTMAX);
      if (__all_sync(0xffffffffu, good)) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        const int q = q0 + g * tstride + row;
        if (kSplit) {
          // this key range's O / l (f32) and log2 of its exponential sum
          float* po = p.part_o + ((size_t)ksplit * p.seq + q) * ((size_t)p.n_heads * HD) +
                      (size_t)head * HD;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(o_addr + c * 32, r);
            tmem_wait_ld();
            if (q < p.seq) {
              float4* d4 = reinterpret_cast<float4*>(po + c * 32);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                d4[i] = make_float4(__uint_as_float(r[4 * i]) * inv_l, __uint_as_float(r[4 * i + 1]) * inv_l,
                                    __uint_as_float(r[4 * i + 2]) * inv_l,
                                    __uint_as_float(r[4 * i + 3]) * inv_l);
            }
          }
          if (q < p.seq)
            p.part_lse[((size_t)ksplit * p.n_heads + head) * p.seq + q] = m + __log2f(l);
        } else {
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
    }
    tc_fence_before();
    __syncwarp();
    if constexpr (kPair)
      cluster_sync_all();
    else if (lane == 0)
      bar_arrive(sm_done);
  }
}

// Merges the kv_split partial outputs of each (query row, head): with
// lse_s = log2 of range s's exponential sum, out = sum_s 2^(lse_s - lse) O_s
// where lse = log2 sum_s 2^lse_s (the ranges' softmax weights).  One thread
// per 8 dims of one (row, head); f16 stores to out, or to the row's owner
// under routes (as the attention epilogue does).
__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                               int kv_split, int seq, int n_heads, __half* out, long long ld_out,
                               RowRoutes routes) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long total = (long long)seq * n_heads * (HD / 8);
  if (idx >= total) return;
  const int d8 = (int)(idx % (HD / 8));
  const int h = (int)((idx / (HD / 8)) % n_heads);
  const int q = (int)(idx / ((long long)(HD / 8) * n_heads));
  float mx = -INFINITY;
  for (int sp = 0; sp < kv_split; ++sp)
    mx = fmaxf(mx, part_lse[((size_t)sp * n_heads + h) * seq + q]);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  const size_t row_stride = (size_t)n_heads * HD;
  for (int sp = 0; sp < kv_split; ++sp) {
    const float w = exp2f(part_lse[((size_t)sp * n_heads + h) * seq + q] - mx);
    wsum += w;
    const float4* src = reinterpret_cast<const float4*>(part_o + ((size_t)sp * seq + q) * row_stride +
                                                        (size_t)h * HD + d8 * 8);
    const float4 a = src[0], b = src[1];
    acc[0] += w * a.x; acc[1] += w * a.y; acc[2] += w * a.z; acc[3] += w * a.w;
    acc[4] += w * b.x; acc[5] += w * b.y; acc[6] += w * b.z; acc[7] += w * b.w;
  }
  const float inv = 1.0f / wsum;
  __half* base = out;
  if (routes.n > 0) {
    int r = 0;
    while (r + 1 < routes.n && q >= routes.row_bound[r + 1]) ++r;
    base = routes.outs[r];
  }
  uint32_t hv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h2 = __floats2half2_rn(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    hv[i] = *reinterpret_cast<const uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(base + (size_t)q * ld_out + (size_t)h * HD + d8 * 8) =
      make_uint4(hv[0], hv[1], hv[2], hv[3]);
  if (routes.n > 0) __threadfence_system();  // peer stores ordered before the kernel's end
}

// ------------------------------------------------------------------------
// attention_pair128_kernel (BONSAI_ATTN=v2): a cluster of two CTAs per head
// x 256 queries -- one 128-query tile per CTA, every product one
// cta_group::2 MMA of M = 256 -- with keys in blocks of 128.  Q K^T then has
// N = 128: per SM and k-step it reads Q (4 KB) and this CTA's 64 keys (2 KB)
// in 64 clocks, 96 B/clk, under shared memory's 128 B/clk (with 64-key
// blocks it needs 160 B/clk and waits on shared memory).  The 128 keys of a
// block feed two independent online softmaxes: warps 0-3 take keys [0, 64)
// of every block, warps 4-7 keys [64, 128), each half with its own running
// max, row sum and O accumulator in TMEM (O_a, O_b), merged in the
// epilogue, so neither half ever waits for the other's max.  S is
// double-buffered by block parity.  TMEM: S(even) [0,128) S(odd) [128,256)
// O_a [256,384) O_b [384,512); P of half h (f16 pairs) overwrites the first
// 32 columns of that half's S.  MMA order: S(0) S(1), then per block j:
// P_a V_a(j), P_b V_b(j), S(j + 2) -- S(j + 2) reuses the buffer whose P the
// two products before it have read.
namespace v2 {
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int HALF = 64;
constexpr int KS = 4;
constexpr int VS = 4;
constexpr int Q_BYTES = BQ * HD * 2;       // 32 KB: two 64-dim halves of 16 KB
constexpr int Q_HALF = Q_BYTES / 2;
constexpr int K_SLOT = HALF * HD * 2;      // this CTA's 64 keys x 128 dims: 16 KB
constexpr int K_SLOT_HALF = K_SLOT / 2;    // 64 keys x 64 dims
constexpr int V_SLOT = BKV * 64 * 2;       // this CTA's 64 dims x 128 keys: 16 KB
constexpr int BAR_BYTES = 512;
constexpr int STAT_BYTES = 4 * BQ * 4;     // (max, sum) of both halves, per row
constexpr int SMEM_BYTES = 1024 + Q_BYTES + (KS + VS) * K_SLOT + BAR_BYTES + STAT_BYTES;
constexpr int S_COL = 0, O_COL = 256;
static_assert(K_SLOT == V_SLOT, "K and V stages share the slot size");
}  // namespace v2

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attention_pair128_kernel(const __grid_constant__ CUtensorMap qmap,
                             const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + v2::Q_BYTES;
  uint8_t* vs = ks + v2::KS * v2::K_SLOT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + v2::VS * v2::V_SLOT);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + v2::KS;
  uint64_t* v_full = k_empty + v2::KS;
  uint64_t* v_empty = v_full + v2::VS;
  uint64_t* s_full = v_empty + v2::VS;  // [2] by block parity
  uint64_t* p_ready = s_full + 2;       // [4] key half * 2 + block parity
  uint64_t* pv_done = p_ready + 4;      // [4] key half * 2 + block parity
  uint64_t* drain = pv_done + 4;
  uint64_t* stat_bar = drain + 1;       // both halves' (max, sum) published
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stat_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* st_m = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + v2::BAR_BYTES);
  float* st_l = st_m + 2 * v2::BQ;  // st_m / st_l [half][row]

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const int head = blockIdx.y;
  const uint32_t rank = cluster_ctarank();
  const int q0 = (int)(blockIdx.x >> 1) * 2 * v2::BQ + (int)rank * v2::BQ;
  const bool leader = rank == 0;
  const int nkv = (p.seq + v2::BKV - 1) / v2::BKV;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int s = 0; s < v2::KS; ++s) {
      bar_init(&k_full[s], 1);
      bar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < v2::VS; ++s) {
      bar_init(&v_full[s], 1);
      bar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) bar_init(&s_full[i], 1);
    for (int i = 0; i < 4; ++i) {
      bar_init(&p_ready[i], 8);  // 4 warps of the half in each CTA
      bar_init(&pv_done[i], 1);
    }
    bar_init(drain, 1);
    bar_init(stat_bar, 8 * 32);  // every softmax thread of this CTA
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
  auto lead_bar = [&](uint64_t* b) -> uint32_t { return mapa_shared(smem_u32(b), 0); };

  if (warp >= 8) {
    regs_dec<kAuxRegs>();
    if (warp == WARP_TMA) {
      if (elect_one()) {
        tma_prefetch_desc(&qmap);
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
        if (leader) bar_arrive_expect_tx(q_full, 2 * v2::Q_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d_pair(qs + h * v2::Q_HALF, &qmap, lead_bar(q_full), h * 64, q0, head);
        bool ok = true;
        for (int j = 0; j < nkv && ok; ++j) {
          const int sk = j % v2::KS;
          if (!wait_bar(&k_empty[sk], ((j / v2::KS) & 1) ^ 1, abort_flag, p.err,
                        DEV_ERR_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          if (leader) bar_arrive_expect_tx(&k_full[sk], 2 * v2::K_SLOT);
          for (int h = 0; h < 2; ++h)  // this CTA's 64 keys of the block, two 64-dim halves
            tma_load_3d_pair(ks + sk * v2::K_SLOT + h * v2::K_SLOT_HALF, &kmap,
                             lead_bar(&k_full[sk]), h * 64, j * v2::BKV + (int)rank * v2::HALF,
                             head);
          const int sv = j % v2::VS;
          if (!wait_bar(&v_empty[sv], ((j / v2::VS) & 1) ^ 1, abort_flag, p.err,
                        DEV_ERR_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          if (leader) bar_arrive_expect_tx(&v_full[sv], 2 * v2::V_SLOT);
          // this CTA's 64 dims of the block's 128 keys
          tma_load_3d_pair(vs + sv * v2::V_SLOT, &vmap, lead_bar(&v_full[sv]), (int)rank * 64,
                           j * v2::BKV, head);
        }
        if (!ok) {
          const unsigned long long t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 1000000ull) {
          }
        }
      }
      __syncwarp();
      cluster_sync_all();
    } else if (warp == WARP_MMA) {
      if (elect_one()) {
        if (leader) {
          constexpr uint32_t idesc_s = make_idesc_f16(2 * v2::BQ, v2::BKV, 0, 0, 0);
          constexpr uint32_t idesc_o = make_idesc_f16(2 * v2::BQ, HD, 0, 0, 1);  // V MN-major
          bool ok = wait_bar(q_full, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA);
          // S(j) = Q K_j^T (N = 128) into S(j & 1); the K stage is released after it.
          auto issue_s = [&](int j) -> bool {
            const int sk = j % v2::KS;
            if (!wait_bar(&k_full[sk], (j / v2::KS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
              return false;
            tc_fence_after();
            const uint32_t q_addr = smem_u32(qs);
            const uint32_t k_addr = smem_u32(ks + sk * v2::K_SLOT);
            const uint32_t d = tmem + v2::S_COL + (j & 1) * v2::BKV;
#pragma unroll
            for (int k16 = 0; k16 < HD / 16; ++k16) {
              const uint32_t qo = (k16 >> 2) * v2::Q_HALF + (k16 & 3) * 32;
              const uint32_t ko = (k16 >> 2) * v2::K_SLOT_HALF + (k16 & 3) * 32;
              mma_ss_pair(d, make_smem_desc(q_addr + qo, 16, 1024),
                          make_smem_desc(k_addr + ko, 16, 1024), idesc_s, k16 > 0 ? 1u : 0u);
            }
            tc_commit_pair(&s_full[j & 1], 0x3);
            tc_commit_pair(&k_empty[sk], 0x3);
            return true;
          };
          // O_h += P_h(j) V_h(j): P_h over the first 32 columns of half h of
          // S(j & 1), V_h = keys [64 h, 64 h + 64) of the V stage; the stage
          // is released after the second half's product.
          auto issue_pv = [&](int j, int h) -> bool {
            const int b = j & 1;
            if (!wait_bar(&p_ready[h * 2 + b], (j >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
              return false;
            const int sv = j % v2::VS;
            if (h == 0 &&
                !wait_bar(&v_full[sv], (j / v2::VS) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA))
              return false;
            tc_fence_after();
            const uint32_t v_addr = smem_u32(vs + sv * v2::V_SLOT) + h * v2::HALF * 128;
#pragma unroll
            for (int k16 = 0; k16 < v2::HALF / 16; ++k16) {
              const uint32_t a = tmem + v2::S_COL + b * v2::BKV + h * v2::HALF + k16 * 8;
              const uint64_t vd = make_smem_desc(v_addr + k16 * 16 * 128, v2::V_SLOT / 2, 1024);
              mma_ts_pair(tmem + v2::O_COL + h * HD, a, vd, idesc_o, (j > 0 || k16 > 0) ? 1u : 0u);
            }
            tc_commit_pair(&pv_done[h * 2 + b], 0x3);
            if (h == 1) tc_commit_pair(&v_empty[sv], 0x3);
            return true;
          };
          if (ok) ok = issue_s(0);
          if (ok && nkv > 1) ok = issue_s(1);
          for (int j = 0; j < nkv && ok; ++j) {
            ok = issue_pv(j, 0);
            if (ok) ok = issue_pv(j, 1);
            if (ok && j + 2 < nkv) ok = issue_s(j + 2);
          }
          tc_commit_pair(drain, 0x3);
        }
        // Both CTAs: wait until every MMA has completed (the commit above
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
      __syncwarp();
      // Every warp of both CTAs ends at this cluster barrier, after its last
      // MMA, remote arrive and TMEM access.
      cluster_sync_all();
      tc_fence_after();
      tmem_dealloc_pair(tmem, TMEM_COLS);
    } else {
      cluster_sync_all();  // warps 10-11
    }
  } else {
    regs_inc<kSoftmaxRegs>();
    // softmax warps: 0..3 -> keys [0, 64) of every block, 4..7 -> keys [64, 128)
    const int hf = warp >> 2;
    const int qd = warp & 3;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + v2::O_COL + hf * HD;
    const int row = qd * 32 + (int)lane;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int buf = j & 1;
      const uint32_t s_addr = tmem + lane_base + v2::S_COL + buf * v2::BKV + hf * v2::HALF;
      bool good = wait_bar(&s_full[buf], (j >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX);
      if (!__all_sync(0xffffffffu, good)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kbase = j * v2::BKV + hf * v2::HALF;
      if (kbase >= p.seq) {
        // This half of the last block holds no key (seq % 128 <= 64): P = 0,
        // and the max / sum stay as they are.
        uint32_t z[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) z[i] = 0u;
        tmem_st16(s_addr, z);
        tmem_st16(s_addr + 16, z);
      } else {
        float s[v2::HALF];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(s_addr, r0);
          tmem_ld32(s_addr + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s[i] = __uint_as_float(r0[i]);
            s[32 + i] = __uint_as_float(r1[i]);
          }
        }
        if (kbase + v2::HALF > p.seq) {
#pragma unroll
          for (int c = 0; c < v2::HALF; ++c)
            if (kbase + c >= p.seq) s[c] = -INFINITY;
        }
        auto row_max = [&]() -> float {
          float m8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = fmaxf(s[i], s[8 + i]);
#pragma unroll
          for (int c = 16; c < v2::HALF; c += 16) {
#pragma unroll
            for (int i = 0; i < 8; ++i) m8[i] = max3f(m8[i], s[c + i], s[c + 8 + i]);
          }
          return max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]),
                       fmaxf(m8[6], m8[7])) * p.scale_log2;
        };
        auto exps = [&](float mref) -> float {
          unsigned long long rs2[4] = {0ull, 0ull, 0ull, 0ull};
          const unsigned long long sc2 = pack2(p.scale_log2, p.scale_log2);
          const unsigned long long nm2 = pack2(-mref, -mref);
#pragma unroll
          for (int ch = 0; ch < v2::HALF / 32; ++ch) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int c = ch * 16 + i;
              const unsigned long long x2 = fma2(pack2(s[2 * c], s[2 * c + 1]), sc2, nm2);
              float a, b;
              if ((kPolyPairsPair >> i) & 1) {
                ex2_poly2(x2, a, b);
              } else {
                float x0, x1;
                unpack2(x2, x0, x1);
                a = ex2(x0);
                b = ex2(x1);
              }
              rs2[c & 3] = add2(rs2[c & 3], pack2(a, b));
              pk[i] = cvt_h2(a, b);
            }
            tmem_st16(s_addr + ch * 16, pk);
          }
          float rsv[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) unpack2(rs2[i], rsv[2 * i], rsv[2 * i + 1]);
          return ((rsv[0] + rsv[1]) + (rsv[2] + rsv[3])) + ((rsv[4] + rsv[5]) + (rsv[6] + rsv[7]));
        };
        float alpha = 1.0f;
        float rs = 0.0f;
        auto rescale_step = [&]() -> bool {
          const float mx = row_max();
          if (mx > m + kRescaleThreshold) {
            alpha = ex2(m - mx);
            m = mx;
          }
          if (__any_sync(0xffffffffu, alpha != 1.0f)) {
            // O_h is rescaled once P_h(j - 1) V_h(j - 1) has completed.
            const int pb = (j - 1) & 1;
            bool good2 = wait_bar(&pv_done[hf * 2 + pb], ((j - 1) >> 1) & 1, abort_flag, p.err,
                                  DEV_ERR_TIMEOUT_SOFTMAX);
            if (!__all_sync(0xffffffffu, good2)) return false;
            tc_fence_after();
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
          return true;
        };
        // Speculative exponentials as in the 64-key pair kernel: from the
        // second block on, taken against the running max first; a block whose
        // row sum exceeds 2^15 is redone with its own max.
        if (j == 0) m = row_max();
#pragma unroll 1
        for (int pass = 0; pass < 2; ++pass) {
          rs = exps(m);
          if (j == 0 || pass == 1 || !__any_sync(0xffffffffu, !(rs <= kSpeculativeSumLimit)))
            break;
          if (!rescale_step()) {
            ok = false;
            break;
          }
          tmem_wait_st();  // the first pass's P stores land before they are overwritten
        }
        if (!ok) break;
        l = l * alpha + rs;
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive_remote(lead_bar(&p_ready[hf * 2 + buf]));
    }
    if (ok) {
      // Publish this half's (max, sum) per row, then merge both halves.
      st_m[hf * v2::BQ + row] = m;
      st_l[hf * v2::BQ + row] = l;
      bar_arrive(stat_bar);
      const int lb = (nkv - 1) & 1;
      const uint32_t lph = ((nkv - 1) >> 1) & 1;
      const bool good = wait_bar(stat_bar, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX) &&
                        wait_bar(&pv_done[lb], lph, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX) &&
                        wait_bar(&pv_done[2 + lb], lph, abort_flag, p.err, DEV_ERR_TIMEOUT_SOFTMAX);
      if (__all_sync(0xffffffffu, good)) {
        tc_fence_after();
        const float ma = st_m[row], mb = st_m[v2::BQ + row];
        const float mx = fmaxf(ma, mb);
        const float wa = ex2(ma - mx), wb = ex2(mb - mx);  // 0 for a half that saw no key
        const float inv_l = 1.0f / (st_l[row] * wa + st_l[v2::BQ + row] * wb);
        const float ca = wa * inv_l, cb = wb * inv_l;
        const int q = q0 + row;
        __half* base = p.out;
        if (p.routes.n > 0) {
          int r = 0;
          while (r + 1 < p.routes.n && q >= p.routes.row_bound[r + 1]) ++r;
          base = p.routes.outs[r];
        }
        // this warp writes dims [64 hf, 64 hf + 64) of its rows
        __half* dst = base + (size_t)q * p.ld_out + (size_t)head * HD + hf * v2::HALF;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t ra[32], rb[32];
          tmem_ld32(tmem + lane_base + v2::O_COL + hf * v2::HALF + c * 32, ra);
          tmem_ld32(tmem + lane_base + v2::O_COL + HD + hf * v2::HALF + c * 32, rb);
          tmem_wait_ld();
          if (q < p.seq) {
            uint32_t hv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float x0 = __uint_as_float(ra[2 * i]) * ca + __uint_as_float(rb[2 * i]) * cb;
              const float x1 =
                  __uint_as_float(ra[2 * i + 1]) * ca + __uint_as_float(rb[2 * i + 1]) * cb;
              const __half2 h2 = __floats2half2_rn(x0, x1);
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
    cluster_sync_all();
  }
}

}  // namespace attn

int encode_tmap_heads(CUtensorMap* map, const void* base, int n_heads, int seq, int head_dim,
                      int box_rows);

namespace {
cudaLaunchConfig_t attn_pair_config(cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(attn::NUM_THREADS);
  cfg.dynamicSmemBytes = attn::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// How many clusters of two attention CTAs can be resident at once (0: the
// pair form cannot run and the one-CTA form is used).
int attn_pair_slots() {
  static int slots_dev[64];
  static bool known[64] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  const int d = device_slot();
  if (!known[d]) {
    known[d] = true;
    slots_dev[d] = 0;
    if (cudaFuncSetAttribute(attn::attention_kernel<true, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn::SMEM_BYTES) == cudaSuccess) {
      cudaLaunchAttribute attr[1];
      cudaLaunchConfig_t cfg = attn_pair_config(attr);
      cfg.gridDim = dim3(2);
      int c = 0;
      if (cudaOccupancyMaxActiveClusters(&c, attn::attention_kernel<true, false>, &cfg) == cudaSuccess)
        slots_dev[d] = c > 0 ? c : 0;
    }
    cudaGetLastError();
  }
  return slots_dev[d];
}

// Key split for a launch of `units` equal work units (clusters or CTAs) on
// `slots` resident ones, nkv key blocks per head.  A launch that fills at
// most half of the GPU in a single wave (one or two heads at a long
// sequence) leaves SMs idle for its whole duration: cutting every unit's keys
// into s ranges (units * s <= slots) runs it in about 1/s of the time.  Where
// the units already take more than one wave the split does not pay: on 3
// heads x 16896 tokens (99 clusters on 74 slots) two ranges measured 450 us
// against 438 us unsplit -- the part-filled last wave runs at a higher clock
// than the full ones, and every range adds its pipeline start, f32 partial
// stores and the merge.  Every range keeps >= 16 key blocks.
// BONSAI_ATTN_SPLIT=n forces n ranges (tests).  Returns the number of key
// ranges; *chunk = blocks per range.
int choose_kv_split(long long units, int slots, int nkv, int* chunk) {
  int want = 1;
  if (const char* e = getenv("BONSAI_ATTN_SPLIT")) {
    want = std::max(1, atoi(e));
  } else if (slots > 0) {
    for (int sp = 2; sp <= 4; ++sp)
      if (units * sp <= slots && nkv / sp >= 16) want = sp;
  }
  want = std::min(want, nkv);
  *chunk = (nkv + want - 1) / want;
  return (nkv + *chunk - 1) / *chunk;  // no empty range
}
}  // namespace

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
  // BONSAI_ATTN=single selects the one-CTA form (the tests run both); the
  // CTA-pair form is the default where a cluster of two fits (checked once).
  // Kernel form.  BONSAI_ATTN=single: one CTA per head x 256 queries;
  // pair (or v1): clusters of two CTAs, 512 queries, 64-key blocks; v2:
  // clusters of two CTAs, 256 queries, 128-key blocks with two key-half
  // softmaxes.  Unset: v2 where its smaller work units fill the GPU's waves
  // enough better to make up for its lower per-SM rate (measured alone:
  // 1055 / 1242 TFLOP/s for v2 against 1214 / 1356 for the 64-key pair at
  // L = 4608 / 16896 with 24 heads, 1158 against 1001 with 3 heads at 16896,
  // the 8-GPU head split's shape), else the 64-key pair.  A forced key split
  // (BONSAI_ATTN_SPLIT) runs on the 64-key forms.
  const char* form = getenv("BONSAI_ATTN");
  const int pair_slots = attn_pair_slots();
  const bool pair = !(form && std::strcmp(form, "single") == 0) && pair_slots > 0;
  bool v2form = false;
  if (pair && form && std::strcmp(form, "v2") == 0) {
    v2form = true;
  } else if (pair && !form && !getenv("BONSAI_ATTN_SPLIT")) {
    constexpr double kV2UnitCost = 0.55;  // a v2 cluster's time per 64-key-pair cluster's
    const long long u1 = (long long)((seq + 4 * attn::BQ - 1) / (4 * attn::BQ)) * n_heads;
    const long long u2 = (long long)((seq + 2 * attn::v2::BQ - 1) / (2 * attn::v2::BQ)) * n_heads;
    const double w1 = (double)((u1 + pair_slots - 1) / pair_slots);
    const double w2 = kV2UnitCost * (double)((u2 + pair_slots - 1) / pair_slots);
    v2form = w2 < 0.95 * w1;
  }
  attn::Params p{};
  p.seq = seq;
  p.n_heads = n_heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.ld_out = ld_out;
  if (routes) p.routes = *routes;
  p.err = device_error_word();
  p.kv_split = 1;
  static bool attr_dev[64] = {};
  bool& attr = attr_dev[device_slot()];
  if (!attr) {
    {
      cudaFuncAttributes fa{};
      cudaError_t e = cudaFuncGetAttributes(&fa, attn::attention_pair128_kernel);
      if (e != cudaSuccess) return cuda_status(e, "attention function attributes");
      if (fa.numRegs != attn::kLaunchRegs)
        return fail(-2, "attention: kernel built with " + std::to_string(fa.numRegs) +
                            " registers per thread, the register split needs " +
                            std::to_string(attn::kLaunchRegs));
      e = cudaFuncSetAttribute(attn::attention_pair128_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, attn::v2::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_status(e, "attention set smem attribute");
    }
    // setmaxnreg.inc waits until the block's launch allocation can supply
    // the registers: refuse to launch unless the kernel was built with the
    // per-thread count the split above assumes.
    for (auto kern : {attn::attention_kernel<false, false>, attn::attention_kernel<true, false>,
                      attn::attention_kernel<false, true>, attn::attention_kernel<true, true>}) {
      cudaFuncAttributes fa{};
      cudaError_t e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return cuda_status(e, "attention function attributes");
      if (fa.numRegs != attn::kLaunchRegs)
        return fail(-2, "attention: kernel built with " + std::to_string(fa.numRegs) +
                            " registers per thread, the register split needs " +
                            std::to_string(attn::kLaunchRegs));
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, attn::SMEM_BYTES);
      if (e != cudaSuccess) return cuda_status(e, "attention set smem attribute");
    }
    attr = true;
  }
  if (v2form) {
    CUtensorMap qm, km, vm;
    int rc = encode_tmap_heads(&qm, q, n_heads, seq, head_dim, attn::v2::BQ);
    if (!rc) rc = encode_tmap_heads(&km, k, n_heads, seq, head_dim, attn::v2::HALF);
    if (!rc) rc = encode_tmap_heads(&vm, v, n_heads, seq, head_dim, attn::v2::BKV);
    if (rc) return rc;
    ProfScope prof("attention", 4.0 * (double)seq * seq * head_dim * n_heads,
                   4.0 * (double)seq * n_heads * head_dim * 2, st);
    cudaLaunchAttribute attr_c[1];
    cudaLaunchConfig_t cfg = attn_pair_config(attr_c);
    cfg.gridDim = dim3(2 * (unsigned)((seq + 2 * attn::v2::BQ - 1) / (2 * attn::v2::BQ)),
                       (unsigned)n_heads);
    cfg.dynamicSmemBytes = attn::v2::SMEM_BYTES;
    cfg.stream = st;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attn::attention_pair128_kernel, qm, km, vm, p);
    if (e != cudaSuccess) return cuda_status(e, "attention pair128 launch");
    return launch_status("attention pair128 launch");
  }
  CUtensorMap qm, km, vm;
  int rc = encode_tmap_heads(&qm, q, n_heads, seq, head_dim, attn::BQ);
  if (!rc) rc = encode_tmap_heads(&km, k, n_heads, seq, head_dim, pair ? attn::BKV / 2 : attn::BKV);
  if (!rc) rc = encode_tmap_heads(&vm, v, n_heads, seq, head_dim, attn::BKV);
  if (rc) return rc;
  // work units of the unsplit launch and the key split
  const int nkv = (seq + attn::BKV - 1) / attn::BKV;
  const long long qblocks = pair ? (seq + 4 * attn::BQ - 1) / (4 * attn::BQ)
                                 : (seq + 2 * attn::BQ - 1) / (2 * attn::BQ);
  int chunk = nkv;
  p.kv_split = choose_kv_split(qblocks * n_heads, pair ? pair_slots : num_sms(), nkv, &chunk);
  p.kv_chunk = chunk;
  void* part = nullptr;
  if (p.kv_split > 1) {
    // partial outputs + their log2 sums, stream-ordered, freed after the merge
    const size_t o_bytes = (size_t)p.kv_split * seq * n_heads * attn::HD * sizeof(float);
    const size_t l_bytes = (size_t)p.kv_split * n_heads * seq * sizeof(float);
    cudaError_t e = cudaMallocAsync(&part, o_bytes + l_bytes, st);
    if (e != cudaSuccess) return fail(-6, "attention: partial-output allocation failed");
    p.part_o = static_cast<float*>(part);
    p.part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(part) + o_bytes);
  }
  int rc2 = 0;
  {
    ProfScope prof("attention", 4.0 * (double)seq * seq * head_dim * n_heads,
                   4.0 * (double)seq * n_heads * head_dim * 2, st);
    if (!pair) {
      dim3 grid((unsigned)(qblocks * p.kv_split), n_heads);
      if (p.kv_split > 1)
        attn::attention_kernel<false, true><<<grid, attn::NUM_THREADS, attn::SMEM_BYTES, st>>>(qm, km, vm, p);
      else
        attn::attention_kernel<false, false><<<grid, attn::NUM_THREADS, attn::SMEM_BYTES, st>>>(qm, km, vm, p);
      rc2 = launch_status("attention_kernel launch");
    } else {
      cudaLaunchAttribute attr_c[1];
      cudaLaunchConfig_t cfg = attn_pair_config(attr_c);
      cfg.gridDim = dim3(2 * (unsigned)(qblocks * p.kv_split), (unsigned)n_heads);
      cfg.stream = st;
      const cudaError_t e =
          p.kv_split > 1 ? cudaLaunchKernelEx(&cfg, attn::attention_kernel<true, true>, qm, km, vm, p)
                         : cudaLaunchKernelEx(&cfg, attn::attention_kernel<true, false>, qm, km, vm, p);
      rc2 = e != cudaSuccess ? cuda_status(e, "attention pair launch")
                             : launch_status("attention pair launch");
    }
  }
  if (p.kv_split > 1) {
    if (rc2 == 0) {
      ProfScope prof("attention_combine", 0.0,
                     (double)seq * n_heads * attn::HD * (4.0 * p.kv_split + 2.0), st);
      const long long threads = (long long)seq * n_heads * (attn::HD / 8);
      attn::combine_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
          p.part_o, p.part_lse, p.kv_split, seq, n_heads, out, ld_out, p.routes);
      rc2 = launch_status("attention combine launch");
    }
    cudaFreeAsync(part, st);
  }
  return rc2;
}

}  // namespace bonsai
