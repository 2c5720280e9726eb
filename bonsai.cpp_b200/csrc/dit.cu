// DiT engine: weights, workspace and the denoise-step forward of
// build_diffuser_graph (src/diffuser_graph.cpp:231-561) on sm_100a kernels.
//
// Stage order per step (same tensors as the reference graph):
//   edges      img_in / txt_in linears, timestep embedding -> time MLP (+ the
//              pooled-vector MLP for Flux.1) -> vec, silu(vec) (:283-311)
//   modulation all per-block (Flux.1, B1_0) or shared (klein, f32) modulation
//              vectors computed once from silu(vec) (:307-320, :470-473)
//   double     19/5 double blocks on the text and image rows (:341-466)
//   single     38/20 single blocks on the joint rows (:476-542)
//   head       LayerNorm-modulate + proj_out on the image rows (:544-556)
// The hidden state is one f32 [txt + img][3072] buffer with the text rows
// first, so the reference's ggml_concat(h_txt, h_img) (:468) is free.
#include "../../include/bonsai_cuda.h"
#include "internal.cuh"
#include "ptx.cuh"

#include <cmath>
#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace bonsai {
namespace dit {

// ----------------------------------------------------------- weight RNG
// Counter-based generator: every element is a pure function of
// (seed, tensor id, element index), so tensors can be regenerated on demand.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__host__ __device__ __forceinline__ uint64_t tensor_key(uint64_t seed, uint64_t tid) {
  return splitmix64(seed * 0x100000001B3ull + splitmix64(tid));
}
__device__ __forceinline__ float normal_from(uint64_t r) {
  const uint32_t a = (uint32_t)(r >> 32), b = (uint32_t)r;
  const float u1 = ((float)a + 1.0f) * 2.3283064365386963e-10f;  // (0, 1]
  const float u2 = (float)b * 2.3283064365386963e-10f;
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Packed B1_0 bytes [rows][K/32][6]: signs Bernoulli(0.5), scale |N(0, std)| -> f16.
__global__ void gen_b1_kernel(uint8_t* __restrict__ dst, long long groups, uint64_t key,
                              float scale_std) {
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const uint64_t r1 = splitmix64(key + 2 * (uint64_t)g);
    const uint64_t r2 = splitmix64(key + 2 * (uint64_t)g + 1);
    const uint32_t sign = (uint32_t)r1;
    const __half s = __float2half_rn(fabsf(normal_from(r2)) * scale_std);
    const uint16_t sb = __half_as_ushort(s);
    uint8_t* p = dst + g * 6;
    p[0] = (uint8_t)(sb & 0xFF);
    p[1] = (uint8_t)(sb >> 8);
    p[2] = (uint8_t)(sign & 0xFF);
    p[3] = (uint8_t)((sign >> 8) & 0xFF);
    p[4] = (uint8_t)((sign >> 16) & 0xFF);
    p[5] = (uint8_t)(sign >> 24);
  }
}

__global__ void gen_f32_kernel(float* __restrict__ dst, long long n, uint64_t key, float mean,
                               float stdv) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    dst[i] = mean + stdv * normal_from(splitmix64(key + (uint64_t)i));
}

// --------------------------------------------------------------- config
struct Cfg {
  int preset = BONSAI_PRESET_FLUX1;
  int H = 3072, heads = 24, hd = 128;
  int depth = 19, depth_single = 38;
  int mlp = 12288;          // activation width
  int mlp_in_rows = 12288;  // rows of the MLP-in linear (2*mlp for SwiGLU)
  int in_ch = 64, ctx_dim = 4096, pooled = 768;
  int n_axes = 3;
  int axes[4] = {16, 56, 56, 0};
  float theta = 10000.f;
  bool per_block_mod = true;
  bool edge_bias = true;
  bool swiglu = false;
  int img = 4096, txt = 512, L = 4608;
  int grid_h = 64, grid_w = 64;
  uint64_t seed = 1234;
  int C() const { return H + mlp; }  // width of the single block's to_out input
};

enum Kind { KIND_B1 = 0, KIND_F32 = 1 };
struct TensorInfo {
  Kind kind;
  long long rows, cols;  // B1: out_dim, in_dim; F32: numel in rows*cols
  uint64_t tid;
  float mean, stdv;
  // Where the tensor lives on the device: B1 rows [row_off, row_off + rows)
  // of *b1 (row_off is a multiple of 128), or f32 values at f32.
  B1Weight* b1 = nullptr;
  long long row_off = 0;
  float* f32 = nullptr;
};

struct DoubleW {
  B1Weight img_qkv, txt_qkv, img_out, txt_out, img_mlp_in, img_mlp_out, txt_mlp_in, txt_mlp_out;
  float *nq_img, *nk_img, *nq_txt, *nk_txt;
};
struct SingleW {
  B1Weight proj, out;
  float *nq, *nk;
};

}  // namespace dit
}  // namespace bonsai

using namespace bonsai;
using namespace bonsai::dit;

// Flag words of the peer barrier: [0, kMaxPeers) arrivals, kFlagEpoch own count.
constexpr int kFlagWords = 64;
constexpr int kFlagEpoch = 32;

struct bonsai_dit {
  ~bonsai_dit();
  Cfg c;
  std::map<std::string, TensorInfo> reg;
  std::vector<void*> allocs;
  std::vector<DoubleW> dbl;
  std::vector<SingleW> sgl;
  B1Weight mod_all;  // Flux.1: every block's modulation linear stacked (rows)
  long long mod_rows = 0;
  // f32 edge weights
  float *img_in_w = nullptr, *img_in_b = nullptr, *txt_in_w = nullptr, *txt_in_b = nullptr;
  float *time_w1 = nullptr, *time_b1 = nullptr, *time_w2 = nullptr, *time_b2 = nullptr;
  float *vec_w1 = nullptr, *vec_b1 = nullptr, *vec_w2 = nullptr, *vec_b2 = nullptr;
  float *mod_img_w = nullptr, *mod_txt_w = nullptr, *mod_single_w = nullptr;
  float *norm_out_w = nullptr, *norm_out_b = nullptr, *proj_out_w = nullptr, *proj_out_b = nullptr;
  // The token-wide f32 edge linears (context embedder, image input, output
  // projection) also as bf16x3 weights [N][3K] for the tensor cores, kept in
  // step with the f32 ones; a3 = the split activations [M][3K].
  __nv_bfloat16 *txt_in_w3 = nullptr, *img_in_w3 = nullptr, *proj_out_w3 = nullptr, *a3 = nullptr;
  // workspace
  float* hidden = nullptr;   // [L][H]
  __half* xm = nullptr;      // [L][H]
  __half* qkv = nullptr;     // [3][heads][L][128]
  __half* cat = nullptr;     // [L][C]: attention out at [0,H), MLP activation at [H, H+mlp)
  float* tmp32 = nullptr;    // [img][H] (final LayerNorm-modulate)
  float* mods = nullptr;     // Flux.1: [mod_rows]; klein: [6H img | 6H txt | 3H single]
  float* fin = nullptr;      // [2H] norm_out modulation
  float* te = nullptr;       // [256] timestep embedding
  float* h256 = nullptr;     // [H] time MLP hidden
  float* vec = nullptr;      // [H]
  float* vtmp = nullptr;     // [H]
  float* vec_silu = nullptr; // [H]
  __half* vec_silu16 = nullptr;  // [8][H] (row 0 used; padded for TMA)
  float* cos_t = nullptr;    // [L][64]
  float* sin_t = nullptr;
  // CUDA graph of the step body (everything after the timestep copy), keyed
  // by the caller's buffer pointers; captured on a private stream, replayed
  // on the caller's stream.
  cudaStream_t cap_stream = nullptr;
  // The double blocks run their text-stream chain on `aux`, forked from and
  // joined back into the caller's stream inside each phase.
  cudaStream_t aux = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  cudaGraphExec_t graph = nullptr;
  const void* graph_key[4] = {nullptr, nullptr, nullptr, nullptr};
  long long graph_kernels = 0;
  int forwards = 0;
  // Multi-GPU partition (bonsai_dit_set_partition): this rank owns token
  // rows [r0, r1) and heads [h0, h0 + hl).  world == 1: everything.
  int rank = 0, world = 1;
  int r0 = 0, r1 = 0, h0 = 0, hl = 24;
  // Fused exchanges (bonsai_dit_set_peers): every rank's "xm" and "cat" as
  // seen from this device (peer mappings; [rank] = this model's own).  Phase
  // 0 then stores its xm rows into every rank's xm and phase 1 stores each
  // attention row into its owner's cat: no separate all-gather / all-to-all.
  bool fused = false;
  __half* peer_xm[kMaxPeers] = {};
  __half* peer_cat[kMaxPeers] = {};
  std::vector<void*> ipc_opened;  // peer mappings opened by bonsai_dit_open_peers
  // QKV scatter (bonsai_dit_set_qkv_peers, fused exchanges only): phase 0
  // computes q/k/v of this rank's own rows for every head and the GEMM
  // epilogue stores head h into peer_qkv[h / hl] (its owner's q/k/v buffer),
  // instead of phase 0 broadcasting xm rows and phase 1 computing the own
  // heads' q/k/v over every row.
  bool qkv_scatter = false;
  __half* peer_qkv[kMaxPeers] = {};
  std::vector<void*> ipc_opened_qkv;
  // Peer flag barrier (bonsai_dit_set_flag_peers / bonsai_dit_barrier): this
  // rank's flag words (kFlagWords u32, zeroed: [r] = the last barrier rank r
  // has reached, [kFlagEpoch] = this rank's own barrier count) and every
  // rank's as seen from this device.
  unsigned* flags = nullptr;
  unsigned* peer_flags[kMaxPeers] = {};
  bool flag_barrier = false;
  std::vector<void*> ipc_opened_flags;
  // device copies of caller inputs for the host-buffer entry point
  float *in_img = nullptr, *in_txt = nullptr, *in_pooled = nullptr, *out_buf = nullptr;
};

namespace {

int dev_alloc(bonsai_dit* m, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return fail(BONSAI_ERR_NOMEM, "dit: cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  m->allocs.push_back(*p);
  return 0;
}


int gen_b1_into(const Cfg& c, const TensorInfo& ti, uint8_t* dst, cudaStream_t st) {
  const long long groups = ti.rows * (ti.cols / 32);
  const long long blocks = std::min<long long>((groups + 255) / 256, 65535LL * 8);
  gen_b1_kernel<<<(unsigned)std::max<long long>(blocks, 1), 256, 0, st>>>(
      dst, groups, tensor_key(c.seed, ti.tid), ti.stdv);
  return launch_status("gen_b1 launch");
}
int gen_f32_into(const Cfg& c, const TensorInfo& ti, float* dst, cudaStream_t st) {
  const long long n = ti.rows * ti.cols;
  const long long blocks = std::min<long long>((n + 255) / 256, 65535LL * 8);
  gen_f32_kernel<<<(unsigned)std::max<long long>(blocks, 1), 256, 0, st>>>(
      dst, n, tensor_key(c.seed, ti.tid), ti.mean, ti.stdv);
  return launch_status("gen_f32 launch");
}

// Register and materialise one B1_0 weight (generated packed, then retiled).
int make_b1(bonsai_dit* m, const std::string& name, long long rows, long long cols,
            int swiglu_from, B1Weight& w, uint8_t* staging) {
  TensorInfo ti{KIND_B1, rows, cols, (uint64_t)m->reg.size() + 1, 0.f, 0.02f};
  ti.b1 = &w;
  m->reg[name] = ti;
  int rc = gen_b1_into(m->c, ti, staging, 0);
  if (rc) return rc;
  w = B1Weight{};
  w.n_rows = (int)rows;
  w.k_in = (int)cols;
  w.n_ftiles = (int)((rows + 127) / 128);
  w.k_blocks = (int)((cols + 63) / 64);
  w.swiglu_from = swiglu_from;
  cudaGetDevice(&w.device);
  rc = dev_alloc(m, reinterpret_cast<void**>(&w.chunks),
                 (size_t)w.n_ftiles * w.k_blocks * kChunkWords * 4);
  if (rc) return rc;
  return launch_b1_retile(staging, w, 0);
}

int make_f32(bonsai_dit* m, const std::string& name, long long rows, long long cols, float mean,
             float stdv, float** out) {
  TensorInfo ti{KIND_F32, rows, cols, (uint64_t)m->reg.size() + 1, mean, stdv};
  int rc = dev_alloc(m, reinterpret_cast<void**>(out), (size_t)rows * cols * 4);
  if (rc) return rc;
  ti.f32 = *out;
  m->reg[name] = ti;
  return gen_f32_into(m->c, ti, *out, 0);
}

// Re-split one of the token-wide edge weights into its bf16x3 copy.
int refresh_edge_w3(bonsai_dit* m, const std::string& name, cudaStream_t st) {
  const Cfg& c = m->c;
  if (name == "txt_in.w") return launch_split_bf16x3(m->txt_in_w, c.ctx_dim, c.H, c.ctx_dim, true, m->txt_in_w3, st);
  if (name == "img_in.w") return launch_split_bf16x3(m->img_in_w, c.in_ch, c.H, c.in_ch, true, m->img_in_w3, st);
  if (name == "proj_out.w") return launch_split_bf16x3(m->proj_out_w, c.H, c.in_ch, c.H, true, m->proj_out_w3, st);
  return 0;
}

long long tensor_bytes(const TensorInfo& ti) {
  return ti.kind == KIND_B1 ? ti.rows * (ti.cols / 32) * 6 : ti.rows * ti.cols * 4;
}

// The device B1_0 weight a registered tensor occupies: the whole weight, or
// whole 128-row tiles of a stacked one (the per-block modulation linears).
B1Weight b1_view(const TensorInfo& ti) {
  const B1Weight& w = *ti.b1;
  if (ti.row_off == 0 && ti.rows == w.n_rows) return w;
  B1Weight v = w;
  v.n_rows = (int)ti.rows;
  v.n_ftiles = (int)((ti.rows + 127) / 128);
  v.swiglu_from = -1;
  v.chunks = w.chunks + (size_t)(ti.row_off / 128) * w.k_blocks * kChunkWords;
  return v;
}

EpiSeg seg_of(int mode, int row_begin, int row_end, void* dst, long long ld, int col_off,
              const float* gate) {
  EpiSeg s;
  s.mode = mode;
  s.row_begin = row_begin;
  s.row_end = row_end;
  s.dst = dst;
  s.ld = ld;
  s.col_off = col_off;
  s.gate = gate;
  return s;
}

EpiSeg seg_qkv(const Cfg& c, int row_end, __half* qkv, int tok_off) {
  EpiSeg s;
  s.mode = EPI_QKV_F16;
  s.row_begin = 0;
  s.row_end = row_end;
  s.dst = qkv;
  s.heads = c.heads;
  s.seq_total = c.L;
  s.tok_off = tok_off;
  s.head_dim = c.hd;
  return s;
}

// seg_qkv whose heads go to their owners' q/k/v buffers (QKV scatter).
EpiSeg seg_qkv_routed(const bonsai_dit* m, int tok_off) {
  EpiSeg s = seg_qkv(m->c, 3 * m->c.H, m->qkv, tok_off);
  for (int r = 0; r < m->world; ++r) s.route[r] = m->peer_qkv[r];
  s.route_heads = m->hl;
  return s;
}

#define RC(x)              \
  do {                     \
    int _rc = (x);         \
    if (_rc) return _rc;   \
  } while (0)

// Modulation vectors of double block i: (img, txt) pointers to [6H].
void double_mods(bonsai_dit* m, int i, const float** mi, const float** mt) {
  const Cfg& c = m->c;
  if (c.per_block_mod) {
    *mi = m->mods + (size_t)i * 12 * c.H;
    *mt = *mi + 6 * c.H;
  } else {
    *mi = m->mods;
    *mt = m->mods + 6 * c.H;
  }
}
const float* single_mods(bonsai_dit* m, int i) {
  const Cfg& c = m->c;
  if (c.per_block_mod) return m->mods + (size_t)c.depth * 12 * c.H + (size_t)i * 3 * c.H;
  return m->mods + 12 * c.H;
}

// silu(vec) -> every modulation vector + the output-head modulation.
int compute_mods(bonsai_dit* m, cudaStream_t st) {
  const Cfg& c = m->c;
  RC(launch_silu_f32(m->vec, c.H, m->vec_silu, st));
  if (c.per_block_mod && b1_gemv_supported(m->mod_all)) {
    // every block's modulation linear at once: one row of silu(vec), so the
    // memory-bound B1_0 matrix-vector kernel (f32 activations)
    RC(launch_b1_gemv_f32(m->vec_silu, m->mod_all, m->mods, st));
  } else if (c.per_block_mod) {
    RC(launch_f32_to_f16(m->vec_silu, m->vec_silu16, c.H, st));
    EpiSeg s = seg_of(EPI_F32, 0, (int)m->mod_rows, m->mods, m->mod_rows, 0, nullptr);
    RC(launch_b1_gemm(m->vec_silu16, c.H, 1, m->mod_all, &s, 1, false, st));
  } else {
    RC(launch_linear_f32(m->vec_silu, c.H, 1, c.H, m->mod_img_w, nullptr, 6 * c.H, m->mods, 6 * c.H, false, st));
    RC(launch_linear_f32(m->vec_silu, c.H, 1, c.H, m->mod_txt_w, nullptr, 6 * c.H, m->mods + 6 * c.H, 6 * c.H, false, st));
    RC(launch_linear_f32(m->vec_silu, c.H, 1, c.H, m->mod_single_w, nullptr, 3 * c.H, m->mods + 12 * c.H, 3 * c.H, false, st));
  }
  return launch_linear_f32(m->vec_silu, c.H, 1, c.H, m->norm_out_w, m->norm_out_b, 2 * c.H, m->fin,
                           2 * c.H, false, st);
}

// Row ranges of this rank inside the text [0, Lt) and image [Lt, L) streams.
struct Span {
  int a, b;
  int n() const { return b > a ? b - a : 0; }
};
Span own_txt(const bonsai_dit* m) { return {std::max(0, m->r0), std::min(m->c.txt, m->r1)}; }
Span own_img(const bonsai_dit* m) { return {std::max(m->c.txt, m->r0), std::min(m->c.L, m->r1)}; }

// QKV tiles of this rank's heads: q, k and v parts of the fused [3H] weight.
TileSel head_tiles(const bonsai_dit* m) {
  TileSel t;
  t.groups = 3;
  t.count = m->hl;
  for (int g = 0; g < 3; ++g) t.base[g] = g * m->c.heads + m->h0;
  return t;
}

// The three phases of a double block (src/diffuser_graph.cpp:341-466).
// phase 0: LN-modulate (attention) of this rank's rows -> xm           (:347-352)
// phase 1: Q/K/V of this rank's heads on every row, Q/K RMSNorm + RoPE,
//          joint attention of those heads -> cat[:, heads]           (:354-416)
// phase 2: out-projection + gate-residual, LN-modulate, MLP + gate-residual
//          on this rank's rows (needs cat[own rows, all heads])      (:434-460)
// The stream of the double blocks' text-stream chain: m->aux, or st itself
// while per-launch profiling is on (concurrent kernels would stretch each
// other's event-timed durations).
cudaStream_t txt_stream(bonsai_dit* m, cudaStream_t st) { return profiling_active() ? st : m->aux; }
// The text stream starts after everything issued so far on st ...
int fork_aux(bonsai_dit* m, cudaStream_t st) {
  if (txt_stream(m, st) == st) return 0;
  RC(cuda_status(cudaEventRecord(m->ev_fork, st), "fork record"));
  return cuda_status(cudaStreamWaitEvent(m->aux, m->ev_fork, 0), "fork wait");
}
// ... and st continues only after everything issued on it.
int join_aux(bonsai_dit* m, cudaStream_t st) {
  if (txt_stream(m, st) == st) return 0;
  RC(cuda_status(cudaEventRecord(m->ev_join, m->aux), "join record"));
  return cuda_status(cudaStreamWaitEvent(st, m->ev_join, 0), "join wait");
}

// The other ranks' xm at the rows starting at `row` (fused exchanges only).
PeerCopies xm_copies(const bonsai_dit* m, int row) {
  PeerCopies pc;
  if (!m->fused) return pc;
  for (int r = 0; r < m->world; ++r)
    if (r != m->rank) pc.y[pc.n++] = m->peer_xm[r] + (size_t)row * m->c.H;
  return pc;
}
// Attention rows of this rank's heads routed to their owners' cat.
RowRoutes cat_routes(const bonsai_dit* m) {
  RowRoutes rr;
  if (!m->fused) return rr;
  const int rows = m->c.L / m->world;
  rr.n = m->world;
  for (int r = 0; r < m->world; ++r) {
    rr.outs[r] = m->peer_cat[r] + (size_t)m->h0 * m->c.hd;
    rr.row_bound[r] = r * rows;
  }
  rr.row_bound[m->world] = m->c.L;
  return rr;
}

int double_phase(bonsai_dit* m, int i, int phase, cudaStream_t st) {
  const Cfg& c = m->c;
  const DoubleW& w = m->dbl[i];
  const int H = c.H, Lt = c.txt, C = c.C();
  const float *mi, *mt;
  double_mods(m, i, &mi, &mt);
  const Span tx = own_txt(m), im = own_img(m);
  const cudaStream_t ts = txt_stream(m, st);
  // The text and image streams touch disjoint rows of hidden / xm / cat and
  // disjoint tokens of qkv until the joint attention: the text chain runs on
  // its own stream, concurrently with the image chain, and is joined back
  // into st before anything that reads both (and at the end of every phase).
  if (phase == 0 && m->qkv_scatter) {
    // own rows only: LN-modulate, then q/k/v of every head, each head stored
    // into its owner's q/k/v buffer by the GEMM epilogue
    RC(fork_aux(m, st));
    RC(launch_ln_modulate_f16(m->hidden + (size_t)tx.a * H, tx.n(), H, mt + 0 * H, mt + 1 * H, 1e-6f,
                              m->xm + (size_t)tx.a * H, H, ts));
    EpiSeg s = seg_qkv_routed(m, tx.a);
    RC(launch_b1_gemm(m->xm + (size_t)tx.a * H, H, tx.n(), w.txt_qkv, &s, 1, false, ts));
    RC(launch_ln_modulate_f16(m->hidden + (size_t)im.a * H, im.n(), H, mi + 0 * H, mi + 1 * H, 1e-6f,
                              m->xm + (size_t)im.a * H, H, st));
    s = seg_qkv_routed(m, im.a);
    RC(launch_b1_gemm(m->xm + (size_t)im.a * H, H, im.n(), w.img_qkv, &s, 1, false, st));
    return join_aux(m, st);
  }
  if (phase == 0) {
    RC(fork_aux(m, st));
    RC(launch_ln_modulate_f16_peers(m->hidden + (size_t)tx.a * H, tx.n(), H, mt + 0 * H, mt + 1 * H,
                                    1e-6f, m->xm + (size_t)tx.a * H, H, xm_copies(m, tx.a), ts));
    RC(launch_ln_modulate_f16_peers(m->hidden + (size_t)im.a * H, im.n(), H, mi + 0 * H, mi + 1 * H,
                                    1e-6f, m->xm + (size_t)im.a * H, H, xm_copies(m, im.a), st));
    return join_aux(m, st);
  }
  if (phase == 1 && m->qkv_scatter) {
    // every row of this rank's heads is in its q/k/v buffer (phase 0 of all ranks)
    const size_t hs = (size_t)c.L * c.hd;
    __half* q = m->qkv + (size_t)m->h0 * hs;
    __half* k = m->qkv + (size_t)(c.heads + m->h0) * hs;
    __half* v = m->qkv + (size_t)(2 * c.heads + m->h0) * hs;
    RC(launch_qk_norm_rope(q, k, m->hl, c.L, w.nq_txt, w.nq_img, w.nk_txt, w.nk_img, Lt, 1e-6f,
                           m->cos_t, m->sin_t, st));
    const RowRoutes rr = cat_routes(m);
    return launch_attention(q, k, v, m->hl, c.L, c.hd, 1.0f / sqrtf((float)c.hd),
                            m->cat + (size_t)m->h0 * c.hd, C, st, &rr);
  }
  if (phase == 1) {
    const TileSel sel = head_tiles(m);
    const TileSel* ps = m->world > 1 ? &sel : nullptr;
    RC(fork_aux(m, st));
    EpiSeg s = seg_qkv(c, 3 * H, m->qkv, 0);
    RC(launch_b1_gemm(m->xm, H, Lt, w.txt_qkv, &s, 1, false, ts, ps));
    s = seg_qkv(c, 3 * H, m->qkv, Lt);
    RC(launch_b1_gemm(m->xm + (size_t)Lt * H, H, c.img, w.img_qkv, &s, 1, false, st, ps));
    RC(join_aux(m, st));
    const size_t hs = (size_t)c.L * c.hd;  // one head of one of q/k/v
    __half* q = m->qkv + (size_t)m->h0 * hs;
    __half* k = m->qkv + (size_t)(c.heads + m->h0) * hs;
    __half* v = m->qkv + (size_t)(2 * c.heads + m->h0) * hs;
    // rms_norm_qk (:371-374) + RoPE (:383-384); text rows use the added-stream weights
    RC(launch_qk_norm_rope(q, k, m->hl, c.L, w.nq_txt, w.nq_img, w.nk_txt, w.nk_img, Lt, 1e-6f,
                           m->cos_t, m->sin_t, st));
    // joint attention over [txt; img] (:393-416)
    const RowRoutes rr = cat_routes(m);
    return launch_attention(q, k, v, m->hl, c.L, c.hd, 1.0f / sqrtf((float)c.hd),
                            m->cat + (size_t)m->h0 * c.hd, C, st, m->fused ? &rr : nullptr);
  }
  // phase 2, per stream on this rank's rows (text on its own stream)
  const int act_mode = c.swiglu ? EPI_SWIGLU_F16 : EPI_GELU_F16;
  RC(fork_aux(m, st));
  for (int sidx = 0; sidx < 2; ++sidx) {
    const Span sp = sidx == 0 ? tx : im;
    if (sp.n() == 0) continue;
    const cudaStream_t ss = sidx == 0 ? ts : st;
    const float* md = sidx == 0 ? mt : mi;
    const B1Weight& w_out = sidx == 0 ? w.txt_out : w.img_out;
    const B1Weight& w_in = sidx == 0 ? w.txt_mlp_in : w.img_mlp_in;
    const B1Weight& w_o2 = sidx == 0 ? w.txt_mlp_out : w.img_mlp_out;
    float* h = m->hidden + (size_t)sp.a * H;
    __half* x = m->xm + (size_t)sp.a * H;
    __half* a = m->cat + (size_t)sp.a * C;
    EpiSeg s = seg_of(EPI_RESID_F32, 0, H, h, H, 0, md + 2 * H);
    s.split_ok = m->world > 1;
    RC(launch_b1_gemm(a, C, sp.n(), w_out, &s, 1, false, ss));
    RC(launch_ln_modulate_f16(h, sp.n(), H, md + 3 * H, md + 4 * H, 1e-6f, x, H, ss));
    s = seg_of(act_mode, 0, c.mlp_in_rows, a, C, H, nullptr);
    RC(launch_b1_gemm(x, H, sp.n(), w_in, &s, 1, false, ss));
    s = seg_of(EPI_RESID_F32, 0, H, h, H, 0, md + 5 * H);
    s.split_ok = m->world > 1;
    RC(launch_b1_gemm(a + H, C, sp.n(), w_o2, &s, 1, false, ss));
  }
  return join_aux(m, st);
}

// The three phases of a single block (src/diffuser_graph.cpp:476-542).
// phase 0: LN-modulate of this rank's rows -> xm                      (:479-480)
// phase 1: Q/K/V rows of to_qkv_mlp_proj for this rank's heads on every
//          row, Q/K RMSNorm + RoPE, attention of those heads -> cat    (:482-519)
// phase 2: MLP rows of to_qkv_mlp_proj + activation, then to_out and the
//          gate-residual on this rank's rows                          (:533-538)
int single_phase(bonsai_dit* m, int i, int phase, cudaStream_t st) {
  const Cfg& c = m->c;
  const SingleW& w = m->sgl[i];
  const int H = c.H, L = c.L, C = c.C();
  const float* md = single_mods(m, i);
  const int rows = m->r1 - m->r0;
  if (m->qkv_scatter) {
    const size_t hs = (size_t)L * c.hd;
    if (phase == 0) {
      // own rows: LN-modulate, then to_qkv_mlp_proj in one launch -- q/k/v of
      // every head to the heads' owners, the MLP activation into own cat rows
      RC(launch_ln_modulate_f16(m->hidden + (size_t)m->r0 * H, rows, H, md, md + H, 1e-6f,
                                m->xm + (size_t)m->r0 * H, H, st));
      EpiSeg segs[2];
      segs[0] = seg_qkv_routed(m, m->r0);
      segs[1] = seg_of(c.swiglu ? EPI_SWIGLU_F16 : EPI_GELU_F16, 3 * H, 3 * H + c.mlp_in_rows,
                       m->cat + (size_t)m->r0 * C, C, H, nullptr);
      return launch_b1_gemm(m->xm + (size_t)m->r0 * H, H, rows, w.proj, segs, 2, false, st);
    }
    if (phase == 1) {
      __half* q = m->qkv + (size_t)m->h0 * hs;
      __half* k = m->qkv + (size_t)(c.heads + m->h0) * hs;
      __half* v = m->qkv + (size_t)(2 * c.heads + m->h0) * hs;
      RC(launch_qk_norm_rope(q, k, m->hl, L, w.nq, w.nq, w.nk, w.nk, L, 1e-6f, m->cos_t, m->sin_t, st));
      const RowRoutes rr = cat_routes(m);
      return launch_attention(q, k, v, m->hl, L, c.hd, 1.0f / sqrtf((float)c.hd),
                              m->cat + (size_t)m->h0 * c.hd, C, st, &rr);
    }
    EpiSeg s = seg_of(EPI_RESID_F32, 0, H, m->hidden + (size_t)m->r0 * H, H, 0, md + 2 * H);
    s.split_ok = m->world > 1;
    return launch_b1_gemm(m->cat + (size_t)m->r0 * C, C, rows, w.out, &s, 1, false, st);
  }
  if (phase == 0)
    return launch_ln_modulate_f16_peers(m->hidden + (size_t)m->r0 * H, rows, H, md, md + H, 1e-6f,
                                        m->xm + (size_t)m->r0 * H, H, xm_copies(m, m->r0), st);
  if (phase == 1) {
    TileSel sel = head_tiles(m);
    EpiSeg s = seg_qkv(c, 3 * H, m->qkv, 0);
    RC(launch_b1_gemm(m->xm, H, L, w.proj, &s, 1, false, st, &sel));
    const size_t hs = (size_t)L * c.hd;
    __half* q = m->qkv + (size_t)m->h0 * hs;
    __half* k = m->qkv + (size_t)(c.heads + m->h0) * hs;
    __half* v = m->qkv + (size_t)(2 * c.heads + m->h0) * hs;
    RC(launch_qk_norm_rope(q, k, m->hl, L, w.nq, w.nq, w.nk, w.nk, L, 1e-6f, m->cos_t, m->sin_t, st));
    const RowRoutes rr = cat_routes(m);
    return launch_attention(q, k, v, m->hl, L, c.hd, 1.0f / sqrtf((float)c.hd),
                            m->cat + (size_t)m->h0 * c.hd, C, st, m->fused ? &rr : nullptr);
  }
  // MLP part of to_qkv_mlp_proj (rows [3H, 3H + mlp_in_rows)) on this rank's rows
  TileSel mlp;
  mlp.groups = 1;
  mlp.base[0] = 3 * H / 128;
  mlp.count = (c.mlp_in_rows + 127) / 128;
  EpiSeg s = seg_of(c.swiglu ? EPI_SWIGLU_F16 : EPI_GELU_F16, 3 * H, 3 * H + c.mlp_in_rows,
                    m->cat + (size_t)m->r0 * C, C, H, nullptr);
  RC(launch_b1_gemm(m->xm + (size_t)m->r0 * H, H, rows, w.proj, &s, 1, false, st, &mlp));
  s = seg_of(EPI_RESID_F32, 0, H, m->hidden + (size_t)m->r0 * H, H, 0, md + 2 * H);
  s.split_ok = m->world > 1;
  return launch_b1_gemm(m->cat + (size_t)m->r0 * C, C, rows, w.out, &s, 1, false, st);
}

int run_double(bonsai_dit* m, int i, cudaStream_t st) {
  for (int ph = 0; ph < 3; ++ph) RC(double_phase(m, i, ph, st));
  return 0;
}

int run_single(bonsai_dit* m, int i, cudaStream_t st) {
  if (m->world > 1) {
    for (int ph = 0; ph < 3; ++ph) RC(single_phase(m, i, ph, st));
    return 0;
  }
  // One rank: the fused to_qkv_mlp_proj GEMM covers both segments in one launch.
  const Cfg& c = m->c;
  const SingleW& w = m->sgl[i];
  const int H = c.H, L = c.L, C = c.C();
  const float* md = single_mods(m, i);
  RC(single_phase(m, i, 0, st));
  EpiSeg segs[2];
  segs[0] = seg_qkv(c, 3 * H, m->qkv, 0);
  segs[1] = seg_of(c.swiglu ? EPI_SWIGLU_F16 : EPI_GELU_F16, 3 * H, 3 * H + c.mlp_in_rows, m->cat,
                   C, H, nullptr);
  RC(launch_b1_gemm(m->xm, H, L, w.proj, segs, 2, false, st));
  __half* q = m->qkv;
  __half* k = m->qkv + (size_t)c.heads * L * c.hd;
  __half* v = k + (size_t)c.heads * L * c.hd;
  RC(launch_qk_norm_rope(q, k, c.heads, L, w.nq, w.nq, w.nk, w.nk, L, 1e-6f, m->cos_t, m->sin_t, st));
  RC(launch_attention(q, k, v, c.heads, L, c.hd, 1.0f / sqrtf((float)c.hd), m->cat, C, st));
  EpiSeg s = seg_of(EPI_RESID_F32, 0, H, m->hidden, H, 0, md + 2 * H);
  return launch_b1_gemm(m->cat, C, L, w.out, &s, 1, false, st);
}

}  // namespace

// Stream-ordered barrier of the partitioned ranks over peer memory (one
// process per GPU).  Lane r < world stores this rank's new barrier count into
// word [rank] of rank r's flags (a system-scope release store: the kernels
// issued before it on this stream have completed and ended with a
// system-scope fence after their peer stores), then waits until word [r] of
// this rank's own flags has reached the same count (acquire loads of local
// memory; every rank takes the barriers in the same order, so a rank is at
// most one barrier ahead and counts only grow).  Kernels after it on the
// stream therefore see everything the other ranks wrote into this GPU's
// buffers before their own barrier.  The wait gives up after kWaitLimitNs
// and records DEV_ERR_TIMEOUT_BARRIER (a rank that never arrives).
struct FlagPeers {
  unsigned* f[kMaxPeers];
};
__global__ void peer_barrier_kernel(FlagPeers peers, unsigned* __restrict__ own, int rank,
                                    int world, int* err) {
  const int lane = threadIdx.x;
  unsigned e = 0;
  if (lane == 0) {
    e = own[kFlagEpoch] + 1;
    own[kFlagEpoch] = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  if (lane < world) {
    unsigned* dst = peers.f[0];
#pragma unroll
    for (int r = 1; r < kMaxPeers; ++r)  // static indices: the pointers stay in parameter space
      if (r == lane) dst = peers.f[r];
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst + rank), "r"(e) : "memory");
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own + lane) : "memory");
      if ((int)(v - e) >= 0) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_BARRIER);
        break;
      }
    }
  }
  __syncwarp();
}

extern "C" {

int bonsai_dit_create(const bonsai_dit_config* cfg, bonsai_dit_t* out) {
  if (!cfg || !out) return fail(BONSAI_ERR_ARG, "dit_create: null argument");
  *out = nullptr;
  std::unique_ptr<bonsai_dit> m(new bonsai_dit());
  Cfg& c = m->c;
  if (cfg->preset == BONSAI_PRESET_KLEIN4B) {
    // DiffuserParams (src/diffuser_types.h:13-30)
    c.preset = BONSAI_PRESET_KLEIN4B;
    c.depth = 5;
    c.depth_single = 20;
    c.mlp = 9216;
    c.mlp_in_rows = 2 * 9216;
    c.in_ch = 128;
    c.ctx_dim = 7680;
    c.pooled = 0;
    c.n_axes = 4;
    c.axes[0] = c.axes[1] = c.axes[2] = c.axes[3] = 32;
    c.theta = 2000.f;
    c.per_block_mod = false;
    c.edge_bias = false;
    c.swiglu = true;
  } else if (cfg->preset != BONSAI_PRESET_FLUX1) {
    return fail(BONSAI_ERR_ARG, "dit_create: unknown preset");
  }
  if (cfg->depth > 0) c.depth = std::min(cfg->depth, c.depth);
  if (cfg->depth_single > 0) c.depth_single = std::min(cfg->depth_single, c.depth_single);
  if (cfg->depth < 0 || cfg->depth_single < 0) return fail(BONSAI_ERR_ARG, "dit_create: negative depth");
  c.img = cfg->img_tokens;
  c.txt = cfg->txt_tokens;
  c.L = c.img + c.txt;
  m->r0 = 0;
  m->r1 = c.L;
  m->h0 = 0;
  m->hl = c.heads;
  c.grid_h = cfg->grid_h;
  c.grid_w = cfg->grid_w;
  c.seed = cfg->seed;
  if (c.img <= 0 || c.txt < 0 || c.grid_h * c.grid_w != c.img)
    return fail(BONSAI_ERR_ARG, "dit_create: need img_tokens > 0 == grid_h * grid_w and txt_tokens >= 0");
  const int H = c.H;
  const long long L = c.L;
  cudaStream_t st = 0;

  // ---------------------------------------------------------- weights
  long long max_rows = 3LL * H + c.mlp_in_rows;
  long long max_cols = std::max<long long>(H, c.mlp) + H;
  long long staging_bytes = max_rows * (max_cols / 32) * 6;
  if (c.per_block_mod) {
    m->mod_rows = (long long)c.depth * 12 * H + (long long)c.depth_single * 3 * H;
    staging_bytes = std::max(staging_bytes, m->mod_rows * (H / 32) * 6);
  }
  uint8_t* staging = nullptr;
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&staging), (size_t)staging_bytes));
  m->dbl.resize(c.depth);
  m->sgl.resize(c.depth_single);
  const int mlp_swiglu_from = c.swiglu ? 0 : -1;
  for (int i = 0; i < c.depth; ++i) {
    DoubleW& w = m->dbl[i];
    const std::string p = "double." + std::to_string(i) + ".";
    RC(make_b1(m.get(), p + "img_qkv", 3 * H, H, -1, w.img_qkv, staging));
    RC(make_b1(m.get(), p + "txt_qkv", 3 * H, H, -1, w.txt_qkv, staging));
    RC(make_b1(m.get(), p + "img_out", H, H, -1, w.img_out, staging));
    RC(make_b1(m.get(), p + "txt_out", H, H, -1, w.txt_out, staging));
    RC(make_b1(m.get(), p + "img_mlp_in", c.mlp_in_rows, H, mlp_swiglu_from, w.img_mlp_in, staging));
    RC(make_b1(m.get(), p + "img_mlp_out", H, c.mlp, -1, w.img_mlp_out, staging));
    RC(make_b1(m.get(), p + "txt_mlp_in", c.mlp_in_rows, H, mlp_swiglu_from, w.txt_mlp_in, staging));
    RC(make_b1(m.get(), p + "txt_mlp_out", H, c.mlp, -1, w.txt_mlp_out, staging));
    RC(make_f32(m.get(), p + "img_norm_q", 1, c.hd, 1.f, 0.1f, &w.nq_img));
    RC(make_f32(m.get(), p + "img_norm_k", 1, c.hd, 1.f, 0.1f, &w.nk_img));
    RC(make_f32(m.get(), p + "txt_norm_q", 1, c.hd, 1.f, 0.1f, &w.nq_txt));
    RC(make_f32(m.get(), p + "txt_norm_k", 1, c.hd, 1.f, 0.1f, &w.nk_txt));
  }
  for (int i = 0; i < c.depth_single; ++i) {
    SingleW& w = m->sgl[i];
    const std::string p = "single." + std::to_string(i) + ".";
    RC(make_b1(m.get(), p + "proj", 3 * H + c.mlp_in_rows, H, c.swiglu ? 3 * H : -1, w.proj, staging));
    RC(make_b1(m.get(), p + "out", H, c.C(), -1, w.out, staging));
    RC(make_f32(m.get(), p + "norm_q", 1, c.hd, 1.f, 0.1f, &w.nq));
    RC(make_f32(m.get(), p + "norm_k", 1, c.hd, 1.f, 0.1f, &w.nk));
  }
  if (c.per_block_mod) {
    // Flux.1 per-block modulation linears (B1_0: 2-D tensors under the block
    // prefixes are quantized by convert_to_b1_0_packed.py:46-54), stacked so
    // one GEMV launch produces every block's vectors.
    long long row = 0;
    for (int i = 0; i < c.depth; ++i)
      for (const char* s : {"img_mod", "txt_mod"}) {
        TensorInfo ti{KIND_B1, 6LL * H, H, (uint64_t)m->reg.size() + 1, 0.f, 0.02f};
        ti.b1 = &m->mod_all;
        ti.row_off = row;
        m->reg["double." + std::to_string(i) + "." + s] = ti;
        RC(gen_b1_into(c, ti, staging + row * (H / 32) * 6, st));
        row += 6LL * H;
      }
    for (int i = 0; i < c.depth_single; ++i) {
      TensorInfo ti{KIND_B1, 3LL * H, H, (uint64_t)m->reg.size() + 1, 0.f, 0.02f};
      ti.b1 = &m->mod_all;
      ti.row_off = row;
      m->reg["single." + std::to_string(i) + ".mod"] = ti;
      RC(gen_b1_into(c, ti, staging + row * (H / 32) * 6, st));
      row += 3LL * H;
    }
    B1Weight& w = m->mod_all;
    w.n_rows = (int)m->mod_rows;
    w.k_in = H;
    w.n_ftiles = (int)((m->mod_rows + 127) / 128);
    w.k_blocks = (H + 63) / 64;
    cudaGetDevice(&w.device);
    RC(dev_alloc(m.get(), reinterpret_cast<void**>(&w.chunks),
                 (size_t)w.n_ftiles * w.k_blocks * kChunkWords * 4));
    RC(launch_b1_retile(staging, w, st));
  } else {
    RC(make_f32(m.get(), "mod_img.w", 6LL * H, H, 0.f, 0.02f, &m->mod_img_w));
    RC(make_f32(m.get(), "mod_txt.w", 6LL * H, H, 0.f, 0.02f, &m->mod_txt_w));
    RC(make_f32(m.get(), "mod_single.w", 3LL * H, H, 0.f, 0.02f, &m->mod_single_w));
  }
  const float bstd = c.edge_bias ? 0.02f : 0.f;
  RC(make_f32(m.get(), "img_in.w", H, c.in_ch, 0.f, 0.02f, &m->img_in_w));
  RC(make_f32(m.get(), "txt_in.w", H, c.ctx_dim, 0.f, 0.02f, &m->txt_in_w));
  RC(make_f32(m.get(), "time.w1", H, 256, 0.f, 0.02f, &m->time_w1));
  RC(make_f32(m.get(), "time.w2", H, H, 0.f, 0.02f, &m->time_w2));
  RC(make_f32(m.get(), "norm_out.w", 2LL * H, H, 0.f, 0.02f, &m->norm_out_w));
  RC(make_f32(m.get(), "proj_out.w", c.in_ch, H, 0.f, 0.02f, &m->proj_out_w));
  if (c.edge_bias) {
    RC(make_f32(m.get(), "img_in.b", 1, H, 0.f, bstd, &m->img_in_b));
    RC(make_f32(m.get(), "txt_in.b", 1, H, 0.f, bstd, &m->txt_in_b));
    RC(make_f32(m.get(), "time.b1", 1, H, 0.f, bstd, &m->time_b1));
    RC(make_f32(m.get(), "time.b2", 1, H, 0.f, bstd, &m->time_b2));
    RC(make_f32(m.get(), "norm_out.b", 1, 2 * H, 0.f, bstd, &m->norm_out_b));
    RC(make_f32(m.get(), "proj_out.b", 1, c.in_ch, 0.f, bstd, &m->proj_out_b));
  }
  if (c.pooled > 0) {
    RC(make_f32(m.get(), "vec.w1", H, c.pooled, 0.f, 0.02f, &m->vec_w1));
    RC(make_f32(m.get(), "vec.b1", 1, H, 0.f, bstd, &m->vec_b1));
    RC(make_f32(m.get(), "vec.w2", H, H, 0.f, 0.02f, &m->vec_w2));
    RC(make_f32(m.get(), "vec.b2", 1, H, 0.f, bstd, &m->vec_b2));
  }

  // bf16x3 copies of the token-wide edge weights
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->txt_in_w3), (size_t)H * 3 * c.ctx_dim * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->img_in_w3), (size_t)H * 3 * c.in_ch * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->proj_out_w3), (size_t)c.in_ch * 3 * H * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->a3),
               (size_t)std::max({(long long)c.txt * c.ctx_dim, (long long)c.img * c.in_ch,
                                 (long long)c.img * H}) * 3 * 2));
  for (const char* n : {"txt_in.w", "img_in.w", "proj_out.w"}) RC(refresh_edge_w3(m.get(), n, st));

  // -------------------------------------------------------- workspace
  const long long C = c.C();
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->hidden), (size_t)L * H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->xm), (size_t)L * H * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->qkv), (size_t)3 * c.heads * L * c.hd * 2));
  // its own allocation, so that its IPC handle maps exactly these words
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->flags), kFlagWords * sizeof(unsigned)));
  RC(cuda_status(cudaMemset(m->flags, 0, kFlagWords * sizeof(unsigned)), "dit_create: flags"));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->cat), (size_t)L * C * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->tmp32), (size_t)c.img * H * 4));
  const long long nmods = c.per_block_mod ? m->mod_rows : 15LL * H;
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->mods), (size_t)nmods * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->fin), (size_t)2 * H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->te), 256 * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->h256), (size_t)H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->vec), (size_t)H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->vtmp), (size_t)H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->vec_silu), (size_t)H * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->vec_silu16), (size_t)8 * H * 2));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->cos_t), (size_t)L * 64 * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->sin_t), (size_t)L * 64 * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->in_img), (size_t)c.img * c.in_ch * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->in_txt), (size_t)std::max(c.txt, 1) * c.ctx_dim * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->in_pooled), (size_t)std::max(c.pooled, 1) * 4));
  RC(dev_alloc(m.get(), reinterpret_cast<void**>(&m->out_buf), (size_t)c.img * c.in_ch * 4));
  // The image-stream chain (captured on cap_stream) outranks the text-stream
  // chain (aux): the persistent image GEMMs take every SM first and the
  // 512-token text GEMMs fill the SMs their last, partly filled wave leaves
  // idle, instead of delaying their start (measured -0.35 ms per step).
  int prio_least = 0, prio_greatest = 0;
  RC(cuda_status(cudaDeviceGetStreamPriorityRange(&prio_least, &prio_greatest), "stream priorities"));
  RC(cuda_status(cudaStreamCreateWithPriority(&m->cap_stream, cudaStreamNonBlocking, prio_greatest),
                 "capture stream"));
  RC(cuda_status(cudaStreamCreateWithPriority(&m->aux, cudaStreamNonBlocking, prio_least), "aux stream"));
  RC(cuda_status(cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming), "fork event"));
  RC(cuda_status(cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming), "join event"));
  cudaMemset(m->vec_silu16, 0, (size_t)8 * H * 2);

  // RoPE ids (src/diffuser.cpp:240-249): text rows 0, image rows (.., y, x)
  // on the last two axes; tables built once (they do not change per step).
  {
    std::vector<float> ids((size_t)L * c.n_axes, 0.f);
    for (int y = 0; y < c.grid_h; ++y)
      for (int x = 0; x < c.grid_w; ++x) {
        const size_t t = (size_t)c.txt + (size_t)y * c.grid_w + x;
        ids[t * c.n_axes + c.n_axes - 2] = (float)y;
        ids[t * c.n_axes + c.n_axes - 1] = (float)x;
      }
    float* ids_d = nullptr;
    RC(dev_alloc(m.get(), reinterpret_cast<void**>(&ids_d), ids.size() * 4));
    int half = 0;
    for (int a = 0; a < c.n_axes; ++a) half += c.axes[a] / 2;
    if (half != 64) return fail(BONSAI_ERR_UNSUPPORTED, "dit_create: RoPE axes must cover head_dim 128");
    std::vector<int> pa(half);
    std::vector<float> pf(half);
    rope_pair_table(c.axes, c.n_axes, c.theta, pa.data(), pf.data());
    int* tab = nullptr;
    RC(dev_alloc(m.get(), reinterpret_cast<void**>(&tab), (size_t)half * 8));
    RC(cuda_status(cudaMemcpy(ids_d, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice), "ids copy"));
    RC(cuda_status(cudaMemcpy(tab, pa.data(), half * 4, cudaMemcpyHostToDevice), "rope table copy"));
    RC(cuda_status(cudaMemcpy(tab + half, pf.data(), half * 4, cudaMemcpyHostToDevice), "rope table copy"));
    RC(launch_rope_tables(ids_d, (int)L, c.n_axes, tab, reinterpret_cast<float*>(tab + half), half,
                          m->cos_t, m->sin_t, st));
  }
  RC(cuda_status(cudaDeviceSynchronize(), "dit_create"));
  *out = m.release();
  return 0;
}

// Releases everything the model owns (also when bonsai_dit_create fails
// part-way and its unique_ptr deletes the half-built model).
bonsai_dit::~bonsai_dit() {
  cudaDeviceSynchronize();
  for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
  for (void* p : ipc_opened_qkv) cudaIpcCloseMemHandle(p);
  for (void* p : ipc_opened_flags) cudaIpcCloseMemHandle(p);
  if (graph) cudaGraphExecDestroy(graph);
  if (cap_stream) cudaStreamDestroy(cap_stream);
  if (aux) cudaStreamDestroy(aux);
  if (ev_fork) cudaEventDestroy(ev_fork);
  if (ev_join) cudaEventDestroy(ev_join);
  for (void* p : allocs) cudaFree(p);
}

int bonsai_dit_destroy(bonsai_dit_t m) {
  delete m;
  return 0;
}

// ggml_timestep_embedding(t, 256, 10000) with the [sin, cos] half swap
// (src/diffuser_graph.cpp:288-292), evaluated on the host in f32 and copied
// into the device buffer m->te.  The source is a stack array (pageable): the
// runtime stages it before returning, so back-to-back calls cannot race on it.
static int dit_upload_timestep(bonsai_dit* m, float timestep, cudaStream_t st) {
  float te[256];
  for (int j = 0; j < 128; ++j) {
    const float freq = expf(-logf(10000.0f) * (float)j / 128.0f);
    const float arg = timestep * freq;
    te[j] = sinf(arg);
    te[128 + j] = cosf(arg);
  }
  return cuda_status(cudaMemcpyAsync(m->te, te, sizeof(te), cudaMemcpyHostToDevice, st), "te copy");
}

static int dit_prepare_vec(bonsai_dit* m, const float* pooled, cudaStream_t st) {
  const Cfg& c = m->c;
  // time MLP (:294-305): vec = W2 silu(W1 te + b1) + b2
  RC(launch_linear_f32(m->te, 256, 1, 256, m->time_w1, m->time_b1, c.H, m->h256, c.H, false, st));
  RC(launch_linear_f32(m->h256, c.H, 1, c.H, m->time_w2, m->time_b2, c.H, m->vec, c.H, true, st));
  if (c.pooled > 0) {
    if (!pooled) return fail(BONSAI_ERR_ARG, "dit_forward: the Flux.1 preset needs the pooled vector");
    RC(launch_linear_f32(pooled, c.pooled, 1, c.pooled, m->vec_w1, m->vec_b1, c.H, m->h256, c.H, false, st));
    RC(launch_linear_f32(m->h256, c.H, 1, c.H, m->vec_w2, m->vec_b2, c.H, m->vtmp, c.H, true, st));
    RC(launch_add_f32(m->vec, m->vtmp, c.H, m->vec, st));
  }
  return compute_mods(m, st);
}

// A token-wide f32 edge linear: on the tensor cores as bf16x3 when the
// activations allow it (rows 16-byte aligned, K % 8 == 0), else the f32 CUDA
// core kernel with its split-K workspace.
static int edge_linear(bonsai_dit* m, const float* x, long long ldx, int M, int K, const float* W,
                       const __nv_bfloat16* w3, const float* b, int N, float* y, long long ldy,
                       cudaStream_t st, float* ws, long long ws_elems) {
  if (K % 8 == 0 && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0)
    return launch_linear_bf16x3(x, ldx, M, K, w3, b, N, y, ldy, m->a3, st);
  return launch_linear_f32(x, ldx, M, K, W, b, N, y, ldy, false, st, ws, ws_elems);
}

// Everything of the step after the timestep upload (all stream-ordered kernel
// launches with fixed pointers).
static int dit_forward_body(bonsai_dit* m, const float* img, const float* txt, const float* pooled,
                            float* out, cudaStream_t st) {
  const Cfg& c = m->c;
  // input projections (:283-286), text rows first in the hidden state
  RC(edge_linear(m, txt, c.ctx_dim, c.txt, c.ctx_dim, m->txt_in_w, m->txt_in_w3, m->txt_in_b, c.H,
                 m->hidden, c.H, st, m->tmp32, (long long)c.img * c.H));
  RC(edge_linear(m, img, c.in_ch, c.img, c.in_ch, m->img_in_w, m->img_in_w3, m->img_in_b, c.H,
                 m->hidden + (size_t)c.txt * c.H, c.H, st, nullptr, 0));
  RC(dit_prepare_vec(m, pooled, st));
  for (int i = 0; i < c.depth; ++i) RC(run_double(m, i, st));
  for (int i = 0; i < c.depth_single; ++i) RC(run_single(m, i, st));
  // output head (:544-556): norm_out modulation is (scale, shift)
  const float* h_img = m->hidden + (size_t)c.txt * c.H;
  RC(launch_ln_modulate_f32(h_img, c.img, c.H, m->fin + c.H, m->fin, 1e-6f, m->tmp32, c.H, st));
  // (f32 fallback: cat, free by now, holds the split-K partial sums)
  return edge_linear(m, m->tmp32, c.H, c.img, c.H, m->proj_out_w, m->proj_out_w3, m->proj_out_b,
                     c.in_ch, out, c.in_ch, st, reinterpret_cast<float*>(m->cat),
                     (long long)c.L * c.C() / 2);
}

int bonsai_dit_forward(bonsai_dit_t m, const float* img, const float* txt, const float* pooled,
                       float timestep, float* out, void* stream) {
  if (!m || !img || !out || (m->c.txt > 0 && !txt)) return fail(BONSAI_ERR_ARG, "dit_forward: null argument");
  if (m->c.pooled > 0 && !pooled)
    return fail(BONSAI_ERR_ARG, "dit_forward: the Flux.1 preset needs the pooled vector");
  if (m->world > 1)
    return fail(BONSAI_ERR_ARG,
                "dit_forward: a partitioned model is driven with bonsai_dit_begin/phase/end");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RC(dit_upload_timestep(m, timestep, st));
  // The first call runs eagerly (it also performs one-time kernel set-up);
  // later calls replay a CUDA graph of the body.  Profiling runs eagerly so
  // every launch keeps its own events.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  const bool use_graph = m->forwards++ > 0 && !profiling_active() && cs == cudaStreamCaptureStatusNone;
  if (!use_graph) return dit_forward_body(m, img, txt, pooled, out, st);
  const void* key[4] = {img, txt, pooled, out};
  if (!m->graph || memcmp(key, m->graph_key, sizeof(key)) != 0) {
    if (m->graph) {
      cudaGraphExecDestroy(m->graph);
      m->graph = nullptr;
    }
    // the body must see the timestep copy and the caller's earlier work:
    // capture on the private stream, launch on the caller's.
    const long long before = launch_counter();
    RC(cuda_status(cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeThreadLocal),
                   "begin capture"));
    int rc = dit_forward_body(m, img, txt, pooled, out, m->cap_stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->cap_stream, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return cuda_status(e, "end capture");
    e = cudaGraphInstantiate(&m->graph, g, cudaGraphInstantiateFlagUseNodePriority);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      m->graph = nullptr;
      return cuda_status(e, "graph instantiate");
    }
    m->graph_kernels = launch_counter() - before;
    launch_counter_add(-m->graph_kernels);  // counted again when replayed below
    memcpy(m->graph_key, key, sizeof(key));
  }
  RC(cuda_status(cudaGraphLaunch(m->graph, st), "graph launch"));
  launch_counter_add(m->graph_kernels);
  return 0;
}

int bonsai_dit_forward_host(bonsai_dit_t m, const float* host_img, const float* host_txt,
                            const float* host_pooled, float timestep, float* host_out,
                            void* stream) {
  if (!m || !host_img || !host_out) return fail(BONSAI_ERR_ARG, "dit_forward_host: null argument");
  const Cfg& c = m->c;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RC(cuda_status(cudaMemcpyAsync(m->in_img, host_img, (size_t)c.img * c.in_ch * 4, cudaMemcpyHostToDevice, st), "img copy"));
  if (c.txt > 0)
    RC(cuda_status(cudaMemcpyAsync(m->in_txt, host_txt, (size_t)c.txt * c.ctx_dim * 4, cudaMemcpyHostToDevice, st), "txt copy"));
  if (c.pooled > 0 && host_pooled)
    RC(cuda_status(cudaMemcpyAsync(m->in_pooled, host_pooled, (size_t)c.pooled * 4, cudaMemcpyHostToDevice, st), "pooled copy"));
  RC(bonsai_dit_forward(m, m->in_img, m->in_txt, c.pooled > 0 ? m->in_pooled : nullptr, timestep,
                        m->out_buf, stream));
  RC(cuda_status(cudaMemcpyAsync(host_out, m->out_buf, (size_t)c.img * c.in_ch * 4, cudaMemcpyDeviceToHost, st), "out copy"));
  return cuda_status(cudaStreamSynchronize(st), "dit_forward_host sync");
}

int bonsai_dit_set_state(bonsai_dit_t m, const float* hidden, const float* vec, void* stream) {
  if (!m || !hidden || !vec) return fail(BONSAI_ERR_ARG, "dit_set_state: null argument");
  const Cfg& c = m->c;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RC(cuda_status(cudaMemcpyAsync(m->hidden, hidden, (size_t)c.L * c.H * 4, cudaMemcpyDefault, st), "hidden copy"));
  RC(cuda_status(cudaMemcpyAsync(m->vec, vec, (size_t)c.H * 4, cudaMemcpyDefault, st), "vec copy"));
  return compute_mods(m, st);
}

int bonsai_dit_get_state(bonsai_dit_t m, float* hidden, void* stream) {
  if (!m || !hidden) return fail(BONSAI_ERR_ARG, "dit_get_state: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RC(cuda_status(cudaMemcpyAsync(hidden, m->hidden, (size_t)m->c.L * m->c.H * 4, cudaMemcpyDefault, st), "hidden copy"));
  return cuda_status(cudaStreamSynchronize(st), "dit_get_state sync");
}

int bonsai_dit_double_block(bonsai_dit_t m, int i, void* stream) {
  if (!m || i < 0 || i >= m->c.depth) return fail(BONSAI_ERR_ARG, "dit_double_block: bad block index");
  return run_double(m, i, static_cast<cudaStream_t>(stream));
}

int bonsai_dit_single_block(bonsai_dit_t m, int i, void* stream) {
  if (!m || i < 0 || i >= m->c.depth_single) return fail(BONSAI_ERR_ARG, "dit_single_block: bad block index");
  return run_single(m, i, static_cast<cudaStream_t>(stream));
}

int bonsai_dit_set_partition(bonsai_dit_t m, int rank, int world) {
  if (!m || world < 1 || rank < 0 || rank >= world)
    return fail(BONSAI_ERR_ARG, "dit_set_partition: need 0 <= rank < world");
  const Cfg& c = m->c;
  if (c.heads % world != 0 || c.L % world != 0)
    return fail(BONSAI_ERR_ARG, "dit_set_partition: heads (" + std::to_string(c.heads) +
                                    ") and tokens (" + std::to_string(c.L) +
                                    ") must both divide by world");
  m->rank = rank;
  m->world = world;
  const int rows = c.L / world;
  m->r0 = rank * rows;
  m->r1 = m->r0 + rows;
  m->hl = c.heads / world;
  m->h0 = rank * m->hl;
  m->fused = false;  // peers belong to a partition: set them again after a change
  m->qkv_scatter = false;
  m->flag_barrier = false;
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  return 0;
}

int bonsai_dit_set_peers(bonsai_dit_t m, void* const* xm, void* const* cat, int world) {
  if (!m) return fail(BONSAI_ERR_ARG, "dit_set_peers: null model");
  if (!xm || !cat) {
    m->fused = false;
    m->qkv_scatter = false;
    return 0;
  }
  if (world != m->world || world < 2 || world > kMaxPeers)
    return fail(BONSAI_ERR_ARG, "dit_set_peers: world must match bonsai_dit_set_partition (2..8)");
  if (xm[m->rank] != m->xm || cat[m->rank] != m->cat)
    return fail(BONSAI_ERR_ARG, "dit_set_peers: entry [rank] must be this model's own xm / cat");
  for (int r = 0; r < world; ++r) {
    if (!xm[r] || !cat[r] || (reinterpret_cast<uintptr_t>(xm[r]) & 15) ||
        (reinterpret_cast<uintptr_t>(cat[r]) & 15))
      return fail(BONSAI_ERR_ARG, "dit_set_peers: null or misaligned buffer");
    m->peer_xm[r] = static_cast<__half*>(xm[r]);
    m->peer_cat[r] = static_cast<__half*>(cat[r]);
  }
  m->fused = true;
  return 0;
}

int bonsai_dit_ipc_handles(bonsai_dit_t m, void* out) {
  if (!m || !out) return fail(BONSAI_ERR_ARG, "dit_ipc_handles: null argument");
  cudaIpcMemHandle_t h[2];
  RC(cuda_status(cudaIpcGetMemHandle(&h[0], m->xm), "dit_ipc_handles: xm"));
  RC(cuda_status(cudaIpcGetMemHandle(&h[1], m->cat), "dit_ipc_handles: cat"));
  std::memcpy(out, h, sizeof(h));
  return 0;
}

int bonsai_dit_open_peers(bonsai_dit_t m, const void* handles, int world) {
  if (!m || !handles) return fail(BONSAI_ERR_ARG, "dit_open_peers: null argument");
  if (world != m->world || world < 2 || world > kMaxPeers)
    return fail(BONSAI_ERR_ARG, "dit_open_peers: world must match bonsai_dit_set_partition (2..8)");
  for (void* p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  m->ipc_opened.clear();
  m->fused = false;
  m->qkv_scatter = false;
  void* xm[kMaxPeers] = {};
  void* cat[kMaxPeers] = {};
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < world; ++r) {
    if (r == m->rank) {
      xm[r] = m->xm;
      cat[r] = m->cat;
      continue;
    }
    for (int b = 0; b < 2; ++b) {
      void* p = nullptr;
      RC(cuda_status(cudaIpcOpenMemHandle(&p, h[2 * r + b], cudaIpcMemLazyEnablePeerAccess),
                     "dit_open_peers: open handle"));
      m->ipc_opened.push_back(p);
      (b == 0 ? xm : cat)[r] = p;
    }
  }
  return bonsai_dit_set_peers(m, xm, cat, world);
}

int bonsai_dit_set_qkv_peers(bonsai_dit_t m, void* const* qkv, int world) {
  if (!m) return fail(BONSAI_ERR_ARG, "dit_set_qkv_peers: null model");
  if (!qkv) {
    m->qkv_scatter = false;
    return 0;
  }
  if (!m->fused)
    return fail(BONSAI_ERR_ARG, "dit_set_qkv_peers: set the xm / cat peers first (bonsai_dit_set_peers)");
  if (world != m->world) return fail(BONSAI_ERR_ARG, "dit_set_qkv_peers: world must match the partition");
  if (qkv[m->rank] != m->qkv)
    return fail(BONSAI_ERR_ARG, "dit_set_qkv_peers: entry [rank] must be this model's own qkv");
  for (int r = 0; r < world; ++r) {
    if (!qkv[r] || (reinterpret_cast<uintptr_t>(qkv[r]) & 15))
      return fail(BONSAI_ERR_ARG, "dit_set_qkv_peers: null or misaligned buffer");
    m->peer_qkv[r] = static_cast<__half*>(qkv[r]);
  }
  m->qkv_scatter = true;
  return 0;
}

int bonsai_dit_ipc_handle(bonsai_dit_t m, const char* name, void* out) {
  if (!m || !name || !out) return fail(BONSAI_ERR_ARG, "dit_ipc_handle: null argument");
  void* ptr = nullptr;
  RC(bonsai_dit_buffer(m, name, &ptr, nullptr));
  cudaIpcMemHandle_t h;
  RC(cuda_status(cudaIpcGetMemHandle(&h, ptr), "dit_ipc_handle"));
  std::memcpy(out, &h, sizeof(h));
  return 0;
}

int bonsai_dit_open_qkv_peers(bonsai_dit_t m, const void* handles, int world) {
  if (!m || !handles) return fail(BONSAI_ERR_ARG, "dit_open_qkv_peers: null argument");
  if (world != m->world || world < 2 || world > kMaxPeers)
    return fail(BONSAI_ERR_ARG, "dit_open_qkv_peers: world must match bonsai_dit_set_partition (2..8)");
  for (void* p : m->ipc_opened_qkv) cudaIpcCloseMemHandle(p);
  m->ipc_opened_qkv.clear();
  m->qkv_scatter = false;
  void* qkv[kMaxPeers] = {};
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < world; ++r) {
    if (r == m->rank) {
      qkv[r] = m->qkv;
      continue;
    }
    void* p = nullptr;
    RC(cuda_status(cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess),
                   "dit_open_qkv_peers: open handle"));
    m->ipc_opened_qkv.push_back(p);
    qkv[r] = p;
  }
  return bonsai_dit_set_qkv_peers(m, qkv, world);
}

int bonsai_dit_set_flag_peers(bonsai_dit_t m, void* const* flags, int world) {
  if (!m) return fail(BONSAI_ERR_ARG, "dit_set_flag_peers: null model");
  if (!flags) {
    m->flag_barrier = false;
    return 0;
  }
  if (world != m->world || world < 2 || world > kMaxPeers)
    return fail(BONSAI_ERR_ARG, "dit_set_flag_peers: world must match bonsai_dit_set_partition (2..8)");
  if (flags[m->rank] != m->flags)
    return fail(BONSAI_ERR_ARG, "dit_set_flag_peers: entry [rank] must be this model's own flags");
  for (int r = 0; r < world; ++r) {
    if (!flags[r] || (reinterpret_cast<uintptr_t>(flags[r]) & 15))
      return fail(BONSAI_ERR_ARG, "dit_set_flag_peers: null or misaligned buffer");
    m->peer_flags[r] = static_cast<unsigned*>(flags[r]);
  }
  // every rank starts counting from zero (the caller orders the ranks after
  // this call, before the first barrier)
  RC(cuda_status(cudaMemset(m->flags, 0, kFlagWords * sizeof(unsigned)), "dit_set_flag_peers: reset"));
  RC(cuda_status(cudaDeviceSynchronize(), "dit_set_flag_peers: reset"));
  m->flag_barrier = true;
  return 0;
}

int bonsai_dit_open_flag_peers(bonsai_dit_t m, const void* handles, int world) {
  if (!m || !handles) return fail(BONSAI_ERR_ARG, "dit_open_flag_peers: null argument");
  if (world != m->world || world < 2 || world > kMaxPeers)
    return fail(BONSAI_ERR_ARG, "dit_open_flag_peers: world must match bonsai_dit_set_partition (2..8)");
  for (void* p : m->ipc_opened_flags) cudaIpcCloseMemHandle(p);
  m->ipc_opened_flags.clear();
  m->flag_barrier = false;
  void* flags[kMaxPeers] = {};
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < world; ++r) {
    if (r == m->rank) {
      flags[r] = m->flags;
      continue;
    }
    void* p = nullptr;
    RC(cuda_status(cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess),
                   "dit_open_flag_peers: open handle"));
    m->ipc_opened_flags.push_back(p);
    flags[r] = p;
  }
  return bonsai_dit_set_flag_peers(m, flags, world);
}

int bonsai_dit_barrier(bonsai_dit_t m, void* stream) {
  if (!m) return fail(BONSAI_ERR_ARG, "dit_barrier: null model");
  if (!m->flag_barrier) return fail(BONSAI_ERR_ARG, "dit_barrier: set the flag peers first");
  FlagPeers fp{};
  for (int r = 0; r < m->world; ++r) fp.f[r] = m->peer_flags[r];
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fp, m->flags, m->rank,
                                                                       m->world, device_error_word());
  return launch_status("peer_barrier_kernel launch");
}

int bonsai_dit_buffer(bonsai_dit_t m, const char* name, void** ptr, long long* bytes) {
  if (!m || !name || !ptr) return fail(BONSAI_ERR_ARG, "dit_buffer: null argument");
  const Cfg& c = m->c;
  const std::string n = name;
  long long b = 0;
  if (n == "hidden") { *ptr = m->hidden; b = (long long)c.L * c.H * 4; }
  else if (n == "xm") { *ptr = m->xm; b = (long long)c.L * c.H * 2; }
  else if (n == "cat") { *ptr = m->cat; b = (long long)c.L * c.C() * 2; }
  else if (n == "qkv") { *ptr = m->qkv; b = 3LL * c.heads * c.L * c.hd * 2; }
  else if (n == "flags") { *ptr = m->flags; b = kFlagWords * (long long)sizeof(unsigned); }
  else return fail(BONSAI_ERR_ARG, "dit_buffer: unknown buffer " + n);
  if (bytes) *bytes = b;
  return 0;
}

int bonsai_dit_begin(bonsai_dit_t m, const float* img, const float* txt, const float* pooled,
                     float timestep, void* stream) {
  if (!m || !img || (m->c.txt > 0 && !txt)) return fail(BONSAI_ERR_ARG, "dit_begin: null argument");
  if (m->c.pooled > 0 && !pooled) return fail(BONSAI_ERR_ARG, "dit_begin: the Flux.1 preset needs the pooled vector");
  const Cfg& c = m->c;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RC(dit_upload_timestep(m, timestep, st));
  // input projections of this rank's rows (:283-286)
  const Span tx = own_txt(m), im = own_img(m);
  RC(edge_linear(m, txt + (size_t)tx.a * c.ctx_dim, c.ctx_dim, tx.n(), c.ctx_dim, m->txt_in_w,
                 m->txt_in_w3, m->txt_in_b, c.H, m->hidden + (size_t)tx.a * c.H, c.H, st, m->tmp32,
                 (long long)c.img * c.H));
  RC(edge_linear(m, img + (size_t)(im.a - c.txt) * c.in_ch, c.in_ch, im.n(), c.in_ch, m->img_in_w,
                 m->img_in_w3, m->img_in_b, c.H, m->hidden + (size_t)im.a * c.H, c.H, st, nullptr,
                 0));
  return dit_prepare_vec(m, pooled, st);
}

int bonsai_dit_phase(bonsai_dit_t m, int kind, int block, int phase, void* stream) {
  if (!m || phase < 0 || phase > 2) return fail(BONSAI_ERR_ARG, "dit_phase: bad phase");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (kind == 0) {
    if (block < 0 || block >= m->c.depth) return fail(BONSAI_ERR_ARG, "dit_phase: bad double block");
    return double_phase(m, block, phase, st);
  }
  if (kind == 1) {
    if (block < 0 || block >= m->c.depth_single) return fail(BONSAI_ERR_ARG, "dit_phase: bad single block");
    return single_phase(m, block, phase, st);
  }
  return fail(BONSAI_ERR_ARG, "dit_phase: kind must be 0 (double) or 1 (single)");
}

int bonsai_dit_end(bonsai_dit_t m, float* out, void* stream) {
  if (!m || !out) return fail(BONSAI_ERR_ARG, "dit_end: null argument");
  const Cfg& c = m->c;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // output head (:544-556) on every image row (the caller has gathered them)
  const float* h_img = m->hidden + (size_t)c.txt * c.H;
  RC(launch_ln_modulate_f32(h_img, c.img, c.H, m->fin + c.H, m->fin, 1e-6f, m->tmp32, c.H, st));
  // (f32 fallback: cat, free by now, holds the split-K partial sums)
  return edge_linear(m, m->tmp32, c.H, c.img, c.H, m->proj_out_w, m->proj_out_w3, m->proj_out_b,
                     c.in_ch, out, c.in_ch, st, reinterpret_cast<float*>(m->cat),
                     (long long)c.L * c.C() / 2);
}

long long bonsai_dit_weight(bonsai_dit_t m, const char* name, void* buf, long long cap) {
  if (!m || !name) return fail(BONSAI_ERR_ARG, "dit_weight: null argument");
  auto it = m->reg.find(name);
  if (it == m->reg.end()) return fail(BONSAI_ERR_ARG, std::string("dit_weight: unknown tensor ") + name);
  const TensorInfo& ti = it->second;
  const long long bytes = tensor_bytes(ti);
  if (!buf) return bytes;
  if (cap < bytes) return fail(BONSAI_ERR_ARG, "dit_weight: buffer too small");
  RC(cuda_status(cudaDeviceSynchronize(), "dit_weight: synchronize"));
  if (ti.kind == KIND_F32)
    return cuda_status(cudaMemcpy(buf, ti.f32, bytes, cudaMemcpyDeviceToHost), "dit_weight copy") ? BONSAI_ERR_CUDA : bytes;
  // B1_0: the device copy, turned back into the packed file layout.
  void* tmp = nullptr;
  if (cudaMalloc(&tmp, bytes) != cudaSuccess) return fail(BONSAI_ERR_NOMEM, "dit_weight: staging allocation failed");
  int rc = launch_b1_unretile(b1_view(ti), static_cast<uint8_t*>(tmp), 0);
  if (!rc) rc = cuda_status(cudaMemcpy(buf, tmp, bytes, cudaMemcpyDeviceToHost), "dit_weight copy");
  cudaFree(tmp);
  return rc ? rc : bytes;
}

int bonsai_dit_set_weight(bonsai_dit_t m, const char* name, const void* host, long long bytes) {
  if (!m || !name || !host) return fail(BONSAI_ERR_ARG, "dit_set_weight: null argument");
  auto it = m->reg.find(name);
  if (it == m->reg.end())
    return fail(BONSAI_ERR_ARG, std::string("dit_set_weight: unknown tensor ") + name);
  const TensorInfo& ti = it->second;
  if (bytes != tensor_bytes(ti))
    return fail(BONSAI_ERR_ARG, std::string("dit_set_weight: ") + name + " takes " +
                                    std::to_string(tensor_bytes(ti)) + " bytes, got " +
                                    std::to_string(bytes));
  // No forward of this model may be running while its weights change.
  RC(cuda_status(cudaDeviceSynchronize(), "dit_set_weight: synchronize"));
  if (ti.kind == KIND_F32) {
    RC(cuda_status(cudaMemcpy(ti.f32, host, bytes, cudaMemcpyHostToDevice), "dit_set_weight copy"));
    RC(refresh_edge_w3(m, name, 0));
    return cuda_status(cudaDeviceSynchronize(), "dit_set_weight: edge split");
  }
  void* tmp = nullptr;
  if (cudaMalloc(&tmp, bytes) != cudaSuccess) return fail(BONSAI_ERR_NOMEM, "dit_set_weight: staging allocation failed");
  int rc = cuda_status(cudaMemcpy(tmp, host, bytes, cudaMemcpyHostToDevice), "dit_set_weight copy");
  B1Weight v = b1_view(ti);
  if (!rc) rc = launch_b1_retile(static_cast<const uint8_t*>(tmp), v, 0);
  if (!rc) rc = cuda_status(cudaDeviceSynchronize(), "dit_set_weight: retile");
  cudaFree(tmp);
  return rc;
}

int bonsai_dit_load_safetensors(bonsai_dit_t m, const char* path) {
  if (!m || !path) return fail(BONSAI_ERR_ARG, "dit_load_safetensors: null argument");
  if (m->c.preset != BONSAI_PRESET_KLEIN4B)
    return fail(BONSAI_ERR_UNSUPPORTED,
                "dit_load_safetensors: the reference's checkpoint layout (src/diffuser.cpp:88-186) "
                "exists for the klein4b preset only");
  StFile f;
  RC(st_open(path, f));
  // Our tensor <- the reference's tensors, stacked by rows in this order.
  std::vector<std::pair<std::string, std::vector<std::string>>> map = {
      {"img_in.w", {"x_embedder.weight"}},
      {"txt_in.w", {"context_embedder.weight"}},
      {"time.w1", {"time_guidance_embed.timestep_embedder.linear_1.weight"}},
      {"time.w2", {"time_guidance_embed.timestep_embedder.linear_2.weight"}},
      {"mod_img.w", {"double_stream_modulation_img.linear.weight"}},
      {"mod_txt.w", {"double_stream_modulation_txt.linear.weight"}},
      {"mod_single.w", {"single_stream_modulation.linear.weight"}},
      {"norm_out.w", {"norm_out.linear.weight"}},
      {"proj_out.w", {"proj_out.weight"}},
  };
  for (int d = 0; d < m->c.depth; ++d) {
    const std::string o = "double." + std::to_string(d) + ".";
    const std::string r = "transformer_blocks." + std::to_string(d) + ".";
    map.push_back({o + "img_qkv", {r + "attn.to_q.weight", r + "attn.to_k.weight", r + "attn.to_v.weight"}});
    map.push_back({o + "txt_qkv", {r + "attn.add_q_proj.weight", r + "attn.add_k_proj.weight",
                                   r + "attn.add_v_proj.weight"}});
    map.push_back({o + "img_out", {r + "attn.to_out.0.weight"}});
    map.push_back({o + "txt_out", {r + "attn.to_add_out.weight"}});
    map.push_back({o + "img_norm_q", {r + "attn.norm_q.weight"}});
    map.push_back({o + "img_norm_k", {r + "attn.norm_k.weight"}});
    map.push_back({o + "txt_norm_q", {r + "attn.norm_added_q.weight"}});
    map.push_back({o + "txt_norm_k", {r + "attn.norm_added_k.weight"}});
    map.push_back({o + "img_mlp_in", {r + "ff.linear_in.weight"}});
    map.push_back({o + "img_mlp_out", {r + "ff.linear_out.weight"}});
    map.push_back({o + "txt_mlp_in", {r + "ff_context.linear_in.weight"}});
    map.push_back({o + "txt_mlp_out", {r + "ff_context.linear_out.weight"}});
  }
  for (int s = 0; s < m->c.depth_single; ++s) {
    const std::string o = "single." + std::to_string(s) + ".";
    const std::string r = "single_transformer_blocks." + std::to_string(s) + ".attn.";
    map.push_back({o + "proj", {r + "to_qkv_mlp_proj.weight"}});
    map.push_back({o + "out", {r + "to_out.weight"}});
    map.push_back({o + "norm_q", {r + "norm_q.weight"}});
    map.push_back({o + "norm_k", {r + "norm_k.weight"}});
  }
  std::vector<uint8_t> buf;
  for (const auto& e : map) {
    auto it = m->reg.find(e.first);
    if (it == m->reg.end()) return fail(BONSAI_ERR_ARG, "dit_load_safetensors: model lacks " + e.first);
    const TensorInfo& ti = it->second;
    const long long want = tensor_bytes(ti);
    buf.resize((size_t)want);
    long long off = 0, rows = 0;
    for (const std::string& src : e.second) {
      auto ts = f.tensors.find(src);
      if (ts == f.tensors.end())
        return fail(BONSAI_ERR_ARG, "dit_load_safetensors: tensor '" + src + "' not found in " + path);
      const StTensor& t = ts->second;
      const long long n = t.end - t.begin;
      if (ti.kind == KIND_B1) {
        // packed [out][in/32*6] bytes (convert_to_b1_0_packed.py:21-43)
        if ((t.dtype != "U8" && t.dtype != "I8") || t.shape.size() != 2 ||
            t.shape[1] != (ti.cols / 32) * 6 || n != t.shape[0] * t.shape[1])
          return fail(BONSAI_ERR_ARG, "dit_load_safetensors: '" + src + "' is not a packed B1_0 [" +
                                          "rows][" + std::to_string((ti.cols / 32) * 6) + "] U8 tensor");
        rows += t.shape[0];
      } else if (t.dtype != "F32") {
        return fail(BONSAI_ERR_ARG, "dit_load_safetensors: '" + src + "' must be F32, found " + t.dtype);
      }
      if (off + n > want)
        return fail(BONSAI_ERR_ARG, "dit_load_safetensors: '" + src + "' is larger than " + e.first);
      RC(st_read(f, t, buf.data() + off, n));
      off += n;
    }
    if (off != want || (ti.kind == KIND_B1 && rows != ti.rows))
      return fail(BONSAI_ERR_ARG, "dit_load_safetensors: the tensors for " + e.first + " hold " +
                                      std::to_string(off) + " bytes, the model needs " +
                                      std::to_string(want));
    RC(bonsai_dit_set_weight(m, e.first.c_str(), buf.data(), want));
  }
  return 0;
}

int bonsai_dit_sample(bonsai_dit_t m, float* latents, const float* txt, const float* pooled,
                      int n_steps, float* stats, void* stream) {
  if (!m || !latents || n_steps < 1) return fail(BONSAI_ERR_ARG, "dit_sample: bad argument");
  if (m->world > 1)
    return fail(BONSAI_ERR_ARG, "dit_sample: a partitioned model is driven with bonsai_dit_begin/phase/end");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n = (long long)m->c.img * m->c.in_ch;
  float* dstats = nullptr;
  RC(cuda_status(cudaMallocAsync(reinterpret_cast<void**>(&dstats), (size_t)n_steps * 5 * 4, st),
                 "dit_sample: stats allocation"));
  int rc = 0;
  // Timesteps and step sizes exactly as the reference's loop computes them
  // (src/diffuser.cpp:251-255, :258-259), in float.
  for (int step = 0; step < n_steps && !rc; ++step) {
    const float t = 1.0f - (float)step / n_steps;
    const float t_next = 1.0f - (float)(step + 1) / n_steps;
    const float dt = (step < n_steps - 1) ? t - t_next : t;
    rc = bonsai_dit_forward(m, latents, txt, pooled, t * 1000.0f, m->out_buf, stream);
    if (!rc) rc = launch_euler_stats(latents, m->out_buf, n, dt, dstats + 5LL * step, st);
  }
  if (!rc && stats)
    rc = cuda_status(cudaMemcpyAsync(stats, dstats, (size_t)n_steps * 5 * 4, cudaMemcpyDeviceToHost, st),
                     "dit_sample: stats copy");
  cudaFreeAsync(dstats, st);
  if (!rc && stats) rc = cuda_status(cudaStreamSynchronize(st), "dit_sample: synchronize");
  return rc;
}

}  // extern "C"
