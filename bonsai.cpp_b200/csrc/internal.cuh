// Internal declarations shared by the kernel translation units and the
// host-side engine.  Nothing here is part of the public C ABI
// (include/bonsai_cuda.h).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace bonsai {

// ------------------------------------------------------------------ status
void set_error(const std::string& msg);  // stores the message for bonsai_last_error()
int fail(int code, const std::string& msg);  // set_error + return code
int cuda_status(cudaError_t e, const char* what);  // 0 or BONSAI_ERR_CUDA
int launch_status(const char* what);  // checks cudaGetLastError() and counts the launch
// RAII per-launch timer used by bonsai_profile_start/stop: records a CUDA
// event before and after the launch on its stream when profiling is on.
class ProfScope {
 public:
  ProfScope(const char* kind, double flop, double bytes, cudaStream_t st);
  ~ProfScope();
 private:
  cudaStream_t st_;
  long long idx_ = -1;
};
int* device_error_word();
long long launch_counter();           // launches counted on this thread so far
void launch_counter_add(long long n);  // account for kernels replayed from a CUDA graph
bool profiling_active();              // bonsai_profile_start() in effect on this thread  // device address of the per-device error word (lazily resolved)
int num_sms();
// Index (0..63) of the current CUDA device: per-device caches of launch set-up
// (shared-memory attributes, cluster occupancy) are kept per device, since a
// process may drive several GPUs.
int device_slot();

// ------------------------------------------------------- B1_0 device weights
// Device layout ("chunked"): the packed reference layout [N][K/32][6 bytes]
// is retiled on upload into chunks of 128 output rows x 64 inputs.  Chunk
// (ftile, kb) holds three arrays of 128 u32: the sign word of group 2kb, the
// sign word of group 2kb+1 (both in "pair-split" bit order: bit j = input
// 2j, bit j+16 = input 2j+1), and both fp16 scales packed (lo = group 2kb).
// Rows beyond N and groups beyond K/32 are zero (scale 0).  The size is the
// same 6 bytes per 32 weights as the packed file (plus tile padding).
struct B1Weight {
  int n_rows = 0;      // output features N
  int k_in = 0;        // input features K
  int n_ftiles = 0;    // ceil(N / 128)
  int k_blocks = 0;    // ceil(K / 64)
  int swiglu_from = -1;  // rows [swiglu_from, N) are stored gate/value interleaved
  uint32_t* chunks = nullptr;  // n_ftiles * k_blocks * 384 words
  int device = 0;
};

constexpr int kChunkWords = 384;  // 3 x 128 u32 per (128-row, 64-input) chunk

// ------------------------------------------------------------- epilogues
enum EpiMode : int {
  EPI_F32 = 0,         // dst f32 [t][ld] at col_off + (row - row_begin)
  EPI_F16 = 1,         // dst f16
  EPI_GELU_F16 = 2,    // dst f16 = gelu_tanh(acc)
  EPI_RESID_F32 = 3,   // dst f32 += gate[row - row_begin] * acc  (gate may be null -> 1)
  EPI_QKV_F16 = 4,     // head-major scatter: dst[(which*heads + h)*seq_total + tok_off + t][d]
  EPI_SWIGLU_F16 = 5,  // interleaved gate/value rows -> dst f16 silu(g)*v at col_off + (row-row_begin)/2
};

constexpr int kMaxPeers = 8;

struct EpiSeg {
  int mode = EPI_F32;
  int row_begin = 0, row_end = 0;
  void* dst = nullptr;
  long long ld = 0;   // elements
  int col_off = 0;
  const float* gate = nullptr;
  int heads = 0, seq_total = 0, tok_off = 0, head_dim = 128;
  // EPI_QKV_F16 only: with route_heads > 0, head h is stored through
  // route[h / route_heads] (at the same offsets) instead of dst -- each rank's
  // q/k/v buffer of a head split, peer-mapped -- and the kernel ends with a
  // system-scope fence after its stores.
  __half* route[kMaxPeers] = {};
  int route_heads = 0;
  // EPI_RESID_F32 only: the launcher may split K between two CTA pairs whose
  // epilogues both add into dst (f32 atomic adds, in no fixed order: the sum
  // can differ in the last bit from run to run).
  int split_ok = 0;
};

constexpr int kMaxSegs = 2;
constexpr int kMaxTileGroups = 3;

// Optional selection of 128-row weight tiles for a GEMM launch: the tiles
// base[g] + i for g < groups, i < count (e.g. one rank's heads of the q, k
// and v parts of a fused QKV weight).  Null = every tile.
struct TileSel {
  int groups = 1;
  int count = 0;
  int base[kMaxTileGroups] = {0, 0, 0};
};

// Launch the tcgen05 B1_0 GEMM: for every token t < tokens and weight row n,
// acc[t][n] = sum_k x[t][k] * W[n][k]; acc is routed through the segment that
// covers n.  x is f16 (or bf16 when x_bf16) row-major with leading dimension
// ldx (elements); it must be 16-byte aligned with ldx % 8 == 0.
int launch_b1_gemm(const void* x, long long ldx, int tokens, const B1Weight& w,
                   const EpiSeg* segs, int nseg, bool x_bf16, cudaStream_t st,
                   const TileSel* sel = nullptr);

// B1_0 matrix-vector product for one f32 activation row: y[n] = sum_k
// W[n][k] x[k] (f32 x and accumulation), memory-bound, no tensor cores.
// Supported for in_dim <= 8192 and weights without the SwiGLU interleave.
bool b1_gemv_supported(const B1Weight& w);
int launch_b1_gemv_f32(const float* x, const B1Weight& w, float* y, cudaStream_t st);

// Retile packed reference bytes (device copy) into the chunked layout.
int launch_b1_retile(const uint8_t* dev_packed, B1Weight& w, cudaStream_t st);
// Inverse of launch_b1_retile: device chunks of w back to the packed
// [n_rows][k_in/32][6] bytes (dev_packed, device memory).
int launch_b1_unretile(const B1Weight& w, uint8_t* dev_packed, cudaStream_t st);

// ------------------------------------------------------------ safetensors
// Index of a .safetensors file: 8-byte little-endian header length, JSON
// header {name: {"dtype", "shape", "data_offsets": [begin, end]}}, then the
// tensor bytes (offsets relative to the end of the header).
struct StTensor {
  std::string dtype;
  std::vector<long long> shape;
  long long begin = 0, end = 0;
};
struct StFile {
  FILE* f = nullptr;
  long long data_start = 0, file_size = 0;
  std::map<std::string, StTensor> tensors;
  ~StFile();
};
int st_open(const char* path, StFile& out);                     // 0 or a BONSAI_ERR_* code
int st_read(StFile& f, const StTensor& t, void* dst, long long bytes);

// Peer copies of an f16 output: the same rows are also stored, at the same
// offsets, into copies[0..n) (other GPUs' buffers reached through peer
// mappings, or other buffers of this GPU).  The kernel ends with a
// system-scope fence after its stores.
struct PeerCopies {
  __half* y[kMaxPeers - 1] = {};
  int n = 0;
};

// ------------------------------------------------------------- attention
// q, k, v: f16 [n_heads][seq][128]; out: f16 [seq][ld_out], head h at columns h*128.
// routes (optional): query row t is stored through outs[r] for the r with
// row_bound[r] <= t < row_bound[r + 1] instead of out (each rank's buffer
// of a head/row split, peer-mapped); the kernel then ends with a
// system-scope fence after its stores.
struct RowRoutes {
  __half* outs[kMaxPeers] = {};
  int row_bound[kMaxPeers + 1] = {};
  int n = 0;
};
int launch_attention(const __half* q, const __half* k, const __half* v, int n_heads, int seq,
                     int head_dim, float scale, __half* out, long long ld_out, cudaStream_t st,
                     const RowRoutes* routes = nullptr);

// ------------------------------------------------------------ pointwise
int launch_f32_to_f16(const float* src, __half* dst, long long n, cudaStream_t st);
int launch_ln_modulate_f16(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, __half* y, long long ld_y,
                           cudaStream_t st);
int launch_ln_modulate_f16_peers(const float* x, int rows, int dim, const float* shift,
                                 const float* scale, float eps, __half* y, long long ld_y,
                                 const PeerCopies& copies, cudaStream_t st);
int launch_ln_modulate_f32(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, float* y, long long ld_y,
                           cudaStream_t st);
// q and k head-major [n_heads][seq][128] f16, in place (k may be null).
int launch_qk_norm_rope(__half* q, __half* k, int n_heads, int seq, const float* wq_lo,
                        const float* wq_hi, const float* wk_lo, const float* wk_hi, int split,
                        float eps, const float* cos_t, const float* sin_t, cudaStream_t st);
int launch_rope_2d_f32(const float* x, const float* c, const float* s, int head_dim, int n_heads,
                       int seq, float* out, cudaStream_t st);
int launch_rms_norm_f32(const float* x, const float* w, int rows, int dim, float eps, float* y,
                        cudaStream_t st);
int launch_rope_tables(const float* ids, int seq, int n_axes, const int* pair_axis_dev,
                       const float* pair_freq_dev, int half, float* cos_out, float* sin_out,
                       cudaStream_t st);
// Host-side pair -> (axis, frequency) map of compute_rope_freqs_data
// (src/diffuser_graph.cpp:126-140) with the axes concatenated in order.
void rope_pair_table(const int* axes_dim, int n_axes, float theta, int* pair_axis,
                     float* pair_freq);

// ------------------------------------------------------------ edge ops
// workspace (optional): f32 scratch for split-K partial sums of large-K, few-tile shapes.
int launch_linear_f32(const float* x, long long ldx, int T, int K, const float* W, const float* b,
                      int N, float* y, long long ldy, bool silu_in, cudaStream_t st,
                      float* workspace = nullptr, long long workspace_elems = 0);
// f32 linear on the tensor cores as bf16x3: x = x_hi + x_lo and
// W = W_hi + W_lo in bf16, y = x_hi W_hi + x_hi W_lo + x_lo W_hi (+ bias)
// with f32 accumulation (every bf16 product is exact in f32; the dropped
// x_lo W_lo term is ~2^-16 relative).  w3 = the weight [N][K] split once by
// launch_split_bf16x3(weights = true) into [N][3K]; a3: scratch [M][3K].
// K % 8 == 0, x rows 16-byte aligned.  One split kernel + one GEMM launch.
int launch_split_bf16x3(const float* x, long long ldx, int M, int K, bool weights,
                        __nv_bfloat16* out, cudaStream_t st);
int launch_linear_bf16x3(const float* x, long long ldx, int M, int K, const __nv_bfloat16* w3,
                         const float* bias, int N, float* y, long long ldy, __nv_bfloat16* a3,
                         cudaStream_t st);
int launch_silu_f32(const float* x, long long n, float* y, cudaStream_t st);
int launch_add_f32(const float* a, const float* b, long long n, float* y, cudaStream_t st);
// *dev_count += number of NaN / Inf values in x[0, n).
int launch_count_nonfinite(const float* x, long long n, unsigned long long* dev_count,
                           cudaStream_t st);
// lat += dt * pred and stats[0..4] = {NaN count, Inf count, min, max, mean} of pred.
int launch_euler_stats(float* lat, const float* pred, long long n, float dt, float* stats,
                       cudaStream_t st);

}  // namespace bonsai

// Opaque handle behind bonsai_b1_t (include/bonsai_cuda.h).
struct bonsai_b1_weight {
  bonsai::B1Weight w;
};
