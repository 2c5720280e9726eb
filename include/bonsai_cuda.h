/*
 * bonsai_cuda.h - C ABI of the B200 (sm_100a) diffuser-transformer engine.
 *
 * Drop-in boundary for bonsai.cpp's diffuser step.  The reference builds a
 * ggml graph whose custom ops are recognised by a magic number in their
 * user data (src/b1_0_kernel.h:32 "1B1B" b1_linear, src/b1_0_kernel.h:303
 * "ROPE" rope_2d_fwd) next to built-in ggml ops (norm, rms_norm,
 * flash_attn_ext, swiglu) called from build_diffuser_graph
 * (src/diffuser_graph.cpp:231-561).  Every entry point here replaces one of
 * those ops, one block, or the whole step, with the same tensors.
 *
 * Conventions
 *   - All tensor arguments are DEVICE pointers unless the name says host_.
 *   - Row-major; "[a][b]" means a rows of b contiguous elements.  A ggml
 *     tensor with ne = {b, a} has exactly this layout.
 *   - f16 = IEEE binary16 stored as uint16_t.  Activations that feed the
 *     tensor cores are f16; the residual stream and drop-in outputs are f32.
 *   - stream is a cudaStream_t passed as void* (NULL = legacy stream).
 *     Calls are asynchronous and stream-ordered; none synchronises the host.
 *   - Every function returns 0 on success or a negative BONSAI_ERR_* code;
 *     bonsai_last_error() describes the most recent failure of the calling
 *     thread.  Nothing aborts the process (the reference aborts on NaN /
 *     missing weights: src/b1_0_kernel.h:195-198, src/diffuser.cpp:52-56).
 */
#ifndef BONSAI_CUDA_H
#define BONSAI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BONSAI_OK 0
#define BONSAI_ERR_ARG (-1)         /* bad argument / shape */
#define BONSAI_ERR_UNSUPPORTED (-2) /* shape or mode not supported */
#define BONSAI_ERR_CUDA (-3)        /* CUDA runtime error */
#define BONSAI_ERR_DEVICE (-4)      /* a kernel reported a device-side error (bounded wait expired) */
#define BONSAI_ERR_DRIVER (-5)      /* driver entry point (tensor-map encoder) unavailable */
#define BONSAI_ERR_NOMEM (-6)       /* device allocation failed */

/* Magic numbers of the reference's custom-op user data; a ggml backend that
 * routes nodes to this library matches on them (src/b1_0_kernel.h:32, :303). */
#define BONSAI_B1_MAGIC 0x31423142
#define BONSAI_ROPE_MAGIC 0x524F5045

/* B1_0 block format: 32 weights per 6-byte block = fp16 scale (LE) + u32
 * sign bits (LE, bit i -> input 32*blk+i, 1 = +scale, 0 = -scale).
 * src/diffuser_types.h:10-11, convert_to_b1_0_packed.py:21-43. */
#define BONSAI_B1_BLOCK_SIZE 32
#define BONSAI_B1_BLOCK_BYTES 6

/* ------------------------------------------------------------- runtime */

/* Message for the most recent failure on the calling thread ("" if none). */
const char* bonsai_last_error(void);

/* Select the CUDA device used by later calls from this thread and check it
 * is an sm_100 part.  Replaces ggml_backend_cpu_init()
 * (src/diffuser.cpp:214). */
int bonsai_init(int device);

/* Read and clear the device-side error word of the current device: 0, or the
 * code of the first bounded wait that expired since the last call.
 * Synchronises the device. */
int bonsai_device_error(void);

/* Wait for the current device and release what the library allocated
 * lazily for the calling thread on it (bonsai_b1_linear_f32's activation
 * scratch, pending profiling events).  Weight handles and models stay valid.
 * The counterpart of ggml_backend_free (src/diffuser.cpp:310). */
int bonsai_shutdown(void);

/* *count = number of NaN / Inf values in the device array x[0, n);
 * synchronises the stream.  Replaces the reference's NaN/Inf abort() checks
 * (src/b1_0_kernel.h:45-69, :195-198) with a value the caller can test. */
int bonsai_count_nonfinite(const float* x, long long n, long long* count, void* stream);

/* Testing hook for the bounded waits that replace the reference's abort()
 * (src/b1_0_kernel.h:193-198): the next B1_0 GEMM launched by the calling
 * thread runs the one-CTA kernel with its load warp idle, so every other role
 * waits on a barrier that nothing completes.  Each wait gives up after its
 * 2 s limit, the kernel records a DEV_ERR_TIMEOUT_* code in the device error
 * word and returns through its abort path (nothing is in flight: no copy was
 * issued and no MMA started), leaving the context usable.  Read (and clear)
 * the code with bonsai_device_error().  The launch's output is not written. */
int bonsai_debug_stall_next_gemm(void);

/* Number of kernel launches this library has issued on the current thread
 * since the last call (launch accounting for benchmarks); resets to 0. */
long long bonsai_launch_count(void);

/* Per-kernel timing for benchmarks and tracing: between start and stop,
 * every launch of the library is bracketed by two CUDA events recorded on
 * its own stream.  stop synchronises the device and writes a JSON object
 * {kernel: {"launches", "ms", "flop", "bytes"}} (algorithmic work) into
 * json (truncated to cap); it returns the full length.  Per thread. */
int bonsai_profile_start(void);
int bonsai_profile_stop(char* json, int cap);

/* ------------------------------------------------------ B1_0 weights */

typedef struct bonsai_b1_weight* bonsai_b1_t;

/* Upload one packed B1_0 matrix exactly as written by
 * convert_to_b1_0_packed.py and loaded by load_b1 (src/diffuser.cpp:39-50):
 * host_packed = [out_dim][in_dim/32][6] bytes.  The device copy is retiled
 * (same 6 bytes per 32 weights); the on-disk layout is unchanged.
 * swiglu_from: -1, or the first row of a trailing [gate; value] pair of
 * halves that should be stored interleaved so the SwiGLU epilogue can fuse
 * (rows [swiglu_from, out_dim) must split into two equal halves).
 * in_dim % 32 == 0 is required (src/diffuser.cpp:43). */
int bonsai_b1_upload(const uint8_t* host_packed, int out_dim, int in_dim, int swiglu_from,
                     bonsai_b1_t* out);
int bonsai_b1_free(bonsai_b1_t w);
int bonsai_b1_shape(bonsai_b1_t w, int* out_dim, int* in_dim);

/* Drop-in for b1_linear_f32_f32 (src/b1_0_kernel.h:37-288) as invoked by
 * b1_linear() (src/b1_0_kernel.h:290-300):
 *   out[t][r] = sum_blk scale[r][blk] * sum_i (bit ? +act : -act)
 * act: f32 [tokens][in_dim]; out: f32 [tokens][out_dim].
 * The activations are rounded to f16 for the tensor cores (f32
 * accumulation); a single token (tokens == 1, in_dim <= 8192) instead runs
 * a memory-bound matrix-vector kernel on the f32 activations, with no
 * scratch.  The f16 copy of act lives in a scratch buffer the library
 * keeps per (calling thread, device, stream), grown on demand with
 * cudaMallocAsync on that stream and released by bonsai_shutdown: calls on
 * different streams never share a buffer, so they may overlap on the GPU.
 * The weight must live on the current device (BONSAI_ERR_ARG otherwise). */
int bonsai_b1_linear_f32(const float* act, int tokens, bonsai_b1_t w, float* out, void* stream);

/* Same operation as bonsai_b1_linear_f32, for callers that cannot let the
 * library allocate device memory (no counterpart in the reference).  Hosts
 * that own every device byte through their own allocator (a ggml graph
 * allocator) or loops that must not block on an allocation use this form:
 * it calls no cudaMalloc/cudaFree or allocating library routine.  The f16
 * copy of act lives in one fixed 8 MiB device array inside the library
 * (tokens * in_dim <= 4,194,304 elements; larger calls return
 * BONSAI_ERR_UNSUPPORTED), which every GPU that loads the library keeps until
 * the process exits.  The first call on a device looks up that array's device
 * address (cudaGetSymbolAddress) with the device current: make that first
 * call before any stream capture.  All calls share the one array, so calls
 * that may overlap on the GPU (different streams, or different host threads
 * on one device) race: serialise them.  A single token (tokens == 1,
 * in_dim <= 8192) runs the same f32 matrix-vector kernel as
 * bonsai_b1_linear_f32 and does not touch the array.  The weight must live
 * on the current device (BONSAI_ERR_ARG otherwise). */
int bonsai_b1_linear_f32_noalloc(const float* act, int tokens, bonsai_b1_t w, float* out,
                                 void* stream);

/* Fused-epilogue B1_0 GEMM on f16 activations (the form the engine uses).
 * x: f16 [tokens][ldx] (16-byte aligned, ldx % 8 == 0).  The accumulator
 * acc[t][r] is written according to mode:
 *   BONSAI_EPI_F32    out f32  [t][ld_out] at column r
 *   BONSAI_EPI_F16    out f16  [t][ld_out] at column r
 *   BONSAI_EPI_GELU   out f16  = gelu_tanh(acc)
 *   BONSAI_EPI_RESID  out f32 += gate[r] * acc   (gate may be NULL = 1)
 *                      (adaLN gate-residual, src/diffuser_graph.cpp:439-460, :538)
 *   BONSAI_EPI_SWIGLU out f16 [t][ld_out] at column r/2 = silu(g)*v for a
 *                      weight uploaded with swiglu_from = 0
 *                      (ggml_swiglu, src/diffuser_graph.cpp:227-229)
 */
#define BONSAI_EPI_F32 0
#define BONSAI_EPI_F16 1
#define BONSAI_EPI_GELU 2
#define BONSAI_EPI_RESID 3
#define BONSAI_EPI_SWIGLU 5
int bonsai_b1_gemm(const uint16_t* x, long long ldx, int tokens, bonsai_b1_t w, int mode,
                   void* out, long long ld_out, const float* gate, void* stream);

/* ------------------------------------------------------ pointwise ops */

/* Drop-in for rope_2d_fwd_f32 (src/b1_0_kernel.h:309-361): for every
 * (s, h, d) pair, (a, b) = (x[s][h][2d], x[s][h][2d+1]) ->
 * (a*c - b*s, a*s + b*c) with c = cos_t[s][d], s = sin_t[s][d].
 * x, out: f32 [seq][n_heads][head_dim]; cos_t, sin_t: f32 [seq][head_dim/2].
 * out may equal x. */
int bonsai_rope_2d_f32(const float* x, const float* cos_t, const float* sin_t, int head_dim,
                       int n_heads, int seq, float* out, void* stream);

/* RoPE angle tables of build_rope_cos_sin (src/diffuser_graph.cpp:126-182):
 * freq[a][j] = 1 / theta^(2j/axes_dim[a]); pair d of the head belongs to the
 * axis whose half-range contains it (axes concatenated in order);
 * angle[s][d] = ids[s][a] * freq[a][j].  ids: f32 [seq][n_axes] (device);
 * cos_out / sin_out: f32 [seq][sum(axes_dim)/2]. */
int bonsai_rope_tables(const float* ids, int seq, int n_axes, const int* host_axes_dim,
                       float theta, float* cos_out, float* sin_out, void* stream);

/* f32 linear y[t][o] = sum_k x[t][k] * W[o][k] (+ bias[o]), the ggml_mul_mat
 * of the reference's f32 edge projections (x_embedder / context_embedder /
 * proj_out, src/diffuser_graph.cpp:283-286, :544-556) in f32 arithmetic.
 * x: f32 [tokens][in_dim]; W: f32 [out_dim][in_dim] (PyTorch layout);
 * bias: f32 [out_dim] or NULL; y: f32 [tokens][out_dim].  Narrow or short
 * problems split the K sum (partials in a stream-ordered allocation,
 * reduced in a fixed order: deterministic). */
int bonsai_linear_f32(const float* x, int tokens, int in_dim, const float* W, const float* bias,
                      int out_dim, float* y, void* stream);

/* Q/K RMSNorm of rms_norm_qk (src/diffuser_graph.cpp:71-79): for each row
 * of head_dim values, y = x / sqrt(mean(x^2) + eps) * w.
 * x, out: f32 [rows][head_dim]; w: f32 [head_dim]. */
int bonsai_rms_norm_f32(const float* x, const float* w, int rows, int head_dim, float eps,
                        float* out, void* stream);

/* adaLN modulate of the blocks (src/diffuser_graph.cpp:347-352, :444-448,
 * :479-480, :546-552): y = LayerNorm(x; eps, no affine) * (1 + scale) + shift.
 * x: f32 [rows][dim]; shift, scale: f32 [dim]; y: f16 [rows][ld_y]. */
int bonsai_ln_modulate(const float* x, int rows, int dim, const float* shift, const float* scale,
                       float eps, uint16_t* y, long long ld_y, void* stream);

/* Same, f32 output (the reference's own ggml_norm + mul/add chain). */
int bonsai_ln_modulate_f32(const float* x, int rows, int dim, const float* shift,
                           const float* scale, float eps, float* y, void* stream);

/* ------------------------------------------------------ attention */

/* Joint non-causal attention (ggml_flash_attn_ext with scale, no mask,
 * GGML_PREC_F32: src/diffuser_graph.cpp:403-416, :506-519).
 * q, k, v: f16 head-major [n_heads][seq][head_dim] (head_dim = 128).
 * out: f16 token-major [seq][ld_out] with head h at columns h*head_dim.
 * scale: softmax scale (the reference uses 1/sqrt(head_dim)).
 * Runs as clusters of two CTAs where they fit: 512 queries per cluster in
 * 64-key blocks, or, where its smaller work units fill the GPU's waves
 * better (few heads at long sequences), 256 queries per cluster in 128-key
 * blocks.  BONSAI_ATTN=pair | v2 | single forces one form (results equal
 * within the tolerance, not bit-identical); BONSAI_ATTN_SPLIT=n splits each
 * head's keys into n ranges merged by a second kernel (used by itself only
 * for launches that fill at most half of the GPU; partials in stream-ordered
 * scratch). */
int bonsai_joint_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int n_heads,
                           int seq, int head_dim, float scale, uint16_t* out, long long ld_out,
                           void* stream);

/* Q/K RMSNorm + RoPE fused, in place on head-major f16 q or k
 * [n_heads][seq][head_dim]: rows with token index < split use w_lo, the
 * rest w_hi (double blocks normalise text and image tokens with different
 * weights: src/diffuser_graph.cpp:371-374).  cos_t/sin_t: f32 [seq][head_dim/2]. */
int bonsai_qk_norm_rope(uint16_t* qk, int n_heads, int seq, int head_dim, const float* w_lo,
                        const float* w_hi, int split, float eps, const float* cos_t,
                        const float* sin_t, void* stream);

/* ------------------------------------------------------ whole model */

/* Model presets.  KLEIN4B = the reference's compiled-in DiffuserParams
 * (src/diffuser_types.h:13-30): 5 double + 20 single blocks, SwiGLU MLP
 * 9216, axes (32,32,32,32), theta 2000, shared modulation, in 128, ctx 7680.
 * FLUX1 = Flux.1-schnell dims: 19 + 38 blocks, GELU-tanh MLP 12288, axes
 * (16,56,56), theta 10000, per-block modulation (B1_0), pooled 768, in 64,
 * ctx 4096. */
#define BONSAI_PRESET_KLEIN4B 0
#define BONSAI_PRESET_FLUX1 1

typedef struct bonsai_dit* bonsai_dit_t;

typedef struct {
  int preset;          /* BONSAI_PRESET_* */
  int depth;           /* double blocks to run (0 = preset value) */
  int depth_single;    /* single blocks to run (0 = preset value) */
  int img_tokens;      /* image tokens (latent H*W after 2x2 packing) */
  int txt_tokens;      /* text tokens */
  int grid_h, grid_w;  /* image token grid for RoPE ids (grid_h*grid_w == img_tokens) */
  unsigned long long seed; /* random-init weights (no checkpoint is read) */
} bonsai_dit_config;

/* Create a model with seeded random B1_0 block weights and f32 edge weights
 * (signs Bernoulli(0.5), scales |N(0, 0.02)| as f16; f32 weights N(0, 0.02);
 * norm weights N(1, 0.1)), plus the activation workspace for the given
 * token counts.  The weights are generated on the host with the same
 * generator the CPU oracle uses, so both see identical tensors. */
int bonsai_dit_create(const bonsai_dit_config* cfg, bonsai_dit_t* out);
int bonsai_dit_destroy(bonsai_dit_t m);

/* One denoise-step forward of build_diffuser_graph (src/diffuser_graph.cpp:231-561)
 * on device buffers: img f32 [img_tokens][in_ch], txt f32 [txt_tokens][ctx_dim],
 * pooled f32 [768] (FLUX1 only, else NULL), timestep t (the graph input, i.e.
 * already x1000 as src/diffuser.cpp:264 does); out f32 [img_tokens][in_ch]. */
int bonsai_dit_forward(bonsai_dit_t m, const float* img, const float* txt, const float* pooled,
                       float timestep, float* out, void* stream);

/* Same with host buffers: copies in, runs, copies the prediction back and
 * synchronises the stream (what a ggml backend's graph_compute does). */
int bonsai_dit_forward_host(bonsai_dit_t m, const float* host_img, const float* host_txt,
                            const float* host_pooled, float timestep, float* host_out,
                            void* stream);

/* Run only double block i (0-based) or single block i on the model's
 * current hidden state; used by block-level parity tests.  The hidden
 * state is f32 [txt_tokens + img_tokens][3072] (text rows first, as
 * ggml_concat(h_txt, h_img) in src/diffuser_graph.cpp:468). */
int bonsai_dit_set_state(bonsai_dit_t m, const float* hidden, const float* vec, void* stream);
int bonsai_dit_get_state(bonsai_dit_t m, float* hidden, void* stream);
int bonsai_dit_double_block(bonsai_dit_t m, int i, void* stream);
int bonsai_dit_single_block(bonsai_dit_t m, int i, void* stream);

/* ---- Multi-GPU: one long image split across GPUs (2048^2, 16896 tokens).
 * Each of `world` ranks (one process per GPU, each with its own model holding
 * the full weights) owns token rows [rank*L/world, (rank+1)*L/world) and
 * heads [rank*24/world, (rank+1)*24/world).  A step is driven as
 *   bonsai_dit_begin                       (edges of own rows, modulation)
 *   for each double block i, then each single block i (kind 0 / 1):
 *     bonsai_dit_phase(kind, i, 0)         LN-modulate own rows -> "xm"
 *     all-gather the rows of "xm"          (caller: NCCL, in place)
 *     bonsai_dit_phase(kind, i, 1)         Q/K/V of own heads on all rows,
 *                                          Q/K norm + RoPE, attention -> "cat"
 *     all-to-all of "cat" columns [0, 3072): own heads x all rows ->
 *                                          all heads x own rows (caller)
 *     bonsai_dit_phase(kind, i, 2)         out-proj / MLP / gate-residual, own rows
 *   all-gather the rows of "hidden", then bonsai_dit_end -> out (every rank).
 * No GEMM FLOP is repeated across ranks (Q/K/V weights are split by head,
 * the rest by token rows).  With world == 1 the phases are exactly
 * bonsai_dit_forward.  The reference has no multi-device path. */
int bonsai_dit_set_partition(bonsai_dit_t m, int rank, int world);
/* Fused exchanges: give the partitioned model every rank's "xm" and "cat"
 * as device pointers valid on this GPU (entry [rank] = its own buffers,
 * the others peer-mapped, e.g. by bonsai_dit_open_peers).  Phase 0 then also
 * stores its LN-modulated rows into every rank's xm, and phase 1's attention
 * stores each output row into its owner's cat (this rank's head columns):
 * the caller drops the all-gather and the all-to-all and only has to order
 * the ranks after phases 0 and 1 (a stream-ordered barrier: bonsai_dit_barrier,
 * or e.g. a one-element NCCL all-reduce), because a rank writes into the
 * others' buffers.  Both
 * kernels end with a system-scope fence after their peer stores.  NULL
 * pointers switch back to caller-side exchanges; bonsai_dit_set_partition
 * does too. */
int bonsai_dit_set_peers(bonsai_dit_t m, void* const* xm, void* const* cat, int world);
/* CUDA IPC handles (2 x 64 bytes: xm, cat) of this model's buffers, for the
 * other ranks' bonsai_dit_open_peers. */
int bonsai_dit_ipc_handles(bonsai_dit_t m, void* out);
/* Open the handles of all ranks (world x 2 x 64 bytes, rank-major, this
 * rank's own entry ignored) and set them as peers; the mappings are closed
 * by the next call or bonsai_dit_destroy. */
int bonsai_dit_open_peers(bonsai_dit_t m, const void* handles, int world);
/* QKV scatter form of the fused exchanges (after bonsai_dit_set_peers /
 * bonsai_dit_open_peers): every rank's q/k/v buffer ("qkv") as a device
 * pointer valid on this GPU (entry [rank] = its own).  Phase 0 then computes
 * q, k and v of this rank's own token rows for EVERY head, and the GEMM's
 * epilogue stores head h straight into the q/k/v buffer of the rank that
 * owns h (the split's all-to-all, fused into the GEMM); phase 0 no longer
 * stores xm rows into the other ranks, and phase 1 runs only the Q/K norm +
 * RoPE and the attention of this rank's heads.  Per rank and block this
 * sends 3 * L/world * 3072 * 2 * (world-1)/world bytes instead of the xm
 * broadcast's L/world * 3072 * 2 * (world-1), overlapped with the GEMM: fewer
 * bytes from world = 4 on.  The caller's ordering between the phases is
 * unchanged.  NULL switches back to the xm broadcast;
 * bonsai_dit_set_partition and bonsai_dit_set_peers(NULL) do too. */
int bonsai_dit_set_qkv_peers(bonsai_dit_t m, void* const* qkv, int world);
/* CUDA IPC handle (64 bytes) of one engine buffer: "hidden", "xm", "cat",
 * "qkv" or "flags" (bonsai_dit_buffer's names). */
int bonsai_dit_ipc_handle(bonsai_dit_t m, const char* name, void* out);
/* Peer flag barrier: the stream-ordered ordering of the ranks after phases 0
 * and 1 of the fused exchanges, without a collective library.  flags: every
 * rank's "flags" buffer (64 u32, allocated with the model) as a device
 * pointer valid on this GPU, entry [rank] = its own.  The call zeroes this
 * rank's flags and synchronises the device; the caller must then order the
 * ranks once (e.g. a host barrier) before any rank calls bonsai_dit_barrier.
 * NULL switches it off; bonsai_dit_set_partition does too. */
int bonsai_dit_set_flag_peers(bonsai_dit_t m, void* const* flags, int world);
/* Open the "flags" IPC handles of all ranks (world x 64 bytes, rank-major,
 * this rank's own entry ignored) and call bonsai_dit_set_flag_peers; the
 * mappings are closed by the next call or bonsai_dit_destroy. */
int bonsai_dit_open_flag_peers(bonsai_dit_t m, const void* handles, int world);
/* Enqueue the barrier on stream: one 32-thread kernel that stores this
 * rank's barrier count into every rank's flags (system-scope release) and
 * waits, on its own GPU's memory, until every rank has stored the same
 * count.  Work enqueued after it sees everything the other ranks wrote into
 * this GPU's buffers before their barrier.  Every rank must call it the same
 * number of times, one process per GPU (ranks that share a GPU cannot use
 * it: their barrier kernels would wait on one another).  A rank that never
 * arrives makes the wait give up after 2 s with DEV_ERR_TIMEOUT_BARRIER
 * (bonsai_device_error).  The reference has no multi-device path. */
int bonsai_dit_barrier(bonsai_dit_t m, void* stream);
/* Open every rank's "qkv" handle (world x 64 bytes, rank-major, this rank's
 * own entry ignored) and pass them to bonsai_dit_set_qkv_peers; the mappings
 * are closed by the next call or bonsai_dit_destroy. */
int bonsai_dit_open_qkv_peers(bonsai_dit_t m, const void* handles, int world);
/* Device pointer and size of an engine buffer shared with the caller's
 * collectives: "hidden" f32 [L][3072], "xm" f16 [L][3072],
 * "cat" f16 [L][3072 + mlp], "qkv" f16 [3][24][L][128]. */
int bonsai_dit_buffer(bonsai_dit_t m, const char* name, void** ptr, long long* bytes);
int bonsai_dit_begin(bonsai_dit_t m, const float* img, const float* txt, const float* pooled,
                     float timestep, void* stream);
int bonsai_dit_phase(bonsai_dit_t m, int kind, int block, int phase, void* stream);
int bonsai_dit_end(bonsai_dit_t m, float* out, void* stream);

/* Export one weight of the model as it is on the device, by the engine's
 * name ("double.<i>.img_qkv", "single.<i>.proj", "mod_img.w", "img_in.w",
 * ...): packed B1_0 bytes [out][in/32][6] (the layout of
 * convert_to_b1_0_packed.py:21-43) or f32 values [out][in].  Returns the byte
 * size when buf is NULL.  Synchronises the device.  Used by the CPU oracle
 * to run on identical weights. */
long long bonsai_dit_weight(bonsai_dit_t m, const char* name, void* buf, long long cap);

/* Replace one weight from host bytes in the layout bonsai_dit_weight
 * exports (B1_0 weights are retiled on the device).  bytes must match the
 * tensor.  Synchronises the device; no forward of this model may be running.
 * The per-tensor form of load_b1 / load_f32_2d (src/diffuser.cpp:27-50). */
int bonsai_dit_set_weight(bonsai_dit_t m, const char* name, const void* host, long long bytes);

/* Load a packed checkpoint in the reference's safetensors layout: the
 * tensor names, dtypes and shapes that src/diffuser.cpp:88-186 reads
 * (x_embedder.weight, transformer_blocks.<d>.attn.to_q.weight, ...;
 * B1_0 tensors U8 [out][in/32*6], the rest F32 [out][in]).  Q/K/V are
 * stacked into the engine's fused weights; blocks beyond the model's depth
 * are ignored (the reference's --max-depth / --max-single).  The same
 * tensors in a GGUF file (convert_to_b1_0.py) load too.  klein4b preset
 * only (BONSAI_ERR_UNSUPPORTED otherwise).  Missing tensors or wrong shapes
 * return BONSAI_ERR_ARG instead of the reference's abort()
 * (src/diffuser.cpp:52-56); tensors are set in order, so after an error the
 * model may hold a mix of old and new weights. */
int bonsai_dit_load_safetensors(bonsai_dit_t m, const char* path);

/* The tensor index of a .safetensors file (src/safetensors.h reads the
 * same container) or of a GGUF file (recognised by its magic; B1_0 is tensor
 * type 100 as convert_to_b1_0.py writes it, listed as U8 [out][in/32*6]
 * under the reference's safetensors names): one line per tensor, sorted by name,
 * "name<TAB>dtype<TAB>d0,d1,...<TAB>begin<TAB>end\n" (data offsets relative to
 * the end of the header).  Host only, no device work.  Returns the full text
 * length (out may be NULL to size it; at most cap-1 bytes are written) or a
 * negative BONSAI_ERR_* code for an unreadable or malformed file. */
int bonsai_safetensors_list(const char* path, char* out, int cap);

/* The reference's whole diffusion loop (src/diffuser.cpp:251-294) on the
 * device: for step s < n_steps, t = 1 - s/n_steps, pred = forward(latents,
 * t*1000), latents += dt*pred with dt = t - t_next (the last step: dt = t).
 * latents: device f32 [img_tokens][in_ch], updated in place.  stats (host,
 * optional): 5 floats per step = the reference's per-step printout {NaN
 * count, Inf count, min, max, mean} of pred (:276-288); when given, the call
 * synchronises the stream. */
int bonsai_dit_sample(bonsai_dit_t m, float* latents, const float* txt, const float* pooled,
                      int n_steps, float* stats, void* stream);

/* ------------------------------------------------------------------ VAE
 * The Flux VAE decoder of the reference's bonsai_vae program
 * (src/vae_decoder.cpp:281-547, graph src/vae_graph.cpp:174-212) on the
 * device.  A decoder is created for one encoded-latent size h x w
 * (128 channels, the reference's --H / --W) and decodes it to a
 * 3 x 16h x 16w image of raw decoder values. */
typedef struct bonsai_vae* bonsai_vae_t;

/* Allocate a decoder with seeded synthetic weights (conv / linear weights
 * N(0, 1/fan_in), norm scales 1 + N(0, 0.1), biases N(0, 0.05), BatchNorm
 * mean N(0, 0.25) and var U(0.25, 4)); load real ones with
 * bonsai_vae_load_safetensors.  Replaces load_vae_weights
 * (src/vae_decoder.cpp:214-250) plus the activation context of :427-444. */
int bonsai_vae_create(int latent_h, int latent_w, unsigned long long seed, bonsai_vae_t* out);
int bonsai_vae_destroy(bonsai_vae_t v);
/* Load flux2-vae.safetensors: every tensor load_vae_weights reads
 * (post_quant_conv.*, decoder.conv_in.*, decoder.mid_block.*,
 * decoder.up_blocks.<i>.*, decoder.conv_norm_out.*, decoder.conv_out.*) and
 * bn.running_mean / bn.running_var (:353-373), PyTorch layouts, F32 (F16
 * and BF16 are converted).  A missing tensor or a wrong shape returns
 * BONSAI_ERR_ARG (the reference throws); tensors are set in order. */
int bonsai_vae_load_safetensors(bonsai_vae_t v, const char* path);
/* latent: device f32 [128][h][w] (the reference's --latent .bin layout);
 * image: device f32 [3][16h][16w].  Inverse BatchNorm + 2x2 un-tiling
 * (:402-421) then the decoder graph; asynchronous on stream. */
int bonsai_vae_decode(bonsai_vae_t v, const float* latent, float* image, void* stream);
/* The same with host buffers: copies in, decodes, copies out, synchronises. */
int bonsai_vae_decode_host(bonsai_vae_t v, const float* host_latent, float* host_image,
                           void* stream);
/* chw_f32_to_hwc_u8 (src/vae_decoder.cpp:262-281) on the device: rgb[y][x][c]
 * = clamp((int)(sigmoid(image[c][y][x]) * 255), 0, 255). */
int bonsai_vae_rgb8(const float* image, int height, int width, unsigned char* rgb, void* stream);
/* One stride-1 'same'-padded convolution of the decoder, ggml_conv_2d_direct
 * (w, x, 1, 1, k/2, k/2, 1, 1) + bias [+ resid] as src/vae_graph.cpp uses it,
 * on the tcgen05 implicit-GEMM kernel: x device NHWC [H][W][cin] f16 (bf16
 * when x_bf16), cin % 8 == 0; w device f32 PyTorch layout [cout][cin][k][k]
 * (k = 1 or 3, converted to x's type per call); bias [cout] and resid
 * (NHWC f32 [H][W][cout]) optional; y device NHWC f32 [H][W][cout]. */
int bonsai_conv2d_nhwc(const void* x, int H, int W, int cin, int x_bf16, const float* w, int cout,
                       int k, const float* bias, const float* resid, float* y, void* stream);
/* Output image size of a decoder (16h x 16w). */
int bonsai_vae_info(bonsai_vae_t v, int* image_h, int* image_w);

#ifdef __cplusplus
}
#endif
#endif /* BONSAI_CUDA_H */
