/*
 * CPU oracle for the bonsai.cpp diffuser-transformer step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the algorithm of
 * the reference's diffuser graph so that the CUDA engine can be checked
 * against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load it; the product library never links or calls it.
 *
 * Every function cites the reference file:line it follows (paths relative to
 * the bonsai.cpp repository).  The reference's custom ops (b1_linear_f32_f32,
 * rope_2d_fwd_f32) are restated here and additionally available verbatim
 * through oracle/_ref (ref_bridge.cpp).  The ggml built-ins the graph uses
 * (ggml_norm, ggml_rms_norm, ggml_flash_attn_ext, ggml_swiglu, ggml_mul_mat,
 * ggml_timestep_embedding) come from the reference's un-vendored ggml fork, so
 * their restatement follows ggml's published algorithms: parity for those is
 * pinned by this restatement, not by the fork's code.
 *
 * Layouts: row-major, "[a][b]" = a rows of b elements (ggml ne = {b, a}).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------ fp16 helpers */
static float f16_bits_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}
/* Round-to-nearest-even f32 -> f16 -> f32 (ggml_cast F32->F16). */
static float round_f16(float x) { return (float)(_Float16)x; }

ORC_EXPORT void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------- B1_0 linear
 * b1_linear_f32_f32, scalar path (src/b1_0_kernel.h:240-287):
 * for each output row r and token b: sum over 32-weight blocks of
 * scale * (sum_i bit_i ? +a : -a), accumulated in the same order.
 * act f32 [tokens][in_dim]; w packed [out_dim][in_dim/32][6]; out [tokens][out_dim]. */
ORC_EXPORT void orc_b1_linear(const float* act, int tokens, int in_dim, const uint8_t* w,
                              int out_dim, float* out) {
  const int nblk = in_dim / 32;
  const int row_stride = nblk * 6;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < out_dim; ++r) {
    for (int b = 0; b < tokens; ++b) {
      const float* a = act + (size_t)b * in_dim;
      float sum = 0.0f;
      for (int blk = 0; blk < nblk; ++blk) {
        const uint8_t* p = w + (size_t)r * row_stride + blk * 6;
        uint16_t sb;
        uint32_t bits;
        memcpy(&sb, p, 2);
        memcpy(&bits, p + 2, 4);
        const float scale = f16_bits_to_f32(sb);
        float bs = 0.0f;
        for (int i = 0; i < 32; ++i) {
          const float v = a[blk * 32 + i];
          if ((bits >> i) & 1u) bs += v; else bs -= v;
        }
        sum += scale * bs;
      }
      out[(size_t)b * out_dim + r] = sum;
    }
  }
}

/* The B1_0 linear used inside the oracle's blocks.  By default the C
 * restatement above; orc_use_reference_b1() swaps in the reference's own
 * b1_linear_f32_f32 (oracle/_ref, AVX2 build) so a block runs the
 * reference's exact kernel for every linear. */
typedef void (*ref_b1_fn)(const float*, int, int, const uint8_t*, int, float*, int);
static ref_b1_fn g_ref_b1 = 0;
static int g_ref_threads = 1;
ORC_EXPORT void orc_use_reference_b1(void* fn, int nthreads) {
  g_ref_b1 = (ref_b1_fn)fn;
  g_ref_threads = nthreads > 0 ? nthreads : 1;
}
static void block_b1(const float* act, int tokens, int in_dim, const uint8_t* w, int out_dim,
                     float* out) {
  if (g_ref_b1)
    g_ref_b1(act, tokens, in_dim, w, out_dim, out, g_ref_threads);
  else
    orc_b1_linear(act, tokens, in_dim, w, out_dim, out);
}

/* Attention input rounding: 1 (default) rounds q, k, v to f16 as the
 * reference's graph does; 0 gives the fp32 dequantised-weight oracle. */
static int g_attn_f16 = 1;
ORC_EXPORT void orc_set_attention_f16(int on) { g_attn_f16 = on; }

/* Dense f32 linear, ggml_mul_mat(W, x) with W [out][in] (src/diffuser_graph.cpp:283-311):
 * y[t][o] = sum_i W[o][i] * x[t][i] (+ bias[o] when given). */
ORC_EXPORT void orc_linear_f32(const float* x, int tokens, int in_dim, const float* W,
                               const float* bias, int out_dim, float* y) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < tokens; ++t)
    for (int o = 0; o < out_dim; ++o) {
      double s = 0.0;
      const float* xr = x + (size_t)t * in_dim;
      const float* wr = W + (size_t)o * in_dim;
      for (int i = 0; i < in_dim; ++i) s += (double)wr[i] * xr[i];
      y[(size_t)t * out_dim + o] = (float)s + (bias ? bias[o] : 0.0f);
    }
}

/* ------------------------------------------------------------------- RoPE
 * compute_rope_freqs_data (src/diffuser_graph.cpp:126-140):
 * values[a][j] = 1 / theta^((2j)/axes_dim[a]) for j < axes_dim[a]/2. */
ORC_EXPORT void orc_rope_freqs(const int* axes_dim, int n_axes, float theta, float* values,
                               int max_half) {
  for (int a = 0; a < n_axes; ++a) {
    for (int j = 0; j < max_half; ++j) values[a * max_half + j] = 0.0f;
    for (int j = 0; j < axes_dim[a] / 2; ++j) {
      const float scale = (float)(j * 2) / (float)axes_dim[a];
      values[a * max_half + j] = 1.0f / powf(theta, scale);
    }
  }
}

/* build_rope_cos_sin (src/diffuser_graph.cpp:142-182): per axis a, angles
 * [ax_half][seq] = freq[a][j] * ids[s][a] (a 1x1 mul_mat per element), the
 * axes concatenated along the pair dimension, then cos / sin.
 * ids f32 [seq][n_axes]; cos_out/sin_out f32 [seq][sum(axes_dim)/2]. */
ORC_EXPORT void orc_rope_cos_sin(const float* ids, int seq, const int* axes_dim, int n_axes,
                                 float theta, float* cos_out, float* sin_out) {
  int max_half = 0, half = 0;
  for (int a = 0; a < n_axes; ++a) {
    if (axes_dim[a] / 2 > max_half) max_half = axes_dim[a] / 2;
    half += axes_dim[a] / 2;
  }
  float* freqs = (float*)malloc(sizeof(float) * (size_t)max_half * n_axes);
  orc_rope_freqs(axes_dim, n_axes, theta, freqs, max_half);
  for (int s = 0; s < seq; ++s) {
    int d = 0;
    for (int a = 0; a < n_axes; ++a)
      for (int j = 0; j < axes_dim[a] / 2; ++j, ++d) {
        const float ang = freqs[a * max_half + j] * ids[(size_t)s * n_axes + a];
        cos_out[(size_t)s * half + d] = cosf(ang);
        sin_out[(size_t)s * half + d] = sinf(ang);
      }
  }
  free(freqs);
}

/* rope_2d_fwd_f32 (src/b1_0_kernel.h:309-361): pairs (2d, 2d+1) of every
 * (token, head) rotate by the angle of (token, d).
 * x/out f32 [seq][n_heads][head_dim]; cos/sin f32 [seq][head_dim/2]. */
ORC_EXPORT void orc_rope_apply(const float* x, const float* c, const float* s, int head_dim,
                               int n_heads, int seq, float* out) {
  const int half = head_dim / 2;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < seq; ++t)
    for (int h = 0; h < n_heads; ++h) {
      const size_t base = (size_t)t * n_heads * head_dim + (size_t)h * head_dim;
      for (int d = 0; d < half; ++d) {
        const float cv = c[(size_t)t * half + d], sv = s[(size_t)t * half + d];
        const float a = x[base + 2 * d], b = x[base + 2 * d + 1];
        out[base + 2 * d] = a * cv - b * sv;
        out[base + 2 * d + 1] = a * sv + b * cv;
      }
    }
}

/* ------------------------------------------------------------ norms
 * rms_norm_qk (src/diffuser_graph.cpp:71-79): ggml_rms_norm(eps) over each
 * head_dim row (sum of squares in double, scale = 1/sqrtf(mean + eps)),
 * then * w. */
ORC_EXPORT void orc_rms_norm(const float* x, const float* w, int rows, int dim, float eps,
                             float* y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * dim;
    double s2 = 0.0;
    for (int i = 0; i < dim; ++i) s2 += (double)xr[i] * xr[i];
    const float mean = (float)(s2 / dim);
    const float sc = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < dim; ++i) y[(size_t)r * dim + i] = (xr[i] * sc) * w[i];
  }
}

/* adaLN modulate (src/diffuser_graph.cpp:347-352, :444-448, :479-480,
 * :546-552): ggml_norm(x, eps) (mean and variance in double, no affine),
 * then y * (scale + 1) + shift. */
ORC_EXPORT void orc_ln_modulate(const float* x, int rows, int dim, const float* shift,
                                const float* scale, float eps, float* y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * dim;
    float* yr = y + (size_t)r * dim;
    double s = 0.0;
    for (int i = 0; i < dim; ++i) s += xr[i];
    const float mean = (float)(s / dim);
    double s2 = 0.0;
    for (int i = 0; i < dim; ++i) {
      const float v = xr[i] - mean;
      s2 += (double)(v * v);
    }
    const float var = (float)(s2 / dim);
    const float sc = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < dim; ++i) {
      const float n = (xr[i] - mean) * sc;
      yr[i] = n * (scale[i] + 1.0f) + shift[i];
    }
  }
}

/* --------------------------------------------------------- activations */
static float silu_f(float x) { return x / (1.0f + expf(-x)); }
static float gelu_tanh_f(float x) {
  const float k0 = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}
/* ggml_swiglu (src/diffuser_graph.cpp:227-229, tests/ops/test_all_ops.py:29-46):
 * x [rows][2n] -> silu(x[:, :n]) * x[:, n:]. */
ORC_EXPORT void orc_swiglu(const float* x, int rows, int n, float* y, int ld_y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int i = 0; i < n; ++i)
      y[(size_t)r * ld_y + i] = silu_f(x[(size_t)r * 2 * n + i]) * x[(size_t)r * 2 * n + n + i];
}
/* GELU-tanh for the Flux.1 preset (not in the reference; restated from its
 * definition). x [rows][n] -> y [rows][ld_y]. */
ORC_EXPORT void orc_gelu(const float* x, int rows, int n, float* y, int ld_y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int i = 0; i < n; ++i) y[(size_t)r * ld_y + i] = gelu_tanh_f(x[(size_t)r * n + i]);
}

/* ------------------------------------------------------------ attention
 * Joint attention (src/diffuser_graph.cpp:395-416, :502-519): K and V are
 * cast to f16 (:409-410) and ggml's CPU flash_attn_ext converts Q to the K
 * type for its dot products, so q, k, v are all rounded to f16; scores and
 * the softmax are f32 (GGML_PREC_F32), no mask, non-causal.
 * q, k, v f32 [seq][n_heads][hd] (ggml [hd, H, S]); out f32 [seq][n_heads*hd]. */
ORC_EXPORT void orc_attention(const float* q, const float* k, const float* v, int seq,
                              int n_heads, int hd, float scale, float* out) {
  const size_t n = (size_t)seq * n_heads * hd;
  float* q16 = (float*)malloc(n * sizeof(float));
  float* k16 = (float*)malloc(n * sizeof(float));
  float* v16 = (float*)malloc(n * sizeof(float));
  for (size_t i = 0; i < n; ++i) {
    q16[i] = g_attn_f16 ? round_f16(q[i]) : q[i];
    k16[i] = g_attn_f16 ? round_f16(k[i]) : k[i];
    v16[i] = g_attn_f16 ? round_f16(v[i]) : v[i];
  }
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)seq);
    float* acc = (float*)malloc(sizeof(float) * (size_t)hd);
#pragma omp for collapse(2) schedule(static)
    for (int h = 0; h < n_heads; ++h)
      for (int i = 0; i < seq; ++i) {
        const float* qi = q16 + ((size_t)i * n_heads + h) * hd;
        float mx = -INFINITY;
        for (int j = 0; j < seq; ++j) {
          const float* kj = k16 + ((size_t)j * n_heads + h) * hd;
          /* eight fixed partial sums: a deterministic order that vectorises */
          float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          int d = 0;
          for (; d + 8 <= hd; d += 8)
            for (int u = 0; u < 8; ++u) part[u] += qi[d + u] * kj[d + u];
          float s = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
          for (; d < hd; ++d) s += qi[d] * kj[d];
          s *= scale;
          sc[j] = s;
          if (s > mx) mx = s;
        }
        float l = 0.0f;
        for (int d = 0; d < hd; ++d) acc[d] = 0.0f;
        for (int j = 0; j < seq; ++j) {
          const float p = expf(sc[j] - mx);
          l += p;
          const float* vj = v16 + ((size_t)j * n_heads + h) * hd;
          for (int d = 0; d < hd; ++d) acc[d] += p * vj[d];
        }
        float* o = out + (size_t)i * n_heads * hd + (size_t)h * hd;
        for (int d = 0; d < hd; ++d) o[d] = acc[d] / l;
      }
    free(sc);
    free(acc);
  }
  free(q16);
  free(k16);
  free(v16);
}

/* ------------------------------------------------------- timestep embedding
 * ggml_timestep_embedding(t, 256, 10000) then the half swap of
 * src/diffuser_graph.cpp:288-292: freq_j = exp(-ln(10000) * j / 128),
 * result = [sin(t*freq), cos(t*freq)]. */
ORC_EXPORT void orc_timestep_embedding(float t, int dim, float max_period, float* out) {
  const int half = dim / 2;
  for (int j = 0; j < half; ++j) {
    const float freq = expf(-logf(max_period) * (float)j / (float)half);
    const float arg = t * freq;
    out[j] = sinf(arg);
    out[half + j] = cosf(arg);
  }
}

/* ------------------------------------------------------------ blocks */
typedef struct {
  int preset;      /* 0 = klein4b (SwiGLU), 1 = flux1 (GELU-tanh) */
  int hidden;      /* 3072 */
  int heads;       /* 24 */
  int head_dim;    /* 128 */
  int mlp;         /* MLP hidden width (after the activation) */
} orc_dims;

/* Shared helper: per-head RMSNorm (+RoPE) on a [L][3*H] qkv buffer in place
 * for q (offset 0) and k (offset H); tokens < split use w_lo, else w_hi. */
static void qk_norm_rope(float* qkv, int L, const orc_dims* D, const float* wq_lo,
                         const float* wk_lo, const float* wq_hi, const float* wk_hi, int split,
                         const float* cos_t, const float* sin_t) {
  const int H = D->hidden, hd = D->head_dim, nh = D->heads, half = hd / 2;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < L; ++t) {
    for (int which = 0; which < 2; ++which) {
      const float* w = which == 0 ? (t < split ? wq_lo : wq_hi) : (t < split ? wk_lo : wk_hi);
      for (int h = 0; h < nh; ++h) {
        float* x = qkv + (size_t)t * 3 * H + (size_t)which * H + (size_t)h * hd;
        double s2 = 0.0;
        for (int i = 0; i < hd; ++i) s2 += (double)x[i] * x[i];
        const float sc = 1.0f / sqrtf((float)(s2 / hd) + 1e-6f);
        float tmp[512];
        for (int i = 0; i < hd; ++i) tmp[i] = (x[i] * sc) * w[i];
        for (int d = 0; d < half; ++d) {
          const float cv = cos_t[(size_t)t * half + d], sv = sin_t[(size_t)t * half + d];
          const float a = tmp[2 * d], b = tmp[2 * d + 1];
          x[2 * d] = a * cv - b * sv;
          x[2 * d + 1] = a * sv + b * cv;
        }
      }
    }
  }
}

/* Exported form of the fused Q/K RMSNorm + RoPE for head-major tensors:
 * x f32 [n_heads][seq][hd] in place; tokens < split use w_lo else w_hi. */
ORC_EXPORT void orc_qk_norm_rope_heads(float* x, int n_heads, int seq, int hd, const float* w_lo,
                                       const float* w_hi, int split, float eps,
                                       const float* cos_t, const float* sin_t) {
  const int half = hd / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < n_heads; ++h)
    for (int t = 0; t < seq; ++t) {
      float* r = x + ((size_t)h * seq + t) * hd;
      const float* w = t < split ? w_lo : w_hi;
      double s2 = 0.0;
      for (int i = 0; i < hd; ++i) s2 += (double)r[i] * r[i];
      const float sc = 1.0f / sqrtf((float)(s2 / hd) + eps);
      float tmp[512];
      for (int i = 0; i < hd; ++i) tmp[i] = (r[i] * sc) * w[i];
      for (int d = 0; d < half; ++d) {
        const float cv = cos_t[(size_t)t * half + d], sv = sin_t[(size_t)t * half + d];
        r[2 * d] = tmp[2 * d] * cv - tmp[2 * d + 1] * sv;
        r[2 * d + 1] = tmp[2 * d] * sv + tmp[2 * d + 1] * cv;
      }
    }
}

/* Split a [L][3H] qkv buffer into q, k, v [L][H] (head-interleaved rows). */
static void split3(const float* qkv, int L, int H, float* q, float* k, float* v) {
  for (int t = 0; t < L; ++t) {
    memcpy(q + (size_t)t * H, qkv + (size_t)t * 3 * H, sizeof(float) * H);
    memcpy(k + (size_t)t * H, qkv + (size_t)t * 3 * H + H, sizeof(float) * H);
    memcpy(v + (size_t)t * H, qkv + (size_t)t * 3 * H + 2 * H, sizeof(float) * H);
  }
}

/* One double-stream block (src/diffuser_graph.cpp:341-466).
 * h: f32 [L_txt + L_img][H], text rows first; updated in place.
 * mod_img / mod_txt: f32 [6H] = shift1, scale1, gate1, shift2, scale2, gate2
 * (split_mod, src/diffuser_graph.cpp:33-41).
 * w_*_qkv: packed [3H][H/32*6] = the to_q, to_k, to_v matrices stacked.
 * w_*_mlp_in: packed [mlp_in_rows][H/32*6] (2*mlp rows for SwiGLU, mlp for GELU).
 * cos_t/sin_t: f32 [L][hd/2] for the joint sequence (text first). */
ORC_EXPORT void orc_double_block(const orc_dims* D, int L_txt, int L_img, float* h,
                                 const float* mod_img, const float* mod_txt,
                                 const uint8_t* w_img_qkv, const uint8_t* w_txt_qkv,
                                 const uint8_t* w_img_out, const uint8_t* w_txt_out,
                                 const uint8_t* w_img_mlp_in, const uint8_t* w_img_mlp_out,
                                 const uint8_t* w_txt_mlp_in, const uint8_t* w_txt_mlp_out,
                                 const float* nq_img, const float* nk_img, const float* nq_txt,
                                 const float* nk_txt, const float* cos_t, const float* sin_t) {
  const int H = D->hidden, L = L_txt + L_img;
  const int mlp_in_rows = D->preset == 0 ? 2 * D->mlp : D->mlp;
  float* xm = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)L * 3 * H);
  float* q = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* k = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* v = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* att = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* y = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* mi = (float*)malloc(sizeof(float) * (size_t)L * mlp_in_rows);
  float* ma = (float*)malloc(sizeof(float) * (size_t)L * D->mlp);
  float* h_txt = h;
  float* h_img = h + (size_t)L_txt * H;
  const float* mods[2] = {mod_txt, mod_img};
  float* hs[2] = {h_txt, h_img};
  const int Ls[2] = {L_txt, L_img};
  const int offs[2] = {0, L_txt};
  const uint8_t* wqkv[2] = {w_txt_qkv, w_img_qkv};
  const uint8_t* wout[2] = {w_txt_out, w_img_out};
  const uint8_t* wmi[2] = {w_txt_mlp_in, w_img_mlp_in};
  const uint8_t* wmo[2] = {w_txt_mlp_out, w_img_mlp_out};

  /* attention sub-block: LN-modulate (:347-352), q/k/v (:354-361) */
  for (int sidx = 0; sidx < 2; ++sidx) {
    const float* m = mods[sidx];
    orc_ln_modulate(hs[sidx], Ls[sidx], H, m + 0 * H, m + 1 * H, 1e-6f,
                    xm + (size_t)offs[sidx] * H);
    block_b1(xm + (size_t)offs[sidx] * H, Ls[sidx], H, wqkv[sidx], 3 * H,
                  qkv + (size_t)offs[sidx] * 3 * H);
  }
  /* rms_norm_qk (:371-374) with per-stream weights, RoPE (:383-384) */
  qk_norm_rope(qkv, L, D, nq_txt, nk_txt, nq_img, nk_img, L_txt, cos_t, sin_t);
  /* joint attention over [txt; img] (:395-416) */
  split3(qkv, L, H, q, k, v);
  orc_attention(q, k, v, L, D->heads, D->head_dim, 1.0f / sqrtf((float)D->head_dim), att);
  for (int sidx = 0; sidx < 2; ++sidx) {
    const float* m = mods[sidx];
    /* out projections (:434-437) and gate-residual (:440-442) */
    block_b1(att + (size_t)offs[sidx] * H, Ls[sidx], H, wout[sidx], H, y);
    for (int t = 0; t < Ls[sidx]; ++t)
      for (int i = 0; i < H; ++i) hs[sidx][(size_t)t * H + i] += m[2 * H + i] * y[(size_t)t * H + i];
    /* MLP sub-block (:444-460) */
    orc_ln_modulate(hs[sidx], Ls[sidx], H, m + 3 * H, m + 4 * H, 1e-6f, xm);
    block_b1(xm, Ls[sidx], H, wmi[sidx], mlp_in_rows, mi);
    if (D->preset == 0)
      orc_swiglu(mi, Ls[sidx], D->mlp, ma, D->mlp);
    else
      orc_gelu(mi, Ls[sidx], D->mlp, ma, D->mlp);
    block_b1(ma, Ls[sidx], D->mlp, wmo[sidx], H, y);
    for (int t = 0; t < Ls[sidx]; ++t)
      for (int i = 0; i < H; ++i) hs[sidx][(size_t)t * H + i] += m[5 * H + i] * y[(size_t)t * H + i];
  }
  free(xm); free(qkv); free(q); free(k); free(v); free(att); free(y); free(mi); free(ma);
}

/* One single-stream block (src/diffuser_graph.cpp:476-542).
 * h: f32 [L][H] (combined, text first), updated in place.
 * mod: f32 [3H] = shift, scale, gate (split_mod_single, :43-48).
 * w_proj: packed [3H + mlp_in_rows][H/32*6] (to_qkv_mlp_proj);
 * w_out: packed [H][(H + mlp)/32*6] (to_out on concat(attn, mlp_act), :534-536). */
ORC_EXPORT void orc_single_block(const orc_dims* D, int L, float* h, const float* mod,
                                 const uint8_t* w_proj, const uint8_t* w_out, const float* nq,
                                 const float* nk, const float* cos_t, const float* sin_t) {
  const int H = D->hidden;
  const int mlp_in_rows = D->preset == 0 ? 2 * D->mlp : D->mlp;
  const int P = 3 * H + mlp_in_rows;
  const int C = H + D->mlp;
  float* xm = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* proj = (float*)malloc(sizeof(float) * (size_t)L * P);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)L * 3 * H);
  float* mi = (float*)malloc(sizeof(float) * (size_t)L * mlp_in_rows);
  float* q = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* k = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* v = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* cat = (float*)malloc(sizeof(float) * (size_t)L * C);
  float* att = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* y = (float*)malloc(sizeof(float) * (size_t)L * H);
  orc_ln_modulate(h, L, H, mod + 0, mod + H, 1e-6f, xm); /* :479-480 */
  block_b1(xm, L, H, w_proj, P, proj);               /* :482 */
  for (int t = 0; t < L; ++t) {                            /* views :484-486 */
    memcpy(qkv + (size_t)t * 3 * H, proj + (size_t)t * P, sizeof(float) * 3 * H);
    memcpy(mi + (size_t)t * mlp_in_rows, proj + (size_t)t * P + 3 * H, sizeof(float) * mlp_in_rows);
  }
  qk_norm_rope(qkv, L, D, nq, nk, nq, nk, L, cos_t, sin_t); /* :490-499 */
  split3(qkv, L, H, q, k, v);
  orc_attention(q, k, v, L, D->heads, D->head_dim, 1.0f / sqrtf((float)D->head_dim), att);
  for (int t = 0; t < L; ++t) memcpy(cat + (size_t)t * C, att + (size_t)t * H, sizeof(float) * H);
  if (D->preset == 0) /* :533-534 */
    orc_swiglu(mi, L, D->mlp, cat + H, C);
  else
    orc_gelu(mi, L, D->mlp, cat + H, C);
  block_b1(cat, L, C, w_out, H, y); /* :536 */
  for (int t = 0; t < L; ++t)           /* :538 */
    for (int i = 0; i < H; ++i) h[(size_t)t * H + i] += mod[2 * H + i] * y[(size_t)t * H + i];
  free(xm); free(proj); free(qkv); free(mi); free(q); free(k); free(v); free(cat); free(att); free(y);
}

/* silu applied elementwise (ggml_silu). */
ORC_EXPORT void orc_silu(const float* x, int n, float* y) {
  for (int i = 0; i < n; ++i) y[i] = silu_f(x[i]);
}
