// Internal declarations of the Flux VAE decoder kernels (vae_conv.cu,
// vae_ops.cu) used by the decoder engine (vae.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace bonsai {

// Output layouts of the implicit-GEMM epilogue.
enum VaeOut : int {
  VOUT_F32 = 0,       // f32 [pix][ld_out] + n
  VOUT_F16 = 1,       // f16 [pix][ld_out] + n
  VOUT_BF16 = 2,      // bf16 [pix][ld_out] + n
  VOUT_F16_T = 3,     // f16 [n][ld_out] + pix (transposed)
  VOUT_F32_NCHW = 4,  // f32 [n][H*W] + pix (planar image)
};

// out[pix][n] = row_scale[pix] * sum_{tap, c} in[pix + off(tap)][c] * w[n][tap*k_per_tap + c]
//               + bias[n] + resid[pix][n]
// in: NHWC 16-bit [H][W][ld_in] (channels 0..cin-1 used), zero outside the
// image (taps = 9: 3x3 'same' convolution; taps = 1: pointwise / plain GEMM).
// w: 16-bit [w_rows][w_ld] (same type as in); for taps = 9, k_per_tap >= cin
// rounded up to 64 and the padding columns hold zeros.  bias, row_scale and
// resid are optional.  in, w, resid and out must be 16-byte aligned.
//
// phases = 4 (with taps = 4) computes conv3x3(upsample_nearest_2x(in)) on the
// 2H x 2W output without forming the upsampled tensor: output pixel
// (2y + a, 2x + b) is a 2x2 convolution of `in` around (y, x) (row offsets
// {a - 1, a}, column offsets {b - 1, b}) with the phase's weights
// w[(2a + b) * w_rows + n] (launch_vae_pack_subpixel_weight folds the 3x3
// kernel into the four 2x2 ones).
//
// Optional epilogue extras (NHWC outputs only): out2, a bf16 NHWC copy of the
// output (ld_out2, N % 32 == 0); stats, GroupNorm(32) partials of the output
// for launch_vae_gn_finalize (N in {128, 256, 512}; stats_slots = capacity,
// *stats_slots_used = slots written).  prof_name labels the launch for
// bonsai_profile_stop (a static string; by default the shape decides).
struct VaeConvArgs {
  const void* in = nullptr;
  long long ld_in = 0;
  int H = 0, W = 0, cin = 0;
  bool bf16 = false;
  int taps = 1;
  const void* w = nullptr;
  long long w_ld = 0;
  int k_per_tap = 0;
  int N = 0;
  int w_rows = 0;  // weight rows in memory (>= N); 0 = N
  const float* bias = nullptr;
  const float* row_scale = nullptr;
  const float* resid = nullptr;
  long long ld_resid = 0;
  void* out = nullptr;
  long long ld_out = 0;
  int out_mode = VOUT_F32;
  int bn = 0;  // output-channel tile (0 = automatic)
  int phases = 1;
  void* out2 = nullptr;
  long long ld_out2 = 0;
  float* stats = nullptr;
  long long stats_slots = 0;
  long long* stats_slots_used = nullptr;
  const char* prof_name = nullptr;
};
int launch_vae_conv(const VaeConvArgs& a, cudaStream_t st);
// GroupNorm partial slots a launch over an H x W input grid writes (upper bound).
long long vae_conv_stat_slots(int H, int W, int phases);
constexpr int kStatGroups = 32;   // partial slot = 32 float4 {sum, M2, count, 0}

// GroupNorm(32) statistics from the conv epilogue's partials (slots x 32
// float4 {sum, M2 about the slot mean, count}): mean_rstd[32][2] = {mean,
// 1/sqrt(var + eps)}, reduced in f64 in a fixed order (deterministic).
// scratch: kGnMergeBlocks * 32 * 4 doubles.
constexpr int kGnMergeBlocks = 148;
int launch_vae_gn_finalize(const float* partials, long long slots, float eps, float* mean_rstd,
                           double* scratch, cudaStream_t st);
// y = [silu]((x - mean_g) * rstd_g * gamma_c + beta_c), f32 [pixels][C] ->
// f16 / bf16 (C = 128, 256, 512 or 1024).
int launch_vae_gn_apply(const float* x, long long pixels, int C, const float* mean_rstd,
                        const float* gamma, const float* beta, bool silu, void* y, bool y_bf16,
                        cudaStream_t st);
// Encoded latent f32 [128][h][w] -> f16 NHWC [2h][2w][64]: channel c < 32 of
// pixel (2i + di, 2j + dj) = latent[4c + 2di + dj][i][j] * bn_std + bn_mean,
// channels 32..63 zero.
int launch_vae_preprocess(const float* latent, int h, int w, const float* bn_mean,
                          const float* bn_std, __half* y, cudaStream_t st);
// Row softmax numerators: P[r][c] = exp(scale * (S[r][c] - max_c S[r][c])) as
// f16, rowinv[r] = 1 / sum_c P[r][c] (f32 sum of the unrounded values).
int launch_vae_softmax(const float* S, long long ld_s, int rows, int cols, float scale,
                       __half* P, long long ld_p, float* rowinv, cudaStream_t st);
// PyTorch-layout f32 weight [cout][cin][taps] -> 16-bit [rows][taps][cin_pad]
// (zero rows >= cout and columns >= cin).
int launch_vae_pack_weight(const float* src, int cout, int cin, int taps, int rows, int cin_pad,
                           void* dst, bool bf16, cudaStream_t st);
// The 3x3 kernel src [cout][cin][3][3] f32 folded into the four 2x2 kernels
// of conv3x3(upsample_nearest_2x(x)): dst 16-bit [4 phases][cout][4 taps][cin_pad],
// phase 2a + b, tap 2ry + rx = the sum of src[ky][kx] over the 3x3 taps
// that read input row offset ry + a - 1 and column offset rx + b - 1.
int launch_vae_pack_subpixel_weight(const float* src, int cout, int cin, int cin_pad, void* dst,
                                    bool bf16, cudaStream_t st);
// Seeded synthetic values: dst[i] = mean + std * N(0,1) (uniform = false) or
// mean + std * U[0,1) (uniform = true), from a counter-based hash of (seed, i).
int launch_vae_fill(float* dst, long long n, unsigned long long seed, float mean, float std,
                    bool uniform, cudaStream_t st);

}  // namespace bonsai
