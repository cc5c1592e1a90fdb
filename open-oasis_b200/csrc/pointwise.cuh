// Launchers for the memory-bound kernels (LayerNorm, SiLU, patch embed, DDIM,
// bridge, post-quant) and the attention kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace oasis {

inline int num_sms_cached() { return num_sms(); }

struct LayerNormParams {
  int rows_out = 0;
  // Row map: in_row = (r / P) * in_group + in_off + r % P; frame = (r / P) * frame_mul + frame_add
  int P = 1;
  long long in_group = 1;
  long long in_off = 0;
  long long frame_mul = 1;
  long long frame_add = 0;
  float eps = 1e-6f;
  // adaLN modulation table [frames, ld_mod]: shift at shift_off, (1 + scale) at scale_off
  const float* mod = nullptr;
  long long ld_mod = 0;
  long long shift_off = 0;
  long long scale_off = 0;
  // or LayerNorm affine weights (VAE)
  const float* affine_w = nullptr;
  const float* affine_b = nullptr;
};

struct PatchEmbedParams {
  int rows = 0;  // input rows of 64 values
  // out_row = (r / P) * out_group + out_off + r % P
  int P = 144;
  long long out_group = 144;
  long long out_off = 0;
};

struct DdimCoeffs {
  float at_sqrt, one_minus_at_sqrt, inv_at_sqrt, inv_sigma, an_sqrt, one_minus_an_sqrt;
};

int layernorm_launch(const float* x, __nv_bfloat16* y, const LayerNormParams& p, cudaStream_t s);
int silu_bf16_launch(const float* x, __nv_bfloat16* y, long long n, cudaStream_t s);
int patch_embed_launch(const float* chunk, const float* w, const float* b, float* z, const PatchEmbedParams& p,
                       cudaStream_t s);
int ddim_launch(float* chunk, const float* v, const DdimCoeffs& c, long long n, cudaStream_t s);
int bridge_launch(const float* chunk, float* latent, int batch, float inv_scale, cudaStream_t s);
int gated_residual_launch(float* z, const float* x, const float* bias, const float* gate, long long ldg,
                          int rows_per_frame, int rows, cudaStream_t s);
// The same with bf16 x (the reduce-scattered partial of sequence-parallel TP).
int gated_residual_bf16_launch(float* z, const __nv_bfloat16* x, const float* bias, const float* gate, long long ldg,
                               int rows_per_frame, int rows, cudaStream_t s);
int post_quant_launch(const float* lat, const float* w, const float* b, float* z, int rows, cudaStream_t s);
// VAE encoder: image [B, 3, 360, 640] -> bf16 patch rows [B * 576, kp] (kp >= 1200, zero-padded);
// moments [B * 576, 32] -> latent [B, 576, 16] and/or chunk [B, 144, 64], both scaled by `scale`.
int image_patchify_launch(const float* img, __nv_bfloat16* out, int batch, int kp, cudaStream_t s);
int moments_to_latent_launch(const float* mom, float* lat, float* chunk, int batch, float scale, cudaStream_t s);

// Attention over a packed qkv buffer [rows, 3 * 1024] bf16 (q | k | v, 16 heads x 64).
// Full (non-causal) attention within groups of `seq` consecutive rows.
int attention_full_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int groups, int seq, int H, cudaStream_t s);
// tcgen05 version for seq a multiple of 144 (attention_tc.cu).
bool attention_tc_supported(int seq);
int attention_tc_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int groups, int seq, int H, cudaStream_t s);
int read_device_error_tc(int reset);
// Causal attention across the T frames of each session, per (patch, head):
// row of (b, t, p) = (b * T + t) * P + p.
int attention_temporal_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int batch, int frames, int P, int H,
                              cudaStream_t s);
int attention_temporal_cached_launch(const __nv_bfloat16* past, const __nv_bfloat16* cur, __nv_bfloat16* out,
                                     int batch, int past_frames, int P, int H, cudaStream_t s);

}  // namespace oasis
