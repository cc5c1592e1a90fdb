// Memory-bound kernels of the frame path: LayerNorm (+adaLN modulate or affine),
// SiLU of the conditioning, the noisy-chunk patch embed, the DDIM update, the
// DiT->VAE bridge (unpatchify + 1/scaling), the VAE post-quant projection and
// the VAE encoder's image patchify and posterior-mean readout.
//
// All are HBM-bound row/element kernels: fp32 vectorised loads (float4),
// warp-shuffle reductions, bf16 stores where the consumer is a GEMM operand.
#include <cstdlib>

#include "common.cuh"
#include "pointwise.cuh"
#include "status.h"

namespace oasis {
namespace {

constexpr int D = 1024;  // model width of both the DiT and the VAE decoder

// One warp per run of `R` consecutive output rows. x is fp32 [*, 1024]; y is
// bf16 [rows_out, 1024]. Row map (gathers the last frame of each session for the
// final layer):
//   in_row = (r / P) * in_group + in_off + r % P
//   frame  = (r / P) * frame_mul + frame_add
// Modulated: y = LN(x) * scale1p[frame] + shift[frame] (scale1p holds 1+scale).
// Affine:    y = LN(x) * w + b.
// A run never crosses a group of P rows (R divides P), so the warp loads its
// lanes' 64 modulation (or affine) values once and reuses them for all R rows:
// the per-row L2 traffic is the 4 KB row instead of the row plus 8 KB of
// modulation. (Issuing the next row's loads before the current row's reduction
// measured slower: the extra 32 registers halve the resident warps.)
__device__ __forceinline__ void ln_load_row(const float* xr, int lane, float4 (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = reinterpret_cast<const float4*>(xr)[lane + 32 * j];
}

__global__ void __launch_bounds__(256, 2)
    layernorm_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, LayerNormParams p, int R) {
  pdl_trigger();
  pdl_wait();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = warp_global * R;
  if (r0 >= p.rows_out) return;
  const int r1 = min(r0 + R, p.rows_out);
  const int grp = r0 / p.P;
  auto in_row = [&](int r) { return (long long)grp * p.in_group + p.in_off + (r - grp * p.P); };

  const float* mul;
  const float* add;
  if (p.affine_w) {
    mul = p.affine_w;
    add = p.affine_b;
  } else {
    const long long frame = (long long)grp * p.frame_mul + p.frame_add;
    mul = p.mod + frame * p.ld_mod + p.scale_off;
    add = p.mod + frame * p.ld_mod + p.shift_off;
  }
  float4 v[8], m[8], a[8];
  ln_load_row(x + in_row(r0) * D, lane, v);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = 4 * (lane + 32 * j);
    m[j] = __ldg(reinterpret_cast<const float4*>(mul + c));
    a[j] = add ? __ldg(reinterpret_cast<const float4*>(add + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r = r0; r < r1; ++r) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.f / D);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a0 = v[j].x - mean, b0 = v[j].y - mean, c0 = v[j].z - mean, d0 = v[j].w - mean;
      q += (a0 * a0 + b0 * b0) + (c0 * c0 + d0 * d0);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q * (1.f / D) + p.eps);
    __nv_bfloat16* yr = y + (long long)r * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = 4 * (lane + 32 * j);
      const float o0 = (v[j].x - mean) * rstd * m[j].x + a[j].x;
      const float o1 = (v[j].y - mean) * rstd * m[j].y + a[j].y;
      const float o2 = (v[j].z - mean) * rstd * m[j].z + a[j].z;
      const float o3 = (v[j].w - mean) * rstd * m[j].w + a[j].w;
      *reinterpret_cast<uint2*>(yr + c) = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
    }
    if (r + 1 < r1) ln_load_row(x + in_row(r + 1) * D, lane, v);
  }
}

__global__ void silu_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n4) {
  pdl_trigger();
  pdl_wait();
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x)[i];
    const float s0 = a.x / (1.f + __expf(-a.x));
    const float s1 = a.y / (1.f + __expf(-a.y));
    const float s2 = a.z / (1.f + __expf(-a.z));
    const float s3 = a.w / (1.f + __expf(-a.w));
    reinterpret_cast<uint2*>(y)[i] = make_uint2(pack_bf16x2(s0, s1), pack_bf16x2(s2, s3));
  }
}

// z[out_row, :] = chunk[r, :64] . W[64, 1024] + b, fp32 throughout.
// Block: 256 threads x 4 columns = one full row width; kEmbedRows rows per block
// (16; 2 for a few hundred rows, so a single frame still spreads over ~70 SMs).
template <int kEmbedRows>
__global__ void __launch_bounds__(256) patch_embed_kernel(const float* __restrict__ chunk, const float* __restrict__ w,
                                                          const float* __restrict__ b, float* __restrict__ z,
                                                          PatchEmbedParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float xs[kEmbedRows][64];
  const int r0 = blockIdx.x * kEmbedRows;
  for (int i = threadIdx.x; i < kEmbedRows * 64; i += 256) {
    const int rr = r0 + i / 64;
    xs[i / 64][i % 64] = rr < p.rows ? chunk[(long long)rr * 64 + (i % 64)] : 0.f;
  }
  __syncthreads();
  const int c = threadIdx.x * 4;
  float4 acc[kEmbedRows];
  const float4 bias = b ? *reinterpret_cast<const float4*>(b + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kEmbedRows; ++i) acc[i] = bias;
#pragma unroll 8
  for (int k = 0; k < 64; ++k) {
    const float4 wk = __ldg(reinterpret_cast<const float4*>(w + k * D + c));
#pragma unroll
    for (int i = 0; i < kEmbedRows; ++i) {
      const float xv = xs[i][k];
      acc[i].x = fmaf(xv, wk.x, acc[i].x);
      acc[i].y = fmaf(xv, wk.y, acc[i].y);
      acc[i].z = fmaf(xv, wk.z, acc[i].z);
      acc[i].w = fmaf(xv, wk.w, acc[i].w);
    }
  }
#pragma unroll
  for (int i = 0; i < kEmbedRows; ++i) {
    const int r = r0 + i;
    if (r >= p.rows) break;
    const int grp = r / p.P, within = r - grp * p.P;
    const long long out_row = (long long)grp * p.out_group + p.out_off + within;
    *reinterpret_cast<float4*>(z + out_row * D + c) = acc[i];
  }
}

__global__ void ddim_kernel(float* __restrict__ chunk, const float* __restrict__ v, DdimCoeffs c, long long n) {
  pdl_trigger();
  pdl_wait();
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float x = chunk[i];
    const float x_start = c.at_sqrt * x - c.one_minus_at_sqrt * v[i];
    const float x_noise = (c.inv_at_sqrt * x - x_start) * c.inv_sigma;
    chunk[i] = c.an_sqrt * x_start + c.one_minus_an_sqrt * x_noise;
  }
}

// chunk [B, 144, 64] in (h, w, p, q, c) order -> latent tokens [B, 576, 16]:
// latent[b, (2h+p)*32 + (2w+q), c] = chunk[b, h*16+w, p*32 + q*16 + c] * inv_scale.
__global__ void bridge_kernel(const float* __restrict__ chunk, float* __restrict__ lat, int batch, float inv_scale) {
  pdl_trigger();
  pdl_wait();
  const long long n = (long long)batch * 576 * 16;
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int c = i & 15;
    const long long t = i >> 4;
    const int tok = t % 576;
    const long long bidx = t / 576;
    const int row = tok >> 5, col = tok & 31;
    const int h = row >> 1, pp = row & 1, w = col >> 1, qq = col & 1;
    lat[i] = chunk[(bidx * 144 + h * 16 + w) * 64 + pp * 32 + qq * 16 + c] * inv_scale;
  }
}

// z[r, :] = lat[r, :16] . W[16, 1024] + b  (VAE post_quant_conv as a linear map)
__global__ void __launch_bounds__(256) post_quant_kernel(const float* __restrict__ lat, const float* __restrict__ w,
                                                         const float* __restrict__ b, float* __restrict__ z, int rows) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= rows) return;
  __shared__ float xs[16];
  if (threadIdx.x < 16) xs[threadIdx.x] = lat[(long long)r * 16 + threadIdx.x];
  __syncthreads();
  const int c = threadIdx.x * 4;
  float4 acc = b ? *reinterpret_cast<const float4*>(b + c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float4 wk = __ldg(reinterpret_cast<const float4*>(w + k * D + c));
    acc.x = fmaf(xs[k], wk.x, acc.x);
    acc.y = fmaf(xs[k], wk.y, acc.y);
    acc.z = fmaf(xs[k], wk.z, acc.z);
    acc.w = fmaf(xs[k], wk.w, acc.w);
  }
  *reinterpret_cast<float4*>(z + (long long)r * D + c) = acc;
}

int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  const long long cap = (long long)num_sms_cached() * 16;
  return (int)(g < cap ? (g > 0 ? g : 1) : cap);
}

// z[r, :] += gate[r / rows_per_frame, :] * (x[r, :] + bias)   (gate NULL: plain residual)
// x is the all-reduced output of a row-parallel projection (tensor parallelism).
template <typename TX>
__global__ void __launch_bounds__(256) gated_residual_kernel(float* __restrict__ z, const TX* __restrict__ x,
                                                             const float* __restrict__ bias,
                                                             const float* __restrict__ gate, long long ldg,
                                                             int rows_per_frame, long long n4) {
  pdl_trigger();
  pdl_wait();
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 4;
    const long long r = e / D;
    const int c = (int)(e - r * D);
    float4 v;
    if constexpr (sizeof(TX) == 4) {
      v = reinterpret_cast<const float4*>(x)[i];
    } else {  // bf16 partial sums (sequence-parallel tensor parallelism)
      const uint2 u = reinterpret_cast<const uint2*>(x)[i];
      v = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                      __uint_as_float(u.y & 0xffff0000u));
    }
    if (bias) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(bias + c));
      v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
    }
    if (gate) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(gate + (r / rows_per_frame) * ldg + c));
      v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
    }
    float4 o = reinterpret_cast<float4*>(z)[i];
    o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
    reinterpret_cast<float4*>(z)[i] = o;
  }
}

// VAE encoder input: image [B, 3, 360, 640] fp32 -> patch rows [B * 576, kp] bf16,
// the 20x20 stride-20 patch_embed conv as a GEMM operand. Row = token (i, j) of the
// 18 x 32 grid; column k = c * 400 + p * 20 + q (the conv weight's flattening order),
// zero for 1200 <= k < kp. Each thread writes 8 columns (one 16-byte store).
__global__ void __launch_bounds__(256) image_patchify_kernel(const float* __restrict__ img,
                                                             __nv_bfloat16* __restrict__ out, int batch, int kp) {
  pdl_trigger();
  pdl_wait();
  const int vec = kp >> 3;
  const long long n = (long long)batch * 576 * vec;
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int k0 = (int)(i % vec) * 8;
    const long long r = i / vec;
    const int tok = (int)(r % 576);
    const long long b = r / 576;
    const int ti = tok >> 5, tj = tok & 31;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      float x = 0.f;
      if (k < 1200) {
        const int c = k / 400, pq = k % 400, pp = pq / 20, qq = pq % 20;
        x = __ldg(img + ((b * 3 + c) * 360 + ti * 20 + pp) * 640 + tj * 20 + qq);
      }
      v[e] = __float2bfloat16(x);
    }
    *reinterpret_cast<uint4*>(out + r * kp + k0) = *reinterpret_cast<const uint4*>(v);
  }
}

// VAE encoder output: moments [B * 576, 32] fp32 (mean | logvar of the posterior)
// -> latent [B, 576, 16] = mean * scale and, if chunk != NULL, the same latent in
// the DiT's patch layout: chunk[b, h*16 + w, p*32 + q*16 + c] = latent[b, (2h+p)*32 + 2w+q, c]
// (the inverse of bridge_kernel without the 1/scale).
__global__ void moments_to_latent_kernel(const float* __restrict__ mom, float* __restrict__ lat,
                                         float* __restrict__ chunk, int batch, float scale) {
  pdl_trigger();
  pdl_wait();
  const long long n = (long long)batch * 576 * 16;
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int c = i & 15;
    const long long t = i >> 4;
    const float x = mom[t * 32 + c] * scale;
    if (lat) lat[i] = x;
    if (chunk) {
      const int tok = t % 576;
      const long long b = t / 576;
      const int row = tok >> 5, col = tok & 31;
      chunk[(b * 144 + (row >> 1) * 16 + (col >> 1)) * 64 + (row & 1) * 32 + (col & 1) * 16 + c] = x;
    }
  }
}

}  // namespace

int gated_residual_launch(float* z, const float* x, const float* bias, const float* gate, long long ldg,
                          int rows_per_frame, int rows, cudaStream_t s) {
  OASIS_REQUIRE(z && x && rows >= 0, "gated_residual: bad arguments");
  OASIS_REQUIRE(!gate || rows_per_frame > 0, "gated_residual: rows_per_frame");
  const long long n4 = (long long)rows * D / 4;
  if (n4 == 0) return OASIS_OK;
  launch_pdl(gated_residual_kernel<float>, dim3(grid_for(n4, 256)), dim3(256), 0, s, z, x, bias, gate, ldg,
             rows_per_frame, n4);
  return check_launch("gated_residual_kernel");
}

int gated_residual_bf16_launch(float* z, const __nv_bfloat16* x, const float* bias, const float* gate, long long ldg,
                               int rows_per_frame, int rows, cudaStream_t s) {
  OASIS_REQUIRE(z && x && rows >= 0, "gated_residual: bad arguments");
  OASIS_REQUIRE(!gate || rows_per_frame > 0, "gated_residual: rows_per_frame");
  const long long n4 = (long long)rows * D / 4;
  if (n4 == 0) return OASIS_OK;
  launch_pdl(gated_residual_kernel<__nv_bfloat16>, dim3(grid_for(n4, 256)), dim3(256), 0, s, z, x, bias, gate, ldg,
             rows_per_frame, n4);
  return check_launch("gated_residual_kernel");
}

int layernorm_launch(const float* x, __nv_bfloat16* y, const LayerNormParams& p, cudaStream_t s) {
  OASIS_REQUIRE(x && y, "layernorm: null pointer");
  OASIS_REQUIRE(p.rows_out >= 0 && p.P > 0, "layernorm: bad row map");
  OASIS_REQUIRE(p.affine_w || p.mod, "layernorm: need affine weights or a modulation table");
  if (p.rows_out == 0) return OASIS_OK;
  // Rows per warp: enough rows that every SM still gets several warps of eight
  // rows (at 73 728 rows: 9 216 warps), else one row per warp; R divides P so a
  // warp's rows share their modulation row.
  static const int force_r = [] {
    const char* e = getenv("OASIS_LN_ROWS");
    return e ? atoi(e) : 0;
  }();
  int R = 1;
  if (force_r > 0) {
    R = p.P % force_r == 0 ? force_r : 1;
  } else if (p.rows_out >= num_sms() * 8 * 16) {
    const int cand[] = {4, 6, 3, 2};  // 73 728 rows: R = 1 / 2 / 4 / 8 / 16 -> 89.0 / 77.8 / 75.5 / 77.2 / 80.6 us
    for (int c : cand)
      if (p.P % c == 0) {
        R = c;
        break;
      }
  }
  const int warps = (p.rows_out + R - 1) / R;
  // a few hundred rows: 2 warps per block, so the rows spread over every SM
  const int warps_per_block = warps < num_sms() * 8 ? 2 : 8;
  const int grid = (warps + warps_per_block - 1) / warps_per_block;
  launch_pdl(layernorm_kernel, dim3(grid), dim3(32 * warps_per_block), 0, s, x, y, p, R);
  return check_launch("layernorm_kernel");
}

int silu_bf16_launch(const float* x, __nv_bfloat16* y, long long n, cudaStream_t s) {
  OASIS_REQUIRE(n % 4 == 0, "silu: n must be a multiple of 4");
  if (n == 0) return OASIS_OK;
  launch_pdl(silu_bf16_kernel, dim3(grid_for(n / 4, 256)), dim3(256), 0, s, x, y, n / 4);
  return check_launch("silu_bf16_kernel");
}

int patch_embed_launch(const float* chunk, const float* w, const float* b, float* z, const PatchEmbedParams& p,
                       cudaStream_t s) {
  OASIS_REQUIRE(chunk && w && z, "patch_embed: null pointer");
  if (p.rows == 0) return OASIS_OK;
  if (p.rows <= 2304)
    launch_pdl(patch_embed_kernel<2>, dim3((p.rows + 1) / 2), dim3(256), 0, s, chunk, w, b, z, p);
  else
    launch_pdl(patch_embed_kernel<16>, dim3((p.rows + 15) / 16), dim3(256), 0, s, chunk, w, b, z, p);
  return check_launch("patch_embed_kernel");
}

int ddim_launch(float* chunk, const float* v, const DdimCoeffs& c, long long n, cudaStream_t s) {
  OASIS_REQUIRE(chunk && v, "ddim: null pointer");
  if (n == 0) return OASIS_OK;
  launch_pdl(ddim_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, chunk, v, c, n);
  return check_launch("ddim_kernel");
}

int bridge_launch(const float* chunk, float* latent, int batch, float inv_scale, cudaStream_t s) {
  OASIS_REQUIRE(chunk && latent && batch >= 0, "bridge: bad arguments");
  if (batch == 0) return OASIS_OK;
  launch_pdl(bridge_kernel, dim3(grid_for((long long)batch * 576 * 16, 256)), dim3(256), 0, s, chunk, latent, batch, inv_scale);
  return check_launch("bridge_kernel");
}

int post_quant_launch(const float* lat, const float* w, const float* b, float* z, int rows, cudaStream_t s) {
  OASIS_REQUIRE(lat && w && z, "post_quant: null pointer");
  if (rows == 0) return OASIS_OK;
  launch_pdl(post_quant_kernel, dim3(rows), dim3(256), 0, s, lat, w, b, z, rows);
  return check_launch("post_quant_kernel");
}

int image_patchify_launch(const float* img, __nv_bfloat16* out, int batch, int kp, cudaStream_t s) {
  OASIS_REQUIRE(img && out && batch >= 0, "image_patchify: bad arguments");
  OASIS_REQUIRE(kp >= 1200 && kp % 8 == 0, "image_patchify: kp=%d", kp);
  if (batch == 0) return OASIS_OK;
  launch_pdl(image_patchify_kernel, dim3(grid_for((long long)batch * 576 * (kp / 8), 256)), dim3(256), 0, s, img, out,
             batch, kp);
  return check_launch("image_patchify_kernel");
}

int moments_to_latent_launch(const float* mom, float* lat, float* chunk, int batch, float scale, cudaStream_t s) {
  OASIS_REQUIRE(mom && (lat || chunk) && batch >= 0, "moments_to_latent: bad arguments");
  if (batch == 0) return OASIS_OK;
  launch_pdl(moments_to_latent_kernel, dim3(grid_for((long long)batch * 576 * 16, 256)), dim3(256), 0, s, mom, lat,
             chunk, batch, scale);
  return check_launch("moments_to_latent_kernel");
}

}  // namespace oasis
