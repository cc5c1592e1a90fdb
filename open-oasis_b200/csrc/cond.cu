// Frame conditioning on the GPU: the timestep MLP and the action projection of
// compute_cond_for_frame (oasis_inference.py:1406-1427), which the reference runs
// on the host in fp32 once per frame and DDIM level:
//   cond[r] = W2 silu(W0 emb(t_r) + b0) + b2 + (actions[r] We^T + be)
//   emb(t)  = [cos(t f_i) | sin(t f_i)], f_i = exp(-ln(1e4) i / 128), i < 128
// Everything stays fp32 (the reference keeps this path in fp32 "for precision"),
// on CUDA cores: two register-tiled SGEMMs over all rows of a frame (every DDIM
// step x session x frame), the first generating its A operand (the sinusoidal
// embedding) on the fly, the second adding the action projection in its epilogue.
// At 64 sessions x 8 frames x 4 steps that is 2048 rows, 4.3 GFLOP.
#include "../../include/oasis_b200.h"
#include "common.cuh"
#include "status.h"

namespace oasis {
namespace {

constexpr int kFreq = 256;  // timestep embedding width
constexpr int kD = 1024;
constexpr int kAct = 25;
constexpr int TM = 64, TN = 64, TK = 16;  // CTA tile; 256 threads x (4 rows x 4 cols)

// Stage 0: h = silu(emb(levels) W0^T + b0), K = 256.
// Stage 1: cond = h W2^T + b2 (+ actions[r % action_rows] We^T + be), K = 1024.
template <int kStage>
__global__ void __launch_bounds__(256) cond_gemm_kernel(const float* __restrict__ levels,
                                                        const float* __restrict__ freqs,
                                                        const float* __restrict__ a_in,  // stage 1: h [n, 1024]
                                                        const float* __restrict__ w, const float* __restrict__ b,
                                                        const float* __restrict__ actions, int action_rows,
                                                        const float* __restrict__ ext_w,
                                                        const float* __restrict__ ext_b, float* __restrict__ out,
                                                        int n) {
  constexpr int K = kStage == 0 ? kFreq : kD;
  __shared__ float As[TK][TM + 4];
  __shared__ float Ws[TK][TN + 4];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int r0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  // loader roles: row (or output column) tid / 4, four consecutive k at (tid % 4) * 4
  const int lr = tid >> 2, lk = (tid & 3) * 4;
  const int ar = r0 + lr;
  const float t = (kStage == 0 && ar < n) ? levels[ar] : 0.f;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    float4 av = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ar < n) {
      if constexpr (kStage == 0) {
        float e[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = k0 + lk + j;
          const float arg = t * freqs[k & 127];
          e[j] = k < 128 ? cosf(arg) : sinf(arg);
        }
        av = make_float4(e[0], e[1], e[2], e[3]);
      } else {
        av = *reinterpret_cast<const float4*>(a_in + (size_t)ar * K + k0 + lk);
      }
    }
    const float4 wv = *reinterpret_cast<const float4*>(w + (size_t)(n0 + lr) * K + k0 + lk);
    __syncthreads();
    As[lk + 0][lr] = av.x;
    As[lk + 1][lr] = av.y;
    As[lk + 2][lr] = av.z;
    As[lk + 3][lr] = av.w;
    Ws[lk + 0][lr] = wv.x;
    Ws[lk + 1][lr] = wv.y;
    Ws[lk + 2][lr] = wv.z;
    Ws[lk + 3][lr] = wv.w;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 w4 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float ai[4] = {a4.x, a4.y, a4.z, a4.w};
      const float wj[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ai[i], wj[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= n) break;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      float v = acc[i][j] + b[c];
      if constexpr (kStage == 0) {
        v = v / (1.f + expf(-v));  // SiLU
      } else if (actions) {
        const float* ar_ = actions + (size_t)(r % action_rows) * kAct;
        const float* we = ext_w + (size_t)c * kAct;
        float e = 0.f;
#pragma unroll
        for (int q = 0; q < kAct; ++q) e = fmaf(ar_[q], we[q], e);
        v += e + ext_b[c];
      }
      o[j] = v;
    }
    *reinterpret_cast<float4*>(out + (size_t)r * kD + n0 + tx * 4) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// Few rows (one session's frame: 4 steps x 2 frames = 8): the tiled kernel
// would put 16 CTAs on a 4 MB weight stream, 64 dependent K steps each. Here a
// warp owns one output column and its 32 lanes stride K, so each weight row is
// read as whole 128-byte runs by 256 warps at once; the kRows A rows sit in
// shared memory (generated, for stage 0). Same arithmetic as the tiled kernel,
// summed in another order.
constexpr int kGemvRows = 8;
template <int kStage>
__global__ void __launch_bounds__(256) cond_gemv_kernel(const float* __restrict__ levels,
                                                        const float* __restrict__ freqs,
                                                        const float* __restrict__ a_in,
                                                        const float* __restrict__ w, const float* __restrict__ b,
                                                        const float* __restrict__ actions, int action_rows,
                                                        const float* __restrict__ ext_w,
                                                        const float* __restrict__ ext_b, float* __restrict__ out,
                                                        int n) {
  constexpr int K = kStage == 0 ? kFreq : kD;
  __shared__ float As[kGemvRows][K];
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < n * K; i += blockDim.x) {
    const int r = i / K, k = i - r * K;
    if constexpr (kStage == 0) {
      const float arg = levels[r] * freqs[k & 127];
      As[r][k] = k < 128 ? cosf(arg) : sinf(arg);
    } else {
      As[r][k] = a_in[(size_t)r * K + k];
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int c = blockIdx.x * 8 + warp;
    const float* wr = w + (size_t)c * K;
    float acc[kGemvRows];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) acc[r] = 0.f;
    for (int k = lane; k < K; k += 32) {
      const float wv = __ldg(wr + k);
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r)
        if (r < n) acc[r] = fmaf(As[r][k], wv, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    if (lane < n) {
      float v = b[c];
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r)
        if (r == lane) v += acc[r];
      const int r = lane;
      if constexpr (kStage == 0) {
        v = v / (1.f + expf(-v));  // SiLU
      } else if (actions) {
        const float* ar_ = actions + (size_t)(r % action_rows) * kAct;
        const float* we = ext_w + (size_t)c * kAct;
        float e = 0.f;
#pragma unroll
        for (int q = 0; q < kAct; ++q) e = fmaf(ar_[q], we[q], e);
        v += e + ext_b[c];
      }
      out[(size_t)r * kD + c] = v;
    }
  }
}

}  // namespace

int cond_launch(const OasisCondWeights* w, const float* levels, int n, const float* actions, int action_rows,
                float* cond, void* ws, size_t ws_bytes, cudaStream_t st) {
  OASIS_REQUIRE(w && w->t_freqs && w->t_w0 && w->t_b0 && w->t_w2 && w->t_b2, "compute_cond: missing weights");
  OASIS_REQUIRE(n > 0 && levels && cond, "compute_cond: n=%d", n);
  if (actions) {
    OASIS_REQUIRE(action_rows > 0 && w->ext_w && w->ext_b, "compute_cond: actions need action_rows > 0 and ext_w/ext_b");
  }
  const size_t need = (size_t)n * kD * sizeof(float);
  if (!ws || ws_bytes < need)
    return set_error(OASIS_ERR_WORKSPACE, "compute_cond: workspace %zu bytes < %zu", ws_bytes, need);
  float* h = static_cast<float*>(ws);
  if (n <= kGemvRows) {
    launch_pdl(cond_gemv_kernel<0>, dim3(kD / 8), dim3(256), 0, st, levels, w->t_freqs, (const float*)nullptr,
               w->t_w0, w->t_b0, (const float*)nullptr, 1, (const float*)nullptr, (const float*)nullptr, h, n);
    OASIS_TRY(check_launch("cond_gemv_kernel<0>"));
    launch_pdl(cond_gemv_kernel<1>, dim3(kD / 8), dim3(256), 0, st, levels, w->t_freqs, (const float*)h, w->t_w2,
               w->t_b2, actions, action_rows > 0 ? action_rows : 1, w->ext_w, w->ext_b, cond, n);
    return check_launch("cond_gemv_kernel<1>");
  }
  const dim3 grid(kD / TN, (n + TM - 1) / TM);
  launch_pdl(cond_gemm_kernel<0>, grid, dim3(256), 0, st, levels, w->t_freqs, (const float*)nullptr, w->t_w0,
             w->t_b0, (const float*)nullptr, 1, (const float*)nullptr, (const float*)nullptr, h, n);
  OASIS_TRY(check_launch("cond_gemm_kernel<0>"));
  launch_pdl(cond_gemm_kernel<1>, grid, dim3(256), 0, st, levels, w->t_freqs, (const float*)h, w->t_w2, w->t_b2,
             actions, action_rows > 0 ? action_rows : 1, w->ext_w, w->ext_b, cond, n);
  return check_launch("cond_gemm_kernel<1>");
}

}  // namespace oasis

extern "C" size_t oasis_cond_workspace_size(int n) { return n > 0 ? (size_t)n * oasis::kD * sizeof(float) : 0; }

extern "C" int oasis_compute_cond(const OasisCondWeights* w, const float* levels, int n, const float* actions,
                                  int action_rows, float* cond, void* workspace, size_t workspace_bytes,
                                  oasis_stream_t stream) {
  return oasis::cond_launch(w, levels, n, actions, action_rows, cond, workspace, workspace_bytes,
                            reinterpret_cast<cudaStream_t>(stream));
}
