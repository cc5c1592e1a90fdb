// tcgen05 / TMEM / TMA GEMM for sm_100a with fused Oasis epilogues.
//
// C[M,N] = A[M,K] . W[N,K]^T, bf16 operands, fp32 accumulation in tensor memory.
// Every projection on the frame-generation path runs through this kernel:
// adaLN parameters, QKV (+RoPE), O (+bias, gate, residual), FC1 (+bias, GELU),
// FC2 (+bias, gate, residual), VAE QKV/proj/FC1/FC2, and the VAE predictor
// (+bias, unpatchify, clamp).
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and W tiles (128B swizzle) into a STAGES-deep ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: tcgen05.ld the fp32 accumulator, apply the fused op,
//               stage 128-byte rows in swizzled shared memory, TMA bulk store
// Two TMEM accumulators alternate so the epilogue of tile i overlaps the
// mainloop of tile i+1. Optional split-K: partial tiles go to a workspace and the
// last-arriving split (tile counter) sums them in split order (deterministic)
// before running the epilogue.
//
// Waits are bounded (see common.cuh); no TMA multicast is used anywhere.
#include <cudaTypedefs.h>
#include <cstdlib>
#include <mutex>
#include <stdio.h>

#include "common.cuh"
#include "gemm.cuh"
#include "status.h"

namespace oasis {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
#ifndef OASIS_EPI_WARPS
#define OASIS_EPI_WARPS 8
#endif
constexpr int kEpiWarps = OASIS_EPI_WARPS;     // kGroups per TMEM lane quarter
constexpr int kGroups = kEpiWarps / 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer + MMA + epilogue
constexpr int kStgBytes = 32 * 128;          // per-warp store staging: 32 rows x 128 B

// kDeep: the configuration for launches where every CTA has at most one output
// tile (a few hundred rows, e.g. one session). There is no next tile for the
// epilogue to overlap, so the epilogue keeps one staging buffer per warp and the
// shared memory goes to more mainloop stages.
template <int BN, bool kDeep = false>
struct Cfg {
  // Two staging buffers per epilogue warp (the store of one chunk overlaps the
  // next; residual tiles are TMA-loaded into them ahead of time). Measured on
  // B200: worth a pipeline stage even at BN = 256.
  static constexpr int NBUF = (kDeep || kEpiWarps >= 16) ? 1 : 2;
  // Narrow tiles load two 64-wide K atoms per TMA instruction (a stage covers
  // K = 128): the per-instruction cost, not bytes, bounds small-M GEMMs.
  static constexpr int KA = BN <= 128 ? 2 : 1;
  static constexpr int BASE_STAGES = BN == 256 ? 3 : (BN == 128 ? 2 : (BN == 64 ? 3 : 4));
  static constexpr int A_ATOM = BM * BK * 2;  // bytes of one 64-wide K atom of the A tile
  static constexpr int B_ATOM = BN * BK * 2;
  static constexpr int A_BYTES = A_ATOM * KA;
  static constexpr int B_BYTES = B_ATOM * KA;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators; 128/256/512 (power of 2)
  static constexpr int STG_BYTES = kEpiWarps * kStgBytes * NBUF;
  static constexpr int BAR_BYTES = 512;
  // row-statistic exchange of the LN epilogue: [2 row blocks][4 quarters][2 halves][32 rows] float2
  static constexpr int LN_BYTES = BN == 256 ? 2 * 4 * 2 * 32 * 8 : 0;
  static constexpr int DEEP_STAGES = (232448 - 1024 - STG_BYTES - BAR_BYTES - LN_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = kDeep ? (DEEP_STAGES > 6 ? 6 : DEEP_STAGES) : BASE_STAGES;
  static constexpr int SMEM = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES + LN_BYTES;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};


struct SplitK {
  float* partials;  // [tiles][splits][BM][BN]
  int splits;       // CTAs per tile (one cluster), each summing K / splits
};

__host__ __device__ constexpr bool bf16_out(int mode) {
  return mode == kEpiBF16 || mode == kEpiGeluTanhBF16 || mode == kEpiGeluErfBF16 || mode == kEpiRopeBF16;
}
__host__ __device__ constexpr bool gated(int mode) { return mode == kEpiGatedResid || mode == kEpiGatedResidLN; }
__host__ __device__ constexpr bool reads_resid(int mode) { return gated(mode) || mode == kEpiResid; }

// Residual prefetch for one 32-column group of row r (zeros past the last row).
__device__ __forceinline__ void load_resid(const EpiParams& e, int r, int nb, int M, float4 (&res)[8]) {
  if (r < M) {
    const float4* src = reinterpret_cast<const float4*>(e.resid + (long long)r * e.ldr + nb);
#pragma unroll
    for (int i = 0; i < 8; ++i) res[i] = src[i];
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) res[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Applies the epilogue to 32 consecutive accumulator columns [nb, nb + 32) of row r, in place.
// bpre / blane: the bias of these columns spread over the warp's lanes (four
// consecutive columns per lane, starting at lane blane), broadcast by shuffles.
__device__ __forceinline__ void epilogue_math(const EpiParams& e, int r, int nb, float (&v)[32],
                                              const float4 (&res)[8], const float4* gpre = nullptr,
                                              const float4* bpre = nullptr, int blane = 0) {
  if (bpre) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      v[i] += __shfl_sync(0xffffffffu, bpre->x, blane + i / 4);
      v[i + 1] += __shfl_sync(0xffffffffu, bpre->y, blane + i / 4);
      v[i + 2] += __shfl_sync(0xffffffffu, bpre->z, blane + i / 4);
      v[i + 3] += __shfl_sync(0xffffffffu, bpre->w, blane + i / 4);
    }
  } else if (e.bias) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(e.bias + nb + i));
      v[i] += b.x; v[i + 1] += b.y; v[i + 2] += b.z; v[i + 3] += b.w;
    }
  }
  switch (e.mode) {
    case kEpiGeluTanhBF16:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
      break;
    case kEpiGeluErfBF16:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
      break;
    case kEpiRopeBF16:
      if (nb < 2 * e.rope_dim) {
        // pairs (2j, 2j+1) of a 64-wide head rotate by the angle of (pos, pair)
        const int pos = (r / e.rope_div) % e.rope_mod;
        // pair quads q0 .. q0 + 7 of these 32 columns; consecutive rows of a warp
        // read consecutive positions of one quad row
        const float4* tab = reinterpret_cast<const float4*>(e.rope) + (long long)((nb & 63) >> 2) * e.rope_stride + pos;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 cs = __ldg(tab + (long long)j * e.rope_stride);  // (cos, sin) of two consecutive pairs
          const float x0 = v[4 * j], x1 = v[4 * j + 1], x2 = v[4 * j + 2], x3 = v[4 * j + 3];
          v[4 * j] = x0 * cs.x - x1 * cs.y;
          v[4 * j + 1] = x1 * cs.x + x0 * cs.y;
          v[4 * j + 2] = x2 * cs.z - x3 * cs.w;
          v[4 * j + 3] = x3 * cs.z + x2 * cs.w;
        }
      }
      break;
    case kEpiGatedResid:
    case kEpiGatedResidLN:
    case kEpiResid:
      if (gated(e.mode)) {
        const float4* g = reinterpret_cast<const float4*>(e.gate + (long long)(r / e.rows_per_frame) * e.ldg + nb);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 gg = gpre ? gpre[i] : __ldg(g + i);
          v[4 * i] *= gg.x; v[4 * i + 1] *= gg.y; v[4 * i + 2] *= gg.z; v[4 * i + 3] *= gg.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[4 * i] += res[i].x; v[4 * i + 1] += res[i].y; v[4 * i + 2] += res[i].z; v[4 * i + 3] += res[i].w;
      }
      break;
    default:
      break;
  }
}

// VAE predictor: row r = frame * tokens + (hh * grid_w + ww); column n = ch * P*P + p * P + q.
__device__ __forceinline__ void store_image(const EpiParams& e, int r, int nb, int N, const float (&v)[32]) {
  const int P = e.img_patch;
  const int frame = r / e.img_tokens;
  const int tok = r - frame * e.img_tokens;
  const int hh = tok / e.img_grid_w, ww = tok - hh * e.img_grid_w;
  const int grid_h = e.img_tokens / e.img_grid_w;
  const long long H = (long long)grid_h * P, Wd = (long long)e.img_grid_w * P;
  float* img = static_cast<float*>(e.out) + (long long)frame * 3 * H * Wd;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int nn = nb + i;
    if (nn < N) {
      const int ch = nn / (P * P);
      const int rem = nn - ch * P * P;
      const int p = rem / P, q = rem - p * P;
      img[(long long)ch * H * Wd + (long long)(hh * P + p) * Wd + (ww * P + q)] = fminf(1.f, fmaxf(-1.f, v[i]));
    }
  }
}

// The warp's staging tile holds one 32-row x 128-byte box for a TMA store; row
// `lane` belongs to this thread and its 16-byte chunks are XOR-swizzled by
// lane % 8 (TMA's 128-byte swizzle), so the writes are bank-conflict free.
__device__ __forceinline__ void stage_begin(int lane, int nbuf) {
  // the store that last used the buffer about to be written has read it
  if (lane == 0) {
    if (nbuf == 2)
      bulk_wait_read1();
    else
      bulk_wait_read0();
  }
  __syncwarp();
}

// Writes 32 values at 16-byte chunks [j0, j0 + 8 or 4) of this thread's staging row.
__device__ __forceinline__ void stage_write(uint8_t* stg, int lane, bool bf16, int j0, const float (&v)[32]) {
  uint8_t* row = stg + lane * 128;
  if (bf16) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(row + (((j0 + j) ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                     pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) =
          make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                     __float_as_uint(v[4 * j + 3]));
  }
}

__device__ __forceinline__ void stage_commit(const CUtensorMap* tm_out, uint8_t* stg, int lane, int row0, int nb) {
  fence_proxy_async();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tm_out, stg, nb, row0);
    bulk_commit();
  }
}

// Epilogue of one output tile for one warp. A chunk is 128 output bytes per row
// (32 fp32 or 64 bf16 columns), processed as 32-column groups; the warp takes
// chunks c = half, half + 2, ...
__device__ __forceinline__ void epilogue_tile(const EpiParams& e, const SplitK& sk, const CUtensorMap* tm_out,
                                              uint8_t* stg, int nbuf, int& sbuf, uint32_t t_acc, int M, int N,
                                              int BN, int m0q, int n0, int tile, int split, int quarter, int half,
                                              int lane, uint64_t* acc_bar, uint32_t acc_parity, bool& ok,
                                              bool spread_bias = false) {
  const int r = m0q + lane;
  const bool bf16 = bf16_out(e.mode);
  const int W = bf16 ? 64 : 32;
  const int nchunks = BN / W;
  const bool resid = reads_resid(e.mode) && sk.splits == 1;  // fp32 modes: W == 32
  float4 rcur[8];
  if (resid && half < nchunks && n0 + half * W < N) load_resid(e, r, n0 + half * W, M, rcur);
  // spread_bias (single-tile launches, where the epilogue is a serial tail):
  // the bias of this warp's chunks, four columns per lane, read while the
  // accumulator is still being computed (chunk k of the warp: lanes k W/4 ..).
  // Measured slower at large M, where the epilogue overlaps the next tile.
  const int per = W / 4;
  const bool bias_pre = spread_bias && e.bias && sk.splits == 1 && e.mode != kEpiImage;
  float4 bpre = make_float4(0.f, 0.f, 0.f, 0.f);
  if (bias_pre) {
    const int c = half + (lane / per) * kGroups, col = n0 + c * W + (lane % per) * 4;
    if (c < nchunks && col < N) bpre = __ldg(reinterpret_cast<const float4*>(e.bias + col));
  }
  bool acc_ready;
  {
    acc_ready = mbar_wait(acc_bar, acc_parity, kDevTimeoutAccFull);
  }
  if (!acc_ready) {
    ok = false;
    return;
  }
  tc_fence_after();
  float* part = nullptr;
  if (sk.splits > 1) part = sk.partials + ((long long)tile * sk.splits + split) * (BM * BN) + (quarter * 32 + lane) * BN;
#pragma unroll 1
  for (int c = half; c < nchunks; c += kGroups) {
    const int nb = n0 + c * W;
    if (sk.splits == 1 && nb >= N) break;  // warp-uniform
    float4 rnext[8];
    if (resid && c + kGroups < nchunks && nb + kGroups * W < N) load_resid(e, r, nb + kGroups * W, M, rnext);
    uint8_t* buf = stg + sbuf * kStgBytes;
    if (sk.splits == 1 && e.mode != kEpiImage) stage_begin(lane, nbuf);
#pragma unroll 1
    for (int g = 0; g < W / 32; ++g) {
      float v[32];
      __syncwarp();
      tmem_ld32(t_acc + c * W + g * 32, v);
      if (sk.splits > 1) {
        float4* dst = reinterpret_cast<float4*>(part + c * W + g * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) __stcg(dst + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
      } else {
        epilogue_math(e, r, nb + g * 32, v, rcur, nullptr, bias_pre ? &bpre : nullptr,
                      ((c - half) / kGroups) * per + g * 8);
        if (e.mode == kEpiImage) {
          if (r < M) store_image(e, r, nb, N, v);
        } else {
          stage_write(buf, lane, bf16, g * 4, v);
        }
      }
    }
    if (sk.splits == 1) {
      if (e.mode != kEpiImage) {
        stage_commit(tm_out, buf, lane, m0q, nb);
        if (nbuf == 2) sbuf ^= 1;
      }
      if (resid) {
#pragma unroll
        for (int i = 0; i < 8; ++i) rcur[i] = rnext[i];
      }
    }
  }
}

// Epilogue of a residual tile (fp32 in and out, no split-K): the warp's 32-column
// residual boxes are TMA-loaded into its two staging buffers (the first two before
// the accumulator is ready, later ones as soon as a buffer's store has read it),
// the result is computed in place and TMA-stored from the same buffer.
__device__ __forceinline__ void epilogue_tile_resid(const EpiParams& e, const CUtensorMap* tm_out,
                                                    const CUtensorMap* tm_res, uint8_t* stg, int nbuf, uint64_t* rbar,
                                                    uint32_t& rphase, uint32_t t_acc, int M, int N, int BN, int m0q,
                                                    int n0, int half, int lane, uint64_t* acc_bar,
                                                    uint32_t acc_parity, bool& ok, float* stats = nullptr,
                                                    bool early = false) {
  const int r = m0q + lane;
  const int nchunks = BN / 32;
  int mine = 0;  // this warp's chunks: c = half + kGroups i, i < mine
  while (half + kGroups * mine < nchunks && n0 + (half + kGroups * mine) * 32 < N) ++mine;
  // early (single-tile launches, where the epilogue is a serial tail): the first
  // chunk's gate row and the warp's bias (four columns per lane, broadcast by
  // shuffles) are read before the accumulator wait
  float4 gate[8];
  auto load_gate = [&](int nb) {
    const float4* g = reinterpret_cast<const float4*>(e.gate + (long long)((r < M ? r : M - 1) / e.rows_per_frame) * e.ldg + nb);
#pragma unroll
    for (int j = 0; j < 8; ++j) gate[j] = __ldg(g + j);
  };
  const bool bias_pre = early && e.bias;
  float4 bpre = make_float4(0.f, 0.f, 0.f, 0.f);
  if (early) {
    if (gated(e.mode) && mine > 0) load_gate(n0 + half * 32);
    const int c = half + (lane >> 3) * kGroups, col = n0 + c * 32 + (lane & 7) * 4;
    if (bias_pre && c < nchunks && col < N) bpre = __ldg(reinterpret_cast<const float4*>(e.bias + col));
  }
  if (lane == 0) {
    bulk_wait_read0();  // earlier stores no longer read the buffers
    for (int i = 0; i < nbuf && i < mine; ++i) {
      mbar_arrive_expect_tx(&rbar[i], kStgBytes);
      tma_load_2d(stg + i * kStgBytes, tm_res, &rbar[i], n0 + (half + kGroups * i) * 32, m0q);
    }
  }
  __syncwarp();
  bool acc_ready;
  {
    acc_ready = mbar_wait(acc_bar, acc_parity, kDevTimeoutAccFull);
  }
  if (!acc_ready) {
    ok = false;
    return;
  }
  tc_fence_after();
#pragma unroll 1
  for (int i = 0; i < mine; ++i) {
    const int b = i % nbuf;
    const int c = half + kGroups * i;
    const int nb = n0 + c * 32;
    uint8_t* buf = stg + b * kStgBytes;
    // issued before the waits so its latency overlaps them
    if (gated(e.mode) && !(early && i == 0)) load_gate(nb);
    if (!mbar_wait(&rbar[b], (rphase >> b) & 1, kDevTimeoutAccFull)) {
      ok = false;
      return;
    }
    rphase ^= 1u << b;
    float v[32];
    __syncwarp();
    tmem_ld32(t_acc + c * 32, v);
    uint8_t* row = buf + lane * 128;
    float4 res[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) res[j] = *reinterpret_cast<const float4*>(row + ((j ^ (lane & 7)) << 4));
    epilogue_math(e, r, nb, v, res, gated(e.mode) ? gate : nullptr, bias_pre ? &bpre : nullptr, i * 8);
    if (stats) {  // row statistics of the new values: chunk mean / M2, then Chan's combination
      float cm = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) cm += v[j];
      cm *= (1.f / 32.f);
      float c2 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) c2 = fmaf(v[j] - cm, v[j] - cm, c2);
      const float na = stats[0], nn = na + 32.f, d = cm - stats[1];
      stats[1] += d * (32.f / nn);
      stats[2] += c2 + d * d * (na * 32.f / nn);
      stats[0] = nn;
    }
    stage_write(buf, lane, false, 0, v);
    stage_commit(tm_out, buf, lane, m0q, nb);
    if (i + nbuf < mine) {  // refill this buffer with chunk i + nbuf once the store has read it
      if (lane == 0) {
        bulk_wait_read0();
        mbar_arrive_expect_tx(&rbar[b], kStgBytes);
        tma_load_2d(buf, tm_res, &rbar[b], n0 + (c + nbuf * kGroups) * 32, m0q);
      }
      __syncwarp();
    }
  }
}

// LayerNorm pass of the kEpiGatedResidLN epilogue, run by each epilogue warp once
// all n-tiles of its 128-row block are written: half `half` of the lane quarter
// normalises columns [half 512, half 512 + 512) of its 32 rows in 64-column
// chunks (two 32-column fp32 boxes of the new z TMA-loaded into the staging
// buffers, bf16 result stored from the first one with the xn tensor map).
__device__ __forceinline__ bool ln_pass(const EpiParams& e, const LnParams& ln, const CUtensorMap* tm_z,
                                       const CUtensorMap* tm_x,
                                       uint8_t* stg, uint64_t* rbar, uint32_t& rphase, int M, int m0q, int half,
                                       int lane, float mean, float rstd) {
  const int r = m0q + lane;
  const long long frame = (long long)((r < M ? r : M - 1) / e.rows_per_frame);
  const float* mul = ln.mod + frame * ln.ld_mod + ln.scale_off;
  const float* add = ln.mod + frame * ln.ld_mod + ln.shift_off;
#pragma unroll 1
  for (int ch = 0; ch < 8; ++ch) {
    const int c0 = half * 512 + ch * 64;
    if (lane == 0) {
      bulk_wait_read0();  // the previous chunk's store has read the staging buffer
      for (int b = 0; b < 2; ++b) {
        mbar_arrive_expect_tx(&rbar[b], kStgBytes);
        tma_load_2d(stg + b * kStgBytes, tm_z, &rbar[b], c0 + b * 32, m0q);
      }
    }
    __syncwarp();
    float v[2][32];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      if (!mbar_wait(&rbar[b], (rphase >> b) & 1, kDevTimeoutAccFull)) return false;
      rphase ^= 1u << b;
      const uint8_t* row = stg + b * kStgBytes + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = *reinterpret_cast<const float4*>(row + ((j ^ (lane & 7)) << 4));
        const int c = c0 + b * 32 + 4 * j;
        const float4 mm = __ldg(reinterpret_cast<const float4*>(mul + c));
        const float4 aa = __ldg(reinterpret_cast<const float4*>(add + c));
        v[b][4 * j] = (x.x - mean) * rstd * mm.x + aa.x;
        v[b][4 * j + 1] = (x.y - mean) * rstd * mm.y + aa.y;
        v[b][4 * j + 2] = (x.z - mean) * rstd * mm.z + aa.z;
        v[b][4 * j + 3] = (x.w - mean) * rstd * mm.w + aa.w;
      }
    }
    __syncwarp();  // both buffers read before the first is overwritten
    stage_write(stg, lane, true, 0, v[0]);
    stage_write(stg, lane, true, 4, v[1]);
    stage_commit(tm_x, stg, lane, m0q, c0);
  }
  return true;
}

// Split-K fix-up. The `splits` CTAs of a tile form one thread-block cluster;
// after every CTA has written its fp32 partial tile and the cluster barrier has
// passed, CTA `split` sums rows [split BM / splits, (split + 1) BM / splits) of
// the tile over the partials in split order (deterministic) and applies the
// epilogue. `tid` / `nthr` enumerate the threads taking part.
__device__ __forceinline__ void splitk_cluster_reduce(const EpiParams& e, const SplitK& sk, int M, int N, int BN,
                                                      int m0, int n0, int tile, int split, int tid, int nthr) {
  const int rows = BM / sk.splits;
  const int groups = BN / 32;
  const bool bf16 = bf16_out(e.mode);
  const float* base = sk.partials + (long long)tile * sk.splits * (BM * BN);
  for (int it = tid; it < rows * groups; it += nthr) {
    const int lr = split * rows + it / groups;  // row within the tile
    const int g = it - (it / groups) * groups;
    const int r = m0 + lr, nb = n0 + g * 32;
    if (r >= M || nb >= N) continue;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    for (int s2 = 0; s2 < sk.splits; ++s2) {
      const float4* src = reinterpret_cast<const float4*>(base + (long long)s2 * (BM * BN) + lr * BN + g * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 y = __ldcg(src + i);
        v[4 * i] += y.x; v[4 * i + 1] += y.y; v[4 * i + 2] += y.z; v[4 * i + 3] += y.w;
      }
    }
    float4 res[8];
    if (reads_resid(e.mode)) load_resid(e, r, nb, M, res);
    epilogue_math(e, r, nb, v, res);
    if (e.mode == kEpiImage) {
      store_image(e, r, nb, N, v);
    } else if (nb + 32 <= N) {
      if (bf16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(e.out) + (long long)r * e.ldo + nb);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                              pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
      } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(e.out) + (long long)r * e.ldo + nb);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
    } else {  // ragged last column group (N is a multiple of 16)
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (nb + i < N) {
          if (bf16)
            static_cast<__nv_bfloat16*>(e.out)[(long long)r * e.ldo + nb + i] = __float2bfloat16(v[i]);
          else
            static_cast<float*>(e.out)[(long long)r * e.ldo + nb + i] = v[i];
        }
      }
    }
  }
}

// The k-th unit (tile x split index) this CTA processes, or -1 when none is left.
// The LN-fused epilogue takes whole 128-row blocks instead: m-blocks blockIdx.x,
// + gridDim.x, ..., each with all its n-tiles, so that one CTA writes every
// column of its rows.
__device__ __forceinline__ int unit_at(int k, bool row_blocks, int units, int n_tiles, int m_tiles) {
  if (!row_blocks) {
    const int u = blockIdx.x + k * gridDim.x;
    return u < units ? u : -1;
  }
  // n-tiles in a rotated order (starting at blockIdx.x % n_tiles) so that the
  // CTAs do not all stream the same weight slice at the same time
  const int mb = blockIdx.x + (k / n_tiles) * gridDim.x;
  return mb < m_tiles ? mb * n_tiles + (k + blockIdx.x) % n_tiles : -1;
}

// kLN: the kEpiGatedResidLN instantiation (whole-row blocks, row statistics and
// the LayerNorm pass); kept separate so the other epilogues' register budget is
// not shared with it.
template <int BN, bool kLN, bool kDeep = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                const __grid_constant__ CUtensorMap tmX, const int M,
                const int N, const int K,
                const EpiParams epi, const SplitK sk, const LnParams lnp) {
  using C = Cfg<BN, kDeep>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(tmem_base_slot + 4);  // [kEpiWarps][2], 8-byte aligned
  float2* lnx = reinterpret_cast<float2*>(full + C::BAR_BYTES / 8);   // LN_BYTES: (mean, M2) per row half

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();

  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int splits = sk.splits;
  const int units = m_tiles * n_tiles * splits;
  const int kb_total = K / (BK * C::KA);  // stages of K
  const int kb_per_split = kb_total / splits;  // host guarantees divisibility
  constexpr bool row_blocks = kLN;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    if (epi.mode != kEpiImage) prefetch_tmap(&tmO);
    if (reads_resid(epi.mode)) prefetch_tmap(&tmR);
    if (row_blocks) prefetch_tmap(&tmX);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  if (warp != 0) pdl_wait();  // the producer waits after prefetching weights

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // stage kb covers K atoms [kb KA, kb KA + KA)
    auto load_a = [&](void* dst, uint64_t* bar, int kb, int m0) {
      if constexpr (C::KA == 1) tma_load_2d(dst, &tmA, bar, kb * BK, m0);
      else tma_load_3d(dst, &tmA, bar, 0, m0, kb * C::KA);
    };
    auto load_w = [&](void* dst, uint64_t* bar, int kb, int n0) {
      if constexpr (C::KA == 1) tma_load_2d(dst, &tmW, bar, kb * BK, n0);
      else tma_load_3d(dst, &tmW, bar, 0, n0, kb * C::KA);
    };
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Weights are never written by an earlier kernel: start streaming the first
      // stages' W tiles before waiting for the upstream kernel (programmatic
      // dependent launch), then add the A tiles once its output is visible.
      int pre = 0;
      const int u_first = unit_at(0, row_blocks, units, n_tiles, m_tiles);
      if (u_first >= 0) {
        const int tile = u_first / splits, split = u_first - tile * splits;
        const int n0 = (tile % n_tiles) * BN, kb0 = split * kb_per_split;
        pre = kb_per_split < C::STAGES ? kb_per_split : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          load_w(smem + i * C::STAGE_BYTES + C::A_BYTES, &full[i], kb0 + i, n0);
        }
      }
      pdl_wait();
      for (int k = 0, u; ok && (u = unit_at(k, row_blocks, units, n_tiles, m_tiles)) >= 0; ++k) {
        const int tile = u / splits, split = u - tile * splits;
        const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
        const int kb0 = split * kb_per_split;
        for (int kb = kb0; kb < kb0 + kb_per_split; ++kb) {
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          if (k == 0 && kb - kb0 < pre) {
            load_a(sa, &full[stage], kb, m0);  // W already in flight
          } else {
            bool got;
            got = mbar_wait(&empty[stage], phase ^ 1, kDevTimeoutSmemEmpty);
            if (!got) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            load_a(sa, &full[stage], kb, m0);
            load_w(sa + C::A_BYTES, &full[stage], kb, n0);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int k = 0; ok && unit_at(k, row_blocks, units, n_tiles, m_tiles) >= 0; ++k) {
        bool got;
        got = mbar_wait(&acc_empty[acc], acc_phase ^ 1, kDevTimeoutAccEmpty);
        if (!got) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kb_per_split; ++kb) {
          got = mbar_wait(&full[stage], phase, kDevTimeoutTmaFull);
          if (!got) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
#pragma unroll
          for (int at = 0; at < C::KA; ++at) {
            const uint64_t adesc = smem_desc_sw128(a_addr + at * C::A_ATOM);
            const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES + at * C::B_ATOM);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              // +32 bytes per 16-element K step inside the 128-byte swizzle atom
              tc_mma_bf16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                          (kb > 0 || at > 0 || k > 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        tc_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..9) ----------------
    // Warp w reads TMEM lanes [32 (w % 4), +32) - the rows it may access - and
    // every other chunk of 128 output bytes per row (half = (w - 2) / 4). Each
    // thread owns one row; results leave through a swizzled staging tile and a
    // TMA bulk store, residual inputs are prefetched a chunk ahead.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* stg = staging + (warp - 2) * kStgBytes * C::NBUF;
    uint64_t* my_rbar = rbar + 2 * (warp - 2);
    const bool resid_tma = reads_resid(epi.mode) && splits == 1;
    int sbuf = 0;
    uint32_t rphase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    float stats[3] = {0.f, 0.f, 0.f};  // LN epilogue: this thread's row (count, mean, M2) so far
    int mblk = 0;
    for (int k = 0, u; ok && (u = unit_at(k, row_blocks, units, n_tiles, m_tiles)) >= 0; ++k) {
      const int tile = u / splits, split = u - tile * splits;
      const int m0q = (tile / n_tiles) * BM + quarter * 32, n0 = (tile % n_tiles) * BN;
      const uint32_t t_acc = tmem_base + lane_off + acc * BN;
      if (resid_tma)
        epilogue_tile_resid(epi, &tmO, &tmR, stg, C::NBUF, my_rbar, rphase, t_acc, M, N, BN, m0q, n0, half, lane,
                            &acc_full[acc], acc_phase, ok, kLN ? stats : nullptr, kDeep && BN == 32);
      else
        epilogue_tile(epi, sk, &tmO, stg, C::NBUF, sbuf, t_acc, M, N, BN, m0q, n0, tile, split, quarter, half,
                      lane, &acc_full[acc], acc_phase, ok, kDeep);
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if constexpr (kLN && C::LN_BYTES > 0) {
        if (k % n_tiles == n_tiles - 1) {  // the row block's last tile in this CTA's order
          // every column of these rows is written: combine the two halves' row
          // statistics (512 columns each) and normalise into the LN output
          if (lane == 0) bulk_wait0();  // this warp's z stores have completed
          __syncwarp();
          float2* slot = lnx + (mblk & 1) * 256 + quarter * 64;
          slot[half * 32 + lane] = make_float2(stats[1], stats[2]);
          named_barrier_sync(1 + quarter, 64);
          const float2 o = slot[(half ^ 1) * 32 + lane];
          const float d = stats[1] - o.x;
          const float mean = 0.5f * (stats[1] + o.x);
          const float m2 = stats[2] + o.y + d * d * 256.f;  // n_a n_b / n = 512 x 512 / 1024
          const float rstd = rsqrtf(m2 * (1.f / 1024.f) + lnp.eps);
          if (!ln_pass(epi, lnp, &tmR, &tmX, stg, my_rbar, rphase, M, m0q, half, lane, mean, rstd)) {
            ok = false;
            break;
          }
          stats[0] = stats[1] = stats[2] = 0.f;
          ++mblk;
        }
      }
    }
    if (lane == 0) bulk_wait0();  // stores complete before the staging memory goes away
  }

  if (splits > 1) {
    // one unit per CTA here (grid = tiles x splits, clusters of `splits`): once
    // every CTA of the cluster has written its partial, reduce this CTA's rows
    __threadfence();
    cluster_sync_all();
    const int tile = blockIdx.x / splits, split = blockIdx.x - tile * splits;
    splitk_cluster_reduce(epi, sk, M, N, BN, (tile / n_tiles) * BM, (tile % n_tiles) * BN, tile, split,
                          threadIdx.x, blockDim.x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// CTA-pair GEMM: 256 x 256 output tiles, one 2-CTA cluster per tile.
// ---------------------------------------------------------------------------
// Each CTA of the pair stages its own 128 rows of A and its own 128 rows of W
// (so a pair reads A and W once per 256 x 256 tile: a third less L2 -> shared
// traffic per FLOP than a 128 x 256 tile per CTA). The leader (rank 0) issues
// cta_group::2 MMAs of M = 256, N = 256 that read both CTAs' shared memory and
// accumulate into both CTAs' TMEM (rank r holds rows [128 r, 128 r + 128) of the
// tile). TMA completion of both CTAs' loads counts on the leader's `full`
// barrier; the MMA commit arrives on the `empty` and `acc_full` barriers of both
// CTAs; both CTAs' epilogue warps release an accumulator on the leader's
// `acc_empty`. No TMA multicast. Every wait is bounded as in gemm_kernel.
struct PairCfg {
  static constexpr int BNP = 256;                 // output columns per tile
  static constexpr int A_BYTES = BM * BK * 2;     // this CTA's 128 A rows x 64 K
  static constexpr int B_BYTES = 128 * BK * 2;    // this CTA's 128 W rows x 64 K
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 5;
  static constexpr int NBUF = 2;
  static constexpr int TMEM_COLS = 2 * BNP;       // two accumulators
  static constexpr int STG_BYTES = kEpiWarps * kStgBytes * NBUF;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(2 * STAGES + 4 + 2 * kEpiWarps + 2 <= BAR_BYTES / 8, "barrier area");
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, const int M,
                     const int N, const int K, const EpiParams epi) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(tmem_base_slot + 4);  // [kEpiWarps][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  pdl_trigger();

  const int m_tiles = (M + 2 * BM - 1) / (2 * BM);
  const int n_tiles = (N + C::BNP - 1) / C::BNP;
  const int units = m_tiles * n_tiles;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int kb_total = K / BK;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmO);
    if (reads_resid(epi.mode)) prefetch_tmap(&tmR);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // both CTAs' epilogue warps (used on the leader)
    }
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // barriers initialised and TMEM allocated in both CTAs before either uses the other's
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  if (warp != 0) pdl_wait();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int pre = 0;
      // W is never written by an earlier kernel: start its first stages before
      // waiting for the upstream kernel, then add the A tiles
      if (pair < units) {
        const int n0 = (pair % n_tiles) * C::BNP + (int)rank * 128;
        pre = kb_total < C::STAGES ? kb_total : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          if (leader) mbar_arrive_expect_tx(&full[i], 2 * C::STAGE_BYTES);
          tma_load_2d_pair(smem + i * C::STAGE_BYTES + C::A_BYTES, &tmW, mapa_shared(smem_u32(&full[i]), 0),
                           i * BK, n0);
        }
      }
      pdl_wait();
      for (int k = 0, u = pair; ok && u < units; ++k, u += pairs) {
        const int m0 = (u / n_tiles) * 2 * BM + (int)rank * BM;
        const int n0 = (u % n_tiles) * C::BNP + (int)rank * 128;
        for (int kb = 0; kb < kb_total; ++kb) {
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (k == 0 && kb < pre) {
            tma_load_2d_pair(sa, &tmA, bar, kb * BK, m0);  // W already in flight
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, kDevTimeoutSmemEmpty)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            tma_load_2d_pair(sa, &tmA, bar, kb * BK, m0);
            tma_load_2d_pair(sa + C::A_BYTES, &tmW, bar, kb * BK, n0);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * BM, C::BNP);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; ok && u < units; u += pairs) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BNP;
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&full[stage], phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint64_t adesc = smem_desc_sw128(a_addr);
          const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_bf16_pair(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                             (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..9, both CTAs) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* stg = staging + (warp - 2) * kStgBytes * C::NBUF;
    uint64_t* my_rbar = rbar + 2 * (warp - 2);
    const bool resid_tma = reads_resid(epi.mode);
    const SplitK nosplit{nullptr, 1};
    int sbuf = 0;
    uint32_t rphase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = pair; ok && u < units; u += pairs) {
      const int m0q = (u / n_tiles) * 2 * BM + (int)rank * BM + quarter * 32, n0 = (u % n_tiles) * C::BNP;
      const uint32_t t_acc = tmem_base + lane_off + acc * C::BNP;
      if (resid_tma)
        epilogue_tile_resid(epi, &tmO, &tmR, stg, C::NBUF, my_rbar, rphase, t_acc, M, N, C::BNP, m0q, n0, half, lane,
                            &acc_full[acc], acc_phase, ok);
      else
        epilogue_tile(epi, nosplit, &tmO, stg, C::NBUF, sbuf, t_acc, M, N, C::BNP, m0q, n0, u, 0, quarter, half,
                      lane, &acc_full[acc], acc_phase, ok);
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait0();  // stores complete before the staging memory goes away
  }

  // neither CTA frees TMEM or exits while the other may still signal its barriers
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  return OASIS_OK;
}

// K-major bf16 tile map: dims {K, rows}, box {64, box_rows}, 128-byte swizzle, OOB -> 0.
int make_map(CUtensorMap* map, const void* ptr, long long rows, long long K, long long ld, int box_rows,
             int atoms = 1) {
  OASIS_TRY(get_encoder());
  OASIS_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "GEMM operand not 16-byte aligned");
  OASIS_REQUIRE((ld * 2) % 16 == 0, "GEMM operand row stride not a multiple of 16 bytes");
  CUresult r;
  if (atoms == 1) {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // {64, rows, K / 64} view: one box = `atoms` consecutive 64-wide K atoms of
    // box_rows rows, laid out atom after atom (each atom the 128B-swizzled tile).
    cuuint64_t dims[3] = {(cuuint64_t)BK, (cuuint64_t)rows, (cuuint64_t)(K / BK)};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(BK * 2)};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)atoms};
    cuuint32_t estr[3] = {1, 1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return set_error(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OASIS_OK;
}

// Output store map: dims {N, M}, box {128 bytes of columns, 32 rows}, 128-byte swizzle.
int make_out_map(CUtensorMap* map, void* ptr, long long M, long long N, long long ld, bool bf16) {
  OASIS_TRY(get_encoder());
  const int es = bf16 ? 2 : 4;
  OASIS_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "GEMM output not 16-byte aligned");
  OASIS_REQUIRE((ld * es) % 16 == 0, "GEMM output row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return OASIS_OK;
}

std::atomic<int> g_num_sms[64];  // per device, zero until first queried

template <int BN, bool kLN, bool kDeep = false>
int launch_bn(const GemmProblem& p, int splits, cudaStream_t stream) {
  using C = Cfg<BN, kDeep>;
  static std::atomic<bool> attr_set[64];  // per device; host threads may launch concurrently
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, kLN, kDeep>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta, tw, to, tr;
  OASIS_TRY(make_map(&ta, p.A, p.M, p.K, p.lda, BM, C::KA));
  OASIS_TRY(make_map(&tw, p.W, p.N, p.K, p.K, BN, C::KA));
  if (p.epi.mode == kEpiImage)
    to = ta;  // unused: the image epilogue scatters directly
  else
    OASIS_TRY(make_out_map(&to, p.epi.out, p.M, p.N, p.epi.ldo, bf16_out(p.epi.mode)));
  if (reads_resid(p.epi.mode))
    OASIS_TRY(make_out_map(&tr, const_cast<float*>(p.epi.resid), p.M, p.N, p.epi.ldr, false));  // same box as the output
  else
    tr = to;
  CUtensorMap tx = to;
  if (p.epi.mode == kEpiGatedResidLN) OASIS_TRY(make_out_map(&tx, p.ln.out, p.M, p.N, p.N, true));
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  SplitK sk{nullptr, splits};
  if (splits > 1) {
    const size_t need = (size_t)tiles * splits * BM * BN * sizeof(float);
    if (!p.workspace || p.workspace_bytes < need)
      return set_error(OASIS_ERR_WORKSPACE, "split-K GEMM needs %zu workspace bytes, got %zu", need,
                       p.workspace_bytes);
    sk.partials = static_cast<float*>(p.workspace);
    // one CTA per (tile, split); the splits of a tile are one cluster
    launch_pdl_cluster(gemm_kernel<BN, kLN, kDeep>, dim3(tiles * splits), dim3(kThreads), C::SMEM, stream, splits, ta, tw, to,
                       tr, tx, p.M, p.N, p.K, p.epi, sk, p.ln);
    return check_launch("gemm_kernel");
  }
  const int work = p.epi.mode == kEpiGatedResidLN ? (p.M + BM - 1) / BM : tiles;  // row blocks or tiles
  const int grid = work < grid_sms() ? work : grid_sms();
  launch_pdl(gemm_kernel<BN, kLN, kDeep>, dim3(grid), dim3(kThreads), C::SMEM, stream, ta, tw, to, tr, tx, p.M, p.N, p.K, p.epi,
             sk, p.ln);
  return check_launch("gemm_kernel");
}

// 256 x 256 tiles on CTA pairs (gemm_pair_kernel); no split-K, no LN epilogue.
int launch_pair(const GemmProblem& p, cudaStream_t stream) {
  using C = PairCfg;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta, tw, to, tr;
  OASIS_TRY(make_map(&ta, p.A, p.M, p.K, p.lda, BM, 1));
  OASIS_TRY(make_map(&tw, p.W, p.N, p.K, p.K, 128, 1));
  OASIS_TRY(make_out_map(&to, p.epi.out, p.M, p.N, p.epi.ldo, bf16_out(p.epi.mode)));
  if (reads_resid(p.epi.mode))
    OASIS_TRY(make_out_map(&tr, const_cast<float*>(p.epi.resid), p.M, p.N, p.epi.ldr, false));
  else
    tr = to;
  const int units = ((p.M + 2 * BM - 1) / (2 * BM)) * ((p.N + C::BNP - 1) / C::BNP);
  const int max_pairs = grid_sms() / 2;
  const int pairs = units < max_pairs ? units : max_pairs;
  launch_pdl_cluster(gemm_pair_kernel, dim3(2 * pairs), dim3(kThreads), C::SMEM, stream, 2, ta, tw, to, tr, p.M, p.N,
                     p.K, p.epi);
  return check_launch("gemm_pair_kernel");
}

// Which large GEMMs run on CTA pairs. Isolated launches at C4 shapes (TFLOP/s,
// single 128 x 256 tiles -> pairs): FC2 1158 -> 1370-1445, O ~860 -> 830-905,
// FC1 ~1100-1200 either way, QKV 1107 -> 1038-1110; the whole C4 frame, per MHz
// of SM clock under the power cap: no pairs 0.139 frames/s/MHz, pairs for the
// fp32 residual epilogues only 0.148, pairs everywhere 0.153-0.155 (the lower
// L2 -> shared traffic buys clock). Default: every eligible GEMM.
// OASIS_GEMM_PAIR=0: never; =resid: the residual epilogues only.
enum PairMode { kPairOff = 0, kPairResid = 1, kPairAll = 2 };
int pair_mode() {
  static const int m = [] {
    const char* e = getenv("OASIS_GEMM_PAIR");
    if (e && e[0] == '0') return (int)kPairOff;
    if (e && e[0] == 'r') return (int)kPairResid;
    return (int)kPairAll;
  }();
  return m;
}

// The deep-pipeline configuration for single-wave launches (OASIS_GEMM_DEEP=0:
// never). Measured on one session at T = 2 (three A/B pairs): C3 frame 8.515 ->
// 8.235 ms, C2 step 1.918 -> 1.850 ms.
bool deep_enabled() {
  static const bool on = [] {
    const char* e = getenv("OASIS_GEMM_DEEP");
    return !(e && e[0] == '0');
  }();
  return on;
}

struct Plan {
  int bn;
  int splits;
  bool pair;  // 256 x 256 tiles on a CTA pair
};

Plan choose_plan(int M, int N, int K) {
  const int sms = num_sms();
  const int mt = (M + BM - 1) / BM;
  const int t256 = mt * ((N + 255) / 256);
  if (t256 >= sms && N % 256 == 0) return {256, 1, false};
  const int t128 = mt * ((N + 127) / 128);
  if (t128 >= sms) return {128, 1, false};
  // Small problems (a handful of sessions): narrow tiles so most SMs stream a
  // slice of the weights. A long K over at most three row tiles (the B = 1 FC2,
  // M = 288, K = 4096) runs as 128-wide tiles x 4 K splits, one cluster per tile
  // (measured 17.2 -> 15.0 us); elsewhere at M = 288-576 split-K measured slower.
  if (mt <= 3 && K >= 4096 && N <= 1024 && (K / 128) % 4 == 0 && mt * ((N + 127) / 128) * 4 <= sms)
    return {128, 4, false};
  return {t128 >= sms / 2 ? 128 : 64, 1, false};
}

// The final tile plan of a problem: heuristic choice, the caller's overrides and
// every rule the launch applies on top. gemm_launch dispatches on it and the
// workspace queries size from it, so the two cannot disagree.
int resolve_plan(const GemmProblem& p, Plan* out) {
  Plan pl = choose_plan(p.M, p.N, p.K);
  pl.pair = false;
  // fp32-output epilogues (32-column chunks) can use 32-wide tiles: at a few
  // hundred rows and N = 1024 that doubles the SMs streaming the weights.
  if (pl.bn == 64 && !bf16_out(p.epi.mode) && p.epi.mode != kEpiImage &&
      ((p.M + BM - 1) / BM) * ((p.N + 63) / 64) < num_sms() / 2)
    pl.bn = 32;
  if (p.block_n == 512) {  // explicit request: 256 x 256 tiles on a CTA pair
    OASIS_REQUIRE(p.splits <= 1 && p.epi.mode != kEpiImage && p.epi.mode != kEpiGatedResidLN,
                  "GEMM: CTA-pair tiles take no split-K, image or LN epilogue");
    *out = Plan{256, 1, true};
    return OASIS_OK;
  }
  if (p.block_n) pl.bn = p.block_n;
  if (p.splits) pl.splits = p.splits;
  if (pl.splits > 1 && !p.workspace) pl.splits = 1;
  if (p.epi.mode == kEpiGatedResidLN) {  // whole rows per CTA, 4 tiles of 256
    pl.bn = 256;
    pl.splits = 1;
  }
  OASIS_REQUIRE(pl.bn != 32 || !bf16_out(p.epi.mode), "GEMM: block_n=32 needs an fp32 epilogue");
  if (pl.bn <= 128 && p.K % (2 * BK)) pl.bn = 256;  // narrower tiles stage K in 128-wide steps
  const int k_stages = p.K / (pl.bn <= 128 ? 2 * BK : BK);
  OASIS_REQUIRE(pl.splits >= 1 && pl.splits <= 8, "GEMM: splits=%d outside [1, 8] (one cluster per tile)", pl.splits);
  OASIS_REQUIRE(k_stages % pl.splits == 0, "GEMM: splits=%d must divide the %d K stages", pl.splits, k_stages);
  // Large problems: 256 x 256 tiles on CTA pairs, when there are enough of them
  // to fill the GPU (one pair per two SMs).
  const int pm = pair_mode();
  pl.pair = !p.block_n && pl.bn == 256 && pl.splits == 1 && pm != kPairOff && p.epi.mode != kEpiImage &&
            p.epi.mode != kEpiGatedResidLN && (pm == kPairAll || reads_resid(p.epi.mode)) && p.N % 256 == 0 &&
            p.M >= 2 * BM &&  // a pair's second CTA would hold no rows (M = 8 adaLN rows: 104.7 -> 88.1 us)
            ((p.M + 2 * BM - 1) / (2 * BM)) * (p.N / 256) >= num_sms() / 2;
  *out = pl;
  return OASIS_OK;
}

size_t plan_splitk_bytes(int M, int N, const Plan& pl) {
  if (pl.pair || pl.splits <= 1) return 0;
  const size_t tiles = (size_t)((M + BM - 1) / BM) * ((N + pl.bn - 1) / pl.bn);
  return tiles * pl.splits * BM * pl.bn * sizeof(float);
}

}  // namespace

thread_local int t_sm_reserve = 0;

void set_sm_reserve(int n) { t_sm_reserve = n > 0 ? n : 0; }

int grid_sms() {
  const int n = num_sms() - t_sm_reserve;
  return n >= 2 ? n : 2;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (g_num_sms[dev & 63] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev & 63] = n > 0 ? n : 148;
  }
  return g_num_sms[dev & 63];
}

int gemm_plan(int M, int N, int K, int mode, int block_n, int splits, int* bn, int* splits_out, int* pair,
              size_t* splitk_bytes) {
  OASIS_REQUIRE(M > 0 && N > 0 && K > 0 && K % BK == 0, "GEMM plan: bad shape %d x %d x %d", M, N, K);
  GemmProblem p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.epi.mode = mode;
  p.block_n = block_n;
  p.splits = splits;
  p.workspace = reinterpret_cast<void*>(uintptr_t(256));  // "a workspace is given": split-K stays allowed
  Plan pl;
  OASIS_TRY(resolve_plan(p, &pl));
  if (bn) *bn = pl.pair ? 512 : pl.bn;
  if (splits_out) *splits_out = pl.splits;
  if (pair) *pair = pl.pair ? 1 : 0;
  if (splitk_bytes) *splitk_bytes = plan_splitk_bytes(M, N, pl);
  return OASIS_OK;
}

size_t gemm_workspace_bytes(int M, int N, int K) {
  size_t b = 0;
  if (M <= 0 || N <= 0 || K <= 0 || K % BK) return 0;
  if (gemm_plan(M, N, K, kEpiF32, 0, 0, nullptr, nullptr, nullptr, &b) != OASIS_OK) return 0;
  return b;
}

size_t gemm_splitk_bytes(int M, int N, int K, int mode, int block_n, int splits) {
  size_t b = 0;
  if (M <= 0 || N <= 0 || K <= 0 || K % BK) return 0;
  if (gemm_plan(M, N, K, mode, block_n, splits, nullptr, nullptr, nullptr, &b) != OASIS_OK) return 0;
  return b;
}

int gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  OASIS_REQUIRE(p.A && p.W, "GEMM: null operand");
  OASIS_REQUIRE(p.M > 0 && p.N > 0 && p.K > 0, "GEMM: bad shape %d x %d x %d", p.M, p.N, p.K);
  OASIS_REQUIRE(p.K % BK == 0, "GEMM: K=%d must be a multiple of %d", p.K, BK);
  OASIS_REQUIRE(p.N % 16 == 0, "GEMM: N=%d must be a multiple of 16", p.N);
  OASIS_REQUIRE(p.epi.out, "GEMM: null output");
  OASIS_REQUIRE(p.lda >= p.K, "GEMM: lda < K");
  if (reads_resid(p.epi.mode)) OASIS_REQUIRE(p.epi.resid, "GEMM: residual epilogue without residual input");
  if (gated(p.epi.mode)) OASIS_REQUIRE(p.epi.gate && p.epi.rows_per_frame > 0, "GEMM: gate missing");
  if (p.epi.mode == kEpiGatedResidLN) {
    OASIS_REQUIRE(p.N == 1024 && p.epi.ldo == 1024 && p.epi.ldr == 1024, "GEMM: the LN epilogue needs N = 1024 rows");
    OASIS_REQUIRE(p.ln.out && p.ln.mod, "GEMM: LN epilogue without output or modulation table");
    OASIS_REQUIRE(p.block_n == 0 || p.block_n == 256, "GEMM: the LN epilogue uses 256-wide tiles");
    OASIS_REQUIRE(p.splits <= 1, "GEMM: the LN epilogue does not split K");
  }
  if (p.epi.mode == kEpiRopeBF16) OASIS_REQUIRE(p.epi.rope && p.epi.rope_mod > 0 && p.epi.rope_div > 0, "GEMM: rope table missing");
  Plan pl;
  OASIS_TRY(resolve_plan(p, &pl));
  if (pl.pair) return launch_pair(p, stream);
  // one output tile per CTA at most: the deep-pipeline configuration
  const int units = ((p.M + BM - 1) / BM) * ((p.N + pl.bn - 1) / pl.bn) * pl.splits;
  if (deep_enabled() && p.epi.mode != kEpiGatedResidLN && units <= num_sms()) {
    switch (pl.bn) {
      case 32: return launch_bn<32, false, true>(p, pl.splits, stream);
      case 64: return launch_bn<64, false, true>(p, pl.splits, stream);
      case 128: return launch_bn<128, false, true>(p, pl.splits, stream);
      default: break;
    }
  }
  switch (pl.bn) {
    case 32: return launch_bn<32, false>(p, pl.splits, stream);
    case 64: return launch_bn<64, false>(p, pl.splits, stream);
    case 128: return launch_bn<128, false>(p, pl.splits, stream);
    case 256:
      if (p.epi.mode == kEpiGatedResidLN) return launch_bn<256, true>(p, pl.splits, stream);
      return launch_bn<256, false>(p, pl.splits, stream);
    default: return set_error(OASIS_ERR_INVALID_ARG, "GEMM: block_n=%d unsupported", pl.bn);
  }
}

}  // namespace oasis

namespace oasis {

int make_tma_bf16_2d(CUtensorMap* map, const void* ptr, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer) {
  OASIS_TRY(get_encoder());
  OASIS_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA source not 16-byte aligned");
  OASIS_REQUIRE((ld * 2) % 16 == 0, "TMA row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OASIS_OK;
}

int read_device_error(int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error reset: %s", cudaGetErrorString(e));
  }
  return v;
}

}  // namespace oasis
