// Tensor-core (tcgen05 / TMEM) attention within groups of `seq` consecutive rows:
// the DiT spatial attention (seq = 144, one frame) and the VAE attention
// (seq = 576). Non-causal softmax(q k^T / 8) v per (group, head), head dim 64,
// reading q/k/v straight out of the packed QKV rows [rows, 3 H 64] (RoPE already
// applied) and writing [rows, H 64].
//
// Work unit: 128 consecutive query rows of the token stream x one head. Because
// seq >= 128 such a tile touches at most two groups; its keys are visited in
// blocks of KB keys (KB divides seq), each block lying inside one group, and a
// row only takes the blocks of its own group (the others are masked to zero in
// P and leave its running max untouched).
//
// Per key block j (online softmax; P V of a block is accumulated after the next
// block's softmax, across unit boundaries too):
//   S_j  = Q K_j^T       tcgen05.mma M=128 N=KB K=64, fp32 in TMEM (two buffers)
//   P_j  = exp2(S_j * c - m_j)   softmax warps, one TMEM lane (query row) per
//                                thread (SWQ threads per row, each with a share
//                                of the columns), S read from TMEM once, bf16 P
//                                written to shared memory in the K-major
//                                128-byte-swizzled operand layout
//   PV_j = P_j V_j       tcgen05.mma M=128 N=64 K=KB with V as an MN-major
//                        operand (V rows are key-major as they sit in memory)
//   O    = O alpha_j + PV_j  in registers (alpha_j rescales to the new max)
// Warp 0 streams Q (one buffer: the next unit's Q loads while the last block of
// the current unit is in softmax) and K/V blocks (3-stage ring) with
// TMA, warp 1 owns TMEM and issues the MMAs from one thread, SWQ warps per TMEM
// lane quarter do the softmax and the output. Persistent over units. Every wait
// is bounded and records a code in this file's device error word.
#include <cuda.h>

#include "common.cuh"
#include "gemm.cuh"
#include "pointwise.cuh"
#include "status.h"

namespace oasis {
namespace {

constexpr int kTcRows = 128;    // query rows per unit = TMEM lanes
// Warp 0 TMA, warp 1 MMA, then 4 SWQ softmax warps from warp 4 (from warp 2 when
// SWQ = 4): SWQ warps share each TMEM lane quarter (32 query rows), splitting
// the key columns of a block and the 64 output dims between them. SWQ = 2
// (measured: 4 ties at three more warps and spills).
#ifndef OASIS_TC_SWQ
#define OASIS_TC_SWQ 2
#endif
constexpr int kTcSWQ = OASIS_TC_SWQ;
constexpr int kTcSoftWarp0 = kTcSWQ >= 4 ? 2 : 4;
constexpr int kTcThreads = 32 * (kTcSoftWarp0 + 4 * kTcSWQ);
constexpr int kTcSCols = 192;    // TMEM columns reserved per S buffer (KB <= 192)
// (all callers use KB = 144: shared memory then holds one Q tile, three K/V
// stages and two P tiles within the 227 KB limit)
constexpr int kTcPVCol = 384;    // PV buffers at columns 384 and 448

template <int KB>
struct TcCfg {
  static_assert(KB % 16 == 0 && KB <= kTcSCols, "key block");
  static constexpr int Q_BYTES = kTcRows * 128;
  static constexpr int KV_BYTES = KB * 128;  // one K or V block: KB rows of 64 bf16
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int STAGES = 3;   // K/V ring depth
  static constexpr int Q_BUFS = 1;   // the next unit's Q loads during the last block's softmax
  static constexpr int P_ATOMS = (KB + 63) / 64;  // 64-key atoms of the P operand
  static constexpr int P_BYTES = P_ATOMS * kTcRows * 128;
  static constexpr int BAR_BYTES = 256 + 2 * kTcSWQ * kTcRows * 4;  // barriers + row max/sum exchange
  static constexpr int SMEM = 1024 + Q_BUFS * Q_BYTES + STAGES * STAGE_BYTES + 2 * P_BYTES + BAR_BYTES;
  static_assert(SMEM <= 232448, "shared memory");
};

// K-major operands (Q, K, P): S = Q K^T reads K like a weight matrix. MN-major B
// (bit 16) for V: its 64 head dims are the contiguous direction.
__host__ __device__ constexpr uint32_t idesc_tc(int m, int n, bool b_mn_major) {
  return idesc_bf16_f32(m, n) | (b_mn_major ? (1u << 16) : 0u);
}

__device__ int g_tc_error = 0;


__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int code, int site = 0) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(addr, parity)) {
    if (clock64() - t0 > kWaitClockLimit) {
      atomicCAS(&g_tc_error, 0, code);
      return false;
    }
  }
  (void)site;
  return true;
}

struct TcUnit {
  int q0, head, g0, nblk;
};

__device__ __forceinline__ TcUnit tc_unit(int u, int H, int seq, int rows, int nsub) {
  TcUnit t;
  const int tile = u / H;
  t.head = u - tile * H;
  t.q0 = tile * kTcRows;
  const int last = min(t.q0 + kTcRows, rows) - 1;
  t.g0 = t.q0 / seq;
  t.nblk = (last / seq - t.g0 + 1) * nsub;
  return t;
}

template <int KB>
__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                        __nv_bfloat16* __restrict__ out, int rows, int seq, int H) {
  using C = TcCfg<KB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [Q_BUFS][128 rows x 128 B]
  uint8_t* sKV = sQ + C::Q_BUFS * C::Q_BYTES;           // [STAGES][K block | V block]
  uint8_t* sP = sKV + C::STAGES * C::STAGE_BYTES;       // [2][P_ATOMS][128 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* q_full = bars;        // [Q_BUFS <= 2]
  uint64_t* q_empty = bars + 2;   // [Q_BUFS <= 2]
  uint64_t* kv_full = bars + 4;   // [STAGES <= 3]
  uint64_t* kv_empty = bars + 7;  // [STAGES <= 3]
  uint64_t* s_full = bars + 10;   // [2]
  uint64_t* p_full = bars + 12;   // [2]
  uint64_t* pv_full = bars + 14;  // [2]
  uint64_t* pv_free = bars + 16;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  float* xch = reinterpret_cast<float*>(bars + 32);  // [2 rounds][SWQ parts][128 rows]
  static_assert(C::Q_BUFS <= 2 && C::STAGES <= 3, "barrier slots");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HD = H * 64;
  const int nsub = seq / KB;
  const int units = ((rows + kTcRows - 1) / kTcRows) * H;
  pdl_trigger();

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmKV);
    for (int i = 0; i < C::Q_BUFS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4 * kTcSWQ);
      mbar_init(&pv_full[i], 1);
      mbar_init(&pv_free[i], 4 * kTcSWQ);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      pdl_wait();
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x, qi = 0; u < units && ok; u += gridDim.x, ++qi) {
        const TcUnit t = tc_unit(u, H, seq, rows, nsub);
        const int qb = qi % C::Q_BUFS;
        if (!tc_wait(&q_empty[qb], ((qi / C::Q_BUFS) & 1) ^ 1, kDevTimeoutSmemEmpty, 1)) break;
        mbar_arrive_expect_tx(&q_full[qb], C::Q_BYTES);
        tma_load_2d(sQ + qb * C::Q_BYTES, &tmQ, &q_full[qb], t.head * 64, t.q0);
        for (int i = 0; i < t.nblk; ++i) {
          if (!tc_wait(&kv_empty[st], ph ^ 1, kDevTimeoutSmemEmpty, 2)) { ok = false; break; }
          const int kb0 = t.g0 * seq + i * KB;
          uint8_t* dst = sKV + st * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&kv_full[st], C::STAGE_BYTES);
          tma_load_2d(dst, &tmKV, &kv_full[st], HD + t.head * 64, kb0);
          tma_load_2d(dst + C::KV_BYTES, &tmKV, &kv_full[st], 2 * HD + t.head * 64, kb0);
          if (++st == C::STAGES) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tc(kTcRows, KB, false);
      constexpr uint32_t idPV = idesc_tc(kTcRows, 64, true);
      int st = 0, st_prev = 0;
      uint32_t ph = 0;
      int jb = 0;
      bool ok = true;
      // PV_j = P_j V_j for global block j whose K/V sit in stage `stj`
      auto issue_pv = [&](int j, int stj) -> bool {
        const int b = j & 1;
        if (!tc_wait(&p_full[b], (j >> 1) & 1, kDevTimeoutTmaFull, 3)) return false;
        if (j >= 2 && !tc_wait(&pv_free[b], ((j >> 1) - 1) & 1, kDevTimeoutAccEmpty, 4)) return false;
        tc_fence_after();
        const uint32_t d = tmem + kTcPVCol + b * 64;
        const uint32_t p_addr = smem_u32(sP + b * C::P_BYTES);
        const uint32_t v_addr = smem_u32(sKV + stj * C::STAGE_BYTES + C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk) {
          // P: atom kk / 4, +32 B per 16 keys inside it; V: +16 key rows = 2048 B
          const uint64_t a = smem_desc_sw128(p_addr + (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32);
          const uint64_t bd = smem_desc_sw128(v_addr + kk * 2048);
          tc_mma_bf16(d, a, bd, idPV, kk > 0 ? 1u : 0u);
        }
        tc_commit(&pv_full[b]);
        tc_commit(&kv_empty[stj]);
        return true;
      };
      bool pending = false;  // PV of block jb - 1 not yet issued
      for (int u = blockIdx.x, qi = 0; u < units && ok; u += gridDim.x, ++qi) {
        const TcUnit t = tc_unit(u, H, seq, rows, nsub);
        const int qb = qi % C::Q_BUFS;
        if (!tc_wait(&q_full[qb], (qi / C::Q_BUFS) & 1, kDevTimeoutTmaFull, 5)) break;
        const uint32_t q_addr = smem_u32(sQ + qb * C::Q_BYTES);
        for (int i = 0; i < t.nblk; ++i, ++jb) {
          const int b = jb & 1;
          if (!tc_wait(&kv_full[st], ph, kDevTimeoutTmaFull, 6)) { ok = false; break; }
          // S[b] is free once the softmax of block jb - 2 has read it (it then wrote P)
          if (jb >= 2 && !tc_wait(&p_full[b], ((jb >> 1) - 1) & 1, kDevTimeoutAccEmpty, 0)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sKV + st * C::STAGE_BYTES);
          const uint32_t d = tmem + b * kTcSCols;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_bf16(d, smem_desc_sw128(q_addr) + (uint64_t)(k * 2), smem_desc_sw128(k_addr) + (uint64_t)(k * 2),
                        idS, k > 0 ? 1u : 0u);
          tc_commit(&s_full[b]);
          if (i == t.nblk - 1) tc_commit(&q_empty[qb]);  // last S of the unit: Q buffer reusable
          // the previous block's P V (possibly of the previous unit) overlaps this S
          if (pending && !issue_pv(jb - 1, st_prev)) { ok = false; break; }
          pending = true;
          st_prev = st;
          if (++st == C::STAGES) { st = 0; ph ^= 1; }
        }
      }
      if (ok && pending) issue_pv(jb - 1, st_prev);
    }
  } else if (warp >= kTcSoftWarp0) {
    // ---------------- softmax + output ----------------
    // Blocks are handled in one stream across units, P V of block j being
    // accumulated after the softmax of block j + 1 (so its MMA latency is hidden);
    // a unit's output is written when its last block has been accumulated.
    // Half `hf` of a lane quarter takes the 32-column chunks c with c % SWQ == hf
    // (the 16-column tail of KB = 144 goes to the last half) and output dims
    // [hf 64 / SWQ, (hf + 1) 64 / SWQ); row max and sum are exchanged through
    // shared memory with a named barrier per quarter.
    constexpr int ODIM = 64 / kTcSWQ;
    constexpr int NCH = KB / 32;
    const int quarter = warp & 3;
    const int hf = (warp - kTcSoftWarp0) >> 2;  // which part of the quarter's columns
    const int row_t = quarter * 32 + lane;  // TMEM lane = query row in the unit
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sc = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) in log2 units
    auto pair_sync = [&]() {
      if constexpr (kTcSWQ > 1) named_barrier_sync(1 + quarter, 32 * kTcSWQ);
    };
    int jb = 0;
    bool ok = true;
    float o[ODIM];
#pragma unroll
    for (int i = 0; i < ODIM; ++i) o[i] = 0.f;
    bool pending = false, pending_last = false;
    float alpha_prev = 0.f, l_done = 0.f;
    int r_done = 0, head_done = 0;
    // O = O alpha + PV_j (this half's dims) for global block j
    auto accumulate = [&](int j, float alpha) -> bool {
      const int b = j & 1;
      if (!tc_wait(&pv_full[b], (j >> 1) & 1, kDevTimeoutAccFull, 8)) return false;
      tc_fence_after();
      if constexpr (ODIM >= 32) {
#pragma unroll
        for (int h = 0; h < ODIM / 32; ++h) {
          float pv[32];
          tmem_ld32(lane_base + kTcPVCol + b * 64 + hf * ODIM + h * 32, pv);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h * 32 + i] = fmaf(o[h * 32 + i], alpha, pv[i]);
        }
      } else {
        float pv[16];
        tmem_ld16(lane_base + kTcPVCol + b * 64 + hf * ODIM, pv);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = fmaf(o[i], alpha, pv[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pv_free[b]);
      return true;
    };
    auto finish = [&]() {  // write the finished unit's row (this half's dims), clear O
      if (r_done < rows && l_done > 0.f) {
        const float inv = 1.f / l_done;
        uint4* dst = reinterpret_cast<uint4*>(out + (long long)r_done * HD + head_done * 64 + hf * ODIM);
#pragma unroll
        for (int q = 0; q < ODIM / 8; ++q)
          dst[q] = make_uint4(pack_bf16x2(o[8 * q] * inv, o[8 * q + 1] * inv),
                              pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                              pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv),
                              pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
      }
#pragma unroll
      for (int i = 0; i < ODIM; ++i) o[i] = 0.f;
    };
    auto store_p = [&](uint8_t* prow, int chunk, const uint32_t (&pk)[4]) {  // 16-byte chunk = 8 keys
      uint8_t* dst = prow + (chunk >> 3) * (kTcRows * 128) + (((chunk & 7) ^ (row_t & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const TcUnit t = tc_unit(u, H, seq, rows, nsub);
      const int r = t.q0 + row_t;
      const int g_r = r < rows ? r / seq : -1;
      float m = -1e30f, l = 0.f;
      for (int i = 0; i < t.nblk; ++i, ++jb) {
        const int b = jb & 1;
        const bool mine = (g_r == t.g0 + i / nsub);
        if (!tc_wait(&s_full[b], (jb >> 1) & 1, kDevTimeoutAccFull, 9)) { ok = false; break; }
        tc_fence_after();
        uint8_t* prow = sP + b * C::P_BYTES + row_t * 128;
        float alpha = 1.f;
#define TC_SECTION(i)
        if (__any_sync(0xffffffffu, mine)) {  // same rows, same decision in both halves
          const uint32_t sbase = lane_base + b * kTcSCols;
          // this part's S columns into registers with one TMEM round trip
          // (loads are warp-collective), then the row max and p = exp2(s c - m)
          constexpr int CPT = (NCH + kTcSWQ - 1) / kTcSWQ;  // 32-column chunks per part
          constexpr bool TAIL = KB % 32 != 0;
          const bool has_tail = TAIL && hf == kTcSWQ - 1;
          uint32_t sr[CPT][32];
          uint32_t st16[16];
#pragma unroll
          for (int i2 = 0; i2 < CPT; ++i2)
            if (hf + i2 * kTcSWQ < NCH) tmem_ld32_issue(sbase + (hf + i2 * kTcSWQ) * 32, sr[i2]);
          if (has_tail) tmem_ld16_issue(sbase + NCH * 32, st16);
#pragma unroll
          for (int i2 = 0; i2 < CPT; ++i2) tmem_wait_ld(sr[i2]);
          tmem_wait_ld(st16);
          float bm = -1e30f;
#pragma unroll
          for (int i2 = 0; i2 < CPT; ++i2)
            if (hf + i2 * kTcSWQ < NCH)
#pragma unroll
              for (int k = 0; k < 32; ++k) bm = fmaxf(bm, __uint_as_float(sr[i2][k]));
          if (has_tail)
#pragma unroll
            for (int k = 0; k < 16; ++k) bm = fmaxf(bm, __uint_as_float(st16[k]));
          if constexpr (kTcSWQ > 1) {
            xch[hf * kTcRows + row_t] = bm;
            pair_sync();
#pragma unroll
            for (int w2 = 0; w2 < kTcSWQ; ++w2) bm = fmaxf(bm, xch[w2 * kTcRows + row_t]);
          }
          TC_SECTION(11)
          const float mnew = mine ? fmaxf(m, bm * sc) : m;
          alpha = mine ? ex2_approx(m - mnew) : 1.f;
          float rs = 0.f;
          auto emit = [&](const uint32_t* sv, int chunk) {  // 8 keys -> one 16-byte P chunk
            uint32_t pk[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float p0 = mine ? ex2_approx(fmaf(__uint_as_float(sv[2 * k]), sc, -mnew)) : 0.f;
              const float p1 = mine ? ex2_approx(fmaf(__uint_as_float(sv[2 * k + 1]), sc, -mnew)) : 0.f;
              rs += p0 + p1;
              pk[k] = pack_bf16x2(p0, p1);
            }
            store_p(prow, chunk, pk);
          };
#pragma unroll
          for (int i2 = 0; i2 < CPT; ++i2) {
            const int c = hf + i2 * kTcSWQ;
            if (c < NCH)
#pragma unroll
              for (int q = 0; q < 4; ++q) emit(&sr[i2][8 * q], c * 4 + q);
          }
          if (has_tail) {
            emit(&st16[0], NCH * 4);
            emit(&st16[8], NCH * 4 + 1);
          }
          TC_SECTION(12)
          if constexpr (kTcSWQ > 1) {
            xch[(kTcSWQ + hf) * kTcRows + row_t] = rs;
            pair_sync();
            rs = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kTcSWQ; ++w2) rs += xch[(kTcSWQ + w2) * kTcRows + row_t];
          }
          if (mine) {
            l = l * alpha + rs;
            m = mnew;
          }
          TC_SECTION(13)
        } else {
          // no row of this warp belongs to the block's group: zero this half's P chunks
          const uint32_t zero[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int c = hf; c < NCH; c += kTcSWQ)
#pragma unroll
            for (int q = 0; q < 4; ++q) store_p(prow, c * 4 + q, zero);
          if constexpr (KB % 32 != 0) {
            if (hf == kTcSWQ - 1) {
              store_p(prow, NCH * 4, zero);
              store_p(prow, NCH * 4 + 1, zero);
            }
          }
        }
        tc_fence_before();    // S[b] reads done before the MMA may overwrite it
        fence_proxy_async();  // P writes visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
        TC_SECTION(14)
        if (pending) {
          if (!accumulate(jb - 1, alpha_prev)) { ok = false; break; }
          TC_SECTION(15)
          if (pending_last) finish();
          TC_SECTION(7)
        }
        pending = true;
        alpha_prev = alpha;
        pending_last = (i == t.nblk - 1);
        if (pending_last) {
          l_done = l;
          r_done = r;
          head_done = t.head;
        }
      }
    }
    if (ok && pending && accumulate(jb - 1, alpha_prev)) finish();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <int KB>
int launch_tc(const __nv_bfloat16* qkv, __nv_bfloat16* out, int groups, int seq, int H, cudaStream_t s) {
  using C = TcCfg<KB>;
  static std::atomic<bool> attr[64];  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr[dev & 63] = true;
  }
  const long long rows = (long long)groups * seq;
  const int ld = 3 * H * 64;
  CUtensorMap tq, tkv;
  OASIS_TRY(make_tma_bf16_2d(&tq, qkv, ld, rows, ld, 64, kTcRows));
  OASIS_TRY(make_tma_bf16_2d(&tkv, qkv, ld, rows, ld, 64, KB));
  const int units = (int)((rows + kTcRows - 1) / kTcRows) * H;
  const int grid = units < grid_sms() ? units : grid_sms();
  launch_pdl(attention_tc_kernel<KB>, dim3(grid), dim3(kTcThreads), C::SMEM, s, tq, tkv, out, (int)rows, seq, H);
  return check_launch("attention_tc_kernel");
}

}  // namespace

bool attention_tc_supported(int seq) { return seq >= 144 && seq % 144 == 0; }

int attention_tc_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int groups, int seq, int H, cudaStream_t s) {
  OASIS_REQUIRE(qkv && out, "attention_tc: null pointer");
  OASIS_REQUIRE(H >= 1 && H <= 16, "attention_tc: heads=%d outside [1, 16]", H);
  OASIS_REQUIRE(attention_tc_supported(seq), "attention_tc: seq=%d unsupported", seq);
  OASIS_REQUIRE((long long)groups * seq < (1LL << 31), "attention_tc: too many rows");
  if (groups == 0) return OASIS_OK;
  return launch_tc<144>(qkv, out, groups, seq, H, s);  // key blocks of 144 (VAE: 4 per 576-token frame)
}


int read_device_error_tc(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error reset: %s", cudaGetErrorString(e));
  }
  return v;
}

}  // namespace oasis
