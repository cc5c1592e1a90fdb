// Attention kernels of the Oasis frame path.
//
// Both read q/k/v straight out of the packed QKV GEMM output [rows, 3072] bf16
// (q | k | v, 16 heads x 64; RoPE already applied by the GEMM epilogue), so the
// reference's separate RoPE/layout kernels and reshapes disappear: a head is a
// 128-byte column slice of each row.
//
// attention_spatial (seq = 144, the DiT spatial case): persistent, one whole
//   (frame, head) problem per CTA iteration, see below.
// attention_full: non-causal softmax(q k^T / 8) v within groups of `seq`
//   consecutive rows (VAE: one frame, seq = 576; other lengths: key tail masked).
//   Flash-style: K/V tiles of 64 keys staged in swizzled shared memory with
//   cp.async double buffering, online softmax in fp32, bf16 mma.sync m16n8k16.
// attention_temporal: causal softmax over the T frames of one session, per
//   (patch, head). A warp covers 256 columns (four heads) of one (session,
//   patch), 16 bytes per lane per row, so every q/k/v access is a coalesced
//   512-byte run; T <= 8 holds all frames in registers, longer T shares key
//   loads across blocks of four queries with an online softmax.
// attention_temporal_cached: the generated frame's query only, with the context
//   frames' keys/values read from a cache written once per frame.
#include "common.cuh"
#include "pointwise.cuh"
#include "status.h"

namespace oasis {
namespace {

constexpr int kDh = 64;
// Head count H is a runtime argument (16 for the full model, 16 / n per rank
// under n-way tensor parallelism): a qkv row is 3 H 64 wide, an output row H 64.
constexpr int kKeyTile = 64;

__device__ __forceinline__ int swz(int row, int col) {
  return row * kDh + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Loads `rows` rows (64 bf16 each) of one head slice into a swizzled tile; rows past
// `valid` are zero-filled.
template <int NT>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int rows, int valid,
                                          int ld) {
  for (int i = threadIdx.x; i < rows * 8; i += NT) {
    const int r = i >> 3, c = (i & 7) * 8;
    const bool ok = r < valid;
    cp_async16(dst + swz(r, c), src + (long long)(ok ? r : 0) * ld + c, ok);
  }
}

template <int NW>
__global__ void __launch_bounds__(NW * 32) attention_full_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                 __nv_bfloat16* __restrict__ out, int seq, int H) {
  pdl_trigger();
  pdl_wait();
  constexpr int NT = NW * 32;
  constexpr int QROWS = NW * 16;
  __shared__ __align__(128) __nv_bfloat16 sQ[QROWS * kDh];
  __shared__ __align__(128) __nv_bfloat16 sK[2][kKeyTile * kDh];
  __shared__ __align__(128) __nv_bfloat16 sV[2][kKeyTile * kDh];

  const int q0 = blockIdx.x * QROWS;
  const int head = blockIdx.y;
  const long long grp_row = (long long)blockIdx.z * seq;
  const int kQkvLd = 3 * H * kDh, kOutLd = H * kDh;
  const __nv_bfloat16* qb = qkv + grp_row * kQkvLd + head * kDh;
  const __nv_bfloat16* kb = qb + kOutLd;
  const __nv_bfloat16* vb = qb + 2 * kOutLd;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ntiles = (seq + kKeyTile - 1) / kKeyTile;

  load_tile<NT>(sQ, qb + (long long)q0 * kQkvLd, QROWS, seq - q0, kQkvLd);
  load_tile<NT>(sK[0], kb, kKeyTile, seq, kQkvLd);
  load_tile<NT>(sV[0], vb, kKeyTile, seq, kQkvLd);
  cp_async_commit();

  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sc = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      const int k0n = (j + 1) * kKeyTile;
      load_tile<NT>(sK[buf ^ 1], kb + (long long)k0n * kQkvLd, kKeyTile, seq - k0n, kQkvLd);
      load_tile<NT>(sV[buf ^ 1], vb + (long long)k0n * kQkvLd, kKeyTile, seq - k0n, kQkvLd);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qa[kk], sQ + swz(r, c));
      }
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b[4];
        const int m = lane >> 3;
        const int key = np * 16 + (lane & 7) + (m >> 1) * 8;
        const int c = kk * 16 + (m & 1) * 8;
        ldsm_x4(b, sK[buf] + swz(key, c));
        mma_bf16(s[2 * np], qa[kk], b[0], b[1]);
        mma_bf16(s[2 * np + 1], qa[kk], b[2], b[3]);
      }
    }
    // scale, mask the key tail, online softmax (rows g and g+8 of this warp)
    const int kbase = j * kKeyTile;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + i * 8 + 2 * t + (e & 1);
        s[i][e] = key < seq ? s[i][e] * sc : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[i][0], s[i][1]));
      mx1 = fmaxf(mx1, fmaxf(s[i][2], s[i][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float alpha0 = ex2_approx(m0 - mx0), alpha1 = ex2_approx(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = ex2_approx(s[i][0] - mx0);
      s[i][1] = ex2_approx(s[i][1] - mx0);
      s[i][2] = ex2_approx(s[i][2] - mx1);
      s[i][3] = ex2_approx(s[i][3] - mx1);
      rs0 += s[i][0] + s[i][1];
      rs1 += s[i][2] + s[i][3];
    }
    l0 = l0 * alpha0 + rs0;
    l1 = l1 * alpha1 + rs1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= alpha0; o[i][1] *= alpha0;
      o[i][2] *= alpha1; o[i][3] *= alpha1;
    }
    // O += P V : 4 k-steps of 16 keys, 8 n-tiles of 8 head dims
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {  // pairs of d n-tiles
        uint32_t b[4];
        const int m = lane >> 3;
        const int key = kk * 16 + (lane & 7) + (m & 1) * 8;
        const int c = dp * 16 + (m >> 1) * 8;
        ldsm_x4_t(b, sV[buf] + swz(key, c));
        mma_bf16(o[2 * dp], pa, b[0], b[1]);
        mma_bf16(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  // row sums across the 4 lanes of a quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
  __nv_bfloat16* ob = out + grp_row * kOutLd + head * kDh;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = i * 8 + 2 * t;
    if (r0 < seq)
      *reinterpret_cast<uint32_t*>(ob + (long long)r0 * kOutLd + c) = pack_bf16x2(o[i][0] * inv0, o[i][1] * inv0);
    if (r1 < seq)
      *reinterpret_cast<uint32_t*>(ob + (long long)r1 * kOutLd + c) = pack_bf16x2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

// Spatial attention over exactly 144 tokens: one (frame, head) problem per CTA
// iteration, persistent over problems. 9 warps x 16 query rows cover all 144
// queries, so K and V are staged once per problem; a warp's 16 x 144 score strip
// is computed in two key chunks (80 + 64, no key tail: 144 = 9 x 16) with an
// online softmax, which keeps it under 112 registers so two CTAs share an SM.
// The next problem's q/k/v slices are prefetched into the other half of a double
// buffer with cp.async while the current one is computed.
constexpr int kSpatialSeq = 144;
constexpr int kSpatialWarps = 9;
constexpr int kSpatialTile = kSpatialSeq * kDh;  // bf16 elements per q, k or v slice

__device__ __forceinline__ void spatial_prefetch(__nv_bfloat16* buf, const __nv_bfloat16* qkv, int item, int H) {
  const int kQkvLd = 3 * H * kDh, kOutLd = H * kDh;
  const long long row0 = (long long)(item / H) * kSpatialSeq;
  const __nv_bfloat16* src = qkv + row0 * kQkvLd + (item % H) * kDh;
  for (int i = threadIdx.x; i < 3 * kSpatialSeq * 8; i += kSpatialWarps * 32) {
    const int m = i / (kSpatialSeq * 8), rem = i - m * (kSpatialSeq * 8);
    const int r = rem >> 3, c = (rem & 7) * 8;
    cp_async16(buf + m * kSpatialTile + swz(r, c), src + (long long)r * kQkvLd + m * kOutLd + c, true);
  }
}

__global__ void __launch_bounds__(kSpatialWarps * 32, 2)
    attention_spatial_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out, int items, int H) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) __nv_bfloat16 sm[];  // [2][q | k | v]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const float sc = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
  int item = blockIdx.x;
  if (item >= items) return;
  spatial_prefetch(sm, qkv, item, H);
  cp_async_commit();
  for (int it = 0; item < items; ++it, item += gridDim.x) {
    __nv_bfloat16* cur = sm + (it & 1) * 3 * kSpatialTile;
    const int next = item + gridDim.x;
    if (next < items) spatial_prefetch(sm + ((it + 1) & 1) * 3 * kSpatialTile, qkv, next, H);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* sQ = cur;
    const __nv_bfloat16* sK = cur + kSpatialTile;
    const __nv_bfloat16* sV = cur + 2 * kSpatialTile;

    uint32_t qa[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4(qa[kk], sQ + swz(r, kk * 16 + (lane >> 4) * 8));
    }
    // keys in two chunks (80 + 64) with an online softmax: half the score
    // registers of a single pass, so two CTAs fit on an SM
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int nb0 = ch == 0 ? 0 : 5, nbn = ch == 0 ? 5 : 4;  // 16-key blocks of this chunk
      float s[10][4];
#pragma unroll
      for (int i = 0; i < 10; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int nq = 0; nq < 5; ++nq) {
        if (nq < nbn) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint32_t b[4];
            const int m = lane >> 3;
            ldsm_x4(b, sK + swz((nb0 + nq) * 16 + (lane & 7) + (m >> 1) * 8, kk * 16 + (m & 1) * 8));
            mma_bf16(s[2 * nq], qa[kk], b[0], b[1]);
            mma_bf16(s[2 * nq + 1], qa[kk], b[2], b[3]);
          }
        }
      }
      float mx0 = m0, mx1 = m1;
#pragma unroll
      for (int i = 0; i < 10; ++i) {
        if (i < 2 * nbn) {
          s[i][0] *= sc; s[i][1] *= sc; s[i][2] *= sc; s[i][3] *= sc;
          mx0 = fmaxf(mx0, fmaxf(s[i][0], s[i][1]));
          mx1 = fmaxf(mx1, fmaxf(s[i][2], s[i][3]));
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float a0 = ex2_approx(m0 - mx0), a1 = ex2_approx(m1 - mx1);  // 0 on the first chunk
      m0 = mx0;
      m1 = mx1;
      l0 *= a0;
      l1 *= a1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= a0; o[i][1] *= a0;
        o[i][2] *= a1; o[i][3] *= a1;
      }
#pragma unroll
      for (int i = 0; i < 10; ++i) {
        if (i < 2 * nbn) {
          s[i][0] = ex2_approx(s[i][0] - mx0);
          s[i][1] = ex2_approx(s[i][1] - mx0);
          s[i][2] = ex2_approx(s[i][2] - mx1);
          s[i][3] = ex2_approx(s[i][3] - mx1);
          l0 += s[i][0] + s[i][1];
          l1 += s[i][2] + s[i][3];
        }
      }
#pragma unroll
      for (int kk = 0; kk < 5; ++kk) {
        if (kk < nbn) {
          uint32_t pa[4];
          pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
          pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
          pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
          pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
          for (int dp = 0; dp < 4; ++dp) {
            uint32_t b[4];
            const int m = lane >> 3;
            ldsm_x4_t(b, sV + swz((nb0 + kk) * 16 + (lane & 7) + (m & 1) * 8, dp * 16 + (m >> 1) * 8));
            mma_bf16(o[2 * dp], pa, b[0], b[1]);
            mma_bf16(o[2 * dp + 1], pa, b[2], b[3]);
          }
        }
      }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
    // Stage this warp's 16 output rows in its (no longer needed) rows of the q slice,
    // then write them out as whole 128-byte rows.
    __nv_bfloat16* sO = cur;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = i * 8 + 2 * t;
      *reinterpret_cast<uint32_t*>(sO + swz(warp * 16 + g, c)) = pack_bf16x2(o[i][0] * inv0, o[i][1] * inv0);
      *reinterpret_cast<uint32_t*>(sO + swz(warp * 16 + g + 8, c)) = pack_bf16x2(o[i][2] * inv1, o[i][3] * inv1);
    }
    __syncwarp();
    const int kOutLd = H * kDh;
    __nv_bfloat16* ob = out + (long long)(item / H) * kSpatialSeq * kOutLd + (item % H) * kDh;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = warp * 16 + k * 4 + (lane >> 3), c = (lane & 7) * 8;
      *reinterpret_cast<uint4*>(ob + (long long)r * kOutLd + c) = *reinterpret_cast<const uint4*>(sO + swz(r, c));
    }
    __syncthreads();  // this buffer is refilled two iterations from now
  }
}

// Causal temporal attention for T <= TMAX <= 8 in the lane-per-columns layout
// of the cached kernel below (a warp covers 256 columns = four heads of one
// (session, patch), lane l the 8 columns [8 l, 8 l + 8)): every frame's q, k and
// v segments are loaded up front as 16-byte packets (3 T loads per lane, whole
// 512-byte runs per warp), then each query's scores over the earlier frames are
// reduced across the 8 lanes of its head with three shuffles.
template <int TMAX>
__global__ void __launch_bounds__(256) attention_temporal_rows_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                      __nv_bfloat16* __restrict__ out, int batch,
                                                                      int T, int P, int H);

// Context-cached temporal attention: the one query of the generated frame
// (position Tp) of each (session, patch) against the cached keys/values of the
// Tp context frames plus its own. past: packed QKV rows of the context frames,
// [B, Tp, P, 3 H 64]; cur: packed QKV rows of the generated frame,
// [B, P, 3 H 64]; out: [B, P, H 64]. The causal mask admits every key.
//
// Lane-per-columns layout: a warp covers 256 consecutive columns of the q, k and
// v sections (four heads), lane l the 8 columns [8 l, 8 l + 8) (one 16-byte load
// per row and section), so a key row's K and V segments are read as whole
// coalesced 512-byte runs; the 8 lanes of a head combine their partial dot
// products with three shuffles. Online softmax over the keys; the next key row
// is loaded while the current one is used.
constexpr int kCachedCols = 8;                 // columns per lane
constexpr int kCachedWarpCols = 32 * kCachedCols;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& r, float (&f)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__global__ void __launch_bounds__(256) attention_temporal_cached_kernel(const __nv_bfloat16* __restrict__ past,
                                                                        const __nv_bfloat16* __restrict__ cur,
                                                                        __nv_bfloat16* __restrict__ out, int batch,
                                                                        int Tp, int P, int H) {
  pdl_trigger();
  pdl_wait();
  const int HD = H * kDh, ld = 3 * HD;
  const int wpr = (HD + kCachedWarpCols - 1) / kCachedWarpCols;  // warps per (session, patch)
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)batch * P * wpr) return;  // warp-uniform
  const long long bp = w / wpr;
  const int part = (int)(w - bp * wpr);
  const int p = bp % P;
  const long long b = bp / P;
  int col = part * kCachedWarpCols + kCachedCols * lane;
  const bool active = col < HD;  // whole heads are active or idle together
  if (!active) col = 0;
  const __nv_bfloat16* crow = cur + bp * ld;
  float q[8];
  bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(crow + col)), q);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] *= 0.125f * 1.4426950408889634f;  // 1/sqrt(64), log2 units
  auto key_row = [&](int t) -> const __nv_bfloat16* {
    return t < Tp ? past + ((b * Tp + t) * P + p) * ld : crow;
  };
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float mx = -INFINITY, l = 0.f;
  uint4 kc = __ldg(reinterpret_cast<const uint4*>(key_row(0) + HD + col));
  uint4 vc = __ldg(reinterpret_cast<const uint4*>(key_row(0) + 2 * HD + col));
  for (int t = 0; t <= Tp; ++t) {
    uint4 kn = kc, vn = vc;
    if (t < Tp) {
      const __nv_bfloat16* nr = key_row(t + 1);
      kn = __ldg(reinterpret_cast<const uint4*>(nr + HD + col));
      vn = __ldg(reinterpret_cast<const uint4*>(nr + 2 * HD + col));
    }
    float k[8], v[8];
    bf16x8_to_f32(kc, k);
    float sc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sc = fmaf(q[i], k[i], sc);
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    sc += __shfl_xor_sync(0xffffffffu, sc, 2);
    sc += __shfl_xor_sync(0xffffffffu, sc, 4);
    const float mnew = fmaxf(mx, sc);
    const float corr = ex2_approx(mx - mnew);  // 0 on the first key
    const float e = ex2_approx(sc - mnew);
    l = l * corr + e;
    mx = mnew;
    bf16x8_to_f32(vc, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(e, v[i], acc[i] * corr);
    kc = kn;
    vc = vn;
  }
  if (active) {
    const float inv = 1.f / l;
    *reinterpret_cast<uint4*>(out + bp * HD + col) =
        make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                   pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
  }
}

template <int TMAX>
__global__ void __launch_bounds__(256) attention_temporal_rows_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                      __nv_bfloat16* __restrict__ out, int batch,
                                                                      int T, int P, int H) {
  pdl_trigger();
  pdl_wait();
  const int HD = H * kDh, ld = 3 * HD;
  const int wpr = (HD + kCachedWarpCols - 1) / kCachedWarpCols;
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)batch * P * wpr) return;  // warp-uniform
  const long long bp = w / wpr;
  const int part = (int)(w - bp * wpr);
  const int p = bp % P;
  const long long b = bp / P;
  int col = part * kCachedWarpCols + kCachedCols * lane;
  const bool active = col < HD;
  if (!active) col = 0;
  const __nv_bfloat16* base = qkv + (b * T * P + p) * ld + col;  // frame t: + t P ld
  uint4 qr[TMAX], kr[TMAX], vr[TMAX];
#pragma unroll
  for (int t = 0; t < TMAX; ++t) {
    if (t < T) {
      const __nv_bfloat16* rp = base + (long long)t * P * ld;
      qr[t] = __ldg(reinterpret_cast<const uint4*>(rp));
      kr[t] = __ldg(reinterpret_cast<const uint4*>(rp + HD));
      vr[t] = __ldg(reinterpret_cast<const uint4*>(rp + 2 * HD));
    }
  }
  __nv_bfloat16* obase = out + (b * T * P + p) * (long long)HD + col;
#pragma unroll
  for (int tq = 0; tq < TMAX; ++tq) {
    if (tq < T) {
      float q[8];
      bf16x8_to_f32(qr[tq], q);
      float sc[TMAX];
      float mx = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 <= tq; ++s2) {
        float k[8];
        bf16x8_to_f32(kr[s2], k);
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(q[i], k[i], d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        sc[s2] = d * (0.125f * 1.4426950408889634f);
        mx = fmaxf(mx, sc[s2]);
      }
      float acc[8], l = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
      for (int s2 = 0; s2 <= tq; ++s2) {
        const float e = ex2_approx(sc[s2] - mx);
        float v[8];
        bf16x8_to_f32(vr[s2], v);
        l += e;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(e, v[i], acc[i]);
      }
      if (active) {
        const float inv = 1.f / l;
        *reinterpret_cast<uint4*>(obase + (long long)tq * P * HD) =
            make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                       pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
      }
    }
  }
}

// The same layout for any T <= 32: queries in blocks of four share each key
// row's loads (online softmax per query, keys past a query masked), so a
// (session, patch) reads its key rows about T / 8 times instead of T / 2.
__global__ void __launch_bounds__(128) attention_temporal_rows_long_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                           __nv_bfloat16* __restrict__ out,
                                                                           int batch, int T, int P, int H) {
  pdl_trigger();
  pdl_wait();
  constexpr int QB = 4;
  const int HD = H * kDh, ld = 3 * HD;
  const int wpr = (HD + kCachedWarpCols - 1) / kCachedWarpCols;
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)batch * P * wpr) return;  // warp-uniform
  const long long bp = w / wpr;
  const int part = (int)(w - bp * wpr);
  const int p = bp % P;
  const long long b = bp / P;
  int col = part * kCachedWarpCols + kCachedCols * lane;
  const bool active = col < HD;
  if (!active) col = 0;
  const __nv_bfloat16* base = qkv + (b * T * P + p) * ld + col;
  __nv_bfloat16* obase = out + (b * T * P + p) * (long long)HD + col;
  const long long fstride = (long long)P * ld;
  for (int t0 = 0; t0 < T; t0 += QB) {
    float q[QB][8], acc[QB][8], mx[QB], l[QB];
#pragma unroll
    for (int j = 0; j < QB; ++j) {
      const int tq = t0 + j < T ? t0 + j : T - 1;
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(base + tq * fstride)), q[j]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[j][i] *= 0.125f * 1.4426950408889634f;
        acc[j][i] = 0.f;
      }
      mx[j] = -INFINITY;
      l[j] = 0.f;
    }
    const int last = t0 + QB - 1 < T - 1 ? t0 + QB - 1 : T - 1;
    for (int s2 = 0; s2 <= last; ++s2) {
      float k[8], v[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(base + s2 * fstride + HD)), k);
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(base + s2 * fstride + 2 * HD)), v);
#pragma unroll
      for (int j = 0; j < QB; ++j) {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(q[j][i], k[i], d);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        if (s2 <= t0 + j) {  // causal
          const float mnew = fmaxf(mx[j], d);
          const float corr = ex2_approx(mx[j] - mnew);
          const float e = ex2_approx(d - mnew);
          l[j] = l[j] * corr + e;
          mx[j] = mnew;
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[j][i] = fmaf(e, v[i], acc[j][i] * corr);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < QB; ++j) {
      if (active && t0 + j < T) {
        const float inv = 1.f / l[j];
        *reinterpret_cast<uint4*>(obase + (long long)(t0 + j) * P * HD) = make_uint4(
            pack_bf16x2(acc[j][0] * inv, acc[j][1] * inv), pack_bf16x2(acc[j][2] * inv, acc[j][3] * inv),
            pack_bf16x2(acc[j][4] * inv, acc[j][5] * inv), pack_bf16x2(acc[j][6] * inv, acc[j][7] * inv));
      }
    }
  }
}

}  // namespace

int attention_temporal_cached_launch(const __nv_bfloat16* past, const __nv_bfloat16* cur, __nv_bfloat16* out,
                                     int batch, int past_frames, int P, int H, cudaStream_t s) {
  OASIS_REQUIRE(cur && out && (past || past_frames == 0), "attention_temporal_cached: null pointer");
  OASIS_REQUIRE(past_frames >= 0 && past_frames <= 31, "attention_temporal_cached: past_frames=%d outside [0, 31]",
                past_frames);
  OASIS_REQUIRE(H >= 1 && H <= 16, "attention_temporal_cached: heads=%d outside [1, 16]", H);
  const long long warps = (long long)batch * P * ((H * kDh + kCachedWarpCols - 1) / kCachedWarpCols);
  if (warps == 0) return OASIS_OK;
  const int tpb = warps < 8LL * num_sms() ? 64 : 256;  // few rows: small blocks spread over every SM
  const int grid = (int)((warps * 32 + tpb - 1) / tpb);
  launch_pdl(attention_temporal_cached_kernel, dim3(grid), dim3(tpb), 0, s, past, cur, out, batch, past_frames, P, H);
  return check_launch("attention_temporal_cached_kernel");
}

int attention_full_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int groups, int seq, int H, cudaStream_t s) {
  OASIS_REQUIRE(qkv && out, "attention_full: null pointer");
  OASIS_REQUIRE(groups >= 0 && seq > 0, "attention_full: bad shape");
  OASIS_REQUIRE(H >= 1 && H <= 16, "attention_full: heads=%d outside [1, 16]", H);
  if (groups == 0) return OASIS_OK;
  // The tcgen05 kernel (attention_tc.cu) runs every length it supports
  // (multiples of 144): measured 225 -> 207 us for 512 DiT frames and
  // 400 -> 243 us for 64 VAE frames against the mma.sync kernels below, which
  // serve other lengths. OASIS_ATTN_TC=0 selects the mma.sync kernels.
  static const bool use_tc = [] {
    const char* e = getenv("OASIS_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  if (use_tc && attention_tc_supported(seq)) return attention_tc_launch(qkv, out, groups, seq, H, s);
  if (seq == kSpatialSeq) {
    constexpr int smem = 2 * 3 * kSpatialTile * 2;
    static std::atomic<bool> attr[64];  // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
      cudaError_t e = cudaFuncSetAttribute(attention_spatial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr[dev & 63] = true;
    }
    const int items = groups * H;
    const int g2 = items < 2 * grid_sms() ? items : 2 * grid_sms();  // two CTAs per SM
    launch_pdl(attention_spatial_kernel, dim3(g2), dim3(kSpatialWarps * 32), smem, s, qkv, out, items, H);
  } else if (seq <= 160) {
    constexpr int NW = 3;  // 48 query rows per CTA
    dim3 grid((seq + NW * 16 - 1) / (NW * 16), H, groups);
    launch_pdl(attention_full_kernel<NW>, dim3(grid), dim3(NW * 32), 0, s, qkv, out, seq, H);
  } else if (seq % 96 == 0) {
    constexpr int NW = 6;  // 96 query rows per CTA: 576 = 6 x 96
    dim3 grid(seq / (NW * 16), H, groups);
    launch_pdl(attention_full_kernel<NW>, dim3(grid), dim3(NW * 32), 0, s, qkv, out, seq, H);
  } else {
    constexpr int NW = 4;
    dim3 grid((seq + NW * 16 - 1) / (NW * 16), H, groups);
    launch_pdl(attention_full_kernel<NW>, dim3(grid), dim3(NW * 32), 0, s, qkv, out, seq, H);
  }
  return check_launch("attention_full_kernel");
}

int attention_temporal_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, int batch, int frames, int P, int H,
                              cudaStream_t s) {
  OASIS_REQUIRE(qkv && out, "attention_temporal: null pointer");
  OASIS_REQUIRE(frames >= 1 && frames <= 32, "attention_temporal: frames=%d outside [1, 32]", frames);
  OASIS_REQUIRE(H >= 1 && H <= 16, "attention_temporal: heads=%d outside [1, 16]", H);
  const long long warps = (long long)batch * P * ((H * kDh + kCachedWarpCols - 1) / kCachedWarpCols);
  if (warps == 0) return OASIS_OK;
  const int grid = (int)((warps * 32 + 127) / 128);  // 4-warp blocks
  if (frames <= 2)
    launch_pdl(attention_temporal_rows_kernel<2>, dim3(grid), dim3(128), 0, s, qkv, out, batch, frames, P, H);
  else if (frames <= 4)
    launch_pdl(attention_temporal_rows_kernel<4>, dim3(grid), dim3(128), 0, s, qkv, out, batch, frames, P, H);
  else if (frames <= 8)
    launch_pdl(attention_temporal_rows_kernel<8>, dim3(grid), dim3(128), 0, s, qkv, out, batch, frames, P, H);
  else
    launch_pdl(attention_temporal_rows_long_kernel, dim3(grid), dim3(128), 0, s, qkv, out, batch, frames, P, H);
  return check_launch("attention_temporal_rows_kernel");
}

}  // namespace oasis
