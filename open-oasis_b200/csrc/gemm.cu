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
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator, apply the fused op, store
// Two TMEM accumulators alternate so the epilogue of tile i overlaps the
// mainloop of tile i+1. Optional split-K: partial tiles go to a workspace and the
// last-arriving split (tile counter) sums them in split order (deterministic)
// before running the epilogue.
//
// Waits are bounded (see common.cuh); no TMA multicast is used anywhere.
#include <cudaTypedefs.h>
#include <mutex>
#include <stdio.h>

#include "common.cuh"
#include "gemm.cuh"
#include "status.h"

namespace oasis {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators; 128/256/512 (power of 2)
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 /*align slack*/ + STAGES * STAGE_BYTES + BAR_BYTES;
};

struct SplitK {
  float* partials;  // [tiles][splits][BM][BN]
  int* counters;    // [tiles]
  int splits;
};

// Applies the epilogue to 16 consecutive columns [n, n+16) of row r.
__device__ __forceinline__ void epilogue16(const EpiParams& e, int r, int n, int N, float (&v)[16]) {
  if (e.bias) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      float4 b = __ldg(reinterpret_cast<const float4*>(e.bias + n + i));
      v[i] += b.x; v[i + 1] += b.y; v[i + 2] += b.z; v[i + 3] += b.w;
    }
  }
  switch (e.mode) {
    case kEpiF32: {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + (long long)r * e.ldo + n);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      break;
    }
    case kEpiBF16:
    case kEpiGeluTanhBF16:
    case kEpiGeluErfBF16:
    case kEpiRopeBF16: {
      if (e.mode == kEpiGeluTanhBF16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = gelu_tanh(v[i]);
      } else if (e.mode == kEpiGeluErfBF16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = gelu_erf(v[i]);
      } else if (e.mode == kEpiRopeBF16 && n < 2 * e.rope_dim) {
        const int pos = (r / e.rope_div) % e.rope_mod;
        const int pair0 = (n & 63) >> 1;  // 16 columns never straddle a 64-wide head
        const float2* tab = reinterpret_cast<const float2*>(e.rope) + pos * 32 + pair0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 cs = __ldg(tab + j);
          const float x0 = v[2 * j], x1 = v[2 * j + 1];
          v[2 * j] = x0 * cs.x - x1 * cs.y;
          v[2 * j + 1] = x1 * cs.x + x0 * cs.y;
        }
      }
      uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(e.out) + (long long)r * e.ldo + n);
      o[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                        pack_bf16x2(v[6], v[7]));
      o[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                        pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
      break;
    }
    case kEpiGatedResid:
    case kEpiResid: {
      const float4* rs = reinterpret_cast<const float4*>(e.resid + (long long)r * e.ldr + n);
      float4 res[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) res[i] = rs[i];
      if (e.mode == kEpiGatedResid) {
        const float4* g = reinterpret_cast<const float4*>(
            e.gate + (long long)(r / e.rows_per_frame) * e.ldg + n);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 gg = __ldg(g + i);
          v[4 * i] *= gg.x; v[4 * i + 1] *= gg.y; v[4 * i + 2] *= gg.z; v[4 * i + 3] *= gg.w;
        }
      }
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(e.out) + (long long)r * e.ldo + n);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = make_float4(res[i].x + v[4 * i], res[i].y + v[4 * i + 1], res[i].z + v[4 * i + 2],
                           res[i].w + v[4 * i + 3]);
      break;
    }
    case kEpiImage: {
      // row r = frame * tokens + (hh * grid_w + ww); column n = ch * P*P + p * P + q
      const int P = e.img_patch;
      const int frame = r / e.img_tokens;
      const int tok = r - frame * e.img_tokens;
      const int hh = tok / e.img_grid_w, ww = tok - hh * e.img_grid_w;
      const int grid_h = e.img_tokens / e.img_grid_w;
      const long long H = (long long)grid_h * P, W = (long long)e.img_grid_w * P;
      float* img = static_cast<float*>(e.out) + (long long)frame * 3 * H * W;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int nn = n + i;
        if (nn < N) {
          const int ch = nn / (P * P);
          const int rem = nn - ch * P * P;
          const int p = rem / P, q = rem - p * P;
          const float x = fminf(1.f, fmaxf(-1.f, v[i]));
          img[(long long)ch * H * W + (long long)(hh * P + p) * W + (ww * P + q)] = x;
        }
      }
      break;
    }
    default:
      break;
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const int M, const int N, const int K, const EpiParams epi, const SplitK sk) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* sk_flag = reinterpret_cast<int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int splits = sk.splits;
  const int units = m_tiles * n_tiles * splits;
  const int kb_total = K / BK;
  const int kb_per_split = kb_total / splits;  // host guarantees divisibility

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
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

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int tile = u / splits, split = u - tile * splits;
        const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
        const int kb0 = split * kb_per_split;
        for (int kb = kb0; kb < kb0 + kb_per_split; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, kDevTimeoutSmemEmpty)) { ok = false; break; }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
          tma_load_2d(sa + C::A_BYTES, &tmW, &full[stage], kb * BK, n0);
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
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kb_per_split; ++kb) {
          if (!mbar_wait(&full[stage], phase, kDevTimeoutTmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint64_t adesc = smem_desc_sw128(a_addr);
          const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle atom
            tc_mma_bf16(d_tmem, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc,
                        (kb > 0 || k > 0) ? 1u : 0u);
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
    // ---------------- Epilogue (warps 2..5) ----------------
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const int ep_tid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int tile = u / splits, split = u - tile * splits;
      const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
      const int r = m0 + row_in_tile;
      if (!mbar_wait(&acc_full[acc], acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_off + acc * BN;
      if (splits == 1) {
#pragma unroll 1
        for (int c = 0; c < BN / 16; ++c) {
          const int n = n0 + c * 16;
          if (n >= N) break;  // warp-uniform
          float v[16];
          __syncwarp();
          tmem_ld16(t_acc + c * 16, v);
          if (r < M) epilogue16(epi, r, n, N, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
      } else {
        float* part = sk.partials + ((long long)tile * splits + split) * (BM * BN) + row_in_tile * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 16; ++c) {
          float v[16];
          __syncwarp();
          tmem_ld16(t_acc + c * 16, v);
          float4* dst = reinterpret_cast<float4*>(part + c * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i) __stcg(dst + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        __threadfence();
        named_barrier_sync(1, 128);
        if (ep_tid == 0) {
          const int prev = atomicAdd(&sk.counters[tile], 1);
          const int last = (prev == splits - 1);
          if (last) sk.counters[tile] = 0;  // every split has arrived: ready for the next launch
          *sk_flag = last;
        }
        named_barrier_sync(1, 128);
        if (*sk_flag) {
          __threadfence();
          const float* base = sk.partials + (long long)tile * splits * (BM * BN) + row_in_tile * BN;
#pragma unroll 1
          for (int c = 0; c < BN / 16; ++c) {
            const int n = n0 + c * 16;
            if (n >= N) break;
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int s = 0; s < splits; ++s) {
              const float4* src = reinterpret_cast<const float4*>(base + (long long)s * (BM * BN) + c * 16);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 x = __ldcg(src + i);
                v[4 * i] += x.x; v[4 * i + 1] += x.y; v[4 * i + 2] += x.z; v[4 * i + 3] += x.w;
              }
            }
            if (r < M) epilogue16(epi, r, n, N, v);
          }
        }
        named_barrier_sync(1, 128);  // sk_flag is reused by the next tile
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
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
int make_map(CUtensorMap* map, const void* ptr, long long rows, long long K, long long ld, int box_rows) {
  OASIS_TRY(get_encoder());
  OASIS_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "GEMM operand not 16-byte aligned");
  OASIS_REQUIRE((ld * 2) % 16 == 0, "GEMM operand row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OASIS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OASIS_OK;
}

int g_num_sms[64] = {0};

template <int BN>
int launch_bn(const GemmProblem& p, int splits, cudaStream_t stream) {
  using C = Cfg<BN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta, tw;
  OASIS_TRY(make_map(&ta, p.A, p.M, p.K, p.lda, BM));
  OASIS_TRY(make_map(&tw, p.W, p.N, p.K, p.K, BN));
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  SplitK sk{nullptr, nullptr, splits};
  if (splits > 1) {
    const size_t part_bytes = (size_t)tiles * splits * BM * BN * sizeof(float);
    const size_t need = part_bytes + (size_t)tiles * sizeof(int);
    if (!p.workspace || p.workspace_bytes < need)
      return set_error(OASIS_ERR_WORKSPACE, "split-K GEMM needs %zu workspace bytes, got %zu", need,
                       p.workspace_bytes);
    sk.partials = static_cast<float*>(p.workspace);
    sk.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(p.workspace) + part_bytes);
    cudaError_t e = cudaMemsetAsync(sk.counters, 0, (size_t)tiles * sizeof(int), stream);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "memset counters: %s", cudaGetErrorString(e));
  }
  const int units = tiles * splits;
  const int grid = units < num_sms() ? units : num_sms();
  gemm_kernel<BN><<<grid, kThreads, C::SMEM, stream>>>(ta, tw, p.M, p.N, p.K, p.epi, sk);
  return check_launch("gemm_kernel");
}

struct Plan {
  int bn;
  int splits;
};

Plan choose_plan(int M, int N, int K) {
  const int sms = num_sms();
  const int mt = (M + BM - 1) / BM;
  const int t256 = mt * ((N + 255) / 256);
  if (t256 >= sms && N % 256 == 0) return {256, 1};
  const int t128 = mt * ((N + 127) / 128);
  if (t128 >= sms) return {128, 1};
  // Small problems (a handful of sessions): narrow tiles, then split K until
  // there is roughly one work unit per SM so the weight stream uses all of HBM.
  const int t64 = mt * ((N + 63) / 64);
  const int kb = K / BK;
  int splits = 1;
  while (t64 * splits * 2 <= sms && kb % (splits * 2) == 0 && kb / (splits * 2) >= 4) splits *= 2;
  return {64, splits};
}

}  // namespace

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

size_t gemm_workspace_bytes(int M, int N, int K) {
  Plan pl = choose_plan(M, N, K);
  if (pl.splits <= 1) return 0;
  const size_t tiles = (size_t)((M + BM - 1) / BM) * ((N + pl.bn - 1) / pl.bn);
  return tiles * pl.splits * BM * pl.bn * sizeof(float) + tiles * sizeof(int);
}

int gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  OASIS_REQUIRE(p.A && p.W, "GEMM: null operand");
  OASIS_REQUIRE(p.M > 0 && p.N > 0 && p.K > 0, "GEMM: bad shape %d x %d x %d", p.M, p.N, p.K);
  OASIS_REQUIRE(p.K % BK == 0, "GEMM: K=%d must be a multiple of %d", p.K, BK);
  OASIS_REQUIRE(p.N % 16 == 0, "GEMM: N=%d must be a multiple of 16", p.N);
  OASIS_REQUIRE(p.epi.out, "GEMM: null output");
  OASIS_REQUIRE(p.lda >= p.K, "GEMM: lda < K");
  if (p.epi.mode == kEpiGatedResid || p.epi.mode == kEpiResid)
    OASIS_REQUIRE(p.epi.resid, "GEMM: residual epilogue without residual input");
  if (p.epi.mode == kEpiGatedResid) OASIS_REQUIRE(p.epi.gate && p.epi.rows_per_frame > 0, "GEMM: gate missing");
  if (p.epi.mode == kEpiRopeBF16) OASIS_REQUIRE(p.epi.rope && p.epi.rope_mod > 0 && p.epi.rope_div > 0, "GEMM: rope table missing");
  Plan pl = choose_plan(p.M, p.N, p.K);
  if (p.block_n) pl.bn = p.block_n;
  if (p.splits) pl.splits = p.splits;
  if (pl.splits > 1 && !p.workspace) pl.splits = 1;
  OASIS_REQUIRE((p.K / BK) % pl.splits == 0, "GEMM: splits=%d must divide K/64=%d", pl.splits, p.K / BK);
  switch (pl.bn) {
    case 64: return launch_bn<64>(p, pl.splits, stream);
    case 128: return launch_bn<128>(p, pl.splits, stream);
    case 256: return launch_bn<256>(p, pl.splits, stream);
    default: return set_error(OASIS_ERR_INVALID_ARG, "GEMM: block_n=%d unsupported", pl.bn);
  }
}

}  // namespace oasis

namespace oasis {

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
