// Peer-memory building blocks for the tensor-parallel collectives over NVLink
// (the reference's multi-chip all-reduce after the row-parallel projections,
// oasis_inference.py:1153-1201, on a mesh opened at :289-305).
//
// The bulk data moves on the copy engines (cudaMemcpyAsync into a peer's buffer
// opened through CUDA IPC), which leaves every SM to the projections; these
// kernels only carry the handshakes and the final sum:
//   - signal: one thread stores an epoch into a flag in a peer's memory
//     (release, system scope), after the copies ordered before it on the stream;
//   - wait: one warp polls this rank's flags from the other ranks (acquire,
//     system scope) until each reaches the epoch, with a time limit; past it the
//     kernel records kDevTimeoutPeer in the peer error word and returns, so the
//     context stays usable and the host reads the status;
//   - reduce: sum of the world's slots of a reduce-scatter in rank order in fp32,
//     written once in the partial type.
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "../../include/oasis_b200.h"
#include "status.h"

namespace oasis {
namespace {

constexpr int kDevTimeoutPeer = 16;  // a peer's flag did not reach the epoch in time
__device__ int g_peer_error = 0;

__device__ __forceinline__ long long global_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void peer_signal_kernel(int* flag, int value) {
  // the copies ordered before this kernel on the stream have completed; make
  // them visible system-wide before the flag that announces them
  asm volatile("fence.sc.sys;" ::: "memory");
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

// Lane i watches flags[i] (i < n, i != skip) until it reaches `target`.
__global__ void peer_wait_kernel(const int* flags, int n, int skip, int target, long long timeout_ns) {
  const int i = threadIdx.x;
  bool ok = true;
  if (i < n && i != skip) {
    const long long t0 = global_ns();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if (v - target >= 0) break;  // epochs compare modulo 2^32
      if (global_ns() - t0 > timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(200);
    }
  }
  if (!ok) atomicCAS(&g_peer_error, 0, kDevTimeoutPeer);
  __syncwarp();
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// dst[i] = sum over k < n, in order, of slot_k[i], where slot_k = staging + k
// stride except slot own_slot = own. Eight elements per thread per step.
template <typename T>
__global__ void __launch_bounds__(256) reduce_slots_kernel(T* __restrict__ dst, const T* __restrict__ staging,
                                                           long long stride, const T* __restrict__ own, int own_slot,
                                                           int n, long long count) {
  const long long groups = count / 8;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; ++k) {
      const T* src = (k == own_slot ? own : staging + k * stride) + g * 8;
      T v[8];
      if constexpr (sizeof(T) == 2) {
        *reinterpret_cast<uint4*>(v) = __ldcs(reinterpret_cast<const uint4*>(src));
      } else {
        *reinterpret_cast<float4*>(v) = __ldcs(reinterpret_cast<const float4*>(src));
        *reinterpret_cast<float4*>(v + 4) = __ldcs(reinterpret_cast<const float4*>(src) + 1);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += to_f(v[j]);
    }
    T o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = from_f<T>(acc[j]);
    if constexpr (sizeof(T) == 2) {
      *reinterpret_cast<uint4*>(dst + g * 8) = *reinterpret_cast<uint4*>(o);
    } else {
      *reinterpret_cast<float4*>(dst + g * 8) = *reinterpret_cast<float4*>(o);
      *reinterpret_cast<float4*>(dst + g * 8 + 4) = *reinterpret_cast<float4*>(o + 4);
    }
  }
}

cudaStream_t S(oasis_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

int read_device_error_peer(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(int));
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error (peer): %s", cudaGetErrorString(e));
  if (reset && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "device_error reset (peer): %s", cudaGetErrorString(e));
  }
  return v;
}

}  // namespace oasis

using namespace oasis;

extern "C" int oasis_peer_alloc(size_t bytes, void** ptr) {
  OASIS_REQUIRE(ptr && bytes > 0, "peer_alloc: bytes=%zu", bytes);
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "peer_alloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "peer_alloc memset: %s", cudaGetErrorString(e));
  return OASIS_OK;
}

extern "C" int oasis_peer_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
  return OASIS_OK;
}

extern "C" int oasis_ipc_get_handle(void* ptr, void* handle_out) {
  OASIS_REQUIRE(ptr && handle_out, "ipc_get_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == OASIS_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  return OASIS_OK;
}

extern "C" int oasis_ipc_open_handle(const void* handle, void** ptr) {
  OASIS_REQUIRE(handle && ptr, "ipc_open_handle: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return OASIS_OK;
}

extern "C" int oasis_ipc_close_handle(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return OASIS_OK;
}

extern "C" int oasis_peer_copy(void* dst, const void* src, size_t bytes, oasis_stream_t stream) {
  OASIS_REQUIRE(dst && src, "peer_copy: null pointer");
  if (!bytes) return OASIS_OK;
  // unified addressing: a destination in a peer's (IPC-opened) memory makes this
  // a copy-engine transfer over NVLink
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, S(stream));
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "peer_copy(%zu): %s", bytes, cudaGetErrorString(e));
  return OASIS_OK;
}

extern "C" int oasis_peer_signal(int* flag, int value, oasis_stream_t stream) {
  OASIS_REQUIRE(flag && (reinterpret_cast<uintptr_t>(flag) & 3) == 0, "peer_signal: flag not 4-byte aligned");
  peer_signal_kernel<<<1, 1, 0, S(stream)>>>(flag, value);
  return check_launch("peer_signal_kernel");
}

extern "C" int oasis_peer_wait(const int* flags, int n, int skip, int target, long long timeout_ns,
                               oasis_stream_t stream) {
  OASIS_REQUIRE(flags && n >= 1 && n <= 32, "peer_wait: n=%d (1..32 flags)", n);
  OASIS_REQUIRE(timeout_ns > 0, "peer_wait: timeout_ns=%lld", timeout_ns);
  peer_wait_kernel<<<1, 32, 0, S(stream)>>>(flags, n, skip, target, timeout_ns);
  return check_launch("peer_wait_kernel");
}

extern "C" int oasis_reduce_slots(void* dst, const void* staging, long long slot_stride, const void* own, int own_slot,
                                  int n, long long count, int dtype, oasis_stream_t stream) {
  OASIS_REQUIRE(dst && staging && own && n >= 1 && n <= 32 && own_slot >= 0 && own_slot < n,
                "reduce_slots: n=%d own_slot=%d", n, own_slot);
  OASIS_REQUIRE(count > 0 && count % 8 == 0 && slot_stride % 8 == 0, "reduce_slots: count=%lld stride=%lld (multiples of 8)",
                count, slot_stride);
  OASIS_REQUIRE(dtype == OASIS_DTYPE_F32 || dtype == OASIS_DTYPE_BF16, "reduce_slots: dtype=%d", dtype);
  OASIS_REQUIRE(((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(staging) |
                  reinterpret_cast<uintptr_t>(own)) & 15) == 0,
                "reduce_slots: buffers not 16-byte aligned");
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long groups = count / 8;
  long long blocks = (groups + 255) / 256;
  if (blocks > 4LL * sms) blocks = 4LL * sms;
  if (dtype == OASIS_DTYPE_F32)
    reduce_slots_kernel<float><<<(int)blocks, 256, 0, S(stream)>>>(
        static_cast<float*>(dst), static_cast<const float*>(staging), slot_stride, static_cast<const float*>(own),
        own_slot, n, count);
  else
    reduce_slots_kernel<__nv_bfloat16><<<(int)blocks, 256, 0, S(stream)>>>(
        static_cast<__nv_bfloat16*>(dst), static_cast<const __nv_bfloat16*>(staging), slot_stride,
        static_cast<const __nv_bfloat16*>(own), own_slot, n, count);
  return check_launch("reduce_slots_kernel");
}
