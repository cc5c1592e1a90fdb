// Host-side status codes and the per-thread last-error message of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdio.h>

#define OASIS_OK 0
#define OASIS_ERR_INVALID_ARG (-1)
#define OASIS_ERR_CUDA (-2)
#define OASIS_ERR_WORKSPACE (-3)
#define OASIS_ERR_DEVICE_TIMEOUT (-4)
#define OASIS_ERR_UNSUPPORTED (-5)

namespace oasis {

// Records a printf-style message for oasis_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

// Host-side count of kernels this library has launched (all threads).
void count_launch();

inline int check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return OASIS_OK;
}

}  // namespace oasis

#define OASIS_REQUIRE(cond, ...)                                    \
  do {                                                              \
    if (!(cond)) return ::oasis::set_error(OASIS_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define OASIS_TRY(expr)          \
  do {                           \
    int _rc = (expr);            \
    if (_rc != OASIS_OK) return _rc; \
  } while (0)
