// Shared helpers for the fsctep_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "fsctep_b200.h"

namespace fsc {

// Per-host-thread message of the last failure (returned by fsc_last_error()).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FSC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return FSC_OK;
}

#define FSC_TRY(expr)            \
  do {                           \
    int _st = (expr);            \
    if (_st != FSC_OK) return _st; \
  } while (0)

#define FSC_REQUIRE(cond, msg)                                  \
  do {                                                          \
    if (!(cond)) return ::fsc::fail(FSC_ERR_ARGUMENT, (msg));   \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Bump allocator over a caller-provided workspace (256-byte aligned slices).
struct Arena {
  char* base;
  size_t cap;
  size_t off = 0;
  bool measuring;
  Arena(void* p, size_t n) : base(static_cast<char*>(p)), cap(n), measuring(p == nullptr) {}
  template <typename T>
  T* take(int64_t count) {
    size_t bytes = (static_cast<size_t>(count) * sizeof(T) + 255) & ~size_t(255);
    size_t at = off;
    off += bytes;
    if (measuring) return nullptr;
    return off <= cap ? reinterpret_cast<T*>(base + at) : nullptr;
  }
  bool ok() const { return measuring || off <= cap; }
};

// sigmoid through the hardware reciprocal (__fdividef, within 2 ulp); as x -> -inf the
// denominator overflows to +inf and the result is the exact limit 0.
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x * sigmoid_fast(x); }
// d silu / dx = s (1 + x (1 - s)), s = sigmoid(x)
__device__ __forceinline__ float silu_grad(float x) {
  const float s = sigmoid_fast(x);
  return s * (1.0f + x * (1.0f - s));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace fsc
