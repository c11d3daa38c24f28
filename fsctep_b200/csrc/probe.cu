// FP32 CUDA-core throughput probe: the measured denominator of the CUDA-core kernels' FP32
// roofline (the conv2 tensor-product kernels).  Every thread runs 8 independent FMA chains in
// registers (scalar fmaf, or packed two-lane __ffma2_rn), enough warps per SM to hide the FMA
// latency; the caller times the launch with events on `stream`.
#include <cuda_runtime.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace fsc {
namespace {

constexpr int PROBE_THREADS = 256;
constexpr int PROBE_CHAINS = 8;

template <bool PACKED>
__global__ void __launch_bounds__(PROBE_THREADS) fma_probe_kernel(float* __restrict__ out, int iters, float b, float c) {
  float a[PROBE_CHAINS], d[PROBE_CHAINS];
#pragma unroll
  for (int j = 0; j < PROBE_CHAINS; ++j) {
    a[j] = (float)(threadIdx.x + j) * 1e-3f;
    d[j] = (float)(blockIdx.x + j) * 1e-3f;
  }
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 16; ++u) {
#pragma unroll
      for (int j = 0; j < PROBE_CHAINS; ++j) {
        if (PACKED) {
          const float2 t = __ffma2_rn(make_float2(a[j], d[j]), make_float2(b, b), make_float2(c, c));
          a[j] = t.x;
          d[j] = t.y;
        } else {
          a[j] = fmaf(a[j], b, c);
        }
      }
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PROBE_CHAINS; ++j) s += PACKED ? a[j] + d[j] : a[j];
  if (s == 12345.678f) out[blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the chains live
}

// One mbarrier of arrival count 1 that nothing arrives at; thread 0 waits for phase `parity` with
// the bounded wait of the tensor-core kernels (tc::mbar_wait), which records `where` in *err when
// it gives up.
__global__ void bounded_wait_probe_kernel(uint32_t parity, int where, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
    tc::mbar_wait(&bar, parity, err, where);
  }
}

}  // namespace
}  // namespace fsc

extern "C" int fsc_fp32_fma_probe(int packed, int blocks, int iters, float* out, double* flops, void* stream) {
  using namespace fsc;
  FSC_REQUIRE(blocks > 0 && iters > 0 && out && flops, "fsc_fp32_fma_probe: bad arguments");
  cudaStream_t st = as_stream(stream);
  // the multiplier keeps the chains bounded (|a| converges to c / (1 - b))
  if (packed)
    fma_probe_kernel<true><<<blocks, PROBE_THREADS, 0, st>>>(out, iters, 0.999f, 1e-4f);
  else
    fma_probe_kernel<false><<<blocks, PROBE_THREADS, 0, st>>>(out, iters, 0.999f, 1e-4f);
  *flops = 2.0 * (packed ? 2.0 : 1.0) * PROBE_CHAINS * 16.0 * (double)iters * (double)blocks * PROBE_THREADS;
  return check_launch("fma_probe_kernel");
}

extern "C" int fsc_bounded_wait_probe(int parity, int where, int* err_dev, void* stream) {
  using namespace fsc;
  FSC_REQUIRE(err_dev && (parity == 0 || parity == 1) && where != 0, "fsc_bounded_wait_probe: bad arguments");
  bounded_wait_probe_kernel<<<1, 32, 0, as_stream(stream)>>>((uint32_t)parity, where, err_dev);
  return check_launch("bounded_wait_probe_kernel");
}
