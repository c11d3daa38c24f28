// Generic fp32 SIMT GEMM with two-level row addressing (see GemmArgs in kernels.cuh).
// Used for the per-node channel mixes of the ICTD layers and the readout MLP.
// 64x64 output tile per block of 256 threads, 4x4 register tile per thread, K staged
// through shared memory in steps of 16.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace fsc {

constexpr int GT_M = 64, GT_N = 64, GT_K = 16;

__global__ void __launch_bounds__(256) gemm_kernel(GemmArgs a) {
  __shared__ float As[GT_K][GT_M + 4];
  __shared__ float Bs[GT_K][GT_N + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t M = a.G * (int64_t)a.R;
  const int64_t row0 = (int64_t)blockIdx.y * GT_M;
  const int col0 = blockIdx.x * GT_N;

  // rows this thread loads for A: lr = tid / 4 (0..63), k offsets (tid % 4) * 4 .. +3
  const int lr = tid >> 2, lk = (tid & 3) * 4;
  const int64_t arow = row0 + lr;
  const float* aptr = nullptr;
  if (arow < M) {
    const int64_t g = arow / a.R, r = arow % a.R;
    aptr = a.A + g * a.a_gs + r * a.a_rs;
  }
  // B loads: k = tid / 16 (0..15), cols (tid % 16) * 4 .. +3
  const int bk = tid >> 4, bc = (tid & 15) * 4;

  // Each K step of 16 is summed into a fresh partial and the partials are added with Kahan
  // compensation (long K with heavy cancellation: the readout Gram contraction, the sparse fc.4
  // products; 4 extra operations per 16 FMAs).
  float acc[4][4] = {}, comp[4][4] = {};
  for (int k0 = 0; k0 < a.K; k0 += GT_K) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + lk + j;
      As[lk + j][lr] = (aptr && k < a.K) ? aptr[k] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + bk, c = col0 + bc + j;
      float v = 0.f;
      if (k < a.K && c < a.N) v = a.b_trans ? a.B[(int64_t)c * a.ldb + k] : a.B[(int64_t)k * a.ldb + c];
      Bs[bk][bc + j] = v;
    }
    __syncthreads();
    float part[4][4] = {};
#pragma unroll
    for (int k = 0; k < GT_K; ++k) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) part[i][j] = fmaf(av[i], bv[j], part[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float y = part[i][j] - comp[i][j];
        const float t = acc[i][j] + y;
        comp[i][j] = (t - acc[i][j]) - y;
        acc[i][j] = t;
      }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + ty * 4 + i;
    if (row >= M) continue;
    const int64_t g = row / a.R, r = row % a.R;
    float scale = a.alpha != 0.f ? a.alpha : 1.f;
    if (a.deg_rowptr) {
      const int d = a.deg_rowptr[g + 1] - a.deg_rowptr[g];
      scale *= 1.f / (float)(d > 1 ? d : 1);
    }
    float* cptr = a.C + g * a.c_gs + r * a.c_rs;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = col0 + tx * 4 + j;
      if (c >= a.N) continue;
      float v = acc[i][j] * scale;
      if (a.bias) v += a.bias[c];
      if (a.accumulate) v += cptr[c];
      cptr[c] = v;
    }
  }
}

int launch_gemm(const GemmArgs& a, cudaStream_t st) {
  const int64_t M = a.G * (int64_t)a.R;
  if (M == 0 || a.N == 0) return FSC_OK;
  if (a.K < 0) return fail(FSC_ERR_ARGUMENT, "gemm: negative K");
  dim3 grid((unsigned)ceil_div(a.N, GT_N), (unsigned)ceil_div(M, GT_M));
  if (grid.y > 65535u) {
    // split along M in chunks of 65535 row tiles
    const int64_t rows_per = (int64_t)65535 * GT_M;
    for (int64_t m0 = 0; m0 < M; m0 += rows_per) {
      // chunks must align with row groups: require R divides rows_per, else fall back to per-group launch
      if (rows_per % a.R) return fail(FSC_ERR_UNSUPPORTED, "gemm: row count too large for this R");
      GemmArgs b = a;
      const int64_t g0 = m0 / a.R;
      b.G = std::min<int64_t>(a.G - g0, rows_per / a.R);
      b.A = a.A + g0 * a.a_gs;
      b.C = a.C + g0 * a.c_gs;
      if (a.deg_rowptr) b.deg_rowptr = a.deg_rowptr + g0;
      FSC_TRY(launch_gemm(b, st));
    }
    return FSC_OK;
  }
  gemm_kernel<<<grid, 256, 0, st>>>(a);
  return check_launch("gemm_kernel");
}

}  // namespace fsc
