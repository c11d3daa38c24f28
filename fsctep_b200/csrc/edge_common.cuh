// Per-edge device helpers shared by the CUDA-core and tensor-core edge kernels.
#pragma once

#include <math.h>

#include "common.cuh"
#include "ictd_paths.cuh"

namespace fsc {

// Radial basis value and derivative (e3nn soft_one_hot_linspace(..., cutoff=True) times sqrt(nb),
// pure_cartesian_ictd_layers_full.py:930-937).  Entries [nb, NB) are zero, so NB is a padded
// compile-time width and nb <= NB the configured number_of_basis.
template <int NB>
__device__ __forceinline__ void radial_basis(int kind, int nb, float rc, float x, float* emb, float* demb) {
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    emb[b] = 0.f;
    if (demb) demb[b] = 0.f;
  }
  const float scale = sqrtf((float)nb);
  if (kind == 0) {  // gaussian: exp(-((x - mu_b)/step)^2) / 1.12, mu_b = (b+1) step, step = rc/(nb+1)
    const float step = rc / (float)(nb + 1);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b < nb) {
        const float d = (x - (float)(b + 1) * step) / step;
        const float v = expf(-d * d) * (scale / 1.12f);
        emb[b] = v;
        if (demb) demb[b] = v * (-2.f * d / step);
      }
    }
  } else {  // bessel: sqrt(2/c) sin(b pi x / c) / x on 0 < x < c
    const float pre = sqrtf(2.f / rc) * scale;
    const bool inside = (x > 0.f) && (x / rc < 1.f);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b < nb) {
        const float w = (float)(b + 1) * 3.14159265358979323846f / rc;
        float s, c;
        sincosf(w * x, &s, &c);
        emb[b] = inside ? pre * s / x : 0.f;
        if (demb) demb[b] = inside ? pre * (w * c * x - s) / (x * x) : 0.f;
      }
    }
  }
}

// dE/dr of one edge from dE/d|r| (radial part, summed over layers) and dE/dY (direction part):
// Y = Y(n), n = r / max(|r|, 1e-8), dn/dr = (I - n n^T)/|r|.
__device__ __forceinline__ void edge_direction_grad(const float* ypoly, float rx, float ry, float rz,
                                                    const float* dY, float dl, float* g) {
  const float len = sqrtf(rx * rx + ry * ry + rz * rz);
  const float inv = 1.f / fmaxf(len, 1e-8f);
  const float nx = rx * inv, ny = ry * inv, nz = rz * inv;
  float gx[ictd2::NMONO], gy[ictd2::NMONO], gz[ictd2::NMONO];
  ictd2::monomial_grads(nx, ny, nz, gx, gy, gz);
  float dnx = 0.f, dny = 0.f, dnz = 0.f;
#pragma unroll
  for (int m = 0; m < ictd2::NMONO; ++m) {
    float w = 0.f;
#pragma unroll
    for (int k = 0; k < ictd2::NK; ++k) w = fmaf(ypoly[m * ictd2::NK + k], dY[k], w);
    dnx = fmaf(w, gx[m], dnx);
    dny = fmaf(w, gy[m], dny);
    dnz = fmaf(w, gz[m], dnz);
  }
  const float dot = dnx * nx + dny * ny + dnz * nz;
  if (len > 1e-8f) {
    g[0] = dl * nx + (dnx - dot * nx) * inv;
    g[1] = dl * ny + (dny - dot * ny) * inv;
    g[2] = dl * nz + (dnz - dot * nz) * inv;
  } else {
    g[0] = dl * nx + dnx * inv;
    g[1] = dl * ny + dny * inv;
    g[2] = dl * nz + dnz * inv;
  }
}

}  // namespace fsc
