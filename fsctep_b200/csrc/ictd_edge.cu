// Per-edge kernels of the pure-cartesian-ictd path.
//
// edge_forward: geometry (pure_cartesian_ictd_layers_full.py:896-909), direction
//   harmonics Y_l(n) (ictd_irreps.py:371-402, 489-494), radial basis
//   soft_one_hot_linspace(...)*sqrt(nb) (:930-937) and the per-layer radial MLPs
//   fc / fc2_layers (:277-283, 693-699) -> gates.  One thread per edge; the MLP
//   weights of one layer sit in shared memory and every thread of a warp reads the
//   same weight at the same time (broadcast), so the loop is FMA-bound.
// edge_backward: recomputes the MLP activations and back-propagates the per-edge
//   dE/dgates and dE/dY into dE/dr_e (what autograd replays in the reference,
//   evaluation/calculator.py:158-159).
// forces_from_edges: F_i = sum_{e: src=i} g_e - sum_{e: dst=i} g_e  (r_e = pos[dst]-pos[src]+...),
//   two segmented reductions (CSR by dst, transpose CSR by src), no atomics.
#include <math.h>

#include "common.cuh"
#include "edge_common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"

namespace fsc {

constexpr int RAD_H = 64;       // hidden width of the radial MLPs (fixed by the reference)
constexpr int RAD_P = 11;       // gates per layer (paths)
constexpr int EDGE_TPB = 128;   // threads per block of the edge kernels
constexpr int EDGE_EPT = 4;     // edges per thread (weights reused across them)

struct RadialSmem {
  float w1[RAD_H * 16];
  float b1[RAD_H];
  float w2[RAD_H * RAD_H];
  float b2[RAD_H];
  float w3t[RAD_H * 12];   // transposed: [j][q], q < 11 (+pad)
  float b3[12];
};

__device__ __forceinline__ void load_radial(RadialSmem& s, const RadialW& W, int layer, int nb) {
  const float* w1 = W.w1 + (size_t)layer * RAD_H * nb;
  const float* w2 = W.w2 + (size_t)layer * RAD_H * RAD_H;
  const float* w3 = W.w3 + (size_t)layer * RAD_P * RAD_H;
  for (int i = threadIdx.x; i < RAD_H * nb; i += blockDim.x) s.w1[i] = w1[i];
  for (int i = threadIdx.x; i < RAD_H; i += blockDim.x) {
    s.b1[i] = W.b1[layer * RAD_H + i];
    s.b2[i] = W.b2[layer * RAD_H + i];
  }
  for (int i = threadIdx.x; i < RAD_H * RAD_H; i += blockDim.x) s.w2[i] = w2[i];
  for (int i = threadIdx.x; i < RAD_H * 12; i += blockDim.x) {
    int j = i / 12, q = i % 12;
    s.w3t[i] = q < RAD_P ? w3[q * RAD_H + j] : 0.f;
  }
  if (threadIdx.x < 12) s.b3[threadIdx.x] = threadIdx.x < RAD_P ? W.b3[layer * RAD_P + threadIdx.x] : 0.f;
}

// Radial MLP forward for one edge: gates[q] = W3 silu(W2 silu(W1 emb + b1) + b2) + b3.
__device__ __forceinline__ void radial_mlp(const RadialSmem& s, int nb, const float* emb, float* gates) {
  float h1[RAD_H];
#pragma unroll
  for (int k = 0; k < RAD_H; ++k) {
    float a = s.b1[k];
    for (int b = 0; b < nb; ++b) a = fmaf(s.w1[k * nb + b], emb[b], a);
    h1[k] = silu(a);
  }
#pragma unroll
  for (int q = 0; q < 12; ++q) gates[q] = s.b3[q];
  for (int j = 0; j < RAD_H; ++j) {
    float a = s.b2[j];
    const float4* w = reinterpret_cast<const float4*>(s.w2 + j * RAD_H);
#pragma unroll
    for (int k4 = 0; k4 < RAD_H / 4; ++k4) {
      float4 v = w[k4];
      a = fmaf(v.x, h1[4 * k4 + 0], a);
      a = fmaf(v.y, h1[4 * k4 + 1], a);
      a = fmaf(v.z, h1[4 * k4 + 2], a);
      a = fmaf(v.w, h1[4 * k4 + 3], a);
    }
    float h2 = silu(a);
    const float4* w3 = reinterpret_cast<const float4*>(s.w3t + j * 12);
#pragma unroll
    for (int q4 = 0; q4 < 3; ++q4) {
      float4 v = w3[q4];
      gates[4 * q4 + 0] = fmaf(v.x, h2, gates[4 * q4 + 0]);
      gates[4 * q4 + 1] = fmaf(v.y, h2, gates[4 * q4 + 1]);
      gates[4 * q4 + 2] = fmaf(v.z, h2, gates[4 * q4 + 2]);
      gates[4 * q4 + 3] = fmaf(v.w, h2, gates[4 * q4 + 3]);
    }
  }
}

__global__ void __launch_bounds__(EDGE_TPB) edge_forward_kernel(EdgeFwdArgs a) {
  extern __shared__ float4 smem_raw[];
  RadialSmem& s = *reinterpret_cast<RadialSmem*>(smem_raw);
  __shared__ float ypoly[ictd2::NMONO * ictd2::NK];
  for (int i = threadIdx.x; i < ictd2::NMONO * ictd2::NK; i += blockDim.x)
    ypoly[i] = a.tables[ictd2::TAB_YPOLY + i];
  const int64_t base = (int64_t)blockIdx.x * EDGE_TPB * EDGE_EPT;
  for (int layer = 0; layer < a.nint; ++layer) {
    __syncthreads();
    load_radial(s, a.rad, layer, a.nb);
    __syncthreads();
    for (int t = 0; t < EDGE_EPT; ++t) {
      const int64_t e = base + (int64_t)t * EDGE_TPB + threadIdx.x;
      if (e >= a.E) continue;
      float r[3];
      if (layer == 0) {
        const int i = a.src[e], j = a.dst[e];
        const int g = a.batch[i];
        const float* cell = a.cell + 9 * (int64_t)g;
        const float s0 = a.shift[3 * e + 0], s1 = a.shift[3 * e + 1], s2 = a.shift[3 * e + 2];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float sv = s0 * cell[c] + s1 * cell[3 + c] + s2 * cell[6 + c];
          r[c] = a.pos[3 * (int64_t)j + c] - a.pos[3 * (int64_t)i + c] + sv;
        }
        float len = sqrtf(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
        float inv = 1.f / fmaxf(len, 1e-8f);
        float mono[ictd2::NMONO];
        ictd2::monomials(r[0] * inv, r[1] * inv, r[2] * inv, mono);
        float* out = a.edge_y + 12 * e;
        float4* out4 = reinterpret_cast<float4*>(out);
        float y[12];
#pragma unroll
        for (int k = 0; k < ictd2::NK; ++k) {
          float v = 0.f;
#pragma unroll
          for (int m = 0; m < ictd2::NMONO; ++m) v = fmaf(ypoly[m * ictd2::NK + k], mono[m], v);
          y[k] = v;
        }
        y[9] = r[0]; y[10] = r[1]; y[11] = r[2];
        out4[0] = make_float4(y[0], y[1], y[2], y[3]);
        out4[1] = make_float4(y[4], y[5], y[6], y[7]);
        out4[2] = make_float4(y[8], y[9], y[10], y[11]);
      } else {
        const float* ey = a.edge_y + 12 * e;
        r[0] = ey[9]; r[1] = ey[10]; r[2] = ey[11];
      }
      const float len = sqrtf(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
      float emb[16];
      radial_basis<16>(a.basis_kind, a.nb, a.rc, len, emb, nullptr);
      float gates[12];
      radial_mlp(s, a.nb, emb, gates);
      float4* g4 = reinterpret_cast<float4*>(a.gates + ((int64_t)layer * a.E + e) * 12);
      g4[0] = make_float4(gates[0], gates[1], gates[2], gates[3]);
      g4[1] = make_float4(gates[4], gates[5], gates[6], gates[7]);
      g4[2] = make_float4(gates[8], gates[9], gates[10], 0.f);
    }
  }
}

__global__ void __launch_bounds__(EDGE_TPB) edge_backward_kernel(EdgeBwdArgs a) {
  extern __shared__ float4 smem_raw[];
  RadialSmem& s = *reinterpret_cast<RadialSmem*>(smem_raw);
  __shared__ float ypoly[ictd2::NMONO * ictd2::NK];
  for (int i = threadIdx.x; i < ictd2::NMONO * ictd2::NK; i += blockDim.x)
    ypoly[i] = a.tables[ictd2::TAB_YPOLY + i];
  const int64_t base = (int64_t)blockIdx.x * EDGE_TPB * EDGE_EPT;
  float dlen[EDGE_EPT];
#pragma unroll
  for (int t = 0; t < EDGE_EPT; ++t) dlen[t] = 0.f;
  for (int layer = 0; layer < a.nint; ++layer) {
    __syncthreads();
    load_radial(s, a.rad, layer, a.nb);
    __syncthreads();
#pragma unroll
    for (int t = 0; t < EDGE_EPT; ++t) {
      const int64_t e = base + (int64_t)t * EDGE_TPB + threadIdx.x;
      if (e >= a.E) continue;
      const float* ey = a.edge_y + 12 * e;
      const float len = sqrtf(ey[9] * ey[9] + ey[10] * ey[10] + ey[11] * ey[11]);
      float emb[16], demb[16];
      radial_basis<16>(a.basis_kind, a.nb, a.rc, len, emb, demb);
      float dg[12];
      const float4* dg4 = reinterpret_cast<const float4*>(a.dgates + ((int64_t)layer * a.E + e) * 12);
      {
        float4 v0 = dg4[0], v1 = dg4[1], v2 = dg4[2];
        dg[0] = v0.x; dg[1] = v0.y; dg[2] = v0.z; dg[3] = v0.w;
        dg[4] = v1.x; dg[5] = v1.y; dg[6] = v1.z; dg[7] = v1.w;
        dg[8] = v2.x; dg[9] = v2.y; dg[10] = v2.z; dg[11] = 0.f;
      }
      float h1[RAD_H], dh1[RAD_H];
#pragma unroll
      for (int k = 0; k < RAD_H; ++k) {
        float acc = s.b1[k];
        for (int b = 0; b < a.nb; ++b) acc = fmaf(s.w1[k * a.nb + b], emb[b], acc);
        h1[k] = silu(acc);
        dh1[k] = 0.f;
      }
      for (int j = 0; j < RAD_H; ++j) {
        float acc = s.b2[j];
        const float4* w = reinterpret_cast<const float4*>(s.w2 + j * RAD_H);
#pragma unroll
        for (int k4 = 0; k4 < RAD_H / 4; ++k4) {
          float4 v = w[k4];
          acc = fmaf(v.x, h1[4 * k4 + 0], acc);
          acc = fmaf(v.y, h1[4 * k4 + 1], acc);
          acc = fmaf(v.z, h1[4 * k4 + 2], acc);
          acc = fmaf(v.w, h1[4 * k4 + 3], acc);
        }
        const float* w3 = s.w3t + j * 12;
        float dh2 = 0.f;
#pragma unroll
        for (int q = 0; q < RAD_P; ++q) dh2 = fmaf(w3[q], dg[q], dh2);
        const float da2 = dh2 * silu_grad(acc);
#pragma unroll
        for (int k4 = 0; k4 < RAD_H / 4; ++k4) {
          float4 v = w[k4];
          dh1[4 * k4 + 0] = fmaf(v.x, da2, dh1[4 * k4 + 0]);
          dh1[4 * k4 + 1] = fmaf(v.y, da2, dh1[4 * k4 + 1]);
          dh1[4 * k4 + 2] = fmaf(v.z, da2, dh1[4 * k4 + 2]);
          dh1[4 * k4 + 3] = fmaf(v.w, da2, dh1[4 * k4 + 3]);
        }
      }
      float acc_len = 0.f;
#pragma unroll
      for (int k = 0; k < RAD_H; ++k) {
        float pre = s.b1[k];
        for (int b = 0; b < a.nb; ++b) pre = fmaf(s.w1[k * a.nb + b], emb[b], pre);
        const float da1 = dh1[k] * silu_grad(pre);
        for (int b = 0; b < a.nb; ++b) acc_len = fmaf(da1 * s.w1[k * a.nb + b], demb[b], acc_len);
      }
      dlen[t] += acc_len;
    }
  }
  // direction part and output
#pragma unroll
  for (int t = 0; t < EDGE_EPT; ++t) {
    const int64_t e = base + (int64_t)t * EDGE_TPB + threadIdx.x;
    if (e >= a.E) continue;
    const float* ey = a.edge_y + 12 * e;
    const float rx = ey[9], ry = ey[10], rz = ey[11];
    float dYe[ictd2::NK];
#pragma unroll
    for (int k = 0; k < ictd2::NK; ++k) dYe[k] = a.dY[12 * e + k];
    float gg3[3];
    edge_direction_grad(ypoly, rx, ry, rz, dYe, dlen[t], gg3);
    const float g0 = gg3[0], g1 = gg3[1], g2 = gg3[2];
    a.edge_grad[3 * e + 0] = g0;
    a.edge_grad[3 * e + 1] = g1;
    a.edge_grad[3 * e + 2] = g2;
    if (a.virial) {
      const int g = a.batch[a.src[e]];
      double* v = a.virial + 9 * (int64_t)g;
      const float rr[3] = {rx, ry, rz}, gg[3] = {g0, g1, g2};
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int q = 0; q < 3; ++q) atomicAdd(v + 3 * p + q, (double)(rr[p] * gg[q]));
    }
  }
}

// F_i = sum_{e: src=i} g_e - sum_{e: dst=i} g_e
__global__ void forces_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ tr_ptr,
                              const int32_t* __restrict__ tr_eid, const float* __restrict__ g,
                              float* __restrict__ F, int64_t N) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float fx = 0.f, fy = 0.f, fz = 0.f;
  for (int e = tr_ptr[n]; e < tr_ptr[n + 1]; ++e) {
    const int64_t id = tr_eid[e];
    fx += g[3 * id]; fy += g[3 * id + 1]; fz += g[3 * id + 2];
  }
  for (int e = row_ptr[n]; e < row_ptr[n + 1]; ++e) {
    fx -= g[3 * (int64_t)e]; fy -= g[3 * (int64_t)e + 1]; fz -= g[3 * (int64_t)e + 2];
  }
  F[3 * n] = fx; F[3 * n + 1] = fy; F[3 * n + 2] = fz;
}

// dst index of every edge from the CSR row pointers.
__global__ void edge_dst_kernel(const int32_t* __restrict__ row_ptr, int32_t* __restrict__ dst, int64_t N) {
  const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (n >= N) return;
  for (int e = row_ptr[n] + (threadIdx.x & 31); e < row_ptr[n + 1]; e += 32) dst[e] = (int32_t)n;
}

// Edge geometry only: r_e and Y(n_e) into edge_y (the layer-independent part of edge_forward).
__global__ void __launch_bounds__(256) edge_geom_kernel(EdgeFwdArgs a) {
  __shared__ float ypoly[ictd2::NMONO * ictd2::NK];
  for (int i = threadIdx.x; i < ictd2::NMONO * ictd2::NK; i += blockDim.x) ypoly[i] = a.tables[ictd2::TAB_YPOLY + i];
  __syncthreads();
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= a.E) return;
  const int i = a.src[e], j = a.dst[e];
  const float* cell = a.cell + 9 * (int64_t)a.batch[i];
  const float s0 = a.shift[3 * e + 0], s1 = a.shift[3 * e + 1], s2 = a.shift[3 * e + 2];
  float y[12];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float sv = s0 * cell[c] + s1 * cell[3 + c] + s2 * cell[6 + c];
    y[9 + c] = a.pos[3 * (int64_t)j + c] - a.pos[3 * (int64_t)i + c] + sv;
  }
  const float len = sqrtf(y[9] * y[9] + y[10] * y[10] + y[11] * y[11]);
  const float inv = 1.f / fmaxf(len, 1e-8f);
  float mono[ictd2::NMONO];
  ictd2::monomials(y[9] * inv, y[10] * inv, y[11] * inv, mono);
#pragma unroll
  for (int k = 0; k < ictd2::NK; ++k) {
    float v = 0.f;
#pragma unroll
    for (int m = 0; m < ictd2::NMONO; ++m) v = fmaf(ypoly[m * ictd2::NK + k], mono[m], v);
    y[k] = v;
  }
  float4* out4 = reinterpret_cast<float4*>(a.edge_y + 12 * e);
  out4[0] = make_float4(y[0], y[1], y[2], y[3]);
  out4[1] = make_float4(y[4], y[5], y[6], y[7]);
  out4[2] = make_float4(y[8], y[9], y[10], y[11]);
}

int launch_edge_geom(const EdgeFwdArgs& a, cudaStream_t st) {
  if (a.E == 0) return FSC_OK;
  edge_geom_kernel<<<(unsigned)ceil_div(a.E, 256), 256, 0, st>>>(a);
  return check_launch("edge_geom_kernel");
}

int launch_edge_forward(const EdgeFwdArgs& a, cudaStream_t st) {
  if (a.E == 0) return FSC_OK;
  const int64_t blocks = ceil_div(a.E, EDGE_TPB * EDGE_EPT);
  const size_t sm = sizeof(RadialSmem);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(edge_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    cudaFuncSetAttribute(edge_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    attr = true;
  }
  edge_forward_kernel<<<(unsigned)blocks, EDGE_TPB, sm, st>>>(a);
  return check_launch("edge_forward_kernel");
}

int launch_edge_backward(const EdgeBwdArgs& a, cudaStream_t st) {
  if (a.E == 0) return FSC_OK;
  const int64_t blocks = ceil_div(a.E, EDGE_TPB * EDGE_EPT);
  const size_t sm = sizeof(RadialSmem);
  cudaFuncSetAttribute(edge_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  edge_backward_kernel<<<(unsigned)blocks, EDGE_TPB, sm, st>>>(a);
  return check_launch("edge_backward_kernel");
}

int launch_forces(const int32_t* row_ptr, const int32_t* tr_ptr, const int32_t* tr_eid, const float* g,
                  float* F, int64_t N, cudaStream_t st) {
  if (N == 0) return FSC_OK;
  forces_kernel<<<(unsigned)ceil_div(N, 256), 256, 0, st>>>(row_ptr, tr_ptr, tr_eid, g, F, N);
  return check_launch("forces_kernel");
}

// Per transposed-CSR slot t: the receiver of edge tr_eid[t]; per node: 1 / max(in-degree, 1).
__global__ void transpose_aux_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ dst,
                                     const int32_t* __restrict__ tr_eid, int64_t N, int64_t E,
                                     int32_t* __restrict__ tr_dst, float* __restrict__ invdeg) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < E) tr_dst[i] = dst[tr_eid[i]];
  if (i < N) {
    const int d = row_ptr[i + 1] - row_ptr[i];
    invdeg[i] = 1.f / (float)(d > 1 ? d : 1);
  }
}

int launch_transpose_aux(const int32_t* row_ptr, const int32_t* dst, const int32_t* tr_eid, int64_t N, int64_t E,
                         int32_t* tr_dst, float* invdeg, cudaStream_t st) {
  const int64_t n = E > N ? E : N;
  if (n == 0) return FSC_OK;
  transpose_aux_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(row_ptr, dst, tr_eid, N, E, tr_dst, invdeg);
  return check_launch("transpose_aux_kernel");
}

int launch_edge_dst(const int32_t* row_ptr, int32_t* dst, int64_t N, cudaStream_t st) {
  if (N == 0) return FSC_OK;
  edge_dst_kernel<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(row_ptr, dst, N);
  return check_launch("edge_dst_kernel");
}

}  // namespace fsc
