// Message-passing kernels of the pure-cartesian-ictd path (lmax = 2, "full" paths).
//
// Reference computation (HarmonicFullyConnectedTensorProduct fast path, ictd_irreps.py:1003-1133,
// called from pure_cartesian_ictd_layers_full.py:938-951):
//   out_e[o, l3, kk] = sum_p gate_e[p] sum_{i} W[p,o,i] sum_{m1,m2} x[src,i,l1,m1] Y_{l2}[m2] CG_p[m1,m2,kk]
//   f_next[n] = (1/deg n) sum_{e: dst=n} out_e
// Here the channel mix W (edge independent) is moved after the aggregation:
//   Z[n, p, kk, i] = sum_{e->n} sum_{m1} x[src,i,l1,m1] * Yt_e[p,m1,kk]      (this file, SIMT)
//   f_next[n, l3, kk, o] = (1/deg) sum_{p in l3} sum_i W[p,o,i] Z[n,p,kk,i]  (GEMM, gemm.cu)
// which is the same sum in another order.  One warp owns one node; lanes own channels
// (c = lane + 32*j, j < C/32); the per-edge coupled harmonics Yt (115 values) are built
// once per edge by the warp into shared memory and read as broadcasts.
//
// conv1 (ICTDIrrepsE3Conv, pure_cartesian_ictd_layers_full.py:341-473): x2 holds only the l=0
// scalar Ai[dst], so only paths (l,0,l) contribute and
//   f1[n, l, k, o] = (1/deg) sum_i Vsp[Z_n, l, i, o] * S[n, l, k, i],
//   S[n, l, k, i]  = sum_{e->n} gate_e[p(l,0,l)] * Y1_e[l,k] * Ai[Z_src, i],
// with Vsp[s,l,i,o] = sum_j W1[p(l,0,l), o, i, j] Ai[s, j] precomputed per species.
#include "common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"

namespace fsc {

using namespace ictd2;

struct QTab {
  int8_t path[NQ];
  int8_t yb[NQ];
};

constexpr QTab make_qtab() {
  QTab t{};
  for (int p = 0; p < NP; ++p)
    for (int m1 = 0; m1 < 2 * L1(p) + 1; ++m1)
      for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
        const int q = qidx(p, m1, kk);
        t.path[q] = (int8_t)p;
        t.yb[q] = (int8_t)KB(L2(p));
      }
  return t;
}

__constant__ QTab c_qtab = make_qtab();

constexpr int CONV_WARPS = 4;

struct EdgeBuf {
  float y[12];
  float g[12];
  float yt[NQ + 1];
};

// Warp-cooperative: load Y and gates of edge e and build Yt (gated when `gated`).
__device__ __forceinline__ void build_yt(EdgeBuf& b, const float* __restrict__ cg2, const float* __restrict__ edge_y,
                                         const float* __restrict__ gates, int64_t e, int lane, bool gated) {
  if (lane < 12) b.y[lane] = edge_y[12 * e + lane];
  else if (lane < 24) b.g[lane - 12] = gates[12 * e + lane - 12];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = lane + 32 * j;
    if (q < NQ) {
      const int yb = c_qtab.yb[q];
      float v = 0.f;
#pragma unroll
      for (int m = 0; m < 5; ++m) v = fmaf(cg2[5 * q + m], b.y[yb + m], v);
      b.yt[q] = gated ? v * b.g[c_qtab.path[q]] : v;
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void load_cg2(float* cg2, const float* tables) {
  for (int i = threadIdx.x; i < NQ * 5; i += blockDim.x) cg2[i] = tables[TAB_CG2 + i];
}

// ---------------------------------------------------------------- conv2 forward: Z
template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32) conv2_z_kernel(ConvArgs a, const float* __restrict__ x,
                                                                  float* __restrict__ Z) {
  __shared__ float cg2[NQ * 5];
  __shared__ EdgeBuf bufs[CONV_WARPS];
  load_cg2(cg2, a.tables);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (n >= a.N) return;
  const int C = 32 * CPL;
  EdgeBuf& b = bufs[warp];
  float z[NZ][CPL];
#pragma unroll
  for (int r = 0; r < NZ; ++r)
#pragma unroll
    for (int c = 0; c < CPL; ++c) z[r][c] = 0.f;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  for (int e = e0; e < e1; ++e) {
    const int64_t s = a.src[e];
    if (s >= a.src_limit) {  // sender outside the previous layer's evaluated atoms
      if (lane == 0) atomicCAS(a.err, 0, 70);
      continue;
    }
    float xv[NK][CPL];
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) xv[k][c] = x[(s * NK + k) * C + lane + 32 * c];
    build_yt(b, cg2, a.edge_y, a.gates, e, lane, true);
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m1 = 0; m1 < 2 * L1(p) + 1; ++m1)
#pragma unroll
        for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
          const float w = b.yt[qidx(p, m1, kk)];
#pragma unroll
          for (int c = 0; c < CPL; ++c) z[zrow(p, kk)][c] = fmaf(xv[KB(L1(p)) + m1][c], w, z[zrow(p, kk)][c]);
        }
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < NZ; ++r)
#pragma unroll
    for (int c = 0; c < CPL; ++c) Z[(n * NZ + r) * C + lane + 32 * c] = z[r][c];
}

// ---------------------------------------------------------------- conv2 backward: R (src-centric)
template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32) conv2_r_kernel(ConvArgs a, const float* __restrict__ G,
                                                                  float* __restrict__ R) {
  __shared__ float cg2[NQ * 5];
  __shared__ EdgeBuf bufs[CONV_WARPS];
  load_cg2(cg2, a.tables);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t s = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (s >= a.N) return;
  const int C = 32 * CPL;
  EdgeBuf& b = bufs[warp];
  float r[NZ][CPL];
#pragma unroll
  for (int i = 0; i < NZ; ++i)
#pragma unroll
    for (int c = 0; c < CPL; ++c) r[i][c] = 0.f;
  const int t0 = a.tr_ptr[s], t1 = a.tr_ptr[s + 1];
  for (int t = t0; t < t1; ++t) {
    const int64_t e = a.tr_eid[t];
    const int64_t d = a.dst[e];
    if (d >= a.dst_limit) continue;  // receiver not evaluated in this layer: no gradient
    const int deg = a.row_ptr[d + 1] - a.row_ptr[d];
    const float inv = 1.f / (float)(deg > 1 ? deg : 1);
    float gv[NK][CPL];
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) gv[k][c] = G[(d * NK + k) * C + lane + 32 * c] * inv;
    build_yt(b, cg2, a.edge_y, a.gates, e, lane, true);
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m1 = 0; m1 < 2 * L1(p) + 1; ++m1)
#pragma unroll
        for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
          const float w = b.yt[qidx(p, m1, kk)];
#pragma unroll
          for (int c = 0; c < CPL; ++c) r[rrow(p, m1)][c] = fmaf(gv[KB(L3(p)) + kk][c], w, r[rrow(p, m1)][c]);
        }
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < NZ; ++i)
#pragma unroll
    for (int c = 0; c < CPL; ++c) R[(s * NZ + i) * C + lane + 32 * c] = r[i][c];
}

// ---------------------------------------------------------------- conv2 backward: gates and Y (dst-centric)
// One warp per dst node, one lane per incoming edge (rows longer than 32 take several passes).
// Per edge, over all channels:  Q[q] = sum_c x[src][KB(l1)+m1][c] * dZ[dst][zrow(p,kk)][c]
// (dZ already carries 1/deg), then
//   dgate[p]         = sum_{q in p} Q[q] * Yt0[q],     Yt0[q] = sum_m2 CG_p[m1,m2,kk] Y[KB(l2)+m2]
//   dY[KB(l2)+m2]   += sum_{q in p} Q[q] * gate[p] * CG_p[m1,m2,kk]
// Every reduction runs inside one thread: no cross-lane traffic.  dZ rows are read as 16-byte
// vectors that all lanes of the warp share (same node), x rows as 16-byte vectors per lane.
// Paths with l1 = G: p in [P_LO(G), P_HI(G)), their Q entries [QOFF(P_LO), QOFF(P_HI)).
__host__ __device__ constexpr int P_LO(int G) { return G == 0 ? 0 : (G == 1 ? 3 : 7); }
__host__ __device__ constexpr int P_HI(int G) { return G == 0 ? 3 : (G == 1 ? 7 : 11); }
__host__ __device__ constexpr int Q_END(int G) { return G == 2 ? NQ : QOFF(P_HI(G)); }

template <int G, int C>
__device__ __forceinline__ void q_group(const float4* __restrict__ x4, const float4* __restrict__ dz4,
                                        const float* __restrict__ cg2, const float* Y, const float* g, float* dg,
                                        float* dy) {
  constexpr int Q0 = QOFF(P_LO(G)), NQG = Q_END(G) - Q0, M1 = 2 * G + 1;
  float Q[NQG];
#pragma unroll
  for (int i = 0; i < NQG; ++i) Q[i] = 0.f;
#pragma unroll 1
  for (int c4 = 0; c4 < C / 4; ++c4) {
    float4 xv[M1];
#pragma unroll
    for (int m1 = 0; m1 < M1; ++m1) xv[m1] = x4[(KB(G) + m1) * (C / 4) + c4];
#pragma unroll
    for (int p = P_LO(G); p < P_HI(G); ++p)
#pragma unroll
      for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
        const float4 d = dz4[zrow(p, kk) * (C / 4) + c4];
#pragma unroll
        for (int m1 = 0; m1 < M1; ++m1) {
          float acc = Q[qidx(p, m1, kk) - Q0];
          acc = fmaf(xv[m1].x, d.x, acc);
          acc = fmaf(xv[m1].y, d.y, acc);
          acc = fmaf(xv[m1].z, d.z, acc);
          acc = fmaf(xv[m1].w, d.w, acc);
          Q[qidx(p, m1, kk) - Q0] = acc;
        }
      }
  }
#pragma unroll
  for (int p = P_LO(G); p < P_HI(G); ++p)
#pragma unroll
    for (int m1 = 0; m1 < M1; ++m1)
#pragma unroll
      for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
        const int q = qidx(p, m1, kk);
        float y0 = 0.f;
#pragma unroll
        for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2) y0 = fmaf(cg2[5 * q + m2], Y[KB(L2(p)) + m2], y0);
        dg[p] = fmaf(Q[q - Q0], y0, dg[p]);
        const float qg = Q[q - Q0] * g[p];
#pragma unroll
        for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2)
          dy[KB(L2(p)) + m2] = fmaf(qg, cg2[5 * q + m2], dy[KB(L2(p)) + m2]);
      }
}

template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32) conv2_q_kernel(ConvArgs a, const float* __restrict__ x,
                                                                  const float* __restrict__ dZ,
                                                                  float* __restrict__ dgates,
                                                                  float* __restrict__ dY) {
  __shared__ float cg2[NQ * 5];
  load_cg2(cg2, a.tables);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (n >= a.N) return;
  constexpr int C = 32 * CPL;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  if (n >= a.n_active) {  // receiver not evaluated in this layer: its edges' gate gradients are 0
    for (int e = e0 + lane; e < e1; e += 32) {
      float4* dgo = reinterpret_cast<float4*>(dgates + 12 * (int64_t)e);
      dgo[0] = dgo[1] = dgo[2] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  const float4* dz4 = reinterpret_cast<const float4*>(dZ + n * NZ * C);
  for (int base = e0; base < e1; base += 32) {
    const int e = base + lane;
    const bool active = e < e1;
    const int64_t ee = active ? e : e0;
    const int64_t s = a.src[ee];
    const float4* x4 = reinterpret_cast<const float4*>(x + s * NK * C);
    float Y[NK], g[NP], dg[NP], dy[NK];
#pragma unroll
    for (int k = 0; k < NK; ++k) {
      Y[k] = a.edge_y[12 * ee + k];
      dy[k] = 0.f;
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      g[p] = a.gates[12 * ee + p];
      dg[p] = 0.f;
    }
    q_group<0, C>(x4, dz4, cg2, Y, g, dg, dy);
    q_group<1, C>(x4, dz4, cg2, Y, g, dg, dy);
    q_group<2, C>(x4, dz4, cg2, Y, g, dg, dy);
    if (!active) continue;
    float4* dgo = reinterpret_cast<float4*>(dgates + 12 * (int64_t)e);
    dgo[0] = make_float4(dg[0], dg[1], dg[2], dg[3]);
    dgo[1] = make_float4(dg[4], dg[5], dg[6], dg[7]);
    dgo[2] = make_float4(dg[8], dg[9], dg[10], 0.f);
    float* dyo = dY + 12 * (int64_t)e;
#pragma unroll
    for (int k = 0; k < NK; ++k) dyo[k] += dy[k];
  }
}

// ---------------------------------------------------------------- conv1 forward
// Direction harmonics of conv1's first operand Ai[src] (x) Y_l; an external field adds the
// graph's l = 1 vector (pure_cartesian_ictd_layers_o3.py:466-502: f_in[1o] += scale t Ai[src]).
__device__ __forceinline__ void load_conv1_y(const ConvArgs& a, int64_t e, int64_t s, float* yv) {
  const float* y = a.edge_y + 12 * e;
#pragma unroll
  for (int k = 0; k < NK; ++k) yv[k] = y[k];
  if (a.field) {
    const float* f = a.field + 3 * (int64_t)a.batch[s];
    yv[1] += f[0];
    yv[2] += f[1];
    yv[3] += f[2];
  }
}

template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32) conv1_forward_kernel(ConvArgs a, const float* __restrict__ ai,
                                                                        const float* __restrict__ vsp,
                                                                        float* __restrict__ f1) {
  __shared__ float cg1[NK * 5];
  __shared__ float sbuf[CONV_WARPS][NK * 8];
  for (int i = threadIdx.x; i < NK * 5; i += blockDim.x) cg1[i] = a.tables[TAB_CG1 + i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (n >= a.N) return;
  const int C = 32 * CPL;
  // lane owns S entries q = lane + 32 j (q < 72): kidx = q / 8, i = q % 8
  float S[3] = {0.f, 0.f, 0.f};
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  for (int e = e0; e < e1; ++e) {
    const int64_t s = a.src[e];
    float yv[NK];
    load_conv1_y(a, e, s, yv);
    const float* g = a.gates + 12 * (int64_t)e;
    const float* A = ai + 8 * (int64_t)a.species[s];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int q = lane + 32 * j;
      if (q < NK * 8) {
        const int kidx = q >> 3, i = q & 7;
        const int l = kidx == 0 ? 0 : (kidx < 4 ? 1 : 2);
        float y1 = 0.f;
#pragma unroll
        for (int m = 0; m < 5; ++m) y1 = fmaf(cg1[5 * kidx + m], yv[KB(l) + m], y1);
        S[j] = fmaf(g[P1PATH(l)] * y1, A[i], S[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int q = lane + 32 * j;
    if (q < NK * 8) sbuf[warp][q] = S[j];
  }
  __syncwarp();
  const int deg = e1 - e0;
  const float inv = 1.f / (float)(deg > 1 ? deg : 1);
  const float* V = vsp + (int64_t)a.species[n] * 3 * 8 * C;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int o = lane + 32 * c;
    float v[3][8];
#pragma unroll
    for (int l = 0; l < 3; ++l)
#pragma unroll
      for (int i = 0; i < 8; ++i) v[l][i] = V[(l * 8 + i) * C + o];
#pragma unroll
    for (int kidx = 0; kidx < NK; ++kidx) {
      const int l = kidx == 0 ? 0 : (kidx < 4 ? 1 : 2);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf(v[l][i], sbuf[warp][kidx * 8 + i], acc);
      f1[(n * NK + kidx) * C + o] = acc * inv;
    }
  }
}

// ---------------------------------------------------------------- conv1 backward
// dS[kidx][i] = (1/deg) sum_o Vsp[Z_n, l, i, o] G1[n][kidx][o]; per edge (lane = edge):
//   dgate[p(l)] = sum_{k,i} dS[l,k,i] Y1[l,k] Ai[src,i];  dY1[l,k] = gate[p(l)] sum_i dS[l,k,i] Ai[src,i]
//   dY[l*l+m] += sum_k dY1[l,k] cg1[l*l+k][m]
template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32) conv1_backward_kernel(ConvArgs a, const float* __restrict__ ai,
                                                                         const float* __restrict__ vsp,
                                                                         const float* __restrict__ G1,
                                                                         float* __restrict__ dgates,
                                                                         float* __restrict__ dY) {
  __shared__ float cg1[NK * 5];
  __shared__ float ds[CONV_WARPS][NK * 8];
  for (int i = threadIdx.x; i < NK * 5; i += blockDim.x) cg1[i] = a.tables[TAB_CG1 + i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (n >= a.N) return;
  const int C = 32 * CPL;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  if (n >= a.n_active) {  // receiver not evaluated: zero gate gradients, no direction gradient
    for (int e = e0 + lane; e < e1; e += 32)
#pragma unroll
      for (int p = 0; p < 12; ++p) dgates[12 * (int64_t)e + p] = 0.f;
    return;
  }
  const int deg = e1 - e0;
  const float inv = 1.f / (float)(deg > 1 ? deg : 1);
  const float* V = vsp + (int64_t)a.species[n] * 3 * 8 * C;
  float gv[NK][CPL];
#pragma unroll
  for (int k = 0; k < NK; ++k)
#pragma unroll
    for (int c = 0; c < CPL; ++c) gv[k][c] = G1[(n * NK + k) * C + lane + 32 * c];
#pragma unroll
  for (int kidx = 0; kidx < NK; ++kidx) {
    const int l = kidx == 0 ? 0 : (kidx < 4 ? 1 : 2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float t = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) t = fmaf(V[(l * 8 + i) * C + lane + 32 * c], gv[kidx][c], t);
      t = warp_sum(t);
      if (lane == 0) ds[warp][kidx * 8 + i] = t * inv;
    }
  }
  __syncwarp();
  for (int e = e0 + lane; e < e1; e += 32) {
    const int64_t s = a.src[e];
    float yv[NK];
    load_conv1_y(a, e, s, yv);
    const float* g = a.gates + 12 * (int64_t)e;
    const float* A = ai + 8 * (int64_t)a.species[s];
    float Av[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) Av[i] = A[i];
    float dgl[3] = {0.f, 0.f, 0.f};
    float dy[NK];
#pragma unroll
    for (int k = 0; k < NK; ++k) dy[k] = 0.f;
#pragma unroll
    for (int kidx = 0; kidx < NK; ++kidx) {
      const int l = kidx == 0 ? 0 : (kidx < 4 ? 1 : 2);
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) t = fmaf(ds[warp][kidx * 8 + i], Av[i], t);
      float y1 = 0.f;
#pragma unroll
      for (int m = 0; m < 5; ++m) y1 = fmaf(cg1[5 * kidx + m], yv[KB(l) + m], y1);
      dgl[l] = fmaf(t, y1, dgl[l]);
      const float dy1 = t * g[P1PATH(l)];
#pragma unroll
      for (int m = 0; m < 5; ++m)
        if (KB(l) + m < NK) dy[KB(l) + m] = fmaf(dy1, cg1[5 * kidx + m], dy[KB(l) + m]);
    }
    float* dgo = dgates + 12 * (int64_t)e;
#pragma unroll
    for (int p = 0; p < 12; ++p) dgo[p] = 0.f;
    dgo[P1PATH(0)] = dgl[0];
    dgo[P1PATH(1)] = dgl[1];
    dgo[P1PATH(2)] = dgl[2];
    float* dyo = dY + 12 * (int64_t)e;
#pragma unroll
    for (int k = 0; k < NK; ++k) dyo[k] += dy[k];
  }
}

// ---------------------------------------------------------------- launchers
#define FSC_CONV_LAUNCH(KERNEL, ...)                                                        \
  do {                                                                                      \
    const unsigned blocks = (unsigned)ceil_div(a.N, CONV_WARPS);                            \
    if (a.N == 0) return FSC_OK;                                                            \
    if (a.C == 32) KERNEL<1><<<blocks, CONV_WARPS * 32, 0, st>>>(__VA_ARGS__);              \
    else if (a.C == 64) KERNEL<2><<<blocks, CONV_WARPS * 32, 0, st>>>(__VA_ARGS__);         \
    else return fail(FSC_ERR_UNSUPPORTED, "ictd conv kernels support channels 32 or 64");   \
    return check_launch(#KERNEL);                                                           \
  } while (0)

int launch_conv1_forward(const ConvArgs& a, const float* ai, const float* vsp, float* f1, cudaStream_t st) {
  FSC_CONV_LAUNCH(conv1_forward_kernel, a, ai, vsp, f1);
}
int launch_conv1_backward(const ConvArgs& a, const float* ai, const float* vsp, const float* G1, float* dgates,
                          float* dY, cudaStream_t st) {
  FSC_CONV_LAUNCH(conv1_backward_kernel, a, ai, vsp, G1, dgates, dY);
}
int launch_conv2_z(const ConvArgs& a, const float* x, float* Z, cudaStream_t st) {
  FSC_CONV_LAUNCH(conv2_z_kernel, a, x, Z);
}
int launch_conv2_r(const ConvArgs& a, const float* G, float* R, cudaStream_t st) {
  FSC_CONV_LAUNCH(conv2_r_kernel, a, G, R);
}
int launch_conv2_q(const ConvArgs& a, const float* x, const float* dZ, float* dgates, float* dY,
                   cudaStream_t st) {
  FSC_CONV_LAUNCH(conv2_q_kernel, a, x, dZ, dgates, dY);
}

}  // namespace fsc
