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
// once per edge (one lane per edge, 32 edges at a time) into shared memory and read as
// broadcasts.
//
// conv1 (ICTDIrrepsE3Conv, pure_cartesian_ictd_layers_full.py:341-473): x2 holds only the l=0
// scalar Ai[dst], so only paths (l,0,l) contribute and
//   f1[n, l, k, o] = (1/deg) sum_i Vsp[Z_n, l, i, o] * S[n, l, k, i],
//   S[n, l, k, i]  = sum_{e->n} gate_e[p(l,0,l)] * Y1_e[l,k] * Ai[Z_src, i],
// with Vsp[s,l,i,o] = sum_j W1[p(l,0,l), o, i, j] Ai[s, j] precomputed per species.
#include <algorithm>

#include "common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"

namespace fsc {

using namespace ictd2;

constexpr int CONV_WARPS = 4;

// Node walk of the conv2 kernels.  With a work counter, warps take nodes in increasing order as
// they free up (a persistent grid that keeps the nodes in flight, and so their neighbours' rows,
// close together); without one, every warp owns one node.
__device__ __forceinline__ int64_t take_node(int* work, int lane) {
  int v = 0;
  if (lane == 0) v = atomicAdd(work, 1);
  return __shfl_sync(0xffffffffu, v, 0);
}
__device__ __forceinline__ int64_t first_node(const ConvArgs& a, int warp, int lane) {
  return a.work ? take_node(a.work, lane) : (int64_t)blockIdx.x * CONV_WARPS + warp;
}
__device__ __forceinline__ int64_t next_node(const ConvArgs& a, int lane) {
  return a.work ? take_node(a.work, lane) : a.N;
}

// Per-edge coupled harmonics are stored with every path's block padded to a multiple of 4
// entries (offsets QPOFF), so a path's weights are read as 16-byte shared-memory vectors.
__host__ __device__ constexpr int QPOFF(int p) {
  switch (p) {
    case 0: return 0;
    case 1: return 4;
    case 2: return 8;
    case 3: return 16;
    case 4: return 28;
    case 5: return 32;
    case 6: return 48;
    case 7: return 60;
    case 8: return 88;
    case 9: return 104;
    default: return 112;  // p = 10
  }
}
constexpr int NQP = 140;                      // padded row; NQP / 4 odd: 16-byte stores by 8 lanes hit 8 bank groups
__host__ __device__ constexpr int NPATHQ(int p) { return (2 * L1(p) + 1) * (2 * L3(p) + 1); }

constexpr int YT_EDGES = 32;                  // edges whose Yt rows a warp holds at once
constexpr int CG2_FLOATS = (NQ * 5 + 3) / 4 * 4;
constexpr uint32_t ZR_SMEM = 4u * (CG2_FLOATS + CONV_WARPS * YT_EDGES * NQP);

__device__ __forceinline__ void load_cg2(float* cg2, const float* tables) {
  for (int i = threadIdx.x; i < NQ * 5; i += blockDim.x) cg2[i] = tables[TAB_CG2 + i];
}

// One edge's coupled harmonics (the calling lane's), Yt[q] = gate_p sum_m cg2[q][m] Y[KB(l2)+m],
// written to its padded row with 16-byte stores.  Y and g: the edge's 9 harmonics and 11 gates.
__device__ __forceinline__ void build_yt_row(float* __restrict__ row, const float* __restrict__ cg2, const float* Y,
                                             const float* g) {
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    float v[28];
#pragma unroll
    for (int i = 0; i < 28; ++i) {
      if (i < NPATHQ(p)) {
        const int q = QOFF(p) + i;
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < 2 * L2(p) + 1; ++m) acc = fmaf(cg2[5 * q + m], Y[KB(L2(p)) + m], acc);
        v[i] = acc * g[p];
      } else {
        v[i] = 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < (NPATHQ(p) + 3) / 4; ++i)
      reinterpret_cast<float4*>(row + QPOFF(p))[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

// The 12-float rows of edge e in edge_y and gates.
__device__ __forceinline__ void load_edge_yg(const ConvArgs& a, int64_t e, float* Y, float* g) {
  const float4* y4 = reinterpret_cast<const float4*>(a.edge_y + 12 * e);
  const float4* g4 = reinterpret_cast<const float4*>(a.gates + 12 * e);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float4 u = y4[i], v = g4[i];
    Y[4 * i] = u.x; Y[4 * i + 1] = u.y; Y[4 * i + 2] = u.z; Y[4 * i + 3] = u.w;
    g[4 * i] = v.x; g[4 * i + 1] = v.y; g[4 * i + 2] = v.z; g[4 * i + 3] = v.w;
  }
}

// Path p's (2 l1 + 1) x (2 l3 + 1) weights (m1-major) from a padded Yt row into registers.
template <int P>
__device__ __forceinline__ void path_weights(const float* __restrict__ yt, float* w) {
  constexpr int n = NPATHQ(P);
  const float4* v4 = reinterpret_cast<const float4*>(yt + QPOFF(P));
#pragma unroll
  for (int i = 0; i < (n + 3) / 4; ++i) {
    const float4 v = v4[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}

// acc[c] += x[c] * w over this lane's channels; two channels go through one packed fp32 FMA.
template <int CPL>
__device__ __forceinline__ void fma_ch(const float (&x)[CPL], float w, float (&acc)[CPL]) {
  if constexpr (CPL == 2) {
    const float2 t = __ffma2_rn(make_float2(x[0], x[1]), make_float2(w, w), make_float2(acc[0], acc[1]));
    acc[0] = t.x;
    acc[1] = t.y;
  } else {
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = fmaf(x[c], w, acc[c]);
  }
}

template <int P, int CPL>
__device__ __forceinline__ void z_path(const float* yt, const float (&xv)[NK][CPL], float (&z)[NZ][CPL]) {
  float w[28];
  path_weights<P>(yt, w);
  constexpr int n3 = 2 * L3(P) + 1;
#pragma unroll
  for (int m1 = 0; m1 < 2 * L1(P) + 1; ++m1)
#pragma unroll
    for (int kk = 0; kk < n3; ++kk) fma_ch<CPL>(xv[KB(L1(P)) + m1], w[m1 * n3 + kk], z[zrow(P, kk)]);
}

template <int P, int CPL>
__device__ __forceinline__ void r_path(const float* yt, const float (&gv)[NK][CPL], float (&r)[NZ][CPL]) {
  float w[28];
  path_weights<P>(yt, w);
  constexpr int n3 = 2 * L3(P) + 1;
#pragma unroll
  for (int m1 = 0; m1 < 2 * L1(P) + 1; ++m1)
#pragma unroll
    for (int kk = 0; kk < n3; ++kk) fma_ch<CPL>(gv[KB(L3(P)) + kk], w[m1 * n3 + kk], r[rrow(P, m1)]);
}

template <int CPL, template <int, int> class F, typename... T>
__device__ __forceinline__ void all_paths(T&... t) {
  F<0, CPL>::run(t...); F<1, CPL>::run(t...); F<2, CPL>::run(t...); F<3, CPL>::run(t...);
  F<4, CPL>::run(t...); F<5, CPL>::run(t...); F<6, CPL>::run(t...); F<7, CPL>::run(t...);
  F<8, CPL>::run(t...); F<9, CPL>::run(t...); F<10, CPL>::run(t...);
}
template <int P, int CPL>
struct ZPath {
  __device__ __forceinline__ static void run(const float* yt, const float (&xv)[NK][CPL], float (&z)[NZ][CPL]) {
    z_path<P, CPL>(yt, xv, z);
  }
};
template <int P, int CPL>
struct RPath {
  __device__ __forceinline__ static void run(const float* yt, const float (&gv)[NK][CPL], float (&r)[NZ][CPL]) {
    r_path<P, CPL>(yt, gv, r);
  }
};

// ---------------------------------------------------------------- conv2 forward: Z
// Edges are taken 32 at a time: each lane builds the Yt row of one edge (lane = edge) into the
// warp's shared-memory rows and holds its sender; then the warp walks the edges (lanes =
// channels), the next edge's sender row loaded while the current edge is contracted.
template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32, 3) conv2_z_kernel(ConvArgs a, const float* __restrict__ x,
                                                                     float* __restrict__ Z) {
  extern __shared__ float4 zr_smem4[];
  float* cg2 = reinterpret_cast<float*>(zr_smem4);
  load_cg2(cg2, a.tables);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t n = first_node(a, warp, lane); n < a.N; n = next_node(a, lane)) {
    constexpr int C = 32 * CPL;
    float* yt = cg2 + CG2_FLOATS + warp * YT_EDGES * NQP;
    float z[NZ][CPL];
#pragma unroll
    for (int r = 0; r < NZ; ++r)
#pragma unroll
      for (int c = 0; c < CPL; ++c) z[r][c] = 0.f;
    const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
    for (int blk = e0; blk < e1; blk += YT_EDGES) {
      const int nb = min(YT_EDGES, e1 - blk);
      int my_src = 0;
      __syncwarp();  // the previous block's rows are read
      if (lane < nb) {
        float Y[12], g[12];
        my_src = a.src[blk + lane];
        load_edge_yg(a, blk + lane, Y, g);
        build_yt_row(yt + lane * NQP, cg2, Y, g);
      }
      __syncwarp();
      // a sender outside the previous layer's evaluated atoms is skipped and flagged
      auto fetch = [&](int j, float (&xd)[NK][CPL]) -> bool {
        const int64_t s = __shfl_sync(0xffffffffu, my_src, j);
        const bool ok = s < a.src_limit;
#pragma unroll
        for (int k = 0; k < NK; ++k)
#pragma unroll
          for (int c = 0; c < CPL; ++c) xd[k][c] = ok ? __ldcg(x + (s * NK + k) * C + lane + 32 * c) : 0.f;
        return ok;
      };
      float xv[NK][CPL];
      bool ok = fetch(0, xv);
      for (int j = 0; j < nb; ++j) {
        float xn[NK][CPL];
        bool okn = true;
        if (j + 1 < nb) okn = fetch(j + 1, xn);
        if (ok) {
          const float* row = yt + j * NQP;
          all_paths<CPL, ZPath>(row, xv, z);
        } else if (lane == 0) {
          atomicCAS(a.err, 0, 70);
        }
#pragma unroll
        for (int k = 0; k < NK; ++k)
#pragma unroll
          for (int c = 0; c < CPL; ++c) xv[k][c] = xn[k][c];
        ok = okn;
      }
    }
#pragma unroll
    for (int r = 0; r < NZ; ++r)
#pragma unroll
      for (int c = 0; c < CPL; ++c) Z[(n * NZ + r) * C + lane + 32 * c] = z[r][c];
  }
}

// ---------------------------------------------------------------- conv2 backward: R (src-centric)
// Same blocking as conv2_z over the sender's out-edges (transposed order); the receivers are
// precomputed, so no dependent index chain runs through dst[e].
template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32, 3) conv2_r_kernel(ConvArgs a, const float* __restrict__ G,
                                                                     float* __restrict__ R) {
  extern __shared__ float4 zr_smem4[];
  float* cg2 = reinterpret_cast<float*>(zr_smem4);
  load_cg2(cg2, a.tables);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t s = first_node(a, warp, lane); s < a.N; s = next_node(a, lane)) {
    constexpr int C = 32 * CPL;
    float* yt = cg2 + CG2_FLOATS + warp * YT_EDGES * NQP;
    float r[NZ][CPL];
#pragma unroll
    for (int i = 0; i < NZ; ++i)
#pragma unroll
      for (int c = 0; c < CPL; ++c) r[i][c] = 0.f;
    const int t0 = a.tr_ptr[s], t1 = a.tr_ptr[s + 1];
    for (int blk = t0; blk < t1; blk += YT_EDGES) {
      const int nb = min(YT_EDGES, t1 - blk);
      int my_dst = 0;
      float my_inv = 0.f;  // 1/deg(dst), 0 for a receiver not evaluated in this layer
      __syncwarp();  // the previous block's rows are read
      if (lane < nb) {
        const int64_t e = a.tr_eid[blk + lane];
        my_dst = a.tr_dst[blk + lane];
        my_inv = my_dst < a.dst_limit ? a.invdeg[my_dst] : 0.f;
        float Y[12], g[12];
        load_edge_yg(a, e, Y, g);
        build_yt_row(yt + lane * NQP, cg2, Y, g);
      }
      __syncwarp();
      auto fetch = [&](int j, float (&gd)[NK][CPL]) -> bool {
        const int64_t d = __shfl_sync(0xffffffffu, my_dst, j);
        const float inv = __shfl_sync(0xffffffffu, my_inv, j);
        const bool on = d < a.dst_limit;
#pragma unroll
        for (int k = 0; k < NK; ++k)
#pragma unroll
          for (int c = 0; c < CPL; ++c) gd[k][c] = on ? __ldcg(G + (d * NK + k) * C + lane + 32 * c) * inv : 0.f;
        return on;
      };
      float gv[NK][CPL];
      bool on = fetch(0, gv);
      for (int j = 0; j < nb; ++j) {
        float gn[NK][CPL];
        bool onn = false;
        if (j + 1 < nb) onn = fetch(j + 1, gn);
        if (on) {
          const float* row = yt + j * NQP;
          all_paths<CPL, RPath>(row, gv, r);
        }
#pragma unroll
        for (int k = 0; k < NK; ++k)
#pragma unroll
          for (int c = 0; c < CPL; ++c) gv[k][c] = gn[k][c];
        on = onn;
      }
    }
#pragma unroll
    for (int i = 0; i < NZ; ++i)
#pragma unroll
      for (int c = 0; c < CPL; ++c) R[(s * NZ + i) * C + lane + 32 * c] = r[i][c];
  }
}

// ---------------------------------------------------------------- conv2 backward: gates and Y (dst-centric)
// One warp per dst node, one lane per incoming edge (rows longer than 32 take several passes).
// Per edge, over all channels:  Q[q] = sum_c x[src][KB(l1)+m1][c] * dZ[dst][zrow(p,kk)][c]
// (dZ already carries 1/deg), then
//   dgate[p]         = sum_{q in p} Q[q] * Yt0[q],     Yt0[q] = sum_m2 CG_p[m1,m2,kk] Y[KB(l2)+m2]
//   dY[KB(l2)+m2]   += sum_{q in p} Q[q] * gate[p] * CG_p[m1,m2,kk]
// Every reduction runs inside one thread: no cross-lane traffic.  The sender rows of the warp's 32
// edges are staged in shared memory one (l1 group, 16-channel chunk) step at a time by coalesced
// 16-byte asynchronous copies (four lanes per 64-byte row chunk), double-buffered so that the
// next step's copies run under this step's arithmetic; each lane then reads its own edge's rows
// from there, and the dZ rows of the step (same node for all lanes) as broadcasts.  Q is
// accumulated as even / odd channel partial sums with packed fp32 FMAs (two channels per
// instruction).
constexpr int QCH = 16;                       // channels per staged chunk
constexpr int QRMAX = 3;                      // sender rows per pass (the l1 = 2 group in two passes)
constexpr int QES = 4 * QRMAX + 1;            // float4 slots per edge in a chunk (odd: no bank conflicts)
constexpr int QZR = 14;                       // dZ rows of the largest l1 group
constexpr int QBUF_F4 = 32 * QES + 4 * QZR;   // one step: sender rows, then dZ rows
constexpr int QTAB_F4 = (NQ * 5 + 3) / 4 + 9; // cg2, then the dZ row list of every group (35 ints)
constexpr uint32_t QSMEM = 16u * (QTAB_F4 + CONV_WARPS * 2 * QBUF_F4);

// Local index of (p, kk) among the dZ rows of p's l1 group: rows are listed path by path.
__host__ __device__ constexpr int zlocal(int p, int kk) {
  int j = 0;
  for (int pp = P_LO(L1(p)); pp < p; ++pp) j += 2 * L3(pp) + 1;
  return j + kk;
}
__host__ __device__ constexpr int zcount(int G) { return zlocal(P_HI(G) - 1, 2 * L3(P_HI(G) - 1)) + 1; }
__host__ __device__ constexpr int zbase(int G) { return G == 0 ? 0 : (G == 1 ? zcount(0) : zcount(0) + zcount(1)); }

// A pass covers the sender rows m1 in [R0, R1) of l1 group G; its Q entries (p, m1, kk) are held
// path by path, then row by row.
template <int G, int R0, int R1>
__host__ __device__ constexpr int qloc(int p, int m1, int kk) {
  int j = 0;
  for (int pp = P_LO(G); pp < p; ++pp) j += (R1 - R0) * (2 * L3(pp) + 1);
  return j + (m1 - R0) * (2 * L3(p) + 1) + kk;
}
template <int G, int R0, int R1>
__host__ __device__ constexpr int qcount() {
  return qloc<G, R0, R1>(P_HI(G) - 1, R1 - 1, 2 * L3(P_HI(G) - 1)) + 1;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Issues the copies of step (pass, cc) into `buf` as one group: 32 edges x (R1 - R0) rows x 4
// float4 (lane copies slots f = lane + 32 i, f = (edge, row, c4)), then the group's dZ rows.
template <int G, int R0, int R1, int C>
__device__ __forceinline__ void q_stage(float4* __restrict__ buf, const int* __restrict__ zlist,
                                        const float* __restrict__ x, int64_t src_row,
                                        const float* __restrict__ dzn, int cc, int lane) {
  constexpr int NR = R1 - R0, NZG = zcount(G);
  static_assert(NR <= QRMAX && NZG <= QZR, "staging buffer");
#pragma unroll 1
  for (int i = 0; i < 4 * NR; ++i) {
    const int f = lane + 32 * i, e = f / (4 * NR), r = f - e * (4 * NR);
    const int64_t row = __shfl_sync(0xffffffffu, src_row, e);
    cp_async16(buf + e * QES + r, x + (row + KB(G) + R0 + (r >> 2)) * C + cc * QCH + 4 * (r & 3));
  }
  float4* zb = buf + 32 * QES;
  for (int f = lane; f < 4 * NZG; f += 32)
    cp_async16(zb + f, dzn + zlist[zbase(G) + (f >> 2)] * C + cc * QCH + 4 * (f & 3));
  cp_async_commit();
}

__device__ __forceinline__ float2 ffma2(float a0, float a1, float b0, float b1, float2 c) {
  return __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), c);
}

// Pass (G, R0, R1): its Q partial sums over all chunks, then its share of dgate / dY.  On entry
// step (pass, 0) is staged (or in flight) in bufs[0]; the pass stages every following step, the
// first step of the next pass (NG, NR0, NR1; NG < 0: none) included, one step ahead.
template <int G, int R0, int R1, int NG, int NR0, int NR1, int C>
__device__ __forceinline__ void q_pass(float4* __restrict__ bufs, const int* __restrict__ zlist,
                                       const float* __restrict__ x, int64_t src_row, const float* __restrict__ dzn,
                                       const float* __restrict__ cg2, const float4* __restrict__ ey4,
                                       const float4* __restrict__ eg4, float* dg, float* dy) {
  constexpr int NQP = qcount<G, R0, R1>(), NCH = C / QCH;
  static_assert(NCH % 2 == 0, "every pass starts in buffer 0");
  const int lane = threadIdx.x & 31;
  float2 Q[NQP];
#pragma unroll
  for (int i = 0; i < NQP; ++i) Q[i] = make_float2(0.f, 0.f);
#pragma unroll 1
  for (int cc = 0; cc < NCH; ++cc) {
    float4* cur = bufs + (cc & 1) * QBUF_F4;
    float4* nxt = bufs + ((cc + 1) & 1) * QBUF_F4;
    if (cc + 1 < NCH) {
      q_stage<G, R0, R1, C>(nxt, zlist, x, src_row, dzn, cc + 1, lane);
      cp_async_wait<1>();
    } else if constexpr (NG >= 0) {
      q_stage<NG, NR0, NR1, C>(nxt, zlist, x, src_row, dzn, 0, lane);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const float4* zb = cur + 32 * QES;
#pragma unroll 1
    for (int c4 = 0; c4 < QCH / 4; ++c4) {
      float4 xv[R1 - R0];
#pragma unroll
      for (int m1 = R0; m1 < R1; ++m1) xv[m1 - R0] = cur[lane * QES + 4 * (m1 - R0) + c4];
#pragma unroll
      for (int p = P_LO(G); p < P_HI(G); ++p)
#pragma unroll
        for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
          const float4 d = zb[4 * zlocal(p, kk) + c4];
#pragma unroll
          for (int m1 = R0; m1 < R1; ++m1) {
            float2 acc = Q[qloc<G, R0, R1>(p, m1, kk)];
            acc = ffma2(xv[m1 - R0].x, xv[m1 - R0].y, d.x, d.y, acc);
            acc = ffma2(xv[m1 - R0].z, xv[m1 - R0].w, d.z, d.w, acc);
            Q[qloc<G, R0, R1>(p, m1, kk)] = acc;
          }
        }
    }
    __syncwarp();  // every lane is done with `cur` before it is staged again
  }
  float Y[12], g[12];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float4 u = ey4[i], v = eg4[i];
    Y[4 * i] = u.x; Y[4 * i + 1] = u.y; Y[4 * i + 2] = u.z; Y[4 * i + 3] = u.w;
    g[4 * i] = v.x; g[4 * i + 1] = v.y; g[4 * i + 2] = v.z; g[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int p = P_LO(G); p < P_HI(G); ++p)
#pragma unroll
    for (int m1 = R0; m1 < R1; ++m1)
#pragma unroll
      for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
        const int q = qidx(p, m1, kk);
        const float2 qq = Q[qloc<G, R0, R1>(p, m1, kk)];
        const float Qv = qq.x + qq.y;
        float y0 = 0.f;
#pragma unroll
        for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2) y0 = fmaf(cg2[5 * q + m2], Y[KB(L2(p)) + m2], y0);
        dg[p] = fmaf(Qv, y0, dg[p]);
        const float qg = Qv * g[p];
#pragma unroll
        for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2)
          dy[KB(L2(p)) + m2] = fmaf(qg, cg2[5 * q + m2], dy[KB(L2(p)) + m2]);
      }
}

template <int CPL>
__global__ void __launch_bounds__(CONV_WARPS * 32, 3) conv2_q_kernel(ConvArgs a, const float* __restrict__ x,
                                                                     const float* __restrict__ dZ,
                                                                     float* __restrict__ dgates,
                                                                     float* __restrict__ dY) {
  extern __shared__ float4 qsmem[];
  float* cg2 = reinterpret_cast<float*>(qsmem);
  int* zlist = reinterpret_cast<int*>(qsmem + (NQ * 5 + 3) / 4);  // group G's rows at zbase(G) + zlocal
  load_cg2(cg2, a.tables);
  if (threadIdx.x < NP) {
    const int p = threadIdx.x;
    for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) zlist[zbase(L1(p)) + zlocal(p, kk)] = zrow(p, kk);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t n = first_node(a, warp, lane); n < a.N; n = next_node(a, lane)) {
    constexpr int C = 32 * CPL;
    float4* bufs = qsmem + QTAB_F4 + warp * 2 * QBUF_F4;
    const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
    if (n >= a.n_active) {  // receiver not evaluated in this layer: its edges' gate gradients are 0
      for (int e = e0 + lane; e < e1; e += 32) {
        float4* dgo = reinterpret_cast<float4*>(dgates + 12 * (int64_t)e);
        dgo[0] = dgo[1] = dgo[2] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      continue;
    }
    const float* dzn = dZ + n * NZ * C;
    for (int base = e0; base < e1; base += 32) {
      const int e = base + lane;
      const bool active = e < e1;
      const int64_t ee = active ? e : e0;
      const int64_t src_row = (int64_t)a.src[ee] * NK;
      const float4* ey4 = reinterpret_cast<const float4*>(a.edge_y + 12 * ee);
      const float4* eg4 = reinterpret_cast<const float4*>(a.gates + 12 * ee);
      float dg[NP], dy[NK];
#pragma unroll
      for (int k = 0; k < NK; ++k) dy[k] = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p) dg[p] = 0.f;
      q_stage<0, 0, 1, C>(bufs, zlist, x, src_row, dzn, 0, lane);
      q_pass<0, 0, 1, 1, 0, 3, C>(bufs, zlist, x, src_row, dzn, cg2, ey4, eg4, dg, dy);
      q_pass<1, 0, 3, 2, 0, 3, C>(bufs, zlist, x, src_row, dzn, cg2, ey4, eg4, dg, dy);
      q_pass<2, 0, 3, 2, 3, 5, C>(bufs, zlist, x, src_row, dzn, cg2, ey4, eg4, dg, dy);
      q_pass<2, 3, 5, -1, 0, 0, C>(bufs, zlist, x, src_row, dzn, cg2, ey4, eg4, dg, dy);
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
// Kernels with dynamic shared memory above the 48 KB default.  With a work counter (zeroed here)
// the grid is as many CTAs as fit on the device at once; without, one warp per node.
template <typename K>
unsigned conv_blocks(K kernel, uint32_t smem, const ConvArgs& a) {
  if (!a.work) return (unsigned)ceil_div(a.N, CONV_WARPS);
  int dev = 0, sms = 148, occ = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, CONV_WARPS * 32, smem) != cudaSuccess || occ < 1)
    occ = 1;
  return (unsigned)std::min<int64_t>(ceil_div(a.N, CONV_WARPS), (int64_t)occ * sms);
}

#define FSC_CONV_LAUNCH_SMEM(KERNEL, SMEM, ...)                                                    \
  do {                                                                                           \
    if (a.N == 0) return FSC_OK;                                                                 \
    if (a.work && cudaMemsetAsync(a.work, 0, sizeof(int), st) != cudaSuccess)                     \
      return fail(FSC_ERR_CUDA, #KERNEL ": memset work counter");                                \
    if (a.C == 32) {                                                                             \
      cudaFuncSetAttribute(KERNEL<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(SMEM));  \
      KERNEL<1><<<conv_blocks(KERNEL<1>, SMEM, a), CONV_WARPS * 32, SMEM, st>>>(__VA_ARGS__);     \
    } else if (a.C == 64) {                                                                      \
      cudaFuncSetAttribute(KERNEL<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(SMEM));  \
      KERNEL<2><<<conv_blocks(KERNEL<2>, SMEM, a), CONV_WARPS * 32, SMEM, st>>>(__VA_ARGS__);     \
    } else {                                                                                     \
      return fail(FSC_ERR_UNSUPPORTED, "ictd conv kernels support channels 32 or 64");           \
    }                                                                                            \
    return check_launch(#KERNEL);                                                                \
  } while (0)

int launch_conv2_z(const ConvArgs& a, const float* x, float* Z, cudaStream_t st) {
  FSC_CONV_LAUNCH_SMEM(conv2_z_kernel, ZR_SMEM, a, x, Z);
}
int launch_conv2_r(const ConvArgs& a, const float* G, float* R, cudaStream_t st) {
  FSC_CONV_LAUNCH_SMEM(conv2_r_kernel, ZR_SMEM, a, G, R);
}
int launch_conv2_q(const ConvArgs& a, const float* x, const float* dZ, float* dgates, float* dY,
                   cudaStream_t st) {
  FSC_CONV_LAUNCH_SMEM(conv2_q_kernel, QSMEM, a, x, dZ, dgates, dY);
}

}  // namespace fsc
