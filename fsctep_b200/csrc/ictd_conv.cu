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
  uint8_t qpad[NQ];  // position of q in the padded per-edge layout (QPOFF blocks)
};

// Per-edge coupled harmonics are stored with every path's block padded to a multiple of 4
// entries (offsets QPOFF), so a path's weights are read as 16-byte shared-memory vectors.
__host__ __device__ constexpr int QPOFF(int p) {
  constexpr int t[NP] = {0, 4, 8, 16, 28, 32, 48, 60, 88, 104, 112};
  return t[p];
}
constexpr int NQP = 140;

constexpr QTab make_qtab() {
  QTab t{};
  for (int p = 0; p < NP; ++p)
    for (int m1 = 0; m1 < 2 * L1(p) + 1; ++m1)
      for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
        const int q = qidx(p, m1, kk);
        t.path[q] = (int8_t)p;
        t.yb[q] = (int8_t)KB(L2(p));
        t.qpad[q] = (uint8_t)(QPOFF(p) + m1 * (2 * L3(p) + 1) + kk);
      }
  return t;
}

__constant__ QTab c_qtab = make_qtab();

constexpr int CONV_WARPS = 4;

struct __align__(16) EdgeBuf {
  float yt[NQP];
  float yg[24];  // Y (12) then gates (12) of the edge
};

// The Yt entries a lane builds are q = lane + 32 j (j < 4).  Their Y offset and path (byte j of
// `info` = yb | path << 4) and padded position (byte j of `pad`) live in two registers, read once
// per warp: per-lane indices into __constant__ memory serialise, which made the indexed-constant
// path the limiter of the edge loops.
struct LaneQ {
  uint32_t info, pad;
};
__device__ __forceinline__ LaneQ lane_q(int lane) {
  LaneQ r{0u, 0u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = lane + 32 * j;
    if (q < NQ) {
      const int p = c_qtab.path[q];
      r.info |= (uint32_t)(c_qtab.yb[q] | (p << 4)) << (8 * j);
      r.pad |= (uint32_t)(c_qtab.qpad[q]) << (8 * j);
    }
  }
  return r;
}

// This lane's share of edge e's Y and gates (lanes 0-11: Y, 12-23: gates).
__device__ __forceinline__ float load_yg(const ConvArgs& a, int64_t e, int lane) {
  return lane < 12 ? a.edge_y[12 * e + lane] : (lane < 24 ? a.gates[12 * e + lane - 12] : 0.f);
}

// Warp-cooperative: Yt[q] = gate[p(q)] * sum_m cg2[q][m] Y[yb(q) + m] into b.yt (padded layout).
__device__ __forceinline__ void build_yt(EdgeBuf& b, const float* __restrict__ cg2, float yg, int lane, LaneQ lq) {
  if (lane < 24) b.yg[lane] = yg;
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = lane + 32 * j;
    if (q < NQ) {
      const uint32_t t = lq.info >> (8 * j);
      const int yb = (int)(t & 15u);
      float v = 0.f;
#pragma unroll
      for (int m = 0; m < 5; ++m) v = fmaf(cg2[5 * q + m], b.yg[yb + m], v);
      b.yt[(lq.pad >> (8 * j)) & 255u] = v * b.yg[12 + ((t >> 4) & 15u)];
    }
  }
  __syncwarp();
}

// Path p's (2 l1 + 1) x (2 l3 + 1) weights (m1-major) from the padded Yt into registers.
template <int P>
__device__ __forceinline__ void path_weights(const EdgeBuf& b, float* w) {
  constexpr int n = (2 * L1(P) + 1) * (2 * L3(P) + 1);
  const float4* v4 = reinterpret_cast<const float4*>(b.yt + QPOFF(P));
#pragma unroll
  for (int i = 0; i < (n + 3) / 4; ++i) {
    const float4 v = v4[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}

__device__ __forceinline__ void load_cg2(float* cg2, const float* tables) {
  for (int i = threadIdx.x; i < NQ * 5; i += blockDim.x) cg2[i] = tables[TAB_CG2 + i];
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
__device__ __forceinline__ void z_path(const EdgeBuf& b, const float (&xv)[NK][CPL], float (&z)[NZ][CPL]) {
  float w[28];
  path_weights<P>(b, w);
  constexpr int n3 = 2 * L3(P) + 1;
#pragma unroll
  for (int m1 = 0; m1 < 2 * L1(P) + 1; ++m1)
#pragma unroll
    for (int kk = 0; kk < n3; ++kk) fma_ch<CPL>(xv[KB(L1(P)) + m1], w[m1 * n3 + kk], z[zrow(P, kk)]);
}

template <int P, int CPL>
__device__ __forceinline__ void r_path(const EdgeBuf& b, const float (&gv)[NK][CPL], float (&r)[NZ][CPL]) {
  float w[28];
  path_weights<P>(b, w);
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
  __device__ __forceinline__ static void run(const EdgeBuf& b, const float (&xv)[NK][CPL], float (&z)[NZ][CPL]) {
    z_path<P, CPL>(b, xv, z);
  }
};
template <int P, int CPL>
struct RPath {
  __device__ __forceinline__ static void run(const EdgeBuf& b, const float (&gv)[NK][CPL], float (&r)[NZ][CPL]) {
    r_path<P, CPL>(b, gv, r);
  }
};

// ---------------------------------------------------------------- conv2 forward: Z
// The next edge's sender row, Y and gates are loaded while the current edge is contracted.
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
  constexpr int C = 32 * CPL;
  EdgeBuf& b = bufs[warp];
  const LaneQ lq = lane_q(lane);
  float z[NZ][CPL];
#pragma unroll
  for (int r = 0; r < NZ; ++r)
#pragma unroll
    for (int c = 0; c < CPL; ++c) z[r][c] = 0.f;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  // Senders of the edges [blk, blk + 32) are held one per lane and handed out by shuffle, so a
  // row gather does not wait for its index load.
  int blk = e0, my_src = e0 + lane < e1 ? a.src[e0 + lane] : 0;
  // a sender outside the previous layer's evaluated atoms is skipped and flagged
  auto fetch = [&](int e, float (&xd)[NK][CPL], float& yg) -> bool {
    if (e >= blk + 32) {  // warp-uniform
      blk += 32;
      my_src = blk + lane < e1 ? a.src[blk + lane] : 0;
    }
    const int64_t s = __shfl_sync(0xffffffffu, my_src, e - blk);
    yg = load_yg(a, e, lane);
    const bool ok = s < a.src_limit;
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) xd[k][c] = ok ? x[(s * NK + k) * C + lane + 32 * c] : 0.f;
    return ok;
  };
  float xv[NK][CPL], yg = 0.f;
  bool ok = e0 < e1 ? fetch(e0, xv, yg) : true;
  for (int e = e0; e < e1; ++e) {
    float xn[NK][CPL], ygn = 0.f;
    bool okn = true;
    if (e + 1 < e1) okn = fetch(e + 1, xn, ygn);
    if (ok) {
      build_yt(b, cg2, yg, lane, lq);
      all_paths<CPL, ZPath>(b, xv, z);
      __syncwarp();
    } else if (lane == 0) {
      atomicCAS(a.err, 0, 70);
    }
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) xv[k][c] = xn[k][c];
    yg = ygn;
    ok = okn;
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
  constexpr int C = 32 * CPL;
  EdgeBuf& b = bufs[warp];
  const LaneQ lq = lane_q(lane);
  float r[NZ][CPL];
#pragma unroll
  for (int i = 0; i < NZ; ++i)
#pragma unroll
    for (int c = 0; c < CPL; ++c) r[i][c] = 0.f;
  const int t0 = a.tr_ptr[s], t1 = a.tr_ptr[s + 1];
  // Edge ids and receivers of [blk, blk + 32) are held one per lane and handed out by shuffle
  // (receivers precomputed: no dependent index chain through dst[e]).
  int blk = t0, my_eid = 0, my_dst = 0;
  if (t0 + lane < t1) {
    my_eid = a.tr_eid[t0 + lane];
    my_dst = a.tr_dst[t0 + lane];
  }
  // a receiver not evaluated in this layer carries no gradient
  auto fetch = [&](int t, float (&gd)[NK][CPL], float& yg) -> bool {
    if (t >= blk + 32) {  // warp-uniform
      blk += 32;
      my_eid = blk + lane < t1 ? a.tr_eid[blk + lane] : 0;
      my_dst = blk + lane < t1 ? a.tr_dst[blk + lane] : 0;
    }
    const int64_t e = __shfl_sync(0xffffffffu, my_eid, t - blk);
    const int64_t d = __shfl_sync(0xffffffffu, my_dst, t - blk);
    yg = load_yg(a, e, lane);
    const bool on = d < a.dst_limit;
    const float inv = on ? a.invdeg[d] : 0.f;
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) gd[k][c] = on ? G[(d * NK + k) * C + lane + 32 * c] * inv : 0.f;
    return on;
  };
  float gv[NK][CPL], yg = 0.f;
  bool on = t0 < t1 ? fetch(t0, gv, yg) : false;
  for (int t = t0; t < t1; ++t) {
    float gn[NK][CPL], ygn = 0.f;
    bool onn = false;
    if (t + 1 < t1) onn = fetch(t + 1, gn, ygn);
    if (on) {
      build_yt(b, cg2, yg, lane, lq);
      all_paths<CPL, RPath>(b, gv, r);
      __syncwarp();
    }
#pragma unroll
    for (int k = 0; k < NK; ++k)
#pragma unroll
      for (int c = 0; c < CPL; ++c) gv[k][c] = gn[k][c];
    yg = ygn;
    on = onn;
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
// Every reduction runs inside one thread: no cross-lane traffic.  The sender rows of the warp's 32
// edges are staged in shared memory one (l1 group, 16-channel chunk) at a time by coalesced
// 16-byte asynchronous copies (four lanes per 64-byte row chunk), and each lane then reads its own
// edge's rows from there; dZ rows are 16-byte vectors that all lanes share (same node).
constexpr int QCH = 16;                       // channels per staged chunk
constexpr int QES = 4 * 5 + 1;                // float4 slots per edge in a chunk (odd: no bank conflicts)
constexpr int QZR = 14;                       // dZ rows of the largest l1 group
constexpr int QBUF_F4 = 32 * QES + 4 * QZR;   // per warp: sender rows, then dZ rows
constexpr int QTAB_F4 = (NQ * 5 + 3) / 4 + 9; // cg2, then the dZ row list of every group (35 ints)
constexpr uint32_t QSMEM = 16u * (QTAB_F4 + CONV_WARPS * QBUF_F4);

// Local index of (p, kk) among the dZ rows of p's l1 group: rows are listed path by path.
__host__ __device__ constexpr int zlocal(int p, int kk) {
  int j = 0;
  for (int pp = P_LO(L1(p)); pp < p; ++pp) j += 2 * L3(pp) + 1;
  return j + kk;
}
__host__ __device__ constexpr int zcount(int G) { return zlocal(P_HI(G) - 1, 2 * L3(P_HI(G) - 1)) + 1; }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int G, int C>
__device__ __forceinline__ void q_group(float4* __restrict__ buf, const int* __restrict__ zlist,
                                        const float* __restrict__ x, int64_t src_row, const float* __restrict__ dzn,
                                        const float* __restrict__ cg2, const float4* __restrict__ ey4,
                                        const float4* __restrict__ eg4, float* dg, float* dy) {
  constexpr int Q0 = QOFF(P_LO(G)), NQG = Q_END(G) - Q0, M1 = 2 * G + 1, NZG = zcount(G);
  static_assert(NZG <= QZR, "dZ row buffer");
  const int lane = threadIdx.x & 31;
  float4* zb = buf + 32 * QES;
  float Q[NQG];
#pragma unroll
  for (int i = 0; i < NQG; ++i) Q[i] = 0.f;
#pragma unroll 1
  for (int cc = 0; cc < C / QCH; ++cc) {
    __syncwarp();  // every lane is done reading the previous chunk
    // 32 edges x M1 rows x 4 float4: lane copies slots f = lane + 32 i, f = (e, m1, c4)
#pragma unroll 1
    for (int i = 0; i < 4 * M1; ++i) {
      const int f = lane + 32 * i, e = f / (4 * M1), r = f - e * (4 * M1);
      const int64_t row = __shfl_sync(0xffffffffu, src_row, e);
      cp_async16(buf + e * QES + r, x + (row + KB(G) + (r >> 2)) * C + cc * QCH + 4 * (r & 3));
    }
    for (int f = lane; f < 4 * NZG; f += 32)
      cp_async16(zb + f, dzn + zlist[f >> 2] * C + cc * QCH + 4 * (f & 3));
    cp_async_wait_all();
    __syncwarp();
#pragma unroll 1
    for (int c4 = 0; c4 < QCH / 4; ++c4) {
      float4 xv[M1];
#pragma unroll
      for (int m1 = 0; m1 < M1; ++m1) xv[m1] = buf[lane * QES + 4 * m1 + c4];
#pragma unroll
      for (int p = P_LO(G); p < P_HI(G); ++p)
#pragma unroll
        for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
          const float4 d = zb[4 * zlocal(p, kk) + c4];
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
__global__ void __launch_bounds__(CONV_WARPS * 32, 3) conv2_q_kernel(ConvArgs a, const float* __restrict__ x,
                                                                     const float* __restrict__ dZ,
                                                                     float* __restrict__ dgates,
                                                                     float* __restrict__ dY) {
  extern __shared__ float4 qsmem[];
  float* cg2 = reinterpret_cast<float*>(qsmem);
  int* zlist = reinterpret_cast<int*>(qsmem + (NQ * 5 + 3) / 4);  // group G's rows at zlocal order
  load_cg2(cg2, a.tables);
  if (threadIdx.x < NP) {
    const int p = threadIdx.x, base = p < P_HI(0) ? 0 : (p < P_HI(1) ? zcount(0) : zcount(0) + zcount(1));
    for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) zlist[base + zlocal(p, kk)] = zrow(p, kk);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * CONV_WARPS + warp;
  if (n >= a.N) return;
  constexpr int C = 32 * CPL;
  float4* buf = qsmem + QTAB_F4 + warp * QBUF_F4;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  if (n >= a.n_active) {  // receiver not evaluated in this layer: its edges' gate gradients are 0
    for (int e = e0 + lane; e < e1; e += 32) {
      float4* dgo = reinterpret_cast<float4*>(dgates + 12 * (int64_t)e);
      dgo[0] = dgo[1] = dgo[2] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
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
    q_group<0, C>(buf, zlist, x, src_row, dzn, cg2, ey4, eg4, dg, dy);
    q_group<1, C>(buf, zlist + zcount(0), x, src_row, dzn, cg2, ey4, eg4, dg, dy);
    q_group<2, C>(buf, zlist + zcount(0) + zcount(1), x, src_row, dzn, cg2, ey4, eg4, dg, dy);
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
  if (a.N == 0) return FSC_OK;
  const unsigned blocks = (unsigned)ceil_div(a.N, CONV_WARPS);
  if (a.C == 32) {
    cudaFuncSetAttribute(conv2_q_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QSMEM);
    conv2_q_kernel<1><<<blocks, CONV_WARPS * 32, QSMEM, st>>>(a, x, dZ, dgates, dY);
  } else if (a.C == 64) {
    cudaFuncSetAttribute(conv2_q_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QSMEM);
    conv2_q_kernel<2><<<blocks, CONV_WARPS * 32, QSMEM, st>>>(a, x, dZ, dgates, dY);
  } else {
    return fail(FSC_ERR_UNSUPPORTED, "ictd conv kernels support channels 32 or 64");
  }
  return check_launch("conv2_q_kernel");
}

}  // namespace fsc
