// pure-cartesian-sparse energy + forces (models/pure_cartesian_sparse_layers.py:459-855,
// PureCartesianTensorProductO3Sparse with max_rank_other = 1, k_policy = "k0", no epsilon,
// pseudotensors identically zero: models/pure_cartesian.py:736-929).
//
// Node features are true Cartesian tensors f[n][comp][c], comp = roff(L) + row-major index of the
// rank-L tensor (R = sum_L 3^L components).  Every tensor-product path p = (L1, L2, Lout = L1+L2)
// is an outer product: message_p[e][(i, j)][a] = x1[src][roff(L1)+i][a] * n_e^{(x)L2}[j].
//
// The reference forms per-edge channel-mixing weights W_e = fc.4(h2_e), P*C*C1*C2 floats per edge
// (14.7 GB per layer at config 2), and contracts them with the messages.  Here fc.4 is applied
// after aggregation instead:
//   conv2:  out[n][Lout comp][c] = (1/avg) sum_{p(Lout), j, a} W[(p, c, a), j] Z_p[n][comp][j][a],
//           Z_p[n][comp][j][a] = sum_{e -> n} h2'_e[j] message_p[e][comp][a],  h2' = [h2, 1]
//   (one per-node aggregation kernel + one GEMM per Lout); conv1 folds fc.4 and the atom
//   features of both ends into per-species-pair tables.  The reverse pass mirrors it: a GEMM
//   gives dZ, two kernels per receiving node yield dE/dh2', dE/dn^{(x)L} and the feature gradient
//   of the sources, and the radial MLP backward (radial_tc.cu) turns dE/dh2 into dE/d|r|.
#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {
namespace sp {

constexpr int J = 65;          // radial hidden width + the bias row
constexpr int RH = 64;
constexpr int MAXR = 40;       // components up to rank 3
constexpr int MAXROWS = 144;   // sum over paths of 3^Lout (142 at lmax 3)
constexpr int64_t kMaxGraphs = 4096;
// Aggregation buffer budget, 16 GB: the per-rank fc.4 GEMMs over one node chunk have
// chunk x 3^Lout rows, and the low ranks need large chunks to fill the GPU.
constexpr int64_t kZBudgetFloats = (int64_t)1 << 32;
constexpr int64_t kDmBudgetFloats = (int64_t)1 << 31;  // 8 GB of dm rows per conv2-backward sub-chunk
constexpr int64_t kGramChunk = 16384;

__host__ __device__ constexpr int pow3(int L) { return L == 0 ? 1 : 3 * pow3(L - 1); }
__host__ __device__ constexpr int roff(int L) { return (pow3(L) - 1) / 2; }

// conv2 aggregation rows (built on the host).  Row order: Lout, then the component of the
// rank-Lout output, then the rank q of the path among those with that Lout.
struct Rows {
  int nrows, npaths, R, lmax;
  unsigned char c1[MAXROWS];  // x1 component of the row
  unsigned char c2[MAXROWS];  // n^{(x)L2} component of the row
  unsigned char rlist[MAXROWS];
  short c1off[MAXR + 1];      // rows with x1 component c1: rlist[c1off[c1] .. c1off[c1+1])
  int zoff[4], npl[4];        // first row and number of paths of each Lout
  int p1[4];                  // conv1: path index of (L, 0, L)
};

Rows make_rows(int lmax) {
  Rows r{};
  r.lmax = lmax;
  r.R = roff(lmax + 1);
  std::vector<int> L1s, L2s, Ls;
  for (int L1 = 0; L1 <= lmax; ++L1)
    for (int L2 = 0; L2 <= lmax; ++L2)
      if (std::min(L1, L2) <= 1 && L1 + L2 <= lmax) {
        if (L2 == 0) r.p1[L1] = (int)L1s.size();
        L1s.push_back(L1);
        L2s.push_back(L2);
        Ls.push_back(L1 + L2);
      }
  r.npaths = (int)L1s.size();
  int row = 0;
  std::vector<int> c1v, c2v;
  for (int Lo = 0; Lo <= lmax; ++Lo) {
    std::vector<int> ps;
    for (int p = 0; p < r.npaths; ++p)
      if (Ls[p] == Lo) ps.push_back(p);
    r.zoff[Lo] = row;
    r.npl[Lo] = (int)ps.size();
    for (int k = 0; k < pow3(Lo); ++k)
      for (int p : ps) {
        const int L2 = L2s[p], L1 = L1s[p];
        const int i = k / pow3(L2), j = k % pow3(L2);
        c1v.push_back(roff(L1) + i);
        c2v.push_back(roff(L2) + j);
        ++row;
      }
  }
  r.nrows = row;
  for (int q = 0; q < row; ++q) {
    r.c1[q] = (unsigned char)c1v[q];
    r.c2[q] = (unsigned char)c2v[q];
  }
  int pos = 0;
  for (int c = 0; c < r.R; ++c) {
    r.c1off[c] = (short)pos;
    for (int q = 0; q < row; ++q)
      if (c1v[q] == c) r.rlist[pos++] = (unsigned char)q;
  }
  r.c1off[r.R] = (short)pos;
  return r;
}

// n^{(x)L} for L <= lmax, row-major, out[roff(L) + idx]
__device__ __forceinline__ void npow_all(int lmax, float x, float y, float z, float* out) {
  const float n[3] = {x, y, z};
  out[0] = 1.f;
  out[1] = x; out[2] = y; out[3] = z;
  if (lmax >= 2)
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
      for (int j = 0; j < 3; ++j) out[4 + 3 * i + j] = n[i] * n[j];
  if (lmax >= 3)
#pragma unroll
    for (int i = 0; i < 9; ++i)
#pragma unroll
      for (int k = 0; k < 3; ++k) out[13 + 3 * i + k] = out[4 + i] * n[k];
}

// dE/dn from dE/d(n^{(x)L})
__device__ __forceinline__ void npow_grad(int lmax, const float* n, const float* d, float* dn) {
  dn[0] = d[1]; dn[1] = d[2]; dn[2] = d[3];
  if (lmax >= 2)
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) {
        const float g = d[4 + 3 * i + j];
        dn[i] += g * n[j];
        dn[j] += g * n[i];
      }
  if (lmax >= 3)
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j)
        for (int k = 0; k < 3; ++k) {
          const float g = d[13 + 9 * i + 3 * j + k];
          dn[i] += g * n[j] * n[k];
          dn[j] += g * n[i] * n[k];
          dn[k] += g * n[i] * n[j];
        }
}

// Sum over the 32 lanes of t[i] for every i; lane i returns the sum of t[i].
__device__ __forceinline__ float transpose_reduce32(float (&t)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? t[i] : t[i + w];
      const float keep = up ? t[i + w] : t[i];
      t[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return t[0];
}

struct GradList {
  float* p[8];
};

struct Args {
  int64_t N, E;
  int C, R, lmax, S_species;
  const int32_t* row_ptr;
  const int32_t* src;
  const int32_t* dst;
  const int32_t* species;
  const float* edge_y;  // [E][12]: n (0..2), |r| (3), r (9..11)
};

// ---------------------------------------------------------------- geometry
__global__ void geom_kernel(int64_t E, const float* __restrict__ pos, const int32_t* __restrict__ src,
                            const int32_t* __restrict__ dst, const int32_t* __restrict__ batch,
                            const float* __restrict__ cell, const float* __restrict__ shift, float* __restrict__ ey) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const int i = src[e], j = dst[e];
  const float* c = cell + 9 * (int64_t)batch[i];
  const float s0 = shift[3 * e], s1 = shift[3 * e + 1], s2 = shift[3 * e + 2];
  float r[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) r[k] = pos[3 * (int64_t)j + k] - pos[3 * (int64_t)i + k] + (s0 * c[k] + s1 * c[3 + k] + s2 * c[6 + k]);
  const float len = sqrtf(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
  const float inv = 1.f / fmaxf(len, 1e-8f);
  float* o = ey + 12 * e;
  o[0] = r[0] * inv; o[1] = r[1] * inv; o[2] = r[2] * inv; o[3] = len;
  o[4] = o[5] = o[6] = o[7] = o[8] = 0.f;
  o[9] = r[0]; o[10] = r[1]; o[11] = r[2];
}

// ---------------------------------------------------------------- conv1
// Warp per receiving node, lanes over channels: f1[n][comp][c] = (1/deg) sum_e g_L(e)[c] n^{(x)L}[comp],
// g_L[c] = sum_j h2'_e[j] K[s_src][s_n][L][j][c].
template <int CPL>
__global__ void __launch_bounds__(256) conv1_fwd_kernel(Args a, const float* __restrict__ K, const float* __restrict__ h2,
                                                        float* __restrict__ f1) {
  __shared__ float hs[8][J + 3];
  __shared__ float np[8][MAXR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * 8 + warp;
  if (n >= a.N) return;
  const int C = 32 * CPL, R = a.R;
  float acc[MAXR][CPL];
#pragma unroll
  for (int q = 0; q < MAXR; ++q)
#pragma unroll
    for (int i = 0; i < CPL; ++i) acc[q][i] = 0.f;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  const int sn = a.species[n];
  for (int e = e0; e < e1; ++e) {
    const int s = a.src[e];
    const float* kt = K + ((int64_t)a.species[s] * a.S_species + sn) * (a.lmax + 1) * J * C;
    hs[warp][lane] = h2[(int64_t)e * RH + lane];
    hs[warp][lane + 32] = h2[(int64_t)e * RH + lane + 32];
    if (lane == 0) {
      hs[warp][64] = 1.f;
      const float* y = a.edge_y + 12 * (int64_t)e;
      npow_all(a.lmax, y[0], y[1], y[2], np[warp]);
    }
    __syncwarp();
    for (int L = 0; L <= a.lmax; ++L) {
      float g[CPL];
#pragma unroll
      for (int i = 0; i < CPL; ++i) g[i] = 0.f;
      const float* kl = kt + (int64_t)L * J * C;
      for (int j = 0; j < J; ++j) {
        const float h = hs[warp][j];
#pragma unroll
        for (int i = 0; i < CPL; ++i) g[i] = fmaf(h, kl[j * C + lane + 32 * i], g[i]);
      }
      for (int q = roff(L); q < roff(L + 1); ++q) {
        const float v = np[warp][q];
#pragma unroll
        for (int i = 0; i < CPL; ++i) acc[q][i] = fmaf(g[i], v, acc[q][i]);
      }
    }
    __syncwarp();
  }
  const int deg = e1 - e0;
  const float inv = 1.f / (float)(deg > 1 ? deg : 1);
  for (int q = 0; q < R; ++q)
#pragma unroll
    for (int i = 0; i < CPL; ++i) f1[(n * R + q) * C + lane + 32 * i] = acc[q][i] * inv;
}

// conv1 backward: per edge dE/dh2 (layer 0) and dE/dn^{(x)L} (accumulated), from G1 = dE/df1.
// Warp per receiving node, lanes over channels.  Per edge and rank L, with d_L[c] = sum_{q in L}
// G1[n][q][c] n^{(x)L}[q] / deg:
//   g_L[c] = sum_j h2'_e[j] K[L][j][c],   dE/dh2_e[j] = sum_{L, c} d_L[c] K[L][j][c],
//   dE/dn^{(x)L}[q] += sum_c G1[n][q][c] g_L[c] / deg,
// one coalesced pass over K gives both g and the lane's partial dE/dh2; the per-lane partials
// are summed over the warp by transpose reductions (lane l ends with j = l and j = 32 + l).
template <int CPL>
__global__ void __launch_bounds__(256) conv1_bwd_kernel(Args a, const float* __restrict__ K, const float* __restrict__ h2,
                                                        const float* __restrict__ G1, float* __restrict__ dh2,
                                                        float* __restrict__ dnp) {
  __shared__ float hs[8][J + 3];
  __shared__ float np[8][MAXR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * 8 + warp;
  if (n >= a.N) return;
  const int C = 32 * CPL, R = a.R;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  const int deg = e1 - e0;
  const float inv = 1.f / (float)(deg > 1 ? deg : 1);
  const int sn = a.species[n];
  const float* g1n = G1 + n * R * C + lane;
  for (int e = e0; e < e1; ++e) {
    const int s = a.src[e];
    const float* kt = K + ((int64_t)a.species[s] * a.S_species + sn) * (a.lmax + 1) * J * C + lane;
    hs[warp][lane] = h2[(int64_t)e * RH + lane];
    hs[warp][lane + 32] = h2[(int64_t)e * RH + lane + 32];
    if (lane == 0) {
      hs[warp][64] = 1.f;
      const float* y = a.edge_y + 12 * (int64_t)e;
      npow_all(a.lmax, y[0], y[1], y[2], np[warp]);
    }
    __syncwarp();
    float ph[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) ph[j] = 0.f;
    float dn[64];  // this lane's partial dE/dn^{(x)L}[q], q < R (entries q >= R stay 0)
#pragma unroll
    for (int q = 0; q < 64; ++q) dn[q] = 0.f;
#pragma unroll
    for (int L = 0; L < 4; ++L) {
      if (L > a.lmax) break;
      float d[CPL], g[CPL];
#pragma unroll
      for (int i = 0; i < CPL; ++i) d[i] = g[i] = 0.f;
      for (int q = roff(L); q < roff(L + 1); ++q) {
        const float v = np[warp][q] * inv;
#pragma unroll
        for (int i = 0; i < CPL; ++i) d[i] = fmaf(g1n[q * C + 32 * i], v, d[i]);
      }
      const float* kl = kt + (int64_t)L * J * C;
#pragma unroll
      for (int j = 0; j < RH; ++j) {
        const float h = hs[warp][j];
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const float k = kl[j * C + 32 * i];
          g[i] = fmaf(h, k, g[i]);
          t = fmaf(d[i], k, t);
        }
        ph[j] += t;
      }
#pragma unroll
      for (int i = 0; i < CPL; ++i) g[i] += kl[RH * C + 32 * i];  // the bias row, h2'[64] = 1
#pragma unroll
      for (int q = 0; q < 40; ++q) {
        if (q >= roff(L) && q < roff(L + 1)) {
          float t = 0.f;
#pragma unroll
          for (int i = 0; i < CPL; ++i) t = fmaf(g1n[q * C + 32 * i], g[i], t);
          dn[q] = t * inv;
        }
      }
    }
    float lo[32], hi[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      lo[j] = ph[j];
      hi[j] = ph[32 + j];
    }
    const float dlo = transpose_reduce32(lo, lane);
    const float dhi = transpose_reduce32(hi, lane);
    dh2[(int64_t)e * RH + lane] = dlo;
    dh2[(int64_t)e * RH + 32 + lane] = dhi;
    float q0[32], q1[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      q0[q] = dn[q];
      q1[q] = dn[32 + q];
    }
    const float s0 = transpose_reduce32(q0, lane);
    const float s1 = transpose_reduce32(q1, lane);
    if (lane < R) dnp[(int64_t)e * MAXR + lane] += s0;
    if (32 + lane < R) dnp[(int64_t)e * MAXR + 32 + lane] += s1;
    __syncwarp();
  }
}

// ---------------------------------------------------------------- conv2 forward aggregation
// Block per receiving node; thread item (row r, channel a) with 65 accumulators over j:
// Z[n][r][j][a] = sum_e h2'_e[j] x1[src_e][c1(r)][a] n_e^{(x)L2}[c2(r)].
constexpr int ZEB = 32;  // edges staged per batch

__global__ void __launch_bounds__(256) z_kernel(Args a, Rows rows, const float* __restrict__ x,
                                                const float* __restrict__ h2, int64_t n0, float* __restrict__ Z) {
  __shared__ __align__(16) float hs[ZEB][RH];
  __shared__ float np[ZEB][MAXR];
  __shared__ int srcs[ZEB];
  const int64_t n = n0 + blockIdx.x;
  const int C = a.C, R = a.R;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  const int items = rows.nrows * C;
  float* zn = Z + (int64_t)blockIdx.x * rows.nrows * J * C;
  for (int base = 0; base < items; base += blockDim.x) {
    const int item = base + threadIdx.x;
    const bool valid = item < items;
    const int r = valid ? item / C : 0, ch = valid ? item - r * C : 0;
    const int c1 = rows.c1[r], c2 = rows.c2[r];
    float acc[RH];
#pragma unroll
    for (int j = 0; j < RH; ++j) acc[j] = 0.f;
    float accb = 0.f;
    for (int eb = e0; eb < e1; eb += ZEB) {
      const int ne = min(ZEB, e1 - eb);
      __syncthreads();
      for (int t = threadIdx.x; t < ne * RH; t += blockDim.x) hs[t / RH][t % RH] = h2[(int64_t)(eb + t / RH) * RH + t % RH];
      if (threadIdx.x < ne) {
        const int e = eb + threadIdx.x;
        srcs[threadIdx.x] = a.src[e];
        const float* y = a.edge_y + 12 * (int64_t)e;
        npow_all(a.lmax, y[0], y[1], y[2], np[threadIdx.x]);
      }
      __syncthreads();
      if (valid) {
        for (int k = 0; k < ne; ++k) {
          const float m = x[((int64_t)srcs[k] * R + c1) * C + ch] * np[k][c2];
          const float4* h4 = reinterpret_cast<const float4*>(hs[k]);
#pragma unroll
          for (int j4 = 0; j4 < RH / 4; ++j4) {
            const float4 h = h4[j4];
            acc[4 * j4] = fmaf(h.x, m, acc[4 * j4]);
            acc[4 * j4 + 1] = fmaf(h.y, m, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = fmaf(h.z, m, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = fmaf(h.w, m, acc[4 * j4 + 3]);
          }
          accb += m;
        }
      }
    }
    if (valid) {
      float* zr = zn + (int64_t)r * J * C + ch;
#pragma unroll
      for (int j = 0; j < RH; ++j) zr[(int64_t)j * C] = acc[j];
      zr[(int64_t)RH * C] = accb;
    }
  }
}

// ---------------------------------------------------------------- conv2 forward aggregation, tensor cores
// The same Z as z_kernel, as one small GEMM per receiving node n with K = its edges:
//   D[(r, a)][j] = sum_e A[(r, a)][e] B[j][e],   A[(r, a)][e] = x1[src_e][c1(r)][a] n_e^{(x)L2}[c2(r)],
//   B[j][e] = h2'_e[j] (j < 65; rows 65..79 zero),  Z[n][r][j][a] = D[(r, a)][j].
// M = 128 consecutive (r, a) pairs per tile (TMEM lane = pair), N = 80, K = the node's edges in
// chunks of 64.  A is built by the CUDA cores straight into TMEM (tf32 hi / lo split; warps w and
// w + 4 share lanes and build K columns [0, 32) and [32, 64)), B is the node's h2' rows as a
// K-major shared-memory image (hi / lo), so every tile of the node reuses it; the product is
// 3xTF32 (hi*lo and lo*hi issued before hi*hi).  A node with more than ZTC_KMAX edges is done in
// edge groups, the later groups adding into Z.  Persistent grid of two CTAs per SM.
constexpr int ZTC_M = 128, ZTC_N = 80, ZTC_KC = 64, ZTC_KMAX = 128, ZTC_THREADS = 256;
constexpr uint32_t ZTC_IMG = 4u * ZTC_N * ZTC_KMAX;  // bytes of one B image (hi or lo)
struct ZtcSmem {
  static constexpr uint32_t BHI = 0;
  static constexpr uint32_t BLO = ZTC_IMG;
  static constexpr uint32_t NP = 2 * ZTC_IMG;                    // [ZTC_KMAX][MAXR] n^{(x)L}
  static constexpr uint32_t XOFF = NP + 4u * ZTC_KMAX * MAXR;    // [ZTC_KMAX] source row offsets in x
  static constexpr uint32_t BAR = XOFF + 8u * ZTC_KMAX;
  static constexpr uint32_t TOTAL = BAR + 16;
};
static_assert(3 * ZtcSmem::TOTAL > 228u * 1024u, "at most two CTAs per SM (256 TMEM columns each)");

// element (n, k) of a K-major no-swizzle B image with N rows
__device__ __forceinline__ int zimg(int n, int k) { return (k >> 2) * 4 * ZTC_N + 4 * n + (k & 3); }

__global__ void __launch_bounds__(ZTC_THREADS, 2) z_tc_kernel(Args a, Rows rows, const float* __restrict__ x,
                                                              const float* __restrict__ h2, int64_t n0, int64_t nc,
                                                              float* __restrict__ Z, int* err) {
  extern __shared__ __align__(1024) uint8_t smem[];
  float* bhi = reinterpret_cast<float*>(smem + ZtcSmem::BHI);
  float* blo = reinterpret_cast<float*>(smem + ZtcSmem::BLO);
  float* np = reinterpret_cast<float*>(smem + ZtcSmem::NP);
  int64_t* xoff = reinterpret_cast<int64_t*>(smem + ZtcSmem::XOFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + ZtcSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + ZtcSmem::BAR + 8);

  const int tid = threadIdx.x, warp = tid >> 5, half = tid / ZTC_M, row = tid % ZTC_M;
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t tD = tbase, tAhi = tbase + 128u, tAlo = tbase + 192u;  // D: 80 columns, A: 64 + 64
  const uint32_t s_hi = tc::smem_u32(bhi), s_lo = tc::smem_u32(blo);
  constexpr uint32_t idesc = tc::idesc_tf32(ZTC_M, ZTC_N);
  // tile = ZTC_M / C rows (slots) taken in the order of rows.rlist, where rows with the same x1
  // component are adjacent: a thread keeps its gathered x1 values while the component repeats
  const int C = a.C, R = a.R, S = ZTC_M / C, slot = row / C, ch = row - slot * C;
  const int ntiles = (rows.nrows + S - 1) / S;
  uint32_t phase = 0;
  bool ok = true;

  for (int64_t nl = blockIdx.x; nl < nc && ok; nl += gridDim.x) {
    const int64_t n = n0 + nl;
    const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
    float* zn = Z + nl * (int64_t)rows.nrows * J * C;
    for (int g0 = e0, grp = 0; (g0 < e1 || grp == 0) && ok; g0 += ZTC_KMAX, ++grp) {
      const int kg = min(ZTC_KMAX, e1 - g0);  // edges of this group (0 for an isolated node)
      const int nchunks = max(1, (kg + ZTC_KC - 1) / ZTC_KC);
      // ---- the group's edge data and B image (previous MMAs finished: d_ready below)
      __syncthreads();
      if (tid < ZTC_KMAX) {
        if (tid < kg) {
          const int e = g0 + tid;
          xoff[tid] = (int64_t)a.src[e] * R * C;
          const float* y = a.edge_y + 12 * (int64_t)e;
          npow_all(a.lmax, y[0], y[1], y[2], np + tid * MAXR);
        } else {
          xoff[tid] = 0;
        }
      }
      for (int i = tid; i < ZTC_N * nchunks * ZTC_KC; i += ZTC_THREADS) {
        const int k = i / ZTC_N, j = i - k * ZTC_N;
        float v = 0.f;
        if (k < kg && j < J) v = j < RH ? h2[(int64_t)(g0 + k) * RH + j] : 1.f;
        uint32_t hi, lo;
        tc::split_tf32(v, hi, lo);
        bhi[zimg(j, k)] = __uint_as_float(hi);
        blo[zimg(j, k)] = __uint_as_float(lo);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      int cached_c1 = -1;
      float xv[32];
      for (int tile = 0; tile < ntiles && ok; ++tile) {
        const int q = tile * S + slot;
        const bool valid = q < rows.nrows;
        const int r = valid ? rows.rlist[q] : 0;
        const int c1 = rows.c1[r], c2 = rows.c2[r];
        for (int cc = 0; cc < nchunks; ++cc) {
          // ---- A columns [32 half, 32 half + 32) of chunk cc
          const int kb = cc * ZTC_KC + 32 * half;
          if (nchunks > 1 || c1 != cached_c1) {  // warp-uniform: a warp's lanes share the row
            const float* xc = x + (int64_t)c1 * C + ch;
#pragma unroll
            for (int i = 0; i < 32; ++i) xv[i] = (valid && kb + i < kg) ? xc[xoff[kb + i]] : 0.f;
            cached_c1 = nchunks == 1 ? c1 : -1;
          }
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v = kb + i < kg ? xv[i] * np[(kb + i) * MAXR + c2] : 0.f;
            tc::split_tf32(v, hi[i], lo[i]);
          }
          tc::tmem_st32(tAhi + lane_off + 32u * half, hi);
          tc::tmem_st32(tAlo + lane_off + 32u * half, lo);
          tc::tmem_wait_st();
          tc::tc_fence_before();
          __syncthreads();
          if (tid == 0) {
            tc::tc_fence_after();
            const int ksteps = kg > 0 ? min(ZTC_KC, kg - cc * ZTC_KC + 7) / 8 : 1;
            for (int j = 0; j < ksteps; ++j) {  // a fresh chain per chunk: at most 24 MMAs
              const uint32_t off = 32u * ZTC_N * (uint32_t)(cc * (ZTC_KC / 8) + j);
              const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * ZTC_N, 128);
              const uint64_t dl = tc::smem_desc_kmajor(s_lo + off, 16u * ZTC_N, 128);
              tc::mma_tf32_ts(tD, tAhi + 8u * j, dl, idesc, j > 0 ? 1u : 0u);
              tc::mma_tf32_ts(tD, tAlo + 8u * j, dh, idesc, 1u);
            }
            for (int j = 0; j < ksteps; ++j) {
              const uint32_t off = 32u * ZTC_N * (uint32_t)(cc * (ZTC_KC / 8) + j);
              const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * ZTC_N, 128);
              tc::mma_tf32_ts(tD, tAhi + 8u * j, dh, idesc, 1u);
            }
            tc::mma_commit(bar);
          }
          // one thread polls the barrier; the others wait at the CTA barrier without issuing
          const bool w = tid != 0 || tc::mbar_wait(bar, phase, err, 81);
          phase ^= 1u;
          const bool failed = __syncthreads_or(!w);
          tc::tc_fence_after();
          if (failed) {
            ok = false;
            break;
          }
          // ---- epilogue of the chunk -> Z[n][r][j][a]: half 0 columns [0, 32) and the bias column
          // 64, half 1 [32, 64); later chunks and edge groups add in fp32
          uint32_t u[48];
          tc::tmem_ld32(tD + lane_off + 32u * half, u);
          if (half == 0) tc::tmem_ld16(tD + lane_off + 64u, u + 32);
          tc::tmem_wait_ld();
          if (valid) {
            float* zr = zn + (int64_t)r * J * C + ch + (int64_t)32 * half * C;
            if (grp == 0 && cc == 0) {
#pragma unroll
              for (int i = 0; i < 32; ++i) zr[(int64_t)i * C] = __uint_as_float(u[i]);
              if (half == 0) zr[(int64_t)RH * C] = __uint_as_float(u[32]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) zr[(int64_t)i * C] += __uint_as_float(u[i]);
              if (half == 0) zr[(int64_t)RH * C] += __uint_as_float(u[32]);
            }
          }
          tc::tc_fence_before();
        }
        if (!ok) break;
      }
    }
  }
  if (!ok && tid == 0) {  // a wait gave up: let the last committed chain finish before freeing TMEM
    const long long t0 = clock64();
    while (!tc::mbar_try_wait(bar, phase ^ 1u))
      if (clock64() - t0 > tc::kWaitCycles) break;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

int launch_z_tc(const Args& a, const Rows& rows, const float* x, const float* h2, int64_t n0, int64_t nc, float* Z,
                int* err, cudaStream_t st) {
  if (nc <= 0) return FSC_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaFuncSetAttribute(z_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ZtcSmem::TOTAL) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "z_tc_kernel: shared memory attribute");
  const unsigned blocks = (unsigned)std::min<int64_t>(nc, 2 * (int64_t)sms);
  z_tc_kernel<<<blocks, ZTC_THREADS, ZtcSmem::TOTAL, st>>>(a, rows, x, h2, n0, nc, Z, err);
  return check_launch("sparse z_tc_kernel");
}

// ---------------------------------------------------------------- conv2 backward
// Both kernels take one receiving node per block and read its dZ block once.
// dm_kernel: thread = column (row r, channel a) holding dZ[n][r][:][a] in registers; per edge
//   dm = sum_j dZ[n][r][j][a] h2'_e[j],  written to the chunk's dm rows dmbuf[e - e_base][r][a].
// The two contractions of dm (dE/dx1 of the sources and dE/dn^{(x)L2} of the edges) are
// dm_gx_kernel and dm_dn_kernel below: reductions in a fixed order, no atomics.
__global__ void __launch_bounds__(256) bwd_dm_kernel(Args a, Rows rows, const float* __restrict__ h2,
                                                     const float* __restrict__ dZ, int64_t n0,
                                                     float* __restrict__ dmbuf, int64_t e_base) {
  __shared__ __align__(16) float hs[ZEB][RH];
  const int64_t n = n0 + blockIdx.x;
  const int C = a.C;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  const int cols = rows.nrows * C;
  const float* dzn = dZ + (int64_t)blockIdx.x * rows.nrows * J * C;
  for (int base = 0; base < cols; base += blockDim.x) {
    const int col = base + threadIdx.x;
    const bool valid = col < cols;  // warp-uniform: cols and blockDim are multiples of 32
    const int r = valid ? col / C : 0, ch = valid ? col - r * C : 0;
    float dz[RH];
    float dzb = 0.f;
    if (valid) {
      const float* zc = dzn + (int64_t)r * J * C + ch;
#pragma unroll
      for (int j = 0; j < RH; ++j) dz[j] = zc[(int64_t)j * C];
      dzb = zc[(int64_t)RH * C];
    } else {
#pragma unroll
      for (int j = 0; j < RH; ++j) dz[j] = 0.f;
    }
    for (int eb = e0; eb < e1; eb += ZEB) {
      const int ne = min(ZEB, e1 - eb);
      __syncthreads();
      for (int t = threadIdx.x; t < ne * RH; t += blockDim.x) hs[t / RH][t % RH] = h2[(int64_t)(eb + t / RH) * RH + t % RH];
      __syncthreads();
      if (valid) {
        for (int k = 0; k < ne; ++k) {
          const float4* h4 = reinterpret_cast<const float4*>(hs[k]);
          float d0 = dzb, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
          for (int j4 = 0; j4 < RH / 4; ++j4) {
            const float4 h = h4[j4];
            d0 = fmaf(dz[4 * j4], h.x, d0);
            d1 = fmaf(dz[4 * j4 + 1], h.y, d1);
            d2 = fmaf(dz[4 * j4 + 2], h.z, d2);
            d3 = fmaf(dz[4 * j4 + 3], h.w, d3);
          }
          dmbuf[((int64_t)(eb + k - e_base) * rows.nrows + r) * C + ch] = (d0 + d1) + (d2 + d3);
        }
      }
    }
  }
}

// dE/dx1 of the sources, warp per source atom s: its out-edges in [e_base, e_end) taken in
// increasing edge order (the transpose CSR rows are sorted), 32 at a time with their
// n^{(x)L2} in shared memory; per x1 component c1 (lanes over channels)
//   gx[s][c1][a] += sum_e sum_{r: c1(r) = c1} dm_e[r][a] n_e^{(x)L2}[c2(r)]
// with the rows of c1 in rows.rlist order: a fixed summation order, so the result repeats bit for
// bit.  A source with no out-edge in the range returns after one binary search.
template <int CPL>
__global__ void __launch_bounds__(256) dm_gx_kernel(Args a, Rows rows, const int32_t* __restrict__ tr_ptr,
                                                    const int32_t* __restrict__ tr_eid, const float* __restrict__ dmbuf,
                                                    int64_t e_base, int64_t e_end, float* __restrict__ gx) {
  __shared__ float nps[8][32][MAXR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int C = 32 * CPL;
  const int R = a.R, NR = rows.nrows;
  for (int64_t s = (int64_t)blockIdx.x * 8 + warp; s < a.N; s += (int64_t)gridDim.x * 8) {
    const int t0 = tr_ptr[s], t1 = tr_ptr[s + 1];
    int lo = t0, hi = t1;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (tr_eid[mid] < e_base) lo = mid + 1;
      else hi = mid;
    }
    for (int t = lo; t < t1; t += 32) {
      const int me = t + lane < t1 ? tr_eid[t + lane] : (int)e_end;
      const unsigned in = __ballot_sync(0xffffffffu, me < e_end);
      const int nb = __popc(in);  // edges sorted: the ones in the range are a prefix
      if (nb == 0) break;
      if (lane < nb) {
        const float* y = a.edge_y + 12 * (int64_t)me;
        npow_all(a.lmax, y[0], y[1], y[2], nps[warp][lane]);
      }
      __syncwarp();
      for (int c1 = 0; c1 < R; ++c1) {
        float acc[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[j] = 0.f;
        for (int i = 0; i < nb; ++i) {
          const int64_t e = __shfl_sync(0xffffffffu, me, i);
          const float* dme = dmbuf + (e - e_base) * NR * C + lane;
          for (int qq = rows.c1off[c1]; qq < rows.c1off[c1 + 1]; ++qq) {
            const int r = rows.rlist[qq];
            const float w = nps[warp][i][rows.c2[r]];
#pragma unroll
            for (int j = 0; j < CPL; ++j) acc[j] = fmaf(dme[(int64_t)r * C + 32 * j], w, acc[j]);
          }
        }
        float* g = gx + (s * R + c1) * C + lane;
#pragma unroll
        for (int j = 0; j < CPL; ++j) g[32 * j] += acc[j];
      }
      __syncwarp();
      if (nb < 32) break;
    }
  }
}

// dE/dn^{(x)L2} of the edges, warp per edge e in [e_base, e_base + count): lanes over channels,
//   dnp[e][c2] += sum_{r: c2(r) = c2} sum_a dm_e[r][a] x1[src_e][c1(r)][a]
// each lane's partial sums per c2 kept in shared memory, then summed over the lanes in order.
template <int CPL>
__global__ void __launch_bounds__(256) dm_dn_kernel(Args a, Rows rows, const float* __restrict__ x,
                                                    const float* __restrict__ dmbuf, int64_t e_base, int64_t count,
                                                    float* __restrict__ dnp) {
  __shared__ float part[8][MAXR][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int C = 32 * CPL;
  const int R = a.R, NR = rows.nrows;
  for (int64_t w = (int64_t)blockIdx.x * 8 + warp; w < count; w += (int64_t)gridDim.x * 8) {
    const int64_t e = e_base + w;
    const int64_t s = a.src[e];
    for (int c = 0; c < R; ++c) part[warp][c][lane] = 0.f;
    const float* dme = dmbuf + w * NR * C + lane;
    const float* xs = x + s * R * C + lane;
    for (int r = 0; r < NR; ++r) {
      const int c1 = rows.c1[r];
      float t = 0.f;
#pragma unroll
      for (int j = 0; j < CPL; ++j) t = fmaf(dme[(int64_t)r * C + 32 * j], xs[(int64_t)c1 * C + 32 * j], t);
      part[warp][rows.c2[r]][lane] += t;
    }
    __syncwarp();
    for (int c = lane; c < R; c += 32) {  // R = 40 components at lmax 3
      float v = 0.f;
      for (int l = 0; l < 32; ++l) v += part[warp][c][l];
      dnp[e * MAXR + c] += v;
    }
    __syncwarp();
  }
}

// dm on tensor cores, per receiving node n and 128 consecutive (r, a) pairs (rows.rlist order):
//   D[(r, a)][e] = sum_{j < 64} dZ[n][r][j][a] h2_e[j]      (M = 128, N = 64 edges, K = 64, 3xTF32)
//   dm = D + dZ[n][r][64][a]                                (the bias row of h2' = [h2, 1])
// A (the dZ rows) is written to TMEM by the CUDA cores, B is the node's h2 rows as a K-major image
// in shared memory (up to two 64-edge chunks).  The epilogue writes dm to the sub-chunk's dm rows
// (as bwd_dm_kernel); dm_gx_kernel and dm_dn_kernel reduce them.
constexpr int DTC_NE = 64;
struct DtcSmem {
  static constexpr uint32_t IMG = 4u * DTC_NE * 64u * 2u;        // one hi or lo image, two edge chunks
  static constexpr uint32_t BHI = 0;
  static constexpr uint32_t BLO = IMG;
  static constexpr uint32_t NP = 2 * IMG;                          // [ZTC_KMAX][MAXR]
  static constexpr uint32_t SDN = NP + 4u * ZTC_KMAX * MAXR;       // [ZTC_KMAX][MAXR] dE/dn^{(x)L} partials
  static constexpr uint32_t XOFF = SDN + 4u * ZTC_KMAX * MAXR;     // [ZTC_KMAX]
  static constexpr uint32_t BAR = XOFF + 8u * ZTC_KMAX;
  static constexpr uint32_t TOTAL = BAR + 16;
};
static_assert(3 * DtcSmem::TOTAL > 228u * 1024u, "at most two CTAs per SM (256 TMEM columns each)");

__device__ __forceinline__ int dimg(int n, int k) { return (k >> 2) * 4 * DTC_NE + 4 * n + (k & 3); }

__global__ void __launch_bounds__(ZTC_THREADS, 2) dm_tc_kernel(Args a, Rows rows, const float* __restrict__ h2,
                                                               const float* __restrict__ dZ, int64_t n0, int64_t nc,
                                                               float* __restrict__ dmbuf, int64_t e_base, int* err) {
  extern __shared__ __align__(1024) uint8_t smem[];
  float* bhi = reinterpret_cast<float*>(smem + DtcSmem::BHI);
  float* blo = reinterpret_cast<float*>(smem + DtcSmem::BLO);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + DtcSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + DtcSmem::BAR + 8);

  const int tid = threadIdx.x, warp = tid >> 5, half = tid / ZTC_M, row = tid % ZTC_M;
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t tD = tbase, tAhi = tbase + 128u, tAlo = tbase + 192u;  // D: 64 columns, A: 64 + 64
  const uint32_t s_hi = tc::smem_u32(bhi), s_lo = tc::smem_u32(blo);
  constexpr uint32_t idesc = tc::idesc_tf32(ZTC_M, DTC_NE);
  const int C = a.C, S = ZTC_M / C, slot = row / C, ch = row - slot * C;
  const int ntiles = (rows.nrows + S - 1) / S;
  uint32_t phase = 0;
  bool ok = true;

  for (int64_t nl = blockIdx.x; nl < nc && ok; nl += gridDim.x) {
    const int64_t n = n0 + nl;
    const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
    const float* dzn = dZ + nl * (int64_t)rows.nrows * J * C;
    for (int g0 = e0; g0 < e1 && ok; g0 += ZTC_KMAX) {
      const int kg = min(ZTC_KMAX, e1 - g0);
      const int nch = (kg + DTC_NE - 1) / DTC_NE;
      __syncthreads();
      for (int i = tid; i < nch * DTC_NE * 64; i += ZTC_THREADS) {
        const int k = i >> 6, j = i & 63;  // edge of the group, hidden unit
        const float v = k < kg ? h2[(int64_t)(g0 + k) * RH + j] : 0.f;
        uint32_t hi, lo;
        tc::split_tf32(v, hi, lo);
        const int o = (k / DTC_NE) * DTC_NE * 64 + dimg(k % DTC_NE, j);
        bhi[o] = __uint_as_float(hi);
        blo[o] = __uint_as_float(lo);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      for (int tile = 0; tile < ntiles && ok; ++tile) {
        const int q = tile * S + slot;
        const bool valid = q < rows.nrows;
        const int r = valid ? rows.rlist[q] : 0;
        const float* dzc = dzn + (int64_t)r * J * C + ch;
        // ---- A = dZ[n][r][j][a], columns j in [32 half, 32 half + 32)
        {
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v = valid ? dzc[(int64_t)(32 * half + i) * C] : 0.f;
            tc::split_tf32(v, hi[i], lo[i]);
          }
          tc::tmem_st32(tAhi + lane_off + 32u * half, hi);
          tc::tmem_st32(tAlo + lane_off + 32u * half, lo);
        }
        const float bias = valid ? dzc[(int64_t)RH * C] : 0.f;
        tc::tmem_wait_st();
        for (int cc = 0; cc < nch; ++cc) {
          tc::tc_fence_before();
          __syncthreads();  // A written (first chunk) / previous chunk's D read (later chunks)
          if (tid == 0) {
            tc::tc_fence_after();
            const uint32_t base = 4u * DTC_NE * 64u * (uint32_t)cc;
            for (int j = 0; j < 8; ++j) {
              const uint32_t off = base + 32u * DTC_NE * (uint32_t)j;
              const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * DTC_NE, 128);
              const uint64_t dl = tc::smem_desc_kmajor(s_lo + off, 16u * DTC_NE, 128);
              tc::mma_tf32_ts(tD, tAhi + 8u * j, dl, idesc, j > 0 ? 1u : 0u);
              tc::mma_tf32_ts(tD, tAlo + 8u * j, dh, idesc, 1u);
            }
            for (int j = 0; j < 8; ++j) {
              const uint32_t off = base + 32u * DTC_NE * (uint32_t)j;
              const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * DTC_NE, 128);
              tc::mma_tf32_ts(tD, tAhi + 8u * j, dh, idesc, 1u);
            }
            tc::mma_commit(bar);
          }
          const bool w = tid != 0 || tc::mbar_wait(bar, phase, err, 83);
          phase ^= 1u;
          const bool failed = __syncthreads_or(!w);
          tc::tc_fence_after();
          if (failed) {
            ok = false;
            break;
          }
          // ---- epilogue: dm of this thread's 32 edges kb .. kb + 31 of the group, written to the
          // chunk's dm rows (a warp writes 32 consecutive channels of one row: 128-byte runs)
          const int kb = cc * DTC_NE + 32 * half;
          uint32_t u[32];
          tc::tmem_ld32(tD + lane_off + 32u * half, u);
          tc::tmem_wait_ld();
          if (valid) {
            float* out = dmbuf + ((int64_t)(g0 - e_base) * rows.nrows + r) * C + ch;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (kb + i < kg) out[(int64_t)(kb + i) * rows.nrows * C] = __uint_as_float(u[i]) + bias;
          }
        }
      }
    }
  }
  if (!ok && tid == 0) {
    const long long t0 = clock64();
    while (!tc::mbar_try_wait(bar, phase ^ 1u))
      if (clock64() - t0 > tc::kWaitCycles) break;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

int launch_dm_tc(const Args& a, const Rows& rows, const float* h2, const float* dZ, int64_t n0, int64_t nc,
                 float* dmbuf, int64_t e_base, int* err, cudaStream_t st) {
  if (nc <= 0) return FSC_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaFuncSetAttribute(dm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DtcSmem::TOTAL) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "dm_tc_kernel: shared memory attribute");
  const unsigned blocks = (unsigned)std::min<int64_t>(nc, 2 * (int64_t)sms);
  dm_tc_kernel<<<blocks, ZTC_THREADS, DtcSmem::TOTAL, st>>>(a, rows, h2, dZ, n0, nc, dmbuf, e_base, err);
  return check_launch("sparse dm_tc_kernel");
}

// The fixed-order reductions of a sub-chunk's dm rows (edges [e_base, e_end)).
int launch_dm_reduce(const Args& a, const Rows& rows, const int32_t* tr_ptr, const int32_t* tr_eid, const float* x,
                     const float* dmbuf, int64_t e_base, int64_t e_end, float* gx, float* dnp, cudaStream_t st) {
  if (e_end <= e_base) return FSC_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned gs = (unsigned)std::min<int64_t>(ceil_div(a.N, 8), 16 * (int64_t)sms);
  const unsigned ge = (unsigned)std::min<int64_t>(ceil_div(e_end - e_base, 8), 16 * (int64_t)sms);
  auto go = [&](auto cpl) {
    constexpr int CPL = decltype(cpl)::value;
    dm_gx_kernel<CPL><<<gs, 256, 0, st>>>(a, rows, tr_ptr, tr_eid, dmbuf, e_base, e_end, gx);
    dm_dn_kernel<CPL><<<ge, 256, 0, st>>>(a, rows, x, dmbuf, e_base, e_end - e_base, dnp);
    return check_launch("sparse dm_gx / dm_dn kernels");
  };
  if (a.C == 32) return go(std::integral_constant<int, 1>{});
  if (a.C == 64) return go(std::integral_constant<int, 2>{});
  return go(std::integral_constant<int, 4>{});
}

// dh_kernel: dE/dh2_e[j] = sum_{(r, a)} dZ[n][r][j][a] * x1[src_e][c1(r)][a] * n_e^{(x)L2}[c2(r)],
// a (edges x columns) . (columns x 64) product tiled through shared memory (64 edges x 64 j per
// pass, 32 columns per step, 4 x 4 outputs per thread).
constexpr int DH_E = 64, DH_K = 32;

__global__ void __launch_bounds__(256) bwd_dh_kernel(Args a, Rows rows, const float* __restrict__ x,
                                                     const float* __restrict__ dZ, int64_t n0, float* __restrict__ dh2) {
  __shared__ float zt[DH_K][RH + 4];
  __shared__ float mt[DH_E][DH_K + 1];
  __shared__ float np[DH_E][MAXR];
  __shared__ int srcs[DH_E];
  const int64_t n = n0 + blockIdx.x;
  const int C = a.C, R = a.R;
  const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
  const int cols = rows.nrows * C;
  const float* dzn = dZ + (int64_t)blockIdx.x * rows.nrows * J * C;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int eb = e0; eb < e1; eb += DH_E) {
    const int ne = min(DH_E, e1 - eb);
    __syncthreads();
    if (threadIdx.x < ne) {
      const int e = eb + threadIdx.x;
      srcs[threadIdx.x] = a.src[e];
      const float* y = a.edge_y + 12 * (int64_t)e;
      npow_all(a.lmax, y[0], y[1], y[2], np[threadIdx.x]);
    }
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int col0 = 0; col0 < cols; col0 += DH_K) {
      __syncthreads();
      // dZ tile: zt[c][j] = dZ[n][r][j][a], (r, a) = column col0 + c
      for (int t = threadIdx.x; t < DH_K * RH; t += blockDim.x) {
        const int c = t % DH_K, j = t / DH_K;
        const int col = col0 + c;
        const int r = col / C, ch = col - r * C;
        zt[c][j] = dzn[((int64_t)r * J + j) * C + ch];
      }
      // message tile: mt[e][c] = x1[src_e][c1(r)][a] * n_e^{(x)L2}[c2(r)]
      for (int t = threadIdx.x; t < DH_E * DH_K; t += blockDim.x) {
        const int c = t % DH_K, k = t / DH_K;
        float v = 0.f;
        if (k < ne) {
          const int col = col0 + c;
          const int r = col / C, ch = col - r * C;
          v = x[((int64_t)srcs[k] * R + rows.c1[r]) * C + ch] * np[k][rows.c2[r]];
        }
        mt[k][c] = v;
      }
      __syncthreads();
#pragma unroll 8
      for (int c = 0; c < DH_K; ++c) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = mt[ty * 4 + i][c];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = zt[c][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = ty * 4 + i;
      if (k < ne)
#pragma unroll
        for (int j = 0; j < 4; ++j) dh2[(int64_t)(eb + k) * RH + tx * 4 + j] = acc[i][j];
    }
  }
}

// dh on tensor cores, per receiving node n and up to 128 of its edges (TMEM lane = edge):
//   D[e][j] = sum_{(r, a)} A[e][(r, a)] B[j][(r, a)],  A[e][(r, a)] = x1[src_e][c1(r)][a] n_e^{(x)L2}[c2(r)],
//   B[j][(r, a)] = dZ[n][r][j][a]   (M = 128, N = 64, K = rows x C in chunks of 32 channels, 3xTF32).
// Each chunk is a fresh 12-MMA chain; every second chunk the accumulator is added into fp32
// registers (short tensor-core chains, sums rounded to nearest), and dh2_e = the register sums.
// Warps w and w + 4 share lanes: each builds 16 of a chunk's 32 A columns and drains 32 of D's 64.
constexpr int HTC_KC = 32;
struct HtcSmem {
  static constexpr uint32_t IMG = 4u * 64u * HTC_KC;           // one hi or lo image: N = 64, K = 32
  static constexpr uint32_t BHI = 0;
  static constexpr uint32_t BLO = IMG;
  static constexpr uint32_t NP = 2 * IMG;                       // [ZTC_KMAX][MAXR]
  static constexpr uint32_t XOFF = NP + 4u * ZTC_KMAX * MAXR;   // [ZTC_KMAX]
  static constexpr uint32_t BAR = XOFF + 8u * ZTC_KMAX;
  static constexpr uint32_t USED = BAR + 16;
  static constexpr uint32_t TOTAL = USED > 80u * 1024u ? USED : 80u * 1024u;  // at most two CTAs per SM
};

__device__ __forceinline__ int himg(int n, int k) { return (k >> 2) * 4 * 64 + 4 * n + (k & 3); }

__global__ void __launch_bounds__(ZTC_THREADS, 2) dh_tc_kernel(Args a, Rows rows, const float* __restrict__ x,
                                                               const float* __restrict__ dZ, int64_t n0, int64_t nc,
                                                               float* __restrict__ dh2, int* err) {
  extern __shared__ __align__(1024) uint8_t smem[];
  float* bhi = reinterpret_cast<float*>(smem + HtcSmem::BHI);
  float* blo = reinterpret_cast<float*>(smem + HtcSmem::BLO);
  float* np = reinterpret_cast<float*>(smem + HtcSmem::NP);
  int64_t* xoff = reinterpret_cast<int64_t*>(smem + HtcSmem::XOFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + HtcSmem::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + HtcSmem::BAR + 8);

  const int tid = threadIdx.x, warp = tid >> 5, half = tid / ZTC_M, row = tid % ZTC_M;
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t tD = tbase, tAhi = tbase + 128u, tAlo = tbase + 192u;  // D: 64 columns, A: 32 + 32
  const uint32_t s_hi = tc::smem_u32(bhi), s_lo = tc::smem_u32(blo);
  constexpr uint32_t idesc = tc::idesc_tf32(ZTC_M, 64);
  const int C = a.C, R = a.R, cpr = C / HTC_KC;  // chunks per row
  const int nchunks = rows.nrows * cpr;
  uint32_t phase = 0;
  bool ok = true;

  for (int64_t nl = blockIdx.x; nl < nc && ok; nl += gridDim.x) {
    const int64_t n = n0 + nl;
    const int e0 = a.row_ptr[n], e1 = a.row_ptr[n + 1];
    const float* dzn = dZ + nl * (int64_t)rows.nrows * J * C;
    for (int g0 = e0; g0 < e1 && ok; g0 += ZTC_KMAX) {
      const int kg = min(ZTC_KMAX, e1 - g0);
      __syncthreads();
      if (tid < ZTC_KMAX) {
        if (tid < kg) {
          const int e = g0 + tid;
          xoff[tid] = (int64_t)a.src[e] * R * C;
          const float* y = a.edge_y + 12 * (int64_t)e;
          npow_all(a.lmax, y[0], y[1], y[2], np + tid * MAXR);
        } else {
          xoff[tid] = 0;
        }
      }
      __syncthreads();
      const bool erow = row < kg;
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0.f;
      for (int kc = 0; kc < nchunks && ok; ++kc) {
        const int r = kc / cpr, a0 = (kc - r * cpr) * HTC_KC;
        const int c1 = rows.c1[r], c2 = rows.c2[r];
        // ---- A columns [16 half, 16 half + 16) of the chunk: this lane's edge
        {
          float v[16];
          if (erow) {
            const float4* xs = reinterpret_cast<const float4*>(x + xoff[row] + (int64_t)c1 * C + a0 + 16 * half);
            const float w = np[row * MAXR + c2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 t = xs[i];
              v[4 * i] = t.x * w; v[4 * i + 1] = t.y * w; v[4 * i + 2] = t.z * w; v[4 * i + 3] = t.w * w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
          }
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) tc::split_tf32(v[i], hi[i], lo[i]);
          tc::tmem_st16(tAhi + lane_off + 16u * half, hi);
          tc::tmem_st16(tAlo + lane_off + 16u * half, lo);
        }
        // ---- B = dZ[n][r][j][a0 .. a0 + 32) for j < 64 (thread: one j, four channels, two passes)
        {
          const float* dzr = dzn + (int64_t)r * J * C + a0;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int i = tid + ZTC_THREADS * t, j = i & 63, k4 = i >> 6;
            const float4 v = *reinterpret_cast<const float4*>(dzr + (int64_t)j * C + 4 * k4);
            uint32_t h0, l0, h1, l1, h2_, l2, h3, l3;
            tc::split_tf32(v.x, h0, l0);
            tc::split_tf32(v.y, h1, l1);
            tc::split_tf32(v.z, h2_, l2);
            tc::split_tf32(v.w, h3, l3);
            const int o = himg(j, 4 * k4);
            *reinterpret_cast<uint4*>(bhi + o) = make_uint4(h0, h1, h2_, h3);
            *reinterpret_cast<uint4*>(blo + o) = make_uint4(l0, l1, l2, l3);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncthreads();
        if (tid == 0) {
          tc::tc_fence_after();
          const uint32_t acc0 = (kc & 1) ? 1u : 0u;  // chunks are summed in pairs on the tensor core
          for (int j = 0; j < HTC_KC / 8; ++j) {
            const uint32_t off = 32u * 64u * (uint32_t)j;
            const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * 64u, 128);
            const uint64_t dl = tc::smem_desc_kmajor(s_lo + off, 16u * 64u, 128);
            tc::mma_tf32_ts(tD, tAhi + 8u * j, dl, idesc, (j > 0 || acc0) ? 1u : 0u);
            tc::mma_tf32_ts(tD, tAlo + 8u * j, dh, idesc, 1u);
          }
          for (int j = 0; j < HTC_KC / 8; ++j) {
            const uint32_t off = 32u * 64u * (uint32_t)j;
            const uint64_t dh = tc::smem_desc_kmajor(s_hi + off, 16u * 64u, 128);
            tc::mma_tf32_ts(tD, tAhi + 8u * j, dh, idesc, 1u);
          }
          tc::mma_commit(bar);
        }
        const bool w = tid != 0 || tc::mbar_wait(bar, phase, err, 84);
        phase ^= 1u;
        const bool failed = __syncthreads_or(!w);
        tc::tc_fence_after();
        if (failed) {
          ok = false;
          break;
        }
        if ((kc & 1) || kc == nchunks - 1) {  // drain the pair's sum into the registers
          uint32_t u[32];
          tc::tmem_ld32(tD + lane_off + 32u * half, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(u[i]);
        }
        tc::tc_fence_before();
      }
      if (ok && erow) {
        float4* o = reinterpret_cast<float4*>(dh2 + (int64_t)(g0 + row) * RH + 32 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
      }
    }
  }
  if (!ok && tid == 0) {
    const long long t0 = clock64();
    while (!tc::mbar_try_wait(bar, phase ^ 1u))
      if (clock64() - t0 > tc::kWaitCycles) break;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

int launch_dh_tc(const Args& a, const Rows& rows, const float* x, const float* dZ, int64_t n0, int64_t nc, float* dh2,
                 int* err, cudaStream_t st) {
  if (nc <= 0) return FSC_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaFuncSetAttribute(dh_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)HtcSmem::TOTAL) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "dh_tc_kernel: shared memory attribute");
  const unsigned blocks = (unsigned)std::min<int64_t>(nc, 2 * (int64_t)sms);
  dh_tc_kernel<<<blocks, ZTC_THREADS, HtcSmem::TOTAL, st>>>(a, rows, x, dZ, n0, nc, dh2, err);
  return check_launch("sparse dh_tc_kernel");
}

// ---------------------------------------------------------------- edge gradient
// g_e = dE/d|r| n + (I - n n^T) / |r| dE/dn,  dE/dn from dE/dn^{(x)L}; dE/d|r| in g_e[0] on entry.
__global__ void edge_grad_kernel(int64_t E, int lmax, const float* __restrict__ ey, const float* __restrict__ dnp,
                                 float* __restrict__ g) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const float* y = ey + 12 * e;
  const float n[3] = {y[0], y[1], y[2]};
  const float len = y[3];
  float d[MAXR];
  for (int q = 0; q < MAXR; ++q) d[q] = dnp[e * MAXR + q];
  float dn[3];
  npow_grad(lmax, n, d, dn);
  const float dl = g[3 * e];
  const float inv = 1.f / fmaxf(len, 1e-8f);
  const float dot = dn[0] * n[0] + dn[1] * n[1] + dn[2] * n[2];
#pragma unroll
  for (int k = 0; k < 3; ++k) g[3 * e + k] = dl * n[k] + (len > 1e-8f ? (dn[k] - dot * n[k]) : dn[k]) * inv;
}

// ---------------------------------------------------------------- readout
// t_L[c'][m] = feats[c' / C][n][roff(L) + m][c' % C]; Gram over m < 3^L.
struct RdArgs {
  int64_t N;
  int C, R, nint, S;
  const float* feats[8];
};

// Gp[nl][j] = sum_m t_L[c][m] t_L[d][m], (c, d) = pairs[j]; grid (pair blocks, nodes)
// Gram operand of one node for Lout = L (M = 3^L components): Gp[n][j(c, d)] = sum_m t[c][m] t[d][m]
// over the packed upper triangle c <= d of the nC = C * nint concatenated channels, pair j(c, d) =
// c nC - c (c - 1) / 2 + d - c (the order of the W_read image).  One CTA per node holds the node's
// t as [M][nC] in shared memory; each warp walks triangle rows c, its lanes taking aligned quads
// d4 .. d4 + 3 (one float4 read per component), and a row's results leave through a per-warp
// staging buffer as coalesced runs.
template <int M>
__global__ void __launch_bounds__(256) gram_pack_kernel(RdArgs a, int L, int64_t n0, int64_t nn, int64_t npairs,
                                                        float* __restrict__ Gp) {
  extern __shared__ float4 gp_smem4[];
  float* ts = reinterpret_cast<float*>(gp_smem4);  // [M][nC], then [8 warps][128] staging
  const int nC = a.C * a.nint;
  const int64_t nl = blockIdx.x;
  const int64_t n = n0 + nl;
  for (int i = threadIdx.x; i < M * nC; i += blockDim.x) {
    const int m = i / nC, cp = i - m * nC, k = cp / a.C, c = cp - k * a.C;
    ts[i] = a.feats[k][(n * a.R + roff(L) + m) * a.C + c];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float* stage = ts + M * nC + warp * 128;
  float* gout = Gp + nl * npairs;
  for (int c = warp; c < nC; c += nw) {
    const int64_t j0 = (int64_t)c * nC - (int64_t)c * (c - 1) / 2 - c;  // pair index of (c, d) = j0 + d
    float tc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) tc[m] = ts[m * nC + c];
    for (int base = c & ~3; base < nC; base += 128) {
      const int d4 = base + 4 * lane;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (d4 < nC) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float4 t4 = reinterpret_cast<const float4*>(ts + m * nC)[d4 >> 2];
          acc.x = fmaf(tc[m], t4.x, acc.x);
          acc.y = fmaf(tc[m], t4.y, acc.y);
          acc.z = fmaf(tc[m], t4.z, acc.z);
          acc.w = fmaf(tc[m], t4.w, acc.w);
        }
      }
      reinterpret_cast<float4*>(stage)[lane] = acc;
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = base + lane + 32 * i;
        if (d >= c && d < nC) gout[j0 + d] = stage[lane + 32 * i];
      }
      __syncwarp();
    }
  }
}

// grads at t_L[c'][m] += 2 sum_d H[n][c'][d] t_L[d][m]; one CTA per node, two channels c' per
// thread.  t is held as [nC][M] in shared memory (a row of M values read as float4 broadcasts); H
// is symmetric (ds times the symmetrised W_read), so H[n][d][c'] is read: coalesced over c'.
template <int M>
__global__ void __launch_bounds__(192) gram_apply_kernel(RdArgs a, GradList g, int L, int64_t n0, int64_t nn,
                                                         const float* __restrict__ H) {
  constexpr int MP = (M + 3) / 4 * 4;
  extern __shared__ float4 ga_smem4[];
  float* ts = reinterpret_cast<float*>(ga_smem4);  // [nC][MP]
  const int nC = a.C * a.nint;
  const int64_t nl = blockIdx.x;
  const int64_t n = n0 + nl;
  for (int i = threadIdx.x; i < nC * MP; i += blockDim.x) {
    const int d = i / MP, m = i - d * MP, k = d / a.C, dd = d - k * a.C;
    ts[i] = m < M ? a.feats[k][(n * a.R + roff(L) + m) * a.C + dd] : 0.f;
  }
  __syncthreads();
  const int half = (nC + 1) / 2;
  const int c0 = threadIdx.x, c1 = threadIdx.x + half;
  const bool v0 = c0 < half, v1 = c1 < nC && v0;
  float acc0[MP], acc1[MP];
#pragma unroll
  for (int m = 0; m < MP; ++m) acc0[m] = acc1[m] = 0.f;
  const float* h = H + nl * (int64_t)nC * nC;
  if (v0) {
    for (int d = 0; d < nC; ++d) {
      const float h0 = h[(int64_t)d * nC + c0];
      const float h1 = v1 ? h[(int64_t)d * nC + c1] : 0.f;
      const float4* t4 = reinterpret_cast<const float4*>(ts + d * MP);
#pragma unroll
      for (int q = 0; q < MP / 4; ++q) {
        const float4 t = t4[q];
        acc0[4 * q] = fmaf(h0, t.x, acc0[4 * q]);
        acc0[4 * q + 1] = fmaf(h0, t.y, acc0[4 * q + 1]);
        acc0[4 * q + 2] = fmaf(h0, t.z, acc0[4 * q + 2]);
        acc0[4 * q + 3] = fmaf(h0, t.w, acc0[4 * q + 3]);
        acc1[4 * q] = fmaf(h1, t.x, acc1[4 * q]);
        acc1[4 * q + 1] = fmaf(h1, t.y, acc1[4 * q + 1]);
        acc1[4 * q + 2] = fmaf(h1, t.z, acc1[4 * q + 2]);
        acc1[4 * q + 3] = fmaf(h1, t.w, acc1[4 * q + 3]);
      }
    }
  }
  if (v0) {
    const int k = c0 / a.C, c = c0 - k * a.C;
    float* gp = g.p[k] + (n * a.R + roff(L)) * a.C + c;
#pragma unroll
    for (int m = 0; m < M; ++m) gp[m * a.C] += 2.f * acc0[m];
  }
  if (v1) {
    const int k = c1 / a.C, c = c1 - k * a.C;
    float* gp = g.p[k] + (n * a.R + roff(L)) * a.C + c;
#pragma unroll
    for (int m = 0; m < M; ++m) gp[m * a.C] += 2.f * acc1[m];
  }
}

int launch_gram_pack(const RdArgs& a, int L, int nC, int64_t n0, int64_t nn, int64_t npairs, float* Gp,
                     cudaStream_t st) {
  if (nn <= 0) return FSC_OK;
  const int M = pow3(L);
  const size_t smem = sizeof(float) * ((size_t)M * nC + 8 * 128);
  if (nC % 4 || smem > 227u * 1024u) return fail(FSC_ERR_UNSUPPORTED, "sparse gram_pack: channel count");
  auto go = [&](auto kernel) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "sparse gram_pack: shared memory attribute");
    kernel<<<(unsigned)nn, 256, smem, st>>>(a, L, n0, nn, npairs, Gp);
    return check_launch("sparse gram_pack_kernel");
  };
  switch (L) {
    case 0: return go(gram_pack_kernel<1>);
    case 1: return go(gram_pack_kernel<3>);
    case 2: return go(gram_pack_kernel<9>);
    case 3: return go(gram_pack_kernel<27>);
    default: return fail(FSC_ERR_UNSUPPORTED, "sparse gram_pack: lmax <= 3");
  }
}

int launch_gram_apply(const RdArgs& a, const GradList& g, int L, int nC, int64_t n0, int64_t nn, const float* H,
                      cudaStream_t st) {
  if (nn <= 0) return FSC_OK;
  const int M = pow3(L), MP = (M + 3) / 4 * 4;
  const int threads = (int)ceil_div((nC + 1) / 2, 32) * 32;
  const size_t smem = sizeof(float) * (size_t)nC * MP;
  if (threads > 192 || smem > 227u * 1024u) return fail(FSC_ERR_UNSUPPORTED, "sparse gram_apply: channel count");
  auto go = [&](auto kernel) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "sparse gram_apply: shared memory attribute");
    kernel<<<(unsigned)nn, threads, smem, st>>>(a, g, L, n0, nn, H);
    return check_launch("sparse gram_apply_kernel");
  };
  switch (L) {
    case 0: return go(gram_apply_kernel<1>);
    case 1: return go(gram_apply_kernel<3>);
    case 2: return go(gram_apply_kernel<9>);
    case 3: return go(gram_apply_kernel<27>);
    default: return fail(FSC_ERR_UNSUPPORTED, "sparse gram_apply: lmax <= 3");
  }
}

// MainNet input [layer k: L = 0..lmax: C] x nint | scalars^2 (S)
__global__ void p5_fwd_kernel(RdArgs a, int lmax, const float* __restrict__ scal, float* __restrict__ p5) {
  const int W = a.C * (lmax + 1);
  const int D0 = a.nint * W + a.S;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= a.N * D0) return;
  const int64_t n = idx / D0;
  const int j = (int)(idx - n * D0);
  float v;
  if (j < a.nint * W) {
    const int k = j / W, w = j - k * W, L = w / a.C, c = w - L * a.C;
    const float* f = a.feats[k] + (n * a.R + roff(L)) * a.C + c;
    float acc = 0.f;
    for (int m = 0; m < pow3(L); ++m) acc = fmaf(f[m * a.C], f[m * a.C], acc);
    v = acc * rsqrtf((float)pow3(L));
  } else {
    const float s = scal[n * a.S + (j - a.nint * W)];
    v = s * s;
  }
  p5[idx] = v;
}

__global__ void p5_bwd_kernel(RdArgs a, GradList g, int lmax, const float* __restrict__ scal,
                              const float* __restrict__ dp5, float* __restrict__ dscal) {
  const int W = a.C * (lmax + 1);
  const int D0 = a.nint * W + a.S;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= a.N * D0) return;
  const int64_t n = idx / D0;
  const int j = (int)(idx - n * D0);
  const float d = dp5[idx];
  if (j < a.nint * W) {
    const int k = j / W, w = j - k * W, L = w / a.C, c = w - L * a.C;
    const int64_t off = (n * a.R + roff(L)) * a.C + c;
    const float sc = 2.f * rsqrtf((float)pow3(L)) * d;
    for (int m = 0; m < pow3(L); ++m) g.p[k][off + m * a.C] = sc * a.feats[k][off + m * a.C];
  } else {
    const int o = j - a.nint * W;
    dscal[n * a.S + o] = 2.f * scal[n * a.S + o] * d;
  }
}

// per-graph sums of r (x) g (virial) or S (x) g (cell gradient), double atomics
__global__ void to_float_kernel(const double* __restrict__ in, int64_t n, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (float)in[i];
}

// ---------------------------------------------------------------- plan
struct Plan {
  int C, R, lmax, nint, S, nC, D0, nb, n_hidden, hidden[4];
  int64_t N, E, B, npairs, chunk, gchunk, zstride;
  Rows rows;
  int32_t* dst;
  float* edge_y;
  float* h2;
  float* feats[8];
  float* zbuf;
  float* scalars;
  float* p5;
  float* x0;
  float* act_pre[4];
  float* act_post[4];
  double* acc_d;  // energy [4096] | virial [4096][9] | cell grad [4096][9]
  float* grads[8];
  float* dscalars;
  float* dp5;
  float* dxa;
  float* dxb;
  float* dh2;
  float* dnp;
  float* dmbuf;    // [dmcap][nrows][C] dm rows of one sub-chunk of receivers (conv2 backward)
  int64_t dmcap;   // edges of a sub-chunk
  float* edge_grad;
  float* gbuf;
  int* err;
  // tensor-core GEMM operand images of the weights (null: CUDA-core GEMM)
  bool gtc;
  bool atc;  // per-node aggregation kernels (z / dm / dh) on tensor cores
  float* img_mix[8][4];    // conv2 layer k, Lout: fc.4 regrouped, forward
  float* img_mixT[8][4];   // its transpose (backward dZ)
  float* img_gf[4];        // packed Gram x W_read (forward), per L
  float* img_gb[4];        // ds x W_read (backward), per L
  float* img_mnf[4];
  float* img_mnb[4];
};

int validate(const fsc_sparse_config* cfg) {
  FSC_REQUIRE(cfg != nullptr, "config is null");
  if (cfg->lmax != 2 && cfg->lmax != 3) return fail(FSC_ERR_UNSUPPORTED, "sparse engine supports lmax 2 or 3");
  if (cfg->channels != 32 && cfg->channels != 64 && cfg->channels != 128)
    return fail(FSC_ERR_UNSUPPORTED, "sparse engine supports channels 32, 64 or 128");
  if (cfg->num_interaction < 2 || cfg->num_interaction > 8) return fail(FSC_ERR_UNSUPPORTED, "num_interaction in [2, 8]");
  if (cfg->number_of_basis < 1 || cfg->number_of_basis > 16) return fail(FSC_ERR_UNSUPPORTED, "number_of_basis in [1, 16]");
  if (cfg->basis_kind != 0 && cfg->basis_kind != 1) return fail(FSC_ERR_UNSUPPORTED, "gaussian or bessel basis");
  if (cfg->n_hidden < 1 || cfg->n_hidden > 4) return fail(FSC_ERR_UNSUPPORTED, "MainNet needs 1..4 hidden layers");
  if (cfg->num_species < 1 || cfg->num_species > 128) return fail(FSC_ERR_UNSUPPORTED, "num_species in [1, 128]");
  if (cfg->invariant_channels < 1) return fail(FSC_ERR_ARGUMENT, "invariant_channels must be >= 1");
  if (cfg->channels * cfg->num_interaction > 65535) return fail(FSC_ERR_UNSUPPORTED, "too many channels");
  if (!(cfg->avg_num_neighbors >= 0.f) || !std::isfinite(cfg->avg_num_neighbors))
    return fail(FSC_ERR_ARGUMENT, "avg_num_neighbors must be finite and >= 0");
  return FSC_OK;
}

void layout(Plan& p, Arena& ar, const fsc_sparse_config* cfg, int64_t N, int64_t E) {
  p.C = cfg->channels;
  p.lmax = cfg->lmax;
  p.R = roff(p.lmax + 1);
  p.nint = cfg->num_interaction;
  p.S = (p.nint - 1) * cfg->invariant_channels;
  p.nC = p.C * p.nint;
  p.D0 = p.nint * p.C * (p.lmax + 1) + p.S;
  p.nb = cfg->number_of_basis;
  p.n_hidden = cfg->n_hidden;
  for (int k = 0; k < 4; ++k) p.hidden[k] = k < p.n_hidden ? cfg->hidden[k] : 0;
  p.N = N;
  p.E = E;
  p.rows = make_rows(p.lmax);
  p.zstride = (int64_t)p.rows.nrows * J * p.C;
  p.chunk = std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>(N, 1), kZBudgetFloats / p.zstride));
  p.npairs = (int64_t)p.nC * (p.nC + 1) / 2;
  p.gchunk = std::max<int64_t>(1, std::min<int64_t>(N, kGramChunk));
  int maxw = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) maxw = std::max(maxw, p.hidden[k]);
  const int64_t fsz = N * p.R * p.C;
  p.dst = ar.take<int32_t>(E);
  p.edge_y = ar.take<float>(E * 12);
  p.h2 = ar.take<float>((int64_t)p.nint * E * RH);
  for (int k = 0; k < p.nint; ++k) p.feats[k] = ar.take<float>(fsz);
  p.zbuf = ar.take<float>(p.chunk * p.zstride);
  p.scalars = ar.take<float>(N * p.S);
  p.p5 = ar.take<float>(N * p.D0);
  p.x0 = ar.take<float>(N * p.D0);
  for (int k = 0; k < p.n_hidden; ++k) {
    p.act_pre[k] = ar.take<float>(N * p.hidden[k]);
    p.act_post[k] = ar.take<float>(N * p.hidden[k]);
  }
  p.acc_d = ar.take<double>(kMaxGraphs * 19);
  for (int k = 0; k < p.nint; ++k) p.grads[k] = ar.take<float>(fsz);
  p.dscalars = ar.take<float>(N * p.S);
  p.dp5 = ar.take<float>(N * p.D0);
  p.dxa = ar.take<float>(N * maxw);
  p.dxb = ar.take<float>(N * maxw);
  p.dh2 = ar.take<float>((int64_t)p.nint * E * RH);
  p.dnp = ar.take<float>(E * MAXR);
  p.dmcap = std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>(E, 1), kDmBudgetFloats / ((int64_t)p.rows.nrows * p.C)));
  p.dmbuf = ar.take<float>(p.dmcap * p.rows.nrows * p.C);
  p.edge_grad = ar.take<float>(E * 3);
  p.gbuf = ar.take<float>(p.gchunk * std::max<int64_t>(p.npairs, (int64_t)p.nC * p.nC));
  p.err = ar.take<int>(64);
  // gemm_path 0: both on tensor cores; 1: both on CUDA cores; 2: tensor-core aggregation with
  // CUDA-core GEMMs; 3: CUDA-core aggregation with tensor-core GEMMs
  p.gtc = gemm_path() == 0 || gemm_path() == 3;
  p.atc = gemm_path() == 0 || gemm_path() == 2;
  for (int k = 0; k < 8; ++k)
    for (int L = 0; L < 4; ++L) p.img_mix[k][L] = p.img_mixT[k][L] = nullptr;
  for (int k = 0; k < 4; ++k) p.img_gf[k] = p.img_gb[k] = p.img_mnf[k] = p.img_mnb[k] = nullptr;
  if (p.gtc) {
    for (int k = 1; k < p.nint; ++k)
      for (int L = 0; L <= p.lmax; ++L) {
        const int K = p.rows.npl[L] * J * p.C;
        p.img_mix[k][L] = ar.take<float>(gemm_image_floats(K, p.C));
        p.img_mixT[k][L] = ar.take<float>(gemm_image_floats(p.C, K));
      }
    for (int L = 0; L <= p.lmax; ++L) {
      p.img_gf[L] = ar.take<float>(gemm_image_floats((int)p.npairs, p.S));
      p.img_gb[L] = ar.take<float>(gemm_image_floats(p.S, p.nC * p.nC));
    }
    int din = p.D0;
    for (int k = 0; k < p.n_hidden; ++k) {
      p.img_mnf[k] = ar.take<float>(gemm_image_floats(din, p.hidden[k]));
      p.img_mnb[k] = ar.take<float>(gemm_image_floats(p.hidden[k], din));
      din = p.hidden[k];
    }
  }
}

struct Ctx {
  const fsc_sparse_config* cfg;
  const fsc_sparse_weights* w;
  const fsc_graph* g;
  Plan p;
  cudaStream_t st;
  std::vector<int32_t> row_ptr_host;  // conv2 backward: sub-chunks of at most p.dmcap edges
};

Args args(const Ctx& c) {
  Args a{};
  a.N = c.p.N;
  a.E = c.p.E;
  a.C = c.p.C;
  a.R = c.p.R;
  a.lmax = c.p.lmax;
  a.S_species = c.cfg->num_species;
  a.row_ptr = c.g->row_ptr;
  a.src = c.g->src;
  a.dst = c.p.dst;
  a.species = c.g->species;
  a.edge_y = c.p.edge_y;
  return a;
}

RdArgs rd_args(const Plan& p) {
  RdArgs r{};
  r.N = p.N;
  r.C = p.C;
  r.R = p.R;
  r.nint = p.nint;
  r.S = p.S;
  for (int k = 0; k < p.nint; ++k) r.feats[k] = p.feats[k];
  return r;
}

RadialW radial(const fsc_sparse_weights* w) {
  RadialW r{};
  r.w1 = w->rad_w1;
  r.b1 = w->rad_b1;
  r.w2 = w->rad_w2;
  r.b2 = w->rad_b2;
  r.w3 = nullptr;
  r.b3 = nullptr;
  return r;
}

GemmArgs gemm(const float* A, int64_t a_gs, int64_t a_rs, const float* B, int64_t ldb, int b_trans, float* C,
              int64_t c_gs, int64_t c_rs, int64_t G, int R, int K, int N) {
  GemmArgs g{};
  g.A = A; g.a_gs = a_gs; g.a_rs = a_rs;
  g.B = B; g.ldb = ldb; g.b_trans = b_trans;
  g.C = C; g.c_gs = c_gs; g.c_rs = c_rs;
  g.G = G; g.R = R; g.K = K; g.N = N;
  return g;
}

// offset (floats) of layer k's mix block of rank Lout
int64_t mix_offset(const Plan& p, int k, int Lout);

// Builds every weight image the tensor-core GEMMs of this call read.
int build_gemm_images(const Plan& p, const fsc_sparse_weights* w, cudaStream_t st) {
  if (!p.gtc) return FSC_OK;
  GemmImageBatch jobs;
  for (int k = 1; k < p.nint; ++k)
    for (int L = 0; L <= p.lmax; ++L) {
      const int K = p.rows.npl[L] * J * p.C;
      FSC_TRY(jobs.add(w->mix + mix_offset(p, k, L), p.C, 0, K, p.C, p.img_mix[k][L], st));
      FSC_TRY(jobs.add(w->mixT + mix_offset(p, k, L), K, 0, p.C, K, p.img_mixT[k][L], st));
    }
  for (int L = 0; L <= p.lmax; ++L) {
    FSC_TRY(jobs.add(w->wread_p + (int64_t)L * p.S * p.npairs, p.npairs, 1, (int)p.npairs, p.S, p.img_gf[L], st));
    FSC_TRY(jobs.add(w->wread_s + (int64_t)L * p.S * p.nC * p.nC, (int64_t)p.nC * p.nC, 0, p.S, p.nC * p.nC,
                     p.img_gb[L], st));
  }
  int din = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) {
    FSC_TRY(jobs.add(w->mn_w[k], din, 1, din, p.hidden[k], p.img_mnf[k], st));
    FSC_TRY(jobs.add(w->mn_w[k], din, 0, p.hidden[k], din, p.img_mnb[k], st));
    din = p.hidden[k];
  }
  return jobs.flush(st);
}

int64_t mix_offset(const Plan& p, int k, int Lout) {
  int64_t per_layer = 0;
  for (int L = 0; L <= p.lmax; ++L) per_layer += (int64_t)p.rows.npl[L] * J * p.C * p.C;
  int64_t off = (int64_t)(k - 1) * per_layer;
  for (int L = 0; L < Lout; ++L) off += (int64_t)p.rows.npl[L] * J * p.C * p.C;
  return off;
}

template <typename F>
int by_cpl(int C, F f) {
  if (C == 32) return f(std::integral_constant<int, 1>{});
  if (C == 64) return f(std::integral_constant<int, 2>{});
  return f(std::integral_constant<int, 4>{});
}

// avg_num_neighbors of the conv2 layers: the caller's value, else E / N of this graph
float conv2_norm(const Ctx& c) {
  if (c.cfg->avg_num_neighbors > 0.f) return c.cfg->avg_num_neighbors;
  return (float)std::max(1e-8, (double)c.p.E / (double)std::max<int64_t>(c.p.N, 1));
}

// Forward in steps (fsc_sparse_forward_step): 0 = edge geometry, radial MLPs and conv1; k in
// [1, nint) = conv2 layer k; nint = readout.
int forward_step0(Ctx& c) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  prof::mark("begin", st);
  FSC_TRY(build_gemm_images(p, w, st));
  FSC_TRY(launch_edge_dst(g->row_ptr, p.dst, p.N, st));
  if (p.E > 0) {
    geom_kernel<<<(unsigned)ceil_div(p.E, 256), 256, 0, st>>>(p.E, g->pos, g->src, p.dst, g->batch, g->cell, g->shift,
                                                             p.edge_y);
    FSC_TRY(check_launch("sparse geom_kernel"));
  }
  RadialTcArgs ra{};
  ra.E = p.E; ra.rad = radial(w); ra.nint = p.nint; ra.nb = p.nb; ra.basis_kind = c.cfg->basis_kind;
  ra.rc = c.cfg->max_radius; ra.edge_y = p.edge_y; ra.err = p.err; ra.hout = p.h2;
  FSC_TRY(launch_radial_fwd_tc(ra, st));
  prof::mark("sparse_radial_forward", st);
  Args a = args(c);
  if (p.N > 0) {
    FSC_TRY(by_cpl(p.C, [&](auto cpl) {
      conv1_fwd_kernel<decltype(cpl)::value><<<(unsigned)ceil_div(p.N, 8), 256, 0, st>>>(a, w->pair_k, p.h2, p.feats[0]);
      return check_launch("sparse conv1_fwd_kernel");
    }));
  }
  prof::mark("sparse_conv1_forward", st);
  return FSC_OK;
}

int forward_conv2(Ctx& c, int k) {
  Plan& p = c.p;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  Args a = args(c);
  const float avg = conv2_norm(c);
  {
    for (int64_t n0 = 0; n0 < p.N; n0 += p.chunk) {
      const int64_t nc = std::min(p.chunk, p.N - n0);
      if (p.atc) {
        FSC_TRY(launch_z_tc(a, p.rows, p.feats[k - 1], p.h2 + (int64_t)k * p.E * RH, n0, nc, p.zbuf, p.err, st));
      } else {
        z_kernel<<<(unsigned)nc, 256, 0, st>>>(a, p.rows, p.feats[k - 1], p.h2 + (int64_t)k * p.E * RH, n0, p.zbuf);
        FSC_TRY(check_launch("sparse z_kernel"));
      }
      for (int Lo = 0; Lo <= p.lmax; ++Lo) {
        const int K = p.rows.npl[Lo] * J * p.C;
        GemmArgs ga = gemm(p.zbuf + (int64_t)p.rows.zoff[Lo] * J * p.C, p.zstride, K, w->mix + mix_offset(p, k, Lo),
                           p.C, 0, p.feats[k] + (n0 * p.R + roff(Lo)) * p.C, (int64_t)p.R * p.C, p.C, nc, pow3(Lo),
                           K, p.C);
        ga.alpha = 1.f / avg;
        FSC_TRY(run_gemm(ga, p.img_mix[k][Lo], p.err, st));
      }
    }
    prof::mark("sparse_conv2_forward", st);
  }
  return FSC_OK;
}

int forward_readout(Ctx& c) {
  Plan& p = c.p;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  // readout: bilinear invariants of the channel concatenation, 0e products, MainNet
  RdArgs rd = rd_args(p);
  if (cudaMemsetAsync(p.scalars, 0, sizeof(float) * p.N * p.S, st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset");
  for (int L = 0; L <= p.lmax; ++L) {
    const float* Wp = w->wread_p + (int64_t)L * p.S * p.npairs;
    for (int64_t n0 = 0; n0 < p.N; n0 += p.gchunk) {
      const int64_t nn = std::min(p.gchunk, p.N - n0);
      FSC_TRY(launch_gram_pack(rd, L, p.C * p.nint, n0, nn, p.npairs, p.gbuf, st));
      GemmArgs ga = gemm(p.gbuf, p.npairs, 0, Wp, p.npairs, 1, p.scalars + n0 * p.S, p.S, 0, nn, 1, (int)p.npairs, p.S);
      ga.accumulate = 1;
      ga.precise = 1;  // K = nC (nC + 1) / 2 Gram pairs whose terms cancel heavily
      FSC_TRY(run_gemm(ga, p.img_gf[L], p.err, st));
    }
  }
  prof::mark("sparse_readout_gram_forward", st);
  if (p.N > 0) {
    p5_fwd_kernel<<<(unsigned)ceil_div(p.N * p.D0, 256), 256, 0, st>>>(rd, p.lmax, p.scalars, p.p5);
    FSC_TRY(check_launch("sparse p5_fwd_kernel"));
  }
  FSC_TRY(launch_layernorm(p.p5, p.N, p.D0, w->mn_in_g, w->mn_in_b, 0, p.x0, st));
  const float* xin = p.x0;
  int din = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) {
    GemmArgs ga = gemm(xin, din, 0, w->mn_w[k], din, 1, p.act_pre[k], p.hidden[k], 0, p.N, 1, din, p.hidden[k]);
    ga.bias = w->mn_b[k];
    FSC_TRY(run_gemm(ga, p.img_mnf[k], p.err, st));
    FSC_TRY(launch_layernorm(p.act_pre[k], p.N, p.hidden[k], w->mn_g[k], w->mn_beta[k], 1, p.act_post[k], st));
    xin = p.act_post[k];
    din = p.hidden[k];
  }
  prof::mark("sparse_readout_mlp_forward", st);
  return FSC_OK;
}

// Backward in steps (fsc_sparse_backward_step): nint = readout backward; k in [1, nint) = conv2
// layer k backward (adds into layer k - 1's feature gradient); 0 = conv1 backward and the edge part.
int backward_readout(Ctx& c) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  const int H = p.hidden[p.n_hidden - 1];
  FSC_TRY(launch_energy_seed(p.N, H, w->out_v, g->energy_weight, g->num_local, p.dxa, st));
  float* dcur = p.dxa;
  float* dnext = p.dxb;
  for (int k = p.n_hidden - 1; k >= 0; --k) {
    const int din = k == 0 ? p.D0 : p.hidden[k - 1];
    FSC_TRY(launch_layernorm_backward(p.act_pre[k], dcur, p.N, p.hidden[k], w->mn_g[k], w->mn_beta[k], 1, dnext, st));
    GemmArgs ga = gemm(dnext, p.hidden[k], 0, w->mn_w[k], din, 0, dcur, din, 0, p.N, 1, p.hidden[k], din);
    FSC_TRY(run_gemm(ga, p.img_mnb[k], p.err, st));
  }
  FSC_TRY(launch_layernorm_backward(p.p5, dcur, p.N, p.D0, w->mn_in_g, w->mn_in_b, 0, p.dp5, st));
  RdArgs rd = rd_args(p);
  GradList gl{};
  for (int k = 0; k < p.nint; ++k) gl.p[k] = p.grads[k];
  if (p.N > 0) {
    p5_bwd_kernel<<<(unsigned)ceil_div(p.N * p.D0, 256), 256, 0, st>>>(rd, gl, p.lmax, p.scalars, p.dp5, p.dscalars);
    FSC_TRY(check_launch("sparse p5_bwd_kernel"));
  }
  prof::mark("sparse_readout_mlp_backward", st);
  for (int L = 0; L <= p.lmax; ++L) {
    const float* Ws = w->wread_s + (int64_t)L * p.S * p.nC * p.nC;
    for (int64_t n0 = 0; n0 < p.N; n0 += p.gchunk) {
      const int64_t nn = std::min(p.gchunk, p.N - n0);
      GemmArgs ga = gemm(p.dscalars + n0 * p.S, p.S, 0, Ws, (int64_t)p.nC * p.nC, 0, p.gbuf, (int64_t)p.nC * p.nC, 0,
                         nn, 1, p.S, p.nC * p.nC);
      FSC_TRY(run_gemm(ga, p.img_gb[L], p.err, st));
      FSC_TRY(launch_gram_apply(rd, gl, L, p.C * p.nint, n0, nn, p.gbuf, st));
    }
  }
  prof::mark("sparse_readout_gram_backward", st);
  if (cudaMemsetAsync(p.dnp, 0, sizeof(float) * p.E * MAXR, st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset");
  return FSC_OK;
}

int backward_conv2(Ctx& c, int k) {
  Plan& p = c.p;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  Args a = args(c);
  const float avg = conv2_norm(c);
  if ((int64_t)c.row_ptr_host.size() != p.N + 1) {  // once per call: the sub-chunk boundaries
    c.row_ptr_host.resize(p.N + 1);
    if (cudaMemcpyAsync(c.row_ptr_host.data(), c.g->row_ptr, sizeof(int32_t) * (p.N + 1), cudaMemcpyDeviceToHost,
                        st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "row_ptr readback");
  }
  {
    for (int64_t n0 = 0; n0 < p.N; n0 += p.chunk) {
      const int64_t nc = std::min(p.chunk, p.N - n0);
      for (int Lo = 0; Lo <= p.lmax; ++Lo) {
        const int K = p.rows.npl[Lo] * J * p.C;
        GemmArgs ga = gemm(p.grads[k] + (n0 * p.R + roff(Lo)) * p.C, (int64_t)p.R * p.C, p.C,
                           w->mixT + mix_offset(p, k, Lo), K, 0, p.zbuf + (int64_t)p.rows.zoff[Lo] * J * p.C,
                           p.zstride, K, nc, pow3(Lo), p.C, K);
        ga.alpha = 1.f / avg;
        FSC_TRY(run_gemm(ga, p.img_mixT[k][Lo], p.err, st));
      }
      // dm rows of sub-chunks of at most dmcap edges, each reduced in a fixed order (no atomics)
      for (int64_t m0 = n0; m0 < n0 + nc;) {
        const int64_t eb = c.row_ptr_host[m0];
        int64_t m1 = m0 + 1;
        while (m1 < n0 + nc && c.row_ptr_host[m1 + 1] - eb <= p.dmcap) ++m1;
        const int64_t ee = c.row_ptr_host[m1];
        if (ee - eb > p.dmcap) return fail(FSC_ERR_CAPACITY, "sparse conv2 backward: a receiver has more edges "
                                                           "than the dm buffer holds");
        const float* dz = p.zbuf + (m0 - n0) * p.zstride;
        if (p.atc) {
          FSC_TRY(launch_dm_tc(a, p.rows, p.h2 + (int64_t)k * p.E * RH, dz, m0, m1 - m0, p.dmbuf, eb, p.err, st));
        } else if (m1 > m0) {
          bwd_dm_kernel<<<(unsigned)(m1 - m0), 256, 0, st>>>(a, p.rows, p.h2 + (int64_t)k * p.E * RH, dz, m0,
                                                              p.dmbuf, eb);
          FSC_TRY(check_launch("sparse bwd_dm_kernel"));
        }
        FSC_TRY(launch_dm_reduce(a, p.rows, c.g->tr_ptr, c.g->tr_eid, p.feats[k - 1], p.dmbuf, eb, ee,
                                 p.grads[k - 1], p.dnp, st));
        m0 = m1;
      }
      if (p.atc) {
        FSC_TRY(launch_dh_tc(a, p.rows, p.feats[k - 1], p.zbuf, n0, nc, p.dh2 + (int64_t)k * p.E * RH, p.err, st));
      } else {
        bwd_dh_kernel<<<(unsigned)nc, 256, 0, st>>>(a, p.rows, p.feats[k - 1], p.zbuf, n0,
                                                     p.dh2 + (int64_t)k * p.E * RH);
        FSC_TRY(check_launch("sparse bwd_dh_kernel"));
      }
    }
    prof::mark("sparse_conv2_backward", st);
  }
  return FSC_OK;
}

int backward_conv1(Ctx& c) {
  Plan& p = c.p;
  const fsc_sparse_weights* w = c.w;
  cudaStream_t st = c.st;
  Args a = args(c);
  if (p.N > 0) {
    FSC_TRY(by_cpl(p.C, [&](auto cpl) {
      conv1_bwd_kernel<decltype(cpl)::value><<<(unsigned)ceil_div(p.N, 8), 256, 0, st>>>(a, w->pair_k, p.h2, p.grads[0],
                                                                                         p.dh2, p.dnp);
      return check_launch("sparse conv1_bwd_kernel");
    }));
  }
  prof::mark("sparse_conv1_backward", st);
  return FSC_OK;
}

int prepare(Ctx& c, void* workspace, size_t bytes) {
  const fsc_graph* g = c.g;
  FSC_TRY(validate(c.cfg));
  FSC_REQUIRE(c.w && g, "weights/graph is null");
  FSC_REQUIRE(g->num_atoms >= 0 && g->num_edges >= 0 && g->num_graphs >= 1, "bad graph sizes");
  FSC_REQUIRE(g->num_atoms < (int64_t)INT32_MAX && g->num_edges < (int64_t)INT32_MAX, "graph too large");
  FSC_REQUIRE(g->num_graphs <= kMaxGraphs, "too many graphs per call (max 4096)");
  FSC_REQUIRE(g->num_local >= 0 && g->num_local <= g->num_atoms, "num_local out of range");
  if (g->layer_atoms) return fail(FSC_ERR_UNSUPPORTED, "layer_atoms is supported by the ictd engine only");
  Arena ar(workspace, bytes);
  layout(c.p, ar, c.cfg, g->num_atoms, g->num_edges);
  if (!ar.ok() || workspace == nullptr)
    return fail(FSC_ERR_CAPACITY, "workspace too small: need " + std::to_string(ar.off) + " bytes");
  c.p.B = g->num_graphs;
  return FSC_OK;
}

int run_forward_step(Ctx& c, int step, float* energy, float* atom_energy) {
  Plan& p = c.p;
  if (step == 0) {
    if (cudaMemsetAsync(p.acc_d, 0, sizeof(double) * kMaxGraphs * 19, c.st) != cudaSuccess ||
        cudaMemsetAsync(p.err, 0, sizeof(int) * 64, c.st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset accumulators");
    return forward_step0(c);
  }
  if (step < p.nint) return forward_conv2(c, step);
  FSC_TRY(forward_readout(c));
  const int H = p.hidden[p.n_hidden - 1];
  float* ebuf = atom_energy ? atom_energy : p.dxb;
  FSC_TRY(launch_energy(p.act_post[p.n_hidden - 1], p.N, H, c.w->out_v, c.w->out_c0, c.g->batch, c.g->num_local, ebuf,
                        nullptr, c.st));
  FSC_TRY(launch_graph_reduce(1, ebuf, nullptr, nullptr, nullptr, c.g->batch, p.N, c.g->num_local, p.acc_d, nullptr,
                              c.st));
  if (energy) {
    to_float_kernel<<<(unsigned)ceil_div(p.B, 256), 256, 0, c.st>>>(p.acc_d, p.B, energy);
    FSC_TRY(check_launch("sparse to_float_kernel"));
  }
  return FSC_OK;
}

int run_forward(Ctx& c, float* energy, float* atom_energy) {
  for (int step = 0; step <= c.p.nint; ++step) FSC_TRY(run_forward_step(c, step, energy, atom_energy));
  return FSC_OK;
}

int run_backward_edges(Ctx& c, fsc_ictd_outputs* out);

int run_backward_step(Ctx& c, int step, fsc_ictd_outputs* out) {
  if (step == c.p.nint) return backward_readout(c);
  if (step > 0) return backward_conv2(c, step);
  FSC_TRY(backward_conv1(c));
  return run_backward_edges(c, out);
}

int run_backward(Ctx& c, fsc_ictd_outputs* out) {
  for (int step = c.p.nint; step >= 0; --step) FSC_TRY(run_backward_step(c, step, out));
  return FSC_OK;
}

int run_backward_edges(Ctx& c, fsc_ictd_outputs* out) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  float* eg = out->edge_grad ? out->edge_grad : p.edge_grad;
  RadialTcArgs ra{};
  ra.E = p.E; ra.rad = radial(c.w); ra.nint = p.nint; ra.nb = p.nb; ra.basis_kind = c.cfg->basis_kind;
  ra.rc = c.cfg->max_radius; ra.edge_y = p.edge_y; ra.err = p.err; ra.edge_grad = eg; ra.hout_grad = p.dh2;
  FSC_TRY(launch_radial_bwd_tc(ra, c.st));
  if (p.E > 0) {
    edge_grad_kernel<<<(unsigned)ceil_div(p.E, 256), 256, 0, c.st>>>(p.E, p.lmax, p.edge_y, p.dnp, eg);
    FSC_TRY(check_launch("sparse edge_grad_kernel"));
  }
  prof::mark("sparse_edge_backward", c.st);
  if (out->forces) FSC_TRY(launch_forces(g->row_ptr, g->tr_ptr, g->tr_eid, eg, out->forces, p.N, c.st));
  double* vir = p.acc_d + kMaxGraphs;
  double* cg = p.acc_d + 10 * kMaxGraphs;
  if (out->virial) {
    if (cudaMemsetAsync(vir, 0, sizeof(double) * 9 * kMaxGraphs, c.st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset");
    FSC_TRY(launch_graph_reduce(9, nullptr, p.edge_y, eg, g->src, g->batch, p.E, p.E, vir, nullptr, c.st));
    to_float_kernel<<<(unsigned)ceil_div(9 * p.B, 256), 256, 0, c.st>>>(vir, 9 * p.B, out->virial);
    FSC_TRY(check_launch("sparse virial"));
  }
  if (out->cell_grad) {
    if (cudaMemsetAsync(cg, 0, sizeof(double) * 9 * kMaxGraphs, c.st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset");
    FSC_TRY(launch_graph_reduce(9, nullptr, p.edge_y, eg, g->src, g->batch, p.E, p.E, cg, g->shift, c.st));
    to_float_kernel<<<(unsigned)ceil_div(9 * p.B, 256), 256, 0, c.st>>>(cg, 9 * p.B, out->cell_grad);
    FSC_TRY(check_launch("sparse cell grad"));
  }
  prof::mark("sparse_forces_virial", c.st);
  return FSC_OK;
}

}  // namespace sp
}  // namespace fsc

using namespace fsc;

extern "C" {

size_t fsc_sparse_workspace_bytes(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges) {
  if (!cfg || sp::validate(cfg) != FSC_OK) return 0;
  sp::Plan p{};
  Arena ar(nullptr, 0);
  sp::layout(p, ar, cfg, num_atoms, num_edges);
  return ar.off;
}

int fsc_sparse_forward(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g, float* energy,
                       float* atom_energy, void* workspace, size_t workspace_bytes, void* stream) {
  sp::Ctx c{cfg, w, g, sp::Plan{}, as_stream(stream)};
  FSC_TRY(sp::prepare(c, workspace, workspace_bytes));
  return sp::run_forward(c, energy, atom_energy);
}

int fsc_sparse_backward(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g,
                        fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(out != nullptr, "outputs required");
  sp::Ctx c{cfg, w, g, sp::Plan{}, as_stream(stream)};
  FSC_TRY(sp::prepare(c, workspace, workspace_bytes));
  return sp::run_backward(c, out);
}

int fsc_sparse_forward_step(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g, int step,
                            float* energy, float* atom_energy, void* workspace, size_t workspace_bytes, void* stream) {
  sp::Ctx c{cfg, w, g, sp::Plan{}, as_stream(stream)};
  FSC_TRY(sp::prepare(c, workspace, workspace_bytes));
  FSC_REQUIRE(step >= 0 && step <= c.p.nint, "forward step out of range [0, num_interaction]");
  return sp::run_forward_step(c, step, energy, atom_energy);
}

int fsc_sparse_backward_step(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g, int step,
                             fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream) {
  sp::Ctx c{cfg, w, g, sp::Plan{}, as_stream(stream)};
  FSC_TRY(sp::prepare(c, workspace, workspace_bytes));
  FSC_REQUIRE(step >= 0 && step <= c.p.nint, "backward step out of range [0, num_interaction]");
  FSC_REQUIRE(step > 0 || out != nullptr, "outputs required for backward step 0");
  return sp::run_backward_step(c, step, out);
}

int fsc_sparse_feature_buffer(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                              int which, int layer, float** out) {
  FSC_REQUIRE(out && workspace, "workspace and output pointer required");
  FSC_TRY(sp::validate(cfg));
  FSC_REQUIRE(which == 0 || which == 1, "which must be 0 (features) or 1 (gradients)");
  FSC_REQUIRE(layer >= 0 && layer < cfg->num_interaction, "layer out of range");
  sp::Plan p{};
  Arena ar(workspace, (size_t)-1);
  sp::layout(p, ar, cfg, num_atoms, num_edges);
  *out = which == 0 ? p.feats[layer] : p.grads[layer];
  return FSC_OK;
}

int fsc_sparse_status(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace, void* stream,
                      int* status_host) {
  FSC_REQUIRE(status_host && workspace, "status output and workspace required");
  FSC_TRY(sp::validate(cfg));
  sp::Plan p{};
  Arena ar(workspace, (size_t)-1);
  sp::layout(p, ar, cfg, num_atoms, num_edges);
  cudaStream_t st = as_stream(stream);
  if (cudaMemcpyAsync(status_host, p.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "status readback");
  return FSC_OK;
}

}  // extern "C"
