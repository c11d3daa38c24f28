// Neighbour list with the semantics of radius_graph_pbc_gpu (utils/graph_utils.py:192-258).
//
// Edge (src=i, dst=j, S): |(pos[j] + S@cell) - pos[i]| < cutoff, S in {-1,0,1}^3 on periodic axes,
// no i == j at S == 0.  Float64 arithmetic in a fixed order without FMA contraction
// (shift_c = (S0*c0c + S1*c1c) + S2*c2c; d_c = (pos[j,c] + shift_c) - pos[i,c];
//  r2 = (dx*dx + dy*dy) + dz*dz; edge iff r2 < cutoff*cutoff), so the edge set is bit-exact
// with the CPU oracle.  Output: CSR by dst with rows sorted by (src, sidx),
// sidx = (S0+1)*9 + (S1+1)*3 + (S2+1).
//
// Two searches, identical results:
//  * all pairs within a frame (any cell shape, any pbc), one thread per dst atom, candidates
//    visited in (src, sidx) order so rows come out sorted;
//  * cell list for a frame whose periodic cell vectors are axis-aligned, with positions in
//    [0, L) along periodic axes and anywhere along open axes (the grid spans the atoms'
//    bounding box there): cells of side >= cutoff + 1e-6, the 27 neighbour cells of the dst
//    atom's cell are visited, periodic axes with their wrap count q (S = -q), open axes only
//    inside the grid (S = 0); every (src, S) candidate is met exactly once for any cell count
//    per axis >= 1; rows are sorted afterwards (warp-per-row rank sort).  Mixed periodicity is
//    what a spatial-decomposition rank has: open along the split axes (explicit ghost images),
//    periodic along the others.
#include <cub/cub.cuh>

#include <algorithm>
#include <mutex>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace fsc {

namespace {

struct FrameDev {
  const int64_t* frame_ptr;  // [F+1]
  const double* cell;        // [F][9]
  int64_t F;
};

__device__ __forceinline__ int find_frame(const int64_t* fp, int64_t F, int64_t a) {
  int64_t lo = 0, hi = F;  // fp[lo] <= a < fp[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (fp[mid] <= a) lo = mid;
    else hi = mid;
  }
  return (int)lo;
}

__device__ __forceinline__ bool within(const double* pj, const double* pi, const double* sv, double r2max) {
  const double dx = __dadd_rn(__dadd_rn(pj[0], sv[0]), -pi[0]);
  const double dy = __dadd_rn(__dadd_rn(pj[1], sv[1]), -pi[1]);
  const double dz = __dadd_rn(__dadd_rn(pj[2], sv[2]), -pi[2]);
  const double r2 = __dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz));
  return r2 < r2max;
}

__device__ __forceinline__ void shift_vec(const double* c, int s0, int s1, int s2, double* sv) {
#pragma unroll
  for (int k = 0; k < 3; ++k)
    sv[k] = __dadd_rn(__dadd_rn(__dmul_rn((double)s0, c[k]), __dmul_rn((double)s1, c[3 + k])),
                      __dmul_rn((double)s2, c[6 + k]));
}

// mode 0: count into counts[j]; mode 1: write src/sidx at row_ptr[j]...
__global__ void brute_kernel(const double* __restrict__ pos, FrameDev fr, int64_t j0, int64_t j1, int p0, int p1,
                             int p2, double r2max, int mode, int32_t* __restrict__ counts,
                             const int32_t* __restrict__ row_ptr, int32_t* __restrict__ src,
                             int8_t* __restrict__ sidx) {
  const int64_t j = j0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= j1) return;
  const int f = find_frame(fr.frame_ptr, fr.F, j);
  const int64_t a0 = fr.frame_ptr[f], a1 = fr.frame_ptr[f + 1];
  const double* c = fr.cell + 9 * f;
  const double pj[3] = {pos[3 * j], pos[3 * j + 1], pos[3 * j + 2]};
  int32_t n = 0;
  int64_t out = mode ? row_ptr[j] : 0;
  for (int64_t i = a0; i < a1; ++i) {
    const double pi[3] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
    for (int s0 = -p0; s0 <= p0; ++s0)
      for (int s1 = -p1; s1 <= p1; ++s1)
        for (int s2 = -p2; s2 <= p2; ++s2) {
          if (i == j && s0 == 0 && s1 == 0 && s2 == 0) continue;
          double sv[3];
          shift_vec(c, s0, s1, s2, sv);
          if (within(pj, pi, sv, r2max)) {
            if (mode) {
              src[out] = (int32_t)i;
              sidx[out] = (int8_t)((s0 + 1) * 9 + (s1 + 1) * 3 + (s2 + 1));
              ++out;
            } else {
              ++n;
            }
          }
        }
  }
  if (!mode) counts[j] = n;
}

struct CellGrid {
  int nc[3];
  int per[3];        // periodic axis
  double lo[3];      // grid origin (0 on periodic axes)
  double inv_cs[3];  // cells per unit length
};

__device__ __forceinline__ int cell_coord(double x, double lo, double inv_cs, int n) {
  int c = (int)floor((x - lo) * inv_cs);
  return c < 0 ? 0 : (c >= n ? n - 1 : c);
}

__global__ void cell_assign_kernel(const double* __restrict__ pos, int64_t a0, int64_t na, CellGrid g,
                                   int32_t* __restrict__ cell_of, int32_t* __restrict__ cell_count) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= na) return;
  const int64_t a = a0 + t;
  const int cx = cell_coord(pos[3 * a], g.lo[0], g.inv_cs[0], g.nc[0]);
  const int cy = cell_coord(pos[3 * a + 1], g.lo[1], g.inv_cs[1], g.nc[1]);
  const int cz = cell_coord(pos[3 * a + 2], g.lo[2], g.inv_cs[2], g.nc[2]);
  const int id = (cx * g.nc[1] + cy) * g.nc[2] + cz;
  cell_of[t] = id;
  atomicAdd(cell_count + id, 1);
}

__global__ void cell_fill_kernel(int64_t a0, int64_t na, const int32_t* __restrict__ cell_of,
                                 const int32_t* __restrict__ cell_start, int32_t* __restrict__ cursor,
                                 int32_t* __restrict__ cell_atoms) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= na) return;
  const int id = cell_of[t];
  const int slot = atomicAdd(cursor + id, 1);
  cell_atoms[cell_start[id] + slot] = (int32_t)(a0 + t);
}

__global__ void cell_search_kernel(const double* __restrict__ pos, int64_t a0, int64_t na, CellGrid g,
                                   const double* __restrict__ cellm, const int32_t* __restrict__ cell_of,
                                   const int32_t* __restrict__ cell_start, const int32_t* __restrict__ cell_atoms,
                                   double r2max, int mode, int32_t* __restrict__ counts,
                                   const int32_t* __restrict__ row_ptr, int32_t* __restrict__ src,
                                   int8_t* __restrict__ sidx) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= na) return;
  const int64_t j = a0 + t;
  const int id = cell_of[t];
  const int cz = id % g.nc[2], cy = (id / g.nc[2]) % g.nc[1], cx = id / (g.nc[2] * g.nc[1]);
  const double pj[3] = {pos[3 * j], pos[3 * j + 1], pos[3 * j + 2]};
  int32_t n = 0;
  int64_t out = mode ? row_ptr[j] : 0;
  for (int dx = -1; dx <= 1; ++dx) {
    const int ux = cx + dx;
    const int qx = ux < 0 ? -1 : (ux >= g.nc[0] ? 1 : 0);
    if (qx != 0 && !g.per[0]) continue;
    const int wx = ux - qx * g.nc[0];
    for (int dy = -1; dy <= 1; ++dy) {
      const int uy = cy + dy;
      const int qy = uy < 0 ? -1 : (uy >= g.nc[1] ? 1 : 0);
      if (qy != 0 && !g.per[1]) continue;
      const int wy = uy - qy * g.nc[1];
      for (int dz = -1; dz <= 1; ++dz) {
        const int uz = cz + dz;
        const int qz = uz < 0 ? -1 : (uz >= g.nc[2] ? 1 : 0);
        if (qz != 0 && !g.per[2]) continue;
        const int wz = uz - qz * g.nc[2];
        const int s0 = -qx, s1 = -qy, s2 = -qz;
        double sv[3];
        shift_vec(cellm, s0, s1, s2, sv);
        const int nid = (wx * g.nc[1] + wy) * g.nc[2] + wz;
        for (int k = cell_start[nid]; k < cell_start[nid + 1]; ++k) {
          const int64_t i = cell_atoms[k];
          if (i == j && s0 == 0 && s1 == 0 && s2 == 0) continue;
          const double pi[3] = {pos[3 * i], pos[3 * i + 1], pos[3 * i + 2]};
          if (within(pj, pi, sv, r2max)) {
            if (mode) {
              src[out] = (int32_t)i;
              sidx[out] = (int8_t)((s0 + 1) * 9 + (s1 + 1) * 3 + (s2 + 1));
              ++out;
            } else {
              ++n;
            }
          }
        }
      }
    }
  }
  if (!mode) counts[j] = n;
}

// Warp per row: sort (key = src*27 + sidx) ascending by rank counting; rows of any length.
__global__ void row_sort_kernel(const int32_t* __restrict__ row_ptr, int64_t N, int32_t* __restrict__ src,
                                int8_t* __restrict__ sidx, int32_t* __restrict__ tmp_src, int8_t* __restrict__ tmp_sidx) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= N) return;
  const int e0 = row_ptr[r], e1 = row_ptr[r + 1];
  for (int e = e0 + lane; e < e1; e += 32) {
    const int64_t key = (int64_t)src[e] * 27 + sidx[e];
    int rank = 0;
    for (int f = e0; f < e1; ++f) {
      const int64_t k2 = (int64_t)src[f] * 27 + sidx[f];
      rank += (k2 < key) ? 1 : 0;
    }
    tmp_src[e0 + rank] = src[e];
    tmp_sidx[e0 + rank] = sidx[e];
  }
  __syncwarp();
  for (int e = e0 + lane; e < e1; e += 32) {
    src[e] = tmp_src[e];
    sidx[e] = tmp_sidx[e];
  }
}

// Order-preserving int64 key of a double (for atomicMin / atomicMax).
__device__ __forceinline__ long long dkey(double x) {
  const long long b = __double_as_longlong(x);
  return b >= 0 ? b : (b ^ 0x7FFFFFFFFFFFFFFFLL);
}
__host__ __device__ inline double dkey_inv(long long k) {
  const long long b = k >= 0 ? k : (k ^ 0x7FFFFFFFFFFFFFFFLL);
  double x;
  memcpy(&x, &b, sizeof(x));
  return x;
}

// flag |= 1 if a position is outside [0, L) on a periodic axis or not finite; mm[2k] / mm[2k+1]
// = min / max keys of coordinate k.
__global__ void box_kernel(const double* __restrict__ pos, int64_t a0, int64_t na, int p0, int p1, int p2, double L0,
                           double L1, double L2, int32_t* __restrict__ flag, long long* __restrict__ mm) {
  __shared__ long long smin[3][8], smax[3][8];
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per[3] = {p0, p1, p2};
  const double L[3] = {L0, L1, L2};
  long long kmin[3], kmax[3];
  bool bad = false;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    kmin[k] = 0x7FFFFFFFFFFFFFFFLL;
    kmax[k] = -0x7FFFFFFFFFFFFFFFLL - 1;
  }
  if (t < na) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const double x = pos[3 * (a0 + t) + k];
      if (!isfinite(x) || (per[k] && !(x >= 0.0 && x < L[k]))) bad = true;
      kmin[k] = kmax[k] = dkey(x);
    }
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    for (int o = 16; o > 0; o >>= 1) {
      kmin[k] = min(kmin[k], __shfl_xor_sync(0xffffffffu, kmin[k], o));
      kmax[k] = max(kmax[k], __shfl_xor_sync(0xffffffffu, kmax[k], o));
    }
    if (lane == 0) {
      smin[k][warp] = kmin[k];
      smax[k][warp] = kmax[k];
    }
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    const int k = threadIdx.x;
    long long a = smin[k][0], b = smax[k][0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      a = min(a, smin[k][w]);
      b = max(b, smax[k][w]);
    }
    atomicMin(mm + 2 * k, a);
    atomicMax(mm + 2 * k + 1, b);
  }
}

// transpose CSR
__global__ void tr_count_kernel(const int32_t* __restrict__ src, int64_t E, int32_t* __restrict__ cnt) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e < E) atomicAdd(cnt + src[e], 1);
}
__global__ void tr_fill_kernel(const int32_t* __restrict__ src, int64_t E, const int32_t* __restrict__ tr_ptr,
                               int32_t* __restrict__ cursor, int32_t* __restrict__ tr_eid) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const int s = src[e];
  tr_eid[tr_ptr[s] + atomicAdd(cursor + s, 1)] = (int32_t)e;
}
__global__ void tr_sort_kernel(const int32_t* __restrict__ tr_ptr, int64_t N, int32_t* __restrict__ tr_eid,
                               int32_t* __restrict__ tmp) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= N) return;
  const int e0 = tr_ptr[r], e1 = tr_ptr[r + 1];
  for (int e = e0 + lane; e < e1; e += 32) {
    const int key = tr_eid[e];
    int rank = 0;
    for (int f = e0; f < e1; ++f) rank += (tr_eid[f] < key) ? 1 : 0;
    tmp[e0 + rank] = key;
  }
  __syncwarp();
  for (int e = e0 + lane; e < e1; e += 32) tr_eid[e] = tmp[e];
}

// Per-source neighbour cap (max_num_neighbors of radius_graph_pbc_gpu, utils/graph_utils.py:192,
// 240): the reference runs one torch_cluster radius search per image shift S, and that search
// keeps, for every source i, the first `cap` candidates j in ascending index order with
// |pos[j] + S@cell - pos[i]| < cutoff; the self pair (j == i at S == 0) takes a slot before it is
// removed.  One thread per source walks its out-edges in the transpose CSR (ascending edge id =
// ascending dst, then shift) with one counter per shift.
__device__ __forceinline__ int64_t row_of(const int32_t* __restrict__ row_ptr, int64_t N, int64_t e) {
  int64_t lo = 0, hi = N;  // row_ptr[lo] <= e < row_ptr[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (row_ptr[mid] <= e) lo = mid;
    else hi = mid;
  }
  return lo;
}
__global__ void cap_mark_kernel(const int32_t* __restrict__ row_ptr, int64_t N, const int8_t* __restrict__ sidx,
                                const int32_t* __restrict__ tr_ptr, const int32_t* __restrict__ tr_eid, int cap,
                                uint8_t* __restrict__ keep) {
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= N) return;
  int cnt[27];
#pragma unroll
  for (int k = 0; k < 27; ++k) cnt[k] = 0;
  bool self_counted = false;
  for (int t = tr_ptr[s]; t < tr_ptr[s + 1]; ++t) {
    const int e = tr_eid[t];
    const int k = min(max((int)sidx[e], 0), 26);
    if (k == 13 && !self_counted && row_of(row_ptr, N, e) > s) {  // past j == i in the S == 0 search
      ++cnt[13];
      self_counted = true;
    }
    keep[e] = cnt[k] < cap ? 1 : 0;
    ++cnt[k];
  }
}
__global__ void cap_count_kernel(const int32_t* __restrict__ row_ptr, int64_t N, const uint8_t* __restrict__ keep,
                                 int32_t* __restrict__ counts) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r > N) return;
  int n = 0;
  if (r < N)
    for (int e = row_ptr[r]; e < row_ptr[r + 1]; ++e) n += keep[e];
  counts[r] = n;
}
__global__ void cap_fill_kernel(const int32_t* __restrict__ row_ptr, int64_t N, const uint8_t* __restrict__ keep,
                                const int32_t* __restrict__ src, const int8_t* __restrict__ sidx,
                                const int32_t* __restrict__ out_ptr, int32_t* __restrict__ out_src,
                                int8_t* __restrict__ out_sidx) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= N) return;
  int o = out_ptr[r];
  for (int e = row_ptr[r]; e < row_ptr[r + 1]; ++e)
    if (keep[e]) {
      out_src[o] = src[e];
      out_sidx[o] = sidx[e];
      ++o;
    }
}

size_t scan_temp_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, bytes, (int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  return bytes;
}

struct NbrWs {
  int32_t* counts;      // [N+1]
  int32_t* cell_of;     // [N]
  int32_t* cell_count;  // [N+2]
  int32_t* cell_start;  // [N+2]
  int32_t* cursor;      // [N+2]
  int32_t* cell_atoms;  // [N]
  int64_t* frame_ptr;   // [F+1] (F <= N+1)
  double* cell;         // [F][9]
  int32_t* flag;        // [4]
  long long* mm;        // [6] coordinate min / max keys
  void* scan_tmp;
  size_t scan_bytes;
};

void nbr_layout(NbrWs& w, Arena& ar, int64_t N, int64_t F) {
  w.counts = ar.take<int32_t>(N + 1);
  w.cell_of = ar.take<int32_t>(N + 1);
  w.cell_count = ar.take<int32_t>(N + 2);
  w.cell_start = ar.take<int32_t>(N + 2);
  w.cursor = ar.take<int32_t>(N + 2);
  w.cell_atoms = ar.take<int32_t>(N + 1);
  w.frame_ptr = ar.take<int64_t>(F + 1);
  w.cell = ar.take<double>(9 * F + 9);
  w.flag = ar.take<int32_t>(4);
  w.mm = ar.take<long long>(6);
  w.scan_bytes = scan_temp_bytes(N + 2);
  w.scan_tmp = ar.take<char>((int64_t)w.scan_bytes + 16);
}

// Periodic cell vectors axis-aligned (the rows of open axes are not used).
bool aligned_periodic(const double* c, const int32_t* pbc) {
  for (int k = 0; k < 3; ++k) {
    if (!pbc[k]) continue;
    if (!(c[4 * k] > 0.0)) return false;
    for (int j = 0; j < 3; ++j)
      if (j != k && c[3 * k + j] != 0.0) return false;
  }
  return true;
}

// lo / hi: grid extent per axis ([0, L) on periodic axes, the bounding box on open ones).
CellGrid make_grid(const int32_t* pbc, const double* lo, const double* hi, double cutoff, int64_t natoms) {
  CellGrid g{};
  int64_t nc[3];
  double L[3];
  for (int k = 0; k < 3; ++k) {
    L[k] = hi[k] - lo[k];
    nc[k] = L[k] > 0.0 ? std::max<int64_t>(1, (int64_t)std::floor(L[k] / (cutoff + 1e-6))) : 1;
  }
  const int64_t cap = std::max<int64_t>(1, natoms);
  while (nc[0] * nc[1] * nc[2] > cap) {
    int k = 0;
    if (nc[1] > nc[k]) k = 1;
    if (nc[2] > nc[k]) k = 2;
    nc[k] -= 1;
  }
  for (int k = 0; k < 3; ++k) {
    g.nc[k] = (int)nc[k];
    g.per[k] = pbc[k] ? 1 : 0;
    g.lo[k] = lo[k];
    g.inv_cs[k] = L[k] > 0.0 ? (double)nc[k] / L[k] : 0.0;
  }
  return g;
}

// Run the search (mode 0 count / 1 fill) over all frames.
int search(const double* pos, const double* cell_host, const int64_t* fp_host, int64_t F, int64_t N,
           const int32_t* pbc, double cutoff, int mode, int32_t* counts, const int32_t* row_ptr, int32_t* src,
           int8_t* sidx, NbrWs& w, cudaStream_t st) {
  const double r2max = cutoff * cutoff;
  std::vector<int64_t> brute_frames;
  for (int64_t f = 0; f < F; ++f) {
    const int64_t a0 = fp_host[f], na = fp_host[f + 1] - fp_host[f];
    const double* c = cell_host + 9 * f;
    bool use_cells = aligned_periodic(c, pbc) && na > 512;
    double lo[3] = {0.0, 0.0, 0.0}, hi[3] = {c[0], c[4], c[8]};
    if (use_cells) {
      const long long init[6] = {0x7FFFFFFFFFFFFFFFLL, -0x7FFFFFFFFFFFFFFFLL - 1, 0x7FFFFFFFFFFFFFFFLL,
                                 -0x7FFFFFFFFFFFFFFFLL - 1, 0x7FFFFFFFFFFFFFFFLL, -0x7FFFFFFFFFFFFFFFLL - 1};
      if (cudaMemsetAsync(w.flag, 0, sizeof(int32_t), st) != cudaSuccess ||
          cudaMemcpyAsync(w.mm, init, sizeof(init), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail(FSC_ERR_CUDA, "box check setup");
      box_kernel<<<(unsigned)ceil_div(na, 256), 256, 0, st>>>(pos, a0, na, pbc[0], pbc[1], pbc[2], c[0], c[4], c[8],
                                                              w.flag, w.mm);
      int32_t flag = 0;
      long long mm[6];
      if (cudaMemcpyAsync(&flag, w.flag, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
          cudaMemcpyAsync(mm, w.mm, sizeof(mm), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
          cudaStreamSynchronize(st) != cudaSuccess)
        return fail(FSC_ERR_CUDA, "neighbour box check");
      use_cells = (flag == 0);
      for (int k = 0; k < 3; ++k)
        if (!pbc[k]) {
          lo[k] = dkey_inv(mm[2 * k]);
          hi[k] = dkey_inv(mm[2 * k + 1]);
        }
    }
    if (!use_cells) {
      brute_frames.push_back(f);
      continue;
    }
    CellGrid g = make_grid(pbc, lo, hi, cutoff, na);
    const int64_t ncell = (int64_t)g.nc[0] * g.nc[1] * g.nc[2];
    if (cudaMemsetAsync(w.cell_count, 0, sizeof(int32_t) * (ncell + 1), st) != cudaSuccess ||
        cudaMemsetAsync(w.cursor, 0, sizeof(int32_t) * (ncell + 1), st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset cells");
    const unsigned blocks = (unsigned)ceil_div(na, 256);
    cell_assign_kernel<<<blocks, 256, 0, st>>>(pos, a0, na, g, w.cell_of, w.cell_count);
    size_t sb = w.scan_bytes;
    if (cub::DeviceScan::ExclusiveSum(w.scan_tmp, sb, w.cell_count, w.cell_start, (int)(ncell + 1), st) !=
        cudaSuccess)
      return fail(FSC_ERR_CUDA, "cell scan");
    cell_fill_kernel<<<blocks, 256, 0, st>>>(a0, na, w.cell_of, w.cell_start, w.cursor, w.cell_atoms);
    cell_search_kernel<<<blocks, 256, 0, st>>>(pos, a0, na, g, w.cell + 9 * f, w.cell_of, w.cell_start, w.cell_atoms,
                                               r2max, mode, counts, row_ptr, src, sidx);
    FSC_TRY(check_launch("cell_search_kernel"));
  }
  if (!brute_frames.empty()) {
    // one launch over all atoms of the brute-force frames (contiguous runs are launched together)
    size_t k = 0;
    while (k < brute_frames.size()) {
      size_t k2 = k + 1;
      while (k2 < brute_frames.size() && brute_frames[k2] == brute_frames[k2 - 1] + 1) ++k2;
      const int64_t f0 = brute_frames[k], f1 = brute_frames[k2 - 1] + 1;
      const int64_t a0 = fp_host[f0], a1 = fp_host[f1];
      FrameDev fr{w.frame_ptr, w.cell, F};
      const int64_t na = a1 - a0;
      if (na > 0) {
        brute_kernel<<<(unsigned)ceil_div(na, 128), 128, 0, st>>>(pos, fr, a0, a1, pbc[0], pbc[1], pbc[2], r2max,
                                                                  mode, counts, row_ptr, src, sidx);
        FSC_TRY(check_launch("brute_kernel"));
      }
      k = k2;
    }
  }
  return FSC_OK;
}

}  // namespace
}  // namespace fsc

using namespace fsc;

extern "C" {

size_t fsc_neighbor_workspace_bytes(int64_t num_atoms, int64_t num_edges) {
  NbrWs w{};
  Arena ar(nullptr, 0);
  nbr_layout(w, ar, num_atoms, num_atoms + 1);
  ar.take<int32_t>(num_edges);
  ar.take<int8_t>(num_edges);
  return ar.off;
}

static int nbr_prepare(const double* cell, const int64_t* frame_ptr_host, int64_t F, int64_t N, const int32_t* pbc,
                       NbrWs& w, void* workspace, size_t bytes, std::vector<double>& cell_host, cudaStream_t st) {
  FSC_REQUIRE(F >= 1 && N >= 0, "bad frame/atom counts");
  FSC_REQUIRE(frame_ptr_host && frame_ptr_host[0] == 0 && frame_ptr_host[F] == N, "frame_ptr must span [0, N]");
  for (int64_t f = 0; f < F; ++f) FSC_REQUIRE(frame_ptr_host[f + 1] >= frame_ptr_host[f], "frame_ptr not monotone");
  FSC_REQUIRE(F <= N + 1, "more frames than atoms");
  FSC_REQUIRE(N < (int64_t)1 << 26, "neighbour builder supports < 2^26 atoms");
  FSC_REQUIRE(pbc != nullptr, "pbc flags required");
  Arena ar(workspace, bytes);
  nbr_layout(w, ar, N, F);
  if (!ar.ok()) return fail(FSC_ERR_CAPACITY, "neighbour workspace too small");
  cell_host.resize(9 * F);
  if (cudaMemcpyAsync(cell_host.data(), cell, sizeof(double) * 9 * F, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(w.cell, cell, sizeof(double) * 9 * F, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(w.frame_ptr, frame_ptr_host, sizeof(int64_t) * (F + 1), cudaMemcpyHostToDevice, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "neighbour setup copies");
  return FSC_OK;
}

int fsc_neighbor_count(const double* pos, const double* cell, const int64_t* frame_ptr_host, int64_t num_frames,
                       int64_t num_atoms, const int32_t* pbc_host, double cutoff, int32_t* row_ptr,
                       int64_t* num_edges_host, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(num_edges_host && row_ptr, "row_ptr / num_edges output required");
  FSC_REQUIRE(cutoff > 0.0, "cutoff must be positive");
  cudaStream_t st = as_stream(stream);
  NbrWs w{};
  std::vector<double> cell_host;
  FSC_TRY(nbr_prepare(cell, frame_ptr_host, num_frames, num_atoms, pbc_host, w, workspace, workspace_bytes, cell_host,
                      st));
  const int64_t N = num_atoms;
  if (cudaMemsetAsync(w.counts, 0, sizeof(int32_t) * (N + 1), st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset");
  FSC_TRY(search(pos, cell_host.data(), frame_ptr_host, num_frames, N, pbc_host, cutoff, 0, w.counts, nullptr,
                 nullptr, nullptr, w, st));
  size_t sb = w.scan_bytes;
  if (cub::DeviceScan::ExclusiveSum(w.scan_tmp, sb, w.counts, row_ptr, (int)(N + 1), st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "edge scan");
  int32_t total = 0;
  if (cudaMemcpyAsync(&total, row_ptr + N, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "edge count readback");
  *num_edges_host = total;
  return FSC_OK;
}

int fsc_neighbor_fill(const double* pos, const double* cell, const int64_t* frame_ptr_host, int64_t num_frames,
                      int64_t num_atoms, const int32_t* pbc_host, double cutoff, const int32_t* row_ptr, int32_t* src,
                      int8_t* sidx, int64_t capacity, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(src && sidx && row_ptr, "outputs required");
  cudaStream_t st = as_stream(stream);
  NbrWs w{};
  std::vector<double> cell_host;
  FSC_TRY(nbr_prepare(cell, frame_ptr_host, num_frames, num_atoms, pbc_host, w, workspace, workspace_bytes, cell_host,
                      st));
  const int64_t N = num_atoms;
  int32_t total = 0;
  if (cudaMemcpyAsync(&total, row_ptr + N, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "edge count readback");
  if (total > capacity) return fail(FSC_ERR_CAPACITY, "edge capacity " + std::to_string(capacity) + " < " +
                                                          std::to_string(total));
  FSC_TRY(search(pos, cell_host.data(), frame_ptr_host, num_frames, N, pbc_host, cutoff, 1, nullptr, row_ptr, src,
                 sidx, w, st));
  // rows from the cell-list search are unordered: sort every row (sorted rows stay as they are)
  if (total > 0 && N > 0) {
    Arena ar2(workspace, workspace_bytes);
    NbrWs dummy{};
    nbr_layout(dummy, ar2, N, num_frames);
    int32_t* tmp_src = ar2.take<int32_t>(total);
    int8_t* tmp_sidx = ar2.take<int8_t>(total);
    if (!ar2.ok() || !tmp_src)
      return fail(FSC_ERR_CAPACITY, "neighbour workspace too small for the fill phase; size it with "
                                    "fsc_neighbor_workspace_bytes(num_atoms, num_edges)");
    row_sort_kernel<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(row_ptr, N, src, sidx, tmp_src, tmp_sidx);
    FSC_TRY(check_launch("row_sort_kernel"));
  }
  return FSC_OK;
}

int fsc_csr_transpose(const int32_t* row_ptr, const int32_t* src, int64_t num_atoms, int64_t num_edges,
                      int32_t* tr_ptr, int32_t* tr_eid, void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = as_stream(stream);
  const int64_t N = num_atoms, E = num_edges;
  FSC_REQUIRE(tr_ptr && row_ptr && (E == 0 || (tr_eid && src)), "null pointer");
  Arena ar(workspace, workspace_bytes);
  int32_t* cnt = ar.take<int32_t>(N + 1);
  int32_t* cursor = ar.take<int32_t>(N + 1);
  int32_t* tmp = ar.take<int32_t>(E + 1);
  const size_t sbytes = scan_temp_bytes(N + 1);
  void* stmp = ar.take<char>((int64_t)sbytes + 16);
  if (!ar.ok() || (workspace == nullptr)) return fail(FSC_ERR_CAPACITY, "transpose workspace too small");
  if (cudaMemsetAsync(cnt, 0, sizeof(int32_t) * (N + 1), st) != cudaSuccess ||
      cudaMemsetAsync(cursor, 0, sizeof(int32_t) * (N + 1), st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "memset");
  if (E > 0) tr_count_kernel<<<(unsigned)ceil_div(E, 256), 256, 0, st>>>(src, E, cnt);
  size_t sb = sbytes;
  if (cub::DeviceScan::ExclusiveSum(stmp, sb, cnt, tr_ptr, (int)(N + 1), st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "transpose scan");
  if (E > 0) {
    tr_fill_kernel<<<(unsigned)ceil_div(E, 256), 256, 0, st>>>(src, E, tr_ptr, cursor, tr_eid);
    tr_sort_kernel<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(tr_ptr, N, tr_eid, tmp);
  }
  return check_launch("csr_transpose");
}

// ---- allocation-free transpose ----------------------------------------------------------
// For callers that cannot allocate device memory (a host program bound to its own fixed
// memory pool, an FFI binding with no allocator): the scratch lives
// in a file-scope __device__ array that every GPU loading this library keeps until exit.
namespace {
constexpr int64_t kStaticMaxAtoms = 262144;       // rows of the CSR
constexpr int64_t kStaticMaxEdges = 4194304;      // edges
constexpr size_t kStaticScanBytes = (1u << 20) + 4096;  // scan temporaries + arena rounding
constexpr size_t kStaticScratchBytes = sizeof(int32_t) * (2 * (kStaticMaxAtoms + 1) + kStaticMaxEdges + 64) +
                                       kStaticScanBytes;
__device__ __align__(256) unsigned char g_transpose_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};

// Device address of g_transpose_scratch on the current device (looked up once per device).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(FSC_ERR_CUDA, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_transpose_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FSC_ERR_CUDA, std::string("cudaGetSymbolAddress(g_transpose_scratch): ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FSC_OK;
}
}  // namespace

int fsc_csr_transpose_static(const int32_t* row_ptr, const int32_t* src, int64_t num_atoms, int64_t num_edges,
                             int32_t* tr_ptr, int32_t* tr_eid, void* stream) {
  FSC_REQUIRE(num_atoms >= 0 && num_edges >= 0, "negative size");
  if (num_atoms > kStaticMaxAtoms || num_edges > kStaticMaxEdges)
    return fail(FSC_ERR_CAPACITY, "fsc_csr_transpose_static handles at most " + std::to_string(kStaticMaxAtoms) +
                                      " atoms and " + std::to_string(kStaticMaxEdges) + " edges (got " +
                                      std::to_string(num_atoms) + ", " + std::to_string(num_edges) +
                                      "); use fsc_csr_transpose with a caller workspace");
  // the same arithmetic (per-block rounding included) that fsc_csr_transpose's arena applies
  const size_t need = fsc_csr_transpose_workspace_bytes(num_atoms, num_edges);
  if (need > kStaticScratchBytes)
    return fail(FSC_ERR_CAPACITY, "fsc_csr_transpose_static: " + std::to_string(num_atoms) + " atoms and " +
                                      std::to_string(num_edges) + " edges need " + std::to_string(need) +
                                      " scratch bytes, more than the static " + std::to_string(kStaticScratchBytes) +
                                      " (at most " + std::to_string(kStaticMaxAtoms) + " atoms and " +
                                      std::to_string(kStaticMaxEdges) + " edges); use fsc_csr_transpose");
  void* scratch = nullptr;
  FSC_TRY(static_scratch(&scratch));
  // Same kernels and layout as fsc_csr_transpose; the counters are cleared on every call.
  return fsc_csr_transpose(row_ptr, src, num_atoms, num_edges, tr_ptr, tr_eid, scratch, kStaticScratchBytes,
                           stream);
}

size_t fsc_csr_transpose_workspace_bytes(int64_t num_atoms, int64_t num_edges) {
  Arena ar(nullptr, 0);
  ar.take<int32_t>(num_atoms + 1);
  ar.take<int32_t>(num_atoms + 1);
  ar.take<int32_t>(num_edges + 1);
  ar.take<char>((int64_t)scan_temp_bytes(num_atoms + 1) + 16);
  return ar.off;
}

size_t fsc_neighbor_cap_workspace_bytes(int64_t num_atoms, int64_t num_edges) {
  Arena ar(nullptr, 0);
  ar.take<uint8_t>(num_edges + 1);
  ar.take<int32_t>(num_atoms + 1);
  ar.take<char>((int64_t)scan_temp_bytes(num_atoms + 1) + 16);
  return ar.off;
}

int fsc_neighbor_cap(const int32_t* row_ptr, const int32_t* src, const int8_t* sidx, int64_t num_atoms,
                     int64_t num_edges, const int32_t* tr_ptr, const int32_t* tr_eid, int max_num_neighbors,
                     int32_t* out_row_ptr, int32_t* out_src, int8_t* out_sidx, int64_t* out_num_edges_host,
                     void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(row_ptr && out_row_ptr && out_num_edges_host, "null pointer");
  FSC_REQUIRE(num_atoms >= 0 && num_edges >= 0, "negative size");
  FSC_REQUIRE(num_edges == 0 || (src && sidx && tr_ptr && tr_eid && out_src && out_sidx), "null edge arrays");
  FSC_REQUIRE(max_num_neighbors >= 1, "max_num_neighbors must be >= 1");
  FSC_REQUIRE(num_atoms < (int64_t)INT32_MAX && num_edges < (int64_t)INT32_MAX, "graph too large");
  cudaStream_t st = as_stream(stream);
  const int64_t N = num_atoms, E = num_edges;
  Arena ar(workspace, workspace_bytes);
  uint8_t* keep = ar.take<uint8_t>(E + 1);
  int32_t* counts = ar.take<int32_t>(N + 1);
  const size_t sbytes = scan_temp_bytes(N + 1);
  void* stmp = ar.take<char>((int64_t)sbytes + 16);
  if (!ar.ok() || workspace == nullptr)
    return fail(FSC_ERR_CAPACITY, "neighbour cap workspace too small; size it with fsc_neighbor_cap_workspace_bytes");
  if (E > 0 && N > 0) {
    cap_mark_kernel<<<(unsigned)ceil_div(N, 128), 128, 0, st>>>(row_ptr, N, sidx, tr_ptr, tr_eid, max_num_neighbors,
                                                                keep);
    FSC_TRY(check_launch("cap_mark_kernel"));
  }
  cap_count_kernel<<<(unsigned)ceil_div(N + 1, 256), 256, 0, st>>>(row_ptr, N, keep, counts);
  FSC_TRY(check_launch("cap_count_kernel"));
  size_t sb = sbytes;
  if (cub::DeviceScan::ExclusiveSum(stmp, sb, counts, out_row_ptr, (int)(N + 1), st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "neighbour cap scan");
  if (E > 0 && N > 0) {
    cap_fill_kernel<<<(unsigned)ceil_div(N, 256), 256, 0, st>>>(row_ptr, N, keep, src, sidx, out_row_ptr, out_src,
                                                                out_sidx);
    FSC_TRY(check_launch("cap_fill_kernel"));
  }
  int32_t total = 0;
  if (cudaMemcpyAsync(&total, out_row_ptr + N, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "capped edge count readback");
  *out_num_edges_host = total;
  return FSC_OK;
}

}  // extern "C"
