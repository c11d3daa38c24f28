// conv2 backward, gate and harmonic gradients, on the tensor cores.
//
// The quantities of conv2_q_kernel (ictd_conv.cu; reference: the backward of the conv2 tensor
// product, ictd_irreps.py:1003-1133).  Per edge e -> n with sender s and q = (p, m1, kk):
//   Q_e[q]   = sum_c x[s][KB(l1(p)) + m1][c] * dZ[n][zrow(p, kk)][c]      (dZ already carries 1/deg n)
//   dgates[e][p]         = sum_{m1, kk} Q_e[q] * Yt0_e[q],   Yt0_e[q] = sum_m2 cg2[q][m2] Y_e[KB(l2) + m2]
//   dY[e][KB(l2) + m2]  += sum_{m1, kk} Q_e[q] * gate_e[p] * cg2[q][m2]
// For one receiver n, Q of up to 14 of its edges is one matrix product over the channels:
//   D[row][j] = sum_c A[row][c] B[j][c],   A[row] = x[s_e][KB(G) + m1],   B[j] = dZ[n][j]
// with row = (l1 group G, m1, edge) -- 14 G = 0 rows, 42 G = 1 rows, 70 G = 2 rows, 2 unused --
// and j < 35 the dZ rows (48 with zero padding), so M = 128, N = 48, K = C: 3xTF32 (hi*lo and
// lo*hi issued before hi*hi), one chain of 3 C / 8 <= 24 MMAs.  D[row][zrow(p, kk)] is Q for the
// paths of group G; the epilogue (one thread per row) reduces them to per-row gate and harmonic
// partials, and the per-edge sums over the nine rows run in a fixed order (no atomics).
//
// One persistent CTA per SM, warp-specialised, every hand-off an mbarrier:
//  * warp 9, producer: takes receivers from a work counter (in increasing order, which keeps the
//    senders' rows of the receivers in flight close together in L2) and per tile of up to 14
//    edges issues bulk copies of the senders' 9 x C rows (contiguous in x: one copy per edge, into
//    a slot of stride 9 C + 4 floats so that the rows read in one shared-memory phase fall in
//    distinct bank groups) and of the edges' harmonics and gates (two contiguous blocks), through
//    four stages; per receiver, its 35 dZ rows;
//  * warps 0-3, builders (thread = tile row = TMEM lane): per receiver they split dZ into a K-major
//    tf32 hi / lo image (one of two, written in a diagonal (row, K-quad) order, free of bank
//    conflicts on both sides); per tile they split the sender rows into one of two TMEM A buffers
//    and copy the tile's edge data into the matching tile record;
//  * warp 8, MMA issuer: one chain per tile into one of two TMEM D buffers;
//  * warps 4-7, epilogue: read D, release it, reduce.
// So the operand build of tile t + 1 and the epilogue of tile t - 1 run under the MMAs of tile t.
// Every wait is bounded (status 61-69).
#include <algorithm>

#include "common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {

using namespace ictd2;

namespace {

constexpr int QT_EDGES = 14;      // edges per tile
constexpr int QT_ROWS = 126;      // 9 rows per edge
constexpr int QT_M = 128;
constexpr int QT_N = 48;          // 35 dZ rows + zero padding (N % 16 == 0)
constexpr int QT_GROUP = 256;     // builders (warps 0-7) and epilogue (warps 8-15): two threads per row
constexpr int QT_THREADS = 576;   // + the MMA issuer (warp 16) and the producer (warp 17)
constexpr int QT_STAGES = 4;
constexpr int QT_RED = 13;        // per row: 4 gate partials, 9 harmonic partials
constexpr int QT_OUT = 21;        // per edge: 11 gate gradients, the zero pad, 9 harmonic gradients
constexpr int QT_EREC = 36;      // per edge in a tile record: Y (12), gates (12), dY before this kernel (12)
constexpr int QT_REC = 4 + QT_EDGES * QT_EREC;  // tile record: eb, nk, B image, end flag; edge data
constexpr int QT_BATCH = 8;       // receivers per work-counter take
constexpr int QT_BSRC = 1024;     // senders of a batch held in shared memory (more: loaded per tile)
static_assert(QT_EDGES * QT_OUT <= 2 * QT_GROUP, "two output items per epilogue thread");

template <int C>
struct QtcSmem {
  static constexpr int ES = NK * C + 4;                                      // floats per staging slot
  static constexpr uint32_t XSTAGE = 4u * QT_EDGES * ES;
  static constexpr uint32_t ESTAGE = 4u * QT_EDGES * 12;
  static constexpr uint32_t BIMG = 4u * QT_N * C;                            // one B image (hi or lo)
  static constexpr uint32_t XS = 0;                                           // [4][14][ES] sender rows
  static constexpr uint32_t EY = XS + QT_STAGES * XSTAGE;                     // [4][14][12] harmonics
  static constexpr uint32_t EG = EY + QT_STAGES * ESTAGE;                     // [4][14][12] gates
  static constexpr uint32_t ED = EG + QT_STAGES * ESTAGE;                     // [4][14][12] dY
  static constexpr uint32_t ZS = ED + QT_STAGES * ESTAGE;                     // [2][35][C] dZ rows
  static constexpr uint32_t B0 = (ZS + 2u * 4u * NZ * C + 127u) / 128u * 128u;  // [2][hi, lo][C/4][48][4]
  static constexpr uint32_t REC = B0 + 4u * BIMG;                             // [2][QT_REC] tile records
  static constexpr uint32_t RED = REC + 2u * 4u * QT_REC;                     // [2 halves][128][13]
  static constexpr uint32_t CG = RED + 2u * 4u * QT_M * QT_RED;               // [115][5]
  static constexpr uint32_t BSRC = CG + (4u * NQ * 5 + 15u) / 16u * 16u;      // [1024] senders of a batch
  static constexpr uint32_t INFO = BSRC + 4u * QT_BSRC;                       // [4] {receiver, eb, nk, first}
  static constexpr uint32_t BAR = INFO + 16u * QT_STAGES;
  // full[4], empty[4], zfull[2], zempty[2], a_full[2], mma_done[2], d_free[2]; TMEM slot
  static constexpr uint32_t TOTAL = BAR + 8u * 19;
};
static_assert(QtcSmem<64>::TOTAL <= 227u * 1024u, "shared memory of one CTA");
static_assert((QtcSmem<64>::ES / 4) % 8 == 1 && (QtcSmem<32>::ES / 4) % 8 == 1, "staging slot stride");
static_assert(QtcSmem<64>::XSTAGE % 16 == 0 && QtcSmem<32>::XSTAGE % 16 == 0, "bulk copy alignment");
static_assert(QtcSmem<64>::REC % 16 == 0 && (4 * QT_REC) % 16 == 0 && (4 * QT_EREC) % 16 == 0, "record alignment");
static_assert(QtcSmem<64>::ZS % 16 == 0 && QtcSmem<32>::ZS % 16 == 0 && (4 * NZ * 32) % 16 == 0, "dZ staging");

// Dynamic shared memory requested: at least 116 KB, so that two CTAs never share an SM.
template <int C>
constexpr uint32_t qtc_smem() { return QtcSmem<C>::TOTAL > 116u * 1024u ? QtcSmem<C>::TOTAL : 116u * 1024u; }
// one CTA per SM: it allocates all 512 TMEM columns
static_assert(2u * qtc_smem<32>() > 228u * 1024u && 2u * qtc_smem<64>() > 228u * 1024u, "one CTA per SM");

// Row t of a tile: l1 group G, component m1 within the group, edge k.
__device__ __forceinline__ void qtc_coords(int t, int& G, int& m1, int& k) {
  if (t < QT_EDGES) {
    G = 0; m1 = 0; k = t;
  } else if (t < 4 * QT_EDGES) {
    G = 1; m1 = (t - QT_EDGES) / QT_EDGES; k = (t - QT_EDGES) % QT_EDGES;
  } else {
    G = 2; m1 = (t - 4 * QT_EDGES) / QT_EDGES; k = (t - 4 * QT_EDGES) % QT_EDGES;
  }
}
__device__ __forceinline__ int qtc_row_of(int G, int m1, int k) {
  return G == 0 ? k : (G == 1 ? QT_EDGES + QT_EDGES * m1 + k : 4 * QT_EDGES + QT_EDGES * m1 + k);
}

// The two epilogue threads of a row split its paths: [P_LO(G), P_SPLIT(G)) and [P_SPLIT(G), P_HI(G))
// (about equal multiply counts: the last path of each group is the widest).
__host__ __device__ constexpr int P_SPLIT(int G) { return G == 0 ? 2 : (G == 1 ? 6 : 10); }
__host__ __device__ constexpr int P_HALF(int p) { return p >= P_SPLIT(L1(p)) ? 1 : 0; }

// Gate partials (paths of group G in half H, local index p - P_LO(G)) and harmonic partials of
// one row from its D columns u[zrow(p, kk)].
template <int G, int H>
__device__ __forceinline__ void qtc_row(const uint32_t* u, int m1, const float* Y, const float* g,
                                        const float* __restrict__ cg2, float* dg, float* dy) {
#pragma unroll
  for (int p = H == 0 ? P_LO(G) : P_SPLIT(G); p < (H == 0 ? P_SPLIT(G) : P_HI(G)); ++p)
#pragma unroll
    for (int kk = 0; kk < 2 * L3(p) + 1; ++kk) {
      const int q = QOFF(p) + m1 * (2 * L3(p) + 1) + kk;
      const float Qv = __uint_as_float(u[zrow(p, kk)]);
      float y0 = 0.f;
#pragma unroll
      for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2) y0 = fmaf(cg2[5 * q + m2], Y[KB(L2(p)) + m2], y0);
      dg[p - P_LO(G)] = fmaf(Qv, y0, dg[p - P_LO(G)]);
      const float qg = Qv * g[p];
#pragma unroll
      for (int m2 = 0; m2 < 2 * L2(p) + 1; ++m2)
        dy[KB(L2(p)) + m2] = fmaf(qg, cg2[5 * q + m2], dy[KB(L2(p)) + m2]);
    }
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Named barrier `ID` of one 256-thread group; the _or form returns the OR of `v` over it.
template <int ID>
__device__ __forceinline__ bool group_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(ID)
      : "memory");
  return r != 0;
}
template <int ID>
__device__ __forceinline__ void group_sync() { asm volatile("bar.sync %0, 256;" ::"n"(ID) : "memory"); }

// Wait of a 256-thread group: one thread (`leader`) polls the barrier, the others block at named
// barrier ID without issuing; returns false (for every thread of the group) if the wait failed.
template <int ID>
__device__ __forceinline__ bool group_wait(bool leader, uint64_t* bar, uint32_t parity, int* err, int where) {
  const bool w = !leader || tc::mbar_wait(bar, parity, err, where);
  return !group_sync_or<ID>(!w);
}

// Bounded wait for the completion of phase `parity` on the way out.
__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!tc::mbar_try_wait(bar, parity))
    if (clock64() - t0 > tc::kWaitCycles) break;
}

}  // namespace


template <int C>
__global__ void __launch_bounds__(QT_THREADS, 1)
    conv2_q_tc_kernel(ConvArgs a, const float* __restrict__ x, const float* __restrict__ dZ,
                      float* __restrict__ dgates, float* __restrict__ dY) {
  using L = QtcSmem<C>;
  extern __shared__ __align__(1024) uint8_t smem[];
  float* recs = reinterpret_cast<float*>(smem + L::REC);
  float* red = reinterpret_cast<float*>(smem + L::RED);
  float* cg2 = reinterpret_cast<float*>(smem + L::CG);
  int* bsrc = reinterpret_cast<int*>(smem + L::BSRC);
  int4* info = reinterpret_cast<int4*>(smem + L::INFO);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR);  // [4] stage copies landed
  uint64_t* empty = full + 4;                                   // [4] stage consumed
  uint64_t* zfull = full + 8;                                   // [2] dZ rows landed
  uint64_t* zempty = full + 10;                                 // [2] dZ rows consumed
  uint64_t* a_full = full + 12;                                 // [2] A buffer and tile record written
  uint64_t* mma_done = full + 14;                               // [2] MMA chain into D buffer done
  uint64_t* d_free = full + 16;                                 // [2] D buffer and tile record read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 18);
  auto xs = [&](int s) { return reinterpret_cast<float*>(smem + L::XS + (uint32_t)s * L::XSTAGE); };
  auto ey = [&](int s) { return reinterpret_cast<float*>(smem + L::EY + (uint32_t)s * L::ESTAGE); };
  auto eg = [&](int s) { return reinterpret_cast<float*>(smem + L::EG + (uint32_t)s * L::ESTAGE); };
  auto ed = [&](int s) { return reinterpret_cast<float*>(smem + L::ED + (uint32_t)s * L::ESTAGE); };
  auto zs = [&](int z) { return reinterpret_cast<float*>(smem + L::ZS + (uint32_t)z * 4u * NZ * C); };
  auto bimg = [&](int i) { return reinterpret_cast<float*>(smem + L::B0 + (uint32_t)i * L::BIMG); };  // 2 bsel + lo

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_act = a.n_active < a.N ? a.n_active : a.N;

  // receivers not evaluated in this layer: zero gate gradients (grid-stride over their edges)
  {
    const int64_t z0 = a.row_ptr[n_act], z1 = a.row_ptr[a.N];
    for (int64_t e = z0 + (int64_t)blockIdx.x * QT_THREADS + tid; e < z1; e += (int64_t)gridDim.x * QT_THREADS) {
      float4* d = reinterpret_cast<float4*>(dgates + 12 * e);
      d[0] = d[1] = d[2] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 18; ++i) tc::mbar_init(full + i, 1);
    tc::fence_mbar_init();
  }
  for (int i = tid; i < NQ * 5; i += QT_THREADS) cg2[i] = a.tables[TAB_CG2 + i];
  for (int i = tid; i < 4 * QT_N * C; i += QT_THREADS) bimg(0)[i] = 0.f;  // rows >= 35 stay zero
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 17) {
    // ================================================================ producer
    int s = 0, zb = 0;
    uint32_t pe = 0xFu, pze = 3u;  // parity bits; a fresh barrier's "previous phase" counts as complete
    uint32_t iss = 0u, par = 0u;   // per stage: issued at all, parity of the next phase
    uint32_t ziss = 0u, zpar = 0u;
    bool ok = true;
    while (ok) {
      // a batch of consecutive receivers; their senders into shared memory when they fit
      int64_t n0 = 0;
      if (lane == 0) n0 = (int64_t)atomicAdd(a.work, QT_BATCH);
      n0 = __shfl_sync(0xffffffffu, n0, 0);
      if (n0 >= n_act) {  // end marker in the next stage
        if (lane == 0 && tc::mbar_wait(empty + s, (pe >> s) & 1u, a.err, 65)) {
          info[s] = make_int4(-1, 0, 0, 0);
          tc::mbar_arrive(full + s);
          iss |= 1u << s;
          par ^= 1u << s;
        }
        break;
      }
      const int nb = (int)min((int64_t)QT_BATCH, n_act - n0);
      const int rp = lane <= nb ? a.row_ptr[n0 + lane] : 0;
      const int E0 = __shfl_sync(0xffffffffu, rp, 0), E1 = __shfl_sync(0xffffffffu, rp, nb);
      const bool held = E1 - E0 <= QT_BSRC;
      __syncwarp();  // the previous batch's senders are no longer read
      if (held)
        for (int e = E0 + lane; e < E1; e += 32) bsrc[e - E0] = a.src[e];
      __syncwarp();
      for (int j = 0; j < nb && ok; ++j) {
        const int e0 = __shfl_sync(0xffffffffu, rp, j), e1 = __shfl_sync(0xffffffffu, rp, j + 1);
        if (e1 == e0) continue;
        const int64_t n = n0 + j;
        // its dZ rows into staging buffer zb, once the builders have split what was there
        if (!__shfl_sync(0xffffffffu, lane != 0 || tc::mbar_wait(zempty + zb, (pze >> zb) & 1u, a.err, 64), 0)) {
          ok = false;
          break;
        }
        pze ^= 1u << zb;
        if (lane == 0) {
          fence_proxy_async();
          tc::mbar_arrive_expect_tx(zfull + zb, 4u * NZ * C);
          tc::bulk_g2s(zs(zb), dZ + n * NZ * C, 4u * NZ * C, zfull + zb);
          ziss |= 1u << zb;
          zpar ^= 1u << zb;
        }
        zb ^= 1;
        for (int eb = e0; eb < e1; eb += QT_EDGES) {
          const int nk = min(QT_EDGES, e1 - eb);
          const int src = lane < nk ? (held ? bsrc[eb - E0 + lane] : a.src[eb + lane]) : 0;
          if (!__shfl_sync(0xffffffffu, lane != 0 || tc::mbar_wait(empty + s, (pe >> s) & 1u, a.err, 65), 0)) {
            ok = false;
            break;
          }
          pe ^= 1u << s;
          if (lane == 0) {
            info[s] = make_int4((int)n, eb, nk, eb == e0 ? 1 : 0);
            fence_proxy_async();
            tc::mbar_arrive_expect_tx(full + s, 4u * (uint32_t)nk * (NK * C + 36));
            iss |= 1u << s;
            par ^= 1u << s;
          }
          __syncwarp();
          if (lane < nk) tc::bulk_g2s(xs(s) + lane * L::ES, x + (int64_t)src * NK * C, 4u * NK * C, full + s);
          if (lane == 0) {
            tc::bulk_g2s(ey(s), a.edge_y + 12 * (int64_t)eb, 48u * nk, full + s);
            tc::bulk_g2s(eg(s), a.gates + 12 * (int64_t)eb, 48u * nk, full + s);
            tc::bulk_g2s(ed(s), dY + 12 * (int64_t)eb, 48u * nk, full + s);
          }
          s = (s + 1) & (QT_STAGES - 1);
        }
      }
    }
    if (lane == 0) {  // every copy issued has landed before the CTA exits
      for (int i = 0; i < QT_STAGES; ++i)
        if ((iss >> i) & 1u) drain(full + i, ((par >> i) & 1u) ^ 1u);
      for (int i = 0; i < 2; ++i)
        if ((ziss >> i) & 1u) drain(zfull + i, ((zpar >> i) & 1u) ^ 1u);
    }
  }
  else if (warp < 8) {
    // ================================================================ builders (two threads per row)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int row = tid & (QT_M - 1), half = tid >> 7;
    int G, m1, k;
    qtc_coords(row, G, m1, k);
    int s = 0, bsel = 1, zb = 0;
    uint32_t pf = 0u, pz = 0u;  // parity bits per stage / per dZ buffer
    for (uint32_t t = 0;; ++t) {
      const int b = (int)(t & 1u);
      const uint32_t pb = ((t >> 1) & 1u) ^ 1u;  // parity of tile t - 2's phases on buffer b
      {
        const bool w = group_wait<1>(tid == 0, full + s, (pf >> s) & 1u, a.err, 61);
        pf ^= 1u << s;
        if (!w) break;
      }
      const int4 inf = info[s];
      {  // A buffer b (MMAs of tile t - 2) and tile record b (epilogue of tile t - 2) are free
        const bool w = tid != 0 || (tc::mbar_wait(mma_done + b, pb, a.err, 66) && tc::mbar_wait(d_free + b, pb, a.err, 67));
        if (group_sync_or<1>(!w)) break;
      }
      float* rec = recs + b * QT_REC;
      if (inf.x < 0) {  // no more tiles: tell the MMA issuer and the epilogue
        if (tid == 0) {
          reinterpret_cast<int4*>(rec)[0] = make_int4(0, 0, 0, 1);
          tc::mbar_arrive(a_full + b);
        }
        break;
      }
      const int eb = inf.y, nk = inf.z;
      if (inf.w) {  // first tile of a receiver: its dZ rows -> the other B image (hi / lo)
        const bool w = group_wait<1>(tid == 0, zfull + zb, (pz >> zb) & 1u, a.err, 62);
        pz ^= 1u << zb;
        if (!w) break;
        const float* zsrc = zs(zb);
        bsel ^= 1;
        float* bhi = bimg(2 * bsel);
        float* blo = bimg(2 * bsel + 1);
        for (int f = tid; f < 10 * C; f += QT_GROUP) {  // 40 rows x C/4 K-quads, 8 x 8 diagonal blocks
          const int blk = f >> 6, w8 = f & 63, ph = w8 >> 3, i8 = w8 & 7;
          const int row = 8 * (blk / (C / 32)) + i8, kc = 8 * (blk % (C / 32)) + ((i8 + ph) & 7);
          if (row < NZ) {
            const float4 v = reinterpret_cast<const float4*>(zsrc + row * C)[kc];
            uint4 h, l;
            tc::split_tf32(v.x, h.x, l.x);
            tc::split_tf32(v.y, h.y, l.y);
            tc::split_tf32(v.z, h.z, l.z);
            tc::split_tf32(v.w, h.w, l.w);
            reinterpret_cast<uint4*>(bhi)[kc * QT_N + row] = h;
            reinterpret_cast<uint4*>(blo)[kc * QT_N + row] = l;
          }
        }
        fence_proxy_async();  // the image is read by the tensor cores
        group_sync<1>();
        if (tid == 0) tc::mbar_arrive(zempty + zb);
        zb ^= 1;
      }
      // ---- A rows -> TMEM buffer b (hi in columns [0, C), lo in [C, 2C); this thread's half of
      // the row's columns); edge data -> record b
      {
        const bool valid = row < QT_ROWS && k < nk;
        const float* xr = xs(s) + (valid ? k * L::ES + (KB(G) + m1) * C : 0) + half * (C / 2);
        const uint32_t tA = tbase + 128u * (uint32_t)b + lane_off + (uint32_t)(half * (C / 2));
#pragma unroll
        for (int h = 0; h < C / 32; ++h) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = valid ? reinterpret_cast<const float4*>(xr)[4 * h + i] : make_float4(0.f, 0.f, 0.f, 0.f);
            tc::split_tf32(v.x, hi[4 * i], lo[4 * i]);
            tc::split_tf32(v.y, hi[4 * i + 1], lo[4 * i + 1]);
            tc::split_tf32(v.z, hi[4 * i + 2], lo[4 * i + 2]);
            tc::split_tf32(v.w, hi[4 * i + 3], lo[4 * i + 3]);
          }
          tc::tmem_st16(tA + 16u * h, hi);
          tc::tmem_st16(tA + (uint32_t)C + 16u * h, lo);
        }
        if (tid < 9 * nk) {  // Y, gates, dY of the tile's edges
          const int ke = tid / 9, j = tid % 9, blk = j / 3;
          const float4* src4 = reinterpret_cast<const float4*>(blk == 0 ? ey(s) : (blk == 1 ? eg(s) : ed(s)));
          reinterpret_cast<float4*>(rec + 4)[ke * 9 + j] = src4[ke * 3 + j - 3 * blk];
        }
        if (tid == 0) reinterpret_cast<int4*>(rec)[0] = make_int4(eb, nk, bsel, 0);
        tc::tmem_wait_st();
      }
      tc::tc_fence_before();
      group_sync<1>();  // A and the record written; stage s is read
      if (tid == 0) {
        tc::mbar_arrive(empty + s);
        tc::mbar_arrive(a_full + b);
      }
      s = (s + 1) & (QT_STAGES - 1);
    }
  } else if (warp == 16) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(QT_M, QT_N);
      const uint32_t s_b0 = tc::smem_u32(smem + L::B0);
      int last0 = -1, last1 = -1;  // last tile committed on each D buffer
      for (uint32_t t = 0;; ++t) {
        const int b = (int)(t & 1u);
        const uint32_t pcur = (t >> 1) & 1u;
        if (!tc::mbar_wait(a_full + b, pcur, a.err, 63)) break;
        const int4 hdr = reinterpret_cast<const int4*>(recs + b * QT_REC)[0];
        if (hdr.w) break;
        if (!tc::mbar_wait(d_free + b, pcur ^ 1u, a.err, 67)) break;
        tc::tc_fence_after();
        const uint32_t tA = tbase + 128u * (uint32_t)b, tD = tbase + 256u + 64u * (uint32_t)b;
        const uint32_t s_hi = s_b0 + (uint32_t)(2 * hdr.z) * L::BIMG, s_lo = s_hi + L::BIMG;
#pragma unroll
        for (int j = 0; j < C / 8; ++j) {  // small products first, then hi * hi: one chain
          const uint64_t dh = tc::smem_desc_kmajor(s_hi + 1536u * j, 16u * QT_N, 128);
          const uint64_t dl = tc::smem_desc_kmajor(s_lo + 1536u * j, 16u * QT_N, 128);
          tc::mma_tf32_ts(tD, tA + 8u * j, dl, idesc, j > 0 ? 1u : 0u);
          tc::mma_tf32_ts(tD, tA + (uint32_t)C + 8u * j, dh, idesc, 1u);
        }
#pragma unroll
        for (int j = 0; j < C / 8; ++j) {
          const uint64_t dh = tc::smem_desc_kmajor(s_hi + 1536u * j, 16u * QT_N, 128);
          tc::mma_tf32_ts(tD, tA + 8u * j, dh, idesc, 1u);
        }
        tc::mma_commit(mma_done + b);
        if (b) last1 = (int)t; else last0 = (int)t;
      }
      // the last chain on each buffer has finished before TMEM is released
      if (last0 >= 0) drain(mma_done, ((uint32_t)last0 >> 1) & 1u);
      if (last1 >= 0) drain(mma_done + 1, ((uint32_t)last1 >> 1) & 1u);
    }
  }
  else {
    // ================================================================ epilogue (warps 8-15, two threads per row)
    const int et = tid - QT_GROUP, row = et & (QT_M - 1), half = et >> 7;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    int G, m1, k;
    qtc_coords(row, G, m1, k);
    for (uint32_t t = 0;; ++t) {
      const int b = (int)(t & 1u);
      const uint32_t pcur = (t >> 1) & 1u;
      if (!group_wait<2>(et == 0, a_full + b, pcur, a.err, 68)) break;
      const float* rec = recs + b * QT_REC;
      const int4 hdr = reinterpret_cast<const int4*>(rec)[0];
      if (hdr.w) break;
      const int eb = hdr.x, nk = hdr.y;
      {
        const bool w = group_wait<2>(et == 0, mma_done + b, pcur, a.err, 69);
        tc::tc_fence_after();
        if (!w) break;
      }
      uint32_t u[QT_N];
      tc::tmem_ld32(tbase + 256u + 64u * (uint32_t)b + lane_off, u);
      tc::tmem_ld16(tbase + 256u + 64u * (uint32_t)b + lane_off + 32u, u + 32);
      const bool valid = row < QT_ROWS && k < nk;
      float Y[NK], g[NP];
      {
        const float* ek = rec + 4 + (valid ? k * QT_EREC : 0);
#pragma unroll
        for (int j = 0; j < NK; ++j) Y[j] = ek[j];
#pragma unroll
        for (int j = 0; j < NP; ++j) g[j] = ek[12 + j];
      }
      // dY of this thread's output items (before this kernel): item it = et + 256 r is edge
      // it / 21, output it % 21, a harmonic gradient from output 12 on
      float dy_old[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int it = et + QT_GROUP * r, ke = it / QT_OUT, o = it - ke * QT_OUT;
        dy_old[r] = it < nk * QT_OUT && o > NP ? rec[4 + ke * QT_EREC + 24 + (o - NP - 1)] : 0.f;
      }
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      group_sync<2>();  // D buffer b and record b are read
      if (et == 0) tc::mbar_arrive(d_free + b);
      {  // per-row partials of this thread's half of the row's paths
        float dg[4] = {0.f, 0.f, 0.f, 0.f}, dy[NK];
#pragma unroll
        for (int j = 0; j < NK; ++j) dy[j] = 0.f;
        if (valid) {
          if (half == 0) {
            if (G == 0) qtc_row<0, 0>(u, m1, Y, g, cg2, dg, dy);
            else if (G == 1) qtc_row<1, 0>(u, m1, Y, g, cg2, dg, dy);
            else qtc_row<2, 0>(u, m1, Y, g, cg2, dg, dy);
          } else {
            if (G == 0) qtc_row<0, 1>(u, m1, Y, g, cg2, dg, dy);
            else if (G == 1) qtc_row<1, 1>(u, m1, Y, g, cg2, dg, dy);
            else qtc_row<2, 1>(u, m1, Y, g, cg2, dg, dy);
          }
        }
        float* rr = red + et * QT_RED;
#pragma unroll
        for (int j = 0; j < 4; ++j) rr[j] = dg[j];
#pragma unroll
        for (int j = 0; j < NK; ++j) rr[4 + j] = dy[j];
      }
      group_sync<2>();
      // per-edge sums over the edge's rows and the two halves, in a fixed order
      // (nk * 21 <= 294 < 2 * 256 items)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int it = et + QT_GROUP * r;
        if (it >= nk * QT_OUT) break;
        const int ke = it / QT_OUT, o = it - ke * QT_OUT;
        const int64_t e = eb + ke;
        if (o < NP) {
          const int Gp = L1(o), loc = o - P_LO(Gp);
          const float* rh = red + P_HALF(o) * QT_M * QT_RED + loc;
          float v = 0.f;
          for (int m = 0; m < 2 * Gp + 1; ++m) v += rh[qtc_row_of(Gp, m, ke) * QT_RED];
          dgates[12 * e + o] = v;
        } else if (o == NP) {
          dgates[12 * e + NP] = 0.f;
        } else {
          const int j = o - NP - 1;
          float v = 0.f;
          for (int h = 0; h < 2; ++h) {
            const float* rh = red + h * QT_M * QT_RED + 4 + j;
            v += rh[qtc_row_of(0, 0, ke) * QT_RED];
            for (int m = 0; m < 3; ++m) v += rh[qtc_row_of(1, m, ke) * QT_RED];
            for (int m = 0; m < 5; ++m) v += rh[qtc_row_of(2, m, ke) * QT_RED];
          }
          dY[12 * e + j] = dy_old[r] + v;
        }
      }
      group_sync<2>();  // red is rewritten by the next tile
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

int launch_conv2_q_tc(const ConvArgs& a, const float* x, const float* dZ, float* dgates, float* dY,
                      cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  if (!a.work) return fail(FSC_ERR_ARGUMENT, "conv2_q_tc_kernel needs a work counter");
  if (cudaMemsetAsync(a.work, 0, sizeof(int), st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "conv2_q_tc_kernel: memset work counter");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n_act = std::min<int64_t>(std::max<int64_t>(a.n_active, 0), a.N);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(sms, n_act));
  auto go = [&](auto kernel, uint32_t smem) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "conv2_q_tc_kernel: shared memory attribute");
    kernel<<<grid, QT_THREADS, smem, st>>>(a, x, dZ, dgates, dY);
    return check_launch("conv2_q_tc_kernel");
  };
  if (a.C == 32) return go(conv2_q_tc_kernel<32>, qtc_smem<32>());
  if (a.C == 64) return go(conv2_q_tc_kernel<64>, qtc_smem<64>());
  return fail(FSC_ERR_UNSUPPORTED, "conv2_q_tc_kernel supports channels 32 or 64");
}

}  // namespace fsc
