// Readout Gram contraction on the 5th-generation tensor cores (tcgen05, TMEM, bulk TMA).
//
// Forward   scalars[n, o] = sum_l sum_{c,d} Ws_l[o, c, d] G_l[n, c, d],  G_l[n] = t_l t_l^T (over m)
// Backward  dt_l[n, c, m] = 2 sum_d H_l[n, c, d] t_l[n, d, m],  H_l[n] = sum_o ds[n, o] Ws_l[o]
// (pure_cartesian_ictd_layers_full.py:990-1000 and its adjoint; Ws = (W_read + W_read^T)/2/sqrt(2l+1)).
//
// The (c, d) plane is cut into 8x8 blocks of 64 pairs.  One CTA owns 128 nodes (= the 128 TMEM
// lanes / MMA rows) and has a producer warp (bulk copies of W blocks and of the t rows a block
// needs into shared-memory rings), an MMA warp and 16 generator / epilogue warps:
//  * forward, per block (c-block <= d-block): the generator warps build the 128 x 64 Gram block on
//    CUDA cores from shared memory straight into TMEM and the MMA warp multiplies it with the W
//    block (doubled off the diagonal) into one of four TMEM accumulators, which the generators
//    add to fp32 registers a few blocks later;
//  * backward, per pair of d-blocks: the MMA warp forms the 128 x 128 block of H from ds (TMEM)
//    and two W blocks (N = 128 runs the tensor core at full rate) while the epilogue warps
//    contract an earlier one with t.
// Precision: the MMAs are kind::f16 on a two-term split, hi = fp16(x s), lo = fp16(x s - hi),
// summing hi*hi + hi*lo + lo*hi (~22 significant bits, like 3xTF32, at twice the K per
// instruction).  s is a power of two per node (from the Gram bound (2l+1) max t^2, or max |ds|)
// and per W image (host), so the range fits fp16 and unscaling is exact.  Products accumulate in
// fp32; every block is a fresh 12-MMA chain and the block sums are added in fp32 registers.
// All hand-offs go through mbarriers with bounded waits.
//
// t is read from Fg, a tile-blocked copy of the Gram operand (node n, row r at
// (n / 128) * nrows * 128 + r * 128 + n % 128, rows in the order of the reference's flat split,
// row = l-offset + c*(2l+1) + m; built by fg_gather_kernel): the rows one block needs are one
// contiguous chunk, moved by a single bulk copy.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {

namespace {

constexpr int TILE = 128;
constexpr int NGEN_WARPS = 16;  // 4 per TMEM lane quadrant
constexpr int THREADS = (NGEN_WARPS + 2) * 32;  // + MMA warp + producer (bulk copy) warp
constexpr int NSTB = 3;                          // W block ring
constexpr int NSTT = 4;                          // d-row chunk ring
constexpr int NSTC = 2;                          // c-row chunk ring (forward)
constexpr uint32_t TBYTES = 40u * TILE * 4u;     // one chunk: 8 rows x (2l+1 <= 5) x 128 nodes
constexpr int NSD = 4;                           // TMEM accumulator slots (MMA runs NSD - 1 blocks ahead)

// W images: a 64-byte header (float 0 = inverse of the power-of-two range scale applied to W),
// then fp16 hi / lo planes per block.
constexpr uint32_t WHEADER = 64u;

template <int S>
struct Smem {
  static constexpr uint32_t BBYTES = 256u * S;  // one W block (64 pairs x S), fp16 hi + lo
  static constexpr uint32_t T_OFF = NSTB * BBYTES;
  static constexpr uint32_t C_OFF = T_OFF + NSTT * TBYTES;
  static constexpr uint32_t BAR_FWD = C_OFF + NSTC * TBYTES;
  static constexpr uint32_t TOTAL_FWD = BAR_FWD + 256;
};

// Backward: the MMA forms H for two d-blocks at once (N = 128 pairs runs the tensor core at its
// full rate; N = 64 reaches ~70 %), so its rings hold W block pairs and 16-row t chunks.
constexpr int NSTB2 = 2, NSTT2 = 2, NSD2 = 3;
constexpr uint32_t TBYTES2 = 2 * TBYTES;
template <int S>
struct SmemBwd {
  static constexpr uint32_t BBYTES = 512u * S;  // two W blocks (128 pairs x S), fp16 hi + lo
  static constexpr uint32_t T_OFF = NSTB2 * BBYTES;
  static constexpr uint32_t BAR = T_OFF + NSTT2 * TBYTES2;
  static constexpr uint32_t TOTAL = BAR + 256;
};

// Ring-slot wait: slot k % n of use k waits for phase (k / n) & 1 of its barrier.
__device__ __forceinline__ bool ring_full(uint64_t* bars, int k, int n, int* err, int where) {
  return tc::mbar_wait(bars + k % n, (k / n) & 1, err, where);
}
// A producer's use k of a ring slot first waits for the consumers of use k - n.
__device__ __forceinline__ bool ring_empty(uint64_t* bars, int k, int n, int* err, int where) {
  return k < n || tc::mbar_wait(bars + k % n, ((k / n) - 1) & 1, err, where);
}

// Bulk copy of one chunk (or W block) into a ring slot with its byte count on the slot's barrier.
__device__ __forceinline__ void put(uint8_t* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  tc::mbar_arrive_expect_tx(bar, bytes);
  tc::bulk_g2s(dst, src, bytes, bar);
}

// Every CTA walks the Gram-block rows (b, cb) starting at its own row (and wrapping), so that at
// any moment the CTAs stream different W blocks: all CTAs reading the same 32 KB block at once
// would queue on the few L2 slices that hold it.
struct RowOrder {
  int rows, r0, nb;
  __device__ RowOrder(int ngram, int nb_) : rows(ngram * nb_), r0(0), nb(nb_) {
    r0 = (int)(blockIdx.x % (unsigned)rows);
  }
  __device__ __forceinline__ void at(int i, int& b, int& cb) const {
    const int r = (i + r0) % rows;
    b = r / nb;
    cb = r - b * nb;
  }
};
// Index of forward W block (b, cb, db >= cb) in the image (rows of nb - cb blocks).
__device__ __forceinline__ int fwd_block(int b, int cb, int db, int nb) {
  return b * (nb * (nb + 1) / 2) + cb * nb - cb * (cb - 1) / 2 + (db - cb);
}

// ------------------------------------------------------------------ forward
// Roles (one CTA = 128 nodes = the 128 TMEM lanes / MMA rows):
//  * producer warp: for every block s (Gram block b, c-block cb <= d-block db) bulk-copies the W
//    block s and the d-block's 8 (2l+1) t rows (one contiguous chunk of the tile-blocked Fg), and
//    once per (b, cb) the c-block's rows, into shared-memory rings;
//  * 16 generator warps: thread = node (TMEM lane) and quarter qq of the block: c-rows
//    4(qq & 1) + ci (held in registers for the whole block row), d-rows 4(qq >> 1) + di; builds
//    its 16 pairs of the Gram block (packed fp32 FMAs), scales them by the node's
//    power-of-two range factor (from gmax) and splits them into fp16 hi + lo in TMEM; adds output
//    columns [16qq, 16qq + 16) of an earlier block's fresh 12-MMA accumulator, unscaled (exact
//    powers of two), to fp32 registers, so the tensor core never carries a long accumulation chain;
//  * MMA warp: 12 tcgen05.mma kind::f16 (hi*hi + hi*lo + lo*hi over 4 K=16 steps; A = Gram block
//    in TMEM, B = W block in shared memory) per block.  kind::f16 moves K = 16 per instruction,
//    twice the K of kind::tf32 at the same instruction cost, with the same ~22-bit products.
template <int S>
__global__ void __launch_bounds__(THREADS, 1) readout_fwd_tc_kernel(ReadoutTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using SM = Smem<S>;
  uint8_t* sB = smem;
  const float* sT = reinterpret_cast<const float*>(smem + SM::T_OFF);
  const float* sC = reinterpret_cast<const float*>(smem + SM::C_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::BAR_FWD);
  uint64_t* full_B = bars;        // [3]
  uint64_t* empty_B = bars + 3;   // [3]
  uint64_t* full_T = bars + 6;    // [4]
  uint64_t* empty_T = bars + 10;  // [4]
  uint64_t* full_C = bars + 14;   // [2]
  uint64_t* empty_C = bars + 16;  // [2]
  uint64_t* full_A = bars + 18;   // [2]
  uint64_t* empty_A = bars + 20;  // [2]
  uint64_t* d_full = bars + 22;   // [NSD]
  uint64_t* d_empty = bars + 26;  // [NSD]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 30);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.nC / 8;
  const int64_t n0 = (int64_t)blockIdx.x * TILE;
  const int nblk = a.ngram * nb * (nb + 1) / 2;
  const float* Ftile = a.Fg + (int64_t)blockIdx.x * a.nrows * TILE;

  if (warp == NGEN_WARPS) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTB; ++i) {
      tc::mbar_init(full_B + i, 1);
      tc::mbar_init(empty_B + i, 1);
    }
    for (int i = 0; i < NSTT; ++i) {
      tc::mbar_init(full_T + i, 1);
      tc::mbar_init(empty_T + i, NGEN_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(full_C + i, 1);
      tc::mbar_init(empty_C + i, NGEN_WARPS);
      tc::mbar_init(full_A + i, NGEN_WARPS);
      tc::mbar_init(empty_A + i, 1);
    }
    for (int i = 0; i < NSD; ++i) {
      tc::mbar_init(d_full + i, 1);
      tc::mbar_init(d_empty + i, NGEN_WARPS);
    }
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  auto tD = [&](int st) { return tbase + 64u * st; };                             // cols [0, 256)
  auto tA = [&](int st, int lo) { return tbase + 256u + 64u * st + 32u * lo; };  // cols [256, 384)
  const float w_inv = a.wimg[0];

  if (warp < NGEN_WARPS) {
    // ---------------- Gram generators + block accumulation
    const int q4 = warp & 3, qq = warp >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool has_cols = 16 * qq < S;  // this warp owns output columns [16qq, 16qq+16)
    float2 acc[8];                      // columns 2i, 2i + 1
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
    bool ok = true;
    int s = 0, rr = 0;
    const int64_t n = n0 + row;
    // unscale factor of the rows in flight: rows start at blocks r_start[0] > [1] > [2]
    int r_start[3] = {0, 0, 0};
    float r_inv[3] = {1.f, 1.f, 1.f};
    auto flush = [&](int t) {
      const int dst = t % NSD;
      if (!ring_full(d_full, t, NSD, a.err, 16)) {
        ok = false;
        return;
      }
      tc::tc_fence_after();
      if (has_cols) {
        const float inv = t >= r_start[0] ? r_inv[0] : (t >= r_start[1] ? r_inv[1] : r_inv[2]);
        uint32_t v[16];
        tc::tmem_ld16(tD(dst) + lane_off + 16u * qq, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          acc[i] = __ffma2_rn(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), make_float2(inv, inv),
                              acc[i]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(d_empty + dst);
    };
    // one Gram block row (b, cb): c-rows from the C ring (held for the row), d-rows of every
    // db >= cb from the T ring
    auto gen_row = [&](auto mconst, int b, int cb) {
      constexpr int M = decltype(mconst)::value;
      const float scale = tc::f16_range_scale((float)M * a.gmax[(int64_t)b * a.n_pad + n]);
      r_start[2] = r_start[1];
      r_inv[2] = r_inv[1];
      r_start[1] = r_start[0];
      r_inv[1] = r_inv[0];
      r_start[0] = s;
      r_inv[0] = w_inv / scale;
      if (!ring_full(full_C, rr, NSTC, a.err, 12)) {
        ok = false;
        return;
      }
      float2 tcv[4][M];  // (t, t): the packed Gram FMA's broadcast operand, ready for the whole row
      {
        const float* pc = sC + (rr % NSTC) * (TBYTES / 4) + 4 * (qq & 1) * M * TILE + row;
#pragma unroll
        for (int ci = 0; ci < 4; ++ci)
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float t = pc[(ci * M + m) * TILE] * scale;  // power of two: exact
            tcv[ci][m] = make_float2(t, t);
          }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(empty_C + rr % NSTC);
      ++rr;
      for (int db = cb; db < nb; ++db, ++s) {
        if (!ring_full(full_T, s, NSTT, a.err, 10)) {
          ok = false;
          return;
        }
        float tdv[4][M];
        const float* pt = sT + (s % NSTT) * (TBYTES / 4) + 4 * (qq >> 1) * M * TILE + row;
#pragma unroll
        for (int di = 0; di < 4; ++di)
#pragma unroll
          for (int m = 0; m < M; ++m) tdv[di][m] = pt[(di * M + m) * TILE];
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty_T + s % NSTT);
        const int st = s & 1;
        if (s >= 2 && !tc::mbar_wait(empty_A + st, ((s >> 1) - 1) & 1, a.err, 11)) {
          ok = false;
          return;
        }
        // pairs (c = 4(qq&1) + ci, d = 4(qq>>1) + di) -> A element 16qq + 4ci + di (the forward W
        // images use this order), fp16 packed two per TMEM column: column 8qq + 2ci + di/2
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int ci = 0; ci < 4; ++ci)
#pragma unroll
          for (int dp = 0; dp < 2; ++dp) {
            float2 g = make_float2(0.f, 0.f);
#pragma unroll
            for (int m = 0; m < M; ++m)
              g = __ffma2_rn(tcv[ci][m], make_float2(tdv[2 * dp][m], tdv[2 * dp + 1][m]), g);
            tc::split_f16x2(g.x, g.y, hi[2 * ci + dp], lo[2 * ci + dp]);
          }
        tc::tmem_st8(tA(st, 0) + lane_off + 8u * qq, hi);
        tc::tmem_st8(tA(st, 1) + lane_off + 8u * qq, lo);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(full_A + st);
        if (s >= 2) {  // two blocks behind: that chain has long finished
          flush(s - 2);
          if (!ok) return;
        }
      }
    };
    const RowOrder order(a.ngram, nb);
    for (int i = 0; i < order.rows && ok; ++i) {
      int b, cb;
      order.at(i, b, cb);
      const int M = 2 * a.gl[b] + 1;
      if (M == 1) gen_row(std::integral_constant<int, 1>{}, b, cb);
      else if (M == 3) gen_row(std::integral_constant<int, 3>{}, b, cb);
      else gen_row(std::integral_constant<int, 5>{}, b, cb);
    }
    for (int t = nblk - 2; t < nblk && ok; ++t)
      if (t >= 0) flush(t);
    if (ok && has_cols && n < a.N) {
      float4* out = reinterpret_cast<float4*>(a.scalars + n * S + 16 * qq);
#pragma unroll
      for (int i = 0; i < 4; ++i) out[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
    }
  } else if (warp == NGEN_WARPS) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16(TILE, S);
      const uint32_t sB0 = tc::smem_u32(sB);
      for (int s = 0; s < nblk; ++s) {
        const int bst = s % NSTB, ast = s & 1, dst = s % NSD;
        if (!tc::mbar_wait(full_B + bst, (s / NSTB) & 1, a.err, 13)) break;
        if (!tc::mbar_wait(full_A + ast, (s >> 1) & 1, a.err, 14)) break;
        if (!ring_empty(d_empty, s, NSD, a.err, 17)) break;
        tc::tc_fence_after();
        const uint32_t bhi = sB0 + bst * SM::BBYTES, blo = bhi + SM::BBYTES / 2;
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // K = 16 pairs per step: 8 packed columns of A
          const uint64_t dh = tc::smem_desc_kmajor(bhi + j * 2 * 16 * S, 16 * S, 128);
          const uint64_t dl = tc::smem_desc_kmajor(blo + j * 2 * 16 * S, 16 * S, 128);
          tc::mma_f16_ts(tD(dst), tA(ast, 0) + 8 * j, dh, idesc, j != 0);
          tc::mma_f16_ts(tD(dst), tA(ast, 0) + 8 * j, dl, idesc, 1);
          tc::mma_f16_ts(tD(dst), tA(ast, 1) + 8 * j, dh, idesc, 1);
        }
        tc::mma_commit(empty_A + ast);
        tc::mma_commit(empty_B + bst);
        tc::mma_commit(d_full + dst);
      }
    }
  } else {
    // ---------------- producer: W blocks, d-row and c-row chunks (bulk copies)
    if (lane == 0) {
      const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(a.wimg) + WHEADER;
      uint8_t* tring = smem + SM::T_OFF;
      uint8_t* cring = smem + SM::C_OFF;
      int s = 0;
      bool ok = true;
      const RowOrder order(a.ngram, nb);
      for (int rr = 0; rr < order.rows && ok; ++rr) {
        int b, cb;
        order.at(rr, b, cb);
        const int M = 2 * a.gl[b] + 1, off = a.goff[b];
        const uint32_t cbytes = 8u * M * TILE * 4u;
        if (!(ok = ring_empty(empty_C, rr, NSTC, a.err, 18))) break;
        put(cring + (rr % NSTC) * TBYTES, Ftile + (int64_t)(off + 8 * cb * M) * TILE, cbytes, full_C + rr % NSTC);
        for (int db = cb; db < nb; ++db, ++s) {
          if (!(ok = ring_empty(empty_T, s, NSTT, a.err, 19))) break;
          put(tring + (s % NSTT) * TBYTES, Ftile + (int64_t)(off + 8 * db * M) * TILE, cbytes, full_T + s % NSTT);
          if (!(ok = ring_empty(empty_B, s, NSTB, a.err, 15))) break;
          const size_t wb = (size_t)fwd_block(b, cb, db, nb);
          put(sB + (s % NSTB) * SM::BBYTES, wsrc + wb * SM::BBYTES, SM::BBYTES, full_B + s % NSTB);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NGEN_WARPS) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------ backward
// Roles: the MMA warp forms H for two d-blocks at a time (A = ds, range-scaled and split into
// fp16 hi / lo in TMEM, B = the W block pair in shared memory; 3 x S/16 kind::f16 MMAs) into one of
// three TMEM accumulators; the producer streams W blocks and the d-block's t
// rows; 16 epilogue warps (thread = node, quarter qq of the c-rows: c = 2qq, 2qq + 1) contract
// the other accumulator with t from shared memory: dt[c][m] += 2 sum_d H[c][d] t[d][m] over all
// d-blocks of a row.
template <int S>
__global__ void __launch_bounds__(THREADS, 1) readout_bwd_tc_kernel(ReadoutTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using SM = SmemBwd<S>;
  uint8_t* sB = smem;
  const float* sT = reinterpret_cast<const float*>(smem + SM::T_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::BAR);
  uint64_t* full_B = bars;        // [NSTB2]
  uint64_t* empty_B = bars + 2;   // [NSTB2]
  uint64_t* full_T = bars + 4;    // [NSTT2]
  uint64_t* empty_T = bars + 6;   // [NSTT2]
  uint64_t* d_full = bars + 8;    // [NSD2]
  uint64_t* d_empty = bars + 11;  // [NSD2]
  uint64_t* a_ready = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  __shared__ float xch[4 * TILE * 10];  // row-end exchange of the epilogue quarters (2 c-rows x M <= 5)
  __shared__ uint64_t xbar[2];
  uint64_t* xfull = xbar;               // every epilogue warp wrote its exchange rows
  uint64_t* xempty = xbar + 1;          // every epilogue warp read them

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.nC / 8, np = nb / 2;  // d-block pairs per row
  const int64_t n0 = (int64_t)blockIdx.x * TILE;
  const int ngrp = a.ngram * nb * np;
  const float* Ftile = a.Fg + (int64_t)blockIdx.x * a.nrows * TILE;

  if (warp == NGEN_WARPS) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTB2; ++i) {
      tc::mbar_init(full_B + i, 1);
      tc::mbar_init(empty_B + i, 1);
    }
    for (int i = 0; i < NSTT2; ++i) {
      tc::mbar_init(full_T + i, 1);
      tc::mbar_init(empty_T + i, NGEN_WARPS);
    }
    for (int i = 0; i < NSD2; ++i) {
      tc::mbar_init(d_full + i, 1);
      tc::mbar_init(d_empty + i, NGEN_WARPS);
    }
    tc::mbar_init(a_ready, NGEN_WARPS);
    tc::mbar_init(xfull, NGEN_WARPS);
    tc::mbar_init(xempty, NGEN_WARPS);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tAhi = tbase, tAlo = tbase + 32u;                   // ds fp16 split, cols [0, 64)
  auto tD = [&](int st) { return tbase + 128u + 128u * st; };        // H block pairs, cols [128, 512)
  const float w_inv = a.wimg[0];
  __shared__ float dmax[4][TILE];

  if (warp < NGEN_WARPS) {
    const int q4 = warp & 3, qq = warp >> 2;
    const int row = q4 * 32 + lane;
    const int64_t n = n0 + row;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    // A operand: ds (128 x S) times the node's power-of-two range factor, split into fp16
    // hi / lo; warp quarter qq holds elements [16qq, 16qq+16) = packed columns [8qq, 8qq+8)
    float dv[16];
    float vmax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      dv[i] = (16 * qq < S && n < a.N) ? a.dscal[n * S + 16 * qq + i] : 0.f;
      vmax = fmaxf(vmax, fabsf(dv[i]));
    }
    dmax[qq][row] = vmax;
    asm volatile("bar.sync 1, %0;" ::"n"(NGEN_WARPS * 32) : "memory");  // generator warps only
    const float scale = tc::f16_range_scale(fmaxf(fmaxf(dmax[0][row], dmax[1][row]), fmaxf(dmax[2][row], dmax[3][row])));
    const float unscale = 2.f * w_inv / scale;  // dt = 2 H t; H carries scale / w_inv
    if (16 * qq < S) {
      uint32_t hi[8], lo[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) tc::split_f16x2(dv[2 * i] * scale, dv[2 * i + 1] * scale, hi[i], lo[i]);
      tc::tmem_st8(tAhi + lane_off + 8u * qq, hi);
      tc::tmem_st8(tAlo + lane_off + 8u * qq, lo);
      tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(a_ready);
    // epilogue over block pairs: quarter qq = 2 dblk + cq2 contracts c-rows 4 cq2 .. 4 cq2 + 3
    // with the 8 d-rows of d-block dblk of each pair (columns [32qq, 32qq + 32) of the pair's H:
    // 4d + c % 4, see the image order); at the end of a row the two d-block halves are summed
    // through shared memory and the thread writes c-rows 4 cq2 + 2 dblk, + 1.
    const int dblk = qq >> 1, cq2 = qq & 1;
    float* dFt = a.dFg + (int64_t)blockIdx.x * a.nrows * TILE + row;
    int s = 0, xrow = 0;
    bool ok = true;
    auto epi_row = [&](auto mconst, int off, int cb) {
      constexpr int M = decltype(mconst)::value;
      float acc[4][M];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[c][m] = 0.f;
      for (int dp = 0; dp < np; ++dp, ++s) {
        if (!ring_full(full_T, s, NSTT2, a.err, 20)) {
          ok = false;
          return;
        }
        const int st = s % NSD2;
        if (!ring_full(d_full, s, NSD2, a.err, 21)) {
          ok = false;
          return;
        }
        tc::tc_fence_after();
        uint32_t hv[32];
        tc::tmem_ld32(tD(st) + lane_off + 32u * qq, hv);
        const float* pt = sT + (s % NSTT2) * (TBYTES2 / 4) + 8 * dblk * M * TILE + row;
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          float td[M];
#pragma unroll
          for (int m = 0; m < M; ++m) td[m] = pt[(d * M + m) * TILE];
          if (d == 0) tc::tmem_wait_ld();
#pragma unroll
          for (int cp = 0; cp < 2; ++cp) {
            const float2 h2 = make_float2(__uint_as_float(hv[4 * d + 2 * cp]), __uint_as_float(hv[4 * d + 2 * cp + 1]));
#pragma unroll
            for (int m = 0; m < M; ++m) {
              const float2 t2 =
                  __ffma2_rn(h2, make_float2(td[m], td[m]), make_float2(acc[2 * cp][m], acc[2 * cp + 1][m]));
              acc[2 * cp][m] = t2.x;
              acc[2 * cp + 1][m] = t2.y;
            }
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(d_empty + st);
          tc::mbar_arrive(empty_T + s % NSTT2);
        }
      }
      // hand the partner quarter (other d-block, same c-rows) the two c-rows it writes; the
      // exchange rows are reused row after row (bounded mbarrier waits, no block barrier)
      if (xrow > 0 && !tc::mbar_wait(xempty, (uint32_t)((xrow - 1) & 1), a.err, 27)) {
        ok = false;
        return;
      }
      float* xs = xch + (qq * TILE + row) * 10;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) xs[j * M + m] = dblk ? acc[j][m] : acc[2 + j][m];
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(xfull);
      if (!tc::mbar_wait(xfull, (uint32_t)(xrow & 1), a.err, 28)) {
        ok = false;
        return;
      }
      const float* xr = xch + (((1 - dblk) * 2 + cq2) * TILE + row) * 10;
      float* pd = dFt + (int64_t)(off + (8 * cb + 4 * cq2 + 2 * dblk) * M) * TILE;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int m = 0; m < M; ++m) pd[(j * M + m) * TILE] = unscale * ((dblk ? acc[2 + j][m] : acc[j][m]) + xr[j * M + m]);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(xempty);
      ++xrow;
    };
    const RowOrder order(a.ngram, nb);
    for (int i = 0; i < order.rows && ok; ++i) {
      int b, cb;
      order.at(i, b, cb);
      const int M = 2 * a.gl[b] + 1, off = a.goff[b];
      if (M == 1) epi_row(std::integral_constant<int, 1>{}, off, cb);
      else if (M == 3) epi_row(std::integral_constant<int, 3>{}, off, cb);
      else epi_row(std::integral_constant<int, 5>{}, off, cb);
    }
  } else if (warp == NGEN_WARPS) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16(TILE, 128);
      const uint32_t sB0 = tc::smem_u32(sB);
      bool ok = tc::mbar_wait(a_ready, 0, a.err, 22);
      tc::tc_fence_after();
      for (int s = 0; s < ngrp && ok; ++s) {
        const int bst = s % NSTB2, dst = s % NSD2;
        if (!ring_full(full_B, s, NSTB2, a.err, 23)) break;
        if (!ring_empty(d_empty, s, NSD2, a.err, 24)) break;
        tc::tc_fence_after();
        const uint32_t bhi = sB0 + bst * SM::BBYTES, blo = bhi + SM::BBYTES / 2;
#pragma unroll
        for (int j = 0; j < S / 16; ++j) {  // K = 16 outputs per step: 8 packed columns of A
          const uint64_t dh = tc::smem_desc_kmajor(bhi + j * 2 * 16 * 128, 16 * 128, 128);
          const uint64_t dl = tc::smem_desc_kmajor(blo + j * 2 * 16 * 128, 16 * 128, 128);
          tc::mma_f16_ts(tD(dst), tAhi + 8 * j, dh, idesc, j != 0);
          tc::mma_f16_ts(tD(dst), tAhi + 8 * j, dl, idesc, 1);
          tc::mma_f16_ts(tD(dst), tAlo + 8 * j, dh, idesc, 1);
        }
        tc::mma_commit(empty_B + bst);
        tc::mma_commit(d_full + dst);
      }
    }
  } else {
    // ---------------- producer: W block pairs and 16-row t chunks
    if (lane == 0) {
      const uint8_t* wsrc = reinterpret_cast<const uint8_t*>(a.wimg) + WHEADER;
      uint8_t* tring = smem + SM::T_OFF;
      int s = 0;
      bool ok = true;
      const RowOrder order(a.ngram, nb);
      for (int rr = 0; rr < order.rows && ok; ++rr) {
        int b, cb;
        order.at(rr, b, cb);
        const int M = 2 * a.gl[b] + 1, off = a.goff[b];
        const uint32_t cbytes = 16u * M * TILE * 4u;
        for (int dp = 0; dp < np; ++dp, ++s) {
          if (!(ok = ring_empty(empty_T, s, NSTT2, a.err, 26))) break;
          put(tring + (s % NSTT2) * TBYTES2, Ftile + (int64_t)(off + 16 * dp * M) * TILE, cbytes, full_T + s % NSTT2);
          if (!(ok = ring_empty(empty_B, s, NSTB2, a.err, 25))) break;
          const size_t wg = (size_t)(b * nb + cb) * np + dp;
          put(sB + (s % NSTB2) * SM::BBYTES, wsrc + wg * SM::BBYTES, SM::BBYTES, full_B + s % NSTB2);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NGEN_WARPS) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------ Fg gather / scatter
// Fg[r][n] = feats[layer(r)][n][kc(r)] via xinv (storage -> row); tile of 32 nodes x one layer.
constexpr int FG_NODES = 32;


// Also: gmax[b][n] = max of t^2 over the Gram operand rows of block b (atomic max over the
// layers' CTAs; non-negative floats order like their bit patterns).  The rows of a block are the
// reference's flat split of the concatenated features, so t_b[c][m] is an arbitrary feature
// element; |G_cd| = |sum_m t_cm t_dm| <= (2l+1) gmax bounds the fp16 split's range.
// Both passes keep several 16-byte loads per thread in flight (memory bound transposes).
template <int C>
__global__ void __launch_bounds__(256) fg_gather_kernel(FgArgs a) {
  constexpr int W = 9 * C, W4 = W / 4, TS = W + 1, ROUND = 6;
  constexpr int PER = FG_NODES * W4 / 256;  // float4 loads per thread
  extern __shared__ float tile[];  // [FG_NODES][TS], then xinv of this layer [W]
  int* sinv = reinterpret_cast<int*>(tile + FG_NODES * TS);
  __shared__ unsigned int nmax[4][FG_NODES];
  const int layer = blockIdx.y, tid = threadIdx.x;
  const int64_t n0 = (int64_t)blockIdx.x * FG_NODES;
  const float4* src4 = reinterpret_cast<const float4*>(a.feats[layer]);
  if (tid < 4 * FG_NODES) (&nmax[0][0])[tid] = 0u;
  for (int i = tid; i < W; i += 256) sinv[i] = a.xinv[(int64_t)layer * W + i];
#pragma unroll
  for (int j0 = 0; j0 < PER; j0 += ROUND) {
    float4 v[ROUND];
#pragma unroll
    for (int j = 0; j < ROUND; ++j) {
      const int i = tid + 256 * (j0 + j), nl = i / W4, k4 = i - nl * W4;
      v[j] = (j0 + j < PER && n0 + nl < a.N) ? src4[(n0 + nl) * W4 + k4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < ROUND; ++j) {
      if (j0 + j >= PER) break;
      const int i = tid + 256 * (j0 + j), nl = i / W4, k4 = i - nl * W4;
      float* t = tile + nl * TS + 4 * k4;
      t[0] = v[j].x;
      t[1] = v[j].y;
      t[2] = v[j].z;
      t[3] = v[j].w;
    }
  }
  __syncthreads();
  // thread = one node (nl) and every 8th storage column; a warp writes one 128-byte row segment
  const int nl = tid & (FG_NODES - 1);
  const int64_t n = n0 + nl;
  float* fg = a.Fg + (n / TILE) * a.nrows * TILE + (n % TILE);
  float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll 8
  for (int kc = tid >> 5; kc < W; kc += 8) {
    const int r = sinv[kc];
    const float v = tile[nl * TS + kc];
    fg[(int64_t)r * TILE] = v;
    const float q = v * v;
    if (r < a.goff[1] || a.ngram == 1) m0 = fmaxf(m0, q);
    else if (r < a.goff[2] || a.ngram == 2) m1 = fmaxf(m1, q);
    else if (r < a.goff[3] || a.ngram == 3) m2 = fmaxf(m2, q);
    else m3 = fmaxf(m3, q);
  }
  atomicMax(&nmax[0][nl], __float_as_uint(m0));
  atomicMax(&nmax[1][nl], __float_as_uint(m1));
  atomicMax(&nmax[2][nl], __float_as_uint(m2));
  atomicMax(&nmax[3][nl], __float_as_uint(m3));
  __syncthreads();
  if (tid < 4 * FG_NODES) {
    const int b = tid / FG_NODES, l = tid - b * FG_NODES;
    if (b < a.ngram && n0 + l < a.n_pad)
      atomicMax(reinterpret_cast<unsigned int*>(a.gmax) + (int64_t)b * a.n_pad + n0 + l, nmax[b][l]);
  }
}

// grads[layer][n][kc] += dFg[r(kc)][n].  Both phases keep all of a thread's 16-byte loads in
// flight: dFg rows as float4 of 4 nodes (8 lanes cover the block's 32 nodes of one row), the
// gradient rows as float4 of 4 columns.
template <int C>
__global__ void __launch_bounds__(256, 2) fg_scatter_add_kernel(FgArgs a) {
  constexpr int W = 9 * C, W4 = W / 4, TS = W + 1;
  constexpr int PER = FG_NODES * W4 / 256;  // float4 per thread in either phase
  constexpr int RND = (PER + 1) / 2;        // loads in flight per round (two rounds: 2 CTAs per SM)
  static_assert(FG_NODES == 32 && W % 32 == 0 && PER * 256 == FG_NODES * W4, "tile shape");
  extern __shared__ float tile[];
  int* sinv = reinterpret_cast<int*>(tile + FG_NODES * TS);
  const int layer = blockIdx.y, tid = threadIdx.x;
  const int64_t n0 = (int64_t)blockIdx.x * FG_NODES;
  for (int i = tid; i < W; i += 256) sinv[i] = a.xinv[(int64_t)layer * W + i];
  __syncthreads();
  {
    // rows of the padded operand exist for every node of the 128-node tile
    const int g = tid & 7, rr = tid >> 3;
    const float* fg = a.dFg + (n0 / TILE) * a.nrows * TILE + (n0 % TILE) + 4 * g;
#pragma unroll
    for (int j0 = 0; j0 < PER; j0 += RND) {
      float4 v[RND];
#pragma unroll
      for (int j = 0; j < RND; ++j)
        if (j0 + j < PER) v[j] = *reinterpret_cast<const float4*>(fg + (int64_t)sinv[rr + 32 * (j0 + j)] * TILE);
#pragma unroll
      for (int j = 0; j < RND; ++j) {
        if (j0 + j >= PER) break;
        float* t = tile + (4 * g) * TS + rr + 32 * (j0 + j);
        t[0] = v[j].x;
        t[TS] = v[j].y;
        t[2 * TS] = v[j].z;
        t[3 * TS] = v[j].w;
      }
    }
  }
  __syncthreads();
  float4* dst4 = reinterpret_cast<float4*>(a.grads[layer]);
#pragma unroll
  for (int j0 = 0; j0 < PER; j0 += RND) {
    float4 g[RND];
#pragma unroll
    for (int j = 0; j < RND; ++j) {
      const int i = tid + 256 * (j0 + j), nl = i / W4, k4 = i - nl * W4;
      if (j0 + j < PER && n0 + nl < a.N) g[j] = dst4[(n0 + nl) * W4 + k4];
    }
#pragma unroll
    for (int j = 0; j < RND; ++j) {
      const int i = tid + 256 * (j0 + j), nl = i / W4, k4 = i - nl * W4;
      if (j0 + j >= PER || n0 + nl >= a.N) continue;
      const float* t = tile + nl * TS + 4 * k4;
      g[j].x += t[0];
      g[j].y += t[1];
      g[j].z += t[2];
      g[j].w += t[3];
      dst4[(n0 + nl) * W4 + k4] = g[j];
    }
  }
}

template <int S>
int launch_fwd(const ReadoutTcArgs& a, cudaStream_t st) {
  const int sm = Smem<S>::TOTAL_FWD;
  cudaFuncSetAttribute(readout_fwd_tc_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  readout_fwd_tc_kernel<S><<<(unsigned)ceil_div(a.N, TILE), THREADS, sm, st>>>(a);
  return check_launch("readout_fwd_tc_kernel");
}
template <int S>
int launch_bwd(const ReadoutTcArgs& a, cudaStream_t st) {
  const int sm = SmemBwd<S>::TOTAL;
  cudaFuncSetAttribute(readout_bwd_tc_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  readout_bwd_tc_kernel<S><<<(unsigned)ceil_div(a.N, TILE), THREADS, sm, st>>>(a);
  return check_launch("readout_bwd_tc_kernel");
}

}  // namespace

bool readout_tc_supported(int nC, int S) { return (S == 32 || S == 64) && nC % 8 == 0 && nC <= 512; }

int64_t readout_tc_blocks(int nC, int ngram, bool backward) {
  const int64_t nb = nC / 8;
  return backward ? ngram * nb * nb : ngram * nb * (nb + 1) / 2;
}

int launch_readout_fwd_tc(const ReadoutTcArgs& a, cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  if (a.ngram < 1 || a.ngram > 4) return fail(FSC_ERR_ARGUMENT, "readout: 1..4 Gram blocks");
  if (a.S == 64) return launch_fwd<64>(a, st);
  if (a.S == 32) return launch_fwd<32>(a, st);
  return fail(FSC_ERR_UNSUPPORTED, "tensor-core readout needs S in {32, 64}");
}

int launch_readout_bwd_tc(const ReadoutTcArgs& a, cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  if (a.ngram < 1 || a.ngram > 4) return fail(FSC_ERR_ARGUMENT, "readout: 1..4 Gram blocks");
  if (a.S == 64) return launch_bwd<64>(a, st);
  if (a.S == 32) return launch_bwd<32>(a, st);
  return fail(FSC_ERR_UNSUPPORTED, "tensor-core readout needs S in {32, 64}");
}

int launch_fg_gather(const FgArgs& a, cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  if (a.C != 32 && a.C != 64) return fail(FSC_ERR_UNSUPPORTED, "fg_gather: C must be 32 or 64");
  const int sm = (FG_NODES * (9 * a.C + 1) + 9 * a.C) * (int)sizeof(float);
  dim3 grid((unsigned)ceil_div(a.n_pad, FG_NODES), (unsigned)a.nint);
  if (a.C == 64) {
    cudaFuncSetAttribute(fg_gather_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    fg_gather_kernel<64><<<grid, 256, sm, st>>>(a);
  } else {
    cudaFuncSetAttribute(fg_gather_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    fg_gather_kernel<32><<<grid, 256, sm, st>>>(a);
  }
  return check_launch("fg_gather_kernel");
}

int launch_fg_scatter_add(const FgArgs& a, cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  if (a.C != 32 && a.C != 64) return fail(FSC_ERR_UNSUPPORTED, "fg_scatter_add: C must be 32 or 64");
  const int sm = (FG_NODES * (9 * a.C + 1) + 9 * a.C) * (int)sizeof(float);
  dim3 grid((unsigned)ceil_div(a.n_pad, FG_NODES), (unsigned)a.nint);
  if (a.C == 64) {
    cudaFuncSetAttribute(fg_scatter_add_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    fg_scatter_add_kernel<64><<<grid, 256, sm, st>>>(a);
  } else {
    cudaFuncSetAttribute(fg_scatter_add_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    fg_scatter_add_kernel<32><<<grid, 256, sm, st>>>(a);
  }
  return check_launch("fg_scatter_add_kernel");
}

}  // namespace fsc
