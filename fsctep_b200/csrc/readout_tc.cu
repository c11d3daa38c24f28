// Readout Gram contraction on the 5th-generation tensor cores (tcgen05, TMEM, bulk TMA).
//
// Forward   scalars[n, o] = sum_l sum_{c,d} Ws_l[o, c, d] G_l[n, c, d],  G_l[n] = t_l t_l^T (over m)
// Backward  dt_l[n, c, m] = 2 sum_d H_l[n, c, d] t_l[n, d, m],  H_l[n] = sum_o ds[n, o] Ws_l[o]
// (pure_cartesian_ictd_layers_full.py:990-1000 and its adjoint; Ws = (W_read + W_read^T)/2/sqrt(2l+1)).
//
// The (c, d) plane is cut into 8x8 blocks of 64 pairs.  One CTA owns 128 nodes (= the 128 TMEM
// lanes / MMA rows):
//  * forward, per block (c-block <= d-block): 8 generator warps build the 128 x 64 Gram block
//    on CUDA cores straight into TMEM (thread = node = TMEM lane) and an elected thread issues
//    tcgen05.mma with A from TMEM and the pre-formatted W block (doubled off the diagonal) from
//    shared memory, accumulating the 128 x S scalars in TMEM;
//  * backward, per block (all c-, d-blocks): tcgen05.mma forms the 128 x 64 block of H from ds
//    (in TMEM) and the W block (shared memory) into one of two TMEM accumulators while the 8
//    epilogue warps contract the other with t on CUDA cores.
// W blocks are streamed by 1-D bulk TMA into a 3-stage shared-memory ring; all hand-offs go
// through mbarriers with bounded waits.  fp32 accuracy comes from the 3xTF32 split
// (hi*hi + hi*lo + lo*hi; the W split is precomputed on the host).
//
// t is read from Fg, a node-innermost copy of the Gram operand (Fg[row][n], row = l-offset +
// c*(2l+1) + m, rows in the order of the reference's flat split; built by fg_gather_kernel),
// so that one warp's 32 nodes read one 128-byte line per (c, m).
#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {

namespace {

constexpr int TILE = 128;
constexpr int NGEN_WARPS = 8;
constexpr int THREADS = (NGEN_WARPS + 2) * 32;  // + MMA warp + TMA warp
constexpr int NSTB = 3;


template <int S>
struct Smem {
  static constexpr uint32_t BBYTES = 512u * S;  // one W block, hi + lo
  static constexpr uint32_t BAR_OFF = NSTB * BBYTES;
  static constexpr uint32_t TOTAL = BAR_OFF + 256;
  // the forward allocates all 512 TMEM columns: keep it at one CTA per SM through shared memory
  static constexpr uint32_t TOTAL_FWD = TOTAL > 120u * 1024u ? TOTAL : 120u * 1024u;
};

// ------------------------------------------------------------------ forward
// Each 64-pair block is accumulated fresh in one of two TMEM accumulators (24 MMAs) and added to
// per-thread fp32 registers (round-to-nearest) by the generator warps, so the tensor core never
// carries a long accumulation chain.
template <int S>
__global__ void __launch_bounds__(THREADS, 1) readout_fwd_tc_kernel(ReadoutTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using SM = Smem<S>;
  uint8_t* sB = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::BAR_OFF);
  uint64_t* full_B = bars;        // [3]
  uint64_t* empty_B = bars + 3;   // [3]
  uint64_t* full_A = bars + 6;    // [2]
  uint64_t* empty_A = bars + 8;   // [2]
  uint64_t* d_full = bars + 10;   // [2]
  uint64_t* d_empty = bars + 12;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nC = a.nC, nb = nC / 8;
  const int64_t n0 = (int64_t)blockIdx.x * TILE;
  const int nblk = a.ngram * nb * (nb + 1) / 2;

  if (warp == NGEN_WARPS) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTB; ++i) {
      tc::mbar_init(full_B + i, 1);
      tc::mbar_init(empty_B + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(full_A + i, NGEN_WARPS);
      tc::mbar_init(empty_A + i, 1);
      tc::mbar_init(d_full + i, 1);
      tc::mbar_init(d_empty + i, NGEN_WARPS);
    }
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  auto tD = [&](int st) { return tbase + 64u * st; };                              // cols [0, 128)
  auto tA = [&](int st, int lo) { return tbase + 128u + 128u * st + 64u * lo; };  // cols [128, 384)

  if (warp < NGEN_WARPS) {
    // ---------------- Gram generators + block accumulation
    const int q4 = warp & 3, h = warp >> 2;
    const int row = q4 * 32 + lane;
    const int64_t n = n0 + row;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool has_cols = 32 * h < S;  // this warp half owns output columns [32h, 32h+32)
    const float* Fg = a.Fg + n;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    bool ok = true;
    auto flush = [&](int t) {
      const int dst = t & 1;
      if (!tc::mbar_wait(d_full + dst, (t >> 1) & 1, a.err, 16)) {
        ok = false;
        return;
      }
      tc::tc_fence_after();
      if (has_cols) {
        uint32_t v[32];
        tc::tmem_ld32(tD(dst) + lane_off + 32u * h, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] += __uint_as_float(v[i]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(d_empty + dst);
    };
    int s = 0;
    for (int b = 0; b < a.ngram && ok; ++b) {
      const int M = 2 * a.gl[b] + 1, off = a.goff[b];
      for (int cb = 0; cb < nb && ok; ++cb) {
        float tcv[4][5];
#pragma unroll
        for (int cq = 0; cq < 4; ++cq)
#pragma unroll
          for (int m = 0; m < 5; ++m)
            tcv[cq][m] = m < M ? Fg[(int64_t)(off + (8 * cb + 4 * h + cq) * M + m) * a.n_pad] : 0.f;
        for (int db = cb; db < nb && ok; ++db, ++s) {
          float tdv[8][5];
#pragma unroll
          for (int dq = 0; dq < 8; ++dq)
#pragma unroll
            for (int m = 0; m < 5; ++m)
              tdv[dq][m] = m < M ? Fg[(int64_t)(off + (8 * db + dq) * M + m) * a.n_pad] : 0.f;
          const int st = s & 1;
          if (s >= 2 && !tc::mbar_wait(empty_A + st, ((s >> 1) - 1) & 1, a.err, 11)) {
            ok = false;
            break;
          }
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int cq = 0; cq < 4; ++cq)
#pragma unroll
            for (int dq = 0; dq < 8; ++dq) {
              float g = 0.f;
#pragma unroll
              for (int m = 0; m < 5; ++m) g = fmaf(tcv[cq][m], tdv[dq][m], g);
              tc::split_tf32(g, hi[cq * 8 + dq], lo[cq * 8 + dq]);
            }
          tc::tmem_st32(tA(st, 0) + lane_off + 32u * h, hi);
          tc::tmem_st32(tA(st, 1) + lane_off + 32u * h, lo);
          tc::tmem_wait_st();
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(full_A + st);
          if (s >= 1) flush(s - 1);
        }
      }
    }
    if (ok) flush(nblk - 1);
    if (ok && has_cols && n < a.N) {
      float4* out = reinterpret_cast<float4*>(a.scalars + n * S + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
    }
  } else if (warp == NGEN_WARPS) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(TILE, S);
      const uint32_t sB0 = tc::smem_u32(sB);
      for (int s = 0; s < nblk; ++s) {
        const int bst = s % NSTB, ast = s & 1;
        if (!tc::mbar_wait(full_B + bst, (s / NSTB) & 1, a.err, 13)) break;
        if (!tc::mbar_wait(full_A + ast, (s >> 1) & 1, a.err, 14)) break;
        if (s >= 2 && !tc::mbar_wait(d_empty + ast, ((s >> 1) - 1) & 1, a.err, 17)) break;
        tc::tc_fence_after();
        const uint32_t bhi = sB0 + bst * SM::BBYTES, blo = bhi + SM::BBYTES / 2;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t dh = tc::smem_desc_kmajor(bhi + j * 2 * 16 * S, 16 * S, 128);
          const uint64_t dl = tc::smem_desc_kmajor(blo + j * 2 * 16 * S, 16 * S, 128);
          tc::mma_tf32_ts(tD(ast), tA(ast, 0) + 8 * j, dh, idesc, j != 0);
          tc::mma_tf32_ts(tD(ast), tA(ast, 0) + 8 * j, dl, idesc, 1);
          tc::mma_tf32_ts(tD(ast), tA(ast, 1) + 8 * j, dh, idesc, 1);
        }
        tc::mma_commit(empty_A + ast);
        tc::mma_commit(empty_B + bst);
        tc::mma_commit(d_full + ast);
      }
    }
  } else {
    // ---------------- W block producer (bulk TMA)
    if (lane == 0) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.wimg);
      for (int s = 0; s < nblk; ++s) {
        const int bst = s % NSTB;
        if (s >= NSTB && !tc::mbar_wait(empty_B + bst, ((s / NSTB) - 1) & 1, a.err, 15)) break;
        tc::mbar_arrive_expect_tx(full_B + bst, SM::BBYTES);
        tc::bulk_g2s(sB + bst * SM::BBYTES, src + (size_t)s * SM::BBYTES, SM::BBYTES, full_B + bst);
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
template <int S>
__global__ void __launch_bounds__(THREADS, 1) readout_bwd_tc_kernel(ReadoutTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using SM = Smem<S>;
  uint8_t* sB = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::BAR_OFF);
  uint64_t* full_B = bars;       // [3]
  uint64_t* empty_B = bars + 3;  // [3]
  uint64_t* d_full = bars + 6;   // [2]
  uint64_t* d_empty = bars + 8;  // [2]
  uint64_t* a_ready = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nC = a.nC, nb = nC / 8;
  const int64_t n0 = (int64_t)blockIdx.x * TILE;
  const int nblk = a.ngram * nb * nb;

  if (warp == NGEN_WARPS) {
    tc::tmem_alloc(tmem_slot, 256);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTB; ++i) {
      tc::mbar_init(full_B + i, 1);
      tc::mbar_init(empty_B + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(d_full + i, 1);
      tc::mbar_init(d_empty + i, NGEN_WARPS);
    }
    tc::mbar_init(a_ready, NGEN_WARPS);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tAhi = tbase, tAlo = tbase + 64u;                  // ds split, cols [0, 128)
  auto tD = [&](int st) { return tbase + 128u + 64u * st; };         // H blocks, cols [128, 256)

  if (warp < NGEN_WARPS) {
    const int q4 = warp & 3, h = warp >> 2;
    const int row = q4 * 32 + lane;
    const int64_t n = n0 + row;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    // A operand: ds (128 x S), split into hi / lo; warp half h stores columns [32h, 32h+32)
    if (32 * h < S) {
      uint32_t hi[32], lo[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float v = n < a.N ? a.dscal[n * S + 32 * h + i] : 0.f;
        tc::split_tf32(v, hi[i], lo[i]);
      }
      tc::tmem_st32(tAhi + lane_off + 32u * h, hi);
      tc::tmem_st32(tAlo + lane_off + 32u * h, lo);
      tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(a_ready);
    // epilogue over blocks
    const float* Fg = a.Fg + n;
    float* dFg = a.dFg + n;
    int s = 0;
    bool ok = true;
    for (int b = 0; b < a.ngram && ok; ++b) {
      const int M = 2 * a.gl[b] + 1, off = a.goff[b];
      for (int cb = 0; cb < nb && ok; ++cb) {
        float acc[4][5];
#pragma unroll
        for (int cq = 0; cq < 4; ++cq)
#pragma unroll
          for (int m = 0; m < 5; ++m) acc[cq][m] = 0.f;
        for (int db = 0; db < nb; ++db, ++s) {
          float tdv[8][5];
#pragma unroll
          for (int dq = 0; dq < 8; ++dq)
#pragma unroll
            for (int m = 0; m < 5; ++m)
              tdv[dq][m] = m < M ? Fg[(int64_t)(off + (8 * db + dq) * M + m) * a.n_pad] : 0.f;
          const int st = s & 1;
          if (!tc::mbar_wait(d_full + st, (s >> 1) & 1, a.err, 21)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          uint32_t hv[32];
          tc::tmem_ld32(tD(st) + lane_off + 32u * h, hv);
          tc::tmem_wait_ld();
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(d_empty + st);
#pragma unroll
          for (int cq = 0; cq < 4; ++cq)
#pragma unroll
            for (int dq = 0; dq < 8; ++dq) {
              const float hcd = __uint_as_float(hv[cq * 8 + dq]);
#pragma unroll
              for (int m = 0; m < 5; ++m) acc[cq][m] = fmaf(hcd, tdv[dq][m], acc[cq][m]);
            }
        }
        if (!ok) break;
#pragma unroll
        for (int cq = 0; cq < 4; ++cq)
#pragma unroll
          for (int m = 0; m < 5; ++m)
            if (m < M) dFg[(int64_t)(off + (8 * cb + 4 * h + cq) * M + m) * a.n_pad] = 2.f * acc[cq][m];
      }
    }
  } else if (warp == NGEN_WARPS) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(TILE, 64);
      const uint32_t sB0 = tc::smem_u32(sB);
      bool ok = tc::mbar_wait(a_ready, 0, a.err, 22);
      tc::tc_fence_after();
      for (int s = 0; s < nblk && ok; ++s) {
        const int bst = s % NSTB, dst = s & 1;
        if (!tc::mbar_wait(full_B + bst, (s / NSTB) & 1, a.err, 23)) break;
        if (s >= 2 && !tc::mbar_wait(d_empty + dst, ((s >> 1) - 1) & 1, a.err, 24)) break;
        tc::tc_fence_after();
        const uint32_t bhi = sB0 + bst * SM::BBYTES, blo = bhi + SM::BBYTES / 2;
#pragma unroll
        for (int j = 0; j < S / 8; ++j) {
          const uint64_t dh = tc::smem_desc_kmajor(bhi + j * 2 * 16 * 64, 16 * 64, 128);
          const uint64_t dl = tc::smem_desc_kmajor(blo + j * 2 * 16 * 64, 16 * 64, 128);
          tc::mma_tf32_ts(tD(dst), tAhi + 8 * j, dh, idesc, j != 0);
          tc::mma_tf32_ts(tD(dst), tAhi + 8 * j, dl, idesc, 1);
          tc::mma_tf32_ts(tD(dst), tAlo + 8 * j, dh, idesc, 1);
        }
        tc::mma_commit(empty_B + bst);
        tc::mma_commit(d_full + dst);
      }
    }
  } else {
    if (lane == 0) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.wimg);
      for (int s = 0; s < nblk; ++s) {
        const int bst = s % NSTB;
        if (s >= NSTB && !tc::mbar_wait(empty_B + bst, ((s / NSTB) - 1) & 1, a.err, 25)) break;
        tc::mbar_arrive_expect_tx(full_B + bst, SM::BBYTES);
        tc::bulk_g2s(sB + bst * SM::BBYTES, src + (size_t)s * SM::BBYTES, SM::BBYTES, full_B + bst);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == NGEN_WARPS) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 256);
  }
}

// ------------------------------------------------------------------ Fg gather / scatter
// Fg[r][n] = feats[layer(r)][n][kc(r)] via xinv (storage -> row); tile of 32 nodes x one layer.
constexpr int FG_NODES = 32;

__global__ void fg_gather_kernel(FgArgs a) {
  extern __shared__ float tile[];  // [FG_NODES][9C + 1]
  const int layer = blockIdx.y;
  const int W = 9 * a.C;
  const int64_t n0 = (int64_t)blockIdx.x * FG_NODES;
  const float* src = a.feats[layer];
  for (int i = threadIdx.x; i < FG_NODES * W; i += blockDim.x) {
    const int nl = i / W, kc = i - nl * W;
    const int64_t n = n0 + nl;
    tile[nl * (W + 1) + kc] = n < a.N ? src[n * W + kc] : 0.f;
  }
  __syncthreads();
  const int32_t* inv = a.xinv + (int64_t)layer * W;
  for (int i = threadIdx.x; i < FG_NODES * W; i += blockDim.x) {
    const int kc = i / FG_NODES, nl = i - kc * FG_NODES;
    a.Fg[(int64_t)inv[kc] * a.n_pad + n0 + nl] = tile[nl * (W + 1) + kc];
  }
}

// grads[layer][n][kc] += dFg[r(kc)][n]
__global__ void fg_scatter_add_kernel(FgArgs a) {
  extern __shared__ float tile[];
  const int layer = blockIdx.y;
  const int W = 9 * a.C;
  const int64_t n0 = (int64_t)blockIdx.x * FG_NODES;
  const int32_t* inv = a.xinv + (int64_t)layer * W;
  for (int i = threadIdx.x; i < FG_NODES * W; i += blockDim.x) {
    const int kc = i / FG_NODES, nl = i - kc * FG_NODES;
    tile[nl * (W + 1) + kc] = a.dFg[(int64_t)inv[kc] * a.n_pad + n0 + nl];
  }
  __syncthreads();
  float* dst = a.grads[layer];
  for (int i = threadIdx.x; i < FG_NODES * W; i += blockDim.x) {
    const int nl = i / W, kc = i - nl * W;
    const int64_t n = n0 + nl;
    if (n < a.N) dst[n * W + kc] += tile[nl * (W + 1) + kc];
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
  const int sm = Smem<S>::TOTAL;
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
  const int sm = FG_NODES * (9 * a.C + 1) * (int)sizeof(float);
  cudaFuncSetAttribute(fg_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  dim3 grid((unsigned)ceil_div(a.n_pad, FG_NODES), (unsigned)a.nint);
  fg_gather_kernel<<<grid, 256, sm, st>>>(a);
  return check_launch("fg_gather_kernel");
}

int launch_fg_scatter_add(const FgArgs& a, cudaStream_t st) {
  if (a.N == 0) return FSC_OK;
  const int sm = FG_NODES * (9 * a.C + 1) * (int)sizeof(float);
  cudaFuncSetAttribute(fg_scatter_add_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  dim3 grid((unsigned)ceil_div(a.n_pad, FG_NODES), (unsigned)a.nint);
  fg_scatter_add_kernel<<<grid, 256, sm, st>>>(a);
  return check_launch("fg_scatter_add_kernel");
}

}  // namespace fsc
