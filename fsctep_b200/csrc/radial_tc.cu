// Per-edge radial MLPs of the ictd layers on the 5th-generation tensor cores.
//
// Forward, per layer (fc / fc2_layers, pure_cartesian_ictd_layers_full.py:277-283, 693-699):
//   gates = W3 silu(W2 silu(W1 emb + b1) + b2) + b3,   emb = radial basis of |r_e| (nb <= 16)
// Backward, per layer (the adjoint autograd replays, evaluation/calculator.py:158-159):
//   dh2 = W3^T dgates, da2 = dh2 * silu'(a2), dh1 = W2^T da2, da1 = dh1 * silu'(a1),
//   dE/d|r| += (W1^T da1) . demb/d|r|
// and, after the last layer, the direction part dE/dY -> dE/dr (edge_grad).
//
// One CTA owns a tile of 128 edges (edge = TMEM lane = MMA row) and walks its tiles persistently.
// Every matrix product of the MLP is a chain of tcgen05.mma (kind::tf32, M = 128) with the
// activations as the A operand in TMEM and the layer's weights as B operand images in shared
// memory.  fp32 accuracy comes from the 3xTF32 split (hi*hi + hi*lo + lo*hi).  The element-wise
// steps (bias, SiLU and its derivative, tf32 split) run on the CUDA cores between the MMA chains,
// reading the accumulators with tcgen05.ld and writing the next A with tcgen05.st: two threads per
// edge (warps w and w + 4 share TMEM lanes 32 (w % 4) ...), each owning 32 of the 64 hidden
// columns, so 16 warps per SM share the latency of those steps.  Two CTAs share an SM (256 TMEM
// columns each) so one CTA's element-wise work overlaps the other's MMAs.
//
#include "common.cuh"
#include "edge_common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {

namespace {

constexpr int RT = 128;      // edges per tile
constexpr int RTH = 2 * RT;  // threads per CTA: two per edge
constexpr int RH = 64;       // hidden width (fixed by the reference)
constexpr int RP = 11;       // gates per layer
constexpr int RT_PER_SM = 2; // CTAs per SM
constexpr uint32_t kMinSmem = 80u * 1024u;  // keeps at most two CTAs (512 TMEM columns) per SM

// B-operand image of a row-major N x K matrix for a K-major, no-swizzle descriptor: element
// (n, k) at float (k/4)*4N + 4n + k%4.  The 8-wide K step j starts at byte 32*N*j; the second
// 4-wide K half is LBO = 16*N bytes further, the next 8 rows SBO = 128 bytes further.
__device__ __forceinline__ int bimg(int n, int k, int N) { return (k >> 2) * 4 * N + 4 * n + (k & 3); }

template <int NBP>
struct FwdImg {
  static constexpr int W1 = 0;                // [64][NBP]   B[k][b] = W1[k][b]
  static constexpr int W2 = W1 + RH * NBP;    // [64][64]    B[j][k] = W2[j][k]
  static constexpr int W3 = W2 + RH * RH;     // [16][64]    B[q][j] = W3[q][j] (q >= 11 zero)
  static constexpr int SIZE = W3 + 16 * RH;
};

template <int NBP>
struct BwdImg {
  static constexpr int W1 = 0;                // [64][NBP]   B[k][b] = W1[k][b]
  static constexpr int W3P = W1 + RH * NBP;   // [64][16]    B[j][q] = W3[q][j]
  static constexpr int W2 = W3P + RH * 16;    // [64][64]    B[j][k] = W2[j][k]
  static constexpr int W2T = W2 + RH * RH;    // [64][64]    B[k][j] = W2[j][k]
  static constexpr int W1T = W2T + RH * RH;   // [16][64]    B[b][k] = W1[k][b] (b >= nb zero)
  static constexpr int SIZE = W1T + 16 * RH;
};

// Shared memory: hi images, lo images, biases, ypoly, the exchange rows of the two column
// halves (an N = 16 product's partial sums), mbarrier, TMEM slot.
constexpr int XST = 17;  // exchange row stride (odd: no bank conflicts)
template <int SIZE>
struct RtSmem {
  static constexpr uint32_t HI = 0;
  static constexpr uint32_t LO = 4u * SIZE;
  static constexpr uint32_t BIAS = 8u * SIZE;                   // b1[64], b2[64], b3[16]
  static constexpr uint32_t YPOLY = BIAS + 4u * 144;            // [NMONO][NK]
  static constexpr uint32_t XCH = YPOLY + 4u * 96;              // [RT][XST]
  static constexpr uint32_t BAR = (XCH + 4u * RT * XST + 15u) & ~15u;
  static constexpr uint32_t TOTAL_RAW = BAR + 16;
  static constexpr uint32_t TOTAL = TOTAL_RAW > kMinSmem ? TOTAL_RAW : kMinSmem;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Writes element (n, k) of a B image, split into tf32 hi and lo.
__device__ __forceinline__ void put_b(float* hi, float* lo, int off, int N, int n, int k, float v) {
  uint32_t h, l;
  tc::split_tf32(v, h, l);
  hi[off + bimg(n, k, N)] = __uint_as_float(h);
  lo[off + bimg(n, k, N)] = __uint_as_float(l);
}

__device__ __forceinline__ void load_bias(float* bias, const RadialW& W, int layer) {
  for (int i = threadIdx.x; i < 144; i += blockDim.x) {
    float v;
    if (i < RH) v = W.b1[layer * RH + i];
    else if (i < 2 * RH) v = W.b2[layer * RH + i - RH];
    else v = ((i - 2 * RH) < RP && W.b3) ? W.b3[layer * RP + i - 2 * RH] : 0.f;
    bias[i] = v;
  }
}

// D = A x B^T over `ksteps` 8-wide K steps with the 3xTF32 split.  The tensor core truncates
// every accumulation toward zero, which biases long chains; so the two small cross terms of all
// K steps are accumulated before the hi*hi terms, and K step j goes to accumulator j % nacc
// (at column d + (j % nacc) * acc_cols), which the CUDA cores add up with round-to-nearest.
__device__ __forceinline__ void mma_3xtf32(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                           int N, int ksteps, uint32_t idesc, int nacc = 1, uint32_t acc_cols = 0) {
  for (int j = 0; j < ksteps; ++j) {
    const uint32_t dj = d + (uint32_t)(j % nacc) * acc_cols;
    const uint64_t dh = tc::smem_desc_kmajor(b_hi + 32u * N * j, 16u * N, 128);
    const uint64_t dl = tc::smem_desc_kmajor(b_lo + 32u * N * j, 16u * N, 128);
    tc::mma_tf32_ts(dj, a_hi + 8u * j, dl, idesc, j >= nacc);
    tc::mma_tf32_ts(dj, a_lo + 8u * j, dh, idesc, 1);
  }
  for (int j = 0; j < ksteps; ++j) {
    const uint32_t dj = d + (uint32_t)(j % nacc) * acc_cols;
    const uint64_t dh = tc::smem_desc_kmajor(b_hi + 32u * N * j, 16u * N, 128);
    tc::mma_tf32_ts(dj, a_hi + 8u * j, dh, idesc, 1);
  }
}

// Sum of four of the eight 16-column accumulators of an N = 16 product: columns [t, t + 64).
__device__ __forceinline__ void ld_sum16x4(uint32_t t, float* out) {
  uint32_t u[32], w[32];
  tc::tmem_ld32(t, u);
  tc::tmem_ld32(t + 32u, w);
  tc::tmem_wait_ld();
#pragma unroll
  for (int q = 0; q < 16; ++q)
    out[q] = (__uint_as_float(u[q]) + __uint_as_float(u[16 + q])) + (__uint_as_float(w[q]) + __uint_as_float(w[16 + q]));
}

// Full sum of the eight accumulators in the threads of column half 0: half 1 hands its partial
// sums over through shared memory.  Block-wide (contains a barrier).
__device__ __forceinline__ void sum16x8_halves(uint32_t t_lane, int half, int row, float* xch, float* out) {
  ld_sum16x4(t_lane + 64u * half, out);
  if (half == 1) {
#pragma unroll
    for (int q = 0; q < 16; ++q) xch[row * XST + q] = out[q];
  }
  __syncthreads();
  if (half == 0) {
#pragma unroll
    for (int q = 0; q < 16; ++q) out[q] += xch[row * XST + q];
  }
}

// Splits 32 values into tf32 hi / lo and stores them as 32 A columns at `col`.
__device__ __forceinline__ void store_a32(uint32_t t_ahi, uint32_t t_alo, uint32_t col, const float* v) {
  uint32_t hi[32], lo[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) tc::split_tf32(v[i], hi[i], lo[i]);
  tc::tmem_st32(t_ahi + col, hi);
  tc::tmem_st32(t_alo + col, lo);
}

// Splits NC (8 or 16) values into tf32 hi / lo and stores them as NC A columns at `col`.
template <int NC>
__device__ __forceinline__ void store_a_n(uint32_t t_ahi, uint32_t t_alo, uint32_t col, const float* v) {
  static_assert(NC == 8 || NC == 16, "8 or 16 columns");
  uint32_t hi[NC], lo[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) tc::split_tf32(v[i], hi[i], lo[i]);
  if constexpr (NC == 8) {
    tc::tmem_st8(t_ahi + col, hi);
    tc::tmem_st8(t_alo + col, lo);
  } else {
    tc::tmem_st16(t_ahi + col, hi);
    tc::tmem_st16(t_alo + col, lo);
  }
}

// Hand-off from the CUDA-core phase to the MMA issuer: every thread's tcgen05.st is complete and
// ordered before the barrier.
__device__ __forceinline__ void a_ready() {
  tc::tmem_wait_st();
  tc::tc_fence_before();
  __syncthreads();
}

// Waits for the commit of the last MMA chain (all threads).  Returns false block-uniformly when
// the wait timed out anywhere in the block.
__device__ __forceinline__ bool d_ready(uint64_t* bar, uint32_t& phase, int* err, int where) {
  const bool ok = tc::mbar_wait(bar, phase, err, where);
  phase ^= 1u;
  tc::tc_fence_after();
  return !__syncthreads_or(!ok);
}

// After a timed-out wait: bounded wait for the chain still committed to `bar` before the TMEM
// it writes is released.
__device__ __forceinline__ void drain(uint64_t* bar, uint32_t phase) {
  const long long t0 = clock64();
  while (!tc::mbar_try_wait(bar, phase ^ 1u))
    if (clock64() - t0 > tc::kWaitCycles) return;
}

// ------------------------------------------------------------------ forward
// HOUT: stop after the second hidden layer and write h2 = silu(W2 h1 + b2) ([nint][E][64]) for
// callers that fold the last linear layer into their own contraction (pure-cartesian-sparse).
template <int NBP, bool HOUT>
__global__ void __launch_bounds__(RTH, RT_PER_SM) radial_fwd_tc_kernel(RadialTcArgs a) {
  using IM = FwdImg<NBP>;
  using SM = RtSmem<IM::SIZE>;
  extern __shared__ __align__(1024) uint8_t smem[];
  float* img_hi = reinterpret_cast<float*>(smem + SM::HI);
  float* img_lo = reinterpret_cast<float*>(smem + SM::LO);
  float* bias = reinterpret_cast<float*>(smem + SM::BIAS);
  float* xch = reinterpret_cast<float*>(smem + SM::XCH);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::BAR + 8);

  // thread = (column half, edge row); warps w and w + 4 read and write TMEM lanes 32 (w % 4) ...
  const int tid = threadIdx.x, warp = tid >> 5, half = tid / RT, row = tid % RT;
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
  const uint32_t tD0 = tbase, tD1 = tbase + 64u, tAhi = tbase + 128u, tAlo = tbase + 192u;
  const uint32_t hcol = 32u * half;  // this thread's hidden columns [hcol, hcol + 32)
  const uint32_t s_hi = tc::smem_u32(img_hi), s_lo = tc::smem_u32(img_lo);
  constexpr uint32_t id64 = tc::idesc_tf32(RT, 64), id16 = tc::idesc_tf32(RT, 16);
  const int64_t ntiles = (a.E + RT - 1) / RT;
  uint32_t phase = 0;
  bool ok = true;

  for (int layer = 0; layer < a.nint && ok; ++layer) {
    // ---- this layer's weights as B images
    __syncthreads();
    const float* w1 = a.rad.w1 + (size_t)layer * RH * a.nb;
    const float* w2 = a.rad.w2 + (size_t)layer * RH * RH;
    const float* w3 = a.rad.w3 + (size_t)layer * RP * RH;
    for (int i = tid; i < RH * NBP; i += RTH) {
      const int k = i / NBP, b = i - k * NBP;
      put_b(img_hi, img_lo, IM::W1, RH, k, b, b < a.nb ? w1[k * a.nb + b] : 0.f);
    }
    for (int i = tid; i < RH * RH; i += RTH) put_b(img_hi, img_lo, IM::W2, RH, i >> 6, i & 63, w2[i]);
    if (!HOUT) {
      for (int i = tid; i < 16 * RH; i += RTH) {
        const int q = i >> 6, j = i & 63;
        put_b(img_hi, img_lo, IM::W3, 16, q, j, q < RP ? w3[q * RH + j] : 0.f);
      }
    }
    load_bias(bias, a.rad, layer);
    fence_proxy_async_smem();
    __syncthreads();

    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t e = tile * RT + row;
      const bool valid = e < a.E;
      // ---- A = emb (columns [0, NBP), written by half 0; the MMA reads no further)
      if (half == 0) {
        float v[NBP];
#pragma unroll
        for (int i = 0; i < NBP; ++i) v[i] = 0.f;
        if (valid) {
          const float4 ry = reinterpret_cast<const float4*>(a.edge_y + 12 * e)[2];
          const float len = sqrtf(ry.y * ry.y + ry.z * ry.z + ry.w * ry.w);
          radial_basis<NBP>(a.basis_kind, a.nb, a.rc, len, v, nullptr);
        }
        store_a_n<NBP>(tAhi + lane_off, tAlo + lane_off, 0, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W1, s_lo + 4u * IM::W1, 64, NBP / 8, id64);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 41))) break;
      // ---- h1 = silu(D0 + b1) -> A ; D0 = h1 W2^T
      {
        uint32_t u[32];
        float v[32];
        tc::tmem_ld32(tD0 + lane_off + hcol, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = silu(__uint_as_float(u[i]) + bias[hcol + i]);
        store_a32(tAhi + lane_off, tAlo + lane_off, hcol, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W2, s_lo + 4u * IM::W2, 64, RH / 8, id64, 2, 64);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 42))) break;
      // ---- h2 = silu(D0 + D1 + b2) -> A ; D0..D1 = h2 W3^T (eight 16-column accumulators)
      {
        uint32_t u[32], w[32];
        float v[32];
        tc::tmem_ld32(tD0 + lane_off + hcol, u);
        tc::tmem_ld32(tD1 + lane_off + hcol, w);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = silu((__uint_as_float(u[i]) + __uint_as_float(w[i])) + bias[RH + hcol + i]);
        if (HOUT) {
          if (valid) {
            float4* o = reinterpret_cast<float4*>(a.hout + ((int64_t)layer * a.E + e) * RH + hcol);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        } else {
          store_a32(tAhi + lane_off, tAlo + lane_off, hcol, v);
        }
      }
      if (HOUT) {
        tc::tc_fence_before();
        continue;
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W3, s_lo + 4u * IM::W3, 16, RH / 8, id16, 8, 16);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 43))) break;
      // ---- gates = sum of the accumulators + b3
      {
        float gs[16];
        sum16x8_halves(tD0 + lane_off, half, row, xch, gs);
        if (half == 0 && valid) {
          float g[12];
#pragma unroll
          for (int q = 0; q < 12; ++q) g[q] = q < RP ? gs[q] + bias[2 * RH + q] : 0.f;
          float4* g4 = reinterpret_cast<float4*>(a.gates + ((int64_t)layer * a.E + e) * 12);
          g4[0] = make_float4(g[0], g[1], g[2], g[3]);
          g4[1] = make_float4(g[4], g[5], g[6], g[7]);
          g4[2] = make_float4(g[8], g[9], g[10], 0.f);
        }
      }
      tc::tc_fence_before();  // the next tile's tcgen05.st into A follows this tile's loads
    }
  }
  if (!ok && tid == 0) drain(bar, phase);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 256);
  }
}

// ------------------------------------------------------------------ backward
// HOUT: dE/dh2 comes from hout_grad ([nint][E][64]) instead of the gates, and every layer only
// accumulates dE/d|r| into edge_grad[e][0] (the caller adds the direction part).
template <int NBP, bool HOUT>
__global__ void __launch_bounds__(RTH, RT_PER_SM) radial_bwd_tc_kernel(RadialTcArgs a) {
  using IM = BwdImg<NBP>;
  using SM = RtSmem<IM::SIZE>;
  extern __shared__ __align__(1024) uint8_t smem[];
  float* img_hi = reinterpret_cast<float*>(smem + SM::HI);
  float* img_lo = reinterpret_cast<float*>(smem + SM::LO);
  float* bias = reinterpret_cast<float*>(smem + SM::BIAS);
  float* ypoly = reinterpret_cast<float*>(smem + SM::YPOLY);
  float* xch = reinterpret_cast<float*>(smem + SM::XCH);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::BAR + 8);

  // thread = (column half, edge row); warps w and w + 4 read and write TMEM lanes 32 (w % 4) ...
  const int tid = threadIdx.x, warp = tid >> 5, half = tid / RT, row = tid % RT;
  if (!HOUT)
    for (int i = tid; i < ictd2::NMONO * ictd2::NK; i += RTH) ypoly[i] = a.tables[ictd2::TAB_YPOLY + i];
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
  const uint32_t tD0 = tbase, tD1 = tbase + 64u, tAhi = tbase + 128u, tAlo = tbase + 192u;
  const uint32_t hcol = 32u * half;  // this thread's hidden columns [hcol, hcol + 32)
  const uint32_t s_hi = tc::smem_u32(img_hi), s_lo = tc::smem_u32(img_lo);
  constexpr uint32_t id64 = tc::idesc_tf32(RT, 64), id16 = tc::idesc_tf32(RT, 16);
  const int64_t ntiles = (a.E + RT - 1) / RT;
  uint32_t phase = 0;
  bool ok = true;

  for (int layer = 0; layer < a.nint && ok; ++layer) {
    __syncthreads();
    const float* w1 = a.rad.w1 + (size_t)layer * RH * a.nb;
    const float* w2 = a.rad.w2 + (size_t)layer * RH * RH;
    const float* w3 = a.rad.w3 + (size_t)layer * RP * RH;
    for (int i = tid; i < RH * NBP; i += RTH) {
      const int k = i / NBP, b = i - k * NBP;
      const float v = b < a.nb ? w1[k * a.nb + b] : 0.f;
      put_b(img_hi, img_lo, IM::W1, RH, k, b, v);
    }
    for (int i = tid; i < RH * 16; i += RTH) {  // W1T rows b < 16
      const int b = i >> 6, k = i & 63;
      put_b(img_hi, img_lo, IM::W1T, 16, b, k, b < a.nb ? w1[k * a.nb + b] : 0.f);
    }
    for (int i = tid; i < RH * RH; i += RTH) {
      const int j = i >> 6, k = i & 63;
      put_b(img_hi, img_lo, IM::W2, RH, j, k, w2[i]);
      put_b(img_hi, img_lo, IM::W2T, RH, k, j, w2[i]);
    }
    if (!HOUT) {
      for (int i = tid; i < RH * 16; i += RTH) {
        const int j = i >> 4, q = i & 15;
        put_b(img_hi, img_lo, IM::W3P, RH, j, q, q < RP ? w3[q * RH + j] : 0.f);
      }
    }
    load_bias(bias, a.rad, layer);
    fence_proxy_async_smem();
    __syncthreads();

    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t e = tile * RT + row;
      const bool valid = e < a.E;
      float demb[NBP];  // half 0
      float ry[3] = {0.f, 0.f, 0.f};
      // ---- A = [emb (NBP, half 0) | dgates (16, half 1)] ; D0 = emb W1^T (a1 - b1), D1 = dg W3 (dh2)
      if (half == 0) {
        float v[NBP];
#pragma unroll
        for (int i = 0; i < NBP; ++i) v[i] = 0.f;
#pragma unroll
        for (int b = 0; b < NBP; ++b) demb[b] = 0.f;
        if (valid) {
          const float4 r4 = reinterpret_cast<const float4*>(a.edge_y + 12 * e)[2];
          ry[0] = r4.y; ry[1] = r4.z; ry[2] = r4.w;
          const float len = sqrtf(r4.y * r4.y + r4.z * r4.z + r4.w * r4.w);
          radial_basis<NBP>(a.basis_kind, a.nb, a.rc, len, v, demb);
        }
        store_a_n<NBP>(tAhi + lane_off, tAlo + lane_off, 0, v);
      } else if (!HOUT) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        if (valid) {
          const float4* dg4 = reinterpret_cast<const float4*>(a.dgates + ((int64_t)layer * a.E + e) * 12);
          const float4 g0 = dg4[0], g1 = dg4[1], g2 = dg4[2];
          v[0] = g0.x; v[1] = g0.y; v[2] = g0.z; v[3] = g0.w;
          v[4] = g1.x; v[5] = g1.y; v[6] = g1.z; v[7] = g1.w;
          v[8] = g2.x; v[9] = g2.y; v[10] = g2.z;
        }
        store_a_n<16>(tAhi + lane_off, tAlo + lane_off, NBP, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W1, s_lo + 4u * IM::W1, 64, NBP / 8, id64);
        if (!HOUT)
          mma_3xtf32(tD1, tAhi + NBP, tAlo + NBP, s_hi + 4u * IM::W3P, s_lo + 4u * IM::W3P, 64, 2, id64);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 51))) break;
      // ---- h1 = silu(a1) -> A, keep silu'(a1) ; D0 = h1 W2^T (a2 - b2)
      float sg1[32];
      {
        uint32_t u[32];
        float v[32];
        tc::tmem_ld32(tD0 + lane_off + hcol, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = __uint_as_float(u[i]) + bias[hcol + i];
          v[i] = silu(x);
          sg1[i] = silu_grad(x);
        }
        store_a32(tAhi + lane_off, tAlo + lane_off, hcol, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W2, s_lo + 4u * IM::W2, 64, RH / 8, id64);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 52))) break;
      // ---- da2 = dh2 * silu'(a2) -> A ; D0 = da2 W2 (dh1)
      {
        uint32_t u[32], w[32];
        float v[32];
        tc::tmem_ld32(tD0 + lane_off + hcol, u);
        if (!HOUT) tc::tmem_ld32(tD1 + lane_off + hcol, w);
        tc::tmem_wait_ld();
        if (HOUT) {
          const float4* g4 = reinterpret_cast<const float4*>(a.hout_grad + ((int64_t)layer * a.E + e) * RH + hcol);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 t = valid ? g4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            w[4 * i] = __float_as_uint(t.x); w[4 * i + 1] = __float_as_uint(t.y);
            w[4 * i + 2] = __float_as_uint(t.z); w[4 * i + 3] = __float_as_uint(t.w);
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(w[i]) * silu_grad(__uint_as_float(u[i]) + bias[RH + hcol + i]);
        store_a32(tAhi + lane_off, tAlo + lane_off, hcol, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W2T, s_lo + 4u * IM::W2T, 64, RH / 8, id64, 2, 64);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 53))) break;
      // ---- da1 = (D0 + D1) * silu'(a1) -> A ; D0..D1 = da1 W1 (dE/demb, eight accumulators)
      {
        uint32_t u[32], w[32];
        float v[32];
        tc::tmem_ld32(tD0 + lane_off + hcol, u);
        tc::tmem_ld32(tD1 + lane_off + hcol, w);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = (__uint_as_float(u[i]) + __uint_as_float(w[i])) * sg1[i];
        store_a32(tAhi + lane_off, tAlo + lane_off, hcol, v);
      }
      a_ready();
      if (tid == 0) {
        tc::tc_fence_after();
        mma_3xtf32(tD0, tAhi, tAlo, s_hi + 4u * IM::W1T, s_lo + 4u * IM::W1T, 16, RH / 8, id16, 8, 16);
        tc::mma_commit(bar);
      }
      if (!(ok = d_ready(bar, phase, a.err, 54))) break;
      // ---- dE/d|r| of this layer; the last layer also applies the direction part (half 0)
      {
        float de[16];
        sum16x8_halves(tD0 + lane_off, half, row, xch, de);
        if (half == 0 && valid) {
          float dl = 0.f;
#pragma unroll
          for (int b = 0; b < NBP; ++b) dl = fmaf(de[b], demb[b], dl);
          float* eg = a.edge_grad + 3 * e;
          if (layer > 0) dl += eg[0];
          if (HOUT || layer + 1 < a.nint) {
            eg[0] = dl;
          } else {
            float dYe[ictd2::NK], g[3];
            const float4* d4 = reinterpret_cast<const float4*>(a.dY + 12 * e);
            const float4 d0 = d4[0], d1 = d4[1], d2 = d4[2];
            dYe[0] = d0.x; dYe[1] = d0.y; dYe[2] = d0.z; dYe[3] = d0.w;
            dYe[4] = d1.x; dYe[5] = d1.y; dYe[6] = d1.z; dYe[7] = d1.w; dYe[8] = d2.x;
            edge_direction_grad(ypoly, ry[0], ry[1], ry[2], dYe, dl, g);
            eg[0] = g[0]; eg[1] = g[1]; eg[2] = g[2];
          }
        }
      }
      tc::tc_fence_before();
    }
  }
  if (!ok && tid == 0) drain(bar, phase);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 256);
  }
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <typename K>
int launch_rt(K kernel, uint32_t smem, const RadialTcArgs& a, cudaStream_t st, const char* name) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(FSC_ERR_CUDA, std::string(name) + ": cannot set shared memory size");
  const int64_t ntiles = ceil_div(a.E, RT);
  const int64_t grid = ntiles < (int64_t)RT_PER_SM * num_sms() ? ntiles : (int64_t)RT_PER_SM * num_sms();
  kernel<<<(unsigned)grid, RTH, smem, st>>>(a);
  return check_launch(name);
}

}  // namespace

bool radial_tc_supported(int nb) { return nb >= 1 && nb <= 16; }

int launch_radial_fwd_tc(const RadialTcArgs& a, cudaStream_t st) {
  if (a.E == 0) return FSC_OK;
  if (!radial_tc_supported(a.nb)) return fail(FSC_ERR_UNSUPPORTED, "radial_fwd_tc: number_of_basis must be 1..16");
  if (a.hout) {
    if (a.nb <= 8)
      return launch_rt(radial_fwd_tc_kernel<8, true>, RtSmem<FwdImg<8>::SIZE>::TOTAL, a, st, "radial_fwd_tc_kernel<8,h>");
    return launch_rt(radial_fwd_tc_kernel<16, true>, RtSmem<FwdImg<16>::SIZE>::TOTAL, a, st,
                     "radial_fwd_tc_kernel<16,h>");
  }
  if (a.nb <= 8)
    return launch_rt(radial_fwd_tc_kernel<8, false>, RtSmem<FwdImg<8>::SIZE>::TOTAL, a, st, "radial_fwd_tc_kernel<8>");
  return launch_rt(radial_fwd_tc_kernel<16, false>, RtSmem<FwdImg<16>::SIZE>::TOTAL, a, st, "radial_fwd_tc_kernel<16>");
}

int launch_radial_bwd_tc(const RadialTcArgs& a, cudaStream_t st) {
  if (a.E == 0) return FSC_OK;
  if (!radial_tc_supported(a.nb)) return fail(FSC_ERR_UNSUPPORTED, "radial_bwd_tc: number_of_basis must be 1..16");
  if (a.hout_grad) {
    if (a.nb <= 8)
      return launch_rt(radial_bwd_tc_kernel<8, true>, RtSmem<BwdImg<8>::SIZE>::TOTAL, a, st, "radial_bwd_tc_kernel<8,h>");
    return launch_rt(radial_bwd_tc_kernel<16, true>, RtSmem<BwdImg<16>::SIZE>::TOTAL, a, st,
                     "radial_bwd_tc_kernel<16,h>");
  }
  if (a.nb <= 8)
    return launch_rt(radial_bwd_tc_kernel<8, false>, RtSmem<BwdImg<8>::SIZE>::TOTAL, a, st, "radial_bwd_tc_kernel<8>");
  return launch_rt(radial_bwd_tc_kernel<16, false>, RtSmem<BwdImg<16>::SIZE>::TOTAL, a, st, "radial_bwd_tc_kernel<16>");
}

}  // namespace fsc
