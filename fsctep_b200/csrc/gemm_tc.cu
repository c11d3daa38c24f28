// Channel-mixing and MainNet GEMMs on the 5th-generation tensor cores (TMA, tcgen05, TMEM).
//
//   C[row, n] (+)= scale(row) * sum_k A[row, k] B[k, n] (+ bias[n]),  rows (g, r): g < G, r < R,
//   A row (g, r) at A + g*a_gs + r*a_rs (K contiguous), C row at C + g*c_gs + r*c_rs.
//
// One CTA = 128 rows (the TMEM lanes; Gb = 128 / R whole row groups) x NT output columns.
//  * producer warp: per K-chunk of 32, one 3-D TMA load of the A tile (dims K, R, G: the two-level
//    row addressing needs no copy; 128-byte swizzle, so each row is one swizzle row) and one bulk
//    copy of the B chunk from a pre-formatted image, into a shared-memory ring;
//  * 4 math warps: split the staged A in place into tf32 hi = round_tf32(a) and write lo =
//    round_tf32(a - hi) to a second buffer of the same layout (elementwise, so the swizzle needs
//    no decoding); after the last chunk they read the accumulators and write C;
//  * MMA warp: per chunk the 8 small products (hi*lo, lo*hi of 4 K-steps) and then the 4 hi*hi
//    kind::tf32 MMAs (A and B from shared memory): the small terms accumulate before the large
//    ones, so they are not truncated against the full magnitude (tensor-core accumulation rounds
//    toward zero); no accumulator carries a long chain (see GCfg).
// B images (hi / lo planes, K-major, no swizzle) are built from the weights by gemm_image_kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace fsc {

namespace {

constexpr int KC = 32;                      // K per chunk: one 128-byte row per A row
constexpr int MT = 128;                     // rows per tile
constexpr uint32_t ABYTES = MT * KC * 4u;   // 16 KB
constexpr int GT_THREADS = 6 * 32;          // 4 math warps, producer warp, MMA warp

// NT <= 128 (FLUSH): every group of GC K-chunks (12 GC MMAs) accumulates into a fresh one of two
// TMEM slots, which the math warps add to fp32 registers (tensor-core accumulation truncates, so
// long chains over large K would bias the result).  PRECISE (long K with heavy cancellation, e.g.
// the readout's Gram contraction): a fresh slot every chunk (12 MMAs, 4 of them hi*hi).  Wider
// tiles (gemm_tc_nt gives them only for K <= 128) rotate the chunks over NACC accumulators summed
// in the epilogue.
template <int NT, bool PRECISE = false>
struct GCfg {
  static constexpr bool FLUSH = NT <= 128;
  static constexpr int GC = PRECISE ? 1 : 2;
  static constexpr int NACC = FLUSH ? 2 : 2;
  // shared-memory ring depth: NT = 128 runs one CTA per SM and has room for a third stage;
  // NT = 64 keeps two stages so that two CTAs share an SM
  static constexpr int NST = NT == 128 ? 3 : 2;
  static constexpr uint32_t BBYTES = 2u * KC * NT * 4u;  // hi + lo planes of one chunk
  static constexpr uint32_t ALO_OFF = NST * ABYTES;
  static constexpr uint32_t B_OFF = 2 * NST * ABYTES;
  static constexpr uint32_t BAR_OFF = B_OFF + NST * BBYTES;
  static constexpr uint32_t TOTAL = BAR_OFF + 128 + 1024;  // + slack for 1024-byte alignment
  static constexpr uint32_t TCOLS = NT * NACC <= 256 ? 256 : 512;
};

// K-major, 128-byte swizzle smem descriptor: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(tc::smem_u32(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(tc::smem_u32(bar))
      : "memory");
}

struct GemmTcArgs {
  const float* bimg;       // [ntiles][K/KC][2][KC/4][NT][4]
  int K, N;
  int64_t G;
  int R, Gb;
  uint32_t abox;           // bytes of one A box: KC * R * Gb * 4
  float* C;
  int64_t c_gs, c_rs;
  const int32_t* deg_rowptr;
  const float* bias;
  int accumulate;
  float alpha;
  int* err;
};

template <int NT, bool PRECISE>
__global__ void __launch_bounds__(GT_THREADS) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, GemmTcArgs a) {
  using CF = GCfg<NT, PRECISE>;
  constexpr int NST = CF::NST, NACC = CF::NACC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sAlo = smem + CF::ALO_OFF;
  uint8_t* sB = smem + CF::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::BAR_OFF);
  uint64_t* full = bars;                  // [NST] TMA + bulk bytes landed
  uint64_t* lo_ready = bars + NST;        // [NST] math warps split the chunk
  uint64_t* empty = bars + 2 * NST;       // [NST] MMAs done with the stage
  uint64_t* d_ready = bars + 3 * NST;     // all MMAs done
  uint64_t* grp_full = bars + 3 * NST + 1;   // [2] FLUSH: a group's MMAs done
  uint64_t* grp_empty = bars + 3 * NST + 3;  // [2] FLUSH: math warps read the slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * NST + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = (a.K + KC - 1) / KC;  // a K tail reads TMA zero fill and zero image rows
  const int64_t g0 = (int64_t)blockIdx.x * a.Gb;

  if (warp == 4) {
    tc::tmem_alloc(tmem_slot, CF::TCOLS);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      tc::mbar_init(full + i, 1);
      tc::mbar_init(lo_ready + i, 4);
      tc::mbar_init(empty + i, 1);
    }
    tc::mbar_init(d_ready, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(grp_full + i, 1);
      tc::mbar_init(grp_empty + i, 4);
    }
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int ngroups = (nchunks + CF::GC - 1) / CF::GC;

  if (warp < 4) {
    // ---------------- split A into tf32 hi (in place) and lo, per chunk
    bool ok = true;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float sum[CF::FLUSH ? NT : 1];
#pragma unroll
    for (int i = 0; i < (CF::FLUSH ? NT : 1); ++i) sum[i] = 0.f;
    auto flush = [&](int g) {  // FLUSH: add group g's slot to the fp32 sums and free it
      const int slot = g & 1;
      if (!(ok = tc::mbar_wait(grp_full + slot, (g >> 1) & 1, a.err, 86))) return;
      tc::tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < (CF::FLUSH ? NT / 16 : 0); ++cb) {
        uint32_t u[16];
        tc::tmem_ld16(tbase + (uint32_t)(slot * NT) + lane_off + 16u * cb, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[16 * cb + i] += __uint_as_float(u[i]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(grp_empty + slot);
    };
    for (int c = 0; c < nchunks && ok; ++c) {
      const int st = c % NST;
      if (!(ok = tc::mbar_wait(full + st, (c / NST) & 1, a.err, 81))) break;
      float4* pa = reinterpret_cast<float4*>(sA + st * ABYTES);
      float4* pl = reinterpret_cast<float4*>(sAlo + st * ABYTES);
#pragma unroll
      for (int i = 0; i < (int)(ABYTES / 16) / MT; ++i) {
        const int idx = threadIdx.x + MT * i;
        float4 v = pa[idx];
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
        tc::split_tf32(v.x, h0, l0);
        tc::split_tf32(v.y, h1, l1);
        tc::split_tf32(v.z, h2, l2);
        tc::split_tf32(v.w, h3, l3);
        pa[idx] = make_float4(__uint_as_float(h0), __uint_as_float(h1), __uint_as_float(h2), __uint_as_float(h3));
        pl[idx] = make_float4(__uint_as_float(l0), __uint_as_float(l1), __uint_as_float(l2), __uint_as_float(l3));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(lo_ready + st);
      if (CF::FLUSH && (c % CF::GC == CF::GC - 1 || c == nchunks - 1) && c / CF::GC >= 1) flush(c / CF::GC - 1);
    }
    if (CF::FLUSH && ok) flush(ngroups - 1);
    // ---------------- epilogue: thread = tile row = TMEM lane
    if (ok) ok = tc::mbar_wait(d_ready, 0, a.err, 82);
    tc::tc_fence_after();
    const int t = warp * 32 + lane;
    const int64_t g = g0 + t / a.R;
    const int r = t % a.R;
    const bool valid = ok && t < a.R * a.Gb && g < a.G;
    float scale = a.alpha != 0.f ? a.alpha : 1.f;
    if (valid && a.deg_rowptr) {
      const int d = a.deg_rowptr[g + 1] - a.deg_rowptr[g];
      scale *= 1.f / (float)(d > 1 ? d : 1);
    }
    float* crow = valid ? a.C + g * a.c_gs + r * a.c_rs : nullptr;
    const int n0 = blockIdx.y * NT;
    const int nacc = nchunks < NACC ? nchunks : NACC;
#pragma unroll
    for (int cb = 0; cb < NT / 16; ++cb) {
      float v[16];
      if (CF::FLUSH) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = sum[(CF::FLUSH ? 16 * cb + i : 0)];
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        for (int q = 0; q < nacc; ++q) {
          uint32_t u[16];
          tc::tmem_ld16(tbase + (uint32_t)(q * NT) + lane_off + 16u * cb, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += __uint_as_float(u[i]);
        }
      }
      const int nc = n0 + 16 * cb;
      if (crow && nc < a.N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] *= scale;
          if (a.bias && nc + i < a.N) v[i] += a.bias[nc + i];
        }
        float* cp = crow + nc;
        if (nc + 16 <= a.N && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
          float4* c4 = reinterpret_cast<float4*>(cp);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if (a.accumulate) {
              const float4 p = c4[i];
              o.x += p.x;
              o.y += p.y;
              o.z += p.z;
              o.w += p.w;
            }
            c4[i] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (nc + i < a.N) cp[i] = a.accumulate ? cp[i] + v[i] : v[i];
        }
      }
    }
  } else if (warp == 4) {
    // ---------------- producer
    if (lane == 0) {
      const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(a.bimg) + (size_t)blockIdx.y * nchunks * CF::BBYTES;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % NST;
        if (c >= NST && !tc::mbar_wait(empty + st, ((c / NST) - 1) & 1, a.err, 83)) break;
        tc::mbar_arrive_expect_tx(full + st, a.abox + CF::BBYTES);
        tma_load_3d(sA + st * ABYTES, &tmA, c * KC, 0, (int)g0, full + st);
        tc::bulk_g2s(sB + st * CF::BBYTES, bsrc + (size_t)c * CF::BBYTES, CF::BBYTES, full + st);
      }
    }
  } else {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(MT, NT);
      const uint32_t a0 = tc::smem_u32(sA), l0 = tc::smem_u32(sAlo), b0 = tc::smem_u32(sB);
      bool ok = true;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % NST;
        if (!(ok = tc::mbar_wait(lo_ready + st, (c / NST) & 1, a.err, 84))) break;
        const int g = c / CF::GC;
        const bool first = CF::FLUSH ? c % CF::GC == 0 : c < NACC;
        if (CF::FLUSH && first && g >= 2 && !(ok = tc::mbar_wait(grp_empty + (g & 1), ((g >> 1) - 1) & 1, a.err, 87)))
          break;
        tc::tc_fence_after();
        const uint32_t d = tbase + (uint32_t)((CF::FLUSH ? (g & 1) : (c % NACC)) * NT);
#pragma unroll
        for (int j = 0; j < KC / 8; ++j) {  // small products first
          const uint64_t ah = desc_sw128(a0 + st * ABYTES + 32 * j);
          const uint64_t al = desc_sw128(l0 + st * ABYTES + 32 * j);
          const uint32_t bh_addr = b0 + st * CF::BBYTES + j * 2 * 16 * NT;
          const uint64_t bh = tc::smem_desc_kmajor(bh_addr, 16 * NT, 128);
          const uint64_t bl = tc::smem_desc_kmajor(bh_addr + CF::BBYTES / 2, 16 * NT, 128);
          mma_tf32_ss(d, ah, bl, idesc, (!first || j > 0) ? 1u : 0u);
          mma_tf32_ss(d, al, bh, idesc, 1u);
        }
#pragma unroll
        for (int j = 0; j < KC / 8; ++j) {
          const uint64_t ah = desc_sw128(a0 + st * ABYTES + 32 * j);
          const uint64_t bh = tc::smem_desc_kmajor(b0 + st * CF::BBYTES + j * 2 * 16 * NT, 16 * NT, 128);
          mma_tf32_ss(d, ah, bh, idesc, 1u);
        }
        tc::mma_commit(empty + st);
        if (CF::FLUSH && (c % CF::GC == CF::GC - 1 || c == nchunks - 1)) tc::mma_commit(grp_full + (g & 1));
      }
      tc::mma_commit(d_ready);  // also when a wait failed: whatever was issued completes first
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    // the MMA warp commits d_ready on every path: wait (bounded) until no MMA still writes TMEM
    if (lane == 0) tc::mbar_wait(d_ready, 0, a.err, 85);
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, CF::TCOLS);
  }
}

// ------------------------------------------------------------------ streaming, A split into TMEM
// The same product for NT <= 128 with the A operand in tensor memory: the math warps read the
// staged A tile (thread = tile row = TMEM lane; the 128-byte swizzle is undone by XOR-ing the
// 16-byte chunk index with the row), split it into tf32 hi / lo straight into one of NAB TMEM
// A buffers (64 columns each), and the MMAs read A from TMEM and B from shared memory.  No hi / lo
// copy of A is written back to shared memory, so a stage holds only the raw A tile and the B
// chunk: four stages for NT = 128 (one CTA per SM, all 512 TMEM columns), three for NT = 64 (two
// CTAs per SM, 256 columns each).  Accumulation as in gemm_tc_kernel (FLUSH groups of GC chunks).
template <int NT, bool PRECISE = false>
struct GmCfg {
  static_assert(NT == 64 || NT == 128, "A-in-TMEM tiles");
  static constexpr int GC = PRECISE ? 1 : 2;
  static constexpr int NST = NT == 128 ? 4 : 3;
  static constexpr int NAB = NT == 128 ? 4 : 2;
  static constexpr uint32_t TCOLS = NT == 128 ? 512 : 256;
  static constexpr uint32_t ACOL = 2 * NT;                 // A buffers after the two D slots
  static constexpr uint32_t BBYTES = 2u * KC * NT * 4u;
  static constexpr uint32_t B_OFF = NST * ABYTES;
  static constexpr uint32_t BAR_OFF = B_OFF + NST * BBYTES;
  static constexpr uint32_t TOTAL = BAR_OFF + 256 + 1024;  // + slack for 1024-byte alignment
};
static_assert(GmCfg<128>::ACOL + 64 * GmCfg<128>::NAB <= GmCfg<128>::TCOLS, "TMEM plan");
static_assert(GmCfg<64>::ACOL + 64 * GmCfg<64>::NAB <= GmCfg<64>::TCOLS, "TMEM plan");
static_assert(GmCfg<128>::TOTAL <= 227u * 1024u && GmCfg<128>::TOTAL > 114u * 1024u, "one CTA per SM at NT = 128");
static_assert(2u * (GmCfg<64>::TOTAL + 1024u) <= 228u * 1024u, "two CTAs per SM at NT = 64");
static_assert(2 * GmCfg<64, true>::NST + 2 * GmCfg<64, true>::NAB + 5 <= 31, "barrier space");

template <int NT, bool PRECISE>
__global__ void __launch_bounds__(GT_THREADS) gemm_tcm_kernel(const __grid_constant__ CUtensorMap tmA, GemmTcArgs a) {
  using CF = GmCfg<NT, PRECISE>;
  constexpr int NST = CF::NST, NAB = CF::NAB, GC = CF::GC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + CF::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CF::BAR_OFF);
  uint64_t* full = bars;                         // [NST] TMA + bulk bytes landed
  uint64_t* empty = bars + NST;                  // [NST] MMAs done with the stage
  uint64_t* a_ready = bars + 2 * NST;            // [NAB] math warps split the chunk into the buffer
  uint64_t* a_free = bars + 2 * NST + NAB;       // [NAB] MMAs done with the buffer
  uint64_t* d_ready = bars + 2 * NST + 2 * NAB;  // all MMAs done
  uint64_t* grp_full = d_ready + 1;              // [2] a group's MMAs done
  uint64_t* grp_empty = d_ready + 3;             // [2] math warps read the slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_ready + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = (a.K + KC - 1) / KC;  // a K tail reads TMA zero fill and zero image rows
  const int64_t g0 = (int64_t)blockIdx.x * a.Gb;

  if (warp == 4) {
    tc::tmem_alloc(tmem_slot, CF::TCOLS);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      tc::mbar_init(full + i, 1);
      tc::mbar_init(empty + i, 1);
    }
    for (int i = 0; i < NAB; ++i) {
      tc::mbar_init(a_ready + i, 4);
      tc::mbar_init(a_free + i, 1);
    }
    tc::mbar_init(d_ready, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(grp_full + i, 1);
      tc::mbar_init(grp_empty + i, 4);
    }
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int ngroups = (nchunks + GC - 1) / GC;

  if (warp < 4) {
    // ---------------- split the staged A rows into TMEM (thread = row = lane), flush groups
    bool ok = true;
    const int t = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float sum[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) sum[i] = 0.f;
    auto flush = [&](int g) {  // add group g's slot to the fp32 sums and free it
      const int slot = g & 1;
      if (!(ok = tc::mbar_wait(grp_full + slot, (g >> 1) & 1, a.err, 86))) return;
      tc::tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < NT / 16; ++cb) {
        uint32_t u[16];
        tc::tmem_ld16(tbase + (uint32_t)(slot * NT) + lane_off + 16u * cb, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[16 * cb + i] += __uint_as_float(u[i]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(grp_empty + slot);
    };
    for (int c = 0; c < nchunks && ok; ++c) {
      const int st = c % NST, ab = c % NAB;
      if (!(ok = tc::mbar_wait(full + st, (c / NST) & 1, a.err, 81))) break;
      if (c >= NAB && !(ok = tc::mbar_wait(a_free + ab, ((c / NAB) - 1) & 1, a.err, 88))) break;
      const uint8_t* row = sA + st * ABYTES + t * 128;
      const uint32_t tA = tbase + CF::ACOL + 64u * (uint32_t)ab + lane_off;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = 4 * h + q;  // 16-byte chunk of the 128-byte row (4 K values)
          const float4 v = *reinterpret_cast<const float4*>(row + ((j ^ (t & 7)) << 4));
          tc::split_tf32(v.x, hi[4 * q], lo[4 * q]);
          tc::split_tf32(v.y, hi[4 * q + 1], lo[4 * q + 1]);
          tc::split_tf32(v.z, hi[4 * q + 2], lo[4 * q + 2]);
          tc::split_tf32(v.w, hi[4 * q + 3], lo[4 * q + 3]);
        }
        tc::tmem_st16(tA + 16u * h, hi);
        tc::tmem_st16(tA + 32u + 16u * h, lo);
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(a_ready + ab);
      if ((c % GC == GC - 1 || c == nchunks - 1) && c / GC >= 1) flush(c / GC - 1);
    }
    if (ok) flush(ngroups - 1);
    // ---------------- epilogue: thread = tile row = TMEM lane
    if (ok) ok = tc::mbar_wait(d_ready, 0, a.err, 82);
    tc::tc_fence_after();
    const int64_t g = g0 + t / a.R;
    const int r = t % a.R;
    const bool valid = ok && t < a.R * a.Gb && g < a.G;
    float scale = a.alpha != 0.f ? a.alpha : 1.f;
    if (valid && a.deg_rowptr) {
      const int d = a.deg_rowptr[g + 1] - a.deg_rowptr[g];
      scale *= 1.f / (float)(d > 1 ? d : 1);
    }
    float* crow = valid ? a.C + g * a.c_gs + r * a.c_rs : nullptr;
    const int n0 = blockIdx.y * NT;
#pragma unroll
    for (int cb = 0; cb < NT / 16; ++cb) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = sum[16 * cb + i];
      const int nc = n0 + 16 * cb;
      if (crow && nc < a.N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] *= scale;
          if (a.bias && nc + i < a.N) v[i] += a.bias[nc + i];
        }
        float* cp = crow + nc;
        if (nc + 16 <= a.N && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
          float4* c4 = reinterpret_cast<float4*>(cp);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if (a.accumulate) {
              const float4 p = c4[i];
              o.x += p.x;
              o.y += p.y;
              o.z += p.z;
              o.w += p.w;
            }
            c4[i] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (nc + i < a.N) cp[i] = a.accumulate ? cp[i] + v[i] : v[i];
        }
      }
    }
  } else if (warp == 4) {
    // ---------------- producer
    if (lane == 0) {
      const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(a.bimg) + (size_t)blockIdx.y * nchunks * CF::BBYTES;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % NST;
        if (c >= NST && !tc::mbar_wait(empty + st, ((c / NST) - 1) & 1, a.err, 83)) break;
        tc::mbar_arrive_expect_tx(full + st, a.abox + CF::BBYTES);
        tma_load_3d(sA + st * ABYTES, &tmA, c * KC, 0, (int)g0, full + st);
        tc::bulk_g2s(sB + st * CF::BBYTES, bsrc + (size_t)c * CF::BBYTES, CF::BBYTES, full + st);
      }
    }
  } else {
    // ---------------- MMA issuer: A from TMEM, B from shared memory
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(MT, NT);
      const uint32_t b0 = tc::smem_u32(sB);
      bool ok = true;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % NST, ab = c % NAB;
        if (!(ok = tc::mbar_wait(a_ready + ab, (c / NAB) & 1, a.err, 84))) break;
        const int g = c / GC;
        const bool first = c % GC == 0;
        if (first && g >= 2 && !(ok = tc::mbar_wait(grp_empty + (g & 1), ((g >> 1) - 1) & 1, a.err, 87))) break;
        tc::tc_fence_after();
        const uint32_t d = tbase + (uint32_t)((g & 1) * NT);
        const uint32_t tA = tbase + CF::ACOL + 64u * (uint32_t)ab;
#pragma unroll
        for (int j = 0; j < KC / 8; ++j) {  // small products first
          const uint32_t bh_addr = b0 + st * CF::BBYTES + j * 2 * 16 * NT;
          const uint64_t bh = tc::smem_desc_kmajor(bh_addr, 16 * NT, 128);
          const uint64_t bl = tc::smem_desc_kmajor(bh_addr + CF::BBYTES / 2, 16 * NT, 128);
          tc::mma_tf32_ts(d, tA + 8u * j, bl, idesc, (!first || j > 0) ? 1u : 0u);
          tc::mma_tf32_ts(d, tA + 32u + 8u * j, bh, idesc, 1u);
        }
#pragma unroll
        for (int j = 0; j < KC / 8; ++j) {
          const uint64_t bh = tc::smem_desc_kmajor(b0 + st * CF::BBYTES + j * 2 * 16 * NT, 16 * NT, 128);
          tc::mma_tf32_ts(d, tA + 8u * j, bh, idesc, 1u);
        }
        tc::mma_commit(empty + st);
        tc::mma_commit(a_free + ab);
        if (c % GC == GC - 1 || c == nchunks - 1) tc::mma_commit(grp_full + (g & 1));
      }
      tc::mma_commit(d_ready);  // also when a wait failed: whatever was issued completes first
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    // the MMA warp commits d_ready on every path: wait (bounded) until no MMA still writes TMEM
    if (lane == 0) tc::mbar_wait(d_ready, 0, a.err, 85);
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, CF::TCOLS);
  }
}

// ------------------------------------------------------------------ persistent, B resident
// For short K and N <= 256 (the dZ channel mix and the MainNet layers here) the whole B image
// fits in shared memory: one CTA per SM loads it once and walks row tiles.  Roles: producer warp (B once,
// then A chunks by TMA into an NST-stage ring), 4 split warps (tf32 hi in place + lo), MMA warp,
// 4 epilogue warps (thread = row = TMEM lane).  Two TMEM slots of 256 columns let tile i's
// epilogue run under tile i + 1's loads and MMAs.  Within a slot, chunk group a (GC <= 2 chunks,
// <= 24 MMAs) accumulates at column a * NT; the epilogue sums the groups in fp32.
constexpr int TP_THREADS = 10 * 32;         // split 0-3, epilogue 4-7, producer 8, MMA 9
constexpr uint32_t TP_BMAX = 128u * 1024u;  // B image bytes held in shared memory

template <int NT>
struct TpCfg {
  static constexpr int NACC_MAX = 256 / NT;               // chunk groups per TMEM slot
  static constexpr uint32_t BBYTES = 2u * KC * NT * 4u;   // one chunk's hi + lo planes
  static constexpr uint32_t RING = 2u * ABYTES;           // one stage: A hi + A lo
};

struct TpShape {
  int nchunks, nst, gc;
  uint32_t b_off, bar_off, total;
};

template <int NT>
__host__ __device__ inline TpShape tp_shape(int K) {
  TpShape sh{};
  sh.nchunks = (K + KC - 1) / KC;
  const int nacc = sh.nchunks < TpCfg<NT>::NACC_MAX ? sh.nchunks : TpCfg<NT>::NACC_MAX;
  sh.gc = (sh.nchunks + nacc - 1) / nacc;
  const uint32_t bbytes = (uint32_t)sh.nchunks * TpCfg<NT>::BBYTES;
  sh.nst = bbytes + 4u * TpCfg<NT>::RING <= 200u * 1024u ? 4 : 2;
  sh.b_off = (uint32_t)sh.nst * TpCfg<NT>::RING;
  sh.bar_off = sh.b_off + bbytes;
  const uint32_t raw = sh.bar_off + 256u + 1024u;  // barriers, TMEM slot, 1024-byte alignment slack
  sh.total = raw < 120u * 1024u ? 120u * 1024u : raw;  // one CTA per SM (512 TMEM columns)
  return sh;
}

template <int NT>
__global__ void __launch_bounds__(TP_THREADS, 1) gemm_tcp_kernel(const __grid_constant__ CUtensorMap tmA, GemmTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TpShape sh = tp_shape<NT>(a.K);
  const int NST = sh.nst, nchunks = sh.nchunks, GC = sh.gc;
  uint8_t* sB = smem + sh.b_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sh.bar_off);
  uint64_t* full = bars;                 // [NST] A chunk landed
  uint64_t* lo_ready = bars + 4;         // [NST] split done
  uint64_t* empty = bars + 8;            // [NST] MMAs done with the stage
  uint64_t* acc_full = bars + 12;        // [2] a tile's MMAs done
  uint64_t* acc_empty = bars + 14;       // [2] epilogue done with the slot
  uint64_t* b_full = bars + 16;          // B image landed
  uint64_t* done = bars + 17;            // every MMA issued by this CTA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (a.G + a.Gb - 1) / a.Gb;

  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      tc::mbar_init(full + i, 1);
      tc::mbar_init(lo_ready + i, 4);
      tc::mbar_init(empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(acc_full + i, 1);
      tc::mbar_init(acc_empty + i, 4);
    }
    tc::mbar_init(b_full, 1);
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp < 4) {
    // ---------------- split A chunks into tf32 hi (in place) and lo
    int64_t q = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      bool ok = true;
      for (int c = 0; c < nchunks; ++c, ++q) {
        const int st = (int)(q % NST);
        if (!(ok = tc::mbar_wait(full + st, (uint32_t)((q / NST) & 1), a.err, 91))) break;
        float4* pa = reinterpret_cast<float4*>(smem + st * TpCfg<NT>::RING);
        float4* pl = reinterpret_cast<float4*>(smem + st * TpCfg<NT>::RING + ABYTES);
#pragma unroll
        for (int i = 0; i < (int)(ABYTES / 16) / MT; ++i) {
          const int idx = threadIdx.x + MT * i;
          const float4 v = pa[idx];
          uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
          tc::split_tf32(v.x, h0, l0);
          tc::split_tf32(v.y, h1, l1);
          tc::split_tf32(v.z, h2, l2);
          tc::split_tf32(v.w, h3, l3);
          pa[idx] = make_float4(__uint_as_float(h0), __uint_as_float(h1), __uint_as_float(h2), __uint_as_float(h3));
          pl[idx] = make_float4(__uint_as_float(l0), __uint_as_float(l1), __uint_as_float(l2), __uint_as_float(l3));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(lo_ready + st);
      }
      if (!ok) break;
    }
  } else if (warp < 8) {
    // ---------------- epilogue: thread = tile row = TMEM lane
    const int t = (warp - 4) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp - 4) * 32) << 16;
    const int ngroups = (nchunks + GC - 1) / GC;
    int64_t i = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int slot = (int)(i & 1);
      if (!tc::mbar_wait(acc_full + slot, (uint32_t)((i >> 1) & 1), a.err, 92)) break;
      tc::tc_fence_after();
      const int64_t g = tile * a.Gb + t / a.R;
      const int r = t % a.R;
      const bool valid = t < a.R * a.Gb && g < a.G;
      float scale = a.alpha != 0.f ? a.alpha : 1.f;
      if (valid && a.deg_rowptr) {
        const int d = a.deg_rowptr[g + 1] - a.deg_rowptr[g];
        scale *= 1.f / (float)(d > 1 ? d : 1);
      }
      float* crow = valid ? a.C + g * a.c_gs + r * a.c_rs : nullptr;
      const uint32_t tslot = tbase + (uint32_t)(slot * 256) + lane_off;
#pragma unroll 1
      for (int cb = 0; cb < NT / 16; ++cb) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = 0.f;
        for (int ga = 0; ga < ngroups; ++ga) {
          uint32_t u[16];
          tc::tmem_ld16(tslot + (uint32_t)(ga * NT) + 16u * cb, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 16; ++k) v[k] += __uint_as_float(u[k]);
        }
        const int nc = 16 * cb;
        if (!crow || nc >= a.N) continue;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          v[k] *= scale;
          if (a.bias && nc + k < a.N) v[k] += a.bias[nc + k];
        }
        float* cp = crow + nc;
        if (nc + 16 <= a.N && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
          float4* c4 = reinterpret_cast<float4*>(cp);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float4 o = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            if (a.accumulate) {
              const float4 pv = c4[k];
              o.x += pv.x;
              o.y += pv.y;
              o.z += pv.z;
              o.w += pv.w;
            }
            c4[k] = o;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k)
            if (nc + k < a.N) cp[k] = a.accumulate ? cp[k] + v[k] : v[k];
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty + slot);
    }
  } else if (warp == 8) {
    // ---------------- producer
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(b_full, (uint32_t)nchunks * TpCfg<NT>::BBYTES);
      for (int c = 0; c < nchunks; ++c)
        tc::bulk_g2s(sB + c * TpCfg<NT>::BBYTES, reinterpret_cast<const uint8_t*>(a.bimg) + (size_t)c * TpCfg<NT>::BBYTES,
                     TpCfg<NT>::BBYTES, b_full);
      int64_t q = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int c = 0; c < nchunks; ++c, ++q) {
          const int st = (int)(q % NST);
          if (q >= NST && !(ok = tc::mbar_wait(empty + st, (uint32_t)(((q / NST) - 1) & 1), a.err, 93))) break;
          tc::mbar_arrive_expect_tx(full + st, a.abox);
          tma_load_3d(smem + st * TpCfg<NT>::RING, &tmA, c * KC, 0, (int)(tile * a.Gb), full + st);
        }
      }
    }
  } else {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_tf32(MT, NT);
      const uint32_t s0 = tc::smem_u32(smem), b0 = tc::smem_u32(sB);
      bool ok = tc::mbar_wait(b_full, 0, a.err, 94);
      int64_t q = 0, i = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++i) {
        const int slot = (int)(i & 1);
        if (i >= 2 && !(ok = tc::mbar_wait(acc_empty + slot, (uint32_t)(((i >> 1) - 1) & 1), a.err, 95))) break;
        tc::tc_fence_after();
        for (int c = 0; c < nchunks; ++c, ++q) {
          const int st = (int)(q % NST);
          if (!(ok = tc::mbar_wait(lo_ready + st, (uint32_t)((q / NST) & 1), a.err, 96))) break;
          tc::tc_fence_after();
          const uint32_t d = tbase + (uint32_t)(slot * 256 + (c / GC) * NT);
          const bool first = c % GC == 0;
          const uint32_t ah0 = s0 + st * TpCfg<NT>::RING, al0 = ah0 + ABYTES;
#pragma unroll
          for (int j = 0; j < KC / 8; ++j) {
            const uint64_t ah = desc_sw128(ah0 + 32 * j);
            const uint64_t al = desc_sw128(al0 + 32 * j);
            const uint32_t bh_addr = b0 + c * TpCfg<NT>::BBYTES + j * 2 * 16 * NT;
            const uint64_t bh = tc::smem_desc_kmajor(bh_addr, 16 * NT, 128);
            const uint64_t bl = tc::smem_desc_kmajor(bh_addr + TpCfg<NT>::BBYTES / 2, 16 * NT, 128);
            mma_tf32_ss(d, ah, bl, idesc, (!first || j > 0) ? 1u : 0u);
            mma_tf32_ss(d, al, bh, idesc, 1u);
            mma_tf32_ss(d, ah, bh, idesc, 1u);
          }
          tc::mma_commit(empty + st);
        }
        if (!ok) break;
        tc::mma_commit(acc_full + slot);
      }
      tc::mma_commit(done);  // also when a wait failed: whatever was issued completes first
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    if (lane == 0) tc::mbar_wait(done, 0, a.err, 97);
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, 512);
  }
}

// B image: element (k, n) of B[k][n] (b_trans: B[n*ldb + k]) at
//   [n / NT][k / KC][hi|lo][(k % KC) / 4][n % NT][k % 4], zero for n >= N or k >= K (K padded to
//   whole chunks).
__global__ void gemm_image_kernel(GemmImageJobs jobs) {
  const GemmImageJob& j = jobs.job[blockIdx.y];
  const int Kp = (j.K + KC - 1) / KC * KC;
  const int64_t total = (int64_t)Kp * j.ntiles * j.NT;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i % Kp);
    const int64_t n = i / Kp;  // padded column
    float x = 0.f;
    if (n < j.N && k < j.K) x = j.b_trans ? j.B[n * j.ldb + k] : j.B[(int64_t)k * j.ldb + n];
    uint32_t hi, lo;
    tc::split_tf32(x, hi, lo);
    const int64_t tile = n / j.NT, nl = n % j.NT;
    const int64_t nch = Kp / KC;
    const int64_t base = ((tile * nch + k / KC) * 2) * (KC * j.NT) + ((k % KC) / 4) * (4 * j.NT) + nl * 4 + (k % 4);
    j.out[base] = __uint_as_float(hi);
    j.out[base + KC * j.NT] = __uint_as_float(lo);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <int NT, bool PRECISE>
int launch_nt(const GemmArgs& g, const CUtensorMap& map, GemmTcArgs t, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(g.G, (int64_t)t.Gb), (unsigned)ceil_div(g.N, NT));
  if constexpr (NT <= 128) {  // A split into TMEM
    const int sm = (int)GmCfg<NT, PRECISE>::TOTAL;
    cudaFuncSetAttribute(gemm_tcm_kernel<NT, PRECISE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    gemm_tcm_kernel<NT, PRECISE><<<grid, GT_THREADS, sm, st>>>(map, t);
    return check_launch("gemm_tcm_kernel");
  } else {
    const int sm = (int)GCfg<NT, PRECISE>::TOTAL;
    cudaFuncSetAttribute(gemm_tc_kernel<NT, PRECISE>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    gemm_tc_kernel<NT, PRECISE><<<grid, GT_THREADS, sm, st>>>(map, t);
    return check_launch("gemm_tc_kernel");
  }
}

// The persistent kernel holds B (whole K) in shared memory and keeps every chunk group at <= 2
// chunks within 256 TMEM columns.  It is used for K <= 128: with a longer K the resident B leaves
// room for too few A stages to stream A (measured: the K = 192 / 256 channel mixes ran slower
// than the two-CTA-per-SM kernel, the K = 64 / 128 dZ mix and MainNet layers faster).
bool gemm_tcp_fits(int NT, int K) {
  const int nchunks = (K + KC - 1) / KC;
  const int nacc_max = 256 / NT;
  return nchunks <= 4 && (uint32_t)nchunks * 2u * KC * NT * 4u <= TP_BMAX && (nchunks + nacc_max - 1) / nacc_max <= 2;
}

template <int NT>
int launch_tp(const GemmArgs& g, const CUtensorMap& map, GemmTcArgs t, cudaStream_t st) {
  const TpShape sh = tp_shape<NT>(g.K);
  if (cudaFuncSetAttribute(gemm_tcp_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh.total) !=
      cudaSuccess)
    return fail(FSC_ERR_CUDA, "gemm_tcp: cannot set shared memory size");
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int64_t ntiles = ceil_div(g.G, (int64_t)t.Gb);
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sms);
  gemm_tcp_kernel<NT><<<grid, TP_THREADS, sh.total, st>>>(map, t);
  return check_launch("gemm_tcp_kernel");
}

}  // namespace

// Output tile width.  Tiles wider than 128 hold no fp32 register sums (their K chunks rotate over
// two TMEM accumulators), so they are used only while those chains stay short (K <= 4 chunks).
int gemm_tc_nt(int N, int K) {
  if (N > 128 && K > 4 * KC) return 128;
  return N <= 64 ? 64 : (N <= 128 ? 128 : (N <= 192 ? 192 : (N <= 256 ? 256 : 128)));
}

bool gemm_tc_supported(const GemmArgs& g) {
  if (g.K % 4 || g.K <= 0 || g.R < 1 || g.R > MT || g.N <= 0) return false;
  const auto a = reinterpret_cast<uintptr_t>(g.A);
  if (a % 16 || (g.a_rs * 4) % 16 || (g.a_gs * 4) % 16) return false;
  if (g.R > 1 && g.a_rs < g.K) return false;
  return encode_fn() != nullptr;
}

int64_t gemm_image_floats(int K, int N) {
  const int NT = gemm_tc_nt(N, K);
  return (int64_t)ceil_div(N, NT) * NT * ((K + KC - 1) / KC * KC) * 2;
}

int launch_gemm_images(const GemmImageJobs& jobs, int njobs, cudaStream_t st) {
  if (njobs <= 0) return FSC_OK;
  if (njobs > kMaxImageJobs) return fail(FSC_ERR_ARGUMENT, "too many GEMM image jobs");
  gemm_image_kernel<<<dim3(64, (unsigned)njobs), 256, 0, st>>>(jobs);
  return check_launch("gemm_image_kernel");
}

int GemmImageBatch::add(const float* B, int64_t ldb, int b_trans, int K, int N, float* out, cudaStream_t st) {
  GemmImageJob& j = jobs.job[n++];
  j.B = B;
  j.ldb = ldb;
  j.b_trans = b_trans;
  j.K = K;
  j.N = N;
  j.NT = gemm_tc_nt(N, K);
  j.ntiles = (int)ceil_div(N, j.NT);
  j.out = out;
  return n == kMaxImageJobs ? flush(st) : FSC_OK;
}

int GemmImageBatch::flush(cudaStream_t st) {
  const int m = n;
  n = 0;
  return launch_gemm_images(jobs, m, st);
}

int run_gemm(const GemmArgs& g, const float* img, int* err, cudaStream_t st) {
  if (img && gemm_tc_supported(g)) return launch_gemm_tc(g, img, err, st);
  return launch_gemm(g, st);
}

int launch_gemm_tc(const GemmArgs& g, const float* bimg, int* err, cudaStream_t st) {
  const int64_t M = g.G * (int64_t)g.R;
  if (M == 0 || g.N == 0) return FSC_OK;
  if (!gemm_tc_supported(g)) return fail(FSC_ERR_UNSUPPORTED, "gemm_tc: unsupported shape or alignment");
  const int NT = gemm_tc_nt(g.N, g.K);
  GemmTcArgs t{};
  t.bimg = bimg;
  t.K = g.K;
  t.N = g.N;
  t.G = g.G;
  t.R = g.R;
  t.Gb = MT / g.R;
  t.abox = (uint32_t)(KC * g.R * t.Gb * 4);
  t.C = g.C;
  t.c_gs = g.c_gs;
  t.c_rs = g.c_rs;
  t.deg_rowptr = g.deg_rowptr;
  t.bias = g.bias;
  t.accumulate = g.accumulate;
  t.alpha = g.alpha;
  t.err = err;
  // A as a 3-D tensor (K, R, G) with byte strides a_rs*4, a_gs*4
  CUtensorMap map;
  const cuuint64_t dims[3] = {(cuuint64_t)g.K, (cuuint64_t)g.R, (cuuint64_t)g.G};
  const cuuint64_t strides[2] = {(cuuint64_t)(g.R > 1 ? g.a_rs : g.K) * 4, (cuuint64_t)g.a_gs * 4};
  const cuuint32_t box[3] = {(cuuint32_t)KC, (cuuint32_t)g.R, (cuuint32_t)t.Gb};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult rc = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(g.A), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return fail(FSC_ERR_CUDA, "cuTensorMapEncodeTiled failed for a GEMM operand");
  if (g.N <= NT && gemm_tcp_fits(NT, g.K)) {
    switch (NT) {
      case 64: return launch_tp<64>(g, map, t, st);
      case 128: return launch_tp<128>(g, map, t, st);
      case 192: return launch_tp<192>(g, map, t, st);
      default: return launch_tp<256>(g, map, t, st);
    }
  }
  if (g.precise) {
    if (NT == 64) return launch_nt<64, true>(g, map, t, st);
    if (NT == 128) return launch_nt<128, true>(g, map, t, st);
  }
  switch (NT) {
    case 64: return launch_nt<64, false>(g, map, t, st);
    case 128: return launch_nt<128, false>(g, map, t, st);
    case 192: return launch_nt<192, false>(g, map, t, st);
    default: return launch_nt<256, false>(g, map, t, st);
  }
}

}  // namespace fsc

extern "C" int fsc_gemm_tc_plan(int K, int N, int precise, int* tile_n, int* max_chain) {
  using namespace fsc;
  if (K <= 0 || N <= 0 || !tile_n || !max_chain) return fail(FSC_ERR_ARGUMENT, "fsc_gemm_tc_plan: bad arguments");
  const int NT = gemm_tc_nt(N, K);
  const int nchunks = (K + KC - 1) / KC;
  constexpr int kPerChunk = 3 * (KC / 8);  // 3xTF32 MMAs per 32-wide K chunk
  *tile_n = NT;
  if (N <= NT && gemm_tcp_fits(NT, K)) {  // persistent kernel: chunk groups of gc chunks
    const int nacc = std::min(nchunks, 256 / NT);
    *max_chain = kPerChunk * ((nchunks + nacc - 1) / nacc);
  } else if (NT <= 128) {  // flushed to fp32 registers every GC chunks
    *max_chain = kPerChunk * std::min(nchunks, precise ? 1 : 2);
  } else {  // chunks rotate over two accumulators
    *max_chain = kPerChunk * ((nchunks + 1) / 2);
  }
  return FSC_OK;
}
