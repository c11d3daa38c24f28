// Readout of the pure-cartesian-ictd model (pure_cartesian_ictd_layers_full.py:956-1054):
//   scalars[n,o] = sum_l sum_{c,d} W_read[l][o,c,d] G_l[n,c,d] / sqrt(2l+1),  G_l = t_l t_l^T (over m)
//   T_0 = [t_0 | scalars], T_l = t_l;  p5 = concat_l factor_l * sum_m T_l[c,m]^2   (product_5, 0e)
//   e = MainNet(p5) . weighted_sum  (models/mlp.py:55-66, 117-133)
// with the features of all layers concatenated along channels (c' = layer*C + c).
// The Gram contraction runs as  packed Gram (this file) x symmetrised W_read (GEMM); its
// backward as  H = dscalars x W_sym (GEMM) then dt = 2 H t (this file).
#include <algorithm>

#include "common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"

namespace fsc {

using ictd2::KB;
using ictd2::NK;

struct GradPtrs {
  float* p[8];
};

__device__ __forceinline__ const float* feat_row(const ReadoutArgs& a, int64_t n, int comp, int cprime, int& c) {
  const int k = cprime / a.C;
  c = cprime - k * a.C;
  return a.feats[k] + (n * NK + comp) * a.C;
}

// Gram operand t_b[c'][m] = flat element goff[b] + c'*(2l+1) + m of the layer concatenation (see
// xmap); returns its offset in feats[layer] relative to the node's row, or -1 for an element
// with no storage (the zero 1e block of the o3 model).
__device__ __forceinline__ int64_t xoff(const ReadoutArgs& a, int b, int cprime, int m, int& layer) {
  const int l = a.gl[b];
  const int32_t code = a.xmap[a.goff[b] + cprime * (2 * l + 1) + m];
  if (code < 0) {
    layer = 0;
    return -1;
  }
  layer = code >> 16;
  return code & 0xffff;
}

__device__ __forceinline__ float xval(const ReadoutArgs& a, int b, int cprime, int m, int64_t base) {
  int layer;
  const int64_t o = xoff(a, b, cprime, m, layer);
  return o < 0 ? 0.f : a.feats[layer][base + o];
}

__global__ void gram_pack_kernel(ReadoutArgs a, int b, int64_t n0, int64_t nn, const int32_t* __restrict__ pairs,
                                 int64_t npairs, float* __restrict__ Gp) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nn * npairs) return;
  const int64_t nl = idx / npairs, j = idx - nl * npairs;
  const int64_t n = n0 + nl;
  const int32_t pr = pairs[j];
  const int cp = pr & 0xffff, dp = pr >> 16;
  const int64_t base = n * NK * a.C;
  const int l = a.gl[b];
  float acc = 0.f;
  for (int m = 0; m < 2 * l + 1; ++m) acc = fmaf(xval(a, b, cp, m, base), xval(a, b, dp, m, base), acc);
  Gp[idx] = acc;
}

// grads at t_b[c'][m] += 2 sum_d H[n][c'][d] t_b[d][m]
__global__ void gram_apply_kernel(ReadoutArgs a, GradPtrs g, int b, int64_t n0, int64_t nn,
                                  const float* __restrict__ H) {
  const int nC = a.C * a.nint;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nn * nC) return;
  const int64_t nl = idx / nC;
  const int cp = (int)(idx - nl * nC);
  const int64_t n = n0 + nl;
  const int64_t base = n * NK * a.C;
  const int l = a.gl[b];
  const float* h = H + (nl * nC + cp) * (int64_t)nC;
  float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  for (int d = 0; d < nC; ++d) {
    const float hv = h[d];
#pragma unroll
    for (int m = 0; m < 5; ++m)
      if (m < 2 * l + 1) acc[m] = fmaf(hv, xval(a, b, d, m, base), acc[m]);
  }
  for (int m = 0; m < 2 * l + 1; ++m) {
    int lc;
    const int64_t oc = xoff(a, b, cp, m, lc);
    if (oc >= 0) g.p[lc][base + oc] += 2.f * acc[m];
  }
}

// Physical-tensor heads: out[h][graph][m] = sum_n sum_c w[h][c] t_{blocks[h]}[n][c][m] (m < 5).
// One warp per (node, head): lanes split the channels, one double atomic per component.
struct HeadBlocks {
  int b[4];
};

__global__ void heads_kernel(ReadoutArgs a, const int32_t* __restrict__ batch, int nheads, HeadBlocks blocks,
                             const float* __restrict__ w, double* __restrict__ acc) {
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (wid >= a.N * nheads) return;
  const int64_t n = wid / nheads;
  const int h = (int)(wid - n * nheads);
  const int b = blocks.b[h];
  const int l = a.gl[b];
  const int nC = a.C * a.nint;
  const int64_t base = n * NK * a.C;
  float v[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  for (int c = lane; c < nC; c += 32) {
    const float wc = w[(int64_t)h * nC + c];
#pragma unroll
    for (int m = 0; m < 5; ++m)
      if (m < 2 * l + 1) v[m] = fmaf(wc, xval(a, b, c, m, base), v[m]);
  }
#pragma unroll
  for (int m = 0; m < 5; ++m) v[m] = warp_sum(v[m]);
  if (lane == 0) {
    double* o = acc + ((int64_t)h * 4096 + batch[n]) * 5;
    for (int m = 0; m < 2 * l + 1; ++m) atomicAdd(o + m, (double)v[m]);
  }
}

__global__ void heads_finalize_kernel(const double* __restrict__ acc, int nheads, int64_t B, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nheads * B * 5) return;
  const int64_t h = i / (B * 5), r = i - h * B * 5;
  out[i] = (float)acc[h * 4096 * 5 + r];
}

// MainNet input [0e | scalars | (o3: zero 1e) | 1 | 2] (product_5 of the concatenated per-layer
// features, pure_cartesian_ictd_layers_o3.py:1046-1057 for o3).
__global__ void __launch_bounds__(128) p5_forward_kernel(ReadoutArgs a, const float* __restrict__ scalars,
                                                         float* __restrict__ p5) {
  const int nC = a.C * a.nint;
  const int z = a.o3 ? nC : 0;
  const int D0 = 3 * nC + a.S + z;
  const float* f = a.tables + ictd2::TAB_P5;
  for (int64_t n = blockIdx.x; n < a.N; n += gridDim.x) {  // one node per CTA pass: no index division
    for (int j = threadIdx.x; j < D0; j += blockDim.x) {
      float v;
      if (j < nC) {
        int c;
        const float* r = feat_row(a, n, 0, j, c);
        v = f[0] * r[c] * r[c];
      } else if (j < nC + a.S) {
        const float s = scalars[n * a.S + (j - nC)];
        v = f[0] * s * s;
      } else if (j < nC + a.S + z) {
        v = 0.f;
      } else {
        const int l = j < 2 * nC + a.S + z ? 1 : 2;
        const int cp = j - (nC + a.S + z) - (l - 1) * nC;
        const int k = cp / a.C, c = cp - k * a.C;
        const float* r = a.feats[k] + (n * NK + KB(l)) * a.C + c;
        float acc = 0.f;
        for (int m = 0; m < 2 * l + 1; ++m) acc = fmaf(r[m * a.C], r[m * a.C], acc);
        v = f[l] * acc;
      }
      p5[n * D0 + j] = v;
    }
  }
}

__global__ void __launch_bounds__(128) p5_backward_kernel(ReadoutArgs a, GradPtrs g, const float* __restrict__ scalars,
                                                          const float* __restrict__ dp5, float* __restrict__ dscalars) {
  const int nC = a.C * a.nint;
  const int z = a.o3 ? nC : 0;
  const int D0 = 3 * nC + a.S + z;
  const float* f = a.tables + ictd2::TAB_P5;
  for (int64_t n = blockIdx.x; n < a.N; n += gridDim.x) {  // one node per CTA pass: no index division
    for (int j = threadIdx.x; j < D0; j += blockDim.x) {
      const float d = dp5[n * D0 + j];
      if (j < nC) {
        const int k = j / a.C, c = j - k * a.C;
        const int64_t off = (n * NK) * a.C + c;
        g.p[k][off] = 2.f * f[0] * a.feats[k][off] * d;
      } else if (j < nC + a.S) {
        const int o = j - nC;
        dscalars[n * a.S + o] = 2.f * f[0] * scalars[n * a.S + o] * d;
      } else if (j < nC + a.S + z) {
        // zero 1e slot: no input depends on it
      } else {
        const int l = j < 2 * nC + a.S + z ? 1 : 2;
        const int cp = j - (nC + a.S + z) - (l - 1) * nC;
        const int k = cp / a.C, c = cp - k * a.C;
        for (int m = 0; m < 2 * l + 1; ++m) {
          const int64_t off = (n * NK + KB(l) + m) * a.C + c;
          g.p[k][off] = 2.f * f[l] * a.feats[k][off] * d;
        }
      }
    }
  }
}

// One warp per row; D <= 1024.
__global__ void layernorm_kernel(const float* __restrict__ X, int64_t rows, int D, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, int silu_flag, float* __restrict__ Y) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = X + row * D;
  float s = 0.f;
  for (int i = lane; i < D; i += 32) s += x[i];
  const float mean = warp_sum(s) / (float)D;
  float v = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float t = x[i] - mean;
    v = fmaf(t, t, v);
  }
  const float rstd = rsqrtf(warp_sum(v) / (float)D + 1e-5f);
  float* y = Y + row * D;
  for (int i = lane; i < D; i += 32) {
    float u = (x[i] - mean) * rstd * gamma[i] + beta[i];
    y[i] = silu_flag ? silu(u) : u;
  }
}

__global__ void layernorm_backward_kernel(const float* __restrict__ X, const float* __restrict__ dY, int64_t rows,
                                          int D, const float* __restrict__ gamma, const float* __restrict__ beta,
                                          int silu_flag, float* __restrict__ dX) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = X + row * D;
  const float* dy = dY + row * D;
  float s = 0.f;
  for (int i = lane; i < D; i += 32) s += x[i];
  const float mean = warp_sum(s) / (float)D;
  float v = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float t = x[i] - mean;
    v = fmaf(t, t, v);
  }
  const float rstd = rsqrtf(warp_sum(v) / (float)D + 1e-5f);
  // g_i = dL/dxhat_i = dy_i * (silu'(u_i)) * gamma_i
  float s1 = 0.f, s2 = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float xh = (x[i] - mean) * rstd;
    float gi = dy[i];
    if (silu_flag) gi *= silu_grad(xh * gamma[i] + beta[i]);
    gi *= gamma[i];
    s1 += gi;
    s2 = fmaf(gi, xh, s2);
  }
  s1 = warp_sum(s1) / (float)D;
  s2 = warp_sum(s2) / (float)D;
  float* dx = dX + row * D;
  for (int i = lane; i < D; i += 32) {
    const float xh = (x[i] - mean) * rstd;
    float gi = dy[i];
    if (silu_flag) gi *= silu_grad(xh * gamma[i] + beta[i]);
    gi *= gamma[i];
    dx[i] = rstd * (gi - s1 - xh * s2);
  }
}

__global__ void energy_kernel(const float* __restrict__ x, int64_t N, int H, const float* __restrict__ v, float c0,
                              const int32_t* __restrict__ batch, int64_t num_local, float* __restrict__ atom_energy,
                              double* __restrict__ energy) {
  const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  float s = 0.f;
  for (int i = lane; i < H; i += 32) s = fmaf(x[n * H + i], v[i], s);
  s = warp_sum(s) + c0;
  if (lane == 0) {
    if (atom_energy) atom_energy[n] = s;
    if (energy && n < num_local) atomicAdd(energy + batch[n], (double)s);
  }
}

__global__ void energy_seed_kernel(int64_t N, int H, const float* __restrict__ v, const float* __restrict__ weight,
                                   int64_t num_local, float* __restrict__ dx) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= N * H) return;
  const int64_t n = idx / H;
  const float wn = weight ? weight[n] : (n < num_local ? 1.f : 0.f);
  dx[idx] = wn * v[idx - n * H];
}

static GradPtrs to_ptrs(float* const* g, int nint) {
  GradPtrs p{};
  for (int k = 0; k < nint && k < 8; ++k) p.p[k] = g[k];
  return p;
}

int launch_heads(const ReadoutArgs& a, const int32_t* batch, int nheads, const int32_t* blocks, const float* w,
                 double* acc, float* out, int64_t B, cudaStream_t st) {
  if (cudaMemsetAsync(acc, 0, sizeof(double) * nheads * 4096 * 5, st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "memset heads");
  if (a.N > 0) {
    HeadBlocks hb{};
    for (int h = 0; h < nheads && h < 4; ++h) hb.b[h] = blocks[h];
    heads_kernel<<<(unsigned)ceil_div(a.N * nheads, 8), 256, 0, st>>>(a, batch, nheads, hb, w, acc);
    FSC_TRY(check_launch("heads_kernel"));
  }
  heads_finalize_kernel<<<(unsigned)ceil_div((int64_t)nheads * B * 5, 256), 256, 0, st>>>(acc, nheads, B, out);
  return check_launch("heads_finalize_kernel");
}

int launch_gram_pack(const ReadoutArgs& a, int l, int64_t n0, int64_t nn, const int32_t* pairs, int64_t npairs,
                     float* Gp, cudaStream_t st) {
  const int64_t total = nn * npairs;
  if (total == 0) return FSC_OK;
  gram_pack_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(a, l, n0, nn, pairs, npairs, Gp);
  return check_launch("gram_pack_kernel");
}

int launch_gram_apply(const ReadoutArgs& a, int l, int64_t n0, int64_t nn, const float* H, float* const* grads,
                      cudaStream_t st) {
  const int64_t total = nn * a.C * a.nint;
  if (total == 0) return FSC_OK;
  gram_apply_kernel<<<(unsigned)ceil_div(total, 128), 128, 0, st>>>(a, to_ptrs(grads, a.nint), l, n0, nn, H);
  return check_launch("gram_apply_kernel");
}

int launch_p5_forward(const ReadoutArgs& a, const float* scalars, float* p5, cudaStream_t st) {
  const int64_t total = a.N * ((a.o3 ? 4 : 3) * a.C * a.nint + a.S);
  if (total == 0) return FSC_OK;
  p5_forward_kernel<<<(unsigned)std::min<int64_t>(a.N, 1 << 20), 128, 0, st>>>(a, scalars, p5);
  return check_launch("p5_forward_kernel");
}

int launch_p5_backward(const ReadoutArgs& a, const float* scalars, const float* dp5, float* const* grads,
                       float* dscalars, cudaStream_t st) {
  const int64_t total = a.N * ((a.o3 ? 4 : 3) * a.C * a.nint + a.S);
  if (total == 0) return FSC_OK;
  p5_backward_kernel<<<(unsigned)std::min<int64_t>(a.N, 1 << 20), 128, 0, st>>>(a, to_ptrs(grads, a.nint), scalars, dp5,
                                                                       dscalars);
  return check_launch("p5_backward_kernel");
}

int launch_layernorm(const float* X, int64_t rows, int D, const float* gamma, const float* beta, int silu_flag,
                     float* Y, cudaStream_t st) {
  if (rows == 0) return FSC_OK;
  layernorm_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(X, rows, D, gamma, beta, silu_flag, Y);
  return check_launch("layernorm_kernel");
}

int launch_layernorm_backward(const float* X, const float* dY, int64_t rows, int D, const float* gamma,
                              const float* beta, int silu_flag, float* dX, cudaStream_t st) {
  if (rows == 0) return FSC_OK;
  layernorm_backward_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(X, dY, rows, D, gamma, beta, silu_flag,
                                                                           dX);
  return check_launch("layernorm_backward_kernel");
}

int launch_energy(const float* x, int64_t N, int H, const float* v, float c0, const int32_t* batch,
                  int64_t num_local, float* atom_energy, double* energy, cudaStream_t st) {
  if (N == 0) return FSC_OK;
  energy_kernel<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(x, N, H, v, c0, batch, num_local, atom_energy, energy);
  return check_launch("energy_kernel");
}

int launch_energy_seed(int64_t N, int H, const float* v, const float* weight, int64_t num_local, float* dx,
                       cudaStream_t st) {
  if (N == 0) return FSC_OK;
  energy_seed_kernel<<<(unsigned)ceil_div(N * H, 256), 256, 0, st>>>(N, H, v, weight, num_local, dx);
  return check_launch("energy_seed_kernel");
}

}  // namespace fsc
