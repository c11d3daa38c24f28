// pure-cartesian-ictd energy + forces: forward of PureCartesianICTDTransformerLayer
// (pure_cartesian_ictd_layers_full.py:867-1078) and a hand-written reverse pass that yields
// dE/dr per edge, forces and the virial without autograd replay.  All buffers come from the
// caller's workspace; nothing is allocated here.
#include <algorithm>
#include <cmath>
#include <vector>

#include "common.cuh"
#include "ictd_paths.cuh"
#include "kernels.cuh"

namespace fsc {

using namespace ictd2;

// Optional per-stage CUDA-event timing of the engine (off by default).
namespace prof {
constexpr int kMax = 64;
bool enabled = false;
int count = 0;
const char* names[kMax];
cudaEvent_t events[kMax];
bool created = false;

void mark(const char* name, cudaStream_t st) {
  if (!enabled || count >= kMax) return;
  if (!created) {
    for (int i = 0; i < kMax; ++i) cudaEventCreate(&events[i]);
    created = true;
  }
  names[count] = name;
  cudaEventRecord(events[count], st);
  ++count;
}
}  // namespace prof

namespace {

constexpr int64_t kGramChunk = 16384;  // nodes per readout chunk
constexpr int64_t kMaxGraphs = 4096;   // graphs per call (float64 accumulators in the workspace)

struct Plan {
  int C, nint, S, nC, D0, nb;
  int o3;                   // parity-keyed model: 4 Gram blocks, zero 1e slot in the MainNet input
  int ngram;                // Gram blocks of the readout (3, or 4 with o3)
  int goff[4], gl[4];       // block offset in the flat split (units of nC) and its l
  int64_t nrows;            // Gram operand rows: nC * sum_b (2 l_b + 1)
  int64_t N, E, B, npairs, chunk;
  int64_t nk[8];            // receiving atoms evaluated per interaction layer (graph layer_atoms)
  int64_t nro;              // atoms of the readout: nk[nint - 1]
  int hidden[4];
  int n_hidden;
  // workspace
  int32_t* dst;
  int32_t* tr_dst;
  float* invdeg;
  float* edge_y;
  float* gates;
  float* feats[8];
  float* zbuf;
  float* scalars;
  float* p5;
  float* x0;
  float* act_pre[4];
  float* act_post[4];
  double* energy_d;
  float* grads[8];
  float* dscalars;
  float* dp5;
  float* dxa;
  float* dxb;
  float* dgates;
  float* dY;
  float* edge_grad;
  double* virial_d;
  double* cellg_d;
  float* chunkbuf;
  double* heads_d;          // [4][kMaxGraphs][5] physical-tensor head accumulators
  // tensor-core readout
  bool tc;
  bool rtc;  // radial MLPs on tensor cores
  int64_t n_pad;
  float* Fg;
  float* dFg;
  float* gmax;
  int* err;
  int* work;  // conv2 node counter
  // tensor-core GEMM operand images of the weights (null: CUDA-core GEMM)
  bool gtc;
  float* img_fwd[8][3];     // conv2 layer k, l3
  float* img_dz[8][3];
  float* img_dx[8][3];      // by l1
  float* img_mnf[4];
  float* img_mnb[4];
};

int g_readout_path = 0;  // 0: tensor cores where supported, 1: CUDA cores
int g_radial_path = 0;   // 0: tensor cores where supported, 1: CUDA cores
int g_gemm_path = 0;     // 0: tensor cores where supported, 1: CUDA cores
int g_conv2_path = 0;    // conv2 gate gradients: 0 CUDA cores (faster), 1 tensor cores

int validate(const fsc_ictd_config* cfg) {
  FSC_REQUIRE(cfg != nullptr, "config is null");
  if (cfg->lmax != 2) return fail(FSC_ERR_UNSUPPORTED, "ictd engine supports lmax = 2 only");
  if (cfg->channels != 32 && cfg->channels != 64)
    return fail(FSC_ERR_UNSUPPORTED, "ictd engine supports channels 32 or 64");
  if (cfg->num_interaction < 2 || cfg->num_interaction > 8)
    return fail(FSC_ERR_UNSUPPORTED, "num_interaction must be in [2, 8]");
  if (cfg->number_of_basis < 1 || cfg->number_of_basis > 16)
    return fail(FSC_ERR_UNSUPPORTED, "number_of_basis must be in [1, 16]");
  if (cfg->basis_kind != 0 && cfg->basis_kind != 1)
    return fail(FSC_ERR_UNSUPPORTED, "radial basis must be gaussian (0) or bessel (1)");
  if (cfg->output_size != 8) return fail(FSC_ERR_UNSUPPORTED, "output_size must be 8");
  if (cfg->n_hidden < 1 || cfg->n_hidden > 4) return fail(FSC_ERR_UNSUPPORTED, "MainNet needs 1..4 hidden layers");
  for (int k = 0; k < cfg->n_hidden; ++k)
    if (cfg->hidden[k] < 1 || cfg->hidden[k] > 1024) return fail(FSC_ERR_UNSUPPORTED, "MainNet hidden size out of range");
  if (cfg->invariant_channels < 1) return fail(FSC_ERR_ARGUMENT, "invariant_channels must be >= 1");
  return FSC_OK;
}

void layout(Plan& p, Arena& ar, const fsc_ictd_config* cfg, int64_t N, int64_t E) {
  p.C = cfg->channels;
  p.nint = cfg->num_interaction;
  p.S = (p.nint - 1) * cfg->invariant_channels;
  p.nC = p.C * p.nint;
  p.o3 = cfg->o3 ? 1 : 0;
  p.ngram = p.o3 ? 4 : 3;
  {
    const int ls[4] = {0, 1, p.o3 ? 1 : 2, 2};
    int off = 0;
    for (int b = 0; b < p.ngram; ++b) {
      p.gl[b] = ls[b];
      p.goff[b] = off * p.nC;
      off += 2 * ls[b] + 1;
    }
    p.nrows = (int64_t)off * p.nC;
  }
  p.D0 = p.ngram * p.nC + p.S;
  p.nb = cfg->number_of_basis;
  p.N = N;
  p.E = E;
  p.npairs = (int64_t)p.nC * (p.nC + 1) / 2;
  p.chunk = std::max<int64_t>(1, std::min<int64_t>(N, kGramChunk));
  p.n_hidden = cfg->n_hidden;
  for (int k = 0; k < 4; ++k) p.hidden[k] = k < cfg->n_hidden ? cfg->hidden[k] : 0;
  int maxw = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) maxw = std::max(maxw, p.hidden[k]);
  const int64_t fsz = N * NK * p.C;
  p.dst = ar.take<int32_t>(E);
  p.tr_dst = ar.take<int32_t>(E);
  p.invdeg = ar.take<float>(N);
  p.edge_y = ar.take<float>(E * 12);
  p.gates = ar.take<float>((int64_t)p.nint * E * 12);
  for (int k = 0; k < p.nint; ++k) p.feats[k] = ar.take<float>(fsz);
  p.zbuf = ar.take<float>(N * NZ * p.C);
  p.scalars = ar.take<float>(N * p.S);
  p.p5 = ar.take<float>(N * p.D0);
  p.x0 = ar.take<float>(N * p.D0);
  for (int k = 0; k < p.n_hidden; ++k) {
    p.act_pre[k] = ar.take<float>(N * p.hidden[k]);
    p.act_post[k] = ar.take<float>(N * p.hidden[k]);
  }
  p.energy_d = ar.take<double>(kMaxGraphs * 19);
  p.virial_d = p.energy_d ? p.energy_d + kMaxGraphs : nullptr;
  p.cellg_d = p.energy_d ? p.energy_d + 10 * kMaxGraphs : nullptr;
  for (int k = 0; k < p.nint; ++k) p.grads[k] = ar.take<float>(fsz);
  p.dscalars = ar.take<float>(N * p.S);
  p.dp5 = ar.take<float>(N * p.D0);
  p.dxa = ar.take<float>(N * maxw);
  p.dxb = ar.take<float>(N * maxw);
  p.dgates = ar.take<float>((int64_t)p.nint * E * 12);
  p.dY = ar.take<float>(E * 12);
  p.edge_grad = ar.take<float>(E * 3);
  p.heads_d = ar.take<double>(4 * kMaxGraphs * 5);
  p.tc = g_readout_path == 0 && readout_tc_supported(p.nC, p.S);
  p.gtc = g_gemm_path == 0 || g_gemm_path == 3;  // 3: tensor-core GEMMs with CUDA-core sparse aggregation
  for (int k = 0; k < 8; ++k)
    for (int l = 0; l < 3; ++l) p.img_fwd[k][l] = p.img_dz[k][l] = p.img_dx[k][l] = nullptr;
  for (int k = 0; k < 4; ++k) p.img_mnf[k] = p.img_mnb[k] = nullptr;
  if (p.gtc) {
    const int C = p.C;
    for (int k = 1; k < p.nint; ++k)
      for (int l = 0; l < 3; ++l) {
        p.img_fwd[k][l] = ar.take<float>(gemm_image_floats(NP3(l) * C, C));
        p.img_dz[k][l] = ar.take<float>(gemm_image_floats(C, NP3(l) * C));
        p.img_dx[k][l] = ar.take<float>(gemm_image_floats(NP1(l) * C, C));
      }
    int din = p.D0;
    for (int k = 0; k < p.n_hidden; ++k) {
      p.img_mnf[k] = ar.take<float>(gemm_image_floats(din, p.hidden[k]));
      p.img_mnb[k] = ar.take<float>(gemm_image_floats(p.hidden[k], din));
      din = p.hidden[k];
    }
  }
  p.rtc = g_radial_path == 0 && radial_tc_supported(p.nb);
  p.n_pad = ceil_div(std::max<int64_t>(N, 1), 128) * 128;
  p.err = ar.take<int>(64);
  p.work = ar.take<int>(16);
  if (p.tc) {
    p.chunkbuf = nullptr;
    p.Fg = ar.take<float>(p.nrows * p.n_pad);
    p.dFg = ar.take<float>(p.nrows * p.n_pad);
    p.gmax = ar.take<float>(4 * p.n_pad);
  } else {
    p.Fg = p.dFg = p.gmax = nullptr;
    p.chunkbuf = ar.take<float>(p.chunk * std::max<int64_t>(p.npairs, (int64_t)p.nC * p.nC));
  }
}

FgArgs fg_args(const Plan& p, const fsc_ictd_weights* w) {
  FgArgs f{};
  f.N = p.nro;
  f.n_pad = p.n_pad;
  f.C = p.C;
  f.nint = p.nint;
  for (int k = 0; k < p.nint; ++k) {
    f.feats[k] = p.feats[k];
    f.grads[k] = p.grads[k];
  }
  f.xinv = w->xinv;
  f.Fg = p.Fg;
  f.dFg = p.dFg;
  f.gmax = p.gmax;
  f.ngram = p.ngram;
  for (int b = 0; b < 4; ++b) f.goff[b] = p.goff[b];
  f.nrows = p.nrows;
  return f;
}

ReadoutTcArgs tc_args(const Plan& p, const float* wimg) {
  ReadoutTcArgs r{};
  r.N = p.nro;
  r.n_pad = p.n_pad;
  r.nrows = p.nrows;
  r.nC = p.nC;
  r.S = p.S;
  r.Fg = p.Fg;
  r.gmax = p.gmax;
  r.wimg = wimg;
  r.scalars = p.scalars;
  r.dscal = p.dscalars;
  r.dFg = p.dFg;
  r.err = p.err;
  r.ngram = p.ngram;
  for (int b = 0; b < 4; ++b) {
    r.goff[b] = p.goff[b];
    r.gl[b] = p.gl[b];
  }
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

// Block offset of l-block l inside one layer's mix weights (3, 4, 4 paths of C x C).
inline int64_t mix_boff(int l, int C) { return (int64_t)(l == 0 ? 0 : (l == 1 ? 3 : 7)) * C * C; }

// Builds every weight image the tensor-core GEMMs of this call read.
int build_gemm_images(const Plan& p, const fsc_ictd_weights* w, cudaStream_t st) {
  if (!p.gtc) return FSC_OK;
  GemmImageBatch jobs;
  const int C = p.C;
  for (int k = 1; k < p.nint; ++k) {
    const int64_t lo = (int64_t)(k - 1) * NP * C * C;
    for (int l = 0; l < 3; ++l) {
      FSC_TRY(jobs.add(w->mix_fwd + lo + mix_boff(l, C), C, 0, NP3(l) * C, C, p.img_fwd[k][l], st));
      FSC_TRY(jobs.add(w->mix_bwd + lo + mix_boff(l, C), NP3(l) * C, 0, C, NP3(l) * C, p.img_dz[k][l], st));
      FSC_TRY(jobs.add(w->mix_dx + lo + mix_boff(l, C), C, 0, NP1(l) * C, C, p.img_dx[k][l], st));
    }
  }
  int din = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) {
    FSC_TRY(jobs.add(w->mn_w[k], din, 1, din, p.hidden[k], p.img_mnf[k], st));
    FSC_TRY(jobs.add(w->mn_w[k], din, 0, p.hidden[k], din, p.img_mnb[k], st));
    din = p.hidden[k];
  }
  return jobs.flush(st);
}

__global__ void finalize_kernel(const double* __restrict__ e, const double* __restrict__ v, int64_t B, float* energy,
                                float* virial) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < B && energy) energy[i] = (float)e[i];
  if (i < 9 * B && virial) virial[i] = (float)v[i];
}

struct Ctx {
  const fsc_ictd_config* cfg;
  const fsc_ictd_weights* w;
  const fsc_graph* g;
  Plan p;
  cudaStream_t st;
};

ConvArgs conv_args(const Ctx& c, int layer) {
  ConvArgs a{};
  a.N = c.p.N;
  a.E = c.p.E;
  a.C = c.p.C;
  a.row_ptr = c.g->row_ptr;
  a.src = c.g->src;
  a.dst = c.p.dst;
  a.tr_ptr = c.g->tr_ptr;
  a.tr_eid = c.g->tr_eid;
  a.species = c.g->species;
  a.tables = c.w->tables;
  a.edge_y = c.p.edge_y;
  a.gates = c.p.gates + (int64_t)layer * c.p.E * 12;
  a.field = c.g->field;
  a.batch = c.g->batch;
  a.N = c.p.nk[layer];
  a.n_active = c.p.nk[layer];
  a.dst_limit = c.p.nk[layer];
  a.src_limit = layer > 0 ? c.p.nk[layer - 1] : c.p.N;
  a.err = c.p.err;
  a.tr_dst = c.p.tr_dst;
  a.invdeg = c.p.invdeg;
  a.work = c.p.work;
  return a;
}

ReadoutArgs readout_args(const Ctx& c) {
  ReadoutArgs r{};
  r.N = c.p.nro;
  r.C = c.p.C;
  r.nint = c.p.nint;
  r.S = c.p.S;
  for (int k = 0; k < c.p.nint; ++k) r.feats[k] = c.p.feats[k];
  r.tables = c.w->tables;
  r.xmap = c.w->xmap;
  r.o3 = c.p.o3;
  r.ngram = c.p.ngram;
  for (int b = 0; b < 4; ++b) {
    r.goff[b] = c.p.goff[b];
    r.gl[b] = c.p.gl[b];
  }
  return r;
}

RadialW radial(const fsc_ictd_weights* w) {
  return RadialW{w->rad_w1, w->rad_b1, w->rad_w2, w->rad_b2, w->rad_w3, w->rad_b3};
}

// Forward in steps (fsc_ictd_forward_step): 0 = edge geometry, radial MLPs and conv1; k in
// [1, nint) = conv2 layer k; nint = readout.
int forward_step0(Ctx& c) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  prof::mark("begin", st);
  FSC_TRY(build_gemm_images(p, w, st));
  FSC_TRY(launch_edge_dst(g->row_ptr, p.dst, p.N, st));
  FSC_TRY(launch_transpose_aux(g->row_ptr, p.dst, g->tr_eid, p.N, p.E, p.tr_dst, p.invdeg, st));
  EdgeFwdArgs ef{};
  ef.E = p.E; ef.pos = g->pos; ef.src = g->src; ef.dst = p.dst; ef.batch = g->batch; ef.cell = g->cell;
  ef.shift = g->shift; ef.tables = w->tables; ef.rad = radial(w); ef.nint = p.nint; ef.nb = p.nb;
  ef.basis_kind = c.cfg->basis_kind; ef.rc = c.cfg->max_radius; ef.edge_y = p.edge_y; ef.gates = p.gates;
  if (p.rtc) {
    FSC_TRY(launch_edge_geom(ef, st));
    RadialTcArgs ra{};
    ra.E = p.E; ra.rad = ef.rad; ra.nint = p.nint; ra.nb = p.nb; ra.basis_kind = ef.basis_kind; ra.rc = ef.rc;
    ra.tables = w->tables; ra.edge_y = p.edge_y; ra.gates = p.gates; ra.err = p.err;
    FSC_TRY(launch_radial_fwd_tc(ra, st));
  } else {
    FSC_TRY(launch_edge_forward(ef, st));
  }
  prof::mark("edge_forward", st);
  FSC_TRY(launch_conv1_forward(conv_args(c, 0), w->ai, w->vsp, p.feats[0], st));
  prof::mark("conv1_forward", st);
  return FSC_OK;
}

int forward_conv2(Ctx& c, int k) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  const int C = p.C;
  FSC_TRY(launch_conv2_z(conv_args(c, k), p.feats[k - 1], p.zbuf, st));
  prof::mark("conv2_edge_forward", st);
  const float* W = w->mix_fwd + (int64_t)(k - 1) * NP * C * C;
  int64_t boff = 0;
  for (int l3 = 0; l3 < 3; ++l3) {
    GemmArgs ga = gemm(p.zbuf + OFF3(l3) * C, NZ * C, NP3(l3) * C, W + boff, C, 0, p.feats[k] + KB(l3) * C,
                       NK * C, C, p.nk[k], 2 * l3 + 1, NP3(l3) * C, C);
    ga.deg_rowptr = g->row_ptr;
    FSC_TRY(run_gemm(ga, p.img_fwd[k][l3], p.err, st));
    boff += (int64_t)NP3(l3) * C * C;
  }
  prof::mark("conv2_mix_forward", st);
  return FSC_OK;
}

int forward_readout(Ctx& c) {
  Plan& p = c.p;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  // readout scalars: packed Gram x symmetrised W_read
  ReadoutArgs ra = readout_args(c);
  if (p.tc) {
    // o3: the Gram operand rows of the (zero) 1e block have no storage and stay zero
    if (p.o3 && cudaMemsetAsync(p.Fg, 0, sizeof(float) * p.nrows * p.n_pad, st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset Fg");
    if (cudaMemsetAsync(p.gmax, 0, sizeof(float) * p.ngram * p.n_pad, st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset gmax");
    FSC_TRY(launch_fg_gather(fg_args(p, w), st));
    prof::mark("readout_gather", st);
    FSC_TRY(launch_readout_fwd_tc(tc_args(p, w->wimg_fwd), st));
  }
  if (!p.tc && cudaMemsetAsync(p.scalars, 0, sizeof(float) * p.nro * p.S, st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "memset scalars");
  for (int b = 0; b < p.ngram && !p.tc; ++b) {
    const float* Wp = w->wread_p + (int64_t)b * p.S * p.npairs;
    for (int64_t n0 = 0; n0 < p.nro; n0 += p.chunk) {
      const int64_t nn = std::min(p.chunk, p.nro - n0);
      FSC_TRY(launch_gram_pack(ra, b, n0, nn, w->pairs, p.npairs, p.chunkbuf, st));
      GemmArgs ga = gemm(p.chunkbuf, p.npairs, 0, Wp, p.npairs, 1, p.scalars + n0 * p.S, p.S, 0, nn, 1,
                         (int)p.npairs, p.S);
      ga.accumulate = 1;
      ga.precise = 1;
      FSC_TRY(launch_gemm(ga, st));
    }
  }
  prof::mark("readout_gram_forward", st);
  FSC_TRY(launch_p5_forward(ra, p.scalars, p.p5, st));
  FSC_TRY(launch_layernorm(p.p5, p.nro, p.D0, w->mn_in_g, w->mn_in_b, 0, p.x0, st));
  const float* xin = p.x0;
  int din = p.D0;
  for (int k = 0; k < p.n_hidden; ++k) {
    GemmArgs ga = gemm(xin, din, 0, w->mn_w[k], din, 1, p.act_pre[k], p.hidden[k], 0, p.nro, 1, din, p.hidden[k]);
    ga.bias = w->mn_b[k];
    FSC_TRY(run_gemm(ga, p.img_mnf[k], p.err, st));
    FSC_TRY(launch_layernorm(p.act_pre[k], p.nro, p.hidden[k], w->mn_g[k], w->mn_beta[k], 1, p.act_post[k], st));
    xin = p.act_post[k];
    din = p.hidden[k];
  }
  prof::mark("readout_mlp_forward", st);
  return FSC_OK;
}

// Backward in steps (fsc_ictd_backward_step): nint = readout backward (every layer's feature
// gradient from the readout); k in [1, nint) = conv2 layer k backward (adds into layer k - 1's
// gradient); 0 = conv1 backward (then the edge part, run_backward_edges).
int backward_readout(Ctx& c) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  const int C = p.C;
  const int H = p.hidden[p.n_hidden - 1];
  FSC_TRY(launch_energy_seed(p.nro, H, w->out_v, g->energy_weight, g->num_local, p.dxa, st));
  float* dcur = p.dxa;
  float* dnext = p.dxb;
  for (int k = p.n_hidden - 1; k >= 0; --k) {
    const int din = k == 0 ? p.D0 : p.hidden[k - 1];
    // da_k = LN_bwd(a_k, dx_{k+1}) into dnext, then dx_k = da_k @ W_k into dcur
    FSC_TRY(launch_layernorm_backward(p.act_pre[k], dcur, p.nro, p.hidden[k], w->mn_g[k], w->mn_beta[k], 1, dnext, st));
    GemmArgs ga = gemm(dnext, p.hidden[k], 0, w->mn_w[k], din, 0, dcur, din, 0, p.nro, 1, p.hidden[k], din);
    FSC_TRY(run_gemm(ga, p.img_mnb[k], p.err, st));
  }
  FSC_TRY(launch_layernorm_backward(p.p5, dcur, p.nro, p.D0, w->mn_in_g, w->mn_in_b, 0, p.dp5, st));
  ReadoutArgs ra = readout_args(c);
  FSC_TRY(launch_p5_backward(ra, p.scalars, p.dp5, p.grads, p.dscalars, st));
  prof::mark("readout_mlp_backward", st);
  if (p.tc) {
    FSC_TRY(launch_readout_bwd_tc(tc_args(p, w->wimg_bwd), st));
    prof::mark("readout_gram_backward", st);
    FSC_TRY(launch_fg_scatter_add(fg_args(p, w), st));
  }
  for (int b = 0; b < p.ngram && !p.tc; ++b) {
    const float* Ws = w->wread_s + (int64_t)b * p.S * p.nC * p.nC;
    for (int64_t n0 = 0; n0 < p.nro; n0 += p.chunk) {
      const int64_t nn = std::min(p.chunk, p.nro - n0);
      GemmArgs ga = gemm(p.dscalars + n0 * p.S, p.S, 0, Ws, (int64_t)p.nC * p.nC, 0, p.chunkbuf,
                         (int64_t)p.nC * p.nC, 0, nn, 1, p.S, p.nC * p.nC);
      FSC_TRY(launch_gemm(ga, st));
      FSC_TRY(launch_gram_apply(ra, b, n0, nn, p.chunkbuf, p.grads, st));
    }
  }
  prof::mark(p.tc ? "readout_scatter" : "readout_gram_backward", st);
  // the readout only seeded atoms [0, nro): the rest of each evaluated layer starts at zero
  for (int k = 0; k + 1 < p.nint; ++k)
    if (p.nk[k] > p.nro &&
        cudaMemsetAsync(p.grads[k] + p.nro * NK * C, 0, sizeof(float) * (p.nk[k] - p.nro) * NK * C, st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset grads");
  if (cudaMemsetAsync(p.dY, 0, sizeof(float) * p.E * 12, st) != cudaSuccess) return fail(FSC_ERR_CUDA, "memset dY");
  return FSC_OK;
}

int backward_conv2(Ctx& c, int k) {
  Plan& p = c.p;
  const fsc_graph* g = c.g;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  const int C = p.C;
  {
    ConvArgs ca = conv_args(c, k);
    // dZ = (1/deg) G_k x W   (l3 blocks)
    const float* Wb = w->mix_bwd + (int64_t)(k - 1) * NP * C * C;
    int64_t boff = 0;
    for (int l3 = 0; l3 < 3; ++l3) {
      GemmArgs ga = gemm(p.grads[k] + KB(l3) * C, NK * C, C, Wb + boff, NP3(l3) * C, 0, p.zbuf + OFF3(l3) * C,
                         NZ * C, NP3(l3) * C, p.nk[k], 2 * l3 + 1, C, NP3(l3) * C);
      ga.deg_rowptr = g->row_ptr;
      FSC_TRY(run_gemm(ga, p.img_dz[k][l3], p.err, st));
      boff += (int64_t)NP3(l3) * C * C;
    }
    prof::mark("conv2_mix_backward_dz", st);
    ConvArgs cq = ca;
    cq.N = p.N;  // every receiver: the ones not evaluated zero their gate gradients
    if (g_conv2_path == 1)
      FSC_TRY(launch_conv2_q_tc(cq, p.feats[k - 1], p.zbuf, p.dgates + (int64_t)k * p.E * 12, p.dY, st));
    else
      FSC_TRY(launch_conv2_q(cq, p.feats[k - 1], p.zbuf, p.dgates + (int64_t)k * p.E * 12, p.dY, st));
    prof::mark("conv2_edge_backward_gates", st);
    ConvArgs cr = ca;
    cr.N = p.nk[k - 1];  // senders whose layer k-1 features were evaluated
    FSC_TRY(launch_conv2_r(cr, p.grads[k], p.zbuf, st));
    prof::mark("conv2_edge_backward_x", st);
    const float* Wx = w->mix_dx + (int64_t)(k - 1) * NP * C * C;
    boff = 0;
    for (int l1 = 0; l1 < 3; ++l1) {
      GemmArgs ga = gemm(p.zbuf + OFF1(l1) * C, NZ * C, NP1(l1) * C, Wx + boff, C, 0, p.grads[k - 1] + KB(l1) * C,
                         NK * C, C, p.nk[k - 1], 2 * l1 + 1, NP1(l1) * C, C);
      ga.accumulate = 1;
      FSC_TRY(run_gemm(ga, p.img_dx[k][l1], p.err, st));
      boff += (int64_t)NP1(l1) * C * C;
    }
    prof::mark("conv2_mix_backward_dx", st);
  }
  return FSC_OK;
}

int backward_conv1(Ctx& c) {
  Plan& p = c.p;
  const fsc_ictd_weights* w = c.w;
  cudaStream_t st = c.st;
  ConvArgs c1 = conv_args(c, 0);
  c1.N = p.N;
  FSC_TRY(launch_conv1_backward(c1, w->ai, w->vsp, p.grads[0], p.dgates, p.dY, st));
  prof::mark("conv1_backward", st);
  return FSC_OK;
}

// Per-graph sums in float64: out[b*W + w] += sum of vals over items of graph b.
// Items: atoms (W = 1, value e[n], counted when n < limit) or edges (W = 9, r_e (x) g_e).
template <int W>
__global__ void graph_reduce_kernel(const float* __restrict__ e, const float* __restrict__ edge_y,
                                    const float* __restrict__ grad, const int32_t* __restrict__ item_atom,
                                    const int32_t* __restrict__ batch, int64_t count, int64_t limit,
                                    double* __restrict__ out, const float* __restrict__ shift) {
  __shared__ double red[W][8];
  __shared__ int first_graph;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double v[W];
  int gid = -1;
#pragma unroll
  for (int w = 0; w < W; ++w) v[w] = 0.0;
  if (i < count) {
    const int64_t atom = item_atom ? item_atom[i] : i;
    gid = batch[atom];
    if (W == 1) {
      if (i < limit) v[0] = (double)e[i];
    } else {
      const float* r = shift ? shift + 3 * i : edge_y + 12 * i + 9;
      const float* g = grad + 3 * i;
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = 0; b < 3; ++b) v[(3 * a + b) % W] = (double)r[a] * (double)g[b];
    }
  }
  if (threadIdx.x == 0) first_graph = gid;
  __syncthreads();
  const bool uniform = __syncthreads_and(gid == first_graph || gid < 0);
  if (!uniform) {
    if (gid >= 0)
#pragma unroll
      for (int w = 0; w < W; ++w) atomicAdd(out + (int64_t)gid * W + w, v[w]);
    return;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    double t = v[w];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[w][warp] = t;
  }
  __syncthreads();
  if (threadIdx.x < W && first_graph >= 0) {
    double t = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[threadIdx.x][k];
    atomicAdd(out + (int64_t)first_graph * W + threadIdx.x, t);
  }
}

int prepare(Ctx& c, void* workspace, size_t bytes) {
  const fsc_graph* g = c.g;
  FSC_TRY(validate(c.cfg));
  FSC_REQUIRE(c.w && g, "weights/graph is null");
  FSC_REQUIRE(g->num_atoms >= 0 && g->num_edges >= 0 && g->num_graphs >= 1, "bad graph sizes");
  FSC_REQUIRE(g->num_atoms < (int64_t)INT32_MAX && g->num_edges < (int64_t)INT32_MAX,
              "graph too large for int32 indices");
  FSC_REQUIRE(g->num_graphs <= kMaxGraphs, "too many graphs per call (max 4096)");
  FSC_REQUIRE(g->num_local >= 0 && g->num_local <= g->num_atoms, "num_local out of range");
  Arena ar(workspace, bytes);
  layout(c.p, ar, c.cfg, g->num_atoms, g->num_edges);
  if (!ar.ok() || workspace == nullptr)
    return fail(FSC_ERR_CAPACITY, "workspace too small: need " + std::to_string(ar.off) + " bytes");
  c.p.B = g->num_graphs;
  Plan& p = c.p;
  for (int k = 0; k < p.nint; ++k) {
    const int64_t v = g->layer_atoms ? g->layer_atoms[k] : g->num_atoms;
    FSC_REQUIRE(v >= 0 && v <= g->num_atoms && (k == 0 || v <= p.nk[k - 1]),
                "layer_atoms must be non-increasing and within [0, num_atoms]");
    p.nk[k] = v;
  }
  p.nro = p.nk[p.nint - 1];
  FSC_REQUIRE(g->energy_weight || p.nro >= g->num_local, "layer_atoms[last] must be >= num_local");
  p.n_pad = ceil_div(std::max<int64_t>(p.nro, 1), 128) * 128;  // Fg stride of this call (<= allocated)
  return FSC_OK;
}

int run_forward_step(Ctx& c, int step, float* energy, float* atom_energy) {
  if (step == 0) {
    if (cudaMemsetAsync(c.p.energy_d, 0, sizeof(double) * kMaxGraphs * 19, c.st) != cudaSuccess ||
        cudaMemsetAsync(c.p.err, 0, sizeof(int) * 64, c.st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset accumulators");
    return forward_step0(c);
  }
  if (step < c.p.nint) return forward_conv2(c, step);
  FSC_TRY(forward_readout(c));
  const int H = c.p.hidden[c.p.n_hidden - 1];
  float* ebuf = atom_energy ? atom_energy : c.p.dxb;  // dxb is free until the backward starts
  FSC_TRY(launch_energy(c.p.act_post[c.p.n_hidden - 1], c.p.nro, H, c.w->out_v, c.w->out_c0, c.g->batch,
                        c.g->num_local, ebuf, nullptr, c.st));
  if (atom_energy && c.p.N > c.p.nro &&
      cudaMemsetAsync(atom_energy + c.p.nro, 0, sizeof(float) * (c.p.N - c.p.nro), c.st) != cudaSuccess)
    return fail(FSC_ERR_CUDA, "memset atom_energy");
  if (c.p.nro > 0) {
    graph_reduce_kernel<1><<<(unsigned)ceil_div(c.p.nro, 256), 256, 0, c.st>>>(
        ebuf, nullptr, nullptr, nullptr, c.g->batch, c.p.nro, c.g->num_local, c.p.energy_d, nullptr);
    FSC_TRY(check_launch("graph_reduce_kernel<1>"));
  }
  if (energy) {
    finalize_kernel<<<(unsigned)ceil_div(c.p.B, 256), 256, 0, c.st>>>(c.p.energy_d, nullptr, c.p.B, energy, nullptr);
    FSC_TRY(check_launch("finalize_kernel"));
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

// radial / direction backward, forces, virial and cell gradient from dgates and dY
int run_backward_edges(Ctx& c, fsc_ictd_outputs* out) {
  const fsc_graph* g = c.g;
  EdgeBwdArgs eb{};
  eb.E = c.p.E; eb.src = g->src; eb.batch = g->batch; eb.tables = c.w->tables; eb.rad = radial(c.w);
  eb.nint = c.p.nint; eb.nb = c.p.nb; eb.basis_kind = c.cfg->basis_kind; eb.rc = c.cfg->max_radius;
  eb.edge_y = c.p.edge_y; eb.dgates = c.p.dgates; eb.dY = c.p.dY;
  eb.edge_grad = out->edge_grad ? out->edge_grad : c.p.edge_grad;
  eb.virial = nullptr;
  if (c.p.rtc) {
    RadialTcArgs ra{};
    ra.E = c.p.E; ra.rad = eb.rad; ra.nint = c.p.nint; ra.nb = c.p.nb; ra.basis_kind = eb.basis_kind; ra.rc = eb.rc;
    ra.tables = c.w->tables; ra.edge_y = c.p.edge_y; ra.dgates = c.p.dgates; ra.dY = c.p.dY;
    ra.edge_grad = eb.edge_grad; ra.err = c.p.err;
    FSC_TRY(launch_radial_bwd_tc(ra, c.st));
  } else {
    FSC_TRY(launch_edge_backward(eb, c.st));
  }
  prof::mark("edge_backward", c.st);
  if (out->forces) FSC_TRY(launch_forces(g->row_ptr, g->tr_ptr, g->tr_eid, eb.edge_grad, out->forces, c.p.N, c.st));
  const int64_t nfin = 9 * c.p.B;
  if (out->virial) {
    if (cudaMemsetAsync(c.p.virial_d, 0, sizeof(double) * 9 * kMaxGraphs, c.st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset virial");
    if (c.p.E > 0) {
      graph_reduce_kernel<9><<<(unsigned)ceil_div(c.p.E, 256), 256, 0, c.st>>>(
          nullptr, c.p.edge_y, eb.edge_grad, g->src, g->batch, c.p.E, c.p.E, c.p.virial_d, nullptr);
      FSC_TRY(check_launch("graph_reduce_kernel<9>"));
    }
    finalize_kernel<<<(unsigned)ceil_div(nfin, 256), 256, 0, c.st>>>(c.p.energy_d, c.p.virial_d, c.p.B, nullptr,
                                                                     out->virial);
    FSC_TRY(check_launch("finalize_kernel (virial)"));
  }
  if (out->cell_grad) {
    if (cudaMemsetAsync(c.p.cellg_d, 0, sizeof(double) * 9 * kMaxGraphs, c.st) != cudaSuccess)
      return fail(FSC_ERR_CUDA, "memset cell grad");
    if (c.p.E > 0) {
      graph_reduce_kernel<9><<<(unsigned)ceil_div(c.p.E, 256), 256, 0, c.st>>>(
          nullptr, c.p.edge_y, eb.edge_grad, g->src, g->batch, c.p.E, c.p.E, c.p.cellg_d, g->shift);
      FSC_TRY(check_launch("graph_reduce_kernel<9> (cell)"));
    }
    finalize_kernel<<<(unsigned)ceil_div(nfin, 256), 256, 0, c.st>>>(c.p.energy_d, c.p.cellg_d, c.p.B, nullptr,
                                                                     out->cell_grad);
    FSC_TRY(check_launch("finalize_kernel (cell)"));
  }
  prof::mark("forces_virial", c.st);
  return FSC_OK;
}

}  // namespace

int gemm_path() { return g_gemm_path; }

int launch_graph_reduce(int width, const float* e, const float* edge_y, const float* grad, const int32_t* item_atom,
                        const int32_t* batch, int64_t count, int64_t limit, double* out, const float* shift,
                        cudaStream_t st) {
  if (count <= 0) return FSC_OK;
  const unsigned blocks = (unsigned)ceil_div(count, 256);
  if (width == 1)
    graph_reduce_kernel<1><<<blocks, 256, 0, st>>>(e, edge_y, grad, item_atom, batch, count, limit, out, shift);
  else
    graph_reduce_kernel<9><<<blocks, 256, 0, st>>>(e, edge_y, grad, item_atom, batch, count, limit, out, shift);
  return check_launch("graph_reduce_kernel");
}

}  // namespace fsc

extern "C" {

size_t fsc_ictd_workspace_bytes(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges) {
  if (!cfg || fsc::validate(cfg) != FSC_OK) return 0;
  fsc::Plan p{};
  fsc::Arena ar(nullptr, 0);
  fsc::layout(p, ar, cfg, num_atoms, num_edges);
  return ar.off;
}

int fsc_ictd_forward(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, float* energy,
                     float* atom_energy, void* workspace, size_t workspace_bytes, void* stream) {
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  return fsc::run_forward(c, energy, atom_energy);
}

int fsc_ictd_backward(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g,
                      fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(out != nullptr, "outputs required");
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  return fsc::run_backward(c, out);
}

int fsc_ictd_energy_forces(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g,
                           fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(out && out->forces && out->energy, "outputs (energy, forces) required");
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  FSC_TRY(fsc::run_forward(c, out->energy, out->atom_energy));
  return fsc::run_backward(c, out);
}

int fsc_ictd_forward_step(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int step,
                          float* energy, float* atom_energy, void* workspace, size_t workspace_bytes, void* stream) {
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  FSC_REQUIRE(step >= 0 && step <= c.p.nint, "forward step out of range [0, num_interaction]");
  return fsc::run_forward_step(c, step, energy, atom_energy);
}

int fsc_ictd_backward_step(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int step,
                           fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream) {
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  FSC_REQUIRE(step >= 0 && step <= c.p.nint, "backward step out of range [0, num_interaction]");
  FSC_REQUIRE(step > 0 || out != nullptr, "outputs required for backward step 0");
  return fsc::run_backward_step(c, step, out);
}

int fsc_ictd_feature_buffer(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                            int which, int layer, float** out) {
  FSC_REQUIRE(out && workspace, "workspace and output pointer required");
  FSC_TRY(fsc::validate(cfg));
  FSC_REQUIRE(which == 0 || which == 1, "which must be 0 (features) or 1 (gradients)");
  FSC_REQUIRE(layer >= 0 && layer < cfg->num_interaction, "layer out of range");
  fsc::Plan p{};
  fsc::Arena ar(workspace, (size_t)-1);
  fsc::layout(p, ar, cfg, num_atoms, num_edges);
  *out = which == 0 ? p.feats[layer] : p.grads[layer];
  return FSC_OK;
}

int fsc_ictd_energy(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, float* energy,
                    float* atom_energy, void* workspace, size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(energy, "energy output required");
  return fsc_ictd_forward(cfg, w, g, energy, atom_energy, workspace, workspace_bytes, stream);
}

int fsc_ictd_heads(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int nheads,
                   const int32_t* block_host, const float* weights, float* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  FSC_REQUIRE(nheads >= 1 && nheads <= 4, "1..4 heads");
  FSC_REQUIRE(block_host && weights && out, "head blocks, weights and output required");
  fsc::Ctx c{cfg, w, g, fsc::Plan{}, fsc::as_stream(stream)};
  FSC_TRY(fsc::prepare(c, workspace, workspace_bytes));
  for (int h = 0; h < nheads; ++h)
    FSC_REQUIRE(block_host[h] >= 0 && block_host[h] < c.p.ngram, "head block index out of range");
  return fsc::launch_heads(fsc::readout_args(c), g->batch, nheads, block_host, weights, c.p.heads_d, out,
                           g->num_graphs, c.st);
}

int64_t fsc_ictd_tables_floats(void) { return ictd2::TAB_FLOATS; }

int fsc_ictd_status(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                    void* stream, int* status_host) {
  FSC_REQUIRE(status_host && workspace, "status output and workspace required");
  FSC_TRY(fsc::validate(cfg));
  fsc::Plan p{};
  fsc::Arena ar(workspace, (size_t)-1);
  fsc::layout(p, ar, cfg, num_atoms, num_edges);
  cudaStream_t st = fsc::as_stream(stream);
  if (cudaMemcpyAsync(status_host, p.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return fsc::fail(FSC_ERR_CUDA, "status readback");
  return FSC_OK;
}

void fsc_ictd_set_readout_path(int path) { fsc::g_readout_path = path; }
void fsc_ictd_set_radial_path(int path) { fsc::g_radial_path = path; }
void fsc_ictd_set_gemm_path(int path) { fsc::g_gemm_path = path; }
void fsc_ictd_set_conv2_path(int path) { fsc::g_conv2_path = path; }

void fsc_profile_enable(int enable) {
  fsc::prof::enabled = enable != 0;
  fsc::prof::count = 0;
}

int fsc_profile_read(const char** names, float* ms, int max_stages) {
  using namespace fsc::prof;
  if (count < 2) {
    count = 0;
    return 0;
  }
  if (cudaEventSynchronize(events[count - 1]) != cudaSuccess) return -1;
  int n = 0;
  for (int i = 1; i < count && n < max_stages; ++i, ++n) {
    names[n] = fsc::prof::names[i];
    cudaEventElapsedTime(&ms[n], events[i - 1], events[i]);
  }
  count = 0;
  return n;
}

}  // extern "C"
