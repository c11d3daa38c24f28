// Internal kernel-launch interfaces shared by the .cu files (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fsc {

struct RadialW {
  const float *w1, *b1, *w2, *b2, *w3, *b3;
};

struct EdgeFwdArgs {
  int64_t E;
  const float* pos;
  const int32_t* src;
  const int32_t* dst;
  const int32_t* batch;
  const float* cell;
  const float* shift;
  const float* tables;
  RadialW rad;
  int nint, nb, basis_kind;
  float rc;
  float* edge_y;   // [E][12]: Y[9], r[3]
  float* gates;    // [nint][E][12]
};

struct EdgeBwdArgs {
  int64_t E;
  const int32_t* src;
  const int32_t* batch;
  const float* tables;
  RadialW rad;
  int nint, nb, basis_kind;
  float rc;
  const float* edge_y;
  const float* dgates;   // [nint][E][12]
  const float* dY;       // [E][12]
  float* edge_grad;      // [E][3]
  double* virial;        // [B][9] or null (accumulated)
};

int launch_edge_forward(const EdgeFwdArgs& a, cudaStream_t st);
int launch_edge_geom(const EdgeFwdArgs& a, cudaStream_t st);

// Radial MLPs on tcgen05 (radial_tc.cu).
struct RadialTcArgs {
  int64_t E;
  RadialW rad;
  int nint, nb, basis_kind;
  float rc;
  const float* tables;   // ypoly
  const float* edge_y;   // [E][12]
  float* gates;          // forward output [nint][E][12]
  const float* dgates;   // backward input [nint][E][12]
  const float* dY;       // backward input [E][12]
  float* edge_grad;      // backward output [E][3]
  int* err;              // first failing wait site (0 = ok)
  float* hout;           // forward: non-null -> write h2 [nint][E][64] instead of gates
  const float* hout_grad;// backward: non-null -> dE/dh2 [nint][E][64]; dE/d|r| summed into edge_grad[e][0]
};
bool radial_tc_supported(int nb);
int launch_radial_fwd_tc(const RadialTcArgs& a, cudaStream_t st);
int launch_radial_bwd_tc(const RadialTcArgs& a, cudaStream_t st);
int launch_edge_backward(const EdgeBwdArgs& a, cudaStream_t st);
int launch_forces(const int32_t* row_ptr, const int32_t* tr_ptr, const int32_t* tr_eid, const float* g,
                  float* F, int64_t N, cudaStream_t st);
int launch_edge_dst(const int32_t* row_ptr, int32_t* dst, int64_t N, cudaStream_t st);
int launch_transpose_aux(const int32_t* row_ptr, const int32_t* dst, const int32_t* tr_eid, int64_t N, int64_t E,
                         int32_t* tr_dst, float* invdeg, cudaStream_t st);

struct ConvArgs {
  int64_t N, E;
  int C;
  const int32_t* row_ptr;
  const int32_t* src;
  const int32_t* dst;
  const int32_t* tr_ptr;
  const int32_t* tr_eid;
  const int32_t* species;
  const float* tables;
  const float* edge_y;   // [E][12]
  const float* gates;    // [E][12] of this layer
  const float* field;    // [B][3] or null: added to the l = 1 harmonic in conv1
  const int32_t* batch;  // [N] graph of each atom (for field)
  // Receptive-field restriction (all default to "no restriction" when left at 0 / null):
  int64_t n_active;      // conv1_backward / conv2_q: nodes in [n_active, N) only zero their dgates
  int64_t dst_limit;     // conv2_r: edges whose dst >= dst_limit carry no gradient
  int64_t src_limit;     // conv2_z: an edge whose src >= src_limit is skipped and flags err (70)
  int* err;
  const int32_t* tr_dst; // [E] receiver of edge tr_eid[t] (conv2_r)
  const float* invdeg;   // [N] 1 / max(in-degree, 1) (conv2_r)
  int* work;             // conv2 z / r / q: node counter for dynamic scheduling (zeroed by the
                         // launcher; null: one node per warp, one launch-wide grid)
};

// conv1: f1[n][k][c]
int launch_conv1_forward(const ConvArgs& a, const float* ai, const float* vsp, float* f1, cudaStream_t st);
// conv1 backward: dgates (this layer, all 11 written) and dY (+=)
int launch_conv1_backward(const ConvArgs& a, const float* ai, const float* vsp, const float* G1,
                          float* dgates, float* dY, cudaStream_t st);
// conv2 forward: Z[n][35][C] (not yet divided by the degree)
int launch_conv2_z(const ConvArgs& a, const float* x, float* Z, cudaStream_t st);
// conv2 backward, src-centric: R[s][35][C] = sum_{e: src=s} sum_k Yt * G[dst]/deg(dst)
int launch_conv2_r(const ConvArgs& a, const float* G, float* R, cudaStream_t st);
// conv2 backward, dst-centric: dgates[e][p], dY[e][k] += from x[src] and dZ[dst]
int launch_conv2_q(const ConvArgs& a, const float* x, const float* dZ, float* dgates, float* dY,
                   cudaStream_t st);
// the same on the tensor cores (conv2_q_tc.cu); needs a.work
int launch_conv2_q_tc(const ConvArgs& a, const float* x, const float* dZ, float* dgates, float* dY,
                      cudaStream_t st);

// Generic fp32 GEMM with two-level row addressing:
//   row (g, r), g < G, r < R:  A + g*a_gs + r*a_rs (K contiguous), C + g*c_gs + r*c_rs (N contiguous)
//   B[k][n] = b_trans ? B[n*ldb + k] : B[k*ldb + n]
//   C = scale_g * (A @ B) + bias  (+ C if accumulate);  scale_g = 1/max(deg,1) from deg_rowptr if set
struct GemmArgs {
  const float* A;
  int64_t a_gs, a_rs;
  const float* B;
  int64_t ldb;
  int b_trans;
  float* C;
  int64_t c_gs, c_rs;
  int64_t G;
  int R, K, N;
  const int32_t* deg_rowptr;
  const float* bias;
  int accumulate;
  float alpha;  // extra scale of the product (0 means 1)
  int precise;  // long K with heavy cancellation: shortest tensor-core chains
};
int launch_gemm(const GemmArgs& a, cudaStream_t st);

// The same GEMM on tcgen05 (gemm_tc.cu): A staged by TMA (two-level rows as a 3-D tensor map),
// B from a pre-formatted hi/lo image (gemm_image_kernel), 3xTF32.  Needs K % 4 == 0, A and its
// row strides 16-byte aligned, rows of one group contiguous (a_rs >= K) when R > 1.
bool gemm_tc_supported(const GemmArgs& a);
int gemm_tc_nt(int N, int K);
int64_t gemm_image_floats(int K, int N);
int launch_gemm_tc(const GemmArgs& a, const float* bimg, int* err, cudaStream_t st);
constexpr int kMaxImageJobs = 32;
struct GemmImageJob {
  const float* B;     // logical B[k][n] = b_trans ? B[n*ldb + k] : B[k*ldb + n]
  int64_t ldb;
  int b_trans, K, N, NT, ntiles;
  float* out;         // gemm_image_floats(K, N) floats
};
struct GemmImageJobs {
  GemmImageJob job[kMaxImageJobs];
};
int launch_gemm_images(const GemmImageJobs& jobs, int njobs, cudaStream_t st);
// Collects image jobs and launches them in batches of kMaxImageJobs.
struct GemmImageBatch {
  GemmImageJobs jobs{};
  int n = 0;
  int add(const float* B, int64_t ldb, int b_trans, int K, int N, float* out, cudaStream_t st);
  int flush(cudaStream_t st);
};
// Tensor-core GEMM when an image is given and the shape qualifies, else the CUDA-core kernel.
int run_gemm(const GemmArgs& a, const float* img, int* err, cudaStream_t st);
// Process-wide GEMM path (fsc_ictd_set_gemm_path): 0 = tensor cores where supported.
int gemm_path();
// Per-graph float64 sums, block-reduced where a block's items share one graph:
// width 1: out[b] += e[i] over atoms i < min(count, limit) of graph b;
// width 9: out[b][3p+q] += r_i[p] g_i[q] over edges i (r = edge_y[i][9..11], or shift[i] if given),
// graph of edge i = batch[item_atom[i]].
int launch_graph_reduce(int width, const float* e, const float* edge_y, const float* grad, const int32_t* item_atom,
                        const int32_t* batch, int64_t count, int64_t limit, double* out, const float* shift,
                        cudaStream_t st);

// Readout (pure_cartesian_ictd_layers_full.py:956-1054)
struct ReadoutArgs {
  int64_t N;
  int C, nint, S;
  const float* feats[8];       // nint pointers to [N][9][C]
  const float* tables;
  const int32_t* xmap;         // [nrows] Gram operand element -> (layer << 16) | (k*C + c), -1 = zero
  int o3;                      // MainNet input has a zero 1e slot after [0e | scalars]
  int ngram;                   // Gram blocks
  int goff[4], gl[4];          // block offsets (elements) and l
};
// Packed Gram of Gram block b for nodes [n0, n0+nn): Gp[n][pair] = sum_m t[c][m] t[d][m]
int launch_gram_pack(const ReadoutArgs& a, int b, int64_t n0, int64_t nn, const int32_t* pairs, int64_t npairs,
                     float* Gp, cudaStream_t st);
// grads at t_b[n][c'][m] += 2 sum_d H[n][c'][d] t_b[n][d][m] for nodes [n0, n0+nn), H [nn][nC][nC]
int launch_gram_apply(const ReadoutArgs& a, int b, int64_t n0, int64_t nn, const float* H, float* const* grads,
                      cudaStream_t st);
// Physical-tensor heads: out[h][graph][m] = sum_n sum_c w[h][c] t_{block[h]}[n][c][m]; acc: double
// scratch [nheads][4096][5] (graphs < 4096); blocks: host array of <= 4 block indices; w on the device.
int launch_heads(const ReadoutArgs& a, const int32_t* batch, int nheads, const int32_t* blocks, const float* w,
                 double* acc, float* out, int64_t B, cudaStream_t st);
int launch_p5_forward(const ReadoutArgs& a, const float* scalars, float* p5, cudaStream_t st);
// Writes (not accumulates) grads[k] for all components, and dscalars.
int launch_p5_backward(const ReadoutArgs& a, const float* scalars, const float* dp5, float* const* grads,
                       float* dscalars, cudaStream_t st);
// Tensor-core readout (readout_tc.cu)
// Fg / dFg (Gram operand and its gradient) are tile-blocked: node n, row r at
//   (n / 128) * nrows * 128 + r * 128 + n % 128,
// so one tile's rows are 512-byte lines at compile-time-friendly offsets.
struct ReadoutTcArgs {
  int64_t N, n_pad;     // nodes, padded node count (multiple of 128)
  int nC, S;
  int64_t nrows;        // Gram operand rows per node
  const float* Fg;      // [n_pad / 128][nrows][128] Gram operand
  const float* wimg;    // pre-formatted W blocks (hi/lo), forward or backward order
  float* scalars;       // forward output [N][S]
  const float* dscal;   // backward input [N][S]
  float* dFg;           // backward output, layout of Fg
  const float* gmax;    // [ngram][n_pad] max t^2 per node over each Gram block's rows (fp16 range scaling)
  int* err;             // first failing wait site (0 = ok)
  int ngram;            // Gram blocks (rows of block b start at goff[b], m-width 2 gl[b] + 1)
  int goff[4], gl[4];
};
bool readout_tc_supported(int nC, int S);
int64_t readout_tc_blocks(int nC, int ngram, bool backward);
int launch_readout_fwd_tc(const ReadoutTcArgs& a, cudaStream_t st);
int launch_readout_bwd_tc(const ReadoutTcArgs& a, cudaStream_t st);
struct FgArgs {
  int64_t N, n_pad;
  int C, nint;
  const float* feats[8];
  float* grads[8];
  const int32_t* xinv;  // [nint][9*C] storage (layer, k*C + c) -> Gram operand row
  float* Fg;
  const float* dFg;
  int64_t nrows;        // Gram operand rows
  float* gmax;          // gather: [ngram][n_pad] max t^2 over the rows of each Gram block (zeroed by the caller)
  int ngram;
  int goff[4];          // first row of each Gram block
};
int launch_fg_gather(const FgArgs& a, cudaStream_t st);
int launch_fg_scatter_add(const FgArgs& a, cudaStream_t st);

// LayerNorm over the last dim (rows x D), eps 1e-5, optional SiLU after.
int launch_layernorm(const float* X, int64_t rows, int D, const float* gamma, const float* beta, int silu,
                     float* Y, cudaStream_t st);
// Backward: dX = LN_backward(dY * (silu ? silu'(u) : 1)), u = LN(X)
int launch_layernorm_backward(const float* X, const float* dY, int64_t rows, int D, const float* gamma,
                              const float* beta, int silu, float* dX, cudaStream_t st);
// e[n] = x[n] . v + c0;  energy[batch[n]] += e[n] for n < num_local (double accumulate)
int launch_energy(const float* x, int64_t N, int H, const float* v, float c0, const int32_t* batch,
                  int64_t num_local, float* atom_energy, double* energy, cudaStream_t st);
// dx[n] = v * weight[n]  (weight NULL: 1 for n < num_local, else 0)
int launch_energy_seed(int64_t N, int H, const float* v, const float* weight, int64_t num_local, float* dx,
                       cudaStream_t st);

// Optional per-stage CUDA-event timing (engine.cu).
namespace prof {
void mark(const char* name, cudaStream_t st);
}

}  // namespace fsc
