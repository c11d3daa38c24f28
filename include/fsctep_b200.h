/*
 * fsctep_b200 -- C ABI of the B200-native (sm_100a) FSCTEP message-passing hot path.
 *
 * Everything here takes plain pointers and sizes: no torch types.  All data
 * pointers are DEVICE pointers unless a comment says otherwise; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Every function
 * returns an fsc_status; on failure fsc_last_error() gives a message (per host
 * thread).  Nothing in this library allocates device memory: callers pass
 * outputs and workspaces they own (sizes from the *_workspace_bytes queries).
 *
 * Reference interfaces replaced (paths inside the Parity-LRX/FSCTEP project):
 *   - the `_C_ictd_tp` pybind operator family       csrc/ictd_tp.cpp:498-523
 *   - the per-edge TP layers + autograd force/virial pure_cartesian_ictd_layers_full.py:867-1078,
 *     evaluation/calculator.py:152-159, training/trainer.py:1213-1310
 *   - the LibTorch engine E/F/virial call           lammps_user_mfftorch/src/USER-MFFTORCH/
 *                                                   mff_torch_engine.cpp:740-864 (MFFTorchEngine::compute)
 *   - the neighbour search                          utils/graph_utils.py:192-258 (radius_graph_pbc_gpu)
 */
#ifndef FSCTEP_B200_H
#define FSCTEP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FSC_OK = 0,
  FSC_ERR_ARGUMENT = 1,     /* bad shape / pointer / unsupported size        */
  FSC_ERR_CUDA = 2,         /* a CUDA runtime call or kernel launch failed   */
  FSC_ERR_UNSUPPORTED = 3,  /* configuration outside what the kernels cover  */
  FSC_ERR_CAPACITY = 4      /* an output buffer is too small (see message)   */
} fsc_status;

typedef enum { FSC_F32 = 0, FSC_F64 = 1 } fsc_dtype;

/* ---- library ------------------------------------------------------------ */
const char* fsc_last_error(void);
int fsc_version(void);
/* 1 when the library was built with its CUDA kernels (always, for this build).
 * Replaces `_C_ictd_tp.has_cuda()` (csrc/ictd_tp.cpp:516-522). */
int fsc_has_cuda(void);
/* FP32 CUDA-core throughput probe: launches `blocks` x 256 threads, each running 8 independent
 * fp32 FMA chains of 16 * iters steps (packed != 0: two-lane packed FMAs), and writes the launch's
 * FLOP count to *flops; the caller times it with events on `stream`.  `out`: a device buffer of
 * blocks * 256 floats (written only to keep the chains live).  No reference counterpart: the
 * measured denominator of the CUDA-core kernels' FP32 roofline. */
int fsc_fp32_fma_probe(int packed, int blocks, int iters, float* out, double* flops, void* stream);
/* Bounded-wait check: one thread of one block runs the mbarrier wait that every tensor-core
 * kernel of this library uses on a fresh barrier of arrival count 1 that nothing arrives at,
 * waiting for phase `parity`.  Parity 0 is never completed: the wait gives up after its limit
 * (about 2e9 SM clock cycles, ~1 s), writes `where` to *err_dev (a device int, if it was 0) and
 * the kernel returns; parity 1 counts as the completed previous phase and returns at once.  No
 * reference counterpart: it shows that a stalled pipeline ends with an error status that the host
 * reads, leaving the context usable. */
int fsc_bounded_wait_probe(int parity, int where, int* err_dev, void* stream);

/* ---- `_C_ictd_tp` operator family (csrc/ictd_tp.cpp:137-497) -------------
 * Shapes follow the reference TORCH_CHECKs (csrc/ictd_tp.cpp:78-108):
 *   a (B, I, m1), b (B, J, m2), u (m1*m2, P*K), y (B, P, K, I*J),
 *   w (P, O, I*J), gates (B, P), out (B, O, K).  All C-contiguous.
 * J (mul_in2) may be any value >= 1 (the reference CUDA path needs J == 1).
 * Outputs are fully overwritten (no accumulation).                           */
int fsc_project_bucket_forward(int dtype, const void* a, const void* b, const void* u, void* y,
                               int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2,
                               int64_t P, int64_t K, void* stream);        /* ictd_tp.cpp:137 */
int fsc_project_bucket_transpose_a(int dtype, const void* grad_y, const void* b, const void* u,
                                   void* grad_a, int64_t B, int64_t I, int64_t J, int64_t m1,
                                   int64_t m2, int64_t P, int64_t K, void* stream); /* :175 */
int fsc_project_bucket_transpose_b(int dtype, const void* grad_y, const void* a, const void* u,
                                   void* grad_b, int64_t B, int64_t I, int64_t J, int64_t m1,
                                   int64_t m2, int64_t P, int64_t K, void* stream); /* :210 */
int fsc_project_bucket_transpose_u(int dtype, const void* grad_y, const void* a, const void* b,
                                   void* grad_u, int64_t B, int64_t I, int64_t J, int64_t m1,
                                   int64_t m2, int64_t P, int64_t K, void* stream); /* :242 */
int fsc_mix_bucket_forward(int dtype, const void* y, const void* w, const void* gates, void* out,
                           int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O,
                           void* stream);                                  /* :270 */
int fsc_mix_bucket_transpose_y(int dtype, const void* grad_out, const void* w, const void* gates,
                               void* grad_y, int64_t B, int64_t P, int64_t K, int64_t IJ,
                               int64_t O, void* stream);                   /* :293 */
int fsc_mix_bucket_transpose_w(int dtype, const void* grad_out, const void* y, const void* gates,
                               void* grad_w, int64_t B, int64_t P, int64_t K, int64_t IJ,
                               int64_t O, void* stream);                   /* :322 */
int fsc_mix_bucket_transpose_g(int dtype, const void* grad_out, const void* y, const void* w,
                               void* grad_g, int64_t B, int64_t P, int64_t K, int64_t IJ,
                               int64_t O, void* stream);                   /* :346 */
/* y-free fused forward of one same-kdim bucket: out = mix(project(a,b,u), w, gates) (:372). */
int fsc_bucketed_tp_forward(int dtype, const void* a, const void* b, const void* u, const void* w,
                            const void* gates, void* out, int64_t B, int64_t I, int64_t J,
                            int64_t m1, int64_t m2, int64_t P, int64_t K, int64_t O, void* stream);
/* Double-backward fused terms (ictd_tp.cpp:387-495, ictd_tp_cuda.cu:528-534, 780-786):
 *   grad_h  = PF(gga,b,u) + PF(a,ggb,u) + PF(a,b,ggu)        -> (B,P,K,I*J)
 *   grad_a2 = PAT(h,ggb,u) + PAT(h,b,ggu)                    -> (B,I,m1)
 *   grad_b2 = PBT(h,gga,u) + PBT(h,a,ggu)                    -> (B,J,m2)
 *   grad_u2 = PUT(h,gga,b) + PUT(h,a,ggb)                    -> (m1*m2,P*K)
 *   grad_g_out = MF(ggy,w,g) + MF(y,ggw,g) + MF(y,w,ggg)     -> (B,O,K)
 *   grad_y2 = MYT(g_out,ggw,g) + MYT(g_out,w,ggg)            -> (B,P,K,IJ)
 *   grad_w2 = MWT(g_out,ggy,g) + MWT(g_out,y,ggg)            -> (P,O,IJ)
 *   grad_g2 = MGT(g_out,ggy,w) + MGT(g_out,y,ggw)            -> (B,P)              */
int fsc_project_dbl_bwd_grad_h(int dtype, const void* a, const void* gga, const void* b,
                               const void* ggb, const void* u, const void* ggu, void* out,
                               int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2,
                               int64_t P, int64_t K, void* stream);
int fsc_project_dbl_bwd_grad_a(int dtype, const void* h, const void* b, const void* ggb,
                               const void* u, const void* ggu, void* out, int64_t B, int64_t I,
                               int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                               void* stream);
int fsc_project_dbl_bwd_grad_b(int dtype, const void* h, const void* a, const void* gga,
                               const void* u, const void* ggu, void* out, int64_t B, int64_t I,
                               int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                               void* stream);
int fsc_project_dbl_bwd_grad_u(int dtype, const void* h, const void* a, const void* gga,
                               const void* b, const void* ggb, void* out, int64_t B, int64_t I,
                               int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                               void* stream);
int fsc_mix_dbl_bwd_grad_g_out(int dtype, const void* y, const void* ggy, const void* w,
                               const void* ggw, const void* gates, const void* ggg, void* out,
                               int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O,
                               void* stream);
int fsc_mix_dbl_bwd_grad_y(int dtype, const void* g_out, const void* w, const void* ggw,
                           const void* gates, const void* ggg, void* out, int64_t B, int64_t P,
                           int64_t K, int64_t IJ, int64_t O, void* stream);
int fsc_mix_dbl_bwd_grad_w(int dtype, const void* g_out, const void* y, const void* ggy,
                           const void* gates, const void* ggg, void* out, int64_t B, int64_t P,
                           int64_t K, int64_t IJ, int64_t O, void* stream);
int fsc_mix_dbl_bwd_grad_g(int dtype, const void* g_out, const void* y, const void* ggy,
                           const void* w, const void* ggw, void* out, int64_t B, int64_t P,
                           int64_t K, int64_t IJ, int64_t O, void* stream);

/* ---- neighbour list (utils/graph_utils.py:192-258) ------------------------
 * Edges (src=i, dst=j, S) with |(pos[j] + S@cell) - pos[i]| < cutoff, S in
 * {-1,0,1}^3 on periodic axes ({0} on open ones), no self pair at S = 0;
 * float64 arithmetic in the fixed order documented in oracle/neighbors.py.
 * Output is a CSR by dst: row_ptr[N+1]; per edge src[e] and the packed image
 * index sidx[e] = (S0+1)*9 + (S1+1)*3 + (S2+1); rows sorted by (src, sidx).
 * Frames: atoms of frame g are [frame_ptr[g], frame_ptr[g+1]) (host array);
 * edges never cross frames.  `cell` is [num_frames][3][3] (device), rows =
 * lattice vectors.  The builder uses a cell list when a frame is periodic and
 * orthorhombic with all positions inside [0, L), else an all-pairs search.
 * Two phases: count (fills row_ptr, returns the edge count in *num_edges,
 * host; workspace >= fsc_neighbor_workspace_bytes(N, 0)) then fill (needs
 * capacity >= *num_edges and workspace >= fsc_neighbor_workspace_bytes(N, E)).
 * Both phases synchronise `stream` (the edge count is read back to the host). */
size_t fsc_neighbor_workspace_bytes(int64_t num_atoms, int64_t num_edges);
/* pos [N][3] (device), cell [num_frames][3][3] (device); pbc_host[3] (host). */
int fsc_neighbor_count(const double* pos, const double* cell, const int64_t* frame_ptr_host,
                       int64_t num_frames, int64_t num_atoms, const int32_t* pbc_host,
                       double cutoff, int32_t* row_ptr, int64_t* num_edges_host,
                       void* workspace, size_t workspace_bytes, void* stream);
int fsc_neighbor_fill(const double* pos, const double* cell, const int64_t* frame_ptr_host,
                      int64_t num_frames, int64_t num_atoms, const int32_t* pbc_host,
                      double cutoff, const int32_t* row_ptr, int32_t* src, int8_t* sidx,
                      int64_t capacity, void* workspace, size_t workspace_bytes, void* stream);
/* Transpose CSR (edges grouped by src, ascending edge id within a group). */
size_t fsc_csr_transpose_workspace_bytes(int64_t num_atoms, int64_t num_edges);
int fsc_csr_transpose(const int32_t* row_ptr, const int32_t* src, int64_t num_atoms,
                      int64_t num_edges, int32_t* tr_ptr, int32_t* tr_eid, void* workspace,
                      size_t workspace_bytes, void* stream);
/* Per-source cap of radius_graph_pbc_gpu's max_num_neighbors (utils/graph_utils.py:192, 240):
 * the reference runs one torch_cluster radius search per image shift, which keeps for every
 * source i the first max_num_neighbors candidates j (ascending j) inside the cutoff, the self
 * pair at S = 0 taking a slot before it is dropped.  Input: a CSR from fsc_neighbor_fill and
 * its transpose; output: the capped CSR (out_row_ptr[N+1], out_src / out_sidx with room for
 * num_edges entries, rows in the input order) and its edge count (host).  Synchronises
 * `stream`.  Workspace >= fsc_neighbor_cap_workspace_bytes(N, E).                            */
size_t fsc_neighbor_cap_workspace_bytes(int64_t num_atoms, int64_t num_edges);
int fsc_neighbor_cap(const int32_t* row_ptr, const int32_t* src, const int8_t* sidx,
                     int64_t num_atoms, int64_t num_edges, const int32_t* tr_ptr,
                     const int32_t* tr_eid, int max_num_neighbors, int32_t* out_row_ptr,
                     int32_t* out_src, int8_t* out_sidx, int64_t* out_num_edges_host,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free transpose, for callers that cannot call cudaMalloc (a host program that
 * hands all device memory to its own fixed pool, an FFI binding without a device allocator,
 * a plugin inside another program that owns the device's memory).  No counterpart in the reference.  Same result as fsc_csr_transpose,
 * but its scratch is a file-scope __device__ array of this library (about 19 MiB, held on
 * every GPU that loads the library until exit), so it accepts at most 262,144 atoms and
 * 4,194,304 edges and returns FSC_ERR_CAPACITY beyond that.  It allocates nothing.  The
 * first call on a device looks up the array's device address (cudaGetSymbolAddress, once
 * per device, with that device current); make that first call before any stream capture.
 * All calls share the one array and it keeps the last call's contents: calls that overlap
 * on the GPU (different streams, or different host threads on one device) race.        */
int fsc_csr_transpose_static(const int32_t* row_ptr, const int32_t* src, int64_t num_atoms,
                             int64_t num_edges, int32_t* tr_ptr, int32_t* tr_eid, void* stream);

/* ---- pure-cartesian-ictd energy + forces + virial -------------------------
 * One call = PureCartesianICTDTransformerLayer forward (pure_cartesian_ictd_layers_full.py:
 * 867-1078) followed by a hand-written backward giving dE/dpos and the per-edge
 * dE/dr (no autograd replay).  Covers lmax = 2, path_policy "full",
 * channels 32 or 64, any num_interaction in [2, 8], number_of_basis <= 16,
 * radial basis gaussian/bessel, MainNet with up to 4 hidden layers, no external
 * tensor, no physical heads, no long-range module.                           */
typedef struct {
  int32_t channels;          /* C (hidden_dim_conv): 32 or 64                    */
  int32_t lmax;              /* must be 2                                        */
  int32_t num_interaction;   /* 2..8                                             */
  int32_t number_of_basis;   /* radial basis size, <= 16                         */
  int32_t basis_kind;        /* 0 = gaussian, 1 = bessel                         */
  float max_radius;          /* cutoff of the radial basis                       */
  int32_t num_species;       /* max_atomvalue (rows of the per-species tables)  */
  int32_t output_size;       /* conv1 scalar width, must be 8                    */
  int32_t invariant_channels;/* readout scalar channels per extra interaction   */
  int32_t n_hidden;          /* MainNet hidden layers, 1..4                      */
  int32_t hidden[4];         /* MainNet hidden sizes (<= 1024)                   */
  int32_t n_out;             /* MainNet output width (17)                        */
  int32_t o3;                /* 0 = pure-cartesian-ictd; 1 = pure-cartesian-ictd-o3 with
                                active irreps 0e,1e,1o,2e (pure_cartesian_ictd_layers_o3.py):
                                the canonical-parity blocks 0e,1o,2e carry the 11 SO(3) paths
                                of its 17, 1e has no source without a 1e input and stays zero;
                                readout over 4 Gram blocks, MainNet input 4*nC + S          */
} fsc_ictd_config;

/* Packed fp32 device weights.  The host side derives them from the reference
 * state_dict (key names in comments); layouts are row-major.
 *   P = 11 paths, nint = num_interaction, nb = number_of_basis, C = channels,
 *   nC = C*nint, S = (nint-1)*invariant_channels, npairs = nC*(nC+1)/2.   */
typedef struct {
  const float* tables;   /* ictd tables, fsc_ictd_tables_floats() floats: Y polynomials,
                            conv2 CG (115x5), conv1 CG (9x5), product_5 factors (3)       */
  const float* ai;       /* [num_species][8]   atom_mlp(atom_embedding(Z))                 */
  const float* vsp;      /* [num_species][3][8][C]  V[s][l][i][o] = sum_j e3_conv_emb.tp2.weight[p(l,0,l),o,i,j]*ai[s,j] */
  const float* rad_w1;   /* [nint][64][nb]   fc.0 / fc2_layers.k.0 weight                  */
  const float* rad_b1;   /* [nint][64]                                                      */
  const float* rad_w2;   /* [nint][64][64]   fc.2 / fc2_layers.k.2                          */
  const float* rad_b2;   /* [nint][64]                                                      */
  const float* rad_w3;   /* [nint][11][64]   fc.4 / fc2_layers.k.4                          */
  const float* rad_b3;   /* [nint][11]                                                      */
  /* Channel mixes of conv2..N (tp2_layers.k.weight W[p][o][i]), 11*C*C floats per layer,
   * three blocks per layer for l3 (l1) = 0, 1, 2 holding the paths with that l3 (l1) in
   * path order (P3 = P1 = {3, 4, 4} paths):                                                 */
  const float* mix_fwd;  /* [nint-1] x blocks [(rank,i)][o] = W[p_rank][o][i]                */
  const float* mix_bwd;  /* [nint-1] x blocks [o][(rank,i)] = W[p_rank][o][i]                */
  const float* mix_dx;   /* [nint-1] x blocks (by l1) [(rank,o)][i] = W[p_rank][o][i]        */
  const float* wread_p;  /* [3][S][npairs]   W_read.l symmetrised, upper-triangle packed,
                                             off-diagonal doubled, scaled 1/sqrt(2l+1)    */
  const float* wread_s;  /* [3][S][nC][nC]   W_read.l symmetrised (W+W^T)/2, scaled 1/sqrt(2l+1) */
  const int32_t* pairs;  /* [npairs] packed (c | d<<16), c <= d, row-major upper triangle       */
  /* The Gram invariants read t_l[c][m] = F[off_l + c*(2l+1) + m] from the flat concatenation
   * F of all layers' features in the reference layout (pure_cartesian_ictd_layers_full.py:
   * 956-958 splits torch.cat(features) into l blocks of nC*(2l+1)); off_l = 0, nC, 4nC.
   * xmap[off_l + c*(2l+1) + m] = (layer << 16) | (k*C + channel) locates that element in
   * the [N][9][C] feature buffers.                                                          */
  const int32_t* xmap;   /* [9*nC]                                                          */
  const int32_t* xinv;   /* [nint][9*C] inverse of xmap: storage (layer, k*C+c) -> element   */
  /* Tensor-core readout: W_read in 8x8 (c, d) blocks as shared-memory images of K-major fp16
   * tcgen05 (kind::f16) operands.  Each image starts with a 64-byte header whose first float is
   * 1/s, s = the power of two bringing max |W| in the image to <= 2^14; then per block the fp16
   * hi plane and lo plane of s*W (hi = fp16(s w), lo = fp16(s w - hi)).  nb = nC/8,
   * pair = (c - 8cb, d - 8db), Ws = (W_read.l + W_read.l^T)/2/sqrt(2l+1):
   *   wimg_fwd: for l, cb <= db:  [k/8][o][k%8], K = 64 pairs ordered (d/4, c/4, c%4, d%4), Ws x2
   *             off the diagonal block
   *   wimg_bwd: for l, cb, db pairs (db even, db+1):  [o/8][n][o%8],
   *             n = 64 (db odd) + 32 (c/4) + 4d + c%4                                           */
  const float* wimg_fwd; /* header + [3*nb*(nb+1)/2][2][8][S][8] fp16                         */
  const float* wimg_bwd; /* header + [3*nb*nb/2][2][S/8][128][8] fp16                         */
  const float* mn_in_g;  /* [D0]  proj_total.input_norm.weight, D0 = 3*nC + S             */
  const float* mn_in_b;  /* [D0]  proj_total.input_norm.bias                              */
  const float* mn_w[4];  /* [hidden[k]][in_k]  proj_total.layers.k.weight (as stored)      */
  const float* mn_b[4];  /* [hidden[k]]        proj_total.layers.k.bias                    */
  const float* mn_g[4];  /* [hidden[k]]        proj_total.layer_norms.k.weight            */
  const float* mn_beta[4];/* [hidden[k]]       proj_total.layer_norms.k.bias              */
  /* proj_total.output followed by weighted_sum collapse to one dot product:
   *   e = x_last . out_v + out_c0,  out_v = output.weight^T weighted_sum.weights,
   *   out_c0 = output.bias . weighted_sum.weights                                        */
  const float* out_v;    /* [hidden[last]]                                                  */
  float out_c0;
} fsc_ictd_weights;

/* Number of floats in the `tables` block. */
int64_t fsc_ictd_tables_floats(void);

typedef struct {
  int64_t num_atoms;        /* N (owned + ghost)                                     */
  int64_t num_local;        /* energy = sum over atoms [0, num_local)                */
  int64_t num_edges;        /* E                                                     */
  int64_t num_graphs;       /* B                                                     */
  const float* pos;         /* [N][3]                                                */
  const int32_t* species;   /* [N] atomic numbers, < num_species                     */
  const int32_t* batch;     /* [N] graph of each atom                                */
  const float* cell;        /* [B][3][3] rows = lattice vectors                      */
  const int32_t* row_ptr;   /* [N+1] CSR by dst                                      */
  const int32_t* src;       /* [E] edge sources, sorted by dst                       */
  const float* shift;       /* [E][3] integer image shift S (as float), r = pos[dst]-pos[src]+S@cell[batch[src]] */
  const int32_t* tr_ptr;    /* [N+1] CSR by src                                      */
  const int32_t* tr_eid;    /* [E] edge ids grouped by src                           */
  const float* energy_weight;/* [N] or NULL: backward seed dL/de_n; NULL = 1 for atoms
                                [0, num_local), 0 for the rest (LAMMPS ghost convention,
                                mff_torch_engine.cpp:812-820)                           */
  const float* field;       /* [B][3] or NULL: per-graph vector added to the l = 1 direction
                                harmonic of conv1 (external 1o field of the o3 model: the
                                field's ICTD l = 1 components times external_tensor_scale,
                                pure_cartesian_ictd_layers_o3.py:466-502)               */
  const int64_t* layer_atoms;/* HOST [num_interaction] or NULL (= all atoms).  Receptive-field
                                restriction of a spatial-decomposition rank: interaction layer k
                                (conv1 = 0) is evaluated for receiving atoms [0, layer_atoms[k])
                                and the readout for atoms [0, layer_atoms[last]).  Non-increasing,
                                layer_atoms[last] >= num_local, and every edge whose dst is below
                                layer_atoms[k] (k >= 1) has src below layer_atoms[k-1] (atoms
                                ordered by distance shell from the owned region); a violated edge
                                sets status 70 and is skipped.  Atoms past layer_atoms[last] get
                                atom_energy 0 and no backward seed.  ictd engine only.       */
} fsc_graph;

typedef struct {
  float* energy;            /* [B] per-graph energy (sum of atom energies, local atoms) */
  float* atom_energy;       /* [N] or NULL                                            */
  float* forces;            /* [N][3] = -dE/dpos                                      */
  float* virial;            /* [B][9] or NULL: sum_e r_e (x) dE/dr_e (row-major a,b)  */
  float* edge_grad;         /* [E][3] or NULL: dE/dr_e per edge (LAMMPS atom virial)  */
  float* cell_grad;         /* [B][9] or NULL: dE/dcell = sum_e S_e (x) dE/dr_e        */
} fsc_ictd_outputs;

size_t fsc_ictd_workspace_bytes(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges);
int fsc_ictd_energy_forces(const fsc_ictd_config* cfg, const fsc_ictd_weights* w,
                           const fsc_graph* g, fsc_ictd_outputs* out, void* workspace,
                           size_t workspace_bytes, void* stream);
/* The same call split in two: forward leaves its intermediates in `workspace`;
 * backward (same cfg, weights, graph and workspace, no other call on that workspace
 * in between) produces the outputs' forces / virial / edge_grad / cell_grad with the
 * seed graph->energy_weight.  This pair is what an autograd wrapper binds. */
int fsc_ictd_forward(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g,
                     float* energy, float* atom_energy, void* workspace, size_t workspace_bytes,
                     void* stream);
int fsc_ictd_backward(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g,
                      fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream);
/* Stepwise evaluation, for callers that act on the node features between interaction layers:
 * the reference's sync_after_scatter hook (pure_cartesian_ictd_layers_full.py:923-924, 952-953;
 * pure_cartesian_ictd_layers_o3.py:947-948, 971-972) or a per-layer ghost-feature exchange of a
 * spatial decomposition (cli/inference_ddp.py:143-340).  Forward steps: 0 = edge geometry, radial
 * MLPs and conv1 (layer 0's features); k in [1, num_interaction) = conv2 layer k; num_interaction
 * = readout (energy, atom_energy; both may be NULL before it).  Steps 0..num_interaction in order
 * equal fsc_ictd_forward.  Backward steps, after a forward on the same workspace: num_interaction
 * = readout backward (every layer's feature gradient from the readout); k in [1, num_interaction)
 * = conv2 layer k backward (needs layer k's gradient complete, adds into layer k - 1's); 0 =
 * conv1 backward and the edge part (forces / virial / edge_grad / cell_grad into `out`).  Steps
 * num_interaction..0 in order equal fsc_ictd_backward.  Between steps the caller may rewrite the
 * buffers fsc_ictd_feature_buffer names, on the same stream. */
int fsc_ictd_forward_step(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int step,
                          float* energy, float* atom_energy, void* workspace, size_t workspace_bytes, void* stream);
int fsc_ictd_backward_step(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int step,
                           fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream);
/* Device address, inside a workspace laid out for (cfg, num_atoms, num_edges), of layer `layer`'s
 * node features (which = 0) or of their gradient (which = 1): float [num_atoms][9][C], row
 * l^2 + m (l = 0..2; with the o3 model the rows are 0e, 1o, 2e), channel innermost. */
int fsc_ictd_feature_buffer(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                            int which, int layer, float** out);
/* Device status word of the last call on `workspace` (0 = ok; else the id of a bounded
 * wait in a tensor-core kernel that timed out).  Synchronises `stream`.  */
int fsc_ictd_status(const fsc_ictd_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                    void* stream, int* status_host);
/* Readout path: 0 = tensor cores where supported (default), 1 = CUDA-core kernels. */
void fsc_ictd_set_readout_path(int path);
/* Radial MLP path (per-edge fc / fc2_layers and their backward): 0 = tensor cores where
 * supported (default; number_of_basis <= 16), 1 = CUDA-core kernels.  Process-wide. */
void fsc_ictd_set_radial_path(int path);
/* Channel-mixing and MainNet GEMMs, and the pure-cartesian-sparse per-node aggregation kernels
 * (forward Z and its two reverse contractions): 0 = tensor cores (tcgen05, 3xTF32) where the
 * shape qualifies (default), 1 = CUDA-core kernels, 2 = tensor-core aggregation with CUDA-core
 * GEMMs, 3 = CUDA-core aggregation with tensor-core GEMMs.  Process-wide. */
void fsc_ictd_set_gemm_path(int path);
/* conv2 gate / harmonic gradients (the reverse of the per-edge contraction with the sender
 * rows): 0 = CUDA-core kernel (default, the faster one), 1 = tensor cores (tcgen05, 3xTF32,
 * one 128 x 48 product per 14 edges of a receiver, warp-specialised pipeline).  Process-wide. */
void fsc_ictd_set_conv2_path(int path);
/* Plan of the tensor-core GEMM for a K x N product (host arithmetic, no device work): the output
 * tile width and the longest chain of tcgen05.mma instructions that accumulate into one TMEM
 * accumulator before the partial sum moves to fp32 registers (tensor-core accumulation rounds
 * toward zero, so the engines keep these chains at <= 24).  `precise` selects the variant used
 * for long K with heavy cancellation (the readout's Gram contraction).  No reference
 * counterpart: a diagnostic of this library's accumulation order. */
int fsc_gemm_tc_plan(int K, int N, int precise, int* tile_n, int* max_chain);
/* Physical-tensor heads of the o3 model (pure_cartesian_ictd_layers_o3.py:1010-1044), from the
 * features left in the workspace by the last fsc_ictd_forward on it: for head h,
 *   out[h][b][m] = sum_{n in graph b} sum_c weights[h][c] * t_{block[h]}[n][c][m],  m < 2l+1,
 * t_block = Gram operand block (0e, 1e, 1o, 2e for o3; l = 0, 1, 2 otherwise) of the readout's
 * flat split of the concatenated features, c < nC.  weights [nheads][nC], out [nheads][B][5]
 * (entries m >= 2l+1 are set to 0).  block_host: host array of nheads block indices. */
int fsc_ictd_heads(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g, int nheads,
                   const int32_t* block_host, const float* weights, float* out, void* workspace,
                   size_t workspace_bytes, void* stream);
/* Forward only (per-atom energy), same workspace. */
int fsc_ictd_energy(const fsc_ictd_config* cfg, const fsc_ictd_weights* w, const fsc_graph* g,
                    float* energy, float* atom_energy, void* workspace, size_t workspace_bytes,
                    void* stream);

/* ---- pure-cartesian-sparse model ------------------------------------------------
 * PureCartesianSparseTransformerLayer (models/pure_cartesian_sparse_layers.py:459-855) with
 * max_rank_other = 1, k_policy = "k0", no epsilon paths: node features are true Cartesian
 * tensors of rank L <= lmax (3^L components per channel; the pseudotensor half is identically
 * zero), every tensor-product path (L1, L2 -> L1 + L2, min(L1, L2) <= 1) is an outer product,
 * and the per-edge channel-mixing weights come from the radial MLP (fc.4 of each layer).
 * The engine never forms those per-edge weights: conv1 uses per-species-pair tables, conv2
 * aggregates h2 (x) message per receiving node and applies fc.4 as one GEMM.
 * Same graph (fsc_graph) and outputs (fsc_ictd_outputs) as the ictd engine; field unused. */
typedef struct {
  int32_t channels;          /* C: 32, 64 or 128                                  */
  int32_t lmax;              /* 2 or 3                                            */
  int32_t num_interaction;   /* 2..8                                              */
  int32_t number_of_basis;   /* <= 16                                             */
  int32_t basis_kind;        /* 0 = gaussian, 1 = bessel                          */
  float max_radius;
  int32_t num_species;       /* max_atomvalue                                     */
  int32_t invariant_channels;
  int32_t n_hidden;
  int32_t hidden[4];
  int32_t n_out;             /* 17                                                */
  float avg_num_neighbors;   /* conv2 normaliser: 0 = E / N of the call's graph, as the reference
                                (pure_cartesian_sparse_layers.py:418); > 0 = this value (the
                                whole system's E / N when a spatial-decomposition rank passes its
                                local graph of owned atoms and ghosts)                        */
} fsc_sparse_config;

/* Packed fp32 device weights (host derives them from the reference state_dict):
 *   R = sum_{L<=lmax} 3^L components, P paths in the reference order, J = 65 (64 hidden + 1). */
typedef struct {
  const float* rad_w1;   /* [nint][64][nb]  e3_conv_layers.k.fc.0.weight (k = 0 is e3_conv_emb.fc) */
  const float* rad_b1;   /* [nint][64]                                                         */
  const float* rad_w2;   /* [nint][64][64]  fc.2                                               */
  const float* rad_b2;   /* [nint][64]                                                         */
  /* conv1, paths (L, 0, L): K[ss][sd][L][j][c] = sum_{a,b} W_fc4[(p_L*C + c)*64 + a*8 + b][j] ai[ss][a] ai[sd][b]
   * (j = 64: the fc.4 bias), ai = atom_mlp(atom_embedding) per species                         */
  const float* pair_k;   /* [S][S][lmax+1][J][C]                                               */
  /* conv2 layer k (k = 1..nint-1), per output rank Lout, the paths with that Lout in order
   * (rank q): mix[k-1][Lout][(q, j, a)][c] = W_fc4[(p_q*C + c)*C + a][j] (j = 64: bias), and
   * mixT[k-1][Lout][c][(q, j, a)] its transpose.                                               */
  const float* mix;
  const float* mixT;
  const float* wread_p;  /* [lmax+1][S][npairs] product_3.W.L symmetrised, packed, / sqrt(3^L)  */
  const float* wread_s;  /* [lmax+1][S][nC][nC] product_3.W.L symmetrised / sqrt(3^L)           */
  const int32_t* pairs;  /* [npairs] (c | d << 16), c <= d                                        */
  const float* mn_in_g;
  const float* mn_in_b;
  const float* mn_w[4];
  const float* mn_b[4];
  const float* mn_g[4];
  const float* mn_beta[4];
  const float* out_v;
  float out_c0;
} fsc_sparse_weights;

size_t fsc_sparse_workspace_bytes(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges);
int fsc_sparse_forward(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g,
                       float* energy, float* atom_energy, void* workspace, size_t workspace_bytes, void* stream);
int fsc_sparse_backward(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g,
                        fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream);
int fsc_sparse_status(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                      void* stream, int* status_host);
/* Stepwise pure-cartesian-sparse evaluation, as fsc_ictd_forward_step / fsc_ictd_backward_step
 * (same step numbering; the reference sparse model has no sync_after_scatter hook, but a
 * per-layer ghost-feature exchange of a spatial decomposition uses the steps).  Feature buffers:
 * float [num_atoms][R][C], R = sum_{L <= lmax} 3^L rows (rank-L Cartesian components, row-major),
 * channel innermost. */
int fsc_sparse_forward_step(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g, int step,
                            float* energy, float* atom_energy, void* workspace, size_t workspace_bytes, void* stream);
int fsc_sparse_backward_step(const fsc_sparse_config* cfg, const fsc_sparse_weights* w, const fsc_graph* g, int step,
                             fsc_ictd_outputs* out, void* workspace, size_t workspace_bytes, void* stream);
int fsc_sparse_feature_buffer(const fsc_sparse_config* cfg, int64_t num_atoms, int64_t num_edges, void* workspace,
                              int which, int layer, float** out);

/* ---- stage timing ------------------------------------------------------
 * When enabled, the engine records a CUDA event after each stage on its stream;
 * fsc_profile_read waits for the last one and returns per-stage milliseconds (stage
 * i spans from mark i-1 to mark i; the same name may repeat, once per layer) and
 * clears the record.  Process-wide, not thread-safe; meant for benchmarks. */
void fsc_profile_enable(int enable);
int fsc_profile_read(const char** names, float* ms, int max_stages);

#ifdef __cplusplus
}
#endif
#endif /* FSCTEP_B200_H */
