// TorchScript custom ops for core.pt: per-atom energies of the pure-cartesian-ictd, -ictd-o3 and
// -sparse models from precomputed edge vectors, with the native reverse pass as their autograd
// backward (fsctep::ictd_atom_energy, fsctep::ictd_o3_atom_energy with the o3 model's external
// field, fsctep::sparse_atom_energy).
//
// The reference exports core.pt by tracing _TorchScriptEdgeVecCore (interfaces/lammps_mliap.py:
// 372-420, 615-684): forward(pos, A, batch, edge_src, edge_dst, edge_shifts, cell, edge_vec,
// external_tensor) -> atom_energy (N, 1).  The LAMMPS engine (mff_torch_engine.cpp:459-569)
// builds edge_vec = pos[dst] - pos[src] + shift with autograd, runs core.pt and calls
// torch::autograd::grad(sum(atom_energy[:nlocal]), {pos, shift}).  The model's dependence on
// positions is entirely through edge_vec, so one op
//
//   fsctep::ictd_atom_energy(edge_vec, species, edge_src, edge_dst, blob, icfg, fcfg) -> (N, 1)
//
// with backward  grad_edge_vec[e] = sum_i grad_atom[i] dE_i/dr_e  covers that contract.  The op
// feeds the engine with positions 0, one graph with an identity cell and shift = edge_vec, so
// the engine's r_e = pos[dst] - pos[src] + shift . cell is edge_vec itself, and passes the
// upstream gradient as the engine's per-atom energy weights.  Loaded into LAMMPS through
// MFF_CUSTOM_OPS_LIB (dlopen, no libpython).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/autograd.h>
#include <torch/library.h>

#include <vector>

#include "fsctep_b200.h"

namespace {

using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

// icfg: channels, lmax, num_interaction, number_of_basis, basis_kind, num_species, output_size,
//       invariant_channels, n_hidden, hidden[4], n_out, o3, then one element offset into the blob per
//       weight field in the order of kFields (-1 = absent).
// fcfg: max_radius, out_c0.
constexpr int kCfgInts = 15;
constexpr int kFields = 38;

struct Packed {
  fsc_ictd_config cfg;
  fsc_ictd_weights w;
};

Packed unpack(const at::Tensor& blob, c10::IntArrayRef ic, c10::ArrayRef<double> fc) {
  TORCH_CHECK(ic.size() == kCfgInts + kFields, "fsctep::ictd_atom_energy: icfg must have ", kCfgInts + kFields,
              " entries, got ", ic.size());
  TORCH_CHECK(fc.size() == 2, "fsctep::ictd_atom_energy: fcfg must be [max_radius, out_c0]");
  TORCH_CHECK(blob.is_cuda() && blob.scalar_type() == at::kFloat && blob.is_contiguous(),
              "fsctep::ictd_atom_energy: blob must be a contiguous float32 CUDA tensor");
  Packed p{};
  p.cfg.channels = (int32_t)ic[0];
  p.cfg.lmax = (int32_t)ic[1];
  p.cfg.num_interaction = (int32_t)ic[2];
  p.cfg.number_of_basis = (int32_t)ic[3];
  p.cfg.basis_kind = (int32_t)ic[4];
  p.cfg.num_species = (int32_t)ic[5];
  p.cfg.output_size = (int32_t)ic[6];
  p.cfg.invariant_channels = (int32_t)ic[7];
  p.cfg.n_hidden = (int32_t)ic[8];
  for (int k = 0; k < 4; ++k) p.cfg.hidden[k] = (int32_t)ic[9 + k];
  p.cfg.n_out = (int32_t)ic[13];
  p.cfg.o3 = (int32_t)ic[14];
  p.cfg.max_radius = (float)fc[0];
  const float* base = blob.data_ptr<float>();
  const int64_t n = blob.numel();
  auto at_ = [&](int k) -> const float* {
    const int64_t off = ic[kCfgInts + k];
    if (off < 0) return nullptr;
    TORCH_CHECK(off < n, "fsctep::ictd_atom_energy: weight offset out of range");
    return base + off;
  };
  int k = 0;
  fsc_ictd_weights& w = p.w;
  w.tables = at_(k++);
  w.ai = at_(k++);
  w.vsp = at_(k++);
  w.rad_w1 = at_(k++);
  w.rad_b1 = at_(k++);
  w.rad_w2 = at_(k++);
  w.rad_b2 = at_(k++);
  w.rad_w3 = at_(k++);
  w.rad_b3 = at_(k++);
  w.mix_fwd = at_(k++);
  w.mix_bwd = at_(k++);
  w.mix_dx = at_(k++);
  w.wread_p = at_(k++);
  w.wread_s = at_(k++);
  w.pairs = reinterpret_cast<const int32_t*>(at_(k++));
  w.xmap = reinterpret_cast<const int32_t*>(at_(k++));
  w.xinv = reinterpret_cast<const int32_t*>(at_(k++));
  w.wimg_fwd = at_(k++);
  w.wimg_bwd = at_(k++);
  w.mn_in_g = at_(k++);
  w.mn_in_b = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_w[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_b[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_g[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_beta[h] = at_(k++);
  w.out_v = at_(k++);
  TORCH_CHECK(k == kFields, "internal: field count");
  w.out_c0 = (float)fc[1];
  return p;
}

// Sparse icfg: channels, lmax, num_interaction, number_of_basis, basis_kind, num_species,
//   invariant_channels, n_hidden, hidden[4], n_out, then one blob offset per field of kSparseFields
//   (-1 = absent).  fcfg: max_radius, out_c0.
constexpr int kSparseCfgInts = 13;
constexpr int kSparseFields = 29;

struct SparsePacked {
  fsc_sparse_config cfg;
  fsc_sparse_weights w;
};

SparsePacked unpack_sparse(const at::Tensor& blob, c10::IntArrayRef ic, c10::ArrayRef<double> fc) {
  TORCH_CHECK(ic.size() == kSparseCfgInts + kSparseFields, "fsctep::sparse_atom_energy: icfg must have ",
              kSparseCfgInts + kSparseFields, " entries, got ", ic.size());
  TORCH_CHECK(fc.size() == 2, "fsctep::sparse_atom_energy: fcfg must be [max_radius, out_c0]");
  TORCH_CHECK(blob.is_cuda() && blob.scalar_type() == at::kFloat && blob.is_contiguous(),
              "fsctep::sparse_atom_energy: blob must be a contiguous float32 CUDA tensor");
  SparsePacked p{};
  fsc_sparse_config& c = p.cfg;
  c.channels = (int32_t)ic[0];
  c.lmax = (int32_t)ic[1];
  c.num_interaction = (int32_t)ic[2];
  c.number_of_basis = (int32_t)ic[3];
  c.basis_kind = (int32_t)ic[4];
  c.num_species = (int32_t)ic[5];
  c.invariant_channels = (int32_t)ic[6];
  c.n_hidden = (int32_t)ic[7];
  for (int k = 0; k < 4; ++k) c.hidden[k] = (int32_t)ic[8 + k];
  c.n_out = (int32_t)ic[12];
  c.max_radius = (float)fc[0];
  c.avg_num_neighbors = 0.f;  // E / N of the call's graph, as the reference
  const float* base = blob.data_ptr<float>();
  const int64_t n = blob.numel();
  auto at_ = [&](int k) -> const float* {
    const int64_t off = ic[kSparseCfgInts + k];
    if (off < 0) return nullptr;
    TORCH_CHECK(off < n, "fsctep::sparse_atom_energy: weight offset out of range");
    return base + off;
  };
  int k = 0;
  fsc_sparse_weights& w = p.w;
  w.rad_w1 = at_(k++);
  w.rad_b1 = at_(k++);
  w.rad_w2 = at_(k++);
  w.rad_b2 = at_(k++);
  w.pair_k = at_(k++);
  w.mix = at_(k++);
  w.mixT = at_(k++);
  w.wread_p = at_(k++);
  w.wread_s = at_(k++);
  w.pairs = reinterpret_cast<const int32_t*>(at_(k++));
  w.mn_in_g = at_(k++);
  w.mn_in_b = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_w[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_b[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_g[h] = at_(k++);
  for (int h = 0; h < 4; ++h) w.mn_beta[h] = at_(k++);
  w.out_v = at_(k++);
  TORCH_CHECK(k == kSparseFields, "internal: sparse field count");
  w.out_c0 = (float)fc[1];
  return p;
}

// The engine behind an op: pure-cartesian-ictd (-o3) or pure-cartesian-sparse.
enum Kind : int64_t { kIctd = 0, kSparse = 1 };

void check(int st, const char* what) {
  TORCH_CHECK(st == 0, "fsctep::ictd_atom_energy: ", what, " failed: ", fsc_last_error());
}

// dst-sorted CSR of the caller's edges, its transpose, and the engine inputs of the identity-cell
// formulation.  order[k] = caller's index of CSR slot k.
struct Graph {
  at::Tensor order, row_ptr, src, shift, tr_ptr, tr_eid, pos, species, batch, cell;
  int64_t N, E;
};

Graph make_graph(const at::Tensor& edge_vec, const at::Tensor& species, const at::Tensor& edge_src,
                 const at::Tensor& edge_dst, cudaStream_t st) {
  TORCH_CHECK(edge_vec.is_cuda() && edge_vec.dim() == 2 && edge_vec.size(1) == 3,
              "fsctep::ictd_atom_energy: edge_vec must be a CUDA (E, 3) tensor");
  TORCH_CHECK(edge_src.dim() == 1 && edge_dst.dim() == 1 && edge_src.size(0) == edge_vec.size(0) &&
                  edge_dst.size(0) == edge_vec.size(0),
              "fsctep::ictd_atom_energy: edge_src / edge_dst must be (E,)");
  Graph g;
  g.N = species.size(0);
  g.E = edge_vec.size(0);
  auto dev = edge_vec.device();
  auto i32 = at::TensorOptions().dtype(at::kInt).device(dev);
  auto dst = edge_dst.to(dev, at::kLong);
  g.order = std::get<1>(at::sort(dst, /*stable=*/true, /*dim=*/0, /*descending=*/false));
  auto counts = at::bincount(dst, {}, g.N);
  g.row_ptr = at::zeros({g.N + 1}, i32);
  if (g.N > 0) g.row_ptr.slice(0, 1).copy_(at::cumsum(counts, 0).to(at::kInt));
  g.src = edge_src.to(dev, at::kLong).index_select(0, g.order).to(at::kInt).contiguous();
  g.shift = edge_vec.detach().to(at::kFloat).index_select(0, g.order).contiguous();
  g.tr_ptr = at::empty({g.N + 1}, i32);
  g.tr_eid = at::empty({std::max<int64_t>(g.E, 1)}, i32);
  const size_t twb = fsc_csr_transpose_workspace_bytes(g.N, g.E);
  auto tws = at::empty({(int64_t)std::max<size_t>(twb, 1)}, at::TensorOptions().dtype(at::kByte).device(dev));
  check(fsc_csr_transpose(g.row_ptr.data_ptr<int32_t>(), g.src.data_ptr<int32_t>(), g.N, g.E,
                          g.tr_ptr.data_ptr<int32_t>(), g.tr_eid.data_ptr<int32_t>(), tws.data_ptr(), twb, st),
        "fsc_csr_transpose");
  auto f32 = at::TensorOptions().dtype(at::kFloat).device(dev);
  g.pos = at::zeros({std::max<int64_t>(g.N, 1), 3}, f32);
  g.species = species.to(dev, at::kInt).contiguous();
  g.batch = at::zeros({std::max<int64_t>(g.N, 1)}, i32);
  g.cell = at::eye(3, f32).reshape({1, 3, 3}).contiguous();
  return g;
}

fsc_graph engine_graph(const Graph& g, const float* energy_weight, const at::Tensor& field) {
  fsc_graph s{};
  s.num_atoms = g.N;
  s.num_local = g.N;
  s.num_edges = g.E;
  s.num_graphs = 1;
  s.pos = g.pos.data_ptr<float>();
  s.species = g.species.data_ptr<int32_t>();
  s.batch = g.batch.data_ptr<int32_t>();
  s.cell = g.cell.data_ptr<float>();
  s.row_ptr = g.row_ptr.data_ptr<int32_t>();
  s.src = g.src.data_ptr<int32_t>();
  s.shift = g.shift.data_ptr<float>();
  s.tr_ptr = g.tr_ptr.data_ptr<int32_t>();
  s.tr_eid = g.tr_eid.data_ptr<int32_t>();
  s.energy_weight = energy_weight;
  s.field = (field.defined() && field.numel() > 0) ? field.data_ptr<float>() : nullptr;
  return s;
}

at::Tensor no_field(const at::Tensor& edge_vec) {
  return at::empty({0}, edge_vec.options().dtype(at::kFloat));
}

// (1, 3) float32 field of the o3 op on the edge vectors' device (the engine's l = 1 conv1 term)
at::Tensor field_arg(const at::Tensor& field, const at::Tensor& edge_vec) {
  TORCH_CHECK(field.numel() == 3, "fsctep::ictd_o3_atom_energy: field must hold 3 values (one graph)");
  return field.detach().to(edge_vec.device(), at::kFloat).reshape({1, 3}).contiguous();
}

// Forward; returns (atom_energy (N, 1), workspace holding the intermediates).
std::pair<at::Tensor, at::Tensor> forward_impl(int64_t kind, const at::Tensor& blob, c10::IntArrayRef icfg,
                                               c10::ArrayRef<double> fcfg, const Graph& g, const at::Tensor& field,
                                               cudaStream_t st) {
  auto dev = g.shift.device();
  auto energy = at::empty({1}, at::TensorOptions().dtype(at::kFloat).device(dev));
  auto atom_e = at::empty({g.N}, at::TensorOptions().dtype(at::kFloat).device(dev));
  fsc_graph s = engine_graph(g, nullptr, field);
  at::Tensor ws;
  if (kind == kSparse) {
    const SparsePacked p = unpack_sparse(blob, icfg, fcfg);
    const size_t wb = fsc_sparse_workspace_bytes(&p.cfg, g.N, g.E);
    TORCH_CHECK(wb > 0, "fsctep::sparse_atom_energy: unsupported configuration: ", fsc_last_error());
    ws = at::empty({(int64_t)wb}, at::TensorOptions().dtype(at::kByte).device(dev));
    check(fsc_sparse_forward(&p.cfg, &p.w, &s, energy.data_ptr<float>(), atom_e.data_ptr<float>(), ws.data_ptr(),
                             wb, st),
          "fsc_sparse_forward");
  } else {
    const Packed p = unpack(blob, icfg, fcfg);
    const size_t wb = fsc_ictd_workspace_bytes(&p.cfg, g.N, g.E);
    TORCH_CHECK(wb > 0, "fsctep::ictd_atom_energy: unsupported configuration: ", fsc_last_error());
    ws = at::empty({(int64_t)wb}, at::TensorOptions().dtype(at::kByte).device(dev));
    check(fsc_ictd_forward(&p.cfg, &p.w, &s, energy.data_ptr<float>(), atom_e.data_ptr<float>(), ws.data_ptr(), wb,
                           st),
          "fsc_ictd_forward");
  }
  return {atom_e.reshape({g.N, 1}), ws};
}

cudaStream_t current_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// No-grad kernels (inference mode, or no input requires grad).
at::Tensor atom_energy_nograd(int64_t kind, const at::Tensor& edge_vec, const at::Tensor& species,
                              const at::Tensor& edge_src, const at::Tensor& edge_dst, const at::Tensor& field,
                              const at::Tensor& blob, c10::IntArrayRef icfg, c10::ArrayRef<double> fcfg) {
  cudaStream_t st = current_stream(edge_vec);
  Graph g = make_graph(edge_vec, species, edge_src, edge_dst, st);
  return forward_impl(kind, blob, icfg, fcfg, g, field, st).first.to(edge_vec.scalar_type());
}

at::Tensor ictd_atom_energy_cuda(const at::Tensor& edge_vec, const at::Tensor& species, const at::Tensor& edge_src,
                                 const at::Tensor& edge_dst, const at::Tensor& blob, c10::IntArrayRef icfg,
                                 c10::ArrayRef<double> fcfg) {
  return atom_energy_nograd(kIctd, edge_vec, species, edge_src, edge_dst, at::Tensor(), blob, icfg, fcfg);
}

at::Tensor ictd_o3_atom_energy_cuda(const at::Tensor& edge_vec, const at::Tensor& species, const at::Tensor& edge_src,
                                    const at::Tensor& edge_dst, const at::Tensor& field, const at::Tensor& blob,
                                    c10::IntArrayRef icfg, c10::ArrayRef<double> fcfg) {
  return atom_energy_nograd(kIctd, edge_vec, species, edge_src, edge_dst, field_arg(field, edge_vec), blob, icfg,
                            fcfg);
}

at::Tensor sparse_atom_energy_cuda(const at::Tensor& edge_vec, const at::Tensor& species, const at::Tensor& edge_src,
                                   const at::Tensor& edge_dst, const at::Tensor& blob, c10::IntArrayRef icfg,
                                   c10::ArrayRef<double> fcfg) {
  return atom_energy_nograd(kSparse, edge_vec, species, edge_src, edge_dst, at::Tensor(), blob, icfg, fcfg);
}

// Autograd: the backward is the engine's reverse pass with the upstream gradient as per-atom
// energy weights; dE/d(edge_vec) is its per-edge dE/dr.  The field (o3) is not differentiated;
// ops without one pass an empty tensor (custom autograd functions take defined tensors only).
class AtomEnergy : public torch::autograd::Function<AtomEnergy> {
 public:
  static at::Tensor forward(AutogradContext* ctx, const at::Tensor& edge_vec, const at::Tensor& species,
                            const at::Tensor& edge_src, const at::Tensor& edge_dst, const at::Tensor& field,
                            const at::Tensor& blob, c10::IntArrayRef icfg, c10::ArrayRef<double> fcfg, int64_t kind) {
    at::AutoDispatchBelowADInplaceOrView guard;
    cudaStream_t st = current_stream(edge_vec);
    Graph g = make_graph(edge_vec, species, edge_src, edge_dst, st);
    auto out = forward_impl(kind, blob, icfg, fcfg, g, field, st);
    ctx->saved_data["kind"] = kind;
    ctx->saved_data["field"] = field;
    ctx->saved_data["ws"] = out.second;
    ctx->saved_data["order"] = g.order;
    ctx->saved_data["row_ptr"] = g.row_ptr;
    ctx->saved_data["src"] = g.src;
    ctx->saved_data["shift"] = g.shift;
    ctx->saved_data["tr_ptr"] = g.tr_ptr;
    ctx->saved_data["tr_eid"] = g.tr_eid;
    ctx->saved_data["pos"] = g.pos;
    ctx->saved_data["species"] = g.species;
    ctx->saved_data["batch"] = g.batch;
    ctx->saved_data["cell"] = g.cell;
    ctx->saved_data["blob"] = blob;
    ctx->saved_data["icfg"] = std::vector<int64_t>(icfg.begin(), icfg.end());
    ctx->saved_data["fcfg"] = std::vector<double>(fcfg.begin(), fcfg.end());
    ctx->saved_data["dtype"] = (int64_t)edge_vec.scalar_type();
    return out.first.to(edge_vec.scalar_type());
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    at::Tensor go = grads[0];
    TORCH_CHECK(!at::GradMode::is_enabled() && !(go.defined() && go.requires_grad()),
                "fsctep atom energy ops: double backward (create_graph=True) is not implemented");
    auto& sd = ctx->saved_data;
    Graph g;
    g.order = sd["order"].toTensor();
    g.row_ptr = sd["row_ptr"].toTensor();
    g.src = sd["src"].toTensor();
    g.shift = sd["shift"].toTensor();
    g.tr_ptr = sd["tr_ptr"].toTensor();
    g.tr_eid = sd["tr_eid"].toTensor();
    g.pos = sd["pos"].toTensor();
    g.species = sd["species"].toTensor();
    g.batch = sd["batch"].toTensor();
    g.cell = sd["cell"].toTensor();
    g.N = g.species.size(0);
    g.E = g.shift.size(0);
    const auto icfg = sd["icfg"].toIntVector();
    const auto fcfg = sd["fcfg"].toDoubleVector();
    at::Tensor blob = sd["blob"].toTensor();
    const int64_t kind = sd["kind"].toInt();
    at::Tensor field = sd["field"].toTensor();
    at::Tensor ws = sd["ws"].toTensor();
    cudaStream_t st = current_stream(g.shift);
    auto dev = g.shift.device();
    if (!go.defined()) go = at::zeros({g.N, 1}, at::TensorOptions().dtype(at::kFloat).device(dev));
    auto w = go.reshape({g.N}).to(dev, at::kFloat).contiguous();
    auto edge_grad = at::empty({std::max<int64_t>(g.E, 1), 3}, at::TensorOptions().dtype(at::kFloat).device(dev));
    fsc_graph s = engine_graph(g, w.data_ptr<float>(), field);
    fsc_ictd_outputs o{};
    o.edge_grad = edge_grad.data_ptr<float>();
    if (kind == kSparse) {
      const SparsePacked p = unpack_sparse(blob, icfg, fcfg);
      check(fsc_sparse_backward(&p.cfg, &p.w, &s, &o, ws.data_ptr(), (size_t)ws.numel(), st), "fsc_sparse_backward");
    } else {
      const Packed p = unpack(blob, icfg, fcfg);
      check(fsc_ictd_backward(&p.cfg, &p.w, &s, &o, ws.data_ptr(), (size_t)ws.numel(), st), "fsc_ictd_backward");
    }
    auto out = at::zeros({g.E, 3}, edge_grad.options());
    if (g.E > 0) out.index_copy_(0, g.order, edge_grad.slice(0, 0, g.E));
    const auto dt = (at::ScalarType)sd["dtype"].toInt();
    return {out.to(dt), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(),
            at::Tensor(), at::Tensor()};
  }
};

at::Tensor ictd_atom_energy_autograd(const at::Tensor& edge_vec, const at::Tensor& species, const at::Tensor& edge_src,
                                     const at::Tensor& edge_dst, const at::Tensor& blob, c10::IntArrayRef icfg,
                                     c10::ArrayRef<double> fcfg) {
  return AtomEnergy::apply(edge_vec, species, edge_src, edge_dst, no_field(edge_vec), blob, icfg, fcfg,
                           (int64_t)kIctd);
}

at::Tensor ictd_o3_atom_energy_autograd(const at::Tensor& edge_vec, const at::Tensor& species,
                                        const at::Tensor& edge_src, const at::Tensor& edge_dst,
                                        const at::Tensor& field, const at::Tensor& blob, c10::IntArrayRef icfg,
                                        c10::ArrayRef<double> fcfg) {
  return AtomEnergy::apply(edge_vec, species, edge_src, edge_dst, field_arg(field, edge_vec), blob, icfg, fcfg,
                           (int64_t)kIctd);
}

at::Tensor sparse_atom_energy_autograd(const at::Tensor& edge_vec, const at::Tensor& species,
                                       const at::Tensor& edge_src, const at::Tensor& edge_dst, const at::Tensor& blob,
                                       c10::IntArrayRef icfg, c10::ArrayRef<double> fcfg) {
  return AtomEnergy::apply(edge_vec, species, edge_src, edge_dst, no_field(edge_vec), blob, icfg, fcfg,
                           (int64_t)kSparse);
}

}  // namespace

TORCH_LIBRARY(fsctep, m) {
  m.def("ictd_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, Tensor edge_dst, Tensor blob, "
        "int[] icfg, float[] fcfg) -> Tensor");
  m.def("ictd_o3_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, Tensor edge_dst, Tensor field, "
        "Tensor blob, int[] icfg, float[] fcfg) -> Tensor");
  m.def("sparse_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, Tensor edge_dst, Tensor blob, "
        "int[] icfg, float[] fcfg) -> Tensor");
}

TORCH_LIBRARY_IMPL(fsctep, CUDA, m) {
  m.impl("ictd_atom_energy", &ictd_atom_energy_cuda);
  m.impl("ictd_o3_atom_energy", &ictd_o3_atom_energy_cuda);
  m.impl("sparse_atom_energy", &sparse_atom_energy_cuda);
}

TORCH_LIBRARY_IMPL(fsctep, Autograd, m) {
  m.impl("ictd_atom_energy", &ictd_atom_energy_autograd);
  m.impl("ictd_o3_atom_energy", &ictd_o3_atom_energy_autograd);
  m.impl("sparse_atom_energy", &sparse_atom_energy_autograd);
}
