// The `_C_ictd_tp` operator family (csrc/ictd_tp.cpp:137-523 of the reference) for fp32/fp64.
//
// Notation: a (B,I,m1), b (B,J,m2), u (m1*m2, P*K) viewed as u[m1][m2][p*K+k],
// y / h (B,P,K,I*J) with ij = i*J + j, w (P,O,IJ), gates (B,P), out (B,O,K).
//   PF  y[b,p,k,ij]  = sum_{m1,m2} a[b,i,m1] b[b,j,m2] u[m1,m2,pk]            (project forward)
//   PAT ga[b,i,m1]   = sum_{j,p,k} h[b,p,k,ij] sum_{m2} b[b,j,m2] u[m1,m2,pk]
//   PBT gb[b,j,m2]   = sum_{i,p,k} h[b,p,k,ij] sum_{m1} a[b,i,m1] u[m1,m2,pk]
//   PUT gu[m1,m2,pk] = sum_{b,i,j} h[b,p,k,ij] a[b,i,m1] b[b,j,m2]
//   MF  out[b,o,k]   = sum_p g[b,p] sum_q y[b,p,k,q] w[p,o,q]                  (mix forward)
//   MYT gy[b,p,k,q]  = g[b,p] sum_o go[b,o,k] w[p,o,q]
//   MWT gw[p,o,q]    = sum_{b,k} g[b,p] go[b,o,k] y[b,p,k,q]
//   MGT gg[b,p]      = sum_{o,k} go[b,o,k] sum_q y[b,p,k,q] w[p,o,q]
// Double-backward ops are sums of two or three of these with the operand triples of
// ictd_tp_cuda.cu:528-534 and :780-786.  One thread per output element; the two ops that reduce
// over the batch (PUT, MWT) use one block per output element and a deterministic block reduction.
#include "common.cuh"

namespace fsc {
namespace {

struct Dims {
  int64_t B, I, J, m1, m2, P, K, O, IJ;
};

template <typename T>
struct Trip {
  const T* x0;
  const T* x1;
  const T* x2;
};

template <typename T>
__device__ T pf(const Dims& d, const T* a, const T* b, const T* u, int64_t bb, int64_t p, int64_t k, int64_t i,
                int64_t j) {
  const int64_t PK = d.P * d.K, pk = p * d.K + k;
  T acc = 0;
  for (int64_t x = 0; x < d.m1; ++x) {
    const T av = a[(bb * d.I + i) * d.m1 + x];
    T t = 0;
    for (int64_t z = 0; z < d.m2; ++z) t += b[(bb * d.J + j) * d.m2 + z] * u[(x * d.m2 + z) * PK + pk];
    acc += av * t;
  }
  return acc;
}

template <typename T>
__device__ T pat(const Dims& d, const T* h, const T* b, const T* u, int64_t bb, int64_t i, int64_t x) {
  const int64_t PK = d.P * d.K;
  T acc = 0;
  for (int64_t pk = 0; pk < PK; ++pk)
    for (int64_t j = 0; j < d.J; ++j) {
      T t = 0;
      for (int64_t z = 0; z < d.m2; ++z) t += b[(bb * d.J + j) * d.m2 + z] * u[(x * d.m2 + z) * PK + pk];
      acc += h[(bb * PK + pk) * d.IJ + i * d.J + j] * t;
    }
  return acc;
}

template <typename T>
__device__ T pbt(const Dims& d, const T* h, const T* a, const T* u, int64_t bb, int64_t j, int64_t z) {
  const int64_t PK = d.P * d.K;
  T acc = 0;
  for (int64_t pk = 0; pk < PK; ++pk)
    for (int64_t i = 0; i < d.I; ++i) {
      T t = 0;
      for (int64_t x = 0; x < d.m1; ++x) t += a[(bb * d.I + i) * d.m1 + x] * u[(x * d.m2 + z) * PK + pk];
      acc += h[(bb * PK + pk) * d.IJ + i * d.J + j] * t;
    }
  return acc;
}

template <typename T>
__device__ T mf(const Dims& d, const T* y, const T* w, const T* g, int64_t bb, int64_t o, int64_t k) {
  T acc = 0;
  for (int64_t p = 0; p < d.P; ++p) {
    T t = 0;
    for (int64_t q = 0; q < d.IJ; ++q) t += y[((bb * d.P + p) * d.K + k) * d.IJ + q] * w[(p * d.O + o) * d.IJ + q];
    acc += g[bb * d.P + p] * t;
  }
  return acc;
}

template <typename T>
__device__ T myt(const Dims& d, const T* go, const T* w, const T* g, int64_t bb, int64_t p, int64_t k, int64_t q) {
  T t = 0;
  for (int64_t o = 0; o < d.O; ++o) t += go[(bb * d.O + o) * d.K + k] * w[(p * d.O + o) * d.IJ + q];
  return g[bb * d.P + p] * t;
}

template <typename T>
__device__ T mgt(const Dims& d, const T* go, const T* y, const T* w, int64_t bb, int64_t p) {
  T acc = 0;
  for (int64_t o = 0; o < d.O; ++o)
    for (int64_t k = 0; k < d.K; ++k) {
      T t = 0;
      for (int64_t q = 0; q < d.IJ; ++q) t += y[((bb * d.P + p) * d.K + k) * d.IJ + q] * w[(p * d.O + o) * d.IJ + q];
      acc += go[(bb * d.O + o) * d.K + k] * t;
    }
  return acc;
}

enum Kind { K_PF, K_PAT, K_PBT, K_MF, K_MYT, K_MGT };

template <typename T, int KIND>
__global__ void elem_kernel(Dims d, Trip<T> t0, Trip<T> t1, Trip<T> t2, int nterms, T* out, int64_t total) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const Trip<T> ts[3] = {t0, t1, t2};
  T acc = 0;
  for (int s = 0; s < nterms; ++s) {
    const Trip<T>& t = ts[s];
    if (KIND == K_PF) {  // out (B,P,K,I,J)
      int64_t r = idx;
      const int64_t j = r % d.J; r /= d.J;
      const int64_t i = r % d.I; r /= d.I;
      const int64_t k = r % d.K; r /= d.K;
      const int64_t p = r % d.P; r /= d.P;
      acc += pf(d, t.x0, t.x1, t.x2, r, p, k, i, j);
    } else if (KIND == K_PAT) {  // out (B,I,m1)
      const int64_t x = idx % d.m1, i = (idx / d.m1) % d.I, bb = idx / (d.m1 * d.I);
      acc += pat(d, t.x0, t.x1, t.x2, bb, i, x);
    } else if (KIND == K_PBT) {  // out (B,J,m2)
      const int64_t z = idx % d.m2, j = (idx / d.m2) % d.J, bb = idx / (d.m2 * d.J);
      acc += pbt(d, t.x0, t.x1, t.x2, bb, j, z);
    } else if (KIND == K_MF) {  // out (B,O,K)
      const int64_t k = idx % d.K, o = (idx / d.K) % d.O, bb = idx / (d.K * d.O);
      acc += mf(d, t.x0, t.x1, t.x2, bb, o, k);
    } else if (KIND == K_MYT) {  // out (B,P,K,IJ)
      int64_t r = idx;
      const int64_t q = r % d.IJ; r /= d.IJ;
      const int64_t k = r % d.K; r /= d.K;
      const int64_t p = r % d.P; r /= d.P;
      acc += myt(d, t.x0, t.x1, t.x2, r, p, k, q);
    } else {  // K_MGT out (B,P)
      const int64_t p = idx % d.P, bb = idx / d.P;
      acc += mgt(d, t.x0, t.x1, t.x2, bb, p);
    }
  }
  out[idx] = acc;
}

// PUT: out[(m1,m2), pk] = sum_{b,i,j} h[b,pk,ij] a[b,i,m1] b[b,j,m2]  (one block per output)
// MWT: out[p,o,q]       = sum_{b,k} g[b,p] go[b,o,k] y[b,p,k,q]
template <typename T, int PUT>
__global__ void reduce_kernel(Dims d, Trip<T> t0, Trip<T> t1, int nterms, T* out) {
  __shared__ T red[256];
  const int64_t idx = blockIdx.x;
  const Trip<T> ts[2] = {t0, t1};
  T acc = 0;
  for (int s = 0; s < nterms; ++s) {
    const Trip<T>& t = ts[s];
    if (PUT) {
      const int64_t PK = d.P * d.K;
      const int64_t pk = idx % PK, mm = idx / PK, x = mm / d.m2, z = mm % d.m2;
      const int64_t n = d.B * d.I * d.J;
      for (int64_t r = threadIdx.x; r < n; r += blockDim.x) {
        const int64_t j = r % d.J, i = (r / d.J) % d.I, bb = r / (d.J * d.I);
        acc += t.x0[(bb * PK + pk) * d.IJ + i * d.J + j] * t.x1[(bb * d.I + i) * d.m1 + x] *
               t.x2[(bb * d.J + j) * d.m2 + z];
      }
    } else {
      const int64_t q = idx % d.IJ, o = (idx / d.IJ) % d.O, p = idx / (d.IJ * d.O);
      const int64_t n = d.B * d.K;
      // t.x0 = go, t.x1 = y, t.x2 = g
      for (int64_t r = threadIdx.x; r < n; r += blockDim.x) {
        const int64_t k = r % d.K, bb = r / d.K;
        acc += t.x2[bb * d.P + p] * t.x0[(bb * d.O + o) * d.K + k] * t.x1[((bb * d.P + p) * d.K + k) * d.IJ + q];
      }
    }
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[idx] = red[0];
}

template <typename T, int KIND>
int run_elem(const Dims& d, std::initializer_list<Trip<T>> terms, void* out, int64_t total, void* stream) {
  if (total <= 0) return FSC_OK;
  Trip<T> t[3] = {};
  int n = 0;
  for (const auto& x : terms) t[n++] = x;
  elem_kernel<T, KIND><<<(unsigned)ceil_div(total, 128), 128, 0, as_stream(stream)>>>(d, t[0], t[1], t[2], n,
                                                                                    static_cast<T*>(out), total);
  return check_launch("tp_ops elem_kernel");
}

template <typename T, int PUT>
int run_reduce(const Dims& d, std::initializer_list<Trip<T>> terms, void* out, int64_t total, void* stream) {
  if (total <= 0) return FSC_OK;
  if (total > 2147483647LL) return fail(FSC_ERR_ARGUMENT, "tp_ops: output too large");
  Trip<T> t[2] = {};
  int n = 0;
  for (const auto& x : terms) t[n++] = x;
  reduce_kernel<T, PUT><<<(unsigned)total, 256, 0, as_stream(stream)>>>(d, t[0], t[1], n, static_cast<T*>(out));
  return check_launch("tp_ops reduce_kernel");
}

int check_dims(int dtype, int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K) {
  FSC_REQUIRE(dtype == FSC_F32 || dtype == FSC_F64, "dtype must be FSC_F32 or FSC_F64");
  FSC_REQUIRE(B >= 0 && I >= 1 && J >= 1 && m1 >= 1 && m2 >= 1 && P >= 1 && K >= 1, "bad projection dims");
  return FSC_OK;
}
int check_mix(int dtype, int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O) {
  FSC_REQUIRE(dtype == FSC_F32 || dtype == FSC_F64, "dtype must be FSC_F32 or FSC_F64");
  FSC_REQUIRE(B >= 0 && P >= 1 && K >= 1 && IJ >= 1 && O >= 1, "bad mix dims");
  return FSC_OK;
}

Dims pdims(int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K) {
  return Dims{B, I, J, m1, m2, P, K, 0, I * J};
}
Dims mdims(int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O) { return Dims{B, 0, 0, 0, 0, P, K, O, IJ}; }

template <typename T>
Trip<T> tr(const void* a, const void* b, const void* c) {
  return Trip<T>{static_cast<const T*>(a), static_cast<const T*>(b), static_cast<const T*>(c)};
}

#define FSC_DISPATCH(dtype, ...)          \
  if ((dtype) == FSC_F32) {               \
    using T = float;                      \
    __VA_ARGS__;                          \
  } else {                                \
    using T = double;                     \
    __VA_ARGS__;                          \
  }

}  // namespace
}  // namespace fsc

namespace fsc {
namespace {
template <typename T>
__global__ void bucketed_kernel(Dims d, const T* a, const T* b, const T* u, const T* w, const T* g, T* out,
                                int64_t total) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int64_t k = idx % d.K, o = (idx / d.K) % d.O, bb = idx / (d.K * d.O);
  T acc = 0;
  for (int64_t p = 0; p < d.P; ++p) {
    T t = 0;
    for (int64_t i = 0; i < d.I; ++i)
      for (int64_t j = 0; j < d.J; ++j) t += w[(p * d.O + o) * d.IJ + i * d.J + j] * pf(d, a, b, u, bb, p, k, i, j);
    acc += g[bb * d.P + p] * t;
  }
  out[idx] = acc;
}
}  // namespace
}  // namespace fsc

using namespace fsc;

extern "C" {

int fsc_project_bucket_forward(int dtype, const void* a, const void* b, const void* u, void* y, int64_t B, int64_t I,
                               int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PF>(d, {tr<T>(a, b, u)}, y, B * P * K * I * J, stream)));
}

int fsc_project_bucket_transpose_a(int dtype, const void* grad_y, const void* b, const void* u, void* grad_a,
                                   int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                                   void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PAT>(d, {tr<T>(grad_y, b, u)}, grad_a, B * I * m1, stream)));
}

int fsc_project_bucket_transpose_b(int dtype, const void* grad_y, const void* a, const void* u, void* grad_b,
                                   int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                                   void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PBT>(d, {tr<T>(grad_y, a, u)}, grad_b, B * J * m2, stream)));
}

int fsc_project_bucket_transpose_u(int dtype, const void* grad_y, const void* a, const void* b, void* grad_u,
                                   int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                                   void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_reduce<T, 1>(d, {tr<T>(grad_y, a, b)}, grad_u, m1 * m2 * P * K, stream)));
}

int fsc_mix_bucket_forward(int dtype, const void* y, const void* w, const void* gates, void* out, int64_t B, int64_t P,
                           int64_t K, int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MF>(d, {tr<T>(y, w, gates)}, out, B * O * K, stream)));
}

int fsc_mix_bucket_transpose_y(int dtype, const void* grad_out, const void* w, const void* gates, void* grad_y,
                               int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MYT>(d, {tr<T>(grad_out, w, gates)}, grad_y, B * P * K * IJ, stream)));
}

int fsc_mix_bucket_transpose_w(int dtype, const void* grad_out, const void* y, const void* gates, void* grad_w,
                               int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_reduce<T, 0>(d, {tr<T>(grad_out, y, gates)}, grad_w, P * O * IJ, stream)));
}

int fsc_mix_bucket_transpose_g(int dtype, const void* grad_out, const void* y, const void* w, void* grad_g, int64_t B,
                               int64_t P, int64_t K, int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MGT>(d, {tr<T>(grad_out, y, w)}, grad_g, B * P, stream)));
}


int fsc_bucketed_tp_forward(int dtype, const void* a, const void* b, const void* u, const void* w, const void* gates,
                            void* out, int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P, int64_t K,
                            int64_t O, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  FSC_REQUIRE(O >= 1, "bad mul_out");
  Dims d = pdims(B, I, J, m1, m2, P, K);
  d.O = O;
  const int64_t total = B * O * K;
  if (total == 0) return FSC_OK;
  FSC_DISPATCH(dtype, {
    bucketed_kernel<T><<<(unsigned)ceil_div(total, 128), 128, 0, as_stream(stream)>>>(
        d, static_cast<const T*>(a), static_cast<const T*>(b), static_cast<const T*>(u), static_cast<const T*>(w),
        static_cast<const T*>(gates), static_cast<T*>(out), total);
    return check_launch("bucketed_kernel");
  });
}

int fsc_project_dbl_bwd_grad_h(int dtype, const void* a, const void* gga, const void* b, const void* ggb,
                               const void* u, const void* ggu, void* out, int64_t B, int64_t I, int64_t J, int64_t m1,
                               int64_t m2, int64_t P, int64_t K, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PF>(d, {tr<T>(gga, b, u), tr<T>(a, ggb, u), tr<T>(a, b, ggu)}, out,
                                                  B * P * K * I * J, stream)));
}

int fsc_project_dbl_bwd_grad_a(int dtype, const void* h, const void* b, const void* ggb, const void* u, const void* ggu,
                               void* out, int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P,
                               int64_t K, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PAT>(d, {tr<T>(h, ggb, u), tr<T>(h, b, ggu)}, out, B * I * m1, stream)));
}

int fsc_project_dbl_bwd_grad_b(int dtype, const void* h, const void* a, const void* gga, const void* u, const void* ggu,
                               void* out, int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P,
                               int64_t K, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype, return (run_elem<T, K_PBT>(d, {tr<T>(h, gga, u), tr<T>(h, a, ggu)}, out, B * J * m2, stream)));
}

int fsc_project_dbl_bwd_grad_u(int dtype, const void* h, const void* a, const void* gga, const void* b, const void* ggb,
                               void* out, int64_t B, int64_t I, int64_t J, int64_t m1, int64_t m2, int64_t P,
                               int64_t K, void* stream) {
  FSC_TRY(check_dims(dtype, B, I, J, m1, m2, P, K));
  const Dims d = pdims(B, I, J, m1, m2, P, K);
  FSC_DISPATCH(dtype,
               return (run_reduce<T, 1>(d, {tr<T>(h, gga, b), tr<T>(h, a, ggb)}, out, m1 * m2 * P * K, stream)));
}

int fsc_mix_dbl_bwd_grad_g_out(int dtype, const void* y, const void* ggy, const void* w, const void* ggw,
                               const void* gates, const void* ggg, void* out, int64_t B, int64_t P, int64_t K,
                               int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MF>(d, {tr<T>(ggy, w, gates), tr<T>(y, ggw, gates), tr<T>(y, w, ggg)},
                                                  out, B * O * K, stream)));
}

int fsc_mix_dbl_bwd_grad_y(int dtype, const void* g_out, const void* w, const void* ggw, const void* gates,
                           const void* ggg, void* out, int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O,
                           void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MYT>(d, {tr<T>(g_out, ggw, gates), tr<T>(g_out, w, ggg)}, out,
                                                   B * P * K * IJ, stream)));
}

int fsc_mix_dbl_bwd_grad_w(int dtype, const void* g_out, const void* y, const void* ggy, const void* gates,
                           const void* ggg, void* out, int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O,
                           void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_reduce<T, 0>(d, {tr<T>(g_out, ggy, gates), tr<T>(g_out, y, ggg)}, out, P * O * IJ,
                                                 stream)));
}

int fsc_mix_dbl_bwd_grad_g(int dtype, const void* g_out, const void* y, const void* ggy, const void* w, const void* ggw,
                           void* out, int64_t B, int64_t P, int64_t K, int64_t IJ, int64_t O, void* stream) {
  FSC_TRY(check_mix(dtype, B, P, K, IJ, O));
  const Dims d = mdims(B, P, K, IJ, O);
  FSC_DISPATCH(dtype, return (run_elem<T, K_MGT>(d, {tr<T>(g_out, ggy, w), tr<T>(g_out, y, ggw)}, out, B * P,
                                                   stream)));
}

}  // extern "C"
