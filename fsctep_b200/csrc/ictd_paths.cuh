// Compile-time structure of the lmax = 2, path_policy = "full" ICTD tensor product.
//
// Paths (l1, l2, l3) in the reference enumeration order (models/ictd_irreps.py:801-821):
//   p:  0       1       2       3       4       5       6       7       8       9       10
//      (0,0,0) (0,1,1) (0,2,2) (1,0,1) (1,1,0) (1,1,2) (1,2,1) (2,0,2) (2,1,1) (2,2,0) (2,2,2)
// Node features are stored [node][k][c] with k = l*l + m (9 components) and c the channel.
//
// Per-node accumulators of a conv2 layer use two layouts (each row holds C channels):
//   Z (forward, grouped by l3):  zrow(p, kk) = OFF3[l3] + kk * NP3[l3] + RANK3[p], kk < 2*l3+1
//   R (backward dx, grouped by l1): rrow(p, m1) = OFF1[l1] + m1 * NP1[l1] + RANK1[p], m1 < 2*l1+1
// so that for every l3 (l1) the rows of one node that feed one output component are contiguous
// and the channel mix is a plain GEMM with K = NP3[l3]*C (NP1[l1]*C).
// Per-edge coupled harmonics Yt[q], q = QOFF[p] + m1*(2*l3+1) + kk (115 entries):
//   Yt[q] = gate_p * sum_{m2} CG_p[m1, m2, kk] * Y_{l2}[m2]
#pragma once

// Tables are switch statements rather than local arrays: with a loop index that the compiler
// unrolls they fold to constants, where a local array may be materialised in local memory.

namespace ictd2 {

constexpr int NP = 11;
constexpr int NK = 9;
constexpr int NZ = 35;
constexpr int NQ = 115;
constexpr int NMONO = 10;

__host__ __device__ constexpr int L1(int p) {
  return p < 3 ? 0 : (p < 7 ? 1 : 2);
}
__host__ __device__ constexpr int L2(int p) {
  switch (p) {
    case 0: case 3: case 7: return 0;
    case 1: case 4: case 5: case 8: return 1;
    default: return 2;  // p = 2, 6, 9, 10
  }
}
__host__ __device__ constexpr int L3(int p) {
  switch (p) {
    case 0: case 4: case 9: return 0;
    case 1: case 3: case 6: case 8: return 1;
    default: return 2;  // p = 2, 5, 7, 10
  }
}
__host__ __device__ constexpr int KB(int l) { return l * l; }
__host__ __device__ constexpr int NP3(int l3) { return l3 == 0 ? 3 : 4; }
__host__ __device__ constexpr int OFF3(int l3) { return l3 == 0 ? 0 : (l3 == 1 ? 3 : 15); }
__host__ __device__ constexpr int RANK3(int p) {
  switch (p) {
    case 0: case 1: case 2: return 0;
    case 3: case 4: case 5: return 1;
    case 6: case 7: case 9: return 2;
    default: return 3;  // p = 8, 10
  }
}
__host__ __device__ constexpr int NP1(int l1) { return l1 == 0 ? 3 : 4; }
__host__ __device__ constexpr int OFF1(int l1) { return l1 == 0 ? 0 : (l1 == 1 ? 3 : 15); }
__host__ __device__ constexpr int RANK1(int p) {
  switch (p) {
    case 0: case 3: case 7: return 0;
    case 1: case 4: case 8: return 1;
    case 2: case 5: case 9: return 2;
    default: return 3;  // p = 6, 10
  }
}
__host__ __device__ constexpr int QOFF(int p) {
  switch (p) {
    case 0: return 0;
    case 1: return 1;
    case 2: return 4;
    case 3: return 9;
    case 4: return 18;
    case 5: return 21;
    case 6: return 36;
    case 7: return 45;
    case 8: return 70;
    case 9: return 85;
    default: return 90;  // p = 10
  }
}
__host__ __device__ constexpr int zrow(int p, int kk) { return OFF3(L3(p)) + kk * NP3(L3(p)) + RANK3(p); }
__host__ __device__ constexpr int rrow(int p, int m1) { return OFF1(L1(p)) + m1 * NP1(L1(p)) + RANK1(p); }
__host__ __device__ constexpr int qidx(int p, int m1, int kk) { return QOFF(p) + m1 * (2 * L3(p) + 1) + kk; }

// Paths with l1 = G: p in [P_LO(G), P_HI(G)), their Q entries [QOFF(P_LO), Q_END(G)).
__host__ __device__ constexpr int P_LO(int G) { return G == 0 ? 0 : (G == 1 ? 3 : 7); }
__host__ __device__ constexpr int P_HI(int G) { return G == 0 ? 3 : (G == 1 ? 7 : 11); }
__host__ __device__ constexpr int Q_END(int G) { return G == 2 ? NQ : QOFF(P_HI(G)); }

// conv1 paths (l, 0, l): 0, 3, 7
__host__ __device__ constexpr int P1PATH(int l) { return l == 0 ? 0 : (l == 1 ? 3 : 7); }

// Layout of the float `tables` block (fsc_ictd_weights::tables).
constexpr int TAB_YPOLY = 0;    // [NMONO][NK]: Y[k] = sum_j ypoly[j][k] * mono_j(n)
constexpr int TAB_CG2 = 90;     // [NQ][5]:  Yt0[q] = sum_m cg2[q][m] * Y[KB(l2)+m]
constexpr int TAB_CG1 = 665;    // [NK][5]:  Y1[l*l+k] = sum_m cg1[l*l+k][m] * Y[l*l+m]
constexpr int TAB_P5 = 710;     // [3] product_5 0e factors
constexpr int TAB_FLOATS = 720;

// Monomials of n = (x, y, z): 1, z, y, x, zz, yz, yy, xz, xy, xx (ictd_fast.py:41-48 order).
__device__ __forceinline__ void monomials(float x, float y, float z, float* m) {
  m[0] = 1.f; m[1] = z; m[2] = y; m[3] = x;
  m[4] = z * z; m[5] = y * z; m[6] = y * y; m[7] = x * z; m[8] = x * y; m[9] = x * x;
}
// d mono_j / d(x, y, z)
__device__ __forceinline__ void monomial_grads(float x, float y, float z, float* gx, float* gy, float* gz) {
  gx[0] = 0; gy[0] = 0; gz[0] = 0;
  gx[1] = 0; gy[1] = 0; gz[1] = 1;
  gx[2] = 0; gy[2] = 1; gz[2] = 0;
  gx[3] = 1; gy[3] = 0; gz[3] = 0;
  gx[4] = 0; gy[4] = 0; gz[4] = 2 * z;
  gx[5] = 0; gy[5] = z; gz[5] = y;
  gx[6] = 0; gy[6] = 2 * y; gz[6] = 0;
  gx[7] = z; gy[7] = 0; gz[7] = x;
  gx[8] = y; gy[8] = x; gz[8] = 0;
  gx[9] = 2 * x; gy[9] = 0; gz[9] = 0;
}

}  // namespace ictd2
