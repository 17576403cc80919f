// Screened exact Hartree energy over the significant pairs (gs_dft/coulomb/stream.py:249-320):
//   E_J = 1/2 sum_{a,b} q_a q_b (a|b),  q_a = w_a sum_o occ_o C_io C_jo,
//   (a|b) = KN_a KN_b (2/sqrt(pi)) pi^3 sum_t w_t det(G_t)^-1/2 exp(-v^T G_t^-1 v)
// with G_t the 6x6 precision [[A_a + t^2, -t^2], [-t^2, A_b + t^2]]. Written through
// H = A_a^-1 + A_b^-1 (C = H^-1): det G_t = det A_a det A_b det H D(t^2) and the exponent is
// t^2 N(t^2)/D(t^2), D(s) = det(C + s I) = s^3 + I1 s^2 + I2 s + I3 and
// N(s) = d.C adj(C + s I) d = q2 s^2 + (I1 q2 - |C d|^2) s + I3 |d|^2, d = P_a - P_b, where
// I1 = tr adj(H) / det H, I2 = tr H / det H, I3 = 1 / det H, q2 = d.adj(H) d / det H. The same
// 20-node rule as the reference's Schur kernel integrates the same function of t.
// One bra representative per thread, ket tiles staged in shared memory, ket splits filling the
// waves, fixed-order reductions (bitwise reproducible).
#include "common.cuh"

namespace gsdft {

constexpr int kXF = 12;          // per pair: A^-1 (xx yy zz xy xz yz), P (3), g = KN det(A)^-1/2, q, 0
constexpr int kXThreads = 128;   // bra representatives per CTA
constexpr int kXTile = 64;       // ket records per staged tile
constexpr int kXBits = 6;
constexpr size_t kXDynSmem = sizeof(double) * GSDFT_NQUAD * (1 << kXBits);

__global__ void exact_prep_kernel(const double* __restrict__ rec, int64_t n,
                                  double* __restrict__ xr) {
  const int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n) return;
  const double* r = rec + a * GSDFT_REC_FIELDS;
  double il[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) il[c] = 1.0 / r[GSDFT_REC_L0 + c];
  auto U = [&](int row, int col) { return r[GSDFT_REC_U00 + 3 * row + col]; };
  auto ainv = [&](int p, int s) {
    return U(p, 0) * U(s, 0) * il[0] + U(p, 1) * U(s, 1) * il[1] + U(p, 2) * U(s, 2) * il[2];
  };
  double* o = xr + a * kXF;
  o[0] = ainv(0, 0);
  o[1] = ainv(1, 1);
  o[2] = ainv(2, 2);
  o[3] = ainv(0, 1);
  o[4] = ainv(0, 2);
  o[5] = ainv(1, 2);
  o[6] = r[GSDFT_REC_P0];
  o[7] = r[GSDFT_REC_P1];
  o[8] = r[GSDFT_REC_P2];
  const double detA = r[GSDFT_REC_L0] * r[GSDFT_REC_L1] * r[GSDFT_REC_L2];
  o[9] = (r[GSDFT_REC_KN] * (1.0 / kPref)) * rsqrt_pos(detA);
  o[10] = r[GSDFT_REC_Q];
  o[11] = 0.0;
}

// part[split][a] = sum over the split's kets b of q_b (a|b).
__global__ void __launch_bounds__(kXThreads)
    exact_j_kernel(const double* __restrict__ xr, int64_t n, int64_t per_split,
                   double* __restrict__ part) {
  __shared__ double tile[kXTile * kXF];
  extern __shared__ __align__(16) double etab[];
  load_wexp2_tables<kXBits>(etab);
  const int64_t a = blockIdx.x * (int64_t)kXThreads + threadIdx.x;
  const bool has = a < n;
  const double* ra = xr + (has ? a : 0) * kXF;
  const double h0a = has ? ra[0] : 1.0, h1a = has ? ra[1] : 1.0, h2a = has ? ra[2] : 1.0;
  const double h3a = has ? ra[3] : 0.0, h4a = has ? ra[4] : 0.0, h5a = has ? ra[5] : 0.0;
  const double pxa = has ? ra[6] : 0.0, pya = has ? ra[7] : 0.0, pza = has ? ra[8] : 0.0;
  const double ga = has ? ra[9] : 0.0;
  const int64_t b0 = blockIdx.y * per_split;
  const int64_t b1 = imin64(b0 + per_split, n);
  double J = 0.0;
  for (int64_t t0 = b0; t0 < b1; t0 += kXTile) {
    const int cnt = (int)imin64(kXTile, b1 - t0);
    __syncthreads();  // previous tile consumed (and the exp2 table loaded)
    for (int k = threadIdx.x; k < cnt * kXF; k += kXThreads) tile[k] = xr[t0 * kXF + k];
    __syncthreads();
    if (!has) continue;
    for (int k = 0; k < cnt; ++k) {
      const double* rb = tile + k * kXF;
      const double h00 = h0a + rb[0], h11 = h1a + rb[1], h22 = h2a + rb[2];
      const double h01 = h3a + rb[3], h02 = h4a + rb[4], h12 = h5a + rb[5];
      // adjugate of the symmetric H, its determinant and trace
      const double c00 = h11 * h22 - h12 * h12, c11 = h00 * h22 - h02 * h02;
      const double c22 = h00 * h11 - h01 * h01, c01 = h02 * h12 - h01 * h22;
      const double c02 = h01 * h12 - h02 * h11, c12 = h01 * h02 - h00 * h12;
      const double detH = h00 * c00 + h01 * c01 + h02 * c02;
      const double rd = 1.0 / detH;
      const double I1 = (c00 + c11 + c22) * rd;
      const double I2 = (h00 + h11 + h22) * rd;
      const double I3 = rd;
      const double d0 = pxa - rb[6], d1 = pya - rb[7], d2 = pza - rb[8];
      const double e0 = c00 * d0 + c01 * d1 + c02 * d2;
      const double e1 = c01 * d0 + c11 * d1 + c12 * d2;
      const double e2 = c02 * d0 + c12 * d1 + c22 * d2;
      const double q2 = (d0 * e0 + d1 * e1 + d2 * e2) * rd;
      const double cd2 = (e0 * e0 + e1 * e1 + e2 * e2) * (rd * rd);
      const double q1 = fma(I1, q2, -cd2);
      const double q0 = I3 * (d0 * d0 + d1 * d1 + d2 * d2);
      double acc = 0.0;
#pragma unroll
      for (int nq = 0; nq < GSDFT_NQUAD; ++nq) {
        const double s = kQuadT2[nq];
        const double D = fma(fma(s + I1, s, I2), s, I3);
        const double N = fma(fma(q2, s, q1), s, q0);
        const double y = rsqrt_pos(D);
        const double ex = (-kLog2e * N) * (y * y);
        acc = fma(y, wexp2<kXBits>(ex, s, etab + (nq << kXBits)), acc);
      }
      J = fma(rb[10] * rb[9] * rsqrt_pos(detH), acc, J);
    }
  }
  if (has) part[blockIdx.y * n + a] = (kPref * ga) * J;
}

// J[a] = sum_s part[s][a] in split order; e[blk] = block sums of q_a J_a (fixed tree).
__global__ void __launch_bounds__(256)
    exact_fold_kernel(const double* __restrict__ part, int S, int64_t n,
                      const double* __restrict__ xr, double* __restrict__ J,
                      double* __restrict__ blk) {
  __shared__ double s[256];
  const int64_t a = blockIdx.x * 256LL + threadIdx.x;
  double e = 0.0;
  if (a < n) {
    double acc = 0.0;
    for (int k = 0; k < S; ++k) acc += part[(int64_t)k * n + a];
    J[a] = acc;
    e = xr[a * kXF + 10] * acc;
  }
  s[threadIdx.x] = e;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) blk[blockIdx.x] = s[0];
}

__global__ void __launch_bounds__(256)
    exact_energy_kernel(const double* __restrict__ blk, int64_t nb, double* __restrict__ E) {
  __shared__ double s[256];
  double acc = 0.0;
  for (int64_t b = threadIdx.x; b < nb; b += 256) acc += blk[b];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *E = 0.5 * s[0];
}

// ------------------------------------------------------------------------------------------------
// Reverse pass of E_J = 1/2 sum_{a,b} q_a q_b (a|b) (the gradient the reference takes by autodiff of
// gs_dft/coulomb/stream.py:249-320). With H = A_a^-1 + A_b^-1, d = P_a - P_b, g = KN det(A)^-1/2:
//   (a|b) = kPref g_a g_b F(H, d),  F = sum_n w_n det(I + s_n H)^-1/2 exp(-s_n d.K_n d),
//   K_n = (I + s_n H)^-1 = [I + s_n (tr H I - H) + s_n^2 adj H] / Delta_n, Delta_n = det(I + s_n H),
// so with u_n = K_n d and f_n = w_n Delta_n^-1/2 exp(-s_n d.u_n):
//   dF/dH = sum_n f_n (-1/2 s_n K_n + s_n^2 u_n u_n^T),   dF/dd = -2 sum_n f_n s_n u_n.
// Expanding K_n and u_n = (d + s_n v + s_n^2 e) / Delta_n (v = tr H d - H d, e = adj H d) in powers
// of s_n, the node loop only sums nine scalars: F, c_k = sum f s^k / Delta (k = 1..3) and
// b_k = sum f s^k / Delta^2 (k = 2..6); the matrices are assembled once per (a, b):
//   dF/dH = -1/2 [c1 I + c2 (tr H I - H) + c3 adj H] + d alpha^T + v beta^T + e gamma^T,
//   alpha = b2 d + b3 v + b4 e, beta = b3 d + b4 v + b5 e, gamma = b4 d + b5 v + b6 e,
//   dF/dd = -2 (c1 d + c2 v + c3 e).
// part[split][f][a] (f < kXV): T = sum_b q_b g_b F, then the six entries of
// sum_b q_b g_b dF/dH (xx yy zz xy xz yz), then the three of sum_b q_b g_b dF/dd.
// ------------------------------------------------------------------------------------------------
constexpr int kXV = 10;

__global__ void __launch_bounds__(kXThreads)
    exact_vjp_kernel(const double* __restrict__ xr, int64_t n, int64_t per_split,
                     double* __restrict__ part) {
  __shared__ double tile[kXTile * kXF];
  extern __shared__ __align__(16) double etab[];
  load_wexp2_tables<kXBits>(etab);
  const int64_t a = blockIdx.x * (int64_t)kXThreads + threadIdx.x;
  const bool has = a < n;
  const double* ra = xr + (has ? a : 0) * kXF;
  const double h0a = has ? ra[0] : 1.0, h1a = has ? ra[1] : 1.0, h2a = has ? ra[2] : 1.0;
  const double h3a = has ? ra[3] : 0.0, h4a = has ? ra[4] : 0.0, h5a = has ? ra[5] : 0.0;
  const double pxa = has ? ra[6] : 0.0, pya = has ? ra[7] : 0.0, pza = has ? ra[8] : 0.0;
  const int64_t b0 = blockIdx.y * per_split;
  const int64_t b1 = imin64(b0 + per_split, n);
  double acc[kXV];
#pragma unroll
  for (int f = 0; f < kXV; ++f) acc[f] = 0.0;
  for (int64_t t0 = b0; t0 < b1; t0 += kXTile) {
    const int cnt = (int)imin64(kXTile, b1 - t0);
    __syncthreads();  // previous tile consumed (and the exp2 table loaded)
    for (int k = threadIdx.x; k < cnt * kXF; k += kXThreads) tile[k] = xr[t0 * kXF + k];
    __syncthreads();
    if (!has) continue;
    for (int k = 0; k < cnt; ++k) {
      const double* rb = tile + k * kXF;
      const double h00 = h0a + rb[0], h11 = h1a + rb[1], h22 = h2a + rb[2];
      const double h01 = h3a + rb[3], h02 = h4a + rb[4], h12 = h5a + rb[5];
      const double c00 = h11 * h22 - h12 * h12, c11 = h00 * h22 - h02 * h02;
      const double c22 = h00 * h11 - h01 * h01, c01 = h02 * h12 - h01 * h22;
      const double c02 = h01 * h12 - h02 * h11, c12 = h01 * h02 - h00 * h12;
      const double detH = h00 * c00 + h01 * c01 + h02 * c02;
      const double trH = h00 + h11 + h22, trC = c00 + c11 + c22;
      const double d0 = pxa - rb[6], d1 = pya - rb[7], d2 = pza - rb[8];
      const double e0 = c00 * d0 + c01 * d1 + c02 * d2;
      const double e1 = c01 * d0 + c11 * d1 + c12 * d2;
      const double e2 = c02 * d0 + c12 * d1 + c22 * d2;
      const double v0 = trH * d0 - (h00 * d0 + h01 * d1 + h02 * d2);
      const double v1 = trH * d1 - (h01 * d0 + h11 * d1 + h12 * d2);
      const double v2 = trH * d2 - (h02 * d0 + h12 * d1 + h22 * d2);
      const double n0 = d0 * d0 + d1 * d1 + d2 * d2;
      const double m0 = -kLog2e * n0;                                  // d.adj(I + sH) d, -log2 e
      const double m1 = -kLog2e * (d0 * v0 + d1 * v1 + d2 * v2);
      const double m2 = -kLog2e * (d0 * e0 + d1 * e1 + d2 * e2);
      double F = 0.0, c1 = 0.0, c2 = 0.0, c3 = 0.0;
      double b2 = 0.0, b3 = 0.0, b4 = 0.0, b5 = 0.0, b6 = 0.0;
#pragma unroll 4  // full unrolling spills (255 registers); 4 keeps 126
      for (int nq = 0; nq < GSDFT_NQUAD; ++nq) {
        const double s = kQuadT2[nq];
        const double D = fma(fma(fma(detH, s, trC), s, trH), s, 1.0);  // det(I + sH)
        const double y = rsqrt_pos(D);
        const double iD = y * y;
        const double ex = fma(fma(m2, s, m1), s, m0) * iD;             // -log2e d.K d
        const double f = y * wexp2<kXBits>(ex, s, etab + (nq << kXBits));
        const double fD = f * iD, fD2 = fD * iD;
        F += f;
        c1 = fma(s, fD, c1);
        c2 = fma(kQuadSPow[0][nq], fD, c2);
        c3 = fma(kQuadSPow[1][nq], fD, c3);
        b2 = fma(kQuadSPow[0][nq], fD2, b2);
        b3 = fma(kQuadSPow[1][nq], fD2, b3);
        b4 = fma(kQuadSPow[2][nq], fD2, b4);
        b5 = fma(kQuadSPow[3][nq], fD2, b5);
        b6 = fma(kQuadSPow[4][nq], fD2, b6);
      }
      const double wb = rb[10] * rb[9];  // q_b g_b
      acc[0] = fma(wb, F, acc[0]);
      // -1/2 [c1 I + c2 (tr H I - H) + c3 adj H] + d alpha^T + v beta^T + e gamma^T
      const double al0 = b2 * d0 + b3 * v0 + b4 * e0, al1 = b2 * d1 + b3 * v1 + b4 * e1,
                   al2 = b2 * d2 + b3 * v2 + b4 * e2;
      const double be0 = b3 * d0 + b4 * v0 + b5 * e0, be1 = b3 * d1 + b4 * v1 + b5 * e1,
                   be2 = b3 * d2 + b4 * v2 + b5 * e2;
      const double ga0 = b4 * d0 + b5 * v0 + b6 * e0, ga1 = b4 * d1 + b5 * v1 + b6 * e1,
                   ga2 = b4 * d2 + b5 * v2 + b6 * e2;
      const double k00 = -0.5 * (c1 + c2 * (trH - h00) + c3 * c00);
      const double k11 = -0.5 * (c1 + c2 * (trH - h11) + c3 * c11);
      const double k22 = -0.5 * (c1 + c2 * (trH - h22) + c3 * c22);
      const double k01 = -0.5 * (c3 * c01 - c2 * h01);
      const double k02 = -0.5 * (c3 * c02 - c2 * h02);
      const double k12 = -0.5 * (c3 * c12 - c2 * h12);
      acc[1] = fma(wb, k00 + d0 * al0 + v0 * be0 + e0 * ga0, acc[1]);
      acc[2] = fma(wb, k11 + d1 * al1 + v1 * be1 + e1 * ga1, acc[2]);
      acc[3] = fma(wb, k22 + d2 * al2 + v2 * be2 + e2 * ga2, acc[3]);
      acc[4] = fma(wb, k01 + d0 * al1 + v0 * be1 + e0 * ga1, acc[4]);
      acc[5] = fma(wb, k02 + d0 * al2 + v0 * be2 + e0 * ga2, acc[5]);
      acc[6] = fma(wb, k12 + d1 * al2 + v1 * be2 + e1 * ga2, acc[6]);
      const double w2 = -2.0 * wb;
      acc[7] = fma(w2, c1 * d0 + c2 * v0 + c3 * e0, acc[7]);
      acc[8] = fma(w2, c1 * d1 + c2 * v1 + c3 * e1, acc[8]);
      acc[9] = fma(w2, c1 * d2 + c2 * v2 + c3 * e2, acc[9]);
    }
  }
  if (has) {
#pragma unroll
    for (int f = 0; f < kXV; ++f) part[((int64_t)blockIdx.y * kXV + f) * n + a] = acc[f];
  }
}

// Per representative: the splits' sums in split order, then the cotangents of (A_hat, P, KN) and
// dE/dq of g_E E_J (xc, GSDFT_XC_FIELDS per representative). With G the H-sum and T the F-sum,
//   dE/dq_a = kPref g_a T,  A^-1 bar = q_a kPref g_a G,  P bar = q_a kPref g_a (d-sum),
//   g bar = q_a kPref T  ->  KN bar = g bar det(A)^-1/2,
//   A_hat bar = -A^-1 (A^-1 bar) A^-1 - 1/2 g bar g_a A^-1   (g's det(A)^-1/2).
__global__ void exact_vjp_fold_kernel(const double* __restrict__ part, int S, int64_t n,
                                      const double* __restrict__ xr,
                                      const double* __restrict__ rec,
                                      const double* __restrict__ g_E, double* __restrict__ xc) {
  const int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n) return;
  double v[kXV];
#pragma unroll
  for (int f = 0; f < kXV; ++f) {
    double t = 0.0;
    for (int s = 0; s < S; ++s) t += part[((int64_t)s * kXV + f) * n + a];
    v[f] = t;
  }
  const double ge = g_E ? *g_E : 1.0;
  const double* x = xr + a * kXF;
  const double* r = rec + a * GSDFT_REC_FIELDS;
  const double g = x[9], q = x[10];
  const double Jq = ge * kPref * g * v[0];
  const double sc = ge * q * kPref * g;       // scale of the H- and d-sums
  const double gbar = ge * q * kPref * v[0];
  const double rdet = rsqrt_pos(r[GSDFT_REC_L0] * r[GSDFT_REC_L1] * r[GSDFT_REC_L2]);
  // A^-1 (symmetric) and X = A^-1 G A^-1 with G = sc * (H-sum)
  const double Ai[3][3] = {{x[0], x[3], x[4]}, {x[3], x[1], x[5]}, {x[4], x[5], x[2]}};
  const double G[3][3] = {{sc * v[1], sc * v[4], sc * v[5]},
                          {sc * v[4], sc * v[2], sc * v[6]},
                          {sc * v[5], sc * v[6], sc * v[3]}};
  double AG[3][3];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) AG[i][j] = Ai[i][0] * G[0][j] + Ai[i][1] * G[1][j] + Ai[i][2] * G[2][j];
  auto X = [&](int i, int j) { return AG[i][0] * Ai[0][j] + AG[i][1] * Ai[1][j] + AG[i][2] * Ai[2][j]; };
  const double hg = -0.5 * gbar * g;
  double* o = xc + a * GSDFT_XC_FIELDS;
  o[GSDFT_XC_A00] = fma(hg, Ai[0][0], -X(0, 0));
  o[GSDFT_XC_A11] = fma(hg, Ai[1][1], -X(1, 1));
  o[GSDFT_XC_A22] = fma(hg, Ai[2][2], -X(2, 2));
  o[GSDFT_XC_A01] = fma(hg, Ai[0][1], -0.5 * (X(0, 1) + X(1, 0)));
  o[GSDFT_XC_A02] = fma(hg, Ai[0][2], -0.5 * (X(0, 2) + X(2, 0)));
  o[GSDFT_XC_A12] = fma(hg, Ai[1][2], -0.5 * (X(1, 2) + X(2, 1)));
  o[GSDFT_XC_P0] = sc * v[7];
  o[GSDFT_XC_P1] = sc * v[8];
  o[GSDFT_XC_P2] = sc * v[9];
  o[GSDFT_XC_KN] = gbar * rdet;
  o[GSDFT_XC_J] = Jq;
}

static int exact_splits(int64_t n) {
  static const int per_sm = [] {
    int v = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, exact_j_kernel, kXThreads, kXDynSmem);
    return v > 0 ? v : 1;
  }();
  const int sms = device_sms();
  const int64_t tiles = (n + kXThreads - 1) / kXThreads;
  const int64_t max_s = imin64(64, imax64(1, n / kXTile));
  return best_splits(tiles, (int64_t)sms * per_sm, max_s);
}

}  // namespace gsdft

using namespace gsdft;

static int exact_vjp_splits(int64_t n) {
  static const int per_sm = [] {
    int v = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, exact_vjp_kernel, kXThreads, kXDynSmem);
    return v > 0 ? v : 1;
  }();
  const int sms = device_sms();
  const int64_t tiles = (n + kXThreads - 1) / kXThreads;
  const int64_t max_s = imin64(64, imax64(1, n / kXTile));
  return best_splits(tiles, (int64_t)sms * per_sm, max_s);
}

extern "C" size_t gsdft_exact_j_workspace_size(int64_t n_rep) {
  const int64_t n = imax64(n_rep, 1);
  const int S = exact_splits(n);
  Sizer z;
  z.take<double>((size_t)n * kXF);
  z.take<double>((size_t)S * n);
  z.take<double>((size_t)(n + 255) / 256);
  return z.off + 256;
}

extern "C" int gsdft_exact_j(const double* rec, int64_t n_rep, double* J, double* E, void* ws,
                             size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_rep < (int64_t(1) << 31), "bad sizes");
  GSDFT_REQUIRE(E && ws, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(E, 0, sizeof(double), st));
    return GSDFT_OK;
  }
  GSDFT_REQUIRE(rec && J, "null pointer");
  const int64_t n = n_rep;
  const int S = exact_splits(n);
  Carver c(ws, ws_bytes);
  double* xr = c.take<double>((size_t)n * kXF);
  double* part = c.take<double>((size_t)S * n);
  double* blk = c.take<double>((size_t)(n + 255) / 256);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "exact-J workspace too small");
  exact_prep_kernel<<<grid_1d(n, 256), 256, 0, st>>>(rec, n, xr);
  GSDFT_LAUNCHED("exact_prep");
  const int64_t per_split = (n + S - 1) / S;
  dim3 grid((unsigned)((n + kXThreads - 1) / kXThreads), (unsigned)S);
  exact_j_kernel<<<grid, kXThreads, kXDynSmem, st>>>(xr, n, per_split, part);
  GSDFT_LAUNCHED("exact_j");
  const int64_t nb = (n + 255) / 256;
  exact_fold_kernel<<<(unsigned)nb, 256, 0, st>>>(part, S, n, xr, J, blk);
  GSDFT_LAUNCHED("exact_fold");
  exact_energy_kernel<<<1, 256, 0, st>>>(blk, nb, E);
  GSDFT_LAUNCHED("exact_energy");
  return GSDFT_OK;
}

extern "C" size_t gsdft_exact_j_vjp_workspace_size(int64_t n_rep) {
  const int64_t n = imax64(n_rep, 1);
  const int S = exact_vjp_splits(n);
  Sizer z;
  z.take<double>((size_t)n * kXF);
  z.take<double>((size_t)S * kXV * n);
  return z.off + 256;
}

extern "C" int gsdft_exact_j_vjp(const double* rec, int64_t n_rep, const double* g_E, double* xc,
                                 void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_rep < (int64_t(1) << 31), "bad sizes");
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && xc && ws, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = n_rep;
  const int S = exact_vjp_splits(n);
  Carver c(ws, ws_bytes);
  double* xr = c.take<double>((size_t)n * kXF);
  double* part = c.take<double>((size_t)S * kXV * n);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "exact-J reverse workspace too small");
  exact_prep_kernel<<<grid_1d(n, 256), 256, 0, st>>>(rec, n, xr);
  GSDFT_LAUNCHED("exact_prep");
  const int64_t per_split = (n + S - 1) / S;
  dim3 grid((unsigned)((n + kXThreads - 1) / kXThreads), (unsigned)S);
  exact_vjp_kernel<<<grid, kXThreads, kXDynSmem, st>>>(xr, n, per_split, part);
  GSDFT_LAUNCHED("exact_vjp");
  exact_vjp_fold_kernel<<<grid_1d(n, 128), 128, 0, st>>>(part, S, n, xr, rec, g_E, xc);
  GSDFT_LAUNCHED("exact_vjp_fold");
  return GSDFT_OK;
}
