// Screened exact Hartree energy over the significant pairs (gs_dft/coulomb/stream.py:249-458) and
// its reverse pass:
//   E_J = 1/2 sum_{a,b} q_a q_b (a|b),  q_a = w_a sum_o occ_o C_io C_jo,
//   (a|b) = KN_a KN_b (2/sqrt(pi)) pi^3 integral_0^inf dt det(G_t)^-1/2 exp(-v^T G_t^-1 v)
// with G_t the 6x6 precision [[A_a + t^2, -t^2], [-t^2, A_b + t^2]]. With H = A_a^-1 + A_b^-1 and
// d = P_a - P_b, det G_t = det A_a det A_b det(I + s H) and the exponent is s d.(I + s H)^-1 d at
// s = t^2, so with g = KN det(A)^-1/2:
//   (a|b) = kPref g_a g_b F(H, d),  F = sum_n w_n Delta_n^-1/2 exp(-s_n d.K_n d),
//   Delta_n = det(I + s_n H) = 1 + s_n (tr H + s_n (tr adj H + s_n det H)),
//   d.K_n d = d.adj(I + s_n H) d / Delta_n = (|d|^2 + s_n d.v + s_n^2 d.e) / Delta_n,
// v = tr H d - H d, e = adj H d (adj(I + sH) = I + s (tr H I - H) + s^2 adj H).
// Two quadrature rules of the reference (the `rule` argument):
//   GSDFT_EXACT_SCHUR20: the 20-node half-line rule of full_eri_block_schur (:249-283),
//       s_n = t_n^2, w_n its weights;
//   GSDFT_EXACT_FUSED32: the 32-node Boys-scaled rule of full_eri_block_fused (:323-458), s_k =
//       rho c_k with the per-(a, b) scale rho = I3^(1/3) / (1 + q2), I3 = 1 / det H,
//       q2 = d.H^-1 d, and F = sqrt(rho) sum_k e_k Delta_k^-1/2 exp(-s_k d.K_k d).
// One bra representative per thread, ket tiles staged in shared memory, ket splits filling the
// waves, fixed-order reductions (bitwise reproducible).
#include "common.cuh"

namespace gsdft {

constexpr int kXF = 12;          // per pair: A^-1 (xx yy zz xy xz yz), P (3), g = KN det(A)^-1/2, q, 0
constexpr int kXThreads = 128;   // bra representatives per CTA
constexpr int kXTile = 64;       // ket records per staged tile
constexpr int kXBits = 6;
constexpr int kXV = 10;          // reverse-pass sums per representative

template <int kRule>
__host__ __device__ constexpr int rule_nodes() {
  return kRule == GSDFT_EXACT_FUSED32 ? GSDFT_NBOYS : GSDFT_NQUAD;
}
template <int kRule>
__host__ __device__ constexpr size_t rule_smem() {
  return sizeof(double) * rule_nodes<kRule>() * (1 << kXBits);
}

// The rule's per-node weighted exp2 tables into shared memory (all threads; the caller syncs).
template <int kRule>
__device__ __forceinline__ void load_rule_tables(double* dst) {
  const double* src = kRule == GSDFT_EXACT_FUSED32 ? kExp2WTabBoys6 : kExp2WTab6;
  for (int k = threadIdx.x; k < rule_nodes<kRule>() * (1 << kXBits); k += blockDim.x)
    dst[k] = src[k];
}

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

// The bra's own A^-1 and P (registers), and the pair-pair quantities of one (a, b).
struct Bra {
  double h0, h1, h2, h3, h4, h5, px, py, pz;
};

struct PairPair {
  double h00, h11, h22, h01, h02, h12;  // H = A_a^-1 + A_b^-1
  double c00, c11, c22, c01, c02, c12;  // adj H
  double detH, trH, trC;                // det H, tr H, tr adj H
  double d0, d1, d2, v0, v1, v2, e0, e1, e2;
  double n0, n1, n2;                    // |d|^2, d.v, d.e
};

__device__ __forceinline__ void pair_pair(const Bra& A, const double* __restrict__ rb, PairPair& g) {
  g.h00 = A.h0 + rb[0];
  g.h11 = A.h1 + rb[1];
  g.h22 = A.h2 + rb[2];
  g.h01 = A.h3 + rb[3];
  g.h02 = A.h4 + rb[4];
  g.h12 = A.h5 + rb[5];
  g.c00 = g.h11 * g.h22 - g.h12 * g.h12;
  g.c11 = g.h00 * g.h22 - g.h02 * g.h02;
  g.c22 = g.h00 * g.h11 - g.h01 * g.h01;
  g.c01 = g.h02 * g.h12 - g.h01 * g.h22;
  g.c02 = g.h01 * g.h12 - g.h02 * g.h11;
  g.c12 = g.h01 * g.h02 - g.h00 * g.h12;
  g.detH = g.h00 * g.c00 + g.h01 * g.c01 + g.h02 * g.c02;
  g.trH = g.h00 + g.h11 + g.h22;
  g.trC = g.c00 + g.c11 + g.c22;
  g.d0 = A.px - rb[6];
  g.d1 = A.py - rb[7];
  g.d2 = A.pz - rb[8];
  g.e0 = g.c00 * g.d0 + g.c01 * g.d1 + g.c02 * g.d2;
  g.e1 = g.c01 * g.d0 + g.c11 * g.d1 + g.c12 * g.d2;
  g.e2 = g.c02 * g.d0 + g.c12 * g.d1 + g.c22 * g.d2;
  g.v0 = g.trH * g.d0 - (g.h00 * g.d0 + g.h01 * g.d1 + g.h02 * g.d2);
  g.v1 = g.trH * g.d1 - (g.h01 * g.d0 + g.h11 * g.d1 + g.h12 * g.d2);
  g.v2 = g.trH * g.d2 - (g.h02 * g.d0 + g.h12 * g.d1 + g.h22 * g.d2);
  g.n0 = g.d0 * g.d0 + g.d1 * g.d1 + g.d2 * g.d2;
  g.n1 = g.d0 * g.v0 + g.d1 * g.v1 + g.d2 * g.v2;
  g.n2 = g.d0 * g.e0 + g.d1 * g.e1 + g.d2 * g.e2;
}

// The fused rule's scale rho = det(H)^-1/3 / (1 + q2), q2 = d.adj H d / det H.
__device__ __forceinline__ double rule_rho(const PairPair& g) {
  return rcbrt(g.detH) / (1.0 + g.n2 / g.detH);
}

__device__ __forceinline__ Bra load_bra(const double* __restrict__ xr, int64_t a, bool has) {
  const double* ra = xr + (has ? a : 0) * kXF;
  Bra b;
  b.h0 = has ? ra[0] : 1.0;
  b.h1 = has ? ra[1] : 1.0;
  b.h2 = has ? ra[2] : 1.0;
  b.h3 = has ? ra[3] : 0.0;
  b.h4 = has ? ra[4] : 0.0;
  b.h5 = has ? ra[5] : 0.0;
  b.px = has ? ra[6] : 0.0;
  b.py = has ? ra[7] : 0.0;
  b.pz = has ? ra[8] : 0.0;
  return b;
}

// part[split][a] = sum over the split's kets b of q_b (a|b).
template <int kRule>
__global__ void __launch_bounds__(kXThreads)
    exact_j_kernel(const double* __restrict__ xr, int64_t n, int64_t per_split,
                   double* __restrict__ part) {
  __shared__ double tile[kXTile * kXF];
  extern __shared__ __align__(16) double etab[];
  load_rule_tables<kRule>(etab);
  const int64_t a = blockIdx.x * (int64_t)kXThreads + threadIdx.x;
  const bool has = a < n;
  const Bra A = load_bra(xr, a, has);
  const double ga = has ? xr[a * kXF + 9] : 0.0;
  const int64_t b0 = blockIdx.y * per_split;
  const int64_t b1 = imin64(b0 + per_split, n);
  double J = 0.0;
  for (int64_t t0 = b0; t0 < b1; t0 += kXTile) {
    const int cnt = (int)imin64(kXTile, b1 - t0);
    __syncthreads();  // previous tile consumed (and the exp2 tables loaded)
    for (int k = threadIdx.x; k < cnt * kXF; k += kXThreads) tile[k] = xr[t0 * kXF + k];
    __syncthreads();
    if (!has) continue;
    for (int k = 0; k < cnt; ++k) {
      const double* rb = tile + k * kXF;
      PairPair g;
      pair_pair(A, rb, g);
      const double m0 = -kLog2e * g.n0, m1 = -kLog2e * g.n1, m2 = -kLog2e * g.n2;
      double rho = 1.0;
      if (kRule == GSDFT_EXACT_FUSED32) rho = rule_rho(g);
      double acc = 0.0;
#pragma unroll 4
      for (int nq = 0; nq < rule_nodes<kRule>(); ++nq) {
        const double s = kRule == GSDFT_EXACT_FUSED32 ? rho * kBoysC[nq] : kQuadT2[nq];
        const double D = fma(fma(fma(g.detH, s, g.trC), s, g.trH), s, 1.0);  // det(I + sH)
        const double y = rsqrt_pos(D);
        const double ex = s * (fma(fma(m2, s, m1), s, m0) * (y * y));        // -log2e s d.K d
        acc = fma(y, wexp2x<kXBits>(ex, etab + (nq << kXBits)), acc);
      }
      if (kRule == GSDFT_EXACT_FUSED32) acc *= sqrt(rho);
      J = fma(rb[10] * rb[9], acc, J);
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
// Reverse pass of E_J (the gradient the reference takes by autodiff of its streamed blocks, with
// the fused rule's hand-written node VJP, gs_dft/coulomb/stream.py:144-189, 356-398). At fixed s,
// with u_n = K_n d and f_n = w_n Delta_n^-1/2 exp(-s_n d.u_n):
//   dF/dH = sum_n f_n (-1/2 s_n K_n + s_n^2 u_n u_n^T),   dF/dd = -2 sum_n f_n s_n u_n.
// Expanding K_n and u_n = (d + s_n v + s_n^2 e) / Delta_n in powers of s_n, the node loop sums nine
// scalars: F, c_k = sum f s^k / Delta (k = 1..3) and b_k = sum f s^k / Delta^2 (k = 2..6); the
// matrices are assembled once per (a, b):
//   dF/dH = -1/2 [c1 I + c2 (tr H I - H) + c3 adj H] + d alpha^T + v beta^T + e gamma^T,
//   alpha = b2 d + b3 v + b4 e, beta = b3 d + b4 v + b5 e, gamma = b4 d + b5 v + b6 e,
//   dF/dd = -2 (c1 d + c2 v + c3 e).
// The fused rule also depends on H and d through rho (F = sqrt(rho) sum_k f_k at s_k = rho c_k):
//   dF/drho = F / (2 rho) + sqrt(rho) sum_k c_k df_k/ds,  df/ds = f (-1/2 Delta'/Delta - |u|^2),
//   Delta' = tr H + 2 s tr adj H + 3 s^2 det H,  |u|^2 = |d + s v + s^2 e|^2 / Delta^2,
//   drho/dH = rho (-1/3 H^-1 + w w^T / (1 + q2)),  drho/dd = -2 rho w / (1 + q2),  w = H^-1 d.
// part[split][f][a] (f < kXV): T = sum_b q_b g_b F, then the six entries of
// sum_b q_b g_b dF/dH (xx yy zz xy xz yz), then the three of sum_b q_b g_b dF/dd.
// ------------------------------------------------------------------------------------------------
template <int kRule>
__global__ void __launch_bounds__(kXThreads)
    exact_vjp_kernel(const double* __restrict__ xr, int64_t n, int64_t per_split,
                     double* __restrict__ part) {
  constexpr bool kFused = kRule == GSDFT_EXACT_FUSED32;
  __shared__ double tile[kXTile * kXF];
  extern __shared__ __align__(16) double etab[];
  load_rule_tables<kRule>(etab);
  const int64_t a = blockIdx.x * (int64_t)kXThreads + threadIdx.x;
  const bool has = a < n;
  const Bra A = load_bra(xr, a, has);
  const int64_t b0 = blockIdx.y * per_split;
  const int64_t b1 = imin64(b0 + per_split, n);
  double acc[kXV];
#pragma unroll
  for (int f = 0; f < kXV; ++f) acc[f] = 0.0;
  for (int64_t t0 = b0; t0 < b1; t0 += kXTile) {
    const int cnt = (int)imin64(kXTile, b1 - t0);
    __syncthreads();  // previous tile consumed (and the exp2 tables loaded)
    for (int k = threadIdx.x; k < cnt * kXF; k += kXThreads) tile[k] = xr[t0 * kXF + k];
    __syncthreads();
    if (!has) continue;
    for (int k = 0; k < cnt; ++k) {
      const double* rb = tile + k * kXF;
      PairPair g;
      pair_pair(A, rb, g);
      const double m0 = -kLog2e * g.n0, m1 = -kLog2e * g.n1, m2 = -kLog2e * g.n2;
      double rho = 1.0, p1 = 0.0, p2 = 0.0, p3 = 0.0, p4 = 0.0;
      if (kFused) {
        rho = rule_rho(g);
        p1 = 2.0 * g.n1;
        p2 = (g.v0 * g.v0 + g.v1 * g.v1 + g.v2 * g.v2) + 2.0 * g.n2;
        p3 = 2.0 * (g.v0 * g.e0 + g.v1 * g.e1 + g.v2 * g.e2);
        p4 = g.e0 * g.e0 + g.e1 * g.e1 + g.e2 * g.e2;
      }
      double F = 0.0, c1 = 0.0, c2 = 0.0, c3 = 0.0;
      double b2 = 0.0, b3 = 0.0, b4 = 0.0, b5 = 0.0, b6 = 0.0;
      double A1 = 0.0, A2 = 0.0;  // fused: sum c_k f Delta'/Delta, sum c_k f |u|^2
#pragma unroll 4  // full unrolling spills; 4 keeps the fixed rule at 126 registers
      for (int nq = 0; nq < rule_nodes<kRule>(); ++nq) {
        const double s = kFused ? rho * kBoysC[nq] : kQuadT2[nq];
        const double D = fma(fma(fma(g.detH, s, g.trC), s, g.trH), s, 1.0);  // det(I + sH)
        const double y = rsqrt_pos(D);
        const double iD = y * y;
        const double ex = s * (fma(fma(m2, s, m1), s, m0) * iD);           // -log2e s d.K d
        const double f = y * wexp2x<kXBits>(ex, etab + (nq << kXBits));
        const double fD = f * iD, fD2 = fD * iD;
        double s2, s3, s4, s5, s6;
        if (kFused) {
          s2 = s * s;
          s3 = s2 * s;
          s4 = s2 * s2;
          s5 = s4 * s;
          s6 = s3 * s3;
        } else {
          s2 = kQuadSPow[0][nq];
          s3 = kQuadSPow[1][nq];
          s4 = kQuadSPow[2][nq];
          s5 = kQuadSPow[3][nq];
          s6 = kQuadSPow[4][nq];
        }
        F += f;
        c1 = fma(s, fD, c1);
        c2 = fma(s2, fD, c2);
        c3 = fma(s3, fD, c3);
        b2 = fma(s2, fD2, b2);
        b3 = fma(s3, fD2, b3);
        b4 = fma(s4, fD2, b4);
        b5 = fma(s5, fD2, b5);
        b6 = fma(s6, fD2, b6);
        if (kFused) {
          const double ck = kBoysC[nq];
          const double Dp = fma(fma(3.0 * g.detH, s, 2.0 * g.trC), s, g.trH);
          const double uu = fma(fma(fma(fma(p4, s, p3), s, p2), s, p1), s, g.n0);
          A1 = fma(ck * fD, Dp, A1);
          A2 = fma(ck * fD2, uu, A2);
        }
      }
      // the rho chain of the fused rule: F -> sqrt(rho) F, the fixed-s sums scaled alike, and
      // dF/drho times drho/dH (coefficients of adj H and e e^T) and drho/dd (coefficient of e)
      double rA = 0.0, rE = 0.0, rD = 0.0;
      if (kFused) {
        const double sq = sqrt(rho);
        const double dFdr = 0.5 * F / sq - sq * fma(0.5, A1, A2);
        F *= sq;
        c1 *= sq;
        c2 *= sq;
        c3 *= sq;
        b2 *= sq;
        b3 *= sq;
        b4 *= sq;
        b5 *= sq;
        b6 *= sq;
        const double iH = 1.0 / g.detH;
        const double kr = dFdr * rho;
        const double iq = 1.0 / (1.0 + g.n2 * iH);
        rA = (-1.0 / 3.0) * kr * iH;   // H^-1 = adj H / det H
        rE = kr * iq * (iH * iH);      // w w^T = e e^T / det H^2
        rD = -2.0 * kr * iq * iH;      // w = e / det H
      }
      const double wb = rb[10] * rb[9];  // q_b g_b
      acc[0] = fma(wb, F, acc[0]);
      const double al0 = b2 * g.d0 + b3 * g.v0 + b4 * g.e0, al1 = b2 * g.d1 + b3 * g.v1 + b4 * g.e1,
                   al2 = b2 * g.d2 + b3 * g.v2 + b4 * g.e2;
      const double be0 = b3 * g.d0 + b4 * g.v0 + b5 * g.e0, be1 = b3 * g.d1 + b4 * g.v1 + b5 * g.e1,
                   be2 = b3 * g.d2 + b4 * g.v2 + b5 * g.e2;
      const double ga0 = b4 * g.d0 + b5 * g.v0 + b6 * g.e0, ga1 = b4 * g.d1 + b5 * g.v1 + b6 * g.e1,
                   ga2 = b4 * g.d2 + b5 * g.v2 + b6 * g.e2;
      double k00 = -0.5 * (c1 + c2 * (g.trH - g.h00) + c3 * g.c00);
      double k11 = -0.5 * (c1 + c2 * (g.trH - g.h11) + c3 * g.c11);
      double k22 = -0.5 * (c1 + c2 * (g.trH - g.h22) + c3 * g.c22);
      double k01 = -0.5 * (c3 * g.c01 - c2 * g.h01);
      double k02 = -0.5 * (c3 * g.c02 - c2 * g.h02);
      double k12 = -0.5 * (c3 * g.c12 - c2 * g.h12);
      if (kFused) {
        k00 += rA * g.c00 + rE * g.e0 * g.e0;
        k11 += rA * g.c11 + rE * g.e1 * g.e1;
        k22 += rA * g.c22 + rE * g.e2 * g.e2;
        k01 += rA * g.c01 + rE * g.e0 * g.e1;
        k02 += rA * g.c02 + rE * g.e0 * g.e2;
        k12 += rA * g.c12 + rE * g.e1 * g.e2;
      }
      acc[1] = fma(wb, k00 + g.d0 * al0 + g.v0 * be0 + g.e0 * ga0, acc[1]);
      acc[2] = fma(wb, k11 + g.d1 * al1 + g.v1 * be1 + g.e1 * ga1, acc[2]);
      acc[3] = fma(wb, k22 + g.d2 * al2 + g.v2 * be2 + g.e2 * ga2, acc[3]);
      acc[4] = fma(wb, k01 + g.d0 * al1 + g.v0 * be1 + g.e0 * ga1, acc[4]);
      acc[5] = fma(wb, k02 + g.d0 * al2 + g.v0 * be2 + g.e0 * ga2, acc[5]);
      acc[6] = fma(wb, k12 + g.d1 * al2 + g.v1 * be2 + g.e1 * ga2, acc[6]);
      const double w2 = -2.0 * wb;
      acc[7] = fma(w2, c1 * g.d0 + c2 * g.v0 + c3 * g.e0, fma(wb * rD, g.e0, acc[7]));
      acc[8] = fma(w2, c1 * g.d1 + c2 * g.v1 + c3 * g.e1, fma(wb * rD, g.e1, acc[8]));
      acc[9] = fma(w2, c1 * g.d2 + c2 * g.v2 + c3 * g.e2, fma(wb * rD, g.e2, acc[9]));
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

// Ket splits filling the waves of resident CTAs of a kernel (occupancy queried once per kernel;
// thread-safe statics).
template <typename Kern>
static int x_per_sm(Kern kern, size_t smem) {
  int v = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, kXThreads, smem);
  return v > 0 ? v : 1;
}

static int x_splits(int64_t n, int per_sm) {
  const int64_t tiles = (n + kXThreads - 1) / kXThreads;
  const int64_t max_s = imin64(64, imax64(1, n / kXTile));
  return best_splits(tiles, (int64_t)device_sms() * per_sm, max_s);
}

static int exact_splits(int64_t n, int rule) {
  static const int p0 = x_per_sm(exact_j_kernel<GSDFT_EXACT_SCHUR20>,
                                 rule_smem<GSDFT_EXACT_SCHUR20>());
  static const int p1 = x_per_sm(exact_j_kernel<GSDFT_EXACT_FUSED32>,
                                 rule_smem<GSDFT_EXACT_FUSED32>());
  return x_splits(n, rule == GSDFT_EXACT_FUSED32 ? p1 : p0);
}

static int exact_vjp_splits(int64_t n, int rule) {
  static const int p0 = x_per_sm(exact_vjp_kernel<GSDFT_EXACT_SCHUR20>,
                                 rule_smem<GSDFT_EXACT_SCHUR20>());
  static const int p1 = x_per_sm(exact_vjp_kernel<GSDFT_EXACT_FUSED32>,
                                 rule_smem<GSDFT_EXACT_FUSED32>());
  return x_splits(n, rule == GSDFT_EXACT_FUSED32 ? p1 : p0);
}

}  // namespace gsdft

using namespace gsdft;

extern "C" size_t gsdft_exact_j_workspace_size(int64_t n_rep) {
  const int64_t n = imax64(n_rep, 1);
  const int S = imax64(exact_splits(n, GSDFT_EXACT_SCHUR20), exact_splits(n, GSDFT_EXACT_FUSED32));
  Sizer z;
  z.take<double>((size_t)n * kXF);
  z.take<double>((size_t)S * n);
  z.take<double>((size_t)(n + 255) / 256);
  return z.off + 256;
}

extern "C" int gsdft_exact_j(const double* rec, int64_t n_rep, int rule, double* J, double* E,
                             void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_rep < (int64_t(1) << 31), "bad sizes");
  GSDFT_REQUIRE(rule == GSDFT_EXACT_SCHUR20 || rule == GSDFT_EXACT_FUSED32, "unknown rule");
  GSDFT_REQUIRE(E && ws, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(E, 0, sizeof(double), st));
    return GSDFT_OK;
  }
  GSDFT_REQUIRE(rec && J, "null pointer");
  const int64_t n = n_rep;
  const int S = exact_splits(n, rule);
  Carver c(ws, ws_bytes);
  double* xr = c.take<double>((size_t)n * kXF);
  double* part = c.take<double>((size_t)S * n);
  double* blk = c.take<double>((size_t)(n + 255) / 256);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "exact-J workspace too small");
  exact_prep_kernel<<<grid_1d(n, 256), 256, 0, st>>>(rec, n, xr);
  GSDFT_LAUNCHED("exact_prep");
  const int64_t per_split = (n + S - 1) / S;
  dim3 grid((unsigned)((n + kXThreads - 1) / kXThreads), (unsigned)S);
  if (rule == GSDFT_EXACT_FUSED32)
    exact_j_kernel<GSDFT_EXACT_FUSED32>
        <<<grid, kXThreads, rule_smem<GSDFT_EXACT_FUSED32>(), st>>>(xr, n, per_split, part);
  else
    exact_j_kernel<GSDFT_EXACT_SCHUR20>
        <<<grid, kXThreads, rule_smem<GSDFT_EXACT_SCHUR20>(), st>>>(xr, n, per_split, part);
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
  const int S = imax64(exact_vjp_splits(n, GSDFT_EXACT_SCHUR20),
                       exact_vjp_splits(n, GSDFT_EXACT_FUSED32));
  Sizer z;
  z.take<double>((size_t)n * kXF);
  z.take<double>((size_t)S * kXV * n);
  return z.off + 256;
}

extern "C" int gsdft_exact_j_vjp(const double* rec, int64_t n_rep, int rule, const double* g_E,
                                 double* xc, void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_rep < (int64_t(1) << 31), "bad sizes");
  GSDFT_REQUIRE(rule == GSDFT_EXACT_SCHUR20 || rule == GSDFT_EXACT_FUSED32, "unknown rule");
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && xc && ws, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = n_rep;
  const int S = exact_vjp_splits(n, rule);
  Carver c(ws, ws_bytes);
  double* xr = c.take<double>((size_t)n * kXF);
  double* part = c.take<double>((size_t)S * kXV * n);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "exact-J reverse workspace too small");
  exact_prep_kernel<<<grid_1d(n, 256), 256, 0, st>>>(rec, n, xr);
  GSDFT_LAUNCHED("exact_prep");
  const int64_t per_split = (n + S - 1) / S;
  dim3 grid((unsigned)((n + kXThreads - 1) / kXThreads), (unsigned)S);
  if (rule == GSDFT_EXACT_FUSED32)
    exact_vjp_kernel<GSDFT_EXACT_FUSED32>
        <<<grid, kXThreads, rule_smem<GSDFT_EXACT_FUSED32>(), st>>>(xr, n, per_split, part);
  else
    exact_vjp_kernel<GSDFT_EXACT_SCHUR20>
        <<<grid, kXThreads, rule_smem<GSDFT_EXACT_SCHUR20>(), st>>>(xr, n, per_split, part);
  GSDFT_LAUNCHED("exact_vjp");
  exact_vjp_fold_kernel<<<grid_1d(n, 128), 128, 0, st>>>(part, S, n, xr, rec, g_E, xc);
  GSDFT_LAUNCHED("exact_vjp_fold");
  return GSDFT_OK;
}
