/*
 * CPU oracle, C restatement of the O(N_aux x N_pairs) loops of the RI-J path — TEST
 * INFRASTRUCTURE ONLY (used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs;
 * never by the product). OpenMP over aux functions (forward) and pairs (reverse).
 *
 * Forward: gamma_P = sum_a KN_P KN_a pref q_a sum_t w_t (G0G1G2)^-1/2 exp(-t^2 num/(G0G1G2)), in the
 * reference's division-lean node form (gs_dft/coulomb/ri.py:167-185) with dp2 = (U^T (R_P - P_a))^2
 * (ri.py:145-147) and pref = 2 pi^3 / sqrt(pi) (ri.py:150). Per-pair inputs (eigenvalues lam,
 * eigenvectors U as columns, centre P, KN, q) come from the NumPy oracle (gsdft_oracle.py).
 *
 * Reverse: with c_P = dbar_P KN_P and per node f = w (G0G1G2)^-1/2 exp(-t^2 S),
 *   SJ     = sum_P c_P sum_t f
 *   SD_k   = sum_P c_P sum_t f (beta + t^2) / G_k
 *   SV_k   = sum_P c_P beta y_k sum_t f t^2 / G_k
 *   SZ_kl  = sum_P c_P beta^2 y_k y_l sum_t f t^4 / (G_k G_l)
 * from which the NumPy side forms J, the eigenframe cotangent of A_hat and that of P (see
 * gsdft_oracle.py::_pair_vjp_integral for the derivation).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>

void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

int orc_get_threads(void) { return omp_get_max_threads(); }

static double QT[20], QW[20];

void orc_set_nodes(const double* t, const double* w) {
  for (int n = 0; n < 20; ++n) {
    QT[n] = t[n];
    QW[n] = w[n];
  }
}

static const double PREF = 34.986836655249725; /* 2 pi^3 / sqrt(pi) */

/* pair records (n_pairs x 17): lam0..2, U00..U22 (row-major, columns = eigenvectors), P0..2, KN, q */
void orc_gamma(const double* pr, int64_t n_pairs, const double* beta, const double* R,
               const double* KNa, int64_t n_aux, double* gamma) {
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t P = 0; P < n_aux; ++P) {
    const double b = beta[P];
    double acc = 0.0;
    for (int64_t a = 0; a < n_pairs; ++a) {
      const double* r = pr + a * 17;
      const double d0 = R[3 * P] - r[12], d1 = R[3 * P + 1] - r[13], d2 = R[3 * P + 2] - r[14];
      double dp2[3];
      for (int c = 0; c < 3; ++c) {
        double y = r[3 + c] * d0 + r[6 + c] * d1 + r[9 + c] * d2;
        dp2[c] = y * y;
      }
      const double L0 = r[0], L1 = r[1], L2 = r[2];
      double coul = 0.0;
      for (int n = 0; n < 20; ++n) {
        const double t2 = QT[n] * QT[n];
        const double G0 = b * L0 + t2 * (b + L0);
        const double G1 = b * L1 + t2 * (b + L1);
        const double G2 = b * L2 + t2 * (b + L2);
        const double invp = 1.0 / (G0 * G1 * G2);
        const double num = b * (L0 * dp2[0] * G1 * G2 + L1 * dp2[1] * G0 * G2 + L2 * dp2[2] * G0 * G1);
        coul += QW[n] * sqrt(invp) * exp(-t2 * num * invp);
      }
      acc += r[15] * PREF * r[16] * coul;
    }
    gamma[P] = KNa[P] * acc;
  }
}

/* sums (n_pairs x 13): SJ, SD0..2, SV0..2, SZ00, SZ11, SZ22, SZ01, SZ02, SZ12 ; c_P = dbar_P KN_P */
void orc_vjp(const double* pr, int64_t n_pairs, const double* beta, const double* R,
             const double* cP, int64_t n_aux, double* sums) {
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t a = 0; a < n_pairs; ++a) {
    const double* r = pr + a * 17;
    double SJ = 0, SD[3] = {0, 0, 0}, SV[3] = {0, 0, 0}, SZ[6] = {0, 0, 0, 0, 0, 0};
    for (int64_t P = 0; P < n_aux; ++P) {
      const double b = beta[P];
      const double d0 = R[3 * P] - r[12], d1 = R[3 * P + 1] - r[13], d2 = R[3 * P + 2] - r[14];
      double y[3];
      for (int c = 0; c < 3; ++c) y[c] = r[3 + c] * d0 + r[6 + c] * d1 + r[9 + c] * d2;
      double cf = 0, B[3] = {0, 0, 0}, C[3] = {0, 0, 0}, Z[6] = {0, 0, 0, 0, 0, 0};
      for (int n = 0; n < 20; ++n) {
        const double t2 = QT[n] * QT[n];
        double G[3], iG[3];
        double S = 0.0;
        for (int c = 0; c < 3; ++c) {
          G[c] = b * r[c] + t2 * (b + r[c]);
          iG[c] = 1.0 / G[c];
          S += b * r[c] * y[c] * y[c] * iG[c];
        }
        const double f = QW[n] * sqrt(iG[0] * iG[1] * iG[2]) * exp(-t2 * S);
        cf += f;
        for (int c = 0; c < 3; ++c) {
          B[c] += f * iG[c];
          C[c] += f * t2 * iG[c];
        }
        const double f4 = f * t2 * t2;
        Z[0] += f4 * iG[0] * iG[0];
        Z[1] += f4 * iG[1] * iG[1];
        Z[2] += f4 * iG[2] * iG[2];
        Z[3] += f4 * iG[0] * iG[1];
        Z[4] += f4 * iG[0] * iG[2];
        Z[5] += f4 * iG[1] * iG[2];
      }
      const double c0 = cP[P];
      SJ += c0 * cf;
      for (int c = 0; c < 3; ++c) {
        SD[c] += c0 * (b * B[c] + C[c]);
        SV[c] += c0 * b * y[c] * C[c];
      }
      const double cb2 = c0 * b * b;
      SZ[0] += cb2 * y[0] * y[0] * Z[0];
      SZ[1] += cb2 * y[1] * y[1] * Z[1];
      SZ[2] += cb2 * y[2] * y[2] * Z[2];
      SZ[3] += cb2 * y[0] * y[1] * Z[3];
      SZ[4] += cb2 * y[0] * y[2] * Z[4];
      SZ[5] += cb2 * y[1] * y[2] * Z[5];
    }
    double* o = sums + a * 13;
    o[0] = SJ;
    for (int c = 0; c < 3; ++c) {
      o[1 + c] = SD[c];
      o[4 + c] = SV[c];
    }
    for (int c = 0; c < 6; ++c) o[7 + c] = SZ[c];
  }
}

/* ---- significant-pair list (gs_dft/screening/pairs.py:50-118, 225-315, 342-345) ---------------------
 * The same screening as gsdft_oracle.py::_significant_flat, in C for the large configurations: |S| of
 * the (min, max) orientation, S = N_i N_j exp(-d.A_i A_hat^-1 A_j d) pi^1.5 / sqrt(det A_hat), with
 * the 3x3 algebra of gs_dft/integrals/linalg3.py:17-51 in the oracle's operation order (built with
 * FMA contraction off, so each operation rounds once as NumPy's does). A9 (M,9) row-major, mu (M,3),
 * N (M) come from the NumPy oracle's chart. Rows are independent (OpenMP over i). */
static double det3c(const double* A) {
  return A[0] * (A[4] * A[8] - A[5] * A[7]) - A[1] * (A[3] * A[8] - A[5] * A[6]) +
         A[2] * (A[3] * A[7] - A[4] * A[6]);
}

static void solve3c(const double* A, const double* b, double* x) {
  double c[9];
  c[0] = A[4] * A[8] - A[5] * A[7];
  c[1] = A[2] * A[7] - A[1] * A[8];
  c[2] = A[1] * A[5] - A[2] * A[4];
  c[3] = A[5] * A[6] - A[3] * A[8];
  c[4] = A[0] * A[8] - A[2] * A[6];
  c[5] = A[2] * A[3] - A[0] * A[5];
  c[6] = A[3] * A[7] - A[4] * A[6];
  c[7] = A[1] * A[6] - A[0] * A[7];
  c[8] = A[0] * A[4] - A[1] * A[3];
  const double det = det3c(A);
  for (int k = 0; k < 3; ++k) x[k] = (c[3 * k] * b[0] + c[3 * k + 1] * b[1] + c[3 * k + 2] * b[2]) / det;
}

static double abs_overlap(const double* A9, const double* mu, const double* N, int64_t i, int64_t j,
                          double pi15) {
  const int64_t lo = i < j ? i : j, hi = i < j ? j : i;
  const double *Ai = A9 + 9 * lo, *Aj = A9 + 9 * hi, *mi = mu + 3 * lo, *mj = mu + 3 * hi;
  double Ah[9], d[3], Ajd[3], s[3], x[3];
  for (int k = 0; k < 9; ++k) Ah[k] = Ai[k] + Aj[k];
  for (int k = 0; k < 3; ++k) d[k] = mi[k] - mj[k];
  for (int k = 0; k < 3; ++k) Ajd[k] = Aj[3 * k] * d[0] + Aj[3 * k + 1] * d[1] + Aj[3 * k + 2] * d[2];
  solve3c(Ah, Ajd, s);
  for (int k = 0; k < 3; ++k) x[k] = Ai[3 * k] * s[0] + Ai[3 * k + 1] * s[1] + Ai[3 * k + 2] * s[2];
  const double quad = d[0] * x[0] + d[1] * x[1] + d[2] * x[2];
  const double NK = N[lo] * N[hi] * exp(-quad);
  return fabs(NK * pi15 / sqrt(det3c(Ah)));
}

/* counts[i] = number of j (j >= i when unique) with |S_ij| > eps; near[i] = number of those within
 * relative `band` of eps either side (the guard band: decisions a last-bit change could flip). */
void orc_pairs_count(const double* A9, const double* mu, const double* N, int64_t M, double eps,
                     int unique, double pi15, double band, int64_t* counts, int64_t* near) {
#pragma omp parallel for schedule(dynamic, 8)
  for (int64_t i = 0; i < M; ++i) {
    int64_t c = 0, nb = 0;
    for (int64_t j = unique ? i : 0; j < M; ++j) {
      const double s = abs_overlap(A9, mu, N, i, j, pi15);
      c += s > eps;
      nb += fabs(s / eps - 1.0) < band;
    }
    counts[i] = c;
    near[i] = nb;
  }
}

/* The lexsorted significant list: row i's entries start at offsets[i] (exclusive prefix of counts). */
void orc_pairs_fill(const double* A9, const double* mu, const double* N, int64_t M, double eps,
                    int unique, double pi15, const int64_t* offsets, int32_t* pi, int32_t* pj,
                    double* absS) {
#pragma omp parallel for schedule(dynamic, 8)
  for (int64_t i = 0; i < M; ++i) {
    int64_t o = offsets[i];
    for (int64_t j = unique ? i : 0; j < M; ++j) {
      const double s = abs_overlap(A9, mu, N, i, j, pi15);
      if (s > eps) {
        pi[o] = (int32_t)i;
        pj[o] = (int32_t)j;
        absS[o] = s;
        ++o;
      }
    }
  }
}

/* ---- aux metric (gs_dft/coulomb/ri.py:63-76, 267-275) -----------------------------------------------
 * V_PQ = KN_P KN_Q 2 pi^2.5 / (b_P b_Q sqrt(b_P + b_Q)) F0(b_P b_Q / (b_P + b_Q) |R_P - R_Q|^2),
 * F0(T) = 1/2 sqrt(pi/T) erf(sqrt T) (Taylor below 1e-8), as gsdft_oracle.py::coulomb_block; C libm's
 * erf, so entries may differ from the NumPy oracle's in the last bits. For the CPU baseline's refresh
 * at sizes where the NumPy temporaries (n^2 x 3 doubles) are too large. */
static double boys0c(double T) {
  if (T < 1e-8) return 1.0 - T / 3.0 + T * T / 10.0 - T * T * T / 42.0;
  return 0.5 * sqrt(3.141592653589793 / T) * erf(sqrt(T));
}

void orc_metric(const double* beta, const double* R, const double* KN, int64_t n, double* V) {
  const double c = 2.0 * pow(3.141592653589793, 2.5);
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t p = 0; p < n; ++p) {
    for (int64_t q = 0; q < n; ++q) {
      const double g1 = beta[p], g2 = beta[q];
      const double gab = g1 * g2, gsum = g1 + g2;
      const double dx = R[3 * p] - R[3 * q], dy = R[3 * p + 1] - R[3 * q + 1],
                   dz = R[3 * p + 2] - R[3 * q + 2];
      const double T = gab / gsum * (dx * dx + dy * dy + dz * dz);
      V[p * n + q] = (KN[p] * KN[q]) * (c / (gab * sqrt(gsum)) * boys0c(T));
    }
  }
}
