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
