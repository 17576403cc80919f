// Screened density-fitted exchange (RI-K) over the significant pairs (gs_dft/coulomb/ri.py:497-544):
//   D[P,o,o'] = sum_{live (i,k)} (P|ik) C_io C_ko',   E_K = -tr((V + lam I)^-1 M),
//   M_PQ = sum_{o,o'} D[P,o,o'] D[Q,o,o'] = (D D^T)_PQ,  so  E_K = -|L^-1 D|_F^2  with V + lam I = L L^T.
// Layout (row-major): Bt[a][P] = (P|a) for the representatives a (thread per aux, coalesced
// stores), X[a][o n + o'] = C_io C_ko' (+ C_ko C_io' for a merged transposed twin, whose integral
// is the same), D = Bt^T X. The contractions are the library's own DMMA GEMMs (dense.cu): D split
// over the pairs (its n_aux x n_occ^2 tiles alone cannot fill the device), Z = L^-1 D and its
// reverse as products with the packed inverse factor read as a lower-triangular operand; the
// integral block and every reduction are this file's kernels, all in a fixed order (bitwise
// reproducible).
// Reverse: Ybar = dE/dD = -2 g L^-T L^-1 D; dE/dX = Bt Ybar; dE/d(P|a) = W[P][a] = (Ybar X^T)[P][a],
// which drives the same integral reverse pass as RI-J with a per-(P,a) weight
// (gsdft_j_vjp_weighted, W stored aux-major so that a warp's pairs read consecutive entries);
// dE/dC from dE/dX per splat over the plan's groupings.
#include "common.cuh"

extern "C" size_t gsdft_j_vjp_weighted_workspace_size(int64_t n_live, int64_t n_aux);
extern "C" int gsdft_j_vjp_weighted(const double* rec, int64_t n_live, const double* beta,
                                    const double* R, const double* KN, const double* Wt,
                                    int64_t ldw, int64_t n_aux, double* sums, void* ws,
                                    size_t ws_bytes, gsdft_stream_t stream);

namespace gsdft {

int gemm_dmma(bool ta, bool tb, bool tri_a, int64_t M, int64_t N, int64_t K, double alpha,
              const double* A, int64_t lda, const double* B, int64_t ldb, double beta, double* C,
              int64_t ldc, cudaStream_t st);
int gemm_dmma_splitk(bool ta, int64_t M, int64_t N, int64_t K, double alpha, const double* A,
                     int64_t lda, const double* B, int64_t ldb, double beta, double* C, int64_t ldc,
                     double* part, int S, cudaStream_t st);
int splitk_count(int64_t M, int64_t N, int64_t K);

constexpr int kKThreads = 128;  // aux per CTA in the integral block kernel
constexpr int kKTile = 32;      // pair records per CTA iteration
constexpr int kKBits = 6;       // 2^6-entry weighted exp2 table per node
constexpr size_t kKDynSmem = sizeof(double) * GSDFT_NQUAD * (1 << kKBits);
constexpr int kKRedBlocks = 256;  // fixed block count of the sum of squares

// Bt[a * n_aux + P] = (P|a) = KN_P (KN_a pref) sum_n w_n (G0 G1 G2)^-1/2 2^(t^2 sum_k m_k / G_k),
// the integrand of the RI-J kernels without q. One aux per thread; the CTA walks tiles of kKTile
// records (grid-stride over tiles), staged in shared memory.
__global__ void __launch_bounds__(kKThreads)
    k_block_kernel(const double* __restrict__ rec, int64_t n_rep, const double* __restrict__ beta,
                   const double* __restrict__ R, const double* __restrict__ KN, int64_t n_aux,
                   double* __restrict__ Bt) {
  __shared__ double tile[kKTile * GSDFT_REC_FIELDS];
  extern __shared__ __align__(16) double etab[];
  load_wexp2_tables<kKBits>(etab);
  const int64_t P = blockIdx.x * (int64_t)kKThreads + threadIdx.x;
  const bool has = P < n_aux;
  const double b = has ? beta[P] : 1.0;
  const double r0 = has ? R[3 * P] : 0.0, r1 = has ? R[3 * P + 1] : 0.0;
  const double r2 = has ? R[3 * P + 2] : 0.0;
  const double knP = has ? KN[P] : 0.0;
  const double cP = -kLog2e * b;
  const int64_t ntiles = (n_rep + kKTile - 1) / kKTile;
  for (int64_t t = blockIdx.y; t < ntiles; t += gridDim.y) {
    const int64_t a0 = t * kKTile;
    const int cnt = (int)imin64(kKTile, n_rep - a0);
    __syncthreads();  // the previous tile is consumed (and the table is loaded)
    for (int k = threadIdx.x; k < cnt * GSDFT_REC_FIELDS; k += kKThreads)
      tile[k] = rec[a0 * GSDFT_REC_FIELDS + k];
    __syncthreads();
    if (!has) continue;
    for (int k = 0; k < cnt; ++k) {
      const double* rr = tile + k * GSDFT_REC_FIELDS;
      const double d0 = r0 - rr[GSDFT_REC_P0], d1 = r1 - rr[GSDFT_REC_P1];
      const double d2 = r2 - rr[GSDFT_REC_P2];
      double m[3], g[3], h[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const double y = rr[GSDFT_REC_U00 + c] * d0 + rr[GSDFT_REC_U10 + c] * d1 +
                         rr[GSDFT_REC_U20 + c] * d2;
        const double L = rr[GSDFT_REC_L0 + c];
        m[c] = (cP * L) * (y * y);
        g[c] = L * b;
        h[c] = L + b;
      }
      double coul = 0.0;
#pragma unroll
      for (int n = 0; n < GSDFT_NQUAD; ++n) {
        const double t2 = kQuadT2[n];
        const double G0 = fma(t2, h[0], g[0]);
        const double G1 = fma(t2, h[1], g[1]);
        const double G2 = fma(t2, h[2], g[2]);
        const double p12 = G1 * G2;
        const double prod = G0 * p12;
        const double num = fma(m[0], p12, G0 * fma(m[1], G2, m[2] * G1));
        const double y = rsqrt_pos(prod);
        const double inv = y * y;
        coul = fma(y, wexp2<kKBits>(num * inv, t2, etab + (n << kKBits)), coul);
      }
      Bt[(a0 + k) * n_aux + P] = (knP * rr[GSDFT_REC_KN]) * coul;
    }
  }
}

// X[a][o n + q] = C_io C_kq + (merged twin ? C_ko C_iq : 0), (i, k) the representative's pair.
__global__ void k_xbuild_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                const int32_t* __restrict__ rep_pos,
                                const int32_t* __restrict__ rep_twin, int64_t n_rep,
                                const double* __restrict__ C, int64_t no, double* __restrict__ X) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t K2 = no * no;
  if (idx >= n_rep * K2) return;
  const int64_t a = idx / K2, r = idx - a * K2;
  const int64_t o = r / no, q = r - o * no;
  const int64_t e = rep_pos[a];
  const double* ci = C + (int64_t)pi[e] * no;
  const double* ck = C + (int64_t)pj[e] * no;
  double v = ci[o] * ck[q];
  if (rep_twin[a] >= 0) v = fma(ck[o], ci[q], v);
  X[idx] = v;
}

// Partial sums of squares over kKRedBlocks fixed contiguous ranges; then E = -g * total.
__global__ void __launch_bounds__(256)
    k_sumsq_kernel(const double* __restrict__ Z, int64_t n, double* __restrict__ part) {
  __shared__ double s[256];
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * per, hi = imin64(lo + per, n);
  double acc = 0.0;
  for (int64_t k = lo + threadIdx.x; k < hi; k += 256) acc = fma(Z[k], Z[k], acc);
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = s[0];
}

__global__ void __launch_bounds__(256)
    k_energy_kernel(const double* __restrict__ part, int nb, double* __restrict__ E) {
  __shared__ double s[256];
  double acc = 0.0;
  for (int b = threadIdx.x; b < nb; b += 256) acc += part[b];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *E = -s[0];
}

// Y *= -2 g (g a device scalar, NULL = 1): Ybar = dE/dD.
__global__ void k_scale_kernel(double* __restrict__ Y, int64_t n, const double* __restrict__ gE) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k < n) Y[k] *= -2.0 * (gE ? gE[0] : 1.0);
}

// rec_K = rec with q = 1 (Q = 1, QK = KN pref): the chain then maps the weighted reverse sums,
// which already carry the exchange weights, to splat cotangents.
__global__ void k_unit_q_kernel(const double* __restrict__ rec, int64_t n_rep,
                                double* __restrict__ out) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= n_rep * GSDFT_REC_FIELDS) return;
  const int64_t a = k / GSDFT_REC_FIELDS;
  const int f = (int)(k - a * GSDFT_REC_FIELDS);
  double v = rec[k];
  if (f == GSDFT_REC_Q) v = 1.0;
  if (f == GSDFT_REC_QK) v = rec[a * GSDFT_REC_FIELDS + GSDFT_REC_KN];
  out[k] = v;
}

// g_C[s][o] = sum over the by-pi segment of s of ((Xb + tw Xb^T) C_k)[o] + over the by-pj segment of
// ((Xb^T + tw Xb) C_i)[o], Xb the representative's dE/dX as an n x n matrix (fixed order).
__global__ void k_cgrad_kernel(const int32_t* __restrict__ order_i, const int64_t* __restrict__ seg_i,
                               const int32_t* __restrict__ partner_i,
                               const int32_t* __restrict__ order_j, const int64_t* __restrict__ seg_j,
                               const int32_t* __restrict__ partner_j,
                               const int32_t* __restrict__ rep_twin, const double* __restrict__ Xbar,
                               const double* __restrict__ C, int64_t no, double* __restrict__ gC) {
  const int64_t s = blockIdx.x;
  const int64_t K2 = no * no;
  for (int64_t o = threadIdx.x; o < no; o += blockDim.x) {
    double acc = 0.0;
    for (int64_t e = seg_i[s]; e < seg_i[s + 1]; ++e) {
      const int64_t r = order_i[e];
      const bool tw = rep_twin[r] >= 0;
      const double* Xb = Xbar + r * K2;
      const double* ck = C + (int64_t)partner_i[e] * no;
      for (int64_t q = 0; q < no; ++q) {
        const double x = tw ? Xb[o * no + q] + Xb[q * no + o] : Xb[o * no + q];
        acc = fma(x, ck[q], acc);
      }
    }
    for (int64_t e = seg_j[s]; e < seg_j[s + 1]; ++e) {
      const int64_t r = order_j[e];
      const bool tw = rep_twin[r] >= 0;
      const double* Xb = Xbar + r * K2;
      const double* ci = C + (int64_t)partner_j[e] * no;
      for (int64_t q = 0; q < no; ++q) {
        const double x = tw ? Xb[q * no + o] + Xb[o * no + q] : Xb[q * no + o];
        acc = fma(x, ci[q], acc);
      }
    }
    gC[s * no + o] = acc;
  }
}

struct KLayout {
  double *Bt, *X, *Xbar, *Y, *part, *split;
  int S;
  void* vjp_ws;
  size_t vjp_bytes;
  bool ok;
};

static KLayout k_layout(void* ws, size_t ws_bytes, int64_t n_rep, int64_t n_aux, int64_t no) {
  const int64_t K2 = no * no;
  Carver c(ws, ws_bytes);
  KLayout l;
  l.Bt = c.take<double>((size_t)imax64(n_rep, 1) * n_aux);
  l.X = c.take<double>((size_t)imax64(n_rep, 1) * K2);
  l.Xbar = c.take<double>((size_t)imax64(n_rep, 1) * K2);
  l.Y = c.take<double>((size_t)n_aux * K2);
  l.part = c.take<double>(kKRedBlocks);
  l.S = splitk_count(n_aux, K2, imax64(n_rep, 1));
  l.split = c.take<double>((size_t)l.S * n_aux * K2);
  l.vjp_bytes = gsdft_j_vjp_weighted_workspace_size(imax64(n_rep, 1), n_aux);
  l.vjp_ws = c.take<unsigned char>(l.vjp_bytes);
  l.ok = c.ok;
  return l;
}

static int k_block_and_x(const double* rec, const int32_t* pi, const int32_t* pj,
                         const int32_t* rep_pos, const int32_t* rep_twin, int64_t n_rep,
                         const double* beta, const double* R, const double* KN, int64_t n_aux,
                         const double* C, int64_t no, const KLayout& l, cudaStream_t st) {
  const int64_t ntiles = (n_rep + kKTile - 1) / kKTile;
  dim3 grid((unsigned)((n_aux + kKThreads - 1) / kKThreads), (unsigned)imin64(ntiles, 65535));
  k_block_kernel<<<grid, kKThreads, kKDynSmem, st>>>(rec, n_rep, beta, R, KN, n_aux, l.Bt);
  GSDFT_LAUNCHED("k_block");
  const int64_t nx = n_rep * no * no;
  k_xbuild_kernel<<<grid_1d(nx, 256), 256, 0, st>>>(pi, pj, rep_pos, rep_twin, n_rep, C, no, l.X);
  GSDFT_LAUNCHED("k_xbuild");
  return GSDFT_OK;
}

}  // namespace gsdft

using namespace gsdft;

extern "C" size_t gsdft_k_workspace_size(int64_t n_rep, int64_t n_aux, int64_t n_occ) {
  const int64_t K2 = n_occ * n_occ;
  Sizer z;
  z.take<double>((size_t)imax64(n_rep, 1) * n_aux);
  z.take<double>((size_t)imax64(n_rep, 1) * K2);
  z.take<double>((size_t)imax64(n_rep, 1) * K2);
  z.take<double>((size_t)n_aux * K2);
  z.take<double>(kKRedBlocks);
  z.take<double>((size_t)splitk_count(n_aux, K2, imax64(n_rep, 1)) * n_aux * K2);
  z.take<unsigned char>(gsdft_j_vjp_weighted_workspace_size(imax64(n_rep, 1), n_aux));
  return z.off + 256;
}

extern "C" int gsdft_k_forward(const double* rec, const int32_t* pi, const int32_t* pj,
                               const int32_t* rep_pos, const int32_t* rep_twin, int64_t n_rep,
                               const double* beta, const double* R, const double* KN,
                               int64_t n_aux, const double* Linv, const double* C_occ,
                               int64_t n_occ, double* Z, double* E, void* ws, size_t ws_bytes,
                               gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31) && n_occ > 0 &&
                    n_occ * n_occ < (int64_t(1) << 31) && n_rep < (int64_t(1) << 31),
                "bad sizes");
  GSDFT_REQUIRE(beta && R && KN && Linv && C_occ && Z && E && ws, "null pointer");
  GSDFT_REQUIRE(n_rep == 0 || (rec && pi && pj && rep_pos && rep_twin), "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  KLayout l = k_layout(ws, ws_bytes, n_rep, n_aux, n_occ);
  if (!l.ok) return fail(GSDFT_ERR_ARG, "exchange workspace too small");
  const int64_t K2 = n_occ * n_occ;
  int rc = GSDFT_OK;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(Z, 0, (size_t)n_aux * K2 * sizeof(double), st));
  } else {
    rc = k_block_and_x(rec, pi, pj, rep_pos, rep_twin, n_rep, beta, R, KN, n_aux, C_occ, n_occ, l,
                       st);
    if (rc) return rc;
    // D (n_aux x K2, in Y) = Bt^T X, split over the pairs
    rc = gemm_dmma_splitk(true, n_aux, K2, n_rep, 1.0, l.Bt, n_aux, l.X, K2, 0.0, l.Y, K2, l.split,
                          l.S, st);
    if (rc) return rc;
    // Z = L^-1 D: the packed inverse's lower triangle
    rc = gemm_dmma(false, false, true, n_aux, K2, n_aux, 1.0, Linv, n_aux, l.Y, K2, 0.0, Z, K2, st);
    if (rc) return rc;
  }
  k_sumsq_kernel<<<kKRedBlocks, 256, 0, st>>>(Z, n_aux * K2, l.part);
  GSDFT_LAUNCHED("k_sumsq");
  k_energy_kernel<<<1, 256, 0, st>>>(l.part, kKRedBlocks, E);
  GSDFT_LAUNCHED("k_energy");
  return GSDFT_OK;
}

extern "C" int gsdft_k_backward(const double* rec, const int32_t* pi, const int32_t* pj,
                                const int32_t* rep_pos, const int32_t* rep_twin, int64_t n_rep,
                                const double* beta, const double* R, const double* KN,
                                int64_t n_aux, const double* Linv, const double* C_occ,
                                int64_t n_occ, const double* Z, const double* g_E,
                                const int32_t* order_i, const int64_t* seg_i,
                                const int32_t* partner_i, const int32_t* order_j,
                                const int64_t* seg_j, const int32_t* partner_j, int64_t M,
                                double* sums, double* g_C, void* ws, size_t ws_bytes,
                                gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31) && n_occ > 0 && M > 0 &&
                    n_occ * n_occ < (int64_t(1) << 31) && n_rep < (int64_t(1) << 31),
                "bad sizes");
  GSDFT_REQUIRE(beta && R && KN && Linv && C_occ && Z && g_C && ws && seg_i && seg_j,
                "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(g_C, 0, (size_t)M * n_occ * sizeof(double), st));
    return GSDFT_OK;
  }
  GSDFT_REQUIRE(rec && pi && pj && rep_pos && rep_twin && sums && order_i && partner_i &&
                    order_j && partner_j,
                "null pointer");
  KLayout l = k_layout(ws, ws_bytes, n_rep, n_aux, n_occ);
  if (!l.ok) return fail(GSDFT_ERR_ARG, "exchange workspace too small");
  const int64_t K2 = n_occ * n_occ;
  // Bt and X from the forward (the same workspace, untouched in between)
  // Y = L^-T Z (the packed inverse's lower triangle, transposed), then Ybar = -2 g_E Y
  int rc = gemm_dmma(true, false, true, n_aux, K2, n_aux, 1.0, Linv, n_aux, Z, K2, 0.0, l.Y, K2, st);
  if (rc) return rc;
  k_scale_kernel<<<grid_1d(n_aux * K2, 256), 256, 0, st>>>(l.Y, n_aux * K2, g_E);
  GSDFT_LAUNCHED("k_scale");
  // Xbar (n_rep x K2) = Bt Ybar
  rc = gemm_dmma(false, false, false, n_rep, K2, n_aux, 1.0, l.Bt, n_aux, l.Y, K2, 0.0, l.Xbar, K2,
                 st);
  if (rc) return rc;
  // W (n_aux x n_rep) = Ybar X^T, into Bt's storage (Bt is no longer needed)
  double* Wt = l.Bt;
  rc = gemm_dmma(false, true, false, n_aux, n_rep, K2, 1.0, l.Y, K2, l.X, K2, 0.0, Wt, n_rep, st);
  if (rc) return rc;
  rc = gsdft_j_vjp_weighted(rec, n_rep, beta, R, KN, Wt, n_rep, n_aux, sums, l.vjp_ws,
                            l.vjp_bytes, stream);
  if (rc) return rc;
  k_cgrad_kernel<<<(unsigned)M, 128, 0, st>>>(order_i, seg_i, partner_i, order_j, seg_j, partner_j,
                                             rep_twin, l.Xbar, C_occ, n_occ, g_C);
  GSDFT_LAUNCHED("k_cgrad");
  return GSDFT_OK;
}

extern "C" int gsdft_k_unit_q(const double* rec, int64_t n_rep, double* rec_out,
                              gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0, "bad sizes");
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && rec_out, "null pointer");
  k_unit_q_kernel<<<grid_1d(n_rep * GSDFT_REC_FIELDS, 256), 256, 0, (cudaStream_t)stream>>>(
      rec, n_rep, rec_out);
  GSDFT_LAUNCHED("k_unit_q");
  return GSDFT_OK;
}
