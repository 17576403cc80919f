// Product auxiliary basis, its Coulomb metric, the metric's Cholesky factor and the per-step solve.
// Reference: gs_dft/basis/isotropic.py:22-39,81-116 (aux); gs_dft/coulomb/ri.py:63-123,267-275
// (metric), :243-264 (factor), :472-482 (solve). The factorisations themselves (Cholesky, the
// factor's inverse, blocked substitution) are the DMMA routines of dense.cu.
#include "common.cuh"

namespace gsdft {

struct Scales {
  double v[64];
};

__global__ void product_aux_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                   const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                   const double* __restrict__ w, int64_t n, Scales scales,
                                   int n_scales, double* __restrict__ log_alpha,
                                   double* __restrict__ R) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n) return;
  int i = pi ? pi[a] : (int)a;
  int j = pj ? pj[a] : (int)a;
  double Ai[9], Aj[9], mui[3], muj[3];
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    Ai[k] = A9[9 * (int64_t)i + k];
    Aj[k] = A9[9 * (int64_t)j + k];
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    mui[k] = mu[3 * (int64_t)i + k];
    muj[k] = mu[3 * (int64_t)j + k];
  }
  double Ah[9], P[3], KN, det;
  pair_quantities_rn(Ai, Aj, mui, muj, 1.0, 1.0, Ah, P, &KN, &det);
  double alpha0 = pow(det, 1.0 / 3.0);
  if (w && w[a] == 0.0) alpha0 = 1.0;
  for (int s = 0; s < n_scales; ++s) {
    int64_t o = (int64_t)s * n + a;
    log_alpha[o] = log(alpha0 * scales.v[s]);
    R[3 * o + 0] = P[0];
    R[3 * o + 1] = P[1];
    R[3 * o + 2] = P[2];
  }
}

__global__ void aux_quantities_kernel(const double* __restrict__ log_alpha, int64_t n,
                                      double* __restrict__ beta, double* __restrict__ KN) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n) return;
  double b = exp(log_alpha[a]);
  beta[a] = b;
  KN[a] = pow(2.0 * b / kPi, 0.75);
}

// F0(T) = 1/2 sqrt(pi/T) erf(sqrt T), Taylor series below 1e-8.
__device__ __forceinline__ double boys0(double T) {
  if (T < 1e-8) return 1.0 - T / 3.0 + T * T / 10.0 - T * T * T / 42.0;
  return 0.5 * sqrt(kPi / T) * erf(sqrt(T));
}

// One metric entry in the canonical orientation (lo, hi) so V is exactly symmetric.
// omega > 0: the long-range erf(omega r)/r kernel, F0(T) -> sqrt(z) F0(z T), z = omega^2 /
// (omega^2 + rho) (gs_dft/coulomb/ri.py:63-76).
__global__ void aux_metric_kernel(const double* __restrict__ beta, const double* __restrict__ R,
                                  const double* __restrict__ KN, int64_t n, double omega,
                                  double* __restrict__ V) {
  int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (q >= n) return;
  for (int64_t p = blockIdx.y; p < n; p += gridDim.y) {
    int64_t lo = p < q ? p : q, hi = p < q ? q : p;
    double g1 = beta[lo], g2 = beta[hi];
    double gab = g1 * g2;
    double gsum = g1 + g2;
    double dx = R[3 * lo] - R[3 * hi], dy = R[3 * lo + 1] - R[3 * hi + 1];
    double dz = R[3 * lo + 2] - R[3 * hi + 2];
    double PQ2 = dx * dx + dy * dy + dz * dz;
    double rho = gab / gsum;
    double T = rho * PQ2;
    double F0;
    if (omega > 0.0) {
      const double z = (omega * omega) / (omega * omega + rho);
      F0 = sqrt(z) * boys0(z * T);
    } else {
      F0 = boys0(T);
    }
    double coul = 34.986836655249725 / (gab * sqrt(gsum)) * F0;   // 2 pi^2.5
    V[p * n + q] = (KN[lo] * KN[hi]) * coul;
  }
}

// E = 1/2 gamma . d, one block, fixed-order tree: deterministic.
__global__ void half_dot_kernel(const double* __restrict__ g, const double* __restrict__ d,
                                int64_t n, double* E) {
  __shared__ double s[1024];
  double acc = 0.0;
  for (int64_t k = threadIdx.x; k < n; k += blockDim.x) acc = fma(g[k], d[k], acc);
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] += s[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *E = 0.5 * s[0];
}

// One-CTA blocked triangular solves for the per-step tail, N_aux <= kSmallSolveMax:
// L y = gamma (forward), L^T d = y (backward), E = 1/2 gamma.d. Blocks of 32 rows: the panel of
// rows below/right of the solved part is applied with coalesced reads of row-major L (a warp per row
// for the forward sweep, warps over rows and lanes over the block's columns for the backward
// sweep), then the 32x32 diagonal triangle is solved inside one warp. The solution lives in shared
// memory; every reduction has a fixed order.
// --- per-step solve through the inverse factor ----------------------------------------------------
// With X = L^-1 (computed once per refresh), d = X^T (X gamma) and E = 1/2 |X gamma|^2 =
// 1/2 gamma.(L L^T)^-1 gamma are two triangular mat-vecs: every row is independent, so they spread
// over the SMs instead of walking a dependent chain of substitution steps, and the two of them
// stream the factor's n^2 doubles once. Both read ONE packed n x n matrix: its lower triangle (with
// the diagonal) is L^-1 and its strict upper triangle is L^-T's, i.e. the mirror of the strict lower
// one, so row i holds L^-1's row i in [0, i] and L^-T's row i in [i, n) (the diagonal is shared).
// One warp per row; each lane keeps four partial sums; the warp's shuffle tree fixes the summation
// order (bitwise reproducible).
constexpr int kTriWarps = 4;

// In place, X[c][r] = X[r][c] for r > c: the strict lower triangle mirrored into the strict upper
// one, through 32 x 33 shared tiles (coalesced both ways). A block reads one lower (or diagonal)
// tile and writes its mirror tile, which no other block reads; a diagonal tile is read whole before
// its upper half is written.
__global__ void mirror_lower_kernel(double* X, int64_t n) {
  __shared__ double t[32][33];
  if (blockIdx.x > blockIdx.y) return;  // strictly upper tiles are written by their mirror's block
  const int64_t r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < n && c < n) t[k][threadIdx.x] = X[r * n + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = c0 + k, c = r0 + threadIdx.x;  // destination (r, c) = mirror of (c, r)
    if (r < n && c < n && r < c) X[r * n + c] = t[threadIdx.x][k];
  }
}

// y[i] = sum_{j in row i's triangle} A[i][j] x[j]: columns [0, i] (kLower) or [i, n) (upper);
// kMode 1 gives y = b - (that), kMode 2 y = b + (that). With E != nullptr, block 0 also writes
// E = 1/2 x.x.
template <bool kLower, int kMode>
__global__ void __launch_bounds__(kTriWarps * 32)
    tri_rows_kernel(const double* __restrict__ A, const double* __restrict__ x, int64_t n,
                    double* __restrict__ y, double* __restrict__ E, const double* __restrict__ b) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = blockIdx.x * (int64_t)kTriWarps + warp;
  if (i < n) {
    const double* row = A + i * n;
    const int64_t lo = kLower ? 0 : i, hi = kLower ? i + 1 : n;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    int64_t j = lo + lane;
    for (; j + 96 < hi; j += 128) {
      a0 = fma(row[j], x[j], a0);
      a1 = fma(row[j + 32], x[j + 32], a1);
      a2 = fma(row[j + 64], x[j + 64], a2);
      a3 = fma(row[j + 96], x[j + 96], a3);
    }
    for (; j < hi; j += 32) a0 = fma(row[j], x[j], a0);
    double v = (a0 + a1) + (a2 + a3);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) y[i] = kMode == 1 ? b[i] - v : (kMode == 2 ? b[i] + v : v);
  }
  if (E != nullptr && blockIdx.x == 0) {
    __shared__ double part[kTriWarps];
    double a0 = 0.0, a1 = 0.0;
    int64_t k = threadIdx.x;
    for (; k + kTriWarps * 32 < n; k += 2 * kTriWarps * 32) {
      a0 = fma(x[k], x[k], a0);
      a1 = fma(x[k + kTriWarps * 32], x[k + kTriWarps * 32], a1);
    }
    if (k < n) a0 = fma(x[k], x[k], a0);
    double v = a0 + a1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) part[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kTriWarps; ++w) sum += part[w];
      *E = 0.5 * sum;
    }
  }
}

// part[s][i] = sum_{j in chunk s, j >= i} L[j][i] x[j]: the transposed lower-triangular product
// L^T x read down columns, one column per thread (a warp's loads are consecutive in a row), the
// rows cut into gridDim.y chunks for parallelism.
constexpr int kLtCols = 128;
constexpr int kLtChunks = 16;
__global__ void __launch_bounds__(kLtCols)
    trmv_lt_part_kernel(const double* __restrict__ L, const double* __restrict__ x, int64_t n,
                        double* __restrict__ part) {
  const int64_t i = blockIdx.x * (int64_t)kLtCols + threadIdx.x;
  const int64_t chunk = (n + gridDim.y - 1) / gridDim.y;
  const int64_t c0 = blockIdx.x * (int64_t)kLtCols;
  const int64_t j0 = imax64(blockIdx.y * chunk, c0), j1 = imin64((blockIdx.y + 1) * chunk, n);
  double a0 = 0.0, a1 = 0.0;
  int64_t j = j0;
  if (i < n) {
    for (; j + 1 < j1; j += 2) {
      if (j >= i) a0 = fma(L[j * n + i], x[j], a0);
      if (j + 1 >= i) a1 = fma(L[(j + 1) * n + i], x[j + 1], a1);
    }
    if (j < j1 && j >= i) a0 = fma(L[j * n + i], x[j], a0);
    part[blockIdx.y * n + i] = a0 + a1;
  }
}

// t[i] = sum_s part[s][i] in split order.
__global__ void sum_parts_kernel(const double* __restrict__ part, int S, int64_t n,
                                 double* __restrict__ t) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  double acc = 0.0;
  for (int s = 0; s < S; ++s) acc += part[(int64_t)s * n + i];
  t[i] = acc;
}

int potrf_dmma(double* V, int64_t n, double lam, double* Dinv, int* info_dev, cudaStream_t st);
int trtri_dmma(const double* L, int64_t n, double* X, cudaStream_t st);
int trsv_llt(const double* L, int64_t n, double* d, cudaStream_t st);

}  // namespace gsdft

using namespace gsdft;

extern "C" int gsdft_product_aux(const double* A9, const double* mu, const double* N, int64_t M,
                                 const int32_t* pi, const int32_t* pj, const double* w,
                                 int64_t n_pairs, const double* scales_host, int n_scales,
                                 double* log_alpha, double* R, gsdft_stream_t stream) {
  (void)N;
  GSDFT_REQUIRE(M > 0 && n_scales >= 1 && n_scales <= 64, "bad M or n_scales (1..64)");
  GSDFT_REQUIRE(A9 && mu && scales_host && log_alpha && R, "null pointer");
  GSDFT_REQUIRE((pi == nullptr) == (pj == nullptr), "pi and pj must both be given or both NULL");
  int64_t n = pi ? n_pairs : M;
  if (n == 0) return GSDFT_OK;
  Scales sc;
  for (int s = 0; s < n_scales; ++s) sc.v[s] = scales_host[s];
  product_aux_kernel<<<grid_1d(n, 128), 128, 0, (cudaStream_t)stream>>>(A9, mu, pi, pj, w, n, sc,
                                                                       n_scales, log_alpha, R);
  GSDFT_LAUNCHED("product_aux");
  return GSDFT_OK;
}

extern "C" int gsdft_aux_quantities(const double* log_alpha, int64_t n_aux, double* beta,
                                    double* KN, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux >= 0, "n_aux < 0");
  if (n_aux == 0) return GSDFT_OK;
  GSDFT_REQUIRE(log_alpha && beta && KN, "null pointer");
  aux_quantities_kernel<<<grid_1d(n_aux, 128), 128, 0, (cudaStream_t)stream>>>(log_alpha, n_aux,
                                                                              beta, KN);
  GSDFT_LAUNCHED("aux_quantities");
  return GSDFT_OK;
}

extern "C" int gsdft_aux_metric(const double* beta, const double* R, const double* KN,
                                int64_t n_aux, double* V, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux > 0 && n_aux < (int64_t(1) << 31), "n_aux out of range");
  GSDFT_REQUIRE(beta && R && KN && V, "null pointer");
  dim3 grid(grid_1d(n_aux, 128), (unsigned)imin64(n_aux, 65535));
  aux_metric_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(beta, R, KN, n_aux, 0.0, V);
  GSDFT_LAUNCHED("aux_metric");
  return GSDFT_OK;
}

extern "C" int gsdft_aux_metric_lr(const double* beta, const double* R, const double* KN,
                                   int64_t n_aux, double omega, double* V, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux > 0 && n_aux < (int64_t(1) << 31), "n_aux out of range");
  GSDFT_REQUIRE(omega > 0.0, "omega must be positive");
  GSDFT_REQUIRE(beta && R && KN && V, "null pointer");
  dim3 grid(grid_1d(n_aux, 128), (unsigned)imin64(n_aux, 65535));
  aux_metric_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(beta, R, KN, n_aux, omega, V);
  GSDFT_LAUNCHED("aux_metric");
  return GSDFT_OK;
}

namespace gsdft {
// Gauss-Legendre on [0, upper] (nq <= GSDFT_NQUAD nodes, ascending) as a runtime node table:
// table[n] = t_n^2, table[GSDFT_NQUAD + n] = t_n^4, and from 2 GSDFT_NQUAD on, node n's row of 64
// weighted exp2 entries w_n 2^(j/64). The roots of P_nq by Newton's method from the standard
// cosine guesses (each thread one root, in FP64; the iteration stops at a relative step of 1e-16 or
// after 100 steps), the weights 2 / ((1 - x^2) P'_nq(x)^2), mapped t = upper (x + 1)/2,
// w = upper w_GL / 2 (gs_dft/integrals/dense.py:56-76).
__device__ void legendre_eval(int nq, double x, double* p, double* dp) {
  double p0 = 1.0, p1 = x;
  for (int k = 1; k < nq; ++k) {
    const double p2 = ((2.0 * k + 1.0) * x * p1 - k * p0) / (k + 1.0);
    p0 = p1;
    p1 = p2;
  }
  *p = p1;
  *dp = nq * (x * p1 - p0) / (x * x - 1.0);
}

__global__ void lr_node_table_kernel(double upper, int nq, double* __restrict__ table) {
  __shared__ double w[GSDFT_NQUAD];
  const int n = threadIdx.x;
  if (n < nq) {
    const int i = nq - 1 - n;  // the guesses descend in x
    double x = cos(3.14159265358979323846 * (i + 0.75) / (nq + 0.5));
    double p, dp;
    for (int it = 0; it < 100; ++it) {
      legendre_eval(nq, x, &p, &dp);
      const double dx = p / dp;
      x -= dx;
      if (fabs(dx) <= 1e-16 * fmax(fabs(x), 1e-3)) break;
    }
    legendre_eval(nq, x, &p, &dp);
    const double t = 0.5 * upper * (x + 1.0);
    table[n] = t * t;
    table[GSDFT_NQUAD + n] = (t * t) * (t * t);
    w[n] = 0.5 * upper * (2.0 / ((1.0 - x * x) * dp * dp));
  } else if (n < GSDFT_NQUAD) {
    table[n] = 0.0;
    table[GSDFT_NQUAD + n] = 0.0;
  }
  __syncthreads();
  for (int k = threadIdx.x; k < nq * 64; k += blockDim.x)
    table[2 * GSDFT_NQUAD + k] = w[k / 64] * exp2((k % 64) / 64.0);
}
}  // namespace gsdft

extern "C" int gsdft_lr_node_table(double upper, int n_nodes, double* table,
                                   gsdft_stream_t stream) {
  GSDFT_REQUIRE(upper > 0.0 && n_nodes >= 1 && n_nodes <= GSDFT_NQUAD, "bad node rule");
  GSDFT_REQUIRE(table, "null pointer");
  lr_node_table_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(upper, n_nodes, table);
  GSDFT_LAUNCHED("lr_node_table");
  return GSDFT_OK;
}

extern "C" size_t gsdft_aux_cholesky_workspace_size(int64_t n_aux) {
  (void)n_aux;
  Sizer z;
  z.take<double>(64 * 64);  // inverse of the current diagonal block
  z.take<int>(1);           // first non-positive pivot
  return z.off + 256;
}

extern "C" int gsdft_aux_cholesky(double* V, int64_t n_aux, double lam, void* ws, size_t ws_bytes,
                                  gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux > 0 && n_aux < (int64_t(1) << 31), "n_aux out of range");
  GSDFT_REQUIRE(V, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  Carver c(ws, ws_bytes);
  double* Dinv = c.take<double>(64 * 64);
  int* info = c.take<int>(1);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "cholesky workspace too small (%zu < %zu)", ws_bytes, c.off);
  int rc = potrf_dmma(V, n_aux, lam, Dinv, info, st);
  if (rc) return rc;
  int info_h = 0;
  GSDFT_CUDA(cudaMemcpyAsync(&info_h, info, sizeof(int), cudaMemcpyDeviceToHost, st));
  GSDFT_CUDA(cudaStreamSynchronize(st));
  if (info_h != 0)
    return fail(GSDFT_ERR_LINALG,
                "aux metric + lam I is not positive definite (pivot %d of %lld not positive)",
                info_h, (long long)n_aux);
  return GSDFT_OK;
}

extern "C" size_t gsdft_j_solve_workspace_size(int64_t n_aux) {
  (void)n_aux;
  return 0;
}

extern "C" int gsdft_j_solve(const double* L, const double* gamma, int64_t n_aux, double* d,
                             double* E, void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  (void)ws;
  (void)ws_bytes;
  GSDFT_REQUIRE(n_aux > 0 && n_aux < (int64_t(1) << 31), "n_aux out of range");
  GSDFT_REQUIRE(L && gamma && d && E, "null pointer");
  GSDFT_REQUIRE(d != gamma, "d must not alias gamma");
  cudaStream_t st = (cudaStream_t)stream;
  GSDFT_CUDA(cudaMemcpyAsync(d, gamma, n_aux * sizeof(double), cudaMemcpyDeviceToDevice, st));
  int rc = trsv_llt(L, n_aux, d, st);
  if (rc) return rc;
  half_dot_kernel<<<1, 1024, 0, st>>>(gamma, d, n_aux, E);
  GSDFT_LAUNCHED("half_dot");
  return GSDFT_OK;
}

extern "C" int gsdft_j_solve_inverse(const double* L, int64_t n_aux, double* Linv,
                                     gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux > 0 && n_aux <= GSDFT_SOLVE_INV_MAX, "n_aux out of range (1..%d)",
                GSDFT_SOLVE_INV_MAX);
  GSDFT_REQUIRE(L && Linv, "null pointer");
  GSDFT_REQUIRE(L != Linv, "Linv must not alias L");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = n_aux;
  // L^-1 in the lower triangle (DMMA recursive doubling), then its mirror into the strict upper one
  int rc = trtri_dmma(L, n, Linv, st);
  if (rc) return rc;
  const dim3 tg((unsigned)((n + 31) / 32), (unsigned)((n + 31) / 32));
  mirror_lower_kernel<<<tg, dim3(32, 8), 0, st>>>(Linv, n);
  GSDFT_LAUNCHED("mirror_lower");
  return GSDFT_OK;
}

extern "C" size_t gsdft_j_solve_inv_workspace_size(int64_t n_aux) {
  Sizer z;
  z.take<double>((size_t)imax64(n_aux, 1));                 // y
  z.take<double>((size_t)imax64(n_aux, 1));                 // t = L^T d
  z.take<double>((size_t)imax64(n_aux, 1));                 // residual
  z.take<double>((size_t)kLtChunks * imax64(n_aux, 1));     // partial sums of L^T d
  return z.off;
}

extern "C" int gsdft_j_solve_inv(const double* Linv, const double* L, const double* gamma,
                                 int64_t n_aux, double* d, double* E, void* ws, size_t ws_bytes,
                                 gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_aux > 0 && n_aux <= GSDFT_SOLVE_INV_MAX, "n_aux out of range");
  GSDFT_REQUIRE(Linv && gamma && d && E && ws, "null pointer");
  GSDFT_REQUIRE(ws_bytes >= gsdft_j_solve_inv_workspace_size(n_aux), "workspace too small");
  GSDFT_REQUIRE(d != gamma, "d must not alias gamma");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = n_aux;
  Carver c(ws, ws_bytes);
  double* y = c.take<double>((size_t)imax64(n, 1));
  double* t = c.take<double>((size_t)imax64(n, 1));
  double* r = c.take<double>((size_t)imax64(n, 1));
  double* part = c.take<double>((size_t)kLtChunks * imax64(n, 1));
  const unsigned grid = (unsigned)((n + kTriWarps - 1) / kTriWarps);
  // d = L^-T (L^-1 gamma)
  tri_rows_kernel<true, 0><<<grid, kTriWarps * 32, 0, st>>>(Linv, gamma, n, y, nullptr, nullptr);
  GSDFT_LAUNCHED("tri_rows");
  tri_rows_kernel<false, 0><<<grid, kTriWarps * 32, 0, st>>>(Linv, y, n, d, L ? nullptr : E,
                                                             nullptr);
  GSDFT_LAUNCHED("tri_rows");
  if (L == nullptr) return GSDFT_OK;  // E = 1/2 |L^-1 gamma|^2 written above
  // one step of refinement with the factor: r = gamma - L (L^T d), d += L^-T L^-1 r
  dim3 lt((unsigned)((n + kLtCols - 1) / kLtCols), kLtChunks);
  trmv_lt_part_kernel<<<lt, kLtCols, 0, st>>>(L, d, n, part);
  GSDFT_LAUNCHED("trmv_lt");
  sum_parts_kernel<<<grid_1d(n, 256), 256, 0, st>>>(part, kLtChunks, n, t);
  GSDFT_LAUNCHED("sum_parts");
  tri_rows_kernel<true, 1><<<grid, kTriWarps * 32, 0, st>>>(L, t, n, r, nullptr, gamma);
  GSDFT_LAUNCHED("tri_rows");
  tri_rows_kernel<true, 0><<<grid, kTriWarps * 32, 0, st>>>(Linv, r, n, y, nullptr, nullptr);
  GSDFT_LAUNCHED("tri_rows");
  tri_rows_kernel<false, 2><<<grid, kTriWarps * 32, 0, st>>>(Linv, y, n, d, nullptr, d);
  GSDFT_LAUNCHED("tri_rows");
  half_dot_kernel<<<1, 1024, 0, st>>>(gamma, d, n, E);
  GSDFT_LAUNCHED("half_dot");
  return GSDFT_OK;
}
