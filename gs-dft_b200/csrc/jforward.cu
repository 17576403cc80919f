// Per-step pair preparation and the fused forward fit-vector contraction
//   gamma_P = sum_a (P|a) q_a,   (P|a) = KN_P KN_a pref sum_t w_t (G0 G1 G2)^(-1/2) exp(-t^2 S),
// the 3-centre integral never stored. Reference: gs_dft/coulomb/ri.py:126-185 (block + nodes),
// :436-469 (gamma stream), gs_dft/coulomb/stream.py:203-215 (pair quantities), ri.py:456 (q).
#include <mutex>

#include "common.cuh"

namespace gsdft {

// ------------------------------------------------------------------------------------------------
// Pair prep: geometry + symmetric eigen-decomposition of A_hat (cyclic Jacobi).
// ------------------------------------------------------------------------------------------------

// Cyclic Jacobi on a symmetric 3x3 (Golub & Van Loan, symmetric Schur decomposition). a is
// overwritten; lam gets the eigenvalues ascending and V (row-major) the matching eigenvectors as
// columns.
__device__ void jacobi_eig3(double a[3][3], double lam[3], double V[9]) {
  double v[3][3] = {{1, 0, 0}, {0, 1, 0}, {0, 0, 1}};
  for (int sweep = 0; sweep < 12; ++sweep) {
    double off = a[0][1] * a[0][1] + a[0][2] * a[0][2] + a[1][2] * a[1][2];
    double dia = a[0][0] * a[0][0] + a[1][1] * a[1][1] + a[2][2] * a[2][2];
    if (off <= 1e-36 * dia) break;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int p = r == 2 ? 1 : 0;
      const int q = r == 0 ? 1 : 2;
      double apq = a[p][q];
      if (apq == 0.0) continue;
      double theta = (a[q][q] - a[p][p]) / (2.0 * apq);
      double t = (theta >= 0.0 ? 1.0 : -1.0) / (fabs(theta) + sqrt(theta * theta + 1.0));
      double c = 1.0 / sqrt(t * t + 1.0);
      double s = t * c;
      a[p][p] -= t * apq;
      a[q][q] += t * apq;
      a[p][q] = a[q][p] = 0.0;
      const int o = 3 - p - q;
      double aop = a[o][p], aoq = a[o][q];
      a[o][p] = a[p][o] = c * aop - s * aoq;
      a[o][q] = a[q][o] = s * aop + c * aoq;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        double vkp = v[k][p], vkq = v[k][q];
        v[k][p] = c * vkp - s * vkq;
        v[k][q] = s * vkp + c * vkq;
      }
    }
  }
  int idx[3] = {0, 1, 2};
  double d[3] = {a[0][0], a[1][1], a[2][2]};
  if (d[idx[1]] < d[idx[0]]) { int t = idx[0]; idx[0] = idx[1]; idx[1] = t; }
  if (d[idx[2]] < d[idx[1]]) { int t = idx[1]; idx[1] = idx[2]; idx[2] = t; }
  if (d[idx[1]] < d[idx[0]]) { int t = idx[0]; idx[0] = idx[1]; idx[1] = t; }
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    lam[c] = d[idx[c]];
#pragma unroll
    for (int r = 0; r < 3; ++r) V[3 * r + c] = v[r][idx[c]];
  }
}

__global__ void pair_prep_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                 const double* __restrict__ N, const int32_t* __restrict__ pi,
                                 const int32_t* __restrict__ pj,
                                 const int32_t* __restrict__ live_idx, int64_t n_live,
                                 double* __restrict__ rec) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_live) return;
  int64_t e = live_idx[a];
  int i = pi[e], j = pj[e];
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
  pair_quantities_rn(Ai, Aj, mui, muj, N[i], N[j], Ah, P, &KN, &det);
  double s[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) s[r][c] = 0.5 * (Ah[3 * r + c] + Ah[3 * c + r]);
  double lam[3], U[9];
  jacobi_eig3(s, lam, U);
  double* o = rec + a * GSDFT_REC_FIELDS;
  o[GSDFT_REC_L0] = lam[0];
  o[GSDFT_REC_L1] = lam[1];
  o[GSDFT_REC_L2] = lam[2];
#pragma unroll
  for (int k = 0; k < 9; ++k) o[GSDFT_REC_U00 + k] = U[k];
  o[GSDFT_REC_P0] = P[0];
  o[GSDFT_REC_P1] = P[1];
  o[GSDFT_REC_P2] = P[2];
  o[GSDFT_REC_KN] = KN * kPref;
}

// q_a = w_a sum_o occ_o C_io C_jo, w_a the representative's (summed) weight; one warp per pair
// (lanes stride o; fixed-order reduce).
__global__ void pair_density_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                    const double* __restrict__ rep_w,
                                    const int32_t* __restrict__ live_idx, int64_t n_live,
                                    const double* __restrict__ C, const double* __restrict__ occ,
                                    int64_t n_occ, double* __restrict__ rec) {
  int64_t a = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (a >= n_live) return;
  int64_t e = live_idx[a];
  const double* ci = C + (int64_t)pi[e] * n_occ;
  const double* cj = C + (int64_t)pj[e] * n_occ;
  double acc = 0.0;
  for (int64_t o = lane; o < n_occ; o += 32) acc = fma(occ[o] * ci[o], cj[o], acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    double q = rep_w[a] * acc;
    double* r = rec + a * GSDFT_REC_FIELDS;
    r[GSDFT_REC_Q] = q;
    r[GSDFT_REC_QK] = q * r[GSDFT_REC_KN];
  }
}

// The same for few orbitals (n_occ <= 32): one thread per pair, orbitals in order.
__global__ void pair_density_thread_kernel(const int32_t* __restrict__ pi,
                                           const int32_t* __restrict__ pj,
                                           const double* __restrict__ rep_w,
                                           const int32_t* __restrict__ live_idx, int64_t n_live,
                                           const double* __restrict__ C,
                                           const double* __restrict__ occ, int64_t n_occ,
                                           double* __restrict__ rec) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_live) return;
  int64_t e = live_idx[a];
  const double* ci = C + (int64_t)pi[e] * n_occ;
  const double* cj = C + (int64_t)pj[e] * n_occ;
  double acc = 0.0;
  for (int64_t o = 0; o < n_occ; ++o) acc = fma(occ[o] * ci[o], cj[o], acc);
  double q = rep_w[a] * acc;
  double* r = rec + a * GSDFT_REC_FIELDS;
  r[GSDFT_REC_Q] = q;
  r[GSDFT_REC_QK] = q * r[GSDFT_REC_KN];
}

// ------------------------------------------------------------------------------------------------
// Forward: a block holds kFwAux aux functions resident in shared memory for its whole run and
// streams its slice of the pair representatives past them in chunks of 128, one representative
// per thread (eigenframe, centre and q KN in registers), two aux at a time per thread. The 32
// lanes of a warp are 32 consecutive representatives (mostly one row of the lexsorted list, so
// neighbouring pairs), which keeps node screening's per-warp node count close to the per-pair one.
// gamma_P is reduced over the warp's lanes by a fixed shuffle tree and accumulated per warp in
// shared memory; the warps' partial sums are added in warp order at the end. The loop has no
// block-wide barrier and no asynchronous copy: warps needing different numbers of nodes never wait
// for each other.
// ------------------------------------------------------------------------------------------------
constexpr int kFwThreads = 128;  // representatives per chunk (one per thread)
constexpr int kFwWarps = kFwThreads / 32;
#ifndef GSDFT_FW_AUX
#define GSDFT_FW_AUX 256
#endif
constexpr int kFwAux = GSDFT_FW_AUX;  // aux resident per block (at most)
#ifndef GSDFT_FW_EXP2_BITS
#define GSDFT_FW_EXP2_BITS 6
#endif
// Minimum resident CTAs per SM for the register budget (0: the compiler's choice).
#ifndef GSDFT_FW_MINB
#define GSDFT_FW_MINB 0
#endif
#if GSDFT_FW_MINB > 0
#define GSDFT_FW_BOUNDS __launch_bounds__(kFwThreads, GSDFT_FW_MINB)
#else
#define GSDFT_FW_BOUNDS __launch_bounds__(kFwThreads)
#endif
#ifndef GSDFT_FW_NA
#define GSDFT_FW_NA 2
#endif
constexpr int kFwNA = GSDFT_FW_NA;  // aux evaluated together per thread (independent chains)
constexpr int kFwBits = GSDFT_FW_EXP2_BITS;  // 2^kFwBits-entry weighted exp2 table per node
constexpr size_t kFwDynSmem = sizeof(double) * GSDFT_NQUAD * (1 << kFwBits);
static_assert(kFwAux % kFwNA == 0, "aux groups must tile the resident block");

// Node evaluations of the forward kernel since the last reset: (aux, pair) units times the nodes
// each evaluated (20 without screening). Read by gsdft_node_evals.
static __device__ unsigned long long g_fw_node_evals;

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__global__ void GSDFT_FW_BOUNDS
    j_forward_kernel(const double* __restrict__ rec, int64_t n_live,
                     const double* __restrict__ beta, const double* __restrict__ R,
                     const double* __restrict__ KN, int64_t n_aux, int64_t per_split,
                     int aux_per_block, double skip2, double* __restrict__ partial) {
  __shared__ double sb[kFwAux], scp[kFwAux], sr0[kFwAux], sr1[kFwAux], sr2[kFwAux];
  __shared__ double red[kFwWarps][kFwAux];
  extern __shared__ __align__(16) double etab[];  // GSDFT_NQUAD x 2^kFwBits weighted table
  load_wexp2_tables<kFwBits>(etab);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t P0 = blockIdx.x * (int64_t)aux_per_block;
  const int naux = (int)imin64(aux_per_block, n_aux - P0);
  for (int k = threadIdx.x; k < kFwAux; k += kFwThreads) {
    const bool in = k < naux;
    const double b = in ? beta[P0 + k] : 1.0;
    sb[k] = b;
    scp[k] = -kLog2e * b;
    sr0[k] = in ? R[3 * (P0 + k)] : 0.0;
    sr1[k] = in ? R[3 * (P0 + k) + 1] : 0.0;
    sr2[k] = in ? R[3 * (P0 + k) + 2] : 0.0;
#pragma unroll
    for (int w = 0; w < kFwWarps; ++w) red[w][k] = 0.0;
  }
  __syncthreads();  // tables and the resident aux; the only block-wide barrier before the end
  const int64_t a0 = blockIdx.y * per_split;
  const int64_t a1 = imin64(a0 + per_split, n_live);
  const int ngroups = (naux + kFwNA - 1) / kFwNA;
  unsigned long long evals = 0;  // node evaluations of real (aux, pair) units, warp-uniform
  for (int64_t c0 = a0; c0 < a1; c0 += kFwThreads) {
    const int64_t a = c0 + threadIdx.x;
    const bool live = a < a1;
    const unsigned lanes = __popc(__ballot_sync(0xffffffffu, live));
    if (lanes == 0) continue;  // warp-uniform: the tail chunk's empty warps
    const double* rr = rec + (live ? a : a0) * GSDFT_REC_FIELDS;
    double L[3], U[9], Pc[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) L[k] = rr[GSDFT_REC_L0 + k];
#pragma unroll
    for (int k = 0; k < 9; ++k) U[k] = rr[GSDFT_REC_U00 + k];
#pragma unroll
    for (int k = 0; k < 3; ++k) Pc[k] = rr[GSDFT_REC_P0 + k];
    const double qk = live ? rr[GSDFT_REC_QK] : 0.0;  // a tail lane stands in with weight 0
#pragma unroll 1
    for (int grp = 0; grp < ngroups; ++grp) {
      double m[kFwNA][3], g[kFwNA][3], h[kFwNA][3], coul[kFwNA], e0[kFwNA];
#pragma unroll
      for (int u = 0; u < kFwNA; ++u) {
        const int k = grp * kFwNA + u;  // k < kFwAux always; beyond naux a dummy aux, dropped
        const double b = sb[k], cP = scp[k];
        const double d0 = sr0[k] - Pc[0], d1 = sr1[k] - Pc[1], d2 = sr2[k] - Pc[2];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const double y = U[c] * d0 + U[3 + c] * d1 + U[6 + c] * d2;
          m[u][c] = (cP * L[c]) * (y * y);
          g[u][c] = L[c] * b;
          h[u][c] = L[c] + b;
        }
        coul[u] = 0.0;
        e0[u] = 0.0;
      }
      int nodes = GSDFT_NQUAD;
#pragma unroll
      for (int n = 0; n < GSDFT_NQUAD; ++n) {
        const double t2 = kQuadT2[n];
        bool far = node_check(n);  // tested at the check nodes only (the exponent is monotone)
#pragma unroll
        for (int u = 0; u < kFwNA; ++u) {
          const double G0 = fma(t2, h[u][0], g[u][0]);
          const double G1 = fma(t2, h[u][1], g[u][1]);
          const double G2 = fma(t2, h[u][2], g[u][2]);
          const double p12 = G1 * G2;
          const double prod = G0 * p12;
          const double num = fma(m[u][0], p12, G0 * fma(m[u][1], G2, m[u][2] * G1));
          const double y = rsqrt_pos(prod);
          const double inv = y * y;
          const double x = num * inv;  // node exponent / t^2, log2 units
          const double ew = wexp2<kFwBits>(x, t2, etab + (n << kFwBits));
          coul[u] = fma(y, ew, coul[u]);
          if (n == 0) e0[u] = x * t2;
          if (node_check(n)) far = far && fma(x, t2, -e0[u]) < -skip2;
        }
        // node screening (warp-uniform): every later node is below the last bit of every lane's sum
        if (node_check(n) && __all_sync(0xffffffffu, far)) {
          nodes = n + 1;
          break;
        }
      }
      const int real = (int)imin64(kFwNA, naux - grp * kFwNA);
      evals += (unsigned long long)nodes * (unsigned long long)(real * lanes);
      // gamma_k += sum over the warp's representatives (fixed shuffle tree), per warp in order
      double v[kFwNA];
#pragma unroll
      for (int u = 0; u < kFwNA; ++u) v[u] = warp_sum(qk * coul[u]);
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < kFwNA; ++u) red[warp][grp * kFwNA + u] += v[u];
      }
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < naux; k += kFwThreads) {
    double acc = red[0][k];
#pragma unroll
    for (int w = 1; w < kFwWarps; ++w) acc += red[w][k];
    partial[blockIdx.y * n_aux + P0 + k] = acc * KN[P0 + k];
  }
  if (lane == 0 && evals) atomicAdd(&g_fw_node_evals, evals);
}

// gamma_P = sum_s partial[s][P], fixed order.
__global__ void sum_splits_kernel(const double* __restrict__ partial, int S, int64_t n,
                                  double* __restrict__ out) {
  int64_t P = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (P >= n) return;
  // four independent partial sums, combined in a fixed order
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  int s = 0;
  for (; s + 3 < S; s += 4) {
    a0 += partial[(int64_t)s * n + P];
    a1 += partial[(int64_t)(s + 1) * n + P];
    a2 += partial[(int64_t)(s + 2) * n + P];
    a3 += partial[(int64_t)(s + 3) * n + P];
  }
  for (; s < S; ++s) a0 += partial[(int64_t)s * n + P];
  out[P] = (a0 + a1) + (a2 + a3);
}

// Aux per block: the fewest blocks of at most kFwAux, equally sized (a multiple of kFwNA), so that no
// block is left with a short remainder while the others run full.
static int forward_aux_per_block(int64_t n_aux) {
  const int64_t blocks = (n_aux + kFwAux - 1) / kFwAux;
  int64_t per = (n_aux + blocks - 1) / blocks;
  per = (per + kFwNA - 1) / kFwNA * kFwNA;
  return (int)imin64(per, kFwAux);
}

// Pair splits of the forward grid: aux blocks x S CTAs filling whole waves of resident CTAs, with at
// least two chunks of representatives per split. The occupancy query runs once (a thread-safe
// static).
static int forward_splits(int64_t n_live, int64_t n_aux) {
  static const int per_sm = [] {
    int v = 0;
    cudaFuncSetAttribute(j_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kFwDynSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, j_forward_kernel, kFwThreads, kFwDynSmem);
    return v > 0 ? v : 1;
  }();
  const int apb = forward_aux_per_block(n_aux);
  int64_t aux_blocks = (n_aux + apb - 1) / apb;
  int64_t cap = (int64_t)device_sms() * per_sm;
  int64_t max_s = imin64(4096, imax64(1, n_live / (2 * kFwThreads)));
  return best_splits(aux_blocks, cap, max_s);
}

}  // namespace gsdft

using namespace gsdft;

namespace gsdft {
int device_status_forward(int* out, int clear) {
  GSDFT_CUDA(cudaMemcpyFromSymbol(out, g_device_status, sizeof(int)));
  if (clear) {
    int z = 0;
    GSDFT_CUDA(cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)));
  }
  return GSDFT_OK;
}
int device_status_vjp(int* out, int clear);
int node_evals_forward(unsigned long long* out, int clear) {
  GSDFT_CUDA(cudaMemcpyFromSymbol(out, g_fw_node_evals, sizeof(unsigned long long)));
  if (clear) {
    unsigned long long z = 0;
    GSDFT_CUDA(cudaMemcpyToSymbol(g_fw_node_evals, &z, sizeof(z)));
  }
  return GSDFT_OK;
}
}  // namespace gsdft

extern "C" int gsdft_device_status(int* status_host, int clear) {
  GSDFT_REQUIRE(status_host, "null pointer");
  GSDFT_CUDA(cudaDeviceSynchronize());
  int a = 0, b = 0;
  int rc = device_status_forward(&a, clear);
  if (rc) return rc;
  rc = device_status_vjp(&b, clear);
  if (rc) return rc;
  *status_host = a | b;
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// Estimated integral cost of each representative, for a cost-balanced partition across devices:
// over a strided sample of the aux, the node screening rule of the integral kernels applied per
// (aux, pair) (first node at which the exponent has grown kNodeSkipLog2 past the first node's, at the
// same check nodes), plus one node's worth of per-(aux, pair) fixed work. Integer, so the prefix
// sums that cut the list are exact and identical on every rank.
// ------------------------------------------------------------------------------------------------
__global__ void rep_cost_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                const int32_t* __restrict__ rep_pos, int64_t n_rep,
                                const double* __restrict__ beta, const double* __restrict__ R,
                                int64_t n_aux, int64_t stride, double skip2,
                                int64_t* __restrict__ cost) {
  const int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_rep) return;
  const int64_t e = rep_pos[a];
  const int i = pi[e], j = pj[e];
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
  double sm[3][3];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) sm[r][c] = 0.5 * (Ah[3 * r + c] + Ah[3 * c + r]);
  double lam[3], U[9];
  jacobi_eig3(sm, lam, U);
  int64_t total = 0;
  for (int64_t q = 0; q < n_aux; q += stride) {
    const double b = beta[q];
    const double d0 = R[3 * q] - P[0], d1 = R[3 * q + 1] - P[1], d2 = R[3 * q + 2] - P[2];
    double m[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double y = U[c] * d0 + U[3 + c] * d1 + U[6 + c] * d2;
      m[c] = -kLog2e * b * lam[c] * y * y;
    }
    int nodes = GSDFT_NQUAD;
    double e0 = 0.0;
    for (int n = 0; n < GSDFT_NQUAD; ++n) {
      const double t2 = kQuadT2[n];
      double x = 0.0;
#pragma unroll
      for (int c = 0; c < 3; ++c) x += m[c] / fma(t2, lam[c] + b, lam[c] * b);
      if (n == 0) e0 = x * t2;
      if (node_check(n) && x * t2 - e0 < -skip2) {
        nodes = n + 1;
        break;
      }
    }
    total += nodes + 1;
  }
  cost[a] = total;
}

extern "C" int gsdft_rep_cost(const double* A9, const double* mu, int64_t M, const int32_t* pi,
                              const int32_t* pj, const int32_t* rep_pos, int64_t n_rep,
                              const double* beta, const double* R, int64_t n_aux, int64_t n_sample,
                              int64_t* cost, gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_rep >= 0 && n_aux > 0 && n_sample > 0, "bad sizes");
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(A9 && mu && pi && pj && rep_pos && beta && R && cost, "null pointer");
  const int64_t stride = imax64(1, n_aux / n_sample);
  rep_cost_kernel<<<grid_1d(n_rep, 128), 128, 0, (cudaStream_t)stream>>>(
      A9, mu, pi, pj, rep_pos, n_rep, beta, R, n_aux, stride, node_skip_threshold(), cost);
  GSDFT_LAUNCHED("rep_cost");
  return GSDFT_OK;
}

extern "C" int gsdft_pair_prep(const double* A9, const double* mu, const double* N, int64_t M,
                               const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                               const double* rep_w, int64_t n_rep, const double* C_occ,
                               const double* occ, int64_t n_occ, double* rec,
                               gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_rep >= 0 && n_occ >= 0, "bad sizes");
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(A9 && mu && N && pi && pj && rep_pos && rep_w && rec, "null pointer");
  GSDFT_REQUIRE(n_occ == 0 || (C_occ && occ), "null C_occ/occ");
  GSDFT_REQUIRE((reinterpret_cast<uintptr_t>(rec) & 15) == 0, "rec must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  pair_prep_kernel<<<grid_1d(n_rep, 128), 128, 0, st>>>(A9, mu, N, pi, pj, rep_pos, n_rep, rec);
  GSDFT_LAUNCHED("pair_prep");
  if (n_occ == 0 && !C_occ) return GSDFT_OK;  // q and qk come from gsdft_block_density
  if (n_occ <= 32) {
    pair_density_thread_kernel<<<grid_1d(n_rep, 128), 128, 0, st>>>(pi, pj, rep_w, rep_pos, n_rep,
                                                                   C_occ, occ, n_occ, rec);
  } else {
    pair_density_kernel<<<grid_1d(n_rep * 32, 256), 256, 0, st>>>(pi, pj, rep_w, rep_pos, n_rep,
                                                                  C_occ, occ, n_occ, rec);
  }
  GSDFT_LAUNCHED("pair_density");
  return GSDFT_OK;
}

extern "C" size_t gsdft_j_forward_workspace_size(int64_t n_live, int64_t n_aux) {
  int S = forward_splits(n_live, n_aux);
  return align_up((size_t)S * n_aux * sizeof(double), 256) + 256;
}

extern "C" int gsdft_j_forward(const double* rec, int64_t n_live, const double* beta,
                               const double* R, const double* KN, int64_t n_aux, double* gamma,
                               void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_live >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31), "bad sizes");
  GSDFT_REQUIRE(beta && R && KN && gamma, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_live == 0) {
    GSDFT_CUDA(cudaMemsetAsync(gamma, 0, n_aux * sizeof(double), st));
    return GSDFT_OK;
  }
  GSDFT_REQUIRE(rec && (reinterpret_cast<uintptr_t>(rec) & 15) == 0, "rec must be 16-byte aligned");
  int S = forward_splits(n_live, n_aux);
  Carver c(ws, ws_bytes);
  double* partial = c.take<double>((size_t)S * n_aux);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "forward workspace too small (%zu < %zu)", ws_bytes, c.off);
  int64_t per_split = (n_live + S - 1) / S;
  const int apb = forward_aux_per_block(n_aux);
  dim3 grid((unsigned)((n_aux + apb - 1) / apb), (unsigned)S);
  j_forward_kernel<<<grid, kFwThreads, kFwDynSmem, st>>>(rec, n_live, beta, R, KN, n_aux,
                                                         per_split, apb, node_skip_threshold(),
                                                         partial);
  GSDFT_LAUNCHED("j_forward");
  sum_splits_kernel<<<grid_1d(n_aux, 256), 256, 0, st>>>(partial, S, n_aux, gamma);
  GSDFT_LAUNCHED("sum_splits");
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// No-allocation variant of gsdft_j_forward.
//
// For callers that cannot allocate device memory at call time and cannot hand in a workspace —
// for example a handler running inside a framework that owns the device memory pool (XLA
// preallocates most of the GPU for its own allocator, so a cudaMalloc from inside a custom call can
// fail or fragment that pool), or a caller with a fixed memory budget decided up front. The
// per-split partial sums that gsdft_j_forward keeps in its workspace live here in one fixed array
// of kNoAllocScratchDoubles doubles (8 MiB) that every device holds from library load until exit.
// ------------------------------------------------------------------------------------------------
namespace gsdft {

constexpr int64_t kNoAllocScratchDoubles = int64_t(1) << 20;
static __device__ __align__(256) double g_forward_scratch[kNoAllocScratchDoubles];

static std::mutex g_scratch_mu;
static double* g_scratch_dev[256];  // device address of g_forward_scratch, per device ordinal

// The host-side name g_forward_scratch is only a stand-in for the device array; its device address
// is looked up once per device (with that device current) and cached.
static int forward_scratch(double** out) {
  int dev = 0;
  GSDFT_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return fail(GSDFT_ERR_ARG, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_forward_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(GSDFT_ERR_CUDA, "cudaGetSymbolAddress(forward scratch) on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_scratch_dev[dev] = static_cast<double*>(p);
  }
  *out = g_scratch_dev[dev];
  return GSDFT_OK;
}

}  // namespace gsdft

extern "C" int gsdft_j_forward_noalloc(const double* rec, int64_t n_rep, const double* beta,
                                       const double* R, const double* KN, int64_t n_aux,
                                       double* gamma, gsdft_stream_t stream) {
  using namespace gsdft;
  GSDFT_REQUIRE(n_rep >= 0 && n_aux > 0, "bad sizes");
  if (n_aux > kNoAllocScratchDoubles)
    return fail(GSDFT_ERR_ARG,
                "gsdft_j_forward_noalloc: n_aux = %lld exceeds the fixed scratch of %lld doubles; "
                "use gsdft_j_forward with a workspace",
                (long long)n_aux, (long long)kNoAllocScratchDoubles);
  GSDFT_REQUIRE(beta && R && KN && gamma, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  double* scratch = nullptr;
  int rc = forward_scratch(&scratch);
  if (rc) return rc;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(gamma, 0, n_aux * sizeof(double), st));
    return GSDFT_OK;
  }
  GSDFT_REQUIRE(rec && (reinterpret_cast<uintptr_t>(rec) & 15) == 0, "rec must be 16-byte aligned");
  // Every entry the reduction reads (S rows of n_aux) is written by the kernel first, so the
  // array needs no clearing; the split count is capped so the partial sums fit.
  int64_t S = forward_splits(n_rep, n_aux);
  S = imin64(S, kNoAllocScratchDoubles / n_aux);
  int64_t per_split = (n_rep + S - 1) / S;
  const int apb = forward_aux_per_block(n_aux);
  dim3 grid((unsigned)((n_aux + apb - 1) / apb), (unsigned)S);
  j_forward_kernel<<<grid, kFwThreads, kFwDynSmem, st>>>(rec, n_rep, beta, R, KN, n_aux, per_split,
                                                         apb, node_skip_threshold(), scratch);
  GSDFT_LAUNCHED("j_forward_noalloc");
  sum_splits_kernel<<<grid_1d(n_aux, 256), 256, 0, st>>>(scratch, (int)S, n_aux, gamma);
  GSDFT_LAUNCHED("sum_splits_noalloc");
  return GSDFT_OK;
}
