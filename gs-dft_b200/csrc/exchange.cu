// Screened density-fitted exchange (RI-K) over the significant pairs (gs_dft/coulomb/ri.py:497-544):
//   D[P,o,o'] = sum_{live (i,k)} (P|ik) C_io C_ko',   E_K = -tr((V + lam I)^-1 M),
//   M_PQ = sum_{o,o'} D[P,o,o'] D[Q,o,o'] = (D D^T)_PQ,  so  E_K = -|L^-1 D|_F^2  with V + lam I = L L^T.
// Layout (row-major): Bt[a][P] = (P|a) for the representatives a (thread per aux, coalesced
// stores), kept for the whole step. The orbital products are streamed over chunks of orbitals o
// (the reference's occ_chunk): X_c[a][(o - o0) n + o'] = C_io C_ko' (+ C_ko C_io' for a merged
// transposed twin, whose integral is the same) for o in the chunk, D[:, chunk] = Bt^T X_c, so only
// n_rep x occ_chunk x n products are ever held (the whole X would be n_rep x n^2). The contractions
// are the library's own DMMA GEMMs (dense.cu): D split over the pairs, Z = L^-1 D and its reverse
// as products with the packed inverse factor read as a lower-triangular operand; the integral
// block and every reduction are this file's kernels, all in a fixed order (bitwise reproducible).
// Reverse: Ybar = dE/dD = -2 g L^-T L^-1 D; dE/dX_c = Bt Ybar[:, chunk] (into g_C chunk by chunk);
// dE/d(P|a) = W[P][a] = sum_c (Ybar[:, chunk] X_c^T)[P][a], which drives the same integral reverse
// pass as RI-J with a per-(P,a) weight (gsdft_j_vjp_weighted, W stored aux-major in the integral
// block's storage once the block is no longer needed).
// Range separation (gs_dft/coulomb/ri.py:149,232-235): the long-range exchange E_K[erf(omega r)/r]
// is the same computation on a different node rule (the 12-node segment rule on [0, omega], a
// runtime table from gsdft_lr_node_table) with the attenuated metric's factor.
#include "common.cuh"

extern "C" size_t gsdft_j_vjp_weighted_workspace_size(int64_t n_live, int64_t n_aux);
extern "C" int gsdft_j_vjp_weighted(const double* rec, int64_t n_live, const double* beta,
                                    const double* R, const double* KN, const double* Wt,
                                    int64_t ldw, int64_t n_aux, const double* nodes, int n_nodes,
                                    double* sums, void* ws, size_t ws_bytes,
                                    gsdft_stream_t stream);

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
// records (grid-stride over tiles), staged in shared memory. kLR: the nodes come from a runtime
// table (nq <= GSDFT_NQUAD nodes: t^2 rows, then the weighted exp2 rows).
template <bool kLR>
__global__ void __launch_bounds__(kKThreads)
    k_block_kernel(const double* __restrict__ rec, int64_t n_rep, const double* __restrict__ beta,
                   const double* __restrict__ R, const double* __restrict__ KN, int64_t n_aux,
                   double* __restrict__ Bt, const double* __restrict__ nodes, int nq) {
  __shared__ double tile[kKTile * GSDFT_REC_FIELDS];
  __shared__ double lrt[kLR ? GSDFT_NQUAD : 1];
  extern __shared__ __align__(16) double etab[];
  if (kLR) {
    for (int k = threadIdx.x; k < nq * 64; k += blockDim.x) etab[k] = nodes[2 * GSDFT_NQUAD + k];
    for (int k = threadIdx.x; k < GSDFT_NQUAD; k += blockDim.x) lrt[k] = nodes[k];
  } else {
    load_wexp2_tables<kKBits>(etab);
  }
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
        if (kLR && n >= nq) break;
        const double t2 = kLR ? lrt[n] : kQuadT2[n];
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

// X_c[a][(o - o0) n + q] = C_io C_kq + (merged twin ? C_ko C_iq : 0) for o in [o0, o0 + nc), (i, k)
// the representative's pair.
__global__ void k_xbuild_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                const int32_t* __restrict__ rep_pos,
                                const int32_t* __restrict__ rep_twin, int64_t n_rep,
                                const double* __restrict__ C, int64_t no, int64_t o0, int64_t nc,
                                double* __restrict__ X) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t W = nc * no;
  if (idx >= n_rep * W) return;
  const int64_t a = idx / W, r = idx - a * W;
  const int64_t o = o0 + r / no, q = r % no;
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

// g_C[s][p] += the chunk's part of dE/dC: with Xb the representative's dE/dX_c (nc x n rows
// o in [o0, o0 + nc)), over the by-pi segment of s (s = i, partner k): [p in chunk] sum_q Xb[p][q]
// C_kq + [twin] sum_o Xb[o][p] C_ko; over the by-pj segment (s = k, partner i):
// sum_o Xb[o][p] C_io + [twin, p in chunk] sum_q Xb[p][q] C_iq. Fixed order; chunks add in order.
__global__ void k_cgrad_kernel(const int32_t* __restrict__ order_i, const int64_t* __restrict__ seg_i,
                               const int32_t* __restrict__ partner_i,
                               const int32_t* __restrict__ order_j, const int64_t* __restrict__ seg_j,
                               const int32_t* __restrict__ partner_j,
                               const int32_t* __restrict__ rep_twin, const double* __restrict__ Xbar,
                               const double* __restrict__ C, int64_t no, int64_t o0, int64_t nc,
                               double* __restrict__ gC) {
  const int64_t s = blockIdx.x;
  const int64_t W = nc * no;
  for (int64_t p = threadIdx.x; p < no; p += blockDim.x) {
    const bool in_c = p >= o0 && p < o0 + nc;
    const int64_t pl = p - o0;
    double acc = 0.0;
    for (int64_t e = seg_i[s]; e < seg_i[s + 1]; ++e) {
      const int64_t r = order_i[e];
      const double* Xb = Xbar + r * W;
      const double* ck = C + (int64_t)partner_i[e] * no;
      if (in_c)
        for (int64_t q = 0; q < no; ++q) acc = fma(Xb[pl * no + q], ck[q], acc);
      if (rep_twin[r] >= 0)
        for (int64_t o = 0; o < nc; ++o) acc = fma(Xb[o * no + p], ck[o0 + o], acc);
    }
    for (int64_t e = seg_j[s]; e < seg_j[s + 1]; ++e) {
      const int64_t r = order_j[e];
      const double* Xb = Xbar + r * W;
      const double* ci = C + (int64_t)partner_j[e] * no;
      for (int64_t o = 0; o < nc; ++o) acc = fma(Xb[o * no + p], ci[o0 + o], acc);
      if (rep_twin[r] >= 0 && in_c)
        for (int64_t q = 0; q < no; ++q) acc = fma(Xb[pl * no + q], ci[q], acc);
    }
    gC[s * no + p] += acc;
  }
}

struct KLayout {
  double *Bt, *XB, *Y, *Dc, *part, *split;
  int S;
  int64_t nc;
  void* vjp_ws;
  size_t vjp_bytes;
  bool ok;
};

static int64_t k_chunk(int64_t no, int64_t occ_chunk) {
  return occ_chunk <= 0 ? no : imin64(occ_chunk, no);
}

// Workspace: the integral block (later the weights W), one chunk of products X_c or their
// cotangents, Y = L^-T Z over all orbitals, one chunk of D and its split-K partials, the
// sum-of-squares partials, and the weighted reverse pass's workspace.
static KLayout k_layout(void* ws, size_t ws_bytes, int64_t n_rep, int64_t n_aux, int64_t no,
                        int64_t occ_chunk) {
  const int64_t K2 = no * no, nc = k_chunk(no, occ_chunk), Wc = nc * no;
  const int64_t nr = imax64(n_rep, 1);
  Carver c(ws, ws_bytes);
  KLayout l;
  l.nc = nc;
  l.Bt = c.take<double>((size_t)nr * n_aux);
  l.XB = c.take<double>((size_t)nr * Wc);
  l.Y = c.take<double>((size_t)n_aux * K2);
  l.Dc = c.take<double>((size_t)n_aux * Wc);
  l.part = c.take<double>(kKRedBlocks);
  l.S = splitk_count(n_aux, Wc, nr);
  l.split = c.take<double>((size_t)l.S * n_aux * Wc);
  l.vjp_bytes = gsdft_j_vjp_weighted_workspace_size(nr, n_aux);
  l.vjp_ws = c.take<unsigned char>(l.vjp_bytes);
  l.ok = c.ok;
  return l;
}

static int k_xbuild(const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                    const int32_t* rep_twin, int64_t n_rep, const double* C, int64_t no,
                    int64_t o0, int64_t nc, double* X, cudaStream_t st) {
  k_xbuild_kernel<<<grid_1d(n_rep * nc * no, 256), 256, 0, st>>>(pi, pj, rep_pos, rep_twin, n_rep,
                                                                 C, no, o0, nc, X);
  GSDFT_LAUNCHED("k_xbuild");
  return GSDFT_OK;
}

}  // namespace gsdft

using namespace gsdft;

extern "C" size_t gsdft_k_workspace_size(int64_t n_rep, int64_t n_aux, int64_t n_occ,
                                         int64_t occ_chunk) {
  const int64_t K2 = n_occ * n_occ, nc = k_chunk(n_occ, occ_chunk), Wc = nc * n_occ;
  const int64_t nr = imax64(n_rep, 1);
  Sizer z;
  z.take<double>((size_t)nr * n_aux);
  z.take<double>((size_t)nr * Wc);
  z.take<double>((size_t)n_aux * K2);
  z.take<double>((size_t)n_aux * Wc);
  z.take<double>(kKRedBlocks);
  z.take<double>((size_t)splitk_count(n_aux, Wc, nr) * n_aux * Wc);
  z.take<unsigned char>(gsdft_j_vjp_weighted_workspace_size(nr, n_aux));
  return z.off + 256;
}

static int k_check(int64_t n_rep, int64_t n_aux, int64_t n_occ, const double* nodes, int n_nodes) {
  GSDFT_REQUIRE(n_rep >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31) && n_occ > 0 &&
                    n_occ * n_occ < (int64_t(1) << 31) && n_rep < (int64_t(1) << 31),
                "bad sizes");
  GSDFT_REQUIRE(!nodes || (n_nodes >= 1 && n_nodes <= GSDFT_NQUAD), "bad node count");
  return GSDFT_OK;
}

extern "C" int gsdft_k_forward(const double* rec, const int32_t* pi, const int32_t* pj,
                               const int32_t* rep_pos, const int32_t* rep_twin, int64_t n_rep,
                               const double* beta, const double* R, const double* KN,
                               int64_t n_aux, const double* nodes, int n_nodes,
                               const double* Linv, const double* C_occ, int64_t n_occ,
                               int64_t occ_chunk, double* Z, double* E, void* ws, size_t ws_bytes,
                               gsdft_stream_t stream) {
  int rc = k_check(n_rep, n_aux, n_occ, nodes, n_nodes);
  if (rc) return rc;
  GSDFT_REQUIRE(beta && R && KN && Linv && C_occ && Z && E && ws, "null pointer");
  GSDFT_REQUIRE(n_rep == 0 || (rec && pi && pj && rep_pos && rep_twin), "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  KLayout l = k_layout(ws, ws_bytes, n_rep, n_aux, n_occ, occ_chunk);
  if (!l.ok) return fail(GSDFT_ERR_ARG, "exchange workspace too small");
  const int64_t K2 = n_occ * n_occ;
  if (n_rep == 0) {
    GSDFT_CUDA(cudaMemsetAsync(Z, 0, (size_t)n_aux * K2 * sizeof(double), st));
  } else {
    const int64_t ntiles = (n_rep + kKTile - 1) / kKTile;
    dim3 grid((unsigned)((n_aux + kKThreads - 1) / kKThreads), (unsigned)imin64(ntiles, 65535));
    if (nodes)
      k_block_kernel<true><<<grid, kKThreads, kKDynSmem, st>>>(rec, n_rep, beta, R, KN, n_aux, l.Bt,
                                                               nodes, n_nodes);
    else
      k_block_kernel<false><<<grid, kKThreads, kKDynSmem, st>>>(rec, n_rep, beta, R, KN, n_aux,
                                                                l.Bt, nullptr, 0);
    GSDFT_LAUNCHED("k_block");
    for (int64_t o0 = 0; o0 < n_occ; o0 += l.nc) {
      const int64_t nc = imin64(l.nc, n_occ - o0), Wc = nc * n_occ;
      rc = k_xbuild(pi, pj, rep_pos, rep_twin, n_rep, C_occ, n_occ, o0, nc, l.XB, st);
      if (rc) return rc;
      // D[:, chunk] (n_aux x Wc) = Bt^T X_c, split over the pairs
      rc = gemm_dmma_splitk(true, n_aux, Wc, n_rep, 1.0, l.Bt, n_aux, l.XB, Wc, 0.0, l.Dc, Wc,
                            l.split, splitk_count(n_aux, Wc, n_rep), st);
      if (rc) return rc;
      // Z[:, chunk] = L^-1 D[:, chunk]: the packed inverse's lower triangle
      rc = gemm_dmma(false, false, true, n_aux, Wc, n_aux, 1.0, Linv, n_aux, l.Dc, Wc, 0.0,
                     Z + o0 * n_occ, K2, st);
      if (rc) return rc;
    }
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
                                int64_t n_aux, const double* nodes, int n_nodes,
                                const double* Linv, const double* C_occ, int64_t n_occ,
                                int64_t occ_chunk, const double* Z, const double* g_E,
                                const int32_t* order_i, const int64_t* seg_i,
                                const int32_t* partner_i, const int32_t* order_j,
                                const int64_t* seg_j, const int32_t* partner_j, int64_t M,
                                double* sums, double* g_C, void* ws, size_t ws_bytes,
                                gsdft_stream_t stream) {
  int rc = k_check(n_rep, n_aux, n_occ, nodes, n_nodes);
  if (rc) return rc;
  GSDFT_REQUIRE(M > 0, "bad sizes");
  GSDFT_REQUIRE(beta && R && KN && Linv && C_occ && Z && g_C && ws && seg_i && seg_j,
                "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  GSDFT_CUDA(cudaMemsetAsync(g_C, 0, (size_t)M * n_occ * sizeof(double), st));
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && pi && pj && rep_pos && rep_twin && sums && order_i && partner_i &&
                    order_j && partner_j,
                "null pointer");
  KLayout l = k_layout(ws, ws_bytes, n_rep, n_aux, n_occ, occ_chunk);
  if (!l.ok) return fail(GSDFT_ERR_ARG, "exchange workspace too small");
  const int64_t K2 = n_occ * n_occ;
  // Bt from the forward (the same workspace, untouched in between)
  // Y = L^-T Z (the packed inverse's lower triangle, transposed), then Ybar = -2 g_E Y
  rc = gemm_dmma(true, false, true, n_aux, K2, n_aux, 1.0, Linv, n_aux, Z, K2, 0.0, l.Y, K2, st);
  if (rc) return rc;
  k_scale_kernel<<<grid_1d(n_aux * K2, 256), 256, 0, st>>>(l.Y, n_aux * K2, g_E);
  GSDFT_LAUNCHED("k_scale");
  // dE/dX_c = Bt Ybar[:, chunk] (n_rep x Wc), folded into g_C chunk by chunk
  for (int64_t o0 = 0; o0 < n_occ; o0 += l.nc) {
    const int64_t nc = imin64(l.nc, n_occ - o0), Wc = nc * n_occ;
    rc = gemm_dmma(false, false, false, n_rep, Wc, n_aux, 1.0, l.Bt, n_aux, l.Y + o0 * n_occ, K2,
                   0.0, l.XB, Wc, st);
    if (rc) return rc;
    k_cgrad_kernel<<<(unsigned)M, 128, 0, st>>>(order_i, seg_i, partner_i, order_j, seg_j,
                                               partner_j, rep_twin, l.XB, C_occ, n_occ, o0, nc,
                                               g_C);
    GSDFT_LAUNCHED("k_cgrad");
  }
  // W (n_aux x n_rep) = sum_c Ybar[:, chunk] X_c^T, into Bt's storage (Bt is no longer needed)
  double* Wt = l.Bt;
  for (int64_t o0 = 0; o0 < n_occ; o0 += l.nc) {
    const int64_t nc = imin64(l.nc, n_occ - o0), Wc = nc * n_occ;
    rc = k_xbuild(pi, pj, rep_pos, rep_twin, n_rep, C_occ, n_occ, o0, nc, l.XB, st);
    if (rc) return rc;
    rc = gemm_dmma(false, true, false, n_aux, n_rep, Wc, 1.0, l.Y + o0 * n_occ, K2, l.XB, Wc,
                   o0 == 0 ? 0.0 : 1.0, Wt, n_rep, st);
    if (rc) return rc;
  }
  return gsdft_j_vjp_weighted(rec, n_rep, beta, R, KN, Wt, n_rep, n_aux, nodes, n_nodes, sums,
                              l.vjp_ws, l.vjp_bytes, stream);
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
