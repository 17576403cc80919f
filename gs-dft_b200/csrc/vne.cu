// Screened nuclear attraction on the pair list (gs_dft/screening/pairs.py:348-370, 409-440):
//   V_a = -2 pi KN_a sum_A Z_A sum_n w_n det(B_n)^-1/2 exp(-t_n^2 d.A_hat B_n^-1 d),
//   B_n = A_hat + t_n^2 I, d = R_A - P_a (the reference's t^2|d|^2 - t^4 d.adj(B)d/det B),
//   E_ne = sum_a q_a V_a.
// In the eigenframe of A_hat (lam, U from the pair record) B_n is diagonal, lam_k + t^2, and with
// y = U^T d the exponent is t^2 sum_k lam_k y_k^2 / (lam_k + t^2): the integrand of the RI-J
// kernels with the aux exponent taken to infinity (a point charge). Its reverse pass
//   df/dA_hat = f (-1/2 B^-1 - t^4 z z^T),   df/dP = 2 t^2 f A_hat z,   z = B^-1 d
// is the RI-J one with beta = 1 in the weights, so the 13 per-pair sums come out in
// gsdft_j_vjp's layout and scale and the same chain (gsdft_pair_chain -> gsdft_splat_reduce ->
// gsdft_density_grad -> gsdft_chart_vjp) turns them into splat and orbital gradients; added onto
// the RI-J sums, one chain carries E_J + E_ne.
#include "common.cuh"

namespace gsdft {

constexpr int kVneThreads = 64;   // representatives per CTA (one per thread)
constexpr int kVneBits = 6;       // 2^6-entry weighted exp2 table per node
constexpr size_t kVneDynSmem = sizeof(double) * GSDFT_NQUAD * (1 << kVneBits);
constexpr double kVnePref = 2.0 * kPi;  // (2/sqrt(pi)) pi^(3/2)

// One representative per thread, every atom in turn (atom loads are warp-uniform broadcasts).
// B_n depends on the pair and the node only, so 1/(lam_k + t_n^2) and det(B_n)^-1/2 are computed
// once per thread (80 values, held in registers) and every atom reuses them; the exponent is then
// sum_k m_k / (lam_k + t^2), m_k = -log2(e) lam_k y_k^2.
// Writes V (by representative or at its list positions), the block's sum of q V, and with kGrad
// the reverse-pass sums scaled by g_E (-2 pi / pref) so that gsdft_pair_chain, which multiplies
// by q KN pref, sees -2 pi q KN.
template <bool kGrad>
__global__ void __launch_bounds__(kVneThreads)
    vne_kernel(const double* __restrict__ rec, int64_t n_rep, const double4* __restrict__ atoms,
               int64_t n_atoms, const double* __restrict__ gE, const int32_t* __restrict__ rep_pos,
               const int32_t* __restrict__ rep_twin, double* __restrict__ V,
               double* __restrict__ sums, int add, double* __restrict__ block_E) {
  extern __shared__ __align__(16) double etab[];  // GSDFT_NQUAD x 2^kVneBits weighted table
  __shared__ double warp_E[kVneThreads / 32];
  load_wexp2_tables<kVneBits>(etab);
  __syncthreads();
  const int tid = threadIdx.x;
  const int64_t a = blockIdx.x * (int64_t)kVneThreads + tid;
  const bool live = a < n_rep;
  const double* rr = rec + (live ? a : 0) * GSDFT_REC_FIELDS;  // dereferenced only when live
  double L[3], U[9], Pc[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) L[k] = live ? rr[GSDFT_REC_L0 + k] : 1.0;
#pragma unroll
  for (int k = 0; k < 9; ++k) U[k] = live ? rr[GSDFT_REC_U00 + k] : (k % 4 == 0 ? 1.0 : 0.0);
#pragma unroll
  for (int k = 0; k < 3; ++k) Pc[k] = live ? rr[GSDFT_REC_P0 + k] : 0.0;
  // Nodes in passes of kPass (all 20 for the value alone; two passes of 10 with the reverse sums,
  // which are linear in the node terms, so that the pass's constants and the sums fit in registers).
  constexpr int kPass = kGrad ? GSDFT_NQUAD / 2 : GSDFT_NQUAD;
  double SJ = 0.0, SD[3] = {0, 0, 0}, SV[3] = {0, 0, 0}, SZ[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll 1
  for (int n0 = 0; live && n0 < GSDFT_NQUAD; n0 += kPass) {
    double iG[kPass][3], yn[kPass];
#pragma unroll
    for (int j = 0; j < kPass; ++j) {
      const double t2 = kQuadT2[n0 + j];
      const double G0 = L[0] + t2, G1 = L[1] + t2, G2 = L[2] + t2;
      const double p12 = G1 * G2;
      const double yy = rsqrt_pos(G0 * p12);
      const double inv = yy * yy;
      iG[j][0] = p12 * inv;
      iG[j][1] = (G0 * G2) * inv;
      iG[j][2] = (G0 * G1) * inv;
      yn[j] = yy;
    }
#pragma unroll 1
    for (int64_t A = 0; A < n_atoms; ++A) {
      const double4 at = atoms[A];
      const double d0 = at.x - Pc[0], d1 = at.y - Pc[1], d2 = at.z - Pc[2];
      double y[3], m[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        y[c] = U[c] * d0 + U[3 + c] * d1 + U[6 + c] * d2;
        m[c] = (-kLog2e * L[c]) * (y[c] * y[c]);
      }
      double cf = 0.0, B[3] = {0, 0, 0}, C[3] = {0, 0, 0}, Z[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < kPass; ++j) {
        const int n = n0 + j;
        const double t2 = kQuadT2[n];
        const double iG0 = iG[j][0], iG1 = iG[j][1], iG2 = iG[j][2];
        const double ex = fma(m[0], iG0, fma(m[1], iG1, m[2] * iG2));
        const double f = yn[j] * wexp2<kVneBits>(ex, t2, etab + (n << kVneBits));
        cf += f;
        if (kGrad) {
          const double t4 = kQuadT4[n];
          const double g0 = f * iG0, g1 = f * iG1, g2 = f * iG2;
          B[0] += g0;
          B[1] += g1;
          B[2] += g2;
          C[0] = fma(t2, g0, C[0]);
          C[1] = fma(t2, g1, C[1]);
          C[2] = fma(t2, g2, C[2]);
          const double h0 = t4 * g0, h1 = t4 * g1, h2 = t4 * g2;
          Z[0] = fma(h0, iG0, Z[0]);
          Z[1] = fma(h1, iG1, Z[1]);
          Z[2] = fma(h2, iG2, Z[2]);
          Z[3] = fma(h0, iG1, Z[3]);
          Z[4] = fma(h0, iG2, Z[4]);
          Z[5] = fma(h1, iG2, Z[5]);
        }
      }
      const double zA = at.w;
      SJ = fma(zA, cf, SJ);
      if (kGrad) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          SD[c] = fma(zA, B[c], SD[c]);
          SV[c] = fma(zA, y[c] * C[c], SV[c]);
        }
        SZ[0] = fma(zA, (y[0] * y[0]) * Z[0], SZ[0]);
        SZ[1] = fma(zA, (y[1] * y[1]) * Z[1], SZ[1]);
        SZ[2] = fma(zA, (y[2] * y[2]) * Z[2], SZ[2]);
        SZ[3] = fma(zA, (y[0] * y[1]) * Z[3], SZ[3]);
        SZ[4] = fma(zA, (y[0] * y[2]) * Z[4], SZ[4]);
        SZ[5] = fma(zA, (y[1] * y[2]) * Z[5], SZ[5]);
      }
    }
  }
  // rec holds KN * pref; V = -2 pi KN SJ
  const double ratio = -kVnePref / kPref;
  const double v = live ? (ratio * rr[GSDFT_REC_KN]) * SJ : 0.0;
  double e = live ? rr[GSDFT_REC_Q] * v : 0.0;
  if (live && V != nullptr) {
    if (rep_pos != nullptr) {
      V[rep_pos[a]] = v;
      if (rep_twin != nullptr && rep_twin[a] >= 0) V[rep_twin[a]] = v;
    } else {
      V[a] = v;
    }
  }
  if (kGrad && live) {
    const double s = ratio * (gE ? gE[0] : 1.0);
    double* o = sums + a * GSDFT_VJP_FIELDS;
    double vals[GSDFT_VJP_FIELDS];
    vals[GSDFT_VJP_SJ] = SJ;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      vals[GSDFT_VJP_SD0 + c] = SD[c];
      vals[GSDFT_VJP_SV0 + c] = SV[c];
    }
#pragma unroll
    for (int c = 0; c < 6; ++c) vals[GSDFT_VJP_SZ00 + c] = SZ[c];
#pragma unroll
    for (int f = 0; f < GSDFT_VJP_FIELDS; ++f) o[f] = add ? fma(s, vals[f], o[f]) : s * vals[f];
  }
  // block sum of q V in a fixed order: lanes by shuffle tree, then warps in order
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
  if ((tid & 31) == 0) warp_E[tid >> 5] = e;
  __syncthreads();
  if (tid == 0) {
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kVneThreads / 32; ++w) s += warp_E[w];
    block_E[blockIdx.x] = s;
  }
}

// E = sum of the block partials, each thread over a fixed stride, then a fixed tree.
__global__ void __launch_bounds__(256)
    vne_sum_kernel(const double* __restrict__ block_E, int64_t nb, double* __restrict__ E) {
  __shared__ double part[256];
  double s = 0.0;
  for (int64_t b = threadIdx.x; b < nb; b += 256) s += block_E[b];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *E = part[0];
}

}  // namespace gsdft

using namespace gsdft;

extern "C" size_t gsdft_vne_workspace_size(int64_t n_rep) {
  const int64_t nb = (imax64(n_rep, 1) + kVneThreads - 1) / kVneThreads;
  return ((size_t)nb * sizeof(double) + 255) & ~(size_t)255;
}

extern "C" int gsdft_vne(const double* rec, int64_t n_rep, const double* atoms, int64_t n_atoms,
                         const double* g_E, const int32_t* rep_pos, const int32_t* rep_twin,
                         int64_t n, double* V, double* E, double* sums, int add, void* ws,
                         size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_atoms >= 0 && n >= 0, "bad sizes");
  GSDFT_REQUIRE(E && ws, "null pointer");
  GSDFT_REQUIRE(ws_bytes >= gsdft_vne_workspace_size(n_rep), "workspace too small");
  GSDFT_REQUIRE(n_rep == 0 || rec, "null rec");
  GSDFT_REQUIRE(n_atoms == 0 || atoms, "null atoms");
  GSDFT_REQUIRE(n_atoms == 0 || (reinterpret_cast<uintptr_t>(atoms) & 31) == 0,
                "atoms must be 32-byte aligned");
  GSDFT_REQUIRE(rep_pos == nullptr || n >= n_rep, "list shorter than the representatives");
  cudaStream_t st = (cudaStream_t)stream;
  if (V != nullptr && rep_pos != nullptr && n > 0)
    GSDFT_CUDA(cudaMemsetAsync(V, 0, n * sizeof(double), st));
  const int64_t nb = (imax64(n_rep, 1) + kVneThreads - 1) / kVneThreads;
  double* block_E = static_cast<double*>(ws);
  const double4* at = reinterpret_cast<const double4*>(atoms);
  if (sums != nullptr) {
    vne_kernel<true><<<(unsigned)nb, kVneThreads, kVneDynSmem, st>>>(
        rec, n_rep, at, n_atoms, g_E, rep_pos, rep_twin, V, sums, add, block_E);
  } else {
    vne_kernel<false><<<(unsigned)nb, kVneThreads, kVneDynSmem, st>>>(
        rec, n_rep, at, n_atoms, g_E, rep_pos, rep_twin, V, nullptr, 0, block_E);
  }
  GSDFT_LAUNCHED("vne");
  vne_sum_kernel<<<1, 256, 0, st>>>(block_E, nb, E);
  GSDFT_LAUNCHED("vne_sum");
  return GSDFT_OK;
}

namespace gsdft {
// P_a = sum_o occ_o C[pi_a, o] C[pj_a, o]: one warp per pair, lanes over orbitals, shuffle tree.
__global__ void density_pairs_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                     int64_t n, const double* __restrict__ C,
                                     const double* __restrict__ occ, int64_t n_occ,
                                     double* __restrict__ out) {
  const int64_t a = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (a >= n) return;
  const double* ci = C + (int64_t)pi[a] * n_occ;
  const double* cj = C + (int64_t)pj[a] * n_occ;
  double s = 0.0;
  for (int64_t o = lane; o < n_occ; o += 32) s = fma(occ[o] * ci[o], cj[o], s);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) out[a] = s;
}
}  // namespace gsdft

extern "C" int gsdft_density_pairs(const int32_t* pi, const int32_t* pj, int64_t n,
                                   const double* C_occ, const double* occ, int64_t n_occ,
                                   double* P, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n >= 0 && n_occ >= 0, "bad sizes");
  if (n == 0) return GSDFT_OK;
  GSDFT_REQUIRE(pi && pj && P && (n_occ == 0 || (C_occ && occ)), "null pointer");
  density_pairs_kernel<<<grid_1d(n * 32, 256), 256, 0, (cudaStream_t)stream>>>(pi, pj, n, C_occ,
                                                                               occ, n_occ, P);
  GSDFT_LAUNCHED("density_pairs");
  return GSDFT_OK;
}
