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
