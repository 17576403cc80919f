// Reverse pass of the RI-J energy E = 1/2 gamma^T (V + lam I)^-1 gamma with respect to the splat
// quantities, aux frozen. With dbar_P = g_E d_P and per node
//   f = w det(G)^(-1/2) exp(-t^2 beta d^T A_hat G^-1 d),  G = (beta+t^2) A_hat + t^2 beta I,
//   df/dA_hat = f (-1/2 (beta+t^2) G^-1 - t^4 beta^2 z z^T),   df/dP = 2 t^2 beta f A_hat z,  z = G^-1 d,
// evaluated in the eigenframe of A_hat (where G is diagonal). This avoids the 1/(lam_i - lam_j)
// terms of an eigh VJP. Reference for the quantities being differentiated: gs_dft/coulomb/ri.py
// :126-222 (block, nodes, nodes_bwd), :436-494 (gamma, solve); gs_dft/coulomb/stream.py:203-215
// (pair quantities); gs_dft/coulomb/ri.py:456 (q).
#include "common.cuh"

namespace gsdft {

// Tuning knobs (compile-time): minimum resident CTAs per SM for the reverse kernel's register
// budget, and the size 2^bits of the per-node weighted exp2 table.
#ifndef GSDFT_VJP_MINB
#define GSDFT_VJP_MINB 0
#endif
#if GSDFT_VJP_MINB > 0
#define GSDFT_VJP_BOUNDS __launch_bounds__(kVjpThreads, GSDFT_VJP_MINB)
#else
#define GSDFT_VJP_BOUNDS __launch_bounds__(kVjpThreads)
#endif
#ifndef GSDFT_VJP_EXP2_BITS
#define GSDFT_VJP_EXP2_BITS 6
#endif

constexpr int kAuxRec = 8;        // [beta, -log2e beta, R0, R1, R2, dbar KN, beta^2, 0]
constexpr int kVjpThreads = 128;  // pairs per CTA (one per thread)
constexpr int kVjpTile = 64;      // aux records per staged tile (64 x 64 B)
constexpr int kVjpBits = GSDFT_VJP_EXP2_BITS;
constexpr size_t kVjpDynSmem = sizeof(double) * GSDFT_NQUAD * (1 << kVjpBits);

__global__ void aux_vjp_pack_kernel(const double* __restrict__ beta, const double* __restrict__ R,
                                    const double* __restrict__ KN, const double* __restrict__ d,
                                    const double* __restrict__ gE, int64_t n,
                                    double* __restrict__ out) {
  int64_t P = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (P >= n) return;
  double b = beta[P];
  double g = gE ? gE[0] : 1.0;
  double dP = d ? d[P] : 1.0;
  double* o = out + P * kAuxRec;
  o[0] = b;
  o[1] = -kLog2e * b;
  o[2] = R[3 * P];
  o[3] = R[3 * P + 1];
  o[4] = R[3 * P + 2];
  o[5] = (g * dP) * KN[P];
  o[6] = b * b;
  o[7] = 0.0;
}

// kW: the per-(P,a) weight of the reverse pass is W[P * ldw + a] x (the aux record's dbar KN)
// (E = sum_{P,a} W[P][a] (P|a), as the RI-K gradient needs); without it the weight is dbar_P KN_P.
// Node evaluations of the reverse kernel since the last reset ((aux, pair) units times the nodes
// each evaluated). Read by gsdft_node_evals.
static __device__ unsigned long long g_vjp_node_evals;

// kLR: the node rule is a runtime table (gsdft_lr_node_table: t^2, t^4 and the weighted exp2 rows
// of nq <= GSDFT_NQUAD nodes, e.g. the long-range kernel's segment rule) instead of the half-line
// one; node screening is off for it (its weights are not monotone along the nodes).
template <bool kW, bool kLR = false>
__global__ void GSDFT_VJP_BOUNDS
    j_vjp_kernel(const double* __restrict__ rec, int64_t n_live, const double* __restrict__ auxr,
                 int64_t n_aux, int64_t per_split, double skip2, double* __restrict__ out,
                 const double* __restrict__ Wt, int64_t ldw, const double* __restrict__ nodes,
                 int nq) {
  __shared__ __align__(128) double tile[2][kVjpTile * kAuxRec];
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ double lrt[kLR ? 2 * GSDFT_NQUAD : 1];  // runtime rule: t^2, then t^4
  extern __shared__ __align__(16) double etab[];  // GSDFT_NQUAD x 2^kVjpBits weighted table
  if (kLR) {
    static_assert(!kLR || kVjpBits == 6, "runtime node tables have 64-entry rows");
    for (int k = threadIdx.x; k < nq * 64; k += blockDim.x) etab[k] = nodes[2 * GSDFT_NQUAD + k];
    for (int k = threadIdx.x; k < 2 * GSDFT_NQUAD; k += blockDim.x) lrt[k] = nodes[k];
  } else {
    load_wexp2_tables<kVjpBits>(etab);
  }
  const int64_t a = blockIdx.x * (int64_t)kVjpThreads + threadIdx.x;
  const bool live = a < n_live;
  const int64_t aa = live ? a : 0;
  const bool warp_active = __any_sync(0xffffffffu, live);
  const double* rr = rec + aa * GSDFT_REC_FIELDS;
  double L[3], U[9], Pc[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) L[k] = live ? rr[GSDFT_REC_L0 + k] : 1.0;
#pragma unroll
  for (int k = 0; k < 9; ++k) U[k] = live ? rr[GSDFT_REC_U00 + k] : (k % 4 == 0 ? 1.0 : 0.0);
#pragma unroll
  for (int k = 0; k < 3; ++k) Pc[k] = live ? rr[GSDFT_REC_P0 + k] : 0.0;

  const int64_t P0 = blockIdx.y * per_split;
  const int64_t P1 = imin64(P0 + per_split, n_aux);
  const int64_t naux = P1 > P0 ? P1 - P0 : 0;
  const int ntiles = (int)((naux + kVjpTile - 1) / kVjpTile);
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
  }
  __syncthreads();
  auto issue = [&](int t) {
    int64_t s = P0 + (int64_t)t * kVjpTile;
    int cnt = (int)imin64(kVjpTile, P1 - s);
    uint32_t bytes = (uint32_t)cnt * kAuxRec * sizeof(double);
    fence_proxy_async();
    mbar_expect_tx(&bar[t & 1], bytes);
    bulk_g2s(tile[t & 1], auxr + s * kAuxRec, bytes, &bar[t & 1]);
  };
  if (threadIdx.x == 0) {
    if (ntiles > 0) issue(0);
    if (ntiles > 1) issue(1);
  }

  double SJ = 0.0, SD[3] = {0, 0, 0}, SV[3] = {0, 0, 0}, SZ[6] = {0, 0, 0, 0, 0, 0};
  unsigned long long evals = 0;  // node evaluations per (aux, pair), warp-uniform
  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    ok = __syncthreads_and(mbar_wait(&bar[t & 1], (t >> 1) & 1));
    if (!ok) break;
    const double* tl = tile[t & 1];
    const int cnt = (int)imin64(kVjpTile, P1 - (P0 + (int64_t)t * kVjpTile));
    // a warp with no live pair (the tail of the last pair tile) only takes part in the barriers
    for (int k = 0; warp_active && k < cnt; ++k) {
      const double* ar = tl + k * kAuxRec;
      const double b = ar[0], cP = ar[1], b2 = ar[6];
      double dk = ar[5];
      // aux-major weights: the warp's pairs read consecutive entries of row P
      if constexpr (kW) dk *= Wt[(P0 + (int64_t)t * kVjpTile + k) * ldw + aa];
      const double d0 = ar[2] - Pc[0], d1 = ar[3] - Pc[1], d2 = ar[4] - Pc[2];
      double y[3], m[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        y[c] = U[c] * d0 + U[3 + c] * d1 + U[6 + c] * d2;
        m[c] = (cP * L[c]) * (y[c] * y[c]);
      }
      double cf = 0.0, B[3] = {0, 0, 0}, C[3] = {0, 0, 0}, Z[6] = {0, 0, 0, 0, 0, 0};
      double e0 = 0.0;
      int nodes_done = kLR ? nq : GSDFT_NQUAD;
#pragma unroll
      for (int n = 0; n < GSDFT_NQUAD; ++n) {
        if (kLR && n >= nq) break;
        const double t2 = kLR ? lrt[n] : kQuadT2[n], t4 = kLR ? lrt[GSDFT_NQUAD + n] : kQuadT4[n];
        // Gamma_k = lam_k (beta + t^2) + t^2 beta, rebuilt from two per-node scalars
        const double sn = b + t2, un = t2 * b;
        const double G0 = fma(L[0], sn, un);
        const double G1 = fma(L[1], sn, un);
        const double G2 = fma(L[2], sn, un);
        const double p12 = G1 * G2, p02 = G0 * G2, p01 = G0 * G1;
        const double prod = G0 * p12;
        const double num = fma(m[0], p12, fma(m[1], p02, m[2] * p01));
        const double yy = rsqrt_pos(prod);
        const double inv = yy * yy;
        const double x = num * inv;  // node exponent / t^2, log2 units
        const double f = yy * wexp2<kVjpBits>(x, t2, etab + (n << kVjpBits));
        if (n == 0) e0 = x * t2;
        cf += f;
        const double iG0 = p12 * inv, iG1 = p02 * inv, iG2 = p01 * inv;
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
        // node screening (warp-uniform): every later node is below the last bit of every lane's sums
        if (!kLR && node_check(n) && __all_sync(0xffffffffu, fma(x, t2, -e0) < -skip2)) {
          nodes_done = n + 1;
          break;
        }
      }
      evals += (unsigned long long)nodes_done;
      SJ = fma(dk, cf, SJ);
      const double dkb = dk * b, dkb2 = dk * b2;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        SD[c] = fma(dk, fma(b, B[c], C[c]), SD[c]);
        SV[c] = fma(dkb, y[c] * C[c], SV[c]);
      }
      SZ[0] = fma(dkb2, (y[0] * y[0]) * Z[0], SZ[0]);
      SZ[1] = fma(dkb2, (y[1] * y[1]) * Z[1], SZ[1]);
      SZ[2] = fma(dkb2, (y[2] * y[2]) * Z[2], SZ[2]);
      SZ[3] = fma(dkb2, (y[0] * y[1]) * Z[3], SZ[3]);
      SZ[4] = fma(dkb2, (y[0] * y[2]) * Z[4], SZ[4]);
      SZ[5] = fma(dkb2, (y[1] * y[2]) * Z[5], SZ[5]);
    }
    __syncthreads();
    if (threadIdx.x == 0 && t + 2 < ntiles) issue(t + 2);
  }
  if (live) {
    double* o = out + ((int64_t)blockIdx.y * n_live + a) * GSDFT_VJP_FIELDS;
    const double bad = __longlong_as_double(-1LL);
    o[GSDFT_VJP_SJ] = ok ? SJ : bad;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      o[GSDFT_VJP_SD0 + c] = ok ? SD[c] : bad;
      o[GSDFT_VJP_SV0 + c] = ok ? SV[c] : bad;
    }
#pragma unroll
    for (int c = 0; c < 6; ++c) o[GSDFT_VJP_SZ00 + c] = ok ? SZ[c] : bad;
  }
  const unsigned lanes = __popc(__ballot_sync(0xffffffffu, live));
  if ((threadIdx.x & 31) == 0 && lanes) atomicAdd(&g_vjp_node_evals, evals * lanes);
}

__global__ void sum_vjp_splits_kernel(const double* __restrict__ part, int S, int64_t n,
                                      double* __restrict__ out) {
  int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t tot = n * GSDFT_VJP_FIELDS;
  if (k >= tot) return;
  double acc = 0.0;
  for (int s = 0; s < S; ++s) acc += part[s * tot + k];
  out[k] = acc;
}

// ------------------------------------------------------------------------------------------------
// Chain: per-pair sums -> cotangents of (A_hat, P, KN) -> per-side (A, mu, N) contributions.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void sym6_add_outer(double* s6, double c, const double* u,
                                               const double* v) {
  // s6 += c * sym(u v^T), [xx,yy,zz,xy,xz,yz]
  s6[0] += c * u[0] * v[0];
  s6[1] += c * u[1] * v[1];
  s6[2] += c * u[2] * v[2];
  s6[3] += c * 0.5 * (u[0] * v[1] + u[1] * v[0]);
  s6[4] += c * 0.5 * (u[0] * v[2] + u[2] * v[0]);
  s6[5] += c * 0.5 * (u[1] * v[2] + u[2] * v[1]);
}

__global__ void pair_chain_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                  const double* __restrict__ N, const int32_t* __restrict__ pi,
                                  const int32_t* __restrict__ pj,
                                  const int32_t* __restrict__ live_idx,
                                  const int32_t* __restrict__ twin,
                                  const double* __restrict__ rep_w, int64_t n_live,
                                  const double* __restrict__ rec, const double* __restrict__ sums,
                                  const double* __restrict__ xc, double* __restrict__ side,
                                  double* __restrict__ J, double* __restrict__ jw) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_live) return;
  const double* r = rec + a * GSDFT_REC_FIELDS;
  const int64_t e = live_idx[a];
  const int i = pi[e], j = pj[e];
  const double q = r[GSDFT_REC_Q], kn = r[GSDFT_REC_KN], qk = r[GSDFT_REC_QK];
  double Ab[3][3] = {{0.0, 0.0, 0.0}, {0.0, 0.0, 0.0}, {0.0, 0.0, 0.0}};
  double Pb[3] = {0.0, 0.0, 0.0};
  double Jq = 0.0, KNbar = 0.0;
  if (sums) {
    const double* sm = sums + a * GSDFT_VJP_FIELDS;
    const double SJ = sm[GSDFT_VJP_SJ];
    Jq = kn * SJ;
    KNbar = q * kPref * SJ;
    // eigenframe cotangent of A_hat: M_kl = -qk SZ_kl - 1/2 qk SD_k delta_kl
    double Mm[3][3];
    Mm[0][0] = -qk * sm[GSDFT_VJP_SZ00] - 0.5 * qk * sm[GSDFT_VJP_SD0];
    Mm[1][1] = -qk * sm[GSDFT_VJP_SZ11] - 0.5 * qk * sm[GSDFT_VJP_SD1];
    Mm[2][2] = -qk * sm[GSDFT_VJP_SZ22] - 0.5 * qk * sm[GSDFT_VJP_SD2];
    Mm[0][1] = Mm[1][0] = -qk * sm[GSDFT_VJP_SZ01];
    Mm[0][2] = Mm[2][0] = -qk * sm[GSDFT_VJP_SZ02];
    Mm[1][2] = Mm[2][1] = -qk * sm[GSDFT_VJP_SZ12];
    double U[3][3], Pe[3];
    for (int rr = 0; rr < 3; ++rr)
      for (int c = 0; c < 3; ++c) U[rr][c] = r[GSDFT_REC_U00 + 3 * rr + c];
    for (int k = 0; k < 3; ++k) Pe[k] = 2.0 * qk * r[GSDFT_REC_L0 + k] * sm[GSDFT_VJP_SV0 + k];
    // Abar = U M U^T (symmetric), Pbar = U Pe
    double UM[3][3];
    for (int rr = 0; rr < 3; ++rr)
      for (int c = 0; c < 3; ++c) UM[rr][c] = U[rr][0] * Mm[0][c] + U[rr][1] * Mm[1][c] + U[rr][2] * Mm[2][c];
    for (int rr = 0; rr < 3; ++rr)
      for (int c = 0; c < 3; ++c) Ab[rr][c] = UM[rr][0] * U[c][0] + UM[rr][1] * U[c][1] + UM[rr][2] * U[c][2];
    for (int rr = 0; rr < 3; ++rr) Pb[rr] = U[rr][0] * Pe[0] + U[rr][1] * Pe[1] + U[rr][2] * Pe[2];
  }
  if (xc) {  // cotangents given directly
    const double* x = xc + a * GSDFT_XC_FIELDS;
    Ab[0][0] += x[GSDFT_XC_A00];
    Ab[1][1] += x[GSDFT_XC_A11];
    Ab[2][2] += x[GSDFT_XC_A22];
    Ab[0][1] += x[GSDFT_XC_A01];
    Ab[1][0] += x[GSDFT_XC_A01];
    Ab[0][2] += x[GSDFT_XC_A02];
    Ab[2][0] += x[GSDFT_XC_A02];
    Ab[1][2] += x[GSDFT_XC_A12];
    Ab[2][1] += x[GSDFT_XC_A12];
    for (int k = 0; k < 3; ++k) Pb[k] += x[GSDFT_XC_P0 + k];
    KNbar += x[GSDFT_XC_KN];
    Jq += x[GSDFT_XC_J];
  }
  J[e] = Jq;
  if (twin[a] >= 0) J[twin[a]] = Jq;  // the merged transpose carries the same integral
  jw[a] = Jq * rep_w[a];              // J w, the weight of q_a's gradient

  double Ai[9], Aj[9], mui[3], muj[3];
  for (int k = 0; k < 9; ++k) {
    Ai[k] = A9[9 * (int64_t)i + k];
    Aj[k] = A9[9 * (int64_t)j + k];
  }
  for (int k = 0; k < 3; ++k) {
    mui[k] = mu[3 * (int64_t)i + k];
    muj[k] = mu[3 * (int64_t)j + k];
  }
  double Ah[9], adj[9];
  for (int k = 0; k < 9; ++k) Ah[k] = Ai[k] + Aj[k];
  adj3_rn(Ah, adj);
  const double idet = 1.0 / det3_rn(Ah);
  auto ahinv = [&](const double* x, double* out3) {
    for (int k = 0; k < 3; ++k)
      out3[k] = (adj[3 * k] * x[0] + adj[3 * k + 1] * x[1] + adj[3 * k + 2] * x[2]) * idet;
  };
  const double P[3] = {r[GSDFT_REC_P0], r[GSDFT_REC_P1], r[GSDFT_REC_P2]};
  double v[3];
  ahinv(Pb, v);
  // sym(A_hat bar) = Abar - sym(v P^T)
  double gAi[6] = {Ab[0][0], Ab[1][1], Ab[2][2], Ab[0][1], Ab[0][2], Ab[1][2]};
  sym6_add_outer(gAi, -1.0, v, P);
  double gAj[6];
  for (int k = 0; k < 6; ++k) gAj[k] = gAi[k];
  sym6_add_outer(gAi, 1.0, v, mui);
  sym6_add_outer(gAj, 1.0, v, muj);
  double gmui[3], gmuj[3];
  for (int k = 0; k < 3; ++k) {
    gmui[k] = Ai[k] * v[0] + Ai[3 + k] * v[1] + Ai[6 + k] * v[2];
    gmuj[k] = Aj[k] * v[0] + Aj[3 + k] * v[1] + Aj[6 + k] * v[2];
  }
  // KN = N_i N_j exp(-d^T A_i A_hat^-1 A_j d)
  const double dd[3] = {mui[0] - muj[0], mui[1] - muj[1], mui[2] - muj[2]};
  double Ajd[3], ev[3], fv[3], Hd[3];
  for (int k = 0; k < 3; ++k) Ajd[k] = Aj[3 * k] * dd[0] + Aj[3 * k + 1] * dd[1] + Aj[3 * k + 2] * dd[2];
  ahinv(Ajd, ev);
  for (int k = 0; k < 3; ++k) fv[k] = dd[k] - ev[k];
  for (int k = 0; k < 3; ++k) Hd[k] = Ai[3 * k] * ev[0] + Ai[3 * k + 1] * ev[1] + Ai[3 * k + 2] * ev[2];
  const double K = exp(-(dd[0] * Hd[0] + dd[1] * Hd[1] + dd[2] * Hd[2]));
  const double Ni = N[i], Nj = N[j];
  const double KNv = Ni * Nj * K;
  const double gNi = KNbar * Nj * K, gNj = KNbar * Ni * K;
  const double Qbar = -KNbar * KNv;
  for (int k = 0; k < 3; ++k) {
    gmui[k] += 2.0 * Qbar * Hd[k];
    gmuj[k] -= 2.0 * Qbar * Hd[k];
  }
  sym6_add_outer(gAi, Qbar, ev, ev);
  sym6_add_outer(gAj, Qbar, fv, fv);
  double* o = side + a * GSDFT_SIDE_FIELDS;
  for (int k = 0; k < 6; ++k) {
    o[k] = gAi[k];
    o[10 + k] = gAj[k];
  }
  for (int k = 0; k < 3; ++k) {
    o[6 + k] = gmui[k];
    o[16 + k] = gmuj[k];
  }
  o[9] = gNi;
  o[19] = gNj;
}

// One warp per splat: the i-side contributions of its pi-segment plus the j-side contributions of
// its pj-segment, lanes striding the segments, then a fixed-order warp reduction.
__global__ void splat_reduce_kernel(const double* __restrict__ side,
                                    const int32_t* __restrict__ order_i,
                                    const int64_t* __restrict__ seg_i,
                                    const int32_t* __restrict__ order_j,
                                    const int64_t* __restrict__ seg_j, int64_t M,
                                    double* __restrict__ gA6, double* __restrict__ gmu,
                                    double* __restrict__ gN) {
  int64_t s = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (s >= M) return;
  double acc[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) acc[k] = 0.0;
  for (int64_t e = seg_i[s] + lane; e < seg_i[s + 1]; e += 32) {
    const double* o = side + (int64_t)order_i[e] * GSDFT_SIDE_FIELDS;
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] += o[k];
  }
  for (int64_t e = seg_j[s] + lane; e < seg_j[s + 1]; e += 32) {
    const double* o = side + (int64_t)order_j[e] * GSDFT_SIDE_FIELDS + 10;
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] += o[k];
  }
#pragma unroll
  for (int k = 0; k < 10; ++k)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], off);
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < 6; ++k) gA6[6 * s + k] = acc[k];
#pragma unroll
    for (int k = 0; k < 3; ++k) gmu[3 * s + k] = acc[6 + k];
    gN[s] = acc[9];
  }
}

// g_C[s, o] = occ_o sum_{e in s's by-pi and by-pj segments} (J w)_e C[partner_e, o], partner_e
// the other splat of entry e's representative. One block of kDgWarps warps per splat row.
// Few orbitals (n_occ <= 32): lanes take segment entries, each lane accumulates the whole row in
// registers, then a fixed-order reduction over lanes and warps. Many orbitals: warps take entries,
// lanes cover o in strides of 32, warps' partial rows added in warp order. Deterministic either way.
constexpr int kDgWarps = 8;
constexpr int kDgMaxOcc = 512;   // orbitals per pass of the shared-memory row buffer

template <int NO>
__global__ void __launch_bounds__(kDgWarps * 32)
    density_grad_small_kernel(const int32_t* __restrict__ order_i,
                              const int64_t* __restrict__ seg_i,
                              const int32_t* __restrict__ partner_i,
                              const int32_t* __restrict__ order_j,
                              const int64_t* __restrict__ seg_j,
                              const int32_t* __restrict__ partner_j, const double* __restrict__ jw,
                              const double* __restrict__ C, const double* __restrict__ occ,
                              int n_occ, double* __restrict__ gC) {
  __shared__ double part[kDgWarps][NO];
  const int64_t s = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = seg_i[s], ni = seg_i[s + 1] - i0;
  const int64_t j0 = seg_j[s], nj = seg_j[s + 1] - j0;
  double acc[NO];
#pragma unroll
  for (int o = 0; o < NO; ++o) acc[o] = 0.0;
  for (int64_t e = threadIdx.x; e < ni + nj; e += kDgWarps * 32) {
    const bool is_i = e < ni;
    const int64_t k = is_i ? i0 + e : j0 + (e - ni);
    const double w = jw[is_i ? order_i[k] : order_j[k]];
    const double* crow = C + (int64_t)(is_i ? partner_i[k] : partner_j[k]) * n_occ;
#pragma unroll
    for (int o = 0; o < NO; ++o)
      if (o < n_occ) acc[o] = fma(w, crow[o], acc[o]);
  }
#pragma unroll
  for (int o = 0; o < NO; ++o) {
    double v = acc[o];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) part[warp][o] = v;
  }
  __syncthreads();
  for (int o = threadIdx.x; o < n_occ; o += blockDim.x) {
    double sum = 0.0;
#pragma unroll
    for (int w = 0; w < kDgWarps; ++w) sum += part[w][o];
    gC[s * n_occ + o] = occ[o] * sum;
  }
}

__global__ void __launch_bounds__(kDgWarps * 32)
    density_grad_kernel(const int32_t* __restrict__ order_i, const int64_t* __restrict__ seg_i,
                        const int32_t* __restrict__ partner_i,
                        const int32_t* __restrict__ order_j, const int64_t* __restrict__ seg_j,
                        const int32_t* __restrict__ partner_j, const double* __restrict__ jw,
                        const double* __restrict__ C, const double* __restrict__ occ,
                        int64_t n_occ, double* __restrict__ gC) {
  __shared__ double part[kDgWarps][kDgMaxOcc / 32][32];
  const int64_t s = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = seg_i[s], ni = seg_i[s + 1] - i0;
  const int64_t j0 = seg_j[s], nj = seg_j[s + 1] - j0;
  for (int64_t ob = 0; ob < n_occ; ob += kDgMaxOcc) {
    const int nchunk = (int)((imin64(kDgMaxOcc, n_occ - ob) + 31) / 32);
    double acc[kDgMaxOcc / 32];
#pragma unroll
    for (int c = 0; c < kDgMaxOcc / 32; ++c) acc[c] = 0.0;
    for (int64_t e = warp; e < ni + nj; e += kDgWarps) {
      const bool is_i = e < ni;
      const int64_t k = is_i ? i0 + e : j0 + (e - ni);
      const double w = jw[is_i ? order_i[k] : order_j[k]];
      const double* crow = C + (int64_t)(is_i ? partner_i[k] : partner_j[k]) * n_occ + ob;
#pragma unroll
      for (int c = 0; c < kDgMaxOcc / 32; ++c) {
        const int64_t o = (int64_t)c * 32 + lane;
        if (c < nchunk && ob + o < n_occ) acc[c] = fma(w, crow[o], acc[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < kDgMaxOcc / 32; ++c)
      if (c < nchunk) part[warp][c][lane] = acc[c];
    __syncthreads();
    for (int64_t o = threadIdx.x; o < imin64(kDgMaxOcc, n_occ - ob); o += blockDim.x) {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kDgWarps; ++w) sum += part[w][o >> 5][o & 31];
      gC[s * n_occ + ob + o] = occ[ob + o] * sum;
    }
    __syncthreads();
  }
}

// Aux splits: pair tiles x S CTAs filling whole waves of resident CTAs (S <= 8, since the partial
// sums take S x n_live x 13 doubles). The occupancy query runs once per template (a thread-safe
// static).
template <bool kW, bool kLR = false>
static int vjp_splits(int64_t n_live, int64_t n_aux) {
  static const int per_sm = [] {
    int v = 0;
    cudaFuncSetAttribute(j_vjp_kernel<kW, kLR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kVjpDynSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, j_vjp_kernel<kW, kLR>, kVjpThreads,
                                                  kVjpDynSmem);
    return v > 0 ? v : 1;
  }();
  int64_t tiles = (n_live + kVjpThreads - 1) / kVjpThreads;
  int64_t cap = (int64_t)device_sms() * per_sm;
  int64_t max_s = imin64(8, imax64(1, n_aux / kVjpTile));
  return best_splits(tiles, cap, max_s);
}

int node_evals_vjp(unsigned long long* out, int clear) {
  GSDFT_CUDA(cudaMemcpyFromSymbol(out, g_vjp_node_evals, sizeof(unsigned long long)));
  if (clear) {
    unsigned long long z = 0;
    GSDFT_CUDA(cudaMemcpyToSymbol(g_vjp_node_evals, &z, sizeof(z)));
  }
  return GSDFT_OK;
}

int device_status_vjp(int* out, int clear) {
  GSDFT_CUDA(cudaMemcpyFromSymbol(out, g_device_status, sizeof(int)));
  if (clear) {
    int z = 0;
    GSDFT_CUDA(cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)));
  }
  return GSDFT_OK;
}

}  // namespace gsdft

using namespace gsdft;

namespace gsdft {
template <bool kW>
static size_t vjp_workspace_size(int64_t n_live, int64_t n_aux) {
  int S = vjp_splits<kW>(n_live, n_aux);
  if constexpr (kW) S = (int)imax64(S, vjp_splits<kW, true>(n_live, n_aux));  // either rule
  Sizer z;
  z.take<double>((size_t)n_aux * kAuxRec);
  if (S > 1) z.take<double>((size_t)S * n_live * GSDFT_VJP_FIELDS);
  return z.off + 256;
}

template <bool kW, bool kLR = false>
static int vjp_run(const double* rec, int64_t n_live, const double* beta, const double* R,
                   const double* KN, const double* d, const double* g_E, const double* Wt,
                   int64_t ldw, int64_t n_aux, double* sums, void* ws, size_t ws_bytes,
                   cudaStream_t st, const double* nodes = nullptr, int nq = 0) {
  int S = vjp_splits<kW, kLR>(n_live, n_aux);
  Carver c(ws, ws_bytes);
  double* auxr = c.take<double>((size_t)n_aux * kAuxRec);
  double* part = S > 1 ? c.take<double>((size_t)S * n_live * GSDFT_VJP_FIELDS) : sums;
  if (!c.ok) return fail(GSDFT_ERR_ARG, "vjp workspace too small (%zu < %zu)", ws_bytes, c.off);
  aux_vjp_pack_kernel<<<grid_1d(n_aux, 256), 256, 0, st>>>(beta, R, KN, d, g_E, n_aux, auxr);
  GSDFT_LAUNCHED("aux_vjp_pack");
  int64_t per_split = (n_aux + S - 1) / S;
  dim3 grid((unsigned)((n_live + kVjpThreads - 1) / kVjpThreads), (unsigned)S);
  j_vjp_kernel<kW, kLR><<<grid, kVjpThreads, kVjpDynSmem, st>>>(
      rec, n_live, auxr, n_aux, per_split, node_skip_threshold(), part, Wt, ldw, nodes, nq);
  GSDFT_LAUNCHED("j_vjp");
  if (S > 1) {
    sum_vjp_splits_kernel<<<grid_1d(n_live * GSDFT_VJP_FIELDS, 256), 256, 0, st>>>(part, S, n_live,
                                                                                   sums);
    GSDFT_LAUNCHED("sum_vjp_splits");
  }
  return GSDFT_OK;
}
}  // namespace gsdft

extern "C" size_t gsdft_j_vjp_workspace_size(int64_t n_live, int64_t n_aux) {
  return vjp_workspace_size<false>(n_live, n_aux);
}

extern "C" int gsdft_j_vjp(const double* rec, int64_t n_live, const double* beta, const double* R,
                           const double* KN, const double* d, const double* g_E, int64_t n_aux,
                           double* sums, void* ws, size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_live >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31), "bad sizes");
  if (n_live == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && beta && R && KN && d && sums, "null pointer");
  return vjp_run<false>(rec, n_live, beta, R, KN, d, g_E, nullptr, 0, n_aux, sums, ws, ws_bytes,
                        (cudaStream_t)stream);
}

extern "C" size_t gsdft_j_vjp_weighted_workspace_size(int64_t n_live, int64_t n_aux) {
  return vjp_workspace_size<true>(n_live, n_aux);
}

extern "C" int gsdft_j_vjp_weighted(const double* rec, int64_t n_live, const double* beta,
                                    const double* R, const double* KN, const double* Wt,
                                    int64_t ldw, int64_t n_aux, const double* nodes, int n_nodes,
                                    double* sums, void* ws, size_t ws_bytes,
                                    gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_live >= 0 && n_aux > 0 && n_aux < (int64_t(1) << 31) && ldw >= n_live,
                "bad sizes");
  GSDFT_REQUIRE(!nodes || (n_nodes >= 1 && n_nodes <= GSDFT_NQUAD), "bad node count");
  if (n_live == 0) return GSDFT_OK;
  GSDFT_REQUIRE(rec && beta && R && KN && Wt && sums, "null pointer");
  if (nodes)
    return vjp_run<true, true>(rec, n_live, beta, R, KN, nullptr, nullptr, Wt, ldw, n_aux, sums,
                               ws, ws_bytes, (cudaStream_t)stream, nodes, n_nodes);
  return vjp_run<true>(rec, n_live, beta, R, KN, nullptr, nullptr, Wt, ldw, n_aux, sums, ws,
                       ws_bytes, (cudaStream_t)stream);
}

extern "C" int gsdft_pair_chain(const double* A9, const double* mu, const double* N, int64_t M,
                                const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                                const int32_t* rep_twin, const double* rep_w, int64_t n_rep,
                                int64_t n, const double* rec, const double* sums,
                                const double* xc, double* side, double* J, double* jw,
                                gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_rep >= 0 && n >= n_rep, "bad sizes");
  cudaStream_t st = (cudaStream_t)stream;
  if (n > 0) {
    GSDFT_REQUIRE(J, "null J");
    GSDFT_CUDA(cudaMemsetAsync(J, 0, n * sizeof(double), st));
  }
  if (n_rep == 0) return GSDFT_OK;
  GSDFT_REQUIRE(A9 && mu && N && pi && pj && rep_pos && rep_twin && rep_w && rec && side && jw,
                "null pointer");
  pair_chain_kernel<<<grid_1d(n_rep, 128), 128, 0, st>>>(A9, mu, N, pi, pj, rep_pos, rep_twin,
                                                         rep_w, n_rep, rec, sums, xc, side, J, jw);
  GSDFT_LAUNCHED("pair_chain");
  return GSDFT_OK;
}

extern "C" int gsdft_splat_reduce(const double* side, const int32_t* order_i, const int64_t* seg_i,
                                  const int32_t* order_j, const int64_t* seg_j, int64_t n_live,
                                  int64_t M, double* gA6, double* gmu, double* gN,
                                  gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_live >= 0, "bad sizes");
  GSDFT_REQUIRE(seg_i && seg_j && gA6 && gmu && gN, "null pointer");
  GSDFT_REQUIRE(n_live == 0 || (side && order_i && order_j), "null pointer");
  splat_reduce_kernel<<<grid_1d(M * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      side, order_i, seg_i, order_j, seg_j, M, gA6, gmu, gN);
  GSDFT_LAUNCHED("splat_reduce");
  return GSDFT_OK;
}

extern "C" int gsdft_density_grad(const int32_t* order_i, const int64_t* seg_i,
                                  const int32_t* partner_i, const int32_t* order_j,
                                  const int64_t* seg_j, const int32_t* partner_j, const double* jw,
                                  int64_t n_rep, int64_t M, const double* C_occ, const double* occ,
                                  int64_t n_occ, double* g_C, gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_rep >= 0 && n_occ >= 0, "bad sizes");
  if (n_occ == 0) return GSDFT_OK;
  GSDFT_REQUIRE(seg_i && seg_j && C_occ && occ && g_C, "null pointer");
  GSDFT_REQUIRE(n_rep == 0 || (order_i && partner_i && order_j && partner_j && jw), "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (n_occ <= 16) {
    density_grad_small_kernel<16><<<(unsigned)M, kDgWarps * 32, 0, st>>>(
        order_i, seg_i, partner_i, order_j, seg_j, partner_j, jw, C_occ, occ, (int)n_occ, g_C);
  } else if (n_occ <= 32) {
    density_grad_small_kernel<32><<<(unsigned)M, kDgWarps * 32, 0, st>>>(
        order_i, seg_i, partner_i, order_j, seg_j, partner_j, jw, C_occ, occ, (int)n_occ, g_C);
  } else {
    density_grad_kernel<<<(unsigned)M, kDgWarps * 32, 0, st>>>(
        order_i, seg_i, partner_i, order_j, seg_j, partner_j, jw, C_occ, occ, n_occ, g_C);
  }
  GSDFT_LAUNCHED("density_grad");
  return GSDFT_OK;
}
