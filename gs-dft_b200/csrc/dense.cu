// Dense FP64 linear algebra on the tensor cores (DMMA): a tiled GEMM built on mma.sync f64, and on it
// the refresh-time factorisations of the aux metric — the blocked Cholesky of V + lam I
// (gs_dft/coulomb/ri.py:243-264), the inverse of its factor for the per-step solve, and the blocked
// triangular solves of a one-shot solve (gs_dft/coulomb/ri.py:472-482). No library is called.
//
// GEMM: C = alpha op(A) op(B) + beta C, row-major FP64, op = identity or transpose. A block of 128
// threads computes a 64 x 64 tile of C; each of its four warps a 32 x 32 sub-tile as 2 x 4
// m16n8k4 DMMA tiles (32 FP64 accumulators per thread). K advances in stages of 16: the next
// stage's operand tiles are loaded into registers while the tensor cores work on the current one in
// shared memory (rows padded so that the fragment reads are free of bank conflicts). Tiles at the
// matrix edges are zero-filled; an operand can be declared lower-triangular (entries above its
// diagonal read as zero), and the output restricted to tiles on or below the diagonal (for the
// symmetric rank-k update of the Cholesky). A batch index (gridDim.z) walks equally spaced
// sub-problems of one matrix, the last of which may be smaller.
#include "common.cuh"

namespace gsdft {

constexpr int kGT = 64;    // output tile (rows and columns) per block
constexpr int kGK = 16;    // K per shared-memory stage
constexpr int kGPad = 4;   // row padding (doubles) of the shared tiles

struct GemmArgs {
  int64_t M, N, K;
  double alpha, beta;
  const double* A;
  int64_t lda;
  const double* B;
  int64_t ldb;
  double* C;
  int64_t ldc;
  // batch z: operands offset by z * s{a,b,c} elements; sizes min(M, Mclip - z Mstep) (same for N, K)
  int64_t sa, sb, sc;
  int64_t Mclip, Mstep, Nclip, Nstep, Kclip, Kstep;
};

__device__ __forceinline__ void dmma_m16n8k4(double (&d)[4], double a0, double a1, double b0) {
  asm("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
      : "d"(a0), "d"(a1), "d"(b0));
}

// kTA / kTB: A is stored K x M / B is stored N x K (op = transpose). kTriA / kTriB: the stored
// operand is lower-triangular (entries above its diagonal read as zero). kLower: only output tiles on
// or below the diagonal are computed.
template <bool kTA, bool kTB, bool kTriA, bool kTriB, bool kLower>
__global__ void __launch_bounds__(128) dmma_gemm_kernel(GemmArgs g) {
  const int64_t z = blockIdx.z;
  const int64_t M = imin64(g.M, g.Mclip - z * g.Mstep);
  const int64_t N = imin64(g.N, g.Nclip - z * g.Nstep);
  const int64_t K = imin64(g.K, g.Kclip - z * g.Kstep);
  const int64_t m0 = (int64_t)blockIdx.y * kGT, n0 = (int64_t)blockIdx.x * kGT;
  if (m0 >= M || n0 >= N) return;
  if (kLower && n0 > m0) return;
  const double* __restrict__ A = g.A + z * g.sa;
  const double* __restrict__ B = g.B + z * g.sb;
  double* __restrict__ C = g.C + z * g.sc;

  // shared tiles: A as [m][k] (kTA: [k][m]), B as [k][n] (kTB: [n][k])
  __shared__ double As[kTA ? kGK : kGT][(kTA ? kGT : kGK) + kGPad];
  __shared__ double Bs[kTB ? kGT : kGK][(kTB ? kGK : kGT) + kGPad];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
  // global -> register mapping: 8 consecutive elements of one stored row per thread
  const int ar = kTA ? (tid >> 3) : (tid >> 1), ac = kTA ? (tid & 7) * 8 : (tid & 1) * 8;
  const int br = kTB ? (tid >> 1) : (tid >> 3), bc = kTB ? (tid & 1) * 8 : (tid & 7) * 8;
  double ra[8], rb[8];

  auto load = [&](int64_t k0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // A stored (row, col): !kTA (m, k), kTA (k, m)
      const int64_t r = kTA ? k0 + ar : m0 + ar, c = kTA ? m0 + ac + e : k0 + ac + e;
      const bool in = kTA ? (r < K && c < M) : (r < M && c < K);
      ra[e] = (in && !(kTriA && c > r)) ? A[r * g.lda + c] : 0.0;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // B stored (row, col): !kTB (k, n), kTB (n, k)
      const int64_t r = kTB ? n0 + br : k0 + br, c = kTB ? k0 + bc + e : n0 + bc + e;
      const bool in = kTB ? (r < N && c < K) : (r < K && c < N);
      rb[e] = (in && !(kTriB && c > r)) ? B[r * g.ldb + c] : 0.0;
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int e = 0; e < 8; ++e) As[ar][ac + e] = ra[e];
#pragma unroll
    for (int e = 0; e < 8; ++e) Bs[br][bc + e] = rb[e];
  };

  double acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.0;

  load(0);
  store();
  __syncthreads();
  for (int64_t k0 = 0; k0 < K; k0 += kGK) {
    const bool more = k0 + kGK < K;
    if (more) load(k0 + kGK);
#pragma unroll
    for (int kk = 0; kk < kGK; kk += 4) {
      double a0[2], a1[2], b[4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int m = wm + mi * 16 + gq;
        a0[mi] = kTA ? As[kk + tq][m] : As[m][kk + tq];
        a1[mi] = kTA ? As[kk + tq][m + 8] : As[m + 8][kk + tq];
      }
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const int n = wn + ni * 8 + gq;
        b[ni] = kTB ? Bs[n][kk + tq] : Bs[kk + tq][n];
      }
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) dmma_m16n8k4(acc[mi][ni], a0[mi], a1[mi], b[ni]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }

#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t row = m0 + wm + mi * 16 + gq + (r >> 1) * 8;
        const int64_t col = n0 + wn + ni * 8 + 2 * tq + (r & 1);
        if (row < M && col < N) {
          double* p = C + row * g.ldc + col;
          const double v = g.alpha * acc[mi][ni][r];
          *p = g.beta == 0.0 ? v : fma(g.beta, *p, v);
        }
      }
}

// ------------------------------------------------------------------------------------------------
// The same GEMM for large, 16-byte-aligned operands: a 128 x 64 tile of C per block of 256 threads
// (eight warps of 32 x 32, 2 x 4 DMMA tiles each), the operand tiles of three K stages of 16 in
// flight at once through cp.async (16-byte copies straight into shared memory, no register
// staging), one barrier per stage. A copy's source size zero-fills what lies beyond the matrix edge
// or above a triangular operand's diagonal, so edges and triangles need no second path.
// ------------------------------------------------------------------------------------------------
#ifndef GSDFT_GEMM_V2
#define GSDFT_GEMM_V2 1
#endif
constexpr int kBM = 128, kBN = 64, kBK = 16, kStages = 3, kV2Threads = 256;

template <bool kTA>
__host__ __device__ constexpr int v2_a_cols() { return (kTA ? kBM : kBK) + 4; }
template <bool kTA>
__host__ __device__ constexpr int v2_a_size() { return (kTA ? kBK : kBM) * v2_a_cols<kTA>(); }
template <bool kTB>
__host__ __device__ constexpr int v2_b_cols() { return (kTB ? kBK : kBN) + 4; }
template <bool kTB>
__host__ __device__ constexpr int v2_b_size() { return (kTB ? kBN : kBK) * v2_b_cols<kTB>(); }
template <bool kTA, bool kTB>
__host__ __device__ constexpr size_t v2_smem() {
  return sizeof(double) * kStages * (v2_a_size<kTA>() + v2_b_size<kTB>());
}

__device__ __forceinline__ void cp_async16(double* dst, const double* src, int bytes) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// One 16-byte chunk (two doubles from (gr, gc) on) of a stored operand with rows x cols elements:
// how many of its doubles exist (0, 1, 2), after the edge and, for a lower-triangular operand, the
// diagonal (entries with column > row read as zero).
template <bool kTri>
__device__ __forceinline__ int chunk_doubles(int64_t gr, int64_t gc, int64_t rows, int64_t cols) {
  if (gr >= rows) return 0;
  int64_t v = imin64(2, imax64(0, cols - gc));
  if (kTri) v = imin64(v, imax64(0, gr - gc + 1));
  return (int)v;
}

template <bool kTA, bool kTB, bool kTriA, bool kTriB, bool kLower>
__global__ void __launch_bounds__(kV2Threads) dmma_gemm_v2_kernel(GemmArgs g) {
  const int64_t z = blockIdx.z;
  const int64_t M = imin64(g.M, g.Mclip - z * g.Mstep);
  const int64_t N = imin64(g.N, g.Nclip - z * g.Nstep);
  const int64_t K = imin64(g.K, g.Kclip - z * g.Kstep);
  const int64_t m0 = (int64_t)blockIdx.y * kBM, n0 = (int64_t)blockIdx.x * kBN;
  if (m0 >= M || n0 >= N) return;
  if (kLower && n0 > m0 + kGT) return;  // both 64-row halves lie above the block diagonal
  const double* __restrict__ A = g.A + z * g.sa;
  const double* __restrict__ B = g.B + z * g.sb;
  double* __restrict__ C = g.C + z * g.sc;

  extern __shared__ __align__(16) double sm2[];
  constexpr int AC = v2_a_cols<kTA>(), AS = v2_a_size<kTA>();
  constexpr int BC = v2_b_cols<kTB>(), BS = v2_b_size<kTB>();
  double* As = sm2;
  double* Bs = sm2 + kStages * AS;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
  const int64_t arows = kTA ? K : M, acols = kTA ? M : K;
  const int64_t brows = kTB ? N : K, bcols = kTB ? K : N;

  auto issue = [&](int stage, int64_t k0) {
    double* as = As + stage * AS;
    double* bs = Bs + stage * BS;
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // A: 1024 chunks of the 128 x 16 (or 16 x 128) tile
      const int id = tid + q * kV2Threads;
      const int r = kTA ? id >> 6 : id >> 3, c = kTA ? (id & 63) * 2 : (id & 7) * 2;
      const int64_t gr = kTA ? k0 + r : m0 + r, gc = kTA ? m0 + c : k0 + c;
      const int nd = chunk_doubles<kTriA>(gr, gc, arows, acols);
      cp_async16(as + r * AC + c, nd ? A + gr * g.lda + gc : A, nd * 8);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {  // B: 512 chunks of the 16 x 64 (or 64 x 16) tile
      const int id = tid + q * kV2Threads;
      const int r = kTB ? id >> 3 : id >> 5, c = kTB ? (id & 7) * 2 : (id & 31) * 2;
      const int64_t gr = kTB ? n0 + r : k0 + r, gc = kTB ? k0 + c : n0 + c;
      const int nd = chunk_doubles<kTriB>(gr, gc, brows, bcols);
      cp_async16(bs + r * BC + c, nd ? B + gr * g.ldb + gc : B, nd * 8);
    }
  };

  double acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.0;

  const int64_t KT = (K + kBK - 1) / kBK;
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < KT) issue(s, (int64_t)s * kBK);
    cp_async_commit();
  }
  for (int64_t kt = 0; kt < KT; ++kt) {
    cp_async_wait<kStages - 2>();  // this thread's copies of stage kt have landed
    __syncthreads();               // everyone's have; stage kt - 1 is no longer read
    const int64_t nk = kt + kStages - 1;
    if (nk < KT) issue((int)(nk % kStages), nk * kBK);
    cp_async_commit();
    const double* as = As + (kt % kStages) * AS;
    const double* bs = Bs + (kt % kStages) * BS;
#pragma unroll
    for (int kk = 0; kk < kBK; kk += 4) {
      double a0[2], a1[2], b[4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int m = wm + mi * 16 + gq;
        a0[mi] = kTA ? as[(kk + tq) * AC + m] : as[m * AC + kk + tq];
        a1[mi] = kTA ? as[(kk + tq) * AC + m + 8] : as[(m + 8) * AC + kk + tq];
      }
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const int n = wn + ni * 8 + gq;
        b[ni] = kTB ? bs[n * BC + kk + tq] : bs[(kk + tq) * BC + n];
      }
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) dmma_m16n8k4(acc[mi][ni], a0[mi], a1[mi], b[ni]);
    }
  }
  cp_async_wait<0>();

#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t row = m0 + wm + mi * 16 + gq + (r >> 1) * 8;
        const int64_t col = n0 + wn + ni * 8 + 2 * tq + (r & 1);
        // kLower: the 64 x 64 blocks on or below the block diagonal, as the 64-tile kernel writes
        if (row < M && col < N && !(kLower && n0 > (row / kGT) * kGT)) {
          double* p = C + row * g.ldc + col;
          const double v = g.alpha * acc[mi][ni][r];
          *p = g.beta == 0.0 ? v : fma(g.beta, *p, v);
        }
      }
}

// Host launcher: picks the instantiation; grid (N tiles, M tiles, batch). Large products whose
// operands are 16-byte aligned (bases, leading dimensions and batch strides even) take the
// pipelined kernel.
template <bool kTA, bool kTB, bool kTriA, bool kTriB, bool kLower>
static int gemm_launch(const GemmArgs& g, int64_t batch, cudaStream_t st) {
  if (g.M <= 0 || g.N <= 0 || batch <= 0) return GSDFT_OK;
  const bool aligned = (reinterpret_cast<uintptr_t>(g.A) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(g.B) & 15) == 0 && g.lda % 2 == 0 &&
                       g.ldb % 2 == 0 && g.sa % 2 == 0 && g.sb % 2 == 0;
  if (GSDFT_GEMM_V2 && aligned && g.M >= kBM && g.N >= kBN && g.K >= kBK) {
    constexpr size_t smem = v2_smem<kTA, kTB>();
    static const bool attr = [] {
      return cudaFuncSetAttribute(dmma_gemm_v2_kernel<kTA, kTB, kTriA, kTriB, kLower>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem) == cudaSuccess;
    }();
    GSDFT_REQUIRE(attr, "gemm: shared-memory attribute refused");
    dim3 grid((unsigned)((g.N + kBN - 1) / kBN), (unsigned)((g.M + kBM - 1) / kBM),
              (unsigned)batch);
    GSDFT_REQUIRE(grid.y <= 65535 && grid.z <= 65535, "gemm grid too large");
    dmma_gemm_v2_kernel<kTA, kTB, kTriA, kTriB, kLower><<<grid, kV2Threads, smem, st>>>(g);
    GSDFT_LAUNCHED("dmma_gemm");
    return GSDFT_OK;
  }
  dim3 grid((unsigned)((g.N + kGT - 1) / kGT), (unsigned)((g.M + kGT - 1) / kGT),
            (unsigned)batch);
  GSDFT_REQUIRE(grid.y <= 65535 && grid.z <= 65535, "gemm grid too large");
  dmma_gemm_kernel<kTA, kTB, kTriA, kTriB, kLower><<<grid, 128, 0, st>>>(g);
  GSDFT_LAUNCHED("dmma_gemm");
  return GSDFT_OK;
}

static GemmArgs gemm_args(int64_t M, int64_t N, int64_t K, double alpha, const double* A,
                          int64_t lda, const double* B, int64_t ldb, double beta, double* C,
                          int64_t ldc) {
  GemmArgs g;
  g.M = M, g.N = N, g.K = K, g.alpha = alpha, g.beta = beta;
  g.A = A, g.lda = lda, g.B = B, g.ldb = ldb, g.C = C, g.ldc = ldc;
  g.sa = g.sb = g.sc = 0;
  g.Mclip = M, g.Nclip = N, g.Kclip = K;
  g.Mstep = g.Nstep = g.Kstep = 0;
  return g;
}

// General entry for the other translation units: op(A) lower-triangular when tri_a.
int gemm_dmma(bool ta, bool tb, bool tri_a, int64_t M, int64_t N, int64_t K, double alpha,
              const double* A, int64_t lda, const double* B, int64_t ldb, double beta, double* C,
              int64_t ldc, cudaStream_t st) {
  const GemmArgs g = gemm_args(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  if (tri_a) {
    if (ta && tb) return gemm_launch<true, true, true, false, false>(g, 1, st);
    if (ta) return gemm_launch<true, false, true, false, false>(g, 1, st);
    if (tb) return gemm_launch<false, true, true, false, false>(g, 1, st);
    return gemm_launch<false, false, true, false, false>(g, 1, st);
  }
  if (ta && tb) return gemm_launch<true, true, false, false, false>(g, 1, st);
  if (ta) return gemm_launch<true, false, false, false, false>(g, 1, st);
  if (tb) return gemm_launch<false, true, false, false, false>(g, 1, st);
  return gemm_launch<false, false, false, false, false>(g, 1, st);
}

// C = alpha sum_s partial_s + beta C over S split-K partial products, in split order.
__global__ void splitk_sum_kernel(const double* __restrict__ part, int S, int64_t M, int64_t N,
                                  double alpha, double beta, double* __restrict__ C, int64_t ldc) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= M * N) return;
  double acc = 0.0;
  for (int s = 0; s < S; ++s) acc += part[(int64_t)s * M * N + k];
  double* p = C + (k / N) * ldc + (k % N);
  *p = beta == 0.0 ? alpha * acc : fma(beta, *p, alpha * acc);
}

// Split-K count for a GEMM whose M x N tiles cannot fill the device, and its partial buffer size
// (doubles): the K range is cut into S chunks (multiples of 16) computed as a batch, then summed
// in a fixed order.
int splitk_count(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ((M + kGT - 1) / kGT) * ((N + kGT - 1) / kGT);
  const int64_t want = (2 * (int64_t)device_sms() + tiles - 1) / tiles;  // ~2 blocks per SM
  const int64_t by_k = imax64(1, K / (4 * kGK));                          // >= 4 stages per chunk
  return (int)imax64(1, imin64(imin64(want, by_k), 64));
}

// C = alpha op(A) B + beta C with op(A) = A^T when ta (A stored K x M), B stored K x N, split over K.
int gemm_dmma_splitk(bool ta, int64_t M, int64_t N, int64_t K, double alpha, const double* A,
                     int64_t lda, const double* B, int64_t ldb, double beta, double* C, int64_t ldc,
                     double* part, int S, cudaStream_t st) {
  if (S <= 1) return gemm_dmma(ta, false, false, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, st);
  int64_t chunk = (K + S - 1) / S;
  chunk = (chunk + kGK - 1) / kGK * kGK;
  const int64_t nb = (K + chunk - 1) / chunk;
  GemmArgs g = gemm_args(M, N, chunk, 1.0, A, lda, B, ldb, 0.0, part, N);
  g.sa = ta ? chunk * lda : chunk;
  g.sb = chunk * ldb;
  g.sc = M * N;
  g.Kclip = K, g.Kstep = chunk;
  const int rc = ta ? gemm_launch<true, false, false, false, false>(g, nb, st)
                    : gemm_launch<false, false, false, false, false>(g, nb, st);
  if (rc) return rc;
  splitk_sum_kernel<<<grid_1d(M * N, 256), 256, 0, st>>>(part, (int)nb, M, N, alpha, beta, C, ldc);
  GSDFT_LAUNCHED("splitk_sum");
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// Cholesky, right-looking in panels of 64: factor the diagonal block in shared memory (and invert
// it), the panel below as a GEMM with the inverse's transpose, and the trailing lower triangle
// updated by a rank-64 DMMA GEMM.
// ------------------------------------------------------------------------------------------------
constexpr int kNb = 64;

// The kb x kb diagonal block at A (lower part) factored in place, A = L L^T (unblocked,
// right-looking), its strict upper part zeroed, and inv(L) written to Dinv (64 x 64, leading
// dimension 64, zero above the diagonal). A non-positive pivot records its global index + 1 in
// *info (first one only) and continues with pivot 1.
__global__ void __launch_bounds__(256) potf2_inv_kernel(double* A, int64_t lda, int kb,
                                                        double* Dinv, int* info, int64_t k0) {
  // s: the factor in the lower triangle, then inv(L) transposed into the strict upper one
  // (inv(L)[i][c] at s[c][i]) with its diagonal in xd
  __shared__ double s[kNb][kNb + 1];
  __shared__ double xd[kNb];
  const int tid = threadIdx.x;
  for (int idx = tid; idx < kNb * kNb; idx += blockDim.x) {
    const int i = idx / kNb, j = idx % kNb;
    s[i][j] = (i < kb && j <= i) ? A[(int64_t)i * lda + j] : (i == j ? 1.0 : 0.0);
  }
  __syncthreads();
  for (int j = 0; j < kb; ++j) {
    if (tid == 0) {
      double d = s[j][j];
      if (!(d > 0.0)) {
        if (*info == 0) *info = (int)(k0 + j + 1);
        d = 1.0;
      }
      s[j][j] = sqrt(d);
    }
    __syncthreads();
    const double djj = s[j][j];
    for (int i = j + 1 + tid; i < kb; i += blockDim.x) s[i][j] = s[i][j] / djj;
    __syncthreads();
    const int w = kb - j - 1;
    for (int idx = tid; idx < w * w; idx += blockDim.x) {
      const int i = j + 1 + idx / w, l = j + 1 + idx % w;
      if (l <= i) s[i][l] = fma(-s[i][j], s[l][j], s[i][l]);
    }
    __syncthreads();
  }
  // inverse of the lower triangle, one column c per thread (forward substitution on e_c); thread c
  // writes only row c of the upper triangle and reads the factor's lower triangle
  if (tid < kb) {
    const int c = tid;
    xd[c] = 1.0 / s[c][c];
    for (int i = c + 1; i < kb; ++i) {
      double acc = s[i][c] * xd[c];
      for (int l = c + 1; l < i; ++l) acc = fma(s[i][l], s[c][l], acc);
      s[c][i] = -acc / s[i][i];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < kNb * kNb; idx += blockDim.x) {
    const int i = idx / kNb, j = idx % kNb;
    if (i < kb && j < kb) A[(int64_t)i * lda + j] = j <= i ? s[i][j] : 0.0;
    Dinv[idx] = (i < kb && j <= i) ? (i == j ? xd[i] : s[j][i]) : 0.0;
  }
}

__global__ void shift_diag_kernel2(double* V, int64_t n, double lam) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) V[i * n + i] += lam;
}

// Zero the strict upper triangle of a row-major n x n matrix.
__global__ void zero_strict_upper_kernel(double* V, int64_t n) {
  const int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (q >= n) return;
  for (int64_t p = blockIdx.y; p < q; p += gridDim.y) V[p * n + q] = 0.0;
}

int potrf_dmma(double* V, int64_t n, double lam, double* Dinv, int* info_dev, cudaStream_t st) {
  shift_diag_kernel2<<<grid_1d(n, 256), 256, 0, st>>>(V, n, lam);
  GSDFT_LAUNCHED("shift_diag");
  GSDFT_CUDA(cudaMemsetAsync(info_dev, 0, sizeof(int), st));
  for (int64_t k0 = 0; k0 < n; k0 += kNb) {
    const int kb = (int)imin64(kNb, n - k0);
    double* Akk = V + k0 * n + k0;
    potf2_inv_kernel<<<1, 256, 0, st>>>(Akk, n, kb, Dinv, info_dev, k0);
    GSDFT_LAUNCHED("potf2_inv");
    const int64_t rows = n - k0 - kb;
    if (rows <= 0) break;
    double* P = V + (k0 + kb) * n + k0;  // rows x kb panel below the block
    // P <- P inv(L_kk)^T
    int rc = gemm_launch<false, true, false, false, false>(
        gemm_args(rows, kb, kb, 1.0, P, n, Dinv, kNb, 0.0, P, n), 1, st);
    if (rc) return rc;
    // trailing lower triangle: A22 <- A22 - P P^T
    double* A22 = V + (k0 + kb) * n + (k0 + kb);
    rc = gemm_launch<false, true, false, false, true>(
        gemm_args(rows, rows, kb, -1.0, P, n, P, n, 1.0, A22, n), 1, st);
    if (rc) return rc;
  }
  dim3 grid(grid_1d(n, 256), (unsigned)imin64(n, 65535));
  zero_strict_upper_kernel<<<grid, 256, 0, st>>>(V, n);
  GSDFT_LAUNCHED("zero_upper");
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// Inverse of a lower-triangular factor by recursive doubling: with blocks of size s,
// [L11 0; L21 L22]^-1 = [X11 0; -X22 L21 X11  X22]. The 64 x 64 diagonal blocks are inverted in
// shared memory (all at once); then for s = 64, 128, ... every adjacent pair of inverted s-blocks
// is joined by two batched GEMMs: T^T = X11^T L21^T, written into the (still unused) strict upper
// block of the pair, and X21 = -X22 T. X11 and X22 are read as lower-triangular operands (their
// upper parts hold earlier levels' T). The strict upper triangle is garbage until the caller
// overwrites it (the packed inverse mirrors the lower triangle into it).
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(64) diag_inv_kernel(const double* __restrict__ L, int64_t n,
                                                      double* __restrict__ X) {
  // the block's factor in the lower triangle of s, its inverse transposed into the strict upper
  // triangle (inv[i][c] at s[c][i]) with the diagonal in xd
  __shared__ double s[kNb][kNb + 1];
  __shared__ double xd[kNb];
  const int64_t b0 = (int64_t)blockIdx.x * kNb;
  const int kb = (int)imin64(kNb, n - b0);
  const int tid = threadIdx.x;
  for (int i = 0; i < kNb; ++i)
    s[i][tid] = (i < kb && tid <= i) ? L[(b0 + i) * n + b0 + tid] : (i == tid ? 1.0 : 0.0);
  __syncthreads();
  if (tid < kb) {
    const int c = tid;
    xd[c] = 1.0 / s[c][c];
    for (int i = c + 1; i < kb; ++i) {
      double acc = s[i][c] * xd[c];
      for (int l = c + 1; l < i; ++l) acc = fma(s[i][l], s[c][l], acc);
      s[c][i] = -acc / s[i][i];
    }
  }
  __syncthreads();
  for (int i = 0; i < kb; ++i)
    if (tid < kb) X[(b0 + i) * n + b0 + tid] = tid < i ? s[tid][i] : (tid == i ? xd[i] : 0.0);
}

int trtri_dmma(const double* L, int64_t n, double* X, cudaStream_t st) {
  const int64_t nblk = (n + kNb - 1) / kNb;
  diag_inv_kernel<<<(unsigned)nblk, 64, 0, st>>>(L, n, X);
  GSDFT_LAUNCHED("diag_inv");
  for (int64_t s = kNb; s < n; s *= 2) {
    const int64_t batch = (n - s + 2 * s - 1) / (2 * s);  // pairs with a second block
    // T^T (s x s2) = X11^T (s x s) L21^T (s x s2), into X[b1 : b1+s, b2 : b2+s2]
    GemmArgs g1 = gemm_args(s, s, s, 1.0, X, n, L + s * n, n, 0.0, X + s, n);
    g1.sa = g1.sb = g1.sc = 2 * s * (n + 1);
    g1.Nclip = n - s, g1.Nstep = 2 * s;
    int rc = gemm_launch<true, true, true, false, false>(g1, batch, st);
    if (rc) return rc;
    // X21 (s2 x s) = -X22 (s2 x s2) T (s2 x s), T read through its transpose stored above
    GemmArgs g2 = gemm_args(s, s, s, -1.0, X + s * (n + 1), n, X + s, n, 0.0, X + s * n, n);
    g2.sa = g2.sb = g2.sc = 2 * s * (n + 1);
    g2.Mclip = n - s, g2.Mstep = 2 * s;
    g2.Kclip = n - s, g2.Kstep = 2 * s;
    rc = gemm_launch<false, true, true, false, false>(g2, batch, st);
    if (rc) return rc;
  }
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// One-shot solve (L L^T) d = gamma by blocked substitution in panels of 64: per panel, the diagonal
// block is solved in shared memory by one block, then the rest of the right-hand side is updated
// by a row-parallel panel product (forward: rows below; backward: columns to the left, read as the
// panel's rows of L). Every reduction has a fixed order.
// ------------------------------------------------------------------------------------------------
// Forward: y[p0:p0+kb] = L_pp^-1 r[p0:p0+kb] (in place in r). One warp.
__global__ void trsv_diag_fwd_kernel(const double* __restrict__ L, int64_t n, int64_t p0, int kb,
                                     double* __restrict__ r) {
  __shared__ double y[kNb];
  const int lane = threadIdx.x;
  for (int i = 0; i < kb; ++i) {
    const double* row = L + (p0 + i) * n + p0;
    double acc = 0.0;
    for (int l = lane; l < i; l += 32) acc = fma(row[l], y[l], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) y[i] = (r[p0 + i] - acc) / row[i];
    __syncwarp();
  }
  for (int i = lane; i < kb; i += 32) r[p0 + i] = y[i];
}

// Forward update: r[i] -= L[i, p0:p0+kb] . y for i >= p0 + kb; one warp per row.
__global__ void trsv_update_fwd_kernel(const double* __restrict__ L, int64_t n, int64_t p0, int kb,
                                       double* __restrict__ r) {
  const int64_t i = p0 + kb + ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const double* row = L + i * n + p0;
  double acc = 0.0;
  for (int l = lane; l < kb; l += 32) acc = fma(row[l], r[p0 + l], acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) r[i] -= acc;
}

// Backward: d[p0:p0+kb] = L_pp^-T r[p0:p0+kb] (in place). One warp.
__global__ void trsv_diag_bwd_kernel(const double* __restrict__ L, int64_t n, int64_t p0, int kb,
                                     double* __restrict__ r) {
  __shared__ double d[kNb];
  const int lane = threadIdx.x;
  for (int i = kb - 1; i >= 0; --i) {
    double acc = 0.0;
    for (int l = i + 1 + lane; l < kb; l += 32) acc = fma(L[(p0 + l) * n + p0 + i], d[l], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) d[i] = (r[p0 + i] - acc) / L[(p0 + i) * n + p0 + i];
    __syncwarp();
  }
  for (int i = lane; i < kb; i += 32) r[p0 + i] = d[i];
}

// Backward update: r[j] -= sum_{i in panel} L[i][j] d[i] for j < p0; one thread per column.
__global__ void trsv_update_bwd_kernel(const double* __restrict__ L, int64_t n, int64_t p0, int kb,
                                       double* __restrict__ r) {
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (j >= p0) return;
  double acc = 0.0;
  for (int i = 0; i < kb; ++i) acc = fma(L[(p0 + i) * n + j], r[p0 + i], acc);
  r[j] -= acc;
}

int trsv_llt(const double* L, int64_t n, double* d, cudaStream_t st) {
  for (int64_t p0 = 0; p0 < n; p0 += kNb) {
    const int kb = (int)imin64(kNb, n - p0);
    trsv_diag_fwd_kernel<<<1, 32, 0, st>>>(L, n, p0, kb, d);
    GSDFT_LAUNCHED("trsv_diag_fwd");
    const int64_t rows = n - p0 - kb;
    if (rows > 0) {
      trsv_update_fwd_kernel<<<grid_1d(rows * 32, 256), 256, 0, st>>>(L, n, p0, kb, d);
      GSDFT_LAUNCHED("trsv_update_fwd");
    }
  }
  for (int64_t p0 = ((n - 1) / kNb) * kNb; p0 >= 0; p0 -= kNb) {
    const int kb = (int)imin64(kNb, n - p0);
    trsv_diag_bwd_kernel<<<1, 32, 0, st>>>(L, n, p0, kb, d);
    GSDFT_LAUNCHED("trsv_diag_bwd");
    if (p0 > 0) {
      trsv_update_bwd_kernel<<<grid_1d(p0, 256), 256, 0, st>>>(L, n, p0, kb, d);
      GSDFT_LAUNCHED("trsv_update_bwd");
    }
  }
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// Orbital contractions on the pair list, as dense DMMA tiles over row blocks (gs_dft/coulomb/
// ri.py:456 and its gradient). The splats are cut into blocks of 64 consecutive rows; block b's
// partner list J_b is the sorted set of splats paired with its rows (consecutive splats sit on the
// same atoms, so their neighbour sets nearly coincide and the 64 x |J_b| block is mostly live).
// SDDMM: Q_b = (C_I diag(occ)) C_J^T into the block's dense tile, from which each representative
//   reads its q (one cell per representative).
// SpMM:  G_I (+)= T_b (C_J diag(occ)) with T_b the block's dense tile of per-representative values
//   (J w), giving g_C row by row.
// The partner rows of C are gathered by index inside the tile loads; every sum has a fixed order.
// ------------------------------------------------------------------------------------------------
struct BlockArgs {
  const double* C;        // (M, n_occ)
  const double* occ;      // (n_occ)
  int64_t M, n_occ;
  const int64_t* boff;    // per block: offset of its dense tile (elements), rows x nj
  const int32_t* nj;      // per block: partners
  const int64_t* joff;    // per block: offset into jidx
  const int32_t* jidx;    // concatenated partner lists
  double* buf;            // the blocks' dense tiles
  double* out;            // SpMM: g_C (M, n_occ)
  double beta;            // SpMM: out = beta out + tile products
};

// kSpmm = false (SDDMM): tile (64 rows of block b) x (64 partners), K = n_occ.
// kSpmm = true (SpMM): tile (64 rows of block b) x (64 orbitals), K = nj_b.
template <bool kSpmm>
__global__ void __launch_bounds__(128) block_contract_kernel(BlockArgs g) {
  const int64_t b = blockIdx.z;
  const int64_t r0 = b * kGT;
  const int64_t M = imin64(kGT, g.M - r0);
  const int64_t nj = g.nj[b];
  const int64_t N = kSpmm ? g.n_occ : nj;
  const int64_t K = kSpmm ? nj : g.n_occ;
  const int64_t n0 = (int64_t)blockIdx.x * kGT;
  if (M <= 0 || n0 >= N) return;
  const int32_t* __restrict__ J = g.jidx + g.joff[b];
  double* __restrict__ T = g.buf + g.boff[b];

  // A as [m][k]; B as [k][n] (SpMM: C_J rows) or [n][k] (SDDMM: C_J rows as the transposed operand)
  __shared__ double As[kGT][kGK + kGPad];
  __shared__ double Bs[kSpmm ? kGK : kGT][(kSpmm ? kGT : kGK) + kGPad];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
  const int ar = tid >> 1, ac = (tid & 1) * 8;
  const int br = kSpmm ? (tid >> 3) : (tid >> 1), bc = kSpmm ? (tid & 7) * 8 : (tid & 1) * 8;
  double ra[8], rb[8];

  auto load = [&](int64_t k0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t r = ar, c = k0 + ac + e;
      double v = 0.0;
      if (r < M && c < K) {
        if (kSpmm) v = T[r * nj + c];                                  // the block's tile
        else v = g.C[(r0 + r) * g.n_occ + c] * g.occ[c];             // C_I diag(occ)
      }
      ra[e] = v;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      double v = 0.0;
      if (kSpmm) {  // stored (k, n): row k is partner J[k], column n an orbital
        const int64_t k = k0 + br, n = n0 + bc + e;
        if (k < K && n < N) v = g.C[(int64_t)J[k] * g.n_occ + n] * g.occ[n];
      } else {      // stored (n, k): row n is partner J[n], column k an orbital
        const int64_t n = n0 + br, k = k0 + bc + e;
        if (n < N && k < K) v = g.C[(int64_t)J[n] * g.n_occ + k];
      }
      rb[e] = v;
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int e = 0; e < 8; ++e) As[ar][ac + e] = ra[e];
#pragma unroll
    for (int e = 0; e < 8; ++e) Bs[br][bc + e] = rb[e];
  };

  double acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.0;
  load(0);
  store();
  __syncthreads();
  for (int64_t k0 = 0; k0 < K; k0 += kGK) {
    const bool more = k0 + kGK < K;
    if (more) load(k0 + kGK);
#pragma unroll
    for (int kk = 0; kk < kGK; kk += 4) {
      double a0[2], a1[2], bv[4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int m = wm + mi * 16 + gq;
        a0[mi] = As[m][kk + tq];
        a1[mi] = As[m + 8][kk + tq];
      }
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const int n = wn + ni * 8 + gq;
        bv[ni] = kSpmm ? Bs[kk + tq][n] : Bs[n][kk + tq];
      }
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) dmma_m16n8k4(acc[mi][ni], a0[mi], a1[mi], bv[ni]);
    }
    __syncthreads();
    if (more) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t row = wm + mi * 16 + gq + (r >> 1) * 8;
        const int64_t col = n0 + wn + ni * 8 + 2 * tq + (r & 1);
        if (row < M && col < N) {
          if (kSpmm) {
            double* p = g.out + (r0 + row) * g.n_occ + col;
            *p = g.beta == 0.0 ? acc[mi][ni][r] : fma(g.beta, *p, acc[mi][ni][r]);
          } else {
            T[row * nj + col] = acc[mi][ni][r];
          }
        }
      }
}

// rec[a].q = w_a Q[cell_a] and rec[a].qk = q KN pref, after the SDDMM.
__global__ void block_q_gather_kernel(const double* __restrict__ buf, const int64_t* __restrict__ cell,
                                      const double* __restrict__ rep_w, int64_t n_rep,
                                      double* __restrict__ rec) {
  const int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_rep) return;
  const double q = rep_w[a] * buf[cell[a]];
  double* r = rec + a * GSDFT_REC_FIELDS;
  r[GSDFT_REC_Q] = q;
  r[GSDFT_REC_QK] = q * r[GSDFT_REC_KN];
}

// buf[cell_a] = v_a (every other cell zero), before an SpMM.
__global__ void block_scatter_kernel(const double* __restrict__ v, const int64_t* __restrict__ cell,
                                     int64_t n, double* __restrict__ buf) {
  const int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a < n) buf[cell[a]] = v[a];
}

static int block_launch(bool spmm, const BlockArgs& g, int64_t n_blocks, int64_t max_nj,
                        cudaStream_t st) {
  if (n_blocks <= 0) return GSDFT_OK;
  GSDFT_REQUIRE(n_blocks <= 65535, "too many row blocks for one launch");
  const int64_t ncols = spmm ? g.n_occ : max_nj;
  if (ncols <= 0) return GSDFT_OK;
  dim3 grid((unsigned)((ncols + kGT - 1) / kGT), 1, (unsigned)n_blocks);
  if (spmm) block_contract_kernel<true><<<grid, 128, 0, st>>>(g);
  else block_contract_kernel<false><<<grid, 128, 0, st>>>(g);
  GSDFT_LAUNCHED("block_contract");
  return GSDFT_OK;
}

}  // namespace gsdft

using namespace gsdft;

extern "C" int gsdft_block_density(const double* C_occ, const double* occ, int64_t M,
                                   int64_t n_occ, int64_t n_blocks, const int64_t* boff,
                                   const int32_t* nj, const int64_t* joff, const int32_t* jidx,
                                   int64_t max_nj, const int64_t* cell, const double* rep_w,
                                   int64_t n_rep, double* buf, double* rec,
                                   gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_occ > 0 && n_blocks == (M + kGT - 1) / kGT && n_rep >= 0 && max_nj >= 0,
                "bad sizes");
  GSDFT_REQUIRE(C_occ && occ && boff && nj && joff && buf, "null pointer");
  GSDFT_REQUIRE(n_rep == 0 || (jidx && cell && rep_w && rec), "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  BlockArgs g{C_occ, occ, M, n_occ, boff, nj, joff, jidx, buf, nullptr, 0.0};
  int rc = block_launch(false, g, n_blocks, max_nj, st);
  if (rc || n_rep == 0) return rc;
  block_q_gather_kernel<<<grid_1d(n_rep, 256), 256, 0, st>>>(buf, cell, rep_w, n_rep, rec);
  GSDFT_LAUNCHED("block_q_gather");
  return GSDFT_OK;
}

extern "C" int gsdft_block_density_grad(const double* vals, const int64_t* cell, int64_t n_rep,
                                        const double* C_occ, const double* occ, int64_t M,
                                        int64_t n_occ, int64_t n_blocks, const int64_t* boff,
                                        const int32_t* nj, const int64_t* joff,
                                        const int32_t* jidx, int64_t buf_len, double* buf,
                                        double beta, double* g_C, gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && n_occ > 0 && n_blocks == (M + kGT - 1) / kGT && n_rep >= 0 &&
                    buf_len >= 0,
                "bad sizes");
  GSDFT_REQUIRE(C_occ && occ && boff && nj && joff && g_C && (buf_len == 0 || buf), "null pointer");
  GSDFT_REQUIRE(n_rep == 0 || (vals && cell && jidx), "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (buf_len > 0) GSDFT_CUDA(cudaMemsetAsync(buf, 0, (size_t)buf_len * sizeof(double), st));
  if (n_rep > 0) {
    block_scatter_kernel<<<grid_1d(n_rep, 256), 256, 0, st>>>(vals, cell, n_rep, buf);
    GSDFT_LAUNCHED("block_scatter");
  }
  BlockArgs g{C_occ, occ, M, n_occ, boff, nj, joff, jidx, buf, g_C, beta};
  return block_launch(true, g, n_blocks, 0, st);
}

extern "C" int gsdft_dense_gemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
                                double alpha, const double* A, int64_t lda, const double* B,
                                int64_t ldb, double beta, double* C, int64_t ldc,
                                gsdft_stream_t stream) {
  GSDFT_REQUIRE(M >= 0 && N >= 0 && K >= 0, "bad sizes");
  if (M == 0 || N == 0) return GSDFT_OK;
  GSDFT_REQUIRE(C && (K == 0 || (A && B)), "null pointer");
  GSDFT_REQUIRE(lda >= (trans_a ? M : K) && ldb >= (trans_b ? K : N) && ldc >= N,
                "leading dimension too small");
  GSDFT_REQUIRE(M <= int64_t(65535) * kGT, "M too large for one launch");
  const GemmArgs g = gemm_args(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  cudaStream_t st = (cudaStream_t)stream;
  if (trans_a && trans_b) return gemm_launch<true, true, false, false, false>(g, 1, st);
  if (trans_a) return gemm_launch<true, false, false, false, false>(g, 1, st);
  if (trans_b) return gemm_launch<false, true, false, false, false>(g, 1, st);
  return gemm_launch<false, false, false, false, false>(g, 1, st);
}
