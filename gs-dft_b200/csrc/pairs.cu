// Significant-pair list on the GPU: |S_ij| > eps over all M^2 ordered candidates, compacted in
// lexsorted (flat i*M+j ascending) order, padded to pad_to; overflow keeps the pad_to largest |S|.
// Reference: gs_dft/screening/pairs.py:50-164 (builders), :225-315 (neighbor_pairs), :318-322
// (weights), :342-345 (overlap); gs_dft/ks/shard.py:146-166 (stripe_pairs).
//
// The overlap of a pair is evaluated once per unordered pair, in the (min, max) orientation, with
// FMA contraction disabled and the reference's operation order, and shared by (i,j) and (j,i).
#include <cub/cub.cuh>
#include <thrust/iterator/counting_iterator.h>

#include "common.cuh"

namespace gsdft {

constexpr int kRowThreads = 256;
constexpr double kPi15 = 5.568327996831708;  // pi ** 1.5 as the reference's float computes it

__device__ __forceinline__ double abs_overlap(const double* __restrict__ A9,
                                              const double* __restrict__ mu,
                                              const double* __restrict__ N, int i, int j) {
  int lo = min(i, j), hi = max(i, j);
  double Ai[9], Aj[9], mui[3], muj[3];
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    Ai[k] = A9[9 * (int64_t)lo + k];
    Aj[k] = A9[9 * (int64_t)hi + k];
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    mui[k] = mu[3 * (int64_t)lo + k];
    muj[k] = mu[3 * (int64_t)hi + k];
  }
  double Ah[9], P[3], KN, det;
  pair_quantities_rn(Ai, Aj, mui, muj, N[lo], N[hi], Ah, P, &KN, &det);
  return fabs(__ddiv_rn(DM(KN, kPi15), __dsqrt_rn(det)));
}

constexpr int kRowWarps = kRowThreads / 32;

// Per-row count of significant columns (j >= i when unique): per warp the population count of
// its significance ballots, then the warps' counts added in warp order.
__global__ void pairs_count_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                   const double* __restrict__ N, int M, double eps, int unique,
                                   int64_t* __restrict__ row_count) {
  __shared__ int s_warp[kRowWarps];
  const int i = blockIdx.x;
  const int j0 = unique ? i : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int cnt = 0;  // warp-uniform
  for (int jb = j0; jb < M; jb += kRowThreads) {
    const int j = jb + threadIdx.x;
    const bool sig = j < M && abs_overlap(A9, mu, N, i, j) > eps;
    cnt += __popc(__ballot_sync(0xffffffffu, sig));
  }
  if (lane == 0) s_warp[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t tot = 0;
    for (int w = 0; w < kRowWarps; ++w) tot += s_warp[w];
    row_count[i] = tot;
  }
}

// Ordered write of row i's significant columns at row_off[i]: a warp-ballot + prefix-scan
// compaction. Per chunk of kRowThreads columns, each warp's ballot of the significance flags gives
// a lane its rank inside the warp (popc of the lower lanes' bits) and the warp its count; an
// exclusive scan of the kRowWarps counts in shared memory gives each warp's offset, so the columns
// land in ascending j. Direct mode writes (pi,pj,w); ranking mode writes (flat index, |S|) for the
// overflow selection.
__global__ void pairs_build_kernel(const double* __restrict__ A9, const double* __restrict__ mu,
                                   const double* __restrict__ N, int M, double eps, int unique,
                                   const int64_t* __restrict__ row_off, int ranking,
                                   int32_t* __restrict__ pi, int32_t* __restrict__ pj,
                                   double* __restrict__ w, int64_t* __restrict__ flat,
                                   double* __restrict__ val) {
  __shared__ int s_warp[kRowWarps];
  const int i = blockIdx.x;
  const int j0 = unique ? i : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lower = (1u << lane) - 1u;
  int64_t base = row_off[i];
  for (int jb = j0; jb < M; jb += kRowThreads) {
    const int j = jb + threadIdx.x;
    double s = 0.0;
    int sig = 0;
    if (j < M) {
      s = abs_overlap(A9, mu, N, i, j);
      sig = s > eps ? 1 : 0;
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, sig);
    if (lane == 0) s_warp[warp] = __popc(ballot);
    __syncthreads();
    int offset = 0, total = 0;
    for (int w2 = 0; w2 < kRowWarps; ++w2) {
      const int c = s_warp[w2];
      offset += w2 < warp ? c : 0;
      total += c;
    }
    const int rank = offset + __popc(ballot & lower);
    if (sig) {
      int64_t pos = base + rank;
      if (ranking) {
        flat[pos] = (int64_t)i * M + j;
        val[pos] = s;
      } else {
        pi[pos] = i;
        pj[pos] = j;
        w[pos] = unique ? (i == j ? 1.0 : 2.0) : 1.0;
      }
    }
    base += total;
    __syncthreads();  // every warp has read s_warp before the next chunk overwrites it
  }
}

__global__ void fill_pad_kernel(int64_t start, int64_t n, int32_t* pi, int32_t* pj, double* w) {
  int64_t k = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= n) return;
  pi[k] = 0;
  pj[k] = 0;
  w[k] = 0.0;
}

__global__ void decode_flat_kernel(const int64_t* __restrict__ flat, int64_t n, int M, int unique,
                                   int32_t* pi, int32_t* pj, double* w) {
  int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= n) return;
  int64_t f = flat[k];
  int i = (int)(f / M), j = (int)(f % M);
  pi[k] = i;
  pj[k] = j;
  w[k] = unique ? (i == j ? 1.0 : 2.0) : 1.0;
}

// |S| > 0 doubles order like their bit patterns as unsigned integers.
__global__ void val_bits_kernel(const double* __restrict__ val, int64_t n, uint64_t* bits) {
  int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k < n) bits[k] = (uint64_t)__double_as_longlong(val[k]);
}

__global__ void stripe_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                              const double* __restrict__ w, int64_t n, int G, int32_t* pio,
                              int32_t* pjo, double* wo) {
  int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k >= n) return;
  int64_t d = n / G;
  int64_t g = k / d, j = k % d;       // new[g*d + j] = old[j*G + g]
  int64_t src = j * G + g;
  pio[k] = pi[src];
  pjo[k] = pj[src];
  wo[k] = w[src];
}

// ------------------------------------------------------------------------------------------------
// Pair plan helpers
// ------------------------------------------------------------------------------------------------
__global__ void live_flags_kernel(const double* __restrict__ w, int64_t n, char* flags) {
  int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k < n) flags[k] = w[k] != 0.0;
}

__global__ void flat_keys_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                                 const int32_t* __restrict__ live, int64_t n_live, int64_t M,
                                 int64_t* __restrict__ keys, int32_t* __restrict__ iota) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_live) return;
  int32_t e = live[a];
  keys[a] = (int64_t)pi[e] * M + pj[e];
  iota[a] = (int32_t)a;
}

// Position of `key` in the sorted keys if it occurs exactly once, else -1.
__device__ __forceinline__ int64_t find_unique(const int64_t* __restrict__ sk, int64_t n,
                                               int64_t key) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (sk[mid] < key) lo = mid + 1; else hi = mid;
  }
  if (lo >= n || sk[lo] != key) return -1;
  if (lo + 1 < n && sk[lo + 1] == key) return -1;
  return lo;
}

// Twin merge: a live (i,j), i < j, whose transpose (j,i) is also live (each key occurring once)
// becomes the representative of both; (j,i) is absorbed. Every other live entry represents itself.
__global__ void twin_kernel(const int32_t* __restrict__ pi, const int32_t* __restrict__ pj,
                            const int32_t* __restrict__ live, int64_t n_live, int64_t M,
                            const int64_t* __restrict__ sk, const int32_t* __restrict__ sv,
                            int merge, char* __restrict__ is_rep, int32_t* __restrict__ twin) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n_live) return;
  int32_t e = live[a];
  int64_t i = pi[e], j = pj[e];
  int32_t tw = -1;
  char rep = 1;
  if (merge && i != j && find_unique(sk, n_live, i * M + j) >= 0) {
    int64_t s = find_unique(sk, n_live, j * M + i);
    if (s >= 0) {
      if (i < j) tw = live[sv[s]];
      else rep = 0;
    }
  }
  is_rep[a] = rep;
  twin[a] = tw;
}

__global__ void rep_gather_kernel(const int32_t* __restrict__ live, const int32_t* __restrict__ sel,
                                  const int32_t* __restrict__ twin, const double* __restrict__ w,
                                  int64_t n_rep, int32_t* __restrict__ rep_pos,
                                  double* __restrict__ rep_w, int32_t* __restrict__ rep_twin) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n_rep) return;
  int32_t a = sel[r];
  int32_t e = live[a];
  int32_t t = twin[a];
  rep_pos[r] = e;
  rep_twin[r] = t;
  rep_w[r] = t >= 0 ? w[e] + w[t] : w[e];
}

__global__ void gather_keys_kernel(const int32_t* __restrict__ key, const int32_t* __restrict__ pos,
                                   int64_t n, int32_t* __restrict__ out,
                                   int32_t* __restrict__ iota) {
  int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (a >= n) return;
  out[a] = key[pos[a]];
  iota[a] = (int32_t)a;
}

// partner[e] = the other splat of the representative at sorted position e (pj for the by-pi
// grouping, pi for the by-pj grouping).
__global__ void partner_kernel(const int32_t* __restrict__ other, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ order, int64_t n,
                               int32_t* __restrict__ partner) {
  int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e < n) partner[e] = other[pos[order[e]]];
}

// seg[s] = first position in the sorted keys with key >= s, s in [0, M].
__global__ void segment_bounds_kernel(const int32_t* __restrict__ sorted, int64_t n, int64_t M,
                                      int64_t* __restrict__ seg) {
  int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (s > M) return;
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (sorted[mid] < s) lo = mid + 1; else hi = mid;
  }
  seg[s] = lo;
}

struct PairsWs {
  int64_t* row_count;
  int64_t* row_off;
  void* scan_tmp;
  size_t scan_bytes;
  int64_t* flat;
  double* val;
  uint64_t* bits;
  uint64_t* bits_sorted;
  int64_t* flat_sorted;
  int64_t* keep;
  int64_t* keep_sorted;
  void* sort_tmp;
  size_t sort_bytes;
};

template <class C>
static void layout_pairs_ws(C& c, int64_t M, int64_t pad_to, PairsWs* p, size_t scan_bytes,
                            size_t sort_bytes) {
  int64_t cap = 2 * (pad_to > 0 ? pad_to : 0);
  auto rc = c.template take<int64_t>(M + 1);
  auto ro = c.template take<int64_t>(M + 1);
  auto st = c.template take<char>(scan_bytes);
  auto fl = c.template take<int64_t>(cap + 1);
  auto va = c.template take<double>(cap + 1);
  auto bi = c.template take<uint64_t>(cap + 1);
  auto bs = c.template take<uint64_t>(cap + 1);
  auto fs = c.template take<int64_t>(cap + 1);
  auto ke = c.template take<int64_t>(cap + 1);
  auto ks = c.template take<int64_t>(cap + 1);
  auto so = c.template take<char>(sort_bytes);
  if (p) {
    *p = PairsWs{(int64_t*)rc, (int64_t*)ro, st, scan_bytes, (int64_t*)fl, (double*)va,
                 (uint64_t*)bi, (uint64_t*)bs, (int64_t*)fs, (int64_t*)ke, (int64_t*)ks, so,
                 sort_bytes};
  }
}

// Sizer::take returns void; wrap so both carve paths share one layout routine.
struct SizerP {
  Sizer s;
  template <class T>
  T* take(size_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

static void cub_sizes(int64_t M, int64_t pad_to, size_t* scan_bytes, size_t* sort_bytes) {
  size_t sb = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, sb, (int64_t*)nullptr, (int64_t*)nullptr, (int)(M + 1));
  int64_t cap = 2 * (pad_to > 0 ? pad_to : 0);
  size_t s1 = 0, s2 = 0;
  if (cap > 0) {
    cub::DeviceRadixSort::SortPairsDescending(nullptr, s1, (uint64_t*)nullptr, (uint64_t*)nullptr,
                                              (int64_t*)nullptr, (int64_t*)nullptr, (int)cap);
    cub::DeviceRadixSort::SortKeys(nullptr, s2, (int64_t*)nullptr, (int64_t*)nullptr, (int)cap);
  }
  *scan_bytes = sb;
  *sort_bytes = s1 > s2 ? s1 : s2;
}

}  // namespace gsdft

using namespace gsdft;

extern "C" size_t gsdft_pairs_workspace_size(int64_t M, int64_t pad_to) {
  size_t sb, so;
  cub_sizes(M, pad_to, &sb, &so);
  SizerP z;
  layout_pairs_ws(z, M, pad_to, nullptr, sb, so);
  return z.s.off + 256;
}

static int pairs_counts(const double* A9, const double* mu, const double* N, int64_t M,
                        double eps, int unique, const PairsWs& ws, int64_t* n_sig_host,
                        cudaStream_t st) {
  pairs_count_kernel<<<(int)M, kRowThreads, 0, st>>>(A9, mu, N, (int)M, eps, unique,
                                                       ws.row_count);
  GSDFT_LAUNCHED("pairs_count");
  GSDFT_CUDA(cudaMemsetAsync(ws.row_count + M, 0, sizeof(int64_t), st));
  size_t sb = ws.scan_bytes;
  GSDFT_CUDA(cub::DeviceScan::ExclusiveSum(ws.scan_tmp, sb, ws.row_count, ws.row_off,
                                           (int)(M + 1), st));
  GSDFT_CUDA(cudaMemcpyAsync(n_sig_host, ws.row_off + M, sizeof(int64_t), cudaMemcpyDeviceToHost,
                             st));
  GSDFT_CUDA(cudaStreamSynchronize(st));
  return GSDFT_OK;
}

static int carve_pairs_ws(void* ws, size_t ws_bytes, int64_t M, int64_t pad_to, PairsWs* p) {
  size_t sb, so;
  cub_sizes(M, pad_to, &sb, &so);
  Carver c(ws, ws_bytes);
  layout_pairs_ws(c, M, pad_to, p, sb, so);
  if (!c.ok)
    return fail(GSDFT_ERR_ARG, "pairs workspace too small: need %zu bytes, got %zu", c.off,
                ws_bytes);
  return GSDFT_OK;
}

extern "C" int gsdft_pairs_count(const double* A9, const double* mu, const double* N, int64_t M,
                                 double eps, int unique, int64_t* n_sig_host, void* ws,
                                 size_t ws_bytes, gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && M < (int64_t(1) << 31), "M out of range");
  GSDFT_REQUIRE(A9 && mu && N && n_sig_host, "null pointer");
  PairsWs p;
  int rc = carve_pairs_ws(ws, ws_bytes, M, 0, &p);
  if (rc) return rc;
  return pairs_counts(A9, mu, N, M, eps, unique, p, n_sig_host, (cudaStream_t)stream);
}

extern "C" int gsdft_pairs_build(const double* A9, const double* mu, const double* N, int64_t M,
                                 double eps, int unique, int64_t pad_to, int32_t* pi, int32_t* pj,
                                 double* w, int64_t* n_sig_host, void* ws, size_t ws_bytes,
                                 gsdft_stream_t stream) {
  GSDFT_REQUIRE(M > 0 && M < (int64_t(1) << 31), "M out of range");
  GSDFT_REQUIRE(pad_to >= 0 && pad_to < (int64_t(1) << 31), "pad_to out of range");
  GSDFT_REQUIRE(A9 && mu && N && n_sig_host, "null pointer");
  GSDFT_REQUIRE(pad_to == 0 || (pi && pj && w), "null output pointer");
  cudaStream_t st = (cudaStream_t)stream;
  PairsWs p;
  int rc = carve_pairs_ws(ws, ws_bytes, M, pad_to, &p);
  if (rc) return rc;
  rc = pairs_counts(A9, mu, N, M, eps, unique, p, n_sig_host, st);
  if (rc) return rc;
  int64_t n_sig = *n_sig_host;
  if (n_sig <= pad_to) {
    pairs_build_kernel<<<(int)M, kRowThreads, 0, st>>>(A9, mu, N, (int)M, eps, unique, p.row_off,
                                                         0, pi, pj, w, nullptr, nullptr);
    GSDFT_LAUNCHED("pairs_build");
    if (pad_to > n_sig) {
      fill_pad_kernel<<<grid_1d(pad_to - n_sig, 256), 256, 0, st>>>(n_sig, pad_to, pi, pj, w);
      GSDFT_LAUNCHED("fill_pad");
    }
    return GSDFT_OK;
  }
  if (n_sig > 2 * pad_to)
    return fail(GSDFT_ERR_OVERFLOW,
                "neighbor_pairs: %lld significant pairs exceed 2x the pad (%lld); raise the pad",
                (long long)n_sig, (long long)(2 * pad_to));
  // Overflow: all significant (flat, |S|), then a stable descending sort by |S| (ties keep the
  // ascending flat order), the first pad_to, and an ascending sort of their flat indices.
  pairs_build_kernel<<<(int)M, kRowThreads, 0, st>>>(A9, mu, N, (int)M, eps, unique, p.row_off, 1,
                                                       nullptr, nullptr, nullptr, p.flat, p.val);
  GSDFT_LAUNCHED("pairs_build_rank");
  val_bits_kernel<<<grid_1d(n_sig, 256), 256, 0, st>>>(p.val, n_sig, p.bits);
  GSDFT_LAUNCHED("val_bits");
  size_t sb = p.sort_bytes;
  GSDFT_CUDA(cub::DeviceRadixSort::SortPairsDescending(p.sort_tmp, sb, p.bits, p.bits_sorted,
                                                       p.flat, p.flat_sorted, (int)n_sig, 0, 64,
                                                       st));
  sb = p.sort_bytes;
  GSDFT_CUDA(cub::DeviceRadixSort::SortKeys(p.sort_tmp, sb, p.flat_sorted, p.keep_sorted,
                                            (int)pad_to, 0, 64, st));
  decode_flat_kernel<<<grid_1d(pad_to, 256), 256, 0, st>>>(p.keep_sorted, pad_to, (int)M, unique,
                                                           pi, pj, w);
  GSDFT_LAUNCHED("decode_flat");
  return GSDFT_OK;
}

extern "C" int gsdft_stripe_pairs(const int32_t* pi, const int32_t* pj, const double* w, int64_t n,
                                  int G, int32_t* pi_out, int32_t* pj_out, double* w_out,
                                  gsdft_stream_t stream) {
  GSDFT_REQUIRE(n >= 0 && G >= 1, "bad n or G");
  if (n == 0) return GSDFT_OK;
  GSDFT_REQUIRE(pi && pj && w && pi_out && pj_out && w_out, "null pointer");
  GSDFT_REQUIRE(pi_out != pi && pj_out != pj && w_out != w, "stripe_pairs is out of place");
  cudaStream_t st = (cudaStream_t)stream;
  if (G <= 1 || n % G) {
    GSDFT_CUDA(cudaMemcpyAsync(pi_out, pi, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    GSDFT_CUDA(cudaMemcpyAsync(pj_out, pj, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    GSDFT_CUDA(cudaMemcpyAsync(w_out, w, n * sizeof(double), cudaMemcpyDeviceToDevice, st));
    return GSDFT_OK;
  }
  stripe_kernel<<<grid_1d(n, 256), 256, 0, st>>>(pi, pj, w, n, G, pi_out, pj_out, w_out);
  GSDFT_LAUNCHED("stripe");
  return GSDFT_OK;
}

// ------------------------------------------------------------------------------------------------
// Pair plan: representatives (live entries, transposed twins merged) and their groupings
// ------------------------------------------------------------------------------------------------
namespace {
static int bits_for(int64_t v) {
  int b = 1;
  while (b < 63 && (int64_t(1) << b) <= v) ++b;
  return b;
}

struct RepsWs {
  char* flags;
  int64_t* n_sel;
  int32_t* live;
  int64_t* keys;
  int64_t* keys_sorted;
  int32_t* iota;
  int32_t* vals_sorted;
  char* is_rep;
  int32_t* twin;
  int32_t* sel;
  void* tmp;
  size_t tmp_bytes;
};

size_t reps_tmp_bytes(int64_t n) {
  size_t a = 0, b = 0, c = 0;
  cub::DeviceSelect::Flagged(nullptr, a, thrust::counting_iterator<int32_t>(0), (char*)nullptr,
                             (int32_t*)nullptr, (int64_t*)nullptr, (int)n);
  cub::DeviceRadixSort::SortPairs(nullptr, b, (int64_t*)nullptr, (int64_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  cub::DeviceRadixSort::SortPairs(nullptr, c, (int32_t*)nullptr, (int32_t*)nullptr,
                                  (int32_t*)nullptr, (int32_t*)nullptr, (int)n);
  size_t m = a > b ? a : b;
  return m > c ? m : c;
}

template <class C>
void layout_reps(C& c, int64_t n, RepsWs* p, size_t tmp) {
  auto f = c.template take<char>(n + 1);
  auto ns = c.template take<int64_t>(1);
  auto lv = c.template take<int32_t>(n + 1);
  auto k = c.template take<int64_t>(n + 1);
  auto ks = c.template take<int64_t>(n + 1);
  auto io = c.template take<int32_t>(n + 1);
  auto vs = c.template take<int32_t>(n + 1);
  auto ir = c.template take<char>(n + 1);
  auto tw = c.template take<int32_t>(n + 1);
  auto se = c.template take<int32_t>(n + 1);
  auto t = c.template take<char>(tmp);
  if (p)
    *p = RepsWs{(char*)f,      (int64_t*)ns,  (int32_t*)lv, (int64_t*)k,  (int64_t*)ks,
                (int32_t*)io,  (int32_t*)vs,  (char*)ir,    (int32_t*)tw, (int32_t*)se,
                t,             tmp};
}
}  // namespace

extern "C" size_t gsdft_pair_plan_workspace_size(int64_t n, int64_t M) {
  (void)M;
  SizerP z;
  layout_reps(z, n, nullptr, reps_tmp_bytes(n));
  return z.s.off + 256;
}

extern "C" int gsdft_pair_reps(const int32_t* pi, const int32_t* pj, const double* w, int64_t n,
                               int64_t M, int merge_twins, int32_t* rep_pos, double* rep_w,
                               int32_t* rep_twin, int64_t* n_rep_host, void* ws, size_t ws_bytes,
                               gsdft_stream_t stream) {
  GSDFT_REQUIRE(n >= 0 && n < (int64_t(1) << 31) && M > 0 && M < (int64_t(1) << 31),
                "bad n or M");
  GSDFT_REQUIRE(n_rep_host, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  *n_rep_host = 0;
  if (n == 0) return GSDFT_OK;
  GSDFT_REQUIRE(pi && pj && w && rep_pos && rep_w && rep_twin, "null pointer");
  RepsWs p;
  size_t tmp = reps_tmp_bytes(n);
  Carver c(ws, ws_bytes);
  layout_reps(c, n, &p, tmp);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "pair plan workspace too small (%zu < %zu)", ws_bytes, c.off);
  live_flags_kernel<<<grid_1d(n, 256), 256, 0, st>>>(w, n, p.flags);
  GSDFT_LAUNCHED("live_flags");
  size_t tb = tmp;
  GSDFT_CUDA(cub::DeviceSelect::Flagged(p.tmp, tb, thrust::counting_iterator<int32_t>(0), p.flags,
                                        p.live, p.n_sel, (int)n, st));
  int64_t nl = 0;
  GSDFT_CUDA(cudaMemcpyAsync(&nl, p.n_sel, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  GSDFT_CUDA(cudaStreamSynchronize(st));
  if (nl == 0) return GSDFT_OK;
  flat_keys_kernel<<<grid_1d(nl, 256), 256, 0, st>>>(pi, pj, p.live, nl, M, p.keys, p.iota);
  GSDFT_LAUNCHED("flat_keys");
  tb = tmp;
  GSDFT_CUDA(cub::DeviceRadixSort::SortPairs(p.tmp, tb, p.keys, p.keys_sorted, p.iota,
                                             p.vals_sorted, (int)nl, 0, bits_for(M * M), st));
  twin_kernel<<<grid_1d(nl, 256), 256, 0, st>>>(pi, pj, p.live, nl, M, p.keys_sorted,
                                                p.vals_sorted, merge_twins, p.is_rep, p.twin);
  GSDFT_LAUNCHED("twin");
  tb = tmp;
  GSDFT_CUDA(cub::DeviceSelect::Flagged(p.tmp, tb, thrust::counting_iterator<int32_t>(0),
                                        p.is_rep, p.sel, p.n_sel, (int)nl, st));
  int64_t nr = 0;
  GSDFT_CUDA(cudaMemcpyAsync(&nr, p.n_sel, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  GSDFT_CUDA(cudaStreamSynchronize(st));
  if (nr > 0) {
    rep_gather_kernel<<<grid_1d(nr, 256), 256, 0, st>>>(p.live, p.sel, p.twin, w, nr, rep_pos,
                                                        rep_w, rep_twin);
    GSDFT_LAUNCHED("rep_gather");
  }
  *n_rep_host = nr;
  return GSDFT_OK;
}

extern "C" size_t gsdft_pair_groups_workspace_size(int64_t n_rep, int64_t M) {
  (void)M;
  return gsdft_pair_plan_workspace_size(n_rep, M);
}

extern "C" int gsdft_pair_groups(const int32_t* pi, const int32_t* pj, const int32_t* rep_pos,
                                 int64_t n_rep, int64_t M, int32_t* order_i, int64_t* seg_i,
                                 int32_t* partner_i, int32_t* order_j, int64_t* seg_j,
                                 int32_t* partner_j, void* ws, size_t ws_bytes,
                                 gsdft_stream_t stream) {
  GSDFT_REQUIRE(n_rep >= 0 && n_rep < (int64_t(1) << 31) && M > 0, "bad n_rep or M");
  GSDFT_REQUIRE(seg_i && seg_j, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  RepsWs p;
  size_t tmp = reps_tmp_bytes(n_rep);
  Carver c(ws, ws_bytes);
  layout_reps(c, n_rep, &p, tmp);
  if (!c.ok) return fail(GSDFT_ERR_ARG, "pair groups workspace too small (%zu < %zu)", ws_bytes, c.off);
  GSDFT_REQUIRE(n_rep == 0 || (pi && pj && rep_pos && order_i && order_j && partner_i && partner_j),
                "null pointer");
  int eb = bits_for(M);
  const int32_t* keysrc[2] = {pi, pj};
  const int32_t* othersrc[2] = {pj, pi};
  int32_t* order[2] = {order_i, order_j};
  int32_t* partner[2] = {partner_i, partner_j};
  int64_t* seg[2] = {seg_i, seg_j};
  int32_t* k32 = reinterpret_cast<int32_t*>(p.keys);
  int32_t* k32s = reinterpret_cast<int32_t*>(p.keys_sorted);
  for (int s = 0; s < 2; ++s) {
    if (n_rep > 0) {
      gather_keys_kernel<<<grid_1d(n_rep, 256), 256, 0, st>>>(keysrc[s], rep_pos, n_rep, k32, p.iota);
      GSDFT_LAUNCHED("gather_keys");
      size_t tb = tmp;
      GSDFT_CUDA(cub::DeviceRadixSort::SortPairs(p.tmp, tb, k32, k32s, p.iota, order[s],
                                                 (int)n_rep, 0, eb, st));
      partner_kernel<<<grid_1d(n_rep, 256), 256, 0, st>>>(othersrc[s], rep_pos, order[s], n_rep,
                                                          partner[s]);
      GSDFT_LAUNCHED("partner");
    }
    segment_bounds_kernel<<<grid_1d(M + 1, 256), 256, 0, st>>>(k32s, n_rep, M, seg[s]);
    GSDFT_LAUNCHED("segment_bounds");
  }
  return GSDFT_OK;
}
