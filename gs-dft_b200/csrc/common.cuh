// Shared device helpers and host error plumbing for the gs-dft B200 RI-J library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include <stdio.h>

#include "quad_table.h"
#include "../../include/gsdft_b200.h"

namespace gsdft {

// ------------------------------------------------------------------------------------------------
// Host: last-error string (thread-local), status helpers
// ------------------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

#define GSDFT_CUDA(call)                                                                    \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess)                                                                  \
      return ::gsdft::fail(GSDFT_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call,        \
                           cudaGetErrorString(e_));                                         \
  } while (0)

void count_launch();

#define GSDFT_LAUNCHED(name)                                                                \
  do {                                                                                      \
    ::gsdft::count_launch();                                                                \
    cudaError_t e_ = cudaGetLastError();                                                    \
    if (e_ != cudaSuccess)                                                                  \
      return ::gsdft::fail(GSDFT_ERR_CUDA, "launch %s: %s", name, cudaGetErrorString(e_));  \
  } while (0)

#define GSDFT_REQUIRE(cond, ...)                                                            \
  do {                                                                                      \
    if (!(cond)) return ::gsdft::fail(GSDFT_ERR_ARG, __VA_ARGS__);                           \
  } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace; every carve is 256-byte aligned.
struct Carver {
  char* base;
  size_t cap;
  size_t off = 0;
  bool ok = true;
  Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <class T>
  T* take(size_t n) {
    off = align_up(off, 256);
    size_t bytes = align_up(n * sizeof(T), 256);
    if (base == nullptr || off + bytes > cap) {
      ok = false;
      off += bytes;
      return nullptr;
    }
    T* p = reinterpret_cast<T*>(base + off);
    off += bytes;
    return p;
  }
};

// Counts the bytes a Carver sequence will need (same alignment rules).
struct Sizer {
  size_t off = 0;
  template <class T>
  void take(size_t n) {
    off = align_up(off, 256);
    off += align_up(n * sizeof(T), 256);
  }
};

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

// Number of splits S of a second axis that best fills whole waves: `base` independent work items
// become base*S items of 1/S the work each; resident capacity is `cap` CTAs. Returns the smallest
// S in [1, max_s] within 1% of the best wave efficiency base*S / (ceil(base*S/cap) * cap).
inline int best_splits(int64_t base, int64_t cap, int64_t max_s) {
  if (cap < 1) cap = 1;
  if (max_s < 1) max_s = 1;
  double best = 0.0;
  for (int64_t s = 1; s <= max_s; ++s) {
    int64_t items = base * s;
    int64_t waves = (items + cap - 1) / cap;
    best = fmax(best, (double)items / (double)(waves * cap));
  }
  for (int64_t s = 1; s <= max_s; ++s) {
    int64_t items = base * s;
    int64_t waves = (items + cap - 1) / cap;
    if ((double)items / (double)(waves * cap) >= best - 0.01) return (int)s;
  }
  return 1;
}

// Streaming multiprocessors of the device current at the first call (148 on B200); a thread-safe
// static, queried once per process.
int device_sms();

inline int grid_1d(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// ------------------------------------------------------------------------------------------------
// Device: 3x3 algebra in the reference's operation order (gs_dft/integrals/linalg3.py:17-51).
// Matrices are row-major 9-vectors. Plain +,-,* with FMA contraction disabled by the __d*_rn
// intrinsics where bit-faithful screening decisions matter.
// ------------------------------------------------------------------------------------------------
#define DM(a, b) __dmul_rn((a), (b))
#define DA(a, b) __dadd_rn((a), (b))
#define DS(a, b) __dsub_rn((a), (b))

__device__ __forceinline__ double det3_rn(const double* A) {
  double c0 = DS(DM(A[4], A[8]), DM(A[5], A[7]));
  double c1 = DS(DM(A[3], A[8]), DM(A[5], A[6]));
  double c2 = DS(DM(A[3], A[7]), DM(A[4], A[6]));
  return DA(DS(DM(A[0], c0), DM(A[1], c1)), DM(A[2], c2));
}

__device__ __forceinline__ void adj3_rn(const double* A, double* C) {
  C[0] = DS(DM(A[4], A[8]), DM(A[5], A[7]));
  C[1] = DS(DM(A[2], A[7]), DM(A[1], A[8]));
  C[2] = DS(DM(A[1], A[5]), DM(A[2], A[4]));
  C[3] = DS(DM(A[5], A[6]), DM(A[3], A[8]));
  C[4] = DS(DM(A[0], A[8]), DM(A[2], A[6]));
  C[5] = DS(DM(A[2], A[3]), DM(A[0], A[5]));
  C[6] = DS(DM(A[3], A[7]), DM(A[4], A[6]));
  C[7] = DS(DM(A[1], A[6]), DM(A[0], A[7]));
  C[8] = DS(DM(A[0], A[4]), DM(A[1], A[3]));
}

__device__ __forceinline__ void matvec3_rn(const double* A, const double* b, double* y) {
#pragma unroll
  for (int k = 0; k < 3; ++k)
    y[k] = DA(DA(DM(A[3 * k + 0], b[0]), DM(A[3 * k + 1], b[1])), DM(A[3 * k + 2], b[2]));
}

// solve3: adj(A) b / det(A)  (gs_dft/integrals/linalg3.py:49-51)
__device__ __forceinline__ void solve3_rn(const double* A, const double* b, double* x) {
  double C[9];
  adj3_rn(A, C);
  double det = det3_rn(A);
  double y[3];
  matvec3_rn(C, b, y);
#pragma unroll
  for (int k = 0; k < 3; ++k) x[k] = __ddiv_rn(y[k], det);
}

// Pair quantities of gs_dft/coulomb/stream.py:203-215, evaluated without FMA contraction in the
// reference's operation order. Outputs A_hat (9), P (3), KN and det(A_hat).
__device__ __forceinline__ void pair_quantities_rn(const double* Ai, const double* Aj,
                                                   const double* mui, const double* muj,
                                                   double Ni, double Nj, double* Ah, double* P,
                                                   double* KN, double* detAh) {
#pragma unroll
  for (int k = 0; k < 9; ++k) Ah[k] = DA(Ai[k], Aj[k]);
  double r1[3], r2[3], rhs[3];
  matvec3_rn(Ai, mui, r1);
  matvec3_rn(Aj, muj, r2);
#pragma unroll
  for (int k = 0; k < 3; ++k) rhs[k] = DA(r1[k], r2[k]);
  double C[9];
  adj3_rn(Ah, C);
  double det = det3_rn(Ah);
  double y[3];
  matvec3_rn(C, rhs, y);
#pragma unroll
  for (int k = 0; k < 3; ++k) P[k] = __ddiv_rn(y[k], det);
  double d[3] = {DS(mui[0], muj[0]), DS(mui[1], muj[1]), DS(mui[2], muj[2])};
  double Ajd[3], s[3], AiAinvAjd[3];
  matvec3_rn(Aj, d, Ajd);
  matvec3_rn(C, Ajd, y);
#pragma unroll
  for (int k = 0; k < 3; ++k) s[k] = __ddiv_rn(y[k], det);
  matvec3_rn(Ai, s, AiAinvAjd);
  double quad = DA(DA(DM(d[0], AiAinvAjd[0]), DM(d[1], AiAinvAjd[1])), DM(d[2], AiAinvAjd[2]));
  double K = exp(-quad);
  *KN = DM(DM(Ni, Nj), K);
  *detAh = det;
}

// ------------------------------------------------------------------------------------------------
// Device: fast FP64 transcendentals for the node loop.
//
// wexp2<B>(a, t2, tab) = w_n 2^(a t2) for a t2 <= 0, table-driven (Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2),
// 1989). x = a t2 is never rounded on its own: kd = fma(a, t2, 1.5*2^(52-B)) rounds it to a multiple
// n/2^B (n exact for |x| < 2^(31-B)), r = fma(a, t2, -n/2^B) is the reduced argument
// (|r| <= 2^-(B+1)), and w_n 2^x = 2^k (w_n 2^(j/2^B)) p(r) with n = 2^B k + j. `tab` is node n's row
// of kExp2WTab<B> in shared memory, so the quadrature weight comes for free; p is the Taylor
// polynomial kExp2T5 (B = 6) or kExp2T4 (B = 8). Results below 2^-1000 are flushed to zero by
// integer selects (nothing that small reaches a sum). 8-9 FP64 operations.
// ------------------------------------------------------------------------------------------------
template <int B>
__device__ __forceinline__ double wexp2(double a, double t2, const double* __restrict__ tab) {
  const double kRound = 6755399441055744.0 / (double)(1 << B);  // 1.5 * 2^(52-B)
  const double kd = fma(a, t2, kRound);
  const int n = __double2loint(kd);
  const double nd = kd - kRound;
  const double r = fma(a, t2, -nd);
  double p;
  if (B == 8) {
    p = kExp2T4[4];
    p = fma(p, r, kExp2T4[3]);
    p = fma(p, r, kExp2T4[2]);
    p = fma(p, r, kExp2T4[1]);
    p = fma(p, r, kExp2T4[0]);
  } else {
    p = kExp2T5[5];
    p = fma(p, r, kExp2T5[4]);
    p = fma(p, r, kExp2T5[3]);
    p = fma(p, r, kExp2T5[2]);
    p = fma(p, r, kExp2T5[1]);
    p = fma(p, r, kExp2T5[0]);
  }
  const double v = tab[n & ((1 << B) - 1)] * p;
  const int k = n >> B;
  const bool keep = k >= -1000;
  const int hi = keep ? __double2hiint(v) + (k << 20) : 0;
  const int lo = keep ? __double2loint(v) : 0;
  return __hiloint2double(hi, lo);
}

// wexp2x<B>(x, tab) = w 2^x for an already formed exponent x (the product rounded once), clamped
// at -2048 so that the table index and the exponent field stay in range for any x <= 0 (2^-2048 is
// flushed to zero). For the exact (pair|pair) kernels, whose exponents reach far beyond the
// 3-centre ones; the rounding of x adds a relative error |x| 2^-53 to a term of size 2^x.
template <int B>
__device__ __forceinline__ double wexp2x(double x, const double* __restrict__ tab) {
  const double kRound = 6755399441055744.0 / (double)(1 << B);
  x = fmax(x, -2048.0);
  const double kd = x + kRound;
  const int n = __double2loint(kd);
  const double r = x - (kd - kRound);
  double p = kExp2T5[5];
  p = fma(p, r, kExp2T5[4]);
  p = fma(p, r, kExp2T5[3]);
  p = fma(p, r, kExp2T5[2]);
  p = fma(p, r, kExp2T5[1]);
  p = fma(p, r, kExp2T5[0]);
  static_assert(B == 6, "wexp2x uses the degree-5 polynomial of the 64-entry tables");
  const double v = tab[n & ((1 << B) - 1)] * p;
  const int k = n >> B;
  const bool keep = k >= -1000;
  const int hi = keep ? __double2hiint(v) + (k << 20) : 0;
  const int lo = keep ? __double2loint(v) : 0;
  return __hiloint2double(hi, lo);
}

// Copy the per-node weighted tables kExp2WTab<B> (GSDFT_NQUAD x 2^B doubles) into shared memory
// (all threads; the caller synchronises before use).
template <int B>
__device__ __forceinline__ void load_wexp2_tables(double* dst) {
  const double* src = (B == 8) ? kExp2WTab8 : kExp2WTab6;
  for (int k = threadIdx.x; k < GSDFT_NQUAD * (1 << B); k += blockDim.x) dst[k] = src[k];
}

// rsqrt_pos(p) = 1/sqrt(p), p > 0 normal. Seed from the PTX instruction rsqrt.approx.ftz.f64, then one
// third-order (Halley-type) correction y = y0 (1 + e/2 + 3e^2/8), e = 1 - p y0^2, which triples the
// number of correct bits of the seed.
__device__ __forceinline__ double rsqrt_pos(double p) {
  double y0;
#if GSDFT_RSQRT_SEED_F32
  y0 = (double)rsqrtf(__double2float_rn(p));
#else
  asm("rsqrt.approx.ftz.f64 %0, %1;" : "=d"(y0) : "d"(p));
#endif
  double t = p * y0;
  double e = fma(-t, y0, 1.0);
  double c = fma(0.375, e, 0.5);
  c = c * e;
  return fma(y0, c, y0);
}

// ------------------------------------------------------------------------------------------------
// Device: bulk copies global -> shared (the non-tensor TMA path, cp.async.bulk, no multicast) with
// an mbarrier transaction count, and a BOUNDED wait. A wait that runs out sets the library's device
// status word and the caller abandons its loop; nothing spins forever.
// ------------------------------------------------------------------------------------------------
// Each translation unit that waits on mbarriers owns one status word (whole-program compilation,
// no relocatable device code); gsdft_device_status() reads all of them.
static __device__ int g_device_status;

constexpr int kStatusMbarTimeout = 1;
// A wait gives up after 2 s of wall-clock time (the %globaltimer nanosecond clock), and in any case
// after 2^30 polls; a healthy tile copy completes in microseconds.
constexpr unsigned long long kMbarTimeoutNs = 2000000000ull;
constexpr unsigned kMbarMaxPolls = 1u << 30;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Returns true once phase `parity` of `bar` has completed; false (status set) after the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  unsigned long long t0 = 0;
  for (unsigned it = 0; it < kMbarMaxPolls; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255u) == 0u) {
      const unsigned long long t = global_ns();
      if (it == 0u) t0 = t;
      else if (t - t0 > kMbarTimeoutNs) break;
    }
  }
  atomicExch(&g_device_status, kStatusMbarTimeout);
  return false;
}

// ------------------------------------------------------------------------------------------------
// Node screening of the 20-node Laplace sum. Along the nodes (t ascending) the exponent
//   E(t) = t^2 beta sum_k lam_k dp2_k / Gamma_k(t),   Gamma_k = beta lam_k + t^2 (beta + lam_k)
// never decreases (each t^2 / Gamma_k(t) does), and the prefactor (G0 G1 G2)^(-1/2) never
// increases. So once E has grown by more than kNodeSkipLog2 (in log2 units) past its value at the
// first node, every later node contributes at most (sum_m w_m / w_0) 2^-kNodeSkipLog2 ~ 1e-21 of
// the first node's term: below the last bit of the sum. The integral kernels then stop the node loop
// for a warp once all of its lanes (every (aux, pair) it holds) are that far along; the check is
// warp-uniform, so no lane diverges. The reverse-pass sums also weight nodes by t^2 / Gamma_k and
// t^4 / (Gamma_k Gamma_l) (bounded, increasing in t); their truncation error measured over 2.5e6
// (aux, pair) samples of the water clusters fell from 1e-12 to below one rounding as the threshold
// rose from 40 to 48 nats, and the threshold here is 60 nats. A CPU emulation of the same rule is
// in the tests. Distant (aux, pair) combinations dominate large systems: at configuration 3 a warp
// evaluates ~10 of the 20 nodes, at configuration 4 ~7; at a compact molecule all 20.
// gsdft_set_node_screening(0) turns it off (every node evaluated, as the reference does).
// ------------------------------------------------------------------------------------------------
// The warp checks after node kNodeSkipFirst and then every kNodeSkipEvery nodes: a check is a vote
// and a branch, which also ends the compiler's interleaving of consecutive nodes, so checking
// every node costs ~10% where nothing can be skipped (compact molecules).
#ifndef GSDFT_SKIP_FIRST
#define GSDFT_SKIP_FIRST 5
#endif
#ifndef GSDFT_SKIP_EVERY
#define GSDFT_SKIP_EVERY 2
#endif
constexpr double kNodeSkipLog2 = 87.0;  // 2^-87 = e^-60.3
constexpr int kNodeSkipFirst = GSDFT_SKIP_FIRST;  // nodes 0..kNodeSkipFirst are always evaluated
constexpr int kNodeSkipEvery = GSDFT_SKIP_EVERY;
__host__ __device__ constexpr bool node_check(int n) {
  return n >= kNodeSkipFirst && (n - kNodeSkipFirst) % kNodeSkipEvery == 0 && n + 1 < 20;
}
// Host: the skip threshold the launches pass (kNodeSkipLog2, or +inf when screening is off).
double node_skip_threshold();

constexpr double kPi = 3.141592653589793;
constexpr double kLog2e = 1.4426950408889634;           // log2(e)
// 2 pi^3 / sqrt(pi), the 3-centre prefactor of gs_dft/coulomb/ri.py:150
constexpr double kPref = 34.986836655249725;

}  // namespace gsdft
