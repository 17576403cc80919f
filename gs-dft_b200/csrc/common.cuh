// Shared device helpers and host error plumbing for the gs-dft B200 RI-J library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
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
// exp2_nonpos(x) = 2^x for x <= 0. Reduction x = k + f with k = rint(x) (the 1.5*2^52 rounding
// constant), 2^f from the degree-11 Chebyshev interpolant kExp2C (gen_constants.py), then the
// exponent field is raised by k. x is clamped at -1020 so the result stays normal (the clamped
// value, ~1e-307, is far below anything that reaches a sum).
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ double exp2_nonpos(double x) {
  x = fmax(x, -1020.0);
  const double kRound = 6755399441055744.0;   // 1.5 * 2^52
  double kd = x + kRound;
  int k = __double2loint(kd);
  kd = kd - kRound;
  double f = x - kd;
  double p = kExp2C[11];
  p = fma(p, f, kExp2C[10]);
  p = fma(p, f, kExp2C[9]);
  p = fma(p, f, kExp2C[8]);
  p = fma(p, f, kExp2C[7]);
  p = fma(p, f, kExp2C[6]);
  p = fma(p, f, kExp2C[5]);
  p = fma(p, f, kExp2C[4]);
  p = fma(p, f, kExp2C[3]);
  p = fma(p, f, kExp2C[2]);
  p = fma(p, f, kExp2C[1]);
  p = fma(p, f, kExp2C[0]);
  int hi = __double2hiint(p) + (k << 20);
  return __hiloint2double(hi, __double2loint(p));
}

// rsqrt_pos(p) = 1/sqrt(p), p > 0 normal. Seed from the PTX instruction rsqrt.approx.f64, then one
// third-order (Halley-type) correction y = y0 (1 + e/2 + 3e^2/8), e = 1 - p y0^2, which triples the
// number of correct bits of the seed.
__device__ __forceinline__ double rsqrt_pos(double p) {
  double y0;
  asm("rsqrt.approx.f64 %0, %1;" : "=d"(y0) : "d"(p));
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
constexpr long long kMbarMaxPolls = 1LL << 22;

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
  for (long long it = 0; it < kMbarMaxPolls; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicExch(&g_device_status, kStatusMbarTimeout);
  return false;
}

constexpr double kPi = 3.141592653589793;
constexpr double kLog2e = 1.4426950408889634;           // log2(e)
// 2 pi^3 / sqrt(pi), the 3-centre prefactor of gs_dft/coulomb/ri.py:150
constexpr double kPref = 34.986836655249725;

}  // namespace gsdft
