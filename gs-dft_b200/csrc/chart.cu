// Splat chart A = R(q) diag(exp l) R(q)^T, N = (8 det A / pi^3)^(1/4), and its reverse.
// Reference: gs_dft/basis/spectral.py:33-40 (quat_to_rotation), :71-76 (A), :78-82 (norm).
#include <stdarg.h>

#include "common.cuh"

namespace gsdft {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// Rotation of the normalised quaternion, row-major (gs_dft/basis/spectral.py:33-40).
__device__ __forceinline__ void quat_rotation(const double* q4, double* R, double* qh,
                                              double* nrm) {
  double n = sqrt(DA(DA(DA(DM(q4[0], q4[0]), DM(q4[1], q4[1])), DM(q4[2], q4[2])),
                     DM(q4[3], q4[3])));
  double den = DA(n, 1e-12);
  double w = __ddiv_rn(q4[0], den), x = __ddiv_rn(q4[1], den);
  double y = __ddiv_rn(q4[2], den), z = __ddiv_rn(q4[3], den);
  qh[0] = w; qh[1] = x; qh[2] = y; qh[3] = z;
  *nrm = n;
  R[0] = DS(1.0, DM(2.0, DA(DM(y, y), DM(z, z))));
  R[1] = DM(2.0, DS(DM(x, y), DM(w, z)));
  R[2] = DM(2.0, DA(DM(x, z), DM(w, y)));
  R[3] = DM(2.0, DA(DM(x, y), DM(w, z)));
  R[4] = DS(1.0, DM(2.0, DA(DM(x, x), DM(z, z))));
  R[5] = DM(2.0, DS(DM(y, z), DM(w, x)));
  R[6] = DM(2.0, DS(DM(x, z), DM(w, y)));
  R[7] = DM(2.0, DA(DM(y, z), DM(w, x)));
  R[8] = DS(1.0, DM(2.0, DA(DM(x, x), DM(y, y))));
}

__global__ void splat_quantities_kernel(const double* __restrict__ quat,
                                        const double* __restrict__ log_scale, int64_t M,
                                        double* __restrict__ A9, double* __restrict__ N) {
  int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (m >= M) return;
  double q4[4] = {quat[4 * m], quat[4 * m + 1], quat[4 * m + 2], quat[4 * m + 3]};
  double R[9], qh[4], nrm;
  quat_rotation(q4, R, qh, &nrm);
  double l0 = log_scale[3 * m], l1 = log_scale[3 * m + 1], l2 = log_scale[3 * m + 2];
  double a[3] = {exp(l0), exp(l1), exp(l2)};
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      A9[9 * m + 3 * i + k] = DA(DA(DM(DM(R[3 * i + 0], a[0]), R[3 * k + 0]),
                                    DM(DM(R[3 * i + 1], a[1]), R[3 * k + 1])),
                                 DM(DM(R[3 * i + 2], a[2]), R[3 * k + 2]));
  double detA = exp(DA(DA(l0, l1), l2));
  const double pi3 = 31.006276680299816;  // pi ** 3 as the reference's float computes it
  N[m] = pow(__ddiv_rn(DM(8.0, detA), pi3), 0.25);
}

// Reverse of the chart. gA6 = symmetric cotangent [xx,yy,zz,xy,xz,yz].
__global__ void chart_vjp_kernel(const double* __restrict__ quat,
                                 const double* __restrict__ log_scale,
                                 const double* __restrict__ gA6, const double* __restrict__ gN,
                                 int64_t M, double* __restrict__ g_quat,
                                 double* __restrict__ g_log) {
  int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (m >= M) return;
  double q4[4] = {quat[4 * m], quat[4 * m + 1], quat[4 * m + 2], quat[4 * m + 3]};
  double R[9], qh[4], n;
  quat_rotation(q4, R, qh, &n);
  double l[3] = {log_scale[3 * m], log_scale[3 * m + 1], log_scale[3 * m + 2]};
  double a[3] = {exp(l[0]), exp(l[1]), exp(l[2])};
  const double* g6 = gA6 + 6 * m;
  double S[9] = {g6[0], g6[3], g6[4], g6[3], g6[1], g6[5], g6[4], g6[5], g6[2]};
  double Nm = pow(exp(l[0] + l[1] + l[2]) * 8.0 / 31.006276680299816, 0.25);
  // gR = 2 S R diag(a);  g_l_k = a_k r_k^T S r_k + gN N / 4
  double SR[9];
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 3; ++k)
      SR[3 * i + k] = S[3 * i] * R[k] + S[3 * i + 1] * R[3 + k] + S[3 * i + 2] * R[6 + k];
  double gl[3];
  for (int k = 0; k < 3; ++k)
    gl[k] = a[k] * (R[k] * SR[k] + R[3 + k] * SR[3 + k] + R[6 + k] * SR[6 + k]) + gN[m] * Nm * 0.25;
  double g[9];
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 3; ++k) g[3 * i + k] = 2.0 * SR[3 * i + k] * a[k];
  double w = qh[0], x = qh[1], y = qh[2], z = qh[3];
  double gw = 2 * (-z * g[1] + y * g[2] + z * g[3] - x * g[5] - y * g[6] + x * g[7]);
  double gx = 2 * (y * g[1] + z * g[2] + y * g[3] - 2 * x * g[4] - w * g[5] + z * g[6] + w * g[7] -
                   2 * x * g[8]);
  double gy = 2 * (-2 * y * g[0] + x * g[1] + w * g[2] + x * g[3] + z * g[5] - w * g[6] +
                   z * g[7] - 2 * y * g[8]);
  double gz = 2 * (-2 * z * g[0] - w * g[1] + x * g[2] + w * g[3] - 2 * z * g[4] + y * g[5] +
                   x * g[6] + y * g[7]);
  double den = n + 1e-12;
  double dot = q4[0] * gw + q4[1] * gx + q4[2] * gy + q4[3] * gz;
  double coef = dot / (fmax(n, 1e-300) * den * den);
  g_quat[4 * m + 0] = gw / den - q4[0] * coef;
  g_quat[4 * m + 1] = gx / den - q4[1] * coef;
  g_quat[4 * m + 2] = gy / den - q4[2] * coef;
  g_quat[4 * m + 3] = gz / den - q4[3] * coef;
  g_log[3 * m + 0] = gl[0];
  g_log[3 * m + 1] = gl[1];
  g_log[3 * m + 2] = gl[2];
}

}  // namespace gsdft

using namespace gsdft;

extern "C" const char* gsdft_last_error_string(void) { return g_err; }
extern "C" int gsdft_version(void) { return GSDFT_ABI_VERSION; }

extern "C" int gsdft_splat_quantities(const double* quat, const double* log_scale, int64_t M,
                                      double* A9, double* N, gsdft_stream_t stream) {
  GSDFT_REQUIRE(M >= 0, "M < 0");
  if (M == 0) return GSDFT_OK;
  GSDFT_REQUIRE(quat && log_scale && A9 && N, "null pointer");
  splat_quantities_kernel<<<grid_1d(M, 128), 128, 0, (cudaStream_t)stream>>>(quat, log_scale, M,
                                                                            A9, N);
  GSDFT_LAUNCHED("splat_quantities");
  return GSDFT_OK;
}

extern "C" int gsdft_chart_vjp(const double* quat, const double* log_scale, const double* gA6,
                               const double* gN, int64_t M, double* g_quat, double* g_log_scale,
                               gsdft_stream_t stream) {
  GSDFT_REQUIRE(M >= 0, "M < 0");
  if (M == 0) return GSDFT_OK;
  GSDFT_REQUIRE(quat && log_scale && gA6 && gN && g_quat && g_log_scale, "null pointer");
  chart_vjp_kernel<<<grid_1d(M, 128), 128, 0, (cudaStream_t)stream>>>(quat, log_scale, gA6, gN, M,
                                                                     g_quat, g_log_scale);
  GSDFT_LAUNCHED("chart_vjp");
  return GSDFT_OK;
}
