// Launch accounting and the FP64 FMA throughput probe.
#include <atomic>

#include "common.cuh"

namespace gsdft {

static std::atomic<int64_t> g_launches{0};
static std::atomic<int> g_node_screening{1};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int device_sms() {
  static const int sms = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return sms;
}

double node_skip_threshold() {
  return g_node_screening.load(std::memory_order_relaxed) ? kNodeSkipLog2 : (double)INFINITY;
}

int node_evals_forward(unsigned long long* out, int clear);
int node_evals_vjp(unsigned long long* out, int clear);

// 16 independent FMA chains per thread; the coefficients keep every value finite.
__global__ void dfma_probe_kernel(double* out, int64_t iters) {
  double a[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) a[k] = 1.0 + 1e-3 * (threadIdx.x + k);
  const double m = 0.999999999, c = 1e-9;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = fma(a[k], m, c);
  }
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < 16; ++k) s += a[k];
  out[blockIdx.x * (int64_t)blockDim.x + threadIdx.x] = s;
}

}  // namespace gsdft

using namespace gsdft;

extern "C" int64_t gsdft_kernel_launches(void) { return g_launches.load(); }

extern "C" int gsdft_dfma_probe(double* out, int64_t iters, int blocks, int threads,
                                gsdft_stream_t stream) {
  GSDFT_REQUIRE(out && iters > 0 && blocks > 0 && threads > 0 && threads <= 1024, "bad arguments");
  dfma_probe_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(out, iters);
  GSDFT_LAUNCHED("dfma_probe");
  return GSDFT_OK;
}

extern "C" int gsdft_set_node_screening(int enabled) {
  g_node_screening.store(enabled ? 1 : 0, std::memory_order_relaxed);
  return GSDFT_OK;
}

extern "C" int gsdft_node_screening(void) { return g_node_screening.load(); }

extern "C" int gsdft_node_evals(uint64_t* forward_host, uint64_t* reverse_host, int clear) {
  GSDFT_REQUIRE(forward_host && reverse_host, "null pointer");
  GSDFT_CUDA(cudaDeviceSynchronize());
  unsigned long long f = 0, r = 0;
  int rc = node_evals_forward(&f, clear);
  if (rc) return rc;
  rc = node_evals_vjp(&r, clear);
  if (rc) return rc;
  *forward_host = f;
  *reverse_host = r;
  return GSDFT_OK;
}
