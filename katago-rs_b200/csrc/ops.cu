// Standalone operator entry points of the katago-rs B200 backend (C ABI): KataGo's masked global pooling followed
// by the gpool-to-bias matmul, on reference-layout (NCHW float32) device tensors. This is the computation of a
// gpool block's bias branch and of the policy head's g1 branch (tools/bin2onnx/bin2onnx.py gpool :1222-1230 and
// the matmul that follows it at :1255 and :1501), for callers that run it outside a whole forward pass.

#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <string>

#include "../../include/katago_cuda.h"
#include "common.h"
#include "kernels.cuh"

namespace kc {

// pooled[b][c], [C + c], [2C + c] = mean, mean * (sqrt(area) - 14) / 10, max(x + (mask * 1e4 - 1e4)) over the
// board's 361 points of channel c (x already masked). One warp per (board, channel); block (32, 8).
__global__ void gpool_nchw_kernel(const float* __restrict__ x, const float* __restrict__ mask, int n, int C,
                                  float* __restrict__ pooled) {
  const int b = blockIdx.x;
  const int c = blockIdx.y * 8 + threadIdx.y;
  if (c >= C) return;
  const float* xr = x + ((size_t)b * C + c) * 361;
  const float* mr = mask + (size_t)b * 361;
  float s = 0.0f, ms = 0.0f, mx = -INFINITY;
  for (int i = threadIdx.x; i < 361; i += 32) {
    const float v = xr[i], m = mr[i];
    s += v;
    ms += m;
    const float biasv = m * 1e4f - 1e4f;
    mx = fmaxf(mx, v + biasv);
  }
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ms += __shfl_xor_sync(0xffffffffu, ms, o);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (threadIdx.x == 0) {
    const float mean = s / ms;
    const float cen = sqrtf(ms) - 14.0f;
    float* o = pooled + (size_t)b * 3 * C;
    o[c] = mean;
    o[C + c] = mean * (cen * 0.1f);
    o[2 * C + c] = mx;
  }
}

void check_gpool_args(const float* x, const float* mask, int n, int c, const float* w, int oc, const float* out) {
  if (!x || !mask || !w || !out) fail(KC_ERR_INVALID, "CUDA backend: gpool: null tensor");
  if (n < 1 || c < 1 || oc < 1) fail(KC_ERR_INVALID, "CUDA backend: gpool: sizes must be positive");
  if (3 * c > 12 * 1024) fail(KC_ERR_INVALID, "CUDA backend: gpool: 3 * channels above 12288");
}

// fc_kernel<1> with up to 3 * 4096 input floats: above the 48 KB of shared memory a kernel gets without opting in
// (its inputs plus its static reduction buffer). Once per device; not a stream operation.
void allow_fc_smem() {
  static std::mutex mu;
  static std::set<int> done;
  int dev = 0;
  KC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(dev)) return;
  KC_CUDA(cudaFuncSetAttribute(fc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 12 * 1024 * sizeof(float)));
  done.insert(dev);
}

// pooled (scratch [n][3c]) -> out = pooled x w ([3c][oc]), both launched on `st`.
void launch_gpool_fc(const float* x, const float* mask, int n, int c, const float* w, int oc, float* out,
                     float* pooled, cudaStream_t st) {
  gpool_nchw_kernel<<<dim3(n, (c + 7) / 8), dim3(32, 8), 0, st>>>(x, mask, n, c, pooled);
  KC_CUDA(cudaGetLastError());
  allow_fc_smem();
  fc_kernel<1><<<dim3(n, (oc + 31) / 32), FC_THREADS, 3 * c * sizeof(float), st>>>(pooled, 3 * c, 3 * c, w, oc,
                                                                              nullptr, 0, out, oc, 0, 1, n);
  KC_CUDA(cudaGetLastError());
}

// Failure-detection self-test: one thread waits on an mbarrier that nothing arrives at, with the bounded wait
// every kernel of the forward pass uses but a short limit; when the limit runs out it records `code` in the error
// word (first error wins) and the kernel returns.
__global__ void wait_selftest_kernel(int* err, long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, err, DEV_TIMEOUT_TEST, limit_cycles);
  __syncthreads();
}

void launch_wait_selftest(int* err, long long limit_cycles, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(err, limit_cycles);
  KC_CUDA(cudaGetLastError());
}

}  // namespace kc

namespace {
template <typename F>
int guard_op(F&& f) {
  try {
    f();
    kc::set_last_error("");
    return KC_OK;
  } catch (const kc::Error& e) {
    kc::set_last_error(e.what());
    return e.status;
  }
}
}  // namespace

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free variant. Its scratch (the pooled [n][3c] vector) is this fixed device array, present on every
// GPU that loads the library for as long as the process lives. Host code must not pass the symbol itself to a
// kernel: on the host, g_gpool_scratch names a host-side stand-in, not device memory. The device address is looked
// up once per device with cudaGetSymbolAddress (with that device current) and cached.
// ---------------------------------------------------------------------------------------------------------------
static __device__ __align__(256) float g_gpool_scratch[KC_GPOOL_NOALLOC_MAX_FLOATS];

namespace {
std::mutex g_scratch_mu;
float* g_scratch_addr[128] = {nullptr};

float* gpool_scratch_for_current_device() {
  int dev = -1;
  KC_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 128) kc::fail(KC_ERR_INVALID, "CUDA backend: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    KC_CUDA(cudaGetSymbolAddress(&p, g_gpool_scratch));
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  return g_scratch_addr[dev];
}
}  // namespace

extern "C" int kc_gpool_fc_noalloc(const float* d_x, const float* d_mask, int n, int c, const float* d_w, int oc,
                                   float* d_out, void* stream) {
  return guard_op([&] {
    kc::check_gpool_args(d_x, d_mask, n, c, d_w, oc, d_out);
    if ((long long)n * 3 * c > KC_GPOOL_NOALLOC_MAX_FLOATS)
      kc::fail(KC_ERR_INVALID, "CUDA backend: kc_gpool_fc_noalloc: n * 3 * c = " + std::to_string((long long)n * 3 * c) +
                                   " floats exceeds its fixed scratch of " +
                                   std::to_string(KC_GPOOL_NOALLOC_MAX_FLOATS) + " floats; use kc_gpool_fc");
    float* scratch = gpool_scratch_for_current_device();
    // every entry of the scratch that the matmul reads is written by the pooling kernel first: nothing to clear
    kc::launch_gpool_fc(d_x, d_mask, n, c, d_w, oc, d_out, scratch, static_cast<cudaStream_t>(stream));
  });
}

extern "C" int kc_gpool_fc(const float* d_x, const float* d_mask, int n, int c, const float* d_w, int oc,
                           float* d_out, void* stream) {
  return guard_op([&] {
    kc::check_gpool_args(d_x, d_mask, n, c, d_w, oc, d_out);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* pooled = nullptr;
    KC_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&pooled), (size_t)n * 3 * c * sizeof(float), st));
    try {
      kc::launch_gpool_fc(d_x, d_mask, n, c, d_w, oc, d_out, pooled, st);
    } catch (...) {
      cudaFreeAsync(pooled, st);
      throw;
    }
    KC_CUDA(cudaFreeAsync(pooled, st));
  });
}
