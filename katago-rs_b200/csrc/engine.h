// The forward-pass engine of one compute handle: device weights, activation buffers and the launch plan of one
// KataGo net on one GPU, for batches of up to max_batch boards.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "model.h"
#include "../../include/katago_cuda.h"

namespace kc {

enum Precision : int { PREC_F32 = 0, PREC_F16 = 1, PREC_BF16 = 2 };

// Launch classes for per-kernel timing (kc_handle_profile).
enum LaunchClass : int { CLS_CONV3 = 0, CLS_LINEAR = 1, CLS_STEM = 2, CLS_ATTN = 3, CLS_OTHER = 4, CLS_COUNT = 5 };

struct OutputLayout {
  int row_len = 0, policy_off = 0, value_off = 0, score_off = 0, own_off = 0;
};

class Engine {
 public:
  Engine(const ModelDesc& m, int device, int max_batch, int precision);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  // Enqueue the forward pass of n boards on `stream`: inputs and outputs are device pointers (NCHW float32 spatial
  // [n][C][361], global [n][G], meta [n][192] or null; out [n][row_len] float32). Instead of d_spatial: bit-packed
  // planes d_bits [n][C][12] with one symmetry per board d_sym [n], applied on the device.
  void forward(int n, cudaStream_t stream, const float* d_spatial, const float* d_global, const float* d_meta,
               float* d_out, const uint32_t* d_bits = nullptr, const int* d_sym = nullptr);

  const OutputLayout& layout() const { return layout_; }
  int max_batch() const { return max_batch_; }
  int precision() const { return precision_; }
  int device() const { return device_; }
  // Kernel launches of a forward pass of n boards (an entry of the plan may choose between forms by batch).
  int launches_per_forward(int n) const {
    int k = 0;
    for (const Launch& l : plan_) k += l.kernels ? l.kernels(n) : 1;
    return k;
  }
  // Non-zero after a kernel reported a device-side error (a bounded wait expired).
  int device_error();
  int* error_word();  // device address of the error word kernels write (first error wins)
  void clear_device_error();

  void set_profiling(bool on);
  // Accumulate the per-launch event times of the last profiled forward (waits for it), then report.
  void profile(double* ms, int64_t* launches, int n);
  void reset_profile();
  void set_use_graphs(bool on) { use_graphs_ = on; }

  struct Impl;
  struct Launch {
    int cls;
    std::function<void(cudaStream_t, int)> fn;
    std::function<int(int)> kernels;  // kernels fn launches for n boards (empty: one)
  };

 private:
  int device_, max_batch_, precision_;
  OutputLayout layout_;
  std::vector<Launch> plan_;
  std::unique_ptr<Impl> impl_;
  bool use_graphs_ = true;
  bool profiling_ = false;
  bool prof_pending_ = false;
  std::vector<cudaEvent_t> prof_events_;  // 2 per launch
  double prof_ms_[CLS_COUNT] = {0};
  int64_t prof_n_[CLS_COUNT] = {0};
  template <typename T> void build_model(const ModelDesc& m);
  void run_plan(int n, cudaStream_t stream, bool events);
  void collect_profile();
};

// copy_outputs on the device (io.cu): the forward's raw output rows [n][row_len] -> NNOutput rows
// [n][KC_FINISHED_ROW_LEN] (policy with the optimism mix and the inverse symmetry, value, misc by model version,
// ownership with the inverse symmetry).
struct FinishParams {
  const float* rows = nullptr;
  int row_len = 0, policy_off = 0, value_off = 0, score_off = 0, own_off = 0;
  int P = 1, version = 0, has_own = 1;
  const int* sym = nullptr;
  const float* optimism = nullptr;
  float* out = nullptr;
};
void launch_finish_outputs(const FinishParams& p, int n, cudaStream_t st);

// Failure-detection self-test (ops.cu): enqueue on `st` one kernel whose bounded wait runs out after
// `limit_cycles` SM cycles and records DEV_TIMEOUT_TEST in `err`.
void launch_wait_selftest(int* err, long long limit_cycles, cudaStream_t st);

// Algorithmic FLOPs per board (direct-convolution MACs x 2 over the 361 points, attention over 361 x 361).
void model_flops(const ModelDesc& m, double* total, double* conv3x3);

}  // namespace kc
