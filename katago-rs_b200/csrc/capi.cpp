// The C ABI of the katago-rs B200 backend (include/katago_cuda.h): models, contexts, handles, the asynchronous
// enqueue/wait pair, and the whole get_output of the reference backend with its host-side symmetry handling.
//
// Reference behaviour followed here (crates/katago-nn-burn/src/backend.rs): create_compute_context rejects
// nnXLen/nnYLen != 19 (:327-333), create_compute_handle rejects NHWC inputs (:371-373), get_output copies each row
// with its symmetry (:497-546), runs the net, then mixes policy optimism, undoes the symmetry and fills the score
// fields by model version (:622-731).

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <string>
#include <vector>

#include "common.h"
#include "engine.h"
#include "model.h"

namespace kc {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }

}  // namespace kc

struct kc_model {
  kc::ModelDesc desc;
};

struct kc_context {
  std::vector<int> gpus;
  int nn_x_len = 19, nn_y_len = 19;
  int precision = kc::PREC_F32;
  const kc_model* model = nullptr;
};

struct kc_handle {
  const kc_model* model = nullptr;
  std::unique_ptr<kc::Engine> engine;
  int device = 0;
  int max_batch = 0;
  int n_spatial = 0, n_global = 0, n_meta = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
  float* h_spatial = nullptr;  // pinned
  float* h_global = nullptr;
  float* h_meta = nullptr;
  float* h_out = nullptr;
  int* h_err = nullptr;
  float* d_spatial = nullptr;
  float* d_global = nullptr;
  float* d_meta = nullptr;
  float* d_out = nullptr;
  // Bit-packed input staging: one pinned block and its device copy with the same layout, moved by one copy:
  // [symmetry int32 x max_batch | optimism float x max_batch | global x max_batch G | meta x max_batch M |
  //  spatial bits uint32 x max_batch C 12]
  uint8_t* h_pk = nullptr;
  uint8_t* d_pk = nullptr;
  size_t pk_prefix = 0, pk_row_bits = 0;  // bytes before the bits; bytes of one row's bits
  int32_t* pk_sym(uint8_t* base) const { return reinterpret_cast<int32_t*>(base); }
  float* pk_opt(uint8_t* base) const { return reinterpret_cast<float*>(base + 4 * (size_t)max_batch); }
  float* pk_global(uint8_t* base) const { return pk_opt(base) + max_batch; }
  float* pk_meta(uint8_t* base) const { return pk_global(base) + (size_t)max_batch * n_global; }
  uint32_t* pk_bits(uint8_t* base) const { return reinterpret_cast<uint32_t*>(base + pk_prefix); }
  // NNOutput rows of the device copy_outputs: [max_batch][KC_FINISHED_ROW_LEN]
  float* d_fin = nullptr;
  float* h_fin = nullptr;
  bool last_finished = false;  // the last enqueue read back NNOutput rows (h_fin) instead of raw rows (h_out)
  int last_n = 0;
  bool pending = false;
  // host time of the last completion mark and a running estimate of how long a batch takes from there, per batch
  // size class: a waiter sleeps through most of that and polls the rest
  std::chrono::steady_clock::time_point t_mark;
  double est_us[2] = {0.0, 0.0};  // batches of up to / above half the maximum
  bool mark_is_batch = false;     // the last mark follows a forward pass (kc_synchronize's marks do not count)

  std::vector<float> scratch;  // get_output: one row's symmetric copy

  ~kc_handle() {
    if (stream) {
      cudaSetDevice(device);
      cudaStreamSynchronize(stream);
    }
    engine.reset();
    if (done) cudaEventDestroy(done);
    if (stream) cudaStreamDestroy(stream);
    cudaFreeHost(h_spatial);
    cudaFreeHost(h_global);
    cudaFreeHost(h_meta);
    cudaFreeHost(h_out);
    cudaFreeHost(h_err);
    cudaFreeHost(h_pk);
    cudaFreeHost(h_fin);
    cudaFree(d_pk);
    cudaFree(d_fin);
    cudaFree(d_spatial);
    cudaFree(d_global);
    cudaFree(d_meta);
    cudaFree(d_out);
  }
};

namespace {

using kc::Error;
using kc::fail;

template <typename F>
int guard(F&& f) {
  try {
    f();
    kc::set_last_error("");
    return KC_OK;
  } catch (const Error& e) {
    kc::set_last_error(e.what());
    return e.status;
  } catch (const std::exception& e) {
    kc::set_last_error(std::string("CUDA backend: ") + e.what());
    return KC_ERR_INVALID;
  }
}

void need(const void* p, const char* what) {
  if (!p) fail(KC_ERR_INVALID, std::string("CUDA backend: ") + what + " is null");
}

// SymmetryHelpers copy_with_symmetry, NCHW branch (nninputs.rs:756-831): a symmetry is 3 bits flipY (bit 0),
// flipX (bit 1), transpose (bit 2), applied in that order; `reverse` applies the inverse (copyOutputsWithSymmetry).
void copy_with_symmetry(const float* src, float* dst, int n_size, int h_size, int w_size, int c_size, int symmetry,
                        bool reverse) {
  bool transpose = (symmetry & 0x4) != 0 && h_size == w_size;
  bool flip_x = (symmetry & 0x2) != 0;
  bool flip_y = (symmetry & 0x1) != 0;
  if (transpose && !reverse) std::swap(flip_x, flip_y);
  const int nc_size = n_size * c_size;
  const int nc_stride = h_size * w_size;
  const int h_stride = w_size, w_stride = 1;
  int h_base_new = 0, h_stride_new = h_stride, w_base_new = 0, w_stride_new = w_stride;
  if (flip_y) {
    h_base_new = (h_size - 1) * h_stride_new;
    h_stride_new = -h_stride_new;
  }
  if (flip_x) {
    w_base_new = (w_size - 1) * w_stride_new;
    w_stride_new = -w_stride_new;
  }
  if (transpose) std::swap(h_stride_new, w_stride_new);
  for (int nc = 0; nc < nc_size; nc++)
    for (int h = 0; h < h_size; h++) {
      int nch_old = nc * nc_stride + h * h_stride;
      int nch_new = nc * nc_stride + h_base_new + h * h_stride_new;
      for (int w = 0; w < w_size; w++) dst[nch_new + w_base_new + w * w_stride_new] = src[nch_old + w * w_stride];
    }
}

int resolve_precision(int precision, const kc::ModelDesc& m) {
  if (precision == KC_PRECISION_AUTO) return m.has_any_transformer_blocks() ? kc::PREC_BF16 : kc::PREC_F16;
  if (precision < 0 || precision > 2) fail(KC_ERR_INVALID, "CUDA backend: unknown precision " + std::to_string(precision));
  return precision;
}

void check_device(int dev) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    fail(KC_ERR_NO_DEVICE, "CUDA backend: no CUDA device available");
  }
  if (dev < 0 || dev >= count) fail(KC_ERR_INVALID, "CUDA backend: gpu index " + std::to_string(dev) + " out of range");
  cudaDeviceProp prop;
  KC_CUDA(cudaGetDeviceProperties(&prop, dev));
  if (prop.major != 10)
    fail(KC_ERR_NO_DEVICE, "CUDA backend: device " + std::to_string(dev) + " (" + prop.name +
                               ") is not an sm_100 (Blackwell B200) GPU");
}

// Record completion of everything enqueued so far on the handle's stream (`batch`: behind a forward pass).
void mark_batch(kc_handle* h, bool batch = true) {
  KC_CUDA(cudaEventRecord(h->done, h->stream));
  h->t_mark = std::chrono::steady_clock::now();
  h->mark_is_batch = batch;
  h->pending = true;
}

// Wait for the last mark: sleep through 85% of the estimated batch time, then poll the event, yielding the thread
// between queries (a few microseconds from completion to return, and no spinning for most of the batch); past the
// estimate, poll every 20 us. timeout_ms < 0: no limit.
void wait_event(kc_handle* h, int timeout_ms) {
  using clock = std::chrono::steady_clock;
  const auto t0 = clock::now();
  const int cls = h->last_n > h->max_batch / 2 ? 1 : 0;
  const double est = h->mark_is_batch ? h->est_us[cls] : 0.0;
  const auto deadline = t0 + std::chrono::milliseconds(timeout_ms < 0 ? 0 : timeout_ms);
  if (est > 0) {
    auto wake = h->t_mark + std::chrono::microseconds((long long)(0.8 * est));
    if (timeout_ms >= 0 && wake > deadline) wake = deadline;
    if (wake > t0 && cudaEventQuery(h->done) == cudaErrorNotReady) std::this_thread::sleep_until(wake);
  }
  while (true) {
    cudaError_t e = cudaEventQuery(h->done);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) KC_CUDA(e);
    const auto now = clock::now();
    if (timeout_ms >= 0 && now > deadline)
      fail(KC_ERR_TIMEOUT, "CUDA backend: batch did not finish within " + std::to_string(timeout_ms) + " ms");
    const double since_mark = std::chrono::duration<double, std::micro>(now - h->t_mark).count();
    if (est <= 0 || since_mark < 1.5 * est + 200) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  // the estimate follows a shorter batch at once (oversleeping costs latency) and a longer one slowly (a batch
  // held up by other work on the stream moves it by at most a factor 1.1)
  if (h->mark_is_batch) {
    const double took = std::chrono::duration<double, std::micro>(clock::now() - h->t_mark).count();
    h->est_us[cls] = est <= 0 || took < est ? took : 0.9 * est + 0.1 * std::min(took, 2.0 * est);
  }
  h->pending = false;
  if (*h->h_err != 0) {
    int code = *h->h_err;
    h->engine->clear_device_error();
    *h->h_err = 0;
    fail(KC_ERR_DEVICE, "CUDA backend: a kernel gave up waiting (device error code " + std::to_string(code) + ")");
  }
}

void check_enqueue(kc_handle* h, int n) {
  if (n < 1 || n > h->max_batch)
    fail(KC_ERR_INVALID, "CUDA backend: batch of " + std::to_string(n) + " rows outside [1, " +
                             std::to_string(h->max_batch) + "]");
  if (h->pending) fail(KC_ERR_INVALID, "CUDA backend: kc_enqueue while the previous batch was not waited for");
  KC_CUDA(cudaSetDevice(h->device));
}

// Float planes: rows [0, n) of the pinned float inputs to the device.
void upload_float(kc_handle* h, int n) {
  KC_CUDA(cudaMemcpyAsync(h->d_spatial, h->h_spatial, (size_t)n * h->n_spatial * sizeof(float), cudaMemcpyHostToDevice,
                          h->stream));
  KC_CUDA(cudaMemcpyAsync(h->d_global, h->h_global, (size_t)n * h->n_global * sizeof(float), cudaMemcpyHostToDevice,
                          h->stream));
  if (h->n_meta)
    KC_CUDA(cudaMemcpyAsync(h->d_meta, h->h_meta, (size_t)n * h->n_meta * sizeof(float), cudaMemcpyHostToDevice,
                            h->stream));
}

// Packed staging: symmetries, optimism, globals, meta and rows [0, n) of the bits in one copy (or the symmetries
// and optimism alone).
void upload_packed(kc_handle* h, int n, bool prefix_only) {
  const size_t bytes = prefix_only ? (size_t)h->max_batch * 8 : h->pk_prefix + (size_t)n * h->pk_row_bits;
  KC_CUDA(cudaMemcpyAsync(h->d_pk, h->h_pk, bytes, cudaMemcpyHostToDevice, h->stream));
}

void run_forward(kc_handle* h, int n, bool packed) {
  if (packed)
    h->engine->forward(n, h->stream, nullptr, h->pk_global(h->d_pk), h->n_meta ? h->pk_meta(h->d_pk) : nullptr,
                       h->d_out, h->pk_bits(h->d_pk), h->pk_sym(h->d_pk));
  else
    h->engine->forward(n, h->stream, h->d_spatial, h->d_global, h->n_meta ? h->d_meta : nullptr, h->d_out);
}

// Read the batch back: the raw output rows, or (finish) the NNOutput rows of the device copy_outputs, which reads
// the symmetries and optimism of the packed staging; then the device error word and the completion mark.
void readback(kc_handle* h, int n, bool finish) {
  if (finish) {
    const kc::OutputLayout& L = h->engine->layout();
    const kc::ModelDesc& m = h->model->desc;
    kc::FinishParams fp;
    fp.rows = h->d_out;
    fp.row_len = L.row_len;
    fp.policy_off = L.policy_off;
    fp.value_off = L.value_off;
    fp.score_off = L.score_off;
    fp.own_off = L.own_off;
    fp.P = m.num_policy_channels;
    fp.version = m.version;
    fp.has_own = m.num_ownership_channels() > 0;
    fp.sym = h->pk_sym(h->d_pk);
    fp.optimism = h->pk_opt(h->d_pk);
    fp.out = h->d_fin;
    kc::launch_finish_outputs(fp, n, h->stream);
    KC_CUDA(cudaMemcpyAsync(h->h_fin, h->d_fin, (size_t)n * KC_FINISHED_ROW_LEN * sizeof(float),
                            cudaMemcpyDeviceToHost, h->stream));
  } else {
    const int row_len = h->engine->layout().row_len;
    KC_CUDA(cudaMemcpyAsync(h->h_out, h->d_out, (size_t)n * row_len * sizeof(float), cudaMemcpyDeviceToHost,
                            h->stream));
  }
  KC_CUDA(cudaMemcpyAsync(h->h_err, h->engine->error_word(), sizeof(int), cudaMemcpyDeviceToHost, h->stream));
  mark_batch(h);
  h->last_n = n;
  h->last_finished = finish;
}

void enqueue_host(kc_handle* h, int n) {
  check_enqueue(h, n);
  upload_float(h, n);
  run_forward(h, n, false);
  readback(h, n, false);
}

// Pack one row's float planes [c][361] into c x 12 words (bit p % 32 of word p / 32 = point p); false if a value
// is neither 0 nor 1 (the row then cannot travel packed).
bool pack_row(const float* src, int c, uint32_t* dst) {
  for (int k = 0; k < c; k++) {
    const float* pl = src + (size_t)k * 361;
    uint32_t* w = dst + (size_t)k * KC_PACKED_WORDS_PER_PLANE;
    uint32_t bad = 0;
    for (int j = 0; j < KC_PACKED_WORDS_PER_PLANE; j++) {
      const int p0 = j * 32, cnt = std::min(32, 361 - p0);
      uint32_t word = 0;
      for (int i = 0; i < cnt; i++) {
        const float v = pl[p0 + i];
        word |= (uint32_t)(v != 0.0f) << i;
        bad |= (uint32_t)(v != 0.0f && v != 1.0f);
      }
      w[j] = word;
    }
    if (bad) return false;
  }
  return true;
}

}  // namespace

extern "C" {

const char* kc_last_error(void) { return kc::g_last_error.c_str(); }

int kc_device_count(int* count) {
  return guard([&] {
    need(count, "count");
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    int usable = 0;
    for (int i = 0; i < c; i++) {
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, i) == cudaSuccess && prop.major == 10) usable++;
    }
    *count = usable;
  });
}

int kc_model_load(const void* bytes, size_t n, const char* file_name, kc_model** out) {
  return guard([&] {
    need(bytes, "model bytes");
    need(out, "out");
    *out = nullptr;
    int binary = -1;
    bool onnx = false;
    if (file_name) {
      std::string f(file_name);
      for (auto& c : f) c = (char)std::tolower((unsigned char)c);
      auto ends = [&](const char* s) {
        size_t k = std::strlen(s);
        return f.size() >= k && f.compare(f.size() - k, k, s) == 0;
      };
      binary = (ends(".txt") || ends(".txt.gz")) ? 0 : 1;
      onnx = ends(".onnx");
    } else {
      // an ONNX ModelProto starts with its ir_version field (tag 0x08); a KataGo file starts with its name (text) or
      // the gzip magic
      onnx = n > 16 && static_cast<const uint8_t*>(bytes)[0] == 0x08;
    }
    try {
      auto m = std::make_unique<kc_model>();
      m->desc = onnx ? kc::parse_onnx(static_cast<const uint8_t*>(bytes), n)
                     : kc::parse_model(static_cast<const uint8_t*>(bytes), n, binary);
      *out = m.release();
    } catch (const Error& e) {
      fail(e.status, std::string("Error loading or parsing model file ") + (file_name ? file_name : "<memory>") + ": " +
                         e.what());
    }
  });
}

int kc_model_desc(const kc_model* model, kc_desc* out) {
  return guard([&] {
    need(model, "model");
    need(out, "out");
    const kc::ModelDesc& m = model->desc;
    std::memset(out, 0, sizeof(*out));
    std::snprintf(out->name, sizeof(out->name), "%s", m.name.c_str());
    out->model_version = m.version;
    out->num_input_channels = m.num_input_channels;
    out->num_input_global_channels = m.num_input_global_channels;
    out->num_input_meta_channels = m.num_input_meta_channels;
    out->meta_encoder_version = m.meta_encoder_version;
    out->num_policy_channels = m.num_policy_channels;
    out->num_value_channels = m.num_value_channels();
    out->num_score_value_channels = m.num_score_value_channels();
    out->num_ownership_channels = m.num_ownership_channels();
    out->trunk_num_blocks = (int)m.blocks.size();
    out->trunk_num_channels = m.trunk_c;
    out->trunk_norm_kind = m.trunk_norm_kind;
    out->has_any_transformer_blocks = m.has_any_transformer_blocks();
    out->has_any_nested_bottleneck_blocks = m.has_any_nested_bottleneck_blocks();
    out->post_process_from_header = m.post_process_from_header;
    out->prefer_pass_alive_under_suicide_rules = m.prefer_pass_alive;
    out->prefer_exclude_territory_adjacent_to_atari = m.prefer_exclude_atari;
    out->num_parameters = m.num_parameters();
    out->trunk_spatial_conv_depth = m.trunk_spatial_conv_depth();
    for (int i = 0; i < 8; i++) out->post_process[i] = m.post_process[i];
  });
}

int kc_model_destroy(kc_model* model) {
  delete model;
  return KC_OK;
}

int kc_model_flops(const kc_model* model, double* flops_per_row, double* conv3x3_flops_per_row) {
  return guard([&] {
    need(model, "model");
    kc::model_flops(model->desc, flops_per_row, conv3x3_flops_per_row);
  });
}

int kc_context_create(const int* gpu_idxs, int n_gpu_idxs, int nn_x_len, int nn_y_len, int precision,
                      const kc_model* model, kc_context** out) {
  return guard([&] {
    need(model, "model");
    need(out, "out");
    *out = nullptr;
    if (nn_x_len != 19 || nn_y_len != 19) fail(KC_ERR_INVALID, "CUDA backend: nnXLen and nnYLen must equal the network's posLen 19");
    auto c = std::make_unique<kc_context>();
    for (int i = 0; i < n_gpu_idxs; i++) c->gpus.push_back(gpu_idxs ? gpu_idxs[i] : -1);
    if (c->gpus.empty()) c->gpus.push_back(-1);
    c->nn_x_len = nn_x_len;
    c->nn_y_len = nn_y_len;
    c->precision = resolve_precision(precision, model->desc);
    c->model = model;
    *out = c.release();
  });
}

int kc_context_precision(const kc_context* ctx, int* precision) {
  return guard([&] {
    need(ctx, "context");
    need(precision, "precision");
    *precision = ctx->precision;
  });
}

int kc_context_destroy(kc_context* ctx) {
  delete ctx;
  return KC_OK;
}

int kc_handle_create(kc_context* ctx, int gpu_idx, int max_batch, int inputs_use_nhwc, kc_handle** out) {
  return guard([&] {
    need(ctx, "context");
    need(out, "out");
    *out = nullptr;
    if (inputs_use_nhwc) fail(KC_ERR_INVALID, "CUDA backend: inputsUseNHWC = true unsupported");
    if (max_batch < 1) fail(KC_ERR_INVALID, "CUDA backend: max batch size must be positive");
    int dev = gpu_idx >= 0 ? gpu_idx : (ctx->gpus[0] >= 0 ? ctx->gpus[0] : 0);
    check_device(dev);
    KC_CUDA(cudaSetDevice(dev));
    auto h = std::make_unique<kc_handle>();
    const kc::ModelDesc& m = ctx->model->desc;
    h->model = ctx->model;
    h->device = dev;
    h->max_batch = max_batch;
    h->n_spatial = m.num_input_channels * 361;
    h->n_global = m.num_input_global_channels;
    h->n_meta = m.num_input_meta_channels;
    KC_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    KC_CUDA(cudaEventCreateWithFlags(&h->done, cudaEventDisableTiming));
    h->engine = std::make_unique<kc::Engine>(m, dev, max_batch, ctx->precision);
    // KATAGO_CUDA_NO_GRAPHS=1 launches the forward kernel by kernel instead of through a CUDA graph (profilers)
    const char* ng = std::getenv("KATAGO_CUDA_NO_GRAPHS");
    if (ng && ng[0] == '1') h->engine->set_use_graphs(false);
    const int row_len = h->engine->layout().row_len;
    KC_CUDA(cudaMallocHost(&h->h_spatial, (size_t)max_batch * h->n_spatial * sizeof(float)));
    KC_CUDA(cudaMallocHost(&h->h_global, (size_t)max_batch * h->n_global * sizeof(float)));
    KC_CUDA(cudaMallocHost(&h->h_meta, (size_t)max_batch * std::max(1, h->n_meta) * sizeof(float)));
    KC_CUDA(cudaMallocHost(&h->h_out, (size_t)max_batch * row_len * sizeof(float)));
    KC_CUDA(cudaMallocHost(&h->h_err, sizeof(int)));
    std::memset(h->h_spatial, 0, (size_t)max_batch * h->n_spatial * sizeof(float));
    std::memset(h->h_global, 0, (size_t)max_batch * h->n_global * sizeof(float));
    std::memset(h->h_meta, 0, (size_t)max_batch * std::max(1, h->n_meta) * sizeof(float));
    *h->h_err = 0;
    KC_CUDA(cudaMalloc(&h->d_spatial, (size_t)max_batch * h->n_spatial * sizeof(float)));
    KC_CUDA(cudaMalloc(&h->d_global, (size_t)max_batch * h->n_global * sizeof(float)));
    KC_CUDA(cudaMalloc(&h->d_meta, (size_t)max_batch * std::max(1, h->n_meta) * sizeof(float)));
    KC_CUDA(cudaMalloc(&h->d_out, (size_t)max_batch * row_len * sizeof(float)));
    h->pk_prefix = ((size_t)max_batch * (2 + h->n_global + h->n_meta) * 4 + 255) / 256 * 256;
    h->pk_row_bits = (size_t)m.num_input_channels * KC_PACKED_WORDS_PER_PLANE * 4;
    const size_t pk_bytes = h->pk_prefix + (size_t)max_batch * h->pk_row_bits;
    KC_CUDA(cudaMallocHost(&h->h_pk, pk_bytes));
    std::memset(h->h_pk, 0, pk_bytes);
    KC_CUDA(cudaMalloc(&h->d_pk, pk_bytes));
    KC_CUDA(cudaMemset(h->d_pk, 0, pk_bytes));
    KC_CUDA(cudaMallocHost(&h->h_fin, (size_t)max_batch * KC_FINISHED_ROW_LEN * sizeof(float)));
    KC_CUDA(cudaMalloc(&h->d_fin, (size_t)max_batch * KC_FINISHED_ROW_LEN * sizeof(float)));
    h->scratch.resize(h->n_spatial);
    *out = h.release();
  });
}

int kc_handle_destroy(kc_handle* h) {
  delete h;
  return KC_OK;
}

int kc_handle_input_ptrs(kc_handle* h, float** spatial, float** global, float** meta) {
  return guard([&] {
    need(h, "handle");
    if (spatial) *spatial = h->h_spatial;
    if (global) *global = h->h_global;
    if (meta) *meta = h->n_meta ? h->h_meta : nullptr;
  });
}

int kc_handle_output_layout(const kc_handle* h, int* row_len, int* policy_off, int* value_off, int* score_off,
                            int* ownership_off) {
  return guard([&] {
    need(h, "handle");
    const kc::OutputLayout& L = h->engine->layout();
    if (row_len) *row_len = L.row_len;
    if (policy_off) *policy_off = L.policy_off;
    if (value_off) *value_off = L.value_off;
    if (score_off) *score_off = L.score_off;
    if (ownership_off) *ownership_off = L.own_off;
  });
}

int kc_enqueue(kc_handle* h, int n) {
  return guard([&] {
    need(h, "handle");
    enqueue_host(h, n);
  });
}

int kc_wait(kc_handle* h, int timeout_ms, const float** out_rows) {
  return guard([&] {
    need(h, "handle");
    if (!h->pending && h->last_n == 0) fail(KC_ERR_INVALID, "CUDA backend: kc_wait without kc_enqueue");
    KC_CUDA(cudaSetDevice(h->device));
    if (h->pending) wait_event(h, timeout_ms);
    if (out_rows) *out_rows = h->last_finished ? h->h_fin : h->h_out;
  });
}

int kc_handle_packed_input_ptrs(kc_handle* h, uint32_t** spatial_bits, float** global, float** meta,
                                int32_t** symmetry, float** policy_optimism) {
  return guard([&] {
    need(h, "handle");
    if (spatial_bits) *spatial_bits = h->pk_bits(h->h_pk);
    if (global) *global = h->pk_global(h->h_pk);
    if (meta) *meta = h->n_meta ? h->pk_meta(h->h_pk) : nullptr;
    if (symmetry) *symmetry = h->pk_sym(h->h_pk);
    if (policy_optimism) *policy_optimism = h->pk_opt(h->h_pk);
  });
}

int kc_enqueue_packed(kc_handle* h, int n, int finish) {
  return guard([&] {
    need(h, "handle");
    check_enqueue(h, n);
    const int32_t* sym = h->pk_sym(h->h_pk);
    for (int i = 0; i < n; i++)
      if (sym[i] < 0 || sym[i] > 7) fail(KC_ERR_INVALID, "CUDA backend: symmetry " + std::to_string(sym[i]) + " outside [0, 8)");
    upload_packed(h, n, false);
    run_forward(h, n, true);
    readback(h, n, finish != 0);
  });
}

int kc_pack_spatial(const float* planes, int n_planes, uint32_t* bits) {
  return guard([&] {
    need(planes, "planes");
    need(bits, "bits");
    if (n_planes < 1) fail(KC_ERR_INVALID, "CUDA backend: no planes to pack");
    if (!pack_row(planes, n_planes, bits))
      fail(KC_ERR_INVALID, "CUDA backend: a spatial input value is neither 0 nor 1 and cannot be bit-packed");
  });
}

int kc_enqueue_device(kc_handle* h, int n, const float* d_spatial, const float* d_global, const float* d_meta,
                      float* d_out) {
  return guard([&] {
    need(h, "handle");
    need(d_spatial, "spatial");
    need(d_global, "global");
    need(d_out, "out");
    if (h->n_meta) need(d_meta, "meta");
    if (h->pending) fail(KC_ERR_INVALID, "CUDA backend: kc_enqueue_device while the previous batch was not waited for");
    KC_CUDA(cudaSetDevice(h->device));
    h->engine->forward(n, h->stream, d_spatial, d_global, h->n_meta ? d_meta : nullptr, d_out);
    KC_CUDA(cudaMemcpyAsync(h->h_err, h->engine->error_word(), sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    mark_batch(h);
    h->last_n = n;
  });
}

int kc_handle_stream(kc_handle* h, void** stream) {
  return guard([&] {
    need(h, "handle");
    need(stream, "stream");
    *stream = (void*)h->stream;
  });
}

int kc_synchronize(kc_handle* h, int timeout_ms) {
  return guard([&] {
    need(h, "handle");
    KC_CUDA(cudaSetDevice(h->device));
    mark_batch(h, false);
    wait_event(h, timeout_ms);
  });
}

int kc_get_output(kc_handle* h, int n, const float* const* spatial_rows, const float* const* global_rows,
                  const float* const* meta_rows, const int* symmetry, const float* policy_optimism, int timeout_ms,
                  float* policy_out, float* value_out, float* misc_out, float* ownership_out) {
  return guard([&] {
    need(h, "handle");
    need(spatial_rows, "spatial rows");
    need(global_rows, "global rows");
    need(symmetry, "symmetry");
    need(policy_optimism, "policy optimism");
    need(policy_out, "policy out");
    need(value_out, "value out");
    need(misc_out, "misc out");
    if (n < 1 || n > h->max_batch) fail(KC_ERR_INVALID, "CUDA backend: batch size out of range");
    // the staging buffers below are still read by an earlier batch's copies while it is in flight
    if (h->pending) fail(KC_ERR_INVALID, "CUDA backend: kc_get_output while an enqueued batch was not waited for");
    const kc::ModelDesc& m = h->model->desc;
    const int C = m.num_input_channels;
    // copy_inputs (backend.rs:497-546): symmetry and optimism are read here, before the batch runs. Rows go to the
    // device bit-packed, the symmetry applied there, unless a spatial value is neither 0 nor 1; then every row is
    // copied as floats with its symmetry applied here, as the reference does.
    int32_t* sym = h->pk_sym(h->h_pk);
    float* opt = h->pk_opt(h->h_pk);
    for (int row = 0; row < n; row++) {
      if (symmetry[row] < 0 || symmetry[row] > 7)
        fail(KC_ERR_INVALID, "CUDA backend: symmetry " + std::to_string(symmetry[row]) + " outside [0, 8)");
      sym[row] = symmetry[row];
      opt[row] = policy_optimism[row];
      need(spatial_rows[row], "spatial row");
      need(global_rows[row], "global row");
      if (h->n_meta && (!meta_rows || !meta_rows[row]))
        fail(KC_ERR_INVALID, "CUDA backend: model needs SGF metadata rows");
    }
    bool packed = true;
    for (int row = 0; row < n && packed; row++)
      packed = pack_row(spatial_rows[row], C, h->pk_bits(h->h_pk) + (size_t)row * C * KC_PACKED_WORDS_PER_PLANE);
    float* glob = packed ? h->pk_global(h->h_pk) : h->h_global;
    float* meta = packed ? h->pk_meta(h->h_pk) : h->h_meta;
    for (int row = 0; row < n; row++) {
      std::memcpy(glob + (size_t)row * h->n_global, global_rows[row], h->n_global * sizeof(float));
      if (h->n_meta) std::memcpy(meta + (size_t)row * h->n_meta, meta_rows[row], h->n_meta * sizeof(float));
      if (!packed)
        copy_with_symmetry(spatial_rows[row], h->h_spatial + (size_t)row * h->n_spatial, 1, 19, 19, C, sym[row],
                           false);
    }
    KC_CUDA(cudaSetDevice(h->device));
    if (packed) {
      upload_packed(h, n, false);
    } else {
      upload_float(h, n);
      upload_packed(h, n, true);  // the symmetries and optimism the device copy_outputs reads
    }
    run_forward(h, n, packed);
    readback(h, n, true);
    wait_event(h, timeout_ms);
    // copy_outputs (backend.rs:622-731) ran on the device: each row's NNOutput fields are copied out
    for (int row = 0; row < n; row++) {
      const float* f = h->h_fin + (size_t)row * KC_FINISHED_ROW_LEN;
      std::memcpy(policy_out + (size_t)row * 362, f + KC_FINISHED_POLICY, 362 * sizeof(float));
      std::memcpy(value_out + (size_t)row * 3, f + KC_FINISHED_VALUE, 3 * sizeof(float));
      std::memcpy(misc_out + (size_t)row * 6, f + KC_FINISHED_MISC, 6 * sizeof(float));
      if (ownership_out)
        std::memcpy(ownership_out + (size_t)row * 361, f + KC_FINISHED_OWNERSHIP, 361 * sizeof(float));
    }
  });
}

int kc_handle_set_profiling(kc_handle* h, int on) {
  return guard([&] {
    need(h, "handle");
    KC_CUDA(cudaSetDevice(h->device));
    KC_CUDA(cudaStreamSynchronize(h->stream));
    h->engine->reset_profile();
    h->engine->set_profiling(on != 0);
  });
}

int kc_handle_profile(kc_handle* h, double* ms_by_class, int64_t* launches_by_class, int n_classes) {
  return guard([&] {
    need(h, "handle");
    h->engine->profile(ms_by_class, launches_by_class, n_classes);
  });
}

int kc_handle_launch_count(kc_handle* h, int n, int* launches) {
  return guard([&] {
    need(h, "handle");
    need(launches, "launches");
    if (n < 1 || n > h->max_batch) fail(KC_ERR_INVALID, "CUDA backend: launch count for a batch outside [1, max_batch]");
    *launches = h->engine->launches_per_forward(n);
  });
}

int kc_selftest_device_timeout(kc_handle* h, int limit_us) {
  return guard([&] {
    need(h, "handle");
    if (limit_us < 1 || limit_us > 2000000) fail(KC_ERR_INVALID, "CUDA backend: self-test limit outside [1 us, 2 s]");
    if (h->pending) fail(KC_ERR_INVALID, "CUDA backend: self-test while an enqueued batch was not waited for");
    KC_CUDA(cudaSetDevice(h->device));
    int khz = 0;
    KC_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, h->device));
    const long long cycles = (long long)limit_us * (khz > 0 ? khz : 2000000) / 1000;
    kc::launch_wait_selftest(h->engine->error_word(), cycles, h->stream);
    KC_CUDA(cudaMemcpyAsync(h->h_err, h->engine->error_word(), sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    mark_batch(h, false);
  });
}

int kc_copy_with_symmetry(const float* src, float* dst, int n_size, int h_size, int w_size, int c_size, int symmetry,
                          int reverse) {
  return guard([&] {
    need(src, "src");
    need(dst, "dst");
    copy_with_symmetry(src, dst, n_size, h_size, w_size, c_size, symmetry, reverse != 0);
  });
}

}  // extern "C"
