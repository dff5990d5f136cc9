/*
 * katago_cuda.h — the C ABI of the katago-rs B200 (sm_100a) neural-net backend.
 *
 * This is the boundary a `cuda` backend of katago-rs binds to. Each entry point replaces one piece of the
 * reference's `NeuralNet` trait (crates/katago-core/src/neuralnet/nninterface.rs:79-214) as implemented by the
 * burn backend (crates/katago-nn-burn/src/backend.rs); the citation is on each declaration. Plain pointers and
 * sizes only; no callbacks; the library never keeps a caller-owned pointer beyond the call.
 *
 * Every function returns an int status (KC_OK = 0). On failure kc_last_error() gives a message for this thread,
 * which the Rust side maps to KataError::StringError (nninterface.rs:202-205).
 *
 * Threading follows the reference: a model and a context may be shared; a handle is used by one thread at a time
 * ("Not thread-safe, each handle should only be used by one thread", nninterface.rs:33-34).
 */
#ifndef KATAGO_CUDA_H
#define KATAGO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KC_OK 0
#define KC_ERR_INVALID 1    /* bad argument (sizes, null pointers, unsupported option) */
#define KC_ERR_PARSE 2      /* model file could not be parsed */
#define KC_ERR_CUDA 3       /* a CUDA call failed */
#define KC_ERR_TIMEOUT 4    /* kc_wait gave up before the batch finished (the batch is still in flight) */
#define KC_ERR_DEVICE 5     /* a kernel reported a device-side error (a bounded wait expired) */
#define KC_ERR_NO_DEVICE 6  /* no usable sm_100 device */

/* Precision of a context (the reference's useFP16 enabled_t plus an explicit choice, backend.rs:300-340). */
#define KC_PRECISION_F32 0   /* float32 everywhere: the parity tier (SIMT kernels) */
#define KC_PRECISION_F16 1   /* f16 activations and weights, f32 accumulation (tcgen05) */
#define KC_PRECISION_BF16 2  /* bf16 activations and weights, f32 accumulation (tcgen05) */
#define KC_PRECISION_AUTO 3  /* f16 for convolution nets, bf16 for nets with transformer blocks */

typedef struct kc_model kc_model;
typedef struct kc_context kc_context;
typedef struct kc_handle kc_handle;

/* ModelDesc fields the host needs (crates/katago-core/src/neuralnet/desc.rs; the ONNX metadata keys the reference
 * writes in tools/bin2onnx/bin2onnx.py:1566-1614). */
typedef struct kc_desc {
  char name[128];
  int32_t model_version;
  int32_t num_input_channels;
  int32_t num_input_global_channels;
  int32_t num_input_meta_channels;
  int32_t meta_encoder_version;
  int32_t num_policy_channels;
  int32_t num_value_channels;
  int32_t num_score_value_channels;
  int32_t num_ownership_channels;
  int32_t trunk_num_blocks;
  int32_t trunk_num_channels;
  int32_t trunk_norm_kind;
  int32_t has_any_transformer_blocks;
  int32_t has_any_nested_bottleneck_blocks;
  int32_t post_process_from_header;
  int32_t prefer_pass_alive_under_suicide_rules;
  int32_t prefer_exclude_territory_adjacent_to_atari;
  int64_t num_parameters;
  double trunk_spatial_conv_depth;
  /* td_score, score_mean, score_stdev, lead, variance_time, shortterm_value_error, shortterm_score_error,
   * output_scale multipliers (ModelPostProcessParams, bin2onnx.py:843-854) */
  float post_process[8];
} kc_desc;

/* Message of the last failed call on this thread ("" if none). Valid until the next call on this thread. */
const char* kc_last_error(void);

/* Number of CUDA devices the library can run on (sm_100). NeuralNet::printDevices / getNumEffectiveDevices. */
int kc_device_count(int* count);

/* Parse a KataGo model file (.bin, .bin.gz, .txt, .txt.gz) from memory. `file_name` (may be NULL) decides text vs
 * binary floats as the reference does (bin2onnx.py:1074-1082); NULL means: binary if the data holds "@BIN@".
 * A name ending in ".onnx" (or, without a name, data that starts as an ONNX ModelProto) is read as the ONNX export
 * the reference's tools/bin2onnx/bin2onnx.py writes (the files the reference's burn backend is generated from,
 * crates/katago-nn-burn/build.rs:25-30): its layers are rebuilt from the graph and its metadata_props.
 * Replaces NeuralNet::load_model_file (nninterface.rs:137; backend.rs:277-292). No device is touched. */
int kc_model_load(const void* bytes, size_t n, const char* file_name, kc_model** out);

/* NeuralNet::get_model_desc (nninterface.rs:140; backend.rs:295-297). */
int kc_model_desc(const kc_model* model, kc_desc* out);

/* NeuralNet::free of LoadedModel (Drop). Safe on NULL. */
int kc_model_destroy(kc_model* model);

/* NeuralNet::create_compute_context (nninterface.rs:148-162; backend.rs:300-340). `gpu_idxs` lists the devices
 * handles of this context will use (-1 = default device); nn_x_len and nn_y_len must be 19 (the reference's fixed
 * posLen, backend.rs:327-333); `precision` is a KC_PRECISION_* value. */
int kc_context_create(const int* gpu_idxs, int n_gpu_idxs, int nn_x_len, int nn_y_len, int precision,
                      const kc_model* model, kc_context** out);
int kc_context_precision(const kc_context* ctx, int* precision);
int kc_context_destroy(kc_context* ctx);

/* NeuralNet::create_compute_handle (nninterface.rs:166-186; backend.rs:343-389): uploads packed weights to
 * `gpu_idx` (-1 = the context's first device), allocates device activations and pinned host I/O for `max_batch`
 * rows, and prepares the forward pass. `inputs_use_nhwc` must be 0 (NCHW, as the reference). */
int kc_handle_create(kc_context* ctx, int gpu_idx, int max_batch, int inputs_use_nhwc, kc_handle** out);
int kc_handle_destroy(kc_handle* h);

/* Pinned host input buffers of the handle (the reference's BurnInputBuffers, backend.rs:150-212): spatial
 * [max_batch, C, 19, 19] NCHW float32, global [max_batch, G], meta [max_batch, M] (NULL when M = 0). */
int kc_handle_input_ptrs(kc_handle* h, float** spatial, float** global, float** meta);

/* Floats per output row and the offsets of its parts, as the reference's readback concatenates them
 * (backend.rs:584-617): policy [P, 362] (pass last), value [3], score [S_v], ownership [1, 361]. */
int kc_handle_output_layout(const kc_handle* h, int* row_len, int* policy_off, int* value_off, int* score_off,
                            int* ownership_off);

/* Non-blocking: copy rows [0, n) of the pinned inputs to the device, run the forward pass, copy the n output rows
 * into the handle's pinned output buffer, and record completion. The device half of run_network
 * (backend.rs:549-619). */
int kc_enqueue(kc_handle* h, int n);

/* Block until the last enqueue finished, at most `timeout_ms` (negative = no limit). On success `*out_rows` points
 * at n rows of kc_handle_output_layout's row_len floats in pinned memory, valid until the next kc_enqueue. The
 * reference waits on a helper thread (backend.rs:743-753); KC_ERR_TIMEOUT leaves the batch in flight. */
int kc_wait(kc_handle* h, int timeout_ms, const float** out_rows);

/* Bit-packed inputs. Every spatial input feature of the reference (nninputs.rs fill_row_v7 :1336) is 0 or 1, so a
 * row's planes travel as bits: plane c of a row is KC_PACKED_WORDS_PER_PLANE 32-bit words, point p = y * 19 + x at bit
 * p % 32 of word p / 32 (bits past 361 zero); 22 planes are 1,056 bytes instead of 31,768. Each row's symmetry is
 * applied on the device as the planes are read (the inverse of SymmetryHelpers::copy_inputs_with_symmetry,
 * nninputs.rs:872, which the reference runs on the host per row in copy_inputs, backend.rs:497-546). */
#define KC_PACKED_WORDS_PER_PLANE 12

/* NNOutput rows (the reference's copy_outputs, backend.rs:622-731, run on the device): per row KC_FINISHED_ROW_LEN
 * floats: policy [362] (optimism mixed for v12+ nets, symmetry undone, pass last), value [3] (win, loss, noresult),
 * misc [6] (scoreMean, scoreMeanSq, lead, varTimeLeft, shorttermWinlossError, shorttermScoreError, by model version),
 * ownership [361] (symmetry undone). */
#define KC_FINISHED_ROW_LEN 732
#define KC_FINISHED_POLICY 0
#define KC_FINISHED_VALUE 362
#define KC_FINISHED_MISC 365
#define KC_FINISHED_OWNERSHIP 371

/* The handle's pinned staging for kc_enqueue_packed: spatial_bits [max_batch][C][KC_PACKED_WORDS_PER_PLANE],
 * global [max_batch][G], meta [max_batch][M] (NULL when M = 0), symmetry [max_batch] (0..7: bit 0 flipY, bit 1
 * flipX, bit 2 transpose), policy_optimism [max_batch]. The binding of BurnInputBuffers (backend.rs:150-212) for
 * callers that write packed rows. */
int kc_handle_packed_input_ptrs(kc_handle* h, uint32_t** spatial_bits, float** global, float** meta,
                                int32_t** symmetry, float** policy_optimism);

/* kc_enqueue for the packed staging: one host-to-device copy of rows [0, n), the forward pass with each row's
 * symmetry applied on the device, and the readback. finish = 0 reads back the raw output rows (as kc_enqueue);
 * finish = 1 runs the reference's copy_outputs on the device and reads back NNOutput rows of KC_FINISHED_ROW_LEN
 * floats. kc_wait returns the rows of whichever the last enqueue read back. */
int kc_enqueue_packed(kc_handle* h, int n, int finish);

/* Pack one row's float planes [n_planes][361] into [n_planes][KC_PACKED_WORDS_PER_PLANE] words; KC_ERR_INVALID when a
 * value is neither 0 nor 1. */
int kc_pack_spatial(const float* planes, int n_planes, uint32_t* bits);

/* The point mappings of the device-side symmetry, for tests of the host logic (no device is used): reverse = 0:
 * table[y * 19 + x] = the input point the network sees at (y, x); reverse = 1: table[p] = the point an output p is
 * moved to. Equal to kc_copy_with_symmetry's moves (nninputs.rs:756-831). */
int kc_symmetry_table(int symmetry, int reverse, int* table);

/* Same as kc_enqueue but the inputs and outputs are device pointers (no host copies): spatial [n,C,19,19],
 * global [n,G], meta [n,M] (may be NULL when M = 0), out [n,row_len] float32. For callers that keep their
 * batches on the GPU. */
int kc_enqueue_device(kc_handle* h, int n, const float* d_spatial, const float* d_global, const float* d_meta,
                      float* d_out);

/* The CUDA stream (cudaStream_t) the handle's work runs on, for callers that order their own work or timing
 * events against it. */
int kc_handle_stream(kc_handle* h, void** stream);

/* Synchronise the handle's stream (bounded like kc_wait). */
int kc_synchronize(kc_handle* h, int timeout_ms);

/* The whole reference get_output for one batch (backend.rs:410-731): per row, copy the inputs into the handle's
 * staging buffers with `symmetry[i]` (SymmetryHelpers::copy_inputs_with_symmetry, nninputs.rs:872), run the net,
 * then for each row mix the optimistic policy with `policy_optimism[i]` (v12+ nets), undo the symmetry on policy
 * and ownership, and write the NNOutput fields. Rows travel bit-packed with the symmetry applied on the device when
 * every spatial value is 0 or 1 (always, for the reference's inputs), else as floats with the symmetry applied on
 * the host; the output handling runs on the device (kc_enqueue_packed with finish = 1). Row inputs: `spatial_rows[i]` [C*19*19] NCHW,
 * `global_rows[i]` [G], `meta_rows[i]` [M] (NULL when M = 0). Outputs per row i:
 *   policy_out + i*362 (362 floats, pass last), value_out + i*3 (win, loss, noresult),
 *   misc_out + i*6 (scoreMean, scoreMeanSq, lead, varTimeLeft, shorttermWinlossError, shorttermScoreError,
 *   filled per model version as backend.rs:690-729), ownership_out + i*361 (may be NULL: no ownership map). */
int kc_get_output(kc_handle* h, int n, const float* const* spatial_rows, const float* const* global_rows,
                  const float* const* meta_rows, const int* symmetry, const float* policy_optimism, int timeout_ms,
                  float* policy_out, float* value_out, float* misc_out, float* ownership_out);

/* Per-kernel-class device time of the forward passes since profiling was switched on, in ms: with profiling on,
 * each kernel launch of the forward is bracketed by CUDA events on the handle's stream (recorded inside the CUDA
 * graph when graphs are used), and kc_handle_profile waits for the last pass and accumulates its launches.
 * class: 0 conv3x3 GEMM, 1 conv1x1/linear GEMM, 2 stem GEMM, 3 attention, 4 other kernels. */
int kc_handle_set_profiling(kc_handle* h, int on);
int kc_handle_profile(kc_handle* h, double* ms_by_class, int64_t* launches_by_class, int n_classes);
/* Kernel launches per forward pass of n positions (1 <= n <= the handle's max_batch; some boundaries of a net take
 * one fused kernel or two kernels depending on n), and algorithmic FLOPs per row. */
int kc_handle_launch_count(kc_handle* h, int n, int* launches);
int kc_model_flops(const kc_model* model, double* flops_per_row, double* conv3x3_flops_per_row);

/* KataGo's masked global pooling followed by the gpool-to-bias matmul, on device tensors in the reference layout:
 * x [n][c][19*19] float32 (already masked), mask [n][19*19] (input channel 0), w [3c][oc], out [n][oc]:
 *   out[b] = [mean, mean * (sqrt(area) - 14) / 10, max over on-board points] x w
 * (tools/bin2onnx/bin2onnx.py gpool :1222-1230 and the matmul after it, :1255 / :1501). Enqueued on `stream`
 * (a cudaStream_t, NULL = legacy default stream); the pooled [n][3c] scratch is taken from the stream-ordered
 * allocator (cudaMallocAsync) and released after use. 3c <= 12288. */
int kc_gpool_fc(const float* d_x, const float* d_mask, int n, int c, const float* d_w, int oc, float* d_out,
                void* stream);

/* kc_gpool_fc for callers that cannot allocate GPU memory — for instance a host that reserves the device memory up
 * front for its own pools and forbids later allocations, or a latency-critical thread that cannot afford
 * cudaMalloc's device-wide synchronisation. This entry point has no counterpart in the reference; it allocates
 * nothing (no cudaMalloc, cudaFree or allocating library call). Its pooled [n][3c] scratch is one fixed array of
 * KC_GPOOL_NOALLOC_MAX_FLOATS floats (1 MiB) in device memory, present on every GPU that loads this library until
 * the process exits; larger n * 3c is rejected with KC_ERR_INVALID. The first call on a device looks up that
 * array's device address (once per device, with that device current), so make the first call on each device
 * before any stream capture. With CUDA's lazy module loading (the default) the array is only placed in device
 * memory when that first call loads this part of the library on the device: make the first call before reserving
 * the device's memory for other pools (or load modules eagerly, CUDA_MODULE_LOADING=EAGER). All calls share the one array and it keeps the last call's contents (every entry a
 * call reads is written by that call first): calls whose work overlaps on the GPU (different streams, or
 * different host threads on one device) race on it and must be ordered by the caller. Inputs, outputs and
 * stream are as for kc_gpool_fc. */
#define KC_GPOOL_NOALLOC_MAX_FLOATS 262144
int kc_gpool_fc_noalloc(const float* d_x, const float* d_mask, int n, int c, const float* d_w, int oc, float* d_out,
                        void* stream);

/* Failure-detection self-test. Every spin-wait in this library's kernels is bounded: when a wait runs out, the
 * kernel records an error code in the handle's device error word, releases what it holds and returns, and the next
 * kc_wait / kc_synchronize reports KC_ERR_DEVICE (the handle stays usable). This enqueues on the handle's stream
 * one kernel that makes the same bounded wait on a barrier nothing completes, with a limit of `limit_us`
 * microseconds (1 .. 2,000,000) instead of the forward pass's 2 s, so that a caller can check the whole error path
 * without a fault. No counterpart in the reference, whose kernels have no bounded waits. */
int kc_selftest_device_timeout(kc_handle* h, int limit_us);

/* Host-side symmetry helpers of the reference (nninputs.rs:756-879), exported for tests of the host logic.
 * NCHW copy of one row with `c_size` channels; `reverse` = copyOutputsWithSymmetry semantics. */
int kc_copy_with_symmetry(const float* src, float* dst, int n_size, int h_size, int w_size, int c_size,
                          int symmetry, int reverse);

#ifdef __cplusplus
}
#endif

#endif /* KATAGO_CUDA_H */
