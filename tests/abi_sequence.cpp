// The call sequence of the katago-nn-cuda Rust crate's NeuralNet (load_model_file, create_compute_context,
// create_compute_handle, get_output), made through the same C ABI from C++, for a test on the GPU: the crate cannot
// be compiled where cargo is absent, so this program stands in for it call for call.
//
//   abi_sequence <model file> <inputs file> <out file> <precision> <float path 0|1>
//
// inputs file: int32 n, int32 C, int32 G, then per row: C*361 floats (spatial), G floats (global), int32 symmetry,
// float optimism. out file: n rows of KC_FINISHED_ROW_LEN floats (policy 362 | value 3 | misc 6 | ownership 361).
// With float path = 1 the rows go as floats moved by kc_copy_with_symmetry (the crate's fallback for features that
// are not 0 / 1) and copy_outputs runs here, as the crate's copy_outputs_raw does.

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "../include/katago_cuda.h"

#define CHECK(call)                                                              \
  do {                                                                           \
    int st_ = (call);                                                            \
    if (st_ != KC_OK) {                                                          \
      std::fprintf(stderr, "%s failed (%d): %s\n", #call, st_, kc_last_error()); \
      std::exit(1);                                                              \
    }                                                                            \
  } while (0)

static std::vector<char> read_file(const char* path) {
  FILE* f = std::fopen(path, "rb");
  if (!f) {
    std::perror(path);
    std::exit(1);
  }
  std::vector<char> d;
  char buf[65536];
  size_t k;
  while ((k = std::fread(buf, 1, sizeof(buf), f)) > 0) d.insert(d.end(), buf, buf + k);
  std::fclose(f);
  return d;
}

int main(int argc, char** argv) {
  if (argc != 6) {
    std::fprintf(stderr, "usage: %s model inputs out precision float_path\n", argv[0]);
    return 2;
  }
  const int precision = std::atoi(argv[4]);
  const bool float_path = std::atoi(argv[5]) != 0;
  // load_model_file
  std::vector<char> bytes = read_file(argv[1]);
  kc_model* model = nullptr;
  CHECK(kc_model_load(bytes.data(), bytes.size(), argv[1], &model));
  kc_desc d;
  CHECK(kc_model_desc(model, &d));
  // inputs
  std::vector<char> in = read_file(argv[2]);
  const int32_t* hdr = reinterpret_cast<const int32_t*>(in.data());
  const int n = hdr[0], C = hdr[1], G = hdr[2];
  if (C != d.num_input_channels || G != d.num_input_global_channels) {
    std::fprintf(stderr, "input sizes do not match the model\n");
    return 1;
  }
  const size_t row_bytes = ((size_t)C * 361 + G) * 4 + 8;
  auto row = [&](int i) { return in.data() + 12 + (size_t)i * row_bytes; };
  // create_compute_context, create_compute_handle
  const int gpus[1] = {0};
  kc_context* ctx = nullptr;
  CHECK(kc_context_create(gpus, 1, 19, 19, precision, model, &ctx));
  kc_handle* h = nullptr;
  CHECK(kc_handle_create(ctx, 0, n, 0, &h));
  uint32_t* pk_bits;
  float *pk_glob, *pk_meta, *pk_opt;
  int32_t* pk_sym;
  CHECK(kc_handle_packed_input_ptrs(h, &pk_bits, &pk_glob, &pk_meta, &pk_sym, &pk_opt));
  float *f_spatial, *f_glob, *f_meta;
  CHECK(kc_handle_input_ptrs(h, &f_spatial, &f_glob, &f_meta));
  int row_len, policy_off, value_off, score_off, own_off;
  CHECK(kc_handle_output_layout(h, &row_len, &policy_off, &value_off, &score_off, &own_off));
  // get_output: copy_inputs
  std::vector<int> sym(n);
  std::vector<float> opt(n);
  for (int i = 0; i < n; i++) {
    const float* sp = reinterpret_cast<const float*>(row(i));
    const float* gl = sp + (size_t)C * 361;
    std::memcpy(&sym[i], gl + G, 4);
    std::memcpy(&opt[i], gl + G + 1, 4);
    if (float_path) {
      CHECK(kc_copy_with_symmetry(sp, f_spatial + (size_t)i * C * 361, 1, 19, 19, C, sym[i], 0));
      std::memcpy(f_glob + (size_t)i * G, gl, (size_t)G * 4);
    } else {
      CHECK(kc_pack_spatial(sp, C, pk_bits + (size_t)i * C * KC_PACKED_WORDS_PER_PLANE));
      std::memcpy(pk_glob + (size_t)i * G, gl, (size_t)G * 4);
      pk_sym[i] = sym[i];
      pk_opt[i] = opt[i];
    }
  }
  // run_network: enqueue here, wait on a helper thread (the crate's wait_on_helper_thread)
  if (float_path) CHECK(kc_enqueue(h, n));
  else CHECK(kc_enqueue_packed(h, n, 1));
  const float* rows = nullptr;
  int wait_status = -1;
  std::thread helper([&] { wait_status = kc_wait(h, -1, &rows); });
  helper.join();
  if (wait_status != KC_OK) {
    std::fprintf(stderr, "kc_wait failed (%d)\n", wait_status);
    return 1;
  }
  // copy_outputs
  std::vector<float> out((size_t)n * KC_FINISHED_ROW_LEN, 0.0f);
  for (int i = 0; i < n; i++) {
    float* o = out.data() + (size_t)i * KC_FINISHED_ROW_LEN;
    if (!float_path) {
      std::memcpy(o, rows + (size_t)i * KC_FINISHED_ROW_LEN, KC_FINISHED_ROW_LEN * 4);
      continue;
    }
    const float* rd = rows + (size_t)i * row_len;
    const float* pol = rd + policy_off;
    float tmp[361];
    const bool mix = d.num_policy_channels == 2 || (d.num_policy_channels == 4 && d.model_version >= 16);
    for (int p = 0; p < 361; p++) tmp[p] = mix ? pol[p] + (pol[362 + p] - pol[p]) * opt[i] : pol[p];
    CHECK(kc_copy_with_symmetry(tmp, o + KC_FINISHED_POLICY, 1, 19, 19, 1, sym[i], 1));
    o[KC_FINISHED_POLICY + 361] = mix ? pol[361] + (pol[362 + 361] - pol[361]) * opt[i] : pol[361];
    for (int k = 0; k < 3; k++) o[KC_FINISHED_VALUE + k] = rd[value_off + k];
    const float* s = rd + score_off;
    float* m = o + KC_FINISHED_MISC;
    if (d.model_version >= 9) {
      for (int k = 0; k < 6; k++) m[k] = s[k];
    } else if (d.model_version >= 8) {
      m[0] = s[0], m[1] = s[1], m[2] = s[2], m[3] = s[3];
    } else if (d.model_version >= 4) {
      m[0] = s[0], m[1] = s[1], m[2] = s[0];
    } else {
      m[0] = s[0], m[1] = s[0] * s[0], m[2] = s[0];
    }
    CHECK(kc_copy_with_symmetry(rd + own_off, o + KC_FINISHED_OWNERSHIP, 1, 19, 19, 1, sym[i], 1));
  }
  FILE* f = std::fopen(argv[3], "wb");
  if (!f || std::fwrite(out.data(), 4, out.size(), f) != out.size()) return 1;
  std::fclose(f);
  CHECK(kc_handle_destroy(h));
  CHECK(kc_context_destroy(ctx));
  CHECK(kc_model_destroy(model));
  return 0;
}
