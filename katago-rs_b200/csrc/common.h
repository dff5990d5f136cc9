// Shared definitions of the katago-rs B200 backend: status codes, the thread-local error message of the C ABI,
// and CUDA error checks that turn a failed call into an exception the C ABI maps to a status.
#pragma once

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include <cuda_runtime.h>

#include "../../include/katago_cuda.h"

namespace kc {

// An error with the C ABI status it maps to. The message is what the reference backend would put into a
// KataError::StringError (crates/katago-nn-burn/src/backend.rs:280-289,327,335,371 use the same texts).
struct Error : std::runtime_error {
  int status;
  Error(int st, const std::string& m) : std::runtime_error(m), status(st) {}
};

[[noreturn]] inline void fail(int status, const std::string& msg) { throw Error(status, msg); }

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
  if (e != cudaSuccess) {
    char buf[512];
    std::snprintf(buf, sizeof(buf), "CUDA backend: %s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    throw Error(KC_ERR_CUDA, buf);
  }
}

void set_last_error(const std::string& msg);

}  // namespace kc

#define KC_CUDA(call) ::kc::cuda_check((call), #call, __FILE__, __LINE__)
