// Device side of the reference backend's host-side row handling (crates/katago-nn-burn/src/backend.rs): the
// copy_outputs step of get_output (:622-731) run on the GPU behind the forward pass, so that a batch's readback is
// the NNOutput fields of every row instead of the raw output rows, and the host only copies them out.

#include <cuda_runtime.h>

#include "common.h"
#include "engine.h"
#include "kernels.cuh"

namespace kc {

// Destination of a row's output point (h, w) under copyOutputsWithSymmetry (SymmetryHelpers copy_with_symmetry with
// reverse = true, nninputs.rs:756-831, 877): flipY / flipX of (h, w), transposed after the flips.
__host__ __device__ __forceinline__ int sym_dst_reverse(int sym, int h, int w) {
  const bool fy = (sym & 1) != 0, fx = (sym & 2) != 0;
  int hs = fy ? -19 : 19, ws = fx ? -1 : 1;
  const int base = (fy ? 18 * 19 : 0) + (fx ? 18 : 0);
  if (sym & 4) {
    const int t = hs;
    hs = ws;
    ws = t;
  }
  return base + h * hs + w * ws;
}

// One block of 384 threads per row: thread t < 361 owns point t of the policy (optimism mix, then its inverse
// symmetry) and of the ownership map, thread 361 the pass logit, threads 362.. the value and score fields.
// The mix p + (p_opt - p) * o is rounded step by step (no fused multiply-add), as the reference computes it.
__global__ void __launch_bounds__(384) finish_outputs_kernel(const __grid_constant__ FinishParams p) {
  const int row = blockIdx.x, t = threadIdx.x;
  const float* rd = p.rows + (size_t)row * p.row_len;
  float* out = p.out + (size_t)row * KC_FINISHED_ROW_LEN;
  const int sym = p.sym[row];
  const float o = p.optimism[row];
  const bool mix = p.P == 2 || (p.P == 4 && p.version >= 16);
  const float* pol = rd + p.policy_off;
  if (t < 361) {
    float v = pol[t];
    if (mix) v = __fadd_rn(v, __fmul_rn(__fsub_rn(pol[362 + t], v), o));
    const int d = sym_dst_reverse(sym, t / 19, t % 19);
    out[KC_FINISHED_POLICY + d] = v;
    out[KC_FINISHED_OWNERSHIP + d] = p.has_own ? rd[p.own_off + t] : 0.0f;
  } else if (t == 361) {
    float v = pol[361];
    if (mix) v = __fadd_rn(v, __fmul_rn(__fsub_rn(pol[362 + 361], v), o));
    out[KC_FINISHED_POLICY + 361] = v;
  } else if (t < 362 + 3) {
    out[KC_FINISHED_VALUE + (t - 362)] = rd[p.value_off + (t - 362)];
  } else if (t < 362 + 3 + 6) {
    // misc fields by model version (backend.rs:690-729): scoreMean, scoreMeanSq, lead, varTimeLeft,
    // shorttermWinlossError, shorttermScoreError
    const int i = t - 365;
    const float* s = rd + p.score_off;
    float v = 0.0f;
    if (p.version >= 9) v = s[i];
    else if (p.version >= 8) v = i < 4 ? s[i] : 0.0f;
    else if (p.version >= 4) v = i == 0 ? s[0] : i == 1 ? s[1] : i == 2 ? s[0] : 0.0f;
    else v = i == 0 ? s[0] : i == 1 ? __fmul_rn(s[0], s[0]) : i == 2 ? s[0] : 0.0f;
    out[KC_FINISHED_MISC + i] = v;
  }
}

void launch_finish_outputs(const FinishParams& p, int n, cudaStream_t st) {
  finish_outputs_kernel<<<n, 384, 0, st>>>(p);
  KC_CUDA(cudaGetLastError());
}

}  // namespace kc

// The point mappings the device applies, exported for tests of the host-side semantics (no device is used):
// reverse = 0: table[y * 19 + x] = the row's input point the network sees at (y, x) (sym_src);
// reverse = 1: table[p] = the NNOutput point an output point p goes to (sym_dst_reverse).
extern "C" int kc_symmetry_table(int symmetry, int reverse, int* table) {
  if (!table || symmetry < 0 || symmetry > 7) {
    kc::set_last_error("CUDA backend: kc_symmetry_table: bad arguments");
    return KC_ERR_INVALID;
  }
  for (int p = 0; p < 361; p++)
    table[p] = reverse ? kc::sym_dst_reverse(symmetry, p / 19, p % 19) : kc::sym_src(symmetry, p / 19, p % 19);
  kc::set_last_error("");
  return KC_OK;
}
