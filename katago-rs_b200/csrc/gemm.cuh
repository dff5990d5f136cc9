// Implicit-GEMM convolutions and token linears of the katago-rs B200 backend.
//
// Every 3x3 / 5x5 / 1x1 convolution and every transformer linear of the reference forward pass
// (tools/bin2onnx/bin2onnx.py GraphBuilder.conv :1140, matmul_tokens :1326) is one GEMM over the board-point rows
// of an activation tensor in the padded board layout (PBL):
//
//   out[r, n] = sum_{tap, c} A[r + tap_off[tap], c] * W[n, tap * cin + c]
//
// A is NHWC with one row per point of a 20-column grid per board (19 board columns + 1 zero column shared by the
// left and right halo) and 20 rows per board (a zero row shared by the boards above and below), so a 3x3 tap is a
// constant row offset dy*20+dx and the whole convolution is nine shifted row windows of the same tensor: no
// gather. Zero halo rows are maintained by every epilogue (it writes 0 there). The stem's 5x5 / 3x3 taps over the
// 22 input planes are either a one-tap GEMM over an im2col operand in the PBL (tensor-core tiers, built by
// prep_im2col_kernel) or, in the float32 tier, taps over a 21-column / 2-halo layout whose epilogue remaps rows
// into the PBL.
//
// Kernels sharing this file's epilogue:
//  * gemm_tc_kernel (f16 / bf16): persistent, warp-specialised one-CTA tcgen05 kernel. Warp 0 issues TMA loads of
//    the A window (128 rows x 64 channels at the tap's row offset) and the weight tile into a STAGES-deep ring,
//    warp 1 issues tcgen05.mma (M = 128, N = BN, K = 16) into one of two TMEM accumulators, warps 2-9 (two per
//    TMEM lane quarter) drain the other accumulator (tcgen05.ld) through the fused epilogue while the next tile's
//    MMAs run. Most GEMMs of the tensor-core tiers run on the CTA-pair kernel instead (gemm_pair.cuh); this one
//    takes the rest (three output segments, float32 outputs with an activation output, narrow RoPE heads).
//  * gemm_simt_kernel (f32 parity tier): 64 x 64 register-tiled SIMT GEMM over the same row geometry.
//
// Fused epilogue (per row r, column c): + per-board bias (stem: global-feature matmul), x mask (transformer
// residual branches), + residual, raw output, BN + activation + mask output for the next layer
// (bin2onnx.py bn_act_mask :1170), or SwiGLU (silu(a) * gate, bin2onnx.py :1433) or 2D RoPE on Q and K
// (bin2onnx.py rope :1342, applied to the f32 accumulators).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "ptx.cuh"

namespace kc {

enum EpiFlags : int {
  EPI_BOARD_BIAS = 1,  // acc += board_bias[board][col]
  EPI_MASK_ACC = 2,    // acc *= mask before the residual add (transformer branch outputs are masked)
  EPI_RESIDUAL = 4,    // y = acc + residual[row][col]
  EPI_RAW = 8,         // out_raw[row][col] = y * mask
  EPI_ACT = 16,        // out_act[row][col] = act(y * scale[col] + bias[col]) * mask
  EPI_RES_F32 = 32,    // the residual is float32 (the bf16 tier keeps the residual stream in float32)
  EPI_RAW_F32 = 64,    // the raw output is float32
};

enum GemmMode : int { MODE_SEGMENTS = 0, MODE_SWIGLU = 1, MODE_ROPE = 2 };

struct EpiSeg {
  int n0 = 0, n1 = 0;  // GEMM columns [n0, n1) (multiples of 16)
  int flags = 0, act = 0;
  const float* scale = nullptr;       // [n1 - n0]
  const float* bias = nullptr;        // [n1 - n0]
  const float* board_bias = nullptr;  // [boards][ld_bb]
  int ld_bb = 0;
  const void* res = nullptr;
  int ld_res = 0, res_c0 = 0;
  void* out_raw = nullptr;
  int ld_raw = 0, raw_c0 = 0;
  void* out_act = nullptr;
  int ld_act = 0, act_c0 = 0;
};

// Row space of a GEMM: which rows to compute and how a row maps to (board, y, x).
struct GemmGeom {
  int rows = 0;        // rows [0, rows) are computed; tiles cover ceil(rows / 128) * 128
  int board_rows = 400;
  int stride = 20;     // row within board -> y = rr / stride - pad, x = rr % stride
  int pad = 1;
  int remap = 0;       // 1: output row = PBL row of the same (board, y, x) (stem)
  const float* rowmask = nullptr;  // [PBL rows]: 1 on board, 0 elsewhere
};

struct alignas(16) GemmParams {
  GemmGeom g;
  int n_total = 0;     // N (multiple of the tile width)
  int cin = 0;         // A channels per tap (multiple of 64 on the tensor-core path)
  int taps = 1;
  int tap_off[25] = {0};
  int mode = MODE_SEGMENTS;
  int nseg = 1;
  EpiSeg seg[3];
  // RoPE (MODE_ROPE): columns [0, rot_cols) are Q then K heads of head_dim, rotated in halves
  const float* rope_cos = nullptr;  // [tables][361][head_dim/2]
  const float* rope_sin = nullptr;
  int rope_table_stride = 0;        // floats between tables (0: one shared table)
  int rope_q_cols = 0, rope_rot_cols = 0, head_dim = 0, rope_group = 1;
  int* err = nullptr;
  // windowed A (CTA-pair kernel, 3x3 convolutions): one window of win_rows rows starting halo rows above the tile
  int halo = 0, win_rows = 0;
  // CTA-pair kernel, windowed tiles of width >= 128: work items from split_from on are column halves of the tiles
  // from split_from on (two items per tile), so that a last, partly filled round of tiles becomes one round of
  // half-width items on up to twice as many pairs. Honoured only when every pair gets at most one half item, as its
  // last item: split_from a multiple of the launched pairs and 2 x (tiles - split_from) <= pairs.
  int split_from = 1 << 30;
  // CTA-pair kernel: columns >= pair_split belong to segment 1; the x coordinate of an output / residual box is
  // pair_*_x + GEMM column (the segment's c0 minus its first column)
  int pair_split = 0, pair_raw_x = 0, pair_act_x = 0, pair_res_x = 0;
  // SIMT kernel only
  const void* a = nullptr;
  int lda = 0;
  int a_rows = 0;      // allocated rows of A (rows outside [0, a_rows) read as 0)
  const void* w = nullptr;  // [n_total][taps * cin]
};

// ---- element conversions ----
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// mish(x) = x * tanh(softplus(x)), with tanh(log(1 + e)) = (e^2 + 2e) / (e^2 + 2e + 2), e = exp(x), and the
// identity above 20 (burn's softplus threshold, crates/katago-nn-burn/src/wino/kernels.rs:131).
// silu(x) = x / (exp(-x) + 1) (bin2onnx.py:1163-1168), 0 below -80 where exp(-x) leaves the fast-divide range.
// Both divide with __fdividef: the divisors stay below 2^126 on the branches taken.
template <int ACT>
__device__ __forceinline__ float act_fn(float x) {
  if constexpr (ACT == 1) {
    return fmaxf(x, 0.0f);
  } else if constexpr (ACT == 2) {
    float e = __expf(fminf(x, 20.0f));
    float n = e * (e + 2.0f);
    float y = x * __fdividef(n, n + 2.0f);
    return x > 20.0f ? x : y;
  } else if constexpr (ACT == 3) {
    float y = __fdividef(x, __expf(-x) + 1.0f);
    return x < -80.0f ? 0.0f : y;
  } else {
    return x;
  }
}

// Runtime-selected activation, for the small kernels (per-element dispatch; the GEMM epilogue dispatches once per
// 16-column unit on act_fn<ACT> instead).
__device__ __forceinline__ float act_apply(float x, int act) {
  if (act == 1) return act_fn<1>(x);
  if (act == 2) return act_fn<2>(x);
  if (act == 3) return act_fn<3>(x);
  return x;
}

struct RowInfo {
  int out_row;
  int board;
  int pos;      // y * 19 + x
  float mask;
  bool write;
};

__device__ __forceinline__ RowInfo row_info(const GemmGeom& g, int r) {
  RowInfo ri;
  int b = r / g.board_rows;
  int rr = r - b * g.board_rows;
  int q = rr / g.stride;
  int yy = q - g.pad;
  int xx = rr - q * g.stride;
  bool in_grid = r < g.rows && yy >= 0 && yy < 19 && xx < 19;
  if (g.remap) {
    ri.write = in_grid;
    ri.out_row = in_grid ? b * 400 + (yy + 1) * 20 + xx : 0;
  } else {
    ri.write = true;
    ri.out_row = r;
  }
  ri.board = in_grid ? b : 0;
  ri.pos = in_grid ? yy * 19 + xx : 0;
  ri.mask = in_grid ? __ldg(g.rowmask + ri.out_row) : 0.0f;
  return ri;
}

// Load CNT consecutive T (CNT * sizeof(T) a multiple of 16 bytes, 16-byte aligned) as floats.
template <typename T, int CNT>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[CNT]) {
  static_assert((CNT * sizeof(T)) % 16 == 0, "vector width");
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < CNT; i += PER) {
    uint4 u = *reinterpret_cast<const uint4*>(p + i);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < PER; j++) v[i + j] = to_f<T>(e[j]);
  }
}

template <typename T, int CNT>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[CNT]) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < CNT; i += PER) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < PER; j++) e[j] = from_f<T>(v[i + j]);
    *reinterpret_cast<uint4*>(p + i) = u;
  }
}

template <typename T, int CNT>
__device__ __forceinline__ void store_zero(T* p) {
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < CNT; i += PER) *reinterpret_cast<uint4*>(p + i) = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ const EpiSeg& seg_of(const GemmParams& p, int col) {
  if (p.nseg > 2 && col >= p.seg[1].n1) return p.seg[2];
  if (p.nseg > 1 && col >= p.seg[0].n1) return p.seg[1];
  return p.seg[0];
}

// The residual of CNT columns [c, c + CNT) of a segment (issued before the accumulator is read, to overlap).
template <typename T, int CNT>
__device__ __forceinline__ void epi_load_res(const EpiSeg& s, const RowInfo& ri, int c, float (&rv)[CNT]) {
  if ((s.flags & EPI_RESIDUAL) && ri.write) {
    const size_t off = (size_t)ri.out_row * s.ld_res + s.res_c0 + c;
    if (s.flags & EPI_RES_F32) load_vec<float, CNT>(reinterpret_cast<const float*>(s.res) + off, rv);
    else load_vec<T, CNT>(reinterpret_cast<const T*>(s.res) + off, rv);
  } else {
#pragma unroll
    for (int i = 0; i < CNT; i++) rv[i] = 0.0f;
  }
}

// o = act(v * scale + bias) * mask (bin2onnx.py bn_act_mask :1170), the activation fixed at compile time.
template <int CNT, int ACT>
__device__ __forceinline__ void bn_act(const float (&v)[CNT], const float* sc, const float* bi, float m,
                                       float (&o)[CNT]) {
#pragma unroll
  for (int i = 0; i < CNT; i++) {
    float t = v[i] * sc[i];
    t = t + bi[i];
    o[i] = act_fn<ACT>(t) * m;
  }
}

// Segment epilogue for CNT consecutive columns [c, c + CNT) of segment s (c relative to the segment) of one row.
// sc / bi: the BN scale and bias of those columns (shared or global memory).
template <typename T, int CNT>
__device__ __forceinline__ void epi_apply(const EpiSeg& s, const RowInfo& ri, int c, float (&v)[CNT],
                                          const float (&rv)[CNT], const float* sc, const float* bi) {
  if (!ri.write) return;
  const int f = s.flags;
  const float m = ri.mask;
  if ((f & EPI_BOARD_BIAS) && m != 0.0f) {
    const float* bb = s.board_bias + (size_t)ri.board * s.ld_bb + c;
#pragma unroll
    for (int i = 0; i < CNT; i++) v[i] += __ldg(bb + i);
  }
  if (f & EPI_MASK_ACC) {
#pragma unroll
    for (int i = 0; i < CNT; i++) v[i] *= m;
  }
  if (f & EPI_RESIDUAL) {
#pragma unroll
    for (int i = 0; i < CNT; i++) v[i] += rv[i];
  }
  if (f & EPI_RAW) {
    float o[CNT];
#pragma unroll
    for (int i = 0; i < CNT; i++) o[i] = v[i] * m;
    const size_t off = (size_t)ri.out_row * s.ld_raw + s.raw_c0 + c;
    if (f & EPI_RAW_F32) store_vec<float, CNT>(reinterpret_cast<float*>(s.out_raw) + off, o);
    else store_vec<T, CNT>(reinterpret_cast<T*>(s.out_raw) + off, o);
  }
  if (f & EPI_ACT) {
    float o[CNT];
    switch (s.act) {
      case 1: bn_act<CNT, 1>(v, sc, bi, m, o); break;
      case 2: bn_act<CNT, 2>(v, sc, bi, m, o); break;
      case 3: bn_act<CNT, 3>(v, sc, bi, m, o); break;
      default: bn_act<CNT, 0>(v, sc, bi, m, o); break;
    }
    store_vec<T, CNT>(reinterpret_cast<T*>(s.out_act) + (size_t)ri.out_row * s.ld_act + s.act_c0 + c, o);
  }
}

// ================================================================================================================
// tcgen05 persistent kernel
// ================================================================================================================

// Shared-memory plan of the tensor-core kernel: a stage holds one A tile (128 rows x 64 channels) and one B tile.
template <int BN>
struct TcCfg {
  static constexpr int A_BYTES = 128 * 64 * 2;
  static constexpr int B_BYTES = BN * 64 * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PARAM_COLS = 768;  // per-column BN scale and bias staged in shared memory
  static constexpr int PARAM_BYTES = PARAM_COLS * 2 * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int PCOPY_BYTES = 1024;  // a shared-memory copy of GemmParams
  static constexpr int SMEM_LIMIT = 227 * 1024;
  static constexpr int FIT =
      (SMEM_LIMIT - 1024 - BAR_BYTES - PARAM_BYTES - PCOPY_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr uint32_t ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
  static constexpr int SMEM =
      1024 /*align slack*/ + STAGES * STAGE_BYTES + BAR_BYTES + PARAM_BYTES + PCOPY_BYTES;
  static constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, splitting the tile's columns
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};

// Epilogue of one 128 x BN accumulator by the warp pair of one TMEM lane quarter; `half` selects this warp's
// columns (interleaved 16-column chunks for segments, contiguous halves for SwiGLU and RoPE).
// Residual of one 16-column unit as raw 32-bit words (8 for 2-byte types, 16 for float32), loaded early.
template <typename T, bool RF32>
__device__ __forceinline__ void res_fetch(const EpiSeg& s, const RowInfo& ri, int c, uint32_t* w) {
  constexpr int WORDS = RF32 ? 16 : 8;
  if ((s.flags & EPI_RESIDUAL) && ri.write) {
    const size_t off = (size_t)ri.out_row * s.ld_res + s.res_c0 + c;
    const uint4* src = RF32 ? reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(s.res) + off)
                            : reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(s.res) + off);
#pragma unroll
    for (int j = 0; j < WORDS / 4; j++) {
      uint4 q = src[j];
      w[4 * j] = q.x;
      w[4 * j + 1] = q.y;
      w[4 * j + 2] = q.z;
      w[4 * j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < WORDS; j++) w[j] = 0;
  }
}

template <typename T, bool RF32>
__device__ __forceinline__ void res_unpack(const uint32_t* w, float (&rv)[16]) {
  if constexpr (RF32) {
#pragma unroll
    for (int i = 0; i < 16; i++) rv[i] = __uint_as_float(w[i]);
  } else {
    const T* e = reinterpret_cast<const T*>(w);
#pragma unroll
    for (int i = 0; i < 16; i++) rv[i] = to_f<T>(e[i]);
  }
}

// The segment of a column: with SINGLE (one-segment GEMMs, the trunk's convolutions and linears) always the
// register-resident copy s0, so the per-unit epilogue code reads no descriptor memory at all.
template <bool SINGLE>
struct SegPick {
  const GemmParams& p;
  const EpiSeg& s0;
  __device__ __forceinline__ const EpiSeg& operator()(int col) const {
    if constexpr (SINGLE) return s0;
    else return seg_of(p, col);
  }
};

template <typename T, int BN, bool RF32, bool SINGLE>
__device__ __forceinline__ void tc_epilogue_tile(const GemmParams& p, const EpiSeg& s0, const RowInfo& ri,
                                                 const float* s_scale, const float* s_bias, uint32_t tacc, int n0,
                                                 int half) {
  const SegPick<SINGLE> pick{p, s0};
  if (p.mode == MODE_SEGMENTS) {
    // This warp's 16-column units are half, half + 2, half + 4, ... The residuals of a group of G units are all
    // loaded before any of them is used (the whole tile for 2-byte residuals), so that one memory latency covers
    // the group; then two units at a time share one TMEM wait.
    constexpr int WORDS = RF32 ? 16 : 8;  // residual words per 16 columns
    if constexpr (BN % 32 == 0) {
      // 32-column blocks: block j goes to warp half j % 2; one 32-column TMEM load per block
      constexpr int BLK = BN / 32;
      constexpr int MY = (BLK + 1) / 2;
      constexpr int G = RF32 ? (MY < 2 ? MY : 2) : MY;
#pragma unroll 1
      for (int g0 = 0; g0 < MY; g0 += G) {
        uint32_t rw[G][2 * WORDS];
#pragma unroll
        for (int k = 0; k < G; k++) {
          const int b = half + 2 * (g0 + k);
          if (b < BLK) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              const int col = n0 + b * 32 + hh * 16;
              const EpiSeg& s = pick(col);
              res_fetch<T, RF32>(s, ri, col - s.n0, &rw[k][hh * WORDS]);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < G; k++) {
          const int b = half + 2 * (g0 + k);
          if (b >= BLK) break;
          uint32_t x[32];
          tmem_ld32(tacc + b * 32, x);
          tmem_wait_ld();
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            const int col = n0 + b * 32 + hh * 16;
            const EpiSeg& s = pick(col);
            float v[16], rv[16], sc[16], bi[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __uint_as_float(x[hh * 16 + i]);
            res_unpack<T, RF32>(&rw[k][hh * WORDS], rv);
            if (s.flags & EPI_ACT) {  // the tables only cover GEMMs with a BN segment (at most PARAM_COLS wide)
              lds16(s_scale + col, sc);
              lds16(s_bias + col, bi);
            }
            epi_apply<T, 16>(s, ri, col - s.n0, v, rv, sc, bi);
          }
        }
      }
    } else {
      // 16-column units: unit u goes to warp half u % 2
      constexpr int UNITS = BN / 16;
      constexpr int MY = (UNITS + 1) / 2;
#pragma unroll 1
      for (int k = 0; k < MY; k++) {
        const int u = half + 2 * k;
        if (u >= UNITS) break;
        const int col = n0 + u * 16;
        const EpiSeg& s = pick(col);
        uint32_t rw[WORDS];
        res_fetch<T, RF32>(s, ri, col - s.n0, rw);
        uint32_t x[16];
        tmem_ld16(tacc + u * 16, x);
        tmem_wait_ld();
        float v[16], rv[16], sc[16], bi[16];
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = __uint_as_float(x[i]);
        res_unpack<T, RF32>(rw, rv);
        if (s.flags & EPI_ACT) {
          lds16(s_scale + col, sc);
          lds16(s_bias + col, bi);
        }
        epi_apply<T, 16>(s, ri, col - s.n0, v, rv, sc, bi);
      }
    }
  } else if (p.mode == MODE_SWIGLU) {
    const EpiSeg& s = p.seg[0];
#pragma unroll 1
    for (int c = half * (BN / 4); c < (half + 1) * (BN / 4); c += 16) {
      uint32_t ua[16], ug[16];
      tmem_ld16(tacc + c, ua);
      tmem_ld16(tacc + BN / 2 + c, ug);
      tmem_wait_ld();
      float h[16];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float a = __uint_as_float(ua[i]);
        float g = __uint_as_float(ug[i]);
        h[i] = act_fn<3>(a) * g * ri.mask;
      }
      if (ri.write)
        store_vec<T, 16>(reinterpret_cast<T*>(s.out_raw) + (size_t)ri.out_row * s.ld_raw + n0 / 2 + c, h);
    }
  } else {  // MODE_ROPE: Q|K|V columns, Q and K heads rotated in halves of head_dim / 2
    const EpiSeg& s = p.seg[0];
    const int hd = p.head_dim, hh = hd / 2;
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
      const int gcol = n0 + c;
      if (gcol < p.rope_rot_cols) {
        const int within = gcol % hd;
        if (within >= hh) continue;  // written with its pair
        uint32_t u0[16], u1[16];
        tmem_ld16(tacc + c, u0);
        tmem_ld16(tacc + c + hh, u1);
        tmem_wait_ld();
        const int head = gcol / hd;
        int table;
        if (gcol < p.rope_q_cols) table = head / p.rope_group;
        else table = head - p.rope_q_cols / hd;
        const float* ct = p.rope_cos + (size_t)table * p.rope_table_stride + (size_t)ri.pos * hh + within;
        const float* st = p.rope_sin + (size_t)table * p.rope_table_stride + (size_t)ri.pos * hh + within;
        float r0[16], r1[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          float x0 = __uint_as_float(u0[i]), x1 = __uint_as_float(u1[i]);
          float cs = __ldg(ct + i), sn = __ldg(st + i);
          r0[i] = (x0 * cs - x1 * sn) * ri.mask;
          r1[i] = (x0 * sn + x1 * cs) * ri.mask;
        }
        if (ri.write) {
          T* o = reinterpret_cast<T*>(s.out_raw) + (size_t)ri.out_row * s.ld_raw + gcol;
          store_vec<T, 16>(o, r0);
          store_vec<T, 16>(o + hh, r1);
        }
      } else {
        uint32_t u[16];
        tmem_ld16(tacc + c, u);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = __uint_as_float(u[i]) * ri.mask;
        if (ri.write) store_vec<T, 16>(reinterpret_cast<T*>(s.out_raw) + (size_t)ri.out_row * s.ld_raw + gcol, v);
      }
    }
  }
}

// RF32: the residual segments read a float32 residual stream (the bf16 tier).
template <typename T, int BN, bool RF32>
__global__ void __launch_bounds__(TcCfg<BN>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ GemmParams p) {
  using C = TcCfg<BN>;
  constexpr int fmt = sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC = make_idesc_f16(fmt, 128, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_scale = reinterpret_cast<float*>(stages + C::STAGES * C::STAGE_BYTES + C::BAR_BYTES);
  float* s_bias = s_scale + C::PARAM_COLS;
  GemmParams* s_params = reinterpret_cast<GemmParams*>(s_bias + C::PARAM_COLS);

  // The roles read the parameters from a shared-memory copy: fields of the __grid_constant__ struct reached through
  // references with run-time indices (segment lookups per 16 columns) cost hundreds of cycles each.
  static_assert(sizeof(GemmParams) <= C::PCOPY_BYTES && sizeof(GemmParams) % 16 == 0, "parameter copy");
  for (int i = threadIdx.x; i < (int)(sizeof(GemmParams) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(s_params)[i] = reinterpret_cast<const uint4*>(&p)[i];

  // per-column BN scale / bias of the act segments, staged once per CTA (zero where a segment has no BN); the
  // plan builder only gives segments with EPI_ACT to GEMMs of at most PARAM_COLS columns
  if (p.mode == MODE_SEGMENTS && p.n_total <= C::PARAM_COLS) {
    for (int col = threadIdx.x; col < p.n_total; col += blockDim.x) {
      const EpiSeg& s = seg_of(p, col);
      const bool act = (s.flags & EPI_ACT) != 0;
      s_scale[col] = act ? s.scale[col - s.n0] : 0.0f;
      s_bias[col] = act ? s.bias[col - s.n0] : 0.0f;
    }
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (p.g.rows + 127) / 128;
  const int n_tiles = p.n_total / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_per_tap = p.cin / 64;
  const int KB = p.taps * kb_per_tap;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * C::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above (barriers, TMEM, parameter and BN-table copies) overlaps the previous kernel's tail
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * 128;
        const int n0 = (tile % n_tiles) * BN;
        {
          for (int kb = 0; kb < KB; kb++) {
            if (!mbar_wait(&empty[stage], phase ^ 1, p.err, DEV_TIMEOUT_PRODUCER) || *abort_flag) {
              ok = false;
              *abort_flag = 1;
              break;
            }
            const int tap = kb / kb_per_tap;
            const int c0 = (kb - tap * kb_per_tap) * 64;
            uint8_t* sa = stages + stage * C::STAGE_BYTES;
            mbar_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sa, &tmA, &full[stage], c0, m0 + s_params->tap_off[tap]);
            tma_load_2d(sa + C::A_BYTES, &tmB, &full[stage], kb * 64, n0);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        // let copies already issued land before the CTA exits (bounded)
        unsigned long long t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, local++) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, DEV_TIMEOUT_MMA) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
        {
          // Two K-blocks (8 MMAs) per barrier wait and commit: tcgen05.mma issue blocks once a few MMAs are
          // queued, so the wait / commit latency between groups would otherwise idle the tensor pipe; with 4 MMAs
          // per group it cost a third of the throughput, with 8 under 2%.
          for (int kb = 0; kb < KB && ok; kb += 2) {
            const int nk = KB - kb >= 2 ? 2 : 1;
            int st[2];
            uint32_t ph[2];
            for (int j = 0; j < nk; j++) {
              st[j] = stage;
              ph[j] = phase;
              if (++stage == C::STAGES) {
                stage = 0;
                phase ^= 1;
              }
            }
            for (int j = 0; j < nk; j++) {
              if (!mbar_try_wait(&full[st[j]], ph[j]) &&
                  (*abort_flag || !mbar_wait(&full[st[j]], ph[j], p.err, DEV_TIMEOUT_MMA))) {
                ok = false;
                break;
              }
            }
            if (!ok) break;
            tc_fence_after();
            for (int j = 0; j < nk; j++) {
              const uint32_t sa = smem_u32(stages + st[j] * C::STAGE_BYTES);
              const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
              for (int k = 0; k < 4; k++)
                umma_f16(d_tmem, make_sw128_desc(sa + k * 32), make_sw128_desc(sb + k * 32), IDESC,
                         (kb | j | k) != 0);
            }
            for (int j = 0; j < nk; j++) umma_commit(&empty[st[j]]);
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(drain);  // wait for MMAs in flight before TMEM is released
        mbar_wait(drain, 0, p.err, DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue warps 2..9: TMEM lane quarter = warp % 4, column half = (warp - 2) / 4 ----
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const GemmParams& sp = *s_params;
    int local = 0;
    RowInfo ri_next = row_info(sp.g, (blockIdx.x / n_tiles) * 128 + row_in_tile);
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, local++) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int n0 = (tile % n_tiles) * BN;
      const RowInfo ri = ri_next;
      // the next tile's row (and its mask load) is fetched now, so the load overlaps this tile's epilogue
      const int tnext = tile + gridDim.x;
      if (tnext < num_tiles) ri_next = row_info(sp.g, (tnext / n_tiles) * 128 + row_in_tile);
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, DEV_TIMEOUT_EPILOGUE) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t tacc = tmem_base + acc * C::ACC_COLS + ((uint32_t)(q * 32) << 16);
      tc_epilogue_tile<T, BN, RF32, false>(sp, sp.seg[0], ri, s_scale, s_bias, tacc, n0, half);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ================================================================================================================
// SIMT kernel (the f32 tier): 64 x 64 tile, 128 threads, 8 rows x 4 columns per thread, K chunks of 16 channels of
// one tap, double-buffered in shared memory with the next chunk's 16-byte global loads in flight during the FMAs.
// Every output sums its K terms in the same order (taps, then channels) whatever its tile: results do not depend on
// the batch position. Needs lda % 4 == 0 and cin % 16 == 0 (checked by the host).
// ================================================================================================================

constexpr int SIMT_THREADS = 128;

template <typename T>
__global__ void __launch_bounds__(SIMT_THREADS) gemm_simt_kernel(const __grid_constant__ GemmParams p) {
  pdl_wait();
  pdl_trigger();
  static_assert(sizeof(T) == 4, "the SIMT GEMM is the float32 path");
  __shared__ __align__(16) float As[2][16][64 + 4];  // [buffer][k][row]
  __shared__ __align__(16) float Ws[2][16][64 + 4];  // [buffer][k][column]
  const int t = threadIdx.x;
  const int tx = t & 15, ty = t >> 4;  // columns tx * 4 .. + 3, rows ty * 8 .. + 7
  const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
  const float* A = reinterpret_cast<const float*>(p.a);
  const float* W = reinterpret_cast<const float*>(p.w);
  const int K = p.taps * p.cin;
  const int chunks_per_tap = p.cin / 16;
  const int nchunks = p.taps * chunks_per_tap;
  // this thread's two 16-byte loads of each operand per chunk: rows / columns (t >> 2) and (t >> 2) + 32, channels
  // (t & 3) * 4 .. + 3
  const int lr = t >> 2, lk = (t & 3) * 4;
  float4 ra[2], rw[2];
  auto fetch = [&](int ch) {
    const int tap = ch / chunks_per_tap;
    const int c0 = (ch - tap * chunks_per_tap) * 16 + lk;
    const int off = p.tap_off[tap];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int row = m0 + lr + 32 * h + off;
      ra[h] = row >= 0 && row < p.a_rows ? *reinterpret_cast<const float4*>(A + (size_t)row * p.lda + c0)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      const int n = n0 + lr + 32 * h;
      rw[h] = n < p.n_total ? *reinterpret_cast<const float4*>(W + (size_t)n * K + tap * p.cin + c0)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int rr = lr + 32 * h;
      As[buf][lk + 0][rr] = ra[h].x;
      As[buf][lk + 1][rr] = ra[h].y;
      As[buf][lk + 2][rr] = ra[h].z;
      As[buf][lk + 3][rr] = ra[h].w;
      Ws[buf][lk + 0][rr] = rw[h].x;
      Ws[buf][lk + 1][rr] = rw[h].y;
      Ws[buf][lk + 2][rr] = rw[h].z;
      Ws[buf][lk + 3][rr] = rw[h].w;
    }
  };
  float acc[8][4] = {};
  fetch(0);
  stash(0);
  __syncthreads();
  for (int ch = 0; ch < nchunks; ch++) {
    const int buf = ch & 1;
    if (ch + 1 < nchunks) fetch(ch + 1);
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
      const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], wv[j], acc[i][j]);
    }
    if (ch + 1 < nchunks) stash(buf ^ 1);
    __syncthreads();
  }
  const int ncol = n0 + tx * 4;
  if (ncol >= p.n_total) return;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int r = m0 + ty * 8 + i;
    const RowInfo ri = row_info(p.g, r);
    float v[4] = {acc[i][0], acc[i][1], acc[i][2], acc[i][3]};
    const EpiSeg& s = seg_of(p, ncol);
    const int c = ncol - s.n0;
    float rv[4];
    epi_load_res<T, 4>(s, ri, c, rv);
    epi_apply<T, 4>(s, ri, c, v, rv, s.scale + c, s.bias + c);
  }
}

}  // namespace kc
