// Memory-bound kernels of the katago-rs B200 forward pass: input layout conversion, per-board statistics and
// biases, masked global pooling, the small head matmuls, batch-norm/RMSNorm elementwise passes, and the SIMT
// attention / RoPE / SwiGLU paths of the float32 tier. Semantics follow tools/bin2onnx/bin2onnx.py GraphBuilder
// (line numbers on each kernel).
#pragma once

#include "gemm.cuh"
#include "../../include/katago_cuda.h"

namespace kc {

// Positions of a board in the padded board layout (PBL): row of (b, y, x) = b * 400 + (y + 1) * 20 + x.
__host__ __device__ __forceinline__ int pbl_row(int b, int y, int x) { return b * 400 + (y + 1) * 20 + x; }

// The point of a row's input that the network sees at (y, x) under `sym` (bit 0 flipY, bit 1 flipX, bit 2
// transpose): the inverse of SymmetryHelpers::copy_inputs_with_symmetry's NCHW copy (nninputs.rs:756-831, 872),
// which moves source point (h, w) to (h', w') = flipY/flipX of (h, w), transposed after the flips (with the flips
// exchanged first when transposing).
__host__ __device__ __forceinline__ int sym_src(int sym, int y, int x) {
  const bool fy = (sym & 1) != 0, fx = (sym & 2) != 0;
  int h, w;
  if (sym & 4) {
    w = fx ? 18 - y : y;
    h = fy ? 18 - x : x;
  } else {
    h = fy ? 18 - y : y;
    w = fx ? 18 - x : x;
  }
  return h * 19 + w;
}

// The spatial input of a forward pass: float32 planes [n][cin][361] in the reference layout, or bit-packed planes
// [n][cin][12] (point p of a plane at bit p % 32 of word p / 32; every spatial feature of the reference's inputs is
// 0 or 1, nninputs.rs fill_row_v7 :1336) with one symmetry per board applied as the planes are read.
constexpr int kPackedWordsPerPlane = KC_PACKED_WORDS_PER_PLANE;
struct InputSrc {
  const float* f = nullptr;
  const uint32_t* bits = nullptr;
  const int* sym = nullptr;
};

// Plane c of board b at the network's (y, x).
__device__ __forceinline__ float input_at(const InputSrc& in, int b, int cin, int c, int y, int x) {
  if (in.bits) {
    const int p = sym_src(__ldg(in.sym + b), y, x);
    const uint32_t w = __ldg(in.bits + ((size_t)b * cin + c) * kPackedWordsPerPlane + (p >> 5));
    return (float)((w >> (p & 31)) & 1u);
  }
  return __ldg(in.f + ((size_t)b * cin + c) * 361 + y * 19 + x);
}

// ---------------------------------------------------------------------------------------------------------------
// Input: NCHW float32 [n][cin][19*19] -> stem layout T rows [b * brows + (y + pad) * stride + x][cpad], and the
// per-PBL-row on-board mask (input channel 0, bin2onnx.py setup_mask :1203-1206).
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void prep_input_kernel(const __grid_constant__ InputSrc in, int n, int cin, T* __restrict__ out, int cpad,
                                  int brows, int stride, int pad, float* __restrict__ rowmask) {
  pdl_wait();
  pdl_trigger();
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * 361) return;
  int b = idx / 361, pos = idx - b * 361;
  int y = pos / 19, x = pos - y * 19;
  T* dst = out + ((size_t)b * brows + (size_t)(y + pad) * stride + x) * cpad;
  // cpad is a multiple of 8: the row is written as 16-byte vectors of 8 channels
  for (int c0 = 0; c0 < cpad; c0 += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = c0 + i < cin ? input_at(in, b, cin, c0 + i, y, x) : 0.0f;
    store_vec<T, 8>(dst + c0, v);
  }
  rowmask[pbl_row(b, y, x)] = input_at(in, b, cin, 0, y, x);
}

// ---------------------------------------------------------------------------------------------------------------
// Input -> the stem's im2col operand (tensor-core tiers), in two steps.
// prep_pixels_kernel: planes [n][cin][361] float32 -> pixel-major px [n][G][G][CP] (G = 19 + 2 pad, CP = cin
// rounded up to 8; the pad-wide border and planes [cin, CP) zero), and the per-PBL-row on-board mask (input channel
// 0, bin2onnx.py setup_mask :1203-1206). One thread per grid pixel.
// prep_im2col_kernel: row = PBL row of (b, y, x), columns [tap * CP, tap * CP + CP) = px[b][y + ky d][x + kx d]
// (tap = ky * k + kx; the border supplies the stem conv's zero padding), columns [k * k * CP, kpad) and halo rows
// zero: K = kpad (640 for a 5x5 stem over 22 planes) instead of 25 taps of 64 padded channels. One thread per
// (row, tap) copying CP / 8 16-byte vectors; tap k * k zeroes the tail.
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void prep_pixels_kernel(const __grid_constant__ InputSrc in, int n, int cin, int pad, T* __restrict__ px,
                                   int cp, float* __restrict__ rowmask) {
  pdl_wait();
  pdl_trigger();
  const int G = 19 + 2 * pad;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * G * G) return;
  const int b = idx / (G * G), q = idx - b * G * G;
  const int gy = q / G, gx = q - gy * G;
  const int y = gy - pad, x = gx - pad;
  const bool on = y >= 0 && y < 19 && x >= 0 && x < 19;
  T* dst = px + (size_t)idx * cp;
  if (on && in.bits) {
    // one packed word per plane holds this point's bit
    const int p = sym_src(__ldg(in.sym + b), y, x);
    const uint32_t* wp = in.bits + (size_t)b * cin * kPackedWordsPerPlane + (p >> 5);
    const int sh = p & 31;
    for (int c0 = 0; c0 < cp; c0 += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; i++)
        v[i] = c0 + i < cin ? (float)((__ldg(wp + (size_t)(c0 + i) * kPackedWordsPerPlane) >> sh) & 1u) : 0.0f;
      store_vec<T, 8>(dst + c0, v);
      if (c0 == 0) rowmask[pbl_row(b, y, x)] = v[0];
    }
    return;
  }
  const float* src = in.f + (size_t)b * cin * 361 + (on ? y * 19 + x : 0);
  for (int c0 = 0; c0 < cp; c0 += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = on && c0 + i < cin ? __ldg(src + (size_t)(c0 + i) * 361) : 0.0f;
    store_vec<T, 8>(dst + c0, v);
  }
  if (on) rowmask[pbl_row(b, y, x)] = __ldg(src);
}

template <typename T>
__global__ void prep_im2col_kernel(const T* __restrict__ px, int n, int k, int d, int pad, int cp,
                                   T* __restrict__ out, int kpad) {
  pdl_wait();
  pdl_trigger();
  const int taps = k * k;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * 400 * (taps + 1)) return;
  const int r = idx / (taps + 1), t = idx - r * (taps + 1);
  const int b = r / 400, rr = r - b * 400;
  const int y = rr / 20 - 1, x = rr - (rr / 20) * 20;
  const bool on = y >= 0 && x < 19;
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)r * kpad);
  const int nv = cp >> 3;
  if (t < taps) {
    uint4* d0 = dst + t * nv;
    if (on) {
      const int ky = t / k, kx = t - ky * k;
      const int G = 19 + 2 * pad;
      const uint4* s = reinterpret_cast<const uint4*>(px + ((size_t)b * G * G + (size_t)(y + ky * d) * G + (x + kx * d)) * cp);
      for (int v = 0; v < nv; v++) d0[v] = __ldg(s + v);
    } else {
      for (int v = 0; v < nv; v++) d0[v] = make_uint4(0, 0, 0, 0);
    }
  } else {
    for (int v = taps * nv; v < (kpad >> 3); v++) dst[v] = make_uint4(0, 0, 0, 0);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Per board: mask sum and the pooling scales (bin2onnx.py setup_mask :1207-1215), and the trunk's per-board bias:
// global features x initial matmul, plus the SGF-metadata encoder for human-SL nets (bin2onnx.py :1467-1487).
// ---------------------------------------------------------------------------------------------------------------
struct BoardParams {
  const float* spatial;  // [n][cin][361] (channel 0 = mask), or null with bits
  const uint32_t* bits;  // [n][cin][12] bit-packed planes (InputSrc), or null
  int cin;
  const float* glob;     // [n][G]
  int G;
  const float* wg;       // [G][C]
  int C;
  const float* meta;     // [n][192] or null
  const float* m1; const float* b1; int h1; int act1;   // [192][h1]
  const float* m2; const float* b2; int h2; int act2;   // [h1][h2]
  const float* m3;                                      // [h2][C]
  float* board_bias;     // [n][C]
  float* mask_sum;       // [n]
  float* scale1;         // [n]
  float* scale2;         // [n]
};

static __global__ void board_kernel(const __grid_constant__ BoardParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[256];
  __shared__ float hbuf[2][512];
  const int b = blockIdx.x;
  float s = 0.0f;
  if (p.bits) {
    // plane 0 (the mask) as bits: the count of on-board points (a symmetry moves points, it does not change it)
    if (threadIdx.x < kPackedWordsPerPlane)
      s = (float)__popc(__ldg(p.bits + (size_t)b * p.cin * kPackedWordsPerPlane + threadIdx.x));
  } else {
    for (int i = threadIdx.x; i < 361; i += blockDim.x) s += p.spatial[(size_t)b * p.cin * 361 + i];
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float ms = red[0];
    float cen = sqrtf(ms) - 14.0f;
    p.mask_sum[b] = ms;
    p.scale1[b] = cen * 0.1f;
    float sq = cen * cen;
    sq = sq * 0.01f;
    p.scale2[b] = sq - 0.1f;
  }
  if (p.meta) {
    const float* mi = p.meta + (size_t)b * 192;
    for (int o = threadIdx.x; o < p.h1; o += blockDim.x) {
      float a = 0.0f;
      for (int i = 0; i < 192; i++) a += mi[i] * p.m1[(size_t)i * p.h1 + o];
      hbuf[0][o] = act_apply(a + p.b1[o], p.act1);
    }
    __syncthreads();
    for (int o = threadIdx.x; o < p.h2; o += blockDim.x) {
      float a = 0.0f;
      for (int i = 0; i < p.h1; i++) a += hbuf[0][i] * p.m2[(size_t)i * p.h2 + o];
      hbuf[1][o] = act_apply(a + p.b2[o], p.act2);
    }
    __syncthreads();
  }
  for (int c = threadIdx.x; c < p.C; c += blockDim.x) {
    float a = 0.0f;
    for (int i = 0; i < p.G; i++) a += p.glob[(size_t)b * p.G + i] * p.wg[(size_t)i * p.C + c];
    if (p.meta) {
      float m = 0.0f;
      for (int i = 0; i < p.h2; i++) m += hbuf[1][i] * p.m3[(size_t)i * p.C + c];
      a = a + m;
    }
    p.board_bias[(size_t)b * p.C + c] = a;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Masked pooling over a board's 361 points of channels [c0, c0 + C) of a PBL tensor (already masked):
// gpool (bin2onnx.py :1222-1230): [mean, mean * scale1, max(x + (mask * 1e4 - 1e4))];
// value (bin2onnx.py :1232-1239): [mean, mean * scale1, mean * scale2]. out [n][3C] float32.
// One block of POOL_THREADS per board: thread t takes the 8 channels (t % CG) * 8.. (CG = ceil(C / 8) groups) of
// every RL-th point (RL = POOL_THREADS / CG row lanes), reading 16-byte vectors, then the row lanes are reduced in
// shared memory ([RL][CG * 8] floats, twice). C is at most 8 * POOL_THREADS; c0 and the row pitch are multiples of 8
// (the channels up to the next multiple of 8 are read and dropped).
// ---------------------------------------------------------------------------------------------------------------
constexpr int POOL_THREADS = 512;
// Shared memory of one board's pooling: [RL][Cp] sums, then [RL][Cp] maxima.
__host__ __device__ constexpr int pool_red_floats(int C) {
  return 2 * (POOL_THREADS / ((C + 7) / 8)) * ((C + 7) / 8) * 8;
}
// Board b's pooled [3C] into o, by a block of POOL_THREADS threads (red: pool_red_floats(C) floats of shared memory;
// o may be shared or global memory). Ends with the block synchronised when o is shared.
template <typename T>
__device__ __forceinline__ void pool_board(const T* __restrict__ x, int ld, int c0, int C, const float* __restrict__ rowmask,
                                           const float* __restrict__ mask_sum, const float* __restrict__ scale1,
                                           const float* __restrict__ scale2, int value_mode, int b, float* red,
                                           float* o) {
  const int CG = (C + 7) >> 3, Cp = CG * 8, RL = POOL_THREADS / CG;
  const int g = threadIdx.x % CG, rl = threadIdx.x / CG;
  float* ssum = red;
  float* smax = red + RL * Cp;
  if (rl < RL) {
    float s[8], mx[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      s[i] = 0.0f;
      mx[i] = -INFINITY;
    }
#pragma unroll 4
    for (int pos = rl; pos < 361; pos += RL) {
      const int y = pos / 19, xx = pos - y * 19;
      const int r = pbl_row(b, y, xx);
      float v[8];
      load_vec<T, 8>(x + (size_t)r * ld + c0 + g * 8, v);
      const float biasv = __ldg(rowmask + r) * 1e4f - 1e4f;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        s[i] += v[i];
        mx[i] = fmaxf(mx[i], v[i] + biasv);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      ssum[rl * Cp + g * 8 + i] = s[i];
      smax[rl * Cp + g * 8 + i] = mx[i];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += POOL_THREADS) {
    float s = 0.0f, mx = -INFINITY;
    for (int i = 0; i < RL; i++) {
      s += ssum[i * Cp + c];
      mx = fmaxf(mx, smax[i * Cp + c]);
    }
    const float mean = s / mask_sum[b];
    o[c] = mean;
    o[C + c] = mean * scale1[b];
    o[2 * C + c] = value_mode ? mean * scale2[b] : mx;
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(POOL_THREADS) pool_kernel(const T* __restrict__ x, int ld, int c0, int C,
                                                            const float* __restrict__ rowmask,
                                                            const float* __restrict__ mask_sum,
                                                            const float* __restrict__ scale1,
                                                            const float* __restrict__ scale2, int value_mode,
                                                            float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float pool_red[];
  const int b = blockIdx.x;
  pool_board<T>(x, ld, c0, C, rowmask, mask_sum, scale1, scale2, value_mode, b, pool_red, out + (size_t)b * 3 * C);
}

// ---------------------------------------------------------------------------------------------------------------
// Small per-board matmul: out[b][off + o * ostride] = act(sum_i in[b][i] * W[i][o] (+ bias[o])).
// A block computes 32 outputs (blockIdx.y) for NB boards (blockIdx.x): its 8 warps split the input dimension,
// lane = output (coalesced weight rows), and the 8 partial sums are added in shared memory. grid (ceil(n / NB),
// ceil(oc / 32)), block FC_THREADS, shared memory NB * ic floats (the boards' inputs).
// ---------------------------------------------------------------------------------------------------------------
constexpr int FC_BOARDS = 4;
constexpr int FC_THREADS = 256;
template <int NB>
__global__ void __launch_bounds__(FC_THREADS) fc_kernel(const float* __restrict__ in, int in_ld, int ic,
                                                        const float* __restrict__ w, int oc,
                                                        const float* __restrict__ bias, int act,
                                                        float* __restrict__ out, int out_ld, int out_off,
                                                        int out_stride, int n) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xin[];  // [NB][ic]
  __shared__ float part[FC_THREADS / 32][NB][32];
  const int b0 = blockIdx.x * NB;
  const int nb = n - b0 < NB ? n - b0 : NB;
  for (int i = threadIdx.x; i < NB * ic; i += blockDim.x) {
    const int k = i / ic;
    xin[i] = k < nb ? in[(size_t)(b0 + k) * in_ld + (i - k * ic)] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.y * 32 + lane;
  constexpr int NW = FC_THREADS / 32;
  const int i0 = (int)((long long)ic * warp / NW), i1 = (int)((long long)ic * (warp + 1) / NW);
  float a[NB];
#pragma unroll
  for (int k = 0; k < NB; k++) a[k] = 0.0f;
  if (o < oc) {
#pragma unroll 4
    for (int i = i0; i < i1; i++) {
      const float wv = __ldg(w + (size_t)i * oc + o);
#pragma unroll
      for (int k = 0; k < NB; k++) a[k] += xin[k * ic + i] * wv;
    }
  }
#pragma unroll
  for (int k = 0; k < NB; k++) part[warp][k][lane] = a[k];
  __syncthreads();
  if (threadIdx.x < NB * 32) {
    const int k = threadIdx.x >> 5;
    const int oo = blockIdx.y * 32 + (threadIdx.x & 31);
    if (k < nb && oo < oc) {
      float v = 0.0f;
#pragma unroll
      for (int j = 0; j < NW; j++) v += part[j][k][threadIdx.x & 31];
      if (bias) v = v + bias[oo];
      out[(size_t)(b0 + k) * out_ld + out_off + (size_t)oo * out_stride] = act_apply(v, act);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// y[r][c] = act((x[r][xc0 + c] (+ board_bias[b][c])) * scale[c] + bias[c]) * mask[r]  for c < C;
// the gpool-biased regular branch (bin2onnx.py :1256-1258), the policy head's p1 (:1503-1504), and the standalone
// bn_act_mask (:1170) where a producer could not fuse it. Rows [0, rows); y's channels [C, Cw) are written as 0.
// ---------------------------------------------------------------------------------------------------------------
// One thread per 8 channels of a row (16-byte loads and stores); the activation fixed at compile time. x's and y's
// row pitches and xc0 are multiples of 8 elements, Cw a multiple of 8.
// Channels [c, c + 8) of row r with mask m; bb: the row's board bias (or null).
template <typename TI, typename T, int ACT>
__device__ __forceinline__ void bias_bnact_vec(const TI* __restrict__ x, int xld, int xc0, const float* bb,
                                               const float* __restrict__ scale, const float* __restrict__ bias,
                                               float m, int r, int c, int C, T* __restrict__ y, int yld) {
  float o[8];
  if (c < C && m != 0.0f) {
    float v[8];
    load_vec<TI, 8>(x + (size_t)r * xld + xc0 + c, v);
    if (c + 8 <= C && (C & 3) == 0) {
      // whole vector inside the channels: parameters as 16-byte loads
      float sc[8], bi[8], bv[8];
      load_vec<float, 8>(scale + c, sc);
      load_vec<float, 8>(bias + c, bi);
      if (bb) load_vec<float, 8>(bb + c, bv);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float t = v[i];
        if (bb) t = t + bv[i];
        t = t * sc[i];
        t = t + bi[i];
        o[i] = act_fn<ACT>(t) * m;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int cc = c + i;
        if (cc < C) {
          float t = v[i];
          if (bb) t = t + bb[cc];
          t = t * __ldg(scale + cc);
          t = t + __ldg(bias + cc);
          o[i] = act_fn<ACT>(t) * m;
        } else {
          o[i] = 0.0f;
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) o[i] = 0.0f;
  }
  store_vec<T, 8>(y + (size_t)r * yld + c, o);
}

template <typename TI, typename T, int ACT>
__global__ void bias_bnact_kernel(const TI* __restrict__ x, int xld, int xc0, const float* __restrict__ board_bias,
                                  const float* __restrict__ scale, const float* __restrict__ bias,
                                  const float* __restrict__ rowmask, int rows, int C, int Cw, T* __restrict__ y,
                                  int yld) {
  pdl_wait();
  pdl_trigger();
  const int per_row = Cw >> 3;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int r = idx / per_row;
  const int c = (idx - r * per_row) << 3;
  const float* bb = board_bias ? board_bias + (size_t)(r / 400) * C : nullptr;
  bias_bnact_vec<TI, T, ACT>(x, xld, xc0, bb, scale, bias, __ldg(rowmask + r), r, c, C, y, yld);
}

// ---------------------------------------------------------------------------------------------------------------
// The gpool block's middle in one launch (bin2onnx.py gpool_block :1250-1261 after the two convolutions): per board
// (one block of POOL_THREADS), pool the gpool branch G (pool_board), the pooled vector times gpool_to_bias
// ([3 gc][rc], fc_kernel's arithmetic: eight input slices summed in order) into the regular branch's bias, then
// T1 = act((REG + bias) * scale + shift) * mask over the board's 400 rows (bias_bnact_vec). Shared memory:
// pool_red_floats(gc) + 3 gc + 8 rc + rc floats. With gridDim.y = S > 1 (small batches, where one block per board
// leaves most SMs idle) block (b, s) pools the whole board but computes only its column group's bias entries and
// output vectors: vectors [cw/8 * s / S, cw/8 * (s + 1) / S) of each row. Every output value takes the same
// arithmetic in the same order whatever S is.
// ---------------------------------------------------------------------------------------------------------------
struct GpoolMidParams {
  const void* g;     // gpool branch [rows][ld_g], channels [0, gc)
  int ld_g, gc;
  const void* reg;   // regular branch [rows][ld_reg], channels [0, rc)
  int ld_reg, rc;
  const float* w;    // [3 gc][rc]
  const float* scale;
  const float* shift;
  const float* rowmask;
  const float* mask_sum;
  const float* scale1;
  const float* scale2;
  void* y;           // T1 [rows][ld_y], channels [0, cw) written (zero from rc on)
  int ld_y, cw;
};

template <typename T, int ACT>
__global__ void __launch_bounds__(POOL_THREADS) gpool_mid_kernel(const __grid_constant__ GpoolMidParams p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float gm_smem[];
  float* red = gm_smem;
  float* pooled = red + pool_red_floats(p.gc);
  float* part = pooled + 3 * p.gc;  // [8][rc]
  float* gb = part + 8 * p.rc;
  const int b = blockIdx.x;
  pool_board<T>(static_cast<const T*>(p.g), p.ld_g, 0, p.gc, p.rowmask, p.mask_sum, p.scale1, p.scale2, 0, b, red,
                pooled);
  // this block's output vectors [v0, v1) of each row and bias columns [o0, o1)
  const int per_row = p.cw >> 3;
  const int v0 = per_row * (int)blockIdx.y / (int)gridDim.y, v1 = per_row * ((int)blockIdx.y + 1) / (int)gridDim.y;
  const int o0 = v0 * 8, o1 = v1 * 8 < p.rc ? v1 * 8 : p.rc, ncol = o1 - o0;
  const int ic = 3 * p.gc;
  constexpr int NS = 8;  // input slices, as fc_kernel's eight warps
  for (int q = threadIdx.x; q < NS * ncol; q += POOL_THREADS) {
    const int sl = q / ncol, o = o0 + q - sl * ncol;
    const int i0 = (int)((long long)ic * sl / NS), i1 = (int)((long long)ic * (sl + 1) / NS);
    float a = 0.0f;
    for (int i = i0; i < i1; i++) a += pooled[i] * __ldg(p.w + (size_t)i * p.rc + o);
    part[sl * p.rc + o] = a;
  }
  __syncthreads();
  for (int o = o0 + (int)threadIdx.x; o < o1; o += POOL_THREADS) {
    float v = 0.0f;
#pragma unroll
    for (int j = 0; j < NS; j++) v += part[j * p.rc + o];
    gb[o] = v;
  }
  __syncthreads();
  const int nv = v1 - v0;
  for (int idx = threadIdx.x; idx < 400 * nv; idx += POOL_THREADS) {
    const int rr = idx / nv;
    const int r = b * 400 + rr;
    const int c = (v0 + idx - rr * nv) << 3;
    bias_bnact_vec<T, T, ACT>(static_cast<const T*>(p.reg), p.ld_reg, 0, gb, p.scale, p.shift, __ldg(p.rowmask + r),
                              r, c, p.rc, static_cast<T*>(p.y), p.ld_y);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Transformer RMSNorm per row (bin2onnx.py transformer_rmsnorm :1330-1340): x * (1 / sqrt(sum(x^2) / C + eps)) * w
// * mask. One warp per row.
// ---------------------------------------------------------------------------------------------------------------
template <typename TI, typename T>
__global__ void rmsnorm_kernel(const TI* __restrict__ x, int ld, int C, const float* __restrict__ w, float eps,
                               const float* __restrict__ rowmask, int rows, T* __restrict__ y, int yld) {
  pdl_wait();
  pdl_trigger();
  int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const TI* xr = x + (size_t)r * ld;
  float ss = 0.0f;
  for (int c = lane; c < C; c += 32) {
    float v = to_f<TI>(xr[c]);
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  float ms = ss / (float)C;
  float den = sqrtf(ms + eps);
  float rms = 1.0f / den;
  float m = rowmask[r];
  T* yr = y + (size_t)r * yld;
  for (int c = lane; c < C; c += 32) yr[c] = from_f<T>(to_f<TI>(xr[c]) * rms * w[c] * m);
}

// ---------------------------------------------------------------------------------------------------------------
// Row RMSNorm with 128-bit loads: one warp per PBL row, the row's C channels (C = 128 nv, nv <= 8) held in
// registers as 4-channel vectors (lane l holds channels 128 i + 4 l .. + 3). TIP = false: the transformer block
// norm, y = x * rms * w * mask (bin2onnx.py transformer_rmsnorm :1330-1340); TIP = true: the per-point trunk tip,
// y = act(x * rms * gamma + beta) * mask (trunk_tip_rmsnorm :1440-1463). rms = 1 / sqrt(sum(x^2) / C + eps).
// ---------------------------------------------------------------------------------------------------------------
template <typename U>
__device__ __forceinline__ float4 load4(const U* p) {
  if constexpr (std::is_same<U, float>::value) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const U* e = reinterpret_cast<const U*>(&u);
    return make_float4(to_f<U>(e[0]), to_f<U>(e[1]), to_f<U>(e[2]), to_f<U>(e[3]));
  }
}

template <typename U>
__device__ __forceinline__ void store4(U* p, float a, float b, float c, float d) {
  if constexpr (std::is_same<U, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
    return;
  }
  uint2 u;
  U* e = reinterpret_cast<U*>(&u);
  e[0] = from_f<U>(a);
  e[1] = from_f<U>(b);
  e[2] = from_f<U>(c);
  e[3] = from_f<U>(d);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename TI, typename T, bool TIP>
__global__ void rms_rows_kernel(const TI* __restrict__ x, int ld, int nv, const float* __restrict__ w,
                                const float* __restrict__ beta, int act, float eps,
                                const float* __restrict__ rowmask, int rows, T* __restrict__ y, int yld) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const TI* xr = x + (size_t)r * ld + lane * 4;
  float4 v[8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i < nv) {
      v[i] = load4<TI>(xr + i * 128);
      ss += v[i].x * v[i].x;
      ss += v[i].y * v[i].y;
      ss += v[i].z * v[i].z;
      ss += v[i].w * v[i].w;
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float ms = ss / (float)(nv * 128);
  const float den = sqrtf(ms + eps);
  const float rms = 1.0f / den;
  const float m = rowmask[r];
  T* yr = y + (size_t)r * yld + lane * 4;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i < nv) {
      const int c = i * 128 + lane * 4;
      const float4 g = __ldg(reinterpret_cast<const float4*>(w + c));
      float o[4] = {v[i].x * rms, v[i].y * rms, v[i].z * rms, v[i].w * rms};
      const float gg[4] = {g.x, g.y, g.z, g.w};
      if constexpr (TIP) {
        const float4 bt = __ldg(reinterpret_cast<const float4*>(beta + c));
        const float bb[4] = {bt.x, bt.y, bt.z, bt.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          float t = o[k] * gg[k];
          t = t + bb[k];
          o[k] = act_apply(t, act) * m;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; k++) o[k] = o[k] * gg[k] * m;
      }
      store4<T>(yr + i * 128, o[0], o[1], o[2], o[3]);
    }
  }
}

// Spatial trunk-tip RMSNorm (trunk_tip_rmsnorm :1440-1463 with one rms per board over its channels x on-board
// points) in two row-parallel steps. Step 1: the sum of squares of each PBL row's C = 128 nv channels, one warp per
// row.
template <typename TI>
__global__ void row_sumsq_kernel(const TI* __restrict__ x, int ld, int nv, int rows, float* __restrict__ ss) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const TI* xr = x + (size_t)r * ld + lane * 4;
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i < nv) {
      const float4 v = load4<TI>(xr + i * 128);
      s += v.x * v.x;
      s += v.y * v.y;
      s += v.z * v.z;
      s += v.w * v.w;
    }
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) ss[r] = s;
}

// Step 2, one warp per row (8 rows per block of 256 threads): the board total of the on-board rows' sums of squares
// (each block adds the 400 values of the one or two boards its rows belong to, in the same order for every block),
// rms = 1 / sqrt(total / (on-board points x C) + eps), then y = act(x * rms * gamma + beta) * mask as the per-point
// tip.
template <typename TI, typename T>
__global__ void tip_spatial_apply_kernel(const TI* __restrict__ x, int ld, int nv, const float* __restrict__ ss,
                                         const float* __restrict__ rowmask, const float* __restrict__ mask_sum,
                                         const float* __restrict__ gamma, const float* __restrict__ beta, int act,
                                         float eps, int rows, T* __restrict__ y, int yld) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[2][8];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  const int bfirst = (blockIdx.x * 8) / 400;
  const int blast = min(blockIdx.x * 8 + 7, rows - 1) / 400;
#pragma unroll
  for (int bi = 0; bi < 2; bi++) {
    float t = 0.0f;
    if (bfirst + bi <= blast) {
      const int b0 = (bfirst + bi) * 400;
      for (int k = threadIdx.x; k < 400; k += 256) t += ss[b0 + k] * rowmask[b0 + k];
    }
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) part[bi][warp] = t;
  }
  __syncthreads();
  if (r >= rows) return;
  const int bi = r / 400 - bfirst;
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) t += part[bi][w];
  const float count = mask_sum[r / 400] * (float)(nv * 128);
  const float ms = t / count;
  const float rms = 1.0f / sqrtf(ms + eps);
  const float m = rowmask[r];
  const TI* xr = x + (size_t)r * ld + lane * 4;
  T* yr = y + (size_t)r * yld + lane * 4;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i < nv) {
      const int c = i * 128 + lane * 4;
      const float4 v = load4<TI>(xr + i * 128);
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + c));
      const float4 bt = __ldg(reinterpret_cast<const float4*>(beta + c));
      const float xv[4] = {v.x * rms, v.y * rms, v.z * rms, v.w * rms};
      const float gg[4] = {g.x, g.y, g.z, g.w}, bb[4] = {bt.x, bt.y, bt.z, bt.w};
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        float u = xv[k] * gg[k];
        u = u + bb[k];
        o[k] = act_apply(u, act) * m;
      }
      store4<T>(yr + i * 128, o[0], o[1], o[2], o[3]);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Trunk-tip RMSNorm (bin2onnx.py trunk_tip_rmsnorm :1440-1463): act(x * rms * gamma + beta) * mask, rms per point
// over channels, or (spatial) one rms per board over channels x on-board points. One block per board.
// ---------------------------------------------------------------------------------------------------------------
template <typename TI, typename T>
__global__ void tip_rms_kernel(const TI* __restrict__ x, int ld, int C, const float* __restrict__ gamma,
                               const float* __restrict__ beta, float eps, int spatial, int act,
                               const float* __restrict__ rowmask, const float* __restrict__ mask_sum,
                               T* __restrict__ y, int yld) {
  pdl_wait();
  pdl_trigger();
  __shared__ float rms_s[361];
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31, nw = blockDim.x / 32;
  for (int pos = warp; pos < 361; pos += nw) {
    int r = pbl_row(b, pos / 19, pos % 19);
    float ss = 0.0f;
    for (int c = lane; c < C; c += 32) {
      float v = to_f<TI>(x[(size_t)r * ld + c]);
      ss += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) rms_s[pos] = spatial ? ss * rowmask[r] : ss;
  }
  __syncthreads();
  if (spatial) {
    float s = 0.0f;
    for (int pos = threadIdx.x; pos < 361; pos += blockDim.x) s += rms_s[pos];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int i = 0; i < nw; i++) t += red[i];
      float count = mask_sum[b] * (float)C;
      float ms = t / count;
      red[0] = 1.0f / sqrtf(ms + eps);
    }
    __syncthreads();
    float rr = red[0];
    __syncthreads();
    for (int pos = threadIdx.x; pos < 361; pos += blockDim.x) rms_s[pos] = rr;
  } else {
    __syncthreads();
    for (int pos = threadIdx.x; pos < 361; pos += blockDim.x) {
      float ms = rms_s[pos] / (float)C;
      rms_s[pos] = 1.0f / sqrtf(ms + eps);
    }
  }
  __syncthreads();
  for (int pos = warp; pos < 361; pos += nw) {
    int r = pbl_row(b, pos / 19, pos % 19);
    float m = rowmask[r], rr = rms_s[pos];
    for (int c = lane; c < C; c += 32) {
      float v = to_f<TI>(x[(size_t)r * ld + c]) * rr;
      v = v * gamma[c];
      v = v + beta[c];
      y[(size_t)r * yld + c] = from_f<T>(act_apply(v, act) * m);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Policy p2 (1x1 conv p1 -> P, bin2onnx.py :1505) and ownership (1x1 conv v1 -> 1, :1530) per board point, written
// into the output rows: policy[p * 362 + pos], ownership[own_off + pos]. One thread per (board, point).
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void head_spatial_kernel(const T* __restrict__ p1a, int p1ld, int p1c, const float* __restrict__ w2,
                                    int P, const T* __restrict__ v1a, int v1ld, int v1c0, int v1c,
                                    const float* __restrict__ wown, float* __restrict__ out, int row_len, int own_off,
                                    int n) {
  pdl_wait();
  pdl_trigger();
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * 361) return;
  int b = idx / 361, pos = idx - b * 361;
  int r = pbl_row(b, pos / 19, pos % 19);
  float* o = out + (size_t)b * row_len;
  constexpr int VW = 16 / (int)sizeof(T);  // elements per 16-byte vector
  const T* pr = p1a + (size_t)r * p1ld;
  if (P <= 4 && p1ld % VW == 0) {
    // the row's channels as 16-byte vectors, all (up to 4) policy outputs at once; each output still sums its
    // channels in order
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int c = 0;
    for (; c + VW <= p1c; c += VW) {
      const uint4 u = *reinterpret_cast<const uint4*>(pr + c);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < VW; k++) {
        const float a = to_f<T>(e[k]);
#pragma unroll
        for (int p = 0; p < 4; p++)
          if (p < P) acc[p] += a * __ldg(w2 + (size_t)(c + k) * P + p);
      }
    }
    for (; c < p1c; c++) {
      const float a = to_f<T>(pr[c]);
#pragma unroll
      for (int p = 0; p < 4; p++)
        if (p < P) acc[p] += a * __ldg(w2 + (size_t)c * P + p);
    }
#pragma unroll
    for (int p = 0; p < 4; p++)
      if (p < P) o[p * 362 + pos] = acc[p];
  } else {
    for (int p = 0; p < P; p++) {
      float a = 0.0f;
      for (int c = 0; c < p1c; c++) a += to_f<T>(pr[c]) * __ldg(w2 + (size_t)c * P + p);
      o[p * 362 + pos] = a;
    }
  }
  const T* vr = v1a + (size_t)r * v1ld + v1c0;
  float a = 0.0f;
  int c = 0;
  if (v1ld % VW == 0 && v1c0 % VW == 0)
    for (; c + VW <= v1c; c += VW) {
      const uint4 u = *reinterpret_cast<const uint4*>(vr + c);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < VW; k++) a += to_f<T>(e[k]) * __ldg(wown + c + k);
    }
  for (; c < v1c; c++) a += to_f<T>(vr[c]) * __ldg(wown + c);
  o[own_off + pos] = a;
}

// ---------------------------------------------------------------------------------------------------------------
// float32-tier RoPE (in place on the QKV buffer) and SwiGLU, where the GEMM epilogue does not fuse them.
// Q columns [0, qc), K columns [qc, qc + kc); head h's channels are [x0 of each pair..., x1 of each pair...]
// (the projection columns are permuted so, bin2onnx.py :1369-1374). Tables [tables][361][hd/2].
// ---------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void rope_kernel(T* __restrict__ qkv, int ld, int qc, int kc, int hd, const float* __restrict__ cosv,
                            const float* __restrict__ sinv, int table_stride, int group, int rows) {
  pdl_wait();
  pdl_trigger();
  const int half = hd / 2;
  const int pairs_per_row = (qc + kc) / 2;
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)rows * pairs_per_row) return;
  int r = (int)(idx / pairs_per_row), pr = (int)(idx - (size_t)r * pairs_per_row);
  int head = pr / half, j = pr - head * half;
  int rr = r % 400, yy = rr / 20 - 1, xx = rr % 20;
  if (yy < 0 || xx >= 19) return;
  int pos = yy * 19 + xx;
  int qheads = qc / hd;
  int table = head < qheads ? head / group : head - qheads;
  float c = cosv[(size_t)table * table_stride + (size_t)pos * half + j];
  float s = sinv[(size_t)table * table_stride + (size_t)pos * half + j];
  T* base = qkv + (size_t)r * ld + head * hd;
  float x0 = to_f<T>(base[j]), x1 = to_f<T>(base[j + half]);
  float a0 = x0 * c, b1 = x1 * s;
  float c0 = x0 * s, d1 = x1 * c;
  base[j] = from_f<T>(a0 - b1);
  base[j + half] = from_f<T>(c0 + d1);
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ ag, int ld, int F, const float* __restrict__ rowmask, int rows,
                              T* __restrict__ h, int hld) {
  pdl_wait();
  pdl_trigger();
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)rows * F) return;
  int r = (int)(idx / F), j = (int)(idx - (size_t)r * F);
  float a = to_f<T>(ag[(size_t)r * ld + j]);
  float g = to_f<T>(ag[(size_t)r * ld + F + j]);
  float s = a / (expf(-a) + 1.0f);
  h[(size_t)r * hld + j] = from_f<T>(s * g * rowmask[r]);
}

// ---------------------------------------------------------------------------------------------------------------
// SIMT attention (bin2onnx.py transformer_attention_block :1359-1423 after the projections): per board and head,
// softmax(q k^T * scale + bias) v over the board's 361 points, bias = mask * 3e4 - 3e4 (:1313-1323), GQA kv head =
// h / (heads / kv_heads). One thread per query with an online softmax; K and V of the board staged in shared
// memory. grid (ceil(400 / 128), heads, n), block 128.
// ---------------------------------------------------------------------------------------------------------------
template <typename T, int HD>
__global__ void __launch_bounds__(128) attention_simt_kernel(const T* __restrict__ qkv, int ld, int qc, int kc,
                                                             int heads, int kv_heads, float scale,
                                                             const float* __restrict__ rowmask, T* __restrict__ out,
                                                             int out_ld) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t sm[];
  T* Ks = reinterpret_cast<T*>(sm);
  T* Vs = Ks + 361 * HD;
  float* kb = reinterpret_cast<float*>(Vs + 361 * HD);
  const int b = blockIdx.z, h = blockIdx.y;
  const int kvh = h / (heads / kv_heads);
  for (int i = threadIdx.x; i < 361 * HD; i += blockDim.x) {
    int pos = i / HD, d = i - pos * HD;
    int r = pbl_row(b, pos / 19, pos % 19);
    Ks[i] = qkv[(size_t)r * ld + qc + kvh * HD + d];
    Vs[i] = qkv[(size_t)r * ld + qc + kc + kvh * HD + d];
  }
  for (int pos = threadIdx.x; pos < 361; pos += blockDim.x) {
    float m = rowmask[pbl_row(b, pos / 19, pos % 19)];
    kb[pos] = m * 3e4f - 3e4f;
  }
  __syncthreads();
  const int rr = blockIdx.x * 128 + threadIdx.x;
  if (rr >= 400) return;
  const int r = b * 400 + rr;
  const int yy = rr / 20 - 1, xx = rr % 20;
  T* o = out + (size_t)r * out_ld + h * HD;
  if (yy < 0 || xx >= 19) {
    for (int d = 0; d < HD; d++) o[d] = from_f<T>(0.0f);
    return;
  }
  float q[HD], acc[HD];
  for (int d = 0; d < HD; d++) {
    q[d] = to_f<T>(qkv[(size_t)r * ld + h * HD + d]);
    acc[d] = 0.0f;
  }
  float mx = -INFINITY, l = 0.0f;
  for (int k = 0; k < 361; k++) {
    float s = 0.0f;
#pragma unroll
    for (int d = 0; d < HD; d++) s += q[d] * to_f<T>(Ks[k * HD + d]);
    s = s * scale + kb[k];
    float mn = fmaxf(mx, s);
    float corr = expf(mx - mn);
    float pw = expf(s - mn);
    l = l * corr + pw;
#pragma unroll
    for (int d = 0; d < HD; d++) acc[d] = acc[d] * corr + pw * to_f<T>(Vs[k * HD + d]);
    mx = mn;
  }
  float inv = 1.0f / l;
  for (int d = 0; d < HD; d++) o[d] = from_f<T>(acc[d] * inv);
}

}  // namespace kc
