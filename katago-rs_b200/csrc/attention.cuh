// Tensor-core attention of the transformer blocks (tools/bin2onnx/bin2onnx.py transformer_attention_block
// :1359-1423 after the projections): per board and head, softmax(q k^T * scale + bias) v over the board's points,
// bias = 0 on board and -3e4 off board (:1313-1323). Head dim 64 (q and v), GQA kv head = h / (heads / kv_heads).
//
// One CTA per (head, board). A board's 400 PBL rows (361 points plus zero halo rows) are the keys, so every key of
// the board is in one tile and the softmax is a single exact pass, no online rescaling. K [416 x 64] and
// V [448 x 64] are loaded once (128B-swizzled TMA boxes) and the board's queries run as three 128-row tiles from
// the board's row 20 (rows 0..19 are the halo row above the board, no query): rows 20..403 cover every point
// (rows 400..403 belong to the next board and are neither kept nor written).
// Sixteen warps, four per TMEM lane quarter, each one query row per thread and a quarter of the keys:
//   S = Q K^T (M = 128, N = 2 x 208, K = 64) into TMEM [0, 416);
//   row max over S (exchanged in shared memory), p = 2^((s - max) * scale * log2 e) for on-board keys (0 for
//   off-board, halo and out-of-board keys: an additive -inf key bias), P (bf16 / f16) into shared memory in the
//   K-major 128B-swizzled layout of an MMA A operand, in five 64-key buffers: the first pass keys 0..191 (buffers
//   0..2); the second pass first keys 192..255 (buffer 3) and 384..447 (buffer 4; keys 416..447 zero), which the
//   first pass's MMAs do not read, then, once they have read buffers 0 and 1, keys 256..383 there;
//   O = P V (M = 128, N = 64, K = 448, V as an MN-major B operand) into TMEM [416, 480) after each pass, the
//   K-blocks in key order, then O divided by the row sum.
// There are no producer or MMA warps: one elected thread of warp 0 issues the TMA loads and the MMAs at the points
// where its warp waits for all warps anyway (after each pass), so the CTA is 512 threads with 128 registers
// each. The next tile's S is computed while the warps write the current tile's output.
// Off-board keys get weight exactly 0 here; in the reference their weight exp(-3e4 + ...) underflows to 0 too.
#pragma once

#include "gemm.cuh"

namespace kc {

struct AttnParams {
  int qc = 0, kc = 0;            // column offsets of K (= qc) and V (= qc + kc) in the QKV rows
  int heads = 1, kv_heads = 1;
  float scale = 0.125f;          // 1 / sqrt(head_dim)
  const float* rowmask = nullptr;
  void* out = nullptr;           // [rows][out_ld], head h at columns h * 64
  int out_ld = 0;
  int* err = nullptr;
};

struct AttnCfg {
  static constexpr int KEYS = 416;         // S columns: the board's 400 rows padded to 2 x 208
  static constexpr int PKEYS = 448;        // P / V keys: 7 x 64
  static constexpr int QTILES = 3;         // 128-row query tiles covering the board's rows 20..399
  static constexpr int QROW0 = 20;         // first query row: the board's first point
  static constexpr int K_OFF = 0;
  static constexpr int K_BYTES = KEYS * 128;           // 53248
  static constexpr int V_OFF = K_OFF + K_BYTES;
  static constexpr int V_BYTES = PKEYS * 128;          // 57344
  static constexpr int Q_OFF = V_OFF + V_BYTES;        // 110592
  static constexpr int Q_BYTES = 128 * 128;            // 16384
  static constexpr int P_OFF = Q_OFF + Q_BYTES;        // 126976: P buffers 0..4, tiles of 128 queries x 64 keys
  static constexpr int P_BYTES = 5 * 128 * 128;        // 81920
  static constexpr int BIAS_OFF = P_OFF + P_BYTES;     // 208896: key bias, 0 or -inf
  static constexpr int WARPS = 16;                     // 4 per TMEM lane quarter, one per key quarter
  static constexpr int RED_OFF = BIAS_OFF + KEYS * 4;  // row max and row sum of each key quarter: [2][4][128]
  static constexpr int BAR_OFF = RED_OFF + 2 * 4 * 128 * 4;
  static constexpr int SMEM = 1024 + BAR_OFF + 128;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t O_COL = 416;
};

// Shared-memory descriptor of an MN-major operand stored as 128-byte rows along K with the 128B swizzle (a TMA load
// of [K rows][64 elements]): 8-row K groups 1024 B apart (stride byte offset), one 64-element MN atom.
__device__ __forceinline__ uint64_t make_sw128_mn_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (one MN atom: unused)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset between 8-row K groups
  d |= (uint64_t)1 << 46;                 // sm_100 descriptor version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One 32-key (or 16-key) group of a query row: p = 2^(s * sl - msl) for the keys, their sum added to `sum`, written
// as bf16 / f16 into row r of the half-P buffer `P` (keys kp.. relative to the half: tile kp / 64, 16-byte chunk).
// Row max of N keys of S (N a multiple of 4) with the keys' additive bias (0 or -inf, 16-byte aligned).
template <int N>
__device__ __forceinline__ float attn_max(const uint32_t* x, const float* bias, float m) {
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    const float4 b = *reinterpret_cast<const float4*>(bias + i);
    m = fmaxf(m, __uint_as_float(x[i]) + b.x);
    m = fmaxf(m, __uint_as_float(x[i + 1]) + b.y);
    m = fmaxf(m, __uint_as_float(x[i + 2]) + b.z);
    m = fmaxf(m, __uint_as_float(x[i + 3]) + b.w);
  }
  return m;
}

// One group of N keys (a multiple of 8) of a query row: p = 2^((s + bias) * sl - msl), their sum added to `sum`,
// written as bf16 / f16 into row r of the half-P buffer `P` (keys kp.. relative to the half: tile kp / 64, 16-byte
// chunk (kp % 64) / 8; a group may cross a tile boundary).
template <typename T, int N>
__device__ __forceinline__ void attn_exp_group(const uint32_t* x, const float* bias, float sl, float msl, float& sum,
                                               uint8_t* P, int r, int kp) {
#pragma unroll
  for (int j = 0; j < N / 8; j++) {
    const float4 b0 = *reinterpret_cast<const float4*>(bias + j * 8);
    const float4 b1 = *reinterpret_cast<const float4*>(bias + j * 8 + 4);
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float pv = ex2_approx(fmaf(__uint_as_float(x[j * 8 + k]) + bb[k], sl, -msl));
      sum += pv;
      e[k] = from_f<T>(pv);
    }
    const int key = kp + j * 8;
    *reinterpret_cast<uint4*>(P + (key >> 6) * 16384 + r * 128 + ((((key >> 3) & 7) ^ (r & 7)) * 16)) = u;
  }
}

template <typename T>
__global__ void __launch_bounds__(AttnCfg::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  using C = AttnCfg;
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_S = make_idesc_f16(fmt, 128, 208);
  constexpr uint32_t IDESC_O = make_idesc_f16(fmt, 128, 64) | (1u << 16);  // B (V) MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bar + 0;
  uint64_t* q_full = bar + 1;
  uint64_t* s_full = bar + 2;   // S of the current tile in TMEM (MMA commit)
  uint64_t* pa_full = bar + 3;  // first half of P written (one arrival per warp)
  uint64_t* pa_free = bar + 4;  // the MMAs have read the first half (MMA commit)
  uint64_t* pb_full = bar + 5;  // second half of P written (one arrival per warp)
  uint64_t* o_full = bar + 6;   // O in TMEM (MMA commit)
  uint64_t* o_empty = bar + 7;  // O read (one arrival per warp)
  uint64_t* drain = bar + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 9);
  float* kbias = reinterpret_cast<float*>(smem + C::BIAS_OFF);
  float* red = reinterpret_cast<float*>(smem + C::RED_OFF);  // [max | sum][key quarter][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (p.heads / p.kv_heads);
  const int row0 = b * 400;
  const bool ctl = threadIdx.x == 0;  // issues the TMA loads and the MMAs

  if (ctl) {
    for (int i = 0; i < 9; i++) mbar_init(&bar[i], (i == 3 || i == 5 || i == 7) ? C::WARPS : 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();
  // key bias: 0 for the board's on-board points, -inf for halo rows and keys past the board's 400 rows
  for (int k = threadIdx.x; k < C::KEYS; k += blockDim.x)
    kbias[k] = k < 400 && p.rowmask[row0 + k] != 0.0f ? 0.0f : -INFINITY;

  const uint32_t sq = smem_u32(smem + C::Q_OFF), sk = smem_u32(smem + C::K_OFF);
  const uint32_t sp = smem_u32(smem + C::P_OFF), sv = smem_u32(smem + C::V_OFF);
  bool cok = true;  // the control thread's waits all succeeded
  auto issue_s = [&](int t) {  // S = Q_t K^T once Q_t has landed
    cok = cok && mbar_wait(q_full, t & 1, p.err, DEV_TIMEOUT_MMA);
    if (!cok) return;
    tc_fence_after();
#pragma unroll
    for (int nh = 0; nh < 2; nh++)
#pragma unroll
      for (int k = 0; k < 4; k++)
        umma_f16(tmem + nh * 208, make_sw128_desc(sq + k * 32), make_sw128_desc(sk + nh * 208 * 128 + k * 32),
                 IDESC_S, k != 0);
    umma_commit(s_full);
  };
  if (ctl) {
    mbar_expect_tx(kv_full, C::K_BYTES + C::V_BYTES);
    tma_load_2d(smem + C::K_OFF, &tmK, kv_full, p.qc + kvh * 64, row0);
    tma_load_2d(smem + C::K_OFF + 208 * 128, &tmK, kv_full, p.qc + kvh * 64, row0 + 208);
    tma_load_2d(smem + C::V_OFF, &tmV, kv_full, p.qc + p.kc + kvh * 64, row0);
    tma_load_2d(smem + C::V_OFF + 224 * 128, &tmV, kv_full, p.qc + p.kc + kvh * 64, row0 + 224);
    mbar_expect_tx(q_full, C::Q_BYTES);
    tma_load_2d(smem + C::Q_OFF, &tmQ, q_full, h * 64, row0 + C::QROW0);
    cok = mbar_wait(kv_full, 0, p.err, DEV_TIMEOUT_MMA);
    issue_s(0);
  }
  __syncthreads();  // the key bias is written

  const int q = warp & 3;    // TMEM lane quarter
  const int kq = warp >> 2;  // key quarter
  const int r = q * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
  const float sl = p.scale * 1.4426950408889634f;  // exp(x) = 2^(x log2 e)
  uint8_t* P = smem + C::P_OFF;
  float* rmax = red;            // [4][128]
  float* rsum = red + 4 * 128;  // [4][128]
  const uint32_t bar_id = 1 + q;  // named barrier of the lane quarter's four warps
  bool ok = true;
  for (int t = 0; t < C::QTILES; t++) {
    const uint32_t ph = t & 1;
    const int qrow = C::QROW0 + t * 128 + r;  // query row within the board
    // the quarter's warps whose 32 rows are all past the board's 400 rows only keep the barrier protocol
    const bool live = C::QROW0 + t * 128 + q * 32 < 400;
    const float mq = qrow < 400 ? __ldg(p.rowmask + row0 + qrow) : 0.0f;  // for the output, loaded early
    ok = ok && mbar_wait(s_full, ph, p.err, DEV_TIMEOUT_EPILOGUE);
    __syncwarp();
    tc_fence_after();
    float m = -INFINITY;
    if (ok && live) {
      // row max over this warp's 104 keys
      const int k0 = kq * 104;
      uint32_t x[32], y[32];
      tmem_ld32(trow + k0, x);
      tmem_ld32(trow + k0 + 32, y);
      tmem_wait_ld();
      m = attn_max<32>(x, kbias + k0, m);
      m = attn_max<32>(y, kbias + k0 + 32, m);
      uint32_t z[8];
      tmem_ld32(trow + k0 + 64, x);
      tmem_ld8(trow + k0 + 96, z);
      tmem_wait_ld();
      m = attn_max<32>(x, kbias + k0 + 64, m);
      m = attn_max<8>(z, kbias + k0 + 96, m);
    }
    rmax[kq * 128 + r] = m;
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
    m = fmaxf(fmaxf(rmax[r], rmax[128 + r]), fmaxf(rmax[256 + r], rmax[384 + r]));
    if (m == -INFINITY) m = 0.0f;  // no on-board key: every p is 0
    const float msl = m * sl;
    float sum = 0.0f;
    // first pass, keys 0..191: this warp's 48 keys -> P buffers 0..2
    if (ok && live) {
      uint32_t x[32], y[16];
      tmem_ld32(trow + kq * 48, x);
      tmem_ld16(trow + kq * 48 + 32, y);
      tmem_wait_ld();
      attn_exp_group<T, 32>(x, kbias + kq * 48, sl, msl, sum, P, r, kq * 48);
      attn_exp_group<T, 16>(y, kbias + kq * 48 + 32, sl, msl, sum, P, r, kq * 48 + 32);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(pa_full);
    if (ctl) {
      // O = P[keys 0..191] V once every warp wrote its part and the previous tile's O was read; then the next
      // query tile into the Q buffer (S_t has completed: its commit was observed above)
      cok = cok && mbar_wait(pa_full, ph, p.err, DEV_TIMEOUT_MMA) &&
            (t == 0 || mbar_wait(o_empty, (t - 1) & 1, p.err, DEV_TIMEOUT_MMA));
      if (cok) {
        tc_fence_after();
        for (int kb = 0; kb < 3; kb++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + C::O_COL, make_sw128_desc(sp + kb * 16384 + k * 32),
                     make_sw128_mn_desc(sv + (kb * 64 + k * 16) * 128), IDESC_O, (kb | k) != 0);
        umma_commit(pa_free);
        if (t + 1 < C::QTILES) {
          mbar_expect_tx(q_full, C::Q_BYTES);
          tma_load_2d(smem + C::Q_OFF, &tmQ, q_full, h * 64, row0 + C::QROW0 + (t + 1) * 128);
        }
      }
    }
    // second pass, into the buffers the first pass's MMAs do not read: this warp's 16 of keys 192..255 (buffer 3)
    // and 8 of keys 384..415 (buffer 4), and 8 of buffer 4's zero keys 416..447 (V rows there are finite: the next
    // board or TMA's zero fill)
    uint8_t* P4 = P + 4 * 16384;
    if (ok && live) {
      uint32_t x[16], z[8];
      tmem_ld16(trow + 192 + kq * 16, x);
      tmem_ld8(trow + 384 + kq * 8, z);
      tmem_wait_ld();
      attn_exp_group<T, 16>(x, kbias + 192 + kq * 16, sl, msl, sum, P, r, 192 + kq * 16);
      attn_exp_group<T, 8>(z, kbias + 384 + kq * 8, sl, msl, sum, P4, r, kq * 8);
      *reinterpret_cast<uint4*>(P4 + r * 128 + (((4 + kq) ^ (r & 7)) * 16)) = make_uint4(0, 0, 0, 0);
    }
    // then, once the first pass's MMAs have read buffers 0 and 1: this warp's 32 of keys 256..383 there
    ok = ok && mbar_wait(pa_free, ph, p.err, DEV_TIMEOUT_EPILOGUE);
    __syncwarp();
    tc_fence_after();
    if (ok && live) {
      uint32_t x[32];
      tmem_ld32(trow + 256 + kq * 32, x);
      tmem_wait_ld();
      attn_exp_group<T, 32>(x, kbias + 256 + kq * 32, sl, msl, sum, P, r, kq * 32);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(pb_full);
    if (ctl) {
      // O += P[keys 192..447] V, K-blocks 3..6 from buffers 3, 0, 1, 4; then the next tile's S (every warp has
      // read S_t)
      cok = cok && mbar_wait(pb_full, ph, p.err, DEV_TIMEOUT_MMA);
      if (cok) {
        tc_fence_after();
        for (int kb = 3; kb < 7; kb++) {
          const int buf = kb == 3 ? 3 : kb == 6 ? 4 : kb - 4;
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + C::O_COL, make_sw128_desc(sp + buf * 16384 + k * 32),
                     make_sw128_mn_desc(sv + (kb * 64 + k * 16) * 128), IDESC_O, 1);
        }
        umma_commit(o_full);
        if (t + 1 < C::QTILES) issue_s(t + 1);
      }
    }
    __syncwarp();
    rsum[kq * 128 + r] = sum;
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
    const float total = (rsum[r] + rsum[128 + r]) + (rsum[256 + r] + rsum[384 + r]);
    // output: this warp's 16 of the head's 64 dimensions
    ok = ok && mbar_wait(o_full, ph, p.err, DEV_TIMEOUT_EPILOGUE);
    __syncwarp();
    tc_fence_after();
    if (ok && live) {
      uint32_t o[16];
      tmem_ld16(trow + C::O_COL + kq * 16, o);
      tmem_wait_ld();
      if (qrow < 400) {
        const float inv = total > 0.0f ? mq / total : 0.0f;
        T* dst = reinterpret_cast<T*>(p.out) + (size_t)(row0 + qrow) * p.out_ld + h * 64 + kq * 16;
#pragma unroll
        for (int j = 0; j < 2; j++) {
          uint4 u;
          T* e = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int tt = 0; tt < 8; tt++) e[tt] = from_f<T>(__uint_as_float(o[j * 8 + tt]) * inv);
          *reinterpret_cast<uint4*>(dst + j * 8) = u;
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(o_empty);
  }
  if (ctl && !cok) {
    umma_commit(drain);  // the MMAs issued so far complete before TMEM is released
    mbar_wait(drain, 0, p.err, DEV_TIMEOUT_DRAIN);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace kc
