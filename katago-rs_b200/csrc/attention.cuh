// Tensor-core attention of the transformer blocks (tools/bin2onnx/bin2onnx.py transformer_attention_block
// :1359-1423 after the projections): per board and head, softmax(q k^T * scale + bias) v over the board's points,
// bias = 0 on board and -3e4 off board (:1313-1323). Head dim 64 (q and v), GQA kv head = h / (heads / kv_heads).
//
// One CTA per (head, board). A board's 400 PBL rows (361 points plus zero halo rows) are the keys, so every key of
// the board is in one tile and the softmax is a single exact pass, no online rescaling. K [416 x 64] and
// V [448 x 64] are loaded once (128B-swizzled TMA boxes) and the board's queries run as four 128-row tiles
// through a pipeline:
//   MMA warp:     S = Q K^T (M = 128, N = 2 x 208, K = 64) into TMEM [0, 416); later O = P V (M = 128, N = 64,
//                 K = 448, V as an MN-major B operand) into TMEM [416, 480), in two halves of P;
//   TMA warp:     the next query tile as soon as the MMAs have read the current one;
//   8 softmax warps (two per TMEM lane quarter, one query row per thread, each half of the keys): row max over
//                 S (exchanged between the pair in shared memory), p = 2^((s - max) * scale * log2 e) for on-board
//                 keys (0 for off-board, halo and out-of-board keys: an additive -inf key bias), P (bf16 / f16) into
//                 shared memory in the K-major 128B-swizzled layout of an MMA A operand, keys 0..255 then, once the
//                 MMAs have read those, keys 256..447 (keys 416..447 zero); then O divided by the row sum.
// The MMA warp computes the next tile's S while the softmax warps write the current tile's output.
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
  static constexpr int QTILES = 4;         // 128-row query tiles covering the board's 400 rows
  static constexpr int K_OFF = 0;
  static constexpr int K_BYTES = KEYS * 128;           // 53248
  static constexpr int V_OFF = K_OFF + K_BYTES;
  static constexpr int V_BYTES = PKEYS * 128;          // 57344
  static constexpr int Q_OFF = V_OFF + V_BYTES;        // 110592
  static constexpr int Q_BYTES = 128 * 128;            // 16384
  static constexpr int P_OFF = Q_OFF + Q_BYTES;        // 126976: half of P, 4 tiles of 128 queries x 64 keys
  static constexpr int P_BYTES = 4 * 128 * 128;        // 65536
  static constexpr int BIAS_OFF = P_OFF + P_BYTES;     // 192512: key bias, 0 or -inf
  static constexpr int RED_OFF = BIAS_OFF + KEYS * 4;  // row max and row sum of each warp of a pair: [2][2][128]
  static constexpr int BAR_OFF = RED_OFF + 2 * 2 * 128 * 4;
  static constexpr int SMEM = 1024 + BAR_OFF + 128;
  static constexpr int SM_WARPS = 8;                   // softmax warps
  static constexpr int THREADS = 64 + 32 * SM_WARPS;  // TMA warp, MMA warp, softmax warps
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
template <typename T, int N>
__device__ __forceinline__ void attn_exp_group(const uint32_t* x, const float* bias, float sl, float msl, float& sum,
                                               uint8_t* P, int r, int kp) {
  float pv[N];
#pragma unroll
  for (int i = 0; i < N; i++) {
    pv[i] = ex2_approx(fmaf(__uint_as_float(x[i]) + bias[i], sl, -msl));
    sum += pv[i];
  }
#pragma unroll
  for (int j = 0; j < N / 8; j++) {
    const int key = kp + j * 8;  // a group may cross a 64-key tile boundary
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int t = 0; t < 8; t++) e[t] = from_f<T>(pv[j * 8 + t]);
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
  uint64_t* q_empty = bar + 2;
  uint64_t* s_full = bar + 3;
  uint64_t* pa_full = bar + 4;
  uint64_t* pa_free = bar + 5;
  uint64_t* pb_full = bar + 6;
  uint64_t* o_full = bar + 7;
  uint64_t* o_empty = bar + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 9);
  float* kbias = reinterpret_cast<float*>(smem + C::BIAS_OFF);
  float* red = reinterpret_cast<float*>(smem + C::RED_OFF);  // [max | sum][pair member][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (p.heads / p.kv_heads);
  const int row0 = b * 400;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 9; i++) mbar_init(&bar[i], (i == 4 || i == 6 || i == 8) ? C::SM_WARPS : 1);
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
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: K and V once, then the query tiles ----
      mbar_expect_tx(kv_full, C::K_BYTES + C::V_BYTES);
      tma_load_2d(smem + C::K_OFF, &tmK, kv_full, p.qc + kvh * 64, row0);
      tma_load_2d(smem + C::K_OFF + 208 * 128, &tmK, kv_full, p.qc + kvh * 64, row0 + 208);
      tma_load_2d(smem + C::V_OFF, &tmV, kv_full, p.qc + p.kc + kvh * 64, row0);
      tma_load_2d(smem + C::V_OFF + 224 * 128, &tmV, kv_full, p.qc + p.kc + kvh * 64, row0 + 224);
      for (int t = 0; t < C::QTILES; t++) {
        if (t > 0 && !mbar_wait(q_empty, (t - 1) & 1, p.err, DEV_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(q_full, C::Q_BYTES);
        tma_load_2d(smem + C::Q_OFF, &tmQ, q_full, h * 64, row0 + t * 128);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      const uint32_t sq = smem_u32(smem + C::Q_OFF), sk = smem_u32(smem + C::K_OFF);
      const uint32_t sp = smem_u32(smem + C::P_OFF), sv = smem_u32(smem + C::V_OFF);
      bool ok = mbar_wait(kv_full, 0, p.err, DEV_TIMEOUT_MMA);
      for (int t = 0; t < C::QTILES && ok; t++) {
        const uint32_t ph = t & 1;
        ok = mbar_wait(q_full, ph, p.err, DEV_TIMEOUT_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int nh = 0; nh < 2; nh++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + nh * 208, make_sw128_desc(sq + k * 32), make_sw128_desc(sk + nh * 208 * 128 + k * 32),
                     IDESC_S, k != 0);
        umma_commit(q_empty);
        umma_commit(s_full);
        // O = P[keys 0..255] V, once the previous tile's O has been read
        ok = mbar_wait(pa_full, ph, p.err, DEV_TIMEOUT_MMA) &&
             (t == 0 || mbar_wait(o_empty, (t - 1) & 1, p.err, DEV_TIMEOUT_MMA));
        if (!ok) break;
        tc_fence_after();
        for (int kb = 0; kb < 4; kb++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + C::O_COL, make_sw128_desc(sp + kb * 16384 + k * 32),
                     make_sw128_mn_desc(sv + (kb * 64 + k * 16) * 128), IDESC_O, (kb | k) != 0);
        umma_commit(pa_free);
        // O += P[keys 256..447] V (the same buffer, refilled)
        ok = mbar_wait(pb_full, ph, p.err, DEV_TIMEOUT_MMA);
        if (!ok) break;
        tc_fence_after();
        for (int kb = 4; kb < 7; kb++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + C::O_COL, make_sw128_desc(sp + (kb - 4) * 16384 + k * 32),
                     make_sw128_mn_desc(sv + (kb * 64 + k * 16) * 128), IDESC_O, 1);
        umma_commit(o_full);
      }
      if (!ok) {
        umma_commit(o_full);  // drains the MMAs issued so far
        mbar_wait(o_full, 0, p.err, DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  } else {
    // ---- softmax / output warps: TMEM lane quarter q, query row r = q * 32 + lane, key half `hs` ----
    const int q = warp & 3;
    const int hs = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const float sl = p.scale * 1.4426950408889634f;  // exp(x) = 2^(x log2 e)
    uint8_t* P = smem + C::P_OFF;
    float* rmax = red;           // [2][128]
    float* rsum = red + 2 * 128;  // [2][128]
    bool ok = true;
    for (int t = 0; t < C::QTILES; t++) {
      const uint32_t ph = t & 1;
      const int qrow = t * 128 + r;  // query row within the board
      // a pair whose 32 rows are all past the board's 400 rows only keeps the barrier protocol
      const bool live = t * 128 + q * 32 < 400;
      ok = ok && mbar_wait(s_full, ph, p.err, DEV_TIMEOUT_EPILOGUE);
      __syncwarp();
      tc_fence_after();
      float m = -INFINITY;
      if (ok && live) {
        // row max over this warp's 208 keys
        const int k0 = hs * 208;
#pragma unroll 1
        for (int c = 0; c < 192; c += 32) {
          uint32_t x[32];
          tmem_ld32(trow + k0 + c, x);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) m = fmaxf(m, __uint_as_float(x[i]) + kbias[k0 + c + i]);
        }
        uint32_t x[16];
        tmem_ld16(trow + k0 + 192, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; i++) m = fmaxf(m, __uint_as_float(x[i]) + kbias[k0 + 192 + i]);
      }
      rmax[hs * 128 + r] = m;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
      m = fmaxf(rmax[r], rmax[128 + r]);
      if (m == -INFINITY) m = 0.0f;  // no on-board key: every p is 0
      const float msl = m * sl;
      float sum = 0.0f;
      // keys 0..255: this warp's 128 keys -> P tiles 2 hs, 2 hs + 1
      if (ok && live) {
#pragma unroll 1
        for (int c = hs * 128; c < hs * 128 + 128; c += 32) {
          uint32_t x[32];
          tmem_ld32(trow + c, x);
          tmem_wait_ld();
          attn_exp_group<T, 32>(x, kbias + c, sl, msl, sum, P, r, c);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pa_full);
      // keys 256..447, once the MMAs have read the first half: this warp's 80 keys (and hs 1: the zero keys)
      ok = ok && mbar_wait(pa_free, ph, p.err, DEV_TIMEOUT_EPILOGUE);
      __syncwarp();
      tc_fence_after();
      if (ok && live) {
        const int c0 = 256 + hs * 80;
        uint32_t x[32];
        tmem_ld32(trow + c0, x);
        tmem_wait_ld();
        attn_exp_group<T, 32>(x, kbias + c0, sl, msl, sum, P, r, c0 - 256);
        tmem_ld32(trow + c0 + 32, x);
        tmem_wait_ld();
        attn_exp_group<T, 32>(x, kbias + c0 + 32, sl, msl, sum, P, r, c0 + 32 - 256);
        uint32_t y[16];
        tmem_ld16(trow + c0 + 64, y);
        tmem_wait_ld();
        attn_exp_group<T, 16>(y, kbias + c0 + 64, sl, msl, sum, P, r, c0 + 64 - 256);
        if (hs == 1) {
          // keys 416..447: P zero (V rows there are finite: the next board or TMA's zero fill)
          uint8_t* tile = P + 2 * 16384 + r * 128;
#pragma unroll
          for (int j = 4; j < 8; j++) *reinterpret_cast<uint4*>(tile + ((j ^ (r & 7)) * 16)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pb_full);
      rsum[hs * 128 + r] = sum;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
      const float total = rsum[r] + rsum[128 + r];
      // output: this warp's 32 of the head's 64 dimensions
      ok = ok && mbar_wait(o_full, ph, p.err, DEV_TIMEOUT_EPILOGUE);
      __syncwarp();
      tc_fence_after();
      if (ok && live) {
        uint32_t o[32];
        tmem_ld32(trow + C::O_COL + hs * 32, o);
        tmem_wait_ld();
        if (qrow < 400) {
          const float mq = p.rowmask[row0 + qrow];
          const float inv = total > 0.0f ? mq / total : 0.0f;
          T* dst = reinterpret_cast<T*>(p.out) + (size_t)(row0 + qrow) * p.out_ld + h * 64 + hs * 32;
#pragma unroll
          for (int j = 0; j < 4; j++) {
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace kc
