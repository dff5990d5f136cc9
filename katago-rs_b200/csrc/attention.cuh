// Tensor-core attention of the transformer blocks (tools/bin2onnx/bin2onnx.py transformer_attention_block
// :1359-1423 after the projections): per board and head, softmax(q k^T * scale + bias) v over the board's points,
// bias = 0 on board and -3e4 off board (:1313-1323). Head dim 64 (q and v), GQA kv head = h / (heads / kv_heads).
//
// One CTA per (128-query tile, head, board). A board's 400 PBL rows (361 points plus zero halo rows) are the keys,
// so every key of the board is in one tile and the softmax is a single exact pass, no online rescaling:
//   1. TMA: Q tile [128 x 64], K [416 x 64] (two 208-row boxes), V [448 x 64] (two 224-row boxes), 128B swizzle.
//   2. tcgen05.mma: S = Q K^T, M = 128, N = 2 x 208, K = 64, into TMEM columns [0, 416).
//   3. Four warps (one TMEM lane quarter each, one query row per thread) read S twice (row max, then
//      p = exp((s - max) * scale) for on-board keys, 0 for off-board, halo and out-of-board keys), keep the row sum in
//      float32 and write P (bf16 / f16) into shared memory in the K-major 128B-swizzled layout of an MMA A operand
//      (7 tiles of 128 queries x 64 keys, keys 416..447 zero).
//   4. tcgen05.mma: O = P V, M = 128, N = 64, K = 448, with V as an MN-major B operand, into TMEM [416, 480).
//   5. The same warps read O, divide by the row sum and store the heads' output rows.
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
  static constexpr int V_OFF = 0;
  static constexpr int V_BYTES = PKEYS * 128;          // 57344
  static constexpr int Q_OFF = V_OFF + V_BYTES;
  static constexpr int Q_BYTES = 128 * 128;            // 16384
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int K_BYTES = KEYS * 128;           // 53248
  static constexpr int P_OFF = Q_OFF;                  // P reuses Q and K once S is computed
  static constexpr int P_BYTES = 7 * 128 * 128;        // 114688
  static constexpr int BAR_OFF = P_OFF + P_BYTES;      // 172032
  static constexpr int MASK_OFF = BAR_OFF + 128;
  static constexpr int SMEM = 1024 + MASK_OFF + KEYS * 4;
  static constexpr int THREADS = 192;                  // producer, MMA, 4 softmax warps
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

template <typename T>
__global__ void __launch_bounds__(AttnCfg::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  pdl_wait();
  pdl_trigger();
  using C = AttnCfg;
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_S = make_idesc_f16(fmt, 128, 208);
  constexpr uint32_t IDESC_O = make_idesc_f16(fmt, 128, 64) | (1u << 16);  // B (V) MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* qk_full = bar + 0;
  uint64_t* v_full = bar + 1;
  uint64_t* s_full = bar + 2;
  uint64_t* p_full = bar + 3;
  uint64_t* o_full = bar + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 5);
  float* kmask = reinterpret_cast<float*>(smem + C::MASK_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.heads / p.kv_heads);
  const int row0 = b * 400;

  // key validity: on-board points of this board (halo rows and keys past the board's 400 rows excluded)
  for (int k = threadIdx.x; k < C::KEYS; k += blockDim.x) kmask[k] = k < 400 ? p.rowmask[row0 + k] : 0.0f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; i++) mbar_init(&bar[i], i == 3 ? 128 : 1);
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

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(qk_full, C::Q_BYTES + C::K_BYTES);
      tma_load_2d(smem + C::Q_OFF, &tmQ, qk_full, h * 64, row0 + qt * 128);
      tma_load_2d(smem + C::K_OFF, &tmK, qk_full, p.qc + kvh * 64, row0);
      tma_load_2d(smem + C::K_OFF + 208 * 128, &tmK, qk_full, p.qc + kvh * 64, row0 + 208);
      mbar_expect_tx(v_full, C::V_BYTES);
      tma_load_2d(smem + C::V_OFF, &tmV, v_full, p.qc + p.kc + kvh * 64, row0);
      tma_load_2d(smem + C::V_OFF + 224 * 128, &tmV, v_full, p.qc + p.kc + kvh * 64, row0 + 224);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(qk_full, 0, p.err, DEV_TIMEOUT_MMA);
      if (ok) {
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + C::Q_OFF), sk = smem_u32(smem + C::K_OFF);
#pragma unroll
        for (int nh = 0; nh < 2; nh++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + nh * 208, make_sw128_desc(sq + k * 32), make_sw128_desc(sk + nh * 208 * 128 + k * 32),
                     IDESC_S, k != 0);
        umma_commit(s_full);
        ok = mbar_wait(p_full, 0, p.err, DEV_TIMEOUT_MMA) && mbar_wait(v_full, 0, p.err, DEV_TIMEOUT_MMA);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + C::P_OFF), sv = smem_u32(smem + C::V_OFF);
        for (int kb = 0; kb < 7; kb++)
#pragma unroll
          for (int k = 0; k < 4; k++)
            umma_f16(tmem + C::O_COL, make_sw128_desc(sp + kb * 16384 + k * 32),
                     make_sw128_mn_desc(sv + (kb * 64 + k * 16) * 128), IDESC_O, (kb | k) != 0);
      }
      umma_commit(o_full);  // also drains the MMAs issued so far on the error path
      if (!ok) mbar_wait(o_full, 0, p.err, DEV_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else {
    // ---- softmax / output warps: query row r = TMEM lane ----
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const bool ok = mbar_wait(s_full, 0, p.err, DEV_TIMEOUT_EPILOGUE);
    __syncwarp();
    tc_fence_after();
    float mx = -INFINITY;
    if (ok) {
      static_assert(C::KEYS % 32 == 0, "S is read in 32-column loads");
#pragma unroll 1
      for (int c = 0; c < C::KEYS; c += 32) {
        uint32_t x[32];
        tmem_ld32(trow + c, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (kmask[c + i] != 0.0f) mx = fmaxf(mx, __uint_as_float(x[i]));
      }
    }
    const float sl = p.scale * 1.4426950408889634f;  // exp(x) = exp2(x * log2 e)
    float sum = 0.0f;
    uint8_t* P = smem + C::P_OFF;
#pragma unroll 1
    for (int c = 0; c < C::PKEYS; c += 32) {
      uint32_t x[32];
#pragma unroll
      for (int i = 0; i < 32; i++) x[i] = 0;
      if (ok && c < C::KEYS) {
        tmem_ld32(trow + c, x);
        tmem_wait_ld();
      }
      float pv[32];
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const int k = c + i;
        const bool valid = ok && k < C::KEYS && kmask[k < C::KEYS ? k : 0] != 0.0f;
        pv[i] = valid ? exp2f((__uint_as_float(x[i]) - mx) * sl) : 0.0f;
        sum += pv[i];
      }
      // 4 chunks of 8 keys -> 16-byte swizzled slots of row r in P tile (c / 64)
      uint8_t* tile = P + (c / 64) * 16384 + r * 128;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int chunk = ((c % 64) / 8) + j;
        uint4 u;
        T* e = reinterpret_cast<T*>(&u);
#pragma unroll
        for (int t = 0; t < 8; t++) e[t] = from_f<T>(pv[j * 8 + t]);
        *reinterpret_cast<uint4*>(tile + ((chunk ^ (r & 7)) * 16)) = u;
      }
    }
    // make the generic-proxy P writes visible to the tensor core, then hand P to the MMA warp
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    mbar_arrive(p_full);
    const bool ok2 = mbar_wait(o_full, 0, p.err, DEV_TIMEOUT_EPILOGUE);
    __syncwarp();
    tc_fence_after();
    const int rr = qt * 128 + r;  // row within the board
    const float m = rr < 400 ? p.rowmask[row0 + rr] : 0.0f;
    const float inv = sum > 0.0f ? m / sum : 0.0f;
    T* dst = reinterpret_cast<T*>(p.out) + (size_t)(row0 + (rr < 400 ? rr : 0)) * p.out_ld + h * 64;
#pragma unroll
    for (int half_o = 0; half_o < 2; half_o++) {
      uint32_t o[32];
      tmem_ld32(trow + C::O_COL + half_o * 32, o);
      tmem_wait_ld();
      if (ok && ok2 && rr < 400) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          uint4 u;
          T* e = reinterpret_cast<T*>(&u);
#pragma unroll
          for (int t = 0; t < 8; t++) e[t] = from_f<T>(__uint_as_float(o[j * 8 + t]) * inv);
          *reinterpret_cast<uint4*>(dst + half_o * 32 + j * 8) = u;
        }
      }
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
