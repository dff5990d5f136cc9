// A nested bottleneck block's closing 1x1 convolution chained with the next nested block's opening 1x1 on one CTA
// pair (bin2onnx.py nested_bottleneck_block :1263-1269, two consecutive blocks of the trunk):
//   X  <- X + MA W1^T                      (closing 1x1, 192 -> 384, residual add; raw trunk written back)
//   XA  = act1(bn1(X)) * mask               (the next block's pre batch norm: kept in tensor memory, never stored)
//   M   = XA W2^T * mask, MA = act2(bn2(XA W2^T)) * mask    (opening 1x1, 384 -> 192, raw + act outputs)
// The separate launches write XA (384 channels) to HBM and read it straight back; here each 256-row tile's XA stays
// in the pair's tensor memory as the second GEMM's A operand.
//
// Per tile of 256 rows (128 per CTA), tensor memory (512 columns per CTA):
//   G1: two M = 256, N = 192 MMAs per K step into columns [0, 192) and [192, 384) (the 384 trunk channels).
//   E1: epilogue warp group h (0..2, 128 channels each) drains its columns [128 h, 128 h + 128) chunk by chunk (32
//       columns), adds the residual box, stores the trunk through a staging box, and writes the chunk's 32 XA values
//       as 16 packed 2-byte pairs over columns it has already drained: [128 h + 16 c, 128 h + 16 c + 16).
//   G2: 24 K steps (16 channels each) with A from tensor memory (channel block k at column 128 (k / 8) + 8 (k % 8))
//       into columns [320, 512), free once E1 is done (group 2's upper half and the unused [384, 512)).
//   E2: 64 output columns per epilogue warp group: raw and act outputs through staging boxes.
// The next tile's G1 overwrites the XA columns (dead once G2 is complete) and G2's columns [320, 384), which only
// epilogue group 0 reads: it starts as soon as G2 is complete and group 0 has loaded its E2 columns, so it runs
// beside the rest of E2. G2 itself reuses [384, 512) only after every warp has passed the next tile's E1, and so
// its E2. The epilogue warps wait out one GEMM per tile (G2). The TMA producer runs ahead through the stage ring
// (G1 stages: A + both weight halves; G2 stages: three weight K-blocks).
// The epilogue arithmetic is the CTA-pair kernel's (residual add, raw = v * mask, pair_act), so the outputs equal the
// two separate launches'.
#pragma once

#include "gemm_pair.cuh"

namespace kc {

struct ChainParams {
  int rows;                 // PBL rows of this batch
  const float* rowmask;
  int* err;
  const float* scale1;      // the next block's pre batch norm over the 384 trunk channels, act1
  const float* bias1;
  int act1;
  const float* scale2;      // the first inner batch norm over the opening's 192 outputs, act2
  const float* bias2;
  int act2;
  int trunk_x, raw2_x, act2_x;  // first column of each in its box map's tensor
};

struct ChainCfg {
  static constexpr int N1 = 384, K1 = 192, N2 = 192, K2 = 384;
  static constexpr int KB1 = K1 / 64, KB2 = K2 / 64;  // 64-channel K-blocks of the two GEMMs
  static constexpr int A_BYTES = 128 * 128;           // one K-block of this CTA's 128 rows
  static constexpr int B_BYTES = 96 * 128;            // one K-block of 96 weight rows (half of an N = 192 MMA)
  static constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;  // G1: A + two halves; G2: three weight K-blocks
  static constexpr int G2_KBS = 3;
  static_assert(G2_KBS * B_BYTES <= STAGE_BYTES && KB2 % G2_KBS == 0, "G2 stages");
  static constexpr int STAGES = 3;
  static constexpr int EPI_WARPS = 12, EPI_WARP0 = 4;
  static constexpr int BOX = 32 * 32 * 2;              // 32 x 32 staging / residual box of 2-byte values
  static constexpr int NRES = 2;                       // residual boxes in flight per epilogue warp
  static constexpr int EPI_WARP_BYTES = 2 * BOX + NRES * BOX;  // raw, act, residual ring
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_WARP_BYTES;
  static constexpr int PARAM_FLOATS = 2 * N1 + 2 * N2;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + PARAM_FLOATS * 4 + BAR_BYTES;
  static_assert(SMEM <= 227 * 1024, "chain shared memory");
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t ACC2 = 320;  // G2's accumulator: columns [320, 512)
  static_assert(ACC2 + N2 <= TMEM_COLS && ACC2 >= 2 * 128 + 64, "G2 columns free after E1");
  // the next tile's G1 may start once epilogue group 0 has read its E2 columns [ACC2, ACC2 + 64): G1's columns
  // [0, N1) must meet G2's only there
  static_assert(N1 - ACC2 <= N2 / 3, "G1 / G2 column overlap inside group 0's E2 columns");
  // registers: as the 12-warp pair tiles (warpgroup 0: producer, MMA issuer, two idle warps)
  static constexpr int WG0_REGS = 48, EPI_REGS = 152;
  static_assert(4 * 32 * WG0_REGS + 12 * 32 * EPI_REGS <= 65536, "register split");
};

template <typename T>
__device__ __forceinline__ void chain_act(int a, const float (&v)[32], const float* sc, const float* bi, float m,
                                          float (&o)[32]) {
  switch (a) {
    case 1: pair_act<1>(v, sc, bi, m, o); break;
    case 2: pair_act<2>(v, sc, bi, m, o); break;
    case 3: pair_act<3>(v, sc, bi, m, o); break;
    default: pair_act<0>(v, sc, bi, m, o); break;
  }
}

template <typename T>
__global__ void __launch_bounds__(ChainCfg::THREADS, 1)
    gemm_chain_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW1,
                      const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmTrunk,
                      const __grid_constant__ CUtensorMap tmRaw2, const __grid_constant__ CUtensorMap tmAct2,
                      const __grid_constant__ ChainParams p) {
  using C = ChainCfg;
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC = make_idesc_f16(fmt, 256, 192);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* epi = stages + C::STAGES * C::STAGE_BYTES;
  float* s_sc1 = reinterpret_cast<float*>(epi + C::EPI_BYTES);
  float* s_bi1 = s_sc1 + C::N1;
  float* s_sc2 = s_bi1 + C::N1;
  float* s_bi2 = s_sc2 + C::N2;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_bi2 + C::N2);
  uint64_t* empty = full + C::STAGES;
  uint64_t* t1full = empty + C::STAGES;  // G1 accumulated
  uint64_t* actready = t1full + 1;       // E1 done: XA in tensor memory, G1's columns drained
  uint64_t* t2full = actready + 1;       // G2 accumulated
  uint64_t* e2lo = t2full + 1;           // epilogue group 0 has read its E2 columns [320, 384)
  uint64_t* drain = e2lo + 1;
  uint64_t* rbar = drain + 1;            // [EPI_WARPS][NRES]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + C::NRES * C::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert((2 * C::STAGES + 5 + C::NRES * C::EPI_WARPS) * 8 + 8 <= C::BAR_BYTES, "barrier area");

  for (int i = threadIdx.x; i < C::N1; i += blockDim.x) {
    s_sc1[i] = p.scale1[i];
    s_bi1[i] = p.bias1[i];
  }
  for (int i = threadIdx.x; i < C::N2; i += blockDim.x) {
    s_sc2[i] = p.scale2[i];
    s_bi2[i] = p.bias2[i];
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_tiles = (p.rows + 255) / 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(t1full, 1);
    mbar_init(t2full, 1);
    mbar_init(actready, 2 * C::EPI_WARPS);  // one arrival per epilogue warp of both CTAs
    mbar_init(e2lo, 2 * 4);  // group 0's four warps in both CTAs
    mbar_init(drain, 1);
    for (int i = 0; i < C::NRES * C::EPI_WARPS; i++) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmX);
    prefetch_tensormap(&tmW1);
    prefetch_tensormap(&tmW2);
  }
  if (warp == 0) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp < C::EPI_WARP0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::WG0_REGS));
    if (warp == 0) {
      if (lane == 0) {
        // ---- TMA producer (both CTAs): this CTA's 128 rows of MA and its halves of the weights
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        auto slot_free = [&](uint64_t* bar, uint32_t parity) {
          if (mbar_try_wait(bar, parity)) return true;
          if (!*abort_flag && mbar_wait(bar, parity, p.err, DEV_TIMEOUT_PRODUCER)) return true;
          *abort_flag = 1;
          return false;
        };
        auto next = [&]() {
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        };
        for (int it = pair; it < num_tiles && ok; it += npairs) {
          const int m0 = it * 256 + (int)rank * 128;
          for (int kb = 0; kb < C::KB1 && ok; kb++) {
            if (!(ok = slot_free(&empty[stage], phase ^ 1))) break;
            if (leader) mbar_expect_tx(&full[stage], 2u * C::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            uint8_t* dst = stages + stage * C::STAGE_BYTES;
            tma_load_2d_pair(dst, &tmX, fb, kb * 64, m0);
            tma_load_2d_pair(dst + C::A_BYTES, &tmW1, fb, kb * 64, (int)rank * 96);
            tma_load_2d_pair(dst + C::A_BYTES + C::B_BYTES, &tmW1, fb, kb * 64, 192 + (int)rank * 96);
            next();
          }
          for (int s2 = 0; s2 < C::KB2 / C::G2_KBS && ok; s2++) {
            if (!(ok = slot_free(&empty[stage], phase ^ 1))) break;
            if (leader) mbar_expect_tx(&full[stage], 2u * C::G2_KBS * C::B_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            uint8_t* dst = stages + stage * C::STAGE_BYTES;
            for (int j = 0; j < C::G2_KBS; j++)
              tma_load_2d_pair(dst + j * C::B_BYTES, &tmW2, fb, (s2 * C::G2_KBS + j) * 64, (int)rank * 96);
            next();
          }
        }
        if (!ok) {
          unsigned long long t0 = globaltimer();
          while (globaltimer() - t0 < 2000000ull) {
          }
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      if (lane == 0 && leader) {
        // ---- MMA issuer (leader CTA only)
        const uint32_t peer = 1;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        auto data_ready = [&](uint64_t* bar, uint32_t parity) {
          if (mbar_try_wait(bar, parity)) return true;
          return !*abort_flag && mbar_wait(bar, parity, p.err, DEV_TIMEOUT_MMA);
        };
        auto commit_both = [&](uint64_t* bar) {
          const uint32_t b = smem_u32(bar);
          umma_commit_pair(b);
          umma_commit_pair(mapa_shared(b, peer));
        };
        auto next = [&]() {
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        };
        int lt = 0;
        for (int it = pair; it < num_tiles && ok; it += npairs, lt++) {
          const uint32_t ph = lt & 1;
          // G1 overwrites the previous tile's XA columns (G2 complete) and its G2 columns [320, 384) (group 0's E2
          // loads done)
          if (!(ok = data_ready(t2full, ph ^ 1) && data_ready(e2lo, ph ^ 1))) break;
          tc_fence_after();
          for (int kb = 0; kb < C::KB1; kb++) {
            if (!(ok = data_ready(&full[stage], phase))) break;
            tc_fence_after();
            const uint32_t sa = smem_u32(stages + stage * C::STAGE_BYTES);
            const uint32_t sb0 = sa + C::A_BYTES, sb1 = sb0 + C::B_BYTES;
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const uint64_t ad = make_sw128_desc(sa + k * 32);
              umma_f16_pair(tmem_base, ad, make_sw128_desc(sb0 + k * 32), IDESC, (kb | k) != 0);
              umma_f16_pair(tmem_base + 192, ad, make_sw128_desc(sb1 + k * 32), IDESC, (kb | k) != 0);
            }
            commit_both(&empty[stage]);
            next();
          }
          if (!ok) break;
          commit_both(t1full);
          // G2 reads the XA values the epilogue warps of both CTAs wrote into tensor memory
          if (!(ok = data_ready(actready, ph))) break;
          tc_fence_after();
          for (int s2 = 0; s2 < C::KB2 / C::G2_KBS; s2++) {
            if (!(ok = data_ready(&full[stage], phase))) break;
            tc_fence_after();
            const uint32_t sb = smem_u32(stages + stage * C::STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < C::G2_KBS; j++) {
#pragma unroll
              for (int k = 0; k < 4; k++) {
                const int kk = (s2 * C::G2_KBS + j) * 4 + k;  // 16-channel block of XA
                const uint32_t a_t = tmem_base + 128u * (uint32_t)(kk >> 3) + 8u * (uint32_t)(kk & 7);
                umma_f16_pair_ts(tmem_base + C::ACC2, a_t, make_sw128_desc(sb + j * C::B_BYTES + k * 32), IDESC,
                                 (s2 | j | k) != 0);
              }
            }
            commit_both(&empty[stage]);
            next();
          }
          if (!ok) break;
          commit_both(t2full);
        }
        if (!ok) {
          *abort_flag = 1;
          umma_commit_pair(smem_u32(drain));  // wait for MMAs in flight before TMEM is released
          mbar_wait(drain, 0, p.err, DEV_TIMEOUT_DRAIN);
        }
      }
      __syncwarp();
    }  // warps 2, 3: idle
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::EPI_REGS));
    // ---- epilogue warps (both CTAs): TMEM lane quarter warp % 4, channel group (warp - EPI_WARP0) / 4
    const int ew = warp - C::EPI_WARP0;
    const int q = warp & 3;
    const int h = ew >> 2;
    uint8_t* wbuf = epi + ew * C::EPI_WARP_BYTES;
    uint8_t* st_raw = wbuf;
    uint8_t* st_act = wbuf + C::BOX;
    uint8_t* ring = wbuf + 2 * C::BOX;
    uint64_t* rb = rbar + C::NRES * ew;
    const uint32_t actready_l = mapa_shared(smem_u32(actready), 0);
    const uint32_t e2lo_l = mapa_shared(smem_u32(e2lo), 0);
    constexpr int E1_CHUNKS = 4, E2_CHUNKS = 2;  // 32-column chunks per warp: 128 trunk / 64 opening channels
    // residual box u (this warp's u-th E1 chunk over its tiles) into ring buffer u % NRES, NRES boxes ahead
    auto res_issue = [&](int u) {
      const int i = u / E1_CHUNKS, k = u - i * E1_CHUNKS;
      const int it = pair + i * npairs;
      if (it >= num_tiles) return;
      const int mrow = it * 256 + (int)rank * 128 + q * 32;
      mbar_expect_tx(&rb[u % C::NRES], C::BOX);
      tma_load_2d(ring + (u % C::NRES) * C::BOX, &tmTrunk, &rb[u % C::NRES], p.trunk_x + h * 128 + k * 32, mrow);
    };
    if (lane == 0)
      for (int i = 0; i < C::NRES; i++) res_issue(i);

    int u = 0, lt = 0;
    bool ok = true;
    for (int it = pair; it < num_tiles && ok; it += npairs, lt++) {
      const uint32_t ph = lt & 1;
      const int mrow = it * 256 + (int)rank * 128 + q * 32;
      const int r = mrow + lane;
      const float m = r < p.rows ? __ldg(p.rowmask + r) : 0.0f;
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16);
      // ---- E1: trunk = acc + residual (raw, stored); XA = act1(bn1(trunk)) * mask into tensor memory
      if (!mbar_wait(t1full, ph, p.err, DEV_TIMEOUT_EPILOGUE) || *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < E1_CHUNKS; cc++, u++) {
        const int col = h * 128 + cc * 32;
        uint32_t x[32];
        tmem_ld32(tl + col, x);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(x[i]);
        if (!mbar_wait(&rb[u % C::NRES], (u / C::NRES) & 1, p.err, DEV_TIMEOUT_EPILOGUE)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        const uint8_t* rbox = ring + (u % C::NRES) * C::BOX;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          uint4 w = *reinterpret_cast<const uint4*>(rbox + sw64_off(lane, j));
          const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
          for (int k = 0; k < 8; k++) v[8 * j + k] += to_f<T>(e[k]);
        }
        __syncwarp();
        if (lane == 0) {
          fence_proxy_async_smem();
          res_issue(u + C::NRES);
        }
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        {
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const f32x2 y = mul2({v[i], v[i + 1]}, {m, m});
            o[i] = y.x;
            o[i + 1] = y.y;
          }
          stage_row<T>(st_raw, lane, o);
        }
        {
          float o[32];
          chain_act<T>(p.act1, v, s_sc1 + col, s_bi1 + col, m, o);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; i++) pk[i] = pack2<T>(o[2 * i], o[2 * i + 1]);
          // columns this warp has drained: [128 h + 16 cc, + 16) lies inside chunk cc / 2's 32 columns
          tmem_st16(tl + h * 128 + cc * 16, pk);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmTrunk, st_raw, p.trunk_x + col, mrow);
          bulk_commit_group();
        }
      }
      if (!ok) break;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(actready_l);
      // ---- E2: the opening's raw and act outputs from G2's accumulator
      if (!mbar_wait(t2full, ph, p.err, DEV_TIMEOUT_EPILOGUE) || *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < E2_CHUNKS; cc++) {
        const int col = h * 64 + cc * 32;
        uint32_t x[32];
        tmem_ld32(tl + C::ACC2 + col, x);
        tmem_wait_ld();
        if (h == 0 && cc == E2_CHUNKS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(e2lo_l);
        }
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __uint_as_float(x[i]);
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        {
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const f32x2 y = mul2({v[i], v[i + 1]}, {m, m});
            o[i] = y.x;
            o[i + 1] = y.y;
          }
          stage_row<T>(st_raw, lane, o);
        }
        {
          float o[32];
          chain_act<T>(p.act2, v, s_sc2 + col, s_bi2 + col, m, o);
          stage_row<T>(st_act, lane, o);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmRaw2, st_raw, p.raw2_x + col, mrow);
          tma_store_2d(&tmAct2, st_act, p.act2_x + col, mrow);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait0();
    if (!ok) {
      // residual boxes may still be in flight towards this warp's buffers: let them land (bounded)
      unsigned long long t0 = globaltimer();
      while (globaltimer() - t0 < 2000000ull) {
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace kc
