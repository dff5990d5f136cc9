// The trunk's convolution / linear GEMM on a CTA pair: tcgen05 MMAs of M = 256 rows (cta_group::2, 128 rows per
// CTA), operand tiles by TMA in 128-channel pipeline stages, accumulators in TMEM, and an epilogue that stages each
// 32 x 32 output box in shared memory and writes it with a TMA store (residuals arrive the same way, by TMA loads).
//
// It computes what gemm_tc_kernel computes for
//  * MODE_SEGMENTS: one or two column segments of 2-byte outputs and residuals (the raw / residual /
//    batch-norm-activation epilogue of bin2onnx.py residual_block :1243-1248 and nested_bottleneck_block
//    :1263-1269): y = A * W^T (* mask) (+ residual); raw = y * mask; act = act(y * scale + bias) * mask. RF32: the
//    residual and the raw output are float32 (the bf16 tier's residual stream; transformer_attention_block and
//    transformer_ffn_block's output linears, :1359-1438, with the branch output masked before the add);
//  * MODE_ROPE: the attention block's Q|K|V linear with 2D RoPE on the Q and K heads (head dim 64, the head's two
//    rotation halves at columns [0, 32) and [32, 64), :1369-1374 and :449-484): one head per epilogue warp; the
//    cos / sin tables indexed by board row (GemmParams::rope_cos / rope_sin: [tables][432][32]);
//  * MODE_SWIGLU: the FFN's first linear and gate, SiLU(x W1) * (x Wg) * mask (:1425-1438), each tile's columns
//    [linear1 | gate] halves.
//
// Why the layout is what it is (measured on B200):
//  * tcgen05.mma issue blocks the issuing thread once about four MMAs are queued, and each barrier wait + commit
//    costs it a few hundred cycles, so a stage carries two or three 64-channel K-blocks (8-12 MMAs per wait);
//  * M = 256 over a CTA pair halves the B (weight) bytes each SM loads and stages, which leaves the shared memory
//    for two such stages plus the epilogue's staging boxes;
//  * row-per-thread global stores cost one memory transaction per 16 bytes; a TMA store writes a whole box.
#pragma once

#include "gemm.cuh"

namespace kc {

// Tiles that may run as column halves: windowed 3x3 tiles and residual-free 1x1 tiles of width >= 128. Rows of one
// TMA load of their weights (B): half of a CTA's BH rows (a whole tile loads both halves, a half tile one), BH
// otherwise.
__host__ __device__ constexpr bool pair_split_tiles(int bn, bool win, bool nores) { return (win || nores) && bn >= 128; }
__host__ __device__ constexpr int pair_b_box_rows(int bn, bool win, bool nores) {
  return pair_split_tiles(bn, win, nores) ? bn / 4 : bn / 2;
}

// WIN (3x3 convolutions, 9 taps): per 64-channel chunk, each CTA loads one A window (its 128 rows plus the taps'
// halo above and below) into one of two window slots, and every tap's MMA reads its 128 rows at the tap's row offset
// inside the window; the pipeline stages carry the weight boxes (three taps per stage: 12 MMAs per wait). The
// window travels with its chunk's first stage, on that stage's barrier: no barriers of its own. Slot ch % 2 is free
// when that stage's slot is (its MMAs follow chunk ch - 2's whenever STAGES <= 4, with 3 stages per chunk). This cuts the TMA bytes of a
// 3x3 convolution's K-block from 28 KB to about 14 KB per CTA, below what TMA delivers per SM.
// NORES: the tile has no residual input, so its epilogue warps need no residual boxes; the shared memory goes to
// pipeline stages instead (the 1x1 convolutions without a residual: a third stage).
// SPLIT (pair_split_tiles): the tiles of a launch's last, partly filled round may run as column halves
// (MMAs of N = BN / 2 on the same accumulator, one weight box per K-block instead of two, the epilogue warps' boxes
// shared out over the half), one half per pair, so that the round takes about half a tile's time on up to twice
// as many pairs (GemmParams::split_from).
template <int BN, bool WIN = false, bool RF32 = false, bool NORES = false>
struct PairCfg {
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "pair tile width");
  static_assert(!(WIN && RF32), "float32 residual tiles are linears");
  static constexpr int BH = BN / 2;               // B rows (output columns) staged by each CTA of the pair
  static constexpr int A_BYTES = 128 * 64 * 2;    // one 64-channel K-block of this CTA's 128 rows
  static constexpr int B_BYTES = BH * 64 * 2;     // one K-block of this CTA's half of the weights
  static constexpr bool SPLIT = pair_split_tiles(BN, WIN, NORES);  // work items may be column halves of tiles
  static constexpr int BBOX = pair_b_box_rows(BN, WIN, NORES);     // weight rows per TMA load
  static constexpr int HALF_CHUNKS = BN / 64;               // 32-column boxes of a half tile
  static constexpr int KB_BYTES = (WIN ? 0 : A_BYTES) + B_BYTES;  // one K-block's slot in a stage
  static constexpr int KBS = WIN ? 3 : 2;         // K-blocks per pipeline stage (WIN: a row of three taps)
  static constexpr int WIN_TAPS = 9;
  static constexpr int STAGE_BYTES = KBS * KB_BYTES;
  static constexpr int WIN_MAX_ROWS = 176;        // 128 rows + a halo of up to 24 rows on each side
  static constexpr int A_WIN_BYTES = WIN_MAX_ROWS * 128;
  static constexpr int A_RING_BYTES = WIN ? 2 * A_WIN_BYTES : 0;
  // Epilogue warps: 2 or (1x1 tiles of BN = 192, whose time is the epilogue's) 3 per TMEM lane quarter, splitting
  // the tile's columns; the windowed 3x3 keeps 2 (its third weight stage is worth more), and so do float32
  // residual tiles (their boxes are twice as large). With 12 epilogue warps
  // the CTA has 16 (512 threads, 128 registers each at launch) and setmaxnreg moves registers from warpgroup 0
  // (TMA producer, MMA issuer, two idle warps: 48 each) to the three epilogue warpgroups (152 each):
  // 4 x 32 x 48 + 12 x 32 x 152 = 64,512 <= 65,536, per SMSP 48 + 3 x 152 = 504 <= 4 x 128. (With 56 for
  // warpgroup 0 the compiler spilled in the residual 1x1 instance; with 48 it does not.)
  static constexpr int EPI_WARPS = BN == 192 && !WIN && !RF32 ? 12 : 8;
  static constexpr int EPI_WARP0 = EPI_WARPS == 12 ? 4 : 2;  // first epilogue warp (a warpgroup boundary with 12)
  static constexpr int WG0_REGS = 48, EPI_REGS = 152;
  static_assert(WG0_REGS + 3 * EPI_REGS <= 4 * 128 && WG0_REGS % 8 == 0 && EPI_REGS % 8 == 0, "register split");
  static constexpr int WARP_COLS = BN / (EPI_WARPS / 4);
  static constexpr int CHUNKS = WARP_COLS / 32;   // 32-column boxes per warp and tile
  // staging boxes of 32 rows x 32 columns: 2-byte outputs in 64-byte rows (64-byte swizzle), float32 raw outputs
  // and residuals in 128-byte rows (128-byte swizzle)
  static constexpr int BOX_BYTES = 32 * 32 * 2;
  static constexpr int RBOX_BYTES = RF32 ? 32 * 32 * 4 : BOX_BYTES;  // raw output and residual boxes
  static constexpr int ABOX_BYTES = RF32 ? 0 : BOX_BYTES;            // act output box (none with RF32)
  static constexpr int NRES = NORES ? 0 : WIN || RF32 || BN > 128 ? 2 : 4;  // residual boxes in flight per warp
  static constexpr int EPI_WARP_BYTES = RBOX_BYTES + ABOX_BYTES + NRES * RBOX_BYTES;  // raw, act, residual ring
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_WARP_BYTES;
  static constexpr int PARAM_COLS = 768;          // per-column BN scale / bias in shared memory
  static constexpr int PARAM_BYTES = 2 * PARAM_COLS * 4;
  static constexpr int PCOPY_BYTES = 1024;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_LIMIT = 227 * 1024;
  static constexpr int FIXED =
      1024 /*align slack*/ + A_RING_BYTES + EPI_BYTES + PARAM_BYTES + PCOPY_BYTES + BAR_BYTES;
  static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 4 ? 4 : FIT;
  static_assert(STAGES >= 2 && (!WIN || STAGES <= 4), "pair pipeline depth");
  static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
  static constexpr uint32_t ACC_COLS = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
  static_assert(WARP_COLS % 32 == 0, "epilogue warp columns");
};

// The 16-byte chunk `j` (0..3) of row `r` of a 32 x 64-byte box written by TMA with CU_TENSOR_MAP_SWIZZLE_64B:
// the chunk index is XORed with address bits 7-8, i.e. with (r / 2) % 4 for 64-byte rows. Thread r of a warp
// touching chunk j of its own row hits 8 distinct 16-byte bank groups per 8 threads: no conflicts.
__device__ __forceinline__ uint32_t sw64_off(int r, int j) { return (uint32_t)(r * 64 + ((j ^ ((r >> 1) & 3)) << 4)); }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Write 32 floats of this thread's row into a 64-byte-swizzled staging box as T.
template <typename T>
__device__ __forceinline__ void stage_row(uint8_t* box, int r, const float (&o)[32]) {
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint4 u;
    u.x = pack2<T>(o[8 * j + 0], o[8 * j + 1]);
    u.y = pack2<T>(o[8 * j + 2], o[8 * j + 3]);
    u.z = pack2<T>(o[8 * j + 4], o[8 * j + 5]);
    u.w = pack2<T>(o[8 * j + 6], o[8 * j + 7]);
    *reinterpret_cast<uint4*>(box + sw64_off(r, j)) = u;
  }
}

// Write 32 floats of this thread's row into a 128-byte-swizzled float32 staging box (CU_TENSOR_MAP_SWIZZLE_128B:
// 16-byte chunk j of row r at chunk j ^ (r % 8); conflict-free for the 8 threads of a 128-bit store phase).
__device__ __forceinline__ void stage_row_f32(uint8_t* box, int r, const float (&o)[32]) {
#pragma unroll
  for (int j = 0; j < 8; j++)
    *reinterpret_cast<float4*>(box + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
}

// Packed two-lane float32 arithmetic (sm_100 fma / mul / add .f32x2): two elements per instruction, float32
// rounding per element.
struct f32x2 {
  float x, y;
};
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// mish(t) * m for two elements t = v * s + b, as act_fn<2> (x * n / (n + 2), n = e^2 + 2e, e = exp(min(x, 20)))
// but with one MUFU operation per element: 1 / (n + 2) by Newton-Raphson from an integer-subtraction seed on the
// float's bit pattern (J. Blinn, "Floating-Point Tricks", IEEE CG&A 17(4), 1997: the bit pattern is a scaled,
// offset piecewise-linear log2, so kSeed - bits(d) approximates the bits of 1 / d). kSeed is the constant with the
// smallest largest relative error of the seed over a binade (an exhaustive search over the 2^23 significands): 5.05%
// for every d in [2, 2.4e17] seen here; two steps r <- r (2 - d r) bring it below 7e-6, under the 2-byte outputs'
// rounding (tests/test_mish_seed.py checks both in float32 arithmetic). Above x = 20, where act_fn<2> returns x,
// n / (n + 2) evaluates to 1 within that error, so no select is needed.
constexpr int kRcpSeed = 0x7EF311C2;
__device__ __forceinline__ f32x2 mish2(f32x2 v, f32x2 s, f32x2 b, float m) {
  const f32x2 t = fma2(v, s, b);
  const f32x2 e = {__expf(fminf(t.x, 20.0f)), __expf(fminf(t.y, 20.0f))};
  const f32x2 two = {2.0f, 2.0f};
  const f32x2 n = mul2(e, add2(e, two));
  const f32x2 d = add2(n, two);
  const f32x2 nd = {-d.x, -d.y};
  f32x2 r = {__int_as_float(kRcpSeed - __float_as_int(d.x)), __int_as_float(kRcpSeed - __float_as_int(d.y))};
  r = mul2(r, fma2(nd, r, two));
  r = mul2(r, fma2(nd, r, two));
  return mul2(mul2(t, mul2(n, r)), f32x2{m, m});
}

// act(v * scale + bias) * mask over 32 columns, scale / bias from shared memory (broadcast reads).
template <int ACT>
__device__ __forceinline__ void pair_act(const float (&v)[32], const float* sc, const float* bi, float m,
                                         float (&o)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 16) {
    float s[16], b[16];
    lds16(sc + j, s);
    lds16(bi + j, b);
    if constexpr (ACT == 2) {
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const f32x2 y = mish2({v[j + i], v[j + i + 1]}, {s[i], s[i + 1]}, {b[i], b[i + 1]}, m);
        o[j + i] = y.x;
        o[j + i + 1] = y.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float t = v[j + i] * s[i];
        t = t + b[i];
        o[j + i] = act_fn<ACT>(t) * m;
      }
    }
  }
}

template <typename T, int BN, bool WIN, int MODE = MODE_SEGMENTS, bool RF32 = false, bool NORES = false>
__global__ void __launch_bounds__(PairCfg<BN, WIN, RF32, NORES>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmRes, const __grid_constant__ CUtensorMap tmRaw,
                     const __grid_constant__ CUtensorMap tmAct, const __grid_constant__ GemmParams p) {
  using C = PairCfg<BN, WIN, RF32, NORES>;
  static_assert(MODE != MODE_ROPE || C::WARP_COLS == 64, "RoPE tiles give each epilogue warp one head of 64");
  static_assert(MODE != MODE_ROPE || (C::NRES * C::RBOX_BYTES >= 4096 && C::RBOX_BYTES + C::ABOX_BYTES == 4096),
                "RoPE table rows: cos in the residual ring, sin in the raw and act staging boxes");
  static_assert(MODE != MODE_SWIGLU || (BN % 128 == 0 && C::EPI_WARPS == 8), "SwiGLU tile halves");
  static_assert(MODE == MODE_SEGMENTS || (!WIN && !RF32), "RoPE / SwiGLU tiles are linears");
  constexpr int fmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC = make_idesc_f16(fmt, 256, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* awin = smem;  // WIN: the two A windows
  uint8_t* stages = smem + C::A_RING_BYTES;
  uint8_t* epi = stages + C::STAGES * C::STAGE_BYTES;
  float* s_scale = reinterpret_cast<float*>(epi + C::EPI_BYTES);
  float* s_bias = s_scale + C::PARAM_COLS;
  GemmParams* s_params = reinterpret_cast<GemmParams*>(s_bias + C::PARAM_COLS);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_params) + C::PCOPY_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* rbar = drain + 1;  // [EPI_WARPS][NRES]: the residual boxes of each epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + C::NRES * C::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  static_assert(sizeof(GemmParams) <= C::PCOPY_BYTES && sizeof(GemmParams) % 16 == 0, "parameter copy");
  static_assert((2 * C::STAGES + 5 + C::NRES * C::EPI_WARPS) * 8 + 8 <= C::BAR_BYTES, "barrier area");
  for (int i = threadIdx.x; i < (int)(sizeof(GemmParams) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(s_params)[i] = reinterpret_cast<const uint4*>(&p)[i];
  // one or two column segments: [0, split) segment 0, [split, n_total) segment 1 (split a multiple of 32); a
  // one-segment GEMM never reads segment 1
  const int split = p.nseg > 1 ? p.pair_split : p.n_total;
  const int f0 = p.seg[0].flags, f1 = p.nseg > 1 ? p.seg[1].flags : f0;
  const int flags = f0 | f1;
  if ((flags & EPI_ACT) && p.n_total <= C::PARAM_COLS) {
    for (int col = threadIdx.x; col < p.n_total; col += blockDim.x) {
      const bool s1 = col >= split;
      const bool act = ((s1 ? f1 : f0) & EPI_ACT) != 0;
      s_scale[col] = act ? (s1 ? p.seg[1].scale[col - split] : p.seg[0].scale[col]) : 0.0f;
      s_bias[col] = act ? (s1 ? p.seg[1].bias[col - split] : p.seg[0].bias[col]) : 0.0f;
    }
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int n_tiles = p.n_total / BN;
  const int num_tiles = ((p.g.rows + 255) / 256) * n_tiles;
  const int kb_per_tap = p.cin / 64;
  const int KB = p.taps * kb_per_tap;
  const int NST = (KB + C::KBS - 1) / C::KBS;
  // work items: tiles [0, sf) whole, then two column halves per tile (SPLIT); each pair takes items pair,
  // pair + npairs, ... and so at most one half item, its last
  int sf = num_tiles;
  if constexpr (C::SPLIT) {
    if (p.split_from < num_tiles && p.split_from % npairs == 0 && 2 * (num_tiles - p.split_from) <= npairs)
      sf = p.split_from;
  }
  const int num_items = sf + 2 * (num_tiles - sf);
  // item -> tile and column half (-1: the whole tile)
  auto item_tile = [&](int it, int& hf) {
    if (!C::SPLIT || it < sf) {
      hf = -1;
      return it;
    }
    hf = (it - sf) & 1;
    return sf + ((it - sf) >> 1);
  };
  constexpr uint32_t IDESC_HALF = make_idesc_f16(fmt, 256, C::SPLIT ? BN / 2 : BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * C::EPI_WARPS);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    for (int i = 0; i < C::NRES * C::EPI_WARPS; i++) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 0) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or transaction
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above (barriers, TMEM, cluster barrier, parameter and BN-table copies) overlaps the previous
  // kernel's tail
  pdl_wait();
  pdl_trigger();

  if (warp < C::EPI_WARP0) {
  if constexpr (C::EPI_WARPS == 12) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::WG0_REGS));
  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): this CTA's A rows and half of B; the bytes count on the leader's barrier
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int as = 0;
      // wait for a ring slot this CTA may refill; false (and abort) on a timeout
      auto slot_free = [&](uint64_t* bar, uint32_t parity) {
        if (mbar_try_wait(bar, parity)) return true;
        if (!*abort_flag && mbar_wait(bar, parity, p.err, DEV_TIMEOUT_PRODUCER)) return true;
        *abort_flag = 1;
        return false;
      };
      for (int it = pair; it < num_items && ok; it += npairs) {
        int hf;
        const int tile = item_tile(it, hf);
        const int m0 = (tile / n_tiles) * 256 + (int)rank * 128;
        // this CTA's weight rows: half of the tile's columns, or (half item) half of the item's BN / 2
        const int nb = (tile % n_tiles) * BN + (hf < 0 ? (int)rank * C::BH : hf * (BN / 2) + (int)rank * (BN / 4));
        if constexpr (WIN) {
          const uint32_t b_bytes = hf < 0 ? C::B_BYTES : C::B_BYTES / 2;
          for (int ch = 0; ch < kb_per_tap && ok; ch++) {
            for (int t0 = 0; t0 < C::WIN_TAPS; t0 += C::KBS) {
              if (!(ok = slot_free(&empty[stage], phase ^ 1))) break;
              const uint32_t win_bytes = t0 == 0 ? (uint32_t)p.win_rows * 128u : 0u;
              if (leader) mbar_expect_tx(&full[stage], 2u * (C::KBS * b_bytes + win_bytes));
              const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
              if (t0 == 0) {  // the chunk's A window rides on its first stage
                tma_load_2d_pair(awin + as * C::A_WIN_BYTES, &tmA, fb, ch * 64, m0 - p.halo);
                as ^= 1;
              }
              for (int j = 0; j < C::KBS; j++) {
                uint8_t* dst = stages + stage * C::STAGE_BYTES + j * C::KB_BYTES;
                const int x = (t0 + j) * p.cin + ch * 64;
                tma_load_2d_pair(dst, &tmB, fb, x, nb);
                // a whole tile's second weight box: the rows after the first, where one box of BH rows would put
                // them (BBOX rows of 128 bytes = whole 1024-byte swizzle atoms)
                if (C::SPLIT && hf < 0) tma_load_2d_pair(dst + C::BBOX * 128, &tmB, fb, x, nb + C::BBOX);
              }
              if (++stage == C::STAGES) {
                stage = 0;
                phase ^= 1;
              }
            }
          }
        } else {
          const uint32_t kb_bytes = hf < 0 ? C::KB_BYTES : C::A_BYTES + C::B_BYTES / 2;
          for (int st = 0; st < NST; st++) {
            if (!(ok = slot_free(&empty[stage], phase ^ 1))) break;
            const int kb0 = st * C::KBS;
            const int nk = KB - kb0 < C::KBS ? KB - kb0 : C::KBS;
            if (leader) mbar_expect_tx(&full[stage], 2u * (uint32_t)nk * kb_bytes);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            uint8_t* sbase = stages + stage * C::STAGE_BYTES;
            for (int j = 0; j < nk; j++) {
              const int kb = kb0 + j;
              const int tap = kb / kb_per_tap;
              const int c0 = (kb - tap * kb_per_tap) * 64;
              uint8_t* dst = sbase + j * C::KB_BYTES + C::A_BYTES;
              tma_load_2d_pair(sbase + j * C::KB_BYTES, &tmA, fb, c0, m0 + s_params->tap_off[tap]);
              tma_load_2d_pair(dst, &tmB, fb, kb * 64, nb);
              if (C::SPLIT && hf < 0) tma_load_2d_pair(dst + C::BBOX * 128, &tmB, fb, kb * 64, nb + C::BBOX);
            }
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
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader CTA only): one M = 256 MMA covers both CTAs' rows
      const uint32_t peer = 1;
      int stage = 0;
      uint32_t phase = 0;
      int as = 0;
      int local = 0;
      bool ok = true;
      // WIN: byte offset of each tap's 128 rows inside the window (halo + tap row offset; any row works: the
      // 128-byte swizzle follows the absolute address, so the descriptors' base offset stays 0). Held in registers:
      // a shared-memory read between a commit and the next MMAs stalls the issuing thread.
      uint32_t win_off[C::WIN_TAPS];
#pragma unroll
      for (int t = 0; t < C::WIN_TAPS; t++) win_off[t] = WIN ? (uint32_t)(p.halo + s_params->tap_off[t]) * 128u : 0u;
      for (int it = pair; it < num_items && ok; it += npairs, local++) {
        int hf;
        item_tile(it, hf);
        const uint32_t idesc = hf < 0 ? IDESC : IDESC_HALF;  // a half item: N = BN / 2
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, DEV_TIMEOUT_MMA) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
        auto data_ready = [&](uint64_t* bar, uint32_t parity) {
          if (mbar_try_wait(bar, parity)) return true;
          return !*abort_flag && mbar_wait(bar, parity, p.err, DEV_TIMEOUT_MMA);
        };
        // the pair's MMAs have read this stage: both CTAs may refill it
        auto release = [&](uint64_t* bar) {
          const uint32_t b = smem_u32(bar);
          umma_commit_pair(b);
          umma_commit_pair(mapa_shared(b, peer));
        };
        if constexpr (WIN) {
          for (int ch = 0; ch < kb_per_tap && ok; ch++) {
            const uint32_t swin = smem_u32(awin + as * C::A_WIN_BYTES);
            as ^= 1;
#pragma unroll
            for (int g = 0; g < C::WIN_TAPS / C::KBS; g++) {
              if (!(ok = data_ready(&full[stage], phase))) break;
              tc_fence_after();
              const uint32_t sbase = smem_u32(stages + stage * C::STAGE_BYTES);
#pragma unroll
              for (int j = 0; j < C::KBS; j++) {
                const uint32_t sa = swin + win_off[g * C::KBS + j];
                const uint32_t sb = sbase + j * C::KB_BYTES;
#pragma unroll
                for (int k = 0; k < 4; k++)
                  umma_f16_pair(d_tmem, make_sw128_desc(sa + k * 32), make_sw128_desc(sb + k * 32), idesc,
                                (ch | g | j | k) != 0);
              }
              release(&empty[stage]);
              if (++stage == C::STAGES) {
                stage = 0;
                phase ^= 1;
              }
            }
            if (!ok) break;
          }
        } else {
          for (int st = 0; st < NST; st++) {
            if (!(ok = data_ready(&full[stage], phase))) break;
            tc_fence_after();
            const int nk = KB - st * C::KBS < C::KBS ? KB - st * C::KBS : C::KBS;
            const uint32_t sbase = smem_u32(stages + stage * C::STAGE_BYTES);
            for (int j = 0; j < nk; j++) {
              const uint32_t sa = sbase + j * C::KB_BYTES, sb = sa + C::A_BYTES;
#pragma unroll
              for (int k = 0; k < 4; k++)
                umma_f16_pair(d_tmem, make_sw128_desc(sa + k * 32), make_sw128_desc(sb + k * 32), idesc,
                              (st | j | k) != 0);
            }
            release(&empty[stage]);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        if (!ok) break;
        const uint32_t tb = smem_u32(&tfull[acc]);
        umma_commit_pair(tb);
        umma_commit_pair(mapa_shared(tb, peer));
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit_pair(smem_u32(drain));  // wait for MMAs in flight before TMEM is released
        mbar_wait(drain, 0, p.err, DEV_TIMEOUT_DRAIN);
      }
    }
    __syncwarp();
  }  // warps 2 .. EPI_WARP0 - 1: idle
  } else {
    if constexpr (C::EPI_WARPS == 12) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::EPI_REGS));
    // ---- epilogue warps (both CTAs): TMEM lane quarter warp % 4, column part (warp - EPI_WARP0) / 4
    const int ew = warp - C::EPI_WARP0;
    const int q = warp & 3;
    const int h = ew >> 2;
    uint8_t* wbuf = epi + ew * C::EPI_WARP_BYTES;
    uint8_t* st_raw = wbuf;
    uint8_t* st_act = wbuf + C::RBOX_BYTES;  // RoPE: the head's second rotation half
    constexpr int RES_OFF = C::RBOX_BYTES + C::ABOX_BYTES;  // the residual ring after the raw and act boxes
    constexpr int NRING = C::NRES > 0 ? C::NRES : 1;         // its length (NORES: no ring, never indexed)
    uint64_t* rb = rbar + C::NRES * ew;
    const bool has_res = !NORES && (flags & EPI_RESIDUAL) != 0;  // one-segment GEMMs only
    const int a0 = p.seg[0].act, a1 = p.nseg > 1 ? p.seg[1].act : a0;
    const int res_x = p.pair_res_x, raw_x = p.pair_raw_x, act_x = p.pair_act_x;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);

    // this warp's 32-column boxes of an item, [cb, ce) counted from the item's first column: CHUNKS of a whole
    // tile, or its column group's share of a half tile's HALF_CHUNKS (the first groups take the odd ones)
    constexpr int GROUPS = C::EPI_WARPS / 4;
    auto chunk_range = [&](int hf, int& cb, int& ce) {
      if (!C::SPLIT || hf < 0) {
        cb = h * C::CHUNKS;
        ce = cb + C::CHUNKS;
      } else {
        constexpr int per = (C::HALF_CHUNKS + GROUPS - 1) / GROUPS;
        cb = h * per;
        ce = cb + per < C::HALF_CHUNKS ? cb + per : C::HALF_CHUNKS;
      }
    };
    static_assert(!C::SPLIT || (GROUPS - 1) * ((C::HALF_CHUNKS + GROUPS - 1) / GROUPS) < C::HALF_CHUNKS,
                  "every epilogue warp has a box of a half tile");

    // residual boxes run NRES boxes ahead: box u (this warp's u-th 32-column chunk over its items; CHUNKS per whole
    // tile, and fewer for a pair's last item if that is a half tile) goes to buffer u % NRES
    auto res_issue = [&](int u) {
      const int i = u / C::CHUNKS, k = u - i * C::CHUNKS;
      const int it = pair + i * npairs;
      if (it >= num_items) return;
      int hf, cb, ce;
      const int tile = item_tile(it, hf);
      chunk_range(hf, cb, ce);
      if (cb + k >= ce) return;
      const int mrow = (tile / n_tiles) * 256 + (int)rank * 128 + q * 32;
      const int col = (tile % n_tiles) * BN + (hf > 0 ? BN / 2 : 0) + (cb + k) * 32;
      mbar_expect_tx(&rb[u % NRING], C::RBOX_BYTES);
      tma_load_2d(wbuf + RES_OFF + (u % NRING) * C::RBOX_BYTES, &tmRes, &rb[u % NRING], res_x + col, mrow);
    };
    if (has_res && lane == 0)
      for (int i = 0; i < C::NRES; i++) res_issue(i);

    int local = 0, u = 0;
    bool ok = true;
    for (int it = pair; it < num_items && ok; it += npairs, local++) {
      int hf, cb, ce;
      const int tile = item_tile(it, hf);
      chunk_range(hf, cb, ce);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int mrow = (tile / n_tiles) * 256 + (int)rank * 128 + q * 32;
      const int r = mrow + lane;
      const float m = r < p.g.rows ? __ldg(p.g.rowmask + r) : 0.0f;
      const int icol0 = (tile % n_tiles) * BN + (hf > 0 ? BN / 2 : 0);  // the item's first column
      const int ncol0 = icol0 + h * C::WARP_COLS;                         // RoPE / SwiGLU: whole tiles
      // RoPE: this warp's 32 rows of the head's cos / sin table (board-row-indexed, 432 rows per table so that 32
      // rows from any board row stay inside it), 4 KB blocks read with coalesced 128-bit loads while the
      // accumulator is computed, into shared memory as 128-byte rows with the 128-byte swizzle, from where each
      // thread reads its row: cos in the residual ring (unused here), sin in the raw and act staging boxes, free
      // until this tile's outputs are staged once the previous tile's stores have read them
      bool rot = false;
      uint8_t* tab = wbuf + RES_OFF;
      uint8_t* tab_s = wbuf;
      if constexpr (MODE == MODE_ROPE) {
        rot = ncol0 < p.rope_rot_cols;
        if (rot) {
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          const int head = ncol0 / 64;
          const int table = ncol0 < p.rope_q_cols ? head / p.rope_group : head - p.rope_q_cols / 64;
          const size_t toff = (size_t)table * p.rope_table_stride + (size_t)(mrow % 400) * 32 + lane * 4;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float4 c = __ldg(reinterpret_cast<const float4*>(p.rope_cos + toff + i * 128));
            const float4 sn = __ldg(reinterpret_cast<const float4*>(p.rope_sin + toff + i * 128));
            const int row = (lane >> 3) + 4 * i, chunk = lane & 7;
            const uint32_t off = row * 128 + ((chunk ^ (row & 7)) << 4);
            *reinterpret_cast<float4*>(tab + off) = c;
            *reinterpret_cast<float4*>(tab_s + off) = sn;
          }
        }
      }
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, DEV_TIMEOUT_EPILOGUE) || *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      if constexpr (MODE == MODE_SEGMENTS) {
        const uint32_t tacc = tmem_base + acc * C::ACC_COLS + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
        for (int cc = cb; cc < ce; cc++, u++) {
          uint32_t x[32];
          tmem_ld32(tacc + cc * 32, x);
          tmem_wait_ld();
          if (cc == ce - 1) {
            // the accumulator is in registers: hand it back to the MMA issuer before the math
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
          }
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = __uint_as_float(x[i]);
          if ((f0 & EPI_BOARD_BIAS) && m != 0.0f) {
            // per-board bias (one-segment GEMMs: the stem's global-feature term), 32 columns of this row's board
            const float* bb = p.seg[0].board_bias + (size_t)(r / 400) * p.seg[0].ld_bb + icol0 + cc * 32;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 q = __ldg(reinterpret_cast<const float4*>(bb + j));
              v[j] += q.x;
              v[j + 1] += q.y;
              v[j + 2] += q.z;
              v[j + 3] += q.w;
            }
          }
          // one-segment GEMMs of 8 epilogue warps (the 12-warp tiles have no registers to spare): the transformer
          // branch output is masked before the add
          if (C::EPI_WARPS == 8 && (f0 & EPI_MASK_ACC)) {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] *= m;
          }
          if (has_res) {
            if (!mbar_wait(&rb[u % NRING], (u / NRING) & 1, p.err, DEV_TIMEOUT_EPILOGUE)) {
              *abort_flag = 1;
              ok = false;
              break;
            }
            const uint8_t* rbox = wbuf + RES_OFF + (u % NRING) * C::RBOX_BYTES;
            if constexpr (RF32) {
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const float4 w = *reinterpret_cast<const float4*>(rbox + lane * 128 + ((j ^ (lane & 7)) << 4));
                v[4 * j] += w.x;
                v[4 * j + 1] += w.y;
                v[4 * j + 2] += w.z;
                v[4 * j + 3] += w.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; j++) {
                uint4 w = *reinterpret_cast<const uint4*>(rbox + sw64_off(lane, j));
                const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
                for (int k = 0; k < 8; k++) v[8 * j + k] += to_f<T>(e[k]);
              }
            }
            __syncwarp();
            if (lane == 0) {
              fence_proxy_async_smem();
              res_issue(u + C::NRES);
            }
          }
          // the previous box's stores must have read the staging boxes before they are overwritten
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          const int col = icol0 + cc * 32;
          const int cf = col < split ? f0 : f1;  // this box's segment
          if (cf & EPI_RAW) {
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const f32x2 y = mul2({v[i], v[i + 1]}, {m, m});
              o[i] = y.x;
              o[i + 1] = y.y;
            }
            if constexpr (RF32) stage_row_f32(st_raw, lane, o);
            else stage_row<T>(st_raw, lane, o);
          }
          if (!RF32 && (cf & EPI_ACT)) {
            float o[32];
            switch (col < split ? a0 : a1) {
              case 1: pair_act<1>(v, s_scale + col, s_bias + col, m, o); break;
              case 2: pair_act<2>(v, s_scale + col, s_bias + col, m, o); break;
              case 3: pair_act<3>(v, s_scale + col, s_bias + col, m, o); break;
              default: pair_act<0>(v, s_scale + col, s_bias + col, m, o); break;
            }
            stage_row<T>(st_act, lane, o);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (cf & EPI_RAW) tma_store_2d(&tmRaw, st_raw, raw_x + col, mrow);
            if (!RF32 && (cf & EPI_ACT)) tma_store_2d(&tmAct, st_act, act_x + col, mrow);
            bulk_commit_group();
          }
        }
      } else if constexpr (MODE == MODE_ROPE) {
        // one head of 64 columns per warp: Q and K heads rotated in halves of 32 (x0 at [0, 32), x1 at [32, 64)),
        // V heads as they are (the table rows were staged above; __syncwarp below orders them before the reads)
        const uint32_t tacc = tmem_base + acc * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + h * C::WARP_COLS;
        uint32_t x0[32], x1[32];
        tmem_ld32(tacc, x0);
        tmem_ld32(tacc + 32, x1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
        float o0[32], o1[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 cs = make_float4(1.0f, 1.0f, 1.0f, 1.0f), sn = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (rot) {
            const uint32_t off = lane * 128 + (((j >> 2) ^ (lane & 7)) << 4);
            cs = *reinterpret_cast<const float4*>(tab + off);
            sn = *reinterpret_cast<const float4*>(tab_s + off);
          }
          const float c4[4] = {cs.x, cs.y, cs.z, cs.w}, s4[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float a = __uint_as_float(x0[j + i]), b = __uint_as_float(x1[j + i]);
            o0[j + i] = (a * c4[i] - b * s4[i]) * m;
            o1[j + i] = (a * s4[i] + b * c4[i]) * m;
          }
        }
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        stage_row<T>(st_raw, lane, o0);
        stage_row<T>(st_act, lane, o1);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmRaw, st_raw, raw_x + ncol0, mrow);
          tma_store_2d(&tmRaw, st_act, raw_x + ncol0 + 32, mrow);
          bulk_commit_group();
        }
      } else {
        // SwiGLU: this warp's BN / 4 output columns, linear1 at accumulator columns [h BN / 4, ...) of the tile's
        // first half and the gate at the same place in its second half
        constexpr int OCH = BN / 128;
        const int ocol0 = (tile % n_tiles) * (BN / 2) + h * (BN / 4);
        const uint32_t tacc = tmem_base + acc * C::ACC_COLS + ((uint32_t)(q * 32) << 16) + h * (BN / 4);
#pragma unroll 1
        for (int c = 0; c < OCH; c++) {
          uint32_t xa[32], xg[32];
          tmem_ld32(tacc + c * 32, xa);
          tmem_ld32(tacc + BN / 2 + c * 32, xg);
          tmem_wait_ld();
          if (c == OCH - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
          }
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] = act_fn<3>(__uint_as_float(xa[i])) * __uint_as_float(xg[i]) * m;
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          stage_row<T>(st_raw, lane, o);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmRaw, st_raw, raw_x + ocol0 + c * 32, mrow);
            bulk_commit_group();
          }
        }
      }
    }
    if (lane == 0) bulk_wait0();
    if (!ok && has_res) {
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
