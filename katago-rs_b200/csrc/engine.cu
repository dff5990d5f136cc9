// Forward-pass engine: packs a parsed KataGo net into device layouts and builds the launch plan that evaluates it
// on boards in the padded board layout (PBL, see gemm.cuh). The plan follows the reference graph
// (tools/bin2onnx/bin2onnx.py GraphBuilder.trunk :1477, block_stack :1271, residual/gpool/nested blocks :1243-1269,
// transformer blocks :1359-1438, heads :1495-1531) with batch norm + activation + mask fused into the epilogue of
// the GEMM that produces each tensor, and the residual add fused into the GEMM that closes each block.

#include "engine.h"

#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <tuple>

#include "common.h"
#include "attention.cuh"
#include "gemm_chain.cuh"
#include "gemm_pair.cuh"
#include "kernels.cuh"

namespace kc {

namespace {

int round_up(int a, int b) { return (a + b - 1) / b * b; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up once per process (a function-local static: its initialisation is
// thread-safe, and handles are built from several host threads at once when one process serves several GPUs).
EncodeTiledFn encode_fn() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    KC_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess) fail(KC_ERR_CUDA, "CUDA backend: cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2D tensor map over a row-major [rows][cols] matrix of 2-byte elements, box [box_rows][64 elements], 128B swizzle.
CUtensorMap make_map(const void* base, bool bf16, int cols, int rows, int box_rows) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * 2) % 16 != 0 || cols % 64 != 0)
    fail(KC_ERR_INVALID, "CUDA backend: tensor map operand not 16-byte aligned");
  CUresult r = encode_fn()(&map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(KC_ERR_CUDA, "CUDA backend: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

// A 32-row x 32-column box map with the 64-byte swizzle: the epilogue boxes (outputs and residuals) of the
// CTA-pair GEMM.
CUtensorMap make_box_map(const void* base, bool bf16, int cols, int rows, bool f32 = false) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 32 != 0)
    fail(KC_ERR_INVALID, "CUDA backend: epilogue box operand not aligned");
  const CUtensorMapDataType dt = f32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // 32 columns: 64-byte rows of a 2-byte type, 128-byte rows of float32
  CUresult r = encode_fn()(&map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(KC_ERR_CUDA, "CUDA backend: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

// Opt the kernel instances into large dynamic shared memory, once per device (plan-build time, never while a
// stream is being captured).
template <typename K>
void allow_smem(K* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  KC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  if (done.count(key)) return;
  KC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert(key);
}

// Programmatic dependent launch: every kernel of a forward pass is launched with programmatic stream
// serialization, so that it can start (and run its prologue) on SMs the previous kernel has left; each kernel
// waits (griddepcontrol.wait) before its first access to memory an earlier kernel writes. KATAGO_CUDA_PDL=0 turns
// it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KATAGO_CUDA_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  KC_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

template <typename T, int BN, bool RF32>
void launch_tc_bn(bool prepare, int grid, cudaStream_t s, const CUtensorMap& a, const CUtensorMap& b,
                  const GemmParams& p) {
  using C = TcCfg<BN>;
  if (prepare) {
    allow_smem(gemm_tc_kernel<T, BN, RF32>, C::SMEM);
    return;
  }
  launch_pdl(gemm_tc_kernel<T, BN, RF32>, dim3(grid), dim3(C::THREADS), C::SMEM, s, a, b, p);
}

template <typename T, bool RF32>
void launch_tc_rf(bool prepare, int bn, int grid, cudaStream_t s, const CUtensorMap& a, const CUtensorMap& b,
                  const GemmParams& p) {
  switch (bn) {
    case 16: launch_tc_bn<T, 16, RF32>(prepare, grid, s, a, b, p); break;
    case 32: launch_tc_bn<T, 32, RF32>(prepare, grid, s, a, b, p); break;
    case 48: launch_tc_bn<T, 48, RF32>(prepare, grid, s, a, b, p); break;
    case 64: launch_tc_bn<T, 64, RF32>(prepare, grid, s, a, b, p); break;
    case 96: launch_tc_bn<T, 96, RF32>(prepare, grid, s, a, b, p); break;
    case 128: launch_tc_bn<T, 128, RF32>(prepare, grid, s, a, b, p); break;
    case 192: launch_tc_bn<T, 192, RF32>(prepare, grid, s, a, b, p); break;
    case 256: launch_tc_bn<T, 256, RF32>(prepare, grid, s, a, b, p); break;
    default: fail(KC_ERR_INVALID, "CUDA backend: unsupported GEMM tile width " + std::to_string(bn));
  }
}

// rf32: the GEMM's residual is a float32 stream (only the bf16 tier has those)
template <typename T>
void launch_tc(bool prepare, bool rf32, int bn, int grid, cudaStream_t s, const CUtensorMap& a, const CUtensorMap& b,
               const GemmParams& p) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (rf32) {
      launch_tc_rf<T, true>(prepare, bn, grid, s, a, b, p);
      return;
    }
  } else {
    if (rf32) fail(KC_ERR_INVALID, "CUDA backend: float32 residual stream outside the bf16 tier");
  }
  launch_tc_rf<T, false>(prepare, bn, grid, s, a, b, p);
}

// The CTA-pair GEMM, launched as clusters of two CTAs. `prepare` (plan-build time) opts the instance into its
// shared memory and returns how many pairs fit on the device at once; otherwise launches `pairs` pairs.
struct PairMaps {
  CUtensorMap a, b, res, raw, act;
};

template <typename T, int BN, bool WIN, int MODE, bool RF32, bool NORES = false>
int launch_pair_bn(bool prepare, int pairs, cudaStream_t s, const PairMaps& m, const GemmParams& p) {
  using C = PairCfg<BN, WIN, RF32, NORES>;
  auto kernel = gemm_pair_kernel<T, BN, WIN, MODE, RF32, NORES>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (prepare) {
    allow_smem(kernel, C::SMEM);
    cfg.gridDim = dim3(2);
    int clusters = 0;
    KC_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg));
    if (clusters <= 0) fail(KC_ERR_CUDA, "CUDA backend: no CTA pair of the trunk GEMM fits on this device");
    return clusters;
  }
  cudaLaunchAttribute at2[2] = {at[0], {}};
  at2[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at2[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at2;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cfg.gridDim = dim3(2 * pairs);
  KC_CUDA(cudaLaunchKernelEx(&cfg, kernel, m.a, m.b, m.res, m.raw, m.act, p));
  return pairs;
}

// The chained closing / opening 1x1 kernel of two consecutive nested blocks (gemm_chain.cuh), launched as clusters
// of two CTAs like the pair GEMM; `prepare` returns how many pairs fit on the device at once.
struct ChainMaps {
  CUtensorMap x, w1, w2, trunk, raw2, act2;
};

template <typename T>
int launch_chain(bool prepare, int pairs, cudaStream_t s, const ChainMaps& m, const ChainParams& p) {
  using C = ChainCfg;
  auto kernel = gemm_chain_kernel<T>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (prepare) {
    allow_smem(kernel, C::SMEM);
    cfg.gridDim = dim3(2);
    int clusters = 0;
    KC_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg));
    if (clusters <= 0) fail(KC_ERR_CUDA, "CUDA backend: no CTA pair of the chained 1x1 kernel fits on this device");
    return clusters;
  }
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cfg.gridDim = dim3(2 * pairs);
  KC_CUDA(cudaLaunchKernelEx(&cfg, kernel, m.x, m.w1, m.w2, m.trunk, m.raw2, m.act2, p));
  return pairs;
}

// How a pair launch of `tiles` tiles of width `w` runs on at most `P` pairs: how many pairs, from which work item on
// tiles are column halves (`split`: when the last, partly filled round of tiles then fits one round of half items),
// and its cost in column units: a tile costs about its width plus a fixed ~74 columns' worth (prologue, pipeline
// fill, epilogue), a round the cost of its largest item.
struct PairPlan {
  int pairs, split_from;
  long long cost;
};
PairPlan plan_pair(int tiles, int P, int w, bool split) {
  const int rounds = tiles / P, rem = tiles % P;
  if (split && rem > 0 && 2 * rem <= P) {
    if (rounds == 0) return {2 * rem, 0, w / 2 + 74};
    return {P, rounds * P, rounds * (w + 74LL) + (w / 2 + 74)};
  }
  return {std::min(tiles, P), 1 << 30, (long long)((tiles + P - 1) / P) * (w + 74)};
}

// The pair kernel instances: tile width x (windowed 3x3 | linear | float32 residual | RoPE | SwiGLU), as chosen by
// Impl::pair_tile.
enum PairKind { PAIR_SEG = 0, PAIR_WIN = 1, PAIR_F32 = 2, PAIR_ROPE = 3, PAIR_SWIGLU = 4, PAIR_SEG_NORES = 5 };

template <typename T>
int launch_pair(bool prepare, int bn, int kind, int pairs, cudaStream_t s, const PairMaps& m, const GemmParams& p) {
  const int key = kind * 1000 + bn;
  switch (key) {
    case PAIR_SEG * 1000 + 64: return launch_pair_bn<T, 64, false, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_SEG * 1000 + 128: return launch_pair_bn<T, 128, false, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_SEG * 1000 + 192: return launch_pair_bn<T, 192, false, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_SEG * 1000 + 256: return launch_pair_bn<T, 256, false, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_SEG_NORES * 1000 + 64: return launch_pair_bn<T, 64, false, MODE_SEGMENTS, false, true>(prepare, pairs, s, m, p);
    case PAIR_SEG_NORES * 1000 + 128: return launch_pair_bn<T, 128, false, MODE_SEGMENTS, false, true>(prepare, pairs, s, m, p);
    case PAIR_SEG_NORES * 1000 + 192: return launch_pair_bn<T, 192, false, MODE_SEGMENTS, false, true>(prepare, pairs, s, m, p);
    case PAIR_SEG_NORES * 1000 + 256: return launch_pair_bn<T, 256, false, MODE_SEGMENTS, false, true>(prepare, pairs, s, m, p);
    case PAIR_WIN * 1000 + 64: return launch_pair_bn<T, 64, true, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_WIN * 1000 + 128: return launch_pair_bn<T, 128, true, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_WIN * 1000 + 192: return launch_pair_bn<T, 192, true, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_WIN * 1000 + 256: return launch_pair_bn<T, 256, true, MODE_SEGMENTS, false>(prepare, pairs, s, m, p);
    case PAIR_F32 * 1000 + 128: return launch_pair_bn<T, 128, false, MODE_SEGMENTS, true>(prepare, pairs, s, m, p);
    case PAIR_F32 * 1000 + 192: return launch_pair_bn<T, 192, false, MODE_SEGMENTS, true>(prepare, pairs, s, m, p);
    case PAIR_ROPE * 1000 + 128: return launch_pair_bn<T, 128, false, MODE_ROPE, false>(prepare, pairs, s, m, p);
    case PAIR_ROPE * 1000 + 192: return launch_pair_bn<T, 192, false, MODE_ROPE, false>(prepare, pairs, s, m, p);
    case PAIR_SWIGLU * 1000 + 128: return launch_pair_bn<T, 128, false, MODE_SWIGLU, false>(prepare, pairs, s, m, p);
    case PAIR_SWIGLU * 1000 + 256: return launch_pair_bn<T, 256, false, MODE_SWIGLU, false>(prepare, pairs, s, m, p);
    default:
      fail(KC_ERR_INVALID, "CUDA backend: unsupported pair tile (" + std::to_string(kind) + ", " + std::to_string(bn) + ")");
  }
  return 0;
}

// RoPE tables [tables][361][half] (desc.cpp computeRopeCosSin as restated in bin2onnx.py:449-484: float32 steps,
// cos/sin of the float32 angle evaluated in float64 and rounded).
void rope_tables(const BlockDesc& b, std::vector<float>& cs, std::vector<float>& sn, int& tables) {
  const int half = b.head_dim / 2, P = half;
  if (!b.rope_cos.empty()) {  // tables stored in the file
    tables = b.rope_ntables;
    cs = b.rope_cos;
    sn = b.rope_sin;
    return;
  }
  if (b.learnable_rope) {
    tables = b.kv_heads;
    cs.assign((size_t)tables * 361 * half, 0.0f);
    sn.assign(cs.size(), 0.0f);
    for (int h = 0; h < b.kv_heads; h++)
      for (int p = 0; p < P; p++) {
        float fx = b.rope_freqs[((size_t)h * P + p) * 2], fy = b.rope_freqs[((size_t)h * P + p) * 2 + 1];
        for (int s = 0; s < 361; s++) {
          volatile float ax = (float)(s % 19) * fx;
          volatile float ay = (float)(s / 19) * fy;
          volatile float a = (float)ax + (float)ay;
          cs[((size_t)h * 361 + s) * half + p] = (float)std::cos((double)a);
          sn[((size_t)h * 361 + s) * half + p] = (float)std::sin((double)a);
        }
      }
  } else {
    tables = 1;
    cs.assign((size_t)361 * half, 0.0f);
    sn.assign(cs.size(), 0.0f);
    int ppd = P / 2, dim_half = b.head_dim / 2;
    for (int p = 0; p < P; p++) {
      int padj = p < ppd ? p : p - ppd;
      volatile float expo = (float)(2 * padj) / (float)dim_half;
      float powv = (float)std::pow((double)b.rope_theta, (double)(float)expo);
      volatile float freq = 1.0f / powv;
      for (int s = 0; s < 361; s++) {
        float pos = p < ppd ? (float)(s / 19) : (float)(s % 19);
        volatile float a = pos * (float)freq;
        cs[(size_t)s * half + p] = (float)std::cos((double)a);
        sn[(size_t)s * half + p] = (float)std::sin((double)a);
      }
    }
  }
}

struct BnAct {
  const BNDesc* bn = nullptr;
  Act act = ACT_IDENTITY;
};

bool is_conv_block(const BlockDesc& b) {
  return b.kind == BLOCK_ORDINARY || b.kind == BLOCK_GPOOL || b.kind == BLOCK_NESTED;
}

// The batch norm that the consumer of a block stack's stream applies first: the next block's pre-BN, or `after`.
BnAct consumer_bn(const std::vector<BlockDesc>& v, size_t i, BnAct after) {
  if (i < v.size()) {
    if (is_conv_block(v[i])) return {&v[i].pre_bn, v[i].pre_act};
    return {};
  }
  return after;
}

struct Tensor {
  void* p = nullptr;
  int ld = 0;
  bool f32 = false;  // float32 storage (the residual stream of the bf16 tier) instead of the tier's type
};

}  // namespace

struct Engine::Impl {
  std::vector<void*> allocs;
  int sm_count = 148;
  int R = 0;
  int stem_rows = 0;
  const float* in_spatial = nullptr;
  const uint32_t* in_bits = nullptr;  // bit-packed spatial planes (instead of in_spatial) and their symmetries
  const int* in_sym = nullptr;
  const float* in_global = nullptr;
  const float* in_meta = nullptr;
  float* out = nullptr;
  int* d_err = nullptr;
  float* rowmask = nullptr;
  float* mask_sum = nullptr;
  float* scale1 = nullptr;
  float* scale2 = nullptr;
  float* board_bias = nullptr;
  // Captured forward passes by (batch size and profiling, caller's buffers), least recently used first out of
  // `graph_lru` once more than kMaxGraphs are held (a caller that rotates buffers or batch sizes would otherwise
  // keep one graph per combination). An evicted graph that is still running is freed when it completes.
  using GraphKey = std::tuple<int, const void*, const void*, const void*, const void*, const void*, void*>;
  static constexpr size_t kMaxGraphs = 64;
  std::map<GraphKey, std::pair<cudaGraphExec_t, uint64_t>> graphs;
  uint64_t graph_clock = 0;

  InputSrc input() const {
    InputSrc s;
    s.f = in_bits ? nullptr : in_spatial;
    s.bits = in_bits;
    s.sym = in_sym;
    return s;
  }
  void* alloc(size_t bytes) {
    void* p = nullptr;
    KC_CUDA(cudaMalloc(&p, bytes));
    allocs.push_back(p);
    KC_CUDA(cudaMemset(p, 0, bytes));
    return p;
  }
  template <typename U>
  U* upload(const std::vector<U>& v) {
    if (v.empty()) return nullptr;
    U* p = static_cast<U*>(alloc(v.size() * sizeof(U)));
    KC_CUDA(cudaMemcpy(p, v.data(), v.size() * sizeof(U), cudaMemcpyHostToDevice));
    return p;
  }
  ~Impl() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.second.first);
    for (void* p : allocs) cudaFree(p);
  }
};

// ================================================================================================================
// Plan builder. Runs twice: pass 0 sizes the shared scratch tensors, pass 1 allocates and records launches.
// ================================================================================================================

namespace {

enum Role : int {
  R_T1, R_REG, R_G, R_XN, R_QKV, R_O, R_H, R_AG, R_HEAD, R_P1A, R_STEM, R_TIPH,
  R_LEVEL0 = 16,  // + 2 * depth (+0 stream, +1 act)
  R_COUNT = 32
};
enum FRole : int { F_POOL, F_GBIAS, F_VPOOL, F_V2, F_PASS, F_PIX, F_TIPSS, F_COUNT };

template <typename T>
struct Builder {
  // The heads' operand type: the bf16 tier runs the policy and value heads (under 0.3% of a transformer net's
  // FLOPs) in f16, whose 11-bit significand keeps their rounding, the largest error term of the tier's outputs at
  // bf16, well inside the tier's tolerance; the other tiers use their own type.
  using H = typename std::conditional<std::is_same<T, __nv_bfloat16>::value, __half, T>::type;
  Engine::Impl& I;
  std::vector<Engine::Launch>& plan;
  const ModelDesc& m;
  int max_batch;
  int pass = 0;
  bool tc;
  bool bf16;
  int ld_max[R_COUNT] = {0};
  int rows_of[R_COUNT] = {0};
  Tensor tens[R_COUNT];
  int f_max[F_COUNT] = {0};
  float* fbuf[F_COUNT] = {nullptr};
  int stem_k = 1, stem_pad = 0, stem_stride = 20, stem_brows = 400, stem_cin = 64;

  Builder(Engine::Impl& i, std::vector<Engine::Launch>& pl, const ModelDesc& md, int mb, bool bf)
      : I(i), plan(pl), m(md), max_batch(mb), tc(sizeof(T) == 2), bf16(bf) {}

  int pbl_rows_alloc() const { return round_up(max_batch * 400, 128) + 128; }

  // The residual streams (trunk and nested-block levels) are float32 in the bf16 tier: bf16's 8-bit mantissa
  // would otherwise round every residual add.
  bool is_stream(int role) const { return role >= R_LEVEL0 && (role - R_LEVEL0) % 2 == 0; }

  Tensor tensor(int role, int c) {
    int ld = round_up(std::max(c, 16), 64);
    if (pass == 0) {
      ld_max[role] = std::max(ld_max[role], ld);
      return {};
    }
    if (ld > tens[role].ld) fail(KC_ERR_INVALID, "CUDA backend: internal scratch sizing error");
    return tens[role];
  }
  float* fbuffer(int role, int per_board) {
    if (pass == 0) {
      f_max[role] = std::max(f_max[role], per_board);
      return nullptr;
    }
    return fbuf[role];
  }
  void allocate() {
    for (int r = 0; r < R_COUNT; r++) {
      if (!ld_max[r]) continue;
      int rows = r == R_STEM ? I.stem_rows : I.R;
      tens[r].ld = ld_max[r];
      tens[r].f32 = bf16 && is_stream(r);
      tens[r].p = I.alloc((size_t)rows * ld_max[r] * (tens[r].f32 ? sizeof(float) : sizeof(T)));
      rows_of[r] = rows;
    }
    for (int f = 0; f < F_COUNT; f++)
      if (f_max[f]) fbuf[f] = static_cast<float*>(I.alloc((size_t)max_batch * f_max[f] * sizeof(float)));
  }
  int rows_for(const Tensor& t) const {
    for (int r = 0; r < R_COUNT; r++)
      if (tens[r].p == t.p) return rows_of[r];
    return I.R;
  }

  template <typename U>
  U* up(const std::vector<U>& v) { return pass == 0 ? nullptr : I.upload(v); }

  void add(int cls, std::function<void(cudaStream_t, int)> fn) {
    if (pass == 1) plan.push_back({cls, std::move(fn)});
  }

  // ---- weights ----
  // W [N][taps * cin_pad]: conv (file order [ky][kx][ic][oc]) at output rows [n_off, n_off + oc)
  // W[n_off + o][tap * cin_pad + i] = conv weight (tap = ky * kx_n + kx); cin_pad 0 packs the taps densely
  // (tap * ic + i, the stem's im2col operand)
  static void pack_conv(std::vector<float>& W, int K, int cin_pad, int n_off, const ConvDesc& c) {
    const int stride = cin_pad ? cin_pad : c.ic;
    for (int ky = 0; ky < c.ky; ky++)
      for (int kx = 0; kx < c.kx; kx++)
        for (int i = 0; i < c.ic; i++)
          for (int o = 0; o < c.oc; o++)
            W[(size_t)(n_off + o) * K + (ky * c.kx + kx) * stride + i] =
                c.w[(((size_t)ky * c.kx + kx) * c.ic + i) * c.oc + o];
  }
  static void pack_linear(std::vector<float>& W, int K, int n_off, const MatMulDesc& mm, const int* perm = nullptr,
                          int ncols = -1, int col0 = 0) {
    if (ncols < 0) ncols = mm.oc;
    for (int o = 0; o < ncols; o++)
      for (int i = 0; i < mm.ic; i++)
        W[(size_t)(n_off + o) * K + i] = mm.w[(size_t)i * mm.oc + (perm ? perm[col0 + o] : col0 + o)];
  }

  // ---- GEMM ----
  struct Seg {
    int width = 0;
    int flags = 0;
    int act = 0;
    std::vector<float> scale, bias;
    const float* board_bias = nullptr;
    int ld_bb = 0;
    Tensor res, raw, actout;
    int res_c0 = 0, raw_c0 = 0, act_c0 = 0;
  };

  struct Spec {
    int cls = CLS_LINEAR;
    Tensor A;
    int cin = 0;
    std::vector<int> taps{0};
    int N = 0;
    std::vector<float> W;
    int mode = MODE_SEGMENTS;
    std::vector<Seg> segs;
    bool stem = false;
    // RoPE (MODE_ROPE)
    const float* rope_cos = nullptr;
    const float* rope_sin = nullptr;
    int rope_table_stride = 0, rope_q_cols = 0, rope_rot_cols = 0, head_dim = 0, rope_group = 1;
    // the same tables indexed by board row for the pair kernel: [tables][432][head_dim / 2], rows 400..431
    // repeating rows 0..31, halo rows zero
    const float* rope_cos_rows = nullptr;
    const float* rope_sin_rows = nullptr;
  };

  // Tile width of the CTA-pair kernel for this GEMM, or 0 when the one-CTA kernel must run it; `f32` is set for
  // float32 raw outputs (and residuals). Taken: one or two column segments of 2-byte raw / batch-norm-activation
  // outputs (a 2-byte residual, a per-board bias or a masked accumulator only with one segment), each kind of output
  // in at most one segment, on 32-column-aligned operands; one segment of float32 raw output (+ float32 residual)
  // without an activation output; RoPE Q|K|V linears of head dim 64; SwiGLU linears. KATAGO_CUDA_PAIR=0 sends every
  // GEMM to the one-CTA kernel.
  int pair_tile(const Spec& s, const GemmParams& p, bool& f32) const {
    f32 = false;
    const char* e = std::getenv("KATAGO_CUDA_PAIR");
    if (e && e[0] == '0') return 0;
    if (s.stem || p.nseg < 1 || p.nseg > 2) return 0;
    auto aligned = [](const Tensor& t, int c0) { return !t.p || (t.ld % 32 == 0 && c0 % 32 == 0); };
    if (s.mode == MODE_ROPE || s.mode == MODE_SWIGLU) {
      const Seg& g = s.segs[0];
      if (p.nseg != 1 || g.raw.f32 || !aligned(g.raw, g.raw_c0)) return 0;
      if (s.mode == MODE_ROPE) {
        // one head of 64 per epilogue warp: 192 columns (three warps per lane quarter) or 128 (two)
        if (s.head_dim != 64) return 0;
        for (int bn : {192, 128})
          if (s.N % bn == 0) return bn;
        return 0;
      } else {
        for (int bn : {256, 128})
          if (s.N % bn == 0) return bn;
      }
      return 0;
    }
    if (s.mode != MODE_SEGMENTS) return 0;
    int n_raw = 0, n_act = 0, n_res = 0;
    for (int i = 0; i < p.nseg; i++) {
      const int f = p.seg[i].flags;
      if ((f & ~(EPI_RAW | EPI_ACT | EPI_RESIDUAL | EPI_BOARD_BIAS | EPI_MASK_ACC | EPI_RES_F32 | EPI_RAW_F32)) ||
          !(f & (EPI_RAW | EPI_ACT)))
        return 0;
      // per-board bias: one segment, 16-byte aligned rows (the stem)
      if ((f & EPI_BOARD_BIAS) && (p.nseg != 1 || p.seg[i].ld_bb % 4 != 0)) return 0;
      if ((f & EPI_MASK_ACC) && p.nseg != 1) return 0;
      const Seg& g = s.segs[i];
      if (f & (EPI_RES_F32 | EPI_RAW_F32)) {
        // float32 tile: one segment, raw float32 output, float32 residual if any, no activation output
        const bool res_ok = !(f & EPI_RESIDUAL) || ((f & EPI_RES_F32) && g.res.f32);
        if (p.nseg != 1 || !(f & EPI_RAW_F32) || !g.raw.f32 || (f & EPI_ACT) || !res_ok) return 0;
        f32 = true;
      } else {
        for (const Tensor* t : {&g.res, &g.raw, &g.actout})
          if (t->p && t->f32) return 0;
      }
      n_raw += (f & EPI_RAW) != 0;
      n_act += (f & EPI_ACT) != 0;
      n_res += (f & EPI_RESIDUAL) != 0;
      if (!aligned(g.res, g.res_c0) || !aligned(g.raw, g.raw_c0) || !aligned(g.actout, g.act_c0)) return 0;
    }
    if (n_raw > 1 || n_act > 1 || n_res > 1) return 0;
    if (p.nseg == 2 && (n_res || p.seg[0].n1 % 32)) return 0;
    if (n_act && s.N > PairCfg<256>::PARAM_COLS) return 0;
    // float32 tiles: 256 columns would leave one pipeline stage; a masked accumulator needs a tile of 8 epilogue
    // warps (not the 2-byte 192-wide tile)
    const bool mask_acc = (p.seg[0].flags & EPI_MASK_ACC) != 0;
    for (int bn : {256, 192, 128})
      if (s.N % bn == 0 && !(f32 && bn == 256) && !(mask_acc && !f32 && bn == 192)) return bn;
    return 0;
  }

  static int pick_bn(int N, int mult) {
    const int cands[] = {256, 192, 128, 96, 64, 48, 32, 16};
    for (int c : cands)
      if (N % c == 0 && c % mult == 0) return c;
    return 0;
  }

  // E: the operand type of this GEMM (the tier's type, or __half for the heads of the bf16 tier)
  template <typename E = T>
  void gemm(Spec s) {
    if (pass == 0) return;
    constexpr bool ebf = std::is_same<E, __nv_bfloat16>::value;
    GemmParams p;
    p.n_total = s.N;
    p.cin = s.cin;
    p.taps = (int)s.taps.size();
    for (int i = 0; i < p.taps; i++) p.tap_off[i] = s.taps[i];
    p.mode = s.mode;
    p.nseg = (int)s.segs.size();
    int n0 = 0;
    for (int i = 0; i < p.nseg; i++) {
      Seg& g = s.segs[i];
      EpiSeg& e = p.seg[i];
      e.n0 = n0;
      e.n1 = n0 + g.width;
      n0 = e.n1;
      e.flags = g.flags;
      e.act = g.act;
      if (g.flags & EPI_ACT) {
        g.scale.resize(g.width, 0.0f);
        g.bias.resize(g.width, 0.0f);
        e.scale = up(g.scale);
        e.bias = up(g.bias);
      }
      e.board_bias = g.board_bias;
      e.ld_bb = g.ld_bb;
      e.res = g.res.p;
      e.ld_res = g.res.ld;
      e.res_c0 = g.res_c0;
      e.out_raw = g.raw.p;
      e.ld_raw = g.raw.ld;
      e.raw_c0 = g.raw_c0;
      e.out_act = g.actout.p;
      e.ld_act = g.actout.ld;
      e.act_c0 = g.act_c0;
    }
    if (s.mode == MODE_SEGMENTS && n0 != s.N) fail(KC_ERR_INVALID, "CUDA backend: GEMM segment widths != N");
    for (int i = 0; i < p.nseg; i++)
      if ((p.seg[i].flags & EPI_ACT) && s.N > TcCfg<256>::PARAM_COLS)
        fail(KC_ERR_INVALID, "CUDA backend: batch-norm epilogue on a GEMM wider than 768 columns");
    p.rope_cos = s.rope_cos;
    p.rope_sin = s.rope_sin;
    p.rope_table_stride = s.rope_table_stride;
    p.rope_q_cols = s.rope_q_cols;
    p.rope_rot_cols = s.rope_rot_cols;
    p.head_dim = s.head_dim;
    p.rope_group = s.rope_group;
    p.err = I.d_err;
    if (s.stem) {
      p.g.board_rows = stem_brows;
      p.g.stride = stem_stride;
      p.g.pad = stem_pad;
      p.g.remap = 1;
    }
    p.g.rowmask = I.rowmask;
    const int brows = p.g.board_rows;
    const int a_rows = rows_for(s.A);
    if (s.cin > s.A.ld) fail(KC_ERR_INVALID, "CUDA backend: GEMM reads more channels than its input holds");
    const int K = p.taps * s.cin;
    Engine::Impl* Ip = &I;
    if constexpr (sizeof(E) == 2) {
      // SwiGLU splits each tile's linear1 half between two epilogue warps (BN % 64); RoPE gives each warp whole
      // heads (BN % (2 * head_dim))
      int bn = pick_bn(s.N, s.mode == MODE_SWIGLU ? 64 : s.mode == MODE_ROPE ? 2 * s.head_dim : 16);
      if (!bn) fail(KC_ERR_INVALID, "CUDA backend: no GEMM tile width for N = " + std::to_string(s.N));
      if (s.cin % 64 != 0) fail(KC_ERR_INVALID, "CUDA backend: GEMM input channels not padded");
      bool pf32 = false;
      const int pbn = pair_tile(s, p, pf32);
      // SwiGLU tiles: the weight columns in tiles of the kernel's width
      const int tbn = pbn ? pbn : bn;
      std::vector<float> Wp = s.W;
      if (s.mode == MODE_SWIGLU) {
        // columns [0, F) = linear1, [F, 2F) = gate  ->  per tile of tbn: [tbn/2 linear1 | tbn/2 gate]
        const int F = s.N / 2, hb = tbn / 2;
        for (int t = 0; t < s.N / tbn; t++)
          for (int j = 0; j < hb; j++) {
            std::memcpy(&Wp[(size_t)(t * tbn + j) * K], &s.W[(size_t)(t * hb + j) * K], K * sizeof(float));
            std::memcpy(&Wp[(size_t)(t * tbn + hb + j) * K], &s.W[(size_t)(F + t * hb + j) * K], K * sizeof(float));
          }
      }
      std::vector<E> Wt(Wp.size());
      for (size_t i = 0; i < Wp.size(); i++) Wt[i] = E(Wp[i]);
      E* dW = up(Wt);
      if (pbn) {
        // CTA-pair kernel with TMA-staged epilogue boxes (the trunk's convolutions, the token linears); the raw,
        // act and residual boxes each come from the (single) segment that has them
        const Tensor *raw = nullptr, *act = nullptr, *res = nullptr;
        p.pair_split = p.nseg > 1 ? p.seg[0].n1 : p.n_total;
        if (s.mode != MODE_SEGMENTS) raw = &s.segs[0].raw, p.pair_raw_x = s.segs[0].raw_c0;  // RoPE / SwiGLU
        for (int i = 0; i < p.nseg; i++) {
          const Seg& g = s.segs[i];
          const int n0 = p.seg[i].n0;
          if (p.seg[i].flags & EPI_RAW) raw = &g.raw, p.pair_raw_x = g.raw_c0 - n0;
          if (p.seg[i].flags & EPI_ACT) act = &g.actout, p.pair_act_x = g.act_c0 - n0;
          if (p.seg[i].flags & EPI_RESIDUAL) res = &g.res, p.pair_res_x = g.res_c0 - n0;
        }
        const Tensor& out0 = raw ? *raw : *act;
        auto box = [&](const Tensor* t) { return make_box_map(t ? t->p : out0.p, ebf, t ? t->ld : out0.ld,
                                                              rows_for(t ? *t : out0), t && t->f32); };
        // 3x3 convolutions read one A window per 64-channel chunk (KATAGO_CUDA_PAIR_WIN=0: one A tile per tap)
        const char* pw = std::getenv("KATAGO_CUDA_PAIR_WIN");
        bool pwin = p.taps == PairCfg<256, true>::WIN_TAPS && !pf32 && !(pw && pw[0] == '0');
        if (pwin) {
          int halo = 0;
          for (int i = 0; i < p.taps; i++) halo = std::max(halo, std::abs(p.tap_off[i]));
          p.halo = halo;
          p.win_rows = round_up(128 + 2 * halo, 8);
          if (p.win_rows > PairCfg<256, true>::WIN_MAX_ROWS) pwin = false;
        }
        // linears and 1x1 convolutions without a residual: the instance without residual boxes (a deeper pipeline;
        // KATAGO_CUDA_PAIR_NORES=0: the general one)
        const char* nr = std::getenv("KATAGO_CUDA_PAIR_NORES");
        bool any_res = false;
        for (int i = 0; i < p.nseg; i++) any_res = any_res || (p.seg[i].flags & EPI_RESIDUAL);
        const bool nores = !any_res && !(nr && nr[0] == '0');
        const int kind = s.mode == MODE_ROPE ? PAIR_ROPE : s.mode == MODE_SWIGLU ? PAIR_SWIGLU : pf32 ? PAIR_F32
                         : pwin ? PAIR_WIN : nores ? PAIR_SEG_NORES : PAIR_SEG;
        const bool kwin = kind == PAIR_WIN, knores = kind == PAIR_SEG_NORES;
        PairMaps pm;
        pm.a = make_map(s.A.p, ebf, s.A.ld, a_rows, pwin ? p.win_rows : 128);
        pm.b = make_map(dW, ebf, K, s.N, pair_b_box_rows(pbn, kwin, knores));
        pm.res = box(res);
        pm.raw = box(raw);
        pm.act = box(act);
        if (kind == PAIR_ROPE) {
          p.rope_cos = s.rope_cos_rows;
          p.rope_sin = s.rope_sin_rows;
          p.rope_table_stride = s.rope_table_stride ? 432 * (s.head_dim / 2) : 0;
        }
        const int max_pairs = launch_pair<E>(true, pbn, kind, 0, 0, pm, p);
        // Small batches: the convolutions also get 64-column tiles (three or six per row tile instead of one or two)
        // when that spreads a launch over more SM pairs than it adds tile rounds (KATAGO_CUDA_PAIR_NARROW=0: off).
        // A tile costs about its width plus a fixed ~74 columns' worth (prologue, pipeline fill, epilogue).
        const char* ne = std::getenv("KATAGO_CUDA_PAIR_NARROW");
        const bool narrow = (kind == PAIR_SEG || kind == PAIR_SEG_NORES || kind == PAIR_WIN) && pbn > 64 && s.N % 64 == 0 &&
                            !(ne && ne[0] == '0');
        PairMaps pm64 = pm;
        int max_pairs64 = 0;
        if (narrow) {
          pm64.b = make_map(dW, ebf, K, s.N, pair_b_box_rows(64, kwin, knores));
          max_pairs64 = launch_pair<E>(true, 64, kind, 0, 0, pm64, p);
        }
        // windowed and residual-free tiles: the last, partly filled round as column halves (KATAGO_CUDA_PAIR_SPLIT=0:
        // off)
        const char* se = std::getenv("KATAGO_CUDA_PAIR_SPLIT");
        const bool split = pair_split_tiles(pbn, kwin, knores) && !(se && se[0] == '0');
        add(s.cls, [=](cudaStream_t st, int n) {
          GemmParams q = p;
          q.g.rows = n * brows;
          const int mt = (q.g.rows + 255) / 256;
          const PairPlan pl = plan_pair(mt * (q.n_total / pbn), max_pairs, pbn, split);
          if (narrow) {
            const PairPlan pl64 = plan_pair(mt * (q.n_total / 64), max_pairs64, 64, false);
            if (pl64.cost < pl.cost) {
              launch_pair<E>(false, 64, kind, pl64.pairs, st, pm64, q);
              return;
            }
          }
          q.split_from = pl.split_from;
          launch_pair<E>(false, pbn, kind, pl.pairs, st, pm, q);
        });
        return;
      }
      CUtensorMap ta = make_map(s.A.p, ebf, s.A.ld, a_rows, 128);
      CUtensorMap tb = make_map(dW, ebf, K, s.N, bn);
      bool rf32 = false;
      for (int i = 0; i < p.nseg; i++) rf32 = rf32 || (p.seg[i].flags & EPI_RES_F32);
      launch_tc<E>(true, rf32, bn, 0, 0, ta, tb, p);
      add(s.cls, [=](cudaStream_t st, int n) {
        GemmParams q = p;
        q.g.rows = n * brows;
        int tiles = ((q.g.rows + 127) / 128) * (q.n_total / bn);
        int grid = std::min(tiles, Ip->sm_count);
        launch_tc<E>(false, rf32, bn, grid, st, ta, tb, q);
      });
    } else {
      p.a = s.A.p;
      p.lda = s.A.ld;
      p.a_rows = a_rows;
      p.w = up(s.W);
      if (s.mode != MODE_SEGMENTS) fail(KC_ERR_INVALID, "CUDA backend: fused SwiGLU/RoPE needs the tensor-core path");
      if (s.A.ld % 4 != 0 || s.cin % 16 != 0 || reinterpret_cast<uintptr_t>(s.A.p) % 16 != 0)
        fail(KC_ERR_INVALID, "CUDA backend: float32 GEMM operand not 16-byte aligned");
      add(s.cls, [=](cudaStream_t st, int n) {
        GemmParams q = p;
        q.g.rows = n * brows;
        dim3 grid((q.g.rows + 63) / 64, (q.n_total + 63) / 64);
        launch_pdl(gemm_simt_kernel<E>, dim3(grid), dim3(SIMT_THREADS), 0, st, q);
      });
    }
  }

  std::vector<int> taps_pbl(int k) {
    std::vector<int> t;
    for (int ky = 0; ky < k; ky++)
      for (int kx = 0; kx < k; kx++) t.push_back((ky - k / 2) * 20 + (kx - k / 2));
    return t;
  }

  void check_conv(const ConvDesc& c) {
    if (!((c.ky == 1 && c.kx == 1) || (c.ky == 3 && c.kx == 3)) || c.dy != 1 || c.dx != 1)
      fail(KC_ERR_INVALID, "CUDA backend: " + c.name + ": only 1x1 and 3x3 undilated convolutions are supported "
                           "inside the trunk and heads");
  }

  // conv from A (channels cin) into segments; returns the Spec with W packed
  Spec conv_spec(int cls, Tensor A, int cin, const std::vector<const ConvDesc*>& convs, std::vector<Seg> segs) {
    Spec s;
    s.cls = cls;
    s.A = A;
    s.cin = round_up(cin, tc ? 64 : 16);
    int k = convs[0]->ky;
    for (auto* c : convs) {
      check_conv(*c);
      if (c->ky != k) fail(KC_ERR_INVALID, "CUDA backend: fused convolutions differ in size");
    }
    s.taps = taps_pbl(k);
    s.N = 0;
    for (auto& g : segs) s.N += g.width;
    const int K = (int)s.taps.size() * s.cin;
    if (pass == 1) {
      s.W.assign((size_t)s.N * K, 0.0f);
      int off = 0;
      for (size_t i = 0; i < convs.size(); i++) {
        pack_conv(s.W, K, s.cin, off, *convs[i]);
        off += segs[i].width;
      }
    }
    s.segs = std::move(segs);
    return s;
  }

  static int w16(int c) { return round_up(c, 16); }

  Seg act_seg(int width, const BNDesc& bn, Act act, Tensor out, int c0 = 0) {
    Seg g;
    g.width = width;
    g.flags = EPI_ACT;
    g.act = act;
    g.scale = bn.merged_scale;
    g.bias = bn.merged_bias;
    g.actout = out;
    g.act_c0 = c0;
    return g;
  }
  // residual-closing segment: y = acc (* mask) + X; X = y; XA = act(next(y)). raw_live false: nothing reads X
  // after this block (the last block of a nested block's inner stack, whose closing 1x1 reads only XA), so y is
  // not written back when XA is (2-byte residual streams).
  Seg close_seg(int width, Tensor X, Tensor XA, BnAct next, bool mask_acc, bool raw_live = true) {
    Seg g;
    g.width = width;
    const bool raw = raw_live || !next.bn || X.f32;
    g.flags = EPI_RESIDUAL | (raw ? EPI_RAW : 0) | (mask_acc ? EPI_MASK_ACC : 0) |
              (X.f32 ? EPI_RES_F32 | EPI_RAW_F32 : 0);
    g.res = X;
    if (raw) g.raw = X;
    if (next.bn) {
      g.flags |= EPI_ACT;
      g.act = next.act;
      g.scale = next.bn->merged_scale;
      g.bias = next.bn->merged_bias;
      g.actout = XA;
    }
    return g;
  }

  // ---- elementwise / reduction launches ----
  template <typename TI = T, typename TO = T>
  void bias_bnact(Tensor x, int xc0, const float* board_bias, const BNDesc& bn, Act act, int C, Tensor y) {
    const float* sc = up(bn.merged_scale);
    const float* bi = up(bn.merged_bias);
    Engine::Impl* Ip = &I;
    // written width: the channels plus the zero padding a consumer GEMM reads (its input channels are padded to a
    // multiple of 64), not the whole row of the shared buffer
    const int Cw = std::min(y.ld, round_up(C, 64));
    if (xc0 % 8 != 0 || x.ld % 8 != 0 || Cw % 8 != 0)
      fail(KC_ERR_INVALID, "CUDA backend: biased batch-norm pass on unaligned channels");
    add(CLS_OTHER, [=](cudaStream_t st, int n) {
      const int rows = n * 400;
      const unsigned blocks = (unsigned)(((size_t)rows * (Cw / 8) + 255) / 256);
      auto go = [&](auto kernel) {
        launch_pdl(kernel, dim3(blocks), dim3(256), 0, st, (const TI*)x.p, x.ld, xc0, board_bias, sc, bi, Ip->rowmask,
                   rows, C, Cw, (TO*)y.p, y.ld);
      };
      switch (act) {
        case 1: go(bias_bnact_kernel<TI, TO, 1>); break;
        case 2: go(bias_bnact_kernel<TI, TO, 2>); break;
        case 3: go(bias_bnact_kernel<TI, TO, 3>); break;
        default: go(bias_bnact_kernel<TI, TO, 0>); break;
      }
    });
  }
  template <typename E = T>
  void pool(Tensor x, int c0, int C, bool value_mode, float* out) {
    Engine::Impl* Ip = &I;
    const int CG = (C + 7) / 8;
    if (CG > POOL_THREADS || c0 % 8 != 0 || x.ld % 8 != 0)
      fail(KC_ERR_INVALID, "CUDA backend: pooled channels unaligned or too many");
    const int smem = 2 * (POOL_THREADS / CG) * CG * 8 * (int)sizeof(float);
    add(CLS_OTHER, [=](cudaStream_t st, int n) {
      launch_pdl(pool_kernel<E>, dim3(n), dim3(POOL_THREADS), smem, st, (const E*)x.p, x.ld, c0, C, Ip->rowmask, Ip->mask_sum,
                                                    Ip->scale1, Ip->scale2, value_mode ? 1 : 0, out);
    });
  }
  // The gpool block's pooling, bias matmul and biased batch-norm + activation as one launch per board
  // (gpool_mid_kernel), bit-identical to the three launches it replaces; false where its shapes do not fit (the
  // caller then emits pool, fc and bias_bnact). KATAGO_CUDA_GPOOL_FUSED=0: always the three launches. Each board's
  // columns are shared out over S blocks so that a launch has at least one block per SM (S = 1 from one board per
  // SM up: at batch 256, two groups per board took 0.40 ms of a b18 step against 0.37 ms with one);
  // KATAGO_CUDA_GPOOL_GROUPS=k fixes S at k (tests: the outputs do not depend on it).
  bool gpool_mid(Tensor G, int gc, Tensor REG, int rc, const MatMulDesc& mm, const BNDesc& bn, Act act, Tensor y) {
    const char* e = std::getenv("KATAGO_CUDA_GPOOL_FUSED");
    if (e && e[0] == '0') return false;
    if (gc % 8 || rc % 8 || G.ld % 8 || REG.ld % 8 || y.ld % 8 || mm.ic != 3 * gc || mm.oc != rc ||
        (gc + 7) / 8 > POOL_THREADS)
      return false;
    const int smem = (pool_red_floats(gc) + 3 * gc + 9 * rc) * (int)sizeof(float);
    if (smem > 227 * 1024) return false;
    if (pass == 0) return true;
    const float* w = up(mm.w);
    const float* sc = up(bn.merged_scale);
    const float* sh = up(bn.merged_bias);
    const int cw = std::min(y.ld, round_up(rc, 64));
    auto kernel_for = [](Act a) {
      switch (a) {
        case 1: return gpool_mid_kernel<T, 1>;
        case 2: return gpool_mid_kernel<T, 2>;
        case 3: return gpool_mid_kernel<T, 3>;
        default: return gpool_mid_kernel<T, 0>;
      }
    };
    auto kernel = kernel_for(act);
    if (smem > 48 * 1024) allow_smem(kernel, smem);
    Engine::Impl* Ip = &I;
    const char* ge = std::getenv("KATAGO_CUDA_GPOOL_GROUPS");
    const int groups = ge ? std::atoi(ge) : 0;
    add(CLS_OTHER, [=](cudaStream_t st, int n) {
      const int per_row = cw / 8;
      int S = groups > 0 ? groups : (Ip->sm_count + n - 1) / n;
      S = std::max(1, std::min(S, per_row));
      GpoolMidParams q;
      q.g = G.p, q.ld_g = G.ld, q.gc = gc;
      q.reg = REG.p, q.ld_reg = REG.ld, q.rc = rc;
      q.w = w, q.scale = sc, q.shift = sh;
      q.rowmask = Ip->rowmask, q.mask_sum = Ip->mask_sum, q.scale1 = Ip->scale1, q.scale2 = Ip->scale2;
      q.y = y.p, q.ld_y = y.ld, q.cw = cw;
      launch_pdl(kernel, dim3(n, S), dim3(POOL_THREADS), smem, st, q);
    });
    return true;
  }
  void fc(const float* in, int in_ld, const MatMulDesc& mm, const MatBiasDesc* mb, Act act, float* out, int out_ld,
          int out_off, int out_stride) {
    const float* w = up(mm.w);
    const float* b = mb ? up(mb->b) : nullptr;
    const int ic = mm.ic, oc = mm.oc;
    const int smem = FC_BOARDS * ic * (int)sizeof(float);
    if (smem > 227 * 1024) fail(KC_ERR_INVALID, "CUDA backend: head matmul input too wide");
    if (smem > 48 * 1024) allow_smem(fc_kernel<FC_BOARDS>, smem);
    Engine::Impl* Ip = &I;
    const bool to_out = out == nullptr;  // null = the forward's output rows
    add(CLS_OTHER, [=](cudaStream_t st, int n) {
      float* o = to_out ? Ip->out : out;
      launch_pdl(fc_kernel<FC_BOARDS>, dim3((n + FC_BOARDS - 1) / FC_BOARDS, (oc + 31) / 32), dim3(FC_THREADS), smem, st, in, in_ld, ic, w, oc, b, act, o, out_ld, out_off,
                                                                    out_stride, n);
    });
  }
  // The row RMSNorm kernel with 128-bit loads takes C = 128 k channels (k <= 8) on 4-element-aligned rows.
  static bool rms_vec(Tensor x, int C, Tensor y) {
    return C % 128 == 0 && C <= 1024 && x.ld % 4 == 0 && y.ld % 4 == 0;
  }

  void rmsnorm(Tensor x, int C, const TfRmsDesc& d, Tensor y) {
    const float* w = up(d.w);
    float eps = d.eps;
    Engine::Impl* Ip = &I;
    if (rms_vec(x, C, y)) {
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        const int rows = n * 400;
        if (x.f32)
          launch_pdl(rms_rows_kernel<float, T, false>, dim3((rows + 7) / 8), dim3(256), 0, st, (const float*)x.p,
                     x.ld, C / 128, w, (const float*)nullptr, 0, eps, Ip->rowmask, rows, (T*)y.p, y.ld);
        else
          launch_pdl(rms_rows_kernel<T, T, false>, dim3((rows + 7) / 8), dim3(256), 0, st, (const T*)x.p, x.ld,
                     C / 128, w, (const float*)nullptr, 0, eps, Ip->rowmask, rows, (T*)y.p, y.ld);
      });
      return;
    }
    add(CLS_OTHER, [=](cudaStream_t st, int n) {
      int rows = n * 400;
      if (x.f32)
        launch_pdl(rmsnorm_kernel<float, T>, dim3((rows + 7) / 8), dim3(256), 0, st, (const float*)x.p, x.ld, C, w, eps, Ip->rowmask, rows,
                                                                (T*)y.p, y.ld);
      else
        launch_pdl(rmsnorm_kernel<T, T>, dim3((rows + 7) / 8), dim3(256), 0, st, (const T*)x.p, x.ld, C, w, eps, Ip->rowmask, rows,
                                                            (T*)y.p, y.ld);
    });
  }

  // ---- blocks ----
  // raw_live: whether the stack's residual stream is read after its last block
  void emit_stack(const std::vector<BlockDesc>& v, int depth, int C, BnAct after, bool raw_live = true) {
    bool pre_done = false;
    for (size_t i = 0; i < v.size(); i++)
      pre_done = emit_block(v[i], depth, C, consumer_bn(v, i + 1, after), i + 1 < v.size() || raw_live, pre_done,
                            i + 1 < v.size() ? &v[i + 1] : nullptr);
  }

  // A nested block's closing 1x1 and the next nested block's opening 1x1 as one launch (gemm_chain_kernel): the
  // trunk's batch norm + activation for the opening (XA) stays in tensor memory instead of a 384-channel HBM write
  // and read per boundary. Taken for the 2-byte tiers' 384-channel trunks with 192-channel bottlenecks (the
  // b18c384nbt shape) when a batch has at least half as many 256-row tiles as SM pairs: below that the two separate
  // launches, whose narrow tiles spread over more pairs, are faster (batch 1: 804 against 764 evals/s, batch 8:
  // 5,928 against 5,821; batch 32: 18,090 against 18,926), so both are built and each forward picks one.
  // KATAGO_CUDA_CHAIN=0: always the two launches. Returns whether it emitted the boundary.
  bool chain_boundary(const BlockDesc& b, const BlockDesc& nb, int depth, int C, BnAct next, Tensor X, Tensor XA,
                      Tensor MA) {
    if constexpr (sizeof(T) != 2) {
      return false;
    } else {
      const char* e = std::getenv("KATAGO_CUDA_CHAIN");
      if (pass == 0 || !tc || (e && e[0] == '0')) return false;
      using CC = ChainCfg;
      const ConvDesc &c1 = b.post_conv, &c2 = nb.pre_conv;
      if (nb.kind != BLOCK_NESTED || C != CC::N1 || c1.ky != 1 || c1.kx != 1 || c2.ky != 1 || c2.kx != 1 ||
          c1.ic != CC::K1 || c1.oc != CC::N1 || c2.ic != CC::K2 || c2.oc != CC::N2)
        return false;
      const BnAct first = consumer_bn(nb.inner, 0, {&nb.post_bn, nb.post_act});
      if (!next.bn || !first.bn) return false;
      Tensor M2 = tensor(R_LEVEL0 + 2 * (depth + 1), c2.oc);
      Tensor MA2 = tensor(R_LEVEL0 + 2 * (depth + 1) + 1, c2.oc);
      if (X.f32 || MA.f32 || M2.f32 || MA2.f32 || MA.ld % 64 || X.ld % 32 || M2.ld % 32 || MA2.ld % 32) return false;
      // the weights as the separate launches pack them: [384][192] and [192][384], K-major
      std::vector<float> W1((size_t)CC::N1 * CC::K1, 0.0f), W2((size_t)CC::N2 * CC::K2, 0.0f);
      pack_conv(W1, CC::K1, CC::K1, 0, c1);
      pack_conv(W2, CC::K2, CC::K2, 0, c2);
      std::vector<T> w1(W1.size()), w2(W2.size());
      for (size_t i = 0; i < W1.size(); i++) w1[i] = T(W1[i]);
      for (size_t i = 0; i < W2.size(); i++) w2[i] = T(W2[i]);
      std::vector<float> sc1 = next.bn->merged_scale, bi1 = next.bn->merged_bias;
      std::vector<float> sc2 = first.bn->merged_scale, bi2 = first.bn->merged_bias;
      sc1.resize(CC::N1, 0.0f);
      bi1.resize(CC::N1, 0.0f);
      sc2.resize(CC::N2, 0.0f);
      bi2.resize(CC::N2, 0.0f);
      ChainParams cp = {};
      cp.rowmask = I.rowmask;
      cp.err = I.d_err;
      cp.scale1 = up(sc1);
      cp.bias1 = up(bi1);
      cp.act1 = next.act;
      cp.scale2 = up(sc2);
      cp.bias2 = up(bi2);
      cp.act2 = first.act;
      constexpr bool ebf = std::is_same<T, __nv_bfloat16>::value;
      ChainMaps cm;
      cm.x = make_map(MA.p, ebf, MA.ld, rows_for(MA), 128);
      cm.w1 = make_map(up(w1), ebf, CC::K1, CC::N1, 96);
      cm.w2 = make_map(up(w2), ebf, CC::K2, CC::N2, 96);
      cm.trunk = make_box_map(X.p, ebf, X.ld, rows_for(X));
      cm.raw2 = make_box_map(M2.p, ebf, M2.ld, rows_for(M2));
      cm.act2 = make_box_map(MA2.p, ebf, MA2.ld, rows_for(MA2));
      const int max_pairs = launch_chain<T>(true, 0, 0, cm, cp);
      // the two separate launches (as emit_block would record them), taken out of the plan for small batches
      const size_t mark = plan.size();
      gemm(conv_spec(CLS_LINEAR, MA, c1.ic, {&c1}, {close_seg(w16(C), X, XA, next, false)}));
      Seg so;
      so.width = w16(c2.oc);
      so.flags = EPI_RAW | EPI_ACT;
      so.raw = M2;
      so.act = first.act;
      so.scale = first.bn->merged_scale;
      so.bias = first.bn->merged_bias;
      so.actout = MA2;
      gemm(conv_spec(CLS_LINEAR, XA, C, {&c2}, {so}));
      std::vector<std::function<void(cudaStream_t, int)>> sep;
      for (size_t i = mark; i < plan.size(); i++) sep.push_back(plan[i].fn);
      plan.resize(mark);
      auto chained = [max_pairs](int n) { return 2 * ((n * 400 + 255) / 256) >= max_pairs; };
      add(CLS_LINEAR, [=](cudaStream_t st, int n) {
        ChainParams q = cp;
        q.rows = n * 400;
        const int tiles = (q.rows + 255) / 256;
        if (chained(n)) {
          launch_chain<T>(false, std::min(tiles, max_pairs), st, cm, q);
        } else {
          for (const auto& f : sep) f(st, n);
        }
      });
      const int n_sep = (int)sep.size();
      plan.back().kernels = [chained, n_sep](int n) { return chained(n) ? 1 : n_sep; };
      return true;
    }
  }

  // Returns whether the next block's opening 1x1 was emitted with this block's closing one (pre_done for it).
  bool emit_block(const BlockDesc& b, int depth, int C, BnAct next, bool raw_live = true, bool pre_done = false,
                  const BlockDesc* nb = nullptr) {
    Tensor X = tensor(R_LEVEL0 + 2 * depth, C);
    Tensor XA = tensor(R_LEVEL0 + 2 * depth + 1, C);
    if (b.kind == BLOCK_ORDINARY) {
      // bin2onnx.py residual_block :1243-1248
      Tensor T1 = tensor(R_T1, b.regular.oc);
      gemm(conv_spec(CLS_CONV3, XA, C, {&b.regular}, {act_seg(w16(b.regular.oc), b.mid_bn, b.mid_act, T1)}));
      gemm(conv_spec(b.final_conv.ky == 3 ? CLS_CONV3 : CLS_LINEAR, T1, b.final_conv.ic, {&b.final_conv},
                     {close_seg(w16(C), X, XA, next, false, raw_live)}));
    } else if (b.kind == BLOCK_GPOOL) {
      // bin2onnx.py gpool_block :1250-1261: regular and gpool convs share one GEMM
      const int rc = b.regular.oc, gc = b.gpool_conv.oc;
      Tensor REG = tensor(R_REG, rc), G = tensor(R_G, gc), T1 = tensor(R_T1, rc);
      Seg s0;
      s0.width = w16(rc);
      s0.flags = EPI_RAW;
      s0.raw = REG;
      gemm(conv_spec(CLS_CONV3, XA, C, {&b.regular, &b.gpool_conv},
                     {s0, act_seg(w16(gc), b.gpool_bn, b.gpool_act, G)}));
      if (!gpool_mid(G, gc, REG, rc, b.gpool_to_bias, b.mid_bn, b.mid_act, T1)) {
        float* pooled = fbuffer(F_POOL, 3 * gc);
        float* gbias = fbuffer(F_GBIAS, rc);
        pool(G, 0, gc, false, pooled);
        fc(pooled, 3 * gc, b.gpool_to_bias, nullptr, ACT_IDENTITY, gbias, rc, 0, 1);
        bias_bnact(REG, 0, gbias, b.mid_bn, b.mid_act, rc, T1);
      }
      gemm(conv_spec(CLS_CONV3, T1, rc, {&b.final_conv}, {close_seg(w16(C), X, XA, next, false, raw_live)}));
    } else if (b.kind == BLOCK_NESTED) {
      // bin2onnx.py nested_bottleneck_block :1263-1269
      const int mid = b.pre_conv.oc;
      Tensor M = tensor(R_LEVEL0 + 2 * (depth + 1), mid);
      Tensor MA = tensor(R_LEVEL0 + 2 * (depth + 1) + 1, mid);
      BnAct first = consumer_bn(b.inner, 0, {&b.post_bn, b.post_act});
      Seg s;
      s.width = w16(mid);
      s.flags = EPI_RAW | (M.f32 ? EPI_RAW_F32 : 0);
      s.raw = M;
      if (first.bn) {
        s.flags |= EPI_ACT;
        s.act = first.act;
        s.scale = first.bn->merged_scale;
        s.bias = first.bn->merged_bias;
        s.actout = MA;
      }
      if (!pre_done) gemm(conv_spec(CLS_LINEAR, XA, C, {&b.pre_conv}, {s}));
      emit_stack(b.inner, depth + 1, mid, {&b.post_bn, b.post_act}, false);
      if (nb && raw_live && chain_boundary(b, *nb, depth, C, next, X, XA, MA)) return true;
      gemm(conv_spec(CLS_LINEAR, MA, mid, {&b.post_conv}, {close_seg(w16(C), X, XA, next, false, raw_live)}));
    } else if (b.kind == BLOCK_ATTENTION) {
      emit_attention(b, X, XA, C, next);
    } else {
      emit_ffn(b, X, XA, C, next);
    }
    return false;
  }

  void emit_attention(const BlockDesc& b, Tensor X, Tensor XA, int C, BnAct next) {
    // bin2onnx.py transformer_attention_block :1359-1423
    const int nh = b.heads, nkv = b.kv_heads, hd = b.head_dim, vhd = b.v_head_dim;
    if (vhd != hd) fail(KC_ERR_INVALID, "CUDA backend: " + b.name + ": vHeadDim != qHeadDim is not supported");
    if (hd != 16 && hd != 32 && hd != 64)
      fail(KC_ERR_INVALID, "CUDA backend: " + b.name + ": head dim must be 16, 32 or 64");
    const int qc = nh * hd, kc = nkv * hd, vc = nkv * vhd, N = qc + kc + vc;
    Tensor XN = tensor(R_XN, C), QKV = tensor(R_QKV, N), O = tensor(R_O, nh * vhd);
    rmsnorm(X, C, b.ln, XN);
    // Q and K columns permuted per head to [x0 of each pair..., x1 of each pair...] (bin2onnx.py :1369-1374)
    std::vector<int> pq, pk;
    for (int h = 0; h < nh; h++) {
      for (int j = 0; j < hd; j += 2) pq.push_back(h * hd + j);
      for (int j = 1; j < hd; j += 2) pq.push_back(h * hd + j);
    }
    for (int h = 0; h < nkv; h++) {
      for (int j = 0; j < hd; j += 2) pk.push_back(h * hd + j);
      for (int j = 1; j < hd; j += 2) pk.push_back(h * hd + j);
    }
    Spec s;
    s.cls = CLS_LINEAR;
    s.A = XN;
    s.cin = round_up(C, tc ? 64 : 16);
    s.N = N;
    if (pass == 1) {
      const int K = s.cin;
      s.W.assign((size_t)N * K, 0.0f);
      pack_linear(s.W, K, 0, b.q, b.use_rope ? pq.data() : nullptr);
      pack_linear(s.W, K, qc, b.k, b.use_rope ? pk.data() : nullptr);
      pack_linear(s.W, K, qc + kc, b.v);
    }
    const float* dcos = nullptr;
    const float* dsin = nullptr;
    const float* dcos_rows = nullptr;
    const float* dsin_rows = nullptr;
    int tables = 1;
    if (b.use_rope) {
      std::vector<float> cs, sn;
      rope_tables(b, cs, sn, tables);
      dcos = up(cs);
      dsin = up(sn);
      // board-row-indexed copies (the pair kernel's RoPE epilogue loads 32 consecutive rows per warp)
      const int half = hd / 2;
      std::vector<float> cr((size_t)tables * 432 * half, 0.0f), sr(cr.size(), 0.0f);
      for (int t = 0; t < tables; t++)
        for (int pr = 0; pr < 432; pr++) {
          const int rr = pr % 400, y = rr / 20 - 1, x = rr % 20;
          if (y < 0 || y >= 19 || x >= 19) continue;
          const size_t src = ((size_t)t * 361 + y * 19 + x) * half, dst = ((size_t)t * 432 + pr) * half;
          std::copy(cs.begin() + src, cs.begin() + src + half, cr.begin() + dst);
          std::copy(sn.begin() + src, sn.begin() + src + half, sr.begin() + dst);
        }
      dcos_rows = up(cr);
      dsin_rows = up(sr);
    }
    const int tstride = b.use_rope && b.learnable_rope ? 361 * (hd / 2) : 0;
    const bool fuse_rope = tc && b.use_rope && hd % 32 == 0 && pick_bn(N, 2 * hd) != 0;
    if (fuse_rope) {
      s.mode = MODE_ROPE;
      Seg g;
      g.width = N;
      g.raw = QKV;
      s.segs = {g};
      s.rope_cos = dcos;
      s.rope_sin = dsin;
      s.rope_cos_rows = dcos_rows;
      s.rope_sin_rows = dsin_rows;
      s.rope_table_stride = tstride;
      s.rope_q_cols = qc;
      s.rope_rot_cols = qc + kc;
      s.head_dim = hd;
      s.rope_group = nh / nkv;
    } else {
      Seg g;
      g.width = N;
      g.flags = EPI_RAW;
      g.raw = QKV;
      s.segs = {g};
    }
    gemm(std::move(s));
    Engine::Impl* Ip = &I;
    if (b.use_rope && !fuse_rope) {
      const int group = nh / nkv;
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        int rows = n * 400;
        size_t total = (size_t)rows * ((qc + kc) / 2);
        launch_pdl(rope_kernel<T>, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, (T*)QKV.p, QKV.ld, qc, kc, hd, dcos, dsin,
                                                                        tstride, group, rows);
      });
    }
    // attention
    const float scale = 1.0f / std::sqrt((float)hd);
    if constexpr (sizeof(T) == 2) {
      const char* te = std::getenv("KATAGO_CUDA_TC_ATTN");
      if (hd == 64 && vhd == 64 && !(te && te[0] == '0')) {
        // tensor-core attention (attention.cuh): Q, K and V tiles straight from the QKV rows by TMA
        // (KATAGO_CUDA_TC_ATTN=0: the CUDA-core attention kernel below)
        if (pass == 1) {
          const int qkv_rows = rows_for(QKV);
          CUtensorMap tq = make_map(QKV.p, bf16, QKV.ld, qkv_rows, 128);
          CUtensorMap tk = make_map(QKV.p, bf16, QKV.ld, qkv_rows, 208);
          CUtensorMap tv = make_map(QKV.p, bf16, QKV.ld, qkv_rows, 224);
          AttnParams ap;
          ap.qc = qc;
          ap.kc = kc;
          ap.heads = nh;
          ap.kv_heads = nkv;
          ap.scale = scale;
          ap.rowmask = I.rowmask;
          ap.out = O.p;
          ap.out_ld = O.ld;
          ap.err = I.d_err;
          allow_smem(attention_tc_kernel<T>, AttnCfg::SMEM);
          add(CLS_ATTN, [=](cudaStream_t st, int n) {
            launch_pdl(attention_tc_kernel<T>, dim3(nh, n), dim3(AttnCfg::THREADS), AttnCfg::SMEM, st, tq, tk, tv, ap);
          });
        }
        Spec so;
        so.cls = CLS_LINEAR;
        so.A = O;
        so.cin = round_up(nh * vhd, 64);
        so.N = w16(C);
        if (pass == 1) {
          so.W.assign((size_t)so.N * so.cin, 0.0f);
          pack_linear(so.W, so.cin, 0, b.out);
        }
        so.segs = {close_seg(w16(C), X, XA, next, true)};
        gemm(std::move(so));
        return;
      }
    }
    if (pass == 1) {
      const int smem_need = 361 * hd * (int)sizeof(T) * 2 + 361 * (int)sizeof(float);
      if (hd == 16) allow_smem(attention_simt_kernel<T, 16>, smem_need);
      else if (hd == 32) allow_smem(attention_simt_kernel<T, 32>, smem_need);
      else allow_smem(attention_simt_kernel<T, 64>, smem_need);
    }
    add(CLS_ATTN, [=](cudaStream_t st, int n) {
      dim3 grid(4, nh, n);
      size_t smem = (size_t)361 * hd * sizeof(T) * 2 + 361 * sizeof(float);
      switch (hd) {
        case 16: launch_attn<16>(grid, smem, st, QKV, qc, kc, nh, nkv, scale, Ip->rowmask, O); break;
        case 32: launch_attn<32>(grid, smem, st, QKV, qc, kc, nh, nkv, scale, Ip->rowmask, O); break;
        default: launch_attn<64>(grid, smem, st, QKV, qc, kc, nh, nkv, scale, Ip->rowmask, O); break;
      }
    });
    // output projection, masked, + residual (bin2onnx.py :1420-1423)
    Spec so;
    so.cls = CLS_LINEAR;
    so.A = O;
    so.cin = round_up(nh * vhd, tc ? 64 : 16);
    so.N = w16(C);
    if (pass == 1) {
      so.W.assign((size_t)so.N * so.cin, 0.0f);
      pack_linear(so.W, so.cin, 0, b.out);
    }
    so.segs = {close_seg(w16(C), X, XA, next, true)};
    gemm(std::move(so));
  }

  template <int HD>
  static void launch_attn(dim3 grid, size_t smem, cudaStream_t st, Tensor QKV, int qc, int kc, int nh, int nkv,
                          float scale, const float* rowmask, Tensor O) {
    launch_pdl(attention_simt_kernel<T, HD>, dim3(grid), dim3(128), smem, st, (const T*)QKV.p, QKV.ld, qc, kc, nh, nkv, scale, rowmask,
                                                         (T*)O.p, O.ld);
  }

  void emit_ffn(const BlockDesc& b, Tensor X, Tensor XA, int C, BnAct next) {
    // bin2onnx.py transformer_ffn_block :1425-1438 (SwiGLU)
    const int F = b.ffn;
    Tensor XN = tensor(R_XN, C), H = tensor(R_H, F);
    rmsnorm(X, C, b.ln, XN);
    Spec s;
    s.cls = CLS_LINEAR;
    s.A = XN;
    s.cin = round_up(C, tc ? 64 : 16);
    s.N = 2 * F;
    if (pass == 1) {
      s.W.assign((size_t)s.N * s.cin, 0.0f);
      pack_linear(s.W, s.cin, 0, b.w1);
      pack_linear(s.W, s.cin, F, b.wgate);
    }
    const bool fuse = tc && F % 16 == 0 && pick_bn(2 * F, 64) != 0;
    if (fuse) {
      s.mode = MODE_SWIGLU;
      Seg g;
      g.width = 2 * F;
      g.raw = H;
      s.segs = {g};
      gemm(std::move(s));
    } else {
      Tensor AG = tensor(R_AG, 2 * F);
      Seg g;
      g.width = 2 * F;
      g.flags = EPI_RAW;
      g.raw = AG;
      s.segs = {g};
      if (F % 16 != 0) fail(KC_ERR_INVALID, "CUDA backend: " + b.name + ": ffn width must be a multiple of 16");
      gemm(std::move(s));
      Engine::Impl* Ip = &I;
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        int rows = n * 400;
        size_t total = (size_t)rows * F;
        launch_pdl(swiglu_kernel<T>, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, (const T*)AG.p, AG.ld, F, Ip->rowmask, rows,
                                                                         (T*)H.p, H.ld);
      });
    }
    Spec s2;
    s2.cls = CLS_LINEAR;
    s2.A = H;
    s2.cin = round_up(F, tc ? 64 : 16);
    s2.N = w16(C);
    if (pass == 1) {
      s2.W.assign((size_t)s2.N * s2.cin, 0.0f);
      pack_linear(s2.W, s2.cin, 0, b.w2);
    }
    s2.segs = {close_seg(w16(C), X, XA, next, true)};
    gemm(std::move(s2));
  }

  // ---- whole net ----
  void build_all(OutputLayout& L) {
    const int C = m.trunk_c;
    const ConvDesc& ic = m.initial_conv;
    if (ic.ky != ic.kx) fail(KC_ERR_INVALID, "CUDA backend: non-square initial convolution");
    stem_k = ic.ky;
    stem_pad = (ic.ky / 2) * std::max(ic.dy, ic.dx);
    if (ic.dy != ic.dx) fail(KC_ERR_INVALID, "CUDA backend: anisotropic dilation of the initial convolution");
    stem_stride = 19 + stem_pad;
    stem_brows = (19 + stem_pad) * stem_stride;
    stem_cin = round_up(m.num_input_channels, tc ? 64 : 16);
    I.stem_rows = round_up(max_batch * stem_brows, 128) + 2 * (stem_pad * stem_stride + stem_pad) + 128;
    // tensor-core tiers: the stem reads an im2col operand in the PBL (one tap, K = taps x planes padded to 64)
    const bool im2col = tc;
    const int stem_dil = std::max(ic.dy, 1);
    const int pix_c = round_up(m.num_input_channels, 8);  // planes per pixel of the im2col staging grid
    if (im2col) {
      stem_cin = round_up(stem_k * stem_k * pix_c, 64);
      I.stem_rows = round_up(max_batch * 400, 128) + 128;
    }

    Tensor X = tensor(R_LEVEL0, C), XA = tensor(R_LEVEL0 + 1, C);
    Tensor STEM = tensor(R_STEM, stem_cin);
    // stem input layout + per-board statistics and trunk bias
    {
      const int cin = m.num_input_channels, brows = stem_brows, stride = stem_stride, pad = stem_pad;
      Engine::Impl* Ip = &I;
      const int sk = stem_k, grid_px = (19 + 2 * pad) * (19 + 2 * pad);
      // im2col staging: [n][G][G][pix_c] of T, as a per-board float buffer
      T* pix = im2col ? reinterpret_cast<T*>(fbuffer(F_PIX, (grid_px * pix_c * (int)sizeof(T) + 3) / 4)) : nullptr;
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        if (im2col) {
          launch_pdl(prep_pixels_kernel<T>, dim3((n * grid_px + 255) / 256), dim3(256), 0, st, Ip->input(), n, cin,
                     pad, pix, pix_c, Ip->rowmask);
          launch_pdl(prep_im2col_kernel<T>, dim3((n * 400 * (sk * sk + 1) + 255) / 256), dim3(256), 0, st,
                     (const T*)pix, n, sk, stem_dil, pad, pix_c, (T*)STEM.p, STEM.ld);
        } else
          launch_pdl(prep_input_kernel<T>, dim3((n * 361 + 127) / 128), dim3(128), 0, st, Ip->input(), n, cin,
                     (T*)STEM.p, STEM.ld, brows, stride, pad, Ip->rowmask);
      });
      BoardParams bp;
      std::memset(&bp, 0, sizeof(bp));
      bp.cin = cin;
      bp.G = m.num_input_global_channels;
      bp.wg = up(m.initial_matmul.w);
      bp.C = C;
      if (m.has_meta) {
        bp.m1 = up(m.meta_mul1.w); bp.b1 = up(m.meta_bias1.b); bp.h1 = m.meta_mul1.oc; bp.act1 = m.meta_act1;
        bp.m2 = up(m.meta_mul2.w); bp.b2 = up(m.meta_bias2.b); bp.h2 = m.meta_mul2.oc; bp.act2 = m.meta_act2;
        bp.m3 = up(m.meta_mul3.w);
        if (bp.h1 > 512 || bp.h2 > 512) fail(KC_ERR_INVALID, "CUDA backend: metadata encoder wider than 512");
      }
      bp.board_bias = I.board_bias;
      bp.mask_sum = I.mask_sum;
      bp.scale1 = I.scale1;
      bp.scale2 = I.scale2;
      const bool meta = m.has_meta;
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        BoardParams q = bp;
        q.spatial = Ip->in_spatial;
        q.bits = Ip->in_bits;
        q.glob = Ip->in_global;
        q.meta = meta ? Ip->in_meta : nullptr;
        launch_pdl(board_kernel, dim3(n), dim3(256), 0, st, q);
      });
    }
    // stem conv + per-board bias -> X (remapped into the PBL), XA = first block's pre-BN act
    {
      BnAct first = consumer_bn(m.blocks, 0, {});
      Spec s;
      s.cls = CLS_STEM;
      s.A = STEM;
      s.cin = stem_cin;
      s.taps.clear();
      if (im2col) {
        s.taps.push_back(0);  // one tap over the im2col operand, ordinary PBL rows
      } else {
        s.stem = true;
        for (int ky = 0; ky < stem_k; ky++)
          for (int kx = 0; kx < stem_k; kx++)
            s.taps.push_back(((ky - stem_k / 2) * stem_stride + (kx - stem_k / 2)) * stem_dil);
      }
      s.N = w16(C);
      const int K = (int)s.taps.size() * s.cin;
      if (pass == 1) {
        s.W.assign((size_t)s.N * K, 0.0f);
        // im2col column of (tap, plane) = tap * planes padded to 8 + plane; else tap * padded planes + plane
        pack_conv(s.W, K, im2col ? pix_c : s.cin, 0, ic);
      }
      Seg g;
      g.width = w16(C);
      g.flags = EPI_BOARD_BIAS | EPI_RAW | (X.f32 ? EPI_RAW_F32 : 0);
      g.board_bias = I.board_bias;
      g.ld_bb = C;
      g.raw = X;
      if (first.bn) {
        g.flags |= EPI_ACT;
        g.act = first.act;
        g.scale = first.bn->merged_scale;
        g.bias = first.bn->merged_bias;
        g.actout = XA;
      }
      s.segs = {g};
      gemm(std::move(s));
    }
    // trunk; with heads in another type than the trunk (the bf16 tier) the tip writes its own buffer in that type
    constexpr bool hsplit = !std::is_same<H, T>::value;
    BnAct tip;
    if (m.trunk_norm_kind == 0 && !hsplit) tip = {&m.tip_bn, m.tip_act};
    emit_stack(m.blocks, 0, C, tip);
    const Tensor XH = hsplit ? tensor(R_TIPH, C) : XA;
    if (m.trunk_norm_kind == 0 && hsplit) {
      if (X.f32) bias_bnact<float, H>(X, 0, nullptr, m.tip_bn, m.tip_act, C, XH);
      else bias_bnact<T, H>(X, 0, nullptr, m.tip_bn, m.tip_act, C, XH);
    }
    if (m.trunk_norm_kind != 0) {
      const float* g = up(m.tip_rms_gamma);
      const float* bb = up(m.tip_rms_beta);
      float eps = m.tip_rms_eps;
      int spatial = m.tip_rms_spatial ? 1 : 0;
      int act = m.tip_act;
      Engine::Impl* Ip = &I;
      if (!spatial && rms_vec(X, C, XH)) {
        // per-point tip: one warp per row
        add(CLS_OTHER, [=](cudaStream_t st, int n) {
          const int rows = n * 400;
          if (X.f32)
            launch_pdl(rms_rows_kernel<float, H, true>, dim3((rows + 7) / 8), dim3(256), 0, st, (const float*)X.p,
                       X.ld, C / 128, g, bb, act, eps, Ip->rowmask, rows, (H*)XH.p, XH.ld);
          else
            launch_pdl(rms_rows_kernel<T, H, true>, dim3((rows + 7) / 8), dim3(256), 0, st, (const T*)X.p, X.ld,
                       C / 128, g, bb, act, eps, Ip->rowmask, rows, (H*)XH.p, XH.ld);
        });
      } else if (spatial && rms_vec(X, C, XH)) {
        // spatial tip: row sums of squares, then per row its board's rms and the affine + activation
        float* tss = fbuffer(F_TIPSS, 400);
        add(CLS_OTHER, [=](cudaStream_t st, int n) {
          const int rows = n * 400;
          const dim3 grid((rows + 7) / 8), block(256);
          if (X.f32) {
            launch_pdl(row_sumsq_kernel<float>, grid, block, 0, st, (const float*)X.p, X.ld, C / 128, rows, tss);
            launch_pdl(tip_spatial_apply_kernel<float, H>, grid, block, 0, st, (const float*)X.p, X.ld, C / 128,
                       (const float*)tss, Ip->rowmask, Ip->mask_sum, g, bb, act, eps, rows, (H*)XH.p, XH.ld);
          } else {
            launch_pdl(row_sumsq_kernel<T>, grid, block, 0, st, (const T*)X.p, X.ld, C / 128, rows, tss);
            launch_pdl(tip_spatial_apply_kernel<T, H>, grid, block, 0, st, (const T*)X.p, X.ld, C / 128,
                       (const float*)tss, Ip->rowmask, Ip->mask_sum, g, bb, act, eps, rows, (H*)XH.p, XH.ld);
          }
        });
      } else {
        add(CLS_OTHER, [=](cudaStream_t st, int n) {
          if (X.f32)
            launch_pdl(tip_rms_kernel<float, H>, dim3(n), dim3(512), 0, st, (const float*)X.p, X.ld, C, g, bb, eps,
                       spatial, act, Ip->rowmask, Ip->mask_sum, (H*)XH.p, XH.ld);
          else
            launch_pdl(tip_rms_kernel<T, H>, dim3(n), dim3(512), 0, st, (const T*)X.p, X.ld, C, g, bb, eps, spatial,
                       act, Ip->rowmask, Ip->mask_sum, (H*)XH.p, XH.ld);
        });
      }
    }
    // heads: one GEMM for p1 | g1 | v1 (bin2onnx.py policy_head :1495, value_head :1518)
    const int p1c = m.p1_conv.oc, g1c = m.g1_conv.oc, v1c = m.v1_conv.oc;
    const int P1p = w16(p1c), G1p = w16(g1c), V1p = w16(v1c);
    Tensor HEAD = tensor(R_HEAD, P1p + G1p + V1p);
    Tensor P1A = tensor(R_P1A, p1c);
    {
      Seg s0;
      s0.width = P1p;
      s0.flags = EPI_RAW;
      s0.raw = HEAD;
      // HEAD column = GEMM column: each segment's output base is its first GEMM column
      Seg s1 = act_seg(G1p, m.g1_bn, m.g1_act, HEAD, P1p);
      Seg s2 = act_seg(V1p, m.v1_bn, m.v1_act, HEAD, P1p + G1p);
      gemm<H>(conv_spec(CLS_LINEAR, XH, C, {&m.p1_conv, &m.g1_conv, &m.v1_conv}, {s0, s1, s2}));
    }
    L.policy_off = 0;
    L.value_off = m.num_policy_channels * 362;
    L.score_off = L.value_off + m.num_value_channels();
    L.own_off = L.score_off + m.num_score_value_channels();
    L.row_len = L.own_off + 361 * m.num_ownership_channels();
    const int row_len = L.row_len;
    float* g1pool = fbuffer(F_POOL, 3 * g1c);
    float* p1bias = fbuffer(F_GBIAS, p1c);
    pool<H>(HEAD, P1p, g1c, false, g1pool);
    fc(g1pool, 3 * g1c, m.gpool_to_bias_mul, nullptr, ACT_IDENTITY, p1bias, p1c, 0, 1);
    bias_bnact<H, H>(HEAD, 0, p1bias, m.p1_bn, m.p1_act, p1c, P1A);
    {
      // p2 weights [p1c][P] and ownership weights [v1c] (1x1 convs, file order [ic][oc])
      const float* w2 = up(m.p2_conv.w);
      const float* wo = up(m.v_ownership_conv.w);
      const int P = m.num_policy_channels, own_off = L.own_off;
      const int v1c0 = P1p + G1p;
      Engine::Impl* Ip = &I;
      add(CLS_OTHER, [=](cudaStream_t st, int n) {
        launch_pdl(head_spatial_kernel<H>, dim3((n * 361 + 127) / 128), dim3(128), 0, st, (const H*)P1A.p, P1A.ld,
                   p1c, w2, P, (const H*)HEAD.p, HEAD.ld, v1c0, v1c, wo, Ip->out, row_len, own_off, n);
      });
    }
    // pass logit: policy[p * 362 + 361]
    if (m.pass_mlp) {
      float* tmp = fbuffer(F_PASS, m.gpool_to_pass_mul.oc);
      fc(g1pool, 3 * g1c, m.gpool_to_pass_mul, &m.gpool_to_pass_bias, m.pass_act, tmp, m.gpool_to_pass_mul.oc, 0, 1);
      fc(tmp, m.gpool_to_pass_mul.oc, m.gpool_to_pass_mul2, nullptr, ACT_IDENTITY, nullptr, row_len, 361, 362);
    } else {
      fc(g1pool, 3 * g1c, m.gpool_to_pass_mul, nullptr, ACT_IDENTITY, nullptr, row_len, 361, 362);
    }
    // value head
    float* vpool = fbuffer(F_VPOOL, 3 * v1c);
    float* v2 = fbuffer(F_V2, m.v2_mul.oc);
    pool<H>(HEAD, P1p + G1p, v1c, true, vpool);
    fc(vpool, 3 * v1c, m.v2_mul, &m.v2_bias, m.v2_act, v2, m.v2_mul.oc, 0, 1);
    fc(v2, m.v2_mul.oc, m.v3_mul, &m.v3_bias, ACT_IDENTITY, nullptr, row_len, L.value_off, 1);
    fc(v2, m.v2_mul.oc, m.sv3_mul, &m.sv3_bias, ACT_IDENTITY, nullptr, row_len, L.score_off, 1);
  }
};

}  // namespace

Engine::Engine(const ModelDesc& m, int device, int max_batch, int precision)
    : device_(device), max_batch_(max_batch), precision_(precision), impl_(new Impl) {
  if (max_batch < 1) fail(KC_ERR_INVALID, "CUDA backend: max batch size must be positive");
  KC_CUDA(cudaSetDevice(device));
  Impl& I = *impl_;
  int dev_sms = 0;
  KC_CUDA(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, device));
  I.sm_count = dev_sms;
  I.R = round_up(max_batch * 400, 128) + 128;
  I.d_err = static_cast<int*>(I.alloc(sizeof(int) * 4));
  I.rowmask = static_cast<float*>(I.alloc((size_t)I.R * sizeof(float)));
  I.mask_sum = static_cast<float*>(I.alloc((size_t)max_batch * sizeof(float)));
  I.scale1 = static_cast<float*>(I.alloc((size_t)max_batch * sizeof(float)));
  I.scale2 = static_cast<float*>(I.alloc((size_t)max_batch * sizeof(float)));
  I.board_bias = static_cast<float*>(I.alloc((size_t)max_batch * m.trunk_c * sizeof(float)));
  switch (precision) {
    case PREC_F32: build_model<float>(m); break;
    case PREC_F16: build_model<__half>(m); break;
    case PREC_BF16: build_model<__nv_bfloat16>(m); break;
    default: fail(KC_ERR_INVALID, "CUDA backend: unknown precision");
  }
  KC_CUDA(cudaDeviceSynchronize());
}

Engine::~Engine() {
  if (impl_) {
    cudaSetDevice(device_);
    cudaDeviceSynchronize();
  }
  for (auto e : prof_events_) cudaEventDestroy(e);
}

template <typename T>
void Engine::build_model(const ModelDesc& m) {
  Builder<T> b(*impl_, plan_, m, max_batch_, std::is_same<T, __nv_bfloat16>::value);
  b.pass = 0;
  OutputLayout L;
  b.build_all(L);
  b.pass = 1;
  b.allocate();
  b.build_all(L);
  layout_ = L;
}

int Engine::device_error() {
  int e = 0;
  KC_CUDA(cudaMemcpy(&e, impl_->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  return e;
}

int* Engine::error_word() { return impl_->d_err; }

void Engine::clear_device_error() { KC_CUDA(cudaMemset(impl_->d_err, 0, sizeof(int))); }

void Engine::set_profiling(bool on) {
  if (on && prof_events_.empty()) {
    KC_CUDA(cudaSetDevice(device_));
    prof_events_.resize(2 * plan_.size());
    for (auto& e : prof_events_) KC_CUDA(cudaEventCreate(&e));
  }
  profiling_ = on;
}

void Engine::reset_profile() {
  for (int i = 0; i < CLS_COUNT; i++) {
    prof_ms_[i] = 0;
    prof_n_[i] = 0;
  }
  prof_pending_ = false;
}

void Engine::collect_profile() {
  if (!prof_pending_) return;
  KC_CUDA(cudaEventSynchronize(prof_events_.back()));
  for (size_t j = 0; j < plan_.size(); j++) {
    float ms = 0;
    KC_CUDA(cudaEventElapsedTime(&ms, prof_events_[2 * j], prof_events_[2 * j + 1]));
    prof_ms_[plan_[j].cls] += ms;
    prof_n_[plan_[j].cls] += 1;
  }
  prof_pending_ = false;
}

void Engine::profile(double* ms, int64_t* launches, int n) {
  collect_profile();
  for (int i = 0; i < n && i < CLS_COUNT; i++) {
    if (ms) ms[i] = prof_ms_[i];
    if (launches) launches[i] = prof_n_[i];
  }
}

void Engine::run_plan(int n, cudaStream_t stream, bool events) {
  for (size_t j = 0; j < plan_.size(); j++) {
    // external event nodes: recorded each time a captured graph runs
    if (events) KC_CUDA(cudaEventRecordWithFlags(prof_events_[2 * j], stream, cudaEventRecordExternal));
    plan_[j].fn(stream, n);
    KC_CUDA(cudaGetLastError());
    if (events) KC_CUDA(cudaEventRecordWithFlags(prof_events_[2 * j + 1], stream, cudaEventRecordExternal));
  }
}

void Engine::forward(int n, cudaStream_t stream, const float* d_spatial, const float* d_global, const float* d_meta,
                     float* d_out, const uint32_t* d_bits, const int* d_sym) {
  if (n < 1 || n > max_batch_)
    fail(KC_ERR_INVALID, "CUDA backend: batch of " + std::to_string(n) + " rows outside [1, " +
                             std::to_string(max_batch_) + "]");
  Impl& I = *impl_;
  KC_CUDA(cudaSetDevice(device_));
  if (prof_pending_) collect_profile();
  if (!d_bits == !d_spatial || (d_bits && !d_sym))
    fail(KC_ERR_INVALID, "CUDA backend: a forward pass takes float planes or bit-packed planes with symmetries");
  I.in_spatial = d_spatial;
  I.in_bits = d_bits;
  I.in_sym = d_sym;
  I.in_global = d_global;
  I.in_meta = d_meta;
  I.out = d_out;
  const bool events = profiling_;
  if (!use_graphs_) {
    run_plan(n, stream, events);
  } else {
    auto key = std::make_tuple(n * 2 + (events ? 1 : 0), (const void*)d_spatial, (const void*)d_bits,
                               (const void*)d_sym, (const void*)d_global, (const void*)d_meta, (void*)d_out);
    auto it = I.graphs.find(key);
    if (it == I.graphs.end()) {
      cudaGraph_t g;
      KC_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      try {
        run_plan(n, stream, events);
      } catch (...) {
        cudaStreamEndCapture(stream, &g);
        cudaGetLastError();
        throw;
      }
      KC_CUDA(cudaStreamEndCapture(stream, &g));
      cudaGraphExec_t ge;
      KC_CUDA(cudaGraphInstantiate(&ge, g, 0));
      cudaGraphDestroy(g);
      if (I.graphs.size() >= Impl::kMaxGraphs) {
        auto lru = I.graphs.begin();
        for (auto j = I.graphs.begin(); j != I.graphs.end(); ++j)
          if (j->second.second < lru->second.second) lru = j;
        cudaGraphExecDestroy(lru->second.first);
        I.graphs.erase(lru);
      }
      it = I.graphs.emplace(key, std::make_pair(ge, uint64_t(0))).first;
    }
    it->second.second = ++I.graph_clock;
    KC_CUDA(cudaGraphLaunch(it->second.first, stream));
  }
  if (events) prof_pending_ = true;
}

void model_flops(const ModelDesc& m, double* total, double* conv3x3) {
  const double area = 361;
  double t = 0, c3 = 0;
  std::function<void(const std::vector<BlockDesc>&)> walk = [&](const std::vector<BlockDesc>& v) {
    for (auto& b : v) {
      auto conv = [&](const ConvDesc& c) {
        double f = 2.0 * area * c.ky * c.kx * c.ic * c.oc;
        t += f;
        if (c.ky == 3) c3 += f;
      };
      switch (b.kind) {
        case BLOCK_ORDINARY: conv(b.regular); conv(b.final_conv); break;
        case BLOCK_GPOOL: conv(b.regular); conv(b.gpool_conv); conv(b.final_conv); break;
        case BLOCK_NESTED: conv(b.pre_conv); walk(b.inner); conv(b.post_conv); break;
        case BLOCK_ATTENTION:
          t += 2.0 * area * (b.q.ic * (double)b.q.oc + b.k.ic * (double)b.k.oc + b.v.ic * (double)b.v.oc +
                             b.out.ic * (double)b.out.oc);
          t += 2.0 * area * area * b.heads * (b.head_dim + b.v_head_dim);
          break;
        case BLOCK_FFN: t += 2.0 * area * (b.w1.ic * (double)b.w1.oc * 2 + b.w2.ic * (double)b.w2.oc); break;
      }
    }
  };
  walk(m.blocks);
  const ConvDesc& ic = m.initial_conv;
  t += 2.0 * area * ic.ky * ic.kx * ic.ic * ic.oc;
  t += 2.0 * area * m.trunk_c * (double)(m.p1_conv.oc + m.g1_conv.oc + m.v1_conv.oc);
  if (total) *total = t;
  if (conv3x3) *conv3x3 = c3;
}

}  // namespace kc
