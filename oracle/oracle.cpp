// CPU ORACLE — test infrastructure only, never part of the product path.
//
// A plain C++ restatement of the reference's neural-net forward pass, used by tests/ (parity checks), by
// __graft_entry__.smoke() and by bench.py's CPU-baseline leg. Nothing in katago-rs_b200/ links or calls it.
//
// What it restates (file:line in the katago-rs reference checkout):
//   * the model-file parser: tools/bin2onnx/bin2onnx.py ModelReader :61-125, parse_conv :149, parse_bn :186,
//     parse_activation :208, parse_matmul :225, parse_matbias :240, blocks :232-338, RMSNorm :383-420,
//     transformer blocks :489-560, block stack :575-599, meta encoder :639-668, trunk :718-765, policy head
//     :774-823, value head :833-857, parse_model :1009-1071;
//   * the forward graph: bin2onnx.py GraphBuilder :1088-1531 (setup_mask :1203, gpool :1222, value_pool :1232,
//     residual / gpool / nested blocks :1243-1269, block_stack :1271, transformer_rmsnorm :1330, rope :1342,
//     attention :1359, ffn :1425, trunk tip RMSNorm :1440, meta encoder :1467, trunk :1477, heads :1495-1531),
//     with every constant as the graph holds it (float32 scalars such as 0.1f, eps, 1/sqrt(d); RoPE tables in
//     float32 from float64 cos/sin, desc.cpp computeRopeCosSin as bin2onnx.py:449-484 restates it);
//   * batch-norm merge in float32 (bin2onnx.py:179-183); mish with burn's softplus (identity above 20,
//     crates/katago-nn-burn/src/wino/kernels.rs:131); SiLU as x / (exp(-x) + 1) (bin2onnx.py:1163-1168).
// It runs in float (the flex-like tier) or double (the error yardstick). Pinned by tests/test_oracle_golden.py
// against tests/golden/*.npz, which are the reference graph itself evaluated in float64.
//
// Build: oracle/Makefile (-ffp-contract=off so float32 steps round like the numpy reference).

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace orc {

enum Act { ACT_ID = 0, ACT_RELU = 1, ACT_MISH = 2, ACT_SILU = 3 };

struct Conv { int ky = 0, kx = 0, ic = 0, oc = 0, dy = 1, dx = 1; std::vector<float> w; };  // w [oc][ic][ky][kx]
struct BN { int c = 0; std::vector<float> scale, bias; };                                    // merged, float32
struct MatMul { int ic = 0, oc = 0; std::vector<float> w; };                                 // [ic][oc]
struct MatBias { int c = 0; std::vector<float> b; };
struct TfRms { int c = 0; float eps = 0; std::vector<float> w; };

enum Kind { K_ORD, K_GPOOL, K_NESTED, K_ATTN, K_FFN };

struct Block {
  Kind kind;
  // ordinary / gpool / nested
  BN pre_bn; Act pre_act = ACT_RELU;
  Conv regular, gpool_conv, final_conv, pre_conv, post_conv;
  BN gpool_bn, mid_bn, post_bn; Act gpool_act = ACT_RELU, mid_act = ACT_RELU, post_act = ACT_RELU;
  MatMul gpool_to_bias;
  std::vector<Block> inner;
  // transformer
  int nh = 0, nkv = 0, hd = 0, vhd = 0; bool rope = false, learn = false; float theta = 0;
  TfRms ln; MatMul q, k, v, out, w1, wg, w2; int ffn = 0;
  std::vector<float> freqs;  // [nkv][pairs][2]
  std::vector<float> cos_t, sin_t;  // learnable: [nkv][P][S]; fixed: [P][S]
};

struct Model {
  std::string name;
  int version = 0, n_in = 0, n_glob = 0, n_meta = 0, meta_ver = 0;
  int trunk_c = 0, norm_kind = 0;
  Conv initial_conv; MatMul initial_matmul;
  bool has_meta = false; MatMul m1, m2, m3; MatBias mb1, mb2; Act ma1 = ACT_ID, ma2 = ACT_ID;
  std::vector<Block> blocks;
  BN tip_bn; bool tip_rms = false, tip_spatial = false; float tip_eps = 0; std::vector<float> tip_gamma, tip_beta;
  Act tip_act = ACT_RELU;
  // policy head
  int P = 1; Conv p1, g1, p2; BN g1_bn, p1_bn; Act g1_act = ACT_RELU, p1_act = ACT_RELU, pass_act = ACT_ID;
  MatMul gpool_to_bias_p, pass_mul, pass_mul2; MatBias pass_bias; bool pass_mlp = false;
  // value head
  Conv v1, own; BN v1_bn; Act v1_act = ACT_RELU, v2_act = ACT_RELU; MatMul v2, v3, sv3; MatBias v2b, v3b, sv3b;
};

// --------------------------------------------------------------------------------------------------------------
// Parser (bin2onnx.py ModelReader and parse_*)
// --------------------------------------------------------------------------------------------------------------

struct Reader {
  const uint8_t* d; size_t n; size_t pos = 0;
  static bool ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; }
  void skip() { while (pos < n && ws(d[pos])) pos++; }
  std::string tok() {
    skip();
    size_t s = pos;
    while (pos < n && !ws(d[pos])) pos++;
    if (pos == s) throw std::runtime_error("Unexpected end of model file");
    return std::string((const char*)d + s, pos - s);
  }
  int i() { return std::stoi(tok()); }
  float f() { return std::strtof(tok().c_str(), nullptr); }
  bool b() { int v = i(); if (v != 0 && v != 1) throw std::runtime_error("Expected bool 0/1"); return v == 1; }
  std::vector<float> floats(size_t cnt, const std::string& name) {
    int before = 0;
    while (true) {
      if (pos >= n) throw std::runtime_error(name + ": could not find binary float block");
      uint8_t c = d[pos++];
      if (c == '@') break;
      if (++before > 100) throw std::runtime_error(name + ": could not read float weights (no @BIN@ header)");
    }
    if (pos + 4 > n || memcmp(d + pos, "BIN@", 4) != 0) throw std::runtime_error(name + ": bad binary header");
    pos += 4;
    if (pos + 4 * cnt > n) throw std::runtime_error(name + ": too few floats");
    std::vector<float> v(cnt);
    memcpy(v.data(), d + pos, 4 * cnt);
    pos += 4 * cnt;
    for (float x : v) if (!std::isfinite(x)) throw std::runtime_error(name + ": non-finite weight");
    return v;
  }
};

static void check(bool c, const std::string& m) { if (!c) throw std::runtime_error(m); }

static Conv parse_conv(Reader& r) {
  std::string name = r.tok();
  Conv c;
  c.ky = r.i(); c.kx = r.i(); c.ic = r.i(); c.oc = r.i(); c.dy = r.i(); c.dx = r.i();
  check(c.ky > 0 && c.kx > 0 && c.ic > 0 && c.oc > 0 && c.dy > 0 && c.dx > 0, name + ": bad conv dims");
  check(c.ky % 2 == 1 && c.kx % 2 == 1, name + ": convolution filter sizes must be odd");
  auto raw = r.floats((size_t)c.ky * c.kx * c.ic * c.oc, name);  // file order y,x,ic,oc
  c.w.resize(raw.size());
  for (int y = 0; y < c.ky; y++)
    for (int x = 0; x < c.kx; x++)
      for (int i = 0; i < c.ic; i++)
        for (int o = 0; o < c.oc; o++)
          c.w[(((size_t)o * c.ic + i) * c.ky + y) * c.kx + x] = raw[(((size_t)y * c.kx + x) * c.ic + i) * c.oc + o];
  return c;
}

static BN parse_bn(Reader& r) {
  std::string name = r.tok();
  BN b; b.c = r.i();
  float eps = r.f();
  bool hs = r.b(), hb = r.b();
  check(b.c >= 1 && eps > 0, name + ": bad bn");
  auto mean = r.floats(b.c, name), var = r.floats(b.c, name);
  std::vector<float> scale = hs ? r.floats(b.c, name) : std::vector<float>(b.c, 1.0f);
  std::vector<float> bias = hb ? r.floats(b.c, name) : std::vector<float>(b.c, 0.0f);
  b.scale.resize(b.c); b.bias.resize(b.c);
  for (int i = 0; i < b.c; i++) {
    volatile float v = var[i] + eps;
    volatile float sq = std::sqrt((float)v);
    volatile float ms = scale[i] / sq;
    volatile float prod = ms * mean[i];
    b.scale[i] = ms;
    b.bias[i] = bias[i] - prod;
  }
  return b;
}

static Act parse_act(Reader& r, int version) {
  std::string name = r.tok();
  if (version >= 11) {
    std::string k = r.tok();
    if (k == "ACTIVATION_IDENTITY") return ACT_ID;
    if (k == "ACTIVATION_RELU") return ACT_RELU;
    if (k == "ACTIVATION_MISH") return ACT_MISH;
    if (k == "ACTIVATION_SILU") return ACT_SILU;
    throw std::runtime_error(name + ": unknown activation " + k);
  }
  return ACT_RELU;
}

static MatMul parse_matmul(Reader& r) {
  std::string name = r.tok();
  MatMul m; m.ic = r.i(); m.oc = r.i();
  check(m.ic > 0 && m.oc > 0, name + ": bad matmul");
  m.w = r.floats((size_t)m.ic * m.oc, name);
  return m;
}

static MatBias parse_matbias(Reader& r) {
  std::string name = r.tok();
  MatBias b; b.c = r.i();
  b.b = r.floats(b.c, name);
  return b;
}

static TfRms parse_tfrms(Reader& r) {
  std::string name = r.tok();
  TfRms t; t.c = r.i(); t.eps = r.f();
  t.w = r.floats(t.c, name);
  return t;
}

static std::vector<Block> parse_stack(Reader& r, int version, int nblocks, int c);

static void rope_tables(Block& b) {
  // computeRopeCosSin (bin2onnx.py:449-484), float32 steps, cos/sin of the float32 angle in float64
  const int S = 361, L = 19;
  int P = b.hd / 2;
  if (b.learn) {
    b.cos_t.assign((size_t)b.nkv * P * S, 0); b.sin_t.assign((size_t)b.nkv * P * S, 0);
    for (int h = 0; h < b.nkv; h++)
      for (int p = 0; p < P; p++) {
        float fx = b.freqs[((size_t)h * P + p) * 2 + 0], fy = b.freqs[((size_t)h * P + p) * 2 + 1];
        for (int s = 0; s < S; s++) {
          volatile float ax = (float)(s % L) * fx;
          volatile float ay = (float)(s / L) * fy;
          volatile float a = ax + ay;
          b.cos_t[((size_t)h * P + p) * S + s] = (float)std::cos((double)a);
          b.sin_t[((size_t)h * P + p) * S + s] = (float)std::sin((double)a);
        }
      }
  } else {
    b.cos_t.assign((size_t)P * S, 0); b.sin_t.assign((size_t)P * S, 0);
    int ppd = P / 2, dim_half = b.hd / 2;
    for (int p = 0; p < P; p++) {
      int padj = p < ppd ? p : p - ppd;
      volatile float expo = (float)(2 * padj) / (float)dim_half;
      float powv = (float)std::pow((double)b.theta, (double)expo);
      volatile float freq = 1.0f / powv;
      for (int s = 0; s < S; s++) {
        float pos = p < ppd ? (float)(s / L) : (float)(s % L);
        volatile float a = pos * freq;
        b.cos_t[(size_t)p * S + s] = (float)std::cos((double)a);
        b.sin_t[(size_t)p * S + s] = (float)std::sin((double)a);
      }
    }
  }
}

static Block parse_block(Reader& r, int version, const std::string& kind, int c) {
  Block b;
  if (kind == "ordinary_block") {
    b.kind = K_ORD; r.tok();
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version); b.regular = parse_conv(r);
    b.mid_bn = parse_bn(r); b.mid_act = parse_act(r, version); b.final_conv = parse_conv(r);
  } else if (kind == "gpool_block") {
    b.kind = K_GPOOL; r.tok();
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version);
    b.regular = parse_conv(r); b.gpool_conv = parse_conv(r);
    b.gpool_bn = parse_bn(r); b.gpool_act = parse_act(r, version);
    b.gpool_to_bias = parse_matmul(r);
    b.mid_bn = parse_bn(r); b.mid_act = parse_act(r, version); b.final_conv = parse_conv(r);
  } else if (kind == "nested_bottleneck_block") {
    b.kind = K_NESTED; r.tok();
    int nb = r.i();
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version); b.pre_conv = parse_conv(r);
    b.inner = parse_stack(r, version, nb, b.pre_conv.oc);
    b.post_bn = parse_bn(r); b.post_act = parse_act(r, version); b.post_conv = parse_conv(r);
  } else if (kind == "transformer_attention_block") {
    b.kind = K_ATTN; std::string name = r.tok();
    b.nh = r.i(); b.nkv = r.i(); b.hd = r.i(); b.vhd = r.i(); b.rope = r.i() != 0; b.learn = r.i() != 0;
    b.ln = parse_tfrms(r); b.q = parse_matmul(r); b.k = parse_matmul(r); b.v = parse_matmul(r); b.out = parse_matmul(r);
    if (b.rope) {
      if (b.learn) {
        std::string fname = r.tok();
        int a = r.i(), p = r.i(), d2 = r.i();
        check(a == b.nkv && p == b.hd / 2 && d2 == 2, name + ": bad rope freqs");
        b.freqs = r.floats((size_t)a * p * 2, name);
      } else {
        r.tok();
        b.theta = r.f();
      }
      rope_tables(b);
    }
  } else if (kind == "transformer_ffn_block") {
    b.kind = K_FFN; std::string name = r.tok();
    int cc = r.i(); b.ffn = r.i(); bool swiglu = r.i() != 0;
    check(cc == c, name + ": channels");
    b.ln = parse_tfrms(r); b.w1 = parse_matmul(r);
    check(swiglu, name + ": non-SwiGLU transformer FFN is not supported");
    b.wg = parse_matmul(r); b.w2 = parse_matmul(r);
  } else {
    throw std::runtime_error("found unknown block kind " + kind);
  }
  return b;
}

static std::vector<Block> parse_stack(Reader& r, int version, int nblocks, int c) {
  std::vector<Block> v;
  for (int i = 0; i < nblocks; i++) v.push_back(parse_block(r, version, r.tok(), c));
  return v;
}

static Model parse_model(const uint8_t* d, size_t n) {
  Reader r{d, n};
  Model m;
  m.name = r.tok(); m.version = r.i(); m.n_in = r.i(); m.n_glob = r.i();
  check(m.version >= 3 && m.version <= 17, "unsupported model version");
  if (m.version >= 13) for (int i = 0; i < 7; i++) r.f();
  if (m.version >= 15) {
    m.meta_ver = r.i();
    m.n_meta = m.meta_ver == 1 ? 192 : 0;
    for (int i = 0; i < 7; i++) r.i();
  }
  // trunk
  r.tok();
  int nb = r.i(); m.trunk_c = r.i(); r.i(); r.i(); r.i(); r.i();
  if (m.version >= 15) { m.norm_kind = r.i(); for (int i = 0; i < 5; i++) r.i(); }
  m.initial_conv = parse_conv(r);
  m.initial_matmul = parse_matmul(r);
  if (m.meta_ver > 0) {
    m.has_meta = true;
    r.tok(); r.i();
    m.m1 = parse_matmul(r); m.mb1 = parse_matbias(r); m.ma1 = parse_act(r, m.version);
    m.m2 = parse_matmul(r); m.mb2 = parse_matbias(r); m.ma2 = parse_act(r, m.version);
    m.m3 = parse_matmul(r);
  }
  m.blocks = parse_stack(r, m.version, nb, m.trunk_c);
  if (m.norm_kind == 0) {
    m.tip_bn = parse_bn(r);
  } else {
    m.tip_rms = true;
    r.tok(); r.i(); m.tip_eps = r.f(); m.tip_spatial = r.i() != 0; r.i();
    m.tip_gamma = r.floats(m.trunk_c, "rms"); m.tip_beta = r.floats(m.trunk_c, "rms");
  }
  m.tip_act = parse_act(r, m.version);
  // policy head
  r.tok();
  if (m.version >= 17) { m.P = r.i(); for (int i = 0; i < 3; i++) r.i(); }
  else if (m.version == 16) m.P = 4;
  else if (m.version >= 12) m.P = 2;
  else m.P = 1;
  m.p1 = parse_conv(r); m.g1 = parse_conv(r); m.g1_bn = parse_bn(r); m.g1_act = parse_act(r, m.version);
  m.gpool_to_bias_p = parse_matmul(r); m.p1_bn = parse_bn(r); m.p1_act = parse_act(r, m.version);
  m.p2 = parse_conv(r); m.pass_mul = parse_matmul(r);
  if (m.version >= 15) {
    m.pass_mlp = true;
    m.pass_bias = parse_matbias(r); m.pass_act = parse_act(r, m.version); m.pass_mul2 = parse_matmul(r);
  }
  // value head
  r.tok();
  if (m.version >= 17) for (int i = 0; i < 3; i++) r.i();
  m.v1 = parse_conv(r); m.v1_bn = parse_bn(r); m.v1_act = parse_act(r, m.version);
  m.v2 = parse_matmul(r); m.v2b = parse_matbias(r); m.v2_act = parse_act(r, m.version);
  m.v3 = parse_matmul(r); m.v3b = parse_matbias(r); m.sv3 = parse_matmul(r); m.sv3b = parse_matbias(r);
  m.own = parse_conv(r);
  r.skip();
  check(r.pos == r.n, "unparsed trailing bytes in model file");
  return m;
}

// --------------------------------------------------------------------------------------------------------------
// Forward (GraphBuilder semantics), NCHW with H = W = 19
// --------------------------------------------------------------------------------------------------------------

constexpr int L = 19, S = 361;

template <typename T>
struct Ctx {
  int N;
  std::vector<T> mask, mask_sum, scale1, scale2;  // mask [N][S]
};

template <typename T>
static inline T act(T x, Act a) {
  switch (a) {
    case ACT_ID: return x;
    case ACT_RELU: return x > T(0) ? x : T(0);
    case ACT_MISH: {
      T sp = x > T(20) ? x : std::log1p(std::exp(x));
      return x * std::tanh(sp);
    }
    case ACT_SILU: return x / (std::exp(-x) + T(1));
  }
  return x;
}

// out[N][oc][S] = conv(in[N][ic][S]) ("same" padding, dilation, stride 1)
template <typename T>
static std::vector<T> conv(const std::vector<T>& in, int N, const Conv& c) {
  std::vector<T> out((size_t)N * c.oc * S, T(0));
  int py = (c.ky / 2) * c.dy, px = (c.kx / 2) * c.dx;
  std::vector<T> w(c.w.begin(), c.w.end());
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; n++)
    for (int o = 0; o < c.oc; o++) {
      T acc[S];
      for (int s = 0; s < S; s++) acc[s] = T(0);
      for (int i = 0; i < c.ic; i++) {
        const T* src = &in[((size_t)n * c.ic + i) * S];
        for (int ky = 0; ky < c.ky; ky++) {
          int oy = ky * c.dy - py;
          for (int kx = 0; kx < c.kx; kx++) {
            int ox = kx * c.dx - px;
            T wv = w[(((size_t)o * c.ic + i) * c.ky + ky) * c.kx + kx];
            int y0 = oy < 0 ? -oy : 0, y1 = oy > 0 ? L - oy : L;
            int x0 = ox < 0 ? -ox : 0, x1 = ox > 0 ? L - ox : L;
            for (int y = y0; y < y1; y++) {
              const T* row = src + (y + oy) * L + ox;
              T* arow = acc + y * L;
              for (int x = x0; x < x1; x++) arow[x] += wv * row[x];
            }
          }
        }
      }
      std::memcpy(&out[((size_t)n * c.oc + o) * S], acc, sizeof(acc));
    }
  return out;
}

template <typename T>
static std::vector<T> matmul(const std::vector<T>& x, int N, const MatMul& m) {
  std::vector<T> y((size_t)N * m.oc, T(0));
  for (int n = 0; n < N; n++)
    for (int i = 0; i < m.ic; i++) {
      T xv = x[(size_t)n * m.ic + i];
      for (int o = 0; o < m.oc; o++) y[(size_t)n * m.oc + o] += xv * T(m.w[(size_t)i * m.oc + o]);
    }
  return y;
}

template <typename T>
static void matbias(std::vector<T>& x, int N, const MatBias& b) {
  for (int n = 0; n < N; n++)
    for (int c = 0; c < b.c; c++) x[(size_t)n * b.c + c] += T(b.b[c]);
}

template <typename T>
static void bn_act_mask(std::vector<T>& x, const Ctx<T>& cx, const BN& bn, Act a) {
  int C = bn.c;
#pragma omp parallel for collapse(2)
  for (int n = 0; n < cx.N; n++)
    for (int c = 0; c < C; c++) {
      T* p = &x[((size_t)n * C + c) * S];
      T s = T(bn.scale[c]), b = T(bn.bias[c]);
      for (int i = 0; i < S; i++) {
        T v = p[i] * s;
        v = v + b;
        p[i] = act(v, a) * cx.mask[(size_t)n * S + i];
      }
    }
}

template <typename T>
static void add(std::vector<T>& x, const std::vector<T>& y) {
  for (size_t i = 0; i < x.size(); i++) x[i] += y[i];
}

// [N,C,S] (already masked) -> [N,3C]: mean, mean*scale1, masked max (gpool, bin2onnx.py:1222-1230)
template <typename T>
static std::vector<T> gpool(const std::vector<T>& x, const Ctx<T>& cx, int C) {
  std::vector<T> out((size_t)cx.N * 3 * C);
  for (int n = 0; n < cx.N; n++)
    for (int c = 0; c < C; c++) {
      const T* p = &x[((size_t)n * C + c) * S];
      T s = 0, mx = -INFINITY;
      for (int i = 0; i < S; i++) {
        s += p[i];
        T biasv = cx.mask[(size_t)n * S + i] * T(1e4f) - T(1e4f);
        T v = p[i] + biasv;
        mx = v > mx ? v : mx;
      }
      T mean = s / cx.mask_sum[n];
      out[(size_t)n * 3 * C + c] = mean;
      out[(size_t)n * 3 * C + C + c] = mean * cx.scale1[n];
      out[(size_t)n * 3 * C + 2 * C + c] = mx;
    }
  return out;
}

template <typename T>
static std::vector<T> value_pool(const std::vector<T>& x, const Ctx<T>& cx, int C) {
  std::vector<T> out((size_t)cx.N * 3 * C);
  for (int n = 0; n < cx.N; n++)
    for (int c = 0; c < C; c++) {
      const T* p = &x[((size_t)n * C + c) * S];
      T s = 0;
      for (int i = 0; i < S; i++) s += p[i];
      T mean = s / cx.mask_sum[n];
      out[(size_t)n * 3 * C + c] = mean;
      out[(size_t)n * 3 * C + C + c] = mean * cx.scale1[n];
      out[(size_t)n * 3 * C + 2 * C + c] = mean * cx.scale2[n];
    }
  return out;
}

template <typename T>
static void add_nc_bias(std::vector<T>& x, int N, int C, const std::vector<T>& bias) {
  for (int n = 0; n < N; n++)
    for (int c = 0; c < C; c++) {
      T b = bias[(size_t)n * C + c];
      T* p = &x[((size_t)n * C + c) * S];
      for (int i = 0; i < S; i++) p[i] += b;
    }
}

// ---- transformer blocks, on tokens [N][S][C] ----

template <typename T>
static std::vector<T> to_tokens(const std::vector<T>& x, int N, int C) {
  std::vector<T> t(x.size());
  for (int n = 0; n < N; n++)
    for (int c = 0; c < C; c++)
      for (int s = 0; s < S; s++) t[((size_t)n * S + s) * C + c] = x[((size_t)n * C + c) * S + s];
  return t;
}

template <typename T>
static std::vector<T> to_nchw(const std::vector<T>& t, int N, int C) {
  std::vector<T> x(t.size());
  for (int n = 0; n < N; n++)
    for (int c = 0; c < C; c++)
      for (int s = 0; s < S; s++) x[((size_t)n * C + c) * S + s] = t[((size_t)n * S + s) * C + c];
  return x;
}

template <typename T>
static std::vector<T> tf_rms(const std::vector<T>& x, const Ctx<T>& cx, const TfRms& d) {
  int C = d.c;
  std::vector<T> y(x.size());
  for (size_t r = 0; r < (size_t)cx.N * S; r++) {
    const T* p = &x[r * C];
    T ss = 0;
    for (int c = 0; c < C; c++) ss += p[c] * p[c];
    T ms = ss / T(float(C));
    T den = std::sqrt(ms + T(d.eps));
    T rms = T(1) / den;
    for (int c = 0; c < C; c++) y[r * C + c] = p[c] * rms * T(d.w[c]) * cx.mask[r];
  }
  return y;
}

// tokens [R][ic] x [ic][oc] (optionally with permuted columns)
template <typename T>
static std::vector<T> tok_matmul(const std::vector<T>& x, size_t R, const MatMul& m, const std::vector<int>* perm = nullptr) {
  std::vector<T> y(R * m.oc, T(0));
  std::vector<T> w((size_t)m.ic * m.oc);
  for (int i = 0; i < m.ic; i++)
    for (int o = 0; o < m.oc; o++) w[(size_t)i * m.oc + o] = T(m.w[(size_t)i * m.oc + (perm ? (*perm)[o] : o)]);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < (long)R; r++) {
    T* yr = &y[r * m.oc];
    for (int i = 0; i < m.ic; i++) {
      T xv = x[r * m.ic + i];
      const T* wr = &w[(size_t)i * m.oc];
      for (int o = 0; o < m.oc; o++) yr[o] += xv * wr[o];
    }
  }
  return y;
}

template <typename T>
static void attention_block(std::vector<T>& x, const Ctx<T>& cx, const Block& b, int C) {
  int N = cx.N, nh = b.nh, nkv = b.nkv, hd = b.hd, vhd = b.vhd, g = nh / nkv, half = hd / 2;
  size_t R = (size_t)N * S;
  auto xn = tf_rms(x, cx, b.ln);
  std::vector<int> pq, pk;
  std::vector<int>* ppq = nullptr; std::vector<int>* ppk = nullptr;
  if (b.rope) {
    // per head: interleaved pair channels (2p, 2p+1) -> [2p for all p] + [2p+1 for all p] (bin2onnx.py:1369-1374)
    for (int h = 0; h < nh; h++) {
      for (int j = 0; j < hd; j += 2) pq.push_back(h * hd + j);
      for (int j = 1; j < hd; j += 2) pq.push_back(h * hd + j);
    }
    for (int h = 0; h < nkv; h++) {
      for (int j = 0; j < hd; j += 2) pk.push_back(h * hd + j);
      for (int j = 1; j < hd; j += 2) pk.push_back(h * hd + j);
    }
    ppq = &pq; ppk = &pk;
  }
  auto q = tok_matmul(xn, R, b.q, ppq);
  auto k = tok_matmul(xn, R, b.k, ppk);
  auto v = tok_matmul(xn, R, b.v);
  int P = hd / 2;
  auto rope = [&](std::vector<T>& t, int nheads, int h, size_t n) {
    // rotate head h of tokens of board n in place; table row: learnable -> kv head, fixed -> shared
    int kvh = b.learn ? (nheads == nh ? h * nkv / nh : h) : 0;
    for (int s = 0; s < S; s++) {
      T* p = &t[((n * S + s) * nheads + h) * hd];
      for (int j = 0; j < half; j++) {
        size_t ti = b.learn ? ((size_t)kvh * P + j) * S + s : (size_t)j * S + s;
        T c = T(b.cos_t[ti]), sn = T(b.sin_t[ti]);
        T x0 = p[j], x1 = p[j + half];
        T a0 = x0 * c, b1 = x1 * sn;
        T r0 = a0 - b1;
        T c0 = x0 * sn, d1 = x1 * c;
        T r1 = c0 + d1;
        p[j] = r0; p[j + half] = r1;
      }
    }
  };
  if (b.rope) {
    for (int n = 0; n < N; n++) {
      for (int h = 0; h < nh; h++) rope(q, nh, h, n);
      for (int h = 0; h < nkv; h++) rope(k, nkv, h, n);
    }
  }
  const float scalef = 1.0f / std::sqrt((float)hd);
  T scale = T(scalef);
  std::vector<T> o(R * nh * vhd, T(0));
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < N; n++)
    for (int h = 0; h < nh; h++) {
      int kvh = h / g;
      std::vector<T> sc(S);
      for (int qi = 0; qi < S; qi++) {
        const T* qp = &q[(((size_t)n * S + qi) * nh + h) * hd];
        T mx = -INFINITY;
        for (int ki = 0; ki < S; ki++) {
          const T* kp = &k[(((size_t)n * S + ki) * nkv + kvh) * hd];
          T d = 0;
          for (int j = 0; j < hd; j++) d += qp[j] * kp[j];
          T biasv = cx.mask[(size_t)n * S + ki] * T(3e4f) - T(3e4f);
          d = d * scale + biasv;
          sc[ki] = d;
          mx = d > mx ? d : mx;
        }
        T sum = 0;
        for (int ki = 0; ki < S; ki++) { sc[ki] = std::exp(sc[ki] - mx); sum += sc[ki]; }
        T* op = &o[(((size_t)n * S + qi) * nh + h) * vhd];
        for (int ki = 0; ki < S; ki++) {
          T pw = sc[ki] / sum;
          const T* vp = &v[(((size_t)n * S + ki) * nkv + kvh) * vhd];
          for (int j = 0; j < vhd; j++) op[j] += pw * vp[j];
        }
      }
    }
  auto y = tok_matmul(o, R, b.out);
  for (size_t r = 0; r < R; r++)
    for (int c = 0; c < C; c++) x[r * C + c] += y[r * C + c] * cx.mask[r];
}

template <typename T>
static void ffn_block(std::vector<T>& x, const Ctx<T>& cx, const Block& b, int C) {
  size_t R = (size_t)cx.N * S;
  auto xn = tf_rms(x, cx, b.ln);
  auto a = tok_matmul(xn, R, b.w1);
  auto gt = tok_matmul(xn, R, b.wg);
  for (size_t i = 0; i < a.size(); i++) a[i] = act(a[i], ACT_SILU) * gt[i];
  auto y = tok_matmul(a, R, b.w2);
  for (size_t r = 0; r < R; r++)
    for (int c = 0; c < C; c++) x[r * C + c] += y[r * C + c] * cx.mask[r];
}

template <typename T>
static std::vector<T> block_stack(std::vector<T> x, const Ctx<T>& cx, const std::vector<Block>& blocks, int C);

template <typename T>
static std::vector<T> apply_block(const std::vector<T>& x, const Ctx<T>& cx, const Block& b, int C) {
  int N = cx.N;
  if (b.kind == K_ORD) {
    auto t = x;
    bn_act_mask(t, cx, b.pre_bn, b.pre_act);
    t = conv(t, N, b.regular);
    bn_act_mask(t, cx, b.mid_bn, b.mid_act);
    t = conv(t, N, b.final_conv);
    add(t, x);
    return t;
  }
  if (b.kind == K_GPOOL) {
    auto t = x;
    bn_act_mask(t, cx, b.pre_bn, b.pre_act);
    auto reg = conv(t, N, b.regular);
    auto g = conv(t, N, b.gpool_conv);
    bn_act_mask(g, cx, b.gpool_bn, b.gpool_act);
    auto pooled = gpool(g, cx, b.gpool_bn.c);
    auto bias = matmul(pooled, N, b.gpool_to_bias);
    add_nc_bias(reg, N, b.gpool_to_bias.oc, bias);
    bn_act_mask(reg, cx, b.mid_bn, b.mid_act);
    reg = conv(reg, N, b.final_conv);
    add(reg, x);
    return reg;
  }
  if (b.kind == K_NESTED) {
    auto t = x;
    bn_act_mask(t, cx, b.pre_bn, b.pre_act);
    t = conv(t, N, b.pre_conv);
    t = block_stack(t, cx, b.inner, b.pre_conv.oc);
    bn_act_mask(t, cx, b.post_bn, b.post_act);
    t = conv(t, N, b.post_conv);
    add(t, x);
    return t;
  }
  throw std::runtime_error("apply_block: transformer block outside a token run");
}

template <typename T>
static std::vector<T> block_stack(std::vector<T> x, const Ctx<T>& cx, const std::vector<Block>& blocks, int C) {
  bool tokens = false;
  for (const Block& b : blocks) {
    bool tf = b.kind == K_ATTN || b.kind == K_FFN;
    if (tf && !tokens) { x = to_tokens(x, cx.N, C); tokens = true; }
    else if (!tf && tokens) { x = to_nchw(x, cx.N, C); tokens = false; }
    if (b.kind == K_ATTN) attention_block(x, cx, b, C);
    else if (b.kind == K_FFN) ffn_block(x, cx, b, C);
    else x = apply_block(x, cx, b, C);
  }
  if (tokens) x = to_nchw(x, cx.N, C);
  return x;
}

template <typename T>
static void forward(const Model& m, int N, const float* bin, const float* glob, const float* meta,
                    float* policy, float* value, float* score, float* own) {
  Ctx<T> cx; cx.N = N;
  cx.mask.resize((size_t)N * S); cx.mask_sum.resize(N); cx.scale1.resize(N); cx.scale2.resize(N);
  for (int n = 0; n < N; n++) {
    T s = 0;
    for (int i = 0; i < S; i++) { cx.mask[(size_t)n * S + i] = T(bin[((size_t)n * m.n_in) * S + i]); s += cx.mask[(size_t)n * S + i]; }
    cx.mask_sum[n] = s;
    T cen = std::sqrt(s) - T(14.0f);
    cx.scale1[n] = cen * T(0.1f);
    T sq = cen * cen;
    sq = sq * T(0.01f);
    cx.scale2[n] = sq - T(0.1f);
  }
  int C = m.trunk_c;
  std::vector<T> in((size_t)N * m.n_in * S);
  for (size_t i = 0; i < in.size(); i++) in[i] = T(bin[i]);
  auto x = conv(in, N, m.initial_conv);
  std::vector<T> g((size_t)N * m.n_glob);
  for (size_t i = 0; i < g.size(); i++) g[i] = T(glob[i]);
  add_nc_bias(x, N, C, matmul(g, N, m.initial_matmul));
  if (m.has_meta) {
    std::vector<T> mi((size_t)N * m.n_meta);
    for (size_t i = 0; i < mi.size(); i++) mi[i] = T(meta[i]);
    auto h = matmul(mi, N, m.m1); matbias(h, N, m.mb1); for (auto& v : h) v = act(v, m.ma1);
    h = matmul(h, N, m.m2); matbias(h, N, m.mb2); for (auto& v : h) v = act(v, m.ma2);
    h = matmul(h, N, m.m3);
    add_nc_bias(x, N, C, h);
  }
  x = block_stack(x, cx, m.blocks, C);
  // trunk tip
  if (!m.tip_rms) {
    bn_act_mask(x, cx, m.tip_bn, m.tip_act);
  } else {
    for (int n = 0; n < N; n++) {
      std::vector<T> rms(S);
      if (!m.tip_spatial) {
        for (int i = 0; i < S; i++) {
          T ss = 0;
          for (int c = 0; c < C; c++) { T v = x[((size_t)n * C + c) * S + i]; ss += v * v; }
          T ms = ss / T(float(C));
          T den = std::sqrt(ms + T(m.tip_eps));
          rms[i] = T(1) / den;
        }
      } else {
        // ReduceSum over C x 361 terms: blocked (one partial per channel, then the partials), as a vectorised
        // reduction sums, rather than one running float32 sum whose rounding error grows with the 277k terms
        T ss = 0;
        for (int c = 0; c < C; c++) {
          T part = 0;
          for (int i = 0; i < S; i++) { T v = x[((size_t)n * C + c) * S + i]; part += (v * v) * cx.mask[(size_t)n * S + i]; }
          ss += part;
        }
        T count = cx.mask_sum[n] * T(float(C));
        T ms = ss / count;
        T den = std::sqrt(ms + T(m.tip_eps));
        for (int i = 0; i < S; i++) rms[i] = T(1) / den;
      }
      for (int c = 0; c < C; c++)
        for (int i = 0; i < S; i++) {
          T& v = x[((size_t)n * C + c) * S + i];
          T y = v * rms[i];
          y = y * T(m.tip_gamma[c]);
          y = y + T(m.tip_beta[c]);
          v = act(y, m.tip_act) * cx.mask[(size_t)n * S + i];
        }
    }
  }
  // policy head
  auto p1 = conv(x, N, m.p1);
  auto g1 = conv(x, N, m.g1);
  bn_act_mask(g1, cx, m.g1_bn, m.g1_act);
  auto g1p = gpool(g1, cx, m.g1_bn.c);
  add_nc_bias(p1, N, m.p1.oc, matmul(g1p, N, m.gpool_to_bias_p));
  bn_act_mask(p1, cx, m.p1_bn, m.p1_act);
  auto p2 = conv(p1, N, m.p2);
  std::vector<T> pass;
  if (m.pass_mlp) {
    pass = matmul(g1p, N, m.pass_mul); matbias(pass, N, m.pass_bias);
    for (auto& v : pass) v = act(v, m.pass_act);
    pass = matmul(pass, N, m.pass_mul2);
  } else {
    pass = matmul(g1p, N, m.pass_mul);
  }
  for (int n = 0; n < N; n++)
    for (int p = 0; p < m.P; p++) {
      for (int i = 0; i < S; i++) policy[((size_t)n * m.P + p) * (S + 1) + i] = (float)p2[((size_t)n * m.P + p) * S + i];
      policy[((size_t)n * m.P + p) * (S + 1) + S] = (float)pass[(size_t)n * m.P + p];
    }
  // value head
  auto v1 = conv(x, N, m.v1);
  bn_act_mask(v1, cx, m.v1_bn, m.v1_act);
  auto vp = value_pool(v1, cx, m.v1_bn.c);
  auto v2 = matmul(vp, N, m.v2); matbias(v2, N, m.v2b);
  for (auto& v : v2) v = act(v, m.v2_act);
  auto v3 = matmul(v2, N, m.v3); matbias(v3, N, m.v3b);
  auto sv = matmul(v2, N, m.sv3); matbias(sv, N, m.sv3b);
  auto ow = conv(v1, N, m.own);
  for (size_t i = 0; i < v3.size(); i++) value[i] = (float)v3[i];
  for (size_t i = 0; i < sv.size(); i++) score[i] = (float)sv[i];
  for (size_t i = 0; i < ow.size(); i++) own[i] = (float)ow[i];
}

}  // namespace orc

// --------------------------------------------------------------------------------------------------------------
// C ABI for ctypes (tests, smoke, bench cpu_baseline)
// --------------------------------------------------------------------------------------------------------------

extern "C" {

void* orc_load(const uint8_t* bytes, size_t n, char* err, int errlen) {
  try {
    return new orc::Model(orc::parse_model(bytes, n));
  } catch (const std::exception& e) {
    if (err && errlen > 0) { std::snprintf(err, errlen, "%s", e.what()); }
    return nullptr;
  }
}

void orc_free(void* m) { delete (orc::Model*)m; }

// dims: [version, n_in, n_glob, n_meta, P, n_value, n_score, n_own, trunk_c]
void orc_dims(void* mp, int* d) {
  auto* m = (orc::Model*)mp;
  d[0] = m->version; d[1] = m->n_in; d[2] = m->n_glob; d[3] = m->n_meta; d[4] = m->P;
  d[5] = m->v3.oc; d[6] = m->sv3.oc; d[7] = m->own.oc; d[8] = m->trunk_c;
}

int orc_forward(void* mp, int n, const float* bin, const float* glob, const float* meta, int use_double, int threads,
                float* policy, float* value, float* score, float* own, char* err, int errlen) {
  try {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    auto* m = (orc::Model*)mp;
    if (use_double) orc::forward<double>(*m, n, bin, glob, meta, policy, value, score, own);
    else orc::forward<float>(*m, n, bin, glob, meta, policy, value, score, own);
    return 0;
  } catch (const std::exception& e) {
    if (err && errlen > 0) { std::snprintf(err, errlen, "%s", e.what()); }
    return 1;
  }
}

}  // extern "C"
