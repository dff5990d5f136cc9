// ONNX model loading: a KataGo net exported by the reference's tools/bin2onnx/bin2onnx.py (build_onnx :1571-1615)
// is read back into the same ModelDesc the .bin parser produces, so that the engine plans it identically.
//
// The file is protobuf (the public onnx.proto schema: ModelProto, GraphProto, NodeProto, TensorProto,
// AttributeProto, StringStringEntryProto), decoded here from the wire format. The graph holds no layer list:
// GraphBuilder (:1088-1531) writes each layer as a fixed sequence of nodes (batch norms already merged into
// per-channel Mul / Add initializers, activations as op patterns), in a fixed order per block kind. The parser walks
// the node list in that order, checking each node's op and wiring, and rebuilds the blocks; where two block kinds
// begin alike (a residual block, a nested bottleneck block, the trunk tip) it tries one and backs up, since every
// block ends with the residual Add whose first input is the block's input.

#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "common.h"
#include "model.h"

namespace kc {

namespace {

[[noreturn]] void bad(const std::string& m) { fail(KC_ERR_PARSE, "ONNX model: " + m); }

// ---- protobuf wire format ----

struct Pb {
  const uint8_t* p;
  const uint8_t* e;
  bool more() const { return p < e; }
  uint64_t varint() {
    uint64_t v = 0;
    for (int s = 0; s < 64; s += 7) {
      if (p >= e) bad("truncated varint");
      const uint8_t b = *p++;
      v |= (uint64_t)(b & 0x7F) << s;
      if (!(b & 0x80)) return v;
    }
    bad("varint too long");
  }
  Pb sub() {  // a length-delimited field's bytes
    const uint64_t n = varint();
    if (n > (uint64_t)(e - p)) bad("truncated field");
    Pb r{p, p + n};
    p += n;
    return r;
  }
  std::string str() {
    Pb s = sub();
    return std::string(reinterpret_cast<const char*>(s.p), s.e - s.p);
  }
  uint32_t fixed32() {
    if (e - p < 4) bad("truncated fixed32");
    uint32_t v;
    std::memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  void skip(int wire) {
    switch (wire) {
      case 0: varint(); break;
      case 1:
        if (e - p < 8) bad("truncated fixed64");
        p += 8;
        break;
      case 2: sub(); break;
      case 5: fixed32(); break;
      default: bad("unsupported wire type " + std::to_string(wire));
    }
  }
};

struct Attr {
  std::string name;
  int64_t i = 0;
  float f = 0;
  std::vector<int64_t> ints;
};

struct Node {
  std::string op, name;
  std::vector<std::string> in, out;
  std::vector<Attr> attrs;
  const Attr* attr(const char* n) const {
    for (auto& a : attrs)
      if (a.name == n) return &a;
    return nullptr;
  }
};

struct Tensor {
  std::vector<int64_t> dims;
  int type = 0;  // TensorProto.DataType: 1 FLOAT, 7 INT64
  std::vector<float> f;
  std::vector<int64_t> i64;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct Graph {
  std::vector<Node> nodes;
  std::map<std::string, Tensor> inits;
  std::map<std::string, std::string> meta;
};

void read_packed_ints(Pb& f, int wire, std::vector<int64_t>& v) {
  if (wire == 2) {
    Pb s = f.sub();
    while (s.more()) v.push_back((int64_t)s.varint());
  } else {
    v.push_back((int64_t)f.varint());
  }
}

Attr read_attr(Pb b) {
  Attr a;
  while (b.more()) {
    const uint64_t key = b.varint();
    const int field = (int)(key >> 3), wire = (int)(key & 7);
    if (field == 1 && wire == 2) a.name = b.str();
    else if (field == 2 && wire == 5) {
      const uint32_t u = b.fixed32();
      std::memcpy(&a.f, &u, 4);
    } else if (field == 3 && wire == 0) a.i = (int64_t)b.varint();
    else if (field == 8) read_packed_ints(b, wire, a.ints);
    else b.skip(wire);
  }
  return a;
}

Node read_node(Pb b) {
  Node n;
  while (b.more()) {
    const uint64_t key = b.varint();
    const int field = (int)(key >> 3), wire = (int)(key & 7);
    if (field == 1 && wire == 2) n.in.push_back(b.str());
    else if (field == 2 && wire == 2) n.out.push_back(b.str());
    else if (field == 3 && wire == 2) n.name = b.str();
    else if (field == 4 && wire == 2) n.op = b.str();
    else if (field == 5 && wire == 2) n.attrs.push_back(read_attr(b.sub()));
    else b.skip(wire);
  }
  return n;
}

void read_tensor(Pb b, Graph& g) {
  Tensor t;
  std::string name;
  Pb raw{nullptr, nullptr};
  while (b.more()) {
    const uint64_t key = b.varint();
    const int field = (int)(key >> 3), wire = (int)(key & 7);
    if (field == 1) read_packed_ints(b, wire, t.dims);
    else if (field == 2 && wire == 0) t.type = (int)b.varint();
    else if (field == 4) {  // float_data
      if (wire == 2) {
        Pb s = b.sub();
        while (s.more()) {
          const uint32_t u = s.fixed32();
          float x;
          std::memcpy(&x, &u, 4);
          t.f.push_back(x);
        }
      } else {
        const uint32_t u = b.fixed32();
        float x;
        std::memcpy(&x, &u, 4);
        t.f.push_back(x);
      }
    } else if (field == 7) read_packed_ints(b, wire, t.i64);
    else if (field == 8 && wire == 2) name = b.str();
    else if (field == 9 && wire == 2) raw = b.sub();
    else b.skip(wire);
  }
  const int64_t n = t.numel();
  if (raw.p) {  // raw_data: little-endian values
    const size_t bytes = raw.e - raw.p;
    if (t.type == 1) {
      if (bytes != (size_t)n * 4) bad(name + ": raw_data size does not match its dims");
      t.f.resize(n);
      std::memcpy(t.f.data(), raw.p, bytes);
    } else if (t.type == 7) {
      if (bytes != (size_t)n * 8) bad(name + ": raw_data size does not match its dims");
      t.i64.resize(n);
      std::memcpy(t.i64.data(), raw.p, bytes);
    } else {
      bad(name + ": unsupported tensor type " + std::to_string(t.type));
    }
  }
  if (t.type == 1 && (int64_t)t.f.size() != n) bad(name + ": float data size does not match its dims");
  if (t.type == 7 && (int64_t)t.i64.size() != n) bad(name + ": int64 data size does not match its dims");
  g.inits[name] = std::move(t);
}

Graph read_model(const uint8_t* data, size_t n) {
  Graph g;
  Pb m{data, data + n};
  bool have_graph = false;
  while (m.more()) {
    const uint64_t key = m.varint();
    const int field = (int)(key >> 3), wire = (int)(key & 7);
    if (field == 7 && wire == 2) {  // graph
      have_graph = true;
      Pb gb = m.sub();
      while (gb.more()) {
        const uint64_t k2 = gb.varint();
        const int f2 = (int)(k2 >> 3), w2 = (int)(k2 & 7);
        if (f2 == 1 && w2 == 2) g.nodes.push_back(read_node(gb.sub()));
        else if (f2 == 5 && w2 == 2) read_tensor(gb.sub(), g);
        else gb.skip(w2);
      }
    } else if (field == 14 && wire == 2) {  // metadata_props
      Pb e = m.sub();
      std::string k, v;
      while (e.more()) {
        const uint64_t k3 = e.varint();
        const int f3 = (int)(k3 >> 3), w3 = (int)(k3 & 7);
        if (f3 == 1 && w3 == 2) k = e.str();
        else if (f3 == 2 && w3 == 2) v = e.str();
        else e.skip(w3);
      }
      g.meta[k] = v;
    } else {
      m.skip(wire);
    }
  }
  if (!have_graph) bad("no graph");
  return g;
}

// ---- the graph, read back into layers ----

// Thrown when the nodes at the cursor do not follow the pattern being tried; the caller backs up.
struct Mismatch {};

std::string strip(const std::string& s, const char* suffix) {
  const size_t k = std::strlen(suffix);
  return s.size() > k && s.compare(s.size() - k, k, suffix) == 0 ? s.substr(0, s.size() - k) : s;
}

struct Parser {
  const Graph& g;
  size_t pos = 0;
  std::string mask, mask_sum, mask_tok, attn_bias;

  explicit Parser(const Graph& gr) : g(gr) {}

  [[noreturn]] static void miss() { throw Mismatch{}; }
  const Node& at(size_t off = 0) const {
    if (pos + off >= g.nodes.size()) miss();
    return g.nodes[pos + off];
  }
  bool is(const char* op, size_t off = 0) const {
    return pos + off < g.nodes.size() && g.nodes[pos + off].op == op;
  }
  const Node& take(const char* op) {
    const Node& n = at();
    if (n.op != op || n.out.empty()) miss();
    pos++;
    return n;
  }
  // take a node of `op` whose first inputs are exactly `ins` (empty strings match anything)
  const Node& take(const char* op, std::initializer_list<std::string> ins) {
    const Node& n = take(op);
    size_t i = 0;
    for (const std::string& want : ins) {
      if (i >= n.in.size() || (!want.empty() && n.in[i] != want)) miss();
      i++;
    }
    return n;
  }
  const Tensor* init(const std::string& name) const {
    auto it = g.inits.find(name);
    return it == g.inits.end() ? nullptr : &it->second;
  }
  const Tensor& finit(const std::string& name) const {  // a float initializer
    const Tensor* t = init(name);
    if (!t || t->type != 1) miss();
    return *t;
  }
  float scalar(const std::string& name) const {
    const Tensor& t = finit(name);
    if (t.f.size() != 1) miss();
    return t.f[0];
  }
  std::vector<int64_t> ints(const std::string& name) const {
    const Tensor* t = init(name);
    if (!t || t->type != 7) miss();
    return t->i64;
  }

  // ---- layers (GraphBuilder conv / activation / bn_act_mask / matmul / matbias, bin2onnx.py:1135-1186) ----
  std::string conv(const std::string& x, ConvDesc& c) {
    const Node& n = take("Conv", {x, ""});
    const Tensor& w = finit(n.in[1]);
    if (w.dims.size() != 4) miss();
    c.name = n.name;
    c.oc = (int)w.dims[0];
    c.ic = (int)w.dims[1];
    c.ky = (int)w.dims[2];
    c.kx = (int)w.dims[3];
    c.dy = c.dx = 1;
    if (const Attr* d = n.attr("dilations")) {
      if (d->ints.size() == 2) {
        c.dy = (int)d->ints[0];
        c.dx = (int)d->ints[1];
      }
    }
    // ONNX [oc][ic][ky][kx] -> the file order [ky][kx][ic][oc]
    c.w.assign(w.f.size(), 0.0f);
    for (int o = 0; o < c.oc; o++)
      for (int i = 0; i < c.ic; i++)
        for (int y = 0; y < c.ky; y++)
          for (int xx = 0; xx < c.kx; xx++)
            c.w[(((size_t)y * c.kx + xx) * c.ic + i) * c.oc + o] =
                w.f[(((size_t)o * c.ic + i) * c.ky + y) * c.kx + xx];
    return n.out[0];
  }
  std::string act(const std::string& x, Act& a) {
    if (is("Relu") && at().in.size() == 1 && at().in[0] == x) {
      a = ACT_RELU;
      return take("Relu").out[0];
    }
    if (is("Softplus") && at().in[0] == x) {  // mish: x * tanh(softplus(x))
      const Node& sp = take("Softplus", {x});
      const Node& th = take("Tanh", {sp.out[0]});
      const Node& m = take("Mul", {x, th.out[0]});
      a = ACT_MISH;
      return m.out[0];
    }
    if (is("Mul") && is("Exp", 1) && at().in.size() == 2 && at().in[0] == x && init(at().in[1])) {  // SiLU
      const Node& neg = take("Mul", {x, ""});
      if (scalar(neg.in[1]) != -1.0f) miss();
      const Node& e = take("Exp", {neg.out[0]});
      const Node& d = take("Add", {e.out[0], ""});
      if (scalar(d.in[1]) != 1.0f) miss();
      const Node& q = take("Div", {x, d.out[0]});
      a = ACT_SILU;
      return q.out[0];
    }
    a = ACT_IDENTITY;
    return x;
  }
  std::string bn_act_mask(const std::string& x, BNDesc& bn, Act& a) {
    const Node& m = take("Mul", {x, ""});
    const Tensor& sc = finit(m.in[1]);
    const Node& ad = take("Add", {m.out[0], ""});
    const Tensor& bi = finit(ad.in[1]);
    if (sc.f.size() != bi.f.size() || sc.f.empty()) miss();
    bn.name = strip(m.name, ".mul");
    bn.c = (int)sc.f.size();
    bn.merged_scale = sc.f;
    bn.merged_bias = bi.f;
    const std::string y = act(ad.out[0], a);
    return take("Mul", {y, mask}).out[0];
  }
  std::string matmul(const std::string& x, MatMulDesc& mm) {
    const Node& n = take("MatMul", {x, ""});
    const Tensor& w = finit(n.in[1]);
    if (w.dims.size() != 2) miss();
    mm.name = n.name;
    mm.ic = (int)w.dims[0];
    mm.oc = (int)w.dims[1];
    mm.w = w.f;
    return n.out[0];
  }
  std::string matbias(const std::string& x, MatBiasDesc& mb) {
    const Node& n = take("Add", {x, ""});
    const Tensor& b = finit(n.in[1]);
    mb.name = n.name;
    mb.c = (int)b.f.size();
    mb.b = b.f;
    return n.out[0];
  }
  std::string reshape(const std::string& x) { return take("Reshape", {x, ""}).out[0]; }
  // gpool (:1222-1230) and value_pool (:1232-1239)
  std::string gpool(const std::string& x) {
    const std::string f = reshape(x);
    const Node& s = take("ReduceSum", {f, ""});
    const Node& mean = take("Div", {s.out[0], mask_sum});
    const Node& ms = take("Mul", {mean.out[0], ""});
    const Node& sh = take("Add", {f, ""});
    const Node& mx = take("ReduceMax", {sh.out[0]});
    return take("Concat", {mean.out[0], ms.out[0], mx.out[0]}).out[0];
  }
  std::string value_pool(const std::string& x) {
    const std::string f = reshape(x);
    const Node& s = take("ReduceSum", {f, ""});
    const Node& mean = take("Div", {s.out[0], mask_sum});
    const Node& m1 = take("Mul", {mean.out[0], ""});
    const Node& m2 = take("Mul", {mean.out[0], ""});
    return take("Concat", {mean.out[0], m1.out[0], m2.out[0]}).out[0];
  }

  // ---- blocks (residual_block, gpool_block, nested_bottleneck_block :1243-1269) ----
  std::string close(const std::string& x, const std::string& r, BlockDesc& b, BlockDesc& out) {
    const Node& ad = take("Add", {x, r});
    b.name = strip(ad.name, ".residual");
    out = std::move(b);
    return ad.out[0];
  }
  std::string conv_block(const std::string& x, BlockDesc& out) {
    BlockDesc b;
    const std::string pre = bn_act_mask(x, b.pre_bn, b.pre_act);
    ConvDesc c1;
    const std::string y1 = conv(pre, c1);
    const size_t after_c1 = pos;
    if (is("Conv") && at().in[0] == pre) {  // a second conv of the same input: global pooling block
      b.kind = BLOCK_GPOOL;
      b.regular = std::move(c1);
      std::string t = conv(pre, b.gpool_conv);
      t = bn_act_mask(t, b.gpool_bn, b.gpool_act);
      t = gpool(t);
      t = matmul(t, b.gpool_to_bias);
      t = reshape(t);
      const Node& ad = take("Add", {y1, t});
      std::string r = bn_act_mask(ad.out[0], b.mid_bn, b.mid_act);
      r = conv(r, b.final_conv);
      return close(x, r, b, out);
    }
    try {  // an ordinary residual block: batch norm, conv, then the residual add of the block's input
      BlockDesc o = b;
      o.kind = BLOCK_ORDINARY;
      o.regular = c1;
      std::string r = bn_act_mask(y1, o.mid_bn, o.mid_act);
      r = conv(r, o.final_conv);
      return close(x, r, o, out);
    } catch (const Mismatch&) {
      pos = after_c1;
    }
    b.kind = BLOCK_NESTED;  // else a nested bottleneck: the 1x1 pre conv, an inner stack, post BN-act, 1x1 post conv
    b.pre_conv = std::move(c1);
    std::string r = block_stack(y1, b.inner);
    if (b.inner.empty()) miss();
    r = bn_act_mask(r, b.post_bn, b.post_act);
    r = conv(r, b.post_conv);
    return close(x, r, b, out);
  }

  // ---- transformer blocks (:1313-1438), on tokens ----
  void token_masks() {  // setup_token_masks, emitted inside the first transformer block
    if (!mask_tok.empty() || !is("Reshape") || at().in.empty() || at().in[0] != mask) return;
    const Node& mt = take("Reshape", {mask, ""});
    const Node& mk = take("Reshape", {mask, ""});
    const Node& sc = take("Mul", {mk.out[0], ""});
    const Node& b = take("Sub", {sc.out[0], ""});
    mask_tok = mt.out[0];
    attn_bias = b.out[0];
  }
  std::string rmsnorm(const std::string& x, TfRmsDesc& d) {
    const Node& sq = take("Mul", {x, x});
    const Node& ss = take("ReduceSum", {sq.out[0], ""});
    const Node& ms = take("Div", {ss.out[0], ""});
    const Node& den = take("Add", {ms.out[0], ""});
    d.eps = scalar(den.in[1]);
    const Node& sr = take("Sqrt", {den.out[0]});
    const Node& rms = take("Div", {"", sr.out[0]});
    const Node& y = take("Mul", {x, rms.out[0]});
    const Node& w = take("Mul", {y.out[0], ""});
    d.w = finit(w.in[1]).f;
    d.c = (int)d.w.size();
    return take("Mul", {w.out[0], mask_tok}).out[0];
  }
  // heads(): Reshape [-1, S, heads, dim] + Transpose; returns the head count and dim
  std::string heads(const std::string& t, int& nh, int& dim) {
    const Node& r = take("Reshape", {t, ""});
    const std::vector<int64_t> shape = ints(r.in[1]);
    if (shape.size() != 4) miss();
    nh = (int)shape[2];
    dim = (int)shape[3];
    return take("Transpose", {r.out[0]}).out[0];
  }
  // rope(): two Slices, x0 cos - x1 sin, x0 sin + x1 cos, Concat; returns the cos / sin initializers
  std::string rope(const std::string& x, std::string& cos, std::string& sin) {
    const Node& x0 = take("Slice", {x, "", "", ""});
    const Node& x1 = take("Slice", {x, "", "", ""});
    const Node& a = take("Mul", {x0.out[0], ""});
    const Node& b = take("Mul", {x1.out[0], ""});
    const Node& r0 = take("Sub", {a.out[0], b.out[0]});
    const Node& c = take("Mul", {x0.out[0], b.in[1]});
    const Node& d = take("Mul", {x1.out[0], a.in[1]});
    const Node& r1 = take("Add", {c.out[0], d.out[0]});
    cos = a.in[1];
    sin = b.in[1];
    return take("Concat", {r0.out[0], r1.out[0]}).out[0];
  }
  std::string attention(const std::string& x, BlockDesc& out) {
    BlockDesc b;
    b.kind = BLOCK_ATTENTION;
    token_masks();
    const std::string xn = rmsnorm(x, b.ln);
    const std::string q = matmul(xn, b.q), k = matmul(xn, b.k), v = matmul(xn, b.v);
    int qd = 0, kd = 0;
    std::string qh = heads(q, b.heads, qd), kh = heads(k, b.kv_heads, kd), vh = heads(v, b.kv_heads, b.v_head_dim);
    b.head_dim = qd;
    if (kd != qd || b.heads % b.kv_heads != 0) miss();
    if (is("Slice") && at().in[0] == qh) {
      b.use_rope = true;
      std::string cq, sq, ck, sk;
      qh = rope(qh, cq, sq);
      kh = rope(kh, ck, sk);
      // tables per KV head: the K tables (learnable RoPE with fewer KV heads), else the Q tables ([1, T, S, P],
      // T = 1 for a fixed theta, T = heads otherwise)
      const Tensor& c = finit(ck);
      const Tensor& s = finit(sk);
      if (c.dims.size() != 4 || c.dims[2] != 361 || c.dims[3] != qd / 2 || s.f.size() != c.f.size()) miss();
      b.rope_ntables = (int)c.dims[1];
      if (b.rope_ntables != 1 && b.rope_ntables != b.kv_heads) miss();
      b.learnable_rope = b.rope_ntables > 1;
      b.rope_cos = c.f;
      b.rope_sin = s.f;
      // the export permuted each head's Q / K columns to [x0 of every pair..., x1 of every pair...] (:1369-1374);
      // the layer keeps the file's interleaved order
      auto unpermute = [&](MatMulDesc& m, int nheads) {
        std::vector<float> w(m.w.size());
        for (int i = 0; i < m.ic; i++)
          for (int h = 0; h < nheads; h++)
            for (int j = 0; j < qd; j++) {
              const int src = j < qd / 2 ? 2 * j : 2 * (j - qd / 2) + 1;
              w[(size_t)i * m.oc + h * qd + src] = m.w[(size_t)i * m.oc + h * qd + j];
            }
        m.w = std::move(w);
      };
      unpermute(b.q, b.heads);
      unpermute(b.k, b.kv_heads);
    }
    if (b.heads != b.kv_heads) qh = reshape(qh);
    const Node& kt = take("Transpose", {kh});
    const Node& sc = take("MatMul", {qh, kt.out[0]});
    const Node& sm = take("Mul", {sc.out[0], ""});
    const Node& mb = take("Add", {sm.out[0], attn_bias});
    const Node& pr = take("Softmax", {mb.out[0]});
    std::string o = take("MatMul", {pr.out[0], vh}).out[0];
    if (b.heads != b.kv_heads) o = reshape(o);
    o = take("Transpose", {o}).out[0];
    o = reshape(o);
    o = matmul(o, b.out);
    o = take("Mul", {o, mask_tok}).out[0];
    return close(x, o, b, out);
  }
  std::string ffn(const std::string& x, BlockDesc& out) {
    BlockDesc b;
    b.kind = BLOCK_FFN;
    token_masks();
    const std::string xn = rmsnorm(x, b.ln);
    const std::string a = matmul(xn, b.w1), gt = matmul(xn, b.wgate);
    Act sa;
    const std::string s = act(a, sa);
    if (sa != ACT_SILU) miss();
    std::string o = take("Mul", {s, gt}).out[0];
    o = matmul(o, b.w2);
    o = take("Mul", {o, mask_tok}).out[0];
    b.ffn = b.w1.oc;
    return close(x, o, b, out);
  }

  // block_stack (:1271-1300): blocks until the next nodes are no block of this stack's stream
  std::string block_stack(std::string x, std::vector<BlockDesc>& blocks) {
    bool tokens = false;
    while (true) {
      const size_t save = pos;
      const std::string x_save = x;
      const bool tokens_save = tokens;
      try {
        std::string y = x;
        bool tf = false;
        if (!tokens && is("Reshape") && is("Transpose", 1) && at().in[0] == y) {
          y = take("Transpose", {reshape(y)}).out[0];  // into tokens
          tokens = tf = true;
        } else if (tokens) {
          const bool masks_next = mask_tok.empty() && is("Reshape") && at().in[0] == mask;
          const bool norm_next = is("Mul") && at().in.size() == 2 && at().in[0] == y && at().in[1] == y;
          if (masks_next || norm_next) {
            tf = true;
          } else {
            y = reshape(take("Transpose", {y}).out[0]);  // back to NCHW
            tokens = false;
          }
        }
        BlockDesc b;
        if (tf) {
          const size_t p0 = pos;
          try {
            y = attention(y, b);
          } catch (const Mismatch&) {
            pos = p0;
            y = ffn(y, b);
          }
        } else {
          y = conv_block(y, b);
        }
        blocks.push_back(std::move(b));
        x = y;
      } catch (const Mismatch&) {
        pos = save;
        x = x_save;
        tokens = tokens_save;
        break;
      }
    }
    if (tokens) x = reshape(take("Transpose", {x}).out[0]);
    return x;
  }

  // ---- the whole graph: setup_mask, trunk, policy head, value head (:1202-1220, :1477-1531) ----
  void model(ModelDesc& m) {
    const Node& sl = take("Slice", {"bin_input", "", "", ""});
    mask = sl.out[0];
    const std::string mflat = reshape(mask);
    mask_sum = take("ReduceSum", {mflat, ""}).out[0];
    const char* rest[] = {"Sqrt", "Sub", "Mul", "Mul", "Mul", "Sub", "Mul", "Sub"};  // pool scales, max-pool bias
    for (const char* op : rest) take(op);
    // trunk
    std::string x = conv("bin_input", m.initial_conv);
    std::string gl = reshape(matmul("global_input", m.initial_matmul));
    x = take("Add", {x, gl}).out[0];
    if (is("MatMul") && at().in[0] == "meta_input") {
      m.has_meta = true;
      std::string t = matbias(matmul("meta_input", m.meta_mul1), m.meta_bias1);
      t = act(t, m.meta_act1);
      t = matbias(matmul(t, m.meta_mul2), m.meta_bias2);
      t = act(t, m.meta_act2);
      t = reshape(matmul(t, m.meta_mul3));
      x = take("Add", {x, t}).out[0];
    }
    x = block_stack(x, m.blocks);
    if (is("Mul") && at().in.size() == 2 && at().in[0] == x && at().in[1] == x) {  // RMSNorm tip (:1440-1463)
      m.trunk_norm_kind = 1;
      const Node& sq = take("Mul", {x, x});
      std::string ms;
      if (is("Mul") && at().in[0] == sq.out[0]) {
        m.tip_rms_spatial = true;
        const Node& ob = take("Mul", {sq.out[0], mask});
        const Node& ss = take("ReduceSum", {reshape(ob.out[0]), ""});
        const Node& cnt = take("Mul", {mask_sum, ""});
        ms = reshape(take("Div", {ss.out[0], cnt.out[0]}).out[0]);
      } else {
        const Node& ss = take("ReduceSum", {sq.out[0], ""});
        ms = take("Div", {ss.out[0], ""}).out[0];
      }
      const Node& den = take("Add", {ms, ""});
      m.tip_rms_eps = scalar(den.in[1]);
      const Node& sr = take("Sqrt", {den.out[0]});
      const Node& rms = take("Div", {"", sr.out[0]});
      const Node& y = take("Mul", {x, rms.out[0]});
      const Node& ga = take("Mul", {y.out[0], ""});
      const Node& be = take("Add", {ga.out[0], ""});
      m.tip_rms_gamma = finit(ga.in[1]).f;
      m.tip_rms_beta = finit(be.in[1]).f;
      x = take("Mul", {act(be.out[0], m.tip_act), mask}).out[0];
    } else {
      x = bn_act_mask(x, m.tip_bn, m.tip_act);
    }
    // policy head
    const std::string p1 = conv(x, m.p1_conv);
    std::string g1 = conv(x, m.g1_conv);
    g1 = bn_act_mask(g1, m.g1_bn, m.g1_act);
    const std::string gp = gpool(g1);
    const std::string pb = reshape(matmul(gp, m.gpool_to_bias_mul));
    std::string p = take("Add", {p1, pb}).out[0];
    p = bn_act_mask(p, m.p1_bn, m.p1_act);
    const std::string p2 = conv(p, m.p2_conv);
    std::string pass = matmul(gp, m.gpool_to_pass_mul);
    if (is("Add") && at().in[0] == pass) {  // v15+ pass MLP
      m.pass_mlp = true;
      pass = act(matbias(pass, m.gpool_to_pass_bias), m.pass_act);
      pass = matmul(pass, m.gpool_to_pass_mul2);
    }
    const std::string sp = reshape(p2), ps = reshape(pass);
    if (take("Concat", {sp, ps}).out[0] != "policy") miss();
    m.num_policy_channels = m.p2_conv.oc;
    // value head
    std::string v1 = conv(x, m.v1_conv);
    v1 = bn_act_mask(v1, m.v1_bn, m.v1_act);
    std::string v2 = matbias(matmul(value_pool(v1), m.v2_mul), m.v2_bias);
    v2 = act(v2, m.v2_act);
    if (matbias(matmul(v2, m.v3_mul), m.v3_bias) != "value") miss();
    if (matbias(matmul(v2, m.sv3_mul), m.sv3_bias) != "scorevalue") miss();
    if (conv(v1, m.v_ownership_conv) != "ownership") miss();
    if (pos != g.nodes.size()) miss();
  }
};

int meta_int(const Graph& g, const char* k, int dflt, bool required) {
  auto it = g.meta.find(k);
  if (it == g.meta.end()) {
    if (required) bad(std::string("metadata key ") + k + " missing");
    return dflt;
  }
  try {
    return std::stoi(it->second);
  } catch (...) {
    bad(std::string("metadata key ") + k + " is not an integer: " + it->second);
  }
}

double meta_num(const Graph& g, const char* k, double dflt) {
  auto it = g.meta.find(k);
  if (it == g.meta.end()) return dflt;
  try {
    return std::stod(it->second);
  } catch (...) {
    bad(std::string("metadata key ") + k + " is not a number: " + it->second);
  }
}

}  // namespace

ModelDesc parse_onnx(const uint8_t* data, size_t n) {
  const Graph g = read_model(data, n);
  ModelDesc m;
  auto nm = g.meta.find("name");
  m.name = nm != g.meta.end() ? nm->second : "";
  m.version = meta_int(g, "modelVersion", 0, true);
  if (meta_int(g, "posLen", 19, false) != 19) bad("posLen must be 19");
  m.meta_encoder_version = meta_int(g, "metaEncoderVersion", 0, false);
  m.post_process_from_header = meta_int(g, "postProcessParamsFromHeader", 0, false) != 0;
  const char* pp[8] = {"tdScoreMultiplier", "scoreMeanMultiplier", "scoreStdevMultiplier", "leadMultiplier",
                       "varianceTimeMultiplier", "shorttermValueErrorMultiplier", "shorttermScoreErrorMultiplier",
                       "outputScaleMultiplier"};
  for (int i = 0; i < 8; i++) m.post_process[i] = (float)meta_num(g, pp[i], m.post_process[i]);
  m.prefer_pass_alive = meta_int(g, "preferPassAliveUnderSuicideRules", 0, false) != 0;
  m.prefer_exclude_atari = meta_int(g, "preferExcludeTerritoryAdjacentToAtari", 0, false) != 0;
  m.arch_num_parameters = (int64_t)meta_num(g, "numParameters", -1);
  m.arch_conv_depth = meta_num(g, "trunkSpatialConvDepth", -1);
  Parser p(g);
  try {
    p.model(m);
  } catch (const Mismatch&) {
    const std::string at = p.pos < g.nodes.size() ? g.nodes[p.pos].op + " node " + g.nodes[p.pos].name : "the end";
    bad("the graph is not one tools/bin2onnx/bin2onnx.py writes (unexpected " + at + " at node " +
        std::to_string(p.pos) + ")");
  }
  // the metadata and the graph must agree
  m.num_input_channels = m.initial_conv.ic;
  m.num_input_global_channels = m.initial_matmul.ic;
  m.num_input_meta_channels = m.has_meta ? m.meta_mul1.ic : 0;
  m.trunk_c = m.initial_conv.oc;
  m.mid_c = m.regular_c = m.gpool_c = m.trunk_c;
  auto agree = [&](const char* k, int have) {
    const int v = meta_int(g, k, have, false);
    if (v != have) bad(std::string("metadata ") + k + " = " + std::to_string(v) + " but the graph has " + std::to_string(have));
  };
  agree("numInputChannels", m.num_input_channels);
  agree("numInputGlobalChannels", m.num_input_global_channels);
  agree("numInputMetaChannels", m.num_input_meta_channels);
  agree("trunkNumChannels", m.trunk_c);
  agree("trunkNumBlocks", (int)m.blocks.size());
  agree("trunkNormKind", m.trunk_norm_kind);
  agree("numPolicyChannels", m.num_policy_channels);
  agree("numValueChannels", m.num_value_channels());
  agree("numScoreValueChannels", m.num_score_value_channels());
  agree("numOwnershipChannels", m.num_ownership_channels());
  if (m.has_meta != (m.meta_encoder_version > 0)) bad("metaEncoderVersion does not match the graph's meta input");
  return m;
}

}  // namespace kc
