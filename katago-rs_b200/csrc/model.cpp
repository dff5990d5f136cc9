// KataGo model-file parser of the katago-rs B200 backend.
//
// Token stream and checks follow the reference's parser, tools/bin2onnx/bin2onnx.py (ModelReader :61-125,
// parse_conv :149, parse_bn :186, parse_activation :208, parse_matmul :225, parse_matbias :240, blocks :232-338,
// parse_rmsnorm :383, transformer blocks :406-560, block stack :575-599, meta encoder :639-668, parse_trunk :718,
// policy head :774, value head :833, parse_model :1009-1071, num_parameters :918, spatial_conv_depth :972), which
// mirrors upstream KataGo's desc.cpp. Error messages keep the reference's wording.

#include "model.h"

#include <zlib.h>

#include <cmath>
#include <cstring>

#include "common.h"

namespace kc {

namespace {

[[noreturn]] void perr(const std::string& m) { fail(KC_ERR_PARSE, m); }
void pcheck(bool c, const std::string& m) {
  if (!c) perr(m);
}

std::vector<uint8_t> gunzip(const uint8_t* data, size_t n) {
  z_stream zs;
  std::memset(&zs, 0, sizeof(zs));
  if (inflateInit2(&zs, 16 + MAX_WBITS) != Z_OK) perr("could not initialise gzip decoder");
  std::vector<uint8_t> out;
  out.resize(n * 4 + 1024);
  zs.next_in = const_cast<Bytef*>(data);
  zs.avail_in = (uInt)n;
  int rc = Z_OK;
  while (true) {
    if (zs.total_out >= out.size()) out.resize(out.size() * 2);
    zs.next_out = out.data() + zs.total_out;
    zs.avail_out = (uInt)(out.size() - zs.total_out);
    rc = inflate(&zs, Z_NO_FLUSH);
    if (rc == Z_STREAM_END) break;
    if (rc != Z_OK && rc != Z_BUF_ERROR) {
      inflateEnd(&zs);
      perr("gzip data is corrupt");
    }
    if (rc == Z_BUF_ERROR && zs.avail_in == 0) {
      inflateEnd(&zs);
      perr("gzip data is truncated");
    }
  }
  out.resize(zs.total_out);
  inflateEnd(&zs);
  return out;
}

struct Reader {
  const uint8_t* d;
  size_t n;
  bool binary;
  size_t pos = 0;

  static bool ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; }
  void skip_ws() {
    while (pos < n && ws(d[pos])) pos++;
  }
  std::string token() {
    skip_ws();
    size_t s = pos;
    while (pos < n && !ws(d[pos])) pos++;
    if (pos == s) perr("Unexpected end of model file");
    return std::string(reinterpret_cast<const char*>(d) + s, pos - s);
  }
  int integer() {
    std::string t = token();
    char* end = nullptr;
    long v = std::strtol(t.c_str(), &end, 10);
    if (end == t.c_str() || *end != 0) perr("Expected integer but got " + t);
    return (int)v;
  }
  float flt() {
    std::string t = token();
    char* end = nullptr;
    float v = std::strtof(t.c_str(), &end);
    if (end == t.c_str() || *end != 0) perr("Expected float but got " + t);
    return v;
  }
  bool boolean() {
    int v = integer();
    if (v != 0 && v != 1) perr("Expected bool 0/1 but got " + std::to_string(v));
    return v == 1;
  }
  std::vector<float> floats(size_t cnt, const std::string& name) {
    std::vector<float> v(cnt);
    if (!binary) {
      for (size_t i = 0; i < cnt; i++) v[i] = flt();
    } else {
      int before = 0;
      while (true) {
        if (pos >= n) perr(name + ": could not find binary float block");
        uint8_t c = d[pos++];
        if (c == '@') break;
        if (++before > 100) perr(name + ": could not read float weights (no @BIN@ header)");
      }
      if (pos + 4 > n || std::memcmp(d + pos, "BIN@", 4) != 0)
        perr(name + ": did not find expected header for binary float block");
      pos += 4;
      if (pos + 4 * cnt > n) perr(name + ": did not find the expected number of floats in binary float block");
      std::memcpy(v.data(), d + pos, 4 * cnt);
      pos += 4 * cnt;
    }
    for (float x : v)
      if (!std::isfinite(x)) perr(name + ": Nan or infinite neural net weight or parameter");
    return v;
  }
};

ConvDesc parse_conv(Reader& r) {
  ConvDesc c;
  c.name = r.token();
  c.ky = r.integer(); c.kx = r.integer(); c.ic = r.integer(); c.oc = r.integer();
  c.dy = r.integer(); c.dx = r.integer();
  pcheck(c.kx > 0 && c.ky > 0, c.name + ": convolution filter sizes must be positive");
  pcheck(c.ic > 0 && c.oc > 0, c.name + ": number of in and out channels must be positive");
  pcheck(c.dx > 0 && c.dy > 0, c.name + ": dilation factors must be positive");
  pcheck(c.kx % 2 == 1 && c.ky % 2 == 1, c.name + ": convolution filter sizes must be odd");
  c.w = r.floats((size_t)c.ky * c.kx * c.ic * c.oc, c.name);
  return c;
}

BNDesc parse_bn(Reader& r) {
  BNDesc b;
  b.name = r.token();
  b.c = r.integer();
  float eps = r.flt();
  b.has_scale = r.boolean();
  b.has_bias = r.boolean();
  pcheck(b.c >= 1, b.name + ": numChannels < 1");
  pcheck(eps > 0 && std::isfinite(eps), b.name + ": epsilon is not positive and finite");
  std::vector<float> mean = r.floats(b.c, b.name), var = r.floats(b.c, b.name);
  std::vector<float> scale = b.has_scale ? r.floats(b.c, b.name) : std::vector<float>(b.c, 1.0f);
  std::vector<float> bias = b.has_bias ? r.floats(b.c, b.name) : std::vector<float>(b.c, 0.0f);
  b.merged_scale.resize(b.c);
  b.merged_bias.resize(b.c);
  for (int i = 0; i < b.c; i++) {
    // float32 steps, each rounded: scale / sqrt(var + eps); bias - mergedScale * mean
    volatile float ve = var[i] + eps;
    volatile float sq = std::sqrt((float)ve);
    volatile float ms = scale[i] / (float)sq;
    volatile float pm = (float)ms * mean[i];
    b.merged_scale[i] = ms;
    b.merged_bias[i] = bias[i] - (float)pm;
  }
  return b;
}

Act parse_act(Reader& r, int version) {
  std::string name = r.token();
  if (version >= 11) {
    std::string k = r.token();
    if (k == "ACTIVATION_IDENTITY") return ACT_IDENTITY;
    if (k == "ACTIVATION_RELU") return ACT_RELU;
    if (k == "ACTIVATION_MISH") return ACT_MISH;
    if (k == "ACTIVATION_SILU") return ACT_SILU;
    perr(name + ": unknown activation " + k);
  }
  return ACT_RELU;
}

MatMulDesc parse_matmul(Reader& r) {
  MatMulDesc m;
  m.name = r.token();
  m.ic = r.integer();
  m.oc = r.integer();
  pcheck(m.ic > 0 && m.oc > 0, m.name + ": number of in and out channels must be positive");
  m.w = r.floats((size_t)m.ic * m.oc, m.name);
  return m;
}

MatBiasDesc parse_matbias(Reader& r) {
  MatBiasDesc b;
  b.name = r.token();
  b.c = r.integer();
  pcheck(b.c > 0, b.name + ": number of channels must be positive");
  b.b = r.floats(b.c, b.name);
  return b;
}

TfRmsDesc parse_tf_rms(Reader& r) {
  TfRmsDesc t;
  std::string name = r.token();
  t.c = r.integer();
  t.eps = r.flt();
  pcheck(t.c >= 1, name + ": transformer rmsnorm numChannels < 1");
  pcheck(t.eps > 0 && t.eps <= 1.0f, name + ": transformer rmsnorm epsilon is not positive or is too large");
  t.w = r.floats(t.c, name);
  return t;
}

std::vector<BlockDesc> parse_stack(Reader& r, int version, const std::string& name, int nblocks, int trunk_c);

BlockDesc parse_block(Reader& r, int version, const std::string& kind) {
  BlockDesc b;
  if (kind == "ordinary_block") {
    b.kind = BLOCK_ORDINARY;
    b.name = r.token();
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version); b.regular = parse_conv(r);
    b.mid_bn = parse_bn(r); b.mid_act = parse_act(r, version); b.final_conv = parse_conv(r);
    pcheck(b.pre_bn.c == b.regular.ic, b.name + ": preBN.numChannels != regularConv.inChannels");
    pcheck(b.mid_bn.c == b.regular.oc, b.name + ": midBN.numChannels != regularConv.outChannels");
    pcheck(b.mid_bn.c == b.final_conv.ic, b.name + ": midBN.numChannels != finalConv.inChannels");
  } else if (kind == "gpool_block") {
    b.kind = BLOCK_GPOOL;
    b.name = r.token();
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version);
    b.regular = parse_conv(r); b.gpool_conv = parse_conv(r);
    b.gpool_bn = parse_bn(r); b.gpool_act = parse_act(r, version);
    b.gpool_to_bias = parse_matmul(r);
    b.mid_bn = parse_bn(r); b.mid_act = parse_act(r, version); b.final_conv = parse_conv(r);
    pcheck(b.pre_bn.c == b.regular.ic, b.name + ": preBN.numChannels != regularConv.inChannels");
    pcheck(b.pre_bn.c == b.gpool_conv.ic, b.name + ": preBN.numChannels != gpoolConv.inChannels");
    pcheck(b.gpool_bn.c == b.gpool_conv.oc, b.name + ": gpoolBN.numChannels != gpoolConv.outChannels");
    pcheck(b.gpool_bn.c * 3 == b.gpool_to_bias.ic, b.name + ": gpoolBN.numChannels*3 != gpoolToBiasMul.inChannels");
    pcheck(b.mid_bn.c == b.regular.oc, b.name + ": midBN.numChannels != regularConv.outChannels");
    pcheck(b.mid_bn.c == b.gpool_to_bias.oc, b.name + ": midBN.numChannels != gpoolToBiasMul.outChannels");
    pcheck(b.mid_bn.c == b.final_conv.ic, b.name + ": midBN.numChannels != finalConv.inChannels");
  } else if (kind == "nested_bottleneck_block") {
    b.kind = BLOCK_NESTED;
    b.name = r.token();
    int nb = r.integer();
    pcheck(nb >= 1, b.name + ": nested bottleneck res block num blocks must be positive");
    b.pre_bn = parse_bn(r); b.pre_act = parse_act(r, version); b.pre_conv = parse_conv(r);
    b.inner = parse_stack(r, version, b.name, nb, b.pre_conv.oc);
    b.post_bn = parse_bn(r); b.post_act = parse_act(r, version); b.post_conv = parse_conv(r);
    pcheck(b.pre_bn.c == b.pre_conv.ic, b.name + ": preBN.numChannels != preConv.inChannels");
    pcheck(b.post_bn.c == b.pre_conv.oc, b.name + ": postBN.numChannels != preConv.outChannels");
    pcheck(b.post_bn.c == b.post_conv.ic, b.name + ": postBN.numChannels != postConv.inChannels");
  } else if (kind == "transformer_attention_block") {
    b.kind = BLOCK_ATTENTION;
    b.name = r.token();
    b.heads = r.integer(); b.kv_heads = r.integer(); b.head_dim = r.integer(); b.v_head_dim = r.integer();
    b.use_rope = r.integer() != 0;
    b.learnable_rope = r.integer() != 0;
    pcheck(b.heads >= 1 && b.kv_heads >= 1, b.name + ": transformer attention numHeads and numKVHeads must be positive");
    pcheck(b.heads % b.kv_heads == 0, b.name + ": numHeads must be divisible by numKVHeads");
    pcheck(b.head_dim >= 1 && b.v_head_dim >= 1, b.name + ": head dims must be positive");
    pcheck(!b.use_rope || b.head_dim % 2 == 0, b.name + ": qHeadDim must be even when RoPE is used");
    b.ln = parse_tf_rms(r);
    b.q = parse_matmul(r); b.k = parse_matmul(r); b.v = parse_matmul(r); b.out = parse_matmul(r);
    pcheck(b.q.oc == b.heads * b.head_dim, b.name + ": qProj.outChannels != numHeads*qHeadDim");
    pcheck(b.k.oc == b.kv_heads * b.head_dim, b.name + ": kProj.outChannels != numKVHeads*qHeadDim");
    pcheck(b.v.oc == b.kv_heads * b.v_head_dim, b.name + ": vProj.outChannels != numKVHeads*vHeadDim");
    pcheck(b.out.ic == b.heads * b.v_head_dim, b.name + ": outProj.inChannels != numHeads*vHeadDim");
    if (b.use_rope) {
      if (b.learnable_rope) {
        r.token();
        int kvh = r.integer(), np = r.integer(), d2 = r.integer();
        pcheck(kvh == b.kv_heads, b.name + ": ropeNumKVHeads != numKVHeads");
        pcheck(np == b.head_dim / 2, b.name + ": ropeNumPairs != qHeadDim/2");
        pcheck(d2 == 2, b.name + ": rope freq dim2 must be 2");
        b.rope_freqs = r.floats((size_t)kvh * np * 2, b.name);
      } else {
        r.token();
        b.rope_theta = r.flt();
        pcheck(b.rope_theta > 0 && std::isfinite(b.rope_theta), b.name + ": rope theta must be positive and finite");
      }
    }
  } else if (kind == "transformer_ffn_block") {
    b.kind = BLOCK_FFN;
    b.name = r.token();
    int c = r.integer();
    b.ffn = r.integer();
    bool swiglu = r.integer() != 0;
    pcheck(c >= 1 && b.ffn >= 1, b.name + ": transformer ffn channels must be positive");
    b.ln = parse_tf_rms(r);
    b.w1 = parse_matmul(r);
    if (swiglu) b.wgate = parse_matmul(r);
    b.w2 = parse_matmul(r);
    pcheck(b.w1.ic == c, b.name + ": linear1.inChannels != numChannels");
    pcheck(b.w1.oc == b.ffn, b.name + ": linear1.outChannels != ffnChannels");
    pcheck(b.w2.ic == b.ffn, b.name + ": linear2.inChannels != ffnChannels");
    pcheck(b.w2.oc == c, b.name + ": linear2.outChannels != numChannels");
    // As the reference (bin2onnx.py:1428-1430) and upstream's Eigen backend: the plain FFN has no defined
    // activation and is rejected.
    pcheck(swiglu, b.name + ": non-SwiGLU transformer FFN is not supported");
    pcheck(b.wgate.ic == c && b.wgate.oc == b.ffn, b.name + ": linearGate shape mismatch");
  } else {
    perr("found unknown block kind " + kind);
  }
  return b;
}

std::vector<BlockDesc> parse_stack(Reader& r, int version, const std::string& name, int nblocks, int trunk_c) {
  std::vector<BlockDesc> v;
  for (int i = 0; i < nblocks; i++) {
    std::string kind = r.token();
    BlockDesc b = parse_block(r, version, kind);
    pcheck(b.in_channels() == trunk_c, name + ": " + b.name + " input channels != trunk channels");
    pcheck(b.out_channels() == trunk_c, name + ": " + b.name + " output channels != trunk channels");
    v.push_back(std::move(b));
  }
  return v;
}

bool any_tf(const std::vector<BlockDesc>& v) {
  for (auto& b : v) {
    if (b.kind == BLOCK_ATTENTION || b.kind == BLOCK_FFN) return true;
    if (b.kind == BLOCK_NESTED && any_tf(b.inner)) return true;
  }
  return false;
}

int64_t np_conv(const ConvDesc& c) { return (int64_t)c.w.size(); }
int64_t np_bn(const BNDesc& b) { return (b.has_scale ? b.c : 0) + (b.has_bias ? b.c : 0); }
int64_t np_mm(const MatMulDesc& m) { return (int64_t)m.w.size(); }
int64_t np_mb(const MatBiasDesc& m) { return (int64_t)m.b.size(); }

int64_t np_block(const BlockDesc& b) {
  switch (b.kind) {
    case BLOCK_ORDINARY:
      return np_bn(b.pre_bn) + np_conv(b.regular) + np_bn(b.mid_bn) + np_conv(b.final_conv);
    case BLOCK_GPOOL:
      return np_bn(b.pre_bn) + np_conv(b.regular) + np_conv(b.gpool_conv) + np_bn(b.gpool_bn) +
             np_mm(b.gpool_to_bias) + np_bn(b.mid_bn) + np_conv(b.final_conv);
    case BLOCK_NESTED: {
      int64_t n = np_bn(b.pre_bn) + np_conv(b.pre_conv);
      for (auto& ib : b.inner) n += np_block(ib);
      return n + np_bn(b.post_bn) + np_conv(b.post_conv);
    }
    case BLOCK_ATTENTION:
      return (int64_t)b.ln.w.size() + np_mm(b.q) + np_mm(b.k) + np_mm(b.v) + np_mm(b.out) + (int64_t)b.rope_freqs.size();
    case BLOCK_FFN:
      return (int64_t)b.ln.w.size() + np_mm(b.w1) + np_mm(b.wgate) + np_mm(b.w2);
  }
  return 0;
}

double depth_conv(const ConvDesc& c) { return (c.ky + c.kx - 2) / 4.0; }

double depth_stack(const std::vector<BlockDesc>& v) {
  double d = 0;
  for (auto& b : v) {
    if (b.kind == BLOCK_ATTENTION || b.kind == BLOCK_FFN) d += 2;
    else if (b.kind == BLOCK_NESTED) d += depth_conv(b.pre_conv) + depth_stack(b.inner) + depth_conv(b.post_conv);
    else d += depth_conv(b.regular) + depth_conv(b.final_conv);
  }
  return d;
}

}  // namespace

int BlockDesc::in_channels() const {
  switch (kind) {
    case BLOCK_ORDINARY: case BLOCK_GPOOL: case BLOCK_NESTED: return pre_bn.c;
    case BLOCK_ATTENTION: return q.ic;
    case BLOCK_FFN: return w1.ic;
  }
  return 0;
}

int BlockDesc::out_channels() const {
  switch (kind) {
    case BLOCK_ORDINARY: case BLOCK_GPOOL: return final_conv.oc;
    case BLOCK_NESTED: return post_conv.oc;
    case BLOCK_ATTENTION: return out.oc;
    case BLOCK_FFN: return w2.oc;
  }
  return 0;
}

bool ModelDesc::has_any_transformer_blocks() const { return any_tf(blocks); }

bool ModelDesc::has_any_nested_bottleneck_blocks() const {
  for (auto& b : blocks)
    if (b.kind == BLOCK_NESTED) return true;
  return false;
}

int64_t ModelDesc::num_parameters() const {
  if (arch_num_parameters >= 0) return arch_num_parameters;
  int64_t n = np_conv(initial_conv) + np_mm(initial_matmul);
  if (has_meta) n += np_mm(meta_mul1) + np_mb(meta_bias1) + np_mm(meta_mul2) + np_mb(meta_bias2) + np_mm(meta_mul3);
  for (auto& b : blocks) n += np_block(b);
  n += np_bn(tip_bn) + (int64_t)tip_rms_gamma.size() + (int64_t)tip_rms_beta.size();
  n += np_conv(p1_conv) + np_conv(g1_conv) + np_bn(g1_bn) + np_mm(gpool_to_bias_mul) + np_bn(p1_bn) + np_conv(p2_conv) +
       np_mm(gpool_to_pass_mul) + np_mb(gpool_to_pass_bias) + np_mm(gpool_to_pass_mul2);
  n += np_conv(v1_conv) + np_bn(v1_bn) + np_mm(v2_mul) + np_mb(v2_bias) + np_mm(v3_mul) + np_mb(v3_bias) +
       np_mm(sv3_mul) + np_mb(sv3_bias) + np_conv(v_ownership_conv);
  return n;
}

double ModelDesc::trunk_spatial_conv_depth() const {
  return arch_conv_depth >= 0 ? arch_conv_depth : depth_conv(initial_conv) + depth_stack(blocks);
}

ModelDesc parse_model(const uint8_t* data, size_t n, int binary_floats) {
  std::vector<uint8_t> inflated;
  if (n >= 2 && data[0] == 0x1f && data[1] == 0x8b) {
    inflated = gunzip(data, n);
    data = inflated.data();
    n = inflated.size();
  }
  if (binary_floats < 0) {
    static const char tag[] = "@BIN@";
    binary_floats = 0;
    for (size_t i = 0; i + 5 <= n; i++)
      if (data[i] == '@' && std::memcmp(data + i, tag, 5) == 0) {
        binary_floats = 1;
        break;
      }
  }
  Reader r{data, n, binary_floats != 0};
  ModelDesc m;
  m.name = r.token();
  m.version = r.integer();
  pcheck(!m.name.empty() && m.name.size() <= 96, "Model name must be 1..96 chars");
  for (char c : m.name)
    pcheck((c >= '0' && c <= '9') || (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || c == '_' || c == '-',
           "Model name must contain only alphanumeric characters, underscores, and hyphens: " + m.name);
  pcheck(m.version >= 3, m.name + ": model version " + std::to_string(m.version) + " is too old");
  pcheck(m.version <= 17, m.name + ": model version " + std::to_string(m.version) + " is newer than supported (17)");
  m.num_input_channels = r.integer();
  pcheck(m.num_input_channels > 0, m.name + ": numInputChannels must be positive");
  m.num_input_global_channels = r.integer();
  pcheck(m.num_input_global_channels > 0, m.name + ": numInputGlobalChannels must be positive");
  if (m.version >= 13) {
    for (int i = 0; i < 7; i++) {
      m.post_process[i] = r.flt();
      pcheck(m.post_process[i] > 0, m.name + ": post-process params must be positive");
    }
    m.post_process_from_header = true;
  }
  if (m.version >= 15) {
    m.meta_encoder_version = r.integer();
    pcheck(m.meta_encoder_version >= 0 && m.meta_encoder_version <= 1, m.name + ": unsupported metaEncoderVersion");
    m.num_input_meta_channels = m.meta_encoder_version == 1 ? 192 : 0;
    int a = r.integer(), b = r.integer();
    pcheck((a == 0 || a == 1) && (b == 0 || b == 1), m.name + ": model flag unexpected value");
    m.prefer_pass_alive = a == 1;
    m.prefer_exclude_atari = b == 1;
    for (int i = 0; i < 5; i++) pcheck(r.integer() == 0, m.name + ": unknown/unsupported model option");
  }
  // trunk
  std::string tname = r.token();
  int nb = r.integer();
  m.trunk_c = r.integer(); m.mid_c = r.integer(); m.regular_c = r.integer();
  r.integer();  // dilated channels, unused
  m.gpool_c = r.integer();
  if (m.version >= 15) {
    m.trunk_norm_kind = r.integer();
    for (int i = 0; i < 5; i++) pcheck(r.integer() == 0, tname + ": unknown/unsupported trunk option");
    pcheck(m.trunk_norm_kind == 0 || m.trunk_norm_kind == 1, tname + ": unknown or unsupported trunk norm kind");
  }
  pcheck(nb >= 1, tname + ": trunk num blocks must be positive");
  pcheck(m.trunk_c > 0 && m.mid_c > 0 && m.regular_c > 0 && m.gpool_c > 0, tname + ": channel counts must be positive");
  m.initial_conv = parse_conv(r);
  pcheck(m.initial_conv.oc == m.trunk_c, m.initial_conv.name + ": outChannels != trunkNumChannels");
  m.initial_matmul = parse_matmul(r);
  pcheck(m.initial_matmul.oc == m.trunk_c, m.initial_matmul.name + ": outChannels != trunkNumChannels");
  if (m.meta_encoder_version > 0) {
    m.has_meta = true;
    std::string ename = r.token();
    int nin = r.integer();
    pcheck(nin == 192, ename + ": number of in channels did not match expected (192)");
    m.meta_mul1 = parse_matmul(r); m.meta_bias1 = parse_matbias(r); m.meta_act1 = parse_act(r, m.version);
    m.meta_mul2 = parse_matmul(r); m.meta_bias2 = parse_matbias(r); m.meta_act2 = parse_act(r, m.version);
    m.meta_mul3 = parse_matmul(r);
    pcheck(m.meta_mul1.ic == 192 && m.meta_mul1.oc == m.meta_bias1.c && m.meta_mul2.ic == m.meta_mul1.oc &&
               m.meta_mul2.oc == m.meta_bias2.c && m.meta_mul3.ic == m.meta_mul2.oc && m.meta_mul3.oc == m.trunk_c,
           ename + ": SGF metadata encoder shape mismatch");
  }
  m.blocks = parse_stack(r, m.version, tname, nb, m.trunk_c);
  if (m.trunk_norm_kind == 0) {
    m.tip_bn = parse_bn(r);
    pcheck(m.tip_bn.c == m.trunk_c, tname + ": trunkTipBN.numChannels != trunkNumChannels");
  } else {
    std::string rname = r.token();
    int c = r.integer();
    m.tip_rms_eps = r.flt();
    m.tip_rms_spatial = r.integer() != 0;
    int cg = r.integer();
    pcheck(m.tip_rms_eps > 0 && m.tip_rms_eps <= 1.0f, rname + ": rmsnorm epsilon is not positive or is too large");
    pcheck(c == m.trunk_c, tname + ": trunkTipRMSNorm.numChannels != trunkNumChannels");
    pcheck(cg == 0, rname + ": rmsnorm cgroupSize != 0, grouped spatial RMSNorm is not supported");
    m.tip_rms_gamma = r.floats(c, rname);
    m.tip_rms_beta = r.floats(c, rname);
  }
  m.tip_act = parse_act(r, m.version);

  // policy head
  std::string pname = r.token();
  if (m.version >= 17) {
    m.num_policy_channels = r.integer();
    pcheck(m.num_policy_channels == 2 || m.num_policy_channels == 4,
           pname + ": policy head got invalid policyOutChannels " + std::to_string(m.num_policy_channels));
    for (int i = 0; i < 3; i++) pcheck(r.integer() == 0, pname + ": unknown/unsupported policy option");
  } else if (m.version == 16) {
    m.num_policy_channels = 4;
  } else if (m.version >= 12) {
    m.num_policy_channels = 2;
  } else {
    m.num_policy_channels = 1;
  }
  m.p1_conv = parse_conv(r); m.g1_conv = parse_conv(r); m.g1_bn = parse_bn(r); m.g1_act = parse_act(r, m.version);
  m.gpool_to_bias_mul = parse_matmul(r); m.p1_bn = parse_bn(r); m.p1_act = parse_act(r, m.version);
  m.p2_conv = parse_conv(r); m.gpool_to_pass_mul = parse_matmul(r);
  if (m.version >= 15) {
    m.pass_mlp = true;
    m.gpool_to_pass_bias = parse_matbias(r); m.pass_act = parse_act(r, m.version); m.gpool_to_pass_mul2 = parse_matmul(r);
  }
  pcheck(m.p1_conv.oc == m.p1_bn.c, pname + ": p1Conv.outChannels != p1BN.numChannels");
  pcheck(m.g1_conv.oc == m.g1_bn.c, pname + ": g1Conv.outChannels != g1BN.numChannels");
  pcheck(m.gpool_to_bias_mul.ic == m.g1_bn.c * 3, pname + ": gpoolToBiasMul.inChannels != g1BN.numChannels*3");
  pcheck(m.gpool_to_bias_mul.oc == m.p1_bn.c, pname + ": gpoolToBiasMul.outChannels != p1BN.numChannels");
  pcheck(m.p2_conv.ic == m.p1_bn.c, pname + ": p2Conv.inChannels != p1BN.numChannels");
  pcheck(m.gpool_to_pass_mul.ic == m.g1_bn.c * 3, pname + ": gpoolToPassMul.inChannels != g1BN.numChannels*3");
  pcheck(m.p2_conv.oc == m.num_policy_channels, pname + ": p2Conv.outChannels != policyOutChannels");
  if (m.pass_mlp) {
    pcheck(m.gpool_to_pass_mul.oc == m.gpool_to_pass_bias.c && m.gpool_to_pass_mul.oc == m.gpool_to_pass_mul2.ic &&
               m.gpool_to_pass_mul2.oc == m.num_policy_channels,
           pname + ": gpoolToPass shape mismatch");
  } else {
    pcheck(m.gpool_to_pass_mul.oc == m.num_policy_channels, pname + ": gpoolToPassMul.outChannels != policyOutChannels");
  }

  // value head
  std::string vname = r.token();
  if (m.version >= 17)
    for (int i = 0; i < 3; i++) pcheck(r.integer() == 0, vname + ": unknown/unsupported value option");
  m.v1_conv = parse_conv(r); m.v1_bn = parse_bn(r); m.v1_act = parse_act(r, m.version);
  m.v2_mul = parse_matmul(r); m.v2_bias = parse_matbias(r); m.v2_act = parse_act(r, m.version);
  m.v3_mul = parse_matmul(r); m.v3_bias = parse_matbias(r);
  m.sv3_mul = parse_matmul(r); m.sv3_bias = parse_matbias(r);
  m.v_ownership_conv = parse_conv(r);
  pcheck(m.v1_conv.oc == m.v1_bn.c, vname + ": v1Conv.outChannels != v1BN.numChannels");
  pcheck(m.v2_mul.ic == m.v1_bn.c * 3, vname + ": v2Mul.inChannels != v1BN.numChannels*3");
  pcheck(m.v2_mul.oc == m.v2_bias.c && m.v2_mul.oc == m.v3_mul.ic, vname + ": v2 shape mismatch");
  pcheck(m.v3_mul.oc == 3 && m.v3_bias.c == 3, vname + ": v3 must have 3 outputs");
  int expected_sv = m.version >= 9 ? 6 : m.version >= 8 ? 4 : m.version >= 4 ? 2 : 1;
  pcheck(m.sv3_mul.ic == m.v2_mul.oc, vname + ": sv3Mul.inChannels != v2Mul.outChannels");
  pcheck(m.sv3_mul.oc == expected_sv && m.sv3_bias.c == expected_sv,
         vname + ": sv3 must have " + std::to_string(expected_sv) + " outputs for model version " + std::to_string(m.version));
  pcheck(m.v_ownership_conv.ic == m.v1_conv.oc, vname + ": vOwnershipConv.inChannels != v1Conv.outChannels");
  pcheck(m.v_ownership_conv.oc == 1, vname + ": vOwnershipConv.outChannels != 1");

  pcheck(m.num_input_channels == m.initial_conv.ic, m.name + ": numInputChannels != initialConv.inChannels");
  pcheck(m.num_input_global_channels == m.initial_matmul.ic, m.name + ": numInputGlobalChannels != initialMatMul.inChannels");
  pcheck(m.trunk_c == m.p1_conv.ic && m.trunk_c == m.g1_conv.ic && m.trunk_c == m.v1_conv.ic,
         m.name + ": trunk channels != head input channels");
  r.skip_ws();
  pcheck(r.pos == r.n, m.name + ": " + std::to_string(r.n - r.pos) + " unparsed trailing bytes in model file");
  return m;
}

}  // namespace kc
