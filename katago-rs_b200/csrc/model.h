// Host-side model description of the katago-rs B200 backend: the parsed KataGo model file with float32 weights.
//
// The layer and block structure is KataGo's desc.h as the reference restates it in
// tools/bin2onnx/bin2onnx.py:138-905; parse() follows the same token order, version gates and checks. The engine
// (engine.cu) packs these weights into device layouts.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace kc {

enum Act : int { ACT_IDENTITY = 0, ACT_RELU = 1, ACT_MISH = 2, ACT_SILU = 3 };

struct ConvDesc {
  std::string name;
  int ky = 0, kx = 0, ic = 0, oc = 0, dy = 1, dx = 1;
  std::vector<float> w;  // file order [ky][kx][ic][oc]
};

struct BNDesc {
  std::string name;
  int c = 0;
  bool has_scale = false, has_bias = false;
  std::vector<float> merged_scale, merged_bias;  // computeMerged() in float32 (bin2onnx.py:179-183)
};

struct MatMulDesc {
  std::string name;
  int ic = 0, oc = 0;
  std::vector<float> w;  // [ic][oc]
};

struct MatBiasDesc {
  std::string name;
  int c = 0;
  std::vector<float> b;
};

struct TfRmsDesc {
  int c = 0;
  float eps = 0;
  std::vector<float> w;
};

enum BlockKind : int { BLOCK_ORDINARY, BLOCK_GPOOL, BLOCK_NESTED, BLOCK_ATTENTION, BLOCK_FFN };

struct BlockDesc {
  BlockKind kind = BLOCK_ORDINARY;
  std::string name;
  // ordinary / gpool / nested bottleneck
  BNDesc pre_bn, mid_bn, gpool_bn, post_bn;
  Act pre_act = ACT_RELU, mid_act = ACT_RELU, gpool_act = ACT_RELU, post_act = ACT_RELU;
  ConvDesc regular, gpool_conv, final_conv, pre_conv, post_conv;
  MatMulDesc gpool_to_bias;
  std::vector<BlockDesc> inner;
  // transformer attention / SwiGLU FFN
  int heads = 0, kv_heads = 0, head_dim = 0, v_head_dim = 0;
  bool use_rope = false, learnable_rope = false;
  float rope_theta = 0;
  std::vector<float> rope_freqs;  // [kv_heads][head_dim/2][2]
  // RoPE tables as a file stores them (ONNX models): [rope_ntables][361][head_dim / 2] cos and sin; empty: the
  // engine computes them from rope_freqs / rope_theta
  std::vector<float> rope_cos, rope_sin;
  int rope_ntables = 0;
  TfRmsDesc ln;
  MatMulDesc q, k, v, out;
  int ffn = 0;
  MatMulDesc w1, wgate, w2;

  int in_channels() const;
  int out_channels() const;
};

struct ModelDesc {
  std::string name;
  int version = 0;
  int num_input_channels = 0, num_input_global_channels = 0, num_input_meta_channels = 0;
  int meta_encoder_version = 0;
  bool post_process_from_header = false;
  float post_process[8] = {20, 20, 20, 20, 40, 0.25f, 30, 1};
  bool prefer_pass_alive = false, prefer_exclude_atari = false;

  // trunk
  int trunk_c = 0, mid_c = 0, regular_c = 0, gpool_c = 0;
  int trunk_norm_kind = 0;  // 0 batch norm, 1 RMSNorm
  ConvDesc initial_conv;
  MatMulDesc initial_matmul;
  bool has_meta = false;
  MatMulDesc meta_mul1, meta_mul2, meta_mul3;
  MatBiasDesc meta_bias1, meta_bias2;
  Act meta_act1 = ACT_IDENTITY, meta_act2 = ACT_IDENTITY;
  std::vector<BlockDesc> blocks;
  BNDesc tip_bn;
  bool tip_rms_spatial = false;
  float tip_rms_eps = 0;
  std::vector<float> tip_rms_gamma, tip_rms_beta;
  Act tip_act = ACT_RELU;

  // policy head
  int num_policy_channels = 1;
  ConvDesc p1_conv, g1_conv, p2_conv;
  BNDesc g1_bn, p1_bn;
  Act g1_act = ACT_RELU, p1_act = ACT_RELU, pass_act = ACT_IDENTITY;
  MatMulDesc gpool_to_bias_mul, gpool_to_pass_mul, gpool_to_pass_mul2;
  MatBiasDesc gpool_to_pass_bias;
  bool pass_mlp = false;

  // value head
  ConvDesc v1_conv, v_ownership_conv;
  BNDesc v1_bn;
  Act v1_act = ACT_RELU, v2_act = ACT_RELU;
  MatMulDesc v2_mul, v3_mul, sv3_mul;
  MatBiasDesc v2_bias, v3_bias, sv3_bias;

  int num_value_channels() const { return v3_mul.oc; }
  int num_score_value_channels() const { return sv3_mul.oc; }
  int num_ownership_channels() const { return v_ownership_conv.oc; }
  bool has_any_transformer_blocks() const;
  bool has_any_nested_bottleneck_blocks() const;
  int64_t num_parameters() const;
  double trunk_spatial_conv_depth() const;
  // the architecture summary a file states (ONNX metadata numParameters / trunkSpatialConvDepth, written because a
  // graph has no layer list to recompute them from); < 0: computed from the layers
  int64_t arch_num_parameters = -1;
  double arch_conv_depth = -1;
};

// Parse a KataGo net exported as ONNX by the reference's tools/bin2onnx/bin2onnx.py (the graph GraphBuilder emits,
// :1088-1615, and its metadata_props): the layer list is rebuilt from the graph. Throws kc::Error(KC_ERR_PARSE, ...).
ModelDesc parse_onnx(const uint8_t* data, size_t n);

// Parse a model file held in memory. `binary_floats` selects "@BIN@" float blocks (.bin) or text floats (.txt).
// gzip data is detected by its magic bytes and inflated first. Throws kc::Error(KC_ERR_PARSE, ...) on failure.
ModelDesc parse_model(const uint8_t* data, size_t n, int binary_floats /* 1, 0, or -1 = detect */);

}  // namespace kc
