"""The product's model parser (kc_model_load) against the reference parser's ModelDesc (tests/golden/descs.json is
tools/bin2onnx/bin2onnx.py parse_model on the same bytes), plus the reference's error behaviour. CPU only."""

import gzip
import json
import os

import pytest

from katago_cuda import api, netgen

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DESCS = json.load(open(os.path.join(GOLDEN, "descs.json")))
FIELDS = {
    "modelVersion": "model_version", "numInputChannels": "num_input_channels",
    "numInputGlobalChannels": "num_input_global_channels", "numInputMetaChannels": "num_input_meta_channels",
    "numPolicyChannels": "num_policy_channels", "numValueChannels": "num_value_channels",
    "numScoreValueChannels": "num_score_value_channels", "numOwnershipChannels": "num_ownership_channels",
    "trunkNumBlocks": "trunk_num_blocks", "trunkNumChannels": "trunk_num_channels", "trunkNormKind": "trunk_norm_kind",
    "numParameters": "num_parameters", "hasAnyTransformerBlocks": "has_any_transformer_blocks",
    "hasAnyNestedBottleneckBlocks": "has_any_nested_bottleneck_blocks",
}


@pytest.mark.parametrize("name", sorted(DESCS))
def test_desc_matches_reference_parser(name):
    m = api.Model(netgen.net_bytes(name), "net.bin")
    d = DESCS[name]
    for k, attr in FIELDS.items():
        assert getattr(m.desc, attr) == d[k], (k, getattr(m.desc, attr), d[k])
    assert abs(m.desc.trunk_spatial_conv_depth - d["trunkSpatialConvDepth"]) < 1e-9
    assert m.desc.name.decode() == d["name"]
    for i, v in enumerate(d["postProcess"]):
        assert abs(m.desc.post_process[i] - v) < 1e-6


def test_gzip_and_detection():
    raw = netgen.net_bytes("tiny-resnet")
    a = api.Model(gzip.compress(raw), "net.bin.gz")
    b = api.Model(raw, None)
    assert a.desc.num_parameters == b.desc.num_parameters == DESCS["tiny-resnet"]["numParameters"]


def test_truncated_file_is_rejected():
    raw = netgen.net_bytes("tiny-resnet")
    with pytest.raises(api.KcError) as e:
        api.Model(raw[: len(raw) // 2], "net.bin")
    assert e.value.status == api.KC_ERR_PARSE
    assert "Error loading or parsing model file net.bin" in str(e.value)


def test_trailing_bytes_rejected():
    raw = netgen.net_bytes("tiny-resnet") + b" junk"
    with pytest.raises(api.KcError, match="unparsed trailing bytes"):
        api.Model(raw, "net.bin")


def test_newer_version_rejected():
    raw = netgen.net_bytes("tiny-resnet").replace(b"tiny-resnet 8 ", b"tiny-resnet 18 ", 1)
    with pytest.raises(api.KcError, match="newer than supported"):
        api.Model(raw, "net.bin")


def test_nonfinite_weight_rejected():
    import numpy as np
    raw = bytearray(netgen.net_bytes("tiny-resnet"))
    i = raw.index(b"@BIN@") + 5
    raw[i:i + 4] = np.float32(np.nan).tobytes()
    with pytest.raises(api.KcError, match="Nan or infinite"):
        api.Model(bytes(raw), "net.bin")


def test_context_rejects_other_board_sizes():
    m = api.Model(netgen.net_bytes("tiny-resnet"))
    with pytest.raises(api.KcError, match="posLen 19"):
        api.Context(m, nn_x_len=13, nn_y_len=13)


def test_auto_precision():
    assert api.Context(api.Model(netgen.net_bytes("tiny-nbt"))).precision == api.PRECISION_F16
    assert api.Context(api.Model(netgen.net_bytes("tiny-tf-learn"))).precision == api.PRECISION_BF16
    assert api.Context(api.Model(netgen.net_bytes("tiny-nbt")), precision=api.PRECISION_F32).precision == 0
