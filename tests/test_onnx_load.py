"""ONNX models (§8f: the files the reference's burn backend is generated from, crates/katago-nn-burn/build.rs:25-30)
through kc_model_load: the fixtures tests/golden/*.onnx are the reference's own export (tools/bin2onnx/bin2onnx.py
build_onnx, made by tests/golden/make_onnx.py) of the seeded .bin nets; loaded, each must describe the same net as
its .bin. CPU only (no device is touched); tests/test_gpu_onnx.py compares the forward passes."""

import os

import pytest

import katago_cuda as kc
from katago_cuda import api, netgen

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NETS = ["tiny-resnet", "tiny-nbt", "tiny-v15-meta", "tiny-tf-learn", "tiny-tf-spatial"]
FIELDS = [f for f, _ in api.Desc._fields_ if f != "post_process"]


def onnx_bytes(name):
    with open(os.path.join(GOLDEN, f"{name}.onnx"), "rb") as f:
        return f.read()


@pytest.mark.parametrize("name", NETS)
@pytest.mark.parametrize("file_name", ["model.onnx", None])
def test_onnx_desc_matches_bin(name, file_name):
    got = kc.Model(onnx_bytes(name), file_name)
    want = kc.Model(netgen.net_bytes(name))
    for f in FIELDS:
        assert getattr(got.desc, f) == getattr(want.desc, f), f
    assert list(got.desc.post_process) == list(want.desc.post_process)
    assert got.flops() == want.flops()


def test_truncated_onnx_is_a_parse_error():
    data = onnx_bytes("tiny-nbt")
    with pytest.raises(kc.KcError) as e:
        kc.Model(data[: len(data) // 2], "cut.onnx")
    assert e.value.status == api.KC_ERR_PARSE
    assert "Error loading or parsing model file cut.onnx" in str(e.value)


def test_foreign_graph_is_refused():
    # a well-formed ModelProto whose graph is not GraphBuilder's: one Relu node
    def varint(v):
        out = bytearray()
        while True:
            b, v = v & 0x7F, v >> 7
            out.append(b | (0x80 if v else 0))
            if not v:
                return bytes(out)

    def ld(field, payload):
        return varint(field << 3 | 2) + varint(len(payload)) + payload

    node = ld(1, b"x") + ld(2, b"y") + ld(3, b"r") + ld(4, b"Relu")
    model = varint(1 << 3) + varint(8) + ld(7, ld(1, node)) + ld(14, ld(1, b"modelVersion") + ld(2, b"8"))
    with pytest.raises(kc.KcError) as e:
        kc.Model(model, "foreign.onnx")
    assert e.value.status == api.KC_ERR_PARSE
    assert "not one tools/bin2onnx/bin2onnx.py writes" in str(e.value)
