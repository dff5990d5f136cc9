"""Forward passes of the ONNX-loaded nets (tests/golden/*.onnx, the reference's own export) against the same nets
loaded from .bin, through the C ABI: identical layers give identical outputs in every tier. The RoPE tables are
the ones the export stores (float32, from float64 cos / sin as bin2onnx.py:449-484 computes them); the .bin path
computes them the same way."""

import os

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
KEYS = ("policy", "value", "scorevalue", "ownership")


@pytest.mark.parametrize("name", ["tiny-resnet", "tiny-nbt", "tiny-v15-meta", "tiny-tf-learn", "tiny-tf-spatial"])
@pytest.mark.parametrize("prec", [kc.PRECISION_F32, kc.PRECISION_AUTO])
def test_onnx_forward_equals_bin(name, prec):
    with open(os.path.join(GOLDEN, f"{name}.onnx"), "rb") as f:
        mo = kc.Model(f.read(), f"{name}.onnx")
    mb = kc.Model(netgen.net_bytes(name))
    d = mb.desc
    n = 11
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, 61, (9, 13, 19), d.num_input_channels,
                                                     d.num_input_global_channels, d.num_input_meta_channels,
                                                     rich=True)
    outs = []
    for m in (mo, mb):
        h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=prec), max_batch=n, gpu_idx=0)
        outs.append(h.forward(spatial, glob, meta))
    for k in KEYS:
        assert np.all(np.isfinite(outs[0][k])), k
        np.testing.assert_array_equal(outs[0][k], outs[1][k])
