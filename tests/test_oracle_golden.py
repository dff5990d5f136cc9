"""The CPU oracle against the golden fixtures (the reference's own graph, tools/bin2onnx/bin2onnx.py GraphBuilder,
evaluated in float64 by tests/golden/make_golden.py). Pins the oracle before it is trusted as the GPU checker."""

import json
import os

import numpy as np
import pytest

from katago_cuda import netgen
from oracle.oracle import OracleNet

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAMES = sorted(json.load(open(os.path.join(GOLDEN, "descs.json"))))


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_graph(name):
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    net = OracleNet(netgen.net_bytes(name))
    out64 = net.forward(g["bin_input"], g["global_input"], g["meta_input"], double=True)
    out32 = net.forward(g["bin_input"], g["global_input"], g["meta_input"], double=False)
    for k in ("policy", "value", "scorevalue", "ownership"):
        ref = g[k]
        assert out64[k].shape == ref.shape
        # float64 oracle == float64 reference graph up to the float32 rounding of the outputs
        np.testing.assert_allclose(out64[k], ref, rtol=0, atol=1e-6 + 1e-6 * np.abs(ref).max())
        # float32 oracle (the flex tier) within the reference's CPU tolerance (nn_parity.rs flex tier 1e-5 scale)
        assert np.abs(out32[k] - ref).max() < 2e-5, (k, np.abs(out32[k] - ref).max())


def test_writer_bytes_match_golden_hash():
    import hashlib
    descs = json.load(open(os.path.join(GOLDEN, "descs.json")))
    for name, d in descs.items():
        assert hashlib.sha256(netgen.net_bytes(name)).hexdigest() == d["sha256"], name


def test_oracle_detects_planted_error():
    """A mistake planted in the oracle's inputs (one flipped stone) must show up at the golden tolerance."""
    g = np.load(os.path.join(GOLDEN, "tiny-nbt.npz"))
    net = OracleNet(netgen.net_bytes("tiny-nbt"))
    x = g["bin_input"].copy()
    x[0, 1, 3, 3] = 1.0 - x[0, 1, 3, 3]
    out = net.forward(x, g["global_input"], g["meta_input"], double=True)
    assert np.abs(out["policy"] - g["policy"]).max() > 1e-4
