"""The trunk's CTA-pair GEMM (the default for one- and two-segment convolutions with 2-byte outputs) against the
one-CTA GEMM (KATAGO_CUDA_PAIR=0), the pair kernel without A windows (KATAGO_CUDA_PAIR_WIN=0) and the float64
oracle, on the tile widths the pair kernel has (128, 192, 256: b10c128, small-nbt, wide-nbt) and on ragged batches
whose last 256-row pair tile is mostly past the batch's rows. Tolerance: the f16 tier's 2e-2 (north_star)."""

import os

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")
TOL = 2e-2


def forward(name, env, spatial, glob):
    """A fresh plan built under `env` (the GEMM selection is read when the plan is built)."""
    saved = {k: os.environ.get(k) for k in ("KATAGO_CUDA_PAIR", "KATAGO_CUDA_PAIR_WIN")}
    try:
        for k in saved:
            os.environ.pop(k, None)
        os.environ.update(env)
        m = kc.Model(netgen.net_bytes(name))
        h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=kc.PRECISION_F16), max_batch=len(spatial), gpu_idx=0)
        return h.forward(spatial, glob)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.mark.parametrize("name", ["wide-nbt", "b10c128", "small-nbt"])
@pytest.mark.parametrize("batch", [1, 5, 37])
def test_pair_gemm_matches_one_cta_gemm_and_oracle(name, batch):
    spatial, glob, _, _ = inputs.synthetic_inputs(batch, 4000 + batch, (9, 13, 19), rich=True)
    want = OracleNet(netgen.net_bytes(name)).forward(spatial, glob, double=True)
    runs = {"pair": forward(name, {}, spatial, glob),
            "pair without windows": forward(name, {"KATAGO_CUDA_PAIR_WIN": "0"}, spatial, glob),
            "one-CTA": forward(name, {"KATAGO_CUDA_PAIR": "0"}, spatial, glob)}
    for label, got in runs.items():
        for k in KEYS:
            assert np.all(np.isfinite(got[k])), (label, k)
        errs = {k: float(np.abs(got[k] - want[k]).max()) for k in KEYS}
        assert max(errs.values()) <= TOL, (label, errs)
    diff = {k: float(np.abs(runs["pair"][k] - runs["one-CTA"][k]).max()) for k in KEYS}
    assert max(diff.values()) <= TOL, diff
