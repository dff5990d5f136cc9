"""The CTA-pair GEMM (the default for one- and two-segment convolutions and token linears) against the one-CTA GEMM
(KATAGO_CUDA_PAIR=0), the pair kernel without A windows (KATAGO_CUDA_PAIR_WIN=0), the pair kernel without the
64-column tiles that small batches get (KATAGO_CUDA_PAIR_NARROW=0), without the column-half items of a last, partly
filled round of tiles (KATAGO_CUDA_PAIR_SPLIT=0) and the float64 oracle: the trunk's tile widths (128, 192,
256: b10c128, small-nbt, wide-nbt; 64 at batches 1 and 5) on ragged batches whose last 256-row pair tile is mostly
past the batch's rows, and the transformer's token linears (fused RoPE, SwiGLU, masked accumulators, the float32
residual stream of the bf16 tier). Tolerance: the 2-byte tiers' 2e-2 (north_star)."""

import os

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")
TOL = 2e-2


def forward(name, env, spatial, glob, meta=None, prec=kc.PRECISION_F16):
    """A fresh plan built under `env` (the GEMM selection is read when the plan is built)."""
    saved = {k: os.environ.get(k) for k in ("KATAGO_CUDA_PAIR", "KATAGO_CUDA_PAIR_WIN", "KATAGO_CUDA_PAIR_NARROW",
                                            "KATAGO_CUDA_PAIR_SPLIT", "KATAGO_CUDA_GPOOL_FUSED",
                                            "KATAGO_CUDA_GPOOL_GROUPS", "KATAGO_CUDA_CHAIN")}
    try:
        for k in saved:
            os.environ.pop(k, None)
        os.environ.update(env)
        m = kc.Model(netgen.net_bytes(name))
        h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=prec), max_batch=len(spatial), gpu_idx=0)
        return h.forward(spatial, glob, meta)
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
            "pair, wide tiles only": forward(name, {"KATAGO_CUDA_PAIR_NARROW": "0"}, spatial, glob),
            "pair, whole tiles only": forward(name, {"KATAGO_CUDA_PAIR_NARROW": "0", "KATAGO_CUDA_PAIR_SPLIT": "0"},
                                              spatial, glob),
            "one-CTA": forward(name, {"KATAGO_CUDA_PAIR": "0"}, spatial, glob)}
    for label, got in runs.items():
        for k in KEYS:
            assert np.all(np.isfinite(got[k])), (label, k)
        errs = {k: float(np.abs(got[k] - want[k]).max()) for k in KEYS}
        assert max(errs.values()) <= TOL, (label, errs)
    diff = {k: float(np.abs(runs["pair"][k] - runs["one-CTA"][k]).max()) for k in KEYS}
    assert max(diff.values()) <= TOL, diff


@pytest.mark.parametrize("name", ["gqa-tf", "small-tf"])
@pytest.mark.parametrize("prec", [kc.PRECISION_F16, kc.PRECISION_BF16])
def test_pair_token_linears(name, prec):
    """The transformer's token linears on the pair kernel (the Q|K|V linear with fused RoPE, the SwiGLU linear, the
    output linears with a masked accumulator and, at bf16, the float32 residual stream) and on the one-CTA kernel,
    against the float64 oracle; at f16 also against each other."""
    batch = 13
    m = kc.Model(netgen.net_bytes(name))
    spatial, glob, meta, _ = inputs.synthetic_inputs(batch, 5000 + batch, (9, 13, 19), m.desc.num_input_channels,
                                                     m.desc.num_input_global_channels,
                                                     m.desc.num_input_meta_channels, rich=True)
    want = OracleNet(netgen.net_bytes(name)).forward(spatial, glob, meta, double=True)
    runs = {"pair": forward(name, {}, spatial, glob, meta, prec),
            "one-CTA": forward(name, {"KATAGO_CUDA_PAIR": "0"}, spatial, glob, meta, prec)}
    for label, got in runs.items():
        for k in KEYS:
            assert np.all(np.isfinite(got[k])), (label, k)
        errs = {k: float(np.abs(got[k] - want[k]).max()) for k in KEYS}
        assert max(errs.values()) <= TOL, (label, errs)
    if prec == kc.PRECISION_F16:
        diff = {k: float(np.abs(runs["pair"][k] - runs["one-CTA"][k]).max()) for k in KEYS}
        assert max(diff.values()) <= TOL, diff


@pytest.mark.parametrize("prec", [kc.PRECISION_F16, kc.PRECISION_F32])
def test_gpool_mid_fused_is_bit_identical(prec):
    """The gpool block's pooling, bias matmul and biased batch norm as one launch give the outputs of the three
    launches they replace, bit for bit (small-nbt: two gpool blocks of 128 + 64 channels; mixed boards), whether a
    board's columns go to one block or are shared out over several (the default at this batch: 16 groups of one
    16-byte vector per row; 3 groups: uneven)."""
    spatial, glob, _, _ = inputs.synthetic_inputs(7, 4242, (9, 13, 19), rich=True)
    three = forward("small-nbt", {"KATAGO_CUDA_GPOOL_FUSED": "0"}, spatial, glob, prec=prec)
    for env in ({}, {"KATAGO_CUDA_GPOOL_GROUPS": "1"}, {"KATAGO_CUDA_GPOOL_GROUPS": "3"}):
        fused = forward("small-nbt", env, spatial, glob, prec=prec)
        for k in KEYS:
            np.testing.assert_array_equal(fused[k], three[k], err_msg=str(env))


@pytest.mark.parametrize("batch", [1, 37, 100])
def test_chained_boundary_1x1s_match_separate_launches(batch):
    """b18c384nbt's nested-block boundaries (closing 1x1 of one block + opening 1x1 of the next, with the trunk's
    batch norm + mish kept in tensor memory) give the outputs of the two separate launches, bit for bit, on mixed
    boards: 37 and 100 boards (58 and 157 row tiles, the last partly filled) run the chained kernel; one board (two
    row tiles) runs the separate launches that small batches take."""
    spatial, glob, _, _ = inputs.synthetic_inputs(batch, 6100 + batch, (9, 13, 19), rich=True)
    chained = forward("b18c384nbt", {}, spatial, glob)
    separate = forward("b18c384nbt", {"KATAGO_CUDA_CHAIN": "0"}, spatial, glob)
    for k in KEYS:
        np.testing.assert_array_equal(chained[k], separate[k], err_msg=k)


def test_launch_count_follows_the_boundary_form():
    """The handle's launch count is per batch: b18c384nbt's 17 nested-block boundaries take two launches each at one
    board and one chained launch at 64 boards (at least half as many 256-row tiles as the B200's 74 SM pairs)."""
    m = kc.Model(netgen.net_bytes("b18c384nbt"))
    h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=kc.PRECISION_F16), max_batch=64, gpu_idx=0)
    assert h.launch_count(1) - h.launch_count(64) == 17
