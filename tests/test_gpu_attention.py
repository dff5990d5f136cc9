"""The tensor-core attention kernel (head dim 64, one CTA per head and board, the board's query tiles pipelined
through S = Q K^T, an exact softmax over the board's keys and O = P V) against the float64 oracle: grouped-query
heads (gqa-tf: 6 query heads over 2 KV heads, 4 over 1), the b10c384h6 benchmark net, f16 and bf16, and mixed
9x9 / 13x13 / 19x19 boards (off-board keys weigh 0, off-board query rows are 0). Tolerance: the 2-byte tier's 2e-2
(north_star)."""

import os

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")
TOL = 2e-2


def handle(m, prec, n, tc):
    saved = os.environ.get("KATAGO_CUDA_TC_ATTN")
    os.environ["KATAGO_CUDA_TC_ATTN"] = tc
    try:
        return kc.Handle(kc.Context(m, gpu_idxs=[0], precision=prec), max_batch=n, gpu_idx=0)
    finally:
        if saved is None:
            os.environ.pop("KATAGO_CUDA_TC_ATTN")
        else:
            os.environ["KATAGO_CUDA_TC_ATTN"] = saved


def case(name, n, seed, sizes):
    m = kc.Model(netgen.net_bytes(name))
    spatial, glob, meta, _ = inputs.synthetic_inputs(n, seed, sizes, m.desc.num_input_channels,
                                                     m.desc.num_input_global_channels,
                                                     m.desc.num_input_meta_channels, rich=True)
    return m, (spatial, glob, meta)


def max_err(got, want):
    for k in KEYS:
        assert np.all(np.isfinite(got[k])), k
    return {k: float(np.abs(got[k] - want[k]).max()) for k in KEYS}


@pytest.mark.parametrize("n", [1, 13])
def test_gqa_mixed_boards_f16(n):
    m, x = case("gqa-tf", n, 4321 + n, (9, 13, 19))
    got = handle(m, kc.PRECISION_F16, n, "1").forward(*x)
    errs = max_err(got, OracleNet(netgen.net_bytes("gqa-tf")).forward(*x))
    assert max(errs.values()) <= TOL, errs


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_gqa_mixed_boards_bf16(seed):
    """The bf16 tier (bf16 trunk, f16 heads) with the tensor-core attention kernel and with the CUDA-core one
    (KATAGO_CUDA_TC_ATTN=0), each within the 2e-2 tier of the float64 oracle."""
    n = 13
    m, x = case("gqa-tf", n, 4321 + 100 * seed, (9, 13, 19))
    want = OracleNet(netgen.net_bytes("gqa-tf")).forward(*x, double=True)
    for tc in ("1", "0"):
        errs = max_err(handle(m, kc.PRECISION_BF16, n, tc).forward(*x), want)
        assert max(errs.values()) <= TOL, (tc, errs)


@pytest.mark.parametrize("prec,seed", [(kc.PRECISION_F16, 77), (kc.PRECISION_BF16, 77), (kc.PRECISION_BF16, 78),
                                       (kc.PRECISION_BF16, 79)])
def test_b10c384h6(prec, seed):
    """The benchmark transformer net on mixed 9x9 / 13x13 / 19x19 boards, batch 8, against the float64 oracle."""
    n = 8
    m, x = case("b10c384h6", n, seed, (9, 13, 19))
    got = handle(m, prec, n, "1").forward(*x)
    errs = max_err(got, OracleNet(netgen.net_bytes("b10c384h6")).forward(*x, double=True))
    assert max(errs.values()) <= TOL, errs
