"""Several compute handles of one context driven from several host threads at once, as katago-rs runs one NN
server thread per handle (crates/katago-core/src/program/setup.rs:456-496; one handle per thread,
nninterface.rs:33-34). The handles are created concurrently (plan building, shared-memory opt-in, the driver's
tensor-map encoder) and then run batches concurrently; every output must be bit-identical to the same handle's
output when it runs alone."""

import threading

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import inputs, netgen

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")


@pytest.mark.parametrize("name,prec", [("small-nbt", kc.PRECISION_F16), ("gqa-tf", kc.PRECISION_BF16)])
def test_two_handles_two_threads(name, prec):
    m = kc.Model(netgen.net_bytes(name))
    ctx = kc.Context(m, gpu_idxs=[0], precision=prec)
    n_threads, n, reps = 2, 24, 6
    batches = [inputs.synthetic_inputs(n, 700 + t, (9, 13, 19), rich=True)[:2] for t in range(n_threads)]
    handles = [None] * n_threads
    errors = []

    def create(t):
        try:
            handles[t] = kc.Handle(ctx, max_batch=n, gpu_idx=0)
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=create, args=(t,)) for t in range(n_threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    alone = [handles[t].forward(*batches[t]) for t in range(n_threads)]
    results = [[] for _ in range(n_threads)]

    def run(t):
        try:
            for _ in range(reps):
                results[t].append(handles[t].forward(*batches[t]))
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=run, args=(t,)) for t in range(n_threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    for t in range(n_threads):
        assert len(results[t]) == reps
        for got in results[t]:
            for k in KEYS:
                np.testing.assert_array_equal(got[k], alone[t][k])
