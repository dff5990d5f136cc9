"""Failure detection without a GPU fault, through the C ABI.

* A device wait that runs out: kc_selftest_device_timeout enqueues a kernel whose bounded mbarrier wait (the same
  wait every kernel of the forward pass makes, with a limit of a millisecond instead of 2 s) is on a barrier nothing
  completes. The kernel records its error code and returns; the next wait reports KC_ERR_DEVICE, and the handle
  keeps working.
* A host wait that runs out: kc_wait with a 0 ms limit on a batch still in flight returns KC_ERR_TIMEOUT and leaves
  the batch in flight; a later wait without a limit returns its outputs. The handle's stream is held busy by a
  bounded sleep kernel (torch) queued ahead of the batch.
"""

import numpy as np
import pytest

import katago_cuda as kc
from katago_cuda import api, inputs, netgen
from oracle.oracle import OracleNet

pytestmark = pytest.mark.gpu

KEYS = ("policy", "value", "scorevalue", "ownership")


def make(name="tiny-nbt", n=8):
    m = kc.Model(netgen.net_bytes(name))
    h = kc.Handle(kc.Context(m, gpu_idxs=[0], precision=kc.PRECISION_F16), max_batch=n, gpu_idx=0)
    x = inputs.synthetic_inputs(n, 31, (9, 13, 19), rich=True)[:2]
    return h, x


def test_device_wait_runs_out_and_handle_recovers():
    h, (spatial, glob) = make()
    want = OracleNet(netgen.net_bytes("tiny-nbt")).forward(spatial, glob)
    h.selftest_device_timeout(1000)
    with pytest.raises(api.KcError) as e:
        h.wait(10000)
    assert e.value.status == api.KC_ERR_DEVICE
    assert "gave up waiting" in str(e.value) and "code 6" in str(e.value)
    # the error word was cleared and the context is usable: a normal batch follows
    got = h.forward(spatial, glob)
    for k in KEYS:
        assert float(np.abs(got[k] - want[k]).max()) <= 2e-2, k


def test_host_wait_times_out_then_completes():
    torch = pytest.importorskip("torch")
    h, (spatial, glob) = make("small-nbt", 16)
    first = h.forward(spatial, glob)
    h.spatial[:16] = spatial
    h.glob[:16] = glob
    with torch.cuda.device(0):
        busy = torch.cuda.ExternalStream(h.stream_ptr(), device=0)
        with torch.cuda.stream(busy):
            torch.cuda._sleep(200_000_000)  # ~0.1 s of spinning on the handle's stream, bounded
    h.enqueue(16)
    with pytest.raises(api.KcError) as e:
        h.wait(0)
    assert e.value.status == api.KC_ERR_TIMEOUT
    # the batch is still in flight: another enqueue is refused, the staging buffers are not touched
    with pytest.raises(api.KcError) as e2:
        h.enqueue(16)
    assert e2.value.status == api.KC_ERR_INVALID
    rows = np.array(h.wait(-1)[:16])
    got = h.split(rows)
    for k in KEYS:
        np.testing.assert_array_equal(got[k], first[k])
