"""GPU: omc_moe_forward_async / omc_moe_wait, the pipelined host entry.

Calls overlap (upload of the next x, forward, download of the previous out
on three streams, three staging slots).  Every call's results must equal the
blocking entry's (omc_moe_forward) bit for bit, including when more calls are
submitted than there are slots (a fourth submit waits for the oldest), when
T changes between calls (a slot's buffers grow) and when results are waited
for out of submission order.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_common import next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu


def _submit(gpu, lid, x, out, idx, w):
    t = C.c_longlong(-1)
    rc = gpu.lib().omc_moe_forward_async(lid, x.ctypes.data_as(C.c_void_p), x.shape[0],
                                         out.ctypes.data_as(C.c_void_p), idx.ctypes.data_as(C.c_void_p),
                                         w.ctypes.data_as(C.c_void_p), C.byref(t))
    assert rc == 0, gpu.last_error()
    return t.value


@pytest.mark.parametrize("family", ["olmoe", "qwen"])
def test_async_equals_blocking(gpu, oracle, family):
    L = olmoe_full() if family == "olmoe" else qwen_full()
    lid = next_layer_id()
    m = gpu.MoELayer.from_oracle_layer(lid, L)
    Ts = [512, 512, 64, 512, 1, 200, 512, 512, 33]
    xs = [oracle.normal(5100 + i, (T, L.D)) for i, T in enumerate(Ts)]
    want = [m.forward(x) for x in xs]
    outs = [(np.full((T, L.D), np.nan, np.float32), np.full((T, L.k), -1, np.int32), np.zeros((T, L.k), np.float32))
            for T in Ts]
    tickets = [_submit(gpu, lid, xs[i], *outs[i]) for i in range(len(Ts))]
    assert tickets == sorted(tickets) and len(set(tickets)) == len(Ts)
    # wait the newest first: waiting for a ticket also completes every older one
    assert gpu.lib().omc_moe_wait(tickets[-1]) == 0, gpu.last_error()
    for i in range(len(Ts)):
        assert gpu.lib().omc_moe_wait(tickets[i]) == 0
        o, idx, w = outs[i]
        assert np.array_equal(idx, want[i][1]), i
        assert np.array_equal(w.view(np.uint32), want[i][2].view(np.uint32)), i
        assert np.array_equal(o.view(np.uint32), want[i][0].view(np.uint32)), f"call {i} (T={Ts[i]}) differs"


def test_async_rejects_bad_ticket(gpu, oracle):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 16, 4, seed=88)
    lid = next_layer_id()
    gpu.MoELayer.from_oracle_layer(lid, L)
    assert gpu.lib().omc_moe_wait(1 << 40) == gpu.EINVAL
