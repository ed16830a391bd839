"""GPU: the tiered expert store (omc_tier_enable) -- a layer with only some
of its experts in HBM slots, every expert's home in pinned host memory, and
the reference's LFRU hot-store policy (include/tier.h:30-58) moving the hot
ones into the slots.

A tiered layer never lets a kernel read host memory: after routing, the
routed experts outside the HBM slots are copied into an HBM miss area
(tier.cu), and the expert kernels read that.  Its T = 1 forwards take the
router + CUDA-core path (the fused decode kernel routes and runs the
experts in one launch, leaving no point to copy them in).

Bar:
  * outputs and routing of a tiered layer are bit-identical to the same
    layer fully resident on the same expert path (CUDA-core GEMV,
    tensor-core grouped GEMM), through swaps, misses, graph replay, the
    device-pointer entry and the no-alloc entry;
  * the device heat counters equal the oracle's accounting of the routing
    the forwards returned, and the device's miss count equals the routed
    experts that were outside the slots;
  * every swap is the one the oracle's tier.h restatement picks from those
    counters, and the hot experts end up resident.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_common import next_layer_id

pytestmark = pytest.mark.gpu

D, I, E, K = 1024, 512, 32, 4
HOT = np.arange(20, 28)      # routed most often; not among the first slots
SLOTS = 8


@pytest.fixture(scope="module")
def layer(oracle):
    return oracle.make_layer(oracle.FAMILY_OLMOE, D, I, E, K, seed=8800)


def _inputs(oracle, L, seed, T):
    r = L.arrays["router"]
    m = r[HOT].sum(0)
    m = (m / np.linalg.norm(m)).astype(np.float32)
    return np.ascontiguousarray(oracle.normal(seed, (T, D)) + np.float32(3.0) * m)


def _predict(oracle, heat, last, clock, pinned):
    return oracle.Tier("oracle").pick_lfru(heat, last, clock, pinned)


SEQ = [1, 1, 1, 4, 4, 16, 16, 16, 64, 64, 256, 256, 256, 1, 1, 8, 8, 512, 512, 1]


def test_tier_bit_identical_and_policy(gpu, oracle, layer):
    """Automatic mode (a decision after every forward): each forward equals
    the resident layer's bit for bit; heat equals the oracle's count; each
    swap is the oracle's pick from the counters the previous forward left."""
    A = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer)
    B = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer, tier=(SLOTS, 1, 0))
    orc = oracle.Tier("oracle")
    heat, last, clock = np.zeros(E, np.uint32), np.zeros(E, np.uint32), 0
    pinned = np.arange(SLOTS, dtype=np.int32)
    _, _, _, slots, swaps, misses = B.tier_stats(SLOTS)
    assert np.array_equal(slots, pinned) and swaps == 0 and misses == 0
    want_misses = 0
    for i, T in enumerate(SEQ * 2):
        x = _inputs(oracle, layer, 9000 + i, T)
        # the decision made at this forward's entry: from the counters so far
        pick = _predict(oracle, heat, last, clock, pinned) if i > 0 else None
        if T == 1:   # the resident layer on the tiered layer's T = 1 path
            gpu.set_path(gpu.PATH_GEMV)
        try:
            oa, ia, wa = A.forward(x)
        finally:
            gpu.set_path(gpu.PATH_AUTO)
        ob, ib, wb = B.forward(x)
        assert np.array_equal(ia, ib) and np.array_equal(wa.view(np.uint32), wb.view(np.uint32))
        assert np.array_equal(oa.view(np.uint32), ob.view(np.uint32)), f"forward {i} T={T}"
        if pick is not None:
            pinned = pinned.copy()
            pinned[pick[0]] = pick[1]
        # this forward copied in every routed expert outside the slots it found
        want_misses += len(set(np.unique(ib).tolist()) - set(pinned.tolist()))
        heat, last, clock = orc.account(ib, E, heat, last, clock)
        h, l, c, slots, swaps, misses = B.tier_stats(SLOTS)
        assert c == clock and np.array_equal(h, heat) and np.array_equal(l, last), f"counters after forward {i}"
        assert np.array_equal(slots, pinned), f"slots after forward {i}: {slots} vs {pinned}"
        assert misses == want_misses, f"misses after forward {i}"
    assert swaps >= SLOTS // 2
    assert len(set(slots.tolist()) & set(HOT.tolist())) >= SLOTS - 2


def test_tier_step_and_decay(gpu, oracle, layer):
    """Manual mode (interval 0) with decay: nothing moves until omc_tier_step,
    which makes exactly the oracle's pick; halving every 3 forwards."""
    B = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer, tier=(SLOTS, 0, 3))
    orc = oracle.Tier("oracle")
    heat, last, clock = np.zeros(E, np.uint32), np.zeros(E, np.uint32), 0
    pinned = np.arange(SLOTS, dtype=np.int32)
    ref = oracle.oracle_moe
    for i in range(14):
        x = _inputs(oracle, layer, 9500 + i, 96)
        out, idx, _ = B.forward(x)
        ro, ridx, _ = ref(layer, x)
        assert np.array_equal(idx, ridx)
        heat, last, clock = orc.account(idx, E, heat, last, clock, decay_every=3)
        h, l, c, slots, swaps, _ = B.tier_stats(SLOTS)
        assert c == clock and np.array_equal(h, heat) and np.array_equal(l, last)
        assert np.array_equal(slots, pinned)          # no automatic decisions
        if i % 2 == 1:
            pick = _predict(oracle, heat, last, clock, pinned)
            e = B.tier_step()
            assert e == (pick[1] if pick else -1)
            if pick:
                pinned = pinned.copy()
                pinned[pick[0]] = pick[1]
            assert np.array_equal(B.tier_stats(SLOTS)[3], pinned)


def test_tier_dev_noalloc_and_gemma(gpu, oracle, layer):
    """The device-pointer and no-alloc entries on a tiered layer, and a
    tiered GEMMA layer: results equal the resident layer's."""
    import torch
    A = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer)
    B = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer, tier=(4, 1, 0))
    s = torch.cuda.current_stream().cuda_stream
    for i, T in enumerate([2, 32, 256, 2, 32, 256, 256]):
        x = torch.from_numpy(_inputs(oracle, layer, 9700 + i, T)).cuda()
        outs = []
        for m, entry in ((A, "dev"), (B, "dev"), (B, "noalloc")):
            out = torch.empty_like(x)
            idx = torch.empty((T, K), dtype=torch.int32, device="cuda")
            if entry == "dev":
                m.forward_dev(x.data_ptr(), T, out.data_ptr(), idx.data_ptr(), 0, s)
            else:
                gpu.check(gpu.lib().omc_moe_forward_noalloc(m.layer, C.c_void_p(x.data_ptr()), T,
                                                            C.c_void_p(out.data_ptr()), C.c_void_p(idx.data_ptr()),
                                                            None, C.c_void_p(s)), "noalloc")
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
    assert B.tier_stats(4)[4] > 0
    G = oracle.make_layer(oracle.FAMILY_GEMMA, 512, 256, 16, 4, seed=8810)
    GA = gpu.MoELayer.from_oracle_layer(next_layer_id(), G)
    GB = gpu.MoELayer.from_oracle_layer(next_layer_id(), G, tier=(3, 1, 0))
    for i, T in enumerate([2, 24, 200, 2, 24, 200]):
        x = oracle.normal(9800 + i, (T, 512), 2.0)
        oa, ia, _ = GA.forward(x)
        ob, ib, _ = GB.forward(x)
        assert np.array_equal(ia, ib) and np.array_equal(oa.view(np.uint32), ob.view(np.uint32))


def test_tier_rejects_rows_entry_and_forced_decode(gpu, oracle, layer):
    import torch
    from gpu_common import experts_dev
    B = gpu.MoELayer.from_oracle_layer(next_layer_id(), layer, tier=(SLOTS, 1, 0))
    rows = torch.from_numpy(oracle.normal(8830, (4, D))).cuda()
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(gpu.OmcError):
        experts_dev(B, rows, ids, torch.ones(4, device="cuda"))
    gpu.set_path(gpu.PATH_DECODE)
    try:
        with pytest.raises(gpu.OmcError):
            B.forward(oracle.normal(8831, (1, D)))
    finally:
        gpu.set_path(gpu.PATH_AUTO)


def test_tier_enable_rules(gpu, oracle):
    L = oracle.make_layer(oracle.FAMILY_OLMOE, 256, 128, 8, 2, seed=8820)
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    with pytest.raises(gpu.OmcError):          # experts already uploaded
        m.tier_enable(4)
    a = L.arrays
    n = gpu.MoELayer(next_layer_id(), L.family, L.D, L.I, L.E, L.k, a["router"])
    for bad in ((0, 1, 0), (9, 1, 0), (4, -1, 0), (4, 1, -2)):
        with pytest.raises(gpu.OmcError):
            n.tier_enable(*bad)
    n.tier_enable(8, 1, 0)                     # every expert resident: a valid store that never swaps
    with pytest.raises(gpu.OmcError):
        n.tier_enable(4)                       # already tiered
    n.set_experts_packed(a["g"], a["gs"], a["u"], a["us"], a["d"], a["ds"])
    x = oracle.normal(8821, (40, 256))
    out, idx, _ = n.forward(x)
    ro, ridx, _ = oracle.oracle_moe(L, x)
    assert np.array_equal(idx, ridx)
    assert n.tier_stats(8)[4] == 0
