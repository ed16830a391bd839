"""Expert parallelism on two GPUs through the library's NCCL data plane, one
process per GPU.

Each rank joins the library's NCCL group (omc_ep_unique_id on rank 0, the id
passed to rank 1 over a gloo group, omc_ep_init), holds half of a full-size
layer's routed experts and brings its own tokens; omc_moe_forward runs the
whole exchange (route, f16 rows out, experts, f32 partials back, combine).
The gathered result must equal a single-GPU tensor-core forward of all tokens
bit for bit, and the oracle within the parity tolerance.

The failure test: after one good forward, rank 1 leaves (exits between steps,
nothing of its own in flight); rank 0's next forward must come back with
OMC_ETIMEOUT or OMC_ENCCL within its deadline instead of hanging, and the
forward after that with OMC_ENCCL.  NVLS is off (NCCL_NVLS_ENABLE=0) and the
library's own kernels never wait on a peer.

Skipped when fewer than two GPUs are visible.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch

from conftest import assert_close
from gpu_common import next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _layer(kind):
    import pyoracle as P
    if kind == "olmoe":
        return olmoe_full()
    if kind == "qwen_zipf":
        return P.make_layer(P.FAMILY_QWEN, 2048, 512, 256, 8, seed=2, renorm=1, router_i8=1, has_shared=1, Is=512,
                            router_bias=P.zipf_bias(256, 1.1, seed=22))
    return qwen_full()


def _join(rank, world, port):
    """gloo group for the id exchange and barriers; the library's own NCCL group."""
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, HERE)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import overhang_b200 as ob
    ob.init(rank, 4 << 30)
    obj = [ob.ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    ob.ep_init(rank, world, obj[0])
    return dist, ob


def _rank_main(rank, world, port, kind, counts, out_dir, combine="exact"):
    dist, ob = _join(rank, world, port)
    try:
        if combine == "ranksum":
            ob.ep_set_combine(ob.EP_RANKSUM)
        import pyoracle as P
        L = _layer(kind)
        layer = ob.MoELayer.from_oracle_layer(3, L)
        x_all = P.normal(9100 + sum(counts), (sum(counts), L.D))
        a = sum(counts[:rank])
        x = np.ascontiguousarray(x_all[a:a + counts[rank]])
        out, idx, w = layer.forward(x)
        out2, _, _ = layer.forward(x)          # a second forward on the grown buffers
        assert np.array_equal(out.view(np.uint32), out2.view(np.uint32)), "EP forward not deterministic"
        ob.sync()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out, idx=idx, w=w)
        dist.barrier()
        ob.shutdown()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


needs_two = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


@needs_two
@pytest.mark.parametrize("kind,counts", [("olmoe", (128, 128)), ("qwen", (64, 64)), ("qwen", (100, 28)),
                                         ("olmoe", (40, 0)), ("qwen_zipf", (256, 256))])
def test_ep_two_gpus_equals_single_gpu(gpu, oracle, tmp_path, kind, counts):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), kind, counts, str(tmp_path)), nprocs=2, join=True)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    out = np.concatenate([p["out"] for p in parts])
    idx = np.concatenate([p["idx"] for p in parts])
    L = _layer(kind)
    x_all = oracle.normal(9100 + sum(counts), (sum(counts), L.D))
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    gpu.set_path(gpu.PATH_MMA)
    try:
        o1, i1, _ = m.forward(x_all)
    finally:
        gpu.set_path(gpu.PATH_AUTO)
    assert np.array_equal(idx, i1)
    assert np.array_equal(out.view(np.uint32), o1.view(np.uint32)), "EP result differs from the single-GPU forward"
    sub = np.arange(0, sum(counts), 8)
    ro, ridx, _ = oracle.oracle_moe(L, x_all[sub])
    assert np.array_equal(idx[sub], ridx)
    assert_close(out[sub], ro, what=f"EP {kind}")


@needs_two
@pytest.mark.parametrize("kind,counts", [("olmoe", (96, 160)), ("qwen_zipf", (128, 128))])
def test_ep_rank_sums_within_tolerance(gpu, oracle, tmp_path, kind, counts):
    """OMC_EP_RANKSUM: the expert ranks return one row per (token, rank); the
    same terms summed in another order, so the result is the single-GPU
    forward's within the parity tolerance (not bit for bit)."""
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), kind, counts, str(tmp_path), "ranksum"), nprocs=2, join=True)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    out = np.concatenate([p["out"] for p in parts])
    idx = np.concatenate([p["idx"] for p in parts])
    L = _layer(kind)
    x_all = oracle.normal(9100 + sum(counts), (sum(counts), L.D))
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    gpu.set_path(gpu.PATH_MMA)
    try:
        o1, i1, _ = m.forward(x_all)
    finally:
        gpu.set_path(gpu.PATH_AUTO)
    assert np.array_equal(idx, i1)
    assert_close(out, o1, what=f"EP rank sums {kind} vs one GPU")
    sub = np.arange(0, sum(counts), 8)
    ro, ridx, _ = oracle.oracle_moe(L, x_all[sub])
    assert np.array_equal(idx[sub], ridx)
    assert_close(out[sub], ro, what=f"EP {kind}")


def _leave_main(rank, world, port, out_dir):
    dist, ob = _join(rank, world, port)
    import pyoracle as P
    L = olmoe_full()
    layer = ob.MoELayer.from_oracle_layer(3, L)
    x = P.normal(9300 + rank, (32, L.D))
    layer.forward(x)                            # one good step on both ranks
    ob.sync()
    dist.barrier()
    if rank == 1:
        os._exit(0)                             # leaves between steps, nothing in flight
    ob.ep_set_timeout(3000)
    t0 = time.perf_counter()
    try:
        layer.forward(x)
        status = 0
    except ob.OmcError as e:
        status = e.status
    dt = time.perf_counter() - t0
    try:
        layer.forward(x)
        status2 = 0
    except ob.OmcError as e:
        status2 = e.status
    np.savez(os.path.join(out_dir, "leave.npz"), status=status, status2=status2, seconds=dt)
    ob.shutdown()
    os._exit(0)                                 # the gloo peer is gone: no group teardown


@needs_two
def test_ep_rank_leaves_between_steps(gpu, tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.spawn(_leave_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False)
    deadline = time.time() + 120
    while not ctx.join(timeout=5):
        assert time.time() < deadline, "ranks did not finish"
    r = np.load(tmp_path / "leave.npz")
    assert int(r["status"]) in (gpu.ETIMEOUT, gpu.ENCCL), int(r["status"])
    assert float(r["seconds"]) < 3.0 + 10.0, float(r["seconds"])
    assert int(r["status2"]) == gpu.ENCCL
