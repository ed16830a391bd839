"""Expert parallelism on two GPUs (NCCL), one process per GPU.

Each rank holds half of a full-size layer's routed experts (ep_init before
the layer is created) and its own tokens; overhang_b200.ep exchanges rows
with all_to_all and the library computes routing and expert rows.  The
gathered result must equal a single-GPU forward of all tokens bit for bit
(the exchange only moves rows; every product and sum is the same operation
in the same order), and the oracle within the parity tolerance.

Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import assert_close
from gpu_common import next_layer_id, olmoe_full, qwen_full

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _rank_main(rank, world, port, kind, T, out_dir):
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, HERE)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import overhang_b200 as ob
        import pyoracle as P
        from overhang_b200.ep import ExpertParallel, LibCompute
        from gpu_common import olmoe_full, qwen_full
        ob.init(rank, 1 << 30)
        ob.ep_init(rank, world)
        L = olmoe_full() if kind == "olmoe" else qwen_full()
        layer = ob.MoELayer.from_oracle_layer(3, L)
        x_all = P.normal(9100 + T, (world * T, L.D))
        x = torch.from_numpy(np.ascontiguousarray(x_all[rank * T:(rank + 1) * T])).cuda()
        ep = ExpertParallel(LibCompute(layer), L.E, L.k, L.D, L.has_shared)
        out, idx, w = ep.forward(x)
        torch.cuda.synchronize()
        ob.sync()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out.cpu().numpy(), idx=idx.cpu().numpy(),
                 w=w.cpu().numpy())
        dist.barrier()
        ob.shutdown()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kind,T", [("olmoe", 128), ("qwen", 64)])
def test_ep_two_gpus_equals_single_gpu(gpu, oracle, tmp_path, kind, T):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), kind, T, str(tmp_path)), nprocs=2, join=True)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    out = np.concatenate([p["out"] for p in parts])
    idx = np.concatenate([p["idx"] for p in parts])
    L = olmoe_full() if kind == "olmoe" else qwen_full()
    x_all = oracle.normal(9100 + T, (2 * T, L.D))
    m = gpu.MoELayer.from_oracle_layer(next_layer_id(), L)
    gpu.set_path(gpu.PATH_MMA)
    try:
        o1, i1, _ = m.forward(x_all)
    finally:
        gpu.set_path(gpu.PATH_AUTO)
    assert np.array_equal(idx, i1)
    assert np.array_equal(out.view(np.uint32), o1.view(np.uint32)), "EP result differs from the single-GPU forward"
    sub = np.arange(0, 2 * T, 16)
    ro, ridx, _ = oracle.oracle_moe(L, x_all[sub])
    assert np.array_equal(idx[sub], ridx)
    assert_close(out[sub], ro, what=f"EP {kind}")
