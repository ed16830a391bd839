"""Expert parallelism on CPU ranks (gloo, world size 2).

The exchange of overhang_b200.ep runs for real between two processes; the
oracle supplies each rank's routing and the rows of the experts it holds
(a test double of the library's device passes, refusing any expert the rank
does not hold).  The gathered outputs must equal the oracle's single-process
forward of all tokens bit for bit: the exchange may move rows anywhere but
must sum them in the reference's order.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _layer(kind):
    import pyoracle as P
    if kind == "olmoe":
        return P.make_layer(P.FAMILY_OLMOE, 128, 64, 8, 2, seed=41)
    return P.make_layer(P.FAMILY_QWEN, 128, 64, 8, 2, seed=42, renorm=1, router_i8=1, has_shared=1, Is=64)


class OracleCompute:
    """One rank's device work, done by the oracle (test double)."""

    def __init__(self, L, lo, hi):
        self.L, self.lo, self.hi = L, lo, hi

    def route(self, x):
        import pyoracle as P
        idx, w = P.oracle_route(self.L, x.numpy())
        sg = torch.from_numpy(P.oracle_shared_gate(self.L, x.numpy())) if self.L.has_shared else None
        return torch.from_numpy(idx), torch.from_numpy(w), sg

    def experts(self, x_rows, ids, w):
        import pyoracle as P
        ids_np = ids.numpy()
        held = ((ids_np >= self.lo) & (ids_np < self.hi)) | (ids_np == self.L.E)
        assert held.all(), "a row reached a rank that does not hold its expert"
        y = P.oracle_expert_rows(self.L, x_rows.numpy(), ids_np)
        return torch.from_numpy((w.numpy()[:, None] * y).astype(np.float32))


def _rank_main(rank, world, port, kind, counts, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import pyoracle as P
        from overhang_b200.ep import ExpertParallel
        L = _layer(kind)
        x_all = P.normal(77, (sum(counts), L.D))
        a = sum(counts[:rank])
        x = torch.from_numpy(np.ascontiguousarray(x_all[a:a + counts[rank]]))
        per = L.E // world
        ep = ExpertParallel(OracleCompute(L, rank * per, (rank + 1) * per), L.E, L.k, L.D, L.has_shared)
        out, idx, w = ep.forward(x)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out.numpy(), idx=idx.numpy(), w=w.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("kind,counts", [("olmoe", (5, 3)), ("qwen", (4, 4)), ("olmoe", (6, 0))])
def test_ep_exchange_matches_single_process(oracle, tmp_path, kind, counts):
    mp.spawn(_rank_main, args=(2, _free_port(), kind, counts, str(tmp_path)), nprocs=2, join=True)
    L = _layer(kind)
    x_all = oracle.normal(77, (sum(counts), L.D))
    ro, ridx, rw = oracle.oracle_moe(L, x_all)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    out = np.concatenate([p["out"] for p in parts])
    idx = np.concatenate([p["idx"] for p in parts])
    w = np.concatenate([p["w"] for p in parts])
    assert np.array_equal(idx, ridx)
    assert np.array_equal(w.view(np.uint32), rw.view(np.uint32))
    assert np.array_equal(out.view(np.uint32), ro.view(np.uint32)), "EP sum differs from the single-process forward"
