"""Expert parallelism on CPU ranks (gloo, world size 2): the library's own
index arithmetic of the exchange.

The device path (omc_ep.c + ep.cu) places every row and slot with the
functions of overhang_b200/csrc/omc_ep_plan.h; the library exports the same
functions run on the host (omc_ep_layout_host, omc_ep_unpack_host), which
need no GPU.  Here two processes use them to pack, exchange (gloo
all_to_all, the stand-in for NCCL's grouped send/recv), unpack and combine,
with the oracle computing the expert rows (f32 rows instead of the device's
f16 ones, so the result can be compared exactly).  The gathered outputs must
equal the oracle's single-process forward of all tokens bit for bit: the
exchange may move rows anywhere but must return every slot to its place and
sum in the reference's order.
"""
import ctypes as C
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
        return P.make_layer(P.FAMILY_OLMOE, 128, 64, 8, 3, seed=41)
    return P.make_layer(P.FAMILY_QWEN, 128, 64, 8, 3, seed=42, renorm=1, router_i8=1, has_shared=1, Is=64)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _a2a(send, send_counts, recv_counts, width, dtype):
    """all_to_all of row blocks (rows of `width` values), gloo."""
    out = torch.empty((int(sum(recv_counts)), width), dtype=dtype)
    dist.all_to_all_single(out, torch.from_numpy(np.ascontiguousarray(send)).reshape(-1, width),
                           [int(c) for c in recv_counts], [int(c) for c in send_counts])
    return out.numpy()


def _rank_main(rank, world, port, kind, counts_tok, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import pyoracle as P
        import overhang_b200 as ob
        lib = ob.lib()
        L = _layer(kind)
        E, k, D = L.E, L.k, L.D
        x_all = P.normal(77, (sum(counts_tok), D))
        a = sum(counts_tok[:rank])
        T = counts_tok[rank]
        x = np.ascontiguousarray(x_all[a:a + T])
        idx, w = P.oracle_route(L, x)
        sg = P.oracle_shared_gate(L, x) if L.has_shared else None
        M = 2 + 2 * k
        # 1. the library's layout: positions, counts, meta rows
        tok_pos = np.full((T, world), -1, np.int32)
        slot_pos = np.full((T, k), -1, np.int32)
        cnt = np.zeros(4 * world, np.int32)
        meta = np.zeros((max(T * world, 1), M), np.int32)
        nsent = lib.omc_ep_layout_host(_p(idx), _p(w), T, k, E, world, _p(tok_pos), _p(slot_pos), _p(cnt), _p(meta))
        assert nsent == int(cnt[:world].sum())
        send_rows, send_slots = cnt[:world], cnt[world:2 * world]
        send_x = np.zeros((max(nsent, 1), D), np.float32)
        for t in range(T):
            for r in range(world):
                if tok_pos[t, r] >= 0:
                    send_x[tok_pos[t, r]] = x[t]
        # 2. counts, then rows and meta
        pairs = np.stack([send_rows, send_slots], 1).astype(np.int64)
        recv_pairs = _a2a(pairs, [1] * world, [1] * world, 2, torch.int64)
        recv_rows, recv_slots = recv_pairs[:, 0].astype(np.int32), recv_pairs[:, 1].astype(np.int32)
        rx = _a2a(send_x[:nsent], send_rows, recv_rows, D, torch.float32)
        rm = _a2a(meta[:nsent], send_rows, recv_rows, M, torch.int32)
        # 3. the library's unpack: slots numbered in the senders' return order
        Rr, Sr = int(recv_rows.sum()), int(recv_slots.sum())
        Ntot = Sr + (T if L.has_shared else 0)
        slot_tok = np.zeros(max(Ntot, 1), np.int32)
        slot_e = np.zeros(max(Ntot, 1), np.int32)
        slot_w = np.zeros(max(Ntot, 1), np.float32)
        n = lib.omc_ep_unpack_host(_p(np.ascontiguousarray(rm, np.int32)), _p(recv_rows), _p(recv_slots), world, k,
                                   T, E, L.has_shared, _p(slot_tok), _p(slot_e), _p(slot_w))
        assert n == Ntot
        per = E // world
        held = ((slot_e[:Ntot] >= rank * per) & (slot_e[:Ntot] < (rank + 1) * per)) | (slot_e[:Ntot] == E)
        assert held.all(), "a slot reached a rank that does not hold its expert"
        opnd = np.concatenate([x, rx]) if Rr else x
        y = np.zeros((max(Ntot, 1), D), np.float32)
        if Ntot:
            yy = P.oracle_expert_rows(L, np.ascontiguousarray(opnd[slot_tok[:Ntot]]), slot_e[:Ntot])
            y[:Ntot] = (slot_w[:Ntot, None] * yy).astype(np.float32)
        # 4. partials back, combine in the reference's order
        ret = _a2a(y[:Sr], recv_slots, send_slots, D, torch.float32)
        out = np.zeros((T, D), np.float32)
        for t in range(T):
            acc = (np.float32(sg[t]) * y[Sr + t]).astype(np.float32) if L.has_shared else np.zeros(D, np.float32)
            for kk in range(k):
                acc = (acc + ret[slot_pos[t, kk]]).astype(np.float32)
            out[t] = acc
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out, idx=idx, w=w)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("kind,counts", [("olmoe", (5, 3)), ("qwen", (4, 4)), ("olmoe", (6, 0)), ("qwen", (9, 7))])
def test_ep_exchange_matches_single_process(oracle, omc_lib, tmp_path, kind, counts):
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


def test_layout_host_positions(omc_lib):
    """The layout's definitions on a hand-made routing (E=8, k=3, 4 ranks):
    rows deduplicated per rank, blocks in rank order, slots in token then
    selection order."""
    lib = omc_lib.lib()
    idx = np.array([[0, 1, 7], [6, 2, 3], [5, 4, 0]], np.int32)     # owners: r = e // 2
    w = np.arange(9, dtype=np.float32).reshape(3, 3) / 10
    P, k, E, T = 4, 3, 8, 3
    tok_pos = np.zeros((T, P), np.int32)
    slot_pos = np.zeros((T, k), np.int32)
    cnt = np.zeros(4 * P, np.int32)
    meta = np.zeros((T * P, 2 + 2 * k), np.int32)
    n = lib.omc_ep_layout_host(_p(idx), _p(w), T, k, E, P, _p(tok_pos), _p(slot_pos), _p(cnt), _p(meta))
    # rank 0 gets tokens 0 (experts 0,1) and 2 (expert 0); rank 1 tokens 1 (2,3);
    # rank 2 token 2 (5,4); rank 3 tokens 0 (7) and 1 (6)
    assert list(cnt[:P]) == [2, 1, 1, 2] and list(cnt[P:2 * P]) == [3, 2, 2, 2] and n == 6
    assert list(cnt[2 * P:3 * P]) == [0, 2, 3, 4] and list(cnt[3 * P:]) == [0, 3, 5, 7]
    assert tok_pos.tolist() == [[0, -1, -1, 4], [-1, 2, -1, 5], [1, -1, 3, -1]]
    assert slot_pos.tolist() == [[0, 1, 7], [8, 3, 4], [5, 6, 2]]
    # token 2 on rank 2: its block's first slot (offset 0), two experts 5 then 4
    assert meta[3, :4].tolist() == [0, 2, 5, 4] and meta[3, 4] == -1
