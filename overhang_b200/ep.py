"""Expert parallelism for one MoE layer: one process per GPU, torch.distributed.

The experts of a layer are split into `world` contiguous ranges; rank r holds
routed experts [r*E/world, (r+1)*E/world) (call ``overhang_b200.ep_init``
before creating the layer) and the shared expert, if any.  Every rank brings
its own tokens (their *home* rank).  A forward is the reference's MoE block
(engines/olmoe.c:344-402, engines/qwen.c:453-495) with one exchange each way:

1. route the home tokens (bit-exact top-k and weights, the shared gate);
2. send each routed slot's token row, its expert id and its weight to the
   rank holding that expert (counts first, then rows; all_to_all_single);
3. run the received rows through the local experts; each row comes back
   already weighted, w * y, rounded as the reference rounds it;
4. send the weighted rows back along the same splits;
5. at home, out = sigmoid(gate) * shared(x) (or 0), then + row_k for k in
   selection order: the reference's combine order, so the result equals a
   single-GPU forward bit for bit.

The exchange is written against ``torch.distributed`` (NCCL between GPUs;
gloo works for host tensors) and a *compute* object that supplies the
per-rank device work; ``LibCompute`` is the library's (omc_moe_route_dev /
omc_moe_experts_dev on this rank's GPU).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import check, lib


class LibCompute:
    """The library's passes for one layer on this rank's GPU (device tensors,
    enqueued on torch's current stream)."""

    def __init__(self, layer):
        self.layer = layer
        self.E, self.k, self.D = layer.E, layer.k, layer.D
        self.has_shared = bool(layer.has_shared)

    def route(self, x: torch.Tensor):
        T = x.shape[0]
        idx = torch.empty((T, self.k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.k), dtype=torch.float32, device=x.device)
        sg = torch.empty(T, dtype=torch.float32, device=x.device) if self.has_shared else None
        s = torch.cuda.current_stream(x.device).cuda_stream
        check(lib().omc_moe_route_dev(self.layer.layer, C.c_void_p(x.data_ptr()), T, C.c_void_p(idx.data_ptr()),
                                      C.c_void_p(w.data_ptr()), C.c_void_p(sg.data_ptr() if sg is not None else None),
                                      C.c_void_p(s)), "omc_moe_route_dev")
        return idx, w, sg

    def experts(self, x_rows: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        R = x_rows.shape[0]
        y = torch.empty((R, self.D), dtype=torch.float32, device=x_rows.device)
        if R == 0:
            return y
        x_rows = x_rows.contiguous()
        ids = ids.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        s = torch.cuda.current_stream(x_rows.device).cuda_stream
        check(lib().omc_moe_experts_dev(self.layer.layer, C.c_void_p(x_rows.data_ptr()), R, C.c_void_p(ids.data_ptr()),
                                        C.c_void_p(w.data_ptr()), C.c_void_p(y.data_ptr()), C.c_void_p(s)),
              "omc_moe_experts_dev")
        return y


class ExpertParallel:
    """The exchange of one expert-parallel MoE layer (see the module doc)."""

    def __init__(self, compute, E: int, k: int, D: int, has_shared: bool, group=None):
        self.compute, self.group = compute, group
        self.E, self.k, self.D, self.has_shared = E, k, D, bool(has_shared)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if E % self.world:
            raise ValueError(f"E={E} is not divisible by {self.world} ranks")
        self.per_rank = E // self.world

    def forward(self, x: torch.Tensor):
        """x [T, D] f32 on this rank's device -> (out [T, D], topk_idx [T, k], topk_w [T, k])."""
        T, D, k, dev = x.shape[0], self.D, self.k, x.device
        x = x.contiguous()
        idx, w, sg = self.compute.route(x)
        # 2. slots grouped by the rank holding their expert (stable: by slot within a rank)
        dest = (idx.to(torch.int64) // self.per_rank).reshape(-1)
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_split = send_counts.tolist()
        recv_split = recv_counts.tolist()
        n_recv = int(sum(recv_split))
        self.last_recv_rows = n_recv
        send_rows = x.index_select(0, order // k)
        meta = torch.stack([idx.reshape(-1)[order], w.reshape(-1)[order].view(torch.int32)], 1).contiguous()
        recv_rows = torch.empty((n_recv, D), dtype=x.dtype, device=dev)
        recv_meta = torch.empty((n_recv, 2), dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_split, send_split, group=self.group)
        # 3. the local experts, rows weighted as the reference weights them
        y = self.compute.experts(recv_rows, recv_meta[:, 0].contiguous(),
                                 recv_meta[:, 1].contiguous().view(torch.float32))
        # 4. back along the same splits: back[j] belongs to slot order[j]
        back = torch.empty((T * k, D), dtype=torch.float32, device=dev)
        dist.all_to_all_single(back, y.contiguous(), send_split, recv_split, group=self.group)
        rows = torch.empty_like(back)
        rows[order] = back
        rows = rows.view(T, k, D)
        # 5. the reference's combine order
        if self.has_shared:
            sh = self.compute.experts(x, torch.full((T,), self.E, dtype=torch.int32, device=dev),
                                      torch.ones(T, dtype=torch.float32, device=dev))
            out = sg[:, None] * sh
        else:
            out = torch.zeros((T, D), dtype=torch.float32, device=dev)
        for kk in range(k):
            out = out + rows[:, kk]
        return out, idx, w
