"""Expert parallelism for the FP4 MoE FFN over torch.distributed.

The routed experts are sharded contiguously over the ranks of a process group
(rank r owns experts [r*E_l, (r+1)*E_l)); the shared expert is replicated.  One
forward on every rank:

    dispatch (act quant, one row per route, grouped by destination rank)
    all-to-all of the per-(rank, expert) counts, all-to-all of the rows
    expert FFN on the received rows (grouped tcgen05 GEMMs) + shared expert
    all-to-all of the f32 result rows back to their token's rank
    combine (ascending expert id, w / sum(w)) + shared

The collective sequence (`ep_step`) is written once against a small device-ops
interface: `DeviceOps` runs the library's kernels through the C ABI (NCCL
process group on the GPU); the CPU tests drive the same sequence over gloo with
a numpy stand-in for the kernels.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

from . import (Context, DeepSeekV4Fp4Expert, Fp4ExpertSpec, MoeDesc, _check, _ptr, _stream,
               lib)


def ep_step(ops, x, ids, weights, world: int, local_experts: int, group=None):
    """One expert-parallel MoE step for this rank's tokens x [T, hidden] with
    routes ids/weights [T, topk].  `ops` provides dispatch / expert_ffn /
    combine and the tensor factory; the all-to-alls go over `group`."""
    import torch.distributed as dist

    send, send_counts, pos = ops.dispatch(x, ids)
    recv_counts = ops.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    per_dest = ops.to_list(send_counts.view(world, local_experts).sum(1))
    per_src = ops.to_list(recv_counts.view(world, local_experts).sum(1))
    R = sum(per_src)
    recv = ops.empty_rows(R)
    dist.all_to_all_single(recv, send, output_split_sizes=per_src, input_split_sizes=per_dest,
                           group=group)
    y_rows = ops.expert_ffn(recv, recv_counts, R, x)
    y_back = ops.empty_results(send.shape[0])
    dist.all_to_all_single(y_back, y_rows[:R], output_split_sizes=per_dest,
                           input_split_sizes=per_src, group=group)
    return ops.combine(ids, weights, pos, y_back, y_rows[R:])


class DeviceOps:
    """The C-ABI kernels (wh_ep_dispatch / wh_ep_expert_ffn / wh_ep_combine)."""

    def __init__(self, layer: "EpMoeLayer"):
        self.l = layer

    def empty_like(self, t):
        import torch

        return torch.empty_like(t)

    def to_list(self, t):
        return [int(v) for v in t.tolist()]

    def empty_rows(self, n):
        import torch

        return torch.empty(n, self.l.row_bytes, dtype=torch.uint8, device=self.l.device)

    def empty_results(self, n):
        import torch

        return torch.empty(n, self.l.hidden, dtype=torch.float32, device=self.l.device)

    def dispatch(self, x, ids):
        import torch

        l = self.l
        T = x.shape[0]
        send = torch.empty(T * l.topk, l.row_bytes, dtype=torch.uint8, device=l.device)
        counts = torch.empty(l.world * l.local_experts, dtype=torch.int32, device=l.device)
        pos = torch.empty(T * l.topk, dtype=torch.int32, device=l.device)
        l._ensure_scratch(T, 0)
        _check(lib().wh_ep_dispatch(l.ctx.handle, l.plan, l.world, _ptr(x), T, _ptr(ids),
                                    _ptr(send), _ptr(counts), _ptr(pos), _ptr(l.scratch),
                                    l.scratch.numel(), _stream(None)))
        self.pos = pos
        return send, counts, pos

    def expert_ffn(self, recv, recv_counts, R, x):
        import torch

        l = self.l
        T = x.shape[0]
        y_rows = torch.empty(R + T, l.hidden, dtype=torch.float32, device=l.device)
        l._ensure_scratch(T, R)
        _check(lib().wh_ep_expert_ffn(l.ctx.handle, l.plan, l.world, _ptr(recv),
                                      _ptr(recv_counts), R, _ptr(x), T, _ptr(y_rows),
                                      _ptr(l.scratch), l.scratch.numel(), _stream(None)))
        return y_rows

    def combine(self, ids, weights, pos, y_back, y_shared):
        import torch

        l = self.l
        T = ids.shape[0]
        y = torch.empty(T, l.hidden, dtype=torch.float32, device=l.device)
        _check(lib().wh_ep_combine(l.ctx.handle, l.plan, _ptr(ids), _ptr(weights), _ptr(pos), T,
                                   _ptr(y_back), _ptr(y_shared), _ptr(y), _stream(None)))
        return y


class EpMoeLayer:
    """This rank's shard of an expert-parallel MoE FFN layer.

    local_experts: the experts [rank*E_l, (rank+1)*E_l) of the layer;
    shared: the replicated shared expert (or None).  forward(x, ids, weights)
    takes this rank's tokens and their routes (global expert ids) and returns
    the layer output for them."""

    def __init__(self, ctx: Context, local_experts: Sequence[DeepSeekV4Fp4Expert],
                 shared: Optional[DeepSeekV4Fp4Expert], world: int, topk: int = 6,
                 group=None):
        self.ctx = ctx
        self.world = world
        self.group = group
        self.topk = topk
        self.local_experts = len(local_experts)
        self.hidden = local_experts[0].w1.cols
        self.inter = local_experts[0].w1.rows
        self.device = f"cuda:{ctx.device}"
        self._keep = (list(local_experts), shared)
        arr = (Fp4ExpertSpec * len(local_experts))(*[e.spec() for e in local_experts])
        sh = shared.spec() if shared is not None else None
        d = MoeDesc(len(local_experts), self.hidden, self.inter, arr,
                    C.pointer(sh) if sh is not None else None, None, None, topk, 0, 1.0, 1, 0)
        h = C.c_void_p()
        _check(lib().wh_moe_plan_create(ctx.handle, C.byref(d), C.byref(h)))
        self.plan = h
        self.row_bytes = lib().wh_ep_row_bytes(self.hidden)
        self.scratch = None

    def _ensure_scratch(self, tokens: int, recv_rows: int):
        import torch

        need = lib().wh_ep_scratch_bytes(self.plan, self.world, tokens, recv_rows)
        if self.scratch is None or self.scratch.numel() < need:
            self.scratch = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8,
                                       device=self.device)

    def forward(self, x, ids, weights):
        return ep_step(DeviceOps(self), x, ids, weights, self.world, self.local_experts,
                       self.group)

    def close(self):
        if getattr(self, "plan", None):
            lib().wh_moe_plan_destroy(self.plan)
            self.plan = None
