"""Expert parallelism for the FP4 MoE FFN over torch.distributed.

The routed experts are sharded contiguously over the ranks of a process group
(rank r owns experts [r*E_l, (r+1)*E_l)); the shared expert is replicated.  One
forward on every rank:

    dispatch (act quant, one row per route, grouped by destination rank)
    all-to-all of the per-(rank, expert) counts, all-to-all of the rows
    expert FFN on the received rows (grouped tcgen05 GEMMs) + shared expert
    all-to-all of the f32 result rows back to their token's rank
    combine (ascending expert id, w / sum(w)) + shared

Two transports move the rows:

* "p2p" (default): no collective and no host synchronisation per step.  Every
  rank exports a window of device memory over CUDA IPC (handles exchanged once
  with the process group); the dispatch kernel stores each route's row into its
  destination's window over NVLink, the down GEMM's epilogue stores each result
  row into the window of the token's rank, and arrival flags with bounded
  device-side waits order the three calls (wh_ep_p2p_*).
* "nccl": the collective sequence `ep_step` (all-to-all of counts, rows and
  results over the process group), written once against a small device-ops
  interface: `DeviceOps` runs the library's kernels through the C ABI; the CPU
  tests drive the same sequence over gloo with a numpy stand-in for the
  kernels.
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
    # one host synchronisation for both split lists
    both = ops.to_list(ops.cat([send_counts.view(world, local_experts).sum(1),
                                recv_counts.view(world, local_experts).sum(1)]))
    per_dest, per_src = both[:world], both[world:]
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

    def cat(self, ts):
        import torch

        return torch.cat(ts)

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
                 group=None, transport: str = "p2p", max_tokens: int = 1024):
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"transport must be 'p2p' or 'nccl', not {transport!r}")
        self.ctx = ctx
        self.world = world
        self.group = group
        self.transport = transport
        self.max_tokens = max_tokens
        self.window = None
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
        if transport == "p2p":
            self._connect()

    def _connect(self):
        """Create this rank's window and connect to every rank's (collective)."""
        import torch.distributed as dist

        rank = dist.get_rank(self.group) if self.world > 1 else 0
        handle = (C.c_uint8 * 64)()
        win = C.c_void_p()
        _check(lib().wh_ep_window_create(self.ctx.handle, self.plan, self.world, rank,
                                         self.max_tokens, C.byref(win), handle))
        self.window = win
        mine = bytes(handle)
        if self.world > 1:
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=self.group)
        else:
            allh = [mine]
        buf = (C.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(allh))
        _check(lib().wh_ep_window_connect(self.window, buf))

    def _ensure_scratch(self, tokens: int, recv_rows: int):
        import torch

        need = lib().wh_ep_scratch_bytes(self.plan, self.world, tokens, recv_rows)
        if self.scratch is None or self.scratch.numel() < need:
            self.scratch = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8,
                                       device=self.device)

    def forward(self, x, ids, weights):
        if self.transport == "nccl":
            return ep_step(DeviceOps(self), x, ids, weights, self.world, self.local_experts,
                           self.group)
        return self.forward_p2p(x, ids, weights)

    def forward_p2p(self, x, ids, weights, marks=None):
        """The peer-transport step: one wh_ep_moe_layer call, or, when
        `marks(i)` is given, its three calls with marks(i) called before the
        first and after each (event records for phase times)."""
        import torch

        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        L, s, h = lib(), _stream(None), self.ctx.handle
        if marks is None:
            y = torch.empty(T, self.hidden, dtype=torch.float32, device=self.device)
            _check(L.wh_ep_moe_layer(h, self.window, _ptr(x), T, _ptr(ids), _ptr(weights),
                                     _ptr(y), s))
            return y
        pos = torch.empty(T * self.topk, dtype=torch.int32, device=self.device)
        ysh = torch.empty(T, self.hidden, dtype=torch.float32, device=self.device)
        y = torch.empty(T, self.hidden, dtype=torch.float32, device=self.device)
        if marks:
            marks(0)
        _check(L.wh_ep_p2p_dispatch(h, self.window, _ptr(x), T, _ptr(ids), _ptr(pos), s))
        if marks:
            marks(1)
        _check(L.wh_ep_p2p_expert_ffn(h, self.window, _ptr(x), T, _ptr(ysh), s))
        if marks:
            marks(2)
        _check(L.wh_ep_p2p_combine(h, self.window, _ptr(ids), _ptr(weights), _ptr(pos), T,
                                   _ptr(ysh), _ptr(y), s))
        if marks:
            marks(3)
        return y

    def close(self):
        """Collective for the peer transport: no rank may still store into a
        window that is being freed."""
        if self.window is not None:
            import torch
            import torch.distributed as dist

            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            lib().wh_ep_window_destroy(self.window)
            self.window = None
        if getattr(self, "plan", None):
            lib().wh_moe_plan_destroy(self.plan)
            self.plan = None
