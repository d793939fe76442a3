"""Peer-memory expert parallelism, host side, on CPU ranks over gloo.

EpMoeLayer(transport="p2p") creates one window per rank, all-gathers the
64-byte IPC handles over the process group and connects each window to every
rank's handle in rank order; close() barriers before the window is freed.
The C library is replaced by a recorder (no device work), so the test checks
the exchange itself: every rank passes the same handle table, ordered by rank,
its own handle included at its own index, and no rank frees its window before
every rank has finished its last step (the barrier)."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")


class FakeLib:
    """The C entry points EpMoeLayer calls, recording what they receive."""

    def __init__(self, rank):
        self.rank = rank
        self.calls = []

    def wh_moe_plan_create(self, ctx, desc, out):
        self.calls.append(("plan_create",))
        out._obj.value = 0x1000  # a non-null handle
        return 0

    def wh_ep_row_bytes(self, hidden):
        return hidden + hidden // 32

    def wh_ep_window_create(self, ctx, plan, world, rank, max_tokens, out, handle):
        self.calls.append(("window_create", world, rank, max_tokens))
        out._obj.value = 0x2000
        for i in range(64):
            handle[i] = (17 * rank + i) & 0xFF
        return 0

    def wh_ep_window_connect(self, win, handles):
        self.calls.append(("window_connect", bytes(handles)))
        return 0

    def wh_ep_window_destroy(self, win):
        self.calls.append(("window_destroy",))

    def wh_moe_plan_destroy(self, plan):
        self.calls.append(("plan_destroy",))


class FakeMatvec:
    def __init__(self, rows, cols):
        self.rows, self.cols = rows, cols


class FakeExpert:
    def __init__(self, hidden, inter):
        self.w1 = FakeMatvec(inter, hidden)

    def spec(self):
        import wohper_b200 as W

        return W.Fp4ExpertSpec()


class FakeCtx:
    handle = None
    device = 0


def _worker(rank, world, port, results):
    import torch.distributed as dist

    import wohper_b200 as W
    import wohper_b200.ep as ep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = FakeLib(rank)
    ep.lib = lambda: fake  # the module's bound name; no library is loaded
    orig_sync = torch.cuda.synchronize
    torch.cuda.synchronize = lambda *a, **k: None
    try:
        layer = ep.EpMoeLayer(FakeCtx(), [FakeExpert(64, 32) for _ in range(4)], None, world,
                              transport="p2p", max_tokens=8)
        layer.close()
        results[rank] = fake.calls
    finally:
        torch.cuda.synchronize = orig_sync
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_p2p_window_handle_exchange_over_gloo(world):
    import torch.multiprocessing as mp

    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), results), nprocs=world, join=True)
    want = b"".join(bytes((17 * r + i) & 0xFF for i in range(64)) for r in range(world))
    for r in range(world):
        calls = results[r]
        names = [c[0] for c in calls]
        assert names == ["plan_create", "window_create", "window_connect", "window_destroy",
                         "plan_destroy"], names
        assert calls[1] == ("window_create", world, r, 8)
        assert calls[2][1] == want  # same table on every rank, rank order
