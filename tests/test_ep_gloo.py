"""Expert-parallel exchange logic (wohper_b200.ep.ep_step) on CPU ranks over gloo.

The device kernels are replaced by a numpy stand-in with the same contract
(dispatch rows ordered by global expert id, received rows source-major in
(rank, local expert) segments, results returned in send order, combine in
ascending expert id with w / sum(w)); toy experts make every routed row's
result identifiable (expert e scales its input by e + 1, the shared expert by
0.5), so a misrouted, misordered or dropped row changes the output."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


class NumpyOps:
    def __init__(self, rank, world, local_experts, hidden):
        self.rank, self.world, self.El, self.hidden = rank, world, local_experts, hidden

    def empty_like(self, t):
        return torch.empty_like(t)

    def to_list(self, t):
        return [int(v) for v in t.tolist()]

    def cat(self, ts):
        return torch.cat(ts)

    def empty_rows(self, n):
        return torch.empty(n, self.hidden, dtype=torch.float32)

    def empty_results(self, n):
        return torch.empty(n, self.hidden, dtype=torch.float32)

    def dispatch(self, x, ids):
        T, K = ids.shape
        flat = ids.reshape(-1).numpy()
        order = np.argsort(flat, kind="stable")  # by global expert id
        send = torch.from_numpy(np.ascontiguousarray(x.numpy()[order // K]))
        pos = np.empty(T * K, np.int32)
        pos[order] = np.arange(T * K, dtype=np.int32)
        counts = np.bincount(flat, minlength=self.world * self.El).astype(np.int32)
        return send, torch.from_numpy(counts), torch.from_numpy(pos)

    def expert_ffn(self, recv, recv_counts, R, x):
        rc = recv_counts.numpy().reshape(self.world, self.El)
        out = np.empty((R + x.shape[0], self.hidden), np.float32)
        row = 0
        for src in range(self.world):
            for le in range(self.El):
                e = self.rank * self.El + le
                n = int(rc[src, le])
                out[row:row + n] = recv.numpy()[row:row + n] * (e + 1)
                row += n
        assert row == R
        out[R:] = 0.5 * x.numpy()
        return torch.from_numpy(out)

    def combine(self, ids, weights, pos, y_back, y_shared):
        ids, w, pos = ids.numpy(), weights.numpy(), pos.numpy().reshape(ids.shape)
        yb, ys = y_back.numpy(), y_shared.numpy()
        y = np.empty_like(ys)
        for t in range(ids.shape[0]):
            s = np.float32(w[t].sum())
            acc = np.zeros(self.hidden, np.float32)
            for k in np.argsort(ids[t], kind="stable"):
                acc = acc + yb[pos[t, k]] * np.float32(w[t, k] / s)
            y[t] = ys[t] + acc
        return torch.from_numpy(y)


def _worker(rank, world, port, tokens, E, hidden):
    import torch.distributed as dist

    from wohper_b200.ep import ep_step

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.random.default_rng(100 + rank)
        T, K = tokens[rank], 6
        x = g.standard_normal((T, hidden)).astype(np.float32)
        ids = np.array([g.choice(E, K, replace=False) for _ in range(T)],
                       np.int32).reshape(T, K)
        w = g.uniform(0.1, 1.0, (T, K)).astype(np.float32)
        ops = NumpyOps(rank, world, E // world, hidden)
        y = ep_step(ops, torch.from_numpy(x), torch.from_numpy(ids).reshape(T, K),
                    torch.from_numpy(w), world, E // world).numpy()
        want = 0.5 * x + np.stack([
            sum((w[t, k] / w[t].sum()) * (ids[t, k] + 1) for k in range(K)) * x[t]
            for t in range(T)]) if T else np.zeros((0, hidden), np.float32)
        np.testing.assert_allclose(y, want, rtol=1e-5, atol=1e-5)
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,tokens", [(2, (13, 5)), (4, (7, 0, 9, 3))])
def test_ep_exchange_over_gloo(world, tokens):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(world, _port(), tokens, 8 * world, 64), nprocs=world, join=True)
