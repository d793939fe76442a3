"""Expert-parallel MoE check on `world` GPUs (one process per GPU).

Every rank builds the same seeded layer (all experts, so rank 0 can compute the
single-rank result), keeps its contiguous shard in two expert-parallel layers
(peer-memory and NCCL transports), runs its share of the tokens through both
and gathers the outputs on rank 0, which compares them with a world-1 layer
over all tokens (same routes).  Three steps: two even splits (the second
reuses the windows) and one with every token on rank 0 (the other ranks send
nothing).  Launched by tests/test_gpu_ep.py with torch.distributed.run.

argv[1] = "small" (default: 16 experts, 1024 -> 512, 96 tokens) or "v4"
(256 experts, 4096 -> 2048 -> 4096, 8192 tokens, uniform
top-6 routes); with "v4" rank 0 also checks a sample of tokens against the
CPU oracle (the reference's batched path)."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    import wohper_b200 as W
    from tests import helpers as H
    from wohper_b200.ep import EpMoeLayer

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    shape = sys.argv[1] if len(sys.argv) > 1 else "small"
    E, Hd, I, T = (256, 4096, 2048, 8192) if shape == "v4" else (16, 1024, 512, 96)
    ctx = W.Context(rank)
    stack = H.torch_fp4_experts(91, E + 1, Hd, I, device=f"cuda:{rank}")

    def wexp(e):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, I, Hd, Hd // 32),
                                     W.Fp4Matvec(w3, s3, I, Hd, Hd // 32),
                                     W.Fp4Matvec(w2, s2, Hd, I, I // 32))

    El = E // world
    mine = [wexp(e) for e in range(rank * El, (rank + 1) * El)]
    layers = {t: EpMoeLayer(ctx, mine, wexp(E), world, transport=t, max_tokens=T)
              for t in ("nccl", "p2p")}
    solo = dist.new_group([0])  # collective: every rank creates it
    ref = (EpMoeLayer(ctx, [wexp(e) for e in range(E)], wexp(E), 1, group=solo,
                      transport="nccl") if rank == 0 else None)
    # steps: even split, a second input (window reuse), everything on rank 0
    for step, (seed, split) in enumerate([(92, "even"), (94, "even"), (96, "rank0")]):
        x = torch.from_numpy(H.activations(seed, T, Hd)).cuda()
        g = np.random.default_rng(seed + 1)
        ids = torch.from_numpy(np.array([g.choice(E, 6, replace=False) for _ in range(T)],
                                        np.int32)).cuda()
        w = torch.from_numpy(g.uniform(0.1, 1.0, (T, 6)).astype(np.float32)).cuda()
        bounds = ([r * T // world for r in range(world + 1)] if split == "even"
                  else [0] + [T] * world)
        lo, hi = bounds[rank], bounds[rank + 1]
        outs = {t: l.forward(x[lo:hi].contiguous(), ids[lo:hi].contiguous(),
                             w[lo:hi].contiguous()) for t, l in layers.items()}
        ctx.sync()
        same = bool(torch.equal(outs["p2p"], outs["nccl"]))
        flags = [None] * world
        dist.all_gather_object(flags, same)
        got = {}
        for t in ("p2p", "nccl"):
            parts = [torch.empty(bounds[r + 1] - bounds[r], Hd, device=x.device)
                     for r in range(world)]
            dist.all_gather(parts, outs[t])
            got[t] = torch.cat(parts)
        if rank == 0:
            want = ref.forward(x, ids, w)
            ctx.sync()
            scale = float(want.abs().max())
            for t in ("p2p", "nccl"):
                diff = float((got[t] - want).abs().max())
                print(f"ep world={world} step {step} ({split}) {t}: max |diff| vs world 1 = "
                      f"{diff:.3e} of max {scale:.3e}; p2p == nccl bitwise on every rank: "
                      f"{all(flags)}", flush=True)
                assert diff <= 1e-6 * scale, (t, diff)
            if shape == "v4" and step == 0:
                _oracle_sample(stack, x, ids, w, got["p2p"], E, Hd, I, world)
    if ref is not None:
        ref.close()
    dist.barrier()
    for l in layers.values():
        l.close()
    ctx.close()
    dist.destroy_process_group()


def _oracle_sample(stack, x, ids, w, y, E, Hd, I, world, n=16):
    """A seeded sample of tokens against the oracle's batched path: the layer's
    tensor-core tolerance (exact products, tensor-core accumulation, rare
    act-quant grid flips of the hidden; tests/grouped_check.py holds the tight
    per-flip gate of the same kernels)."""
    import oracle as O

    sample = np.sort(np.random.default_rng(7).choice(x.shape[0], n, replace=False))
    ids_np, w_np = ids.cpu().numpy()[sample], w.cpu().numpy()[sample]
    keep = []
    arr = (O.Fp4Expert * (E + 1))()
    for e in set(ids_np.reshape(-1).tolist()) | {E}:
        w1, s1, w3, s3, w2, s2 = [t.cpu().numpy() for t in H_views(stack, e)]
        arr[e] = O.Fp4Expert(O.fp4_spec(w1, s1, I, Hd, Hd // 32, keep),
                             O.fp4_spec(w3, s3, I, Hd, Hd // 32, keep),
                             O.fp4_spec(w2, s2, Hd, I, I // 32, keep))
    st, want = O.moe_batched(arr, E, np.ascontiguousarray(ids_np), np.ascontiguousarray(w_np),
                             arr[E], np.ascontiguousarray(x.cpu().numpy()[sample]))
    assert st == O.OK
    got = y.cpu().numpy()[sample]
    err = float(np.abs(got - want).max() / np.abs(want).max())
    rms = float(np.sqrt(((got - want) ** 2).mean() / (want ** 2).mean()))
    print(f"ep world={world} v4 shape: {n} tokens vs the CPU oracle: max |diff| / max|ref| = "
          f"{err:.2e}, rms ratio {rms:.2e}", flush=True)
    assert err <= 2e-3 and rms <= 1e-4, (err, rms)


def H_views(stack, e):
    from tests import helpers as H

    return H.expert_views(stack, e)


if __name__ == "__main__":
    main()
