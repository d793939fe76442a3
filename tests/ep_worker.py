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
        single = None
        if shape == "v4" and step == 0:
            # the routes of a single-GPU layer's own router, so that the same
            # tokens also run through wh_moe_ffn (all experts on rank 0)
            single = _single_gpu_layer(W, H, ctx, stack, E, Hd, I, T, x, ids, w, rank)
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
            if single is not None:
                _check_single(W, single, stack, x, ids, w, got["p2p"], E, world)
    if ref is not None:
        ref.close()
    dist.barrier()
    for l in layers.values():
        l.close()
    ctx.close()
    dist.destroy_process_group()


def _single_gpu_layer(W, H, ctx, stack, E, Hd, I, T, x, ids, w, rank):
    """Rank 0 routes x with a single-GPU MoeLayer (wh_moe_ffn, all experts,
    the tensor-core path at this token count); every rank then takes those
    routes (ids and w are overwritten in place).  Returns (layer, y) on rank 0."""
    out = None
    if rank == 0:
        gate = H.router_gate(97, E, Hd)

        def wexp(e):
            w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
            return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, I, Hd, Hd // 32),
                                         W.Fp4Matvec(w3, s3, I, Hd, Hd // 32),
                                         W.Fp4Matvec(w2, s2, Hd, I, I // 32))

        layer = W.MoeLayer(ctx, [wexp(e) for e in range(E)], wexp(E),
                           torch.from_numpy(gate.view(np.int16)).cuda(), topk=6, max_tokens=T)
        y = layer.forward(x, ids=ids, weights=w)
        ctx.sync()
        out = (layer, y)
    dist.broadcast(ids, 0)
    dist.broadcast(w, 0)
    return out


def _check_single(W, single, stack, x, ids, w, y_ep, E, world, n=64):
    """The expert-parallel output against the single-GPU layer on the same
    routes, and that layer against the oracle through the tensor-core gate of
    tests/grouped_check.py (exact products; the act-quant grid flips of the
    hidden accounted for exactly; the rest within 2e-6 of sum|w x|) on a
    seeded sample of tokens."""
    from tests.grouped_check import check_grouped

    layer, y1 = single
    scale = float(y1.abs().max())
    diff = float((y_ep - y1).abs().max())
    print(f"ep world={world} v4 shape: max |diff| vs the single-GPU layer (wh_moe_ffn) = "
          f"{diff:.3e} of max {scale:.3e}", flush=True)
    assert diff <= 1e-5 * scale, diff
    sample = np.sort(np.random.default_rng(7).choice(x.shape[0], n, replace=False))
    m = check_grouped(torch, W, layer, stack, x.cpu().numpy(), y1.cpu().numpy(),
                      ids.cpu().numpy(), w.cpu().numpy(), E, sample=sample)
    print(f"ep world={world} v4 shape: {n} tokens through the grouped gate: {m}", flush=True)
    layer.close()


if __name__ == "__main__":
    main()
