"""Expert-parallel MoE check on `world` GPUs (one process per GPU).

Every rank builds the same seeded layer (all experts, so rank 0 can compute the
single-rank result), keeps its contiguous shard in two expert-parallel layers
(peer-memory and NCCL transports), runs its share of the tokens through both
and gathers the outputs on rank 0, which compares them with a world-1 layer
over all tokens (same routes).  Three steps: two even splits (the second
reuses the windows) and one with every token on rank 0 (the other ranks send
nothing).  Launched by tests/test_gpu_ep.py with torch.distributed.run."""
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
    E, Hd, I, T = 16, 1024, 512, 96
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
    if ref is not None:
        ref.close()
    dist.barrier()
    for l in layers.values():
        l.close()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
