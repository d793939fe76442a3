"""Expert-parallel MoE check on `world` GPUs (one process per GPU, NCCL).

Every rank builds the same seeded layer (all experts, so rank 0 can compute the
single-GPU result), keeps its contiguous shard for the expert-parallel layer,
runs its share of the tokens through EpMoeLayer and gathers the outputs on
rank 0, which compares them with the single-GPU MoeLayer on all tokens (same
routes).  Launched by tests/test_gpu_ep.py with torch.distributed.run."""
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
    ep = EpMoeLayer(ctx, [wexp(e) for e in range(rank * El, (rank + 1) * El)], wexp(E), world)
    x = torch.from_numpy(H.activations(92, T, Hd)).cuda()
    g = np.random.default_rng(93)
    ids = torch.from_numpy(np.array([g.choice(E, 6, replace=False) for _ in range(T)],
                                    np.int32)).cuda()
    w = torch.from_numpy(g.uniform(0.1, 1.0, (T, 6)).astype(np.float32)).cuda()
    lo, hi = rank * T // world, (rank + 1) * T // world
    y = ep.forward(x[lo:hi].contiguous(), ids[lo:hi].contiguous(), w[lo:hi].contiguous())
    ctx.sync()
    parts = [torch.empty((r + 1) * T // world - r * T // world, Hd, device=y.device)
             for r in range(world)]
    dist.all_gather(parts, y)
    solo = dist.new_group([0])  # collective: every rank creates it
    if rank == 0:
        ref = EpMoeLayer(ctx, [wexp(e) for e in range(E)], wexp(E), 1, group=solo)
        want = ref.forward(x, ids, w)
        ctx.sync()
        got = torch.cat(parts)
        diff = float((got - want).abs().max())
        scale = float(want.abs().max())
        print(f"ep world={world}: max |diff| = {diff:.3e} of max {scale:.3e}", flush=True)
        assert diff <= 1e-6 * scale, diff
        ref.close()
    dist.barrier()
    ep.close()
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
