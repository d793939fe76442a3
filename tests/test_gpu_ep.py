"""Expert parallelism on the GPU: the expert-parallel layer at world size 1
(both transports, several steps through the same window) reproduces the
single-GPU batched layer given the same routes, and (when two or more GPUs are
visible) 2-rank runs of both transports reproduce it too (tests/ep_worker.py)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from tests import helpers as H

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_world1_matches_batched_layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch.distributed as dist

    import wohper_b200 as W
    from wohper_b200.ep import EpMoeLayer

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_port())
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        E, Hd, I, T = 16, 1024, 512, 64
        ctx = W.Context(0)
        stack = H.torch_fp4_experts(95, E + 1, Hd, I)
        gate = H.router_gate(96, E, Hd)

        def wexp(e):
            w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
            return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, I, Hd, Hd // 32),
                                         W.Fp4Matvec(w3, s3, I, Hd, Hd // 32),
                                         W.Fp4Matvec(w2, s2, Hd, I, I // 32))

        experts = [wexp(e) for e in range(E)]
        layer = W.MoeLayer(ctx, experts, wexp(E), torch.from_numpy(gate.view(np.int16)).cuda(),
                           topk=6, max_tokens=T)
        x = torch.from_numpy(H.activations(97, T, Hd)).cuda()
        ids = torch.zeros(T, 6, dtype=torch.int32, device="cuda")
        w = torch.zeros(T, 6, device="cuda")
        want = layer.forward(x, ids=ids, weights=w)
        for transport in ("nccl", "p2p"):
            ep = EpMoeLayer(ctx, experts, wexp(E), 1, transport=transport, max_tokens=T)
            for step in range(3):  # the peer transport reuses its window (epochs)
                n = (T, T // 2, 0)[step]
                got = ep.forward(x[:n].contiguous(), ids[:n].contiguous(), w[:n].contiguous())
                ctx.sync()
                diff = float((got - want[:n]).abs().max()) if n else 0.0
                assert diff <= 1e-6 * float(want.abs().max()), (transport, step, diff)
            ep.close()
        layer.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_ep_two_ranks():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1",
                        f"--master-port={_port()}", str(ROOT / "tests" / "ep_worker.py")],
                       env=env, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert "ep world=2" in r.stdout


def test_ep_all_gpus_config4_shape():
    """BASELINE config 4 at its own shape on every visible GPU (4 or 8): 256
    experts sharded contiguously, 8192 tokens; both transports equal the
    world-1 layer and each other, and a token sample matches the CPU oracle."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 4:
        pytest.skip("needs 4 or more GPUs")
    n = 8 if torch.cuda.device_count() >= 8 else 4
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        f"--nproc-per-node={n}", "--master-addr=127.0.0.1",
                        f"--master-port={_port()}", str(ROOT / "tests" / "ep_worker.py"), "v4"],
                       env=env, cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert f"ep world={n} v4 shape" in r.stdout
    print(r.stdout[-2500:])
