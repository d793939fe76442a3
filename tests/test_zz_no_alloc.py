"""wh_fp4_expert_forward_noalloc: the FP4 expert forward whose scratch is a
static device array of the library (no allocation on the call path).

Checked against the existing entry point wh_fp4_expert_forward on the same
inputs, with two calls in a row on one stream before any synchronisation, and
against the CPU oracle.  The file name sorts last so that it also runs after
every other GPU test in one process; it passes alone in a fresh process too.
"""
import numpy as np
import pytest

import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import wohper_b200

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return wohper_b200


@pytest.fixture(scope="module")
def ctx(W):
    c = W.Context(0)
    yield c
    c.close()


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _w_expert(W, stack, e):
    w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
    inter, hb = w1.shape
    hidden = hb * 2
    return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, inter, hidden, hidden // 32),
                                 W.Fp4Matvec(w3, s3, inter, hidden, hidden // 32),
                                 W.Fp4Matvec(w2, s2, hidden, inter, inter // 32))


def _oracle_expert(stack, e, keep):
    w1, s1, w3, s3, w2, s2 = [t.cpu().numpy() for t in H.expert_views(stack, e)]
    inter, hb = w1.shape
    hidden = hb * 2
    return O.Fp4Expert(O.fp4_spec(w1, s1, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w3, s3, inter, hidden, hidden // 32, keep),
                       O.fp4_spec(w2, s2, hidden, inter, inter // 32, keep))


# (4096, 2048) and (1024, 512) take the TMA fast path in wh_fp4_expert_forward,
# (160, 96) its generic path; both compute in the reference's order, so the
# static-scratch entry point must agree with either bit for bit.
@pytest.mark.parametrize("hidden,inter", [(4096, 2048), (1024, 512), (160, 96)])
def test_noalloc_matches_existing_entry_point_two_calls(ctx, W, hidden, inter):
    stack = H.torch_fp4_experts(61, 2, hidden, inter)
    xs = [H.activations(62 + i, 1, hidden).reshape(-1) for i in range(2)]
    experts = [_w_expert(W, stack, e) for e in range(2)]
    # two calls in a row, different experts and inputs, one sync at the end
    got = [torch.zeros(hidden, device="cuda") for _ in range(2)]
    for e in range(2):
        W.deepseek_v4_fp4_expert_forward_noalloc(ctx, experts[e], torch.from_numpy(xs[e]).cuda(),
                                                 got[e])
    ctx.sync()
    keep = []
    for e in range(2):
        ref = torch.zeros(hidden, device="cuda")
        W.deepseek_v4_fp4_expert_forward(ctx, experts[e], torch.from_numpy(xs[e]).cuda(), ref,
                                         torch.zeros(2 * inter, device="cuda"))
        ctx.sync()
        g, r = got[e].cpu().numpy(), ref.cpu().numpy()
        assert np.all(np.isfinite(g))
        nd = int(np.sum(_bits(g) != _bits(r)))
        assert nd == 0, f"{nd} outputs differ from wh_fp4_expert_forward"
        # and the static-scratch path is the reference order itself
        st, want = O.fp4_expert_forward(_oracle_expert(stack, e, keep), xs[e])
        assert st == O.OK
        assert np.array_equal(_bits(g), _bits(want))


def test_noalloc_rejects_experts_beyond_the_static_scratch(ctx, W):
    hidden, inter = 4096, 32768  # hidden + 2 * inter = 69632 > 65536 floats
    w13 = torch.empty(inter, hidden // 2, dtype=torch.uint8, device="cuda")
    s13 = torch.empty(inter, hidden // 32, dtype=torch.uint8, device="cuda")
    w2 = torch.empty(hidden, inter // 2, dtype=torch.uint8, device="cuda")
    s2 = torch.empty(hidden, inter // 32, dtype=torch.uint8, device="cuda")
    e = W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w13, s13, inter, hidden, hidden // 32),
                              W.Fp4Matvec(w13, s13, inter, hidden, hidden // 32),
                              W.Fp4Matvec(w2, s2, hidden, inter, inter // 32))
    out = torch.zeros(hidden, device="cuda")
    with pytest.raises(W.WohperError) as err:
        W.deepseek_v4_fp4_expert_forward_noalloc(ctx, e, torch.zeros(hidden, device="cuda"), out)
    assert err.value.kind == "ScratchTooSmall"
    assert "65536" in str(err.value)
    ctx.sync()


def test_noalloc_calls_leave_device_memory_unchanged(ctx, W):
    """The promise itself: once the library is loaded on the device, calls --
    here at a larger expert than the other tests, still inside the array --
    take no device memory, from the driver or from torch's caching allocator."""
    hidden, inter = 8192, 16384  # hidden + 2 * inter = 40960 <= 65536 floats
    stack = H.torch_fp4_experts(71, 1, hidden, inter)
    e = _w_expert(W, stack, 0)
    x = torch.from_numpy(H.activations(72, 1, hidden).reshape(-1)).cuda()
    out = torch.zeros(hidden, device="cuda")
    W.deepseek_v4_fp4_expert_forward_noalloc(ctx, e, x, out)  # loads every kernel it uses
    ctx.sync()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch0 = torch.cuda.memory_allocated()
    for _ in range(4):
        W.deepseek_v4_fp4_expert_forward_noalloc(ctx, e, x, out)
    ctx.sync()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    assert torch.cuda.memory_allocated() == torch0
    assert np.all(np.isfinite(out.cpu().numpy()))
