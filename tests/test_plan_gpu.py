"""GPU: execution plans (MatcorePlan semantics, include/matcore/plan.h:37-107).

A plan freezes the operator and its tensors' metadata; execute rejects other
shapes; graph plans capture the launches once and replay them, rejecting data
pointer changes as the reference does (src/jit_runner.cpp:1060-1111).
"""
import numpy as np
import pytest

from tests import gpu_util as gu

pytestmark = pytest.mark.gpu


def _gemm_inputs(m=256, k=512, n=384, seed=1):
    import torch
    rng = np.random.default_rng(seed)
    x = gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((m, k), dtype=np.float32))[0])
    w = gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((k, n), dtype=np.float32) / 20)[0])
    b = gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal(n, dtype=np.float32) / 50)[0])
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    return x, w, b, y


@pytest.mark.parametrize("graph", [False, True])
def test_gemm_plan_matches_direct_call(mcb, graph):
    import torch
    x, w, b, y = _gemm_inputs()
    ref = mcb.gemm_epilogue(x, w, b, act="gelu_tanh", out_dtype="bf16")
    plan = mcb.Plan("gemm_epilogue", y, x, w, b, graph=graph, bias_mode="row", act="gelu_tanh")
    for _ in range(3):
        y.zero_()
        plan.execute(y, x, w, b)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    assert plan.generation > 0
    plan.close()


def test_graph_plan_rejects_pointer_change_and_shape_change(mcb):
    import torch
    x, w, b, y = _gemm_inputs()
    plan = mcb.Plan("gemm_epilogue", y, x, w, b, graph=True, bias_mode="row", act="gelu_tanh")
    plan.execute(y, x, w, b)
    x2 = x.clone()
    with pytest.raises(mcb.McbError) as e:
        plan.execute(y, x2, w, b)
    assert e.value.name == "INVALID_ARGUMENT"
    xs, ws, bs, ys = _gemm_inputs(m=128)
    with pytest.raises(mcb.McbError) as e:
        plan.execute(ys, xs, ws, bs)
    assert e.value.name == "SHAPE_MISMATCH"
    # a non-graph plan follows new buffers of the same shape
    p2 = mcb.Plan("gemm_epilogue", y, x, w, b, bias_mode="row", act="gelu_tanh")
    p2.execute(y, x2, w, b)
    torch.cuda.synchronize()
    assert p2.generation > plan.generation


def test_graph_plans_for_msm_chain_and_region(mcb, orc):
    import torch
    rng = np.random.default_rng(2)
    q, k, v = (gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((1, 2, 256, 128),
                                                               dtype=np.float32))[0])
               for _ in range(3))
    o = torch.empty_like(q)
    ref = mcb.msm(q, k, v, 128 ** -0.5)
    p = mcb.Plan("msm", o, q, k, v, graph=True, scale=128 ** -0.5)
    p.execute(o, q, k, v)
    p.execute(o, q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(o, ref)

    x, w, _, _ = _gemm_inputs(m=256, k=256, n=256)
    w2 = w.clone()
    e = torch.empty(256, 256, dtype=torch.float32, device="cuda")
    ref = mcb.gemm_chain(x, w, w2, act="relu", out_dtype="f32")
    pc = mcb.Plan("gemm_chain", e, x, w, None, w2, graph=True, act="relu")
    pc.execute(e, x, w, None, w2)
    torch.cuda.synchronize()
    assert torch.equal(e, ref)

    xb = gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((1, 256, 512), dtype=np.float32))[0])
    wts = [gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((512, 512), dtype=np.float32)
                                        / np.float32(22.6))[0]) for _ in range(4)]
    yb = torch.empty_like(xb)
    ref = mcb.attn_block(xb, *wts, 4, 1e-6)
    pr = mcb.Plan("attn_block", yb, xb, *wts, graph=True, heads=4, eps=1e-6)
    pr.execute(yb, xb, *wts)
    torch.cuda.synchronize()
    assert torch.equal(yb, ref)
    assert mcb.device_status(0) == 0


@pytest.mark.parametrize("graph", [False, True])
def test_epilogue_chain_plan(mcb, orc, graph):
    """A Family A chain with two boundaries (MatcorePlan freezes any accepted
    Family A graph, src/jit_runner.cpp:881-1125): the plan replays the direct
    call bit for bit; a graph plan rejects a moved boundary and a new shape."""
    import torch
    m, k, n = 256, 512, 384
    x, w, _, _ = _gemm_inputs(m, k, n, seed=5)
    rng = np.random.default_rng(6)
    b0 = torch.from_numpy(rng.standard_normal((m, n), dtype=np.float32)).cuda()
    b1 = gu.to_dev_bf16(gu.bf16_pair(rng.standard_normal((m, n), dtype=np.float32))[0])
    chain = [("add", b0), "gelu_tanh", ("mul", b1, "right"), "tanh"]
    ref = mcb.gemm_epilogue(x, w, chain=chain, out_dtype="f32")
    y = torch.empty(m, n, dtype=torch.float32, device="cuda")
    plan = mcb.Plan("gemm_epilogue_chain", y, x, w, graph=graph, chain=chain)
    for _ in range(3):
        y.fill_(float("nan"))
        plan.execute(y, x, w, b0, b1)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    # and the result is the chain itself (fp64 oracle of the same ops)
    xf = x.float().cpu().numpy()
    wf = w.float().cpu().numpy()
    acc = xf.astype(np.float64) @ wf.astype(np.float64) + b0.cpu().numpy()
    acc = 0.5 * acc * (1 + np.tanh(0.7978845608 * (acc + 0.044715 * acc ** 3)))
    expect = np.tanh(b1.float().cpu().numpy() * acc)
    assert orc.rel_frobenius(gu.from_dev(y), expect) < 1e-5
    if graph:
        with pytest.raises(mcb.McbError) as e:
            plan.execute(y, x, w, b0.clone(), b1)
        assert e.value.name == "INVALID_ARGUMENT"
    with pytest.raises(mcb.McbError) as e:
        plan.execute(y[:128], x[:128], w, b0[:128], b1[:128])
    assert e.value.name == "SHAPE_MISMATCH"
    plan.close()
