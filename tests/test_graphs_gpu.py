"""GPU: the forward and the training step are CUDA-graph capturable (fast_reduction.graphs: no host
synchronisation, no allocation outside the graph pool, launches on the capturing stream and forked
side streams), and a replay equals eager execution bit for bit, also after new data is copied into
the static inputs."""

import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _static_inputs(B, H, V, seed):
    h, w, t = rm.make_inputs(B, H, V, seed=seed, weight_std=0.2, ignore_frac=0.03)
    return h.to(DEV), w.to(DEV), t.to(DEV)


def test_forward_graph_replay_equals_eager():
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy
    from fast_reduction.graphs import graphed_forward

    B, H, V, chunk = 640, 256, 3001, 256
    h, w, t = _static_inputs(B, H, V, seed=41)
    run = graphed_forward(h, w, t, chunk_size=chunk)
    for seed in (41, 42):
        h2, w2, t2 = _static_inputs(B, H, V, seed=seed)
        h.copy_(h2)
        w.copy_(w2)
        t.copy_(t2)
        outs = run()
        ref = gemm_fused_ce_entropy(h2, w2, t2, chunk_size=chunk)
        torch.cuda.synchronize()
        for a, b in zip(outs, ref):
            assert torch.equal(a, b)


@pytest.mark.parametrize("with_bias", [False, True])
def test_training_step_graph_replay_equals_eager(with_bias):
    from fast_reduction.gemm_kernel import gemm_megakernel_fast
    from fast_reduction.graphs import graphed_training_step

    B, H, V, chunk = 512, 128, 1500, 128
    h, w, t = _static_inputs(B, H, V, seed=43)
    h_leaf = h.clone().requires_grad_(True)
    w_leaf = w.clone().requires_grad_(True)
    b_leaf = (torch.randn(V, device=DEV) * 0.5).to(torch.bfloat16).requires_grad_(True) if with_bias else None
    run = graphed_training_step(h_leaf, w_leaf, t, bias=b_leaf, chunk_size=chunk)
    h2, w2, t2 = _static_inputs(B, H, V, seed=44)
    with torch.no_grad():
        h_leaf.copy_(h2)
        w_leaf.copy_(w2)
    t.copy_(t2)
    loss_g, ce_g, _ = run()
    torch.cuda.synchronize()
    he = h2.clone().requires_grad_(True)
    we = w2.clone().requires_grad_(True)
    be = None if b_leaf is None else b_leaf.detach().clone().requires_grad_(True)
    loss_e, ce_e, _ = gemm_megakernel_fast(he, we, t2, bias=be, chunk_size=chunk)
    loss_e.backward()
    torch.cuda.synchronize()
    assert torch.equal(loss_g, loss_e.detach()) and torch.equal(ce_g, ce_e)
    assert torch.equal(h_leaf.grad, he.grad)
    assert torch.equal(w_leaf.grad, we.grad)
    if with_bias:
        assert torch.equal(b_leaf.grad, be.grad)
