"""GPU: the forward and the training step are CUDA-graph capturable (no host synchronisation, no
allocation outside the graph pool, launches on the capturing stream and forked side streams), and a
replay equals eager execution bit for bit, also after new data is copied into the static inputs."""

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

    B, H, V, chunk = 640, 256, 3001, 256
    h, w, t = _static_inputs(B, H, V, seed=41)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            gemm_fused_ce_entropy(h, w, t, chunk_size=chunk)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = gemm_fused_ce_entropy(h, w, t, chunk_size=chunk)
    for seed in (41, 42):
        h2, w2, t2 = _static_inputs(B, H, V, seed=seed)
        h.copy_(h2)
        w.copy_(w2)
        t.copy_(t2)
        graph.replay()
        ref = gemm_fused_ce_entropy(h2, w2, t2, chunk_size=chunk)
        torch.cuda.synchronize()
        for a, b in zip(outs, ref):
            assert torch.equal(a, b)


def test_training_step_graph_replay_equals_eager():
    from fast_reduction.gemm_kernel import gemm_megakernel_fast

    B, H, V, chunk = 512, 128, 1500, 128
    h, w, t = _static_inputs(B, H, V, seed=43)
    h_leaf = h.clone().requires_grad_(True)
    w_leaf = w.clone().requires_grad_(True)

    def step():
        h_leaf.grad = None
        w_leaf.grad = None
        loss, _, _ = gemm_megakernel_fast(h_leaf, w_leaf, t, chunk_size=chunk)
        loss.backward()
        return loss

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    h_leaf.grad = None
    w_leaf.grad = None
    with torch.cuda.graph(graph):
        loss_g = step()
    h2, w2, t2 = _static_inputs(B, H, V, seed=44)
    with torch.no_grad():
        h_leaf.copy_(h2)
        w_leaf.copy_(w2)
    t.copy_(t2)
    graph.replay()
    torch.cuda.synchronize()
    got = (loss_g.detach().clone(), h_leaf.grad.clone(), w_leaf.grad.clone())
    he = h2.clone().requires_grad_(True)
    we = w2.clone().requires_grad_(True)
    loss_e, _, _ = gemm_megakernel_fast(he, we, t2, chunk_size=chunk)
    loss_e.backward()
    torch.cuda.synchronize()
    assert torch.equal(got[0], loss_e.detach())
    assert torch.equal(got[1], he.grad)
    assert torch.equal(got[2], we.grad)
