"""GPU, multi-process (NCCL): the vocabulary-sharded forward and training at the full BASELINE.json
shapes that are defined as multi-GPU runs, against the single-GPU engine on the same inputs (which
tests/test_configs_gpu.py checks against fp32 ground truth at these sizes):

* hidden [8, 2048, 4096] (B = 16384), V = 256000, weight N(0, 0.05), 5% of targets = -100
  (chosen by a seeded randperm);
* B = 65536, H = 5120, V = 152064, chunk 8192, weight N(0, 0.02), 1% of the targets of every
  shard placed in that shard's last vocabulary tile (ragged at 4 and 8 GPUs: 38016 = 148.5 x 256 and
  19008 = 74.25 x 256 columns per shard).

Every rank generates the same inputs on its own GPU from a seeded CUDA generator. Skipped when fewer
than two GPUs are visible; runs on up to 8."""

import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CONFIGS = {
    # name: (batch shape, H, V, chunk, weight std, ignore fraction, per-shard last-tile fraction)
    "configs3": ((8, 2048), 4096, 256000, 4096, 0.05, 0.05, 0.0),
    "configs4": ((65536,), 5120, 152064, 8192, 0.02, 0.0, 0.01),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(name, world, dev):
    from fast_reduction.vocab_parallel import shard_bounds

    shape, H, V, chunk, wstd, ignore, tail = CONFIGS[name]
    B = 1
    for s in shape:
        B *= s
    g = torch.Generator(device=dev).manual_seed(20240 + len(name))
    h = torch.randn(B, H, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(V, H, device=dev, generator=g) * wstd).to(torch.bfloat16)
    t = torch.randint(0, V, (B,), device=dev, generator=g)
    if tail:
        per = max(1, int(tail * B / world))
        for r in range(world):
            a, b = shard_bounds(V, world, r)
            last = a + (b - a - 1) // 256 * 256  # first column of the shard's last tile
            rows = torch.arange(r, B, world, device=dev)[:per]
            t[rows] = last + torch.randint(0, b - last, (rows.numel(),), device=dev, generator=g)
    if ignore:
        t[torch.randperm(B, device=dev, generator=g)[: int(ignore * B)]] = -100
    return h.view(*shape, H), w, t.view(*shape), chunk


def _worker(rank, world, port, q, name):
    try:
        import datetime
        import sys
        from pathlib import Path

        repo = Path(__file__).resolve().parents[1]
        for p in (str(repo / "fast-reduction_b200"), str(repo)):
            if p not in sys.path:
                sys.path.insert(0, p)
        import torch.distributed as dist

        from fast_reduction import _native as nat
        from fast_reduction.gemm_kernel import gemm_fused_ce_entropy, gemm_megakernel_fast
        from fast_reduction.vocab_parallel import shard_bounds, vocab_parallel_ce_entropy, vocab_parallel_megakernel

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        h, w, t, chunk = _inputs(name, world, dev)
        V = w.shape[0]
        a, b = shard_bounds(V, world, rank)

        out = vocab_parallel_ce_entropy(h, w[a:b], t, a, V, chunk_size=chunk)
        ref = gemm_fused_ce_entropy(h, w, t, chunk_size=chunk)
        err_fwd = max(float((x - y).abs().max()) for x, y in zip(out, ref))
        finite = all(bool(torch.isfinite(x).all()) for x in out)
        del out, ref

        h_leaf = h.clone().requires_grad_(True)
        w_leaf = w[a:b].clone().requires_grad_(True)
        loss, _, _ = vocab_parallel_megakernel(h_leaf, w_leaf, t, a, V, chunk_size=chunk)
        loss.backward()
        dh, dw = h_leaf.grad.float(), w_leaf.grad.float()
        del h_leaf, w_leaf
        torch.cuda.empty_cache()
        h1 = h.clone().requires_grad_(True)
        w1 = w.clone().requires_grad_(True)
        loss1, _, _ = gemm_megakernel_fast(h1, w1, t, chunk_size=chunk)
        loss1.backward()
        dh1, dw1 = h1.grad.float(), w1.grad[a:b].float()
        dh_rel = float((dh - dh1).norm() / dh1.norm())
        dw_rel = float((dw - dw1).norm() / dw1.norm())
        loss_rel = abs(float(loss) - float(loss1)) / abs(float(loss1))
        torch.cuda.synchronize()
        bits = nat.read_status(dev)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", err_fwd, finite, dh_rel, dw_rel, loss_rel, bits))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least two GPUs")
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_vocab_parallel_full_size_config(name):
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, name)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r in results:
        assert r[1] == "ok", r[2]
    for rank, _, err_fwd, finite, dh_rel, dw_rel, loss_rel, bits in results:
        assert finite, rank
        # the shard merge regroups the same per-tile partials: fp32 rounding of the merge only
        assert err_fwd < 5e-5, (rank, err_fwd)
        # d_hidden: per-shard fp32 products summed by NCCL, then one cast to bf16; d_weight: identical
        # GEMM per shard, but its dlogits come from the merged statistics
        assert dh_rel < 5e-3, (rank, dh_rel)
        assert dw_rel < 5e-3, (rank, dw_rel)
        assert loss_rel < 1e-5, (rank, loss_rel)
        assert bits == 0, (rank, bits)
