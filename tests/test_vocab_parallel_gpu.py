"""GPU, multi-process (NCCL): vocabulary-parallel forward and training over 2+ GPUs agree with the
single-GPU engine on the same inputs. Skipped when fewer than two GPUs are visible."""

import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, nvls, dtype_name="bfloat16", dh_collective="rs_ag"):
    try:
        import datetime
        import os
        import sys
        from pathlib import Path

        os.environ["FRX_NVLS"] = "1" if nvls else "0"  # read when fast_reduction.vocab_parallel is imported
        os.environ["FRX_DH_COLLECTIVE"] = dh_collective
        repo = Path(__file__).resolve().parents[1]
        for p in (str(repo / "fast-reduction_b200"), str(repo)):
            if p not in sys.path:
                sys.path.insert(0, p)
        import torch.distributed as dist

        from fast_reduction import _native as nat
        from fast_reduction.gemm_kernel import gemm_fused_ce_entropy, gemm_megakernel_fast
        from fast_reduction.vocab_parallel import shard_bounds, vocab_parallel_ce_entropy, vocab_parallel_megakernel
        from oracle import reference_math as rm

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        B, H, V, chunk = 520, 256, 3001, 200
        dtype = getattr(torch, dtype_name)
        h, w, t = rm.make_inputs(B, H, V, seed=5, weight_std=0.1, ignore_frac=0.05, tail_frac=0.02)
        h, w = h.to(dtype), w.to(dtype)
        bias = (torch.randn(V, generator=torch.Generator().manual_seed(9)) * 0.5).to(dtype)
        a, b = shard_bounds(V, world, rank)
        hd, td = h.to(dev), t.to(dev)
        ce, ent, lp = vocab_parallel_ce_entropy(hd, w[a:b].to(dev), td, a, V, chunk_size=chunk,
                                                bias_shard=bias[a:b].to(dev))
        ce1, ent1, lp1 = gemm_fused_ce_entropy(hd, w.to(dev), td, bias=bias.to(dev), chunk_size=chunk)
        err_fwd = max(float((ce - ce1).abs().max()), float((ent - ent1).abs().max()), float((lp - lp1).abs().max()))
        # host inputs: each rank uploads a share of the hidden rows, all-gathers them, streams its weight slice
        host = vocab_parallel_ce_entropy(h.pin_memory(), w[a:b].pin_memory(), t.pin_memory(), a, V,
                                         chunk_size=chunk, bias_shard=bias[a:b].pin_memory())
        if not all(x.device.type == "cpu" and torch.equal(x, y.cpu()) for x, y in zip(host, (ce, ent, lp))):
            err_fwd = float("inf")

        h_leaf = h.to(dev).requires_grad_(True)
        w_leaf = w[a:b].to(dev).requires_grad_(True)
        b_leaf = bias[a:b].to(dev).requires_grad_(True)
        loss, ce2, ent2 = vocab_parallel_megakernel(h_leaf, w_leaf, td, a, V, chunk_size=chunk, bias_shard=b_leaf)
        loss.backward()
        h1 = h.to(dev).requires_grad_(True)
        w1 = w.to(dev).requires_grad_(True)
        b1 = bias.to(dev).requires_grad_(True)
        loss1, _, _ = gemm_megakernel_fast(h1, w1, td, bias=b1, chunk_size=chunk)
        loss1.backward()
        dh_rel = float((h_leaf.grad.float() - h1.grad.float()).norm() / h1.grad.float().norm())
        dw_rel = float((w_leaf.grad.float() - w1.grad[a:b].float()).norm() / w1.grad[a:b].float().norm())
        db_rel = float((b_leaf.grad.float() - b1.grad[a:b].float()).norm() / b1.grad[a:b].float().norm())
        dw_rel = max(dw_rel, db_rel)
        loss_err = abs(float(loss) - float(loss1))
        torch.cuda.synchronize()
        bits = nat.read_status(dev)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", err_fwd, dh_rel, dw_rel, loss_err, float(loss1), bits))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least two GPUs")
@pytest.mark.parametrize("nvls,dtype_name,dh_collective", [
    (True, "bfloat16", "rs_ag"), (False, "bfloat16", "rs_ag"), (False, "bfloat16", "allreduce"),
    (False, "float16", "rs_ag"), (False, "float32", "rs_ag")],
    ids=["nvls-fused-dhidden", "nccl-rs-ag", "nccl-allreduce", "nccl-fp16", "nccl-fp32"])
def test_vocab_parallel_matches_single_gpu(nvls, dtype_name, dh_collective):
    """The d_hidden reductions: NCCL reduce-scatter + cast + all-gather (default), one NCCL fp32
    all-reduce (FRX_DH_COLLECTIVE=allreduce), and the reduction fused into the GEMM through NVLS
    multicast (FRX_NVLS=1; when the GPUs lack NVLS this case runs the default path); fp16 and fp32
    operands on the default path. B = 520 rows do not split evenly over 4 ranks' shares."""
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, nvls, dtype_name, dh_collective))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in results:
        assert r[1] == "ok", r[2]
    for rank, _, err_fwd, dh_rel, dw_rel, loss_err, loss1, bits in results:
        assert err_fwd < 2e-5, (rank, err_fwd)
        assert dh_rel < 5e-3, (rank, dh_rel)
        assert dw_rel < 5e-3, (rank, dw_rel)
        assert loss_err <= 1e-4 * abs(loss1) + 1e-2, (rank, loss_err)
        assert bits == 0, (rank, bits)
