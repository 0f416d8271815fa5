"""CPU, multi-process (gloo): the vocabulary-parallel exchange protocol of
fast_reduction.vocab_parallel, run with the oracle's arithmetic in place of the CUDA kernels.

Each rank reduces its vocabulary slice to per-row (M, S, U, ZT), the ranks all-gather the
[B, 4] rows, and every rank merges them; the result must equal the unsharded computation.
Also checks the slice bounds, the d_hidden all-reduce, and that a failing rank surfaces as an
error on the other ranks instead of a hang.
"""

import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_math as rm


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _protocol_worker(rank, world, port, q):
    try:
        from fast_reduction.vocab_parallel import shard_bounds

        _init(rank, world, port)
        B, H, V = 48, 32, 1000
        h, w, t = rm.make_inputs(B, H, V, seed=3, weight_std=0.3, ignore_frac=0.1)
        z = (h.double() @ w.double().T).numpy()
        a, b = shard_bounds(V, world, rank)
        local = rm.finalize_partials(rm.tile_partials(z[:, a:b], t.numpy(), vocab_offset=a))[4]
        local_t = torch.from_numpy(local.astype(np.float64))
        gathered = torch.empty((world * local_t.shape[0],) + tuple(local_t.shape[1:]), dtype=local_t.dtype)
        dist.all_gather_into_tensor(gathered, local_t)
        gathered = gathered.view((world,) + tuple(local_t.shape))
        ce, ent, lse, lp, _ = rm.finalize_partials(gathered.numpy(), target=t.numpy(), vocab_size=V)
        # backward: each rank's d_hidden contribution from its slice, summed by all-reduce
        dz = rm.dlogits(z[:, a:b], t.numpy(), lse, ent, 1.0, -1.0, vocab_offset=a)
        dh = torch.from_numpy(dz @ w.double().numpy()[a:b])
        dist.all_reduce(dh)
        dw_slice = dz.T @ h.double().numpy()
        q.put((rank, ce, ent, lse, dh.numpy(), (a, b), dw_slice))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_parallel_protocol_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_protocol_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in results:
        assert not (isinstance(r[1], str) and r[1] == "error"), r[2]
    B, H, V = 48, 32, 1000
    h, w, t = rm.make_inputs(B, H, V, seed=3, weight_std=0.3, ignore_frac=0.1)
    ce_ref, ent_ref, lp_ref, lse_ref = rm.fp32_reference(h.double(), w.double(), t)
    _, _, dh_ref, dw_ref = rm.fp32_reference_grads(h.double(), w.double(), t)
    covered = []
    for rank, ce, ent, lse, dh, (a, b), dw_slice in sorted(results, key=lambda r: r[0]):
        np.testing.assert_allclose(ce, ce_ref.numpy(), atol=1e-5)
        np.testing.assert_allclose(ent, ent_ref.numpy(), atol=1e-5)
        np.testing.assert_allclose(lse, lse_ref.numpy(), atol=1e-5)
        np.testing.assert_allclose(dh, dh_ref.numpy(), atol=1e-5)
        np.testing.assert_allclose(dw_slice, dw_ref.numpy()[a:b], atol=1e-5)
        covered.append((a, b))
    assert covered[0][0] == 0 and covered[-1][1] == V
    assert all(covered[i][1] == covered[i + 1][0] for i in range(len(covered) - 1))


def test_shard_bounds_cover_and_balance():
    from fast_reduction.vocab_parallel import shard_bounds

    for V in (1000, 128256, 152064, 256000, 7):
        for world in (1, 2, 3, 4, 8):
            bounds = [shard_bounds(V, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == V
            sizes = [b - a for a, b in bounds]
            assert max(sizes) - min(sizes) <= 1
            assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _failing_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("rank 1 fails before the exchange")
        x = torch.zeros(4)
        out = torch.empty(world * 4)
        try:
            dist.all_gather_into_tensor(out, x)
            q.put((rank, "completed"))
        except Exception as exc:  # the peer is gone: the collective must fail, not hang
            q.put((rank, "raised", type(exc).__name__))
    except Exception as exc:
        q.put((rank, "raised", type(exc).__name__))


def test_failed_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1][0] == "raised"
    assert results[0][0] == "raised", results


def test_empty_shard_is_rejected_before_any_collective():
    from fast_reduction.vocab_parallel import vocab_parallel_ce_entropy

    h = torch.randn(4, 16).to(torch.bfloat16)
    w = torch.empty(0, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="non-empty vocabulary slice"):
        vocab_parallel_ce_entropy(h, w, torch.zeros(4, dtype=torch.int64), 0, 3)
