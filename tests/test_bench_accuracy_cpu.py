"""CPU, multi-process (gloo): the accuracy checker bench.py runs at every number of GPUs.

bench.sharded_accuracy builds the fp32 ground truth from each rank's own vocabulary shard and merges
it over the ranks. Fed with exact results, its errors must be ~0 at world sizes 1 and 2, and with
results whose CE / d_hidden / d_weight carry a planted offset it must report that offset: the gate
numbers that the bench lines carry at N > 1 are then trustworthy.
"""

import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_math as rm


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    B, H, V = 40, 24, 700
    h, w, t = rm.make_inputs(B, H, V, seed=5, weight_std=0.3, ignore_frac=0.1)
    ce, ent, _, _ = rm.fp32_reference(h, w, t)
    _, _, dh, dw = rm.fp32_reference_grads(h, w, t)
    return h, w, t, ce, ent, dh, dw


def _check(rank, world, offset):
    import bench
    from fast_reduction.vocab_parallel import shard_bounds

    h, w, t, ce, ent, dh, dw = _case()
    V = w.shape[0]
    a, b = shard_bounds(V, world, rank)
    acc, _ = bench.sharded_accuracy(ce + offset, ent, h, w[a:b], t, a, world, grads=(dh + offset, dw[a:b] + offset),
                                    dh_rows=16, dw_rows=24)
    return acc


def _worker(rank, world, port, q):
    try:
        import datetime

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        q.put((rank, _check(rank, world, 0.0), _check(rank, world, 1e-3)))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _assert_exact_and_offset(acc0, acc1):
    for k in ("ce_mae", "ent_mae", "dh_mae", "dw_mae"):
        assert acc0[k] < 1e-5, (k, acc0[k])
    assert acc1["ce_mae"] == pytest.approx(1e-3, rel=0.02)
    assert acc1["dh_mae"] == pytest.approx(1e-3, rel=0.02)
    assert acc1["dw_mae"] == pytest.approx(1e-3, rel=0.02)
    assert acc1["ent_mae"] < 1e-5


def test_single_process_checker():
    acc0 = _check(0, 1, 0.0)
    acc1 = _check(0, 1, 1e-3)
    assert acc0["rows_checked"] == 40 and acc0["dh_rows_checked"] == 16
    _assert_exact_and_offset(acc0, acc1)


def test_two_rank_checker_matches_the_whole_vocabulary():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(60)
    for item in out:
        assert item[1] != "error", item[2]
        _assert_exact_and_offset(item[1], item[2])
