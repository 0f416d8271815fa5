#!/usr/bin/env python
"""Benchmark of the fused linear + CE + entropy engine (one JSON line on rank 0).

Workload: B=32768, H=4096, V=128256, bf16, chunk 4096; hidden ~ N(0,1),
weight ~ N(0, 0.02), targets uniform. One step = one forward over the whole batch through the
public API (`gemm_fused_ce_entropy`; vocabulary-parallel `vocab_parallel_ce_entropy` for N > 1).
The same line also reports the training step (`gemm_megakernel_fast` + loss.backward(), configs[2])
under "fwd_bwd", BASELINE.json configs[3] and configs[4] under "configs" (few steps each), and at every
N the accuracy of the sharded result against an fp32 ground truth merged over the shards (forward CE /
entropy over all rows, d_hidden rows, d_weight rows of every shard).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --micro        (HBM-bound kernels alone: finalize, dlogits, column sums, fp32 split,
                                    CE over logits)
    torchrun --nproc-per-node N bench.py --gpus N ...      (vocabulary sharded over N GPUs)

Timing: CUDA events on the launching stream, barrier + synchronize on both sides, max over ranks.
Inputs (1 GiB weight, 256 MiB hidden) are far larger than L2, so no flush is needed between steps.
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "fast-reduction_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "fwd & fwd+bwd ms @B32768 H4096 V128256 bf16; % dense BF16 tensor peak"
WORKLOAD = "configs[1] forward headline: B=32768 H=4096 V=128256 bf16 chunk 4096"
# The reference's own published numbers for this metric and shape (its README.md:15 and :32: Level-5
# forward and 5M training step at B=32768, H=4096, V=128256, bf16, chunk 4096, on one H100).
REFERENCE_PUBLISHED_MS = {"fwd": 67.0, "fwd_bwd": 243.0}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------------------------------------ utils
def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    if world != n_gpus and rank == 0:
        print(f"[bench] note: --gpus {n_gpus} but WORLD_SIZE={world}; using {world}", file=sys.stderr)
    return world, rank, local


def barrier(world: int):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while a timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, maxes, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            try:
                sm = float(row[1])
                mx = float(row[2])
            except ValueError:
                continue
            sms.append(sm)
            maxes.append(mx)
            try:
                power.append(float(row[3]))
            except ValueError:
                pass
            for n, v in zip(names, row[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = ([s for s, p in zip(sms, power) if p > 300] or sms) if len(power) == len(sms) else sms
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms), "power_w_max": max(power) if power else None}


class KernelTimer:
    """Launch observer for fast_reduction.ops: CUDA events around every libfrx launch."""

    def __init__(self):
        self.pending = []
        self.count = 0

    def before(self, name, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        self.pending.append([name, ev, None])

    def after(self, name, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        self.pending[-1][2] = ev
        self.count += 1

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for name, a, b in self.pending:
            d = out.setdefault(name, {"launches": 0, "total_ms": 0.0})
            d["launches"] += 1
            d["total_ms"] += a.elapsed_time(b)
        return out


_PROBE_SMS = 256
# Dense bf16 tensor work per SM per clock: B200's nominal 2.25 PFLOP/s dense bf16 is 148 SMs x 8,192
# FLOP x 1.855 GHz; the forward GEMM's ncu tensor-pipe utilisation agrees with this rate.
_FLOP_PER_CLK_SM = 8192


def _clock_frac(tflops_per_gpu: float, clocks) -> float | None:
    """Achieved TFLOP/s per GPU over the dense bf16 peak at the SM clock the timed region actually ran
    (frx_clock_probe): how close the kernels come to what the power cap lets the clock allow."""
    mhz = (clocks or {}).get("sm_mhz_effective")
    if not mhz:
        return None
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return round(tflops_per_gpu / (sms * _FLOP_PER_CLK_SM * mhz * 1e6 / 1e12), 4)


def _clock_probe_start():
    """Stamps every SM's %clock64 with %globaltimer (frx_clock_probe) before a timed region."""
    from fast_reduction import _native as nat

    buf = torch.zeros(2, 2 * _PROBE_SMS, dtype=torch.int64, device="cuda")
    nat.check(nat.load().frx_clock_probe(buf[0].data_ptr(), _PROBE_SMS, nat.stream_of(buf.device)),
              "frx_clock_probe")
    return buf


def _clock_probe_stop(buf):
    """Second stamp after the region; returns a function giving the region's average SM clock in MHz
    (median over the SMs stamped both times; cycle counters are per SM)."""
    from fast_reduction import _native as nat

    nat.check(nat.load().frx_clock_probe(buf[1].data_ptr(), _PROBE_SMS, nat.stream_of(buf.device)),
              "frx_clock_probe")

    def read():
        b = buf.cpu().view(2, _PROBE_SMS, 2)
        rates = [(int(b[1, s, 0]) - int(b[0, s, 0])) / (int(b[1, s, 1]) - int(b[0, s, 1])) * 1000.0
                 for s in range(_PROBE_SMS)
                 if int(b[0, s, 1]) and int(b[1, s, 1]) and int(b[1, s, 1]) > int(b[0, s, 1])]
        return round(statistics.median(rates), 1) if rates else None

    return read


def time_steps(step, steps: int, warmup: int, world: int, timer: KernelTimer | None = None, sampler=None):
    from fast_reduction import ops

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    prev = ops.set_launch_observer(timer) if timer is not None else None
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    probe = _clock_probe_start()
    start.record()
    for _ in range(steps):
        step()
    end.record()
    effective_mhz = _clock_probe_stop(probe)
    torch.cuda.synchronize()
    if timer is not None:
        ops.set_launch_observer(prev)
    clocks = sampler.stop() if sampler is not None else None
    if clocks is not None:
        clocks["sm_mhz_effective"] = effective_mhz()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    return max_over_ranks(ms, world), clocks


# ------------------------------------------------------------------------------------------------ inputs
def make_headline_inputs(B, H, V, vstart, vend, seed=0, weight_std=0.02):
    """hidden ~ N(0, 1) [B, H], this rank's rows [vstart, vend) of a weight ~ N(0, weight_std) [V, H],
    targets uniform in [0, V): bf16, drawn on the device. The weight is drawn in 8192-row blocks with
    per-block seeds, so every rank sees the same slice values for any number of ranks."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn(B, H, device="cuda", generator=g).to(torch.bfloat16)
    weight = torch.empty(vend - vstart, H, device="cuda", dtype=torch.bfloat16)
    blk = 8192
    for r0 in range(0, V, blk):
        r1 = min(r0 + blk, V)
        lo, hi = max(r0, vstart), min(r1, vend)
        if lo >= hi:
            continue
        gb = torch.Generator(device="cuda").manual_seed(seed * 1_000_003 + r0 + 1)
        rows = (torch.randn(r1 - r0, H, device="cuda", generator=gb) * weight_std).to(torch.bfloat16)
        weight[lo - vstart:hi - vstart] = rows[lo - r0:hi - r0]
    target = torch.randint(0, V, (B,), device="cuda", generator=g)
    return hidden, weight, target


def make_config_inputs(cfg: dict, world: int, rank: int):
    """BASELINE.json configs[3] / configs[4] inputs for this rank (seeded, identical on every rank):
    configs[3] sets a seeded 5% of the targets to ignore_index -100; configs[4] moves a seeded 1% of
    the targets into the last 256-column tile of a vocabulary shard (the ragged one when the shard
    width is not a multiple of 256), spread over the shards of this run."""
    from fast_reduction import vocab_parallel as vp

    B, H, V = cfg["B"], cfg["H"], cfg["V"]
    vstart, vend = vp.shard_bounds(V, world, rank)
    hidden, weight, target = make_headline_inputs(B, H, V, vstart, vend, seed=cfg["seed"], weight_std=cfg["wstd"])
    g = torch.Generator().manual_seed(cfg["seed"] + 7)
    t = target.cpu()
    if cfg.get("tail_frac"):
        n = int(round(cfg["tail_frac"] * B))
        idx = torch.randperm(B, generator=g)[:n]
        for j, i in enumerate(idx.tolist()):
            a, b = vp.shard_bounds(V, world, j % world)
            last = a + (b - a - 1) // 256 * 256
            t[i] = int(torch.randint(last, b, (1,), generator=g))
    if cfg.get("ignore_frac"):
        n = int(round(cfg["ignore_frac"] * B))
        t[torch.randperm(B, generator=g)[:n]] = -100
    return hidden, weight, t.to(hidden.device), vstart, vend


# ------------------------------------------------------------------------------------------------ accuracy
def fp32_stats(hidden, weight_shard, target, vstart, world, rows=None, chunk=2048):
    """fp32 ground truth per row over the whole vocabulary (fp32 logits, TF32 off, fp64 reductions):
    each rank reduces its shard's fp32 logits to (m, s, u, zt), the ranks all-gather them and merge.
    Returns fp64 (lse, entropy, ce-before-ignore) for the first `rows` rows (default all)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    B = hidden.shape[0] if rows is None else rows
    V_r = weight_shard.shape[0]
    wf = weight_shard.float()
    st = torch.empty(B, 4, device=hidden.device, dtype=torch.float64)
    for r0 in range(0, B, chunk):
        r1 = min(B, r0 + chunk)
        z = (hidden[r0:r1].float() @ wf.T).double()
        m = z.max(dim=1).values
        d = z - m[:, None]
        e = d.exp()
        st[r0:r1, 0] = m
        st[r0:r1, 1] = e.sum(1)
        st[r0:r1, 2] = (d * e).sum(1)
        lt = target[r0:r1] - vstart
        inside = (lt >= 0) & (lt < V_r)
        zt = torch.zeros(r1 - r0, device=z.device, dtype=torch.float64)
        zt[inside] = z[inside.nonzero().squeeze(1), lt[inside]]
        st[r0:r1, 3] = zt
        del z, d, e
    if world > 1:
        allst = torch.empty(world * B, 4, device=st.device, dtype=st.dtype)
        dist.all_gather_into_tensor(allst, st)
        allst = allst.view(world, B, 4)
    else:
        allst = st.view(1, B, 4)
    M = allst[:, :, 0].max(dim=0).values
    dm = allst[:, :, 0] - M[None]
    sc = dm.exp()
    S = (allst[:, :, 1] * sc).sum(0)
    U = ((allst[:, :, 2] + dm * allst[:, :, 1]) * sc).sum(0)
    ZT = allst[:, :, 3].sum(0)
    lse = M + S.log()
    ent = S.log() - U / S
    return lse, ent, lse - ZT


def _dz_fp32(z, target_rows, cols_global, lse, ent, ce_weight=1.0, ent_weight=-1.0):
    """dlogits of loss = ce_weight sum ce + ent_weight sum H for fp32 logits z [R, C] whose columns
    are the global vocabulary ids `cols_global`, given fp64 per-row lse / entropy (ignore_index
    -100 rows drop the CE term)."""
    lp = z.double() - lse[:, None]
    p = lp.exp()
    gce = torch.where(target_rows == -100, 0.0, ce_weight).double()
    dz = p * (gce - ent_weight * ent)[:, None] - ent_weight * p * lp
    hit = target_rows[:, None] == cols_global[None, :]
    dz = dz - hit.double() * gce[:, None]
    return dz


def sharded_accuracy(ce, ent, hidden, weight_shard, target, vstart, world, grads=None, rows_check=None,
                     dh_rows=256, dw_rows=256):
    """Forward (and, with grads = (d_hidden, d_weight_shard), training) accuracy of the engine against
    the fp32 ground truth at any number of ranks, with the north-star gates (CE MAE <= 2e-3, entropy
    MAE <= 1e-4, dH / dW MAE <= 2e-3). d_hidden is checked on its first dh_rows rows (each rank's fp32
    contribution from its shard, summed over ranks); d_weight on dw_rows vocabulary rows spread over
    each rank's own shard (incl. its last, possibly ragged, tile), against every row of the batch;
    the reported dW MAE is the maximum over ranks."""
    lse, ent32, ce_raw = fp32_stats(hidden, weight_shard, target, vstart, world, rows=rows_check)
    n = lse.shape[0]
    ign = target[:n] == -100
    ce32 = torch.where(ign, 0.0, ce_raw)
    out = {"rows_checked": n,
           "ce_mae": float((ce.reshape(-1)[:n].double() - ce32).abs().mean()),
           "ent_mae": float((ent.reshape(-1)[:n].double() - ent32).abs().mean()),
           "reference": "fp32 logits (TF32 off), fp64 reductions, merged over shards"}
    if grads is None:
        return out, (lse, ent32)
    d_hidden, d_weight = grads
    V_r = weight_shard.shape[0]
    wf = weight_shard.float()
    # d_hidden rows [0, dh_rows): this shard's fp32 contribution, summed over ranks
    R = min(dh_rows, n)
    z = hidden[:R].float() @ wf.T
    cols = torch.arange(vstart, vstart + V_r, device=z.device)
    dz = _dz_fp32(z, target[:R], cols, lse[:R], ent32[:R])
    dh = (dz.float() @ wf)
    if world > 1:
        dist.all_reduce(dh)
    out["dh_mae"] = float((d_hidden.reshape(-1, hidden.shape[1])[:R].float() - dh).abs().mean())
    out["dh_rows_checked"] = R
    # d_weight rows of this shard, against every row (needs the fp32 statistics of all rows)
    if n == hidden.shape[0]:
        sel = torch.unique(torch.cat([torch.linspace(0, V_r - 1, dw_rows - 8, device=z.device).round().long(),
                                      torch.arange(max(0, V_r - 8), V_r, device=z.device)]))
        zs = hidden.float() @ wf[sel].T
        dzs = _dz_fp32(zs, target, vstart + sel, lse, ent32)
        dws = dzs.float().T @ hidden.float()
        mae = torch.tensor([float((d_weight[sel].float() - dws).abs().mean())], device=z.device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(mae, op=dist.ReduceOp.MAX)
        out["dw_mae"] = float(mae)
        out["dw_rows_checked_per_rank"] = int(sel.numel())
    return out, (lse, ent32)


# ------------------------------------------------------------------------------------------------ cpu baseline
def cpu_baseline(B, H, V, chunk, budget_s: float = 12.0) -> dict:
    """Times the oracle port of the reference's chunked torch path (baseline.py:207-241) on the
    host cores over a row sample of the headline workload, extrapolated linearly to B rows."""
    from oracle import reference_math as rm

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    weight = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16)
    rows = 64
    h = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    t = torch.randint(0, V, (rows,), generator=g)
    t0 = time.perf_counter()
    rm.chunked_linear_xent_entropy(h, weight, t, chunk_size=chunk)
    probe = time.perf_counter() - t0
    rows = int(max(64, min(B, rows * budget_s / max(probe, 1e-3)))) // 64 * 64
    h = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    t = torch.randint(0, V, (rows,), generator=g)
    t0 = time.perf_counter()
    rm.chunked_linear_xent_entropy(h, weight, t, chunk_size=chunk)
    el = time.perf_counter() - t0
    ms_full = el * 1000.0 * B / rows

    # training step (the chunked autograd loop of the reference's benchmarks/bench_fwd_bwd.py:177-195)
    # on a smaller row sample, extrapolated the same way
    rows_fb = max(64, rows // 4 // 64 * 64)
    hf = h[:rows_fb]
    t0 = time.perf_counter()
    rm.chunked_fwd_bwd(hf, weight, t[:rows_fb], chunk_size=chunk)
    el_fb = time.perf_counter() - t0
    del hf

    # configs[0] (B=1024, H=1024, V=32000, chunk 512), timed whole after one warm-up call
    g0 = torch.Generator().manual_seed(0)
    h0 = torch.randn(1024, 1024, generator=g0).to(torch.bfloat16)
    w0 = (torch.randn(32000, 1024, generator=g0) / math.sqrt(1024)).to(torch.bfloat16)
    t0_ = torch.randint(0, 32000, (1024,), generator=g0)
    rm.chunked_linear_xent_entropy(h0, w0, t0_, chunk_size=512)
    t0 = time.perf_counter()
    rm.chunked_linear_xent_entropy(h0, w0, t0_, chunk_size=512)
    el0 = time.perf_counter() - t0
    return {"value": round(ms_full, 1), "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"{rows} of {B} rows (full V={V}, H={H}) in {el:.1f} s on {threads} threads, "
                      f"extrapolated linearly to B={B}; oracle/reference_math.chunked_linear_xent_entropy "
                      f"(restates reference baseline.py:207-241), torch CPU bf16 matmul",
            "fwd_bwd_ms": round(el_fb * 1000.0 * B / rows_fb, 1),
            "fwd_bwd_sample": f"{rows_fb} of {B} rows in {el_fb:.1f} s, extrapolated linearly; "
                              f"oracle/reference_math.chunked_fwd_bwd (restates benchmarks/bench_fwd_bwd.py:177-195)",
            "config0_fwd_ms": round(el0 * 1000.0, 1),
            "cpu_model": _cpu_model(), "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# Bound on the whole --impl reference run (warm-up + timed steps) on the host cores.
_REFERENCE_BUDGET_S = 240.0


def run_reference(args, world, rank):
    """--impl reference: the reference's own algorithm for this path on the host cores: the oracle
    restatement of baseline.chunked_linear_xent_entropy (baseline.py:207-241), bit-exact against the
    reference's golden outputs (tests/test_oracle.py). The reference package itself cannot be
    installed here (its build backend, hatchling, is not in the offline wheelhouse), and its Python
    cannot travel to the GPU box. Each step runs the whole batch of B rows when warm-up + timed
    steps fit _REFERENCE_BUDGET_S (no extrapolation), else an equal row sample per step, scaled to B.
    Under torchrun only rank 0 runs; the other ranks exit without work."""
    if rank != 0:
        return
    from oracle import reference_math as rm

    B, H, V, chunk = args.B, args.H, args.V, args.chunk
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    weight = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16)
    hidden = torch.randn(B, H, generator=g).to(torch.bfloat16)
    target = torch.randint(0, V, (B,), generator=g)
    # probe one chunk to size the step
    t0 = time.perf_counter()
    rm.chunked_linear_xent_entropy(hidden[:chunk], weight, target[:chunk], chunk_size=chunk)
    per_row = (time.perf_counter() - t0) / min(chunk, B)
    n_steps = max(1, args.steps + args.warmup)
    rows = B
    if per_row * B * n_steps > _REFERENCE_BUDGET_S:
        rows = max(chunk, int(_REFERENCE_BUDGET_S / n_steps / per_row) // chunk * chunk)
    h, t = hidden[:rows], target[:rows]
    for _ in range(args.warmup):
        rm.chunked_linear_xent_entropy(h, weight, t, chunk_size=chunk)
    times = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        rm.chunked_linear_xent_entropy(h, weight, t, chunk_size=chunk)
        times.append(time.perf_counter() - t0)
    timed_s = time.perf_counter() - t_all
    per_step = sum(times) / len(times)
    ms_full = per_step * 1000.0 * B / rows
    flops = 2.0 * B * H * V
    full = rows == B
    sample = (f"each step: all {B} rows (full V={V}, H={H}), mean of {args.steps} steps; timed region {timed_s:.1f} s"
              if full else
              f"each step: {rows} of {B} rows (full V, H), mean of {args.steps} steps = {per_step:.2f} s, scaled "
              f"linearly to B={B} (the whole batch x {n_steps} steps would exceed {_REFERENCE_BUDGET_S:.0f} s)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms_full, 1), "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_full, 1), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "B": B, "H": H, "V": V, "chunk": chunk, "parallelism": "cpu",
                   "l2": "inputs larger than L2"},
        "tflops": round(flops / (ms_full / 1000.0) / 1e12, 3),
        "cpu_baseline": {"value": round(ms_full, 1), "unit": "ms", "cores": threads, "kind": "port",
                         "sample": sample, "extrapolated": not full, "cpu_model": _cpu_model(),
                         "implementation": "oracle/reference_math.chunked_linear_xent_entropy (restates reference "
                                           "baseline.py:207-241; reference install unavailable: no hatchling)"},
        "e2e": {"value": round(ms_full, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ our engine
# BASELINE.json configs[3] (large-vocabulary entropy stress) and configs[4] (ragged tail), timed with
# few steps at every N beside the headline, each with its own accuracy check.
CONFIGS = {
    "configs[3]": {"workload": "configs[3] large-vocab stress: hidden [8, 2048, 4096], V=256000, weight N(0, 0.05), "
                               "5% targets ignore_index", "B": 16384, "H": 4096, "V": 256000, "chunk": 4096,
                   "wstd": 0.05, "ignore_frac": 0.05, "seed": 3, "hidden_shape": (8, 2048)},
    "configs[4]": {"workload": "configs[4] ragged tail: B=65536, H=5120, V=152064, chunk 8192, 1% targets in a "
                               "shard's last vocabulary tile", "B": 65536, "H": 5120, "V": 152064, "chunk": 8192,
                   "wstd": 0.02, "tail_frac": 0.01, "seed": 4},
}
# The N=1 run leaves its clock-normalised fractions here, so later N>1 runs of the same workload on
# the same box can report their efficiency at equal clocks.
_N1_STATE = Path("/tmp/frx_bench_n1.json")


def _train_fn(gk, vp, world, h_leaf, w_leaf, target, vstart, V, chunk):
    def train_step():
        h_leaf.grad = None
        w_leaf.grad = None
        if world == 1:
            loss, _, _ = gk.gemm_megakernel_fast(h_leaf, w_leaf, target, chunk_size=chunk)
        else:
            loss, _, _ = vp.vocab_parallel_megakernel(h_leaf, w_leaf, target, vstart, V, chunk_size=chunk)
        loss.backward()
    return train_step


def _fwd_fn(gk, vp, world, hidden, weight, target, vstart, V, chunk):
    if world == 1:
        return lambda: gk.gemm_fused_ce_entropy(hidden, weight, target, chunk_size=chunk)
    return lambda: vp.vocab_parallel_ce_entropy(hidden, weight, target, vstart, V, chunk_size=chunk)


def _gpu_numa_node(index: int):
    """NUMA node of GPU `index` from its PCI address (None when the system does not say)."""
    try:
        pr = torch.cuda.get_device_properties(index)
        addr = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{addr}/numa_node").read_text().strip())
        return node if node >= 0 else None
    except Exception:
        return None


def _node_cpus(node: int):
    try:
        out = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            a, _, b = part.partition("-")
            out.update(range(int(a), int(b or a) + 1))
        return out
    except Exception:
        return None


def run_config(name, cfg, world, rank, local, steps, warmup, peaks):
    """Forward and training step of one BASELINE config at this N (few steps), with accuracy."""
    from fast_reduction import gemm_kernel as gk
    from fast_reduction import vocab_parallel as vp

    B, H, V, chunk = cfg["B"], cfg["H"], cfg["V"], cfg["chunk"]
    hidden, weight, target, vstart, vend = make_config_inputs(cfg, world, rank)
    shape = cfg.get("hidden_shape")
    hs = hidden.view(*shape, H) if shape else hidden
    ts = target.view(*shape) if shape else target
    fwd = _fwd_fn(gk, vp, world, hs, weight, ts, vstart, V, chunk)
    fwd_ms, fclk = time_steps(fwd, steps, warmup, world, sampler=ClockSampler(local))
    h_leaf = hs.detach().requires_grad_(True)
    w_leaf = weight.detach().requires_grad_(True)
    train = _train_fn(gk, vp, world, h_leaf, w_leaf, ts, vstart, V, chunk)
    fb_ms, bclk = time_steps(train, steps, warmup, world, sampler=ClockSampler(local))
    train()
    ce, ent, _ = fwd()
    acc, _ = sharded_accuracy(ce, ent, hidden, weight, target, vstart, world, grads=(h_leaf.grad, w_leaf.grad),
                              rows_check=1024, dh_rows=128)
    peak_tf = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    ff, fbf = 2.0 * B * H * V, 6.0 * B * H * V
    res = {"workload": cfg["workload"], "B": B, "H": H, "V": V, "chunk": chunk, "steps": steps, "warmup": warmup,
           "fwd_ms": round(fwd_ms, 3), "fwd_bwd_ms": round(fb_ms, 3),
           "fwd_frac_of_peak": round(ff / (fwd_ms / 1e3) / 1e12 / (peak_tf * world), 4),
           "fwd_bwd_frac_of_peak": round(fbf / (fb_ms / 1e3) / 1e12 / (peak_tf * world), 4),
           "fwd_frac_of_clock_limited_peak": _clock_frac(ff / (fwd_ms / 1e3) / 1e12 / world, fclk),
           "fwd_bwd_frac_of_clock_limited_peak": _clock_frac(fbf / (fb_ms / 1e3) / 1e12 / world, bclk),
           "sm_mhz_effective": {"fwd": (fclk or {}).get("sm_mhz_effective"),
                                "fwd_bwd": (bclk or {}).get("sm_mhz_effective")},
           "accuracy": acc}
    del hidden, weight, target, hs, ts, h_leaf, w_leaf, ce, ent
    torch.cuda.empty_cache()
    return res


def run_ours(args, world, rank, local):
    from fast_reduction import _native as nat
    from fast_reduction import gemm_kernel as gk
    from fast_reduction import vocab_parallel as vp

    nat.load()
    B, H, V, chunk = args.B, args.H, args.V, args.chunk
    vstart, vend = vp.shard_bounds(V, world, rank)
    Vr = vend - vstart
    peaks = load_peaks()
    hidden, weight, target = make_headline_inputs(B, H, V, vstart, vend, seed=0)
    torch.cuda.synchronize()
    fwd = _fwd_fn(gk, vp, world, hidden, weight, target, vstart, V, chunk)

    # ---- forward (headline value) with per-kernel event timing and clock sampling
    timer = KernelTimer()
    sampler = ClockSampler(local)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.cuda.reset_peak_memory_stats(dev)
    mem_base = torch.cuda.memory_allocated(dev)
    fwd_ms, clocks = time_steps(fwd, args.steps, args.warmup, world, timer, sampler)
    peak_extra_fwd = (torch.cuda.max_memory_allocated(dev) - mem_base) / 1e9
    ksum = timer.summary()
    launches_fwd = timer.count
    flops_fwd = 2.0 * B * H * V
    gemm = ksum.get("fwd_partials", {"launches": 1, "total_ms": float("nan")})
    gemm_avg_ms = gemm["total_ms"] / max(gemm["launches"], 1)
    # The forward launches chunk-size row groups, merged while a launch's partials stay small
    # (gemm_kernel._launch_rows): count the launches of a step rather than assume one per chunk.
    launches_per_step = max(gemm["launches"] / args.steps, 1.0)
    rows_per_launch = int(round(B / launches_per_step))
    gemm_flops = 2.0 * B * Vr * H / launches_per_step
    achieved_tflops = gemm_flops / (gemm_avg_ms / 1000.0) / 1e12
    peak_tf = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    peak_sus = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    ce, ent, lp = fwd()

    # ---- configs[0] (B=1024, H=1024, V=32000, chunk 512): a launch-bound size, eager vs CUDA graph
    small = None
    if world == 1 and not args.no_config0:
        from fast_reduction.graphs import graphed_forward

        g0 = torch.Generator().manual_seed(0)
        h0 = torch.randn(1024, 1024, generator=g0).to(torch.bfloat16).cuda()
        w0 = (torch.randn(32000, 1024, generator=g0) / math.sqrt(1024)).to(torch.bfloat16).cuda()
        t0 = torch.randint(0, 32000, (1024,), generator=g0).cuda()
        eager_ms, _ = time_steps(lambda: gk.gemm_fused_ce_entropy(h0, w0, t0, chunk_size=512), 50, 5, 1)
        run0 = graphed_forward(h0, w0, t0, chunk_size=512)
        graph_ms, _ = time_steps(run0, 50, 5, 1)
        small = {"workload": "configs[0] forward: B=1024 H=1024 V=32000 bf16 chunk 512",
                 "note": "launch-overhead comparison; the 65 MB weight stays in L2 between steps (no flush)",
                 "eager_ms": round(eager_ms, 4), "graph_ms": round(graph_ms, 4),
                 "tflops_graph": round(2.0 * 1024 * 1024 * 32000 / (graph_ms / 1000.0) / 1e12, 1)}
        del h0, w0, t0, run0

    # ---- fwd+bwd (training step, configs[2])
    fb = None
    grads = None
    if not args.no_fwd_bwd:
        h_leaf = hidden.detach().requires_grad_(True)
        w_leaf = weight.detach().requires_grad_(True)
        train_step = _train_fn(gk, vp, world, h_leaf, w_leaf, target, vstart, V, chunk)
        timer_fb = KernelTimer()
        fb_steps = max(1, min(args.steps, 10))
        torch.cuda.reset_peak_memory_stats(dev)
        mem_base_fb = torch.cuda.memory_allocated(dev)
        fb_ms, fb_clocks = time_steps(train_step, fb_steps, max(args.warmup, 1), world, timer_fb, ClockSampler(local))
        peak_extra_fb = (torch.cuda.max_memory_allocated(dev) - mem_base_fb) / 1e9
        kfb = timer_fb.summary()
        # The same step with the dlogits pass serialised on the main stream: per-kernel times without
        # the side stream's waits for SMs (the overlapped figures above include them).
        prev_overlap = gk._OVERLAP_DLOGITS
        gk._OVERLAP_DLOGITS = False
        timer_ser = KernelTimer()
        ser_ms, _ = time_steps(train_step, 2, 1, world, timer_ser)
        gk._OVERLAP_DLOGITS = prev_overlap
        kser = timer_ser.summary()
        flops_fb = 6.0 * B * H * V
        fb = {"ms": round(fb_ms, 3), "tflops": round(flops_fb / (fb_ms / 1000.0) / 1e12, 1),
              "frac_of_peak": round(flops_fb / (fb_ms / 1000.0) / 1e12 / (peak_tf * world), 4),
              "frac_of_sustained_peak": round(flops_fb / (fb_ms / 1000.0) / 1e12 / (peak_sus * world), 4),
              "frac_of_clock_limited_peak": _clock_frac(flops_fb / (fb_ms / 1000.0) / 1e12 / world, fb_clocks),
              "steps": fb_steps,
              "workload": "configs[2] gemm_megakernel_fast + loss.backward(), ce_weight 1, ent_weight -1",
              "peak_extra_mem_gb": round(peak_extra_fb, 3),
              "kernels_ms_per_step_wall": {k: round(v["total_ms"] / fb_steps, 3) for k, v in kfb.items()},
              "kernels_ms_per_step_wall_note": "events around each launch on its own stream while the dlogits pass "
                                               "overlaps the next forward GEMM: includes time spent waiting for SMs",
              "kernels_ms_per_step": {k: round(v["total_ms"] / 2, 3) for k, v in kser.items()},
              "kernels_ms_per_step_note": f"serialised pass (FRX_OVERLAP_DLOGITS=0, 2 steps, {ser_ms:.2f} ms/step): "
                                          "each kernel alone on the stream",
              "gpu_launches_per_step": timer_fb.count // fb_steps, "clocks": fb_clocks}
        train_step()
        grads = (h_leaf.grad, w_leaf.grad)

    # ---- accuracy at every N: fp32 ground truth over the shards, forward over all rows, gradients
    acc, _ = sharded_accuracy(ce, ent, hidden, weight, target, vstart, world, grads=grads)
    if fb is not None:
        fb["accuracy"] = {k: acc[k] for k in ("dh_mae", "dh_rows_checked", "dw_mae", "dw_rows_checked_per_rank")
                          if k in acc}
        fb["accuracy"]["gate"] = "dH / dW MAE <= 2e-3 vs fp32"
        h_leaf.grad = None
        w_leaf.grad = None
        del h_leaf, w_leaf, grads
    acc = {k: acc[k] for k in ("rows_checked", "ce_mae", "ent_mae", "reference")}
    acc["gate"] = "CE MAE <= 2e-3, entropy MAE <= 1e-4 vs fp32"
    del ce, ent, lp
    torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers (H2D inputs, D2H results inside)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(gk, vp, world, rank, local, hidden, weight, target, vstart, V, chunk, args)

    # ---- BASELINE configs[3] / configs[4] at this N
    cfgs = None
    if not args.no_configs:
        del hidden, weight, target
        torch.cuda.empty_cache()
        cfgs = {name: run_config(name, cfg, world, rank, local, args.config_steps, 3, peaks)
                for name, cfg in CONFIGS.items()}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(B, H, V, chunk)

    traffic = None
    tp = REPO / "profiles" / "traffic.json"
    if tp.exists():
        try:
            tj = json.loads(tp.read_text())
            ent_ = tj.get("fwd_partials")
            if ent_ and ent_.get("rows_per_launch") == rows_per_launch and ent_.get("vocab_shard"):
                traffic = round(ent_["dram_bytes_per_launch"] * Vr / ent_["vocab_shard"])
        except Exception:
            traffic = None

    if rank != 0:
        return
    tflops = flops_fwd / (fwd_ms / 1000.0) / 1e12
    headline_shape = (B, H, V, chunk) == (32768, 4096, 128256, 4096)
    if fb is not None and headline_shape:
        fb["vs_baseline"] = round(fb["ms"] / REFERENCE_PUBLISHED_MS["fwd_bwd"], 4)
    fwd_clock_frac = _clock_frac(tflops / world, clocks)
    scaling_cn = _clock_normalised_scaling(world, (B, H, V, chunk), fwd_clock_frac,
                                           None if fb is None else fb["frac_of_clock_limited_peak"])
    line = {
        "metric": METRIC,
        "value": round(fwd_ms, 3),
        "unit": "ms",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(fwd_ms, 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": round(fwd_ms / REFERENCE_PUBLISHED_MS["fwd"], 4) if headline_shape else None,
        "vs_baseline_source": ("reference's published Level-5 forward, 67 ms on one H100 (its README.md:15); "
                               "value / 67, lower is better") if headline_shape else None,
        "dtype": "bf16",
        "data": "synthetic (seeded: hidden N(0,1), weight N(0,0.02), uniform targets)",
        "config": {"workload": WORKLOAD, "B": B, "H": H, "V": V, "chunk": chunk,
                   "parallelism": f"vocab-sharded x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (no flush needed)"},
        "tflops": round(tflops, 1),
        "frac_of_peak": round(tflops / (peak_tf * world), 4),
        "frac_of_sustained_peak": round(tflops / (peak_sus * world), 4),
        "frac_of_clock_limited_peak": fwd_clock_frac,
        "scaling_clock_normalised": scaling_cn,
        "peak_bf16_tflops": peak_tf,
        "peak_bf16_tflops_sustained": peak_sus,
        "peak_source": peaks.get("source"),
        "roofline": {"bound": "tensor", "kernel": "gemm_tcgen05_pair_kernel<CEPartialsEpilogue> (frx_fwd_partials)",
                     "achieved": round(achieved_tflops, 1), "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": round(achieved_tflops / peak_tf, 4), "traffic": traffic,
                     "algorithmic_flop_per_launch": gemm_flops, "avg_launch_ms": round(gemm_avg_ms, 4),
                     "launches_timed": gemm["launches"]},
        "kernels_ms_per_step": {k: round(v["total_ms"] / args.steps, 4) for k, v in ksum.items()},
        "gpu_launches": launches_fwd,
        "peak_extra_mem_gb": round(peak_extra_fwd, 3),
        "clocks": clocks,
        "accuracy": acc,
        "fwd_bwd": fb,
        "config0": small,
        "configs": cfgs,
        "e2e": e2e,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def _clock_normalised_scaling(world, shape, fwd_frac, fb_frac):
    """Each N's fraction of the clock-limited peak over the N=1 run's, for the forward and the training
    step (per-GPU efficiency at equal clocks). The N=1 run stores its fractions on the box for the
    N>1 runs that follow it; without that record the ratios are null."""
    now = time.time()
    if world == 1:
        try:
            _N1_STATE.write_text(json.dumps({"shape": list(shape), "fwd": fwd_frac, "fwd_bwd": fb_frac, "t": now}))
        except OSError:
            pass
        return {"fwd": 1.0 if fwd_frac else None, "fwd_bwd": 1.0 if fb_frac else None,
                "basis": "N=1 run of this command"}
    try:
        ref = json.loads(_N1_STATE.read_text())
    except (OSError, ValueError):
        return {"fwd": None, "fwd_bwd": None, "basis": "no N=1 record on this box"}
    if ref.get("shape") != list(shape) or now - ref.get("t", 0) > 6 * 3600:
        return {"fwd": None, "fwd_bwd": None, "basis": "no matching N=1 record on this box"}

    def ratio(a, b):
        return round(a / b, 4) if a and b else None

    return {"fwd": ratio(fwd_frac, ref.get("fwd")), "fwd_bwd": ratio(fb_frac, ref.get("fwd_bwd")),
            "basis": f"N=1 run {now - ref['t']:.0f} s earlier on this box"}


def run_e2e(gk, vp, world, rank, local, hidden, weight, target, vstart, V, chunk, args):
    """e2e: the public API with pinned host hidden / weight (shard) / target in and host results out.
    With N ranks every rank uploads only its 1/N share of the hidden rows (the API's host path), so
    only that share is pinned (cudaHostRegister on a pageable full-size tensor); host buffers are
    allocated from CPUs of the GPU's NUMA node when the system reports one."""
    B, H = hidden.shape
    node = _gpu_numa_node(local)
    cpus = _node_cpus(node) if node is not None else None
    old_aff = None
    if cpus:
        try:
            old_aff = os.sched_getaffinity(0)
            os.sched_setaffinity(0, cpus)
        except OSError:
            old_aff = None
    c = (B + world - 1) // world
    lo, hi = min(B, rank * c), min(B, (rank + 1) * c)
    registered = None
    if world > 1:
        h_host = torch.empty(B, H, dtype=hidden.dtype)
        h_host[lo:hi].copy_(hidden[lo:hi])
        try:
            cr = torch.cuda.cudart()
            nbytes = (hi - lo) * H * hidden.element_size()
            if nbytes and int(cr.cudaHostRegister(h_host[lo:hi].data_ptr(), nbytes, 0)) == 0:
                registered = h_host[lo:hi].data_ptr()
        except Exception:
            registered = None
        if registered is None:  # fall back to pinning everything
            h_host = h_host.pin_memory()
    else:
        h_host = torch.empty(B, H, dtype=hidden.dtype, pin_memory=True)
        h_host.copy_(hidden)
    w_host = torch.empty(weight.shape, dtype=weight.dtype, pin_memory=True)
    w_host.copy_(weight)
    t_host = torch.empty(target.shape, dtype=target.dtype, pin_memory=True)
    t_host.copy_(target)

    # This rank's H2D rate for its upload (hidden share + weight shard), all ranks at once.
    up = hi - lo
    dst_h = torch.empty(max(up, 1), H, dtype=hidden.dtype, device=hidden.device)
    dst_w = torch.empty_like(weight)
    barrier(world)
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(3):
        if up:
            dst_h[:up].copy_(h_host[lo:hi], non_blocking=True)
        dst_w.copy_(w_host, non_blocking=True)
    e_ev.record()
    torch.cuda.synchronize()
    up_bytes = (up * H + weight.numel()) * hidden.element_size()
    gbs = up_bytes * 3 / (s_ev.elapsed_time(e_ev) / 1e3) / 1e9
    del dst_h, dst_w
    rates = torch.tensor([gbs], device=hidden.device, dtype=torch.float64)
    if world > 1:
        allr = torch.empty(world, device=hidden.device, dtype=torch.float64)
        dist.all_gather_into_tensor(allr, rates)
        rates = allr

    def e2e_step():
        if world == 1:
            res = gk.gemm_fused_ce_entropy(h_host, w_host, t_host, chunk_size=chunk)
        else:
            res = vp.vocab_parallel_ce_entropy(h_host, w_host, t_host, vstart, V, chunk_size=chunk)
        assert res[0].device.type == "cpu"

    e2e_ms, _ = time_steps(e2e_step, max(1, min(args.steps, 10)), max(args.warmup, 3), world)
    if registered is not None:
        torch.cuda.cudart().cudaHostUnregister(registered)
    if old_aff is not None:
        os.sched_setaffinity(0, old_aff)
    h2d = up * H * 2 + w_host.numel() * 2 + t_host.numel() * 8
    return {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(3 * B * 4),
            "path": "pinned host hidden/weight(shard)/target -> gemm_fused_ce_entropy / vocab_parallel_ce_entropy "
                    "(host in, host out; bytes per rank)",
            "h2d_gbs_per_rank": [round(float(x), 1) for x in rates.tolist()],
            "h2d_gbs_note": "each rank's own upload (hidden share + weight shard) copied alone, all ranks at once",
            "numa": {"gpu_node": node, "host_buffers_bound_to_node": bool(cpus) and old_aff is not None,
                     "hidden_pinned": "share only (cudaHostRegister)" if registered is not None else "whole tensor"}}


def run_micro(args):
    """--micro: each HBM-bound libfrx kernel alone on inputs larger than L2, timed with CUDA events on
    the launching stream; one JSON line per kernel with its algorithmic bytes and achieved GB/s."""
    from fast_reduction import ops

    peaks = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)

    def timeit(fn, iters=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / iters

    def report(kernel, shape, ms, nbytes, note):
        gbs = nbytes / (ms / 1000.0) / 1e9
        print(json.dumps({"micro": kernel, "shape": shape, "ms": round(ms, 4), "algorithmic_bytes": int(nbytes),
                          "achieved_gbs": round(gbs, 1), "peak_gbs": hbm, "frac_of_hbm_peak": round(gbs / hbm, 4),
                          "peak_source": peaks.get("source"), "bytes": note}), flush=True)

    # finalize: partials of all 32768 rows over the 501 vocabulary tiles of V=128256 (the host-streamed
    # forward's single finalize), 16 B per (tile, row) in, 12 B per row out (ce, entropy, log_probs).
    sc = max(1, args.micro_scale)
    T, R = ops.n_vocab_tiles(128256), 32768
    part = torch.randn(T, R, 4, device=dev, generator=g).abs_() + 1.0
    tgt = torch.randint(0, 128256, (R,), device=dev, generator=g)
    outs = [torch.empty(R, device=dev) for _ in range(3)]
    ms = timeit(lambda: ops.finalize(part, T, R, R, target=tgt, vocab_size=128256, ce=outs[0], entropy=outs[1],
                                     log_probs=outs[2]))
    report("finalize", [T, R], ms, T * R * 16 + R * (8 + 12), "16 B per (tile, row) + 8 B target + 12 B out per row")
    del part, outs

    # dlogits: one 4096-row chunk of the headline training step (fp32 logits in, bf16 dlogits out).
    M, V = 4096 // sc, 128256
    ld = ops.round_up(V, 4)
    z = torch.randn(M, ld, device=dev, generator=g)
    lse = torch.full((M,), 12.0, device=dev)
    ent = torch.full((M,), 10.0, device=dev)
    tg = torch.randint(0, V, (M,), device=dev, generator=g)
    dz = torch.empty(M, ops.round_up(V, 8), device=dev, dtype=torch.bfloat16)
    ms = timeit(lambda: ops.dlogits(z, tg, lse, ent, dz, rows=M, vocab_shard=V))
    report("dlogits", [M, V], ms, M * V * 6 + M * 16, "4 B logit read + 2 B dlogit write per element + row stats")
    del z
    # the training pass's form: fp16 z - m_tile in, the tile maxima from the partials
    T = ops.n_vocab_tiles(V)
    zr = torch.randn(M, ops.round_up(V, 8), device=dev, generator=g).mul_(-3.0).to(torch.float16)
    pt = torch.randn(T, M, 4, device=dev, generator=g)
    ms = timeit(lambda: ops.dlogits_tilerel(zr, pt, M, tg, lse, ent, dz, rows=M, vocab_shard=V))
    report("dlogits_tilerel", [M, V], ms, M * V * 4 + M * 16 + T * M * 4,
           "2 B fp16 logit read + 2 B dlogit write per element + row stats + 4 B tile max per (tile, row)")
    del zr, pt

    # column sums: d_bias of the headline training step (bf16 dlogits [32768, 128256] -> fp32 [V]).
    R2 = 32768 // sc
    big = torch.empty(R2, ops.round_up(V, 8), device=dev, dtype=torch.bfloat16).normal_(generator=g)
    db = torch.empty(V, device=dev)
    ms = timeit(lambda: ops.column_sums(big, db, rows=R2, cols=V), iters=5)
    report("column_sums", [R2, V], ms, R2 * V * 2 + V * 4, "2 B per element read + 4 B per column written")
    del big, dz

    # fp32 -> bf16 hi / mid / lo parts (the fp32 input path's split), a [32768, 4096] hidden
    R4, C4 = 32768 // sc, 4096
    xf = torch.randn(R4, C4, device=dev, generator=g)
    parts = torch.empty(3, R4, C4, device=dev, dtype=torch.bfloat16)
    ms = timeit(lambda: ops.split_f32(xf, parts[0], (0, 1, 2), part_stride=R4 * C4))
    report("split_f32", [R4, C4], ms, R4 * C4 * (4 + 3 * 2), "4 B fp32 read + three 2 B parts written per element")
    del xf, parts

    # standalone CE / entropy over materialised bf16 logits [32768, 32000] (configs[0]'s vocabulary).
    M3, N3 = 32768 // sc, 32000
    logits = torch.empty(M3, N3, device=dev, dtype=torch.bfloat16).normal_(generator=g)
    tg3 = torch.randint(0, N3, (M3,), device=dev, generator=g)
    from fast_reduction.cute_cross_entropy import ce_entropy_fwd
    ms = timeit(lambda: ce_entropy_fwd(logits, tg3))
    report("logits_partials+finalize (ce_entropy_fwd)", [M3, N3], ms, M3 * N3 * 2 + M3 * 16,
           "2 B per logit read + 8 B target + 8 B out per row")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--B", type=int, default=32768)
    ap.add_argument("--H", type=int, default=4096)
    ap.add_argument("--V", type=int, default=128256)
    ap.add_argument("--chunk", type=int, default=4096)
    ap.add_argument("--no-fwd-bwd", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config0", action="store_true", help="skip the configs[0] eager-vs-graph line")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[3] / configs[4] block")
    ap.add_argument("--config-steps", type=int, default=3, help="timed steps per configs[3] / configs[4] leg")
    ap.add_argument("--micro", action="store_true", help="time the HBM-bound kernels alone (one line each)")
    ap.add_argument("--micro-scale", type=int, default=1, help="divide the --micro row counts (small ncu cases)")
    args = ap.parse_args()
    if args.micro:
        run_micro(args)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
