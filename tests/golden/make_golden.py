"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's own code.

Run in the build container, where the reference checkout is readable:
    python tests/golden/make_golden.py --ref /path/to/fast-reduction

It imports the reference's fast_reduction/baseline.py by file path (pure torch, runs on CPU)
under a private module name and records its outputs on small seeded inputs. The fixtures are
committed; nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import math
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference_baseline(ref_root: Path):
    path = ref_root / "fast_reduction" / "baseline.py"
    spec = importlib.util.spec_from_file_location("_reference_baseline", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a checkout of the reference (justinchiu/fast-reduction)")
    args = ap.parse_args()
    ref = load_reference_baseline(Path(args.ref))
    torch.set_num_threads(8)
    out = {}

    # 1. Unfused baseline on fp32 inputs (the reference's own CPU test shape, tests/test_ce_impls.py:28-40).
    torch.manual_seed(42)
    B, H, V = 32, 64, 128
    h = torch.randn(B, H)
    w = torch.randn(V, H)
    t = torch.randint(0, V, (B,))
    ce, ent, lp = ref.baseline_linear_xent_entropy(h, w, t)
    out.update(unfused_hidden=h.numpy(), unfused_weight=w.numpy(), unfused_target=t.numpy(),
               unfused_ce=ce.numpy(), unfused_ent=ent.numpy(), unfused_lp=lp.numpy())

    # 2. Chunked bf16 path, ragged vocab (V not a multiple of 256) and ragged last chunk.
    torch.manual_seed(7)
    B, H, V, chunk = 72, 64, 1000, 32
    h = torch.randn(B, H).to(torch.bfloat16)
    w = (torch.randn(V, H) / math.sqrt(H)).to(torch.bfloat16)
    t = torch.randint(0, V, (B,))
    ce, ent, lp = ref.chunked_linear_xent_entropy(h, w, t, chunk_size=chunk)
    out.update(chunked_hidden=h.view(torch.int16).numpy(), chunked_weight=w.view(torch.int16).numpy(),
               chunked_target=t.numpy(), chunked_chunk=np.int64(chunk),
               chunked_ce=ce.numpy(), chunked_ent=ent.numpy(), chunked_lp=lp.numpy())

    # 2b. The same chunked path on fp16 inputs (the reference's matmul runs in the input dtype, so its
    #     logits are rounded to fp16 before the fp32 reduction).
    torch.manual_seed(8)
    B, H, V, chunk = 72, 64, 1000, 32
    h = torch.randn(B, H).to(torch.float16)
    w = (torch.randn(V, H) / math.sqrt(H)).to(torch.float16)
    t = torch.randint(0, V, (B,))
    ce, ent, lp = ref.chunked_linear_xent_entropy(h, w, t, chunk_size=chunk)
    out.update(chunked16_hidden=h.view(torch.int16).numpy(), chunked16_weight=w.view(torch.int16).numpy(),
               chunked16_target=t.numpy(), chunked16_chunk=np.int64(chunk),
               chunked16_ce=ce.numpy(), chunked16_ent=ent.numpy(), chunked16_lp=lp.numpy())

    # 3. fp32 autograd ground truth for gradients (baseline.py:91-150), default g_ce=1, g_ent=-1,
    #    and with per-row upstream gradients.
    torch.manual_seed(123)
    B, H, V = 24, 32, 300
    h = torch.randn(B, H)
    w = torch.randn(V, H) * 0.2
    t = torch.randint(0, V, (B,))
    ce, ent, dh, dw, _ = ref.baseline_linear_xent_entropy_backward(h, w, t)
    gce = torch.rand(B)
    gent = torch.randn(B)
    _, _, dh2, dw2, _ = ref.baseline_linear_xent_entropy_backward(h, w, t, g_ce=gce, g_ent=gent)
    out.update(bwd_hidden=h.numpy(), bwd_weight=w.numpy(), bwd_target=t.numpy(), bwd_ce=ce.numpy(),
               bwd_ent=ent.numpy(), bwd_dh=dh.numpy(), bwd_dw=dw.numpy(), bwd_gce=gce.numpy(),
               bwd_gent=gent.numpy(), bwd_dh_g=dh2.numpy(), bwd_dw_g=dw2.numpy())

    # 3b. the same with a bias (baseline.py:115-142 adds it to the logits and returns d_bias).
    torch.manual_seed(321)
    B, H, V = 20, 32, 300
    h = torch.randn(B, H)
    w = torch.randn(V, H) * 0.2
    b = torch.randn(V) * 0.5
    t = torch.randint(0, V, (B,))
    ce, ent, dh, dw, db = ref.baseline_linear_xent_entropy_backward(h, w, t, bias=b)
    out.update(bias_hidden=h.numpy(), bias_weight=w.numpy(), bias_bias=b.numpy(), bias_target=t.numpy(),
               bias_ce=ce.numpy(), bias_ent=ent.numpy(), bias_dh=dh.numpy(), bias_dw=dw.numpy(), bias_db=db.numpy())

    # 3c. fp16 inputs through the reference's backward: it differentiates in fp32 and casts the
    #     gradients back to fp16 (baseline.py:140-141).
    torch.manual_seed(654)
    B, H, V = 40, 64, 500
    h = torch.randn(B, H).to(torch.float16)
    w = (torch.randn(V, H) * 0.2).to(torch.float16)
    t = torch.randint(0, V, (B,))
    ce, ent, dh, dw, _ = ref.baseline_linear_xent_entropy_backward(h, w, t)
    out.update(bwd16_hidden=h.view(torch.int16).numpy(), bwd16_weight=w.view(torch.int16).numpy(),
               bwd16_target=t.numpy(), bwd16_ce=ce.numpy(), bwd16_ent=ent.numpy(),
               bwd16_dh=dh.view(torch.int16).numpy(), bwd16_dw=dw.view(torch.int16).numpy())

    # 4. BASELINE configs[0] (B=1024, H=1024, V=32000, chunk 512, seed 0): inputs are regenerated
    #    from the seed at test time (checked by digest); only the reference's outputs are stored.
    g = torch.Generator().manual_seed(0)
    B, H, V = 1024, 1024, 32000
    h = torch.randn(B, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g) * (1.0 / math.sqrt(H))).to(torch.bfloat16)
    t = torch.randint(0, V, (B,), generator=g, dtype=torch.int64)
    ce, ent, lp = ref.chunked_linear_xent_entropy(h, w, t, chunk_size=512)
    out.update(cfg0_digest=np.array(digest(h, w, t)), cfg0_ce=ce.numpy(), cfg0_ent=ent.numpy(),
               cfg0_lp=lp.numpy())

    np.savez_compressed(HERE / "reference_baseline.npz", **out)
    print("wrote", HERE / "reference_baseline.npz")


if __name__ == "__main__":
    main()
