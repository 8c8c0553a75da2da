"""The DSpark draft attention on the GPU (``dsm.attention``) against golden vectors from the
reference's own ``DSparkAttention`` (``tests/golden/make_golden_attn.py``) and against the
oracle at larger widths.

Every step of a golden case is replayed: the prefill that seeds the sliding KV window, the
decode steps and ``advance_window``. The outputs and the window after each step are
compared. Tolerances are max|out - ref| / max|ref|:
* bf16 allows 2e-2: the five projections round to bf16 after fp32 sums taken in another
  order.
* fp32 allows 2e-3: fp32 activations are staged hi + lo and keep fp32 precision, but fp32
  weights are held as f16 in the packed tiles, 2^-12 relative each."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle
from dsm import _lib
from dsm.attention import DSparkAttention
from helpers import max_rel_err
from oracle.attention_oracle import AttnDims
from test_oracle_attn import DIMS, HERE, _t

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "attn_*.npz")))


def _module(dims: dict, weights: dict) -> DSparkAttention:
    a = DSparkAttention(dims, max_seq_len=64).to(DEV)
    with torch.no_grad():
        for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b"):
            getattr(a, k).weight = torch.nn.Parameter(weights[k].to(DEV), requires_grad=False)
        a.q_norm.weight.copy_(weights["q_norm"])
        a.kv_norm.weight.copy_(weights["kv_norm"])
        a.attn_sink.copy_(weights["attn_sink"])
    return a


@pytest.mark.parametrize("name", CASES)
def test_attention_matches_reference_goldens(name, attn_kernel):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    bf16 = bool(z["dtype_bf16"])
    if attn_kernel == 0 and not bf16:
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    tol = 2e-2 if bf16 else 2e-3
    w = {k: _t(z[k]) for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b")}
    w.update(q_norm=_t(z["q_norm"]), kv_norm=_t(z["kv_norm"]), attn_sink=_t(z["sink"]))
    a = _module(DIMS, w)
    x0 = _t(z["prefill_x"]).to(DEV)
    ret = a(x0, 0, _t(z["prefill_main"]).to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(ret.cpu(), x0.cpu())
    assert max_rel_err(a.window, _t(z["window_0"])) < tol
    for i, kind in enumerate(z["plan"]):
        if kind == "advance":
            a.advance_window(_t(z[f"s{i}_main"]).to(DEV), int(z[f"s{i}_pos"]))
        else:
            out = a(_t(z[f"s{i}_x"]).to(DEV), int(z[f"s{i}_pos"]), _t(z[f"s{i}_main"]).to(DEV))
            torch.cuda.synchronize()
            ref = _t(z[f"s{i}_out"])
            assert out.dtype == ref.dtype and out.shape == ref.shape
            assert max_rel_err(out, ref) < tol, (name, i, max_rel_err(out, ref))
        assert max_rel_err(a.window, _t(z[f"window_{i + 1}"])) < tol, (name, i)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_matches_oracle_at_larger_widths(dtype, attn_kernel):
    """dim 1024, 16 heads of 128 (rope 64), q rank 256, 4 output groups of rank 128, a 32-slot
    window, 4 sequences x 7 draft positions; prefill of 40 positions, then 3 decode steps."""
    if attn_kernel == 0 and dtype == torch.float32:
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    g = torch.Generator().manual_seed(7)
    dims = dict(dim=1024, n_heads=16, head_dim=128, rope_head_dim=64, q_lora_rank=256, o_groups=4, o_lora_rank=128,
                window_size=32, norm_eps=1e-6, rope_theta=10000.0)
    d, h, hd, ql, og, orank = 1024, 16, 128, 256, 4, 128
    r = lambda *s, std: (torch.randn(*s, generator=g) * std).to(dtype)  # noqa: E731
    w = {"wq_a": r(ql, d, std=d ** -0.5), "wq_b": r(h * hd, ql, std=ql ** -0.5), "wkv": r(hd, d, std=d ** -0.5),
         "wo_a": r(og * orank, h * hd // og, std=(h * hd // og) ** -0.5), "wo_b": r(d, og * orank, std=0.05),
         "q_norm": 1 + 0.1 * torch.randn(ql, generator=g), "kv_norm": 1 + 0.1 * torch.randn(hd, generator=g),
         "attn_sink": torch.randn(h, generator=g)}
    a = _module(dims, w)
    od = AttnDims(n_heads=h, head_dim=hd, rope_head_dim=64, o_groups=og, o_lora_rank=orank, window_size=32, eps=1e-6)
    cos, sin = oracle.rope_tables(64, 64, 10000.0)
    cache = oracle.KVWindow(32)
    b, blk = 4, 7
    main = torch.randn(b, 40, d, generator=g).to(dtype)
    x0 = torch.randn(b, blk, d, generator=g).to(dtype)
    a(x0.to(DEV), 0, main.to(DEV))
    oracle.attention_forward(w, od, x0, 0, main, cache, cos, sin)
    tol = 2e-2 if dtype == torch.bfloat16 else 2e-3
    assert max_rel_err(a.window, cache.window) < tol
    pos = 40
    for step in range(3):
        mx1 = torch.randn(b, 1, d, generator=g).to(dtype)
        xs = torch.randn(b, blk, d, generator=g).to(dtype)
        out = a(xs.to(DEV), pos, mx1.to(DEV))
        ref = oracle.attention_forward(w, od, xs, pos, mx1, cache, cos, sin)
        torch.cuda.synchronize()
        assert max_rel_err(out, ref) < tol, (step, max_rel_err(out, ref))
        assert max_rel_err(a.window, cache.window) < tol
        pos += 1
    assert _lib.device_error() == 0
