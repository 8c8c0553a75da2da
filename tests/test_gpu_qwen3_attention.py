"""The Qwen3 DSpark draft attention on the GPU (``dsm.qwen3_attention``) against golden vectors
from the reference's own ``Qwen3DSparkAttention`` (``tests/golden/make_golden_qwen3_attn.py``)
and against the oracle at the Qwen3-4B draft layer's widths.

Tolerances are max|out - ref| / max|ref|:
* bf16 allows 2e-2: q, k, v and o round to bf16 after fp32 sums taken in another order, and
  the attention's softmax runs in another order.
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
from dsm.qwen3_attention import Qwen3DSparkAttention, rope_tables
from helpers import max_rel_err
from test_oracle_qwen3_attn import DIMS, HERE, _t, _weights

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_attn_*.npz")))


def _module(args: dict, w: dict) -> Qwen3DSparkAttention:
    a = Qwen3DSparkAttention(args).to(DEV)
    for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(a, k).weight = torch.nn.Parameter(w[k].to(DEV), requires_grad=False)
    with torch.no_grad():
        a.q_norm.weight.copy_(w["q_norm"])
        a.k_norm.weight.copy_(w["k_norm"])
    return a


def _golden_args():
    return dict(hidden_size=96, num_attention_heads=DIMS["nh"], num_key_value_heads=DIMS["nkv"], head_dim=DIMS["hd"],
                rms_norm_eps=DIMS["eps"])


@pytest.mark.parametrize("name", CASES)
def test_qwen3_attention_matches_reference_goldens(name, attn_kernel):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    if attn_kernel == 0 and not bool(z["dtype_bf16"]):
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    tol = 2e-2 if bool(z["dtype_bf16"]) else 2e-3
    a = _module(_golden_args(), _weights(z))
    hidden, target = _t(z["hidden"]), _t(z["target_ctx"])
    b, q, _ = hidden.shape
    ctx = target.shape[1]
    hd, theta = DIMS["hd"], DIMS["theta"]
    cos, sin = rope_tables(torch.arange(ctx + q), hd, theta)
    full = a(hidden.to(DEV), target.to(DEV), cos, sin)
    torch.cuda.synchronize()
    ref = _t(z["full_out"])
    assert full.dtype == ref.dtype and full.shape == ref.shape
    assert max_rel_err(full, ref) < tol, (name, max_rel_err(full, ref))

    # the cached form: the context in two appends into preallocated caches, then the block
    split = {5: 2, 13: 9}[ctx]
    kc = torch.zeros(b, DIMS["nkv"], ctx + 3, hd, dtype=hidden.dtype, device=DEV)
    vc = torch.zeros_like(kc)
    for lo, hi in ((0, split), (split, ctx)):
        c, s = rope_tables(torch.arange(lo, hi), hd, theta)
        a.context_kv(target[:, lo:hi].to(DEV), c, s, out=(kc, vc), row0=lo)
    torch.cuda.synchronize()
    assert max_rel_err(kc[:, :, :ctx], _t(z["ctx_k"])) < tol
    assert max_rel_err(vc[:, :, :ctx], _t(z["ctx_v"])) < tol
    c, s = rope_tables(torch.arange(ctx, ctx + q), hd, theta)
    cached = a.attend_cached(hidden.to(DEV), kc[:, :, :ctx], vc[:, :, :ctx], c, s)
    k2, v2 = a.context_kv(target.to(DEV), *rope_tables(torch.arange(ctx), hd, theta))  # one call, fresh tensors
    cached2 = a.attend_cached(hidden.to(DEV), k2, v2, c, s)
    c0, s0 = rope_tables(torch.arange(q), hd, theta)
    alone = a.attend_cached(hidden.to(DEV), None, None, c0, s0)
    torch.cuda.synchronize()
    assert max_rel_err(cached, _t(z["cached_out"])) < tol
    assert max_rel_err(cached2, _t(z["cached_out"])) < tol
    assert max_rel_err(alone, _t(z["nocontext_out"])) < tol
    assert _lib.device_error() == 0


def _oracle_case(dtype, b, q, ctx, h, nh, nkv, hd, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, std: (torch.randn(*s, generator=g) * std).to(dtype)  # noqa: E731
    w = {"q_proj": r(nh * hd, h, std=h ** -0.5), "k_proj": r(nkv * hd, h, std=h ** -0.5),
         "v_proj": r(nkv * hd, h, std=h ** -0.5), "o_proj": r(h, nh * hd, std=(nh * hd) ** -0.5),
         "q_norm": 1 + 0.1 * torch.randn(hd, generator=g), "k_norm": 1 + 0.1 * torch.randn(hd, generator=g)}
    hidden = torch.randn(b, q, h, generator=g).to(dtype)
    target = torch.randn(b, ctx, h, generator=g).to(dtype)
    return w, hidden, target


def test_qwen3_attention_8bit_projections_match_oracle(attn_kernel):
    """Projections quantised as quantize_drafter leaves them (MLX affine, 8 bits, groups of 64)
    run split along K (dsm_linear_splitk). The oracle multiplies by the dequantised weights in
    fp32; the GPU's bf16 activations round after every product."""
    from oracle.formats import affine_dequantize

    dtype, b, q, ctx, h, nh, nkv, hd = torch.bfloat16, 2, 7, 300, 2560, 32, 8, 128
    theta, eps = 1000000.0, 1e-6
    w, hidden, target = _oracle_case(dtype, b, q, ctx, h, nh, nkv, hd, seed=11)
    a = _module(dict(hidden_size=h, num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd, rms_norm_eps=eps),
                w)
    wd = dict(w)
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        proj = getattr(a, n)
        assert proj.quantize(bits=8, group_size=64)
        wd[n] = affine_dequantize(proj.q.cpu(), proj.scales.cpu(), proj.biases.cpu(), 64, 8)
    cos, sin = rope_tables(torch.arange(ctx + q), hd, theta)
    out = a(hidden.to(DEV), target.to(DEV), cos, sin)
    torch.cuda.synchronize()
    ref = oracle.qwen3_attention(wd, nh, nkv, hd, eps, hidden.float(), target.float(), cos, sin)
    assert out.dtype == torch.bfloat16
    assert max_rel_err(out, ref) < 2e-2, max_rel_err(out, ref)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dtype,b,q,ctx,h,nh,nkv,hd", [
    (torch.bfloat16, 2, 7, 2048, 2560, 32, 8, 128),   # the Qwen3-4B draft layer, 2048 context rows
    (torch.bfloat16, 3, 7, 333, 1024, 16, 2, 64),     # 8 heads per KV head: 56 query rows, two row blocks
    (torch.float32, 1, 5, 1000, 512, 4, 1, 256),      # head_dim 256, one KV head
    (torch.bfloat16, 4, 7, 0, 512, 8, 4, 128),        # no context at all
])
def test_qwen3_attention_matches_oracle(dtype, b, q, ctx, h, nh, nkv, hd, attn_kernel):
    if attn_kernel == 0 and not dtype == torch.bfloat16:
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    theta, eps = 1000000.0, 1e-6
    w, hidden, target = _oracle_case(dtype, b, q, ctx, h, nh, nkv, hd, seed=ctx + hd)
    a = _module(dict(hidden_size=h, num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd, rms_norm_eps=eps),
                w)
    cos, sin = rope_tables(torch.arange(ctx + q), hd, theta)
    out = a(hidden.to(DEV), target.to(DEV), cos, sin)
    torch.cuda.synchronize()
    ref = oracle.qwen3_attention(w, nh, nkv, hd, eps, hidden, target, cos, sin)
    tol = 2e-2 if dtype == torch.bfloat16 else 2e-3
    assert max_rel_err(out, ref) < tol, max_rel_err(out, ref)
    if ctx:
        k, v = a.context_kv(target.to(DEV), cos[:ctx], sin[:ctx])
        rk, rv = oracle.qwen3_context_kv(w, nkv, hd, eps, target, cos[:ctx], sin[:ctx])
        torch.cuda.synchronize()
        assert max_rel_err(k, rk) < tol and max_rel_err(v, rv) < tol
    assert _lib.device_error() == 0


def test_qwen3_attention_context_order_invariance_at_bench_shape(attn_kernel):
    """At the bench's shape (16 sequences x 7 block tokens over 2048 cached context rows,
    Qwen3-4B widths) the CPU oracle is too slow, so a size-independent property stands in:
    attention over the cached rows does not depend on their order. Permuting the context rows
    (K and V alike) moves them across the kernel's key ranges and tiles; the output must agree
    to bf16 rounding of the same sums in another order."""
    from dsm import workloads as W

    wl = W.WORKLOADS["qwen3_attn_q8"]
    t = W.make_gqa_tensors(wl, device=DEV, seed=3)
    attn = W.build_gqa(wl, t, DEV)
    a = wl.args
    s, ctx = wl.block, wl.extra["ctx"]
    cos, sin = rope_tables(torch.arange(ctx, ctx + s), a["head_dim"], a["rope_theta"])
    kc, vc = t["ctx_k"], t["ctx_v"]
    perm = torch.randperm(ctx, generator=torch.Generator().manual_seed(1)).to(DEV)
    y0 = attn.attend_cached(t["x"], kc, vc, cos, sin)
    y1 = attn.attend_cached(t["x"], kc[:, :, perm].contiguous(), vc[:, :, perm].contiguous(), cos, sin)
    torch.cuda.synchronize()
    assert torch.isfinite(y0.float()).all()
    assert max_rel_err(y1, y0) < 1e-2, max_rel_err(y1, y0)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("ctx", [2048, 2011, 25])
def test_qwen3_attention_kernels_agree(ctx):
    """The tensor-core kernel (gqa_mma_kernel) against the CUDA-core one on the same inputs at
    Qwen3-4B widths: 2048 context rows (the bench shape), 2011 (the last 64-key tile of each
    range partly filled) and 25 (with the 7 block rows, one tile of 32 keys: the second key half
    of every tile is empty). The tensor-core kernel rounds the softmax weights to bf16 for the
    p.v products and sums the same rounded weights in the denominator, so the two agree to a
    few bf16 ulps of the output."""
    from dsm import workloads as W

    L = _lib.lib()
    wl = W.WORKLOADS["qwen3_attn_q8"]
    t = W.make_gqa_tensors(wl, device=DEV, seed=5)
    attn = W.build_gqa(wl, t, DEV)
    a = wl.args
    s = wl.block
    cos, sin = rope_tables(torch.arange(ctx, ctx + s), a["head_dim"], a["rope_theta"])
    kc, vc = t["ctx_k"][:, :, :ctx], t["ctx_v"][:, :, :ctx]
    outs = []
    for k in (1, 0):
        _lib.check(L.dsm_set_attn_kernel(k))
        try:
            outs.append(attn.attend_cached(t["x"], kc, vc, cos, sin))
            torch.cuda.synchronize()
        finally:
            _lib.check(L.dsm_set_attn_kernel(_lib.ATTN_KERNEL_DEFAULT))
    assert torch.isfinite(outs[1].float()).all()
    assert max_rel_err(outs[1], outs[0]) < 1e-2, max_rel_err(outs[1], outs[0])
    assert _lib.device_error() == 0
