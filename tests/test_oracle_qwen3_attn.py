"""The oracle's restatement of the Qwen3 DSpark draft attention against golden vectors from the
reference's own ``Qwen3DSparkAttention`` (``dspark_mlx/arch/qwen3.py:84-143``): the full path
over ``[context || block]``, the cached context K/V built in two appends, and the cached
attention with and without a context; and the whole draft layer (``Qwen3DSparkLayer``,
``qwen3.py:157-176``) on both paths (``tests/golden/make_golden_qwen3_attn.py``)."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_attn_*.npz")))
LAYER_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_layer_*.npz")))
BACKBONE_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_backbone_*.npz")))
LAYER_KEYS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "q_norm", "k_norm",
              "input_layernorm", "post_attention_layernorm")
DIMS = dict(nh=4, nkv=2, hd=32, eps=1e-6, theta=1000000.0)


def _t(a):
    return torch.from_numpy(a).view(torch.bfloat16) if a.dtype == np.int16 else torch.from_numpy(a)


def _weights(z):
    p = {k: _t(z[k]) for k in ("q_proj", "k_proj", "v_proj", "o_proj")}
    p.update(q_norm=_t(z["q_norm"]), k_norm=_t(z["k_norm"]))
    return p


def test_golden_cases_exist():
    assert len(CASES) == 2 and len(LAYER_CASES) == 2 and len(BACKBONE_CASES) == 1


def backbone_tensors(z):
    return {k: _t(v) for k, v in z.items() if k.endswith(".weight")}


@pytest.mark.parametrize("name", BACKBONE_CASES)
def test_backbone_oracle_matches_reference_goldens(name):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    t = backbone_tensors(z)
    nh, nkv, hd, eps, theta = (DIMS[k] for k in ("nh", "nkv", "hd", "eps", "theta"))
    tctx = oracle.qwen3_project_context(t, eps, _t(z["target_hidden"]))
    assert torch.equal(tctx, _t(z["target_ctx"]))
    noise = _t(z["noise_embed"])
    q, ctx = noise.shape[1], tctx.shape[1]
    n_layers = len({k.split(".")[1] for k in t if k.startswith("layers.")})
    cos, sin = oracle.qwen3_rope_tables(torch.arange(ctx + q), hd, theta)
    out = oracle.qwen3_backbone(t, n_layers, nh, nkv, hd, eps, noise, tctx, cos, sin)
    assert torch.equal(out, _t(z["full_out"]))


@pytest.mark.parametrize("name", LAYER_CASES)
def test_layer_oracle_matches_reference_goldens(name):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    p = {k: _t(z[k]) for k in LAYER_KEYS}
    nh, nkv, hd, eps, theta = (DIMS[k] for k in ("nh", "nkv", "hd", "eps", "theta"))
    hidden, target = _t(z["hidden"]), _t(z["target_ctx"])
    q, ctx = hidden.shape[1], target.shape[1]
    cos, sin = oracle.qwen3_rope_tables(torch.arange(ctx + q), hd, theta)
    full = oracle.qwen3_layer(p, nh, nkv, hd, eps, hidden, target, cos, sin)
    assert full.dtype == hidden.dtype and torch.equal(full, _t(z["full_out"]))
    c, s = oracle.qwen3_rope_tables(torch.arange(ctx), hd, theta)
    ck, cv = oracle.qwen3_context_kv(p, nkv, hd, eps, target, c, s)
    c, s = oracle.qwen3_rope_tables(torch.arange(ctx, ctx + q), hd, theta)
    assert torch.equal(oracle.qwen3_layer_cached(p, nh, nkv, hd, eps, hidden, ck, cv, c, s), _t(z["cached_out"]))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_goldens(name):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    p = _weights(z)
    nh, nkv, hd, eps, theta = (DIMS[k] for k in ("nh", "nkv", "hd", "eps", "theta"))
    hidden, target = _t(z["hidden"]), _t(z["target_ctx"])
    b, q, _ = hidden.shape
    ctx = target.shape[1]
    cos, sin = oracle.qwen3_rope_tables(torch.arange(ctx + q), hd, theta)
    # the same torch operations in the same order as the reference run: bit-identical
    assert torch.equal(cos, _t(z["cos_full"])) and torch.equal(sin, _t(z["sin_full"]))
    full = oracle.qwen3_attention(p, nh, nkv, hd, eps, hidden, target, cos, sin)
    assert full.dtype == hidden.dtype and torch.equal(full, _t(z["full_out"]))

    split = {5: 2, 13: 9}[ctx]
    ks, vs = [], []
    for lo, hi in ((0, split), (split, ctx)):
        c, s = oracle.qwen3_rope_tables(torch.arange(lo, hi), hd, theta)
        k, v = oracle.qwen3_context_kv(p, nkv, hd, eps, target[:, lo:hi], c, s)
        ks.append(k)
        vs.append(v)
    ctx_k, ctx_v = torch.cat(ks, dim=2), torch.cat(vs, dim=2)
    assert torch.equal(ctx_k, _t(z["ctx_k"])) and torch.equal(ctx_v, _t(z["ctx_v"]))
    c, s = oracle.qwen3_rope_tables(torch.arange(ctx, ctx + q), hd, theta)
    cached = oracle.qwen3_attend_cached(p, nh, nkv, hd, eps, hidden, ctx_k, ctx_v, c, s)
    assert torch.equal(cached, _t(z["cached_out"]))
    c0, s0 = oracle.qwen3_rope_tables(torch.arange(q), hd, theta)
    assert torch.equal(oracle.qwen3_attend_cached(p, nh, nkv, hd, eps, hidden, None, None, c0, s0),
                       _t(z["nocontext_out"]))


@pytest.mark.parametrize("name", CASES)
def test_cached_path_equals_full_path_up_to_rounding(name):
    """Caching post-RoPE context K/V is the full path's computation split in two
    (``qwen3.py:118-120``): the two agree to a few bf16 ulps (the block's q sits at the same
    positions, only the K rows are taken from separate projections)."""
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    full, cached = _t(z["full_out"]).float(), _t(z["cached_out"]).float()
    tol = 2e-2 if bool(z["dtype_bf16"]) else 1e-5
    assert (full - cached).abs().max() <= tol * full.abs().max()
