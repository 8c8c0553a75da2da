"""The Qwen3 DSpark draft layer on the GPU (``dsm.qwen3_layer``) against golden vectors from the
reference's own ``Qwen3DSparkLayer`` (``tests/golden/make_golden_qwen3_attn.py``) and against
the oracle at the Qwen3-4B draft layer's widths.

Tolerances are max|out - ref| / max|ref|:
* bf16 allows 2e-2, as for the attention alone.
* fp32 allows 5e-3: the MLP stages its fp32 input as one f16 row (2^-11 relative), and fp32
  weights are held as f16 (2^-12)."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle
from dsm import _lib
from dsm.qwen3_attention import rope_tables
from dsm.qwen3_layer import Qwen3DSparkLayer
from helpers import max_rel_err
from test_oracle_qwen3_attn import DIMS, HERE, LAYER_KEYS, _t

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_layer_*.npz")))


def _layer(args: dict, w: dict) -> Qwen3DSparkLayer:
    layer = Qwen3DSparkLayer(args).to(DEV)
    for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(layer.self_attn, k).weight = torch.nn.Parameter(w[k].to(DEV), requires_grad=False)
    for k in ("gate_proj", "up_proj", "down_proj"):
        getattr(layer.mlp, k).weight = torch.nn.Parameter(w[k].to(DEV), requires_grad=False)
    with torch.no_grad():
        layer.self_attn.q_norm.weight.copy_(w["q_norm"])
        layer.self_attn.k_norm.weight.copy_(w["k_norm"])
        layer.input_layernorm.weight.copy_(w["input_layernorm"])
        layer.post_attention_layernorm.weight.copy_(w["post_attention_layernorm"])
    return layer


@pytest.mark.parametrize("name", CASES)
def test_qwen3_layer_matches_reference_goldens(name, attn_kernel):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    if attn_kernel == 0 and not bool(z["dtype_bf16"]):
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    tol = 2e-2 if bool(z["dtype_bf16"]) else 5e-3
    w = {k: _t(z[k]) for k in LAYER_KEYS}
    inter = w["gate_proj"].shape[0]
    args = dict(hidden_size=96, num_attention_heads=DIMS["nh"], num_key_value_heads=DIMS["nkv"], head_dim=DIMS["hd"],
                rms_norm_eps=DIMS["eps"], intermediate_size=inter)
    layer = _layer(args, w)
    hidden, target = _t(z["hidden"]), _t(z["target_ctx"])
    q, ctx = hidden.shape[1], target.shape[1]
    hd, theta = DIMS["hd"], DIMS["theta"]
    full = layer(hidden.to(DEV), target.to(DEV), *rope_tables(torch.arange(ctx + q), hd, theta))
    ck, cv = layer.context_kv(target.to(DEV), *rope_tables(torch.arange(ctx), hd, theta))
    cached = layer.forward_cached(hidden.to(DEV), ck, cv, *rope_tables(torch.arange(ctx, ctx + q), hd, theta))
    torch.cuda.synchronize()
    ref_full, ref_cached = _t(z["full_out"]), _t(z["cached_out"])
    assert full.dtype == ref_full.dtype and full.shape == ref_full.shape
    assert max_rel_err(full, ref_full) < tol, (name, max_rel_err(full, ref_full))
    assert max_rel_err(cached, ref_cached) < tol, (name, max_rel_err(cached, ref_cached))
    assert _lib.device_error() == 0


def test_qwen3_layer_matches_oracle_at_qwen3_4b_widths(attn_kernel):
    """hidden 2560, MLP 9728, 32 query / 8 KV heads of 128; 2 sequences x 7 block tokens over
    256 cached context rows, bf16."""
    g = torch.Generator().manual_seed(5)
    h, inter, nh, nkv, hd, b, q, ctx = 2560, 9728, 32, 8, 128, 2, 7, 256
    r = lambda *s, std: (torch.randn(*s, generator=g) * std).to(torch.bfloat16)  # noqa: E731
    w = {"q_proj": r(nh * hd, h, std=h ** -0.5), "k_proj": r(nkv * hd, h, std=h ** -0.5),
         "v_proj": r(nkv * hd, h, std=h ** -0.5), "o_proj": r(h, nh * hd, std=(nh * hd) ** -0.5),
         "gate_proj": r(inter, h, std=h ** -0.5), "up_proj": r(inter, h, std=h ** -0.5),
         "down_proj": r(h, inter, std=inter ** -0.5),
         "q_norm": 1 + 0.1 * torch.randn(hd, generator=g), "k_norm": 1 + 0.1 * torch.randn(hd, generator=g),
         "input_layernorm": 1 + 0.1 * torch.randn(h, generator=g),
         "post_attention_layernorm": 1 + 0.1 * torch.randn(h, generator=g)}
    args = dict(hidden_size=h, num_attention_heads=nh, num_key_value_heads=nkv, head_dim=hd, rms_norm_eps=1e-6,
                intermediate_size=inter)
    layer = _layer(args, w)
    hidden = torch.randn(b, q, h, generator=g).to(torch.bfloat16)
    target = torch.randn(b, ctx, h, generator=g).to(torch.bfloat16)
    c, s = rope_tables(torch.arange(ctx), hd, 1e6)
    ck, cv = layer.context_kv(target.to(DEV), c, s)
    cb, sb = rope_tables(torch.arange(ctx, ctx + q), hd, 1e6)
    out = layer.forward_cached(hidden.to(DEV), ck, cv, cb, sb)
    torch.cuda.synchronize()
    rk, rv = oracle.qwen3_context_kv(w, nkv, hd, 1e-6, target, c, s)
    ref = oracle.qwen3_layer_cached(w, nh, nkv, hd, 1e-6, hidden, rk, rv, cb, sb)
    assert max_rel_err(out, ref) < 2e-2, max_rel_err(out, ref)
    assert _lib.device_error() == 0


BACKBONE_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "qwen3_backbone_*.npz")))


@pytest.mark.parametrize("name", BACKBONE_CASES)
def test_qwen3_backbone_matches_reference_goldens(name):
    """``Qwen3Backbone``: the context projection, two layers and the final norm (bf16, 2e-2)."""
    from dsm.qwen3_layer import Qwen3Backbone

    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    t = {k: _t(v) for k, v in z.items() if k.endswith(".weight")}
    n_layers = len({k.split(".")[1] for k in t if k.startswith("layers.")})
    fc_in = t["fc.weight"].shape[1]
    inter = t["layers.0.mlp.gate_proj.weight"].shape[0]
    args = dict(hidden_size=96, num_attention_heads=DIMS["nh"], num_key_value_heads=DIMS["nkv"], head_dim=DIMS["hd"],
                rms_norm_eps=DIMS["eps"], intermediate_size=inter, num_hidden_layers=n_layers,
                target_layer_ids=list(range(fc_in // 96)))
    bb = Qwen3Backbone(args).to(DEV)
    for name_, v in t.items():
        *path, leaf = name_.split(".")
        obj = bb
        for part in path:
            obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
        if leaf == "weight" and isinstance(obj, torch.nn.Module) and v.dtype == torch.float32 and v.dim() == 1:
            with torch.no_grad():
                obj.weight.copy_(v)  # norm weights (fp32)
        else:
            setattr(obj, leaf, torch.nn.Parameter(v.to(DEV), requires_grad=False))
    tctx = bb.project_context(_t(z["target_hidden"]).to(DEV))
    noise = _t(z["noise_embed"])
    q, ctx = noise.shape[1], tctx.shape[1]
    out = bb(noise.to(DEV), tctx, *rope_tables(torch.arange(ctx + q), DIMS["hd"], DIMS["theta"]))
    torch.cuda.synchronize()
    assert max_rel_err(tctx, _t(z["target_ctx"])) < 2e-2
    ref = _t(z["full_out"])
    assert out.dtype == ref.dtype and max_rel_err(out, ref) < 2e-2, max_rel_err(out, ref)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_add_rms_norm_entry_point(dtype):
    """``dsm_add_rms_norm`` through the C ABI: s = x + delta rounded once, y = RMSNorm(s) * w, each
    output optional; against the oracle's add and RMSNorm (bf16 within one rounding, fp32 1e-6)."""
    from dsm._lib import dtype_code, lib, ptr, stream_ptr

    g = torch.Generator().manual_seed(3)
    n, dim = 37, 2560
    x = torch.randn(n, dim, generator=g).to(dtype)
    d = torch.randn(n, dim, generator=g).to(dtype)
    w = 1 + 0.1 * torch.randn(dim, generator=g)
    xs, ds, ws = x.to(DEV), d.to(DEV), w.to(DEV)
    s, y, y0 = torch.empty_like(xs), torch.empty_like(xs), torch.empty_like(xs)
    L = lib()
    _lib.check(L.dsm_add_rms_norm(ptr(xs), ptr(ds), dtype_code(dtype), n, dim, ptr(ws), 1e-6, ptr(s), ptr(y),
                                  stream_ptr()), "dsm_add_rms_norm")
    _lib.check(L.dsm_add_rms_norm(ptr(xs), None, dtype_code(dtype), n, dim, ptr(ws), 1e-6, None, ptr(y0),
                                  stream_ptr()), "dsm_add_rms_norm")
    torch.cuda.synchronize()
    ref_s = (x.float() + d.float()).to(dtype)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-6
    assert torch.equal(s.cpu(), ref_s)
    assert max_rel_err(y, oracle.rms_norm(ref_s, w, 1e-6)) < tol
    assert max_rel_err(y0, oracle.rms_norm(x, w, 1e-6)) < tol
