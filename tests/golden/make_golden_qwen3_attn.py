"""Generate golden vectors for the Qwen3 DSpark draft attention by running the reference's
own ``Qwen3DSparkAttention`` (``dspark_mlx/arch/qwen3.py``, RMSNorm from
``dspark_mlx/model/norm_rope.py``) on seeded inputs and weights, with the ``mlx`` API served
by ``mlx_torch_shim``. Each case records
* the full path ``attn(hidden, target_ctx, cos_full, sin_full)`` over contiguous positions
  ``0 .. ctx + block - 1``;
* the cached path: ``context_kv`` of the committed context in two pieces (as
  ``extend_context`` appends them), then ``attend_cached`` of the block at its own absolute
  positions, and ``attend_cached`` with no context at all.
Layer cases run the whole ``Qwen3DSparkLayer`` (``qwen3.py:157-176``: RMSNorms, residual adds,
the attention and the MLP) on the full and the cached path; backbone cases run
``Qwen3Backbone`` (``qwen3.py:178-197``: the context projection, the layers, the final norm).
Everything goes to ``qwen3_attn_*.npz`` / ``qwen3_layer_*.npz`` / ``qwen3_backbone_*.npz``
next to this script; the tests read only the fixtures.

    python tests/golden/make_golden_qwen3_attn.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import mlx_torch_shim as shim  # noqa: E402

DIMS = dict(hidden_size=96, num_attention_heads=4, num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6,
            rope_theta=1000000.0)
CASES = {
    # dtype, batch, block, committed context length, split of the context into two appends
    "qwen3_attn_bf16_b2_c13": dict(dtype=torch.bfloat16, b=2, block=7, ctx=13, split=9),
    "qwen3_attn_f32_b3_c5": dict(dtype=torch.float32, b=3, block=4, ctx=5, split=2),
}


def load_reference(ref_root: str):
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model"),
                      ("dspark_mlx.arch", "dspark_mlx/arch")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    return importlib.import_module("dspark_mlx.arch.qwen3")


def build_case(q3, spec: dict, rng) -> dict:
    mx = shim
    dt = spec["dtype"]
    args = q3.Qwen3DSparkArgs.from_dict(dict(DIMS))
    attn = q3.Qwen3DSparkAttention(args)
    h, nh, nkv, hd = (DIMS[k] for k in ("hidden_size", "num_attention_heads", "num_key_value_heads", "head_dim"))

    def w(*shape, std):
        return torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(dt)

    weights = {"q_proj": w(nh * hd, h, std=h ** -0.5), "k_proj": w(nkv * hd, h, std=h ** -0.5),
               "v_proj": w(nkv * hd, h, std=h ** -0.5), "o_proj": w(h, nh * hd, std=(nh * hd) ** -0.5)}
    norms = {"q_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
             "k_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)}
    for k, v in weights.items():
        getattr(attn, k).weight = mx.array(v)
    attn.q_norm.weight = mx.array(norms["q_norm"])
    attn.k_norm.weight = mx.array(norms["k_norm"])

    def raw(t):
        tt = t.t if isinstance(t, shim.array) else t
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.to(torch.float32).numpy()

    b, block, ctx, split = spec["b"], spec["block"], spec["ctx"], spec["split"]
    out = {"dtype_bf16": np.array(dt == torch.bfloat16), **{k: raw(v) for k, v in weights.items()}, **norms}
    hidden = torch.from_numpy(rng.standard_normal((b, block, h)).astype(np.float32)).to(dt)
    target = torch.from_numpy(rng.standard_normal((b, ctx, h)).astype(np.float32)).to(dt)
    out["hidden"], out["target_ctx"] = raw(hidden), raw(target)

    cos, sin = q3.rope_tables(mx.arange(ctx + block), hd, DIMS["rope_theta"])
    out["cos_full"], out["sin_full"] = raw(cos), raw(sin)
    out["full_out"] = raw(attn(mx.array(hidden), mx.array(target), cos, sin))

    ks, vs = [], []
    for lo, hi in ((0, split), (split, ctx)):
        c, s = q3.rope_tables(mx.arange(lo, hi), hd, DIMS["rope_theta"])
        k, v = attn.context_kv(mx.array(target[:, lo:hi]), c, s)
        ks.append(k)
        vs.append(v)
    ctx_k, ctx_v = mx.concatenate(ks, axis=2), mx.concatenate(vs, axis=2)
    out["ctx_k"], out["ctx_v"] = raw(ctx_k), raw(ctx_v)
    c, s = q3.rope_tables(mx.arange(ctx, ctx + block), hd, DIMS["rope_theta"])
    out["cached_out"] = raw(attn.attend_cached(mx.array(hidden), ctx_k, ctx_v, c, s))
    c0, s0 = q3.rope_tables(mx.arange(0, block), hd, DIMS["rope_theta"])
    out["nocontext_out"] = raw(attn.attend_cached(mx.array(hidden), None, None, c0, s0))
    return out


LAYER_CASES = {
    "qwen3_layer_bf16_b2_c9": dict(dtype=torch.bfloat16, b=2, block=7, ctx=9, inter=160),
    "qwen3_layer_f32_b1_c4": dict(dtype=torch.float32, b=1, block=3, ctx=4, inter=64),
}


def build_layer_case(q3, spec: dict, rng) -> dict:
    mx = shim
    dt = spec["dtype"]
    args = q3.Qwen3DSparkArgs.from_dict(dict(DIMS, intermediate_size=spec["inter"]))
    layer = q3.Qwen3DSparkLayer(args)
    h, nh, nkv, hd = (DIMS[k] for k in ("hidden_size", "num_attention_heads", "num_key_value_heads", "head_dim"))
    inter = spec["inter"]

    def w(*shape, std):
        return torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(dt)

    weights = {"q_proj": w(nh * hd, h, std=h ** -0.5), "k_proj": w(nkv * hd, h, std=h ** -0.5),
               "v_proj": w(nkv * hd, h, std=h ** -0.5), "o_proj": w(h, nh * hd, std=(nh * hd) ** -0.5),
               "gate_proj": w(inter, h, std=h ** -0.5), "up_proj": w(inter, h, std=h ** -0.5),
               "down_proj": w(h, inter, std=inter ** -0.5)}
    norms = {"q_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
             "k_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
             "input_layernorm": (1 + 0.1 * rng.standard_normal(h)).astype(np.float32),
             "post_attention_layernorm": (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)}
    for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(layer.self_attn, k).weight = mx.array(weights[k])
    for k in ("gate_proj", "up_proj", "down_proj"):
        getattr(layer.mlp, k).weight = mx.array(weights[k])
    layer.self_attn.q_norm.weight = mx.array(norms["q_norm"])
    layer.self_attn.k_norm.weight = mx.array(norms["k_norm"])
    layer.input_layernorm.weight = mx.array(norms["input_layernorm"])
    layer.post_attention_layernorm.weight = mx.array(norms["post_attention_layernorm"])

    def raw(t):
        tt = t.t if isinstance(t, shim.array) else t
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.to(torch.float32).numpy()

    b, block, ctx = spec["b"], spec["block"], spec["ctx"]
    out = {"dtype_bf16": np.array(dt == torch.bfloat16), **{k: raw(v) for k, v in weights.items()}, **norms}
    hidden = torch.from_numpy(rng.standard_normal((b, block, h)).astype(np.float32)).to(dt)
    target = torch.from_numpy(rng.standard_normal((b, ctx, h)).astype(np.float32)).to(dt)
    out["hidden"], out["target_ctx"] = raw(hidden), raw(target)
    cos, sin = q3.rope_tables(mx.arange(ctx + block), hd, DIMS["rope_theta"])
    out["full_out"] = raw(layer(mx.array(hidden), mx.array(target), cos, sin))
    c, s = q3.rope_tables(mx.arange(ctx), hd, DIMS["rope_theta"])
    ck, cv = layer.context_kv(mx.array(target), c, s)
    c, s = q3.rope_tables(mx.arange(ctx, ctx + block), hd, DIMS["rope_theta"])
    out["cached_out"] = raw(layer.forward_cached(mx.array(hidden), ck, cv, c, s))
    return out


BACKBONE_CASES = {
    "qwen3_backbone_bf16_b2_c6": dict(dtype=torch.bfloat16, b=2, block=7, ctx=6, inter=160, layers=2, targets=3),
}


def build_backbone_case(q3, spec: dict, rng) -> dict:
    """``Qwen3Backbone`` (``qwen3.py:178-197``): project_context, then the layers and the norm."""
    mx = shim
    dt = spec["dtype"]
    args = q3.Qwen3DSparkArgs.from_dict(dict(DIMS, intermediate_size=spec["inter"], num_hidden_layers=spec["layers"],
                                             target_layer_ids=list(range(spec["targets"]))))
    bb = q3.Qwen3Backbone(args)
    h, nh, nkv, hd = (DIMS[k] for k in ("hidden_size", "num_attention_heads", "num_key_value_heads", "head_dim"))
    inter, fc_in = spec["inter"], h * spec["targets"]

    def w(*shape, std):
        return torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(dt)

    def norm(n):
        return (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    def raw(t):
        tt = t.t if isinstance(t, shim.array) else t
        if isinstance(tt, np.ndarray):
            return tt
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.to(torch.float32).numpy()

    out = {"dtype_bf16": np.array(dt == torch.bfloat16)}
    t = {"fc.weight": w(h, fc_in, std=fc_in ** -0.5), "hidden_norm.weight": norm(h), "norm.weight": norm(h)}
    for i in range(spec["layers"]):
        p = f"layers.{i}."
        t.update({p + "self_attn.q_proj.weight": w(nh * hd, h, std=h ** -0.5),
                  p + "self_attn.k_proj.weight": w(nkv * hd, h, std=h ** -0.5),
                  p + "self_attn.v_proj.weight": w(nkv * hd, h, std=h ** -0.5),
                  p + "self_attn.o_proj.weight": w(h, nh * hd, std=(nh * hd) ** -0.5),
                  p + "self_attn.q_norm.weight": norm(hd), p + "self_attn.k_norm.weight": norm(hd),
                  p + "mlp.gate_proj.weight": w(inter, h, std=h ** -0.5), p + "mlp.up_proj.weight": w(inter, h, std=h ** -0.5),
                  p + "mlp.down_proj.weight": w(h, inter, std=inter ** -0.5),
                  p + "input_layernorm.weight": norm(h), p + "post_attention_layernorm.weight": norm(h)})
    for name, v in t.items():
        *path, leaf = name.split(".")
        obj = bb
        for part in path:
            obj = obj[int(part)] if isinstance(obj, list) else getattr(obj, part)
        setattr(obj, leaf, mx.array(v))
    out.update({k: raw(v) for k, v in t.items()})
    b, block, ctx = spec["b"], spec["block"], spec["ctx"]
    target_hidden = w(b, ctx, fc_in, std=1.0)
    noise = w(b, block, h, std=1.0)
    out["target_hidden"], out["noise_embed"] = raw(target_hidden), raw(noise)
    tctx = bb.project_context(mx.array(target_hidden))
    out["target_ctx"] = raw(tctx)
    cos, sin = q3.rope_tables(mx.arange(ctx + block), hd, DIMS["rope_theta"])
    out["full_out"] = raw(bb(mx.array(noise), tctx, cos, sin))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    q3 = load_reference(args.reference)
    rng = np.random.default_rng(20263)
    for name, spec in CASES.items():
        case = build_case(q3, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, sorted(k for k in case if k.endswith("_out")))
    rng = np.random.default_rng(20264)
    for name, spec in LAYER_CASES.items():
        case = build_layer_case(q3, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, sorted(k for k in case if k.endswith("_out")))
    rng = np.random.default_rng(20266)
    for name, spec in BACKBONE_CASES.items():
        case = build_backbone_case(q3, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, sorted(k for k in case if k.endswith("_out")))


if __name__ == "__main__":
    main()
