"""Generate the golden MoE vectors by running the reference's own ``moe.py``.

The reference (``dspark_mlx``) is imported from its source tree with the ``mlx`` API served
by ``mlx_torch_shim`` (MLX itself cannot be installed here). Its ``MoE``, ``Gate`` and the
``loading.py`` dequant helpers run unmodified on seeded inputs; inputs and outputs are
written as ``.npz`` fixtures next to this script. The fixtures are committed; the tests read
only the fixtures, never the reference tree.

    python tests/golden/make_golden.py [--reference PATH]
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


def load_reference(ref_root: str):
    """Import ``dspark_mlx.model.moe``, ``.model.config`` and ``.loading`` from the reference tree.

    The package ``__init__`` files are bypassed (they import the whole product, including
    mlx-lm); ``dspark_mlx.model.drafter`` is replaced by an empty stub because ``loading.py``
    imports it only for a type it does not use in the helpers exercised here.
    """
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    drafter = types.ModuleType("dspark_mlx.model.drafter")
    drafter.DSparkDrafter = object
    sys.modules["dspark_mlx.model.drafter"] = drafter
    moe = importlib.import_module("dspark_mlx.model.moe")
    config = importlib.import_module("dspark_mlx.model.config")
    loading = importlib.import_module("dspark_mlx.loading")
    return moe, config, loading


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy()


def _e4m3_codes(rng, shape):
    vals = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).clamp(-448, 448)
    return vals.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def _e4m3_value(codes: np.ndarray) -> np.ndarray:
    return torch.from_numpy(codes).view(torch.float8_e4m3fn).to(torch.float32).numpy()


E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def build_case(moe_mod, config_mod, loading, name: str, spec: dict, rng) -> dict:
    mx = shim
    args = config_mod.DSparkArgs.from_dict(spec["args"])
    layer_id = spec.get("layer_id", 0)
    moe = moe_mod.MoE(args, layer_id)
    E, dim, inter = args.n_routed_experts, args.dim, args.moe_inter_dim
    N = spec["n_tokens"]
    xdt = spec.get("x_dtype", torch.bfloat16)
    out = {"name": name}

    gate_w = (rng.standard_normal((E, dim)) * spec.get("gate_std", 0.02)).astype(np.float32)
    moe.gate.weight = mx.array(gate_w)
    out["gate_weight"] = gate_w
    if moe.gate.hash:
        k = args.n_activated_experts
        t2e = np.stack([rng.choice(E, size=k, replace=False) for _ in range(args.vocab_size)]).astype(np.int32)
        moe.gate.tid2eid = mx.array(t2e)
        out["tid2eid"] = t2e
    else:
        bias = (rng.standard_normal(E) * spec.get("bias_std", 0.02)).astype(np.float32)
        moe.gate.bias = mx.array(bias)
        out["gate_bias"] = bias

    wfmt = spec["wfmt"]
    std = spec.get("w_std", 0.02)
    shapes = {"w1": (E, inter, dim), "w3": (E, inter, dim), "w2": (E, dim, inter)}
    for n, shp in shapes.items():
        if wfmt == "bf16":
            w = torch.from_numpy((rng.standard_normal(shp) * std).astype(np.float32)).to(torch.bfloat16)
            moe[n] = mx.array(w)
            out[n + "_bf16"] = _bits16(w)
        elif wfmt == "f32":
            w = (rng.standard_normal(shp) * std).astype(np.float32)
            moe[n] = mx.array(w)
            out[n + "_f32"] = w
        elif wfmt == "fp8":
            codes = _e4m3_codes(rng, shp)
            sb = (shp[0], -(-shp[1] // 128), -(-shp[2] // 128))
            scales = np.exp2(rng.uniform(-10, -4, size=sb)).astype(np.float32)
            deq = np.stack([loading.dequant_fp8_blockwise(_e4m3_value(codes[e]), scales[e], 128)
                            for e in range(shp[0])])
            moe[n] = mx.array(deq)
            out[n + "_codes"], out[n + "_scales"] = codes, scales
        elif wfmt == "fp4":
            nib = rng.integers(0, 16, size=shp).astype(np.uint8)
            packed = (nib[..., 0::2] | (nib[..., 1::2] << 4)).astype(np.uint8)
            gsh = (shp[0], shp[1], shp[2] // 32)
            gcodes = torch.from_numpy(np.exp2(rng.uniform(-3, 3, size=gsh)).astype(np.float32)).to(
                torch.float8_e4m3fn).view(torch.uint8).numpy()
            tscale = np.exp2(rng.uniform(-9, -7, size=(shp[0],))).astype(np.float32)
            deq = np.stack([loading.dequant_fp4_groupwise(E2M1[nib[e]], _e4m3_value(gcodes[e]), 32)
                            for e in range(shp[0])]) * tscale[:, None, None]
            moe[n] = mx.array(deq.astype(np.float32))
            out[n + "_codes"], out[n + "_scales"], out[n + "_tscale"] = packed, gcodes, tscale
        elif wfmt.startswith("affine"):
            w = torch.from_numpy((rng.standard_normal(shp) * std).astype(np.float32)).to(torch.bfloat16)
            moe[n] = mx.array(w)
        else:
            raise ValueError(wfmt)
    if wfmt.startswith("affine"):
        bits = int(wfmt[len("affine"):])
        moe.quantize(bits=bits, group_size=64)
        for n in shapes:
            out[n + "_codes"] = moe[n + "_q"].t.numpy()
            out[n + "_scales"] = _bits16(moe[n + "_scales"].t)
            out[n + "_biases"] = _bits16(moe[n + "_biases"].t)
        out["bits"] = np.int32(bits)

    sdt = spec.get("shared_dtype", torch.bfloat16)
    for n, shp in (("w1", (inter, dim)), ("w2", (dim, inter)), ("w3", (inter, dim))):
        w = torch.from_numpy((rng.standard_normal(shp) * std).astype(np.float32)).to(sdt)
        getattr(moe.shared_experts, n).weight = mx.array(w)
        out["shared_" + n] = _bits16(w) if sdt == torch.bfloat16 else w.numpy()
    out["shared_dtype"] = np.array("bf16" if sdt == torch.bfloat16 else "f32")

    x = torch.from_numpy(rng.standard_normal((N, dim)).astype(np.float32)).to(xdt)
    out["x"] = _bits16(x) if xdt == torch.bfloat16 else x.numpy()
    out["x_dtype"] = np.array("bf16" if xdt == torch.bfloat16 else "f32")
    n_ids = spec.get("n_ids", N)
    ids = rng.integers(0, args.vocab_size, size=(n_ids,)).astype(np.int32)
    out["ids"] = ids

    y = moe(mx.array(x), mx.array(ids))
    xf = mx.array(x).reshape(-1, dim)
    weights, indices = moe.gate(xf, mx.array(ids).reshape(-1))
    if weights.shape[0] != N:  # hash anchor broadcast: take_along_axis already broadcast
        pass
    out["y"] = _bits16(y.t) if y.dtype == torch.bfloat16 else y.t.numpy()
    out["route_weights"] = weights.t.to(torch.float32).numpy()
    out["route_indices"] = np.broadcast_to(indices.t.numpy(), (N, indices.shape[-1])).astype(np.int32).copy()
    out["args"] = np.array(repr(spec["args"]))
    out["layer_id"] = np.int32(layer_id)
    return out


BASE = dict(n_shared_experts=1, swiglu_limit=10.0, n_hash_layers=0)

CASES = {
    # hash routing at the tiny hash-MoE layer's shapes (dim 256, 16 experts, top-2, inter 128)
    "hash_tiny_bf16": dict(args=dict(BASE, vocab_size=1024, dim=256, moe_inter_dim=128, n_routed_experts=16,
                                     n_activated_experts=2, n_hash_layers=1, score_func="sqrtsoftplus",
                                     route_scale=1.5), n_tokens=7, wfmt="bf16", seed=11),
    # draft-block form: one anchor id for the whole block (broadcast over the 7 tokens)
    "hash_anchor_bf16": dict(args=dict(BASE, vocab_size=64, dim=128, moe_inter_dim=64, n_routed_experts=8,
                                       n_activated_experts=2, n_hash_layers=1, score_func="sqrtsoftplus",
                                       route_scale=1.5), n_tokens=7, n_ids=1, wfmt="bf16", seed=12),
    "sigmoid_fp8": dict(args=dict(BASE, vocab_size=64, dim=256, moe_inter_dim=128, n_routed_experts=8,
                                  n_activated_experts=3, score_func="sigmoid", route_scale=2.5),
                        n_tokens=12, wfmt="fp8", seed=13),
    "sigmoid_fp4": dict(args=dict(BASE, vocab_size=64, dim=256, moe_inter_dim=128, n_routed_experts=8,
                                  n_activated_experts=2, score_func="sigmoid", route_scale=2.5),
                        n_tokens=10, wfmt="fp4", seed=14),
    "sqrtsoftplus_affine8": dict(args=dict(BASE, vocab_size=64, dim=128, moe_inter_dim=64, n_routed_experts=8,
                                           n_activated_experts=2, score_func="sqrtsoftplus", route_scale=1.5),
                                 n_tokens=6, wfmt="affine8", w_std=0.1, gate_std=0.1, bias_std=0.1, seed=15),
    "sqrtsoftplus_affine4": dict(args=dict(BASE, vocab_size=64, dim=128, moe_inter_dim=64, n_routed_experts=8,
                                           n_activated_experts=2, score_func="sqrtsoftplus", route_scale=1.5),
                                 n_tokens=6, wfmt="affine4", w_std=0.1, gate_std=0.1, bias_std=0.1, seed=16),
    "softmax_bf16": dict(args=dict(BASE, vocab_size=64, dim=128, moe_inter_dim=64, n_routed_experts=8,
                                   n_activated_experts=2, score_func="softmax", route_scale=1.0),
                         n_tokens=9, wfmt="bf16", seed=17),
    # the reference unit test's configuration: fp32 activations and weights
    "sqrtsoftplus_f32": dict(args=dict(BASE, vocab_size=64, dim=128, moe_inter_dim=64, n_routed_experts=8,
                                       n_activated_experts=2, score_func="sqrtsoftplus", route_scale=1.5),
                             n_tokens=6, wfmt="f32", x_dtype=torch.float32, shared_dtype=torch.float32,
                             w_std=0.1, gate_std=0.1, bias_std=0.1, seed=18),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DSPARK_REFERENCE", "/root/reference"))
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    moe_mod, config_mod, loading = load_reference(a.reference)
    for name, spec in CASES.items():
        torch.manual_seed(spec["seed"])
        rng = np.random.default_rng(spec["seed"])
        case = build_case(moe_mod, config_mod, loading, name, spec, rng)
        path = os.path.join(a.out, f"{name}.npz")
        np.savez_compressed(path, **case)
        print(f"{name}: {os.path.getsize(path) / 1e3:.0f} kB, indices[0]={case['route_indices'][0].tolist()}")


if __name__ == "__main__":
    main()
