"""Generate golden vectors for the DSpark draft attention by running the reference's own
``DSparkAttention`` (``dspark_mlx/model/attention.py``, with ``sparse_attn`` from
``dspark_mlx/kernels.py`` and RoPE / RMSNorm from ``dspark_mlx/model/norm_rope.py``) on
seeded inputs and weights, with the ``mlx`` API served by ``mlx_torch_shim``. Each case runs
a prefill that seeds the sliding KV window, then decode steps (and one
``advance_window``), recording the outputs and the window after each step. Everything goes
to ``attn_*.npz`` next to this script; the tests read only the fixtures.

    python tests/golden/make_golden_attn.py [--reference PATH]
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

DIMS = dict(dim=64, n_heads=4, head_dim=32, rope_head_dim=16, q_lora_rank=48, o_groups=2, o_lora_rank=24,
            window_size=8, norm_eps=1e-6, rope_theta=10000.0)
CASES = {
    # dtype, batch, block, prefill length, decode plan: ("decode", n_main) or ("advance",)
    "attn_bf16_b2_p11": dict(dtype=torch.bfloat16, b=2, block=5, prefill=11,
                             plan=[("decode", 1), ("decode", 1), ("advance",), ("decode", 1)]),
    "attn_f32_b3_p3": dict(dtype=torch.float32, b=3, block=4, prefill=3, plan=[("decode", 1), ("decode", 2)]),
}


def load_reference(ref_root: str):
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    return importlib.import_module("dspark_mlx.model.attention"), importlib.import_module("dspark_mlx.model.config")


def build_case(attn_mod, config, spec: dict, rng) -> dict:
    mx = shim
    dt = spec["dtype"]
    args = config.DSparkArgs.from_dict(dict(DIMS))
    attn = attn_mod.DSparkAttention(args, max_seq_len=64)
    d, h, hd, ql, og, orank = (DIMS[k] for k in ("dim", "n_heads", "head_dim", "q_lora_rank", "o_groups", "o_lora_rank"))

    def w(*shape, std):
        return torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(dt)

    weights = {"wq_a": w(ql, d, std=d ** -0.5), "wq_b": w(h * hd, ql, std=ql ** -0.5), "wkv": w(hd, d, std=d ** -0.5),
               "wo_a": w(og * orank, h * hd // og, std=(h * hd // og) ** -0.5), "wo_b": w(d, og * orank, std=0.1)}
    norms = {"q_norm": (1 + 0.1 * rng.standard_normal(ql)).astype(np.float32),
             "kv_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)}
    sink = rng.standard_normal(h).astype(np.float32)
    for k, v in weights.items():
        getattr(attn, k).weight = mx.array(v)
    attn.q_norm.weight = mx.array(norms["q_norm"])
    attn.kv_norm.weight = mx.array(norms["kv_norm"])
    attn.attn_sink = mx.array(sink)

    b, block = spec["b"], spec["block"]

    def raw(t):
        tt = t.t if isinstance(t, shim.array) else t
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.to(torch.float32).numpy()

    out = {"dtype_bf16": np.array(dt == torch.bfloat16), "sink": sink, **{k: raw(v) for k, v in weights.items()},
           **norms}
    p = spec["prefill"]
    main = torch.from_numpy(rng.standard_normal((b, p, d)).astype(np.float32)).to(dt)
    xb = torch.from_numpy(rng.standard_normal((b, block, d)).astype(np.float32)).to(dt)
    ret = attn(mx.array(xb), 0, mx.array(main))
    out["prefill_main"], out["prefill_x"] = raw(main), raw(xb)
    out["prefill_ret"], out["window_0"] = raw(ret), raw(attn.cache.read())
    pos = p
    steps = []
    for i, step in enumerate(spec["plan"]):
        if step[0] == "advance":
            mx1 = torch.from_numpy(rng.standard_normal((b, d)).astype(np.float32)).to(dt)
            attn.advance_window(mx.array(mx1), pos)
            out[f"s{i}_main"] = raw(mx1)
            out[f"s{i}_pos"] = np.array(pos)
            pos += 1
            steps.append("advance")
        else:
            n_main = step[1]
            mx_ = torch.from_numpy(rng.standard_normal((b, n_main, d)).astype(np.float32)).to(dt)
            xs = torch.from_numpy(rng.standard_normal((b, block, d)).astype(np.float32)).to(dt)
            o = attn(mx.array(xs), pos, mx.array(mx_))
            out[f"s{i}_main"], out[f"s{i}_x"], out[f"s{i}_pos"] = raw(mx_), raw(xs), np.array(pos)
            out[f"s{i}_out"] = raw(o)
            pos += n_main
            steps.append("decode")
        out[f"window_{i + 1}"] = raw(attn.cache.read())
    out["plan"] = np.array(steps)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    attn_mod, config = load_reference(args.reference)
    rng = np.random.default_rng(20262)
    for name, spec in CASES.items():
        case = build_case(attn_mod, config, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, sorted(k for k in case if k.endswith("_out")))


if __name__ == "__main__":
    main()
