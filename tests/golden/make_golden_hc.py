"""Generate golden vectors for the MoE's neighbours in the draft block by running the
reference's own code: ``hc_pre`` / ``hc_post`` (``dspark_mlx/model/hyper.py``),
``hc_split_sinkhorn`` (``dspark_mlx/kernels.py``) and ``RMSNorm``
(``dspark_mlx/model/norm_rope.py``), on seeded inputs, with the ``mlx`` API served by
``mlx_torch_shim``. Inputs and outputs go to ``hc_*.npz`` next to this script; the tests read
only the fixtures.

    python tests/golden/make_golden_hc.py [--reference PATH]
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

CASES = {
    # name: x dtype, [b, s], hc_mult, dim, sinkhorn iterations, scale of the mix projections
    "hc_bf16_b2s4_d256": dict(dtype=torch.bfloat16, bs=(2, 4), hc=4, dim=256, iters=20, fn_std=0.05),
    "hc_f32_b1s7_d512": dict(dtype=torch.float32, bs=(1, 7), hc=4, dim=512, iters=20, fn_std=0.05),
    "hc_bf16_b3s5_d384_it5": dict(dtype=torch.bfloat16, bs=(3, 5), hc=4, dim=384, iters=5, fn_std=0.2),
}
NORM_EPS = 1e-6
HC_EPS = 1e-6


def load_reference(ref_root: str):
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    hyper = importlib.import_module("dspark_mlx.model.hyper")
    norm = importlib.import_module("dspark_mlx.model.norm_rope")
    return hyper, norm


def build_case(hyper, norm, spec: dict, rng) -> dict:
    mx = shim
    b, s = spec["bs"]
    hc, dim = spec["hc"], spec["dim"]
    mix = (2 + hc) * hc
    dt = spec["dtype"]
    x = torch.from_numpy(rng.standard_normal((b, s, hc, dim)).astype(np.float32)).to(dt)
    fn = (rng.standard_normal((mix, hc * dim)) * spec["fn_std"]).astype(np.float32)
    scale = rng.standard_normal(3).astype(np.float32)
    base = (rng.standard_normal(mix) * 0.5).astype(np.float32)
    weight = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    h = torch.from_numpy(rng.standard_normal((b, s, dim)).astype(np.float32)).to(dt)  # a sublayer output

    y, post, comb = hyper.hc_pre(mx.array(x), mx.array(fn), mx.array(scale), mx.array(base), hc, spec["iters"],
                                 NORM_EPS, HC_EPS)
    rms = norm.RMSNorm(dim, NORM_EPS)
    rms.weight = mx.array(weight)
    yn = rms(y)
    out = hyper.hc_post(mx.array(h), mx.array(x), post, comb)

    def raw(t):  # bf16 as int16 bits, else float32
        tt = t.t if isinstance(t, shim.array) else t
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.to(torch.float32).numpy()

    return {"x": raw(x), "x_bf16": np.array(dt == torch.bfloat16), "fn": fn, "scale": scale, "base": base,
            "weight": weight, "h": raw(h), "iters": np.array(spec["iters"]), "y": raw(y), "post": raw(post),
            "comb": raw(comb), "yn": raw(yn), "out": raw(out)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    hyper, norm = load_reference(args.reference)
    rng = np.random.default_rng(20260)
    for name, spec in CASES.items():
        case = build_case(hyper, norm, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path)


if __name__ == "__main__":
    main()
