"""Generate golden vectors for the DSpark draft head by running the reference's own code:
``hc_head`` (``dspark_mlx/model/hyper.py``), ``RMSNorm`` (``dspark_mlx/model/norm_rope.py``),
the Markov and confidence heads (``dspark_mlx/model/heads.py``) and the block walk
``draft_block_decode`` (``dspark_mlx/recipe.py``), composed as ``DSparkBlock.forward_head``
does (``dspark_mlx/model/block.py:111-116``). Seeded inputs; the ``mlx`` API is served by
``mlx_torch_shim``, whose ``mx.random.uniform`` records the uniforms the sampler drew at a
temperature above 0. Inputs and outputs go to ``head_*.npz`` next to this script; the tests
read only the fixtures.

    python tests/golden/make_golden_head.py [--reference PATH]
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
    # x dtype, weight dtype (LM head, Markov tables), [b, s], hc, dim, vocab, rank, temperature
    "head_bf16_b2s5_v512": dict(dtype=torch.bfloat16, wdtype=torch.bfloat16, bs=(2, 5), hc=4, dim=256, vocab=512,
                                rank=16, temperature=0.0),
    "head_f32_b3s7_v1000": dict(dtype=torch.float32, wdtype=torch.float32, bs=(3, 7), hc=4, dim=256, vocab=1000,
                                rank=32, temperature=0.0),
    "head_bf16_b4s4_v640_t1": dict(dtype=torch.bfloat16, wdtype=torch.bfloat16, bs=(4, 4), hc=4, dim=256, vocab=640,
                                   rank=16, temperature=1.0),
}
NORM_EPS = 1e-6
HC_EPS = 1e-6


def load_reference(ref_root: str):
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    mods = {n: importlib.import_module(f"dspark_mlx.{n}") for n in ("model.hyper", "model.norm_rope", "model.heads",
                                                                   "recipe")}
    return mods


def build_case(mods, spec: dict, rng, seed: int) -> dict:
    mx = shim
    hyper, norm, heads, recipe = (mods[k] for k in ("model.hyper", "model.norm_rope", "model.heads", "recipe"))
    b, s = spec["bs"]
    hc, dim, vocab, rank = spec["hc"], spec["dim"], spec["vocab"], spec["rank"]
    dt, wdt = spec["dtype"], spec["wdtype"]
    x = torch.from_numpy(rng.standard_normal((b, s, hc, dim)).astype(np.float32)).to(dt)
    fn = (rng.standard_normal((hc, hc * dim)) * 0.05).astype(np.float32)
    scale = rng.standard_normal(1).astype(np.float32)
    base = (rng.standard_normal(hc) * 0.5).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    head_w = torch.from_numpy((rng.standard_normal((vocab, dim)) * 0.05).astype(np.float32)).to(wdt)
    w1 = torch.from_numpy((rng.standard_normal((vocab, rank)) * 0.5).astype(np.float32)).to(wdt)
    w2 = torch.from_numpy((rng.standard_normal((vocab, rank)) * 0.5).astype(np.float32)).to(wdt)
    wc = (rng.standard_normal((1, dim + rank)) * 0.05).astype(np.float32)
    anchor = rng.integers(0, vocab, size=(b,)).astype(np.int32)

    # DSparkBlock.forward_head (block.py:111-116), its modules holding the weights above
    y = hyper.hc_head(mx.array(x), mx.array(fn), mx.array(scale), mx.array(base), NORM_EPS, HC_EPS)
    rms = norm.RMSNorm(dim, NORM_EPS)
    rms.weight = mx.array(norm_w)
    head = shim.Linear(dim, vocab, bias=False)
    head.weight = mx.array(head_w)
    logits = head(rms(y).astype(mx.float32))
    markov = heads.DSparkMarkovHead(vocab, rank)
    markov.markov_w1.weight = mx.array(w1)
    markov.markov_w2.weight = mx.array(w2)
    conf = heads.DSparkConfidenceHead(dim + rank)
    conf.proj.weight = mx.array(wc)
    shim.random_seed(seed)
    out_ids, biased, confidence = recipe.draft_block_decode(logits, y, mx.array(anchor), markov, conf, s,
                                                            spec["temperature"])
    uniforms = (torch.stack(shim.random_draws).numpy() if shim.random_draws
                else np.zeros((0, b, vocab), np.float32))

    def raw(t):  # bf16 as int16 bits, else float32 / int32
        tt = t.t if isinstance(t, shim.array) else t
        if tt.dtype == torch.bfloat16:
            return tt.view(torch.int16).numpy()
        return tt.numpy() if tt.dtype == torch.int32 else tt.to(torch.float32).numpy()

    return {"x": raw(x), "x_bf16": np.array(dt == torch.bfloat16), "w_bf16": np.array(wdt == torch.bfloat16),
            "fn": fn, "scale": scale, "base": base, "norm_w": norm_w, "head_w": raw(head_w), "w1": raw(w1),
            "w2": raw(w2), "wc": wc, "anchor": anchor, "temperature": np.array(spec["temperature"], np.float32),
            "uniforms": uniforms, "y": raw(y), "logits": raw(logits), "out_ids": raw(out_ids),
            "biased": raw(biased), "confidence": raw(confidence)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    mods = load_reference(args.reference)
    rng = np.random.default_rng(20261)
    for i, (name, spec) in enumerate(CASES.items()):
        case = build_case(mods, spec, rng, seed=100 + i)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, {k: v.shape for k, v in case.items() if k in ("out_ids", "biased", "uniforms")})


if __name__ == "__main__":
    main()
