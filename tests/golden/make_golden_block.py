"""Generate golden vectors for the whole DSpark draft block by running the reference's own
``DSparkBlock`` (``dspark_mlx/model/block.py``, with its attention, MoE, hyper-connections,
norms and heads) on seeded inputs and weights, with the ``mlx`` API served by
``mlx_torch_shim``. One stage that is both the first and the last (``n_mtp_layers = 1``), so
``forward_embed`` and ``forward_head`` run too. The sequence per case:
* ``forward_embed(main_hidden, input_ids, embed)`` -> the block input and the main rows;
* ``block(x, 0, ids, main_x)``, the prefill that seeds the attention's window;
* decode calls ``block(x, pos, ids, main_x1)`` and one ``advance(main_x1, pos)``;
* ``forward_head(y, ids, head)`` at temperature 0 on the last decode output.
Everything goes to ``block_*.npz`` next to this script; the tests read only the fixtures.

    python tests/golden/make_golden_block.py [--reference PATH]
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

ARGS = dict(vocab_size=512, dim=256, moe_inter_dim=128, n_layers=2, n_mtp_layers=1, n_hash_layers=0, n_heads=4,
            n_routed_experts=8, n_shared_experts=1, n_activated_experts=2, score_func="sigmoid", route_scale=2.5,
            swiglu_limit=10.0, q_lora_rank=48, head_dim=32, rope_head_dim=16, o_groups=2, o_lora_rank=24,
            window_size=8, norm_eps=1e-6, hc_mult=4, hc_sinkhorn_iters=20, hc_eps=1e-6, rope_theta=10000.0,
            dspark_block_size=5, dspark_noise_token_id=500, dspark_markov_rank=16, temperature=0.0,
            dspark_target_layer_ids=[1, 3, 5])
CASES = {
    # weight / activation dtype, batch, prefill length, decode plan
    "block_bf16_b2_p10": dict(dtype=torch.bfloat16, b=2, prefill=10, plan=["decode", "advance", "decode"]),
    "block_f32_b1_p4": dict(dtype=torch.float32, b=1, prefill=4, plan=["decode"]),
}


def load_reference(ref_root: str):
    shim.install()
    for name, sub in (("dspark_mlx", "dspark_mlx"), ("dspark_mlx.model", "dspark_mlx/model")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(ref_root, sub)]
        sys.modules[name] = mod
    return importlib.import_module("dspark_mlx.model.block"), importlib.import_module("dspark_mlx.model.config")


def build_case(block_mod, config, spec: dict, rng) -> dict:
    mx = shim
    dt = spec["dtype"]
    a = dict(ARGS)
    args = config.DSparkArgs.from_dict(a)
    blk = block_mod.DSparkBlock(args, 0, max_seq_len=64)
    d, hc, E, inter = a["dim"], a["hc_mult"], a["n_routed_experts"], a["moe_inter_dim"]
    h, hd, ql, og, orank = a["n_heads"], a["head_dim"], a["q_lora_rank"], a["o_groups"], a["o_lora_rank"]
    vocab, rank = a["vocab_size"], a["dspark_markov_rank"]
    mix = (2 + hc) * hc

    def w(*shape, std, dtype=None):
        return torch.from_numpy((rng.standard_normal(shape) * std).astype(np.float32)).to(dtype or dt)

    def f32(*shape, std, mean=0.0):
        return (mean + rng.standard_normal(shape) * std).astype(np.float32)

    t = {  # every tensor of the block, under its reference name
        "attn.wq_a.weight": w(ql, d, std=d ** -0.5), "attn.wq_b.weight": w(h * hd, ql, std=ql ** -0.5),
        "attn.wkv.weight": w(hd, d, std=d ** -0.5),
        "attn.wo_a.weight": w(og * orank, h * hd // og, std=(h * hd // og) ** -0.5),
        "attn.wo_b.weight": w(d, og * orank, std=(og * orank) ** -0.5),
        "attn.q_norm.weight": f32(ql, std=0.1, mean=1.0), "attn.kv_norm.weight": f32(hd, std=0.1, mean=1.0),
        "attn.attn_sink": f32(h, std=1.0),
        "ffn.gate.weight": f32(E, d, std=0.1), "ffn.gate.bias": f32(E, std=0.1),
        "ffn.w1": w(E, inter, d, std=d ** -0.5), "ffn.w3": w(E, inter, d, std=d ** -0.5),
        "ffn.w2": w(E, d, inter, std=inter ** -0.5),
        "ffn.shared_experts.w1.weight": w(inter, d, std=d ** -0.5),
        "ffn.shared_experts.w3.weight": w(inter, d, std=d ** -0.5),
        "ffn.shared_experts.w2.weight": w(d, inter, std=inter ** -0.5),
        "attn_norm.weight": f32(d, std=0.1, mean=1.0), "ffn_norm.weight": f32(d, std=0.1, mean=1.0),
        "hc_attn_fn": f32(mix, hc * d, std=0.05), "hc_ffn_fn": f32(mix, hc * d, std=0.05),
        "hc_attn_base": f32(mix, std=0.5), "hc_ffn_base": f32(mix, std=0.5),
        "hc_attn_scale": f32(3, std=1.0), "hc_ffn_scale": f32(3, std=1.0),
        "main_proj.weight": w(d, d * len(a["dspark_target_layer_ids"]), std=(3 * d) ** -0.5),
        "main_norm.weight": f32(d, std=0.1, mean=1.0), "norm.weight": f32(d, std=0.1, mean=1.0),
        "markov_head.markov_w1.weight": w(vocab, rank, std=0.5), "markov_head.markov_w2.weight": w(vocab, rank, std=0.5),
        "confidence_head.proj.weight": f32(1, d + rank, std=0.05),
        "hc_head_fn": f32(hc, hc * d, std=0.05), "hc_head_base": f32(hc, std=0.5), "hc_head_scale": f32(1, std=1.0),
    }
    for name, v in t.items():
        *path, leaf = name.split(".")
        obj = blk
        for p in path:
            obj = getattr(obj, p)
        setattr(obj, leaf, mx.array(v))
    embed_w = w(vocab, d, std=1.0)
    head_w = w(vocab, d, std=0.05)
    embed = shim.Embedding(vocab, d)
    embed.weight = mx.array(embed_w)
    head = shim.Linear(d, vocab, bias=False)
    head.weight = mx.array(head_w)

    def raw(x):
        tt = x.t if isinstance(x, shim.array) else x
        if isinstance(tt, np.ndarray):
            return tt
        return tt.view(torch.int16).numpy() if tt.dtype == torch.bfloat16 else tt.numpy()

    out = {"dtype_bf16": np.array(dt == torch.bfloat16), "embed.weight": raw(embed_w), "head.weight": raw(head_w)}
    out.update({k: raw(v) for k, v in t.items()})
    b, pre = spec["b"], spec["prefill"]
    k_main = len(a["dspark_target_layer_ids"])
    main_hidden = w(b, pre, d * k_main, std=1.0)
    ids = rng.integers(0, vocab, size=(b,)).astype(np.int32)
    x, main_x = blk.forward_embed(mx.array(main_hidden), mx.array(ids), embed)
    out["main_hidden"], out["input_ids"] = raw(main_hidden), ids
    out["embed_x"], out["embed_main_x"] = raw(x), raw(main_x)
    ret = blk(x, 0, mx.array(ids), main_x)
    out["prefill_ret"] = raw(ret)
    out["window_0"] = raw(blk.attn.cache.read())
    pos = pre
    y = None
    for i, kind in enumerate(spec["plan"]):
        m1 = w(b, 1, d * k_main, std=1.0)
        out[f"s{i}_main_hidden"], out[f"s{i}_pos"] = raw(m1), np.array(pos)
        m1x = blk.main_norm(blk.main_proj(mx.array(m1)))
        out[f"s{i}_main_x"] = raw(m1x)
        if kind == "advance":
            blk.advance(m1x.reshape(b, d), pos)
        else:
            y = blk(x, pos, mx.array(ids), m1x)
            out[f"s{i}_out"] = raw(y)
        out[f"window_{i + 1}"] = raw(blk.attn.cache.read())
        pos += 1
    ids_out, biased, conf = blk.forward_head(y, mx.array(ids), head)
    out["head_ids"], out["head_logits"], out["head_conf"] = raw(ids_out), raw(biased), raw(conf)
    out["plan"] = np.array(spec["plan"])
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    block_mod, config = load_reference(args.reference)
    rng = np.random.default_rng(20265)
    for name, spec in CASES.items():
        case = build_case(block_mod, config, spec, rng)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **case)
        print("wrote", path, sorted(k for k in case if k.endswith("_out") or k.startswith("head_")))


if __name__ == "__main__":
    main()
