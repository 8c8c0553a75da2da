"""The oracle's restatement of the whole DSpark draft block against golden vectors from the
reference's own ``DSparkBlock`` (``dspark_mlx/model/block.py``; ``tests/golden/make_golden_block.py``):
``forward_embed``, the prefill, decode steps, ``advance``, the window after each step, and
``forward_head`` at temperature 0.

Everything is bit-identical except the fp32 decode outputs. There the MoE's fp32 matmuls run
over the block's token shape, and the CPU BLAS sums them in another order than the reference
run's batched ``gather_mm``. They agree within 1e-6 relative; the attention half alone is
bit-identical."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "block_*.npz")))
ARGS = dict(vocab_size=512, dim=256, moe_inter_dim=128, n_layers=2, n_mtp_layers=1, n_hash_layers=0, n_heads=4,
            n_routed_experts=8, n_shared_experts=1, n_activated_experts=2, score_func="sigmoid", route_scale=2.5,
            swiglu_limit=10.0, q_lora_rank=48, head_dim=32, rope_head_dim=16, o_groups=2, o_lora_rank=24,
            window_size=8, norm_eps=1e-6, hc_mult=4, hc_sinkhorn_iters=20, hc_eps=1e-6, rope_theta=10000.0,
            dspark_block_size=5, dspark_noise_token_id=500, dspark_markov_rank=16, temperature=0.0,
            dspark_target_layer_ids=[1, 3, 5])
SKIP = {"dtype_bf16", "plan", "main_hidden", "input_ids", "embed_x", "embed_main_x", "prefill_ret", "head_ids",
        "head_logits", "head_conf"}


def _t(a):
    return torch.from_numpy(a).view(torch.bfloat16) if a.dtype == np.int16 else torch.from_numpy(a)


def load_case(name):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    t = {k: _t(v) for k, v in z.items() if "." in k or k.startswith("hc_")}
    return z, t


def test_golden_cases_exist():
    assert len(CASES) == 2


@pytest.mark.parametrize("name", CASES)
def test_block_oracle_matches_reference_goldens(name):
    z, t = load_case(name)
    a = ARGS
    ids = torch.from_numpy(z["input_ids"])
    x, main_x = oracle.block_forward_embed(t, a, _t(z["main_hidden"]), ids, t["embed.weight"])
    assert torch.equal(x, _t(z["embed_x"])) and torch.equal(main_x, _t(z["embed_main_x"]))
    cos, sin = oracle.rope_tables(a["rope_head_dim"], 64, a["rope_theta"])
    cache = oracle.KVWindow(a["window_size"])
    ret = oracle.block_forward(t, a, x, 0, ids, main_x, cache, cos, sin)
    assert torch.equal(ret, _t(z["prefill_ret"]))
    assert torch.equal(cache.window, _t(z["window_0"]))
    y = None
    for i, kind in enumerate(z["plan"]):
        pos = int(z[f"s{i}_pos"])
        m1x = oracle.rms_norm(oracle.linear(_t(z[f"s{i}_main_hidden"]), t["main_proj.weight"]), t["main_norm.weight"],
                              a["norm_eps"])
        assert torch.equal(m1x, _t(z[f"s{i}_main_x"]))
        if kind == "advance":
            oracle.block_advance(t, a, m1x.reshape(m1x.shape[0], -1), pos, cache, cos, sin)
        else:
            y = oracle.block_forward(t, a, x, pos, ids, m1x, cache, cos, sin)
            ref = _t(z[f"s{i}_out"])
            assert y.dtype == x.dtype
            if x.dtype == torch.bfloat16:
                assert torch.equal(y, ref), (name, i)
            else:
                assert float((y - ref).abs().max()) <= 1e-6 * float(ref.abs().max()), (name, i)
                y = ref  # the head below starts from the reference's block output
        assert torch.equal(cache.window, _t(z[f"window_{i + 1}"])), (name, i)
    out_ids, biased, conf = oracle.block_forward_head(t, a, y, ids, t["head.weight"])
    assert torch.equal(out_ids.to(torch.int32), torch.from_numpy(z["head_ids"]).to(torch.int32))
    assert torch.equal(biased, _t(z["head_logits"])) and torch.equal(conf, _t(z["head_conf"]))
