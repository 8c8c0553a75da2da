"""The oracle's restatement of the DSpark draft attention against golden vectors from the
reference's own ``DSparkAttention`` (attention.py, kernels.sparse_attn, norm_rope.py):
prefill of the sliding KV window, decode steps and ``advance_window``
(``tests/golden/make_golden_attn.py``)."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle
from oracle.attention_oracle import AttnDims

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "attn_*.npz")))
DIMS = dict(dim=64, n_heads=4, head_dim=32, rope_head_dim=16, q_lora_rank=48, o_groups=2, o_lora_rank=24,
            window_size=8, norm_eps=1e-6, rope_theta=10000.0)


def _t(a):
    return torch.from_numpy(a).view(torch.bfloat16) if a.dtype == np.int16 else torch.from_numpy(a)


def test_golden_cases_exist():
    assert len(CASES) == 2


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_goldens(name):
    z = dict(np.load(os.path.join(HERE, name + ".npz")))
    p = {k: _t(z[k]) for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b")}
    p.update(q_norm=_t(z["q_norm"]), kv_norm=_t(z["kv_norm"]), attn_sink=_t(z["sink"]))
    dims = AttnDims(n_heads=DIMS["n_heads"], head_dim=DIMS["head_dim"], rope_head_dim=DIMS["rope_head_dim"],
                    o_groups=DIMS["o_groups"], o_lora_rank=DIMS["o_lora_rank"], window_size=DIMS["window_size"],
                    eps=DIMS["norm_eps"])
    cos, sin = oracle.rope_tables(DIMS["rope_head_dim"], 64, DIMS["rope_theta"])
    cache = oracle.KVWindow(DIMS["window_size"])
    x0 = _t(z["prefill_x"])
    ret = oracle.attention_forward(p, dims, x0, 0, _t(z["prefill_main"]), cache, cos, sin)
    assert ret is x0
    # the same torch operations in the same order as the reference run: bit-identical
    assert torch.equal(cache.window, _t(z["window_0"]))
    for i, kind in enumerate(z["plan"]):
        if kind == "advance":
            main = _t(z[f"s{i}_main"])
            pos = int(z[f"s{i}_pos"])
            kv = oracle.rms_norm(oracle.linear(main, p["wkv"]), p["kv_norm"], dims.eps)[:, None, :]
            kv = oracle.rope_last(kv, cos[pos:pos + 1], sin[pos:pos + 1], dims.rope_head_dim)
            cache.update(pos, kv[:, 0])
        else:
            out = oracle.attention_forward(p, dims, _t(z[f"s{i}_x"]), int(z[f"s{i}_pos"]), _t(z[f"s{i}_main"]),
                                           cache, cos, sin)
            ref = _t(z[f"s{i}_out"])
            assert out.dtype == ref.dtype and torch.equal(out, ref), (name, i)
        assert torch.equal(cache.window, _t(z[f"window_{i + 1}"])), (name, i)


def test_sparse_attn_sink_and_mask():
    """The sink only enlarges the denominator; masked slots (-1) take no weight."""
    g = torch.Generator().manual_seed(2)
    q = torch.randn(1, 2, 3, 8, generator=g)
    kv = torch.randn(1, 5, 8, generator=g)
    idx = torch.tensor([[[0, 1, 2, -1], [3, 4, -1, -1]]], dtype=torch.int32)
    far = torch.full((3,), -1e4)
    o = oracle.sparse_attn(q, kv, far, idx, 0.5)
    for m, rows in enumerate(([0, 1, 2], [3, 4])):  # plain softmax attention over the unmasked rows
        s = (q[0, m] @ kv[0, rows].T) * 0.5
        torch.testing.assert_close(o[0, m], torch.softmax(s, -1) @ kv[0, rows], rtol=1e-5, atol=1e-6)
    o2 = oracle.sparse_attn(q, kv, torch.zeros(3), idx, 0.5)
    assert (o2.norm(dim=-1) < o.norm(dim=-1)).all()  # a sink at logit 0 shrinks every output
