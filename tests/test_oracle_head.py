"""The oracle's restatement of the DSpark draft head against golden vectors from the
reference's own hyper.py (hc_head), norm_rope.py, heads.py and recipe.py
(``tests/golden/make_golden_head.py``), plus the reference's own head test values."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "head_*.npz")))
NORM_EPS = HC_EPS = 1e-6


def load_head(name):
    z = np.load(os.path.join(HERE, name + ".npz"))

    def t(k):
        a = z[k]
        return torch.from_numpy(a).view(torch.bfloat16) if a.dtype == np.int16 else torch.from_numpy(a)

    c = {k: t(k) for k in ("x", "fn", "scale", "base", "norm_w", "head_w", "w1", "w2", "wc", "anchor", "uniforms",
                           "y", "logits", "out_ids", "biased", "confidence")}
    c["temperature"] = float(z["temperature"])
    c["bf16"] = bool(z["x_bf16"])
    return c


def oracle_head(c, **over):
    kw = dict(head_w=c["head_w"], hc_fn=c["fn"], hc_scale=c["scale"], hc_base=c["base"], norm_w=c["norm_w"],
              w1=c["w1"], w2=c["w2"], wc=c["wc"], norm_eps=NORM_EPS, hc_eps=HC_EPS, temperature=c["temperature"],
              uniforms=list(c["uniforms"]) if len(c["uniforms"]) else None)
    kw.update(over)
    return oracle.forward_head(c["x"], c["anchor"], **kw)


def test_golden_cases_exist():
    assert len(CASES) == 3


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_goldens(name):
    c = load_head(name)
    y = oracle.hc_head(c["x"], c["fn"], c["scale"], c["base"], NORM_EPS, HC_EPS)
    # the same torch fp32 operations in the same order as the reference run: bit-identical
    assert y.dtype == c["y"].dtype and torch.equal(y, c["y"])
    ids, biased, conf = oracle_head(c)
    assert torch.equal(ids, c["out_ids"])
    assert torch.equal(biased, c["biased"])
    assert torch.equal(conf, c["confidence"])
    assert ids.shape == (c["x"].shape[0], c["x"].shape[1] + 1) and torch.equal(ids[:, 0], c["anchor"])


def test_temperature_case_consumed_one_uniform_draw_per_position():
    c = load_head("head_bf16_b4s4_v640_t1")
    b, s = c["x"].shape[:2]
    assert c["uniforms"].shape == (s, b, c["head_w"].shape[0])
    # other uniforms give other samples somewhere in the block
    ids, _, _ = oracle_head(c, uniforms=list(torch.rand_like(c["uniforms"])))
    assert not torch.equal(ids, c["out_ids"])


def test_reference_head_values():
    """tests/test_heads_parity.py:21-60 of the reference: the Markov and confidence heads on
    its seeded inputs, against a direct fp32 restatement."""
    vocab, dim, rank, b, k = 512, 64, 16, 2, 5
    rng = np.random.default_rng(0)
    w1 = torch.from_numpy((rng.standard_normal((vocab, rank)) * 0.02).astype(np.float32))
    w2 = torch.from_numpy((rng.standard_normal((vocab, rank)) * 0.02).astype(np.float32))
    tok = torch.from_numpy(rng.integers(0, vocab, size=(b,)).astype(np.int64))
    logits, embed = oracle.markov_head(tok, w1, w2)
    assert torch.equal(embed, w1[tok])
    torch.testing.assert_close(logits, w1[tok] @ w2.T, rtol=0, atol=1e-6)
    rng = np.random.default_rng(1)
    wc = torch.from_numpy((rng.standard_normal((1, dim + rank)) * 0.02).astype(np.float32))
    hidden = torch.from_numpy((rng.standard_normal((b, k, dim)) * 0.5).astype(np.float32))
    membed = torch.from_numpy((rng.standard_normal((b, k, rank)) * 0.5).astype(np.float32))
    conf = oracle.confidence_head(hidden, membed, wc)
    torch.testing.assert_close(conf, (torch.cat([hidden, membed], -1) @ wc.T)[..., 0], rtol=0, atol=1e-6)
