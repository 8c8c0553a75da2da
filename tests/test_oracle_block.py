"""The oracle's restatement of the draft block's hyper-connection mixing and RMSNorm against
golden vectors from the reference's own hyper.py / kernels.py / norm_rope.py."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "hc_*.npz")))
NORM_EPS = HC_EPS = 1e-6


def load_hc(name):
    z = np.load(os.path.join(HERE, name + ".npz"))
    bf16 = bool(z["x_bf16"])

    def t(k):
        a = z[k]
        return torch.from_numpy(a).view(torch.bfloat16) if a.dtype == np.int16 else torch.from_numpy(a)

    return {k: t(k) for k in ("x", "h", "y", "post", "comb", "yn", "out")} | {
        k: torch.from_numpy(z[k]) for k in ("fn", "scale", "base", "weight")} | {"iters": int(z["iters"]), "bf16": bf16}


def test_golden_cases_exist():
    assert len(CASES) == 3


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_goldens(name):
    c = load_hc(name)
    hc = c["x"].shape[2]
    y, post, comb = oracle.hc_pre(c["x"], c["fn"], c["scale"], c["base"], hc, c["iters"], NORM_EPS, HC_EPS)
    # the same fp32 operations in the same order as the reference run: bit-identical
    assert torch.equal(y, c["y"]) and torch.equal(post, c["post"]) and torch.equal(comb, c["comb"])
    assert torch.equal(oracle.rms_norm(c["y"], c["weight"], NORM_EPS), c["yn"])
    out = oracle.hc_post(c["h"], c["x"], c["post"], c["comb"])
    assert out.shape == c["x"].shape and torch.equal(out, c["out"])


def test_sinkhorn_is_doubly_stochastic():
    g = torch.Generator().manual_seed(3)
    mixes = torch.randn(5, 24, generator=g)
    pre, post, comb = oracle.hc_split_sinkhorn(mixes, torch.ones(3), torch.zeros(24), 4, 20, 1e-6)
    assert torch.all(pre > 0) and torch.all((post > 0) & (post < 2))
    torch.testing.assert_close(comb.sum(-2), torch.ones(5, 4), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(comb.sum(-1), torch.ones(5, 4), rtol=2e-3, atol=2e-3)
