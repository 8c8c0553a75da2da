"""The DSpark draft head on the GPU (``dsm.head``) against golden vectors from the
reference's own hyper.py / norm_rope.py / heads.py / recipe.py and against the oracle.

Token choices are compared exactly up to the first position where the reference's two best
candidates are closer than the logit tolerance. From there a row may legitimately take
another path, so it is compared only up to that point. The LM head's products run in f16
with fp32 accumulation: bf16 weights are exact, fp32 weights are rounded to f16."""

from __future__ import annotations

import pytest
import torch

import oracle
from dsm import _lib
from dsm.head import DSparkHead, DSparkMarkovHead
from test_oracle_head import CASES, HC_EPS, NORM_EPS, load_head, oracle_head

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _head_from(c, conf_bias=None):
    b, s, hc, dim = c["x"].shape
    vocab, rank = c["w1"].shape
    args = dict(vocab_size=vocab, dim=dim, hc_mult=hc, dspark_markov_rank=rank, dspark_block_size=s,
                temperature=c["temperature"], norm_eps=NORM_EPS, hc_eps=HC_EPS)
    h = DSparkHead(args, conf_bias=conf_bias is not None).to(DEV)
    with torch.no_grad():
        h.hc_head_fn.copy_(c["fn"])
        h.hc_head_scale.copy_(c["scale"])
        h.hc_head_base.copy_(c["base"])
        h.norm.weight.copy_(c["norm_w"])
        h.markov_head.markov_w1.weight = torch.nn.Parameter(c["w1"].to(DEV), requires_grad=False)
        h.markov_head.markov_w2.weight = torch.nn.Parameter(c["w2"].to(DEV), requires_grad=False)
        h.confidence_head.proj.weight.copy_(c["wc"])
        if conf_bias is not None:
            h.confidence_head.proj.bias.fill_(conf_bias)
        h.head.weight = torch.nn.Parameter(c["head_w"].to(DEV), requires_grad=False)
    return h


def _compare_walk(ids, biased, conf, ref_ids, ref_biased, ref_conf, atol):
    """ids equal up to a near tie of the reference; logits and confidence close up to there."""
    b, s1 = ref_ids.shape
    compared = 0
    for r in range(b):
        for i in range(s1 - 1):
            lr = ref_biased[r, i]
            err = (biased[r, i] - lr).abs().max().item()
            scale = max(1.0, lr.abs().max().item())
            assert err <= atol * scale, (r, i, err)
            assert abs(conf[r, i].item() - ref_conf[r, i].item()) <= 1e-3 * max(1.0, abs(ref_conf[r, i].item()))
            compared += 1
            if ids[r, i + 1] != ref_ids[r, i + 1]:
                top2 = torch.topk(lr, 2).values
                assert (top2[0] - top2[1]).item() <= 2 * atol * scale, (r, i, "not a near tie")
                break
    return compared


@pytest.mark.parametrize("name", CASES)
def test_draft_head_matches_reference_goldens(name):
    c = load_head(name)
    h = _head_from(c)
    uni = c["uniforms"].to(DEV) if len(c["uniforms"]) else None
    ids, biased, conf = h(c["x"].to(DEV), c["anchor"].to(DEV), uniforms=uni)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert ids.dtype == torch.int32 and ids.shape == c["out_ids"].shape
    assert torch.equal(ids[:, 0].cpu(), c["anchor"])
    # fp32 weights are rounded to f16 for the LM head; a bf16 hidden may differ from the
    # reference's by one last bit (fp32 sums in another order before the cast)
    atol = 2e-3
    n = _compare_walk(ids.cpu(), biased.cpu(), conf.cpu(), c["out_ids"], c["biased"], c["confidence"], atol)
    assert n >= c["x"].shape[0]


def test_hc_head_norm_kernel_matches_golden_hidden():
    c = load_head("head_bf16_b2s5_v512")
    b, s, hc, dim = c["x"].shape
    n = b * s
    x = c["x"].to(DEV).contiguous()
    y = torch.empty(n, dim, dtype=x.dtype, device=DEV)
    xn = torch.empty_like(y)
    conf = torch.empty(n, device=DEV)
    f = lambda t: t.to(DEV).float().contiguous()  # noqa: E731
    fn, sc, base, nw, wc = f(c["fn"]), f(c["scale"]), f(c["base"]), f(c["norm_w"]), f(c["wc"].reshape(-1))
    _lib.check(_lib.lib().dsm_hc_head_norm(x.data_ptr(), _lib.DT_BF16, n, hc, dim, fn.data_ptr(), sc.data_ptr(),
                                           base.data_ptr(), NORM_EPS, HC_EPS, nw.data_ptr(), wc.data_ptr(),
                                           y.data_ptr(), xn.data_ptr(), conf.data_ptr(), _lib.stream_ptr()))
    torch.cuda.synchronize()
    ref_y = c["y"].reshape(n, dim)
    # fp32 reductions in another order than the reference's: a last-bit flip of the bf16 cast
    diff = (y.cpu().float() - ref_y.float()).abs()
    assert (diff <= ref_y.float().abs() * 2 ** -7 + 1e-6).all()
    assert (diff == 0).float().mean() > 0.95
    ref_xn = oracle.rms_norm(ref_y, c["norm_w"], NORM_EPS)
    assert ((xn.cpu().float() - ref_xn.float()).abs() <= ref_xn.float().abs() * 2 ** -6 + 1e-5).all()
    torch.testing.assert_close(conf.cpu(), ref_y.float() @ c["wc"].reshape(-1)[:dim], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_markov_head_matches_oracle(dtype):
    g = torch.Generator().manual_seed(11)
    vocab, rank = 1000, 64
    m = DSparkMarkovHead(vocab, rank).to(DEV)
    w1, w2 = (torch.randn(vocab, rank, generator=g) * 0.3).to(dtype), (torch.randn(vocab, rank, generator=g) * 0.3).to(dtype)
    m.markov_w1.weight = torch.nn.Parameter(w1.to(DEV), requires_grad=False)
    m.markov_w2.weight = torch.nn.Parameter(w2.to(DEV), requires_grad=False)
    ids = torch.randint(0, vocab, (3, 5), generator=g)
    logits, embed = m(ids.to(DEV))
    torch.cuda.synchronize()
    rl, re = oracle.markov_head(ids, w1, w2)
    assert logits.shape == (3, 5, vocab) and embed.dtype == dtype and torch.equal(embed.cpu(), re)
    torch.testing.assert_close(logits.cpu(), rl, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("b,temperature", [(8, 0.0), (8, 0.7), (20, 0.0), (32, 0.7)])
def test_draft_head_large_batch_and_vocab(b, temperature):
    """DeepSeek-V4 widths (dim 4096, hc 4, rank 256) with a 32000-word vocabulary, b x 7 draft
    tokens, bf16 weights and activations, a confidence bias. Batches above 8 run the walk's
    32-row instance (four 8-row tensor-core tiles, the last ones partly padding)."""
    g = torch.Generator().manual_seed(5 + b)
    s, hc, dim, vocab, rank = 7, 4, 4096, 32000, 256
    c = {"x": torch.randn(b, s, hc, dim, generator=g).to(torch.bfloat16),
         "fn": torch.randn(hc, hc * dim, generator=g) * 0.02, "scale": torch.randn(1, generator=g),
         "base": torch.randn(hc, generator=g) * 0.5, "norm_w": 1 + 0.1 * torch.randn(dim, generator=g),
         "head_w": (torch.randn(vocab, dim, generator=g) * 0.02).to(torch.bfloat16),
         "w1": (torch.randn(vocab, rank, generator=g) * 0.2).to(torch.bfloat16),
         "w2": (torch.randn(vocab, rank, generator=g) * 0.2).to(torch.bfloat16),
         "wc": torch.randn(1, dim + rank, generator=g) * 0.02,
         "anchor": torch.randint(0, vocab, (b,), generator=g, dtype=torch.int32), "temperature": temperature,
         "uniforms": torch.zeros(0)}
    uni = [torch.rand(b, vocab, generator=g) for _ in range(s)] if temperature > 0 else None
    h = _head_from(c, conf_bias=0.25)
    ids, biased, conf = h(c["x"].to(DEV), c["anchor"].to(DEV), uniforms=torch.stack(uni).to(DEV) if uni else None)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ref = oracle_head(c, uniforms=uni, conf_bias=torch.tensor([0.25]))
    n = _compare_walk(ids.cpu(), biased.cpu(), conf.cpu(), *ref, atol=2e-3)
    assert n >= b
    # deterministic: the same call gives the same tokens and logits
    ids2, biased2, _ = h(c["x"].to(DEV), c["anchor"].to(DEV), uniforms=torch.stack(uni).to(DEV) if uni else None)
    assert torch.equal(ids, ids2) and torch.equal(biased, biased2)
