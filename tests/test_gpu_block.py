"""The MoE's neighbours in the draft block on the GPU: hc_pre + ffn_norm and hc_post
(dspark_mlx/model/block.py:83-86) against the reference's golden vectors and the oracle, and
the whole FFN sub-layer (DSparkFFN) against the oracle composition."""

from __future__ import annotations

import pytest
import torch

import oracle
from dsm import _lib, workloads as W
from dsm.block import DSparkFFN
from helpers import MOE_TOL, max_rel_err, oracle_weights, small_workload
from test_oracle_block import CASES, NORM_EPS, HC_EPS, load_hc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pre_norm(x, fn, scale, base, weight, iters):
    n, hc, dim = x.shape[0] * x.shape[1], x.shape[2], x.shape[3]
    xr = x.reshape(n, hc, dim).to(DEV).contiguous()
    xn = torch.empty(n, dim, dtype=x.dtype, device=DEV)
    post = torch.empty(n, hc, device=DEV)
    comb = torch.empty(n, hc, hc, device=DEV)
    f, s, b, w = (t.to(DEV).float().contiguous() for t in (fn, scale, base, weight))
    _lib.check(_lib.lib().dsm_hc_pre_norm(xr.data_ptr(), _lib.dtype_code(x.dtype), n, hc, dim, f.data_ptr(),
                                          s.data_ptr(), b.data_ptr(), iters, NORM_EPS, HC_EPS, w.data_ptr(),
                                          xn.data_ptr(), post.data_ptr(), comb.data_ptr(), _lib.stream_ptr()))
    torch.cuda.synchronize()
    return xn.cpu().reshape(*x.shape[:2], dim), post.cpu().reshape(*x.shape[:3]), comb.cpu().reshape(*x.shape[:3], hc)


def _post(h, x, post, comb):
    n, hc, dim = x.shape[0] * x.shape[1], x.shape[2], x.shape[3]
    out = torch.empty(n, hc, dim, dtype=x.dtype, device=DEV)
    hd, xd = h.reshape(n, dim).to(DEV).contiguous(), x.reshape(n, hc, dim).to(DEV).contiguous()
    pd, cd = post.reshape(n, hc).to(DEV).contiguous(), comb.reshape(n, hc, hc).to(DEV).contiguous()
    _lib.check(_lib.lib().dsm_hc_post(hd.data_ptr(), xd.data_ptr(), _lib.dtype_code(x.dtype), n, hc, dim,
                                      pd.data_ptr(), cd.data_ptr(), out.data_ptr(), _lib.stream_ptr()))
    torch.cuda.synchronize()
    return out.cpu().reshape(x.shape)


@pytest.mark.parametrize("name", CASES)
def test_pre_norm_and_post_match_reference_goldens(name):
    c = load_hc(name)
    xn, post, comb = _pre_norm(c["x"], c["fn"], c["scale"], c["base"], c["weight"], c["iters"])
    # fp32 reductions in another order than the reference's: a few ulps in the mixes
    torch.testing.assert_close(post, c["post"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(comb, c["comb"], rtol=1e-4, atol=1e-4)
    tol = 2e-2 if c["bf16"] else 1e-5  # bf16 outputs: a last-bit flip of the cast
    assert xn.dtype == c["yn"].dtype and max_rel_err(xn, c["yn"]) < tol
    out = _post(c["h"], c["x"], c["post"], c["comb"])
    assert out.dtype == c["out"].dtype and max_rel_err(out, c["out"]) < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pre_norm_without_weight_and_large_dim(dtype):
    g = torch.Generator().manual_seed(9)
    hc, dim = 4, 4096
    x = torch.randn(2, 7, hc, dim, generator=g).to(dtype)
    fn = torch.randn((2 + hc) * hc, hc * dim, generator=g) * 0.01
    scale, base = torch.randn(3, generator=g), torch.randn((2 + hc) * hc, generator=g) * 0.5
    ones = torch.ones(dim)
    xn, post, comb = _pre_norm(x, fn, scale, base, ones, 20)
    y, rpost, rcomb = oracle.hc_pre(x, fn, scale, base, hc, 20, NORM_EPS, HC_EPS)
    ref = oracle.rms_norm(y, None, NORM_EPS)
    torch.testing.assert_close(post, rpost, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(comb, rcomb, rtol=1e-4, atol=1e-4)
    assert max_rel_err(xn, ref) < (2e-2 if dtype == torch.bfloat16 else 1e-5)


def _ffn_case(routing: str, dtype=torch.bfloat16):
    if routing == "hash":
        wl = W.WORKLOADS["tiny_hash"]
    else:
        wl = small_workload("fp8_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=28, seed=17)
    t = W.make_moe_tensors(wl, device="cpu", n_tokens=28)
    a = t["args"]
    ffn = DSparkFFN(a, wl.layer_id).to(DEV)
    ffn.ffn = W.build_moe(wl, t, DEV)
    g = torch.Generator().manual_seed(5)
    hc, dim = ffn.hc_mult, a["dim"]
    mix = (2 + hc) * hc
    with torch.no_grad():
        ffn.hc_ffn_fn.copy_(torch.randn(mix, hc * dim, generator=g) * 0.05)
        ffn.hc_ffn_scale.copy_(torch.randn(3, generator=g))
        ffn.hc_ffn_base.copy_(torch.randn(mix, generator=g) * 0.5)
        ffn.ffn_norm.weight.copy_(1 + 0.1 * torch.randn(dim, generator=g))
    x = torch.randn(4, 7, hc, dim, generator=g).to(dtype)
    ids = t.get("input_ids")
    ids = ids.reshape(4, 7) if ids is not None else None
    return wl, t, ffn, x, ids


@pytest.mark.parametrize("routing", ["hash", "score"])
def test_ffn_sublayer_matches_oracle(routing):
    wl, t, ffn, x, ids = _ffn_case(routing)
    a = t["args"]
    out = ffn(x.to(DEV), ids.to(DEV) if ids is not None else None)
    torch.cuda.synchronize()
    assert out.shape == x.shape and out.dtype == x.dtype and _lib.device_error() == 0
    ws = oracle_weights(wl, t)
    shared = (t["shared_w1"], t["shared_w2"], t["shared_w3"])

    def moe(xn, input_ids):
        return oracle.moe_forward(xn, input_ids, gate_weight=t["gate_weight"], topk=a["n_activated_experts"],
                                  score_func=a["score_func"], route_scale=a["route_scale"],
                                  swiglu_limit=a["swiglu_limit"], w1=ws["w1"], w3=ws["w3"], w2=ws["w2"], shared=shared,
                                  gate_bias=t.get("gate_bias"), tid2eid=t.get("tid2eid"))

    hc_args = dict(hc_fn=ffn.hc_ffn_fn.cpu(), hc_scale=ffn.hc_ffn_scale.cpu(), hc_base=ffn.hc_ffn_base.cpu(),
                   norm_weight=ffn.ffn_norm.weight.cpu(), hc=ffn.hc_mult, iters=ffn.hc_sinkhorn_iters,
                   norm_eps=ffn.norm_eps, hc_eps=ffn.hc_eps)
    if routing == "hash":  # routing depends on the ids only: the whole sub-layer against the oracle
        ref = oracle.ffn_sublayer(x, ids, moe=moe, **hc_args)
    else:  # score routing: the oracle MoE runs on the GPU's own MoE input, so that a last-bit
        # difference of the normalised input cannot flip a near-tie expert choice
        xn, post, comb = _pre_norm(x, hc_args["hc_fn"], hc_args["hc_scale"], hc_args["hc_base"],
                                   hc_args["norm_weight"], hc_args["iters"])
        y, rpost, rcomb = oracle.hc_pre(x, hc_args["hc_fn"], hc_args["hc_scale"], hc_args["hc_base"], ffn.hc_mult,
                                        ffn.hc_sinkhorn_iters, ffn.norm_eps, ffn.hc_eps)
        assert max_rel_err(xn, oracle.rms_norm(y, hc_args["norm_weight"], ffn.norm_eps)) < 2e-2
        ref = oracle.hc_post(moe(xn, None), x, rpost, rcomb)
    assert max_rel_err(out, ref) < MOE_TOL, max_rel_err(out, ref)
