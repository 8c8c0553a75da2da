"""The whole DSpark draft block on the GPU (``dsm.draft_block.DSparkBlock``) against golden
vectors from the reference's own ``DSparkBlock`` (``tests/golden/make_golden_block.py``):
``forward_embed``, the prefill's window, decode steps through both hyper-connection halves,
``advance`` and ``forward_head``.

Tolerances (max|out - ref| / max|ref|): the block outputs 2e-2 in bf16 and 1e-2 in fp32 (the
MoE stages fp32 activations as one f16 row, as the MoE tests allow); the window as the
attention tests (2e-2 / 2e-3). ``forward_head`` runs on the reference's own block output and is
held to the draft head's comparison: ids equal up to a near tie, logits within 2e-3."""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

from dsm import _lib
from dsm.draft_block import DSparkBlock
from helpers import max_rel_err
from test_gpu_head import _compare_walk
from test_oracle_draft_block import ARGS, HERE, _t, load_case

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "block_*.npz")))


class _W(torch.nn.Module):
    def __init__(self, w):
        super().__init__()
        self.weight = torch.nn.Parameter(w, requires_grad=False)


def _block(t) -> DSparkBlock:
    """The block with every golden tensor under its reference name: buffers (the MoE's gate and
    stacked experts) take plain tensors, parameters take Parameters."""
    blk = DSparkBlock(ARGS, 0, max_seq_len=64).to(DEV)
    for name, v in t.items():
        if name in ("embed.weight", "head.weight"):
            continue
        *path, leaf = name.split(".")
        obj = blk
        for p in path:
            obj = getattr(obj, p)
        if leaf in obj._buffers:
            setattr(obj, leaf, v.to(DEV))
        else:
            setattr(obj, leaf, torch.nn.Parameter(v.to(DEV), requires_grad=False))
    return blk


@pytest.mark.parametrize("name", CASES)
def test_draft_block_matches_reference_goldens(name, attn_kernel):
    z, t = load_case(name)
    bf16 = bool(z["dtype_bf16"])
    if attn_kernel == 0 and not bf16:
        pytest.skip("fp32 attention always runs the CUDA-core kernels")
    tol, wtol = (2e-2, 2e-2) if bf16 else (1e-2, 2e-3)
    blk = _block(t)
    ids = torch.from_numpy(z["input_ids"]).to(DEV)
    x, main_x = blk.forward_embed(_t(z["main_hidden"]).to(DEV), ids, _W(t["embed.weight"].to(DEV)))
    torch.cuda.synchronize()
    assert torch.equal(x.cpu(), _t(z["embed_x"]))  # a row gather: exact
    assert max_rel_err(main_x, _t(z["embed_main_x"])) < wtol
    ret = blk(x, 0, ids, _t(z["embed_main_x"]).to(DEV))
    assert torch.equal(ret.cpu(), x.cpu())
    assert max_rel_err(blk.attn.window, _t(z["window_0"])) < wtol
    for i, kind in enumerate(z["plan"]):
        pos = int(z[f"s{i}_pos"])
        m1x = _t(z[f"s{i}_main_x"]).to(DEV)
        if kind == "advance":
            blk.advance(m1x.reshape(m1x.shape[0], -1), pos)
        else:
            y = blk(x, pos, ids, m1x)
            torch.cuda.synchronize()
            ref = _t(z[f"s{i}_out"])
            assert y.dtype == ref.dtype and y.shape == ref.shape
            assert max_rel_err(y, ref) < tol, (name, i, max_rel_err(y, ref))
        assert max_rel_err(blk.attn.window, _t(z[f"window_{i + 1}"])) < wtol, (name, i)
    last = max(i for i, k in enumerate(z["plan"]) if k == "decode")
    out_ids, biased, conf = blk.forward_head(_t(z[f"s{last}_out"]).to(DEV), ids, _W(t["head.weight"].to(DEV)))
    torch.cuda.synchronize()
    ref_ids = torch.from_numpy(z["head_ids"]).to(torch.int32)
    assert out_ids.dtype == torch.int32 and out_ids.shape == ref_ids.shape
    assert torch.equal(out_ids[:, 0].cpu(), ref_ids[:, 0])
    n = _compare_walk(out_ids.cpu(), biased.cpu(), conf.cpu(), ref_ids, _t(z["head_logits"]), _t(z["head_conf"]), 2e-3)
    assert n >= ref_ids.shape[0]
    assert _lib.device_error() == 0


def test_draft_block_full_width_matches_oracle():
    """The bench's whole-block workload at its own widths (DeepSeek-V4: dim 4096, 64 heads of
    512, 4 hyper-connection streams, 256 fp8 experts top-6): one decode step of 8 sequences
    after a 160-token prefill, the first sequence against the oracle's block (the experts it
    routes to dequantised on the CPU)."""
    import oracle
    from dsm import workloads as W
    from oracle.attention_oracle import AttnDims

    wl = W.WORKLOADS["draft_block_dsv4"]
    a = wl.args
    t = W.make_block_tensors(wl, device=DEV, seed=3)
    blk = W.build_block(wl, t, DEV)
    pos = wl.extra["prefill"]
    blk(t["x"], 0, None, t["attn_prefill_main"])
    y = blk(t["x"], pos, None, t["attn_main"])
    torch.cuda.synchronize()
    assert _lib.device_error() == 0

    class _Lazy(oracle.OracleWeights):
        def matrix(self, e):
            return oracle.fp8_weight_dequant(self.data[e].cpu(), self.scales[e].cpu())

    p = {k: t[f"attn_{k}"].cpu() for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "q_norm", "kv_norm", "attn_sink")}
    dims = AttnDims(n_heads=a["n_heads"], head_dim=a["head_dim"], rope_head_dim=a["rope_head_dim"],
                    o_groups=a["o_groups"], o_lora_rank=a["o_lora_rank"], window_size=a["window_size"],
                    eps=a["norm_eps"])
    cos, sin = oracle.rope_tables(a["rope_head_dim"], wl.extra["max_seq_len"], a["rope_theta"])
    cache = oracle.KVWindow(a["window_size"])
    oracle.attention_forward(p, dims, t["x"][:1, :, 0].cpu(), 0, t["attn_prefill_main"][:1].cpu(), cache, cos, sin)
    ffn = dict(gate_weight=t["moe_gate_weight"].cpu(), gate_bias=t["moe_gate_bias"].cpu(),
               topk=a["n_activated_experts"], score_func=a["score_func"], route_scale=a["route_scale"],
               swiglu_limit=a["swiglu_limit"],
               **{n: _Lazy("fp8", t[f"moe_{n}_codes"], scales=t[f"moe_{n}_scale"]) for n in ("w1", "w3", "w2")},
               shared=tuple(t[f"moe_shared_{n}"].cpu() for n in ("w1", "w2", "w3")))
    hc = dict(hc=a["hc_mult"], iters=a["hc_sinkhorn_iters"], norm_eps=a["norm_eps"], hc_eps=a["hc_eps"])
    halves = {h: dict(hc_fn=t[f"hc_{h}_fn"].cpu(), hc_scale=t[f"hc_{h}_scale"].cpu(),
                      hc_base=t[f"hc_{h}_base"].cpu(), norm_weight=t[f"norm_{h}"].cpu()) for h in ("attn", "ffn")}
    x, main = t["x"][:1].cpu(), t["attn_main"][:1].cpu()
    h = oracle.ffn_sublayer(x, None, moe=lambda v, _i: oracle.attention_forward(p, dims, v, pos, main, cache, cos, sin),
                            **halves["attn"], **hc)
    ref = oracle.ffn_sublayer(h, None, moe=lambda v, ids: oracle.moe_forward(v, ids, **ffn), **halves["ffn"], **hc)
    assert ref.shape == y[:1].shape and ref.dtype == y.dtype
    assert max_rel_err(y[:1], ref) < 2e-2, max_rel_err(y[:1], ref)
