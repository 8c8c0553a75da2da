"""Toy end-to-end draft/verify loop with the MoE block inside.

The reference pins losslessness with its drafter against an order-1 Markov base
(tests/test_generate_lossless.py:30-86): whatever the drafter proposes, the emitted stream
equals plain greedy decoding of the base. The drafter's attention and hyper-connections are
outside this module's scope, so the drafter here is a toy with the same block shape: the
anchor token's embedding plus per-position offsets ``[1, K, dim]`` -> the MoE block (score
routing, or hash routing on the anchor id broadcast over the block as
dspark_mlx/model/moe.py:71-72 allows) -> an LM head -> greedy drafts. The loop runs with
``dsm.MoE`` on the GPU and with the oracle's MoE on the CPU. The draft tokens must be
identical block by block, and both emitted streams must equal the base's greedy stream.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from dsm import workloads as W
from helpers import oracle_weights, small_workload

pytestmark = pytest.mark.gpu
DEV = "cuda"
V, K, N_NEW = 32, 4, 40
NEAR_TIE = 1e-2  # top-2 logit gap below which the last bit of the block output may decide


def _plain_greedy(transition: torch.Tensor, start: int, steps: int):
    out, last = [], start
    for _ in range(steps):
        last = int(transition[last].argmax())
        out.append(last)
    return out


def _verify(transition, last, drafts):
    """Accept the longest prefix of drafts that the base's greedy chain reproduces, then the
    base's own next token (the correction, or the bonus after a full accept)."""
    emitted = []
    for d in drafts:
        g = int(transition[last].argmax())
        emitted.append(g)
        last = g
        if d != g:
            return emitted
    emitted.append(int(transition[last].argmax()))
    return emitted


@pytest.mark.parametrize("routing", ["score", "hash"])
def test_toy_draft_loop_drafts_match_and_stream_is_lossless(routing):
    if routing == "hash":
        wl = W.WORKLOADS["tiny_hash"]  # hidden 256, 16 experts, top-2, sqrtsoftplus, bf16
    else:
        wl = small_workload("fp8_decode", dim=256, inter=128, experts=16, topk=2, n_tokens=K, wfmt="bf16", seed=11)
    t = W.make_moe_tensors(wl, device="cpu", n_tokens=K)
    moe = W.build_moe(wl, t, DEV)
    a = t["args"]
    ws = oracle_weights(wl, t)
    shared = (t["shared_w1"], t["shared_w2"], t["shared_w3"])
    dim = a["dim"]

    g = torch.Generator().manual_seed(0)
    transition = torch.randn(V, V, generator=g)
    embed = torch.randn(V, dim, generator=g)
    pos = torch.randn(K, dim, generator=g) * 0.5
    # block outputs are ~0.1 here: scale the head so logit gaps sit well above the
    # bf16 rounding of the block output (~1e-4 in logits)
    head = torch.randn(dim, V, generator=g) * 10 / dim ** 0.5

    def block_logits(impl: str, anchor: int) -> torch.Tensor:
        x = (embed[anchor] + pos).to(torch.bfloat16).unsqueeze(0)  # [1, K, dim]
        ids = torch.tensor([anchor], dtype=torch.int32) if routing == "hash" else None
        if impl == "gpu":
            y = moe(x.to(DEV), ids.to(DEV) if ids is not None else None).cpu()
        else:
            y = oracle.moe_forward(x, ids, gate_weight=t["gate_weight"], topk=a["n_activated_experts"],
                                   score_func=a["score_func"], route_scale=a["route_scale"],
                                   swiglu_limit=a["swiglu_limit"], w1=ws["w1"], w3=ws["w3"], w2=ws["w2"],
                                   shared=shared, gate_bias=t.get("gate_bias"), tid2eid=t.get("tid2eid"))
        assert y.shape == (1, K, dim) and y.dtype == torch.bfloat16
        return y[0].float() @ head  # [K, V]

    prompt_last = 5
    # loop driven by the oracle's drafts; the GPU drafts are compared at the same anchors
    compared = skipped = blocks = 0
    emitted, last = [], prompt_last
    while len(emitted) < N_NEW:
        lo = block_logits("oracle", last)
        lg = block_logits("gpu", last)
        d_ref = lo.argmax(dim=-1).tolist()
        d_gpu = lg.argmax(dim=-1).tolist()
        top2 = lo.topk(2, dim=-1).values
        for i in range(K):
            if float(top2[i, 0] - top2[i, 1]) < NEAR_TIE:
                skipped += 1
                continue
            compared += 1
            assert d_gpu[i] == d_ref[i], (blocks, i, d_gpu, d_ref)
        out = _verify(transition, last, d_ref)
        emitted += out
        last = out[-1]
        blocks += 1
    assert emitted[:N_NEW] == _plain_greedy(transition, prompt_last, N_NEW)
    assert compared >= 0.8 * (compared + skipped) and blocks >= N_NEW // (K + 1)

    # the GPU-driven loop on its own: same stream (lossless whatever the drafts)
    emitted, last = [], prompt_last
    while len(emitted) < N_NEW:
        out = _verify(transition, last, block_logits("gpu", last).argmax(dim=-1).tolist())
        emitted += out
        last = out[-1]
    assert emitted[:N_NEW] == _plain_greedy(transition, prompt_last, N_NEW)
