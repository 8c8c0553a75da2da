"""The MoE call through the C ABI captured in a CUDA graph: every launch of dsm_moe_forward
(router, permutation, staging, grouped products, the shared expert on its side stream,
combine) is stream-ordered on the caller's stream with a caller-owned workspace, so one
capture replays the whole layer. A replay must equal the eager call bit for bit, on the
captured input and on new input written into the same buffer."""

from __future__ import annotations

import ctypes

import pytest
import torch

from dsm import _lib, workloads as W
from helpers import MOE_TOL, max_rel_err, oracle_moe, small_workload

pytestmark = pytest.mark.gpu
DEV = "cuda"

CASES = {
    "tiny_hash": lambda: W.WORKLOADS["tiny_hash"],
    "fp8_small": lambda: small_workload("fp8_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=14),
    "fp4_small": lambda: small_workload("fp4_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=56),
}


@pytest.mark.parametrize("name", list(CASES))
def test_moe_forward_replays_in_a_cuda_graph(name):
    wl = CASES[name]()
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, DEV)
    L = _lib.lib()
    x = t["x"].to(DEV).contiguous()
    N, dim = x.shape
    topk = wl.args["n_activated_experts"]
    ids = t.get("input_ids")
    ids = ids.to(DEV) if ids is not None else None
    desc, keep = moe.describe(N, torch.bfloat16)
    wsb = L.dsm_moe_workspace_bytes(ctypes.byref(desc))
    ws = torch.empty(max(1, wsb), dtype=torch.uint8, device=DEV)
    y = torch.empty(N, dim, dtype=torch.bfloat16, device=DEV)
    rw = torch.empty(N, topk, dtype=torch.float32, device=DEV)
    ri = torch.empty(N, topk, dtype=torch.int32, device=DEV)

    def call():
        _lib.check(L.dsm_moe_forward(ctypes.byref(desc), x.data_ptr(), _lib.DT_BF16,
                                     ids.data_ptr() if ids is not None else None, _lib.DT_I32,
                                     N if ids is not None else 0, y.data_ptr(), rw.data_ptr(), ri.data_ptr(),
                                     ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream))

    call()
    torch.cuda.synchronize()
    y_eager, i_eager = y.clone(), ri.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    y.zero_()
    ri.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(ri, i_eager)
    assert torch.equal(y, y_eager)
    ref_y, _, ref_i = oracle_moe(wl, t)
    assert torch.equal(ri.cpu(), ref_i)
    assert max_rel_err(y, ref_y) < MOE_TOL

    # new tokens in the captured input buffer: the replay computes on them
    x2 = torch.randn(N, dim, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    x.copy_(x2.to(DEV))
    g.replay()
    torch.cuda.synchronize()
    y_graph, i_graph = y.clone(), ri.clone()
    call()
    torch.cuda.synchronize()
    assert torch.equal(i_graph, ri)
    assert torch.equal(y_graph, y)
    del g


def _graph_matches_eager(call, inputs):
    """``call(x)`` captured once on the first input; each replay after new data is written into
    that input equals the eager call on the same data, bit for bit."""
    x0 = inputs[0]
    call(x0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = call(x0)
    outs = out if isinstance(out, tuple) else (out,)
    for x in inputs:
        x0.copy_(x)
        g.replay()
        torch.cuda.synchronize()
        got = [o.clone() for o in outs]
        want = call(x0)
        want = want if isinstance(want, tuple) else (want,)
        torch.cuda.synchronize()
        assert len(got) == len(want)
        for a, b in zip(got, want):
            assert torch.equal(a, b)
    del g


def _variants(x, n=2, seed=9):
    gen = torch.Generator(device=x.device).manual_seed(seed)
    return [x.clone()] + [torch.randn(x.shape, generator=gen, device=x.device).to(x.dtype) for _ in range(n)]


def test_qwen3_attention_replays_in_a_cuda_graph():
    from dsm.qwen3_attention import rope_tables

    wl = W.WORKLOADS["qwen3_attn_q8"]
    t = W.make_gqa_tensors(wl, device=DEV, seed=0)
    attn = W.build_gqa(wl, t, DEV)
    a = wl.args
    cos, sin = rope_tables(torch.arange(wl.extra["ctx"], wl.extra["ctx"] + wl.block), a["head_dim"], a["rope_theta"])
    cos, sin = cos.to(DEV), sin.to(DEV)
    kc, vc = t["ctx_k"], t["ctx_v"]
    _graph_matches_eager(lambda x: attn.attend_cached(x, kc, vc, cos, sin), _variants(t["x"]))


def test_draft_attention_replays_in_a_cuda_graph():
    wl = W.WORKLOADS["draft_attn_dsv4"]
    t = W.make_dsattn_tensors(wl, device=DEV, seed=0)
    attn = W.build_dsattn(wl, t, DEV)
    pos = wl.extra["prefill"]
    attn(t["x"], 0, t["prefill_main"])  # the window holds the prefill's last positions
    main = t["main"]
    _graph_matches_eager(lambda x: attn(x, pos, main), _variants(t["x"]))


def test_draft_head_replays_in_a_cuda_graph():
    wl = W.WORKLOADS["draft_head"]
    t = W.make_head_tensors(wl, device=DEV, seed=0)
    head = W.build_head(wl, t, DEV)
    anchor = t["anchor"]

    _graph_matches_eager(lambda x: tuple(head(x, anchor)), _variants(t["x"]))
