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
