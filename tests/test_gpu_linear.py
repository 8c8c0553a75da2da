"""The linear entry points beside ``dsm_linear``, through the C ABI.

``dsm_linear_splitk`` (K split across the GPU: the tensor-memory weight formats, and bf16 weights
on the streaming kernel) against ``dsm_linear`` on the same staged rows and packed weights.

Both multiply the same products; the split one sums fp32 partial slabs over K ranges in range
order, so the two agree to fp32 rounding (1e-5 relative). Outputs go to a column slice of a
wider buffer (row stride ``ldo``): the columns outside the slice must keep their contents.

``dsm_grouped_linear`` and ``dsm_grouped_linear_splitk`` (several weight matrices over row groups,
one launch, scattered output rows) against fp32 products of the same rows and (dequantised)
weights."""

from __future__ import annotations

import pytest
import torch

from dsm import _lib
from dsm._lib import dtype_code, lib, ptr, stream_ptr
from dsm.weights import affine_quantize, pack
from helpers import max_rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("bits,n,k,out", [(8, 112, 2560, 1024), (8, 300, 2560, 2560), (4, 56, 4096, 512),
                                          (8, 14, 4096, 4096),
                                          # bf16 weights on the streaming kernel: the draft attention's
                                          # wo_b, wq_a and wkv over a 56-row draft step, and 9 rows
                                          (0, 56, 8192, 4096), (0, 56, 4096, 1024), (0, 9, 4096, 512)])
def test_splitk_matches_whole_k_linear(bits, n, k, out):
    g = torch.Generator().manual_seed(n + k + out)
    w = (torch.randn(out, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    if bits:
        q, s, b = affine_quantize(w, group_size=64, bits=bits)
        pm = pack("affine", data=q, scales=s, biases=b, group_size=64, bits=bits, device=DEV)
    else:
        pm = pack("dense", data=w, device=DEV)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16).to(DEV)
    L = lib()
    cap = L.dsm_stage_rows_cap(n)
    staged = torch.empty(L.dsm_stage_bytes(cap, k), dtype=torch.uint8, device=DEV)
    xs = torch.empty(cap, dtype=torch.float32, device=DEV)
    _lib.check(L.dsm_stage_rows(ptr(x), dtype_code(x.dtype), n, k, None, n, 1, ptr(staged), cap, ptr(xs),
                                stream_ptr()), "dsm_stage_rows")
    ldo, c0 = out + 32, 16
    whole = torch.full((n, ldo), 7.0, device=DEV)
    split = torch.full((n, ldo), 7.0, device=DEV)
    _lib.check(L.dsm_linear(ptr(staged), ptr(xs), cap, k, pm.wfmt, pm.group_size, ptr(pm.packed), out,
                            ptr(whole[:, c0:]), ldo, n, stream_ptr()), "dsm_linear")
    ws_bytes = L.dsm_linear_splitk_workspace_bytes(n, out)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    for _ in range(2):  # a second call on the same workspace gives the same result
        _lib.check(L.dsm_linear_splitk(ptr(staged), ptr(xs), cap, k, pm.wfmt, pm.group_size, ptr(pm.packed), out,
                                       ptr(split[:, c0:]), ldo, n, ptr(ws), ws_bytes, stream_ptr()),
                   "dsm_linear_splitk")
    torch.cuda.synchronize()
    assert max_rel_err(split[:, c0:c0 + out], whole[:, c0:c0 + out]) < 1e-5
    assert torch.all(split[:, :c0] == 7.0) and torch.all(split[:, c0 + out:] == 7.0)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("fmt", ["dense", "affine8"])
def test_grouped_linear_matches_per_group_products(fmt, split):
    """The draft attention's grouped output projection as one call: 4 groups of rank 256 over
    group-major rows (56 tokens x 512 values per group), row r = (g, t) written to output row
    t * 4 + g of a [56, 4 * 256] buffer. split: through dsm_grouped_linear_splitk (K split for
    the dense weights: four ranges of 128; the affine weights take the unsplit product)."""
    from oracle.formats import affine_dequantize

    g = torch.Generator().manual_seed(9)
    groups, n, d, rank = 4, 56, 512, 256
    o = torch.randn(groups, n, d, generator=g).to(torch.bfloat16)
    w = (torch.randn(groups, rank, d, generator=g) * d ** -0.5).to(torch.bfloat16)
    if fmt == "dense":
        pm = pack("dense", data=w.to(DEV), device=DEV)
        wf = w.float()
    else:
        q, s, b = affine_quantize(w.to(DEV), group_size=64, bits=8)
        pm = pack("affine", data=q, scales=s, biases=b, group_size=64, bits=8, device=DEV)
        wf = affine_dequantize(q.cpu(), s.cpu(), b.cpu(), 64, 8)
    L = lib()
    rows = groups * n
    x = o.reshape(rows, d).to(DEV)
    cap = L.dsm_stage_rows_cap(rows)
    staged = torch.empty(L.dsm_stage_bytes(cap, d), dtype=torch.uint8, device=DEV)
    xs = torch.empty(cap, dtype=torch.float32, device=DEV)
    _lib.check(L.dsm_stage_rows(ptr(x), dtype_code(x.dtype), rows, d, None, rows, 1, ptr(staged), cap, ptr(xs),
                                stream_ptr()), "dsm_stage_rows")
    offsets = (torch.arange(groups + 1, dtype=torch.int32) * n).to(DEV)
    gi, t = torch.meshgrid(torch.arange(groups), torch.arange(n), indexing="ij")
    row_map = (t * groups + gi).reshape(-1).to(torch.int32).to(DEV)
    y = torch.full((n, groups * rank), 7.0, device=DEV)
    ws_bytes = L.dsm_linear_splitk_workspace_bytes(rows, rank)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    for _ in range(2):
        if split:
            _lib.check(L.dsm_grouped_linear_splitk(ptr(staged), ptr(xs), cap, d, pm.wfmt, pm.group_size,
                                                   ptr(pm.packed), groups, ptr(offsets), rank, ptr(y), rank,
                                                   ptr(row_map), rows, ptr(ws), ws_bytes, stream_ptr()),
                       "dsm_grouped_linear_splitk")
        else:
            _lib.check(L.dsm_grouped_linear(ptr(staged), ptr(xs), cap, d, pm.wfmt, pm.group_size, ptr(pm.packed),
                                            groups, ptr(offsets), rank, ptr(y), rank, ptr(row_map), rows,
                                            stream_ptr()), "dsm_grouped_linear")
    torch.cuda.synchronize()
    ref = torch.einsum("gtd,grd->tgr", o.float(), wf.reshape(groups, rank, d)).reshape(n, groups * rank)
    # bf16 weights are exact in the f16 tiles; dequantised 8-bit weights are formed in f16 in
    # tensor memory (2^-11 relative each)
    tol = 1e-5 if fmt == "dense" else 2e-3
    assert max_rel_err(y, ref) < tol, max_rel_err(y, ref)
    assert _lib.device_error() == 0
