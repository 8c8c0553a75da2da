"""The router entry point that allocates nothing (``dsm_router_noalloc``).

It exists for callers that cannot allocate device memory -- an engine whose memory arena
owns the whole GPU, or a latency-critical loop that must not touch an allocator -- and keeps
its scratch in a fixed array inside the library. Checked here through the C ABI against the
workspace-taking ``dsm_router`` on two calls in a row (the shared array is reused), and for
the clear rejection of a call that would need more than the fixed scratch.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from dsm import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed: int, n_tokens: int, dim: int, n_experts: int):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n_tokens, dim, generator=g).to(torch.bfloat16).to(DEV)
    gw = (torch.randn(n_experts, dim, generator=g) * 0.02).to(DEV)
    gb = (torch.randn(n_experts, generator=g) * 0.02).to(DEV)
    return x, gw, gb


def _call(fn, x, gw, gb, topk, ws=None):
    n, dim = x.shape
    w = torch.empty(n, topk, dtype=torch.float32, device=DEV)
    i = torch.empty(n, topk, dtype=torch.int32, device=DEV)
    args = [x.data_ptr(), _lib.DT_BF16, n, dim, gw.data_ptr(), gw.shape[0], gb.data_ptr(), None, 0, None,
            _lib.DT_I32, 0, topk, _lib.SCORE["sigmoid"], 2.5]
    if ws is not None:
        args.append(ws.data_ptr())
    args += [w.data_ptr(), i.data_ptr(), _lib.stream_ptr()]
    _lib.check(fn(*args))
    return w, i


@pytest.mark.parametrize("shape", [(56, 4096, 256, 6), (19, 1024, 64, 4), (512, 1024, 64, 6), (900, 2048, 32, 4)],
                         ids=["56tok_E256", "19tok_E64", "512tok_E64", "900tok_E32"])
def test_router_noalloc_matches_router_two_calls_in_a_row(shape):
    """Up to 256 tokens the router splits K into 256-wide slices; above that the split
    follows the SM count and the scratch size changes with it, so the 512- and 900-token cases
    run that path through the fixed array (each still within its size)."""
    L = _lib.lib()
    n, dim, E, k = shape
    need = L.dsm_router_workspace_bytes(n, dim, E)
    assert need <= 8 << 20  # DSM_ROUTER_NOALLOC_MAX_SCRATCH_BYTES
    for seed in (0, 1):  # two calls in a row on the shared array, different inputs
        x, gw, gb = _inputs(seed + 7 * n, n, dim, E)
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        w_ref, i_ref = _call(L.dsm_router, x, gw, gb, k, ws)
        w_got, i_got = _call(L.dsm_router_noalloc, x, gw, gb, k)
        torch.cuda.synchronize()
        assert torch.equal(i_got, i_ref)
        assert torch.allclose(w_got, w_ref, rtol=1e-5, atol=1e-6)
    assert _lib.device_error() == 0


def test_router_noalloc_rejects_oversized_calls():
    L = _lib.lib()
    n, dim, E = 200, 4096, 1024  # 200 x 1024 cells x 132 bytes > 8 MiB
    assert L.dsm_router_workspace_bytes(n, dim, E) > 8 << 20
    x, gw, gb = _inputs(2, n, dim, E)
    w = torch.empty(n, 6, dtype=torch.float32, device=DEV)
    i = torch.empty(n, 6, dtype=torch.int32, device=DEV)
    rc = L.dsm_router_noalloc(x.data_ptr(), _lib.DT_BF16, n, dim, gw.data_ptr(), E, gb.data_ptr(), None, 0, None,
                              _lib.DT_I32, 0, 6, _lib.SCORE["sigmoid"], 2.5, w.data_ptr(), i.data_ptr(),
                              _lib.stream_ptr())
    assert rc == 3  # DSM_ERR_WORKSPACE
    assert "scratch" in L.dsm_last_error_message().decode()
