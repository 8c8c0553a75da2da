"""Pin the CPU oracle: the reference's own known-answer tests and the golden vectors.

* Dequant block maths: the exact cases of ``tests/test_loading.py:74-95`` (reference).
* Sparse == dense-loop equivalence: ``tests/test_moe_gather_mm.py:36-58`` (reference).
* Expert stacking: ``tests/test_moe_gather_mm.py:82-96`` (reference).
* Golden vectors produced by the reference's own ``moe.py`` (``tests/golden/make_golden.py``).
* Code decoding against the library casts, permutation invariants, affine round trip.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io
import oracle


def test_dequant_fp8_blockwise_kat():
    w = torch.arange(16, dtype=torch.float32).reshape(4, 4)
    scale = torch.tensor([[2.0, 3.0], [4.0, 5.0]])
    out = oracle.dequant_fp8_blockwise(w, scale, block=2)
    exp = w.clone()
    exp[0:2, 0:2] *= 2
    exp[0:2, 2:4] *= 3
    exp[2:4, 0:2] *= 4
    exp[2:4, 2:4] *= 5
    assert torch.equal(out, exp)


def test_dequant_fp4_groupwise_kat():
    w = torch.arange(16, dtype=torch.float32).reshape(2, 8)
    scale = torch.tensor([[2.0, 3.0], [4.0, 5.0]])
    out = oracle.dequant_fp4_groupwise(w, scale, group=4)
    exp = w.clone()
    exp[0, 0:4] *= 2
    exp[0, 4:8] *= 3
    exp[1, 0:4] *= 4
    exp[1, 4:8] *= 5
    assert torch.equal(out, exp)


def test_e4m3_decode_matches_torch_cast():
    codes = np.arange(256, dtype=np.uint8)
    mine = oracle.e4m3_decode(codes)
    lib = torch.from_numpy(codes).view(torch.float8_e4m3fn).to(torch.float32)
    both_nan = torch.isnan(mine) & torch.isnan(lib)
    assert torch.equal(torch.where(both_nan, 0.0, mine), torch.where(both_nan, 0.0, lib))
    vals = torch.randn(4096, generator=torch.Generator().manual_seed(0)) * 40
    enc = oracle.e4m3_encode(vals)
    assert torch.equal(enc, vals.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8))


def test_e2m1_decode_table():
    vals = oracle.e2m1_decode(np.arange(16, dtype=np.uint8))
    exp = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6])
    assert torch.equal(vals, exp)


def _rand_moe(seed, E=8, dim=128, inter=64, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(E, inter, dim, generator=g) * 0.1).to(dtype)
    w3 = (torch.randn(E, inter, dim, generator=g) * 0.1).to(dtype)
    w2 = (torch.randn(E, dim, inter, generator=g) * 0.1).to(dtype)
    gw = torch.randn(E, dim, generator=g) * 0.1
    gb = torch.randn(E, generator=g) * 0.1
    shared = tuple((torch.randn(*s, generator=g) * 0.1).to(dtype) for s in ((inter, dim), (dim, inter), (inter, dim)))
    return w1, w2, w3, gw, gb, shared


def test_sparse_matches_dense_loop():
    """``tests/test_moe_gather_mm.py:47-58``: sparse routing == O(E) dense loop, < 1e-4."""
    w1, w2, w3, gw, gb, shared = _rand_moe(0)
    x = torch.randn(6, 128, generator=torch.Generator().manual_seed(1)) * 0.5
    kw = dict(gate_weight=gw, topk=2, score_func="sqrtsoftplus", route_scale=1.5, swiglu_limit=10.0,
              w1=oracle.OracleWeights("dense", w1), w3=oracle.OracleWeights("dense", w3),
              w2=oracle.OracleWeights("dense", w2), shared=shared, gate_bias=gb)
    sparse, weights, indices = oracle.moe_forward(x, None, return_routing=True, **kw)
    dense = oracle.dense_combine(x, w1, w2, w3, weights, indices, 10.0)
    dense = dense + oracle.expert_forward(x, shared[0], shared[1], shared[2], 10.0).float()
    assert float((sparse - dense).abs().max()) < 1e-4


def test_affine_quantized_close_to_bf16():
    """``tests/test_moe_gather_mm.py:61-79``: q8 within 0.05 and q4 within 0.40 of bf16."""
    w1, w2, w3, gw, gb, shared = _rand_moe(2, dtype=torch.bfloat16)
    x = torch.randn(6, 128, generator=torch.Generator().manual_seed(1)) * 0.5
    base = dict(gate_weight=gw, topk=2, score_func="sqrtsoftplus", route_scale=1.5, swiglu_limit=10.0,
                shared=shared, gate_bias=gb)
    ref = oracle.moe_forward(x, None, w1=oracle.OracleWeights("dense", w1), w3=oracle.OracleWeights("dense", w3),
                             w2=oracle.OracleWeights("dense", w2), **base)
    scale = float(ref.abs().max()) + 1e-6
    for bits, tol in ((8, 0.05), (4, 0.40)):
        q = {n: oracle.affine_quantize(w, 64, bits) for n, w in (("w1", w1), ("w2", w2), ("w3", w3))}
        ws = {n: oracle.OracleWeights("affine", *q[n], group_size=64, bits=bits) for n in q}
        out = oracle.moe_forward(x, None, w1=ws["w1"], w3=ws["w3"], w2=ws["w2"], **base)
        assert float((out - ref).abs().max()) / scale < tol


def test_stack_experts():
    """``tests/test_moe_gather_mm.py:82-96``: row e of the stack is expert e."""
    g = torch.Generator().manual_seed(3)
    per = {e: torch.randn(6, 8, generator=g) for e in range(4)}
    params = {f"blocks.2.ffn.experts.{e}.w1.weight": per[e] for e in range(4)}
    params["blocks.2.attn.q_proj.weight"] = torch.zeros(4, 4)
    oracle.stack_experts(params)
    assert params["blocks.2.ffn.w1"].shape == (4, 6, 8)
    for e in range(4):
        assert torch.equal(params["blocks.2.ffn.w1"][e], per[e])
    assert "blocks.2.attn.q_proj.weight" in params


def test_affine_roundtrip_error_bound():
    w = torch.randn(16, 256, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    for bits in (4, 8):
        codes, s, b = oracle.affine_quantize(w, 64, bits)
        deq = oracle.affine_dequantize(codes, s, b, 64, bits)
        step = s.float().abs().repeat_interleave(64, -1)
        bias = b.float().abs().repeat_interleave(64, -1)
        # Snapping the edge so that zero is exact can clip the far end of the range by up
        # to one step; storing scale and bias in bf16 adds up to 2**bits * 2**-8 steps.
        bound = step * (1.5 + ((1 << bits) - 1) * 2.0 ** -8) + bias * 2.0 ** -8 + 1e-6
        assert bool(((deq - w.float()).abs() <= bound).all())


def test_permutation_invariants():
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(0, 16, (37, 3), generator=g).to(torch.int32)
    counts, offsets, perm, inv = oracle.permutation(idx, 16)
    flat = idx.reshape(-1)
    assert int(counts.sum()) == flat.numel()
    assert torch.equal(offsets[1:] - offsets[:-1], counts)
    sorted_e = flat[perm.long()]
    assert bool((sorted_e[1:] >= sorted_e[:-1]).all())
    for e in range(16):  # stable: ascending pair ids inside each expert
        seg = perm[offsets[e]:offsets[e + 1]]
        assert bool((seg[1:] > seg[:-1]).all())
    assert torch.equal(perm[inv.long()], torch.arange(flat.numel(), dtype=torch.int32))


@pytest.mark.parametrize("name", golden_io.names())
def test_oracle_matches_reference_golden(name):
    c = golden_io.load(name)
    y, w, idx = golden_io.oracle_forward(c)
    assert torch.equal(idx, c.route_indices), "routing indices differ from the reference"
    assert torch.allclose(w, c.route_weights, rtol=1e-5, atol=1e-6)
    assert y.dtype == c.y.dtype
    assert golden_io.max_rel_err(y, c.y) < 1e-2
