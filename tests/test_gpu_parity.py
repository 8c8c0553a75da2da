"""Parity of the CUDA path (through the C ABI) against the CPU oracle and the golden vectors.

Bars: routing indices, permutation and per-expert counts bit-exact; MoE outputs within a
max relative error of 1e-2 (``helpers.MOE_TOL``).
"""

from __future__ import annotations

import pytest
import torch

import golden_io
import oracle
from dsm import _lib, workloads as W
from dsm.config import DSparkArgs
from dsm.moe import MoE
from dsm.weights import affine_quantize
from helpers import MOE_TOL, check_routing, max_rel_err, oracle_moe, small_workload

pytestmark = pytest.mark.gpu
DEV = "cuda"


# ------------------------------------------------------------------------------ golden
def _moe_from_golden(c: golden_io.GoldenCase) -> MoE:
    moe = MoE(DSparkArgs.from_dict(c.args), c.layer_id)
    moe.gate.weight = c.gate_weight.to(DEV)
    if c.tid2eid is not None:
        moe.gate.tid2eid = c.tid2eid.to(DEV)
    else:
        moe.gate.bias = c.gate_bias.to(DEV)
    w = c.weights
    if c.wfmt in ("bf16", "f32"):
        for n in ("w1", "w3", "w2"):
            setattr(moe, n, w[n].data.to(DEV))
    elif c.wfmt == "fp8":
        moe.load_fp8_experts(**{n: (w[n].data.to(DEV), w[n].scales.to(DEV)) for n in ("w1", "w3", "w2")})
    elif c.wfmt == "fp4":
        moe.load_fp4_experts(**{n: (w[n].data.to(DEV), w[n].scales.to(DEV), w[n].tscale.to(DEV))
                                for n in ("w1", "w3", "w2")})
    else:  # affine: install the reference's quantized triple directly
        bits = w["w1"].bits
        moe._drop_routed()
        for n in ("w1", "w3", "w2"):
            moe.register_buffer(f"{n}_q", w[n].data.to(DEV))
            moe.register_buffer(f"{n}_scales", w[n].scales.to(DEV))
            moe.register_buffer(f"{n}_biases", w[n].biases.to(DEV))
        moe.quant = (bits, 64)
        moe.expert_format = "affine"
    for n in ("w1", "w2", "w3"):
        getattr(moe.shared_experts, n).weight = torch.nn.Parameter(c.shared[n].to(DEV), requires_grad=False)
    return moe.to(DEV)


@pytest.mark.parametrize("name", golden_io.names())
def test_golden_cases(name):
    c = golden_io.load(name)
    moe = _moe_from_golden(c)
    y, w, idx = moe(c.x.to(DEV), c.ids.to(DEV), return_routing=True)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(idx.cpu(), c.route_indices), "routing indices differ from the reference's"
    assert torch.allclose(w.cpu(), c.route_weights, rtol=1e-5, atol=1e-6)
    assert y.dtype == c.y.dtype and y.shape == c.y.shape
    assert max_rel_err(y, c.y) < MOE_TOL


# ------------------------------------------------------------------------------ router
@pytest.mark.parametrize("wname,n_tokens", [("fp8_decode", 56), ("fp4_decode", 448), ("prefill_fp8", 2048)])
def test_router_bit_exact_full_width(wname, n_tokens):
    """Full router width (4096 x 256): indices bit-exact, weights close; margins reported."""
    wl = W.WORKLOADS[wname]
    g = torch.Generator().manual_seed(11)
    a = wl.args
    x = torch.randn(n_tokens, a["dim"], generator=g).to(torch.bfloat16)
    gw = torch.randn(a["n_routed_experts"], a["dim"], generator=g) * 0.02
    gb = torch.randn(a["n_routed_experts"], generator=g) * 0.02
    if wl.zipf_alpha:
        gb = gb + W.zipf_offsets(a["n_routed_experts"], wl.zipf_alpha, g)
    args = DSparkArgs.from_dict(a)
    moe = MoE(args, 0)
    moe.gate.weight = gw.to(DEV)
    moe.gate.bias = gb.to(DEV)
    w, idx = moe.gate(x.to(DEV))
    ref_w, ref_idx = oracle.gate_forward(x, gw, topk=a["n_activated_experts"], score_func=a["score_func"],
                                         route_scale=a["route_scale"], bias=gb)
    # A token whose k-th and (k+1)-th biased scores lie within a few fp32 ulps of each other
    # can legitimately flip with the last bit of the activation function; such near-ties are
    # counted (and must be rare), every other token must match bit for bit.
    margin = oracle.topk_margin(x, gw, gb, a["n_activated_experts"], a["score_func"])
    clear = margin > 1e-6
    assert float(clear.float().mean()) > 0.99
    assert torch.equal(idx.cpu()[clear], ref_idx[clear])
    assert torch.allclose(w.cpu()[clear], ref_w[clear], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("score_func", ["softmax", "sigmoid", "sqrtsoftplus"])
def test_router_score_functions(score_func):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(33, 384, generator=g)
    gw = torch.randn(40, 384, generator=g) * 0.05
    gb = torch.randn(40, generator=g) * 0.05
    args = DSparkArgs(dim=384, n_routed_experts=40, n_activated_experts=5, score_func=score_func, route_scale=1.7,
                      n_hash_layers=0)
    moe = MoE(args, 0)
    moe.gate.weight = gw.to(DEV)
    moe.gate.bias = gb.to(DEV)
    w, idx = moe.gate(x.to(DEV))
    ref_w, ref_idx = oracle.gate_forward(x, gw, topk=5, score_func=score_func, route_scale=1.7, bias=gb)
    assert torch.equal(idx.cpu(), ref_idx)
    assert torch.allclose(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)


def test_router_hash_anchor_broadcast_and_int64_ids():
    g = torch.Generator().manual_seed(6)
    args = DSparkArgs(dim=128, n_routed_experts=8, n_activated_experts=2, vocab_size=50, n_hash_layers=2,
                      score_func="sqrtsoftplus", route_scale=1.5)
    moe = MoE(args, 1)
    moe.gate.weight = (torch.randn(8, 128, generator=g) * 0.1).to(DEV)
    t2e = torch.stack([torch.randperm(8, generator=g)[:2] for _ in range(50)]).to(torch.int32)
    moe.gate.tid2eid = t2e.to(DEV)
    x = torch.randn(7, 128, generator=g)
    for ids in (torch.tensor([17]), torch.randint(0, 50, (7,), generator=g)):
        w, idx = moe.gate(x.to(DEV), ids.to(DEV))  # int64 ids
        ref_w, ref_idx = oracle.gate_forward(x, moe.gate.weight.cpu(), topk=2, score_func="sqrtsoftplus",
                                             route_scale=1.5, tid2eid=t2e, input_ids=ids)
        assert torch.equal(idx.cpu(), ref_idx)
        assert torch.allclose(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------------------ permute
def _permute(idx: torch.Tensor, E: int):
    L = _lib.lib()
    P = idx.numel()
    d = idx.to(DEV).to(torch.int32).contiguous()
    counts = torch.empty(E, dtype=torch.int32, device=DEV)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=DEV)
    perm = torch.empty(max(P, 1), dtype=torch.int32, device=DEV)
    inv = torch.empty(max(P, 1), dtype=torch.int32, device=DEV)
    wsb = L.dsm_permute_workspace_bytes(P, E)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    _lib.check(L.dsm_permute(d.data_ptr(), P, E, counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
                             inv.data_ptr(), ws.data_ptr(), wsb, _lib.stream_ptr()))
    torch.cuda.synchronize()
    return counts.cpu(), offsets.cpu(), perm[:P].cpu(), inv[:P].cpu()


@pytest.mark.parametrize("n_tokens,topk,E", [(1, 1, 1), (7, 2, 16), (56, 6, 256), (448, 6, 256), (3000, 8, 256),
                                             (16384, 8, 256), (100, 3, 1024), (5, 4, 7)])
def test_permute_bit_exact(n_tokens, topk, E):
    g = torch.Generator().manual_seed(n_tokens * 31 + E)
    if n_tokens * topk >= 10000:  # skewed: some experts empty, some with thousands of pairs
        p = torch.exp(-0.05 * torch.arange(E, dtype=torch.float64))
        idx = torch.multinomial(p.expand(n_tokens, E), topk, replacement=False, generator=g)
    else:
        idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(n_tokens)])
    idx = idx.to(torch.int32)
    got = _permute(idx, E)
    ref = oracle.permutation(idx, E)
    for a, b, what in zip(got, ref, ("counts", "offsets", "perm", "inv")):
        assert torch.equal(a, b), what


def test_permute_empty_and_device_error_flag():
    counts, offsets, perm, inv = _permute(torch.zeros(0, dtype=torch.int32), 8)
    assert int(counts.sum()) == 0 and int(offsets[-1]) == 0
    assert _lib.device_error() == 0
    # an expert id outside [0, E): the kernel skips it and records the error word
    bad = torch.tensor([0, 3, 9, 1], dtype=torch.int32)
    _permute(bad, 8)
    assert _lib.device_error(clear=True) == 0x10
    assert _lib.device_error() == 0


# ------------------------------------------------------------------------------ MoE forward
FORMAT_CASES = [
    dict(base="tiny_hash"),
    dict(base="fp8_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=24),
    dict(base="fp8_decode", dim=384, inter=200, experts=12, topk=3, n_tokens=9),  # ragged (padding) shapes
    dict(base="fp4_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=40),
    dict(base="fp4_decode", dim=512, inter=256, experts=8, topk=2, n_tokens=200),  # > 8 rows per expert
    # many rows per expert on the tensor-memory kernel: units of up to 128 rows (3 row tiles)
    # and of up to 64 rows (16 row tiles: 128-row units would exceed one wave)
    dict(base="fp4_decode", dim=512, inter=384, experts=16, topk=4, n_tokens=700),
    dict(base="fp4_decode", dim=512, inter=2048, experts=16, topk=4, n_tokens=700),
    dict(base="fp8_decode", dim=512, inter=256, experts=16, topk=6, n_tokens=300, wfmt="bf16"),
]


@pytest.mark.parametrize("case", FORMAT_CASES, ids=lambda c: "-".join(str(v) for v in c.values()))
def test_moe_forward_formats(case):
    case = dict(case)
    base = case.pop("base")
    wl = W.WORKLOADS[base] if not case else small_workload(base, **case)
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, DEV)
    ids = t.get("input_ids")
    y, rw, ri = moe(t["x"].to(DEV), ids.to(DEV) if ids is not None else None, return_routing=True)
    ref_y, ref_w, ref_i = oracle_moe(wl, t)
    assert _lib.device_error() == 0
    assert torch.equal(ri.cpu(), ref_i)
    assert max_rel_err(y, ref_y) < MOE_TOL, max_rel_err(y, ref_y)


@pytest.mark.parametrize("bits,n_tokens,gs", [(8, 20, 64), (4, 20, 64), (8, 400, 64), (4, 400, 64), (8, 20, 32),
                                              (8, 40, 128), (4, 40, 128)])
def test_affine_quantize_matches_oracle_and_forward(bits, n_tokens, gs):
    g = torch.Generator().manual_seed(21)
    w = (torch.randn(8, 256, 512, generator=g) * 0.05).to(torch.bfloat16)
    codes, s, b = affine_quantize(w.to(DEV), group_size=gs, bits=bits)
    rc, rs, rb = oracle.affine_quantize(w, gs, bits)
    assert torch.equal(codes.cpu(), rc)
    assert torch.equal(s.cpu().view(torch.int16), rs.view(torch.int16))
    assert torch.equal(b.cpu().view(torch.int16), rb.view(torch.int16))
    # quantised MoE vs the oracle's gather_qmm path
    wl = small_workload("fp8_decode", dim=512, inter=256, experts=8, topk=2, n_tokens=n_tokens, wfmt="bf16", seed=4,
                        zipf_alpha=1.2 if n_tokens > 100 else None)
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, DEV)
    moe.quantize(bits=bits, group_size=gs)
    assert moe.quant == (bits, gs) and "w1" not in moe._buffers and "w1_q" in moe._buffers
    y = moe(t["x"].to(DEV))
    qs = {n: oracle.OracleWeights("affine", getattr(moe, f"{n}_q").cpu(), scales=getattr(moe, f"{n}_scales").cpu(),
                                  biases=getattr(moe, f"{n}_biases").cpu(), group_size=gs, bits=bits)
          for n in ("w1", "w3", "w2")}
    a = t["args"]
    ref = oracle.moe_forward(t["x"], None, gate_weight=t["gate_weight"], topk=2, score_func=a["score_func"],
                             route_scale=a["route_scale"], swiglu_limit=a["swiglu_limit"], w1=qs["w1"], w3=qs["w3"],
                             w2=qs["w2"], shared=(t["shared_w1"], t["shared_w2"], t["shared_w3"]),
                             gate_bias=t["gate_bias"])
    assert max_rel_err(y, ref) < MOE_TOL


def test_shared_expert_standalone():
    g = torch.Generator().manual_seed(8)
    x = torch.randn(13, 384, generator=g).to(torch.bfloat16)
    ws = [(torch.randn(*s, generator=g) * 0.03).to(torch.bfloat16) for s in ((160, 384), (384, 160), (160, 384))]
    from dsm.moe import Expert

    ex = Expert(384, 160, 10.0)
    for n, w in zip(("w1", "w2", "w3"), ws):
        getattr(ex, n).weight = torch.nn.Parameter(w.to(DEV), requires_grad=False)
    y = ex.to(DEV)(x.to(DEV))
    ref = oracle.expert_forward(x, ws[0], ws[1], ws[2], 10.0)
    assert y.dtype == ref.dtype
    assert max_rel_err(y, ref) < MOE_TOL


def _full_size_case(name: str):
    """Runs the full-size workload on the GPU and checks, against the oracle:
    routing indices (near-tie rule, count reported), per-expert counts / offsets /
    permutation of the GPU's routing (bit-exact against ``oracle.permutation``), and the MoE
    output of every token whose routing is clear of near ties."""
    wl = W.WORKLOADS[name]
    t = W.make_moe_tensors(wl, device=DEV)
    moe = W.build_moe(wl, t, DEV)
    y, rw, ri = moe(t["x"], None, return_routing=True)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert bool(torch.isfinite(y.float()).all())
    a = t["args"]
    clear, ref_i, n_ties = check_routing(ri, t["x"], t["gate_weight"], t["gate_bias"], a["n_activated_experts"],
                                         a["score_func"], a["route_scale"])
    print(f"{name}: {n_ties} near-tie tokens of {wl.n_tokens} excluded from the bit-exact routing check")
    got = _permute(ri.cpu(), a["n_routed_experts"])
    for g_, r_, what in zip(got, oracle.permutation(ri.cpu(), a["n_routed_experts"]), ("counts", "offsets", "perm",
                                                                                      "inv")):
        assert torch.equal(g_, r_), what
    return wl, t, moe, y, ri, clear


def test_fp8_decode_full_size_all_tokens():
    """The 56-token fp8 decode block at full size (hidden 4096, 256 experts, top-6): every
    token against the oracle, which dequantises one expert at a time."""
    wl, t, moe, y, ri, clear = _full_size_case("fp8_decode")
    tokens = torch.nonzero(clear).flatten().tolist()
    ref_y, _, ref_i = oracle_moe(wl, t, tokens=tokens)
    assert torch.equal(ri.cpu()[tokens], ref_i)
    assert max_rel_err(y[tokens], ref_y) < MOE_TOL, max_rel_err(y[tokens], ref_y)


def test_fp4_decode_full_size_all_tokens():
    """The 448-token fp4 block (Zipf-skewed routing) at full size: every token against the
    oracle."""
    wl, t, moe, y, ri, clear = _full_size_case("fp4_decode")
    counts = torch.bincount(ri.flatten().long(), minlength=256)
    assert int(counts.max()) > 4 * int(counts.float().mean())  # the skew is there
    tokens = torch.nonzero(clear).flatten().tolist()
    ref_y, _, ref_i = oracle_moe(wl, t, tokens=tokens)
    assert torch.equal(ri.cpu()[tokens], ref_i)
    assert max_rel_err(y[tokens], ref_y) < MOE_TOL, max_rel_err(y[tokens], ref_y)


def test_prefill_full_size():
    """The prefill stress case at its own shapes: 16384 tokens, 256 experts, top-8, hidden
    4096, inter 2048, fp8 128x128 block scales, Zipf(1.2) popularity, on the tcgen05 regime.
    Routing and the permutation are checked for all 16384 tokens; the MoE output on a sample
    that holds rows of the most-loaded expert (first, last and middle), every row of the
    least-loaded busy expert, and random tokens."""
    wl, t, moe, y, ri, clear = _full_size_case("prefill_fp8")
    E = wl.args["n_routed_experts"]
    counts = torch.bincount(ri.cpu().flatten().long(), minlength=E)
    assert int(counts.max()) > 1000 and int(counts.min()) <= 4  # the Zipf skew: >1000 rows and (near-)empty experts
    pairs_tok = torch.arange(ri.shape[0]).repeat_interleave(ri.shape[1])
    flat = ri.cpu().flatten().long()
    e_max = int(counts.argmax())
    busy = torch.nonzero(counts > 0).flatten()
    e_min = int(busy[counts[busy].argmin()])
    tok_max = pairs_tok[flat == e_max]
    tok_min = pairs_tok[flat == e_min]
    g = torch.Generator().manual_seed(99)
    sample = {int(tok_max[0]), int(tok_max[len(tok_max) // 2]), int(tok_max[-1])}
    sample |= {int(v) for v in tok_min[:4]}
    sample |= {int(v) for v in torch.randint(0, wl.n_tokens, (6,), generator=g)}
    tokens = sorted(v for v in sample if bool(clear[v]))
    print(f"prefill: expert {e_max} has {int(counts[e_max])} rows, expert {e_min} {int(counts[e_min])}; "
          f"{int((counts == 0).sum())} experts empty; output checked on tokens {tokens}")
    assert len(tokens) >= 8
    ref_y, _, ref_i = oracle_moe(wl, t, tokens=tokens)
    assert torch.equal(ri.cpu()[tokens], ref_i)
    assert max_rel_err(y[tokens], ref_y) < MOE_TOL, max_rel_err(y[tokens], ref_y)


def test_fp8_decode_batch_invariance():
    """Size-independent property: a token's output does not depend on its batch neighbours."""
    wl = W.WORKLOADS["fp8_decode"]
    t = W.make_moe_tensors(wl, device=DEV)
    moe = W.build_moe(wl, t, DEV)
    y_all = moe(t["x"])
    y_part = moe(t["x"][:9].clone())
    y_one = moe(t["x"][40:41].clone())
    assert torch.equal(y_all[:9], y_part)
    assert torch.equal(y_all[40:41], y_one)
