"""Qwen3 dense draft-layer MLP (dspark_mlx/arch/qwen3.py:146-154) after quantize_drafter
(dspark_mlx/quant.py:29-45): the GPU module against the oracle's restatement."""

from __future__ import annotations

import pytest
import torch

from dsm import _lib, workloads as W
from dsm.qwen3 import Qwen3MLP
from helpers import MOE_TOL, max_rel_err
import oracle

DEV = "cuda"


def _oracle_weights(mlp: Qwen3MLP):
    out = []
    for p in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
        if p.quant is None:
            out.append(oracle.OracleWeights("dense", p.weight.detach().cpu().unsqueeze(0)))
        else:
            bits, gs = p.quant
            out.append(oracle.OracleWeights("affine", p.q.cpu().unsqueeze(0), scales=p.scales.cpu().unsqueeze(0),
                                            biases=p.biases.cpu().unsqueeze(0), group_size=gs, bits=bits))
    return out


def test_predicate_skips_projections_whose_input_dim_is_not_a_group_multiple():
    # quant.py:36-39: a Linear is quantised only when weight.shape[-1] % group_size == 0
    mlp = Qwen3MLP({"hidden_size": 96, "intermediate_size": 128})
    assert mlp.gate_proj.quantize(8, 64) is False and mlp.gate_proj.quant is None
    assert mlp.up_proj.quantize(8, 64) is False
    assert tuple(mlp.down_proj.weight.shape) == (96, 128)


def test_constructor_mirrors_reference_shapes():
    mlp = Qwen3MLP({"hidden_size": 2560, "intermediate_size": 9728})
    assert tuple(mlp.gate_proj.weight.shape) == (9728, 2560)
    assert tuple(mlp.up_proj.weight.shape) == (9728, 2560)
    assert tuple(mlp.down_proj.weight.shape) == (2560, 9728)


def _case(hidden, inter, n_tokens, wfmt="affine8", seed=0):
    wl = W.Workload("qwen3_small", dict(hidden_size=hidden, intermediate_size=inter), n_tokens=n_tokens, wfmt=wfmt,
                    seed=seed)
    return wl, W.make_qwen3_tensors(wl, device="cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("shape", [(512, 384, 24), (640, 1088, 7), (384, 512, 113)])
def test_quantised_mlp_matches_oracle(bits, shape):
    hidden, inter, n = shape
    wl, t = _case(hidden, inter, n, seed=bits + n)
    mlp = W.build_qwen3_mlp(wl, t, DEV, bits=bits)
    assert all(p.quant == (bits, 64) for p in (mlp.gate_proj, mlp.up_proj, mlp.down_proj))
    # the codes are MLX's: bit-exact against the oracle's quantize
    rq, rs, rb = oracle.affine_quantize(t["gate_proj"], 64, bits)
    assert torch.equal(mlp.gate_proj.q.cpu(), rq)
    assert torch.equal(mlp.gate_proj.scales.cpu().view(torch.int16), rs.view(torch.int16))
    assert torch.equal(mlp.gate_proj.biases.cpu().view(torch.int16), rb.view(torch.int16))
    y = mlp(t["x"].to(DEV))
    torch.cuda.synchronize()
    ref = oracle.qwen3_mlp(t["x"], *_oracle_weights(mlp))
    assert y.dtype == ref.dtype == torch.bfloat16 and y.shape == ref.shape
    assert max_rel_err(y, ref) < MOE_TOL, max_rel_err(y, ref)


@pytest.mark.gpu
def test_dense_bf16_mlp_matches_oracle():
    wl, t = _case(512, 768, 30, wfmt="bf16", seed=5)
    mlp = W.build_qwen3_mlp(wl, t, DEV)
    assert mlp.gate_proj.quant is None
    y = mlp(t["x"].to(DEV))
    ref = oracle.qwen3_mlp(t["x"], *_oracle_weights(mlp))
    assert y.dtype == ref.dtype
    assert max_rel_err(y, ref) < MOE_TOL, max_rel_err(y, ref)


@pytest.mark.gpu
def test_full_size_q8_mlp_matches_oracle():
    """The measured shape: hidden 2560, inter 9728, 8-bit group 64, 112 tokens (16 x 7)."""
    wl = W.WORKLOADS["qwen3_mlp_q8"]
    t = W.make_qwen3_tensors(wl, device="cpu")
    mlp = W.build_qwen3_mlp(wl, t, DEV)
    x = t["x"].to(DEV)
    y = mlp(x)
    y2 = mlp(x)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # deterministic
    ref = oracle.qwen3_mlp(t["x"], *_oracle_weights(mlp))
    assert max_rel_err(y, ref) < MOE_TOL, max_rel_err(y, ref)
    # leading dims are kept: [16, 7, 2560] in, [16, 7, 2560] out
    y3 = mlp(x.reshape(16, 7, -1))
    assert y3.shape == (16, 7, 2560) and torch.equal(y3.reshape(112, -1), y)
    # the K-split down product (fp32 partial slabs added in a fixed order) against the whole-K
    # product the streaming regime keeps: the same sums in another order, so at most a
    # last-bit flip of the bf16 output here and there
    L = _lib.lib()
    try:
        L.dsm_set_expert_regime(1)
        y_whole = mlp(x)
        torch.cuda.synchronize()
    finally:
        L.dsm_set_expert_regime(0)
    assert max_rel_err(y_whole, y) < 1e-2
    assert (y_whole == y).float().mean() > 0.95
