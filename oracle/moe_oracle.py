"""CPU oracle for the DSpark draft-layer MoE block (test infrastructure only).

This module restates, in PyTorch on the CPU, the arithmetic of the reference MoE block
``dspark_mlx/model/moe.py:31-161`` with the reference's rounding points, plus the dense
Qwen3 MLP ``dspark_mlx/arch/qwen3.py:146-154`` and the expert stacking of
``dspark_mlx/loading.py:88-100``. It is the checker the CUDA path is measured against:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
import it, and the product path never does.

MLX dtype rules it follows (``mx.matmul`` / ``gather_mm`` return the promoted dtype of
their operands, accumulating in fp32; ``gather_qmm`` / quantized matmul return the
activation dtype): with bf16 activations and bf16 expert weights the gate/up/down products
are rounded to bf16; with fp32 (dequantised fp8/fp4) expert weights they stay fp32; the
SwiGLU hidden is always cast back to the activation dtype (``moe.py:142,147``); the combine
is fp32 (``moe.py:159-160``).

Two choices are this oracle's own and are documented where they are made:

* Router logits are computed in fp64 and rounded once to fp32 (``moe.py:63`` computes
  them in fp32 with MLX's own summation order, which cannot be run here). The routing
  parity tests also report the top-k margin so a near-tie cannot pass by luck.
* ``mx.argsort`` tie order is not specified by MLX; ties are broken as a stable ascending
  sort would (equal biased scores keep ascending expert order, so the higher expert id
  ranks higher).

The permutation / per-expert counts are not tensors the reference materialises
(``gather_mm`` takes unsorted ``rhs_indices``, ``moe.py:145-148``); they are defined here
as the stable sort of the flattened ``(token, slot)`` pairs by expert id.

Parity pin status: partial -- pinned by the reference's own known-answer tests and by
golden vectors from the reference's own ``moe.py`` executed over a PyTorch stand-in for the
``mlx`` API; MLX's kernel numerics themselves are unpinned (``mlx`` cannot be installed).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from .formats import affine_dequantize, fp4_weight_dequant, fp8_weight_dequant

__all__ = [
    "sqrtsoftplus",
    "swiglu",
    "gate_forward",
    "topk_margin",
    "permutation",
    "OracleWeights",
    "route_experts",
    "expert_forward",
    "moe_forward",
    "dense_combine",
    "qwen3_mlp",
    "stack_experts",
]


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


def _mm(a: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """``a @ w.T`` accumulated in fp32 and returned in ``out_dtype`` (MLX matmul semantics)."""
    return (a.to(torch.float32) @ w.to(torch.float32).T).to(out_dtype)


def sqrtsoftplus(x: torch.Tensor) -> torch.Tensor:
    """``moe.py:31-34``: ``sqrt(max(x,0) + log1p(exp(-|x|)))``."""
    softplus = torch.clamp(x, min=0.0) + torch.log1p(torch.exp(-x.abs()))
    return torch.sqrt(softplus)


def swiglu(gate: torch.Tensor, up: torch.Tensor, limit: float) -> torch.Tensor:
    """``moe.py:37-44``: fp32; ``up`` clipped to +-limit, ``gate`` capped at limit; silu(gate)*up."""
    gate = gate.to(torch.float32)
    up = up.to(torch.float32)
    if limit > 0:
        up = torch.clamp(up, -limit, limit)
        gate = torch.clamp(gate, max=limit)
    return gate * torch.sigmoid(gate) * up


def _scores(x: torch.Tensor, weight: torch.Tensor, score_func: str) -> torch.Tensor:
    logits = (x.to(torch.float64) @ weight.to(torch.float64).T).to(torch.float32)  # moe.py:63
    if score_func == "softmax":  # moe.py:64-65
        return torch.softmax(logits, dim=-1)
    if score_func == "sigmoid":  # moe.py:66-67
        return torch.sigmoid(logits)
    return sqrtsoftplus(logits)  # moe.py:68-69


def gate_forward(
    x: torch.Tensor,
    weight: torch.Tensor,
    *,
    topk: int,
    score_func: str,
    route_scale: float,
    bias: Optional[torch.Tensor] = None,
    tid2eid: Optional[torch.Tensor] = None,
    input_ids: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``Gate.__call__`` (``moe.py:62-79``) -> ``(weights [N,k] fp32, indices [N,k] int32)``.

    Hash mode (``tid2eid`` given, ``moe.py:71-72``): ``indices = tid2eid[input_ids]``; the ids
    broadcast against the N tokens exactly like ``take_along_axis`` does (length N, or length
    1 for the draft-block case where every token routes like the anchor).
    Score mode (``moe.py:74-75``): indices of the top-k of ``scores + bias`` in ascending
    order (the best expert is the last slot); the bias steers selection only.
    """
    scores = _scores(x, weight, score_func)
    n = scores.shape[0]
    if tid2eid is not None:
        if input_ids is None:
            raise ValueError("hash routing needs input_ids")
        ids = input_ids.reshape(-1).to(torch.int64)
        idx = tid2eid.to(torch.int64)[ids]
        if idx.shape[0] == 1 and n != 1:
            idx = idx.expand(n, idx.shape[1])
        elif idx.shape[0] != n:
            raise ValueError(f"input_ids of length {idx.shape[0]} do not broadcast against {n} tokens")
    else:
        biased = scores + bias.to(torch.float32)
        order = torch.sort(biased, dim=-1, stable=True).indices
        idx = order[..., -topk:]
    weights = torch.gather(scores, -1, idx)  # moe.py:76
    if score_func != "softmax":  # moe.py:77-78
        weights = weights / weights.sum(dim=-1, keepdim=True)
    return weights * route_scale, idx.to(torch.int32)  # moe.py:79


def topk_margin(x, weight, bias, topk: int, score_func: str) -> torch.Tensor:
    """Per token: gap between the k-th and (k+1)-th largest biased score (tie guard)."""
    scores = _scores(x, weight, score_func) + bias.to(torch.float32)
    top = torch.topk(scores.to(torch.float64), topk + 1, dim=-1).values
    return top[:, topk - 1] - top[:, topk]


def permutation(indices: torch.Tensor, n_experts: int):
    """Expert-sorted order of the flattened ``(token, slot)`` pairs.

    Returns ``counts [E]``, ``offsets [E+1]`` (exclusive scan), ``perm [N*k]`` (sorted
    position -> pair id ``token*k + slot``; stable, so pairs of one expert stay in
    ascending pair order) and ``inv [N*k]`` (pair id -> sorted position). All int32.
    """
    flat = indices.reshape(-1).to(torch.int64)
    counts = torch.bincount(flat, minlength=n_experts)
    offsets = torch.zeros(n_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    perm = torch.sort(flat, stable=True).indices
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    return (counts.to(torch.int32), offsets.to(torch.int32), perm.to(torch.int32), inv.to(torch.int32))


@dataclass
class OracleWeights:
    """One stacked expert matrix ``[E, out, in]`` in one of the supported storage formats.

    ``kind`` is ``"dense"`` (``data`` is a bf16 / fp32 tensor), ``"fp8"`` (``data`` e4m3
    codes, ``scales`` fp32 128x128 blocks; the reference dequantises to fp32 at load,
    ``loading.py:7-18``), ``"fp4"`` (packed e2m1 codes, e4m3 group-32 ``scales``, fp32
    per-tensor ``tscale [E]``; dequantised to fp32), or ``"affine"`` (MLX quantized triple,
    used through ``gather_qmm``).
    """

    kind: str
    data: torch.Tensor
    scales: Optional[torch.Tensor] = None
    biases: Optional[torch.Tensor] = None
    tscale: Optional[torch.Tensor] = None
    group_size: int = 64
    bits: int = 8

    def matrix(self, e: int) -> torch.Tensor:
        if self.kind == "dense":
            return self.data[e]
        if self.kind == "fp8":
            return fp8_weight_dequant(self.data[e], self.scales[e])
        if self.kind == "fp4":
            return fp4_weight_dequant(self.data[e], self.scales[e], self.tscale[e])
        if self.kind == "affine":
            return affine_dequantize(self.data[e], self.scales[e], self.biases[e], self.group_size, self.bits)
        raise ValueError(self.kind)

    def product_dtype(self, act_dtype: torch.dtype) -> torch.dtype:
        if self.kind == "dense":
            return torch.promote_types(act_dtype, self.data.dtype)
        if self.kind == "affine":
            return act_dtype  # gather_qmm returns the activation dtype
        return torch.promote_types(act_dtype, torch.float32)  # fp32 after host dequant


def route_experts(x: torch.Tensor, indices: torch.Tensor, w1: OracleWeights, w3: OracleWeights,
                  w2: OracleWeights, limit: float) -> torch.Tensor:
    """``MoE._route_experts`` (``moe.py:132-149``) -> ``o [N, k, dim]``.

    ``gather_mm(x[N,1,1,dim], w.swapaxes(-1,-2), rhs_indices=idx)`` is one independent
    vector-matrix product per ``(token, slot)``; they are evaluated here grouped by expert.
    """
    n, k = indices.shape
    dim = x.shape[-1]
    pdt1 = w1.product_dtype(x.dtype)
    pdt2 = w2.product_dtype(x.dtype)
    out = torch.zeros(n, k, dim, dtype=pdt2)
    for e in torch.unique(indices).tolist():
        tok, slot = torch.nonzero(indices == e, as_tuple=True)
        xs = x[tok]
        g = _mm(xs, w1.matrix(e), pdt1)
        u = _mm(xs, w3.matrix(e), w3.product_dtype(x.dtype))
        h = swiglu(g, u, limit).to(x.dtype)  # moe.py:142,147
        out[tok, slot] = _mm(h, w2.matrix(e), pdt2)
    return out


def expert_forward(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor,
                   limit: float) -> torch.Tensor:
    """``Expert.__call__`` (``moe.py:95-97``), the always-on shared expert (nn.Linear layout)."""
    g = _mm(x, w1, torch.promote_types(x.dtype, w1.dtype))
    u = _mm(x, w3, torch.promote_types(x.dtype, w3.dtype))
    h = swiglu(g, u, limit).to(x.dtype)
    return _mm(h, w2, torch.promote_types(x.dtype, w2.dtype))


def moe_forward(x: torch.Tensor, input_ids: Optional[torch.Tensor], *, gate_weight: torch.Tensor,
                topk: int, score_func: str, route_scale: float, swiglu_limit: float,
                w1: OracleWeights, w3: OracleWeights, w2: OracleWeights,
                shared: Tuple[torch.Tensor, torch.Tensor, torch.Tensor],
                gate_bias: Optional[torch.Tensor] = None, tid2eid: Optional[torch.Tensor] = None,
                return_routing: bool = False):
    """``MoE.__call__`` (``moe.py:151-161``): flatten, gate, route, fp32 combine, + shared, cast."""
    shape, in_dtype = x.shape, x.dtype
    dim = shape[-1]
    x2 = x.reshape(-1, dim)
    ids = input_ids.reshape(-1) if input_ids is not None else None
    weights, indices = gate_forward(x2, gate_weight, topk=topk, score_func=score_func,
                                    route_scale=route_scale, bias=gate_bias, tid2eid=tid2eid,
                                    input_ids=ids)
    o = route_experts(x2, indices, w1, w3, w2, swiglu_limit)
    y = (o.to(torch.float32) * weights[..., None]).sum(dim=-2)  # moe.py:159
    s1, s2, s3 = shared
    y = y + expert_forward(x2, s1, s2, s3, swiglu_limit).to(torch.float32)  # moe.py:160
    y = y.to(in_dtype).reshape(shape)  # moe.py:161
    if return_routing:
        return y, weights, indices
    return y


def dense_combine(x, w1, w2, w3, weights, indices, limit):
    """The O(E) loop the reference pins its sparse path against (``tests/test_moe_gather_mm.py:36-44``)."""
    y = torch.zeros(x.shape, dtype=torch.float32)
    for e in range(w1.shape[0]):
        h = swiglu(_mm(x, w1[e], torch.promote_types(x.dtype, w1.dtype)),
                   _mm(x, w3[e], torch.promote_types(x.dtype, w3.dtype)), limit)
        oe = _mm(h.to(x.dtype), w2[e], torch.promote_types(x.dtype, w2.dtype))
        w_e = torch.where(indices == e, weights, torch.zeros_like(weights)).sum(-1, keepdim=True)
        y = y + oe.to(torch.float32) * w_e
    return y


def qwen3_mlp(x: torch.Tensor, gate: OracleWeights, up: OracleWeights, down: OracleWeights) -> torch.Tensor:
    """``Qwen3MLP.__call__`` (``arch/qwen3.py:153-154``) after ``quantize_drafter`` (``quant.py:36-41``).

    ``down(silu(gate(x)) * up(x))`` with no clamp; each QuantizedLinear returns the
    activation dtype and each elementwise op (``sigmoid``, the two products) rounds to it.
    """
    dt = x.dtype
    g = _mm(x, gate.matrix(0), gate.product_dtype(dt))
    u = _mm(x, up.matrix(0), up.product_dtype(dt))
    sig = torch.sigmoid(g.to(torch.float32)).to(g.dtype)
    s = (g.to(torch.float32) * sig.to(torch.float32)).to(g.dtype)
    h = (s.to(torch.float32) * u.to(torch.float32)).to(torch.promote_types(g.dtype, u.dtype))
    return _mm(h, down.matrix(0), down.product_dtype(h.dtype))


def stack_experts(params: dict) -> dict:
    """``_stack_moe_experts`` (``loading.py:88-100``): ``...ffn.experts.{e}.wK.weight`` -> ``...ffn.wK``."""
    import re

    pat = re.compile(r"^(.*\.ffn)\.experts\.(\d+)\.(w[123])\.weight$")
    groups = {}
    for key in [k for k in params if pat.match(k)]:
        m = pat.match(key)
        groups.setdefault((m.group(1), m.group(3)), {})[int(m.group(2))] = params.pop(key)
    for (prefix, wk), by_eid in groups.items():
        params[f"{prefix}.{wk}"] = torch.stack([by_eid[e] for e in sorted(by_eid)], dim=0)
    return params
