"""The Qwen3 dense DSpark draft layer's MLP on B200: ``Qwen3MLP``.

Mirrors ``dspark_mlx/arch/qwen3.py:146-154`` -- ``gate_proj``/``up_proj``/``down_proj``
(``nn.Linear`` layout ``[out, in]``, no bias) and ``mlp(x) = down(silu(gate(x)) * up(x))``
with no clamp -- and the quantisation ``quantize_drafter`` applies to it
(``dspark_mlx/quant.py:29-45``: every Linear whose input dimension is a multiple of the
group size becomes an MLX affine QuantizedLinear).

The MLP runs on the grouped expert kernels as a single expert holding every token: one
staging launch, the fused gate/up product with ``silu(g) * u`` in its epilogue (MLX's bf16
elementwise rounding: ``sigmoid``, the two products), and the down product. Quantised
projections stream MLX's own 8/4-bit codes, scales and biases.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .weights import PackedMatrix, affine_quantize, pack


class Projection(nn.Module):
    """A bias-free projection: dense ``weight [out, in]``, or after :meth:`quantize` MLX affine
    ``q``/``scales``/``biases`` (the QuantizedLinear triple)."""

    def __init__(self, in_dim: int, out_dim: int):
        super().__init__()
        self.in_dim, self.out_dim = in_dim, out_dim
        self.weight = nn.Parameter(torch.empty(out_dim, in_dim, dtype=torch.float32), requires_grad=False)
        nn.init.uniform_(self.weight, -in_dim ** -0.5, in_dim ** -0.5)
        self.quant: Optional[Tuple[int, int]] = None
        self._cache = None

    def quantize(self, bits: int, group_size: int) -> bool:
        """Quantise in place when ``in_dim % group_size == 0`` (``quant.py:36-39``); returns whether it did."""
        if self.quant is not None or self.in_dim % group_size:
            return False
        q, s, b = affine_quantize(self.weight.detach().cuda(), group_size=group_size, bits=bits)
        del self.weight
        self.register_buffer("q", q)
        self.register_buffer("scales", s)
        self.register_buffer("biases", b)
        self.quant = (bits, group_size)
        return True

    def packed(self) -> PackedMatrix:
        srcs = (self.weight,) if self.quant is None else (self.q, self.scales, self.biases)
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in srcs)
        if self._cache is None or self._cache[0] != key:
            if self.quant is None:
                p = pack("dense", data=self.weight.detach(), device=self.weight.device)
            else:
                bits, gs = self.quant
                p = pack("affine", data=self.q, scales=self.scales, biases=self.biases, group_size=gs, bits=bits,
                         device=self.q.device)
            self._cache = (key, p)
        return self._cache[1]

    def product_dtype(self, x_dtype: torch.dtype) -> torch.dtype:
        """dtype of ``proj(x)`` in MLX: a QuantizedLinear returns x's dtype; a Linear promotes."""
        if self.quant is not None:
            return x_dtype
        return torch.promote_types(x_dtype, self.weight.dtype)


class Qwen3MLP(nn.Module):
    """``Qwen3MLP(args)``: ``args`` carries ``hidden_size`` and ``intermediate_size`` (a
    ``Qwen3DSparkArgs``, or any object / dict with those fields)."""

    def __init__(self, args):
        super().__init__()
        get = (lambda k: args[k]) if isinstance(args, dict) else (lambda k: getattr(args, k))
        h, i = int(get("hidden_size")), int(get("intermediate_size"))
        self.gate_proj = Projection(h, i)
        self.up_proj = Projection(h, i)
        self.down_proj = Projection(i, h)
        self._ws: Optional[torch.Tensor] = None

    def quantize(self, bits: int = 8, group_size: int = 64) -> "Qwen3MLP":
        """``nn.quantize`` of the three projections with ``quantize_drafter``'s predicate."""
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            p.quantize(bits, group_size)
        if (self.gate_proj.quant is None) != (self.up_proj.quant is None):
            raise ValueError("gate_proj and up_proj must share a format (both quantised or both dense)")
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise ValueError("Qwen3MLP runs on the GPU only: x must be a CUDA tensor")
        shape, dt = x.shape, x.dtype
        x2 = x.reshape(-1, shape[-1]).contiguous()
        pg, pu, pd = self.gate_proj.packed(), self.up_proj.packed(), self.down_proj.packed()
        if pg.wfmt != pu.wfmt or pg.group_size != pu.group_size:
            raise ValueError("gate_proj and up_proj must share a weight format")
        n = x2.shape[0]
        g_dt = self.gate_proj.product_dtype(dt)
        u_dt = self.up_proj.product_dtype(dt)
        h_dt = torch.promote_types(g_dt, u_dt)
        o_dt = self.down_proj.product_dtype(h_dt)
        # bit 0: g and u rounded to bf16; bit 1: h rounded to bf16 (the elementwise ops' dtype)
        rgu = int(g_dt == torch.bfloat16 and u_dt == torch.bfloat16) | (2 if h_dt == torch.bfloat16 else 0)
        act = _lib.ACT_SILU_MUL_BF16 if g_dt == torch.bfloat16 else _lib.ACT_SWIGLU_CLAMP
        y = torch.empty(n, pd.rows, dtype=o_dt, device=x.device)
        if n == 0:
            return y.reshape(*shape[:-1], pd.rows)
        L = lib()
        need = L.dsm_dense_mlp_workspace_bytes(n, pg.cols, pg.rows)
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        check(L.dsm_dense_mlp(ptr(x2), dtype_code(dt), n, pg.cols, pg.rows, pg.wfmt, pg.group_size, ptr(pg.packed),
                              ptr(pu.packed), ptr(pd.packed), act, 0.0, rgu, int(o_dt == torch.bfloat16), ptr(y),
                              dtype_code(o_dt), ptr(self._ws), self._ws.numel(), stream_ptr()), "dsm_dense_mlp")
        return y.reshape(*shape[:-1], pd.rows)
