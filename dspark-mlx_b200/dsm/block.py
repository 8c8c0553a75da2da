"""The MoE with its neighbours in the DSpark draft block: ``DSparkFFN``.

``DSparkBlock.__call__`` (``dspark_mlx/model/block.py:83-86``) wraps the MoE in
hyper-connection mixing and the FFN's RMSNorm:

    residual = x                                    # [b, s, hc, d]
    h, post, comb = hc_pre(x, hc_ffn_fn, hc_ffn_scale, hc_ffn_base)
    h = ffn(ffn_norm(h), input_ids)
    return hc_post(h, residual, post, comb)

``DSparkFFN`` is that sub-layer with the reference's parameter names (``hc_ffn_fn``
``[(2+hc)*hc, hc*dim]``, ``hc_ffn_scale [3]``, ``hc_ffn_base [(2+hc)*hc]``,
``ffn_norm.weight [dim]``, ``ffn`` the :class:`dsm.MoE`). ``hc_pre`` and the RMSNorm run as
one kernel producing the MoE input, ``hc_post`` as one kernel after it; the MoE is the
fused ``dsm_moe_forward``.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .config import DSparkArgs
from .moe import MoE


class RMSNorm(nn.Module):
    """``RMSNorm`` (``dspark_mlx/model/norm_rope.py:22-39``): fp32 weight of ones, ``eps``."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.float32), requires_grad=False)
        self.eps = eps


class DSparkFFN(nn.Module):
    """The FFN sub-layer of a DSpark draft block: ``forward(x [b, s, hc, d], input_ids)``."""

    def __init__(self, args, layer_id: int):
        super().__init__()
        if isinstance(args, dict):
            args = DSparkArgs.from_dict(args)
        self.hc_mult = args.hc_mult
        self.hc_sinkhorn_iters = args.hc_sinkhorn_iters
        self.hc_eps = args.hc_eps
        self.norm_eps = args.norm_eps
        mix = (2 + self.hc_mult) * self.hc_mult
        self.hc_ffn_fn = nn.Parameter(torch.zeros(mix, self.hc_mult * args.dim, dtype=torch.float32),
                                      requires_grad=False)
        self.hc_ffn_base = nn.Parameter(torch.zeros(mix, dtype=torch.float32), requires_grad=False)
        self.hc_ffn_scale = nn.Parameter(torch.zeros(3, dtype=torch.float32), requires_grad=False)
        self.ffn_norm = RMSNorm(args.dim, args.norm_eps)
        self.ffn = MoE(args, layer_id)

    def forward(self, x: torch.Tensor, input_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda:
            raise ValueError("DSparkFFN runs on the GPU only: x must be a CUDA tensor")
        if x.dim() < 2 or x.shape[-2] != self.hc_mult:
            raise ValueError(f"x must be [..., hc_mult={self.hc_mult}, dim], got {tuple(x.shape)}")
        shape, dt = x.shape, x.dtype
        dim = shape[-1]
        xr = x.reshape(-1, self.hc_mult, dim).contiguous()
        n = xr.shape[0]
        dev = x.device
        xn = torch.empty(n, dim, dtype=dt, device=dev)
        post = torch.empty(n, self.hc_mult, dtype=torch.float32, device=dev)
        comb = torch.empty(n, self.hc_mult, self.hc_mult, dtype=torch.float32, device=dev)
        params = [t.detach().to(device=dev, dtype=torch.float32).contiguous()
                  for t in (self.hc_ffn_fn, self.hc_ffn_scale, self.hc_ffn_base, self.ffn_norm.weight)]
        s = stream_ptr()
        L = lib()
        check(L.dsm_hc_pre_norm(ptr(xr), dtype_code(dt), n, self.hc_mult, dim, ptr(params[0]), ptr(params[1]),
                                ptr(params[2]), self.hc_sinkhorn_iters, float(self.norm_eps), float(self.hc_eps),
                                ptr(params[3]), ptr(xn), ptr(post), ptr(comb), s), "dsm_hc_pre_norm")
        h = self.ffn(xn, input_ids)
        out = torch.empty_like(xr)
        check(L.dsm_hc_post(ptr(h), ptr(xr), dtype_code(dt), n, self.hc_mult, dim, ptr(post), ptr(comb), ptr(out),
                            s), "dsm_hc_post")
        return out.reshape(shape)
