"""CPU restatement of the MoE's neighbours in the DSpark draft block (test infrastructure
only: the checker the CUDA path is compared against, never part of the product).

The FFN half of ``DSparkBlock.__call__`` (``dspark_mlx/model/block.py:83-86``) is

    residual = x                                   # [b, s, hc, d] hyper-connection copies
    h, post, comb = hc_pre(x, hc_ffn_fn, hc_ffn_scale, hc_ffn_base)
    h = ffn(ffn_norm(h), input_ids)                # the MoE
    return hc_post(h, residual, post, comb)

restated here in PyTorch with MLX's dtype rules: every reduction and mix in fp32, results
cast back to the activation dtype where the reference casts them.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

__all__ = ["hc_split_sinkhorn", "hc_pre", "hc_post", "rms_norm", "ffn_sublayer"]


def hc_split_sinkhorn(mixes: torch.Tensor, hc_scale: torch.Tensor, hc_base: torch.Tensor, hc: int, iters: int,
                      eps: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``kernels.hc_split_sinkhorn`` (``dspark_mlx/kernels.py:60-85``): the first ``hc`` mixes
    give ``pre`` (sigmoid + eps), the next ``hc`` give ``post`` (2 sigmoid), the last ``hc*hc``
    a row-softmax matrix normalised by alternating column / row sums (``iters`` column passes,
    ``iters - 1`` row passes) toward doubly stochastic."""
    m = mixes.to(torch.float32)
    pre = torch.sigmoid(m[..., :hc] * hc_scale[0] + hc_base[:hc]) + eps
    post = 2.0 * torch.sigmoid(m[..., hc:2 * hc] * hc_scale[1] + hc_base[hc:2 * hc])
    logits = (m[..., 2 * hc:] * hc_scale[2] + hc_base[2 * hc:]).reshape(*m.shape[:-1], hc, hc)
    comb = torch.softmax(logits, dim=-1) + eps
    comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        comb = comb / (comb.sum(dim=-1, keepdim=True) + eps)
        comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    return pre, post, comb


def hc_pre(x: torch.Tensor, hc_fn: torch.Tensor, hc_scale: torch.Tensor, hc_base: torch.Tensor, hc: int,
           iters: int, norm_eps: float, hc_eps: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``hyper.hc_pre`` (``dspark_mlx/model/hyper.py:24-42``): ``[b, s, hc, d] -> [b, s, d]``.

    The mix projections of the flattened copies are scaled by their inverse RMS; ``pre``
    weights the copies' sum (in fp32, cast to x's dtype)."""
    shape = x.shape
    xf = x.reshape(*shape[:2], -1).to(torch.float32)
    inv_rms = torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + norm_eps)
    mixes = (xf @ hc_fn.to(torch.float32).T) * inv_rms
    pre, post, comb = hc_split_sinkhorn(mixes, hc_scale.to(torch.float32), hc_base.to(torch.float32), hc, iters,
                                        hc_eps)
    y = (pre[..., None] * xf.reshape(shape)).sum(dim=2)
    return y.to(x.dtype), post, comb


def hc_post(h: torch.Tensor, residual: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """``hyper.hc_post`` (``dspark_mlx/model/hyper.py:45-51``): ``[b, s, d] -> [b, s, hc, d]``,
    ``out[c] = post[c] * h + sum_a comb[a, c] * residual[a]`` in fp32, cast to h's dtype."""
    term1 = post[..., None] * h[..., None, :].to(torch.float32)
    term2 = (comb[..., :, :, None] * residual[..., :, None, :].to(torch.float32)).sum(dim=-3)
    return (term1 + term2).to(h.dtype)


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """``RMSNorm.__call__`` (``dspark_mlx/model/norm_rope.py:22-39``): fp32 normalisation,
    optional fp32 weight, cast back to x's dtype."""
    xf = x.to(torch.float32)
    xf = xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
    if weight is not None:
        xf = weight.to(torch.float32) * xf
    return xf.to(x.dtype)


def ffn_sublayer(x: torch.Tensor, input_ids: Optional[torch.Tensor], *, hc_fn, hc_scale, hc_base, norm_weight,
                 moe: Callable, hc: int, iters: int, norm_eps: float, hc_eps: float) -> torch.Tensor:
    """The FFN half of ``DSparkBlock.__call__`` (``dspark_mlx/model/block.py:83-86``)."""
    h, post, comb = hc_pre(x, hc_fn, hc_scale, hc_base, hc, iters, norm_eps, hc_eps)
    h = moe(rms_norm(h, norm_weight, norm_eps), input_ids)
    return hc_post(h, x, post, comb)
