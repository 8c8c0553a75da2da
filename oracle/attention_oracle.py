"""CPU oracle for the DSpark draft attention (test infrastructure only).

Restates, in PyTorch on the CPU with MLX's dtype rules, the draft block's MLA attention in
its ``compress_ratio == 0`` form (``dspark_mlx/model/attention.py``):

* low-rank queries ``wq_a -> q_norm -> wq_b`` with a per-head RMS;
* one shared KV head ``wkv -> kv_norm``;
* interleaved-pair RoPE on the last ``rope_head_dim`` dims (``norm_rope.py:43-77``);
* a sliding-window KV ring buffer (``attention.py:27-57``);
* top-k gathered attention over ``[window || block]`` with a denominator-only sink
  (``dspark_mlx/kernels.py:20-57``);
* the inverse rotation of the output and the grouped low-rank output projection
  (``attention.py:117-129``).

``nn.Linear`` is a matmul accumulated in fp32 with the result in the promoted dtype of
input and weight.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from .block_oracle import rms_norm

__all__ = ["rope_tables", "apply_rotary_emb", "rope_last", "dspark_topk_idxs", "sparse_attn", "KVWindow",
           "linear", "attention_forward"]


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``nn.Linear`` without bias: fp32 accumulation, the promoted dtype out."""
    return (x.to(torch.float32) @ w.to(torch.float32).T).to(torch.promote_types(x.dtype, w.dtype))


def rope_tables(dim: int, seqlen: int, base: float = 10000.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """``precompute_rope`` (``norm_rope.py:43-49``): ``(cos, sin)`` ``[seqlen, dim/2]``."""
    freqs = 1.0 / (base ** (torch.arange(0, dim, 2).to(torch.float32) / dim))
    theta = torch.outer(torch.arange(seqlen).to(torch.float32), freqs)
    return torch.cos(theta), torch.sin(theta)


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Interleaved-pair RoPE (``norm_rope.py:52-77``); position axis 1, x ``[b, s, rd]`` or ``[b, s, h, rd]``."""
    rd = x.shape[-1]
    half, seqlen = rd // 2, x.shape[1]
    xf = x.to(torch.float32).reshape(*x.shape[:-1], half, 2)
    xr, xi = xf[..., 0], xf[..., 1]
    shape = (1, seqlen, half) if x.dim() == 3 else (1, seqlen, 1, half)
    c, s = cos.reshape(shape), sin.reshape(shape)
    if inverse:
        s = -s
    out = torch.stack([xr * c - xi * s, xr * s + xi * c], dim=-1).reshape(x.shape)
    return out.to(x.dtype)


def rope_last(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rd: int, inverse: bool = False) -> torch.Tensor:
    """Rotate only the last ``rd`` dims (``attention.py:60-62``)."""
    return torch.cat([x[..., :-rd], apply_rotary_emb(x[..., -rd:], cos, sin, inverse)], dim=-1)


def dspark_topk_idxs(window_size: int, bsz: int, block_size: int, start_pos: int) -> torch.Tensor:
    """``attention.py:65-69``: the filled window slots, then the block's own rows."""
    win = torch.arange(min(window_size, start_pos + 1))
    block = window_size + torch.arange(block_size)
    row = torch.cat([win, block]).to(torch.int32)
    return row[None, None, :].expand(bsz, block_size, row.shape[0])


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor, topk_idxs: torch.Tensor,
                softmax_scale: float) -> torch.Tensor:
    """``kernels.py:20-57``: gathered single-KV-head attention, denominator-only sink."""
    b, m, h, d = q.shape
    t = topk_idxs.shape[-1]
    mask = topk_idxs != -1
    safe = torch.where(mask, topk_idxs, torch.zeros_like(topk_idxs)).to(torch.int64)
    kv_g = torch.take_along_dim(kv.to(torch.float32), safe.reshape(b, m * t)[:, :, None].expand(b, m * t, d),
                                dim=1).reshape(b, m, t, d)
    qf = q.to(torch.float32)
    scores = (qf @ kv_g.transpose(-1, -2)) * softmax_scale
    scores = torch.where(mask[:, :, None, :], scores, torch.tensor(float("-inf")))
    smax = scores.amax(dim=-1, keepdim=True)
    ex = torch.exp(scores - smax)
    num = ex @ kv_g
    sink = torch.exp(attn_sink.to(torch.float32)[None, None, :, None] - smax)
    denom = ex.sum(dim=-1, keepdim=True) + sink
    return (num / denom).to(q.dtype)


class KVWindow:
    """``DSparkKVCache`` (``attention.py:27-57``): slot ``p % window`` holds position ``p``."""

    def __init__(self, window_size: int):
        self.window_size = window_size
        self.window: Optional[torch.Tensor] = None

    def prefill(self, main_kv: torch.Tensor) -> None:
        b, seqlen, d = main_kv.shape
        win = self.window_size
        if seqlen <= win:
            self.window = torch.cat([main_kv, torch.zeros(b, win - seqlen, d, dtype=main_kv.dtype)], dim=1)
        else:
            cutoff = seqlen % win
            last = main_kv[:, seqlen - win:]
            self.window = torch.cat([last[:, win - cutoff:], last[:, :win - cutoff]], dim=1)

    def update(self, start_pos: int, v: torch.Tensor) -> None:
        sel = torch.arange(self.window_size) == (start_pos % self.window_size)
        self.window = torch.where(sel[None, :, None], v[:, None, :], self.window)


@dataclass
class AttnDims:
    n_heads: int
    head_dim: int
    rope_head_dim: int
    o_groups: int
    o_lora_rank: int
    window_size: int
    eps: float


def attention_forward(p: Dict[str, torch.Tensor], dims: AttnDims, x: torch.Tensor, start_pos: int,
                      main_x: torch.Tensor, cache: KVWindow, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``DSparkAttention.__call__`` (``attention.py:99-129``). ``p`` holds ``wq_a``,
    ``q_norm``, ``wq_b``, ``wkv``, ``kv_norm``, ``wo_a``, ``wo_b``, ``attn_sink``."""
    rd = dims.rope_head_dim
    b, seqlen, _ = main_x.shape
    main_kv = rms_norm(linear(main_x, p["wkv"]), p["kv_norm"], dims.eps)
    main_kv = rope_last(main_kv, cos[start_pos:start_pos + seqlen], sin[start_pos:start_pos + seqlen], rd)
    if start_pos == 0:
        cache.prefill(main_kv)
        return x
    block_size = x.shape[1]
    bcos = cos[start_pos + seqlen:start_pos + seqlen + block_size]
    bsin = sin[start_pos + seqlen:start_pos + seqlen + block_size]
    q = linear(rms_norm(linear(x, p["wq_a"]), p["q_norm"], dims.eps), p["wq_b"])
    q = q.reshape(b, block_size, dims.n_heads, dims.head_dim)
    ms = (q * q).mean(dim=-1, keepdim=True) + dims.eps  # in q's dtype, as MLX evaluates it
    q = q * torch.rsqrt(ms.to(torch.float32)).to(ms.dtype)
    q = rope_last(q, bcos, bsin, rd)
    kv = rope_last(rms_norm(linear(x, p["wkv"]), p["kv_norm"], dims.eps), bcos, bsin, rd)
    cache.update(start_pos, main_kv[:, 0])
    kv_full = torch.cat([cache.window, kv], dim=1)
    topk = dspark_topk_idxs(dims.window_size, b, block_size, start_pos)
    o = sparse_attn(q, kv_full, p["attn_sink"], topk, dims.head_dim ** -0.5)
    o = rope_last(o, bcos, bsin, rd, inverse=True)
    o = o.reshape(b, block_size, dims.o_groups, -1)
    wo_a = p["wo_a"].reshape(dims.o_groups, dims.o_lora_rank, -1)
    dt = torch.promote_types(o.dtype, wo_a.dtype)
    o = (o.to(dt)[..., None, :] * wo_a.to(dt)[None, None, :, :, :]).sum(dim=-1)
    return linear(o.reshape(b, block_size, dims.o_groups * dims.o_lora_rank), p["wo_b"])
