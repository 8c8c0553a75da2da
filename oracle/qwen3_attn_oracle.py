"""CPU oracle for the Qwen3 DSpark draft attention (test infrastructure only).

Restates ``Qwen3DSparkAttention`` (``dspark_mlx/arch/qwen3.py:84-143``) in PyTorch on the
CPU with MLX's dtype rules:
* grouped-query attention, ``num_attention_heads`` query heads over ``num_key_value_heads``
  KV heads;
* per-head RMSNorm on q and k;
* NeoX half-split RoPE (``qwen3.py:64-81``), whose tables are cast to the activation dtype
  before the rotation;
* unmasked scaled dot-product attention of the draft block over ``[context || block]``;
* the cached form, whose context K/V are projected once and reused (``qwen3.py:122-143``).

The attention is softmax(q k^T * scale) v accumulated in fp32 with q's dtype out, as
``mx.fast.scaled_dot_product_attention`` documents.

The whole draft layer (``Qwen3DSparkLayer``, ``qwen3.py:157-176``) adds the pre-attention and
pre-MLP RMSNorms, the residual adds and the MLP (``qwen3.py:146-154``).
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from .attention_oracle import linear
from .block_oracle import rms_norm

__all__ = ["qwen3_rope_tables", "qwen3_apply_rope", "qwen3_sdpa", "qwen3_attention", "qwen3_context_kv",
           "qwen3_attend_cached", "qwen3_layer", "qwen3_layer_cached", "qwen3_layer_params", "qwen3_project_context",
           "qwen3_backbone"]


def qwen3_rope_tables(position_ids: torch.Tensor, head_dim: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``rope_tables`` (``qwen3.py:76-81``): cos/sin ``[len(position_ids), head_dim]``."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).to(torch.float32) / head_dim))
    freqs = position_ids.to(torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return torch.cos(emb), torch.sin(emb)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def qwen3_apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``_apply_rope`` (``qwen3.py:69-73``): x ``[b, seq, heads, hd]``, all in x's dtype."""
    c = cos[None, :, None, :].to(x.dtype)
    s = sin[None, :, None, :].to(x.dtype)
    return x * c + _rotate_half(x) * s


def qwen3_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Unmasked attention, q ``[b, nh, q, hd]`` over k, v ``[b, nkv, n, hd]``."""
    rep = q.shape[1] // k.shape[1]
    kf = k.to(torch.float32).repeat_interleave(rep, dim=1)
    vf = v.to(torch.float32).repeat_interleave(rep, dim=1)
    s = (q.to(torch.float32) @ kf.transpose(-1, -2)) * scale
    return (torch.softmax(s, dim=-1) @ vf).to(q.dtype)


def _heads_norm(x: torch.Tensor, heads: int, hd: int, w: torch.Tensor, eps: float) -> torch.Tensor:
    b, n, _ = x.shape
    return rms_norm(x.reshape(b, n, heads, hd), w, eps)


def qwen3_attention(p: Dict[str, torch.Tensor], nh: int, nkv: int, hd: int, eps: float, hidden: torch.Tensor,
                    target_ctx: torch.Tensor, cos_full: torch.Tensor, sin_full: torch.Tensor) -> torch.Tensor:
    """``Qwen3DSparkAttention.__call__`` (``qwen3.py:97-116``)."""
    b, q, _ = hidden.shape
    ctx = target_ctx.shape[1]
    qh = _heads_norm(linear(hidden, p["q_proj"]), nh, hd, p["q_norm"], eps)
    k = rms_norm(torch.cat([linear(target_ctx, p["k_proj"]), linear(hidden, p["k_proj"])], dim=1)
                 .reshape(b, ctx + q, nkv, hd), p["k_norm"], eps)
    v = torch.cat([linear(target_ctx, p["v_proj"]), linear(hidden, p["v_proj"])], dim=1).reshape(b, ctx + q, nkv, hd)
    qh = qwen3_apply_rope(qh, cos_full[-q:], sin_full[-q:])
    k = qwen3_apply_rope(k, cos_full, sin_full)
    out = qwen3_sdpa(qh.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), hd ** -0.5)
    return linear(out.transpose(1, 2).reshape(b, q, nh * hd), p["o_proj"])


def qwen3_context_kv(p: Dict[str, torch.Tensor], nkv: int, hd: int, eps: float, proj_ctx: torch.Tensor,
                     cos: torch.Tensor, sin: torch.Tensor):
    """``context_kv`` (``qwen3.py:122-128``): RoPE'd context K, V ``[b, nkv, n, hd]``."""
    k = _heads_norm(linear(proj_ctx, p["k_proj"]), nkv, hd, p["k_norm"], eps)
    b, n, _ = proj_ctx.shape
    v = linear(proj_ctx, p["v_proj"]).reshape(b, n, nkv, hd)
    k = qwen3_apply_rope(k, cos, sin)
    return k.transpose(1, 2), v.transpose(1, 2)


def qwen3_attend_cached(p: Dict[str, torch.Tensor], nh: int, nkv: int, hd: int, eps: float, noise: torch.Tensor,
                        ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor], cos: torch.Tensor,
                        sin: torch.Tensor) -> torch.Tensor:
    """``attend_cached`` (``qwen3.py:130-143``): the noise block over ``[cached context || block]``."""
    b, q, _ = noise.shape
    qh = _heads_norm(linear(noise, p["q_proj"]), nh, hd, p["q_norm"], eps)
    nk = _heads_norm(linear(noise, p["k_proj"]), nkv, hd, p["k_norm"], eps)
    nv = linear(noise, p["v_proj"]).reshape(b, q, nkv, hd)
    qh = qwen3_apply_rope(qh, cos, sin).transpose(1, 2)
    nk = qwen3_apply_rope(nk, cos, sin).transpose(1, 2)
    nv = nv.transpose(1, 2)
    k = nk if ctx_k is None else torch.cat([ctx_k, nk], dim=2)
    v = nv if ctx_v is None else torch.cat([ctx_v, nv], dim=2)
    out = qwen3_sdpa(qh, k, v, hd ** -0.5)
    return linear(out.transpose(1, 2).reshape(b, q, nh * hd), p["o_proj"])


def _qwen3_mlp(p: Dict[str, torch.Tensor], x: torch.Tensor) -> torch.Tensor:
    """``Qwen3MLP.__call__`` (``qwen3.py:153-154``) on dense weights: ``nn.silu`` is
    ``x * sigmoid(x)``, each elementwise op rounded to the activation dtype."""
    g = linear(x, p["gate_proj"])
    u = linear(x, p["up_proj"])
    sig = torch.sigmoid(g.to(torch.float32)).to(g.dtype)
    s = (g.to(torch.float32) * sig.to(torch.float32)).to(g.dtype)
    h = (s.to(torch.float32) * u.to(torch.float32)).to(torch.promote_types(g.dtype, u.dtype))
    return linear(h, p["down_proj"])


def _add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a + b`` as MLX evaluates it: in the promoted dtype, one rounding."""
    dt = torch.promote_types(a.dtype, b.dtype)
    return (a.to(torch.float32) + b.to(torch.float32)).to(dt)


def qwen3_layer(p: Dict[str, torch.Tensor], nh: int, nkv: int, hd: int, eps: float, hidden: torch.Tensor,
                target_ctx: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``Qwen3DSparkLayer.__call__`` (``qwen3.py:165-167``): ``p`` holds the attention's weights,
    ``input_layernorm``, ``post_attention_layernorm``, ``gate_proj``, ``up_proj``, ``down_proj``."""
    a = qwen3_attention(p, nh, nkv, hd, eps, rms_norm(hidden, p["input_layernorm"], eps), target_ctx, cos, sin)
    hidden = _add(hidden, a)
    return _add(hidden, _qwen3_mlp(p, rms_norm(hidden, p["post_attention_layernorm"], eps)))


def qwen3_layer_cached(p: Dict[str, torch.Tensor], nh: int, nkv: int, hd: int, eps: float, hidden: torch.Tensor,
                       ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor], cos: torch.Tensor,
                       sin: torch.Tensor) -> torch.Tensor:
    """``Qwen3DSparkLayer.forward_cached`` (``qwen3.py:174-176``)."""
    a = qwen3_attend_cached(p, nh, nkv, hd, eps, rms_norm(hidden, p["input_layernorm"], eps), ctx_k, ctx_v, cos, sin)
    hidden = _add(hidden, a)
    return _add(hidden, _qwen3_mlp(p, rms_norm(hidden, p["post_attention_layernorm"], eps)))


def qwen3_layer_params(t: Dict[str, torch.Tensor], i: int) -> Dict[str, torch.Tensor]:
    """Layer ``i``'s tensors under the short names the layer functions take, from the
    backbone's reference names (``layers.{i}.self_attn.q_proj.weight`` -> ``q_proj`` ...)."""
    pre = f"layers.{i}."
    return {k[len(pre):].split(".")[-2]: v for k, v in t.items() if k.startswith(pre)}


def qwen3_project_context(t: Dict[str, torch.Tensor], eps: float, target_hidden: torch.Tensor) -> torch.Tensor:
    """``Qwen3Backbone.project_context`` (``qwen3.py:189-191``): ``hidden_norm(fc(target_hidden))``."""
    return rms_norm(linear(target_hidden, t["fc.weight"]), t["hidden_norm.weight"], eps)


def qwen3_backbone(t: Dict[str, torch.Tensor], n_layers: int, nh: int, nkv: int, hd: int, eps: float,
                   noise_embed: torch.Tensor, target_ctx: torch.Tensor, cos: torch.Tensor,
                   sin: torch.Tensor) -> torch.Tensor:
    """``Qwen3Backbone.__call__`` (``qwen3.py:193-197``): the layers, then the final norm."""
    h = noise_embed
    for i in range(n_layers):
        h = qwen3_layer(qwen3_layer_params(t, i), nh, nkv, hd, eps, h, target_ctx, cos, sin)
    return rms_norm(h, t["norm.weight"], eps)
