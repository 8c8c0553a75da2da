"""The Qwen3 DSpark draft layer on the GPU: ``Qwen3DSparkLayer``
(``dspark_mlx/arch/qwen3.py:157-176``), and the backbone that stacks it, ``Qwen3Backbone``
(``qwen3.py:178-197``).

Same constructor (``Qwen3DSparkLayer(args)``), parameter names (``self_attn``, ``mlp``,
``input_layernorm``, ``post_attention_layernorm``) and calls as the reference:

* ``layer(hidden, target_ctx, cos, sin)``: ``hidden + attn(norm(hidden))``, then
  ``+ mlp(norm(.))`` (``qwen3.py:165-167``);
* ``context_kv(proj_ctx, cos, sin)``: the attention's cached context K/V, no norm
  (``qwen3.py:171-172``);
* ``forward_cached(hidden, ctx_k, ctx_v, cos, sin)``: the same over cached context K/V
  (``qwen3.py:174-176``).

The attention is :class:`dsm.qwen3_attention.Qwen3DSparkAttention`, the MLP
:class:`dsm.qwen3.Qwen3MLP` (``quantize`` quantises both as ``quantize_drafter`` does). The
norms and residual adds are ``dsm_add_rms_norm``: the input norm alone, the first residual add
fused with the post-attention norm, the last residual add alone. Hidden, weights and outputs
share one dtype (bf16 or fp32), as the reference's arrays do in a bf16 or fp32 drafter.

``Qwen3Backbone(args)`` holds ``fc``, ``hidden_norm``, ``layers`` and ``norm``:
``project_context(target_hidden)`` is ``hidden_norm(fc(.))`` (the projection on ``dsm_linear``,
rounded and normalised by ``dsm_rows_norm_rope``), and ``backbone(noise_embed, target_ctx,
cos, sin)`` runs the layers and the final norm.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import nn

from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .block import RMSNorm
from .qwen3 import Projection, Qwen3MLP
from .qwen3_attention import Qwen3DSparkAttention, _get


class Qwen3DSparkLayer(nn.Module):
    def __init__(self, args):
        super().__init__()
        h = int(_get(args, "hidden_size"))
        eps = float(_get(args, "rms_norm_eps"))
        self.hidden = h
        self.self_attn = Qwen3DSparkAttention(args)
        self.mlp = Qwen3MLP(args)
        self.input_layernorm = RMSNorm(h, eps)
        self.post_attention_layernorm = RMSNorm(h, eps)

    def quantize(self, bits: int = 8, group_size: int = 64) -> "Qwen3DSparkLayer":
        """``quantize_drafter``'s pass over this layer's Linears (``quant.py:36-41``)."""
        for p in (self.self_attn.q_proj, self.self_attn.k_proj, self.self_attn.v_proj, self.self_attn.o_proj):
            p.quantize(bits, group_size)
        self.mlp.quantize(bits, group_size)
        return self

    def _norm(self, x: torch.Tensor, norm: RMSNorm, delta: Optional[torch.Tensor] = None, want_sum: bool = False,
              want_norm: bool = True):
        """(x + delta, RMSNorm(x + delta)) as requested; one launch."""
        n = x.numel() // self.hidden
        s = torch.empty_like(x) if want_sum else None
        y = torch.empty_like(x) if want_norm else None
        w = norm.weight.detach().to(device=x.device, dtype=torch.float32).contiguous() if want_norm else None
        check(lib().dsm_add_rms_norm(ptr(x), ptr(delta), dtype_code(x.dtype), n, self.hidden, ptr(w), float(norm.eps),
                                     ptr(s), ptr(y), stream_ptr()), "dsm_add_rms_norm")
        return s, y

    def _check(self, hidden: torch.Tensor) -> torch.Tensor:
        if not hidden.is_cuda:
            raise ValueError("Qwen3DSparkLayer runs on the GPU only (hidden is on the CPU)")
        if hidden.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"hidden dtype {hidden.dtype} unsupported (bf16 or fp32)")
        if hidden.dim() != 3 or hidden.shape[-1] != self.hidden:
            raise ValueError(f"hidden must be [batch, seq, {self.hidden}], got {tuple(hidden.shape)}")
        return hidden.contiguous()

    def _finish(self, hidden: torch.Tensor, attn: torch.Tensor) -> torch.Tensor:
        if attn.dtype != hidden.dtype:
            raise ValueError(f"the attention returns {attn.dtype} for {hidden.dtype} hidden: weights and hidden "
                             "must share a dtype")
        h1, x2 = self._norm(hidden, self.post_attention_layernorm, delta=attn, want_sum=True)
        m = self.mlp(x2)
        if m.dtype != hidden.dtype:
            raise ValueError(f"the MLP returns {m.dtype} for {hidden.dtype} hidden: weights and hidden must share "
                             "a dtype")
        out, _ = self._norm(h1, self.post_attention_layernorm, delta=m, want_sum=True, want_norm=False)
        return out

    def forward(self, hidden: torch.Tensor, target_ctx: torch.Tensor, cos, sin) -> torch.Tensor:
        hidden = self._check(hidden)
        _, x = self._norm(hidden, self.input_layernorm)
        return self._finish(hidden, self.self_attn(x, target_ctx, cos, sin))

    def context_kv(self, proj_ctx: torch.Tensor, cos, sin, **kw):
        return self.self_attn.context_kv(proj_ctx, cos, sin, **kw)

    def forward_cached(self, hidden: torch.Tensor, ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor], cos,
                       sin) -> torch.Tensor:
        hidden = self._check(hidden)
        _, x = self._norm(hidden, self.input_layernorm)
        return self._finish(hidden, self.self_attn.attend_cached(x, ctx_k, ctx_v, cos, sin))


class Qwen3Backbone(nn.Module):
    def __init__(self, args):
        super().__init__()
        h = int(_get(args, "hidden_size"))
        eps = float(_get(args, "rms_norm_eps"))
        n_layers = int(_get(args, "num_hidden_layers"))
        fc_in = h * len(tuple(_get(args, "target_layer_ids")))
        self.hidden = h
        self.fc = Projection(fc_in, h)
        self.hidden_norm = RMSNorm(h, eps)
        self.layers = nn.ModuleList([Qwen3DSparkLayer(args) for _ in range(n_layers)])
        self.norm = RMSNorm(h, eps)

    def quantize(self, bits: int = 8, group_size: int = 64) -> "Qwen3Backbone":
        self.fc.quantize(bits, group_size)
        for layer in self.layers:
            layer.quantize(bits, group_size)
        return self

    def project_context(self, target_hidden: torch.Tensor) -> torch.Tensor:
        """``[b, ctx, fc_in]`` -> ``[b, ctx, hidden]`` = ``hidden_norm(fc(target_hidden))`` in the
        projection's dtype (``qwen3.py:189-191``)."""
        if not target_hidden.is_cuda:
            raise ValueError("Qwen3Backbone runs on the GPU only (target_hidden is on the CPU)")
        dt = self.fc.product_dtype(target_hidden.dtype)
        if dt not in (torch.bfloat16, torch.float32):
            raise ValueError(f"projection dtype {dt} unsupported (bf16 or fp32)")
        xin = target_hidden if target_hidden.dtype in (torch.bfloat16, torch.float32) else target_hidden.to(dt)
        lead = xin.shape[:-1]
        x2 = xin.reshape(-1, xin.shape[-1]).contiguous()
        n = x2.shape[0]
        st = Qwen3DSparkAttention._stage(x2)
        rows = st[3]
        o = torch.empty(rows, self.hidden, dtype=torch.float32, device=x2.device)
        Qwen3DSparkAttention._project(st, self.fc, o, self.hidden)
        y = torch.empty(n, self.hidden, dtype=dt, device=x2.device)
        w = self.hidden_norm.weight.detach().to(device=x2.device, dtype=torch.float32).contiguous()
        check(lib().dsm_rows_norm_rope(ptr(o), ptr(o[n:]) if rows == 2 * n else None, n, self.hidden, ptr(w),
                                       float(self.hidden_norm.eps), 0, None, None, 0, 1, ptr(y), dtype_code(dt),
                                       stream_ptr()), "dsm_rows_norm_rope")
        return y.reshape(*lead, self.hidden)

    def forward(self, noise_embed: torch.Tensor, target_ctx: torch.Tensor, cos, sin) -> torch.Tensor:
        """The layers over ``[context || block]``, then the final norm (``qwen3.py:193-197``)."""
        h = noise_embed
        for layer in self.layers:
            h = layer(h, target_ctx, cos, sin)
        h = h.contiguous()
        y = torch.empty_like(h)
        w = self.norm.weight.detach().to(device=h.device, dtype=torch.float32).contiguous()
        check(lib().dsm_add_rms_norm(ptr(h), None, dtype_code(h.dtype), h.numel() // self.hidden, self.hidden, ptr(w),
                                     float(self.norm.eps), None, ptr(y), stream_ptr()), "dsm_add_rms_norm")
        return y
