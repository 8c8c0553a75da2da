"""CPU oracle for the whole DSpark draft block (test infrastructure only).

Restates ``DSparkBlock`` (``dspark_mlx/model/block.py:28-116``) from the oracle's pieces:
* ``__call__`` (``block.py:74-86``): the prefill seeds the attention's window and returns x;
  a decode step is the attention half (``hc_pre`` -> ``attn_norm`` -> ``DSparkAttention`` ->
  ``hc_post``) then the FFN half (the same around the MoE);
* ``advance`` (``block.py:88-90``): the window over one committed token;
* ``forward_embed`` (``block.py:92-101``): the main rows ``main_norm(main_proj(main_hidden))``
  and the draft block's embeddings (anchor, then noise tokens) copied to every
  hyper-connection;
* ``forward_head`` (``block.py:103-116``): the head oracle.
``t`` maps the reference's parameter names to tensors (``attn.wq_a.weight``,
``ffn.gate.weight``, ``hc_attn_fn``, ``main_proj.weight`` ...).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from .attention_oracle import AttnDims, KVWindow, attention_forward, linear, rope_last
from .block_oracle import ffn_sublayer, rms_norm
from .head_oracle import forward_head
from .moe_oracle import OracleWeights, moe_forward

__all__ = ["block_attn_params", "block_forward", "block_advance", "block_forward_embed", "block_forward_head"]


def block_attn_params(t: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    return {k: t[f"attn.{k}.weight"] for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "q_norm", "kv_norm")} | {
        "attn_sink": t["attn.attn_sink"]}


def _dims(a: dict) -> AttnDims:
    return AttnDims(n_heads=a["n_heads"], head_dim=a["head_dim"], rope_head_dim=a["rope_head_dim"],
                    o_groups=a["o_groups"], o_lora_rank=a["o_lora_rank"], window_size=a["window_size"],
                    eps=a["norm_eps"])


def block_forward(t: Dict[str, torch.Tensor], a: dict, x: torch.Tensor, start_pos: int,
                  input_ids: Optional[torch.Tensor], main_x: torch.Tensor, cache: KVWindow, cos: torch.Tensor,
                  sin: torch.Tensor) -> torch.Tensor:
    """``DSparkBlock.__call__`` (``block.py:74-86``); ``cos``/``sin`` are the attention's tables."""
    p, dims = block_attn_params(t), _dims(a)
    if start_pos == 0:
        return attention_forward(p, dims, x, 0, main_x, cache, cos, sin)
    hc = dict(hc=a["hc_mult"], iters=a["hc_sinkhorn_iters"], norm_eps=a["norm_eps"], hc_eps=a["hc_eps"])
    x = ffn_sublayer(x, None, hc_fn=t["hc_attn_fn"], hc_scale=t["hc_attn_scale"], hc_base=t["hc_attn_base"],
                     norm_weight=t["attn_norm.weight"],
                     moe=lambda h, _ids: attention_forward(p, dims, h, start_pos, main_x, cache, cos, sin), **hc)
    ffn = dict(gate_weight=t["ffn.gate.weight"], gate_bias=t["ffn.gate.bias"], topk=a["n_activated_experts"],
               score_func=a["score_func"], route_scale=a["route_scale"], swiglu_limit=a["swiglu_limit"],
               w1=OracleWeights("dense", t["ffn.w1"]), w3=OracleWeights("dense", t["ffn.w3"]),
               w2=OracleWeights("dense", t["ffn.w2"]),
               shared=tuple(t[f"ffn.shared_experts.{n}.weight"] for n in ("w1", "w2", "w3")))
    return ffn_sublayer(x, input_ids, hc_fn=t["hc_ffn_fn"], hc_scale=t["hc_ffn_scale"], hc_base=t["hc_ffn_base"],
                        norm_weight=t["ffn_norm.weight"], moe=lambda h, ids: moe_forward(h, ids, **ffn), **hc)


def block_advance(t: Dict[str, torch.Tensor], a: dict, main_x: torch.Tensor, position: int, cache: KVWindow,
                  cos: torch.Tensor, sin: torch.Tensor) -> None:
    """``DSparkBlock.advance`` -> ``DSparkAttention.advance_window`` (``attention.py:131-142``)."""
    kv = rms_norm(linear(main_x.reshape(main_x.shape[0], 1, -1), t["attn.wkv.weight"]), t["attn.kv_norm.weight"],
                  a["norm_eps"])
    kv = rope_last(kv, cos[position:position + 1], sin[position:position + 1], a["rope_head_dim"])
    cache.update(position, kv[:, 0])


def block_forward_embed(t: Dict[str, torch.Tensor], a: dict, main_hidden: torch.Tensor, input_ids: torch.Tensor,
                        embed_w: torch.Tensor):
    """``DSparkBlock.forward_embed`` (``block.py:92-101``): ``(x [b, block, hc, dim], main_x)``."""
    main_x = rms_norm(linear(main_hidden, t["main_proj.weight"]), t["main_norm.weight"], a["norm_eps"])
    b = input_ids.shape[0]
    noise = torch.full((b, a["dspark_block_size"] - 1), a["dspark_noise_token_id"], dtype=torch.int64)
    draft_ids = torch.cat([input_ids.reshape(b, 1).to(torch.int64), noise], dim=1)
    x = embed_w[draft_ids]
    return x[:, :, None, :].expand(b, a["dspark_block_size"], a["hc_mult"], x.shape[-1]), main_x


def block_forward_head(t: Dict[str, torch.Tensor], a: dict, x: torch.Tensor, input_ids: torch.Tensor,
                       head_w: torch.Tensor, temperature: float = 0.0):
    """``DSparkBlock.forward_head`` (``block.py:103-116``) with the drafter's LM head."""
    return forward_head(x, input_ids, head_w=head_w, hc_fn=t["hc_head_fn"], hc_scale=t["hc_head_scale"],
                        hc_base=t["hc_head_base"], norm_w=t["norm.weight"], w1=t["markov_head.markov_w1.weight"],
                        w2=t["markov_head.markov_w2.weight"], wc=t["confidence_head.proj.weight"],
                        norm_eps=a["norm_eps"], hc_eps=a["hc_eps"], temperature=temperature)
