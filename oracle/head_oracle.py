"""CPU oracle for the DSpark draft head (test infrastructure only).

Restates, in PyTorch on the CPU with MLX's dtype rules, the last-stage head of the draft
stack:

* ``hc_head``: the hyper-connection copies reduced to one hidden
  (``dspark_mlx/model/hyper.py:52-67``);
* the final ``RMSNorm`` (``dspark_mlx/model/norm_rope.py:22-39``) and the LM head in fp32
  (``dspark_mlx/model/block.py:111-112``);
* the Markov transition head (``dspark_mlx/model/heads.py:11-31``);
* the confidence head (``dspark_mlx/model/heads.py:34-49``);
* the left-to-right block walk that adds the Markov bias and samples each next token
  (``dspark_mlx/recipe.py:21-63``).

The sampler at temperature 0 is argmax. Above 0 it is Gumbel-max over softmax probabilities
with uniforms drawn by ``mx.random.uniform``. Here the uniforms are an argument, one
``[b, vocab]`` tensor per block position, so a run is reproducible.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from .block_oracle import rms_norm

__all__ = ["hc_head", "markov_head", "confidence_head", "sample", "draft_block_decode", "forward_head"]


def hc_head(x: torch.Tensor, hc_fn: torch.Tensor, hc_scale: torch.Tensor, hc_base: torch.Tensor, norm_eps: float,
            hc_eps: float) -> torch.Tensor:
    """``[b, s, hc, d] -> [b, s, d]`` in x's dtype (``hyper.py:52-67``)."""
    shape = x.shape
    xf = x.reshape(*shape[:2], -1).to(torch.float32)
    rsqrt = torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + norm_eps)
    mixes = (xf @ hc_fn.to(torch.float32).T) * rsqrt
    pre = torch.sigmoid(mixes * hc_scale.to(torch.float32) + hc_base.to(torch.float32)) + hc_eps
    y = (pre[..., None] * xf.reshape(shape)).sum(dim=2)
    return y.to(x.dtype)


def markov_head(token_ids: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(logits fp32 [..., vocab], embed [..., rank] in w1's dtype)`` (``heads.py:26-30``)."""
    embed = w1[token_ids.to(torch.int64)]
    logits = embed.to(torch.float32) @ w2.to(torch.float32).T
    return logits, embed


def confidence_head(hidden: torch.Tensor, markov_embed: torch.Tensor, wc: torch.Tensor,
                    bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``proj([hidden || markov_embed])[..., 0]`` in fp32 (``heads.py:46-48``)."""
    dt = torch.promote_types(hidden.dtype, markov_embed.dtype)
    x = torch.cat([hidden.to(dt), markov_embed.to(dt)], dim=-1).to(torch.float32)
    y = x @ wc.to(torch.float32).T
    if bias is not None:
        y = y + bias.to(torch.float32)
    return y[..., 0]


def sample(logits: torch.Tensor, temperature: float, uniforms: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``recipe.py:21-27``: argmax at temperature 0 (first maximum), else Gumbel-max."""
    if temperature == 0:
        return logits.argmax(dim=-1).to(torch.int32)
    probs = torch.softmax(logits.to(torch.float32) / max(temperature, 1e-5), dim=-1)
    g = uniforms.to(torch.float32)
    return (probs / (-torch.log(g + 1e-20))).argmax(dim=-1).to(torch.int32)


def draft_block_decode(logits: torch.Tensor, conf_hidden: torch.Tensor, anchor: torch.Tensor, w1: torch.Tensor,
                       w2: torch.Tensor, wc: torch.Tensor, block_size: int, temperature: float,
                       uniforms: Optional[Sequence[torch.Tensor]] = None, conf_bias: Optional[torch.Tensor] = None):
    """``recipe.py:30-63``: ``(output_ids [b, s+1], biased_logits [b, s, vocab], confidence [b, s])``."""
    prev = anchor.to(torch.int32)
    out_ids, biased, membeds = [prev], [], []
    for i in range(block_size):
        bias, membed = markov_head(prev, w1, w2)
        li = logits[:, i] + bias
        biased.append(li)
        membeds.append(membed)
        prev = sample(li, temperature, None if uniforms is None else uniforms[i])
        out_ids.append(prev)
    output_ids = torch.stack(out_ids, dim=1)
    logits_out = torch.stack(biased, dim=1)
    confidence = confidence_head(conf_hidden, torch.stack(membeds, dim=1), wc, conf_bias)
    return output_ids, logits_out, confidence


def forward_head(x: torch.Tensor, input_ids: torch.Tensor, *, head_w: torch.Tensor, hc_fn: torch.Tensor,
                 hc_scale: torch.Tensor, hc_base: torch.Tensor, norm_w: torch.Tensor, w1: torch.Tensor,
                 w2: torch.Tensor, wc: torch.Tensor, norm_eps: float, hc_eps: float, temperature: float,
                 uniforms: Optional[Sequence[torch.Tensor]] = None, conf_bias: Optional[torch.Tensor] = None):
    """``DSparkBlock.forward_head`` (``block.py:103-116``) with the drafter's LM head ``head_w``."""
    y = hc_head(x, hc_fn, hc_scale, hc_base, norm_eps, hc_eps)
    xn = rms_norm(y, norm_w, norm_eps).to(torch.float32)
    logits = xn @ head_w.to(torch.float32).T
    return draft_block_decode(logits, y, input_ids, w1, w2, wc, x.shape[1], temperature, uniforms, conf_bias)
