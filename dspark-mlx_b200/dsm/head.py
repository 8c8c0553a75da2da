"""The DSpark draft head on the GPU: ``DSparkHead`` (``DSparkBlock.forward_head`` with the
drafter's LM head) and the Markov head module.

``forward_head`` (``dspark_mlx/model/block.py:103-116``) reduces the last block's
hyper-connection copies (``hc_head``, ``hyper.py:52-67``) and applies the final ``norm``.
It reads the LM head over the vocabulary in fp32 (``drafter.py:29``), then walks the draft
block left to right (``recipe.py:30-63``). Each position adds the Markov transition bias of
the previous token (``heads.py:11-31``) and samples the next token. The confidence head
(``heads.py:34-49``) scores every position.

Parameter names follow the reference: ``hc_head_fn`` ``[hc, hc*dim]``, ``hc_head_base``
``[hc]``, ``hc_head_scale`` ``[1]``, ``norm.weight``, ``markov_head.markov_w1.weight`` /
``markov_head.markov_w2.weight`` ``[vocab, rank]``, ``confidence_head.proj.weight``
``[1, dim + rank]`` (plus ``.bias`` where the architecture has one), and ``head.weight``
``[vocab, dim]``, the drafter's LM head. The whole head is one ``dsm_draft_head`` call
(``include/dsm.h``). CPU tensors are rejected: there is no CPU path.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
from torch import nn

from . import _lib
from ._lib import HeadDesc, check, dtype_code, lib, ptr, stream_ptr
from .block import RMSNorm
from .config import DSparkArgs
from .weights import PackedMatrix, pack


def _param(*shape, dtype=torch.float32, fill=0.0):
    return nn.Parameter(torch.full(shape, fill, dtype=dtype), requires_grad=False)


class _Weight(nn.Module):
    """A module holding only ``weight`` (the reference's Embedding / Linear slots)."""

    def __init__(self, *shape, bias: bool = False):
        super().__init__()
        self.weight = _param(*shape)
        if bias:
            self.bias = _param(shape[0])


def _markov_tables(w1: torch.Tensor, w2: torch.Tensor):
    dt = torch.bfloat16 if w1.dtype == torch.bfloat16 and w2.dtype == torch.bfloat16 else torch.float32
    return w1.to(dt).contiguous(), w2.to(dt).contiguous(), dtype_code(dt)


class DSparkMarkovHead(nn.Module):
    """``DSparkMarkovHead`` (``heads.py:11-31``): ``(logits fp32 [..., vocab], embed [..., rank])``."""

    def __init__(self, vocab_size: int, rank: int):
        super().__init__()
        self.markov_w1 = _Weight(vocab_size, rank)
        self.markov_w2 = _Weight(vocab_size, rank)

    def forward(self, token_ids: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        if not token_ids.is_cuda:
            raise ValueError("DSparkMarkovHead runs on the GPU only")
        w1, w2, wdt = _markov_tables(self.markov_w1.weight, self.markov_w2.weight)
        ids = token_ids.reshape(-1).contiguous()
        if ids.dtype not in (torch.int32, torch.int64):
            ids = ids.to(torch.int32)
        n, (vocab, rank) = ids.numel(), w1.shape
        logits = torch.empty(n, vocab, dtype=torch.float32, device=ids.device)
        embed = torch.empty(n, rank, dtype=w1.dtype, device=ids.device)
        check(lib().dsm_markov_head(ptr(ids), dtype_code(ids.dtype), n, vocab, rank, ptr(w1), ptr(w2), wdt, ptr(logits),
                                    ptr(embed), stream_ptr()), "dsm_markov_head")
        shape = tuple(token_ids.shape)
        return logits.reshape(*shape, vocab), embed.to(self.markov_w1.weight.dtype).reshape(*shape, rank)


class DSparkHead(nn.Module):
    """The last draft block's head with the LM head:
    ``forward(x [b, s, hc, dim], input_ids [b]) -> (output_ids [b, s+1] int32, biased_logits
    [b, s, vocab] fp32, confidence [b, s] fp32)``."""

    def __init__(self, args, conf_bias: bool = False):
        super().__init__()
        if isinstance(args, dict):
            args = DSparkArgs.from_dict(args)
        self.hc_mult, self.dim, self.vocab = args.hc_mult, args.dim, args.vocab_size
        self.rank = args.dspark_markov_rank
        self.block_size = args.dspark_block_size
        self.temperature = args.temperature
        self.norm_eps, self.hc_eps = args.norm_eps, args.hc_eps
        hc, dim = self.hc_mult, self.dim
        self.hc_head_fn = _param(hc, hc * dim)
        self.hc_head_base = _param(hc)
        self.hc_head_scale = _param(1)
        self.norm = RMSNorm(dim, args.norm_eps)
        self.markov_head = DSparkMarkovHead(self.vocab, self.rank)
        self.confidence_head = nn.Module()
        self.confidence_head.proj = _Weight(1, dim + self.rank, bias=conf_bias)
        self.head = _Weight(self.vocab, dim)
        self._cache = None
        self._ws: Optional[torch.Tensor] = None

    def packed_head(self) -> PackedMatrix:
        w = self.head.weight
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        if self._cache is None or self._cache[0] != key:
            self._cache = (key, pack("dense", data=w.detach(), device=w.device))
        return self._cache[1]

    def forward(self, x: torch.Tensor, input_ids: torch.Tensor, *, temperature: Optional[float] = None,
                uniforms: Optional[torch.Tensor] = None):
        """``uniforms`` ``[s, b, vocab]`` (one ``mx.random.uniform`` draw per position) are
        used above temperature 0; drawn here when not given."""
        if not x.is_cuda:
            raise ValueError("DSparkHead runs on the GPU only: x must be a CUDA tensor")
        return run_draft_head(self, self.packed_head(), x, input_ids, temperature=temperature, uniforms=uniforms)


def run_draft_head(owner, hp: PackedMatrix, x: torch.Tensor, input_ids: torch.Tensor, *,
                   temperature: Optional[float] = None, uniforms: Optional[torch.Tensor] = None):
    """The draft head of ``owner`` (a module with the head's parameters under the reference's
    names: ``hc_head_fn`` / ``hc_head_scale`` / ``hc_head_base``, ``norm``, ``markov_head``,
    ``confidence_head``, and the settings ``hc_mult``, ``dim``, ``vocab``, ``rank``,
    ``temperature``, ``norm_eps``, ``hc_eps``; ``_ws`` caches the workspace) over the packed
    LM head ``hp``."""
    if not x.is_cuda:
        raise ValueError("DSparkHead runs on the GPU only: x must be a CUDA tensor")
    b, s, hc, dim = x.shape
    if hc != owner.hc_mult or dim != owner.dim:
        raise ValueError(f"x must be [b, s, {owner.hc_mult}, {owner.dim}], got {tuple(x.shape)}")
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.to(torch.float32)
    x = x.contiguous()
    dev = x.device
    temp = float(owner.temperature if temperature is None else temperature)
    ids = input_ids.reshape(-1).contiguous()
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    if ids.numel() != b:
        raise ValueError("input_ids must hold one anchor token per batch row")
    if temp > 0 and uniforms is None:
        uniforms = torch.rand(s, b, owner.vocab, device=dev)
    if uniforms is not None:
        uniforms = uniforms.to(device=dev, dtype=torch.float32).contiguous()
        if tuple(uniforms.shape) != (s, b, owner.vocab):
            raise ValueError(f"uniforms must be [{s}, {b}, {owner.vocab}], got {tuple(uniforms.shape)}")
    f32 = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    fn, sc, base, nw = f32(owner.hc_head_fn), f32(owner.hc_head_scale), f32(owner.hc_head_base), f32(owner.norm.weight)
    proj = owner.confidence_head.proj
    cw = f32(proj.weight.reshape(-1))
    w1, w2, wdt = _markov_tables(owner.markov_head.markov_w1.weight.detach().to(dev),
                                 owner.markov_head.markov_w2.weight.detach().to(dev))
    d = HeadDesc()
    d.batch, d.block, d.hc_mult, d.dim, d.vocab, d.rank = b, s, hc, dim, owner.vocab, owner.rank
    d.norm_eps, d.hc_eps = float(owner.norm_eps), float(owner.hc_eps)
    d.hc_fn, d.hc_scale, d.hc_base, d.norm_weight = ptr(fn), ptr(sc), ptr(base), ptr(nw)
    d.head_wfmt, d.head_group_size, d.head_w = hp.wfmt, hp.group_size, ptr(hp.packed)
    d.markov_dtype, d.markov_w1, d.markov_w2 = wdt, ptr(w1), ptr(w2)
    d.conf_w = ptr(cw)
    d.conf_bias = float(proj.bias.reshape(-1)[0]) if hasattr(proj, "bias") else 0.0
    L = lib()
    need = L.dsm_draft_head_workspace_bytes(ctypes.byref(d), dtype_code(x.dtype))
    if owner._ws is None or owner._ws.numel() < need or owner._ws.device != dev:
        owner._ws = torch.empty(need, dtype=torch.uint8, device=dev)
    out_ids = torch.empty(b, s + 1, dtype=torch.int32, device=dev)
    biased = torch.empty(b, s, owner.vocab, dtype=torch.float32, device=dev)
    conf = torch.empty(b, s, dtype=torch.float32, device=dev)
    check(L.dsm_draft_head(ctypes.byref(d), ptr(x), dtype_code(x.dtype), ptr(ids), dtype_code(ids.dtype), temp,
                           ptr(uniforms), ptr(out_ids), ptr(biased), ptr(conf), None, ptr(owner._ws),
                           owner._ws.numel(), stream_ptr()), "dsm_draft_head")
    return out_ids, biased, conf
