"""The whole DSpark draft block on the GPU: ``DSparkBlock`` (``dspark_mlx/model/block.py:28-116``).

Same constructor (``DSparkBlock(args, stage_id, max_seq_len)``), calls and parameter names as
the reference:
* ``block(x [b, s, hc, dim], start_pos, input_ids, main_x)``. The prefill (``start_pos ==
  0``) seeds the attention's window and returns x. A decode step is the attention half
  (``hc_pre`` -> ``attn_norm`` -> ``attn`` -> ``hc_post``) and then the FFN half, the same
  around the MoE (``block.py:74-86``).
* ``advance(main_x, position)``: the window over one committed token (``block.py:88-90``).
* ``forward_embed(main_hidden, input_ids, embed)`` (stage 0): ``main_norm(main_proj(.))``
  and the draft block's embeddings copied to every hyper-connection (``block.py:92-101``).
* ``forward_head(x, input_ids, head)`` (last stage): the draft head with the drafter's LM
  head module (``block.py:103-116``).

Parameters: ``attn`` (:class:`dsm.attention.DSparkAttention`), ``ffn`` (:class:`dsm.MoE`),
``attn_norm``, ``ffn_norm``, ``hc_attn_fn`` / ``hc_attn_base`` / ``hc_attn_scale`` and the
``hc_ffn_*`` triple; ``main_proj``, ``main_norm`` on stage 0; ``norm``, ``markov_head``,
``confidence_head``, ``hc_head_*`` on the last stage. Every step runs on ``libdsm`` kernels:
``dsm_hc_pre_norm`` / ``dsm_hc_post`` around each half, the attention's and the MoE's own
kernels, ``dsm_linear`` + ``dsm_rows_norm_rope`` for the main projection, ``dsm_gather_rows``
for the embedding rows, and ``dsm_draft_head``. CPU tensors are rejected.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
from torch import nn

from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .attention import DSparkAttention, _Linear
from .block import RMSNorm
from .config import DSparkArgs
from .head import DSparkMarkovHead, _Weight, run_draft_head
from .moe import MoE
from .weights import PackedMatrix, pack


def _param(*shape):
    return nn.Parameter(torch.zeros(shape, dtype=torch.float32), requires_grad=False)


class DSparkBlock(nn.Module):
    def __init__(self, args, stage_id: int, max_seq_len: int = 8192):
        super().__init__()
        if isinstance(args, dict):
            args = DSparkArgs.from_dict(args)
        self.stage_id = stage_id
        self.hc_mult, self.hc_sinkhorn_iters, self.hc_eps = args.hc_mult, args.hc_sinkhorn_iters, args.hc_eps
        self.norm_eps = args.norm_eps
        self.block_size, self.noise_token_id = args.dspark_block_size, args.dspark_noise_token_id
        self.temperature = args.temperature
        self.dim, self.vocab, self.rank = args.dim, args.vocab_size, args.dspark_markov_rank
        self.is_last = stage_id == args.n_mtp_layers - 1
        self.attn = DSparkAttention(args, max_seq_len)
        self.ffn = MoE(args, args.n_layers + stage_id)
        self.attn_norm = RMSNorm(args.dim, args.norm_eps)
        self.ffn_norm = RMSNorm(args.dim, args.norm_eps)
        hc, mix = self.hc_mult, (2 + self.hc_mult) * self.hc_mult
        self.hc_attn_fn, self.hc_ffn_fn = _param(mix, hc * args.dim), _param(mix, hc * args.dim)
        self.hc_attn_base, self.hc_ffn_base = _param(mix), _param(mix)
        self.hc_attn_scale, self.hc_ffn_scale = _param(3), _param(3)
        if stage_id == 0:
            self.main_proj = _Linear(args.dim * len(args.dspark_target_layer_ids), args.dim)
            self.main_norm = RMSNorm(args.dim, args.norm_eps)
        if self.is_last:
            self.norm = RMSNorm(args.dim, args.norm_eps)
            self.markov_head = DSparkMarkovHead(self.vocab, self.rank)
            self.confidence_head = nn.Module()
            self.confidence_head.proj = _Weight(1, args.dim + self.rank)
            self.hc_head_fn, self.hc_head_base, self.hc_head_scale = _param(hc, hc * args.dim), _param(hc), _param(1)
        self._ws: Optional[torch.Tensor] = None
        self._head_cache = None
        self._main_cache = None

    # ---------------------------------------------------------------- hyper-connection halves
    def _half(self, x: torch.Tensor, fn, scale, base, norm: RMSNorm, inner: Callable[[torch.Tensor], torch.Tensor]):
        """residual = x; h, post, comb = hc_pre(x); h = inner(norm(h)); hc_post(h, residual, post, comb)."""
        b, s, hc, dim = x.shape
        n = b * s
        dev, dt = x.device, x.dtype
        xn = torch.empty(n, dim, dtype=dt, device=dev)
        post = torch.empty(n, hc, dtype=torch.float32, device=dev)
        comb = torch.empty(n, hc, hc, dtype=torch.float32, device=dev)
        f32 = [t.detach().to(device=dev, dtype=torch.float32).contiguous() for t in (fn, scale, base, norm.weight)]
        L = lib()
        check(L.dsm_hc_pre_norm(ptr(x), dtype_code(dt), n, hc, dim, ptr(f32[0]), ptr(f32[1]), ptr(f32[2]),
                                self.hc_sinkhorn_iters, float(self.norm_eps), float(self.hc_eps), ptr(f32[3]), ptr(xn),
                                ptr(post), ptr(comb), stream_ptr()), "dsm_hc_pre_norm")
        h = inner(xn.reshape(b, s, dim))
        if h.dtype != dt:
            raise ValueError(f"the sub-layer returns {h.dtype} for {dt} input: weights and activations must share "
                             "a dtype")
        h = h.reshape(n, dim).contiguous()
        out = torch.empty_like(x)
        check(L.dsm_hc_post(ptr(h), ptr(x), dtype_code(dt), n, hc, dim, ptr(post), ptr(comb), ptr(out), stream_ptr()),
              "dsm_hc_post")
        return out

    def forward(self, x: torch.Tensor, start_pos: int, input_ids: Optional[torch.Tensor],
                main_x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise ValueError("DSparkBlock runs on the GPU only: x must be a CUDA tensor")
        if start_pos == 0:
            return self.attn(x, start_pos, main_x)  # the prefill seeds the window only
        if x.dim() != 4 or x.shape[2] != self.hc_mult or x.shape[3] != self.dim:
            raise ValueError(f"x must be [b, s, {self.hc_mult}, {self.dim}], got {tuple(x.shape)}")
        x = x.contiguous()
        x = self._half(x, self.hc_attn_fn, self.hc_attn_scale, self.hc_attn_base, self.attn_norm,
                       lambda h: self.attn(h, start_pos, main_x))
        return self._half(x, self.hc_ffn_fn, self.hc_ffn_scale, self.hc_ffn_base, self.ffn_norm,
                          lambda h: self.ffn(h, input_ids))

    def advance(self, main_x: torch.Tensor, position: int) -> None:
        self.attn.advance_window(main_x, position)

    # ---------------------------------------------------------------- stage 0 / last stage
    def _packed_main(self) -> PackedMatrix:
        w = self.main_proj.weight
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        if self._main_cache is None or self._main_cache[0] != key:
            self._main_cache = (key, pack("dense", data=w.detach(), device=w.device))
        return self._main_cache[1]

    def project_main(self, main_hidden: torch.Tensor) -> torch.Tensor:
        """``main_norm(main_proj(main_hidden))`` over the last dimension (stage 0), the rows the
        window and the attention read (``block.py:96`` and ``drafter.py:50-51``)."""
        if self.stage_id != 0:
            raise ValueError("the main projection belongs to stage 0")
        if not main_hidden.is_cuda:
            raise ValueError("DSparkBlock runs on the GPU only")
        dt = main_hidden.dtype if main_hidden.dtype in (torch.bfloat16, torch.float32) else torch.float32
        mh = main_hidden.to(dt).contiguous()
        lead = mh.shape[:-1]
        mh2 = mh.reshape(-1, mh.shape[-1])
        main_x = self.attn._norm_rope(mh2, self._packed_main(), self.main_norm.weight, False, 0, 1)
        return main_x.reshape(*lead, self.dim)

    def forward_embed(self, main_hidden: torch.Tensor, input_ids: torch.Tensor, embed: nn.Module):
        """``(x [b, block, hc, dim], main_x [b, seqlen, dim])``; ``embed`` holds ``weight [vocab, dim]``."""
        if self.stage_id != 0:
            raise ValueError("forward_embed belongs to stage 0")
        if not (main_hidden.is_cuda and input_ids.is_cuda):
            raise ValueError("DSparkBlock runs on the GPU only")
        main_x = self.project_main(main_hidden)
        b = input_ids.shape[0]
        w = embed.weight.detach()
        if w.dtype not in (torch.bfloat16, torch.float32):
            w = w.to(torch.float32)
        w = w.contiguous()
        draft = torch.full((b, self.block_size), self.noise_token_id, dtype=torch.int32, device=w.device)
        draft[:, 0] = input_ids.reshape(b).to(torch.int32)
        rows = draft.reshape(-1).repeat_interleave(self.hc_mult).contiguous()  # one row per hyper-connection
        x = torch.empty(rows.numel(), self.dim, dtype=w.dtype, device=w.device)
        check(lib().dsm_gather_rows(ptr(w), dtype_code(w.dtype), w.shape[0], self.dim, ptr(rows), rows.numel(), 1,
                                    ptr(x), stream_ptr()), "dsm_gather_rows")
        return x.reshape(b, self.block_size, self.hc_mult, self.dim), main_x

    def forward_head(self, x: torch.Tensor, input_ids: torch.Tensor, head: nn.Module, *,
                     temperature: Optional[float] = None, uniforms: Optional[torch.Tensor] = None):
        """``(output_ids [b, s+1], biased_logits [b, s, vocab], confidence [b, s])``; ``head``
        holds the drafter's LM head ``weight [vocab, dim]``."""
        if not self.is_last:
            raise ValueError("forward_head belongs to the last stage")
        if not x.is_cuda:
            raise ValueError("DSparkBlock runs on the GPU only: x must be a CUDA tensor")
        w = head.weight
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        if self._head_cache is None or self._head_cache[0] != key:
            self._head_cache = (key, pack("dense", data=w.detach(), device=w.device))
        return run_draft_head(self, self._head_cache[1], x, input_ids, temperature=temperature, uniforms=uniforms)
