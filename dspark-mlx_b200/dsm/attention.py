"""The DSpark draft attention on the GPU: ``DSparkAttention``, the ``compress_ratio == 0`` MLA
of the draft blocks (``dspark_mlx/model/attention.py``).

Same constructor (``DSparkAttention(args, max_seq_len)``), call
(``attn(x [b, s, dim], start_pos, main_x [b, seqlen, dim])``) and ``advance_window`` as the
reference, and the same parameter names. Those are ``wq_a``, ``q_norm``, ``wq_b``, ``wkv``,
``kv_norm``, ``wo_a``, ``wo_b`` and ``attn_sink``. A prefill call (``start_pos == 0``) seeds
the sliding KV window and returns x. A decode call drafts the block.

The five projections run on ``dsm_linear_splitk`` over packed weights (K split where the row
tiles alone would leave SMs idle). A bf16 activation is staged
exactly. An fp32 activation is staged as two f16 rows (hi + lo), so its products keep fp32
precision. The norms, RoPE, the window ring, the gathered attention with its sink and the
output's inverse rotation are the ``dsm_*`` kernels of ``csrc/attn.cu``. The grouped output
projection is one ``dsm_grouped_linear`` launch over the group-major attention output (bf16;
fp32 rows, staged hi + lo, take one ``dsm_linear`` per group). CPU tensors are rejected.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
from torch import nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .block import RMSNorm
from .config import DSparkArgs
from .weights import PackedMatrix, pack


class _Linear(nn.Module):
    def __init__(self, in_dim: int, out_dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(out_dim, in_dim), requires_grad=False)


def rope_tables(dim: int, seqlen: int, base: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``precompute_rope`` (``norm_rope.py:43-49``), computed as the reference does, in fp32."""
    freqs = 1.0 / (base ** (torch.arange(0, dim, 2).to(torch.float32) / dim))
    theta = torch.outer(torch.arange(seqlen).to(torch.float32), freqs)
    return torch.cos(theta), torch.sin(theta)


class DSparkAttention(nn.Module):
    def __init__(self, args, max_seq_len: int = 8192):
        super().__init__()
        if isinstance(args, dict):
            args = DSparkArgs.from_dict(args)
        self.n_heads, self.head_dim, self.rope_head_dim = args.n_heads, args.head_dim, args.rope_head_dim
        self.o_lora_rank, self.n_groups, self.window_size = args.o_lora_rank, args.o_groups, args.window_size
        self.eps = args.norm_eps
        self.softmax_scale = args.head_dim ** -0.5
        self.dim = args.dim
        self.wq_a = _Linear(args.dim, args.q_lora_rank)
        self.q_norm = RMSNorm(args.q_lora_rank, args.norm_eps)
        self.wq_b = _Linear(args.q_lora_rank, args.n_heads * args.head_dim)
        self.wkv = _Linear(args.dim, args.head_dim)
        self.kv_norm = RMSNorm(args.head_dim, args.norm_eps)
        self.wo_a = _Linear(args.n_heads * args.head_dim // args.o_groups, args.o_groups * args.o_lora_rank)
        self.wo_b = _Linear(args.o_groups * args.o_lora_rank, args.dim)
        self.attn_sink = nn.Parameter(torch.zeros(args.n_heads), requires_grad=False)
        cos, sin = rope_tables(args.rope_head_dim, max_seq_len, args.rope_theta)
        self.register_buffer("_cos", cos, persistent=False)
        self.register_buffer("_sin", sin, persistent=False)
        self.window: Optional[torch.Tensor] = None  # [b, window, head_dim], slot p % window = position p
        self._packed: Dict[object, tuple] = {}  # packed weights and row maps, by name

    # ---------------------------------------------------------------- projections
    def _pm(self, name: str, w: torch.Tensor) -> PackedMatrix:
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        hit = self._packed.get(name)
        if hit is None or hit[0] != key:
            hit = (key, pack("dense", data=w.detach(), device=w.device))
            self._packed[name] = hit
        return hit[1]

    @staticmethod
    def _stage(x2: torch.Tensor):
        """x2's rows staged for the products (fp32 rows as hi + lo): (staged, xscale, cap, rows, k)."""
        L = lib()
        n, k = x2.shape
        f32 = x2.dtype == torch.float32
        rows = 2 * n if f32 else n
        cap = L.dsm_stage_rows_cap(rows)
        staged = torch.empty(L.dsm_stage_bytes(cap, k), dtype=torch.uint8, device=x2.device)
        xscale = torch.empty(cap, dtype=torch.float32, device=x2.device)
        s = stream_ptr()
        if f32:
            check(L.dsm_stage_rows_hilo(ptr(x2), n, k, ptr(staged), cap, ptr(xscale), s), "dsm_stage_rows_hilo")
        else:
            check(L.dsm_stage_rows(ptr(x2), dtype_code(x2.dtype), n, k, None, n, 1, ptr(staged), cap, ptr(xscale), s),
                  "dsm_stage_rows")
        return staged, xscale, cap, rows, k

    def _linear(self, x2: torch.Tensor, pm: PackedMatrix, out: Optional[torch.Tensor] = None, ldo: int = 0, st=None):
        """fp32 rows of x2 W^T: ``(hi, lo)``; lo is the product of an fp32 input's residual rows.
        st: x2 already staged by ``_stage`` (one staging serves several products of x2)."""
        L = lib()
        staged, xscale, cap, rows, k = self._stage(x2) if st is None else st
        s = stream_ptr()
        if out is None:
            out = torch.empty(rows, pm.rows, dtype=torch.float32, device=x2.device)
            ldo = pm.rows
        # K split across the GPU where the row tiles alone leave SMs idle (wq_a, wkv, wo_b)
        ws_bytes = L.dsm_linear_splitk_workspace_bytes(rows, pm.rows)
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=x2.device)
        check(L.dsm_linear_splitk(ptr(staged), ptr(xscale), cap, k, pm.wfmt, pm.group_size, ptr(pm.packed), pm.rows,
                                  ptr(out), ldo, rows, ptr(ws), ws_bytes, s), "dsm_linear_splitk")
        return out

    def _grouped_wo_a(self, o: torch.Tensor, wo_a: torch.Tensor, y1: torch.Tensor) -> None:
        """y1[t, gi * rank + c] = o[gi, t] . wo_a[gi, c] for every group in one staging and one
        ``dsm_grouped_linear`` launch: the groups are the packed matrix's experts over group-major
        rows, and row gi * n + t goes to y1's row t * groups + gi seen as rows of rank values."""
        g, n, dg = o.shape
        rank = wo_a.shape[1]
        key = (wo_a.data_ptr(), wo_a._version, wo_a.dtype, wo_a.device)
        hit = self._packed.get("wo_a")
        if hit is None or hit[0] != key:
            hit = (key, pack("dense", data=wo_a.detach(), device=wo_a.device))
            self._packed["wo_a"] = hit
        pm = hit[1]
        maps = self._packed.get(("wo_a_rows", g, n))
        if maps is None or maps[0].device != o.device:
            offsets = torch.arange(0, g * n + 1, n, dtype=torch.int32, device=o.device)
            t = torch.arange(n, dtype=torch.int32, device=o.device)
            gi = torch.arange(g, dtype=torch.int32, device=o.device)
            row_map = (t.unsqueeze(0) * g + gi.unsqueeze(1)).reshape(-1).contiguous()
            maps = (offsets, row_map)
            self._packed[("wo_a_rows", g, n)] = maps
        L = lib()
        x_all = o.reshape(g * n, dg)
        cap = L.dsm_stage_rows_cap(g * n)
        staged = torch.empty(L.dsm_stage_bytes(cap, dg), dtype=torch.uint8, device=o.device)
        xscale = torch.empty(cap, dtype=torch.float32, device=o.device)
        s = stream_ptr()
        check(L.dsm_stage_rows(ptr(x_all), dtype_code(x_all.dtype), g * n, dg, None, g * n, 1, ptr(staged), cap,
                               ptr(xscale), s), "dsm_stage_rows")
        ws_bytes = L.dsm_linear_splitk_workspace_bytes(g * n, rank)
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=o.device)
        check(L.dsm_grouped_linear_splitk(ptr(staged), ptr(xscale), cap, dg, pm.wfmt, pm.group_size, ptr(pm.packed), g,
                                          ptr(maps[0]), rank, ptr(y1), rank, ptr(maps[1]), g * n, ptr(ws), ws_bytes,
                                          s), "dsm_grouped_linear_splitk")

    @staticmethod
    def _hilo(o: torch.Tensor, n: int):
        return (o[:n], o[n:]) if o.shape[0] == 2 * n else (o, None)

    def _norm_rope(self, x2: torch.Tensor, pm: PackedMatrix, weight: torch.Tensor, rope: bool, pos0: int, period: int,
                   st=None):
        n = x2.shape[0]
        hi, lo = self._hilo(self._linear(x2, pm, st=st), n)
        out = torch.empty(n, pm.rows, dtype=x2.dtype, device=x2.device)
        w = weight.detach().to(device=x2.device, dtype=torch.float32).contiguous()
        cos, sin = (self._cos, self._sin) if rope else (None, None)
        check(lib().dsm_rows_norm_rope(ptr(hi), ptr(lo), n, pm.rows, ptr(w), float(self.eps),
                                       self.rope_head_dim if rope else 0, ptr(cos), ptr(sin), pos0, period, ptr(out),
                                       dtype_code(x2.dtype), stream_ptr()), "dsm_rows_norm_rope")
        return out

    def _main_kv(self, main_x: torch.Tensor, start_pos: int) -> torch.Tensor:
        b, seqlen, _ = main_x.shape
        kv = self._norm_rope(main_x.reshape(b * seqlen, -1).contiguous(), self._pm("wkv", self.wkv.weight),
                             self.kv_norm.weight, True, start_pos, seqlen)
        return kv.reshape(b, seqlen, self.head_dim)

    def _write_window(self, rows: torch.Tensor, pos0: int) -> None:
        b, n, d = rows.shape
        check(lib().dsm_kv_window_write(ptr(rows), dtype_code(rows.dtype), b, n, d, pos0, self.window_size,
                                        ptr(self.window), stream_ptr()), "dsm_kv_window_write")

    # ---------------------------------------------------------------- calls
    def forward(self, x: torch.Tensor, start_pos: int, main_x: torch.Tensor) -> torch.Tensor:
        if not (x.is_cuda and main_x.is_cuda):
            raise ValueError("DSparkAttention runs on the GPU only")
        dt = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
        x, main_x = x.to(dt).contiguous(), main_x.to(dt).contiguous()
        b, seqlen, _ = main_x.shape
        block = x.shape[1] if start_pos > 0 else 0
        if start_pos < 0 or start_pos + seqlen + block > self._cos.shape[0]:
            raise ValueError(f"positions up to {start_pos + seqlen + block} exceed max_seq_len {self._cos.shape[0]}")
        main_kv = self._main_kv(main_x, start_pos)
        win = self.window_size
        if start_pos == 0:  # DSparkKVCache.prefill: slot p % window holds the last window positions
            self.window = torch.zeros(b, win, self.head_dim, dtype=dt, device=x.device)
            first = max(0, seqlen - win)
            self._write_window(main_kv[:, first:].contiguous(), first)
            return x
        if self.window is None or self.window.shape[0] != b or self.window.dtype != dt:
            raise ValueError("decode before a prefill of this batch")
        _, block, _ = x.shape
        n = b * block
        x2 = x.reshape(n, -1)
        pos_b = start_pos + seqlen  # positions of the block's rows
        h, hd, g = self.n_heads, self.head_dim, self.n_groups
        # q: wq_b(q_norm(wq_a(x))), per-head RMS, RoPE
        st = self._stage(x2)  # one staging of x for wq_a and wkv
        q_lat = self._norm_rope(x2, self._pm("wq_a", self.wq_a.weight), self.q_norm.weight, False, 0, 1, st=st)
        qh, ql = self._hilo(self._linear(q_lat, self._pm("wq_b", self.wq_b.weight)), n)
        q = torch.empty(n, h * hd, dtype=dt, device=x.device)
        check(lib().dsm_q_head_norm_rope(ptr(qh), ptr(ql), n, h, hd, float(self.eps), self.rope_head_dim,
                                         ptr(self._cos), ptr(self._sin), pos_b, block, ptr(q), dtype_code(dt),
                                         stream_ptr()), "dsm_q_head_norm_rope")
        kv = self._norm_rope(x2, self._pm("wkv", self.wkv.weight), self.kv_norm.weight, True, pos_b, block, st=st)
        self._write_window(main_kv[:, :1].contiguous(), start_pos)  # cache.update(start_pos, main_kv[:, 0])
        n_win = min(win, start_pos + 1)
        dg = h * hd // g
        o = torch.empty(g, n, dg, dtype=dt, device=x.device)
        L = lib()
        scratch = torch.empty(max(1, L.dsm_sparse_attn_scratch_bytes(b, block, h, n_win) // 4), dtype=torch.float32,
                              device=x.device)
        sink = self.attn_sink.detach().to(device=x.device, dtype=torch.float32).contiguous()
        check(L.dsm_sparse_attn(ptr(q), ptr(self.window), ptr(kv), dtype_code(dt), ptr(sink), b, block, h, hd, win,
                                n_win, float(self.softmax_scale), self.rope_head_dim, ptr(self._cos), ptr(self._sin),
                                pos_b, g, ptr(o), ptr(scratch), stream_ptr()), "dsm_sparse_attn")
        # grouped low-rank output projection: group gi's rows times wo_a[gi]
        rank = self.o_lora_rank
        rows = 2 * n if dt == torch.float32 else n
        y1 = torch.empty(rows, g * rank, dtype=torch.float32, device=x.device)
        wo_a = self.wo_a.weight.reshape(g, rank, dg)
        if dt == torch.bfloat16:
            self._grouped_wo_a(o, wo_a, y1)
        else:  # fp32 rows are staged hi + lo per group: one product per group
            for gi in range(g):
                self._linear(o[gi], self._pm(f"wo_a{gi}", wo_a[gi]), out=y1[:, gi * rank:], ldo=g * rank)
        y1h, y1l = self._hilo(y1, n)
        y1t = torch.empty(n, g * rank, dtype=dt, device=x.device)
        check(L.dsm_round_rows(ptr(y1h), ptr(y1l), y1t.numel(), ptr(y1t), dtype_code(dt), stream_ptr()),
              "dsm_round_rows")
        yh, yl = self._hilo(self._linear(y1t, self._pm("wo_b", self.wo_b.weight)), n)
        y = torch.empty(n, self.dim, dtype=dt, device=x.device)
        check(L.dsm_round_rows(ptr(yh), ptr(yl), y.numel(), ptr(y), dtype_code(dt), stream_ptr()), "dsm_round_rows")
        return y.reshape(b, block, self.dim)

    def advance_window(self, main_x: torch.Tensor, position: int) -> None:
        """One committed token's main KV into the window (``attention.py:131-142``)."""
        if self.window is None:
            raise ValueError("advance_window before a prefill")
        if not 0 <= position < self._cos.shape[0]:
            raise ValueError(f"position {position} outside max_seq_len {self._cos.shape[0]}")
        mx2 = main_x.reshape(main_x.shape[0], -1).to(self.window.dtype).contiguous()
        kv = self._norm_rope(mx2, self._pm("wkv", self.wkv.weight), self.kv_norm.weight, True, position, 1)
        self._write_window(kv.reshape(mx2.shape[0], 1, self.head_dim), position)
