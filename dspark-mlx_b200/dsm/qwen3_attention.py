"""The Qwen3 DSpark draft attention on the GPU: ``Qwen3DSparkAttention``
(``dspark_mlx/arch/qwen3.py:84-143``).

Same constructor (``Qwen3DSparkAttention(args)``), parameter names (``q_proj``, ``k_proj``,
``v_proj``, ``o_proj``, ``q_norm``, ``k_norm``) and calls as the reference:

* ``attn(hidden [b, q, hidden], target_ctx [b, ctx, hidden], cos_full, sin_full)``: the block
  over ``[context || block]``; the tables have ``ctx + q`` rows and the block's queries take
  the last ``q`` (``qwen3.py:97-116``);
* ``context_kv(proj_ctx [b, n, hidden], cos, sin)`` -> RoPE'd ``(k, v)`` ``[b, n_kv, n,
  head_dim]`` (``qwen3.py:122-128``); ``out=(k_cache, v_cache), row0=`` writes them into
  rows ``row0 ..`` of preallocated ``[b, n_kv, cap, head_dim]`` caches instead;
* ``attend_cached(noise, ctx_k, ctx_v, cos, sin)``: the block over cached context K/V
  (``None`` for none; any view whose rows are ``head_dim`` contiguous values) and its own
  rows (``qwen3.py:130-143``).

The projections are ``Projection``s, dense or MLX affine after ``quantize`` as
``quantize_drafter`` leaves them, on ``dsm_linear`` (quantised ones on
``dsm_linear_splitk``, which spreads K over the GPU). q, k and v share one staging of the
input and one fp32 output slab; quantised alike, they are one packed matrix of stacked rows
and one product. The head norms, NeoX RoPE and the cache layout are one
``dsm_qkv_norm_rope``; the attention is ``dsm_gqa_attn``; ``o_proj`` is one more
``dsm_linear``. The activation dtype is the projections' MLX product dtype (bf16 or fp32).
CPU tensors are rejected.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import nn

from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .block import RMSNorm
from .qwen3 import Projection
from .weights import pack


def rope_tables(position_ids, head_dim: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``rope_tables`` (``qwen3.py:76-81``): cos/sin ``[len(position_ids), head_dim]`` in fp32,
    computed on the CPU as the reference computes them."""
    pos = torch.as_tensor(position_ids).cpu()
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).to(torch.float32) / head_dim))
    freqs = pos.to(torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return torch.cos(emb), torch.sin(emb)


def _get(args, key):
    return args[key] if isinstance(args, dict) else getattr(args, key)


class Qwen3DSparkAttention(nn.Module):
    def __init__(self, args):
        super().__init__()
        h = int(_get(args, "hidden_size"))
        nh, nkv = int(_get(args, "num_attention_heads")), int(_get(args, "num_key_value_heads"))
        hd = int(_get(args, "head_dim"))
        eps = float(_get(args, "rms_norm_eps"))
        if nh % nkv:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")
        self.hidden, self.nh, self.nkv, self.hd = h, nh, nkv, hd
        self.scale = hd ** -0.5
        self.q_proj = Projection(h, nh * hd)
        self.k_proj = Projection(h, nkv * hd)
        self.v_proj = Projection(h, nkv * hd)
        self.o_proj = Projection(nh * hd, h)
        self.q_norm = RMSNorm(hd, eps)
        self.k_norm = RMSNorm(hd, eps)
        self._fused = {}  # with_q -> (source key, packed q/k/v rows): see _fused_packed

    # ---------------------------------------------------------------- helpers
    def _act_dtype(self, x: torch.Tensor) -> torch.dtype:
        dts = {p.product_dtype(x.dtype) for p in (self.q_proj, self.k_proj, self.v_proj)}
        if len(dts) != 1:
            raise ValueError(f"q/k/v projections give different dtypes {sorted(map(str, dts))}")
        dt = dts.pop()
        if dt not in (torch.bfloat16, torch.float32):
            raise ValueError(f"activation dtype {dt} unsupported (bf16 or fp32)")
        return dt

    @staticmethod
    def _stage(x2: torch.Tensor):
        """Stage rows for dsm_linear: bf16 exactly, fp32 as hi + lo f16 rows (2n rows)."""
        L = lib()
        n, k = x2.shape
        f32 = x2.dtype == torch.float32
        rows = 2 * n if f32 else n
        cap = L.dsm_stage_rows_cap(rows)
        staged = torch.empty(L.dsm_stage_bytes(cap, k), dtype=torch.uint8, device=x2.device)
        xscale = torch.empty(cap, dtype=torch.float32, device=x2.device)
        if f32:
            check(L.dsm_stage_rows_hilo(ptr(x2), n, k, ptr(staged), cap, ptr(xscale), stream_ptr()),
                  "dsm_stage_rows_hilo")
        else:
            check(L.dsm_stage_rows(ptr(x2), dtype_code(x2.dtype), n, k, None, n, 1, ptr(staged), cap, ptr(xscale),
                                   stream_ptr()), "dsm_stage_rows")
        return staged, xscale, cap, rows, k

    def _fused_packed(self, with_q: bool):
        """k_proj and v_proj (after q_proj when with_q) as one packed matrix of their stacked
        output rows, when all of them are quantised alike; else None. One product then fills
        the q/k/v slab, instead of one launch per projection with its own pipeline fill and
        split sum. The packed rows are cached and rebuilt when a source tensor changes."""
        projs = ((self.q_proj,) if with_q else ()) + (self.k_proj, self.v_proj)
        quant = projs[0].quant
        if quant is None or any(p.quant != quant for p in projs):
            return None
        srcs = [t for p in projs for t in (p.q, p.scales, p.biases)]
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in srcs)
        hit = self._fused.get(with_q)
        if hit is None or hit[0] != key:
            bits, gs = quant
            q = torch.cat([p.q for p in projs], 0)
            sc = torch.cat([p.scales for p in projs], 0)
            bi = torch.cat([p.biases for p in projs], 0)
            hit = (key, pack("affine", data=q, scales=sc, biases=bi, group_size=gs, bits=bits, device=q.device))
            self._fused[with_q] = hit
        return hit[1]

    @staticmethod
    def _project(st, proj: Projection, out: torch.Tensor, ldo: int, pm=None) -> None:
        """out[:, :proj.out_dim] (row stride ldo) = the staged rows times the projection (or times
        the packed matrix pm, quantised like proj). Quantised projections split K across the GPU
        (``dsm_linear_splitk``)."""
        staged, xscale, cap, rows, k = st
        pm = proj.packed() if pm is None else pm
        L = lib()
        if proj.quant is None:
            check(L.dsm_linear(ptr(staged), ptr(xscale), cap, k, pm.wfmt, pm.group_size, ptr(pm.packed), pm.rows,
                               ptr(out), ldo, rows, stream_ptr()), "dsm_linear")
            return
        ws_bytes = L.dsm_linear_splitk_workspace_bytes(rows, pm.rows)
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=out.device)
        check(L.dsm_linear_splitk(ptr(staged), ptr(xscale), cap, k, pm.wfmt, pm.group_size, ptr(pm.packed), pm.rows,
                                  ptr(out), ldo, rows, ptr(ws), ws_bytes, stream_ptr()), "dsm_linear_splitk")

    def _prep(self, x: torch.Tensor, name: str) -> Tuple[torch.Tensor, torch.dtype]:
        if not x.is_cuda:
            raise ValueError(f"Qwen3DSparkAttention runs on the GPU only ({name} is on the CPU)")
        if x.dim() != 3 or x.shape[-1] != self.hidden:
            raise ValueError(f"{name} must be [batch, seq, {self.hidden}], got {tuple(x.shape)}")
        dt = self._act_dtype(x)
        xin = x if x.dtype in (torch.bfloat16, torch.float32) else x.to(dt)
        return xin.contiguous(), dt

    def _tables(self, cos: torch.Tensor, sin: torch.Tensor, device) -> Tuple[torch.Tensor, torch.Tensor]:
        cos = torch.as_tensor(cos).to(device=device, dtype=torch.float32).contiguous()
        sin = torch.as_tensor(sin).to(device=device, dtype=torch.float32).contiguous()
        if cos.dim() != 2 or cos.shape[1] != self.hd or cos.shape != sin.shape:
            raise ValueError(f"cos/sin must be [positions, {self.hd}], got {tuple(cos.shape)} / {tuple(sin.shape)}")
        return cos, sin

    def _heads(self, x: torch.Tensor, dt: torch.dtype, with_q: bool, cos, sin, tab0: int, k_out, v_out, kv_cap: int,
               row0: int) -> Optional[torch.Tensor]:
        """q (optional), k and v of x's rows: q -> [b, s, nh, hd]; k, v -> caches at row0 + t."""
        b, s, _ = x.shape
        n = b * s
        nq = self.nh if with_q else 0
        cols = (nq + 2 * self.nkv) * self.hd
        st = self._stage(x.reshape(n, -1))
        rows = st[3]
        slab = torch.empty(rows, cols, dtype=torch.float32, device=x.device)
        fused = self._fused_packed(with_q)
        if fused is not None:
            self._project(st, self.k_proj, slab, cols, pm=fused)
        else:
            c = 0
            for proj, used in ((self.q_proj, with_q), (self.k_proj, True), (self.v_proj, True)):
                if used:
                    self._project(st, proj, slab[:, c:], cols)
                    c += proj.out_dim
        lo = slab[n:] if rows == 2 * n else None
        q = torch.empty(b, s, self.nh, self.hd, dtype=dt, device=x.device) if with_q else None
        qw = self.q_norm.weight.detach().to(device=x.device, dtype=torch.float32).contiguous()
        kw = self.k_norm.weight.detach().to(device=x.device, dtype=torch.float32).contiguous()
        check(lib().dsm_qkv_norm_rope(ptr(slab), ptr(lo), n, nq, self.nkv, self.hd, ptr(qw), ptr(kw),
                                      float(self.q_norm.eps), ptr(cos), ptr(sin), cos.shape[0], tab0, s, ptr(q),
                                      ptr(k_out), ptr(v_out), kv_cap, row0, dtype_code(dt), stream_ptr()),
              "dsm_qkv_norm_rope")
        return q

    def _attend(self, q: torch.Tensor, ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor],
                blk_k: torch.Tensor, blk_v: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
        b, s = q.shape[:2]
        n_ctx, sb, sh = 0, 0, 0
        if ctx_k is not None:
            for name, t in (("ctx_k", ctx_k), ("ctx_v", ctx_v)):
                if t is None or t.dim() != 4 or t.shape[0] != b or t.shape[1] != self.nkv or t.shape[3] != self.hd:
                    raise ValueError(f"{name} must be [{b}, {self.nkv}, n, {self.hd}]")
                if t.dtype != dt or t.device != q.device:
                    raise ValueError(f"{name} must be {dt} on {q.device}")
                if t.stride(3) != 1 or t.stride(2) != self.hd:
                    raise ValueError(f"{name} rows must be {self.hd} contiguous values")
            if ctx_v.shape != ctx_k.shape or ctx_v.stride() != ctx_k.stride():
                raise ValueError("ctx_k and ctx_v must have the same shape and strides")
            n_ctx, sb, sh = ctx_k.shape[2], ctx_k.stride(0), ctx_k.stride(1)
        L = lib()
        out = torch.empty(b, s, self.nh * self.hd, dtype=dt, device=q.device)
        ws_bytes = L.dsm_gqa_attn_workspace_bytes(b, s, self.nh, self.nkv, self.hd, n_ctx)
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=q.device)
        check(L.dsm_gqa_attn(ptr(q), ptr(ctx_k) if n_ctx else None, ptr(ctx_v) if n_ctx else None, sb, sh, n_ctx,
                             ptr(blk_k), ptr(blk_v), dtype_code(dt), b, s, self.nh, self.nkv, self.hd,
                             float(self.scale), ptr(out), ptr(ws), ws_bytes, stream_ptr()), "dsm_gqa_attn")
        return out

    def _out(self, attn: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
        b, s, _ = attn.shape
        n = b * s
        st = self._stage(attn.reshape(n, -1))
        rows = st[3]
        o = torch.empty(rows, self.hidden, dtype=torch.float32, device=attn.device)
        self._project(st, self.o_proj, o, self.hidden)
        y = torch.empty(b, s, self.hidden, dtype=dt, device=attn.device)
        check(lib().dsm_round_rows(ptr(o), ptr(o[n:]) if rows == 2 * n else None, y.numel(), ptr(y),
                                   dtype_code(dt), stream_ptr()), "dsm_round_rows")
        return y

    # ---------------------------------------------------------------- calls
    def forward(self, hidden: torch.Tensor, target_ctx: torch.Tensor, cos_full, sin_full) -> torch.Tensor:
        hidden, dt = self._prep(hidden, "hidden")
        target_ctx, dt_c = self._prep(target_ctx, "target_ctx")
        if dt_c != dt or target_ctx.shape[0] != hidden.shape[0]:
            raise ValueError("hidden and target_ctx must share batch and dtype")
        b, q, _ = hidden.shape
        ctx = target_ctx.shape[1]
        cos, sin = self._tables(cos_full, sin_full, hidden.device)
        if cos.shape[0] != ctx + q:
            raise ValueError(f"cos_full/sin_full must have ctx + q = {ctx + q} rows, got {cos.shape[0]}")
        ck = torch.empty(b, self.nkv, ctx, self.hd, dtype=dt, device=hidden.device)
        cv = torch.empty_like(ck)
        if ctx:
            self._heads(target_ctx, dt, False, cos, sin, 0, ck, cv, ctx, 0)
        bk = torch.empty(b, self.nkv, q, self.hd, dtype=dt, device=hidden.device)
        bv = torch.empty_like(bk)
        qh = self._heads(hidden, dt, True, cos, sin, ctx, bk, bv, q, 0)
        return self._out(self._attend(qh, ck if ctx else None, cv if ctx else None, bk, bv, dt), dt)

    def context_kv(self, proj_ctx: torch.Tensor, cos, sin, out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                   row0: int = 0):
        proj_ctx, dt = self._prep(proj_ctx, "proj_ctx")
        b, n, _ = proj_ctx.shape
        cos, sin = self._tables(cos, sin, proj_ctx.device)
        if cos.shape[0] != n:
            raise ValueError(f"cos/sin must have {n} rows, got {cos.shape[0]}")
        if out is None:
            k = torch.empty(b, self.nkv, n, self.hd, dtype=dt, device=proj_ctx.device)
            v = torch.empty_like(k)
            cap, row0 = n, 0
        else:
            k, v = out
            for name, t in (("k cache", k), ("v cache", v)):
                if (t.dim() != 4 or t.shape[0] != b or t.shape[1] != self.nkv or t.shape[3] != self.hd
                        or not t.is_contiguous() or t.dtype != dt or t.device != proj_ctx.device):
                    raise ValueError(f"{name} must be a contiguous [{b}, {self.nkv}, cap, {self.hd}] {dt} tensor")
            if v.shape != k.shape:
                raise ValueError("k and v caches must have the same shape")
            cap = k.shape[2]
            if row0 < 0 or row0 + n > cap:
                raise ValueError(f"rows {row0}..{row0 + n} outside the cache's {cap}")
        if n:
            self._heads(proj_ctx, dt, False, cos, sin, 0, k, v, cap, row0)
        return k, v

    def attend_cached(self, noise: torch.Tensor, ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor], cos,
                      sin) -> torch.Tensor:
        noise, dt = self._prep(noise, "noise")
        b, q, _ = noise.shape
        cos, sin = self._tables(cos, sin, noise.device)
        if cos.shape[0] != q:
            raise ValueError(f"cos/sin must have {q} rows, got {cos.shape[0]}")
        if (ctx_k is None) != (ctx_v is None):
            raise ValueError("ctx_k and ctx_v must both be given or both be None")
        bk = torch.empty(b, self.nkv, q, self.hd, dtype=dt, device=noise.device)
        bv = torch.empty_like(bk)
        qh = self._heads(noise, dt, True, cos, sin, 0, bk, bv, q, 0)
        return self._out(self._attend(qh, ctx_k, ctx_v, bk, bv, dt), dt)
