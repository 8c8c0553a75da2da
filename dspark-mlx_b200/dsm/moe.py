"""Drop-in DSpark draft-layer MoE for B200: ``Gate``, ``Expert`` and ``MoE``.

Mirrors the reference module ``dspark_mlx/model/moe.py`` -- the same constructor
(``MoE(args, layer_id)``), call signature (``moe(x, input_ids) -> y`` of x's shape and
dtype), ``quantize(bits, group_size)`` and parameter names (``gate.weight``,
``gate.bias`` | ``gate.tid2eid``, stacked ``w1``/``w3`` ``[E, inter, dim]`` and ``w2``
``[E, dim, inter]``, ``w{n}_q``/``_scales``/``_biases`` after quantisation,
``shared_experts.w{1,2,3}.weight``) -- so callers of the reference MoE
(``DSparkBlock.__call__``, ``dspark_mlx/model/block.py:85``) are unchanged.

PyTorch tensors are only the containers: every call goes through ``libdsm.so``
(hand-written sm_100a kernels). There is no CPU path; CPU tensors are rejected.

Beyond the reference, the routed experts can also be held in the checkpoint's own fp8
(128x128 block scales) and fp4 (group-32 scales) formats without dequantising them
(:meth:`MoE.load_fp8_experts`, :meth:`MoE.load_fp4_experts`).
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
from torch import nn

from . import _lib
from ._lib import MoEDesc, check, dtype_code, lib, ptr, stream_ptr
from .weights import PackedMatrix, affine_quantize, pack

_ROUTED = ("w1", "w3", "w2")


def _cuda_contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libdsm has no CPU path)")
    return t if t.is_contiguous() else t.contiguous()


def _ids_arg(input_ids: Optional[torch.Tensor]):
    if input_ids is None:
        return None, None, _lib.DT_I32, 0
    ids = _cuda_contig(input_ids, "input_ids").reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.to(torch.int32)
    return ids, ptr(ids), dtype_code(ids.dtype), ids.numel()


class Gate(nn.Module):
    """Expert routing (``dspark_mlx/model/moe.py:47-79``): hash routing when
    ``layer_id < n_hash_layers``, else score routing with a selection-only bias."""

    def __init__(self, args, layer_id: int):
        super().__init__()
        self.topk = args.n_activated_experts
        self.score_func = args.score_func
        self.route_scale = args.route_scale
        self.hash = layer_id < args.n_hash_layers
        self.register_buffer("weight", torch.zeros(args.n_routed_experts, args.dim, dtype=torch.float32))
        if self.hash:
            self.register_buffer("tid2eid", torch.zeros(args.vocab_size, args.n_activated_experts, dtype=torch.int32))
        else:
            self.register_buffer("bias", torch.zeros(args.n_routed_experts, dtype=torch.float32))

    def router_args(self):
        w = _cuda_contig(self.weight.to(torch.float32), "gate.weight")
        if self.hash:
            t2e = _cuda_contig(self.tid2eid.to(torch.int32), "gate.tid2eid")
            return w, None, t2e
        return w, _cuda_contig(self.bias.to(torch.float32), "gate.bias"), None

    def forward(self, x: torch.Tensor, input_ids: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """``(weights [N, k] fp32, indices [N, k] int32)`` for ``x [N, dim]``."""
        x = _cuda_contig(x, "x")
        if x.dtype not in (torch.float32, torch.bfloat16):
            x = x.to(torch.float32)
        n, dim = x.shape
        w, b, t2e = self.router_args()
        ids, ids_p, ids_dt, n_ids = _ids_arg(input_ids)
        if self.hash and ids is None:
            raise ValueError("hash routing needs input_ids")
        scores = torch.empty(lib().dsm_router_workspace_bytes(n, dim, w.shape[0]), dtype=torch.uint8, device=x.device)
        weights = torch.empty(n, self.topk, dtype=torch.float32, device=x.device)
        indices = torch.empty(n, self.topk, dtype=torch.int32, device=x.device)
        check(lib().dsm_router(ptr(x), dtype_code(x.dtype), n, dim, ptr(w), w.shape[0], ptr(b), ptr(t2e),
                               t2e.shape[0] if t2e is not None else 0, ids_p, ids_dt, n_ids, self.topk,
                               _lib.SCORE[self.score_func], float(self.route_scale), ptr(scores), ptr(weights),
                               ptr(indices), stream_ptr()), "dsm_router")
        return weights, indices


class _Linear(nn.Module):
    """Bias-free linear weight holder (``nn.Linear`` layout ``[out, in]``). A ``meta`` weight
    marks a matrix the owning :class:`Expert` holds packed; it stays a placeholder through
    ``.to()`` / ``.cuda()``."""

    def __init__(self, in_dim: int, out_dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_dim, in_dim, dtype=torch.float32), requires_grad=False)
        nn.init.uniform_(self.weight, -in_dim ** -0.5, in_dim ** -0.5)

    def _apply(self, fn, recurse=True):
        w = self._parameters.get("weight")
        if w is None or not w.is_meta:
            return super()._apply(fn, recurse)
        self._parameters["weight"] = None
        try:
            return super()._apply(fn, recurse)
        finally:
            self._parameters["weight"] = w


class Expert(nn.Module):
    """The always-on shared expert (``dspark_mlx/model/moe.py:82-97``): ``w2(swiglu(w1 x, w3 x))``."""

    def __init__(self, dim: int, inter_dim: int, swiglu_limit: float = 0.0):
        super().__init__()
        self.w1 = _Linear(dim, inter_dim)
        self.w2 = _Linear(inter_dim, dim)
        self.w3 = _Linear(dim, inter_dim)
        self.swiglu_limit = swiglu_limit
        self._cache = None

    @property
    def format(self) -> str:
        """``"fp8"`` after :meth:`load_fp8` (the weights are then placeholders), else ``"dense"``."""
        return "fp8" if self.w1.weight.is_meta else "dense"

    def weight_dtype(self, name: str) -> torch.dtype:
        """The dtype the reference computes this matrix in: its loader dequantises an fp8
        checkpoint matrix to fp32 (``dspark_mlx/loading.py:103-107``)."""
        return torch.float32 if self.format == "fp8" else getattr(self, name).weight.dtype

    def load_fp8(self, **mats) -> None:
        """Hold the shared expert as e4m3 codes + fp32 128x128 block scales, the checkpoint's
        format for projection weights. Keywords ``w1``, ``w3``, ``w2``: ``(codes
        uint8|float8_e4m3fn [out, in], scales fp32 [ceil(out/128), ceil(in/128)])``."""
        for n in ("w1", "w3", "w2"):
            codes, scales = mats[n]
            lin = getattr(self, n)
            shape = tuple(lin.weight.shape)
            if tuple(codes.shape) != shape:
                raise ValueError(f"shared expert {n}: codes must be {shape}, got {tuple(codes.shape)}")
            lin.weight = nn.Parameter(torch.empty(shape, dtype=torch.float32, device="meta"), requires_grad=False)
            self.register_buffer(f"{n}_codes", codes.view(torch.uint8) if codes.dtype != torch.uint8 else codes)
            self.register_buffer(f"{n}_scale", scales.to(torch.float32))
        self._cache = None

    def packed(self) -> Tuple[PackedMatrix, PackedMatrix, PackedMatrix]:
        names = ("w1", "w3", "w2")
        if self.format == "fp8":
            srcs = tuple(getattr(self, f"{n}_{s}") for n in names for s in ("codes", "scale"))
        else:
            srcs = tuple(getattr(self, n).weight for n in names)
        key = tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in srcs)
        if self._cache is None or self._cache[0] != key:
            if self.format == "fp8":
                mats = tuple(pack("fp8", data=srcs[2 * i], scales=srcs[2 * i + 1], device=srcs[2 * i].device)
                             for i in range(3))
            else:
                mats = tuple(pack("dense", data=t.detach(), device=t.device) for t in srcs)
            self._cache = (key, mats)
        return self._cache[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Standalone call: the same kernels with a single group holding every row."""
        shape, dt = x.shape, x.dtype
        x2 = _cuda_contig(x.reshape(-1, shape[-1]), "x")
        p1, p3, p2 = self.packed()
        n = x2.shape[0]
        L = lib()
        cap = L.dsm_stage_rows_cap(n)
        dev = x.device
        offsets = torch.tensor([0, n], dtype=torch.int32, device=dev)
        xs = torch.empty(L.dsm_stage_bytes(cap, p1.cols), dtype=torch.uint8, device=dev)
        xscale = torch.empty(cap, dtype=torch.float32, device=dev)
        hs = torch.empty(L.dsm_stage_bytes(cap, p1.rows), dtype=torch.uint8, device=dev)
        o = torch.empty(n, p2.rows, dtype=torch.float32, device=dev)
        s = stream_ptr()
        check(L.dsm_stage_rows(ptr(x2), dtype_code(x2.dtype), n, p1.cols, None, n, 1, ptr(xs), cap, ptr(xscale), s),
              "dsm_stage_rows")
        bf16x = x2.dtype == torch.bfloat16
        rgu = int(bf16x and self.weight_dtype("w1") == torch.bfloat16) | (2 if bf16x else 0)
        rgo = int(bf16x and self.weight_dtype("w2") == torch.bfloat16)
        hsc = 1.0 if 0 < self.swiglu_limit and self.swiglu_limit ** 2 < 30000 else 1.0 / 256
        check(L.dsm_expert_gate_up(ptr(xs), ptr(xscale), cap, p1.cols, ptr(offsets), 1, p1.wfmt, p1.group_size,
                                   ptr(p1.packed), ptr(p3.packed), p1.rows, _lib.ACT_SWIGLU_CLAMP,
                                   float(self.swiglu_limit), rgu, ptr(hs), hsc, n, s), "dsm_expert_gate_up")
        check(L.dsm_expert_down(ptr(hs), hsc, cap, p2.cols, ptr(offsets), 1, p2.wfmt, p2.group_size, ptr(p2.packed),
                                p2.rows, rgo, ptr(o), p2.rows, None, n, s), "dsm_expert_down")
        out_dt = torch.promote_types(dt, self.weight_dtype("w2"))
        return o.to(out_dt).reshape(*shape[:-1], p2.rows)


class MoE(nn.Module):
    """Top-k routed experts (stacked, grouped by expert on the GPU) plus the shared expert
    (``dspark_mlx/model/moe.py:100-161``)."""

    def __init__(self, args, layer_id: int):
        super().__init__()
        self.dim = args.dim
        self.inter_dim = args.moe_inter_dim
        self.n_routed_experts = args.n_routed_experts
        self.swiglu_limit = args.swiglu_limit
        self.gate = Gate(args, layer_id)
        E, dim, inter = args.n_routed_experts, args.dim, args.moe_inter_dim
        # Shape-only placeholders until weights are assigned (the reference's mx.zeros is
        # lazy; eager fp32 zeros would cost 25 GB at DeepSeek-V4 sizes).
        self.register_buffer("w1", torch.empty(E, inter, dim, dtype=torch.float32, device="meta"))
        self.register_buffer("w3", torch.empty(E, inter, dim, dtype=torch.float32, device="meta"))
        self.register_buffer("w2", torch.empty(E, dim, inter, dtype=torch.float32, device="meta"))
        self.shared_experts = Expert(dim, inter, args.swiglu_limit)
        self.quant: Optional[Tuple[int, int]] = None
        self.expert_format = "dense"
        self._packed = None
        self._ws: Optional[torch.Tensor] = None

    def _apply(self, fn, recurse=True):
        # unassigned (meta) expert stacks stay placeholders through .to() / .cuda()
        meta = {k: v for k, v in self._buffers.items() if v is not None and v.is_meta}
        for k in meta:
            self._buffers[k] = None
        try:
            return super()._apply(fn, recurse)
        finally:
            for k, v in meta.items():
                if self._buffers.get(k) is None:
                    self._buffers[k] = v

    # ------------------------------------------------------------------ weight formats
    def _sources(self):
        if self.expert_format == "dense":
            return [getattr(self, n) for n in _ROUTED]
        if self.expert_format == "affine":
            return [getattr(self, f"{n}_{s}") for n in _ROUTED for s in ("q", "scales", "biases")]
        if self.expert_format == "fp8":
            return [getattr(self, f"{n}_{s}") for n in _ROUTED for s in ("codes", "scale")]
        return [getattr(self, f"{n}_{s}") for n in _ROUTED for s in ("codes", "scale", "tensor_scale")]

    def _drop_routed(self):
        for n in _ROUTED:
            for suffix in ("", "_q", "_scales", "_biases", "_codes", "_scale", "_tensor_scale"):
                name = n + suffix
                if name in self._buffers:
                    del self._buffers[name]
        self._packed = None

    def quantize(self, bits: int = 8, group_size: int = 64) -> None:
        """Quantise the stacked routed experts in place (``moe.py:124-130``): MLX affine, on the GPU."""
        if self.expert_format != "dense":
            raise ValueError("quantize() needs dense routed experts")
        out = {}
        for n in _ROUTED:
            out[n] = affine_quantize(_cuda_contig(getattr(self, n), n), group_size=group_size, bits=bits)
        self._drop_routed()
        for n in _ROUTED:
            q, s, b = out[n]
            self.register_buffer(f"{n}_q", q)
            self.register_buffer(f"{n}_scales", s)
            self.register_buffer(f"{n}_biases", b)
        self.quant = (bits, group_size)
        self.expert_format = "affine"

    def load_fp8_experts(self, **mats) -> None:
        """Hold the routed experts as e4m3 codes + fp32 128x128 block scales.

        Keywords ``w1``, ``w3``, ``w2``: ``(codes uint8|float8_e4m3fn [E,out,in], scales fp32)``.
        """
        self._drop_routed()
        for n in _ROUTED:
            codes, scales = mats[n]
            self.register_buffer(f"{n}_codes", codes.view(torch.uint8) if codes.dtype != torch.uint8 else codes)
            self.register_buffer(f"{n}_scale", scales.to(torch.float32))
        self.quant = None
        self.expert_format = "fp8"

    def load_fp4_experts(self, **mats) -> None:
        """Hold the routed experts as packed e2m1 codes + e4m3 group-32 scales + fp32 per-expert scale.

        Keywords ``w1``, ``w3``, ``w2``: ``(codes uint8 [E,out,in/2], scales uint8 e4m3
        [E,out,in/32], tensor_scale fp32 [E])``.
        """
        self._drop_routed()
        for n in _ROUTED:
            codes, scales, ts = mats[n]
            self.register_buffer(f"{n}_codes", codes)
            self.register_buffer(f"{n}_scale", scales.view(torch.uint8) if scales.dtype != torch.uint8 else scales)
            self.register_buffer(f"{n}_tensor_scale", ts.to(torch.float32))
        self.quant = None
        self.expert_format = "fp4"

    def packed_experts(self) -> Tuple[PackedMatrix, PackedMatrix, PackedMatrix]:
        srcs = self._sources()
        if any(t.is_meta for t in srcs):
            raise ValueError("routed expert weights are not assigned (w1/w3/w2 are placeholders)")
        key = (self.expert_format,) + tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in srcs)
        if self._packed is None or self._packed[0] != key:
            f = self.expert_format
            mats = []
            for n in _ROUTED:
                if f == "dense":
                    mats.append(pack("dense", data=getattr(self, n)))
                elif f == "affine":
                    bits, gs = self.quant
                    mats.append(pack("affine", data=getattr(self, f"{n}_q"), scales=getattr(self, f"{n}_scales"),
                                     biases=getattr(self, f"{n}_biases"), group_size=gs, bits=bits))
                elif f == "fp8":
                    mats.append(pack("fp8", data=getattr(self, f"{n}_codes"), scales=getattr(self, f"{n}_scale")))
                else:
                    mats.append(pack("fp4", data=getattr(self, f"{n}_codes"), scales=getattr(self, f"{n}_scale"),
                                     tensor_scale=getattr(self, f"{n}_tensor_scale")))
            self._packed = (key, tuple(mats))
        return self._packed[1]

    # ------------------------------------------------------------------ forward
    def routed_round_flags(self, x_dtype: torch.dtype) -> Tuple[int, int]:
        """(gate/up flags, down flag) following the reference's dtypes for the routed experts."""
        bf16x = x_dtype == torch.bfloat16
        f = self.expert_format
        if f == "dense":
            prod_bf16 = bf16x and self.w1.dtype == torch.bfloat16
            o_bf16 = bf16x and self.w2.dtype == torch.bfloat16
        elif f == "affine":
            prod_bf16 = o_bf16 = bf16x  # gather_qmm returns the activation dtype
        else:
            prod_bf16 = o_bf16 = False  # fp8/fp4 weights are dequantised to fp32 by the reference
        return int(prod_bf16) | (2 if bf16x else 0), int(o_bf16)

    def _round_flags(self, x_dtype: torch.dtype):
        bf16x = x_dtype == torch.bfloat16
        rgu, ro = self.routed_round_flags(x_dtype)
        sh = self.shared_experts
        s_gu = bf16x and sh.weight_dtype("w1") == torch.bfloat16
        s_o = bf16x and sh.weight_dtype("w2") == torch.bfloat16
        hbit = 2 if bf16x else 0
        return rgu, ro, int(s_gu) | hbit, int(s_o)

    def describe(self, n_tokens: int, x_dtype: torch.dtype) -> Tuple[MoEDesc, tuple]:
        """The C descriptor for a call on ``n_tokens`` tokens (and the tensors it points into)."""
        p1, p3, p2 = self.packed_experts()
        s1, s3, s2 = self.shared_experts.packed()
        gw, gb, t2e = self.gate.router_args()
        rgu, ro, srgu, sro = self._round_flags(x_dtype)
        d = MoEDesc()
        d.n_tokens = n_tokens
        d.dim, d.inter, d.n_experts, d.topk = self.dim, self.inter_dim, self.n_routed_experts, self.gate.topk
        d.score_func = _lib.SCORE[self.gate.score_func]
        d.route_scale, d.swiglu_limit = float(self.gate.route_scale), float(self.swiglu_limit)
        d.gate_weight, d.gate_bias, d.tid2eid = ptr(gw), ptr(gb), ptr(t2e)
        d.vocab = t2e.shape[0] if t2e is not None else 0
        d.wfmt, d.group_size = p1.wfmt, p1.group_size
        d.w1, d.w3, d.w2 = ptr(p1.packed), ptr(p3.packed), ptr(p2.packed)
        d.round_gu, d.round_o = rgu, ro
        d.shared_wfmt, d.shared_group_size = s1.wfmt, s1.group_size
        d.s1, d.s3, d.s2 = ptr(s1.packed), ptr(s3.packed), ptr(s2.packed)
        d.shared_inter, d.shared_round_gu, d.shared_round_o = s1.rows, srgu, sro
        d.act = _lib.ACT_SWIGLU_CLAMP
        return d, (p1, p3, p2, s1, s3, s2, gw, gb, t2e)

    def workspace(self, desc: MoEDesc, device) -> torch.Tensor:
        need = lib().dsm_moe_workspace_bytes(ctypes.byref(desc))
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
        return self._ws

    def forward(self, x: torch.Tensor, input_ids: Optional[torch.Tensor] = None, *, return_routing: bool = False):
        """``MoE.__call__`` (``moe.py:151-161``): ``x [..., dim]`` -> ``y`` of x's shape and dtype."""
        shape, in_dtype = x.shape, x.dtype
        x2 = _cuda_contig(x.reshape(-1, self.dim), "x")
        if x2.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("x must be bf16 or fp32")
        n = x2.shape[0]
        ids, ids_p, ids_dt, n_ids = _ids_arg(input_ids)
        if self.gate.hash and ids is None:
            raise ValueError("hash routing needs input_ids")
        desc, keep = self.describe(n, x2.dtype)
        ws = self.workspace(desc, x2.device)
        y = torch.empty_like(x2)
        rw = torch.empty(n, self.gate.topk, dtype=torch.float32, device=x2.device) if return_routing else None
        ri = torch.empty(n, self.gate.topk, dtype=torch.int32, device=x2.device) if return_routing else None
        check(lib().dsm_moe_forward(ctypes.byref(desc), ptr(x2), dtype_code(x2.dtype), ids_p, ids_dt, n_ids, ptr(y),
                                    ptr(rw), ptr(ri), ptr(ws), ws.numel(), stream_ptr()), "dsm_moe_forward")
        del keep
        y = y.to(in_dtype).reshape(shape)
        if return_routing:
            return y, rw, ri
        return y
