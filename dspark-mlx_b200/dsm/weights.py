"""Expert weight formats and their packing into the kernel tile stream.

A stacked expert matrix ``[E, out, in]`` (nn.Linear layout, ``dspark_mlx/model/moe.py:103-120``)
can be held as

* ``dense``  bf16 / fp32 weights (the reference's unquantised experts); packed as f16 with a
  per-expert power-of-two prescale (exact for bf16 sources),
* ``fp8``    e4m3 codes with fp32 128x128 block scales (the bundled DeepSeek draft's
  checkpoint format; the reference dequantises it with ``dequant_fp8_blockwise``,
  ``dspark_mlx/loading.py:103-107``),
* ``fp4``    e2m1 codes (two per byte, element ``2j`` in the low nibble) with e4m3 scales per 32
  along K and an fp32 per-expert scale (``dequant_fp4_groupwise``, ``loading.py:110-114``,
  times the per-tensor scale),
* ``affine`` MLX affine 8/4-bit codes with per-group scale and bias (``MoE.quantize``,
  ``moe.py:124-130``).

``pack`` converts any of them, on the GPU, into the layout the expert kernels stream.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_ptr


@dataclass
class PackedMatrix:
    wfmt: int
    group_size: int
    n_experts: int
    rows: int
    cols: int
    packed: torch.Tensor  # uint8, device

    @property
    def nbytes(self) -> int:
        return self.packed.numel()


def _dev_u8(t: torch.Tensor, device) -> torch.Tensor:
    if t.dtype != torch.uint8 and t.element_size() == 1:  # e4m3 / e8m0 / packed e2m1 / int8 bytes
        t = t.view(torch.uint8)
    return t.to(device=device).contiguous()


def pack(kind: str, *, data: torch.Tensor, scales: Optional[torch.Tensor] = None,
         biases: Optional[torch.Tensor] = None, tensor_scale: Optional[torch.Tensor] = None,
         group_size: int = 64, bits: int = 8, device=None) -> PackedMatrix:
    """Pack one stacked expert matrix. ``data`` is ``[E, out, in]`` (or ``[out, in]``: one expert)."""
    device = torch.device(device) if device is not None else (data.device if data.is_cuda else torch.device("cuda"))
    if data.dim() == 2:
        data = data.unsqueeze(0)
        scales = scales.unsqueeze(0) if scales is not None else None
        biases = biases.unsqueeze(0) if biases is not None else None
        if tensor_scale is not None:
            tensor_scale = tensor_scale.reshape(1)
    E, R = data.shape[0], data.shape[1]
    if kind == "dense":
        wfmt, K = _lib.WFMT_F16, data.shape[2]
        src = data.to(device=device).contiguous()
        if src.dtype not in (torch.float32, torch.bfloat16):
            src = src.to(torch.float32)
        args = (ptr(src), None, None, None, dtype_code(src.dtype))
        keep = (src,)
        gs = 0
    elif kind == "fp8":
        wfmt, K = _lib.WFMT_FP8_B128, data.shape[2]
        codes = _dev_u8(data, device)
        sc = scales.to(device=device, dtype=torch.float32).contiguous()
        if tuple(sc.shape) != (E, -(-R // 128), -(-K // 128)):
            raise ValueError(f"fp8 scales must be [E, ceil(out/128), ceil(in/128)], got {tuple(sc.shape)}")
        args = (ptr(codes), ptr(sc), None, None, _lib.DT_F32)
        keep = (codes, sc)
        gs = 128
    elif kind == "fp4":
        wfmt, K = _lib.WFMT_FP4_G32, data.shape[2] * 2
        codes = _dev_u8(data, device)
        gsc = _dev_u8(scales, device)
        ts = tensor_scale.to(device=device, dtype=torch.float32).reshape(E).contiguous()
        if tuple(gsc.shape) != (E, R, K // 32):
            raise ValueError(f"fp4 group scales must be [E, out, in/32], got {tuple(gsc.shape)}")
        args = (ptr(codes), ptr(gsc), None, ptr(ts), _lib.DT_F32)
        keep = (codes, gsc, ts)
        gs = 32
    elif kind == "affine":
        wfmt = _lib.WFMT_AFFINE8 if bits == 8 else _lib.WFMT_AFFINE4
        K = data.shape[2] * 8 // bits
        codes = _dev_u8(data, device)
        sc = scales.to(device=device, dtype=torch.bfloat16).contiguous()
        bi = biases.to(device=device, dtype=torch.bfloat16).contiguous()
        args = (ptr(codes), ptr(sc), ptr(bi), None, _lib.DT_BF16)
        keep = (codes, sc, bi)
        gs = group_size
    else:
        raise ValueError(f"unknown weight kind {kind!r}")
    nbytes = lib().dsm_packed_bytes(wfmt, E, R, K, gs)
    if nbytes == 0:
        raise ValueError("unsupported packing shape")
    packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
    codes_p, scales_p, biases_p, ts_p, src_dt = args
    with torch.cuda.device(device):
        check(lib().dsm_pack_weights(wfmt, E, R, K, gs, src_dt, codes_p, scales_p, biases_p, ts_p,
                                     ptr(packed), stream_ptr()), "dsm_pack_weights")
    del keep
    return PackedMatrix(wfmt, gs, E, R, K, packed)


def affine_quantize(w: torch.Tensor, group_size: int = 64, bits: int = 8):
    """MLX affine quantize of ``w [..., K]`` on the GPU -> ``(codes uint8, scales, biases)``.

    Scales and biases keep ``w``'s dtype (bf16 or fp32), as ``mx.quantize`` does.
    """
    if not w.is_cuda:
        raise ValueError("affine_quantize expects a CUDA tensor")
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.to(torch.float32)
    w = w.contiguous()
    K = w.shape[-1]
    rows = w.numel() // K
    codes = torch.empty(*w.shape[:-1], K * bits // 8, dtype=torch.uint8, device=w.device)
    scales = torch.empty(*w.shape[:-1], K // group_size, dtype=w.dtype, device=w.device)
    biases = torch.empty_like(scales)
    with torch.cuda.device(w.device):
        check(lib().dsm_affine_quantize(ptr(w), dtype_code(w.dtype), rows, K, group_size, bits, ptr(codes),
                                        ptr(scales), ptr(biases), stream_ptr()), "dsm_affine_quantize")
    return codes, scales, biases
