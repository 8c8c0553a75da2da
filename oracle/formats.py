"""Weight-format arithmetic of the oracle (test infrastructure only).

Restates, on the CPU, the dequantisation maths the reference applies to the bundled
DeepSeek fp8/fp4 expert weights (``dspark_mlx/loading.py:103-114``) and the affine
quantiser the reference's ``MoE.quantize`` calls (``dspark_mlx/model/moe.py:124-130`` ->
``mlx.core.quantize``; third-party MLX, ``mlx>=0.31.0`` at ``pyproject.toml:20``, no lock
file, so no exact version is pinned).

Code decoding is written from the bit definitions (OCP 8-bit float e4m3 "fn" variant:
bias 7, no infinities, S.1111.111 is NaN; OCP 4-bit e2m1: bias 1, no NaN/inf) rather than
through a library cast, so the oracle does not inherit the product's conversions.

Layout conventions shared with the product (they are the formats' definitions):

* fp8 block weights: codes ``uint8 [..., out, in]`` (e4m3 bit patterns) and fp32 scales
  ``[..., ceil(out/128), ceil(in/128)]``; ``w = code * scale[row//128, col//128]``.
* fp4 group weights: codes ``uint8 [..., out, in/2]`` with element ``2j`` in the low nibble
  and ``2j+1`` in the high nibble; e4m3 group scales ``uint8 [..., out, in/32]``; an fp32
  per-tensor scale ``[...]``; ``w = (code * gscale) * tensor_scale``.
* affine (MLX) weights: codes packed little-endian (the byte view of MLX's uint32 packing:
  for 8 bits byte ``j`` is element ``j``; for 4 bits byte ``j`` holds element ``2j`` in the
  low nibble); scales and biases ``[..., out, in/group]`` in the weight dtype;
  ``w = q * scale + bias``.
"""

from __future__ import annotations

import numpy as np
import torch

__all__ = [
    "e4m3_decode",
    "e2m1_decode",
    "e4m3_encode",
    "e8m0_decode",
    "dequant_fp8_blockwise",
    "dequant_fp4_groupwise",
    "fp8_weight_dequant",
    "fp4_weight_dequant",
    "affine_quantize",
    "affine_unpack",
    "affine_dequantize",
]


def _e4m3_fields(c: torch.Tensor) -> torch.Tensor:
    """e4m3 (fn) bit patterns (int32) -> fp32 values, from the bit fields."""
    sign = torch.where((c & 0x80) != 0, -1.0, 1.0)
    exp = (c >> 3) & 0xF
    man = (c & 0x7).to(torch.float64)
    normal = (1.0 + man / 8.0) * torch.pow(2.0, (exp - 7).to(torch.float64))
    sub = (man / 8.0) * 2.0 ** -6
    val = torch.where(exp == 0, sub, normal) * sign
    val = torch.where((c & 0x7F) == 0x7F, torch.tensor(float("nan"), dtype=torch.float64), val)
    return val.to(torch.float32)


def _e2m1_fields(c: torch.Tensor) -> torch.Tensor:
    """e2m1 nibbles (int32, 0..15) -> fp32 values, from the bit fields."""
    sign = torch.where((c & 0x8) != 0, -1.0, 1.0)
    exp = (c >> 1) & 0x3
    man = (c & 0x1).to(torch.float64)
    normal = (1.0 + man / 2.0) * torch.pow(2.0, (exp - 1).to(torch.float64))
    sub = man * 0.5
    return (torch.where(exp == 0, sub, normal) * sign).to(torch.float32)


# Every code's value, decoded once from the bit fields above; decoding a tensor of codes is
# then a table lookup (the same values, without re-running the field arithmetic per element).
_E4M3_TABLE = _e4m3_fields(torch.arange(256, dtype=torch.int32))
_E2M1_TABLE = _e2m1_fields(torch.arange(16, dtype=torch.int32))


def _code_index(codes) -> torch.Tensor:
    if isinstance(codes, torch.Tensor):
        return codes.to(torch.int64) & 0xFF
    return torch.as_tensor(np.asarray(codes, dtype=np.uint8)).to(torch.int64)


def e4m3_decode(codes) -> torch.Tensor:
    """e4m3 (fn) bit patterns -> fp32 values (the bit-field decode of each code)."""
    return _E4M3_TABLE[_code_index(codes)]


def e2m1_decode(codes) -> torch.Tensor:
    """e2m1 nibbles (values 0..15) -> fp32 values (the bit-field decode of each code)."""
    return _E2M1_TABLE[_code_index(codes) & 0xF]


def e8m0_decode(codes) -> torch.Tensor:
    """e8m0 scale bytes -> fp32 ``2^(code - 127)`` (the checkpoint's block scales,
    ``dspark_mlx/loading.py:7-18``; 255 is NaN). Computed in float64, where every such power
    of two is exact, then rounded to fp32, where it is exact too (``2^-127`` as a subnormal)."""
    c = torch.as_tensor(np.asarray(codes, dtype=np.uint8)).to(torch.float64)
    val = torch.pow(torch.tensor(2.0, dtype=torch.float64), c - 127.0)
    return torch.where(c == 255, torch.tensor(float("nan"), dtype=torch.float64), val).to(torch.float32)


def e4m3_encode(values: torch.Tensor) -> torch.Tensor:
    """fp32 -> nearest e4m3 (fn) bit pattern, ties to even, saturating at +-448.

    Brute force over the 254 finite codes: used only to build small test inputs.
    """
    table = e4m3_decode(np.arange(256, dtype=np.uint8)).to(torch.float64)
    finite = ~torch.isnan(table)
    codes = torch.arange(256)[finite]
    vals = table[finite]
    v = values.to(torch.float64).clamp(-448.0, 448.0).reshape(-1, 1)
    d = (v - vals.reshape(1, -1)).abs()
    best = d.min(dim=1, keepdim=True).values
    cand = d == best
    # tie -> even mantissa (bit 0 clear); also prefer +0 over -0
    even = ((codes & 1) == 0).reshape(1, -1) & cand
    pick = torch.where(even.any(dim=1, keepdim=True), even, cand)
    pick = pick & ~((codes == 0x80).reshape(1, -1) & pick.sum(1, keepdim=True).gt(1))
    idx = pick.to(torch.int64).argmax(dim=1)
    return codes[idx].to(torch.uint8).reshape(values.shape)


def dequant_fp8_blockwise(weight: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """``dspark_mlx/loading.py:103-107``: f32 weight times a 2-D block-repeated scale."""
    out, inn = weight.shape[-2:]
    full = scale.repeat_interleave(block, dim=-2).repeat_interleave(block, dim=-1)
    return (weight * full[..., :out, :inn]).to(torch.float32)


def dequant_fp4_groupwise(weight: torch.Tensor, scale: torch.Tensor, group: int = 32) -> torch.Tensor:
    """``dspark_mlx/loading.py:110-114``: f32 weight times a 1-D (along K) group scale."""
    inn = weight.shape[-1]
    full = scale.repeat_interleave(group, dim=-1)
    return (weight * full[..., :inn]).to(torch.float32)


def fp8_weight_dequant(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """e4m3 codes ``[..., out, in]`` + fp32 128x128 block scales -> fp32 weights."""
    return dequant_fp8_blockwise(e4m3_decode(codes.numpy()), scales.to(torch.float32), 128)


def fp4_weight_dequant(codes: torch.Tensor, gscales: torch.Tensor, tscale: torch.Tensor) -> torch.Tensor:
    """Packed e2m1 codes ``[..., out, in/2]`` + e4m3 group-32 scales + fp32 per-tensor scale.

    ``(code * group_scale)`` is the reference's ``dequant_fp4_groupwise`` (exact in fp32);
    the per-tensor fp32 scale multiplies that product.
    """
    c = codes.to(torch.int64)
    w = torch.stack([e2m1_decode(c & 0xF), e2m1_decode(c >> 4)], dim=-1).reshape(*c.shape[:-1], c.shape[-1] * 2)
    gs = e4m3_decode(gscales.numpy())
    wg = dequant_fp4_groupwise(w, gs, 32)
    ts = tscale.to(torch.float32).reshape(*tscale.shape, 1, 1)
    return (wg * ts).to(torch.float32)


def affine_quantize(w: torch.Tensor, group_size: int = 64, bits: int = 8):
    """Restatement of MLX's affine ``quantize`` (per group of ``group_size`` along the last dim).

    Per group: ``scale = max((max - min) / (2**bits - 1), 1e-7)``, signed towards the edge
    of larger magnitude; the edge value is snapped so that it is exactly representable
    (``scale = edge / round(edge / scale)``), ``bias = edge`` (0 if the edge rounds to 0);
    ``q = clip(round((w - bias) / scale), 0, 2**bits - 1)``. Arithmetic in fp32; scales and
    biases are stored in the weight dtype. ``round`` is round-half-to-even.
    Returns ``(codes uint8 [..., K*bits/8], scales, biases)``.
    """
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    shape = w.shape
    K = shape[-1]
    if K % group_size:
        raise ValueError("last dim must be a multiple of group_size")
    wf = w.to(torch.float32).reshape(-1, K // group_size, group_size)
    n_bins = float((1 << bits) - 1)
    w_max = wf.amax(dim=-1, keepdim=True)
    w_min = wf.amin(dim=-1, keepdim=True)
    mask = w_min.abs() > w_max.abs()
    scale = torch.clamp((w_max - w_min) / n_bins, min=1e-7)
    scale = torch.where(mask, scale, -scale)
    edge = torch.where(mask, w_min, w_max)
    q0 = torch.round(edge / scale)
    scale = torch.where(q0 != 0, edge / q0, scale)
    bias = torch.where(q0 == 0, torch.zeros_like(edge), edge)
    q = torch.clamp(torch.round((wf - bias) / scale), 0, n_bins).to(torch.uint8)
    q = q.reshape(*shape[:-1], K)
    if bits == 8:
        codes = q
    else:
        codes = (q[..., 0::2] | (q[..., 1::2] << 4)).to(torch.uint8)
    scales = scale.reshape(*shape[:-1], K // group_size).to(w.dtype)
    biases = bias.reshape(*shape[:-1], K // group_size).to(w.dtype)
    return codes, scales, biases


def affine_unpack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Packed affine codes -> integer levels ``[..., K]`` (int32)."""
    c = codes.to(torch.int32)
    if bits == 8:
        return c
    lo = c & 0xF
    hi = (c >> 4) & 0xF
    return torch.stack([lo, hi], dim=-1).reshape(*c.shape[:-1], c.shape[-1] * 2)


def affine_dequantize(codes: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                      group_size: int, bits: int) -> torch.Tensor:
    """``w = q * scale + bias`` per group, in fp32 (the values gather_qmm multiplies by)."""
    q = affine_unpack(codes, bits).to(torch.float32)
    s = scales.to(torch.float32).repeat_interleave(group_size, dim=-1)
    b = biases.to(torch.float32).repeat_interleave(group_size, dim=-1)
    return q * s + b
