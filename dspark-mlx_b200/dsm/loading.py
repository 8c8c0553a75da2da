"""Checkpoint ingestion for the draft layer's FFN: the bundled DeepSeek-V4 ``mtp.*`` tensors
go straight into the packed expert formats, without the fp32 dequantisation the reference's
loader applies.

The reference (``dspark_mlx/loader.py:87-107``) reads only the safetensors shards that hold
``mtp.*`` plus the shared ``embed``/``head`` weights. It maps ``mtp.N.*`` to the drafter's
``blocks.N.*`` (``dspark_mlx/loading.py:49-54``). It stacks the per-expert
``...ffn.experts.{e}.{w1,w2,w3}.weight`` into ``[E, out, in]`` in ascending expert id
(``loading.py:88-100``). Quantised tensors carry a sibling ``.scale`` of block-wise e8m0
powers of two (``loading.py:7-18``):

* routed experts: fp4 (e2m1, two per byte) with a 1-D scale per 32 along K, dequantised as
  ``code * scale`` (``dequant_fp4_groupwise``, ``loading.py:110-114``);
* projections (the shared expert among them): fp8 (e4m3) with a 128x128 scale, dequantised
  as ``code * scale`` (``dequant_fp8_blockwise``, ``loading.py:103-107``).

Here those tensors stay packed:

* fp8 matrices keep their codes. Each e8m0 scale becomes the fp32 power of two it
  denotes, which is exact.
* fp4 experts keep their codes. Each expert matrix's e8m0 group scales ``2^x`` split into
  an fp32 per-expert scale ``2^(xmax-8)`` and e4m3 group scales ``2^(x-xmax+8)``. Every
  power of two from ``2^-9`` to ``2^8`` is an exact e4m3 value, so the dequantised weight
  is unchanged bit for bit whenever an expert's nonzero groups span at most 18 octaves. A
  group whose codes are all zero takes any scale. A nonzero group outside that range is an
  error.

e2m1 pairs are read with element ``2j`` in the low nibble of byte ``j``. That is the OCP
microscaling packing and torch's ``float4_e2m1fn_x2`` layout.
"""

from __future__ import annotations

import json
import os
import re
from typing import Dict, Iterable, List, Mapping, Optional, Set, Tuple

import torch

_MTP_RE = re.compile(r"mtp\.(\d+)\.(.+)$")
_EXPERT_RE = re.compile(r"^(.*)\.experts\.(\d+)\.(w[123])\.weight$")
DRAFT_SHARED: Tuple[str, ...] = ("embed.weight", "head.weight")
E4M3_MIN_EXP, E4M3_MAX_EXP = -9, 8  # the powers of two e4m3 holds exactly


def map_checkpoint_key(key: str) -> Optional[str]:
    """Checkpoint key -> drafter parameter path (``loading.py:49-54``): ``mtp.N.rest`` ->
    ``blocks.N.rest``, ``embed.weight``/``head.weight`` unchanged, anything else (base-model
    keys) ``None``."""
    if key in DRAFT_SHARED:
        return key
    m = _MTP_RE.match(key)
    return f"blocks.{m.group(1)}.{m.group(2)}" if m else None


def draft_shards(weight_map: Mapping[str, str]) -> Tuple[Set[str], List[str]]:
    """The draft's keys and the shards holding them (``loader.py:87-91``)."""
    keep = {k for k in weight_map if k.startswith("mtp.") or k in DRAFT_SHARED}
    return keep, sorted({weight_map[k] for k in keep})


def read_draft_tensors(ckpt_dir: str, device="cpu", keys: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Read the draft tensors of a sharded safetensors checkpoint (``loader.py:94-107``).

    Only the shards listed for the draft's keys in ``model.safetensors.index.json`` are opened,
    and only those keys are read from them, straight onto ``device``. ``keys`` narrows the
    selection further (e.g. to one block's FFN).
    """
    from safetensors import safe_open

    with open(os.path.join(ckpt_dir, "model.safetensors.index.json")) as f:
        weight_map = json.load(f)["weight_map"]
    keep, shards = draft_shards(weight_map)
    if keys is not None:
        want = set(keys)
        keep &= want
        shards = sorted({weight_map[k] for k in keep})
    out: Dict[str, torch.Tensor] = {}
    dev = str(torch.device(device))
    for shard in shards:
        with safe_open(os.path.join(ckpt_dir, shard), framework="pt", device=dev) as f:
            for k in f.keys():
                if k in keep and weight_map.get(k) == shard:
                    out[k] = f.get_tensor(k)
    return out


# ---------------------------------------------------------------------------- scale formats
def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def e8m0_exponents(scale: torch.Tensor) -> torch.Tensor:
    """The unbiased exponents ``x`` of e8m0 scales ``2^x`` as int32.

    Accepts e8m0 bytes (``float8_e8m0fnu`` or ``uint8``, biased by 127; 255 is NaN and
    rejected) or a float tensor already holding powers of two (a host that decoded them).
    """
    if scale.dtype in (torch.float8_e8m0fnu, torch.uint8):
        b = _bytes(scale).to(torch.int32)
        if bool((b == 255).any()):
            raise ValueError("e8m0 scale holds NaN (0xFF)")
        return b - 127
    if not scale.is_floating_point():
        raise ValueError(f"scales must be e8m0 bytes or powers of two, got {scale.dtype}")
    m, e = torch.frexp(scale.to(torch.float32))
    if bool((m != 0.5).any()):
        raise ValueError("float scales must be positive powers of two (an e8m0 scale)")
    return e.to(torch.int32) - 1


def e8m0_to_fp32(scale: torch.Tensor) -> torch.Tensor:
    """e8m0 scales -> the fp32 powers of two they denote, exactly (``2^-127`` is an fp32
    subnormal, the rest are normal numbers)."""
    x = e8m0_exponents(scale)
    bits = torch.where(x >= -126, (x + 127) << 23, torch.full_like(x, 1 << 22))
    return bits.view(torch.float32)


def _e4m3_pow2_codes(g: torch.Tensor) -> torch.Tensor:
    """e4m3 bit patterns of ``2^g`` for ``-9 <= g <= 8``: normal numbers have exponent field
    ``g + 7`` and a zero mantissa; ``2^-7 .. 2^-9`` are the subnormals with mantissa
    ``2^(g+9)`` (value ``mantissa/8 * 2^-6``)."""
    normal = (g + 7) << 3
    sub = torch.ones_like(g) << (g + 9).clamp(min=0)
    return torch.where(g >= -6, normal, sub).to(torch.uint8)


def fp4_scales_from_e8m0(codes: torch.Tensor, scale: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Split e8m0 group-32 scales of packed e2m1 experts into e4m3 group scales and an fp32
    per-expert scale, exactly.

    ``codes`` ``[E, out, in/2]`` (packed e2m1), ``scale`` ``[E, out, in/32]`` e8m0. Returns
    ``(group_scales uint8 e4m3 [E, out, in/32], tensor_scale fp32 [E])``, with
    ``e4m3(group) * tensor == 2^x`` for every group that holds a nonzero code.
    """
    if codes.dim() != 3 or scale.dim() != 3:
        raise ValueError("codes and scales must be [E, out, in/2] and [E, out, in/32]")
    E, R, half = codes.shape
    G = scale.shape[2]
    if half % 16 or tuple(scale.shape) != (E, R, half // 16):
        raise ValueError(f"fp4 scales must be [E, out, in/32] = {(E, R, half // 16)}, got {tuple(scale.shape)}")
    x = e8m0_exponents(scale)
    # a group is nonzero when a byte has a magnitude bit set in either nibble (e2m1 +-0 is 0x0 / 0x8)
    nz = (_bytes(codes).reshape(E, R, G, 16) & 0x77).ne(0).any(dim=-1)
    lowest = torch.iinfo(torch.int32).min
    xmax = torch.where(nz, x, torch.full_like(x, lowest)).reshape(E, -1).max(dim=1).values
    xmax = torch.where(xmax == lowest, torch.zeros_like(xmax), xmax)  # an all-zero expert
    g = x - (xmax - E4M3_MAX_EXP).reshape(E, 1, 1)
    bad = nz & (g < E4M3_MIN_EXP)
    if bool(bad.any()):
        e = int(bad.reshape(E, -1).any(dim=1).nonzero()[0, 0])
        raise ValueError(f"expert {e}: {int(bad[e].sum())} nonzero fp4 groups sit more than "
                         f"{E4M3_MAX_EXP - E4M3_MIN_EXP} octaves below the expert's largest scale; "
                         "their e8m0 scale has no exact e4m3 form")
    if bool((xmax - E4M3_MAX_EXP < -127).any()):
        raise ValueError("fp4 expert scales all below 2^-119: no e8m0-style per-expert scale holds them")
    gs = _e4m3_pow2_codes(g.clamp(min=E4M3_MIN_EXP))  # all-zero groups: any scale is exact
    ts = e8m0_to_fp32((xmax - E4M3_MAX_EXP + 127).to(torch.uint8))
    return gs, ts


# ---------------------------------------------------------------------------- experts
def stack_experts(tensors: Mapping[str, torch.Tensor], prefix: str) -> Dict[str, Tuple[torch.Tensor, Optional[torch.Tensor]]]:
    """Stack ``{prefix}.experts.{e}.w{1,2,3}.weight`` (and their ``.scale``) in ascending
    expert id (``loading.py:88-100``): ``{"w1": (weight [E, ...], scale [E, ...] | None), ...}``."""
    groups: Dict[str, Dict[int, str]] = {}
    for k in tensors:
        m = _EXPERT_RE.match(k)
        if m and m.group(1) == prefix:
            groups.setdefault(m.group(3), {})[int(m.group(2))] = k
    out = {}
    for wk, by_eid in groups.items():
        eids = sorted(by_eid)
        if eids != list(range(len(eids))):
            raise ValueError(f"{prefix}.experts.*.{wk}: expert ids are not 0..{len(eids) - 1}")
        skeys = [by_eid[e][: -len("weight")] + "scale" for e in eids]
        have = [s in tensors for s in skeys]
        if any(have) and not all(have):
            raise ValueError(f"{prefix}.experts.*.{wk}: some experts have a .scale and some do not")
        parts = [[tensors[by_eid[e]] for e in eids]] + ([[tensors[s] for s in skeys]] if all(have) else [])
        for ts in parts:
            if any(t.shape != ts[0].shape or t.dtype != ts[0].dtype for t in ts):
                raise ValueError(f"{prefix}.experts.*.{wk}: experts differ in shape or dtype")
        out[wk] = (_stack(parts[0]), _stack(parts[1]) if all(have) else None)
    return out


def _stack(ts: List[torch.Tensor]) -> torch.Tensor:
    """``torch.stack`` that also takes the one-byte float formats (stacked as their bytes)."""
    dt = ts[0].dtype
    if ts[0].element_size() == 1 and dt not in (torch.uint8, torch.int8):
        return torch.stack([t.view(torch.uint8) for t in ts]).view(dt)
    return torch.stack(ts)


def _matrix_kind(w: torch.Tensor, scale: Optional[torch.Tensor], out_dim: int, in_dim: int, what: str) -> str:
    """``"dense"``, ``"fp8"`` or ``"fp4"`` from a ``[..., out, cols]`` weight and its scale."""
    rows, cols = w.shape[-2:]
    if scale is None:
        if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            raise ValueError(f"{what}: {w.dtype} weights need a .scale")
        kind = "dense"
    elif w.dtype == torch.float4_e2m1fn_x2 or (w.element_size() == 1 and w.dtype != torch.float8_e4m3fn
                                                and scale.shape[-2] == rows and cols * 2 == in_dim):
        kind = "fp4"
        cols *= 2
    elif w.element_size() == 1:
        kind = "fp8"
        want = (-(-rows // 128), -(-cols // 128))
        if tuple(scale.shape[-2:]) != want:
            raise ValueError(f"{what}: fp8 scales must be {want} blocks of 128x128, got {tuple(scale.shape[-2:])}")
    else:
        raise ValueError(f"{what}: cannot tell the format of {w.dtype} weights with a .scale")
    if (rows, cols) != (out_dim, in_dim):
        raise ValueError(f"{what}: expected [{out_dim}, {in_dim}], got [{rows}, {cols}] ({kind})")
    return kind


def load_moe(moe, tensors: Mapping[str, torch.Tensor], prefix: str) -> List[str]:
    """Assign one MoE's checkpoint tensors (keys ``{prefix}.gate.*``, ``{prefix}.experts.*``,
    ``{prefix}.shared_experts.*``, e.g. ``prefix="mtp.0.ffn"``) into a :class:`dsm.MoE`.

    fp4 routed experts go to :meth:`MoE.load_fp4_experts`, fp8 ones to
    :meth:`MoE.load_fp8_experts`, bf16/fp32 ones to the stacked dense ``w1``/``w3``/``w2``;
    an fp8 shared expert to :meth:`Expert.load_fp8`. Tensors stay on their device. Returns
    the keys consumed.
    """
    used: List[str] = []

    def take(key: str) -> torch.Tensor:
        used.append(key)
        return tensors[key]

    g = moe.gate
    with torch.no_grad():
        g.weight = take(f"{prefix}.gate.weight").to(torch.float32)
        if g.hash:
            g.tid2eid = take(f"{prefix}.gate.tid2eid").to(torch.int32)
        elif f"{prefix}.gate.bias" in tensors:
            g.bias = take(f"{prefix}.gate.bias").to(torch.float32)

    stacks = stack_experts(tensors, prefix)
    if set(stacks) != {"w1", "w2", "w3"}:
        raise ValueError(f"{prefix}.experts: need w1, w2 and w3, found {sorted(stacks)}")
    E, dim, inter = moe.n_routed_experts, moe.dim, moe.inter_dim
    shapes = {"w1": (inter, dim), "w3": (inter, dim), "w2": (dim, inter)}
    kinds = set()
    for wk, (w, s) in stacks.items():
        if w.shape[0] != E:
            raise ValueError(f"{prefix}.experts.*.{wk}: {w.shape[0]} experts, the MoE has {E}")
        kinds.add(_matrix_kind(w, s, *shapes[wk], what=f"{prefix}.experts.*.{wk}"))
    if len(kinds) != 1:
        raise ValueError(f"{prefix}.experts: mixed formats {sorted(kinds)}")
    kind = kinds.pop()
    for k in tensors:
        m = _EXPERT_RE.match(k[: -len("scale")] + "weight") if k.endswith(".scale") else _EXPERT_RE.match(k)
        if m and m.group(1) == prefix:
            used.append(k)
    if kind == "fp4":
        mats = {}
        for wk, (w, s) in stacks.items():
            codes = _bytes(w)
            gs, ts = fp4_scales_from_e8m0(codes, s)
            mats[wk] = (codes, gs, ts)
        moe.load_fp4_experts(**mats)
    elif kind == "fp8":
        moe.load_fp8_experts(**{wk: (_bytes(w), e8m0_to_fp32(s)) for wk, (w, s) in stacks.items()})
    else:
        moe._drop_routed()
        for wk, (w, _) in stacks.items():
            moe.register_buffer(wk, w)
        moe.quant = None
        moe.expert_format = "dense"

    sh = moe.shared_experts
    sk = {wk: f"{prefix}.shared_experts.{wk}" for wk in ("w1", "w2", "w3")}
    if any(f"{v}.weight" in tensors for v in sk.values()):
        sshapes = {wk: tuple(getattr(sh, wk).weight.shape) for wk in sk}
        mats, skinds = {}, set()
        for wk, base in sk.items():
            w = take(f"{base}.weight")
            s = take(f"{base}.scale") if f"{base}.scale" in tensors else None
            skinds.add(_matrix_kind(w, s, *sshapes[wk], what=f"{base}"))
            mats[wk] = (w, s)
        if skinds == {"fp8"}:
            sh.load_fp8(**{wk: (_bytes(w), e8m0_to_fp32(s)) for wk, (w, s) in mats.items()})
        elif skinds == {"dense"}:
            for wk, (w, _) in mats.items():
                getattr(sh, wk).weight = torch.nn.Parameter(w, requires_grad=False)
            sh._cache = None
        else:
            raise ValueError(f"{prefix}.shared_experts: unsupported formats {sorted(skinds)}")
    return used


def load_ffn_sublayer(ffn, tensors: Mapping[str, torch.Tensor], prefix: str) -> List[str]:
    """Assign a draft block's FFN half (``prefix`` = ``"mtp.N"`` or ``"blocks.N"``) into a
    :class:`dsm.block.DSparkFFN`: ``hc_ffn_fn``/``hc_ffn_base``/``hc_ffn_scale``,
    ``ffn_norm.weight`` and the MoE under ``{prefix}.ffn``. Returns the keys consumed."""
    used = []
    with torch.no_grad():
        for name in ("hc_ffn_fn", "hc_ffn_base", "hc_ffn_scale"):
            key = f"{prefix}.{name}"
            p = getattr(ffn, name)
            t = tensors[key]
            if tuple(t.shape) != tuple(p.shape):
                raise ValueError(f"{key}: expected {tuple(p.shape)}, got {tuple(t.shape)}")
            setattr(ffn, name, torch.nn.Parameter(t.to(torch.float32), requires_grad=False))
            used.append(key)
        key = f"{prefix}.ffn_norm.weight"
        ffn.ffn_norm.weight = torch.nn.Parameter(tensors[key].to(torch.float32), requires_grad=False)
        used.append(key)
    return used + load_moe(ffn.ffn, tensors, f"{prefix}.ffn")
