"""Seeded synthetic MoE workloads (the shapes the DSpark draft MoE is measured on).

No dataset is involved: every tensor is drawn from a seeded ``torch.Generator``.

* ``tiny_hash``    hidden 256, 16 routed + 1 shared expert, top-2 hash routing over a
                   1024-token vocabulary (seeded map, 2 distinct experts per id), expert
                   inter 128, bf16 weights N(0, 0.02), x N(0, 1) [7, 256].
* ``fp8_decode``   hidden 4096, 256 experts, top-6 sigmoid + bias N(0, 0.02), route scale
                   2.5, inter 2048; e4m3 codes of N(0, 1) draws with fp32 128x128 block
                   scales log-uniform in [2^-10, 2^-4]; bf16 shared expert N(0, 0.02);
                   x bf16 N(0, 1) [56, 4096] (8 sequences x 7 draft tokens).
* ``fp4_decode``   as fp8_decode with e2m1 codes (uniform over the 16 codes), e4m3 group-32
                   scales 2^U(-3, 3) and an fp32 per-expert scale 2^U(-9, -7); 448 tokens
                   (64 x 7); Zipf(1.1) routing skew.
* ``qwen3_mlp_q8`` the Qwen3-4B-shaped dense draft layer's MLP: hidden 2560, inter 9728,
                   bf16 weights N(0, 0.02) quantised to MLX affine 8-bit group 64 (bf16
                   scale and bias), x bf16 N(0, 1) [112, 2560] (16 sequences x 7), no clamp.
* ``prefill_fp8``  16384 tokens, 256 experts, top-8, fp8 experts, Zipf(1.2) skew.

Zipf skew: expert ``e`` with popularity rank ``r_e`` (a seeded permutation) gets a selection
offset ``-alpha * beta * ln(r_e)`` added to its gate bias. With Gumbel-like score noise of
scale ``beta`` the top-1 choice frequency would fall off as ``r^-alpha``; top-k selection
competes in the saturated upper tail of the sigmoid scores, where the noise is a few
hundredths, and ``beta = 0.05`` gives the prefill case its stated shape (16384 tokens x top-8:
the busiest experts take over 4000 tokens, a dozen take none, the median ~200). The bias
steers selection only, as in the reference gate (``dspark_mlx/model/moe.py:74-75``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import torch

ZIPF_BETA = 0.05


@dataclass
class Workload:
    name: str
    args: Dict
    n_tokens: int
    wfmt: str  # "bf16" | "fp8" | "fp4" | "affine8"
    layer_id: int = 0
    zipf_alpha: Optional[float] = None
    seed: int = 0
    batch: int = 1
    block: int = 7
    notes: str = ""
    extra: Dict = field(default_factory=dict)


def _args(**kw):
    base = dict(n_shared_experts=1, swiglu_limit=10.0, n_hash_layers=0)
    base.update(kw)
    return base


WORKLOADS = {
    "tiny_hash": Workload(
        "tiny_hash", _args(vocab_size=1024, dim=256, moe_inter_dim=128, n_routed_experts=16, n_activated_experts=2,
                           n_hash_layers=1, score_func="sqrtsoftplus", route_scale=1.5),
        n_tokens=7, wfmt="bf16", layer_id=0, batch=1),
    "fp8_decode": Workload(
        "fp8_decode", _args(vocab_size=129280, dim=4096, moe_inter_dim=2048, n_routed_experts=256,
                            n_activated_experts=6, score_func="sigmoid", route_scale=2.5),
        n_tokens=56, wfmt="fp8", batch=8),
    "fp4_decode": Workload(
        "fp4_decode", _args(vocab_size=129280, dim=4096, moe_inter_dim=2048, n_routed_experts=256,
                            n_activated_experts=6, score_func="sigmoid", route_scale=2.5),
        n_tokens=448, wfmt="fp4", zipf_alpha=1.1, batch=64),
    "qwen3_mlp_q8": Workload(
        "qwen3_mlp_q8", dict(hidden_size=2560, intermediate_size=9728), n_tokens=112, wfmt="affine8", batch=16),
    "prefill_fp8": Workload(
        "prefill_fp8", _args(vocab_size=129280, dim=4096, moe_inter_dim=2048, n_routed_experts=256,
                             n_activated_experts=8, score_func="sigmoid", route_scale=2.5),
        n_tokens=16384, wfmt="fp8", zipf_alpha=1.2, batch=1, block=16384),
    # the draft head of the last block: hc_head + norm, LM head over the DeepSeek-V4
    # vocabulary, Markov-biased walk over a 7-token block for 8 sequences
    "draft_head": Workload(
        "draft_head", dict(vocab_size=129280, dim=4096, hc_mult=4, dspark_markov_rank=256, dspark_block_size=7,
                           temperature=0.0),
        n_tokens=56, wfmt="bf16", batch=8, block=7),
    # the Qwen3-4B draft layer's attention (32 query / 8 KV heads of 128) on its cached path:
    # 16 sequences x a 7-token block over 2048 cached context rows, 8-bit affine projections
    # as quantize_drafter leaves them
    "qwen3_attn_q8": Workload(
        "qwen3_attn_q8", dict(hidden_size=2560, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                              rms_norm_eps=1e-6, rope_theta=1000000.0),
        n_tokens=112, wfmt="affine8", batch=16, block=7, extra={"ctx": 2048}),
    # the whole Qwen3-4B draft layer (norms, the attention above, the 9728-wide MLP) on the
    # cached path, every Linear 8-bit affine as quantize_drafter leaves it
    "qwen3_layer_q8": Workload(
        "qwen3_layer_q8", dict(hidden_size=2560, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                               rms_norm_eps=1e-6, rope_theta=1000000.0, intermediate_size=9728),
        n_tokens=112, wfmt="affine8", batch=16, block=7, extra={"ctx": 2048}),
    # the DeepSeek-V4 draft attention (compress_ratio 0 MLA: 64 heads of 512, q rank 1024,
    # 8 output groups of rank 1024, a 128-slot window) decoding 7-token blocks for 8
    # sequences after a 160-token prefill: the window is full
    "draft_attn_dsv4": Workload(
        "draft_attn_dsv4", dict(dim=4096, n_heads=64, head_dim=512, rope_head_dim=64, q_lora_rank=1024, o_groups=8,
                                o_lora_rank=1024, window_size=128, norm_eps=1e-6, rope_theta=10000.0),
        n_tokens=56, wfmt="bf16", batch=8, block=7, extra={"prefill": 160, "max_seq_len": 4096}),
    # the whole DeepSeek-V4 DSpark draft block, a middle stage: over 4 hyper-connection
    # streams, hc_pre -> attn_norm -> the draft attention above -> hc_post, then hc_pre ->
    # ffn_norm -> the fp8 MoE of the decode workload -> hc_post; 8 sequences x 7-token
    # blocks after a 160-token prefill (full window)
    "draft_block_dsv4": Workload(
        "draft_block_dsv4", _args(vocab_size=129280, dim=4096, moe_inter_dim=2048, n_routed_experts=256,
                                  n_activated_experts=6, score_func="sigmoid", route_scale=2.5, n_heads=64,
                                  head_dim=512, rope_head_dim=64, q_lora_rank=1024, o_groups=8, o_lora_rank=1024,
                                  window_size=128, norm_eps=1e-6, rope_theta=10000.0, hc_mult=4,
                                  hc_sinkhorn_iters=20, hc_eps=1e-6, n_layers=43, n_mtp_layers=3,
                                  dspark_block_size=7),
        n_tokens=56, wfmt="fp8", layer_id=44, batch=8, block=7,
        extra={"prefill": 160, "max_seq_len": 4096, "stage": 1}),
}


def zipf_offsets(n_experts: int, alpha: float, gen: torch.Generator) -> torch.Tensor:
    ranks = torch.randperm(n_experts, generator=gen).to(torch.float64) + 1.0
    return (-alpha * ZIPF_BETA * torch.log(ranks)).to(torch.float32)


def _randn(shape, gen, device, std=1.0, dtype=torch.float32):
    return (torch.randn(shape, generator=gen, device=device) * std).to(dtype)


def e4m3_codes(shape, gen, device) -> torch.Tensor:
    v = torch.randn(shape, generator=gen, device=device).clamp_(-448, 448)
    return v.to(torch.float8_e4m3fn).view(torch.uint8)


def make_moe_tensors(wl: Workload, device="cpu", seed: Optional[int] = None, n_tokens: Optional[int] = None,
                     experts_subset: Optional[int] = None, routed: bool = True) -> Dict[str, torch.Tensor]:
    """All tensors of one MoE call of workload ``wl``, generated on ``device``.

    ``experts_subset`` shrinks the routed expert count (keeping every other shape) for
    tests that must fit a CPU oracle; ``n_tokens`` overrides the token count;
    ``routed=False`` skips the routed expert stacks (see :func:`expert_tensors`).
    """
    a = dict(wl.args)
    if experts_subset:
        a["n_routed_experts"] = experts_subset
    E, dim, inter, k = a["n_routed_experts"], a["dim"], a["moe_inter_dim"], a["n_activated_experts"]
    N = n_tokens or wl.n_tokens
    gen = torch.Generator(device=device)
    gen.manual_seed(wl.seed if seed is None else seed)
    out: Dict[str, torch.Tensor] = {"args": a}
    out["x"] = _randn((N, dim), gen, device, dtype=torch.bfloat16)
    out["gate_weight"] = _randn((E, dim), gen, device, std=0.02)
    if wl.layer_id < a.get("n_hash_layers", 0):
        vocab = a["vocab_size"]
        keys = torch.rand((vocab, E), generator=gen, device=device)
        out["tid2eid"] = keys.argsort(dim=1)[:, :k].to(torch.int32)
        out["input_ids"] = torch.randint(0, vocab, (N,), generator=gen, device=device, dtype=torch.int32)
    else:
        bias = _randn((E,), gen, device, std=0.02)
        if wl.zipf_alpha:
            g2 = torch.Generator(device="cpu")
            g2.manual_seed((wl.seed if seed is None else seed) + 7919)
            bias = bias + zipf_offsets(E, wl.zipf_alpha, g2).to(device)
        out["gate_bias"] = bias
    shapes = {"w1": (E, inter, dim), "w3": (E, inter, dim), "w2": (E, dim, inter)}
    for n, shp in (shapes.items() if routed else ()):
        if wl.wfmt == "bf16":
            out[n] = _randn(shp, gen, device, std=0.02, dtype=torch.bfloat16)
        elif wl.wfmt == "fp8":
            out[n + "_codes"] = e4m3_codes(shp, gen, device)
            sb = (shp[0], -(-shp[1] // 128), -(-shp[2] // 128))
            out[n + "_scale"] = torch.exp2(torch.rand(sb, generator=gen, device=device) * 6.0 - 10.0)
        elif wl.wfmt == "fp4":
            nib = torch.randint(0, 16, shp, generator=gen, device=device, dtype=torch.int32)
            out[n + "_codes"] = (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)
            gsh = (shp[0], shp[1], shp[2] // 32)
            gs = torch.exp2(torch.rand(gsh, generator=gen, device=device) * 6.0 - 3.0)
            out[n + "_scale"] = gs.to(torch.float8_e4m3fn).view(torch.uint8)
            out[n + "_tensor_scale"] = torch.exp2(torch.rand((shp[0],), generator=gen, device=device) * 2.0 - 9.0)
        else:
            raise ValueError(wl.wfmt)
    for n, shp in (("shared_w1", (inter, dim)), ("shared_w2", (dim, inter)), ("shared_w3", (inter, dim))):
        out[n] = _randn(shp, gen, device, std=0.02, dtype=torch.bfloat16)
    return out


def build_moe(wl: Workload, t: Dict[str, torch.Tensor], device="cuda"):
    """A ``dsm.MoE`` holding the tensors of ``make_moe_tensors``."""
    from .config import DSparkArgs
    from .moe import MoE

    args = DSparkArgs.from_dict(t["args"])
    moe = MoE(args, wl.layer_id)
    moe.gate.weight = t["gate_weight"].to(device)
    if "tid2eid" in t:
        moe.gate.tid2eid = t["tid2eid"].to(device)
    else:
        moe.gate.bias = t["gate_bias"].to(device)
    if wl.wfmt == "bf16":
        for n in ("w1", "w3", "w2"):
            setattr(moe, n, t[n].to(device))
    elif wl.wfmt == "fp8":
        moe.load_fp8_experts(**{n: (t[n + "_codes"].to(device), t[n + "_scale"].to(device)) for n in ("w1", "w3", "w2")})
    elif wl.wfmt == "fp4":
        moe.load_fp4_experts(**{n: (t[n + "_codes"].to(device), t[n + "_scale"].to(device),
                                    t[n + "_tensor_scale"].to(device)) for n in ("w1", "w3", "w2")})
    for n in ("w1", "w2", "w3"):
        getattr(moe.shared_experts, n).weight = torch.nn.Parameter(t["shared_" + n].to(device), requires_grad=False)
    return moe.to(device)


def routed_weight_bytes(wl: Workload, counts: torch.Tensor, args: Optional[Dict] = None) -> int:
    """Bytes of routed expert weights a call must read: every expert with a nonzero count."""
    a = args or wl.args
    dim, inter = a["dim"], a["moe_inter_dim"]
    touched = int((counts > 0).sum())
    per = 3 * inter * dim
    if wl.wfmt == "fp8":
        per_b = per + 3 * math.ceil(inter / 128) * math.ceil(dim / 128) * 4
    elif wl.wfmt == "fp4":
        per_b = per // 2 + 3 * inter * dim // 32 + 3 * 4
    elif wl.wfmt == "bf16":
        per_b = per * 2
    else:
        per_b = per + 3 * inter * (dim // 64) * 4
    return touched * per_b


def expert_tensors(wl: Workload, experts, seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Routed expert weights for the listed experts only, stacked in that order, on the CPU.

    Each expert comes from its own generator (seeded by the workload seed and the expert
    id), so any subset can be produced without materialising the whole stack.
    """
    a = wl.args
    dim, inter = a["dim"], a["moe_inter_dim"]
    base = (wl.seed if seed is None else seed) * 1_000_003 + 17
    parts: Dict[str, list] = {}
    for e in experts:
        gen = torch.Generator()
        gen.manual_seed(base + int(e))
        one = Workload(wl.name, dict(a, n_routed_experts=1), n_tokens=1, wfmt=wl.wfmt)
        shapes = {"w1": (1, inter, dim), "w3": (1, inter, dim), "w2": (1, dim, inter)}
        for n, shp in shapes.items():
            if wl.wfmt == "bf16":
                vals = {n: _randn(shp, gen, "cpu", std=0.02, dtype=torch.bfloat16)}
            elif wl.wfmt == "fp8":
                sb = (1, -(-shp[1] // 128), -(-shp[2] // 128))
                vals = {n + "_codes": e4m3_codes(shp, gen, "cpu"),
                        n + "_scale": torch.exp2(torch.rand(sb, generator=gen) * 6.0 - 10.0)}
            else:
                nib = torch.randint(0, 16, shp, generator=gen, dtype=torch.int32)
                gs = torch.exp2(torch.rand((1, shp[1], shp[2] // 32), generator=gen) * 6.0 - 3.0)
                vals = {n + "_codes": (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8),
                        n + "_scale": gs.to(torch.float8_e4m3fn).view(torch.uint8),
                        n + "_tensor_scale": torch.exp2(torch.rand((1,), generator=gen) * 2.0 - 9.0)}
            for k, v in vals.items():
                parts.setdefault(k, []).append(v)
        del one
    return {k: torch.cat(v, 0) for k, v in parts.items()}


def make_qwen3_tensors(wl: Workload, device="cpu", seed: Optional[int] = None,
                       n_tokens: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """x and the three bf16 projection weights of the Qwen3 MLP workload (before quantisation)."""
    h, i = wl.args["hidden_size"], wl.args["intermediate_size"]
    gen = torch.Generator(device=device)
    gen.manual_seed(wl.seed if seed is None else seed)
    out: Dict[str, torch.Tensor] = {"args": dict(wl.args)}
    out["x"] = _randn((n_tokens or wl.n_tokens, h), gen, device, dtype=torch.bfloat16)
    out["gate_proj"] = _randn((i, h), gen, device, std=0.02, dtype=torch.bfloat16)
    out["up_proj"] = _randn((i, h), gen, device, std=0.02, dtype=torch.bfloat16)
    out["down_proj"] = _randn((h, i), gen, device, std=0.02, dtype=torch.bfloat16)
    return out


def build_qwen3_mlp(wl: Workload, t: Dict[str, torch.Tensor], device="cuda", bits: int = 8, group_size: int = 64):
    """A :class:`dsm.qwen3.Qwen3MLP` holding ``t``'s weights, quantised as ``quantize_drafter`` does."""
    from .qwen3 import Qwen3MLP

    mlp = Qwen3MLP(t["args"])
    for n in ("gate_proj", "up_proj", "down_proj"):
        getattr(mlp, n).weight = torch.nn.Parameter(t[n].to(device), requires_grad=False)
    if wl.wfmt == "affine8":
        mlp.quantize(bits=bits, group_size=group_size)
    return mlp


def make_head_tensors(wl: Workload, device="cpu", seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Inputs and bf16 weights of the draft head workload (seeded normal values)."""
    a = wl.args
    g = torch.Generator(device=device)
    g.manual_seed(wl.seed if seed is None else seed)
    b, s, hc, dim, vocab, rank = wl.batch, wl.block, a["hc_mult"], a["dim"], a["vocab_size"], a["dspark_markov_rank"]
    r = lambda *shape, std=1.0: torch.randn(shape, generator=g, device=device) * std  # noqa: E731
    return {"args": a, "x": r(b, s, hc, dim).to(torch.bfloat16), "fn": r(hc, hc * dim, std=0.02), "scale": r(1),
            "base": r(hc, std=0.5), "norm_w": 1 + r(dim, std=0.1), "head_w": r(vocab, dim, std=0.02).to(torch.bfloat16),
            "w1": r(vocab, rank, std=0.2).to(torch.bfloat16), "w2": r(vocab, rank, std=0.2).to(torch.bfloat16),
            "wc": r(1, dim + rank, std=0.02),
            "anchor": torch.randint(0, vocab, (b,), generator=g, device=device, dtype=torch.int32)}


def build_head(wl: Workload, t: Dict[str, torch.Tensor], device="cuda"):
    """A :class:`dsm.head.DSparkHead` holding ``t``'s weights."""
    from .head import DSparkHead

    h = DSparkHead(wl.args).to(device)
    with torch.no_grad():
        h.hc_head_fn.copy_(t["fn"])
        h.hc_head_scale.copy_(t["scale"])
        h.hc_head_base.copy_(t["base"])
        h.norm.weight.copy_(t["norm_w"])
        h.confidence_head.proj.weight.copy_(t["wc"])
    h.markov_head.markov_w1.weight = torch.nn.Parameter(t["w1"].to(device), requires_grad=False)
    h.markov_head.markov_w2.weight = torch.nn.Parameter(t["w2"].to(device), requires_grad=False)
    h.head.weight = torch.nn.Parameter(t["head_w"].to(device), requires_grad=False)
    return h


def make_gqa_tensors(wl: Workload, device="cpu", seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Inputs, cached context K/V (N(0, 1)) and bf16 weights of the Qwen3 attention workload."""
    a = wl.args
    g = torch.Generator(device=device)
    g.manual_seed(wl.seed if seed is None else seed)
    h, nh, nkv, hd = a["hidden_size"], a["num_attention_heads"], a["num_key_value_heads"], a["head_dim"]
    b, s, ctx = wl.batch, wl.block, wl.extra["ctx"]
    r = lambda *shape, std=1.0: torch.randn(shape, generator=g, device=device) * std  # noqa: E731
    return {"q_proj": r(nh * hd, h, std=h ** -0.5).to(torch.bfloat16),
            "k_proj": r(nkv * hd, h, std=h ** -0.5).to(torch.bfloat16),
            "v_proj": r(nkv * hd, h, std=h ** -0.5).to(torch.bfloat16),
            "o_proj": r(h, nh * hd, std=(nh * hd) ** -0.5).to(torch.bfloat16),
            "q_norm": 1 + r(hd, std=0.1), "k_norm": 1 + r(hd, std=0.1),
            "x": r(b, s, h).to(torch.bfloat16),
            "ctx_k": r(b, nkv, ctx, hd).to(torch.bfloat16), "ctx_v": r(b, nkv, ctx, hd).to(torch.bfloat16)}


def make_qwen3_layer_tensors(wl: Workload, device="cpu", seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """The attention workload's tensors plus the MLP's bf16 weights and the two layer norms."""
    t = make_gqa_tensors(wl, device=device, seed=seed)
    a = wl.args
    g = torch.Generator(device=device)
    g.manual_seed((wl.seed if seed is None else seed) + 1)
    h, i = a["hidden_size"], a["intermediate_size"]
    r = lambda *shape, std=1.0: torch.randn(shape, generator=g, device=device) * std  # noqa: E731
    t.update({"gate_proj": r(i, h, std=h ** -0.5).to(torch.bfloat16), "up_proj": r(i, h, std=h ** -0.5).to(torch.bfloat16),
              "down_proj": r(h, i, std=i ** -0.5).to(torch.bfloat16),
              "input_layernorm": 1 + r(h, std=0.1), "post_attention_layernorm": 1 + r(h, std=0.1)})
    return t


def build_qwen3_layer(wl: Workload, t: Dict[str, torch.Tensor], device="cuda", bits: int = 8, group_size: int = 64):
    """A :class:`dsm.qwen3_layer.Qwen3DSparkLayer` holding ``t``'s weights, quantised like
    ``quantize_drafter`` when the workload is affine."""
    from .qwen3_layer import Qwen3DSparkLayer

    layer = Qwen3DSparkLayer(wl.args).to(device)
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(layer.self_attn, n).weight = torch.nn.Parameter(t[n].to(device), requires_grad=False)
    for n in ("gate_proj", "up_proj", "down_proj"):
        getattr(layer.mlp, n).weight = torch.nn.Parameter(t[n].to(device), requires_grad=False)
    with torch.no_grad():
        layer.self_attn.q_norm.weight.copy_(t["q_norm"])
        layer.self_attn.k_norm.weight.copy_(t["k_norm"])
        layer.input_layernorm.weight.copy_(t["input_layernorm"])
        layer.post_attention_layernorm.weight.copy_(t["post_attention_layernorm"])
    if wl.wfmt == "affine8":
        layer.quantize(bits=bits, group_size=group_size)
    return layer


def build_gqa(wl: Workload, t: Dict[str, torch.Tensor], device="cuda", bits: int = 8, group_size: int = 64):
    """A :class:`dsm.qwen3_attention.Qwen3DSparkAttention` holding ``t``'s weights, quantised
    like ``quantize_drafter`` when the workload is affine."""
    from .qwen3_attention import Qwen3DSparkAttention

    attn = Qwen3DSparkAttention(wl.args).to(device)
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(attn, n).weight = torch.nn.Parameter(t[n].to(device), requires_grad=False)
        if wl.wfmt == "affine8":
            getattr(attn, n).quantize(bits=bits, group_size=group_size)
    with torch.no_grad():
        attn.q_norm.weight.copy_(t["q_norm"])
        attn.k_norm.weight.copy_(t["k_norm"])
    return attn


def make_dsattn_tensors(wl: Workload, device="cpu", seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Inputs and bf16 weights of the DeepSeek draft attention workload (seeded normal values)."""
    a = wl.args
    g = torch.Generator(device=device)
    g.manual_seed(wl.seed if seed is None else seed)
    d, h, hd, ql, og, orank = (a[k] for k in ("dim", "n_heads", "head_dim", "q_lora_rank", "o_groups", "o_lora_rank"))
    b, s, pre = wl.batch, wl.block, wl.extra["prefill"]
    r = lambda *shape, std=1.0: torch.randn(shape, generator=g, device=device) * std  # noqa: E731
    bf = torch.bfloat16
    return {"wq_a": r(ql, d, std=d ** -0.5).to(bf), "wq_b": r(h * hd, ql, std=ql ** -0.5).to(bf),
            "wkv": r(hd, d, std=d ** -0.5).to(bf), "wo_a": r(og * orank, h * hd // og, std=(h * hd // og) ** -0.5).to(bf),
            "wo_b": r(d, og * orank, std=(og * orank) ** -0.5).to(bf),
            "q_norm": 1 + r(ql, std=0.1), "kv_norm": 1 + r(hd, std=0.1), "attn_sink": r(h),
            "prefill_main": r(b, pre, d).to(bf), "x": r(b, s, d).to(bf), "main": r(b, 1, d).to(bf)}


def make_block_tensors(wl: Workload, device="cpu", seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Inputs and weights of the whole draft block workload: the draft attention's tensors
    (``attn_*``), the fp8 MoE's (``moe_*``), the hyper-connection mixers (``hc_*``), the two
    norms (``norm_attn``, ``norm_ffn``) and the block input ``x [b, s, hc, dim]``."""
    a = wl.args
    sd = wl.seed if seed is None else seed
    t = {f"attn_{k}": v for k, v in make_dsattn_tensors(wl, device, sd).items()}
    t.update({f"moe_{k}": v for k, v in make_moe_tensors(wl, device, seed=sd + 1).items()})
    g = torch.Generator(device=device)
    g.manual_seed(sd + 2)
    d, hc = a["dim"], a["hc_mult"]
    mix = (2 + hc) * hc
    r = lambda *shape, std=1.0: torch.randn(shape, generator=g, device=device) * std  # noqa: E731
    for half in ("attn", "ffn"):
        t[f"hc_{half}_fn"] = r(mix, hc * d, std=(hc * d) ** -0.5)
        t[f"hc_{half}_base"] = r(mix, std=0.1)
        t[f"hc_{half}_scale"] = 1 + r(3, std=0.1)
        t[f"norm_{half}"] = 1 + r(d, std=0.1)
    t["x"] = r(wl.batch, wl.block, hc, d).to(torch.bfloat16)
    return t


def build_block(wl: Workload, t: Dict[str, torch.Tensor], device="cuda"):
    """A :class:`dsm.draft_block.DSparkBlock` (stage ``wl.extra["stage"]``) holding ``t``'s
    weights; its MoE is the one :func:`build_moe` makes from the ``moe_*`` tensors."""
    from .config import DSparkArgs
    from .draft_block import DSparkBlock

    blk = DSparkBlock(DSparkArgs.from_dict(wl.args), wl.extra["stage"], max_seq_len=wl.extra["max_seq_len"])
    blk = blk.to(device)
    at = {k[5:]: v for k, v in t.items() if k.startswith("attn_")}
    ref = build_dsattn(wl, at, device)
    blk.attn = ref
    blk.ffn = build_moe(wl, {k[4:]: v for k, v in t.items() if k.startswith("moe_")}, device)
    with torch.no_grad():
        for half in ("attn", "ffn"):
            getattr(blk, f"hc_{half}_fn").copy_(t[f"hc_{half}_fn"])
            getattr(blk, f"hc_{half}_base").copy_(t[f"hc_{half}_base"])
            getattr(blk, f"hc_{half}_scale").copy_(t[f"hc_{half}_scale"])
            getattr(blk, f"{half}_norm").weight.copy_(t[f"norm_{half}"])
    return blk


def build_dsattn(wl: Workload, t: Dict[str, torch.Tensor], device="cuda"):
    """A :class:`dsm.attention.DSparkAttention` holding ``t``'s weights."""
    from .attention import DSparkAttention

    attn = DSparkAttention(wl.args, max_seq_len=wl.extra["max_seq_len"]).to(device)
    for n in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b"):
        getattr(attn, n).weight = torch.nn.Parameter(t[n].to(device), requires_grad=False)
    with torch.no_grad():
        attn.q_norm.weight.copy_(t["q_norm"])
        attn.kv_norm.weight.copy_(t["kv_norm"])
        attn.attn_sink.copy_(t["attn_sink"])
    return attn
