"""Synthetic DeepSeek-V4-style draft checkpoints for the loader tests.

The bundled draft stores one MoE per block under ``mtp.{N}.ffn``:

* per-expert routed weights ``experts.{e}.{w1,w2,w3}.weight`` as packed e2m1
  (``float4_e2m1fn_x2``, ``[out, in/2]``) with an e8m0 ``.scale`` per 32 along K;
* an fp8 (e4m3) shared expert with 128x128 e8m0 scales;
* an fp32 gate with a bias (score routing) or a ``tid2eid`` table (hash routing);
* the block's hyper-connection mixes and ``ffn_norm`` beside it.

The layout follows ``dspark_mlx/loading.py:7-18``; the values are seeded random. The
reference-side weights come from the oracle's restatement of the reference's dequant helpers.
"""

from __future__ import annotations

import json
import os
from typing import Dict

import torch

import oracle


def _e8m0(exps: torch.Tensor) -> torch.Tensor:
    return (exps + 127).to(torch.uint8).view(torch.float8_e8m0fnu)


def make_checkpoint(args: Dict, layer_id: int, block: int = 0, experts: str = "fp4", shared: str = "fp8",
                    seed: int = 0, octaves: int = 6) -> Dict[str, torch.Tensor]:
    """Checkpoint tensors of block ``block``'s FFN half (keys ``mtp.{block}.*``).

    ``experts``: ``"fp4"`` | ``"fp8"`` | ``"bf16"``; ``shared``: ``"fp8"`` | ``"bf16"``;
    ``octaves``: spread of the e8m0 scale exponents within one expert matrix.
    """
    g = torch.Generator().manual_seed(seed)
    E, dim, inter, k = args["n_routed_experts"], args["dim"], args["moe_inter_dim"], args["n_activated_experts"]
    hc = args.get("hc_mult", 4)
    p = f"mtp.{block}"
    t: Dict[str, torch.Tensor] = {}
    t[f"{p}.hc_ffn_fn"] = torch.randn((2 + hc) * hc, hc * dim, generator=g) * 0.05
    t[f"{p}.hc_ffn_base"] = torch.randn((2 + hc) * hc, generator=g) * 0.5
    t[f"{p}.hc_ffn_scale"] = torch.randn(3, generator=g)
    t[f"{p}.ffn_norm.weight"] = (1 + 0.1 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    t[f"{p}.ffn.gate.weight"] = (torch.randn(E, dim, generator=g) * 0.02).to(torch.bfloat16)
    if layer_id < args.get("n_hash_layers", 0):
        keys = torch.rand(args["vocab_size"], E, generator=g)
        t[f"{p}.ffn.gate.tid2eid"] = keys.argsort(dim=1)[:, :k].to(torch.int32)
    else:
        t[f"{p}.ffn.gate.bias"] = torch.randn(E, generator=g) * 0.02
    shapes = {"w1": (inter, dim), "w3": (inter, dim), "w2": (dim, inter)}
    for e in range(E):
        for wk, (o, i) in shapes.items():
            key = f"{p}.ffn.experts.{e}.{wk}"
            if experts == "fp4":
                nib = torch.randint(0, 16, (o, i), generator=g, dtype=torch.int32)
                t[key + ".weight"] = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8).view(torch.float4_e2m1fn_x2)
                base = -9 - int(torch.randint(0, 3, (1,), generator=g))
                t[key + ".scale"] = _e8m0(base + torch.randint(0, octaves + 1, (o, i // 32), generator=g))
            elif experts == "fp8":
                t[key + ".weight"] = (torch.randn(o, i, generator=g) * 32).clamp(-448, 448).to(torch.float8_e4m3fn)
                t[key + ".scale"] = _e8m0(-12 + torch.randint(0, 4, (-(-o // 128), -(-i // 128)), generator=g))
            else:
                t[key + ".weight"] = (torch.randn(o, i, generator=g) * 0.02).to(torch.bfloat16)
    for wk, (o, i) in shapes.items():
        key = f"{p}.ffn.shared_experts.{wk}"
        if shared == "fp8":
            t[key + ".weight"] = (torch.randn(o, i, generator=g) * 32).clamp(-448, 448).to(torch.float8_e4m3fn)
            t[key + ".scale"] = _e8m0(-12 + torch.randint(0, 4, (-(-o // 128), -(-i // 128)), generator=g))
        else:
            t[key + ".weight"] = (torch.randn(o, i, generator=g) * 0.02).to(torch.bfloat16)
    return t


def reference_matrix(w: torch.Tensor, scale) -> torch.Tensor:
    """What the reference's loader makes of one checkpoint matrix: the host casts the codes
    to fp32 and ``dequant_fp8_blockwise`` / ``dequant_fp4_groupwise`` apply the e8m0 scale
    (``dspark_mlx/loading.py:103-114``); unscaled weights are cast to fp32."""
    if scale is None:
        return w.to(torch.float32)
    s = oracle.e8m0_decode(scale.view(torch.uint8).numpy())
    if w.dtype == torch.float4_e2m1fn_x2:
        c = w.view(torch.uint8)
        nib = torch.stack([c & 0xF, c >> 4], dim=-1).reshape(c.shape[0], c.shape[1] * 2)
        return oracle.dequant_fp4_groupwise(oracle.e2m1_decode(nib.numpy()), s, 32)
    return oracle.dequant_fp8_blockwise(oracle.e4m3_decode(w.view(torch.uint8).numpy()), s, 128)


def reference_moe_weights(t: Dict[str, torch.Tensor], prefix: str, n_experts: int):
    """Stacked fp32 routed weights and the fp32 shared expert, as the reference holds them."""
    routed = {}
    for wk in ("w1", "w2", "w3"):
        mats = []
        for e in range(n_experts):
            key = f"{prefix}.experts.{e}.{wk}"
            mats.append(reference_matrix(t[key + ".weight"], t.get(key + ".scale")))
        routed[wk] = torch.stack(mats)
    shared = []
    for wk in ("w1", "w2", "w3"):
        key = f"{prefix}.shared_experts.{wk}"
        shared.append(reference_matrix(t[key + ".weight"], t.get(key + ".scale")))
    return routed, tuple(shared)


def write_sharded(t: Dict[str, torch.Tensor], ckpt_dir: str, n_shards: int = 2, base_shard: bool = True) -> None:
    """Write ``t`` as a sharded safetensors checkpoint with its index. With ``base_shard``, a
    base-model shard is listed too; it holds bytes that are not safetensors, so a loader that
    opens it fails."""
    from safetensors.torch import save_file

    os.makedirs(ckpt_dir, exist_ok=True)
    keys = sorted(t)
    weight_map = {}
    for s in range(n_shards):
        name = f"model-{s + 1:05d}-of-{n_shards + base_shard:05d}.safetensors"
        part = {k: t[k].contiguous() for k in keys[s::n_shards]}
        save_file(part, os.path.join(ckpt_dir, name))
        weight_map.update({k: name for k in part})
    if base_shard:
        name = f"model-{n_shards + 1:05d}-of-{n_shards + 1:05d}.safetensors"
        with open(os.path.join(ckpt_dir, name), "wb") as f:
            f.write(b"not a safetensors file: the base model's layers")
        weight_map.update({"layers.0.attn.wq_a.weight": name, "layers.0.ffn.gate.weight": name})
    with open(os.path.join(ckpt_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
