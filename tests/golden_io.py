"""Read the golden MoE fixtures (``tests/golden/*.npz``) into torch tensors.

Each fixture holds the inputs of one MoE call (activations, ids, router parameters, the
routed expert weights in their storage format, the shared expert) and the outputs the
reference's own ``moe.py`` produced for them (layer output, routing weights and indices).
"""

from __future__ import annotations

import ast
import glob
import os
from dataclasses import dataclass
from typing import Dict, Optional

import numpy as np
import torch

from oracle import OracleWeights

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16)


@dataclass
class GoldenCase:
    name: str
    args: Dict
    layer_id: int
    x: torch.Tensor
    ids: torch.Tensor
    gate_weight: torch.Tensor
    gate_bias: Optional[torch.Tensor]
    tid2eid: Optional[torch.Tensor]
    wfmt: str
    raw: Dict[str, np.ndarray]
    weights: Dict[str, OracleWeights]
    shared: Dict[str, torch.Tensor]
    y: torch.Tensor
    route_weights: torch.Tensor
    route_indices: torch.Tensor


def names():
    """The MoE golden cases (the hyper-connection ``hc_*``, draft-head ``head_*`` and
    draft-attention ``attn_*`` / ``qwen3_attn_*``, draft-layer ``qwen3_layer_*`` /
    ``qwen3_backbone_*`` and draft-block ``block_*`` fixtures have their own loaders)."""
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith(("hc_", "head_", "attn_", "qwen3_attn_", "qwen3_layer_", "qwen3_backbone_", "block_")))


def load(name: str) -> GoldenCase:
    z = dict(np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")))
    args = ast.literal_eval(str(z["args"]))
    xdt = str(z["x_dtype"])
    x = _bf16(z["x"]) if xdt == "bf16" else torch.from_numpy(z["x"])
    sdt = str(z["shared_dtype"])
    shared = {n: (_bf16(z["shared_" + n]) if sdt == "bf16" else torch.from_numpy(z["shared_" + n]))
              for n in ("w1", "w2", "w3")}
    weights = {}
    if "w1_bf16" in z:
        wfmt = "bf16"
        for n in ("w1", "w2", "w3"):
            weights[n] = OracleWeights("dense", _bf16(z[n + "_bf16"]))
    elif "w1_f32" in z:
        wfmt = "f32"
        for n in ("w1", "w2", "w3"):
            weights[n] = OracleWeights("dense", torch.from_numpy(z[n + "_f32"]))
    elif "w1_tscale" in z:
        wfmt = "fp4"
        for n in ("w1", "w2", "w3"):
            weights[n] = OracleWeights("fp4", torch.from_numpy(z[n + "_codes"]),
                                       scales=torch.from_numpy(z[n + "_scales"]),
                                       tscale=torch.from_numpy(z[n + "_tscale"]))
    elif "w1_biases" in z:
        bits = int(z["bits"])
        wfmt = f"affine{bits}"
        for n in ("w1", "w2", "w3"):
            weights[n] = OracleWeights("affine", torch.from_numpy(z[n + "_codes"]),
                                       scales=_bf16(z[n + "_scales"]), biases=_bf16(z[n + "_biases"]),
                                       group_size=64, bits=bits)
    else:
        wfmt = "fp8"
        for n in ("w1", "w2", "w3"):
            weights[n] = OracleWeights("fp8", torch.from_numpy(z[n + "_codes"]),
                                       scales=torch.from_numpy(z[n + "_scales"]))
    y = _bf16(z["y"]) if xdt == "bf16" else torch.from_numpy(z["y"])
    return GoldenCase(
        name=name, args=args, layer_id=int(z["layer_id"]), x=x, ids=torch.from_numpy(z["ids"]),
        gate_weight=torch.from_numpy(z["gate_weight"]),
        gate_bias=torch.from_numpy(z["gate_bias"]) if "gate_bias" in z else None,
        tid2eid=torch.from_numpy(z["tid2eid"]) if "tid2eid" in z else None,
        wfmt=wfmt, raw=z, weights=weights, shared=shared, y=y,
        route_weights=torch.from_numpy(z["route_weights"]),
        route_indices=torch.from_numpy(z["route_indices"]),
    )


def oracle_forward(c: GoldenCase):
    """Run the oracle on a golden case; returns ``(y, weights, indices)``."""
    import oracle

    a = c.args
    return oracle.moe_forward(
        c.x, c.ids, gate_weight=c.gate_weight, topk=a["n_activated_experts"],
        score_func=a["score_func"], route_scale=a["route_scale"], swiglu_limit=a["swiglu_limit"],
        w1=c.weights["w1"], w3=c.weights["w3"], w2=c.weights["w2"],
        shared=(c.shared["w1"], c.shared["w2"], c.shared["w3"]),
        gate_bias=c.gate_bias, tid2eid=c.tid2eid, return_routing=True)


def max_rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    """``max|out - ref| / max|ref|`` -- the reference's own closeness measure."""
    o, r = out.to(torch.float32), ref.to(torch.float32)
    return float((o - r).abs().max() / r.abs().max().clamp_min(1e-12))
