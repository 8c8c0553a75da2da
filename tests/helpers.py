"""Shared test helpers: workload tensors -> oracle weights, small MoE cases, tolerances."""

from __future__ import annotations

import torch

import oracle
from dsm import workloads as W

# MoE output tolerance: max|out - ref| / max|ref| (the reference's own closeness measure,
# tests/test_moe_gather_mm.py:69-79) -- 1e-2 for bf16 outputs.
MOE_TOL = 1e-2


class _PerExpertCPU(oracle.OracleWeights):
    """Oracle weights whose stacks may live on the GPU: each expert is copied to the CPU
    only when the oracle asks for it (the oracle itself always computes on the CPU)."""

    def matrix(self, e: int) -> torch.Tensor:
        cpu = oracle.OracleWeights(self.kind, self.data[e:e + 1].cpu(),
                                   None if self.scales is None else self.scales[e:e + 1].cpu(),
                                   None if self.biases is None else self.biases[e:e + 1].cpu(),
                                   None if self.tscale is None else self.tscale[e:e + 1].cpu(),
                                   self.group_size, self.bits)
        return cpu.matrix(0)


def oracle_weights(wl: W.Workload, t: dict):
    ws = {}
    for n in ("w1", "w3", "w2"):
        if wl.wfmt == "bf16":
            ws[n] = _PerExpertCPU("dense", t[n])
        elif wl.wfmt == "fp8":
            ws[n] = _PerExpertCPU("fp8", t[n + "_codes"], scales=t[n + "_scale"])
        elif wl.wfmt == "fp4":
            ws[n] = _PerExpertCPU("fp4", t[n + "_codes"], scales=t[n + "_scale"], tscale=t[n + "_tensor_scale"])
    return ws


def oracle_moe(wl: W.Workload, t: dict, tokens=None):
    """Oracle forward for workload tensors (optionally only rows ``tokens`` of x)."""
    a = t["args"]
    x = t["x"].cpu()
    ids = t.get("input_ids")
    ids = ids.cpu() if ids is not None else None
    if tokens is not None:
        x = x[tokens]
        ids = ids[tokens] if ids is not None else None
    ws = oracle_weights(wl, t)
    shared = (t["shared_w1"].cpu(), t["shared_w2"].cpu(), t["shared_w3"].cpu())
    return oracle.moe_forward(
        x, ids, gate_weight=t["gate_weight"].cpu(), topk=a["n_activated_experts"], score_func=a["score_func"],
        route_scale=a["route_scale"], swiglu_limit=a["swiglu_limit"], w1=ws["w1"], w3=ws["w3"], w2=ws["w2"],
        shared=shared, gate_bias=t["gate_bias"].cpu() if "gate_bias" in t else None,
        tid2eid=t["tid2eid"].cpu() if "tid2eid" in t else None, return_routing=True)


def max_rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.detach().float().cpu(), ref.detach().float().cpu()
    return float((o - r).abs().max() / r.abs().max().clamp_min(1e-12))


def small_workload(base: str, *, dim=512, inter=256, experts=16, topk=4, n_tokens=24, seed=3, **over):
    wl = W.WORKLOADS[base]
    args = dict(wl.args, dim=dim, moe_inter_dim=inter, n_routed_experts=experts, n_activated_experts=topk)
    args.update(over.pop("args", {}))
    return W.Workload(f"{base}_small", args, n_tokens=n_tokens, wfmt=over.pop("wfmt", wl.wfmt),
                      layer_id=wl.layer_id, zipf_alpha=over.pop("zipf_alpha", wl.zipf_alpha), seed=seed, **over)
