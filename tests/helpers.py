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


def check_routing(idx_gpu: torch.Tensor, x: torch.Tensor, gate_weight: torch.Tensor, gate_bias: torch.Tensor,
                  topk: int, score_func: str, route_scale: float, tie_eps: float = 1e-6):
    """Routing indices of the GPU against the oracle's, with the near-tie rule.

    A token whose top-(k+1) biased scores hold two neighbours within ``tie_eps`` of each
    other may legitimately order them differently (the last bit of the activation function
    decides). Such tokens are counted and must be rare (< 1%); for them the GPU's set of
    experts must still lie within the oracle's top-(k+1) and hold its top-(k-1) whenever the
    only near tie is the k-th/(k+1)-th. Every other token must match bit for bit, slot order
    included. Returns ``(clear mask, oracle indices, number of near-tie tokens)``."""
    x, gw, gb = x.cpu(), gate_weight.cpu(), gate_bias.cpu()
    _, ref_idx = oracle.gate_forward(x, gw, topk=topk, score_func=score_func, route_scale=route_scale, bias=gb)
    scores = oracle.moe_oracle._scores(x, gw, score_func) + gb.to(torch.float32)
    top = torch.topk(scores.to(torch.float64), topk + 1, dim=-1)
    gaps = top.values[:, :-1] - top.values[:, 1:]  # neighbours in descending order
    clear = gaps.min(dim=-1).values > tie_eps
    got = idx_gpu.cpu().to(torch.int64)
    assert torch.equal(got[clear], ref_idx[clear].to(torch.int64)), "routing indices differ on clear tokens"
    n_ties = int((~clear).sum())
    for t in torch.nonzero(~clear).flatten().tolist():
        allowed = set(top.indices[t].tolist())
        assert set(got[t].tolist()) <= allowed, f"token {t}: an expert outside the oracle's top-{topk + 1}"
        if float(gaps[t, :-1].min()) > tie_eps:  # only the k-th / (k+1)-th are near
            assert set(top.indices[t, :topk - 1].tolist()) <= set(got[t].tolist()), f"token {t}: top-(k-1) lost"
    assert n_ties < max(1, 0.01 * got.shape[0]), f"{n_ties} near-tie tokens of {got.shape[0]}"
    return clear, ref_idx, n_ties
