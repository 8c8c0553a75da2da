"""Expert-parallel DSpark MoE: routed experts sharded over the ranks of a process group.

The reference runs the whole MoE on one device (``dspark_mlx/model/moe.py:151-161``; its test
harness forces ``world_size=1``, ``tests/reference_model.py:55-56``). Here rank ``r`` of ``W``
owns experts ``[r*E/W, (r+1)*E/W)``; the router and the shared expert are replicated and every
rank routes its own tokens. One call:

1. route the local tokens, sort the (token, slot) pairs by expert -- expert order is owner
   order, so the sorted pairs are already grouped by destination rank;
2. all-to-all the per-expert counts (equal splits of ``E/W``), and copy them to the host on a
   side stream while the shared expert runs;
3. all-to-all the pair rows (bf16) with those splits; the receiver groups the rows of all
   sources by its local experts (segment ids + a local permutation);
4. grouped gate/up + down on the local experts; the down kernel writes each result row back
   to the position its input row arrived at;
5. all-to-all the fp32 result rows back (reversed splits) and combine them with the routing
   weights and the shared expert, exactly as the single-GPU path does.

The exchanges are NCCL all-to-alls (torch.distributed); the compute is ``libdsm.so``.
"""

from __future__ import annotations

import copy
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
from torch import nn

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_ptr
from .moe import Expert, Gate, MoE, _cuda_contig, _ids_arg


# ---------------------------------------------------------------------------- exchange steps
def rank_expert_range(n_experts: int, world: int, rank: int) -> Tuple[int, int]:
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not shard evenly over {world} ranks")
    el = n_experts // world
    return rank * el, el


def exchange_counts(counts: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """``counts [E]`` (pairs this rank sends to each expert) -> ``[W * E/W]``: row ``s`` holds the
    pairs source ``s`` sends to each of this rank's experts."""
    recv = torch.empty_like(counts)
    if world == 1:
        recv.copy_(counts)
    else:
        dist.all_to_all_single(recv, counts, group=group)
    return recv


def splits(counts: torch.Tensor, world: int) -> List[int]:
    """Rows per rank from per-expert counts laid out rank-major ([W, E/W] or [E])."""
    return counts.view(world, -1).sum(dim=1).tolist()


def exchange_rows(send: torch.Tensor, send_splits: List[int], recv_splits: List[int], world: int,
                  group=None) -> torch.Tensor:
    """Rows grouped by destination rank -> rows grouped by source rank (same order within)."""
    recv = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
    if world == 1:
        recv.copy_(send)
    else:
        dist.all_to_all_single(recv, send, recv_splits, send_splits, group=group)
    return recv


# ---------------------------------------------------------------------------- module
class ExpertParallelMoE(nn.Module):
    """``MoE`` with the routed experts sharded over ``group``; call it like ``MoE``."""

    def __init__(self, args, layer_id: int, group=None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dim, self.inter_dim = args.dim, args.moe_inter_dim
        self.n_routed_experts = args.n_routed_experts
        self.swiglu_limit = args.swiglu_limit
        self.e0, self.e_local = rank_expert_range(args.n_routed_experts, self.world, self.rank)
        self.gate = Gate(args, layer_id)
        self.shared_experts = Expert(args.dim, args.moe_inter_dim, args.swiglu_limit)
        local_args = copy.copy(args)
        local_args.n_routed_experts = self.e_local
        self.local = MoE(local_args, layer_id)  # holds this rank's routed experts (any format)
        del self.local.gate, self.local.shared_experts
        self._side = None
        self._host = None

    @classmethod
    def from_moe(cls, moe: MoE, args, layer_id: int, group=None) -> "ExpertParallelMoE":
        """Shard a full ``MoE``'s routed experts; router and shared expert are copied."""
        ep = cls(args, layer_id, group)
        # share the replicated modules as they are: their dtypes decide the reference's
        # rounding points (bf16 products for bf16 weights), so they must not be re-cast
        ep.gate = moe.gate
        ep.shared_experts = moe.shared_experts
        sl = slice(ep.e0, ep.e0 + ep.e_local)
        f = moe.expert_format
        if f == "dense":
            for n in ("w1", "w3", "w2"):
                setattr(ep.local, n, getattr(moe, n)[sl].contiguous())
        elif f == "fp8":
            ep.local.load_fp8_experts(**{n: (getattr(moe, f"{n}_codes")[sl].contiguous(),
                                             getattr(moe, f"{n}_scale")[sl].contiguous()) for n in ("w1", "w3", "w2")})
        elif f == "fp4":
            ep.local.load_fp4_experts(**{n: (getattr(moe, f"{n}_codes")[sl].contiguous(),
                                             getattr(moe, f"{n}_scale")[sl].contiguous(),
                                             getattr(moe, f"{n}_tensor_scale")[sl].contiguous())
                                         for n in ("w1", "w3", "w2")})
        else:
            ep.local._drop_routed()
            for n in ("w1", "w3", "w2"):
                for s in ("q", "scales", "biases"):
                    ep.local.register_buffer(f"{n}_{s}", getattr(moe, f"{n}_{s}")[sl].contiguous())
            ep.local.quant = moe.quant
            ep.local.expert_format = "affine"
        return ep.to(moe.gate.weight.device)

    def _shared(self, x2: torch.Tensor, sgu: int, so: int, hsc: float, s: int) -> torch.Tensor:
        L = lib()
        n, dim = x2.shape
        p1, p3, p2 = self.shared_experts.packed()
        cap = L.dsm_stage_rows_cap(n)
        dev = x2.device
        xs = torch.empty(L.dsm_stage_bytes(cap, dim), dtype=torch.uint8, device=dev)
        xsc = torch.empty(cap, dtype=torch.float32, device=dev)
        hs = torch.empty(L.dsm_stage_bytes(cap, p1.rows), dtype=torch.uint8, device=dev)
        o = torch.empty(n, dim, dtype=torch.float32, device=dev)
        check(L.dsm_stage_rows(ptr(x2), dtype_code(x2.dtype), n, dim, None, n, 1, ptr(xs), cap, ptr(xsc), s),
              "dsm_stage_rows")
        check(L.dsm_expert_gate_up(ptr(xs), ptr(xsc), cap, dim, None, 1, p1.wfmt, p1.group_size, ptr(p1.packed),
                                   ptr(p3.packed), p1.rows, _lib.ACT_SWIGLU_CLAMP, float(self.swiglu_limit), sgu,
                                   ptr(hs), hsc, n, s), "dsm_expert_gate_up")
        check(L.dsm_expert_down(ptr(hs), hsc, cap, p2.cols, None, 1, p2.wfmt, p2.group_size, ptr(p2.packed), dim, so,
                                ptr(o), dim, None, n, s), "dsm_expert_down")
        return o

    def forward(self, x: torch.Tensor, input_ids: Optional[torch.Tensor] = None, *, return_routing: bool = False):
        L = lib()
        shape, in_dtype = x.shape, x.dtype
        x2 = _cuda_contig(x.reshape(-1, self.dim), "x")
        n, dim = x2.shape
        dev = x2.device
        E, El, W, k = self.n_routed_experts, self.e_local, self.world, self.gate.topk
        P = n * k
        s = stream_ptr()
        # 1. route and sort the pairs by (global) expert
        w, idx = self.gate(x2, input_ids)
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        perm = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        inv = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        pws = torch.empty(max(1, L.dsm_permute_workspace_bytes(P, E)), dtype=torch.uint8, device=dev)
        check(L.dsm_permute(ptr(idx), P, E, ptr(counts), ptr(offsets), ptr(perm), ptr(inv), ptr(pws), pws.numel(),
                            s), "dsm_permute")
        x_send = torch.empty(P, dim, dtype=x2.dtype, device=dev)
        check(L.dsm_gather_rows(ptr(x2), dtype_code(x2.dtype), n, dim, ptr(perm), P, k, ptr(x_send), s),
              "dsm_gather_rows")
        # 2. counts to the expert owners; to the host on a side stream while the shared expert runs
        recv_counts = exchange_counts(counts, W, self.group)
        if self._side is None:
            self._side = torch.cuda.Stream(device=dev)
            self._host = torch.empty(2 * E, dtype=torch.int32).pin_memory()
        main = torch.cuda.current_stream(dev)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            self._host[:E].copy_(counts, non_blocking=True)
            self._host[E:].copy_(recv_counts, non_blocking=True)
        rgu, ro = self.local.routed_round_flags(x2.dtype)
        if x2.dtype == torch.bfloat16:
            sgu = int(self.shared_experts.weight_dtype("w1") == torch.bfloat16) | 2
            so = int(self.shared_experts.weight_dtype("w2") == torch.bfloat16)
        else:
            sgu, so = 0, 0
        hsc = 1.0 if 0 < self.swiglu_limit and self.swiglu_limit ** 2 < 30000 else 1.0 / 256
        o_shared = self._shared(x2, sgu, so, hsc, s)
        self._side.synchronize()
        host = self._host.clone()
        send_splits = splits(host[:E], W)
        recv_splits = splits(host[E:], W)
        # 3. rows to the owners; group all sources' rows by local expert
        x_recv = exchange_rows(x_send, send_splits, recv_splits, W, self.group)
        R = x_recv.shape[0]
        o_recv = torch.empty(max(R, 1), dim, dtype=torch.float32, device=dev)
        if R:
            seg = torch.empty(R, dtype=torch.int32, device=dev)
            check(L.dsm_segment_ids(ptr(recv_counts), W * El, El, ptr(seg), R, s), "dsm_segment_ids")
            lc = torch.empty(El, dtype=torch.int32, device=dev)
            lo = torch.empty(El + 1, dtype=torch.int32, device=dev)
            lperm = torch.empty(R, dtype=torch.int32, device=dev)
            linv = torch.empty(R, dtype=torch.int32, device=dev)
            lws = torch.empty(max(1, L.dsm_permute_workspace_bytes(R, El)), dtype=torch.uint8, device=dev)
            check(L.dsm_permute(ptr(seg), R, El, ptr(lc), ptr(lo), ptr(lperm), ptr(linv), ptr(lws), lws.numel(), s),
                  "dsm_permute")
            # 4. local grouped expert products; results land in arrival order
            p1, p3, p2 = self.local.packed_experts()
            cap = L.dsm_stage_rows_cap(R)
            xs = torch.empty(L.dsm_stage_bytes(cap, dim), dtype=torch.uint8, device=dev)
            xsc = torch.empty(cap, dtype=torch.float32, device=dev)
            hs = torch.empty(L.dsm_stage_bytes(cap, self.inter_dim), dtype=torch.uint8, device=dev)
            check(L.dsm_stage_rows(ptr(x_recv), dtype_code(x_recv.dtype), R, dim, ptr(lperm), R, 1, ptr(xs), cap,
                                   ptr(xsc), s), "dsm_stage_rows")
            check(L.dsm_expert_gate_up(ptr(xs), ptr(xsc), cap, dim, ptr(lo), El, p1.wfmt, p1.group_size,
                                       ptr(p1.packed), ptr(p3.packed), self.inter_dim, _lib.ACT_SWIGLU_CLAMP,
                                       float(self.swiglu_limit), rgu, ptr(hs), hsc, R, s), "dsm_expert_gate_up")
            check(L.dsm_expert_down(ptr(hs), hsc, cap, self.inter_dim, ptr(lo), El, p2.wfmt, p2.group_size,
                                    ptr(p2.packed), dim, ro, ptr(o_recv), dim, ptr(lperm), R, s), "dsm_expert_down")
        # 5. results back to the token owners (in the order the rows were sent), combine
        o_back = exchange_rows(o_recv[:R], recv_splits, send_splits, W, self.group)
        y = torch.empty_like(x2)
        check(L.dsm_combine(ptr(o_back), ptr(inv), ptr(w), n, k, dim, ptr(o_shared), ptr(y), dtype_code(x2.dtype), s),
              "dsm_combine")
        y = y.to(in_dtype).reshape(shape)
        if return_routing:
            return y, w, idx
        return y
