"""Expert parallelism: the exchange's index arithmetic (gloo, CPU, world size 2), its C ABI
sizes, and the GPU path (ranks emulated on one GPU, and two GPUs).

The device kernels (csrc/ep.cu) place rows by three rules, restated here in Python:
* dispatch: sorted row i of expert e goes to owner d = e // El, slot j = i - offsets[d * El]
  of the sender's block; row_map[pair] = d * C + j;
* receive: an owner lays the arrived rows out by local expert, senders ascending, each
  sender's order kept: staged position -> arrival row (sender * C + slot);
* return: arrival row (s, q) goes back to sender s at slot q, where row_map finds it.
The gloo test runs those rules on two ranks with all-to-alls standing in for the peer stores
and checks that every (token, slot) pair gets its own owner's result back.
"""

from __future__ import annotations

import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsm import _lib, ep as EP


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def dispatch_slots(idx_flat: torch.Tensor, perm: torch.Tensor, offsets: torch.Tensor, e_local: int, cap: int):
    """(owner, slot) of every sorted row, and row_map [pairs] (owner * cap + slot)."""
    e = idx_flat[perm]
    d = e // e_local
    j = torch.arange(perm.numel()) - offsets[d * e_local]
    assert bool((j < cap).all())
    row_map = torch.empty_like(perm)
    row_map[perm] = d * cap + j
    return d, j, row_map


def receive_layout(cnt: torch.Tensor, cap: int):
    """cnt [W, El] rows per (sender, local expert) -> offsets [El + 1], lperm, n_valid [1 + W]."""
    W, El = cnt.shape
    tot = cnt.sum(0)
    offsets = torch.zeros(El + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(tot, 0)
    src_pos = torch.cumsum(cnt, 1) - cnt          # rows of the sender's earlier experts
    before = torch.cumsum(cnt, 0) - cnt           # rows of earlier senders, per expert
    lperm = torch.empty(int(tot.sum()), dtype=torch.int64)
    for s in range(W):
        for e in range(El):
            c = int(cnt[s, e])
            base = int(offsets[e] + before[s, e])
            lperm[base:base + c] = s * cap + src_pos[s, e] + torch.arange(c)
    n_valid = torch.cat([tot.sum().reshape(1), cnt.sum(1)])
    return offsets, lperm, n_valid


def _layout_worker(rank: int, world: int, port: int, E: int, n_tokens: int, topk: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(100 + rank)
        El = E // world
        cap = EP.capacity(n_tokens, topk, El)
        idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(n_tokens)])
        flat = idx.flatten()
        counts = torch.bincount(flat, minlength=E)
        offsets = torch.zeros(E + 1, dtype=torch.int64)
        offsets[1:] = torch.cumsum(counts, 0)
        perm = torch.sort(flat, stable=True).indices
        d, j, row_map = dispatch_slots(flat, perm, offsets, El, cap)
        # the payload of a row: (sender, pair id, expert)
        send = torch.full((world, cap, 3), -1, dtype=torch.int64)
        send[d, j] = torch.stack([torch.full_like(perm, rank), perm, flat[perm]], 1)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)  # stands in for the peer stores into [sender] blocks
        cnt = torch.empty(world, El, dtype=torch.int64)
        dist.all_to_all_single(cnt, counts.view(world, El).clone())
        loff, lperm, n_valid = receive_layout(cnt, cap)
        rows = recv.view(world * cap, 3)[lperm]
        # staged rows are grouped by local expert, in offsets order
        for e in range(El):
            assert bool((rows[loff[e]:loff[e + 1], 2] == rank * El + e).all())
        # "expert compute" in staged order, written back at the arrival positions
        result = torch.full((world * cap,), -1, dtype=torch.int64)
        result[lperm] = rows[:, 0] * 1_000_000 + rows[:, 1] * 1_000 + rows[:, 2]
        back_send = torch.full((world, cap), -1, dtype=torch.int64)
        for s in range(world):
            nq = int(n_valid[1 + s])
            back_send[s, :nq] = result.view(world, cap)[s, :nq]
        back = torch.empty_like(back_send)
        dist.all_to_all_single(back, back_send)  # stands in for the return stores
        got = back.view(-1)[row_map]
        expect = rank * 1_000_000 + torch.arange(flat.numel()) * 1_000 + flat
        q.put((rank, bool(torch.equal(got, expect))))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("E,n_tokens,topk", [(8, 7, 2), (16, 33, 4), (4, 20, 4)])
def test_ep_exchange_layout_gloo_world2(E, n_tokens, topk):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layout_worker, args=(r, 2, port, E, n_tokens, topk, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res


def test_rank_expert_range_capacity_and_buffer_bytes():
    assert EP.rank_expert_range(256, 8, 3) == (96, 32)
    with pytest.raises(ValueError):
        EP.rank_expert_range(10, 4, 0)
    assert EP.capacity(56, 6, 32) == 336 and EP.capacity(56, 6, 2) == 112
    L = _lib.lib()
    d = _lib.EpDesc(8, 3, 32, 4096, _lib.DT_BF16, 336)
    rows = 2 * 8 * 336 * 4096 * 2
    back = 2 * 8 * 336 * 4096 * 4
    r256 = lambda v: (v + 255) // 256 * 256  # noqa: E731
    want = r256(rows) + r256(2 * 8 * 32 * 4) + r256(2 * 8 * 4) + r256(back) + r256(2 * 8 * 4)
    assert L.dsm_ep_buffer_bytes(ctypes.byref(d)) == want
    assert L.dsm_ep_rows_offset(ctypes.byref(d), 1) == 8 * 336 * 4096 * 2
    assert L.dsm_ep_results_offset(ctypes.byref(d), 2) == r256(rows) + r256(2 * 8 * 32 * 4) + r256(2 * 8 * 4)
    for bad in (_lib.EpDesc(8, 8, 32, 4096, _lib.DT_BF16, 336), _lib.EpDesc(8, 0, 32, 4100, _lib.DT_BF16, 336),
                _lib.EpDesc(0, 0, 32, 4096, _lib.DT_BF16, 336), _lib.EpDesc(2, 0, 32, 4096, _lib.DT_I32, 336)):
        assert L.dsm_ep_buffer_bytes(ctypes.byref(bad)) == 0


# ----------------------------------------------------------------------------------- GPU
def _small(wfmt="fp8", n_tokens=40, experts=16, topk=4, seed=9):
    from helpers import small_workload

    base = "fp4_decode" if wfmt == "fp4" else "fp8_decode"
    return small_workload(base, dim=512, inter=256, experts=experts, topk=topk, n_tokens=n_tokens, wfmt=wfmt, seed=seed)


@pytest.mark.gpu
@pytest.mark.parametrize("wfmt", ["fp8", "fp4", "bf16"])
def test_ep_world1_matches_single_gpu(wfmt):
    from dsm import workloads as W
    from dsm.config import DSparkArgs

    wl = _small(wfmt)
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, "cuda")
    epm = EP.ExpertParallelMoE.from_moe(moe, DSparkArgs.from_dict(t["args"]), wl.layer_id, max_tokens=64)
    x = t["x"].cuda()
    y1, _, i1 = moe(x, None, return_routing=True)
    for _ in range(3):  # both buffer sets, twice
        y2, _, i2 = epm(x, None, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(i1, i2)
        assert torch.equal(y1, y2)
    assert _lib.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("world,wfmt,n_tokens", [(2, "fp8", 40), (4, "fp4", 33), (4, "bf16", 1), (8, "fp8", 21)])
def test_ep_ranks_emulated_on_one_gpu_match_single_gpu(world, wfmt, n_tokens):
    """W ranks' modules on one GPU, driven phase by phase (every dispatch, every compute, every
    combine: each wait finds its signals raised by earlier launches). Each rank routes its own
    tokens; its output must equal the single-GPU module's on those tokens, bit for bit, and the
    receive kernel's layout must equal the restatement above."""
    from dsm import workloads as W
    from dsm.config import DSparkArgs

    wl = _small(wfmt, n_tokens=n_tokens * world, experts=16, topk=4)
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, "cuda")
    args = DSparkArgs.from_dict(t["args"])
    mods = [EP.ExpertParallelMoE.from_moe(moe, args, wl.layer_id, max_tokens=n_tokens, world=world, rank=r)
            for r in range(world)]
    EP.connect_on_one_device(mods, torch.bfloat16, "cuda")
    xs = [t["x"][r * n_tokens:(r + 1) * n_tokens].cuda() for r in range(world)]
    for step in range(3):
        sts = [m.dispatch(x) for m, x in zip(mods, xs)]
        for m, st in zip(mods, sts):
            m.compute(st)
        ys = [m.combine(st) for m, st in zip(mods, sts)]
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        for r in range(world):
            assert torch.equal(ys[r], moe(xs[r])), (step, r)
    # the receive layout against the restatement, from the last step's counts
    E, El = args.n_routed_experts, args.n_routed_experts // world
    cap = EP.capacity(n_tokens, 4, El)
    counts = [torch.bincount(st["idx"].flatten().long().cpu(), minlength=E).view(world, El) for st in sts]
    for r in range(world):
        cnt = torch.stack([c[r] for c in counts])
        loff, lperm, n_valid = receive_layout(cnt, cap)
        got_off, got_perm, got_nv = sts[r]["keep_compute"][:3]
        assert torch.equal(got_off.cpu().long(), loff)
        assert torch.equal(got_nv.cpu().long(), n_valid)
        assert torch.equal(got_perm[:lperm.numel()].cpu().long(), lperm)


def _nccl_worker(rank: int, world: int, port: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from dsm import workloads as W
        from dsm.config import DSparkArgs
        from helpers import MOE_TOL, max_rel_err, oracle_moe, small_workload

        wl = small_workload("fp8_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=64, seed=13)
        t = W.make_moe_tensors(wl, device="cpu")  # same weights on every rank
        moe = W.build_moe(wl, t, f"cuda:{rank}")
        epm = EP.ExpertParallelMoE.from_moe(moe, DSparkArgs.from_dict(t["args"]), wl.layer_id, max_tokens=32)
        rows = list(range(rank * 32, (rank + 1) * 32))
        x = t["x"][rows].cuda()
        ok = True
        for _ in range(3):
            y_ep = epm(x)
            y_ref = moe(x)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(y_ep, y_ref))
        ref_y, _, _ = oracle_moe(wl, t, tokens=rows)
        ok = ok and max_rel_err(y_ep, ref_y) < MOE_TOL and _lib.device_error() == 0
        q.put((rank, ok))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_two_gpus_matches_single_gpu_and_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res
