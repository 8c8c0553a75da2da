"""Expert parallelism: the exchange plumbing (gloo, CPU, world size 2) and the GPU path.

The plumbing test drives the same ``dsm.ep`` exchange functions the GPU module uses with
CPU tensors over gloo: each rank routes random tokens, ships (token, slot) rows to the
expert owners, the owners group them by local expert and "compute" a known function of
(row, expert), and the results come back to the right pairs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsm import ep as EP


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _segment_ids(counts: np.ndarray, e_local: int) -> np.ndarray:
    """Host restatement of dsm_segment_ids: row -> local expert of its segment."""
    return np.concatenate([np.full(int(c), s % e_local, dtype=np.int64) for s, c in enumerate(counts)] or
                          [np.zeros(0, np.int64)])


def _plumbing_worker(rank: int, world: int, port: int, E: int, n_tokens: int, topk: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(100 + rank)
        idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(n_tokens)]).to(torch.int32)
        flat = idx.flatten().long()
        counts = torch.bincount(flat, minlength=E).to(torch.int32)
        perm = torch.sort(flat, stable=True).indices  # pairs in expert (= owner) order
        payload = torch.stack([torch.full_like(perm, rank), perm, flat[perm]], 1).to(torch.int64)
        recv_counts = EP.exchange_counts(counts, world)
        e0, el = EP.rank_expert_range(E, world, rank)
        send_splits, recv_splits = EP.splits(counts, world), EP.splits(recv_counts, world)
        rows = EP.exchange_rows(payload, send_splits, recv_splits, world)
        seg = _segment_ids(recv_counts.numpy(), el)
        assert rows.shape[0] == len(seg)
        # every received row is for one of my experts, in the segment the counts say
        assert bool((rows[:, 2] == torch.from_numpy(seg) + e0).all())
        # "expert compute": a function of (source, pair id, expert) the sender can check
        result = rows[:, 0] * 1_000_000 + rows[:, 1] * 1_000 + rows[:, 2]
        back = EP.exchange_rows(result.unsqueeze(1), recv_splits, send_splits, world)[:, 0]
        expect = rank * 1_000_000 + perm * 1_000 + flat[perm]
        q.put((rank, bool(torch.equal(back, expect))))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("E,n_tokens,topk", [(8, 7, 2), (16, 33, 4)])
def test_ep_exchange_plumbing_gloo_world2(E, n_tokens, topk):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plumbing_worker, args=(r, 2, port, E, n_tokens, topk, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res


def test_rank_expert_range_and_splits():
    assert EP.rank_expert_range(256, 8, 3) == (96, 32)
    with pytest.raises(ValueError):
        EP.rank_expert_range(10, 4, 0)
    c = torch.tensor([1, 2, 3, 4, 5, 6], dtype=torch.int32)
    assert EP.splits(c, 3) == [3, 7, 11]


# ----------------------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("wfmt", ["fp8", "fp4", "bf16"])
def test_ep_world1_matches_single_gpu(wfmt):
    from dsm import workloads as W
    from dsm.config import DSparkArgs
    from helpers import small_workload

    base = "fp4_decode" if wfmt == "fp4" else "fp8_decode"
    wl = small_workload(base, dim=512, inter=256, experts=16, topk=4, n_tokens=40, wfmt=wfmt, seed=9)
    t = W.make_moe_tensors(wl, device="cpu")
    moe = W.build_moe(wl, t, "cuda")
    epm = EP.ExpertParallelMoE.from_moe(moe, DSparkArgs.from_dict(t["args"]), wl.layer_id)
    x = t["x"].cuda()
    y1, _, i1 = moe(x, None, return_routing=True)
    y2, _, i2 = epm(x, None, return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2)
    assert torch.equal(y1, y2)


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
        from helpers import small_workload

        wl = small_workload("fp8_decode", dim=512, inter=256, experts=16, topk=4, n_tokens=64, seed=13)
        t = W.make_moe_tensors(wl, device="cpu")  # same weights on every rank
        moe = W.build_moe(wl, t, f"cuda:{rank}")
        epm = EP.ExpertParallelMoE.from_moe(moe, DSparkArgs.from_dict(t["args"]), wl.layer_id)
        x = t["x"][rank * 32:(rank + 1) * 32].cuda()
        y_ep = epm(x)
        y_ref = moe(x)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(y_ep, y_ref))))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_two_gpus_matches_single_gpu():
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
