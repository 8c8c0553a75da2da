"""Benchmark of the DSpark draft-layer MoE block on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

One step = one MoE-layer call (router, permutation, grouped fp8 expert SwiGLU, combine,
shared expert) on one draft block of synthetic tokens: by default the fp8 decode workload
(hidden 4096, 256 experts, top-6, inter 2048, e4m3 experts with 128x128 fp32 block
scales, 8 sequences x 7 draft tokens). The routed expert weights touched per step
(~4.7 GB) are far larger than L2, and steps rotate over several token batches, so no step
is served from cache.

Prints one JSON line (rank 0). ``value`` is whole-job tokens/s with inputs resident in HBM;
``e2e`` is the same metric through the public ``dsm.MoE`` call with the tokens copied from
pinned host memory and the output copied back inside the timed region.
``--impl reference`` times the CPU restatement of the reference block on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "dspark-mlx_b200"))
sys.path.insert(0, ROOT)

METRIC = "MoE-layer tokens/s & draft-block latency; HBM GB/s vs 8 TB/s at 1/2/4/8 B200"
SPEC_HBM_GBS = 8000.0
KERNELS_PER_STEP = 10  # router 3, permute 1, staging 1, routed gate/up + down 2, shared gate/up + down 2, combine 1
# expert-parallel step: router 3, permute 1, dispatch 1, shared expert 3 (staging, gate/up, down), receive 1,
# staging 1, gate/up + down 2, return 1, wait 1, combine 1
KERNELS_PER_STEP_EP = 15


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x1: "gpu_idle", 0x2: "applications_clocks_setting"}

    def __init__(self, index: int, period: float = 0.05):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._h = None
            try:
                import torch

                pr = torch.cuda.get_device_properties(self.index)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._nv = None
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                r = get(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _init_dist(ws, dev):
    """One NCCL process group per run (several workloads may run in one process)."""
    if ws <= 1:
        return
    import datetime

    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)


def _finish_dist():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(v: float, ws: int, device) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class CpuReference:
    """The CPU restatement of the reference block on a sample of the workload's tokens.

    Routed experts are dequantised to fp32 once, before timing, as the reference's loader
    does at load time (``dspark_mlx/loading.py:7-18``); each timed call is ``MoE.__call__``
    restated (router, per-(token, slot) expert products, fp32 combine, shared expert).
    ``t`` holds the small tensors (x, router, shared expert); ``experts(ids)`` returns the
    routed expert stacks of the given experts, in that order.
    """

    def __init__(self, wl, t, experts, sample_tokens: int, threads: int):
        import torch

        import oracle

        torch.set_num_threads(threads)
        self.oracle, self.threads = oracle, threads
        a = t["args"]
        self.a = a
        self.sample = sample_tokens
        self.x = t["x"][:sample_tokens].cpu()
        self.gw = t["gate_weight"].cpu()
        self.gb = t["gate_bias"].cpu() if "gate_bias" in t else None
        self.t2e = t["tid2eid"].cpu() if "tid2eid" in t else None
        self.ids = t["input_ids"][:sample_tokens].cpu() if "input_ids" in t else None
        self.kw = dict(topk=a["n_activated_experts"], score_func=a["score_func"], route_scale=a["route_scale"])
        _, idx = oracle.gate_forward(self.x, self.gw, bias=self.gb, tid2eid=self.t2e, input_ids=self.ids, **self.kw)
        used = sorted(set(idx.flatten().tolist()))
        self.remap = torch.full((a["n_routed_experts"],), -1, dtype=torch.int64)
        self.remap[used] = torch.arange(len(used))
        st = experts(used)
        self.w = {}
        for n in ("w1", "w3", "w2"):
            mats = []
            for j in range(len(used)):
                if wl.wfmt == "fp8":
                    mats.append(oracle.fp8_weight_dequant(st[n + "_codes"][j].cpu(), st[n + "_scale"][j].cpu()))
                elif wl.wfmt == "fp4":
                    mats.append(oracle.fp4_weight_dequant(st[n + "_codes"][j].cpu(), st[n + "_scale"][j].cpu(),
                                                          st[n + "_tensor_scale"][j].cpu()))
                else:
                    mats.append(st[n][j].cpu())
            self.w[n] = oracle.OracleWeights("dense", torch.stack(mats))
        self.shared = (t["shared_w1"].cpu(), t["shared_w2"].cpu(), t["shared_w3"].cpu())

    def call(self):
        import torch

        o = self.oracle
        weights, ind = o.gate_forward(self.x, self.gw, bias=self.gb, tid2eid=self.t2e, input_ids=self.ids, **self.kw)
        out = o.route_experts(self.x, self.remap[ind.long()].to(torch.int32), self.w["w1"], self.w["w3"],
                              self.w["w2"], self.a["swiglu_limit"])
        y = (out.float() * weights[..., None]).sum(-2)
        y = y + o.expert_forward(self.x, *self.shared, self.a["swiglu_limit"]).float()
        return y.to(self.x.dtype)

    def timed(self, budget_s: float, max_calls: int = 1000):
        """tokens/s over repeated calls for about ``budget_s`` seconds."""
        self.call()
        n, t0 = 0, time.perf_counter()
        while True:
            self.call()
            n += 1
            el = time.perf_counter() - t0
            if el > budget_s or n >= max_calls:
                return self.sample * n / el, n, el


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    from dsm import workloads as W

    wl = W.WORKLOADS[args.workload]
    t = W.make_moe_tensors(wl, device="cpu", routed=False)
    threads = os.cpu_count() or 1
    # the whole call for the decode workloads (the GPU arm's own config); a bounded sample of
    # the 16384-token prefill call
    sample = wl.n_tokens if wl.n_tokens <= 512 else 16
    ref = CpuReference(wl, t, lambda ids: W.expert_tensors(wl, ids), sample, threads)
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ref.call()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append(sample / dt)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wl.n_tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16 in/out)",
        "data": "synthetic",
        "config": moe_config(wl, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": (f"the whole {wl.n_tokens}-token call per step" if sample == wl.n_tokens else
                                    f"one call per step on {sample} of the {wl.n_tokens} tokens") +
                                   ", the touched experts dequantised to fp32 before timing (the reference dequantises "
                                   "at load); CPU restatement of MoE.__call__ in PyTorch (mlx is not installable "
                                   "here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def moe_config(wl, ws: int) -> dict:
    """The ``config`` object of a MoE workload's line (the same for the GPU and the reference arm)."""
    a = wl.args
    return {"workload": wl.name, "tokens_per_step_per_gpu": wl.n_tokens, "batch": wl.batch, "draft_block": wl.block,
            "dim": a["dim"], "n_experts": a["n_routed_experts"], "topk": a["n_activated_experts"],
            "inter": a["moe_inter_dim"], "weights": wl.wfmt, "score_func": a["score_func"],
            "routing": "hash" if wl.layer_id < a.get("n_hash_layers", 0) else
            (f"zipf({wl.zipf_alpha})" if wl.zipf_alpha else "uniform"),
            "parallelism": f"ep{ws} (experts sharded, peer stores over NVLink)" if ws > 1 else "single",
            "l2": "inputs larger than L2 (touched expert weights exceed L2, 4 rotating token batches)"
            if wl.name != "tiny_hash" else "tiny: weights (3 MB) L2-resident, as in the reference's latency case"}


# Tokens of each MoE workload that the CPU baseline inside the GPU run takes per call (None:
# the whole call). The large calls are bounded so the default run ends within minutes.
CPU_SAMPLE = {"fp8_decode": None, "tiny_hash": None, "fp4_decode": 56, "prefill_fp8": 16}


def run_gpu(args, wl_name=None, emit=True):
    """One MoE workload on this rank's GPU; returns (and with ``emit`` prints) its JSON line."""
    import ctypes

    import torch

    from dsm import _lib, workloads as W

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    wl = W.WORKLOADS[wl_name or args.workload]
    if args.experts:
        # a smaller expert pool with every per-expert shape unchanged (profiling captures)
        import dataclasses

        wl = dataclasses.replace(wl, args=dict(wl.args, n_routed_experts=args.experts))
    if args.tokens:
        # fewer tokens per call, every other shape unchanged (small profiling captures)
        import dataclasses

        wl = dataclasses.replace(wl, n_tokens=args.tokens)
    # every rank holds the same weights; each rank routes its own tokens
    t = W.make_moe_tensors(wl, device=dev, seed=wl.seed)
    moe = W.build_moe(wl, t, dev)
    N, dim, E = wl.n_tokens, wl.args["dim"], wl.args["n_routed_experts"]
    # several distinct token batches (different routing per step)
    n_batches = 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    xs = [t["x"] if ws == 1 else torch.randn(N, dim, generator=gen, device=dev).to(torch.bfloat16)]
    xs += [torch.randn(N, dim, generator=gen, device=dev).to(torch.bfloat16) for _ in range(n_batches - 1)]
    ids = t.get("input_ids")
    L = _lib.lib()
    stream = torch.cuda.current_stream()
    topk = wl.args["n_activated_experts"]
    if ws == 1:
        model = moe
        desc, keep = moe.describe(N, torch.bfloat16)
        wsb = L.dsm_moe_workspace_bytes(ctypes.byref(desc))
        wsp = torch.empty(wsb, dtype=torch.uint8, device=dev)
        y = torch.empty(N, dim, dtype=torch.bfloat16, device=dev)
        rw = torch.empty(N, topk, dtype=torch.float32, device=dev)
        ri = torch.empty(N, topk, dtype=torch.int32, device=dev)
        ids_p = ids.data_ptr() if ids is not None else None

        def step(i):
            x = xs[i % n_batches]
            _lib.check(L.dsm_moe_forward(ctypes.byref(desc), x.data_ptr(), _lib.DT_BF16, ids_p, _lib.DT_I32,
                                         N if ids is not None else 0, y.data_ptr(), rw.data_ptr(), ri.data_ptr(),
                                         wsp.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream))

        def routing(i):
            step(i)
            return ri
    else:
        from dsm.config import DSparkArgs
        from dsm.ep import ExpertParallelMoE

        model = ExpertParallelMoE.from_moe(moe, DSparkArgs.from_dict(t["args"]), wl.layer_id, max_tokens=N)
        del moe
        t = {k: v for k, v in t.items() if not (k[:2] in ("w1", "w2", "w3"))}
        torch.cuda.empty_cache()

        def step(i):
            model(xs[i % n_batches], ids)

        def routing(i):
            return model(xs[i % n_batches], ids, return_routing=True)[2]

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # routing statistics of the measured batches (for the algorithmic byte count): the routed
    # expert bytes this rank streams are those of its experts that any rank's tokens touch
    touched_bytes = []
    for i in range(n_batches):
        idx = routing(i).flatten().long()
        c = torch.bincount(idx, minlength=E)
        if ws > 1:
            import torch.distributed as dist

            dist.all_reduce(c)
            e0, el = model.e0, model.e_local
            c = c[e0:e0 + el]
        touched_bytes.append(W.routed_weight_bytes(wl, c.cpu()))
    torch.cuda.synchronize()
    # one CUDA graph per token batch: the whole layer call (every launch of dsm_moe_forward,
    # the shared expert's side stream included) replayed as one graph launch
    graphs, graph_note = None, None
    # launch-bound calls (decode-shaped: up to 4096 routed rows) replay as graphs; a prefill
    # call's launches are a negligible share of its ~10 ms
    if ws == 1 and not args.no_graph and N * topk <= 4096:
        try:
            graphs = []
            for b in range(n_batches):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    step(b)
                graphs.append(g)
            for i in range(args.warmup):
                graphs[i % n_batches].replay()
            torch.cuda.synchronize()
        except Exception as exc:  # noqa: BLE001 - report and time the eager calls instead
            graphs, graph_note = None, f"capture failed: {exc}"

    def timed(run):
        _barrier(ws)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk_:
            a.record(stream)
            for i in range(args.steps):
                run(i)
            b.record(stream)
            torch.cuda.synchronize()
        return _max_over_ranks(a.elapsed_time(b) / args.steps, ws, dev), clk_

    eager_ms, clk = timed(step)
    ms = eager_ms
    if graphs:
        ms, clk = timed(lambda i: graphs[i % n_batches].replay())
    _barrier(ws)
    ep_info = ep_measure(model, step, routing, ws, rank, dev, wl) if ws > 1 else None

    # ---- dominant kernel: the fused gate/up expert kernel, timed alone with events (1 GPU)
    sh_bytes = 3 * wl.args["moe_inter_dim"] * dim * 2
    gate_bytes = E * dim * 4
    per_step_bytes = [b + sh_bytes + gate_bytes + 2 * N * dim * 2 for b in touched_bytes]
    avg_step_bytes = sum(per_step_bytes[i % n_batches] for i in range(args.steps)) / args.steps
    hbm_peak, tc_peak, peak_kind = _peaks()
    k_tc = False
    if args.no_kernel_timing or ws > 1:
        k_ms, k_bytes, k_touched, k_flops, achieved = None, None, None, None, None
    else:
        k_ms, k_bytes, k_touched, k_flops, k_tc = time_gate_up(model, xs[0], ids, args, L, dev)
        achieved = k_bytes / (k_ms * 1e-3) / 1e9
    moe = model

    # ---- end to end through the public API: pinned host tokens in, host result out
    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        yh = torch.empty(N, dim, dtype=torch.bfloat16).pin_memory()
        ids_d = ids
        for i in range(3):
            yh.copy_(moe(xh[i % n_batches].to(dev, non_blocking=True), ids_d), non_blocking=True)
        torch.cuda.synchronize()
        _barrier(ws)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for i in range(args.steps):
            xd = xh[i % n_batches].to(dev, non_blocking=True)
            yh.copy_(moe(xd, ids_d), non_blocking=True)
        e3.record(stream)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(e2.elapsed_time(e3) / args.steps, ws, dev)

    # DRAM traffic of the dominant kernel from the committed ncu capture (a smaller expert
    # pool), scaled to this launch by the experts it streams
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            per = json.load(f).get(f"gate_up/{wl.name}")
        if per and k_touched:
            traffic = per["bytes_per_touched_expert"] * k_touched
    except Exception:
        traffic = None

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1

            def experts(ids, t=t):
                keys = [k for k in t if k[:2] in ("w1", "w2", "w3")]
                return {k: t[k][ids].cpu() for k in keys}

            cpu_n = CPU_SAMPLE.get(wl.name) or N
            budget = args.cpu_seconds if wl.name == "fp8_decode" else min(args.cpu_seconds, 8.0)
            v, n, el = CpuReference(wl, t, experts, cpu_n, threads).timed(budget)
            what = f"the whole {N}-token call" if cpu_n >= N else f"{cpu_n} of the {N} tokens per call"
            cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{what}, {n} calls in {el:.1f} s; the touched experts dequantised to fp32 before "
                             f"timing (the reference dequantises at load); CPU restatement of MoE.__call__ in "
                             f"PyTorch"}
        value = ws * N / (ms * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE_DESC.get(wl.wfmt, wl.wfmt),
            "data": "synthetic",
            "config": moe_config(wl, ws),
            "moe_layer_latency_ms": ms,
            "hbm_gbs_step": avg_step_bytes / (ms * 1e-3) / 1e9,
            "hbm_frac_of_8tbs_step": avg_step_bytes / (ms * 1e-3) / 1e9 / SPEC_HBM_GBS,
            "roofline": roofline_entry(ws, k_ms, k_bytes, k_touched, k_flops, k_tc, achieved, avg_step_bytes, ms,
                                       hbm_peak, tc_peak, peak_kind, traffic, wl.wfmt, ep_info),
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * N / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": N * dim * 2,
                "d2h_bytes_per_step": N * dim * 2, "ms_per_step": e2e_ms},
            "gpu_launches": (KERNELS_PER_STEP if ws == 1 else KERNELS_PER_STEP_EP) * args.steps,
            "clocks": clk.summary(),
        }
        if ep_info is not None:
            line["expert_parallel"] = ep_info
        if ws == 1:
            line["launch"] = ("CUDA graph replay of the whole layer call (one graph per token batch)" if graphs
                              else "eager C-ABI calls" + (f" ({graph_note})" if graph_note else ""))
            line["ms_per_step_eager"] = eager_ms
        if emit:
            print(json.dumps(line))
        return line
    return None


def ep_measure(model, step, routing, ws, rank, dev, wl, n=3):
    """Expert parallelism, per rank: the row exchange (dispatch of the routed rows to their
    owners, return of the fp32 results) and the local gate/up product, timed with CUDA events
    around those launches over ``n`` further steps, and the NVLink bytes each rank stores into
    its peers' buffers (from the same steps' routing). Every rank takes the same collective
    steps."""
    import torch
    import torch.distributed as dist

    dim, inter = wl.args["dim"], wl.args["moe_inter_dim"]
    model.phase_events = []
    for i in range(n):
        step(i)
    torch.cuda.synchronize()
    acc = {}
    for name, a, b in model.phase_events:
        acc.setdefault(name, []).append(a.elapsed_time(b))
    model.phase_events = None
    names = ("dispatch", "return", "gate_up")
    t = torch.zeros(ws, len(names), dtype=torch.float64, device=dev)
    for j, name in enumerate(names):
        v = acc.get(name, [])
        t[rank, j] = sum(v) / len(v) if v else 0.0
    pairs = torch.zeros(ws, ws, dtype=torch.float64, device=dev)  # [sender, owner] routed rows
    for i in range(n):
        owner = routing(i).flatten().long() // model.e_local
        pairs[rank] += torch.bincount(owner, minlength=ws).double()
    dist.all_reduce(t)
    dist.all_reduce(pairs)
    t, pairs = t.cpu(), (pairs / n).cpu()
    own = pairs.diagonal()
    rows_in = pairs.sum(0)                        # rows each owner's experts compute
    sent = (pairs.sum(1) - own) * dim * 2         # bf16 rows stored into peers
    back = (rows_in - own) * dim * 4              # fp32 results stored back to their senders
    out_bytes = sent + back
    ex_ms = t[:, 0] + t[:, 1]
    gbs = [float(b / (m * 1e-3) / 1e9) if m > 0 else None for b, m in zip(out_bytes, ex_ms)]
    topk = wl.args["n_activated_experts"]
    hint, busy = wl.n_tokens * topk, min(wl.n_tokens * topk, model.e_local)
    tc = wl.wfmt == "fp8" and hint >= 64 * busy  # the expert products' dispatch rule
    info = {
        "exchange": "peer stores into CUDA-IPC buffers over NVLink (no NCCL on the data path)",
        "dispatch_ms": [float(v) for v in t[:, 0]],
        "return_ms": [float(v) for v in t[:, 1]],
        "a2a_bytes_out_per_step": [float(v) for v in out_bytes],
        "a2a_gbs_per_gpu": gbs,
        "a2a_gbs_per_gpu_mean": sum(g for g in gbs if g) / max(1, sum(1 for g in gbs if g)),
        "nvlink_nominal_gbs_per_direction": 900,
        "rows_per_rank": [float(v) for v in rows_in],
        "gate_up_ms": [float(v) for v in t[:, 2]],
        "gate_up_regime": "tcgen05 (tensor)" if tc else "weight streaming (HBM)",
        "sample": f"{n} steps after the timed ones",
    }
    if tc:
        info["gate_up_tflops"] = [float(2 * 2 * r * dim * inter / (m * 1e-3) / 1e12) if m > 0 else None
                                  for r, m in zip(rows_in, t[:, 2])]
    return info


# arithmetic of the routed expert products per weight format
DTYPE_DESC = {
    "fp8": "fp8 e4m3 weights x bf16 activations (f16 MMA, fp32 accumulate)",
    "fp4": "fp4 e2m1 weights (e4m3 group scales) x bf16 activations (f16 tcgen05 MMA, fp32 accumulate)",
    "bf16": "bf16 weights x bf16 activations (f16 MMA, fp32 accumulate)",
    "affine8": "8-bit affine weights x bf16 activations (f16 tcgen05 MMA, fp32 accumulate)",
}


def graph_replay(make_call, timed, warmup, n_batches=4):
    """Capture ``make_call(b)`` for each token batch ``b`` into its own CUDA graph and time
    the replays with ``timed``: ``(ms, note)``, or ``(None, note)`` when capture fails (the
    eager time then stands)."""
    import torch

    try:
        graphs = []
        for b in range(n_batches):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                make_call(b)
            graphs.append(g)
        for i in range(warmup):
            graphs[i % n_batches].replay()
        torch.cuda.synchronize()
    except Exception as exc:  # noqa: BLE001 - report and keep the eager time
        return None, f"eager calls (capture failed: {exc})"
    return timed(lambda i: graphs[i % n_batches].replay()), "CUDA graph replay of the whole call (one graph per token batch)"


def roofline_entry(ws, k_ms, k_bytes, k_touched, k_flops, k_tc, achieved, step_bytes, ms, hbm_peak, tc_peak,
                   peak_kind, traffic, wfmt="fp8", ep_info=None):
    """The roofline figure of the dominant kernel (or, for expert parallelism, of the step;
    of the local gate/up product on the slowest rank when it runs on the tensor pipe)."""
    if ws > 1 and ep_info and ep_info.get("gate_up_tflops"):
        ms_r = ep_info["gate_up_ms"]
        r = max(range(len(ms_r)), key=lambda i: ms_r[i])  # the rank that bounds the step
        tflops = ep_info["gate_up_tflops"][r]
        return {"bound": "tensor", "kernel": f"expert_tc_kernel<gate_up> on rank {r} (the slowest)",
                "achieved": tflops, "peak": tc_peak, "unit": "TFLOP/s", "frac": tflops / tc_peak,
                "peak_kind": peak_kind + " (dense bf16/f16 burst)", "launch_ms": ms_r[r], "traffic": None}
    if ws > 1:
        gbs = step_bytes / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "kernel": "whole step per rank (expert-parallel)", "achieved": gbs, "peak": hbm_peak,
                "unit": "GB/s", "frac": gbs / hbm_peak, "peak_kind": peak_kind, "traffic": None}
    if achieved is None:
        return None
    if k_tc:  # many rows per expert: the tcgen05 kernel, bound by the tensor pipe
        tflops = k_flops / (k_ms * 1e-3) / 1e12
        return {"bound": "tensor", "kernel": "expert_tc_kernel<gate_up> (tcgen05 kind::f16, TMEM)",
                "achieved": tflops, "peak": tc_peak, "unit": "TFLOP/s", "frac": tflops / tc_peak,
                "peak_kind": peak_kind + " (dense bf16/f16 burst)", "algorithmic_flops_per_launch": k_flops,
                "launch_ms": k_ms, "hbm_gbs": achieved, "traffic": None}
    kernel = ("expert_tm_kernel<gate_up> (e2m1 dequantised into TMEM, tcgen05 kind::f16)" if wfmt == "fp4"
              else f"expert_kernel<{wfmt}, gate_up> (weight streaming, mma.sync)")
    return {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": hbm_peak,
            "unit": "GB/s", "frac": achieved / hbm_peak, "peak_kind": peak_kind,
            "frac_of_8tbs": achieved / SPEC_HBM_GBS, "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms,
            "touched_experts": k_touched, "traffic": traffic,
            "traffic_over_algorithmic": (traffic / k_bytes) if traffic else None}


def time_gate_up(moe, x, ids, args, L, dev):
    """Average duration of the fused gate/up expert kernel (CUDA events) and its algorithmic bytes."""
    import ctypes

    import torch

    from dsm import _lib

    N = x.shape[0]
    desc, keep = moe.describe(N, torch.bfloat16)
    p1, p3 = keep[0], keep[1]
    E, topk = desc.n_experts, desc.topk
    P = N * topk
    s = torch.cuda.current_stream().cuda_stream
    w, idx = moe.gate(x, ids)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(P, dtype=torch.int32, device=dev)
    inv = torch.empty(P, dtype=torch.int32, device=dev)
    pwsb = L.dsm_permute_workspace_bytes(P, E)
    pws = torch.empty(pwsb, dtype=torch.uint8, device=dev)
    _lib.check(L.dsm_permute(idx.data_ptr(), P, E, counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
                             inv.data_ptr(), pws.data_ptr(), pwsb, s))
    cap = L.dsm_stage_rows_cap(P)
    xs = torch.empty(L.dsm_stage_bytes(cap, desc.dim), dtype=torch.uint8, device=dev)
    xsc = torch.empty(cap, dtype=torch.float32, device=dev)
    hs = torch.empty(L.dsm_stage_bytes(cap, desc.inter), dtype=torch.uint8, device=dev)
    _lib.check(L.dsm_stage_rows(x.data_ptr(), _lib.DT_BF16, N, desc.dim, perm.data_ptr(), P, topk, xs.data_ptr(), cap,
                                xsc.data_ptr(), s))

    def launch():
        _lib.check(L.dsm_expert_gate_up(xs.data_ptr(), xsc.data_ptr(), cap, desc.dim, offsets.data_ptr(), E, p1.wfmt,
                                        p1.group_size, p1.packed.data_ptr(), p3.packed.data_ptr(), desc.inter,
                                        desc.act, desc.swiglu_limit, desc.round_gu, hs.data_ptr(), 1.0, P, s))

    for _ in range(5):
        launch()
    torch.cuda.synchronize()
    n = max(20, min(args.steps, 500))
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(n):
        launch()
    a1.record()
    torch.cuda.synchronize()
    k_ms = a0.elapsed_time(a1) / n
    c = counts.cpu()
    touched = int((c > 0).sum())
    header = -(-E * 4 // 256) * 256
    per_expert = (p1.packed.numel() - header) // E  # packed tile bytes (codes + scales) of one expert
    w13 = 2 * touched * per_expert
    act = (P * desc.dim * 2) + (P * desc.inter * 2)
    flops = 2 * 2 * P * desc.dim * desc.inter  # gate and up products over every (token, slot) pair
    busy = max(1, min(P, E))
    tc = p1.wfmt == _lib.WFMT_FP8_B128 and P >= 64 * busy  # the dispatch rule of the expert kernels
    return k_ms, w13 + act, touched, flops, tc


QWEN3_METRIC = "Qwen3 draft-layer MLP tokens/s (8-bit affine, L2 flushed per step); HBM GB/s"
QWEN3_KERNELS_PER_STEP = 4  # staging, gate/up, down (K-split), split sum + cast


def _qwen3_cpu_weights(mlp):
    """The oracle's view of the projections, dequantised to fp32 once (the timed CPU leg then
    measures the three matmuls and the elementwise ops, as the reference does after load)."""
    import oracle

    out = []
    for p in (mlp.gate_proj, mlp.up_proj, mlp.down_proj):
        if p.quant is None:
            w = p.weight.detach().cpu().float()
        else:
            bits, gs = p.quant
            w = oracle.OracleWeights("affine", p.q.cpu().unsqueeze(0), scales=p.scales.cpu().unsqueeze(0),
                                     biases=p.biases.cpu().unsqueeze(0), group_size=gs, bits=bits).matrix(0)
        out.append(oracle.OracleWeights("dense", w.unsqueeze(0).contiguous()))
    return out


def _qwen3_cpu_timed(x, weights, sample, budget_s, max_calls=1000):
    import torch

    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    xs = x[:sample].cpu()
    oracle.qwen3_mlp(xs, *weights)
    n, t0 = 0, time.perf_counter()
    while n < max_calls and time.perf_counter() - t0 < budget_s:
        oracle.qwen3_mlp(xs, *weights)
        n += 1
    el = time.perf_counter() - t0
    return sample * n / el, n, el


def run_qwen3(args, emit=True):
    """One step = one Qwen3 MLP call (hidden 2560, inter 9728, 8-bit affine g64) on 16 x 7
    draft tokens. The quantised weights (79 MB) fit in L2, so L2 is flushed (a 256 MB write)
    before every timed call, outside the CUDA-event bracket of that call."""
    import ctypes

    import torch

    from dsm import _lib, workloads as W

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    wl = W.WORKLOADS["qwen3_mlp_q8"]
    t = W.make_qwen3_tensors(wl, device=dev)
    mlp = W.build_qwen3_mlp(wl, t, dev)
    N, h, inter = wl.n_tokens, wl.args["hidden_size"], wl.args["intermediate_size"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    xs = [t["x"]] + [torch.randn(N, h, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        mlp(xs[i % 4])
    torch.cuda.synchronize()

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.zero_()
            evs[i][0].record(stream)
            fn(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / args.steps

    _barrier(ws)
    with ClockSampler(local) as clk:
        ms = timed(lambda i: mlp(xs[i % 4]))
    eager_ms = _max_over_ranks(ms, ws, dev)
    ms = eager_ms
    # the same call replayed as a CUDA graph (one per token batch)
    graph_note = None
    if not args.no_graph:
        try:
            graphs = []
            for b in range(4):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    mlp(xs[b])
                graphs.append(g)
            for i in range(args.warmup):
                graphs[i % 4].replay()
            torch.cuda.synchronize()
            _barrier(ws)
            with ClockSampler(local) as clk:
                ms = _max_over_ranks(timed(lambda i: graphs[i % 4].replay()), ws, dev)
            graph_note = "CUDA graph replay of the whole MLP call (one graph per token batch)"
        except Exception as exc:  # noqa: BLE001 - report and keep the eager time
            graph_note = f"eager C-ABI calls (capture failed: {exc})"
    pg, pu, pd = mlp.gate_proj.packed(), mlp.up_proj.packed(), mlp.down_proj.packed()
    weight_bytes = pg.nbytes + pu.nbytes + pd.nbytes
    step_bytes = weight_bytes + 2 * N * h * 2
    hbm_peak, _, peak_kind = _peaks()

    # dominant kernel: the fused gate/up product, timed alone after the same flush
    roofline = None
    if not args.no_kernel_timing and ws == 1:
        L = _lib.lib()
        cap = L.dsm_stage_rows_cap(N)
        xsb = torch.empty(L.dsm_stage_bytes(cap, h), dtype=torch.uint8, device=dev)
        xsc = torch.empty(cap, dtype=torch.float32, device=dev)
        hsb = torch.empty(L.dsm_stage_bytes(cap, inter), dtype=torch.uint8, device=dev)
        sp = stream.cuda_stream
        _lib.check(L.dsm_stage_rows(xs[0].data_ptr(), _lib.DT_BF16, N, h, None, N, 1, xsb.data_ptr(), cap,
                                    xsc.data_ptr(), sp))

        def gate_up(_i):
            _lib.check(L.dsm_expert_gate_up(xsb.data_ptr(), xsc.data_ptr(), cap, h, None, 1, pg.wfmt, pg.group_size,
                                            pg.packed.data_ptr(), pu.packed.data_ptr(), inter,
                                            _lib.ACT_SILU_MUL_BF16, 0.0, 3, hsb.data_ptr(), 1.0 / 256, N, sp))

        k_ms = timed(gate_up)
        k_bytes = pg.nbytes + pu.nbytes + N * h * 2 + N * inter * 2
        achieved = k_bytes / (k_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": "expert_tm_kernel<affine8, gate_up> (dequantised into TMEM, tcgen05 kind::f16)",
                    "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                    "peak_kind": peak_kind, "frac_of_8tbs": achieved / SPEC_HBM_GBS,
                    "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms, "traffic": None}

    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        yh = torch.empty(N, h, dtype=torch.bfloat16).pin_memory()
        for i in range(3):
            yh.copy_(mlp(xh[i % 4].to(dev, non_blocking=True)), non_blocking=True)
        torch.cuda.synchronize()

        def e2e(i):
            yh.copy_(mlp(xh[i % 4].to(dev, non_blocking=True)), non_blocking=True)

        e2e_ms = _max_over_ranks(timed(e2e), ws, dev)

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, n, el = _qwen3_cpu_timed(t["x"], _qwen3_cpu_weights(mlp), N, min(args.cpu_seconds, 8.0))
            cpu = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"the whole {N}-token call, {n} calls in {el:.1f} s; weights dequantised to "
                             f"fp32 before timing; CPU restatement of Qwen3MLP.__call__ in PyTorch"}
        line = {
            "metric": QWEN3_METRIC, "value": ws * N / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE_DESC["affine8"], "data": "synthetic",
            "config": {"workload": wl.name, "tokens_per_step_per_gpu": N, "batch": wl.batch, "draft_block": wl.block,
                       "hidden": h, "inter": inter, "weights": "affine8 g64 (bf16 scale, bias)",
                       "parallelism": f"replicas{ws}" if ws > 1 else "single",
                       "l2": "flushed before every timed call (256 MB write outside the timed bracket)"},
            "hbm_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
            "hbm_frac_of_8tbs_step": step_bytes / (ms * 1e-3) / 1e9 / SPEC_HBM_GBS,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * N / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": N * h * 2,
                "d2h_bytes_per_step": N * h * 2, "ms_per_step": e2e_ms},
            "gpu_launches": QWEN3_KERNELS_PER_STEP * args.steps,
            "clocks": clk.summary(),
            "launch": graph_note or "eager C-ABI calls",
            "ms_per_step_eager": eager_ms,
        }
        if emit:
            print(json.dumps(line))
        return line
    return None


def run_reference_qwen3(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    import torch

    from dsm import workloads as W

    wl = W.WORKLOADS[args.workload]
    t = W.make_qwen3_tensors(wl, device="cpu")
    import oracle

    ws_cpu = []
    for n in ("gate_proj", "up_proj", "down_proj"):
        q, sc, b = oracle.affine_quantize(t[n], 64, 8)
        w = oracle.OracleWeights("affine", q.unsqueeze(0), scales=sc.unsqueeze(0), biases=b.unsqueeze(0),
                                 group_size=64, bits=8).matrix(0)
        ws_cpu.append(oracle.OracleWeights("dense", w.unsqueeze(0).contiguous()))
    torch.set_num_threads(os.cpu_count() or 1)
    sample = min(8, wl.n_tokens)
    xs = t["x"][:sample]
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.qwen3_mlp(xs, *ws_cpu)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append(sample / dt)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": QWEN3_METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wl.n_tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16 in/out)",
        "data": "synthetic",
        "config": {"workload": wl.name, "tokens_per_step": wl.n_tokens, "hidden": wl.args["hidden_size"],
                   "inter": wl.args["intermediate_size"], "weights": "affine8 g64"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"one call per step on {sample} of the {wl.n_tokens} tokens, weights dequantised "
                                   f"to fp32 before timing; CPU restatement of Qwen3MLP.__call__ in PyTorch (mlx is "
                                   f"not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


HEAD_METRIC = "Draft-head tokens/s (hc_head + norm + LM head over 129280 words + Markov walk, greedy); HBM GB/s"
HEAD_KERNELS_PER_STEP = 4  # hc_head+norm, staging, LM head product, walk


def _head_oracle_args(t, wl):
    import torch

    a = wl.args
    return dict(head_w=t["head_w"].to(torch.float32), hc_fn=t["fn"], hc_scale=t["scale"], hc_base=t["base"],
                norm_w=t["norm_w"], w1=t["w1"], w2=t["w2"], wc=t["wc"], norm_eps=1e-6, hc_eps=1e-6,
                temperature=float(a["temperature"]))


def _head_cpu_setup(t, wl):
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    kw = _head_oracle_args({k: (v.cpu() if hasattr(v, "cpu") else v) for k, v in t.items()}, wl)
    return kw, t["x"][:1].cpu(), t["anchor"][:1].cpu()


def _head_cpu_timed(t, wl, budget_s, max_calls=50, setup=None):
    """The oracle's forward_head on one batch row (a block of tokens) per call, all host threads."""
    import oracle

    kw, x, anchor = setup or _head_cpu_setup(t, wl)
    if setup is None:
        oracle.forward_head(x, anchor, **kw)
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (n == 0 or time.perf_counter() - t0 < budget_s):
        oracle.forward_head(x, anchor, **kw)
        n += 1
    el = time.perf_counter() - t0
    return n * wl.block / el, n, el


def run_head(args):
    """One step = one draft-head call (8 sequences x 7 draft positions, DeepSeek-V4 widths).
    The LM head (1.06 GB of bf16 weights) exceeds L2, so every step streams it from HBM."""
    import ctypes

    import torch

    from dsm import _lib, workloads as W

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    wl = W.WORKLOADS["draft_head"]
    t = W.make_head_tensors(wl, device=dev, seed=rank)
    head = W.build_head(wl, t, dev)
    b, s = wl.batch, wl.block
    gen = torch.Generator(device=dev)
    gen.manual_seed(777 + rank)
    xs = [t["x"]] + [torch.randn(t["x"].shape, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    anchor = t["anchor"]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        head(xs[i % 4], anchor)
    torch.cuda.synchronize()

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            evs[i][0].record(stream)
            fn(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / args.steps

    _barrier(ws)
    launch_note = "eager calls"
    with ClockSampler(local) as clk:
        ms = timed(lambda i: head(xs[i % 4], anchor))
        eager_ms = ms
        if not args.no_graph:
            gms, launch_note = graph_replay(lambda bb: head(xs[bb], anchor), timed, args.warmup)
            ms = gms if gms is not None else ms
    ms = _max_over_ranks(ms, ws, dev)
    eager_ms = _max_over_ranks(eager_ms, ws, dev)
    hp = head.packed_head()
    vocab, dim, rk = wl.args["vocab_size"], wl.args["dim"], wl.args["dspark_markov_rank"]
    step_bytes = hp.nbytes + 2 * vocab * rk * 2 + b * s * vocab * 4 * 2 + b * s * 4 * dim * 2
    hbm_peak, _, peak_kind = _peaks()

    roofline = None
    if not args.no_kernel_timing and ws == 1:  # the LM head product alone, on the staged normalised rows
        L = _lib.lib()
        n = b * s
        cap = L.dsm_stage_rows_cap(n)
        xn = torch.randn(n, dim, device=dev).to(torch.bfloat16)
        xsb = torch.empty(L.dsm_stage_bytes(cap, dim), dtype=torch.uint8, device=dev)
        xsc = torch.empty(cap, dtype=torch.float32, device=dev)
        out = torch.empty(n, vocab, dtype=torch.float32, device=dev)
        sp = stream.cuda_stream
        _lib.check(L.dsm_stage_rows(xn.data_ptr(), _lib.DT_BF16, n, dim, None, n, 1, xsb.data_ptr(), cap,
                                    xsc.data_ptr(), sp))
        k_ms = timed(lambda i: _lib.check(L.dsm_linear(xsb.data_ptr(), xsc.data_ptr(), cap, dim, hp.wfmt, hp.group_size,
                                                       hp.packed.data_ptr(), vocab, out.data_ptr(), vocab, n, sp)))
        k_bytes = hp.nbytes + n * dim * 2 + n * vocab * 4
        achieved = k_bytes / (k_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": "expert_tc_kernel<f16, down> (LM head over 56 rows, tcgen05)",
                    "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                    "peak_kind": peak_kind, "frac_of_8tbs": achieved / SPEC_HBM_GBS,
                    "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms, "traffic": None}

    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        ah = anchor.cpu().pin_memory()
        ids_h = torch.empty(b, s + 1, dtype=torch.int32).pin_memory()
        conf_h = torch.empty(b, s, dtype=torch.float32).pin_memory()

        def e2e(i):
            ids, _, conf = head(xh[i % 4].to(dev, non_blocking=True), ah.to(dev, non_blocking=True))
            ids_h.copy_(ids, non_blocking=True)
            conf_h.copy_(conf, non_blocking=True)

        for i in range(3):
            e2e(i)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(timed(e2e), ws, dev)

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, calls, el = _head_cpu_timed(t, wl, args.cpu_seconds)
            cpu = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"1 of the {b} sequences ({s} draft tokens) per call, {calls} calls in {el:.1f} s; "
                             f"CPU restatement of DSparkBlock.forward_head + the LM head in PyTorch"}
        line = {
            "metric": HEAD_METRIC, "value": ws * b * s / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 weights x bf16 activations (f16 MMA, fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": wl.name, "tokens_per_step_per_gpu": b * s, "batch": b, "draft_block": s,
                       "dim": dim, "vocab": vocab, "markov_rank": rk, "hc_mult": wl.args["hc_mult"],
                       "sampling": "greedy", "parallelism": f"replicas{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (1.06 GB LM head streamed every step)"},
            "hbm_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * b * s / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": xs[0].numel() * 2 + b * 4, "d2h_bytes_per_step": b * (s + 1) * 4 + b * s * 4,
                "ms_per_step": e2e_ms},
            "gpu_launches": HEAD_KERNELS_PER_STEP * args.steps,
            "clocks": clk.summary(),
            "launch": launch_note,
            "ms_per_step_eager": eager_ms,
        }
        print(json.dumps(line))


def run_reference_head(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    from dsm import workloads as W

    wl = W.WORKLOADS["draft_head"]
    t = W.make_head_tensors(wl, device="cpu")
    setup = _head_cpu_setup(t, wl)
    vals = []
    for i in range(args.warmup + args.steps):
        v, _, _ = _head_cpu_timed(t, wl, 0.0, max_calls=1, setup=setup)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": HEAD_METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wl.n_tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16 weights)",
        "data": "synthetic",
        "config": {"workload": wl.name, "tokens_per_step": wl.n_tokens, "batch": wl.batch, "draft_block": wl.block,
                   "vocab": wl.args["vocab_size"], "dim": wl.args["dim"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"one sequence ({wl.block} draft tokens) per step; CPU restatement of "
                                   f"DSparkBlock.forward_head + the LM head in PyTorch (mlx is not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


GQA_METRIC = ("Qwen3 draft-layer attention tokens/s (attend_cached over 2048 cached context rows, 8-bit affine "
              "projections); HBM GB/s")
# staging, q/k/v products (split K: product + sum each), head norms + RoPE, attention, range
# combine, staging, o_proj (product + sum), cast
GQA_KERNELS_PER_STEP = 1 + 3 * 2 + 1 + 1 + 1 + 1 + 2 + 1
LAYER_METRIC = ("Qwen3 draft layer tokens/s (forward_cached over 2048 cached context rows, every Linear 8-bit "
                "affine); HBM GB/s")
# input norm, the attention, residual add + post-attention norm, the MLP (staging, gate/up, split
# down, split sum + cast), the last residual add
LAYER_KERNELS_PER_STEP = 1 + GQA_KERNELS_PER_STEP + 1 + 4 + 1


def _gqa_cpu_setup(t, wl):
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    from dsm.qwen3_attention import rope_tables

    a, ctx, s = wl.args, wl.extra["ctx"], wl.block
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")
    if "gate_proj" in t:  # the whole layer
        names += ("gate_proj", "up_proj", "down_proj", "input_layernorm", "post_attention_layernorm")
    w = {k: t[k].cpu() for k in names}
    cos, sin = rope_tables(torch.arange(ctx, ctx + s), a["head_dim"], a["rope_theta"])
    return w, t["x"][:1].cpu(), t["ctx_k"][:1].cpu(), t["ctx_v"][:1].cpu(), cos, sin


def _gqa_cpu_timed(wl, setup, budget_s, max_calls=50):
    """The oracle's attend_cached (or the whole layer's forward_cached) on one sequence per call,
    all host threads."""
    import oracle

    a = wl.args
    w, x, ck, cv, cos, sin = setup
    fn = oracle.qwen3_layer_cached if "gate_proj" in w else oracle.qwen3_attend_cached
    call = lambda: fn(w, a["num_attention_heads"], a["num_key_value_heads"],  # noqa: E731
                      a["head_dim"], a["rms_norm_eps"], x, ck, cv, cos, sin)
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (n == 0 or time.perf_counter() - t0 < budget_s):
        call()
        n += 1
    el = time.perf_counter() - t0
    return n * wl.block / el, n, el


def run_gqa(args):
    """One step = ``attend_cached`` of 16 sequences' 7-token blocks over 2048 cached context rows
    each (Qwen3-4B widths). The cached K/V (134 MB) and the projections (~28 MB) exceed L2, so
    every step streams them from HBM. With ``--workload qwen3_layer_q8`` a step is the whole
    layer's ``forward_cached`` (norms, that attention, the 9728-wide MLP: ~107 MB of weights)."""
    import torch

    from dsm import _lib, workloads as W
    from dsm.qwen3_attention import rope_tables

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    _lib.check(_lib.lib().dsm_set_attn_kernel(0 if args.attn_kernel == "mma" else 1), "dsm_set_attn_kernel")
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    layer_mode = args.workload == "qwen3_layer_q8"
    wl = W.WORKLOADS[args.workload]
    a = wl.args
    if layer_mode:
        t = W.make_qwen3_layer_tensors(wl, device=dev, seed=rank)
        layer = W.build_qwen3_layer(wl, t, dev)
        attn = layer.self_attn
        step = lambda x: layer.forward_cached(x, kc, vc, cos, sin)  # noqa: E731
    else:
        t = W.make_gqa_tensors(wl, device=dev, seed=rank)
        attn = W.build_gqa(wl, t, dev)
        step = lambda x: attn.attend_cached(x, kc, vc, cos, sin)  # noqa: E731
    b, s, ctx = wl.batch, wl.block, wl.extra["ctx"]
    nh, nkv, hd, h = a["num_attention_heads"], a["num_key_value_heads"], a["head_dim"], a["hidden_size"]
    cos, sin = rope_tables(torch.arange(ctx, ctx + s), hd, a["rope_theta"])
    cos, sin = cos.to(dev), sin.to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(555 + rank)
    xs = [t["x"]] + [torch.randn(t["x"].shape, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    kc, vc = t["ctx_k"], t["ctx_v"]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(xs[i % 4])
    torch.cuda.synchronize()

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            evs[i][0].record(stream)
            fn(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(x.elapsed_time(y) for x, y in evs) / args.steps

    _barrier(ws)
    launch_note = "eager calls"
    with ClockSampler(local) as clk:
        ms = timed(lambda i: step(xs[i % 4]))
        eager_ms = ms
        if not args.no_graph:
            gms, launch_note = graph_replay(lambda bb: step(xs[bb]), timed, args.warmup)
            ms = gms if gms is not None else ms
    ms = _max_over_ranks(ms, ws, dev)
    eager_ms = _max_over_ranks(eager_ms, ws, dev)
    kv_bytes = 2 * b * nkv * ctx * hd * 2
    w_bytes = sum(getattr(attn, n).packed().nbytes for n in ("q_proj", "k_proj", "v_proj", "o_proj"))
    if layer_mode:
        w_bytes += sum(getattr(layer.mlp, n).packed().nbytes for n in ("gate_proj", "up_proj", "down_proj"))
    act_bytes = b * s * h * 2 * 2  # the block in, the output out
    step_bytes = w_bytes + kv_bytes + act_bytes
    hbm_peak, _, peak_kind = _peaks()

    roofline = None
    if not args.no_kernel_timing and ws == 1:  # dsm_gqa_attn alone (attention + range combine)
        bk = torch.empty(b, nkv, s, hd, dtype=torch.bfloat16, device=dev)
        bv = torch.empty_like(bk)
        q = attn._heads(xs[0], torch.bfloat16, True, cos, sin, 0, bk, bv, s, 0)
        L = _lib.lib()
        wsb = L.dsm_gqa_attn_workspace_bytes(b, s, nh, nkv, hd, ctx)
        wsbuf = torch.empty(wsb, dtype=torch.uint8, device=dev)
        out = torch.empty(b, s, nh * hd, dtype=torch.bfloat16, device=dev)
        sp = stream.cuda_stream
        k_ms = timed(lambda i: _lib.check(L.dsm_gqa_attn(
            q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), ctx, bk.data_ptr(), bv.data_ptr(),
            _lib.DT_BF16, b, s, nh, nkv, hd, float(attn.scale), out.data_ptr(), wsbuf.data_ptr(), wsb, sp),
            "dsm_gqa_attn"))
        k_bytes = kv_bytes + 2 * b * nkv * s * hd * 2 + 2 * b * s * nh * hd * 2
        achieved = k_bytes / (k_ms * 1e-3) / 1e9
        kname = "gqa_mma_kernel<128>" if args.attn_kernel == "mma" else "gqa_attn_kernel<bf16, 128>"
        roofline = {"bound": "hbm", "kernel": kname + " + gqa_combine_kernel",
                    "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                    "peak_kind": peak_kind, "frac_of_8tbs": achieved / SPEC_HBM_GBS,
                    "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms, "traffic": None}

    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        yh = torch.empty(b, s, h, dtype=torch.bfloat16).pin_memory()

        def e2e(i):
            y = step(xh[i % 4].to(dev, non_blocking=True))
            yh.copy_(y, non_blocking=True)

        for i in range(3):
            e2e(i)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(timed(e2e), ws, dev)

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, calls, el = _gqa_cpu_timed(wl, _gqa_cpu_setup(t, wl), args.cpu_seconds)
            cpu = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"1 of the {b} sequences ({s} block tokens over {ctx} context rows) per call, {calls} "
                             f"calls in {el:.1f} s; CPU restatement of "
                             f"{'Qwen3DSparkLayer.forward_cached' if layer_mode else 'Qwen3DSparkAttention.attend_cached'}"
                             f" in PyTorch with the bf16 weights before quantisation"}
        line = {
            "metric": LAYER_METRIC if layer_mode else GQA_METRIC, "value": ws * b * s / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 affine weights x bf16 activations (f16 MMA, fp32 accumulate); fp32 attention",
            "data": "synthetic",
            "config": {"workload": wl.name, "tokens_per_step_per_gpu": b * s, "batch": b, "draft_block": s,
                       "context_rows": ctx, "hidden": h, "heads": nh, "kv_heads": nkv, "head_dim": hd,
                       "attn_kernel": args.attn_kernel,
                       "parallelism": f"replicas{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (134 MB of cached K/V + "
                             f"{w_bytes / 1e6:.0f} MB of weights streamed every step)"},
            "hbm_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * b * s / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": xs[0].numel() * 2, "d2h_bytes_per_step": b * s * h * 2,
                "ms_per_step": e2e_ms},
            "gpu_launches": (LAYER_KERNELS_PER_STEP if layer_mode else GQA_KERNELS_PER_STEP) * args.steps,
            "clocks": clk.summary(),
            "launch": launch_note,
            "ms_per_step_eager": eager_ms,
        }
        print(json.dumps(line))


def run_reference_gqa(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    from dsm import workloads as W

    layer_mode = args.workload == "qwen3_layer_q8"
    wl = W.WORKLOADS[args.workload]
    t = (W.make_qwen3_layer_tensors if layer_mode else W.make_gqa_tensors)(wl, device="cpu")
    setup = _gqa_cpu_setup(t, wl)
    vals = []
    for i in range(args.warmup + args.steps):
        v, _, _ = _gqa_cpu_timed(wl, setup, 0.0, max_calls=1)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": LAYER_METRIC if layer_mode else GQA_METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wl.n_tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16 weights)",
        "data": "synthetic",
        "config": {"workload": wl.name, "tokens_per_step": wl.n_tokens, "batch": wl.batch, "draft_block": wl.block,
                   "context_rows": wl.extra["ctx"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"one sequence ({wl.block} block tokens over {wl.extra['ctx']} context rows) per "
                                   f"step; CPU restatement of "
                                   f"{'Qwen3DSparkLayer.forward_cached' if layer_mode else 'Qwen3DSparkAttention.attend_cached'}"
                                   f" in PyTorch (mlx is not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


DSATTN_METRIC = ("DeepSeek-V4 draft attention tokens/s (MLA decode of 7-token blocks over a full 128-slot window, "
                 "bf16); HBM GB/s")
# staging + product per projection (wq_a, wkv x2, wq_b, 8 wo_a groups, wo_b), 4 norm/RoPE
# kernels (main kv, q latents, q heads, block kv), window write, sparse attention, 2 casts
DSATTN_KERNELS_PER_STEP = 2 * 13 + 4 + 1 + 1 + 2


def _dsattn_cpu_setup(t, wl):
    import torch

    import oracle
    from oracle.attention_oracle import AttnDims

    torch.set_num_threads(os.cpu_count() or 1)
    a = wl.args
    p = {k: t[k].cpu() for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "q_norm", "kv_norm", "attn_sink")}
    dims = AttnDims(n_heads=a["n_heads"], head_dim=a["head_dim"], rope_head_dim=a["rope_head_dim"],
                    o_groups=a["o_groups"], o_lora_rank=a["o_lora_rank"], window_size=a["window_size"],
                    eps=a["norm_eps"])
    cos, sin = oracle.rope_tables(a["rope_head_dim"], wl.extra["max_seq_len"], a["rope_theta"])
    cache = oracle.KVWindow(a["window_size"])
    x, main = t["x"][:1].cpu(), t["main"][:1].cpu()
    oracle.attention_forward(p, dims, x, 0, t["prefill_main"][:1].cpu(), cache, cos, sin)
    return p, dims, x, main, cache, cos, sin


def _dsattn_cpu_timed(wl, setup, budget_s, max_calls=50):
    """The oracle's DSparkAttention decode step on one sequence per call, all host threads."""
    import oracle

    p, dims, x, main, cache, cos, sin = setup
    pos = wl.extra["prefill"]
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (n == 0 or time.perf_counter() - t0 < budget_s):
        oracle.attention_forward(p, dims, x, pos, main, cache, cos, sin)
        n += 1
    el = time.perf_counter() - t0
    return n * wl.block / el, n, el


def run_dsattn(args):
    """One step = one decode call of the DeepSeek draft attention: 8 sequences x 7-token
    blocks, each over its full 128-slot KV window. The projections (214 MB of bf16 weights)
    exceed L2, so every step streams them from HBM."""
    import torch

    from dsm import _lib, workloads as W

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    _lib.check(_lib.lib().dsm_set_attn_kernel(0 if args.attn_kernel == "mma" else 1), "dsm_set_attn_kernel")
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    wl = W.WORKLOADS["draft_attn_dsv4"]
    a = wl.args
    t = W.make_dsattn_tensors(wl, device=dev, seed=rank)
    attn = W.build_dsattn(wl, t, dev)
    b, s, pos = wl.batch, wl.block, wl.extra["prefill"]
    d, h, hd = a["dim"], a["n_heads"], a["head_dim"]
    attn(t["x"], 0, t["prefill_main"])  # seeds the window with the last 128 prefill positions
    gen = torch.Generator(device=dev)
    gen.manual_seed(333 + rank)
    xs = [t["x"]] + [torch.randn(t["x"].shape, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    mains = [t["main"]] + [torch.randn(t["main"].shape, generator=gen, device=dev).to(torch.bfloat16)
                           for _ in range(3)]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        attn(xs[i % 4], pos, mains[i % 4])
    torch.cuda.synchronize()

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            evs[i][0].record(stream)
            fn(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(x.elapsed_time(y) for x, y in evs) / args.steps

    _barrier(ws)
    launch_note = "eager calls"
    with ClockSampler(local) as clk:
        ms = timed(lambda i: attn(xs[i % 4], pos, mains[i % 4]))
        eager_ms = ms
        if not args.no_graph:
            gms, launch_note = graph_replay(lambda bb: attn(xs[bb], pos, mains[bb]), timed, args.warmup)
            ms = gms if gms is not None else ms
    ms = _max_over_ranks(ms, ws, dev)
    eager_ms = _max_over_ranks(eager_ms, ws, dev)
    w_bytes = sum(pm.nbytes for _, pm in attn._packed.values())
    win_bytes = b * a["window_size"] * hd * 2
    step_bytes = w_bytes + win_bytes + b * (2 * s + 1) * d * 2
    hbm_peak, _, peak_kind = _peaks()

    roofline = None
    if not args.no_kernel_timing and ws == 1:  # the largest projection alone: wq_b over the q latents
        L = _lib.lib()
        n = b * s
        pm = attn._pm("wq_b", attn.wq_b.weight)
        k = a["q_lora_rank"]
        cap = L.dsm_stage_rows_cap(n)
        xl = torch.randn(n, k, device=dev).to(torch.bfloat16)
        xsb = torch.empty(L.dsm_stage_bytes(cap, k), dtype=torch.uint8, device=dev)
        xsc = torch.empty(cap, dtype=torch.float32, device=dev)
        out = torch.empty(n, pm.rows, dtype=torch.float32, device=dev)
        sp = stream.cuda_stream
        _lib.check(L.dsm_stage_rows(xl.data_ptr(), _lib.DT_BF16, n, k, None, n, 1, xsb.data_ptr(), cap,
                                    xsc.data_ptr(), sp))
        k_ms = timed(lambda i: _lib.check(L.dsm_linear(xsb.data_ptr(), xsc.data_ptr(), cap, k, pm.wfmt, pm.group_size,
                                                       pm.packed.data_ptr(), pm.rows, out.data_ptr(), pm.rows, n, sp)))
        k_bytes = pm.nbytes + n * k * 2 + n * pm.rows * 4
        achieved = k_bytes / (k_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": "expert_tc_kernel<f16, down> (wq_b over 56 rows, tcgen05)",
                    "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                    "peak_kind": peak_kind, "frac_of_8tbs": achieved / SPEC_HBM_GBS,
                    "algorithmic_bytes_per_launch": k_bytes, "launch_ms": k_ms, "traffic": None}

    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        mh = [m.cpu().pin_memory() for m in mains]
        yh = torch.empty(b, s, d, dtype=torch.bfloat16).pin_memory()

        def e2e(i):
            y = attn(xh[i % 4].to(dev, non_blocking=True), pos, mh[i % 4].to(dev, non_blocking=True))
            yh.copy_(y, non_blocking=True)

        for i in range(3):
            e2e(i)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(timed(e2e), ws, dev)

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, calls, el = _dsattn_cpu_timed(wl, _dsattn_cpu_setup(t, wl), args.cpu_seconds)
            cpu = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"1 of the {b} sequences ({s} block tokens over a full window) per call, {calls} calls "
                             f"in {el:.1f} s; CPU restatement of DSparkAttention.__call__ in PyTorch"}
        line = {
            "metric": DSATTN_METRIC, "value": ws * b * s / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 weights x bf16 activations (f16 MMA, fp32 accumulate); fp32 attention",
            "data": "synthetic",
            "config": {"workload": wl.name, "tokens_per_step_per_gpu": b * s, "batch": b, "draft_block": s,
                       "dim": d, "heads": h, "head_dim": hd, "window": a["window_size"],
                       "attn_kernel": args.attn_kernel,
                       "parallelism": f"replicas{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (214 MB of projection weights streamed every step)"},
            "hbm_gbs_step": step_bytes / (ms * 1e-3) / 1e9,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * b * s / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": (xs[0].numel() + mains[0].numel()) * 2, "d2h_bytes_per_step": b * s * d * 2,
                "ms_per_step": e2e_ms},
            "gpu_launches": DSATTN_KERNELS_PER_STEP * args.steps,
            "clocks": clk.summary(),
            "launch": launch_note,
            "ms_per_step_eager": eager_ms,
        }
        print(json.dumps(line))


BLOCK_METRIC = ("DeepSeek-V4 DSpark draft-block latency (a middle stage: hyper-connections, MLA draft attention over "
                "a full 128-slot window, fp8 MoE; 8 sequences x 7-token blocks); tokens/s")
# two hyper-connection halves (pre+norm, post: 2 each), the attention's launches, the MoE's
BLOCK_KERNELS_PER_STEP = 2 * 2 + DSATTN_KERNELS_PER_STEP + KERNELS_PER_STEP


def _block_cpu_setup(t, wl):
    """The oracle's draft block on the first sequence: reference-named CPU tensors; the routed
    experts are read from the device and dequantised to fp32 on first use, i.e. in the
    untimed first call (the reference dequantises at load)."""
    import torch

    import oracle
    from oracle.attention_oracle import AttnDims

    torch.set_num_threads(os.cpu_count() or 1)
    a = wl.args

    class _Cached(oracle.OracleWeights):
        def __init__(self, codes, scales):
            super().__init__("fp8", codes, scales=scales)
            self._dense = {}

        def matrix(self, e):
            if e not in self._dense:
                self._dense[e] = oracle.fp8_weight_dequant(self.data[e].cpu(), self.scales[e].cpu())
            return self._dense[e]

    p = {k: t[f"attn_{k}"].cpu() for k in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "q_norm", "kv_norm", "attn_sink")}
    dims = AttnDims(n_heads=a["n_heads"], head_dim=a["head_dim"], rope_head_dim=a["rope_head_dim"],
                    o_groups=a["o_groups"], o_lora_rank=a["o_lora_rank"], window_size=a["window_size"],
                    eps=a["norm_eps"])
    cos, sin = oracle.rope_tables(a["rope_head_dim"], wl.extra["max_seq_len"], a["rope_theta"])
    cache = oracle.KVWindow(a["window_size"])
    oracle.attention_forward(p, dims, t["x"][:1, :, 0].cpu(), 0, t["attn_prefill_main"][:1].cpu(), cache, cos, sin)
    ffn = dict(gate_weight=t["moe_gate_weight"].cpu(), gate_bias=t["moe_gate_bias"].cpu(),
               topk=a["n_activated_experts"], score_func=a["score_func"], route_scale=a["route_scale"],
               swiglu_limit=a["swiglu_limit"],
               w1=_Cached(t["moe_w1_codes"], t["moe_w1_scale"]), w3=_Cached(t["moe_w3_codes"], t["moe_w3_scale"]),
               w2=_Cached(t["moe_w2_codes"], t["moe_w2_scale"]),
               shared=tuple(t[f"moe_shared_{n}"].cpu() for n in ("w1", "w2", "w3")))
    hc = dict(hc=a["hc_mult"], iters=a["hc_sinkhorn_iters"], norm_eps=a["norm_eps"], hc_eps=a["hc_eps"])
    halves = {h: dict(hc_fn=t[f"hc_{h}_fn"].cpu(), hc_scale=t[f"hc_{h}_scale"].cpu(),
                      hc_base=t[f"hc_{h}_base"].cpu(), norm_weight=t[f"norm_{h}"].cpu()) for h in ("attn", "ffn")}
    x, main = t["x"][:1].cpu(), t["attn_main"][:1].cpu()
    pos = wl.extra["prefill"]

    def call():
        y = oracle.ffn_sublayer(x, None, moe=lambda h, _i: oracle.attention_forward(p, dims, h, pos, main, cache,
                                                                                    cos, sin),
                                **halves["attn"], **hc)
        return oracle.ffn_sublayer(y, None, moe=lambda h, ids: oracle.moe_forward(h, ids, **ffn), **halves["ffn"], **hc)

    call()  # untimed: dequantises the experts this sequence routes to
    return call


def _block_cpu_timed(call, budget_s, max_calls=20):
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (n == 0 or time.perf_counter() - t0 < budget_s):
        call()
        n += 1
    el = time.perf_counter() - t0
    return n * 7 / el, n, el


def run_block(args):
    """One step = one decode call of a whole DeepSeek-V4 draft block (stage 1 of 3): 8
    sequences x 7-token blocks over 4 hyper-connection streams, the draft attention over a
    full window and the fp8 MoE. The step streams ~4 GB of weights, so every step reads them
    from HBM."""
    import torch

    from dsm import _lib, workloads as W

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    _lib.check(_lib.lib().dsm_set_attn_kernel(0 if args.attn_kernel == "mma" else 1), "dsm_set_attn_kernel")
    dev = torch.device("cuda", local)
    _init_dist(ws, dev)
    wl = W.WORKLOADS["draft_block_dsv4"]
    a = wl.args
    t = W.make_block_tensors(wl, device=dev, seed=rank)
    blk = W.build_block(wl, t, dev)
    b, s, pos, d, hc = wl.batch, wl.block, wl.extra["prefill"], a["dim"], a["hc_mult"]
    blk(t["x"], 0, None, t["attn_prefill_main"])  # seeds the window with the last 128 prefill positions
    gen = torch.Generator(device=dev)
    gen.manual_seed(444 + rank)
    xs = [t["x"]] + [torch.randn(t["x"].shape, generator=gen, device=dev).to(torch.bfloat16) for _ in range(3)]
    mains = [t["attn_main"]] + [torch.randn(t["attn_main"].shape, generator=gen, device=dev).to(torch.bfloat16)
                                for _ in range(3)]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        y = blk(xs[i % 4], pos, None, mains[i % 4])
    torch.cuda.synchronize()
    if not bool(torch.isfinite(y).all()) or _lib.device_error():
        raise RuntimeError("draft block: non-finite output or device error word set")

    def timed(fn):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            evs[i][0].record(stream)
            fn(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(x.elapsed_time(y) for x, y in evs) / args.steps

    _barrier(ws)
    launch_note = "eager calls"
    with ClockSampler(local) as clk:
        ms = timed(lambda i: blk(xs[i % 4], pos, None, mains[i % 4]))
        eager_ms = ms
        if not args.no_graph:
            gms, launch_note = graph_replay(lambda bb: blk(xs[bb], pos, None, mains[bb]), timed, args.warmup)
            ms = gms if gms is not None else ms
    ms = _max_over_ranks(ms, ws, dev)
    eager_ms = _max_over_ranks(eager_ms, ws, dev)

    e2e_ms = None
    if not args.no_e2e:
        xh = [x.cpu().pin_memory() for x in xs]
        mh = [m.cpu().pin_memory() for m in mains]
        yh = torch.empty(b, s, hc, d, dtype=torch.bfloat16).pin_memory()

        def e2e(i):
            y = blk(xh[i % 4].to(dev, non_blocking=True), pos, None, mh[i % 4].to(dev, non_blocking=True))
            yh.copy_(y, non_blocking=True)

        for i in range(3):
            e2e(i)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(timed(e2e), ws, dev)

    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            v, calls, el = _block_cpu_timed(_block_cpu_setup(t, wl), args.cpu_seconds)
            cpu = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"1 of the {b} sequences ({s} block tokens) per call, {calls} calls in {el:.1f} s; the "
                             f"experts it routes to dequantised to fp32 before timing; CPU restatement of "
                             f"DSparkBlock.__call__ in PyTorch"}
        line = {
            "metric": BLOCK_METRIC, "value": ws * b * s / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8 e4m3 experts, bf16 attention weights and activations (f16 MMA, fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": wl.name, "tokens_per_step_per_gpu": b * s, "batch": b, "draft_block": s,
                       "dim": d, "hc_mult": hc, "heads": a["n_heads"], "window": a["window_size"],
                       "n_experts": a["n_routed_experts"], "topk": a["n_activated_experts"], "weights": wl.wfmt,
                       "attn_kernel": args.attn_kernel, "parallelism": f"replicas{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (~4 GB of weights streamed every step)"},
            "draft_block_latency_ms": ms,
            "roofline": None,
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": ws * b * s / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": (xs[0].numel() + mains[0].numel()) * 2, "d2h_bytes_per_step": xs[0].numel() * 2,
                "ms_per_step": e2e_ms},
            "gpu_launches": BLOCK_KERNELS_PER_STEP * args.steps,
            "clocks": clk.summary(),
            "launch": launch_note,
            "ms_per_step_eager": eager_ms,
        }
        print(json.dumps(line))


def run_reference_dsattn(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    from dsm import workloads as W

    wl = W.WORKLOADS["draft_attn_dsv4"]
    t = W.make_dsattn_tensors(wl, device="cpu")
    setup = _dsattn_cpu_setup(t, wl)
    vals = []
    for i in range(args.warmup + args.steps):
        v, _, _ = _dsattn_cpu_timed(wl, setup, 0.0, max_calls=1)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": DSATTN_METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wl.n_tokens / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bf16 weights)",
        "data": "synthetic",
        "config": {"workload": wl.name, "tokens_per_step": wl.n_tokens, "batch": wl.batch, "draft_block": wl.block,
                   "window": wl.args["window_size"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": f"one sequence ({wl.block} block tokens over a full window) per step; CPU "
                                   f"restatement of DSparkAttention.__call__ in PyTorch (mlx is not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# The other single-GPU configurations, measured in the same process and run as the headline
# (fp8 decode) and carried in its line under "configs": the tiny hash-routed layer (latency),
# fp4 decode (448 tokens, Zipf 1.1), the Qwen3 q8 MLP and the 16384-token prefill.
SIDE_CONFIGS = ("tiny_hash", "fp4_decode", "qwen3_mlp_q8", "prefill_fp8")
# expert parallelism: fp4 decode (quoted at 1/2/4/8 GPUs) and the 16384-token prefill (quoted at
# 8 GPUs with its all-to-all GB/s and tensor-pipe figures)
SIDE_CONFIGS_EP = ("fp4_decode", "prefill_fp8")
CONFIG_KEYS = ("metric", "value", "unit", "ms_per_step", "higher_is_better", "dtype", "config", "hbm_gbs_step",
               "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks", "expert_parallel", "launch",
               "ms_per_step_eager")


def run_all(args):
    """The default run: the fp8 decode headline line, with every other configuration's numbers
    (value, roofline, CPU baseline, e2e, clocks) under ``configs``."""
    import torch

    ws, rank, _ = _dist()
    head = run_gpu(args, "fp8_decode", emit=False)
    configs = {}
    for name in (SIDE_CONFIGS if ws == 1 else SIDE_CONFIGS_EP):
        torch.cuda.empty_cache()
        line = run_qwen3(args, emit=False) if name.startswith("qwen3") else run_gpu(args, name, emit=False)
        if rank == 0:
            configs[name] = {k: line.get(k) for k in CONFIG_KEYS}
    if rank == 0:
        head["configs"] = configs
        print(json.dumps(head))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default=None,
                    help="one workload alone (default: fp8 decode with every other configuration under configs)")
    ap.add_argument("--impl", default="dsm", choices=["dsm", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-kernel-timing", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time eager calls only (no CUDA graph replay)")
    ap.add_argument("--experts", type=int, default=0, help="shrink the routed expert pool (profiling)")
    ap.add_argument("--tokens", type=int, default=0, help="override a MoE workload's tokens per call (profiling)")
    ap.add_argument("--attn-kernel", default="mma", choices=["cuda", "mma"],
                    help="attention workloads: CUDA-core kernels, or the tensor-core ones where they apply")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload is None:
        if args.impl == "reference":
            args.workload = "fp8_decode"
        else:
            try:
                run_all(args)
            finally:
                _finish_dist()
            return
    qwen3 = args.workload.startswith("qwen3")
    if args.workload == "draft_head":
        (run_reference_head if args.impl == "reference" else run_head)(args)
    elif args.workload in ("qwen3_attn_q8", "qwen3_layer_q8"):
        (run_reference_gqa if args.impl == "reference" else run_gqa)(args)
    elif args.workload == "draft_attn_dsv4":
        (run_reference_dsattn if args.impl == "reference" else run_dsattn)(args)
    elif args.workload == "draft_block_dsv4":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the whole-block reference arm is not separate: "
                              "the draft_block_dsv4 GPU line carries its own CPU baseline"}))
        else:
            run_block(args)
    elif args.impl == "reference":
        (run_reference_qwen3 if qwen3 else run_reference)(args)
    else:
        try:
            (run_qwen3 if qwen3 else run_gpu)(args)
        finally:
            _finish_dist()
        return
    _finish_dist()


if __name__ == "__main__":
    main()
