"""Benchmark of the INT8 KV-cache decode-attention path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]

One step = one decode of configuration C (default 2: B=64, H=32, D=128,
S=4096, the Llama-7B-like MHA config the headline metric is quoted on) over
a KV cache resident in HBM. The cache is 2.2 GB per step, far larger than the
126 MB L2, so no flush is needed between steps. Multi-GPU (torchrun, one rank
per GPU): every rank decodes its own batch shard with no communication (weak
scaling: per-GPU work fixed, global batch = B*N); the step time is the max over
ranks of CUDA-event time.

Printed: one JSON line (rank 0). `value` = aggregate algorithmic HBM GB/s;
`e2e` = the same metric through the reference-facing C ABI call
(kv_int8_split_launch) with the step's query copied from pinned host memory
and the output copied back inside the timed region (the cache is decode state
and stays resident); `roofline` = achieved / measured HBM copy bandwidth;
`cpu_baseline` = the reference's fp32 host loop on the host cores for a sample
of heads. `--impl reference` times that host loop alone as the reference arm.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cuda-operators_b200"))

METRIC = "INT8 KV decode attn: achieved HBM GB/s (% peak), µs/step at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(config: int):
    """DRAM bytes per launch of the split-KV kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    try:
        return json.loads(path.read_text()).get(f"config{config}", {}).get("dram_bytes_per_step")
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the GPU works."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period: float = 0.02):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- CPU legs
def _cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(cfg, heads: int, seed: int):
    """Host copy of `heads` query heads (each with its own KV rows) of the
    configuration, quantised per token by the oracle quantiser."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle as po

    S, D = cfg.seq_len, cfg.head_dim
    if cfg.ragged:
        S = (cfg.ragged[0] + cfg.ragged[1]) // 2
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((heads, D), dtype=np.float32)
    K = np.empty((heads, S, D), np.int8)
    V = np.empty((heads, S, D), np.int8)
    ks = np.empty((heads, S), np.float32)
    vs = np.empty((heads, S), np.float32)
    for h0 in range(0, heads, 32):
        h1 = min(heads, h0 + 32)
        K[h0:h1], ks[h0:h1] = po.quantize_rows(rng.standard_normal((h1 - h0, S, D), dtype=np.float32))
        V[h0:h1], vs[h0:h1] = po.quantize_rows(rng.standard_normal((h1 - h0, S, D), dtype=np.float32))
    return q, K, V, ks, vs, S


def cpu_measure(cfg, heads: int, steps: int, seed: int = 17):
    """Times the reference fp32 host loop (oracle/_ref build when present, else
    the oracle's restatement) over a sample of heads on all host threads.
    Returns (GB/s, seconds per step, kind, threads, sample description)."""
    import ctypes

    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle as po

    q, K, V, ks, vs, S = cpu_sample(cfg, heads, seed)
    D = cfg.head_dim
    threads = min(_cpu_threads(), heads)
    ref = po.ref_lib("split")
    times = []
    if ref is not None:
        kind = "reference"
        bounds = [round(i * heads / threads) for i in range(threads + 1)]
        jobs = [ref.kvref_cpu_prepare(q[a:b].ctypes.data, K[a:b].ctypes.data, V[a:b].ctypes.data,
                                      ks[a:b].ctypes.data, vs[a:b].ctypes.data, b - a, S, D)
                for a, b in zip(bounds[:-1], bounds[1:])]
        arr = (ctypes.c_void_p * len(jobs))(*jobs)
        for _ in range(steps):
            times.append(ref.kvref_cpu_run_parallel(arr, len(jobs)))
        for j in jobs:
            ref.kvref_cpu_free(j)
    else:
        kind = "port"
        for _ in range(steps):
            t0 = time.perf_counter()
            po.cpu_reference_f32(q, K, V, ks, vs, heads, S, D, threads)
            times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    nbytes = heads * S * (2 * D + 8) + heads * D * 8
    sample = (f"{heads} query heads x {S} tokens x D={D} of config {cfg.name} "
              f"({nbytes / 1e9:.3f} GB/step), median of {steps} steps, {threads} threads")
    return nbytes / sec / 1e9, sec, kind, threads, sample


def run_reference(args) -> None:
    """Reference arm: the reference's own CPU implementation of the path."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import workload as wl

    cfg = wl.CONFIGS[args.config]
    steps = max(1, min(args.steps, 30))  # bounded: the whole arm stays within a few minutes
    gbs, sec, kind, threads, sample = cpu_measure(cfg, args.cpu_heads, steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) Q/K/V, K/V quantised per token",
        "config": {"workload": f"config{args.config} {cfg.name} (host sample)", "sample": sample},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU leg
def to_paged_pool(case, bs: int, Hkv: int, D: int, seed: int, dev):
    """Moves the case's dense cache into block pools [blocks, Hkv, bs, D] in a
    seeded random block order; returns the pools, the block table and the
    lengths (every sequence at its dense length when the case is not ragged)."""
    import torch

    B, _, cap, _ = case.K.shape
    nb = -(-cap // bs)
    pad = nb * bs - cap
    g = torch.Generator(device="cpu").manual_seed(seed)
    table = torch.randperm(B * nb, generator=g).to(torch.int32).view(B, nb).to(dev)
    idx = table.flatten().long()
    pool = {"table": table}
    for name in ("K", "V", "ks", "vs"):
        x = getattr(case, name)
        if pad:
            x = torch.nn.functional.pad(x, ((0, 0, 0, pad) if x.dim() == 4 else (0, pad)))
        if x.dim() == 4:
            blocks = x.view(B, Hkv, nb, bs, D).permute(0, 2, 1, 3, 4).reshape(B * nb, Hkv, bs, D)
        else:
            blocks = x.view(B, Hkv, nb, bs).permute(0, 2, 1, 3).reshape(B * nb, Hkv, bs)
        p = torch.empty_like(blocks)
        p[idx] = blocks
        pool[name] = p
        setattr(case, name, None)  # free the dense copy
    pool["lens"] = (case.seq_lens.clone() if case.seq_lens is not None
                    else torch.full((B,), cap, dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    return pool


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import kvdecode as kvd
    import workload as wl

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    cfg = wl.CONFIGS[args.config]
    B = args.batch or cfg.batch
    # Configuration 3 on N > 1 GPUs splits the sequence: rank g holds tokens
    # [g*S/N, (g+1)*S/N) of every head and the ranks merge (m, l, o) records
    # over NCCL (strong scaling: the job is one configuration-3 step). The other
    # configurations shard the batch with no communication (weak scaling).
    seqsplit = cfg.name == "long_context" and world > 1
    comm = exchange = None
    if seqsplit:
        import dataclasses

        import kvd_mgpu as mg

        lo, hi = mg.seq_shard(cfg.seq_len, world, rank, align=128)
        case = wl.make_case(dataclasses.replace(cfg, seq_len=hi - lo), seed=args.seed + rank, device=str(dev),
                            batch=B)
        job_bytes = wl.step_bytes(cfg, batch=B)
        nbytes = kvd.algorithmic_bytes(B, cfg.q_heads, cfg.kv_heads, cfg.head_dim, hi - lo)
        splitter = mg.SeqSplitDecode(B, cfg.q_heads, cfg.head_dim, dev)
        if args.exchange != "torch":  # a communicator made by the library, its id broadcast by torch
            uid = torch.zeros(128, dtype=torch.uint8, device=dev)
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(kvd.mgpu_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            comm = kvd.MgpuComm(world, rank, bytes(uid.cpu().numpy().tobytes()))
            if args.exchange == "p2p":
                exchange = kvd.P2PExchange(comm, B, cfg.q_heads, cfg.head_dim)
    else:
        case = wl.make_case(cfg, seed=args.seed + rank, device=str(dev), batch=B)
    out = torch.empty((B, cfg.q_heads, cfg.head_dim), dtype=torch.float32, device=dev)
    lens0 = case.seq_lens.clone() if cfg.ragged else None
    lens_final = [n + 1 for n in case.lens_host] if cfg.append else case.lens_host
    if not seqsplit:
        nbytes = wl.step_bytes(cfg, lens_final if cfg.ragged else None, batch=B)
        job_bytes = nbytes * world
    if args.paged and not seqsplit:
        pool = to_paged_pool(case, args.paged, cfg.kv_heads, cfg.head_dim, args.seed, dev)
        pdesc = kvd.make_paged_desc(case.q, pool["K"], pool["ks"], out, pool["table"], pool["lens"])
        ws = torch.empty(max(kvd.paged_workspace_size(pdesc), 1), dtype=torch.uint8, device=dev)
    else:
        pool = None
        desc = kvd.make_desc(case.q, case.K, case.ks, out, case.seq_lens)
        ws = torch.empty(max(kvd.workspace_size(desc), 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    if seqsplit and args.exchange == "nccl":
        ws_split = torch.empty(int(kvd.lib().kvd_mgpu_seq_split_workspace_size(__import__("ctypes").byref(desc),
                                                                            world)), dtype=torch.uint8, device=dev)

    def step():  # launches on the current stream (a capture stream while a graph is recorded)
        if seqsplit:
            if args.exchange == "p2p":
                exchange.decode(case.q, case.K, case.V, case.ks, case.vs, out=out)
            elif args.exchange == "nccl":
                kvd.seq_split_decode(comm, case.q, case.K, case.V, case.ks, case.vs, out=out, workspace=ws_split)
            else:
                splitter(case.q, case.K, case.V, case.ks, case.vs, out=out)
            return
        if pool is not None:
            if cfg.append:
                pool["lens"].copy_(lens0)
                kvd.paged_append(case.k_new, case.v_new, pool["K"], pool["V"], pool["ks"], pool["vs"],
                                 pool["table"], pool["lens"])
            kvd.paged_decode(case.q, pool["K"], pool["V"], pool["ks"], pool["vs"], pool["table"], pool["lens"],
                             out=out, workspace=ws)
            return
        if cfg.append:
            case.seq_lens.copy_(lens0)  # every step appends at the same positions
            if not args.separate_append:  # quantise-on-append inside the decode launch
                kvd.append_decode(case.k_new, case.v_new, case.q, case.K, case.V, case.ks, case.vs, case.seq_lens,
                                  out=out, workspace=ws)
                return
            kvd.append(case.k_new, case.v_new, case.K, case.V, case.ks, case.vs, case.seq_lens)
        kvd.decode(case.q, case.K, case.V, case.ks, case.vs, out=out, seq_lens=case.seq_lens, workspace=ws)

    step()
    if seqsplit and args.exchange == "torch":  # this rank's partial decode, then the record combine
        splitter.local_decode(case.q, case.K, case.V, case.ks, case.vs, splitter.records)
        launches_per_step = kvd.last_launch_count() + 1
    elif seqsplit:  # the library call counts its own launches (decode + exchange/combine)
        launches_per_step = kvd.last_launch_count()
    else:
        separate = cfg.append and (args.separate_append or pool is not None)
        launches_per_step = kvd.last_launch_count() + (1 if separate else 0)
    for _ in range(args.warmup):
        step()

    # Decode steps are replayed from a CUDA graph (G steps per graph) so that
    # host launch overhead does not hide the device time of small configs. The
    # sequence split is captured with the peer-store exchange only (its kernel
    # counts epochs on the device); the NCCL and torch exchanges launch eagerly.
    graphable = not seqsplit or args.exchange == "p2p"
    G = 10 if args.steps % 10 == 0 and not args.no_graph and graphable else 1
    if G > 1:
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            for _ in range(G):
                step()
        torch.cuda.synchronize()
        graph.replay()
        run_steps = graph.replay
    else:
        run_steps = step

    def timed(fn, n):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(local) as clk:
        ms = timed(run_steps, args.steps // G) / G

    # ---- end to end through the reference-facing C ABI with host buffers
    q_host = case.q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    flat = not cfg.ragged and cfg.q_heads == cfg.kv_heads and not seqsplit and pool is None
    if flat:
        H = B * cfg.q_heads
        scratch = torch.empty(H * cfg.seq_len, dtype=torch.float32, device=dev)

    def e2e_step():
        case.q.copy_(q_host, non_blocking=True)
        if flat:
            rc = kvd.kv_int8_split_launch(case.q, case.K, case.V, case.ks, case.vs, out, H, cfg.seq_len,
                                          cfg.head_dim, scratch, torch.cuda.current_stream())  # the capture stream
            if rc != 0:
                raise RuntimeError(f"kv_int8_split_launch returned {rc}")
        else:
            step()
        out_host.copy_(out, non_blocking=True)

    for _ in range(max(3, args.warmup // 2)):
        e2e_step()
    # Replayed from a CUDA graph like the device-timed steps (the copies are in the graph),
    # so that host launch overhead does not stand in for the end-to-end time of small configs.
    run_e2e = e2e_step
    n_e2e = max(10, args.steps // 4)
    if G > 1 and world == 1:
        e2e_graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(e2e_graph):
            for _ in range(G):
                e2e_step()
        torch.cuda.synchronize()
        # the replayed steps must recompute the output: clear it, replay, compare
        expect = out_host.clone()
        out.zero_()
        out_host.zero_()
        e2e_graph.replay()
        torch.cuda.synchronize()
        if not torch.equal(out_host, expect):
            raise RuntimeError("the end-to-end graph does not reproduce the step's output")
        run_e2e = e2e_graph.replay
        n_e2e = max(1, n_e2e // G)
    G_e2e = G if run_e2e is not e2e_step else 1
    e2e_ms = timed(run_e2e, n_e2e) / G_e2e

    peak, peak_kind = measured_peak()
    per_gpu_gbs = nbytes / (ms * 1e-3) / 1e9
    agg_gbs = job_bytes / (ms * 1e-3) / 1e9
    e2e_gbs = job_bytes / (e2e_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": agg_gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "us_per_step": ms * 1e3,
        "pct_of_peak": 100.0 * per_gpu_gbs / peak, "higher_is_better": True,
        "scaling": "strong" if seqsplit else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) Q/K/V (torch Philox on device), K/V quantised per token by the library",
        "config": {
            "workload": (f"config{args.config} {cfg.name}: B={B}/GPU Hq={cfg.q_heads} Hkv={cfg.kv_heads} "
                         f"D={cfg.head_dim} S={cfg.seq_len}" + (" ragged+append" if cfg.ragged else "")
                         + (f" paged cache, {args.paged}-token blocks in random pool order" if pool else "")),
            "global_batch": B if seqsplit else B * world, "seq_len": cfg.seq_len,
            "parallelism": (f"sequence split x{world}, (m, l, o) records exchanged "
                            + ("by peer stores + LSE combine in one kernel" if args.exchange == "p2p"
                               else "by NCCL all-gather + LSE combine")
                            if seqsplit else f"batch shards x{world}, no comm"),
            "bytes_per_step_per_gpu": nbytes,
            "l2": f"no flush: {nbytes / 1e9:.2f} GB of cache read per step > 126 MB L2",
        },
        "roofline": {"bound": "hbm", "achieved": per_gpu_gbs, "peak": peak, "unit": "GB/s",
                     "frac": per_gpu_gbs / peak, "peak_source": f"{peak_kind} copy bandwidth",
                     "traffic": committed_traffic(args.config),
                     "timed": ("decode step: tcgen05 kernel gqa_tc_kernel" if cfg.head_dim == 128
                               else "decode step: CUDA-core split-KV kernel + boundary combine")
                              + ((" + record exchange over NVLink peer stores and LSE combine in one kernel"
                                  if args.exchange == "p2p" else " + NCCL record all-gather + LSE combine")
                                 if seqsplit else "")
                              + ((" with the append fused into it" if not (args.separate_append or pool is not None)
                                  else " after the append kernel") if cfg.append else "")},
        "clocks": clk.summary(),
        "e2e": {"value": e2e_gbs, "unit": "GB/s", "ms_per_step": e2e_ms,
                "launch": f"CUDA graph of {G_e2e} steps, copies included" if G_e2e > 1 else "direct launches",
                "h2d_bytes_per_step": int(q_host.numel() * 4), "d2h_bytes_per_step": int(out_host.numel() * 4),
                "call": ("kv_int8_split_launch" if flat else
                         "kvd_paged_decode_launch" if pool is not None else "kvd_decode_launch")},
        "gpu_launches": launches_per_step * args.steps,
        "launch": f"CUDA graph of {G} steps" if G > 1 else "direct launches",
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        gbs, sec, kind, threads, sample = cpu_measure(cfg, args.cpu_heads, 3)
        line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps its exchange buffers while a peer could still write them
        if exchange is not None:
            exchange.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def run_prefill(args) -> None:
    """Side measurement (not the headline): causal prefill over an INT8 cache.
    --prefill B,Hq,Hkv,L,Lq: B sequences of L cached tokens whose last Lq are
    the queries; fp32 Q and output; seeded random codes and scales. Prints one
    JSON line with attention TFLOP/s (4*D FLOPs per visible query-token pair;
    the MMAs do twice that, hi + lo operands)."""
    import torch
    import kvdecode as kvd

    B, Hq, Hkv, L, Lq = (int(x) for x in args.prefill.split(","))
    D = 128
    dev = "cuda:0"
    g = torch.Generator(device=dev).manual_seed(args.seed)
    K = torch.randint(-127, 128, (B, Hkv, L, D), dtype=torch.int8, device=dev, generator=g)
    V = torch.randint(-127, 128, (B, Hkv, L, D), dtype=torch.int8, device=dev, generator=g)
    ks = torch.rand(B, Hkv, L, device=dev, generator=g) * 0.02
    vs = torch.rand(B, Hkv, L, device=dev, generator=g) * 0.02
    q = torch.randn(B, Hq, Lq, D, device=dev, generator=g)
    out = torch.empty(B, Hq, Lq, D, device=dev)
    for _ in range(args.warmup):
        kvd.prefill(q, K, V, ks, vs, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        kvd.prefill(q, K, V, ks, vs, out=out)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) / args.steps * 1e3
    if kvd.device_status() != kvd.KVD_STATUS_OK:
        raise RuntimeError("prefill kernel reported a bad status")
    pairs = B * Hq * (Lq * (L - Lq) + Lq * (Lq + 1) / 2)
    print(json.dumps({"metric": "INT8 KV causal prefill: attention TFLOP/s", "value": pairs * D * 4 / us / 1e6,
                      "unit": "TFLOP/s", "us_per_step": us, "steps": args.steps, "warmup": args.warmup,
                      "dtype": "f32 in, bf16 hi+lo MMA operands, f32 accumulate", "data": "synthetic",
                      "config": {"workload": "prefill", "batch": B, "q_heads": Hq, "kv_heads": Hkv,
                                 "cache_tokens": L, "queries": Lq, "head_dim": D}}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--seed", type=int, default=17)
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch override (profiling small cases)")
    ap.add_argument("--cpu-heads", type=int, default=512, help="query heads in the CPU sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step directly instead of from a CUDA graph")
    ap.add_argument("--exchange", choices=["p2p", "nccl", "torch"], default="p2p",
                    help="config 3 on N>1 GPUs: record exchange by peer stores (p2p), the library's NCCL call, "
                         "or torch.distributed all_gather")
    ap.add_argument("--separate-append", action="store_true",
                    help="config 4: append kernel then decode (default: one fused append+decode launch)")
    ap.add_argument("--paged", type=int, default=0, metavar="BS",
                    help="decode through the paged-cache entry point with BS-token blocks (0: dense cache)")
    ap.add_argument("--prefill", default="", metavar="B,HQ,HKV,L,LQ",
                    help="time the causal prefill kernel on this shape instead (a side measurement)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.prefill:
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
