"""Benchmark of the INT8 KV-cache decode-attention path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C] [--only]

One step = one decode of a BASELINE configuration over a KV cache resident in
HBM. The headline (`value`) is configuration C (default 2: B=64, H=32, D=128,
S=4096, the Llama-7B-like MHA config the metric is quoted on); the same line
also carries every other configuration under `configs` (skipped with --only).
Caches of configurations 2-5 are 1.1-4.6 GB per step, far larger than the 126 MB
L2, so no flush is needed between steps; configuration 1 (1.1 MB) is
launch-latency bound and stays L2-resident, which its entry says.

Multi-GPU (torchrun, one rank per GPU): configurations 1, 2, 4 and 5 shard the
batch with no communication (weak scaling: every rank decodes a batch of the
configuration's size); configuration 3 splits the sequence across the ranks
and merges (m, l, o) records over NVLink (strong scaling: the job is one
configuration-3 step). Step times are CUDA-event times, max over ranks.

Printed: one JSON line (rank 0). `value` = aggregate algorithmic HBM GB/s;
`e2e` = the same metric through the reference-facing C ABI call with the
step's query copied from pinned host memory and the output copied back inside
the timed region (the cache is decode state and stays resident); `roofline` =
achieved / measured HBM copy bandwidth; `parity` = a sampled FP64 check of the
step's output (torch float64 on the device, at least 64 query rows);
`cpu_baseline` = the reference's fp32 host loop on the host cores for a sample
of heads; `reference_gpu` = the reference's own four kernels built for sm_100a,
timed with CUDA events on configurations 1-3 (outside the timed region).
`--impl reference` times the reference's host loop alone as the reference arm.
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
ATOL, RTOL = 2e-5, 1e-4  # output tolerance of the north-star spec
CPU_STEPS = 10           # timed host-loop steps in both arms (after one warm-up step)


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(config: int):
    """DRAM bytes per launch of the decode kernel from the committed ncu summary."""
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


def cpu_measure(cfg, heads: int, steps: int = CPU_STEPS, seed: int = 17) -> dict:
    """Times the reference fp32 host loop (oracle/_ref build when present, else
    the oracle's restatement) over a sample of heads on all host threads: one
    untimed warm-up step, then `steps` timed steps. Returns GB/s of the median
    step with the min/max spread."""
    import ctypes

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
        ref.kvref_cpu_run_parallel(arr, len(jobs))  # warm-up: first touch of every job's buffers
        for _ in range(steps):
            times.append(ref.kvref_cpu_run_parallel(arr, len(jobs)))
        for j in jobs:
            ref.kvref_cpu_free(j)
    else:
        kind = "port"
        po.cpu_reference_f32(q, K, V, ks, vs, heads, S, D, threads)
        for _ in range(steps):
            t0 = time.perf_counter()
            po.cpu_reference_f32(q, K, V, ks, vs, heads, S, D, threads)
            times.append(time.perf_counter() - t0)
    nbytes = heads * S * (2 * D + 8) + heads * D * 8
    sec = statistics.median(times)
    sample = (f"{heads} query heads x {S} tokens x D={D} of config {cfg.name} ({nbytes / 1e9:.3f} GB/step), "
              f"1 warm-up + median of {steps} steps, {threads} threads")
    return {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample,
            "ms_per_step": sec * 1e3, "min_gbs": nbytes / max(times) / 1e9, "max_gbs": nbytes / min(times) / 1e9,
            "steps": steps}


def run_reference(args) -> None:
    """Reference arm: the reference's own CPU implementation of the path."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import workload as wl

    cfg = wl.CONFIGS[args.config]
    steps = max(CPU_STEPS, min(args.steps, 30))  # bounded: the whole arm stays within a few minutes
    cb = cpu_measure(cfg, args.cpu_heads, steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": 1, "ms_per_step": cb["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) Q/K/V, K/V quantised per token",
        "config": {"workload": f"config{args.config} {cfg.name} (host sample)", "sample": cb["sample"]},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- parity
def _row_records_f64(case, b: int, hk: int, n: int, scale: float):
    """FP64 (m, l, o) of the G query heads of item (b, hk) over the first n tokens
    of this rank's cache (natural-log domain; o unnormalised)."""
    import torch

    cfg = case.cfg
    G, D = cfg.group, cfg.head_dim
    dev = case.q.device
    if n <= 0:
        return (torch.full((G,), float("-inf"), dtype=torch.float64, device=dev),
                torch.zeros(G, dtype=torch.float64, device=dev), torch.zeros(G, D, dtype=torch.float64, device=dev))
    q = case.q[b, hk * G:(hk + 1) * G].double()
    k = case.K[b, hk, :n].double() * case.ks[b, hk, :n, None].double()
    s = (q @ k.T) * scale
    m = s.max(dim=1).values
    p = torch.exp(s - m[:, None])
    v = case.V[b, hk, :n].double() * case.vs[b, hk, :n, None].double()
    return m, p.sum(dim=1), p @ v


def rounded_query(q):
    """The query as the INT8 Q.K mode sees it: each row rounded by the cache's
    quantiser rule (scale = max|q| / 127, code = clamp(rint(q / scale), -127, 127))."""
    import torch

    amax = q.abs().amax(dim=-1, keepdim=True)
    scale = amax / 127.0
    codes = torch.where(amax > 0, torch.clamp(torch.round(q / scale), -127, 127), torch.zeros_like(q))
    return codes * scale


def parity_check(case, out, lens, world: int, seqsplit: bool, qk_int8: bool = False) -> dict:
    """Compares sampled query rows of `out` with a float64 torch restatement of
    the decode (score = (q . code) * k_scale / sqrt(D), value = code * v_scale).
    Sequence split: every rank computes float64 (m, l, o) over its shard and the
    records are all-gathered and merged. With `qk_int8` the reference is the
    exact decode of the per-head rounded query (what that mode computes).
    Returns rows checked, bad elements, max abs and max normalised error (max
    over ranks)."""
    import math

    import torch
    import torch.distributed as dist

    import workload as wl

    cfg = case.cfg
    B = case.q.shape[0]
    G = cfg.group
    scale = 1.0 / math.sqrt(cfg.head_dim)
    items = wl.parity_items(cfg, B, lens)
    q_saved = case.q
    if qk_int8:
        case.q = rounded_query(case.q)
    m_l, l_l, o_l = [], [], []
    for b, hk in items:
        n = lens[b] if lens is not None else case.K.shape[2]
        m, l, o = _row_records_f64(case, b, hk, n, scale)
        m_l.append(m), l_l.append(l), o_l.append(o)
    case.q = q_saved
    M, L, O = torch.stack(m_l), torch.stack(l_l), torch.stack(o_l)  # [items, G], [items, G], [items, G, D]
    if seqsplit:
        rec = torch.cat([M[..., None], L[..., None], O], dim=-1).contiguous()
        allr = [torch.empty_like(rec) for _ in range(world)]
        dist.all_gather(allr, rec)
        allr = torch.stack(allr)
        Mx = allr[..., 0].max(dim=0).values
        f = torch.where(torch.isfinite(allr[..., 0]), torch.exp(allr[..., 0] - Mx), torch.zeros_like(allr[..., 0]))
        L = (f * allr[..., 1]).sum(dim=0)
        O = (f[..., None] * allr[..., 2:]).sum(dim=0)
    ref = torch.where(L[..., None] > 0, O / L.clamp_min(1e-300)[..., None], torch.zeros_like(O))
    got = torch.stack([out[b, hk * G:(hk + 1) * G].double() for b, hk in items])
    err = (got - ref).abs()
    bad_mask = (err > ATOL + RTOL * ref.abs()) | ~torch.isfinite(got)
    res = torch.tensor([float(bad_mask.sum().item()), float(err.nan_to_num(float("inf")).max().item()),
                        float((err / (ATOL + RTOL * ref.abs())).nan_to_num(float("inf")).max().item())],
                       dtype=torch.float64, device=case.q.device)
    if world > 1 and not seqsplit:  # every rank checked its own rows: total bad, worst error
        bad_t = res[:1].clone()
        dist.all_reduce(bad_t)
        mx = res[1:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        res = torch.cat([bad_t, mx])
    rows = len(items) * G * (world if world > 1 and not seqsplit else 1)
    return {"rows": rows, "bad": int(res[0].item()), "max_abs": res[1].item(), "max_norm": res[2].item(),
            "tol": f"|out - f64| <= {ATOL} + {RTOL}|f64|",
            "ref": "torch float64 on the device" + (", per-head int8-rounded query" if qk_int8 else "")}


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


class Env:
    """Process-group facts shared by every measurement."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device(f"cuda:{self.local}")
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=self.dev)
        self.comm = None   # library NCCL communicator (sequence split), made on first use
        self.args = args

    def library_comm(self):
        import torch
        import torch.distributed as dist

        import kvdecode as kvd

        if self.comm is None:
            uid = torch.zeros(128, dtype=torch.uint8, device=self.dev)
            if self.rank == 0:
                uid.copy_(torch.frombuffer(bytearray(kvd.mgpu_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            self.comm = kvd.MgpuComm(self.world, self.rank, bytes(uid.cpu().numpy().tobytes()))
        return self.comm

    def timed(self, fn, n: int, stream) -> float:
        """Milliseconds per call of fn over n calls: CUDA events on `stream`,
        barrier + synchronize on both sides, max over ranks."""
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        if self.world > 1:
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
        if self.world > 1:
            t = torch.tensor([ms], device=self.dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms


def measure_config(env: Env, cid: int, steps: int, warmup: int, batch: int = 0, paged: int = 0,
                   qk_int8: bool = False, head_shards: bool = False) -> dict:
    """Times configuration `cid` on this process group: device steps replayed
    from CUDA graphs, the end-to-end step through the C ABI with host buffers,
    then the sampled parity check. Frees the configuration's memory on return."""
    import dataclasses

    import torch

    import kvd_mgpu as mg
    import kvdecode as kvd
    import workload as wl

    args, world, rank, dev = env.args, env.world, env.rank, env.dev
    cfg = wl.CONFIGS[cid]
    B = batch or cfg.batch
    # Configuration 3 on N > 1 GPUs splits the sequence: rank g holds tokens
    # [g*S/N, (g+1)*S/N) of every head and the ranks merge (m, l, o) records
    # over NVLink (strong scaling). The others shard the batch (weak scaling).
    # head_shards: the comparison point for configuration 3 -- rank g owns
    # H/N heads of every sequence, whole, and nothing crosses NVLink (strong).
    if head_shards:
        cfg = dataclasses.replace(cfg, q_heads=cfg.q_heads // world, kv_heads=cfg.kv_heads // world)
    seqsplit = cfg.name == "long_context" and world > 1 and not head_shards
    exchange = None
    if seqsplit:
        lo, hi = mg.seq_shard(cfg.seq_len, world, rank, align=128)
        case = wl.make_case(dataclasses.replace(cfg, seq_len=hi - lo), seed=args.seed + rank, device=str(dev),
                            batch=B)
        job_bytes = wl.step_bytes(cfg, batch=B)
        nbytes = kvd.algorithmic_bytes(B, cfg.q_heads, cfg.kv_heads, cfg.head_dim, hi - lo)
        splitter = mg.SeqSplitDecode(B, cfg.q_heads, cfg.head_dim, dev)
        if args.exchange != "torch":
            comm = env.library_comm()
            if args.exchange == "p2p":
                exchange = kvd.P2PExchange(comm, B, cfg.q_heads, cfg.head_dim)
    else:
        case = wl.make_case(cfg, seed=args.seed + rank, device=str(dev), batch=B)
    out = torch.empty((B, cfg.q_heads, cfg.head_dim), dtype=torch.float32, device=dev)
    lens0 = case.seq_lens.clone() if cfg.ragged else None
    lens_final = [n + 1 for n in case.lens_host] if cfg.append else (case.lens_host if cfg.ragged else None)
    if not seqsplit:
        nbytes = wl.step_bytes(cfg, lens_final, batch=B)
        job_bytes = nbytes * world  # weak scaling, or the whole step when the heads are sharded
        if world > 1 and cfg.ragged:  # every rank draws its own lengths: add up the ranks' bytes
            import torch.distributed as dist

            t = torch.tensor([float(nbytes)], dtype=torch.float64, device=dev)
            dist.all_reduce(t)
            job_bytes = int(t.item())
    if paged and not seqsplit:
        pool = to_paged_pool(case, paged, cfg.kv_heads, cfg.head_dim, args.seed, dev)
        pdesc = kvd.make_paged_desc(case.q, pool["K"], pool["ks"], out, pool["table"], pool["lens"])
        ws = torch.empty(max(kvd.paged_workspace_size(pdesc), 1), dtype=torch.uint8, device=dev)
    else:
        pool = None
        desc = kvd.make_desc(case.q, case.K, case.ks, out, case.seq_lens)
        ws = torch.empty(max(kvd.workspace_size(desc), 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    if seqsplit and args.exchange == "nccl":
        import ctypes

        ws_split = torch.empty(int(kvd.lib().kvd_mgpu_seq_split_workspace_size(ctypes.byref(desc), world)),
                               dtype=torch.uint8, device=dev)

    def step():  # launches on the current stream (a capture stream while a graph is recorded)
        if seqsplit:
            if args.exchange == "p2p":
                exchange.decode(case.q, case.K, case.V, case.ks, case.vs, out=out)
            elif args.exchange == "nccl":
                kvd.seq_split_decode(env.comm, case.q, case.K, case.V, case.ks, case.vs, out=out, workspace=ws_split)
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
                                  out=out, workspace=ws, qk_int8=qk_int8)
                return
            kvd.append(case.k_new, case.v_new, case.K, case.V, case.ks, case.vs, case.seq_lens)
        kvd.decode(case.q, case.K, case.V, case.ks, case.vs, out=out, seq_lens=case.seq_lens, workspace=ws,
                   qk_int8=qk_int8)

    step()
    if seqsplit and args.exchange == "torch":  # this rank's partial decode, then the record combine
        splitter.local_decode(case.q, case.K, case.V, case.ks, case.vs, splitter.records)
        launches_per_step = kvd.last_launch_count() + 1
    elif seqsplit:  # the library call counts its own launches (decode + exchange/combine)
        launches_per_step = kvd.last_launch_count()
    else:
        separate = cfg.append and (args.separate_append or pool is not None)
        launches_per_step = kvd.last_launch_count() + (1 if separate else 0)
    for _ in range(warmup):
        step()

    # Decode steps are replayed from a CUDA graph (G steps per graph) so that
    # host launch overhead does not hide the device time of small configs. The
    # sequence split is captured with the peer-store exchange only (its kernel
    # counts epochs on the device); the NCCL and torch exchanges launch eagerly.
    graphable = not seqsplit or args.exchange == "p2p"
    G = 10 if steps % 10 == 0 and not args.no_graph and graphable else 1
    graphs = []
    if G > 1:
        graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            for _ in range(G):
                step()
        torch.cuda.synchronize()
        graph.replay()
        graphs.append(graph)
        run_steps = graph.replay
    else:
        run_steps = step

    with ClockSampler(env.local) as clk:
        ms = env.timed(run_steps, steps // G, stream) / G

    # ---- end to end through the reference-facing C ABI with host buffers
    q_host = case.q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    flat = not cfg.ragged and cfg.q_heads == cfg.kv_heads and not seqsplit and pool is None and not qk_int8
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

    for _ in range(max(3, warmup // 2)):
        e2e_step()
    # Replayed from a CUDA graph like the device-timed steps (the copies are in the graph),
    # so that host launch overhead does not stand in for the end-to-end time of small configs.
    run_e2e = e2e_step
    n_e2e = max(10, steps // 4)
    if G > 1 and world == 1:
        e2e_graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(e2e_graph):
            for _ in range(G):
                e2e_step()
        torch.cuda.synchronize()
        graphs.append(e2e_graph)
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
    e2e_ms = env.timed(run_e2e, n_e2e, stream) / G_e2e

    # ---- parity of one more step, outside the timed regions
    out.view(torch.int32).fill_(-1)
    step()
    torch.cuda.synchronize()
    parity = None
    if not args.no_parity:
        if pool is not None:  # the paged pools replaced the dense copy: check against a dense re-decode
            parity = {"rows": 0, "bad": 0, "note": "paged run: parity is covered by tests/test_paged.py"}
        else:
            parity = parity_check(case, out, lens_final, world, seqsplit, qk_int8)
    status = kvd.device_status()

    peak, peak_kind = measured_peak()
    # per GPU: the job's bytes over the ranks (a sequence split divides one step's bytes)
    per_gpu_gbs = job_bytes / world / (ms * 1e-3) / 1e9
    res = {
        "config": cid, "name": cfg.name,
        "workload": (f"config{cid} {cfg.name}: B={B}/GPU Hq={cfg.q_heads} Hkv={cfg.kv_heads} D={cfg.head_dim} "
                     f"S={cfg.seq_len}" + (" ragged+append" if cfg.ragged else "")
                     + (" INT8 Q.K mode (KVD_FLAG_QK_INT8)" if qk_int8 else "")
                     + (f" paged cache, {paged}-token blocks in random pool order" if pool else "")),
        "global_batch": B if (seqsplit or head_shards) else B * world, "seq_len": cfg.seq_len,
        "parallelism": (f"sequence split x{world}, (m, l, o) records exchanged "
                        + ("by peer stores + LSE combine in one kernel" if args.exchange == "p2p"
                           else "by NCCL all-gather + LSE combine")
                        if seqsplit else f"head shards x{world} ({cfg.q_heads} heads per GPU), no comm"
                        if head_shards else f"batch shards x{world}, no comm"),
        "scaling": "strong" if (seqsplit or head_shards) else "weak",
        "ms_per_step": ms, "us_per_step": ms * 1e3, "value": job_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "gbs_per_gpu": per_gpu_gbs, "pct_of_peak": 100.0 * per_gpu_gbs / peak,
        "bytes_per_step_per_gpu": nbytes,
        "l2": (f"no flush: {nbytes / 1e9:.2f} GB of cache read per step > 126 MB L2" if nbytes > 126e6 else
               f"L2-resident: {nbytes / 1e6:.2f} MB per step < 126 MB L2 (launch-latency bound, no flush)"),
        "roofline": {"bound": "hbm", "achieved": per_gpu_gbs, "peak": peak, "unit": "GB/s",
                     "frac": per_gpu_gbs / peak, "peak_source": f"{peak_kind} copy bandwidth",
                     "traffic": committed_traffic(cid)},
        "clocks": clk.summary(),
        "e2e": {"value": job_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "us_per_step": e2e_ms * 1e3,
                "launch": f"CUDA graph of {G_e2e} steps, copies included" if G_e2e > 1 else "direct launches",
                "h2d_bytes_per_step": int(q_host.numel() * 4), "d2h_bytes_per_step": int(out_host.numel() * 4),
                "call": ("kv_int8_split_launch" if flat else "kvd_paged_decode_launch" if pool is not None
                         else "kvd_mgpu_p2p_seq_split_decode" if seqsplit and args.exchange == "p2p"
                         else "kvd_mgpu_seq_split_decode" if seqsplit and args.exchange == "nccl"
                         else "kvd_append_decode_launch" if cfg.append and not args.separate_append
                         else "kvd_decode_launch")},
        "parity": parity, "device_status": status,
        "launches_per_step": launches_per_step, "gpu_launches": launches_per_step * steps,
        "launch": f"CUDA graph of {G} steps" if G > 1 else "direct launches", "steps": steps,
    }
    # release everything this configuration holds before the next one is built
    torch.cuda.synchronize()
    del graphs
    if exchange is not None:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()  # no rank unmaps its exchange buffers while a peer could still write them
        exchange.close()
    del case, out, ws
    torch.cuda.empty_cache()
    return res


def reference_gpu(steps: int) -> dict:
    """The reference's own kernels (kv_cache/*.cu built for sm_100a into
    oracle/_ref by oracle/Makefile) on configurations 1-3 in their flat [H, S, D]
    layout: `solve` of KV_int8.cu and KV_int8_single_buffer.cu (default stream),
    kv_int8_split_launch of KV_int8_split_optimized.cu and kv_int8_simple_launch
    of new_kvint8.cu (caller scratch, so no allocation is timed). CUDA events
    around `steps` calls after one warm-up call. Each output is compared with
    this library's decode of the same inputs (max abs difference)."""
    import ctypes

    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    import kvdecode as kvd
    import pyoracle as po
    import workload as wl

    libs = {name: po.ref_lib(name) for name in ("tiled", "single", "split", "simple")}
    if any(v is None for v in libs.values()):
        return {"unavailable": "oracle/_ref was not built (the reference checkout was absent at build time)"}
    res = {}
    for cid in (1, 2, 3):
        cfg = wl.CONFIGS[cid]
        case = wl.make_case(cfg, seed=17, device="cuda")
        H, S, D = cfg.batch * cfg.q_heads, cfg.seq_len, cfg.head_dim
        ours = kvd.decode(case.q, case.K, case.V, case.ks, case.vs)
        scratch = torch.empty(H * S, dtype=torch.float32, device="cuda")
        out = torch.empty((H, D), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream()
        ptrs = [case.q.data_ptr(), case.K.data_ptr(), case.V.data_ptr(), case.ks.data_ptr(), case.vs.data_ptr(),
                out.data_ptr()]
        calls = {
            "tiled_solve": lambda: libs["tiled"].kvref_tiled_solve(*ptrs, H, S, D),
            "single_buffer_solve": lambda: libs["single"].kvref_single_solve(*ptrs, H, S, D),
            "split_launch": lambda: libs["split"].kvref_split_launch(*ptrs, H, S, D, scratch.data_ptr(),
                                                                    ctypes.c_void_p(stream.cuda_stream)),
            "simple_launch": lambda: libs["simple"].kvref_simple_launch(*ptrs, H, S, D, scratch.data_ptr(),
                                                                       ctypes.c_void_p(stream.cuda_stream)),
        }
        nbytes = kvd.algorithmic_bytes(cfg.batch, cfg.q_heads, cfg.kv_heads, D, S)
        row = {}
        for name, fn in calls.items():
            out.fill_(float("nan"))
            fn()
            torch.cuda.synchronize()
            diff = (out.view(cfg.batch, cfg.q_heads, D) - ours).abs().max().item()
            reps = steps if cid < 3 else max(1, steps // 2)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            row[name] = {"us_per_step": us, "gbs": nbytes / (us * 1e-6) / 1e9, "max_abs_vs_ours": diff,
                         "steps": reps}
        best = min(row, key=lambda k: row[k]["us_per_step"])
        res[str(cid)] = {"variants": row, "best": best, "best_us_per_step": row[best]["us_per_step"]}
        del case, scratch, out, ours
        torch.cuda.empty_cache()
    res["how"] = "CUDA events, 1 warm-up + 5 calls (config 3: 2), same seeded inputs as this bench"
    return res


def run_ours(args) -> None:
    import torch

    env = Env(args)
    world, rank = env.world, env.rank
    head = measure_config(env, args.config, args.steps, args.warmup, batch=args.batch, paged=args.paged,
                          qk_int8=args.qk_int8)
    configs = {}
    if not args.only:
        for cid in (1, 2, 3, 4, 5):
            if cid != args.config:
                configs[str(cid)] = measure_config(env, cid, args.steps, args.warmup)
        # the INT8 Q.K mode on the grouped-query configuration (a looser, stated tolerance)
        configs["5_qk_int8"] = measure_config(env, 5, args.steps, args.warmup, qk_int8=True)
        if world > 1 and 32 % world == 0:  # configuration 3 sharded by heads: the no-communication comparison
            configs["3_head_shards"] = measure_config(env, 3, args.steps, args.warmup, head_shards=True)
    peak, peak_kind = measured_peak()
    line = {
        "metric": METRIC, "value": head["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "us_per_step": head["us_per_step"],
        "pct_of_peak": head["pct_of_peak"], "higher_is_better": True, "scaling": head["scaling"],
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) Q/K/V (torch Philox on device), K/V quantised per token by the library",
        "config": {"workload": head["workload"], "global_batch": head["global_batch"], "seq_len": head["seq_len"],
                   "parallelism": head["parallelism"], "bytes_per_step_per_gpu": head["bytes_per_step_per_gpu"],
                   "l2": head["l2"]},
        "roofline": dict(head["roofline"], timed=(
            "decode step: tcgen05 kernel gqa_tc_kernel" if wl_head_dim(args.config) == 128
            else "decode step: CUDA-core decode kernel")),
        "clocks": head["clocks"], "e2e": head["e2e"], "parity": head["parity"],
        "gpu_launches": head["gpu_launches"], "launch": head["launch"],
    }
    if configs:
        line["configs"] = {cid: {k: v for k, v in c.items() if k not in ("steps",)} for cid, c in configs.items()}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        import workload as wl

        line["cpu_baseline"] = cpu_measure(wl.CONFIGS[args.config], args.cpu_heads)
    if world == 1 and rank == 0 and not args.only and not args.no_reference_gpu:
        line["reference_gpu"] = reference_gpu(5)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier()
        if env.comm is not None:
            env.comm.close()
        dist.destroy_process_group()


def wl_head_dim(cid: int) -> int:
    import workload as wl

    return wl.CONFIGS[cid].head_dim


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
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5], help="headline configuration")
    ap.add_argument("--only", action="store_true", help="measure the headline configuration alone")
    ap.add_argument("--qk-int8", action="store_true", help="headline in the INT8 Q.K mode (KVD_FLAG_QK_INT8)")
    ap.add_argument("--seed", type=int, default=17)
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch override (profiling small cases; implies --only)")
    ap.add_argument("--cpu-heads", type=int, default=512, help="query heads in the CPU sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true", help="skip timing the reference's own GPU kernels")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled FP64 check after the timed region")
    ap.add_argument("--no-graph", action="store_true", help="launch every step directly instead of from a CUDA graph")
    ap.add_argument("--exchange", choices=["p2p", "nccl", "torch"], default="p2p",
                    help="config 3 on N>1 GPUs: record exchange by peer stores (p2p), the library's NCCL call, "
                         "or torch.distributed all_gather")
    ap.add_argument("--separate-append", action="store_true",
                    help="config 4: append kernel then decode (default: one fused append+decode launch)")
    ap.add_argument("--paged", type=int, default=0, metavar="BS",
                    help="decode through the paged-cache entry point with BS-token blocks (0: dense cache; implies --only)")
    ap.add_argument("--prefill", default="", metavar="B,HQ,HKV,L,LQ",
                    help="time the causal prefill kernel on this shape instead (a side measurement)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.batch or args.paged:
        args.only = True
    if args.prefill:
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
