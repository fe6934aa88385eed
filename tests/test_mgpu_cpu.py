"""Multi-GPU host logic on CPU: shard helpers, and the sequence-split
orchestration (partial records -> all-gather -> log-sum-exp combine) run on
two gloo ranks with the FP64 oracle standing in for the device kernels."""
import os
import socket

import numpy as np
import pytest

import kvd_mgpu as mg


def test_batch_and_sequence_shards_cover_everything():
    for world in (1, 2, 3, 8):
        for n in (1, 7, 64, 1000):
            parts = [mg.batch_shard(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert max(h - l for l, h in parts) - min(h - l for l, h in parts) <= 1
        for S in (1, 1000, 131072):
            parts = [mg.seq_shard(S, world, r, align=128) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == S
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert all(l % 128 == 0 for l, _ in parts[1:] if l < S)


def test_lpt_balances_ragged_lengths():
    rng = np.random.default_rng(17)
    lens = rng.integers(256, 8193, size=128)
    for world in (2, 4, 8):
        groups = mg.lpt_assign(lens, world)
        assert sorted(b for g in groups for b in g) == list(range(128))
        loads = [int(lens[g].sum()) for g in groups]
        assert max(loads) - min(loads) <= int(lens.max())  # LPT bound
        assert max(loads) / (lens.sum() / world) < 1.02


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _records_from_oracle(part):
    """Oracle (natural-log m, l, o) rows -> the library's record layout
    (m in base-2 units, l, two unused slots, o)."""
    rec = np.zeros((part.shape[0], part.shape[1] + 2), np.float64)
    rec[:, 0] = part[:, 0] / np.log(2.0)
    rec[:, 1] = part[:, 1]
    rec[:, 4:] = part[:, 2:]
    return rec


def _seq_split_rank(rank, world, port, result):
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "cuda-operators_b200"), os.path.join(root, "oracle")]
    import kvd_mgpu
    import pyoracle as po

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, Hq, Hkv, S, D = 2, 4, 2, 700, 64
        q, K, V, ks, vs = po.random_cache(5, B, Hq, Hkv, S, D)  # identical on every rank
        lo, hi = kvd_mgpu.seq_shard(S, world, rank, align=128)

        def local_decode(q_, K_, V_, ks_, vs_, records, seq_lens=None):
            part = po.partials_f64(q, K, V, ks, vs, lo, hi)  # this rank's token shard
            records.copy_(torch.from_numpy(_records_from_oracle(part)).view(records.shape).float())

        def combine(parts, out):
            p = parts.double().numpy().copy()
            nat = np.concatenate([p[..., :1] * np.log(2.0), p[..., 1:2], p[..., 4:]], axis=-1)
            out.copy_(torch.from_numpy(po.combine_f64(nat)).float())

        dec = kvd_mgpu.SeqSplitDecode(B, Hq, D, "cpu", local_decode=local_decode, combine=combine)
        out = dec(torch.from_numpy(q), None, None, None, None)
        ref = po.decode_f64(q, K, V, ks, vs)
        result[rank] = float(np.abs(out.numpy() - ref).max())
    finally:
        dist.destroy_process_group()


def test_sequence_split_orchestration_on_two_gloo_ranks():
    import torch.multiprocessing as tmp

    ctx = tmp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_seq_split_rank, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert set(result.keys()) == {0, 1}
    assert max(result.values()) < 1e-5  # fp32 records, fp64 combine


def _dropout_rank(rank, world, port, result):
    import datetime
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "cuda-operators_b200"), os.path.join(root, "oracle")]
    import kvd_mgpu

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        result[1] = "left before the collective"
        os._exit(0)  # the rank disappears between steps, with nothing in flight
    dec = kvd_mgpu.SeqSplitDecode(1, 2, 8, "cpu", local_decode=lambda *a: None, combine=lambda parts, out: None)
    try:
        dec(torch.zeros(1, 2, 8), None, None, None, None)
        result[0] = "no error"
    except Exception as exc:  # the survivor must learn of it instead of hanging
        result[0] = f"error: {type(exc).__name__}"
    os._exit(0)


def test_rank_that_leaves_turns_into_an_error_not_a_hang():
    import time

    import torch.multiprocessing as tmp

    ctx = tmp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_rank, args=(r, 2, port, result)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        if p.is_alive():
            p.kill()
    assert time.time() - t0 < 90
    assert result.get(1) == "left before the collective"
    assert str(result.get(0, "")).startswith("error"), result.get(0)
