"""GPU tests of the single-process sequence split (kvd_mgpu_p2p_create_group):
one process drives every rank's GPU, and the exchange kernel links the ranks by
direct peer pointers.

On ONE GPU (what a one-GPU box can run): a group of two ranks placed on the
same device where only rank 0 ever calls -- rank 1's records never arrive, so rank 0's bounded wait must run out, record KVD_STATUS_WAIT_TIMEOUT
and return within seconds, and the CUDA context must stay usable (a decode
right after matches the FP64 oracle). Only one waiting kernel runs. On two
GPUs: the ranks' steps, launched from this thread on one stream per GPU, must
merge into the FP64 oracle's output on both ranks, over several epochs and
after a reset. A one-rank group runs the whole exchange kernel on one GPU."""
import time

import numpy as np
import pytest
import torch

import kvd_mgpu as mg
import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu


def _shard(a, lo, hi, dev):
    return torch.from_numpy(np.ascontiguousarray(a[:, :, lo:hi])).to(dev)


def test_group_exchange_times_out_when_a_rank_never_calls():
    B, Hq, S = 2, 8, 2048
    q, K, V, ks, vs = po.random_cache(71, B, Hq, Hq, S, 128)
    lo, hi = mg.seq_shard(S, 2, 0, align=128)
    shard = [_shard(a, lo, hi, "cuda:0") for a in (K, V, ks, vs)]
    tq = torch.from_numpy(q).to("cuda:0")
    group = kvd.P2PGroup([0, 0], B, Hq, 128)
    try:
        assert kvd.device_status() == kvd.KVD_STATUS_OK
        t0 = time.time()
        group.decode(0, tq, *shard)  # rank 1 never calls: its records never arrive
        st = kvd.device_status()
        dt = time.time() - t0
        assert st & kvd.KVD_STATUS_WAIT_TIMEOUT, f"status {st}"
        assert dt < 10.0, f"the bounded wait took {dt:.1f} s"
        group.reset()
    finally:
        group.close()
    # the context survived: an ordinary decode right after is correct
    out = kvd.decode(tq, *(torch.from_numpy(a).to("cuda:0") for a in (K, V, ks, vs)))
    torch.cuda.synchronize()
    assert po.check(out.cpu().numpy(), po.decode_f64(q, K, V, ks, vs))[0] == 0
    assert kvd.device_status() == kvd.KVD_STATUS_OK


@pytest.mark.parametrize("B,Hq,Hkv,S", [
    (3, 16, 16, 3000),  # group 1: the decode tags its split records, the exchange merges them while it runs
    (2, 32, 4, 2000),   # group 8: float records, the exchange waits for the whole decode grid
    (2, 8, 8, 100),     # one split per row
])
def test_one_rank_group_exchange_matches_the_oracle(B, Hq, Hkv, S):
    """A one-rank group runs the whole exchange on one GPU (the rank pushes its
    records to itself). The query changes every call, so a record or a gather
    buffer parity left over from the previous call would show up."""
    group = kvd.P2PGroup([0], B, Hq, 128)
    try:
        for step in range(5):
            q, K, V, ks, vs = po.random_cache(90 + step, B, Hq, Hkv, S, 128)
            dev = [torch.from_numpy(a).to("cuda:0") for a in (q, K, V, ks, vs)]
            out = group.decode(0, *dev)
            torch.cuda.synchronize()
            bad, max_abs, _ = po.check(out.cpu().numpy(), po.decode_f64(q, K, V, ks, vs))
            assert bad == 0, f"step {step}: {bad} bad, max abs {max_abs:.3g}"
        assert kvd.device_status() == kvd.KVD_STATUS_OK
    finally:
        group.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_group_sequence_split_on_two_gpus():
    B, Hq, Hkv, S = 3, 16, 4, 3000
    q, K, V, ks, vs = po.random_cache(73, B, Hq, Hkv, S, 128)
    ref = po.decode_f64(q, K, V, ks, vs)
    devs = [0, 1]
    shards, queries, streams = [], [], []
    for r, d in enumerate(devs):
        lo, hi = mg.seq_shard(S, 2, r, align=128)
        shards.append([_shard(a, lo, hi, f"cuda:{d}") for a in (K, V, ks, vs)])
        queries.append(torch.from_numpy(q).to(f"cuda:{d}"))
        with torch.cuda.device(d):
            streams.append(torch.cuda.Stream())
    group = kvd.P2PGroup(devs, B, Hq, 128)
    try:
        for step in range(4):
            if step == 2:
                group.reset()
            outs = [group.decode(r, queries[r], *shards[r], stream=streams[r]) for r in range(2)]
            for s_ in streams:
                s_.synchronize()
            for r in range(2):
                bad, max_abs, _ = po.check(outs[r].cpu().numpy(), ref)
                assert bad == 0, f"rank {r} step {step}: {bad} bad, max abs {max_abs:.3g}"
        for d in devs:
            with torch.cuda.device(d):
                assert kvd.device_status() == kvd.KVD_STATUS_OK
    finally:
        group.close()
