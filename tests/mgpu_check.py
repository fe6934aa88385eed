"""Worker for tests/test_mgpu_gpu.py, launched with torch.distributed.run (one
rank per GPU, NCCL). Checks, against the FP64 oracle:
  * sequence split: each rank decodes its token shard into partial records,
    records are all-gathered over NCCL and merged by the combine kernel;
  * batch shards: each rank decodes its own sequences with no communication.
Exits 0 only if every rank's results are within the decode tolerance."""
import datetime
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "cuda-operators_b200"), os.path.join(ROOT, "oracle")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import kvd_mgpu as mg  # noqa: E402
import kvdecode as kvd  # noqa: E402
import pyoracle as po  # noqa: E402


def missed_call_then_reset(comm, rank: int, world: int, dev) -> int:
    """A rank that misses one exchange call (a dropped step, injected on the
    host): rank 0's call must end with KVD_STATUS_WAIT_TIMEOUT within a few
    seconds instead of hanging, and after the collective reset every rank's next
    calls must match the oracle again."""
    bad = 0
    B, Hq, S = 2, 8, 4096
    q, K, V, ks, vs = po.random_cache(37, B, Hq, Hq, S, 128)
    ref = po.decode_f64(q, K, V, ks, vs)
    lo, hi = mg.seq_shard(S, world, rank, align=128)
    shard = [torch.from_numpy(np.ascontiguousarray(a[:, :, lo:hi])).to(dev) for a in (K, V, ks, vs)]
    tq = torch.from_numpy(q).to(dev)
    ex = kvd.P2PExchange(comm, B, Hq, 128)
    try:
        out = ex.decode(tq, *shard)  # every rank: epoch 1
        torch.cuda.synchronize()
        bad += po.check(out.cpu().numpy(), ref)[0]
        if rank == 0:  # the other ranks skip this call
            t0 = time.time()
            ex.decode(tq, *shard)
            st = kvd.device_status()
            dt = time.time() - t0
            print(f"[rank 0] call missed by the peers: status={st} after {dt:.2f} s", flush=True)
            bad += int(not (st & kvd.KVD_STATUS_WAIT_TIMEOUT)) + int(dt > 10.0)
        ex.reset()  # collective: the ranks meet here, then clear their exchange state
        for step in range(3):
            out = ex.decode(tq, *shard)
            torch.cuda.synchronize()
            b, err, _ = po.check(out.cpu().numpy(), ref)
            bad += b
            print(f"[rank {rank}] after reset, step {step}: max_abs={err:.3g} bad={b}", flush=True)
        bad += int(kvd.device_status() != kvd.KVD_STATUS_OK)
    finally:
        dist.barrier()
        ex.close()
    return bad


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    bad = 0
    try:
        for (B, Hq, Hkv, S) in [(2, 8, 8, 4096), (2, 16, 2, 3000)]:
            q, K, V, ks, vs = po.random_cache(11 + Hq, B, Hq, Hkv, S, 128)  # same on every rank
            ref = po.decode_f64(q, K, V, ks, vs)
            lo, hi = mg.seq_shard(S, world, rank, align=128)
            shard = [torch.from_numpy(np.ascontiguousarray(a[:, :, lo:hi])).to(dev) for a in (K, V, ks, vs)]
            dec = mg.SeqSplitDecode(B, Hq, 128, dev)
            for _ in range(2):
                out = dec(torch.from_numpy(q).to(dev), *shard)
                torch.cuda.synchronize()
                b, err, _ = po.check(out.cpu().numpy(), ref)
                bad += b
                print(f"[rank {rank}] seq split B={B} Hq={Hq} Hkv={Hkv} S={S} shard=[{lo},{hi}) "
                      f"max_abs={err:.3g} bad={b}", flush=True)
            # batch shards: no communication
            b0, b1 = mg.batch_shard(B, world, rank)
            if b1 > b0:
                tq, tK, tV, tks, tvs = (torch.from_numpy(np.ascontiguousarray(a[b0:b1])).to(dev)
                                        for a in (q, K, V, ks, vs))
                out = kvd.decode(tq, tK, tV, tks, tvs)
                torch.cuda.synchronize()
                b, err, _ = po.check(out.cpu().numpy(), ref[b0:b1])
                bad += b
        # the C-ABI path: a communicator made by the library, the id broadcast by torch
        uid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(kvd.mgpu_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = kvd.MgpuComm(world, rank, bytes(uid.cpu().numpy().tobytes()))
        try:
            for (B, Hq, Hkv, S, odt) in [(2, 8, 8, 4096, torch.float32), (3, 16, 2, 2500, torch.bfloat16)]:
                q, K, V, ks, vs = po.random_cache(23 + Hq, B, Hq, Hkv, S, 128)
                ref = po.decode_f64(q, K, V, ks, vs)
                lo, hi = mg.seq_shard(S, world, rank, align=128)
                shard = [torch.from_numpy(np.ascontiguousarray(a[:, :, lo:hi])).to(dev) for a in (K, V, ks, vs)]
                for _ in range(2):
                    out = kvd.seq_split_decode(comm, torch.from_numpy(q).to(dev), *shard, out_dtype=odt)
                    torch.cuda.synchronize()
                    o = out.float().cpu().numpy()
                    tol = 2e-5 + (1e-4 + (2.0 ** -8 if odt == torch.bfloat16 else 0.0)) * np.abs(ref)
                    b = int((np.abs(o - ref) > tol).sum()) + int((~np.isfinite(o)).sum())
                    bad += b
                    print(f"[rank {rank}] C-ABI seq split B={B} Hq={Hq} Hkv={Hkv} S={S} out={odt} "
                          f"max_abs={np.abs(o - ref).max():.3g} bad={b} launches={kvd.last_launch_count()}",
                          flush=True)
            # the peer-store exchange: one kernel pushes records over NVLink and merges
            for (B, Hq, Hkv, S, odt) in [(2, 8, 8, 4096, torch.float32), (3, 16, 2, 2500, torch.float16)]:
                q, K, V, ks, vs = po.random_cache(29 + Hq, B, Hq, Hkv, S, 128)
                ref = po.decode_f64(q, K, V, ks, vs)
                lo, hi = mg.seq_shard(S, world, rank, align=128)
                shard = [torch.from_numpy(np.ascontiguousarray(a[:, :, lo:hi])).to(dev) for a in (K, V, ks, vs)]
                ex = kvd.P2PExchange(comm, B, Hq, 128)
                try:
                    for step in range(5):  # several epochs: both buffer parities, epochs counting up
                        out = ex.decode(torch.from_numpy(q).to(dev), *shard, out_dtype=odt)
                        torch.cuda.synchronize()
                        o = out.float().cpu().numpy()
                        extra = 2.0 ** -11 if odt == torch.float16 else 0.0
                        tol = 2e-5 + 2.0 ** -24 + (1e-4 + extra) * np.abs(ref)
                        b = int((np.abs(o - ref) > tol).sum()) + int((~np.isfinite(o)).sum())
                        bad += b
                        if step in (0, 4):
                            print(f"[rank {rank}] P2P seq split B={B} Hq={Hq} S={S} out={odt} step={step} "
                                  f"max_abs={np.abs(o - ref).max():.3g} bad={b} launches={kvd.last_launch_count()}",
                                  flush=True)
                    st = kvd.device_status()
                    bad += int(st != 0)
                finally:
                    dist.barrier()  # no rank unmaps its buffers while a peer could still write them
                    ex.close()
            bad += missed_call_then_reset(comm, rank, world, dev)
        finally:
            comm.close()
        flag = torch.tensor([bad], device=dev)
        dist.all_reduce(flag)
        bad = int(flag.item())
    finally:
        dist.destroy_process_group()
    return 0 if bad == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
