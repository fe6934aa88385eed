"""Failure detection on the GPU without a fault: a bounded wait on a barrier
that nothing completes must time out, report KVD_STATUS_WAIT_TIMEOUT and
return, and the context must stay usable for the next decode."""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
NATIVE = Path(__file__).resolve().parent / "native"
ROOT = NATIVE.parents[1]


def _probe_lib():
    out = NATIVE / "_build" / "libkvd_wait_probe.so"
    src = NATIVE / "wait_probe.cu"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        out.parent.mkdir(exist_ok=True)
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-rdc=true", "-shared",
                        "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}", f"-I{ROOT / 'cuda-operators_b200' / 'csrc'}",
                        str(src), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.kvd_wait_probe.restype = ctypes.c_int
    lib.kvd_wait_probe.argtypes = [ctypes.c_void_p]
    return lib


def test_bounded_wait_times_out_and_context_survives():
    lib = _probe_lib()
    res = np.full(2, -7, np.int32)
    rc = lib.kvd_wait_probe(res.ctypes.data)
    assert rc == 0, f"probe launch failed with CUDA error {rc}"
    assert res[0] == 0, "the wait reported completion on a barrier nothing arrives at"
    assert res[1] & kvd.KVD_STATUS_WAIT_TIMEOUT
    # the CUDA context is intact: a decode right after still matches the oracle
    q, K, V, ks, vs = po.random_cache(3, 1, 4, 4, 300, 128)
    out = kvd.decode(*(torch.from_numpy(a).to("cuda") for a in (q, K, V, ks, vs)))
    torch.cuda.synchronize()
    assert po.check(out.cpu().numpy(), po.decode_f64(q, K, V, ks, vs))[0] == 0
    assert kvd.device_status() == kvd.KVD_STATUS_OK
