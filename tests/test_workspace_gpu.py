"""GPU test of the stream-ordered workspace owner kvd::OrderedWorkspace, the
counterpart of the reference's mur::OrderedWorkspace
(common/ordered_workspace.cuh:10-58): allocation on one stream, handoff to a
second stream through an event (:33-43), release on the last stream by close()
or the destructor (:44-57), and the Audit counters (:17).

A native shim (tests/native/workspace_probe.cu) decodes on stream A with the
owner's buffer, hands it to stream B and decodes again with the same buffer,
then releases it; a second owner is moved and released by its destructor. Both
outputs are checked against the FP64 oracle (the shape uses split records in
the workspace, so a missing handoff would let B overwrite A's records), and the
Audit must read 2 allocations, 2 free submissions and 0 cleanup errors."""
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
PKG = ROOT / "cuda-operators_b200"


def _probe_lib():
    kvd.lib()  # the product library, loaded first: the shim binds to this copy
    out = NATIVE / "_build" / "libkvd_workspace_probe.so"
    src = NATIVE / "workspace_probe.cu"
    hdr = PKG / "csrc" / "kvd_workspace.h"
    if not out.exists() or out.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime):
        out.parent.mkdir(exist_ok=True)
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
                        "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}", f"-I{PKG / 'csrc'}", str(src),
                        f"-L{PKG}", "-lkvdecode_b200", f"-Xlinker=-rpath,{PKG}", "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.kvd_workspace_probe.restype = ctypes.c_int
    lib.kvd_workspace_probe.argtypes = [ctypes.POINTER(kvd.DecodeDesc)] + [ctypes.c_void_p] * 9
    return lib


def test_workspace_handoff_between_streams_and_audit():
    lib = _probe_lib()
    B, H, S, D = 2, 8, 20000, 128  # long heads: the decode splits them and keeps records in the workspace
    q, K, V, ks, vs = po.random_cache(61, B, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = (torch.from_numpy(a).to("cuda") for a in (q, K, V, ks, vs))
    outs = [torch.full((B, H, D), float("nan"), device="cuda") for _ in range(3)]
    desc = kvd.make_desc(tq, tK, tks, outs[0])
    assert kvd.workspace_size(desc) > 0
    res = np.full(5, -1, np.int32)
    torch.cuda.synchronize()
    rc = lib.kvd_workspace_probe(ctypes.byref(desc), tq.data_ptr(), tK.data_ptr(), tV.data_ptr(), tks.data_ptr(),
                                 tvs.data_ptr(), outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
                                 res.ctypes.data)
    assert rc == 0, f"probe returned CUDA error {rc}"
    for i, o in enumerate(outs):
        bad, max_abs, _ = po.check(o.cpu().numpy(), ref)
        assert bad == 0, f"output {i}: {bad} bad elements, max abs {max_abs:.3g}"
    assert res[3] == 1 and res[4] == 1, "the owner does not follow its handoffs"
    assert list(res[:3]) == [2, 2, 0], f"audit {list(res[:3])}: expected 2 allocations, 2 frees, 0 errors"
    assert kvd.device_status() == kvd.KVD_STATUS_OK
