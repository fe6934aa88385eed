"""GPU test of kvd_decode_launch_noalloc, the entry point for callers that may
not allocate device memory while decoding (their host framework owns all
device memory, or their hot path bans allocation). It runs the same decode as
kvd_decode_launch but keeps its scratch in a fixed array inside the library.

Checked through the C ABI against the existing entry point (and the FP64
oracle) within the decode tolerance, on two calls in a row, so stale contents
left in the shared array by one call cannot change the next one's result.
This file is collected last on purpose; it passes alone and after the rest."""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4


def _dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def _poisoned(shape):
    t = torch.empty(shape, dtype=torch.float32, device=DEV)
    t.view(torch.int32).fill_(-1)
    return t


# (B, Hq, Hkv, S, D, ragged, output type): dense MHA on the tensor-core kernel,
# ragged head_dim 64 on the CUDA-core split kernel, head_dim 80 on the generic
# kernel, ragged grouped-query heads on the tensor-core kernel (its tile order
# and split records sit in the shared array), and a bf16 output.
CASES = [(4, 8, 8, 3000, 128, False, torch.float32), (6, 4, 4, 700, 64, True, torch.float32),
         (2, 3, 3, 500, 80, False, torch.float32), (3, 16, 2, 1500, 128, True, torch.float32),
         (3, 16, 2, 2000, 128, False, torch.bfloat16)]


@pytest.mark.parametrize("B,Hq,Hkv,S,D,ragged,odt", CASES)
def test_noalloc_matches_workspace_entry_point_twice(B, Hq, Hkv, S, D, ragged, odt):
    q, K, V, ks, vs = po.random_cache(B * 100 + S, B, Hq, Hkv, S, D)
    lens = np.array([S, 0, 1, 257, S - 1, 128][:B], np.int32) if ragged else None
    tq, tK, tV, tks, tvs = _dev(q, K, V, ks, vs)
    tl = None if lens is None else torch.tensor(lens, device=DEV)
    ref_out = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=tl, out_dtype=odt)  # existing entry point
    torch.cuda.synchronize()
    ref = ref_out.float().cpu().numpy()
    f64 = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    rel16 = 2.0 ** -8 if odt == torch.bfloat16 else 0.0  # one bf16 rounding of the output
    for _ in range(2):
        out = torch.empty((B, Hq, D), dtype=odt, device=DEV)
        out.view(torch.int16 if odt == torch.bfloat16 else torch.int32).fill_(-1)
        kvd.decode_noalloc(tq, tK, tV, tks, tvs, out, seq_lens=tl)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert po.check(got, ref.astype(np.float64), ATOL, RTOL)[0] == 0
        assert po.check(got, f64, ATOL, RTOL + rel16)[0] == 0


def test_noalloc_rejects_long_context_shape():
    """A dense long-context decode (4 sequences x 32 heads x 131,072 tokens) plans
    more split records than the fixed array holds: rejected before any launch."""
    d = kvd.DecodeDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim, d.max_seq_len = 4, 32, 32, 128, 131072
    d.kv_stride_h, d.kv_stride_b = 131072 * 128, 32 * 131072 * 128
    d.sc_stride_h, d.sc_stride_b = 131072, 32 * 131072
    d.q_stride_h, d.q_stride_b = 128, 32 * 128
    d.o_stride_h, d.o_stride_b = 128, 32 * 128
    assert kvd.workspace_size(d) > kvd.NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(64, device=DEV)
    out = torch.full((16,), 7.0, device=DEV)
    p = dummy.data_ptr()
    rc = kvd.lib().kvd_decode_launch_noalloc(ctypes.byref(d), p, p, p, p, p, out.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == kvd.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)


def test_noalloc_rejects_scratch_beyond_its_fixed_size():
    B = 200_000  # the ragged tile plan alone needs (B+1)*4 bytes > 512 KiB
    lens = torch.ones(B, dtype=torch.int32, device=DEV)
    q = torch.zeros((B, 1, 128), device=DEV)
    K = torch.zeros((B, 1, 1, 128), dtype=torch.int8, device=DEV)
    ks = torch.zeros((B, 1, 1), device=DEV)
    out = torch.full((B, 1, 128), 7.0, device=DEV)
    desc = kvd.make_desc(q, K, ks, out, seq_lens=lens)
    assert kvd.workspace_size(desc) > kvd.NOALLOC_SCRATCH_BYTES
    rc = kvd.lib().kvd_decode_launch_noalloc(ctypes.byref(desc), q.data_ptr(), K.data_ptr(), K.data_ptr(),
                                             ks.data_ptr(), ks.data_ptr(), out.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == kvd.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched


def test_noalloc_after_device_reset_in_a_process_of_its_own():
    """A caller that resets its device (cudaDeviceReset) gets a new CUDA context;
    the library must look the fixed array's address up again rather than use
    the stale one. Runs as its own program, because a reset destroys every
    allocation of the process: two rounds of (allocate, decode through the
    workspace entry, decode twice through the no-alloc entry, compare, reset)."""
    native = Path(__file__).resolve().parent / "native"
    root = native.parents[1]
    pkg = root / "cuda-operators_b200"
    kvd.lib()
    exe = native / "_build" / "noalloc_reset"
    src = native / "noalloc_reset.cu"
    if not exe.exists() or exe.stat().st_mtime < max(src.stat().st_mtime, kvd.LIB_PATH.stat().st_mtime):
        exe.parent.mkdir(exist_ok=True)
        subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        f"-I{root / 'include'}", str(src), f"-L{pkg}", "-lkvdecode_b200",
                        f"-Xlinker=-rpath,{pkg}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("max |noalloc - workspace entry|") == 4 and r.stdout.strip().endswith("ok"), r.stdout
