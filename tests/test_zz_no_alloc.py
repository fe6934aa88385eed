"""GPU test of kvd_decode_launch_noalloc, the entry point for callers that may
not allocate device memory while decoding (their host framework owns all
device memory, or their hot path bans allocation). It runs the same decode as
kvd_decode_launch but keeps its scratch in a fixed array inside the library.

Checked through the C ABI against the existing entry point (and the FP64
oracle) within the decode tolerance, on two calls in a row, so stale contents
left in the shared array by one call cannot change the next one's result.
This file is collected last on purpose; it passes alone and after the rest."""
import ctypes

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


@pytest.mark.parametrize("B,H,S,D,ragged", [(4, 8, 3000, 128, False), (6, 4, 700, 64, True), (2, 3, 500, 80, False)])
def test_noalloc_matches_workspace_entry_point_twice(B, H, S, D, ragged):
    q, K, V, ks, vs = po.random_cache(B * 100 + S, B, H, H, S, D)
    lens = np.array([S, 0, 1, 257, S - 1, 128][:B], np.int32) if ragged else None
    tq, tK, tV, tks, tvs = _dev(q, K, V, ks, vs)
    tl = None if lens is None else torch.tensor(lens, device=DEV)
    ref_out = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=tl)  # existing entry point
    torch.cuda.synchronize()
    ref = ref_out.cpu().numpy()
    f64 = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    for _ in range(2):
        out = _poisoned((B, H, D))
        kvd.decode_noalloc(tq, tK, tV, tks, tvs, out, seq_lens=tl)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert po.check(got, ref.astype(np.float64), ATOL, RTOL)[0] == 0
        assert po.check(got, f64, ATOL, RTOL)[0] == 0


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
