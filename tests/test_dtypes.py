"""bf16 / fp16 queries and outputs (KVD_FLAG_Q_*, KVD_FLAG_OUT_*): no
reference counterpart (the reference reads and writes fp32 only,
kv_cache/KV_int8_split_optimized.cu:266-292); parity is anchored on the FP64
oracle of the same cache.

A 16-bit query is widened to fp32 exactly, so the oracle gets the same values
and the usual tolerance (2e-5 abs + 1e-4 rel) holds. A 16-bit output adds one
rounding to nearest: at most 2^-9 (bf16) or 2^-12 (fp16) of |out|, so the
bound grows by that relative term (plus the fp16 subnormal step)."""
import ctypes

import numpy as np
import pytest

import kvdecode as kvd
import pyoracle as po

DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4


def _torch():
    import torch

    return torch


def _check(out, ref, out_dtype, what):
    torch = _torch()
    o = out.float().cpu().numpy().astype(np.float64)
    extra_rel = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}[out_dtype]
    extra_abs = 2.0 ** -24 if out_dtype == torch.float16 else 0.0
    bound = ATOL + extra_abs + (RTOL + extra_rel) * np.abs(ref)
    err = np.abs(o - ref)
    assert np.isfinite(o).all(), what
    assert (err <= bound).all(), f"{what}: max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"


def test_flag_combinations_are_checked():
    L = kvd.lib()
    d = kvd.DecodeDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim, d.max_seq_len = 1, 2, 2, 16, 8
    d.kv_stride_b, d.kv_stride_h, d.sc_stride_b, d.sc_stride_h = 256, 128, 16, 8
    d.q_stride_b, d.q_stride_h, d.o_stride_b, d.o_stride_h = 32, 16, 40, 20
    bad = [kvd.KVD_FLAG_Q_BF16 | kvd.KVD_FLAG_Q_F16, kvd.KVD_FLAG_OUT_BF16 | kvd.KVD_FLAG_OUT_F16,
           kvd.KVD_FLAG_PARTIAL_OUT | kvd.KVD_FLAG_OUT_BF16, 64]
    for f in bad:
        d.flags = f
        assert L.kvd_workspace_size(ctypes.byref(d)) == 0
        assert L.kvd_decode_launch(ctypes.byref(d), 16, 16, 16, 16, 16, 16, None, 0, None) == \
            kvd.CUDA_ERROR_INVALID_VALUE
    assert L.kvd_combine_launch(16, 1, 0, 2, 16, 16, 16, kvd.KVD_FLAG_Q_BF16, None) == kvd.CUDA_ERROR_INVALID_VALUE
    assert L.kvd_combine_launch(16, 1, 0, 2, 16, 16, 16, kvd.KVD_FLAG_PARTIAL_OUT | kvd.KVD_FLAG_OUT_F16,
                                None) == kvd.CUDA_ERROR_INVALID_VALUE


CASES = [
    # name, B, Hq, Hkv, D, lens (None: dense cap)
    ("tc-mha", 2, 8, 8, 128, None),
    ("tc-gqa8-ragged", 3, 16, 2, 128, [3000, 0, 777]),
    ("generic-d64", 2, 4, 4, 64, [500, 129]),
    ("generic-d96", 2, 6, 2, 96, None),
]
DTYPES = [("bfloat16", "float32"), ("float16", "float32"), ("float32", "bfloat16"), ("float32", "float16"),
          ("bfloat16", "bfloat16"), ("float16", "float16")]


@pytest.mark.gpu
@pytest.mark.parametrize("qd,od", DTYPES)
@pytest.mark.parametrize("name,B,Hq,Hkv,D,lens", CASES)
def test_typed_query_and_output(name, B, Hq, Hkv, D, lens, qd, od):
    torch = _torch()
    qdt, odt = getattr(torch, qd), getattr(torch, od)
    cap = 700 if lens is None else max(lens)
    q, K, V, ks, vs = po.random_cache(31 + D, B, Hq, Hkv, cap, D)
    tq = torch.from_numpy(q).to(DEV).to(qdt)
    q_exact = tq.float().cpu().numpy()  # the values the kernel reads
    tK, tV, tks, tvs = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (K, V, ks, vs)]
    tl = None if lens is None else torch.tensor(lens, dtype=torch.int32, device=DEV)
    ref = po.decode_f64(q_exact, K, V, ks, vs, seq_lens=lens)
    for _ in range(2):
        out = torch.full((B, Hq, D), float("nan"), dtype=odt, device=DEV)
        kvd.decode(tq, tK, tV, tks, tvs, out=out, seq_lens=tl)
        torch.cuda.synchronize()
        _check(out, ref, odt, f"{name} q={qd} out={od}")
    assert kvd.device_status() == kvd.KVD_STATUS_OK


@pytest.mark.gpu
@pytest.mark.parametrize("qd,od", [("bfloat16", "bfloat16"), ("float16", "float32")])
def test_typed_paged_decode(qd, od):
    from test_paged import _paged_case

    torch = _torch()
    qdt, odt = getattr(torch, qd), getattr(torch, od)
    lens = np.array([1000, 37, 512], np.int32)
    q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens = _paged_case(61, 3, 16, 2, 128, 16, "bhtd", lens)
    tq = torch.from_numpy(q).to(DEV).to(qdt)
    ref = po.decode_f64(tq.float().cpu().numpy(), K, V, ks, vs, seq_lens=lens)
    tKp, tVp, tksp, tvsp, tt, tl = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
                                     for a in (Kp, Vp, ksp, vsp, table, lens)]
    out = kvd.paged_decode(tq, tKp, tVp, tksp, tvsp, tt, tl, out_dtype=odt)
    torch.cuda.synchronize()
    _check(out, ref, odt, f"paged q={qd} out={od}")


@pytest.mark.gpu
def test_typed_output_of_record_combine():
    torch = _torch()
    B, H, S, D = 2, 8, 900, 128
    q, K, V, ks, vs = po.random_cache(67, B, H, H, S, D)
    tq, tK, tV, tks, tvs = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (q, K, V, ks, vs)]
    halves = []
    for lo, hi in ((0, 384), (384, S)):
        rec = kvd.decode(tq, tK[:, :, lo:hi], tV[:, :, lo:hi], tks[:, :, lo:hi], tvs[:, :, lo:hi], partial=True)
        halves.append(rec.view(B * H, D + 4))
    parts = torch.stack(halves)
    out = kvd.combine(parts, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    _check(out.view(B, H, D), po.decode_f64(q, K, V, ks, vs), torch.bfloat16, "combine bf16")
