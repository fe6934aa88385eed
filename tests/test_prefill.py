"""Causal prefill over the INT8 cache (kvd_prefill_launch): no reference
counterpart (the reference's prefill attention is fp32 without a KV cache,
attention/). Parity is anchored on the FP64 oracle, kvo_prefill_f64, which is
itself pinned on CPU to the decode oracle run once per query over the query's
causal prefix. Tolerance: 2e-5 abs + 1e-4 rel per element (16-bit outputs add
their rounding step)."""
import ctypes

import numpy as np
import pytest

import kvdecode as kvd
import pyoracle as po

DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4


def test_prefill_oracle_equals_per_query_decode():
    B, Hq, Hkv, Lq, cap, D = 2, 4, 2, 6, 50, 16
    _, K, V, ks, vs = po.random_cache(3, B, Hq, Hkv, cap, D)
    q = np.random.default_rng(1).standard_normal((B, Hq, Lq, D), dtype=np.float32)
    lens = np.array([37, 9], np.int32)
    ql = np.array([6, 4], np.int32)
    out = po.prefill_f64(q, K, V, ks, vs, lens, ql)
    for b in range(B):
        for i in range(Lq):
            if i >= ql[b]:
                assert not out[b, :, i].any()
                continue
            pos = lens[b] - ql[b] + i
            ref = po.decode_f64(q[b:b + 1, :, i], K[b:b + 1], V[b:b + 1], ks[b:b + 1], vs[b:b + 1],
                                seq_lens=np.array([pos + 1], np.int32))
            np.testing.assert_allclose(out[b, :, i], ref[0], rtol=1e-12, atol=1e-14)


def test_prefill_argument_checks():
    L = kvd.lib()
    d = kvd.PrefillDesc()
    assert L.kvd_prefill_launch(ctypes.byref(d), *([16] * 6), None, 0, None) == kvd.CUDA_ERROR_INVALID_VALUE
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim, d.max_seq_len, d.max_queries = 1, 4, 2, 64, 8, 4
    d.flags = kvd.KVD_FLAG_PARTIAL_OUT  # records are a decode-only output
    assert L.kvd_prefill_launch(ctypes.byref(d), *([16] * 6), None, 0, None) == kvd.CUDA_ERROR_INVALID_VALUE
    d.flags = 0
    d.num_q_heads = 3  # not a multiple of the kv heads
    assert L.kvd_prefill_launch(ctypes.byref(d), *([16] * 6), None, 0, None) == kvd.CUDA_ERROR_INVALID_VALUE


def _case(seed, B, Hq, Hkv, Lq, cap, D, lens, qlens, qdtype="float32"):
    import torch

    _, K, V, ks, vs = po.random_cache(seed, B, Hq, Hkv, cap, D)
    q = np.random.default_rng(seed + 1).standard_normal((B, Hq, Lq, D), dtype=np.float32)
    tq = torch.from_numpy(q).to(DEV).to(getattr(torch, qdtype))
    q_exact = tq.float().cpu().numpy()
    ref = po.prefill_f64(q_exact, K, V, ks, vs, lens, qlens)
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (K, V, ks, vs)]
    tl = None if lens is None else torch.tensor(lens, dtype=torch.int32, device=DEV)
    tql = None if qlens is None else torch.tensor(qlens, dtype=torch.int32, device=DEV)
    return tq, t, tl, tql, ref


def _check(out, ref, what, out_dtype="float32"):
    o = out.float().cpu().numpy().astype(np.float64)
    extra = {"float32": 0.0, "bfloat16": 2.0 ** -8, "float16": 2.0 ** -11}[out_dtype]
    bound = ATOL + (RTOL + extra) * np.abs(ref) + (2.0 ** -24 if out_dtype == "float16" else 0.0)
    err = np.abs(o - ref)
    assert np.isfinite(o).all(), what
    assert (err <= bound).all(), f"{what}: max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"


PREFILL_CASES = [
    # B, Hq, Hkv, Lq, cap, D, lens, qlens
    (1, 4, 4, 200, 200, 128, None, None),                    # whole prompt, MHA
    (2, 8, 2, 130, 700, 128, [700, 300], [130, 77]),         # GQA 4, queries at the end of a longer cache
    (2, 16, 2, 64, 512, 128, [512, 64], None),               # GQA 8
    (1, 16, 1, 33, 1000, 128, [1000], None),                  # GQA 16
    (2, 4, 4, 50, 300, 64, [300, 120], [50, 20]),            # head_dim 64
    (1, 6, 2, 17, 90, 96, None, None),                       # head_dim 96
    (2, 4, 2, 70, 150, 128, [150, 0], [70, 0]),              # GQA 2, an empty sequence
    (3, 8, 8, 40, 100, 128, [100, 37, 64], [0, 37, 10]),     # a sequence without queries, ragged tails
    (1, 16, 8, 257, 1100, 128, [1100], [257]),               # GQA 2, queries past two 128-row blocks
    (2, 8, 4, 140, 200, 128, [30, 200], [140, 20]),          # more queries than tokens: leading rows are 0
    (1, 4, 4, 20, 40, 64, [12], [20]),                       # the same on the generic kernel
]


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,Lq,cap,D,lens,qlens", PREFILL_CASES)
def test_prefill_matches_fp64(B, Hq, Hkv, Lq, cap, D, lens, qlens):
    import torch

    tq, (tK, tV, tks, tvs), tl, tql, ref = _case(5 + D + Lq, B, Hq, Hkv, Lq, cap, D, lens, qlens)
    for _ in range(2):
        out = torch.full(tq.shape, float("nan"), dtype=torch.float32, device=DEV)
        kvd.prefill(tq, tK, tV, tks, tvs, seq_lens=tl, q_lens=tql, out=out)
        torch.cuda.synchronize()
        _check(out, ref, f"prefill B={B} Hq={Hq} Hkv={Hkv} Lq={Lq} cap={cap} D={D}")
    assert kvd.device_status() == kvd.KVD_STATUS_OK


@pytest.mark.gpu
@pytest.mark.parametrize("qd,od", [("bfloat16", "bfloat16"), ("float16", "float32"), ("float32", "float16")])
def test_prefill_typed(qd, od):
    import torch

    tq, (tK, tV, tks, tvs), tl, tql, ref = _case(71, 2, 8, 2, 96, 400, 128, [400, 200], [96, 40], qd)
    out = kvd.prefill(tq, tK, tV, tks, tvs, seq_lens=tl, q_lens=tql, out_dtype=getattr(torch, od))
    torch.cuda.synchronize()
    _check(out, ref, f"prefill q={qd} out={od}", od)


@pytest.mark.gpu
def test_prefill_single_query_equals_decode():
    """A prefill of one query is a decode over the whole cache."""
    import torch

    tq, (tK, tV, tks, tvs), tl, tql, ref = _case(83, 3, 8, 2, 1, 600, 128, [600, 1, 345], None)
    out = kvd.prefill(tq, tK, tV, tks, tvs, seq_lens=tl)
    dec = kvd.decode(tq[:, :, 0].contiguous(), tK, tV, tks, tvs, seq_lens=tl)
    torch.cuda.synchronize()
    _check(out, ref, "prefill Lq=1")
    _check(dec.unsqueeze(2), ref, "decode")
