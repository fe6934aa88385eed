"""GPU tests of the INT8 Q.K fast mode (KVD_FLAG_QK_INT8; no counterpart in the
reference, whose Q.K is an fp32 product over dequantised codes,
kv_cache/KV_int8_split_optimized.cu:136-143).

The mode rounds each query row (b, hq) to int8 with the cache's quantiser rule
and runs Q.K as one exact int8 tensor-core product per head. Two checks:
  1. against the FP64 oracle fed the ROUNDED query q^ = code_q * scale_q, the
     north-star tolerance |out - f64| <= 2e-5 + 1e-4 |f64| holds (the mode is
     exact attention of q^);
  2. against the FP64 oracle of the original query, the stated looser bound of
     the header: |out - f64(q)| <= 2e-5 + 1.25 * 2 * max_t |ds_t| * max_t,d |v_td|
     per row, where ds_t = (q^ - q) . k_t * softmax_scale is the score change
     the rounding makes (first order, with a margin for the second-order term).
Outputs are poisoned before each of two checked calls."""
import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4


def _rounded_query(q):
    codes, scales = po.quantize_rows(q)
    return (codes.astype(np.float32) * scales[..., None]).astype(np.float32)


def _first_order_bound(q, qh, K, V, ks, vs, lens):
    """Per (b, hq) row: 2 * max_t |(q^ - q) . k_t| * scale * max_t,d |v_td|."""
    B, Hq, D = q.shape
    Hkv = K.shape[1]
    G = Hq // Hkv
    bound = np.zeros((B, Hq))
    for b in range(B):
        n = K.shape[2] if lens is None else int(lens[b])
        if n == 0:
            continue
        for hk in range(Hkv):
            k = K[b, hk, :n].astype(np.float64) * ks[b, hk, :n, None]
            vmax = np.abs(V[b, hk, :n].astype(np.float64) * vs[b, hk, :n, None]).max()
            dq = (qh[b, hk * G:(hk + 1) * G].astype(np.float64) - q[b, hk * G:(hk + 1) * G])
            ds = np.abs(dq @ k.T).max(axis=1) / np.sqrt(D)
            bound[b, hk * G:(hk + 1) * G] = 2.0 * ds * vmax
    return bound


CASES = [  # B, Hq, Hkv, S, ragged, query dtype
    (2, 8, 8, 3000, False, torch.float32),   # MHA (group 1)
    (3, 16, 8, 2500, True, torch.float32),   # group 2, ragged
    (2, 32, 8, 1000, False, torch.float32),  # group 4
    (2, 64, 8, 2048, False, torch.float32),  # group 8: configuration 5's shape
    (3, 32, 2, 1500, True, torch.float32),   # group 16, ragged
    (2, 64, 8, 700, False, torch.bfloat16),  # a bf16 query, widened exactly then rounded
]


@pytest.mark.parametrize("B,Hq,Hkv,S,ragged,qdt", CASES)
def test_qk_int8_is_exact_attention_of_the_rounded_query(B, Hq, Hkv, S, ragged, qdt):
    q, K, V, ks, vs = po.random_cache(B * 31 + Hq + S, B, Hq, Hkv, S, 128)
    if qdt == torch.bfloat16:
        q = torch.from_numpy(q).to(torch.bfloat16).float().numpy()
    lens = None
    if ragged:
        lens = np.random.default_rng(S).integers(0, S + 1, size=B).astype(np.int32)
        lens[0] = S
    qh = _rounded_query(q)
    ref_hat = po.decode_f64(qh, K, V, ks, vs, seq_lens=lens)
    ref = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    tol = ATOL + 1.25 * _first_order_bound(q, qh, K, V, ks, vs, lens)[..., None]
    tq = torch.from_numpy(q).to(DEV).to(qdt)
    tK, tV, tks, tvs = (torch.from_numpy(a).to(DEV) for a in (K, V, ks, vs))
    tl = None if lens is None else torch.from_numpy(lens).to(DEV)
    for _ in range(2):
        out = torch.empty((B, Hq, 128), device=DEV)
        out.view(torch.int32).fill_(-1)
        kvd.decode(tq, tK, tV, tks, tvs, out=out, seq_lens=tl, qk_int8=True)
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        bad, max_abs, _ = po.check(o, ref_hat, ATOL, RTOL)
        assert bad == 0, f"vs the rounded query: {bad} bad, max abs {max_abs:.3g}"
        err = np.abs(o - ref)
        assert np.all(np.isfinite(o)) and np.all(err <= tol), \
            f"vs the original query: max err {err.max():.3g}, worst err/tol {(err / tol).max():.3g}"
    assert kvd.device_status() == kvd.KVD_STATUS_OK


def test_qk_int8_fused_append_matches_two_calls():
    """The fused append + decode with the int8 query gives the bits of the append
    kernel followed by the int8-query decode."""
    B, Hq, Hkv, cap = 4, 32, 4, 1200
    q, K, V, ks, vs = po.random_cache(83, B, Hq, Hkv, cap, 128)
    lens = np.array([1000, 0, 511, 1199], np.int32)
    rng = np.random.default_rng(89)
    kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    outs = []
    for fused in (True, False):
        tq, tK, tV, tks, tvs, tl, tkn, tvn = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
                                              for a in (q, K, V, ks, vs, lens, kn, vn))
        if fused:
            o = kvd.append_decode(tkn, tvn, tq, tK, tV, tks, tvs, tl, qk_int8=True)
        else:
            kvd.append(tkn, tvn, tK, tV, tks, tvs, tl)
            o = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=tl, qk_int8=True)
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert kvd.device_status() == kvd.KVD_STATUS_OK


def test_qk_int8_outside_the_tensor_core_kernel_is_not_supported():
    q, K, V, ks, vs = (torch.from_numpy(a).to(DEV) for a in po.random_cache(3, 1, 4, 4, 100, 64))
    with pytest.raises(kvd.KvdError) as ei:
        kvd.decode(q, K, V, ks, vs, qk_int8=True)
    assert ei.value.code == 801  # cudaErrorNotSupported


@pytest.mark.parametrize("bs,layout", [(16, "bhtd"), (64, "bthd")])
def test_qk_int8_paged_cache(bs, layout):
    """The INT8 Q.K mode through the paged entry point: the same bits as the
    dense ragged decode of the cache the pools were scattered from, and exact
    attention of the rounded query."""
    from test_paged import scatter_to_pool

    B, Hq, Hkv, D = 3, 32, 4, 128
    lens = np.array([1100, 0, 517], np.int32)
    nb = -(-1100 // bs)
    q, K, V, ks, vs = po.random_cache(97 + bs, B, Hq, Hkv, nb * bs, D)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, layout, seed=5)
    tq, tK, tV, tks, tvs, tl = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (q, K, V, ks, vs, lens))
    pK, pV, pks, pvs, tt = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (Kp, Vp, ksp, vsp, table))
    paged = kvd.paged_decode(tq, pK, pV, pks, pvs, tt, tl, layout=layout, qk_int8=True)
    dense = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=tl, qk_int8=True)
    torch.cuda.synchronize()
    assert np.array_equal(paged.cpu().numpy(), dense.cpu().numpy())
    ref_hat = po.decode_f64(_rounded_query(q), K, V, ks, vs, seq_lens=lens)
    bad, max_abs, _ = po.check(paged.cpu().numpy(), ref_hat, ATOL, RTOL)
    assert bad == 0, f"{bad} bad, max abs {max_abs:.3g}"
    assert kvd.device_status() == kvd.KVD_STATUS_OK
