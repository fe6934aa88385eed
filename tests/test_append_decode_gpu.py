"""Fused quantise-on-append + decode (kvd_append_decode_launch): no reference
counterpart (the reference has no append, kv_cache/new_kvint8.cu:83-84).

The fused call must leave exactly the state the two separate calls leave:
the same cache bits, the same lengths, the same status, and -- because the
decode runs the same kernel over the same work plan -- the same output bits.
The output is also checked against the FP64 oracle of the grown cache
(2e-5 abs + 1e-4 rel)."""
import numpy as np
import pytest

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _torch():
    import torch

    return torch


def _state(B, Hq, Hkv, cap, D, lens, seed):
    torch = _torch()
    q, K, V, ks, vs = po.random_cache(seed, B, Hq, Hkv, cap, D)
    rng = np.random.default_rng(seed + 1)
    kn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    vn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    kn[0] = 0.0  # an all-zero row: scale 0, codes 0
    if B > 2:
        vn[2, 0, :4] = [np.nan, 40.0, -40.0, 0.0]  # a NaN and an outlier: both paths give the same bits
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (q, K, V, ks, vs, kn, vn)]
    t.append(torch.tensor(lens, dtype=torch.int32, device=DEV))
    return t


def _clone(ts):
    return [x.clone() for x in ts]


def _run_both(B, Hq, Hkv, cap, D, lens, seed, steps=1):
    torch = _torch()
    base = _state(B, Hq, Hkv, cap, D, lens, seed)
    fused, sep = _clone(base), _clone(base)
    for _ in range(steps):
        q, K, V, ks, vs, kn, vn, tl = fused
        of = kvd.append_decode(kn, vn, q, K, V, ks, vs, tl)
        torch.cuda.synchronize()
        n_fused = kvd.last_launch_count()
        st_f = kvd.device_status()
        q, K, V, ks, vs, kn, vn, tl = sep
        kvd.append(kn, vn, K, V, ks, vs, tl)
        os_ = kvd.decode(q, K, V, ks, vs, seq_lens=tl)
        torch.cuda.synchronize()
        n_sep = 1 + kvd.last_launch_count()
        st_s = kvd.device_status()
        assert st_f == st_s
        for a, b in zip(fused[1:5] + [fused[7]], sep[1:5] + [sep[7]]):
            assert torch.equal(a, b), "cache or lengths differ"
        assert np.array_equal(of.cpu().numpy(), os_.cpu().numpy()), "outputs differ"
    q, K, V, ks, vs, kn, vn, tl = fused
    ref = po.decode_f64(q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy(),
                        seq_lens=tl.cpu().numpy())
    bad, max_abs, _ = po.check(of.cpu().numpy(), ref)
    assert bad == 0, f"vs fp64: max_abs={max_abs:.3g}"
    return n_fused, n_sep, st_f, tl.cpu().numpy()


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 2), (32, 4)])
def test_fused_equals_append_then_decode(Hq, Hkv):
    lens = [0, 1, 127, 128, 255, 2047, 2048, 3000, 4095, 511]
    n_fused, n_sep, st, new = _run_both(len(lens), Hq, Hkv, 4096, 128, lens, seed=Hq)
    assert st == kvd.KVD_STATUS_OK
    assert list(new) == [x + 1 for x in lens]
    assert n_fused <= 3 and n_fused < n_sep  # no separate append kernel


def test_fused_full_cache_is_left_unchanged():
    cap = 640
    lens = [cap, 100, cap - 1, cap]
    n_fused, n_sep, st, new = _run_both(4, 8, 2, cap, 128, lens, seed=5)
    assert st & kvd.KVD_STATUS_CACHE_FULL
    assert list(new) == [cap, 101, cap, cap]


def test_fused_repeated_steps():
    _run_both(3, 16, 2, 1024, 128, [5, 900, 1000], seed=9, steps=4)


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 4, 4), (96, 6, 2), (128, 6, 2)])
def test_other_shapes_take_two_launches_with_the_same_result(D, Hq, Hkv):
    # head_dim 64 / 96 and a group of 3 are not tensor-core shapes: append, then decode
    n_fused, n_sep, st, new = _run_both(3, Hq, Hkv, 700, D, [0, 350, 699], seed=D)
    assert st == kvd.KVD_STATUS_OK and list(new) == [1, 351, 700]
