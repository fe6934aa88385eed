"""GPU tests of the one-launch decode for small dense MHA problems (a thread-block
cluster per head merging (m, l, o) records through distributed shared memory;
configuration 1's kernel). The reference's small shapes run per-head kernels
(kv_cache/KV_int8.cu:49-274) or a three-kernel split
(kv_cache/KV_int8_split_optimized.cu:109-243); here the result must match the
FP64 oracle within 2e-5 + 1e-4 |ref| with ONE kernel launch, for every cluster
size (1..8 CTAs per head), both head dims, partial records, a custom softmax
scale, a cache whose capacity exceeds the decoded length, and extreme scales.
Outputs are poisoned before each of two checked calls."""
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


def _check(out, ref, what):
    bad, max_abs, _ = po.check(out, ref, ATOL, RTOL)
    assert bad == 0, f"{what}: {bad} bad, max abs {max_abs:.3g}"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [1, 100, 128, 129, 255, 256, 257, 640, 1000, 1024, 1537, 2048])
def test_one_launch_for_every_cluster_size(D, S):
    B, H = 2, 4
    q, K, V, ks, vs = po.random_cache(S * 3 + D, B, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = _dev(q, K, V, ks, vs)
    for _ in range(2):
        out = _poisoned((B, H, D))
        kvd.decode(tq, tK, tV, tks, tvs, out=out)
        assert kvd.last_launch_count() == 1
        torch.cuda.synchronize()
        _check(out.cpu().numpy(), ref, f"S={S} D={D}")
    assert kvd.device_status() == kvd.KVD_STATUS_OK


@pytest.mark.parametrize("D", [64, 128])
def test_partial_records_combine_to_the_output(D):
    B, H, S = 1, 8, 1024  # configuration 1's shape (D=64) and its head_dim-128 twin
    q, K, V, ks, vs = po.random_cache(101 + D, B, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = _dev(q, K, V, ks, vs)
    rec = _poisoned((B, H, D + 4))
    kvd.decode(tq, tK, tV, tks, tvs, out=rec, partial=True)
    assert kvd.last_launch_count() == 1
    torch.cuda.synchronize()
    r = rec.cpu().numpy().reshape(B * H, D + 4)
    # the record's normalised output and its log-sum-exp against FP64
    _check((r[:, 4:] / r[:, 1:2]).reshape(B, H, D), ref, "record o / l")
    scale = 1.0 / np.sqrt(D)
    s = np.einsum("hd,htd->ht", q.reshape(H, D).astype(np.float64), K[0].astype(np.float64)) * ks[0] * scale
    lse2 = (s.max(axis=1) + np.log(np.exp(s - s.max(axis=1, keepdims=True)).sum(axis=1))) / np.log(2.0)
    assert np.allclose(r[:, 0] + np.log2(r[:, 1]), lse2, rtol=0, atol=1e-5)
    out = kvd.combine(rec.view(1, B * H, D + 4))
    torch.cuda.synchronize()
    _check(out.cpu().numpy().reshape(B, H, D), ref, "combine of the records")


def test_custom_scale_and_capacity_beyond_length():
    B, H, cap, S, D = 3, 2, 1500, 1100, 64
    q, K, V, ks, vs = po.random_cache(7, B, H, H, cap, D)
    scale = 0.3
    ref = po.decode_f64(q, K[:, :, :S], V[:, :, :S], ks[:, :, :S], vs[:, :, :S], softmax_scale=scale)
    tq, tK, tV, tks, tvs = _dev(q, K, V, ks, vs)
    for _ in range(2):
        out = _poisoned((B, H, D))
        kvd.decode(tq, tK, tV, tks, tvs, out=out, max_seq_len=S, softmax_scale=scale)
        assert kvd.last_launch_count() == 1
        torch.cuda.synchronize()
        _check(out.cpu().numpy(), ref, "capacity > length, custom scale")


def test_extreme_scales_and_a_dominant_token():
    B, H, S, D = 1, 8, 1024, 64
    q, K, V, ks, vs = po.random_cache(13, B, H, H, S, D)
    ks[0, :4] *= np.float32(1e-3)
    vs[0, 4:] *= np.float32(1e3)
    ks[0, 5, 700] *= np.float32(60.0)  # one token dominates head 5 (it sits in the 6th CTA of the cluster)
    ref = po.decode_f64(q, K, V, ks, vs)
    out = kvd.decode(*_dev(q, K, V, ks, vs))
    torch.cuda.synchronize()
    _check(out.cpu().numpy(), ref, "extreme scales")
