"""GPU parity of the decode path against the FP64 oracle, the reference's own
host loop (golden) and, when built, the reference's own kernels compiled for
sm_100a. Every call goes through the C ABI; outputs are poisoned (0xFF) before
each of two checked calls so a missed write cannot pass.

Tolerance (north-star spec): |out - fp64| <= 2e-5 + 1e-4 * |fp64| per element."""
import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4


def dev(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def poisoned(shape):
    t = torch.empty(shape, dtype=torch.float32, device=DEV)
    t.view(torch.int32).fill_(-1)  # 0xFFFFFFFF: a NaN pattern
    return t


def assert_close(out, ref, what=""):
    bad, max_abs, max_norm = po.check(out, ref, ATOL, RTOL)
    assert bad == 0, f"{what}: {bad} bad, max_abs={max_abs:.3g}, max_norm={max_norm:.3g}"
    return max_abs


def decode_checked(q, K, V, ks, vs, seq_lens=None, ref=None, **kw):
    """Two poisoned calls through kvd_decode_launch; both must match `ref`."""
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    tl = None if seq_lens is None else torch.tensor(np.asarray(seq_lens, np.int32), device=DEV)
    if ref is None:
        ref = po.decode_f64(q, K, V, ks, vs, seq_lens=seq_lens)
    for _ in range(2):
        out = poisoned(q.shape)
        kvd.decode(tq, tK, tV, tks, tvs, out=out, seq_lens=tl, **kw)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref, f"shape q{q.shape} k{K.shape}")
    return out


# ------------------------------------------------------------ reference ABI
PATTERN_SHAPES = [(4, 128, 64), (3, 129, 128), (2, 1, 64), (5, 257, 96), (1, 1000, 64), (8, 300, 128)]


@pytest.mark.parametrize("H,S,D", PATTERN_SHAPES)
@pytest.mark.parametrize("entry", ["solve", "kv_int8_split_launch", "kv_int8_simple_launch"])
def test_reference_entry_points_on_reference_test_inputs(golden, H, S, D, entry):
    Q, K, V, ks, vs = po.reference_pattern(H, S, D)
    tQ, tK, tV, tks, tvs = dev(Q, K, V, ks, vs)
    f64 = po.decode_f64(Q.reshape(1, H, D), K.reshape(1, H, S, D), V.reshape(1, H, S, D),
                        ks.reshape(1, H, S), vs.reshape(1, H, S))[0]
    scratch = torch.empty(H * S, dtype=torch.float32, device=DEV)
    for _ in range(2):
        out = poisoned((H, D))
        if entry == "solve":
            kvd.solve(tQ, tK, tV, tks, tvs, out, H, S, D)
        else:
            rc = getattr(kvd, entry)(tQ, tK, tV, tks, tvs, out, H, S, D, scratch, torch.cuda.current_stream())
            assert rc == 0
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        assert_close(o, f64, "vs fp64")
        # the reference's own acceptance test: max abs err <= 1e-4 vs its fp32 host loop
        assert np.abs(o - golden[f"pattern_{H}_{S}_{D}"]).max() <= 1e-4


BOUNDARY_S = [1, 31, 32, 33, 127, 128, 129, 255, 256, 257, 1023, 1024, 1025]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", BOUNDARY_S)
def test_mha_boundary_lengths(D, S):
    q, K, V, ks, vs = po.random_cache(S * 7 + D, 2, 3, 3, S, D)
    decode_checked(q, K, V, ks, vs)


@pytest.mark.parametrize("seed", [17, 29, 101])
@pytest.mark.parametrize("B,H,S,D", [(1, 8, 1024, 64), (4, 8, 5000, 128), (1, 2, 40000, 128), (3, 16, 3333, 64)])
def test_mha_random_parity(seed, B, H, S, D):
    q, K, V, ks, vs = po.random_cache(seed, B, H, H, S, D)
    decode_checked(q, K, V, ks, vs)


@pytest.mark.parametrize("D", [16, 32, 80, 96, 200, 256, 512])
def test_generic_head_dims(D):
    q, K, V, ks, vs = po.random_cache(D, 2, 3, 3, 300, D)
    decode_checked(q, K, V, ks, vs)


def test_unaligned_pointers_take_generic_path():
    q, K, V, ks, vs = po.random_cache(5, 1, 4, 4, 257, 128)
    ref = po.decode_f64(q, K, V, ks, vs)
    # shift K/V by one byte and scales by one float inside larger buffers
    tK = torch.zeros(K.size + 16, dtype=torch.int8, device=DEV)
    tV = torch.zeros(V.size + 16, dtype=torch.int8, device=DEV)
    tK[1:1 + K.size] = torch.from_numpy(K.ravel()).to(DEV)
    tV[1:1 + V.size] = torch.from_numpy(V.ravel()).to(DEV)
    tks = torch.zeros(ks.size + 4, device=DEV)
    tvs = torch.zeros(vs.size + 4, device=DEV)
    tks[1:1 + ks.size] = torch.from_numpy(ks.ravel()).to(DEV)
    tvs[1:1 + vs.size] = torch.from_numpy(vs.ravel()).to(DEV)
    tq = dev(q)[0]
    out = poisoned((4, 128))
    S = torch.empty(4 * 257, device=DEV)
    rc = kvd.kv_int8_split_launch(tq, tK.data_ptr() + 1, tV.data_ptr() + 1, tks.data_ptr() + 4, tvs.data_ptr() + 4,
                                  out, 4, 257, 128, S, torch.cuda.current_stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), ref[0])


# ------------------------------------------------------------ extended API
@pytest.mark.parametrize("seed", [17, 29])
def test_ragged_batch(seed):
    rng = np.random.default_rng(seed)
    cap, D = 3000, 128
    lens = rng.integers(0, cap + 1, size=9).astype(np.int32)
    lens[:3] = [0, 1, cap]
    q, K, V, ks, vs = po.random_cache(seed, 9, 4, 4, cap, D)
    decode_checked(q, K, V, ks, vs, seq_lens=lens)


@pytest.mark.parametrize("D", [64, 128])
def test_ragged_batch_small_workspace_falls_back(D):
    q, K, V, ks, vs = po.random_cache(9, 5, 2, 2, 700, D)
    lens = np.array([700, 3, 0, 256, 257], np.int32)
    ref = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    tl = torch.tensor(lens, device=DEV)
    for ws_bytes in (0, 64, 4096):  # no room for the tile plan, plan only, plan + a few partials
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=DEV)
        out = poisoned(q.shape)
        desc = kvd.make_desc(tq, tK, tks, out, seq_lens=tl)
        import ctypes
        rc = kvd.lib().kvd_decode_launch(ctypes.byref(desc), tq.data_ptr(), tK.data_ptr(), tV.data_ptr(),
                                         tks.data_ptr(), tvs.data_ptr(), out.data_ptr(),
                                         ws.data_ptr() if ws_bytes else None, ws_bytes,
                                         torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref)


@pytest.mark.parametrize("Hq,Hkv", [(16, 2), (8, 8), (12, 4), (64, 8)])
def test_grouped_query_heads(Hq, Hkv):
    q, K, V, ks, vs = po.random_cache(Hq, 3, Hq, Hkv, 777, 128)
    decode_checked(q, K, V, ks, vs)


@pytest.mark.parametrize("B,Hq,Hkv,S", [
    (40, 64, 8, 300),    # 320 (b, kv head) items >= persistent CTAs: one item per group, no split
    (4, 64, 8, 2048),    # config-5 group shape at small batch: split items + record combine
    (2, 8, 4, 1000),     # group 2
    (3, 16, 4, 513),     # group 4
    (2, 32, 2, 700),     # group 16
])
def test_gqa_tensor_core_path(B, Hq, Hkv, S):
    q, K, V, ks, vs = po.random_cache(B * Hq + S, B, Hq, Hkv, S, 128)
    decode_checked(q, K, V, ks, vs)


def test_gqa_ragged_and_records():
    B, Hq, Hkv, cap, D = 5, 32, 4, 1500, 128
    q, K, V, ks, vs = po.random_cache(55, B, Hq, Hkv, cap, D)
    lens = np.array([1500, 0, 1, 129, 640], np.int32)
    decode_checked(q, K, V, ks, vs, seq_lens=lens)
    # partial records: combining one record set must reproduce the output
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    rec = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=torch.tensor(lens, device=DEV), partial=True)
    out = kvd.combine(rec.view(1, B * Hq, D + 4))
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy().reshape(B, Hq, D), po.decode_f64(q, K, V, ks, vs, seq_lens=lens))


def test_gqa_extreme_value_scales():
    """Tiny and huge per-token scales and a dominant token: the fixed-point
    exponents of the query and weight limbs must adapt per head and tile."""
    B, Hq, Hkv, S, D = 2, 16, 2, 600, 128
    q, K, V, ks, vs = po.random_cache(77, B, Hq, Hkv, S, D)
    ks[0] *= np.float32(1e-3)
    vs[1] *= np.float32(1e3)
    ks[1, :, 17] *= np.float32(50.0)  # one token dominates the softmax of every head in batch 1
    q[0, :3] *= np.float32(1e-4)
    decode_checked(q, K, V, ks, vs)


def test_partial_records_and_cross_split_combine():
    """Decode two token halves with KVD_FLAG_PARTIAL_OUT and merge them with
    kvd_combine_launch -- the single-GPU emulation of the sequence split
    across GPUs."""
    B, H, S, D, cut = 2, 8, 4096, 128, 1536
    q, K, V, ks, vs = po.random_cache(21, B, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    parts = poisoned((2, B * H, D + 4))
    for i, (a, b) in enumerate([(0, cut), (cut, S)]):
        pv = parts[i].view(B, H, D + 4)
        kvd.decode(tq, tK[:, :, a:b], tV[:, :, a:b], tks[:, :, a:b], tvs[:, :, a:b], out=pv, partial=True)
    out = kvd.combine(parts)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy().reshape(B, H, D), ref)
    # Records against the fp64 partials. m is a reference point (it may trail
    # the true max by up to 8 because rescaling is lazy), so compare the
    # base-2 log-sum-exp m + log2(l) and the normalised o / l.
    p0 = po.partials_f64(q, K, V, ks, vs, 0, cut)
    rec = parts[0].cpu().numpy().astype(np.float64)
    lse2 = rec[:, 0] + np.log2(rec[:, 1])
    np.testing.assert_allclose(lse2, (p0[:, 0] + np.log(p0[:, 1])) / np.log(2.0), rtol=0, atol=1e-4)
    bad, max_abs, _ = po.check((rec[:, 4:] / rec[:, 1:2]).astype(np.float32), p0[:, 2:] / p0[:, 1:2])
    assert bad == 0, max_abs
    assert np.all(rec[:, 0] <= (p0[:, 0] / np.log(2.0)) + 1e-3)  # m never exceeds the true max


def test_split_count_does_not_change_result():
    H, S, D = 6, 9000, 128
    q, K, V, ks, vs = po.random_cache(4, 1, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = dev(q.reshape(H, D), K, V, ks, vs)
    outs = []
    for nfloats in [H * S, 132 * 2 * 3, 1]:  # full scratch, 3 CTAs' worth, no partial room (1 CTA)
        scratch = torch.empty(max(nfloats, 1), device=DEV)
        out = poisoned((H, D))
        import ctypes
        rc = kvd.lib().kv_int8_split_launch(tq.data_ptr(), tK.data_ptr(), tV.data_ptr(), tks.data_ptr(),
                                            tvs.data_ptr(), out.data_ptr(), H, S, D, scratch.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        assert_close(o, ref[0])
        outs.append(o)


@pytest.mark.skipif(po.ref_lib("split") is None, reason="reference kernels not built (oracle/_ref)")
@pytest.mark.parametrize("H,S,D", [(4, 128, 64), (8, 1024, 64), (16, 4096, 128), (3, 777, 128)])
def test_against_reference_kernels_built_for_sm100a(H, S, D):
    q, K, V, ks, vs = po.random_cache(H + S, 1, H, H, S, D)
    f64 = po.decode_f64(q, K, V, ks, vs)[0]
    tq, tK, tV, tks, tvs = dev(q.reshape(H, D), K, V, ks, vs)
    ours = poisoned((H, D))
    kvd.solve(tq, tK, tV, tks, tvs, ours, H, S, D)
    torch.cuda.synchronize()
    ours = ours.cpu().numpy()
    assert_close(ours, f64, "ours")
    args = [t.data_ptr() for t in (tq, tK, tV, tks, tvs)]
    for name in ["split", "tiled", "single", "simple"]:
        h = po.ref_lib(name)
        out = poisoned((H, D))
        getattr(h, f"kvref_{name}_solve")(*args, out.data_ptr(), H, S, D)
        torch.cuda.synchronize()
        r = out.cpu().numpy()
        # the reference kernels meet the same bound against fp64, and agree with ours
        assert np.abs(r - f64).max() <= 1e-4, name
        assert np.abs(r - ours).max() <= 1e-4, name


def test_decode_replays_from_cuda_graph():
    """The decode allocates nothing and never synchronises, so it can be
    captured once and replayed (how a serving loop amortises launches)."""
    B, H, S, D = 3, 8, 3000, 128
    q, K, V, ks, vs = po.random_cache(33, B, H, H, S, D)
    ref = po.decode_f64(q, K, V, ks, vs)
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    out = poisoned((B, H, D))
    desc = kvd.make_desc(tq, tK, tks, out)
    ws = torch.empty(kvd.workspace_size(desc), dtype=torch.uint8, device=DEV)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kvd.decode(tq, tK, tV, tks, tvs, out=out, workspace=ws)
    for _ in range(2):
        out.view(torch.int32).fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref)


def test_launch_accounting_and_status():
    q, K, V, ks, vs = po.random_cache(1, 2, 4, 4, 2048, 128)
    tq, tK, tV, tks, tvs = dev(q, K, V, ks, vs)
    kvd.decode(tq, tK, tV, tks, tvs)
    assert kvd.last_launch_count() in (1, 2)
    assert kvd.device_status() == kvd.KVD_STATUS_OK
