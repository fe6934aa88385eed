"""Paged KV cache: decode and quantise-on-append over block pools addressed by
a block table (no reference counterpart; the reference's caches are dense
[H][S][D] arrays, kv_cache/new_kvint8.cu:83-84).

Parity is anchored twice: against the FP64 oracle run on the dense cache the
pool was scattered from (tolerance 2e-5 abs + 1e-4 rel), and bit for bit
against the library's dense decode of the same cache (same kernel, same work
plan: the block table only changes where tiles are fetched from). Pool slots
that hold no token of the sequence are filled with random codes and NaN
scales, so a masking error cannot pass. CPU tests cover the scatter helper
and argument checking."""
import ctypes

import numpy as np
import pytest

import kvdecode as kvd
import pyoracle as po

ATOL, RTOL = 2e-5, 1e-4
DEV = "cuda:0"


# ----------------------------------------------------------- host-side layout
def scatter_to_pool(K, V, ks, vs, bs: int, layout: str, seed: int, spare: int = 3):
    """Scatter dense [B,H,cap,D] codes and [B,H,cap] scales into block pools in
    a random block order. Returns (Kp, Vp, ksp, vsp, table); unused slots hold
    random codes and NaN scales."""
    B, H, cap, D = K.shape
    nb = -(-cap // bs)
    NB = B * nb + spare
    rng = np.random.default_rng(seed)
    table = rng.permutation(NB)[: B * nb].reshape(B, nb).astype(np.int32)
    shape = (NB, H, bs, D) if layout == "bhtd" else (NB, bs, H, D)
    Kp = rng.integers(-127, 128, size=shape, dtype=np.int8)
    Vp = rng.integers(-127, 128, size=shape, dtype=np.int8)
    ksp = np.full((NB, H, bs), np.nan, np.float32)
    vsp = np.full((NB, H, bs), np.nan, np.float32)
    for b in range(B):
        for j in range(nb):
            t0, t1 = j * bs, min(cap, (j + 1) * bs)
            blk = table[b, j]
            kb, vb = K[b, :, t0:t1], V[b, :, t0:t1]
            if layout == "bhtd":
                Kp[blk, :, : t1 - t0] = kb
                Vp[blk, :, : t1 - t0] = vb
            else:
                Kp[blk, : t1 - t0] = kb.transpose(1, 0, 2)
                Vp[blk, : t1 - t0] = vb.transpose(1, 0, 2)
            ksp[blk, :, : t1 - t0] = ks[b, :, t0:t1]
            vsp[blk, :, : t1 - t0] = vs[b, :, t0:t1]
    return Kp, Vp, ksp, vsp, table


def gather_from_pool(Kp, ksp, table, bs: int, layout: str, cap: int):
    """Inverse of scatter_to_pool for codes and scales (the test's view of the
    addressing rule in include/kvdecode.h)."""
    B, nb = table.shape
    H = Kp.shape[1] if layout == "bhtd" else Kp.shape[2]
    D = Kp.shape[3]
    K = np.zeros((B, H, nb * bs, D), np.int8)
    ks = np.zeros((B, H, nb * bs), np.float32)
    for b in range(B):
        for j in range(nb):
            blk = table[b, j]
            K[b, :, j * bs:(j + 1) * bs] = Kp[blk] if layout == "bhtd" else Kp[blk].transpose(1, 0, 2)
            ks[b, :, j * bs:(j + 1) * bs] = ksp[blk]
    return K[:, :, :cap], ks[:, :, :cap]


@pytest.mark.parametrize("layout", ["bhtd", "bthd"])
@pytest.mark.parametrize("bs", [1, 8, 24, 128])
def test_scatter_and_gather_round_trip(layout, bs):
    q, K, V, ks, vs = po.random_cache(3, 2, 4, 2, 300, 16)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, layout, seed=5)
    K2, ks2 = gather_from_pool(Kp, ksp, table, bs, layout, 300)
    V2, vs2 = gather_from_pool(Vp, vsp, table, bs, layout, 300)
    assert np.array_equal(K2, K) and np.array_equal(V2, V)
    assert np.array_equal(ks2, ks) and np.array_equal(vs2, vs)
    assert len(set(table.ravel().tolist())) == table.size  # every block used once


def test_paged_symbols_and_argument_checks():
    L = kvd.lib()
    for name in ("kvd_paged_workspace_size", "kvd_paged_decode_launch", "kvd_paged_append_int8_launch"):
        assert hasattr(L, name)
    d = kvd.PagedDesc()
    assert L.kvd_paged_workspace_size(ctypes.byref(d)) == 0  # zero shapes are rejected, size 0
    assert L.kvd_paged_decode_launch(ctypes.byref(d), *([None] * 7), 0, None) == kvd.CUDA_ERROR_INVALID_VALUE
    assert L.kvd_paged_decode_launch(None, *([None] * 7), 0, None) == kvd.CUDA_ERROR_INVALID_VALUE
    assert L.kvd_paged_append_int8_launch(ctypes.byref(d), None, None, 0, 0, *([None] * 5), None) == \
        kvd.CUDA_ERROR_INVALID_VALUE
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim = 2, 8, 2, 128
    d.block_size, d.num_blocks, d.max_blocks_per_seq, d.block_table_stride = 16, 64, 32, 16  # stride < entries
    d.seq_lens = d.block_table = 16
    assert L.kvd_paged_workspace_size(ctypes.byref(d)) == 0
    d.block_table_stride = 32
    d.flags = 64  # unknown flag
    assert L.kvd_paged_workspace_size(ctypes.byref(d)) == 0


# ------------------------------------------------------------------ GPU parity
def _dev(*arrays):
    import torch

    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def _poisoned(shape):
    import torch

    t = torch.empty(shape, dtype=torch.float32, device=DEV)
    t.view(torch.int32).fill_(-1)
    return t


def _check(out, ref, what):
    bad, max_abs, max_norm = po.check(out, ref, ATOL, RTOL)
    assert bad == 0, f"{what}: {bad} bad, max_abs={max_abs:.3g}, max_norm={max_norm:.3g}"


def _paged_case(seed, B, Hq, Hkv, D, bs, layout, lens, cap_blocks=None):
    lens = np.asarray(lens, np.int32)
    nb = cap_blocks or -(-int(lens.max(initial=1)) // bs)
    cap = nb * bs
    q, K, V, ks, vs = po.random_cache(seed, B, Hq, Hkv, cap, D)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, layout, seed=seed + 1)
    # slots past each sequence's length are garbage in a live pool: poison them
    for b in range(B):
        for j in range(nb):
            lo = j * bs
            for t in range(max(lo, int(lens[b])), lo + bs):
                ksp[table[b, j], :, t - lo] = np.nan
                vsp[table[b, j], :, t - lo] = np.nan
    return q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens


def _run_paged(q, Kp, Vp, ksp, vsp, table, lens, layout, partial=False, **kw):
    import torch

    tq, tK, tV, tks, tvs, tt, tl = _dev(q, Kp, Vp, ksp, vsp, table, lens)
    outs = []
    for _ in range(2):
        out = _poisoned(q.shape[:2] + (q.shape[2] + 4 if partial else q.shape[2],))
        kvd.paged_decode(tq, tK, tV, tks, tvs, tt, tl, out=out, layout=layout, partial=partial, **kw)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    assert np.array_equal(outs[0], outs[1], equal_nan=True)  # deterministic
    return outs[0], kvd.last_launch_count()


PAGED_CASES = [
    # B, Hq, Hkv, D, block_size, layout
    (4, 8, 8, 128, 16, "bhtd"),
    (4, 8, 8, 128, 8, "bthd"),
    (3, 16, 2, 128, 32, "bhtd"),
    (3, 32, 4, 128, 64, "bthd"),
    (2, 8, 1, 128, 128, "bhtd"),
    (2, 16, 2, 128, 256, "bthd"),
    (2, 16, 1, 128, 512, "bhtd"),
    (3, 4, 2, 64, 16, "bhtd"),    # head_dim 64: generic kernel
    (2, 4, 4, 128, 24, "bhtd"),   # block size not a power of two: generic kernel
    (2, 6, 2, 96, 8, "bthd"),     # head_dim 96: generic kernel
]


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,D,bs,layout", PAGED_CASES)
def test_paged_decode_matches_fp64_and_dense(B, Hq, Hkv, D, bs, layout):
    import torch

    rng = np.random.default_rng(B * 1000 + bs)
    lens = rng.integers(0, 1500, size=B).astype(np.int32)
    lens[0] = 1537  # one long sequence: several splits
    if B > 2:
        lens[1] = 0  # an empty sequence
    q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens = _paged_case(7 + bs, B, Hq, Hkv, D, bs, layout, lens)
    out, _ = _run_paged(q, Kp, Vp, ksp, vsp, table, lens, layout)
    ref = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    _check(out, ref, f"paged bs={bs} {layout}")
    # the dense decode of the cache the pool was scattered from: same plan, same bits
    tq, tK, tV, tks, tvs, tl = _dev(q, K, V, ks, vs, lens)
    dense = kvd.decode(tq, tK, tV, tks, tvs, seq_lens=tl)
    torch.cuda.synchronize()
    tc = D == 128 and bs >= 8 and (bs & (bs - 1)) == 0
    if tc:
        assert np.array_equal(out, dense.cpu().numpy()), "paged and dense tensor-core decode differ"
    assert kvd.device_status() == kvd.KVD_STATUS_OK


@pytest.mark.gpu
@pytest.mark.parametrize("bs", [16, 128])
def test_paged_partial_records_combine(bs):
    import torch

    B, Hq, Hkv, D = 2, 8, 2, 128
    lens = np.array([900, 433], np.int32)
    q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens = _paged_case(11, B, Hq, Hkv, D, bs, "bhtd", lens)
    rec, _ = _run_paged(q, Kp, Vp, ksp, vsp, table, lens, "bhtd", partial=True)
    # records -> normalised rows through the library's combine (one part each)
    parts = torch.from_numpy(rec.reshape(1, B * Hq, D + 4)).to(DEV)
    out = kvd.combine(parts).cpu().numpy().reshape(B, Hq, D)
    _check(out, po.decode_f64(q, K, V, ks, vs, seq_lens=lens), "paged records")


@pytest.mark.gpu
@pytest.mark.parametrize("D,bs", [(128, 16), (128, 256), (64, 16)])
def test_paged_bad_block_id_is_reported_not_read(D, bs):
    B, Hq, Hkv = 2, 4, 2
    lens = np.array([600, 300], np.int32)
    q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens = _paged_case(19, B, Hq, Hkv, D, bs, "bhtd", lens)
    assert kvd.device_status() == kvd.KVD_STATUS_OK
    table = table.copy()
    NB = Kp.shape[0]
    table[0, 1] = NB + 1000   # past the pool
    table[1, 0] = -7          # negative
    out, _ = _run_paged(q, Kp, Vp, ksp, vsp, table, lens, "bhtd")
    assert kvd.device_status() & kvd.KVD_STATUS_BAD_BLOCK
    assert np.isfinite(out).all()
    # tokens of a bad block count as score 0 with a zero value: check that rule
    # against the oracle on a cache where those tokens carry k = v = 0 codes and
    # scales of 0 (score 0 * scale = 0, value 0)
    Kx, Vx, ksx, vsx = K.copy(), V.copy(), ks.copy(), vs.copy()
    for b, j in ((0, 1), (1, 0)):
        sl = slice(j * bs, (j + 1) * bs)
        Kx[b, :, sl] = 0
        Vx[b, :, sl] = 0
        ksx[b, :, sl] = 0
        vsx[b, :, sl] = 0
    _check(out, po.decode_f64(q, Kx, Vx, ksx, vsx, seq_lens=lens), "bad block rule")


@pytest.mark.gpu
def test_paged_decode_launch_accounting():
    B, Hq, Hkv, D, bs = 4, 32, 32, 128, 16
    lens = np.array([4000, 100, 2048, 1], np.int32)
    q, K, V, ks, vs, Kp, Vp, ksp, vsp, table, lens = _paged_case(23, B, Hq, Hkv, D, bs, "bhtd", lens)
    out, launches = _run_paged(q, Kp, Vp, ksp, vsp, table, lens, "bhtd")
    _check(out, po.decode_f64(q, K, V, ks, vs, seq_lens=lens), "launches")
    assert 1 <= launches <= 3  # order kernel, decode, ragged combine


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["bhtd", "bthd"])
@pytest.mark.parametrize("bs", [16, 128])
def test_paged_append_bit_exact(layout, bs):
    import torch

    B, H, D = 5, 4, 128
    lens = np.array([0, 15, 16, 127, 250], np.int32)
    nb = 3 if bs == 128 else 17  # capacity 384 / 272 tokens
    q, K, V, ks, vs = po.random_cache(29, B, H, H, nb * bs, D)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, layout, seed=31)
    rng = np.random.default_rng(37)
    kn = rng.standard_normal((B, H, D), dtype=np.float32)
    vn = rng.standard_normal((B, H, D), dtype=np.float32)
    kn[2] = 0.0  # all-zero row: scale 0, codes 0
    tkn, tvn, tK, tV, tks, tvs, tt, tl = _dev(kn, vn, Kp, Vp, ksp, vsp, table, lens)
    kvd.paged_append(tkn, tvn, tK, tV, tks, tvs, tt, tl, layout=layout)
    torch.cuda.synchronize()
    assert kvd.device_status() == kvd.KVD_STATUS_OK
    assert np.array_equal(tl.cpu().numpy(), lens + 1)
    kc, kscale = po.quantize_rows(kn.reshape(-1, D))
    vc, vscale = po.quantize_rows(vn.reshape(-1, D))
    Kg, ksg = gather_from_pool(tK.cpu().numpy(), tks.cpu().numpy(), table, bs, layout, nb * bs)
    Vg, vsg = gather_from_pool(tV.cpu().numpy(), tvs.cpu().numpy(), table, bs, layout, nb * bs)
    for b in range(B):
        t = lens[b]
        assert np.array_equal(Kg[b, :, t], kc.reshape(B, H, D)[b])
        assert np.array_equal(Vg[b, :, t], vc.reshape(B, H, D)[b])
        assert np.array_equal(ksg[b, :, t].view(np.uint32), kscale.reshape(B, H)[b].view(np.uint32))
        assert np.array_equal(vsg[b, :, t].view(np.uint32), vscale.reshape(B, H)[b].view(np.uint32))
        # nothing else moved
        Kg[b, :, t] = K[b, :, t]
        Vg[b, :, t] = V[b, :, t]
        ksg[b, :, t] = ks[b, :, t]
        vsg[b, :, t] = vs[b, :, t]
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    assert np.array_equal(ksg, ks) and np.array_equal(vsg, vs)


@pytest.mark.gpu
def test_paged_append_full_and_bad_block():
    import torch

    B, H, D, bs = 3, 2, 64, 16
    q, K, V, ks, vs = po.random_cache(41, B, H, H, 2 * bs, D)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, "bhtd", seed=43)
    table = table.copy()
    table[2, 1] = -1
    lens = np.array([2 * bs, 5, bs + 3], np.int32)  # full, fine, bad block
    kn = np.ones((B, H, D), np.float32)
    tkn, tvn, tK, tV, tks, tvs, tt, tl = _dev(kn, kn, Kp, Vp, ksp, vsp, table, lens)
    before = tK.clone()
    kvd.paged_append(tkn, tvn, tK, tV, tks, tvs, tt, tl)
    torch.cuda.synchronize()
    st = kvd.device_status()
    assert st & kvd.KVD_STATUS_CACHE_FULL and st & kvd.KVD_STATUS_BAD_BLOCK
    assert np.array_equal(tl.cpu().numpy(), [2 * bs, 6, bs + 3])
    changed = (tK != before).nonzero()
    assert changed.shape[0] > 0 and set(changed[:, 0].tolist()) == {int(table[1, 0])}


@pytest.mark.gpu
def test_paged_append_then_decode_equals_dense():
    """The serving step: append one token to each sequence, then decode; paged
    and dense caches give the same bits."""
    import torch

    B, Hq, Hkv, D, bs = 4, 16, 2, 128, 32
    lens = np.array([100, 1023, 0, 511], np.int32)
    nb = 33
    q, K, V, ks, vs = po.random_cache(47, B, Hq, Hkv, nb * bs, D)
    Kp, Vp, ksp, vsp, table = scatter_to_pool(K, V, ks, vs, bs, "bhtd", seed=53)
    rng = np.random.default_rng(59)
    kn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    vn = rng.standard_normal((B, Hkv, D), dtype=np.float32)
    tkn, tvn, tq = _dev(kn, vn, q)
    pK, pV, pks, pvs, tt, pl = _dev(Kp, Vp, ksp, vsp, table, lens)
    dK, dV, dks, dvs, dl = _dev(K, V, ks, vs, lens)
    kvd.paged_append(tkn, tvn, pK, pV, pks, pvs, tt, pl)
    kvd.append(tkn, tvn, dK, dV, dks, dvs, dl)
    po_out = kvd.paged_decode(tq, pK, pV, pks, pvs, tt, pl)
    de_out = kvd.decode(tq, dK, dV, dks, dvs, seq_lens=dl)
    torch.cuda.synchronize()
    assert kvd.device_status() == kvd.KVD_STATUS_OK
    assert np.array_equal(po_out.cpu().numpy(), de_out.cpu().numpy())
    ref = po.decode_f64(q, dK.cpu().numpy(), dV.cpu().numpy(), dks.cpu().numpy(), dvs.cpu().numpy(),
                        seq_lens=lens + 1)
    _check(po_out.cpu().numpy(), ref, "append+decode")
