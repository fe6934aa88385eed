"""CPU tests of the oracle itself: pinned against the reference's own host
loop (golden outputs produced by the reference build, and the live build when
oracle/_ref is present), the quantiser spec, and the split/combine algebra the
GPU path relies on."""
import numpy as np
import pytest

import pyoracle as po

PATTERN_SHAPES = [(4, 128, 64), (3, 129, 128), (2, 1, 64), (5, 257, 96), (1, 1000, 64), (8, 300, 128)]


@pytest.mark.parametrize("H,S,D", PATTERN_SHAPES)
def test_fp32_port_bit_exact_with_reference_golden(golden, H, S, D):
    Q, K, V, ks, vs = po.reference_pattern(H, S, D)
    out = po.cpu_reference_f32(Q, K, V, ks, vs, H, S, D, threads=4)
    ref = golden[f"pattern_{H}_{S}_{D}"]
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("H,S,D", PATTERN_SHAPES)
def test_fp64_oracle_agrees_with_reference_golden(golden, H, S, D):
    Q, K, V, ks, vs = po.reference_pattern(H, S, D)
    f64 = po.decode_f64(Q.reshape(1, H, D), K.reshape(1, H, S, D), V.reshape(1, H, S, D),
                        ks.reshape(1, H, S), vs.reshape(1, H, S))
    bad, max_abs, _ = po.check(golden[f"pattern_{H}_{S}_{D}"], f64[0])
    assert bad == 0, max_abs
    # the reference's own acceptance bound (KV_int8_split_optimized.cu:535)
    assert max_abs <= 1e-4


def test_random_golden(golden):
    q, K, V, ks, vs = (golden[k] for k in ("rand_q", "rand_k", "rand_v", "rand_ks", "rand_vs"))
    H, S, D = K.shape
    out = po.cpu_reference_f32(q, K, V, ks, vs, H, S, D)
    assert np.array_equal(out.view(np.uint32), golden["rand_out"].view(np.uint32))
    f64 = po.decode_f64(q[None], K[None], V[None], ks[None], vs[None])
    assert po.check(golden["rand_out"], f64[0])[0] == 0


def test_quantiser_golden(golden):
    x = golden["quant_x"]
    codes, scales = po.quantize_rows(x)
    assert np.array_equal(codes, golden["quant_codes"])
    assert np.array_equal(scales.view(np.uint32), golden["quant_scale_bits"])
    ncodes, nscales = po.quantize_rows_numpy(x)
    assert np.array_equal(ncodes, codes) and np.array_equal(nscales.view(np.uint32), scales.view(np.uint32))


def test_quantiser_ties_round_half_even():
    x = np.zeros((1, 16), np.float32)
    x[0, 0] = 127.0  # scale exactly 1
    x[0, 1:6] = [0.5, 1.5, 2.5, -0.5, -3.5]
    codes, scales = po.quantize_rows(x)
    assert scales[0] == 1.0
    assert codes[0, :6].tolist() == [127, 0, 2, 2, 0, -4]


@pytest.mark.parametrize("seed", [17, 29, 101])
def test_quantiser_random_bit_exact_c_vs_numpy(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((512, 128)).astype(np.float32) * rng.uniform(1e-3, 1e3, (512, 1)).astype(np.float32)
    c1, s1 = po.quantize_rows(x)
    c2, s2 = po.quantize_rows_numpy(x)
    assert np.array_equal(c1, c2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    assert np.abs(c1.astype(np.int32)).max() == 127  # the max element always maps to +-127


def test_checker_self_test():
    ref = np.array([0.0, 1.0])
    assert po.check(np.array([0.0, 1.0], np.float32), ref)[0] == 0
    assert po.check(np.array([np.nan, 1.0], np.float32), ref)[0] == 1
    assert po.check(np.array([np.inf, 1.0], np.float32), ref)[0] == 1
    assert po.check(np.array([0.0, 1.1], np.float32), ref)[0] == 1


@pytest.mark.parametrize("cuts", [[0, 37, 200], [0, 1, 2, 150, 200], [0, 200, 200]])
def test_split_partials_combine_to_full(cuts):
    q, K, V, ks, vs = po.random_cache(3, 2, 4, 4, 200, 64)
    full = po.decode_f64(q, K, V, ks, vs)
    parts = np.stack([po.partials_f64(q, K, V, ks, vs, a, b) for a, b in zip(cuts[:-1], cuts[1:])])
    comb = po.combine_f64(parts).reshape(full.shape)
    np.testing.assert_allclose(comb, full, rtol=1e-12, atol=1e-14)


def test_gqa_equals_expanded_heads():
    q, K, V, ks, vs = po.random_cache(7, 2, 8, 2, 96, 64)
    gqa = po.decode_f64(q, K, V, ks, vs)
    Ke, Ve = np.repeat(K, 4, axis=1), np.repeat(V, 4, axis=1)
    kse, vse = np.repeat(ks, 4, axis=1), np.repeat(vs, 4, axis=1)
    mha = po.decode_f64(q, Ke, Ve, kse, vse)
    np.testing.assert_array_equal(gqa, mha)


def test_ragged_equals_per_sequence():
    q, K, V, ks, vs = po.random_cache(11, 3, 4, 4, 130, 64)
    lens = np.array([130, 1, 77], np.int32)
    rag = po.decode_f64(q, K, V, ks, vs, seq_lens=lens)
    for b, n in enumerate(lens):
        one = po.decode_f64(q[b:b + 1], K[b:b + 1, :, :n], V[b:b + 1, :, :n], ks[b:b + 1, :, :n], vs[b:b + 1, :, :n])
        np.testing.assert_array_equal(rag[b], one[0])
    zero = po.decode_f64(q, K, V, ks, vs, seq_lens=np.array([0, 5, 0], np.int32))
    assert np.all(zero[0] == 0) and np.all(zero[2] == 0)


@pytest.mark.skipif(po.ref_lib("split") is None, reason="reference not built here (oracle/_ref)")
@pytest.mark.parametrize("H,S,D", [(3, 333, 128), (6, 64, 64), (2, 700, 80)])
def test_live_reference_host_loop_matches_port(H, S, D):
    rng = np.random.default_rng(H * S + D)
    q = rng.standard_normal((H, D), dtype=np.float32)
    K, ks = po.quantize_rows(rng.standard_normal((H, S, D), dtype=np.float32))
    V, vs = po.quantize_rows(rng.standard_normal((H, S, D), dtype=np.float32))
    ref = po.ref_cpu_reference(q, K, V, ks, vs, H, S, D)
    port = po.cpu_reference_f32(q, K, V, ks, vs, H, S, D)
    assert np.array_equal(ref.view(np.uint32), port.view(np.uint32))
