"""GPU tests of the quantiser kernels: bit-exact INT8 codes and fp32 scale bit
patterns against the host spec (oracle), append semantics, and the ragged
configuration end to end (append, then decode with the new lengths)."""
import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_quantize_rows_golden_bit_exact(golden):
    x = torch.from_numpy(golden["quant_x"]).to(DEV)
    codes, scales = kvd.quantize_rows(x)
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), golden["quant_codes"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), golden["quant_scale_bits"])


@pytest.mark.parametrize("dim", [1, 37, 64, 96, 128, 512])
@pytest.mark.parametrize("seed", [17, 29, 101])
def test_quantize_rows_random_bit_exact(dim, seed):
    rng = np.random.default_rng(seed + dim)
    x = (rng.standard_normal((3000, dim)) * rng.uniform(1e-4, 1e4, (3000, 1))).astype(np.float32)
    x[5] = 0.0
    x[6, : dim // 2] = np.float32(0.5)  # ties after scaling
    c_ref, s_ref = po.quantize_rows(x)
    codes, scales = kvd.quantize_rows(torch.from_numpy(x).to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), c_ref)
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_quantize_rows_strided_in_and_out():
    x = np.random.default_rng(3).standard_normal((100, 128)).astype(np.float32)
    tx = torch.zeros((100, 160), device=DEV)
    tx[:, :128] = torch.from_numpy(x).to(DEV)
    codes = torch.zeros((100, 144), dtype=torch.int8, device=DEV)
    scales = torch.empty(100, device=DEV)
    kvd.quantize_rows(tx[:, :128], codes[:, :128], scales)
    torch.cuda.synchronize()
    c_ref, s_ref = po.quantize_rows(x)
    assert np.array_equal(codes[:, :128].cpu().numpy(), c_ref)
    assert torch.all(codes[:, 128:] == 0)


def _cache(B, H, cap, D, seed=0):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    K = torch.randint(-127, 128, (B, H, cap, D), generator=g, device=DEV, dtype=torch.int8)
    V = torch.randint(-127, 128, (B, H, cap, D), generator=g, device=DEV, dtype=torch.int8)
    ks = torch.rand((B, H, cap), generator=g, device=DEV)
    vs = torch.rand((B, H, cap), generator=g, device=DEV)
    return K, V, ks, vs


def test_append_writes_one_token_and_bumps_lengths():
    B, H, cap, D = 5, 4, 10, 128
    K, V, ks, vs = _cache(B, H, cap, D)
    K0, V0, ks0, vs0 = K.clone(), V.clone(), ks.clone(), vs.clone()
    lens0 = np.array([0, 3, 9, 5, 1], np.int32)
    lens = torch.tensor(lens0, device=DEV)
    rng = np.random.default_rng(1)
    kn = rng.standard_normal((B, H, D)).astype(np.float32)
    vn = rng.standard_normal((B, H, D)).astype(np.float32)
    kvd.append(torch.from_numpy(kn).to(DEV), torch.from_numpy(vn).to(DEV), K, V, ks, vs, lens)
    torch.cuda.synchronize()
    assert lens.cpu().numpy().tolist() == (lens0 + 1).tolist()
    ck, sk = po.quantize_rows(kn)
    cv, sv = po.quantize_rows(vn)
    Kh, Vh, ksh, vsh = (t.cpu().numpy() for t in (K, V, ks, vs))
    mask = np.zeros((B, H, cap), bool)
    for b in range(B):
        t = lens0[b]
        assert np.array_equal(Kh[b, :, t], ck[b]) and np.array_equal(Vh[b, :, t], cv[b])
        assert np.array_equal(ksh[b, :, t].view(np.uint32), sk[b].view(np.uint32))
        assert np.array_equal(vsh[b, :, t].view(np.uint32), sv[b].view(np.uint32))
        mask[b, :, t] = True
    # nothing else changed
    assert np.array_equal(Kh[~mask], K0.cpu().numpy()[~mask])
    assert np.array_equal(Vh[~mask], V0.cpu().numpy()[~mask])
    assert np.array_equal(ksh[~mask], ks0.cpu().numpy()[~mask])
    assert np.array_equal(vsh[~mask], vs0.cpu().numpy()[~mask])
    assert kvd.device_status() == kvd.KVD_STATUS_OK


def test_append_to_full_cache_reports_status_and_changes_nothing():
    B, H, cap, D = 2, 2, 4, 64
    K, V, ks, vs = _cache(B, H, cap, D, seed=1)
    K0 = K.clone()
    lens = torch.tensor([4, 2], dtype=torch.int32, device=DEV)
    kn = torch.randn((B, H, D), device=DEV)
    kvd.append(kn, kn.clone(), K, V, ks, vs, lens)
    assert kvd.device_status() == kvd.KVD_STATUS_CACHE_FULL
    assert lens.cpu().tolist() == [4, 3]
    assert torch.equal(K[0], K0[0])
    assert kvd.device_status() == kvd.KVD_STATUS_OK  # reading clears the word


def test_ragged_append_then_decode_end_to_end():
    """Configuration 4 at reduced batch: append one N(0,1) token per sequence,
    then decode with the incremented lengths; compare with the fp64 oracle on
    host copies."""
    import workload as wl

    cfg = wl.CONFIGS[4]
    case = wl.make_case(cfg, seed=17, batch=6)
    kvd.append(case.k_new, case.v_new, case.K, case.V, case.ks, case.vs, case.seq_lens)
    out = kvd.decode(case.q, case.K, case.V, case.ks, case.vs, seq_lens=case.seq_lens)
    torch.cuda.synchronize()
    lens = case.seq_lens.cpu().numpy()
    assert lens.tolist() == [n + 1 for n in case.lens_host]
    maxlen = int(lens.max())
    host = [t[:, :, :maxlen].cpu().numpy() for t in (case.K, case.V, case.ks, case.vs)]
    ref = po.decode_f64(case.q.cpu().numpy(), host[0], host[1], host[2], host[3], seq_lens=lens)
    bad, max_abs, _ = po.check(out.cpu().numpy(), ref)
    assert bad == 0, max_abs
    # the appended token holds exactly the host quantiser's codes
    b = 3
    ck, _ = po.quantize_rows(case.k_new[b].cpu().numpy())
    assert np.array_equal(host[0][b, :, lens[b] - 1], ck)
