"""Parity at the sizes the benchmark measures: every BASELINE configuration is
built at full size on the GPU (workload.make_case, the bench's own inputs), decoded
through the entry point bench.py times, and a seeded sample of at least 64 query
rows -- always the first and last sequence, the last kv head and, for the ragged
batch, the longest and shortest sequence -- is copied to the host and checked
against the FP64 oracle within the north-star tolerance. Outputs are poisoned
(0xFF) before each of two checked calls.

This is the acceptance check of the reference's own test `main`
(kv_cache/KV_int8_split_optimized.cu:515-543: decode, copy back, compare with
the host loop) at the configurations the benchmark reports. Configuration 3 holds
K and V tensors of exactly 2^31 bytes each, where 32-bit offsets would wrap."""
import numpy as np
import pytest
import torch

import kvdecode as kvd
import pyoracle as po
import workload as wl

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-5, 1e-4
SEED = 17


def _poison(t):
    t.view(torch.int32).fill_(-1)
    return t


def _sampled_f64(case, items, lens):
    """FP64 oracle rows for the sampled (b, kv head) items: [len(items), G, D]."""
    cfg = case.cfg
    G, D = cfg.group, cfg.head_dim
    n = len(items)
    L = max(lens[b] for b, _ in items) if lens is not None else case.K.shape[2]
    q = np.empty((n, G, D), np.float32)
    K = np.zeros((n, 1, L, D), np.int8)
    V = np.zeros((n, 1, L, D), np.int8)
    ks = np.zeros((n, 1, L), np.float32)
    vs = np.zeros((n, 1, L), np.float32)
    sl = np.empty(n, np.int32)
    for i, (b, hk) in enumerate(items):
        m = lens[b] if lens is not None else L
        sl[i] = m
        q[i] = case.q[b, hk * G:(hk + 1) * G].cpu().numpy()
        K[i, 0, :m] = case.K[b, hk, :m].cpu().numpy()
        V[i, 0, :m] = case.V[b, hk, :m].cpu().numpy()
        ks[i, 0, :m] = case.ks[b, hk, :m].cpu().numpy()
        vs[i, 0, :m] = case.vs[b, hk, :m].cpu().numpy()
    return po.decode_f64(q, K, V, ks, vs, seq_lens=sl)


def _rows(out, items, G):
    return np.stack([out[b, hk * G:(hk + 1) * G].float().cpu().numpy() for b, hk in items])


def _check(got, ref, what):
    bad, max_abs, max_norm = po.check(got, ref, ATOL, RTOL)
    assert bad == 0, f"{what}: {bad} bad elements, max abs {max_abs:.3g}, max normalised {max_norm:.3g}"


@pytest.mark.parametrize("config", [2, 3, 5])
def test_dense_config_at_full_size(config):
    cfg = wl.CONFIGS[config]
    case = wl.make_case(cfg, seed=SEED, device=DEV)
    items = wl.parity_items(cfg, cfg.batch)
    assert len(items) * cfg.group >= 64
    ref = _sampled_f64(case, items, None)
    out = torch.empty((cfg.batch, cfg.q_heads, cfg.head_dim), device=DEV)
    desc = kvd.make_desc(case.q, case.K, case.ks, out)
    ws = torch.empty(max(kvd.workspace_size(desc), 1), dtype=torch.uint8, device=DEV)
    for _ in range(2):
        _poison(out)
        kvd.decode(case.q, case.K, case.V, case.ks, case.vs, out=out, workspace=ws)
        torch.cuda.synchronize()
        _check(_rows(out, items, cfg.group), ref, f"config {config} kvd_decode_launch")
    assert kvd.device_status() == kvd.KVD_STATUS_OK
    if cfg.q_heads == cfg.kv_heads:  # the reference-facing entry point of the end-to-end timing
        H = cfg.batch * cfg.q_heads
        scratch = torch.empty(H * cfg.seq_len, dtype=torch.float32, device=DEV)
        _poison(out)
        rc = kvd.kv_int8_split_launch(case.q, case.K, case.V, case.ks, case.vs, out, H, cfg.seq_len, cfg.head_dim,
                                      scratch, torch.cuda.current_stream())
        assert rc == 0
        torch.cuda.synchronize()
        _check(_rows(out, items, cfg.group), ref, f"config {config} kv_int8_split_launch")


def test_ragged_append_config_at_full_size():
    cfg = wl.CONFIGS[4]
    case = wl.make_case(cfg, seed=SEED, device=DEV)
    lens0 = list(case.lens_host)
    lens1 = [n + 1 for n in lens0]
    items = wl.parity_items(cfg, cfg.batch, lens0)
    assert len(items) >= 64
    out = torch.empty((cfg.batch, cfg.q_heads, cfg.head_dim), device=DEV)
    desc = kvd.make_desc(case.q, case.K, case.ks, out, case.seq_lens)
    ws = torch.empty(max(kvd.workspace_size(desc), 1), dtype=torch.uint8, device=DEV)
    start = case.seq_lens.clone()
    ref = None
    for call in range(2):
        case.seq_lens.copy_(start)  # every step appends at the same positions, as the bench does
        _poison(out)
        kvd.append_decode(case.k_new, case.v_new, case.q, case.K, case.V, case.ks, case.vs, case.seq_lens,
                          out=out, workspace=ws)
        torch.cuda.synchronize()
        assert case.seq_lens.cpu().tolist() == lens1
        if ref is None:
            # the appended token: codes and scale bits equal the host quantiser's
            for b, hk in items:
                for new, cache, scale in ((case.k_new, case.K, case.ks), (case.v_new, case.V, case.vs)):
                    codes, sc = po.quantize_rows(new[b, hk].cpu().numpy()[None])
                    assert np.array_equal(cache[b, hk, lens0[b]].cpu().numpy(), codes[0])
                    assert scale[b, hk, lens0[b]].cpu().numpy().view(np.uint32) == sc.view(np.uint32)[0]
            ref = _sampled_f64(case, items, lens1)
        _check(_rows(out, items, cfg.group), ref, f"config 4 kvd_append_decode_launch, call {call}")
    assert kvd.device_status() == kvd.KVD_STATUS_OK
