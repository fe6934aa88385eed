"""ctypes wrapper of the CPU oracle (oracle/libkvd_oracle.so) and of the
reference's own builds under oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py, always as the checker or the timed
CPU baseline, never as a product code path.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "libkvd_oracle.so"
REF_DIR = HERE / "_ref"

# Output tolerance of the north-star spec: |out - fp64| <= ATOL + RTOL*|fp64|.
ATOL = 2e-5
RTOL = 1e-4

P = ctypes.c_void_p
_lib = None


class Layout(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("seq_lens", P),
        ("kv_stride_b", ctypes.c_int64),
        ("kv_stride_h", ctypes.c_int64),
        ("sc_stride_b", ctypes.c_int64),
        ("sc_stride_h", ctypes.c_int64),
        ("q_stride_b", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("o_stride_b", ctypes.c_int64),
        ("o_stride_h", ctypes.c_int64),
        ("softmax_scale", ctypes.c_double),
    ]


def build() -> None:
    subprocess.run(["make", "-C", str(HERE), "oracle"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build()
        _lib = ctypes.CDLL(str(ORACLE_LIB))
        _lib.kvo_check.restype = ctypes.c_int64
        _lib.kvo_check.argtypes = [P, P, ctypes.c_int64, ctypes.c_double, ctypes.c_double, P, P]
        _lib.kvo_quantize_rows.argtypes = [P, ctypes.c_int64, ctypes.c_int, P, P]
        _lib.kvo_quantize_row.argtypes = [P, ctypes.c_int, P, P]
        _lib.kvo_cpu_reference_f32.argtypes = [P] * 6 + [ctypes.c_int] * 4
        _lib.kvo_decode_f64.argtypes = [ctypes.POINTER(Layout)] + [P] * 6 + [ctypes.c_int]
        _lib.kvo_partials_f64.argtypes = [ctypes.POINTER(Layout)] + [P] * 5 + [ctypes.c_int32] * 2 + [P]
        _lib.kvo_combine_f64.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        _lib.kvo_prefill_f64.argtypes = [ctypes.c_int] * 6 + [P] * 7 + [ctypes.c_double, P]
        _lib.kvo_fill_reference_pattern.argtypes = [P] * 5 + [ctypes.c_int] * 3
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous or a.ndim == 0
    return a.ctypes.data_as(P)


def quantize_rows(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    codes = np.empty(x.shape, dtype=np.int8)
    scales = np.empty(x.shape[:-1], dtype=np.float32)
    lib().kvo_quantize_rows(_p(x), rows, dim, _p(codes), _p(scales))
    return codes, scales


def quantize_rows_numpy(x: np.ndarray):
    """Independent numpy restatement of the quantiser (cross-checks the C one)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.fmax.reduce(np.abs(x), axis=-1, initial=np.float32(0.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        s = (amax / np.float32(127.0)).astype(np.float32)
        r = np.rint(x / s[..., None]).astype(np.float32)
    r = np.fmin(np.fmax(r, np.float32(-127.0)), np.float32(127.0))
    r = np.where(amax[..., None] == 0, np.float32(0), r)
    s = np.where(amax == 0, np.float32(0), s).astype(np.float32)
    return r.astype(np.int8), s


def cpu_reference_f32(Q, K, V, ks, vs, H: int, S: int, D: int, threads: int = 0) -> np.ndarray:
    out = np.empty(H * D, dtype=np.float32)
    lib().kvo_cpu_reference_f32(_p(Q), _p(K), _p(V), _p(ks), _p(vs), _p(out), H, S, D, threads)
    return out.reshape(H, D)


def _layout(q, k, ks, seq_lens, softmax_scale, max_seq_len=None):
    B, Hq, D = q.shape
    _, Hkv, cap, _ = k.shape
    L = Layout()
    L.batch, L.num_q_heads, L.num_kv_heads, L.head_dim = B, Hq, Hkv, D
    L.max_seq_len = cap if max_seq_len is None else max_seq_len
    L.seq_lens = seq_lens.ctypes.data if seq_lens is not None else None
    L.kv_stride_b, L.kv_stride_h = Hkv * cap * D, cap * D
    L.sc_stride_b, L.sc_stride_h = Hkv * cap, cap
    L.q_stride_b, L.q_stride_h = Hq * D, D
    L.o_stride_b, L.o_stride_h = Hq * D, D
    L.softmax_scale = softmax_scale
    return L


def decode_f64(q, K, V, ks, vs, seq_lens=None, softmax_scale: float = 0.0, threads: int = 0) -> np.ndarray:
    """FP64 oracle: q [B,Hq,D] fp32, K/V [B,Hkv,cap,D] int8, ks/vs [B,Hkv,cap] fp32."""
    q, K, V = (np.ascontiguousarray(a) for a in (q, K, V))
    ks, vs = np.ascontiguousarray(ks, dtype=np.float32), np.ascontiguousarray(vs, dtype=np.float32)
    lens = None if seq_lens is None else np.ascontiguousarray(seq_lens, dtype=np.int32)
    L = _layout(q, K, ks, lens, softmax_scale)
    out = np.empty(q.shape, dtype=np.float64)
    lib().kvo_decode_f64(ctypes.byref(L), _p(q), _p(K), _p(V), _p(ks), _p(vs), _p(out), threads)
    return out


def prefill_f64(q, K, V, ks, vs, seq_lens=None, q_lens=None, softmax_scale: float = 0.0) -> np.ndarray:
    """FP64 causal prefill: q [B,Hq,Lq,D] fp32, K/V [B,Hkv,cap,D] int8, ks/vs [B,Hkv,cap]; the
    queries are the last q_lens[b] of seq_lens[b] cached tokens (query i attends to tokens up
    to and including its own position). Rows past q_lens[b] are 0."""
    q, K, V = (np.ascontiguousarray(a) for a in (q, K, V))
    ks, vs = np.ascontiguousarray(ks, dtype=np.float32), np.ascontiguousarray(vs, dtype=np.float32)
    B, Hq, Lq, D = q.shape
    _, Hkv, cap, _ = K.shape
    lens = None if seq_lens is None else np.ascontiguousarray(seq_lens, dtype=np.int32)
    qls = None if q_lens is None else np.ascontiguousarray(q_lens, dtype=np.int32)
    out = np.empty(q.shape, dtype=np.float64)
    lib().kvo_prefill_f64(B, Hq, Hkv, Lq, cap, D, None if lens is None else _p(lens),
                          None if qls is None else _p(qls), _p(q), _p(K), _p(V), _p(ks), _p(vs),
                          ctypes.c_double(softmax_scale), _p(out))
    return out


def partials_f64(q, K, V, ks, vs, t_begin: int, t_end: int, seq_lens=None, softmax_scale: float = 0.0):
    """(m, l, o) records [B*Hq, D+2] over tokens [t_begin, t_end) (natural-log domain)."""
    q, K, V = (np.ascontiguousarray(a) for a in (q, K, V))
    lens = None if seq_lens is None else np.ascontiguousarray(seq_lens, dtype=np.int32)
    L = _layout(q, K, ks, lens, softmax_scale)
    B, Hq, D = q.shape
    part = np.empty((B * Hq, D + 2), dtype=np.float64)
    lib().kvo_partials_f64(ctypes.byref(L), _p(q), _p(K), _p(V), _p(np.ascontiguousarray(ks)),
                           _p(np.ascontiguousarray(vs)), t_begin, t_end, _p(part))
    return part


def combine_f64(parts: np.ndarray) -> np.ndarray:
    parts = np.ascontiguousarray(parts, dtype=np.float64)
    n, H, R = parts.shape
    out = np.empty((H, R - 2), dtype=np.float64)
    lib().kvo_combine_f64(_p(parts), n, H, R - 2, _p(out))
    return out


def check(actual, ref, atol: float = ATOL, rtol: float = RTOL):
    """Returns (bad_count, max_abs_err, max_normalised_err); NaN/Inf count as bad."""
    a = np.ascontiguousarray(actual, dtype=np.float32).ravel()
    r = np.ascontiguousarray(ref, dtype=np.float64).ravel()
    assert a.size == r.size
    ma, mn = ctypes.c_double(0), ctypes.c_double(0)
    bad = lib().kvo_check(_p(a), _p(r), a.size, atol, rtol, ctypes.byref(ma), ctypes.byref(mn))
    return int(bad), ma.value, mn.value


def reference_pattern(H: int, S: int, D: int):
    """Inputs of the reference's self-test (KV_int8_split_optimized.cu:473-486)."""
    Q = np.empty(H * D, np.float32)
    K = np.empty(H * S * D, np.int8)
    V = np.empty_like(K)
    ks = np.empty(H * S, np.float32)
    vs = np.empty_like(ks)
    lib().kvo_fill_reference_pattern(_p(Q), _p(K), _p(V), _p(ks), _p(vs), H, S, D)
    return Q, K, V, ks, vs


def random_cache(seed: int, B: int, Hq: int, Hkv: int, cap: int, D: int):
    """Seeded N(0,1) q and fp32 K/V quantised per token by the oracle quantiser."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32)
    kf = rng.standard_normal((B, Hkv, cap, D), dtype=np.float32)
    vf = rng.standard_normal((B, Hkv, cap, D), dtype=np.float32)
    K, ks = quantize_rows(kf)
    V, vs = quantize_rows(vf)
    return q, K, V, ks, vs


# --------------------------------------------------------- reference builds
def ref_lib(name: str):
    """oracle/_ref/libkvref_<name>.so, or None when it was not built here."""
    path = REF_DIR / f"libkvref_{name}.so"
    if not path.exists():
        return None
    h = ctypes.CDLL(str(path))
    if name == "split":
        h.kvref_cpu_reference.argtypes = [P] * 6 + [ctypes.c_int] * 3
        h.kvref_cpu_prepare.restype = P
        h.kvref_cpu_prepare.argtypes = [P] * 5 + [ctypes.c_int] * 3
        h.kvref_cpu_run.argtypes = [P]
        h.kvref_cpu_output.argtypes = [P, P]
        h.kvref_cpu_free.argtypes = [P]
        h.kvref_cpu_run_parallel.restype = ctypes.c_double
        h.kvref_cpu_run_parallel.argtypes = [ctypes.POINTER(P), ctypes.c_int]
        h.kvref_split_launch.restype = ctypes.c_int
        h.kvref_split_launch.argtypes = [P] * 6 + [ctypes.c_int] * 3 + [P, P]
        h.kvref_split_solve.argtypes = [P] * 6 + [ctypes.c_int] * 3
    elif name == "simple":
        h.kvref_simple_launch.restype = ctypes.c_int
        h.kvref_simple_launch.argtypes = [P] * 6 + [ctypes.c_int] * 3 + [P, P]
        h.kvref_simple_solve.argtypes = [P] * 6 + [ctypes.c_int] * 3
    else:
        getattr(h, f"kvref_{name}_solve").argtypes = [P] * 6 + [ctypes.c_int] * 3
    return h


def ref_cpu_reference(Q, K, V, ks, vs, H: int, S: int, D: int):
    h = ref_lib("split")
    if h is None:
        return None
    out = np.empty(H * D, np.float32)
    h.kvref_cpu_reference(_p(Q), _p(K), _p(V), _p(ks), _p(vs), _p(out), H, S, D)
    return out.reshape(H, D)
