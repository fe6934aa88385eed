"""Python host side of libkvdecode_b200.so (ctypes over the C ABI in include/kvdecode.h).

The reference (Murmurwkk/cuda-operators kv_cache/*.cu) is driven from host
C++ through ``extern "C"`` entry points; this module exposes the same entry
points with the same names and argument meaning (``solve``,
``kv_int8_split_launch``, ``kv_int8_simple_launch``) plus the extended API
(batched / GQA / ragged decode, quantise-on-append, row quantisation, LSE
combine). Device memory comes from torch tensors; torch is only plumbing
here -- every computation runs in the library's CUDA kernels. There is no
CPU fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import math
import os
import re
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
LIB_PATH = HERE / "libkvdecode_b200.so"
HEADER = ROOT / "include" / "kvdecode.h"

KVD_FLAG_PARTIAL_OUT = 1
KVD_FLAG_Q_BF16 = 2
KVD_FLAG_Q_F16 = 4
KVD_FLAG_OUT_BF16 = 8
KVD_FLAG_OUT_F16 = 16
KVD_FLAG_QK_INT8 = 32
KVD_STATUS_OK = 0
KVD_STATUS_WAIT_TIMEOUT = 1
KVD_STATUS_CACHE_FULL = 2
KVD_STATUS_BAD_BLOCK = 4
CUDA_ERROR_INVALID_VALUE = 1

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_uint32 = ctypes.c_uint32
c_size_t = ctypes.c_size_t
c_float = ctypes.c_float


class DecodeDesc(ctypes.Structure):
    """Mirror of ``kvd_decode_desc``."""

    _fields_ = [
        ("batch", c_int32),
        ("num_q_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("max_seq_len", c_int32),
        ("flags", c_uint32),
        ("seq_lens", c_void_p),
        ("kv_stride_b", c_int64),
        ("kv_stride_h", c_int64),
        ("sc_stride_b", c_int64),
        ("sc_stride_h", c_int64),
        ("q_stride_b", c_int64),
        ("q_stride_h", c_int64),
        ("o_stride_b", c_int64),
        ("o_stride_h", c_int64),
        ("softmax_scale", c_float),
    ]


class AppendDesc(ctypes.Structure):
    """Mirror of ``kvd_append_desc``."""

    _fields_ = [
        ("batch", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("capacity", c_int32),
        ("kv_stride_b", c_int64),
        ("kv_stride_h", c_int64),
        ("sc_stride_b", c_int64),
        ("sc_stride_h", c_int64),
        ("new_stride_b", c_int64),
        ("new_stride_h", c_int64),
    ]


class PagedDesc(ctypes.Structure):
    """Mirror of ``kvd_paged_desc``."""

    _fields_ = [
        ("batch", c_int32),
        ("num_q_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("block_size", c_int32),
        ("num_blocks", c_int32),
        ("max_blocks_per_seq", c_int32),
        ("flags", c_uint32),
        ("seq_lens", c_void_p),
        ("block_table", c_void_p),
        ("block_table_stride", c_int64),
        ("kv_stride_block", c_int64),
        ("kv_stride_h", c_int64),
        ("kv_stride_t", c_int64),
        ("sc_stride_block", c_int64),
        ("sc_stride_h", c_int64),
        ("q_stride_b", c_int64),
        ("q_stride_h", c_int64),
        ("o_stride_b", c_int64),
        ("o_stride_h", c_int64),
        ("softmax_scale", c_float),
    ]


class PrefillDesc(ctypes.Structure):
    """Mirror of ``kvd_prefill_desc``."""

    _fields_ = [
        ("batch", c_int32),
        ("num_q_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("max_seq_len", c_int32),
        ("max_queries", c_int32),
        ("flags", c_uint32),
        ("seq_lens", c_void_p),
        ("q_lens", c_void_p),
        ("kv_stride_b", c_int64),
        ("kv_stride_h", c_int64),
        ("sc_stride_b", c_int64),
        ("sc_stride_h", c_int64),
        ("q_stride_b", c_int64),
        ("q_stride_h", c_int64),
        ("q_stride_t", c_int64),
        ("o_stride_b", c_int64),
        ("o_stride_h", c_int64),
        ("o_stride_t", c_int64),
        ("softmax_scale", c_float),
    ]


_SIGNATURES = {
    "solve": (None, [c_void_p] * 6 + [c_int] * 3),
    "kv_int8_split_launch": (c_int, [c_void_p] * 6 + [c_int] * 3 + [c_void_p, c_void_p]),
    "kv_int8_simple_launch": (c_int, [c_void_p] * 6 + [c_int] * 3 + [c_void_p, c_void_p]),
    "kvd_workspace_size": (c_size_t, [ctypes.POINTER(DecodeDesc)]),
    "kvd_decode_launch": (c_int, [ctypes.POINTER(DecodeDesc)] + [c_void_p] * 7 + [c_size_t, c_void_p]),
    "kvd_combine_launch": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_int64, c_uint32, c_void_p]),
    "kvd_append_int8_launch": (c_int, [ctypes.POINTER(AppendDesc)] + [c_void_p] * 7 + [c_void_p]),
    "kvd_quantize_rows_launch": (c_int, [c_void_p, c_int64, c_int, c_int64, c_void_p, c_int64, c_void_p, c_void_p]),
    "kvd_device_status": (c_int, [ctypes.POINTER(c_int32)]),
    "kvd_last_launch_count": (c_int, []),
    "kvd_abi_version": (c_int, []),
    "kvd_error_string": (ctypes.c_char_p, [c_int]),
    "kvd_decode_launch_noalloc": (c_int, [ctypes.POINTER(DecodeDesc)] + [c_void_p] * 6 + [c_void_p]),
    "kvd_append_decode_launch": (c_int, [ctypes.POINTER(DecodeDesc), c_void_p, c_void_p, c_int64, c_int64]
                                 + [c_void_p] * 6 + [c_void_p, c_size_t, c_void_p]),
    "kvd_mgpu_get_unique_id": (c_int, [c_void_p]),
    "kvd_mgpu_comm_init": (c_int, [ctypes.POINTER(c_void_p), c_int, c_int, c_void_p]),
    "kvd_mgpu_comm_destroy": (c_int, [c_void_p]),
    "kvd_mgpu_seq_split_workspace_size": (c_size_t, [ctypes.POINTER(DecodeDesc), c_int]),
    "kvd_mgpu_seq_split_decode": (c_int, [ctypes.POINTER(DecodeDesc)] + [c_void_p] * 6
                                  + [c_void_p, c_size_t, c_void_p, c_int, c_void_p]),
    "kvd_mgpu_p2p_create": (c_int, [ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_void_p, c_int, c_int]),
    "kvd_mgpu_p2p_destroy": (c_int, [c_void_p]),
    "kvd_mgpu_p2p_reset": (c_int, [c_void_p, c_void_p]),
    "kvd_mgpu_p2p_create_group": (c_int, [ctypes.POINTER(c_void_p), c_int, ctypes.POINTER(c_int), c_int, c_int, c_int]),
    "kvd_mgpu_p2p_workspace_size": (c_size_t, [ctypes.POINTER(DecodeDesc)]),
    "kvd_mgpu_p2p_seq_split_decode": (c_int, [c_void_p, ctypes.POINTER(DecodeDesc)] + [c_void_p] * 6
                                      + [c_void_p, c_size_t, c_void_p]),
    "kvd_prefill_workspace_size": (c_size_t, [ctypes.POINTER(PrefillDesc)]),
    "kvd_prefill_launch": (c_int, [ctypes.POINTER(PrefillDesc)] + [c_void_p] * 7 + [c_size_t, c_void_p]),
    "kvd_paged_workspace_size": (c_size_t, [ctypes.POINTER(PagedDesc)]),
    "kvd_paged_decode_launch": (c_int, [ctypes.POINTER(PagedDesc)] + [c_void_p] * 7 + [c_size_t, c_void_p]),
    "kvd_paged_append_int8_launch": (c_int, [ctypes.POINTER(PagedDesc), c_void_p, c_void_p, c_int64, c_int64]
                                     + [c_void_p] * 5 + [c_void_p]),
}

NOALLOC_SCRATCH_BYTES = 512 * 1024

_lib = None


def build(force: bool = False) -> Path:
    """Compile libkvdecode_b200.so in place with nvcc (sm_100a)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-C", str(HERE), "-j8"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the library (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; build it with `make -C {HERE}`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def header_functions() -> list[str]:
    """Names of every function declared in include/kvdecode.h."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", text, flags=re.M)
    return sorted(set(names))


class KvdError(RuntimeError):
    def __init__(self, code: int, where: str):
        self.code = code
        msg = lib().kvd_error_string(code)
        super().__init__(f"{where} failed: cuda error {code} ({msg.decode() if msg else '?'})")


def _check(code: int, where: str) -> None:
    if code != 0:
        raise KvdError(code, where)


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ---------------------------------------------------------------- reference ABI
def solve(Q, K_int8, V_int8, k_scale, v_scale, output, num_heads: int, seq_len: int, head_dim: int) -> None:
    """``solve`` of kv_cache/*.cu: default stream, no synchronisation, no return value."""
    lib().solve(_ptr(Q), _ptr(K_int8), _ptr(V_int8), _ptr(k_scale), _ptr(v_scale), _ptr(output),
                num_heads, seq_len, head_dim)


def kv_int8_split_launch(Q, K_int8, V_int8, k_scale, v_scale, output, num_heads, seq_len, head_dim, S,
                         stream=None) -> int:
    """Returns the cudaError_t code, like kv_cache/KV_int8_split_optimized.cu:268-292."""
    return lib().kv_int8_split_launch(_ptr(Q), _ptr(K_int8), _ptr(V_int8), _ptr(k_scale), _ptr(v_scale),
                                      _ptr(output), num_heads, seq_len, head_dim, _ptr(S), _stream(stream))


def kv_int8_simple_launch(Q, K_int8, V_int8, k_scale, v_scale, output, num_heads, seq_len, head_dim, S,
                          stream=None) -> int:
    """Returns the cudaError_t code, like kv_cache/new_kvint8.cu:85-100."""
    return lib().kv_int8_simple_launch(_ptr(Q), _ptr(K_int8), _ptr(V_int8), _ptr(k_scale), _ptr(v_scale),
                                       _ptr(output), num_heads, seq_len, head_dim, _ptr(S), _stream(stream))


# ----------------------------------------------------------------- extended API
def dtype_flags(q=None, out=None, partial: bool = False) -> int:
    """Decode flags for the element types of ``q`` and ``out`` (torch tensors:
    float32, bfloat16 or float16)."""
    import torch

    f = KVD_FLAG_PARTIAL_OUT if partial else 0
    qmap = {torch.float32: 0, torch.bfloat16: KVD_FLAG_Q_BF16, torch.float16: KVD_FLAG_Q_F16}
    omap = {torch.float32: 0, torch.bfloat16: KVD_FLAG_OUT_BF16, torch.float16: KVD_FLAG_OUT_F16}
    if q is not None:
        if q.dtype not in qmap:
            raise ValueError(f"unsupported query dtype {q.dtype}")
        f |= qmap[q.dtype]
    if out is not None and out.device.type != "meta":
        if out.dtype not in omap:
            raise ValueError(f"unsupported output dtype {out.dtype}")
        if partial and out.dtype != torch.float32:
            raise ValueError("partial records are float32")
        f |= omap[out.dtype]
    return f


def make_desc(q, k, ks, out, seq_lens=None, max_seq_len: int | None = None, softmax_scale: float = 0.0,
              partial: bool = False, qk_int8: bool = False) -> DecodeDesc:
    """Descriptor for q [B,Hq,D], k/v [B,Hkv,cap,D] int8, ks/vs [B,Hkv,cap], out [B,Hq,D or D+4].
    ``qk_int8`` selects the INT8 Q.K mode (KVD_FLAG_QK_INT8: the query is rounded per head
    to int8 by the cache's quantiser rule)."""
    B, Hq, D = q.shape
    Bk, Hkv, cap, Dk = k.shape
    if Bk != B or Dk != D or Hq % Hkv:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)}")
    if k.stride(3) != 1 or k.stride(2) != D or ks.stride(2) != 1 or q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("token rows must be contiguous (d stride 1, K/V token stride D, scale token stride 1)")
    d = DecodeDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim = B, Hq, Hkv, D
    d.max_seq_len = cap if max_seq_len is None else max_seq_len
    d.flags = dtype_flags(q, out, partial) | (KVD_FLAG_QK_INT8 if qk_int8 else 0)
    d.seq_lens = _ptr(seq_lens)
    d.kv_stride_b, d.kv_stride_h = k.stride(0), k.stride(1)
    d.sc_stride_b, d.sc_stride_h = ks.stride(0), ks.stride(1)
    d.q_stride_b, d.q_stride_h = q.stride(0), q.stride(1)
    d.o_stride_b, d.o_stride_h = out.stride(0), out.stride(1)
    d.softmax_scale = softmax_scale
    return d


def workspace_size(desc: DecodeDesc) -> int:
    return int(lib().kvd_workspace_size(ctypes.byref(desc)))


def decode(q, k, v, ks, vs, out=None, seq_lens=None, softmax_scale: float = 0.0, partial: bool = False,
           workspace=None, max_seq_len: int | None = None, stream=None, out_dtype=None, qk_int8: bool = False):
    """Split-KV INT8 decode attention; returns ``out`` ([B,Hq,D], or [B,Hq,D+4] records if partial).
    ``q`` may be float32, bfloat16 or float16; the output type is ``out``'s (or ``out_dtype``,
    default float32). ``qk_int8`` selects the INT8 Q.K mode (looser, stated tolerance)."""
    import torch

    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq, D + 4 if partial else D), dtype=out_dtype or torch.float32, device=q.device)
    if v.stride() != k.stride() or vs.stride() != ks.stride():
        raise ValueError("K/V and k_scale/v_scale must share strides")
    desc = make_desc(q, k, ks, out, seq_lens, max_seq_len, softmax_scale, partial, qk_int8)
    if workspace is None:
        n = workspace_size(desc)
        workspace = torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)
    rc = lib().kvd_decode_launch(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs), _ptr(out),
                                 _ptr(workspace), workspace.numel(), _stream(stream))
    _check(rc, "kvd_decode_launch")
    return out


def decode_noalloc(q, k, v, ks, vs, out, seq_lens=None, softmax_scale: float = 0.0, partial: bool = False,
                   max_seq_len: int | None = None, stream=None):
    """Same decode for callers that may not allocate device memory: the
    library's fixed scratch array replaces the workspace, so this allocates
    nothing (``out`` must be given). Calls that overlap on the GPU race on that
    array; the first call on a device should not be inside a stream capture."""
    if v.stride() != k.stride() or vs.stride() != ks.stride():
        raise ValueError("K/V and k_scale/v_scale must share strides")
    desc = make_desc(q, k, ks, out, seq_lens, max_seq_len, softmax_scale, partial)
    rc = lib().kvd_decode_launch_noalloc(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs),
                                         _ptr(out), _stream(stream))
    _check(rc, "kvd_decode_launch_noalloc")
    return out


def combine(parts, out=None, partial: bool = False, stream=None, out_dtype=None):
    """LSE-combine records ``parts`` [P, H, D+4] into out [H, D] (or [H, D+4] records)."""
    import torch

    P, H, R = parts.shape
    D = R - 4
    if out is None:
        out = torch.empty((H, R if partial else D), dtype=out_dtype or torch.float32, device=parts.device)
    rc = lib().kvd_combine_launch(_ptr(parts), P, parts.stride(0), H, D, _ptr(out), out.stride(0),
                                  dtype_flags(None, out, partial), _stream(stream))
    _check(rc, "kvd_combine_launch")
    return out


def append(k_new, v_new, K, V, ks, vs, seq_lens, stream=None) -> None:
    """Quantise-on-append of one token per (b, h): k_new/v_new [B,Hkv,D] fp32 into the cache."""
    B, H, D = k_new.shape
    d = AppendDesc()
    d.batch, d.num_kv_heads, d.head_dim, d.capacity = B, H, D, K.shape[2]
    d.kv_stride_b, d.kv_stride_h = K.stride(0), K.stride(1)
    d.sc_stride_b, d.sc_stride_h = ks.stride(0), ks.stride(1)
    d.new_stride_b, d.new_stride_h = k_new.stride(0), k_new.stride(1)
    if v_new.stride() != k_new.stride() or V.stride() != K.stride() or vs.stride() != ks.stride():
        raise ValueError("K/V (and their scales, and the new rows) must share strides")
    rc = lib().kvd_append_int8_launch(ctypes.byref(d), _ptr(k_new), _ptr(v_new), _ptr(K), _ptr(V), _ptr(ks),
                                      _ptr(vs), _ptr(seq_lens), _stream(stream))
    _check(rc, "kvd_append_int8_launch")


def append_decode(k_new, v_new, q, k, v, ks, vs, seq_lens, out=None, workspace=None, softmax_scale: float = 0.0,
                  partial: bool = False, stream=None, out_dtype=None, qk_int8: bool = False):
    """Quantise-on-append of one token per (b, kv head) and the decode over the grown
    cache in one decode launch (``kvd_append_decode_launch``); ``seq_lens`` is updated."""
    import torch

    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq, D + 4 if partial else D), dtype=out_dtype or torch.float32, device=q.device)
    if v.stride() != k.stride() or vs.stride() != ks.stride() or v_new.stride() != k_new.stride():
        raise ValueError("K/V (and their scales, and the new rows) must share strides")
    desc = make_desc(q, k, ks, out, seq_lens, None, softmax_scale, partial, qk_int8)
    if workspace is None:
        workspace = torch.empty(max(workspace_size(desc), 1), dtype=torch.uint8, device=q.device)
    rc = lib().kvd_append_decode_launch(ctypes.byref(desc), _ptr(k_new), _ptr(v_new), k_new.stride(0),
                                        k_new.stride(1), _ptr(q), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs), _ptr(out),
                                        _ptr(workspace), workspace.numel(), _stream(stream))
    _check(rc, "kvd_append_decode_launch")
    return out


def make_prefill_desc(q, k, ks, out, seq_lens=None, q_lens=None, softmax_scale: float = 0.0) -> PrefillDesc:
    """Descriptor for q [B,Hq,Lq,D], k/v [B,Hkv,cap,D] int8, ks/vs [B,Hkv,cap], out [B,Hq,Lq,D]."""
    B, Hq, Lq, D = q.shape
    Bk, Hkv, cap, Dk = k.shape
    if Bk != B or Dk != D or Hq % Hkv or tuple(out.shape) != (B, Hq, Lq, D):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} out{tuple(out.shape)}")
    if k.stride(3) != 1 or k.stride(2) != D or ks.stride(2) != 1 or q.stride(3) != 1 or out.stride(3) != 1:
        raise ValueError("token rows must be contiguous")
    d = PrefillDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim = B, Hq, Hkv, D
    d.max_seq_len, d.max_queries = cap, Lq
    d.flags = dtype_flags(q, out)
    d.seq_lens, d.q_lens = _ptr(seq_lens), _ptr(q_lens)
    d.kv_stride_b, d.kv_stride_h = k.stride(0), k.stride(1)
    d.sc_stride_b, d.sc_stride_h = ks.stride(0), ks.stride(1)
    d.q_stride_b, d.q_stride_h, d.q_stride_t = q.stride(0), q.stride(1), q.stride(2)
    d.o_stride_b, d.o_stride_h, d.o_stride_t = out.stride(0), out.stride(1), out.stride(2)
    d.softmax_scale = softmax_scale
    return d


def prefill(q, k, v, ks, vs, seq_lens=None, q_lens=None, out=None, softmax_scale: float = 0.0, out_dtype=None,
            workspace=None, stream=None):
    """Causal prefill attention over the INT8 cache; q [B,Hq,Lq,D] holds the last q_lens[b]
    (default Lq) of the seq_lens[b] (default cap) cached tokens. Returns out [B,Hq,Lq,D]."""
    import torch

    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype or torch.float32, device=q.device)
    if v.stride() != k.stride() or vs.stride() != ks.stride():
        raise ValueError("K/V and k_scale/v_scale must share strides")
    desc = make_prefill_desc(q, k, ks, out, seq_lens, q_lens, softmax_scale)
    if workspace is None:
        workspace = torch.empty(max(int(lib().kvd_prefill_workspace_size(ctypes.byref(desc))), 1),
                                dtype=torch.uint8, device=q.device)
    rc = lib().kvd_prefill_launch(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs), _ptr(out),
                                  _ptr(workspace), workspace.numel(), _stream(stream))
    _check(rc, "kvd_prefill_launch")
    return out


def quantize_rows(x, codes=None, scales=None, stream=None):
    """Quantise a 2-D fp32 tensor row by row; returns (codes int8 like x, scales [rows])."""
    import torch

    rows, dim = x.shape
    if codes is None:
        codes = torch.empty((rows, dim), dtype=torch.int8, device=x.device)
    if scales is None:
        scales = torch.empty((rows,), dtype=torch.float32, device=x.device)
    rc = lib().kvd_quantize_rows_launch(_ptr(x), rows, dim, x.stride(0), _ptr(codes), codes.stride(0),
                                        _ptr(scales), _stream(stream))
    _check(rc, "kvd_quantize_rows_launch")
    return codes, scales


# ------------------------------------------------------------------ paged cache
def make_paged_desc(q, k_pool, ks_pool, out, block_table, seq_lens, layout: str = "bhtd",
                    softmax_scale: float = 0.0, partial: bool = False, qk_int8: bool = False) -> PagedDesc:
    """Descriptor for a paged cache. ``k_pool`` is [blocks, Hkv, block_size, D]
    (layout "bhtd") or [blocks, block_size, Hkv, D] (layout "bthd"); scale pools
    are [blocks, Hkv, block_size]; ``block_table`` is int32 [B, max_blocks]."""
    B, Hq, D = q.shape
    if layout == "bhtd":
        NB, Hkv, bs, Dk = k_pool.shape
        s_blk, s_h, s_t = k_pool.stride(0), k_pool.stride(1), k_pool.stride(2)
    elif layout == "bthd":
        NB, bs, Hkv, Dk = k_pool.shape
        s_blk, s_t, s_h = k_pool.stride(0), k_pool.stride(1), k_pool.stride(2)
    else:
        raise ValueError(f"unknown pool layout {layout!r}")
    if Dk != D or Hq % Hkv or tuple(ks_pool.shape) != (NB, Hkv, bs):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k_pool{tuple(k_pool.shape)} ks{tuple(ks_pool.shape)}")
    if k_pool.stride(3) != 1 or ks_pool.stride(2) != 1 or q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("dims and scale tokens must be contiguous")
    if block_table.dim() != 2 or block_table.shape[0] != B or block_table.stride(1) != 1:
        raise ValueError("block_table must be int32 [B, max_blocks] with contiguous rows")
    d = PagedDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim = B, Hq, Hkv, D
    d.block_size, d.num_blocks, d.max_blocks_per_seq = bs, NB, block_table.shape[1]
    d.flags = dtype_flags(q if q.device.type != "meta" else None, out, partial) | (KVD_FLAG_QK_INT8 if qk_int8 else 0)
    d.seq_lens, d.block_table = _ptr(seq_lens), _ptr(block_table)
    d.block_table_stride = block_table.stride(0)
    d.kv_stride_block, d.kv_stride_h, d.kv_stride_t = s_blk, s_h, s_t
    d.sc_stride_block, d.sc_stride_h = ks_pool.stride(0), ks_pool.stride(1)
    d.q_stride_b, d.q_stride_h = q.stride(0), q.stride(1)
    d.o_stride_b, d.o_stride_h = out.stride(0), out.stride(1)
    d.softmax_scale = softmax_scale
    return d


def paged_workspace_size(desc: PagedDesc) -> int:
    return int(lib().kvd_paged_workspace_size(ctypes.byref(desc)))


def paged_decode(q, k_pool, v_pool, ks_pool, vs_pool, block_table, seq_lens, out=None, layout: str = "bhtd",
                 softmax_scale: float = 0.0, partial: bool = False, workspace=None, stream=None, out_dtype=None,
                 qk_int8: bool = False):
    """INT8 decode attention over a paged cache; returns ``out`` [B,Hq,D] (or records)."""
    import torch

    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq, D + 4 if partial else D), dtype=out_dtype or torch.float32, device=q.device)
    if v_pool.stride() != k_pool.stride() or vs_pool.stride() != ks_pool.stride():
        raise ValueError("K/V pools and their scale pools must share strides")
    desc = make_paged_desc(q, k_pool, ks_pool, out, block_table, seq_lens, layout, softmax_scale, partial, qk_int8)
    if workspace is None:
        workspace = torch.empty(max(paged_workspace_size(desc), 1), dtype=torch.uint8, device=q.device)
    rc = lib().kvd_paged_decode_launch(ctypes.byref(desc), _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(ks_pool),
                                       _ptr(vs_pool), _ptr(out), _ptr(workspace), workspace.numel(),
                                       _stream(stream))
    _check(rc, "kvd_paged_decode_launch")
    return out


def paged_append(k_new, v_new, k_pool, v_pool, ks_pool, vs_pool, block_table, seq_lens, layout: str = "bhtd",
                 stream=None) -> None:
    """Quantise-on-append of one token per (b, kv head) into a paged cache."""
    import torch

    B, Hkv, D = k_new.shape
    if v_new.stride() != k_new.stride() or v_pool.stride() != k_pool.stride() or vs_pool.stride() != ks_pool.stride():
        raise ValueError("K/V (and their scales, and the new rows) must share strides")
    q_like = torch.empty((B, Hkv, D), dtype=torch.float32, device="meta")
    desc = make_paged_desc(q_like, k_pool, ks_pool, q_like, block_table, seq_lens, layout)
    rc = lib().kvd_paged_append_int8_launch(ctypes.byref(desc), _ptr(k_new), _ptr(v_new), k_new.stride(0),
                                            k_new.stride(1), _ptr(k_pool), _ptr(v_pool), _ptr(ks_pool),
                                            _ptr(vs_pool), _ptr(seq_lens), _stream(stream))
    _check(rc, "kvd_paged_append_int8_launch")


# ------------------------------------------------------------------ multi-GPU
def mgpu_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (made on one rank, broadcast by the caller)."""
    buf = (ctypes.c_ubyte * 128)()
    rc = lib().kvd_mgpu_get_unique_id(ctypes.addressof(buf))
    if rc != 0:
        raise RuntimeError(f"kvd_mgpu_get_unique_id failed: nccl error {rc}")
    return bytes(buf)


class MgpuComm:
    """An NCCL communicator made by the library (kvd_mgpu_comm_init)."""

    def __init__(self, nranks: int, rank: int, uid: bytes):
        buf = (ctypes.c_ubyte * 128).from_buffer_copy(uid)
        h = c_void_p()
        rc = lib().kvd_mgpu_comm_init(ctypes.byref(h), nranks, rank, ctypes.addressof(buf))
        if rc != 0:
            raise RuntimeError(f"kvd_mgpu_comm_init failed: nccl error {rc}")
        self.handle, self.nranks, self.rank = h.value, nranks, rank

    def close(self) -> None:
        if self.handle:
            lib().kvd_mgpu_comm_destroy(self.handle)
            self.handle = None


def seq_split_decode(comm: MgpuComm, q, k, v, ks, vs, out=None, seq_lens=None, workspace=None, stream=None,
                     out_dtype=None):
    """Sequence-split decode (kvd_mgpu_seq_split_decode): this rank passes its own token
    range of the cache; every rank gets the merged output rows."""
    import torch

    B, Hq, D = q.shape
    if out is None:
        out = torch.empty((B, Hq, D), dtype=out_dtype or torch.float32, device=q.device)
    desc = make_desc(q, k, ks, out, seq_lens)
    if workspace is None:
        n = int(lib().kvd_mgpu_seq_split_workspace_size(ctypes.byref(desc), comm.nranks))
        workspace = torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)
    rc = lib().kvd_mgpu_seq_split_decode(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs),
                                         _ptr(out), _ptr(workspace), workspace.numel(), comm.handle, comm.nranks,
                                         _stream(stream))
    _check(rc, "kvd_mgpu_seq_split_decode")
    return out


class P2PExchange:
    """Sequence-split exchange over NVLink peer stores (kvd_mgpu_p2p_*); collective to create."""

    def __init__(self, comm: MgpuComm, batch: int, num_q_heads: int, head_dim: int):
        h = c_void_p()
        _check(lib().kvd_mgpu_p2p_create(ctypes.byref(h), batch, num_q_heads, head_dim, comm.handle, comm.nranks,
                                         comm.rank), "kvd_mgpu_p2p_create")
        self.handle = h.value
        self._ws = None

    def decode(self, q, k, v, ks, vs, out=None, seq_lens=None, stream=None, out_dtype=None):
        import torch

        B, Hq, D = q.shape
        if out is None:
            out = torch.empty((B, Hq, D), dtype=out_dtype or torch.float32, device=q.device)
        desc = make_desc(q, k, ks, out, seq_lens)
        n = int(lib().kvd_mgpu_p2p_workspace_size(ctypes.byref(desc)))
        if self._ws is None or self._ws.numel() < n:
            self._ws = torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)
        rc = lib().kvd_mgpu_p2p_seq_split_decode(self.handle, ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(ks), _ptr(vs), _ptr(out), _ptr(self._ws), self._ws.numel(),
                                                 _stream(stream))
        _check(rc, "kvd_mgpu_p2p_seq_split_decode")
        return out

    def reset(self, stream=None) -> None:
        """Collective: clears the exchange state on every rank after a call timed
        out (KVD_STATUS_WAIT_TIMEOUT), so the ranks' calls pair up again."""
        _check(lib().kvd_mgpu_p2p_reset(self.handle, _stream(stream)), "kvd_mgpu_p2p_reset")

    def close(self) -> None:
        if self.handle:
            lib().kvd_mgpu_p2p_destroy(self.handle)
            self.handle = None


class P2PGroup:
    """Single-process sequence split (kvd_mgpu_p2p_create_group): one context per
    rank, rank r on device devices[r], linked by direct peer pointers."""

    def __init__(self, devices, batch: int, num_q_heads: int, head_dim: int):
        n = len(devices)
        hs = (c_void_p * n)()
        devs = (c_int * n)(*devices)
        _check(lib().kvd_mgpu_p2p_create_group(hs, n, devs, batch, num_q_heads, head_dim),
               "kvd_mgpu_p2p_create_group")
        self.handles = [hs[r] for r in range(n)]
        self.devices = list(devices)
        self._ws = {}

    def decode(self, rank: int, q, k, v, ks, vs, out=None, seq_lens=None, stream=None, out_dtype=None):
        """Launches rank `rank`'s step on its device (tensors on that device); returns without waiting."""
        import torch

        with torch.cuda.device(self.devices[rank]):
            B, Hq, D = q.shape
            if out is None:
                out = torch.empty((B, Hq, D), dtype=out_dtype or torch.float32, device=q.device)
            desc = make_desc(q, k, ks, out, seq_lens)
            n = int(lib().kvd_mgpu_p2p_workspace_size(ctypes.byref(desc)))
            ws = self._ws.get(rank)
            if ws is None or ws.numel() < n:
                ws = self._ws[rank] = torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)
            rc = lib().kvd_mgpu_p2p_seq_split_decode(self.handles[rank], ctypes.byref(desc), _ptr(q), _ptr(k),
                                                     _ptr(v), _ptr(ks), _ptr(vs), _ptr(out), _ptr(ws), ws.numel(),
                                                     _stream(stream))
        _check(rc, "kvd_mgpu_p2p_seq_split_decode")
        return out

    def reset(self) -> None:
        for h in self.handles:
            _check(lib().kvd_mgpu_p2p_reset(h, None), "kvd_mgpu_p2p_reset")

    def close(self) -> None:
        for h in self.handles:
            if h:
                lib().kvd_mgpu_p2p_destroy(h)
        self.handles = []


def device_status() -> int:
    """Synchronise, then read and clear the device status word (KVD_STATUS_* bits)."""
    v = c_int32(0)
    _check(lib().kvd_device_status(ctypes.byref(v)), "kvd_device_status")
    return int(v.value)


def last_launch_count() -> int:
    return int(lib().kvd_last_launch_count())


def algorithmic_bytes(B: int, Hq: int, Hkv: int, D: int, lens) -> int:
    """Bytes a decode step must move: each (b, kv head) reads its codes and two
    scales per token once, plus the fp32 query and output rows."""
    if isinstance(lens, int):
        tokens = B * lens
    else:
        tokens = int(sum(int(x) for x in lens))
    return tokens * Hkv * (2 * D + 8) + B * Hq * D * 4 * 2


def default_softmax_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
