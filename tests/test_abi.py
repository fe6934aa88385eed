"""CPU tests of the C ABI boundary: the library loads, exports every function
include/kvdecode.h declares, rejects bad arguments on the host exactly as the
reference entry points do, and never links the oracle."""
import ctypes
import subprocess

import pytest

import kvdecode as kvd

EINVAL = kvd.CUDA_ERROR_INVALID_VALUE


def test_library_exports_every_header_function():
    names = kvd.header_functions()
    assert {"solve", "kv_int8_split_launch", "kv_int8_simple_launch", "kvd_decode_launch",
            "kvd_append_int8_launch", "kvd_combine_launch"} <= set(names)
    handle = kvd.lib()
    for n in names:
        assert hasattr(handle, n), n
    assert handle.kvd_abi_version() == 1


def test_product_library_does_not_link_the_oracle():
    out = subprocess.run(["nm", "-D", "--defined-only", str(kvd.LIB_PATH)], capture_output=True, text=True).stdout
    assert "kvo_" not in out and "kvref_" not in out
    deps = subprocess.run(["ldd", str(kvd.LIB_PATH)], capture_output=True, text=True).stdout
    assert "oracle" not in deps and "kvref" not in deps


@pytest.mark.parametrize("fn", ["kv_int8_split_launch", "kv_int8_simple_launch"])
def test_reference_launch_rejects_null_and_nonpositive(fn):
    f = getattr(kvd.lib(), fn)
    dummy = 256
    args = [dummy] * 6
    # KV_int8_split_optimized.cu:272-273 / new_kvint8.cu:89-90: any null or non-positive size
    assert f(*args, 4, 128, 64, None, None) == EINVAL
    for i in range(6):
        bad = list(args)
        bad[i] = None
        assert f(*bad, 4, 128, 64, dummy, None) == EINVAL
    for shape in [(0, 128, 64), (4, 0, 64), (4, 128, 0), (-1, 128, 64)]:
        assert f(*args, *shape, dummy, None) == EINVAL


def test_solve_reports_bad_arguments_on_stderr(capfd):
    kvd.lib().solve(None, None, None, None, None, None, 4, 128, 64)
    kvd.lib().solve(16, 16, 16, 16, 16, 16, 0, 128, 64)
    err = capfd.readouterr().err
    assert "null pointer input" in err and "invalid shape" in err


def _desc(**kw):
    d = kvd.DecodeDesc()
    d.batch, d.num_q_heads, d.num_kv_heads, d.head_dim, d.max_seq_len = 1, 8, 8, 128, 64
    d.kv_stride_h, d.sc_stride_h, d.q_stride_h, d.o_stride_h = 64 * 128, 64, 128, 128
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw", [dict(batch=0), dict(num_q_heads=6, num_kv_heads=4), dict(head_dim=0),
                                dict(max_seq_len=-1), dict(flags=64), dict(flags=1 | 8),
                                dict(flags=1, o_stride_h=128)])
def test_decode_launch_rejects_bad_descriptors(kw):
    d = _desc(**kw)
    rc = kvd.lib().kvd_decode_launch(ctypes.byref(d), 256, 256, 256, 256, 256, 256, None, 0, None)
    assert rc == EINVAL
    if "o_stride_h" not in kw:  # record rows too short for partial output: only the launch rejects it
        assert kvd.lib().kvd_workspace_size(ctypes.byref(d)) == 0


def test_other_entry_points_reject_null():
    L = kvd.lib()
    assert L.kvd_decode_launch(None, 1, 1, 1, 1, 1, 1, None, 0, None) == EINVAL
    assert L.kvd_combine_launch(None, 1, 0, 1, 64, 16, 0, 0, None) == EINVAL
    assert L.kvd_combine_launch(16, 2, 10, 4, 64, 16, 0, 0, None) == EINVAL  # part stride too small
    assert L.kvd_append_int8_launch(None, 1, 1, 1, 1, 1, 1, 1, None) == EINVAL
    a = kvd.AppendDesc()
    a.batch, a.num_kv_heads, a.head_dim, a.capacity = 1, 1, 64, 0
    assert L.kvd_append_int8_launch(ctypes.byref(a), 16, 16, 16, 16, 16, 16, 16, None) == EINVAL
    assert L.kvd_quantize_rows_launch(None, 4, 64, 64, 16, 64, 16, None) == EINVAL
    assert L.kvd_quantize_rows_launch(16, 0, 64, 64, 16, 64, 16, None) == 0  # nothing to do
    assert L.kvd_device_status(None) == EINVAL


def test_algorithmic_bytes_match_survey_table():
    # configs 1, 2, 3 and 5 of the north star (per-step HBM bytes)
    assert kvd.algorithmic_bytes(1, 8, 8, 64, 1024) == 1_118_208
    assert kvd.algorithmic_bytes(64, 32, 32, 128, 4096) == 2_216_689_664
    assert kvd.algorithmic_bytes(4, 32, 32, 128, 131072) == 4_429_316_096
    assert kvd.algorithmic_bytes(256, 64, 8, 128, 2048) == 1_124_073_472
