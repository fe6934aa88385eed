"""A plain C host program against the C ABI (tests/native/c_host_example.c),
compiled with gcc -std=c11 -- the way the reference's callers build against its
kv_cache/*.cu entry points. The CPU test compiles, links and checks argument
errors (no GPU needed); the GPU test runs the reference's self-test inputs
(kv_cache/KV_int8_split_optimized.cu:473-486) through `solve` and
`kv_int8_split_launch` with the reference's acceptance tolerance, max abs err
<= 1e-4 (KV_int8_split_optimized.cu:535)."""
import os
import subprocess
from pathlib import Path

import pytest

import kvdecode as kvd

NATIVE = Path(__file__).resolve().parent / "native"
ROOT = NATIVE.parents[1]
PKG = ROOT / "cuda-operators_b200"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _program() -> Path:
    kvd.build()
    exe = NATIVE / "_build" / "c_host_example"
    src = NATIVE / "c_host_example.c"
    hdr = ROOT / "include" / "kvdecode.h"
    if not exe.exists() or exe.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime):
        exe.parent.mkdir(exist_ok=True)
        subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                        f"-I{CUDA / 'include'}", str(src), "-o", str(exe), f"-L{PKG}", "-lkvdecode_b200",
                        f"-Wl,-rpath,{PKG}", f"-L{CUDA / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}",
                        "-lm"], check=True)
    return exe


def test_c_program_compiles_links_and_gets_the_reference_error_codes():
    r = subprocess.run([str(_program()), "args"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "args: ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("H,S,D", [(4, 128, 64), (3, 129, 128), (8, 300, 128), (2, 5000, 64)])
def test_c_program_runs_the_reference_self_test(H, S, D):
    r = subprocess.run([str(_program()), "run", str(H), str(S), str(D)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("max abs err") == 2
