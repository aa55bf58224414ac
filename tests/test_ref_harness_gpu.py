"""The reference's own validators and loadtests, unchanged, against this
library on a B200.

oracle/ref.mk compiles tools/v_{rmsnorm,add_inplace,quantize,swiglu,matmul}_validate.cpp and
tools/b_*_loadtest.cpp from the reference's sources into oracle/_ref/ (they
travel to the GPU box as binaries).  Each loads libv7_threading.so through the
reference's loader (dlopen + 99 dlsym, ms_abi calls) and drives the hot-path
exports with host pointers: the drop-in proof.  Skipped where the binaries
were not built (no reference tree at build time).
"""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "oracle" / "_ref"


def ref_bin(name: str) -> Path:
    p = REF / name
    if not p.exists():
        pytest.skip(f"{p} not built (make -C oracle ref)")
    return p


@pytest.fixture(scope="module")
def db(tmp_path_factory):
    p = tmp_path_factory.mktemp("db") / "v7g.db"
    p.write_bytes(b"not a v7 microdb: the kernels need no key from it\n")
    return p


@pytest.mark.parametrize("validator,expect", [("v_rmsnorm_validate", 94), ("v_add_inplace_validate", 14),
                                               ("v_quantize_validate", 126)])
def test_reference_validator(cuda, native_lib_path, db, validator, expect):
    r = subprocess.run([str(ref_bin(validator)), str(native_lib_path), "--db", str(db)], capture_output=True, text=True,
                       timeout=600)
    tail = r.stdout[-2000:]
    assert r.returncode == 0, tail
    m = re.search(r"(\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(1)) == expect and int(m.group(2)) == 0, tail


def test_reference_matmul_validator_q8_and_batch4(cuda, native_lib_path, db):
    """tools/v_matmul_validate.cpp: its v7d_q8 sweep (the projection shapes
    of Qwen3-0.6B, Llama 3.2 1B, SmolLM2) and its four-token section
    (v7s_q8_batch4 / v7d_q8_batch4 bound by name, against four v7d_q8 calls:
    eight shapes including d = 3 and 7, an edge battery, a row slice, the
    dispatched whole matrix) pass against this library.  Its F32-matmul and
    split-geometry sections drive entries this library does not provide
    (v7d_f32 is a stub that marks the engine dead), so the run as a whole
    reports failures there; the test reads the two sections' own tallies."""
    r = subprocess.run([str(ref_bin("v_matmul_validate")), str(native_lib_path), "--db", str(db)], capture_output=True,
                       text=True, timeout=900)
    tail = r.stdout[-3000:]
    assert r.returncode in (0, 1), tail  # finished, no crash
    q8 = re.search(r"\[matmul Q8\] result: (\d+)/(\d+) passed", r.stdout)
    b4 = re.search(r"\[batch4\] correctness: (\d+)/(\d+) passed", r.stdout)
    assert q8 and int(q8.group(2)) > 0 and q8.group(1) == q8.group(2), tail
    assert b4 and int(b4.group(2)) > 0 and b4.group(1) == b4.group(2), tail
    assert "batch4 mismatch" not in r.stdout and "export missing" not in r.stdout, tail


def test_reference_swiglu_validator(cuda, native_lib_path, db):
    """tools/v_swiglu_validate.cpp (v7d_swiglu and v7d_swiglu_q8 against the
    double C references): the library's outputs equal the oracle's bit for
    bit, so the validator's report -- every case, every printed error -- is
    the one it gives for the oracle behind the same ABI."""
    from oracle.pyoracle import ABI_SHIM
    exe = ref_bin("v_swiglu_validate")

    def run(lib):
        r = subprocess.run([str(exe), str(lib), "--db", str(db)], capture_output=True, text=True, timeout=900)
        lines = [ln for ln in r.stdout.splitlines() if str(lib) not in ln]
        return r.returncode, lines

    rc, ours = run(native_lib_path)
    assert rc == 0, "\n".join(ours[-40:])
    assert any("F32xQ8 10 passed" in ln and "0 hard failures" in ln for ln in ours), "\n".join(ours[-40:])
    _, theirs = run(ABI_SHIM)
    assert ours == theirs


@pytest.mark.parametrize("args", [["b_rmsnorm_loadtest", "2048"], ["b_fused_add_rmsnorm_loadtest", "2048"],
                                  ["b_add_inplace_loadtest", "2048"], ["b_rmsnorm_rope_loadtest", "16", "128", "7", "128"],
                                  ["b_swiglu_q8_loadtest", "2048", "8192"], ["b_swiglu_loadtest", "2048", "8192"]])
def test_reference_loadtest(cuda, native_lib_path, db, args):
    exe = ref_bin(args[0])
    r = subprocess.run([str(exe), str(native_lib_path), *args[1:], "--db", str(db), "--iterations", "200"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "Pass:" in r.stdout and "us / call" in r.stdout, r.stdout
