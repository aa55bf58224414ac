"""The C-ABI library without a GPU: it loads, exports every symbol the
headers in include/ declare and every name the reference's loader resolves
(tests/golden/v7_load_names.txt, from src/v7_lib.h:613-735), validates
arguments on the host, and behaves like the reference's runtime (init, key
store, death reason) when driven through the Microsoft x64 convention from C."""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
NAMES = (ROOT / "tests" / "golden" / "v7_load_names.txt").read_text().split()


def exported(lib_path: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_exports_cover_reference_loader(native_lib_path):
    assert len(NAMES) == 99
    missing = set(NAMES) - exported(native_lib_path)
    assert not missing, missing


def test_exports_cover_headers(native_lib_path):
    from v7multiplikator_b200.build import exported_names
    declared = set(exported_names())
    assert set(NAMES) <= declared
    assert not (declared - exported(native_lib_path))


def test_no_unexpected_exports(native_lib_path):
    from v7multiplikator_b200.build import exported_names
    extra = exported(native_lib_path) - set(exported_names())
    assert not extra, extra


def test_ctypes_load_and_version(native_lib_path):
    import v7multiplikator_b200 as v7g
    assert "sm_100a" in v7g.version()
    assert v7g.launch_count() >= 0


def test_host_argument_validation(native_lib_path):
    """Contract violations are rejected before any device call."""
    import v7multiplikator_b200 as v7g
    L = v7g.lib()
    assert L.v7g_rmsnorm_rows(1, 1, 1, 4, 48, 1e-6, None) == v7g.ops.V7G_ERR_ARG
    assert b"multiple of 32" in L.v7g_last_error()
    assert L.v7g_fused_add_rmsnorm_rows(1, 1, 1, 1, 4, 12, 1e-6, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_swiglu_q8_rows(1, 1, 1, 1, 4, 96, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_rmsnorm_rope_rows(1, 1, 4, 2, 2, 100, 1, 1, 1, 1, 0, 64, 1e-6, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_rmsnorm_rope_rows(1, 1, 4, 2, 2, 2048, 1, 1, 1, 1, 0, 64, 1e-6, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_rmsnorm_rows(0, 0, 0, 4, 64, 1e-6, None) == v7g.ops.V7G_ERR_ARG  # NULL pointers
    assert L.v7g_quantize_rows(1, 1, 1, -1, 64, None) == v7g.ops.V7G_ERR_ARG
    assert L.v7g_add_inplace(1, 1, -5, None) == v7g.ops.V7G_ERR_ARG
    # empty work is a no-op success
    assert L.v7g_rmsnorm_rows(0, 0, 0, 0, 64, 1e-6, None) == 0
    assert L.v7g_swiglu(0, 0, 0, 0, None) == 0


def test_no_device_fails_loudly(native_lib_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    import v7multiplikator_b200 as v7g
    L = v7g.lib()
    rc = L.v7g_rmsnorm_rows(16, 16, 16, 4, 64, 1e-6, None)
    assert rc == v7g.ops.V7G_ERR_NO_DEVICE
    assert L.v7g_last_error()


def test_python_layer_rejects_cpu_tensors(native_lib_path):
    import torch
    import v7multiplikator_b200 as v7g
    x = torch.zeros(2, 64)
    with pytest.raises(ValueError):
        v7g.rmsnorm_rows(torch.empty_like(x), x, torch.ones(64), 1e-6)


def test_rms_eps_global(native_lib_path):
    import v7multiplikator_b200 as v7g
    old = v7g.get_rms_eps()
    v7g.set_rms_eps(1e-5)
    assert abs(v7g.get_rms_eps() - 1e-5) < 1e-12
    v7g.set_rms_eps(old)


def test_launch_overlap_switch(native_lib_path):
    import v7multiplikator_b200 as v7g
    assert v7g.launch_overlap()  # on by default
    try:
        v7g.set_launch_overlap(False)
        assert not v7g.launch_overlap()
        assert v7g.lib().v7g_get_launch_overlap() == 0
    finally:
        v7g.set_launch_overlap(True)
    assert v7g.launch_overlap()


def test_launch_overlap_environment_switch(native_lib_path):
    """V7G_LAUNCH_OVERLAP=0 starts the library with plain launches."""
    import os
    env = dict(os.environ, V7G_LAUNCH_OVERLAP="0")
    code = "import v7multiplikator_b200 as v; print(v.launch_overlap())"
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "False"
    env["V7G_LAUNCH_OVERLAP"] = "1"
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "True"


@pytest.fixture(scope="module")
def abi_probe(tmp_path_factory):
    exe = tmp_path_factory.mktemp("probe") / "abi_probe"
    subprocess.run(["gcc", "-O1", "-std=c11", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "abi_probe.c"), "-o", str(exe),
                    "-ldl", "-lm"], check=True)
    return exe


def test_ms_abi_host_probe(native_lib_path, abi_probe):
    import torch
    mode = ["gpu"] if torch.cuda.is_available() else []
    r = subprocess.run([str(abi_probe), str(native_lib_path), str(ROOT / "tests" / "golden" / "v7_load_names.txt"), *mode],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PROBE PASSED" in r.stdout


def test_batch4_argument_block_layout(tmp_path):
    """The four-token GEMV's argument block, as a C caller compiles it from
    include/v7_threading.h, has the reference's byte offsets
    (src/q8_batch4.h:29-38; q8_batch4_kernel.inc's Q8B_* offsets): 120 bytes,
    xq at 32, xs at 64, wq at 96, ws at 104, n at 112, d at 116."""
    import subprocess
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include "v7_threading.h"\n'
        "_Static_assert(sizeof(v7_q8_batch4_args) == 120, \"size\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, out) == 0, \"out\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, xq) == 32, \"xq\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, xs) == 64, \"xs\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, wq) == 96, \"wq\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, ws) == 104, \"ws\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, n) == 112, \"n\");\n"
        "_Static_assert(offsetof(v7_q8_batch4_args, d) == 116, \"d\");\n"
        "int main(void) { return 0; }\n")
    r = subprocess.run(["gcc", "-std=c11", "-fsyntax-only", f"-I{ROOT / 'include'}", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
