"""Pins the oracle with the reference's own validators: the binaries built
from tools/v_*_validate.cpp (oracle/ref.mk) load libv7_oracle_abi.so -- the
oracle behind the reference's export surface -- through the reference's
loader and run their full case tables, seeds and tolerances against their C
references.  Skipped where the reference tree was not available to build them.
"""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "oracle" / "_ref"


@pytest.mark.parametrize("validator,expect", [("v_rmsnorm_validate", 94), ("v_add_inplace_validate", 14),
                                               ("v_quantize_validate", 126)])
def test_oracle_passes_reference_validator(oracle, tmp_path, validator, expect):
    from oracle.pyoracle import ABI_SHIM
    exe = REF / validator
    if not exe.exists():
        pytest.skip(f"{exe} not built (make -C oracle ref needs the reference tree)")
    db = tmp_path / "empty.db"
    db.write_bytes(b"\n")
    r = subprocess.run([str(exe), str(ABI_SHIM), "--db", str(db)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:]
    m = re.search(r"(\d+) passed, (\d+) failed", r.stdout)
    assert m and int(m.group(1)) == expect and int(m.group(2)) == 0
