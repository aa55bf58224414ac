"""Regenerates the golden fixtures of tests/golden/ from the reference tree.

* ``kt_cref.npz`` -- outputs of the reference's own C reference kernels
  (tools/kt_utils.h: v7s_rmsnorm_c_ref, v7s_fused_add_rmsnorm_c_ref,
  v7s_rmsnorm_rope_heads_c_ref, v7s_add_inplace_c_ref, kt_quantize_c_ref) for
  every case the reference's validators run (tools/v_rmsnorm_validate.cpp,
  v_add_inplace_validate.cpp, v_quantize_validate.cpp).  Inputs are not
  stored: tests/reffills.py regenerates them with glibc rand() exactly as the
  validators do.  Quantiser codes are stored as SHA-256 digests (the check is
  bit-exact), everything else in full.
* ``v7_load_names.txt`` -- the 99 symbol names the reference's loader
  resolves (src/v7_lib.h:613-735).

Usage: python tests/golden/make_golden.py [--ref <reference tree>]
The tree defaults to $V7_REFERENCE_DIR, else a `reference` checkout beside
this repository.  Needs g++ and the reference source tree; the outputs are
committed.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import re
import struct
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("V7_REFERENCE_DIR") or str(HERE.parents[2] / "reference"))
    args = ap.parse_args()
    ref = Path(args.ref)

    names = re.findall(r"V7_RESOLVE\((\w+)\);", (ref / "src" / "v7_lib.h").read_text())
    (HERE / "v7_load_names.txt").write_text("\n".join(names) + "\n")

    with tempfile.TemporaryDirectory() as td:
        exe = Path(td) / "gen_golden"
        inc = [f"-I{ref / p}" for p in ("src/linux/compat", "src/linux", "src", "tools", "tools/zydis_stub")]
        subprocess.run(["g++", "-O0", "-std=c++17", "-D_GNU_SOURCE", "-w", *inc, str(HERE / "gen_golden.cpp"),
                        "-o", str(exe), "-ldl", "-lm", "-pthread"], check=True)
        blob = subprocess.run([str(exe)], check=True, capture_output=True).stdout

    out: dict[str, np.ndarray] = {}
    pos = 0
    while pos < len(blob):
        (nl,) = struct.unpack_from("<I", blob, pos)
        pos += 4
        name = blob[pos:pos + nl].decode()
        pos += nl
        kind, count = struct.unpack_from("<IQ", blob, pos)
        pos += 12
        size = count * (4 if kind == 0 else 1)
        data = blob[pos:pos + size]
        pos += size
        if kind == 1:
            out[name.replace("quant_codes/", "quant_codes_sha256/")] = np.frombuffer(
                hashlib.sha256(data).hexdigest().encode(), dtype=np.uint8)
        else:
            out[name] = np.frombuffer(data, dtype=np.float32).copy()
    np.savez_compressed(HERE / "kt_cref.npz", **out)
    print(f"wrote {len(out)} arrays, {len(names)} loader names")


if __name__ == "__main__":
    main()
