"""v7multiplikator_b200 -- B200-native (sm_100a) kernels for v7's fused
per-layer elementwise and reduction path.

The package is a thin Python host layer over ``lib/libv7_threading.so``, a
C-ABI shared library that

* exports the reference engine's own entry points (``v7s_rmsnorm``,
  ``v7s_fused_add_rmsnorm``, ``v7s_rmsnorm_rope_heads``, ``v7s_add_inplace``,
  ``v7d_quantize``, ``v7s_rmsnorm_quantize`` and the rest of the 99 names its
  loader resolves) with the reference's calling convention, so the
  reference's own host programs run against it unchanged; and
* adds row-batched, device-resident entry points (``v7g_*``, include/v7g.h)
  that process a whole activation tensor per launch.

Every kernel reproduces the reference's AVX2 arithmetic operation for
operation, so results match bit for bit.  See ``ops`` for the Python API.
"""
from .ops import (  # noqa: F401
    LIB_PATH,
    V7GError,
    add_inplace,
    fill_normal,
    fused_add_rmsnorm_rows,
    get_rms_eps,
    launch_count,
    launch_overlap,
    lib,
    pipeline_timeouts,
    q8_fused_gemv,
    q8_gemv,
    quantize_rows,
    rmsnorm_quantize_rows,
    rmsnorm_rope_rows,
    rmsnorm_rows,
    rmsnorm_rows_noalloc,
    rope_freqs,
    rope_init,
    rope_only_rows,
    rope_tables,
    selftest_arith,
    set_launch_overlap,
    set_rms_eps,
    swiglu,
    swiglu_f32q8_gemv,
    swiglu_q8_gemv,
    swiglu_q8_rows,
    v7d_quantize,
    v7s_add_inplace,
    v7s_fused_add_rmsnorm,
    v7s_rmsnorm,
    v7s_rmsnorm_quantize,
    v7s_rmsnorm_rope_heads,
    v7s_rope_only_heads,
    version,
)

__version__ = "0.1.0"
