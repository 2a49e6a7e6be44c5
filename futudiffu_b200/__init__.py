"""futudiffu_b200: B200-native (sm_100a) rebuild of sqcu/futudiffu's quantized DiT hot path.

Modules mirror the reference's operator API:

* ``sage_attention`` / ``attention_srcii`` / ``attention`` -- SageAttention-style
  INT8/FP8 attention (tcgen05) with K smoothing and block masks
* ``fp8_kernels`` / ``fp8`` -- FP8 blockwise activation/weight quantisation,
  the tcgen05 block-scaled GEMM and ``FP8Linear``
* ``fused_kernels`` -- fused RMSNorm / adaLN / RoPE prologues
* ``block_mask`` -- packed-sequence block masks

All compute runs in ``libfd_b200.so`` (C ABI in include/fd_b200.h); there is no
CPU fallback.
"""

from . import _lib  # noqa: F401

__version__ = "0.1.0"


def native_library_path() -> str:
    return str(_lib.LIB_PATH)


def check_status() -> None:
    """Synchronise and raise if any kernel recorded a bounded-wait timeout."""
    _lib.check_status()
