"""gcnasm_b200 -- B200-native (sm_100a) block-scaled FP8 GEMM.

The product is the C ABI in ``include/b2g/gemm.h`` implemented by
``gcnasm_b200/_lib/libb2g.so`` (hand-written tcgen05 / TMA kernels).  This
package binds it (``capi``), mirrors the reference's f4gemm host helpers
(``f4gemm``) and offers torch-tensor wrappers (``ops``).
"""
from . import capi  # noqa: F401

__all__ = ["capi", "f4gemm", "ops", "build"]
