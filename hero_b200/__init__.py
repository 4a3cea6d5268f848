"""hero_b200 -- B200 (sm_100a) attention, KV-cache and gated delta-rule path for the nm engine.

The product is ``libnmg.so`` (CUDA kernels + the C ABI of include/nmg.h).  This
package is its Python face: ``hero_b200.nm`` mirrors the reference's cache and
operator interface over that ABI.
"""
from ._lib import (  # noqa: F401
    BF16, F16, F32, CommError, CudaError, DeviceTimeout, InvalidArgument, LengthError, LogicError, NmgError,
    NoVisibleKeys, OutOfRange, Unsupported, ValueOverflow, lib,
)

__all__ = ["lib", "nm", "NmgError", "InvalidArgument", "OutOfRange", "NoVisibleKeys", "LengthError", "LogicError",
           "CudaError", "DeviceTimeout", "CommError", "Unsupported", "ValueOverflow", "F32", "F16", "BF16"]
