"""B200-native (sm_100a) Gated DeltaNet hot path: T=1 decode and chunked
(C=64) variable-length prefill behind the reference's ``kernel`` API."""

from .kernel import decode, gdn_decode, gdn_prefill, load_tvm_kernel, prefill  # noqa: F401
from ._lib import device_status  # noqa: F401

__all__ = ["decode", "prefill", "gdn_decode", "gdn_prefill", "load_tvm_kernel", "device_status"]
