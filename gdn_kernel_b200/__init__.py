"""B200-native (sm_100a) Gated DeltaNet hot path: T=1 decode and chunked
(C=64) variable-length prefill behind the reference's ``kernel`` API, plus the
serving forms of the decode step (state pool with indices, multi-token
decode)."""

from .kernel import (decode, gdn_decode, gdn_decode_pool, gdn_mtp, gdn_prefill,  # noqa: F401
                     load_tvm_kernel, mtp, prefill)
from ._lib import device_status  # noqa: F401

__all__ = ["decode", "prefill", "gdn_decode", "gdn_prefill", "gdn_decode_pool", "gdn_mtp", "mtp",
           "load_tvm_kernel", "device_status"]
