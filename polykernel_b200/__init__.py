"""pkb200: B200-native (sm_100a) fused MLP and prefill-attention kernels with the
reference's operator interface. See include/pkb200.h for the C ABI."""
from . import ops  # noqa: F401
from ._lib import LIB_PATH, attention_exact_ctas, device_error, lib, path_counters  # noqa: F401

__all__ = ["ops", "lib", "LIB_PATH", "device_error", "path_counters", "attention_exact_ctas"]
