"""strataflow_b200 -- B200-native (sm_100a) per-token MoE decode path for StrataFlow.

libsfk.so (built from csrc/ by strataflow_b200.build) holds every kernel and
the C ABI declared in include/sfk.h; `engine` mirrors engine::Engine and `ops`
exposes the operator-level entry points over torch CUDA tensors.
"""
from .lib import SfkError  # noqa: F401

__all__ = ["SfkError"]
