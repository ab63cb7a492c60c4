"""gollama_b200: sm_100a (B200) backend for the training hot path of gollama.

The compute path is libgollama_cuda.so (hand-written CUDA for sm_100a behind
the C ABI in include/gollama_cuda.h).  This package holds its ctypes binding
and the host-side mirror of the reference's trainer interface
(pkg/train/trainer.go, pkg/train/optimizer.go).
"""
from ._lib import LIB_PATH, load  # noqa: F401
