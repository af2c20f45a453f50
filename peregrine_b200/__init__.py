"""peregrine_b200 — B200-native (sm_100a) KV / prefix-cache hot path of the Peregrine server.

The product is the C-ABI library libperegrine_cuda.so built from csrc/ (see
include/peregrine_cuda.h). `capi` is its ctypes binding; `build` compiles it in-tree.
"""
from . import capi  # noqa: F401

__all__ = ["capi"]
