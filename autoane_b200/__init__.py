"""autoane_b200 — B200-native MeZO-LoRA projection hot path of AutoANE.

The compute lives in libb2p.so (hand-written sm_100a CUDA behind the C ABI of
include/b2p.h); this package is the host-side binding and the Python mirror of
the reference's device boundary. Importing it does not touch the GPU.
"""
from ._lib import B2PError, load, call  # noqa: F401

__all__ = ["B2PError", "load", "call"]
