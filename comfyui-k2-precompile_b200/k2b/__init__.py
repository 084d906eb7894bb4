"""k2b -- B200-native (sm_100a) Krea2 W4A4 DiT block hot path.

Host side of libk2b: ``ops`` (torch wrappers over the C ABI in
include/k2b.h), ``model`` (resident block stack + native block loop),
``native_ops`` (the k2_native / k2_fullgraph torch operator surface).
"""
from . import ops  # noqa: F401
from ._native import K2BError, lib  # noqa: F401

__version__ = "0.1.0"
