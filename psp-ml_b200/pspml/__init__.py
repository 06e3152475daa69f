"""B200 (sm_100a) backend for the cargo-psp-ml TFLite int8 inference path.

The product is libpspml_cuda.so (C ABI in include/pspml.h).  This package is
its host-side mirror: a ctypes binding (capi), synthetic network specs in the
C-ABI form (netspec) and batch sharding across devices (shard).
"""
from . import capi, netspec, shard  # noqa: F401
from .capi import Context, Model, PspmlError, forward_sharded  # noqa: F401
