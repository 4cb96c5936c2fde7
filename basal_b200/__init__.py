"""basal_b200: basal's quantised-linear hot path (rkinas/basal 2.8.1) built for B200 (sm_100a).

Modules mirror the reference's: blockquant, fp8block, int8block, nvfp4, readout, lean; the torch ops (`basal::*`)
are in ops; the C ABI binding in _lib (libbasal200.so, include/basal200.h); row sharding of independent requests
across the GPUs of a box in shard. Importing the package loads libbasal200.so and fails when it is missing.
"""
from . import _lib

_lib.lib()

from . import blockquant, fp8block, int8block, lean, nvfp4, ops, readout  # noqa: E402,F401

__version__ = "0.1.0"
