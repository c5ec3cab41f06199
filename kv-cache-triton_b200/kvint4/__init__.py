"""kvint4: runtime of the B200 INT4 KV-cache library.

* ``kvint4._lib``  -- ctypes binding of ``libkvint4.so`` (C ABI in include/kvint4.h)
* ``kvint4.ops``   -- torch-facing wrappers (pointers, strides, current stream)
* ``kvint4.shard`` -- multi-GPU sharding of the decode (KV-head and sequence shards)
"""

from . import _lib, ops  # noqa: F401

__all__ = ["_lib", "ops"]
