"""flour_b200 — B200 (sm_100a) paged KV pool + paged attention backend for flour.

The compute lives in ``libflour_attn.so`` (CUDA, C ABI in ``include/flour_attn.h``); this
package only binds it (``_lib``), wraps it for torch tensors (``ops``) and mirrors the reference's
host interface (``paged``). The library is loaded on first use; every entry point raises if it
is missing or stale — there is no fallback implementation.
"""

from . import _lib
from ._lib import FlourAttnError

from . import ops, paged  # noqa: E402

__all__ = ["ops", "paged", "FlourAttnError"]
