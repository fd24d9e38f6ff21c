"""flour_b200 — B200 (sm_100a) paged KV pool + paged attention backend for flour.

The compute lives in ``libflour_attn.so`` (CUDA, C ABI in ``include/flour_attn.h``); this
package only binds it (``_lib``), wraps it for torch tensors (``ops``) and mirrors the reference's
host interface (``paged``). Importing it loads the library and fails if it is missing.
"""

from . import _lib
from ._lib import FlourAttnError

_lib.lib()  # fail loudly at import when the CUDA library is absent

from . import ops, paged  # noqa: E402

__all__ = ["ops", "paged", "FlourAttnError"]
