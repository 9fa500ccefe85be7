"""qwen35_b200 -- B200 (sm_100a) backend for the Qwen3.5 engine.

The product is libq35b.so (qwen35_b200/csrc, C ABI in include/q35.h); this
package builds it, binds it (lib.py) and drives its batched engine
(model.py).  There is no CPU fallback: without the shared object, loading
fails.
"""
from .lib import GEOM, TT, load  # noqa: F401
