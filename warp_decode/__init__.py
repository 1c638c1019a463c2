"""The reference's import surface: ``from warp_decode import warp_decode as wd``.

Religious-J/warp_decode is a package named ``warp_decode`` whose attribute
``warp_decode`` is its compiled extension (``__init__.py:36-43``); its
callers import it exactly as above (``tests/test_gate_up_correctness.py:16``,
``tests/test_down_correctness.py:11``, ``benchmark/bench.py:48``).  This
package gives the same name to the warp_decode_b200 extension, so those
callers run unchanged with the B200 kernels underneath: same functions
(``moe_gate_up_3d_batched``, ``moe_down_3d_batched``), argument order, dtypes,
output shapes and ``RuntimeError`` messages.  Nothing is compiled at import
time and there is no fallback: the import fails if the native code is not
built (``python -m warp_decode_b200._build``).
"""
from __future__ import annotations

from warp_decode_b200 import load_extension as _load

warp_decode = _load()

__all__ = ["warp_decode"]
