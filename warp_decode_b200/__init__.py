"""warp_decode_b200 -- fused MoE decode kernels for NVIDIA B200 (sm_100a).

Drop-in for the Religious-J/warp_decode package (``__init__.py:1-6, 36-43``)::

    from warp_decode_b200 import warp_decode as wd
    h = wd.moe_gate_up_3d_batched(x, w_gate_up, topk_ids)          # [B*topk, inter]
    y = wd.moe_down_3d_batched(h, w_down, topk_ids, topk_scale, B)  # [B, hidden]

``warp_decode`` is the compiled PyTorch extension (``csrc/binding.cpp``); all
compute runs in ``libwarp_decode_b200.so`` through the C ABI in
``include/warp_decode.h``.  Nothing is compiled at import time: build once
with ``python -m warp_decode_b200._build`` (or ``__graft_entry__.build()``).
There is no CPU or PyTorch fallback -- importing fails if the extension is
missing.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import sys

__all__ = ["warp_decode", "load_extension"]


def load_extension():
    """Import the prebuilt extension module from this package directory."""
    from . import _build

    name = f"{__name__}.{_build.EXT_NAME}"
    if name in sys.modules:
        return sys.modules[name]
    if not _build.EXT.exists() or not _build.LIB.exists():
        raise ImportError(
            "warp_decode_b200 native code is not built (missing "
            f"{_build.EXT.name} / {_build.LIB.name}); run "
            "`python -m warp_decode_b200._build`")
    import torch  # noqa: F401  (loads libtorch / libc10 for the extension)

    loader = importlib.machinery.ExtensionFileLoader(name, str(_build.EXT))
    spec = importlib.util.spec_from_file_location(name, str(_build.EXT), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def __getattr__(attr):
    # Loaded on first use so that `python -m warp_decode_b200._build` can run
    # before the extension exists.
    if attr == "warp_decode":
        mod = load_extension()
        globals()["warp_decode"] = mod
        return mod
    raise AttributeError(f"module {__name__!r} has no attribute {attr!r}")
