"""ctypes binding of the C ABI in ``include/warp_decode.h``.

This is the binding a non-PyTorch host would write for the C ABI; the tests
use it to drive the kernels through the exact C entry points.  Pointers
are plain integers (device addresses), streams are ``cudaStream_t`` values.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from . import _build

WD_OK = 0
WD_ERR_NULL_POINTER = 1
WD_ERR_SHAPE = 2
WD_ERR_ALIGNMENT = 3
WD_ERR_UNSUPPORTED = 4
WD_ERR_CUDA = 5

WD_STATUS_BAD_EXPERT_ID = 0x1
WD_STATUS_WAIT_TIMEOUT = 0x2
WD_STATUS_ROUTING_CHANGED = 0x4

HEADER = _build.INCLUDE / "warp_decode.h"

_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGS = {
    "wd_version": (_I, []),
    "wd_error_string": (ctypes.c_char_p, [_I]),
    "wd_last_error_message": (ctypes.c_char_p, []),
    "wd_moe_gate_up_3d_batched": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "wd_moe_down_3d_batched": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "wd_moe_gate_up_3d_batched_mxfp8": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "wd_moe_down_3d_batched_mxfp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "wd_status_read": (_I, [ctypes.POINTER(ctypes.c_uint32), _I]),
    "wd_launch_count": (ctypes.c_ulonglong, []),
    "wd_set_gate_up_path": (_I, [_I]),
    "wd_set_down_path": (_I, [_I]),
    "wd_tp_comm_create": (_I, [_I, _I, _I, _I, ctypes.POINTER(ctypes.c_void_p), _P]),
    "wd_tp_comm_open": (_I, [_P, _P]),
    "wd_tp_comm_destroy": (_I, [_P]),
    "wd_tp_comm_set_exchange": (_I, [_P, _I]),
    "wd_moe_down_3d_batched_allreduce": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P,
                                              _P]),
    "wd_moe_ffn_3d_batched": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P,
                                   _P]),
    "wd_set_ffn_path": (_I, [_I]),
    "wd_moe_ffn_3d_batched_kernels": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "wd_moe_ffn_3d_batched_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P,
                                           _P]),
    "wd_moe_router_topk": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _P]),
    "wd_copy_ranges": (_I, [ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t),
                            _I, _P]),
    "wd_moe_ffn_3d_batched_allreduce": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                                             _P, _P, _P]),
}

IPC_HANDLE_BYTES = 64

# Values of wd_set_gate_up_path / wd_set_down_path.
GATE_UP_AUTO, GATE_UP_SIMT, GATE_UP_TC = 0, 1, 2
PATH_AUTO, PATH_SIMT, PATH_TC = 0, 1, 2
# Values of wd_set_ffn_path.
FFN_AUTO, FFN_SPLIT, FFN_FUSED, FFN_TC = 0, 1, 2, 3

_lib = None


def header_symbols(path: Path = HEADER) -> list[str]:
    """Names of every function the header declares with WD_API."""
    text = path.read_text()
    return re.findall(r"^WD_API\s+[^;(]*?\b(wd_\w+)\s*\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    """Load libwarp_decode_b200.so (the same instance the torch extension uses)."""
    global _lib
    if _lib is None:
        if not _build.LIB.exists():
            raise OSError(f"{_build.LIB} is not built; run `python -m warp_decode_b200._build`")
        L = ctypes.CDLL(str(_build.LIB))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class WarpDecodeError(RuntimeError):
    def __init__(self, code: int):
        L = lib()
        self.code = code
        super().__init__(f"{L.wd_error_string(code).decode()}: {L.wd_last_error_message().decode()}")


def check(code: int) -> None:
    if code != WD_OK:
        raise WarpDecodeError(code)


def gate_up(x, w, ids, out, B, E, topk, hidden, inter, status=None, stream=0) -> int:
    return lib().wd_moe_gate_up_3d_batched(x, w, ids, out, B, E, topk, hidden, inter, status, stream)


def down(h, w, ids, scale, out, out_fp32, B, E, topk, hidden, inter, status=None, stream=0) -> int:
    return lib().wd_moe_down_3d_batched(h, w, ids, scale, out, out_fp32, B, E, topk, hidden, inter,
                                        status, stream)


def gate_up_mxfp8(x, wq, ws, ids, out, B, E, topk, hidden, inter, status=None, stream=0) -> int:
    return lib().wd_moe_gate_up_3d_batched_mxfp8(x, wq, ws, ids, out, B, E, topk, hidden, inter,
                                                 status, stream)


def down_mxfp8(h, wq, ws, ids, scale, out, out_fp32, B, E, topk, hidden, inter, status=None,
               stream=0) -> int:
    return lib().wd_moe_down_3d_batched_mxfp8(h, wq, ws, ids, scale, out, out_fp32, B, E, topk,
                                              hidden, inter, status, stream)


def ffn(x, w_gu, w_dn, ids, scale, h, sync, out, out_fp32, B, E, topk, hidden, inter,
        status=None, stream=0) -> int:
    return lib().wd_moe_ffn_3d_batched(x, w_gu, w_dn, ids, scale, h, sync, out, out_fp32, B, E,
                                       topk, hidden, inter, status, stream)


def ffn_noalloc(x, w_gu, w_dn, ids, scale, out, out_fp32, B, E, topk, hidden, inter,
                status=None, stream=0) -> int:
    return lib().wd_moe_ffn_3d_batched_noalloc(x, w_gu, w_dn, ids, scale, out, out_fp32, B, E,
                                               topk, hidden, inter, status, stream)


def router_topk(logits, logits_fp32, ids, weights, B, E, topk, renormalize, stream=0) -> int:
    return lib().wd_moe_router_topk(logits, logits_fp32, ids, weights, B, E, topk, renormalize,
                                    stream)


def copy_ranges(src, dst, nbytes, stream=0) -> int:
    """wd_copy_ranges over parallel lists of addresses (ints) and byte counts."""
    n = len(src)
    sp = (_P * max(n, 1))(*src)
    dp = (_P * max(n, 1))(*dst)
    nb = (ctypes.c_size_t * max(n, 1))(*nbytes)
    return lib().wd_copy_ranges(sp, dp, nb, n, stream)


def set_ffn_path(path: int) -> None:
    """Select the kernels behind wd_moe_ffn_3d_batched (FFN_AUTO / _SPLIT / _FUSED / _TC)."""
    check(lib().wd_set_ffn_path(int(path)))


# Values of ffn_kernels.
FFN_KERNELS_SPLIT, FFN_KERNELS_SIMT_SINGLE, FFN_KERNELS_TC_SINGLE = 0, 1, 2


def ffn_kernels(B: int, E: int, topk: int, hidden: int, inter: int) -> int:
    """Which kernels wd_moe_ffn_3d_batched would run for these sizes (FFN_KERNELS_*)."""
    kind = ctypes.c_int(-1)
    check(lib().wd_moe_ffn_3d_batched_kernels(B, E, topk, hidden, inter, ctypes.byref(kind)))
    return int(kind.value)


def set_gate_up_path(path: int) -> None:
    """Select the gate_up kernel for later calls (GATE_UP_AUTO / _SIMT / _TC)."""
    check(lib().wd_set_gate_up_path(int(path)))


def set_down_path(path: int) -> None:
    """Select the down kernel for later calls (PATH_AUTO / PATH_SIMT / PATH_TC)."""
    check(lib().wd_set_down_path(int(path)))


def tp_comm_create(world: int, rank: int, max_tokens: int, hidden: int):
    """Create this rank's fused-all-reduce communicator; returns (comm, ipc_handle bytes)."""
    comm = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().wd_tp_comm_create(world, rank, max_tokens, hidden, ctypes.byref(comm), handle))
    return comm.value, handle.raw


def tp_comm_open(comm: int, handles: bytes) -> None:
    """Open the peers' buffers; `handles` = every rank's handle, in rank order."""
    buf = ctypes.create_string_buffer(handles, len(handles))
    check(lib().wd_tp_comm_open(comm, buf))


def tp_comm_destroy(comm: int) -> None:
    check(lib().wd_tp_comm_destroy(comm))


# Values of tp_comm_set_exchange.
EXCHANGE_AUTO, EXCHANGE_ONE_SHOT, EXCHANGE_TWO_SHOT = 0, 1, 2


def tp_comm_set_exchange(comm: int, mode: int) -> None:
    """Exchange shape of later fused all-reduce calls (EXCHANGE_AUTO / _ONE_SHOT / _TWO_SHOT)."""
    check(lib().wd_tp_comm_set_exchange(comm, int(mode)))


def torch_ffn_allreduce(x, w_gu, w_dn, ids, scale, comm):
    """bf16 y[B, hidden] = sum over the group's ranks of this rank's FFN shard."""
    import torch

    B, K = ids.shape
    E, two_i, H = w_gu.shape
    I = two_i // 2
    h = torch.empty(B * K, I, dtype=torch.bfloat16, device=x.device)
    y = torch.empty(B, H, dtype=torch.bfloat16, device=x.device)
    check(lib().wd_moe_ffn_3d_batched_allreduce(x.data_ptr(), w_gu.data_ptr(), w_dn.data_ptr(),
                                                ids.data_ptr(), scale.data_ptr(), h.data_ptr(),
                                                None, y.data_ptr(), B, E, K, H, I, comm, None,
                                                _stream()))
    return y


def torch_down_allreduce(h, w, ids, scale, comm):
    """bf16 y[B, hidden] = sum over the group's ranks of down(h_r) (fused all-reduce)."""
    import torch

    B, K = ids.shape
    E, H, I = w.shape
    y = torch.empty(B, H, dtype=torch.bfloat16, device=h.device)
    check(lib().wd_moe_down_3d_batched_allreduce(h.data_ptr(), w.data_ptr(), ids.data_ptr(),
                                                 scale.data_ptr(), y.data_ptr(), B, E, K, H, I,
                                                 comm, None, _stream()))
    return y


def status_read(clear: bool = True) -> int:
    v = ctypes.c_uint32(0)
    check(lib().wd_status_read(ctypes.byref(v), 1 if clear else 0))
    return int(v.value)


def launch_count() -> int:
    """Kernels the library has enqueued in this process (graph captures count
    the launches they record; replays count none)."""
    return int(lib().wd_launch_count())


# ---------------------------------------------------------------------------
# torch-tensor conveniences (device pointers + current stream)
# ---------------------------------------------------------------------------
def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def torch_gate_up(x, w, ids):
    """moe_gate_up_3d_batched through the C ABI (torch tensors in, tensor out)."""
    import torch

    B, H = x.shape
    E, two_i, _ = w.shape
    K = ids.shape[1]
    out = torch.empty(B * K, two_i // 2, dtype=torch.bfloat16, device=x.device)
    check(gate_up(x.data_ptr(), w.data_ptr(), ids.data_ptr(), out.data_ptr(), B, E, K, H,
                  two_i // 2, None, _stream()))
    return out


def torch_down(h, w, ids, scale, fp32_out=False):
    """moe_down_3d_batched through the C ABI."""
    import torch

    B, K = ids.shape
    E, H, I = w.shape
    out = torch.empty(B, H, dtype=torch.float32 if fp32_out else torch.bfloat16, device=h.device)
    check(down(h.data_ptr(), w.data_ptr(), ids.data_ptr(), scale.data_ptr(), out.data_ptr(),
               1 if fp32_out else 0, B, E, K, H, I, None, _stream()))
    return out
