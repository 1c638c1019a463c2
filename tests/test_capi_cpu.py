"""C ABI checks that need no GPU: the library loads, exports exactly what the
header declares, and rejects bad arguments on the host before touching CUDA.

The reference validates in its torch binding (csrc/binding.cpp:29-57, 86-105
of Religious-J/warp_decode); here the same checks live below the binding, in
the C ABI, so a non-PyTorch caller gets them too.
"""
import ctypes
import subprocess

import pytest

from warp_decode_b200 import capi, _build


def test_library_exports_every_header_symbol():
    names = capi.header_symbols()
    assert len(names) == 23, names
    L = capi.lib()
    for n in names:
        assert hasattr(L, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(_build.LIB)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(names), exported ^ set(names)


def test_gate_up_path_selector_validates():
    L = capi.lib()
    assert L.wd_set_gate_up_path(3) == capi.WD_ERR_SHAPE
    assert b"path" in L.wd_last_error_message()
    for p in (capi.GATE_UP_SIMT, capi.GATE_UP_TC, capi.GATE_UP_AUTO):
        assert L.wd_set_gate_up_path(p) == capi.WD_OK
    assert L.wd_set_down_path(-1) == capi.WD_ERR_SHAPE
    for p in (capi.PATH_SIMT, capi.PATH_TC, capi.PATH_AUTO):
        assert L.wd_set_down_path(p) == capi.WD_OK
    assert L.wd_set_ffn_path(4) == capi.WD_ERR_SHAPE
    for p in (capi.FFN_SPLIT, capi.FFN_FUSED, capi.FFN_TC, capi.FFN_AUTO):
        assert L.wd_set_ffn_path(p) == capi.WD_OK


def test_ffn_validates_before_touching_the_device():
    L = capi.lib()
    # shape / pointer / alignment errors come back before any CUDA call
    assert capi.ffn(1, 1, 1, 1, 1, 1, None, 1, 0, 1, 128, 8, 4095, 192) == capi.WD_ERR_SHAPE
    assert capi.ffn(16, 16, 16, 16, 16, None, None, 16, 0, 1, 128, 8, 4096, 192) == \
        capi.WD_ERR_NULL_POINTER
    assert capi.ffn(16, 16, 24, 16, 16, 16, None, 16, 0, 1, 128, 8, 4096, 192) == \
        capi.WD_ERR_ALIGNMENT
    assert capi.ffn(16, 16, 16, 16, 16, 16, 12, 16, 0, 1, 128, 8, 4096, 192) == \
        capi.WD_ERR_ALIGNMENT
    assert b"sync" in L.wd_last_error_message()
    assert capi.ffn(None, None, None, None, None, None, None, None, 0, 0, 128, 8, 4096, 192) == \
        capi.WD_OK


def test_tp_comm_validates_before_touching_the_device():
    import ctypes

    L = capi.lib()
    comm = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(capi.IPC_HANDLE_BYTES)
    assert L.wd_tp_comm_create(1, 0, 64, 4096, ctypes.byref(comm), handle) == capi.WD_ERR_SHAPE
    assert L.wd_tp_comm_create(9, 0, 64, 4096, ctypes.byref(comm), handle) == capi.WD_ERR_SHAPE
    assert L.wd_tp_comm_create(2, 2, 64, 4096, ctypes.byref(comm), handle) == capi.WD_ERR_SHAPE
    assert L.wd_tp_comm_create(2, 0, 64, 4094, ctypes.byref(comm), handle) == capi.WD_ERR_SHAPE
    assert L.wd_tp_comm_create(2, 0, 64, 4096, None, handle) == capi.WD_ERR_NULL_POINTER
    assert L.wd_tp_comm_open(None, handle) == capi.WD_ERR_NULL_POINTER
    assert L.wd_tp_comm_destroy(None) == capi.WD_OK
    rc = L.wd_moe_down_3d_batched_allreduce(1, 1, 1, 1, 1, 1, 8, 8, 4096, 192, None, None, None)
    assert rc == capi.WD_ERR_NULL_POINTER
    assert b"comm" in L.wd_last_error_message()


def test_version_and_error_strings():
    L = capi.lib()
    assert L.wd_version() >= 100
    assert L.wd_error_string(capi.WD_ERR_SHAPE) == b"invalid shape"
    assert L.wd_error_string(99) == b"unknown error"


def test_rejected_calls_launch_nothing():
    L = capi.lib()
    before = L.wd_launch_count()
    assert capi.gate_up(0x1000, 0x2000, 0x3000, 0x4000, -1, 4, 2, 256, 8) == capi.WD_ERR_SHAPE
    assert capi.gate_up(0, 0x2000, 0x3000, 0x4000, 2, 4, 2, 256, 8) == capi.WD_ERR_NULL_POINTER
    assert L.wd_launch_count() == before
    assert capi.launch_count() == before


@pytest.mark.parametrize("args,code,msg", [
    (dict(B=-1), capi.WD_ERR_SHAPE, b"B must be >= 0"),
    (dict(E=0), capi.WD_ERR_SHAPE, b"E (number of experts)"),
    (dict(topk=0), capi.WD_ERR_SHAPE, b"topk must be >= 1"),
    (dict(topk=513), capi.WD_ERR_UNSUPPORTED, b"topk must be <= 512"),
    (dict(hidden=100), capi.WD_ERR_SHAPE, b"hidden must be a multiple of 8"),
    (dict(x=0), capi.WD_ERR_NULL_POINTER, b"null tensor pointer"),
    (dict(x=0x1008), capi.WD_ERR_ALIGNMENT, b"16-byte aligned"),
])
def test_gate_up_host_validation(args, code, msg):
    a = dict(x=0x1000, w=0x2000, ids=0x3000, out=0x4000, B=2, E=4, topk=2, hidden=256, inter=8)
    a.update(args)
    rc = capi.gate_up(a["x"], a["w"], a["ids"], a["out"], a["B"], a["E"], a["topk"], a["hidden"],
                      a["inter"])
    assert rc == code
    assert msg in capi.lib().wd_last_error_message()


@pytest.mark.parametrize("args,code,msg", [
    (dict(inter=12), capi.WD_ERR_SHAPE, b"inter must be a multiple of 8"),
    (dict(scale=0), capi.WD_ERR_NULL_POINTER, b"null tensor pointer"),
    (dict(h=0x1004), capi.WD_ERR_ALIGNMENT, b"16-byte aligned"),
])
def test_down_host_validation(args, code, msg):
    a = dict(h=0x1000, w=0x2000, ids=0x3000, scale=0x5000, out=0x4000, B=2, E=4, topk=2,
             hidden=256, inter=64)
    a.update(args)
    rc = capi.down(a["h"], a["w"], a["ids"], a["scale"], a["out"], 0, a["B"], a["E"], a["topk"],
                   a["hidden"], a["inter"])
    assert rc == code
    assert msg in capi.lib().wd_last_error_message()


def test_mxfp8_host_validation():
    rc = capi.gate_up_mxfp8(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 1, 4, 2, 272, 8)
    assert rc == capi.WD_ERR_SHAPE  # hidden % 32
    rc = capi.down_mxfp8(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000, 0, 1, 4, 2, 256, 48)
    assert rc == capi.WD_ERR_SHAPE  # inter % 32


def test_empty_batch_is_a_no_op():
    # B = 0 returns before any CUDA call (the reference would launch a 0-sized grid)
    assert capi.gate_up(0, 0, 0, 0, 0, 4, 2, 256, 8) == capi.WD_OK
    assert capi.down(0, 0, 0, 0, 0, 0, 0, 4, 2, 256, 64) == capi.WD_OK


def test_torch_binding_rejects_cpu_tensors():
    import torch
    from warp_decode_b200 import warp_decode as wd

    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    w = torch.zeros(4, 16, 256, dtype=torch.bfloat16)
    ids = torch.zeros(1, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="x must be CUDA"):
        wd.moe_gate_up_3d_batched(x, w, ids)
    with pytest.raises(RuntimeError, match="buffer must be CUDA"):
        wd.moe_down_3d_batched(torch.zeros(2, 64, dtype=torch.bfloat16),
                               torch.zeros(4, 256, 64, dtype=torch.bfloat16), ids,
                               torch.zeros(1, 2), 1)


def test_reference_import_surface():
    """`from warp_decode import warp_decode as wd` (the reference's import,
    tests/test_gate_up_correctness.py:16) gives this repository's extension."""
    from warp_decode import warp_decode as wd
    from warp_decode_b200 import warp_decode as wd_b200

    assert wd is wd_b200
    for name in ("moe_gate_up_3d_batched", "moe_down_3d_batched"):
        assert callable(getattr(wd, name))
