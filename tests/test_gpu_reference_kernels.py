"""Our kernels next to the reference's own CUDA kernels on the same B200.

oracle/Makefile rebuilds the reference's moe_gate_up_3d_batched.cu and
moe_down_3d_batched.cu unmodified for sm_100a (test infrastructure, git-
ignored, travels with the tree).  On reference-legal shapes (hidden % 256,
inter % 64) both implementations must agree with the FP32 oracle; the
reference's down rounds every product to bf16 (csrc/moe_down_3d_batched.cu:103)
so it is held to its own 5e-2 tolerance, ours to 1e-2.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import bf16_close
from oracle import moe_ref as O
from warp_decode_b200 import workloads as W

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libwdref.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libwdref.so not built (needs the reference sources)")
    L = ctypes.CDLL(str(LIB))
    P, I = ctypes.c_void_p, ctypes.c_int
    L.wdref_gate_up.argtypes = [P, P, P, P, I, I, I, I, I, P]
    L.wdref_down.argtypes = [P, P, P, P, P, I, I, I, I, I, P]
    return L


def bits(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("B", [1, 8, 64])
def test_reference_kernels_agree(ref, B):
    from warp_decode_b200 import warp_decode as wd

    H, I, E, K = 4096, 192, 128, 8
    w_gu, w_dn = W.make_device_weights(H, I, E, 31)
    x, ids, scale = W.make_device_activations(B, H, E, K, "uniform", 500 + B)
    s = torch.cuda.current_stream().cuda_stream
    h_ref = torch.empty(B * K, I, dtype=torch.bfloat16, device="cuda")
    assert ref.wdref_gate_up(x.data_ptr(), w_gu.data_ptr(), ids.data_ptr(), h_ref.data_ptr(),
                             B, E, K, H, I, s) == 0
    y_ref = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
    assert ref.wdref_down(h_ref.data_ptr(), w_dn.data_ptr(), ids.data_ptr(), scale.data_ptr(),
                          y_ref.data_ptr(), B, E, K, H, I, s) == 0
    h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
    y = wd.moe_down_3d_batched(h_ref, w_dn, ids, scale, B)
    torch.cuda.synchronize()
    ids_h = ids.cpu().numpy()
    touched = {int(e): bits(w_gu[int(e)]) for e in np.unique(ids_h)}
    h_or = O.gate_up(bits(x), touched, ids_h)
    assert bf16_close(bits(h), h_or, 1e-2, 1e-2)[0]
    assert bf16_close(bits(h_ref), h_or, 5e-2, 5e-2)[0]
    touched_d = {int(e): bits(w_dn[int(e)]) for e in np.unique(ids_h)}
    y_or = O.down(bits(h_ref), touched_d, ids_h, scale.cpu().numpy())
    assert bf16_close(bits(y), y_or, 1e-2, 1e-2)[0]
    assert bf16_close(bits(y_ref), y_or, 5e-2, 5e-2)[0]
