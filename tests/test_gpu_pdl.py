"""Programmatic dependent launch of down behind gate_up (WARP_DECODE_PDL=1)
gives the same bits as the default launches, on a B200.

With the variable set, moe_down_3d_batched is launched so that it may start
while the moe_gate_up_3d_batched launch before it on the stream is still
finishing (the gate_up kernels release their dependents after their last h
store; down waits for the whole gate_up grid before reading h or the top-k
weights).  The variable is read once per process, so each mode runs in a
process of its own: the reference's two calls at B = 1 (SIMT down), 2 and 8
(tcgen05 down after the SIMT gate_up) and 16 (after the tcgen05 gate_up),
twice in a row, h and y compared bit for bit, status word clean.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, {root!r})
from warp_decode_b200 import warp_decode as wd
from warp_decode_b200 import workloads as W

H, I, E, K = 4096, 192, 128, 8
w_gu, w_dn = W.make_device_weights(H, I, E, 21)
out = {{}}
for B, gate_up_path in ((1, 0), (2, 0), (8, 0), (16, 2)):
    wd.set_gate_up_path(gate_up_path)
    x, ids, sc = W.make_device_activations(B, H, E, K, "uniform", 300 + B)
    for rep in range(2):
        h = wd.moe_gate_up_3d_batched(x, w_gu, ids)
        y = wd.moe_down_3d_batched(h, w_dn, ids, sc, B)
        torch.cuda.synchronize()
        out[f"h{{B}}_{{rep}}"] = h.view(torch.int16).cpu().numpy()
        out[f"y{{B}}_{{rep}}"] = y.view(torch.int16).cpu().numpy()
    out[f"status{{B}}"] = np.array(wd.status(True, 0))
wd.set_gate_up_path(0)
np.savez({path!r}, **out)
"""


def run_mode(path, pdl):
    env = dict(os.environ, WARP_DECODE_PDL="1" if pdl else "0")
    script = SCRIPT.format(root=str(ROOT), path=str(path))
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return dict(np.load(path))


def test_pdl_same_bits(tmp_path):
    plain = run_mode(tmp_path / "plain.npz", pdl=False)
    pdl = run_mode(tmp_path / "pdl.npz", pdl=True)
    assert plain.keys() == pdl.keys()
    for k in plain:
        if k.startswith("status"):
            assert int(plain[k]) == 0 and int(pdl[k]) == 0, k
        else:
            assert np.array_equal(plain[k], pdl[k]), f"{k}: PDL launch changed the bits"
    # two calls in a row agree with each other too
    for B in (1, 2, 8, 16):
        assert np.array_equal(pdl[f"y{B}_0"], pdl[f"y{B}_1"])
