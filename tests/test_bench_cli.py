"""bench.py's command-line contract on CPU: the reference arm's JSON line for
every BASELINE workload, workload naming across GPU counts, and the refusal
to run a multi-GPU line without torchrun.  (The GPU arm runs on a B200.)"""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from warp_decode_b200 import workloads as W  # noqa: E402


def run_bench(*args):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, cwd=ROOT, timeout=300)


@pytest.mark.parametrize("workload", ["qwen3_235b_tp8", "qwen3_30b_mxfp8", "dsv3_tp8"])
def test_reference_arm_line(workload):
    r = run_bench("--impl", "reference", "--workload", workload, "--batches", "1",
                  "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "us/call"
    assert line["higher_is_better"] is False and line["value"] > 0
    assert line["config"]["workload"] == workload
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "us/call", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_workload_names():
    c = W.CONFIGS
    assert bench.workload_name("qwen3_235b_tp8", c["qwen3_235b_tp8"], 1) == "qwen3_235b_tp8"
    assert bench.workload_name("qwen3_235b_tp8", c["qwen3_235b_tp8"], 8) == \
        "qwen3_235b_inter1536_tp8"
    assert bench.workload_name("qwen3_235b_full", c["qwen3_235b_full"], 4) == "qwen3_235b_full_tp4"
    assert bench.workload_name("dsv3_tp8", c["dsv3_tp8"], 2) == "dsv3_tp8_inter512_tp2"


def test_multi_gpu_needs_torchrun():
    r = run_bench("--gpus", "2", "--steps", "1", "--warmup", "0")
    assert r.returncode == 2
    assert "torchrun" in r.stderr


def test_reference_arm_gpu_bar_absent_without_gpu():
    # the same-box bar of the reference's own CUDA kernels needs a GPU and the
    # rebuilt library; without them the key is present and null
    r = run_bench("--impl", "reference", "--batches", "1", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert "reference_gpu_kernels" in line and line["reference_gpu_kernels"] is None


class _Fused:
    def __init__(self, max_tokens):
        self.max_tokens = max_tokens

    def applies(self, B):
        return 1 <= B <= self.max_tokens


def test_exchange_record(monkeypatch):
    monkeypatch.delenv("WARP_DECODE_TP_TWO_SHOT_BYTES", raising=False)
    H = 4096
    assert bench.exchange_record(None, 8, H, 2) is None
    assert bench.exchange_record(_Fused(64), 8, H, 1) is None
    assert bench.exchange_record(_Fused(64), 128, H, 8) is None  # above the communicator
    # one-shot: every partial row to every peer, 8-byte packets
    r = bench.exchange_record(_Fused(64), 64, H, 8)
    assert r == {"shape": "one-shot", "bytes_sent_per_rank": 64 * H * 8 * 7}
    # two-shot above the threshold (from four ranks): ~2/world of the bytes
    monkeypatch.setenv("WARP_DECODE_TP_TWO_SHOT_BYTES", str(1 << 20))
    r = bench.exchange_record(_Fused(64), 64, H, 8)
    assert r == {"shape": "two-shot", "bytes_sent_per_rank": 2 * 64 * H * 8 * 7 // 8}
    assert bench.exchange_record(_Fused(64), 64, H, 2)["shape"] == "one-shot"
