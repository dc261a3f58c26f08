"""Failure detection under tensor parallelism, without a GPU fault: a rank stops taking part
between steps, and the other rank's next call returns SNL_E_TIMEOUT after about one wait
bound (SNL_TP_WAIT_MS) instead of hanging, with the device error word cleared and the
CUDA context usable afterwards.

`same_device` runs both ranks as processes on GPU 0: rank 1 builds and connects its
engine and runs nothing, so rank 0's exchange waits on words that nothing writes (only
one side ever runs a kernel). `two_gpus` (needs 2 GPUs) runs three steps on both ranks
first, then rank 1 leaves. Both use gloo on the host and no NCCL or NVLS."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
WAIT_MS = 300


def gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.parametrize("mode", ["same_device", "two_gpus"])
def test_peer_that_stops_gives_timeout(torch_cuda, tmp_path, mode):
    if mode == "two_gpus" and gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "tp_timeout.json"
    env = dict(os.environ, SNL_TP_RESULT=str(out), SNL_TP_WAIT_MS=str(WAIT_MS), NCCL_NVLS_ENABLE="0",
               PYTHONUNBUFFERED="1", SNL_TP_SAME_DEVICE="1" if mode == "same_device" else "0")
    port = 29450 + (0 if mode == "same_device" else 1)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(ROOT / "tests" / "tp_timeout_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["code"] == -6, res  # SNL_E_TIMEOUT
    assert "did not answer" in res["message"], res
    # one bound, not one per wait: the old 2 s per wait over 100+ waits took minutes
    assert res["seconds"] < 10.0, res
    assert res["error_word_after"] == 0, res
    assert res["context_ok"], res
    if mode == "two_gpus":
        assert len(res["good_tokens"]) == 3
