"""Tensor parallelism on 2, 4 and 8 GPUs of one node (needs that many GPUs; skipped
otherwise). Each case launches tests/tp_worker.py under torchrun, one process per GPU,
with NVLS off, and checks the rank-0 verdict: logits within 1e-3 of the unsharded oracle,
identical greedy tokens, all ranks agreeing, no device-side wait gave up; and for the
MTP head under tensor parallelism, the oracle's drafts, accept/reject decisions, verify
logits and committed tokens."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
TOL = 1e-3


def gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tensor_parallel_matches_oracle(torch_cuda, tmp_path, n):
    if gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, SNL_TP_RESULT=str(out), NCCL_NVLS_ENABLE="0", PYTHONUNBUFFERED="1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(29400 + n),
           str(ROOT / "tests" / "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["device_error"] == 0
    assert res["ranks_agree"]
    assert res["prefill_rel"] < TOL, res
    assert max(res["decode_rel"]) < TOL, res
    assert res["first_engine_token"] == res["first_oracle_token"]
    assert res["tokens_engine"] == res["tokens_oracle"], res
    # MTP under tensor parallelism: drafts, decisions, verify rows and committed tokens
    mt = res["mtp"]
    assert mt["ranks_agree"], mt
    assert mt["drafts_engine"] == mt["drafts_oracle"], mt
    assert mt["verified_engine"] == mt["verified_oracle"], mt
    assert mt["accept_engine"] == mt["accept_oracle"], mt
    assert any(mt["accept_engine"]) and not all(mt["accept_engine"]), mt
    assert max(mt["verify_rel"]) < TOL, mt
    assert mt["committed_engine"] == mt["committed_oracle"] == mt["greedy"][: len(mt["committed_engine"])], mt
