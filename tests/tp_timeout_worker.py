"""One rank of the tensor-parallel failure check (launched by test_gpu_tp_timeout.py under
torchrun, two ranks, gloo on the host): a rank stops taking part between steps, and the
other rank's next call must come back with SNL_E_TIMEOUT after about one wait bound
instead of hanging, with the device error word cleared and the CUDA context still usable.

SNL_TP_SAME_DEVICE=1 puts both ranks on GPU 0. Then rank 1 builds its engine and
connects, and runs no step at all: rank 0's first exchange waits on words that nothing
writes. Otherwise each rank has its own GPU, both run SNL_TP_GOOD_STEPS decode steps
together, and then rank 1 leaves (it runs no further kernel).
Rank 0 writes a JSON verdict to $SNL_TP_RESULT.
"""
import datetime
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(ROOT / "sense-nova-server_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from sensenova_b200 import ffi  # noqa: E402
from sensenova_b200.config import tp_test  # noqa: E402
from sensenova_b200.engine import Engine  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    same = os.environ.get("SNL_TP_SAME_DEVICE") == "1"
    good = 0 if same else int(os.environ.get("SNL_TP_GOOD_STEPS", "3"))
    dev = 0 if same else int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = tp_test()
    eng = Engine.synthetic(cfg, 64, 7, "q8_0", device=dev, tp=(rank, world))
    res = {"good_tokens": []}
    tok = 5
    for _ in range(good):  # both ranks together
        tok = eng.forward_greedy([tok], None, 1)[0]
        res["good_tokens"].append(tok)
    dist.barrier()  # host only: no kernel of either rank is in flight here
    if rank == 0:
        t0 = time.perf_counter()
        try:
            eng.forward_greedy([tok], None, 1)
            res["code"] = 0
        except ffi.SnlError as ex:
            res["code"] = ex.code
            res["message"] = str(ex)
        res["seconds"] = time.perf_counter() - t0
        res["error_word_after"] = int(eng.lib.snl_device_error(0))
        # the context still works: a small device computation and a synchronize
        a = torch.arange(1024, device="cuda", dtype=torch.float32)
        res["context_ok"] = float((a * 2).sum().item()) == 2.0 * 1023 * 1024 / 2
        Path(os.environ["SNL_TP_RESULT"]).write_text(json.dumps(res))
    dist.barrier()  # rank 1 keeps its exchange region mapped until rank 0 is done with it
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
