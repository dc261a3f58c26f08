"""One rank of the tensor-parallel engine check (launched by test_gpu_tp.py under
torchrun): the TP engine on the `tp_test` model against the oracle's unsharded model.

Rank 0 writes a JSON verdict to $SNL_TP_RESULT: prefill and per-step logits relative
error, greedy tokens of the engine's device decode loop and of forward_greedy, and
whether every rank produced the same tokens. A second engine of the same model with an
MTP head (replicated on every rank, vocabulary-split head) then runs the draft-1 /
verify-2 loop: its drafts, accept/reject decisions, verify logits and committed tokens
go into the verdict beside the oracle's.
"""
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(ROOT / "sense-nova-server_b200"), str(ROOT / "oracle")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from sensenova_b200.config import tp_test  # noqa: E402
from sensenova_b200.engine import Engine  # noqa: E402
from spec_loop import spec_loop  # noqa: E402

MTP_PROMPT = [2, 7, 1, 8, 2, 8, 1, 8, 2, 8]
MTP_STEPS = 10


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = tp_test()
    seed, ctx, steps = 7, 96, int(os.environ.get("SNL_TP_STEPS", "24"))
    eng = Engine.synthetic(cfg, ctx, seed, "q8_0", device=local, tp=(rank, world))
    prompt = [(17 + i * 7919) % cfg.vocab for i in range(13)]
    lg = eng.forward(prompt, True)                 # prefill, full logits on every rank
    toks, lgs = [int(np.argmax(lg))], [lg]
    for _ in range(4):                             # decode with logits (gather path)
        lg = eng.forward([toks[-1]], True)
        lgs.append(lg)
        toks.append(int(np.argmax(lg)))
    g = eng.forward_greedy([toks[-1]], None, 1)[0]  # greedy key exchange
    gen, _ = eng.generate(g, steps)                 # device decode loop (graphs)
    mine = torch.tensor(toks + [g] + list(gen), dtype=torch.int64, device="cuda")
    allt = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allt, mine)
    same = all(bool((t == mine).all()) for t in allt)
    # MTP: the true greedy continuation (from the model without the head, same seed)
    # is verified on odd steps, so both the accept and the reject branch run.
    eng.reset()
    greedy = [int(np.argmax(eng.forward(MTP_PROMPT, True)))]
    for _ in range(2 * MTP_STEPS + 2):
        greedy.append(int(np.argmax(eng.forward([greedy[-1]], True))))

    def forced(i, committed):
        return greedy[len(committed)] if i % 2 == 1 else None

    me = Engine.synthetic(cfg, ctx, seed, "q8_0", mtp=True, device=local, tp=(rank, world))
    mlog, mcommit = spec_loop(me, MTP_PROMPT, MTP_STEPS, forced)
    mine = torch.tensor([x[0] for x in mlog] + mcommit, dtype=torch.int64, device="cuda")
    allt = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allt, mine)
    same_mtp = all(bool((t == mine).all()) for t in allt)
    err = int(eng.lib.snl_device_error(0))
    if rank == 0:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as orc

        o = orc.OracleModel(cfg, ctx, seed=seed, quant=1)
        lo = o.forward(prompt, True)
        res = {"prefill_rel": rel(lgs[0], lo), "decode_rel": [], "tokens_engine": [], "tokens_oracle": []}
        to = int(np.argmax(lo))
        for i in range(1, 5):
            lo = o.forward([toks[i - 1]], True)
            res["decode_rel"].append(rel(lgs[i], lo))
        seq = [toks[-1]]
        ref = []
        t = toks[-1]
        for _ in range(1 + steps):
            lo = o.forward([t], True)
            t = int(np.argmax(lo))
            ref.append(t)
        res["tokens_engine"] = [g] + list(gen)
        res["tokens_oracle"] = ref
        res["ranks_agree"] = same
        res["device_error"] = err
        res["first_oracle_token"] = to
        res["first_engine_token"] = toks[0]
        om = orc.OracleModel(cfg, ctx, seed=seed, quant=1, mtp=True)
        olog, ocommit = spec_loop(om, MTP_PROMPT, MTP_STEPS, forced)
        res["mtp"] = {
            "drafts_engine": [x[0] for x in mlog], "drafts_oracle": [x[0] for x in olog],
            "verified_engine": [x[1] for x in mlog], "verified_oracle": [x[1] for x in olog],
            "accept_engine": [x[2] for x in mlog], "accept_oracle": [x[2] for x in olog],
            "verify_rel": [rel(a[3], b[3]) for a, b in zip(mlog, olog)],
            "committed_engine": mcommit, "committed_oracle": ocommit, "greedy": greedy,
            "ranks_agree": same_mtp,
        }
        Path(os.environ["SNL_TP_RESULT"]).write_text(json.dumps(res))
        om.close()
        o.close()
    me.close()
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
