"""The draft-1 / verify-2 speculative loop shared by the MTP tests (one GPU in
test_gpu_engine.py, tensor parallel in tp_worker.py): it drives an engine or the
oracle's restatement through the same calls."""
import numpy as np


def spec_loop(eng, prompt, steps, forced):
    """The draft-1 / verify-2 loop of worker.rs:197-255 at temperature 0 (as bench.py's
    MTP workload runs it) on an engine or the oracle. On steps where forced(i, committed)
    returns a token, that token is verified instead of the MTP head's draft (the head is
    still run, so its cache advances the same way): with the true greedy continuation
    this takes the accept branch, which a random-weight head never reaches.
    Returns [(mtp draft, verified token, accepted, verify logits)], committed tokens."""
    n = len(prompt)
    lg = eng.forward(prompt, True)
    tok = int(np.argmax(lg))
    eng.mtp(1, prompt[1:], [[i] * 3 for i in range(n - 1)], 0, False)
    committed, log = [tok], []
    rope, mtp_in = n, (n, [tok], [[n - 1] * 3], n - 1)
    for i in range(steps):
        r0, toks, pos, slot0 = mtp_in
        d = eng.mtp(r0, toks, pos, slot0, True)
        f = forced(i, committed)
        v = d if f is None else f
        slot = eng.pos
        lv = eng.forward_mm([tok, v], [[rope] * 3, [rope + 1] * 3], logit_rows=2, ckpt=True)
        a0, a1 = int(np.argmax(lv[0])), int(np.argmax(lv[1]))
        ok = a0 == v
        log.append((d, v, ok, lv))
        if ok:
            tok = a1
            committed += [v, tok]
            mtp_in = (1, [v, tok], [[rope] * 3, [rope + 1] * 3], slot)
            rope += 2
        else:
            eng.rollback()
            tok = a0
            committed.append(tok)
            mtp_in = (1, [tok], [[rope] * 3], slot)
            rope += 1
    return log, committed
