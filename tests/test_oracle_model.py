"""The oracle's Engine restatement on the small configuration: the reference's own
self-consistency checks (README.md:32-47, main.rs:527-545) and its error messages."""
import numpy as np
import pytest

from sensenova_b200.config import nine_b, small


@pytest.fixture(scope="module")
def cfg():
    return small()


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_execution_plan():
    c = nine_b()
    plan = c.execution_plan()
    assert len(plan) == 56
    assert sum(c.full_attention[l] for l in plan) == 14
    assert plan[:4] == [0, 1, 2, 3] and plan[4:28] == list(range(4, 28)) and plan[28:52] == list(range(4, 28))
    assert c.lin_proj_rows == 12352 and c.attn_proj_rows == 10240 and c.conv_dim == 8192


def test_batched_equals_stepwise(orc, cfg):
    # `logits --stepwise` (main.rs:527-545): batched and token-by-token runs agree.
    toks = [(1000 + i * 7919) % cfg.vocab for i in range(12)]
    a = orc.OracleModel(cfg, 64, seed=1)
    la = a.forward(toks, True)
    b = orc.OracleModel(cfg, 64, seed=1)
    for t in toks:
        lb = b.forward([t], True)
    assert rel(la, lb) < 2e-3, rel(la, lb)
    assert int(np.argmax(la)) == int(np.argmax(lb))


def test_rollback_equals_never_fed(orc, cfg):
    a = orc.OracleModel(cfg, 64, seed=2)
    b = orc.OracleModel(cfg, 64, seed=2)
    prompt = [5, 17, 99, 400]
    a.forward(prompt, False)
    b.forward(prompt, False)
    a.forward_mm([7, 8], None, 2, True)  # verify [tok, draft]; the draft is then rejected
    a.rollback()
    assert a.pos == len(prompt) + 1 and a.hid_rows() == 1
    b.forward([7], False)
    la = a.forward([11], True)
    lb = b.forward([11], True)
    assert rel(la, lb) < 2e-3


def test_snapshot_restore_repeats_exactly(orc, cfg):
    a = orc.OracleModel(cfg, 64, seed=3)
    a.forward([1, 2, 3], False)
    a.snapshot(1)
    l1 = a.forward([4, 5], True)
    a.restore(1, 3)
    assert a.pos == 3
    l2 = a.forward([4, 5], True)
    assert np.array_equal(l1, l2)


def test_reset_repeats_exactly(orc, cfg):
    a = orc.OracleModel(cfg, 64, seed=4)
    l1 = a.forward([9, 10, 11], True)
    a.reset()
    l2 = a.forward([9, 10, 11], True)
    assert np.array_equal(l1, l2)


def test_two_logit_rows(orc, cfg):
    a = orc.OracleModel(cfg, 64, seed=5)
    a.forward([3, 4, 5], False)
    lg = a.forward_mm([6, 7], None, 2, False)
    assert lg.shape == (2, cfg.vocab)
    b = orc.OracleModel(cfg, 64, seed=5)
    b.forward([3, 4, 5], False)
    l6 = b.forward([6], True)
    assert rel(lg[0], l6) < 2e-3


def test_errors(orc, cfg):
    a = orc.OracleModel(cfg, 8, seed=6)
    with pytest.raises(orc.OracleError, match=r"context length exceeded \(9 > 8\)"):
        a.forward(list(range(9)), False)
    with pytest.raises(orc.OracleError, match="token id 5000 out of range"):
        a.forward([5000], False)
    with pytest.raises(orc.OracleError, match="unsupported logits or checkpoint request"):
        a.forward_mm([1, 2, 3], None, 3, False)
    with pytest.raises(orc.OracleError, match="unsupported logits or checkpoint request"):
        a.forward_mm([1, 2, 3], None, 1, True)


def test_multi_chunk_prefill(orc, cfg):
    # More than MAX_M = 512 tokens: two chunks, logits of the last.
    a = orc.OracleModel(cfg, 700, seed=7)
    toks = [(i * 31) % cfg.vocab for i in range(520)]
    lg = a.forward(toks, True)
    assert a.pos == 520 and a.hid_rows() == 8 and np.isfinite(lg).all()


def test_mtp_draft(orc, cfg):
    a = orc.OracleModel(cfg, 64, seed=8, mtp=True)
    prompt = [3, 1, 4, 1, 5]
    lg = a.forward(prompt, True)
    tok = int(np.argmax(lg))
    n = len(prompt)
    d = a.mtp(a.hid_rows(), [tok], [[n - 1] * 3], n - 1, True)
    assert 0 <= d < cfg.vocab
    with pytest.raises(orc.OracleError, match="mtp: rows out of range"):
        a.mtp(a.hid_rows() + 1, [tok], [[0] * 3], 0, True)
