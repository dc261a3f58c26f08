"""The generation loop (snl_worker) over the CUDA engine on the small configuration.

Greedy requests give the oracle's greedy tokens with and without MTP drafting; a
request resumed from a snapshot gives the tokens of a cold run with the same step
boundaries (bit-identical states, so sampled tokens match too); the live cache resumes
a continued conversation; a seed fixes the sampled tokens."""
import numpy as np
import pytest

from sensenova_b200.config import small
from sensenova_b200.engine import Engine
from sensenova_b200.worker import GREEDY, SamplingParams, Worker

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg():
    return small()


def oracle_greedy(orc, cfg, prompt, n, seed):
    o = orc.OracleModel(cfg, 320, seed=seed, quant=1)
    lg = o.forward(prompt, True)
    out = [int(np.argmax(lg))]
    while len(out) < n:
        out.append(int(np.argmax(o.forward([out[-1]], True))))
    return out


def test_worker_greedy_matches_oracle_with_and_without_mtp(torch_cuda, orc, cfg):
    prompt = [(17 + i * 7919) % cfg.vocab for i in range(41)]
    want = oracle_greedy(orc, cfg, prompt, 48, seed=21)
    with_mtp = Engine.synthetic(cfg, 320, 21, mtp=True)
    plain = Engine.synthetic(cfg, 320, 21)
    got_m, fin_m = Worker(with_mtp).run(prompt, GREEDY, 48)
    got_p, fin_p = Worker(plain).run(prompt, GREEDY, 48)
    assert got_m == want and got_p == want
    assert fin_m.drafted > 0 and fin_p.drafted == 0
    assert fin_m.completion_tokens == 48 and fin_m.reason == "length"
    with_mtp.close()
    plain.close()


@pytest.mark.parametrize("params", [GREEDY, SamplingParams(temperature=0.8, top_k=20, top_p=0.9, seed=5),
                                    SamplingParams(temperature=1.0, top_k=40, min_p=0.02, presence_penalty=0.2,
                                                   repetition_penalty=1.1, seed=9)])
def test_snapshot_resume_equals_cold_run(torch_cuda, cfg, params):
    rng = np.random.default_rng(3)
    shared = rng.integers(0, cfg.vocab, 70).tolist()
    p1 = shared + rng.integers(0, cfg.vocab, 9).tolist()
    p2 = shared + rng.integers(0, cfg.vocab, 23).tolist()
    warm_e = Engine.synthetic(cfg, 320, 31, mtp=True)
    warm = Worker(warm_e)
    warm.run(p1, params, 16, snapshot_at=len(shared))
    out_w, fin_w = warm.run(p2, params, 24)
    assert fin_w.cached_tokens == len(shared)
    cold_e = Engine.synthetic(cfg, 320, 31, mtp=True)
    out_c, fin_c = Worker(cold_e).run(p2, params, 24, snapshot_at=len(shared))
    assert fin_c.cached_tokens == 0
    assert out_w == out_c
    assert (fin_w.drafted, fin_w.accepted) == (fin_c.drafted, fin_c.accepted)
    warm_e.close()
    cold_e.close()


def test_live_cache_continuation(torch_cuda, orc, cfg):
    e = Engine.synthetic(cfg, 320, 23)
    w = Worker(e)
    prompt = [(5 + i * 104729) % cfg.vocab for i in range(30)]
    w.run(prompt, GREEDY, 12)
    live = w.prefix(-1)[0]
    assert live[:30] == prompt and len(live) == e.pos
    turn = live + [7, 11, 13]
    out, fin = w.run(turn, GREEDY, 16)
    assert fin.cached_tokens == len(live)
    assert out == oracle_greedy(orc, cfg, turn, 16, seed=23)
    e.close()


def test_seed_fixes_sampled_tokens(torch_cuda, cfg):
    prompt = list(range(3, 40))
    outs = []
    for seed in (77, 77, 78):
        e = Engine.synthetic(cfg, 320, 29, mtp=True)
        outs.append(Worker(e).run(prompt, SamplingParams(temperature=1.0, top_k=50, seed=seed), 32)[0])
        e.close()
    assert outs[0] == outs[1]
    assert outs[0] != outs[2]
