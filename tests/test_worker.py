"""The generation loop (snl_worker, worker.rs:118-338) on the CPU, over a host stand-in
for the engine (tests/fake_engine.py) that checks every call against the engine's rules.

The C++ loop is compared with an independent Python restatement of worker.rs on the
same stand-in: same tokens, same Finish counts, same sequence of engine calls. Also:
prefix reuse (live cache and snapshots) gives the tokens of a cold run, LRU eviction of
the snapshot slots, MTP on/off give identical greedy tokens, the self-pause after 16
drafts, EOS / length / disconnect, error recovery, and the generator's ChaCha block
against RFC 8439's known answer."""
from __future__ import annotations

import numpy as np
import pytest

from fake_engine import FakeEngine
from sensenova_b200 import ffi
from sensenova_b200.worker import GREEDY, Prompt, SamplingParams, Worker, uniforms
from test_sampler import py_sample

MASK32 = 0xFFFFFFFF


# ---- the generator -----------------------------------------------------------------------

def test_chacha_block_rfc8439_known_answer():
    """RFC 8439 section 2.3.2: key 00..1f, block count 1, nonce 00:00:00:09:00:00:00:4a:00:00:00:00."""
    key = [int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)]
    state = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574, *key, 1, 0x09000000, 0x4A000000, 0]
    want = [0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3, 0xC7F4D1C7, 0x0368C033, 0x9AAA2204, 0x4E6CD4C3,
            0x466482D2, 0x09AA9F07, 0x05D7C214, 0xA2028BD9, 0xD19C12B5, 0xB94E16DE, 0xE883D0CB, 0x4E3C50A2]
    lib = ffi.load()
    inp = np.array(state, dtype=np.uint32)
    out = np.zeros(16, dtype=np.uint32)
    ffi.check(lib.snl_chacha_block(inp.ctypes.data, 20, out.ctypes.data))
    assert out.tolist() == want


def _py_chacha12_uniforms(seed: int, n: int) -> list[float]:
    """The generator as documented: PCG32 key expansion, ChaCha12 blocks, top 24 bits."""
    def rotl(x, r):
        return ((x << r) | (x >> (32 - r))) & MASK32

    st, key = seed, []
    for _ in range(8):
        st = (st * 6364136223846793005 + 11634580027462260723) & ((1 << 64) - 1)
        xs = (((st >> 18) ^ st) >> 27) & MASK32
        rot = st >> 59
        key.append(((xs >> rot) | (xs << ((32 - rot) & 31))) & MASK32)
    out, ctr = [], 0
    while len(out) < n:
        s = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574, *key, ctr & MASK32, ctr >> 32, 0, 0]
        x = list(s)
        for _ in range(6):
            for a, b, c, d in ((0, 4, 8, 12), (1, 5, 9, 13), (2, 6, 10, 14), (3, 7, 11, 15),
                               (0, 5, 10, 15), (1, 6, 11, 12), (2, 7, 8, 13), (3, 4, 9, 14)):
                x[a] = (x[a] + x[b]) & MASK32; x[d] = rotl(x[d] ^ x[a], 16)
                x[c] = (x[c] + x[d]) & MASK32; x[b] = rotl(x[b] ^ x[c], 12)
                x[a] = (x[a] + x[b]) & MASK32; x[d] = rotl(x[d] ^ x[a], 8)
                x[c] = (x[c] + x[d]) & MASK32; x[b] = rotl(x[b] ^ x[c], 7)
        out += [float(np.float32(((x[i] + s[i]) & MASK32) >> 8) * np.float32(2.0 ** -24)) for i in range(16)]
        ctr += 1
    return out[:n]


@pytest.mark.parametrize("seed", [0, 1, 42, 2**63 + 5])
def test_uniforms_follow_the_documented_generator(seed):
    got = uniforms(seed, 40)
    assert got.tolist() == _py_chacha12_uniforms(seed, 40)
    assert ((got >= 0) & (got < 1)).all()


# ---- worker.rs restated in Python, over the same stand-in --------------------------------

class PyWorker:
    """worker.rs:118-270 and :298-338 in Python (text prompts; draws taken one at a time)."""

    def __init__(self, e: FakeEngine):
        self.e, self.live, self.snaps = e, [], [None] * 4
        self.spec, self.spec_pause, self.clock = False, 0, 0

    def feed(self, toks, pos, a, b, want):
        e = self.e
        for c0 in range(a, b, e.chunk):
            c1 = min(c0 + e.chunk, b)
            assert e.forward(toks[c0:c1], pos[c0:c1], {}, 1 if want and c1 == b else 0, False) == 0
            r0 = 1 if c0 == 0 else 0
            if self.spec and r0 < c1 - c0:
                assert e.mtp(r0, toks[c0 + r0:c1], pos[c0 + r0 - 1:c1 - 1], c0 + r0 - 1, False)[0] == 0

    def run(self, toks, params: SamplingParams, max_tokens, eos=(), snapshot_at=None):
        e, n = self.e, len(toks)
        keys, pos = list(toks), [(i, i, i) for i in range(n)]
        max_tokens = min(max_tokens, e.ctx - n)
        self.spec = e.has_mtp and self.spec_pause == 0
        self.spec_pause = max(self.spec_pause - 1, 0)
        self.clock += 1

        def shared(c, p):
            return len(c) if len(c) < len(p) and p[:len(c)] == c else 0

        live_hit, best = shared(self.live, keys), None
        for i, s in enumerate(self.snaps):
            if s is not None and (best is None or shared(s[0], keys) >= best[1]):
                best = (i, shared(s[0], keys))
        if best is not None and best[1] > live_hit:
            assert e.restore(best[0], best[1]) == 0
            self.snaps[best[0]] = (self.snaps[best[0]][0], self.clock)
            self.live = list(self.snaps[best[0]][0])
        elif live_hit == 0:
            e.reset()
            self.live = []
        cached = len(self.live)
        if snapshot_at is not None and len(self.live) < snapshot_at < n:
            self.feed(toks, pos, len(self.live), snapshot_at, False)
            slot = min(range(4), key=lambda i: 0 if self.snaps[i] is None else self.snaps[i][1])
            e.snapshot(slot)
            self.live = keys[:snapshot_at]
            self.snaps[slot] = (list(self.live), self.clock)
        self.feed(toks, pos, len(self.live), n, True)
        self.live = list(keys)
        rope = n
        u = uniforms(params.seed, 4096).tolist()
        ui, counts = [0], {}
        p = params.to_c()

        def pick(row, draft=-1):
            r = py_sample(p, e.kept[row], list(counts.items()), u[ui[0]:ui[0] + 2], draft)
            ui[0] += r[2]
            return r

        tok = pick(0)[0]
        mtp_in = (e.hid_rows, [tok], [pos[n - 1]], n - 1)
        out, st = [], {"reason": "length", "drafted": 0, "accepted": 0}

        def push(t):
            out.append(t)
            if t in eos:
                st["reason"] = "stop"
                return False
            return len(out) < max_tokens

        dsecs = vsecs = 0.0
        while push(tok):
            counts[tok] = counts.get(tok, 0) + 1
            t0 = e.t
            d = e.mtp(*mtp_in, True)[1] if self.spec else None
            dsecs += e.t - t0
            if d is None:
                e.forward([tok], [(rope,) * 3], {}, 1, False)
                self.live.append(tok)
                rope += 1
                tok = pick(0)[0]
                continue
            slot, tv = e.pos, e.t
            e.forward([tok, d], [(rope,) * 3, (rope + 1,) * 3], {}, 2, True)
            vsecs += e.t - tv
            st["drafted"] += 1
            if st["drafted"] == 16 and dsecs > vsecs * st["accepted"] / st["drafted"]:
                self.spec, self.spec_pause = False, 20
            nxt, ok, _ = pick(0, d)
            self.live.append(tok)
            if ok:
                st["accepted"] += 1
                self.live.append(d)
                if not push(d):
                    break
                counts[d] = counts.get(d, 0) + 1
                tok = pick(1)[0]
                mtp_in = (1, [d, tok], [(rope,) * 3, (rope + 1,) * 3], slot)
                rope += 2
            else:
                e.rollback()
                tok = nxt
                mtp_in = (1, [tok], [(rope,) * 3], slot)
                rope += 1
        return out, st["reason"], cached, st["drafted"], st["accepted"]


def _requests(rng, vocab, n_req):
    """Prompts that share prefixes with earlier prompts and with earlier outputs."""
    base = rng.integers(0, vocab, 30).tolist()
    reqs = []
    for i in range(n_req):
        kind = i % 4
        if kind == 0:
            toks = base[: int(rng.integers(12, 30))] + rng.integers(0, vocab, int(rng.integers(1, 20))).tolist()
        elif kind == 1:
            toks = rng.integers(0, vocab, int(rng.integers(5, 40))).tolist()
        else:
            toks = base + rng.integers(0, vocab, int(rng.integers(1, 9))).tolist()
        snap = int(rng.integers(3, len(toks))) if rng.random() < 0.6 else None
        reqs.append((toks, snap))
    return reqs


PARAMS = [
    SamplingParams(temperature=0.0, top_p=1.0, top_k=1, seed=3),
    SamplingParams(temperature=0.8, top_p=0.9, top_k=20, seed=11),
    SamplingParams(temperature=1.0, top_p=0.95, top_k=5, min_p=0.05, presence_penalty=0.3, repetition_penalty=1.1,
                   frequency_penalty=0.1, seed=7),
    SamplingParams(temperature=0.0, top_p=1.0, top_k=1, repetition_penalty=1.3, seed=1),
]


@pytest.mark.parametrize("mtp", [True, False])
@pytest.mark.parametrize("pi", range(len(PARAMS)))
def test_worker_matches_python_restatement(mtp, pi):
    params = PARAMS[pi]
    rng = np.random.default_rng(100 + pi)
    fc, fp = FakeEngine(mtp=mtp), FakeEngine(mtp=mtp)
    w, pw = Worker(ops=fc.ops), PyWorker(fp)
    eos = (int(rng.integers(0, fc.vocab)),)
    for toks, snap in _requests(rng, fc.vocab, 12):
        max_t = int(rng.integers(0, 30))
        got, fin = w.run(toks, params, max_t, eos=eos, snapshot_at=snap)
        want, reason, cached, drafted, accepted = pw.run(toks, params, max_t, eos=eos, snapshot_at=snap)
        assert got == want
        assert (fin.reason, fin.cached_tokens, fin.drafted, fin.accepted, fin.completion_tokens) == \
            (reason, cached, drafted, accepted, len(want))
        assert fin.prompt_tokens == len(toks)
        assert fc.calls == fp.calls
        assert not fc.violations and not fp.violations, fc.violations + fp.violations
        assert w.prefix(-1)[0] == pw.live
        for s in range(4):
            keys, used = w.prefix(s)
            assert (keys, used) == ((list(pw.snaps[s][0]), pw.snaps[s][1]) if pw.snaps[s] else ([], 0))


@pytest.mark.parametrize("params", [GREEDY, SamplingParams(temperature=0.7, top_k=10, seed=5)])
def test_prefix_reuse_gives_the_cold_tokens(params):
    rng = np.random.default_rng(9)
    shared = rng.integers(0, 48, 40).tolist()
    a = shared + rng.integers(0, 48, 10).tolist()
    b = shared + rng.integers(0, 48, 13).tolist()
    warm_e = FakeEngine()
    warm = Worker(ops=warm_e.ops)
    out_a, fin_a = warm.run(a, params, 12, snapshot_at=len(shared))
    assert fin_a.cached_tokens == 0
    out_b, fin_b = warm.run(b, params, 20)
    assert fin_b.cached_tokens == len(shared)
    assert ("restore", 0, len(shared)) in warm_e.calls
    cold = Worker(ops=FakeEngine().ops)
    assert cold.run(b, params, 20)[0] == out_b
    # Continuing the conversation reuses the live cache: prompt + fed reply + new turn.
    live = warm.prefix(-1)[0]
    assert live[:len(b)] == b and len(live) == warm_e.pos
    c = live + [1, 2, 3]
    out_c, fin_c = warm.run(c, params, 8)
    assert fin_c.cached_tokens == len(live)
    assert Worker(ops=FakeEngine().ops).run(c, params, 8)[0] == out_c
    assert not warm_e.violations, warm_e.violations


def test_live_cache_hit_feeds_only_the_new_tokens():
    e = FakeEngine()
    w = Worker(ops=e.ops)
    p = list(range(20))
    out, _ = w.run(p, GREEDY, 6)
    live = w.prefix(-1)[0]
    assert live[:20] == p and len(live) == e.pos
    nxt = live + [7, 8]
    e.calls.clear()
    _, fin = w.run(nxt, GREEDY, 3)
    assert fin.cached_tokens == len(live)
    assert e.calls[0][0] == "forward" and e.calls[0][1] == len(live) and e.calls[0][2] == [7, 8]


def test_snapshot_slots_evict_least_recently_used():
    e = FakeEngine(mtp=False)
    w = Worker(ops=e.ops)
    prefixes = [[100 + i] * 5 for i in range(4)]
    for i, pre in enumerate(prefixes):  # fills slots 0..3 (empty slots count as unused, first wins)
        w.run([x % 48 for x in pre] + [i], GREEDY, 2, snapshot_at=5)
        assert w.prefix(i)[0] == [x % 48 for x in pre]
    w.run([x % 48 for x in prefixes[0]] + [9, 9], GREEDY, 2)  # touches slot 0
    assert w.prefix(0)[1] == 5
    w.run([1, 2, 3, 4, 5, 6, 7], GREEDY, 2, snapshot_at=5)  # evicts slot 1, the least recently used
    assert w.prefix(1)[0] == [1, 2, 3, 4, 5]
    assert w.prefix(0)[0] == [x % 48 for x in prefixes[0]]
    assert not e.violations


def test_mtp_on_and_off_give_identical_greedy_tokens():
    rng = np.random.default_rng(4)
    on_e, off_e = FakeEngine(mtp=True), FakeEngine(mtp=False)
    on, off = Worker(ops=on_e.ops), Worker(ops=off_e.ops)
    drafted = accepted = 0
    for _ in range(6):
        toks = rng.integers(0, 48, int(rng.integers(3, 50))).tolist()
        a, fa = on.run(toks, GREEDY, 25)
        b, fb = off.run(toks, GREEDY, 25)
        assert a == b
        drafted += fa.drafted
        accepted += fa.accepted
        assert fb.drafted == 0
    assert drafted > 20 and 0 < accepted < drafted
    assert not on_e.violations


def test_mtp_head_sees_every_position():
    e = FakeEngine(mtp=True, chunk=5)
    w = Worker(ops=e.ops)
    toks = list(range(1, 23))
    out, fin = w.run(toks, GREEDY, 10)
    assert set(range(len(toks))) <= e.mtp_filled
    assert not e.violations


def test_drafting_pauses_when_it_does_not_pay_off():
    e = FakeEngine(mtp=True, draft_cost=5.0, fwd_cost=1.0, draft_hit=0.0)
    w = Worker(ops=e.ops)
    _, fin = w.run(list(range(10)), GREEDY, 40)
    assert fin.drafted == 16
    assert w.spec() == (False, 20)
    for i in range(20):
        _, f = w.run([i % 48, 1, 2], GREEDY, 3)
        assert f.drafted == 0
    _, f = w.run([5, 6, 7], GREEDY, 3)
    assert f.drafted > 0 and w.spec() == (True, 0)


def test_drafting_continues_when_it_pays_off():
    e = FakeEngine(mtp=True, draft_cost=0.1, fwd_cost=1.0, draft_hit=0.9)
    w = Worker(ops=e.ops)
    _, fin = w.run(list(range(10)), GREEDY, 60)
    assert fin.drafted > 16 and w.spec() == (True, 0)


def test_finish_reasons():
    e = FakeEngine(mtp=False)
    w = Worker(ops=e.ops)
    free, fin = w.run([3, 4, 5], GREEDY, 12)
    assert fin.reason == "length" and len(free) == 12
    stop_tok = free[4]
    out, fin = w.run([3, 4, 5], GREEDY, 12, eos=(stop_tok,))
    k = free.index(stop_tok)
    assert fin.reason == "stop" and out == free[:k + 1] and fin.completion_tokens == k + 1
    seen = []
    out, fin = w.run([3, 4, 5], GREEDY, 12, on_token=lambda t: seen.append(t) or len(seen) < 3)
    assert fin.cancelled and seen == free[:3] and fin.reason == "length"
    out, fin = w.run([3, 4, 5], GREEDY, 0)
    assert fin.completion_tokens == 1  # the loop pushes once before checking the limit
    out, fin = w.run(list(range(e.ctx - 4)), GREEDY, 100)
    assert fin.completion_tokens == 4  # max_tokens is capped at ctx - n


def test_errors_and_recovery():
    e = FakeEngine(ctx=50)
    w = Worker(ops=e.ops)
    with pytest.raises(ffi.SnlError, match="empty prompt"):
        w.run([], GREEDY, 4)
    with pytest.raises(ffi.SnlError, match=r"prompt is 50 tokens but the context size is 50; restart with a larger --ctx"):
        w.run(list(range(50)), GREEDY, 4)
    w.run(list(range(20)), GREEDY, 4, snapshot_at=10)
    assert w.prefix(0)[0] and w.prefix(-1)[0]
    e.fail_after = e.n_forward + 1
    with pytest.raises(ffi.SnlError):
        w.run(list(range(20)) + [1], GREEDY, 8)
    assert w.prefix(-1)[0] == [] and all(w.prefix(s) == ([], 0) for s in range(4))
    assert e.calls[-1] == ("reset",)
    e.fail_after = None
    out, fin = w.run(list(range(20)) + [1], GREEDY, 8)
    assert fin.cached_tokens == 0
    assert out == Worker(ops=FakeEngine(ctx=50).ops).run(list(range(20)) + [1], GREEDY, 8)[0]


def test_media_rows_reach_the_engine():
    e1, e2 = FakeEngine(mtp=False), FakeEngine(mtp=False)
    toks = list(range(1, 16))
    plain, _ = Worker(ops=e1.ops).run(toks, GREEDY, 8)
    rows = [(i, np.full(4, 0.5 + i, np.float32)) for i in (3, 4, 5, 11)]
    keys = [t if i not in (3, 4, 5, 11) else (1 << 63) | (77 + i) for i, t in enumerate(toks)]
    media, _ = Worker(ops=e2.ops).run(Prompt(toks, keys=keys, media_rows=rows), GREEDY, 8)
    assert media != plain
    assert not e2.violations


def test_worker_rejects_incomplete_ops():
    o = ffi.WorkerOps()
    with pytest.raises(ffi.SnlError, match="operations missing"):
        Worker(ops=o)
