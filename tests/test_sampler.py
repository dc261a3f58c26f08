"""The oracle's restatement of the reference sampler (sampler.rs:54-167) against an
independent Python port of the same code, on seeded random cases: penalties, greedy,
top-k (the top_k_small order), temperature, min-p, top-p, draw and speculative verify
with the caller's uniform draws. CPU only."""
import math

import numpy as np
import pytest

from sensenova_b200.ffi import SampleP


def py_sample(p, logits, hist, u, draft=-1):
    """sampler.rs:54-167 in Python with f32 rounding at each step (np.float32)."""
    f = np.float32
    lg = logits.astype(np.float32).copy()
    for t, c in hist:
        l = lg[t]
        if p.repetition_penalty != 1.0:
            l = f(l / f(p.repetition_penalty)) if l > 0 else f(l * f(p.repetition_penalty))
        lg[t] = f(l - f(f(p.presence_penalty) + f(f(p.frequency_penalty) * f(c))))
    if p.temperature <= 1e-5:
        t = int(np.argmax(lg))  # first maximum
        return t, int(draft == t), 0
    k = len(lg) if p.top_k == 0 else min(p.top_k, len(lg))
    order = sorted(range(len(lg)), key=lambda i: (-float(lg[i]), i))[:k]  # descending, ties by index
    mx = lg[order[0]]
    probs = [f(math.exp(float(f(f(lg[i] - mx) / f(p.temperature))))) for i in order]
    s = f(0)
    for x in probs:
        s = f(s + x)
    probs = [f(x / s) for x in probs]
    keep = k
    if p.min_p > 0:
        th = f(probs[0] * f(p.min_p))
        keep = 0
        while keep < k and probs[keep] >= th:
            keep += 1
        keep = max(keep, 1)
    if p.top_p < 1:
        cum = f(0)
        for i in range(keep):
            cum = f(cum + probs[i])
            if cum >= f(p.top_p):
                keep = i + 1
                break
    tot = f(0)
    for i in range(keep):
        tot = f(tot + probs[i])
    probs = [f(x / tot) for x in probs[:keep]]
    toks = order[:keep]

    def draw(uu, excl):
        total = f(0)
        for t, x in zip(toks, probs):
            if t != excl:
                total = f(total + x)
        r = f(f(uu) * total)
        last = toks[0]
        for t, x in zip(toks, probs):
            if t == excl:
                continue
            r = f(r - x)
            last = t
            if r <= 0:
                return t
        return last

    if draft < 0:
        return draw(u[0], -1), 0, 1
    pd = next((x for t, x in zip(toks, probs) if t == draft), f(0))
    if pd > 0 and f(u[0]) < pd:
        return draft, 1, 1
    return draw(u[1] if pd > 0 else u[0], draft), 0, (2 if pd > 0 else 1)


def params(rng):
    temp = float(rng.choice([0.0, 0.5, 0.8, 1.0, 1.3]))
    return SampleP(temp, float(rng.choice([1.0, 0.95, 0.8, 0.5])), int(rng.choice([1, 5, 20, 64, 256])),
                   float(rng.choice([0.0, 0.05, 0.2])), float(rng.choice([0.0, 0.3])), float(rng.choice([0.0, 0.1])),
                   float(rng.choice([1.0, 1.1, 0.9])), 0)


def case(rng, n):
    logits = (rng.standard_normal(n) * rng.choice([1.0, 3.0])).astype(np.float32)
    ht = rng.choice(n, size=int(rng.integers(0, 12)), replace=False).astype(np.uint32)
    hc = rng.integers(1, 4, size=ht.size).astype(np.uint32)
    u = rng.random(2).astype(np.float32)
    draft = int(rng.integers(-1, n)) if rng.random() < 0.5 else -1
    if draft >= 0 and rng.random() < 0.5:
        draft = int(np.argmax(logits))
    return logits, ht, hc, u, draft


def test_oracle_sampler_matches_python_port(orc):
    rng = np.random.default_rng(2024)
    for _ in range(400):
        p = params(rng)
        logits, ht, hc, u, draft = case(rng, int(rng.choice([50, 300, 1000])))
        got = orc.sample(p, logits.copy(), ht, hc, u, draft)
        want = py_sample(p, logits, list(zip(ht.tolist(), hc.tolist())), u.tolist(), draft)
        assert got == want, (p.temperature, p.top_k, p.top_p, p.min_p, got, want)


def test_oracle_sampler_refuses_large_top_k(orc):
    p = SampleP(1.0, 0.95, 300, 0.0, 0.0, 0.0, 1.0, 0)
    with pytest.raises(RuntimeError):
        orc.sample(p, np.zeros(1000, np.float32), [], [], [0.5, 0.5])
