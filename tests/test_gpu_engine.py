"""The engine (C ABI, engine level) against the oracle's Engine restatement on the
small configuration, plus the reference's own self-consistency checks on the GPU.

Bars: logits within 1e-3 relative; identical greedy
tokens over 256 decode steps; identical MTP accept/reject decisions.
"""
import numpy as np
import pytest

from sensenova_b200 import ffi
from sensenova_b200.config import small
from sensenova_b200.engine import Engine
from spec_loop import spec_loop

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def top2_gap(lg):
    s = np.sort(lg)
    return float(s[-1] - s[-2])


@pytest.fixture(scope="module")
def cfg():
    return small()


def pair(orc, cfg, ctx=320, seed=11, quant="q8_0", mtp=False):
    q = {"q8_0": 1, "q4_0": 2}[quant]
    return Engine.synthetic(cfg, ctx, seed, quant, mtp=mtp), orc.OracleModel(cfg, ctx, seed=seed, quant=q, mtp=mtp)


@pytest.mark.parametrize("quant", ["q8_0", "q4_0"])
def test_prefill_logits_match_oracle(torch_cuda, orc, cfg, quant):
    e, o = pair(orc, cfg, quant=quant)
    prompt = [(1000 + i * 7919) % cfg.vocab for i in range(37)]
    le = e.forward(prompt, True)
    lo = o.forward(prompt, True)
    assert rel(le, lo) < TOL, rel(le, lo)
    assert e.pos == o.pos == 37 and e.hid_rows() == o.hid_rows() == 37
    assert rel(e.read_hidden(0, 38), o.read_hidden(0, 38)) < TOL
    e.close()


def test_greedy_256_steps_identical(torch_cuda, orc, cfg):
    """Greedy decode: identical tokens over 256 steps (north_star), fp32 decode path."""
    e, o = pair(orc, cfg, seed=12)
    prompt = [(1000 + i * 7919) % cfg.vocab for i in range(16)]
    le, lo = e.forward(prompt, True), o.forward(prompt, True)
    te, to = int(np.argmax(le)), int(np.argmax(lo))
    toks_e, toks_o, gaps = [te], [to], []
    for step in range(256):
        le = e.forward([te], True)
        lo = o.forward([to], True)
        assert rel(le, lo) < TOL, (step, rel(le, lo))
        te, to = int(np.argmax(le)), int(np.argmax(lo))
        gaps.append(top2_gap(lo))
        toks_e.append(te)
        toks_o.append(to)
        assert te == to, f"step {step}: {te} != {to}, oracle top-2 gap {gaps[-1]:.3g}"
    assert toks_e == toks_o
    e.close()


def test_simt_fallback_path_matches_oracle(torch_cuda, orc, cfg, monkeypatch):
    """SNL_NO_TC: the same engine on the SIMT GEMVs and separate merge kernels."""
    monkeypatch.setenv("SNL_NO_TC", "1")
    e = Engine.synthetic(cfg, 320, 21)
    monkeypatch.delenv("SNL_NO_TC")
    o = orc.OracleModel(cfg, 320, seed=21)
    prompt = [(3 + i * 101) % cfg.vocab for i in range(9)]
    le, lo = e.forward(prompt, True), o.forward(prompt, True)
    assert rel(le, lo) < TOL
    for _ in range(8):
        t = int(np.argmax(lo))
        le, lo = e.forward([t], True), o.forward([t], True)
        assert rel(le, lo) < TOL and int(np.argmax(le)) == int(np.argmax(lo))
    e.close()


def test_long_context_decode_matches_oracle(torch_cuda, orc, cfg):
    """Decode past 4096 keys of context, where the split-key attention needs more than 64
    parts (a second captured decode graph): logits within 1e-3 and the same greedy
    tokens as the oracle."""
    e, o = pair(orc, cfg, ctx=4400, seed=21)
    prompt = [(1000 + i * 7919) % cfg.vocab for i in range(4200)]
    le, lo = e.forward(prompt, True), o.forward(prompt, True)
    assert rel(le, lo) < TOL, rel(le, lo)
    te, to = int(np.argmax(le)), int(np.argmax(lo))
    for step in range(4):
        assert te == to, (step, te, to)
        le, lo = e.forward([te], True), o.forward([to], True)
        assert rel(le, lo) < TOL, (step, rel(le, lo))
        te, to = int(np.argmax(le)), int(np.argmax(lo))
    e.close()


def test_forward_greedy_matches_logits(torch_cuda, orc, cfg):
    e, _ = pair(orc, cfg, seed=13)
    e2 = Engine.synthetic(cfg, 320, 13)
    prompt = list(range(3, 20))
    lg = e.forward(prompt, True)
    ids = e2.forward_greedy(prompt, None, 1)
    assert ids == [int(np.argmax(lg))]
    for _ in range(20):
        lg = e.forward([ids[0]], True)
        ids = e2.forward_greedy([ids[0]], None, 1)
        assert ids == [int(np.argmax(lg))]
    e.close()
    e2.close()


def test_weight_planes_bitwise(torch_cuda, cfg, monkeypatch):
    """Prefill rows with the engine's weight planes (default) give the same logits, bit
    for bit, as the dequantizing GEMM (SNL_NO_WPLANES)."""
    a = Engine.synthetic(cfg, 320, 33)
    monkeypatch.setenv("SNL_NO_WPLANES", "1")
    b = Engine.synthetic(cfg, 320, 33)
    monkeypatch.delenv("SNL_NO_WPLANES")
    prompt = [(5 + i * 53) % cfg.vocab for i in range(45)]
    la, lb = a.forward(prompt, True), b.forward(prompt, True)
    assert np.array_equal(la, lb)
    t = int(np.argmax(la))
    la, lb = a.forward([t], True), b.forward([t], True)
    assert np.array_equal(la, lb)
    a.close()
    b.close()


def test_engine_sample_on_device_matches_oracle(torch_cuda, orc, cfg):
    """snl_engine_sample on the logits a forward kept on the device gives the oracle
    sampler's result on the same logits (copied out by a twin engine), for sampling and
    for speculative verify, with a growing history of generated tokens."""
    from sensenova_b200.ffi import SampleP

    a = Engine.synthetic(cfg, 320, 41)
    b = Engine.synthetic(cfg, 320, 41)
    rng = np.random.default_rng(5)
    params = [SampleP(1.0, 0.95, 20, 0.0, 0.0, 0.0, 1.0, 0), SampleP(0.7, 0.8, 64, 0.05, 0.2, 0.1, 1.1, 0),
              SampleP(0.0, 1.0, 1, 0.0, 0.0, 0.0, 1.3, 0)]
    hist: dict[int, int] = {}
    tok = [3, 14, 15, 92, 65]
    for step in range(12):
        p = params[step % 3]
        lg = b.forward(tok, True)
        a.forward_keep(tok, 1)
        u = rng.random(2).astype(np.float32)
        draft = -1 if step % 2 == 0 else int(np.argmax(lg))
        want = orc.sample(p, lg.copy().ravel(), list(hist.keys()), list(hist.values()), u, draft)
        got = a.sample(0, p, hist, u, draft)
        assert (got[0], int(got[1]), got[2]) == want, (step, got, want)
        tok = [got[0]]
        hist[got[0]] = hist.get(got[0], 0) + 1
    a.close()
    b.close()


def test_verify_two_rows_and_rollback(torch_cuda, orc, cfg):
    e, o = pair(orc, cfg, seed=14)
    prompt = [5, 17, 99, 400, 1234, 7]
    e.forward(prompt, False)
    o.forward(prompt, False)
    le = e.forward_mm([7, 8], None, (), 2, True)
    lo = o.forward_mm([7, 8], None, 2, True)
    assert le.shape == (2, cfg.vocab) and rel(le, lo) < TOL
    e.rollback()
    o.rollback()
    assert e.pos == o.pos == len(prompt) + 1 and e.hid_rows() == 1
    le, lo = e.forward([11], True), o.forward([11], True)
    assert rel(le, lo) < TOL
    # rollback == never fed the draft (engine.rs:685-697)
    f = Engine.synthetic(cfg, 320, 14)
    f.forward(prompt, False)
    f.forward([7], False)
    lf = f.forward([11], True)
    assert rel(le, lf) < TOL
    assert int(np.argmax(le)) == int(np.argmax(lf))
    e.close()
    f.close()


def test_batched_equals_stepwise(torch_cuda, cfg):
    a = Engine.synthetic(cfg, 320, 15)
    b = Engine.synthetic(cfg, 320, 15)
    toks = [(7 + i * 131) % cfg.vocab for i in range(40)]
    la = a.forward(toks, True)
    for t in toks:
        lb = b.forward([t], True)
    assert rel(la, lb) < 2e-3 and int(np.argmax(la)) == int(np.argmax(lb))


def test_snapshot_restore_and_reset_exact(torch_cuda, cfg):
    e = Engine.synthetic(cfg, 320, 16)
    e.forward([1, 2, 3], False)
    e.snapshot(2)
    l1 = e.forward([4, 5], True)
    e.restore(2, 3)
    l2 = e.forward([4, 5], True)
    assert np.array_equal(l1, l2)
    e.reset()
    l3 = e.forward([1, 2, 3, 4, 5], True)
    assert rel(l3, l1) < 2e-3
    e.close()


def test_multi_chunk_prefill(torch_cuda, orc, cfg):
    e, o = pair(orc, cfg, ctx=700, seed=17)
    toks = [(i * 31) % cfg.vocab for i in range(530)]
    le, lo = e.forward(toks, True), o.forward(toks, True)
    assert rel(le, lo) < TOL and e.hid_rows() == 18
    e.close()


def test_mtp_draft_matches_oracle(torch_cuda, orc, cfg):
    e, o = pair(orc, cfg, seed=18, mtp=True)
    assert e.has_mtp()
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    le, lo = e.forward(prompt, True), o.forward(prompt, True)
    n = len(prompt)
    tok = int(np.argmax(lo))
    assert int(np.argmax(le)) == tok
    # warm-up over the prompt rows (worker.rs:316-318), then a draft
    assert e.mtp(1, prompt[1:], [[i] * 3 for i in range(n - 1)], 0, False) is None
    o.mtp(1, prompt[1:], [[i] * 3 for i in range(n - 1)], 0, False)
    de = e.mtp(n, [tok], [[n - 1] * 3], n - 1, True)
    do = o.mtp(n, [tok], [[n - 1] * 3], n - 1, True)
    assert de == do
    # accept/reject decision: greedy verify accepts iff argmax == draft (sampler.rs:63-66)
    ve = e.forward_mm([tok, de], [[n] * 3, [n + 1] * 3], (), 2, True)
    vo = o.forward_mm([tok, do], [[n] * 3, [n + 1] * 3], 2, True)
    assert (int(np.argmax(ve[0])) == de) == (int(np.argmax(vo[0])) == do)
    e.close()


def test_mtp_accept_and_reject_decisions_match_oracle(torch_cuda, orc, cfg):
    """Every draft, accept/reject decision, verify row and committed token of 12
    speculative steps against the oracle. Odd steps verify the true greedy continuation
    (accept branch: no rollback, both verify rows kept), even steps the MTP head's own
    draft (reject branch with random weights). The committed text equals plain greedy
    decoding (MTP on/off identity, README.md:42)."""
    e, o = pair(orc, cfg, seed=19, mtp=True)
    prompt = [2, 7, 1, 8, 2, 8, 1, 8, 2, 8]
    g = orc.OracleModel(cfg, 320, seed=19, quant=1)
    greedy = [int(np.argmax(g.forward(prompt, True)))]
    for _ in range(40):
        greedy.append(int(np.argmax(g.forward([greedy[-1]], True))))
    g.close()

    def forced(i, committed):
        return greedy[len(committed)] if i % 2 == 1 else None

    le, ce = spec_loop(e, prompt, 12, forced)
    lo, co = spec_loop(o, prompt, 12, forced)
    assert [x[0] for x in le] == [x[0] for x in lo]  # MTP drafts
    assert [x[1] for x in le] == [x[1] for x in lo]  # verified tokens
    assert [x[2] for x in le] == [x[2] for x in lo]  # accept / reject decisions
    assert any(x[2] for x in le) and not all(x[2] for x in le)  # both branches taken
    for (_, _, _, a), (_, _, _, b) in zip(le, lo):
        assert rel(a, b) < TOL
    assert ce == co == greedy[: len(ce)]
    assert e.pos == o.pos
    e.close()


def test_snl_file_roundtrip(torch_cuda, orc, cfg, tmp_path):
    """Engine.load of a .snl file (weights.rs layout) == the same weights generated in place."""
    from sensenova_b200.weights import write_snl
    import sys
    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parent.parent / "sense-nova-server_b200" / "csrc"))

    o = orc.OracleModel(cfg, 64, seed=19)
    tensors = {}
    import ctypes as C

    names = []
    from sensenova_b200.config import ModelConfig  # noqa: F401

    # enumerate the tensor list through the oracle (same list as the engine's generator)
    for nm in ["embed", "lm_head", "norm"] + [f"l{i}.{s}" for i in range(cfg.n_layers) for s in
                                               ("in_ln", "post_ln", "qk_norm", "lin", "qkv", "o_proj", "in_proj",
                                                "out_proj", "mhc_attn", "mhc_ffn", "gate_up", "down")]:
        try:
            p, r, c, s = o.tensor(nm)
        except KeyError:
            continue
        names.append(nm)
        if s:  # quantized (Q8 here)
            q = np.ctypeslib.as_array((C.c_uint8 * (r * c)).from_address(p)).copy()
            sc = np.ctypeslib.as_array((C.c_float * (r * c // 32)).from_address(s)).copy()
            tensors[nm] = ("q8_0", [r, c], q.tobytes(), sc.tobytes())
        else:
            v = np.ctypeslib.as_array((C.c_float * c).from_address(p)).copy()
            tensors[nm] = ("f32", [c], v.tobytes(), b"")
    path = tmp_path / "m.snl"
    write_snl(path, "synthetic", "q8_0", cfg, tensors)
    a = Engine.load(path, 64)
    b = Engine.synthetic(cfg, 64, 19)
    la, lb = a.forward([1, 2, 3, 4], True), b.forward([1, 2, 3, 4], True)
    assert np.array_equal(la, lb)
    a.close()
    b.close()


def test_errors(torch_cuda, cfg):
    e = Engine.synthetic(cfg, 8, 20)
    with pytest.raises(ffi.SnlError, match=r"context length exceeded \(9 > 8\)"):
        e.forward(list(range(9)), False)
    with pytest.raises(ffi.SnlError, match="token id 5000 out of range"):
        e.forward([5000], False)
    with pytest.raises(ffi.SnlError, match="unsupported logits or checkpoint request"):
        e.forward_mm([1, 2, 3], None, (), 3, False)
    with pytest.raises(ffi.SnlError, match="unsupported logits or checkpoint request"):
        e.forward_mm([1, 2, 3], None, (), 1, True)
    assert e.mtp(0, [1], [[0, 0, 0]], 0, True) is None  # no MTP head: None, like the reference
    e.forward([1, 2], False)  # the engine still works after rejected calls
    assert e.pos == 2
    e.close()
