"""The oracle against the reference's OWN kernels: every WGSL entry point of the hot path
(matmul.wgsl with both quant splices of gpu.rs, layers.wgsl, attention.wgsl,
linear.wgsl, vision.wgsl), translated to C++ by oracle/wgsl2cpp.py and run on the host
cores with the reference engine's workgroup grids (oracle/wgslref.py).

Both run in f32 with the same host libm, so the restatement must give the reference's
bits exactly: same operands, same summation order, same tree reductions. This pins the
oracle that every GPU parity test compares against.

Needs the reference tree (present where the CPU suite runs, absent on the GPU box); the
committed golden fixtures (tests/golden/) carry the same evidence to machines without it.
"""
import numpy as np
import pytest

import wgslref as wr
from sensenova_b200.ffi import AttnP, LayerP, LinP, MatP, StepU, VisP, SNL_Q4_0, SNL_Q8_0

pytestmark = pytest.mark.skipif(not wr.available(), reason="reference tree absent")


def same(a: np.ndarray, b: np.ndarray, what: str, live: bool = True) -> None:
    """Bit-identical; live: the output was written (not all zero), so equality means something."""
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape, what
    if live:
        assert np.any(np.nan_to_num(a.astype(np.float64)) != 0), f"{what}: output never written"
    if not np.array_equal(a.view(np.uint32), b.view(np.uint32)):
        d = np.abs(a.astype(np.float64) - b.astype(np.float64))
        raise AssertionError(f"{what}: {int((d > 0).sum())} of {a.size} differ, max |diff| {d.max():.3g}")


def both(fo, fr, *bufs):
    """Run the oracle (fo) and the reference kernel (fr) on separate copies of the
    buffers; return both sets after the call (in-place updates included)."""
    a = [None if b is None else b.copy() for b in bufs]
    r = [None if b is None else b.copy() for b in bufs]
    fo(*a)
    fr(*r)
    return a, r


# ---- matmul.wgsl ----------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m,n,k", [(1, 96, 1024), (1, 45, 4096), (2, 70, 512), (3, 33, 1056), (8, 24, 800),
                                   (9, 37, 288), (40, 130, 320), (130, 21, 256)])
def test_mat(orc, dtype, m, n, k):
    """matvec1 (m=1), matvec2 (m=2), matvec (3..8), matmul (>8; ragged 128-tiles)."""
    rng = np.random.default_rng(m * 100 + n + dtype)
    q, s = orc.gen_quant(5, f"r{dtype}", dtype, n, k)
    xs = k + 8  # x_stride and x_off in whole vec4s, as MatP requires (matmul.wgsl:20-21)
    x = rng.standard_normal(4 + m * xs).astype(np.float32)
    y = np.full(3 + m * (n + 5), np.nan, np.float32)
    p = MatP(n, k, 4, xs, 3, n + 5, 2, 0)
    st = StepU(m, 0, 1, 0)
    (yo,), (yr,) = both(lambda y_: orc.mat(dtype, st, p, x, q, s, y_), lambda y_: wr.mat(dtype, st, p, x, q, s, y_), y)
    same(yo, yr, f"mat dtype {dtype} m {m}")


def test_mat_head_rows(orc):
    """The LM head's use: x_off at the last rows, m_one fixing the row count (engine.rs:835-842)."""
    rng = np.random.default_rng(3)
    n, k, h = 40, 256, 256
    q, s = orc.gen_quant(1, "head", SNL_Q8_0, n, k)
    hid = rng.standard_normal((6, h)).astype(np.float32)
    for m_one in (1, 2):
        p = MatP(n, k, (6 - m_one) * h, h, 0, n, 0, m_one)
        st = StepU(6, 0, 1, 0)
        y = np.zeros((m_one, n), np.float32)
        (yo,), (yr,) = both(lambda y_: orc.mat(SNL_Q8_0, st, p, hid, q, s, y_),
                            lambda y_: wr.mat(SNL_Q8_0, st, p, hid, q, s, y_), y)
        same(yo, yr, f"head m_one {m_one}")


# ---- layers.wgsl ----------------------------------------------------------------------


def layer_p(h, mode=0, last_row=0, eps=1e-6, weight_one=1.0, iterations=20, inter=0, x_stride=0):
    return LayerP(h, mode, last_row, eps, weight_one, iterations, inter, x_stride)


@pytest.mark.parametrize("mode,h", [(0, 512), (1, 512), (1, 4096), (0, 300)])
def test_branch_norm(orc, mode, h):
    rng = np.random.default_rng(mode + h)
    m = 5
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0.1, 1.0, (m, 8)).astype(np.float32)
    w = (0.1 * rng.standard_normal(h)).astype(np.float32)
    out = np.zeros((m, h), np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(h, mode)
    a, r = both(lambda *b: orc.branch_norm(st, p, *b, m), lambda *b: wr.branch_norm(st, p, *b, m), x, coef, w, out)
    same(a[3], r[3], "branch_norm")


def test_branch_norm_last_row_stride(orc):
    rng = np.random.default_rng(5)
    m, h = 4, 256
    x = rng.standard_normal((m, h)).astype(np.float32)
    w = (0.1 * rng.standard_normal(h)).astype(np.float32)
    out = np.zeros(h, np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(h, 0, last_row=1, x_stride=h, weight_one=0.0)
    a, r = both(lambda *b: orc.branch_norm(st, p, *b, 1), lambda *b: wr.branch_norm(st, p, *b, 1),
                x, np.zeros(8 * m, np.float32), w, out)
    same(a[3], r[3], "branch_norm last row")


@pytest.mark.parametrize("h,iters", [(256, 20), (4096, 20), (512, 3)])
def test_mhc_router(orc, h, iters):
    rng = np.random.default_rng(h + iters)
    m, d = 3, 2 * h
    x = rng.standard_normal((m, d)).astype(np.float32)
    w = np.concatenate([0.02 * rng.standard_normal(8 * d), 0.1 * rng.standard_normal(8)]).astype(np.float32)
    raw = np.zeros((m, 9), np.float32)
    coef = np.zeros((m, 8), np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(h, iterations=iters)
    a, r = both(lambda x_, w_, raw_: orc.mhc_dots(st, p, x_, w_, raw_),
                lambda x_, w_, raw_: wr.mhc_dots(st, p, x_, w_, raw_), x, w, raw)
    same(a[2], r[2], "mhc_dots")
    a, r = both(lambda raw_, coef_: orc.mhc_finish(st, p, raw_, w, coef_),
                lambda raw_, coef_: wr.mhc_finish(st, p, raw_, w, coef_), a[2], coef)
    same(a[1], r[1], "mhc_finish")


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_merge(orc, mode):
    rng = np.random.default_rng(mode)
    m, h = 3, 300
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0, 1, (m, 8)).astype(np.float32)
    br = rng.standard_normal((m, h)).astype(np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(h, mode)
    a, r = both(lambda *b: orc.merge(st, p, *b), lambda *b: wr.merge(st, p, *b), x, coef, br)
    same(a[0], r[0], f"merge mode {mode}")


def test_swiglu(orc):
    rng = np.random.default_rng(2)
    m, inter = 3, 700
    gu = rng.standard_normal((m, 2 * inter)).astype(np.float32)
    act = np.zeros((m, inter), np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(64, inter=inter)
    a, r = both(lambda *b: orc.swiglu(st, p, *b), lambda *b: wr.swiglu(st, p, *b), gu, act)
    same(a[1], r[1], "swiglu")


# ---- attention.wgsl -------------------------------------------------------------------

HD = 256


def attn_setup(rng, m, pos0, n_kv=1, rot=64, ctx=96, mrope=(33 << 16) | 30):
    nh = 4 * n_kv
    q_dim, kv_dim = nh * HD, n_kv * HD
    stride = 2 * q_dim + 2 * kv_dim
    p = AttnP(nh, n_kv, rot, stride, 1e7, 1e-6, 1 / 16, mrope)
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    norms = (0.1 * rng.standard_normal(2 * HD)).astype(np.float32)
    kc = np.zeros(ctx * kv_dim // 2, np.uint32)
    vc = np.zeros_like(kc)
    kc[: pos0 * kv_dim // 2] = rng.standard_normal(pos0 * kv_dim).astype(np.float16).view(np.uint32)
    vc[: pos0 * kv_dim // 2] = rng.standard_normal(pos0 * kv_dim).astype(np.float16).view(np.uint32)
    rpos = np.stack([np.arange(pos0, pos0 + m), np.arange(m) * 3 + 1, np.arange(m) * 5 + 2,
                     np.zeros(m, np.int64)], 1).astype(np.uint32)
    return p, proj, norms, kc, vc, rpos


@pytest.mark.parametrize("m,pos0,n_kv,rot", [(3, 5, 1, 64), (2, 0, 2, 256), (1, 60, 2, 64)])
def test_attn_prep(orc, m, pos0, n_kv, rot):
    rng = np.random.default_rng(m + pos0 + rot)
    p, proj, norms, kc, vc, rpos = attn_setup(rng, m, pos0, n_kv, rot)
    qbuf = np.zeros((m, p.n_heads * HD), np.float32)
    st = StepU(m, pos0, 1, 0)
    a, r = both(lambda *b: orc.attn_prep(st, p, proj, *b, norms, rpos),
                lambda *b: wr.attn_prep(st, p, proj, *b, norms, rpos), qbuf, kc, vc)
    same(a[0], r[0], "prep q")
    assert np.array_equal(a[1], r[1]), "prep k cache"
    assert np.array_equal(a[2], r[2]), "prep v cache"


@pytest.mark.parametrize("m,pos0,n_kv,parts", [(1, 40, 1, 1), (2, 37, 2, 1), (2, 37, 2, 3), (1, 90, 1, 4),
                                                (4, 16, 1, 2), (5, 0, 1, 1)])
def test_attend_combine(orc, m, pos0, n_kv, parts):
    rng = np.random.default_rng(m * 7 + pos0 + parts)
    p, proj, norms, kc, vc, rpos = attn_setup(rng, m, pos0 + m, n_kv)
    st = StepU(m, pos0, parts, 0)
    qbuf = rng.standard_normal((m, p.n_heads * HD)).astype(np.float32)
    out = np.zeros((m, p.n_heads * HD), np.float32)
    partial = np.zeros((m * p.n_heads * parts, HD + 2), np.float32)
    a, r = both(lambda o, pt: orc.attend(st, p, proj, qbuf, kc, vc, o, pt),
                lambda o, pt: wr.attend(st, p, proj, qbuf, kc, vc, o, pt), out, partial)
    if parts == 1:
        same(a[0], r[0], "attend out")
        return
    same(a[1], r[1], "attend partials")
    a, r = both(lambda pt, o: orc.attn_combine(st, p, proj, pt, o),
                lambda pt, o: wr.attn_combine(st, p, proj, pt, o), a[1], out)
    same(a[1], r[1], "combine out")


# ---- linear.wgsl ----------------------------------------------------------------------


def lin_setup(rng, m, n_k=2, n_v=4):
    cd = 2 * n_k * 128 + n_v * 128
    stride = cd + n_v * 128 + 2 * n_v
    lp = LinP(cd, stride, n_k, n_v, 1e-6, (0, 0, 0))
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    lw = np.concatenate([0.5 * rng.standard_normal(cd * 4), 0.1 * rng.standard_normal(n_v),
                         0.1 * rng.standard_normal(n_v), 1 + 0.1 * rng.standard_normal(128)]).astype(np.float32)
    return lp, proj, lw, cd


@pytest.mark.parametrize("m,ckpt", [(1, 0), (5, 2), (9, 9)])
def test_conv(orc, m, ckpt):
    rng = np.random.default_rng(8 + m)
    lp, proj, lw, cd = lin_setup(rng, m)
    cs = rng.standard_normal((3, cd)).astype(np.float32)
    out = np.zeros((m, cd), np.float32)
    ck = np.zeros((3, cd), np.float32)
    st = StepU(m, 0, 1, ckpt)
    a, r = both(lambda o, s, c: orc.conv(st, lp, proj, o, s, lw, c), lambda o, s, c: wr.conv(st, lp, proj, o, s, lw, c),
                out, cs, ck)
    for i, what in enumerate(("conv out", "conv state", "conv ckpt")):
        same(a[i], r[i], what, live=i < 2 or ckpt > 0)


@pytest.mark.parametrize("m,n_k,n_v,ckpt", [(1, 2, 4, 0), (4, 2, 4, 3), (3, 1, 4, 0), (6, 4, 4, 6)])
def test_delta(orc, m, n_k, n_v, ckpt):
    rng = np.random.default_rng(9 + m + n_k)
    lp, proj, lw, cd = lin_setup(rng, m, n_k, n_v)
    conv_out = rng.standard_normal((m, cd)).astype(np.float32)
    S = (0.1 * rng.standard_normal((n_v, 128, 128))).astype(np.float32)
    out = np.zeros((m, n_v * 128), np.float32)
    ck = np.zeros_like(S)
    st = StepU(m, 0, 1, ckpt)
    a, r = both(lambda s, o, c: orc.delta(st, lp, proj, conv_out, s, lw, o, c),
                lambda s, o, c: wr.delta(st, lp, proj, conv_out, s, lw, o, c), S, out, ck)
    for i, what in enumerate(("delta state", "delta out", "delta ckpt")):
        same(a[i], r[i], what, live=i < 2 or ckpt > 0)


# ---- vision.wgsl ----------------------------------------------------------------------


def test_vis_layer_norm(orc):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((9, 300)).astype(np.float32)
    w = np.concatenate([1 + 0.1 * rng.standard_normal(300), 0.1 * rng.standard_normal(300)]).astype(np.float32)
    p = VisP(9, 300, 0, 0, 1e-6, 0, 0, 0)
    same(orc.vis_layer_norm(p, a, w), wr.vis_layer_norm(p, a, w), "vision layer_norm")


@pytest.mark.parametrize("mode,act", [(0, 0), (0, 1), (0, 2), (1, 0), (2, 0)])
def test_vis_epilogue(orc, mode, act):
    rng = np.random.default_rng(mode * 3 + act)
    a = (2 * rng.standard_normal((9, 300))).astype(np.float32)
    b = rng.standard_normal((9, 300)).astype(np.float32)
    e = rng.standard_normal((9, 300)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(300)).astype(np.float32)
    p = VisP(9, 300, mode, act, 0, 0, 0, 0)
    ea = None if mode != 2 else e
    x, y = both(lambda a_, b_: orc.vis_epilogue(p, a_, None if mode == 0 else b_, bias, ea),
                lambda a_, b_: wr.vis_epilogue(p, a_, None if mode == 0 else b_, bias, ea), a, b)
    same(x[0], y[0], "vision epilogue a")
    same(x[1], y[1], "vision epilogue b")


@pytest.mark.parametrize("n,grid_w,heads", [(16, 4, 2), (48, 8, 3)])
def test_vis_rope_attend(orc, n, grid_w, heads):
    rng = np.random.default_rng(n + heads)
    qkv = rng.standard_normal((n, 3 * heads * 72)).astype(np.float32)
    p = VisP(n, 0, 0, 0, 0, grid_w, heads, 0)
    a, r = both(lambda q: orc.vis_rope(p, q), lambda q: wr.vis_rope(p, q), qkv)
    same(a[0], r[0], "vision rope")
    same(orc.vis_attend(p, a[0]), wr.vis_attend(p, r[0]), "vision attend")
