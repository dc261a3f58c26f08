"""The CPU oracle against independent float64 numpy statements of the same math,
plus known-answer tests of the Q8_0 / Q4_0 element mapping (bit-exact).

The reference ships no golden vectors for this path (its tests cover only media
preprocessing and chat parsing), so these checks pin the restatement to the
formulas of the WGSL sources it cites.
"""
import numpy as np
import pytest

from sensenova_b200.ffi import AttnP, LayerP, LinP, MatP, StepU, SNL_Q4_0, SNL_Q8_0


def mat_p(n, k, x_stride=None, y_stride=None, x_off=0, m_one=0):
    return MatP(n, k, x_off, x_stride if x_stride is not None else k, 0, y_stride if y_stride is not None else n, 0, m_one)


def dequant(q_bytes: np.ndarray, s: np.ndarray, dtype: int, rows: int, cols: int) -> np.ndarray:
    """Element values (weights.rs:123-162, matmul.wgsl:41-55) in float64."""
    if dtype == SNL_Q8_0:
        v = q_bytes.view(np.int8).astype(np.float64).reshape(rows, cols)
    else:
        w = q_bytes.view(np.uint32).reshape(rows, cols // 8)
        nib = (w[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15
        v = nib.reshape(rows, cols).astype(np.float64) - 8.0
    return v * np.repeat(s.astype(np.float64).reshape(rows, cols // 32), 32, axis=1)


# ---- known answers: every code, every scale edge, bit-exact --------------------------


def test_q8_every_code_bit_exact(orc):
    # 256 codes in 8 blocks of 32; one-hot x picks element j exactly.
    codes = np.arange(-128, 128, dtype=np.int8)
    scales = np.array([1.0, 2.0 ** -24, 65504.0, 0.5, 3.0e-5, 1.0 / 127, 7.62939453125e-06, 0.001], dtype=np.float32)
    rows, k = 1, 256
    q = codes.view(np.uint8).copy()
    for j in range(0, k, 37):
        x = np.zeros(k, dtype=np.float32)
        x[j] = 1.0
        y = np.zeros(1, dtype=np.float32)
        orc.mat(SNL_Q8_0, StepU(1, 0, 1, 0), mat_p(rows, k), x, q, scales, y)
        assert y[0] == np.float32(codes[j]) * scales[j // 32]


def test_q8_dequant_row_all_codes(orc):
    codes = np.arange(-128, 128, dtype=np.int8)
    for s in (1.0, 0.0123, 2.0 ** -20):
        sc = np.full(8, s, dtype=np.float32)
        out = orc.dequant_q8_row(codes, sc)
        assert np.array_equal(out, codes.astype(np.float32) * np.float32(s))


def test_q4_nibble_order_one_hot(orc):
    # nibble i of little-endian word w is element 8w+i, stored as value+8 (weights.rs:135-153)
    k = 32
    x = (np.arange(k, dtype=np.float32) + 1.0) * 0.25
    s = np.array([0.5], dtype=np.float32)
    for e in range(k):
        words = np.full(4, 0x88888888, dtype=np.uint32)
        w, i = divmod(e, 8)
        words[w] = (words[w] & ~np.uint32(0xF << (4 * i))) | np.uint32(15 << (4 * i))
        y = np.zeros(1, dtype=np.float32)
        orc.mat(SNL_Q4_0, StepU(1, 0, 1, 0), mat_p(1, k), x, words.view(np.uint8), s, y)
        assert y[0] == np.float32(7.0) * s[0] * x[e], e


def test_q4_every_nibble(orc):
    k = 32
    for n in range(16):
        words = np.zeros(4, dtype=np.uint32)
        words[0] = n  # element 0 holds nibble n, the rest 0 (value -8)
        x = np.zeros(k, dtype=np.float32)
        x[0] = 1.0
        y = np.zeros(1, dtype=np.float32)
        orc.mat(SNL_Q4_0, StepU(1, 0, 1, 0), mat_p(1, k), x, words.view(np.uint8), np.array([0.25], np.float32), y)
        assert y[0] == np.float32(n - 8) * np.float32(0.25)


# ---- matrix kernels vs float64 ---------------------------------------------------------


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 40])
def test_mat_vs_float64(orc, dtype, m):
    rng = np.random.default_rng(m * 10 + dtype)
    n, k = 96, 1024
    q, s = orc.gen_quant(7, f"w{dtype}", dtype, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = np.full((m, n), np.nan, dtype=np.float32)
    orc.mat(dtype, StepU(m, 0, 1, 0), mat_p(n, k), x, q, s, y)
    ref = x.astype(np.float64) @ dequant(q, s, dtype, n, k).T
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 2e-6, err


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m,n,k", [(1, 67, 4096), (2, 40, 96), (3, 33, 1056), (8, 24, 800), (9, 37, 288),
                                   (17, 19, 512), (40, 21, 320)])
def test_mat_vector_forms_bit_identical(orc, dtype, m, n, k):
    """The AVX2 forms of the oracle's matvec/matmul give the scalar statements' bits:
    block counts that are not multiples of 8 or 32 (partial lane groups), token counts
    with a ragged last group of 8, strided x/y with offsets."""
    rng = np.random.default_rng(m * 1000 + k + dtype)
    q, s = orc.gen_quant(11, f"v{dtype}", dtype, n, k)
    xs = k + 5
    x = rng.standard_normal(3 + m * xs).astype(np.float32)
    p = MatP(n, k, 3, xs, 2, n + 4, 1, 0)
    ys = []
    for vec in (False, True):
        y = np.full(2 + m * (n + 4), np.nan, dtype=np.float32)
        orc.set_vector(vec)
        try:
            orc.mat(dtype, StepU(m, 0, 1, 0), p, x, q, s, y)
        finally:
            orc.set_vector(True)
        ys.append(y)
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))


def test_mat_offsets_and_m_one(orc):
    # The head's use of MatP (engine.rs:835-842): x_off picks the last rows, m_one fixes the count.
    rng = np.random.default_rng(3)
    n, k, h = 40, 256, 256
    q, s = orc.gen_quant(1, "head", SNL_Q8_0, n, k)
    hid = rng.standard_normal((6, h)).astype(np.float32)
    y = np.zeros((2, n), dtype=np.float32)
    orc.mat(SNL_Q8_0, StepU(5, 0, 1, 0), MatP(n, k, 4 * h, h, 0, n, 0, 2), hid, q, s, y)
    ref = hid[4:6].astype(np.float64) @ dequant(q, s, SNL_Q8_0, n, k).T
    assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-6


# ---- layers.wgsl --------------------------------------------------------------------------


def layer_p(h, mode=0, last_row=0, eps=1e-6, weight_one=1.0, iterations=20, inter=0, x_stride=0):
    return LayerP(h, mode, last_row, eps, weight_one, iterations, inter, x_stride)


@pytest.mark.parametrize("mode", [0, 1])
def test_branch_norm(orc, mode):
    rng = np.random.default_rng(mode)
    m, h = 5, 512
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0.1, 1.0, (m, 8)).astype(np.float32)
    w = (0.1 * rng.standard_normal(h)).astype(np.float32)
    out = np.zeros((m, h), dtype=np.float32)
    orc.branch_norm(StepU(m, 0, 1, 0), layer_p(h, mode), x, coef, w, out, m)
    xd = x.astype(np.float64)
    v = xd[:, :h] if mode == 0 else coef[:, :1] * xd[:, :h] + coef[:, 1:2] * xd[:, h:]
    ref = v / np.sqrt((v * v).mean(1, keepdims=True) + 1e-6) * (1.0 + w)
    assert np.abs(out - ref).max() < 1e-5


def test_branch_norm_last_row_and_stride(orc):
    rng = np.random.default_rng(5)
    m, h = 4, 256
    x = rng.standard_normal((m, h)).astype(np.float32)
    w = np.zeros(h, dtype=np.float32)
    out = np.zeros(h, dtype=np.float32)
    orc.branch_norm(StepU(m, 0, 1, 0), layer_p(h, 0, last_row=1, x_stride=h), x, None, w, out, 1)
    v = x[-1].astype(np.float64)
    assert np.abs(out - v / np.sqrt((v * v).mean() + 1e-6)).max() < 1e-5


def sinkhorn_ref(lg, iters):
    a, b, c, e = lg[4:8].astype(np.float64)
    lse = lambda u, v: max(u, v) + np.log(np.exp(u - max(u, v)) + np.exp(v - max(u, v)))
    for _ in range(iters):
        r0, r1 = lse(a, b), lse(c, e)
        a, b, c, e = a - r0, b - r0, c - r1, e - r1
        c0, c1 = lse(a, c), lse(b, e)
        a, c, b, e = a - c0, c - c0, b - c1, e - c1
    sig = lambda z: 1 / (1 + np.exp(-z))
    return np.array([sig(lg[0]), sig(lg[1]), 2 * sig(lg[2]), 2 * sig(lg[3]), np.exp(a), np.exp(b), np.exp(c), np.exp(e)])


def test_mhc_router(orc):
    rng = np.random.default_rng(11)
    m, h = 3, 256
    d = 2 * h
    x = rng.standard_normal((m, d)).astype(np.float32)
    w = np.concatenate([0.02 * rng.standard_normal(8 * d), 0.1 * rng.standard_normal(8)]).astype(np.float32)
    raw = np.zeros((m, 9), dtype=np.float32)
    coef = np.zeros((m, 8), dtype=np.float32)
    st, p = StepU(m, 0, 1, 0), layer_p(h, iterations=20)
    orc.mhc_dots(st, p, x, w, raw)
    orc.mhc_finish(st, p, raw, w, coef)
    W = w[: 8 * d].astype(np.float64).reshape(8, d)
    for r in range(m):
        xd = x[r].astype(np.float64)
        dots = W @ xd
        assert np.abs(raw[r, :8] - dots).max() < 1e-4
        rinv = 1 / np.sqrt((xd * xd).sum() / d + 1e-6)
        lg = dots * rinv + w[8 * d:]
        ref = sinkhorn_ref(lg, 20)
        assert np.abs(coef[r] - ref).max() < 1e-4
        # doubly stochastic mixing after Sinkhorn
        mix = coef[r, 4:].reshape(2, 2)
        assert np.allclose(mix.sum(0), 1, atol=1e-4) and np.allclose(mix.sum(1), 1, atol=1e-4)


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_merge(orc, mode):
    rng = np.random.default_rng(mode)
    m, h = 3, 64
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0, 1, (m, 8)).astype(np.float32)
    br = rng.standard_normal((m, h)).astype(np.float32)
    x0 = x.astype(np.float64).copy()
    orc.merge(StepU(m, 0, 1, 0), layer_p(h, mode), x, coef, br)
    a, b = x0[:, :h], x0[:, h:]
    c = coef.astype(np.float64)
    if mode == 0:
        ref = np.concatenate([a + br, b], 1)
    elif mode == 3:
        ref = np.concatenate([a, a], 1)
    else:
        n0 = c[:, 4:5] * a + c[:, 5:6] * b + c[:, 2:3] * br
        n1 = c[:, 6:7] * a + c[:, 7:8] * b + c[:, 3:4] * br
        ref = np.concatenate([0.5 * (n0 + n1), b], 1) if mode == 2 else np.concatenate([n0, n1], 1)
    assert np.abs(x - ref).max() < 1e-5


def test_swiglu(orc):
    rng = np.random.default_rng(2)
    m, inter = 3, 96
    gu = rng.standard_normal((m, 2 * inter)).astype(np.float32)
    act = np.zeros((m, inter), dtype=np.float32)
    orc.swiglu(StepU(m, 0, 1, 0), layer_p(64, inter=inter), gu, act)
    g, u = gu[:, :inter].astype(np.float64), gu[:, inter:]
    assert np.abs(act - g / (1 + np.exp(-g)) * u).max() < 1e-5


def test_argmax_first_max(orc):
    v = np.array([1.0, 3.0, -2.0, 3.0, 0.5], dtype=np.float32)
    assert orc.argmax(v) == 1
    v = np.array([np.nan, 1.0, 2.0], dtype=np.float32)
    assert orc.argmax(v) == 0  # sampler.rs:169-177 keeps index 0 when v[0] is NaN


# ---- attention.wgsl --------------------------------------------------------------------


def attn_setup(rng, m, pos0, n_kv=1, rot=64, ctx=64):
    nh = 4 * n_kv
    HD = 256
    q_dim, kv_dim = nh * HD, n_kv * HD
    stride = 2 * q_dim + 2 * kv_dim
    p = AttnP(nh, n_kv, rot, stride, 1e7, 1e-6, 1 / 16, (33 << 16) | 30)
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    norms = (0.1 * rng.standard_normal(2 * HD)).astype(np.float32)
    kc = np.zeros(ctx * kv_dim // 2, dtype=np.uint32)
    vc = np.zeros_like(kc)
    # earlier cache entries: random f16 pairs
    pre = (rng.standard_normal(pos0 * kv_dim).astype(np.float16)).view(np.uint32)
    kc[: pre.size] = pre
    vc[: pre.size] = (rng.standard_normal(pos0 * kv_dim).astype(np.float16)).view(np.uint32)
    rpos = np.repeat(np.arange(pos0, pos0 + m, dtype=np.uint32)[:, None], 4, 1).copy()
    return p, proj, norms, kc, vc, rpos


def rope_ref(v, pos, rot, theta):
    v = v.copy()
    half = rot // 2
    fi = np.arange(rot) % half
    ang = pos * theta ** (-(2.0 * fi) / rot)
    sh = v.copy()
    out = v.copy()
    out[:half] = sh[:half] * np.cos(ang[:half]) - sh[half:rot] * np.sin(ang[:half])
    out[half:rot] = sh[half:rot] * np.cos(ang[half:]) + sh[:half] * np.sin(ang[half:])
    return out


def test_attn_prep(orc):
    rng = np.random.default_rng(4)
    m, pos0 = 3, 5
    p, proj, norms, kc, vc, rpos = attn_setup(rng, m, pos0)
    qbuf = np.zeros((m, p.n_heads * 256), dtype=np.float32)
    orc.attn_prep(StepU(m, pos0, 1, 0), p, proj, qbuf, kc, vc, norms, rpos)
    kv_dim = p.n_kv * 256
    for r in range(m):
        for h in range(p.n_heads):
            v = proj[r, h * 512: h * 512 + 256].astype(np.float64)
            v = v / np.sqrt((v * v).mean() + 1e-6) * (1 + norms[:256])
            ref = rope_ref(v, pos0 + r, 64, 1e7)
            assert np.abs(qbuf[r, h * 256:(h + 1) * 256] - ref).max() < 2e-4
        k = proj[r, 2 * 1024: 2 * 1024 + 256].astype(np.float64)
        k = rope_ref(k / np.sqrt((k * k).mean() + 1e-6) * (1 + norms[256:]), pos0 + r, 64, 1e7)
        got = kc[(pos0 + r) * kv_dim // 2:(pos0 + r + 1) * kv_dim // 2].view(np.float16).astype(np.float64)
        assert np.abs(got - k).max() < 4e-3
        vv = proj[r, 2 * 1024 + 256: 2 * 1024 + 512]
        gotv = vc[(pos0 + r) * kv_dim // 2:(pos0 + r + 1) * kv_dim // 2].view(np.float16)
        assert np.array_equal(gotv, vv.astype(np.float16))


def attend_ref(qrow, K, V, gate, scale):
    s = (K @ qrow) * scale
    p = np.exp(s - s.max())
    o = (p[:, None] * V).sum(0) / p.sum()
    return o / (1 + np.exp(-gate))


@pytest.mark.parametrize("parts", [1, 3])
def test_attend_and_combine(orc, parts):
    rng = np.random.default_rng(parts)
    m, pos0, n_kv = 2, 37, 2
    p, proj, norms, kc, vc, rpos = attn_setup(rng, m, pos0, n_kv=n_kv)
    st = StepU(m, pos0, parts, 0)
    qbuf = rng.standard_normal((m, p.n_heads * 256)).astype(np.float32)
    # write this step's keys/values too
    kv_dim = n_kv * 256
    for r in range(m):
        base = (pos0 + r) * kv_dim // 2
        kc[base: base + kv_dim // 2] = rng.standard_normal(kv_dim).astype(np.float16).view(np.uint32)
        vc[base: base + kv_dim // 2] = rng.standard_normal(kv_dim).astype(np.float16).view(np.uint32)
    out = np.zeros((m, p.n_heads * 256), dtype=np.float32)
    partial = np.zeros(((m * p.n_heads) * parts, 258), dtype=np.float32)
    orc.attend(st, p, proj, qbuf, kc, vc, out, partial)
    if parts > 1:
        orc.attn_combine(st, p, proj, partial, out)
    K = kc.view(np.float16).astype(np.float64).reshape(-1, kv_dim)
    V = vc.view(np.float16).astype(np.float64).reshape(-1, kv_dim)
    for r in range(m):
        tot = pos0 + r + 1
        for h in range(p.n_heads):
            kh = h // 4
            gate = proj[r, h * 512 + 256: h * 512 + 512].astype(np.float64)
            ref = attend_ref(qbuf[r, h * 256:(h + 1) * 256].astype(np.float64), K[:tot, kh * 256:(kh + 1) * 256],
                             V[:tot, kh * 256:(kh + 1) * 256], gate, 1 / 16)
            assert np.abs(out[r, h * 256:(h + 1) * 256] - ref).max() < 2e-5


# ---- linear.wgsl ----------------------------------------------------------------------


def lin_setup(rng, m, n_k=2, n_v=4):
    cd = 2 * n_k * 128 + n_v * 128
    stride = cd + n_v * 128 + 2 * n_v
    lp = LinP(cd, stride, n_k, n_v, 1e-6, (0, 0, 0))
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    lw = np.concatenate([0.5 * rng.standard_normal(cd * 4), 0.1 * rng.standard_normal(n_v),
                         0.1 * rng.standard_normal(n_v), 1 + 0.1 * rng.standard_normal(128)]).astype(np.float32)
    return lp, proj, lw, cd


def test_conv_and_ckpt(orc):
    rng = np.random.default_rng(8)
    m = 5
    lp, proj, lw, cd = lin_setup(rng, m)
    cs = rng.standard_normal((3, cd)).astype(np.float32)
    cs0 = cs.astype(np.float64).copy()
    out = np.zeros((m, cd), dtype=np.float32)
    ck = np.zeros((3, cd), dtype=np.float32)
    orc.conv(StepU(m, 0, 1, 2), lp, proj, out, cs, lw, ck)
    W = lw[: cd * 4].astype(np.float64).reshape(cd, 4)
    seq = np.concatenate([cs0, proj[:, :cd].astype(np.float64)], 0)  # [3+m, cd]
    for t in range(m):
        o = (W.T * seq[t: t + 4]).sum(0)
        assert np.abs(out[t] - o / (1 + np.exp(-o))).max() < 1e-5
    assert np.abs(cs - seq[m: m + 3]).max() == 0
    assert np.abs(ck - seq[2: 5]).max() == 0  # state after token ckpt-1 = 1


def delta_ref(proj, conv_out, S, lw, n_k, n_v, cd, eps):
    m = conv_out.shape[0]
    S = S.astype(np.float64).copy()
    key_dim = n_k * 128
    out = np.zeros((m, n_v * 128))
    for t in range(m):
        for h in range(n_v):
            kh = h // (n_v // n_k)
            q = conv_out[t, kh * 128:(kh + 1) * 128].astype(np.float64)
            k = conv_out[t, key_dim + kh * 128: key_dim + (kh + 1) * 128].astype(np.float64)
            v = conv_out[t, 2 * key_dim + h * 128: 2 * key_dim + (h + 1) * 128].astype(np.float64)
            q = q / np.sqrt((q * q).sum() + 1e-6) / np.sqrt(128)
            k = k / np.sqrt((k * k).sum() + 1e-6)
            beta = 1 / (1 + np.exp(-proj[t, cd + n_v * 128 + h]))
            a = proj[t, cd + n_v * 128 + n_v + h] + lw[cd * 4 + n_v + h]
            sp = a if a > 20 else np.log1p(np.exp(a))
            g = np.exp(-np.exp(lw[cd * 4 + h]) * sp)
            Sh = S[h] * g
            dl = (v - Sh.T @ k) * beta
            Sh = Sh + np.outer(k, dl)
            S[h] = Sh
            o = Sh.T @ q
            z = proj[t, cd + h * 128: cd + (h + 1) * 128].astype(np.float64)
            out[t, h * 128:(h + 1) * 128] = o / np.sqrt((o * o).mean() + eps) * lw[cd * 4 + 2 * n_v:] * z / (1 + np.exp(-z))
    return out, S


def test_delta_and_ckpt(orc):
    rng = np.random.default_rng(9)
    m, n_k, n_v = 4, 2, 4
    lp, proj, lw, cd = lin_setup(rng, m, n_k, n_v)
    conv_out = rng.standard_normal((m, cd)).astype(np.float32)
    S = (0.1 * rng.standard_normal((n_v, 128, 128))).astype(np.float32)
    S0 = S.copy()
    out = np.zeros((m, n_v * 128), dtype=np.float32)
    ck = np.zeros_like(S)
    orc.delta(StepU(m, 0, 1, 1), lp, proj, conv_out, S, lw, out, ck)
    ref, Sref = delta_ref(proj, conv_out, S0, lw, n_k, n_v, cd, 1e-6)
    assert np.abs(out - ref).max() / np.abs(ref).max() < 2e-5
    assert np.abs(S - Sref).max() < 1e-5
    _, S1 = delta_ref(proj[:1], conv_out[:1], S0, lw, n_k, n_v, cd, 1e-6)
    assert np.abs(ck - S1).max() < 1e-5
