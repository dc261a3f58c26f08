"""The oracle's restatement of the vision tower (vision.wgsl, Vision::encode) against an
independent numpy statement of the same mathematics, on the CPU: LayerNorm, the
bias/GELU/residual epilogue, 2D RoPE in merge order, bidirectional attention, and the
whole encode (position interpolation, blocks, 2x2 merger) in float64."""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle as orc
from sensenova_b200.ffi import VisP
from sensenova_b200.vision import small_vision

HD = 72


def np_layer_norm(a, w):
    a = a.astype(np.float64)
    cols = a.shape[1]
    mean = a.mean(axis=1, keepdims=True)
    var = ((a - mean) ** 2).mean(axis=1, keepdims=True)
    return (a - mean) / np.sqrt(var + 1e-6) * w[:cols] + w[cols:]


def np_gelu_tanh(x):
    u = np.clip(0.7978845608 * (x + 0.044715 * x ** 3), -15, 15)
    return 0.5 * x * (1 + np.tanh(u))


def np_gelu_erf(x):
    return 0.5 * x * (1 + np.vectorize(math.erf)(x / math.sqrt(2)))


def merge_rc(t, grid_w):
    blk, intra = t // 4, t % 4
    mw = grid_w // 2
    return (blk // mw) * 2 + intra // 2, (blk % mw) * 2 + intra % 2


def np_rope(qkv, heads, grid_w):
    out = qkv.astype(np.float64).copy()
    hidden = heads * HD
    for t in range(qkv.shape[0]):
        r, c = merge_rc(t, grid_w)
        for j in range(36):
            fi = j % 18
            pos = c if j >= 18 else r
            ang = pos * 10000.0 ** (-(2 * fi) / 36)
            cs, sn = math.cos(ang), math.sin(ang)
            for part in range(2):
                for h in range(heads):
                    b = part * hidden + h * HD
                    x1, x2 = out[t, b + j], out[t, b + j + 36]
                    out[t, b + j], out[t, b + j + 36] = x1 * cs - x2 * sn, x2 * cs + x1 * sn
    return out


def np_attend(qkv, heads):
    n = qkv.shape[0]
    hidden = heads * HD
    q = qkv[:, :hidden].reshape(n, heads, HD).astype(np.float64)
    k = qkv[:, hidden:2 * hidden].reshape(n, heads, HD).astype(np.float64)
    v = qkv[:, 2 * hidden:].reshape(n, heads, HD).astype(np.float64)
    s = np.einsum("qhd,khd->hqk", q, k) / math.sqrt(HD)
    p = np.exp(s - s.max(axis=2, keepdims=True))
    p /= p.sum(axis=2, keepdims=True)
    return np.einsum("hqk,khd->qhd", p, v).reshape(n, hidden)


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def test_layer_norm_and_epilogue():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((9, 300)).astype(np.float32) * 3 + 1
    w = rng.standard_normal(600).astype(np.float32)
    assert rel(orc.vis_layer_norm(VisP(9, 300, 0, 0, 1e-6, 0, 0, 0), a, w), np_layer_norm(a, w)) < 1e-5
    bias = rng.standard_normal(300).astype(np.float32)
    for act, f in ((0, lambda x: x), (1, np_gelu_tanh), (2, np_gelu_erf)):
        x = a.copy()
        orc.vis_epilogue(VisP(9, 300, 0, act, 0, 0, 0, 0), x, None, bias)
        assert np.abs(x - f(a.astype(np.float64) + bias)).max() < 2e-6
    b = rng.standard_normal(a.shape).astype(np.float32)
    b1 = b.copy()
    orc.vis_epilogue(VisP(9, 300, 1, 0, 0, 0, 0, 0), a.copy(), b1, bias)
    assert np.abs(b1 - (b + a + bias)).max() < 1e-5
    e = rng.standard_normal(a.shape).astype(np.float32)
    b2 = b.copy()
    orc.vis_epilogue(VisP(9, 300, 2, 0, 0, 0, 0, 0), a.copy(), b2, bias, e)
    assert np.abs(b2 - (a + bias + e)).max() < 1e-5


@pytest.mark.parametrize("n,grid_w", [(8, 4), (24, 6), (36, 12)])
def test_rope_and_attend(n, grid_w):
    rng = np.random.default_rng(n)
    heads = 2
    qkv = rng.standard_normal((n, 3 * heads * HD)).astype(np.float32)
    p = VisP(n, 0, 0, 0, 0, grid_w, heads, 0)
    r = qkv.copy()
    orc.vis_rope(p, r)
    assert np.abs(r - np_rope(qkv, heads, grid_w)).max() < 1e-5
    assert rel(orc.vis_attend(p, r), np_attend(r, heads)) < 1e-5


def np_encode(ov, cfg, patches, frames, h, w):
    """Vision::encode (vision.rs:176-311) in float64 numpy with the oracle's weights."""
    def mat(name):
        dt, q, s, rows, cols = ov.tensor(name)
        return (q.astype(np.float64).reshape(rows, cols // 32, 32) * s.reshape(rows, cols // 32, 1)).reshape(rows, cols)

    def vec(name):
        return ov.tensor(name)[1].astype(np.float64)

    hid, n = cfg.hidden, h * w
    side = cfg.pos_side
    table = vec("v.pos").reshape(side * side, hid)
    lin = lambda m: np.array([0.0] if m == 1 else [(side - 1) * i / (m - 1) for i in range(m)])
    hs, ws = lin(h), lin(w)
    pos = np.zeros((n, hid))
    for t in range(n):
        r, c = merge_rc(t, w)
        fh, fw = int(hs[r]), int(ws[c])
        ch, cw = min(fh + 1, side - 1), min(fw + 1, side - 1)
        dh, dw = hs[r] - fh, ws[c] - fw
        pos[t] = (table[fh * side + fw] * (1 - dh) * (1 - dw) + table[fh * side + cw] * (1 - dh) * dw
                  + table[ch * side + fw] * dh * (1 - dw) + table[ch * side + cw] * dh * dw)
    outs = []
    for f in range(frames):
        x = patches[f].astype(np.float64) @ mat("v.patch").T + vec("v.patch_b") + pos
        for i in range(cfg.depth):
            b = f"v{i}."
            xn = np_layer_norm(x, vec(b + "n1"))
            qkv = xn @ mat(b + "qkv").T + vec(b + "qkv_b")
            qkv = np_rope(qkv, cfg.n_heads, w)
            x = x + np_attend(qkv, cfg.n_heads) @ mat(b + "proj").T + vec(b + "proj_b")
            xn = np_layer_norm(x, vec(b + "n2"))
            m = np_gelu_tanh(xn @ mat(b + "fc1").T + vec(b + "fc1_b"))
            x = x + m @ mat(b + "fc2").T + vec(b + "fc2_b")
        xn = np_layer_norm(x, vec("vm.norm")).reshape(n // 4, 4 * hid)
        m = np_gelu_erf(xn @ mat("vm.fc1").T + vec("vm.fc1_b"))
        outs.append(m @ mat("vm.fc2").T + vec("vm.fc2_b"))
    return np.concatenate(outs)


def test_encode_matches_numpy_statement():
    cfg = small_vision()
    ov = orc.OracleVision(cfg, seed=3)
    h, w, frames = 4, 6, 2
    rng = np.random.default_rng(1)
    patches = rng.standard_normal((frames, h * w, cfg.patch_dim())).astype(np.float32)
    got = ov.encode(patches, frames, h, w)
    want = np_encode(ov, cfg, patches, frames, h, w)
    assert got.shape == (frames * h * w // 4, cfg.out_hidden)
    assert rel(got, want) < 1e-4, rel(got, want)
    ov.close()
