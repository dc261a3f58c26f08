"""Golden-vector cases for the hot-path kernels - TEST INFRASTRUCTURE.

The fixture `reference_kernels.npz` beside this file holds the outputs of the
REFERENCE's own WGSL kernels (translated and run on the host cores by
oracle/wgslref.py) for the cases below; `make_golden.py` wrote it. Inputs are not
stored: `inputs()` regenerates them from an integer hash, so every machine rebuilds the
same bits (no dependence on a random-number library's stream).

`run(case, impl)` runs one case through any implementation with the oracle's kernel
API: oracle/wgslref.py (the reference, to make the fixture) or oracle/oracle.py (the
restatement, to check it against the fixture). The CUDA path has its own runner in
tests/test_gpu_golden.py with the same inputs.
"""
from __future__ import annotations

import hashlib

import numpy as np

from sensenova_b200.ffi import AttnP, LayerP, LinP, MatP, StepU, VisP

Q8, Q4 = 1, 2
HD = 256


def _mix(tag: str, n: int) -> np.ndarray:
    """n 64-bit splitmix64 outputs for (tag, index): deterministic on every machine."""
    seed = np.uint64(int.from_bytes(hashlib.sha256(tag.encode()).digest()[:8], "little"))
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = seed + (i + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def hashed(tag: str, n: int, scale: float = 1.0, offset: float = 0.0) -> np.ndarray:
    """n float32 values, uniform in [offset - scale, offset + scale), 24 random bits each."""
    u = (_mix(tag, n) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return ((2.0 * u - 1.0) * scale + offset).astype(np.float32)


def hashed_f16_words(tag: str, n_halves: int) -> np.ndarray:
    return hashed(tag, n_halves, 2.0).astype(np.float16).view(np.uint32).copy()


def quant(tag: str, dtype: int, n: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Q8_0 codes in [-127, 127] or Q4_0 words (any nibbles), and fp16-exact block scales."""
    if dtype == Q8:
        q = ((_mix(tag + ".q", n * k) % np.uint64(255)).astype(np.int32) - 127).astype(np.int8).view(np.uint8)
    else:
        q = (_mix(tag + ".q", n * k // 8) >> np.uint64(32)).astype(np.uint32).view(np.uint8)
    s = np.abs(hashed(tag + ".s", n * k // 32, 0.02)).astype(np.float16).astype(np.float32) / np.float32(127)
    s = s.astype(np.float16).astype(np.float32)
    return np.ascontiguousarray(q), s


# (name, kernel, shape arguments)
CASES = [
    *[(f"mat_q{8 if d == Q8 else 4}_m{m}", "mat", dict(dtype=d, m=m, n=72, k=256)) for d in (Q8, Q4)
      for m in (1, 2, 5, 20)],
    ("branch_norm_mhc", "branch_norm", dict(m=3, h=512, mode=1, last_row=0)),
    ("branch_norm_last", "branch_norm", dict(m=4, h=256, mode=0, last_row=1)),
    ("mhc", "mhc", dict(m=2, h=256)),
    *[(f"merge_mode{md}", "merge", dict(m=2, h=256, mode=md)) for md in range(4)],
    ("swiglu", "swiglu", dict(m=2, inter=512)),
    ("attn_prep", "attn_prep", dict(m=3, pos0=5, ctx=12)),
    ("attend_1part", "attend", dict(m=2, pos0=29, parts=1, ctx=32)),
    ("attend_3parts", "attend", dict(m=1, pos0=40, parts=3, ctx=44)),
    ("conv", "conv", dict(m=5, ckpt=2)),
    ("delta", "delta", dict(m=3, ckpt=2)),
    # vision.wgsl (the tower's kernels around its matrix products)
    ("vis_layer_norm", "vis_layer_norm", dict(rows=5, cols=300)),
    *[(f"vis_epilogue_mode{md}_act{ac}", "vis_epilogue", dict(rows=5, cols=300, mode=md, act=ac))
      for md, ac in ((0, 1), (0, 2), (1, 0), (2, 0))],
    ("vis_rope_attend", "vis_rope_attend", dict(n=24, grid_w=6, heads=3)),
]


def layer_p(h, mode=0, last_row=0, inter=0, x_stride=0):
    return LayerP(h, mode, last_row, 1e-6, 1.0, 20, inter, x_stride)


def lin_p():
    # one key head and two value heads of 128 (the 9B shape has 16 / 32)
    n_k, n_v = 1, 2
    cd = 2 * n_k * 128 + n_v * 128
    return LinP(cd, cd + n_v * 128 + 2 * n_v, n_k, n_v, 1e-6, (0, 0, 0))


def attn_p():
    n_kv = 1
    return AttnP(4 * n_kv, n_kv, 64, 2 * 4 * n_kv * HD + 2 * n_kv * HD, 1e7, 1e-6, 1 / 16, (33 << 16) | 30)


def inputs(name: str, kernel: str, a: dict) -> dict:
    """The case's inputs (and initial contents of its in/out buffers)."""
    t = lambda s: f"{name}.{s}"  # noqa: E731
    if kernel == "mat":
        q, s = quant(t("w"), a["dtype"], a["n"], a["k"])
        xs = a["k"] + 8
        return dict(q=q, s=s, x=hashed(t("x"), 4 + a["m"] * xs, 2.0), y=np.zeros(3 + a["m"] * (a["n"] + 5), np.float32))
    if kernel == "branch_norm":
        m, h = a["m"], a["h"]
        return dict(x=hashed(t("x"), m * 2 * h, 2.0), coef=hashed(t("c"), m * 8, 0.45, 0.55),
                    w=hashed(t("w"), h, 0.2), out=np.zeros((1 if a["last_row"] else m) * h, np.float32))
    if kernel == "mhc":
        m, d = a["m"], 2 * a["h"]
        return dict(x=hashed(t("x"), m * d, 2.0),
                    w=np.concatenate([hashed(t("w"), 8 * d, 0.04), hashed(t("b"), 8, 0.2)]),
                    raw=np.zeros(m * 9, np.float32), coef=np.zeros(m * 8, np.float32))
    if kernel == "merge":
        m, h = a["m"], a["h"]
        return dict(x=hashed(t("x"), m * 2 * h, 2.0), coef=hashed(t("c"), m * 8, 0.5, 0.5), br=hashed(t("b"), m * h, 2.0))
    if kernel == "swiglu":
        return dict(gu=hashed(t("g"), a["m"] * 2 * a["inter"], 3.0), act=np.zeros(a["m"] * a["inter"], np.float32))
    if kernel in ("attn_prep", "attend"):
        p = attn_p()
        m, pos0, ctx = a["m"], a["pos0"], a["ctx"]
        kv_dim = p.n_kv * HD
        filled = (pos0 if kernel == "attn_prep" else pos0 + m) * kv_dim
        kc = np.zeros(ctx * kv_dim // 2, np.uint32)
        vc = np.zeros_like(kc)
        kc[: filled // 2] = hashed_f16_words(t("k"), filled)
        vc[: filled // 2] = hashed_f16_words(t("v"), filled)
        d = dict(proj=hashed(t("p"), m * p.proj_stride, 2.0), kc=kc, vc=vc)
        if kernel == "attn_prep":
            d.update(norms=hashed(t("n"), 2 * HD, 0.2), qbuf=np.zeros(m * p.n_heads * HD, np.float32),
                     rpos=np.stack([np.arange(pos0, pos0 + m), np.arange(m) * 3 + 1, np.arange(m) * 5 + 2,
                                    np.zeros(m, np.int64)], 1).astype(np.uint32).reshape(-1))
        else:
            d.update(qbuf=hashed(t("q"), m * p.n_heads * HD, 2.0), out=np.zeros(m * p.n_heads * HD, np.float32),
                     partial=np.zeros(m * p.n_heads * a["parts"] * (HD + 2), np.float32))
        return d
    if kernel == "vis_layer_norm":
        r, c = a["rows"], a["cols"]
        return dict(a=hashed(t("a"), r * c, 3.0, 0.5), w=np.concatenate([hashed(t("w"), c, 0.2, 1.0), hashed(t("b"), c, 0.2)]))
    if kernel == "vis_epilogue":
        r, c = a["rows"], a["cols"]
        return dict(a=hashed(t("a"), r * c, 4.0), b=hashed(t("b"), r * c, 2.0), w=hashed(t("w"), c, 0.5),
                    e=hashed(t("e"), r * c, 2.0))
    if kernel == "vis_rope_attend":
        return dict(qkv=hashed(t("qkv"), a["n"] * 3 * a["heads"] * 72, 2.0))
    lp = lin_p()
    m = a["m"]
    lw = np.concatenate([hashed(t("cw"), lp.conv_dim * 4, 0.9), hashed(t("al"), lp.n_v, 0.2),
                         hashed(t("dt"), lp.n_v, 0.2), hashed(t("nw"), 128, 0.2, 1.0)])
    d = dict(proj=hashed(t("p"), m * lp.proj_stride, 2.0), lw=lw)
    if kernel == "conv":
        d.update(conv_out=np.zeros(m * lp.conv_dim, np.float32), conv_state=hashed(t("cs"), 3 * lp.conv_dim, 2.0),
                 conv_ckpt=np.zeros(3 * lp.conv_dim, np.float32))
    else:
        d.update(conv_out=hashed(t("co"), m * lp.conv_dim, 2.0), state=hashed(t("S"), lp.n_v * 128 * 128, 0.2),
                 out=np.zeros(m * lp.n_v * 128, np.float32), state_ckpt=np.zeros(lp.n_v * 128 * 128, np.float32))
    return d


def params(kernel: str, a: dict):
    """(step, struct) of a case."""
    if kernel == "mat":
        return StepU(a["m"], 0, 1, 0), MatP(a["n"], a["k"], 4, a["k"] + 8, 3, a["n"] + 5, 2, 0)
    if kernel == "branch_norm":
        return StepU(a["m"], 0, 1, 0), layer_p(a["h"], a["mode"], a["last_row"])
    if kernel in ("mhc", "merge"):
        return StepU(a["m"], 0, 1, 0), layer_p(a["h"], a.get("mode", 0))
    if kernel == "swiglu":
        return StepU(a["m"], 0, 1, 0), layer_p(64, inter=a["inter"])
    if kernel in ("attn_prep", "attend"):
        return StepU(a["m"], a["pos0"], a.get("parts", 1), 0), attn_p()
    if kernel == "vis_layer_norm":
        return None, VisP(a["rows"], a["cols"], 0, 0, 1e-6, 0, 0, 0)
    if kernel == "vis_epilogue":
        return None, VisP(a["rows"], a["cols"], a["mode"], a["act"], 0, 0, 0, 0)
    if kernel == "vis_rope_attend":
        return None, VisP(a["n"], 0, 0, 0, 0, a["grid_w"], a["heads"], 0)
    return StepU(a["m"], 0, 1, a["ckpt"]), lin_p()


# Outputs each case records (buffers after the call).
OUTPUTS = {"mat": ["y"], "branch_norm": ["out"], "mhc": ["raw", "coef"], "merge": ["x"], "swiglu": ["act"],
           "attn_prep": ["qbuf", "kc", "vc"], "attend": ["out", "partial"], "conv": ["conv_out", "conv_state", "conv_ckpt"],
           "delta": ["out", "state", "state_ckpt"], "vis_layer_norm": ["b"], "vis_epilogue": ["a", "b"],
           "vis_rope_attend": ["qkv", "out"]}


def run(name: str, kernel: str, a: dict, impl) -> dict:
    """Run a case through impl (a module with the oracle's kernel API); return its outputs."""
    d = inputs(name, kernel, a)
    st, p = params(kernel, a)
    if kernel == "mat":
        impl.mat(a["dtype"], st, p, d["x"], d["q"], d["s"], d["y"])
    elif kernel == "branch_norm":
        impl.branch_norm(st, p, d["x"], d["coef"], d["w"], d["out"], 1 if a["last_row"] else a["m"])
    elif kernel == "mhc":
        impl.mhc_dots(st, p, d["x"], d["w"], d["raw"])
        impl.mhc_finish(st, p, d["raw"], d["w"], d["coef"])
    elif kernel == "merge":
        impl.merge(st, p, d["x"], d["coef"], d["br"])
    elif kernel == "swiglu":
        impl.swiglu(st, p, d["gu"], d["act"])
    elif kernel == "attn_prep":
        impl.attn_prep(st, p, d["proj"], d["qbuf"], d["kc"], d["vc"], d["norms"], d["rpos"])
    elif kernel == "attend":
        impl.attend(st, p, d["proj"], d["qbuf"], d["kc"], d["vc"], d["out"], d["partial"])
        if a["parts"] > 1:
            impl.attn_combine(st, p, d["proj"], d["partial"], d["out"])
    elif kernel == "conv":
        impl.conv(st, p, d["proj"], d["conv_out"], d["conv_state"], d["lw"], d["conv_ckpt"])
    elif kernel == "delta":
        impl.delta(st, p, d["proj"], d["conv_out"], d["state"], d["lw"], d["out"], d["state_ckpt"])
    elif kernel == "vis_layer_norm":
        d["b"] = impl.vis_layer_norm(p, d["a"], d["w"])
    elif kernel == "vis_epilogue":
        impl.vis_epilogue(p, d["a"], None if a["mode"] == 0 else d["b"], d["w"], d["e"] if a["mode"] == 2 else None)
    elif kernel == "vis_rope_attend":
        impl.vis_rope(p, d["qkv"])
        d["out"] = impl.vis_attend(p, d["qkv"])
    return {k: d[k] for k in OUTPUTS[kernel]}
