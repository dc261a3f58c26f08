"""The reference's own WGSL kernels on the host cores - TEST INFRASTRUCTURE ONLY.

oracle/wgsl2cpp.py translates the reference's shader sources (read from the reference
tree at build time) into oracle/_ref/libwgslref.so. This module binds buffers to those
translated kernels and dispatches them with the workgroup grids the reference's engine
uses (src/engine.rs:964-1024 `record`, src/gpu.rs:191-218 `MatKind`), so a test can run
the reference's kernel and the oracle restatement on the same inputs.

Used only by tests/ and tests/golden/make_golden.py; available only where the reference
tree exists (this container), never on the GPU box.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))
import wgsl2cpp  # noqa: E402

_lib = None


def available() -> bool:
    return (wgsl2cpp.DEFAULT_REF / "src" / "shaders").is_dir()


def load(path, modules) -> C.CDLL:
    """A library of translated modules (wgsl2cpp.compile_modules) with its dispatchers typed."""
    L = C.CDLL(str(path))
    for m in modules:
        f = getattr(L, f"wr_{m}_dispatch")
        f.restype = C.c_int64
        f.argtypes = [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.POINTER(C.c_int),
                      C.POINTER(C.c_void_p), C.POINTER(C.c_uint64)]
    return L


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = wgsl2cpp.build()
        if path is None:
            raise FileNotFoundError("reference tree absent: the reference shaders cannot be built")
        _lib = load(path, wgsl2cpp.MODULES)
    return _lib


def dispatch(module: str, entry: str, grid: tuple[int, int, int], bindings: dict, library: C.CDLL | None = None) -> None:
    """Run one entry point over grid; bindings maps binding index -> numpy array (storage,
    bound over its whole extent) or ctypes struct (uniform). Raises on an out-of-bounds
    access or a binding the module does not have. library: the reference's modules unless
    given."""
    keep, ids, ptrs, sizes = [], [], [], []
    for b, v in sorted(bindings.items()):
        if isinstance(v, np.ndarray):
            if not v.flags.c_contiguous:
                raise ValueError(f"binding {b}: not contiguous")
            ptrs.append(v.ctypes.data)
            sizes.append(v.nbytes)
        else:
            keep.append(v)
            ptrs.append(C.addressof(v))
            sizes.append(C.sizeof(v))
        ids.append(b)
        keep.append(v)
    n = len(ids)
    rc = getattr(library if library is not None else lib(), f"wr_{module}_dispatch")(
        entry.encode(), *[int(g) for g in grid], n, (C.c_int * n)(*ids), (C.c_void_p * n)(*ptrs),
        (C.c_uint64 * n)(*sizes))
    if rc == -1:
        raise ValueError(f"{module}: no entry point {entry}")
    if rc < -1:
        raise ValueError(f"{module}.{entry}: binding {ids[-2 - rc]} rejected")
    if rc > 0:
        raise IndexError(f"{module}.{entry}: {rc} out-of-bounds accesses")


def _split(n: int) -> tuple[int, int, int]:
    # engine.rs:965 `split`
    return (n, 1, 1) if n <= 65535 else (65535, -(-n // 65535), 1)


def _vec4_view(a: np.ndarray) -> np.ndarray:
    """An f32/u32 buffer padded to whole vec4s (storage arrays of vec4 are read 16 B at a time)."""
    flat = np.ascontiguousarray(a).reshape(-1)
    pad = (-flat.size) % 4
    return np.concatenate([flat, np.zeros(pad, flat.dtype)]) if pad else flat


# ---- matmul.wgsl (matvec / matvec1 / matvec2 / matmul, Q8_0 and Q4_0 splices) ----

def mat(dtype: int, step, p, x: np.ndarray, wq: np.ndarray, ws: np.ndarray, y: np.ndarray) -> None:
    """y as the reference computes it: MatKind::for_rows picks the entry point
    (gpu.rs:211-218), engine.rs:973-982 the grid. dtype 1 = Q8_0, 2 = Q4_0 (snl_b200.h)."""
    m = p.m_one if p.m_one else step.m
    module = "matmul_q8" if dtype == 1 else "matmul_q4"
    if m == 1:
        entry, grid = "matvec1", _split(-(-p.n // 32))
    elif m == 2:
        entry, grid = "matvec2", _split(-(-p.n // 32))
    elif m <= 8:
        entry, grid = "matvec", _split(-(-p.n // 8))
    else:
        entry, grid = "matmul", (-(-p.n // 128), -(-m // 128), 1)
    xv = _vec4_view(np.asarray(x, np.float32))
    wv = _vec4_view(np.asarray(wq).view(np.uint32))
    dispatch(module, entry, grid, {0: step, 1: p, 2: xv, 3: wv, 4: np.ascontiguousarray(ws, np.float32), 5: y})


# ---- layers.wgsl ----

def branch_norm(step, p, x, coef, w, out, n_groups):
    dispatch("layers", "branch_norm", (n_groups, 1, 1), {0: step, 1: p, 2: x, 3: coef, 4: w, 5: out})


def mhc_dots(step, p, x, w, raw):
    dispatch("layers", "mhc_dots", (9, step.m, 1), {0: step, 1: p, 2: x, 4: w, 5: raw, 3: np.zeros(8, np.float32)})


def mhc_finish(step, p, raw, w, coef):
    dispatch("layers", "mhc_finish", _split(-(-step.m // 256)), {0: step, 1: p, 2: np.zeros(4, np.float32), 3: coef,
                                                                   4: w, 5: raw})


def merge(step, p, x, coef, br):
    dispatch("layers", "merge", _split(-(-(step.m * p.h) // 256)), {0: step, 1: p, 2: x, 3: coef,
                                                                    4: np.zeros(4, np.float32), 5: br})


def swiglu(step, p, gu, act):
    dispatch("layers", "swiglu", _split(-(-(step.m * p.inter) // 256)), {0: step, 1: p, 2: gu,
                                                                         3: np.zeros(8, np.float32),
                                                                         4: np.zeros(4, np.float32), 5: act})


# ---- attention.wgsl ----

def _attn_bind(step, p, proj, qbuf, kc, vc, norms, out, partial, rpos):
    z = np.zeros(4, np.float32)
    return {0: step, 1: p, 2: proj, 3: qbuf, 4: kc, 5: vc, 6: z if norms is None else norms,
            7: z if out is None else out, 8: z if partial is None else partial,
            9: np.zeros(4, np.uint32) if rpos is None else rpos}


def attn_prep(step, p, proj, qbuf, kc, vc, norms, rpos):
    dispatch("attention", "prep", (p.n_heads + 2 * p.n_kv, step.m, 1),
             _attn_bind(step, p, proj, qbuf, kc, vc, norms, None, None, np.ascontiguousarray(rpos, np.uint32)))


def attend(step, p, proj, qbuf, kc, vc, out, partial):
    dispatch("attention", "attend", (p.n_kv, step.m, step.parts),
             _attn_bind(step, p, proj, qbuf, kc, vc, None, out, partial, None))


def attn_combine(step, p, proj, partial, out):
    dispatch("attention", "combine", (p.n_heads, step.m, 1),
             _attn_bind(step, p, proj, np.zeros(4, np.float32), np.zeros(4, np.uint32), np.zeros(4, np.uint32),
                        None, out, partial, None))


# ---- linear.wgsl ----

def _lin_bind(step, p, proj, conv_out, conv_state, state, lw, out, conv_ckpt, state_ckpt):
    z = np.zeros(4, np.float32)
    pick = lambda a: z if a is None else a  # noqa: E731
    return {0: step, 1: p, 2: proj, 3: conv_out, 4: pick(conv_state), 5: pick(state), 6: lw, 7: pick(out),
            8: pick(conv_ckpt), 9: pick(state_ckpt)}


def conv(step, p, proj, conv_out, conv_state, lw, conv_ckpt):
    dispatch("linear", "conv", (-(-p.conv_dim // 256), 1, 1),
             _lin_bind(step, p, proj, conv_out, conv_state, None, lw, None, conv_ckpt, None))


def delta(step, p, proj, conv_out, state, lw, out, state_ckpt):
    dispatch("linear", "delta", (p.n_v, 1, 1), _lin_bind(step, p, proj, conv_out, None, state, lw, out, None, state_ckpt))


# ---- vision.wgsl (grids of vision.rs:248-268: `norm`, `epi`, rope and attend) ----

def _vis(entry, p, a, b, w, e, grid):
    z = np.zeros(4, np.float32)
    dispatch("vision", entry, grid, {0: p, 1: a, 2: z if b is None else b, 3: z if w is None else w,
                                     4: z if e is None else e})


def vis_layer_norm(p, a: np.ndarray, w: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.zeros_like(a)
    _vis("layer_norm", p, a, b, np.ascontiguousarray(w, np.float32), None, _split(p.rows))
    return b


def vis_epilogue(p, a: np.ndarray, b, w: np.ndarray, e=None) -> None:
    _vis("epilogue", p, a, b, np.ascontiguousarray(w, np.float32), e, _split(-(-(p.rows * p.cols) // 256)))


def vis_rope(p, qkv: np.ndarray) -> None:
    _vis("rope", p, qkv, None, None, None, _split(-(-(p.rows * p.heads * 36) // 256)))


def vis_attend(p, qkv: np.ndarray) -> np.ndarray:
    out = np.zeros((p.rows, p.heads * 72), np.float32)
    _vis("attend", p, np.ascontiguousarray(qkv, np.float32), out, None, None, (-(-p.rows // 64), p.heads, 1))
    return out
