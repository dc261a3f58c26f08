"""ctypes wrapper of the CPU oracle (oracle/oracle.cpp) - TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference
arm as the checker; never by the product path. Arrays are numpy, host memory.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "sense-nova-server_b200"))
from sensenova_b200.ffi import (AttnP, LayerP, LinP, MatP, ModelConfigC, SampleP, StepU, VisionConfigC,  # noqa: E402
                                 VisP)  # (struct layouts only)
from sensenova_b200.config import ModelConfig  # noqa: E402

LIB_PATH = Path(os.environ.get("SNL_ORACLE_LIB", ROOT / "oracle" / "_build" / "liboracle.so"))
vp, sz, u32, u64, i32 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int
P = C.POINTER

_SIG = {
    "orc_last_error": (C.c_char_p, []),
    "orc_mat": (i32, [i32, P(StepU), P(MatP), vp, vp, vp, vp]),
    "orc_branch_norm": (i32, [P(StepU), P(LayerP), vp, vp, vp, vp, u32]),
    "orc_mhc_dots": (i32, [P(StepU), P(LayerP), vp, vp, vp]),
    "orc_mhc_finish": (i32, [P(StepU), P(LayerP), vp, vp, vp]),
    "orc_merge": (i32, [P(StepU), P(LayerP), vp, vp, vp]),
    "orc_swiglu": (i32, [P(StepU), P(LayerP), vp, vp]),
    "orc_attn_prep": (i32, [P(StepU), P(AttnP), vp, vp, vp, vp, vp, vp]),
    "orc_attend": (i32, [P(StepU), P(AttnP), vp, vp, vp, vp, vp, vp]),
    "orc_attn_combine": (i32, [P(StepU), P(AttnP), vp, vp, vp]),
    "orc_conv": (i32, [P(StepU), P(LinP), vp, vp, vp, vp, vp]),
    "orc_delta": (i32, [P(StepU), P(LinP), vp, vp, vp, vp, vp, vp]),
    "orc_argmax": (u32, [vp, sz]),
    "orc_sample": (i32, [P(SampleP), vp, u32, vp, vp, u32, vp, C.c_int64, vp]),
    "orc_dequant_q8_row": (None, [vp, vp, sz, vp]),
    "orc_gen_quant": (None, [u64, C.c_char_p, i32, sz, sz, vp, vp]),
    "orc_gen_f32": (None, [u64, C.c_char_p, u32, sz, C.c_float, C.c_float, vp]),
    "orc_config_validate": (i32, [P(ModelConfigC)]),
    "orc_model_create": (vp, [P(ModelConfigC), sz, u32, u64, i32]),
    "orc_model_destroy": (None, [vp]),
    "orc_model_reset": (i32, [vp]),
    "orc_model_snapshot": (i32, [vp, sz]),
    "orc_model_restore": (i32, [vp, sz, sz]),
    "orc_model_rollback": (i32, [vp]),
    "orc_model_pos": (sz, [vp]),
    "orc_model_hid_rows": (sz, [vp]),
    "orc_model_read_hidden": (i32, [vp, sz, sz, vp]),
    "orc_model_tensor": (vp, [vp, C.c_char_p, P(sz), P(sz), P(vp)]),
    "orc_model_tensor_dtype": (i32, [vp, C.c_char_p]),
    "orc_model_forward_mm": (i32, [vp, vp, sz, vp, vp, vp, sz, sz, i32, vp]),
    "orc_model_mtp": (i32, [vp, sz, vp, sz, vp, sz, i32, vp]),
    "orc_model_mtp_logits": (vp, [vp]),
    "orc_vis_layer_norm": (i32, [P(VisP), vp, vp, vp]),
    "orc_vis_epilogue": (i32, [P(VisP), vp, vp, vp, vp]),
    "orc_vis_rope": (i32, [P(VisP), vp]),
    "orc_vis_attend": (i32, [P(VisP), vp, vp]),
    "orc_vision_create": (vp, [P(VisionConfigC), u64]),
    "orc_vision_destroy": (None, [vp]),
    "orc_vision_encode": (i32, [vp, vp, sz, sz, sz, vp]),
    "orc_vision_tensor": (i32, [vp, C.c_char_p, P(vp), P(vp), P(sz), P(sz)]),
    "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
    "orc_set_vector": (None, [i32]),
    "orc_set_threads": (None, [i32]),
    "orc_get_threads": (i32, []),
    "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
}

_lib = None


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} missing: python sense-nova-server_b200/build.py --oracle")
        L = C.CDLL(str(LIB_PATH))
        for k, (r, a) in _SIG.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc:
        raise OracleError(rc, lib().orc_last_error().decode())


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


# ---- kernel level --------------------------------------------------------------


def mat(dtype: int, step: StepU, p: MatP, x: np.ndarray, wq: np.ndarray, ws: np.ndarray, y: np.ndarray) -> None:
    _check(lib().orc_mat(dtype, C.byref(step), C.byref(p), _p(x), _p(wq), _p(ws), _p(y)))


def branch_norm(step, p, x, coef, w, out, n_groups):
    _check(lib().orc_branch_norm(C.byref(step), C.byref(p), _p(x), _p(coef), _p(w), _p(out), n_groups))


def mhc_dots(step, p, x, w, raw):
    _check(lib().orc_mhc_dots(C.byref(step), C.byref(p), _p(x), _p(w), _p(raw)))


def mhc_finish(step, p, raw, w, coef):
    _check(lib().orc_mhc_finish(C.byref(step), C.byref(p), _p(raw), _p(w), _p(coef)))


def merge(step, p, x, coef, br):
    _check(lib().orc_merge(C.byref(step), C.byref(p), _p(x), _p(coef), _p(br)))


def swiglu(step, p, gu, act):
    _check(lib().orc_swiglu(C.byref(step), C.byref(p), _p(gu), _p(act)))


def attn_prep(step, p, proj, qbuf, kc, vc, norms, rpos):
    _check(lib().orc_attn_prep(C.byref(step), C.byref(p), _p(proj), _p(qbuf), _p(kc), _p(vc), _p(norms), _p(rpos)))


def attend(step, p, proj, qbuf, kc, vc, out, partial):
    _check(lib().orc_attend(C.byref(step), C.byref(p), _p(proj), _p(qbuf), _p(kc), _p(vc), _p(out), _p(partial)))


def attn_combine(step, p, proj, partial, out):
    _check(lib().orc_attn_combine(C.byref(step), C.byref(p), _p(proj), _p(partial), _p(out)))


def conv(step, p, proj, conv_out, conv_state, lw, conv_ckpt):
    _check(lib().orc_conv(C.byref(step), C.byref(p), _p(proj), _p(conv_out), _p(conv_state), _p(lw), _p(conv_ckpt)))


def delta(step, p, proj, conv_out, state, lw, out, state_ckpt):
    _check(lib().orc_delta(C.byref(step), C.byref(p), _p(proj), _p(conv_out), _p(state), _p(lw), _p(out),
                           _p(state_ckpt)))


def sample(params, logits: np.ndarray, hist_tok, hist_cnt, u, draft: int = -1) -> tuple[int, int, int]:
    """Sampler::sample / verify (sampler.rs:54-167) given the uniform draws u; logits are
    modified in place by the penalties. Returns (token, accepted, draws used)."""
    ht = np.ascontiguousarray(hist_tok, np.uint32)
    hc = np.ascontiguousarray(hist_cnt, np.uint32)
    uu = np.ascontiguousarray(u, np.float32)
    out = np.zeros(3, np.uint32)
    rc = lib().orc_sample(C.byref(params), _p(logits), logits.size, _p(ht), _p(hc), ht.size, _p(uu), int(draft),
                          _p(out))
    if rc:
        raise RuntimeError(lib().orc_last_error().decode())
    return int(out[0]), int(out[1]), int(out[2])


def set_vector(on: bool) -> None:
    """AVX2 forms of the matrix kernels (default) or the scalar statements; both give
    identical bits (tests/test_oracle_kernels.py checks it)."""
    lib().orc_set_vector(1 if on else 0)


def set_threads(n: int) -> None:
    """Threads of the oracle's OpenMP loops (n <= 0 leaves them as they are)."""
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_get_threads())


def argmax(v: np.ndarray) -> int:
    v = f32(v)
    return int(lib().orc_argmax(_p(v), v.size))


def dequant_q8_row(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = f32(s)
    out = np.empty(q.size, dtype=np.float32)
    lib().orc_dequant_q8_row(_p(q), _p(s), q.size, _p(out))
    return out


def gen_quant(seed: int, name: str, dtype: int, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """Seeded synthetic quantized tensor: (quants as u8 bytes, f32 scales)."""
    n = rows * cols
    q = np.empty(n if dtype == 1 else n // 2, dtype=np.uint8)
    s = np.empty(n // 32, dtype=np.float32)
    lib().orc_gen_quant(seed, name.encode(), dtype, rows, cols, _p(q), _p(s))
    return q, s


def gen_f32(seed: int, name: str, sub: int, n: int, mult: float, offset: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_gen_f32(seed, name.encode(), sub, n, mult, offset, _p(out))
    return out


# ---- model level ----------------------------------------------------------------


class OracleModel:
    """The reference's Engine on the CPU, with the seeded synthetic weights."""

    def __init__(self, cfg: ModelConfig, ctx: int, seed: int = 0, quant: int = 1, mtp: bool = False):
        self.cfg = cfg
        cc = cfg.to_c()
        self._h = lib().orc_model_create(C.byref(cc), ctx, 1 if mtp else 0, seed, quant)
        if not self._h:
            raise OracleError(-1, lib().orc_last_error().decode())

    def close(self):
        if self._h:
            lib().orc_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return int(lib().orc_model_pos(self._h))

    def hid_rows(self) -> int:
        return int(lib().orc_model_hid_rows(self._h))

    def reset(self):
        _check(lib().orc_model_reset(self._h))

    def snapshot(self, slot):
        _check(lib().orc_model_snapshot(self._h, slot))

    def restore(self, slot, pos):
        _check(lib().orc_model_restore(self._h, slot, pos))

    def rollback(self):
        _check(lib().orc_model_rollback(self._h))

    def read_hidden(self, row0, rows):
        out = np.empty((rows, self.cfg.hidden), dtype=np.float32)
        _check(lib().orc_model_read_hidden(self._h, row0, rows, _p(out)))
        return out

    def tensor(self, name: str):
        r, c = sz(), sz()
        s = vp()
        ptr = lib().orc_model_tensor(self._h, name.encode(), C.byref(r), C.byref(c), C.byref(s))
        if not ptr:
            raise KeyError(name)
        return ptr, int(r.value), int(c.value), s.value

    def tensor_dtype(self, name: str) -> int:
        """SNL_Q8_0 / SNL_Q4_0 of a matrix, -1 for a vector or an unknown name."""
        return int(lib().orc_model_tensor_dtype(self._h, name.encode()))

    def forward_mm(self, tokens, pos=None, logit_rows=0, ckpt=False, embeds=()):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        n = len(toks)
        pa = None if pos is None else np.ascontiguousarray(np.asarray(pos, dtype=np.uint32).reshape(-1, 3))
        idx = np.ascontiguousarray(np.asarray([i for i, _ in embeds], dtype=np.uint32)) if embeds else None
        emb = np.ascontiguousarray(np.stack([f32(r) for _, r in embeds])) if embeds else None
        rows = min(logit_rows, n - ((max(n - 1, 0)) // 512) * 512) if logit_rows else 0
        out = np.empty((max(rows, 1), self.cfg.vocab), dtype=np.float32) if rows else None
        _check(lib().orc_model_forward_mm(self._h, _p(toks), n, _p(pa), _p(idx), _p(emb),
                                          0 if emb is None else len(emb), logit_rows, int(ckpt), _p(out)))
        return out

    def forward(self, tokens, want_logits):
        out = self.forward_mm(tokens, None, int(want_logits))
        return None if out is None else out[0]

    def mtp(self, r0, tokens, pos, slot0, draft):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        pa = np.ascontiguousarray(np.asarray(pos, dtype=np.uint32).reshape(-1, 3))
        out = np.zeros(1, dtype=np.uint32)
        _check(lib().orc_model_mtp(self._h, r0, _p(toks), len(toks), _p(pa), slot0, int(draft), _p(out)))
        return int(out[0]) if draft else None

    def mtp_logits(self) -> np.ndarray:
        ptr = lib().orc_model_mtp_logits(self._h)
        return np.ctypeslib.as_array((C.c_float * self.cfg.vocab).from_address(ptr)).copy()


# ---- vision tower (vision.wgsl, vision.rs) ----------------------------------------------

def vis_layer_norm(p: VisP, a: np.ndarray, w: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.zeros_like(a)
    _check(lib().orc_vis_layer_norm(C.byref(p), _p(a), _p(b), _p(np.ascontiguousarray(w, np.float32))))
    return b


def vis_epilogue(p: VisP, a: np.ndarray, b: np.ndarray | None, w: np.ndarray, e: np.ndarray | None = None):
    """In place on a (mode 0) or b (modes 1, 2), as the kernel."""
    _check(lib().orc_vis_epilogue(C.byref(p), _p(a), None if b is None else _p(b), _p(np.ascontiguousarray(w, np.float32)),
                                  None if e is None else _p(e)))


def vis_rope(p: VisP, qkv: np.ndarray) -> None:
    _check(lib().orc_vis_rope(C.byref(p), _p(qkv)))


def vis_attend(p: VisP, qkv: np.ndarray) -> np.ndarray:
    out = np.zeros((p.rows, p.heads * 72), np.float32)
    _check(lib().orc_vis_attend(C.byref(p), _p(np.ascontiguousarray(qkv, np.float32)), _p(out)))
    return out


class OracleVision:
    """Vision (vision.rs) on the CPU with the seeded synthetic tower."""

    def __init__(self, cfg, seed: int = 0):
        self.cfg = cfg
        self._c = cfg.to_c()
        self._h = lib().orc_vision_create(C.byref(self._c), seed)

    def close(self):
        if self._h:
            lib().orc_vision_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, patches: np.ndarray, frames: int, h: int, w: int) -> np.ndarray:
        patches = np.ascontiguousarray(patches, np.float32)
        out = np.zeros((frames * h * w // 4, self.cfg.out_hidden), np.float32)
        _check(lib().orc_vision_encode(self._h, _p(patches), frames, h, w, _p(out)))
        return out

    def tensor(self, name: str):
        """(dtype, q bytes / f32 array, f32 scales or None, rows, cols) of one synthetic tensor."""
        q, s, r, c = C.c_void_p(), C.c_void_p(), C.c_size_t(), C.c_size_t()
        dt = lib().orc_vision_tensor(self._h, name.encode(), C.byref(q), C.byref(s), C.byref(r), C.byref(c))
        _check(dt if dt < 0 else 0)
        n = r.value * c.value
        if dt == 1:
            qa = np.ctypeslib.as_array((C.c_int8 * n).from_address(q.value)).copy()
            sa = np.ctypeslib.as_array((C.c_float * (n // 32)).from_address(s.value)).copy()
            return dt, qa, sa, r.value, c.value
        return dt, np.ctypeslib.as_array((C.c_float * n).from_address(q.value)).copy(), None, r.value, c.value
