"""Vision: the Python face of the reference's vision tower (src/vision.rs).

`Vision.encode(patches, frames, h, w)` is `Vision::encode` (vision.rs:176-311): patch
vectors in merge order, frame-major, to `frames * h * w / 4` rows of `out_hidden` floats
that the language model splices in as token embeddings (`forward_mm`'s `embeds`, or a
worker prompt's media rows). Weights come by name as convert.rs:165-199 writes them, or
from the seeded synthetic set.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import ffi


@dataclass
class VisionConfig:
    """VisionConfig (config.rs:40-70); head_dim = hidden / n_heads must be 72 and merge 2."""
    hidden: int = 1152
    intermediate: int = 4304
    intermediate_padded: int = 4320
    depth: int = 27
    n_heads: int = 16
    patch: int = 16
    temporal_patch: int = 2
    merge: int = 2
    out_hidden: int = 4096
    pos_side: int = 48

    def patch_dim(self) -> int:
        return 3 * self.temporal_patch * self.patch * self.patch

    def merged_dim(self) -> int:
        return self.hidden * self.merge * self.merge

    def to_c(self) -> ffi.VisionConfigC:
        return ffi.VisionConfigC(self.hidden, self.intermediate, self.intermediate_padded, self.depth, self.n_heads,
                                 self.patch, self.temporal_patch, self.merge, self.out_hidden, self.pos_side)


def small_vision() -> VisionConfig:
    """A two-block tower with the kernels' fixed head size, for tests."""
    return VisionConfig(hidden=288, intermediate=200, intermediate_padded=224, depth=2, n_heads=4, patch=4,
                        temporal_patch=2, merge=2, out_hidden=128, pos_side=6)


class Vision:
    """The tower on one GPU; not thread-safe."""

    def __init__(self, cfg: VisionConfig, device: int = 0):
        self.lib = ffi.load()
        self.cfg = cfg
        self._h = C.c_void_p()
        cc = cfg.to_c()
        ffi.check(self.lib.snl_vision_create(C.byref(cc), device, C.byref(self._h)))

    @classmethod
    def synthetic(cls, cfg: VisionConfig, seed: int = 0, device: int = 0) -> "Vision":
        v = cls(cfg, device)
        ffi.check(v.lib.snl_vision_fill_synthetic(v._h, seed))
        ffi.check(v.lib.snl_vision_finalize(v._h))
        return v

    def set_tensor(self, name: str, q: np.ndarray, s: np.ndarray | None = None, rows: int = 1,
                   cols: int | None = None) -> None:
        """A Q8_0 matrix (q int8 [rows, cols] bytes, s f32 [rows, cols/32]) or an f32 vector."""
        q = np.ascontiguousarray(q)
        if s is None:
            q = q.astype(np.float32, copy=False)
            ffi.check(self.lib.snl_vision_set_tensor(self._h, name.encode(), ffi.SNL_F32, 1, q.size, q.ctypes.data,
                                                     None))
        else:
            s = np.ascontiguousarray(s, np.float32)
            ffi.check(self.lib.snl_vision_set_tensor(self._h, name.encode(), ffi.SNL_Q8_0, rows, cols, q.ctypes.data,
                                                     s.ctypes.data))

    def finalize(self) -> None:
        ffi.check(self.lib.snl_vision_finalize(self._h))

    def encode(self, patches: np.ndarray, frames: int, h: int, w: int) -> np.ndarray:
        patches = np.ascontiguousarray(patches, np.float32)
        if patches.size != frames * h * w * self.cfg.patch_dim():
            raise ffi.SnlError(ffi.SNL_E_INVALID, "vision input has the wrong shape")
        out = np.zeros((frames * h * w // 4, self.cfg.out_hidden), np.float32)
        ffi.check(self.lib.snl_vision_encode(self._h, patches.ctypes.data, frames, h, w, out.ctypes.data))
        return out

    def close(self) -> None:
        if self._h:
            self.lib.snl_vision_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
