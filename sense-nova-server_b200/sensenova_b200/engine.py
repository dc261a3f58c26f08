"""Engine: the Python face of the reference's Engine (src/engine.rs:151-949).

Same method names, argument meaning and error behaviour as the Rust surface
(`forward`, `forward_mm`, `mtp`, `reset`, `snapshot`, `restore`, `rollback`,
`hid_rows`, `has_mtp`, `pos`, `ctx`), over the C ABI of libsnl_b200.so. Errors
raise `SnlError` carrying the reference's messages ("context length exceeded
(a > b)", "token id t out of range", "forward: unsupported logits or checkpoint
request", "mtp: rows out of range").
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Sequence

import numpy as np

from . import ffi
from .config import ModelConfig

LOGIT_ROWS = 2  # engine.rs:22
SNAPSHOTS = 4  # engine.rs:20


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def gather_tp_handles(rank: int, size: int, mine: bytes, group) -> bytes:
    """All-gathers every rank's exchange-region handle over torch.distributed and returns
    them concatenated in rank order (what snl_engine_tp_connect takes)."""
    import torch.distributed as dist

    handles: list = [None] * size
    dist.all_gather_object(handles, (rank, mine), group=group)
    by_rank = dict(handles)
    if sorted(by_rank) != list(range(size)):
        raise ffi.SnlError(ffi.SNL_E_INVALID, "tensor parallel: ranks of the group do not match tp")
    return b"".join(by_rank[r] for r in range(size))


class Engine:
    """One model on one GPU. Not thread-safe (one owner thread, like the reference)."""

    def __init__(self, cfg: ModelConfig, ctx: int, *, device: int = 0, mtp: bool = False, flags: int = 0,
                 tp: tuple[int, int] | None = None, tp_group=None):
        """tp = (rank, size) builds one tensor-parallel shard; every rank of the group
        constructs its Engine with the same arguments (one process per GPU), and the
        ranks' exchange handles are all-gathered over `tp_group` (a torch.distributed
        process group; None = the default group)."""
        self.lib = ffi.load()
        self.cfg = cfg
        self._h = C.c_void_p()
        cc = cfg.to_c()
        fl = flags | (ffi.SNL_ENGINE_MTP if mtp else 0)
        self.tp = tp if tp is not None else (0, 1)
        if self.tp[1] > 1:
            ffi.check(self.lib.snl_engine_create_tp(C.byref(cc), ctx, device, fl, self.tp[0], self.tp[1],
                                                    C.byref(self._h)))
            self._tp_connect(tp_group)
        else:
            ffi.check(self.lib.snl_engine_create(C.byref(cc), ctx, device, fl, C.byref(self._h)))
        self.quant = "q8_0"
        self.device = device

    def _tp_connect(self, group) -> None:
        buf = (C.c_uint8 * ffi.SNL_TP_HANDLE_BYTES)()
        ffi.check(self.lib.snl_engine_tp_handle(self._h, C.cast(buf, C.c_void_p)))
        allh = gather_tp_handles(self.tp[0], self.tp[1], bytes(buf), group)
        arr = (C.c_uint8 * len(allh)).from_buffer_copy(allh)
        ffi.check(self.lib.snl_engine_tp_connect(self._h, C.cast(arr, C.c_void_p)))

    # ---- construction -------------------------------------------------------------

    @classmethod
    def synthetic(cls, cfg: ModelConfig, ctx: int, seed: int = 0, quant: str = "q8_0", *, mtp: bool = False,
                  device: int = 0, flags: int = 0, tp: tuple[int, int] | None = None, tp_group=None) -> "Engine":
        """The seeded random-init model of the benchmarks, generated on the device."""
        e = cls(cfg, ctx, device=device, mtp=mtp, flags=flags, tp=tp, tp_group=tp_group)
        q = {"q8_0": ffi.SNL_Q8_0, "q4_0": ffi.SNL_Q4_0}[quant]
        ffi.check(e.lib.snl_engine_fill_synthetic(e._h, seed, q))
        ffi.check(e.lib.snl_engine_finalize(e._h))
        e.quant = quant
        return e

    @classmethod
    def load(cls, path: str | Path, ctx: int, mtp: str | Path | None = None, *, device: int = 0) -> "Engine":
        """Engine::load (engine.rs:230) from a `.snl` file (and an optional MTP file)."""
        from .weights import WeightFile

        wf = WeightFile.open(path)
        e = cls(wf.config, ctx, device=device, mtp=mtp is not None)
        e.quant = wf.quant
        files = [wf] + ([WeightFile.open(mtp)] if mtp is not None else [])
        for f in files:
            for name in f.tensors:
                dtype, rows, cols, q, s = f.raw(name)
                ffi.check(e.lib.snl_engine_set_tensor(
                    e._h, name.encode(), dtype, rows, cols, q.ctypes.data,
                    s.ctypes.data if s is not None else None))
        ffi.check(e.lib.snl_engine_finalize(e._h))
        return e

    def close(self) -> None:
        if self._h:
            self.lib.snl_engine_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- state ----------------------------------------------------------------------

    @property
    def pos(self) -> int:
        return int(self.lib.snl_engine_pos(self._h))

    @property
    def ctx(self) -> int:
        return int(self.lib.snl_engine_ctx(self._h))

    @property
    def device_bytes(self) -> int:
        return int(self.lib.snl_engine_device_bytes(self._h))

    def hid_rows(self) -> int:
        return int(self.lib.snl_engine_hid_rows(self._h))

    def has_mtp(self) -> bool:
        return bool(self.lib.snl_engine_has_mtp(self._h))

    def tile_scales(self) -> tuple[int, int]:
        """(matrices whose decode tile layout keeps fp16 block scales, those keeping f32)."""
        a, b = C.c_uint32(), C.c_uint32()
        ffi.check(self.lib.snl_engine_tile_scales(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def reset(self) -> None:
        ffi.check(self.lib.snl_engine_reset(self._h))

    def snapshot(self, slot: int) -> None:
        ffi.check(self.lib.snl_engine_snapshot(self._h, slot))

    def restore(self, slot: int, pos: int) -> None:
        ffi.check(self.lib.snl_engine_restore(self._h, slot, pos))

    def rollback(self) -> None:
        ffi.check(self.lib.snl_engine_rollback(self._h))

    def read_hidden(self, row0: int, rows: int) -> np.ndarray:
        out = np.empty((rows, self.cfg.hidden), dtype=np.float32)
        ffi.check(self.lib.snl_engine_read_hidden(self._h, row0, rows, out.ctypes.data))
        return out

    # ---- forward --------------------------------------------------------------------

    def forward(self, tokens: Sequence[int], want_logits: bool) -> np.ndarray | None:
        """engine.rs:794-796: rotary positions = cache positions; logits of the last token."""
        out = self.forward_mm(tokens, None, (), int(want_logits), False)
        return None if out is None else out[0]

    def forward_mm(self, tokens: Sequence[int], pos: Sequence[Sequence[int]] | None = None,
                   embeds: Sequence[tuple[int, np.ndarray]] = (), logit_rows: int = 0,
                   ckpt: bool = False) -> np.ndarray | None:
        """engine.rs:801-936. Returns logits [logit_rows, vocab] (or None)."""
        toks = _u32(tokens)
        n = len(toks)
        pos_a = None if pos is None else _u32(pos).reshape(-1, 3)
        if pos_a is not None and len(pos_a) != n:
            raise ffi.SnlError(-1, "forward: positions or embeddings do not match the tokens")
        idx = _u32([i for i, _ in embeds]) if embeds else None
        emb = (np.ascontiguousarray(np.stack([np.asarray(r, dtype=np.float32) for _, r in embeds]))
               if embeds else None)
        if emb is not None and emb.shape[1] != self.cfg.hidden:
            raise ffi.SnlError(-1, "forward: positions or embeddings do not match the tokens")
        rows = min(logit_rows, n - (max(n - 1, 0) // 512) * 512) if logit_rows else 0
        out = np.empty((max(rows, 1), self.cfg.vocab), dtype=np.float32) if rows else None
        ffi.check(self.lib.snl_engine_forward_mm(
            self._h, toks.ctypes.data if n else None, n,
            pos_a.ctypes.data if pos_a is not None else None,
            idx.ctypes.data if idx is not None else None,
            emb.ctypes.data if emb is not None else None, 0 if emb is None else len(emb),
            logit_rows, int(bool(ckpt)), out.ctypes.data if out is not None else None))
        return out

    def forward_keep(self, tokens: Sequence[int], logit_rows: int = 1, ckpt: bool = False) -> None:
        """forward_mm whose logits stay on the device for sample() (no 1 MB copy per row)."""
        toks = _u32(tokens)
        ffi.check(self.lib.snl_engine_forward_mm(self._h, toks.ctypes.data if len(toks) else None, len(toks), None,
                                                 None, None, 0, logit_rows, int(bool(ckpt)), None))

    def sample(self, row: int, params, history: dict[int, int] | None = None, u=(0.5, 0.5),
               draft: int = -1) -> tuple[int, bool, int]:
        """Sampler::sample (draft < 0) or Sampler::verify(draft) (sampler.rs:54-167) on the
        device, on logit row `row` of the last forward; u: the host generator's uniform
        draws. Returns (token, accepted, draws used)."""
        hist = history or {}
        ht = np.ascontiguousarray(list(hist.keys()), dtype=np.uint32)
        hc = np.ascontiguousarray(list(hist.values()), dtype=np.uint32)
        uu = np.ascontiguousarray(u, dtype=np.float32)
        out = np.zeros(3, dtype=np.uint32)
        ffi.check(self.lib.snl_engine_sample(self._h, row, C.byref(params), ht.ctypes.data if ht.size else None,
                                             hc.ctypes.data if hc.size else None, ht.size, uu.ctypes.data, int(draft),
                                             out.ctypes.data))
        return int(out[0]), bool(out[1]), int(out[2])

    def forward_greedy(self, tokens: Sequence[int], pos: Sequence[Sequence[int]] | None = None,
                       logit_rows: int = 1, ckpt: bool = False) -> list[int]:
        """forward_mm + argmax on the device; only the token ids come back."""
        toks = _u32(tokens)
        n = len(toks)
        pos_a = None if pos is None else _u32(pos).reshape(-1, 3)
        out = np.zeros(LOGIT_ROWS, dtype=np.uint32)
        ffi.check(self.lib.snl_engine_forward_greedy(
            self._h, toks.ctypes.data if n else None, n, pos_a.ctypes.data if pos_a is not None else None,
            logit_rows, int(bool(ckpt)), out.ctypes.data))
        rows = min(logit_rows, n - (max(n - 1, 0) // 512) * 512)
        return [int(v) for v in out[:rows]]

    def generate(self, first_token: int, n: int) -> tuple[list[int], float]:
        """Greedy generation of n tokens with the argmax fed back on the device.
        Returns (tokens, device milliseconds of the n steps)."""
        out = np.zeros(n, dtype=np.uint32)
        ms = C.c_float(0.0)
        ffi.check(self.lib.snl_engine_generate(self._h, first_token, n, out.ctypes.data, C.byref(ms)))
        return [int(v) for v in out], float(ms.value)

    def profile(self, token: int) -> list[dict]:
        """One decode step op by op (engine.rs:859-886): [{label, calls, ms, bytes}]."""
        cap = 64
        arr = (ffi.OpStat * cap)()
        n = C.c_size_t(0)
        ffi.check(self.lib.snl_engine_profile(self._h, token, arr, cap, C.byref(n)))
        return [{"label": arr[i].label.decode(), "calls": arr[i].calls, "ms": arr[i].ms, "bytes": arr[i].bytes}
                for i in range(n.value)]

    def print_profile(self, rows: list[dict]) -> None:
        """The table of Engine::print_profile (engine.rs:938-949)."""
        total = sum(r["ms"] for r in rows) or 1.0
        print(f"{'op':<28} {'total ms':>10} {'share':>8} {'calls':>10} {'GB/s':>8}")
        for r in sorted(rows, key=lambda r: -r["ms"]):
            gbs = r["bytes"] / (r["ms"] * 1e6) if r["ms"] > 0 else 0.0
            print(f"{r['label']:<28} {r['ms']:>10.3f} {100 * r['ms'] / total:>7.1f}% {r['calls']:>10} {gbs:>8.0f}")

    def mtp(self, r0: int, tokens: Sequence[int], pos: Sequence[Sequence[int]], slot0: int,
            draft: bool) -> int | None:
        """engine.rs:708-774: None without an MTP head or without `draft`."""
        if not self.has_mtp():
            return None
        toks = _u32(tokens)
        pos_a = _u32(pos).reshape(-1, 3)
        if len(pos_a) != len(toks):
            raise ffi.SnlError(-2, "mtp: rows out of range")
        out = np.zeros(1, dtype=np.uint32)
        ffi.check(self.lib.snl_engine_mtp(self._h, r0, toks.ctypes.data if len(toks) else None, len(toks),
                                          pos_a.ctypes.data if len(toks) else None, slot0, int(bool(draft)),
                                          out.ctypes.data))
        return int(out[0]) if draft else None
