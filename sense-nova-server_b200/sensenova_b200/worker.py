"""Worker: the Python face of the reference's generation loop (src/worker.rs).

`Worker.run` is `Worker::run` (worker.rs:118-270) on token ids: it reuses the longest
cached strict prefix (the live cache or one of four snapshot slots, least recently used
first out), snapshots at `snapshot_at`, feeds the prompt in engine chunks (with the MTP
head warmed on every prompt row when drafting), then decodes with draft-1 / verify-2
speculation and rollback, pausing drafting for 20 requests when it does not pay off.
The loop runs in the library (`snl_worker_run`); sampling runs on the device with the
host generator's uniform draws. Text, stop strings and media encoding stay with the
caller: a prompt is token ids, prefix keys and M-RoPE positions, plus any encoded media
rows.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np

from . import ffi

SNAPSHOTS = 4  # engine.rs:20


@dataclass
class SamplingParams:
    """SamplingParams (sampler.rs:4-29), with its defaults."""
    temperature: float = 1.0
    top_p: float = 0.95
    top_k: int = 20
    min_p: float = 0.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    seed: int | None = None

    def to_c(self) -> ffi.SampleP:
        return ffi.SampleP(self.temperature, self.top_p, self.top_k, self.min_p, self.presence_penalty,
                           self.frequency_penalty, self.repetition_penalty, 0)


GREEDY = SamplingParams(temperature=0.0, top_p=1.0, top_k=1)


@dataclass
class Prompt:
    """Prompt (mm.rs:383-409) after tokenisation: ids, prefix-cache keys, (t, h, w)
    positions, and encoded media rows as (prompt index, hidden floats)."""
    tokens: list[int]
    keys: list[int] | None = None
    pos: list[tuple[int, int, int]] | None = None
    media_rows: list[tuple[int, np.ndarray]] = field(default_factory=list)

    @classmethod
    def text(cls, tokens: Sequence[int]) -> "Prompt":
        return cls(list(tokens))

    def next_pos(self) -> int:
        if self.pos is None:
            return len(self.tokens)
        return max((max(p) for p in self.pos), default=-1) + 1


@dataclass
class Finish:
    """Finish (worker.rs:41-55)."""
    reason: str
    prompt_tokens: int
    completion_tokens: int
    cached_tokens: int
    prefill_secs: float
    decode_secs: float
    cancelled: bool
    drafted: int
    accepted: int


class Worker:
    """One generation loop over one engine; not thread-safe (the reference's generation
    thread owns its Worker)."""

    def __init__(self, engine=None, *, ops: ffi.WorkerOps | None = None):
        """engine: a `sensenova_b200.engine.Engine`; or ops: an `ffi.WorkerOps` table
        (any implementation of the engine methods the loop calls)."""
        self.lib = ffi.load()
        self._h = C.c_void_p()
        self._engine = engine
        self._ops = ops
        if engine is not None:
            ffi.check(self.lib.snl_worker_create(engine._h, C.byref(self._h)))
        elif ops is not None:
            ffi.check(self.lib.snl_worker_create_ops(C.byref(ops), C.byref(self._h)))
        else:
            raise ValueError("Worker needs an engine or an ops table")

    def close(self) -> None:
        if self._h:
            self.lib.snl_worker_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def run(self, prompt: Prompt | Sequence[int], params: SamplingParams = GREEDY, max_tokens: int = 256, *,
            eos: Sequence[int] = (), snapshot_at: int | None = None,
            on_token: Callable[[int], bool] | None = None) -> tuple[list[int], Finish]:
        """Generate for one request. Returns the generated ids (the EOS id last when the
        request stopped on it) and the Finish record. on_token(t) streams each non-EOS
        id; returning False ends the request as a client disconnect."""
        if not isinstance(prompt, Prompt):
            prompt = Prompt.text(prompt)
        n = len(prompt.tokens)
        toks = np.ascontiguousarray(np.asarray(prompt.tokens, dtype=np.uint32))
        keys = None if prompt.keys is None else np.ascontiguousarray(np.asarray(prompt.keys, dtype=np.uint64))
        pos = None if prompt.pos is None else np.ascontiguousarray(np.asarray(prompt.pos, dtype=np.uint32).reshape(n, 3))
        eos_a = np.ascontiguousarray(np.asarray(list(eos), dtype=np.uint32))
        req = ffi.GenRequestC()
        req.tokens = toks.ctypes.data if n else None
        req.keys = None if keys is None else keys.ctypes.data
        req.pos = None if pos is None else pos.ctypes.data
        req.n = n
        if prompt.media_rows:
            idx = np.ascontiguousarray(np.asarray([i for i, _ in prompt.media_rows], dtype=np.uint32))
            rows = np.ascontiguousarray(np.stack([np.asarray(r, dtype=np.float32) for _, r in prompt.media_rows]))
            req.embed_idx, req.embeds, req.n_embeds = idx.ctypes.data, rows.ctypes.data, len(idx)
        req.snapshot_at = -1 if snapshot_at is None else int(snapshot_at)
        req.params = params.to_c()
        req.seed = 0 if params.seed is None else int(params.seed)
        req.has_seed = 0 if params.seed is None else 1
        req.max_tokens = int(max_tokens)
        req.eos = eos_a.ctypes.data if len(eos_a) else None
        req.n_eos = len(eos_a)
        cb = None
        if on_token is not None:
            def _cb(_user, t):
                try:
                    return 1 if on_token(int(t)) is not False else 0
                except Exception:
                    return 0
            cb = ffi.TOKEN_FN(_cb)
            req.on_token = cb
        cap = max(int(max_tokens), 0) + 2
        out = np.zeros(cap, dtype=np.uint32)
        fin = ffi.FinishC()
        ffi.check(self.lib.snl_worker_run(self._h, C.byref(req), out.ctypes.data, cap, C.byref(fin)))
        got = out[:min(fin.completion_tokens, cap)].tolist()
        f = Finish("stop" if fin.reason == ffi.SNL_FINISH_STOP else "length", fin.prompt_tokens,
                   fin.completion_tokens, fin.cached_tokens, fin.prefill_secs, fin.decode_secs, bool(fin.cancelled),
                   fin.drafted, fin.accepted)
        return got, f

    def prefix(self, slot: int = -1) -> tuple[list[int], int]:
        """Keys held by the live cache (slot -1) or a snapshot slot, and its last use."""
        n = C.c_size_t()
        ffi.check(self.lib.snl_worker_prefix(self._h, slot, None, 0, C.byref(n), None))
        buf = np.zeros(max(n.value, 1), dtype=np.uint64)
        used = C.c_uint64()
        ffi.check(self.lib.snl_worker_prefix(self._h, slot, buf.ctypes.data, n.value, C.byref(n), C.byref(used)))
        return buf[:n.value].tolist(), used.value

    def spec(self) -> tuple[bool, int]:
        """(drafting in the current request, requests left in a drafting pause)."""
        s, p = C.c_int(), C.c_size_t()
        ffi.check(self.lib.snl_worker_spec(self._h, C.byref(s), C.byref(p)))
        return bool(s.value), p.value


def uniforms(seed: int, n: int) -> np.ndarray:
    """The first n draws of the worker's generator for `seed`."""
    out = np.zeros(n, dtype=np.float32)
    ffi.check(ffi.load().snl_rng_uniforms(seed, n, out.ctypes.data))
    return out
