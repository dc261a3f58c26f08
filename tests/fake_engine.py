"""A host stand-in for the engine, for CPU tests of the generation loop (snl_worker).

It keeps the engine's bookkeeping as engine.rs:651-774 defines it: the cache position,
the hidden rows of the last step (row 0 = the token before the step), hlast, the
checkpoint after the first row of a 2-row step, snapshot slots taken at a position and
the MTP cache slots. Its "recurrent state" is a 64-bit hash of every token fed with its
position, and a row's logits are seeded by that hash, so any mistake in what the loop
feeds, restores or rolls back changes the tokens. Every call is checked against the
engine's rules (rows in range, restore at the position of the snapshot, rollback only
after a checkpointed step, MTP rows paired with the right cache slots and positions);
violations are recorded in `violations` and fail the call.

Sampling follows sampler.rs through `py_sample` (tests/test_sampler.py's port).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from sensenova_b200 import ffi
from test_sampler import py_sample

MASK = (1 << 64) - 1


def mix(h: int, t: int, p: tuple[int, int, int]) -> int:
    v = (t * 0x9E3779B97F4A7C15 + p[0] * 0x1000193 + p[1] * 0x3B9ACA07 + p[2] * 0x2545F491 + 1) & MASK
    h = ((h ^ v) * 0x100000001B3) & MASK
    return h ^ (h >> 29)


def row_logits(h: int, vocab: int) -> np.ndarray:
    return (np.random.default_rng(h).standard_normal(vocab) * 2.0).astype(np.float32)


def first_argmax(v: np.ndarray) -> int:
    return int(np.argmax(v))


class FakeEngine:
    def __init__(self, vocab: int = 48, ctx: int = 400, chunk: int = 7, hidden: int = 4, mtp: bool = True,
                 draft_hit: float = 0.6, fwd_cost: float = 1.0, draft_cost: float = 0.2, fail_after: int | None = None):
        self.vocab, self.ctx, self.chunk, self.hidden, self.has_mtp = vocab, ctx, chunk, hidden, mtp
        self.draft_hit, self.fwd_cost, self.draft_cost = draft_hit, fwd_cost, draft_cost
        self.fail_after = fail_after  # fail the n-th forward call (error injection on the host)
        self.violations: list[str] = []
        self.calls: list[tuple] = []
        self.t = 0.0
        self.snaps: list[tuple | None] = [None] * ffi.SNL_WORKER_SNAPSHOTS
        self.mtp_filled: set[int] = set()
        self.n_forward = 0
        self._reset()
        self.ops = self._make_ops()

    # ---- state ------------------------------------------------------------------------
    def _reset(self):
        self.h = 0
        self.pos = 0
        self.hid_rows = 0
        self.hlast = None  # (slot, pos3, h) of the last fed token
        self.rows: list = [None]
        self.kept: list[np.ndarray] = []
        self.ckpt = None

    def _bad(self, msg: str) -> int:
        self.violations.append(msg)
        return ffi.SNL_E_STATE

    # ---- engine methods ----------------------------------------------------------------
    def forward(self, tokens, pos, embeds, logit_rows, ckpt):
        self.n_forward += 1
        self.t += self.fwd_cost
        if self.fail_after is not None and self.n_forward > self.fail_after:
            return ffi.SNL_E_CUDA
        n = len(tokens)
        self.calls.append(("forward", self.pos, list(tokens), logit_rows, ckpt))
        if n == 0 or self.pos + n > self.ctx:
            return self._bad(f"forward: {n} rows at {self.pos} beyond ctx {self.ctx}")
        if logit_rows > min(2, n) or (ckpt and n != 2):
            return self._bad("forward: unsupported logits or checkpoint request")
        rows = [self.hlast]
        h = self.h
        for i in range(n):
            key = embeds.get(i)
            t = int(tokens[i]) if key is None else key
            h = mix(h, t, tuple(pos[i]))
            rows.append((self.pos + i, tuple(pos[i]), h, int(tokens[i])))
            if ckpt and i == 0:
                self.ckpt = (h, rows[1])
        if not ckpt:
            self.ckpt = None
        self.h = h
        self.rows = rows
        self.hlast = rows[n]
        self.hid_rows = n
        self.pos += n
        self.kept = [row_logits(rows[n - logit_rows + j + 1][2], self.vocab) for j in range(logit_rows)]
        return 0

    def mtp(self, r0, tokens, pos, slot0, draft):
        self.t += self.draft_cost if draft else 0.0
        n = len(tokens)
        self.calls.append(("mtp", r0, list(tokens), slot0, draft))
        if n == 0 or r0 + n > self.hid_rows + 1:
            return self._bad(f"mtp: rows out of range (r0 {r0}, n {n}, hid {self.hid_rows})"), None
        for i in range(n):
            row = self.rows[r0 + i]
            if row is None:
                return self._bad("mtp: row without a token"), None
            if row[0] != slot0 + i or row[1] != tuple(pos[i]):
                return self._bad(f"mtp: row {r0 + i} is slot {row[0]} pos {row[1]}, "
                                 f"paired with slot {slot0 + i} pos {tuple(pos[i])}"), None
            if i + 1 < n:
                nxt = self.rows[r0 + i + 1] if r0 + i + 1 <= self.hid_rows else None
                if nxt is None or nxt[3] != int(tokens[i]):
                    return self._bad(f"mtp: token {tokens[i]} does not follow row {r0 + i}"), None
            self.mtp_filled.add(slot0 + i)
        if not draft:
            return 0, None
        last = self.rows[r0 + n - 1]
        r = last[1][0] + 1
        h = mix(last[2], int(tokens[-1]), (r, r, r))
        true_next = first_argmax(row_logits(h, self.vocab))
        coin = (h >> 7) % 1000 / 1000.0
        return 0, true_next if coin < self.draft_hit else (true_next + 1) % self.vocab

    def sample(self, row, p, hist, u, draft):
        if row >= len(self.kept):
            return self._bad("sample: no logits kept for that row"), None
        return 0, py_sample(p, self.kept[row], hist, u, draft)

    def snapshot(self, slot):
        self.calls.append(("snapshot", slot, self.pos))
        self.snaps[slot] = (self.h, self.hlast, self.pos)
        return 0

    def restore(self, slot, pos):
        self.calls.append(("restore", slot, pos))
        s = self.snaps[slot]
        if s is None or s[2] != pos:
            return self._bad(f"restore: slot {slot} holds {None if s is None else s[2]}, asked for {pos}")
        self.h, self.hlast, _ = s
        self.pos, self.hid_rows, self.rows, self.kept, self.ckpt = pos, 0, [self.hlast], [], None
        return 0

    def rollback(self):
        self.calls.append(("rollback", self.pos))
        if self.ckpt is None:
            return self._bad("rollback without a checkpointed 2-row step")
        self.h, self.hlast = self.ckpt
        self.pos -= 1
        self.hid_rows = 1
        self.ckpt = None
        return 0

    def reset(self):
        self.calls.append(("reset",))
        self._reset()
        return 0

    # ---- the C ops table ----------------------------------------------------------------
    def _make_ops(self) -> ffi.WorkerOps:
        u32a = lambda a, n: np.ctypeslib.as_array((C.c_uint32 * max(n, 1)).from_address(a))[:n].copy() if n else []

        def pos3(a, n):
            return [tuple(int(x) for x in r) for r in u32a(a, 3 * n).reshape(n, 3)] if n else []

        def fwd(_s, tp, n, pp, ei, em, ne, rows, ckpt):
            try:
                emb = {}
                if ne:
                    idx = u32a(ei, ne)
                    vals = np.ctypeslib.as_array((C.c_float * (ne * self.hidden)).from_address(em))
                    for j in range(ne):
                        emb[int(idx[j])] = int(abs(float(vals[j * self.hidden:(j + 1) * self.hidden].sum())) * 1e4) | (1 << 40)
                return self.forward(u32a(tp, n), pos3(pp, n), emb, rows, ckpt)
            except Exception as ex:  # noqa: BLE001
                return self._bad(f"forward raised {ex!r}")

        def fwd_greedy(_s, tp, n, pp, rows, ckpt, out):
            try:
                rc = self.forward(u32a(tp, n), pos3(pp, n), {}, rows, ckpt)
                if rc:
                    return rc
                o = (C.c_uint32 * rows).from_address(out)
                for j in range(rows):
                    o[j] = first_argmax(self.kept[j])
                return 0
            except Exception as ex:  # noqa: BLE001
                return self._bad(f"forward_greedy raised {ex!r}")

        def sample(_s, row, pp, ht, hc, nh, up, draft, out):
            try:
                p = pp.contents
                hist = list(zip(u32a(ht, nh).tolist(), u32a(hc, nh).tolist())) if nh else []
                u = np.ctypeslib.as_array((C.c_float * 2).from_address(up)).tolist()
                rc, res = self.sample(row, p, hist, u, int(draft))
                if rc:
                    return rc
                o = (C.c_uint32 * 3).from_address(out)
                o[0], o[1], o[2] = res
                return 0
            except Exception as ex:  # noqa: BLE001
                return self._bad(f"sample raised {ex!r}")

        def mtp(_s, r0, tp, n, pp, slot0, draft, out):
            try:
                rc, d = self.mtp(r0, u32a(tp, n), pos3(pp, n), slot0, bool(draft))
                if rc:
                    return rc
                if draft:
                    C.c_uint32.from_address(out).value = d
                return 0
            except Exception as ex:  # noqa: BLE001
                return self._bad(f"mtp raised {ex!r}")

        self._cbs = [
            ffi.FWD_FN(fwd), ffi.FWD_GREEDY_FN(fwd_greedy), ffi.SAMPLE_FN(sample), ffi.MTP_FN(mtp),
            ffi.SELF_FN(lambda _s: self.reset()), ffi.SLOT_FN(lambda _s, k: self.snapshot(k)),
            ffi.RESTORE_FN(lambda _s, k, p: self.restore(k, p)), ffi.SELF_FN(lambda _s: self.rollback()),
            ffi.SIZE_FN(lambda _s: self.hid_rows), ffi.SIZE_FN(lambda _s: self.pos), ffi.NOW_FN(lambda _s: self.t),
        ]
        o = ffi.WorkerOps()
        o.self = None
        o.ctx, o.prefill_chunk, o.hidden, o.has_mtp = self.ctx, self.chunk, self.hidden, int(self.has_mtp)
        (o.forward, o.forward_greedy, o.sample, o.mtp, o.reset, o.snapshot, o.restore, o.rollback, o.hid_rows,
         o.pos, o.now) = self._cbs
        return o
