"""The reference's forward pass from its own kernels - TEST INFRASTRUCTURE ONLY.

The op list that src/engine.rs:383-493 records (and forward_mm, :801-936, runs per
prefill chunk), restated in Python over the reference's WGSL kernels translated to C++
(oracle/wgslref.py), with the weights of an oracle model (oracle/oracle.py) so both run
on the same tensors. A test compares its logits with the oracle model's: the same graph,
one side built from the reference's kernel code.

Steps of at most one prefill chunk (512 rows) per call; each matrix in the oracle model's
quantization (Q8_0, or Q4_0 for the matrices a Q4_0 conversion quantizes). `mtp` restates Engine::mtp (engine.rs:700-774) over the MTP layer
that engine.rs:495-580 builds, when the oracle model has one.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))
import wgslref as wr  # noqa: E402
from sensenova_b200.ffi import AttnP, LayerP, LinP, MatP, StepU, VisP  # noqa: E402

Q8 = 1
CHUNK = 512  # engine.rs prefill_chunk


class RefModel:
    def __init__(self, cfg, ctx: int, weights):
        self.cfg, self.ctx, self.w = cfg, ctx, weights
        self.plan = cfg.execution_plan()
        self.pos = 0
        h = cfg.hidden
        self.hlast = np.zeros(h, np.float32)
        n_full = sum(1 for li in self.plan if cfg.full_attention[li])
        n_lin = len(self.plan) - n_full
        kv_words = ctx * cfg.kv_dim // 2
        self.kc = [np.zeros(kv_words, np.uint32) for _ in range(n_full)]
        self.vc = [np.zeros(kv_words, np.uint32) for _ in range(n_full)]
        self.conv = [np.zeros(3 * cfg.conv_dim, np.float32) for _ in range(n_lin)]
        self.state = [np.zeros(cfg.lin_v_heads * 128 * 128, np.float32) for _ in range(n_lin)]
        self.mkc = np.zeros(kv_words, np.uint32)  # the MTP layer's own cache
        self.mvc = np.zeros(kv_words, np.uint32)
        self.hid = np.zeros(h, np.float32)
        self.hid_rows = 0

    # -- weights of the oracle model --
    def q(self, name: str):
        ptr, rows, cols, s = self.w.tensor(name)
        dt = self.w.tensor_dtype(name)
        nbytes = rows * cols if dt == Q8 else rows * cols // 2
        q = np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(ptr)).copy()
        sc = np.ctypeslib.as_array((C.c_float * (rows * cols // 32)).from_address(s)).copy()
        return q, sc, rows, cols, dt

    def f(self, name: str) -> np.ndarray:
        ptr, _, n, _ = self.w.tensor(name)
        return np.ctypeslib.as_array((C.c_float * n).from_address(ptr)).copy()

    def layer_p(self, mode: int, last_row: bool = False) -> LayerP:
        c = self.cfg
        return LayerP(c.hidden, mode, 1 if last_row else 0, c.eps, 1.0, c.mhc.iterations if c.mhc else 0,
                      c.intermediate, 0)

    def mat(self, st, name, x, x_stride, y, y_stride, m_one=0, x_off=0):
        """engine.rs:336-363 (one chunk: n_off 0)."""
        q, s, rows, cols, dt = self.q(name)
        wr.mat(dt, st, MatP(rows, cols, x_off, x_stride, 0, y_stride, 0, m_one), x, q, s, y)

    def embed(self, tokens) -> np.ndarray:
        """engine.rs:777-790: stream 0 the dequantized row, stream 1 zero."""
        h = self.cfg.hidden
        eq, es, _, _, dt = self.q("embed")
        assert dt == Q8, "the embedding stays Q8_0 (convert.rs)"
        x = np.zeros(len(tokens) * 2 * h, np.float32)
        codes = eq.view(np.int8).astype(np.float32)
        for i, t in enumerate(tokens):
            x[i * 2 * h:i * 2 * h + h] = codes[t * h:(t + 1) * h] * np.repeat(es[t * h // 32:(t + 1) * h // 32], 32)
        return x

    def attn_p(self) -> AttnP:
        c = self.cfg
        return AttnP(c.n_heads, c.n_kv_heads, c.rot_dim, c.attn_proj_rows, c.rope_theta, c.eps,
                     float(np.float32(1.0) / np.sqrt(np.float32(c.head_dim))),
                     ((3 * c.mrope_section[1]) << 16) | (3 * c.mrope_section[2]))

    def forward(self, tokens, want_logits: bool):
        c, h = self.cfg, self.cfg.hidden
        m = len(tokens)
        assert 0 < m <= CHUNK and self.pos + m <= self.ctx
        total = self.pos + m
        parts = min(max(-(-total // 256), 1), 64) if m <= 4 else 1  # engine.rs:827
        st = StepU(m, self.pos, parts, 0)
        x = self.embed(tokens)
        rpos = np.repeat(np.arange(self.pos, self.pos + m, dtype=np.uint32)[:, None], 4, 1).reshape(-1).copy()
        coef = np.zeros(m * 8, np.float32)
        xn = np.zeros(m * h, np.float32)
        proj = np.zeros(m * max(c.attn_proj_rows, c.lin_proj_rows, 2 * c.intermediate), np.float32)
        act = np.zeros(m * max(c.intermediate, c.conv_dim), np.float32)
        attn_out = np.zeros(m * max(c.q_dim, c.lin_value_dim), np.float32)
        branch = np.zeros(m * h, np.float32)
        qbuf = np.zeros(m * c.q_dim, np.float32)
        partial = np.zeros(m * c.n_heads * parts * 258, np.float32)
        raw = np.zeros(m * 9, np.float32)

        def push_norm(router, norm_w):
            if router is not None:
                wr.mhc_dots(st, self.layer_p(0), x, router, raw)
                wr.mhc_finish(st, self.layer_p(0), raw, router, coef)
            wr.branch_norm(st, self.layer_p(1 if router is not None else 0), x, coef, norm_w, xn, m)

        lin_slot = full_slot = 0
        mhc_start = c.mhc.start if c.mhc else None
        mhc_end = c.mhc.end if c.mhc else None
        for li in self.plan:
            L = f"l{li}."
            mhc = c.is_mhc(li)
            if mhc and li == mhc_start:
                wr.merge(st, self.layer_p(3), x, coef, branch)
            push_norm(self.f(L + "mhc_attn") if mhc else None, self.f(L + "in_ln"))
            if c.full_attention[li]:
                stride = c.attn_proj_rows
                self.mat(st, L + "qkv", xn, h, proj, stride)
                ap = self.attn_p()
                kc, vc = self.kc[full_slot], self.vc[full_slot]
                wr.attn_prep(st, ap, proj, qbuf, kc, vc, self.f(L + "qk_norm"), rpos)
                wr.attend(st, ap, proj, qbuf, kc, vc, attn_out, partial)
                if parts > 1:
                    wr.attn_combine(st, ap, proj, partial, attn_out)
                self.mat(st, L + "o_proj", attn_out, c.q_dim, branch, h)
                full_slot += 1
            else:
                stride = c.lin_proj_rows
                self.mat(st, L + "in_proj", xn, h, proj, stride)
                lp = LinP(c.conv_dim, stride, c.lin_k_heads, c.lin_v_heads, c.eps, (0, 0, 0))
                lw = self.f(L + "lin")
                ck = np.zeros_like(self.conv[lin_slot])
                sk = np.zeros_like(self.state[lin_slot])
                wr.conv(st, lp, proj, act, self.conv[lin_slot], lw, ck)
                wr.delta(st, lp, proj, act, self.state[lin_slot], lw, attn_out, sk)
                self.mat(st, L + "out_proj", attn_out, c.lin_value_dim, branch, h)
                lin_slot += 1
            wr.merge(st, self.layer_p(1 if mhc else 0), x, coef, branch)
            push_norm(self.f(L + "mhc_ffn") if mhc else None, self.f(L + "post_ln"))
            self.mat(st, L + "gate_up", xn, h, proj, 2 * c.intermediate)
            wr.swiglu(st, self.layer_p(0), proj, act)
            self.mat(st, L + "down", act, c.intermediate, branch, h)
            mode = 0 if not mhc else (2 if li + 1 == mhc_end else 1)
            wr.merge(st, self.layer_p(mode), x, coef, branch)
        # final norm into rows 1..m of hid (row 0: the previous step's last hidden row), head
        hid = np.zeros((m + 1) * h, np.float32)
        hid[:h] = self.hlast
        out_rows = np.zeros(m * h, np.float32)
        wr.branch_norm(st, self.layer_p(0), x, coef, self.f("norm"), out_rows, m)
        hid[h:] = out_rows
        logits = None
        if want_logits:
            logits = np.zeros(c.vocab, np.float32)
            self.mat(st, "lm_head", hid, h, logits, c.vocab, m_one=1, x_off=m * h)
        self.hlast = hid[m * h:(m + 1) * h].copy()
        self.hid, self.hid_rows = hid, m
        self.pos += m
        return logits

    def mtp(self, r0: int, tokens, pos, slot0: int, draft: bool):
        """Engine::mtp: pairs (hidden row r0 + i of the last step, tokens[i]) into MTP cache
        slots slot0.., rotary positions pos [n][3]; with draft, the MTP's logits and argmax."""
        c, h = self.cfg, self.cfg.hidden
        n = len(tokens)
        assert n and r0 + n <= self.hid_rows + 1
        logits = None
        for c0 in range(0, n, CHUNK):
            c1 = min(c0 + CHUNK, n)
            m = c1 - c0
            total = slot0 + c1
            parts = min(max(-(-total // 256), 1), 64) if m <= 4 else 1
            st = StepU(m, slot0 + c0, parts, 0)
            mx = self.embed(tokens[c0:c1])
            rpos = np.array([[p[0], p[1], p[2], 0] for p in pos[c0:c1]], np.uint32).reshape(-1).copy()
            p0 = self.layer_p(0)
            coef = np.zeros(m * 8, np.float32)
            xn = np.zeros(m * h, np.float32)
            hn = np.zeros(m * h, np.float32)
            branch = np.zeros(m * h, np.float32)
            proj = np.zeros(m * max(c.attn_proj_rows, 2 * c.intermediate), np.float32)
            act = np.zeros(m * c.intermediate, np.float32)
            qbuf = np.zeros(m * c.q_dim, np.float32)
            attn_out = np.zeros(m * c.q_dim, np.float32)
            partial = np.zeros(m * c.n_heads * parts * 258, np.float32)
            wr.branch_norm(st, p0, mx, coef, self.f("mtp.norm_e"), xn, m)  # pre (engine.rs:527)
            ph = self.layer_p(0)
            ph.x_stride = h
            rows = np.ascontiguousarray(self.hid[(r0 + c0) * h:(r0 + c0 + m) * h])
            wr.branch_norm(st, ph, rows, coef, self.f("mtp.norm_h"), hn, m)  # norm_h (engine.rs:736-747)
            # engine.rs:549-566
            self.mat(st, "mtp.fc_e", xn, h, mx, 2 * h)
            self.mat(st, "mtp.fc_h", hn, h, branch, h)
            wr.merge(st, p0, mx, coef, branch)
            wr.branch_norm(st, p0, mx, coef, self.f("mtp.in_ln"), xn, m)
            self.mat(st, "mtp.qkv", xn, h, proj, c.attn_proj_rows)
            ap = self.attn_p()
            wr.attn_prep(st, ap, proj, qbuf, self.mkc, self.mvc, self.f("mtp.qk_norm"), rpos)
            wr.attend(st, ap, proj, qbuf, self.mkc, self.mvc, attn_out, partial)
            if parts > 1:
                wr.attn_combine(st, ap, proj, partial, attn_out)
            self.mat(st, "mtp.o_proj", attn_out, c.q_dim, branch, h)
            wr.merge(st, p0, mx, coef, branch)
            wr.branch_norm(st, p0, mx, coef, self.f("mtp.post_ln"), xn, m)
            self.mat(st, "mtp.gate_up", xn, h, proj, 2 * c.intermediate)
            wr.swiglu(st, p0, proj, act)
            self.mat(st, "mtp.down", act, c.intermediate, branch, h)
            wr.merge(st, p0, mx, coef, branch)
            if c1 == n and draft:  # head (engine.rs:567-570): the last row, lm_head
                wr.branch_norm(st, self.layer_p(0, True), mx, coef, self.f("mtp.norm"), xn, 1)
                logits = np.zeros(c.vocab, np.float32)
                self.mat(st, "lm_head", xn, h, logits, c.vocab, m_one=1)
        return logits


class RefVision:
    """Vision::encode (src/vision.rs:195-343) over the reference's vision.wgsl and matmul
    kernels (translated), on an oracle vision tower's weights: the op order of
    vision.rs:252-290 per frame, the position embedding of :160-193 on the host in f32."""

    EPS, GELU_TANH, GELU_ERF = 1e-6, 1, 2  # vision.rs:53-55

    def __init__(self, cfg, tower):
        self.cfg, self.t = cfg, tower

    def f(self, name):
        return self.t.tensor(name)[1]

    def mat(self, name, x, rows, y, y_stride):
        """mat_ops (vision.rs:345-380): x_stride = the weight's k, one chunk."""
        dt, q, s, n, k = self.t.tensor(name)
        wr.mat(dt, StepU(rows, 0, 1, 0), MatP(n, k, 0, k, 0, y_stride, 0, 0), x, q.view(np.uint8), s, y)

    def pos_embed(self, h, w):
        c = self.cfg
        side, hid, m = c.pos_side, c.hidden, c.merge
        f32 = np.float32

        def lin(n):
            return [f32(0) if n == 1 else f32(f32(side - 1) * f32(i)) / f32(n - 1) for i in range(n)]

        hs, ws = lin(h), lin(w)
        pos = self.f("v.pos")
        out = np.zeros((h * w, hid), np.float32)
        for token in range(h * w):
            blk, intra = token // (m * m), token % (m * m)
            r = (blk // (w // m)) * m + intra // m
            cc = (blk % (w // m)) * m + intra % m
            fh, fw = int(hs[r]), int(ws[cc])
            ch, cw = min(fh + 1, side - 1), min(fw + 1, side - 1)
            dh, dw = f32(hs[r] - f32(fh)), f32(ws[cc] - f32(fw))
            one = f32(1)
            corners = [(fh * side + fw, f32((one - dh) * (one - dw))), (fh * side + cw, f32((one - dh) * dw)),
                       (ch * side + fw, f32(dh * (one - dw))), (ch * side + cw, f32(dh * dw))]
            for idx, wt in corners:
                out[token] = out[token] + pos[idx * hid:(idx + 1) * hid] * wt
        return out.reshape(-1)

    def encode(self, patches, frames, h, w):
        c = self.cfg
        n, hid = h * w, c.hidden
        nq = n // (c.merge * c.merge)
        pd = 3 * c.temporal_patch * c.patch * c.patch
        md, ip = hid * c.merge * c.merge, c.intermediate_padded
        pos = self.pos_embed(h, w)
        x = np.zeros(n * hid, np.float32)
        xn, tmp, att = np.zeros_like(x), np.zeros_like(x), np.zeros_like(x)
        qkv = np.zeros(max(n * 3 * hid, nq * c.out_hidden), np.float32)
        mlp = np.zeros(max(n * ip, nq * md), np.float32)

        def norm(wname):
            xn[:] = wr.vis_layer_norm(VisP(n, hid, 0, 0, self.EPS, 0, 0, 0), x, self.f(wname))

        def epi(a, b, bname, e, rows, cols, mode, act):
            wr.vis_epilogue(VisP(rows, cols, mode, act, 0.0, 0, 0, 0), a, b, self.f(bname), e)

        out = []
        for fr in range(frames):
            pin = np.ascontiguousarray(patches.reshape(-1)[fr * n * pd:(fr + 1) * n * pd], np.float32)
            self.mat("v.patch", pin, n, tmp, hid)
            epi(tmp, x, "v.patch_b", pos, n, hid, 2, 0)
            for i in range(c.depth):
                b = f"v{i}."
                norm(b + "n1")
                self.mat(b + "qkv", xn, n, qkv, 3 * hid)
                epi(qkv, None, b + "qkv_b", None, n, 3 * hid, 0, 0)
                rp = VisP(n, 0, 0, 0, 0.0, w, c.n_heads, 0)
                wr.vis_rope(rp, qkv)
                att[:] = wr.vis_attend(rp, qkv[:n * 3 * hid]).reshape(-1)
                self.mat(b + "proj", att, n, tmp, hid)
                epi(tmp, x, b + "proj_b", None, n, hid, 1, 0)
                norm(b + "n2")
                self.mat(b + "fc1", xn, n, mlp, ip)
                epi(mlp, None, b + "fc1_b", None, n, ip, 0, self.GELU_TANH)
                self.mat(b + "fc2", mlp, n, tmp, hid)
                epi(tmp, x, b + "fc2_b", None, n, hid, 1, 0)
            norm("vm.norm")
            self.mat("vm.fc1", xn, nq, mlp, md)
            epi(mlp, None, "vm.fc1_b", None, nq, md, 0, self.GELU_ERF)
            self.mat("vm.fc2", mlp, nq, qkv, c.out_hidden)
            epi(qkv, None, "vm.fc2_b", None, nq, c.out_hidden, 0, 0)
            out.append(qkv[:nq * c.out_hidden].copy())
        return np.concatenate(out).reshape(frames * nq, c.out_hidden)
