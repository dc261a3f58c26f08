"""The CUDA kernels against the committed golden vectors of the reference's own kernels
(tests/golden/reference_kernels.npz: the reference's WGSL run on the host cores), through
the C ABI, on the same hash-generated inputs. The bar is the one BASELINE.json states:
fp32 results within 1e-3 relative error (max |gpu - reference| / max |reference|); the
V cache and the conv state, which the kernels store without arithmetic, bit-exact.
"""
import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from sensenova_b200 import ffi

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import golden_cases as G  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-3  # fp32 accumulate within 1e-3 relative error per kernel
EXACT = {("attn_prep", "vc"), ("conv", "conv_state"), ("conv", "conv_ckpt")}

FIXTURE = np.load(GOLDEN / "reference_kernels.npz")
META = json.loads(FIXTURE["meta"].tobytes().decode())


class Cuda:
    """The kernel-level C ABI behind the oracle's call shapes: numpy buffers in, the same
    buffers updated in place, device memory only for the duration of a call."""

    def __init__(self, torch, lib):
        self.T, self.lib = torch, lib

    def _run(self, fn, *args):
        devs, outs = [], []
        conv = []
        for a in args:
            if isinstance(a, np.ndarray):
                view = a.view(np.int32) if a.dtype == np.uint32 else a
                t = self.T.from_numpy(np.ascontiguousarray(view)).cuda()
                devs.append(t)
                outs.append((a, t))
                conv.append(C.c_void_p(t.data_ptr()))
            elif a is None:
                conv.append(None)
            else:
                conv.append(a)
        ffi.check(fn(*conv, None))
        self.T.cuda.synchronize()
        for a, t in outs:
            a[...] = t.cpu().numpy().view(a.dtype).reshape(a.shape)

    def mat(self, dtype, st, p, x, q, s, y):
        self._run(self.lib.snl_mat, dtype, C.byref(st), C.byref(p), x, q, s, y)

    def branch_norm(self, st, p, x, coef, w, out, n_groups):
        self._run(lambda *a: self.lib.snl_branch_norm(*a[:6], n_groups, a[6]), C.byref(st), C.byref(p), x, coef, w, out)

    def mhc_dots(self, st, p, x, w, raw):
        self._run(self.lib.snl_mhc_dots, C.byref(st), C.byref(p), x, w, raw)

    def mhc_finish(self, st, p, raw, w, coef):
        self._run(self.lib.snl_mhc_finish, C.byref(st), C.byref(p), raw, w, coef)

    def merge(self, st, p, x, coef, br):
        self._run(self.lib.snl_merge, C.byref(st), C.byref(p), x, coef, br)

    def swiglu(self, st, p, gu, act):
        self._run(self.lib.snl_swiglu, C.byref(st), C.byref(p), gu, act)

    def attn_prep(self, st, p, proj, qbuf, kc, vc, norms, rpos):
        self._run(self.lib.snl_attn_prep, C.byref(st), C.byref(p), proj, qbuf, kc, vc, norms, rpos)

    def attend(self, st, p, proj, qbuf, kc, vc, out, partial):
        self._run(self.lib.snl_attend, C.byref(st), C.byref(p), proj, qbuf, kc, vc, out, partial)

    def attn_combine(self, st, p, proj, partial, out):
        self._run(self.lib.snl_attn_combine, C.byref(st), C.byref(p), proj, partial, out)

    def conv(self, st, p, proj, conv_out, conv_state, lw, conv_ckpt):
        self._run(self.lib.snl_conv, C.byref(st), C.byref(p), proj, conv_out, conv_state, lw, conv_ckpt)

    def delta(self, st, p, proj, conv_out, state, lw, out, state_ckpt):
        self._run(self.lib.snl_delta, C.byref(st), C.byref(p), proj, conv_out, state, lw, out, state_ckpt)

    def vis_layer_norm(self, p, a, w):
        b = np.zeros_like(a)
        self._run(self.lib.snl_vis_layer_norm, C.byref(p), a, b, w)
        return b

    def vis_epilogue(self, p, a, b, w, e=None):
        self._run(self.lib.snl_vis_epilogue, C.byref(p), a, b, w, e)

    def vis_rope(self, p, qkv):
        self._run(self.lib.snl_vis_rope, C.byref(p), qkv)

    def vis_attend(self, p, qkv):
        out = np.zeros((p.rows * p.heads * 72,), np.float32)
        self._run(self.lib.snl_vis_attend, C.byref(p), qkv, out)
        return out


@pytest.fixture(scope="module")
def cuda(torch_cuda, lib):
    return Cuda(torch_cuda, lib)


@pytest.mark.parametrize("name,kernel,a", G.CASES, ids=[c[0] for c in G.CASES])
def test_cuda_matches_reference_golden(cuda, name, kernel, a):
    outs = G.run(name, kernel, a, cuda)
    for k, v in outs.items():
        m = META[name]["outputs"][k]
        got = np.ascontiguousarray(v).reshape(-1)[:: m["stride"]]
        want = FIXTURE[f"{name}/{k}"]
        if (kernel, k) in EXACT:
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{name}/{k} not bit-exact"
        elif k in ("kc",):
            g16 = got.view(np.float16).astype(np.float64)
            w16 = want.view(np.float16).astype(np.float64)
            assert np.abs(g16 - w16).max() / np.abs(w16).max() < TOL, f"{name}/{k}"
        else:
            err = np.abs(got.astype(np.float64) - want).max() / max(np.abs(want).max(), 1e-30)
            assert err < TOL, f"{name}/{k}: relative error {err:.3g}"
