"""The vision tower on the GPU against the oracle: each vision.wgsl kernel through its
C ABI entry point, and the whole encode (fused encoder kernels, the tcgen05 GEMM for
frames of >= 8 patches) on the small tower. Bar: 1e-3 relative error per kernel, and
for the encode of a two-block tower."""
import ctypes as C

import numpy as np
import pytest

import oracle as orc
from sensenova_b200 import ffi
from sensenova_b200.ffi import VisP
from sensenova_b200.vision import Vision, VisionConfig, small_vision

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def dev(T, a):
    return T.from_numpy(np.ascontiguousarray(a)).cuda()


def host(T, t):
    T.cuda.synchronize()
    return t.cpu().numpy()


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("rows,cols", [(1, 288), (37, 1152), (200, 4608)])
def test_layer_norm(torch_cuda, lib, rows, cols):
    T = torch_cuda
    rng = np.random.default_rng(rows)
    a = (rng.standard_normal((rows, cols)) * 2 + 0.5).astype(np.float32)
    w = rng.standard_normal(2 * cols).astype(np.float32)
    p = VisP(rows, cols, 0, 0, 1e-6, 0, 0, 0)
    da, db, dw = dev(T, a), T.zeros((rows, cols), device="cuda"), dev(T, w)
    ffi.check(lib.snl_vis_layer_norm(C.byref(p), ptr(da), ptr(db), ptr(dw), None))
    assert rel(host(T, db), orc.vis_layer_norm(p, a, w)) < TOL


@pytest.mark.parametrize("mode,act", [(0, 0), (0, 1), (0, 2), (1, 0), (2, 0), (2, 1)])
@pytest.mark.parametrize("rows,cols", [(5, 224), (33, 4320), (3, 13)])
def test_epilogue(torch_cuda, lib, mode, act, rows, cols):
    T = torch_cuda
    rng = np.random.default_rng(mode * 10 + act)
    a = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    b = rng.standard_normal((rows, cols)).astype(np.float32)
    e = rng.standard_normal((rows, cols)).astype(np.float32)
    w = rng.standard_normal(cols).astype(np.float32)
    p = VisP(rows, cols, mode, act, 0, 0, 0, 0)
    da, db, de, dw = dev(T, a), dev(T, b), dev(T, e), dev(T, w)
    ffi.check(lib.snl_vis_epilogue(C.byref(p), ptr(da), ptr(db), ptr(dw), ptr(de), None))
    ra, rb = a.copy(), b.copy()
    orc.vis_epilogue(p, ra, rb, w, e)
    if mode == 0:
        assert rel(host(T, da), ra) < TOL
    else:
        assert rel(host(T, db), rb) < TOL


@pytest.mark.parametrize("n,grid_w,heads", [(4, 2, 4), (24, 6, 4), (64, 16, 16), (200, 20, 4)])
def test_rope_and_attend(torch_cuda, lib, n, grid_w, heads):
    T = torch_cuda
    rng = np.random.default_rng(n)
    qkv = rng.standard_normal((n, 3 * heads * 72)).astype(np.float32)
    p = VisP(n, 0, 0, 0, 0, grid_w, heads, 0)
    dq = dev(T, qkv)
    ffi.check(lib.snl_vis_rope(C.byref(p), ptr(dq), None))
    want = qkv.copy()
    orc.vis_rope(p, want)
    got = host(T, dq)
    assert rel(got, want) < TOL
    out = T.zeros((n, heads * 72), device="cuda")
    ffi.check(lib.snl_vis_attend(C.byref(p), ptr(dev(T, want)), ptr(out), None))
    assert rel(host(T, out), orc.vis_attend(p, want)) < TOL


@pytest.mark.parametrize("frames,h,w", [(1, 2, 2), (2, 4, 6), (1, 16, 12)])
def test_encode_matches_oracle(torch_cuda, frames, h, w):
    cfg = small_vision()
    rng = np.random.default_rng(h * w)
    patches = rng.standard_normal((frames, h * w, cfg.patch_dim())).astype(np.float32)
    ov = orc.OracleVision(cfg, seed=5)
    want = ov.encode(patches, frames, h, w)
    v = Vision.synthetic(cfg, seed=5)
    got = v.encode(patches, frames, h, w)
    assert got.shape == want.shape
    assert rel(got, want) < TOL, rel(got, want)
    v.close()
    ov.close()


def test_set_tensor_gives_the_synthetic_tower(torch_cuda):
    """Weights loaded by name (the .snl path) give the same features as the tower
    generated on the device."""
    cfg = small_vision()
    ov = orc.OracleVision(cfg, seed=8)
    loaded = Vision(cfg)
    names = ["v.patch", "v.patch_b", "v.pos", "vm.norm", "vm.fc1", "vm.fc1_b", "vm.fc2", "vm.fc2_b"]
    for i in range(cfg.depth):
        names += [f"v{i}.{k}" for k in ("n1", "n2", "qkv", "qkv_b", "proj", "proj_b", "fc1", "fc1_b", "fc2", "fc2_b")]
    for nm in names:
        dt, q, s, rows, cols = ov.tensor(nm)
        loaded.set_tensor(nm, q, s, rows, cols)
    loaded.finalize()
    synth = Vision.synthetic(cfg, seed=8)
    patches = np.random.default_rng(2).standard_normal((1, 8 * 8, cfg.patch_dim())).astype(np.float32)
    assert np.array_equal(loaded.encode(patches, 1, 8, 8), synth.encode(patches, 1, 8, 8))
    loaded.close()
    synth.close()
    ov.close()


def test_vision_errors(torch_cuda):
    with pytest.raises(ffi.SnlError, match="head_dim 72"):
        Vision(VisionConfig(hidden=256, n_heads=4))
    v = Vision.synthetic(small_vision())
    with pytest.raises(ffi.SnlError, match="wrong shape"):
        v.encode(np.zeros((1, 3 * 4, v.cfg.patch_dim()), np.float32), 1, 3, 4)
    with pytest.raises(ffi.SnlError):
        v.set_tensor("v.nothing", np.zeros(4, np.float32))
    v.close()
