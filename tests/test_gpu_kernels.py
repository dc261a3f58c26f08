"""Parity of every CUDA kernel with the CPU oracle, through the C ABI.

Inputs are seeded; device buffers are torch tensors (plumbing only). The bar is the
one BASELINE.json states: fp32 results within 1e-3 relative error per kernel
(max |gpu - oracle| / max |oracle|); quantized values and argmax indices bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

from sensenova_b200 import ffi
from sensenova_b200.ffi import AttnP, LayerP, LinP, MatP, StepU, SNL_Q4_0, SNL_Q8_0

pytestmark = pytest.mark.gpu
TOL = 1e-3  # fp32 accumulate within 1e-3 relative error per kernel


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def T(torch_cuda):
    return torch_cuda


_keep = []  # device tensors stay alive until the test's kernels have run


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    import torch

    torch.cuda.synchronize()
    _keep.clear()


def dev(T, a):
    t = T.from_numpy(np.ascontiguousarray(a)).cuda()
    _keep.append(t)
    return t


def host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def call(rc):
    ffi.check(rc)


# ---- synthetic generator: device == host, bit for bit --------------------------------


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
def test_synth_quant_bit_exact(T, lib, orc, dtype):
    rows, cols = 300, 1024
    q_ref, s_ref = orc.gen_quant(42, "l3.gate_up", dtype, rows, cols)
    q = T.empty(q_ref.size, dtype=T.uint8, device="cuda")
    s = T.empty(s_ref.size, dtype=T.float32, device="cuda")
    call(lib.snl_synth_quant(42, b"l3.gate_up", dtype, rows, cols, ptr(q), ptr(s), None))
    assert np.array_equal(host(q), q_ref)
    assert np.array_equal(host(s).view(np.uint32), s_ref.view(np.uint32))
    # fp16-exact scales (the benchmark's "fp16 scale per block")
    assert np.array_equal(s_ref.astype(np.float16).astype(np.float32), s_ref)


def test_synth_f32_bit_exact(T, lib, orc):
    ref = orc.gen_f32(9, "l0.lin", 3, 5000, 0.1, 1.0)
    out = T.empty(5000, dtype=T.float32, device="cuda")
    call(lib.snl_synth_f32(9, b"l0.lin", 3, 5000, 0.1, 1.0, ptr(out), None))
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))


# ---- matmul.wgsl -------------------------------------------------------------------


def run_mat(T, lib, orc, dtype, n, k, m, x_stride=None, y_stride=None, x_off=0, m_one=0, seed=0):
    rng = np.random.default_rng(seed)
    q, s = orc.gen_quant(seed + 1, "w", dtype, n, k)
    xs = x_stride or k
    ys = y_stride or n
    rows = m_one or m
    x = rng.standard_normal(x_off + max(rows, 1) * xs).astype(np.float32)
    y_ref = np.zeros(rows * ys, dtype=np.float32)
    p = MatP(n, k, x_off, xs, 0, ys, 0, m_one)
    st = StepU(m, 0, 1, 0)
    orc.mat(dtype, st, p, x, q, s, y_ref)
    yd = T.zeros(rows * ys, dtype=T.float32, device="cuda")
    call(lib.snl_mat(dtype, C.byref(st), C.byref(p), ptr(dev(T, x)), ptr(dev(T, q)), ptr(dev(T, s)), ptr(yd), None))
    return host(yd), y_ref


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 64, 130])
def test_mat_rows(T, lib, orc, dtype, m):
    y, ref = run_mat(T, lib, orc, dtype, 200, 1024, m, seed=m)
    assert rel(y, ref) < TOL


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("n,k,m", [(1000, 2048, 256), (1000, 2048, 300), (4096, 4096, 512), (333, 160, 40), (18944, 256, 300),
                                   (12288, 4096, 512)])
def test_mat_prefill_tensor_cores(T, lib, orc, dtype, n, k, m):
    """Prefill rows (m >= 8) run on the tcgen05 GEMM: several token and row tiles, a
    partial last K block (k = 160), against the oracle's f32 GEMM. 12288 x 4096 at 512
    rows is a prefill step's own shape (192-token tiles with weight planes)."""
    y, ref = run_mat(T, lib, orc, dtype, n, k, m, seed=n + m)
    assert rel(y, ref) < TOL
    # Three fp16 hi/lo products; the tensor cores' fp32 accumulation over K leaves
    # ~2e-5 at k = 4096, fifty times inside the bar.
    assert rel(y, ref) < 1e-4


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("n,k,m", [(1000, 2048, 300), (4096, 4096, 512), (333, 160, 40), (18944, 256, 300),
                                   (12288, 4096, 512), (10240, 4096, 400)])
def test_mat_weight_planes_bitwise(T, lib, dtype, n, k, m, orc):
    """Prefill GEMM with precomputed weight planes (A by TMA) == the dequantizing GEMM,
    bit for bit: the same operand values and MMA order over K, whatever the token tile
    (the planes kernel takes 192-token tiles at 12288 x 4096 x 512 and 10240 x 4096 x 400,
    the dequantizing one 256)."""
    rng = np.random.default_rng(n + k + m)
    q, s = orc.gen_quant(n + 3, "wp", dtype, n, k)
    x = rng.standard_normal(m * k).astype(np.float32)
    p, st = MatP(n, k, 0, k, 0, n, 0, 0), StepU(m, 0, 1, 0)
    qd, sd, xd = dev(T, q), dev(T, s), dev(T, x)
    planes = T.empty(2 * n * k, dtype=T.float16, device="cuda")
    call(lib.snl_weight_planes(dtype, n, k, ptr(qd), ptr(sd), ptr(planes), None))
    y0 = T.zeros(m * n, dtype=T.float32, device="cuda")
    y1 = T.zeros(m * n, dtype=T.float32, device="cuda")
    call(lib.snl_mat(dtype, C.byref(st), C.byref(p), ptr(xd), ptr(qd), ptr(sd), ptr(y0), None))
    call(lib.snl_mat_wplanes(dtype, C.byref(st), C.byref(p), ptr(xd), ptr(qd), ptr(sd), ptr(planes), ptr(y1), None))
    assert np.array_equal(host(y0), host(y1))


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
def test_mat_config1_shape(T, lib, orc, dtype):
    # The benchmark GEMV: W [12288 x 4096], one token.
    y, ref = run_mat(T, lib, orc, dtype, 12288, 4096, 1, seed=5)
    assert rel(y, ref) < TOL
    assert rel(y, ref) < 1e-5  # well inside the bar: same fp32 math, another order


@pytest.mark.parametrize("n", [1, 5, 33, 127])
def test_mat_ragged_rows(T, lib, orc, n):
    for m in (1, 2, 11):
        y, ref = run_mat(T, lib, orc, SNL_Q8_0, n, 96, m, seed=n)
        assert rel(y, ref) < TOL


def test_mat_strides_offsets(T, lib, orc):
    # head-style call: x_off picks the last rows, m_one fixes the count, y strided
    y, ref = run_mat(T, lib, orc, SNL_Q8_0, 64, 256, 5, x_stride=256, y_stride=80, x_off=4 * 256, m_one=2, seed=3)
    assert rel(y, ref) < TOL


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("n,k", [(200, 1024), (37, 96), (12288, 4096), (4096, 12288)])
def test_mat_tensor_core(T, lib, orc, dtype, m, n, k):
    """The tensor-core GEMV (x as fp16 hi/lo planes) against the oracle's matvec."""
    rng = np.random.default_rng(n + k + m)
    q, s = orc.gen_quant(n + m, "wtc", dtype, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = np.zeros((m, n), np.float32)
    orc.mat(dtype, StepU(m, 0, 1, 0), MatP(n, k, 0, k, 0, n, 0, 0), x, q, s, ref)
    planes = T.empty(2 * m * k, dtype=T.float16, device="cuda")
    call(lib.snl_xpack(ptr(dev(T, x)), m, k, k, ptr(planes), None))
    y = T.zeros((m, n), device="cuda")
    p = MatP(n, k, 0, k, 0, n, 0, 0)
    call(lib.snl_mat_xpack(dtype, C.byref(p), m, ptr(planes), ptr(dev(T, q)), ptr(dev(T, s)), ptr(y), None))
    err = rel(host(y), ref)
    assert err < TOL and err < 2e-5, err


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("n,k", [(200, 1024), (37, 96), (12288, 4096), (4096, 12288), (33, 160)])
def test_mat_tiles(T, lib, orc, dtype, m, n, k):
    """Tile-layout repack + the tile GEMV (the engine's decode path) against the oracle."""
    rng = np.random.default_rng(n * 3 + k + m)
    q, s = orc.gen_quant(n + 7 * m, "wtile", dtype, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = np.zeros((m, n), np.float32)
    orc.mat(dtype, StepU(m, 0, 1, 0), MatP(n, k, 0, k, 0, n, 0, 0), x, q, s, ref)
    tb, sf = C.c_size_t(), C.c_size_t()
    call(lib.snl_tile_sizes(dtype, n, k, C.byref(tb), C.byref(sf)))
    tiles = T.empty(tb.value, dtype=T.uint8, device="cuda")
    ts = T.empty(sf.value, dtype=T.uint8, device="cuda")
    f16 = C.c_int(-1)
    call(lib.snl_tile_repack(dtype, n, k, ptr(dev(T, q)), ptr(dev(T, s)), ptr(tiles), ptr(ts), C.byref(f16), None))
    assert f16.value == 1  # the synthetic block scales are fp16 numbers
    planes = T.empty(2 * m * k, dtype=T.float16, device="cuda")
    call(lib.snl_xpack(ptr(dev(T, x)), m, k, k, ptr(planes), None))
    y = T.zeros((m, n), device="cuda")
    p = MatP(n, k, 0, k, 0, n, 0, 0)
    call(lib.snl_mat_tiles(dtype, C.byref(p), m, ptr(planes), ptr(tiles), ptr(ts), f16.value, ptr(y), None))
    err = rel(host(y), ref)
    assert err < TOL and err < 2e-5, err


@pytest.mark.parametrize("dtype", [SNL_Q8_0, SNL_Q4_0])
def test_tile_scales_f32_mode(T, lib, orc, dtype):
    """Block scales that are not fp16 numbers (as a converter computing them in f32
    writes) keep the tile layout's f32 scale mode: same results as the file layout."""
    n, k, m = 300, 1024, 2
    rng = np.random.default_rng(41)
    q, s = orc.gen_quant(9, "wtile", dtype, n, k)
    s = (s * np.float32(1.0 + 1e-3)).astype(np.float32)  # off the fp16 grid
    s.flat[0] = np.float32(0.1)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = np.zeros((m, n), np.float32)
    orc.mat(dtype, StepU(m, 0, 1, 0), MatP(n, k, 0, k, 0, n, 0, 0), x, q, s, ref)
    tb, sb = C.c_size_t(), C.c_size_t()
    call(lib.snl_tile_sizes(dtype, n, k, C.byref(tb), C.byref(sb)))
    assert sb.value == ((n + 15) // 16) * ((k // 32 + 3) // 4) * 64 * 4
    tiles = T.empty(tb.value, dtype=T.uint8, device="cuda")
    ts = T.empty(sb.value, dtype=T.uint8, device="cuda")
    f16 = C.c_int(-1)
    call(lib.snl_tile_repack(dtype, n, k, ptr(dev(T, q)), ptr(dev(T, s)), ptr(tiles), ptr(ts), C.byref(f16), None))
    assert f16.value == 0
    planes = T.empty(2 * m * k, dtype=T.float16, device="cuda")
    call(lib.snl_xpack(ptr(dev(T, x)), m, k, k, ptr(planes), None))
    y = T.zeros((m, n), device="cuda")
    call(lib.snl_mat_tiles(dtype, C.byref(MatP(n, k, 0, k, 0, n, 0, 0)), m, ptr(planes), ptr(tiles), ptr(ts), 0,
                           ptr(y), None))
    err = rel(host(y), ref)
    assert err < TOL and err < 2e-5, err


def test_mat_tensor_core_wide_range(T, lib, orc):
    # |x| up to ~5e4: the 1/16 pre-scale keeps the fp16 planes finite and accurate.
    rng = np.random.default_rng(77)
    n, k = 256, 2048
    q, s = orc.gen_quant(5, "wide", SNL_Q8_0, n, k)
    x = (rng.standard_normal((1, k)) * np.exp(rng.uniform(-8, 10, (1, k)))).astype(np.float32)
    ref = np.zeros((1, n), np.float32)
    orc.mat(SNL_Q8_0, StepU(1, 0, 1, 0), MatP(n, k, 0, k, 0, n, 0, 0), x, q, s, ref)
    planes = T.empty(2 * k, dtype=T.float16, device="cuda")
    call(lib.snl_xpack(ptr(dev(T, x)), 1, k, k, ptr(planes), None))
    y = T.zeros((1, n), device="cuda")
    p = MatP(n, k, 0, k, 0, n, 0, 0)
    call(lib.snl_mat_xpack(SNL_Q8_0, C.byref(p), 1, ptr(planes), ptr(dev(T, q)), ptr(dev(T, s)), ptr(y), None))
    assert rel(host(y), ref) < TOL


def test_mat_rejects_misaligned(T, lib):
    st, p = StepU(1, 0, 1, 0), MatP(8, 32, 2, 32, 0, 8, 0, 0)
    buf = T.zeros(1024, device="cuda")
    rc = lib.snl_mat(SNL_Q8_0, C.byref(st), C.byref(p), ptr(buf), ptr(buf), ptr(buf), ptr(buf), None)
    assert rc == -1 and b"multiples of 4" in lib.snl_last_error()


# ---- layers.wgsl --------------------------------------------------------------------


def lp(h, mode=0, last_row=0, inter=0, x_stride=0):
    return LayerP(h, mode, last_row, 1e-6, 1.0, 20, inter, x_stride)


@pytest.mark.parametrize("mode", [0, 1])
def test_branch_norm(T, lib, orc, mode):
    rng = np.random.default_rng(mode)
    m, h = 7, 4096
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0.1, 1, (m, 8)).astype(np.float32)
    w = (0.1 * rng.standard_normal(h)).astype(np.float32)
    ref = np.zeros((m, h), np.float32)
    st, p = StepU(m, 0, 1, 0), lp(h, mode)
    orc.branch_norm(st, p, x, coef, w, ref, m)
    out = T.zeros((m, h), device="cuda")
    call(lib.snl_branch_norm(C.byref(st), C.byref(p), ptr(dev(T, x)), ptr(dev(T, coef)), ptr(dev(T, w)), ptr(out), m, None))
    assert rel(host(out), ref) < TOL


def test_branch_norm_last_row(T, lib, orc):
    rng = np.random.default_rng(2)
    m, h = 5, 512
    x = rng.standard_normal((m, h)).astype(np.float32)
    w = (0.1 * rng.standard_normal(h)).astype(np.float32)
    st, p = StepU(m, 0, 1, 0), lp(h, 0, last_row=1, x_stride=h)
    ref = np.zeros(h, np.float32)
    orc.branch_norm(st, p, x, None, w, ref, 1)
    out = T.zeros(h, device="cuda")
    call(lib.snl_branch_norm(C.byref(st), C.byref(p), ptr(dev(T, x)), None, ptr(dev(T, w)), ptr(out), 1, None))
    assert rel(host(out), ref) < TOL


def test_mhc(T, lib, orc):
    rng = np.random.default_rng(3)
    m, h = 3, 4096
    d = 2 * h
    x = rng.standard_normal((m, d)).astype(np.float32)
    w = np.concatenate([0.02 * rng.standard_normal(8 * d), 0.1 * rng.standard_normal(8)]).astype(np.float32)
    st, p = StepU(m, 0, 1, 0), lp(h)
    raw_ref = np.zeros((m, 9), np.float32)
    coef_ref = np.zeros((m, 8), np.float32)
    orc.mhc_dots(st, p, x, w, raw_ref)
    orc.mhc_finish(st, p, raw_ref, w, coef_ref)
    raw = T.zeros((m, 9), device="cuda")
    coef = T.zeros((m, 8), device="cuda")
    xd, wd = dev(T, x), dev(T, w)
    call(lib.snl_mhc_dots(C.byref(st), C.byref(p), ptr(xd), ptr(wd), ptr(raw), None))
    call(lib.snl_mhc_finish(C.byref(st), C.byref(p), ptr(raw), ptr(wd), ptr(coef), None))
    assert rel(host(raw), raw_ref) < TOL
    assert rel(host(coef), coef_ref) < TOL


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_merge(T, lib, orc, mode):
    rng = np.random.default_rng(mode)
    m, h = 3, 4096
    x = rng.standard_normal((m, 2 * h)).astype(np.float32)
    coef = rng.uniform(0, 1, (m, 8)).astype(np.float32)
    br = rng.standard_normal((m, h)).astype(np.float32)
    st, p = StepU(m, 0, 1, 0), lp(h, mode)
    xr = x.copy()
    orc.merge(st, p, xr, coef, br)
    xd = dev(T, x)
    call(lib.snl_merge(C.byref(st), C.byref(p), ptr(xd), ptr(dev(T, coef)), ptr(dev(T, br)), None))
    assert rel(host(xd), xr) < TOL


def test_swiglu(T, lib, orc):
    rng = np.random.default_rng(4)
    m, inter = 4, 12288
    gu = rng.standard_normal((m, 2 * inter)).astype(np.float32)
    st, p = StepU(m, 0, 1, 0), lp(4096, inter=inter)
    ref = np.zeros((m, inter), np.float32)
    orc.swiglu(st, p, gu, ref)
    out = T.zeros((m, inter), device="cuda")
    call(lib.snl_swiglu(C.byref(st), C.byref(p), ptr(dev(T, gu)), ptr(out), None))
    assert rel(host(out), ref) < TOL


@pytest.mark.parametrize("n", [1, 7, 1000, 248320])
def test_argmax_exact(T, lib, orc, n):
    rng = np.random.default_rng(n)
    v = rng.standard_normal((2, n)).astype(np.float32)
    if n > 10:
        v[0, n // 3] = v[0, n // 2] = 10.0  # tie: the first wins
    out = T.zeros(2, dtype=T.int32, device="cuda")
    call(lib.snl_argmax(ptr(dev(T, v)), 2, n, ptr(out), None))
    got = host(out).view(np.uint32)
    assert list(got) == [orc.argmax(v[0]), orc.argmax(v[1])]


def argmax_edge_rows(n=4096):
    """Rows where the reference's scan (best = 0, move on x > v[best]) differs from a naive
    ordering of floats: -0.0 tied with +0.0, NaN at index 0, NaN elsewhere, all -inf."""
    rows = np.full((6, n), -1.0, np.float32)
    rows[0, 5], rows[0, 9] = -0.0, 0.0      # -0.0 first, +0.0 later: index 5 wins
    rows[1, 5], rows[1, 9] = 0.0, -0.0      # +0.0 first: index 5 wins
    rows[2, 0], rows[2, 7] = np.nan, 3.0    # NaN at index 0: the scan never moves, 0
    rows[3, 3], rows[3, 8] = np.nan, 2.0    # NaN elsewhere never wins: 8
    rows[4, :] = -np.inf                    # all equal: 0
    rows[5, :] = np.nan                     # all NaN: 0
    return rows


@pytest.mark.parametrize("entry", ["snl_argmax", "snl_argmax_noalloc"])
def test_argmax_edge_cases(T, lib, orc, entry):
    v = argmax_edge_rows()
    want = [orc.argmax(r) for r in v]
    assert want == [5, 5, 0, 8, 0, 0]
    out = T.zeros(len(v), dtype=T.int32, device="cuda")
    call(getattr(lib, entry)(ptr(dev(T, v)), len(v), v.shape[1], ptr(out), None))
    T.cuda.synchronize()
    assert list(host(out).view(np.uint32)) == want


# ---- attention.wgsl -------------------------------------------------------------------


def attn_case(rng, m, pos0, n_kv=4, ctx=None):
    nh = 4 * n_kv
    HD = 256
    q_dim, kv_dim = nh * HD, n_kv * HD
    stride = 2 * q_dim + 2 * kv_dim
    ctx = ctx or pos0 + m + 8
    p = AttnP(nh, n_kv, 64, stride, 1e7, 1e-6, 1 / 16, (33 << 16) | 30)
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    norms = (0.1 * rng.standard_normal(2 * HD)).astype(np.float32)
    kc = np.zeros(ctx * kv_dim // 2, np.uint32)
    vc = np.zeros_like(kc)
    kc[: pos0 * kv_dim // 2] = rng.standard_normal(pos0 * kv_dim).astype(np.float16).view(np.uint32)
    vc[: pos0 * kv_dim // 2] = rng.standard_normal(pos0 * kv_dim).astype(np.float16).view(np.uint32)
    rpos = np.stack([np.arange(pos0, pos0 + m), np.arange(pos0, pos0 + m) + 3, np.arange(pos0, pos0 + m) + 7,
                     np.zeros(m)], 1).astype(np.uint32)
    return p, proj, norms, kc, vc, rpos


@pytest.mark.parametrize("m,pos0", [(1, 0), (1, 300), (3, 17), (40, 100)])
def test_attn_prep(T, lib, orc, m, pos0):
    rng = np.random.default_rng(m + pos0)
    p, proj, norms, kc, vc, rpos = attn_case(rng, m, pos0)
    st = StepU(m, pos0, 1, 0)
    q_ref = np.zeros((m, p.n_heads * 256), np.float32)
    kr, vr = kc.copy(), vc.copy()
    orc.attn_prep(st, p, proj, q_ref, kr, vr, norms, rpos)
    qd = T.zeros((m, p.n_heads * 256), device="cuda")
    kd, vd = dev(T, kc.view(np.int32)), dev(T, vc.view(np.int32))
    call(lib.snl_attn_prep(C.byref(st), C.byref(p), ptr(dev(T, proj)), ptr(qd), ptr(kd), ptr(vd), ptr(dev(T, norms)),
                           ptr(dev(T, rpos.view(np.int32))), None))
    assert rel(host(qd), q_ref) < TOL
    kg = host(kd).view(np.uint32).view(np.float16).astype(np.float32)
    assert rel(kg, kr.view(np.float16).astype(np.float32)) < TOL
    assert np.array_equal(host(vd).view(np.uint32), vr)  # V is stored without math: bit-exact


@pytest.mark.parametrize("m,pos0,parts", [(1, 0, 1), (1, 255, 1), (1, 1000, 4), (1, 2047, 8), (2, 5000, 20),
                                          (4, 700, 64), (9, 50, 1), (64, 200, 1),
                                          # prefill chunks (16+ rows): the tiled tensor-core kernel, including
                                          # ragged token blocks, a chunk from position 0, and 32K keys
                                          (16, 0, 1), (37, 100, 1), (512, 0, 1), (300, 4000, 1), (64, 32000, 1)])
def test_attend_combine(T, lib, orc, m, pos0, parts):
    rng = np.random.default_rng(pos0 + m)
    p, proj, norms, kc, vc, rpos = attn_case(rng, m, pos0)
    kv_dim = p.n_kv * 256
    n = (pos0 + m) * kv_dim // 2
    kc[:n] = rng.standard_normal(2 * n).astype(np.float16).view(np.uint32)
    vc[:n] = rng.standard_normal(2 * n).astype(np.float16).view(np.uint32)
    qbuf = rng.standard_normal((m, p.n_heads * 256)).astype(np.float32)
    st = StepU(m, pos0, parts, 0)
    out_ref = np.zeros((m, p.n_heads * 256), np.float32)
    part_ref = np.zeros((m * p.n_heads * parts, 258), np.float32)
    orc.attend(st, p, proj, qbuf, kc, vc, out_ref, part_ref)
    if parts > 1:
        orc.attn_combine(st, p, proj, part_ref, out_ref)
    out = T.zeros((m, p.n_heads * 256), device="cuda")
    part = T.zeros((m * p.n_heads * parts, 258), device="cuda")
    projd = dev(T, proj)
    call(lib.snl_attend(C.byref(st), C.byref(p), ptr(projd), ptr(dev(T, qbuf)), ptr(dev(T, kc.view(np.int32))),
                        ptr(dev(T, vc.view(np.int32))), ptr(out), ptr(part), None))
    if parts > 1:
        call(lib.snl_attn_combine(C.byref(st), C.byref(p), ptr(projd), ptr(part), ptr(out), None))
    assert rel(host(out), out_ref) < TOL


# ---- linear.wgsl --------------------------------------------------------------------


def lin_case(rng, m, n_k=16, n_v=32):
    cd = 2 * n_k * 128 + n_v * 128
    stride = cd + n_v * 128 + 2 * n_v
    lpp = LinP(cd, stride, n_k, n_v, 1e-6, (0, 0, 0))
    proj = rng.standard_normal((m, stride)).astype(np.float32)
    lw = np.concatenate([0.5 * rng.standard_normal(cd * 4), 0.1 * rng.standard_normal(n_v),
                         0.1 * rng.standard_normal(n_v), 1 + 0.1 * rng.standard_normal(128)]).astype(np.float32)
    return lpp, proj, lw, cd


@pytest.mark.parametrize("m,ckpt", [(1, 0), (2, 1), (11, 7), (37, 0), (37, 2)])
def test_conv(T, lib, orc, m, ckpt):
    rng = np.random.default_rng(m)
    lpp, proj, lw, cd = lin_case(rng, m)
    cs = rng.standard_normal((3, cd)).astype(np.float32)
    st = StepU(m, 0, 1, ckpt)
    out_ref, cs_ref, ck_ref = np.zeros((m, cd), np.float32), cs.copy(), np.zeros((3, cd), np.float32)
    orc.conv(st, lpp, proj, out_ref, cs_ref, lw, ck_ref)
    out, csd, ckd = T.zeros((m, cd), device="cuda"), dev(T, cs), T.zeros((3, cd), device="cuda")
    call(lib.snl_conv(C.byref(st), C.byref(lpp), ptr(dev(T, proj)), ptr(out), ptr(csd), ptr(dev(T, lw)), ptr(ckd), None))
    assert rel(host(out), out_ref) < TOL
    assert np.array_equal(host(csd), cs_ref)  # the carried state is copied, not computed
    if ckpt:
        assert np.array_equal(host(ckd), ck_ref)


@pytest.mark.parametrize("m,ckpt", [(1, 0), (2, 1), (7, 3), (40, 0), (512, 0)])
def test_conv_delta_fused(T, lib, orc, m, ckpt):
    """The engine's fused conv + delta kernel (snl_conv_delta) against the oracle's
    conv then delta, states and checkpoints included."""
    rng = np.random.default_rng(30 + m)
    lpp, proj, lw, cd = lin_case(rng, m)
    cs = rng.standard_normal((3, cd)).astype(np.float32)
    S = (0.05 * rng.standard_normal((32, 128, 128))).astype(np.float32)
    st = StepU(m, 0, 1, ckpt)
    conv_out = np.zeros((m, cd), np.float32)
    cs_ref, cck_ref = cs.copy(), np.zeros((3, cd), np.float32)
    orc.conv(st, lpp, proj, conv_out, cs_ref, lw, cck_ref)
    out_ref, S_ref, sck_ref = np.zeros((m, 4096), np.float32), S.copy(), np.zeros_like(S)
    orc.delta(st, lpp, proj, conv_out, S_ref, lw, out_ref, sck_ref)
    out, csd, Sd = T.zeros((m, 4096), device="cuda"), dev(T, cs), dev(T, S)
    cck, sck = T.zeros((3, cd), device="cuda"), T.zeros(S.shape, device="cuda")
    call(lib.snl_conv_delta(C.byref(st), C.byref(lpp), ptr(dev(T, proj)), ptr(csd), ptr(Sd), ptr(dev(T, lw)), ptr(out),
                            ptr(cck), ptr(sck), None))
    assert rel(host(out), out_ref) < TOL
    assert rel(host(Sd), S_ref) < TOL
    assert np.array_equal(host(csd), cs_ref)
    if ckpt:
        assert np.array_equal(host(cck), cck_ref)
        assert rel(host(sck), sck_ref) < TOL


@pytest.mark.slow
def test_deltanet_config2_full_length(T, lib, orc):
    """BASELINE.json configs[1] at its full length: one Gated DeltaNet layer (16 QK / 32 V
    heads of 128) over a 4096-token prefill in 8 chained 512-row steps (the chunked form,
    chunks of 64), then 256 single-token steps (the recurrent form), each carrying the
    conv and delta states of the step before. Inputs as the config states: q, k, v, b, a,
    z ~ N(0,1), A_log = dt_bias = 0 (so g = -softplus(a)), conv weights N(0, 0.5), norm
    weight 1. The oracle runs the reference's token-sequential conv + delta over the same
    steps: every step's output rows and the state after each step within 1e-3, the conv
    state bit-exact."""
    n_k, n_v, D = 16, 32, 128
    cd = 2 * n_k * D + n_v * D
    stride = cd + n_v * D + 2 * n_v
    lpp = LinP(cd, stride, n_k, n_v, 1e-6, (0, 0, 0))
    P, R, chunk = 4096, 256, 512
    rng = np.random.default_rng(2024)
    proj = rng.standard_normal((P + R, stride)).astype(np.float32)
    lw = np.concatenate([np.sqrt(0.5) * rng.standard_normal(cd * 4), np.zeros(2 * n_v), np.ones(D)]).astype(np.float32)
    cs_h, S_h = np.zeros((3, cd), np.float32), np.zeros((n_v, D, D), np.float32)
    dproj, dlw = dev(T, proj), dev(T, lw)
    cs_d, S_d = T.zeros((3, cd), device="cuda"), T.zeros((n_v, D, D), device="cuda")
    out_d = T.zeros((P + R, n_v * D), device="cuda")
    steps = [(r0, chunk) for r0 in range(0, P, chunk)] + [(P + i, 1) for i in range(R)]
    worst_out, worst_state = 0.0, 0.0
    out_ref = np.zeros((P + R, n_v * D), np.float32)
    for i, (r0, m) in enumerate(steps):
        st = StepU(m, r0, 1, 0)
        conv_out = np.zeros((m, cd), np.float32)
        orc.conv(st, lpp, proj[r0:r0 + m], conv_out, cs_h, lw, np.zeros((3, cd), np.float32))
        orc.delta(st, lpp, proj[r0:r0 + m], conv_out, S_h, lw, out_ref[r0:r0 + m], np.zeros_like(S_h))
        call(lib.snl_conv_delta(C.byref(st), C.byref(lpp), C.c_void_p(dproj.data_ptr() + 4 * r0 * stride), ptr(cs_d),
                                ptr(S_d), ptr(dlw), C.c_void_p(out_d.data_ptr() + 4 * r0 * n_v * D), None, None, None))
        if m > 1 or i == len(steps) - 1 or (r0 - P) % 32 == 31:
            worst_out = max(worst_out, rel(host(out_d[r0:r0 + m]), out_ref[r0:r0 + m]))
            worst_state = max(worst_state, rel(host(S_d), S_h))
            assert np.array_equal(host(cs_d), cs_h), (r0, m)
    assert worst_out < TOL, worst_out
    assert worst_state < TOL, worst_state
    assert rel(host(out_d), out_ref) < TOL


@pytest.mark.parametrize("m,ckpt", [(1, 0), (2, 1), (24, 0)])
def test_delta(T, lib, orc, m, ckpt):
    rng = np.random.default_rng(10 + m)
    lpp, proj, lw, cd = lin_case(rng, m)
    conv_out = rng.standard_normal((m, cd)).astype(np.float32)
    S = (0.05 * rng.standard_normal((32, 128, 128))).astype(np.float32)
    st = StepU(m, 0, 1, ckpt)
    out_ref, S_ref, ck_ref = np.zeros((m, 4096), np.float32), S.copy(), np.zeros_like(S)
    orc.delta(st, lpp, proj, conv_out, S_ref, lw, out_ref, ck_ref)
    out, Sd, ckd = T.zeros((m, 4096), device="cuda"), dev(T, S), T.zeros(S.shape, device="cuda")
    call(lib.snl_delta(C.byref(st), C.byref(lpp), ptr(dev(T, proj)), ptr(dev(T, conv_out)), ptr(Sd), ptr(dev(T, lw)),
                       ptr(out), ptr(ckd), None))
    assert rel(host(out), out_ref) < TOL
    assert rel(host(Sd), S_ref) < TOL
    if ckpt:
        assert rel(host(ckd), ck_ref) < TOL


# ---- sampler.rs ------------------------------------------------------------------------


def test_sample_matches_oracle(T, lib, orc):
    """snl_sample (penalties, greedy, top-k order, temperature, min-p, top-p, draw and
    verify with the caller's draws) against the oracle's restatement, at the 9B vocab
    size and small ones."""
    from sensenova_b200.ffi import SampleP

    rng = np.random.default_rng(77)
    scratch = T.empty(int(lib.snl_sample_scratch_bytes()), dtype=T.uint8, device="cuda")
    out = T.zeros(3, dtype=T.int32, device="cuda")
    for i in range(200):
        n = int(rng.choice([37, 1000, 248320]))
        p = SampleP(float(rng.choice([0.0, 0.6, 1.0, 1.4])), float(rng.choice([1.0, 0.95, 0.7])),
                    int(rng.choice([1, 7, 20, 100, 256])), float(rng.choice([0.0, 0.05, 0.3])),
                    float(rng.choice([0.0, 0.4])), float(rng.choice([0.0, 0.15])), float(rng.choice([1.0, 1.2, 0.8])), 0)
        logits = (rng.standard_normal(n) * rng.choice([1.0, 4.0])).astype(np.float32)
        if i % 7 == 0:
            logits[rng.integers(0, n, 20)] = logits.max()  # exact ties: ranked by index
        ht = rng.choice(n, size=min(n, int(rng.integers(0, 16))), replace=False).astype(np.uint32)
        hc = rng.integers(1, 5, size=ht.size).astype(np.uint32)
        u = rng.random(2).astype(np.float32)
        draft = -1 if i % 3 == 0 else (int(np.argmax(logits)) if i % 3 == 1 else int(rng.integers(0, n)))
        want = orc.sample(p, logits.copy(), ht, hc, u, draft)
        ld = dev(T, logits)
        htd = dev(T, ht.view(np.int32)) if ht.size else None
        hcd = dev(T, hc.view(np.int32)) if hc.size else None
        call(lib.snl_sample(C.byref(p), ptr(ld), n, ptr(htd), ptr(hcd), int(ht.size),
                            u.ctypes.data_as(C.c_void_p), draft, ptr(out), ptr(scratch), None))
        got = tuple(int(v) for v in host(out).view(np.uint32))
        assert got == want, (i, n, p.temperature, p.top_k, p.top_p, p.min_p, got, want)


def test_sample_refuses_unordered_top_k(T, lib):
    from sensenova_b200.ffi import SampleP

    scratch = T.empty(int(lib.snl_sample_scratch_bytes()), dtype=T.uint8, device="cuda")
    out = T.zeros(3, dtype=T.int32, device="cuda")
    logits = T.zeros(1000, dtype=T.float32, device="cuda")
    u = np.array([0.5, 0.5], np.float32)
    for k in (0, 257):
        p = SampleP(1.0, 0.95, k, 0.0, 0.0, 0.0, 1.0, 0)
        rc = lib.snl_sample(C.byref(p), ptr(logits), 1000, None, None, 0, u.ctypes.data_as(C.c_void_p), -1, ptr(out),
                            ptr(scratch), None)
        assert rc == -7  # SNL_E_UNSUPPORTED
