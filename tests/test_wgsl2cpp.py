"""The WGSL -> C++ translator and its runtime (oracle/wgsl2cpp.py, oracle/wgsl_rt.h), on
small compute shaders written for this test: the constructs the reference's kernels use
(workgroup memory and barriers, loops, vectors, a matrix, pointers, select, f16 packing,
uniform structs, storage arrays of vec4) must give the values WGSL defines, and an
out-of-bounds access must fail the dispatch. This is what makes the bit-exact checks of
the oracle against the translated reference kernels meaningful."""
import ctypes as C

import numpy as np
import pytest

import wgsl2cpp
import wgslref as wr

SHADER = r"""
struct P {
    n: u32,
    scale: f32,
    _a: u32,
    _b: u32,
}
const W: u32 = 64u;
@group(0) @binding(0) var<uniform> p: P;
@group(0) @binding(1) var<storage, read> x: array<f32>;
@group(0) @binding(2) var<storage, read_write> y: array<f32>;
@group(0) @binding(3) var<storage, read> x4: array<vec4<f32>>;
var<workgroup> red: array<f32, 64>;

fn tree(lid: u32, v: f32) -> f32 {
    red[lid] = v;
    workgroupBarrier();
    for (var s = W / 2u; s > 0u; s >>= 1u) {
        if (lid < s) { red[lid] += red[lid + s]; }
        workgroupBarrier();
    }
    let r = red[0];
    workgroupBarrier();
    return r;
}

// Row sums of x [groups, n] (strided lanes, then a shared-memory tree), times scale.
@compute @workgroup_size(64)
fn rowsum(@builtin(workgroup_id) wid: vec3<u32>, @builtin(local_invocation_index) lid: u32) {
    var acc = 0.0;
    for (var i = lid; i < p.n; i += W) { acc += x[wid.x * p.n + i]; }
    let t = tree(lid, acc);
    if (lid == 0u) { y[wid.x] = t * p.scale; }
}

fn acc4(v: ptr<function, array<vec4<f32>, 2>>) -> vec4<f32> {
    return (*v)[0] + (*v)[1];
}

@compute @workgroup_size(4, 2)
fn vecs(@builtin(global_invocation_id) gid: vec3<u32>) {
    let i = gid.y * 4u + gid.x;
    var pair = array<vec4<f32>, 2>(x4[i], vec4<f32>(0.5));
    let v = acc4(&pair) * 2.0 - vec4<f32>(1.0);
    var m = mat4x4<f32>();
    m[1] = v;
    let h = unpack2x16float(pack2x16float(vec2<f32>(v.x, -v.y)));
    let sgn = i32(u32(i) << 28u) >> 28u;
    y[i] = dot(m[1], vec4<f32>(1.0)) + select(h.x, h.y, i % 2u == 0u) + f32(sgn) + max(v.z, v.w);
}

@compute @workgroup_size(1)
fn oob() {
    y[p.n * 1000u] = 1.0;
}
"""


class P(C.Structure):
    _fields_ = [("n", C.c_uint32), ("scale", C.c_float), ("_a", C.c_uint32), ("_b", C.c_uint32)]


@pytest.fixture(scope="module")
def testlib(tmp_path_factory):
    out = tmp_path_factory.mktemp("wgsl")
    path = wgsl2cpp.compile_modules({"t": SHADER}, out, "libwgsltest.so")
    return wr.load(path, ["t"])


def test_literals():
    assert wgsl2cpp.literal("1.0") == "1.0f"
    assert wgsl2cpp.literal("1e-6") == "1e-6f"
    assert wgsl2cpp.literal("2f") == "2.0f"
    assert wgsl2cpp.literal("0u") == "0u"
    assert wgsl2cpp.literal("3i") == "3"
    assert wgsl2cpp.literal("0xffffu") == "0xffffu"


def test_barrier_tree_reduction(testlib):
    groups, n = 5, 1000
    x = np.random.default_rng(0).standard_normal(groups * n).astype(np.float32)
    y = np.zeros(16, np.float32)
    wr.dispatch("t", "rowsum", (groups, 1, 1), {0: P(n, 0.5, 0, 0), 1: x, 2: y, 3: np.zeros(4, np.float32)},
                library=testlib)
    # the same order in numpy: lane-strided f32 partial sums, then the halving tree
    want = []
    for g in range(groups):
        part = np.zeros(64, np.float32)
        for lid in range(64):
            acc = np.float32(0)
            for i in range(lid, n, 64):
                acc = np.float32(acc + x[g * n + i])
            part[lid] = acc
        s = 32
        while s:
            part[:s] = part[:s] + part[s:2 * s]
            s //= 2
        want.append(np.float32(part[0] * np.float32(0.5)))
    assert np.array_equal(y[:groups], np.array(want, np.float32))


def test_vectors_matrix_pointer_select_f16(testlib):
    x4 = np.random.default_rng(1).standard_normal(8 * 4).astype(np.float32)
    y = np.zeros(8, np.float32)
    wr.dispatch("t", "vecs", (1, 1, 1), {0: P(8, 1.0, 0, 0), 1: np.zeros(4, np.float32), 2: y, 3: x4},
                library=testlib)
    for i in range(8):
        v = (x4[4 * i:4 * i + 4] + np.float32(0.5)) * np.float32(2) - np.float32(1)
        hx, hy = np.float32(np.float16(v[0])), np.float32(np.float16(-v[1]))
        sgn = ((i << 28) & 0xFFFFFFFF)
        sgn = (sgn - (1 << 32) if sgn >= 1 << 31 else sgn) >> 28
        d = np.float32(np.float32(np.float32(v[0] + v[1]) + v[2]) + v[3])
        want = np.float32(np.float32(np.float32(d + (hy if i % 2 == 0 else hx)) + np.float32(sgn)) + max(v[2], v[3]))
        assert y[i] == want, (i, y[i], want)


def test_out_of_bounds_fails_the_dispatch(testlib):
    y = np.zeros(4, np.float32)
    with pytest.raises(IndexError):
        wr.dispatch("t", "oob", (1, 1, 1), {0: P(1, 1.0, 0, 0), 1: np.zeros(4, np.float32), 2: y,
                                            3: np.zeros(4, np.float32)}, library=testlib)
