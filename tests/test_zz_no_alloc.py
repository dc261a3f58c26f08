"""snl_argmax_noalloc: the argmax entry point for callers that must not allocate device
memory when they call it (a host whose device memory is reserved by its own pool
allocator, or a serving loop that cannot take the device-wide wait of cudaFree).

It must return exactly what snl_argmax returns. The static scratch it uses is shared by
every call and keeps the previous call's contents, so the check runs two calls in a row
on different inputs. This file is collected last, so a run that stops at the first
failure has already run every other test; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from sensenova_b200 import ffi

pytestmark = pytest.mark.gpu


def _argmax_both(torch, lib, logits: np.ndarray):
    rows, n = logits.shape
    src = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    out_ref = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    out_new = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    ffi.check(lib.snl_argmax(C.c_void_p(src.data_ptr()), rows, n, C.c_void_p(out_ref.data_ptr()), None))
    ffi.check(lib.snl_argmax_noalloc(C.c_void_p(src.data_ptr()), rows, n, C.c_void_p(out_new.data_ptr()), None))
    torch.cuda.synchronize()
    return out_ref.cpu().numpy().view(np.uint32), out_new.cpu().numpy().view(np.uint32)


def test_noalloc_argmax_matches_snl_argmax_twice(torch_cuda, lib):
    torch = torch_cuda
    rng = np.random.default_rng(1234)
    # Two calls in a row with different inputs and row counts: the second call must not
    # see anything left in the shared scratch by the first.
    for rows, n in ((2, 248320), (5, 4099)):
        logits = rng.standard_normal((rows, n)).astype(np.float32)
        logits[0, n // 3] = logits[0, n // 2] = 50.0  # a tie: the first index wins
        logits[-1, -1] = 60.0
        ref, new = _argmax_both(torch, lib, logits)
        assert np.array_equal(ref, new), (ref, new)  # indices: exact, no tolerance
        assert new[0] == n // 3 and new[-1] == n - 1
        assert list(new) == [int(np.argmax(r)) for r in logits]


def test_noalloc_argmax_rejects_rows_beyond_its_scratch(torch_cuda, lib):
    torch = torch_cuda
    src = torch.zeros(17 * 64, device="cuda")
    out = torch.zeros(17, dtype=torch.int32, device="cuda")
    rc = lib.snl_argmax_noalloc(C.c_void_p(src.data_ptr()), 17, 64, C.c_void_p(out.data_ptr()), None)
    assert rc == -2
    assert b"exceed the static scratch of 16 rows" in lib.snl_last_error()
