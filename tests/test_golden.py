"""The oracle against the committed golden vectors of the reference's own kernels
(tests/golden/reference_kernels.npz, written by tests/golden/make_golden.py from the
reference's WGSL run on the host cores): every output bit-identical. Runs on any
machine, with or without the reference tree; with it, also checks that the fixture is
what the reference's kernels give today.
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import golden_cases as G  # noqa: E402

FIXTURE = np.load(GOLDEN / "reference_kernels.npz")
META = json.loads(FIXTURE["meta"].tobytes().decode())


def check_bits(name: str, outs: dict) -> None:
    for k, v in outs.items():
        v = np.ascontiguousarray(v).reshape(-1)
        m = META[name]["outputs"][k]
        assert v.size == m["size"], (name, k)
        want = FIXTURE[f"{name}/{k}"]
        got = v[:: m["stride"]]
        if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
            d = np.abs(got.astype(np.float64) - want.astype(np.float64))
            raise AssertionError(f"{name}/{k}: {int((d > 0).sum())} sampled values differ, max |diff| {d.max():.3g}")
        assert hashlib.sha256(v.tobytes()).hexdigest() == m["sha256"], f"{name}/{k}: full-output digest differs"


def test_fixture_covers_every_case():
    assert sorted(META) == sorted(n for n, _, _ in G.CASES)


@pytest.mark.parametrize("name,kernel,a", G.CASES, ids=[c[0] for c in G.CASES])
def test_oracle_matches_reference_golden(orc, name, kernel, a):
    check_bits(name, G.run(name, kernel, a, orc))


@pytest.mark.parametrize("name,kernel,a", G.CASES, ids=[c[0] for c in G.CASES])
def test_fixture_is_the_reference_output(name, kernel, a):
    import wgslref as wr

    if not wr.available():
        pytest.skip("reference tree absent")
    check_bits(name, G.run(name, kernel, a, wr))
