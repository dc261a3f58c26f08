"""Write reference_kernels.npz: the reference's own WGSL kernels (translated and run on
the host cores by oracle/wgslref.py) on every case of golden_cases.py.

Run where the reference tree exists: python tests/golden/make_golden.py
Outputs of more than SMALL elements are stored as a SHA-256 of their bits plus every
stride-th value, which keeps the fixture small; the CPU test checks the oracle against
the digest, the GPU test checks the CUDA path against the sampled values.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (str(HERE), str(ROOT / "sense-nova-server_b200"), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)
import golden_cases as G  # noqa: E402

FIXTURE = HERE / "reference_kernels.npz"
SMALL = 8192


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def stride_of(n: int) -> int:
    return 1 if n <= SMALL else -(-n // 2048)


def record(outs: dict) -> dict:
    rec = {}
    for k, v in outs.items():
        v = np.ascontiguousarray(v).reshape(-1)
        s = stride_of(v.size)
        rec[k] = v if s == 1 else v[::s].copy()
    return rec


def main() -> None:
    import wgslref as wr

    arrays, meta = {}, {}
    for name, kernel, a in G.CASES:
        outs = G.run(name, kernel, a, wr)
        for k, v in record(outs).items():
            arrays[f"{name}/{k}"] = v
        meta[name] = {"kernel": kernel, "args": a,
                      "outputs": {k: {"size": int(v.size), "stride": stride_of(v.size), "sha256": digest(v)}
                                  for k, v in outs.items()}}
    arrays["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), np.uint8)
    np.savez_compressed(FIXTURE, **arrays)
    print(f"{FIXTURE}: {len(G.CASES)} cases, {FIXTURE.stat().st_size} bytes")


if __name__ == "__main__":
    main()
