"""The C ABI library on the CPU: it loads, exports every function include/snl_b200.h
declares, and its host-side checks (config validation, argument errors) work
without a device."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from sensenova_b200 import ffi
from sensenova_b200.config import ModelConfig, nine_b, small

ROOT = Path(__file__).resolve().parent.parent


def header_functions() -> set[str]:
    text = (ROOT / "include" / "snl_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return set(re.findall(r"\b(snl_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_abi():
    fns = header_functions()
    assert {"snl_mat", "snl_attend", "snl_delta", "snl_engine_forward_mm", "snl_engine_mtp"} <= fns
    assert len(fns) >= 30


def test_library_exports_every_declared_symbol(lib):
    missing = [f for f in sorted(header_functions()) if not hasattr(lib, f)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert header_functions() <= set(ffi.SIGNATURES), header_functions() - set(ffi.SIGNATURES)


def test_only_abi_symbols_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(ffi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    ours = {s for s in exported if s.startswith("snl_")}
    assert header_functions() <= ours


def test_struct_sizes_match_the_reference_uniforms():
    # #[repr(C)] structs of engine.rs:24-82 are 16 or 32 bytes.
    assert C.sizeof(ffi.StepU) == 16
    for s in (ffi.MatP, ffi.LayerP, ffi.AttnP, ffi.LinP):
        assert C.sizeof(s) == 32


def test_config_validate(lib):
    nine_b().validate()
    small().validate()
    bad = nine_b()
    bad.head_dim = 128
    with pytest.raises(ffi.SnlError, match="head_dim must be 256"):
        bad.validate()
    bad = nine_b()
    bad.mhc.start, bad.mhc.end = 2, 10
    with pytest.raises(ffi.SnlError, match="mHC range crosses a loop boundary"):
        bad.validate()
    bad = nine_b()
    bad.n_kv_heads = 8
    with pytest.raises(ffi.SnlError, match="4 query heads per KV head"):
        bad.validate()


def test_kernel_entry_points_reject_null_arguments(lib):
    st, p = ffi.StepU(1, 0, 1, 0), ffi.MatP(16, 32, 0, 32, 0, 16, 0, 0)
    rc = lib.snl_mat(ffi.SNL_Q8_0, C.byref(st), C.byref(p), None, None, None, None, None)
    assert rc == -1 and b"null" in lib.snl_last_error()


def test_config_json_roundtrip():
    c = nine_b()
    d = c.to_json()
    c2 = ModelConfig.from_json(d)
    assert c2 == c
