"""ctypes binding of include/snl_b200.h (the C ABI of libsnl_b200.so).

The library is the only compute path: if it is missing this module raises at import
time instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("SNL_LIB", PKG_DIR / "libsnl_b200.so"))

SNL_F32, SNL_Q8_0, SNL_Q4_0 = 0, 1, 2
SNL_OK = 0
ERRORS = {
    -1: "SNL_E_INVALID", -2: "SNL_E_RANGE", -3: "SNL_E_CUDA", -4: "SNL_E_OOM",
    -5: "SNL_E_STATE", -6: "SNL_E_TIMEOUT", -7: "SNL_E_UNSUPPORTED", -8: "SNL_E_NCCL",
}
(SNL_E_INVALID, SNL_E_RANGE, SNL_E_CUDA, SNL_E_OOM, SNL_E_STATE, SNL_E_TIMEOUT, SNL_E_UNSUPPORTED,
 SNL_E_NCCL) = -1, -2, -3, -4, -5, -6, -7, -8
SNL_TP_HANDLE_BYTES = 64
SNL_TP_FULL, SNL_TP_ROWS, SNL_TP_COLS, SNL_TP_ELEMS = 0, 1, 2, 3
SNL_ENGINE_MTP = 1
SNL_ENGINE_F16_SCALES = 2
SNL_FINISH_STOP, SNL_FINISH_LENGTH = 0, 1
SNL_WORKER_SNAPSHOTS = 4
SNL_VIS_HEAD_DIM = 72
SNL_VIS_ACT_GELU_TANH, SNL_VIS_ACT_GELU_ERF = 1, 2
MAX_LAYERS = 256


class StepU(C.Structure):
    """StepU (engine.rs:24-32)."""
    _fields_ = [("m", C.c_uint32), ("pos0", C.c_uint32), ("parts", C.c_uint32), ("ckpt", C.c_uint32)]


class SampleP(C.Structure):
    """SamplingParams without the seed (sampler.rs:4-14)."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32), ("min_p", C.c_float),
                ("presence_penalty", C.c_float), ("frequency_penalty", C.c_float),
                ("repetition_penalty", C.c_float), ("pad", C.c_uint32)]


class MatP(C.Structure):
    """MatP (engine.rs:34-45)."""
    _fields_ = [(n, C.c_uint32) for n in ("n", "k", "x_off", "x_stride", "y_off", "y_stride", "n_off", "m_one")]


class LayerP(C.Structure):
    """LayerP (engine.rs:47-58)."""
    _fields_ = [("h", C.c_uint32), ("mode", C.c_uint32), ("last_row", C.c_uint32), ("eps", C.c_float),
                ("weight_one", C.c_float), ("iterations", C.c_uint32), ("inter", C.c_uint32), ("x_stride", C.c_uint32)]


class AttnP(C.Structure):
    """AttnP (engine.rs:60-71)."""
    _fields_ = [("n_heads", C.c_uint32), ("n_kv", C.c_uint32), ("rot_dim", C.c_uint32), ("proj_stride", C.c_uint32),
                ("rope_theta", C.c_float), ("eps", C.c_float), ("scale", C.c_float), ("mrope", C.c_uint32)]


class LinP(C.Structure):
    """LinP (engine.rs:73-82)."""
    _fields_ = [("conv_dim", C.c_uint32), ("proj_stride", C.c_uint32), ("n_k", C.c_uint32), ("n_v", C.c_uint32),
                ("eps", C.c_float), ("pad", C.c_uint32 * 3)]


class ModelConfigC(C.Structure):
    """snl_model_config (the text part of ModelConfig, config.rs:7-37)."""
    _fields_ = [
        ("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("vocab", C.c_uint32), ("n_layers", C.c_uint32),
        ("full_attention", C.c_uint8 * MAX_LAYERS),
        ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("rot_dim", C.c_uint32),
        ("rope_theta", C.c_float), ("mrope_section", C.c_uint32 * 3),
        ("lin_k_heads", C.c_uint32), ("lin_v_heads", C.c_uint32), ("lin_k_dim", C.c_uint32), ("lin_v_dim", C.c_uint32),
        ("conv_kernel", C.c_uint32), ("eps", C.c_float),
        ("loop_start", C.c_uint32), ("loop_end", C.c_uint32), ("loop_count", C.c_uint32),
        ("mhc_start", C.c_int32), ("mhc_end", C.c_int32), ("mhc_streams", C.c_uint32), ("mhc_iterations", C.c_uint32),
        ("max_position", C.c_uint32),
    ]


class OpStat(C.Structure):
    """snl_op_stat: one row of the per-op profile."""
    _fields_ = [("label", C.c_char * 32), ("calls", C.c_uint32), ("ms", C.c_double), ("bytes", C.c_double)]


class VisP(C.Structure):
    """VisP (vision.rs:39-50)."""
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("mode", C.c_uint32), ("act", C.c_uint32),
                ("eps", C.c_float), ("grid_w", C.c_uint32), ("heads", C.c_uint32), ("pad", C.c_uint32)]


class VisionConfigC(C.Structure):
    """snl_vision_config (VisionConfig, config.rs:40-70)."""
    _fields_ = [(n, C.c_uint32) for n in ("hidden", "intermediate", "intermediate_padded", "depth", "n_heads", "patch",
                                          "temporal_patch", "merge", "out_hidden", "pos_side")]


# Callback types of snl_worker_ops and snl_gen_request (include/snl_b200.h).
sz_t = C.c_size_t
FWD_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, sz_t, C.c_void_p, C.c_void_p, C.c_void_p, sz_t, sz_t, C.c_int)
FWD_GREEDY_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, sz_t, C.c_void_p, sz_t, C.c_int, C.c_void_p)
SAMPLE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, sz_t, C.POINTER(SampleP), C.c_void_p, C.c_void_p, sz_t, C.c_void_p,
                        C.c_int64, C.c_void_p)
MTP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, sz_t, C.c_void_p, sz_t, C.c_void_p, sz_t, C.c_int, C.c_void_p)
SELF_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)
SLOT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, sz_t)
RESTORE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, sz_t, sz_t)
SIZE_FN = C.CFUNCTYPE(sz_t, C.c_void_p)
NOW_FN = C.CFUNCTYPE(C.c_double, C.c_void_p)
TOKEN_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32)


class WorkerOps(C.Structure):
    """snl_worker_ops: the engine as the generation loop sees it."""
    _fields_ = [("self", C.c_void_p), ("ctx", sz_t), ("prefill_chunk", sz_t), ("hidden", sz_t), ("has_mtp", C.c_int),
                ("forward", FWD_FN), ("forward_greedy", FWD_GREEDY_FN), ("sample", SAMPLE_FN), ("mtp", MTP_FN),
                ("reset", SELF_FN), ("snapshot", SLOT_FN), ("restore", RESTORE_FN), ("rollback", SELF_FN),
                ("hid_rows", SIZE_FN), ("pos", SIZE_FN), ("now", NOW_FN)]


class GenRequestC(C.Structure):
    """snl_gen_request: GenRequest (worker.rs:17-27) with the Prompt flattened."""
    _fields_ = [("tokens", C.c_void_p), ("keys", C.c_void_p), ("pos", C.c_void_p), ("n", sz_t),
                ("embed_idx", C.c_void_p), ("embeds", C.c_void_p), ("n_embeds", sz_t), ("snapshot_at", C.c_int64),
                ("params", SampleP), ("seed", C.c_uint64), ("has_seed", C.c_int), ("max_tokens", sz_t),
                ("eos", C.c_void_p), ("n_eos", sz_t), ("on_token", TOKEN_FN), ("user", C.c_void_p)]


class FinishC(C.Structure):
    """snl_finish: Finish (worker.rs:41-55)."""
    _fields_ = [("reason", C.c_int), ("cancelled", C.c_int), ("prompt_tokens", sz_t), ("completion_tokens", sz_t),
                ("cached_tokens", sz_t), ("drafted", sz_t), ("accepted", sz_t), ("prefill_secs", C.c_double),
                ("decode_secs", C.c_double)]


class SnlError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code
        self.kind = ERRORS.get(code, str(code))


vp = C.c_void_p
u32 = C.c_uint32
u64 = C.c_uint64
sz = C.c_size_t
i32 = C.c_int
P = C.POINTER

# name -> (restype, argtypes); mirrors include/snl_b200.h.
SIGNATURES = {
    "snl_last_error": (C.c_char_p, []),
    "snl_version": (C.c_char_p, []),
    "snl_launch_count": (u64, []),
    "snl_device_error": (i32, [i32]),
    "snl_config_validate": (i32, [P(ModelConfigC)]),
    "snl_mat": (i32, [i32, P(StepU), P(MatP), vp, vp, vp, vp, vp]),
    "snl_xpack": (i32, [vp, u32, u32, u32, vp, vp]),
    "snl_mat_xpack": (i32, [i32, P(MatP), u32, vp, vp, vp, vp, vp]),
    "snl_weight_planes": (i32, [i32, u32, u32, vp, vp, vp, vp]),
    "snl_sample": (i32, [P(SampleP), vp, u32, vp, vp, u32, vp, C.c_int64, vp, vp, vp]),
    "snl_sample_scratch_bytes": (C.c_size_t, []),
    "snl_mat_wplanes": (i32, [i32, P(StepU), P(MatP), vp, vp, vp, vp, vp, vp]),
    "snl_tile_sizes": (i32, [i32, u32, u32, P(sz), P(sz)]),
    "snl_tile_repack": (i32, [i32, u32, u32, vp, vp, vp, vp, P(i32), vp]),
    "snl_mat_tiles": (i32, [i32, P(MatP), u32, vp, vp, vp, i32, vp, vp]),
    "snl_branch_norm": (i32, [P(StepU), P(LayerP), vp, vp, vp, vp, u32, vp]),
    "snl_mhc_dots": (i32, [P(StepU), P(LayerP), vp, vp, vp, vp]),
    "snl_mhc_finish": (i32, [P(StepU), P(LayerP), vp, vp, vp, vp]),
    "snl_merge": (i32, [P(StepU), P(LayerP), vp, vp, vp, vp]),
    "snl_swiglu": (i32, [P(StepU), P(LayerP), vp, vp, vp]),
    "snl_attn_prep": (i32, [P(StepU), P(AttnP), vp, vp, vp, vp, vp, vp, vp]),
    "snl_attend": (i32, [P(StepU), P(AttnP), vp, vp, vp, vp, vp, vp, vp]),
    "snl_attn_combine": (i32, [P(StepU), P(AttnP), vp, vp, vp, vp]),
    "snl_conv": (i32, [P(StepU), P(LinP), vp, vp, vp, vp, vp, vp]),
    "snl_delta": (i32, [P(StepU), P(LinP), vp, vp, vp, vp, vp, vp, vp]),
    "snl_conv_delta": (i32, [P(StepU), P(LinP), vp, vp, vp, vp, vp, vp, vp, vp]),
    "snl_argmax": (i32, [vp, u32, u32, vp, vp]),
    "snl_argmax_noalloc": (i32, [vp, u32, u32, vp, vp]),
    "snl_synth_quant": (i32, [u64, C.c_char_p, i32, sz, sz, vp, vp, vp]),
    "snl_synth_f32": (i32, [u64, C.c_char_p, u32, sz, C.c_float, C.c_float, vp, vp]),
    "snl_engine_create": (i32, [P(ModelConfigC), sz, i32, u32, P(vp)]),
    "snl_engine_create_tp": (i32, [P(ModelConfigC), sz, i32, u32, i32, i32, P(vp)]),
    "snl_engine_tp_handle": (i32, [vp, vp]),
    "snl_tp_plan": (i32, [P(ModelConfigC), i32, i32, C.c_char_p, P(i32), P(sz), sz, P(sz)]),
    "snl_engine_tp_connect": (i32, [vp, vp]),
    "snl_engine_set_tensor": (i32, [vp, C.c_char_p, i32, sz, sz, vp, vp]),
    "snl_engine_fill_synthetic": (i32, [vp, u64, i32]),
    "snl_engine_finalize": (i32, [vp]),
    "snl_engine_destroy": (None, [vp]),
    "snl_engine_forward_mm": (i32, [vp, vp, sz, vp, vp, vp, sz, sz, i32, vp]),
    "snl_engine_forward_greedy": (i32, [vp, vp, sz, vp, sz, i32, vp]),
    "snl_engine_mtp": (i32, [vp, sz, vp, sz, vp, sz, i32, vp]),
    "snl_engine_generate": (i32, [vp, u32, sz, vp, P(C.c_float)]),
    "snl_engine_profile": (i32, [vp, u32, P(OpStat), sz, P(sz)]),
    "snl_engine_reset": (i32, [vp]),
    "snl_engine_snapshot": (i32, [vp, sz]),
    "snl_engine_restore": (i32, [vp, sz, sz]),
    "snl_engine_rollback": (i32, [vp]),
    "snl_engine_hid_rows": (sz, [vp]),
    "snl_engine_has_mtp": (i32, [vp]),
    "snl_engine_sample": (i32, [vp, C.c_size_t, P(SampleP), vp, vp, C.c_size_t, vp, C.c_int64, vp]),
    "snl_engine_tile_scales": (i32, [vp, P(u32), P(u32)]),
    "snl_engine_pos": (sz, [vp]),
    "snl_engine_ctx": (sz, [vp]),
    "snl_engine_device_bytes": (sz, [vp]),
    "snl_engine_read_hidden": (i32, [vp, sz, sz, vp]),
    "snl_engine_prefill_chunk": (sz, [vp]),
    "snl_vis_layer_norm": (i32, [P(VisP), vp, vp, vp, vp]),
    "snl_vis_epilogue": (i32, [P(VisP), vp, vp, vp, vp, vp]),
    "snl_vis_rope": (i32, [P(VisP), vp, vp]),
    "snl_vis_attend": (i32, [P(VisP), vp, vp, vp]),
    "snl_vision_create": (i32, [P(VisionConfigC), i32, P(vp)]),
    "snl_vision_set_tensor": (i32, [vp, C.c_char_p, i32, sz, sz, vp, vp]),
    "snl_vision_fill_synthetic": (i32, [vp, u64]),
    "snl_vision_finalize": (i32, [vp]),
    "snl_vision_encode": (i32, [vp, vp, sz, sz, sz, vp]),
    "snl_vision_destroy": (None, [vp]),
    "snl_worker_create": (i32, [vp, P(vp)]),
    "snl_worker_create_ops": (i32, [P(WorkerOps), P(vp)]),
    "snl_worker_destroy": (None, [vp]),
    "snl_worker_run": (i32, [vp, P(GenRequestC), vp, sz, P(FinishC)]),
    "snl_worker_prefix": (i32, [vp, i32, vp, sz, P(sz), P(u64)]),
    "snl_worker_spec": (i32, [vp, P(i32), P(sz)]),
    "snl_rng_uniforms": (i32, [u64, sz, vp]),
    "snl_chacha_block": (i32, [vp, i32, vp]),
}

_lib: C.CDLL | None = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Load libsnl_b200.so (once) and declare every exported function."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with `python sense-nova-server_b200/build.py --lib`")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != SNL_OK:
        msg = load().snl_last_error().decode(errors="replace")
        raise SnlError(rc, msg or ERRORS.get(rc, f"error {rc}"))
