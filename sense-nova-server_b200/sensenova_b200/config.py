"""ModelConfig (config.rs:7-37, text part) and the benchmark model shapes.

Field names follow the reference's serde names, so a `.snl` header's "config"
object (weights.rs:76-81) loads directly with `ModelConfig.from_json`.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, asdict

from . import ffi


@dataclass
class MhcConfig:
    start: int
    end: int
    streams: int = 2
    iterations: int = 20


@dataclass
class ModelConfig:
    hidden: int
    intermediate: int
    vocab: int
    n_layers: int
    full_attention: list[bool]
    n_heads: int
    n_kv_heads: int
    head_dim: int
    rot_dim: int
    rope_theta: float
    lin_k_heads: int
    lin_v_heads: int
    lin_k_dim: int
    lin_v_dim: int
    conv_kernel: int
    eps: float
    loop_start: int
    loop_end: int
    loop_count: int
    mhc: MhcConfig | None = None
    mrope_section: list[int] = field(default_factory=lambda: [11, 11, 10])
    eos: list[int] = field(default_factory=list)
    max_position: int = 262144

    # ---- derived dims (config.rs:256-278) ----
    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def lin_key_dim(self) -> int:
        return self.lin_k_heads * self.lin_k_dim

    @property
    def lin_value_dim(self) -> int:
        return self.lin_v_heads * self.lin_v_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.lin_key_dim + self.lin_value_dim

    @property
    def lin_proj_rows(self) -> int:
        return self.conv_dim + self.lin_value_dim + 2 * self.lin_v_heads

    @property
    def attn_proj_rows(self) -> int:
        return 2 * self.q_dim + 2 * self.kv_dim

    def execution_plan(self) -> list[int]:
        """config.rs:242-250: prefix, looped block loop_count times, suffix."""
        plan = list(range(self.loop_start))
        for _ in range(self.loop_count):
            plan.extend(range(self.loop_start, self.loop_end))
        plan.extend(range(self.loop_end, self.n_layers))
        return plan

    def is_mhc(self, layer: int) -> bool:
        return self.mhc is not None and self.mhc.start <= layer < self.mhc.end

    def to_c(self) -> ffi.ModelConfigC:
        c = ffi.ModelConfigC()
        c.hidden, c.intermediate, c.vocab, c.n_layers = self.hidden, self.intermediate, self.vocab, self.n_layers
        if len(self.full_attention) > ffi.MAX_LAYERS:
            raise ValueError("too many layers")
        for i, f in enumerate(self.full_attention):
            c.full_attention[i] = 1 if f else 0
        c.n_heads, c.n_kv_heads, c.head_dim, c.rot_dim = self.n_heads, self.n_kv_heads, self.head_dim, self.rot_dim
        c.rope_theta = self.rope_theta
        for i in range(3):
            c.mrope_section[i] = self.mrope_section[i]
        c.lin_k_heads, c.lin_v_heads = self.lin_k_heads, self.lin_v_heads
        c.lin_k_dim, c.lin_v_dim, c.conv_kernel = self.lin_k_dim, self.lin_v_dim, self.conv_kernel
        c.eps = self.eps
        c.loop_start, c.loop_end, c.loop_count = self.loop_start, self.loop_end, self.loop_count
        if self.mhc is None:
            c.mhc_start, c.mhc_end, c.mhc_streams, c.mhc_iterations = -1, -1, 0, 0
        else:
            c.mhc_start, c.mhc_end = self.mhc.start, self.mhc.end
            c.mhc_streams, c.mhc_iterations = self.mhc.streams, self.mhc.iterations
        c.max_position = min(self.max_position, 2**32 - 1)
        return c

    def validate(self) -> None:
        """ModelConfig::validate (config.rs:194-240), through the library."""
        lib = ffi.load()
        cc = self.to_c()
        ffi.check(lib.snl_config_validate(C.byref(cc)))

    @classmethod
    def from_json(cls, d: dict) -> "ModelConfig":
        d = dict(d)
        d.pop("vision", None)
        mhc = d.pop("mhc", None)
        known = {f for f in cls.__dataclass_fields__}
        cfg = cls(**{k: v for k, v in d.items() if k in known})
        cfg.mhc = MhcConfig(**mhc) if mhc else None
        return cfg

    def to_json(self) -> dict:
        d = asdict(self)
        return d


def nine_b() -> ModelConfig:
    """The 9B-shape model of the benchmarks: hidden 4096, FFN 12288 SwiGLU, 32 layers
    with every 4th a gated full-attention layer (16 Q / 4 KV heads, head_dim 256, 25%
    partial RoPE), the rest Gated DeltaNet (16 QK / 32 V heads of 128), layers 4..27
    looped twice, 2-stream mHC, vocab 248320. The mHC range (the looped block) and its
    20 Sinkhorn iterations are this build's choice (the HF config is not available)."""
    n = 32
    return ModelConfig(
        hidden=4096, intermediate=12288, vocab=248320, n_layers=n,
        full_attention=[(i + 1) % 4 == 0 for i in range(n)],
        n_heads=16, n_kv_heads=4, head_dim=256, rot_dim=64, rope_theta=1e7,
        lin_k_heads=16, lin_v_heads=32, lin_k_dim=128, lin_v_dim=128, conv_kernel=4, eps=1e-6,
        loop_start=4, loop_end=28, loop_count=2, mhc=MhcConfig(start=4, end=28, streams=2, iterations=20),
        mrope_section=[11, 11, 10], max_position=262144,
    )


def small() -> ModelConfig:
    """A reduced model with the same kernels and structure (DeltaNet + gated attention,
    a loop, mHC over the loop) that the CPU checker runs in seconds."""
    n = 8
    return ModelConfig(
        hidden=256, intermediate=512, vocab=2048, n_layers=n,
        full_attention=[(i + 1) % 4 == 0 for i in range(n)],
        n_heads=4, n_kv_heads=1, head_dim=256, rot_dim=64, rope_theta=1e7,
        lin_k_heads=2, lin_v_heads=4, lin_k_dim=128, lin_v_dim=128, conv_kernel=4, eps=1e-6,
        loop_start=2, loop_end=6, loop_count=2, mhc=MhcConfig(start=2, end=6, streams=2, iterations=20),
        mrope_section=[11, 11, 10], max_position=262144,
    )


def tp_test() -> ModelConfig:
    """A reduced model whose head counts and sizes divide by 8 (the 9B shape's 16 Q / 4
    KV heads and 16 / 32 DeltaNet heads, narrower layers), so tensor parallelism over
    2, 4 and 8 GPUs can be checked against the CPU restatement."""
    n = 8
    return ModelConfig(
        hidden=512, intermediate=2048, vocab=8192, n_layers=n,
        full_attention=[(i + 1) % 4 == 0 for i in range(n)],
        n_heads=16, n_kv_heads=4, head_dim=256, rot_dim=64, rope_theta=1e7,
        lin_k_heads=16, lin_v_heads=32, lin_k_dim=128, lin_v_dim=128, conv_kernel=4, eps=1e-6,
        loop_start=2, loop_end=6, loop_count=2, mhc=MhcConfig(start=2, end=6, streams=2, iterations=20),
        mrope_section=[11, 11, 10], max_position=262144,
    )
