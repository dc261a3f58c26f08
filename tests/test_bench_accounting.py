"""The algorithmic byte counts bench.py divides by, checked against the figures derived
from the model shapes: config 1's GEMV (12288 x 4096 Q8_0 blocks, an fp16 scale per 32
weights, plus x and y in f32) and the weight bytes one decode token of the 9B-shape
model streams (56 layer visits plus the LM head; in_proj and the LM head stay Q8_0 in a
Q4_0 model, as convert.rs:232-234 and :286-298 keep them)."""
import importlib.util
from pathlib import Path

from sensenova_b200.config import nine_b

ROOT = Path(__file__).resolve().parent.parent


def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config1_bytes():
    n, k = 12288, 4096
    assert bench().CONFIG1_BYTES == n * k + (n * k // 32) * 2 + 4 * k + 4 * n == 53_542_912


def test_weight_bytes_per_token_9b():
    b, cfg = bench(), nine_b()
    # 13,124,501,504 weight elements per decode token, all Q8_0: 34 bytes per 32.
    assert b.weight_bytes_per_token(cfg, "q8_0") == 13_124_501_504 * 34 // 32 == 13_944_782_848
    # Q4_0 (18 bytes per 32) everywhere but in_proj and the LM head.
    h = cfg.hidden
    q8_elems = cfg.vocab * h + sum(cfg.lin_proj_rows * h for l in cfg.execution_plan() if not cfg.full_attention[l])
    q4_elems = 13_124_501_504 - q8_elems
    assert b.weight_bytes_per_token(cfg, "q4_0") == q8_elems * 34 // 32 + q4_elems * 18 // 32 == 8_953_561_088
