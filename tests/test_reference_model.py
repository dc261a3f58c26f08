"""The whole forward pass from the reference's own kernels against the oracle model.

oracle/wgslref_model.py composes the reference's WGSL kernels (translated to C++ and run
on the host cores) in the op order of src/engine.rs:383-493 and forward_mm (:801-936),
on the oracle model's weights (Q8_0, and the Q4_0 model of BASELINE configs[4]). Every kernel call of the reduced model's graph (DeltaNet
and attention layers, the mHC loop, split-key attention with several parts, the LM head)
must give the oracle's bits, through a prefill and greedy decode steps.
"""
import numpy as np
import pytest

import oracle as orc
import wgslref as wr
from sensenova_b200.config import small

pytestmark = pytest.mark.skipif(not wr.available(), reason="reference tree absent")


@pytest.mark.parametrize("quant", [1, 2], ids=["q8_0", "q4_0"])
def test_reference_kernels_forward_matches_oracle_model(quant):
    from wgslref_model import RefModel

    cfg = small()
    ctx = 320
    om = orc.OracleModel(cfg, ctx, seed=3, quant=quant)
    rm = RefModel(cfg, ctx, om)
    prompt = [(17 + 7919 * i) % cfg.vocab for i in range(258)]  # one tiled-matmul chunk
    lo, lr = om.forward(prompt, True), rm.forward(prompt, True)
    # decode steps past 256 keys: the split-key attention runs with two parts and combine
    steps = 0
    while True:
        assert np.array_equal(lo.view(np.uint32), lr.view(np.uint32)), f"logits differ at step {steps}"
        tok = int(np.argmax(lo))
        steps += 1
        if steps > 3:
            break
        lo, lr = om.forward([tok], True), rm.forward([tok], True)
    om.close()


def test_reference_kernels_mtp_matches_oracle_model():
    """Engine::mtp (engine.rs:700-774) from the reference's kernels: the MTP layer over a
    prompt's hidden rows, then a one-pair draft, logits bit-identical to the oracle's."""
    from wgslref_model import RefModel

    cfg = small()
    ctx = 64
    om = orc.OracleModel(cfg, ctx, seed=4, mtp=True)
    rm = RefModel(cfg, ctx, om)
    prompt = [(29 + 104729 * i) % cfg.vocab for i in range(9)]
    lo, lr = om.forward(prompt, True), rm.forward(prompt, True)
    assert np.array_equal(lo, lr)
    nxt = int(np.argmax(lo))
    # pairs (hidden row i + 1, token i + 1): the prompt's rows with the tokens that follow them
    toks = prompt[1:] + [nxt]
    pos = [[i, i, i] for i in range(len(toks))]
    d_o = om.mtp(1, toks, pos, 0, True)
    lr_m = rm.mtp(1, toks, pos, 0, True)
    lo_m = om.mtp_logits()
    assert np.array_equal(lo_m.view(np.uint32), lr_m.view(np.uint32))
    assert d_o == int(np.argmax(lr_m))
    om.close()


@pytest.mark.parametrize("frames,h,w", [(1, 4, 6), (2, 4, 4)])
def test_reference_kernels_vision_encode_matches_oracle(frames, h, w):
    """Vision::encode (vision.rs:195-343) from the reference's vision and matmul kernels on
    the oracle tower's weights: output rows bit-identical to the oracle's encode."""
    from sensenova_b200.vision import small_vision
    from wgslref_model import RefVision

    cfg = small_vision()
    ov = orc.OracleVision(cfg, seed=5)
    patches = np.random.default_rng(h * w + frames).standard_normal((frames, h * w, cfg.patch_dim())).astype(np.float32)
    want = ov.encode(patches, frames, h, w)
    got = RefVision(cfg, ov).encode(patches, frames, h, w)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
    ov.close()
