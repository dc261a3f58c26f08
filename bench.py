#!/usr/bin/env python
"""Benchmark: decode tok/s at batch 1 on the synthetic 9B-shape Q8_0 model, with the
Q8_0 GEMV's achieved HBM bandwidth against the measured peak.

One step = one greedy decode token of the 9B-shape model (56 layer visits + the
248320-row LM head) after a 2048-token prefill of uniform random ids (BASELINE.json
configs[2]). `value` is device-timed (CUDA events on the engine stream) with every
step's inputs resident in HBM and the argmax fed back on the device; `e2e` is the same
metric through the public API with the token crossing host->device and the next token
device->host every step. The weights (13.9 GB streamed per token) are far larger than
L2, so no L2 flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) the N ranks decode ONE stream together, tensor-parallel: every
quantized matrix is split by rows or columns across the GPUs and the partial sums are
exchanged over NVLink peer memory inside the GEMV epilogue ("scaling": "strong"); time is
the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "sense-nova-server_b200"))

METRIC = "decode tok/s @bs1 Q8_0 9B-shape; Q8 GEMV achieved HBM GB/s vs peak"
PUBLISHED_DECODE_TOK_S = 38.0  # the reference's published decode: ~38 tok/s, batch 1, Q8_0 (RTX 5080, README.md:218)
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--quant", default="q8_0", choices=["q8_0", "q4_0"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--e2e-logits-steps", type=int, default=16)
    ap.add_argument("--no-gemv", action="store_true", help="skip the standalone config-1 GEMV timing")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle parity check (and with it the CPU baseline)")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the BASELINE configs[4] leg (Q4_0 model, 32K context)")
    ap.add_argument("--cpu-budget-s", type=float, default=25.0)
    ap.add_argument("--profile", action="store_true", help="print the per-op table of one decode step")
    ap.add_argument("--turns", type=int, default=4, help="mtp workload: turns (BASELINE configs[3] names 1000)")
    ap.add_argument("--worker-turns", type=int, default=None,
                    help="mtp workload: turns of the snl_worker pass (default: --turns)")
    ap.add_argument("--workload", choices=["decode", "gemv", "gemm", "deltanet", "mtp", "vision"], default="decode",
                    help="gemv: only BASELINE configs[0], the one-token Q8_0 GEMV 12288x4096; "
                         "gemm: one prefill-chunk GEMM (512 tokens x 12288 x 4096) on the tcgen05 kernel")
    ap.add_argument("--iters", type=int, default=40)
    ap.add_argument("--grid", type=int, default=32, help="vision workload: patches per image side")
    ap.add_argument("--gemv-kernel", choices=["tile", "tc", "simt"], default="tile")
    ap.add_argument("--gemm-dequant", action="store_true",
                    help="gemm workload: dequantize in the kernel instead of the engine's weight planes")
    return ap.parse_args()


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, phys_index: int):
        self.idx = phys_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def phys_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


CONFIG1_BYTES = 12288 * 4096 + 12288 * 4096 // 32 * 2 + 4 * 4096 + 4 * 12288  # codes, fp16 block scales, x, y


# ---- CPU side (oracle): the reference's algorithm restated in C++ ------------------------------


def oracle_model(cfg, quant: str, seed: int, ctx: int = 64):
    """The CPU restatement of the reference's kernels (oracle/) for the same seeded model,
    on every host thread (torchrun sets OMP_NUM_THREADS=1 in its workers; the oracle's
    thread count is set explicitly). Returns (oracle module, model, build seconds)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc  # test/baseline infrastructure only

    orc.set_threads(cores())
    t0 = time.perf_counter()
    m = orc.OracleModel(cfg, ctx, seed=seed, quant={"q8_0": 1, "q4_0": 2}[quant])
    return orc, m, time.perf_counter() - t0


def parity_prompt(cfg, seed: int, n: int = 4) -> list[int]:
    return [int(v) for v in np.random.default_rng(seed).integers(0, cfg.vocab, n)]


def first_max(v: np.ndarray) -> int:
    """sampler.rs:169-177 on a host row: the first maximum."""
    return int(np.argmax(v))


PARITY_STEPS = 8


def gpu_parity_run(eng, prompt: list[int], steps: int = PARITY_STEPS):
    """The engine on the parity prompt, twice from a reset state: (a) forward_mm with the
    logits row every step (host argmax), (b) the product greedy path: forward_greedy for
    the prompt, then the device decode loop. Returns (tokens a, logits a, tokens b)."""
    eng.reset()
    lg = [eng.forward(prompt, True)]
    toks = [first_max(lg[0])]
    for _ in range(steps):
        lg.append(eng.forward([toks[-1]], True))
        toks.append(first_max(lg[-1]))
    eng.reset()
    t0 = eng.forward_greedy(prompt, None, 1)[0]
    gen, _ = eng.generate(t0, steps)
    eng.reset()
    return toks, lg, [t0] + list(gen)


def oracle_parity(orc, m, prompt: list[int], gpu_tokens: list[int], gpu_logits: list, greedy_tokens: list[int]):
    """Greedy decode of the oracle on the same prompt (its own tokens fed back), compared
    forward by forward with the GPU's logits: max |gpu - oracle| / max |oracle| per step,
    identical tokens, and at the first differing token the oracle's top-2 gap."""
    lo = m.forward(prompt, True)
    rels, toks, flip = [], [], None
    for i in range(len(gpu_logits)):
        if i:
            lo = m.forward([toks[-1]], True)
        rels.append(float(np.abs(gpu_logits[i].astype(np.float64) - lo).max() / max(np.abs(lo).max(), 1e-30)))
        toks.append(orc.argmax(lo))
        if flip is None and toks[-1] != gpu_tokens[i]:
            top = np.sort(lo)[-2:]
            flip = {"step": i, "oracle": toks[-1], "gpu": gpu_tokens[i], "oracle_top2_gap": float(top[1] - top[0])}
    return {"logits_rel_max": max(rels), "logits_rel_per_step": rels, "tokens_oracle": toks,
            "tokens_gpu_logits_path": gpu_tokens, "tokens_gpu_greedy_path": greedy_tokens,
            "tokens_identical": toks == gpu_tokens == greedy_tokens, "first_flip": flip,
            "tolerance": 1e-3, "within_tolerance": max(rels) < 1e-3}


def oracle_decode(m, orc, first: int, warmup: int, steps: int, budget_s: float):
    """Greedy decode steps of the oracle model from token `first`: `warmup` untimed, then
    up to `steps` timed (fewer when `budget_s` of CPU time runs out). Returns (tok/s, steps)."""
    tok = first
    for _ in range(warmup):
        tok = orc.argmax(m.forward([tok], True))
    n, t = 0, 0.0
    while n < steps and (n == 0 or t < budget_s):
        t1 = time.perf_counter()
        tok = orc.argmax(m.forward([tok], True))
        t += time.perf_counter() - t1
        n += 1
    return n / t, n


def weight_bytes_per_token(cfg, quant: str) -> int:
    """Q8_0/Q4_0 block bytes (codes + an fp16 scale per 32 weights: 34 and 18 bytes) of
    every matrix one decode token streams (56 layer visits + LM head); in_proj and
    lm_head stay Q8_0 (convert.rs:232-234, :286-298). The tile layout the decode GEMV
    reads holds exactly these bytes."""
    h, inter = cfg.hidden, cfg.intermediate
    q8 = lambda r, k: r * k * 34 / 32
    qq = (lambda r, k: r * k * 34 / 32) if quant == "q8_0" else (lambda r, k: r * k * 18 / 32)
    tot = q8(cfg.vocab, h)
    for l in cfg.execution_plan():
        if cfg.full_attention[l]:
            tot += qq(cfg.attn_proj_rows, h) + qq(h, cfg.q_dim)
        else:
            tot += q8(cfg.lin_proj_rows, h) + qq(h, cfg.lin_value_dim)
        tot += qq(2 * inter, h) + qq(h, inter)
    return int(tot)


def gemv_config1(lib, quant: str, copies: int = 8, iters: int = 40, kernel: str = "tile") -> dict:
    """one-token Q8_0 GEMV, W [12288 x 4096], x fp32 ~N(0,1),
    timed alone with CUDA events on the launching stream. `copies` weight copies
    (8 x 56.7 MB > L2) rotate so every launch reads its weights from HBM."""
    import ctypes as C

    import torch

    from sensenova_b200 import ffi

    n, k = 12288, 4096
    dt = ffi.SNL_Q8_0 if quant == "q8_0" else ffi.SNL_Q4_0
    qb = n * k if dt == ffi.SNL_Q8_0 else n * k // 2
    ws = [torch.empty(qb, dtype=torch.uint8, device="cuda") for _ in range(copies)]
    ss = [torch.empty(n * k // 32, dtype=torch.float32, device="cuda") for _ in range(copies)]
    for i in range(copies):
        ffi.check(lib.snl_synth_quant(100 + i, b"gemv", dt, n, k, C.c_void_p(ws[i].data_ptr()),
                                      C.c_void_p(ss[i].data_ptr()), None))
    x = torch.randn(k, device="cuda")
    y = torch.empty(n, device="cuda")
    st, p = ffi.StepU(1, 0, 1, 0), ffi.MatP(n, k, 0, k, 0, n, 0, 0)
    planes = torch.empty(2 * k, dtype=torch.float16, device="cuda")
    ffi.check(lib.snl_xpack(C.c_void_p(x.data_ptr()), 1, k, k, C.c_void_p(planes.data_ptr()), None))
    tiles, tsc = [], []
    scale_mode = "f32"  # the file layout's scales (snl_mat, snl_mat_xpack)
    if kernel == "tile":
        tb, sf = C.c_size_t(), C.c_size_t()
        ffi.check(lib.snl_tile_sizes(dt, n, k, C.byref(tb), C.byref(sf)))
        for i in range(copies):
            tiles.append(torch.empty(tb.value, dtype=torch.uint8, device="cuda"))
            tsc.append(torch.empty(sf.value, dtype=torch.uint8, device="cuda"))
            f16 = C.c_int(-1)
            ffi.check(lib.snl_tile_repack(dt, n, k, C.c_void_p(ws[i].data_ptr()), C.c_void_p(ss[i].data_ptr()),
                                          C.c_void_p(tiles[i].data_ptr()), C.c_void_p(tsc[i].data_ptr()),
                                          C.byref(f16), None))
            scale_mode = "fp16" if f16.value else "f32"

    def run(i, stream=None):
        if kernel == "tile":  # the decode path: tile layout, tensor-core GEMV over packed x
            ffi.check(lib.snl_mat_tiles(dt, C.byref(p), 1, C.c_void_p(planes.data_ptr()), C.c_void_p(tiles[i].data_ptr()),
                                        C.c_void_p(tsc[i].data_ptr()), 1 if scale_mode == "fp16" else 0,
                                        C.c_void_p(y.data_ptr()), stream))
        elif kernel == "tc":  # tensor-core GEMV on the file layout
            ffi.check(lib.snl_mat_xpack(dt, C.byref(p), 1, C.c_void_p(planes.data_ptr()), C.c_void_p(ws[i].data_ptr()),
                                        C.c_void_p(ss[i].data_ptr()), C.c_void_p(y.data_ptr()), stream))
        else:  # snl_mat: the SIMT kernels of the kernel-level entry point
            ffi.check(lib.snl_mat(dt, C.byref(st), C.byref(p), C.c_void_p(x.data_ptr()), C.c_void_p(ws[i].data_ptr()),
                                  C.c_void_p(ss[i].data_ptr()), C.c_void_p(y.data_ptr()), stream))

    for i in range(2 * copies):
        run(i % copies)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(iters):
        run(i % copies)
    b.record()
    torch.cuda.synchronize()
    us_eager = a.elapsed_time(b) * 1000.0 / iters
    # The same launches captured in one CUDA graph, as the decode step runs its kernels:
    # no host launch cost between them, programmatic dependent launch kept. Timed with
    # CUDA events on the graph's stream around whole replays.
    us_graph = None
    if kernel == "tile":
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            run(0, C.c_void_p(side.cuda_stream))  # first call on this stream outside the capture
            side.synchronize()
            with torch.cuda.graph(graph, stream=side):
                for i in range(iters):
                    run(i % copies, C.c_void_p(side.cuda_stream))
            graph.replay()
            side.synchronize()
            reps = 5
            a.record(side)
            for _ in range(reps):
                graph.replay()
            b.record(side)
            side.synchronize()
        us_graph = a.elapsed_time(b) * 1000.0 / (reps * iters)
        del graph
    us = us_graph if us_graph is not None else us_eager
    # Algorithmic bytes: Q8_0/Q4_0 blocks (codes + an fp16 scale per 32), x, y.
    nbytes = qb + n * k // 32 * 2 + 4 * k + 4 * n
    return {"shape": [n, k], "quant": quant, "scales": scale_mode, "kernel": kernel, "us_per_launch": us, "iters": iters,
            "timing": "CUDA graph of the launches" if us_graph is not None else "eager launches",
            "us_per_launch_eager": us_eager, "achieved_gbs_eager": nbytes / (us_eager * 1e3),
            "bytes_per_launch": nbytes,
            "achieved_gbs": nbytes / (us * 1e3), "copies_rotated": copies}


def cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's kernels (the reference is
    a Rust/wgpu crate that cannot be built or run here), greedy decode of the same 9B-shape
    model on all host threads, W warm-up and K timed steps (fewer if ~150 s of CPU time
    runs out). Under torchrun only rank 0 runs it."""
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    from sensenova_b200.config import nine_b

    cfg = nine_b()
    budget = 150.0
    orc, m, build_s = oracle_model(cfg, args.quant, args.seed)
    prompt = parity_prompt(cfg, args.seed)
    first = orc.argmax(m.forward(prompt, True))
    v, n = oracle_decode(m, orc, first, args.warmup, args.steps, budget)
    thr = orc.threads()
    m.close()
    sample = (f"oracle/ (the reference's kernels restated in C++, bit-identical to its WGSL translated and run on the "
              f"host, tests/test_reference_shaders.py): "
              f"9B-shape {args.quant} greedy decode after a {len(prompt)}-token prompt, {args.warmup} warm-up and "
              f"{n} timed tokens (of --steps {args.steps}; capped at ~{budget:.0f} s of CPU work), {thr} OpenMP "
              f"threads, weights generated in {build_s:.0f} s. The prompt is short because a 2048-token prefill "
              f"costs ~54 TFLOP on the CPU; the KV reads at 2K context are <1% of a decode step's bytes")
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": world, "steps": n,
        "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": v / PUBLISHED_DECODE_TOK_S, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"9B-shape {args.quant} greedy decode bs1 after a {len(prompt)}-token prompt",
                   "quant": args.quant, "prompt_tokens": len(prompt)},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": thr, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = CPU restatement of the reference's WGSL kernels (oracle/); the Rust/wgpu reference "
                "cannot be built or run here (no Rust toolchain, no graphics stack)",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    from sensenova_b200 import ffi
    from sensenova_b200.config import nine_b
    from sensenova_b200.engine import Engine

    lib = ffi.load()
    cfg = nine_b()
    K, W = args.steps, max(args.warmup, 3)
    ctx = args.prompt + W + K + args.e2e_steps + 40
    t0 = time.perf_counter()
    # N > 1: one decode stream sharded over the N GPUs (tensor parallel, one process per GPU).
    tp = (rank, world) if world > 1 else None
    eng = Engine.synthetic(cfg, ctx, args.seed, args.quant, device=local_rank, tp=tp)
    n16, n32 = eng.tile_scales()
    scale_mode = f"tile layout: {n16} matrices with fp16 block scales, {n32} with f32"
    build_s = time.perf_counter() - t0

    rng = np.random.default_rng(args.seed)  # every rank feeds the same stream
    prompt = rng.integers(0, cfg.vocab, args.prompt).tolist()

    # Prefill warm-up: one 512-row step (the timed prefill's kernels, their one-time setup
    # and the GPU's clocks), then the engine is reset to an empty context.
    eng.forward_greedy(prompt[:512], None, 1)
    eng.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok = eng.forward_greedy(prompt, None, 1)[0]
    prefill_s = time.perf_counter() - t0

    toks, _ = eng.generate(tok, W)  # warm-up (also captures the decode graph)
    tok = toks[-1]

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(phys_gpu_index(local_rank))
    l0 = lib.snl_launch_count()
    barrier()
    clocks.start()
    gen, ms = eng.generate(tok, K)
    barrier()
    clk = clocks.stop()
    launches = lib.snl_launch_count() - l0
    tok = gen[-1]
    ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = K / (ms_max / 1000.0)  # tokens of the one stream the N GPUs produce together

    # e2e through the public API: token in from host memory, token out to host memory.
    E = args.e2e_steps
    barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        tok = eng.forward_greedy([tok], None, 1)[0]
    barrier()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e = E / float(e2e_t.item())
    # the reference's own call returns the full logits row every token (engine.rs:917-931)
    El = max(args.e2e_logits_steps, 1)
    t0 = time.perf_counter()
    for _ in range(El):
        lg = eng.forward([tok], True)
        tok = int(np.argmax(lg))
    torch.cuda.synchronize()
    e2e_logits = El / (time.perf_counter() - t0)
    # the reference's default sampler (sampler.rs:17-29: temperature 1, top-p 0.95, top-k 20)
    # on the device: the logits stay there, the token comes back (snl_engine_sample)
    Es = max(args.e2e_logits_steps, 1)
    sp = ffi.SampleP(1.0, 0.95, 20, 0.0, 0.0, 0.0, 1.0, 0)
    srng = np.random.default_rng(args.seed + 7)
    hist: dict[int, int] = {}
    t0 = time.perf_counter()
    for _ in range(Es):
        eng.forward_keep([tok], 1)
        tok, _, _ = eng.sample(0, sp, hist, srng.random(2))
        hist[tok] = hist.get(tok, 0) + 1
    e2e_sampled = Es / (time.perf_counter() - t0)

    # One eager decode step op by op, each launch bracketed by CUDA events on the engine
    # stream (so no launch overlaps its predecessor, unlike the captured step): a per-op
    # table of time and algorithmic GB/s, reported beside the device-timed step.
    prof = eng.profile(tok)
    step_ms = sum(r["ms"] for r in prof)
    ops = [{"op": r["label"], "calls": r["calls"], "ms": round(r["ms"], 4), "share": round(r["ms"] / step_ms, 4),
            "gbs": round(r["bytes"] / (r["ms"] * 1e6), 1) if r["ms"] > 0 else 0.0}
           for r in sorted(prof, key=lambda r: -r["ms"])]
    peak, peak_kind = peaks()
    if rank == 0 and args.profile:
        eng.print_profile(prof)
    g1 = None if args.no_gemv else gemv_config1(lib, args.quant)
    # The metric's "GEMV achieved HBM GB/s vs peak" is the config-1 GEMV (BASELINE.json
    # configs[0]): its launches timed back to back with CUDA events on the launching stream.
    # DRAM traffic needs an ncu capture, which this run does not make: null here.
    roofline = None
    if g1:
        roofline = {"bound": "hbm", "achieved": g1["achieved_gbs"], "peak": peak, "unit": "GB/s",
                    "frac": g1["achieved_gbs"] / peak, "traffic": None,
                    "kernel": f"gemv_pg_kernel, BASELINE configs[0] ({args.quant.upper()} 12288x4096, one token): "
                              f"{g1['bytes_per_launch']} algorithmic bytes per launch / {g1['us_per_launch']:.2f} us "
                              f"average over {g1['iters']} back-to-back launches captured in a CUDA graph, as in the decode "
                              f"step (CUDA events around the replays on the graph's stream; eager launches: "
                              f"{g1['us_per_launch_eager']:.2f} us)",
                    "peak_kind": f"{peak_kind} hbm_gbs (burst)"}

    # Parity on this configuration, after the timed legs (the CPU oracle runs only now): the
    # engine (every rank under tensor parallelism), reset, against the oracle's unsharded
    # model of the same seed, on a short prompt and PARITY_STEPS greedy steps; rank 0 runs
    # the oracle.
    pprompt = parity_prompt(cfg, args.seed)
    ptoks, plogits, pgreedy = gpu_parity_run(eng, pprompt) if not args.no_parity else ([], [], [])
    ranks_agree = True
    if dist and ptoks:
        mine = torch.tensor(ptoks + pgreedy, dtype=torch.int64, device="cuda")
        allt = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allt, mine)
        ranks_agree = all(bool((t == mine).all()) for t in allt)
    parity = orc = om = None
    if rank == 0 and not args.no_parity:
        orc, om, obuild_s = oracle_model(cfg, args.quant, args.seed)
        parity = oracle_parity(orc, om, pprompt, ptoks, plogits, pgreedy)
        parity.update({"config": f"9B-shape {args.quant}", "prompt_tokens": len(pprompt), "steps": PARITY_STEPS,
                       "ranks_agree": ranks_agree, "device_error": int(lib.snl_device_error(1)),
                       "oracle_threads": orc.threads()})
    if dist:
        dist.barrier()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and om is not None:
        # the oracle model of the parity check, decoding on from where it stopped
        v, n = oracle_decode(om, orc, parity["tokens_oracle"][-1], 0, 32, args.cpu_budget_s)
        cpu = {"value": v, "unit": "tok/s", "cores": orc.threads(), "kind": "port",
               "sample": f"oracle/ (C++ restatement of the WGSL kernels, bit-identical to the reference's WGSL "
                         f"translated and run on the host; OpenMP, AVX2) greedy decode of the same "
                         f"9B-shape {args.quant} model after a {len(pprompt)}-token prompt, {n} tokens timed; KV "
                         f"reads at 2K context are <1% of the 13.9 GB weight stream, so a short context stands in"}
    if om is not None:
        om.close()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": value / PUBLISHED_DECODE_TOK_S, "dtype": "int8 weights, x as fp16 hi+lo (~22 bits), fp32 accumulate",
            "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
            "config": {"workload": f"9B-shape {args.quant} greedy decode bs1 after a {args.prompt}-token prefill",
                       "prompt_tokens": args.prompt, "decode_tokens": K, "quant": args.quant, "scales": scale_mode,
                       "weight_bytes_per_token": weight_bytes_per_token(cfg, args.quant),
                       "l2": f"inputs larger than L2 ({weight_bytes_per_token(cfg, args.quant) / 1e9:.1f} GB of weights streamed per token)",
                       "parallelism": f"tp{world}" if world > 1 else "single"},
            "roofline": roofline,
            "parity": parity,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 + 16 + 16, "d2h_bytes_per_step": 4,
                    "api": "snl_engine_forward_greedy"},
            "e2e_sampled": {"value": e2e_sampled, "unit": "tok/s", "d2h_bytes_per_step": 12,
                            "api": "snl_engine_forward_mm (logits kept on the device) + snl_engine_sample "
                                   "(temperature 1, top-p 0.95, top-k 20)"},
            "e2e_logits": {"value": e2e_logits, "unit": "tok/s", "d2h_bytes_per_step": 4 * cfg.vocab,
                           "api": "snl_engine_forward_mm (full logits row, as engine.rs:917-931)"},
            "gpu_launches": int(launches),
            "clocks": clk,
            "prefill_tok_s": args.prompt / prefill_s,
            "step_ops_each_timed_alone": {"total_ms": step_ms, "ops": ops},
            "build_s": build_s,
        }
        if g1:
            g1["frac"] = g1["achieved_gbs"] / peak
            line["gemv_config1"] = g1
        if cpu:
            line["cpu_baseline"] = cpu
    eng.close()
    c4 = None if args.no_config4 else config4_leg(args, cfg, world, local_rank, dist, peak)
    if rank == 0:
        if c4:
            line["config4"] = c4
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def config4_leg(args, cfg, world, local_rank, dist, peak):
    """the same model in Q4_0 (in_proj, embedding and LM head
    stay Q8_0) at a 32K context, batch-1 greedy decode, on the run's N GPUs (tensor
    parallel when N > 1). A 32,768-token prefill of uniform random ids, then `steps`
    greedy tokens timed on the device (CUDA events, max over ranks)."""
    import torch

    from sensenova_b200.engine import Engine

    prompt_n, steps, warm = 32768, 32, 4
    tp = (int(os.environ.get("RANK", 0)), world) if world > 1 else None
    eng = Engine.synthetic(cfg, prompt_n + warm + steps + 8, args.seed, "q4_0", device=local_rank, tp=tp)
    prompt = np.random.default_rng(args.seed + 4).integers(0, cfg.vocab, prompt_n).tolist()
    eng.forward_greedy(prompt[:512], None, 1)  # prefill warm-up, as in the headline leg
    eng.reset()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok = eng.forward_greedy(prompt, None, 1)[0]
    prefill_s = time.perf_counter() - t0
    toks, _ = eng.generate(tok, warm)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    _, ms = eng.generate(toks[-1], steps)
    ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    eng.close()
    wb = weight_bytes_per_token(cfg, "q4_0")
    kv = 2 * 2 * cfg.n_kv_heads * cfg.head_dim * sum(1 for l in cfg.execution_plan() if cfg.full_attention[l]) * prompt_n
    tok_s = steps / (ms / 1000.0)
    return {"workload": "BASELINE configs[4]: 9B-shape Q4_0 greedy decode bs1 at a 32K context "
                        "(32768-token prefill of uniform random ids)",
            "value": tok_s, "unit": "tok/s", "steps": steps, "warmup": warm, "ms_per_step": ms / steps,
            "n_gpus": world, "parallelism": f"tp{world}" if world > 1 else "single",
            "prefill_tok_s": prompt_n / prefill_s,
            "bytes_per_token": {"weights": wb, "kv_cache_at_32k": kv},
            "hbm_frac": (wb + kv) / world * tok_s / (peak * 1e9)}


def run_gemv_only(args):
    import torch

    from sensenova_b200 import ffi

    torch.cuda.set_device(0)
    lib = ffi.load()
    g = gemv_config1(lib, args.quant, iters=args.iters, kernel=args.gemv_kernel)
    peak, kind = peaks()
    g["frac"] = g["achieved_gbs"] / peak
    g["peak"] = peak
    print(json.dumps({"workload": "gemv config1", **g}), flush=True)
    return 0


def run_deltanet(args):
    """one Gated DeltaNet layer (16 QK / 32 V heads of 128,
    fp32 state [32,128,128]). Inputs as the config states: q, k, v, b, a, z ~ N(0,1)
    (q, k L2-normalised and beta = sigmoid(b) inside the kernel), A_log = 0 and
    dt_bias = 0 (g = -softplus(a)), conv weights N(0, 0.5), norm weight 1. A prefill of
    4096 tokens in the engine's 512-row steps, then 256 recurrent single-token steps,
    through the engine's fused conv + delta kernel (snl_conv_delta)."""
    import ctypes as C

    import torch

    from sensenova_b200 import ffi

    torch.cuda.set_device(0)
    lib = ffi.load()
    n_k, n_v, D = 16, 32, 128
    cd = 2 * n_k * D + n_v * D
    stride = cd + n_v * D + 2 * n_v
    lp = ffi.LinP(cd, stride, n_k, n_v, 1e-6, (0, 0, 0))
    T, R, chunk = 4096, 256, 512
    rng = np.random.default_rng(args.seed)
    proj = rng.standard_normal((T + R, stride)).astype(np.float32)
    lw = np.concatenate([np.sqrt(0.5) * rng.standard_normal(cd * 4), np.zeros(2 * n_v), np.ones(D)]).astype(np.float32)
    dp, dlw = torch.from_numpy(proj).cuda(), torch.from_numpy(lw).cuda()
    cs, S = torch.zeros(3 * cd, device="cuda"), torch.zeros(n_v * D * D, device="cuda")
    out = torch.zeros((T + R) * n_v * D, device="cuda")
    ptr = lambda t: C.c_void_p(t.data_ptr())

    def step(r0, m):
        st = ffi.StepU(m, r0, 1, 0)
        ffi.check(lib.snl_conv_delta(C.byref(st), C.byref(lp), C.c_void_p(dp.data_ptr() + 4 * r0 * stride), ptr(cs),
                                     ptr(S), ptr(dlw), C.c_void_p(out.data_ptr() + 4 * r0 * n_v * D), None, None, None))

    def timed(fn):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    for _ in range(max(args.warmup, 3)):  # warm-up on a scratch copy of the state
        step(0, chunk)
    cs.zero_()
    S.zero_()
    pf_ms = timed(lambda: [step(c, chunk) for c in range(0, T, chunk)])
    dec_ms = timed(lambda: [step(T + i, 1) for i in range(R)])
    # CPU reference on a bounded sample: the oracle's conv + delta over 64 tokens
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc

    nS = 64
    conv_out = np.zeros((nS, cd), np.float32)
    cs_h, S_h, o_h = np.zeros((3, cd), np.float32), np.zeros((n_v, D, D), np.float32), np.zeros((nS, n_v * D), np.float32)
    stc = ffi.StepU(nS, 0, 1, 0)
    t0 = time.perf_counter()
    orc.conv(stc, lp, proj[:nS], conv_out, cs_h, lw, np.zeros((3, cd), np.float32))
    orc.delta(stc, lp, proj[:nS], conv_out, S_h, lw, o_h, np.zeros_like(S_h))
    cpu_s = time.perf_counter() - t0
    line = {
        "metric": "Gated DeltaNet layer: prefill tok/s (4096 tokens) and recurrent us/token",
        "value": T / (pf_ms / 1000.0), "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
        "prefill_ms": pf_ms, "decode_us_per_token": dec_ms * 1000.0 / R, "decode_tok_s": R / (dec_ms / 1000.0),
        "dtype": "f32", "data": "synthetic (BASELINE configs[1] distributions)",
        "config": {"workload": "BASELINE configs[1]: DeltaNet 16/32 heads x 128, 4096-token prefill in 512-row steps "
                               "then 256 single-token steps",
                   "kernel": "prefill: conv_kernel + chunked gated delta rule (dn_prep_tc_kernel, dn_scan_tc_kernel: "
                             "tcgen05 fp16 hi/lo products into tensor memory; dn_norm_kernel; 64-token chunks); "
                             "decode: conv_delta_split_kernel"},
        "roofline": {"bound": "latency (chunk-sequential state carry; token-sequential recurrence in decode)",
                     "state_bytes_per_token": 2 * n_v * D * D * 4},
        "cpu_baseline": {"value": nS / cpu_s, "unit": "tok/s", "cores": 1, "kind": "port",
                         "sample": f"oracle conv + delta over {nS} tokens"},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_mtp(args):
    """the 9B-shape model with its MTP head. A 12K-token prefix
    is prefilled once (with the MTP layer fed, as worker.rs:330-336) and snapshotted;
    every turn restores it, feeds fresh random ids up to 16K, then decodes greedily with
    draft-1 / verify-2 speculation exactly as worker.rs:197-255 (accept iff the verify
    row's argmax is the draft, else roll back). Reports the acceptance rate and tok/s."""
    import torch

    from sensenova_b200.config import nine_b
    from sensenova_b200.engine import Engine

    torch.cuda.set_device(0)
    cfg = nine_b()
    prefix, full, dec = 12288, 16384, 32
    eng = Engine.synthetic(cfg, full + dec + 64, args.seed, args.quant, mtp=True)
    rng = np.random.default_rng(args.seed)
    chunk = 512

    def feed(toks, start):
        lg = None
        for c0 in range(0, len(toks), chunk):
            c1 = min(c0 + chunk, len(toks))
            pos = [[start + i] * 3 for i in range(c0, c1)]
            lg = eng.forward_mm(toks[c0:c1], pos, (), 1 if c1 == len(toks) else 0, False)
            a, r0 = start + c0, 1 if start + c0 == 0 else 0
            if r0 < c1 - c0:
                eng.mtp(r0, toks[c0 + r0:c1], [[a + i - 1] * 3 for i in range(r0, c1 - c0)], a + r0 - 1, False)
        return lg

    t0 = time.perf_counter()
    prefix_ids = rng.integers(0, cfg.vocab, prefix).tolist()
    feed(prefix_ids, 0)
    eng.snapshot(0)
    torch.cuda.synchronize()
    prefix_s = time.perf_counter() - t0
    drafted = accepted = produced = 0
    dec_s = feed_s = 0.0
    for turn in range(args.turns):
        eng.restore(0, prefix)
        t1 = time.perf_counter()
        lg = feed(rng.integers(0, cfg.vocab, full - prefix).tolist(), prefix)
        torch.cuda.synchronize()
        feed_s += time.perf_counter() - t1
        t2 = time.perf_counter()
        tok = int(np.argmax(lg[0]))
        rope = full
        mtp_in = (eng.hid_rows(), [tok], [[full - 1] * 3], full - 1)
        n_out = 0
        while n_out < dec:
            r0, toks, pos, slot0 = mtp_in
            d = eng.mtp(r0, toks, pos, slot0, True)
            slot = eng.pos
            a0, a1 = eng.forward_greedy([tok, d], [[rope] * 3, [rope + 1] * 3], 2, True)
            drafted += 1
            if a0 == d:
                accepted += 1
                n_out += 2
                tok = a1
                mtp_in = (1, [d, tok], [[rope] * 3, [rope + 1] * 3], slot)
                rope += 2
            else:
                eng.rollback()
                n_out += 1
                tok = a0
                mtp_in = (1, [tok], [[rope] * 3], slot)
                rope += 1
        torch.cuda.synchronize()
        dec_s += time.perf_counter() - t2
        produced += n_out
    # The same turns through the generation loop (snl_worker, worker.rs:118-270): each turn
    # is a request whose prompt is the 12K prefix plus fresh ids, with a snapshot at the
    # prefix. Turn 0 runs cold and leaves the snapshot; later turns restore it. The loop
    # drafts with the MTP head and pauses drafting when the drafts do not pay off.
    from sensenova_b200.worker import GREEDY, Worker

    w = Worker(eng)
    wk = {"turns": 0, "tokens": 0, "decode_s": 0.0, "prefill_s": 0.0, "drafted": 0, "accepted": 0, "cached": 0}
    cold_prefill_s = 0.0
    worker_turns = args.turns if args.worker_turns is None else args.worker_turns
    for turn in range(worker_turns + 1):
        prompt = prefix_ids + rng.integers(0, cfg.vocab, full - prefix).tolist()
        _, fin = w.run(prompt, GREEDY, dec, snapshot_at=prefix)
        wk["drafted"] += fin.drafted
        wk["accepted"] += fin.accepted
        if turn == 0:
            cold_prefill_s = fin.prefill_secs
            continue
        wk["turns"] += 1
        wk["tokens"] += fin.completion_tokens
        wk["decode_s"] += fin.decode_secs
        wk["prefill_s"] += fin.prefill_secs
        wk["cached"] += fin.cached_tokens
    spec_on, pause = w.spec()
    w.close()
    line = {
        "metric": "MTP speculative decode at 16K context: acceptance rate and tok/s",
        "value": produced / dec_s, "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
        "acceptance": accepted / max(drafted, 1), "drafted": drafted, "accepted": accepted,
        "e2e_tok_s_with_feed": produced / (dec_s + feed_s), "feed_tok_s": args.turns * (full - prefix) / feed_s,
        "prefix_prefill_s": prefix_s, "turns": args.turns, "dtype": "int8 weights, x as fp16 hi+lo (~22 bits), fp32 accumulate", "data": "synthetic",
        "worker": {
            "what": "the same turns as requests to snl_worker_run (prefix cache, drafting with self-pause)",
            "decode_tok_s": wk["tokens"] / max(wk["decode_s"], 1e-9),
            "e2e_tok_s_with_feed": wk["tokens"] / max(wk["decode_s"] + wk["prefill_s"], 1e-9),
            "feed_tok_s": wk["turns"] * (full - prefix) / max(wk["prefill_s"], 1e-9),
            "cached_tokens_per_turn": wk["cached"] / max(wk["turns"], 1),
            "cold_turn_prefill_s": cold_prefill_s,
            "drafted": wk["drafted"], "accepted": wk["accepted"],
            "acceptance": wk["accepted"] / max(wk["drafted"], 1),
            "drafting_after": {"on": spec_on, "pause_requests_left": pause},
        },
        "config": {"workload": f"BASELINE configs[3]: 12K-token prefix snapshot, feed to 16K, {dec} tokens per turn "
                               f"with draft-1/verify-2, {args.turns} turns"
                               + ("" if args.turns >= 1000 else " (1000 named; bounded sample)")
                               + f"; worker pass {worker_turns} turns",
                   "quant": args.quant},
    }
    print(json.dumps(line), flush=True)
    eng.close()
    return 0


def run_gemm_only(args):
    """One prefill chunk's largest matrix product: 512 token rows x W [12288 x 4096] in
    Q8_0 (or Q4_0), the shape of BASELINE configs[2]'s 2048-token prefill in 512-row
    steps, through snl_mat (which routes >= 8 rows to the tcgen05 GEMM). Weight copies
    rotate so each launch reads its weights from HBM; CUDA events on the launching stream.
    Achieved TFLOP/s counts the op's 2*m*n*k (the kernel's three fp16 hi/lo products are
    3x that on the tensor pipe)."""
    import ctypes as C

    import torch

    from sensenova_b200 import ffi

    torch.cuda.set_device(0)
    lib = ffi.load()
    m, n, k, copies = 512, 12288, 4096, 4
    dt = ffi.SNL_Q8_0 if args.quant == "q8_0" else ffi.SNL_Q4_0
    qb = n * k if dt == ffi.SNL_Q8_0 else n * k // 2
    ws = [torch.empty(qb, dtype=torch.uint8, device="cuda") for _ in range(copies)]
    ss = [torch.empty(n * k // 32, dtype=torch.float32, device="cuda") for _ in range(copies)]
    for i in range(copies):
        ffi.check(lib.snl_synth_quant(200 + i, b"gemm", dt, n, k, C.c_void_p(ws[i].data_ptr()),
                                      C.c_void_p(ss[i].data_ptr()), None))
    x = torch.randn(m, k, device="cuda")
    y = torch.empty(m, n, device="cuda")
    st, p = ffi.StepU(m, 0, 1, 0), ffi.MatP(n, k, 0, k, 0, n, 0, 0)
    # The engine's form: the weights' fp16 hi/lo planes made once, loaded by TMA
    # (--gemm-dequant: the kernel dequantizes the file layout itself).
    planes = []
    if not args.gemm_dequant:
        for i in range(copies):
            planes.append(torch.empty(2 * n * k, dtype=torch.float16, device="cuda"))
            ffi.check(lib.snl_weight_planes(dt, n, k, C.c_void_p(ws[i].data_ptr()), C.c_void_p(ss[i].data_ptr()),
                                            C.c_void_p(planes[i].data_ptr()), None))

    def run(i):
        if planes:
            ffi.check(lib.snl_mat_wplanes(dt, C.byref(st), C.byref(p), C.c_void_p(x.data_ptr()),
                                          C.c_void_p(ws[i].data_ptr()), C.c_void_p(ss[i].data_ptr()),
                                          C.c_void_p(planes[i].data_ptr()), C.c_void_p(y.data_ptr()), None))
        else:
            ffi.check(lib.snl_mat(dt, C.byref(st), C.byref(p), C.c_void_p(x.data_ptr()), C.c_void_p(ws[i].data_ptr()),
                                  C.c_void_p(ss[i].data_ptr()), C.c_void_p(y.data_ptr()), None))

    for i in range(2 * copies):
        run(i % copies)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.iters):
        run(i % copies)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1000.0 / args.iters
    flops = 2.0 * m * n * k
    try:
        pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        peak, kind = float(pk["bf16_tflops"]), "measured bf16_tflops (burst)"
    except Exception:
        peak, kind = 1590.0, "fallback"
    wbytes = qb + n * k // 32 * 4
    print(json.dumps({"workload": "prefill GEMM", "shape": [m, n, k], "quant": args.quant,
                      "a_operand": "dequantized in the kernel" if args.gemm_dequant else "weight planes by TMA",
                      "us_per_launch": us,
                      "tflops": flops / us / 1e6, "peak_tflops": peak, "peak_kind": kind,
                      "frac": flops / us / 1e6 / peak, "tensor_pipe_flops_per_launch": 3 * flops,
                      "weight_bytes": wbytes, "weight_gbs": wbytes / us / 1e3, "copies_rotated": copies}), flush=True)
    return 0


def run_vision(args):
    """The vision tower (vision.rs Vision::encode) on one image of grid x grid patches, at a
    Qwen3-VL-sized configuration (hidden 1152, 27 blocks, 16 heads of 72, MLP 4304 padded
    to 4320, 16-pixel patches over 2 frames, 2x2 merge to 4096). Seeded synthetic weights
    and patches. Times snl_vision_encode end to end (patches from the host, features back)."""
    import torch

    from sensenova_b200.vision import Vision, VisionConfig

    torch.cuda.set_device(0)
    cfg = VisionConfig()
    v = Vision.synthetic(cfg, seed=args.seed)
    g = args.grid
    n = g * g
    patches = np.random.default_rng(args.seed).standard_normal((1, n, cfg.patch_dim())).astype(np.float32)
    for _ in range(max(args.warmup, 3)):
        v.encode(patches, 1, g, g)
    torch.cuda.synchronize()
    iters = max(1, min(args.iters, 20))
    t0 = time.perf_counter()
    for _ in range(iters):
        out = v.encode(patches, 1, g, g)
    dt = (time.perf_counter() - t0) / iters
    h, ip, md = cfg.hidden, cfg.intermediate_padded, cfg.merged_dim()
    gemm = 2.0 * n * (cfg.patch_dim() * h + cfg.depth * (3 * h * h + h * h + 2 * ip * h)) \
        + 2.0 * (n // 4) * (md * md + md * cfg.out_hidden)
    attn = cfg.depth * 4.0 * n * n * h
    print(json.dumps({
        "workload": "vision tower encode (vision.rs:176-311), one frame", "grid": [g, g], "patches": n,
        "out_tokens": n // 4, "ms_per_frame": dt * 1e3, "frames_per_s": 1.0 / dt,
        "out_tokens_per_s": (n // 4) / dt, "gemm_gflop": gemm / 1e9, "attention_gflop": attn / 1e9,
        "tflops_total": (gemm + attn) / dt / 1e12, "dtype": "f32 (int8 weights)", "data": "synthetic",
        "output_finite": bool(np.isfinite(out).all()),
        "config": {k: getattr(cfg, k) for k in ("hidden", "intermediate", "depth", "n_heads", "patch",
                                                "temporal_patch", "merge", "out_hidden", "pos_side")},
    }), flush=True)
    v.close()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "gemv":
        return run_gemv_only(args)
    if args.workload == "gemm":
        return run_gemm_only(args)
    if args.workload == "deltanet":
        return run_deltanet(args)
    if args.workload == "mtp":
        return run_mtp(args)
    if args.workload == "vision":
        return run_vision(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
