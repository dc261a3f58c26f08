"""Tensor-parallel shard plan (snl_tp_plan, the plan finalize applies) on the CPU.

- Coverage: column-parallel row ranges and row-parallel column ranges tile each
  matrix (replicated only where ranks outnumber KV heads, as designed), and the
  DeltaNet parameter vector splits by head.
- Algebra: with float matrices, the sum over ranks of the row-parallel products of
  the column-parallel shards equals the unsharded MLP and o_proj (the Megatron split).
- N > 1 host path: two `gloo` ranks exchange handles with the engine's own gather and
  reduce their partial MLP outputs to the unsharded result.
"""
import ctypes as C
import os

import numpy as np
import pytest

from sensenova_b200 import ffi
from sensenova_b200.config import nine_b, small, tp_test


def plan(lib, cfg, rank, size, name):
    kind, n = C.c_int(), C.c_size_t()
    buf = (C.c_size_t * 32)()
    cc = cfg.to_c()
    ffi.check(lib.snl_tp_plan(C.byref(cc), rank, size, name.encode(), C.byref(kind), buf, 16, C.byref(n)))
    return kind.value, [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)]


def rows_of(ranges):
    out = []
    for a, n in ranges:
        out.extend(range(a, a + n))
    return out


def dims(cfg):
    q_dim, kv_dim = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    key_dim = cfg.lin_k_heads * cfg.lin_k_dim
    conv_dim = 2 * key_dim + cfg.lin_v_heads * cfg.lin_v_dim
    return dict(qkv=2 * q_dim + 2 * kv_dim, in_proj=conv_dim + cfg.lin_v_heads * cfg.lin_v_dim + 2 * cfg.lin_v_heads,
                gate_up=2 * cfg.intermediate, o_proj=q_dim, out_proj=cfg.lin_v_heads * cfg.lin_v_dim,
                down=cfg.intermediate, lm_head=cfg.vocab, lin=conv_dim * 4 + 2 * cfg.lin_v_heads + cfg.lin_v_dim,
                conv_dim=conv_dim)


CASES = [(nine_b, 2), (nine_b, 4), (nine_b, 8), (tp_test, 2), (tp_test, 4), (tp_test, 8), (small, 2)]


@pytest.mark.parametrize("mk,N", CASES)
def test_plan_tiles_every_matrix(lib, mk, N):
    cfg = mk()
    d = dims(cfg)
    for name, kind_want in (("l0.in_proj", ffi.SNL_TP_ROWS), ("l3.qkv", ffi.SNL_TP_ROWS), ("l0.gate_up", ffi.SNL_TP_ROWS),
                            ("lm_head", ffi.SNL_TP_ROWS), ("l3.o_proj", ffi.SNL_TP_COLS), ("l0.out_proj", ffi.SNL_TP_COLS),
                            ("l0.down", ffi.SNL_TP_COLS)):
        key = name.split(".")[-1]
        count = np.zeros(d[key], np.int64)
        for r in range(N):
            kind, rs = plan(lib, cfg, r, N, name)
            assert kind == kind_want, name
            idx = rows_of(rs)
            assert len(idx) == len(set(idx)), f"{name}: rank {r} repeats a row"
            count[idx] += 1
        if key == "qkv" and N > cfg.n_kv_heads:
            # each GQA group (its G query heads and one KV head) is computed by N / n_kv ranks
            assert (count == N // cfg.n_kv_heads).all(), name
        else:
            assert (count == 1).all(), f"{name}: rows covered {count.min()}..{count.max()} times"
    for name in ("embed", "l0.in_ln", "l0.mhc_attn", "norm", "l3.qk_norm"):
        assert plan(lib, cfg, 0, N, name) == (ffi.SNL_TP_FULL, [])


@pytest.mark.parametrize("mk,N", CASES)
def test_plan_splits_deltanet_params_by_head(lib, mk, N):
    cfg = mk()
    d = dims(cfg)
    cd, nv, dv = d["conv_dim"], cfg.lin_v_heads, cfg.lin_v_dim
    key_dim = cfg.lin_k_heads * cfg.lin_k_dim
    for r in range(N):
        kind, rs = plan(lib, cfg, r, N, "l0.lin")
        assert kind == ffi.SNL_TP_ELEMS
        # the local vector is [conv w of local q, k, v channels | A_log | dt_bias | norm w]
        _, inproj = plan(lib, cfg, r, N, "l0.in_proj")
        chans = rows_of(inproj[:3])
        assert rows_of(rs[:3]) == [4 * c + j for c in chans for j in range(4)]
        heads = [h for h in range(nv) if 2 * key_dim + h * dv in chans]
        assert rows_of([rs[3]]) == [cd * 4 + h for h in heads]
        assert rows_of([rs[4]]) == [cd * 4 + nv + h for h in heads]
        assert rows_of([rs[5]]) == list(range(cd * 4 + 2 * nv, cd * 4 + 2 * nv + dv))
        assert len(rows_of(rs)) == 4 * (2 * key_dim // N + nv * dv // N) + 2 * nv // N + dv


@pytest.mark.parametrize("mk,N", [(tp_test, 2), (tp_test, 4), (tp_test, 8)])
def test_megatron_split_reproduces_mlp_and_o_proj(lib, mk, N):
    cfg = mk()
    rng = np.random.default_rng(5)
    h, I = cfg.hidden, cfg.intermediate
    x = rng.standard_normal(h)
    gu = rng.standard_normal((2 * I, h)) / np.sqrt(h)
    dn = rng.standard_normal((h, I)) / np.sqrt(I)
    silu = lambda v: v / (1 + np.exp(-v))
    g = gu @ x
    full = dn @ (silu(g[:I]) * g[I:])
    acc = np.zeros(h)
    for r in range(N):
        _, gr = plan(lib, cfg, r, N, "l0.gate_up")
        _, (dc,) = plan(lib, cfg, r, N, "l0.down")
        gl = gu[rows_of(gr)] @ x
        il = len(gl) // 2
        acc += dn[:, dc[0]:dc[0] + dc[1]] @ (silu(gl[:il]) * gl[il:])
    assert np.abs(acc - full).max() < 1e-9 * np.abs(full).max() * 1e3
    # o_proj: each rank multiplies the attention output of the query heads it holds.
    q_dim = cfg.n_heads * cfg.head_dim
    att = rng.standard_normal(q_dim)
    op = rng.standard_normal((h, q_dim))
    acc = np.zeros(h)
    for r in range(N):
        _, ((c0, cn),) = plan(lib, cfg, r, N, "l3.o_proj")
        acc += op[:, c0:c0 + cn] @ att[c0:c0 + cn]
    assert np.allclose(acc, op @ att)


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist

    from sensenova_b200 import ffi as f
    from sensenova_b200.config import tp_test as mk
    from sensenova_b200.engine import gather_tp_handles

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        lib = f.load()
        cfg = mk()
        # the engine's handle exchange, with stand-in handles
        mine = bytes([rank + 1]) * f.SNL_TP_HANDLE_BYTES
        allh = gather_tp_handles(rank, world, mine, None)
        ok_handles = allh == b"".join(bytes([r + 1]) * f.SNL_TP_HANDLE_BYTES for r in range(world))
        # each rank's partial MLP output from its shard, summed across ranks
        rng = np.random.default_rng(9)
        h, I = cfg.hidden, cfg.intermediate
        x = rng.standard_normal(h)
        gu = rng.standard_normal((2 * I, h)) / np.sqrt(h)
        dn = rng.standard_normal((h, I)) / np.sqrt(I)
        silu = lambda v: v / (1 + np.exp(-v))
        _, gr = plan(lib, cfg, rank, world, "l0.gate_up")
        _, (dc,) = plan(lib, cfg, rank, world, "l0.down")
        gl = gu[rows_of(gr)] @ x
        il = len(gl) // 2
        part = torch.tensor(dn[:, dc[0]:dc[0] + dc[1]] @ (silu(gl[:il]) * gl[il:]))
        dist.all_reduce(part)
        g = gu @ x
        full = dn @ (silu(g[:I]) * g[I:])
        q.put((rank, ok_handles, float(np.abs(part.numpy() - full).max() / np.abs(full).max())))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, ok, err in res:
        assert ok, f"rank {rank}: handle exchange"
        assert err < 1e-12, err
