"""Tensor-parallel host logic on CPU: world_size 2 (and 4) gloo ranks.

Each rank packs its own K-slice of a matrix (the reference's row-parallel
split, ref/matvec_int4.c:1124-1197 emulates the same in one process),
BFP-packs its own x slice, runs PARTIAL mode (the CPU oracle stands in for
the GPU matvec here), and the partials are all-gathered through
llm.vhdl_b200.tp; the E 2.1 reduction (the oracle's, standing in for
mv4i_tp_reduce) must give the same answer on every rank, stay within the
reference's stated bound of the exact sum, and refuse a y_exp spread above 17
or an out_shift mismatch on every rank alike.  Failure paths are made on the
host: a rank that leaves before the collective, and a mismatched shard.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        sys.path.insert(0, ROOT)
        import datetime

        import torch
        import torch.distributed as dist
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from conftest import load_package
        load_package()
        import llmvhdl_b200.tp as TP

        import oracle as O
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=20))
        M, K = 64, 1024
        rng = np.random.default_rng(42)                       # same matrix on every rank
        idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
        scl = rng.integers(8000, 32000, (M, K // 32), dtype=np.uint16)
        u = rng.integers(-(1 << 24), 1 << 24, K)              # the producer's s32-grid activation
        k0, kn = TP.split(K, world, rank, align=128)
        out_shift = 8 if mode != "oshift" or rank == 0 else 9
        img = O.pack(M, kn, 4, 128, 1, out_shift, O.IQ4_NL, idx[:, k0:k0 + kn],
                     scl[:, k0 // 32:(k0 + kn) // 32])
        # each rank packs ITS OWN slice: a per-rank exponent, as in production
        span = u[k0:k0 + kn] >> (0 if mode != "spread" else (20 * rank))
        xs = np.zeros(kn, np.int16)
        import ctypes as C
        x_exp = O.orc().orc_bfp_pack_s64(span.astype(np.int64).ctypes.data_as(C.c_void_p), kn, 20,
                                         xs.ctypes.data_as(C.c_void_p))
        if mode == "spread" and rank == 1:
            x_exp -= 30                                      # beyond the contractual spread of 17
        rc, r = O.matvec(img, xs, x_exp, M, kn, 2)
        assert rc == 0
        if mode == "leave" and rank == 1:
            q.put((rank, "left"))
            return                                            # never joins the collective

        def reduce_fn(parts, ye, osh):
            prc, out, oe, y32, sat = O.tp_reduce(list(parts.numpy()), list(ye.numpy()), list(osh.numpy()))
            return prc, out, oe, y32

        try:
            prc, out, oe, y32 = TP.row_parallel_golden(torch.from_numpy(r["y_acc"]), r["y_exp"],
                                                       out_shift, reduce_fn)
            q.put((rank, (prc, out.tolist(), oe, y32.tolist(), r["y_exp"])))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error: " + type(e).__name__))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "crash: %r" % (e,)))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, v = q.get(timeout=120)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_golden_identical_on_ranks(world):
    res = _run(world, "ok")
    assert all(isinstance(v, tuple) for v in res.values()), res
    rc0, out0, oe0, y320, _ = res[0]
    assert rc0 == 0
    for r in range(1, world):
        assert res[r][:4] == (rc0, out0, oe0, y320), r
    exps = [res[r][4] for r in range(world)]
    assert len(set(exps)) >= 1
    # the reduced value is close to the unsharded product (15.4b: bounded loss)
    import oracle as O
    M, K = 64, 1024
    rng = np.random.default_rng(42)
    idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
    scl = rng.integers(8000, 32000, (M, K // 32), dtype=np.uint16)
    u = rng.integers(-(1 << 24), 1 << 24, K)
    exact = (O.IQ4_NL[idx].astype(np.float64) * np.repeat(scl, 32, axis=1) / 32768.0) @ u.astype(np.float64)
    exact *= 2.0 ** -(1 + 20)
    got = np.array(out0, np.float64) * 2.0 ** -oe0
    assert np.max(np.abs(got - exact)) <= 2e-3 * np.max(np.abs(exact))


def test_out_shift_mismatch_refused_everywhere():
    res = _run(2, "oshift")
    assert [res[r][0] for r in range(2)] == [-2, -2], res     # oracle code for -13


def test_spread_over_17_refused_everywhere():
    res = _run(2, "spread")
    assert [res[r][0] for r in range(2)] == [-1, -1], res     # oracle code for -12


def test_rank_that_leaves_fails_the_collective_not_the_host():
    res = _run(2, "leave")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error"), res
