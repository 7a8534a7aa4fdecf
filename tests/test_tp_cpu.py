"""Tensor-parallel host logic on CPU: world_size 2 (and 4) gloo ranks.

Each rank packs its own K-slice of a matrix (the reference's row-parallel
split, ref/matvec_int4.c:1124-1197 emulates the same in one process),
BFP-packs its own x slice, runs PARTIAL mode (the CPU oracle stands in for
the GPU matvec here), and writes its E message -- payload, then the trailer
{y_exp, out_shift, sequence number}, sequence last -- with the library's
mv4i_tp_msg_pack.  The messages travel by a gloo all-gather (the transport a
host-side caller might use; GPUs use mv4i_tp_row_parallel's NCCL
all-gather), every rank checks them with the library's mv4i_tp_msgs_check,
and the E 2.1 reduction (the oracle's, standing in for the device's) must
give the same answer on every rank and stay within the reference's stated
bound of the exact sum.  Refusals on every rank alike: a y_exp spread above
17, an out_shift mismatch, and a message carrying the previous collective's
sequence number (E 2.3).  Failure paths are made on the host: a rank that
leaves before the collective.
"""
import os
import socket
import sys

import ctypes as C

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
        from conftest import load_package, split
        pkg = load_package()
        L = pkg.lib()

        import oracle as O
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=20))
        M, K = 64, 1024
        rng = np.random.default_rng(42)                       # same matrix on every rank
        idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
        scl = rng.integers(8000, 32000, (M, K // 32), dtype=np.uint16)
        u = rng.integers(-(1 << 24), 1 << 24, K)              # the producer's s32-grid activation
        k0, kn = split(K, world, rank, align=128)
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

        seq = 41                                              # this collective's sequence number
        try:
            mb = L.mv4i_tp_msg_bytes(M)
            msg = np.zeros(mb, np.uint8)
            my_seq = seq - 1 if (mode == "stale" and rank == world - 1) else seq
            assert L.mv4i_tp_msg_pack(r["y_acc"].ctypes.data, M, r["y_exp"], out_shift, my_seq, msg.ctypes.data) == 0
            bufs = [torch.empty(mb, dtype=torch.uint8) for _ in range(world)]
            dist.all_gather(bufs, torch.from_numpy(msg))
            arrs = [b.numpy() for b in bufs]
            ptrs = (C.c_void_p * world)(*[a.ctypes.data for a in arrs])
            ye = np.zeros(world, np.int32)
            osh = np.zeros(world, np.int32)
            lrc = L.mv4i_tp_msgs_check(world, M, ptrs, seq, ye.ctypes.data, osh.ctypes.data)
            parts = [a[:8 * M].view(np.int64).copy() for a in arrs]
            prc, out, oe, y32, sat = O.tp_reduce(parts, list(ye), list(osh)) if lrc != -15 else (None,) * 5
            q.put((rank, (lrc, prc, None if out is None else out.tolist(), oe,
                          None if y32 is None else y32.tolist(), r["y_exp"])))
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
    lrc0, prc0, out0, oe0, y320, _ = res[0]
    assert lrc0 == 0 and prc0 == 0
    for r in range(1, world):
        assert res[r][:5] == (lrc0, prc0, out0, oe0, y320), r
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
    assert [res[r][0] for r in range(2)] == [-13, -13], res   # the library's check
    assert [res[r][1] for r in range(2)] == [-2, -2], res     # the oracle's code for the same refusal


def test_spread_over_17_refused_everywhere():
    res = _run(2, "spread")
    assert [res[r][0] for r in range(2)] == [-12, -12], res
    assert [res[r][1] for r in range(2)] == [-1, -1], res


@pytest.mark.parametrize("world", [2, 4])
def test_stale_sequence_refused_everywhere(world):
    """One rank's message carries the previous collective's sequence number
    (E 2.3: a stale flag read as completion): every rank refuses it (-15)."""
    res = _run(world, "stale")
    assert [res[r][0] for r in range(world)] == [-15] * world, res


def test_rank_that_leaves_fails_the_collective_not_the_host():
    res = _run(2, "leave")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error"), res


def test_msg_pack_and_check_on_the_host(pkg):
    """The message format on one host: payload, trailer, sequence word last;
    a message of another collective, and each refusal, detected."""
    L = pkg.lib()
    M = 37
    mb = L.mv4i_tp_msg_bytes(M)
    assert mb == ((8 * M + 15) // 16) * 16 + 16 and L.mv4i_tp_msg_bytes(0) == 0
    rng = np.random.default_rng(3)
    msgs = []
    for c in range(3):
        y = rng.integers(-(1 << 40), 1 << 40, M)
        m = np.zeros(mb, np.uint8)
        assert L.mv4i_tp_msg_pack(y.ctypes.data, M, 20 + c, 7, 5, m.ctypes.data) == 0
        assert np.array_equal(m[:8 * M].view(np.int64), y)
        assert list(m[mb - 16:].view(np.int32)[:3].astype(np.int64)) == [20 + c, 7, 5]
        msgs.append(m)

    def check(seq):
        ye, osh = np.zeros(3, np.int32), np.zeros(3, np.int32)
        ptrs = (C.c_void_p * 3)(*[m.ctypes.data for m in msgs])
        return L.mv4i_tp_msgs_check(3, M, ptrs, seq, ye.ctypes.data, osh.ctypes.data), list(ye), list(osh)
    assert check(5) == (0, [20, 21, 22], [7, 7, 7])
    assert check(6)[0] == -15 and check(4)[0] == -15
    msgs[1][mb - 12:mb - 8] = np.array([8], np.int32).view(np.uint8)       # out_shift of rank 1
    assert check(5)[0] == -13
    msgs[1][mb - 12:mb - 8] = np.array([7], np.int32).view(np.uint8)
    msgs[2][mb - 16:mb - 12] = np.array([20 + 18], np.int32).view(np.uint8)  # y_exp spread 18
    assert check(5)[0] == -12
