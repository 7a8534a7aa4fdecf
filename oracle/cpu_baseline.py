"""CPU baseline for bench.py -- TEST INFRASTRUCTURE (the only non-test user of
oracle/ is this module, called from bench.py's cpu_baseline leg and its
`--impl reference` arm).

It times the reference's own mv4i_matvec (ref/matvec_int4.c:329, compiled from
source into oracle/_ref/libref_mv4i.so; kind "reference") -- or, when that
library was not built, the restatement in liboracle.so (kind "port") -- on the
benchmark's config-0 matrix (4096 x 4096, seed 0, the golden-mode image of the
g128 weights: linear codebook, scales * 2^20, w_exp 5, x BFP-packed by the
reg_put rule), BFP output mode.

mv4i_matvec keeps file-static state and is not reentrant, so parallelism is
processes, each running the matvec on its own column-parallel row shard (the
reference's own tensor-parallel split, spec A 14.3); processes start with the
`spawn` method.
"""
import ctypes as C
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN_BYTES = 4096 * 4096 // 2 + 4096 * 128 * 2 + 4096 * 2 + 4096 * 2   # 9,453,568


def _synth():
    import importlib.util
    spec = importlib.util.spec_from_file_location("synth", os.path.join(ROOT, "llm.vhdl_b200", "synth.py"))
    S = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(S)
    return S


def _shard_image(p, P, M=4096, K=4096, seed=0):
    """Rows [p*M/P, (p+1)*M/P) of the config-0 matrix as a .mv4i image + x."""
    import oracle as O
    S = _synth()
    r0, r1 = p * M // P, (p + 1) * M // P
    wq = S.g128_weights(seed, M, K, rows=(r0, r1))
    sc = S.g128_scales(seed, M, K, rows=(r0, r1))
    idx, scl, w_exp = S.g128_to_golden(wq, sc, K)
    xm, xe = O.bfp_pack_f64(S.g128_x(seed, K).astype(np.float64))
    out_shift = 3   # calibrate_out_shift(4096), tools/pack_int4.py:434-446
    img = O.pack(r1 - r0, K, 4, 128, w_exp, out_shift, S.LINEAR_CB, idx, scl)
    return img, xm, xe, r1 - r0, K


def _worker(p, P, kind, barrier, n_iter, budget_s, q):
    sys.path.insert(0, ROOT)
    import oracle as O
    img, xm, xe, rows, K = _shard_image(p, P)
    fn = O.ref_matvec if kind == "reference" else O.matvec
    times = []
    t_end = time.perf_counter() + budget_s
    i = 0
    while True:
        if barrier is not None:
            barrier.wait()
        t0 = time.perf_counter()
        rc, _ = fn(img, xm, xe, rows, K, 0)
        times.append(time.perf_counter() - t0)
        assert rc == 0
        i += 1
        if n_iter is not None and i >= n_iter:
            break
        if n_iter is None and time.perf_counter() > t_end and i >= 2:
            break
    q.put((p, times))


def cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def kind():
    import oracle as O
    return "reference" if O.have_ref() else "port"


def run(P=None, n_iter=None, budget_s=3.0, lockstep=False):
    """Run P processes; returns per-step seconds (max over processes of each
    step when lockstep, else each process's mean) and the kind."""
    P = P or cores()
    k = kind()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    barrier = ctx.Barrier(P) if lockstep else None
    procs = [ctx.Process(target=_worker, args=(p, P, k, barrier, n_iter, budget_s, q)) for p in range(P)]
    for pr in procs:
        pr.start()
    res = dict(q.get() for _ in procs)
    for pr in procs:
        pr.join()
    if lockstep:
        n = min(len(t) for t in res.values())
        steps = [max(res[p][i] for p in res) for i in range(n)]
    else:
        steps = [max(float(np.mean(t)) for t in res.values())]
    return steps, k, P
