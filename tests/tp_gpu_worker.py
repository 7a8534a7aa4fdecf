"""Rank process for tests/test_tp_gpu.py (launched by torchrun, one per GPU).

Row-parallel golden block: every rank uploads its own K-slice of the same
matrix, BFP-packs its own x slice, runs the PARTIAL-mode kernel, the partials
travel over NCCL (all-gather), and every rank reduces with mv4i_tp_reduce; the
result must equal the CPU oracle's reduction of the same partials bit for bit
and be identical on all ranks.  Then a g128 row-parallel block: fp32 partials,
NCCL all-reduce, against the double-precision product of the whole matrix.
Exits 0 on success.
"""
import ctypes as C
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main():
    import torch
    import torch.distributed as dist
    from conftest import load_package
    pkg = load_package()
    import llmvhdl_b200.tp as TP
    import llmvhdl_b200.synth as S

    import oracle as O
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    L = pkg.lib()
    dev = torch.device("cuda", rank)

    # ---- golden row-parallel (config-4 down projection shape, scaled)
    M, K = 5120, 17408 // 4
    rng = np.random.default_rng(7)
    idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
    scl = rng.integers(4000, 32000, (M, K // 32), dtype=np.uint16)
    u = rng.integers(-(1 << 22), 1 << 22, K)
    k0, kn = TP.split(K, world, rank, align=128)
    img = O.pack(M, kn, 4, 128, 2, 9, O.IQ4_NL, idx[:, k0:k0 + kn], scl[:, k0 // 32:(k0 + kn) // 32])
    xs = np.zeros(kn, np.int16)
    x_exp = O.orc().orc_bfp_pack_s64(u[k0:k0 + kn].astype(np.int64).ctypes.data_as(C.c_void_p), kn, 16,
                                     xs.ctypes.data_as(C.c_void_p))
    pi = pkg.ParsedImage(img)
    dm = pkg.DMat()
    assert L.mv4i_dmat_upload(C.byref(pi.f), rank, C.byref(dm)) == 0
    dx = torch.from_numpy(xs).to(dev)
    ya = torch.zeros(M, dtype=torch.int64, device=dev)
    st = torch.zeros(8, dtype=torch.int32, device=dev)
    scratch = torch.zeros(L.mv4i_scratch_bytes(), dtype=torch.uint8, device=dev)
    j = pkg.Job()
    j.w = C.pointer(dm); j.x = dx.data_ptr(); j.x_exp = x_exp; j.n_rows = M; j.n_cols = kn
    j.mode = 2; j.nvec = 1; j.y_acc = ya.data_ptr(); j.status = st.data_ptr()
    assert L.mv4i_launch(C.byref(j), 1, C.c_void_p(scratch.data_ptr()), None) == 0
    torch.cuda.synchronize()
    y_exp = int(st[0].item())
    rc, r = O.matvec(img, xs, x_exp, M, kn, 2)
    assert rc == 0 and np.array_equal(ya.cpu().numpy(), r["y_acc"]) and y_exp == r["y_exp"]
    out, y32, status = TP.row_parallel_golden(ya, y_exp, 9, lambda p, e, o: TP.reduce_partials_device(L, p, e, o))
    torch.cuda.synchronize()
    parts, ye, osh = TP.gather_partials(ya, y_exp, 9)
    prc, oout, oexp, oy32, osat = O.tp_reduce(list(parts.cpu().numpy()), list(ye.cpu().numpy()),
                                            list(osh.cpu().numpy()))
    assert prc == 0 and int(status[4].item()) == 0
    assert np.array_equal(out.cpu().numpy(), oout) and int(status[0].item()) == oexp
    out32 = out.to(torch.int32)                     # NCCL has no int16
    allo = [torch.empty_like(out32) for _ in range(world)]
    dist.all_gather(allo, out32)
    assert all(torch.equal(allo[0], a) for a in allo)

    # ---- g128 row-parallel: fp32 partials + all-reduce
    M2, K2 = 2048, 6144
    wq = torch.empty((M2, K2 // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((M2, K2 // 128), dtype=torch.float16, device=dev)
    x = torch.empty(K2, dtype=torch.float16, device=dev)
    assert L.mv4i_synth_g128(5, 1, M2, K2, C.c_void_p(wq.data_ptr()), C.c_void_p(sc.data_ptr()),
                             C.c_void_p(x.data_ptr()), None) == 0
    c0, cn = TP.split(K2, world, rank, align=128)
    wsl = wq[:, c0 // 2:(c0 + cn) // 2].contiguous()
    ssl = sc[:, c0 // 128:(c0 + cn) // 128].contiguous()
    xsl = x[c0:c0 + cn].contiguous()
    dm2 = pkg.DMat()
    assert L.mv4i_dmat_wrap_g128(C.c_void_p(wsl.data_ptr()), cn // 2, C.c_void_p(ssl.data_ptr()), cn // 128,
                                 M2, cn, rank, C.byref(dm2)) == 0
    y = torch.zeros(M2, dtype=torch.float32, device=dev)
    j2 = pkg.Job()
    j2.w = C.pointer(dm2); j2.x = xsl.data_ptr(); j2.n_rows = M2; j2.n_cols = cn; j2.nvec = 1
    j2.y_f32 = y.data_ptr()
    assert L.mv4i_launch(C.byref(j2), 1, None, None) == 0
    TP.row_parallel_fp32(y)
    torch.cuda.synchronize()
    ref = O.matvec_g128_f64(wq.cpu().numpy(), sc.cpu().numpy(), x.cpu().numpy(), K2)
    err = np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-4, err
    L.mv4i_dmat_free(C.byref(dm))
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_GPU_OK world=%d golden bit-exact, g128 rel err %.2e" % (world, err))


if __name__ == "__main__":
    main()
