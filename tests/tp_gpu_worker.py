"""Rank process for tests/test_tp_gpu.py (launched by torchrun, one per GPU).

Row-parallel golden block: every rank uploads its own K-slice of the same
matrix, BFP-packs its own x slice, runs the PARTIAL-mode kernel, and
mv4i_tp_row_parallel (the library's NCCL communicator) all-gathers the E
messages (partials + {y_exp, out_shift, sequence}) and reduces them on every
rank; the result must equal the CPU oracle's reduction of the same partials
bit for bit and be identical on all ranks.  A second collective whose
sequence number one rank gets wrong is refused (-15) on every rank.  Then a
g128 row-parallel block: fp32 partials, mv4i_tp_allreduce_f32, against the
double-precision product of the whole matrix.  torch.distributed only ships
the communicator's id and compares the ranks' results.  Exits 0 on success.
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
    from conftest import load_package, split
    pkg = load_package()

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
    k0, kn = split(K, world, rank, align=128)
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
    # the library's communicator: rank 0's id shipped over torch.distributed
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        h = (C.c_uint8 * 128)()
        assert L.mv4i_tp_unique_id(h) == 0
        uid = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=dev)
    dist.broadcast(uid, 0)
    comm = C.c_void_p()
    assert L.mv4i_tp_comm_create((C.c_uint8 * 128)(*uid.cpu().tolist()), rank, world, rank, C.byref(comm)) == 0
    mb = L.mv4i_tp_msg_bytes(M)
    work = torch.zeros((world + 1) * mb, dtype=torch.uint8, device=dev)
    out = torch.zeros(M, dtype=torch.int16, device=dev)
    y32 = torch.zeros(M, dtype=torch.int32, device=dev)
    status = torch.zeros(8, dtype=torch.int32, device=dev)
    assert L.mv4i_tp_row_parallel(comm, C.c_void_p(ya.data_ptr()), M, C.c_void_p(st.data_ptr()), 9, 1,
                                  C.c_void_p(work.data_ptr()), C.c_void_p(out.data_ptr()),
                                  C.c_void_p(y32.data_ptr()), C.c_void_p(status.data_ptr()), None) == 0
    torch.cuda.synchronize()
    recv = work[:world * mb].cpu().numpy().reshape(world, mb)
    parts = [recv[c, :8 * M].view(np.int64) for c in range(world)]
    ye = [int(recv[c, mb - 16:mb - 12].view(np.int32)[0]) for c in range(world)]
    osh = [int(recv[c, mb - 12:mb - 8].view(np.int32)[0]) for c in range(world)]
    assert ye[rank] == y_exp and osh == [9] * world
    prc, oout, oexp, oy32, osat = O.tp_reduce(parts, ye, osh)
    assert prc == 0 and int(status[4].item()) == 0
    assert np.array_equal(out.cpu().numpy(), oout) and int(status[0].item()) == oexp
    assert np.array_equal(y32.cpu().numpy(), oy32)
    out32 = out.to(torch.int32)                     # NCCL has no int16
    allo = [torch.empty_like(out32) for _ in range(world)]
    dist.all_gather(allo, out32)
    assert all(torch.equal(allo[0], a) for a in allo)
    # the next collective with the last rank one sequence number behind: refused everywhere
    out.zero_()
    assert L.mv4i_tp_row_parallel(comm, C.c_void_p(ya.data_ptr()), M, C.c_void_p(st.data_ptr()), 9,
                                  2 if rank < world - 1 else 1, C.c_void_p(work.data_ptr()),
                                  C.c_void_p(out.data_ptr()), C.c_void_p(y32.data_ptr()),
                                  C.c_void_p(status.data_ptr()), None) == 0
    torch.cuda.synchronize()
    want = -15
    assert int(status[4].item()) == want and not out.any().item(), int(status[4].item())

    # ---- g128 row-parallel: fp32 partials + all-reduce
    M2, K2 = 2048, 6144
    wq = torch.empty((M2, K2 // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((M2, K2 // 128), dtype=torch.float16, device=dev)
    x = torch.empty(K2, dtype=torch.float16, device=dev)
    assert L.mv4i_synth_g128(5, 1, M2, K2, C.c_void_p(wq.data_ptr()), C.c_void_p(sc.data_ptr()),
                             C.c_void_p(x.data_ptr()), None) == 0
    c0, cn = split(K2, world, rank, align=128)
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
    assert L.mv4i_tp_allreduce_f32(comm, C.c_void_p(y.data_ptr()), M2, None) == 0
    torch.cuda.synchronize()
    ref = O.matvec_g128_f64(wq.cpu().numpy(), sc.cpu().numpy(), x.cpu().numpy(), K2)
    err = np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-4, err
    L.mv4i_dmat_free(C.byref(dm))
    assert L.mv4i_tp_comm_destroy(comm) == 0
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_GPU_OK world=%d golden bit-exact, g128 rel err %.2e" % (world, err))


if __name__ == "__main__":
    main()
