"""Tensor-parallel reduction on GPUs.

* one GPU: N shards emulated in one process (as the reference's 15.4b tests
  do, ref/matvec_int4.c:1124-1197) -- mv4i_tp_reduce, and the message form
  mv4i_tp_msg_pack_dev + mv4i_tp_reduce_msgs, bit-exact against the
  oracle's E 2.1 reduction for N = 2, 4, 8, including the refusals and a
  message of another collective (-15);
* two or more GPUs: tests/tp_gpu_worker.py under torchrun, the messages over
  NCCL through mv4i_tp_row_parallel.
"""
import ctypes as C
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reduce_flat(L, torch, parts, ye, osh):
    N, M = len(parts), len(parts[0])
    dp = torch.from_numpy(np.stack(parts)).cuda()
    dye = torch.tensor(ye, dtype=torch.int32).cuda()
    dos = torch.tensor(osh, dtype=torch.int32).cuda()
    out = torch.empty(M, dtype=torch.int16, device="cuda")
    y32 = torch.empty(M, dtype=torch.int32, device="cuda")
    st = torch.zeros(8, dtype=torch.int32, device="cuda")
    assert L.mv4i_tp_reduce(N, M, C.c_void_p(dp.data_ptr()), C.c_void_p(dye.data_ptr()),
                            C.c_void_p(dos.data_ptr()), C.c_void_p(out.data_ptr()), C.c_void_p(y32.data_ptr()),
                            C.c_void_p(st.data_ptr()), None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy(), y32.cpu().numpy(), st.cpu().numpy()


def _reduce_msgs(L, torch, parts, ye, osh, seqs, seq):
    """Each shard's message written on the device, then the reduction of all N."""
    N, M = len(parts), len(parts[0])
    mb = L.mv4i_tp_msg_bytes(M)
    msgs = torch.zeros(N * mb, dtype=torch.uint8, device="cuda")
    for c in range(N):
        pa = torch.from_numpy(np.asarray(parts[c], np.int64)).cuda()
        assert L.mv4i_tp_msg_pack_dev(C.c_void_p(pa.data_ptr()), M, None, ye[c], osh[c], seqs[c],
                                      C.c_void_p(msgs.data_ptr() + c * mb), None) == 0
        torch.cuda.synchronize()
    out = torch.zeros(M, dtype=torch.int16, device="cuda")
    y32 = torch.zeros(M, dtype=torch.int32, device="cuda")
    st = torch.zeros(8, dtype=torch.int32, device="cuda")
    assert L.mv4i_tp_reduce_msgs(N, M, C.c_void_p(msgs.data_ptr()), seq, C.c_void_p(out.data_ptr()),
                                 C.c_void_p(y32.data_ptr()), C.c_void_p(st.data_ptr()), None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy(), y32.cpu().numpy(), st.cpu().numpy()


@pytest.mark.parametrize("N", [2, 4, 8])
def test_tp_reduce_emulated_shards(cuda, pkg, N):
    torch = cuda
    L = pkg.lib()
    rng = np.random.default_rng(N)
    M = 5120
    for case in ("ok", "spread", "oshift", "stale"):
        parts = [rng.integers(-(1 << 44), 1 << 44, M) for _ in range(N)]
        ye = [int(v) for v in rng.integers(20, 30, N)]
        osh = [9] * N
        if case == "spread":
            ye[-1] = ye[0] + 18 if ye[0] + 18 > max(ye[:-1]) else max(ye) + 18
        if case == "oshift":
            osh[-1] = 10
        prc, oout, oexp, oy32, osat = O.tp_reduce(parts, ye, osh)
        seqs = [77] * N
        if case == "stale":
            seqs[N // 2] = 76
        mout, my32, mst = _reduce_msgs(L, torch, parts, ye, osh, seqs, 77)
        if case == "stale":
            assert mst[4] == -15 and not mout.any()            # refused before anything was summed
            continue
        out, y32, st = _reduce_flat(L, torch, parts, ye, osh)
        if case == "ok":
            assert prc == 0 and st[4] == 0 and mst[4] == 0
            assert np.array_equal(out, oout) and np.array_equal(y32, oy32)
            assert np.array_equal(mout, oout) and np.array_equal(my32, oy32)
            assert st[0] == oexp and st[2] == osat and mst[0] == oexp
        else:
            want = {"spread": -12, "oshift": -13}[case]
            assert st[4] == want and mst[4] == want and prc == {"spread": -1, "oshift": -2}[case]


def test_tp_two_gpus_nccl(cuda):
    torch = cuda
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    s = socket.socket(); s.bind(("127.0.0.1", 0)); port = s.getsockname()[1]; s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(min(n, 2)), "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "tp_gpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_GPU_OK" in r.stdout
