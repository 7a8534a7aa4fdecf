"""Tensor-parallel reduction on GPUs.

* one GPU: N shards emulated in one process (as the reference's 15.4b tests
  do, ref/matvec_int4.c:1124-1197) -- mv4i_tp_reduce bit-exact against the
  oracle's E 2.1 reduction for N = 2, 4, 8, including the refusals;
* two or more GPUs: tests/tp_gpu_worker.py under torchrun, partials over NCCL.
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


@pytest.mark.parametrize("N", [2, 4, 8])
def test_tp_reduce_emulated_shards(cuda, pkg, N):
    torch = cuda
    sys.path.insert(0, ROOT)
    import llmvhdl_b200.tp as TP
    L = pkg.lib()
    rng = np.random.default_rng(N)
    M = 5120
    for case in ("ok", "spread", "oshift"):
        parts = [rng.integers(-(1 << 44), 1 << 44, M) for _ in range(N)]
        ye = [int(v) for v in rng.integers(20, 30, N)]
        osh = [9] * N
        if case == "spread":
            ye[-1] = ye[0] + 18 if ye[0] + 18 > max(ye[:-1]) else max(ye) + 18
        if case == "oshift":
            osh[-1] = 10
        prc, oout, oexp, oy32, osat = O.tp_reduce(parts, ye, osh)
        dp = torch.from_numpy(np.stack(parts)).cuda()
        out, y32, st = TP.reduce_partials_device(L, dp, torch.tensor(ye, dtype=torch.int32).cuda(),
                                                 torch.tensor(osh, dtype=torch.int32).cuda())
        torch.cuda.synchronize()
        err = int(st[4].item())
        if case == "ok":
            assert prc == 0 and err == 0
            assert np.array_equal(out.cpu().numpy(), oout) and np.array_equal(y32.cpu().numpy(), oy32)
            assert int(st[0].item()) == oexp and int(st[2].item()) == osat
        else:
            assert err == {"spread": -12, "oshift": -13}[case] and prc == {"spread": -1, "oshift": -2}[case]


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
