"""Real weights into the decode engine: a float matrix quantised by the
library (mv4i_quantize_g128) and an .mv4i image converted by it
(mv4i_image_to_g128) are written over linears of a model with
dec_load_linear; the device copy must equal the host tensor byte for byte,
and a decode step with the loaded weights must match the float64 oracle
(which reads every weight back from the device) within the tolerance of
tests/test_dec_gpu.py."""
import ctypes as C

import numpy as np
import pytest

from conftest import device_read
from test_dec_gpu import CFG, Dec, check_step, oracle_from

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def O():
    from oracle import dec_oracle
    return dec_oracle


def test_load_linear_then_step(pkg, cuda, O):
    import oracle as OR
    torch = cuda
    L = pkg.lib()
    d = Dec(pkg)
    try:
        rng = np.random.default_rng(4)
        # layer 0 FFN down from a float matrix
        wq0, sc0 = d.linear(torch, 0, "down")
        M, K = wq0.shape[0], wq0.shape[1] * 2
        W = (rng.standard_normal((M, K)) * 0.05).astype(np.float32)
        sp = (K // 128 + 7) & ~7
        wq = np.zeros((M, K // 2), np.uint8)
        sc = np.zeros((M, sp), np.uint16)
        assert L.mv4i_quantize_g128(W.ctypes.data, M, K, wq.ctypes.data, sc.ctypes.data, sp) == 0
        assert d.L.dec_load_linear(d.h, 0, b"down", wq.ctypes.data, sc.ctypes.data, M, K, sp) == 0
        got_wq, got_sc = d.linear(torch, 0, "down")
        assert np.array_equal(got_wq, wq) and np.array_equal(got_sc, sc[:, :K // 128])
        # layer 1 FFN up from an .mv4i image (linear codebook, one scale per 128 columns)
        wq1, _ = d.linear(torch, 1, "up")
        M1, K1 = wq1.shape[0], wq1.shape[1] * 2
        lin = np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8)
        idx = rng.integers(0, 16, (M1, K1), dtype=np.uint8)
        scl = np.repeat(rng.integers(64, 1024, (M1, K1 // 128)).astype(np.uint16) * 16, 4, axis=1)
        pi = pkg.ParsedImage(OR.pack(M1, K1, 4, 128, 5, 3, lin, idx, scl))
        sp1 = (K1 // 128 + 7) & ~7
        wqa = np.zeros((M1, K1 // 2), np.uint8)
        sca = np.zeros((M1, sp1), np.uint16)
        assert L.mv4i_image_to_g128(C.byref(pi.f), wqa.ctypes.data, sca.ctypes.data, sp1) == 0
        assert d.L.dec_load_linear(d.h, 1, b"up", wqa.ctypes.data, sca.ctypes.data, M1, K1, sp1) == 0
        assert d.L.dec_load_linear(d.h, 1, b"up", wqa.ctypes.data, sca.ctypes.data, M1 + 1, K1, sp1) == -11
        assert d.L.dec_load_linear(d.h, 0, b"nope", wq.ctypes.data, sc.ctypes.data, M, K, sp) == -11
        # a step on the loaded weights against the oracle
        assert d.L.dec_prefill_random(d.h, 20, 5) == 0
        tok, pos = 9, 20
        assert d.L.dec_set(d.h, pos, tok) == 0
        M_ = oracle_from(d, torch, O)
        ptrs = d.pointers()
        d.seams_on(torch)
        d.step(torch)
        lg = device_read(torch, ptrs["logits"], (CFG["vocab"],), np.float32).astype(np.float64)
        check_step(O, M_, d.seams(torch), lg, tok, pos)
    finally:
        d.close()
