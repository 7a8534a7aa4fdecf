"""The persistent decode step (one launch per step, grid barriers between
stages; include/dec_b200.h dec_set_persistent) against the launch-per-stage
step on the same model (the default mode, which tests/test_dec_gpu.py checks
against the float64 oracle).

Both modes run the same stage code on the same inputs; only the matvec work
split differs (it is sized for the grid), so fp32 sums may round differently.
Tolerance: logits within 1e-4 of the largest magnitude at every step, and the
same token wherever the top-2 margin exceeds 1e-3 of it.

The barrier waits are bounded: with the wait limit cut to 1 ns a step gives up
at its first barrier that is not complete on arrival, every CTA leaves, and
dec_status reports flag 4 (nothing is made to hang or fault; the wait runs out
on the host-chosen limit).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import device_read
from test_dec_gpu import CFG, Dec

pytestmark = pytest.mark.gpu

CFG_WIDE = dict(hidden=2048, n_layers=4, attn_every=4, vocab=5000, ffn=6144, gdn_kh=16, gdn_vh=16, gdn_hd=128,
                att_qh=16, att_kvh=2, att_hd=128, n_rot=64, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=1024)


def logits(d, torch, nb=1):
    p = d.pointers()
    return device_read(torch, p["logits"], (nb, p["vn"]), np.float32).astype(np.float64)


def top2_margin(lg):
    s = np.sort(lg)
    return (s[-1] - s[-2]) / max(np.max(np.abs(lg)), 1e-30)


@pytest.mark.parametrize("cfg,nb,prefill", [(CFG, 1, 60), (CFG, 4, 40), (CFG_WIDE, 1, 600), (CFG_WIDE, 8, 100)])
def test_persistent_step_equals_launch_mode(pkg, cuda, cfg, nb, prefill):
    torch = cuda
    c = dict(cfg, batch=nb)
    a, b = Dec(pkg, cfg=c, seed=7), Dec(pkg, cfg=c, seed=7)
    try:
        assert a.L.dec_set_persistent(a.h, 1) == 0 and a.L.dec_persistent(a.h) == 1
        assert b.L.dec_set_persistent(b.h, 0) == 0 and b.L.dec_persistent(b.h) == 0
        for d in (a, b):
            assert d.L.dec_prefill_random(d.h, prefill, 3) == 0
            assert d.L.dec_set(d.h, prefill, 17) == 0
        for step in range(5):
            a.step(torch)
            b.step(torch)
            torch.cuda.synchronize()
            la, lb = logits(a, torch, nb), logits(b, torch, nb)
            for s in range(nb):
                err = np.max(np.abs(la[s] - lb[s])) / np.max(np.abs(lb[s]))
                assert err <= 1e-4, (step, s, err)
            pa, pb = a.pointers(), b.pointers()
            ha = device_read(torch, pa["hist"], (nb, c["max_ctx"]), np.int32)[:, prefill + step]
            hb = device_read(torch, pb["hist"], (nb, c["max_ctx"]), np.int32)[:, prefill + step]
            for s in range(nb):
                if top2_margin(lb[s]) > 1e-3:
                    assert ha[s] == hb[s], (step, s)
                    assert ha[s] == int(np.argmax(lb[s]))
        assert device_read(torch, a.pointers()["pos"], (1,), np.int32)[0] == prefill + 5
        fl = C.c_int32(-1)
        assert a.L.dec_status(a.h, C.byref(fl)) == 0 and fl.value == 0
    finally:
        a.close()
        b.close()


def test_stage_clock(pkg, cuda):
    torch = cuda
    d = Dec(pkg)
    try:
        assert d.L.dec_set_persistent(d.h, 1) == 0
        n = d.L.dec_clock_slots(d.h)
        assert n > 2 * CFG["n_layers"]
        clk = torch.zeros(n, dtype=torch.int64, device="cuda")
        assert d.L.dec_set_clock(d.h, C.c_void_p(clk.data_ptr())) == 0
        assert d.L.dec_prefill_random(d.h, 30, 1) == 0
        d.step(torch)
        torch.cuda.synchronize()
        assert d.L.dec_set_clock(d.h, None) == 0
        t = clk.cpu().numpy()
        assert t[0] > 0 and np.all(np.diff(t) >= 0)
        idx = [d.L.dec_layer_clock(d.h, il) for il in range(-1, CFG["n_layers"] + 1)]
        assert idx[0] == 1 and idx[-1] == n - 1 and all(x < y for x, y in zip(idx, idx[1:]))
        assert d.L.dec_layer_clock(d.h, CFG["n_layers"] + 1) < 0
    finally:
        d.close()


def test_barrier_wait_limit_aborts_the_step(pkg, cuda):
    torch = cuda
    d = Dec(pkg)
    try:
        assert d.L.dec_set_persistent(d.h, 1) == 0
        assert d.L.dec_prefill_random(d.h, 30, 1) == 0
        assert d.L.dec_set(d.h, 30, 5) == 0
        assert d.L.dec_set_wait_limit(d.h, 1) == 0
        d.step(torch)
        torch.cuda.synchronize()
        fl = C.c_int32(0)
        assert d.L.dec_status(d.h, C.byref(fl)) == 0
        assert fl.value & 4, fl.value
        assert d.L.dec_status(d.h, C.byref(fl)) == 0 and fl.value == 0          # cleared
        # with the default bound the next steps run through
        assert d.L.dec_set_wait_limit(d.h, 0) == 0
        assert d.L.dec_set(d.h, 30, 5) == 0
        for _ in range(2):
            d.step(torch)
        torch.cuda.synchronize()
        assert d.L.dec_status(d.h, C.byref(fl)) == 0 and fl.value == 0
        assert device_read(torch, d.pointers()["pos"], (1,), np.int32)[0] == 32
    finally:
        d.close()
