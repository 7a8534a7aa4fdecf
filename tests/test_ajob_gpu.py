"""GPU parity of the producers and consumers around the matvec: the
activation BFP pack (reg_put, ref/run9b.c:343-359), the row-window A job
(ref/run9b.c:455-490), and the LM head with argmax_first (ref/run9b.c:399-405,
522-540).  All bit-exact."""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_bfp_pack_matches_reg_put(cuda, pkg, dtype):
    torch = cuda
    rng = np.random.default_rng(11)
    vecs = [rng.normal(size=4096), rng.normal(size=4096) * 1e-4, rng.normal(size=4096) * 3e3,
            np.zeros(4096), rng.uniform(-1, 1, 4096) * 2.0 ** -20, np.full(4096, 0.5),
            np.concatenate([[1.0], np.zeros(4095)]), rng.normal(size=4096) * 7.7]
    if dtype == "f16":
        vecs[4] = rng.uniform(-1, 1, 4096) * 2.0 ** -14      # fp16 subnormals
    npdt = np.float16 if dtype == "f16" else np.float32
    arr = np.stack(vecs).astype(npdt)
    n, cnt = 3000, arr.shape[0]                               # stride 4096, n 3000
    d = torch.from_numpy(arr).cuda()
    mant = torch.zeros((cnt, n), dtype=torch.int16, device="cuda")
    exps = torch.zeros(cnt, dtype=torch.int32, device="cuda")
    assert pkg.lib().mv4i_bfp_pack(_p(d), 0 if dtype == "f16" else 1, n, cnt, 4096, _p(mant), _p(exps), None) == 0
    torch.cuda.synchronize()
    for i in range(cnt):
        m, e = O.bfp_pack_f64(arr[i, :n].astype(np.float64))
        assert np.array_equal(mant[i].cpu().numpy(), m), i
        assert int(exps[i].item()) == e, i


@pytest.mark.parametrize("window", [(0, 300), (0, 100), (64, 200), (299, 1), (123, 77)])
def test_row_window_a_job(cuda, pkg, golden, window):
    torch = cuda
    L = pkg.lib()
    row0, n = window
    M, K = 300, 2048
    rng = np.random.default_rng(row0 + n)
    idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
    scl = rng.integers(0, 32768, (M, K // 32), dtype=np.uint16)
    img = O.pack(M, K, 4, 128, 2, 3, O.IQ4_NL, idx, scl)
    x = rng.integers(-20000, 20000, K).astype(np.int16)
    pi = pkg.ParsedImage(img)
    dm, view = pkg.DMat(), pkg.DMat()
    assert L.mv4i_dmat_upload(C.byref(pi.f), 0, C.byref(dm)) == 0
    assert L.mv4i_dmat_rows(C.byref(dm), row0, n, C.byref(view)) == 0
    dx = torch.from_numpy(x).cuda()
    yd = torch.zeros(n, dtype=torch.int32, device="cuda")
    ym = torch.zeros(n, dtype=torch.int16, device="cuda")
    st = torch.zeros(8, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(L.mv4i_scratch_bytes(), dtype=torch.uint8, device="cuda")
    j = pkg.Job()
    j.w = C.pointer(view); j.x = dx.data_ptr(); j.x_exp = 7; j.n_rows = n; j.n_cols = K; j.mode = 0
    j.nvec = 1; j.y_data = yd.data_ptr(); j.y_mant = ym.data_ptr(); j.status = st.data_ptr()
    assert L.mv4i_launch(C.byref(j), 1, _p(scratch), None) == 0
    torch.cuda.synchronize()
    want, want_e = O.a_job(img, x, 7, K, row0, n)
    assert np.array_equal(ym.cpu().numpy(), want)
    assert int(st[0].item()) == want_e
    L.mv4i_dmat_free(C.byref(dm))


def test_argmax_first_ties(cuda, pkg):
    torch = cuda
    L = pkg.lib()
    work = torch.zeros(1, dtype=torch.int64, device="cuda")
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(2)
    for dt, npdt, code in (("i32", np.int32, 0), ("f32", np.float32, 1), ("f16", np.float16, 2)):
        for n in (1, 7, 1000, 151936):
            v = (rng.integers(-50, 50, n) if dt == "i32" else rng.normal(size=n)).astype(npdt)
            if n > 10:
                v[n // 3] = v[n - 1] = v.max() + (1 if dt == "i32" else 0.5)   # a tie, first wins
            d = torch.from_numpy(v).cuda()
            assert L.mv4i_argmax(_p(d), code, n, _p(work), _p(idx), None) == 0
            assert int(idx.item()) == O.argmax_first(v), (dt, n)
    v = np.array([-3.0, -1.0, -1.0, -2.0], np.float32)                 # negatives
    d = torch.from_numpy(v).cuda()
    assert L.mv4i_argmax(_p(d), 1, 4, _p(work), _p(idx), None) == 0 and int(idx.item()) == 1


def test_lm_head_raw_argmax(cuda, pkg, synth):
    """Config-3 LM head shape: 151936 x 2048, golden RAW logits (one grid)
    bit-exact with the oracle, then argmax_first on the device."""
    torch = cuda
    L = pkg.lib()
    M, K = 151936, 2048
    rng = np.random.default_rng(9)
    wq = synth.g128_weights(2, M, K)
    sc = synth.g128_scales(2, M, K)
    idx, scl, w_exp = synth.g128_to_golden(wq, sc, K)
    img = O.pack(M, K, 4, 128, w_exp, 3, synth.LINEAR_CB, idx, scl)
    x = rng.integers(-16000, 16000, K).astype(np.int16)
    pi = pkg.ParsedImage(img)
    rc, r = pkg.matvec(pi, x, 10, M, K, 1)
    orc, o = O.matvec(img, x, 10, M, K, 1)
    assert rc == 0 and orc == 0
    assert np.array_equal(r["y_data"], o["y_data"]) and r["y_exp"] == o["y_exp"]
    d = torch.from_numpy(r["y_data"]).cuda()
    work = torch.zeros(1, dtype=torch.int64, device="cuda")
    ix = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.mv4i_argmax(_p(d), 0, M, _p(work), _p(ix), None) == 0
    assert int(ix.item()) == O.argmax_first(o["y_data"])
