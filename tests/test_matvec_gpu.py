"""GPU parity of the INT4 streaming matvec (subsystem A) through the C ABI.

Golden mode is compared BIT-EXACT against values produced by the reference's
own ref/matvec_int4.c (committed fixtures) and against the oracle restatement
at full benchmark size.  g128 mode (the benchmark's fp16 format) is compared
against the double-precision oracle with the tolerance written in each test.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _fixture_keys(golden):
    keys = [k[:-5] for k in golden.files if k.endswith("_meta") and not k.startswith("tile")]
    return sorted(keys)


def _img(golden, k):
    meta = golden[k + "_meta"]
    if k.startswith("emit"):
        return golden["img%d" % meta[12]].tobytes()
    return golden[k + "_img"].tobytes()


def test_dropin_matches_reference_fixtures(cuda, pkg, golden):
    """mv4i_matvec (host buffers) vs the reference's outputs, every mode,
    full and partial row/column windows, IQ4_NL and linear codebooks,
    saturation case."""
    for k in _fixture_keys(golden):
        m = [int(v) for v in golden[k + "_meta"]]
        M, K, RI, DW, x_exp, nr, nc, mode, y_exp, sat, nsat, ns = m[:12]
        pi = pkg.ParsedImage(_img(golden, k))
        assert pi.rc == 0
        rc, r = pkg.matvec(pi, golden[k + "_x"], x_exp, nr, nc, mode)
        assert rc == 0, (k, rc)
        got = r["y_acc"] if mode == 2 else (r["y_mant"] if mode == 0 else r["y_data"])
        assert np.array_equal(got.astype(np.int64), golden[k + "_y"]), k
        assert (r["y_exp"], r["sat_event"], r["sat_count"], r["ns"]) == (y_exp, sat, nsat, ns), k
        if mode == 0 and (k + "_ydata") in golden.files:
            assert np.array_equal(r["y_data"], golden[k + "_ydata"]), k


def test_dropin_tile_vectors(cuda, pkg, golden):
    """sim/mv_tile_vec.txt cases (independent model tools/mv_tile_model.py)."""
    keys = sorted({k[:-5] for k in golden.files if k.startswith("tile") and k.endswith("_meta")})
    for k in keys:
        case, tile, osh, mode, sat = [int(v) for v in golden[k + "_meta"]]
        idx, scl, x, cb = golden[k + "_idx"], golden[k + "_scl"], golden[k + "_x"], golden[k + "_cb"]
        K = idx.shape[1]
        pi = pkg.ParsedImage(O.pack(2, K, 2, 128, 0, osh, cb, idx, scl))
        rc, r = pkg.matvec(pi, x, 0, 2, K, 2 if mode == 2 else 1)
        assert rc == 0
        got = r["y_acc"] if mode == 2 else r["y_data"].astype(np.int64)
        assert np.array_equal(got, golden[k + "_y"]), k
        if mode != 2:
            assert r["sat_event"] == sat, k


@pytest.mark.parametrize("shape", [(4096, 4096), (2048, 6144), (5120, 17408), (1, 32), (7, 33),
                                   (300, 2080), (151936 // 16, 2048)])
@pytest.mark.parametrize("cbname", ["linear", "iq4nl"])
def test_golden_full_size_vs_oracle(cuda, pkg, synth, shape, cbname):
    """Benchmark-size shapes (config 0 4096x4096; 2048->6144; 5120->17408;
    an LM-head slice) and ragged ones, bit-exact against the oracle in all
    three modes."""
    M, K = shape
    rng = np.random.default_rng(M + 7 * K)
    nb = (K + 31) // 32
    cb = synth.LINEAR_CB if cbname == "linear" else O.IQ4_NL
    idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
    scl = rng.integers(0, 32768, (M, nb), dtype=np.uint16)
    out_shift = min(40, max(0, 27 + int(np.ceil(np.log2(nb))) - 31)) if nb > 1 else 0
    img = O.pack(M, K, 4, 128, 3, out_shift, cb, idx, scl)
    x = rng.integers(-32768, 32768, K, dtype=np.int16)
    pi = pkg.ParsedImage(img)
    assert pi.rc == 0
    for mode in (0, 1, 2):
        rc, r = pkg.matvec(pi, x, 4, M, K, mode)
        orc, o = O.matvec(img, x, 4, M, K, mode)
        assert rc == 0 and orc == 0
        for f in ("y_exp", "sat_event", "sat_count", "ns"):
            assert r[f] == o[f], (shape, mode, f)
        if mode == 2:
            assert np.array_equal(r["y_acc"], o["y_acc"])
        else:
            assert np.array_equal(r["y_data"], o["y_data"])
            if mode == 0:
                assert np.array_equal(r["y_mant"], o["y_mant"])


def test_dropin_argument_errors_and_contract(cuda, pkg, golden):
    pi = pkg.ParsedImage(_img(golden, "lin1"))
    M, K = pi.M, pi.K
    x = np.zeros(K, np.int16)
    assert pkg.matvec(pi, x, 0, 0, K, 1)[0] == -1
    assert pkg.matvec(pi, x, 0, M, K + 1, 1)[0] == -2
    assert pkg.matvec(pi, x, 0, M + 1, K, 1)[0] == -3
    # a scale with its MSB set breaks the uint15 contract: the reference
    # asserts; this library returns -10
    img = bytearray(_img(golden, "lin1"))
    soff = int.from_bytes(img[0x30:0x34], "little")
    img[soff + 1] |= 0x80
    bad = pkg.ParsedImage(bytes(img))
    rc, _ = pkg.matvec(bad, np.ones(K, np.int16), 0, M, K, 1)
    assert rc == -10
    # the error is reported, not sticky: the good image still works
    rc, r = pkg.matvec(pi, golden["lin1_x"], int(golden["lin1_meta"][4]), M, K, 1)
    assert rc == 0 and np.array_equal(r["y_data"].astype(np.int64), golden["lin1_y"])


def test_dropin_cache_rewrite_and_forget(cuda, pkg, golden):
    """The device copy follows the image: an in-place rewrite inside the
    fingerprinted region is picked up on the next call, and mv4i_forget
    drops the copy outright."""
    pi = pkg.ParsedImage(_img(golden, "lin1"))
    m = [int(v) for v in golden["lin1_meta"]]
    x = golden["lin1_x"]
    rc, r0 = pkg.matvec(pi, x, m[4], m[5], m[6], 1)
    assert rc == 0
    soff = int.from_bytes(bytes(pi.buf[0x30:0x34]), "little")
    pi.buf[soff + 1] ^= 0x40                 # the scale region is hashed whole
    rc, r1 = pkg.matvec(pi, x, m[4], m[5], m[6], 1)
    o = O.matvec(pi.buf.tobytes(), x, m[4], m[5], m[6], 1)[1]
    assert rc == 0 and np.array_equal(r1["y_data"], o["y_data"])
    assert not np.array_equal(r1["y_data"], r0["y_data"])
    assert pkg.lib().mv4i_forget(C.byref(pi.f)) == 0
    rc, r2 = pkg.matvec(pi, x, m[4], m[5], m[6], 1)
    assert rc == 0 and np.array_equal(r2["y_data"], o["y_data"])


# ------------------------------------------------------------ device layer

def _dptr(t):
    return C.c_void_p(t.data_ptr())


def test_device_job_list_mixed(cuda, pkg, golden):
    """Several golden jobs of different shapes and modes in ONE launch; each
    equals the reference fixture; scratch is left zeroed for the next launch."""
    torch = cuda
    L = pkg.lib()
    keys = ["emit0", "emit13", "emit20", "lin0", "lin2", "sat1"]
    mats, jobs, outs = [], [], []
    scratch = torch.zeros(L.mv4i_scratch_bytes(), dtype=torch.uint8, device="cuda")
    status = torch.zeros((len(keys), 8), dtype=torch.int32, device="cuda")
    for i, k in enumerate(keys):
        m = [int(v) for v in golden[k + "_meta"]]
        pi = pkg.ParsedImage(_img(golden, k))
        dm = pkg.DMat()
        assert L.mv4i_dmat_upload(C.byref(pi.f), 0, C.byref(dm)) == 0
        mats.append((pi, dm))
        nr, nc, mode = m[5], m[6], m[7]
        x = torch.from_numpy(golden[k + "_x"].copy()).cuda()
        yd = torch.zeros(nr, dtype=torch.int32, device="cuda")
        ym = torch.zeros(nr, dtype=torch.int16, device="cuda")
        ya = torch.zeros(nr, dtype=torch.int64, device="cuda")
        outs.append((k, m, x, yd, ym, ya))
        j = pkg.Job()
        j.w = C.pointer(dm)
        j.x = x.data_ptr(); j.x_exp = m[4]; j.n_rows = nr; j.n_cols = nc; j.mode = mode; j.nvec = 1
        j.y_data = yd.data_ptr(); j.y_mant = ym.data_ptr(); j.y_acc = ya.data_ptr()
        j.status = status[i].data_ptr()
        jobs.append(j)
    arr = (pkg.Job * len(jobs))(*jobs)
    for rep in range(2):
        assert L.mv4i_launch(arr, len(jobs), _dptr(scratch), None) == 0
        torch.cuda.synchronize()
        assert int(scratch.count_nonzero()) == 0
        st = status.cpu().numpy()
        for i, (k, m, x, yd, ym, ya) in enumerate(outs):
            mode = m[7]
            got = (ya if mode == 2 else (ym if mode == 0 else yd)).cpu().numpy().astype(np.int64)
            assert np.array_equal(got, golden[k + "_y"]), (rep, k)
            assert st[i][0] == m[8] and st[i][1] == m[11] and st[i][2] == m[9] and st[i][4] == 0, k
    for pi, dm in mats:
        assert L.mv4i_dmat_free(C.byref(dm)) == 0


def _g128_operands(torch, pkg, seed, M, K, count=1):
    L = pkg.lib()
    wq = torch.empty((count, M, K // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((count, M, K // 128), dtype=torch.float16, device="cuda")
    x = torch.empty((count, K), dtype=torch.float16, device="cuda")
    assert L.mv4i_synth_g128(seed, count, M, K, _dptr(wq), _dptr(sc), _dptr(x), None) == 0
    torch.cuda.synchronize()
    return wq, sc, x


def _g128_run(torch, pkg, wq, sc, x, M, K):
    L = pkg.lib()
    count = wq.shape[0]
    y16 = torch.zeros((count, M), dtype=torch.float16, device="cuda")
    y32 = torch.zeros((count, M), dtype=torch.float32, device="cuda")
    mats, jobs = [], []
    for i in range(count):
        dm = pkg.DMat()
        assert L.mv4i_dmat_wrap_g128(_dptr(wq[i]), K // 2, _dptr(sc[i]), K // 128, M, K, 0,
                                     C.byref(dm)) == 0
        mats.append(dm)
        j = pkg.Job()
        j.w = C.pointer(dm); j.x = x[i].data_ptr(); j.n_rows = M; j.n_cols = K; j.nvec = 1
        j.y_f16 = y16[i].data_ptr(); j.y_f32 = y32[i].data_ptr()
        jobs.append(j)
    arr = (pkg.Job * count)(*jobs)
    assert L.mv4i_launch(arr, count, None, None) == 0
    torch.cuda.synchronize()
    return y16.cpu().numpy(), y32.cpu().numpy()


def test_synth_matches_host_generator(cuda, pkg, synth):
    """The device generator and llm.vhdl_b200/synth.py agree (W and scales
    bit-exact; x within one fp16 ulp where libm rounding differs)."""
    torch = cuda
    M, K = 256, 1024
    wq, sc, x = _g128_operands(torch, pkg, 0, M, K)
    assert np.array_equal(wq[0].cpu().numpy(), synth.g128_weights(0, M, K))
    assert np.array_equal(sc[0].cpu().numpy(), synth.g128_scales(0, M, K))
    xd = x[0].cpu().numpy().astype(np.float64)
    xh = synth.g128_x(0, K).astype(np.float64)
    assert np.mean(xd == xh) > 0.99 and np.max(np.abs(xd - xh)) <= 2 ** -10 * max(1, np.max(np.abs(xh)))


@pytest.mark.parametrize("shape", [(4096, 4096), (2048, 2048), (6144, 2048), (5120, 17408),
                                   (128, 128), (1, 256), (37, 384)])
def test_g128_vs_double_oracle(cuda, pkg, shape):
    """Config-0 format.  Tolerances: fp32 output max|y-ref| <= 1e-4*max|ref|
    (normwise; x is staged as int16 on a per-128-column exponent, ~2^-15 of the
    group maximum); fp16 output max|y-ref| <= 1e-3*max|ref| and elementwise
    within 2^-11*|ref| + 1e-4*max|ref|."""
    torch = cuda
    M, K = shape
    wq, sc, x = _g128_operands(torch, pkg, 0, M, K)
    y16, y32 = _g128_run(torch, pkg, wq, sc, x, M, K)
    ref = O.matvec_g128_f64(wq[0].cpu().numpy(), sc[0].cpu().numpy(), x[0].cpu().numpy(), K)
    amax = np.max(np.abs(ref))
    e32 = np.max(np.abs(y32[0] - ref)) / amax
    e16 = np.abs(y16[0].astype(np.float64) - ref)
    assert e32 <= 1e-4, e32
    assert np.max(e16) / amax <= 1e-3
    assert np.all(e16 <= 2.0 ** -11 * np.abs(ref) + 1e-4 * amax)


@pytest.mark.parametrize("shape", [(2048, 2048), (512, 6144), (37, 384)])
def test_g128_staging_contract(cuda, pkg, shape):
    """The g128 kernel's only approximation besides fp32 summation is its
    activation staging (int16 on a per-128-column exponent, oracle/dec_oracle.py
    stage_g128): against the double product of the STAGED x the fp32 output
    agrees to 2e-6 of max|y|, with x spanning many octaves inside each group
    (where staging and fp16 differ most)."""
    from oracle import dec_oracle as D
    torch = cuda
    M, K = shape
    wq, sc, _ = _g128_operands(torch, pkg, 1, M, K)
    g = torch.Generator().manual_seed(M)
    xs = (torch.randn(K, generator=g) * torch.exp2(torch.randint(-14, 3, (K,), generator=g).float())).half()
    xs[:5] = 0
    x = xs.cuda().reshape(1, K)
    _, y32 = _g128_run(torch, pkg, wq, sc, x, M, K)
    w = O.matvec_g128_f64
    xh = xs.numpy()
    ref_staged = D.dequant_g128(wq[0].cpu().numpy(), sc[0].cpu().numpy().view(np.uint16)) @ \
        D.stage_g128(xh.astype(np.float64))
    ref_exact = w(wq[0].cpu().numpy(), sc[0].cpu().numpy(), xh, K)
    amax = np.max(np.abs(ref_exact))
    assert np.max(np.abs(y32[0] - ref_staged)) <= 2e-6 * amax
    assert np.max(np.abs(y32[0] - ref_exact)) <= 1e-4 * amax


def test_g128_stack_equals_single(cuda, pkg):
    """A stack of matrices in one launch gives the per-matrix results."""
    torch = cuda
    M, K, G = 1024, 2048, 5
    wq, sc, x = _g128_operands(torch, pkg, 3, M, K, G)
    y16, y32 = _g128_run(torch, pkg, wq, sc, x, M, K)
    for i in range(G):
        a16, a32 = _g128_run(torch, pkg, wq[i:i + 1], sc[i:i + 1], x[i:i + 1], M, K)
        assert np.array_equal(a32[0], y32[i]) and np.array_equal(a16[0], y16[i])


def test_g128_cross_check_golden(cuda, pkg, synth):
    """Same weights through golden mode (linear codebook, scales*2^20, w_exp 5,
    x BFP-packed by the reg_put rule) and g128 mode agree to the BFP
    quantisation of x: |y_g128 - y_golden| <= 2e-4 * max|y|."""
    torch = cuda
    M, K = 1024, 4096
    wq, sc, x = _g128_operands(torch, pkg, 0, M, K)
    _, y32 = _g128_run(torch, pkg, wq, sc, x, M, K)
    idx, scl, w_exp = synth.g128_to_golden(wq[0].cpu().numpy(), sc[0].cpu().numpy(), K)
    xm, xe = O.bfp_pack_f64(x[0].cpu().numpy().astype(np.float64))
    img = O.pack(M, K, 4, 128, w_exp, 0, synth.LINEAR_CB, idx, scl)
    pi = pkg.ParsedImage(img)
    rc, r = pkg.matvec(pi, xm, xe, M, K, 1)
    assert rc == 0
    yg = r["y_data"].astype(np.float64) * 2.0 ** (-r["y_exp"])
    assert np.max(np.abs(yg - y32[0])) <= 2e-4 * np.max(np.abs(y32[0]))


@pytest.mark.parametrize("M,K,n_rows,n_cols,accum", [(37, 1024, 37, 1024, 0), (1000, 2176, 1000, 2176, 0),
                                                    (333, 2048, 300, 1000, 0), (4096, 8192, 4096, 8192, 1),
                                                    (17, 128, 17, 100, 1)])
def test_g128_layouts(cuda, pkg, M, K, n_rows, n_cols, accum):
    """Padded scale rows (a pitch beyond K/128), ragged row counts, a group
    count that is not a power of two, a column window that ends inside a
    group, the accumulate flag, and several jobs sharing CTAs.  Same
    tolerances as test_g128_vs_double_oracle."""
    torch = cuda
    L = pkg.lib()
    ng = (K + 127) // 128
    sp = (ng + 7) & ~7
    G = 3
    wq, sc0, x = _g128_operands(torch, pkg, 5, M, K, G)
    sc = torch.zeros((G, M, sp), dtype=torch.float16, device="cuda")
    sc[:, :, :ng] = sc0
    y16 = torch.zeros((G, M), dtype=torch.float16, device="cuda")
    base = torch.randn((G, M), device="cuda") if accum else torch.zeros((G, M), device="cuda")
    y32 = base.clone()
    mats, jobs = [], []
    for i in range(G):
        dm = pkg.DMat()
        assert L.mv4i_dmat_wrap_g128(_dptr(wq[i]), K // 2, _dptr(sc[i]), sp, M, K, 0, C.byref(dm)) == 0
        mats.append(dm)
        j = pkg.Job()
        j.w = C.pointer(dm); j.x = x[i].data_ptr(); j.n_rows = n_rows; j.n_cols = n_cols; j.nvec = 1
        j.y_f16 = y16[i].data_ptr(); j.y_f32 = y32[i].data_ptr(); j.accum = accum
        jobs.append(j)
    arr = (pkg.Job * G)(*jobs)
    assert L.mv4i_launch(arr, G, None, None) == 0
    torch.cuda.synchronize()
    for i in range(G):
        xc = x[i].cpu().numpy().copy()
        xc[n_cols:] = 0
        ref = O.matvec_g128_f64(wq[i].cpu().numpy(), sc0[i].cpu().numpy(), xc, K)[:n_rows]
        got32 = (y32[i] - base[i]).cpu().numpy()[:n_rows].astype(np.float64)
        amax = np.max(np.abs(ref))
        assert np.max(np.abs(got32 - ref)) <= 1e-4 * amax + (1e-6 * np.max(np.abs(base[i].cpu().numpy())) if accum else 0)
        assert np.all(y32[i].cpu().numpy()[n_rows:] == base[i].cpu().numpy()[n_rows:])
        if not accum:
            e16 = np.abs(y16[i].cpu().numpy()[:n_rows].astype(np.float64) - ref)
            assert np.all(e16 <= 2.0 ** -11 * np.abs(ref) + 1e-4 * amax)


@pytest.mark.parametrize("count", [1, 3, 5, 64])
def test_g128_host_buffer_call_equals_device_launch(cuda, pkg, count):
    """mv4i_g128_matvec_host (pinned host x in, host y out, the end-to-end
    call of the benchmark) gives the device launch's fp16 results bit for bit,
    twice in a row, for one job and for job lists of several sizes."""
    torch = cuda
    L = pkg.lib()
    M, K = 512, 2048
    wq, sc, x = _g128_operands(torch, pkg, 9, M, K, count)
    y16, _ = _g128_run(torch, pkg, wq, sc, x, M, K)
    mats = (pkg.DMat * count)()
    for i in range(count):
        assert L.mv4i_dmat_wrap_g128(_dptr(wq[i]), K // 2, _dptr(sc[i]), K // 128, M, K, 0, C.byref(mats[i])) == 0
    hx = torch.empty((count, K), dtype=torch.float16).pin_memory()
    hx.copy_(x.cpu())
    hy = torch.zeros((count, M), dtype=torch.float16).pin_memory()
    s = torch.cuda.Stream()
    for _ in range(2):
        hy.zero_()
        assert L.mv4i_g128_matvec_host(mats, count, C.c_void_p(hx.data_ptr()), C.c_void_p(hy.data_ptr()),
                                       C.c_void_p(s.cuda_stream)) == 0
        assert np.array_equal(hy.numpy().view(np.uint16), y16.view(np.uint16))
