"""The decode-step matvec (llm.vhdl_b200/csrc/dec_matvec.cu) against the oracle.

Each prologue (fp16 input, RMSNorm of the residual, DeltaNet output norm x
silu(z) per head) and each epilogue (fp32 / fp16 store, residual accumulate,
paired SwiGLU, conv + SiLU with its rolling state, decay / beta gates, LM-head
argmax key) is compared with oracle/dec_oracle.py on identical inputs:

* the staged product is exact up to fp32 summation: against the double
  product of the g128-staged fp16 input (oracle stage_g128) the output agrees to
  2e-6 of its largest magnitude;
* the fp16 input a prologue builds (read back through the seam pointer) equals
  the oracle's fp16 rounding of the same expression except for values within
  fp32 rounding of an fp16 boundary (at most 1 ulp, at most 1% of them);
* epilogue nonlinearities within 1e-3 of the largest magnitude, argmax exact.

Launches are also chained as programmatic dependents (PDL) with each consuming
the previous one's output, which must give the same answer as plain launches.
Batched launches (nvec input vectors sharing each weight load, the decode
step's sequences) must give every vector the single-vector result.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P_ = C.c_void_p
EPI = dict(F32=0, ACC=1, F16=2, SWIGLU=3, CONV=4, GATES=5, ARGMAX=6)
OP = dict(F16=0, RMSNORM=1, GATED=2)


class Job(C.Structure):
    _fields_ = [("wq", P_), ("wq2", P_), ("sc", P_), ("sc2", P_), ("out_f32", P_), ("out2_f32", P_),
                ("out_f16", P_), ("p0", P_), ("p1", P_), ("st", P_), ("st_stride", C.c_int32),
                ("n1", C.c_int32), ("rows", C.c_int32), ("epi", C.c_int32), ("tile0", C.c_int32),
                ("ntiles", C.c_int32), ("s_pitch", C.c_int32), ("ostride", C.c_int32)]


class Params(C.Structure):
    _fields_ = [("jobs", Job * 4), ("njobs", C.c_int32), ("total_tiles", C.c_int32), ("K", C.c_int32),
                ("op", C.c_int32), ("x", P_), ("x2", P_), ("nw", P_), ("eps", C.c_float), ("seam", P_),
                ("key", P_), ("idx0", C.c_int32), ("pf_bytes", C.c_int32), ("ksplit", C.c_int32),
                ("nvec", C.c_int32), ("xs", C.c_int32), ("pad_", C.c_int32),
                ("xst", C.c_void_p)]


@pytest.fixture(scope="module")
def L(pkg):
    D = pkg.declib()
    D.dec_k_matvec.argtypes = [C.POINTER(Params), P_, C.c_int]
    D.dec_k_matvec.restype = C.c_int
    return D


@pytest.fixture(scope="module")
def O():
    from oracle import dec_oracle
    return dec_oracle


def dp(t):
    return t.data_ptr() if t is not None else None


def spitch(K):
    return (K // 128 + 7) & ~7


class Scales:
    """fp16 scales [rows][K/128] stored at a 16-byte row pitch (the kernel's
    layout); .t is the padded device tensor, .v the [rows][K/128] view."""

    def __init__(self, v):
        rows, ng = v.shape
        self.t = torch_mod().zeros(rows, spitch(128 * ng), dtype=v.dtype, device=v.device)
        self.t[:, :ng] = v
        self.v = self.t[:, :ng]

    def data_ptr(self):
        return self.t.data_ptr()

    def __getitem__(self, i):
        return self.v[i]

    def __setitem__(self, i, val):
        self.v[i] = val


def torch_mod():
    import torch
    return torch


def weights(torch, rows, K, seed):
    g = torch.Generator().manual_seed(seed)
    wq = torch.randint(0, 256, (rows, K // 2), generator=g, dtype=torch.uint8)
    sc = (0.002 + 0.018 * torch.rand(rows, K // 128, generator=g)).half()
    return wq.cuda(), Scales(sc.cuda())


def deq(O, wq, sc):
    return O.dequant_g128(wq.cpu().numpy(), sc.v.cpu().numpy().view(np.uint16))


def run(L, torch, p, pdl=0):
    rc = L.dec_k_matvec(C.byref(p), None, pdl)
    assert rc == 0, rc
    torch.cuda.synchronize()


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def seam_ok(got16, want):
    """fp16 seam vs the oracle's fp16 of the same fp64 expression."""
    w16 = want.astype(np.float16)
    g = got16.astype(np.float16)
    diff = g != w16
    if np.any(diff):
        ulp = np.abs(np.spacing(w16[diff]).astype(np.float64))
        assert np.all(np.abs(g[diff].astype(np.float64) - w16[diff].astype(np.float64)) <= ulp * 1.01)
    assert np.mean(diff) <= 0.01, np.mean(diff)


# tall and short K, few and many rows per warp, the column split over warps
@pytest.mark.parametrize("K,rows", [(128, 1), (2048, 7), (2048, 2048), (5120, 33), (17408, 64), (6144, 300),
                                    (4096, 5120), (17408, 5120), (2048, 20000)])
def test_f16_input_staged_product(cuda, L, O, K, rows):
    torch = cuda
    wq, sc = weights(torch, rows, K, K + rows)
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(K, generator=g) * torch.exp2(torch.randint(-10, 3, (K,), generator=g).float())).half().cuda()
    y32 = torch.zeros(rows, device="cuda")
    y16 = torch.zeros(rows, dtype=torch.int16, device="cuda")
    acc = torch.randn(rows, generator=g).cuda()
    acc0 = acc.clone()
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=3, pf_bytes=65536)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y32))
    p.jobs[1] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F16"], out_f16=dp(y16))
    p.jobs[2] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["ACC"], out_f32=dp(acc))
    run(L, torch, p)
    W = deq(O, wq, sc)
    xs = O.stage_g128(x.cpu().numpy().astype(np.float64))
    ref = W @ xs
    got = y32.cpu().numpy().astype(np.float64)
    assert rel(got, ref) <= 2e-6
    assert rel(W @ x.cpu().numpy().astype(np.float64), got) <= 1e-4      # the staging's own cost
    assert np.array_equal(y16.cpu().numpy().view(np.float16), got.astype(np.float32).astype(np.float16))
    assert np.allclose((acc - acc0).cpu().numpy(), got, rtol=0, atol=1e-6 * np.max(np.abs(got)))


@pytest.mark.parametrize("K", [256, 2048, 5120])
def test_rmsnorm_prologue_and_seam(cuda, L, O, K):
    torch = cuda
    rows = 300
    wq, sc = weights(torch, rows, K, 7 + K)
    g = torch.Generator().manual_seed(K + 1)
    res = (torch.randn(K, generator=g) * 3).cuda()
    w = (1 + 0.1 * torch.randn(K, generator=g)).cuda()
    seam = torch.zeros(K, dtype=torch.int16, device="cuda")
    y = torch.zeros(rows, device="cuda")
    p = Params(K=K, op=OP["RMSNORM"], x=dp(res), nw=dp(w), eps=1e-6, seam=dp(seam), njobs=1)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y))
    run(L, torch, p)
    h16 = seam.cpu().numpy().view(np.float16)
    seam_ok(h16, O.rmsnorm(res.double().cpu().numpy(), w.double().cpu().numpy(), 1e-6))
    ref = deq(O, wq, sc) @ O.stage_g128(h16.astype(np.float64))
    assert rel(y.cpu().numpy().astype(np.float64), ref) <= 2e-6


def test_gated_prologue(cuda, L, O):
    torch = cuda
    H, rows = 6, 256
    K = H * 128
    wq, sc = weights(torch, rows, K, 11)
    g = torch.Generator().manual_seed(12)
    o = torch.randn(K, generator=g) * torch.exp2(torch.randint(-6, 2, (H, 1), generator=g).float()).repeat(1, 128).reshape(-1)
    z = 2 * torch.randn(K, generator=g)
    w = 1 + 0.1 * torch.randn(128, generator=g)
    seam = torch.zeros(K, dtype=torch.int16, device="cuda")
    y = torch.zeros(rows, device="cuda")
    od, zd, wd = o.cuda(), z.cuda(), w.cuda()
    p = Params(K=K, op=OP["GATED"], x=dp(od), x2=dp(zd), nw=dp(wd), eps=1e-6, seam=dp(seam), njobs=1)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y))
    run(L, torch, p)
    on, zn, wn = o.double().numpy().reshape(H, 128), z.double().numpy().reshape(H, 128), w.double().numpy()
    want = np.stack([O.rmsnorm(on[i], wn, 1e-6) * O.silu(zn[i]) for i in range(H)]).reshape(-1)
    y16 = seam.cpu().numpy().view(np.float16)
    seam_ok(y16, want)
    ref = deq(O, wq, sc) @ O.stage_g128(y16.astype(np.float64))
    assert rel(y.cpu().numpy().astype(np.float64), ref) <= 2e-6


@pytest.mark.parametrize("K,F", [(2048, 640), (5120, 5120)])
def test_paired_swiglu_epilogue(cuda, L, O, K, F):
    torch = cuda
    wg, sg = weights(torch, F, K, 21)
    wu, su = weights(torch, F, K, 22)
    x = torch.randn(K, generator=torch.Generator().manual_seed(23)).half().cuda()
    h = torch.zeros(F, dtype=torch.int16, device="cuda")
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=1)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wg), wq2=dp(wu), sc=dp(sg), sc2=dp(su), rows=F, epi=EPI["SWIGLU"], out_f16=dp(h))
    run(L, torch, p)
    xs = O.stage_g128(x.cpu().numpy().astype(np.float64))
    want = O.silu(deq(O, wg, sg) @ xs) * (deq(O, wu, su) @ xs)
    got = h.cpu().numpy().view(np.float16).astype(np.float64)
    assert np.all(np.abs(got - want) <= 2.0 ** -10 * np.abs(want) + 1e-6 * np.max(np.abs(want)))


def test_conv_and_gate_epilogues(cuda, L, O):
    """q|k|v channels: 4-tap conv over the rolling state + SiLU to fp16 and
    the state shifted; a|b rows: decay exp(ssm_a * softplus(a + dt_bias))
    (softplus passes x through above 20) and sigmoid beta."""
    torch = cuda
    K, cd, vh = 1024, 768, 6
    g = torch.Generator().manual_seed(31)
    wc, scc = weights(torch, cd, K, 32)
    wa, sa = weights(torch, 2 * vh, K, 33)
    x = torch.randn(K, generator=g).half().cuda()
    cw = (0.5 * torch.randn(cd * 4, generator=g)).cuda()
    st = (0.5 * torch.randn(3 * (cd + 16), generator=g)).cuda()        # stride cd + 16
    st0 = st.clone()
    ssm_a = (-1 + 0.2 * torch.randn(vh, generator=g)).cuda()
    dt = (0.5 * torch.randn(vh, generator=g)).cuda()
    dt[0] = 40.0                                                        # the passthrough branch
    q16 = torch.zeros(cd, dtype=torch.int16, device="cuda")
    raw = torch.zeros(cd, device="cuda")
    eg, beta = torch.zeros(vh, device="cuda"), torch.zeros(vh, device="cuda")
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=2)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wc), sc=dp(scc), rows=cd, epi=EPI["CONV"], out_f16=dp(q16), out_f32=dp(raw),
                    p0=dp(cw), st=dp(st), st_stride=cd + 16)
    p.jobs[1] = Job(s_pitch=spitch(K), wq=dp(wa), sc=dp(sa), rows=2 * vh, epi=EPI["GATES"], out_f32=dp(eg), out2_f32=dp(beta),
                    p0=dp(ssm_a), p1=dp(dt), n1=vh)
    run(L, torch, p)
    xs = O.stage_g128(x.cpu().numpy().astype(np.float64))
    proj = deq(O, wc, scc) @ xs
    assert rel(raw.cpu().numpy().astype(np.float64), proj) <= 2e-6
    S = st0.cpu().numpy().astype(np.float64).reshape(3, cd + 16)[:, :cd]
    w4 = cw.cpu().numpy().astype(np.float64).reshape(cd, 4)
    r = raw.cpu().numpy().astype(np.float64)
    acc = S[0] * w4[:, 0] + S[1] * w4[:, 1] + S[2] * w4[:, 2] + r * w4[:, 3]
    seam_ok(q16.cpu().numpy().view(np.float16), O.silu(acc))
    S1 = st.cpu().numpy().reshape(3, cd + 16)
    S0 = st0.cpu().numpy().reshape(3, cd + 16)
    assert np.array_equal(S1[0, :cd], S0[1, :cd]) and np.array_equal(S1[1, :cd], S0[2, :cd])
    assert np.array_equal(S1[2, :cd], raw.cpu().numpy())
    assert np.array_equal(S1[:, cd:], S0[:, cd:])                       # padding untouched
    ab = deq(O, wa, sa) @ xs
    e_ref = np.exp(ssm_a.double().cpu().numpy() * O.softplus(ab[:vh] + dt.double().cpu().numpy()))
    assert rel(eg.double().cpu().numpy(), e_ref) <= 1e-5
    assert rel(beta.double().cpu().numpy(), O.sigmoid(ab[vh:])) <= 1e-5


def test_argmax_epilogue_first_max(cuda, L, O):
    """Logits and the first-max key; duplicated rows tie exactly and the lower
    global index must win (ref/run9b.c:399-405)."""
    torch = cuda
    K, V = 2048, 20000
    wq, sc = weights(torch, V, K, 41)
    x = torch.randn(K, generator=torch.Generator().manual_seed(42)).half().cuda()
    xs = O.stage_g128(x.cpu().numpy().astype(np.float64))
    top = int(np.argmax(deq(O, wq, sc) @ xs))
    wq[17000] = wq[top]                                  # a later row with the same weights ties
    sc[17000] = sc[top]
    wq[3] = wq[top]                                      # an earlier one wins the tie
    sc[3] = sc[top]
    logits = torch.zeros(V, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=1, key=dp(key), idx0=5000)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=V, epi=EPI["ARGMAX"], out_f32=dp(logits))
    run(L, torch, p)
    lg = logits.cpu().numpy()
    assert lg[3] == lg[top] == lg[17000]
    k = int(key.item()) & 0xFFFFFFFF
    assert 0xFFFFFFFF - k == 5000 + min(3, top)
    assert rel(lg.astype(np.float64), deq(O, wq, sc) @ xs) <= 2e-6


def test_programmatic_dependent_chain(cuda, L, O):
    """Four launches, each reading the previous one's fp16 output, as
    programmatic dependents: same result as plain launches."""
    torch = cuda
    K = 2048
    mats = [weights(torch, K, K, 50 + i) for i in range(4)]
    x0 = torch.randn(K, generator=torch.Generator().manual_seed(51)).half().cuda()
    outs = {}
    s = torch.cuda.Stream()
    for pdl in (0, 1):
        bufs = [x0] + [torch.zeros(K, dtype=torch.float16, device="cuda") for _ in range(4)]
        torch.cuda.synchronize()
        for i, (wq, sc) in enumerate(mats):
            p = Params(K=K, op=OP["F16"], x=dp(bufs[i]), njobs=1, pf_bytes=65536)
            p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=K, epi=EPI["F16"], out_f16=dp(bufs[i + 1]))
            assert L.dec_k_matvec(C.byref(p), C.c_void_p(s.cuda_stream), pdl) == 0
        torch.cuda.synchronize()
        outs[pdl] = bufs[4].cpu().numpy()
    assert np.array_equal(outs[0], outs[1])
    y = x0.cpu().numpy().astype(np.float64)
    for wq, sc in mats:
        y = (deq(O, wq, sc) @ O.stage_g128(y)).astype(np.float16).astype(np.float64)
    assert rel(outs[1].astype(np.float64), y) <= 1e-2     # four fp16 roundings of chained random products


def test_refusals(cuda, L):
    torch = cuda
    wq, sc = weights(torch, 8, 256, 60)
    x = torch.zeros(256, dtype=torch.float16, device="cuda")
    y = torch.zeros(8, device="cuda")

    def p(**kw):
        q = Params(K=kw.pop("K", 256), op=kw.pop("op", 0), x=dp(x), njobs=kw.pop("njobs", 1))
        q.jobs[0] = Job(s_pitch=spitch(256), wq=dp(wq), sc=dp(sc), rows=8, epi=EPI["F32"], out_f32=dp(y))
        for k, v in kw.items():
            setattr(q.jobs[0], k, v)
        return q
    assert L.dec_k_matvec(C.byref(p(K=200)), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p(K=65536)), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p(njobs=0)), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p(njobs=5)), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p(op=1)), None, 0) == -11                   # RMSNORM without weights
    assert L.dec_k_matvec(C.byref(p(out_f32=None)), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p(wq=dp(wq) + 8)), None, 0) == -11          # 16-byte alignment
    assert L.dec_k_matvec(C.byref(p(s_pitch=2)), None, 0) == -11              # scale rows not 16 bytes
    assert L.dec_k_matvec(C.byref(p(epi=EPI["SWIGLU"])), None, 0) == -11      # unpaired SwiGLU
    assert L.dec_k_matvec(C.byref(p(epi=9)), None, 0) == -11
    q = p()
    q.nvec, q.xs = 9, 256                                                    # more than 8 vectors
    assert L.dec_k_matvec(C.byref(q), None, 0) == -11
    q.nvec, q.xs = 2, 128                                                    # inputs overlap
    assert L.dec_k_matvec(C.byref(q), None, 0) == -11
    q = p(ostride=4)
    q.nvec, q.xs = 2, 256                                                    # outputs overlap
    assert L.dec_k_matvec(C.byref(q), None, 0) == -11
    assert L.dec_k_matvec(C.byref(p()), None, 0) == 0
    torch.cuda.synchronize()


# ------------------------------------------------------------------ batches

def staged_ref(O, W, x16):
    return W @ O.stage_g128(np.asarray(x16, dtype=np.float64))


@pytest.mark.parametrize("nv", [2, 3, 4, 8])
@pytest.mark.parametrize("K,rows", [(128, 5), (2048, 96), (2048, 2048), (6144, 2048), (2048, 20000)])
def test_batch_f16_inputs(cuda, L, O, nv, K, rows):
    """nv fp16 vectors at a padded stride: every vector's fp32, fp16 and
    accumulate outputs equal its own staged product; few rows take the
    column split over warps."""
    torch = cuda
    wq, sc = weights(torch, rows, K, 3 * K + rows + nv)
    g = torch.Generator().manual_seed(K + nv)
    xs_ = K + 64
    xb = (torch.randn(nv, xs_, generator=g) * torch.exp2(torch.randint(-8, 3, (nv, xs_), generator=g).float())).half().cuda()
    os_ = rows + 8
    y32 = torch.full((nv, os_), 7.0, device="cuda")
    y16 = torch.zeros(nv, os_, dtype=torch.int16, device="cuda")
    acc = torch.randn(nv, os_, generator=g).cuda()
    acc0 = acc.clone()
    p = Params(K=K, op=OP["F16"], x=dp(xb), njobs=3, pf_bytes=65536, nvec=nv, xs=xs_)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y32), ostride=os_)
    p.jobs[1] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F16"], out_f16=dp(y16), ostride=os_)
    p.jobs[2] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["ACC"], out_f32=dp(acc), ostride=os_)
    run(L, torch, p)
    W = deq(O, wq, sc)
    X = xb.cpu().numpy()[:, :K]
    Y32, Y16 = y32.cpu().numpy(), y16.cpu().numpy().view(np.float16)
    D = (acc - acc0).cpu().numpy()
    for b in range(nv):
        ref = staged_ref(O, W, X[b])
        got = Y32[b, :rows].astype(np.float64)
        assert rel(got, ref) <= 2e-6, b
        assert np.array_equal(Y16[b, :rows], got.astype(np.float32).astype(np.float16))
        assert np.allclose(D[b, :rows], got, rtol=0, atol=1e-6 * np.max(np.abs(got)))
        assert np.all(Y32[b, rows:] == 7.0) and np.all(D[b, rows:] == 0)    # past the rows: untouched


@pytest.mark.parametrize("nv", [2, 8])
def test_batch_rmsnorm_and_seams(cuda, L, O, nv):
    torch = cuda
    K, rows = 2048, 700
    wq, sc = weights(torch, rows, K, 70 + nv)
    g = torch.Generator().manual_seed(71)
    res = (torch.randn(nv, K, generator=g) * (1 + torch.arange(nv).float()[:, None])).cuda()
    w = (1 + 0.1 * torch.randn(K, generator=g)).cuda()
    seam = torch.zeros(nv, K, dtype=torch.int16, device="cuda")
    y = torch.zeros(nv, rows, device="cuda")
    p = Params(K=K, op=OP["RMSNORM"], x=dp(res), nw=dp(w), eps=1e-6, seam=dp(seam), njobs=1, nvec=nv, xs=K)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y), ostride=rows)
    run(L, torch, p)
    W = deq(O, wq, sc)
    H16 = seam.cpu().numpy().view(np.float16)
    R, wn, Y = res.double().cpu().numpy(), w.double().cpu().numpy(), y.cpu().numpy().astype(np.float64)
    for b in range(nv):
        seam_ok(H16[b], O.rmsnorm(R[b], wn, 1e-6))
        assert rel(Y[b], staged_ref(O, W, H16[b])) <= 2e-6


def test_batch_gated_conv_gates(cuda, L, O):
    """DeltaNet shapes at batch 4: the gated prologue per vector, the conv
    epilogue on each sequence's own rolling state, the gates per vector."""
    torch = cuda
    nv, H, cd, vh = 4, 4, 768, 6
    K = H * 128
    g = torch.Generator().manual_seed(81)
    o = torch.randn(nv, K, generator=g).cuda()
    z = (2 * torch.randn(nv, K, generator=g)).cuda()
    w = (1 + 0.1 * torch.randn(128, generator=g)).cuda()
    seam = torch.zeros(nv, K, dtype=torch.int16, device="cuda")
    wc, scc = weights(torch, cd, K, 82)
    wa, sa = weights(torch, 2 * vh, K, 83)
    cw = (0.5 * torch.randn(cd * 4, generator=g)).cuda()
    st = (0.5 * torch.randn(nv, 3, cd, generator=g)).cuda()
    st0 = st.clone()
    ssm_a = (-1 + 0.2 * torch.randn(vh, generator=g)).cuda()
    dt = (0.5 * torch.randn(vh, generator=g)).cuda()
    q16 = torch.zeros(nv, cd, dtype=torch.int16, device="cuda")
    raw = torch.zeros(nv, cd, device="cuda")
    eg, beta = torch.zeros(nv, vh, device="cuda"), torch.zeros(nv, vh, device="cuda")
    p = Params(K=K, op=OP["GATED"], x=dp(o), x2=dp(z), nw=dp(w), eps=1e-6, seam=dp(seam), njobs=2, nvec=nv, xs=K)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wc), sc=dp(scc), rows=cd, epi=EPI["CONV"], out_f16=dp(q16),
                    out_f32=dp(raw), p0=dp(cw), st=dp(st), st_stride=cd, ostride=cd)
    p.jobs[1] = Job(s_pitch=spitch(K), wq=dp(wa), sc=dp(sa), rows=2 * vh, epi=EPI["GATES"], out_f32=dp(eg),
                    out2_f32=dp(beta), p0=dp(ssm_a), p1=dp(dt), n1=vh, ostride=vh)
    run(L, torch, p)
    on, zn, wn = o.double().cpu().numpy(), z.double().cpu().numpy(), w.double().cpu().numpy()
    Wc, Wa = deq(O, wc, scc), deq(O, wa, sa)
    w4 = cw.cpu().numpy().astype(np.float64).reshape(cd, 4)
    S0, S1 = st0.cpu().numpy().astype(np.float64), st.cpu().numpy()
    for b in range(nv):
        want = np.concatenate([O.rmsnorm(on[b, 128 * i:128 * (i + 1)], wn, 1e-6) * O.silu(zn[b, 128 * i:128 * (i + 1)])
                               for i in range(H)])
        y16 = seam.cpu().numpy().view(np.float16)[b]
        seam_ok(y16, want)
        proj = staged_ref(O, Wc, y16)
        r = raw.cpu().numpy()[b].astype(np.float64)
        assert rel(r, proj) <= 2e-6
        a = S0[b, 0] * w4[:, 0] + S0[b, 1] * w4[:, 1] + S0[b, 2] * w4[:, 2] + r * w4[:, 3]
        seam_ok(q16.cpu().numpy().view(np.float16)[b], O.silu(a))
        assert np.array_equal(S1[b, 0], S0[b, 1].astype(np.float32)) and np.array_equal(S1[b, 2], raw.cpu().numpy()[b])
        ab = staged_ref(O, Wa, y16)
        e_ref = np.exp(ssm_a.double().cpu().numpy() * O.softplus(ab[:vh] + dt.double().cpu().numpy()))
        assert rel(eg[b].double().cpu().numpy(), e_ref) <= 1e-5
        assert rel(beta[b].double().cpu().numpy(), O.sigmoid(ab[vh:])) <= 1e-5


@pytest.mark.parametrize("nv", [2, 8])
def test_batch_paired_swiglu(cuda, L, O, nv):
    torch = cuda
    K, F = 2048, 6144
    wg, sg = weights(torch, F, K, 91)
    wu, su = weights(torch, F, K, 92)
    x = torch.randn(nv, K, generator=torch.Generator().manual_seed(93)).half().cuda()
    h = torch.zeros(nv, F, dtype=torch.int16, device="cuda")
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=1, nvec=nv, xs=K)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wg), wq2=dp(wu), sc=dp(sg), sc2=dp(su), rows=F, epi=EPI["SWIGLU"],
                    out_f16=dp(h), ostride=F)
    run(L, torch, p)
    Wg, Wu = deq(O, wg, sg), deq(O, wu, su)
    for b in range(nv):
        xs = O.stage_g128(x[b].cpu().numpy().astype(np.float64))
        want = O.silu(Wg @ xs) * (Wu @ xs)
        got = h[b].cpu().numpy().view(np.float16).astype(np.float64)
        assert np.all(np.abs(got - want) <= 2.0 ** -10 * np.abs(want) + 1e-6 * np.max(np.abs(want))), b


def test_batch_argmax_keys(cuda, L, O):
    """One first-max key per vector; vector 1's winner is planted as a tie
    with an earlier row."""
    torch = cuda
    nv, K, V = 8, 2048, 30000
    wq, sc = weights(torch, V, K, 101)
    x = torch.randn(nv, K, generator=torch.Generator().manual_seed(102)).half().cuda()
    W = deq(O, wq, sc)
    top1 = int(np.argmax(staged_ref(O, W, x[1].cpu().numpy())))
    e = 11 if top1 != 11 else 12
    wq[e] = wq[top1]
    sc[e] = sc[top1]
    W = deq(O, wq, sc)
    logits = torch.zeros(nv, V, device="cuda")
    key = torch.zeros(nv, dtype=torch.int64, device="cuda")
    p = Params(K=K, op=OP["F16"], x=dp(x), njobs=1, key=dp(key), idx0=100, nvec=nv, xs=K)
    p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=V, epi=EPI["ARGMAX"], out_f32=dp(logits), ostride=V)
    run(L, torch, p)
    lg = logits.cpu().numpy()
    for b in range(nv):
        ref = staged_ref(O, W, x[b].cpu().numpy())
        assert rel(lg[b].astype(np.float64), ref) <= 2e-6
        want = int(np.flatnonzero(lg[b] == lg[b].max())[0])
        assert 0xFFFFFFFF - (int(key[b].item()) & 0xFFFFFFFF) == 100 + want, b
    assert 0xFFFFFFFF - (int(key[1].item()) & 0xFFFFFFFF) == 100 + min(e, top1)


@pytest.mark.parametrize("op", ["F16", "RMSNORM", "GATED"])
@pytest.mark.parametrize("nv,K", [(1, 2048), (1, 6144), (1, 17408), (3, 2048), (8, 2048), (8, 6144), (2, 17408)])
def test_prestaged_inputs_equal_in_cta_staging(cuda, L, O, op, nv, K):
    """dec_k_stage stages the inputs once into a global block and the matvec
    copies it: the same arithmetic as staging in every CTA, so outputs and
    seams are bit-identical; chained as programmatic dependents too.  The
    single-sequence RMSNorm prologue keeps its units in registers up to 2 per
    thread (K = 2048, 6144) and reads the residual twice beyond (K = 17408):
    both give the staging launch's bits."""
    torch = cuda
    L.dec_k_stage.argtypes = [C.POINTER(Params), P_, C.c_int]
    L.dec_k_stage.restype = C.c_int
    L.dec_k_stage_bytes.argtypes = [C.c_int, C.c_int]
    L.dec_k_stage_bytes.restype = C.c_longlong
    rows = 1000
    wq, sc = weights(torch, rows, K, 7 * K + nv)
    g = torch.Generator().manual_seed(K + 13 * nv)
    xs_ = K + 64
    if op == "F16":
        x = (torch.randn(nv, xs_, generator=g) * torch.exp2(torch.randint(-8, 3, (nv, xs_), generator=g).float())).half().cuda()
    else:
        x = (torch.randn(nv, xs_, generator=g) * (1 + torch.arange(nv).float()[:, None])).cuda()
    z = (2 * torch.randn(nv, xs_, generator=g)).cuda()
    w = (1 + 0.1 * torch.randn(K, generator=g)).cuda()
    nbytes = L.dec_k_stage_bytes(K, nv)
    assert nbytes > 0
    xst = torch.zeros(nbytes // 4 + 4, dtype=torch.int32, device="cuda")
    outs = []
    for mode in range(3):
        y = torch.zeros(nv, rows, device="cuda")
        acc = torch.ones(nv, rows, device="cuda")
        seam = torch.zeros(nv, K, dtype=torch.int16, device="cuda")
        p = Params(K=K, op=OP[op], x=dp(x), x2=dp(z) if op == "GATED" else None, nw=dp(w), eps=1e-6,
                   seam=dp(seam), njobs=2, nvec=nv, xs=xs_, pf_bytes=65536)
        p.jobs[0] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["F32"], out_f32=dp(y), ostride=rows)
        p.jobs[1] = Job(s_pitch=spitch(K), wq=dp(wq), sc=dp(sc), rows=rows, epi=EPI["ACC"], out_f32=dp(acc),
                        ostride=rows)
        if mode:
            xst.zero_()
            p.xst = dp(xst)
            assert L.dec_k_stage(C.byref(p), None, mode - 1) == 0
            assert L.dec_k_matvec(C.byref(p), None, mode - 1) == 0
        else:
            assert L.dec_k_matvec(C.byref(p), None, 0) == 0
        torch.cuda.synchronize()
        outs.append((y.cpu().numpy(), acc.cpu().numpy(), seam.cpu().numpy()))
    for mode in (1, 2):
        for a, b in zip(outs[0], outs[mode]):
            assert np.array_equal(a, b), mode
    # and the staged product itself against the oracle (vector nv - 1)
    W = deq(O, wq, sc)
    s16 = outs[0][2][nv - 1].view(np.float16)
    assert rel(outs[1][0][nv - 1].astype(np.float64), staged_ref(O, W, s16)) <= 2e-6


def test_stage_refusals(cuda, L):
    torch = cuda
    L.dec_k_stage.argtypes = [C.POINTER(Params), P_, C.c_int]
    L.dec_k_stage.restype = C.c_int
    L.dec_k_stage_bytes.argtypes = [C.c_int, C.c_int]
    L.dec_k_stage_bytes.restype = C.c_longlong
    x = torch.zeros(2048, dtype=torch.float16, device="cuda")
    buf = torch.zeros(8192, dtype=torch.int32, device="cuda")
    assert L.dec_k_stage(C.byref(Params(K=2048, op=OP["F16"], x=dp(x))), None, 0) == -11          # no block
    assert L.dec_k_stage(C.byref(Params(K=2000, op=OP["F16"], x=dp(x), xst=dp(buf))), None, 0) == -11
    assert L.dec_k_stage(C.byref(Params(K=2048, op=OP["F16"], x=dp(x), xst=dp(buf) + 4)), None, 0) == -11
    assert L.dec_k_stage(C.byref(Params(K=2048, op=OP["RMSNORM"], x=dp(x), xst=dp(buf))), None, 0) == -11
    assert L.dec_k_stage_bytes(2048, 9) < 0 and L.dec_k_stage_bytes(100, 1) < 0
    torch.cuda.synchronize()
