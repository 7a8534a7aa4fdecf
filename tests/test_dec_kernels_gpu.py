"""Seam tests: the attention kernel and the step advance of the decode step
on identical inputs against the oracle's restatement of the same ref/run9b.c
stage (oracle/dec_oracle.py), within 1e-3 of the largest magnitude (fp32
arithmetic, fp16 outputs); the advance bit-exact.  The kernels are the
library's internal launchers (exported from libdec_b200.so, not part of the
header).  The projections and the vector ops folded into them are covered by
tests/test_dec_matvec_gpu.py."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3
HD = 128


@pytest.fixture(scope="module")
def K(pkg):
    L = pkg.declib()
    P, I, F, U64 = C.c_void_p, C.c_int, C.c_float, C.c_uint64
    sig = {
        "dec_k_attention": [P, P, P, P, I, I, I, F, F, P, I, I, P, P, P, P, P, I, P, I],
        "dec_k_advance": [P, I, P, P, P, P, I, P, I, P, I],
    }
    for n, a in sig.items():
        getattr(L, n).argtypes = a
        getattr(L, n).restype = C.c_int
    return L


def ptr(t):
    return C.c_void_p(t.data_ptr())


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def h16(t):
    return t.cpu().numpy().view(np.float16).astype(np.float64)


@pytest.fixture(scope="module")
def O():
    from oracle import dec_oracle
    return dec_oracle


def _attention_case(torch, O, qh, kvh, pos, ctx, ch, seed):
    """Random q|gate, k|v projections, norms and a random fp16 cache; returns
    the device tensors, the kernel's outputs and the oracle's."""
    g = torch.Generator().manual_seed(seed)
    nrot, theta = 32, 1e6
    nchunks = (ctx + ch - 1) // ch
    qg = torch.randn(qh * 2 * HD, generator=g) * 2
    kv = torch.randn(2 * kvh * HD, generator=g) * 2
    qn, kn = 1 + 0.1 * torch.randn(HD, generator=g), 1 + 0.1 * torch.randn(HD, generator=g)
    kc = torch.randn(ctx, kvh, HD, generator=g).half()
    vc = torch.randn(ctx, kvh, HD, generator=g).half()
    kc0, vc0 = kc.clone(), vc.clone()
    d = {k: v.cuda() for k, v in dict(qg=qg, kv=kv, qn=qn, kn=kn, kc=kc, vc=vc).items()}
    part = torch.zeros(qh * nchunks * (HD + 4), device="cuda")
    qseam = torch.zeros(qh * HD, device="cuda")
    y = torch.zeros(qh * HD, dtype=torch.int16, device="cuda")
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    return dict(d=d, part=part, qseam=qseam, y=y, dpos=dpos, nrot=nrot, theta=theta, kc0=kc0, vc0=vc0,
                qg=qg.double().numpy(), kv=kv.double().numpy(), qn=qn.double().numpy(), kn=kn.double().numpy())


def _rope(r, pos, nrot, theta):
    r = r.copy()
    half = nrot // 2
    for i in range(half):
        th = pos * theta ** (-2.0 * i / nrot)
        a, b = r[i], r[i + half]
        r[i], r[i + half] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
    return r


def _run_attention(K, torch, c, qh, kvh, pos, ctx, ch):
    d = c["d"]
    rc = K.dec_k_attention(ptr(d["qg"]), ptr(d["kv"]), ptr(d["qn"]), ptr(d["kn"]), qh, kvh, c["nrot"], c["theta"], 1e-6,
                           ptr(c["dpos"]), ctx, ch, ptr(c["part"]), ptr(c["qseam"]), ptr(d["kc"]), ptr(d["vc"]),
                           ptr(c["y"]), 1, None, 0)
    assert rc == 0
    torch.cuda.synchronize()


@pytest.mark.parametrize("qh,kvh,pos,ctx,ch", [(8, 2, 0, 256, 32), (8, 2, 31, 256, 32), (8, 2, 32, 256, 32),
                                               (16, 2, 200, 1024, 32), (4, 4, 255, 256, 32), (32, 1, 130, 4096, 32),
                                               (40, 8, 1000, 8192, 64), (5, 1, 8191, 8192, 64)])
def test_attention_step_against_oracle(cuda, K, O, qh, kvh, pos, ctx, ch):
    """q and the new k: RMSNorm + NeoX RoPE (ref/run9b.c:800-826); k, v into
    the fp16 cache at pos, nothing else written; GQA softmax attention over
    positions 0..pos with the sigmoid gate of the raw projection
    (ref/run9b.c:846-872), fp16 output."""
    torch = cuda
    c = _attention_case(torch, O, qh, kvh, pos, ctx, ch, qh * 1000 + pos)
    _run_attention(K, torch, c, qh, kvh, pos, ctx, ch)
    qgn = c["qg"].reshape(qh, 2, HD)
    q = np.stack([_rope(O.rmsnorm(qgn[h, 0], c["qn"], 1e-6), pos, c["nrot"], c["theta"]) for h in range(qh)])
    assert rel(c["qseam"].double().cpu().numpy().reshape(qh, HD), q) <= 1e-5
    kvn = c["kv"].reshape(2, kvh, HD)
    knew = np.stack([_rope(O.rmsnorm(kvn[0, g], c["kn"], 1e-6), pos, c["nrot"], c["theta"]) for g in range(kvh)])
    kc = c["d"]["kc"].cpu().double().numpy()
    vc = c["d"]["vc"].cpu().double().numpy()
    assert rel(kc[pos], knew) <= 1e-3
    assert np.array_equal(vc[pos], O.f16(kvn[1]))
    others = np.ones(ctx, bool)
    others[pos] = False
    assert np.array_equal(kc[others], c["kc0"].double().numpy()[others])
    assert np.array_equal(vc[others], c["vc0"].double().numpy()[others])
    ref = np.empty((qh, HD))
    for h in range(qh):
        gk = h // (qh // kvh)
        sc = kc[:pos + 1, gk] @ q[h] / np.sqrt(HD)
        e = np.exp(sc - sc.max())
        ref[h] = (e @ vc[:pos + 1, gk]) / e.sum()
    ref *= O.sigmoid(qgn[:, 1])
    assert rel(h16(c["y"]), ref.reshape(-1)) <= TOL


def test_attention_past_capacity_reads_only_the_cache(cuda, K, O):
    """A position at or past max_ctx (a replayed graph that ran past the end)
    writes nothing and attends over the max_ctx cached entries."""
    torch = cuda
    qh, kvh, ctx, ch, pos = 8, 2, 128, 32, 128 + 50
    c = _attention_case(torch, O, qh, kvh, pos, ctx, ch, 7)
    _run_attention(K, torch, c, qh, kvh, pos, ctx, ch)
    assert torch.equal(c["d"]["kc"].cpu(), c["kc0"]) and torch.equal(c["d"]["vc"].cpu(), c["vc0"])
    qgn = c["qg"].reshape(qh, 2, HD)
    q = np.stack([_rope(O.rmsnorm(qgn[h, 0], c["qn"], 1e-6), pos, c["nrot"], c["theta"]) for h in range(qh)])
    kc, vc = c["kc0"].double().numpy(), c["vc0"].double().numpy()
    ref = np.empty((qh, HD))
    for h in range(qh):
        gk = h // (qh // kvh)
        sc = kc[:, gk] @ q[h] / np.sqrt(HD)
        e = np.exp(sc - sc.max())
        ref[h] = (e @ vc[:, gk]) / e.sum()
    ref *= O.sigmoid(qgn[:, 1])
    assert rel(h16(c["y"]), ref.reshape(-1)) <= TOL


def test_advance_picks_first_max_key_and_follows_the_prompt(cuda, K):
    """The largest key wins (keys of equal value: the lower global index,
    ref/run9b.c:399-405); while a prompt lasts its next token is the input."""
    torch = cuda
    keys = torch.tensor([5 << 32 | 0xFFFFFFFF - 900, 7 << 32 | 0xFFFFFFFF - 1200, 7 << 32 | 0xFFFFFFFF - 40],
                        dtype=torch.int64, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    hist = torch.zeros(8, dtype=torch.int32, device="cuda")
    pos = torch.tensor([3], dtype=torch.int32, device="cuda")
    key = torch.ones(1, dtype=torch.int64, device="cuda")
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, None, 1, None, 0) == 0
    torch.cuda.synchronize()
    assert int(tok.item()) == 40 and int(hist[3].item()) == 40 and int(pos.item()) == 4 and int(key.item()) == 0
    prompt = torch.tensor([6, 11, 12, 13, 14, 15, 16], dtype=torch.int32, device="cuda")   # length 6
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, ptr(prompt), 1, None, 0) == 0
    torch.cuda.synchronize()
    assert int(hist[4].item()) == 40 and int(tok.item()) == 16 and int(pos.item()) == 5     # prompt[1 + 5]
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, ptr(prompt), 1, None, 0) == 0
    torch.cuda.synchronize()
    assert int(tok.item()) == 40 and int(pos.item()) == 6                                    # prompt over


def _attention_ref(O, c, qh, kvh, pos, kc, vc):
    qgn = c["qg"].reshape(qh, 2, HD)
    q = np.stack([_rope(O.rmsnorm(qgn[h, 0], c["qn"], 1e-6), pos, c["nrot"], c["theta"]) for h in range(qh)])
    ref = np.empty((qh, HD))
    for h in range(qh):
        gk = h // (qh // kvh)
        sc = kc[:pos + 1, gk] @ q[h] / np.sqrt(HD)
        e = np.exp(sc - sc.max())
        ref[h] = (e @ vc[:pos + 1, gk]) / e.sum()
    return q, ref * O.sigmoid(qgn[:, 1])


def test_attention_batch_of_sequences(cuda, K, O):
    """Three sequences in one launch (grid z): each attends over its own
    cache with its own projections at the shared position, and writes its
    own cache row, q seam and output."""
    torch = cuda
    nseq, qh, kvh, ctx, ch, pos = 3, 16, 2, 512, 32, 300
    cs = [_attention_case(torch, O, qh, kvh, pos, ctx, ch, 500 + b) for b in range(nseq)]
    cat = lambda k: torch.stack([c["d"][k] for c in cs]).contiguous()
    qg, kv, kc, vc = cat("qg"), cat("kv"), cat("kc"), cat("vc")
    nchunks = (ctx + ch - 1) // ch
    part = torch.zeros(nseq * qh * nchunks * (HD + 4), device="cuda")
    qseam = torch.zeros(nseq, qh * HD, device="cuda")
    y = torch.zeros(nseq, qh * HD, dtype=torch.int16, device="cuda")
    c0 = cs[0]
    rc = K.dec_k_attention(ptr(qg), ptr(kv), ptr(c0["d"]["qn"]), ptr(c0["d"]["kn"]), qh, kvh, c0["nrot"], c0["theta"],
                           1e-6, ptr(c0["dpos"]), ctx, ch, ptr(part), ptr(qseam), ptr(kc), ptr(vc), ptr(y), nseq, None, 0)
    assert rc == 0
    torch.cuda.synchronize()
    for b, c in enumerate(cs):
        c["qn"], c["kn"] = c0["qn"], c0["kn"]                 # the norms are shared weights
        kcb, vcb = kc[b].cpu().double().numpy(), vc[b].cpu().double().numpy()
        others = np.ones(ctx, bool)
        others[pos] = False
        assert np.array_equal(kcb[others], c["kc0"].double().numpy()[others])
        kvn = c["kv"].reshape(2, kvh, HD)
        assert np.array_equal(vcb[pos], O.f16(kvn[1]))
        q, ref = _attention_ref(O, c, qh, kvh, pos, kcb, vcb)
        assert rel(qseam[b].double().cpu().numpy().reshape(qh, HD), q) <= 1e-5
        assert rel(h16(y[b]), ref.reshape(-1)) <= TOL, b


def test_advance_batch(cuda, K):
    """Two sequences: each takes its own first max and its own prompt token;
    the shared position advances once."""
    torch = cuda
    big = lambda v, i: v << 32 | 0xFFFFFFFF - i
    keys = torch.tensor([big(5, 900), big(9, 4), big(7, 1200), big(9, 3)], dtype=torch.int64, device="cuda")  # [rank][seq]
    tok = torch.zeros(2, dtype=torch.int32, device="cuda")
    hist = torch.zeros(2, 8, dtype=torch.int32, device="cuda")
    pos = torch.tensor([2], dtype=torch.int32, device="cuda")
    key = torch.ones(2, dtype=torch.int64, device="cuda")
    prompt = torch.tensor([5, 10, 11, 12, 13, 14, 20, 21, 22, 23, 24], dtype=torch.int32, device="cuda")
    assert K.dec_k_advance(ptr(keys), 2, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, ptr(prompt), 2, None, 0) == 0
    torch.cuda.synchronize()
    assert hist[0, 2].item() == 1200 and hist[1, 2].item() == 3
    assert tok.tolist() == [13, 23] and int(pos.item()) == 3 and key.tolist() == [0, 0]
