"""Seam tests: the attention kernels and the step advance of the decode step
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
        "dec_k_attn_pre": [P, P, I, I, I, I, F, F, P, P, P, I, P, P, P, P, P, I],
        "dec_k_attention": [P, P, P, I, I, I, I, I, P, P, P, P, P, I],
        "dec_k_advance": [P, I, P, P, P, P, I, P, P, I],
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


@pytest.mark.parametrize("pos", [0, 1, 77, 4095])
def test_attn_pre_norm_rope_and_cache_write(cuda, K, O, pos):
    torch = cuda
    g = torch.Generator().manual_seed(4 + pos)
    qh, kvh, nrot, theta, ctx = 8, 2, 32, 1e6, 4096
    qg, kv = torch.randn(qh * 2 * HD, generator=g) * 2, torch.randn(2 * kvh * HD, generator=g) * 2
    qn, kn = 1 + 0.1 * torch.randn(HD, generator=g), 1 + 0.1 * torch.randn(HD, generator=g)
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    qo, go = torch.zeros(qh * HD, device="cuda"), torch.zeros(qh * HD, device="cuda")
    kc = torch.zeros(ctx * kvh * HD, dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    assert K.dec_k_attn_pre(ptr(qg.cuda()), ptr(kv.cuda()), qh, kvh, HD, nrot, theta, 1e-6, ptr(qn.cuda()),
                            ptr(kn.cuda()), ptr(dpos), ctx, ptr(qo), ptr(go), ptr(kc), ptr(vc), None, 0) == 0

    def rope(r):
        r = r.copy()
        half = nrot // 2
        for i in range(half):
            th = pos * theta ** (-2.0 * i / nrot)
            a, b = r[i], r[i + half]
            r[i], r[i + half] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
        return r

    qgn = qg.double().numpy().reshape(qh, 2, HD)
    qref = np.stack([rope(O.rmsnorm(qgn[h, 0], qn.double().numpy(), 1e-6)) for h in range(qh)])
    assert rel(qo.double().cpu().numpy(), qref.reshape(-1)) <= TOL
    assert np.array_equal(go.cpu().numpy(), qgn[:, 1].reshape(-1).astype(np.float32))
    kvn = kv.double().numpy().reshape(2, kvh, HD)
    kref = np.stack([rope(O.rmsnorm(kvn[0, h], kn.double().numpy(), 1e-6)) for h in range(kvh)])
    kcn = h16(kc).reshape(ctx, kvh, HD)
    assert rel(kcn[pos], kref) <= TOL
    assert np.array_equal(h16(vc).reshape(ctx, kvh, HD)[pos], O.f16(kvn[1]))
    others = np.delete(kcn, pos, axis=0)
    assert not np.any(others)


@pytest.mark.parametrize("qh,kvh,pos,ctx", [(8, 2, 0, 256), (8, 2, 63, 256), (8, 2, 64, 256), (16, 2, 200, 256),
                                            (4, 4, 255, 256), (32, 1, 130, 4096), (40, 8, 1000, 8192)])
def test_flash_decoding_attention(cuda, K, O, qh, kvh, pos, ctx):
    torch = cuda
    g = torch.Generator().manual_seed(qh * 1000 + pos)
    ch = 64
    nchunks = (ctx + ch - 1) // ch
    q = torch.randn(qh * HD, generator=g)
    kc = (torch.randn(ctx, kvh, HD, generator=g)).half()
    vc = (torch.randn(ctx, kvh, HD, generator=g)).half()
    gate = torch.randn(qh * HD, generator=g)
    part = torch.zeros(qh * nchunks * (HD + 4), device="cuda")
    y = torch.zeros(qh * HD, dtype=torch.int16, device="cuda")
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    kcd, vcd = kc.cuda(), vc.cuda()
    assert K.dec_k_attention(ptr(q.cuda()), ptr(kcd), ptr(vcd), qh, kvh, HD, ch, ctx, ptr(dpos), ptr(part),
                             ptr(gate.cuda()), ptr(y), None, 0) == 0
    qn = q.double().numpy().reshape(qh, HD)
    kn, vn = kc.double().numpy()[:pos + 1], vc.double().numpy()[:pos + 1]
    ref = np.empty((qh, HD))
    for h in range(qh):
        gk = h // (qh // kvh)
        sc = kn[:, gk] @ qn[h] / np.sqrt(HD)
        e = np.exp(sc - sc.max())
        ref[h] = (e @ vn[:, gk]) / e.sum()
    ref *= O.sigmoid(gate.double().numpy().reshape(qh, HD))
    assert rel(h16(y), ref.reshape(-1)) <= TOL


def test_attention_past_capacity_reads_only_the_cache(cuda, K):
    """A position at or past max_ctx (a replayed graph that ran past the end)
    attends over the max_ctx cached entries and writes nothing out of range."""
    torch = cuda
    qh, kvh, ctx = 8, 2, 128
    q = torch.randn(qh * HD, device="cuda")
    kc = torch.randn(ctx, kvh, HD, device="cuda").half()
    vc = torch.randn(ctx, kvh, HD, device="cuda").half()
    gate = torch.randn(qh * HD, device="cuda")
    part = torch.zeros(qh * 2 * (HD + 4), device="cuda")
    ya = torch.zeros(qh * HD, dtype=torch.int16, device="cuda")
    yb = torch.zeros_like(ya)
    for p, y in ((ctx - 1, ya), (ctx + 50, yb)):
        dpos = torch.tensor([p], dtype=torch.int32, device="cuda")
        assert K.dec_k_attention(ptr(q), ptr(kc), ptr(vc), qh, kvh, HD, 64, ctx, ptr(dpos), ptr(part), ptr(gate),
                                 ptr(y), None, 0) == 0
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)


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
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, None, None, 0) == 0
    torch.cuda.synchronize()
    assert int(tok.item()) == 40 and int(hist[3].item()) == 40 and int(pos.item()) == 4 and int(key.item()) == 0
    prompt = torch.tensor([6, 11, 12, 13, 14, 15, 16], dtype=torch.int32, device="cuda")   # length 6
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, ptr(prompt), None, 0) == 0
    torch.cuda.synchronize()
    assert int(hist[4].item()) == 40 and int(tok.item()) == 16 and int(pos.item()) == 5     # prompt[1 + 5]
    assert K.dec_k_advance(ptr(keys), 3, ptr(key), ptr(tok), ptr(hist), ptr(pos), 8, ptr(prompt), None, 0) == 0
    torch.cuda.synchronize()
    assert int(tok.item()) == 40 and int(pos.item()) == 6                                    # prompt over
