"""The public one-token attention entry point gated_attn (include/dec_b200.h)
against a float64 restatement of the reference's float attention layer
(ref/run9b.c:786-872: q/k RMSNorm, NeoX RoPE, fp16 KV cache append, GQA
softmax over positions 0..pos, sigmoid gate of the raw projection).

Tolerance, elementwise: |y - ref| <= 1e-3 * |ref| + 1e-3 * 2^-10 * max|ref|
(fp32 arithmetic, fp16 output: the fp16 rounding alone is 2^-11 relative; the
absolute floor covers outputs that cancel to near zero)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HD = 128


def within(y, ref):
    err = np.abs(y - ref)
    bound = 1e-3 * np.abs(ref) + 1e-3 * 2.0 ** -10 * np.max(np.abs(ref))
    return bool(np.all(err <= bound)), float(np.max(err / (np.abs(ref) + 1e-30)))


def _rope(r, pos, nrot, theta):
    r = r.copy()
    half = nrot // 2
    for i in range(half):
        th = pos * theta ** (-2.0 * i / nrot)
        a, b = r[i], r[i + half]
        r[i], r[i + half] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
    return r


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


@pytest.mark.parametrize("qh,kvh,pos,ctx", [(16, 2, 4096, 4608), (8, 2, 0, 256), (40, 8, 8191, 8192),
                                            (5, 1, 77, 300), (32, 32, 130, 4096)])
def test_gated_attn_against_float64(cuda, pkg, qh, kvh, pos, ctx):
    torch = cuda
    L = pkg.declib()
    g = torch.Generator().manual_seed(qh * 7 + pos)
    nrot, theta, eps = 64, 1e6, 1e-6
    qg = torch.randn(qh * 2 * HD, generator=g)
    kv = torch.randn(2 * kvh * HD, generator=g)
    qn, kn = 1 + 0.1 * torch.randn(HD, generator=g), 1 + 0.1 * torch.randn(HD, generator=g)
    kc = torch.randn(ctx, kvh, HD, generator=g).half()
    vc = torch.randn(ctx, kvh, HD, generator=g).half()
    d = {k: v.cuda() for k, v in dict(qg=qg, kv=kv, qn=qn, kn=kn, kc=kc, vc=vc).items()}
    nb = L.gated_attn_work_bytes(qh, ctx)
    assert nb > 0
    work = torch.zeros(nb // 4, device="cuda")
    y = torch.zeros(qh * HD, dtype=torch.float16, device="cuda")
    qo = torch.zeros(qh * HD, device="cuda")
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    a = pkg.GatedAttnArgs(qh, kvh, HD, nrot, theta, eps, d["qg"].data_ptr(), d["kv"].data_ptr(),
                          d["qn"].data_ptr(), d["kn"].data_ptr(), dpos.data_ptr(), ctx, d["kc"].data_ptr(),
                          d["vc"].data_ptr(), y.data_ptr(), qo.data_ptr(), work.data_ptr(), 0)
    assert L.gated_attn(C.byref(a), None) == 0
    torch.cuda.synchronize()
    qgn = qg.double().numpy().reshape(qh, 2, HD)
    kvn = kv.double().numpy().reshape(2, kvh, HD)
    q = np.stack([_rope(_rms(qgn[h, 0], qn.double().numpy(), eps), pos, nrot, theta) for h in range(qh)])
    kcr, vcr = kc.double().numpy(), vc.double().numpy()
    kdev, vdev = d["kc"].double().cpu().numpy(), d["vc"].double().cpu().numpy()
    if pos < ctx:
        knew = np.stack([_rope(_rms(kvn[0, j], kn.double().numpy(), eps), pos, nrot, theta) for j in range(kvh)])
        assert within(kdev[pos], knew)[0]                  # the appended k (fp16 of the fp32 result)
        vcr[pos] = kvn[1].astype(np.float16)               # v is appended raw
        kcr[pos] = kdev[pos]
    ok, _ = within(qo.double().cpu().numpy().reshape(qh, HD), q)
    assert ok
    assert np.array_equal(kdev, kcr)                       # nothing else in the caches written
    assert np.array_equal(vdev, vcr)
    n = min(pos + 1, ctx)
    ref = np.empty((qh, HD))
    for h in range(qh):
        j = h // (qh // kvh)
        sc = kcr[:n, j] @ q[h] / np.sqrt(HD)
        e = np.exp(sc - sc.max())
        ref[h] = (e @ vcr[:n, j]) / e.sum() / (1 + np.exp(-qgn[h, 1]))
    ok, worst = within(y.double().cpu().numpy().reshape(qh, HD), ref)
    assert ok, worst


def test_gated_attn_refusals(cuda, pkg):
    L = pkg.declib()
    a = pkg.GatedAttnArgs()
    assert L.gated_attn(C.byref(a), None) == -11
    assert L.gated_attn_work_bytes(8, 0) == 0 and L.gated_attn_work_bytes(8, 70000) == 0
