"""The library's offline weight path (llm.vhdl_b200/csrc/mv4i_pack.c) against
the reference's own packer, tools/pack_int4.py: for every case of
tests/golden/pack_golden.npz (seeded float32 matrices over normal, heavy-tailed,
uniform, tiny and zero-row distributions, K % 32 != 0, several ROWS_IF /
AXI_DW geometries) mv4i_quantize must give the reference's indices, scales
and w_exp, mv4i_calibrate_out_shift its out_shift, and mv4i_pack its image
byte for byte.  The image must then parse and read back through the
library's own parse and accessors.  CPU only (host code)."""
import ctypes as C
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "pack_golden.npz")


@pytest.fixture(scope="module")
def pg():
    return np.load(GOLD)


def _cases(pg):
    return sorted({k.split("_")[0] for k in pg.files if k.startswith("c") and k.endswith("_meta")},
                  key=lambda s: int(s[1:]))


def test_quantize_matches_reference(pkg, pg):
    L = pkg.lib()
    cb = np.ascontiguousarray(pg["cb"], np.int8)
    for c in _cases(pg):
        M, K, ri, dw, w_exp, osh = [int(v) for v in pg[c + "_meta"]]
        W = np.ascontiguousarray(pg[c + "_W"], np.float32)
        NB = (K + 31) // 32
        idx = np.zeros((M, NB, 32), np.uint8)
        scl = np.zeros((M, NB), np.uint16)
        we = C.c_int(0)
        assert L.mv4i_quantize(W.ctypes.data, M, K, cb.ctypes.data, idx.ctypes.data, scl.ctypes.data,
                               C.byref(we)) == 0
        assert we.value == w_exp, c
        assert np.array_equal(scl, pg[c + "_scl"]), c
        assert np.array_equal(idx, pg[c + "_idx"]), c


def test_out_shift_matches_reference(pkg, pg):
    L = pkg.lib()
    for K, want in pg["out_shift_K"]:
        assert L.mv4i_calibrate_out_shift(int(K)) == int(want), K
    assert L.mv4i_calibrate_out_shift(0) == -11


def test_pack_matches_reference_and_reads_back(pkg, pg):
    L = pkg.lib()
    cb = np.ascontiguousarray(pg["cb"], np.int8)
    for c in _cases(pg):
        M, K, ri, dw, w_exp, osh = [int(v) for v in pg[c + "_meta"]]
        assert L.mv4i_calibrate_out_shift(K) == osh
        want = pg[c + "_img"]
        n = L.mv4i_pack_size(M, K, ri, dw)
        assert n == want.size, c
        img = np.zeros(n, np.uint8)
        idx = np.ascontiguousarray(pg[c + "_idx"])
        scl = np.ascontiguousarray(pg[c + "_scl"])
        assert L.mv4i_pack(idx.ctypes.data, scl.ctypes.data, w_exp, M, K, ri, osh, cb.ctypes.data, dw,
                           img.ctypes.data) == 0
        assert np.array_equal(img, want), c
        pi = pkg.ParsedImage(img.tobytes())
        assert pi.rc == 0 and (pi.M, pi.K) == (M, K)
        for r in range(0, M, max(1, M // 7)):
            for k in range(0, K, max(1, K // 13)):
                assert L.mv4i_get_widx(C.byref(pi.f), r, k) == idx[r, k // 32, k % 32]
            for b in range(0, (K + 31) // 32, 3):
                assert L.mv4i_get_scale(C.byref(pi.f), r, b) == scl[r, b]


def test_pack_refusals(pkg):
    L = pkg.lib()
    assert L.mv4i_pack_size(8, 64, 3, 256) == 0          # 6.5 invariant does not divide
    assert L.mv4i_pack_size(8, 64, 4, 96) == 0           # not an AXI4 width
    assert L.mv4i_pack_size(8, 64, 4, 128) > 0
    unsorted = np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8)
    W = np.zeros((2, 64), np.float32)
    idx = np.zeros((2, 2, 32), np.uint8)
    scl = np.zeros((2, 2), np.uint16)
    we = C.c_int(0)
    assert L.mv4i_quantize(W.ctypes.data, 2, 64, unsorted.ctypes.data, idx.ctypes.data, scl.ctypes.data,
                           C.byref(we)) == -11


def test_image_to_g128_exact_or_refused(pkg):
    """A linear-codebook image with one scale per 128 columns converts to the
    decode engine's g128 layout exactly (dequantised values equal); a
    codebook or scale pattern g128 cannot hold is refused."""
    import oracle as O
    L = pkg.lib()
    rng = np.random.default_rng(5)
    M, K = 16, 512
    lin = np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8)
    idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
    g = rng.integers(1, 2048, (M, K // 128)).astype(np.uint16) * 8       # exact in fp16 at w_exp 5
    scl = np.repeat(g, 4, axis=1)
    img = O.pack(M, K, 4, 128, 5, 3, lin, idx, scl)
    pi = pkg.ParsedImage(img)
    wq = np.zeros((M, K // 2), np.uint8)
    sc = np.zeros((M, 8), np.uint16)
    assert L.mv4i_image_to_g128(C.byref(pi.f), wq.ctypes.data, sc.ctypes.data, 8) == 0
    nib = np.stack([wq & 15, wq >> 4], axis=2).reshape(M, K).astype(np.int64)
    val = np.where(nib >= 8, nib - 16, nib).astype(np.float64)
    deq_g = val * np.repeat(sc[:, :K // 128].view(np.float16).astype(np.float64), 128, axis=1)
    deq_ref = lin[idx].astype(np.float64) * np.repeat(scl.astype(np.float64), 32, axis=1) / 32768.0 * 2.0 ** -5
    assert np.array_equal(deq_g, deq_ref)
    scl2 = scl.copy()
    scl2[0, 1] += 1                                                         # scales differ inside a group
    pi2 = pkg.ParsedImage(O.pack(M, K, 4, 128, 5, 3, lin, idx, scl2))
    assert L.mv4i_image_to_g128(C.byref(pi2.f), wq.ctypes.data, sc.ctypes.data, 8) == -11
    pi3 = pkg.ParsedImage(O.pack(M, K, 4, 128, 5, 3, O.IQ4_NL, idx, scl))  # not the linear codebook
    assert L.mv4i_image_to_g128(C.byref(pi3.f), wq.ctypes.data, sc.ctypes.data, 8) == -11


def test_quantize_g128_matches_numpy(pkg):
    """The float -> g128 quantiser: scale = fp16(max|w| / 7) per 128 columns,
    q = clamp(rint(w / scale), -8, 7), restated in numpy."""
    L = pkg.lib()
    rng = np.random.default_rng(9)
    M, K = 12, 640
    W = (rng.standard_normal((M, K)) * rng.uniform(1e-4, 3.0, (M, 1))).astype(np.float32)
    W[3, 128:256] = 0.0                                        # an all-zero group
    wq = np.zeros((M, K // 2), np.uint8)
    sc = np.zeros((M, 8), np.uint16)
    assert L.mv4i_quantize_g128(W.ctypes.data, M, K, wq.ctypes.data, sc.ctypes.data, 8) == 0
    g = W.reshape(M, K // 128, 128)
    s16 = (np.abs(g).max(axis=2) / np.float32(7.0)).astype(np.float16)
    s32 = s16.astype(np.float32)[:, :, None]
    q = np.where(s32 > 0, np.clip(np.rint(g / np.where(s32 > 0, s32, 1)), -8, 7), 0).astype(np.int64)
    q = q.reshape(M, K)
    want = ((q[:, 0::2] & 15) | ((q[:, 1::2] & 15) << 4)).astype(np.uint8)
    assert np.array_equal(sc[:, :K // 128], s16.view(np.uint16))
    assert np.array_equal(wq, want)
    big = np.full((1, 128), 1e6, np.float32)
    assert L.mv4i_quantize_g128(big.ctypes.data, 1, 128, wq.ctypes.data, sc.ctypes.data, 8) == -11
