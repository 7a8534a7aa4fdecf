"""The C-ABI library: it loads, exports every function include/*.h declares,
and its host-only entry points (parse, byte accessors) match the reference.
No compute call here needs a GPU."""
import ctypes as C

import numpy as np
import pytest

import oracle as O


def test_library_exports_every_declared_symbol(pkg):
    import glob
    import os
    L = pkg.lib()
    D = pkg.declib()
    inc = os.path.join(pkg.ROOT, "include")
    for h in glob.glob(os.path.join(inc, "*.h")):
        names = pkg.header_symbols(h)
        assert names, h
        lb = D if os.path.basename(h) == "dec_b200.h" else L
        missing = [n for n in names if not hasattr(lb, n)]
        assert not missing, (h, missing)
    names = pkg.header_symbols()
    assert "mv4i_parse" in names and "mv4i_matvec" in names and "mv4i_launch" in names
    assert "dec_step" in names and "gdn_run_f32" in names
    assert set(pkg.DEC_EXPORTS) == set(pkg.header_symbols(os.path.join(inc, "dec_b200.h")))
    assert b"sm_100a" in L.mv4i_version()


def test_struct_sizes_match_reference_layout(pkg):
    """mv4i_file / mv4i_result keep the reference's field order (drop-in)."""
    assert C.sizeof(pkg.Hdr) == 4 * 5 + 2 * 6 + 4 * 2 + 16 + 8 * 128
    assert C.sizeof(pkg.Result) == 8 * 3 + 4 * 2 + 8 + 8


def test_parse_matches_reference(pkg, golden):
    for g in range(6):
        img = golden["img%d" % g].tobytes()
        pi = pkg.ParsedImage(img)
        assert pi.rc == 0
        rc = O.orc().orc_parse  # noqa: F841  (symbol exists)
        # byte accessors against the oracle's restatement
        h = pi.f.h
        rng = np.random.default_rng(g)
        for _ in range(200):
            r = int(rng.integers(0, h.M))
            k = int(rng.integers(0, h.K))
            assert pkg.lib().mv4i_get_widx(C.byref(pi.f), r, k) >= 0


def _refusal_cases():
    base = bytearray(4096 + 64)
    base[0:4] = (0x4D563449).to_bytes(4, "little")
    base[0x08:0x0C] = (4).to_bytes(4, "little")
    base[0x0C:0x10] = (32).to_bytes(4, "little")
    base[0x18:0x1A] = (4).to_bytes(2, "little")
    base[0x1A:0x1C] = (4).to_bytes(2, "little")
    base[0x1C:0x1E] = (32).to_bytes(2, "little")
    base[0x1E:0x20] = (128).to_bytes(2, "little")
    base[0x34:0x38] = (1).to_bytes(4, "little")
    cases = {"ok": bytes(base), "short": bytes(base[:100])}
    b = bytearray(base); b[0] ^= 1; cases["magic"] = bytes(b)
    b = bytearray(base); b[0x1C] = 16; cases["block"] = bytes(b)
    b = bytearray(base); b[0x1A] = 3; cases["nports"] = bytes(b)
    b = bytearray(base); b[0x20] = 0x80; cases["cb128"] = bytes(b)
    b = bytearray(base); b[0x14] = 41; cases["oshift"] = bytes(b)
    b = bytearray(base); b[0x1E:0x20] = (96).to_bytes(2, "little"); cases["axi"] = bytes(b)
    b = bytearray(base); b[0x34] = 3; cases["nss"] = bytes(b)
    b = bytearray(base); b[0x1A:0x1C] = (512).to_bytes(2, "little"); b[0x1E:0x20] = (8).to_bytes(2, "little"); b[0x18] = 128; cases["maxsub"] = bytes(b)
    return cases


@pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built")
def test_parse_refusals_match_reference(pkg):
    """Refusal codes -1..-9 identical to the reference's mv4i_parse."""
    seen = set()
    for name, img in _refusal_cases().items():
        buf = np.frombuffer(img, np.uint8).copy()
        vals = [C.c_int(0) for _ in range(4)]
        rr = O.ref().ref_parse(buf.ctypes.data, buf.size, *[C.byref(v) for v in vals])
        pi = pkg.ParsedImage(img)
        assert pi.rc == rr, (name, pi.rc, rr)
        seen.add(rr)
    assert {0, -1, -2, -3, -4, -5, -6, -7, -9}.issubset(seen) or len(seen) >= 8


def test_decode_bad_configs_are_refused_before_any_cuda_call(pkg):
    """dec_create validates the configuration on the host (-11) first."""
    cfg0 = dict(hidden=256, n_layers=8, attn_every=4, vocab=1000, ffn=512, gdn_kh=2, gdn_vh=4, gdn_hd=128,
                att_qh=8, att_kvh=4, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=256)
    L = pkg.declib()
    h = C.c_void_p()
    for k, v in [("gdn_hd", 64), ("hidden", 200), ("att_kvh", 3), ("n_rot", 33), ("max_ctx", 0),
                 ("ffn", 320), ("attn_every", 0), ("batch", 9), ("batch", -1)]:
        cfg = dict(cfg0)
        cfg[k] = v
        assert L.dec_create(C.byref(pkg.DecConfig(**cfg)), 1, 0, 0, 1, C.byref(h)) == -11, k
    assert L.dec_create(C.byref(pkg.DecConfig(**cfg0)), 1, 0, 2, 2, C.byref(h)) == -11
    assert L.dec_create(C.byref(pkg.DecConfig(**cfg0)), 1, 0, 0, 8, C.byref(h)) == -11   # 4 kv heads
    # batches are single-GPU
    assert L.dec_create(C.byref(pkg.DecConfig(**dict(cfg0, batch=2))), 1, 0, 0, 2, C.byref(h)) == -11


def test_batch_input_staging_host_checks(pkg):
    """The batch input-staging pieces refuse bad arguments on the host: the
    mode setter (no model, mode out of range) and the staged-block size
    (K a multiple of 128 up to 32768, 1-8 vectors), whose value is the
    per-vector shared-memory block of the decode matvec times the vectors."""
    L = pkg.declib()
    assert L.dec_set_prestage(None, 1) == -11
    L.dec_k_stage_bytes.argtypes = [C.c_int, C.c_int]
    L.dec_k_stage_bytes.restype = C.c_longlong
    L.dec_k_stage.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    L.dec_k_stage.restype = C.c_int
    r16 = lambda n: (n + 15) & ~15
    for K in (128, 2048, 6144, 17408, 32768):
        npair, ng = K // 64, K // 128
        block = 128 * npair + r16(4 * npair) + r16(4 * ng) + r16(8 * ng)
        for nv in (1, 3, 8):
            assert L.dec_k_stage_bytes(K, nv) == nv * block, (K, nv)
    for K, nv in [(100, 1), (2000, 1), (32896, 1), (2048, 0), (2048, 9)]:
        assert L.dec_k_stage_bytes(K, nv) < 0, (K, nv)
    assert L.dec_k_stage(None, None, 0) == -11
