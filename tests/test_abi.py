"""The C-ABI library: it loads, exports every function include/*.h declares,
and its host-only entry points (parse, byte accessors) match the reference.
No compute call here needs a GPU."""
import ctypes as C
import os
import subprocess

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


GOLDEN_IMAGES = ["img%d" % g for g in range(6)] + ["lin0_img", "sat0_img"]


@pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built")
def test_accessors_match_reference(pkg, golden):
    """mv4i_parse's header fields and, element by element, mv4i_get_widx /
    mv4i_get_scale against the reference's own parse and static accessors
    (ref/matvec_int4.c:161-307, through oracle/_ref) on every golden image:
    AXI widths 64-256, ROWS_IF 4 and 8, the IQ4_NL and linear codebooks."""
    L, R = pkg.lib(), O.ref()
    R.ref_dump_layout.restype = C.c_int
    R.ref_dump_layout.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    for key in GOLDEN_IMAGES:
        img = golden[key].tobytes()
        pi = pkg.ParsedImage(img)
        assert pi.rc == 0, key
        h = pi.f.h
        M, K, nb = h.M, h.K, (h.K + 31) // 32
        vals = [C.c_int(0) for _ in range(4)]
        buf = np.frombuffer(img, np.uint8).copy()
        assert R.ref_parse(O._p(buf), buf.size, *[C.byref(v) for v in vals]) == 0
        assert (M, K, h.w_exp, h.out_shift) == tuple(v.value for v in vals), key
        widx = np.zeros((M, K), np.uint8)
        scl = np.zeros((M, nb), np.uint16)
        assert R.ref_dump_layout(O._p(buf), buf.size, O._p(widx), O._p(scl)) == 0
        got_w = np.array([[L.mv4i_get_widx(C.byref(pi.f), r, k) for k in range(K)] for r in range(M)])
        got_s = np.array([[L.mv4i_get_scale(C.byref(pi.f), r, b) for b in range(nb)] for r in range(M)])
        assert np.array_equal(got_w, widx), key
        assert np.array_equal(got_s, scl), key


CONSUMER = os.path.join(os.path.dirname(__file__), "c_consumer", "mv4i_consumer.c")


def build_consumer(pkg, out_dir):
    """gcc a plain C program against include/mv4i_b200.h and -lmv4i_b200."""
    exe = os.path.join(out_dir, "mv4i_consumer")
    libdir = os.path.dirname(pkg.LIBPATH)
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-O2", "-I" + os.path.join(pkg.ROOT, "include"),
           "-o", exe, CONSUMER, "-L" + libdir, "-lmv4i_b200", "-Wl,-rpath," + libdir]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


def test_c_consumer_builds_and_parses(pkg, golden, tmp_path):
    """The boundary as a C caller sees it: the header compiles as C11 with
    warnings as errors, the program links against the shared library, and its
    mv4i_parse reads every golden image's header as the reference does (no
    GPU needed for parse)."""
    exe = build_consumer(pkg, str(tmp_path))
    for key in GOLDEN_IMAGES:
        img = golden[key].tobytes()
        path = tmp_path / (key + ".mv4i")
        path.write_bytes(img)
        out = subprocess.run([exe, "parse", str(path)], capture_output=True, text=True, check=True).stdout.split()
        rc, M, K, w_exp, out_shift = [int(v) for v in out[:5]]
        pi = pkg.ParsedImage(img)
        assert (rc, M, K, w_exp, out_shift) == (0, pi.f.h.M, pi.f.h.K, pi.f.h.w_exp, pi.f.h.out_shift)
    bad = tmp_path / "bad.mv4i"
    bad.write_bytes(b"\0" * 100)
    out = subprocess.run([exe, "parse", str(bad)], capture_output=True, text=True, check=True).stdout.split()
    assert int(out[0]) < 0


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
