"""CPU oracle bindings -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, by __graft_entry__.smoke() and by the cpu_baseline leg of
bench.py, and only there, as the checker.  Two libraries:

* liboracle.so        -- the restatement in mv4i_oracle.c (this repository's
                         own code, citing the reference file:line it follows)
* _ref/libref_mv4i.so -- the reference's ref/matvec_int4.c compiled in place
                         from the llm.vhdl tree by oracle/Makefile (present
                         when it was built in a container that has the tree;
                         the built .so travels with the repository snapshot)
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# the llm.vhdl tree: $LLMVHDL_REF, else the directory `reference` beside this repository
REF_TREE = os.environ.get("LLMVHDL_REF") or os.path.normpath(os.path.join(HERE, "..", "..", "reference"))
LIB = os.path.join(HERE, "liboracle.so")
REFLIB = os.path.join(HERE, "_ref", "libref_mv4i.so")
REFBIN = os.path.join(HERE, "_ref", "matvec_int4")


def build():
    """Build liboracle.so; and the _ref artefacts when the reference tree exists."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if os.path.isdir(os.path.join(REF_TREE, "ref")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + REF_TREE], check=True)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


_o = None
_r = None


def orc():
    global _o
    if _o is None:
        L = C.CDLL(LIB)
        sig = {
            "orc_floor_shr": (C.c_int64, [C.c_int64, C.c_int]),
            "orc_round_shift": (C.c_int64, [C.c_int64, C.c_int]),
            "orc_sat32": (C.c_int32, [C.c_int64, C.c_void_p]),
            "orc_sat16": (C.c_int16, [C.c_int64]),
            "orc_msb_pos": (C.c_int, [C.c_uint64]),
            "orc_matvec": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p]),
            "orc_pack_size": (C.c_uint64, [C.c_int, C.c_int, C.c_int, C.c_int]),
            "orc_pack": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
            "orc_bfp_pack_f64": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
            "orc_bfp_pack_s64": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
            "orc_tp_reduce": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
            "orc_matvec_g128_f64": (None, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int64,
                                           C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
        }
        for n, (res, args) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = res, args
        _o = L
    return _o


def have_ref():
    return os.path.exists(REFLIB)


def ref():
    global _r
    if _r is None:
        L = C.CDLL(REFLIB)
        L.ref_matvec.restype = C.c_int
        L.ref_matvec.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_void_p]
        L.ref_pack_geom.restype = C.c_void_p
        L.ref_pack_geom.argtypes = [C.c_int] * 6 + [C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.POINTER(C.c_size_t)]
        L.ref_free.argtypes = [C.c_void_p]
        L.ref_iq4_nl.restype = C.POINTER(C.c_int8)
        L.ref_parse.restype = C.c_int
        L.ref_parse.argtypes = [C.c_void_p, C.c_size_t] + [C.c_void_p] * 4
        _r = L
    return _r


# ------------------------------------------------------------------ helpers

IQ4_NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
                  dtype=np.int8)  # the codebook of ref/matvec_int4.c:544-545 (spec 6.1 default)


def pack(M, K, rows_if, axi_dw, w_exp, out_shift, cb, idx, scl):
    """Restated packer -> bytes of a .mv4i image."""
    n = orc().orc_pack_size(M, K, rows_if, axi_dw)
    if n == 0:
        raise ValueError("unrepresentable geometry")
    img = np.zeros(n, np.uint8)
    cb = np.ascontiguousarray(cb, np.int8)
    idx = np.ascontiguousarray(idx, np.uint8)
    scl = np.ascontiguousarray(scl, np.uint16)
    rc = orc().orc_pack(M, K, rows_if, axi_dw, w_exp, out_shift, _p(cb), _p(idx), _p(scl), _p(img))
    assert rc == 0
    return img.tobytes()


def ref_pack(M, K, rows_if, axi_dw, w_exp, out_shift, cb, idx, scl):
    """The reference's own pack_geom -> bytes."""
    cb = np.ascontiguousarray(cb, np.int8)
    idx = np.ascontiguousarray(idx, np.uint8)
    scl = np.ascontiguousarray(scl, np.uint16)
    n = C.c_size_t(0)
    p = ref().ref_pack_geom(M, K, rows_if, axi_dw, w_exp, out_shift, _p(cb), _p(idx), _p(scl),
                            C.byref(n))
    out = C.string_at(p, n.value)
    ref().ref_free(p)
    return out


def _mv(fn, img, x, x_exp, n_rows, n_cols, mode):
    buf = np.frombuffer(img, np.uint8).copy()
    x = np.ascontiguousarray(x, np.int16)
    yd = np.zeros(max(n_rows, 1), np.int32)
    ya = np.zeros(max(n_rows, 1), np.int64)
    ym = np.zeros(max(n_rows, 1), np.int16)
    ye, se, ns = C.c_int(0), C.c_int(0), C.c_int(0)
    sc = C.c_uint64(0)
    rc = fn(_p(buf), buf.size, _p(x), x_exp, n_rows, n_cols, mode, _p(yd), _p(ya), _p(ym),
            C.byref(ye), C.byref(se), C.byref(sc), C.byref(ns))
    return rc, dict(y_data=yd[:n_rows], y_acc=ya[:n_rows], y_mant=ym[:n_rows], y_exp=ye.value,
                    sat_event=se.value, sat_count=sc.value, ns=ns.value)


def matvec(img, x, x_exp, n_rows, n_cols, mode):
    """Restated mv4i_matvec."""
    return _mv(orc().orc_matvec, img, x, x_exp, n_rows, n_cols, mode)


def ref_matvec(img, x, x_exp, n_rows, n_cols, mode):
    """The reference's mv4i_matvec (compiled from its source)."""
    return _mv(ref().ref_matvec, img, x, x_exp, n_rows, n_cols, mode)


def bfp_pack_f64(v):
    v = np.ascontiguousarray(v, np.float64)
    m = np.zeros(v.size, np.int16)
    e = orc().orc_bfp_pack_f64(_p(v), v.size, _p(m))
    return m, e


def matvec_g128_f64(wq, scales, x, K, G=128):
    """BASELINE config 0 in double (exact dequantisation)."""
    wq = np.ascontiguousarray(wq, np.uint8)
    s = np.ascontiguousarray(scales).view(np.uint16)
    x = np.ascontiguousarray(x).view(np.uint16)
    M = wq.shape[0]
    y = np.zeros(M, np.float64)
    orc().orc_matvec_g128_f64(M, K, G, _p(wq), wq.shape[1], _p(s), s.shape[1], _p(x), _p(y))
    return y


def tp_reduce(parts, y_exps, out_shifts):
    parts = [np.ascontiguousarray(p, np.int64) for p in parts]
    N, n = len(parts), parts[0].size
    arr = (C.c_void_p * N)(*[p.ctypes.data for p in parts])
    ye = np.ascontiguousarray(y_exps, np.int32)
    os_ = np.ascontiguousarray(out_shifts, np.int32)
    out = np.zeros(n, np.int16)
    y32 = np.zeros(n, np.int32)
    oe, sat = C.c_int(0), C.c_int(0)
    rc = orc().orc_tp_reduce(N, n, arr, _p(ye), _p(os_), _p(out), C.byref(oe), _p(y32),
                             C.byref(sat))
    return rc, out, oe.value, y32, sat.value


# ------------------------------------------------------------ DeltaNet (B)

def _gdn_sig():
    L = orc()
    if getattr(L, "_gdn_bound", False):
        return L
    i32p = C.POINTER(C.c_int)
    sig = {
        "orc_fx_init": (None, []),
        "orc_fx_tables": (None, [C.c_void_p, C.c_void_p, C.c_void_p]),
        "orc_gdn_scalar": (None, [C.c_int32, C.c_int, C.c_int32, C.c_int, C.c_int32, C.c_int,
                                  C.c_int32, C.c_int, i32p, i32p, i32p]),
        "orc_gdn_col_fixed": (C.c_int, [C.c_int, C.c_void_p, i32p, C.c_void_p, C.c_void_p, C.c_int32,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, i32p]),
        "orc_gdn_step_fixed": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                         C.c_int, C.c_void_p, C.c_void_p]),
        "orc_gdn_head_emit": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
        "orc_gdn_cfg1_f64": (None, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_double, C.c_void_p]),
        "orc_gdn_cfg1_f32": (None, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_float, C.c_void_p, C.c_int]),
    }
    for n, (res, args) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = res, args
    L._gdn_bound = True
    return L


def gdn_scalar(al_m, al_e, dt_m, dt_e, a_m, a_e, b_m, b_e):
    L = _gdn_sig()
    eg, be, err = C.c_int(0), C.c_int(0), C.c_int(0)
    L.orc_gdn_scalar(al_m, al_e, dt_m, dt_e, a_m, a_e, b_m, b_e, C.byref(eg), C.byref(be), C.byref(err))
    return eg.value, be.value, err.value


def gdn_col_fixed(smant, se_j, kn, qs, v, e_v, eg, beta, tk0):
    """One column of the fixed recurrence; returns (snew, se_new, o_acc, e_o, err)."""
    L = _gdn_sig()
    s = np.ascontiguousarray(smant, np.int16).copy()
    kn = np.ascontiguousarray(kn, np.int16)
    qs = np.ascontiguousarray(qs, np.int16)
    se = C.c_int(int(se_j))
    oacc = np.zeros(1, np.int64)
    eo = C.c_int(0)
    err = L.orc_gdn_col_fixed(s.size, _p(s), C.byref(se), _p(kn), _p(qs), int(v), int(e_v), int(eg),
                              int(beta), int(tk0), _p(oacc), C.byref(eo))
    return s, se.value, int(oacc[0]), eo.value, err


def gdn_step_fixed(smem, se, kn, qs, v, e_v, eg, beta, tk0):
    """All heads; smem [H][D][D] int16 and se [H][D] int32 are updated in place."""
    L = _gdn_sig()
    H, D = smem.shape[0], smem.shape[2]
    KH = kn.shape[0]
    o = np.zeros((H, D), np.int64)
    eo = np.zeros((H, D), np.int32)
    eg = np.ascontiguousarray(eg, np.int32)
    beta = np.ascontiguousarray(beta, np.int32)
    v = np.ascontiguousarray(v, np.int32)
    err = L.orc_gdn_step_fixed(H, KH, D, _p(smem), _p(se), _p(np.ascontiguousarray(kn, np.int16)),
                               _p(np.ascontiguousarray(qs, np.int16)), _p(v), int(e_v), _p(eg), _p(beta),
                               int(tk0), _p(o), _p(eo))
    return o, eo, err


def gdn_head_emit(o_acc, e_o):
    L = _gdn_sig()
    o_acc = np.ascontiguousarray(o_acc, np.int64)
    e_o = np.ascontiguousarray(e_o, np.int32)
    out = np.zeros(o_acc.size, np.int16)
    e = L.orc_gdn_head_emit(o_acc.size, _p(o_acc), _p(e_o), _p(out))
    return out, e


def gdn_cfg1_f64(S, q, k, v, a, b, g, l2=True, q_scale=1.0):
    """Config-1 steps in double.  S [H][D][D] (float64, updated in place);
    q, k, v, g [T][H][D]; a, b [T][H].  Returns out [T][H][D]."""
    L = _gdn_sig()
    T, H, D = q.shape
    arrs = [np.ascontiguousarray(x, np.float64) for x in (q, k, v, a, b, g)]
    out = np.zeros((T, H, D), np.float64)
    L.orc_gdn_cfg1_f64(T, H, D, _p(S), *[_p(x) for x in arrs], int(l2), float(q_scale), _p(out))
    return out


def gdn_cfg1_f32(S, q, k, v, a, b, g, l2=True, q_scale=1.0, threads=1):
    L = _gdn_sig()
    T, H, D = q.shape
    arrs = [np.ascontiguousarray(x, np.float32) for x in (q, k, v, a, b, g)]
    out = np.zeros((T, H, D), np.float32)
    L.orc_gdn_cfg1_f32(T, H, D, _p(S), *[_p(x) for x in arrs], int(l2), float(q_scale), _p(out), int(threads))
    return out


def have_gdn_ref():
    return os.path.exists(os.path.join(HERE, "_ref", "libref_gdn.so"))


def ref_gdn():
    L = C.CDLL(os.path.join(HERE, "_ref", "libref_gdn.so"))
    i32p = C.POINTER(C.c_int)
    L.ref_gdn_scalar.argtypes = [C.c_int32, C.c_int, C.c_int32, C.c_int, C.c_int32, C.c_int,
                                 C.c_int32, C.c_int, i32p, i32p, i32p]
    L.ref_fx_tables.argtypes = [C.c_void_p] * 3
    return L


def a_job(img, x, x_exp, K, row0, n):
    """ref/run9b.c:455-490 restated: (y_mant[n], y_exp)."""
    L = orc()
    if not getattr(L, "_ajob", False):
        L.orc_a_job.restype = C.c_int
        L.orc_a_job.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_void_p, C.POINTER(C.c_int)]
        L._ajob = True
    buf = np.frombuffer(img, np.uint8).copy()
    x = np.ascontiguousarray(x, np.int16)
    y = np.zeros(n, np.int16)
    e = C.c_int(0)
    rc = L.orc_a_job(_p(buf), buf.size, _p(x), x_exp, K, row0, n, _p(y), C.byref(e))
    assert rc == 0, rc
    return y, e.value


def argmax_first(v):
    """ref/run9b.c:399-405: the first maximum wins."""
    v = np.asarray(v)
    return int(np.flatnonzero(v == v.max())[0])


# ---------------------------------------------- DeltaNet block (fixed point)

class Blk(C.Structure):
    """Field for field the caller-owned block record of ref/gdn_block_vec.c:183-202
    (also oracle/gdn_block_oracle.c's orc_blk and the library's gdn_blk_t)."""
    _fields_ = [("xtap", C.c_void_p), ("wtap", C.c_void_p), ("e_t", C.c_void_p),
                ("tvalid", C.c_void_p), ("cw_exp", C.c_void_p), ("sc", C.c_void_p),
                ("zm", C.c_void_p), ("wm", C.c_void_p), ("w_e", C.c_int), ("z_e", C.c_int),
                ("tk0", C.c_int), ("smem", C.c_void_p), ("semem", C.c_void_p), ("y", C.c_void_p),
                ("y_exp", C.c_int), ("err_conv", C.c_int), ("err_g", C.c_int), ("err_se", C.c_int),
                ("y_sat", C.c_int)]


def _blk_sig():
    L = _gdn_sig()
    if getattr(L, "_blk_bound", False):
        return L
    sig = {
        "orc_rsqrt_rom": (None, [C.c_void_p]),
        "orc_to_q12": (C.c_int32, [C.c_int64, C.c_int]),
        "orc_sigma_q15": (C.c_int32, [C.c_int32]),
        "orc_silu": (C.c_int32, [C.c_int32, C.c_int]),
        "orc_conv_seg": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "orc_l2norm_rs": (None, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
        "orc_rmsnorm_bf": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_double,
                                     C.c_void_p, C.POINTER(C.c_int)]),
        "orc_y_emit": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.POINTER(C.c_int)]),
        "orc_emit_chain": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
        "orc_gdn_block_token": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(Blk)]),
    }
    for n, (res, args) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = res, args
    L._blk_bound = True
    return L


def _ref_blk():
    R = ref_gdn()
    if not getattr(R, "_blk_bound", False):
        R.ref_gdn_block_token.restype = None
        R.ref_gdn_block_token.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(Blk)]
        R.ref_l2norm_rs.restype = None
        R.ref_rsqrt_rom.argtypes = [C.c_void_p]
        R.ref_l2norm_rs.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        R.ref_rmsnorm_bf.restype = C.c_int
        R.ref_rmsnorm_bf.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                     C.POINTER(C.c_int)]
        R.ref_silu.restype = C.c_int
        R.ref_silu.argtypes = [C.c_int, C.c_int]
        R._blk_bound = True
    return R


def conv_seg(x, w, e_t, tv, cw_exp):
    """x, w [nch][4] int16 -> (sm[nch] int16, e_seg, sh_seg, err)."""
    L = _blk_sig()
    x = np.ascontiguousarray(x, np.int16)
    w = np.ascontiguousarray(w, np.int16)
    sm = np.zeros(x.shape[0], np.int16)
    es, ss = C.c_int(0), C.c_int(0)
    err = L.orc_conv_seg(x.shape[0], _p(x), _p(w), _p(np.ascontiguousarray(e_t, np.int32)),
                         _p(np.ascontiguousarray(tv, np.int32)), int(cw_exp), _p(sm), C.byref(es),
                         C.byref(ss))
    return sm, es.value, ss.value, err


def l2norm_rs(x, log2n, use_ref=False):
    x = np.ascontiguousarray(x, np.int32)
    k = np.zeros(x.size, np.int32)
    q = np.zeros(x.size, np.int32)
    (_ref_blk().ref_l2norm_rs if use_ref else _blk_sig().orc_l2norm_rs)(_p(x), x.size, log2n, _p(k), _p(q))
    return k, q


def rmsnorm_bf(xm, xe, wm, we, use_ref=False):
    xm = np.ascontiguousarray(xm, np.int16)
    wm = np.ascontiguousarray(wm, np.int16)
    o = np.zeros(xm.size, np.int16)
    oe = C.c_int(0)
    if use_ref:
        _ref_blk().ref_rmsnorm_bf(_p(xm), int(xe), _p(wm), int(we), xm.size, _p(o), C.byref(oe))
    else:
        _blk_sig().orc_rmsnorm_bf(_p(xm), int(xe), _p(wm), int(we), xm.size, 1.0e-6, _p(o), C.byref(oe))
    return o, oe.value


def y_emit(ep, po, pz):
    """ep [H]; po, pz [H][D] int16 -> (y [H*D], y_exp, sat)."""
    L = _blk_sig()
    po = np.ascontiguousarray(po, np.int16)
    pz = np.ascontiguousarray(pz, np.int16)
    H, D = po.shape
    y = np.zeros(H * D, np.int16)
    ye = C.c_int(0)
    sat = L.orc_y_emit(H, D, _p(np.ascontiguousarray(ep, np.int32)), _p(po), _p(pz), _p(y), C.byref(ye))
    return y, ye.value, sat


def emit_chain(o_acc, e_o, zm, wm, we, z_e):
    """o_acc int64 / e_o / zm [H][D] -> (y [H*D], y_exp, sat)."""
    L = _blk_sig()
    o_acc = np.ascontiguousarray(o_acc, np.int64)
    H, D = o_acc.shape
    y = np.zeros(H * D, np.int16)
    ye = C.c_int(0)
    sat = L.orc_emit_chain(H, D, _p(o_acc), _p(np.ascontiguousarray(e_o, np.int32)),
                           _p(np.ascontiguousarray(zm, np.int16)), _p(np.ascontiguousarray(wm, np.int16)),
                           int(we), int(z_e), _p(y), C.byref(ye))
    return y, ye.value, sat


def blk_taps(t, caps):
    """Tap exponents and validity of token t (ref/gdn_block_vec.c:657-669):
    tap 3 is the current token, tap k refers to token t-(3-k); a tap before
    the sequence start is invalid and carries the exponent -47.
    caps [T][3] are the per-token captured segment exponents."""
    n = min(t + 1, 4)
    e_t = np.zeros((3, 4), np.int32)
    tv = np.zeros((3, 4), np.int32)
    for s in range(3):
        for k in range(4):
            src = t - (3 - k)
            ok = k >= 4 - n
            tv[s, k] = ok
            e_t[s, k] = caps[src][s] if ok else -47
    return e_t, tv


def gdn_block_run(KH, VH, D, stim, smem, semem, use_ref=False):
    """Run len(stim['xtap']) tokens through the oracle (or the reference's own
    gdn_block_token).  smem [VH][D][D] int16 and semem [VH][D] int32 are
    updated in place.  Returns y [T][VH*D], y_exp [T], flags [T][4]."""
    fn = _ref_blk().ref_gdn_block_token if use_ref else _blk_sig().orc_gdn_block_token
    T = stim["xtap"].shape[0]
    ys = np.zeros((T, VH * D), np.int16)
    yexp = np.zeros(T, np.int32)
    flags = np.zeros((T, 4), np.int32)
    wtap = np.ascontiguousarray(stim["wtap"], np.int16)
    cw = np.ascontiguousarray(stim["cw_exp"], np.int32)
    wm = np.ascontiguousarray(stim["wm"], np.int16)
    assert smem.dtype == np.int16 and semem.dtype == np.int32
    assert smem.flags.c_contiguous and semem.flags.c_contiguous
    for t in range(T):
        keep = [np.ascontiguousarray(stim[k][t], dt) for k, dt in
                (("xtap", np.int16), ("e_t", np.int32), ("tvalid", np.int32), ("sc", np.int32),
                 ("zm", np.int16))]
        b = Blk()
        b.xtap, b.wtap, b.e_t, b.tvalid = keep[0].ctypes.data, wtap.ctypes.data, keep[1].ctypes.data, \
            keep[2].ctypes.data
        b.cw_exp, b.sc, b.zm, b.wm = cw.ctypes.data, keep[3].ctypes.data, keep[4].ctypes.data, wm.ctypes.data
        b.w_e, b.z_e, b.tk0 = int(stim["w_e"]), int(stim["z_e"]), int(stim["tk0"][t])
        b.smem, b.semem, b.y = smem.ctypes.data, semem.ctypes.data, ys[t].ctypes.data
        rc = fn(KH, VH, D, C.byref(b))
        assert rc in (None, 0), rc
        yexp[t] = b.y_exp
        flags[t] = (b.err_conv, b.err_g, b.err_se, b.y_sat)
    return ys, yexp, flags


def gdn_block_stimulus(KH, VH, D, T, seed):
    """Seeded block stimulus in the reference generator's ranges
    (ref/gdn_block_vec.c:570-618): conv weights and history in +-2047, segment
    exponents 11..13, capture exponents 8..12, norm weights 2000..6000 on 12,
    the scalar-path inputs in the physical band, z in +-8192 on 12, masked taps
    filled with garbage.  Returns (stim, smem, semem)."""
    rng = np.random.default_rng(seed)
    CH = 2 * KH * D + VH * D
    hist = rng.integers(-2047, 2048, (T, CH), dtype=np.int64).astype(np.int16)
    caps = [[8 + (t + s) % 5 for s in range(3)] for t in range(T)]
    stim = dict(wtap=rng.integers(-2047, 2048, (CH, 4)).astype(np.int16),
                cw_exp=np.array([11, 12, 13], np.int32),
                wm=rng.integers(2000, 6001, D).astype(np.int16), w_e=12, z_e=12,
                tk0=np.array([1] + [0] * (T - 1), np.int32))
    xt = np.zeros((T, CH, 4), np.int16)
    et = np.zeros((T, 3, 4), np.int32)
    tv = np.zeros((T, 3, 4), np.int32)
    for t in range(T):
        et[t], tv[t] = blk_taps(t, caps)
        for k in range(4):
            src = t - (3 - k)
            if src >= 0:
                xt[t, :, k] = hist[src]
            else:
                xt[t, :, k] = (-30000 + ((np.arange(CH) * 7 + k * 13) % 60000)).astype(np.int16)
    sc = np.zeros((T, VH, 8), np.int32)
    sc[:, :, 0] = rng.integers(-1000, 1001, (T, VH)); sc[:, :, 1] = 14
    sc[:, :, 2] = -rng.integers(2000, 32001, (T, VH)); sc[:, :, 3] = 12
    sc[:, :, 4] = -rng.integers(1, 3001, (T, VH)); sc[:, :, 5] = 16
    sc[:, :, 6] = rng.integers(-30000, 30001, (T, VH)); sc[:, :, 7] = 12
    stim.update(xtap=xt, e_t=et, tvalid=tv, sc=sc,
                zm=rng.integers(-8192, 8193, (T, VH, D)).astype(np.int16))
    smem = np.zeros((VH, D, D), np.int16)
    semem = np.zeros((VH, D), np.int32)
    for h in range(VH):
        for j in range(D):
            top = int(rng.integers(16384, 32768))
            smem[h, j] = rng.integers(-top, top + 1, D)
            smem[h, j, rng.integers(0, D)] = top
            semem[h, j] = 9 + (h + j) % 4
    return stim, smem, semem
