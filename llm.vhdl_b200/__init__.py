"""Python view of the llm.vhdl B200 hot-path library (ctypes over the C ABI).

The product is the C ABI in include/mv4i_b200.h, implemented by
lib/libmv4i_b200.so (CUDA sm_100a + C host code).  This module only binds it
for the tests and bench.py; it has no compute of its own and no fallback:
``lib()`` raises if the shared library is missing.

Because the directory name contains a dot it is loaded by path:
``load_package()`` in tests/conftest.py and bench.py registers it as the
module ``llmvhdl_b200``.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIBDIR = os.path.join(HERE, "lib")
LIBPATH = os.path.join(LIBDIR, "libmv4i_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["csrc/mv4i_kernels.cu", "csrc/gdn_kernels.cu", "csrc/mv4i_host.c", "csrc/mv4i_pack.c"]   # gdn_kernels.cu includes gdn_block.cuh
DEC_LIBPATH = os.path.join(LIBDIR, "libdec_b200.so")
DEC_SOURCES = ["csrc/dec_step.cu", "csrc/dec_model.c"]   # dec_step.cu includes dec_kernels.cu, dec_matvec.cu

MODE_BFP, MODE_RAW, MODE_PARTIAL = 0, 1, 2
KIND_GOLDEN, KIND_G128 = 0, 1
MAX_JOBS = 64


def build(verbose=False):
    """Compile the CUDA + C sources for sm_100a: lib/libmv4i_b200.so (matvec,
    DeltaNet, drop-in host API) and lib/libdec_b200.so (the decode step,
    linked against the first and NCCL)."""
    os.makedirs(LIBDIR, exist_ok=True)
    cmds = [
        [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
         "-shared", "-o", LIBPATH, *[os.path.join(HERE, s) for s in SOURCES], "-lpthread", "-lnccl"],
        [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
         "-shared", "-o", DEC_LIBPATH, *[os.path.join(HERE, s) for s in DEC_SOURCES],
         "-L" + LIBDIR, "-lmv4i_b200", "-lnccl", "-Xlinker", "-rpath=$ORIGIN"],
    ]
    for cmd in cmds:
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
        if verbose:
            print(r.stdout + r.stderr)
    return LIBPATH


# ----------------------------------------------------------------- structs

class Hdr(C.Structure):
    _fields_ = [("magic", C.c_uint32), ("M", C.c_uint32), ("K", C.c_uint32),
                ("scale_offset", C.c_uint32), ("n_scale_sub", C.c_uint32),
                ("version", C.c_uint16), ("flags", C.c_uint16), ("rows_if", C.c_uint16),
                ("nports_w", C.c_uint16), ("block", C.c_uint16), ("axi_dw", C.c_uint16),
                ("w_exp", C.c_int32), ("out_shift", C.c_int32), ("codebook", C.c_int8 * 16),
                ("w_sub_offset", C.c_uint64 * 64), ("s_sub_offset", C.c_uint64 * 64)]


class File(C.Structure):
    _fields_ = [("h", Hdr), ("base", C.c_void_p), ("nb", C.c_int), ("port_b", C.c_int),
                ("grp", C.c_int)]


class Result(C.Structure):
    _fields_ = [("y_data", C.c_void_p), ("y_acc", C.c_void_p), ("y_mant", C.c_void_p),
                ("y_exp", C.c_int), ("sat_event", C.c_int), ("sat_count", C.c_uint64),
                ("ns", C.c_int)]


class DMat(C.Structure):
    _fields_ = [("wq", C.c_void_p), ("sc", C.c_void_p), ("w_pitch", C.c_int64),
                ("s_pitch", C.c_int64), ("M", C.c_int32), ("K", C.c_int32),
                ("w_exp", C.c_int32), ("out_shift", C.c_int32), ("codebook", C.c_int8 * 16),
                ("kind", C.c_int32), ("device", C.c_int32), ("owned", C.c_void_p)]


class Status(C.Structure):
    _fields_ = [("y_exp", C.c_int32), ("ns", C.c_int32), ("sat_event", C.c_int32),
                ("sat_count", C.c_uint32), ("err", C.c_int32), ("pad", C.c_int32 * 3)]


class GdnFixed(C.Structure):
    _fields_ = [("H", C.c_int32), ("KH", C.c_int32), ("D", C.c_int32), ("smem", C.c_void_p),
                ("semem", C.c_void_p), ("kn", C.c_void_p), ("qs", C.c_void_p), ("v", C.c_void_p),
                ("e_v", C.c_int32), ("eg", C.c_void_p), ("beta", C.c_void_p), ("tk0", C.c_int32),
                ("o_acc", C.c_void_p), ("e_o", C.c_void_p), ("o_head", C.c_void_p),
                ("e_head", C.c_void_p), ("err", C.c_void_p)]


class GdnF32(C.Structure):
    _fields_ = [("T", C.c_int32), ("H", C.c_int32), ("KH", C.c_int32), ("D", C.c_int32),
                ("S", C.c_void_p), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
                ("g", C.c_void_p), ("a", C.c_void_p), ("b", C.c_void_p), ("l2norm", C.c_int32),
                ("q_scale", C.c_float), ("out_f32", C.c_void_p), ("out_f16", C.c_void_p),
                ("eg", C.c_void_p), ("beta", C.c_void_p), ("pdl", C.c_int32), ("nseq", C.c_int32),
                ("seq_in", C.c_int32), ("pad_", C.c_int32)]


class DeltanetArgs(C.Structure):
    """deltanet_args of include/gdn_b200.h (device buffers)."""
    _fields_ = [("KH", C.c_int32), ("VH", C.c_int32), ("D", C.c_int32), ("xtap", C.c_void_p),
                ("wtap", C.c_void_p), ("e_t", (C.c_int32 * 4) * 3), ("tvalid", (C.c_int32 * 4) * 3),
                ("cw_exp", C.c_int32 * 3), ("sc", C.c_void_p), ("zm", C.c_void_p), ("wm", C.c_void_p),
                ("w_e", C.c_int32), ("z_e", C.c_int32), ("tk0", C.c_int32), ("smem", C.c_void_p),
                ("semem", C.c_void_p), ("y", C.c_void_p), ("status", C.c_void_p), ("work", C.c_void_p),
                ("pdl", C.c_int32)]


class Job(C.Structure):
    _fields_ = [("w", C.POINTER(DMat)), ("x", C.c_void_p), ("d_x_exp", C.c_void_p),
                ("x_exp", C.c_int32), ("n_rows", C.c_int32), ("n_cols", C.c_int32),
                ("mode", C.c_int32), ("nvec", C.c_int32), ("x_stride", C.c_int64),
                ("y_stride", C.c_int64), ("y_data", C.c_void_p), ("y_mant", C.c_void_p),
                ("y_acc", C.c_void_p), ("y_f16", C.c_void_p), ("y_f32", C.c_void_p),
                ("status", C.c_void_p), ("accum", C.c_int32), ("pad_", C.c_int32)]


EXPORTS = {
    "mv4i_parse": (C.c_int, [C.POINTER(File), C.c_void_p, C.c_size_t]),
    "mv4i_matvec": (C.c_int, [C.POINTER(File), C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                              C.POINTER(Result)]),
    "mv4i_forget": (C.c_int, [C.POINTER(File)]),
    "mv4i_get_widx": (C.c_int, [C.POINTER(File), C.c_int, C.c_int]),
    "mv4i_get_scale": (C.c_uint16, [C.POINTER(File), C.c_int, C.c_int]),
    "mv4i_dmat_upload": (C.c_int, [C.POINTER(File), C.c_int, C.POINTER(DMat)]),
    "mv4i_dmat_wrap_g128": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int,
                                      C.c_int, C.c_int, C.POINTER(DMat)]),
    "mv4i_dmat_wrap_golden": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                        C.POINTER(DMat)]),
    "mv4i_dmat_free": (C.c_int, [C.POINTER(DMat)]),
    "mv4i_dmat_rows": (C.c_int, [C.POINTER(DMat), C.c_int, C.c_int, C.POINTER(DMat)]),
    "mv4i_argmax": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mv4i_bfp_pack": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int64, C.c_void_p,
                                C.c_void_p, C.c_void_p]),
    "mv4i_scratch_bytes": (C.c_size_t, []),
    "mv4i_launch": (C.c_int, [C.POINTER(Job), C.c_int, C.c_void_p, C.c_void_p]),
    "mv4i_launch_noalloc": (C.c_int, [C.POINTER(Job), C.c_int, C.c_void_p]),
    "mv4i_tp_reduce": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mv4i_synth_g128": (C.c_int, [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_void_p]),
    "mv4i_g128_matvec_host": (C.c_int, [C.POINTER(DMat), C.c_int, C.c_void_p, C.c_void_p,
                                        C.c_void_p]),
    "gdn_scalar_dev": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "gdn_step_fixed": (C.c_int, [C.POINTER(GdnFixed), C.c_void_p]),
    "gdn_run_f32": (C.c_int, [C.POINTER(GdnF32), C.c_void_p]),
    "deltanet_work_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "deltanet_step": (C.c_int, [C.POINTER(DeltanetArgs), C.c_void_p]),
    "gdn_block_token_host": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "gdn_conv_seg_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_void_p]),
    "gdn_silu_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "gdn_l2norm_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "gdn_rmsnorm_bf_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p]),
    "gdn_y_emit_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p]),
    "gdn_emit_chain_dev": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mv4i_quantize": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.POINTER(C.c_int)]),
    "mv4i_calibrate_out_shift": (C.c_int, [C.c_int]),
    "mv4i_pack_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "mv4i_pack": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                            C.c_int, C.c_void_p]),
    "mv4i_image_to_g128": (C.c_int, [C.POINTER(File), C.c_void_p, C.c_void_p, C.c_int]),
    "mv4i_quantize_g128": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int]),
    "mv4i_tp_msg_bytes": (C.c_size_t, [C.c_int]),
    "mv4i_tp_msg_pack": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_void_p]),
    "mv4i_tp_msgs_check": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p]),
    "mv4i_tp_msg_pack_dev": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_uint32, C.c_void_p,
                                       C.c_void_p]),
    "mv4i_tp_reduce_msgs": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p]),
    "mv4i_tp_unique_id": (C.c_int, [C.c_void_p]),
    "mv4i_tp_comm_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "mv4i_tp_comm_destroy": (C.c_int, [C.c_void_p]),
    "mv4i_tp_row_parallel": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_uint32, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mv4i_tp_allreduce_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "mv4i_last_cuda_error": (C.c_int, []),
    "mv4i_version": (C.c_char_p, []),
}

_lib = None


def lib():
    """The loaded C-ABI library.  Raises when it has not been built: there is
    no other implementation to fall back to."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBPATH):
            raise RuntimeError("libmv4i_b200.so is not built (run __graft_entry__.build())")
        L = C.CDLL(LIBPATH)
        for name, (res, args) in EXPORTS.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


class DecConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("n_layers", C.c_int32), ("attn_every", C.c_int32),
                ("vocab", C.c_int32), ("ffn", C.c_int32), ("gdn_kh", C.c_int32),
                ("gdn_vh", C.c_int32), ("gdn_hd", C.c_int32), ("att_qh", C.c_int32),
                ("att_kvh", C.c_int32), ("att_hd", C.c_int32), ("n_rot", C.c_int32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("max_ctx", C.c_int32),
                ("batch", C.c_int32)]


class GatedAttnArgs(C.Structure):
    """gated_attn_args of include/dec_b200.h (device buffers)."""
    _fields_ = [("n_qh", C.c_int32), ("n_kvh", C.c_int32), ("head_dim", C.c_int32), ("n_rot", C.c_int32),
                ("rope_theta", C.c_float), ("eps", C.c_float), ("qg", C.c_void_p), ("kv", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("d_pos", C.c_void_p), ("max_ctx", C.c_int32),
                ("kcache", C.c_void_p), ("vcache", C.c_void_p), ("y", C.c_void_p), ("q_out", C.c_void_p),
                ("work", C.c_void_p), ("pdl", C.c_int32)]


DEC_EXPORTS = {
    "gated_attn_work_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "gated_attn": (C.c_int, [C.POINTER(GatedAttnArgs), C.c_void_p]),
    "dec_load_linear": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                  C.c_int]),
    "dec_create": (C.c_int, [C.POINTER(DecConfig), C.c_uint64, C.c_int, C.c_int, C.c_int,
                             C.POINTER(C.c_void_p)]),
    "dec_destroy": (C.c_int, [C.c_void_p]),
    "dec_nccl_unique_id": (C.c_int, [C.c_void_p]),
    "dec_tp_init": (C.c_int, [C.c_void_p, C.c_void_p]),
    "dec_p2p_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "dec_p2p_open": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "dec_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "dec_prefill_random": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64]),
    "dec_set": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "dec_set_prompt": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "dec_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "dec_pointers": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                               C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                               C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "dec_linear": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_void_p),
                             C.POINTER(C.c_void_p), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                             C.POINTER(C.c_int32)]),
    "dec_param": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_void_p),
                            C.POINTER(C.c_int32)]),
    "dec_step_bytes": (C.c_int64, [C.c_void_p]),
    "dec_layer_bytes": (C.c_int64, [C.c_void_p, C.c_int]),
    "dec_set_layer_events": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "dec_set_residual_seams": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "dec_set_persistent": (C.c_int, [C.c_void_p, C.c_int]),
    "dec_set_prestage": (C.c_int, [C.c_void_p, C.c_int]),
    "dec_persistent": (C.c_int, [C.c_void_p]),
    "dec_set_clock": (C.c_int, [C.c_void_p, C.c_void_p]),
    "dec_set_wait_limit": (C.c_int, [C.c_void_p, C.c_int64]),
    "dec_clock_slots": (C.c_int, [C.c_void_p]),
    "dec_layer_clock": (C.c_int, [C.c_void_p, C.c_int]),
}

_declib = None


def declib():
    """The decode-step library (include/dec_b200.h).  Raises when it has not
    been built."""
    global _declib
    if _declib is None:
        lib()
        if not os.path.exists(DEC_LIBPATH):
            raise RuntimeError("libdec_b200.so is not built (run __graft_entry__.build())")
        L = C.CDLL(DEC_LIBPATH)
        for name, (res, args) in DEC_EXPORTS.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _declib = L
    return _declib


def header_symbols(path=None):
    """Function names declared in include/mv4i_b200.h (and other include/*.h)."""
    import glob
    import re
    names = set()
    paths = [path] if path else glob.glob(os.path.join(ROOT, "include", "*.h"))
    for p in paths:
        src = open(p).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b([a-z][a-z0-9_]*)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(n for n in names if not n.startswith("sizeof"))


# ------------------------------------------------------------ host drop-in

def ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class ParsedImage:
    """A parsed .mv4i image; keeps the bytes alive (the file borrows them)."""

    def __init__(self, img):
        self.buf = np.frombuffer(bytes(img), dtype=np.uint8).copy()
        self.f = File()
        self.rc = lib().mv4i_parse(C.byref(self.f), ptr(self.buf), self.buf.size)

    def forget(self):
        """Drop the library's cached device copy of this image."""
        if self.rc == 0 and _lib is not None:
            _lib.mv4i_forget(C.byref(self.f))

    def __del__(self):
        try:
            self.forget()
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass

    @property
    def M(self):
        return self.f.h.M

    @property
    def K(self):
        return self.f.h.K


def matvec(pi, x_mant, x_exp, n_rows, n_cols, mode):
    """mv4i_matvec through the drop-in C entry point (host buffers)."""
    x = np.ascontiguousarray(x_mant, dtype=np.int16)
    yd = np.zeros(max(n_rows, 1), np.int32)
    ya = np.zeros(max(n_rows, 1), np.int64)
    ym = np.zeros(max(n_rows, 1), np.int16)
    r = Result(yd.ctypes.data, ya.ctypes.data, ym.ctypes.data, 0, 0, 0, 0)
    rc = lib().mv4i_matvec(C.byref(pi.f), ptr(x), x_exp, n_rows, n_cols, mode, C.byref(r))
    return rc, dict(y_data=yd[:n_rows], y_acc=ya[:n_rows], y_mant=ym[:n_rows], y_exp=r.y_exp,
                    sat_event=r.sat_event, sat_count=r.sat_count, ns=r.ns)
