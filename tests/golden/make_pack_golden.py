"""Generate tests/golden/pack_golden.npz from the llm.vhdl reference's own
offline packer, tools/pack_int4.py (imported from the reference tree:
$LLMVHDL_REF, default the directory `reference` beside this repository).

For seeded float32 matrices of several shapes and geometries it records the
reference's quantize() output (indices, uint15 scales, w_exp), its
calibrate_out_shift(K) and its pack() image bytes; tests/test_pack.py requires
the library's mv4i_quantize / mv4i_calibrate_out_shift / mv4i_pack to
reproduce every byte.  Usage: python tests/golden/make_pack_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402

sys.path.insert(0, os.path.join(O.REF_TREE, "tools"))
import pack_int4 as P  # noqa: E402

OUT = os.path.join(HERE, "pack_golden.npz")
# (M, K, rows_if, axi_dw, distribution)
CASES = [(48, 200, 4, 128, "normal"), (64, 1000, 4, 128, "heavy"), (33, 77, 4, 256, "normal"),
         (96, 512, 8, 128, "uniform"), (40, 4096, 4, 128, "normal"), (16, 64, 4, 64, "tiny"),
         (24, 256, 48, 256, "normal"), (8, 96, 1, 128, "zerorow")]


def matrix(M, K, dist, rng):
    if dist == "normal":
        W = rng.standard_normal((M, K)) * 0.02
    elif dist == "heavy":
        W = rng.standard_t(3, (M, K)) * 0.01
    elif dist == "uniform":
        W = rng.uniform(-1.0, 1.0, (M, K))
    elif dist == "tiny":
        W = rng.standard_normal((M, K)) * 1e-6
    else:
        W = rng.standard_normal((M, K)) * 0.05
        W[::3] = 0.0                                   # all-zero rows: scale 0, index 0
    return W.astype(np.float32)


def main():
    rng = np.random.default_rng(20261202)
    d = {}
    for i, (M, K, ri, dw, dist) in enumerate(CASES):
        W = matrix(M, K, dist, rng)
        idx, scl, w_exp = P.quantize(W, P.IQ4_NL)
        osh = P.calibrate_out_shift(K)
        img = P.pack(idx, scl, w_exp, M, K, ri, osh, P.IQ4_NL, axi_dw=dw)
        d["c%d_meta" % i] = np.array([M, K, ri, dw, w_exp, osh], np.int64)
        d["c%d_W" % i] = W
        d["c%d_idx" % i] = idx.astype(np.uint8)
        d["c%d_scl" % i] = scl.astype(np.uint16)
        d["c%d_img" % i] = np.frombuffer(img, np.uint8)
    d["cb"] = P.IQ4_NL.astype(np.int8)
    d["out_shift_K"] = np.array([[k, P.calibrate_out_shift(k)] for k in
                                 (1, 31, 32, 33, 64, 100, 1024, 2048, 4096, 5120, 17408, 65536, 1 << 22)],
                                np.int64)
    np.savez_compressed(OUT, **d)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
