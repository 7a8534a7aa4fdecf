"""Generate tests/golden/mv4i_golden.npz from the llm.vhdl reference itself.

Run in a container that has the reference tree (default /root/reference, or
$LLMVHDL_REF) after `make -C oracle ref`.  Every expected value in the output
comes from the REFERENCE's own code compiled from its source:

* images      -- `matvec_int4 --emit OUT M K ROWS_IF AXI_DW` (the reference's
                 CLI, ref/matvec_int4.c:727-762: its own packer pack_geom with
                 the IQ4_NL codebook and its LCG-drawn indices / scales), plus
                 linear-codebook images from its pack_geom through the shim
* outputs     -- ref/matvec_int4.c mv4i_matvec in BFP, RAW and PARTIAL mode
* tile cases  -- sim/mv_tile_vec.txt (written by tools/mv_tile_model.py), parsed
                 into (codebook, indices, scales, x, out_shift, mode, expected)
* arithmetic  -- sim/arith_vectors.txt (written by tools/gen_arith.py)

The GPU box has no reference tree, so the GPU parity tests read this file.
Usage: python tests/golden/make_golden.py
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402

REF = os.environ.get("LLMVHDL_REF", "/root/reference")
OUT = os.path.join(HERE, "mv4i_golden.npz")


def arith_vectors():
    # site4 = sat16(round_shift(v, sh)), tools/gen_arith.py:261
    ops = {"floor_shr": 0, "round_shift": 1, "sat32": 2, "sat16": 3, "msb_pos": 4, "site4": 5}
    rows = []
    for ln in open(os.path.join(REF, "sim", "arith_vectors.txt")):
        f = ln.split()
        if not f or f[0].startswith("#"):
            continue
        if f[0] not in ops:
            raise ValueError("unknown op " + f[0])
        a = int(f[1], 16)
        e = int(f[3], 16)
        rows.append((ops[f[0]], a - (1 << 64) if a >= 1 << 63 else a, int(f[2]),
                     e - (1 << 64) if e >= 1 << 63 else e))
    return np.array(rows, dtype=np.int64)


def tile_cases():
    """sim/mv_tile_vec.txt -> list of dict.  Each B line packs 2 rows x 32
    nibbles (w256), 32 int16 x (x512) and two 16-bit scales (s32)."""
    cases, cur = [], None
    for ln in open(os.path.join(REF, "sim", "mv_tile_vec.txt")):
        f = ln.split()
        if not f or f[0].startswith("#") or f[0] == "DONE":
            continue
        if f[0] == "CASE":
            cur = dict(id=int(f[1]), out_shift=int(f[2]), mode=int(f[3]), nb=int(f[4]),
                       ntiles=int(f[5]), blocks={}, res={})
        elif f[0] == "CB":
            cur["cb"] = [int(v) for v in f[1:17]]
        elif f[0] == "B":
            cur["blocks"][(int(f[1]), int(f[2]))] = (int(f[3], 16), int(f[4], 16), int(f[5], 16))
        elif f[0] == "R":
            def s48(h):
                v = int(h, 16)
                return v - (1 << 48) if v >= 1 << 47 else v
            cur["res"][int(f[1])] = (s48(f[2]), s48(f[3]), int(f[4]))
        elif f[0] == "END":
            cases.append(cur)
    out = []
    for c in cases:
        nb, nt = c["nb"], c["ntiles"]
        for t in range(nt):
            idx = np.zeros((2, nb * 32), np.uint8)
            x = np.zeros(nb * 32, np.int16)
            scl = np.zeros((2, nb), np.uint16)
            for b in range(nb):
                w, xw, s = c["blocks"][(t, b)]
                for r in range(2):
                    for j in range(32):
                        idx[r, b * 32 + j] = (w >> (4 * (r * 32 + j))) & 15
                for j in range(32):
                    v = (xw >> (16 * j)) & 0xFFFF
                    x[b * 32 + j] = v - 65536 if v >= 32768 else v
                scl[0, b] = s & 0xFFFF
                scl[1, b] = s >> 16
            v0, v1, sat = c["res"][t]
            out.append(dict(case=c["id"], tile=t, out_shift=c["out_shift"], mode=c["mode"],
                            cb=np.array(c["cb"], np.int8), idx=idx, scl=scl, x=x,
                            expect=np.array([v0, v1], np.int64), sat=sat))
    return out


def emitted_image(M, K, RI, DW):
    binp = os.path.join(ROOT, "oracle", "_ref", "matvec_int4")
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "img.mv4i")
        subprocess.run([binp, "--emit", p, str(M), str(K), str(RI), str(DW)], check=True,
                       stdout=subprocess.DEVNULL)
        return open(p, "rb").read()


def main():
    if not O.have_ref():
        raise SystemExit("build the reference first: make -C oracle ref")
    d = {"arith": arith_vectors()}
    rng = np.random.default_rng(20261201)
    geoms = [(8, 96, 4, 128), (50, 200, 4, 128), (33, 77, 4, 256), (64, 1000, 8, 128),
             (16, 64, 4, 64), (40, 4096, 4, 128)]
    n = 0
    for g, (M, K, RI, DW) in enumerate(geoms):
        img = emitted_image(M, K, RI, DW)
        d["img%d" % g] = np.frombuffer(img, np.uint8)
        x = rng.integers(-20000, 20001, K).astype(np.int16)
        x_exp = int(rng.integers(-4, 12))
        for mode in (0, 1, 2):
            for (nr, nc) in ((M, K), (max(1, M - 3), max(1, K - 17))):
                rc, r = O.ref_matvec(img, x, x_exp, nr, nc, mode)
                assert rc == 0
                key = "emit%d" % n
                d[key + "_meta"] = np.array([M, K, RI, DW, x_exp, nr, nc, mode, r["y_exp"],
                                             r["sat_event"], r["sat_count"], r["ns"], g], np.int64)
                d[key + "_x"] = x
                d[key + "_y"] = (r["y_acc"] if mode == 2 else
                                 (r["y_mant"].astype(np.int64) if mode == 0 else r["y_data"].astype(np.int64)))
                if mode == 0:
                    d[key + "_ydata"] = r["y_data"]
                n += 1
    # linear codebook (the benchmark's signed INT4), packed by the reference packer
    from importlib import util
    spec = util.spec_from_file_location("synth", os.path.join(ROOT, "llm.vhdl_b200", "synth.py"))
    S = util.module_from_spec(spec)
    spec.loader.exec_module(S)
    M, K = 64, 512
    wq = S.g128_weights(0, M, K)
    sc = S.g128_scales(0, M, K)
    xf = S.g128_x(0, K)
    idx, scl, w_exp = S.g128_to_golden(wq, sc, K)
    xm, xe = O.bfp_pack_f64(xf.astype(np.float64))
    img = O.ref_pack(M, K, 4, 128, w_exp, 3, S.LINEAR_CB, idx, scl)
    for mode in (0, 1, 2):
        rc, r = O.ref_matvec(img, xm, xe, M, K, mode)
        assert rc == 0
        key = "lin%d" % mode
        d[key + "_img"] = np.frombuffer(img, np.uint8)
        d[key + "_meta"] = np.array([M, K, 4, 128, xe, M, K, mode, r["y_exp"], r["sat_event"],
                                     r["sat_count"], r["ns"]], np.int64)
        d[key + "_x"] = xm
        d[key + "_y"] = (r["y_acc"] if mode == 2 else
                         (r["y_mant"].astype(np.int64) if mode == 0 else r["y_data"].astype(np.int64)))
    # saturation: every weight at -127, every scale 32767, x = -32768, out_shift 0
    M, K = 8, 1024
    idx = np.zeros((M, K), np.uint8)
    scl = np.full((M, K // 32), 32767, np.uint16)
    img = O.ref_pack(M, K, 4, 128, 0, 0, O.IQ4_NL, idx, scl)
    x = np.full(K, -32768, np.int16)
    for mode in (0, 1, 2):
        rc, r = O.ref_matvec(img, x, 0, M, K, mode)
        assert rc == 0
        key = "sat%d" % mode
        d[key + "_img"] = np.frombuffer(img, np.uint8)
        d[key + "_meta"] = np.array([M, K, 4, 128, 0, M, K, mode, r["y_exp"], r["sat_event"],
                                     r["sat_count"], r["ns"]], np.int64)
        d[key + "_x"] = x
        d[key + "_y"] = (r["y_acc"] if mode == 2 else
                         (r["y_mant"].astype(np.int64) if mode == 0 else r["y_data"].astype(np.int64)))
    # tile vectors
    tiles = tile_cases()
    for i, t in enumerate(tiles):
        key = "tile%d" % i
        d[key + "_meta"] = np.array([t["case"], t["tile"], t["out_shift"], t["mode"], t["sat"]], np.int64)
        d[key + "_cb"] = t["cb"]
        d[key + "_idx"] = t["idx"]
        d[key + "_scl"] = t["scl"]
        d[key + "_x"] = t["x"]
        d[key + "_y"] = t["expect"]
    np.savez_compressed(OUT, **d)
    print("wrote", OUT, os.path.getsize(OUT), "bytes;", n, "emit cases,", len(tiles), "tile cases")


if __name__ == "__main__":
    main()
