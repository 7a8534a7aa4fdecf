"""Generate tests/golden/gdn_block_golden.npz from the llm.vhdl reference itself.

Run in a container that has the reference tree ($LLMVHDL_REF, default the
directory `reference` beside this repository) after `make -C oracle ref`.
Every expected value comes from the reference's own code or its committed
vector files:

* block    -- `gdn_block_vec OUT KH VH D TOKENS LAYERS mod SEED`
              (ref/gdn_block_vec.c:539-820, the whole fixed-point DeltaNet
              token: conv, silu, L2 norms, scalar path, recurrence, head emit,
              output rmsnorm, z gate, whole-token renorm) at the regression
              arguments "2 4 32 2 2 mod" (sim/regress.sh) and at the model
              shape KH 16 / VH 32 / D 128 over 3 tokens.  The final state of
              the large run is stored as a SHA-256 (it is 1 MiB of noise).
* units    -- the committed sim/ files: gdn_conv_vec.txt (conv + segment
              requantiser), gdn_silu_vec.txt, gdn_head_emit_vec.txt (site 12),
              gdn_y_emit_vec.txt (site 13), gdn_emit_chain_vec.txt (site 12 ->
              rmsnorm -> z gate -> site 13), rmsnorm_bf_vec.txt
* l2norm   -- `l2norm_rs_vec OUT 128` (ref/l2norm_rs_vec.c; sim/ holds no
              committed file for this unit)

The GPU box has no reference tree, so the GPU parity tests read this file.
Usage: python tests/golden/make_gdn_block_golden.py
"""
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402

REF = O.REF_TREE
OUT = os.path.join(HERE, "gdn_block_golden.npz")
BIN = os.path.join(ROOT, "oracle", "_ref")


def ints(line, dt=np.int64):
    return np.array([int(v) for v in line.split()], dt)


def parse_block(text):
    """The gdn_block_vec output (ref/gdn_block_vec.c:632-730)."""
    L = text.splitlines()
    KH, VH, D, KC, NL, T, w_e, z_e, kdiv = [int(v) for v in L[0].split()]
    assert KC == 4 and kdiv == 0
    CH = 2 * KH * D + VH * D
    d = dict(shape=np.array([KH, VH, D, T, w_e, z_e], np.int64), cw_exp=ints(L[1], np.int32),
             wm=ints(L[2], np.int16), wtap=ints(L[3], np.int16).reshape(CH, 4),
             smem0=ints(L[4], np.int16).reshape(VH, D, D), semem0=ints(L[5], np.int32).reshape(VH, D))
    caps, xt, sc, zm, ye, y = [], [], [], [], [], []
    p = 6
    for t in range(T):
        caps.append(ints(L[p], np.int32))
        xt.append(ints(L[p + 1], np.int16).reshape(CH, 4))
        sc.append(ints(L[p + 2], np.int32).reshape(VH, 8))
        zm.append(ints(L[p + 3], np.int16).reshape(VH, D))
        ye.append(int(L[p + 4]))
        y.append(ints(L[p + 5], np.int16))
        p += 6
    d.update(caps=np.array(caps), xtap=np.array(xt), sc=np.array(sc), zm=np.array(zm),
             y_exp=np.array(ye, np.int32), y=np.array(y))
    d["smem1"] = ints(L[p], np.int16).reshape(VH, D, D)
    d["semem1"] = ints(L[p + 1], np.int32).reshape(VH, D)
    d["flags"] = ints(L[p + 2], np.int32)
    return d


def block_cases(d):
    with tempfile.TemporaryDirectory() as td:
        for name, args in (("reg", ["2", "4", "32", "2", "2", "mod"]),
                           ("m128", ["16", "32", "128", "3", "1", "mod", "20261202"])):
            path = os.path.join(td, name + ".txt")
            subprocess.run([os.path.join(BIN, "gdn_block_vec"), path] + args, check=True,
                           stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            b = parse_block(open(path).read())
            if name == "m128":
                b["smem1_sha256"] = np.frombuffer(hashlib.sha256(b.pop("smem1").tobytes()).digest(),
                                                  np.uint8)
            for k, v in b.items():
                d["blk_%s_%s" % (name, k)] = v


def sim_lines(name):
    return open(os.path.join(REF, "sim", name)).read().splitlines()


def unit_cases(d):
    L = sim_lines("gdn_conv_vec.txt")                       # ref/gdn_conv_vec.c:51,118-123
    n, ch, k = [int(v) for v in L[0].split()]
    meta, x, w, sm = [], [], [], []
    for c in range(n):
        b = 1 + 5 * c
        meta.append(ints(L[b]))
        x.append(ints(L[b + 1], np.int16).reshape(ch, k))
        w.append(ints(L[b + 2], np.int16).reshape(ch, k))
        sm.append(ints(L[b + 3], np.int16))
    d.update(conv_meta=np.array(meta), conv_x=np.array(x), conv_w=np.array(w), conv_sm=np.array(sm))

    L = sim_lines("gdn_silu_vec.txt")                       # ref/gdn_silu_vec.c:107,144-176
    n, m = [int(v) for v in L[0].split()]
    d["silu_e"] = np.array([int(L[1 + 3 * c].split()[1]) for c in range(n)], np.int32)
    d["silu_sm"] = np.array([ints(L[2 + 3 * c], np.int16) for c in range(n)])
    d["silu_y"] = np.array([ints(L[3 + 3 * c], np.int32) for c in range(n)])

    L = sim_lines("gdn_head_emit_vec.txt")                  # ref/gdn_head_emit_vec.c:64,175-185
    n, dim = [int(v) for v in L[0].split()]
    d["hemit_meta"] = np.array([ints(L[1 + 4 * c]) for c in range(n)])
    d["hemit_oacc"] = np.array([[int(float(v)) for v in L[2 + 4 * c].split()] for c in range(n)], np.int64)
    d["hemit_eo"] = np.array([ints(L[3 + 4 * c], np.int32) for c in range(n)])
    d["hemit_o"] = np.array([ints(L[4 + 4 * c], np.int16) for c in range(n)])

    L = sim_lines("gdn_y_emit_vec.txt")                     # ref/gdn_y_emit_vec.c:74,179-187
    n, H, D = [int(v) for v in L[0].split()]
    d["yemit_meta"] = np.array([ints(L[1 + 5 * c]) for c in range(n)])
    d["yemit_ep"] = np.array([ints(L[2 + 5 * c], np.int32) for c in range(n)])
    d["yemit_om"] = np.array([ints(L[3 + 5 * c], np.int16).reshape(H, D) for c in range(n)])
    d["yemit_zm"] = np.array([ints(L[4 + 5 * c], np.int16).reshape(H, D) for c in range(n)])
    d["yemit_y"] = np.array([ints(L[5 + 5 * c], np.int16) for c in range(n)])

    L = sim_lines("gdn_emit_chain_vec.txt")                 # ref/gdn_emit_chain_vec.c:79,208-220
    nb, H, D = [int(v) for v in L[0].split()]
    meta, wm, oacc, eo, zm, y = [], [], [], [], [], []
    p = 1
    for b in range(nb):
        meta.append(ints(L[p]))
        wm.append(ints(L[p + 1], np.int16))
        p += 2
        oa, ee, zz = [], [], []
        for h in range(H):
            oa.append(ints(L[p], np.int64))
            ee.append(ints(L[p + 1], np.int32))
            zz.append(ints(L[p + 2], np.int16))
            p += 3
        oacc.append(oa)
        eo.append(ee)
        zm.append(zz)
        y.append(ints(L[p], np.int16))
        p += 1
    d.update(chain_meta=np.array(meta), chain_wm=np.array(wm), chain_oacc=np.array(oacc),
             chain_eo=np.array(eo), chain_zm=np.array(zm), chain_y=np.array(y))

    L = sim_lines("rmsnorm_bf_vec.txt")                     # ref/rmsnorm_bf_vec.c:653,707-713
    n, N, Q, e_eps, m_eps = [int(v) for v in L[0].split()]
    assert (N, Q, e_eps, m_eps) == (128, 12, 50, 1125899907)
    d["rms_meta"] = np.array([ints(L[1 + 4 * c]) for c in range(n)])
    d["rms_xm"] = np.array([ints(L[2 + 4 * c], np.int16) for c in range(n)])
    d["rms_wm"] = np.array([ints(L[3 + 4 * c], np.int16) for c in range(n)])
    d["rms_o"] = np.array([ints(L[4 + 4 * c], np.int16) for c in range(n)])


def l2norm_cases(d):
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "l2.txt")
        subprocess.run([os.path.join(BIN, "l2norm_rs_vec"), path, "128"], check=True,
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        L = open(path).read().splitlines()
    n, N = [int(v) for v in L[0].split()]
    d["l2_x"] = np.array([ints(L[1 + 3 * c], np.int32) for c in range(n)])
    d["l2_k"] = np.array([ints(L[2 + 3 * c], np.int32) for c in range(n)])
    d["l2_q"] = np.array([ints(L[3 + 3 * c], np.int32) for c in range(n)])


def main():
    if not os.path.exists(os.path.join(BIN, "gdn_block_vec")):
        raise SystemExit("build the reference first: make -C oracle ref")
    d = {}
    block_cases(d)
    unit_cases(d)
    l2norm_cases(d)
    np.savez_compressed(OUT, **d)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
