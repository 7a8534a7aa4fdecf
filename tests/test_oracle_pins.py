"""Pins the CPU oracle (oracle/mv4i_oracle.c) before anything is checked
against it: the reference's arithmetic golden vectors, its tile vectors, its
own mv4i_matvec / pack_geom compiled from source, and the committed fixtures
(tests/golden/mv4i_golden.npz, written by tests/golden/make_golden.py from the
reference's own code).  CPU only."""
import os
import subprocess

import numpy as np
import pytest

import oracle as O

from conftest import REF_TREE  # noqa: E402


def _img_for(golden, key):
    meta = golden[key + "_meta"]
    if key.startswith("emit"):
        return golden["img%d" % meta[12]].tobytes()
    return golden[key + "_img"].tobytes()


def test_arith_vectors(golden):
    """sim/arith_vectors.txt: 4178 primitive vectors (tools/gen_arith.py)."""
    o = O.orc()
    a = golden["arith"]
    assert a.shape[0] == 4178
    bad = 0
    for op, v, sh, e in a:
        op, v, sh, e = int(op), int(v), int(sh), int(e)
        if op == 0:
            got = o.orc_floor_shr(v, sh)
        elif op == 1:
            got = o.orc_round_shift(v, sh)
        elif op == 2:
            got = o.orc_sat32(v, None)
        elif op == 3:
            got = o.orc_sat16(v)
        elif op == 4:
            got = o.orc_msb_pos(v & (2 ** 64 - 1))
        else:
            got = o.orc_sat16(o.orc_round_shift(v, sh))
        bad += got != e
    assert bad == 0


def test_arith_vectors_file_matches_fixture(golden, ref_tree):
    """The fixture is the reference's current file, not a stale copy."""
    n = sum(1 for ln in open(os.path.join(ref_tree, "sim", "arith_vectors.txt"))
            if ln.strip() and not ln.startswith("#"))
    assert n == golden["arith"].shape[0]


def _tile_keys(golden):
    return sorted({k[:-5] for k in golden.files if k.startswith("tile") and k.endswith("_meta")},
                  key=lambda s: int(s[4:]))


def test_tile_vectors(golden):
    """sim/mv_tile_vec.txt (tools/mv_tile_model.py, an independent model of
    subsystem A): each 2-row tile packed by the oracle packer and run through
    the oracle; RAW/BFP compare the s32 pre-pack value, PARTIAL the s48 acc."""
    keys = _tile_keys(golden)
    assert len(keys) == 67
    for k in keys:
        case, tile, osh, mode, sat = [int(v) for v in golden[k + "_meta"]]
        cb, idx, scl, x = golden[k + "_cb"], golden[k + "_idx"], golden[k + "_scl"], golden[k + "_x"]
        K = idx.shape[1]
        img = O.pack(2, K, 2, 128, 0, osh, cb, idx, scl)
        rc, r = O.matvec(img, x, 0, 2, K, 2 if mode == 2 else 1)
        assert rc == 0, k
        got = r["y_acc"] if mode == 2 else r["y_data"].astype(np.int64)
        assert np.array_equal(got, golden[k + "_y"]), k
        if mode != 2:
            assert r["sat_event"] == sat, k


def test_emitted_images_and_outputs(golden):
    """Images written by the reference's `--emit` and outputs of its
    mv4i_matvec, all modes, full and partial row/column windows."""
    keys = [k[:-5] for k in golden.files if k.endswith("_meta") and not k.startswith("tile")]
    assert len(keys) >= 40
    for k in keys:
        m = [int(v) for v in golden[k + "_meta"]]
        M, K, RI, DW, x_exp, nr, nc, mode, y_exp, sat, nsat, ns = m[:12]
        rc, r = O.matvec(_img_for(golden, k), golden[k + "_x"], x_exp, nr, nc, mode)
        assert rc == 0, k
        got = r["y_acc"] if mode == 2 else (r["y_mant"] if mode == 0 else r["y_data"])
        assert np.array_equal(got.astype(np.int64), golden[k + "_y"]), k
        assert (r["y_exp"], r["sat_event"], r["sat_count"], r["ns"]) == (y_exp, sat, nsat, ns), k


needs_ref = pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("geom", [(8, 96, 4, 128), (50, 200, 4, 128), (33, 77, 8, 256),
                                  (17, 64, 4, 64), (9, 1024, 2, 128), (12, 100, 4, 32),
                                  (5, 40, 1, 8), (3, 33, 16, 512)])
def test_oracle_vs_reference_random(geom):
    """Restated packer byte-identical to pack_geom; restated matvec identical
    to mv4i_matvec (all outputs and flags) on random operands."""
    M, K, RI, DW = geom
    rng = np.random.default_rng(M * 1000 + K)
    nb = (K + 31) // 32
    for cb in (O.IQ4_NL, np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], np.int8)):
        idx = rng.integers(0, 16, (M, K), dtype=np.uint8)
        scl = rng.integers(0, 32768, (M, nb), dtype=np.uint16)
        a = O.pack(M, K, RI, DW, 2, 3, cb, idx, scl)
        assert a == O.ref_pack(M, K, RI, DW, 2, 3, cb, idx, scl)
        x = rng.integers(-32768, 32768, K, dtype=np.int16)
        for mode in (0, 1, 2):
            for nr, nc in ((M, K), (max(1, M // 2), max(1, K - 5))):
                r1 = O.matvec(a, x, 5, nr, nc, mode)
                r2 = O.ref_matvec(a, x, 5, nr, nc, mode)
                assert r1[0] == r2[0] == 0
                for f in r1[1]:
                    assert np.array_equal(np.asarray(r1[1][f]), np.asarray(r2[1][f])), (geom, mode, f)


@needs_ref
def test_reference_selftest_passes(ref_tree):
    """The reference's own self-test (ref/matvec_int4.c main), run from its tree."""
    out = subprocess.run([O.REFBIN], cwd=ref_tree, capture_output=True, text=True)
    assert out.returncode == 0 and "OK (0 failures)" in out.stdout


def test_oracle_has_teeth(golden):
    """Negative control: flipping bit 14 of the first scale changes the result."""
    k = "lin1"
    img = bytearray(golden[k + "_img"].tobytes())
    m = [int(v) for v in golden[k + "_meta"]]
    soff = int.from_bytes(img[0x30:0x34], "little")
    img[soff + 1] ^= 0x40
    rc, r = O.matvec(bytes(img), golden[k + "_x"], m[4], m[5], m[6], 1)
    assert rc == 0
    assert not np.array_equal(r["y_data"].astype(np.int64), golden[k + "_y"])


def test_tp_reduce_bounds():
    """E 2.1 option 1 against its own stated properties: the floor-aligned sum
    sits at or below the exact sum by < (N-1) ulp of the min grid; refusals at
    spread > 17 and on out_shift mismatch."""
    rng = np.random.default_rng(7)
    for N in (2, 4, 8):
        n = 64
        parts = [rng.integers(-(1 << 40), 1 << 40, n) for _ in range(N)]
        ye = list(rng.integers(10, 20, N))
        rc, out, oe, y32, sat = O.tp_reduce(parts, ye, [8] * N)
        assert rc == 0
        ymin, ymax = min(ye), max(ye)
        for r in range(n):
            exact = sum(int(parts[c][r]) << (ymax - ye[c]) for c in range(N))
            s1 = sum(int(parts[c][r]) >> (ye[c] - ymin) for c in range(N))
            diff = exact - (s1 << (ymax - ymin))
            assert 0 <= diff < (N - 1) << (ymax - ymin) or (N == 1)
    assert O.tp_reduce([np.zeros(4)] * 2, [0, 18], [3, 3])[0] == -1
    assert O.tp_reduce([np.zeros(4)] * 2, [0, 1], [3, 4])[0] == -2
