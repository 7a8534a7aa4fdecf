"""Pins the fixed-point DeltaNet block oracle (oracle/gdn_block_oracle.c)
before anything is checked against it: every committed unit vector file of the
block's stages (conv + segment requantiser, silu, site-12 head emit, site-13
renorm, the emit chain, rmsnorm_bf), the L2-norm generator's vectors, the
whole-token outputs of the reference's own gdn_block_vec generator
(tests/golden/gdn_block_golden.npz, written by make_gdn_block_golden.py from
the reference's code), and -- where oracle/_ref is built -- the reference's
gdn_block_token, rsqrt ROM and unit cores called directly.  CPU only."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gdn_block_golden.npz")


@pytest.fixture(scope="module")
def gb():
    return np.load(GOLD)


def block_stim(gb, name):
    """A fixture's stimulus in the form oracle.gdn_block_run takes."""
    p = "blk_%s_" % name
    KH, VH, D, T, w_e, z_e = [int(v) for v in gb[p + "shape"]]
    caps = gb[p + "caps"]
    et, tv = zip(*[O.blk_taps(t, caps) for t in range(T)])
    stim = dict(wtap=gb[p + "wtap"], cw_exp=gb[p + "cw_exp"], wm=gb[p + "wm"], w_e=w_e, z_e=z_e,
                tk0=np.array([1] + [0] * (T - 1), np.int32), xtap=gb[p + "xtap"],
                e_t=np.array(et), tvalid=np.array(tv), sc=gb[p + "sc"], zm=gb[p + "zm"])
    return (KH, VH, D, T), stim, gb[p + "smem0"].copy(), gb[p + "semem0"].copy()


def test_conv_vectors(gb):
    """sim/gdn_conv_vec.txt: 128 segments of 256 channels, requantised
    mantissas, e_seg, sh_seg and the range flag."""
    for c in range(gb["conv_meta"].shape[0]):
        vmask, cw, e0, e1, e2, e3, e_seg, sh_seg, err = [int(v) for v in gb["conv_meta"][c]]
        tv = [(vmask >> t) & 1 for t in range(4)]
        sm, es, ss, er = O.conv_seg(gb["conv_x"][c], gb["conv_w"][c], [e0, e1, e2, e3], tv, cw)
        assert np.array_equal(sm, gb["conv_sm"][c]), c
        assert (es, ss, er) == (e_seg, sh_seg, err), c


def test_silu_vectors(gb):
    L = O._blk_sig()
    for c in range(gb["silu_e"].size):
        e = int(gb["silu_e"][c])
        got = [L.orc_silu(int(v), e) for v in gb["silu_sm"][c]]
        assert got == [int(v) for v in gb["silu_y"][c]], c


def test_head_emit_vectors(gb):
    for c in range(gb["hemit_meta"].shape[0]):
        o, e = O.gdn_head_emit(gb["hemit_oacc"][c], gb["hemit_eo"][c])
        assert np.array_equal(o, gb["hemit_o"][c]) and e == int(gb["hemit_meta"][c][1]), c


def test_y_emit_vectors(gb):
    for c in range(gb["yemit_meta"].shape[0]):
        y, ye, sat = O.y_emit(gb["yemit_ep"][c], gb["yemit_om"][c], gb["yemit_zm"][c])
        _, y_exp, sat_any = [int(v) for v in gb["yemit_meta"][c]]
        assert np.array_equal(y, gb["yemit_y"][c]) and (ye, sat) == (y_exp, sat_any), c


def test_emit_chain_vectors(gb):
    for b in range(gb["chain_meta"].shape[0]):
        _, y_exp, sat_any, we, z_e = [int(v) for v in gb["chain_meta"][b]]
        y, ye, sat = O.emit_chain(gb["chain_oacc"][b], gb["chain_eo"][b], gb["chain_zm"][b],
                                  gb["chain_wm"][b], we, z_e)
        assert np.array_equal(y, gb["chain_y"][b]) and (ye, sat) == (y_exp, sat_any), b


def test_rmsnorm_vectors(gb):
    for c in range(gb["rms_meta"].shape[0]):
        _, xe, we, o_exp = [int(v) for v in gb["rms_meta"][c]]
        o, oe = O.rmsnorm_bf(gb["rms_xm"][c], xe, gb["rms_wm"][c], we)
        assert np.array_equal(o, gb["rms_o"][c]) and oe == o_exp, c


def test_l2norm_vectors(gb):
    for c in range(gb["l2_x"].shape[0]):
        k, q = O.l2norm_rs(gb["l2_x"][c], 7)
        assert np.array_equal(k, gb["l2_k"][c]) and np.array_equal(q, gb["l2_q"][c]), c


@pytest.mark.parametrize("name", ["reg", "m128"])
def test_block_fixtures(gb, name):
    """Whole tokens of the reference's gdn_block_vec: every token's y and y_exp,
    the final state (mantissas and exponents) and the flags."""
    (KH, VH, D, T), stim, smem, semem = block_stim(gb, name)
    p = "blk_%s_" % name
    y, ye, fl = O.gdn_block_run(KH, VH, D, stim, smem, semem)
    assert np.array_equal(y, gb[p + "y"]) and np.array_equal(ye, gb[p + "y_exp"])
    assert np.array_equal(semem, gb[p + "semem1"])
    if name == "m128":
        assert hashlib.sha256(smem.tobytes()).digest() == gb[p + "smem1_sha256"].tobytes()
    else:
        assert np.array_equal(smem, gb[p + "smem1"])
    assert np.array_equal(fl.max(axis=0), gb[p + "flags"])


def test_block_negative_control(gb):
    """A masked tap treated as valid (its garbage value and wild exponent let
    into the conv) moves the first token's output: the fixture check sees the
    masking rule."""
    (KH, VH, D, T), stim, smem, semem = block_stim(gb, "reg")
    stim["tvalid"] = stim["tvalid"].copy()
    stim["tvalid"][0, 2, 0] = 1
    y, ye, _ = O.gdn_block_run(KH, VH, D, stim, smem, semem)
    assert not np.array_equal(y[0], gb["blk_reg_y"][0])


needs_ref = pytest.mark.skipif(not O.have_gdn_ref(), reason="oracle/_ref not built")


@needs_ref
def test_rsqrt_rom_matches_reference():
    a, b = np.zeros(64, np.int64), np.zeros(64, np.int64)
    O._blk_sig().orc_rsqrt_rom(O._p(a))
    O._ref_blk().ref_rsqrt_rom(O._p(b))
    assert np.array_equal(a, b)


@needs_ref
def test_units_match_reference_random():
    """rmsnorm_bf, l2norm_rs and silu against the reference's cores on random
    inputs over the exponent ranges that reach every branch."""
    rng = np.random.default_rng(7)
    L = O._blk_sig()
    R = O._ref_blk()
    for it in range(400):
        n = 128
        mag = int(rng.integers(1, 16))
        xm = rng.integers(-(1 << mag), 1 << mag, n).astype(np.int16)
        if it % 17 == 0:
            xm[:] = 0
        wm = rng.integers(-32768, 32768, n).astype(np.int16)
        xe, we = int(rng.integers(-40, 60)), int(rng.integers(-10, 30))
        o1, e1 = O.rmsnorm_bf(xm, xe, wm, we)
        o2, e2 = O.rmsnorm_bf(xm, xe, wm, we, use_ref=True)
        assert np.array_equal(o1, o2) and e1 == e2, it
        x = rng.integers(-32768, 32769, n).astype(np.int32) >> int(rng.integers(0, 16))
        k1, q1 = O.l2norm_rs(x, 7)
        k2, q2 = O.l2norm_rs(x, 7, use_ref=True)
        assert np.array_equal(k1, k2) and np.array_equal(q1, q2), it
        e = int(rng.integers(-45, 70))
        for v in rng.integers(-32768, 32768, 16):
            assert L.orc_silu(int(v), e) == R.ref_silu(int(v), e)


@needs_ref
@pytest.mark.parametrize("shape", [(2, 4, 32, 6), (1, 3, 16, 5), (4, 8, 64, 5), (16, 32, 128, 3),
                                   (2, 2, 128, 4)])
def test_block_matches_reference(shape):
    """The whole token against the reference's gdn_block_token, multi-token,
    on seeded stimulus in the generator's ranges."""
    KH, VH, D, T = shape
    stim, smem, semem = O.gdn_block_stimulus(KH, VH, D, T, seed=11 + D)
    s2, e2 = smem.copy(), semem.copy()
    y1, ye1, f1 = O.gdn_block_run(KH, VH, D, stim, smem, semem)
    y2, ye2, f2 = O.gdn_block_run(KH, VH, D, stim, s2, e2, use_ref=True)
    assert np.array_equal(y1, y2) and np.array_equal(ye1, ye2) and np.array_equal(f1, f2)
    assert np.array_equal(smem, s2) and np.array_equal(semem, e2)
