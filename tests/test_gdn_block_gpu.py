"""GPU parity of the fixed-point Gated DeltaNet block (subsystem B, one token
end to end) through the C ABI: deltanet_step (device buffers), the host-buffer
drop-in gdn_block_token_host, and the unit entry points of the block's
stages.  Every comparison is BIT-EXACT:

* against the reference's own outputs (tests/golden/gdn_block_golden.npz:
  gdn_block_vec at the regression arguments "2 4 32 2 2 mod" and at KH 16 /
  VH 32 / D 128 over 3 tokens, and the committed sim/ unit vector files);
* against the reference's gdn_block_token called directly
  (oracle/_ref/libref_gdn.so, compiled from its source) and the oracle
  restatement, over multi-token runs on seeded stimulus.
"""
import ctypes as C
import hashlib
import os

import numpy as np
import pytest

import oracle as O
from test_gdn_block_pins import block_stim

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "gdn_block_golden.npz")


@pytest.fixture(scope="module")
def gb():
    return np.load(GOLD)


def _p(t):
    return C.c_void_p(t.data_ptr())


def _dev(torch, a, dt=None):
    a = np.ascontiguousarray(a if dt is None else np.asarray(a, dt))
    return torch.from_numpy(a.copy()).cuda()


class DevBlock:
    """Device-resident state + workspace for deltanet_step."""

    def __init__(self, torch, pkg, KH, VH, D, stim, smem, semem):
        self.t, self.pkg, self.KH, self.VH, self.D = torch, pkg, KH, VH, D
        self.stim = stim
        self.smem = _dev(torch, smem, np.int16)
        self.semem = _dev(torch, semem, np.int32)
        self.wtap = _dev(torch, stim["wtap"], np.int16)
        self.wm = _dev(torch, stim["wm"], np.int16)
        nb = pkg.lib().deltanet_work_bytes(KH, VH, D)
        assert nb > 0
        self.work = torch.zeros(nb // 4 + 64, dtype=torch.int32, device="cuda")
        self.y = torch.zeros(VH * D, dtype=torch.int16, device="cuda")
        self.status = torch.zeros(5, dtype=torch.int32, device="cuda")

    def args(self, t, keep, pdl=0):
        s = self.stim
        xt, sc, zm = _dev(self.t, s["xtap"][t], np.int16), _dev(self.t, s["sc"][t], np.int32), \
            _dev(self.t, s["zm"][t], np.int16)
        keep += [xt, sc, zm]
        a = self.pkg.DeltanetArgs()
        a.KH, a.VH, a.D = self.KH, self.VH, self.D
        a.xtap, a.wtap = xt.data_ptr(), self.wtap.data_ptr()
        for sg in range(3):
            a.cw_exp[sg] = int(s["cw_exp"][sg])
            for k in range(4):
                a.e_t[sg][k] = int(s["e_t"][t][sg][k])
                a.tvalid[sg][k] = int(s["tvalid"][t][sg][k])
        a.sc, a.zm, a.wm = sc.data_ptr(), zm.data_ptr(), self.wm.data_ptr()
        a.w_e, a.z_e, a.tk0 = int(s["w_e"]), int(s["z_e"]), int(s["tk0"][t])
        a.smem, a.semem, a.y, a.status = self.smem.data_ptr(), self.semem.data_ptr(), \
            self.y.data_ptr(), self.status.data_ptr()
        w = self.work.data_ptr()
        a.work = (w + 255) & ~255
        a.pdl = pdl
        return a

    def run(self, T, pdl=0):
        """T tokens; returns y [T][VH*D], y_exp [T], flags [T][4]."""
        ys, ye, fl = [], [], []
        for t in range(T):
            keep = []
            a = self.args(t, keep, pdl)
            assert self.pkg.lib().deltanet_step(C.byref(a), None) == 0
            st = self.status.cpu().numpy()
            ys.append(self.y.cpu().numpy())
            ye.append(int(st[0]))
            fl.append(st[1:5].copy())
        return np.array(ys), np.array(ye, np.int32), np.array(fl)


@pytest.mark.parametrize("name", ["reg", "m128"])
def test_block_fixtures(cuda, pkg, gb, name):
    """Every token of the reference's gdn_block_vec output, its final state and
    flags, from deltanet_step with the state resident on the device."""
    (KH, VH, D, T), stim, smem, semem = block_stim(gb, name)
    blk = DevBlock(cuda, pkg, KH, VH, D, stim, smem, semem)
    y, ye, fl = blk.run(T)
    p = "blk_%s_" % name
    assert np.array_equal(ye, gb[p + "y_exp"])
    assert np.array_equal(y, gb[p + "y"])
    sm = blk.smem.cpu().numpy()
    if name == "m128":
        assert hashlib.sha256(sm.tobytes()).digest() == gb[p + "smem1_sha256"].tobytes()
    else:
        assert np.array_equal(sm, gb[p + "smem1"])
    assert np.array_equal(blk.semem.cpu().numpy(), gb[p + "semem1"])
    assert np.array_equal(fl.max(axis=0), gb[p + "flags"])


@pytest.mark.parametrize("shape", [(2, 4, 32, 6), (4, 8, 64, 5), (16, 32, 128, 4), (2, 2, 128, 3),
                                   (8, 8, 128, 5)])
def test_block_matches_reference_multitoken(cuda, pkg, shape):
    """deltanet_step against the reference's gdn_block_token (or, where
    oracle/_ref is absent, the oracle pinned to it) token by token."""
    KH, VH, D, T = shape
    stim, smem, semem = O.gdn_block_stimulus(KH, VH, D, T, seed=100 + KH + D)
    blk = DevBlock(cuda, pkg, KH, VH, D, stim, smem, semem)
    s2, e2 = smem.copy(), semem.copy()
    y2, ye2, f2 = O.gdn_block_run(KH, VH, D, stim, s2, e2, use_ref=O.have_gdn_ref())
    y, ye, fl = blk.run(T)
    assert np.array_equal(ye, ye2) and np.array_equal(y, y2)
    assert np.array_equal(fl, f2)
    assert np.array_equal(blk.smem.cpu().numpy(), s2) and np.array_equal(blk.semem.cpu().numpy(), e2)


def test_block_pdl_chain_equals_serial(cuda, pkg):
    """Tokens launched back to back as programmatic dependents of one another
    (state prefetch overlapping the previous token) equal the oracle."""
    KH, VH, D, T = 16, 32, 128, 6
    stim, smem, semem = O.gdn_block_stimulus(KH, VH, D, T, seed=3)
    blk = DevBlock(cuda, pkg, KH, VH, D, stim, smem, semem)
    keep, ys = [], []
    for t in range(T):
        a = blk.args(t, keep, pdl=1)
        assert pkg.lib().deltanet_step(C.byref(a), None) == 0
        ys.append(blk.y.clone())
    cuda.cuda.synchronize()
    s2, e2 = smem.copy(), semem.copy()
    y2, _, _ = O.gdn_block_run(KH, VH, D, stim, s2, e2)
    assert np.array_equal(np.array([y.cpu().numpy() for y in ys]), y2)
    assert np.array_equal(blk.smem.cpu().numpy(), s2)


def test_block_host_dropin(cuda, pkg, gb):
    """gdn_block_token_host: the reference's record in host memory, updated in
    place, sticky flags -- equal to the reference fixture."""
    (KH, VH, D, T), stim, smem, semem = block_stim(gb, "reg")
    wtap = np.ascontiguousarray(stim["wtap"], np.int16)
    cw = np.ascontiguousarray(stim["cw_exp"], np.int32)
    wm = np.ascontiguousarray(stim["wm"], np.int16)
    for t in range(T):
        keep = [np.ascontiguousarray(stim[k][t], dt) for k, dt in
                (("xtap", np.int16), ("e_t", np.int32), ("tvalid", np.int32), ("sc", np.int32),
                 ("zm", np.int16))]
        y = np.zeros(VH * D, np.int16)
        b = O.Blk()
        b.xtap, b.wtap, b.e_t, b.tvalid = keep[0].ctypes.data, wtap.ctypes.data, keep[1].ctypes.data, \
            keep[2].ctypes.data
        b.cw_exp, b.sc, b.zm, b.wm = cw.ctypes.data, keep[3].ctypes.data, keep[4].ctypes.data, wm.ctypes.data
        b.w_e, b.z_e, b.tk0 = int(stim["w_e"]), int(stim["z_e"]), int(stim["tk0"][t])
        b.smem, b.semem, b.y = smem.ctypes.data, semem.ctypes.data, y.ctypes.data
        assert pkg.lib().gdn_block_token_host(KH, VH, D, C.byref(b)) == 0
        assert b.y_exp == int(gb["blk_reg_y_exp"][t]) and np.array_equal(y, gb["blk_reg_y"][t])
    assert np.array_equal(smem, gb["blk_reg_smem1"]) and np.array_equal(semem, gb["blk_reg_semem1"])


def test_block_refusals(cuda, pkg):
    KH, VH, D = 2, 4, 32
    stim, smem, semem = O.gdn_block_stimulus(KH, VH, D, 1, seed=1)
    blk = DevBlock(cuda, pkg, KH, VH, D, stim, smem, semem)
    keep = []
    a = blk.args(0, keep)
    for k in range(4):
        a.tvalid[1][k] = 0
    assert pkg.lib().deltanet_step(C.byref(a), None) == -11        # a segment without a valid tap
    a = blk.args(0, keep)
    a.D = 48
    assert pkg.lib().deltanet_step(C.byref(a), None) == -11
    a = blk.args(0, keep)
    a.VH = 3
    assert pkg.lib().deltanet_step(C.byref(a), None) == -11        # VH not a multiple of KH
    assert pkg.lib().deltanet_work_bytes(2, 4, 100) == 0


# --------------------------------------------------------------- unit stages

def test_conv_unit_vectors(cuda, pkg, gb):
    torch = cuda
    meta = gb["conv_meta"]
    n, ch = gb["conv_sm"].shape
    cfg = np.zeros((n, 9), np.int32)
    for c in range(n):
        vmask, cw, e0, e1, e2, e3 = [int(v) for v in meta[c][:6]]
        cfg[c] = [(vmask >> t) & 1 for t in range(4)] + [e0, e1, e2, e3, cw]
    x, w, cf = _dev(torch, gb["conv_x"]), _dev(torch, gb["conv_w"]), _dev(torch, cfg)
    sm = torch.zeros((n, ch), dtype=torch.int16, device="cuda")
    info = torch.zeros((n, 3), dtype=torch.int32, device="cuda")
    assert pkg.lib().gdn_conv_seg_dev(n, ch, _p(x), _p(w), _p(cf), _p(sm), _p(info), None) == 0
    assert np.array_equal(sm.cpu().numpy(), gb["conv_sm"])
    assert np.array_equal(info.cpu().numpy(), meta[:, 6:9].astype(np.int32))


def test_silu_unit_vectors(cuda, pkg, gb):
    torch = cuda
    n, m = gb["silu_sm"].shape
    sm, e = _dev(torch, gb["silu_sm"]), _dev(torch, gb["silu_e"])
    y = torch.zeros((n, m), dtype=torch.int32, device="cuda")
    assert pkg.lib().gdn_silu_dev(n, m, _p(sm), _p(e), _p(y), None) == 0
    assert np.array_equal(y.cpu().numpy(), gb["silu_y"])


def test_l2norm_unit_vectors(cuda, pkg, gb):
    torch = cuda
    n, N = gb["l2_x"].shape
    x = _dev(torch, gb["l2_x"])
    k = torch.zeros((n, N), dtype=torch.int16, device="cuda")
    q = torch.zeros((n, N), dtype=torch.int16, device="cuda")
    assert pkg.lib().gdn_l2norm_dev(n, N, _p(x), _p(k), _p(q), None) == 0
    assert np.array_equal(k.cpu().numpy().astype(np.int32), gb["l2_k"])
    assert np.array_equal(q.cpu().numpy().astype(np.int32), gb["l2_q"])


def test_rmsnorm_unit_vectors(cuda, pkg, gb):
    torch = cuda
    n, N = gb["rms_xm"].shape
    meta = gb["rms_meta"]
    xm, wm = _dev(torch, gb["rms_xm"]), _dev(torch, gb["rms_wm"])
    xe, we = _dev(torch, meta[:, 1], np.int32), _dev(torch, meta[:, 2], np.int32)
    o = torch.zeros((n, N), dtype=torch.int16, device="cuda")
    oe = torch.zeros(n, dtype=torch.int32, device="cuda")
    assert pkg.lib().gdn_rmsnorm_bf_dev(n, N, _p(xm), _p(xe), _p(wm), _p(we), _p(o), _p(oe), None) == 0
    assert np.array_equal(o.cpu().numpy(), gb["rms_o"])
    assert np.array_equal(oe.cpu().numpy(), meta[:, 3].astype(np.int32))


def test_y_emit_unit_vectors(cuda, pkg, gb):
    torch = cuda
    st = torch.zeros(5, dtype=torch.int32, device="cuda")
    for c in range(gb["yemit_meta"].shape[0]):
        H, D = gb["yemit_om"][c].shape
        ep, om, zm = _dev(torch, gb["yemit_ep"][c]), _dev(torch, gb["yemit_om"][c]), _dev(torch, gb["yemit_zm"][c])
        y = torch.zeros(H * D, dtype=torch.int16, device="cuda")
        assert pkg.lib().gdn_y_emit_dev(H, D, _p(ep), _p(om), _p(zm), _p(y), _p(st), None) == 0
        s = st.cpu().numpy()
        _, y_exp, sat = [int(v) for v in gb["yemit_meta"][c]]
        assert np.array_equal(y.cpu().numpy(), gb["yemit_y"][c]) and (s[0], s[4]) == (y_exp, sat), c


def test_emit_chain_unit_vectors(cuda, pkg, gb):
    torch = cuda
    st = torch.zeros(5, dtype=torch.int32, device="cuda")
    for b in range(gb["chain_meta"].shape[0]):
        _, y_exp, sat, we, z_e = [int(v) for v in gb["chain_meta"][b]]
        H, D = gb["chain_zm"][b].shape
        nb = pkg.lib().deltanet_work_bytes(1, H, D)
        work = torch.zeros(nb // 4 + 64, dtype=torch.int32, device="cuda")
        oa, eo = _dev(torch, gb["chain_oacc"][b]), _dev(torch, gb["chain_eo"][b])
        zm, wm = _dev(torch, gb["chain_zm"][b]), _dev(torch, gb["chain_wm"][b])
        y = torch.zeros(H * D, dtype=torch.int16, device="cuda")
        wp = (work.data_ptr() + 255) & ~255
        assert pkg.lib().gdn_emit_chain_dev(H, D, _p(oa), _p(eo), _p(zm), _p(wm), we, z_e, _p(y), _p(st),
                                            C.c_void_p(wp), None) == 0
        s = st.cpu().numpy()
        assert np.array_equal(y.cpu().numpy(), gb["chain_y"][b]) and (s[0], s[4]) == (y_exp, sat), b
