"""Pins oracle/dec_oracle.py against the reference's own float decoder.

ref/run9b.c (compiled in place into oracle/_ref/libref_run9b.so by
oracle/Makefile) runs one DeltaNet layer and one gated-attention layer, each
with its SwiGLU tail, at the reference's compiled shapes (hidden 4096, 16/32
DeltaNet heads, 16/4 attention heads of dim 256 with 64 rotary dims, FFN
12288), with activations in double (its --acts f32).  The weights are random
INT4 images packed by the oracle's packer into a synthetic index directory the
reference's own loader reads; the states are random.  The numpy oracle, given
the same dequantised weights and states and no fp16 rounding, must agree to
1e-9 relative on the residual and on every state it updates.  CPU only.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from oracle import dec_oracle as D

REFLIB = os.path.join(O.HERE, "_ref", "libref_run9b.so")
pytestmark = pytest.mark.skipif(not os.path.exists(REFLIB), reason="oracle/_ref/libref_run9b.so not built")

W_EXP = 8
CB = np.arange(-8, 8, dtype=np.int8)          # a linear codebook


def _ref():
    L = C.CDLL(REFLIB)
    L.r9_shape.argtypes = [C.c_void_p]
    L.r9_rms_eps.restype = C.c_double
    L.r9_rope_base.restype = C.c_double
    L.r9_open.argtypes = [C.c_char_p]
    L.r9_layer.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                           C.c_int]
    return L


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


class DeqLinear:
    """W @ x for a packed INT4 matrix, dequantised by w_deq (ref/run9b.c:437-443:
    cb * scale / 32768 * 2^-w_exp, exact in float32) one row block at a time
    into a reused buffer, products and sums in float64."""

    BLOCK = 512

    def __init__(self, idx, scl):
        self.idx, self.scl = idx, scl
        self.M, self.K = idx.shape
        self.buf = np.empty((self.BLOCK, self.K), np.float32)

    def __matmul__(self, x):
        cbf = CB.astype(np.float32) * np.float32(2.0 ** -(15 + W_EXP))
        y = np.empty(self.M)
        for r0 in range(0, self.M, self.BLOCK):
            r1 = min(self.M, r0 + self.BLOCK)
            b = self.buf[:r1 - r0]
            np.take(cbf, self.idx[r0:r1], out=b)
            b.reshape(r1 - r0, self.K // 32, 32)[...] *= self.scl[r0:r1, :, None]
            y[r0:r1] = b @ x
        return y


class Stacked:
    def __init__(self, *parts):
        self.parts = parts

    def __matmul__(self, x):
        return np.concatenate([p @ x for p in self.parts])


class Packed:
    """A synthetic packed directory in the reference's index format
    (ref/run9b.c:236-282: MV4I / BLOB / F32 records)."""

    def __init__(self, d, rng):
        self.d, self.rng, self.lines, self.blob, self.W, self.P = d, rng, [], [], {}, {}

    def linear(self, key, tensor, M, K, segs=None):
        idx = self.rng.integers(0, 16, (M, K), dtype=np.uint8)
        scl = self.rng.integers(8000, 32000, (M, K // 32), dtype=np.uint16)
        img = O.pack(M, K, 4, 128, W_EXP, 8, CB, idx, scl)
        fn = tensor.replace(".", "_") + ".mv4i"
        with open(os.path.join(self.d, fn), "wb") as f:
            f.write(img)
        segs = segs or [("all", 0, M)]
        seg = " ".join("%s %d %d %d" % (n, r0, nr, r0) for n, r0, nr in segs)
        self.lines.append("MV4I %s %s %d %d %d %d %d %s" % (tensor, fn, M, K, W_EXP, 8, len(segs), seg))
        self.W[key] = DeqLinear(idx, scl)

    def vec(self, key, name, n, mean, std):
        v = (mean + std * self.rng.standard_normal(n)).astype(np.float32)
        off = sum(b.nbytes for b in self.blob)
        self.blob.append(v)
        self.lines.append("F32 %s %d %d %d 1" % (name, off, v.nbytes, n))
        self.P[key] = v.astype(np.float64)

    def close(self):
        np.concatenate(self.blob).tofile(os.path.join(self.d, "blob.f32"))
        self.lines.append("BLOB blob.f32")
        with open(os.path.join(self.d, "index.txt"), "w") as f:
            f.write("\n".join(self.lines) + "\n")


def test_oracle_layers_match_run9b_float_layers(tmp_path):
    L = _ref()
    sh = np.zeros(13, np.int32)
    L.r9_shape(_p(sh))
    NL, AI, H, FFN, V, KH, VH, GHD, QH, KVH, AHD, NROT, KCONV = (int(v) for v in sh)
    assert KCONV == 4
    cfg = dict(hidden=H, n_layers=NL, attn_every=AI, vocab=V, ffn=FFN, gdn_kh=KH, gdn_vh=VH, gdn_hd=GHD,
               att_qh=QH, att_kvh=KVH, att_hd=AHD, n_rot=NROT, rope_theta=L.r9_rope_base(),
               rms_eps=L.r9_rms_eps(), max_ctx=16)
    rng = np.random.default_rng(2024)
    pk = Packed(str(tmp_path), rng)
    ig, ia = 0, AI - 1                                       # one DeltaNet, one attention layer
    kd, vd = KH * GHD, VH * GHD
    conv_dim = 2 * kd + vd
    pk.linear((ig, "qkv"), "blk.%d.attn_qkv.weight" % ig, conv_dim, H,
              [("q", 0, kd), ("k", kd, kd), ("v", 2 * kd, vd)])
    pk.linear((ig, "z"), "blk.%d.attn_gate.weight" % ig, vd, H)
    pk.linear((ig, "b"), "blk.%d.ssm_beta.weight" % ig, VH, H)
    pk.linear((ig, "a"), "blk.%d.ssm_alpha.weight" % ig, VH, H)
    pk.linear((ig, "out"), "blk.%d.ssm_out.weight" % ig, H, vd)
    pk.linear((ia, "qg"), "blk.%d.attn_q.weight" % ia, 2 * QH * AHD, H)
    pk.linear((ia, "k"), "blk.%d.attn_k.weight" % ia, KVH * AHD, H)
    pk.linear((ia, "v"), "blk.%d.attn_v.weight" % ia, KVH * AHD, H)
    pk.linear((ia, "o"), "blk.%d.attn_output.weight" % ia, H, QH * AHD)
    for il in (ig, ia):
        pk.linear((il, "gate"), "blk.%d.ffn_gate.weight" % il, FFN, H)
        pk.linear((il, "up"), "blk.%d.ffn_up.weight" % il, FFN, H)
        pk.linear((il, "down"), "blk.%d.ffn_down.weight" % il, H, FFN)
        pk.vec((il, "attn_norm"), "blk.%d.attn_norm.weight" % il, H, 1.0, 0.1)
        pk.vec((il, "post_norm"), "blk.%d.post_attention_norm.weight" % il, H, 1.0, 0.1)
    pk.vec((ig, "conv_w"), "blk.%d.ssm_conv1d.weight" % ig, conv_dim * 4, 0.0, 0.5)
    pk.vec((ig, "ssm_a"), "blk.%d.ssm_a" % ig, VH, -1.0, 0.2)
    pk.vec((ig, "dt_bias"), "blk.%d.ssm_dt.bias" % ig, VH, 0.0, 0.5)
    pk.vec((ig, "ssm_norm"), "blk.%d.ssm_norm.weight" % ig, GHD, 1.0, 0.1)
    pk.vec((ia, "q_norm"), "blk.%d.attn_q_norm.weight" % ia, AHD, 1.0, 0.1)
    pk.vec((ia, "k_norm"), "blk.%d.attn_k_norm.weight" % ia, AHD, 1.0, 0.1)
    pk.close()
    W = dict(pk.W)
    W[ig, "ab"] = Stacked(W.pop((ig, "a")), W.pop((ig, "b")))
    W[ia, "kv"] = Stacked(W.pop((ia, "k")), W.pop((ia, "v")))
    assert L.r9_open(str(tmp_path).encode()) == 0

    # reference-layout states for layers 0..il
    maxpos, pos = cfg["max_ctx"], 9
    conv = np.zeros((ia + 1, KCONV - 1, conv_dim))
    rec = np.zeros((ia + 1, VH, GHD, GHD))                  # [key][val]
    kc = np.zeros((ia + 1, maxpos, KVH * AHD))
    vc = np.zeros((ia + 1, maxpos, KVH * AHD))
    conv[ig] = 0.5 * rng.standard_normal((KCONV - 1, conv_dim))
    rec[ig] = 0.02 * rng.standard_normal((VH, GHD, GHD))
    kc[ia, :pos] = rng.standard_normal((pos, KVH * AHD))
    vc[ia, :pos] = rng.standard_normal((pos, KVH * AHD))
    S = {(ig, "conv_state"): conv[ig].copy(), (ig, "rec_state"): rec[ig].transpose(0, 2, 1).copy(),
         (ia, "kcache"): kc[ia].reshape(maxpos, KVH, AHD).copy(),
         (ia, "vcache"): vc[ia].reshape(maxpos, KVH, AHD).copy()}
    M = D.Model(cfg, W, pk.P, S, fp16=False)

    for il in (ig, ia):
        x = rng.standard_normal(H)
        want = x.copy()
        assert L.r9_layer(il, _p(want), _p(conv), _p(rec), _p(kc), _p(vc), maxpos, pos) == 0
        got = M.attn(il, x, pos) if il == ia else M.gdn(il, x)
        got = M.ffn(il, got)
        assert np.max(np.abs(got - want)) <= 1e-9 * np.max(np.abs(want)), il
    assert np.allclose(S[ig, "conv_state"], conv[ig], rtol=0, atol=1e-12)
    r = rec[ig].transpose(0, 2, 1)
    assert np.max(np.abs(S[ig, "rec_state"] - r)) <= 1e-9 * np.max(np.abs(r))
    k = kc[ia].reshape(maxpos, KVH, AHD)
    assert np.max(np.abs(S[ia, "kcache"][:pos + 1] - k[:pos + 1])) <= 1e-9 * np.max(np.abs(k))
    v = vc[ia].reshape(maxpos, KVH, AHD)
    assert np.max(np.abs(S[ia, "vcache"][:pos + 1] - v[:pos + 1])) <= 1e-9 * np.max(np.abs(v))
