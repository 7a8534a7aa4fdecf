"""Decode-step oracle -- TEST INFRASTRUCTURE ONLY.

Imported by tests/ (and nothing in the product) as the checker for the decode
library (include/dec_b200.h).  A float64 numpy restatement of the reference's
float decoder, ref/run9b.c:

  rmsnorm           ref/run9b.c:557-569   x / sqrt(mean(x^2) + eps) * w
  l2norm            ref/run9b.c:571-581   x / max(sqrt(sum x^2), eps)
  silu / sigmoid / softplus (clamped above 20)   ref/run9b.c:583-590
  layer_gdn         ref/run9b.c:602-756   q|k|v projection, 4-tap causal conv +
                                          SiLU with a rolling state, per-head
                                          L2 norm, delta rule (value head h
                                          reads key head h % KH), output RMSNorm
                                          THEN silu(z) gate, out projection,
                                          residual, SwiGLU tail
  layer_attn        ref/run9b.c:758-900   q|gate interleaved per head, q/k
                                          RMSNorm, NeoX RoPE on the first n_rot
                                          dims, KV cache, GQA softmax
                                          attention (q head h reads kv head
                                          h / (QH/KVH)), sigmoid(gate) on the
                                          raw projection, O projection
  lm_head / argmax_first   ref/run9b.c:399-405, :522-540

The reference stores its registers as block floating point (reg_put); the B200
decoder's floating-point mode stores the activations that feed an INT4
projection, the conv output and the KV cache as fp16 instead.  The oracle rounds
to fp16 at exactly those points (``f16``) and computes everything else in
float64, so a difference against the GPU is fp32-versus-float64 arithmetic
only.  Weights are the INT4 g128 images the library holds (signed nibbles
times the fp16 group scale, the w_deq rule of ref/run9b.c:437-443), and every
projection sees its activation through the g128 kernel's int16 staging
(``stage_g128``), the one approximation of that kernel besides fp32 summation.

A non-zero ``mutant`` plants one of the reference's own documented mistakes
(ref/run9b.c:180-192, the REF9B_MUT list) so the tests can show that the
comparison catches each of them.
"""
import numpy as np


def f16(a):
    return np.asarray(a, np.float64).astype(np.float16).astype(np.float64)


def dequant_g128(wq, sc):
    """[rows][cols/2] packed nibbles (low first) + [rows][cols/128] fp16 scales."""
    rows, half = wq.shape
    q = np.empty((rows, 2 * half), np.int16)
    q[:, 0::2] = wq & 0xF
    q[:, 1::2] = wq >> 4
    q = np.where(q >= 8, q - 16, q)
    s = np.asarray(sc, np.uint16).view(np.float16).astype(np.float64)
    return q.astype(np.float64) * np.repeat(s, 128, axis=1)


def stage_g128(x):
    """The g128 matvec's activation staging (the numeric contract of
    mv4i_kernels.cu stage_x for KIND_G128): per 128-column group, e = 15 -
    (exponent of the group's max |x|, frexp convention), x_i ->
    sat16(rint(x_i * 2^e)) * 2^-e, round half to even.  Finer than the
    reference's own BFP registers (one exponent per whole vector, reg_put at
    ref/run9b.c:343-359), coarser than fp16 for elements below max/16."""
    x = np.asarray(x, np.float64)
    n = x.size
    G = (n + 127) // 128
    g = np.zeros(G * 128)
    g[:n] = x
    g = g.reshape(G, 128)
    am = np.max(np.abs(g), axis=1)
    ex = np.frexp(am)[1]
    e = np.where(am > 0, 15 - ex, 0)[:, None]
    q = np.clip(np.rint(np.ldexp(g, e)), -32768, 32767)
    return np.ldexp(q, -e).reshape(-1)[:n]


def rmsnorm(x, w, eps, mutant=0):
    if mutant == 7:
        return x / (np.sqrt(np.mean(x * x)) + eps) * w
    return x / np.sqrt(np.mean(x * x) + eps) * w


def l2norm(x, eps, mutant=0):
    s = np.sum(x * x)
    d = np.sqrt(s + eps) if mutant == 2 else max(np.sqrt(s), eps)
    return x / d


def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def softplus(x, mutant=0):
    if mutant == 6:
        return np.log1p(np.exp(x))
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


class Model:
    """The whole (unsharded) model: cfg is a dict with the dec_config fields;
    W maps (layer, name) to a dequantised float64 matrix; P maps (layer, name)
    to float64 vectors; S holds the states (conv [3][conv_dim], rec
    [VH][j][i] with value column j over key i, kcache/vcache [ctx][KVH][att_hd]
    fp16 values)."""

    def __init__(self, cfg, W, P, S, mutant=0, fp16=True, stage=None):
        self.c, self.W, self.P, self.S, self.mut = cfg, W, P, S, mutant
        # fp16=False: no storage rounding at all (the reference's --acts f32)
        self.r = f16 if fp16 else (lambda a: np.asarray(a, np.float64))
        # stage: the g128 kernel's int16 activation staging before every
        # projection (default: with fp16 storage)
        self.stage = fp16 if stage is None else stage
        self.seams = {}          # (layer, name) -> value, as the reference's seam()

    def mv(self, w, x):
        return w @ (stage_g128(x) if self.stage else x)

    def is_attn(self, il):
        return ((il + 1) % self.c["attn_every"]) == 0

    def gdn(self, il, x):
        c, W, P, S, mut, f16 = self.c, self.W, self.P, self.S, self.mut, self.r
        eps, KH, VH, HD = c["rms_eps"], c["gdn_kh"], c["gdn_vh"], c["gdn_hd"]
        h = f16(rmsnorm(x, P[il, "attn_norm"], eps, mut))
        mixed = self.mv(W[il, "qkv"], h)
        z = self.mv(W[il, "z"], h)
        ab = self.mv(W[il, "ab"], h)
        cw = P[il, "conv_w"].reshape(-1, 4)
        cs = S[il, "conv_state"]
        acc = cs[0] * cw[:, 0] + cs[1] * cw[:, 1] + cs[2] * cw[:, 2] + mixed * cw[:, 3]
        S[il, "conv_state"] = np.stack([cs[1], cs[2], mixed])
        conv = f16(silu(acc))
        self.seams.update({(il, "qkv"): mixed, (il, "z"): z, (il, "ab"): ab, (il, "qkv16"): conv, (il, "h16"): h})
        kd = KH * HD
        qc, kc, vc = conv[:kd].reshape(KH, HD), conv[kd:2 * kd].reshape(KH, HD), conv[2 * kd:].reshape(VH, HD)
        qc = np.stack([l2norm(r, eps, mut) for r in qc])
        kc = np.stack([l2norm(r, eps, mut) for r in kc])
        beta = sigmoid(ab[VH:])
        gdec = softplus(ab[:VH] + P[il, "dt_bias"], mut) * P[il, "ssm_a"]
        st = S[il, "rec_state"]
        out = np.empty((VH, HD))
        for hh in range(VH):
            ki = hh // 2 if mut == 3 else hh % KH
            Sh = st[hh] * np.exp(gdec[hh])                    # [j][i]
            delta = (vc[hh] - Sh @ kc[ki]) * beta[hh]
            Sh = Sh + np.outer(delta, kc[ki])
            st[hh] = Sh
            out[hh] = (Sh @ qc[ki]) / np.sqrt(HD)
        zz = z.reshape(VH, HD)
        self.seams[il, "o"] = out.reshape(-1)
        if mut == 5:
            y = np.stack([rmsnorm(out[i] * silu(zz[i]), P[il, "ssm_norm"], eps, mut) for i in range(VH)])
        else:
            y = np.stack([rmsnorm(out[i], P[il, "ssm_norm"], eps, mut) * silu(zz[i]) for i in range(VH)])
        self.seams[il, "y16"] = f16(y.reshape(-1))
        return x + self.mv(W[il, "out"], f16(y.reshape(-1)))

    def attn(self, il, x, pos):
        c, W, P, S, mut, f16 = self.c, self.W, self.P, self.S, self.mut, self.r
        eps, QH, KVH, nrot, HD = c["rms_eps"], c["att_qh"], c["att_kvh"], c["n_rot"], c["att_hd"]
        h = f16(rmsnorm(x, P[il, "attn_norm"], eps, mut))
        qg = self.mv(W[il, "qg"], h)
        kv = self.mv(W[il, "kv"], h)
        if mut == 1:
            q, g = qg[:QH * HD].reshape(QH, HD), qg[QH * HD:].reshape(QH, HD)
        else:
            q, g = qg.reshape(QH, 2, HD)[:, 0], qg.reshape(QH, 2, HD)[:, 1]
        q = np.stack([rmsnorm(r, P[il, "q_norm"], eps, mut) for r in q])
        k = np.stack([rmsnorm(r, P[il, "k_norm"], eps, mut) for r in kv[:KVH * HD].reshape(KVH, HD)])
        v = kv[KVH * HD:].reshape(KVH, HD)
        half = nrot // 2
        for vecs in (q, k):
            for r in vecs:
                for i in range(half):
                    th = pos * c["rope_theta"] ** (-2.0 * i / nrot)
                    i0, i1 = (2 * i, 2 * i + 1) if mut == 4 else (i, i + half)
                    a, b = r[i0], r[i1]
                    r[i0], r[i1] = a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)
        S[il, "kcache"][pos] = f16(k)
        S[il, "vcache"][pos] = f16(v)
        kc, vc = S[il, "kcache"][:pos + 1], S[il, "vcache"][:pos + 1]
        t = np.empty((QH, HD))
        for hh in range(QH):
            g_kv = hh % KVH if mut == 9 else hh // (QH // KVH)
            sc = kc[:, g_kv] @ q[hh] / np.sqrt(HD)
            e = np.exp(sc - sc.max())
            t[hh] = (e @ vc[:, g_kv]) / e.sum()
        t = t * sigmoid(g)
        return x + self.mv(W[il, "o"], f16(t.reshape(-1)))

    def ffn(self, il, x):
        eps, f16 = self.c["rms_eps"], self.r
        h = f16(rmsnorm(x, self.P[il, "post_norm"], eps, self.mut))
        hh = f16(silu(self.mv(self.W[il, "gate"], h)) * self.mv(self.W[il, "up"], h))
        self.seams.update({(il, "xmid"): x, (il, "post16"): h, (il, "hf16"): hh})
        return x + self.mv(self.W[il, "down"], hh)

    def step(self, tok, pos, x_in=None):
        """One token: returns (float64 logits, argmax_first token).  x_in
        (optional, [n_layers + 1][hidden]): the residual each layer starts
        from and the LM head's input, taken from the implementation under test
        (its residual seams) instead of this model's own, so each layer is
        compared from identical inputs; self.layer_out[il] is layer il's output
        from that input."""
        x = self.P[-1, "embed"][tok].astype(np.float64)
        self.layer_out = []
        for il in range(self.c["n_layers"]):
            if x_in is not None:
                x = np.asarray(x_in[il], dtype=np.float64)
            x = self.attn(il, x, pos) if self.is_attn(il) else self.gdn(il, x)
            x = self.ffn(il, x)
            self.layer_out.append(x)
        if x_in is not None:
            x = np.asarray(x_in[self.c["n_layers"]], dtype=np.float64)
        self.last_x = x
        h = self.r(rmsnorm(x, self.P[-1, "final_norm"], self.c["rms_eps"], self.mut))
        logits = self.mv(self.W[-1, "lm_head"], h)
        return logits, int(np.argmax(logits))                 # numpy: first maximum
