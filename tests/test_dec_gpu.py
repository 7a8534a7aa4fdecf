"""Decode step (include/dec_b200.h) against the float64 oracle of ref/run9b.c.

A small hybrid stack (DeltaNet layers and gated-attention layers in the 3:1
pattern, INT4 g128 linears, fp16 KV cache pre-filled past one attention chunk)
is stepped on the GPU through the C ABI; every weight, parameter and state is
read back from the device into oracle/dec_oracle.py, which steps the same
tokens in float64 with fp16 rounding at the same storage points.  Before each
step the oracle takes the GPU's states, so every step is compared from the same
inputs: a value that lands on the other side of an fp16 rounding boundary
(fp32 versus float64 arithmetic) then cannot compound over steps.

Within a step, each layer is also compared from identical inputs: the step's
residual seams (the residual stream as every layer starts, and the LM head's
input) are read back, the oracle runs each layer from the GPU's input, and its
output must match the GPU's next seam.

Tolerance (floating-point mode of the benchmark): every layer's output and the
logits from identical inputs within 1e-3 of the largest magnitude, states
within 1e-3, and the same argmax token wherever the oracle's top-2 margin
exceeds that tolerance.  The free-running step (the oracle's own residual
through all 8 layers) must stay within 4e-3: one fp16 rounding flip in an early
layer (float64 versus fp32 on the same side of a rounding boundary) grows by
about 1.6x per layer through this random-weight stack, so free-running logits
can pass 1e-3 for some inputs while every layer is within 1e-4.
The reference's own planted mistakes (ref/run9b.c:180-192) put into the oracle
must each break that agreement.
"""
import ctypes as C
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import device_read

pytestmark = pytest.mark.gpu

HD = 128
CFG = dict(hidden=256, n_layers=8, attn_every=4, vocab=1000, ffn=512, gdn_kh=2, gdn_vh=4, gdn_hd=128,
           att_qh=8, att_kvh=4, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=256)
TOL = 1e-3
FREE_TOL = 4e-3
LINEARS = {"gdn": ["qkv", "z", "ab", "out"], "attn": ["qg", "kv", "o"], "ffn": ["gate", "up", "down"]}


def is_attn(il, cfg=None):
    return ((il + 1) % (cfg or CFG)["attn_every"]) == 0


class Dec:
    def __init__(self, pkg, cfg=CFG, seed=11, device=0, rank=0, world=1):
        self.pkg, self.L, self.cfg = pkg, pkg.declib(), cfg
        self.c = pkg.DecConfig(**cfg)
        self.h = C.c_void_p()
        rc = self.L.dec_create(C.byref(self.c), seed, device, rank, world, C.byref(self.h))
        assert rc == 0, (rc, pkg.lib().mv4i_last_cuda_error())

    def close(self):
        if self.h:
            assert self.L.dec_destroy(self.h) == 0
            self.h = C.c_void_p()

    def linear(self, torch, layer, name):
        wq, sc, r, k, sp = C.c_void_p(), C.c_void_p(), C.c_int32(), C.c_int32(), C.c_int32()
        rc = self.L.dec_linear(self.h, layer, name.encode(), C.byref(wq), C.byref(sc), C.byref(r), C.byref(k),
                               C.byref(sp))
        assert rc == 0, (layer, name)
        r, k, sp = r.value, k.value, sp.value
        assert sp % 8 == 0 and sp >= k // 128
        return (device_read(torch, wq.value, (r, k // 2), np.uint8),
                device_read(torch, sc.value, (r, sp), np.uint16)[:, :k // 128].copy())

    def param(self, torch, layer, name, dtype=np.float32):
        p, n = C.c_void_p(), C.c_int32()
        assert self.L.dec_param(self.h, layer, name.encode(), C.byref(p), C.byref(n)) == 0, (layer, name)
        return device_read(torch, p.value, (n.value,), dtype)

    def pointers(self):
        lg, hist, res, pos = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
        v0, vn = C.c_int32(), C.c_int32()
        assert self.L.dec_pointers(self.h, C.byref(lg), C.byref(hist), C.byref(res), C.byref(pos),
                                   C.byref(v0), C.byref(vn)) == 0
        return dict(logits=lg.value, hist=hist.value, res=res.value, pos=pos.value, v0=v0.value, vn=vn.value)

    def step(self, torch):
        rc = self.L.dec_step(self.h, C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, (rc, self.pkg.lib().mv4i_last_cuda_error())

    def seams_on(self, torch):
        """Residual seams of every step into a [n_layers + 1][batch][hidden]
        device buffer."""
        nb = max(self.cfg.get("batch", 1), 1)
        self.seam_buf = torch.zeros(self.cfg["n_layers"] + 1, nb, self.cfg["hidden"], device="cuda")
        assert self.L.dec_set_residual_seams(self.h, C.c_void_p(self.seam_buf.data_ptr()),
                                             self.cfg["n_layers"] + 1) == 0

    def seams(self, torch, seq=0):
        torch.cuda.synchronize()
        return self.seam_buf[:, seq].double().cpu().numpy()


def check_step(O, M, xs, lg, tok, pos):
    """Compares one GPU step (its logits lg and residual seams xs) with the
    oracle M, whose states already equal the GPU's before the step: every
    layer from the GPU's input and the logits from the GPU's LM-head input
    within TOL; the oracle's free-running step within FREE_TOL.  Returns the
    free-running logits and argmax."""
    Mf = O.Model(M.c, M.W, M.P, {k: v.copy() for k, v in M.S.items()}, M.mut)
    ref_free, rtok = Mf.step(tok, pos)
    ref, _ = M.step(tok, pos, x_in=xs)
    for il, out in enumerate(M.layer_out):
        assert rel(xs[il + 1], out) <= TOL, ("layer", il, rel(xs[il + 1], out))
    assert rel(lg, ref) <= TOL, ("logits", rel(lg, ref))
    assert rel(lg, ref_free) <= FREE_TOL, ("free-running logits", rel(lg, ref_free))
    return ref_free, rtok


def oracle_from(dec, torch, O, mutant=0, seq=0):
    """Everything the oracle needs, read back from a tp_world = 1 model (the
    states of sequence `seq` of a batch)."""
    cfg = dec.cfg
    nb = max(cfg.get("batch", 1), 1)
    W, P, S = {}, {}, {}
    KH, VH, KVH = cfg["gdn_kh"], cfg["gdn_vh"], cfg["att_kvh"]
    conv_dim = 2 * KH * HD + VH * HD
    for il in range(cfg["n_layers"]):
        names = LINEARS["attn" if is_attn(il, cfg) else "gdn"] + LINEARS["ffn"]
        for n in names:
            W[il, n] = O.dequant_g128(*dec.linear(torch, il, n))
        pn = ["attn_norm", "post_norm"] + (["q_norm", "k_norm"] if is_attn(il, cfg)
                                           else ["conv_w", "ssm_a", "dt_bias", "ssm_norm"])
        for n in pn:
            P[il, n] = dec.param(torch, il, n).astype(np.float64)
        if is_attn(il, cfg):
            for n in ("kcache", "vcache"):
                S[il, n] = dec.param(torch, il, n, np.float16).astype(np.float64).reshape(nb, -1, KVH, HD)[seq]
        else:
            S[il, "conv_state"] = dec.param(torch, il, "conv_state").astype(np.float64).reshape(nb, 3, conv_dim)[seq]
            S[il, "rec_state"] = dec.param(torch, il, "rec_state").astype(np.float64).reshape(nb, VH, HD, HD)[seq]
    W[-1, "lm_head"] = O.dequant_g128(*dec.linear(torch, -1, "lm_head"))
    P[-1, "final_norm"] = dec.param(torch, -1, "final_norm").astype(np.float64)
    P[-1, "embed"] = dec.param(torch, -1, "embed", np.float16).astype(np.float64).reshape(cfg["vocab"], -1)
    return O.Model(cfg, W, P, S, mutant)


def sync_states(dec, torch, M, seq=0):
    """Load the GPU's current recurrent, conv and KV states (of sequence
    `seq`) into the oracle, so each step is compared from identical inputs
    (fp16 storage flips do not carry over from one step to the next)."""
    cfg = dec.cfg
    nb = max(cfg.get("batch", 1), 1)
    for il in range(cfg["n_layers"]):
        if is_attn(il, cfg):
            for n in ("kcache", "vcache"):
                M.S[il, n] = dec.param(torch, il, n, np.float16).astype(np.float64).reshape(
                    (nb,) + M.S[il, n].shape)[seq]
        else:
            for n in ("conv_state", "rec_state"):
                M.S[il, n] = dec.param(torch, il, n).astype(np.float64).reshape((nb,) + M.S[il, n].shape)[seq]


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def O():
    from oracle import dec_oracle
    return dec_oracle


@pytest.mark.parametrize("prefill", [0, 100])
def test_decode_steps_match_oracle(pkg, cuda, O, prefill):
    torch = cuda
    d = Dec(pkg)
    try:
        assert d.L.dec_prefill_random(d.h, prefill, 5) == 0
        tok = 7
        assert d.L.dec_set(d.h, prefill, tok) == 0
        M = oracle_from(d, torch, O)
        ptrs = d.pointers()
        d.seams_on(torch)
        pos = prefill
        for s in range(4):
            sync_states(d, torch, M)
            d.step(torch)
            lg = device_read(torch, ptrs["logits"], (CFG["vocab"],), np.float32).astype(np.float64)
            ref, rtok = check_step(O, M, d.seams(torch), lg, tok, pos)
            hist = device_read(torch, ptrs["hist"], (CFG["max_ctx"],), np.int32)
            top2 = np.sort(ref)[-2:]
            if top2[1] - top2[0] > TOL * np.max(np.abs(ref)):
                assert hist[pos] == rtok, (s, hist[pos], rtok)
            assert hist[pos] == int(np.argmax(lg))
            tok = int(hist[pos])                  # the oracle follows the GPU's token
            pos += 1
            assert device_read(torch, ptrs["pos"], (1,), np.int32)[0] == pos
        for il in range(CFG["n_layers"]):
            if is_attn(il):
                kc = d.param(torch, il, "kcache", np.float16).astype(np.float64).reshape(-1, CFG["att_kvh"], HD)
                assert rel(kc[:pos], M.S[il, "kcache"][:pos]) <= TOL, il
            else:
                st = d.param(torch, il, "rec_state").astype(np.float64).reshape(M.S[il, "rec_state"].shape)
                assert rel(st, M.S[il, "rec_state"]) <= TOL, il
                cs = d.param(torch, il, "conv_state").astype(np.float64).reshape(3, -1)
                assert rel(cs, M.S[il, "conv_state"]) <= TOL, il
    finally:
        d.close()


def test_prompt_then_greedy_generation(pkg, cuda, O):
    """dec_set_prompt: a new sequence (zero states) fed the prompt's tokens,
    then its own argmax; every step's prediction lands in the history."""
    torch = cuda
    d = Dec(pkg)
    try:
        prompt = [5, 900, 17, 17, 333]
        arr = C.cast((C.c_int32 * len(prompt))(*prompt), C.c_void_p)
        assert d.L.dec_set_prompt(d.h, arr, len(prompt), None) == 0
        M = oracle_from(d, torch, O)
        assert not any(np.any(M.S[k]) for k in M.S if k[1] in ("conv_state", "rec_state"))
        ptrs = d.pointers()
        d.seams_on(torch)
        tok = prompt[0]
        for pos in range(len(prompt) + 3):
            sync_states(d, torch, M)
            d.step(torch)
            lg = device_read(torch, ptrs["logits"], (CFG["vocab"],), np.float32).astype(np.float64)
            check_step(O, M, d.seams(torch), lg, tok, pos)
            hist = device_read(torch, ptrs["hist"], (CFG["max_ctx"],), np.int32)
            assert hist[pos] == int(np.argmax(lg))
            tok = prompt[pos + 1] if pos + 1 < len(prompt) else int(hist[pos])
        assert d.L.dec_set_prompt(d.h, arr, 0, None) == -11
        bad = C.cast((C.c_int32 * 1)(CFG["vocab"]), C.c_void_p)
        assert d.L.dec_set_prompt(d.h, bad, 1, None) == -11
    finally:
        d.close()


def _batch_steps(d, torch, O, cfg, toks, pos, nsteps, prompts=None):
    """Steps a batched model and every sequence's oracle side by side."""
    nb = cfg["batch"]
    Ms = [oracle_from(d, torch, O, seq=b) for b in range(nb)]
    ptrs = d.pointers()
    d.seams_on(torch)
    plen = len(prompts[0]) if prompts else 0
    for s in range(nsteps):
        for b in range(nb):
            sync_states(d, torch, Ms[b], seq=b)
        d.step(torch)
        lg = device_read(torch, ptrs["logits"], (nb, cfg["vocab"]), np.float32).astype(np.float64)
        hist = device_read(torch, ptrs["hist"], (nb, cfg["max_ctx"]), np.int32)
        for b in range(nb):
            ref, rtok = check_step(O, Ms[b], d.seams(torch, b), lg[b], toks[b], pos)
            assert hist[b, pos] == int(np.argmax(lg[b])), (s, b)
            top2 = np.sort(ref)[-2:]
            if top2[1] - top2[0] > TOL * np.max(np.abs(ref)):
                assert hist[b, pos] == rtok, (s, b)
        toks = [prompts[b][pos + 1] if pos + 1 < plen else int(hist[b, pos]) for b in range(nb)]
        pos += 1
        assert device_read(torch, ptrs["pos"], (1,), np.int32)[0] == pos
    return toks, pos


def test_batched_sequences_match_oracle(pkg, cuda, O):
    """Three sequences decoded together (each weight read once for all three):
    every sequence, from its own pre-filled states, KV cache and token, agrees
    with its own oracle; the sequences differ from one another."""
    torch = cuda
    cfg = dict(CFG, batch=3)
    d = Dec(pkg, cfg)
    try:
        assert d.L.dec_prefill_random(d.h, 100, 5) == 0
        assert d.L.dec_set(d.h, 100, 7) == 0
        _batch_steps(d, torch, O, cfg, [7, 7, 7], 100, 3)
        lg = device_read(torch, d.pointers()["logits"], (3, cfg["vocab"]), np.float32)
        assert not np.array_equal(lg[0], lg[1]) and not np.array_equal(lg[1], lg[2])
    finally:
        d.close()
    # sequence 0 of a batch is the unbatched model's sequence (same draws).
    # A batch streams the projections on the tensor pipe (the exact integer
    # dot of each 128-column group, then one fp32 multiply-add), one sequence
    # on the CUDA cores (one fp32 multiply-add per 64-column half): the fp32
    # sums round differently, an fp16 activation can land on the other side
    # of a rounding boundary, and that grows through the layers -- so the
    # step's tolerance, not bit equality.
    d1, d3 = Dec(pkg), Dec(pkg, cfg)
    try:
        for x in (d1, d3):
            assert x.L.dec_prefill_random(x.h, 50, 9) == 0 and x.L.dec_set(x.h, 50, 3) == 0
            x.step(torch)
        a = device_read(torch, d1.pointers()["logits"], (cfg["vocab"],), np.float32).astype(np.float64)
        b = device_read(torch, d3.pointers()["logits"], (3, cfg["vocab"]), np.float32)[0].astype(np.float64)
        assert rel(b, a) <= TOL
    finally:
        d1.close()
        d3.close()


@pytest.mark.parametrize("nb", [2, 8])
def test_batched_prompts_then_greedy(pkg, cuda, O, nb):
    """dec_set_prompt with one prompt per sequence: teacher forcing per
    sequence, then each sequence's own argmax."""
    torch = cuda
    cfg = dict(CFG, batch=nb)
    d = Dec(pkg, cfg)
    try:
        rng = np.random.default_rng(nb)
        prompts = rng.integers(0, cfg["vocab"], size=(nb, 4)).astype(np.int32)
        arr = prompts.ctypes.data_as(C.c_void_p)
        assert d.L.dec_set_prompt(d.h, arr, 4, None) == 0
        _batch_steps(d, torch, O, cfg, list(prompts[:, 0]), 0, 6, prompts.tolist())
    finally:
        d.close()


@pytest.mark.parametrize("mutant", [1, 3, 4, 5, 9])
def test_planted_mistakes_in_the_oracle_are_caught(pkg, cuda, O, mutant):
    """Each of the reference's documented plausible defects, planted in the
    oracle, moves the logits well past the tolerance.  (Mutants 2, 6 and 7 --
    epsilon placement and the softplus clamp -- change nothing measurable at
    these magnitudes; the reference lists them as below its own harness floor.)"""
    torch = cuda
    d = Dec(pkg)
    try:
        assert d.L.dec_prefill_random(d.h, 100, 5) == 0
        assert d.L.dec_set(d.h, 100, 7) == 0
        M = oracle_from(d, torch, O, mutant)
        d.step(torch)
        lg = device_read(torch, d.pointers()["logits"], (CFG["vocab"],), np.float32).astype(np.float64)
        ref, _ = M.step(7, 100)
        assert rel(lg, ref) > 10 * TOL, (mutant, rel(lg, ref))
    finally:
        d.close()


def _expected_shard(full, name, cfg, R, Wd):
    """Slice of a world-1 weight that rank R of Wd must hold (rows, columns)."""
    KH, VH, QH, KVH = cfg["gdn_kh"], cfg["gdn_vh"], cfg["att_qh"], cfg["att_kvh"]
    vh, qh, kvh, ffn, H = VH // Wd, QH // Wd, KVH // Wd, cfg["ffn"] // Wd, cfg["hidden"]
    v0, q0, kv0, f0 = R * vh, R * qh, R * kvh, R * ffn
    kh = min(KH, vh)
    hd = np.arange(HD)
    if name == "qkv":
        ks = [(v0 + i) % KH for i in range(kh)]
        rows = np.concatenate([g * HD + hd for g in ks] + [KH * HD + g * HD + hd for g in ks]
                              + [2 * KH * HD + (v0 + i) * HD + hd for i in range(vh)])
        return full[rows]
    if name == "z":
        return full[v0 * HD:(v0 + vh) * HD]
    if name == "ab":
        return full[np.r_[v0:v0 + vh, VH + v0:VH + v0 + vh]]
    if name == "out":
        return full[:, v0 * HD:(v0 + vh) * HD]
    if name == "qg":
        return full[(q0 * 2 * HD):(q0 + qh) * 2 * HD]
    if name == "kv":
        return full[np.r_[kv0 * HD:(kv0 + kvh) * HD, KVH * HD + kv0 * HD:KVH * HD + (kv0 + kvh) * HD]]
    if name == "o":
        return full[:, q0 * HD:(q0 + qh) * HD]
    if name in ("gate", "up"):
        return full[f0:f0 + ffn]
    if name == "down":
        return full[:, f0:f0 + ffn]
    if name == "lm_head":
        V = cfg["vocab"]
        n = V // Wd + (1 if R < V % Wd else 0)
        s = R * (V // Wd) + min(R, V % Wd)
        return full[s:s + n]
    assert H and False, name


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_shards_are_slices_of_the_whole(pkg, cuda, O, world):
    """Every rank draws its shard from the same global matrices: the shard of
    rank R equals the column-/row-parallel slice of the tp_world = 1 model."""
    torch = cuda
    full = Dec(pkg)
    parts = [Dec(pkg, rank=R, world=world) for R in range(world)]
    try:
        for il in [0, 3]:
            names = LINEARS["attn" if is_attn(il) else "gdn"] + LINEARS["ffn"]
            for n in names:
                Wf = O.dequant_g128(*full.linear(torch, il, n))
                for R, p in enumerate(parts):
                    got = O.dequant_g128(*p.linear(torch, il, n))
                    assert np.array_equal(got, _expected_shard(Wf, n, CFG, R, world)), (il, n, R)
        Wf = O.dequant_g128(*full.linear(torch, -1, "lm_head"))
        for R, p in enumerate(parts):
            assert np.array_equal(O.dequant_g128(*p.linear(torch, -1, "lm_head")),
                                  _expected_shard(Wf, "lm_head", CFG, R, world))
        a = full.param(torch, 0, "ssm_a")
        for R, p in enumerate(parts):
            vh = CFG["gdn_vh"] // world
            assert np.array_equal(p.param(torch, 0, "ssm_a"), a[R * vh:(R + 1) * vh])
        # the synthetic prefill draws every state entry by its global index
        for d in [full] + parts:
            assert d.L.dec_prefill_random(d.h, 40, 9) == 0
        KH, VH, KVH = CFG["gdn_kh"], CFG["gdn_vh"], CFG["att_kvh"]
        cg = 2 * KH * HD + VH * HD
        cs = full.param(torch, 0, "conv_state").reshape(3, cg)
        st = full.param(torch, 0, "rec_state").reshape(VH, HD, HD)
        kc = full.param(torch, 3, "kcache", np.float16).reshape(-1, KVH, HD)
        for R, p in enumerate(parts):
            vh, kvh = VH // world, KVH // world
            kh = min(KH, vh)
            ks = [(R * vh + i) % KH for i in range(kh)]
            hd = np.arange(HD)
            chan = np.concatenate([g * HD + hd for g in ks] + [KH * HD + g * HD + hd for g in ks]
                                  + [2 * KH * HD + (R * vh + i) * HD + hd for i in range(vh)])
            assert np.array_equal(p.param(torch, 0, "conv_state").reshape(3, -1), cs[:, chan])
            assert np.array_equal(p.param(torch, 0, "rec_state").reshape(vh, HD, HD), st[R * vh:(R + 1) * vh])
            pk = p.param(torch, 3, "kcache", np.float16).reshape(-1, kvh, HD)
            assert np.array_equal(pk[:40], kc[:40, R * kvh:(R + 1) * kvh])
    finally:
        full.close()
        for p in parts:
            p.close()


def test_decode_step_replays_from_a_cuda_graph(pkg, cuda, O):
    """The position and token live on the device, so one captured step
    replayed K times equals K direct steps."""
    torch = cuda
    a, b = Dec(pkg), Dec(pkg)
    try:
        for d in (a, b):
            assert d.L.dec_prefill_random(d.h, 60, 3) == 0
            assert d.L.dec_set(d.h, 60, 11) == 0
        for _ in range(6):
            a.step(torch)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            b.step(torch)                                  # warm-up (step 1)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            b.step(torch)
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        pa, pb = a.pointers(), b.pointers()
        ha = device_read(torch, pa["hist"], (CFG["max_ctx"],), np.int32)
        hb = device_read(torch, pb["hist"], (CFG["max_ctx"],), np.int32)
        assert np.array_equal(ha[60:66], hb[60:66])
        assert device_read(torch, pb["pos"], (1,), np.int32)[0] == 66
        la = device_read(torch, pa["logits"], (CFG["vocab"],), np.float32)
        lb = device_read(torch, pb["logits"], (CFG["vocab"],), np.float32)
        assert np.array_equal(la, lb)
        del g
    finally:
        a.close()
        b.close()


@pytest.mark.parametrize("world,mode", [(2, "nccl"), (4, "nccl"), (2, "p2p"), (4, "p2p"), (2, "p2p_missing")])
def test_tensor_parallel_decode(cuda, world, mode):
    torch = cuda
    n = torch.cuda.device_count()
    if n < world:
        pytest.skip("needs %d GPUs" % world)
    ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    s = socket.socket(); s.bind(("127.0.0.1", 0)); port = s.getsockname()[1]; s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", DEC_TP_MODE=mode)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "dec_tp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "DEC_TP_OK" in r.stdout
