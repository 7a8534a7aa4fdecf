"""BASELINE config 2 at exactly its shape: one DeltaNet block and one
gated-attention block at hidden 2048 (16/16 DeltaNet heads and 16 query / 2 KV
attention heads, head dim 128, SwiGLU 6144, INT4 g128 linears, RoPE 1e6),
the KV cache pre-filled to 4096 positions, batch 1 -- stepped through the C
ABI and compared with the float64 oracle of ref/run9b.c (oracle/dec_oracle.py)
layer by layer from identical inputs, with the tolerance of
tests/test_dec_gpu.py (1e-3 of the largest magnitude per layer output and the
logits; states within 1e-3)."""
import numpy as np
import pytest

from conftest import device_read
from test_dec_gpu import Dec, check_step, is_attn, oracle_from, rel, sync_states, TOL, HD

pytestmark = pytest.mark.gpu

CFG2 = dict(hidden=2048, n_layers=2, attn_every=2, vocab=2048, ffn=6144, gdn_kh=16, gdn_vh=16, gdn_hd=128,
            att_qh=16, att_kvh=2, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=4096 + 64)


@pytest.fixture(scope="module")
def O():
    from oracle import dec_oracle
    return dec_oracle


def test_config2_blocks_match_oracle(pkg, cuda, O):
    torch = cuda
    d = Dec(pkg, cfg=CFG2, seed=2)
    try:
        assert d.L.dec_prefill_random(d.h, 4096, 5) == 0
        tok, pos = 11, 4096
        assert d.L.dec_set(d.h, pos, tok) == 0
        M = oracle_from(d, torch, O)
        kc = M.S[1, "kcache"][:4096]
        assert abs(kc.std() - 1.0) < 0.05 and abs(kc.mean()) < 0.05      # N(0,1) pre-fill
        ptrs = d.pointers()
        d.seams_on(torch)
        for s in range(3):
            sync_states(d, torch, M)
            d.step(torch)
            lg = device_read(torch, ptrs["logits"], (CFG2["vocab"],), np.float32).astype(np.float64)
            check_step(O, M, d.seams(torch), lg, tok, pos)
            hist = device_read(torch, ptrs["hist"], (CFG2["max_ctx"],), np.int32)
            assert hist[pos] == int(np.argmax(lg))
            tok = int(hist[pos])
            pos += 1
        st = d.param(torch, 0, "rec_state").astype(np.float64).reshape(M.S[0, "rec_state"].shape)
        assert rel(st, M.S[0, "rec_state"]) <= TOL
        kc = d.param(torch, 1, "kcache", np.float16).astype(np.float64).reshape(-1, CFG2["att_kvh"], HD)
        assert rel(kc[:pos], M.S[1, "kcache"][:pos]) <= TOL
        assert is_attn(1, CFG2) and not is_attn(0, CFG2)
    finally:
        d.close()
