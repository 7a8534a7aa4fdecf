"""Input staging modes of the launch-mode decode step (include/dec_b200.h
dec_set_prestage): staging each matvec's inputs once in a launch of their
own (mode 1 for batches, the default; mode 2 for every step) or in every CTA
of the matvec (mode 0) runs the same arithmetic, so logits and tokens are
bit-identical across modes, step after step.
"""
import numpy as np
import pytest

from conftest import device_read
from test_dec_gpu import CFG, Dec
from test_dec_persistent_gpu import CFG_WIDE, logits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,nb,prefill", [(CFG, 1, 50), (CFG, 3, 40), (CFG_WIDE, 8, 100)])
def test_prestage_modes_are_bit_identical(pkg, cuda, cfg, nb, prefill):
    torch = cuda
    c = dict(cfg, batch=nb)
    ds = [Dec(pkg, cfg=c, seed=11) for _ in range(3)]
    try:
        for mode, d in enumerate(ds):
            assert d.L.dec_set_prestage(d.h, mode) == 0
            assert d.L.dec_prefill_random(d.h, prefill, 5) == 0
            assert d.L.dec_set(d.h, prefill, 23) == 0
        assert ds[0].L.dec_set_prestage(ds[0].h, 3) == -11
        for step in range(4):
            for d in ds:
                d.step(torch)
            torch.cuda.synchronize()
            lg = [logits(d, torch, nb) for d in ds]
            hs = [device_read(torch, d.pointers()["hist"], (nb, c["max_ctx"]), np.int32)[:, prefill + step] for d in ds]
            for mode in (1, 2):
                assert np.array_equal(lg[0], lg[mode]), (step, mode)
                assert np.array_equal(hs[0], hs[mode]), (step, mode)
    finally:
        for d in ds:
            d.close()
