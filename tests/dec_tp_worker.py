"""Rank process for tests/test_dec_gpu.py (launched by torchrun, one per GPU).

Tensor-parallel decode: every rank builds its shard of the same model
(dec_create with tp_rank / tp_world), rank 0's NCCL id reaches the others over
a gloo group, and all ranks step the same tokens; the row-parallel blocks sum
inside dec_step -- over NCCL (DEC_TP_MODE=nccl) or through peer memory
(DEC_TP_MODE=p2p, handles all-gathered over gloo) -- and the
vocabulary-sharded argmax keys are all-gathered.  DEC_TP_MODE=p2p_missing:
rank 1 never steps, and rank 0's bounded waits must run out and be reported
by dec_status (the failure is made on the host; no GPU hangs or faults).  Rank 0 also runs the unsharded model on its GPU and checks that
the gathered logits agree within 1e-3 of the largest |logit| and that the
tokens agree wherever the top-2 margin exceeds that.  Exits 0 on success.
"""
import ctypes as C
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

STEPS = 4
PREFILL = 100


def run(pkg, torch, dec, steps):
    p = dec.pointers()
    out = []
    for _ in range(steps):
        dec.step(torch)
        torch.cuda.synchronize()
        lg = dec_read(torch, p["logits"], p["vn"])
        out.append(lg)
    from conftest import device_read
    hist = device_read(torch, p["hist"], (dec.cfg["max_ctx"],), np.int32)
    return out, hist[PREFILL:PREFILL + steps], p["v0"]


def dec_read(torch, ptr, n):
    from conftest import device_read
    return device_read(torch, ptr, (n,), np.float32).astype(np.float64)


def main():
    import torch
    import torch.distributed as dist
    from conftest import load_package
    from test_dec_gpu import CFG, TOL, Dec
    pkg = load_package()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    L = pkg.declib()
    uid = (C.c_uint8 * 128)()
    if rank == 0:
        assert L.dec_nccl_unique_id(uid) == 0
    t = torch.tensor(list(bytes(uid)), dtype=torch.uint8)
    dist.broadcast(t, 0)
    uid = (C.c_uint8 * 128)(*t.tolist())
    d = Dec(pkg, device=rank, rank=rank, world=world)
    assert L.dec_tp_init(d.h, uid) == 0
    mode = os.environ.get("DEC_TP_MODE", "nccl")
    if mode.startswith("p2p"):
        hnd = (C.c_uint8 * 64)()
        assert L.dec_p2p_handle(d.h, hnd) == 0
        allh = [None] * world
        dist.all_gather_object(allh, bytes(hnd))
        buf = (C.c_uint8 * (64 * world))(*b"".join(allh))
        assert L.dec_p2p_open(d.h, buf, 20000 if mode == "p2p_missing" else 0) == 0
    if mode == "p2p_missing":
        # rank 1 never steps: rank 0's bounded waits run out and say so
        ok = True
        if rank == 0:
            assert L.dec_prefill_random(d.h, PREFILL, 5) == 0
            assert L.dec_set(d.h, PREFILL, 7) == 0
            d.step(torch)
            torch.cuda.synchronize()
            fl = C.c_int32(0)
            assert L.dec_status(d.h, C.byref(fl)) == 0
            print("flags", fl.value)
            ok = fl.value == 3
            assert L.dec_status(d.h, C.byref(fl)) == 0 and fl.value == 0          # cleared
        dist.barrier()                          # rank 1 keeps its memory mapped until rank 0 is done
        d.close()
        flag = torch.tensor([1 if ok else 0])
        dist.broadcast(flag, 0)
        dist.destroy_process_group()
        if rank == 0 and ok:
            print("DEC_TP_OK")
        sys.exit(0 if int(flag.item()) else 1)
    assert L.dec_prefill_random(d.h, PREFILL, 5) == 0
    assert L.dec_set(d.h, PREFILL, 7) == 0
    logits, hist, v0 = run(pkg, torch, d, STEPS)
    parts = [None] * world
    dist.all_gather_object(parts, (v0, [l.tolist() for l in logits], hist.tolist()))
    ok = True
    if rank == 0:
        full = Dec(pkg, device=0)
        assert L.dec_prefill_random(full.h, PREFILL, 5) == 0
        assert L.dec_set(full.h, PREFILL, 7) == 0
        flog, fhist, _ = run(pkg, torch, full, STEPS)
        parts.sort(key=lambda p: p[0])
        for s in range(STEPS):
            lg = np.concatenate([np.array(p[1][s]) for p in parts])
            err = np.max(np.abs(lg - flog[s])) / np.max(np.abs(flog[s]))
            print("step", s, "rel", err, "tok", parts[0][2][s], fhist[s])
            if err > TOL:
                ok = False
            if any(p[2][s] != parts[0][2][s] for p in parts):
                ok = False
            top2 = np.sort(flog[s])[-2:]
            if parts[0][2][s] != fhist[s]:
                if top2[1] - top2[0] > TOL * np.max(np.abs(flog[s])):
                    ok = False
                break                       # the inputs diverge from here on
        full.close()
    if mode == "p2p":
        fl = C.c_int32(0)
        assert L.dec_status(d.h, C.byref(fl)) == 0
        ok = ok and fl.value == 0
    d.close()
    flag = torch.tensor([1 if ok else 0])
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    if rank == 0 and ok:
        print("DEC_TP_OK")
    sys.exit(0 if int(flag.item()) else 1)


if __name__ == "__main__":
    main()
