"""The allocation-free launch (mv4i_launch_noalloc) against the ordinary one.

mv4i_launch_noalloc serves callers that cannot allocate device memory on
their decode path -- a runtime that has already divided HBM between weights,
caches and state, a loop that cannot take cudaMalloc's synchronisation, or a
foreign-language host with no device allocator.  Its counters live in a fixed
array inside the library instead of caller scratch.  This test runs the same
golden-mode job list through both entry points, twice in a row through the
allocation-free one (its array keeps the previous call's contents), and
requires identical outputs and statuses.  It allocates its own test buffers
with torch; the entry point under test allocates nothing.

Kept in its own file, collected last, so that a failure here comes after
every other test has run.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KEYS = ["emit0", "emit13", "emit20", "lin0", "lin1", "lin2", "sat0"]


def _img(golden, k):
    meta = golden[k + "_meta"]
    if k.startswith("emit"):
        return golden["img%d" % meta[12]].tobytes()
    return golden[k + "_img"].tobytes()


def _setup(torch, pkg, golden):
    L = pkg.lib()
    mats, jobs, outs = [], [], []
    status = torch.zeros((len(KEYS), 8), dtype=torch.int32, device="cuda")
    for i, k in enumerate(KEYS):
        m = [int(v) for v in golden[k + "_meta"]]
        pi = pkg.ParsedImage(_img(golden, k))
        dm = pkg.DMat()
        assert L.mv4i_dmat_upload(C.byref(pi.f), 0, C.byref(dm)) == 0
        mats.append((pi, dm))
        nr, nc, mode = m[5], m[6], m[7]
        x = torch.from_numpy(golden[k + "_x"].copy()).cuda()
        yd = torch.zeros(nr, dtype=torch.int32, device="cuda")
        ym = torch.zeros(nr, dtype=torch.int16, device="cuda")
        ya = torch.zeros(nr, dtype=torch.int64, device="cuda")
        outs.append((x, yd, ym, ya))
        j = pkg.Job()
        j.w = C.pointer(dm)
        j.x = x.data_ptr(); j.x_exp = m[4]; j.n_rows = nr; j.n_cols = nc; j.mode = mode; j.nvec = 1
        j.y_data = yd.data_ptr(); j.y_mant = ym.data_ptr(); j.y_acc = ya.data_ptr()
        j.status = status[i].data_ptr()
        jobs.append(j)
    return L, mats, (pkg.Job * len(jobs))(*jobs), outs, status


def _results(torch, outs, status):
    torch.cuda.synchronize()
    return [tuple(t.cpu().numpy().copy() for t in o[1:]) for o in outs], status.cpu().numpy().copy()


def test_noalloc_matches_launch_twice(cuda, pkg, golden):
    torch = cuda
    L, mats, arr, outs, status = _setup(torch, pkg, golden)
    n = len(KEYS)
    scratch = torch.zeros(L.mv4i_scratch_bytes(), dtype=torch.uint8, device="cuda")
    assert L.mv4i_launch(arr, n, C.c_void_p(scratch.data_ptr()), None) == 0
    want, want_st = _results(torch, outs, status)
    # the reference-produced fixtures agree with the ordinary launch
    for i, k in enumerate(KEYS):
        mode = int(golden[k + "_meta"][7])
        got = want[i][2] if mode == 2 else (want[i][1] if mode == 0 else want[i][0])
        assert np.array_equal(got.astype(np.int64), golden[k + "_y"]), k
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for call in range(2):
        for o in outs:
            for t in o[1:]:
                t.fill_(0)
        status.fill_(0)
        assert L.mv4i_launch_noalloc(arr, n, None) == 0, call
        got, got_st = _results(torch, outs, status)
        for i in range(n):
            for a, b in zip(want[i], got[i]):
                assert np.array_equal(a, b), (call, KEYS[i])
        assert np.array_equal(want_st, got_st), call
    # the entry point allocated nothing: the device's free memory is unchanged
    # across both calls (torch's own caching allocator is not involved: every
    # test buffer above existed before the first call)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0
    for _, dm in mats:
        L.mv4i_dmat_free(C.byref(dm))


def test_noalloc_refuses_more_jobs_than_its_array(cuda, pkg, golden):
    torch = cuda
    L, mats, arr, outs, status = _setup(torch, pkg, golden)
    many = (pkg.Job * 65)(*([arr[0]] * 65))
    assert L.mv4i_launch_noalloc(many, 65, None) == -14
    for _, dm in mats:
        L.mv4i_dmat_free(C.byref(dm))
