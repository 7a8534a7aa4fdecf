#!/usr/bin/env python
"""Benchmark of the INT4 streaming matvec (llm.vhdl subsystem A) on B200.

Workload (streamed): a stack of G = 64 distinct
4096 x 4096 matrices in the benchmark format (signed INT4 uniform in [-8,7],
fp16 scale per 128 columns in [0.002, 0.02], x fp16 ~ N(0,1), y fp16, fp32
accumulation), seeded splitmix64 synthetic data (seed 0 + matrix index, one
disjoint range per rank).  One step = one launch of the 64-job list, i.e. 64
config-0 matvecs; 555 MB of weights per step is larger than the 126 MB L2, so
no flush is needed between steps.

Printed JSON line (rank 0):
  value      HBM GB/s of algorithmic bytes (8,667,136 B per matvec), whole job
  e2e        the same metric through mv4i_g128_matvec_host with pinned HOST
             x / y, copies inside the timed region
  roofline   the g128 kernel: achieved GB/s vs the measured copy bandwidth
  cpu_baseline  the reference's mv4i_matvec (compiled from its C source) on the
             box's cores, golden mode, config 0 (bounded sample)
  golden     the same stack in the reference's bit-exact golden format
             (uint15 scale per 32 columns, int16 BFP x, BFP output)
  single     one 4096x4096 matvec per launch, rotating over the 64 matrices

`--impl reference` times the reference's CPU mv4i_matvec instead (rank 0 only).
"""
import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = K = 4096
G128_BYTES = M * K // 2 + M * (K // 128) * 2 + K * 2 + M * 2        # 8,667,136
GOLDEN_BYTES = M * K // 2 + M * (K // 32) * 2 + K * 2 + M * 2       # 9,453,568
METRIC = "INT4 matvec HBM GB/s (% of peak) and decode tokens/s at 1/2/4/8 B200"
FALLBACK_HBM = 6650.0


def load_pkg():
    import importlib.util
    if "llmvhdl_b200" in sys.modules:
        return sys.modules["llmvhdl_b200"]
    d = os.path.join(ROOT, "llm.vhdl_b200")
    spec = importlib.util.spec_from_file_location(
        "llmvhdl_b200", os.path.join(d, "__init__.py"), submodule_search_locations=[d])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmvhdl_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM, "fallback"


def profiled_traffic(name, key):
    """dram read+write bytes per launch recorded from an ncu capture summary
    in profiles/<name> (line '<key>: <bytes> ...')."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith(key + ":"):
            return float(ln.split(":")[1].split()[0])
    return None


class Clocks:
    """Samples SM clock and clock-event reasons through NVML every 2 ms on a
    thread while the timed region runs (read-only)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, torch_dev):
        self.samples, self.reasons, self.ok = [], 0, False
        try:
            import pynvml as N
            N.nvmlInit()
            bus = torch_dev_bus(torch_dev)
            self.h = N.nvmlDeviceGetHandleByPciBusId(bus) if bus else N.nvmlDeviceGetHandleByIndex(0)
            self.N = N
            self.max = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = str(e)

    def _run(self):
        N = self.N
        while not self.stop:
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                self.reasons |= N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def __enter__(self):
        self.stop = False
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop = True
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": getattr(self, "max", None), "reasons": [],
                    "note": getattr(self, "err", "no samples")}
        rs = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max, "reasons": rs,
                "samples": len(self.samples)}


def torch_dev_bus(dev):
    import torch
    try:
        p = torch.cuda.get_device_properties(dev)
        return "%08X:%02X:%02X.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
    except Exception:  # noqa: BLE001
        return None


def cpu_baseline(budget_s=3.0):
    from oracle import cpu_baseline as CB
    steps, kind, P = CB.run(budget_s=budget_s)
    t = steps[0]
    one, _, _ = CB.run(P=1, budget_s=2.0)
    return {"value": round(CB.GOLDEN_BYTES / t / 1e9, 4), "unit": "GB/s", "cores": P,
            "kind": kind, "ms_per_matvec": round(t * 1e3, 3),
            "sample": "config-0 golden-mode mv4i_matvec (BFP out), %d processes x row shards, "
                      "~%.0f s each" % (P, budget_s),
            "single_thread": {"ms_per_matvec": round(one[0] * 1e3, 3),
                              "GBps": round(CB.GOLDEN_BYTES / one[0] / 1e9, 4), "cores": 1, "kind": kind,
                              "sample": "the whole 4096 x 4096 matvec in one process, ~2 s"}}


def block_cpu_baseline(budget_s=2.0):
    """The reference's own fixed-point gdn_block_token (ref/gdn_block_vec.c:208,
    compiled from source into oracle/_ref/libref_gdn.so) on the bench's block
    stimulus, one thread; the restatement when the reference was not built."""
    import numpy as np
    import oracle as O
    b = block_inputs(1)
    use_ref = O.have_gdn_ref()
    T = 0
    smem, semem = b["smem"].copy(), b["semem"].copy()
    e_t = np.array([[8 + (s + k) % 5 for k in range(4)] for s in range(3)], np.int32)
    stim = dict(wtap=b["wtap"], cw_exp=np.array([11, 12, 13], np.int32), wm=b["wm"], w_e=12, z_e=12)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s or T == 0:
        n = 4
        stim.update(xtap=np.repeat(b["xtap"][None], n, 0), e_t=np.repeat(e_t[None], n, 0),
                    tvalid=np.ones((n, 3, 4), np.int32), sc=np.repeat(b["sc"][None], n, 0),
                    zm=np.repeat(b["zm"][None], n, 0), tk0=np.zeros(n, np.int32))
        O.gdn_block_run(BLK_KH, BLK_VH, BLK_D, stim, smem, semem, use_ref=use_ref)
        T += n
    us = (time.perf_counter() - t0) / T * 1e6
    return {"us_per_token": round(us, 1), "cores": 1, "kind": "reference" if use_ref else "port",
            "sample": "%d block tokens at 16/32 heads x 128, one thread" % T}


# --------------------------------------------------------------------- ours

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    pkg = load_pkg()
    L = pkg.lib()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    G = args.stack
    seed = rank * G
    stream = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(stream.cuda_stream)

    def vp(t):
        return C.c_void_p(t.data_ptr())

    wq = torch.empty((G, M, K // 2), dtype=torch.uint8, device=dev)
    sc = torch.empty((G, M, K // 128), dtype=torch.float16, device=dev)
    x = torch.empty((G, K), dtype=torch.float16, device=dev)
    y16 = torch.empty((G, M), dtype=torch.float16, device=dev)
    assert L.mv4i_synth_g128(seed, G, M, K, vp(wq), vp(sc), vp(x), sp) == 0
    mats = (pkg.DMat * G)()
    jobs = (pkg.Job * G)()
    for i in range(G):
        assert L.mv4i_dmat_wrap_g128(vp(wq[i]), K // 2, vp(sc[i]), K // 128, M, K, local_rank,
                                     C.byref(mats[i])) == 0
        j = jobs[i]
        j.w = C.pointer(mats[i]); j.x = x[i].data_ptr(); j.n_rows = M; j.n_cols = K; j.nvec = 1
        j.y_f16 = y16[i].data_ptr()

    def launch(js=jobs, n=G, scratch=None):
        rc = L.mv4i_launch(js, n, scratch, sp)
        if rc:
            raise RuntimeError("mv4i_launch failed: %d (cuda %d)" % (rc, L.mv4i_last_cuda_error()))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(fn, steps):
        """Run fn() `steps` times between events on `stream`; max over ranks."""
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        barrier()
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # --- headline: the g128 stack
    for _ in range(args.warmup):
        launch()
    clk = Clocks(local_rank)
    with clk:
        ms = timed(launch, args.steps)
    ms_step = ms / args.steps
    value = world * G * G128_BYTES / (ms_step * 1e-3) / 1e9

    # --- golden-mode stack: same nibbles, uint15 scales per 32 columns, BFP x
    gsc = torch.repeat_interleave((sc.float() * 2.0 ** 20).round().to(torch.int16), 4, dim=2).contiguous()
    xm = torch.empty((G, K), dtype=torch.int16, device=dev)
    xe = torch.empty(G, dtype=torch.int32, device=dev)
    assert L.mv4i_bfp_pack(vp(x), 0, K, G, K, vp(xm), vp(xe), sp) == 0
    cb = (C.c_int8 * 16)(*[i if i < 8 else i - 16 for i in range(16)])
    gmats = (pkg.DMat * G)()
    gjobs = (pkg.Job * G)()
    yd = torch.empty((G, M), dtype=torch.int32, device=dev)
    ym = torch.empty((G, M), dtype=torch.int16, device=dev)
    st = torch.zeros((G, 8), dtype=torch.int32, device=dev)
    scratch = torch.zeros(L.mv4i_scratch_bytes(), dtype=torch.uint8, device=dev)
    for i in range(G):
        assert L.mv4i_dmat_wrap_golden(vp(wq[i]), K // 2, vp(gsc[i]), K // 32, M, K, 5, 3, cb,
                                       local_rank, C.byref(gmats[i])) == 0
        j = gjobs[i]
        j.w = C.pointer(gmats[i]); j.x = xm[i].data_ptr(); j.d_x_exp = xe[i].data_ptr()
        j.n_rows = M; j.n_cols = K; j.mode = 0; j.nvec = 1
        j.y_data = yd[i].data_ptr(); j.y_mant = ym[i].data_ptr(); j.status = st[i].data_ptr()
    gscr = vp(scratch)
    for _ in range(args.warmup):
        launch(gjobs, G, gscr)
    gsteps = max(10, args.steps // 2)
    gms = timed(lambda: launch(gjobs, G, gscr), gsteps) / gsteps
    gvalue = world * G * GOLDEN_BYTES / (gms * 1e-3) / 1e9
    assert int(st[:, 4].abs().sum().item()) == 0

    # --- one matvec per launch, rotating over the stack (cold L2 each time),
    # the G launches captured in one CUDA graph as a decode loop would be
    def singles():
        for i in range(G):
            rc = L.mv4i_launch(C.byref(jobs[i]), 1, None, sp)
            if rc:
                raise RuntimeError("single launch failed %d" % rc)
    singles()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        singles()
    for _ in range(3):
        graph.replay()
    nrep = max(3, args.steps // 10)
    sms = timed(graph.replay, nrep) / nrep / G
    del graph

    # --- end to end through the host-buffer entry point
    hx = torch.empty((G, K), dtype=torch.float16).pin_memory()
    hx.copy_(x.cpu())
    hy = torch.empty((G, M), dtype=torch.float16).pin_memory()

    def e2e_call():
        rc = L.mv4i_g128_matvec_host(mats, G, C.c_void_p(hx.data_ptr()), C.c_void_p(hy.data_ptr()), sp)
        if rc:
            raise RuntimeError("mv4i_g128_matvec_host failed %d" % rc)
    for _ in range(3):
        e2e_call()
    esteps = max(10, args.steps // 4)
    ems = timed(e2e_call, esteps) / esteps
    e2e_value = world * G * G128_BYTES / (ems * 1e-3) / 1e9
    assert torch.equal(hy.to(dev), y16), "host-buffer result differs from the device launch"

    gdn = run_gdn(args, pkg, L, torch, dev, stream, sp, timed)
    dec = run_decode(args, pkg, torch, dev, stream, sp, timed, rank, world, local_rank)

    peak, peak_kind = peaks()
    achieved = G * G128_BYTES / (ms_step * 1e-3) / 1e9
    traffic = profiled_traffic("mv4i_g128_stack16.txt", "traffic_bytes_per_launch_stack64") if G == 64 else None
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4 x fp16 (fp32 accumulate)",
        "data": "synthetic (splitmix64 seeds, config-0 distributions)",
        "config": {"workload": "config 0: 64 x [4096x4096 INT4 g128 fp16-scale matvec, batch 1] per step",
                   "stack": G, "M": M, "K": K, "group": 128, "parallelism": "replica%d" % world,
                   "l2": "inputs 555 MB/step per GPU > 126 MB L2 (no flush)"},
        "percent_of_peak": round(100.0 * achieved / peak, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind + " copy bandwidth",
                     "traffic": traffic,
                     "kernel": "mv4i_kernel<G128>", "bytes_per_launch": G * G128_BYTES},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s",
                "h2d_bytes_per_step": G * K * 2, "d2h_bytes_per_step": G * M * 2,
                "call": "mv4i_g128_matvec_host (pinned host x/y)", "ms_per_step": round(ems, 4)},
        "golden": {"value": round(gvalue, 1), "unit": "GB/s", "ms_per_step": round(gms, 5),
                   "bytes_per_matvec": GOLDEN_BYTES, "frac": round(gvalue / world / peak, 4),
                   "mode": "BFP out, linear codebook, bit-exact with ref/matvec_int4.c"},
        "single": {"us_per_matvec": round(sms * 1e3, 2),
                   "GBps": round(G128_BYTES / (sms * 1e-3) / 1e9, 1),
                   "how": "64 one-job launches in a CUDA graph, rotating over the stack"},
        "gdn": gdn,
        "decode": dec,
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    return out


# ------------------------------------------------------------ config 1

GDN_H, GDN_D, GDN_T = 16, 128, 256
# per step, state in HBM: S read + written (2 x 1 MiB fp32), q, k, v (fp16),
# a, b (fp32), gate (fp16), out (fp16)
GDN_STEP_BYTES = 2 * GDN_H * GDN_D * GDN_D * 4 + 3 * GDN_H * GDN_D * 2 + 2 * GDN_H * 4 \
    + GDN_H * GDN_D * 2 + GDN_H * GDN_D * 2


def gdn_inputs(seed=1):
    """Config 1: q, k, v, g fp16 ~ N(0,1); a, b ~ N(0,1); S0 ~ N(0, 0.02)."""
    import numpy as np
    import importlib.util
    spec = importlib.util.spec_from_file_location("synth", os.path.join(ROOT, "llm.vhdl_b200", "synth.py"))
    S = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(S)
    n = GDN_T * GDN_H * GDN_D
    key = 3 * seed
    q = S.normal_f16(key + 100, n).reshape(GDN_T, GDN_H, GDN_D)
    k = S.normal_f16(key + 101, n).reshape(GDN_T, GDN_H, GDN_D)
    v = S.normal_f16(key + 102, n).reshape(GDN_T, GDN_H, GDN_D)
    g = S.normal_f16(key + 103, n).reshape(GDN_T, GDN_H, GDN_D)
    a = S.normal_f16(key + 104, GDN_T * GDN_H).astype(np.float32).reshape(GDN_T, GDN_H)
    b = S.normal_f16(key + 105, GDN_T * GDN_H).astype(np.float32).reshape(GDN_T, GDN_H)
    s0 = (S.normal_f16(key + 106, GDN_H * GDN_D * GDN_D).astype(np.float32) * 0.02).reshape(GDN_H, GDN_D, GDN_D)
    return s0, q, k, v, g, a, b


def run_gdn(args, pkg, L, torch, dev, stream, sp, timed):
    """Config 1 two ways: (1) one launch of all 256 steps with the state on
    chip; (2) one launch per step, the state read and written through HBM
    each step, 256 launches captured in a CUDA graph (a decode loop)."""
    s0, q, k, v, g, a, b = gdn_inputs(1)
    t = {n: torch.from_numpy(x.copy()).to(dev) for n, x in dict(q=q, k=k, v=v, g=g, a=a, b=b).items()}
    S = torch.from_numpy(s0.copy()).to(dev)
    out = torch.empty((GDN_T, GDN_H, GDN_D), dtype=torch.float16, device=dev)
    full = pkg.GdnF32(GDN_T, GDN_H, GDN_H, GDN_D, S.data_ptr(), t["q"].data_ptr(), t["k"].data_ptr(),
                      t["v"].data_ptr(), t["g"].data_ptr(), t["a"].data_ptr(), t["b"].data_ptr(), 1, 1.0,
                      None, out.data_ptr())

    def run_all():
        if L.gdn_run_f32(C.byref(full), sp):
            raise RuntimeError("gdn_run_f32 failed")
    for _ in range(3):
        run_all()
    nrep = max(3, args.steps // 50)
    ms_all = timed(run_all, nrep) / nrep

    steps = []
    for i in range(GDN_T):
        steps.append(pkg.GdnF32(1, GDN_H, GDN_H, GDN_D, S.data_ptr(), t["q"][i].data_ptr(),
                                t["k"][i].data_ptr(), t["v"][i].data_ptr(), t["g"][i].data_ptr(),
                                t["a"][i].data_ptr(), t["b"][i].data_ptr(), 1, 1.0, None,
                                out[i].data_ptr()))

    def run_steps():
        for st in steps:
            if L.gdn_run_f32(C.byref(st), sp):
                raise RuntimeError("gdn_run_f32 failed")
    run_steps()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        run_steps()
    for _ in range(3):
        graph.replay()
    ms_steps = timed(graph.replay, nrep) / nrep
    del graph
    us_step = ms_steps * 1e3 / GDN_T
    blk = run_block(pkg, L, torch, dev, stream, sp, timed, nrep)
    return {
        "workload": "config 1: 16 heads x 128 x 128 fp32 state, 256 sequential steps, seed 1",
        "persistent_us_per_step": round(ms_all * 1e3 / GDN_T, 3),
        "persistent_ms_per_256": round(ms_all, 4),
        "per_step_us": round(us_step, 3),
        "per_step_GBps": round(GDN_STEP_BYTES / (us_step * 1e-6) / 1e9, 1),
        "per_step_bytes": GDN_STEP_BYTES,
        "per_step_how": "one launch per step, state through HBM, 256 launches in a CUDA graph",
        "kernel": "gdn_f32_kernel",
        "fixed_block": blk,
    }


BLK_KH, BLK_VH, BLK_D = 16, 32, 128


def block_inputs(seed=1):
    """Fixed-point DeltaNet block stimulus at the model shape (16 key heads, 32
    value heads, D 128), in the ranges of the reference's generator
    (ref/gdn_block_vec.c:570-618): conv taps/weights +-2047, norm weights
    2000..6000, the scalar path in its physical band, z +-8192, state mantissas
    up to full scale with column exponents 9..12."""
    import numpy as np
    rng = np.random.default_rng(seed)
    KH, VH, D = BLK_KH, BLK_VH, BLK_D
    CH = 2 * KH * D + VH * D
    sc = np.zeros((VH, 8), np.int32)
    sc[:, 0] = rng.integers(-1000, 1001, VH); sc[:, 1] = 14
    sc[:, 2] = -rng.integers(2000, 32001, VH); sc[:, 3] = 12
    sc[:, 4] = -rng.integers(1, 3001, VH); sc[:, 5] = 16
    sc[:, 6] = rng.integers(-30000, 30001, VH); sc[:, 7] = 12
    return dict(xtap=rng.integers(-2047, 2048, (CH, 4)).astype(np.int16),
                wtap=rng.integers(-2047, 2048, (CH, 4)).astype(np.int16), sc=sc,
                zm=rng.integers(-8192, 8193, (VH, D)).astype(np.int16),
                wm=rng.integers(2000, 6001, D).astype(np.int16),
                smem=rng.integers(-30000, 30001, (VH, D, D)).astype(np.int16),
                semem=(9 + (np.arange(VH)[:, None] + np.arange(D)[None]) % 4).astype(np.int32))


BLK_BYTES = 2 * BLK_VH * BLK_D * BLK_D * 2 + 2 * BLK_VH * BLK_D * 4 + (2 * BLK_KH + BLK_VH) * BLK_D * 4 * 2 * 2


def run_block(pkg, L, torch, dev, stream, sp, timed, nrep):
    """The fixed-point block (deltanet_step) per token at the model shape:
    64 tokens per CUDA graph, each a programmatic dependent of the one before,
    the state resident in HBM (read and written every token)."""
    b = block_inputs(1)
    t = {n: torch.from_numpy(x.copy()).to(dev) for n, x in b.items()}
    y = torch.empty(BLK_VH * BLK_D, dtype=torch.int16, device=dev)
    status = torch.zeros(8, dtype=torch.int32, device=dev)
    nb = L.deltanet_work_bytes(BLK_KH, BLK_VH, BLK_D)
    work = torch.empty(nb + 256, dtype=torch.uint8, device=dev)
    a = pkg.DeltanetArgs()
    a.KH, a.VH, a.D = BLK_KH, BLK_VH, BLK_D
    a.xtap, a.wtap, a.sc, a.zm, a.wm = (t[k].data_ptr() for k in ("xtap", "wtap", "sc", "zm", "wm"))
    for s in range(3):
        a.cw_exp[s] = 11 + s
        for k in range(4):
            a.e_t[s][k] = 8 + (s + k) % 5
            a.tvalid[s][k] = 1
    a.w_e, a.z_e, a.tk0 = 12, 12, 0
    a.smem, a.semem, a.y, a.status = t["smem"].data_ptr(), t["semem"].data_ptr(), y.data_ptr(), status.data_ptr()
    a.work = (work.data_ptr() + 255) & ~255
    a.pdl = 1
    T = 64

    def tokens():
        for _ in range(T):
            if L.deltanet_step(C.byref(a), sp):
                raise RuntimeError("deltanet_step failed")
    tokens()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        tokens()
    for _ in range(3):
        g.replay()
    ms = timed(g.replay, nrep) / nrep
    del g
    us = ms * 1e3 / T
    peak, _ = peaks()
    return {"workload": "fixed-point DeltaNet block token (bit-exact with gdn_block_token): 16 key / 32 value "
                        "heads, D 128, int16 state 1 MiB read + written per token",
            "us_per_token": round(us, 3), "bytes_per_token": BLK_BYTES,
            "GBps": round(BLK_BYTES / (us * 1e-6) / 1e9, 1),
            "frac_hbm": round(BLK_BYTES / (us * 1e-6) / 1e9 / peak, 4),
            "how": "2 launches per token (head kernel: D/32 CTAs per value head in clusters; site-13 kernel "
                   "from the head records), 64 tokens per CUDA graph",
            "kernels": ["gdn_blk_head_kernel<128>", "gdn_blk_site13_kernel"]}


# ------------------------------------------------------------ decode (configs 3, 4)

DEC_C3 = dict(hidden=2048, n_layers=24, attn_every=4, vocab=151936, ffn=6144, gdn_kh=16, gdn_vh=16, gdn_hd=128,
              att_qh=16, att_kvh=2, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=1024)
DEC_C2 = dict(hidden=2048, n_layers=2, attn_every=2, vocab=2048, ffn=6144, gdn_kh=16, gdn_vh=16, gdn_hd=128,
              att_qh=16, att_kvh=2, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=4096 + 512)
DEC_C4 = dict(hidden=5120, n_layers=48, attn_every=4, vocab=151936, ffn=17408, gdn_kh=32, gdn_vh=32, gdn_hd=128,
              att_qh=40, att_kvh=8, att_hd=128, n_rot=32, rope_theta=1.0e6, rms_eps=1e-6, max_ctx=8192 + 512)


class _DevArray:
    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 2, "strides": None}


def run_decode(args, pkg, torch, dev, stream, sp, timed, rank, world, local_rank):
    """Decode tokens/s through include/dec_b200.h, one step per CUDA-graph
    replay.  Config 3 (1 GPU): 512-token random-id prompt fed through the
    decode step, then 256 greedy tokens, at batch 1 and batch 8.  Config 4: tensor parallel
    over the `world` ranks (NCCL all-reduce per row-parallel block), KV
    context pre-filled to 8192 with N(0,1), batch 1."""
    import numpy as np
    D = pkg.declib()
    out = {}

    def create(cfg, seed, R, W):
        h = C.c_void_p()
        rc = D.dec_create(C.byref(pkg.DecConfig(**cfg)), seed, local_rank, R, W, C.byref(h))
        if rc:
            raise RuntimeError("dec_create failed %d (cuda %d)" % (rc, pkg.lib().mv4i_last_cuda_error()))
        return h

    def step_fn(h):
        def f():
            rc = D.dec_step(h, sp)
            if rc:
                raise RuntimeError("dec_step failed %d" % rc)
        return f

    def layer_profile(h, cfg, reps=1):
        """One step timed layer by layer: per-layer time and the fraction of
        the HBM peak its bytes reach (DeltaNet / attention layers and the LM
        head, averaged by kind).  The persistent step stamps the GPU global
        timer after every grid barrier (dec_set_clock); the launch-mode step
        records an event after every layer (events between kernels stop
        programmatic launches from overlapping layer boundaries, so those
        fractions are a little below the graph-replay rate)."""
        peak, _ = peaks()
        nl = cfg["n_layers"]
        lb = [D.dec_layer_bytes(h, il) for il in range(nl)] + [D.dec_layer_bytes(h, -1)]
        bounds = []
        if D.dec_persistent(h) == 1:
            slots = D.dec_clock_slots(h)
            clk = torch.zeros(slots, dtype=torch.int64, device=dev)
            assert D.dec_set_clock(h, C.c_void_p(clk.data_ptr())) == 0
            with torch.cuda.stream(stream):
                step_fn(h)()
            torch.cuda.synchronize(dev)
            assert D.dec_set_clock(h, None) == 0
            t = clk.cpu().numpy()
            idx = [D.dec_layer_clock(h, il) for il in range(-1, nl + 1)]
            bounds = [(t[idx[il + 1]] - t[idx[il]]) / 1e3 for il in range(nl + 1)]
        else:
            acc = np.zeros(nl + 1)
            for _ in range(reps):
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(nl + 2)]
                for e in evs:                       # torch creates the CUDA event on first record
                    e.record(stream)
                torch.cuda.synchronize(dev)
                arr = (C.c_void_p * nl)(*[C.c_void_p(e.cuda_event) for e in evs[1:nl + 1]])
                assert D.dec_set_layer_events(h, arr, nl) == 0
                with torch.cuda.stream(stream):
                    evs[0].record(stream)
                    step_fn(h)()
                    evs[nl + 1].record(stream)
                torch.cuda.synchronize(dev)
                assert D.dec_set_layer_events(h, None, 0) == 0
                acc += [evs[il].elapsed_time(evs[il + 1]) * 1e3 for il in range(nl + 1)]
            bounds = list(acc / reps)
        kinds = {"deltanet": [], "attention": [], "lm_head": []}
        for il in range(nl + 1):
            us = float(bounds[il])
            kind = "lm_head" if il == nl else ("attention" if (il + 1) % cfg["attn_every"] == 0 else "deltanet")
            kinds[kind].append((us, lb[il]))
        out = {}
        for k, v in kinds.items():
            if not v:
                continue
            us = sum(x[0] for x in v) / len(v)
            b = sum(x[1] for x in v) / len(v)
            out[k] = {"layers": len(v), "us": round(us, 2), "bytes": int(b),
                      "frac_hbm": round(b / (us * 1e-6) / 1e9 / peak, 4)}
        out["timing"] = "global-timer stamps at the persistent kernel's barriers" if D.dec_persistent(h) == 1 \
            else "CUDA events between layers"
        return out

    def capture(h):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step_fn(h)()
        return g

    def run_c3(nb):
        """Config 3 at batch nb: nb random-id prompts of 512 tokens (sequence
        0's is the batch-1 prompt), fed through the decode step, then 256
        greedy tokens per sequence; tokens/s counts every sequence."""
        cfg = dict(DEC_C3, batch=nb)
        h = create(cfg, 2, 0, 1)
        prompt = np.stack([np.random.default_rng(2 + 1000 * b).integers(0, cfg["vocab"], 512)
                           for b in range(nb)]).astype(np.int32)
        hprompt = torch.from_numpy(prompt).pin_memory()
        pa = C.c_void_p(hprompt.data_ptr())
        assert D.dec_set_prompt(h, pa, 512, sp) == 0
        with torch.cuda.stream(stream):
            for _ in range(3):
                step_fn(h)()
        torch.cuda.synchronize(dev)
        g = capture(h)
        for _ in range(args.warmup):
            g.replay()
        assert D.dec_set_prompt(h, pa, 512, sp) == 0
        ms_prompt = timed(g.replay, 511)
        gen = 256
        ms_gen = timed(g.replay, gen)
        torch.cuda.synchronize(dev)
        hp = C.c_void_p()
        assert D.dec_pointers(h, None, C.byref(hp), None, None, None, None) == 0
        hist = torch.as_tensor(_DevArray(hp.value, nb * cfg["max_ctx"], "<i4"), device=dev).view(nb, -1)
        toks = hist[:, 511:511 + gen].cpu().numpy()
        # end to end: the prompts from pinned host memory, and each step's
        # generated tokens read back to pinned host memory as they are produced
        htok = torch.empty(nb, dtype=torch.int32).pin_memory()

        def e2e_run():
            assert D.dec_set_prompt(h, pa, 512, sp) == 0
            with torch.cuda.stream(stream):
                for _ in range(511):
                    g.replay()
                for i in range(gen):
                    g.replay()
                    htok.copy_(hist[:, 511 + i], non_blocking=True)
                    stream.synchronize()
        e2e_ms = timed(e2e_run, 1)
        sbytes = D.dec_step_bytes(h)
        per_layer = layer_profile(h, cfg)
        mode = "persistent (1 launch per step)" if D.dec_persistent(h) == 1 else "one launch per stage"
        del g
        D.dec_destroy(h)
        peak, _ = peaks()
        us = ms_gen * 1e3 / gen
        return {
            "workload": "config 3: 24-layer hybrid (18 DeltaNet + 6 gated attention), hidden 2048, vocab 151936, "
                        "INT4 g128, seed 2; 512-token random-id prompt, 256 greedy tokens, batch %d" % nb,
            "batch": nb,
            "tokens_per_s": round(nb * gen / (ms_gen * 1e-3), 1),
            "us_per_step": round(us, 2),
            "prompt_tokens_per_s": round(nb * 511 / (ms_prompt * 1e-3), 1),
            "bytes_per_step": sbytes,
            "GBps": round(sbytes / (us * 1e-6) / 1e9, 1),
            "frac_hbm": round(sbytes / (us * 1e-6) / 1e9 / peak, 4),
            "first_tokens": [int(t) for t in toks[0, :8]],
            "step": mode,
            "per_layer": per_layer,
            "e2e": {"tokens_per_s": round(nb * (511 + gen) / (e2e_ms * 1e-3), 1),
                    "how": "prompts H2D from pinned host, 767 graph replays, each step's generated tokens D2H "
                           "(pinned) and synchronised as produced",
                    "h2d_bytes": nb * 512 * 4, "d2h_bytes_per_step": nb * 4},
        }

    def run_c2():
        """Config 2: one DeltaNet block and one gated-attention block at hidden
        2048 (the config-3 layer shapes), KV cache pre-filled to 4096
        positions with N(0,1), batch 1.  Each block timed with CUDA events
        around it, averaged over 64 steps; the pair (plus a 2048-entry LM head,
        2 MB) also as one CUDA-graph replay per step."""
        cfg = DEC_C2
        h = create(cfg, 2, 0, 1)
        assert D.dec_prefill_random(h, 4096, 5) == 0
        assert D.dec_set(h, 4096, 1) == 0
        with torch.cuda.stream(stream):
            for _ in range(3):
                step_fn(h)()
        torch.cuda.synchronize(dev)
        per_block = layer_profile(h, cfg, reps=64)
        assert D.dec_set(h, 4096, 1) == 0
        g = capture(h)
        for _ in range(args.warmup):
            g.replay()
        n = 64
        ms = timed(g.replay, n)
        sbytes = D.dec_step_bytes(h)
        del g
        D.dec_destroy(h)
        peak, _ = peaks()
        us = ms * 1e3 / n
        res = {"workload": "config 2: 1 DeltaNet block (16/16 heads x 128, conv, gates, out 2048x2048) + SwiGLU "
                           "6144, then 1 gated-attention block (16 q / 2 KV heads x 128, RoPE 1e6, sigmoid gate) "
                           "+ SwiGLU 6144; hidden 2048, INT4 g128, KV pre-filled to 4096 with N(0,1), batch 1",
               "deltanet_block": per_block.get("deltanet"), "attention_block": per_block.get("attention"),
               "timing": per_block.get("timing") + ", mean of 64 steps",
               "pair_step_us": round(us, 2), "pair_step_bytes": sbytes,
               "pair_step_frac_hbm": round(sbytes / (us * 1e-6) / 1e9 / peak, 4),
               "pair_step_how": "both blocks + final norm + 2048-entry LM head + argmax, one CUDA-graph replay"}
        if rank == 0:
            res["cpu_baseline"] = c2_cpu_baseline()
        return res

    if world == 1:
        out["config2"] = run_c2()
        out["config3"] = run_c3(1)
        out["config3"]["batch8"] = run_c3(8)

    # config 4, tensor parallel over all ranks
    cfg = DEC_C4
    h = create(cfg, 4, rank, world)
    uid = (C.c_uint8 * 128)()
    if world > 1:
        import torch.distributed as dist
        if rank == 0:
            assert D.dec_nccl_unique_id(uid) == 0
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device=dev)
        dist.broadcast(t, 0)
        uid = (C.c_uint8 * 128)(*t.cpu().tolist())
    assert D.dec_tp_init(h, uid) == 0
    exchange = "none"
    if world > 1:
        # row-parallel sums and argmax keys through peer memory (NVLink stores),
        # not NCCL: each rank's 64-byte IPC handle goes to every rank
        import torch.distributed as dist
        hnd = (C.c_uint8 * 64)()
        assert D.dec_p2p_handle(h, hnd) == 0
        allh = [None] * world
        dist.all_gather_object(allh, bytes(hnd))
        assert D.dec_p2p_open(h, (C.c_uint8 * (64 * world))(*b"".join(allh)), 0) == 0
        exchange = "peer memory (one-shot NVLink stores, bounded waits)"
    assert D.dec_prefill_random(h, 8192, 5) == 0
    assert D.dec_set(h, 8192, 1) == 0
    with torch.cuda.stream(stream):
        for _ in range(2):
            step_fn(h)()
    torch.cuda.synchronize(dev)
    g = capture(h)
    for _ in range(args.warmup):
        g.replay()
    n = 64
    ms = timed(g.replay, n)
    sbytes = D.dec_step_bytes(h)
    per_layer = layer_profile(h, cfg)
    mode = "persistent (1 launch per step)" if D.dec_persistent(h) == 1 else "one launch per stage"
    fl = C.c_int32(0)
    assert D.dec_status(h, C.byref(fl)) == 0 and fl.value == 0, "peer exchange timed out"
    del g
    D.dec_destroy(h)
    peak, _ = peaks()
    us = ms * 1e3 / n
    out["config4"] = {
        "workload": "config 4: 48-layer hybrid (36 DeltaNet + 12 gated attention), hidden 5120, 40/8 heads, "
                    "32 DeltaNet heads, FFN 17408, vocab 151936, INT4 g128; KV context 8192, batch 1",
        "tp": world,
        "tokens_per_s": round(n / (ms * 1e-3), 1),
        "us_per_token": round(us, 2),
        "bytes_per_step_per_rank": sbytes,
        "GBps_per_rank": round(sbytes / (us * 1e-6) / 1e9, 1),
        "frac_hbm": round(sbytes / (us * 1e-6) / 1e9 / peak, 4),
        "step": mode,
        "per_layer_rank0": per_layer,
        "collectives_per_step": (2 * cfg["n_layers"] + 1) if world > 1 else 0,
        "exchange": exchange,
    }
    return out


def profile_decode(args):
    """`--only decode3|decode4`: a short run for profilers -- one model
    (`--batch` sequences), the KV context pre-filled (512 or 8192 positions),
    `--warmup` then `--steps` direct steps on a stream (programmatic
    dependent launches on)."""
    import torch
    pkg = load_pkg()
    D = pkg.declib()
    cfg, pre = (DEC_C3, 512) if args.only == "decode3" else (DEC_C4, 8192)
    cfg = dict(cfg, batch=args.batch)
    h = C.c_void_p()
    assert D.dec_create(C.byref(pkg.DecConfig(**cfg)), 2, 0, 0, 1, C.byref(h)) == 0
    assert D.dec_prefill_random(h, pre, 3) == 0
    assert D.dec_set(h, pre, 1) == 0
    s = torch.cuda.Stream()
    sp = C.c_void_p(s.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            assert D.dec_step(h, sp) == 0
        e0.record(s)
        for _ in range(args.steps):
            assert D.dec_step(h, sp) == 0
        e1.record(s)
    torch.cuda.synchronize()
    print(json.dumps({"only": args.only, "batch": args.batch, "steps": args.steps,
                      "ms_per_step": e0.elapsed_time(e1) / args.steps}))
    D.dec_destroy(h)


def profile_matvec(args):
    """`--only matvec`: a short run for profilers -- the config-0 stack of
    `--stack` 4096x4096 g128 matrices (seeded), `--warmup` then `--steps`
    launches of the whole job list on one stream."""
    import torch
    pkg = load_pkg()
    L = pkg.lib()
    G = args.stack
    wq = torch.empty((G, M, K // 2), dtype=torch.uint8, device="cuda")
    sc = torch.empty((G, M, K // 128), dtype=torch.float16, device="cuda")
    x = torch.empty((G, K), dtype=torch.float16, device="cuda")
    assert L.mv4i_synth_g128(0, G, M, K, C.c_void_p(wq.data_ptr()), C.c_void_p(sc.data_ptr()),
                             C.c_void_p(x.data_ptr()), None) == 0
    y = torch.zeros((G, M), dtype=torch.float16, device="cuda")
    mats = (pkg.DMat * G)()
    jobs = (pkg.Job * G)()
    for i in range(G):
        assert L.mv4i_dmat_wrap_g128(C.c_void_p(wq[i].data_ptr()), K // 2, C.c_void_p(sc[i].data_ptr()), K // 128,
                                     M, K, 0, C.byref(mats[i])) == 0
        j = jobs[i]
        j.w = C.pointer(mats[i]); j.x = x[i].data_ptr(); j.n_rows = M; j.n_cols = K; j.nvec = 1
        j.y_f16 = y[i].data_ptr()
    s = torch.cuda.Stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            assert L.mv4i_launch(jobs, G, None, C.c_void_p(s.cuda_stream)) == 0
        e0.record(s)
        for _ in range(args.steps):
            assert L.mv4i_launch(jobs, G, None, C.c_void_p(s.cuda_stream)) == 0
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"only": "matvec", "stack": G, "steps": args.steps, "ms_per_step": ms,
                      "GBps": round(G * G128_BYTES / (ms * 1e-3) / 1e9, 1)}))


def c2_cpu_baseline(budget_s=4.0):
    """Config 2 on the host cores: the float64 restatement of the reference's
    layer_gdn / layer_attn (oracle/dec_oracle.py, pinned to ref/run9b.c) on
    synthetic weights of the config-2 shapes, KV pre-filled to 4096; mean
    seconds per block over as many steps as fit the budget.  A port (numpy,
    the BLAS threads it is given), not the reference's own C, which is
    compiled for its 9B shapes."""
    import os as _os
    import numpy as np
    from oracle import dec_oracle as DO
    c = DEC_C2
    rng = np.random.default_rng(2)
    H, HD, KH, VH, QH, KVH, F = c["hidden"], 128, c["gdn_kh"], c["gdn_vh"], c["att_qh"], c["att_kvh"], c["ffn"]
    cd = 2 * KH * HD + VH * HD

    def w(r, k):
        return rng.standard_normal((r, k)) * 0.02
    W = {(0, "qkv"): w(cd, H), (0, "z"): w(VH * HD, H), (0, "ab"): w(2 * VH, H), (0, "out"): w(H, VH * HD),
         (1, "qg"): w(2 * QH * HD, H), (1, "kv"): w(2 * KVH * HD, H), (1, "o"): w(H, QH * HD)}
    for il in (0, 1):
        W[il, "gate"], W[il, "up"], W[il, "down"] = w(F, H), w(F, H), w(H, F)
    P = {}
    for il in (0, 1):
        P[il, "attn_norm"] = np.ones(H)
        P[il, "post_norm"] = np.ones(H)
    P[0, "conv_w"] = rng.standard_normal(cd * 4) * 0.3
    P[0, "ssm_a"] = -np.abs(rng.standard_normal(VH))
    P[0, "dt_bias"] = rng.standard_normal(VH)
    P[0, "ssm_norm"] = np.ones(HD)
    P[1, "q_norm"] = np.ones(HD)
    P[1, "k_norm"] = np.ones(HD)
    S = {(0, "conv_state"): np.zeros((3, cd)), (0, "rec_state"): np.zeros((VH, HD, HD)),
         (1, "kcache"): np.zeros((c["max_ctx"], KVH, HD)), (1, "vcache"): np.zeros((c["max_ctx"], KVH, HD))}
    S[1, "kcache"][:4096] = rng.standard_normal((4096, KVH, HD))
    S[1, "vcache"][:4096] = rng.standard_normal((4096, KVH, HD))
    M = DO.Model(c, W, P, S, fp16=False)
    x = rng.standard_normal(H)
    tg = ta = 0.0
    n = 0
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or n == 0:
        t0 = time.perf_counter()
        y = M.gdn(0, x)
        y = M.ffn(0, y)
        t1 = time.perf_counter()
        y = M.attn(1, y, 4096 + n)
        y = M.ffn(1, y)
        t2 = time.perf_counter()
        tg += t1 - t0
        ta += t2 - t1
        n += 1
        if 4096 + n >= c["max_ctx"]:
            break
    thr = _os.environ.get("OMP_NUM_THREADS") or str(_os.cpu_count())
    return {"deltanet_block_us": round(tg / n * 1e6, 1), "attention_block_us": round(ta / n * 1e6, 1),
            "unit": "us per block", "cores": int(thr), "kind": "port",
            "sample": "%d steps of both config-2 blocks, float64 numpy (oracle/dec_oracle.py)" % n}


def gdn_cpu_baseline(budget_s=3.0):
    """The reference's binary32 recurrence (restated in oracle/gdn_oracle.c,
    heads over pthreads as ref/gdn_err.c:447-449 does with OpenMP)."""
    import numpy as np
    import oracle as O
    from oracle import cpu_baseline as CB
    s0, q, k, v, g, a, b = gdn_inputs(1)
    P = CB.cores()
    n, t0 = 0, time.perf_counter()
    while True:
        S = s0.copy()
        O.gdn_cfg1_f32(S, q, k, v, a, b, g.astype(np.float32), threads=P)
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s and n >= 1:
            break
    us = el / n / GDN_T * 1e6
    return {"us_per_step": round(us, 2), "cores": min(P, GDN_H), "kind": "port",
            "sample": "%d runs of the 256 config-1 steps, heads over %d threads" % (n, min(P, GDN_H))}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--stack", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["decode3", "decode4", "matvec"], default=None,
                    help="profiling aid: build one decode model (or the config-0 stack of --stack "
                         "matrices), run --steps direct steps, print ms/step")
    ap.add_argument("--batch", type=int, default=1, help="sequences of the --only decode model")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import cpu_baseline as CB
        steps, kind, P = CB.run(n_iter=args.warmup + args.steps, lockstep=True)
        t = statistics.mean(steps[args.warmup:]) if len(steps) > args.warmup else statistics.mean(steps)
        v = CB.GOLDEN_BYTES / t / 1e9
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 x int16 (integer, bit-exact golden model)",
            "data": "synthetic (splitmix64 seed 0, config-0 distributions)",
            "config": {"workload": "config 0: 4096x4096 INT4 matvec, batch 1, golden-mode image",
                       "M": M, "K": K, "parallelism": "%d processes x row shards" % P},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": P, "kind": kind,
                             "sample": "%d lockstep steps of one config-0 mv4i_matvec split over %d "
                                       "processes" % (args.warmup + args.steps, P)},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    if args.only == "matvec":
        profile_matvec(args)
        return
    if args.only:
        profile_decode(args)
        return

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    cpu = gcpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()          # spawn-started workers, before any CUDA work
        gcpu = gdn_cpu_baseline()
        bcpu = block_cpu_baseline()
    out = run_ours(args, rank, world, local_rank)
    out["cpu_baseline"] = cpu
    if gcpu:
        out["gdn"]["cpu_baseline"] = gcpu
        if isinstance(out["gdn"].get("fixed_block"), dict):
            out["gdn"]["fixed_block"]["cpu_baseline"] = bcpu
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
