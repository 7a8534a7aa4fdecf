"""Tensor-parallel partition of the INT4 matvec (llm.vhdl subsystem E) over
one process per GPU.

Sharding follows spec A 14.2-14.3 (docs/superpowers/specs/2026-08-20-int4-
streaming-matvec-design.md:1539-1716) and the TP design (docs/superpowers/
specs/2026-08-21-tp-collective-design.md):

* column-parallel (Q/K/V/z/alpha/beta, gate/up): each rank owns a contiguous
  range of output rows and the whole x; no collective.
* row-parallel (attention O, DeltaNet ssm_out, FFN down): each rank owns a
  contiguous K-slice (a multiple of 128 columns) and its slice of x.
  - golden mode: each rank BFP-packs ITS x slice (so x_exp, and therefore the
    partial's y_exp, is per rank), runs PARTIAL mode (unrounded s48 sums),
    all-gathers {partials, y_exp, out_shift}, and every rank runs the same
    E 2.1 reduction (min-align by floor, int64 sum, one round_shift, sat32,
    BFP pack) in `mv4i_tp_reduce`, so all ranks hold the identical result.
    Refusals: y_exp spread > 17 (-12), out_shift mismatch (-13).
  - g128 mode: fp32 partial sums, one all-reduce (sum).

The collectives are torch.distributed calls (NCCL between GPUs); the
arithmetic is the C library's.  Head-sharded DeltaNet and attention need no
collective (heads are independent, spec B 4.2).
"""
import ctypes as C

import torch
import torch.distributed as dist


def split(n, world, rank, align=1):
    """Contiguous [start, start+count) of n items for `rank`, in units of
    `align` (the last rank takes the remainder)."""
    units = (n + align - 1) // align
    per = units // world
    extra = units % world
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    s, e = u0 * align, min(n, u1 * align)
    return s, max(0, e - s)


def gather_partials(y_acc, y_exp, out_shift, group=None):
    """All-gather one row-parallel golden partial: y_acc int64 [M] (device
    of the process group's backend), y_exp / out_shift ints.  Returns
    (parts [world, M] int64, y_exps [world] int32, out_shifts [world] int32)."""
    world = dist.get_world_size(group)
    meta = torch.tensor([int(y_exp), int(out_shift)], dtype=torch.int32, device=y_acc.device)
    if dist.get_backend(group) == "nccl":
        parts = torch.empty((world,) + tuple(y_acc.shape), dtype=torch.int64, device=y_acc.device)
        dist.all_gather_into_tensor(parts, y_acc.contiguous(), group=group)
        metas = torch.empty((world, 2), dtype=torch.int32, device=y_acc.device)
        dist.all_gather_into_tensor(metas, meta, group=group)
    else:                                   # gloo has no all_gather_into_tensor
        pl = [torch.empty_like(y_acc) for _ in range(world)]
        dist.all_gather(pl, y_acc.contiguous(), group=group)
        ml = [torch.empty_like(meta) for _ in range(world)]
        dist.all_gather(ml, meta, group=group)
        parts, metas = torch.stack(pl), torch.stack(ml)
    return parts, metas[:, 0].contiguous(), metas[:, 1].contiguous()


def reduce_partials_device(lib, parts, y_exps, out_shifts, stream=None):
    """E 2.1 on the device through mv4i_tp_reduce.  Returns (y_mant int16
    [M], y32 int32 [M], status int32 [8]: y_exp, ns, sat_event, sat_count,
    err)."""
    if not parts.is_cuda:
        raise RuntimeError("mv4i_tp_reduce needs device tensors (the CUDA library has no CPU path)")
    N, M = parts.shape
    out = torch.empty(M, dtype=torch.int16, device=parts.device)
    y32 = torch.empty(M, dtype=torch.int32, device=parts.device)
    st = torch.zeros(8, dtype=torch.int32, device=parts.device)
    rc = lib.mv4i_tp_reduce(N, M, C.c_void_p(parts.data_ptr()), C.c_void_p(y_exps.data_ptr()),
                            C.c_void_p(out_shifts.data_ptr()), C.c_void_p(out.data_ptr()),
                            C.c_void_p(y32.data_ptr()), C.c_void_p(st.data_ptr()),
                            C.c_void_p(stream) if stream else None)
    if rc:
        raise RuntimeError("mv4i_tp_reduce failed: %d" % rc)
    return out, y32, st


def row_parallel_golden(y_acc, y_exp, out_shift, reduce_fn, group=None):
    """One row-parallel golden block: gather every rank's partial, reduce
    identically on every rank.  reduce_fn(parts, y_exps, out_shifts) ->
    (y_mant, y32, status); on GPUs that is reduce_partials_device."""
    parts, ye, osh = gather_partials(y_acc, y_exp, out_shift, group)
    return reduce_fn(parts, ye, osh)


def row_parallel_fp32(y_part, group=None):
    """g128 row-parallel block: sum the fp32 partials of all ranks in place."""
    dist.all_reduce(y_part, op=dist.ReduceOp.SUM, group=group)
    return y_part
