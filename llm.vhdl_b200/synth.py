"""Seeded synthetic inputs for the benchmark shapes (numpy side).

The generator is splitmix64 in counter form: draw ``i`` of key ``k`` is
``mix(k + (i + 1) * 0x9E3779B97F4A7C15)``, which is output ``i`` of a
splitmix64 stream seeded with ``k``.  Unlike the reference's xorshift
generators (ref/vec_seed.h:26-40), seed 0 is legal, which the benchmark
configurations need (seeds 0, 1, 2).  The same formulas run on the device in
``mv4i_synth_g128`` (csrc/mv4i_kernels.cu), so host and device produce the
same integers for the same seed.

Keys per matrix m of a run with seed s: W uses 3*(s+m), scales 3*(s+m)+1,
x 3*(s+m)+2.
"""
import numpy as np

GOLD = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def mix64(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
    return z ^ (z >> np.uint64(31))


def draws(key, start, n):
    """n consecutive draws of stream `key`, beginning at index `start`."""
    i = np.arange(start, start + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return mix64(np.uint64(key) + (i + np.uint64(1)) * GOLD)


def unit(d):
    """draw -> double uniform in [0, 1) (top 53 bits)."""
    return (d >> np.uint64(11)).astype(np.float64) * 2.0 ** -53


def g128_weights(seed, M, K, m=0, rows=None):
    """Packed INT4 [M, K/2] uint8: two's-complement nibbles uniform over
    [-8, 7], k even in the low nibble.  rows=(r0, r1) draws only that slice."""
    r0, r1 = rows or (0, M)
    d = draws(3 * (seed + m), r0 * K, (r1 - r0) * K)
    nib = (d >> np.uint64(60)).astype(np.uint8)
    nib = nib.reshape(r1 - r0, K // 2, 2)
    return (nib[..., 0] | (nib[..., 1] << 4)).astype(np.uint8)


def g128_scales(seed, M, K, m=0, rows=None):
    """fp16 [M, K/128] uniform in [0.002, 0.02] (double -> float32 -> fp16)."""
    r0, r1 = rows or (0, M)
    ng = K // 128
    u = unit(draws(3 * (seed + m) + 1, r0 * ng, (r1 - r0) * ng))
    return (0.002 + 0.018 * u).astype(np.float32).astype(np.float16).reshape(r1 - r0, ng)


def normal_f16(key, n):
    """Box-Muller N(0,1) from pairs of draws, rounded double -> float32 -> fp16."""
    d = draws(key, 0, 2 * n).reshape(n, 2)
    u1 = ((d[:, 0] >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
    u2 = unit(d[:, 1])
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return z.astype(np.float32).astype(np.float16)


def g128_x(seed, K, m=0):
    return normal_f16(3 * (seed + m) + 2, K)


def unpack_int4(wq, K):
    """[M, K/2] packed -> [M, K] int8 in [-8, 7]."""
    lo = (wq & 0x0F).astype(np.int8)
    hi = (wq >> 4).astype(np.int8)
    out = np.empty((wq.shape[0], K), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return np.where(out >= 8, out - 16, out).astype(np.int8)


LINEAR_CB = np.array([0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1], dtype=np.int8)


def g128_to_golden(wq, scales, K):
    """The same weights as a golden-mode operand: nibble indices with the
    linear codebook (cb[i] = sext4(i)), and each fp16 group scale s written as
    the uint15 s * 2^20 into its four 32-blocks (w_exp = 5).  Exact for every
    fp16 in [2^-9, 2^-5): their ulp is >= 2^-19, so s * 2^20 is an integer
    <= 20971."""
    M = wq.shape[0]
    idx = np.empty((M, K), dtype=np.uint8)
    idx[:, 0::2] = wq & 0x0F
    idx[:, 1::2] = wq >> 4
    s = scales.astype(np.float64) * 2.0 ** 20
    q = np.rint(s)
    assert np.all(q == s) and q.max() <= 32767 and q.min() >= 0
    scl = np.repeat(q.astype(np.uint16), 4, axis=1)
    return idx, scl, 5
