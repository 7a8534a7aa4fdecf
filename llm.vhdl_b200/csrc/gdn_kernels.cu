// llm.vhdl_b200/csrc/gdn_kernels.cu -- sm_100a kernels for the Gated DeltaNet
// step (llm.vhdl subsystem B).
//
// Work split (D = 128): a value column j of a head is independent of every
// other column in the recurrence (S'[:,j], sk_j, d_j, S[:,j], o_j), so one
// column is handled by 8 lanes, each owning 16 consecutive key indices; a warp
// carries 4 columns and the per-column sums are 3-level xor shuffles inside
// the 8-lane group.  The column's 128 state values (256 B int16 / 512 B fp32)
// are one contiguous read per column.
//
// * gdn_fixed_kernel: one CTA per value head (32 warps = 128 columns), the
//   exact integer recipe of ref/gdn_block_vec.c:298-361 followed by the
//   stage-6 head emit (:363-378) over the CTA's columns.
// * gdn_scalar_kernel: gdn_scalar_int (ref/gdn_scalar_vec.c:100-156), one
//   thread per head, Q30 LUTs in constant memory.
// * gdn_f32_kernel: T binary32 steps (ref/gdn_err.c:580-590 recurrence) with
//   the state in registers for the whole run, the next step's q/k/v/g/a/b
//   loaded while the current one computes.

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>
#include "../../include/gdn_b200.h"
#include "gdn_f32_step.cuh"

extern "C" int mv4i_g_cuda_err;
static int gdn_fail(cudaError_t e) { mv4i_g_cuda_err = (int)e; return -20; }

__device__ __forceinline__ int64_t g_floor_shr(int64_t v, int sh)
{ return sh <= 0 ? v : (sh >= 63 ? (v < 0 ? -1 : 0) : (v >> sh)); }
__device__ __forceinline__ int64_t g_round_shift(int64_t v, int sh)
{ return sh == 0 ? v : (sh >= 64 ? (v < 0 ? -1 : 0) : g_floor_shr(v + ((int64_t)1 << (sh - 1)), sh)); }
__device__ __forceinline__ int g_msb(uint64_t a) { return a == 0 ? 0 : 63 - __clzll((long long)a); }
__device__ __forceinline__ uint64_t g_abs64(int64_t v) { return v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v; }
__device__ __forceinline__ int16_t g_sat16(int64_t v) { return (int16_t)(v > 32767 ? 32767 : (v < -32768 ? -32768 : v)); }

__device__ __forceinline__ int64_t sum8_i64(int64_t v)
{
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ uint64_t max8_u64(uint64_t v)
{
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o); v = w > v ? w : v; }
    return v;
}

// 16 consecutive int16 (32 bytes, 32-byte aligned) as 8 packed pairs
__device__ __forceinline__ void ld16_i16(const int16_t *p, uint32_t (&w)[8])
{
    const uint4 a = reinterpret_cast<const uint4 *>(p)[0], b = reinterpret_cast<const uint4 *>(p)[1];
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ int32_t lo16(uint32_t w) { return (int32_t)(int16_t)(w & 0xFFFFu); }
__device__ __forceinline__ int32_t hi16(uint32_t w) { return (int32_t)(int16_t)(w >> 16); }

// ------------------------------------------------------------- fixed step

#define GDN_D 128

__global__ void __launch_bounds__(1024, 1)
gdn_fixed_kernel(const gdn_fixed_args A)
{
    __shared__ int64_t s_oacc[GDN_D];
    __shared__ int32_t s_eo[GDN_D];
    __shared__ int s_err;

    const int h = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = warp * 4 + (lane >> 3);          // value column
    const int sl = lane & 7, i0 = 16 * sl;          // key slice
    const int hk = h % A.KH;
    if (threadIdx.x == 0) s_err = 0;
    __syncthreads();

    int16_t *scol = A.smem + ((size_t)h * GDN_D + j) * GDN_D + i0;
    uint32_t sm[8], kn[8], qs[8];
    ld16_i16(scol, sm);
    ld16_i16(A.kn + (size_t)hk * GDN_D + i0, kn);
    ld16_i16(A.qs + (size_t)hk * GDN_D + i0, qs);
    const int se_j = A.semem[h * GDN_D + j];
    const int32_t v_j = A.v[h * GDN_D + j];
    const int egh = A.eg[h], bth = A.beta[h], tk0 = A.tk0, e_v = A.e_v;

    // stage 1-2: decay onto the se_j + 2 grid, sk dot
    int32_t w18[16];
    int64_t sk = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const int32_t a = tk0 ? 0 : lo16(sm[p]) * egh, b = tk0 ? 0 : hi16(sm[p]) * egh;  // |.| < 2^30
        w18[2 * p] = (a + 4096) >> 13;                                                  // round_shift(., 13)
        w18[2 * p + 1] = (b + 4096) >> 13;
        sk += (int64_t)w18[2 * p] * lo16(kn[p]) + (int64_t)w18[2 * p + 1] * hi16(kn[p]);
    }
    sk = sum8_i64(sk);
    int sh_sk = g_msb(g_abs64(sk)) - 14;
    if (sh_sk < 0) sh_sk = 0;
    const int64_t skm = g_round_shift(sk, sh_sk);
    const int ske = se_j + 17 - sh_sk;

    // stage 3: delta on its own grid (masked when tk0 or eg = 0)
    const bool masked = tk0 || egh == 0;
    const int e_d = masked ? e_v : (e_v < ske ? e_v : ske);
    int s1 = e_v - e_d, s2 = ske - e_d;
    if (s1 > 63) s1 = 63;
    if (s2 > 63) s2 = 63;
    const int64_t draw = (g_floor_shr(v_j, s1) - g_floor_shr(skm, s2)) * (int64_t)bth;
    int shd = g_msb(g_abs64(draw)) - 14;
    if (shd < 0) shd = 0;
    const int64_t d_m = g_round_shift(draw, shd);
    const int e_dm = e_d + 16 - shd;

    // stage 4: update on the common grid, write-back quantiser
    const int e_kd = 15 + e_dm;
    const int e_u = masked ? e_kd : (se_j + 2 < e_kd ? se_j + 2 : e_kd);
    int su = se_j + 2 - e_u, sk2 = e_kd - e_u;
    if (su > 63) su = 63;
    if (sk2 > 63) sk2 = 63;
    uint64_t amax = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int32_t k = hlf ? hi16(kn[p]) : lo16(kn[p]);
            const int64_t u = (tk0 ? 0 : g_floor_shr(w18[2 * p + hlf], su)) + g_floor_shr((int64_t)k * d_m, sk2);
            const uint64_t a = g_abs64(u);
            amax = a > amax ? a : amax;
        }
    }
    amax = max8_u64(amax);
    int sh = g_msb(amax) - 14;
    if (sh < 0) sh = 0;
    uint32_t sn[8];
    int64_t od = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
        int32_t r2[2];
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int32_t k = hlf ? hi16(kn[p]) : lo16(kn[p]);
            const int64_t u = (tk0 ? 0 : g_floor_shr(w18[2 * p + hlf], su)) + g_floor_shr((int64_t)k * d_m, sk2);
            r2[hlf] = g_sat16(g_round_shift(u, sh));
        }
        sn[p] = ((uint32_t)(uint16_t)r2[0]) | ((uint32_t)(uint16_t)r2[1] << 16);
        // stage 5: output dot on the requantised mantissas
        od += (int64_t)r2[0] * lo16(qs[p]) + (int64_t)r2[1] * hi16(qs[p]);
    }
    reinterpret_cast<uint4 *>(scol)[0] = make_uint4(sn[0], sn[1], sn[2], sn[3]);
    reinterpret_cast<uint4 *>(scol)[1] = make_uint4(sn[4], sn[5], sn[6], sn[7]);
    od = sum8_i64(od);
    const int se_new = e_u - sh, e_o = se_new + 18;
    if (sl == 0) {
        A.semem[h * GDN_D + j] = se_new;
        A.o_acc[h * GDN_D + j] = od;
        A.e_o[h * GDN_D + j] = e_o;
        s_oacc[j] = od;
        s_eo[j] = e_o;
        if (se_new > 127 || se_new < -128 || e_o > 127 || e_o < -128) atomicOr(&s_err, 1);
    }
    __syncthreads();

    // stage 6 (site 12): fold the head to its minimum exponent, BFP-pack
    if (warp == 0) {
        int emin = 1 << 30;
        for (int c = lane; c < GDN_D; c += 32) emin = min(emin, s_eo[c]);
#pragma unroll
        for (int o = 16; o; o >>= 1) emin = min(emin, __shfl_xor_sync(0xffffffffu, emin, o));
        int64_t al[GDN_D / 32];
        uint64_t am = 0;
#pragma unroll
        for (int t = 0; t < GDN_D / 32; t++) {
            const int c = lane + 32 * t;
            int shj = s_eo[c] - emin;
            if (shj > 63) shj = 63;
            al[t] = g_floor_shr(s_oacc[c], shj);
            const uint64_t a = g_abs64(al[t]);
            am = a > am ? a : am;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) { const uint64_t w = __shfl_xor_sync(0xffffffffu, am, o); am = w > am ? w : am; }
        int shh = g_msb(am) - 14;
        if (shh < 0) shh = 0;
        if (A.o_head) {
#pragma unroll
            for (int t = 0; t < GDN_D / 32; t++) A.o_head[h * GDN_D + lane + 32 * t] = g_sat16(g_round_shift(al[t], shh));
        }
        if (lane == 0) {
            if (A.e_head) A.e_head[h] = emin - shh;
            if (s_err && A.err) atomicOr(A.err, 1);
        }
    }
}

extern "C" int gdn_step_fixed(const gdn_fixed_args *a, void *stream)
{
    if (!a || a->D != GDN_D || a->H <= 0 || a->KH <= 0 || !a->smem || !a->semem || !a->kn || !a->qs
        || !a->v || !a->eg || !a->beta || !a->o_acc || !a->e_o) return -11;
    if ((((uintptr_t)a->smem) | ((uintptr_t)a->kn) | ((uintptr_t)a->qs)) & 31) return -11;
    gdn_fixed_kernel<<<a->H, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

// ------------------------------------------------------------ scalar path

__constant__ int64_t c_exp_lut[257], c_sig_lut[513], c_sp_lut[257];
static unsigned long long g_lut_ready = 0;

// Q30 tables, built exactly as ref/fx.h:51-79 builds them (host libm).
static cudaError_t upload_luts()
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && (g_lut_ready >> dev & 1ull)) return cudaSuccess;
    static int64_t te[257], ts[513], tp[257];
    for (int k = 0; k <= 256; k++) {
        const double z = -16.0 + (double)k * (16.0 / 256.0);
        te[k] = llround(exp(z) * 1073741824.0);
        tp[k] = llround(log1p(exp(z)) * 1073741824.0);
    }
    for (int k = 0; k <= 512; k++) {
        const double z = -16.0 + (double)k * (32.0 / 512.0);
        ts[k] = llround((1.0 / (1.0 + exp(-z))) * 1073741824.0);
    }
    e = cudaMemcpyToSymbol(c_exp_lut, te, sizeof te);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_sig_lut, ts, sizeof ts);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_sp_lut, tp, sizeof tp);
    if (e == cudaSuccess && dev < 64) g_lut_ready |= 1ull << dev;
    return e;
}

__device__ int64_t d_lut_interp(const int64_t *tab, int kmax, int64_t offset, int q)
{
    const int64_t idx_fp = offset * 16;
    int64_t k = idx_fp >> q;
    if (k > kmax - 1) k = kmax - 1;
    if (k < 0) k = 0;
    const int64_t frac = idx_fp - (k << q);
    const int64_t lo = tab[k], hi = tab[k + 1];
    const int64_t v30 = lo + (((hi - lo) * frac) >> q);
    const int sh = 30 - q;
    return sh > 0 ? ((v30 + ((int64_t)1 << (sh - 1))) >> sh) : v30;
}

#define SPQ 18
#define SAT_W ((int64_t)1 << 45)
#define SAT_G ((int64_t)1 << 62)

__device__ int64_t d_to_q_wide(int32_t m, int e)
{
    if (m == 0) return 0;
    const int sh = e - SPQ;
    if (sh >= 0) {
        if (sh > 62) return 0;
        return g_floor_shr((int64_t)m + (sh ? (int64_t)1 << (sh - 1) : 0), sh);
    }
    const int s = -sh;
    if (s > 40) return m > 0 ? SAT_W : -SAT_W;
    int64_t v = (int64_t)m * ((int64_t)1 << s);
    return v > SAT_W ? SAT_W : (v < -SAT_W ? -SAT_W : v);
}

__device__ int64_t d_rshift_r(int64_t v, int s)
{
    if (s <= 0) {
        const int k = -s;
        if (v == 0) return 0;
        if (k > 62) return v > 0 ? SAT_G : -SAT_G;
        if (v > (SAT_G >> k)) return SAT_G;
        if (v < -(SAT_G >> k)) return -SAT_G;
        return v * ((int64_t)1 << k);
    }
    if (s > 62) return 0;
    return g_floor_shr(v + ((int64_t)1 << (s - 1)), s);
}

__global__ void gdn_scalar_kernel(int H, const int32_t *sc, int32_t *eg_o, int32_t *beta_o, int32_t *err_o)
{
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= H) return;
    const int32_t *p = sc + (size_t)h * 8;
    const int64_t arg = d_to_q_wide(p[0], p[1]) + d_to_q_wide(p[2], p[3]);
    const int64_t one = (int64_t)1 << SPQ, lim = 16 * one;
    int64_t sp;
    if (arg <= -lim) sp = 0;
    else if (arg >= lim) sp = arg;
    else {
        const int64_t x = arg, ax = x < 0 ? -x : x, pos = x > 0 ? x : 0;
        const int64_t corr = ax >= lim ? 0 : d_lut_interp(c_sp_lut, 256, lim - ax, SPQ);
        sp = pos + corr;
        if (sp < 0) sp = 0;
        if (sp > 0x7FFFFFFF) sp = 0x7FFFFFFF;
    }
    int64_t g = d_rshift_r(sp * (int64_t)p[4], p[5]);
    if (g > 0) g = 0;
    const int err = g < -lim;
    if (g < -lim) g = -lim;
    int64_t ex = (g < -lim) ? 0 : d_lut_interp(c_exp_lut, 256, g + lim, SPQ);
    if (ex < 0) ex = 0;
    if (ex > 0x7FFFFFFF) ex = 0x7FFFFFFF;
    int64_t egv = d_rshift_r(ex, SPQ - 15);
    egv = egv > 32768 ? 32768 : (egv < 0 ? 0 : egv);
    int64_t bq = d_to_q_wide(p[6], p[7]);
    bq = bq > lim ? lim : (bq < -lim ? -lim : bq);
    int64_t sg;
    if (bq <= -lim) sg = 0;
    else if (bq >= lim) sg = one;
    else {
        sg = d_lut_interp(c_sig_lut, 512, bq + lim, SPQ);
        sg = sg < 0 ? 0 : (sg > one ? one : sg);
    }
    int64_t bv = d_rshift_r(sg, SPQ - 16);
    bv = bv > 65535 ? 65535 : (bv < 0 ? 0 : bv);
    eg_o[h] = (int32_t)egv;
    beta_o[h] = (int32_t)bv;
    if (err_o) err_o[h] = err;
}

extern "C" int gdn_scalar_dev(int H, const int32_t *d_sc, int32_t *d_eg, int32_t *d_beta, int32_t *d_err,
                              void *stream)
{
    if (H <= 0 || !d_sc || !d_eg || !d_beta) return -11;
    cudaError_t e = upload_luts();
    if (e != cudaSuccess) return gdn_fail(e);
    gdn_scalar_kernel<<<(H + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(H, d_sc, d_eg, d_beta, d_err);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

// --------------------------------------------------------- binary32 steps

// grid: H x 8 CTAs of 4 warps; CTA (h, c) owns columns 16c .. 16c+15 of head h
// (the body is gdn_f32_step.cuh, shared with the persistent decode kernel).
__global__ void __launch_bounds__(128)
gdn_f32_kernel(const gdn_f32_args A0)
{
    // the CTA's 16 state columns (8 KB, contiguous) do not depend on the
    // previous kernel: ask L2 for them first
    if (threadIdx.x == 0) {
        const float *S = A0.S + ((size_t)blockIdx.y * A0.H * 128 + (size_t)(blockIdx.x >> 3) * 128 + (blockIdx.x & 7) * 16) * 128;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(S), "r"(8192u) : "memory");
    }
    // a programmatic dependent of the previous kernel: let the next one
    // launch, then wait for this one's inputs (no-ops otherwise)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    gdn_f32_cta<false>(A0, blockIdx.x, blockIdx.y, threadIdx.x);
}

extern "C" int gdn_run_f32(const gdn_f32_args *a, void *stream)
{
    if (!a || a->D != 128 || a->T <= 0 || a->H <= 0 || a->KH <= 0 || !a->S || !a->q || !a->k || !a->v
        || (!a->eg && !a->a) || (!a->beta && !a->b) || (!a->out_f32 && !a->out_f16)) return -11;
    if ((((uintptr_t)a->S) | ((uintptr_t)a->q) | ((uintptr_t)a->k)) & 15) return -11;
    const int nseq = a->nseq > 1 ? a->nseq : 1;
    if (nseq > 1 && (a->T != 1 || a->seq_in <= 0 || (a->seq_in & 7) || nseq > 65535)) return -11;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->H * 8, nseq);
    cfg.blockDim = dim3(128);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a->pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_f32_kernel, *a);
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

// ------------------------------------------------ the fixed-point block

#include "gdn_block.cuh"
