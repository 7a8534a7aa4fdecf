// llm.vhdl_b200/csrc/dec_matvec.cu -- the INT4 g128 matvec of the decode step.
//
// One launch computes up to four projections of the same input vector (the A
// jobs of ref/run9b.c's layer_gdn / layer_attn, :602-900) with the vector ops
// around them folded in:
//   prologue  each CTA builds the fp16 input itself: plain fp16, RMSNorm of the
//             fp32 residual (ref/run9b.c:557-569), or the DeltaNet output norm
//             and z gate per 128-wide head (:708-728); then stages it as int16
//             on a per-128-column exponent (the g128 contract of
//             mv4i_kernels.cu) in shared memory.
//   epilogue  per output row: fp32 / fp16 store, residual accumulate, SwiGLU of
//             paired gate/up rows (:744), the DeltaNet 4-tap conv + SiLU with its
//             rolling state (:634-672), the decay/beta gates (:674-683), or the
//             LM head's first-max argmax key (:399-405).
// Work split: tiles of 8 rows (one warp per row, or per gate/up row pair),
// contiguous tile ranges per CTA, a grid of at most one wave; a warp streams
// up to 4 rows at a time, lanes over 64-column pairs, one batch of loads
// ahead.  Launched as a programmatic dependent of the previous kernel: the
// first weights are requested before waiting for it (they do not depend on
// it), and the next kernel may launch at once.

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>
#include "dec_internal.h"

extern "C" int mv4i_g_cuda_err;

#define DMV_THREADS 256            // CTA of the persistent decode kernel and the staging launch
#define DMV_WARPS 8
#define DMV_WIDE_K 4096            // a single-sequence launch with K at least this runs one CTA
                                   // of 16 warps per SM (the staging split over twice the
                                   // threads), shorter ones two CTAs of 8 warps
#define DMV_G 4                    // rows a warp streams together (2 gate/up pairs)
#define DMV_MAXG 256               // 128-column groups of the widest input (K <= 32768)
#define DMV_HOLD 2                 // units per thread an RMSNorm prologue keeps in registers
#ifndef DMV_MINB
#define DMV_MINB 2                 // resident CTAs per SM the registers are sized for
#endif

#ifndef DEC_PDL_HELPERS
#define DEC_PDL_HELPERS
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}

// 32 bytes of streamed weights (read once: no L1 allocation)
__device__ __forceinline__ void ld_w32(const uint8_t *p, uint32_t (&w)[8])
{
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
        : "l"(p));
}

// a 16-bit scale, issued in program order with the weight loads
__device__ __forceinline__ float ld_scale(const uint16_t *p)
{
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ int dp_uu(uint32_t a, uint32_t b, int c)
{
    int d;
    asm volatile("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp_us(uint32_t a, uint32_t b, int c)
{
    int d;
    asm volatile("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// sat16(rint(f * 2^e)), round half to even; scale = 2^e exactly.  |f * 2^e| <
// 2^15 by the choice of e, so only +32768 (from rounding) needs the clamp.
__device__ __forceinline__ int to_i16(float f, float scale)
{
    return min(__float2int_rn(f * scale), 32767);
}

__device__ __forceinline__ uint32_t prmt_b(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// 2^n for n in [-126, 127]
__device__ __forceinline__ float exp2i(int n) { return __int_as_float((127 + n) << 23); }

// Shared memory (K columns, np = K/64 pairs of 32-column blocks, ng = K/128):
//   planes  uint4 [4 planes][2 block parities][np]: the int16 x split into
//           low bytes (unsigned) and high bytes (signed) of even / odd
//           columns; word q of a block holds columns 8q + {0,2,4,6} (+1)
//   psum    int   [np]  sum of the staged int16 x over the pair
//   gfac    float [ng]  2^-e of each group
//   gs      int2  [ng]  {sum of the staged int16 x over the group, 2^-e bits}
struct Sm {
    uint4 *planes; int *psum; float *gfac; int2 *gs;
};

__host__ __device__ __forceinline__ size_t r16(size_t n) { return (n + 15) & ~(size_t)15; }

__device__ __forceinline__ Sm sm_layout(uint8_t *sm, int K)
{
    const size_t np = K >> 6, ng = K >> 7;
    Sm s;
    s.planes = reinterpret_cast<uint4 *>(sm);
    s.psum = reinterpret_cast<int *>(sm + 128 * np);
    s.gfac = reinterpret_cast<float *>(sm + 128 * np + r16(4 * np));
    s.gs = reinterpret_cast<int2 *>(sm + 128 * np + r16(4 * np) + r16(4 * ng));
    return s;
}

__host__ __device__ __forceinline__ size_t dmv_smem_x_bytes(int K)
{
    const size_t np = K >> 6, ng = K >> 7;
    return 128 * np + r16(4 * np) + r16(4 * ng) + r16(8 * ng);
}

// the 8 fp32 inputs of unit u (columns 8u .. 8u+7): x (fp16 / fp32
// residual / DeltaNet o) and, for the gated prologue, z
__device__ __forceinline__ void unit_load(const dmv_params &P, const void *xv, const float *x2v, int u, bool ok,
                                          float (&v)[8], float (&z)[8])
{
    if (!ok) {
#pragma unroll
        for (int k = 0; k < 8; k++) { v[k] = 0.f; z[k] = 0.f; }
        return;
    }
    if (P.op == DMV_OP_F16) {
        const uint4 r = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(xv) + 8 * u);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
            v[2 * k] = f.x; v[2 * k + 1] = f.y;
        }
    } else {
        const float4 *x = reinterpret_cast<const float4 *>(static_cast<const float *>(xv) + 8 * u);
        const float4 a = x[0], b = x[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        if (P.op == DMV_OP_GATED) {
            const float4 *zp = reinterpret_cast<const float4 *>(x2v + 8 * u);
            const float4 c = zp[0], d = zp[1];
            z[0] = c.x; z[1] = c.y; z[2] = c.z; z[3] = c.w; z[4] = d.x; z[5] = d.y; z[6] = d.z; z[7] = d.w;
        }
    }
}

// sum of squares of a unit's 8 values, then over its half warp: the
// 128-column group's sum (every lane of the half warp gets the same bits)
__device__ __forceinline__ float grp_ssq(const float (&v)[8])
{
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) ss = fmaf(v[k], v[k], ss);
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    return ss;
}

// The RMSNorm statistic of a K-column vector from its 128-column group sums
// gss[0 .. K/128): four interleaved partial sums in group order, then
// (s0 + s1) + (s2 + s3).  Every path (8- and 16-warp CTAs, the staging
// launch, batches) forms the group sums the same way (grp_ssq), so the
// statistic and every result after it are the same bit for bit.
__device__ __forceinline__ float dmv_inv_rms(const float *gss, int K, float eps)
{
    const int ng = K >> 7;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < ng; g += 4) {
#pragma unroll
        for (int j = 0; j < 4; j++) if (g + j < ng) s[j] += gss[g + j];
    }
    return rsqrtf(((s[0] + s[1]) + (s[2] + s[3])) / (float)K + eps);
}

// The group sums of squares of vectors b0 .. b0+NB-1 (those below P.nvec)
// into gss + i * DMV_MAXG (RMSNorm prologue, fp32 residual input); every
// thread of the CTA calls it (shuffles inside), a barrier must follow.
template <int NB, int NW>
__device__ __forceinline__ void dmv_group_ssq(const dmv_params &P, int b0, float *gss)
{
    const int nu = P.K >> 3, tid = threadIdx.x;
    for (int u0 = 0; u0 < nu; u0 += 32 * NW) {           // uniform trip count: shuffles below
        const int u = u0 + tid;
        const bool ok = u < nu;                           // whole half warps
        float v[NB][8];
#pragma unroll
        for (int i = 0; i < NB; i++) {
            const bool oki = ok && b0 + i < P.nvec;
            if (oki) {
                const float4 *x = reinterpret_cast<const float4 *>(static_cast<const float *>(P.x) +
                                                                   (size_t)(b0 + i) * P.xs + 8 * u);
                const float4 a = x[0], c = x[1];
                v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
                v[i][4] = c.x; v[i][5] = c.y; v[i][6] = c.z; v[i][7] = c.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) v[i][k] = 0.f;
            }
        }
#pragma unroll
        for (int i = 0; i < NB; i++) {
            const float ss = grp_ssq(v[i]);
            if (ok && !(u & 15)) gss[i * DMV_MAXG + (u >> 4)] = ss;
        }
    }
}

// fp16 rounding (the storage contract), the group exponent, and unit u's
// int16 x into the byte planes, pair sums and group records of the block s;
// v holds the unit's 8 inputs after the prologue's arithmetic.  Whole half
// warps call it together (shuffles inside); ok is false for padding units.
__device__ __forceinline__ void stage_unit(const Sm &s, int np, int u, bool ok, float (&v)[8], uint16_t *seam)
{
    uint32_t *pw = reinterpret_cast<uint32_t *>(s.planes);
    uint32_t hw[4];
    float m = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const __half2 h2 = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        hw[k] = *reinterpret_cast<const uint32_t *>(&h2);
        const float2 f = __half22float2(h2);
        v[2 * k] = f.x; v[2 * k + 1] = f.y;
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int e = 0;
    // m in [2^(ex-1), 2^ex) (frexp's ex; m is an fp16 value, a normal fp32)
    if (m > 0.f) e = 15 - ((int)((__float_as_uint(m) >> 23) & 0xFF) - 126);
    const float scale = exp2i(e);
    int xi[8], ssum = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) { xi[k] = to_i16(v[k], scale); ssum += xi[k]; }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    const int gsum = ssum + __shfl_xor_sync(0xffffffffu, ssum, 8);
    if (ok) {
        // byte planes by permutes: t = {x0.b0, x2.b0, x0.b1, x2.b1} and
        // {x4.b0, x6.b0, x4.b1, x6.b1}, then their low / high halves
        const uint32_t te0 = prmt_b(xi[0], xi[2], 0x5140u), te1 = prmt_b(xi[4], xi[6], 0x5140u);
        const uint32_t to0 = prmt_b(xi[1], xi[3], 0x5140u), to1 = prmt_b(xi[5], xi[7], 0x5140u);
        const uint32_t le = prmt_b(te0, te1, 0x5410u), he = prmt_b(te0, te1, 0x7632u);
        const uint32_t lo = prmt_b(to0, to1, 0x5410u), ho = prmt_b(to0, to1, 0x7632u);
        const int c = u >> 2, q = u & 3, p = c >> 1, par = c & 1;
        pw[4 * ((0 + par) * np + p) + q] = le;
        pw[4 * ((2 + par) * np + p) + q] = lo;
        pw[4 * ((4 + par) * np + p) + q] = he;
        pw[4 * ((6 + par) * np + p) + q] = ho;
        if (!(u & 7)) s.psum[u >> 3] = ssum;
        if (!(u & 15)) {
            s.gfac[u >> 4] = exp2i(-e);
            s.gs[u >> 4] = make_int2(gsum, __float_as_int(exp2i(-e)));
        }
        if (seam) *reinterpret_cast<uint4 *>(seam + 8 * u) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
}

// Stage units [u_lo, u_hi) of vector b into the block at dst (shared memory,
// or global memory for dec_k_stage: the same layout): unit u = 8 columns per
// thread, so a 128-column group is 16 consecutive lanes (a half warp) and a
// 64-column pair 8 lanes: group max, pair sums and per-head norms are
// shuffle reductions.  u_lo and u_hi are multiples of 16; every thread of
// the CTA calls it.  inv: 1 / rms of the vector (RMSNorm prologue).
template <int NW>
__device__ __forceinline__ void dmv_stage_vec(const dmv_params &P, int b, float inv, uint8_t *dst, int u_lo,
                                              int u_hi, bool seam_cta)
{
    const int K = P.K, np = K >> 6, tid = threadIdx.x;
    const Sm s = sm_layout(dst, K);
    const void *xv = P.op == DMV_OP_F16 ? static_cast<const void *>(static_cast<const uint16_t *>(P.x) + (size_t)b * P.xs)
                                        : static_cast<const void *>(static_cast<const float *>(P.x) + (size_t)b * P.xs);
    const float *x2v = P.x2 ? P.x2 + (size_t)b * P.xs : nullptr;
    uint16_t *seam = P.seam && seam_cta ? P.seam + (size_t)b * K : nullptr;
    for (int u0 = u_lo; u0 < u_hi; u0 += 32 * NW) {       // uniform trip count: shuffles below
        const int u = u0 + tid;
        const bool ok = u < u_hi;                           // whole half warps
        float v[8], z[8];
        unit_load(P, xv, x2v, u, ok, v, z);
        if (P.op == DMV_OP_RMSNORM) {
            if (ok) {
                const float4 *wp = reinterpret_cast<const float4 *>(P.nw + 8 * u);
                const float4 a = wp[0], c = wp[1];
                const float w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
                for (int k = 0; k < 8; k++) v[k] = v[k] * inv * w[k];
            }
        } else if (P.op == DMV_OP_GATED) {
            const float ginv = rsqrtf(grp_ssq(v) / 128.f + P.eps);
            if (ok) {
                const float4 *wp = reinterpret_cast<const float4 *>(P.nw + ((8 * u) & 127));
                const float4 a = wp[0], c = wp[1];
                const float w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
                for (int k = 0; k < 8; k++) v[k] = v[k] * ginv * w[k] * silu_f(z[k]);
            }
        }
        stage_unit(s, np, u, ok, v, seam);
    }
}

// One sequence's RMSNorm prologue in one read of the residual: each thread
// keeps its units (at most DMV_HOLD per thread) and their norm weights in
// registers while the group sums of squares meet in shared memory, then
// scales and stages them.  The same arithmetic as dmv_group_ssq +
// dmv_stage_vec (bit-identical blocks).
template <int NW>
__device__ __forceinline__ void dmv_stage_rms1(const dmv_params &P, uint8_t *dst, float *gss, bool seam_cta)
{
    const int K = P.K, np = K >> 6, nu = K >> 3, tid = threadIdx.x;
    const int nit = (nu + 32 * NW - 1) / (32 * NW);
    const float *x = static_cast<const float *>(P.x);
    float v[DMV_HOLD][8], w[DMV_HOLD][8];
#pragma unroll
    for (int it = 0; it < DMV_HOLD; it++) {
        if (it < nit) {                                     // uniform over the CTA
            const int u = it * 32 * NW + tid;
            if (u < nu) {
                const float4 *xp = reinterpret_cast<const float4 *>(x + 8 * u);
                const float4 *wp = reinterpret_cast<const float4 *>(P.nw + 8 * u);
                const float4 a = xp[0], c = xp[1], d = wp[0], f = wp[1];
                v[it][0] = a.x; v[it][1] = a.y; v[it][2] = a.z; v[it][3] = a.w;
                v[it][4] = c.x; v[it][5] = c.y; v[it][6] = c.z; v[it][7] = c.w;
                w[it][0] = d.x; w[it][1] = d.y; w[it][2] = d.z; w[it][3] = d.w;
                w[it][4] = f.x; w[it][5] = f.y; w[it][6] = f.z; w[it][7] = f.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) { v[it][k] = 0.f; w[it][k] = 0.f; }
            }
        }
    }
#pragma unroll
    for (int it = 0; it < DMV_HOLD; it++) {
        if (it < nit) {
            const int u = it * 32 * NW + tid;
            const float ss = grp_ssq(v[it]);
            if (u < nu && !(u & 15)) gss[u >> 4] = ss;
        }
    }
    __syncthreads();
    const float inv = dmv_inv_rms(gss, K, P.eps);
    const Sm s = sm_layout(dst, K);
    uint16_t *seam = P.seam && seam_cta ? P.seam : nullptr;
#pragma unroll
    for (int it = 0; it < DMV_HOLD; it++) {
        if (it < nit) {
            const int u = it * 32 * NW + tid;
#pragma unroll
            for (int k = 0; k < 8; k++) v[it][k] = v[it][k] * inv * w[it][k];
            stage_unit(s, np, u, u < nu, v[it], seam);
        }
    }
}

// Stage x: NV vectors (the sequences of a batch; those past P.nvec are not
// staged and their results are dropped), vector b into the shared-memory
// block at sm + b * xb.  HOLD: a single sequence's RMSNorm prologue keeps its
// units in registers (one read of the residual) where they fit.
template <int NV, int NW, bool HOLD>
__device__ void dmv_stage(const dmv_params &P, uint8_t *sm, size_t xb, bool seam_cta)
{
    __shared__ float gss[NV * DMV_MAXG];
    if (HOLD && P.op == DMV_OP_RMSNORM && NV == 1 && (P.K >> 3) <= DMV_HOLD * 32 * NW) {
        dmv_stage_rms1<NW>(P, sm, gss, seam_cta);
        __syncthreads();
        return;
    }
    if (P.op == DMV_OP_RMSNORM) {
        dmv_group_ssq<NV, NW>(P, 0, gss);
        __syncthreads();
    }
#pragma unroll 1
    for (int b = 0; b < NV && b < P.nvec; b++)
        dmv_stage_vec<NW>(P, b, P.op == DMV_OP_RMSNORM ? dmv_inv_rms(gss + b * DMV_MAXG, P.K, P.eps) : 0.f,
                          sm + b * xb, 0, P.K >> 3, seam_cta);
    __syncthreads();
}

// The blocks dec_k_stage wrote (vectors 0 .. nvs-1, contiguous) into shared
// memory: 16-byte asynchronous copies, all in flight at once.
template <int NW>
__device__ __forceinline__ void dmv_load_staged(const uint8_t *src, uint8_t *sm, size_t bytes)
{
    const uint32_t base = (uint32_t)__cvta_generic_to_shared(sm);
    for (size_t i = 16 * (size_t)threadIdx.x; i < bytes; i += 16 * 32 * NW)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(base + (uint32_t)i), "l"(src + i) : "memory");
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
}

// sum_j cb_j * x_j over the 64 columns of pair p; w[0..3] block 2p, w[4..7]
// block 2p+1; cb = (nibble ^ 8) - 8, x = 256 * hi + lo.
__device__ __forceinline__ void pair_dot4(const uint32_t (&w)[8], const uint4 (&xp)[8], int (&a)[4])
{
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint4 xle = xp[0 + half], xlo = xp[2 + half], xhe = xp[4 + half], xho = xp[6 + half];
        const uint32_t le[4] = {xle.x, xle.y, xle.z, xle.w}, lo[4] = {xlo.x, xlo.y, xlo.z, xlo.w};
        const uint32_t he[4] = {xhe.x, xhe.y, xhe.z, xhe.w}, ho[4] = {xho.x, xho.y, xho.z, xho.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint32_t wv = w[4 * half + q];
            const uint32_t e = (wv & 0x0F0F0F0Fu) ^ 0x08080808u;     // idx^8 of even columns
            const uint32_t o = (wv & 0xF0F0F0F0u) ^ 0x80808080u;     // 16*(idx^8) of odd columns
            a[0] = dp_uu(e, le[q], a[0]);
            a[1] = dp_uu(o, lo[q], a[1]);
            a[2] = dp_us(e, he[q], a[2]);
            a[3] = dp_us(o, ho[q], a[3]);
        }
    }
}

// the job descriptors live in shared memory (kernel parameters indexed at
// run time would be read through memory loads in the inner loop)
__device__ __forceinline__ int dmv_job_of(const dmv_params &P, const dmv_job *JS, int t)
{
    int j = 0;
    for (int i = 1; i < P.njobs; i++) if (t >= JS[i].tile0) j = i;
    return j;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx)
{
    const uint32_t u = __float_as_uint(v);
    const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)k << 32) | (0xFFFFFFFFull - (uint32_t)idx);
}

// per-row epilogue of vector b (one lane); v2 is the paired row's value.
// Vector b's outputs sit b * ostride elements on, its conv state b * 3 *
// st_stride.
__device__ __forceinline__ void dmv_epilogue(const dmv_params &P, const dmv_job &J, int b, int row, float v,
                                             float v2, unsigned long long &best)
{
    const size_t o = (size_t)b * J.ostride + row;
    switch (J.epi) {
    case DMV_EPI_F32: J.out_f32[o] = v; break;
    case DMV_EPI_ACC: J.out_f32[o] += v; break;
    case DMV_EPI_F16:
        J.out_f16[o] = __half_as_ushort(__float2half_rn(v));
        if (J.out_f32) J.out_f32[o] = v;
        break;
    case DMV_EPI_SWIGLU:
        J.out_f16[o] = __half_as_ushort(__float2half_rn(silu_f(v) * v2));
        break;
    case DMV_EPI_CONV: {
        // taps 0..2 on the stored inputs (oldest first), tap 3 on this one
        const int S = J.st_stride;
        float *st = J.st + (size_t)b * 3 * S;
        const float s0 = st[row], s1 = st[S + row], s2 = st[2 * S + row];
        const float4 cw = reinterpret_cast<const float4 *>(J.p0)[row];
        const float a = s0 * cw.x + s1 * cw.y + s2 * cw.z + v * cw.w;
        st[row] = s1; st[S + row] = s2; st[2 * S + row] = v;
        J.out_f16[o] = __half_as_ushort(__float2half_rn(silu_f(a)));
        if (J.out_f32) J.out_f32[o] = v;
        break;
    }
    case DMV_EPI_GATES:
        if (row < J.n1) {
            const float av = v + J.p1[row];
            const float sp = av > 20.f ? av : log1pf(expf(av));
            J.out_f32[o] = expf(J.p0[row] * sp);
        } else {
            J.out2_f32[o - J.n1] = 1.0f / (1.0f + expf(-v));
        }
        break;
    case DMV_EPI_ARGMAX: {
        J.out_f32[o] = v;
        const unsigned long long k = argmax_key(v, P.idx0 + row);
        best = k > best ? k : best;
        break;
    }
    default: break;
    }
}

// ------------------------------------------------------------ the stream
//
// A CTA owns a contiguous range of tiles; within each job it meets, warp w
// takes row w of every tile, G rows at a time (G = 4, or 2 gate/up pairs),
// and each lane one 64-column pair of each row per batch (a 32-byte load; a
// warp reads 1 KB per row and batch).  The x planes of a pair are read once
// for the G rows.  The first weights are requested (into L2) before the
// kernel waits for its predecessor: they do not depend on it.

template <int NR>
__device__ __forceinline__ void dmv_loads(const uint8_t *const (&wr)[NR], const uint16_t *const (&sr)[NR], int p,
                                          bool on, uint32_t (&w)[NR][8], float (&sc)[NR])
{
#pragma unroll
    for (int k = 0; k < NR; k++) {
        if (on) {
            ld_w32(wr[k] + 32 * (size_t)p, w[k]);
            sc[k] = ld_scale(sr[k] + (p >> 1));
        } else {
#pragma unroll
            for (int q = 0; q < 8; q++) w[k][q] = 0;
            sc[k] = 0.f;
        }
    }
}

template <int NR>
__device__ __forceinline__ void dmv_dots(const Sm &s, int np, int p, const uint32_t (&w)[NR][8],
                                         const float (&sc)[NR], float (&acc)[NR])
{
    int a[NR][4];
#pragma unroll
    for (int k = 0; k < NR; k++) a[k][0] = a[k][1] = a[k][2] = a[k][3] = 0;
    // one block parity at a time: 4 x-plane vectors live, shared by the NR rows
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint4 xle = s.planes[(0 + half) * np + p], xlo = s.planes[(2 + half) * np + p];
        const uint4 xhe = s.planes[(4 + half) * np + p], xho = s.planes[(6 + half) * np + p];
        const uint32_t le[4] = {xle.x, xle.y, xle.z, xle.w}, lo[4] = {xlo.x, xlo.y, xlo.z, xlo.w};
        const uint32_t he[4] = {xhe.x, xhe.y, xhe.z, xhe.w}, ho[4] = {xho.x, xho.y, xho.z, xho.w};
#pragma unroll
        for (int k = 0; k < NR; k++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const uint32_t wv = w[k][4 * half + q];
                const uint32_t e = (wv & 0x0F0F0F0Fu) ^ 0x08080808u;     // idx^8 of even columns
                const uint32_t o = (wv & 0xF0F0F0F0u) ^ 0x80808080u;     // 16*(idx^8) of odd columns
                a[k][0] = dp_uu(e, le[q], a[k][0]);
                a[k][1] = dp_uu(o, lo[q], a[k][1]);
                a[k][2] = dp_us(e, he[q], a[k][2]);
                a[k][3] = dp_us(o, ho[q], a[k][3]);
            }
    }
    const int sx = s.psum[p];
    const float gf = s.gfac[p >> 1];
#pragma unroll
    for (int k = 0; k < NR; k++) {
        const int part = a[k][0] + (a[k][1] >> 4) + (a[k][2] + (a[k][3] >> 4)) * 256 - 8 * sx;   // a1, a3: x16
        acc[k] = fmaf((float)part, sc[k] * gf, acc[k]);
    }
}

// rows of job J in tiles [ta, tb) for this warp; NR dot products per group:
// 4 rows, or (PAIRED) 2 rows of gate and up
// rows of job J in tiles [ta, tb) for this warp; NR dot products per group:
// G rows, or (PAIRED) G/2 rows of gate and up.  The CTA's warps are split
// into rt = 8/ks row slots x ks column slices: a tile is rt rows, warp w takes
// row slot w / ks over column slice w % ks, and the ks partial sums of a row
// meet in shared memory (uniform control flow: every warp walks the same
// groups and the same number of batches).
template <bool PAIRED, int NW>
__device__ __forceinline__ void dmv_segment(const dmv_params &P, const dmv_job &J, const Sm &s, float *red,
                                            int ta, int tb, int warp, int lane, int np, size_t wpitch,
                                            unsigned long long &best)
{
    constexpr int G = PAIRED ? DMV_G / 2 : DMV_G;
    constexpr int NR = DMV_G;
    const int ks = P.ksplit, rt = NW / ks, rs = warp / ks, kq = warp % ks;
    const int npk = np / ks, p0 = kq * npk, p1 = p0 + npk;
    for (int t = ta; t < tb; t += G) {
        const int g = min(G, tb - t);
        const uint8_t *wr[NR];
        const uint16_t *sr[NR];
        int rows[G];
#pragma unroll
        for (int i = 0; i < G; i++) {
            rows[i] = (t + min(i, g - 1) - J.tile0) * rt + rs;
            const int rr = min(rows[i], J.rows - 1);            // past the end: a valid row, discarded
            if (PAIRED) {
                wr[2 * i] = J.wq + (size_t)rr * wpitch;  sr[2 * i] = J.sc + (size_t)rr * J.s_pitch;
                wr[2 * i + 1] = J.wq2 + (size_t)rr * wpitch; sr[2 * i + 1] = J.sc2 + (size_t)rr * J.s_pitch;
            } else {
                wr[i] = J.wq + (size_t)rr * wpitch; sr[i] = J.sc + (size_t)rr * J.s_pitch;
            }
        }
        float acc[NR];
#pragma unroll
        for (int k = 0; k < NR; k++) acc[k] = 0.f;
        for (int pb = p0; pb < p1; pb += 32) {
            const int p = pb + lane;
            uint32_t w[NR][8];
            float sc[NR];
            dmv_loads<NR>(wr, sr, p, p < p1, w, sc);
            if (p < p1) dmv_dots<NR>(s, np, p, w, sc, acc);
        }
        // warp totals by a transposing butterfly: 6 shuffles for 4 values
        // (10 for 2 gate/up pairs) instead of 20; lane L ends with value
        // (L >> 3) & 3 (unpaired) or the pair (L >> 4) (paired)
        const bool hi = lane & 16;
        float k0 = hi ? acc[2] : acc[0], k1 = hi ? acc[3] : acc[1];
        k0 += __shfl_xor_sync(0xffffffffu, hi ? acc[0] : acc[2], 16);
        k1 += __shfl_xor_sync(0xffffffffu, hi ? acc[1] : acc[3], 16);
        float v0, v1;
        int vi;
        bool holder;
        if (PAIRED) {
#pragma unroll
            for (int o = 8; o; o >>= 1) {
                k0 += __shfl_xor_sync(0xffffffffu, k0, o);
                k1 += __shfl_xor_sync(0xffffffffu, k1, o);
            }
            v0 = k0; v1 = k1; vi = lane >> 4; holder = (lane & 15) == 0;
        } else {
            const bool b3 = lane & 8;
            float k = b3 ? k1 : k0;
            k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
#pragma unroll
            for (int o = 4; o; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
            v0 = k; v1 = 0.f; vi = (lane >> 3) & 3; holder = (lane & 7) == 0;
        }
        if (ks > 1) {
            if (holder) {
                red[((rs * 4 + vi) * 2 + 0) * NW + kq] = v0;
                red[((rs * 4 + vi) * 2 + 1) * NW + kq] = v1;
            }
            __syncthreads();
            if (kq == 0 && holder) {
                float a = 0.f, b2 = 0.f;
                for (int q = 0; q < ks; q++) {
                    a += red[((rs * 4 + vi) * 2 + 0) * NW + q];
                    b2 += red[((rs * 4 + vi) * 2 + 1) * NW + q];
                }
                v0 = a; v1 = b2;
            }
            __syncthreads();
        }
        if (kq == 0 && holder && vi < g) {
            const int row = (t + vi - J.tile0) * rt + rs;
            if (row < J.rows) dmv_epilogue(P, J, 0, row, v0, v1, best);
        }
    }
}

// ------------------------------------------------------- the stream on mma
//
// The same integer group dot products on the tensor pipe: mma.sync
// m16n8k32 with A = 16 weight rows x 32 columns as unsigned nibble codes
// (idx ^ 8, so cb = u - 8) and B = 32 columns x 8 input vectors as the low
// (unsigned) and high (signed) bytes of the staged int16 x.  A warp owns a
// tile of 16 rows (or 8 gate/up row pairs: gate in A rows 0-7, up in 8-15)
// and walks its column slice one 128-column group at a time:
//   lane (g, t) = (lane / 4, lane % 4) loads the 16 bytes 16t .. 16t+15 of
//   rows g and g+8 in the group (one 128-bit load each); k-step s (0..3)
//   takes word s of them, i.e. columns 32t + 8s + {0..7}: low nibbles are
//   the fragment's k = 4t + i, high nibbles k = 16 + 4t + i.  The B fragment
//   of the same columns is word s of the x planes of block 4G + t (even
//   columns -> b0, odd -> b1), vector g.
// Per group: lo = -8 * sum(x) + sum(u * xlo), hi = sum(u * xhi) (exact
// int32), then acc += (lo + 256 hi) * scale * 2^-e in fp32, the contract of
// the CUDA-core path.  Lane (g, t) ends with rows g, g+8 of vectors 2t, 2t+1
// (accumulator fragment c0..c3); no lane reduction is needed.

__device__ __forceinline__ void mma_u8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16 bytes of streamed weights (read once: no L1 allocation)
__device__ __forceinline__ uint4 ld_w16(const uint8_t *p)
{
    uint4 w;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w) : "l"(p));
    return w;
}

// 4 consecutive fp16 scales (8-byte aligned)
__device__ __forceinline__ uint2 ld_sc4(const uint16_t *p)
{
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ float h2f_sel(const uint2 &v, int u)
{
    const uint32_t w = (u >> 1) ? v.y : v.x;
    return __half2float(__ushort_as_half((unsigned short)((u & 1) ? (w >> 16) : (w & 0xFFFF))));
}

__device__ __forceinline__ uint32_t u4w(const uint4 &v, int s)
{
    return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

#define DMV_U 4                    // groups per batch of loads

template <int NV, bool PAIRED, int NW>
__device__ __forceinline__ void dmv_segment_mma(const dmv_params &P, const dmv_job &J, uint8_t *sm, size_t xb,
                                                float *red4, int ta, int tb, int warp, int lane, int ng,
                                                size_t wpitch, unsigned long long (&best)[2])
{
    constexpr int TR = PAIRED ? 8 : 16;          // rows (pairs) per warp tile
    const int ks = P.ksplit, rt = NW / ks, rs = warp / ks, kq = warp % ks;
    const int ngk = ng / ks, G0 = kq * ngk, G1 = G0 + ngk;
    const int g = lane >> 2, t = lane & 3, np = P.K >> 6, nv = P.nvec;
    // B fragments: vector g (vectors past the batch read vector 0; their
    // columns are dropped); accumulator columns: vectors 2t, 2t+1
    const Sm sb = sm_layout(sm + (size_t)(NV == 1 ? 0 : min(g, nv - 1)) * xb, P.K);
    const int va = NV == 1 ? 0 : min(2 * t, nv - 1), vb = NV == 1 ? 0 : min(2 * t + 1, nv - 1);
    const int2 *gsa = sm_layout(sm + (size_t)va * xb, P.K).gs;
    const int2 *gsb = sm_layout(sm + (size_t)vb * xb, P.K).gs;
    const int par = t & 1, pq = t >> 1;
    for (int r0 = ta; r0 < tb; r0 += rt) {       // every warp the same rounds
        const int tile = r0 + rs;
        const bool on = tile < tb;
        const int base = (min(tile, tb - 1) - J.tile0) * TR;
        const int ra = min(base + g, J.rows - 1);                  // past the end: valid rows, discarded
        const int rb = PAIRED ? ra : min(base + g + 8, J.rows - 1);
        const uint8_t *pa = J.wq + (size_t)ra * wpitch + 16 * t;
        const uint8_t *pb = (PAIRED ? J.wq2 : J.wq) + (size_t)rb * wpitch + 16 * t;
        const uint16_t *qa = J.sc + (size_t)ra * J.s_pitch;
        const uint16_t *qb = (PAIRED ? J.sc2 : J.sc) + (size_t)rb * J.s_pitch;
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        if (on) {
            // batches of 4 aligned groups: one 8-byte load brings a row's 4
            // scales (rows are 16-byte aligned, s_pitch >= ceil8(K/128))
            for (int Gb = G0 & ~(DMV_U - 1); Gb < G1; Gb += DMV_U) {
                uint4 wa[DMV_U], wb[DMV_U];
                const uint2 qa4 = ld_sc4(qa + Gb), qb4 = ld_sc4(qb + Gb);
#pragma unroll
                for (int u = 0; u < DMV_U; u++) {
                    if (Gb + u >= G0 && Gb + u < G1) {
                        wa[u] = ld_w16(pa + 64 * (size_t)(Gb + u));
                        wb[u] = ld_w16(pb + 64 * (size_t)(Gb + u));
                    } else {
                        wa[u] = wb[u] = make_uint4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int u = 0; u < DMV_U; u++) {
                    if (Gb + u < G0) continue;
                    if (Gb + u >= G1) break;
                    const int G = Gb + u, p = 2 * G + pq;
                    const float sau = h2f_sel(qa4, u), sbu = h2f_sel(qb4, u);
                    const uint4 xle = sb.planes[(0 + par) * np + p], xlo = sb.planes[(2 + par) * np + p];
                    const uint4 xhe = sb.planes[(4 + par) * np + p], xho = sb.planes[(6 + par) * np + p];
                    const int2 ga = gsa[G], gb = gsb[G];
                    int lo[4] = {-8 * ga.x, -8 * gb.x, -8 * ga.x, -8 * gb.x};
                    int hi[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        const uint32_t A = u4w(wa[u], s), B = u4w(wb[u], s);
                        const uint32_t a[4] = {(A & 0x0F0F0F0Fu) ^ 0x08080808u, (B & 0x0F0F0F0Fu) ^ 0x08080808u,
                                               ((A >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u,
                                               ((B >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u};
                        mma_u8u8(lo, a, u4w(xle, s), u4w(xlo, s));
                        mma_u8s8(hi, a, u4w(xhe, s), u4w(xho, s));
                    }
                    const float fa = __int_as_float(ga.y), fb = __int_as_float(gb.y);
                    f[0] = fmaf((float)(lo[0] + 256 * hi[0]), sau * fa, f[0]);
                    f[1] = fmaf((float)(lo[1] + 256 * hi[1]), sau * fb, f[1]);
                    f[2] = fmaf((float)(lo[2] + 256 * hi[2]), sbu * fa, f[2]);
                    f[3] = fmaf((float)(lo[3] + 256 * hi[3]), sbu * fb, f[3]);
                }
            }
        }
        if (ks > 1) {
#pragma unroll
            for (int i = 0; i < 4; i++) red4[(warp * 4 + i) * 32 + lane] = f[i];
            __syncthreads();
            if (kq == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float a = 0.f;
                    for (int q = 0; q < ks; q++) a += red4[((warp + q) * 4 + i) * 32 + lane];
                    f[i] = a;
                }
            }
            __syncthreads();
        }
        if (kq == 0 && on) {
            if (PAIRED) {
                if (base + g < J.rows) {
                    if (2 * t < nv) dmv_epilogue(P, J, 2 * t, base + g, f[0], f[2], best[0]);
                    if (2 * t + 1 < nv) dmv_epilogue(P, J, 2 * t + 1, base + g, f[1], f[3], best[1]);
                }
            } else {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int row = base + g + 8 * h;
                    if (row < J.rows) {
                        if (2 * t < nv) dmv_epilogue(P, J, 2 * t, row, f[2 * h], 0.f, best[0]);
                        if (2 * t + 1 < nv) dmv_epilogue(P, J, 2 * t + 1, row, f[2 * h + 1], 0.f, best[1]);
                    }
                }
            }
        }
    }
}

// L2 prefetch of up to `budget` weight bytes of tiles [t0, t1) (the CTA's
// range of a launch), by one thread; `mma` selects the tile height
__device__ __forceinline__ void dmv_prefetch(const dmv_params &P, const dmv_job *JS, int t0, int t1, int64_t budget,
                                             bool mma, int nw)
{
    const size_t wpitch = (size_t)P.K >> 1;
    for (int t = t0; t < t1 && budget > 0;) {
        const dmv_job &J = JS[dmv_job_of(P, JS, t)];
        const int te = min(t1, J.tile0 + J.ntiles);
        const int TR = mma ? (J.wq2 ? 8 : 16) : nw / P.ksplit;
        const int r0 = (t - J.tile0) * TR;
        const int r1 = min(J.rows, (te - J.tile0) * TR);
        int64_t bytes = (int64_t)(r1 - r0) * (int64_t)wpitch;
        if (bytes > budget) bytes = budget & ~(int64_t)15;
        for (int m = 0; m < (J.wq2 ? 2 : 1); m++) {
            const uint8_t *base = (m ? J.wq2 : J.wq) + (size_t)r0 * wpitch;
            for (int64_t off = 0; off < bytes; off += 65536)
                prefetch_l2(base + off, (uint32_t)min((int64_t)65536, bytes - off));
        }
        budget -= bytes * (J.wq2 ? 2 : 1);
        t = te;
    }
}

// One CTA's share (CTA bid of nb) of a matvec launch.  NV = 1 streams on the
// CUDA cores (dp4a), NV = 2..8 on the tensor pipe (mma.sync, the same integer
// contract): one vector is cheapest as dp4a, several share each mma.
// Standalone launches (pdl) prefetch their own first weights and synchronise
// with the previous kernel; the persistent decode kernel prefetches for the
// next stage itself.  Every thread of the CTA calls it (barriers inside).
template <int NV, int NW, bool HOLD = true>
__device__ __forceinline__ void dmv_body(const dmv_params &P, uint8_t *dmv_sm, int bid, int nb, bool standalone)
{
    constexpr bool MMA = NV > 1;
    __shared__ dmv_job JS[DMV_MAXJ];
    __shared__ float red[NW * 4 * 32];
    if (threadIdx.x < P.njobs) JS[threadIdx.x] = P.jobs[threadIdx.x];
    __syncthreads();
    const int T = P.total_tiles;
    const int t0 = (int)((int64_t)bid * T / nb);
    const int t1 = (int)((int64_t)(bid + 1) * T / nb);
    const int K = P.K, np = K >> 6, ng = K >> 7;
    const size_t wpitch = (size_t)K >> 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int j0 = dmv_job_of(P, JS, min(t0, T - 1));
    if (standalone) {
        // weights do not depend on the previous kernel: ask L2 for the first
        // ones now
        if (threadIdx.x == 0 && P.pf_bytes > 0) dmv_prefetch(P, JS, t0, t1, (int64_t)P.pf_bytes * NW / 8, MMA, NW);
        pdl_trigger();
        pdl_wait();
    }
    if (t0 >= t1) return;                               // uniform over the CTA

    const size_t xb = dmv_smem_x_bytes(K);
    if (P.xst) dmv_load_staged<NW>(P.xst, dmv_sm, xb * (size_t)min(NV, P.nvec));
    else dmv_stage<NV, NW, HOLD>(P, dmv_sm, xb, t0 == 0);    // the first CTA with tiles writes the seam

    unsigned long long best[2] = {0, 0};
    for (int j = j0; j < P.njobs; j++) {
        const dmv_job &J = JS[j];
        const int ta = max(t0, J.tile0), tb = min(t1, J.tile0 + J.ntiles);
        if (ta >= tb) continue;
        if (MMA) {
            if (J.wq2) dmv_segment_mma<NV, true, NW>(P, J, dmv_sm, xb, red, ta, tb, warp, lane, ng, wpitch, best);
            else dmv_segment_mma<NV, false, NW>(P, J, dmv_sm, xb, red, ta, tb, warp, lane, ng, wpitch, best);
        } else {
            const Sm s = sm_layout(dmv_sm, K);
            if (J.wq2) dmv_segment<true, NW>(P, J, s, red, ta, tb, warp, lane, np, wpitch, best[0]);
            else dmv_segment<false, NW>(P, J, s, red, ta, tb, warp, lane, np, wpitch, best[0]);
        }
    }
    if (MMA) {
        // the argmax keys: lanes (g, t) hold vectors 2t and 2t+1; the warp's
        // maximum per vector, then one atomic per vector
#pragma unroll
        for (int h = 0; h < 2; h++) {
            unsigned long long b = best[h];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const unsigned long long c = __shfl_xor_sync(0xffffffffu, b, o);
                b = c > b ? c : b;
            }
            if (b && lane < 4 && 2 * lane + h < P.nvec) atomicMax(P.key + 2 * lane + h, b);
        }
    } else if (best[0]) {
        atomicMax(P.key, best[0]);
    }
}

// The input staging of a matvec as a launch of its own (dec_k_stage): CTA
// (cx, b) stages units [256 cx, 256 cx + 256) of vector b into the global
// block P.xst + b * xb, and every CTA of the matvec that follows copies the
// blocks (dmv_load_staged) instead of staging all vectors itself.  Same
// arithmetic as the in-CTA staging (bit-identical blocks).
__global__ void __launch_bounds__(DMV_THREADS) dmv_stage_kernel(const __grid_constant__ dmv_params P)
{
    __shared__ float gss[DMV_MAXG];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y;
    if (P.op == DMV_OP_RMSNORM) {
        dmv_group_ssq<1, DMV_WARPS>(P, b, gss);
        __syncthreads();
    }
    const int nu = P.K >> 3, u_lo = blockIdx.x * DMV_THREADS;
    dmv_stage_vec<DMV_WARPS>(P, b, P.op == DMV_OP_RMSNORM ? dmv_inv_rms(gss, P.K, P.eps) : 0.f,
                             P.xst + (size_t)b * dmv_smem_x_bytes(P.K), u_lo, min(nu, u_lo + DMV_THREADS), true);
}

template <int NV, int NW>
__global__ void __launch_bounds__(32 * NW, 16 / NW) dmv_kernel(const __grid_constant__ dmv_params P)
{
    extern __shared__ __align__(128) uint8_t dmv_sm[];
    dmv_body<NV, NW>(P, dmv_sm, blockIdx.x, gridDim.x, true);
}

// Validates a parameter block and sets its launch-dependent fields (tiles
// and the column split) for `slots` CTAs; returns the dynamic shared memory
// the kernel needs, or a negative status.
// the input side of a parameter block (prologue, vectors, staged blocks)
static int dmv_check_input(dmv_params &P)
{
    if (P.K < 128 || (P.K & 127) || P.K > 32768 || !P.x) return -11;
    if (P.op == DMV_OP_RMSNORM && !P.nw) return -11;
    if (P.op == DMV_OP_GATED && (!P.nw || !P.x2)) return -11;
    if (P.op < DMV_OP_F16 || P.op > DMV_OP_GATED) return -11;
    if (P.nvec <= 0) P.nvec = 1;
    if (P.nvec > 8 || (P.nvec > 1 && P.xs < P.K) || (P.xs & 7)) return -11;
    if (((uintptr_t)P.xst) & 15) return -11;
    return 0;
}

static long long dmv_prepare(dmv_params &P, int slots, int nw)
{
    if (P.njobs < 1 || P.njobs > DMV_MAXJ || dmv_check_input(P)) return -11;
    const bool mma = P.nvec > 1;
    const int NV = P.nvec == 1 ? 1 : P.nvec == 2 ? 2 : P.nvec <= 4 ? 4 : 8;
    const size_t smem = (size_t)NV * dmv_smem_x_bytes(P.K);
    if (smem > 200 * 1024) return -11;
    // Rows are short of warps when a CTA of nw warps would get fewer than 2 nw
    // (CUDA-core path; nw warp tiles of 16 rows on the mma path): then split
    // each row's columns over up to all nw warps of the CTA.
    long long all_rows = 0, wtiles = 0;
    for (int j = 0; j < P.njobs; j++) {
        const int r = P.jobs[j].rows > 0 ? P.jobs[j].rows : 0;
        all_rows += r;
        wtiles += (r + (P.jobs[j].wq2 ? 7 : 15)) / (P.jobs[j].wq2 ? 8 : 16);
    }
    const int np = P.K / 64, ng = P.K / 128;
    int ks = 1;
    if (mma) {
        while (ks < nw && wtiles * ks < (long long)nw * slots && (ng % (2 * ks)) == 0) ks *= 2;
    } else if (all_rows < 2LL * nw * slots) {
        while (ks < nw && np / ks > 32 && (np % (2 * ks)) == 0) ks *= 2;
    }
    P.ksplit = ks;
    const int rt = nw / ks;
    int tiles = 0;
    for (int j = 0; j < P.njobs; j++) {
        dmv_job &J = P.jobs[j];
        if (!J.wq || !J.sc || J.rows <= 0) return -11;
        if ((((uintptr_t)J.wq) & 15) || (J.wq2 && (((uintptr_t)J.wq2) & 15))) return -11;
        if ((((uintptr_t)J.sc) & 15) || (J.sc2 && (((uintptr_t)J.sc2) & 15))) return -11;
        if ((J.s_pitch & 7) || J.s_pitch < ((P.K / 128 + 7) & ~7)) return -11;
        switch (J.epi) {
        case DMV_EPI_F32: case DMV_EPI_ACC: if (!J.out_f32) return -11; break;
        case DMV_EPI_F16: if (!J.out_f16) return -11; break;
        case DMV_EPI_SWIGLU: if (!J.out_f16 || !J.wq2 || !J.sc2) return -11; break;
        case DMV_EPI_CONV: if (!J.out_f16 || !J.st || !J.p0 || J.st_stride < J.rows) return -11; break;
        case DMV_EPI_GATES: if (!J.out_f32 || !J.out2_f32 || !J.p0 || !J.p1 || J.n1 <= 0 || J.n1 > J.rows)
                                return -11;
                            break;
        case DMV_EPI_ARGMAX: if (!J.out_f32 || !P.key) return -11; break;
        default: return -11;
        }
        if (P.nvec > 1 && J.ostride < J.rows && J.epi != DMV_EPI_GATES) return -11;
        if (P.nvec > 1 && J.epi == DMV_EPI_GATES && (J.ostride < J.n1 || J.ostride < J.rows - J.n1)) return -11;
        if (J.epi != DMV_EPI_SWIGLU && J.wq2) return -11;
        J.tile0 = tiles;
        J.ntiles = mma ? (J.rows + (J.wq2 ? 7 : 15)) / (J.wq2 ? 8 : 16) : (J.rows + rt - 1) / rt;
        tiles += J.ntiles;
    }
    P.total_tiles = tiles;
    return (long long)smem;
}

extern "C" int dec_k_matvec(const dmv_params *p, void *stream, int pdl)
{
    if (!p) return -11;
    dmv_params P = *p;
    const int nvec = P.nvec <= 0 ? 1 : P.nvec;
    if (nvec > 8) return -11;
    const int NV = nvec == 1 ? 1 : nvec == 2 ? 2 : nvec <= 4 ? 4 : 8;
    const bool wide = NV == 1 && P.K >= DMV_WIDE_K;
    const int nw = wide ? 16 : 8;
    const void *fn = wide ? (const void *)dmv_kernel<1, 16> : NV == 1 ? (const void *)dmv_kernel<1, 8>
                   : NV == 2 ? (const void *)dmv_kernel<2, 8> : NV == 4 ? (const void *)dmv_kernel<4, 8>
                   : (const void *)dmv_kernel<8, 8>;
    const int fi = wide ? 4 : NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : 3;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    if (dev < 0 || dev >= 64) return -11;
    // per device and kernel instance: the SM count, and the occupancy of up
    // to 8 shared-memory sizes (the decode step uses 3 or 4)
    static int s_sms[64], s_occ[64][5][8], s_attr[64][5];
    static size_t s_occ_smem[64][5][8];
    if (!s_attr[dev][fi]) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
        s_attr[dev][fi] = 1;
    }
    const size_t smem = (size_t)NV * dmv_smem_x_bytes(P.K > 0 ? P.K : 128);
    int occ = 0;
    for (int i = 0; i < 8; i++) if (s_occ[dev][fi][i] && s_occ_smem[dev][fi][i] == smem) occ = s_occ[dev][fi][i];
    if (!occ) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, 32 * nw, smem);
        if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
        if (occ < 1) occ = 1;
        for (int i = 0; i < 8; i++)
            if (!s_occ[dev][fi][i]) { s_occ[dev][fi][i] = occ; s_occ_smem[dev][fi][i] = smem; break; }
    }
    const int slots = s_sms[dev] * occ;
    const long long rc = dmv_prepare(P, slots, nw);
    if (rc < 0) return (int)rc;
    int grid = slots;
    if (grid > P.total_tiles) grid = P.total_tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * nw);
    cfg.dynamicSmemBytes = (size_t)rc;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void *args[] = {&P};
    e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    return 0;
}

extern "C" long long dec_k_stage_bytes(int K, int nvec)
{
    if (K < 128 || (K & 127) || K > 32768 || nvec < 1 || nvec > 8) return -11;
    return (long long)nvec * (long long)dmv_smem_x_bytes(K);
}

extern "C" int dec_k_stage(const dmv_params *p, void *stream, int pdl)
{
    if (!p || !p->xst) return -11;
    dmv_params P = *p;
    if (dmv_check_input(P)) return -11;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((P.K >> 3) + DMV_THREADS - 1) / DMV_THREADS), (unsigned)P.nvec);
    cfg.blockDim = dim3(DMV_THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void *args[] = {&P};
    const cudaError_t e = cudaLaunchKernelExC(&cfg, (const void *)dmv_stage_kernel, args);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    return 0;
}
