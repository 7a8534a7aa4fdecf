// llm.vhdl_b200/csrc/gdn_f32_step.cuh -- the binary32 Gated DeltaNet step of
// one CTA-sized piece of work (128 threads: 16 value columns of one head),
// shared by gdn_f32_kernel (gdn_kernels.cu) and the persistent decode kernel
// (dec_step.cu).  The recurrence is ref/gdn_err.c:580-590 (decay first, delta
// rule, o = S^T q after the update); see gdn_kernels.cu for the work split.
#ifndef GDN_F32_STEP_CUH
#define GDN_F32_STEP_CUH

#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>
#include "../../include/gdn_b200.h"

__device__ __forceinline__ float gdn_sum8(float v)
{
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

struct GdnStepIn {
    uint32_t k[8], q[8];        // 16 fp16 keys of this lane's slice (packed pairs)
    uint16_t v, g;              // this column's v and gate
    float a, b;                 // the head's decay and beta inputs
};

// PLAIN: ordinary loads (inputs written earlier in the same kernel, as in the
// persistent decode kernel); otherwise the read-only path
template <bool PLAIN, typename T>
__device__ __forceinline__ T gdn_ld(const T *p) { if (PLAIN) return *p; else return __ldg(p); }

template <bool PLAIN>
__device__ __forceinline__ void gdn_load_step(const gdn_f32_args &A, int t, int h, int hk, int j, int i0,
                                              GdnStepIn &s)
{
    const size_t kq = ((size_t)t * A.KH + hk) * 128 + i0;
    const uint4 *kp = reinterpret_cast<const uint4 *>(A.k + kq), *qp = reinterpret_cast<const uint4 *>(A.q + kq);
    const uint4 k0 = gdn_ld<PLAIN>(kp), k1 = gdn_ld<PLAIN>(kp + 1), q0 = gdn_ld<PLAIN>(qp), q1 = gdn_ld<PLAIN>(qp + 1);
    s.k[0] = k0.x; s.k[1] = k0.y; s.k[2] = k0.z; s.k[3] = k0.w; s.k[4] = k1.x; s.k[5] = k1.y; s.k[6] = k1.z; s.k[7] = k1.w;
    s.q[0] = q0.x; s.q[1] = q0.y; s.q[2] = q0.z; s.q[3] = q0.w; s.q[4] = q1.x; s.q[5] = q1.y; s.q[6] = q1.z; s.q[7] = q1.w;
    const size_t vj = ((size_t)t * A.H + h) * 128 + j;
    s.v = gdn_ld<PLAIN>(A.v + vj);
    s.g = A.g ? gdn_ld<PLAIN>(A.g + vj) : (uint16_t)0;
    s.a = A.eg ? gdn_ld<PLAIN>(A.eg + (size_t)t * A.H + h) : gdn_ld<PLAIN>(A.a + (size_t)t * A.H + h);
    s.b = A.beta ? gdn_ld<PLAIN>(A.beta + (size_t)t * A.H + h) : gdn_ld<PLAIN>(A.b + (size_t)t * A.H + h);
}

// Piece (bx, by) of a launch over (H x 8, nseq): sequence by, head bx / 8,
// value columns 16 (bx % 8) .. +15; tid in [0, 128).  A.T steps with the
// state column slice in registers.
template <bool PLAIN>
__device__ __forceinline__ void gdn_f32_cta(const gdn_f32_args &A0, int bx, int by, int tid)
{
    gdn_f32_args A = A0;
    if (by) {
        const size_t n = by, hd = (size_t)A.H * 128;
        A.q += n * A.seq_in; A.k += n * A.seq_in; A.v += n * A.seq_in;
        if (A.g) A.g += n * hd;
        if (A.a) A.a += n * A.H;
        if (A.b) A.b += n * A.H;
        if (A.eg) A.eg += n * A.H;
        if (A.beta) A.beta += n * A.H;
        if (A.out_f32) A.out_f32 += n * hd;
        if (A.out_f16) A.out_f16 += n * hd;
        A.S += n * hd * 128;
    }
    const int h = bx >> 3;
    const int warp = tid >> 5, lane = tid & 31;
    const int j = (bx & 7) * 16 + warp * 4 + (lane >> 3);
    const int sl = lane & 7, i0 = 16 * sl;
    const int hk = h % A.KH;
    float *scol = A.S + ((size_t)h * 128 + j) * 128 + i0;
    float s[16];
#pragma unroll
    for (int t4 = 0; t4 < 4; t4++) {
        const float4 v = reinterpret_cast<const float4 *>(scol)[t4];
        s[4 * t4] = v.x; s[4 * t4 + 1] = v.y; s[4 * t4 + 2] = v.z; s[4 * t4 + 3] = v.w;
    }
    GdnStepIn cur, nxt;
    gdn_load_step<PLAIN>(A, 0, h, hk, j, i0, cur);
    for (int t = 0; t < A.T; t++) {
        if (t + 1 < A.T) gdn_load_step<PLAIN>(A, t + 1, h, hk, j, i0, nxt);
        float kf[16], qf[16];
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const float2 kk = __half22float2(*reinterpret_cast<const __half2 *>(&cur.k[p]));
            const float2 qq = __half22float2(*reinterpret_cast<const __half2 *>(&cur.q[p]));
            kf[2 * p] = kk.x; kf[2 * p + 1] = kk.y; qf[2 * p] = qq.x; qf[2 * p + 1] = qq.y;
        }
        if (A.l2norm) {
            float nk = 0.f, nq = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) { nk = fmaf(kf[i], kf[i], nk); nq = fmaf(qf[i], qf[i], nq); }
            nk = gdn_sum8(nk);
            nq = gdn_sum8(nq);
            const float rk = 1.0f / fmaxf(sqrtf(nk), 1e-12f), rq = A.q_scale / fmaxf(sqrtf(nq), 1e-12f);
#pragma unroll
            for (int i = 0; i < 16; i++) { kf[i] *= rk; qf[i] *= rq; }
        } else if (A.q_scale != 1.0f) {
#pragma unroll
            for (int i = 0; i < 16; i++) qf[i] *= A.q_scale;
        }
        float alpha, beta;
        if (A.eg) { alpha = cur.a; beta = cur.b; }
        else {
            const float sp = cur.a > 30.f ? cur.a : log1pf(expf(cur.a));
            alpha = expf(-sp);
            beta = 1.0f / (1.0f + expf(-cur.b));
        }
        float sk0 = 0.f, sk1 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            s[i] *= alpha; s[i + 1] *= alpha;
            sk0 = fmaf(s[i], kf[i], sk0); sk1 = fmaf(s[i + 1], kf[i + 1], sk1);
        }
        const float sk = gdn_sum8(sk0 + sk1);
        const float d = (__half2float(__ushort_as_half(cur.v)) - sk) * beta;
        float o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            s[i] = fmaf(kf[i], d, s[i]); s[i + 1] = fmaf(kf[i + 1], d, s[i + 1]);
            o0 = fmaf(s[i], qf[i], o0); o1 = fmaf(s[i + 1], qf[i + 1], o1);
        }
        float o = gdn_sum8(o0 + o1);
        if (A.g) o = o / (1.0f + expf(-__half2float(__ushort_as_half(cur.g))));
        if (sl == 0) {
            const size_t oj = ((size_t)t * A.H + h) * 128 + j;
            if (A.out_f32) A.out_f32[oj] = o;
            if (A.out_f16) A.out_f16[oj] = __half_as_ushort(__float2half_rn(o));
        }
        cur = nxt;
    }
#pragma unroll
    for (int t4 = 0; t4 < 4; t4++)
        reinterpret_cast<float4 *>(scol)[t4] = make_float4(s[4 * t4], s[4 * t4 + 1], s[4 * t4 + 2], s[4 * t4 + 3]);
}

#endif
