// llm.vhdl_b200/csrc/dec_kernels.cu -- the kernels of a decode step that are
// not projections (the rest are folded into dec_matvec.cu): embedding gather,
// attention pre-processing (q/k norm, RoPE, KV-cache write), flash-decoding
// attention with its combine, the tensor-parallel residual add and the step
// advance; plus the seeded synthetic weights.  Every kernel reads the position
// from device memory so a step can be replayed from a CUDA graph, and every
// one may be launched as a programmatic dependent of the kernel before it
// (it lets the next one launch, then waits for its inputs).

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>
#include "dec_internal.h"
#include "../../include/dec_b200.h"

extern "C" int mv4i_g_cuda_err;

__device__ __forceinline__ float sigm_f(float x) { return 1.0f / (1.0f + expf(-x)); }
#ifndef DEC_PDL_HELPERS
#define DEC_PDL_HELPERS
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif
#define PDL_ENTER() do { pdl_trigger(); pdl_wait(); } while (0)

// block-wide sum (blockDim.x a multiple of 32, <= 1024); every thread calls it
__device__ __forceinline__ float block_sum(float v, float *red)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < nw ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// x[b][i] = emb[tok[b]][i] for the flat indices i0, i0 + stride, ... of the
// nseq x hidden residual
__device__ __forceinline__ void dec_embed_range(const uint16_t *emb, int hidden, const int32_t *tok, float *x,
                                                int nseq, int i0, int stride)
{
    for (int i = i0; i < nseq * hidden; i += stride) {
        const int b = i / hidden, k = i - b * hidden;
        x[i] = __half2float(__ushort_as_half(emb[(int64_t)tok[b] * hidden + k]));
    }
}

__global__ void dec_embed_kernel(const uint16_t *emb, int hidden, const int32_t *tok, float *x)
{
    PDL_ENTER();
    tok += blockIdx.y;                                   // sequence blockIdx.y of a batch
    x += (size_t)blockIdx.y * hidden;
    dec_embed_range(emb, hidden, tok, x, 1, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// One decode step of gated attention, flash-decoding part 1 with the
// pre-processing folded in (ref/run9b.c:786-869).  Grid (chunks of `ch`
// positions, kv heads); one warp per q head of the GQA group (q head h reads
// kv head h / (qh/kvh), ref/run9b.c:859).  Each CTA builds its group's q from
// the raw projection (q|gate interleaved per head): RMSNorm over the head dim
// with q_norm, NeoX RoPE on the first n_rot dims (pairs i, i + n_rot/2) at the
// current position.  The CTA whose chunk holds the current position builds k
// (k_norm, RoPE) and v the same way, stores both in the fp16 cache and uses
// them.  Then the chunk's scores (scale 1/sqrt(128)), running max, sum and
// unnormalised output per q head go to a record of 132 floats [max, sum, -,
// -, o[128]].  Head dim 128.
#define ATT_HD 128
#define ATT_KS (ATT_HD + 8)          // padded k row in shared memory (272 bytes)

// RMSNorm + RoPE of one 128-dim head held by a warp (lane: dims 4l..4l+3);
// buf is the warp's 128-float scratch
__device__ __forceinline__ void att_norm_rope(const float4 r, const float *w, float eps, int n_rot, float theta,
                                              int pos, float *buf, int lane, float (&out)[4])
{
    float ss = r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)ATT_HD + eps);
    const float4 w4 = reinterpret_cast<const float4 *>(w)[lane];
    const float v[4] = {r.x * inv * w4.x, r.y * inv * w4.y, r.z * inv * w4.z, r.w * inv * w4.w};
#pragma unroll
    for (int i = 0; i < 4; i++) buf[4 * lane + i] = v[i];
    __syncwarp();
    const int half = n_rot / 2;
    // the angle pos * theta^(-2k/n_rot) in double (8192 rad needs more than
    // float's 24 bits), reduced to [-pi, pi] in double, then single-precision
    // sine and cosine of the reduced angle (error ~1e-7)
    const double lt = 4 * lane < n_rot ? log2((double)theta) : 0.0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int d = 4 * lane + i;
        if (d < n_rot) {
            const int k = d < half ? d : d - half;
            const double th = (double)pos * exp2(-2.0 * (double)k / (double)n_rot * lt);
            const double r = th - 6.283185307179586 * rint(th * 0.15915494309189535);
            float sn, cs;
            sincosf((float)r, &sn, &cs);
            const float a = buf[k], b = buf[k + half];
            out[i] = d < half ? a * cs - b * sn : a * sn + b * cs;
        } else {
            out[i] = v[i];
        }
    }
    __syncwarp();
}

// Piece (chunk c, kv head g, sequence b) of the attention step, by `nthr`
// threads (tid < nthr; at least 32 * qh/kvh; warps past the GQA group only help
// load the chunk).  Every thread reaches the same barriers.
__device__ __forceinline__ void dec_attn_cta(const dec_attn_args &A, int c, int g, int b, int tid, int nthr, uint8_t *att_sm)
{
    const int qh = A.qh, kvh = A.kvh, max_ctx = A.max_ctx, ch = A.ch, nchunks = A.nchunks, n_rot = A.n_rot;
    const float theta = A.theta, eps = A.eps;
    const float *qg = A.qg, *kv = A.kv;
    uint16_t *kcache = A.kcache, *vcache = A.vcache;
    float *q_seam = A.q_seam, *part = A.part;
    const int grp = qh / kvh;
    const int warp = tid >> 5, lane = tid & 31;
    const bool qw_on = warp < grp;
    const int h = g * grp + (qw_on ? warp : 0);
    if (b) {
        qg += (size_t)b * 2 * qh * ATT_HD;
        kv += (size_t)b * 2 * kvh * ATT_HD;
        kcache += (size_t)b * max_ctx * kvh * ATT_HD;
        vcache += (size_t)b * max_ctx * kvh * ATT_HD;
        if (q_seam) q_seam += (size_t)b * qh * ATT_HD;
        part += (size_t)b * qh * nchunks * (ATT_HD + 4);
    }
    const int pos = *A.d_pos, len = min(pos + 1, max_ctx), p0 = c * ch;
    float *pp = part + ((size_t)h * nchunks + c) * (ATT_HD + 4);
    if (p0 >= len) {                                   // the whole CTA leaves: no barrier below
        if (qw_on && lane == 0) { pp[0] = -INFINITY; pp[1] = 0.f; }
        return;
    }
    const int n = min(ch, len - p0);
    float *qs = reinterpret_cast<float *>(att_sm);                  // [grp][128]
    float *ps = qs + grp * ATT_HD;                                  // [grp][ch]
    __half *ks = reinterpret_cast<__half *>(ps + grp * ch);         // [ch][ATT_KS]
    __half *vs = ks + ch * ATT_KS;                                  // [ch][128]
    float *kb = reinterpret_cast<float *>(vs + ch * ATT_HD);        // [128] scratch for the new k

    // the chunk's cached k and v rows: 16-byte asynchronous copies, all in
    // flight while q is built (the current position's row is replaced below)
    {
        const uint32_t kb0 = (uint32_t)__cvta_generic_to_shared(ks), vb0 = (uint32_t)__cvta_generic_to_shared(vs);
        for (int i = tid; i < n * 32; i += nthr) {
            const int r = i >> 5, piece = i & 15;
            const size_t off = ((size_t)(p0 + r) * kvh + g) * ATT_HD + 8 * piece;
            if (i & 16)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             :: "r"(vb0 + (uint32_t)(2 * (r * ATT_HD + 8 * piece))), "l"(vcache + off) : "memory");
            else
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             :: "r"(kb0 + (uint32_t)(2 * (r * ATT_KS + 8 * piece))), "l"(kcache + off) : "memory");
        }
    }
    // q of head h
    if (qw_on) {
        float q[4];
        const float4 r = reinterpret_cast<const float4 *>(qg + (size_t)h * 2 * ATT_HD)[lane];
        att_norm_rope(r, A.qn_w, eps, n_rot, theta, pos, qs + warp * ATT_HD, lane, q);
#pragma unroll
        for (int i = 0; i < 4; i++) qs[warp * ATT_HD + 4 * lane + i] = q[i];
        if (c == 0 && q_seam)
            reinterpret_cast<float4 *>(q_seam + (size_t)h * ATT_HD)[lane] = make_float4(q[0], q[1], q[2], q[3]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // the current position: new k and v of kv head g
    if (warp == 0 && pos >= p0 && pos < p0 + n) {
        float k[4];
        const float4 r = reinterpret_cast<const float4 *>(kv + (size_t)g * ATT_HD)[lane];
        att_norm_rope(r, A.kn_w, eps, n_rot, theta, pos, kb, lane, k);
        const float4 vr = reinterpret_cast<const float4 *>(kv + (size_t)(kvh + g) * ATT_HD)[lane];
        const __half2 k01 = __floats2half2_rn(k[0], k[1]), k23 = __floats2half2_rn(k[2], k[3]);
        const __half2 v01 = __floats2half2_rn(vr.x, vr.y), v23 = __floats2half2_rn(vr.z, vr.w);
        uint2 kw, vw;
        kw.x = *reinterpret_cast<const uint32_t *>(&k01); kw.y = *reinterpret_cast<const uint32_t *>(&k23);
        vw.x = *reinterpret_cast<const uint32_t *>(&v01); vw.y = *reinterpret_cast<const uint32_t *>(&v23);
        const int r0 = pos - p0;
        *reinterpret_cast<uint2 *>(ks + r0 * ATT_KS + 4 * lane) = kw;
        *reinterpret_cast<uint2 *>(vs + r0 * ATT_HD + 4 * lane) = vw;
        const size_t off = ((size_t)pos * kvh + g) * ATT_HD + 4 * lane;
        *reinterpret_cast<uint2 *>(kcache + off) = kw;
        *reinterpret_cast<uint2 *>(vcache + off) = vw;
    }
    __syncthreads();
    if (!qw_on) return;                                // no barrier below
    // scores: lanes over positions, q broadcast from shared memory
    const float scale = rsqrtf((float)ATT_HD);
    const float *qw = qs + warp * ATT_HD;
    float *pw = ps + warp * ch;
    float m = -INFINITY;
    for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        if (j < n) {
            float sc = 0.f;
#pragma unroll 4
            for (int d = 0; d < ATT_HD; d += 8) {
                const uint4 kr = *reinterpret_cast<const uint4 *>(ks + j * ATT_KS + d);
                const uint32_t kw[4] = {kr.x, kr.y, kr.z, kr.w};
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&kw[t]));
                    sc = fmaf(qw[d + 2 * t], kf.x, sc);
                    sc = fmaf(qw[d + 2 * t + 1], kf.y, sc);
                }
            }
            sc *= scale;
            pw[j] = sc;
            m = fmaxf(m, sc);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
        const float e = expf(pw[j] - m);
        pw[j] = e;
        l += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncwarp();
    // unnormalised output: lane holds dims 4l..4l+3
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int j = 0; j < n; j++) {
        const float e = pw[j];
        const uint2 vr = *reinterpret_cast<const uint2 *>(vs + j * ATT_HD + 4 * lane);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
        a0 = fmaf(e, v01.x, a0); a1 = fmaf(e, v01.y, a1); a2 = fmaf(e, v23.x, a2); a3 = fmaf(e, v23.y, a3);
    }
    if (lane == 0) { pp[0] = m; pp[1] = l; }
    reinterpret_cast<float4 *>(pp + 4)[lane] = make_float4(a0, a1, a2, a3);
}

__device__ __forceinline__ void prefetch_line(const void *p) { asm volatile("prefetch.global.L2 [%0];" :: "l"(p)); }

// The cached k and v rows of chunk c of kv head g (sequence b) up to the
// position pos_hint + 1, into L2: called before the wait for the previous
// kernel, which does not write them (pos_hint only bounds the request: a
// stale value costs a few useless lines, never a wrong result).
__device__ __forceinline__ void dec_attn_prefetch(const dec_attn_args &A, int c, int g, int b, int tid, int nthr)
{
    const int hint = *(volatile const int *)A.d_pos;
    const int p0 = c * A.ch, p1 = min(min(p0 + A.ch, hint + 2), A.max_ctx);
    const size_t base = (size_t)b * A.max_ctx * A.kvh * ATT_HD;
    for (int i = tid; i < 4 * (p1 - p0); i += nthr) {         // 4 lines a row: k and v, 256 bytes each
        const size_t off = base + ((size_t)(p0 + (i >> 2)) * A.kvh + g) * ATT_HD + 64 * (i & 1);
        prefetch_line((i & 2) ? (const void *)(A.vcache + off) : (const void *)(A.kcache + off));
    }
}

__global__ void __launch_bounds__(1024, 1) dec_attn_kernel(const dec_attn_args A)
{
    extern __shared__ __align__(16) uint8_t att_sm[];
    dec_attn_prefetch(A, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, blockDim.x);
    PDL_ENTER();
    dec_attn_cta(A, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, blockDim.x, att_sm);
}

// Flash-decoding, part 2: combine the chunks of each q head, apply the
// sigmoid output gate (the raw projection, ref/run9b.c:871-872), to fp16.
// Piece (q head h, sequence b) by NW warps (t < 32 NW) with its own scratch
// wc (at least 2 NW + NW * 128 floats): warp w takes chunks w, w + NW, ...,
// R records' loads in flight at a time (lane l holds dims 4l..4l+3), with
// its own running maximum (the online-softmax rescale); then the warps meet in
// shared memory and threads t < 128 write dimension t.  Every thread reaches
// the same barriers.
template <int NW, int R = 8>
__device__ __forceinline__ void dec_attn_combine_cta(const dec_attn_args &A, int h, int b, int t, float *wc)
{
    const int hd = ATT_HD, nchunks = A.nchunks, ch = A.ch, qh = A.qh, gate_stride = 2 * ATT_HD;
    const float *part = A.part, *gate = A.qg + ATT_HD;           // the gate: second half of each q|gate row
    uint16_t *y = A.y;
    if (b) {
        part += (size_t)b * qh * nchunks * (hd + 4);
        gate += (size_t)b * qh * gate_stride;
        y += (size_t)b * qh * hd;
    }
    const int used = min(nchunks, (*A.d_pos + 1 + ch - 1) / ch);
    const float *ph = part + (size_t)h * nchunks * (hd + 4);
    const int w = t >> 5, lane = t & 31;
    float M = -INFINITY, L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int c0 = w; c0 < used; c0 += R * NW) {
        float2 ml[R];
        float4 o[R];
#pragma unroll
        for (int k = 0; k < R; k++) {
            const int c = c0 + NW * k;
            if (c < used) {
                const float *rec = ph + (size_t)c * (hd + 4);
                ml[k] = *reinterpret_cast<const float2 *>(rec);
                o[k] = reinterpret_cast<const float4 *>(rec + 4)[lane];
            } else {
                ml[k] = make_float2(-INFINITY, 0.f);
                o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float Mn = M;
#pragma unroll
        for (int k = 0; k < R; k++) Mn = fmaxf(Mn, ml[k].x);
        const float ro = M == -INFINITY ? 0.f : expf(M - Mn);
        L *= ro; a0 *= ro; a1 *= ro; a2 *= ro; a3 *= ro;
#pragma unroll
        for (int k = 0; k < R; k++) {
            const float f = ml[k].x == -INFINITY ? 0.f : expf(ml[k].x - Mn);
            L = fmaf(ml[k].y, f, L);
            a0 = fmaf(o[k].x, f, a0); a1 = fmaf(o[k].y, f, a1); a2 = fmaf(o[k].z, f, a2); a3 = fmaf(o[k].w, f, a3);
        }
        M = Mn;
    }
    float *mw = wc, *lw = wc + NW, *aw = wc + 2 * NW;          // [NW], [NW], [NW][128]
    if (lane == 0) { mw[w] = M; lw[w] = L; }
    reinterpret_cast<float4 *>(aw + w * hd)[lane] = make_float4(a0, a1, a2, a3);
    __syncthreads();
    if (t < hd) {
        float Mx = mw[0];
#pragma unroll
        for (int i = 1; i < NW; i++) Mx = fmaxf(Mx, mw[i]);    // finite: chunk 0 is in use
        float tot = 0.f, a = 0.f;
#pragma unroll
        for (int i = 0; i < NW; i++) {
            const float f = mw[i] == -INFINITY ? 0.f : expf(mw[i] - Mx);
            tot = fmaf(lw[i], f, tot);
            a = fmaf(aw[i * hd + t], f, a);
        }
        const float gv = gate[(size_t)h * gate_stride + t];
        y[(size_t)h * hd + t] = __half_as_ushort(__float2half_rn(a / tot * sigm_f(gv)));
    }
    __syncthreads();                                       // the scratch may be reused
}

// NW warps x R records in flight: 8 x 8 (one round of loads) up to 64 chunks,
// 16 x 9 up to 144 (more warps for few chunks only lengthen the merge)
#define ATT_COMB_SPLIT 64
template <int NW, int R>
__global__ void __launch_bounds__(32 * NW) dec_attn_combine_kernel(const dec_attn_args A)
{
    __shared__ float wc[2 * NW + NW * ATT_HD];
    PDL_ENTER();
    dec_attn_combine_cta<NW, R>(A, blockIdx.x, blockIdx.y, threadIdx.x, wc);
}

__global__ void dec_add_kernel(float *x, const float *t, int n)
{
    PDL_ENTER();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] += t[i];
}

// Thread b, for sequence b of the batch: pick the largest of its `n` keys
// (one per rank, keys[r * nseq + b]), record it as the prediction at the
// current position in history[b][max_ctx], clear key[b].  The next input
// token is the prompt's while the prompt lasts (prompt[0] holds its length
// len, prompt[1 + b * len + i] sequence b's tokens), else the prediction.
// Then the shared position advances.
// by threads b < nseq of one CTA (all of its threads reach the barrier)
__device__ __forceinline__ void dec_advance_cta(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok,
                                                int32_t *history, int32_t *pos, int max_ctx, const int32_t *prompt,
                                                int b, int nseq)
{
    const int p = *pos;
    if (b < nseq) {
        unsigned long long best = 0;
        for (int i = 0; i < n; i++) best = keys[i * nseq + b] > best ? keys[i * nseq + b] : best;
        // a step whose LM head left no key (0) continues from token 0: the
        // next embedding gather never indexes outside the table
        const int32_t t = best ? (int32_t)(0xFFFFFFFFull - (best & 0xFFFFFFFFull)) : 0;
        if (p < max_ctx) history[(size_t)b * max_ctx + p] = t;
        const int plen = prompt ? prompt[0] : 0;
        tok[b] = (p + 1 < plen) ? prompt[1 + (size_t)b * plen + p + 1] : t;
        key[b] = 0;
    }
    __syncthreads();
    if (b == 0) *pos = p + 1;
}

__global__ void dec_advance_kernel(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok,
                                   int32_t *history, int32_t *pos, int max_ctx, const int32_t *prompt)
{
    PDL_ENTER();
    dec_advance_cta(keys, n, key, tok, history, pos, max_ctx, prompt, threadIdx.x, blockDim.x);
}

// --------------------------------------------------- synthetic weights

__device__ __forceinline__ uint64_t d_mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t d_draw(uint64_t key, uint64_t i)
{ return d_mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL); }

// INT4 g128 shard: local row r is global row rows[r] (or row0 + r when rows is
// NULL); local columns [0, kn) are global columns [k0, k0+kn) of a Kg-column
// matrix; scales at row pitch s_pitch.  Same draws as mv4i_synth_g128 for the
// same key and global index.
__global__ void dec_synth_linear_kernel(uint64_t key, const int32_t *rows, int row0, int nrows, int k0, int kn,
                                        int Kg, uint8_t *wq, uint16_t *sc, int s_pitch)
{
    const int64_t nb = (int64_t)nrows * (kn / 2);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nb; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / (kn / 2), c = i % (kn / 2);
        const int64_t gr = rows ? rows[r] : row0 + r;
        const uint64_t base = (uint64_t)gr * Kg + k0 + 2 * c;
        const uint64_t lo = d_draw(3 * key, base) >> 60, hi = d_draw(3 * key, base + 1) >> 60;
        wq[i] = (uint8_t)(lo | (hi << 4));
    }
    const int ng = kn / 128, ngg = Kg / 128;
    const int64_t ns = (int64_t)nrows * ng;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ns; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ng, g = i % ng;
        const int64_t gr = rows ? rows[r] : row0 + r;
        const double u = (double)(d_draw(3 * key + 1, (uint64_t)gr * ngg + k0 / 128 + g) >> 11) * 0x1.0p-53;
        sc[r * s_pitch + g] = __half_as_ushort(__float2half_rn((float)(0.002 + 0.018 * u)));
    }
}

// fp32 / fp16 parameter vectors: value = mean + std * N(0,1) (Box-Muller);
// global index gi = idx0 + i (or idx[i]).
__global__ void dec_synth_vec_kernel(uint64_t key, const int32_t *idx, int64_t idx0, int64_t n, float mean, float std,
                                     float *f32, uint16_t *f16)
{
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t gi = idx ? (uint64_t)idx[i] : (uint64_t)(idx0 + i);
        const double u1 = ((double)(d_draw(key, 2 * gi) >> 11) + 1.0) * 0x1.0p-53;
        const double u2 = (double)(d_draw(key, 2 * gi + 1) >> 11) * 0x1.0p-53;
        const float v = mean + std * (float)(sqrt(-2.0 * log(u1)) * cospi(2.0 * u2));
        if (f32) f32[i] = v;
        if (f16) f16[i] = __half_as_ushort(__float2half_rn(v));
    }
}

// ------------------------------------------------------------ launchers

static int dk(cudaError_t e) { if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; } return 0; }

// launch on `s`, as a programmatic dependent of the previous kernel when pdl
template <typename... KArgs, typename... Args>
static int launch(void (*k)(KArgs...), dim3 g, dim3 b, void *s, int pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = b;
    cfg.stream = reinterpret_cast<cudaStream_t>(s);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return dk(cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...));
}

extern "C" {

int dec_k_embed(const uint16_t *emb, int hidden, const int32_t *tok, float *x, int nseq, void *s, int pdl)
{ return launch(dec_embed_kernel, dim3((hidden + 255) / 256, nseq), dim3(256), s, pdl, emb, hidden, tok, x); }

size_t dec_attention_smem(int qh, int kvh, int ch)
{
    const int grp = qh / kvh;
    return (size_t)(grp * ATT_HD + grp * ch) * 4 + (size_t)ch * ATT_KS * 2 + (size_t)ch * ATT_HD * 2 + ATT_HD * 4;
}

int dec_attn_prepare(dec_attn_args *A)
{
    if (A->kvh <= 0 || A->qh % A->kvh || A->qh / A->kvh > 32 || A->ch <= 0 || A->ch > 64 || (A->n_rot & 1)
        || A->n_rot > ATT_HD || A->nseq < 1 || A->nseq > 64) return -11;
    A->nchunks = (A->max_ctx + A->ch - 1) / A->ch;
    if (A->nchunks > 1024) return -11;                // at most 65536 positions of 64
    return 0;
}

int dec_k_attention(const float *qg, const float *kv, const float *qn_w, const float *kn_w, int qh, int kvh,
                    int n_rot, float theta, float eps, const int32_t *d_pos, int max_ctx, int ch, float *part,
                    float *q_seam, uint16_t *kcache, uint16_t *vcache, uint16_t *y, int nseq, void *s, int pdl)
{
    dec_attn_args A = {qg, kv, qn_w, kn_w, qh, kvh, n_rot, theta, eps, d_pos, max_ctx, ch, 0, kcache, vcache,
                       q_seam, part, y, nseq};
    int rc = dec_attn_prepare(&A);
    if (rc) return rc;
    const size_t smem = dec_attention_smem(qh, kvh, ch);
    static int attr_set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -11;
    if (!attr_set[dev]) {
        rc = dk(cudaFuncSetAttribute(dec_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
        if (rc) return rc;
        attr_set[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(A.nchunks, kvh, nseq);
    cfg.blockDim = dim3(32 * (qh / kvh));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = reinterpret_cast<cudaStream_t>(s);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    rc = dk(cudaLaunchKernelEx(&cfg, dec_attn_kernel, A));
    if (rc) return rc;
    if (A.nchunks <= ATT_COMB_SPLIT) return launch(dec_attn_combine_kernel<8, 8>, dim3(qh, nseq), dim3(256), s, pdl, A);
    return launch(dec_attn_combine_kernel<16, 9>, dim3(qh, nseq), dim3(512), s, pdl, A);
}

int dec_k_add(float *x, const float *t, int n, void *s, int pdl)
{ return launch(dec_add_kernel, dim3((n + 255) / 256), dim3(256), s, pdl, x, t, n); }

int dec_k_advance(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok, int32_t *hist,
                  int32_t *pos, int max_ctx, const int32_t *prompt, int nseq, void *s, int pdl)
{ return launch(dec_advance_kernel, dim3(1), dim3(nseq), s, pdl, keys, n, key, tok, hist, pos, max_ctx, prompt); }

int dec_k_synth_linear(uint64_t key, const int32_t *rows, int row0, int nrows, int k0, int kn, int Kg,
                       uint8_t *wq, uint16_t *sc, int s_pitch, void *s)
{
    return launch(dec_synth_linear_kernel, dim3(148 * 8), dim3(256), s, 0, key, rows, row0, nrows, k0, kn, Kg, wq,
                  sc, s_pitch);
}

int dec_k_synth_vec(uint64_t key, const int32_t *idx, int64_t idx0, int64_t n, float mean, float std,
                    float *f32, uint16_t *f16, void *s)
{ return launch(dec_synth_vec_kernel, dim3(148 * 4), dim3(256), s, 0, key, idx, idx0, n, mean, std, f32, f16); }

}  // extern "C"

// ------------------------------------------------- peer-memory exchange
//
// Tensor-parallel all-reduce of the row-parallel partial sums and all-gather
// of the argmax keys over NVLink with plain peer stores (no NCCL, no
// multicast).  Every rank owns one exchange region, mapped by every peer:
//   xbuf  float [2][world][hidden]   partial sums, by epoch parity and sender
//   keys  u64   [2][world]           argmax keys
//   xflag u32   [2][world][nslices]  epoch stamps, one per (sender, slice)
//   kflag u32   [2][world]
// An exchange with epoch E (a per-rank device counter, identical on all
// ranks because every rank runs the same sequence) writes buffer E & 1; a
// rank can reach epoch E + 2 only after every peer has stamped epoch E + 1,
// which each peer does after it finished reading its epoch-E buffer, so two
// buffers suffice.  Waits are bounded: after `spin_limit` polls the kernel
// records the failure in `err` and carries on (the step's output is then
// garbage; the host reads `err`).
#define X_SLICE 512                      // floats per CTA of the all-reduce

struct PeerRegion {
    float *xbuf[8];                      // each rank's region, as mapped here
    unsigned long long *keys[8];
    uint32_t *xflag[8], *kflag[8];
};

__device__ __forceinline__ void st_release(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// x[slice] += sum over ranks of their partial t[slice]; one CTA per slice of
// X_SLICE floats, X_SLICE/4 threads
__global__ void __launch_bounds__(X_SLICE / 4) dec_ar_kernel(const __grid_constant__ PeerRegion R, int rank,
                                                             int world, int hidden, const float *t, float *x,
                                                             uint32_t *epoch, uint32_t *done, int *err,
                                                             int spin_limit)
{
    PDL_ENTER();
    const int i = blockIdx.x, tid = threadIdx.x, ns = gridDim.x;
    const uint32_t E = *(volatile uint32_t *)epoch + 1u;
    const int par = E & 1;
    const int base = i * X_SLICE + 4 * tid;
    const bool on = base < hidden;
    float4 mine = make_float4(0.f, 0.f, 0.f, 0.f);
    if (on) mine = *reinterpret_cast<const float4 *>(t + base);
    for (int r = 0; r < world; r++)
        if (on) *reinterpret_cast<float4 *>(R.xbuf[r] + ((size_t)par * world + rank) * hidden + base) = mine;
    __threadfence_system();
    __syncthreads();
    if (tid < world) st_release(R.xflag[tid] + ((size_t)par * world + rank) * ns + i, E);
    if (tid < world) {
        const uint32_t *f = R.xflag[rank] + ((size_t)par * world + tid) * ns + i;
        int n = 0;
        while (ld_acquire(f) != E) {
            if (++n > spin_limit) { atomicOr(err, 1); break; }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (on) {
        float4 a = *reinterpret_cast<const float4 *>(x + base);
        for (int r = 0; r < world; r++) {
            const float4 p = __ldcv(reinterpret_cast<const float4 *>(R.xbuf[rank] + ((size_t)par * world + r) * hidden + base));
            a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
        }
        *reinterpret_cast<float4 *>(x + base) = a;
    }
    __syncthreads();
    if (tid == 0 && atomicAdd(done, 1u) == (uint32_t)ns - 1) { *done = 0; *epoch = E; }
}

// the step advance with the argmax keys exchanged through peer memory
__global__ void dec_advance_p2p_kernel(const __grid_constant__ PeerRegion R, int rank, int world,
                                       unsigned long long *key, int32_t *tok, int32_t *history, int32_t *pos,
                                       int max_ctx, const int32_t *prompt, uint32_t *epoch, int *err,
                                       int spin_limit)
{
    PDL_ENTER();
    const uint32_t E = *epoch + 1u;
    const int par = E & 1;
    const unsigned long long mine = *key;
    for (int r = 0; r < world; r++) R.keys[r][par * world + rank] = mine;
    __threadfence_system();
    for (int r = 0; r < world; r++) st_release(R.kflag[r] + par * world + rank, E);
    unsigned long long best = 0;
    for (int r = 0; r < world; r++) {
        const uint32_t *f = R.kflag[rank] + par * world + r;
        int n = 0;
        while (ld_acquire(f) != E) {
            if (++n > spin_limit) { atomicOr(err, 2); break; }
            __nanosleep(64);
        }
        const unsigned long long k = *(volatile unsigned long long *)(R.keys[rank] + par * world + r);
        best = k > best ? k : best;
    }
    *epoch = E;
    const int32_t tk = best ? (int32_t)(0xFFFFFFFFull - (best & 0xFFFFFFFFull)) : 0;   // no key: token 0
    const int p = *pos;
    if (p < max_ctx) history[p] = tk;
    const int plen = prompt ? prompt[0] : 0;
    *tok = (p + 1 < plen) ? prompt[1 + p + 1] : tk;
    *pos = p + 1;
    *key = 0;
}

extern "C" {

// bytes of one exchange region and the offsets of its parts
size_t dec_p2p_region(int world, int hidden, size_t *off_keys, size_t *off_xflag, size_t *off_kflag)
{
    const int ns = (hidden + X_SLICE - 1) / X_SLICE;
    size_t o = (size_t)2 * world * hidden * 4;
    o = (o + 127) & ~(size_t)127;
    if (off_keys) *off_keys = o;
    o += (size_t)2 * world * 8;
    o = (o + 127) & ~(size_t)127;
    if (off_xflag) *off_xflag = o;
    o += (size_t)2 * world * ns * 4;
    o = (o + 127) & ~(size_t)127;
    if (off_kflag) *off_kflag = o;
    o += (size_t)2 * world * 4;
    return (o + 127) & ~(size_t)127;
}

int dec_k_allreduce_p2p(void *const *regions, int rank, int world, int hidden, const float *t, float *x,
                        uint32_t *epoch, uint32_t *done, int *err, int spin_limit, void *s, int pdl)
{
    if (world < 1 || world > 8 || (hidden & 3)) return -11;
    size_t ok, oxf, okf;
    dec_p2p_region(world, hidden, &ok, &oxf, &okf);
    PeerRegion R = {};
    for (int r = 0; r < world; r++) {
        uint8_t *b = (uint8_t *)regions[r];
        R.xbuf[r] = (float *)b;
        R.keys[r] = (unsigned long long *)(b + ok);
        R.xflag[r] = (uint32_t *)(b + oxf);
        R.kflag[r] = (uint32_t *)(b + okf);
    }
    const int ns = (hidden + X_SLICE - 1) / X_SLICE;
    return launch(dec_ar_kernel, dim3(ns), dim3(X_SLICE / 4), s, pdl, R, rank, world, hidden, t, x, epoch, done,
                  err, spin_limit);
}

int dec_k_advance_p2p(void *const *regions, int rank, int world, int hidden, unsigned long long *key,
                      int32_t *tok, int32_t *hist, int32_t *pos, int max_ctx, const int32_t *prompt,
                      uint32_t *epoch, int *err, int spin_limit, void *s, int pdl)
{
    if (world < 1 || world > 8) return -11;
    size_t ok, oxf, okf;
    dec_p2p_region(world, hidden, &ok, &oxf, &okf);
    PeerRegion R = {};
    for (int r = 0; r < world; r++) {
        uint8_t *b = (uint8_t *)regions[r];
        R.xbuf[r] = (float *)b;
        R.keys[r] = (unsigned long long *)(b + ok);
        R.xflag[r] = (uint32_t *)(b + oxf);
        R.kflag[r] = (uint32_t *)(b + okf);
    }
    return launch(dec_advance_p2p_kernel, dim3(1), dim3(1), s, pdl, R, rank, world, key, tok, hist, pos, max_ctx,
                  prompt, epoch, err, spin_limit);
}

}  // extern "C"

// the public one-token entry (include/dec_b200.h): chunks of 16 positions up
// to a 2048-position cache, 32 up to 6144, 64 beyond (the decode step's choice
// for one sequence)
static int gated_attn_chunk(int max_ctx) { return max_ctx <= 2048 ? 16 : (max_ctx <= 6144 ? 32 : 64); }

extern "C" size_t gated_attn_work_bytes(int n_qh, int max_ctx)
{
    if (n_qh <= 0 || max_ctx <= 0 || max_ctx > 65536) return 0;
    const int ch = gated_attn_chunk(max_ctx);
    return (size_t)4 * n_qh * ((max_ctx + ch - 1) / ch) * (ATT_HD + 4);
}

extern "C" int gated_attn(const gated_attn_args *a, void *stream)
{
    if (!a || a->head_dim != ATT_HD || a->n_qh <= 0 || a->n_kvh <= 0 || !a->qg || !a->kv || !a->q_norm
        || !a->k_norm || !a->d_pos || !a->kcache || !a->vcache || !a->y || !a->work || a->max_ctx <= 0
        || a->max_ctx > 65536)
        return -11;
    if ((((uintptr_t)a->qg) | ((uintptr_t)a->kv) | ((uintptr_t)a->q_norm) | ((uintptr_t)a->k_norm)
         | ((uintptr_t)a->kcache) | ((uintptr_t)a->vcache) | ((uintptr_t)a->work)) & 15)
        return -11;
    return dec_k_attention(a->qg, a->kv, a->q_norm, a->k_norm, a->n_qh, a->n_kvh, a->n_rot, a->rope_theta, a->eps,
                           a->d_pos, a->max_ctx, gated_attn_chunk(a->max_ctx), (float *)a->work, a->q_out,
                           a->kcache, a->vcache, a->y, 1, stream, a->pdl);
}
