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

extern "C" int mv4i_g_cuda_err;

__device__ __forceinline__ float sigm_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
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

__global__ void dec_embed_kernel(const uint16_t *emb, int hidden, const int32_t *tok, float *x)
{
    PDL_ENTER();
    const int64_t base = (int64_t)(*tok) * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        x[i] = __half2float(__ushort_as_half(emb[base + i]));
}

// Attention pre-processing (ref/run9b.c:786-843): q|gate interleaved per
// head, q and k RMSNorm over the head dim, NeoX RoPE on the first n_rot
// dims (pairs i, i + n_rot/2), k and v into the fp16 cache at the current
// position.  One CTA per q head, then one per k head; hd threads.
__global__ void dec_attn_pre_kernel(const float *qg, const float *kv, int qh, int kvh, int hd, int n_rot,
                                    float theta, float eps, const float *qn_w, const float *kn_w,
                                    const int32_t *d_pos, int max_ctx, float *q_out, float *gate_out,
                                    uint16_t *kcache, uint16_t *vcache)
{
    __shared__ float red[32];
    __shared__ float buf[512];
    PDL_ENTER();
    const int hb = blockIdx.x, i = threadIdx.x;
    const int pos = *d_pos;
    const bool isq = hb < qh;
    const int h = isq ? hb : hb - qh;
    const float *src = isq ? qg + (size_t)h * 2 * hd : kv + (size_t)h * hd;
    const float v = i < hd ? src[i] : 0.f;
    const float s = block_sum(v * v, red);
    const float inv = rsqrtf(s / (float)hd + eps);
    if (i < hd) buf[i] = v * inv * (isq ? qn_w[i] : kn_w[i]);
    __syncthreads();
    float r = i < hd ? buf[i] : 0.f;
    const int half = n_rot / 2;
    if (i < n_rot) {
        const int k = i < half ? i : i - half;
        const double th = (double)pos * exp2(-2.0 * (double)k / (double)n_rot * log2((double)theta));
        double sn, cs;
        sincos(th, &sn, &cs);
        const float a = buf[k], b = buf[k + half];
        r = i < half ? (float)(a * cs - b * sn) : (float)(a * sn + b * cs);
    }
    if (i < hd) {
        if (isq) {
            q_out[(size_t)h * hd + i] = r;
            gate_out[(size_t)h * hd + i] = qg[(size_t)h * 2 * hd + hd + i];
        } else if (pos < max_ctx) {          // a full cache takes no more entries
            const size_t off = ((size_t)pos * kvh + h) * hd + i;
            kcache[off] = __half_as_ushort(__float2half_rn(r));
            vcache[off] = __half_as_ushort(__float2half_rn(kv[(size_t)(kvh + h) * hd + i]));
        }
    }
}

// Flash-decoding, part 1: CTA (chunk c of `ch` positions, kv head g), one warp
// per q head of the group (q head h uses kv head h / (qh/kvh),
// ref/run9b.c:859); lane l holds dims 4l..4l+3 (hd = 128).  Writes the
// chunk's running max, sum and unnormalised output per q head into a record
// of hd + 4 floats (max, sum, 2 unused, then hd sums: 16-byte aligned).
__global__ void dec_attn_decode_kernel(const float *q, const uint16_t *kcache, const uint16_t *vcache,
                                       int qh, int kvh, int hd, int ch, const int32_t *d_pos, int max_ctx,
                                       int nchunks, float *part)
{
    PDL_ENTER();
    const int c = blockIdx.x, g = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = qh / kvh, h = g * grp + warp;
    const int len = min(*d_pos + 1, max_ctx);
    const int p0 = c * ch;
    float *pp = part + ((size_t)h * nchunks + c) * (hd + 4);
    if (p0 >= len) {
        if (lane == 0) { pp[0] = -INFINITY; pp[1] = 0.f; }
        return;
    }
    const float scale = rsqrtf((float)hd);
    const float4 qv = reinterpret_cast<const float4 *>(q + (size_t)h * hd)[lane];
    float m = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const int p1 = min(len, p0 + ch);
    for (int p = p0; p < p1; p++) {
        const size_t off = ((size_t)p * kvh + g) * hd + 4 * lane;
        const uint2 kr = *reinterpret_cast<const uint2 *>(kcache + off);
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.x));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.y));
        float s = qv.x * k01.x + qv.y * k01.y + qv.z * k23.x + qv.w * k23.y;
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        s *= scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), e = expf(s - mn);
        const uint2 vr = *reinterpret_cast<const uint2 *>(vcache + off);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
        a0 = a0 * corr + e * v01.x; a1 = a1 * corr + e * v01.y;
        a2 = a2 * corr + e * v23.x; a3 = a3 * corr + e * v23.y;
        l = l * corr + e;
        m = mn;
    }
    if (lane == 0) { pp[0] = m; pp[1] = l; }
    reinterpret_cast<float4 *>(pp + 4)[lane] = make_float4(a0, a1, a2, a3);
}

// Flash-decoding, part 2: combine the chunks of each q head, apply the
// sigmoid output gate (the raw projection, ref/run9b.c:871-872), to fp16.
__global__ void dec_attn_combine_kernel(const float *part, const float *gate, int hd, int nchunks,
                                        const int32_t *d_pos, int ch, uint16_t *y)
{
    PDL_ENTER();
    const int h = blockIdx.x, lane = threadIdx.x;     // 32 threads, 4 dims each
    const int used = min(nchunks, (*d_pos + 1 + ch - 1) / ch);
    float M = -INFINITY;
    for (int c = 0; c < used; c++) M = fmaxf(M, part[((size_t)h * nchunks + c) * (hd + 4)]);
    float L = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int c = 0; c < used; c++) {
        const float *pp = part + ((size_t)h * nchunks + c) * (hd + 4);
        const float w = expf(pp[0] - M);
        L += pp[1] * w;
        const float4 a = reinterpret_cast<const float4 *>(pp + 4)[lane];
        a0 += a.x * w; a1 += a.y * w; a2 += a.z * w; a3 += a.w * w;
    }
    const float inv = 1.0f / L;
    const float4 gv = reinterpret_cast<const float4 *>(gate + (size_t)h * hd)[lane];
    uint16_t *yo = y + (size_t)h * hd + 4 * lane;
    yo[0] = __half_as_ushort(__float2half_rn(a0 * inv * sigm_f(gv.x)));
    yo[1] = __half_as_ushort(__float2half_rn(a1 * inv * sigm_f(gv.y)));
    yo[2] = __half_as_ushort(__float2half_rn(a2 * inv * sigm_f(gv.z)));
    yo[3] = __half_as_ushort(__float2half_rn(a3 * inv * sigm_f(gv.w)));
}

__global__ void dec_add_kernel(float *x, const float *t, int n)
{
    PDL_ENTER();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] += t[i];
}

// Pick the largest of `n` keys (one per rank), record it as the prediction
// at the current position, advance the position, clear `key`.  The next
// input token is the prompt's while the prompt lasts (prompt[0] holds its
// length, prompt[1 + i] its tokens), else the prediction.
__global__ void dec_advance_kernel(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok,
                                   int32_t *history, int32_t *pos, int max_ctx, const int32_t *prompt)
{
    PDL_ENTER();
    unsigned long long best = 0;
    for (int i = 0; i < n; i++) best = keys[i] > best ? keys[i] : best;
    const int32_t t = (int32_t)(0xFFFFFFFFull - (best & 0xFFFFFFFFull));
    const int p = *pos;
    if (p < max_ctx) history[p] = t;
    const int plen = prompt ? prompt[0] : 0;
    *tok = (p + 1 < plen) ? prompt[1 + p + 1] : t;
    *pos = p + 1;
    *key = 0;
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

int dec_k_embed(const uint16_t *emb, int hidden, const int32_t *tok, float *x, void *s, int pdl)
{ return launch(dec_embed_kernel, dim3((hidden + 255) / 256), dim3(256), s, pdl, emb, hidden, tok, x); }

int dec_k_attn_pre(const float *qg, const float *kv, int qh, int kvh, int hd, int n_rot, float theta, float eps,
                   const float *qn_w, const float *kn_w, const int32_t *d_pos, int max_ctx, float *q_out,
                   float *gate_out, uint16_t *kcache, uint16_t *vcache, void *s, int pdl)
{
    return launch(dec_attn_pre_kernel, dim3(qh + kvh), dim3(((hd + 31) / 32) * 32), s, pdl, qg, kv, qh, kvh, hd,
                  n_rot, theta, eps, qn_w, kn_w, d_pos, max_ctx, q_out, gate_out, kcache, vcache);
}

int dec_k_attention(const float *q, const uint16_t *kc, const uint16_t *vc, int qh, int kvh, int hd, int ch,
                    int max_ctx, const int32_t *d_pos, float *part, const float *gate, uint16_t *y, void *s, int pdl)
{
    const int nchunks = (max_ctx + ch - 1) / ch;
    int rc = launch(dec_attn_decode_kernel, dim3(nchunks, kvh), dim3(32 * (qh / kvh)), s, pdl, q, kc, vc, qh, kvh,
                    hd, ch, d_pos, max_ctx, nchunks, part);
    if (rc) return rc;
    return launch(dec_attn_combine_kernel, dim3(qh), dim3(32), s, pdl, part, gate, hd, nchunks, d_pos, ch, y);
}

int dec_k_add(float *x, const float *t, int n, void *s, int pdl)
{ return launch(dec_add_kernel, dim3((n + 255) / 256), dim3(256), s, pdl, x, t, n); }

int dec_k_advance(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok, int32_t *hist,
                  int32_t *pos, int max_ctx, const int32_t *prompt, void *s, int pdl)
{ return launch(dec_advance_kernel, dim3(1), dim3(1), s, pdl, keys, n, key, tok, hist, pos, max_ctx, prompt); }

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
