// llm.vhdl_b200/csrc/dec_kernels.cu -- the small kernels between projections
// in a decode step (the vector ops of ref/run9b.c's layer_gdn / layer_attn):
// embedding gather, RMSNorm to fp16, the DeltaNet conv + SiLU + gate
// activations, the gated output norm, attention pre-processing (q/k norm,
// RoPE, KV-cache write), flash-decoding attention with its combine, SwiGLU,
// residual add, the argmax key and the step advance.  Every kernel reads the
// position from device memory so a step can be replayed from a CUDA graph.

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>

extern "C" int mv4i_g_cuda_err;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigm_f(float x) { return 1.0f / (1.0f + expf(-x)); }

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
    const int64_t base = (int64_t)(*tok) * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        x[i] = __half2float(__ushort_as_half(emb[base + i]));
}

// y = x * (1/sqrt(mean(x^2) + eps)) * w, ref/run9b.c:557-569, to fp16
__global__ void __launch_bounds__(1024) dec_rmsnorm_kernel(const float *x, const float *w, int n, float eps, uint16_t *y)
{
    __shared__ float red[32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
    s = block_sum(s, red);
    const float inv = rsqrtf(s / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        y[i] = __half_as_ushort(__float2half_rn(x[i] * inv * w[i]));
}

// DeltaNet pre-step (ref/run9b.c:634-672): 4-tap causal depthwise conv over
// the [q | k | v] projection with the rolling state (taps 0..2 on the stored
// inputs, oldest first, tap 3 on the current one), SiLU, to fp16; per value
// head beta = sigmoid(b), eg = exp(ssm_a * softplus(a + dt_bias)) (softplus
// returns x above 20).
__global__ void dec_gdn_pre_kernel(const float *qkv, int conv_dim, const float *conv_w, float *conv_state,
                                   uint16_t *qkv16, const float *ab, int vh, const float *ssm_a,
                                   const float *dt_bias, float *eg, float *beta)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < conv_dim) {
        const float x = qkv[c];
        const float s0 = conv_state[c], s1 = conv_state[conv_dim + c], s2 = conv_state[2 * conv_dim + c];
        const float4 w = reinterpret_cast<const float4 *>(conv_w)[c];
        const float acc = s0 * w.x + s1 * w.y + s2 * w.z + x * w.w;
        conv_state[c] = s1;
        conv_state[conv_dim + c] = s2;
        conv_state[2 * conv_dim + c] = x;
        qkv16[c] = __half_as_ushort(__float2half_rn(silu_f(acc)));
    }
    if (c < vh) {
        const float av = ab[c] + dt_bias[c], bv = ab[vh + c];
        const float sp = av > 20.f ? av : log1pf(expf(av));
        eg[c] = expf(ssm_a[c] * sp);
        beta[c] = sigm_f(bv);
    }
}

// Output norm then gate (ref/run9b.c:708-728): per head rmsnorm(o) * silu(z).
__global__ void dec_gated_norm_kernel(const float *o, const float *z, const float *w, int hd, float eps,
                                      uint16_t *y)
{
    __shared__ float red[32];
    const int h = blockIdx.x;
    const float *oh = o + (size_t)h * hd;
    float s = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) s = fmaf(oh[i], oh[i], s);
    s = block_sum(s, red);
    const float inv = rsqrtf(s / (float)hd + eps);
    for (int i = threadIdx.x; i < hd; i += blockDim.x)
        y[(size_t)h * hd + i] = __half_as_ushort(__float2half_rn(oh[i] * inv * w[i] * silu_f(z[(size_t)h * hd + i])));
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

// SwiGLU (ref/run9b.c:744): h = silu(gate) * up, to fp16.
__global__ void dec_swiglu_kernel(const float *g, const float *u, int n, uint16_t *h)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        h[i] = __half_as_ushort(__float2half_rn(silu_f(g[i]) * u[i]));
}

__global__ void dec_add_kernel(float *x, const float *t, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] += t[i];
}

// Argmax key of this rank's logits: order-preserving value in the high
// word, the complemented GLOBAL index in the low word (first max wins).
__global__ void __launch_bounds__(512) dec_argmax_kernel(const float *v, int n, int idx0, unsigned long long *key)
{
    unsigned long long best = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t u = __float_as_uint(v[i]);
        const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        const unsigned long long kk = ((unsigned long long)k << 32) | (0xFFFFFFFFull - (uint32_t)(idx0 + i));
        best = kk > best ? kk : best;
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, best, o);
        best = w > best ? w : best;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(key, best);
}

// Pick the largest of `n` keys (one per rank), record it as the prediction
// at the current position, advance the position, clear `key`.  The next
// input token is the prompt's while the prompt lasts (prompt[0] holds its
// length, prompt[1 + i] its tokens), else the prediction.
__global__ void dec_advance_kernel(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok,
                                   int32_t *history, int32_t *pos, int max_ctx, const int32_t *prompt)
{
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
// matrix.  Same draws as mv4i_synth_g128 for the same key and global index.
__global__ void dec_synth_linear_kernel(uint64_t key, const int32_t *rows, int row0, int nrows, int k0, int kn,
                                        int Kg, uint8_t *wq, uint16_t *sc)
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
        sc[i] = __half_as_ushort(__float2half_rn((float)(0.002 + 0.018 * u)));
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

extern "C" {

static int dk(cudaError_t e) { if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; } return 0; }
#define ST(s) reinterpret_cast<cudaStream_t>(s)

int dec_k_embed(const uint16_t *emb, int hidden, const int32_t *tok, float *x, void *s)
{ dec_embed_kernel<<<(hidden + 255) / 256, 256, 0, ST(s)>>>(emb, hidden, tok, x); return dk(cudaGetLastError()); }

int dec_k_rmsnorm(const float *x, const float *w, int n, float eps, uint16_t *y, void *s)
{ dec_rmsnorm_kernel<<<1, 1024, 0, ST(s)>>>(x, w, n, eps, y); return dk(cudaGetLastError()); }

int dec_k_gdn_pre(const float *qkv, int conv_dim, const float *conv_w, float *conv_state, uint16_t *qkv16,
                  const float *ab, int vh, const float *ssm_a, const float *dt_bias, float *eg, float *beta, void *s)
{
    const int n = conv_dim > vh ? conv_dim : vh;
    dec_gdn_pre_kernel<<<(n + 255) / 256, 256, 0, ST(s)>>>(qkv, conv_dim, conv_w, conv_state, qkv16, ab, vh,
                                                           ssm_a, dt_bias, eg, beta);
    return dk(cudaGetLastError());
}

int dec_k_gated_norm(const float *o, const float *z, const float *w, int heads, int hd, float eps, uint16_t *y, void *s)
{ dec_gated_norm_kernel<<<heads, 128, 0, ST(s)>>>(o, z, w, hd, eps, y); return dk(cudaGetLastError()); }

int dec_k_attn_pre(const float *qg, const float *kv, int qh, int kvh, int hd, int n_rot, float theta, float eps,
                   const float *qn_w, const float *kn_w, const int32_t *d_pos, int max_ctx, float *q_out,
                   float *gate_out, uint16_t *kcache, uint16_t *vcache, void *s)
{
    dec_attn_pre_kernel<<<qh + kvh, ((hd + 31) / 32) * 32, 0, ST(s)>>>(qg, kv, qh, kvh, hd, n_rot, theta, eps, qn_w,
                                                                      kn_w, d_pos, max_ctx, q_out, gate_out, kcache,
                                                                      vcache);
    return dk(cudaGetLastError());
}

int dec_k_attention(const float *q, const uint16_t *kc, const uint16_t *vc, int qh, int kvh, int hd, int ch,
                    int max_ctx, const int32_t *d_pos, float *part, const float *gate, uint16_t *y, void *s)
{
    const int nchunks = (max_ctx + ch - 1) / ch;
    dec_attn_decode_kernel<<<dim3(nchunks, kvh), 32 * (qh / kvh), 0, ST(s)>>>(q, kc, vc, qh, kvh, hd, ch, d_pos,
                                                                              max_ctx, nchunks, part);
    dec_attn_combine_kernel<<<qh, 32, 0, ST(s)>>>(part, gate, hd, nchunks, d_pos, ch, y);
    return dk(cudaGetLastError());
}

int dec_k_swiglu(const float *g, const float *u, int n, uint16_t *h, void *s)
{ dec_swiglu_kernel<<<(n + 255) / 256, 256, 0, ST(s)>>>(g, u, n, h); return dk(cudaGetLastError()); }

int dec_k_add(float *x, const float *t, int n, void *s)
{ dec_add_kernel<<<(n + 255) / 256, 256, 0, ST(s)>>>(x, t, n); return dk(cudaGetLastError()); }

int dec_k_argmax(const float *v, int n, int idx0, unsigned long long *key, void *s)
{
    dec_argmax_kernel<<<min(296, (n + 511) / 512), 512, 0, ST(s)>>>(v, n, idx0, key);
    return dk(cudaGetLastError());
}

int dec_k_advance(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok, int32_t *hist,
                  int32_t *pos, int max_ctx, const int32_t *prompt, void *s)
{
    dec_advance_kernel<<<1, 1, 0, ST(s)>>>(keys, n, key, tok, hist, pos, max_ctx, prompt);
    return dk(cudaGetLastError());
}

int dec_k_synth_linear(uint64_t key, const int32_t *rows, int row0, int nrows, int k0, int kn, int Kg,
                       uint8_t *wq, uint16_t *sc, void *s)
{
    dec_synth_linear_kernel<<<148 * 8, 256, 0, ST(s)>>>(key, rows, row0, nrows, k0, kn, Kg, wq, sc);
    return dk(cudaGetLastError());
}

int dec_k_synth_vec(uint64_t key, const int32_t *idx, int64_t idx0, int64_t n, float mean, float std,
                    float *f32, uint16_t *f16, void *s)
{
    dec_synth_vec_kernel<<<148 * 4, 256, 0, ST(s)>>>(key, idx, idx0, n, mean, std, f32, f16);
    return dk(cudaGetLastError());
}

}  // extern "C"
