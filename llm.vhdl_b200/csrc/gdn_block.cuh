// llm.vhdl_b200/csrc/gdn_block.cuh -- the fixed-point Gated DeltaNet block
// (llm.vhdl subsystem B, one token end to end, bit-exact with the reference's
// gdn_block_token, ref/gdn_block_vec.c:208-423).  Included by gdn_kernels.cu,
// whose integer helpers (g_floor_shr, g_round_shift, g_msb, ...), scalar path
// (d_to_q_wide, ...) and LUT upload it shares.
//
// Two launches per token, each a programmatic dependent of the one before:
//
//   gdn_blk_head_kernel<D> one CTA per value head, D*D/16 threads: the three
//                          conv segments' requantiser maxima (every CTA reduces
//                          whole segments from L2), then one warp each for the
//                          head's q / k (silu, L2 norm with the Newton rsqrt on
//                          the Q30 seed table), v (silu) and scalar path (eg,
//                          beta); the recurrence (stages 1-5, state column j
//                          owned by D/16 lanes of 16 keys each; the state slice
//                          is loaded before the wait on the launch before); then
//                          warp 0 runs the head tail: site-12 head emit, the
//                          output rmsnorm_bf, the z gate.  Tables live in shared
//                          memory, copied before the wait.
//   gdn_blk_tail_kernel    one CTA: site 13, the gated product over all heads
//                          aligned to the minimum head exponent and renormalised
//                          to one token exponent; writes the status word.
//
// Scratch between the launches lives in the caller's workspace
// (deltanet_work_bytes); nothing is allocated here.  Roofline: HBM for the
// state (2*VH*D*D bytes read and written per token, 2 MiB at KH 16 / VH 32 /
// D 128); every other operand is under 200 KB and the launches are latency-
// bound at that size.

#define BLK_FULL 0xffffffffu
#define BLK_EPS_E 50                    /* e_eps = 30 - floor(log2(1e-6))   */
#define BLK_EPS_M 1125899907LL          /* llround(1e-6 * 2^50)             */
#define BLK_INV_SQRT2 759250125LL       /* round(2^30 / sqrt 2)             */

__device__ int64_t d_sig_tab[513];      // the Q30 sigmoid table, global copy for divergent reads
__device__ int64_t d_rsqrt_rom[64];     // round(2^30 / sqrt(1 + k/64))
// global copies of the scalar path's Q30 tables (the constant-bank ones serve
// uniform reads; these are copied into shared memory by every thread)
__device__ int64_t d_sp_tab[257], d_exp_tab[257], d_sg_tab[513];

static unsigned long long g_blk_tab_ready = 0;

static cudaError_t upload_blk_tables()
{
    int dev = 0;
    cudaError_t e = upload_luts();
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && (g_blk_tab_ready >> dev & 1ull)) return cudaSuccess;
    static int64_t ts[513], rom[64];
    for (int k = 0; k <= 512; k++) {
        const double z = -16.0 + (double)k * (32.0 / 512.0);
        ts[k] = llround((1.0 / (1.0 + exp(-z))) * 1073741824.0);
    }
    for (int k = 0; k < 64; k++) rom[k] = llround(1073741824.0 / sqrt(1.0 + (double)k / 64.0));
    e = cudaMemcpyToSymbol(d_sig_tab, ts, sizeof ts);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(d_rsqrt_rom, rom, sizeof rom);
    static int64_t sp[257], ex[257], sg[513];
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(sp, c_sp_lut, sizeof sp);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(ex, c_exp_lut, sizeof ex);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(sg, c_sig_lut, sizeof sg);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(d_sp_tab, sp, sizeof sp);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(d_exp_tab, ex, sizeof ex);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(d_sg_tab, sg, sizeof sg);
    if (e == cudaSuccess && dev < 64) g_blk_tab_ready |= 1ull << dev;
    return e;
}

// ------------------------------------------------------------ fixed-point units

// site-3 Q12 conversion of a mantissa on exponent e (ref/gdn_silu_vec.c:42-57)
__device__ __forceinline__ int32_t fx_to_q12(int64_t x, int e)
{
    const int sh = e - 12;
    if (sh >= 0) return sh > 62 ? 0 : (int32_t)g_round_shift(x, sh);
    const int k = -sh;
    if (k > 40) return x > 0 ? INT32_MAX : (x < 0 ? INT32_MIN : 0);
    const int64_t v = x * ((int64_t)1 << k);
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}

// sigma, Q12 in / Q15 out, interpolated on the Q30 table (ref/gdn_silu_vec.c:59-80)
__device__ __forceinline__ int32_t fx_sigma_q15(int32_t z, const int64_t *tab)
{
    const int64_t lim = (int64_t)16 << 12;
    if ((int64_t)z <= -lim) return 0;
    if ((int64_t)z >= lim) return 1 << 15;
    const int64_t pos = ((int64_t)z + lim) * 16;
    int64_t k = pos >> 12;
    if (k > 511) k = 511;
    const int64_t frac = pos - (k << 12);
    const int64_t lo = tab[k], hi = tab[k + 1];
    const int64_t r = g_round_shift(lo + (((hi - lo) * frac) >> 12), 15);
    return (int32_t)(r < 0 ? 0 : (r > 32768 ? 32768 : r));
}

// silu with the exponent preserved (ref/gdn_block_vec.c:250-253); tab is the
// Q30 sigmoid table (d_sig_tab or a shared-memory copy of it)
__device__ __forceinline__ int32_t fx_silu(int32_t sm, int e, const int64_t *tab)
{
    return (int32_t)g_round_shift((int64_t)sm * fx_sigma_q15(fx_to_q12(sm, e), tab), 15);
}

// numeric_std forms used by rmsnorm_bf (ref/rmsnorm_bf_vec.c:108-157)
__device__ __forceinline__ int64_t fx_sll(int64_t v, int sh)
{ return sh <= 0 ? v : (sh >= 64 ? 0 : (int64_t)((uint64_t)v << sh)); }
__device__ __forceinline__ int64_t fx_narrow(int64_t v, int w)
{
    const int64_t r = (int64_t)((uint64_t)v & (((uint64_t)1 << (w - 1)) - 1));
    return v < 0 ? r - ((int64_t)1 << (w - 1)) : r;
}
__device__ __forceinline__ int fx_msb63(int64_t v)
{
    const uint64_t u = (uint64_t)v & 0x7FFFFFFFFFFFFFFFull;
    return u ? 63 - __clzll((long long)u) : 0;
}

// one L2-norm rsqrt pass (ref/l2norm_rs_vec.c:93-115): Q30 mantissa, exponent he;
// rom is the seed table (d_rsqrt_rom or a shared-memory copy of it)
__device__ __forceinline__ int64_t fx_l2_rsqrt(int64_t arg, int &he, const int64_t *rom)
{
    const int m = fx_msb63(arg);
    const uint64_t mant = m <= 30 ? (uint64_t)arg << (30 - m) : (uint64_t)arg >> (m - 30);
    const int64_t sm = (int64_t)(uint32_t)mant;
    int64_t y = rom[(mant >> 24) & 63];
#pragma unroll
    for (int it = 0; it < 2; it++) {
        const int64_t y2 = (int64_t)(int32_t)((y * y) >> 30);
        const int64_t d = (3LL << 30) - ((sm * y2) >> 30);
        y = (int64_t)(int32_t)((d * y) >> 31);
    }
    if (m & 1) { he = (m - 1) / 2; y = (y * BLK_INV_SQRT2) >> 30; }
    else he = m / 2;
    return y;
}

// the rmsnorm_bf reciprocal (ref/rmsnorm_bf_vec.c:230-331) of a sum of squares
// S of N = 2^lg mantissas on exponent xe: the clamped u31 inv32, Q = 12
__device__ int64_t fx_rms_inv(int64_t S, int xe, int lg, const int64_t *rom)
{
    const int shs = 30 - fx_msb63(S);
    const int e_mean = lg + 2 * xe + shs;
    const int64_t m_mean = S == 0 ? 0 : (shs >= 0 ? fx_sll(S, shs) : g_floor_shr(S, -shs));
    int d, mean_smaller, e_out;
    if (S == 0) { d = 0; mean_smaller = 1; e_out = BLK_EPS_E; }
    else if (e_mean > BLK_EPS_E) { d = e_mean - BLK_EPS_E; mean_smaller = 1; e_out = BLK_EPS_E; }
    else { d = BLK_EPS_E - e_mean; mean_smaller = 0; e_out = e_mean; }
    if (d > 63) d = 63;
    const int64_t align = S == 0 ? 0 : (mean_smaller ? g_floor_shr(m_mean, d) : g_floor_shr(BLK_EPS_M, d));
    const int64_t msq = mean_smaller ? align + BLK_EPS_M : m_mean + align;
    const int p = fx_msb63(msq);
    const uint64_t mant = p <= 30 ? (uint64_t)msq << (30 - p) : (uint64_t)msq >> (p - 30);
    const int64_t sm = (int64_t)(uint32_t)mant;
    int64_t y = rom[(mant >> 24) & 63];
#pragma unroll
    for (int it = 0; it < 2; it++) {
        const int64_t y2 = fx_narrow(g_floor_shr(y * y, 30), 32);
        const int64_t df = fx_narrow((3LL << 30) - fx_narrow(g_floor_shr(sm * y2, 30), 34), 34);
        y = fx_narrow(g_floor_shr(df * y, 31), 32);
    }
    const int rq_d = p - e_out;
    int64_t yf;
    int he;
    if (rq_d % 2 != 0) { yf = fx_narrow(g_floor_shr(y * BLK_INV_SQRT2, 30), 32); he = (rq_d - 1) / 2; }
    else { yf = y; he = rq_d / 2; }
    const int E = 12 - 30 - he;
    int64_t inv;
    if (E > 32) inv = 2147483647LL;
    else if (E >= 0) inv = fx_sll(yf, E);
    else inv = g_floor_shr(yf + fx_sll(1, -E - 1), -E);
    return inv > 2147483647LL ? 2147483647LL : (inv < 0 ? 0 : inv);
}

// warp sum of non-negative 64-bit values (sums of squares) as three 21-bit
// slices, each summed exactly in 32 bits by one reduction; equal to the
// 64-bit sum modulo 2^64
__device__ __forceinline__ int64_t warp_sum_sq(int64_t v)
{
    const uint64_t u = (uint64_t)v;
    const uint64_t lo = __reduce_add_sync(BLK_FULL, (unsigned)(u & 0x1FFFFF));
    const uint64_t mi = __reduce_add_sync(BLK_FULL, (unsigned)((u >> 21) & 0x1FFFFF));
    const uint64_t hi = __reduce_add_sync(BLK_FULL, (unsigned)(u >> 42));
    return (int64_t)((hi << 42) + (mi << 21) + lo);
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) { const uint64_t w = __shfl_xor_sync(BLK_FULL, v, o); v = w > v ? w : v; }
    return v;
}
__device__ __forceinline__ int warp_min_i32(int v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(BLK_FULL, v, o));
    return v;
}
// CTA-wide maximum (every thread gets it); red holds one word per warp
__device__ uint64_t cta_max_u64(uint64_t v, uint64_t *red)
{
    v = warp_max_u64(v);
    const int w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    uint64_t m = 0;
    for (int i = 0; i < nw; i++) m = red[i] > m ? red[i] : m;
    return m;
}

// L2 norm of one head of R*32 silu mantissas held R per lane (element lane + 32 r):
// the k output (exponent 15) or the q output (exponent 18), zeros when the
// sum of squares is 0 (ref/l2norm_rs_vec.c:118-140)
template <int R>
__device__ void fx_l2norm_warp(const int32_t (&x)[R], int log2n, bool q_path, int16_t *out, const int64_t *rom)
{
    int64_t ssq = 0;
#pragma unroll
    for (int r = 0; r < R; r++) ssq += (int64_t)x[r] * x[r];
    ssq = warp_sum_sq(ssq);
    const int lane = threadIdx.x & 31;
    if (ssq == 0) {
#pragma unroll
        for (int r = 0; r < R; r++) out[lane + 32 * r] = 0;
        return;
    }
    int he;
    const int64_t y = fx_l2_rsqrt(q_path ? ssq << log2n : ssq, he, rom);
    const int sh = (q_path ? 12 : 15) + he;
#pragma unroll
    for (int r = 0; r < R; r++)
        out[lane + 32 * r] = g_sat16(((int64_t)x[r] * y + ((int64_t)1 << (sh - 1))) >> sh);
}

// rmsnorm_bf of one head of R*32 int16 mantissas on exponent xe, R per lane,
// weights wm on we (ref/rmsnorm_bf_vec.c:199-389); returns the output exponent
template <int R>
__device__ int fx_rmsnorm_warp(const int32_t (&xm)[R], int xe, const int16_t *wm, int we, int lg,
                               int32_t (&o)[R], int &nsat, const int64_t *rom)
{
    const int lane = threadIdx.x & 31;
    int64_t S = 0;
#pragma unroll
    for (int r = 0; r < R; r++) S += (int64_t)xm[r] * xm[r];
    S = warp_sum_sq(S);
    const int64_t inv = fx_rms_inv(S, xe, lg, rom);
    int64_t raw[R];
    int mb = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
        raw[r] = fx_narrow(xm[r] * inv, 48) * (int64_t)wm[lane + 32 * r];
        mb = max(mb, fx_msb63((int64_t)(uint64_t)(raw[r] < 0 ? -raw[r] : raw[r])));
    }
    mb = __reduce_max_sync(BLK_FULL, mb);            // |raw| < 2^62: the msb of the maximum
    int st = mb - 14;
    if (st < 0) st = 0;
    const int64_t bias = st == 0 ? 0 : fx_sll(1, st - 1);
    nsat = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int64_t v = g_floor_shr(raw[r] + bias, st);
        nsat += (v > 32767 || v < -32768);
        o[r] = g_sat16(v);
    }
    return xe + we + 12 - st;
}

// ------------------------------------------------------------- block kernels

struct BlkWork {                       // device scratch between the two launches of a token
    int16_t *po, *pz;                  // [VH][D] normed output / gated z
    int32_t *ep;                       // [VH] product exponents
    int32_t *err;                      // [VH] bit 0 conv segment exponent, bit 1 g, bit 2 state exponent
    int32_t *pmax, *pmin;              // [VH] largest / smallest product po * pz of each head
};

static size_t blk_al(size_t n) { return (n + 255) & ~(size_t)255; }

static BlkWork blk_work_layout(void *base, int VH, int D, size_t *bytes)
{
    BlkWork w;
    char *p = (char *)base;
    size_t off = 0;
#define BLK_TAKE(field, T, n) w.field = (T *)(p + off); off += blk_al((size_t)(n) * sizeof(T));
    BLK_TAKE(po, int16_t, VH * D)
    BLK_TAKE(pz, int16_t, VH * D)
    BLK_TAKE(ep, int32_t, VH)
    BLK_TAKE(err, int32_t, VH)
    BLK_TAKE(pmax, int32_t, VH)
    BLK_TAKE(pmin, int32_t, VH)
#undef BLK_TAKE
    if (bytes) *bytes = off;
    return w;
}

// floor(v / 2^sh) for a 32-bit v, sh <= 63 (g_floor_shr on int32 values)
__device__ __forceinline__ int32_t blk_floor_shr32(int32_t v, int sh)
{ return sh <= 0 ? v : (sh >= 31 ? (v < 0 ? -1 : 0) : (v >> sh)); }

// conv of one channel over its valid taps, aligned to the smallest valid tap
// exponent by floor (ref/gdn_block_vec.c:231-239)
__device__ __forceinline__ int64_t blk_conv_ch(const int16_t *x, const int16_t *w, int vmask, const int (&tsh)[4])
{
    const uint2 xv = *reinterpret_cast<const uint2 *>(x), wv = *reinterpret_cast<const uint2 *>(w);
    const int32_t xs[4] = {lo16(xv.x), hi16(xv.x), lo16(xv.y), hi16(xv.y)};
    const int32_t ws[4] = {lo16(wv.x), hi16(wv.x), lo16(wv.y), hi16(wv.y)};
    int64_t a = 0;
#pragma unroll
    for (int t = 0; t < 4; t++)
        if (vmask >> t & 1) a += blk_floor_shr32(xs[t] * ws[t], tsh[t]);
    return a;
}

// e_ref = smallest exponent among the valid taps; per-tap alignment shifts
__device__ __forceinline__ int blk_taps(const int32_t (&e_t)[4], const int32_t (&tv)[4], int (&tsh)[4], int &vmask)
{
    int e_ref = 0, have = 0;
    vmask = 0;
#pragma unroll
    for (int t = 0; t < 4; t++)
        if (tv[t]) { vmask |= 1 << t; if (!have || e_t[t] < e_ref) { e_ref = e_t[t]; have = 1; } }
#pragma unroll
    for (int t = 0; t < 4; t++) { const int s = e_t[t] - e_ref; tsh[t] = s > 63 ? 63 : s; }
    return e_ref;
}

// the scalar path of one value head (ref/gdn_block_vec.c:282-290 calling
// gdn_scalar_int, ref/gdn_scalar_vec.c:100-156; the same arithmetic as
// gdn_scalar_kernel): eg (Q15 decay) and beta (Q16) from the head's eight
// inputs; returns 1 when g was clamped at -16
__device__ int blk_scalar(const int32_t *p, int32_t &eg, int32_t &beta, const int64_t *tsp, const int64_t *tex,
                           const int64_t *tsg)
{
    const int64_t arg = d_to_q_wide(p[0], p[1]) + d_to_q_wide(p[2], p[3]);
    const int64_t one = (int64_t)1 << SPQ, lim = 16 * one;
    int64_t sp;
    if (arg <= -lim) sp = 0;
    else if (arg >= lim) sp = arg;
    else {
        const int64_t ax = arg < 0 ? -arg : arg, pos = arg > 0 ? arg : 0;
        sp = pos + (ax >= lim ? 0 : d_lut_interp(tsp, 256, lim - ax, SPQ));
        if (sp < 0) sp = 0;
        if (sp > 0x7FFFFFFF) sp = 0x7FFFFFFF;
    }
    int64_t g = d_rshift_r(sp * (int64_t)p[4], p[5]);
    if (g > 0) g = 0;
    const int err = g < -lim;
    if (g < -lim) g = -lim;
    int64_t ex = d_lut_interp(tex, 256, g + lim, SPQ);
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
        sg = d_lut_interp(tsg, 512, bq + lim, SPQ);
        sg = sg < 0 ? 0 : (sg > one ? one : sg);
    }
    int64_t bv = d_rshift_r(sg, SPQ - 16);
    bv = bv > 65535 ? 65535 : (bv < 0 ? 0 : bv);
    eg = (int32_t)egv;
    beta = (int32_t)bv;
    return err;
}

// one warp: site-12 head emit of a value head's D column outputs (o_acc on
// per-column exponents e_o), the output rmsnorm, the z gate; writes the head's
// po / pz / ep for site 13 (ref/gdn_emit_chain_vec.c).  pz_in, when given,
// holds the head's gated z already (silu(zm) does not depend on the rest);
// w.pmax / w.pmin, when set, receive the head's extreme products po * pz.
// Only the msb of a maximum feeds a shift, so maxima are reduced as msb
// positions (the msb of the largest value is the largest msb).
template <int D>
__device__ void blk_head_tail(int h, const int64_t *s_oacc, const int32_t *s_eo, const int16_t *zm, int z_e,
                              const int16_t *pz_in, const int16_t *wm, int w_e, const BlkWork &w,
                              const int64_t *sig, const int64_t *rom)
{
    constexpr int R = D / 32, LG = D == 32 ? 5 : (D == 64 ? 6 : 7);
    const int lane = threadIdx.x & 31;
    int emin = 1 << 30;
#pragma unroll
    for (int r = 0; r < R; r++) emin = min(emin, s_eo[lane + 32 * r]);
    emin = __reduce_min_sync(BLK_FULL, emin);
    int64_t al[R];
    int mb = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
        int shj = s_eo[lane + 32 * r] - emin;
        if (shj > 63) shj = 63;
        al[r] = g_floor_shr(s_oacc[lane + 32 * r], shj);
        mb = max(mb, g_msb(g_abs64(al[r])));
    }
    mb = __reduce_max_sync(BLK_FULL, mb);
    int shh = mb - 14;
    if (shh < 0) shh = 0;
    int32_t oh[R], po[R];
#pragma unroll
    for (int r = 0; r < R; r++) oh[r] = g_sat16(g_round_shift(al[r], shh));
    int nsat;
    const int o_exp = fx_rmsnorm_warp<R>(oh, emin - shh, wm, w_e, LG, po, nsat, rom);
    int pmx = INT32_MIN, pmn = INT32_MAX;
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int j = lane + 32 * r;
        const int16_t pz = pz_in ? pz_in[j] : g_sat16(fx_silu(zm[h * D + j], z_e, sig));
        w.po[h * D + j] = (int16_t)po[r];
        w.pz[h * D + j] = pz;
        const int32_t pr = po[r] * (int32_t)pz;
        pmx = max(pmx, pr);
        pmn = min(pmn, pr);
    }
    if (w.pmax) {
        pmx = __reduce_max_sync(BLK_FULL, pmx);
        pmn = __reduce_min_sync(BLK_FULL, pmn);
        if (lane == 0) { w.pmax[h] = pmx; w.pmin[h] = pmn; }
    }
    if (lane == 0) w.ep[h] = o_exp + z_e;
}

struct BlkHeadArgs {
    const int16_t *xtap, *wtap;        // [2*KH*D + VH*D][4]
    const int32_t *sc;                 // [VH][8]
    int32_t KH, VH, tk0, w_e, z_e;
    int32_t e_t[3][4], tvalid[3][4], cw_exp[3];
    int16_t *smem;                     // [VH][D][D]
    int32_t *semem;                    // [VH][D]
    const int16_t *zm, *wm;            // [VH][D], [D]
    BlkWork w;
};

// thread-block cluster helpers: the CTA's rank, the cluster's size, loads from
// the same shared-memory variable of CTA `rank`, and the split cluster
// barrier.  A launch without a cluster attribute is a cluster of one.
__device__ __forceinline__ unsigned blk_cl_rank()
{ unsigned r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ unsigned blk_cl_size()
{ unsigned r; asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ unsigned blk_cl_addr(const void *p, unsigned rank)
{
    const unsigned a = (unsigned)__cvta_generic_to_shared(p);
    unsigned ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    return ra;
}
__device__ __forceinline__ int64_t blk_ld_cl_i64(const void *p, unsigned rank)
{
    int64_t v;
    asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(blk_cl_addr(p, rank)) : "memory");
    return v;
}
__device__ __forceinline__ int blk_ld_cl_i32(const void *p, unsigned rank)
{
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(blk_cl_addr(p, rank)) : "memory");
    return v;
}
__device__ __forceinline__ void blk_cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void blk_cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// msb position of |x|, 0 for 0 and 1 (g_msb(g_abs64(x)) for 64-bit values)
__device__ __forceinline__ int blk_msb_abs(int64_t x) { return g_msb(g_abs64(x)); }

// the head kernel's shape for head dimension D: 32 value columns per CTA,
// D/16 lanes per column (16 keys each), D/32 CTAs per value head
template <int D>
struct BlkShape {
    static constexpr int LPC = D / 16, COLS = 32, SPH = D / COLS, NT = COLS * LPC, NW = NT / 32;
    static constexpr int CPW = 32 / LPC, R = D / 32, LG = D == 32 ? 5 : (D == 64 ? 6 : 7);
};

// conv of channel c of the flattened [q | k | v] taps with segment s's tap
// shifts (s selects among the three sets held in registers)
__device__ __forceinline__ int64_t blk_conv_sel(const BlkHeadArgs &A, size_t c, int s, const int (&t0)[4],
                                                const int (&t1)[4], const int (&t2)[4], int v0, int v1, int v2)
{
    int ts[4];
#pragma unroll
    for (int k = 0; k < 4; k++) ts[k] = s == 0 ? t0[k] : (s == 1 ? t1[k] : t2[k]);
    return blk_conv_ch(A.xtap + 4 * c, A.wtap + 4 * c, s == 0 ? v0 : (s == 1 ? v1 : v2), ts);
}

// D/32 CTAs per value head h (CTA part p holds columns 32p .. 32p+31), in
// thread-block clusters of 2-8 CTAs that hold whole heads:
//  1. The three conv segments' requantiser shifts (q, k, v; spec B 2.1.3).
//     One segment shares one shift, so each cluster reduces whole segments
//     (at KH 16 / VH 32 / D 128, 8192 channels, 128 KB of taps from L2), every
//     CTA a slice; only the msb position of the largest |conv| matters, so
//     that is what the CTAs reduce and exchange through distributed shared
//     memory.  The raw conv of the channels this CTA needs itself (q and k of
//     key head h % KH, v of its 32 columns) is kept in shared memory.
//  2. One warp per task: q and k (silu, L2 norm), v (silu), the scalar path.
//  3. The recurrence, stages 1-5, for the CTA's 32 columns (column j owned by
//     D/16 lanes of 16 keys each, ref/gdn_block_vec.c:304-380).
//  4. The head's first CTA gathers the D column results from the others and
//     its warp 0 runs the head tail (site-12 emit, rmsnorm_bf, z gate).
template <int D>
__global__ void __launch_bounds__(2 * D)
gdn_blk_head_kernel(const BlkHeadArgs A)
{
    using S = BlkShape<D>;
    constexpr int NT = S::NT, NW = S::NW, LPC = S::LPC, SPH = S::SPH, CPW = S::CPW, R = S::R, LG = S::LG;
    __shared__ int64_t s_sig[513], s_rom[64], s_raw[2 * D + 32], s_oacc[D], s_loacc[32];
    __shared__ __align__(16) uint4 s_st[2 * NT];        // the state slices, [half][thread]
    __shared__ __align__(16) int16_t s_kn[D], s_qs[D];
    __shared__ int32_t s_eo[D], s_leo[32], s_v[32], s_red[3][NW], s_part[3];
    __shared__ int32_t s_sc[3], s_sh[3], s_es[3], s_errc, s_lerr, s_gerr;
    __shared__ int64_t s_lsp[257], s_lex[257], s_lsg[513];   // the scalar path's Q30 tables
    __shared__ int16_t s_pz[D], s_zmv[D], s_wm[D];
    __shared__ int32_t s_scv[8];
    const int h = blockIdx.x / SPH, part = blockIdx.x % SPH, hk = h % A.KH;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int jl = warp * CPW + lane / LPC;             // local value column
    const int j = 32 * part + jl;                       // value column of the head
    const int i0 = 16 * (lane % LPC);                   // key slice

    // Before the wait: the constant tables and this CTA's state slice (an
    // asynchronous copy into shared memory).  A grid of this kernel starts only
    // once the launch before it has passed its own wait (the site-13 launch of
    // the previous token, or a later kernel), so the previous token's state
    // write-back has completed by then.
    int16_t *scol = A.smem + ((size_t)h * D + j) * D + i0;
    {
        const unsigned d0 = (unsigned)__cvta_generic_to_shared(s_st + threadIdx.x);
        const unsigned d1 = (unsigned)__cvta_generic_to_shared(s_st + NT + threadIdx.x);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(d0), "l"(scol) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(d1), "l"(scol + 8) : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int i = threadIdx.x; i < 513; i += NT) s_sig[i] = d_sig_tab[i];
    for (int i = threadIdx.x; i < 64; i += NT) s_rom[i] = d_rsqrt_rom[i];
    for (int i = threadIdx.x; i < 257; i += NT) { s_lsp[i] = d_sp_tab[i]; s_lex[i] = d_exp_tab[i]; }
    for (int i = threadIdx.x; i < 513; i += NT) s_lsg[i] = d_sg_tab[i];
    const int se_j = A.semem[h * D + j];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // 1. segment shifts
    const int QCH = A.KH * D, NCH = 2 * QCH + A.VH * D;
    const int crank = (int)blk_cl_rank(), csize = (int)blk_cl_size();
    int t0[4], t1[4], t2[4], v0, v1, v2;
    const int er0 = blk_taps(A.e_t[0], A.tvalid[0], t0, v0);
    const int er1 = blk_taps(A.e_t[1], A.tvalid[1], t1, v1);
    const int er2 = blk_taps(A.e_t[2], A.tvalid[2], t2, v2);
    // the taps of this CTA's own channels (q / k of key head hk, v of its 32
    // columns: 2D + 32 <= 2 NT of them) are loaded first, so their latency
    // overlaps the segment loop's
    auto own_ch = [&](int t, int &s) -> size_t {
        s = t < D ? 0 : (t < 2 * D ? 1 : 2);
        return s == 0 ? (size_t)hk * D + t
             : (s == 1 ? (size_t)QCH + (size_t)hk * D + (t - D)
                       : 2 * (size_t)QCH + (size_t)h * D + 32 * part + (t - 2 * D));
    };
    uint2 ox[2], ow[2];
#pragma unroll
    for (int q = 0; q < 2; q++) {
        const int t = threadIdx.x + q * NT;
        int s;
        if (t < 2 * D + 32) {
            const size_t c = own_ch(t, s);
            ox[q] = *reinterpret_cast<const uint2 *>(A.xtap + 4 * c);
            ow[q] = *reinterpret_cast<const uint2 *>(A.wtap + 4 * c);
        }
    }
    // this head's scalar inputs, z row and norm weights: loaded now, kept in
    // shared memory by the end of the phase
    int32_t pre = 0;
    if (part == 0) pre = threadIdx.x < D ? A.zm[(size_t)h * D + threadIdx.x] : A.wm[threadIdx.x - D];
    int32_t scp = threadIdx.x < 8 ? A.sc[(size_t)h * 8 + threadIdx.x] : 0;
    int mb0 = 0, mb1 = 0, mb2 = 0;
#pragma unroll 4
    for (int c = crank * NT + threadIdx.x; c < NCH; c += csize * NT) {
        const int s = c < QCH ? 0 : (c < 2 * QCH ? 1 : 2);
        const int m = blk_msb_abs(blk_conv_sel(A, (size_t)c, s, t0, t1, t2, v0, v1, v2));
        if (s == 0) mb0 = max(mb0, m);
        else if (s == 1) mb1 = max(mb1, m);
        else mb2 = max(mb2, m);
    }
#pragma unroll
    for (int q = 0; q < 2; q++) {
        const int t = threadIdx.x + q * NT;
        if (t < 2 * D + 32) {
            int s;
            own_ch(t, s);
            int ts[4];
#pragma unroll
            for (int k = 0; k < 4; k++) ts[k] = s == 0 ? t0[k] : (s == 1 ? t1[k] : t2[k]);
            s_raw[t] = blk_conv_ch(reinterpret_cast<const int16_t *>(&ox[q]), reinterpret_cast<const int16_t *>(&ow[q]),
                                   s == 0 ? v0 : (s == 1 ? v1 : v2), ts);
        }
    }
    mb0 = __reduce_max_sync(BLK_FULL, mb0);
    mb1 = __reduce_max_sync(BLK_FULL, mb1);
    mb2 = __reduce_max_sync(BLK_FULL, mb2);
    if (lane == 0) { s_red[0][warp] = mb0; s_red[1][warp] = mb1; s_red[2][warp] = mb2; }
    if (part == 0) {
        if (threadIdx.x < D) s_zmv[threadIdx.x] = (int16_t)pre;
        else s_wm[threadIdx.x - D] = (int16_t)pre;
    }
    if (threadIdx.x < 8) s_scv[threadIdx.x] = scp;
    __syncthreads();
    if (threadIdx.x < 3) {
        int m = 0;
#pragma unroll
        for (int w = 0; w < NW; w++) m = max(m, s_red[threadIdx.x][w]);
        s_part[threadIdx.x] = m;
    }
    blk_cl_arrive();
    blk_cl_wait();
    if (warp == 0) {
        int m0 = 0, m1 = 0, m2 = 0;
        if (lane < csize) {
            m0 = blk_ld_cl_i32(&s_part[0], (unsigned)lane);
            m1 = blk_ld_cl_i32(&s_part[1], (unsigned)lane);
            m2 = blk_ld_cl_i32(&s_part[2], (unsigned)lane);
        }
        m0 = __reduce_max_sync(BLK_FULL, m0);
        m1 = __reduce_max_sync(BLK_FULL, m1);
        m2 = __reduce_max_sync(BLK_FULL, m2);
        if (lane == 0) {
            const int ms[3] = {m0, m1, m2}, er[3] = {er0, er1, er2};
            int errc = 0;
#pragma unroll
            for (int s = 0; s < 3; s++) {
                const int x = ms[s] - 14 < 0 ? 0 : ms[s] - 14;
                const int e = er[s] + A.cw_exp[s] - x;
                errc |= e > 127 || e < -128;
                s_sh[s] = x;
                s_es[s] = e;
            }
            s_errc = errc;
        }
    }
    __syncthreads();

    // 2. this CTA's inputs, one warp per task: q, k, v, the scalar path, and
    //    in the head's first CTA the z gate for the head tail
    for (int t = warp; t < 5; t += NW) {
        if (t < 2) {
            int32_t x[R];
#pragma unroll
            for (int r = 0; r < R; r++)
                x[r] = fx_silu(g_sat16(g_round_shift(s_raw[t * D + lane + 32 * r], s_sh[t])), s_es[t], s_sig);
            fx_l2norm_warp<R>(x, LG, t == 0, t == 0 ? s_qs : s_kn, s_rom);
        } else if (t == 2) {
            s_v[lane] = fx_silu(g_sat16(g_round_shift(s_raw[2 * D + lane], s_sh[2])), s_es[2], s_sig);
        } else if (t == 3) {
            if (lane == 0) {
                int32_t eg, bt;
                s_sc[2] = blk_scalar(s_scv, eg, bt, s_lsp, s_lex, s_lsg);
                s_sc[0] = eg;
                s_sc[1] = bt;
            }
        } else if (part == 0) {
            for (int i = lane; i < D; i += 32) s_pz[i] = g_sat16(fx_silu(s_zmv[i], A.z_e, s_sig));
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    // 3. the recurrence; stages 1-2: decay, sk dot
    uint32_t sm[8], kn[8], qs[8];
    {
        const uint4 a0 = s_st[threadIdx.x], a1 = s_st[NT + threadIdx.x];
        sm[0] = a0.x; sm[1] = a0.y; sm[2] = a0.z; sm[3] = a0.w; sm[4] = a1.x; sm[5] = a1.y; sm[6] = a1.z; sm[7] = a1.w;
    }
    ld16_i16(s_kn + i0, kn);
    ld16_i16(s_qs + i0, qs);
    const int32_t v_j = s_v[jl];
    const int egh = s_sc[0], bth = s_sc[1], tk0 = A.tk0, e_v = s_es[2];
    int32_t w18[16];
    int64_t sk = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const int32_t a = tk0 ? 0 : lo16(sm[p]) * egh, b = tk0 ? 0 : hi16(sm[p]) * egh;
        w18[2 * p] = (a + 4096) >> 13;
        w18[2 * p + 1] = (b + 4096) >> 13;
        sk += (int64_t)w18[2 * p] * lo16(kn[p]) + (int64_t)w18[2 * p + 1] * hi16(kn[p]);
    }
#pragma unroll
    for (int o = 1; o < LPC; o <<= 1) sk += __shfl_xor_sync(BLK_FULL, sk, o);
    int sh_sk = g_msb(g_abs64(sk)) - 14;
    if (sh_sk < 0) sh_sk = 0;
    const int64_t skm = g_round_shift(sk, sh_sk);
    const int ske = se_j + 17 - sh_sk;

    // stage 3: delta
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

    // stage 4: update, write-back quantiser.  In 32 bits: |w18| <= 2^17 + 1,
    // |d_m| <= 2^15 and |k| <= 2^15, so |u| < 2^30 + 2^18 and shq <= 16.
    const int e_kd = 15 + e_dm;
    const int e_u = masked ? e_kd : (se_j + 2 < e_kd ? se_j + 2 : e_kd);
    int su = se_j + 2 - e_u, sk2 = e_kd - e_u;
    if (su > 63) su = 63;
    if (sk2 > 63) sk2 = 63;
    const int32_t d32 = (int32_t)d_m;
    uint32_t amax = 0;
#pragma unroll
    for (int p = 0; p < 16; p++) {
        const int32_t k = (p & 1) ? hi16(kn[p >> 1]) : lo16(kn[p >> 1]);
        const int32_t u = (tk0 ? 0 : blk_floor_shr32(w18[p], su)) + blk_floor_shr32(k * d32, sk2);
        const uint32_t a = u < 0 ? 0u - (uint32_t)u : (uint32_t)u;
        amax = a > amax ? a : amax;
    }
#pragma unroll
    for (int o = 1; o < LPC; o <<= 1) amax = max(amax, __shfl_xor_sync(BLK_FULL, amax, o));
    int shq = (amax ? 31 - __clz((int)amax) : 0) - 14;
    if (shq < 0) shq = 0;
    const int32_t rq = shq ? 1 << (shq - 1) : 0;
    uint32_t sn[8];
    int64_t od = 0;
#pragma unroll
    for (int p = 0; p < 8; p++) {
        int32_t r2[2];
#pragma unroll
        for (int hlf = 0; hlf < 2; hlf++) {
            const int32_t k = hlf ? hi16(kn[p]) : lo16(kn[p]);
            const int32_t u = (tk0 ? 0 : blk_floor_shr32(w18[2 * p + hlf], su)) + blk_floor_shr32(k * d32, sk2);
            const int32_t v = (u + rq) >> shq;
            r2[hlf] = v > 32767 ? 32767 : (v < -32768 ? -32768 : v);
        }
        sn[p] = ((uint32_t)(uint16_t)r2[0]) | ((uint32_t)(uint16_t)r2[1] << 16);
        od += (int64_t)r2[0] * lo16(qs[p]) + (int64_t)r2[1] * hi16(qs[p]);     // stage 5
    }
    reinterpret_cast<uint4 *>(scol)[0] = make_uint4(sn[0], sn[1], sn[2], sn[3]);
    reinterpret_cast<uint4 *>(scol)[1] = make_uint4(sn[4], sn[5], sn[6], sn[7]);
#pragma unroll
    for (int o = 1; o < LPC; o <<= 1) od += __shfl_xor_sync(BLK_FULL, od, o);
    const int se_new = e_u - shq, e_o = se_new + 18;
    int err = 0;
    if (lane % LPC == 0) {
        A.semem[h * D + j] = se_new;
        s_loacc[jl] = od;
        s_leo[jl] = e_o;
        err = se_new > 127 || se_new < -128 || e_o > 127 || e_o < -128;
    }
    err = __syncthreads_or(err);
    if (threadIdx.x == 0) s_lerr = err;

    // 4. the head's first CTA gathers its D columns (CTA part p of the head is
    //    cluster rank crank + p), then runs the head tail; the others wait at
    //    the end until it has read their shared memory
    blk_cl_arrive();
    blk_cl_wait();
    if (part == 0) {
        for (int t = threadIdx.x; t < D; t += NT) {
            s_oacc[t] = blk_ld_cl_i64(&s_loacc[t & 31], (unsigned)(crank + (t >> 5)));
            s_eo[t] = blk_ld_cl_i32(&s_leo[t & 31], (unsigned)(crank + (t >> 5)));
        }
        if (threadIdx.x == 0) {
            int e = 0;
#pragma unroll
            for (int p = 0; p < SPH; p++) e |= blk_ld_cl_i32(&s_lerr, (unsigned)(crank + p));
            s_gerr = e;
        }
    }
    blk_cl_arrive();
    if (part == 0) {
        __syncthreads();
        if (warp == 0) {
            blk_head_tail<D>(h, s_oacc, s_eo, A.zm, A.z_e, s_pz, s_wm, A.w_e, A.w, s_sig, s_rom);
            if (lane == 0) A.w.err[h] = (s_errc ? 1 : 0) | (s_sc[2] ? 2 : 0) | (s_gerr ? 4 : 0);
        }
    }
    blk_cl_wait();
}

// the emit chain alone (site 12 -> rmsnorm -> z gate) on o_acc / e_o from
// memory, one warp per head: the unit entry point of the block's tail
struct BlkChainArgs {
    const int64_t *o_acc;              // [H][D]
    const int32_t *e_o;                // [H][D]
    const int16_t *zm, *wm;
    int32_t w_e, z_e;
    BlkWork w;
};

template <int D>
__global__ void __launch_bounds__(32)
gdn_blk_chain_kernel(const BlkChainArgs A)
{
    __shared__ int64_t s_oacc[D];
    __shared__ int32_t s_eo[D];
    const int h = blockIdx.x, lane = threadIdx.x;
    for (int j = lane; j < D; j += 32) { s_oacc[j] = A.o_acc[h * D + j]; s_eo[j] = A.e_o[h * D + j]; }
    __syncwarp();
    blk_head_tail<D>(h, s_oacc, s_eo, A.zm, A.z_e, nullptr, A.wm, A.w_e, A.w, d_sig_tab, d_rsqrt_rom);
}

struct BlkTailArgs {
    int32_t VH, D;
    const int16_t *po, *pz;
    const int32_t *ep;
    int16_t *y;
    int32_t *status;                   // [5] y_exp, err_conv, err_g, err_se, y_sat
    const int32_t *err;                // [VH] the heads' flag words; NULL for the site-13 unit entry
};

// one site-13 product aligned to the token's minimum head exponent e_y:
// |po * pz| <= 2^30, so 32 bits hold it
__device__ __forceinline__ int32_t blk_site13_term(const BlkTailArgs &A, int i, int e_y)
{
    const int s = A.ep[i / A.D] - e_y;
    return blk_floor_shr32((int32_t)A.po[i] * A.pz[i], s > 63 ? 63 : s);
}

__device__ __forceinline__ int blk_msb_abs32(int32_t v)
{
    const uint32_t a = v < 0 ? 0u - (uint32_t)v : (uint32_t)v;
    return a ? 31 - __clz((int)a) : 0;
}

// site 13 (ref/gdn_block_vec.c:396-418) over all VH*D products on their own
// (the unit entry gdn_y_emit_dev, no head records), split over the CTAs of
// one cluster (BLK_TAIL_NT threads each; a launch without a
// cluster is one CTA): each CTA takes a contiguous slice, the msb of the
// largest aligned product is exchanged through distributed shared memory,
// and cluster rank 0 writes the status word.
#define BLK_TAIL_NT 256
__global__ void __launch_bounds__(BLK_TAIL_NT)
gdn_blk_tail_kernel(const BlkTailArgs A)
{
    constexpr int KR = 8, NW = BLK_TAIL_NT / 32;
    __shared__ int32_t s_red[NW], s_ey, s_err, s_part, s_sat;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int crank = (int)blk_cl_rank(), csize = (int)blk_cl_size();
    if (warp == 0) {
        int m = 0x7FFFFFFF, er = 0;
        for (int h = lane; h < A.VH; h += 32) {
            m = min(m, A.ep[h]);
            if (A.err) er |= A.err[h];
        }
        m = __reduce_min_sync(BLK_FULL, m);
        er = (int)__reduce_or_sync(BLK_FULL, (unsigned)er);
        if (lane == 0) { s_ey = m; s_err = er; }
    }
    __syncthreads();
    const int e_y = s_ey, n = A.VH * A.D;
    const int chunk = (n + csize - 1) / csize, lo = crank * chunk, hi = min(n, lo + chunk);
    int32_t pv[KR];
    int mb = 0;
#pragma unroll
    for (int k = 0; k < KR; k++) {
        const int i = lo + threadIdx.x + BLK_TAIL_NT * k;
        pv[k] = i < hi ? blk_site13_term(A, i, e_y) : 0;
        mb = max(mb, blk_msb_abs32(pv[k]));
    }
    for (int i = lo + threadIdx.x + BLK_TAIL_NT * KR; i < hi; i += BLK_TAIL_NT)
        mb = max(mb, blk_msb_abs32(blk_site13_term(A, i, e_y)));
    mb = __reduce_max_sync(BLK_FULL, mb);
    if (lane == 0) s_red[warp] = mb;
    __syncthreads();
    if (threadIdx.x == 0) {
        int m = 0;
#pragma unroll
        for (int w = 0; w < NW; w++) m = max(m, s_red[w]);
        s_part = m;
    }
    blk_cl_arrive();
    blk_cl_wait();
    if (warp == 0) {
        int m = lane < csize ? blk_ld_cl_i32(&s_part, (unsigned)lane) : 0;
        m = __reduce_max_sync(BLK_FULL, m);
        if (lane == 0) s_red[0] = m;                  // the cluster-wide msb, for this CTA's threads
    }
    __syncthreads();
    int sh = s_red[0] - 14;
    if (sh < 0) sh = 0;
    const int32_t rq = sh ? 1 << (sh - 1) : 0;
    int sat = 0;
#pragma unroll
    for (int k = 0; k < KR; k++) {
        const int i = lo + threadIdx.x + BLK_TAIL_NT * k;
        if (i < hi) {
            const int32_t v = (pv[k] + rq) >> sh;
            sat |= v > 32767 || v < -32768;
            A.y[i] = g_sat16(v);
        }
    }
    for (int i = lo + threadIdx.x + BLK_TAIL_NT * KR; i < hi; i += BLK_TAIL_NT) {
        const int32_t v = (blk_site13_term(A, i, e_y) + rq) >> sh;
        sat |= v > 32767 || v < -32768;
        A.y[i] = g_sat16(v);
    }
    sat = __syncthreads_or(sat);
    if (threadIdx.x == 0) s_sat = sat != 0;
    blk_cl_arrive();
    blk_cl_wait();
    if (crank == 0 && threadIdx.x == 0) {
        int st = 0;
        for (int r = 0; r < csize; r++) st |= blk_ld_cl_i32(&s_sat, (unsigned)r);
        A.status[0] = e_y - sh;
        A.status[4] = st;
        if (A.err) {
            A.status[1] = s_err & 1;
            A.status[2] = s_err >> 1 & 1;
            A.status[3] = s_err >> 2 & 1;
        }
    }
    blk_cl_arrive();
    blk_cl_wait();
}

// site 13 of deltanet_step (ref/gdn_block_vec.c:396-418) from the heads'
// records: the token exponent e_y (the smallest head exponent), the shift
// (the msb of the largest aligned product) and the saturation flag all follow
// from each head's exponent and extreme products, because the floor shift and
// the rounding shift are monotone: the extremes of the aligned products are
// the aligned extremes.  So no CTA waits for another: each of the
// ceil(VH*D / 1024) CTAs reduces the VH records itself (one warp) while its
// threads load their four products.
#define BLK_S13_NT 256
#define BLK_S13_PER 4
struct BlkSite13Args {
    int32_t VH, D;
    const int16_t *po, *pz;
    const int32_t *ep, *pmax, *pmin, *err;
    int16_t *y;
    int32_t *status;                   // [5] y_exp, err_conv, err_g, err_se, y_sat
};

__global__ void __launch_bounds__(BLK_S13_NT)
gdn_blk_site13_kernel(const BlkSite13Args A)
{
    __shared__ int32_t s_ey, s_sh, s_sat, s_err;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n = A.VH * A.D;
    const int base = blockIdx.x * BLK_S13_NT * BLK_S13_PER + threadIdx.x;
    int32_t p[BLK_S13_PER], eh[BLK_S13_PER];
#pragma unroll
    for (int k = 0; k < BLK_S13_PER; k++) {
        const int i = base + BLK_S13_NT * k;
        p[k] = i < n ? (int32_t)A.po[i] * A.pz[i] : 0;
        eh[k] = i < n ? A.ep[i / A.D] : 0;
    }
    if (warp == 0) {
        // the first 128 head records in one round of loads, the rest (if any)
        // read again after the minimum
        constexpr int HP = 4;
        int eh_[HP], mx_[HP], mn_[HP], m = 0x7FFFFFFF, er = 0;
#pragma unroll
        for (int k = 0; k < HP; k++) {
            const int h = lane + 32 * k;
            const bool ok = h < A.VH;
            eh_[k] = ok ? A.ep[h] : 0x7FFFFFFF;
            mx_[k] = ok ? A.pmax[h] : INT32_MIN;
            mn_[k] = ok ? A.pmin[h] : INT32_MAX;
            er |= ok ? A.err[h] : 0;
            m = min(m, eh_[k]);
        }
        for (int h = lane + 32 * HP; h < A.VH; h += 32) { m = min(m, A.ep[h]); er |= A.err[h]; }
        m = __reduce_min_sync(BLK_FULL, m);
        er = (int)__reduce_or_sync(BLK_FULL, (unsigned)er);
        int hi = INT32_MIN, lo = INT32_MAX;
#pragma unroll
        for (int k = 0; k < HP; k++) {
            if (lane + 32 * k < A.VH) {
                const int s = min(eh_[k] - m, 63);
                hi = max(hi, blk_floor_shr32(mx_[k], s));
                lo = min(lo, blk_floor_shr32(mn_[k], s));
            }
        }
        for (int h = lane + 32 * HP; h < A.VH; h += 32) {
            const int s = min(A.ep[h] - m, 63);
            hi = max(hi, blk_floor_shr32(A.pmax[h], s));
            lo = min(lo, blk_floor_shr32(A.pmin[h], s));
        }
        hi = __reduce_max_sync(BLK_FULL, hi);
        lo = __reduce_min_sync(BLK_FULL, lo);
        int sh = max(blk_msb_abs32(hi), blk_msb_abs32(lo)) - 14;
        if (sh < 0) sh = 0;
        const int32_t rq = sh ? 1 << (sh - 1) : 0;
        if (lane == 0) {
            s_ey = m;
            s_sh = sh;
            s_sat = ((hi + rq) >> sh) > 32767 || ((lo + rq) >> sh) < -32768;
            s_err = er;
        }
    }
    __syncthreads();
    const int e_y = s_ey, sh = s_sh;
    const int32_t rq = sh ? 1 << (sh - 1) : 0;
#pragma unroll
    for (int k = 0; k < BLK_S13_PER; k++) {
        const int i = base + BLK_S13_NT * k;
        if (i < n) A.y[i] = g_sat16((blk_floor_shr32(p[k], min(eh[k] - e_y, 63)) + rq) >> sh);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        A.status[0] = e_y - sh;
        A.status[1] = s_err & 1;
        A.status[2] = s_err >> 1 & 1;
        A.status[3] = s_err >> 2 & 1;
        A.status[4] = s_sat;
    }
}

// the conv + segment requantiser unit: one CTA per case (no silu)
__global__ void __launch_bounds__(256)
gdn_conv_unit_kernel(int nch, const int16_t *x, const int16_t *w, const int32_t *cfg, int16_t *sm,
                     int32_t *info)
{
    __shared__ uint64_t red[32];
    const int c = blockIdx.x;
    const int32_t *p = cfg + 9 * c;              // tv[4], e_t[4], cw_exp
    const int32_t tv[4] = {p[0], p[1], p[2], p[3]}, et[4] = {p[4], p[5], p[6], p[7]};
    int tsh[4], vmask;
    const int e_ref = blk_taps(et, tv, tsh, vmask);
    const int16_t *xs = x + (size_t)c * nch * 4, *ws = w + (size_t)c * nch * 4;
    uint64_t am = 0;
    for (int i = threadIdx.x; i < nch; i += blockDim.x) {
        const uint64_t a = g_abs64(blk_conv_ch(xs + 4 * i, ws + 4 * i, vmask, tsh));
        am = a > am ? a : am;
    }
    am = cta_max_u64(am, red);
    int sh = g_msb(am) - 14;
    if (sh < 0) sh = 0;
    for (int i = threadIdx.x; i < nch; i += blockDim.x)
        sm[(size_t)c * nch + i] = g_sat16(g_round_shift(blk_conv_ch(xs + 4 * i, ws + 4 * i, vmask, tsh), sh));
    if (threadIdx.x == 0) {
        const int e_seg = e_ref + p[8] - sh;
        info[3 * c] = e_seg;
        info[3 * c + 1] = sh;
        info[3 * c + 2] = e_seg > 127 || e_seg < -128;
    }
}

// silu unit: element-wise over ncase rows of n, row r on exponent e[r]
__global__ void gdn_silu_unit_kernel(int n, int total, const int16_t *sm, const int32_t *e, int32_t *y)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < total) y[i] = fx_silu(sm[i], e[i / n], d_sig_tab);
}

// L2-norm unit: one warp per vector of N = 32 R
template <int R>
__global__ void __launch_bounds__(32)
gdn_l2norm_unit_kernel(const int32_t *x, int log2n, int16_t *k, int16_t *q)
{
    const int v = blockIdx.x, lane = threadIdx.x;
    int32_t xr[R];
#pragma unroll
    for (int r = 0; r < R; r++) xr[r] = x[(size_t)v * 32 * R + lane + 32 * r];
    fx_l2norm_warp<R>(xr, log2n, false, k + (size_t)v * 32 * R, d_rsqrt_rom);
    fx_l2norm_warp<R>(xr, log2n, true, q + (size_t)v * 32 * R, d_rsqrt_rom);
}

// rmsnorm_bf unit: one warp per vector of N = 32 R
template <int R>
__global__ void __launch_bounds__(32)
gdn_rmsnorm_unit_kernel(const int16_t *xm, const int32_t *xe, const int16_t *wm, const int32_t *we,
                        int16_t *o, int32_t *o_exp)
{
    constexpr int LG = R == 1 ? 5 : (R == 2 ? 6 : 7);
    const int v = blockIdx.x, lane = threadIdx.x;
    int32_t x[R], out[R];
#pragma unroll
    for (int r = 0; r < R; r++) x[r] = xm[(size_t)v * 32 * R + lane + 32 * r];
    int nsat;
    const int e = fx_rmsnorm_warp<R>(x, xe[v], wm + (size_t)v * 32 * R, we[v], LG, out, nsat, d_rsqrt_rom);
#pragma unroll
    for (int r = 0; r < R; r++) o[(size_t)v * 32 * R + lane + 32 * r] = (int16_t)out[r];
    if (lane == 0) o_exp[v] = e;
}

// ------------------------------------------------------------- host entries

static cudaError_t blk_launch(const void *fn, dim3 grid, dim3 block, cudaStream_t st, bool pdl, void **args,
                              int cluster = 1)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// the largest cluster of 8, 4 or 2 CTAs (else 1) of `nt` threads that the
// device can co-schedule for kernel fn, asked once per kernel
static int blk_cluster_max(const void *fn, int nt)
{
    static const void *seen[8] = {};
    static int best[8] = {};
    int slot = 0;
    while (slot < 8 && seen[slot] && seen[slot] != fn) slot++;
    if (slot < 8 && seen[slot] == fn) return best[slot];
    int c = 8;
    for (; c > 1; c >>= 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c);
        cfg.blockDim = dim3(nt);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)c;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n >= 1) break;
        cudaGetLastError();
    }
    if (slot < 8) { best[slot] = c; seen[slot] = fn; }
    return c;
}

// the head kernel's cluster: whole heads (a multiple of the CTAs per head
// sph), dividing the grid; 0 when the device cannot co-schedule one head
static int blk_head_cluster(const void *fn, int nt, int grid, int sph)
{
    int c = blk_cluster_max(fn, nt);
    while (c > sph && grid % c) c >>= 1;
    return c >= sph && grid % c == 0 ? c : 0;
}

static bool blk_dim_ok(int D) { return D == 32 || D == 64 || D == 128; }

extern "C" size_t deltanet_work_bytes(int KH, int VH, int D)
{
    if (KH <= 0 || VH <= 0 || !blk_dim_ok(D)) return 0;
    size_t n = 0;
    blk_work_layout(nullptr, VH, D, &n);
    return n;
}

extern "C" int deltanet_step(const deltanet_args *a, void *stream)
{
    if (!a || a->KH <= 0 || a->VH < a->KH || a->VH % a->KH || !blk_dim_ok(a->D) || !a->xtap || !a->wtap
        || !a->sc || !a->zm || !a->wm || !a->smem || !a->semem || !a->y || !a->status || !a->work)
        return -11;
    if ((((uintptr_t)a->smem) & 31) || (((uintptr_t)a->xtap) & 7) || (((uintptr_t)a->wtap) & 7)
        || (((uintptr_t)a->work) & 255))
        return -11;
    for (int s = 0; s < 3; s++) {
        int any = 0;
        for (int t = 0; t < 4; t++) any |= a->tvalid[s][t] != 0;
        if (!any) return -11;                    // a segment with no valid tap
    }
    cudaError_t e = upload_blk_tables();
    if (e != cudaSuccess) return gdn_fail(e);
    const int KH = a->KH, VH = a->VH, D = a->D;
    const BlkWork w = blk_work_layout(a->work, VH, D, nullptr);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    BlkHeadArgs H;
    H.xtap = a->xtap; H.wtap = a->wtap; H.sc = a->sc; H.KH = KH; H.VH = VH; H.tk0 = a->tk0 != 0;
    H.w_e = a->w_e; H.z_e = a->z_e;
    for (int s = 0; s < 3; s++) {
        H.cw_exp[s] = a->cw_exp[s];
        for (int t = 0; t < 4; t++) { H.e_t[s][t] = a->e_t[s][t]; H.tvalid[s][t] = a->tvalid[s][t] != 0; }
    }
    H.smem = a->smem; H.semem = a->semem; H.zm = a->zm; H.wm = a->wm; H.w = w;
    void *ha[] = {&H};
    const void *hk = D == 32 ? (const void *)gdn_blk_head_kernel<32>
                   : (D == 64 ? (const void *)gdn_blk_head_kernel<64> : (const void *)gdn_blk_head_kernel<128>);
    const int sph = D / 32, grid = VH * sph, hcl = blk_head_cluster(hk, 2 * D, grid, sph);
    if (!hcl) return gdn_fail(cudaErrorInvalidClusterSize);
    e = blk_launch(hk, dim3(grid), dim3(2 * D), st, a->pdl != 0, ha, hcl);
    if (e != cudaSuccess) return gdn_fail(e);

    BlkSite13Args T;
    T.VH = VH; T.D = D; T.po = w.po; T.pz = w.pz; T.ep = w.ep; T.pmax = w.pmax; T.pmin = w.pmin; T.err = w.err;
    T.y = a->y; T.status = a->status;
    void *ta[] = {&T};
    const int n13 = (VH * D + BLK_S13_NT * BLK_S13_PER - 1) / (BLK_S13_NT * BLK_S13_PER);
    e = blk_launch((const void *)gdn_blk_site13_kernel, dim3(n13), dim3(BLK_S13_NT), st, true, ta);
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

// The reference's gdn_block_token on host buffers (same record, same in-place
// state, same sticky flags): stages the record through device memory, runs
// deltanet_step on a private stream and copies the state and outputs back.
extern "C" int gdn_block_token_host(int KH, int VH, int D, gdn_blk_t *b)
{
    if (!b || KH <= 0 || VH < KH || VH % KH || !blk_dim_ok(D) || !b->xtap || !b->wtap || !b->e_t
        || !b->tvalid || !b->cw_exp || !b->sc || !b->zm || !b->wm || !b->smem || !b->semem || !b->y)
        return -11;
    const size_t CH = (size_t)(2 * KH + VH) * D, HD = (size_t)VH * D, wb = deltanet_work_bytes(KH, VH, D);
    const size_t off_x = 0, off_w = off_x + blk_al(CH * 8), off_sc = off_w + blk_al(CH * 8),
                 off_z = off_sc + blk_al((size_t)VH * 32), off_wm = off_z + blk_al(HD * 2),
                 off_s = off_wm + blk_al((size_t)D * 2), off_se = off_s + blk_al(HD * D * 2),
                 off_y = off_se + blk_al(HD * 4), off_st = off_y + blk_al(HD * 2),
                 off_wk = off_st + 256, total = off_wk + wb;
    char *dv = nullptr;
    cudaStream_t st = nullptr;
    cudaError_t e = cudaMalloc(&dv, total);
    if (e != cudaSuccess) return gdn_fail(e);
    e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    int rc = 0;
    int32_t status[5] = {0, 0, 0, 0, 0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_x, b->xtap, CH * 8, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_w, b->wtap, CH * 8, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_sc, b->sc, (size_t)VH * 32, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_z, b->zm, HD * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_wm, b->wm, (size_t)D * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_s, b->smem, HD * D * 2, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv + off_se, b->semem, HD * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        deltanet_args a = {};
        a.KH = KH; a.VH = VH; a.D = D;
        a.xtap = (const int16_t *)(dv + off_x); a.wtap = (const int16_t *)(dv + off_w);
        for (int s = 0; s < 3; s++) {
            a.cw_exp[s] = b->cw_exp[s];
            for (int t = 0; t < 4; t++) { a.e_t[s][t] = b->e_t[4 * s + t]; a.tvalid[s][t] = b->tvalid[4 * s + t]; }
        }
        a.sc = (const int32_t *)(dv + off_sc); a.zm = (const int16_t *)(dv + off_z);
        a.wm = (const int16_t *)(dv + off_wm); a.w_e = b->w_e; a.z_e = b->z_e; a.tk0 = b->tk0;
        a.smem = (int16_t *)(dv + off_s); a.semem = (int32_t *)(dv + off_se);
        a.y = (int16_t *)(dv + off_y); a.status = (int32_t *)(dv + off_st); a.work = dv + off_wk;
        rc = deltanet_step(&a, st);
    }
    if (e == cudaSuccess && rc == 0) e = cudaMemcpyAsync(b->smem, dv + off_s, HD * D * 2, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && rc == 0) e = cudaMemcpyAsync(b->semem, dv + off_se, HD * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && rc == 0) e = cudaMemcpyAsync(b->y, dv + off_y, HD * 2, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && rc == 0) e = cudaMemcpyAsync(status, dv + off_st, sizeof status, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && st) e = cudaStreamSynchronize(st);
    if (st) cudaStreamDestroy(st);
    cudaFree(dv);
    if (e != cudaSuccess) return gdn_fail(e);
    if (rc) return rc;
    b->y_exp = status[0];
    if (status[1]) b->err_conv = 1;
    if (status[2]) b->err_g = 1;
    if (status[3]) b->err_se = 1;
    if (status[4]) b->y_sat = 1;
    return 0;
}

extern "C" int gdn_conv_seg_dev(int ncase, int nch, const int16_t *x, const int16_t *w, const int32_t *cfg,
                                int16_t *sm, int32_t *info, void *stream)
{
    if (ncase <= 0 || nch <= 0 || !x || !w || !cfg || !sm || !info || (((uintptr_t)x | (uintptr_t)w) & 7))
        return -11;
    gdn_conv_unit_kernel<<<ncase, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(nch, x, w, cfg, sm, info);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

extern "C" int gdn_silu_dev(int ncase, int n, const int16_t *sm, const int32_t *e_row, int32_t *y, void *stream)
{
    if (ncase <= 0 || n <= 0 || !sm || !e_row || !y) return -11;
    cudaError_t e = upload_blk_tables();
    if (e != cudaSuccess) return gdn_fail(e);
    const int total = ncase * n;
    gdn_silu_unit_kernel<<<(total + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(n, total, sm, e_row, y);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

extern "C" int gdn_l2norm_dev(int nvec, int N, const int32_t *x, int16_t *k, int16_t *q, void *stream)
{
    if (nvec <= 0 || !blk_dim_ok(N) || !x || !k || !q) return -11;
    cudaError_t e = upload_blk_tables();
    if (e != cudaSuccess) return gdn_fail(e);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (N == 32) gdn_l2norm_unit_kernel<1><<<nvec, 32, 0, st>>>(x, 5, k, q);
    else if (N == 64) gdn_l2norm_unit_kernel<2><<<nvec, 32, 0, st>>>(x, 6, k, q);
    else gdn_l2norm_unit_kernel<4><<<nvec, 32, 0, st>>>(x, 7, k, q);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

extern "C" int gdn_rmsnorm_bf_dev(int nvec, int N, const int16_t *xm, const int32_t *xe, const int16_t *wm,
                                  const int32_t *we, int16_t *o, int32_t *o_exp, void *stream)
{
    if (nvec <= 0 || !blk_dim_ok(N) || !xm || !xe || !wm || !we || !o || !o_exp) return -11;
    cudaError_t e = upload_blk_tables();
    if (e != cudaSuccess) return gdn_fail(e);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (N == 32) gdn_rmsnorm_unit_kernel<1><<<nvec, 32, 0, st>>>(xm, xe, wm, we, o, o_exp);
    else if (N == 64) gdn_rmsnorm_unit_kernel<2><<<nvec, 32, 0, st>>>(xm, xe, wm, we, o, o_exp);
    else gdn_rmsnorm_unit_kernel<4><<<nvec, 32, 0, st>>>(xm, xe, wm, we, o, o_exp);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

extern "C" int gdn_y_emit_dev(int H, int D, const int32_t *ep, const int16_t *po, const int16_t *pz,
                              int16_t *y, int32_t *status, void *stream)
{
    if (H <= 0 || D <= 0 || !ep || !po || !pz || !y || !status) return -11;
    BlkTailArgs T = {};
    T.VH = H; T.D = D; T.po = po; T.pz = pz; T.ep = ep; T.y = y; T.status = status;
    void *ta[] = {&T};
    const int tcl = blk_cluster_max((const void *)gdn_blk_tail_kernel, BLK_TAIL_NT);
    cudaError_t e = blk_launch((const void *)gdn_blk_tail_kernel, dim3(tcl), dim3(BLK_TAIL_NT),
                               reinterpret_cast<cudaStream_t>(stream), false, ta, tcl);
    return e == cudaSuccess ? 0 : gdn_fail(e);
}

extern "C" int gdn_emit_chain_dev(int H, int D, const int64_t *o_acc, const int32_t *e_o, const int16_t *zm,
                                  const int16_t *wm, int we, int z_e, int16_t *y, int32_t *status, void *work,
                                  void *stream)
{
    if (H <= 0 || !blk_dim_ok(D) || !o_acc || !e_o || !zm || !wm || !y || !status || !work
        || (((uintptr_t)work) & 255))
        return -11;
    cudaError_t e = upload_blk_tables();
    if (e != cudaSuccess) return gdn_fail(e);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    BlkChainArgs R = {};
    R.o_acc = o_acc; R.e_o = e_o; R.zm = zm; R.wm = wm; R.w_e = we; R.z_e = z_e;
    R.w = blk_work_layout(work, H, D, nullptr);
    if (D == 32) gdn_blk_chain_kernel<32><<<H, 32, 0, st>>>(R);
    else if (D == 64) gdn_blk_chain_kernel<64><<<H, 32, 0, st>>>(R);
    else gdn_blk_chain_kernel<128><<<H, 32, 0, st>>>(R);
    e = cudaGetLastError();
    if (e != cudaSuccess) return gdn_fail(e);
    return gdn_y_emit_dev(H, D, R.w.ep, R.w.po, R.w.pz, y, status, stream);
}
