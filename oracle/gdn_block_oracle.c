/* oracle/gdn_block_oracle.c -- CPU restatement of llm.vhdl's fixed-point Gated
 * DeltaNet BLOCK (subsystem B, one token end to end).  TEST INFRASTRUCTURE
 * ONLY: the checker the parity tests compare the CUDA block against; the
 * shipped library never links it.
 *
 * Paths are relative to the llm.vhdl project root:
 *
 *   orc_rsqrt_rom        the 64-entry Q30 reciprocal-square-root seed table of
 *                        ref/l2norm_rs_vec.c:63-72 / ref/rmsnorm_bf_vec.c:82-91,
 *                        regenerated as round(2^30 / sqrt(1 + k/64)) and pinned
 *                        against the reference's table by the tests
 *   orc_to_q12           ref/gdn_silu_vec.c:42-57   (site-3 Q12 conversion)
 *   orc_sigma_q15        ref/gdn_silu_vec.c:59-80   (Q12 in, Q15 out, Q30 table)
 *   orc_silu             ref/gdn_block_vec.c:250-253 (exponent preserved)
 *   orc_conv_seg         ref/gdn_block_vec.c:217-245 (spec B 2.1.3 conv and
 *                        segment requantiser; same as ref/gdn_conv_vec.c:80-103)
 *   orc_l2norm_rs        ref/l2norm_rs_vec.c:93-140 (both outputs, Newton rsqrt)
 *   orc_rmsnorm_bf       ref/rmsnorm_bf_vec.c:199-389 (the integer path, with
 *                        numeric_std shift / resize semantics)
 *   orc_y_emit           ref/gdn_block_vec.c:396-418 (site 13; same as
 *                        ref/gdn_y_emit_vec.c:124-143)
 *   orc_emit_chain       ref/gdn_block_vec.c:363-418 (site 12 head emit, output
 *                        norm, z gate, site 13; same as ref/gdn_emit_chain_vec.c)
 *   orc_gdn_block_token  ref/gdn_block_vec.c:208-423 (the whole token over the
 *                        caller-owned blk_t of :183-202, value head h reading
 *                        key head h % KH)
 *
 * The recurrence itself (stages 1-5) and the scalar path are the restatements
 * in gdn_oracle.c (orc_gdn_col_fixed, orc_gdn_scalar).  Pinned by
 * tests/test_gdn_block_pins.py against the reference compiled in place
 * (oracle/_ref/libref_gdn.so) and its committed sim/ vector files.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

int64_t orc_floor_shr(int64_t v, int sh);
int64_t orc_round_shift(int64_t v, int sh);
int16_t orc_sat16(int64_t v);
int orc_msb_pos(uint64_t a);
void orc_fx_init(void);
void orc_fx_tables(int64_t *e, int64_t *s, int64_t *p);
void orc_gdn_scalar(int32_t al_m, int al_e, int32_t dt_m, int dt_e, int32_t a_m, int a_e,
                    int32_t b_m, int b_e, int *eg_out, int *beta_out, int *err_g);
int orc_gdn_col_fixed(int D, int16_t *s, int *se, const int16_t *kn, const int16_t *qs,
                      int32_t v, int e_v, int eg, int beta, int tk0, int64_t *o_acc, int *e_o);
int orc_gdn_head_emit(int D, const int64_t *o_acc, const int *e_o, int16_t *o_head);

static uint64_t mag64(int64_t v) { return v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v; }

/* ------------------------------------------------------------- tables */

static int64_t rom[64];
static int64_t sig_tab[513];
static int tabs_ready;

static void tabs_init(void)
{
    if (tabs_ready) return;
    for (int k = 0; k < 64; k++) rom[k] = llround(1073741824.0 / sqrt(1.0 + (double)k / 64.0));
    int64_t e[257], p[257];
    orc_fx_tables(e, sig_tab, p);
    tabs_ready = 1;
}

void orc_rsqrt_rom(int64_t *out)
{
    tabs_init();
    memcpy(out, rom, sizeof rom);
}

#define INV_SQRT2_Q30 759250125LL        /* round(2^30 / sqrt 2) */

/* ------------------------------------------------------ numeric_std forms */

/* shift_right of a signed: floor division by 2^sh, every count */
static int64_t sra(int64_t v, int sh) { return orc_floor_shr(v, sh); }
/* shift_left of a 64-bit signed: bits past the top dropped, >= 64 gives 0 */
static int64_t sll(int64_t v, int sh)
{
    if (sh <= 0) return v;
    if (sh >= 64) return 0;
    return (int64_t)((uint64_t)v << sh);
}
/* resize(signed, w) narrowing: keep the sign bit and the low w-1 bits */
static int64_t narrow(int64_t v, int w)
{
    if (w >= 64) return v;
    int64_t r = (int64_t)((uint64_t)v & (((uint64_t)1 << (w - 1)) - 1));
    return v < 0 ? r - ((int64_t)1 << (w - 1)) : r;
}
/* highest set bit among bits 0..62; 0 for 0 */
static int msb63(int64_t v)
{
    uint64_t u = (uint64_t)v & 0x7FFFFFFFFFFFFFFFull;
    int p = 0;
    while (u >>= 1) p++;
    return p;
}

/* --------------------------------------------------------- silu (site 3) */

int32_t orc_to_q12(int64_t x, int e)
{
    const int sh = e - 12;
    if (sh >= 0) return sh > 62 ? 0 : (int32_t)orc_round_shift(x, sh);
    const int k = -sh;
    if (k > 40) return x > 0 ? INT32_MAX : (x < 0 ? INT32_MIN : 0);
    const int64_t v = x * ((int64_t)1 << k);
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}

int32_t orc_sigma_q15(int32_t z)
{
    tabs_init();
    const int64_t lim = (int64_t)16 << 12;
    if ((int64_t)z <= -lim) return 0;
    if ((int64_t)z >= lim) return 1 << 15;
    const int64_t pos = ((int64_t)z + lim) * 16;
    int64_t k = pos >> 12;
    if (k > 511) k = 511;
    const int64_t frac = pos - (k << 12);
    const int64_t v30 = sig_tab[k] + (((sig_tab[k + 1] - sig_tab[k]) * frac) >> 12);
    int64_t r = orc_round_shift(v30, 15);
    return (int32_t)(r < 0 ? 0 : (r > 32768 ? 32768 : r));
}

int32_t orc_silu(int32_t sm, int e)
{
    return (int32_t)orc_round_shift((int64_t)sm * orc_sigma_q15(orc_to_q12(sm, e)), 15);
}

/* ----------------------------------------------- conv + segment requantiser */

/* One segment of nch channels, 4 taps each (x[c*4+t], w[c*4+t], tap 3 the
 * current token).  Writes the requantised mantissas sm[nch]; returns the
 * exponent-range error, or -1 when no tap is valid. */
int orc_conv_seg(int nch, const int16_t *x, const int16_t *w, const int *e_t, const int *tv,
                 int cw_exp, int16_t *sm, int *e_seg, int *sh_seg)
{
    int e_ref = 0, have = 0;
    for (int t = 0; t < 4; t++)
        if (tv[t] && (!have || e_t[t] < e_ref)) { e_ref = e_t[t]; have = 1; }
    if (!have) return -1;
    int64_t *acc = malloc((size_t)(nch > 0 ? nch : 1) * sizeof *acc);
    uint64_t amax = 0;
    for (int c = 0; c < nch; c++) {
        int64_t a = 0;
        for (int t = 0; t < 4; t++) {
            if (!tv[t]) continue;
            const int sh = e_t[t] - e_ref;
            a += orc_floor_shr((int64_t)x[c * 4 + t] * w[c * 4 + t], sh > 63 ? 63 : sh);
        }
        acc[c] = a;
        if (mag64(a) > amax) amax = mag64(a);
    }
    int sh = orc_msb_pos(amax) - 14;
    if (sh < 0) sh = 0;
    for (int c = 0; c < nch; c++) sm[c] = orc_sat16(orc_round_shift(acc[c], sh));
    free(acc);
    *e_seg = e_ref + cw_exp - sh;
    *sh_seg = sh;
    return *e_seg > 127 || *e_seg < -128;
}

/* ------------------------------------------------------------- L2 norm */

static int64_t l2_rsqrt(int64_t arg, int *he)
{
    tabs_init();
    const int m = msb63(arg);
    const uint64_t mant = m <= 30 ? (uint64_t)arg << (30 - m) : (uint64_t)arg >> (m - 30);
    const int64_t sm = (int64_t)(uint32_t)mant;
    int64_t y = rom[(mant >> 24) & 63];
    for (int it = 0; it < 2; it++) {
        const int64_t y2 = (int64_t)(int32_t)((y * y) >> 30);
        const int64_t d = (3LL << 30) - ((sm * y2) >> 30);
        y = (int64_t)(int32_t)((d * y) >> 31);
    }
    if (m & 1) { *he = (m - 1) / 2; y = (y * INV_SQRT2_Q30) >> 30; }
    else *he = m / 2;
    return y;
}

/* x[N] -> k (exponent 15) and q (exponent 18, the 1/sqrt(N) fold as a shift
 * of the rsqrt argument by log2n); all zero when the sum of squares is 0. */
void orc_l2norm_rs(const int32_t *x, int N, int log2n, int32_t *k, int32_t *q)
{
    int64_t ssq = 0;
    for (int i = 0; i < N; i++) ssq += (int64_t)x[i] * x[i];
    if (ssq == 0) {
        for (int i = 0; i < N; i++) k[i] = q[i] = 0;
        return;
    }
    int hk, hq;
    const int64_t yk = l2_rsqrt(ssq, &hk), yq = l2_rsqrt(ssq << log2n, &hq);
    const int shk = 15 + hk, shq = 12 + hq;
    for (int i = 0; i < N; i++) {
        k[i] = orc_sat16(((int64_t)x[i] * yk + ((int64_t)1 << (shk - 1))) >> shk);
        q[i] = orc_sat16(((int64_t)x[i] * yq + ((int64_t)1 << (shq - 1))) >> shq);
    }
}

/* ------------------------------------------------------------- rmsnorm */

/* The integer rmsnorm of N int16 mantissas on exponent xe with weights wm on
 * we, epsilon eps, Q = 12; returns the number of saturated outputs. */
int orc_rmsnorm_bf(const int16_t *xm, int xe, const int16_t *wm, int we, int N, double eps,
                   int16_t *o, int *o_exp)
{
    tabs_init();
    const int Q = 12;
    const int e_eps = 30 - (int)floor(log2(eps));
    const int64_t m_eps = llround(ldexp(eps, e_eps));
    int lg = 0;
    while ((1L << lg) < N) lg++;
    const int npow2 = (1L << lg) == N;
    const int rk = npow2 ? 0 : 31 - lg;
    const int64_t rn = npow2 ? 1 : llround(ldexp(1.0, lg + rk) / (double)N);

    int64_t S = 0;
    for (int i = 0; i < N; i++) S += (int64_t)xm[i] * xm[i];
    const int64_t Ss = npow2 ? S : S * rn;
    const int shs = 30 - msb63(Ss);
    const int e_mean = lg + rk + 2 * xe + shs;
    const int64_t m_mean = Ss == 0 ? 0 : (shs >= 0 ? sll(Ss, shs) : sra(Ss, -shs));

    int d, mean_smaller, e_out;
    if (S == 0) { d = 0; mean_smaller = 1; e_out = e_eps; }
    else if (e_mean > e_eps) { d = e_mean - e_eps; mean_smaller = 1; e_out = e_eps; }
    else { d = e_eps - e_mean; mean_smaller = 0; e_out = e_mean; }
    if (d > 63) d = 63;
    const int64_t align = S == 0 ? 0 : (mean_smaller ? sra(m_mean, d) : sra(m_eps, d));
    const int64_t msq = mean_smaller ? align + m_eps : m_mean + align;

    const int p = msb63(msq);
    const uint64_t mant = p <= 30 ? (uint64_t)msq << (30 - p) : (uint64_t)msq >> (p - 30);
    const int64_t sm = (int64_t)(uint32_t)mant;
    int64_t y = rom[(mant >> 24) & 63];
    for (int it = 0; it < 2; it++) {
        const int64_t y2 = narrow(sra(y * y, 30), 32);
        const int64_t diff = narrow((3LL << 30) - narrow(sra(sm * y2, 30), 34), 34);
        y = narrow(sra(diff * y, 31), 32);
    }
    const int rq_d = p - e_out;
    int64_t yf;
    int he;
    if (rq_d % 2 != 0) { yf = narrow(sra(y * INV_SQRT2_Q30, 30), 32); he = (rq_d - 1) / 2; }
    else { yf = y; he = rq_d / 2; }
    const int E = Q - 30 - he;
    int64_t inv;
    if (E > 32) inv = 2147483647LL;
    else if (E >= 0) inv = sll(yf, E);
    else inv = sra(yf + sll(1, -E - 1), -E);
    if (inv > 2147483647LL) inv = 2147483647LL;
    if (inv < 0) inv = 0;

    int64_t *raw = malloc((size_t)N * sizeof *raw);
    int64_t mx = 0;
    for (int j = 0; j < N; j++) {
        raw[j] = narrow(xm[j] * inv, 48) * (int64_t)wm[j];
        const int64_t a = raw[j] < 0 ? -raw[j] : raw[j];
        if (a > mx) mx = a;
    }
    int st = msb63(mx) - 14;
    if (st < 0) st = 0;
    *o_exp = xe + we + Q - st;
    const int64_t bias = st == 0 ? 0 : sll(1, st - 1);
    int nsat = 0;
    for (int j = 0; j < N; j++) {
        const int64_t v = sra(raw[j] + bias, st);
        if (v > 32767 || v < -32768) nsat++;
        o[j] = orc_sat16(v);
    }
    free(raw);
    return nsat;
}

/* -------------------------------------------------------- site 13 emit */

/* The gated product prod_o * prod_z of H heads of D, head h on exponent ep[h],
 * aligned to the minimum exponent by floor and renormalised to int16 with one
 * token exponent; returns 1 when any output saturated. */
int orc_y_emit(int H, int D, const int *ep, const int16_t *po, const int16_t *pz, int16_t *y,
               int *y_exp)
{
    int e_y = ep[0];
    for (int h = 1; h < H; h++) if (ep[h] < e_y) e_y = ep[h];
    int64_t *al = malloc((size_t)H * D * sizeof *al);
    uint64_t amax = 0;
    for (int h = 0; h < H; h++) {
        int s = ep[h] - e_y;
        if (s > 63) s = 63;
        for (int j = 0; j < D; j++) {
            al[h * D + j] = orc_floor_shr((int64_t)po[h * D + j] * pz[h * D + j], s);
            if (mag64(al[h * D + j]) > amax) amax = mag64(al[h * D + j]);
        }
    }
    int sh = orc_msb_pos(amax) - 14;
    if (sh < 0) sh = 0;
    *y_exp = e_y - sh;
    int sat = 0;
    for (int i = 0; i < H * D; i++) {
        const int64_t v = orc_round_shift(al[i], sh);
        if (v > 32767 || v < -32768) sat = 1;
        y[i] = orc_sat16(v);
    }
    free(al);
    return sat;
}

/* Site 12 per head, the output rmsnorm (weights wm on we, eps 1e-6), the z
 * gate silu(z) on z_e, then site 13 over all H heads.  o_acc/e_o/zm [H][D]. */
int orc_emit_chain(int H, int D, const int64_t *o_acc, const int *e_o, const int16_t *zm,
                   const int16_t *wm, int we, int z_e, int16_t *y, int *y_exp)
{
    int16_t *po = malloc((size_t)H * D * 2), *pz = malloc((size_t)H * D * 2), *oh = malloc((size_t)D * 2);
    int *ep = malloc((size_t)H * sizeof *ep);
    for (int h = 0; h < H; h++) {
        const int e_head = orc_gdn_head_emit(D, o_acc + (size_t)h * D, e_o + (size_t)h * D, oh);
        int oe;
        orc_rmsnorm_bf(oh, e_head, wm, we, D, 1.0e-6, po + (size_t)h * D, &oe);
        for (int j = 0; j < D; j++)
            pz[h * D + j] = orc_sat16(orc_silu(zm[h * D + j], z_e));
        ep[h] = oe + z_e;
    }
    const int sat = orc_y_emit(H, D, ep, po, pz, y, y_exp);
    free(po); free(pz); free(oh); free(ep);
    return sat;
}

/* --------------------------------------------------------- the block */

/* Field for field the caller-owned block record of ref/gdn_block_vec.c:183-202. */
typedef struct {
    const int16_t *xtap, *wtap;      /* [2*KH*D + VH*D][4] conv taps / weights  */
    const int *e_t, *tvalid;         /* [3][4] tap exponents / validity         */
    const int *cw_exp;               /* [3] conv weight exponent per segment    */
    const int32_t *sc;               /* [VH][8] scalar-path inputs              */
    const int16_t *zm;               /* [VH][D] z gate mantissas on z_e         */
    const int16_t *wm;               /* [D] output-norm weights on w_e          */
    int w_e, z_e, tk0;
    int16_t *smem;                   /* [VH][D][D] state, in place              */
    int *semem;                      /* [VH][D] column exponents, in place      */
    int16_t *y;                      /* [VH*D] output                           */
    int y_exp, err_conv, err_g, err_se, y_sat;
} orc_blk;

int orc_gdn_block_token(int KH, int VH, int D, orc_blk *b)
{
    const int QCH = KH * D, VCH = VH * D, CH = 2 * QCH + VCH;
    int lg = 0;
    while ((1 << lg) < D) lg++;
    int16_t *sm = malloc((size_t)CH * 2);
    int32_t *sil = malloc((size_t)CH * 4), *kq = malloc((size_t)D * 4), *qq = malloc((size_t)D * 4);
    int16_t *kn = malloc((size_t)QCH * 2), *qs = malloc((size_t)QCH * 2);
    int e_seg[3];
    for (int s = 0; s < 3; s++) {
        const int base = s == 0 ? 0 : (s == 1 ? QCH : 2 * QCH), nch = s == 2 ? VCH : QCH;
        int sh;
        const int rc = orc_conv_seg(nch, b->xtap + (size_t)base * 4, b->wtap + (size_t)base * 4,
                                    b->e_t + 4 * s, b->tvalid + 4 * s, b->cw_exp[s], sm + base,
                                    &e_seg[s], &sh);
        if (rc < 0) { free(sm); free(sil); free(kq); free(qq); free(kn); free(qs); return -1; }
        if (rc) b->err_conv = 1;
        for (int c = 0; c < nch; c++) sil[base + c] = orc_silu(sm[base + c], e_seg[s]);
    }
    for (int h = 0; h < KH; h++) {
        orc_l2norm_rs(sil + h * D, D, lg, kq, qq);                  /* q segment -> q_s */
        for (int i = 0; i < D; i++) qs[h * D + i] = (int16_t)qq[i];
        orc_l2norm_rs(sil + QCH + h * D, D, lg, kq, qq);            /* k segment -> k_n */
        for (int i = 0; i < D; i++) kn[h * D + i] = (int16_t)kq[i];
    }
    int64_t *o_acc = malloc((size_t)VCH * 8);
    int *e_o = malloc((size_t)VCH * sizeof(int));
    for (int h = 0; h < VH; h++) {
        int eg, be, eg_err;
        const int32_t *p = b->sc + (size_t)h * 8;
        orc_gdn_scalar(p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7], &eg, &be, &eg_err);
        if (eg_err) b->err_g = 1;
        const int hk = h % KH;
        for (int j = 0; j < D; j++)
            if (orc_gdn_col_fixed(D, b->smem + ((size_t)h * D + j) * D, b->semem + h * D + j,
                                  kn + hk * D, qs + hk * D, sil[2 * QCH + h * D + j], e_seg[2],
                                  eg, be, b->tk0, o_acc + h * D + j, e_o + h * D + j))
                b->err_se = 1;
    }
    if (orc_emit_chain(VH, D, o_acc, e_o, b->zm, b->wm, b->w_e, b->z_e, b->y, &b->y_exp))
        b->y_sat = 1;
    free(sm); free(sil); free(kq); free(qq); free(kn); free(qs); free(o_acc); free(e_o);
    return 0;
}
