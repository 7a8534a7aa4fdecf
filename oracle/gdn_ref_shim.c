/* oracle/gdn_ref_shim.c -- exports pieces of the llm.vhdl reference's own
 * subsystem-B golden model, compiled in place from the reference tree (never
 * copied), so the tests can pin oracle/gdn_oracle.c against it.  TEST
 * INFRASTRUCTURE ONLY; built by oracle/Makefile into oracle/_ref/.
 *
 * ref/gdn_block_vec.c is included with GDN_BLOCK_VEC_NO_MAIN, the guard the
 * reference provides for exactly this (ref/gdn_block_vec.c:532-537); it pulls
 * in gdn_scalar_int (ref/gdn_scalar_vec.c:100) and fx_init (ref/fx.h:51).
 */
#define GDN_BLOCK_VEC_NO_MAIN
#include "gdn_block_vec.c"

void ref_gdn_scalar(int32_t al_m, int al_e, int32_t dt_m, int dt_e, int32_t a_m, int a_e,
                    int32_t b_m, int b_e, int *eg, int *beta, int *err_g)
{
    fx_init();
    gdn_scalar_int(al_m, al_e, dt_m, dt_e, a_m, a_e, b_m, b_e, eg, beta, err_g);
}

void ref_fx_tables(int64_t *e, int64_t *s, int64_t *p)
{
    fx_init();
    for (int k = 0; k <= 256; k++) { e[k] = _fx_exp_lut_q[k]; p[k] = _fx_sp_lut_q[k]; }
    for (int k = 0; k <= 512; k++) s[k] = _fx_sig_lut_q[k];
}

/* The whole fixed-point block token, ref/gdn_block_vec.c:208, with the
 * file globals and one-time set-up its main() performs (:558-561): fx_init,
 * bf_resolve_eps, N = D, SP_Q = 18, the model's key-head map (mod). */
void ref_gdn_block_token(int kh, int vh, int d, blk_t *b)
{
    KH = kh; VH = vh; D = d; N = d; SP_Q = 18; KMAP_DIV = 0;
    fx_init();
    bf_resolve_eps();
    gdn_block_token(b);
}

/* the reference's rsqrt seed ROM (ref/rmsnorm_bf_vec.c:82-91) */
void ref_rsqrt_rom(int64_t *out)
{
    for (int k = 0; k < 64; k++) out[k] = RSQRT_ROM[k];
}

/* ref/l2norm_rs_vec.c:118 */
void ref_l2norm_rs(const int *x, int n, int log2n, int *k, int *q) { l2norm_rs(x, n, log2n, k, q); }

/* ref/rmsnorm_bf_vec.c:199 at N = n, eps 1e-6 */
int ref_rmsnorm_bf(const int16_t *xm, int xe, const int16_t *wm, int we, int n, int16_t *o, int *o_exp)
{
    static bf_out r;
    N = n;
    bf_resolve_eps();
    rmsnorm_bf_int(xm, xe, wm, we, &r);
    for (int j = 0; j < n; j++) o[j] = r.o[j];
    *o_exp = r.o_exp;
    return r.saturations;
}

/* ref/gdn_silu_vec.c:42-80 then the exponent-preserving product */
int ref_silu(int sm, int e)
{
    fx_init();
    return (int)mv4i_round_shift((int64_t)sm * sigma_q15_from_q12(to_q12((int64_t)sm, e)), 15);
}
