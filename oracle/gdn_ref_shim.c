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
