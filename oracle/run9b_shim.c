/* oracle/run9b_shim.c -- exports the float layers of the llm.vhdl reference's
 * whole-model reference (ref/run9b.c, "rung 2": INT4 weights dequantised by
 * w_deq, activations in double) so the tests can pin oracle/dec_oracle.py
 * against it.  Compiled in place from the reference tree (never copied) by
 * oracle/Makefile into oracle/_ref/.  TEST INFRASTRUCTURE ONLY.
 *
 * The reference's main() is renamed away; the tests call load_index
 * (ref/run9b.c:236-282) on a synthetic packed directory, then layer_gdn
 * (:602-756) or layer_attn (:758-900) on one layer, with g_bfp = 0 (the
 * reference's --acts f32).
 */
#define main run9b_main
#include "run9b.c"
#undef main

int r9_shape(int32_t *o)
{
    o[0] = N_LAYER; o[1] = ATTN_INT; o[2] = HIDDEN; o[3] = FFN; o[4] = VOCAB; o[5] = LIN_KH;
    o[6] = LIN_VH; o[7] = LIN_HD; o[8] = ATT_QH; o[9] = ATT_KVH; o[10] = ATT_HD; o[11] = N_ROT;
    o[12] = KCONV;
    return 13;
}

double r9_rms_eps(void) { return RMS_EPS; }
double r9_rope_base(void) { return ROPE_BASE; }

int r9_open(const char *dir)
{
    g_bfp = 0;
    load_index(dir);
    return 0;
}

/* One layer on x[HIDDEN] in place.  The state arrays are the reference's own
 * layouts for layers 0..il (conv [il][KCONV-1][CONV_DIM], rec
 * [il][LIN_VH][key][val], caches [il][maxpos][ATT_KVH*ATT_HD]). */
int r9_layer(int il, double *x, double *conv_state, double *rec_state, double *kcache, double *vcache,
             int maxpos, int pos)
{
    state_t S;
    S.conv_state = conv_state; S.rec_state = rec_state;
    S.kcache = kcache; S.vcache = vcache; S.maxpos = maxpos;
    reg_t RX = reg_new(HIDDEN);
    reg_put(&RX, x);
    if (is_attn(il)) layer_attn(il, &S, &RX, pos);
    else layer_gdn(il, &S, &RX, pos);
    memcpy(x, RX.v, sizeof(double) * HIDDEN);
    free(RX.m); free(RX.v);
    return 0;
}

int r9_argmax_first(const double *v, int n) { return argmax_first(v, n); }
