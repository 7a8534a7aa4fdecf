/* oracle/ref_mv4i_shim.c -- exports the llm.vhdl reference's own subsystem-A
 * golden model, compiled in place from the reference tree (never copied), so
 * the tests can pin the restatement in mv4i_oracle.c against it and bench.py
 * can time it as the CPU baseline.  TEST INFRASTRUCTURE ONLY.
 *
 * Built by oracle/Makefile with -I<reference>/ref; the output goes to
 * oracle/_ref/ only.  The reference file is included WITHOUT MV4I_LIB so its
 * static packer pack_geom (ref/matvec_int4.c:456-530) and its self-test main
 * (ref/matvec_int4.c:764, renamed by -Dmain=ref_mv4i_selftest_main) are
 * reachable; mv4i_parse / mv4i_matvec (ref/matvec_int4.c:161,329) are its
 * public entry points.
 */
#include "matvec_int4.c"

int ref_parse(const uint8_t *img, size_t len, int *M, int *K, int *w_exp, int *out_shift)
{
    mv4i_file f;
    int rc = mv4i_parse(&f, img, len);
    if (rc) return rc;
    *M = (int)f.h.M; *K = (int)f.h.K; *w_exp = f.h.w_exp; *out_shift = f.h.out_shift;
    return 0;
}

/* One mv4i_matvec call on an image; outputs into caller arrays. */
int ref_matvec(const uint8_t *img, size_t len, const int16_t *x, int x_exp,
               int n_rows, int n_cols, int mode,
               int32_t *y_data, int64_t *y_acc, int16_t *y_mant,
               int *y_exp, int *sat_event, unsigned long long *sat_count, int *ns)
{
    mv4i_file f;
    int rc = mv4i_parse(&f, img, len);
    if (rc) return 100 + rc;
    mv4i_result r = { y_data, y_acc, y_mant, 0, 0, 0, 0 };
    rc = mv4i_matvec(&f, x, x_exp, n_rows, n_cols, mode, &r);
    if (rc) return rc;
    *y_exp = r.y_exp; *sat_event = r.sat_event; *sat_count = r.sat_count; *ns = r.ns;
    return 0;
}

/* Reference packer; returns a malloc'd image the caller frees with ref_free. */
uint8_t *ref_pack_geom(int M, int K, int rows_if, int axi_dw, int w_exp, int out_shift,
                       const int8_t cb[16], const uint8_t *idx, const uint16_t *scl,
                       size_t *out_len)
{
    return pack_geom(M, K, rows_if, axi_dw, w_exp, out_shift, cb, idx, scl, out_len);
}

void ref_free(void *p) { free(p); }

const int8_t *ref_iq4_nl(void) { return IQ4_NL; }

/* The reference's static byte accessors (ref/matvec_int4.c:267-307) over a
 * whole image: every weight index [M][K] and every 32-block scale [M][nb]. */
int ref_dump_layout(const uint8_t *img, size_t len, uint8_t *widx, uint16_t *scale)
{
    mv4i_file f;
    int rc = mv4i_parse(&f, img, len);
    if (rc) return rc;
    const int M = (int)f.h.M, K = (int)f.h.K, nb = (K + 31) / 32;
    for (int r = 0; r < M; r++) {
        for (int k = 0; k < K; k++) widx[(size_t)r * K + k] = (uint8_t)get_widx(&f, r, k);
        for (int b = 0; b < nb; b++) scale[(size_t)r * nb + b] = get_scale(&f, r, b);
    }
    return 0;
}
