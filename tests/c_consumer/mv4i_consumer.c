/* tests/c_consumer/mv4i_consumer.c -- a plain C consumer of the drop-in
 * boundary, written the way the reference's own consumers use its golden
 * model: tools/ref9b/mv_step_oracle.c:62-63 and ref/run9b.c:110-111 include
 * ref/matvec_int4.c and call mv4i_parse on an image in memory, then
 * mv4i_matvec with host buffers.  Here the same two calls come from
 * include/mv4i_b200.h, linked against libmv4i_b200.so.  Test harness only.
 *
 *   mv4i_consumer parse IMAGE
 *       prints "rc M K w_exp out_shift rows_if nports_w axi_dw"
 *   mv4i_consumer matvec IMAGE X X_EXP N_ROWS N_COLS MODE OUT
 *       X is raw little-endian int16[K]; writes OUT = the output vector
 *       (int16 BFP / int32 RAW / int64 PARTIAL, N_ROWS entries) and prints
 *       "rc y_exp sat_event sat_count ns"
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "mv4i_b200.h"

static uint8_t *slurp(const char *path, size_t *len)
{
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    uint8_t *b = malloc(n > 0 ? (size_t)n : 1);
    if (b && fread(b, 1, (size_t)n, f) != (size_t)n) { free(b); b = NULL; }
    fclose(f);
    *len = (size_t)n;
    return b;
}

int main(int argc, char **argv)
{
    if (argc < 3) return 2;
    size_t len = 0;
    uint8_t *img = slurp(argv[2], &len);
    if (!img) return 3;
    mv4i_file f;
    int rc = mv4i_parse(&f, img, len);
    if (!strcmp(argv[1], "parse")) {
        printf("%d %u %u %d %d %u %u %u\n", rc, f.h.M, f.h.K, f.h.w_exp, f.h.out_shift,
               (unsigned)f.h.rows_if, (unsigned)f.h.nports_w, (unsigned)f.h.axi_dw);
        free(img);
        return 0;
    }
    if (strcmp(argv[1], "matvec") || argc < 9 || rc) { free(img); return 4; }
    size_t xl = 0;
    int16_t *x = (int16_t *)slurp(argv[3], &xl);
    const int x_exp = atoi(argv[4]), n_rows = atoi(argv[5]), n_cols = atoi(argv[6]), mode = atoi(argv[7]);
    int32_t *y_data = calloc((size_t)f.h.M, sizeof *y_data);
    int64_t *y_acc = calloc((size_t)f.h.M, sizeof *y_acc);
    int16_t *y_mant = calloc((size_t)f.h.M, sizeof *y_mant);
    mv4i_result r;
    memset(&r, 0, sizeof r);
    r.y_data = y_data;
    r.y_acc = y_acc;
    r.y_mant = y_mant;
    rc = mv4i_matvec(&f, x, x_exp, n_rows, n_cols, mode, &r);
    printf("%d %d %d %llu %d\n", rc, r.y_exp, r.sat_event, (unsigned long long)r.sat_count, r.ns);
    FILE *o = fopen(argv[8], "wb");
    if (o) {
        if (mode == MV4I_MODE_PARTIAL) fwrite(y_acc, 8, (size_t)n_rows, o);
        else if (mode == MV4I_MODE_RAW) fwrite(y_data, 4, (size_t)n_rows, o);
        else fwrite(y_mant, 2, (size_t)n_rows, o);
        fclose(o);
    }
    mv4i_forget(&f);
    free(x); free(y_data); free(y_acc); free(y_mant); free(img);
    return rc ? 5 : 0;
}
