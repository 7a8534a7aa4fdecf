/* llm.vhdl_b200/csrc/mv4i_pack.c -- the offline side of the weight path:
 * quantise a float matrix to the .mv4i format, pick out_shift, emit the
 * .mv4i image, and convert an image whose format allows it into the decode
 * engine's g128 layout.  Host code (no device calls).
 *
 * Follows tools/pack_int4.py of the reference (paths relative to the llm.vhdl
 * project root):
 *   mv4i_quantize            quantize()            :280-359  (spec 6.1)
 *   mv4i_calibrate_out_shift calibrate_out_shift() :434-446  (spec 7.4)
 *   mv4i_pack_size           packed_layout()       :451-486  (spec 6.4/6.5a)
 *   mv4i_pack                pack()                :488-559  (spec 6.4/6.5a)
 * The quantiser's arithmetic is the reference's float32 arithmetic, operation
 * for operation, including the order in which a 32-weight block's squared
 * errors are summed (eight strided partial sums, then a fixed tree: the
 * reduction the reference's array library performs), so the per-block
 * least-squares choice -- and therefore the image -- is byte-identical.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "../../include/mv4i_b200.h"

#define PK_BLOCK 32
#define PK_HDR   4096

static size_t al4k(size_t n) { return (n + 4095) & ~(size_t)4095; }

static int gcd_i(int a, int b) { while (b) { const int t = a % b; a = b; b = t; } return a; }

/* NPORTS_W, scale sub-regions and scale groups per superword of a geometry;
 * 0 when the reference refuses it (tools/pack_int4.py check_geometry) */
static int pk_geometry(int rows_if, int axi_dw, int *nports, int *nss, int *grp)
{
    static const int widths[] = {8, 16, 32, 64, 128, 256, 512, 1024};
    const int lane_bits = rows_if * PK_BLOCK * 4;
    int ok = 0;
    for (int i = 0; i < 8; i++) ok |= axi_dw == widths[i];
    if (rows_if <= 0 || !ok || lane_bits % axi_dw) return 0;
    const int sw = rows_if * 16;
    const int lcm = sw / gcd_i(sw, axi_dw) * axi_dw;
    *nports = lane_bits / axi_dw;
    *nss = lcm / axi_dw;
    *grp = *nss * axi_dw / sw;
    if (0x38 + 8 * (*nports + *nss) > PK_HDR) return 0;   /* offset table past the header */
    return 1;
}

size_t mv4i_pack_size(int M, int K, int rows_if, int axi_dw)
{
    int nports, nss, grp;
    if (M <= 0 || K <= 0 || !pk_geometry(rows_if, axi_dw, &nports, &nss, &grp)) return 0;
    const size_t NB = (size_t)(K + PK_BLOCK - 1) / PK_BLOCK, tiles = (size_t)(M + rows_if - 1) / rows_if;
    const size_t port_b = (size_t)axi_dw / 8;
    const size_t sub_sz = al4k(tiles * NB * port_b);
    const size_t nsuper = (tiles * NB + grp - 1) / grp;
    return PK_HDR + sub_sz * nports + al4k(nsuper * port_b) * nss;
}

int mv4i_calibrate_out_shift(int K)
{
    if (K <= 0) return -11;
    const int NB = (K + PK_BLOCK - 1) / PK_BLOCK;
    int lg = 0;
    while ((1 << lg) < NB) lg++;                     /* ceil(log2 NB) */
    const int bits = NB > 1 ? 27 + lg : 27;
    const int s = bits - 31;
    return s < 0 ? 0 : (s > 40 ? 40 : s);
}

static void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static void put32(uint8_t *p, uint32_t v) { for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i)); }
static void put64(uint8_t *p, uint64_t v) { for (int i = 0; i < 8; i++) p[i] = (uint8_t)(v >> (8 * i)); }

int mv4i_pack(const uint8_t *idx, const uint16_t *scale, int w_exp, int M, int K, int rows_if, int out_shift,
              const int8_t cb[16], int axi_dw, uint8_t *out)
{
    int nports, nss, grp;
    if (!idx || !scale || !cb || !out || M <= 0 || K <= 0 || out_shift < 0 || out_shift > 40
        || !pk_geometry(rows_if, axi_dw, &nports, &nss, &grp))
        return -11;
    for (int i = 0; i < 16; i++) if (cb[i] == -128) return -11;
    const size_t NB = (size_t)(K + PK_BLOCK - 1) / PK_BLOCK, tiles = (size_t)(M + rows_if - 1) / rows_if;
    const size_t port_b = (size_t)axi_dw / 8, word_b = (size_t)rows_if * (PK_BLOCK / 2);
    const size_t sub_sz = al4k(tiles * NB * port_b);
    const size_t nsuper = (tiles * NB + grp - 1) / grp, scl_sub_sz = al4k(nsuper * port_b);
    const size_t total = PK_HDR + sub_sz * nports + scl_sub_sz * nss;
    memset(out, 0, total);                           /* pad fill 0x00 (spec 6.4) */
    /* header (spec 6.4, little endian) */
    put32(out + 0x00, MV4I_MAGIC);
    put16(out + 0x04, 1);                            /* version */
    put16(out + 0x06, 1);                            /* flags */
    put32(out + 0x08, (uint32_t)M);
    put32(out + 0x0C, (uint32_t)K);
    put32(out + 0x10, (uint32_t)w_exp);
    put32(out + 0x14, (uint32_t)out_shift);
    put16(out + 0x18, (uint16_t)rows_if);
    put16(out + 0x1A, (uint16_t)nports);
    put16(out + 0x1C, PK_BLOCK);
    put16(out + 0x1E, (uint16_t)axi_dw);
    memcpy(out + 0x20, cb, 16);
    const size_t scl_off = PK_HDR + sub_sz * nports;
    put32(out + 0x30, (uint32_t)scl_off);
    put32(out + 0x34, (uint32_t)nss);
    for (int p = 0; p < nports; p++) put64(out + 0x38 + 8 * p, PK_HDR + sub_sz * p);
    for (int q = 0; q < nss; q++) put64(out + 0x38 + 8 * (nports + q), scl_off + scl_sub_sz * q);
    /* weights (spec 6.5a): the tile word of (t, b) is the ROWS_IF rows' 16-byte
     * chunks with row 0 at the lowest byte; sub-region p holds bytes
     * [p*port_b, (p+1)*port_b) of every word, t-major then b */
    for (size_t t = 0; t < tiles; t++)
        for (size_t b = 0; b < NB; b++)
            for (size_t wb = 0; wb < word_b; wb++) {
                const size_t rr = wb / (PK_BLOCK / 2), j2 = wb % (PK_BLOCK / 2);
                const size_t r = t * rows_if + rr;
                uint8_t v = 0;
                if (r < (size_t)M) {
                    const uint8_t *ix = idx + (r * NB + b) * PK_BLOCK + 2 * j2;
                    v = (uint8_t)((ix[0] & 15) | ((ix[1] & 15) << 4));
                }
                const size_t p = wb / port_b, off = wb % port_b;
                out[PK_HDR + sub_sz * p + (t * NB + b) * port_b + off] = v;
            }
    /* scales: groups of ROWS_IF uint16 in (t, b) order, as superwords of nss
     * beats sliced across the nss sub-regions */
    const size_t gbytes = tiles * NB * (size_t)rows_if * 2, sup_b = (size_t)nss * port_b;
    for (size_t i = 0; i < gbytes; i += 2) {
        const size_t g = i / ((size_t)rows_if * 2), rr = (i / 2) % rows_if;
        const size_t t = g / NB, b = g % NB, r = t * rows_if + rr;
        const uint16_t s = r < (size_t)M ? scale[r * NB + b] : 0;
        for (int h = 0; h < 2; h++) {
            const size_t fb = i + h, su = fb / sup_b, in_su = fb % sup_b;
            const size_t q = in_su / port_b, off = in_su % port_b;
            out[scl_off + scl_sub_sz * q + su * port_b + off] = (uint8_t)(s >> (8 * h));
        }
    }
    return 0;
}

/* sum of 32 floats in the fixed order: eight strided partial sums, then a tree */
static float sum32(const float *a)
{
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    for (int i = 8; i < 32; i += 8)
        for (int j = 0; j < 8; j++) r[j] = r[j] + a[i + j];
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

int mv4i_quantize(const float *W, int M, int K, const int8_t cb[16], uint8_t *idx, uint16_t *scale, int *w_exp)
{
    if (!W || !cb || !idx || !scale || !w_exp || M <= 0 || K <= 0) return -11;
    const int NB = (K + PK_BLOCK - 1) / PK_BLOCK;
    float cbf[16], mids[15], cb_amax = 0.f;
    for (int i = 0; i < 16; i++) { cbf[i] = (float)cb[i]; cb_amax = fmaxf(cb_amax, fabsf(cbf[i])); }
    for (int i = 0; i < 15; i++) {
        if (cb[i + 1] <= cb[i]) return -11;          /* the search needs an ascending codebook */
        mids[i] = (cbf[i] + cbf[i + 1]) * 0.5f;
    }
    float gmax = 0.f;
    for (size_t i = 0; i < (size_t)M * K; i++) gmax = fmaxf(gmax, fabsf(W[i]));
    memset(idx, 0, (size_t)M * NB * PK_BLOCK);
    memset(scale, 0, (size_t)M * NB * 2);
    if (gmax == 0.f) { *w_exp = 0; return 0; }
    const int we = (int)floor(log2((double)cb_amax / (double)gmax));
    *w_exp = we;
    const float pw = (float)ldexp(1.0, we);
    const float kbase = (float)(32768.0 / (double)cb_amax);
    static const float mults[8] = {0.80f, 0.86f, 0.90f, 0.94f, 0.97f, 1.00f, 1.03f, 1.07f};
    float tgt[PK_BLOCK], d2[PK_BLOCK];
    uint8_t ix[PK_BLOCK];
    for (int r = 0; r < M; r++)
        for (int b = 0; b < NB; b++) {
            float amax = 0.f;
            for (int j = 0; j < PK_BLOCK; j++) {
                const int k = b * PK_BLOCK + j;
                tgt[j] = (k < K ? W[(size_t)r * K + k] : 0.f) * pw;
                if (k < K) amax = fmaxf(amax, fabsf(tgt[j]));
            }
            const float base = amax * kbase;
            float best_err = INFINITY;
            uint16_t best_s = 0;
            uint8_t best_ix[PK_BLOCK];
            memset(best_ix, 0, sizeof best_ix);
            for (int m = 0; m < 8; m++) {
                float v = rintf(base * mults[m]);
                v = v < 0.f ? 0.f : (v > 32767.f ? 32767.f : v);
                const uint16_t sc = (uint16_t)v;
                const float s = (float)sc / 32768.0f;
                const float ss = s > 0.f ? s : 1.0f;
                for (int j = 0; j < PK_BLOCK; j++) {
                    const float q = tgt[j] / ss;
                    int n = 0;
                    while (n < 15 && mids[n] < q) n++;   /* first mid >= q */
                    ix[j] = (uint8_t)n;
                    const float e = cbf[n] * ss - tgt[j];
                    const int k = b * PK_BLOCK + j;
                    d2[j] = (e * e) * (k < K ? 1.0f : 0.0f);
                }
                const float err = sum32(d2);
                if (err < best_err) {
                    best_err = err;
                    best_s = sc;
                    memcpy(best_ix, ix, sizeof ix);
                }
            }
            uint8_t *o = idx + ((size_t)r * NB + b) * PK_BLOCK;
            for (int j = 0; j < PK_BLOCK; j++)
                o[j] = (best_s == 0 || b * PK_BLOCK + j >= K) ? 0 : best_ix[j];
            scale[(size_t)r * NB + b] = best_s;
        }
    return 0;
}

/* An image whose values the g128 format holds exactly -> the decode engine's
 * layout (INT4 two's-complement nibbles along K, one fp16 scale per 128
 * columns).  Needs the linear codebook {0..7, -8..-1}, K a multiple of 128,
 * the same uint15 scale in all four 32-blocks of a group, and every scale *
 * 2^-(15 + w_exp) an fp16 normal number or zero. */
int mv4i_image_to_g128(const mv4i_file *f, uint8_t *wq, uint16_t *sc, int sc_pitch)
{
    if (!f || !f->base || !wq || !sc) return -11;
    const int M = (int)f->h.M, K = (int)f->h.K, ng = K / 128;
    if (K % 128 || sc_pitch < ng) return -11;
    for (int i = 0; i < 16; i++) if (f->h.codebook[i] != (i < 8 ? i : i - 16)) return -11;
    for (int r = 0; r < M; r++) {
        for (int g = 0; g < ng; g++) {
            const uint16_t s0 = mv4i_get_scale(f, r, 4 * g);
            for (int b = 1; b < 4; b++) if (mv4i_get_scale(f, r, 4 * g + b) != s0) return -11;
            const double v = ldexp((double)s0, -15 - f->h.w_exp);
            if (v != 0.0 && (v < ldexp(1.0, -14) || v > 65504.0)) return -11;
            /* fp16 of v, exact or refused */
            int e;
            const double m = frexp(v, &e);                   /* v = m * 2^e, m in [0.5, 1) */
            uint16_t h = 0;
            if (v != 0.0) {
                const double mant = ldexp(m, 11);            /* 11 significant bits */
                if (mant != floor(mant)) return -11;
                h = (uint16_t)(((e - 1 + 15) << 10) | ((uint32_t)mant & 0x3FF));
            }
            sc[(size_t)r * sc_pitch + g] = h;
        }
        for (int k = 0; k < K; k += 2) {
            const int a = mv4i_get_widx(f, r, k), b = mv4i_get_widx(f, r, k + 1);
            wq[(size_t)r * (K / 2) + k / 2] = (uint8_t)((a & 15) | ((b & 15) << 4));
        }
    }
    return 0;
}

/* fp16 bits of a finite non-negative float, round to nearest even; 0xFFFF when
 * it overflows fp16 */
static uint16_t f32_to_f16_pos(float f)
{
    if (!(f >= 0.f)) return 0xFFFF;
    if (f == 0.f) return 0;
    int e;
    const double m = frexp((double)f, &e);           /* f = m * 2^e, m in [0.5, 1) */
    if (e > 16) return 0xFFFF;
    if (e >= -13) {                                  /* normal: 11 significant bits */
        double q = rint(ldexp(m, 11));
        if (q == 2048.0) { q = 1024.0; e++; }
        if (e > 16) return 0xFFFF;
        const uint16_t h = (uint16_t)(((e - 1 + 15) << 10) | ((uint32_t)q & 0x3FF));
        return h >= 0x7C00 ? 0xFFFF : h;
    }
    return (uint16_t)rint(ldexp((double)f, 24));     /* subnormal: units of 2^-24 */
}

int mv4i_quantize_g128(const float *W, int M, int K, uint8_t *wq, uint16_t *sc, int sc_pitch)
{
    if (!W || !wq || !sc || M <= 0 || K <= 0 || K % 128 || sc_pitch < K / 128) return -11;
    for (int r = 0; r < M; r++)
        for (int g = 0; g < K / 128; g++) {
            const float *w = W + (size_t)r * K + 128 * g;
            float amax = 0.f;
            for (int j = 0; j < 128; j++) amax = fmaxf(amax, fabsf(w[j]));
            const uint16_t h = f32_to_f16_pos(amax / 7.0f);
            if (h == 0xFFFF) return -11;
            sc[(size_t)r * sc_pitch + g] = h;
            /* the scale as fp16 stores it */
            const float s = (h >> 10) ? ldexpf((float)(1024 | (h & 0x3FF)), (h >> 10) - 25)
                                      : ldexpf((float)h, -24);
            for (int j = 0; j < 128; j += 2) {
                int q[2];
                for (int t = 0; t < 2; t++) {
                    const float v = s > 0.f ? rintf(w[j + t] / s) : 0.f;
                    q[t] = v < -8.f ? -8 : (v > 7.f ? 7 : (int)v);
                }
                wq[(size_t)r * (K / 2) + 64 * g + j / 2] = (uint8_t)((q[0] & 15) | ((q[1] & 15) << 4));
            }
        }
    return 0;
}
