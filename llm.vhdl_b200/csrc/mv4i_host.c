/* llm.vhdl_b200/csrc/mv4i_host.c -- host side of the B200 subsystem-A library.
 *
 *   mv4i_parse        replaces ref/matvec_int4.c:161-255 (same checks, same order,
 *                     same refusal codes; the parsed file borrows the image)
 *   mv4i_get_widx /   replace ref/matvec_int4.c:267-307 (spec 6.5 / 6.5a byte
 *   mv4i_get_scale    layout, any AXI4 width)
 *   mv4i_dmat_upload  .mv4i image -> stream layout in HBM (rows contiguous along K)
 *   mv4i_matvec       replaces ref/matvec_int4.c:329-441 with host buffers; the
 *                     device copy of each image is cached by (base, header)
 *
 * Plain C over the CUDA runtime API.  No allocation happens on the matvec path
 * after the first call for an image except growth of the staging buffers.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <cuda_runtime_api.h>
#include "../../include/mv4i_b200.h"

extern int mv4i_g_cuda_err;      /* defined in mv4i_kernels.cu */
static int fail_cuda(cudaError_t e) { mv4i_g_cuda_err = (int)e; return -20; }

/* ------------------------------------------------------------------ parse */

static uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
static uint32_t rd32(const uint8_t *p) { return rd16(p) | (rd16(p + 2) << 16); }
static uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

static uint32_t gcd32(uint32_t a, uint32_t b) { while (b) { uint32_t t = a % b; a = b; b = t; } return a; }

/* scale sub-regions: smallest n with n*AXI_DW a whole number of ROWS_IF*16-bit groups */
static uint32_t n_scale_sub_of(uint32_t rows_if, uint32_t axi_dw)
{
    uint32_t sw = rows_if * 16u;
    return (sw && axi_dw) ? sw / gcd32(sw, axi_dw) : 0;
}

static int is_axi4(uint32_t w)
{
    switch (w) { case 8: case 16: case 32: case 64: case 128: case 256: case 512: case 1024: return 1; }
    return 0;
}

int mv4i_parse(mv4i_file *f, const uint8_t *img, size_t len)
{
    if (!f || !img) return -11;
    if (len < MV4I_HDR_BYTES) return -1;
    mv4i_hdr *h = &f->h;
    h->magic = rd32(img);
    if (h->magic != MV4I_MAGIC) return -2;
    h->version   = (uint16_t)rd16(img + 0x04);
    h->flags     = (uint16_t)rd16(img + 0x06);
    h->M         = rd32(img + 0x08);
    h->K         = rd32(img + 0x0C);
    h->w_exp     = (int32_t)rd32(img + 0x10);
    h->out_shift = (int32_t)rd32(img + 0x14);
    h->rows_if   = (uint16_t)rd16(img + 0x18);
    h->nports_w  = (uint16_t)rd16(img + 0x1A);
    h->block     = (uint16_t)rd16(img + 0x1C);
    h->axi_dw    = (uint16_t)rd16(img + 0x1E);
    if (h->axi_dw == 0) h->axi_dw = 128;          /* written before the field existed */
    memcpy(h->codebook, img + 0x20, 16);
    h->scale_offset = rd32(img + 0x30);
    h->n_scale_sub  = rd32(img + 0x34);

    if (h->block != MV4I_BLOCK || h->rows_if == 0) return -3;
    if ((uint32_t)h->nports_w * h->axi_dw != (uint32_t)h->rows_if * h->block * 4u) return -4;
    if (!is_axi4(h->axi_dw)) return -7;
    if (h->nports_w == 0 || h->nports_w > MV4I_MAX_SUB) return -8;
    if (h->n_scale_sub == 0) { h->n_scale_sub = 1; h->s_sub_offset[0] = h->scale_offset; }
    if (h->n_scale_sub > MV4I_MAX_SUB) return -8;
    if (h->n_scale_sub != n_scale_sub_of(h->rows_if, h->axi_dw)) return -9;
    if (0x38u + 8u * ((uint32_t)h->nports_w + h->n_scale_sub) > MV4I_HDR_BYTES) return -8;
    for (unsigned i = 0; i < h->nports_w; i++) h->w_sub_offset[i] = rd64(img + 0x38 + 8 * i);
    if (rd32(img + 0x34) != 0)
        for (unsigned i = 0; i < h->n_scale_sub; i++)
            h->s_sub_offset[i] = rd64(img + 0x38 + 8 * h->nports_w + 8 * i);
    f->port_b = (int)(h->axi_dw / 8u);
    f->grp    = (int)(h->n_scale_sub * h->axi_dw / (h->rows_if * 16u));
    for (int i = 0; i < 16; i++) if (h->codebook[i] == -128) return -5;
    if (h->out_shift < 0 || h->out_shift > 40) return -6;
    f->base = img;
    f->nb   = (int)((h->K + MV4I_BLOCK - 1) / MV4I_BLOCK);
    return 0;
}

/* ------------------------------------------------------------- accessors */

int mv4i_get_widx(const mv4i_file *f, int r, int k)
{
    const int ri = f->h.rows_if, t = r / ri, rr = r % ri;
    const int b = k / MV4I_BLOCK, j = k % MV4I_BLOCK;
    const size_t wb = (size_t)rr * (MV4I_BLOCK / 2) + (size_t)(j >> 1);
    const uint8_t *sub = f->base + f->h.w_sub_offset[wb / (size_t)f->port_b];
    const uint8_t byte = sub[((size_t)t * f->nb + b) * (size_t)f->port_b + wb % (size_t)f->port_b];
    return (j & 1) ? (byte >> 4) : (byte & 0x0F);
}

static uint8_t scale_byte(const mv4i_file *f, size_t super, size_t bo)
{
    return f->base[f->h.s_sub_offset[bo / (size_t)f->port_b] + super * (size_t)f->port_b
                   + bo % (size_t)f->port_b];
}

uint16_t mv4i_get_scale(const mv4i_file *f, int r, int b)
{
    const int ri = f->h.rows_if, t = r / ri, rr = r % ri;
    const size_t g = (size_t)t * f->nb + (size_t)b;
    const size_t bo = (g % (size_t)f->grp) * (size_t)ri * 2u + (size_t)rr * 2u;
    const size_t su = g / (size_t)f->grp;
    return (uint16_t)(scale_byte(f, su, bo) | ((uint16_t)scale_byte(f, su, bo + 1) << 8));
}

/* -------------------------------------------------------------- relayout */

/* Stream layout: row r, block b = 16 bytes at r*pitch + 16*b, scale (r, b) at
 * sc[r*spitch + b]; rows are padded with zeros to whole 128-column groups
 * (pitch = 64*ceil(nb/4), spitch = 4*ceil(nb/4)) so every row starts 64-byte
 * aligned.  Row r of tile t sits in the tile word at byte rr*16, so for each
 * (tile, block) beat the word's bytes are scattered to their rows; the
 * sub-region slicing (6.5a) only decides which beat holds which byte. */
static void relayout(const mv4i_file *f, uint8_t *wq, uint16_t *sc, size_t pitch, size_t spitch)
{
    const int M = (int)f->h.M, nb = f->nb, ri = f->h.rows_if, pb = f->port_b;
    const int tiles = (M + ri - 1) / ri;
    const int word_b = ri * 16;
    for (int t = 0; t < tiles; t++)
        for (int b = 0; b < nb; b++) {
            const size_t beat = ((size_t)t * nb + b) * (size_t)pb;
            for (int wb0 = 0; wb0 < word_b; wb0 += pb) {
                const uint8_t *src = f->base + f->h.w_sub_offset[wb0 / pb] + beat;
                for (int o = 0; o < pb; o++) {
                    const int wb = wb0 + o, r = t * ri + wb / 16;
                    if (r < M) wq[(size_t)r * pitch + (size_t)b * 16 + (size_t)(wb % 16)] = src[o];
                }
            }
        }
    for (int r = 0; r < M; r++)
        for (int b = 0; b < nb; b++) sc[(size_t)r * spitch + b] = mv4i_get_scale(f, r, b);
}

int mv4i_dmat_upload(const mv4i_file *f, int device, mv4i_dmat *out)
{
    if (!f || !out || !f->base) return -11;
    memset(out, 0, sizeof *out);
    const int M = (int)f->h.M, nb = f->nb;
    if (M <= 0 || nb <= 0) return -11;
    const size_t ngr = (size_t)(nb + 3) / 4;
    const size_t pitch = ngr * 64, spitch = ngr * 4;
    const size_t wbytes = (size_t)M * pitch, sbytes = (size_t)M * spitch * 2;
    const size_t soff = (wbytes + 255) & ~(size_t)255;
    uint8_t *host = (uint8_t *)calloc(1, soff + sbytes);
    if (!host) return -11;
    relayout(f, host, (uint16_t *)(host + soff), pitch, spitch);
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    void *d = NULL;
    if (e == cudaSuccess) e = cudaMalloc(&d, soff + sbytes);
    if (e == cudaSuccess) e = cudaMemcpy(d, host, soff + sbytes, cudaMemcpyHostToDevice);
    free(host);
    cudaSetDevice(prev);
    if (e != cudaSuccess) { if (d) cudaFree(d); return fail_cuda(e); }
    out->wq = (const uint8_t *)d;
    out->sc = (const uint8_t *)d + soff;
    out->w_pitch = (int64_t)pitch;
    out->s_pitch = (int64_t)spitch;
    out->M = M; out->K = (int32_t)f->h.K;
    out->w_exp = f->h.w_exp; out->out_shift = f->h.out_shift;
    memcpy(out->codebook, f->h.codebook, 16);
    out->kind = MV4I_KIND_GOLDEN;
    out->device = device;
    out->owned = d;
    return 0;
}

int mv4i_dmat_wrap_g128(const uint8_t *d_wq, int64_t w_pitch, const uint16_t *d_scales,
                        int64_t s_pitch, int M, int K, int device, mv4i_dmat *out)
{
    if (!d_wq || !d_scales || !out || M <= 0 || K <= 0 || (K % 128) || (w_pitch & 15)
        || w_pitch < K / 2 || s_pitch < K / 128) return -11;
    memset(out, 0, sizeof *out);
    out->wq = d_wq; out->sc = d_scales;
    out->w_pitch = w_pitch; out->s_pitch = s_pitch;
    out->M = M; out->K = K;
    for (int i = 0; i < 16; i++) out->codebook[i] = (int8_t)(i < 8 ? i : i - 16);
    out->kind = MV4I_KIND_G128;
    out->device = device;
    return 0;
}

int mv4i_dmat_wrap_golden(const uint8_t *d_wq, int64_t w_pitch, const uint16_t *d_scales,
                          int64_t s_pitch, int M, int K, int w_exp, int out_shift,
                          const int8_t codebook[16], int device, mv4i_dmat *out)
{
    const int nb = (K + MV4I_BLOCK - 1) / MV4I_BLOCK;
    if (!d_wq || !d_scales || !out || !codebook || M <= 0 || K <= 0 || (w_pitch & 15)
        || w_pitch < (int64_t)nb * 16 || s_pitch < nb || out_shift < 0 || out_shift > 40) return -11;
    for (int i = 0; i < 16; i++) if (codebook[i] == -128) return -5;
    memset(out, 0, sizeof *out);
    out->wq = d_wq; out->sc = d_scales;
    out->w_pitch = w_pitch; out->s_pitch = s_pitch;
    out->M = M; out->K = K; out->w_exp = w_exp; out->out_shift = out_shift;
    memcpy(out->codebook, codebook, 16);
    out->kind = MV4I_KIND_GOLDEN;
    out->device = device;
    return 0;
}

int mv4i_dmat_rows(const mv4i_dmat *m, int row0, int n, mv4i_dmat *view)
{
    if (!m || !view || row0 < 0 || n <= 0 || row0 + n > m->M) return -11;
    *view = *m;
    view->wq = m->wq + (int64_t)row0 * m->w_pitch;
    view->sc = (const uint8_t *)m->sc + (int64_t)row0 * m->s_pitch * 2;
    view->M = n;
    view->owned = NULL;
    return 0;
}

int mv4i_dmat_free(mv4i_dmat *m)
{
    if (!m) return -11;
    if (m->owned) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(m->device);
        cudaError_t e = cudaFree(m->owned);
        cudaSetDevice(prev);
        if (e != cudaSuccess) return fail_cuda(e);
    }
    memset(m, 0, sizeof *m);
    return 0;
}

/* ------------------------------------------------------ drop-in matvec */

#define CACHE_N 64

typedef struct {
    const uint8_t *base;
    mv4i_hdr       h;
    uint64_t       fp;          /* sampled content fingerprint */
    int            device;
    mv4i_dmat      m;
    uint64_t       stamp;
} cache_ent;

typedef struct {
    int          device;
    cudaStream_t stream;
    void        *d_buf;       /* x | y_data | y_mant | y_acc | status | scratch */
    size_t       cap;
    void        *h_buf;       /* pinned staging */
    size_t       hcap;
} dev_ctx;

static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
static cache_ent g_cache[CACHE_N];
static uint64_t g_stamp;
static dev_ctx g_ctx[16];

static int hdr_same(const mv4i_hdr *a, const mv4i_hdr *b) { return memcmp(a, b, sizeof *a) == 0; }

static uint64_t fnv1a(uint64_t h, const uint8_t *p, size_t n)
{
    for (size_t i = 0; i < n; i++) { h ^= p[i]; h *= 0x100000001B3ull; }
    return h;
}

/* Fingerprint of an image: the 4 KB header plus 128 evenly spaced 32-byte
 * windows of every weight and scale sub-region (~20 KB hashed per call).
 * It catches the usual way a pointer-keyed cache goes stale -- an image freed
 * and another of the same geometry allocated at the same address -- but not
 * an edit of a few bytes between samples; that case needs mv4i_forget. */
static uint64_t image_fp(const mv4i_file *f)
{
    uint64_t h = fnv1a(0xCBF29CE484222325ull, f->base, MV4I_HDR_BYTES);
    const int ri = f->h.rows_if;
    const uint64_t tiles = (f->h.M + (uint64_t)ri - 1) / ri;
    const uint64_t wlen = tiles * (uint64_t)f->nb * (uint64_t)f->port_b;
    const uint64_t slen = ((tiles * (uint64_t)f->nb + (uint64_t)f->grp - 1) / (uint64_t)f->grp) * (uint64_t)f->port_b;
    for (int pass = 0; pass < 2; pass++) {
        const int nsub = pass ? (int)f->h.n_scale_sub : (int)f->h.nports_w;
        const uint64_t len = pass ? slen : wlen;
        for (int s = 0; s < nsub; s++) {
            const uint8_t *base = f->base + (pass ? f->h.s_sub_offset[s] : f->h.w_sub_offset[s]);
            if (len <= 4096) { h = fnv1a(h, base, len); continue; }
            for (int i = 0; i < 128; i++) {
                const uint64_t off = (len - 32) * (uint64_t)i / 127u;
                h = fnv1a(h, base + off, 32);
            }
        }
    }
    return h;
}

static int cache_get(const mv4i_file *f, int device, const mv4i_dmat **out)
{
    int free_i = -1, lru = 0;
    const uint64_t fp = image_fp(f);
    for (int i = 0; i < CACHE_N; i++) {
        cache_ent *c = &g_cache[i];
        if (c->base == f->base && c->device == device && c->fp == fp && hdr_same(&c->h, &f->h)) {
            c->stamp = ++g_stamp; *out = &c->m; return 0;
        }
        if (c->base == f->base && c->device == device) {     /* same address, new content */
            mv4i_dmat_free(&c->m); memset(c, 0, sizeof *c);
        }
        if (!c->base && free_i < 0) free_i = i;
        if (c->stamp < g_cache[lru].stamp) lru = i;
    }
    const int i = free_i >= 0 ? free_i : lru;
    cache_ent *c = &g_cache[i];
    if (c->base) { mv4i_dmat_free(&c->m); memset(c, 0, sizeof *c); }
    int rc = mv4i_dmat_upload(f, device, &c->m);
    if (rc) return rc;
    c->base = f->base; c->h = f->h; c->fp = fp; c->device = device; c->stamp = ++g_stamp;
    *out = &c->m;
    return 0;
}

int mv4i_forget(const mv4i_file *f)
{
    if (!f) return -11;
    pthread_mutex_lock(&g_lock);
    for (int i = 0; i < CACHE_N; i++)
        if (g_cache[i].base == f->base) { mv4i_dmat_free(&g_cache[i].m); memset(&g_cache[i], 0, sizeof g_cache[i]); }
    pthread_mutex_unlock(&g_lock);
    return 0;
}

static size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

static int ctx_reserve(dev_ctx *c, int device, size_t dbytes, size_t hbytes)
{
    cudaError_t e;
    if (!c->stream) {
        e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) return fail_cuda(e);
        c->device = device;
    }
    if (dbytes > c->cap) {
        if (c->d_buf) cudaFree(c->d_buf);
        c->d_buf = NULL; c->cap = 0;
        e = cudaMalloc(&c->d_buf, dbytes);
        if (e != cudaSuccess) return fail_cuda(e);
        e = cudaMemset(c->d_buf, 0, dbytes);        /* scratch must start zeroed */
        if (e != cudaSuccess) return fail_cuda(e);
        c->cap = dbytes;
    }
    if (hbytes > c->hcap) {
        if (c->h_buf) cudaFreeHost(c->h_buf);
        c->h_buf = NULL; c->hcap = 0;
        e = cudaMallocHost(&c->h_buf, hbytes);
        if (e != cudaSuccess) return fail_cuda(e);
        c->hcap = hbytes;
    }
    return 0;
}

int mv4i_matvec(const mv4i_file *f, const int16_t *x_mant, int x_exp,
                int n_rows, int n_cols, int out_mode, mv4i_result *out)
{
    if (!f || !x_mant || !out) return -11;
    if (n_rows <= 0 || n_cols <= 0) return -1;
    if ((uint32_t)n_cols > f->h.K) return -2;
    if ((uint32_t)n_rows > f->h.M) return -3;
    if (out_mode < 0 || out_mode > 2) return -11;
    if (out_mode == MV4I_MODE_PARTIAL ? !out->y_acc : !out->y_data) return -11;
    if (out_mode == MV4I_MODE_BFP && !out->y_mant) return -11;

    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail_cuda(e);
    if (device < 0 || device >= 16) return -11;

    pthread_mutex_lock(&g_lock);
    int rc;
    const mv4i_dmat *m = NULL;
    rc = cache_get(f, device, &m);
    if (rc) goto done;

    dev_ctx *c = &g_ctx[device];
    const size_t xb = up256((size_t)n_cols * 2);
    const size_t yd = up256((size_t)n_rows * 4), ym = up256((size_t)n_rows * 2), ya = up256((size_t)n_rows * 8);
    const size_t stb = 256, scb = up256(mv4i_scratch_bytes());
    const size_t o_x = 0, o_yd = o_x + xb, o_ym = o_yd + yd, o_ya = o_ym + ym, o_st = o_ya + ya, o_sc = o_st + stb;
    const size_t total = o_sc + scb;
    /* the scratch block sits at the END of the buffer so that growth (which
     * re-zeroes everything) never leaves a non-zero scratch behind */
    rc = ctx_reserve(c, device, total, xb + yd + ym + ya + stb);
    if (rc) goto done;
    uint8_t *d = (uint8_t *)c->d_buf;
    uint8_t *hb = (uint8_t *)c->h_buf;
    /* scratch lives at a fixed offset from the end of the capacity */
    void *scratch = d + c->cap - scb;

    memcpy(hb, x_mant, (size_t)n_cols * 2);
    e = cudaMemcpyAsync(d + o_x, hb, (size_t)n_cols * 2, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) { rc = fail_cuda(e); goto done; }

    mv4i_job j;
    memset(&j, 0, sizeof j);
    j.w = m; j.x = d + o_x; j.x_exp = x_exp;
    j.n_rows = n_rows; j.n_cols = n_cols; j.mode = out_mode; j.nvec = 1;
    j.y_data = (int32_t *)(d + o_yd); j.y_mant = (int16_t *)(d + o_ym); j.y_acc = (int64_t *)(d + o_ya);
    j.status = (mv4i_status *)(d + o_st);
    rc = mv4i_launch(&j, 1, scratch, c->stream);
    if (rc) goto done;

    /* results: one D2H of the whole output block + status */
    e = cudaMemcpyAsync(hb + xb, d + o_yd, o_sc - o_yd, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) { rc = fail_cuda(e); goto done; }
    const uint8_t *hy = hb + xb;
    const mv4i_status *st = (const mv4i_status *)(hy + (o_st - o_yd));
    if (st->err) { rc = st->err; goto done; }
    if (out_mode == MV4I_MODE_PARTIAL) {
        memcpy(out->y_acc, hy + (o_ya - o_yd), (size_t)n_rows * 8);
    } else {
        memcpy(out->y_data, hy, (size_t)n_rows * 4);
        if (out_mode == MV4I_MODE_BFP) memcpy(out->y_mant, hy + (o_ym - o_yd), (size_t)n_rows * 2);
    }
    out->y_exp = st->y_exp;
    out->ns = st->ns;
    out->sat_event = st->sat_event;
    out->sat_count = st->sat_count;
    rc = 0;
done:
    pthread_mutex_unlock(&g_lock);
    return rc;
}

int mv4i_g128_matvec_host(const mv4i_dmat *w, int count, const uint16_t *h_x, uint16_t *h_y,
                          void *stream)
{
    if (!w || count <= 0 || count > MV4I_MAX_JOBS || !h_x || !h_y) return -11;
    const int M = w[0].M, K = w[0].K;
    for (int i = 0; i < count; i++)
        if (w[i].kind != MV4I_KIND_G128 || w[i].M != M || w[i].K != K) return -11;
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail_cuda(e);
    if (device < 0 || device >= 16) return -11;
    pthread_mutex_lock(&g_lock);
    int rc = 0;
    dev_ctx *c = &g_ctx[device];
    const size_t xb = up256((size_t)count * K * 2), yb = up256((size_t)count * M * 2);
    const size_t scb = up256(mv4i_scratch_bytes());
    rc = ctx_reserve(c, device, xb + yb + scb, 0);
    if (rc) goto out;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    uint8_t *d = (uint8_t *)c->d_buf;
    e = cudaMemcpyAsync(d, h_x, (size_t)count * K * 2, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { rc = fail_cuda(e); goto out; }
    mv4i_job jobs[MV4I_MAX_JOBS];
    memset(jobs, 0, sizeof jobs);
    for (int i = 0; i < count; i++) {
        jobs[i].w = &w[i];
        jobs[i].x = d + (size_t)i * K * 2;
        jobs[i].n_rows = M; jobs[i].n_cols = K; jobs[i].nvec = 1;
        jobs[i].y_f16 = (uint16_t *)(d + xb + (size_t)i * M * 2);
    }
    rc = mv4i_launch(jobs, count, NULL, st);
    if (rc) goto out;
    e = cudaMemcpyAsync(h_y, d + xb, (size_t)count * M * 2, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = fail_cuda(e);
out:
    pthread_mutex_unlock(&g_lock);
    return rc;
}

const char *mv4i_version(void) { return "llm.vhdl_b200 mv4i 0.1 (sm_100a)"; }

/* ------------------------------------------- tensor-parallel messages */

size_t mv4i_tp_msg_bytes(int n_rows)
{
    if (n_rows <= 0) return 0;
    return (((size_t)n_rows * 8 + 15) & ~(size_t)15) + sizeof(mv4i_tp_trailer);
}

int mv4i_tp_msg_pack(const int64_t *y_acc, int n_rows, int y_exp, int out_shift, uint32_t seq, void *msg)
{
    if (!y_acc || !msg || n_rows <= 0) return -11;
    uint8_t *m = (uint8_t *)msg;
    memcpy(m, y_acc, (size_t)n_rows * 8);
    volatile mv4i_tp_trailer *t = (volatile mv4i_tp_trailer *)(m + mv4i_tp_msg_bytes(n_rows) - sizeof(mv4i_tp_trailer));
    t->y_exp = y_exp;
    t->out_shift = out_shift;
    t->pad_ = 0;
    __atomic_thread_fence(__ATOMIC_RELEASE);   /* the sequence word is stored last */
    t->seq = seq;
    return 0;
}

int mv4i_tp_msgs_check(int N, int n_rows, const void *const *msgs, uint32_t seq, int32_t *y_exps,
                       int32_t *out_shifts)
{
    if (N <= 0 || N > 64 || n_rows <= 0 || !msgs) return -11;
    const size_t off = mv4i_tp_msg_bytes(n_rows) - sizeof(mv4i_tp_trailer);
    int ymin = 0, ymax = 0, osh0 = 0, rc = 0;
    for (int c = 0; c < N; c++) {
        if (!msgs[c]) return -11;
        const mv4i_tp_trailer *t = (const mv4i_tp_trailer *)((const uint8_t *)msgs[c] + off);
        const uint32_t sq = __atomic_load_n(&t->seq, __ATOMIC_ACQUIRE);
        if (sq != seq) return -15;
        if (y_exps) y_exps[c] = t->y_exp;
        if (out_shifts) out_shifts[c] = t->out_shift;
        if (c == 0) { ymin = ymax = t->y_exp; osh0 = t->out_shift; }
        else {
            ymin = t->y_exp < ymin ? t->y_exp : ymin;
            ymax = t->y_exp > ymax ? t->y_exp : ymax;
            if (t->out_shift != osh0) rc = -13;
        }
    }
    if (!rc && ymax - ymin > 17) rc = -12;
    return rc;
}

