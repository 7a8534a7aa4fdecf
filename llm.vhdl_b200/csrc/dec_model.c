/* llm.vhdl_b200/csrc/dec_model.c -- the decode step built on the hot path.
 *
 * One token through a Qwen3.5-style hybrid decoder, composed the way
 * ref/run9b.c composes its A jobs and its delta rule (layer_gdn :602-756,
 * layer_attn :758-900, lm_head :522-540, argmax_first :399-405), in the
 * floating-point mode: fp16 activations into INT4 g128 projections
 * (mv4i_launch job lists), fp32 residual stream, DeltaNet state and
 * accumulation, fp16 KV cache.  Projections that read the same activation go
 * in one launch; the residual add of a single-GPU run is fused into the output
 * projection (accumulate flag).  Tensor parallel: heads and rows are sharded,
 * the row-parallel outputs are summed with one NCCL all-reduce each, and the
 * vocabulary-sharded argmax keys are all-gathered.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <cuda_runtime_api.h>
#include <nccl.h>
#include "../../include/mv4i_b200.h"
#include "../../include/gdn_b200.h"
#include "../../include/dec_b200.h"
#include "dec_internal.h"

extern int mv4i_g_cuda_err;

/* kernels in dec_kernels.cu (pdl: launch as a programmatic dependent) */
int dec_k_embed(const uint16_t *emb, int hidden, const int32_t *tok, float *x, int nseq, void *s, int pdl);
int dec_k_attention(const float *qg, const float *kv, const float *qn_w, const float *kn_w, int qh, int kvh,
                    int n_rot, float theta, float eps, const int32_t *d_pos, int max_ctx, int ch, float *part,
                    float *q_seam, uint16_t *kcache, uint16_t *vcache, uint16_t *y, int nseq, void *s, int pdl);
int dec_k_add(float *x, const float *t, int n, void *s, int pdl);
int dec_k_advance(unsigned long long *keys, int n, unsigned long long *key, int32_t *tok, int32_t *hist,
                  int32_t *pos, int max_ctx, const int32_t *prompt, int nseq, void *s, int pdl);
size_t dec_p2p_region(int world, int hidden, size_t *off_keys, size_t *off_xflag, size_t *off_kflag);
int dec_k_allreduce_p2p(void *const *regions, int rank, int world, int hidden, const float *t, float *x,
                        uint32_t *epoch, uint32_t *done, int *err, int spin_limit, void *s, int pdl);
int dec_k_advance_p2p(void *const *regions, int rank, int world, int hidden, unsigned long long *key,
                      int32_t *tok, int32_t *hist, int32_t *pos, int max_ctx, const int32_t *prompt,
                      uint32_t *epoch, int *err, int spin_limit, void *s, int pdl);
int dec_k_synth_linear(uint64_t key, const int32_t *rows, int row0, int nrows, int k0, int kn, int Kg,
                       uint8_t *wq, uint16_t *sc, int s_pitch, void *s);
int dec_k_synth_vec(uint64_t key, const int32_t *idx, int64_t idx0, int64_t n, float mean, float std,
                    float *f32, uint16_t *f16, void *s);

#define HD 128
#define MAX_ALLOCS 8192
#define CK(x) do { int rc_ = (x); if (rc_) return rc_; } while (0)

typedef struct {
    mv4i_dmat w;
    uint8_t  *wq;
    uint16_t *sc;
    int32_t   rows, cols, s_pitch;   /* scales [rows][s_pitch], 16-byte rows */
} linear_t;

typedef struct {
    int       attn;
    linear_t  qkv, z, ab, out;            /* DeltaNet */
    linear_t  qg, kv, o;                  /* attention */
    linear_t  gate, up, down;
    float    *attn_norm, *post_norm;
    float    *conv_w, *ssm_a, *dt_bias, *ssm_norm, *conv_state, *rec_state;
    float    *q_norm, *k_norm;
    uint16_t *kcache, *vcache;
} layer_t;

struct dec_model {
    dec_config c;
    int device, rank, world;
    /* local shard sizes */
    int kh, vh, v0, qh, q0, kvh, kv0, ffn, f0, vocab, voc0, conv_dim, conv_g, att_ch, nchunks;
    int32_t  *chan;                      /* host: global conv channel of each local one */
    layer_t  *L;
    linear_t  lm;
    float    *final_norm;
    uint16_t *embed;
    /* activations */
    float    *x, *t, *qkv_f, *z_f, *eg, *beta, *o_f, *qg_f, *kv_f, *q_f, *part, *logits;
    uint16_t *h16, *qkv16, *y16, *ya16, *hf16;
    int       B;                         /* sequences decoded together          */
    int       pdl;                       /* programmatic dependent launches     */
    void    **lev;                       /* optional: event after each layer    */
    int       nlev;
    float    *rseam;                     /* optional: residual at each layer input */
    int       nrseam;
    unsigned long long *key, *keys;
    int32_t  *tok, *pos, *hist;
    int32_t  *prompt;                    /* [0] = length, [1..] = tokens     */
    int       hpos;                      /* host mirror of *pos for direct calls */
    ncclComm_t comm;
    int       comm_ok;
    /* peer-memory exchange (tensor parallel without NCCL on the data path) */
    void     *p2p_region, *p2p_peer[8];
    int       p2p_ok, p2p_open[8], spin_limit;
    uint32_t *ar_epoch, *ar_done, *ak_epoch;
    int      *err;
    int64_t   weight_bytes;
    /* the persistent kernel's program (single GPU) */
    mg_prog   mg;
    int       persistent, mega_ok;
    /* launch mode: inputs staged once per matvec by a launch of their own
     * (0 never, 1 batches of 2+ sequences, 2 always) into xst */
    int       prestage;
    uint8_t  *xst;
    long long xst_bytes;                 /* its capacity: every staging is checked against it */
    int32_t  *layer_clock;               /* [n_layers + 1]: clock index at each layer's end */
    void     *allocs[MAX_ALLOCS];
    int       nalloc;
};

static int fail(cudaError_t e) { mv4i_g_cuda_err = (int)e; return -20; }

static int dalloc(dec_model *m, void **p, size_t bytes)
{
    if (m->nalloc >= MAX_ALLOCS) return -11;
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(e);
    e = cudaMemset(*p, 0, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(e);
    m->allocs[m->nalloc++] = *p;
    return 0;
}

static uint64_t mkey(uint64_t seed, int layer, int id)
{ return seed * 1000003ull + (uint64_t)(layer + 2) * 131ull + (uint64_t)id * 7919ull; }

static int to_device_i32(dec_model *m, int32_t **d, const int32_t *h, size_t n)
{
    CK(dalloc(m, (void **)d, sizeof(int32_t) * n));
    cudaError_t e = cudaMemcpy(*d, h, sizeof(int32_t) * n, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? 0 : fail(e);
}

/* A local g128 shard: rows (map or row0..) of a global [*, Kg] matrix,
 * columns [k0, k0+kn). */
static int make_linear(dec_model *m, linear_t *l, uint64_t key, const int32_t *h_rows, int row0, int nrows,
                       int k0, int kn, int Kg)
{
    l->rows = nrows; l->cols = kn; l->s_pitch = ((kn / 128) + 7) & ~7;
    CK(dalloc(m, (void **)&l->wq, (size_t)nrows * kn / 2));
    CK(dalloc(m, (void **)&l->sc, (size_t)nrows * l->s_pitch * 2));
    int32_t *d_rows = NULL;
    if (h_rows) CK(to_device_i32(m, &d_rows, h_rows, (size_t)nrows));
    CK(dec_k_synth_linear(key, d_rows, row0, nrows, k0, kn, Kg, l->wq, l->sc, l->s_pitch, NULL));
    CK(mv4i_dmat_wrap_g128(l->wq, kn / 2, l->sc, l->s_pitch, nrows, kn, m->device, &l->w));
    m->weight_bytes += (int64_t)nrows * kn / 2 + (int64_t)nrows * (kn / 128) * 2;   /* bytes read */
    return 0;
}

static int make_vec(dec_model *m, float **p, uint64_t key, const int32_t *h_idx, int64_t idx0, int64_t n,
                    float mean, float std)
{
    CK(dalloc(m, (void **)p, sizeof(float) * (size_t)n));
    int32_t *d_idx = NULL;
    if (h_idx) CK(to_device_i32(m, &d_idx, h_idx, (size_t)n));
    return dec_k_synth_vec(key, d_idx, idx0, n, mean, std, *p, NULL, NULL);
}

static int mega_build(dec_model *m);

static int is_attn(const dec_config *c, int il) { return ((il + 1) % c->attn_every) == 0; }

int dec_create(const dec_config *cfg, uint64_t seed, int device, int tp_rank, int tp_world, dec_model **out)
{
    if (!cfg || !out || tp_world < 1 || tp_rank < 0 || tp_rank >= tp_world) return -11;
    const dec_config *c = cfg;
    if (c->gdn_hd != HD || c->att_hd != HD || c->hidden % 128 || c->hidden > 16384 || c->ffn % (128 * tp_world)
        || c->gdn_vh % tp_world || c->att_qh % tp_world || c->att_kvh % tp_world || c->att_kvh <= 0
        || (c->att_qh / c->att_kvh) > 32 || c->att_qh % c->att_kvh || c->attn_every < 1
        || c->n_rot > HD || (c->n_rot & 1) || c->max_ctx <= 0 || c->max_ctx > 65536 || c->vocab < tp_world
        || c->batch < 0 || c->batch > 8 || (c->batch > 1 && tp_world > 1))
        return -11;
    dec_model *m = (dec_model *)calloc(1, sizeof *m);
    if (!m) return -11;
    m->c = *c; m->device = device; m->rank = tp_rank; m->world = tp_world;
    m->B = c->batch > 1 ? c->batch : 1;
    m->c.batch = m->B;
    { const char *e = getenv("DEC_PDL"); m->pdl = !(e && e[0] == '0'); }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) { free(m); return fail(e); }
    const int W = tp_world, R = tp_rank;
    m->vh = c->gdn_vh / W; m->v0 = R * m->vh;
    m->kh = c->gdn_kh < m->vh ? c->gdn_kh : m->vh;
    m->qh = c->att_qh / W; m->q0 = R * m->qh;
    m->kvh = c->att_kvh / W; m->kv0 = R * m->kvh;
    m->ffn = c->ffn / W; m->f0 = R * m->ffn;
    m->vocab = c->vocab / W + (R < c->vocab % W ? 1 : 0);
    m->voc0 = R * (c->vocab / W) + (R < c->vocab % W ? R : c->vocab % W);
    m->conv_dim = 2 * m->kh * HD + m->vh * HD;
    /* positions per attention CTA: short caches of one sequence in chunks of
     * 16 (more CTAs on a step that is a latency chain), then 32, then 64 */
    m->att_ch = (c->max_ctx <= 2048 && m->B == 1) ? 16 : (c->max_ctx <= 6144 ? 32 : 64);
    m->nchunks = (c->max_ctx + m->att_ch - 1) / m->att_ch;
    m->L = (layer_t *)calloc((size_t)c->n_layers, sizeof(layer_t));
    const int H = c->hidden, KHg = c->gdn_kh, VHg = c->gdn_vh;
    const int conv_g = 2 * KHg * HD + VHg * HD;
    m->conv_g = conv_g;
    int rc = 0;
    int32_t *rows = (int32_t *)malloc(sizeof(int32_t) * (size_t)(2 * c->att_qh * HD + conv_g + 2 * VHg + 8));
    int32_t *cidx = (int32_t *)malloc(sizeof(int32_t) * (size_t)conv_g * 4);
#define TRY(x) do { rc = (x); if (rc) goto bad; } while (0)
    for (int il = 0; il < c->n_layers; il++) {
        layer_t *l = &m->L[il];
        l->attn = is_attn(c, il);
        TRY(make_vec(m, &l->attn_norm, mkey(seed, il, 1), NULL, 0, H, 1.0f, 0.1f));
        TRY(make_vec(m, &l->post_norm, mkey(seed, il, 2), NULL, 0, H, 1.0f, 0.1f));
        if (!l->attn) {
            int n = 0;
            for (int i = 0; i < m->kh; i++) {            /* local key head i = global (v0 + i) % KH */
                const int g = (m->v0 + i) % KHg;
                for (int d = 0; d < HD; d++) rows[n++] = g * HD + d;
            }
            for (int i = 0; i < m->kh; i++) {
                const int g = (m->v0 + i) % KHg;
                for (int d = 0; d < HD; d++) rows[n++] = KHg * HD + g * HD + d;
            }
            for (int i = 0; i < m->vh; i++)
                for (int d = 0; d < HD; d++) rows[n++] = 2 * KHg * HD + (m->v0 + i) * HD + d;
            TRY(make_linear(m, &l->qkv, mkey(seed, il, 10), rows, 0, n, 0, H, H));
            if (!m->chan) {
                m->chan = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
                if (!m->chan) { rc = -11; goto bad; }
                memcpy(m->chan, rows, sizeof(int32_t) * (size_t)n);
            }
            for (int i = 0; i < n; i++) for (int t = 0; t < 4; t++) cidx[4 * i + t] = rows[i] * 4 + t;
            TRY(make_vec(m, &l->conv_w, mkey(seed, il, 3), cidx, 0, (int64_t)n * 4, 0.0f, 0.5f));
            TRY(make_linear(m, &l->z, mkey(seed, il, 11), NULL, m->v0 * HD, m->vh * HD, 0, H, H));
            n = 0;
            for (int i = 0; i < m->vh; i++) rows[n++] = m->v0 + i;
            for (int i = 0; i < m->vh; i++) rows[n++] = VHg + m->v0 + i;
            TRY(make_linear(m, &l->ab, mkey(seed, il, 12), rows, 0, n, 0, H, H));
            TRY(make_linear(m, &l->out, mkey(seed, il, 13), NULL, 0, H, m->v0 * HD, m->vh * HD, VHg * HD));
            TRY(make_vec(m, &l->ssm_a, mkey(seed, il, 4), NULL, m->v0, m->vh, -1.0f, 0.2f));
            TRY(make_vec(m, &l->dt_bias, mkey(seed, il, 5), NULL, m->v0, m->vh, 0.0f, 0.5f));
            TRY(make_vec(m, &l->ssm_norm, mkey(seed, il, 6), NULL, 0, HD, 1.0f, 0.1f));
            TRY(dalloc(m, (void **)&l->conv_state, sizeof(float) * 3 * (size_t)m->conv_dim * m->B));
            TRY(dalloc(m, (void **)&l->rec_state, sizeof(float) * (size_t)m->vh * HD * HD * m->B));
        } else {
            int n = 0;
            for (int i = 0; i < m->qh; i++)
                for (int j = 0; j < 2 * HD; j++) rows[n++] = (m->q0 + i) * 2 * HD + j;
            TRY(make_linear(m, &l->qg, mkey(seed, il, 20), rows, 0, n, 0, H, H));
            n = 0;
            for (int i = 0; i < m->kvh; i++) for (int d = 0; d < HD; d++) rows[n++] = (m->kv0 + i) * HD + d;
            for (int i = 0; i < m->kvh; i++)
                for (int d = 0; d < HD; d++) rows[n++] = c->att_kvh * HD + (m->kv0 + i) * HD + d;
            TRY(make_linear(m, &l->kv, mkey(seed, il, 21), rows, 0, n, 0, H, H));
            TRY(make_linear(m, &l->o, mkey(seed, il, 22), NULL, 0, H, m->q0 * HD, m->qh * HD, c->att_qh * HD));
            TRY(make_vec(m, &l->q_norm, mkey(seed, il, 7), NULL, 0, HD, 1.0f, 0.1f));
            TRY(make_vec(m, &l->k_norm, mkey(seed, il, 8), NULL, 0, HD, 1.0f, 0.1f));
            TRY(dalloc(m, (void **)&l->kcache, 2 * (size_t)c->max_ctx * m->kvh * HD * m->B));
            TRY(dalloc(m, (void **)&l->vcache, 2 * (size_t)c->max_ctx * m->kvh * HD * m->B));
        }
        TRY(make_linear(m, &l->gate, mkey(seed, il, 30), NULL, m->f0, m->ffn, 0, H, H));
        TRY(make_linear(m, &l->up, mkey(seed, il, 31), NULL, m->f0, m->ffn, 0, H, H));
        TRY(make_linear(m, &l->down, mkey(seed, il, 32), NULL, 0, H, m->f0, m->ffn, c->ffn));
    }
    TRY(make_linear(m, &m->lm, mkey(seed, -1, 40), NULL, m->voc0, m->vocab, 0, H, H));
    TRY(make_vec(m, &m->final_norm, mkey(seed, -1, 9), NULL, 0, H, 1.0f, 0.1f));
    TRY(dalloc(m, (void **)&m->embed, 2 * (size_t)c->vocab * H));
    TRY(dec_k_synth_vec(mkey(seed, -1, 41), NULL, 0, (int64_t)c->vocab * H, 0.0f, 1.0f, NULL, m->embed, NULL));
    /* activations, [batch][...] */
    const int mx = H > m->ffn ? H : m->ffn;
    const size_t B = (size_t)m->B;
    TRY(dalloc(m, (void **)&m->x, 4 * (size_t)H * B));
    TRY(dalloc(m, (void **)&m->t, 4 * (size_t)H * B));
    TRY(dalloc(m, (void **)&m->h16, 2 * (size_t)mx * B));
    TRY(dalloc(m, (void **)&m->qkv_f, 4 * (size_t)m->conv_dim * B));
    TRY(dalloc(m, (void **)&m->qkv16, 2 * (size_t)m->conv_dim * B));
    TRY(dalloc(m, (void **)&m->z_f, 4 * (size_t)m->vh * HD * B));
    TRY(dalloc(m, (void **)&m->eg, 4 * (size_t)m->vh * B));
    TRY(dalloc(m, (void **)&m->beta, 4 * (size_t)m->vh * B));
    TRY(dalloc(m, (void **)&m->o_f, 4 * (size_t)m->vh * HD * B));
    TRY(dalloc(m, (void **)&m->y16, 2 * (size_t)m->vh * HD * B));
    TRY(dalloc(m, (void **)&m->qg_f, 4 * 2 * (size_t)m->qh * HD * B));
    TRY(dalloc(m, (void **)&m->kv_f, 4 * 2 * (size_t)m->kvh * HD * B));
    TRY(dalloc(m, (void **)&m->q_f, 4 * (size_t)m->qh * HD * B));
    TRY(dalloc(m, (void **)&m->part, 4 * (size_t)m->qh * m->nchunks * (HD + 4) * B));
    TRY(dalloc(m, (void **)&m->ya16, 2 * (size_t)m->qh * HD * B));
    TRY(dalloc(m, (void **)&m->hf16, 2 * (size_t)m->ffn * B));
    TRY(dalloc(m, (void **)&m->logits, 4 * (size_t)m->vocab * B));
    TRY(dalloc(m, (void **)&m->key, 8 * B));
    TRY(dalloc(m, (void **)&m->keys, 8 * (size_t)W * B));
    TRY(dalloc(m, (void **)&m->tok, 4 * B));
    TRY(dalloc(m, (void **)&m->pos, 4));
    TRY(dalloc(m, (void **)&m->hist, 4 * (size_t)c->max_ctx * B));
    TRY(dalloc(m, (void **)&m->ar_epoch, 16));
    TRY(dalloc(m, (void **)&m->ar_done, 16));
    TRY(dalloc(m, (void **)&m->ak_epoch, 16));
    TRY(dalloc(m, (void **)&m->err, 16));
    TRY(dalloc(m, (void **)&m->prompt, 4 * ((size_t)c->max_ctx * B + 1)));
    {
        /* the staged inputs of the widest matvec input */
        int kx = mx;
        if (m->vh * HD > kx) kx = m->vh * HD;
        if (m->qh * HD > kx) kx = m->qh * HD;
        const long long xb = dec_k_stage_bytes(kx, m->B);
        if (xb < 0) { rc = -11; goto bad; }
        TRY(dalloc(m, (void **)&m->xst, (size_t)xb));
        m->xst_bytes = xb;
        const char *ps = getenv("DEC_PRESTAGE");
        m->prestage = ps && ps[0] >= '0' && ps[0] <= '2' ? ps[0] - '0' : 1;
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { rc = fail(e); goto bad; }
    m->layer_clock = (int32_t *)calloc((size_t)c->n_layers + 1, sizeof(int32_t));
    if (!m->layer_clock) { rc = -11; goto bad; }
    if (W == 1) {
        const char *pe = getenv("DEC_PERSISTENT");
        m->persistent = pe && pe[0] == '1';
        if (m->persistent) TRY(mega_build(m));
    }
    free(rows); free(cidx);
    *out = m;
    return 0;
bad:
    free(rows); free(cidx);
    dec_destroy(m);
    return rc;
#undef TRY
}

int dec_destroy(dec_model *m)
{
    if (!m) return -11;
    cudaSetDevice(m->device);
    if (m->comm_ok) ncclCommDestroy(m->comm);
    for (int r = 0; r < 8; r++) if (m->p2p_open[r]) cudaIpcCloseMemHandle(m->p2p_peer[r]);
    for (int i = 0; i < m->nalloc; i++) cudaFree(m->allocs[i]);
    if (m->mg.d_prog) cudaFree(m->mg.d_prog);
    if (m->mg.ctl) cudaFree(m->mg.ctl);
    free(m->layer_clock);
    free(m->chan);
    free(m->L);
    free(m);
    return 0;
}

int dec_nccl_unique_id(uint8_t id[128])
{
    ncclUniqueId u;
    if (ncclGetUniqueId(&u) != ncclSuccess) return -20;
    memcpy(id, &u, 128);
    return 0;
}

int dec_tp_init(dec_model *m, const uint8_t id[128])
{
    if (!m) return -11;
    if (m->world == 1) return 0;
    ncclUniqueId u;
    memcpy(&u, id, 128);
    cudaSetDevice(m->device);
    if (ncclCommInitRank(&m->comm, m->world, u, m->rank) != ncclSuccess) return -20;
    m->comm_ok = 1;
    return 0;
}

int dec_p2p_handle(dec_model *m, uint8_t handle[64])
{
    if (!m || !handle || m->world < 2 || m->world > 8) return -11;
    cudaError_t e = cudaSetDevice(m->device);
    if (e != cudaSuccess) return fail(e);
    if (!m->p2p_region) {
        const size_t bytes = dec_p2p_region(m->world, m->c.hidden, NULL, NULL, NULL);
        CK(dalloc(m, &m->p2p_region, bytes));
    }
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, m->p2p_region);
    if (e != cudaSuccess) return fail(e);
    memcpy(handle, &h, 64);
    return 0;
}

int dec_p2p_open(dec_model *m, const uint8_t *handles, int spin_limit)
{
    if (!m || !handles || !m->p2p_region) return -11;
    cudaError_t e = cudaSetDevice(m->device);
    if (e != cudaSuccess) return fail(e);
    for (int r = 0; r < m->world; r++) {
        if (r == m->rank) { m->p2p_peer[r] = m->p2p_region; continue; }
        if (m->p2p_open[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + 64 * (size_t)r, 64);
        e = cudaIpcOpenMemHandle(&m->p2p_peer[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(e);
        m->p2p_open[r] = 1;
    }
    m->spin_limit = spin_limit > 0 ? spin_limit : (1 << 22);
    m->p2p_ok = 1;
    return 0;
}

int dec_status(dec_model *m, int32_t *flags)
{
    if (!m || !flags) return -11;
    int v = 0;
    cudaError_t e = cudaSetDevice(m->device);
    if (e == cudaSuccess) e = cudaMemcpy(&v, m->err, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(m->err, 0, 4);
    if (e == cudaSuccess && m->mg.ctl) {
        mg_ctl ctl;
        e = cudaMemcpy(&ctl, m->mg.ctl, sizeof ctl, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && ctl.abort) {
            v |= 4;
            e = cudaMemset(m->mg.ctl, 0, sizeof ctl);
        }
    }
    if (e != cudaSuccess) return fail(e);
    *flags = v;
    return 0;
}

/* Sequence b of a batch draws from seed ^ (b * golden ratio): sequence 0
 * is the unbatched model's. */
static uint64_t seq_seed(uint64_t seed, int b) { return seed ^ ((uint64_t)b * 0x9E3779B97F4A7C15ull); }

int dec_prefill_random(dec_model *m, int len, uint64_t seed)
{
    if (!m || len < 0 || len >= m->c.max_ctx) return -11;
    cudaSetDevice(m->device);
    const size_t cache_seq = (size_t)m->c.max_ctx * m->kvh * HD;
    /* draw indices: cache [pos][kvh][hd] by (pos, global kv head, d); conv
     * state [3][conv_dim] by (tap, global channel) */
    const int64_t n_kv = (int64_t)len * m->kvh * HD, n_cv = 3 * (int64_t)m->conv_dim;
    const int64_t n_idx = n_kv > n_cv ? n_kv : n_cv;
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)(n_idx > 0 ? n_idx : 1));
    int32_t *d_kv = NULL, *d_cv = NULL;
    int rc = idx ? 0 : -11;
    cudaError_t e = cudaSuccess;
    if (!rc && n_kv > 0) {
        for (int64_t i = 0; i < n_kv; i++) {
            const int64_t p = i / (m->kvh * HD), r = i % (m->kvh * HD);
            idx[i] = (int32_t)((p * m->c.att_kvh + m->kv0 + r / HD) * HD + r % HD);
        }
        e = cudaMalloc((void **)&d_kv, sizeof(int32_t) * (size_t)n_kv);
        if (e == cudaSuccess) e = cudaMemcpy(d_kv, idx, sizeof(int32_t) * (size_t)n_kv, cudaMemcpyHostToDevice);
    }
    if (!rc && e == cudaSuccess && m->chan) {
        for (int64_t i = 0; i < n_cv; i++)
            idx[i] = (int32_t)((i / m->conv_dim) * m->conv_g + m->chan[i % m->conv_dim]);
        e = cudaMalloc((void **)&d_cv, sizeof(int32_t) * (size_t)n_cv);
        if (e == cudaSuccess) e = cudaMemcpy(d_cv, idx, sizeof(int32_t) * (size_t)n_cv, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) rc = fail(e);
    for (int b = 0; b < m->B && !rc; b++) {
        const uint64_t sb = seq_seed(seed, b);
        for (int il = 0; il < m->c.n_layers && !rc; il++) {
            layer_t *l = &m->L[il];
            if (l->attn) {
                if (n_kv == 0) continue;
                rc = dec_k_synth_vec(mkey(sb, il, 50), d_kv, 0, n_kv, 0.f, 1.f, NULL, l->kcache + b * cache_seq, NULL);
                if (!rc) rc = dec_k_synth_vec(mkey(sb, il, 51), d_kv, 0, n_kv, 0.f, 1.f, NULL, l->vcache + b * cache_seq, NULL);
            } else {
                const int64_t ns = (int64_t)m->vh * HD * HD;
                rc = dec_k_synth_vec(mkey(sb, il, 52), NULL, (int64_t)m->v0 * HD * HD, ns, 0.f, 0.02f,
                                     l->rec_state + b * ns, NULL, NULL);
                if (!rc) rc = dec_k_synth_vec(mkey(sb, il, 53), d_cv, 0, n_cv, 0.f, 0.5f, l->conv_state + b * n_cv,
                                              NULL, NULL);
            }
        }
    }
    e = cudaDeviceSynchronize();
    if (d_kv) cudaFree(d_kv);
    if (d_cv) cudaFree(d_cv);
    free(idx);
    if (rc) return rc;
    if (e == cudaSuccess) e = cudaMemcpy(m->pos, &len, 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(e);
    m->hpos = len;
    return 0;
}

int dec_set(dec_model *m, int pos, int token)
{
    if (!m || pos < 0 || pos >= m->c.max_ctx || token < 0 || token >= m->c.vocab) return -11;
    const int32_t zero = 0;
    int32_t toks[8];
    for (int b = 0; b < m->B; b++) toks[b] = token;
    cudaError_t e = cudaMemcpy(m->pos, &pos, 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->tok, toks, 4 * (size_t)m->B, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->prompt, &zero, 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(e);
    m->hpos = pos;
    return 0;
}

int dec_set_prompt(dec_model *m, const int32_t *tokens, int n, void *stream)
{
    if (!m || !tokens || n < 1 || n > m->c.max_ctx) return -11;
    for (int64_t i = 0; i < (int64_t)n * m->B; i++) if (tokens[i] < 0 || tokens[i] >= m->c.vocab) return -11;
    const cudaStream_t s = (cudaStream_t)stream;
    const int32_t zero = 0;
    cudaError_t e = cudaSuccess;
    for (int il = 0; il < m->c.n_layers && e == cudaSuccess; il++) {     /* new sequences */
        layer_t *l = &m->L[il];
        if (l->attn) continue;
        e = cudaMemsetAsync(l->conv_state, 0, sizeof(float) * 3 * (size_t)m->conv_dim * m->B, s);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(l->rec_state, 0, sizeof(float) * (size_t)m->vh * HD * HD * m->B, s);
    }
    int32_t first[8];
    for (int b = 0; b < m->B; b++) first[b] = tokens[(size_t)b * n];
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->prompt, &n, 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->prompt + 1, tokens, 4 * (size_t)n * m->B, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->tok, first, 4 * (size_t)m->B, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, &zero, 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(e);
    m->hpos = 0;
    return 0;
}

#define PF_BYTES (48 * 1024)       /* weight bytes a matvec CTA asks L2 for early, per 8 warps */

/* The step as a program.  dec_program walks the layers once and hands each
 * piece of work to an emitter: in launch mode (rec == NULL) every piece is a
 * kernel launch on the stream (programmatic dependents of one another); in
 * record mode it becomes a stage of the persistent kernel's program, with a
 * grid barrier after every stage whose output a later one reads. */
typedef struct {
    dec_model *m;
    void      *s;
    int        pdl;
    mg_stage  *rec;
    int        n, cap, nbar;
} emit_t;

static mg_stage *em_new(emit_t *E, int op, int sync)
{
    if (E->n == E->cap) {
        const int cap = E->cap ? 2 * E->cap : 256;
        mg_stage *r = (mg_stage *)realloc(E->rec, sizeof(mg_stage) * (size_t)cap);
        if (!r) return NULL;
        E->rec = r; E->cap = cap;
    }
    mg_stage *st = &E->rec[E->n++];
    memset(st, 0, sizeof *st);
    st->op = op; st->sync = sync; st->pf = -1;
    E->nbar += sync ? 1 : 0;
    return st;
}

static int em_matvec(emit_t *E, const dmv_params *P)
{
    dec_model *m = E->m;
    if (!E->rec && m->xst && (m->prestage == 2 || (m->prestage == 1 && m->B > 1))) {
        /* every CTA of the matvec would stage all the batch's vectors: stage
         * them once, the matvec's CTAs copy the blocks */
        dmv_params Q = *P;
        const long long need = dec_k_stage_bytes(P->K, P->nvec > 0 ? P->nvec : 1);
        if (need < 0 || need > m->xst_bytes) return -11;     /* an input wider than the staging block */
        Q.xst = m->xst;
        CK(dec_k_stage(&Q, E->s, E->pdl));
        return dec_k_matvec(&Q, E->s, E->pdl);
    }
    if (!E->rec) return dec_k_matvec(P, E->s, E->pdl);
    mg_stage *st = em_new(E, MG_MATVEC, 1);
    if (!st) return -11;
    st->u.mv = *P;
    return 0;
}

static int em_copy(emit_t *E, float *dst, const float *src, int64_t n)
{
    if (!E->rec)
        return cudaMemcpyAsync(dst, src, sizeof(float) * (size_t)n, cudaMemcpyDeviceToDevice, (cudaStream_t)E->s)
               == cudaSuccess ? 0 : -20;
    /* no barrier: the stage after it reads the residual but does not write it */
    mg_stage *st = em_new(E, MG_COPY, 0);
    if (!st) return -11;
    st->u.cp.dst = dst; st->u.cp.src = src; st->u.cp.n = n;
    return 0;
}

/* inputs [batch][K] */
static void mvparams(dec_model *m, dmv_params *P, int K, int op, const void *x, const float *nw, float eps,
                     uint16_t *seam)
{
    memset(P, 0, sizeof *P);
    P->K = K; P->op = op; P->x = x; P->nw = nw; P->eps = eps; P->seam = seam; P->pf_bytes = PF_BYTES;
    P->nvec = m->B; P->xs = K;
}

/* outputs [batch][rows] */
static void mvjob(dmv_job *J, const linear_t *l, int epi)
{
    memset(J, 0, sizeof *J);
    J->wq = l->wq; J->sc = l->sc; J->rows = l->rows; J->epi = epi; J->s_pitch = l->s_pitch;
    J->ostride = l->rows;
}

/* row-parallel block: a single GPU adds into the residual in the matvec
 * epilogue; tensor parallel sums the partials with one NCCL all-reduce */
static int row_parallel(emit_t *E, dmv_params *P, const linear_t *l)
{
    dec_model *m = E->m;
    void *s = E->s;
    mvjob(&P->jobs[0], l, m->world == 1 ? DMV_EPI_ACC : DMV_EPI_F32);
    P->jobs[0].out_f32 = m->world == 1 ? m->x : m->t;
    P->jobs[0].ostride = m->c.hidden;
    P->njobs = 1;
    CK(em_matvec(E, P));
    if (m->world == 1) return 0;
    if (E->rec) return -11;                       /* tensor parallel runs in launch mode */
    if (m->p2p_ok)
        return dec_k_allreduce_p2p(m->p2p_peer, m->rank, m->world, m->c.hidden, m->t, m->x, m->ar_epoch,
                                   m->ar_done, m->err, m->spin_limit, s, E->pdl);
    if (ncclAllReduce(m->t, m->t, (size_t)m->c.hidden, ncclFloat32, ncclSum, m->comm, (cudaStream_t)s)
        != ncclSuccess) return -20;
    return dec_k_add(m->x, m->t, m->c.hidden, s, E->pdl);
}

static int dec_program(dec_model *m, emit_t *E)
{
    const dec_config *c = &m->c;
    const int H = c->hidden;
    void *s = E->s;
    const int pdl = E->pdl;
    dmv_params P;
    if (E->rec) {
        mg_stage *st = em_new(E, MG_EMBED, 1);
        if (!st) return -11;
        st->u.emb.emb = m->embed; st->u.emb.tok = m->tok; st->u.emb.x = m->x;
        st->u.emb.hidden = H; st->u.emb.nseq = m->B;
    } else {
        CK(dec_k_embed(m->embed, H, m->tok, m->x, m->B, s, pdl));
    }
    const size_t xn = (size_t)H * m->B;
    for (int il = 0; il < c->n_layers; il++) {
        layer_t *l = &m->L[il];
        if (m->rseam && il < m->nrseam) CK(em_copy(E, m->rseam + il * xn, m->x, (int64_t)xn));
        mvparams(m, &P, H, DMV_OP_RMSNORM, m->x, l->attn_norm, c->rms_eps, m->h16);
        if (!l->attn) {
            /* q|k|v with the conv + SiLU epilogue, z, and a|b with the gates */
            mvjob(&P.jobs[0], &l->qkv, DMV_EPI_CONV);
            P.jobs[0].out_f16 = m->qkv16; P.jobs[0].out_f32 = m->qkv_f;
            P.jobs[0].p0 = l->conv_w; P.jobs[0].st = l->conv_state; P.jobs[0].st_stride = m->conv_dim;
            mvjob(&P.jobs[1], &l->z, DMV_EPI_F32);
            P.jobs[1].out_f32 = m->z_f;
            mvjob(&P.jobs[2], &l->ab, DMV_EPI_GATES);
            P.jobs[2].out_f32 = m->eg; P.jobs[2].out2_f32 = m->beta;
            P.jobs[2].p0 = l->ssm_a; P.jobs[2].p1 = l->dt_bias; P.jobs[2].n1 = m->vh; P.jobs[2].ostride = m->vh;
            P.njobs = 3;
            CK(em_matvec(E, &P));
            gdn_f32_args g;
            memset(&g, 0, sizeof g);
            g.T = 1; g.H = m->vh; g.KH = m->kh; g.D = HD; g.S = l->rec_state;
            g.q = m->qkv16; g.k = m->qkv16 + (size_t)m->kh * HD; g.v = m->qkv16 + (size_t)2 * m->kh * HD;
            g.g = NULL; g.eg = m->eg; g.beta = m->beta; g.l2norm = 1; g.q_scale = 1.0f / sqrtf((float)HD);
            g.out_f32 = m->o_f; g.pdl = pdl;
            g.nseq = m->B; g.seq_in = m->conv_dim;
            if (E->rec) {
                mg_stage *st = em_new(E, MG_GDN, 1);
                if (!st) return -11;
                st->u.gdn = g;
            } else {
                CK(gdn_run_f32(&g, s));
            }
            /* output norm and z gate folded into the out projection */
            mvparams(m, &P, m->vh * HD, DMV_OP_GATED, m->o_f, l->ssm_norm, c->rms_eps, m->y16);
            P.x2 = m->z_f;
            CK(row_parallel(E, &P, &l->out));
        } else {
            mvjob(&P.jobs[0], &l->qg, DMV_EPI_F32);
            P.jobs[0].out_f32 = m->qg_f;
            mvjob(&P.jobs[1], &l->kv, DMV_EPI_F32);
            P.jobs[1].out_f32 = m->kv_f;
            P.njobs = 2;
            CK(em_matvec(E, &P));
            /* q/k norm, RoPE and the cache write folded into flash decoding */
            if (E->rec) {
                dec_attn_args A = {m->qg_f, m->kv_f, l->q_norm, l->k_norm, m->qh, m->kvh, c->n_rot, c->rope_theta,
                                   c->rms_eps, m->pos, c->max_ctx, m->att_ch, 0, l->kcache, l->vcache, m->q_f,
                                   m->part, m->ya16, m->B};
                mg_stage *st = em_new(E, MG_ATTN, 1);
                if (!st) return -11;
                st->u.att = A;
                st = em_new(E, MG_COMBINE, 1);
                if (!st) return -11;
                st->u.att = A;
            } else {
                CK(dec_k_attention(m->qg_f, m->kv_f, l->q_norm, l->k_norm, m->qh, m->kvh, c->n_rot, c->rope_theta,
                                   c->rms_eps, m->pos, c->max_ctx, m->att_ch, m->part, m->q_f, l->kcache,
                                   l->vcache, m->ya16, m->B, s, pdl));
            }
            mvparams(m, &P, m->qh * HD, DMV_OP_F16, m->ya16, NULL, 0.f, NULL);
            CK(row_parallel(E, &P, &l->o));
        }
        /* SwiGLU: gate and up rows paired in one warp, silu(g)*u in the epilogue */
        mvparams(m, &P, H, DMV_OP_RMSNORM, m->x, l->post_norm, c->rms_eps, m->h16);
        mvjob(&P.jobs[0], &l->gate, DMV_EPI_SWIGLU);
        P.jobs[0].wq2 = l->up.wq; P.jobs[0].sc2 = l->up.sc; P.jobs[0].out_f16 = m->hf16;
        P.njobs = 1;
        CK(em_matvec(E, &P));
        mvparams(m, &P, m->ffn, DMV_OP_F16, m->hf16, NULL, 0.f, NULL);
        CK(row_parallel(E, &P, &l->down));
        if (E->rec) m->layer_clock[il] = E->nbar;
        else if (m->lev && il < m->nlev && cudaEventRecord((cudaEvent_t)m->lev[il], (cudaStream_t)s) != cudaSuccess)
            return -20;
    }
    if (m->rseam && c->n_layers < m->nrseam) CK(em_copy(E, m->rseam + c->n_layers * xn, m->x, (int64_t)xn));
    /* LM head with the first-max argmax key in its epilogue */
    mvparams(m, &P, H, DMV_OP_RMSNORM, m->x, m->final_norm, c->rms_eps, m->h16);
    mvjob(&P.jobs[0], &m->lm, DMV_EPI_ARGMAX);
    P.jobs[0].out_f32 = m->logits;
    P.key = m->key; P.idx0 = m->voc0; P.njobs = 1;
    CK(em_matvec(E, &P));
    if (E->rec) {
        if (m->world > 1) return -11;
        m->layer_clock[c->n_layers] = E->nbar;
        mg_stage *st = em_new(E, MG_ADVANCE, 0);
        if (!st) return -11;
        st->u.adv.keys = m->key; st->u.adv.key = m->key; st->u.adv.tok = m->tok; st->u.adv.hist = m->hist;
        st->u.adv.pos = m->pos; st->u.adv.prompt = m->prompt; st->u.adv.n = 1; st->u.adv.nseq = m->B;
        st->u.adv.max_ctx = c->max_ctx;
        return 0;
    }
    if (m->world > 1 && m->p2p_ok)
        return dec_k_advance_p2p(m->p2p_peer, m->rank, m->world, H, m->key, m->tok, m->hist, m->pos, c->max_ctx,
                                 m->prompt, m->ak_epoch, m->err, m->spin_limit, s, pdl);
    if (m->world > 1) {
        if (ncclAllGather(m->key, m->keys, 1, ncclUint64, m->comm, (cudaStream_t)s) != ncclSuccess) return -20;
        return dec_k_advance(m->keys, m->world, m->key, m->tok, m->hist, m->pos, c->max_ctx, m->prompt, 1, s, pdl);
    }
    return dec_k_advance(m->key, 1, m->key, m->tok, m->hist, m->pos, c->max_ctx, m->prompt, m->B, s, pdl);
}

/* records the step and uploads it for the persistent kernel (single GPU) */
static int mega_build(dec_model *m)
{
    if (m->world != 1) return 0;
    emit_t E;
    memset(&E, 0, sizeof E);
    E.m = m;
    E.rec = (mg_stage *)malloc(sizeof(mg_stage) * 256);      /* rec != NULL: record mode */
    if (!E.rec) return -11;
    E.cap = 256;
    int rc = dec_program(m, &E);
    if (!rc) {
        if (m->mg.d_prog && m->mg.n != E.n) {
            cudaFree(m->mg.d_prog);
            m->mg.d_prog = NULL;
        }
        rc = dec_mega_upload(E.rec, E.n, m->B, &m->mg);
    }
    free(E.rec);
    m->mega_ok = rc == 0;
    return rc;
}

int dec_step(dec_model *m, void *s)
{
    if (!m) return -11;
    if (m->world > 1 && !m->comm_ok && !m->p2p_ok) return -11;
    if (m->hpos >= m->c.max_ctx) return -11;   /* the KV cache is full */
    m->hpos++;
    if (m->persistent && m->mega_ok) return dec_k_mega(&m->mg, s);
    emit_t E;
    memset(&E, 0, sizeof E);
    E.m = m; E.s = s; E.pdl = m->pdl && s != NULL;   /* not on the legacy default stream */
    return dec_program(m, &E);
}

int dec_set_persistent(dec_model *m, int on)
{
    if (!m) return -11;
    if (on && m->world != 1) return -11;
    m->persistent = on != 0;
    if (m->persistent && !m->mega_ok) CK(mega_build(m));
    return 0;
}

int dec_set_prestage(dec_model *m, int mode)
{
    if (!m || mode < 0 || mode > 2) return -11;
    m->prestage = mode;
    return 0;
}

int dec_persistent(dec_model *m)
{
    return m ? (m->persistent && m->mega_ok) : -11;
}

int dec_set_wait_limit(dec_model *m, int64_t ns)
{
    if (!m || ns < 0) return -11;
    m->mg.timeout_ns = ns > 0 ? ns : 1000000000LL;
    return 0;
}

int dec_set_clock(dec_model *m, uint64_t *d_clock)
{
    if (!m) return -11;
    m->mg.clock = (unsigned long long *)d_clock;
    return 0;
}

int dec_clock_slots(dec_model *m)
{
    if (!m) return -11;
    if (!m->mega_ok) return 0;
    return m->mg.nbar + 1;
}

int dec_layer_clock(dec_model *m, int layer)
{
    if (!m || !m->mega_ok || layer < -1 || layer > m->c.n_layers) return -11;
    if (layer == -1) return 1;                  /* after the embedding */
    return m->layer_clock[layer];
}

int dec_set_layer_events(dec_model *m, void **events, int n)
{
    if (!m || n < 0 || (n && !events)) return -11;
    m->lev = n ? events : NULL;
    m->nlev = n;
    return 0;
}

int dec_set_residual_seams(dec_model *m, float *buf, int n)
{
    if (!m || n < 0 || n > m->c.n_layers + 1 || (n && !buf)) return -11;
    m->rseam = n ? buf : NULL;
    m->nrseam = n;
    if (m->mega_ok || m->persistent) CK(mega_build(m));
    return 0;
}

int64_t dec_layer_bytes(dec_model *m, int layer)
{
    if (!m || layer < -1 || layer >= m->c.n_layers) return -11;
    const linear_t *ls[8];
    int n = 0;
    int64_t b = 0;
    if (layer < 0) {
        ls[n++] = &m->lm;
        b += (int64_t)m->c.hidden * 2 * m->B;          /* the embedding rows */
    } else {
        const layer_t *l = &m->L[layer];
        if (l->attn) {
            ls[n++] = &l->qg; ls[n++] = &l->kv; ls[n++] = &l->o;
            int pos = 0;
            cudaSetDevice(m->device);
            cudaMemcpy(&pos, m->pos, 4, cudaMemcpyDeviceToHost);
            b += (int64_t)2 * (pos + 1) * m->kvh * HD * 2 * m->B;     /* K and V up to the position */
        } else {
            ls[n++] = &l->qkv; ls[n++] = &l->z; ls[n++] = &l->ab; ls[n++] = &l->out;
            b += ((int64_t)2 * m->vh * HD * HD * 4 + (int64_t)2 * 3 * m->conv_dim * 4) * m->B;   /* states r+w */
        }
        ls[n++] = &l->gate; ls[n++] = &l->up; ls[n++] = &l->down;
    }
    for (int i = 0; i < n; i++)
        b += (int64_t)ls[i]->rows * ls[i]->cols / 2 + (int64_t)ls[i]->rows * (ls[i]->cols / 128) * 2;
    return b;
}

int dec_pointers(dec_model *m, float **logits, int32_t **history, float **residual, int32_t **pos,
                 int32_t *vocab0, int32_t *vocab_n)
{
    if (!m) return -11;
    if (logits) *logits = m->logits;
    if (history) *history = m->hist;
    if (residual) *residual = m->x;
    if (pos) *pos = m->pos;
    if (vocab0) *vocab0 = m->voc0;
    if (vocab_n) *vocab_n = m->vocab;
    return 0;
}

int dec_linear(dec_model *m, int layer, const char *name, const uint8_t **d_wq, const uint16_t **d_sc,
               int32_t *rows, int32_t *cols, int32_t *s_pitch)
{
    if (!m || !name) return -11;
    const linear_t *l = NULL;
    if (layer < 0) { if (!strcmp(name, "lm_head")) l = &m->lm; }
    else if (layer < m->c.n_layers) {
        layer_t *L = &m->L[layer];
        const struct { const char *n; linear_t *l; } tab[] = {
            {"qkv", &L->qkv}, {"z", &L->z}, {"ab", &L->ab}, {"out", &L->out}, {"qg", &L->qg},
            {"kv", &L->kv}, {"o", &L->o}, {"gate", &L->gate}, {"up", &L->up}, {"down", &L->down}};
        for (unsigned i = 0; i < sizeof tab / sizeof tab[0]; i++)
            if (!strcmp(name, tab[i].n) && tab[i].l->wq) l = tab[i].l;
    }
    if (!l) return -11;
    *d_wq = l->wq; *d_sc = l->sc; *rows = l->rows; *cols = l->cols;
    if (s_pitch) *s_pitch = l->s_pitch;
    return 0;
}

int dec_load_linear(dec_model *m, int layer, const char *name, const uint8_t *h_wq, const uint16_t *h_sc,
                    int rows, int cols, int sc_pitch)
{
    const uint8_t *d_wq;
    const uint16_t *d_sc;
    int32_t r, k, sp;
    if (!h_wq || !h_sc || sc_pitch < cols / 128) return -11;
    CK(dec_linear(m, layer, name, &d_wq, &d_sc, &r, &k, &sp));
    if (rows != r || cols != k) return -11;          /* the shard this rank holds */
    cudaError_t e = cudaSetDevice(m->device);
    if (e == cudaSuccess) e = cudaMemcpy((void *)d_wq, h_wq, (size_t)r * k / 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy2D((void *)d_sc, (size_t)sp * 2, h_sc, (size_t)sc_pitch * 2, (size_t)(k / 128) * 2, (size_t)r,
                         cudaMemcpyHostToDevice);
    return e == cudaSuccess ? 0 : fail(e);
}

int dec_param(dec_model *m, int layer, const char *name, const void **d_ptr, int32_t *count)
{
    if (!m || !name) return -11;
    const int B = m->B;
    if (layer < 0) {
        const int H = m->c.hidden;
        const struct { const char *n; const void *p; int32_t c; } act[] = {
            {"final_norm", m->final_norm, H}, {"embed", m->embed, m->c.vocab * H},
            /* activation seams of the last step (the last layer that wrote
             * them), [batch][...] */
            {"x", m->x, H * B}, {"h16", m->h16, H * B}, {"qkv", m->qkv_f, m->conv_dim * B},
            {"qkv16", m->qkv16, m->conv_dim * B}, {"z", m->z_f, m->vh * HD * B},
            {"eg", m->eg, m->vh * B}, {"beta", m->beta, m->vh * B}, {"o", m->o_f, m->vh * HD * B},
            {"y16", m->y16, m->vh * HD * B}, {"qg", m->qg_f, 2 * m->qh * HD * B},
            {"kv", m->kv_f, 2 * m->kvh * HD * B}, {"q", m->q_f, m->qh * HD * B},
            {"ya16", m->ya16, m->qh * HD * B}, {"hf16", m->hf16, m->ffn * B}, {"logits", m->logits, m->vocab * B}};
        for (unsigned i = 0; i < sizeof act / sizeof act[0]; i++)
            if (!strcmp(name, act[i].n)) { *d_ptr = act[i].p; *count = act[i].c; return 0; }
        return -11;
    }
    if (layer >= m->c.n_layers) return -11;
    layer_t *L = &m->L[layer];
    const struct { const char *n; const void *p; int32_t c; } tab[] = {
        {"attn_norm", L->attn_norm, m->c.hidden}, {"post_norm", L->post_norm, m->c.hidden},
        {"conv_w", L->conv_w, 4 * m->conv_dim}, {"ssm_a", L->ssm_a, m->vh}, {"dt_bias", L->dt_bias, m->vh},
        {"ssm_norm", L->ssm_norm, HD}, {"q_norm", L->q_norm, HD}, {"k_norm", L->k_norm, HD},
        {"conv_state", L->conv_state, 3 * m->conv_dim * B}, {"rec_state", L->rec_state, m->vh * HD * HD * B},
        {"kcache", L->kcache, m->c.max_ctx * m->kvh * HD * B},
        {"vcache", L->vcache, m->c.max_ctx * m->kvh * HD * B}};
    for (unsigned i = 0; i < sizeof tab / sizeof tab[0]; i++)
        if (!strcmp(name, tab[i].n) && tab[i].p) { *d_ptr = tab[i].p; *count = tab[i].c; return 0; }
    return -11;
}

int64_t dec_step_bytes(dec_model *m)
{
    if (!m) return -11;
    int pos = 0;
    cudaSetDevice(m->device);
    cudaMemcpy(&pos, m->pos, 4, cudaMemcpyDeviceToHost);
    int64_t b = m->weight_bytes;
    for (int il = 0; il < m->c.n_layers; il++) {
        if (m->L[il].attn) b += (int64_t)2 * (pos + 1) * m->kvh * HD * 2 * m->B;
        else b += ((int64_t)2 * m->vh * HD * HD * 4 + (int64_t)2 * 3 * m->conv_dim * 4) * m->B;
    }
    b += (int64_t)m->c.hidden * 2 * m->B;       /* the embedding rows */
    return b;
}
