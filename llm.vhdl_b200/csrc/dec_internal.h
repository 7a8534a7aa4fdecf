/* llm.vhdl_b200/csrc/dec_internal.h -- parameter block of the decode-step
 * matvec (dec_matvec.cu), shared by the kernel and its C caller (dec_model.c).
 * Not part of the public ABI. */
#ifndef DEC_INTERNAL_H
#define DEC_INTERNAL_H

#include <stdint.h>
#include "../../include/gdn_b200.h"

#define DMV_MAXJ 4

/* prologue: how the CTA builds its fp16 input vector x[K] */
enum { DMV_OP_F16 = 0,        /* x16 given                                       */
       DMV_OP_RMSNORM = 1,    /* x = rmsnorm(res[K]) * w[K]          (run9b.c:557) */
       DMV_OP_GATED = 2 };    /* per 128-group: rmsnorm(o) * w[128] * silu(z)    */

/* epilogue: what each output row does with its fp32 dot product v */
enum { DMV_EPI_F32 = 0,       /* out_f32[r] = v                                  */
       DMV_EPI_ACC = 1,       /* out_f32[r] += v  (residual add)                 */
       DMV_EPI_F16 = 2,       /* out_f16[r] = fp16(v)                            */
       DMV_EPI_SWIGLU = 3,    /* paired rows: out_f16[r] = fp16(silu(v) * v2)    */
       DMV_EPI_CONV = 4,      /* DeltaNet 4-tap conv + SiLU on channel r, fp16   */
       DMV_EPI_GATES = 5,     /* r < n1: eg = exp(p0[r]*softplus(v+p1[r]));
                                 else beta[r-n1] = sigmoid(v)                    */
       DMV_EPI_ARGMAX = 6 };  /* out_f32[r] = v and the first-max key           */

typedef struct {
    const uint8_t  *wq, *wq2;      /* [rows][K/2] packed INT4 (wq2: paired rows)  */
    const uint16_t *sc, *sc2;      /* [rows][s_pitch] fp16 scales (K/128 used)    */
    float          *out_f32;       /* F32/ACC/ARGMAX out; CONV: raw projection
                                      (optional); GATES: eg                       */
    float          *out2_f32;      /* GATES: beta                                 */
    uint16_t       *out_f16;       /* F16/SWIGLU/CONV out                         */
    const float    *p0, *p1;       /* CONV: conv_w [rows][4]; GATES: ssm_a, dt_bias */
    float          *st;            /* CONV: conv state [3][st_stride]             */
    int32_t         st_stride, n1;
    int32_t         rows, epi, tile0, ntiles;
    int32_t         s_pitch;       /* scale row pitch in fp16 elements: a
                                      multiple of 8, >= ceil8(K/128)           */
    int32_t         ostride;       /* vector b's outputs (out_f32, out2_f32,
                                      out_f16) at +b*ostride elements; its
                                      CONV state at st + b*3*st_stride       */
} dmv_job;

typedef struct {
    dmv_job   jobs[DMV_MAXJ];
    int32_t   njobs, total_tiles, K, op;
    const void  *x;                /* F16: fp16 [K]; RMSNORM: fp32 residual; GATED: fp32 o */
    const float *x2;               /* GATED: z [K]                                 */
    const float *nw;               /* RMSNORM: w [K]; GATED: w [128]               */
    float        eps;
    uint16_t    *seam;             /* optional: CTA 0 stores the fp16 input here   */
    unsigned long long *key;       /* ARGMAX key (first max, global index)         */
    int32_t      idx0;             /* ARGMAX: global index of row 0                */
    int32_t      pf_bytes;         /* weight bytes each CTA prefetches to L2 early */
    int32_t      ksplit;           /* set by the launcher: warps per row       */
    int32_t      nvec;             /* input vectors (sequences) 1..8, sharing
                                      every weight load: vector b's x and x2
                                      at +b*xs elements, its seam at +b*K, its
                                      argmax key at key[b] (0 means 1)      */
    int32_t      xs;
    int32_t      pad_;
    uint8_t     *xst;              /* optional: the inputs already staged by
                                      dec_k_stage ([nvec] blocks of the
                                      shared-memory layout); the matvec copies
                                      them instead of staging (and leaves the
                                      seam to dec_k_stage)                    */
} dmv_params;

/* the gated-attention step (dec_kernels.cu): flash decoding over chunks of
 * `ch` positions, then the combine with the sigmoid gate */
typedef struct {
    const float *qg, *kv;          /* raw projections: q|gate per head, k|v    */
    const float *qn_w, *kn_w;      /* q / k RMSNorm weights [128]               */
    int32_t      qh, kvh, n_rot;
    float        theta, eps;
    const int32_t *d_pos;          /* the position (device)                     */
    int32_t      max_ctx, ch, nchunks;
    uint16_t    *kcache, *vcache;  /* [nseq][max_ctx][kvh][128] fp16            */
    float       *q_seam, *part;    /* optional q seam; chunk records            */
    uint16_t    *y;                /* fp16 gated output [nseq][qh][128]         */
    int32_t      nseq;
} dec_attn_args;

/* One stage of the persistent decode kernel's program (dec_step.cu): a piece
 * of work every CTA takes its share of, then (sync != 0) a grid-wide barrier.
 * The program of a step is the reference sequencer's per-token layer program
 * in this form: embed, per layer the projection / delta-rule / attention
 * stages, LM head, advance. */
enum { MG_EMBED = 1, MG_MATVEC = 2, MG_GDN = 3, MG_ATTN = 4, MG_COMBINE = 5, MG_ADVANCE = 6, MG_COPY = 7 };

typedef struct {
    const uint16_t *emb; const int32_t *tok; float *x; int32_t hidden, nseq;
} mg_embed_args;

typedef struct {
    unsigned long long *keys, *key; int32_t *tok, *hist, *pos; const int32_t *prompt;
    int32_t n, nseq, max_ctx, pad_;
} mg_advance_args;

typedef struct {
    float *dst; const float *src; int64_t n;
} mg_copy_args;

typedef struct {
    int32_t op, sync;
    int32_t pf;                    /* set on upload: the MATVEC stage whose
                                      weights this stage prefetches, or -1 */
    int32_t pad_;
    union {
        dmv_params      mv;
        gdn_f32_args    gdn;
        dec_attn_args   att;
        mg_embed_args   emb;
        mg_advance_args adv;
        mg_copy_args    cp;
        uint8_t         raw_[544];     /* the record is a whole number of
                                          16-byte words (copied as such) */
    } u;
} mg_stage;
typedef char mg_stage_size_check[(sizeof(mg_stage) % 16) == 0 && sizeof(dmv_params) <= 544 ? 1 : -1];

/* the control block of the persistent kernel (device memory, zeroed) */
typedef struct {
    unsigned long long count;      /* grid-barrier arrivals, never reset        */
    int32_t abort;                 /* a barrier timed out: every CTA leaves     */
    int32_t err_stage;             /* the stage whose barrier timed out         */
} mg_ctl;

/* an uploaded program */
typedef struct {
    mg_stage *d_prog;
    int32_t   n, nbar, grid, nv;
    int64_t   smem;
    mg_ctl   *ctl;
    unsigned long long *clock;     /* optional [nbar + 1] globaltimer stamps */
    int64_t   timeout_ns;
    int32_t   pf_bytes, pad_;
} mg_prog;

#ifdef __cplusplus
extern "C" {
#endif
/* Prepares and uploads a recorded program (host stages, n of them) for the
 * persistent kernel of `nv` sequences on the current device: grid size,
 * matvec tiling for that grid, prefetch plan, shared memory.  *P must hold a
 * zeroed d_prog (first upload: allocated here) or a previous upload of the
 * same length. */
int dec_mega_upload(mg_stage *stages, int n, int nv, mg_prog *P);
int dec_k_mega(const mg_prog *P, void *stream);
/* Launches the decode matvec on `stream`; pdl != 0 launches it as a
 * programmatic dependent of the previous kernel in the stream. */
int dec_k_matvec(const dmv_params *p, void *stream, int pdl);
/* Stages the input vectors of a matvec (prologue, fp16 rounding, int16 byte
 * planes; the seam) into p->xst once for all CTAs of the matvec that follows;
 * dec_k_stage_bytes(K, nvec) is the size p->xst needs. */
int dec_k_stage(const dmv_params *p, void *stream, int pdl);
long long dec_k_stage_bytes(int K, int nvec);
#ifdef __cplusplus
}
#endif
#endif /* DEC_INTERNAL_H */
