/* llm.vhdl_b200/csrc/dec_internal.h -- parameter block of the decode-step
 * matvec (dec_matvec.cu), shared by the kernel and its C caller (dec_model.c).
 * Not part of the public ABI. */
#ifndef DEC_INTERNAL_H
#define DEC_INTERNAL_H

#include <stdint.h>

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
} dmv_params;

#ifdef __cplusplus
extern "C" {
#endif
/* Launches the decode matvec on `stream`; pdl != 0 launches it as a
 * programmatic dependent of the previous kernel in the stream. */
int dec_k_matvec(const dmv_params *p, void *stream, int pdl);
#ifdef __cplusplus
}
#endif
#endif /* DEC_INTERNAL_H */
