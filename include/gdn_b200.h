/* include/gdn_b200.h -- C ABI of the B200 Gated DeltaNet step (llm.vhdl
 * subsystem B): the scalar path, the fixed-point recurrence with its stage-6
 * head emit, and the binary32 recurrence of the benchmark's config 1.
 *
 * The reference runs these inline in gdn_block_token (ref/gdn_block_vec.c:208,
 * a static function over the caller-owned blk_t of ref/gdn_block_vec.c:183-202)
 * and in gdn_err's main (ref/gdn_err.c:460-606).  This library keeps the same
 * state layout -- smem[h][j][i] int16 mantissas, value column j of head h
 * contiguous over key index i, one exponent semem[h][j] per column -- and the
 * same key-head mapping (value head h reads key head h % KH,
 * ref/gdn_block_vec.c:141-166), with the state resident in device memory and
 * updated in place.  Every entry point returns 0 or a negative code (-11 bad
 * argument, -20 CUDA error) and never aborts.  Streams are void* (cudaStream_t).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces gdn_scalar_int (ref/gdn_scalar_vec.c:100-156) for H value heads:
 * d_sc[h*8 .. h*8+7] = {al_m, al_e, dt_m, dt_e, a_m, a_e, b_m, b_e}; writes
 * eg (Q15, <= 32768), beta (Q16, <= 65535) and err_g per head.  The Q30
 * exp / sigmoid / softplus tables are built on the host with the reference's
 * rule (ref/fx.h:51-79) and uploaded once per device. */
int gdn_scalar_dev(int H, const int32_t *d_sc, int32_t *d_eg, int32_t *d_beta, int32_t *d_err,
                   void *stream);

/* One fixed-point step, every head (spec B 2.1.4 stages 1-6):
 * the recurrence of ref/gdn_block_vec.c:298-361 and the site-12 head emit of
 * ref/gdn_block_vec.c:363-378. */
typedef struct {
    int32_t        H, KH, D;        /* value heads, key heads, head dim (<= 128) */
    int16_t       *smem;            /* [H][D][D] state mantissas, in place     */
    int32_t       *semem;           /* [H][D] column exponents, in place       */
    const int16_t *kn;              /* [KH][D] L2-normalised k, Q15            */
    const int16_t *qs;              /* [KH][D] q with 1/sqrt(D) folded, Q18    */
    const int32_t *v;               /* [H][D] v mantissas on exponent e_v      */
    int32_t        e_v;
    const int32_t *eg;              /* [H] decay gate, Q15                     */
    const int32_t *beta;            /* [H] beta, Q16                           */
    int32_t        tk0;             /* first token: the state is taken as 0    */
    int64_t       *o_acc;           /* [H][D] stage-5 output dots              */
    int32_t       *e_o;             /* [H][D] their exponents (se_new + 18)    */
    int16_t       *o_head;          /* [H][D] stage-6 BFP head output (or NULL) */
    int32_t       *e_head;          /* [H] head exponents (or NULL)            */
    int32_t       *err;             /* one int: OR of the exponent-range flags  */
} gdn_fixed_args;

int gdn_step_fixed(const gdn_fixed_args *a, void *stream);

/* T sequential binary32 steps (ref/gdn_err.c:580-590 recurrence) in one
 * launch, the state kept on chip between steps and written back at the end:
 *   alpha = exp(-softplus(a)), beta = sigmoid(b)          (per head, per step)
 *   q, k  <- q/|q|, k/|k| per head when l2norm, then q *= q_scale
 *   S'    = alpha*S;  sk = S'k;  d = (v - sk)*beta;  S = S' + k d^T
 *   out   = (S q) * sigmoid(g)  when g != NULL, else S q
 * S [H][D][D] fp32 (value column j of head h contiguous over key i);
 * q, k [T][KH][D], v [T][H][D], g [T][H][D] fp16; a, b [T][H] fp32;
 * out [T][H][D] fp32 and/or fp16.  T = 1 is one decode step (of nseq
 * sequences at once when nseq > 1). */
typedef struct {
    int32_t         T, H, KH, D;    /* D must be 128                            */
    float          *S;
    const uint16_t *q, *k, *v, *g;
    const float    *a, *b;
    int32_t         l2norm;
    float           q_scale;
    float          *out_f32;
    uint16_t       *out_f16;
    const float    *eg, *beta;      /* optional [T][H]: the decay and beta
                                       already activated (the model's
                                       exp(ssm_a*softplus(.)) and sigmoid);
                                       when set, a and b are not read      */
    int32_t         pdl;            /* launch as a programmatic dependent of
                                       the previous kernel in the stream    */
    int32_t         nseq;           /* independent sequences stepped in one
                                       launch (0 or 1: one).  With nseq > 1,
                                       T must be 1; sequence n reads q, k, v
                                       at +n*seq_in elements, a, b, eg, beta
                                       at +n*H, g and writes out at +n*H*D,
                                       and owns the state S + n*H*D*D      */
    int32_t         seq_in;
    int32_t         pad_;
} gdn_f32_args;

int gdn_run_f32(const gdn_f32_args *a, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GDN_B200_H */
