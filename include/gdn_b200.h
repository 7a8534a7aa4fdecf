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

#include <stddef.h>
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

/* ------------------------------------------------ the fixed-point block */

/* Field for field the caller-owned block record of the reference,
 * blk_t (ref/gdn_block_vec.c:183-202), in HOST memory:
 *   xtap, wtap [2*KH*D + VH*D][4]  conv taps (tap 3 = this token) and weights,
 *                                  channels [q | k | v], head-major
 *   e_t, tvalid [3][4]             per segment: tap exponents, tap validity
 *   cw_exp [3]                     conv weight exponent per segment
 *   sc [VH][8]                     {al_m, al_e, dt_m, dt_e, a_m, a_e, b_m, b_e}
 *   zm [VH][D] on z_e              the z gate input
 *   wm [D] on w_e                  the output rmsnorm weights
 *   tk0                            first token (state taken as zero)
 *   smem [VH][D][D], semem [VH][D] state mantissas / column exponents, in place
 *   y [VH*D], y_exp                output mantissas and the token exponent
 *   err_conv, err_g, err_se, y_sat range flags: set to 1, never cleared       */
typedef struct {
    const int16_t *xtap;
    const int16_t *wtap;
    const int     *e_t;
    const int     *tvalid;
    const int     *cw_exp;
    const int32_t *sc;
    const int16_t *zm;
    const int16_t *wm;
    int            w_e, z_e;
    int            tk0;
    int16_t       *smem;
    int           *semem;
    int16_t       *y;
    int            y_exp;
    int            err_conv, err_g, err_se, y_sat;
} gdn_blk_t;

/* Replaces gdn_block_token (ref/gdn_block_vec.c:208-423), whose shape comes
 * from the file globals KH, VH, D (:138) -- here arguments.  One token of the
 * fixed-point Gated DeltaNet block, bit-exact: conv + segment requantiser,
 * silu, per-key-head L2 norms, scalar path, recurrence, site-12 head emit,
 * output rmsnorm_bf (eps 1e-6), z gate, site-13 whole-token renorm.  Value
 * head h reads key head h % KH.  D is 32, 64 or 128; VH a multiple of KH.
 * Host buffers: the record is staged through device memory on every call
 * (the drop-in form; deltanet_step keeps everything resident).  Returns 0,
 * -11 (bad shape, no valid tap in a segment) or -20 (CUDA error). */
int gdn_block_token_host(int KH, int VH, int D, gdn_blk_t *b);

/* The same token on DEVICE buffers, state resident.  Two launches on
 * `stream` (one CTA per value head, in clusters of up to 8: conv segment
 * maxima, silu, L2 norms, scalar path, recurrence, head emit, rmsnorm, gate;
 * then the site-13 tail), the second a programmatic dependent of the first;
 * with pdl set the first is also a dependent of the kernel before it in the
 * stream.  The small per-token control words
 * (tap exponents, validity, segment weight exponents) are passed by value.
 * status (device, 5 ints) receives {y_exp, err_conv, err_g, err_se, y_sat}
 * for this token.  work: deltanet_work_bytes(KH, VH, D) bytes of device
 * memory, 256-byte aligned, owned by the caller (scratch between the
 * launches; two calls in flight at once need two workspaces). */
typedef struct {
    int32_t        KH, VH, D;
    const int16_t *xtap, *wtap;     /* [2*KH*D + VH*D][4], 8-byte aligned       */
    int32_t        e_t[3][4];
    int32_t        tvalid[3][4];
    int32_t        cw_exp[3];
    const int32_t *sc;              /* [VH][8]                                  */
    const int16_t *zm;              /* [VH][D]                                  */
    const int16_t *wm;              /* [D]                                      */
    int32_t        w_e, z_e, tk0;
    int16_t       *smem;            /* [VH][D][D], 32-byte aligned, in place    */
    int32_t       *semem;           /* [VH][D], in place                        */
    int16_t       *y;               /* [VH*D]                                   */
    int32_t       *status;          /* [5]                                      */
    void          *work;
    int32_t        pdl;
} deltanet_args;

size_t deltanet_work_bytes(int KH, int VH, int D);
int deltanet_step(const deltanet_args *a, void *stream);

/* The block's stages one at a time, on device buffers: the unit cores the
 * reference keeps for its vector generators.
 *   gdn_conv_seg_dev   conv + segment requantiser (ref/gdn_conv_vec.c:80-103):
 *                      ncase segments of nch channels x 4 taps; cfg [ncase][9]
 *                      = {tvalid[4], e_t[4], cw_exp}; sm [ncase][nch] the
 *                      requantised mantissas; info [ncase][3] = {e_seg, sh_seg, err}
 *   gdn_silu_dev       silu with the exponent preserved (ref/gdn_silu_vec.c):
 *                      ncase rows of n int16, row r on exponent e_row[r]
 *   gdn_l2norm_dev     l2norm_rs (ref/l2norm_rs_vec.c:118): nvec vectors of N
 *                      (32/64/128) -> k (exponent 15) and q (exponent 18)
 *   gdn_rmsnorm_bf_dev rmsnorm_bf_int (ref/rmsnorm_bf_vec.c:199), eps 1e-6:
 *                      nvec vectors of N with their own xe, weights, we
 *   gdn_y_emit_dev     site 13 (ref/gdn_y_emit_vec.c:124-143); status[0] =
 *                      y_exp, status[4] = saturation
 *   gdn_emit_chain_dev site 12 -> rmsnorm -> z gate -> site 13
 *                      (ref/gdn_emit_chain_vec.c); work as for deltanet_step
 *                      with KH = 1, VH = H */
int gdn_conv_seg_dev(int ncase, int nch, const int16_t *x, const int16_t *w, const int32_t *cfg,
                     int16_t *sm, int32_t *info, void *stream);
int gdn_silu_dev(int ncase, int n, const int16_t *sm, const int32_t *e_row, int32_t *y, void *stream);
int gdn_l2norm_dev(int nvec, int N, const int32_t *x, int16_t *k, int16_t *q, void *stream);
int gdn_rmsnorm_bf_dev(int nvec, int N, const int16_t *xm, const int32_t *xe, const int16_t *wm,
                       const int32_t *we, int16_t *o, int32_t *o_exp, void *stream);
int gdn_y_emit_dev(int H, int D, const int32_t *ep, const int16_t *po, const int16_t *pz,
                   int16_t *y, int32_t *status, void *stream);
int gdn_emit_chain_dev(int H, int D, const int64_t *o_acc, const int32_t *e_o, const int16_t *zm,
                       const int16_t *wm, int we, int z_e, int16_t *y, int32_t *status, void *work,
                       void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GDN_B200_H */
