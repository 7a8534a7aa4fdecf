/* include/dec_b200.h -- C ABI of the decode loop built on the hot path: a
 * Qwen3.5-style hybrid decoder (Gated DeltaNet and gated-attention layers,
 * SwiGLU MLP, INT4 g128 linears, LM head + first-max argmax) stepping one
 * token per call, on one GPU or tensor-parallel over several (one process per
 * GPU, NCCL).  It composes the matvec (mv4i_b200.h) and DeltaNet step
 * (gdn_b200.h) kernels the way ref/run9b.c composes mv4i_matvec and its
 * delta rule: layer_gdn (ref/run9b.c:602-756), layer_attn (:758-900),
 * lm_head + argmax_first (:399-405, :522-540).  The arithmetic is the
 * benchmark's floating-point mode (fp16 activations into INT4 g128
 * projections, fp32 residual stream, recurrent state and accumulation); the
 * bit-exact integer mode of the golden model is the matvec library's.
 *
 * The position and the current token live in device memory, so one step can
 * be captured in a CUDA graph and replayed for every token.
 */
#ifndef DEC_B200_H
#define DEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t hidden;          /* residual width                                */
    int32_t n_layers;
    int32_t attn_every;      /* layer il is attention when (il+1) % attn_every == 0
                                (ref/run9b.c is_attn)                          */
    int32_t vocab;
    int32_t ffn;             /* SwiGLU intermediate                           */
    int32_t gdn_kh, gdn_vh, gdn_hd;      /* DeltaNet key heads, value heads, dim */
    int32_t att_qh, att_kvh, att_hd;     /* attention heads and dim             */
    int32_t n_rot;           /* rotary dims per head (NeoX pairing i, i+n_rot/2) */
    float   rope_theta;
    float   rms_eps;
    int32_t max_ctx;         /* KV-cache capacity in positions (<= 65536)    */
    int32_t batch;           /* independent sequences decoded together, 1..8
                                (0 means 1; more than 1 only with tp_world 1).
                                They share every weight read of a step and
                                the position; each has its own token, KV
                                cache, DeltaNet and conv states and history */
} dec_config;

typedef struct dec_model dec_model;

/* Random-init weights of the configured architecture (seeded splitmix64,
 * INT4 g128 linears as in the benchmark's config 0), on `device`; tp_world
 * ranks each hold their shard (tp_world = 1: everything).  Shards: heads for
 * DeltaNet and attention, rows for column-parallel projections (qkv, z, a/b,
 * q|gate, k|v, gate, up) and the LM head's vocabulary, columns for the
 * row-parallel ones (DeltaNet out, attention O, FFN down).  Every rank draws
 * its shard from the same global matrices (draws are keyed by global row and
 * column), so any tp_world computes the same model. */
int dec_create(const dec_config *cfg, uint64_t seed, int device, int tp_rank, int tp_world,
               dec_model **out);
int dec_destroy(dec_model *m);

/* NCCL for tp_world > 1: rank 0 calls dec_nccl_unique_id, the caller ships
 * the 128 bytes to every rank (any transport), and every rank calls
 * dec_tp_init before its first step. */
int dec_nccl_unique_id(uint8_t id[128]);
int dec_tp_init(dec_model *m, const uint8_t id[128]);

/* Peer-memory exchange for tensor parallel: replaces the NCCL all-reduce of
 * every row-parallel block and the all-gather of the argmax keys with one-shot
 * stores into the peers' memory over NVLink (one small kernel each, no NCCL
 * on the data path).  Every rank calls dec_p2p_handle (it allocates this
 * rank's exchange region), the host all-gathers the 64-byte handles in rank
 * order (any transport), and every rank calls dec_p2p_open with all of them.
 * Waits on peers are bounded by spin_limit polls (<= 0: about a second); a
 * wait that runs out records a flag and the step goes on, so a rank that never
 * joins cannot hang the others: dec_status returns the flags (1 all-reduce, 2
 * key exchange) and clears them. */
int dec_p2p_handle(dec_model *m, uint8_t handle[64]);
int dec_p2p_open(dec_model *m, const uint8_t *handles, int spin_limit);
int dec_status(dec_model *m, int32_t *flags);

/* Fills the first `len` positions of every attention layer's KV cache with
 * N(0,1) fp16 (the benchmark's pre-filled context), the DeltaNet states with
 * N(0, 0.02) and the conv states with N(0, 0.5), and sets the position to len.
 * Sequence b of a batch draws from seed ^ (b * 0x9E3779B97F4A7C15). */
int dec_prefill_random(dec_model *m, int len, uint64_t seed);

/* Sets the position and the current input token of every sequence (host
 * values); clears any prompt. */
int dec_set(dec_model *m, int pos, int token);

/* Starts the batch's sequences from position 0 (DeltaNet and conv states
 * zeroed) with prompts of n tokens each (host array [batch][n]):
 * steps 0 .. n-2 take the prompt's next token as their next input (teacher
 * forcing, ref/run9b.c's --tokens loop), later steps their own argmax.  The
 * prediction of every step is recorded in the history at its position, so
 * history[n-1 ..] is the generated continuation.  The copies are ordered on
 * `stream` and complete before the call returns. */
int dec_set_prompt(dec_model *m, const int32_t *tokens, int n, void *stream);

/* One decode step on `stream`: embeds the current token, runs every layer,
 * the LM head and argmax; the argmax becomes the current token and is stored
 * in the token history at the current position; the position advances.  No
 * host synchronisation.  Returns -11 once the position reaches max_ctx (a
 * host-side count); replays of a captured step are bounded on the device
 * instead: past max_ctx nothing more is written to the KV cache or history. */
int dec_step(dec_model *m, void *stream);

/* Device pointers for inspection: the fp32 logits of the last step (this
 * rank's vocabulary shard, [batch][vocab_n]), the token history
 * [batch][max_ctx], the fp32 residual [batch][hidden], the position. */
int dec_pointers(dec_model *m, float **logits, int32_t **history, float **residual, int32_t **pos,
                 int32_t *vocab0, int32_t *vocab_n);

/* Weight arrays of one linear, for the oracle: d_wq [rows][cols/2] packed
 * INT4, d_sc [rows][s_pitch] fp16 (cols/128 used; the pitch keeps every row
 * 16-byte aligned).  Names: "qkv", "z", "ab", "out", "qg", "kv", "o", "gate",
 * "up", "down" (per layer) and "lm_head" (layer -1). */
int dec_linear(dec_model *m, int layer, const char *name, const uint8_t **d_wq, const uint16_t **d_sc,
               int32_t *rows, int32_t *cols, int32_t *s_pitch);

/* Real weights into a model: copies a g128 tensor from host memory -- INT4
 * two's-complement nibbles [rows][cols/2] (column k even in the low nibble)
 * and fp16 scales [rows][sc_pitch], one per 128 columns -- over the linear
 * `name` of `layer` (names as dec_linear).  rows x cols must be the shard
 * this rank holds (dec_linear reports it).  An .mv4i image converts to this
 * form with mv4i_image_to_g128 when its values allow it, a float matrix with
 * mv4i_quantize_g128.  No counterpart in the reference, whose weights come
 * to the card as packed images. */
int dec_load_linear(dec_model *m, int layer, const char *name, const uint8_t *h_wq, const uint16_t *h_sc,
                    int rows, int cols, int sc_pitch);

/* Parameter and state vectors: "attn_norm", "post_norm", "conv_w"
 * ([conv_dim][4]), "ssm_a", "dt_bias", "ssm_norm", "q_norm", "k_norm",
 * "conv_state", "rec_state", "kcache", "vcache" (per layer; the states and
 * caches [batch][...]), "final_norm" and
 * the fp16 "embed" [vocab][hidden] (layer -1).  Layer -1 also names the
 * activation seams of the last step, as the last layer to write each left
 * them (the reference's seam records): fp32 "x" (residual), "qkv" (the raw
 * projection), "z", "eg", "beta", "o", "qg", "kv", "q" (after norm and RoPE), "logits"; fp16
 * "h16" (the last RMSNorm output), "qkv16" (after conv + SiLU), "y16" (DeltaNet
 * output after norm and gate), "ya16" (attention output), "hf16" (SwiGLU), each
 * [batch][...]. */
int dec_param(dec_model *m, int layer, const char *name, const void **d_ptr, int32_t *count);

/* Bytes of weights, KV cache and state one step (of every sequence of the
 * batch) reads on this rank. */
int64_t dec_step_bytes(dec_model *m);

/* Per-layer accounting: dec_layer_bytes is what layer `layer` reads in one
 * step on this rank (layer -1: LM head and embedding row); with
 * dec_set_layer_events (n cudaEvent_t handles, NULL/0 to stop) dec_step
 * records events[il] on its stream after layer il, so the host can time each
 * layer (record a start event before the step). */
int64_t dec_layer_bytes(dec_model *m, int layer);
int dec_set_layer_events(dec_model *m, void **events, int n);

/* The persistent step (single GPU; off by default, environment
 * DEC_PERSISTENT=1 turns it on at creation): dec_step is then ONE launch of a
 * kernel that
 * walks the whole layer program -- the counterpart of the reference
 * sequencer's per-token program (ref/run9b.c:1028-1170 issues the same A jobs
 * and delta rule one by one) -- with a grid barrier between dependent stages
 * and the next projection's weights prefetched into L2 during the current
 * stage.  Barrier waits are bounded (about a second); a wait that runs out
 * aborts the step and sets flag 4 of dec_status (which clears it).  Off, every
 * stage is its own kernel launch (programmatic dependent launches).  On B200 a
 * grid barrier costs about as much as a dependent launch (2-3 us), so the
 * launch mode, whose next kernel starts its weight prefetch while the previous
 * one finishes, is the faster default.
 * Tensor-parallel models always step in launch mode.
 * dec_set_persistent(m, on) switches (on: builds and uploads the program;
 * synchronises the device), dec_persistent(m) tells which mode dec_step uses. */
int dec_set_persistent(dec_model *m, int on);
int dec_persistent(dec_model *m);
/* Input staging in launch mode.  Every CTA of a matvec needs the whole input
 * vector of each sequence as int16 byte planes; for a batch, building them
 * in every CTA costs more than the weight stream.  mode 1 (the default)
 * stages a batch's inputs once per matvec in a launch of its own that the
 * matvec's CTAs copy from; 2 does so for single sequences too; 0 never.  The
 * staged values are the same in every mode (bit-identical results);
 * DEC_PRESTAGE=0|1|2 in the environment sets the mode at creation.  No
 * counterpart in the reference (its CPU matvec stages each input once). */
int dec_set_prestage(dec_model *m, int mode);

/* Bound of each grid-barrier wait of the persistent step, in ns (0: the
 * default, one second). */
int dec_set_wait_limit(dec_model *m, int64_t ns);

/* Stage clock of the persistent step: with a device buffer of
 * dec_clock_slots(m) uint64 entries (NULL to stop), each step writes the GPU
 * global timer (ns) at its start (entry 0) and after every grid barrier;
 * dec_layer_clock(m, il) is the entry written at the end of layer il
 * (il = -1: the embedding; il = n_layers: the LM head). */
int dec_set_clock(dec_model *m, uint64_t *d_clock);
int dec_clock_slots(dec_model *m);
int dec_layer_clock(dec_model *m, int layer);

/* Residual seams (the reference's per-layer seam records, for parity
 * checks): with a device buffer of n slots of [batch][hidden] fp32 (n <=
 * n_layers + 1; NULL/0 to stop), dec_step copies the residual stream into
 * slot il as layer il starts, and into slot n_layers after the last layer
 * (the LM head's input).  Copies on the step's stream. */
int dec_set_residual_seams(dec_model *m, float *buf, int n);

/* ------------------------------------------------ one attention token */

/* One token of gated attention on device buffers, the counterpart of the
 * reference's attn_token (ref/attn_block_vec.c:533-541) in the decoder's
 * floating-point mode (ref/run9b.c:786-872, layer_attn without its
 * projections).  For every KV head: k = NeoX-RoPE(RMSNorm(k_in, k_norm)) and
 * the raw v go to the fp16 caches at row pos (the append); for every query
 * head: q = RoPE(RMSNorm(q_in, q_norm)), softmax(q . K[0..pos] / sqrt(128))
 * over its KV head (GQA, contiguous groups: query head h reads KV head
 * h / (n_qh / n_kvh)), times V, times sigmoid(gate), fp16 out.  Past
 * capacity (pos >= max_ctx) the cache is attended as it stands.
 *   qg       [n_qh][2][128] fp32: q then gate, per head (the reference's qg)
 *   kv       [2][n_kvh][128] fp32: k rows, then v rows
 *   q_norm, k_norm [128] fp32; eps the RMSNorm epsilon
 *   d_pos    device int32: the position this token writes and attends up to
 *   kcache, vcache fp16 [max_ctx][n_kvh][128]
 *   y        fp16 [n_qh][128]; q_out (optional) fp32 [n_qh][128] the
 *            normalised, rotated q
 *   work     gated_attn_work_bytes(n_qh, max_ctx) bytes of device memory
 * Two launches (flash decoding over chunks of 16, 32 or 64 positions, then the
 * combine with the gate); pdl makes the first a programmatic dependent of the
 * kernel before it in the stream.  Head dim 128, n_qh / n_kvh <= 32, n_rot
 * even and <= 128, max_ctx <= 65536.  Returns 0, -11 or -20. */
typedef struct {
    int32_t         n_qh, n_kvh, head_dim, n_rot;
    float           rope_theta, eps;
    const float    *qg, *kv;
    const float    *q_norm, *k_norm;
    const int32_t  *d_pos;
    int32_t         max_ctx;
    uint16_t       *kcache, *vcache;
    uint16_t       *y;
    float          *q_out;
    void           *work;
    int32_t         pdl;
} gated_attn_args;

size_t gated_attn_work_bytes(int n_qh, int max_ctx);
int gated_attn(const gated_attn_args *a, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DEC_B200_H */
