/* include/mv4i_b200.h -- C ABI of the B200 INT4 streaming matvec (subsystem A
 * of llm.vhdl) and its tensor-parallel reduction (subsystem E).
 *
 * Two layers:
 *
 *  1. DROP-IN.  mv4i_parse / mv4i_matvec with the reference golden model's
 *     signatures, struct layouts and return codes (ref/matvec_int4.c:51-69,
 *     161-255, 319-441).  Host buffers in, host buffers out; the weight image
 *     is relaid out and kept resident in HBM on first use (see mv4i_matvec).
 *
 *  2. DEVICE-RESIDENT.  Weights uploaded once into the stream layout
 *     (mv4i_dmat), activations and results in device memory, launches on a
 *     caller stream, scalar results (y_exp, ns, sat) in a device-side
 *     mv4i_status.  A launch carries a LIST of matvec jobs (the analogue of
 *     the reference's A_JOB descriptors), so several projections that share
 *     an activation, or a stack of matrices, run as one kernel.
 *
 * Numerics: golden mode is bit-exact with ref/matvec_int4.c (contract 7.4 of
 * docs/superpowers/specs/2026-08-20-int4-streaming-matvec-design.md).  The
 * g128 mode is the fp16 format of the benchmark configuration (signed INT4,
 * fp16 scale per 128 columns, fp16 activations, fp32 accumulation).
 *
 * Every entry point returns an int status (0 = ok) and never aborts.  Codes:
 *   -1..-9   as mv4i_parse / mv4i_matvec in the reference
 *   -10      an operand broke a 7.4 width contract the reference asserts on
 *            (|partial| >= 2^27, scale > 32767, |contrib| >= 2^27,
 *            |acc| >= 2^47); the reference aborts here, this library reports
 *   -11      bad argument (NULL pointer, job count, geometry)
 *   -12      tensor-parallel reduction refused: y_exp spread > 17
 *   -13      tensor-parallel reduction refused: out_shift differs between shards
 *   -14      mv4i_launch_noalloc: more jobs than its fixed counter array holds
 *   -15      tensor-parallel message from another collective (sequence number)
 *   -20      CUDA runtime error (mv4i_last_cuda_error() has the code)
 *
 * Streams are passed as void* (a cudaStream_t; NULL = legacy default stream)
 * so this header needs no CUDA include.
 */
#ifndef MV4I_B200_H
#define MV4I_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------- reference types (drop-in) */

#define MV4I_MAGIC      0x4D563449u   /* "MV4I"            ref/matvec_int4.c:38 */
#define MV4I_BLOCK      32            /* weights per scale ref/matvec_int4.c:39 */
#define MV4I_HDR_BYTES  4096          /*                   ref/matvec_int4.c:40 */
#define MV4I_MAX_SUB    64            /*                   ref/matvec_int4.c:46 */

enum { MV4I_MODE_BFP = 0, MV4I_MODE_RAW = 1, MV4I_MODE_PARTIAL = 2 };

/* Same field order and types as ref/matvec_int4.c:51-59, so code written
 * against the reference compiles and runs unchanged. */
typedef struct {
    uint32_t magic, M, K, scale_offset, n_scale_sub;
    uint16_t version, flags, rows_if, nports_w, block, axi_dw;
    int32_t  w_exp, out_shift;
    int8_t   codebook[16];
    uint64_t w_sub_offset[MV4I_MAX_SUB];
    uint64_t s_sub_offset[MV4I_MAX_SUB];
} mv4i_hdr;

/* ref/matvec_int4.c:61-69: the parsed file BORROWS the image. */
typedef struct {
    mv4i_hdr        h;
    const uint8_t  *base;
    int             nb;
    int             port_b;
    int             grp;
} mv4i_file;

/* ref/matvec_int4.c:319-327 */
typedef struct {
    int32_t *y_data;
    int64_t *y_acc;
    int16_t *y_mant;
    int      y_exp;
    int      sat_event;
    uint64_t sat_count;
    int      ns;
} mv4i_result;

/* Replaces mv4i_parse, ref/matvec_int4.c:161.  Same validation order and
 * refusal codes -1..-9; f->base borrows img. */
int mv4i_parse(mv4i_file *f, const uint8_t *img, size_t len);

/* Replaces mv4i_matvec, ref/matvec_int4.c:329.  Host x_mant in, host arrays
 * of `out` filled exactly as the reference fills them (y_data in RAW and BFP
 * modes, y_mant in BFP, y_acc in PARTIAL; y_exp, sat_event, sat_count, ns).
 * Runs on the current CUDA device.  The first call for an image uploads its
 * stream relayout to HBM and caches it keyed by (f->base, header, a sampled
 * content fingerprint); later calls reuse it, so only x and y cross PCIe.
 * A caller that frees an image, or rewrites its bytes in place, calls
 * mv4i_forget(f) first: the fingerprint samples the image and cannot see
 * every edit.  Thread-safe; calls are serialised on an internal stream. */
int mv4i_matvec(const mv4i_file *f, const int16_t *x_mant, int x_exp,
                int n_rows, int n_cols, int out_mode, mv4i_result *out);

/* Drops the cached device copy of f's image (no-op when none). */
int mv4i_forget(const mv4i_file *f);

/* The reference's byte accessors, ref/matvec_int4.c:267-307 (used by
 * ref/run9b.c:437-443).  Read the borrowed image on the host. */
int      mv4i_get_widx(const mv4i_file *f, int r, int k);
uint16_t mv4i_get_scale(const mv4i_file *f, int r, int b);

/* ------------------------------------------------ device-resident layer */

/* A matrix in the stream layout, resident on one device:
 *   wq  row r, block b (32 nibbles, k even = low nibble) at r*w_pitch + 16*b
 *   sc  golden: uint15 scale of (r, b) at sc[r*s_pitch + b]
 *       g128  : fp16 scale of (r, g) at sc[r*s_pitch + g], g = k/128
 * w_pitch is a multiple of 16 bytes. */
typedef struct {
    const uint8_t *wq;
    const void    *sc;
    int64_t        w_pitch;       /* bytes between rows of wq            */
    int64_t        s_pitch;       /* elements between rows of sc         */
    int32_t        M, K;
    int32_t        w_exp, out_shift;          /* golden only               */
    int8_t         codebook[16];              /* golden only               */
    int32_t        kind;                      /* MV4I_KIND_*               */
    int32_t        device;
    void          *owned;                     /* library allocation or NULL */
} mv4i_dmat;

enum { MV4I_KIND_GOLDEN = 0, MV4I_KIND_G128 = 1 };

/* Scalar results of one job, written on the device by the last CTA of the
 * job.  err is 0 or a negative code from the list above. */
typedef struct {
    int32_t  y_exp;
    int32_t  ns;
    int32_t  sat_event;
    uint32_t sat_count;
    int32_t  err;
    int32_t  pad[3];
} mv4i_status;

/* Relayout f's image and upload it to `device`.  out->owned is set; release
 * with mv4i_dmat_free. */
int mv4i_dmat_upload(const mv4i_file *f, int device, mv4i_dmat *out);

/* Wrap caller-owned device arrays already in the g128 stream layout (the
 * benchmark format: signed INT4 two's-complement nibbles, row-major along K,
 * fp16 scale per 128 columns).  Nothing is allocated. */
int mv4i_dmat_wrap_g128(const uint8_t *d_wq, int64_t w_pitch, const uint16_t *d_scales,
                        int64_t s_pitch, int M, int K, int device, mv4i_dmat *out);

/* Wrap caller-owned device arrays already in the golden stream layout
 * (wq as above, uint15 scales [M][s_pitch] per 32-column block). */
int mv4i_dmat_wrap_golden(const uint8_t *d_wq, int64_t w_pitch, const uint16_t *d_scales,
                          int64_t s_pitch, int M, int K, int w_exp, int out_shift,
                          const int8_t codebook[16], int device, mv4i_dmat *out);

int mv4i_dmat_free(mv4i_dmat *m);

/* A view of rows [row0, row0+n) of a resident matrix (nothing is copied or
 * allocated; the view does not own memory).  A BFP job on the view is the
 * reference's row-window A job, ref/run9b.c:455-490 (RAW over the rows, then
 * the BFP scan over the window only): rows are independent, so computing only
 * the window's rows gives the same RAW values and the window's own ns. */
int mv4i_dmat_rows(const mv4i_dmat *m, int row0, int n, mv4i_dmat *view);

/* One matvec job.
 *   golden: x = int16 mantissas (x_exp, or *d_x_exp when non-NULL);
 *           y_data int32 (RAW, BFP), y_mant int16 (BFP), y_acc int64 (PARTIAL)
 *   g128  : x = fp16 [nvec][K]; y_f16 fp16 [nvec][M] and/or y_f32 fp32
 * n_rows / n_cols select rows [0,n_rows) and columns [0,n_cols) as the
 * reference does (columns past n_cols are masked).  nvec = activation
 * vectors processed against the same weights (1..8; golden requires 1). */
typedef struct {
    const mv4i_dmat *w;
    const void      *x;
    const int32_t   *d_x_exp;
    int32_t          x_exp;
    int32_t          n_rows, n_cols;
    int32_t          mode;            /* golden: MV4I_MODE_*; g128 ignores */
    int32_t          nvec;
    int64_t          x_stride;        /* elements between activation vectors */
    int64_t          y_stride;        /* elements between output vectors     */
    int32_t         *y_data;
    int16_t         *y_mant;
    int64_t         *y_acc;
    uint16_t        *y_f16;
    float           *y_f32;
    mv4i_status     *status;          /* device; may be NULL for g128        */
    int32_t          accum;           /* g128: y_f32[row] += result (residual
                                         add fused into the projection)     */
    int32_t          pad_;
} mv4i_job;

#define MV4I_MAX_JOBS 64

/* Device scratch a launch needs (per-job completion counters and maxima).
 * Must be zero-filled once before first use; every launch leaves it zeroed
 * again.  Launches that share one scratch buffer must not overlap in time. */
size_t mv4i_scratch_bytes(void);

/* Launch njobs (<= MV4I_MAX_JOBS) jobs as one kernel on `stream`.  All jobs
 * of one launch must have the same kind.  Returns after enqueueing; errors in
 * the data (contract violations) land in each job's status->err. */
int mv4i_launch(const mv4i_job *jobs, int njobs, void *d_scratch, void *stream);

/* Allocation-free form of mv4i_launch: the same jobs, the same results, but
 * the per-job completion counters (the only device scratch a launch needs)
 * live in a fixed array compiled into the library -- 16 bytes for each of
 * MV4I_NOALLOC_MAX_JOBS jobs, 1 KiB on every GPU that loads the library,
 * held until the process exits -- instead of in caller-provided memory.
 *
 * It exists for callers that cannot call cudaMalloc on their decode path: a
 * serving runtime that has already divided all of HBM between weights, KV
 * cache and recurrent state (and must not fail or fragment mid-stream), a
 * loop that cannot afford the device-wide synchronisation cudaMalloc may
 * imply while other streams are in flight, or a host in another language
 * that reaches this library through a bare C FFI and owns no device
 * allocator.  It calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * The first call on a device looks up the array's device address with that
 * device current (cudaGetSymbolAddress), so make that first call before any
 * stream capture.  The looked-up address is kept for the life of the
 * process: it does not survive cudaDeviceReset (or any other teardown of the
 * device's primary context), after which this entry point must not be called
 * in that process.  Each call clears the counters it uses on `stream`
 * (cudaMemsetAsync) before its kernel.  All calls on one device share the
 * array and it keeps the last call's contents, so calls that overlap on the
 * GPU (other streams, other host threads) race.  More than
 * MV4I_NOALLOC_MAX_JOBS jobs is refused with -14.  No counterpart in the
 * reference, whose golden model allocates nothing on the device. */
#define MV4I_NOALLOC_MAX_JOBS 64
int mv4i_launch_noalloc(const mv4i_job *jobs, int njobs, void *stream);

/* Host-buffer form of a g128 launch, the end-to-end call: copies count
 * activation vectors h_x[count][K] (fp16) in, runs count jobs over the
 * resident matrices w[0..count-1] (all M x K), copies h_y[count][M] (fp16)
 * out and synchronises.  Staging lives in a per-device library buffer;
 * pinned host arrays make the copies asynchronous DMA.  No counterpart in
 * the reference, whose weights never leave the card (the host-side analogue
 * of ref/run9b.c:455-490 issuing one A job per projection). */
int mv4i_g128_matvec_host(const mv4i_dmat *w, int count, const uint16_t *h_x, uint16_t *h_y,
                          void *stream);

/* -------------------------------------------- tensor-parallel reduction */

/* E 2.1 (docs/superpowers/specs/2026-08-21-tp-collective-design.md:76-103):
 * given the N shards' unrounded s48 partials (PARTIAL mode) on per-shard
 * grids, min-align by floor, sum in int64, round by out_shift, sat32, and
 * BFP-pack.  parts is a device array of N*n_rows int64 (shard-major),
 * y_exps/out_shifts device arrays of N int32.  Writes out_mant (int16) and
 * status (y_exp = out_exp, ns, sat_event; err -12 / -13 on refusal).  The
 * collective that gathers the shards is the caller's (NCCL all-gather). */
int mv4i_tp_reduce(int N, int n_rows, const int64_t *d_parts, const int32_t *d_y_exps,
                   const int32_t *d_out_shifts, int16_t *d_out_mant, int32_t *d_y32,
                   mv4i_status *d_status, void *stream);

/* --------------------------------------------------------- weight packing */

/* The offline weight path of tools/pack_int4.py, as library calls (host
 * memory, no device needed):
 *   mv4i_quantize            quantize() (:280-359, spec 6.1): float W [M][K]
 *                            -> idx [M][NB][32] codebook indices, scale
 *                            [M][NB] uint15 (Q15), w_exp; the per-block scale
 *                            is the least-squares best of 8 candidates around
 *                            the amax-anchored one.  The codebook must be
 *                            ascending (IQ4_NL is); -11 otherwise.  Same bytes
 *                            as the reference's quantiser.
 *   mv4i_calibrate_out_shift calibrate_out_shift() (:434-446, spec 7.4): the
 *                            out_shift for which sat32 cannot fire
 *   mv4i_pack_size           the image size (packed_layout(), :451-486), 0
 *                            for a geometry the reference refuses
 *   mv4i_pack                pack() (:488-559, spec 6.4 / 6.5a): the .mv4i
 *                            image, byte-identical to the reference's
 *   mv4i_image_to_g128       an image the g128 format holds exactly (linear
 *                            codebook {0..7,-8..-1}, K % 128 == 0, equal
 *                            scales in each 128-column group, scales exact
 *                            in fp16) -> INT4 nibbles [M][K/2] and fp16
 *                            scales [M][sc_pitch]; -11 when not exact.  No
 *                            counterpart in the reference (the decode
 *                            engine's layout, see dec_load_linear). */
int    mv4i_quantize(const float *W, int M, int K, const int8_t cb[16], uint8_t *idx, uint16_t *scale,
                     int *w_exp);
int    mv4i_calibrate_out_shift(int K);
size_t mv4i_pack_size(int M, int K, int rows_if, int axi_dw);
int    mv4i_pack(const uint8_t *idx, const uint16_t *scale, int w_exp, int M, int K, int rows_if, int out_shift,
                 const int8_t cb[16], int axi_dw, uint8_t *out);
int    mv4i_image_to_g128(const mv4i_file *f, uint8_t *wq, uint16_t *sc, int sc_pitch);

/* A float matrix W [M][K] (K % 128 == 0) straight to the g128 layout: per row
 * and 128-column group, scale = fp16(max|w| / 7) (round to nearest even),
 * q = clamp(rint(w / scale), -8, 7) as two's-complement nibbles (column k even
 * in the low nibble).  -11 when a scale overflows fp16.  No counterpart in the
 * reference (the benchmark's format, not the .mv4i one). */
int    mv4i_quantize_g128(const float *W, int M, int K, uint8_t *wq, uint16_t *sc, int sc_pitch);

/* ------------------------------------------- tensor-parallel collective */

/* The transport of E (tp-collective-design.md:153-180): the message one rank
 * sends every peer for one row-parallel block -- its n_rows unrounded s48
 * partials in 64-bit slots, then a trailer of its y_exp, its out_shift and
 * the collective's SEQUENCE number, the sequence word stored last.  The
 * receiver accepts a message only when its sequence number is the one it
 * expects for this collective: a message left from collective k read as
 * collective k+1 is refused (-15), not summed.  Refusals (all ranks alike):
 *   -15  a message carries another collective's sequence number
 *   -12  y_exp spread > 17          -13  out_shift differs between ranks */
typedef struct {
    int32_t  y_exp;
    int32_t  out_shift;
    uint32_t seq;
    uint32_t pad_;
} mv4i_tp_trailer;

/* bytes of one message: 8 * n_rows, padded to 16, plus the 16-byte trailer */
size_t mv4i_tp_msg_bytes(int n_rows);

/* Host memory: write one message (payload, then trailer, sequence last), and
 * check N received messages for collective `seq` (their trailers into
 * y_exps / out_shifts, either may be NULL).  Returns 0, -11, -15, -12, -13. */
int mv4i_tp_msg_pack(const int64_t *y_acc, int n_rows, int y_exp, int out_shift, uint32_t seq, void *msg);
int mv4i_tp_msgs_check(int N, int n_rows, const void *const *msgs, uint32_t seq, int32_t *y_exps,
                       int32_t *out_shifts);

/* Device memory: the same message written by a kernel (y_exp read from the
 * PARTIAL job's device status when d_part_status is non-NULL, else y_exp),
 * and the E 2.1 reduction of N messages stored msg_bytes apart in d_msgs,
 * with the sequence / spread / out_shift checks done on the device
 * (d_status->err = -15 / -12 / -13, outputs untouched). */
int mv4i_tp_msg_pack_dev(const int64_t *d_y_acc, int n_rows, const mv4i_status *d_part_status, int y_exp,
                         int out_shift, uint32_t seq, void *d_msg, void *stream);
int mv4i_tp_reduce_msgs(int N, int n_rows, const void *d_msgs, uint32_t seq, int16_t *d_out_mant, int32_t *d_y32,
                        mv4i_status *d_status, void *stream);

/* One row-parallel golden block between the ranks of an NCCL communicator
 * (one process per GPU): pack this rank's message, all-gather the messages
 * (ncclAllGather), reduce them identically on every rank.  d_work holds
 * (world + 1) * mv4i_tp_msg_bytes(n_rows) bytes.  seq must advance by one per
 * collective and be the same on every rank.  The communicator comes from
 * mv4i_tp_comm_create with the 128 bytes rank 0 got from mv4i_tp_unique_id
 * (shipped to the other ranks by any transport).  Row-parallel g128 blocks
 * sum their fp32 partials with mv4i_tp_allreduce_f32. */
int mv4i_tp_unique_id(uint8_t id[128]);
int mv4i_tp_comm_create(const uint8_t id[128], int rank, int world, int device, void **comm);
int mv4i_tp_comm_destroy(void *comm);
int mv4i_tp_row_parallel(void *comm, const int64_t *d_y_acc, int n_rows, const mv4i_status *d_part_status,
                         int out_shift, uint32_t seq, void *d_work, int16_t *d_out_mant, int32_t *d_y32,
                         mv4i_status *d_status, void *stream);
int mv4i_tp_allreduce_f32(void *comm, float *d_y, int n, void *stream);

/* ------------------------------------------------- activation BFP pack */

/* Replaces reg_put, ref/run9b.c:343-359 (value -> BFP16, the producer of every
 * matvec's x): per vector, exp = 14 - floor(log2 max|v|) (0 for an all-zero
 * vector), mant = sat16(floor(v * 2^exp + 0.5)).  count vectors of n values,
 * vector i at d_v + i*stride elements; dtype 0 = fp16, 1 = fp32.  Outputs
 * d_mant[count][n] (int16, stride n) and d_exp[count] (int32).  Bit-exact
 * with the double-precision rule for fp16 and fp32 inputs. */
int mv4i_bfp_pack(const void *d_v, int dtype, int n, int count, int64_t stride,
                  int16_t *d_mant, int32_t *d_exp, void *stream);

/* ------------------------------------------------------------- argmax */

/* Replaces argmax_first (ref/run9b.c:399-405): index of the largest of n
 * values, the FIRST one on ties.  dtype 0 = int32 (golden RAW logits on one
 * grid), 1 = fp32, 2 = fp16.  d_work is 8 bytes of device scratch; *d_idx
 * receives the index.  Two kernels on `stream`. */
int mv4i_argmax(const void *d_v, int dtype, int n, uint64_t *d_work, int32_t *d_idx, void *stream);

/* ----------------------------------------------------------- utilities */

/* Seeded synthetic inputs for the benchmark shape (splitmix64, counter
 * form: draw i of seed s = mix(s + (i+1)*0x9E3779B97F4A7C15)).  Fills the
 * g128 layout on the device: W uniform over [-8,7], scales uniform in
 * [0.002,0.02] rounded to fp16, x ~ N(0,1) (Box-Muller) rounded to fp16.
 * count matrices of M x K back to back (matrix i uses seed + i).  Any
 * pointer may be NULL to skip it. */
int mv4i_synth_g128(uint64_t seed, int count, int M, int K, uint8_t *d_wq,
                    uint16_t *d_scales, uint16_t *d_x, void *stream);

int  mv4i_last_cuda_error(void);
const char *mv4i_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MV4I_B200_H */
