// llm.vhdl_b200/csrc/dec_step.cu -- the decode library's CUDA code as one
// translation unit (the kernels of dec_kernels.cu, dec_matvec.cu and the
// DeltaNet step of gdn_f32_step.cuh are compiled here), and the persistent
// decode kernel.
//
// The persistent kernel runs a whole decode step in one launch.  It executes
// a program of stages (mg_stage, dec_internal.h) -- the counterpart of the
// reference's per-token layer program that its sequencer walks
// (ref/run9b.c:1028-1170 composes the same A jobs and delta rule on the host)
// -- with every CTA taking its share of each stage and a grid-wide barrier
// after each stage whose output the next one reads.  A step thus costs one
// launch instead of five or six per layer, and the weights of the next
// projection are prefetched into L2 while the current stage runs and while
// CTAs wait at barriers: weights never depend on activations, so the HBM
// stream keeps going across stage boundaries.
//
// Barriers: one 64-bit arrival counter in device memory, never reset; the
// k-th barrier of a launch waits for base + k * grid arrivals, where base is
// the count at launch rounded down to a whole number of steps (every launch
// of a program passes the same number of barriers, and no CTA can finish the
// first barrier of a launch before every CTA read the count).  Each wait is
// bounded in time: a barrier that does not complete within timeout_ns sets
// the abort flag, records the stage, and every CTA leaves at its next
// barrier; later launches leave at once until the host clears the flag
// (dec_status).  The grid is the number of CTAs that fit on the device at
// once, launched cooperatively, so all of them are resident.
//
// Measured on B200 (grid 296): a barrier costs about 2.4 us whether arrival
// is a returning atomic or a release reduction -- about what a programmatic
// dependent launch costs -- so this mode is not faster than one launch per
// stage for the benchmark's shapes, and is off by default.

#include "dec_kernels.cu"
#include "dec_matvec.cu"
#include "gdn_f32_step.cuh"

__device__ __forceinline__ unsigned long long mg_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long mg_ld_acquire(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long mg_ld_relaxed(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// every thread of the CTA calls it; returns false when the step is aborted.
// Arrival is a fire-and-forget release reduction (no round trip); the wait
// polls with relaxed loads and takes one acquire fence once the count is in.
__device__ __forceinline__ bool mg_barrier(mg_ctl *ctl, unsigned long long target, long long timeout_ns, int stage,
                                          int *s_ok)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" :: "l"(&ctl->count) : "memory");
        const unsigned long long t0 = mg_now();
        int ok = 1;
        for (unsigned it = 0;; it++) {
            if (mg_ld_relaxed(&ctl->count) >= target) break;
            if ((it & 31) == 31 && *(volatile int32_t *)&ctl->abort) { ok = 0; break; }
            if ((long long)(mg_now() - t0) > timeout_ns) {
                ctl->err_stage = stage;
                atomicExch(&ctl->abort, 1);
                ok = 0;
                break;
            }
        }
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

#define MG_COMBINE_SMEM (2 * (1024 + 32) * 4)

// The stages other than the projections run out of line, so that their
// register needs do not crowd the matvec stream that is inlined in the kernel.
__device__ __noinline__ void mg_gdn_piece(const gdn_f32_args &A, int bx, int by, int tid)
{
    gdn_f32_cta<true>(A, bx, by, tid);
}
__device__ __noinline__ void mg_attn_piece(const dec_attn_args &A, int c, int g, int b, uint8_t *sm)
{
    dec_attn_cta(A, c, g, b, threadIdx.x, blockDim.x, sm);
}
__device__ __noinline__ void mg_combine_piece(const dec_attn_args &A, int h, int b, float *wc)
{
    dec_attn_combine_cta<4>(A, h, b, threadIdx.x & 127, wc);
}

template <int NV>
__global__ void __launch_bounds__(DMV_THREADS, DMV_MINB) dec_mega_kernel(const __grid_constant__ mg_prog P)
{
    extern __shared__ __align__(128) uint8_t mg_sm[];
    __shared__ __align__(16) mg_stage st;
    __shared__ int s_ok;
    __shared__ unsigned long long s_base;
    const mg_stage *prog = P.d_prog;
    if (threadIdx.x == 0) {
        s_ok = !*(volatile int32_t *)&P.ctl->abort;
        const unsigned long long c = mg_ld_acquire(&P.ctl->count);
        const unsigned long long per = (unsigned long long)P.nbar * gridDim.x;
        s_base = per ? c - c % per : c;
        if (P.clock && blockIdx.x == 0) P.clock[0] = mg_now();
    }
    __syncthreads();
    if (!s_ok) return;
    int k = 0;
    for (int i = 0; i < P.n; i++) {
        {
            const uint4 *src = reinterpret_cast<const uint4 *>(prog + i);
            uint4 *dst = reinterpret_cast<uint4 *>(&st);
            for (int w = threadIdx.x; w < (int)(sizeof(mg_stage) / 16); w += blockDim.x) dst[w] = src[w];
        }
        __syncthreads();
        // the next projection's weights (this CTA's share) into L2 now
        if (threadIdx.x == 0 && st.pf >= 0 && P.pf_bytes > 0) {
            const dmv_params &N = prog[st.pf].u.mv;
            const int T = N.total_tiles;
            const int t0 = (int)((int64_t)blockIdx.x * T / gridDim.x);
            const int t1 = (int)((int64_t)(blockIdx.x + 1) * T / gridDim.x);
            dmv_prefetch(N, N.jobs, t0, t1, P.pf_bytes, NV > 1, DMV_WARPS);
        }
        switch (st.op) {
        case MG_MATVEC:
            dmv_body<NV, DMV_WARPS, false>(st.u.mv, mg_sm, blockIdx.x, gridDim.x, false);
            break;
        case MG_GDN: {
            // pieces of 128 threads (16 value columns of a head), two per CTA
            const int per = st.u.gdn.H * 8, nb = per * (st.u.gdn.nseq > 1 ? st.u.gdn.nseq : 1);
            const int half = threadIdx.x >> 7;
            for (int v = 2 * blockIdx.x + half; v < nb; v += 2 * gridDim.x)
                mg_gdn_piece(st.u.gdn, v % per, v / per, threadIdx.x & 127);
            break;
        }
        case MG_ATTN: {
            const dec_attn_args &A = st.u.att;
            const int len = min(*A.d_pos + 1, A.max_ctx), used = (len + A.ch - 1) / A.ch;
            const int nb = used * A.kvh * A.nseq;
            for (int v = blockIdx.x; v < nb; v += gridDim.x) {
                const int c = v % used, g = (v / used) % A.kvh, b = v / (used * A.kvh);
                mg_attn_piece(A, c, g, b, mg_sm);
                __syncthreads();                               // shared memory reused
            }
            break;
        }
        case MG_COMBINE: {
            // pieces of 128 threads (one q head of one sequence), two per CTA;
            // a half past the end repeats the last piece (same values)
            const dec_attn_args &A = st.u.att;
            const int half = threadIdx.x >> 7, nb = A.qh * A.nseq;
            float *wc = reinterpret_cast<float *>(mg_sm) + half * (1024 + 32);
            for (int v = 2 * blockIdx.x; v < nb; v += 2 * gridDim.x) {
                const int vb = min(v + half, nb - 1);
                mg_combine_piece(A, vb % A.qh, vb / A.qh, wc);
                __syncthreads();
            }
            break;
        }
        case MG_EMBED: {
            const mg_embed_args &e = st.u.emb;
            dec_embed_range(e.emb, e.hidden, e.tok, e.x, e.nseq, blockIdx.x * blockDim.x + threadIdx.x,
                            gridDim.x * blockDim.x);
            break;
        }
        case MG_COPY: {
            const mg_copy_args &c = st.u.cp;
            for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < c.n; j += (int64_t)gridDim.x * blockDim.x)
                c.dst[j] = c.src[j];
            break;
        }
        case MG_ADVANCE:
            if (blockIdx.x == 0) {
                const mg_advance_args &a = st.u.adv;
                dec_advance_cta(a.keys, a.n, a.key, a.tok, a.hist, a.pos, a.max_ctx, a.prompt, threadIdx.x, a.nseq);
            }
            break;
        default:
            break;
        }
        if (st.sync) {
            k++;
            if (!mg_barrier(P.ctl, s_base + (unsigned long long)k * gridDim.x, P.timeout_ns, i, &s_ok)) return;
            if (P.clock && blockIdx.x == 0 && threadIdx.x == 0) P.clock[k] = mg_now();
        } else {
            __syncthreads();                                   // st is rewritten next
        }
    }
}

static const void *mega_fn(int nv)
{
    return nv == 1 ? (const void *)dec_mega_kernel<1> : nv == 2 ? (const void *)dec_mega_kernel<2>
         : nv == 4 ? (const void *)dec_mega_kernel<4> : (const void *)dec_mega_kernel<8>;
}

extern "C" int dec_mega_upload(mg_stage *S, int n, int nvec, mg_prog *P)
{
    if (!S || !P || n < 1 || nvec < 1 || nvec > 8) return -11;
    const int NV = nvec == 1 ? 1 : nvec == 2 ? 2 : nvec <= 4 ? 4 : 8;
    const void *fn = mega_fn(NV);
    int dev = 0, sms = 0, occ = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    size_t smem = MG_COMBINE_SMEM;
    for (int i = 0; i < n; i++) {
        if (S[i].op == MG_MATVEC) {
            const size_t b = (size_t)NV * dmv_smem_x_bytes(S[i].u.mv.K);
            if (S[i].u.mv.nvec > 1 && S[i].u.mv.nvec != nvec) return -11;
            smem = b > smem ? b : smem;
        } else if (S[i].op == MG_ATTN || S[i].op == MG_COMBINE) {
            const int rc = dec_attn_prepare(&S[i].u.att);
            if (rc) return rc;
            if (S[i].u.att.nseq > 1 && S[i].u.att.nseq != nvec) return -11;
            const size_t b = dec_attention_smem(S[i].u.att.qh, S[i].u.att.kvh, S[i].u.att.ch);
            smem = b > smem ? b : smem;
            if (S[i].u.att.qh / S[i].u.att.kvh > DMV_WARPS) return -11;     // one warp per q head of a group
        } else if (S[i].op == MG_GDN) {
            if (S[i].u.gdn.T != 1 || S[i].u.gdn.D != 128) return -11;
        } else if (S[i].op == MG_ADVANCE) {
            if (S[i].u.adv.nseq > DMV_THREADS) return -11;
        } else if (S[i].op != MG_EMBED && S[i].op != MG_COPY) {
            return -11;
        }
    }
    if (smem > 200 * 1024) return -11;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, DMV_THREADS, smem);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    if (occ < 1) return -11;
    const int grid = sms * occ;
    int nbar = 0, done = -1;
    for (int i = 0; i < n; i++) {
        if (S[i].op == MG_MATVEC) {
            const long long rc = dmv_prepare(S[i].u.mv, grid, DMV_WARPS);
            if (rc < 0) return (int)rc;
        }
        nbar += S[i].sync ? 1 : 0;
    }
    // prefetch plan: stage i asks for the first projection after it, unless
    // an earlier stage already did
    for (int i = 0; i < n; i++) {
        int j = i + 1;
        while (j < n && S[j].op != MG_MATVEC) j++;
        S[i].pf = -1;
        if (j < n && j != done) { S[i].pf = j; done = j; }
    }
    if (P->d_prog && P->n != n) return -11;
    if (!P->d_prog) {
        e = cudaMalloc((void **)&P->d_prog, sizeof(mg_stage) * (size_t)n);
        if (e != cudaSuccess) { P->d_prog = NULL; mv4i_g_cuda_err = (int)e; return -20; }
    }
    if (!P->ctl) {
        e = cudaMalloc((void **)&P->ctl, sizeof(mg_ctl));
        if (e == cudaSuccess) e = cudaMemset(P->ctl, 0, sizeof(mg_ctl));
        if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    }
    // a new program may pass a different number of barriers: restart the count
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(P->d_prog, S, sizeof(mg_stage) * (size_t)n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(P->ctl, 0, sizeof(mg_ctl));
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    P->n = n; P->nbar = nbar; P->grid = grid; P->nv = NV; P->smem = (int64_t)smem;
    if (P->timeout_ns <= 0) P->timeout_ns = 1000000000LL;
    if (P->pf_bytes <= 0) P->pf_bytes = 192 * 1024;
    return 0;
}

extern "C" int dec_k_mega(const mg_prog *P, void *stream)
{
    if (!P || !P->d_prog || !P->ctl || P->grid < 1) return -11;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P->grid);
    cfg.blockDim = dim3(DMV_THREADS);
    cfg.dynamicSmemBytes = (size_t)P->smem;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {const_cast<mg_prog *>(P)};
    const cudaError_t e = cudaLaunchKernelExC(&cfg, mega_fn(P->nv), args);
    if (e != cudaSuccess) { mv4i_g_cuda_err = (int)e; return -20; }
    return 0;
}
