// frame_fused.cuh — the batch-1 codec frame as two clustered kernels per layer.
//
// A frame is a chain of dependent steps (every projection needs the whole
// output vector of the step before it).  On B200 a dependent kernel launch
// costs ~2.5 us and a grid barrier ~1.3 us, while a barrier across a 16-CTA
// thread-block cluster costs ~0.27 us.  So each transformer layer of the talker
// step and of the code-predictor passes runs as two launches whose inner
// hand-offs stay inside clusters:
//
//   k_ff_attn  one cluster per kv group (8-16 CTAs): the layer input (a partial
//              sum, or a sampled codebook's embedding row), RMSNorm, the
//              group's q|k|v rows, per-head q/k norm + RoPE + KV append +
//              attention, then the group's share of the O-projection: a
//              partial output vector over the group's G x 128 columns.
//   k_ff_ffn   clusters of up to 16 CTAs: layer input + the kv groups' O
//              partials (the residual stream after attention), RMSNorm, a
//              slice of gate/up rows, SwiGLU, and that slice's share of
//              ffn_down; the cluster sums its CTAs' partials over distributed
//              shared memory and writes one partial vector per cluster.
//
// The consumer of partial vectors sums them in a fixed order (partial 0, then
// 1, ...) and then adds the residual, so results do not depend on timing.  The
// samplers run inside the next layer's prologue (every CTA draws the same token
// from the same logits), the heads stay GEMVs over all SMs (k_ff_head), and the
// codec head also advances the frame state.  A frame is 15 code-predictor passes
// x (5 layers x 2 + head) + 28 talker layers x 2 + head = 222 launches (548 as
// one launch per op).
//
// Reduction orders (restated by the CPU oracle's "split" frame mode):
//   q|k|v rows, gate/up rows, heads: the GEMV order of gemv_compute;
//   O-projection of group g: gemv_compute over columns [g G 128, (g+1) G 128);
//     out = ((P_0 + P_1) + ... + P_{NKV-1}) + x;
//   ffn_down, F16 (weight cast to F32, activation F32): CTA s owns rows
//     [s R, s R + R) of the intermediate vector and chains
//     fmaf(W[r][j], h[j], acc) over them in order; the cluster adds its CTAs'
//     partials in rank order, the consumer the clusters' in order, then x;
//   ffn_down, Q8_0: CTA s owns 32-block s: (float) isum x (d_w x d_a), then
//     the same two-level order.
#pragma once
#include "kernels.cuh"

namespace qtts {

constexpr int FF_THREADS = QTTS_WARPS * 32;   // 512: gemv_compute's block size
constexpr int FF_MAX_PF = 6;                  // weight regions prefetched into L2 per launch
constexpr int FF_MAX_CLUSTER = 16;

// How a clustered kernel builds its activation rows.
enum FfInMode : int {
    FIN_PART = 0,     // x[v] = (((p_0[v] + p_1[v]) + ...) + p_{np-1}[v]) + base[v]
    FIN_CB0 = 1,      // sample codebook 0 (talker logits); rows [talker hidden, codec_embd[cb0]]
    FIN_CBG = 2,      // sample code-predictor codebook cb; row cp_embd[cb - 1][code]
    FIN_TALKER = 3,   // sample the last codebook; row = the next talker step's input sum
};

// Frame-wide pointers shared by the launches of a frame.
struct FfFrame {
    DevState * st;
    int * err;                           // set to 3 when a bounded wait gave up
    const SampleParams * sp;
    int * out_codes;
    int out_cap;
    const __half * codec_embd;           // [V0][H]
    const __half * const * cp_embd;      // device array of n_cb - 1 tables [V1][H]
    const float * hidden;                // talker post-norm hidden state [H]
    const float * trailing, * pad;       // trailing text rows [n_trailing][H], tts_pad row [H]
    int H, n_cb, V0, V1;
    float eps;
    unsigned long long * trace;          // optional: [n_launches][FF_TRACE_CTAS][FF_TRACE_N] %globaltimer
    int trace_frame;                     // the frame whose launches are traced
};

// Trace stamps of a launch, per CTA (diagnostics, QTTS_FF_TRACE=1): start,
// dependency wait returned, input built, first GEMV done, first cluster
// barrier passed, attention / ffn_down partial done, second cluster barrier
// passed, end.
constexpr int FF_TRACE_N = 8;
constexpr int FF_TRACE_CTAS = 256;

struct FfInput {
    int mode, cb, np;
    const float * base;                  // FIN_PART: [nv][H]
    const float * part;                  // FIN_PART: [np][nv][H]
    const float * logits;                // sampler modes: the logits to sample from
    float * x_out;                       // the layer input as built, [nv][H] (CTA 0 writes it)
};

// L2 prefetch of weights a later launch reads (split evenly over the CTAs).
struct FfPrefetch {
    const void * p[FF_MAX_PF];
    unsigned long long bytes[FF_MAX_PF];
    int n;
};

struct FfAttnArgs {
    FfFrame fr;
    int launch_id;                       // index of the launch in the frame (trace row)
    FfInput in;
    int nv;                              // rows: 2 for the code-predictor prefill pass, else 1
    DMat qkv;                            // group-major q|k|v: [NKV][(G + 2) 128 rows][H]
    const float * attn_norm;
    DMat o;                              // group-major O: [NKV][H rows][G 128 cols]
    float * qkv_buf;                     // [nv][QD + 2 KD] (standard q | k | v layout)
    float * att_buf;                     // [nv][QD]
    float * part_out;                    // [NKV][nv][H]: the groups' O-projection partials
    FusedAttn att;                       // attention of the layer (qkv = qkv_buf, out = att_buf)
    int att_kind;                        // FF_ATT_UNIT (fused unit) or FF_ATT_CPSTEP (warp per head)
    int n_past;                          // code-predictor position (talker: DevState pos)
    int work_bytes;                      // shared-memory work area (GEMV rows / attention scratch)
    FfPrefetch pf;
};
enum FfAttKind : int { FF_ATT_UNIT = 0, FF_ATT_CPSTEP = 1 };

struct FfFfnArgs {
    FfFrame fr;
    int launch_id;
    FfInput in;
    int nv;
    DMat gate, up;                       // row slices of R rows per CTA
    const float * ffn_norm;
    DMat down;                           // F16: transposed [I][H]; Q8_0: int8 [I/32][H][32], scales [I/32][H]
    int R;                               // intermediate rows per CTA
    float * part_out;                    // [n_clusters][nv][H]
    int set_presence;                    // CTA 0 adds codes[0] to the codebook-0 presence set
    int work_bytes;
    FfPrefetch pf;
};

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ unsigned ff_cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned ff_cluster_id() {
    unsigned r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void ff_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A peer CTA's shared-memory address (same offset) for ld.shared::cluster.
__device__ __forceinline__ uint32_t ff_peer_addr(const void * p, unsigned rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// (no memory clobber: callers read peers only after a cluster barrier, and the
// loads of one reduction must all be in flight before the first add)
__device__ __forceinline__ float ff_ld_peer(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

constexpr int FF_MAX_PART = 16;   // partial vectors a consumer sums (kv groups, FFN clusters)

// x = (((p_0 + p_1) + ...) + p_{np-1}) + base at element e: every load is issued
// before the first add (np <= FF_MAX_PART).
__device__ __forceinline__ float ff_part_sum(const float * part, const float * base, int np, size_t pstride,
                                             size_t e) {
    float pv[FF_MAX_PART];
#pragma unroll
    for (int p = 0; p < FF_MAX_PART; ++p) pv[p] = p < np ? __ldcg(part + (size_t) p * pstride + e) : 0.0f;
    const float b = __ldcg(base + e);
    float acc = pv[0];
#pragma unroll
    for (int p = 1; p < FF_MAX_PART; ++p)
        if (p < np) acc = __fadd_rn(acc, pv[p]);
    return __fadd_rn(acc, b);
}

__device__ __forceinline__ unsigned long long ff_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Stamp k of this CTA in launch `id` when tracing this frame (thread 0).
__device__ __forceinline__ void ff_stamp(const FfFrame & fr, int id, int frame, int k) {
    if (fr.trace && frame == fr.trace_frame && threadIdx.x == 0 && blockIdx.x < FF_TRACE_CTAS)
        fr.trace[((size_t) id * FF_TRACE_CTAS + blockIdx.x) * FF_TRACE_N + k] = ff_now();
}

__device__ __forceinline__ void ff_prefetch(const FfPrefetch & pf) {
    if (threadIdx.x != 0) return;
    for (int i = 0; i < pf.n; ++i) {
        const unsigned long long share = ((pf.bytes[i] + gridDim.x - 1) / gridDim.x + 255) & ~255ull;
        const unsigned long long off = share * blockIdx.x;
        if (off >= pf.bytes[i]) continue;
        unsigned long long n = pf.bytes[i] - off < share ? pf.bytes[i] - off : share;
        const char * c = static_cast<const char *>(pf.p[i]) + off;
        while (n > 0) {
            const unsigned k = (unsigned)(n > 65536 ? 65536 : n);
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(k) : "memory");
            c += k;
            n -= k;
        }
    }
}

// Group block g of a group-major matrix (rows_g rows each).
__device__ __forceinline__ DMat ff_block(const DMat & M, int g, int rows_g, int cols) {
    DMat b = M;
    b.rows = rows_g;
    b.cols = cols;
    const size_t es = M.type == W_Q8_0 ? 1 : 2;
    b.w = static_cast<const char *>(M.w) + (size_t) g * rows_g * cols * es;
    if (M.type == W_Q8_0) b.d = M.d + (size_t) g * rows_g * (cols / 32);
    return b;
}

// Records a sampled token (CTA 0, thread 0).  Codebook 0's presence bit is set
// later (k_ff_ffn) because every CTA of this launch reads the presence set.
__device__ __forceinline__ void ff_commit(int tok, int cb, const FfFrame & fr, const SampleParams & P, int frame) {
    if (cb == 0 && tok == P.eos_id) {
        fr.st->done = 1;
        return;
    }
    fr.st->codes[cb] = tok;
    if (fr.out_codes && frame < fr.out_cap) fr.out_codes[(size_t) frame * P.n_cb + cb] = tok;
}

// Builds the activation rows in the two-plane layout (xs, nv rows of H).
// Returns 1 when codebook 0 sampled EOS (the launch has nothing to do).
template <int NV>
__device__ int ff_build_input(const FfFrame & fr, const FfInput & in, float * xs) {
    __shared__ int s_codes[QTTS_MAX_CB];
    __shared__ const __half * s_tabs[QTTS_MAX_CB];
    __shared__ SampleParams s_sp;
    const int tid = threadIdx.x, nt = blockDim.x, H = fr.H;
    const bool writer = blockIdx.x == 0;
    if (in.mode == FIN_PART) {
        for (int c = tid; c < H; c += nt) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const float x = ff_part_sum(in.part, in.base, in.np, (size_t) NV * H, (size_t) v * H + c);
                xs[v * H + xpos(c, H)] = x;
                if (writer && in.x_out) in.x_out[(size_t) v * H + c] = x;
            }
        }
        return 0;
    }
    // sampler modes
    const DevState * st = fr.st;
    const int frame = st->frame, n_tr = st->n_trailing;
    if (tid == 0) {
        s_sp = *fr.sp;
        if (!writer) s_sp.record_logits = 0;   // CTA 0 records the debug logits
    }
    if (tid < QTTS_MAX_CB) {
        s_codes[tid] = tid < in.cb ? st->codes[tid] : 0;
        s_tabs[tid] = tid >= 1 && tid < fr.n_cb ? fr.cp_embd[tid - 1] : nullptr;
    }
    __syncthreads();
    const int cb = in.cb, V = cb == 0 ? fr.V0 : fr.V1;
    const float * lg = in.logits;
    const int tok = sample_body_l<8>(
        [&](float * l) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int i = tid * 8 + e;
                l[e] = i < V ? __ldcg(lg + i) : -INFINITY;
            }
        },
        V, cb, st, s_sp, frame);
    if (cb == 0 && tok == s_sp.eos_id) {
        if (writer && tid == 0) ff_commit(tok, cb, fr, s_sp, frame);
        return 1;
    }
    if (writer && tid == 0) ff_commit(tok, cb, fr, s_sp, frame);
    if (tid == 0) s_codes[cb] = tok;
    __syncthreads();
    for (int c = tid; c < H; c += nt) {
        float x0, x1 = 0.0f;
        if (in.mode == FIN_CB0) {
            x0 = __ldcg(fr.hidden + c);
            x1 = __half2float(fr.codec_embd[(size_t) tok * H + c]);
        } else if (in.mode == FIN_CBG) {
            x0 = __half2float(s_tabs[cb][(size_t) tok * H + c]);
        } else {   // the same sums, in the same order, as frame_inputs_body
            float s = __half2float(fr.codec_embd[(size_t) s_codes[0] * H + c]);
            for (int q = 1; q < fr.n_cb; ++q) s = __fadd_rn(s, __half2float(s_tabs[q][(size_t) s_codes[q] * H + c]));
            const float t = frame < n_tr ? fr.trailing[(size_t) frame * H + c] : fr.pad[c];
            x0 = __fadd_rn(s, t);
        }
        xs[xpos(c, H)] = x0;
        if (NV == 2) xs[H + xpos(c, H)] = x1;
        if (writer && in.x_out) {
            in.x_out[c] = x0;
            if (NV == 2) in.x_out[H + c] = x1;
        }
    }
    return 0;
}

// q|k|v row r of group g's block -> its column in the standard q | k | v layout.
struct FfQkvStore {
    float * buf;
    int ld, g, G, QD, KD;
    __device__ __forceinline__ void operator()(int r, int, int v, float val) const {
        const int qrows = G * QTTS_HD;
        int col;
        if (r < qrows) col = g * qrows + r;
        else if (r < qrows + QTTS_HD) col = QD + g * QTTS_HD + (r - qrows);
        else col = QD + KD + g * QTTS_HD + (r - qrows - QTTS_HD);
        buf[(size_t) v * ld + col] = val;
    }
};
struct FfRowStore {   // plain [v][ld] store of output rows
    float * y;
    int ld;
    __device__ __forceinline__ void operator()(int r, int, int v, float val) const { y[(size_t) v * ld + r] = val; }
};
struct FfSmemStore {  // this CTA's rows into shared memory [v][ld] (local row index)
    float * y;
    int ld;
    __device__ __forceinline__ void operator()(int, int rl, int v, float val) const { y[v * ld + rl] = val; }
};

// Waits (bounded) for an mbarrier phase this CTA armed, so no bulk copy is in
// flight when the CTA leaves.
__device__ __forceinline__ void ff_drain(uint64_t * m, unsigned parity) {
    if (threadIdx.x == 0) mbar_wait(m, parity);
}

// ---------------------------------------------------------------- attention block
// Grid: NKV clusters of C CTAs (cluster g = kv group g).  Shared memory: one
// weight buffer (the q|k|v slice + attn_norm gain, later the O slice) and the
// work area (activation rows, then the attention scratch, then the O input).
template <int NV>
__global__ void __launch_bounds__(FF_THREADS, 2) k_ff_attn(const FfAttnArgs A) {
    extern __shared__ __align__(128) uint8_t ff_smem[];
    __shared__ __align__(8) uint64_t mbar[2];
    const int tid = threadIdx.x;
    const unsigned rank = ff_cluster_rank();
    const int g = (int) ff_cluster_id();
    unsigned C;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(C));
    const FfFrame & fr = A.fr;
    const int H = fr.H, NH = A.att.n_heads, NKV = A.att.n_kv_heads, G = NH / NKV;
    const int GD = G * QTTS_HD, rows_g = GD + 2 * QTTS_HD;
    const int QD = NH * QTTS_HD, KD = NKV * QTTS_HD;
    const DMat Qg = ff_block(A.qkv, g, rows_g, H);
    const DMat Og = ff_block(A.o, g, H, GD);
    uint8_t * wbuf = ff_smem;
    const size_t wbytes_q = (slice_layout(Qg, false, true, gemv_rpc(rows_g, C)).total + 127) & ~(size_t) 127;
    const size_t wbytes_o = (slice_layout(Og, false, false, gemv_rpc(H, C)).total + 127) & ~(size_t) 127;
    uint8_t * work = ff_smem + (wbytes_q > wbytes_o ? wbytes_q : wbytes_o);
    float * xs = reinterpret_cast<float *>(work);
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue_gemv_slice(Qg, DMat{}, A.attn_norm, wbuf, &mbar[0], (int) rank, (int) C);   // read-only weights
    }
    const unsigned long long t_start = ff_now();
    pdl_trigger();
    ff_prefetch(A.pf);
    __syncthreads();
    pdl_wait();
    const int dn = fr.st->done, pos = fr.st->pos, frame = fr.st->frame;
    if (fr.trace && frame == fr.trace_frame && tid == 0 && blockIdx.x < FF_TRACE_CTAS)
        fr.trace[((size_t) A.launch_id * FF_TRACE_CTAS + blockIdx.x) * FF_TRACE_N] = t_start;
    ff_stamp(fr, A.launch_id, frame, 1);
    if (dn) { ff_drain(&mbar[0], 0u); return; }
    if (ff_build_input<NV>(fr, A.in, xs) == 1) { ff_drain(&mbar[0], 0u); return; }
    __syncthreads();
    ff_stamp(fr, A.launch_id, frame, 2);
    GemvArgs ga{};
    ga.A = Qg;
    ga.nv = NV;
    ga.norm_g = A.attn_norm;
    ga.eps = fr.eps;
    ga.act = ACT_F16;
    ga.epi = EPI_STORE;
    bool ok = gemv_compute<NV>(ga, (int) rank, (int) C, wbuf, work, &mbar[0], 0u,
                               FfQkvStore{A.qkv_buf, QD + 2 * KD, g, G, QD, KD});
    __syncthreads();   // every warp is done with the q|k|v slice
    ff_stamp(fr, A.launch_id, frame, 3);
    if (tid == 0) {    // the O slice into the same buffer; it lands during the attention
        if (!ok) mbar_wait(&mbar[0], 0u);   // no q|k|v copy may still be writing the buffer
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_gemv_slice(Og, DMat{}, nullptr, wbuf, &mbar[1], (int) rank, (int) C);
    }
    ff_cluster_sync();   // the group's q|k|v rows are in qkv_buf
    ff_stamp(fr, A.launch_id, frame, 4);
    const FusedAttn & at = A.att;
    if (A.att_kind == FF_ATT_CPSTEP) {
        const int warp = tid >> 5;
        if (rank == 0 && warp < G) cp_step_attn_body(at, g * G + warp, A.n_past);
    } else if ((int) rank < G * NV) {
        const int i = (int) rank / G, hq = g * G + (int) rank % G;
        fused_attn_body(at, i * NH + hq, work, at.f32_mode ? A.n_past : pos, frame);
    }
    ff_stamp(fr, A.launch_id, frame, 5);
    ff_cluster_sync();   // the group's attention rows are in att_buf
    ff_stamp(fr, A.launch_id, frame, 6);
    for (int t = tid; t < NV * GD; t += blockDim.x) {
        const int v = t / GD, c = t - v * GD;
        xs[v * GD + xpos(c, GD)] = __ldcg(A.att_buf + (size_t) v * QD + (size_t) g * GD + c);
    }
    __syncthreads();
    GemvArgs go{};
    go.A = Og;
    go.nv = NV;
    go.eps = fr.eps;
    go.act = ACT_F16;
    go.epi = EPI_STORE;
    ok = gemv_compute<NV>(go, (int) rank, (int) C, wbuf, work, &mbar[1], 0u,
                          FfRowStore{A.part_out + (size_t) g * NV * H, H}) && ok;
    if (!ok) {
        ff_drain(&mbar[1], 0u);
        if (tid == 0) atomicExch(fr.err, 3);
    }
    ff_stamp(fr, A.launch_id, frame, 7);
}

// ---------------------------------------------------------------- FFN block
// Grid: N CTAs of R intermediate rows each, in clusters of C.  Shared memory:
// gate/up slice + ffn_norm gain | ffn_down slice | work area (activation rows,
// later this CTA's ffn_down partial) | SwiGLU rows.
__host__ __device__ inline size_t ff_down_slice_bytes(int type, int R, int H) {
    return type == W_Q8_0 ? (size_t) H * 32 + (size_t) H * 2 : (size_t) R * H * 2;
}

template <int NV>
__global__ void __launch_bounds__(FF_THREADS) k_ff_ffn(const FfFfnArgs A) {
    extern __shared__ __align__(128) uint8_t ff_smem[];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ int8_t s_qa[NV][32];
    __shared__ float s_da[NV];
    const int tid = threadIdx.x, nt = blockDim.x;
    const unsigned rank = ff_cluster_rank();
    const int cid = (int) ff_cluster_id();
    unsigned C;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(C));
    const FfFrame & fr = A.fr;
    const int H = fr.H, R = A.R, s = blockIdx.x;
    const bool q8 = A.down.type == W_Q8_0;
    const size_t wb_gu = (slice_layout(A.gate, true, true, R).total + 127) & ~(size_t) 127;
    const size_t wb_dn = (ff_down_slice_bytes(A.down.type, R, H) + 127) & ~(size_t) 127;
    uint8_t * wbuf = ff_smem;
    uint8_t * dbuf = ff_smem + wb_gu;
    uint8_t * work = dbuf + wb_dn;
    float * xs = reinterpret_cast<float *>(work);
    float * dpart = reinterpret_cast<float *>(work);   // after the gate/up GEMV
    float * hs = reinterpret_cast<float *>(work + A.work_bytes);
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue_gemv_slice(A.gate, A.up, A.ffn_norm, wbuf, &mbar[0], s, (int) gridDim.x);
        const unsigned dbytes = (unsigned) ff_down_slice_bytes(A.down.type, R, H);
        mbar_expect_tx(&mbar[1], dbytes);
        if (q8) {
            bulk_g2s(dbuf, static_cast<const int8_t *>(A.down.w) + (size_t) s * H * 32, (unsigned)(H * 32), &mbar[1]);
            bulk_g2s(dbuf + (size_t) H * 32, A.down.d + (size_t) s * H, (unsigned)(H * 2), &mbar[1]);
        } else {
            const char * src = static_cast<const char *>(A.down.w) + (size_t) s * R * H * 2;
            for (unsigned o = 0; o < dbytes; o += 32768)
                bulk_g2s(dbuf + o, src + o, dbytes - o < 32768 ? dbytes - o : 32768, &mbar[1]);
        }
    }
    const unsigned long long t_start = ff_now();
    pdl_trigger();
    ff_prefetch(A.pf);
    __syncthreads();
    pdl_wait();
    const int frame = fr.st->frame;
    if (fr.trace && frame == fr.trace_frame && tid == 0 && blockIdx.x < FF_TRACE_CTAS)
        fr.trace[((size_t) A.launch_id * FF_TRACE_CTAS + blockIdx.x) * FF_TRACE_N] = t_start;
    ff_stamp(fr, A.launch_id, frame, 1);
    if (fr.st->done) {
        ff_drain(&mbar[0], 0u);
        ff_drain(&mbar[1], 0u);
        return;
    }
    ff_build_input<NV>(fr, A.in, xs);
    if (A.set_presence && s == 0 && tid == 0) {
        const int c0 = fr.st->codes[0];
        fr.st->presence[c0 >> 5] |= 1u << (c0 & 31);
    }
    __syncthreads();
    GemvArgs gu{};
    gu.A = A.gate;
    gu.B = A.up;
    gu.nv = NV;
    gu.norm_g = A.ffn_norm;
    gu.eps = fr.eps;
    gu.act = ACT_F16;
    gu.epi = EPI_SWIGLU;
    ff_stamp(fr, A.launch_id, frame, 2);
    bool ok = gemv_compute<NV>(gu, s, (int) gridDim.x, wbuf, work, &mbar[0], 0u, FfSmemStore{hs, R});
    if (tid == 0 && !mbar_wait(&mbar[1], 0u)) ok = false;
    ok = !__syncthreads_or(!ok);
    ff_stamp(fr, A.launch_id, frame, 3);
    if (q8) {
        // quantise this CTA's 32-block of each row as quantize_row_q8_0_ref
        const int warp = tid >> 5, lane = tid & 31;
        if (warp < NV) {
            const float x = hs[warp * R + lane];
            float am = fabsf(x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
            const float d = __fdiv_rn(am, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            s_qa[warp][lane] = (int8_t) roundf(__fmul_rn(x, id));
            if (lane == 0) s_da[warp] = __half2float(__float2half_rn(d));
        }
        __syncthreads();
        const int8_t * dq = reinterpret_cast<const int8_t *>(dbuf);
        const __half * dd = reinterpret_cast<const __half *>(dbuf + (size_t) H * 32);
        for (int r = tid; r < H; r += nt) {
            const int4 * wr = reinterpret_cast<const int4 *>(dq + (size_t) r * 32);
            const int4 w0 = wr[0], w1 = wr[1];
            const float dw = __half2float(dd[r]);
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const int4 * qa = reinterpret_cast<const int4 *>(s_qa[v]);
                const int4 a0 = qa[0], a1 = qa[1];
                int is = __dp4a(w0.x, a0.x, 0);
                is = __dp4a(w0.y, a0.y, is);
                is = __dp4a(w0.z, a0.z, is);
                is = __dp4a(w0.w, a0.w, is);
                is = __dp4a(w1.x, a1.x, is);
                is = __dp4a(w1.y, a1.y, is);
                is = __dp4a(w1.z, a1.z, is);
                is = __dp4a(w1.w, a1.w, is);
                dpart[v * H + r] = __fmul_rn((float) is, __fmul_rn(dw, s_da[v]));
            }
        }
    } else {
        const __half * dt = reinterpret_cast<const __half *>(dbuf);   // [R][H]
        for (int r = tid; r < H; r += nt) {
            float acc[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = 0.0f;
            for (int j = 0; j < R; ++j) {
                const float w = __half2float(dt[(size_t) j * H + r]);
#pragma unroll
                for (int v = 0; v < NV; ++v) acc[v] = fmaf(w, hs[v * R + j], acc[v]);
            }
#pragma unroll
            for (int v = 0; v < NV; ++v) dpart[v * H + r] = acc[v];
        }
    }
    __syncthreads();
    ff_stamp(fr, A.launch_id, frame, 4);
    ff_cluster_sync();   // every CTA's partial is in its shared memory
    ff_stamp(fr, A.launch_id, frame, 5);
    {
        const int rows = H / (int) C, r0 = (int) rank * rows;
        for (int t = tid; t < NV * rows; t += nt) {
            const int v = t / rows, r = r0 + t - v * rows;
            const float * src = dpart + v * H + r;
            float pv[FF_MAX_CLUSTER];
#pragma unroll
            for (int p = 0; p < FF_MAX_CLUSTER; ++p) pv[p] = p < (int) C ? ff_ld_peer(ff_peer_addr(src, p)) : 0.0f;
            float acc = pv[0];
#pragma unroll
            for (int p = 1; p < FF_MAX_CLUSTER; ++p)
                if (p < (int) C) acc = __fadd_rn(acc, pv[p]);
            A.part_out[((size_t) cid * NV + v) * H + r] = acc;
        }
    }
    __syncthreads();
    ff_stamp(fr, A.launch_id, frame, 6);
    ff_cluster_sync();   // peers have read this CTA's partial
    if (!ok && tid == 0) atomicExch(fr.err, 3);
    ff_stamp(fr, A.launch_id, frame, 7);
}

// ---------------------------------------------------------------- heads
// Stand-alone GEMV whose input row is a partial sum (row in_row of the
// launch's nv_in-row buffers); the talker head also ends the frame.
struct FfHeadArgs {
    GemvArgs g;                          // A, norm, output (y), xn_out (talker hidden state)
    size_t slice_bytes;
    const float * base, * part;          // [nv_in][H], [np][nv_in][H]
    int np, nv_in, in_row;
    DevState * st;
    int * err;
    int frame_end;                       // advance the frame state at the end
    FfPrefetch pf;
    FfFrame fr;                          // (trace fields only)
    int launch_id;
};

__global__ void __launch_bounds__(FF_THREADS) k_ff_head(const FfHeadArgs A) {
    extern __shared__ __align__(128) uint8_t ff_smem[];
    __shared__ __align__(8) uint64_t mbar;
    const int tid = threadIdx.x, H = A.g.A.cols;
    if (tid == 0) {
        mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue_gemv_slice(A.g.A, DMat{}, A.g.norm_g, ff_smem, &mbar, blockIdx.x, gridDim.x);
    }
    const unsigned long long t_start = ff_now();
    pdl_trigger();
    ff_prefetch(A.pf);
    __syncthreads();
    pdl_wait();
    const int frame = A.st->frame;
    if (A.fr.trace && frame == A.fr.trace_frame && tid == 0 && blockIdx.x < FF_TRACE_CTAS)
        A.fr.trace[((size_t) A.launch_id * FF_TRACE_CTAS + blockIdx.x) * FF_TRACE_N] = t_start;
    ff_stamp(A.fr, A.launch_id, frame, 1);
    if (A.st->done) { ff_drain(&mbar, 0u); return; }
    uint8_t * work = ff_smem + A.slice_bytes;
    float * xs = reinterpret_cast<float *>(work);
    for (int c = tid; c < H; c += blockDim.x)
        xs[xpos(c, H)] = ff_part_sum(A.part, A.base, A.np, (size_t) A.nv_in * H, (size_t) A.in_row * H + c);
    __syncthreads();
    ff_stamp(A.fr, A.launch_id, frame, 2);
    const bool ok = gemv_compute<1>(A.g, blockIdx.x, gridDim.x, ff_smem, work, &mbar, 0u, GemvStorePlain{A.g});
    ff_stamp(A.fr, A.launch_id, frame, 3);
    if (!ok) {
        ff_drain(&mbar, 0u);
        if (tid == 0) atomicExch(A.err, 3);
    }
    ff_stamp(A.fr, A.launch_id, frame, 7);
    if (A.frame_end && blockIdx.x == 0 && tid == 0) {
        A.st->pos += 1;
        A.st->frame += 1;
        A.st->n_out += 1;
    }
}

// ---------------------------------------------------------------- load-time repacking
// ffn_down into the FFN block's layout: F16 [H][I] -> [I][H]; Q8_0 int8
// [H][I] -> [I/32][H][32] and scales [H][I/32] -> [I/32][H].
__global__ void k_ff_repack_down(DMat src, void * dst_w, __half * dst_d) {
    const int H = src.rows, I = src.cols;
    const size_t n = (size_t) H * I;
    for (size_t e = (size_t) blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t) gridDim.x * blockDim.x) {
        const int r = (int)(e / I), j = (int)(e % I);
        if (src.type == W_Q8_0) {
            static_cast<int8_t *>(dst_w)[((size_t)(j >> 5) * H + r) * 32 + (j & 31)] =
                static_cast<const int8_t *>(src.w)[e];
            if ((j & 31) == 0) dst_d[(size_t)(j >> 5) * H + r] = src.d[(size_t) r * (I / 32) + (j >> 5)];
        } else {
            static_cast<__half *>(dst_w)[(size_t) j * H + r] = static_cast<const __half *>(src.w)[e];
        }
    }
}

}  // namespace qtts
