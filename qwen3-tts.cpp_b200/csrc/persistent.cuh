// persistent.cuh — the whole codec frame as one persistent cooperative kernel.
//
// One CTA per SM runs the frame's op list (GEMVs, fused q/k-norm + RoPE + KV
// append + attention, samplers, embedding gathers) with a grid barrier between
// dependent ops.  Kernel-per-op execution pays a launch and a ramp/tail per op,
// and the GEMV ops are only 0.6-1.8 us of HBM time each; here the barrier is the
// only per-op cost, and every CTA issues cp.async.bulk.prefetch.L2 for its
// slice of the GEMV weights LEAD bytes ahead in the weight stream, so HBM keeps
// streaming while the grid waits at barriers.
//
// The grid barrier is a flag array: CTA i publishes the epoch in flags[i]
// (release), warp 0 of every CTA polls all flags (acquire).  Every spin has an
// iteration limit; on expiry the kernel sets *err and returns, and the host
// reports the error (no GPU trap).
#pragma once
#include "kernels.cuh"

namespace qtts {

constexpr int PK_THREADS = 512;
constexpr unsigned long long PK_SPIN_LIMIT = 1ull << 22;   // polls before giving up (a few seconds)

enum POpType : int { P_NOP = 0, P_GEMV = 1, P_ATTN = 2, P_SAMPLE = 3, P_INPUT = 4, P_FRAME_END = 5 };

// q/k RMSNorm + RoPE + KV append + attention for one (kv head, query row) unit.
struct FusedAttn {
    float * qkv;              // raw q|k|v rows [M][ldq]
    int ldq;
    int n_heads, n_kv_heads;
    const float * q_norm, * k_norm;
    float eps;
    const float2 * rope;      // [pos][64]
    __half * kc, * vc;        // cache base of this layer [ctx][NKV][128]
    const int * pos_ptr;
    int pos_static;
    int M;
    int f32_mode;             // 2-token code-predictor prefill: attend over this call's F32 K/V
    float scale;
    float * out;
    int ldo;
    float * dump;             // post-softmax rows [frame][n_heads][dump_stride] or nullptr
    int dump_stride;
};

constexpr int PK_MAX_PF = 3;

struct alignas(16) POp {
    int type;
    int barrier;              // grid barrier after this op
    int nv;                   // GEMV rows (1 or 2)
    int cb, V;                // sampler
    int slot;                 // GEMV: shared-memory weight buffer holding this op's slice
    int issue;                // copy the slice of (iA, iB) into buffer issue_slot at op start
    int issue_slot;
    int n_pf;                 // GEMV weight matrices to prefetch into L2 at op start
    const float * logits;
    DMat iA, iB;
    DMat pfA[PK_MAX_PF], pfB[PK_MAX_PF];
    GemvArgs g;
    FusedAttn a;
    InputArgs in;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned * p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u32(unsigned * p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Returns false (and sets *err) when a peer did not arrive within the limit or
// another CTA reported an error.
__device__ __forceinline__ bool grid_barrier(unsigned * flags, unsigned epoch, int * err) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        if (lane == 0) {
            __threadfence();
            st_release_u32(flags + blockIdx.x, epoch);
        }
        __syncwarp();
        bool ok = false;
        for (unsigned long long it = 0; it < PK_SPIN_LIMIT; ++it) {
            bool mine = true;
            for (int c = lane; c < (int) gridDim.x; c += 32)
                if (ld_relaxed_u32(flags + c) < epoch) mine = false;
            if (__all_sync(0xffffffffu, mine)) { ok = true; break; }
            if (__any_sync(0xffffffffu, *(volatile int *) err != 0)) break;   // warp-uniform exit
        }
        __threadfence();   // acquire side: order the peers' writes before this CTA's reads
        if (lane == 0) {
            if (!ok) atomicExch(err, 1);
            s_ok = ok;
        }
    }
    __syncthreads();
    return s_ok != 0;
}

__device__ __forceinline__ void prefetch_l2(const void * p, size_t bytes) {
    const char * c = static_cast<const char *>(p);
    while (bytes > 0) {
        const unsigned n = (unsigned) (bytes > 65536 ? 65536 : bytes);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}

// This CTA's row slice of a GEMV's weights (same split as gemv_body).
__device__ __forceinline__ void prefetch_mat_slice(const DMat & M, int cta, int ncta) {
    if (!M.w) return;
    const int rows = M.rows, cols = M.cols;
    const int rpc = (rows + ncta - 1) / ncta;
    const int r0 = cta * rpc, r1 = min(rows, r0 + rpc);
    if (r0 >= r1) return;
    const size_t es = M.type == W_F16 ? 2 : 1;
    prefetch_l2(static_cast<const char *>(M.w) + (size_t) r0 * cols * es, (size_t)(r1 - r0) * cols * es);
    if (M.type == W_Q8_0) prefetch_l2(M.d + (size_t) r0 * (cols / 32), (size_t)(r1 - r0) * (cols / 32) * 2);
}
__device__ __forceinline__ void prefetch_gemv_slice(const GemvArgs & g, int cta, int ncta) {
    prefetch_mat_slice(g.A, cta, ncta);
    prefetch_mat_slice(g.B, cta, ncta);
}

// ---- shared-memory weight slices (TMA bulk copies completed on an mbarrier)
__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t * m, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t * m, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t * m, unsigned parity) {
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(smem_u32(m)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: false when the phase did not complete within the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t * m, unsigned parity) {
    for (unsigned long long it = 0; it < PK_SPIN_LIMIT; ++it)
        if (mbar_try_wait(m, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, unsigned bytes, uint64_t * m) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(m)) : "memory");
}

struct SliceGeom {
    int r0, r1;
    size_t bytesA, bytesS;   // per matrix: quants/halves, scales
};
__device__ __forceinline__ SliceGeom slice_geom(const DMat & A, int cta, int ncta) {
    SliceGeom g;
    const int rpc = (A.rows + ncta - 1) / ncta;
    g.r0 = cta * rpc;
    g.r1 = min(A.rows, g.r0 + rpc);
    const int n = g.r1 > g.r0 ? g.r1 - g.r0 : 0;
    g.bytesA = (size_t) n * A.cols * (A.type == W_F16 ? 2 : 1);
    g.bytesS = A.type == W_Q8_0 ? (size_t) n * (A.cols / 32) * 2 : 0;
    return g;
}
// Buffer layout: A rows | B rows | A scales | B scales.
__device__ __forceinline__ WSrc slice_src(const DMat & A, const DMat & B, const uint8_t * buf, int cta, int ncta) {
    const SliceGeom g = slice_geom(A, cta, ncta);
    const int nm = B.w ? 2 : 1;
    WSrc s;
    s.a = buf;
    s.b = buf + g.bytesA;
    s.sa = reinterpret_cast<const __half *>(buf + nm * g.bytesA);
    s.sb = reinterpret_cast<const __half *>(buf + nm * g.bytesA + g.bytesS);
    s.rbase = g.r0;
    return s;
}
// One thread: copy this CTA's slice of (A, B) into buf, completing on m.
__device__ __forceinline__ void issue_slice(const DMat & A, const DMat & B, uint8_t * buf, uint64_t * m, int cta,
                                            int ncta) {
    const SliceGeom g = slice_geom(A, cta, ncta);
    const int nm = B.w ? 2 : 1;
    const size_t es = A.type == W_F16 ? 2 : 1;
    mbar_expect_tx(m, (unsigned)(nm * (g.bytesA + g.bytesS)));
    if (g.r1 <= g.r0) return;
    const DMat * mats[2] = {&A, &B};
    for (int k = 0; k < nm; ++k) {
        const char * src = static_cast<const char *>(mats[k]->w) + (size_t) g.r0 * A.cols * es;
        uint8_t * dst = buf + k * g.bytesA;
        for (size_t o = 0; o < g.bytesA; o += 32768) {
            const unsigned n = (unsigned)(g.bytesA - o < 32768 ? g.bytesA - o : 32768);
            bulk_g2s(dst + o, src + o, n, m);
        }
        if (g.bytesS) {
            const char * ss = reinterpret_cast<const char *>(mats[k]->d + (size_t) g.r0 * (A.cols / 32));
            bulk_g2s(buf + nm * g.bytesA + k * g.bytesS, ss, (unsigned) g.bytesS, m);
        }
    }
}

constexpr int PK_MAX_PG = PK_THREADS / 64;   // PV position groups

__host__ __device__ inline size_t fused_attn_smem(int max_keys, int G, int M) {
    return (size_t) G * max_keys * 4 + (size_t) G * QTTS_HD * 4 + (size_t) PK_MAX_PG * G * QTTS_HD * 4 +
           2 * (size_t) M * QTTS_HD * 4 + 512;
}

__device__ void fused_attn_body(const FusedAttn & a, const int unit, uint8_t * smem, const DevState * st) {
    __shared__ float redf[32];
    __shared__ double redd[32];
    const int NKV = a.n_kv_heads, G = a.n_heads / a.n_kv_heads;
    const int g = unit % NKV, i = unit / NKV;
    const int n_past = a.pos_ptr ? *a.pos_ptr : a.pos_static;
    const int pos = n_past + i;
    const int n = a.f32_mode ? (i + 1) : (n_past + i + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int QD = a.n_heads * QTTS_HD, KD = NKV * QTTS_HD;
    float * qs = reinterpret_cast<float *>(smem);        // [G][D]
    float * part = qs + G * QTTS_HD;                      // [PK_MAX_PG][G][D]
    float * ks = part + PK_MAX_PG * G * QTTS_HD;          // [M][D] (F32 mode)
    float * vs = ks + a.M * QTTS_HD;                      // [M][D]
    float * sc = vs + a.M * QTTS_HD;                      // [G][n]

    if (warp < G) {
        const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
        const float * qh = a.qkv + (size_t) i * a.ldq + (size_t)(g * G + warp) * QTTS_HD + lane * 4;
        float x[4] = {qh[0], qh[1], qh[2], qh[3]};
        head_norm_rope(x, a.q_norm, a.eps, rp, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) qs[warp * QTTS_HD + lane * 4 + k] = a.f32_mode ? x[k] : round_f16(x[k]);
    } else if (warp < G + (a.f32_mode ? i + 1 : 1)) {
        const int j = a.f32_mode ? warp - G : i;                // key row handled by this warp
        const float2 * rp = a.rope + (size_t)(n_past + j) * (QTTS_HD / 2);
        const float * kp = a.qkv + (size_t) j * a.ldq + QD + g * QTTS_HD + lane * 4;
        const float * vp = a.qkv + (size_t) j * a.ldq + QD + KD + g * QTTS_HD + lane * 4;
        float x[4] = {kp[0], kp[1], kp[2], kp[3]};
        head_norm_rope(x, a.k_norm, a.eps, rp, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (a.f32_mode) { ks[j * QTTS_HD + lane * 4 + k] = x[k]; vs[j * QTTS_HD + lane * 4 + k] = vp[k]; }
            if (j == i) {
                a.kc[((size_t) pos * NKV + g) * QTTS_HD + lane * 4 + k] = __float2half_rn(x[k]);
                a.vc[((size_t) pos * NKV + g) * QTTS_HD + lane * 4 + k] = __float2half_rn(vp[k]);
            }
        }
    }
    __syncthreads();

    // uniform trip count per warp (full-mask shuffles below); out-of-range keys use zeros
    const int sub = lane & 7, slot = lane >> 3;
    const int nwarps = blockDim.x >> 5;
    for (int j0 = warp * 4; j0 < n; j0 += nwarps * 4) {
        const int j = j0 + slot;
        const bool jv = j < n;
        float kv[16];
        if (!jv) {
#pragma unroll
            for (int d = 0; d < 16; ++d) kv[d] = 0.0f;
        } else if (a.f32_mode) {
#pragma unroll
            for (int d = 0; d < 16; ++d) kv[d] = ks[j * QTTS_HD + sub * 16 + d];
        } else {
            const uint4 * kp = reinterpret_cast<const uint4 *>(a.kc + ((size_t) j * NKV + g) * QTTS_HD + sub * 16);
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8) {
                uint4 u = kp[h8];
                const __half2 * hp = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float2 f = __half22float2(hp[k]);
                    kv[8 * h8 + 2 * k] = f.x; kv[8 * h8 + 2 * k + 1] = f.y;
                }
            }
        }
        for (int h = 0; h < G; ++h) {
            const float * qh = qs + h * QTTS_HD + sub * 16;
            float s = 0.0f;
#pragma unroll
            for (int d = 0; d < 16; ++d) s = fmaf(kv[d], qh[d], s);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            if (sub == 0 && jv) sc[h * n + j] = __fmul_rn(s, a.scale);
        }
    }
    __syncthreads();
    for (int h = 0; h < G; ++h) {
        float mx = -INFINITY;
        for (int j = tid; j < n; j += blockDim.x) mx = fmaxf(mx, sc[h * n + j]);
        mx = block_max(mx, redf);
        double sum = 0.0;
        for (int j = tid; j < n; j += blockDim.x) {
            const float e = expf(__fsub_rn(sc[h * n + j], mx));
            sc[h * n + j] = e;
            sum += (double) e;
        }
        sum = block_sum_d(sum, redd);
        const float inv = (float)(1.0 / sum);
        float * drow = a.dump ? a.dump + ((size_t) st->frame * a.n_heads + g * G + h) * a.dump_stride : nullptr;
        for (int j = tid; j < n; j += blockDim.x) {
            const float p = __fmul_rn(sc[h * n + j], inv);
            if (drow) drow[j] = p;
            sc[h * n + j] = a.f32_mode ? p : round_f16(p);
        }
        __syncthreads();
    }
    // KQV: position groups of 64 threads, each thread 2 dims of all G heads
    const int npg = blockDim.x >> 6;
    const int pg = tid >> 6, d2 = tid & 63;
    float acc[ATT_MAX_GROUP][2];
#pragma unroll
    for (int h = 0; h < ATT_MAX_GROUP; ++h) acc[h][0] = acc[h][1] = 0.0f;
    for (int j = pg; j < n; j += npg) {
        float2 v;
        if (a.f32_mode) v = make_float2(vs[j * QTTS_HD + 2 * d2], vs[j * QTTS_HD + 2 * d2 + 1]);
        else v = __half22float2(*reinterpret_cast<const __half2 *>(a.vc + ((size_t) j * NKV + g) * QTTS_HD + 2 * d2));
#pragma unroll
        for (int h = 0; h < ATT_MAX_GROUP; ++h)
            if (h < G) {
                const float p = sc[h * n + j];
                acc[h][0] = fmaf(p, v.x, acc[h][0]);
                acc[h][1] = fmaf(p, v.y, acc[h][1]);
            }
    }
    // partial sums of the position groups, then a fixed-order reduction
    float * red = part;
    __syncthreads();
#pragma unroll
    for (int h = 0; h < ATT_MAX_GROUP; ++h)
        if (h < G) {
            red[(pg * G + h) * QTTS_HD + 2 * d2] = acc[h][0];
            red[(pg * G + h) * QTTS_HD + 2 * d2 + 1] = acc[h][1];
        }
    __syncthreads();
    for (int t = tid; t < G * QTTS_HD; t += blockDim.x) {
        float s = 0.0f;
        for (int q = 0; q < npg; ++q) s = __fadd_rn(s, red[q * G * QTTS_HD + t]);
        a.out[(size_t) i * a.ldo + (size_t)(g * G) * QTTS_HD + t] = s;
    }
    __syncthreads();
}

__device__ void frame_inputs_body(const InputArgs & a) {
    const DevState * st = a.st;
    for (int h = threadIdx.x; h < a.H; h += blockDim.x) {
        if (a.mode == IN_CP_PREFILL) {
            a.out[h] = a.hidden[h];
            a.out[a.H + h] = __half2float(a.codec_embd[(size_t) st->codes[0] * a.H + h]);
        } else if (a.mode == IN_CP_STEP) {
            a.out[h] = __half2float(a.cp_embd[a.g - 1][(size_t) st->codes[a.g] * a.H + h]);
        } else {
            float s = __half2float(a.codec_embd[(size_t) st->codes[0] * a.H + h]);
            for (int cb = 1; cb < a.n_cb; ++cb)
                s = __fadd_rn(s, __half2float(a.cp_embd[cb - 1][(size_t) st->codes[cb] * a.H + h]));
            const float * tr = st->frame < st->n_trailing ? a.trailing + (size_t) st->frame * a.H : a.pad;
            a.out[h] = __fadd_rn(s, tr[h]);
        }
    }
}

struct PersistentArgs {
    const POp * ops;
    int n_ops;
    int n_frames;
    DevState * st;
    const SampleParams * sp;
    int * out_codes;
    int out_cap;
    unsigned * flags;          // [gridDim.x], zeroed before the launch
    int * err;
    int wbuf_bytes;            // bytes of each of the two weight buffers
    int n_pf0;                 // GEMVs prefetched into L2 at launch start
    int pf0[16];
    int first_gemv[2];         // the first two GEMV ops (their slices are copied at launch start)
    unsigned long long * trace;  // optional: CTA 0 records %globaltimer per op (start, work done)
};

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void pk_drain(uint64_t * mbar, const int * pending, unsigned * phase) {
    for (int b = 0; b < 2; ++b)
        if (pending[b]) { mbar_wait(&mbar[b], phase[b] & 1u); phase[b]++; }
}

__global__ void __launch_bounds__(PK_THREADS, 1) k_frame_persistent(PersistentArgs P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ POp desc[2];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ int s_done;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    uint8_t * wbuf[2] = {smem, smem + P.wbuf_bytes};
    uint8_t * work = smem + 2 * (size_t) P.wbuf_bytes;
    unsigned phase[2] = {0u, 0u};
    int pending[2] = {0, 0};
    unsigned epoch = 0;
    constexpr int NW = (int)(sizeof(POp) / 8);

    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    {
        const unsigned long long * src = reinterpret_cast<const unsigned long long *>(P.ops);
        unsigned long long * dst = reinterpret_cast<unsigned long long *>(&desc[0]);
        for (int w = tid; w < NW; w += blockDim.x) dst[w] = src[w];
    }
    __syncthreads();
    if (tid == 0) {
        for (int k = 0; k < P.n_pf0; ++k) prefetch_gemv_slice(P.ops[P.pf0[k]].g, cta, ncta);
        for (int b = 0; b < 2; ++b) {
            const POp & g = P.ops[P.first_gemv[b]];
            issue_slice(g.g.A, g.g.B, wbuf[g.slot], &mbar[g.slot], cta, ncta);
        }
    }
    pending[0] = pending[1] = 1;

    long long s = 0;   // position in the op stream
    for (int f = 0; f < P.n_frames; ++f) {
        for (int oi = 0; oi < P.n_ops; ++oi, ++s) {
            const POp & op = desc[s & 1];
            if (P.trace && cta == 0 && tid == 0) P.trace[2 * s] = globaltimer_ns();
            // stage the next descriptor (loads now, shared-memory stores before the barrier)
            const int nx = oi + 1 < P.n_ops ? oi + 1 : 0;
            const unsigned long long * nsrc = reinterpret_cast<const unsigned long long *>(P.ops + nx);
            unsigned long long nw0 = tid < NW ? nsrc[tid] : 0ull;
            unsigned long long nw1 = tid + (int) blockDim.x < NW ? nsrc[tid + blockDim.x] : 0ull;
            if (tid == 0) {
                if (op.issue) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue_slice(op.iA, op.iB, wbuf[op.issue_slot], &mbar[op.issue_slot], cta, ncta);
                }
                for (int k = 0; k < op.n_pf; ++k) {
                    prefetch_mat_slice(op.pfA[k], cta, ncta);
                    prefetch_mat_slice(op.pfB[k], cta, ncta);
                }
            }
            if (op.issue) pending[op.issue_slot] = 1;
            switch (op.type) {
                case P_GEMV: {
                    const int b = op.slot;
                    const bool ok = mbar_wait(&mbar[b], phase[b] & 1u);
                    if (__syncthreads_or(!ok)) {      // block-uniform: a copy did not land in time
                        if (tid == 0) atomicExch(P.err, 2);
                        pk_drain(mbar, pending, phase);
                        return;
                    }
                    phase[b]++;
                    pending[b] = 0;
                    const WSrc src = slice_src(op.g.A, op.g.B, wbuf[b], cta, ncta);
                    if (op.nv == 1) gemv_body<1, true>(op.g, cta, ncta, work, &src);
                    else gemv_body<2, true>(op.g, cta, ncta, work, &src);
                    break;
                }
                case P_ATTN:
                    for (int u = cta; u < op.a.n_kv_heads * op.a.M; u += ncta) fused_attn_body(op.a, u, work, P.st);
                    break;
                case P_SAMPLE:
                    if (cta == 0) {
                        const SampleParams sp = *P.sp;
                        const int frame = P.st->frame;
                        const int tok = sample_body<8>(op.logits, op.V, op.cb, P.st, sp, frame);
                        if (tid == 0) sample_commit(tok, op.cb, P.st, sp, P.out_codes, P.out_cap, frame);
                    }
                    break;
                case P_INPUT:
                    if (cta == 0) frame_inputs_body(op.in);
                    break;
                case P_FRAME_END:
                    if (cta == 0 && tid == 0 && !P.st->done) {
                        P.st->pos += 1;
                        P.st->frame += 1;
                        P.st->n_out += 1;
                    }
                    break;
                default:
                    break;
            }
            __syncthreads();   // everyone is done with desc[s & 1]
            if (P.trace && cta == 0 && tid == 0) P.trace[2 * s + 1] = globaltimer_ns();
            {
                unsigned long long * ndst = reinterpret_cast<unsigned long long *>(&desc[(s + 1) & 1]);
                if (tid < NW) ndst[tid] = nw0;
                if (tid + (int) blockDim.x < NW) ndst[tid + blockDim.x] = nw1;
            }
            const int was_sample0 = op.type == P_SAMPLE && op.cb == 0;
            if (op.barrier) {
                if (!grid_barrier(P.flags, ++epoch, P.err)) { pk_drain(mbar, pending, phase); return; }
                if (was_sample0) {
                    if (tid == 0) s_done = *(volatile int *) &P.st->done;
                    __syncthreads();
                    if (s_done) { pk_drain(mbar, pending, phase); return; }
                }
            } else {
                __syncthreads();
            }
        }
    }
    pk_drain(mbar, pending, phase);
}

}  // namespace qtts
