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

struct alignas(16) POp {
    int type;
    int barrier;              // grid barrier after this op
    int nv;                   // GEMV rows (1 or 2)
    int cb, V;                // sampler
    const float * logits;
    int n_pf;                 // GEMV ops whose weight slices this op prefetches into L2
    int pf[6];
    GemvArgs g;
    FusedAttn a;
    InputArgs in;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
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
                if (ld_acquire_u32(flags + c) < epoch) mine = false;
            if (__all_sync(0xffffffffu, mine)) { ok = true; break; }
            if (__any_sync(0xffffffffu, *(volatile int *) err != 0)) break;   // warp-uniform exit
        }
        if (lane == 0) {
            if (!ok) atomicExch(err, 1);
            __threadfence();
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
__device__ __forceinline__ void prefetch_gemv_slice(const GemvArgs & g, int cta, int ncta) {
    const int rows = g.A.rows, cols = g.A.cols;
    const int rpc = (rows + ncta - 1) / ncta;
    const int r0 = cta * rpc, r1 = min(rows, r0 + rpc);
    if (r0 >= r1) return;
    const size_t es = g.A.type == W_F16 ? 2 : 1;
    const DMat * mats[2] = {&g.A, &g.B};
    for (int m = 0; m < 2; ++m) {
        const DMat & M = *mats[m];
        if (!M.w) continue;
        prefetch_l2(static_cast<const char *>(M.w) + (size_t) r0 * cols * es, (size_t)(r1 - r0) * cols * es);
        if (M.type == W_Q8_0)
            prefetch_l2(M.d + (size_t) r0 * (cols / 32), (size_t)(r1 - r0) * (cols / 32) * 2);
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
    int n_pf0;                 // ops prefetched at launch start
    int pf0[16];
};

__global__ void __launch_bounds__(PK_THREADS, 1) k_frame_persistent(PersistentArgs P) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ POp op;
    __shared__ int s_done;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    unsigned epoch = 0;
    if (tid == 0)
        for (int k = 0; k < P.n_pf0; ++k) prefetch_gemv_slice(P.ops[P.pf0[k]].g, cta, ncta);
    for (int f = 0; f < P.n_frames; ++f) {
        for (int oi = 0; oi < P.n_ops; ++oi) {
            // stage the op descriptor in shared memory
            {
                const unsigned long long * src = reinterpret_cast<const unsigned long long *>(P.ops + oi);
                unsigned long long * dst = reinterpret_cast<unsigned long long *>(&op);
                for (int w = tid; w < (int)(sizeof(POp) / 8); w += blockDim.x) dst[w] = src[w];
            }
            __syncthreads();
            if (tid == 0)
                for (int k = 0; k < op.n_pf; ++k) prefetch_gemv_slice(P.ops[op.pf[k]].g, cta, ncta);
            switch (op.type) {
                case P_GEMV:
                    if (op.nv == 1) gemv_body<1>(op.g, cta, ncta, smem);
                    else gemv_body<2>(op.g, cta, ncta, smem);
                    break;
                case P_ATTN:
                    for (int u = cta; u < op.a.n_kv_heads * op.a.M; u += ncta) fused_attn_body(op.a, u, smem, P.st);
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
            if (op.barrier) {
                if (!grid_barrier(P.flags, ++epoch, P.err)) return;
                if (op.type == P_SAMPLE && op.cb == 0) {
                    if (tid == 0) s_done = *(volatile int *) &P.st->done;
                    __syncthreads();
                    if (s_done) return;
                }
            } else {
                __syncthreads();
            }
        }
    }
}

}  // namespace qtts
