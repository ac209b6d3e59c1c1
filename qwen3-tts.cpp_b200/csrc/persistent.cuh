// persistent.cuh — the whole codec frame as one persistent cooperative kernel.
//
// One CTA per SM runs the frame's op list (GEMVs, fused q/k-norm + RoPE + KV
// append + attention, samplers with the next inputs) with a grid barrier
// between dependent ops.  Kernel-per-op execution pays a launch and a ramp/tail
// per op, and the GEMV ops are only 0.6-1.8 us of HBM time each; here the
// barrier is the only per-op cost.  Each CTA copies its row slice of the next
// GEMVs' weights into a two-buffer shared-memory ring with TMA bulk copies, and
// prefetches slices further ahead into L2, while it waits at barriers.
//
// Every spin has an iteration limit; on expiry the kernel sets *err and
// returns, and the host reports the error (no GPU trap).
#pragma once
#include "kernels.cuh"

namespace qtts {

constexpr int PK_THREADS = 512;

enum POpType : int { P_NOP = 0, P_GEMV = 1, P_ATTN = 2, P_SAMPLE = 3, P_INPUT = 4, P_FRAME_END = 5 };

constexpr int PK_MAX_PF = 3;

struct alignas(16) POp {
    int type;
    int barrier;              // grid barrier after this op
    int nv;                   // GEMV rows (1 or 2)
    int cb, V;                // sampler
    int slot;                 // GEMV: shared-memory weight buffer holding this op's slice
    int issue;                // after this op, copy the slice of (iA, iB) into buffer issue_slot
    int issue_slot;
    int n_pf;                 // GEMV weight matrices to prefetch into L2 after this op
    int has_in;               // P_SAMPLE: CTA 0 then builds the next inputs (in) itself
    const float * logits;
    DMat iA, iB;
    const float * iG;         // RMSNorm gain staged with the slice (nullptr: none)
    DMat pfA[PK_MAX_PF], pfB[PK_MAX_PF];
    GemvArgs g;
    FusedAttn a;
    InputArgs in;
};

// Grid barrier on one arrival counter.  Thread 0 of each CTA adds 1 with
// release semantics (ordering the CTA's writes, made visible to it by the block
// barrier) and polls the counter with acquire loads until all CTAs of this
// epoch arrived: target = epoch * gridDim.x, compared modulo 2^32.  A single
// counter costs 1.45 us per barrier on B200 against 2.49 us for a flag per CTA
// polled by a warp.  While thread 0 waits, thread 32 runs `side` (the weight
// copies and L2 prefetches for later ops), off the critical path.  Returns
// false (and sets *err) when the peers did not arrive within the poll limit or
// another CTA reported an error.
template <class Side>
__device__ __forceinline__ bool grid_barrier(unsigned * ctr, unsigned epoch, int * err, const Side & side) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        const unsigned target = epoch * gridDim.x;
        bool ok = false;
        for (unsigned long long it = 0; it < QTTS_SPIN_LIMIT; ++it) {
            const int e = *(volatile int *) err;   // issued together with the counter load
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
            if ((int)(v - target) >= 0) { ok = true; break; }
            if (e != 0) break;
        }
        if (!ok) atomicExch(err, 1);
        s_ok = ok;
    } else if (threadIdx.x == 32) {
        side();
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

// This CTA's row slice of a GEMV's weights (same split as gemv_slice).
__device__ __forceinline__ void prefetch_mat_slice(const DMat & M, int cta, int ncta) {
    if (!M.w) return;
    const int rows = M.rows, cols = M.cols;
    const int rpc = gemv_rpc(rows, ncta);
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

struct PersistentArgs {
    const POp * ops;
    int n_ops;
    int n_frames;
    DevState * st;
    const SampleParams * sp;
    int * out_codes;
    int out_cap;
    unsigned * flags;          // flags[0]: grid barrier arrival counter, zeroed before the launch
    int * err;
    int wbuf_bytes;            // bytes of each of the two weight buffers
    int n_pf0;                 // GEMVs prefetched into L2 at launch start
    int pf0[16];
    int first_gemv[2];         // the first two GEMV ops (their slices are copied at launch start)
    unsigned long long * trace;  // optional: CTA 0 records %globaltimer per op (PK_TRACE_SLOTS stamps)
};
constexpr int PK_TRACE_SLOTS = 5;   // CTA 0: op start, side work issued; max over CTAs: weights ready; CTA 0: work done; max over CTAs: work done

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Waits (bounded) for the copies still in flight into either weight buffer.
// pending / phase hold one bit per buffer (no per-thread arrays: those would
// live in local memory).
__device__ __forceinline__ void pk_drain(uint64_t * mbar, unsigned pending, unsigned phase) {
    if (threadIdx.x != 0) return;
    for (int b = 0; b < 2; ++b)
        if (pending >> b & 1u) mbar_wait(mbar + b, phase >> b & 1u);
}

__global__ void __launch_bounds__(PK_THREADS, 1) k_frame_persistent(PersistentArgs P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ POp desc[2];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ int s_done;
    __shared__ SampleParams s_sp;
    __shared__ int s_codes[QTTS_MAX_CB];
    __shared__ const __half * s_tabs[QTTS_MAX_CB];
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    uint8_t * work = smem + 2 * (size_t) P.wbuf_bytes;
    unsigned phase = 0u, pending = 0u;   // bit b: parity of buffer b's next completion / copy in flight
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
            issue_gemv_slice(g.g.A, g.g.B, g.g.norm_g, smem + (size_t) g.slot * P.wbuf_bytes, mbar + g.slot, cta, ncta);
        }
    }
    pending = 3u;

    // Every frame advances the position and the frame index by one (a frame
    // that samples EOS ends the launch), so both follow from their values at
    // launch; CTA 0 still writes them back to the frame state at frame end.
    const int pos0 = *(volatile const int *) &P.st->pos;
    const int frame0 = *(volatile const int *) &P.st->frame;
    const int n_trailing = P.st->n_trailing;
    if (tid == 0) s_sp = *P.sp;
    __syncthreads();

    long long s = 0;   // position in the op stream
    for (int f = 0; f < P.n_frames; ++f) {
        for (int oi = 0; oi < P.n_ops; ++oi, ++s) {
            const POp & op = desc[s & 1];
            if (P.trace && cta == 0 && tid == 0) P.trace[PK_TRACE_SLOTS * s] = globaltimer_ns();
            // stage the next descriptor (loads now, shared-memory stores before the barrier)
            const int nx = oi + 1 < P.n_ops ? oi + 1 : 0;
            const unsigned long long * nsrc = reinterpret_cast<const unsigned long long *>(P.ops + nx);
            unsigned long long nw0 = tid < NW ? nsrc[tid] : 0ull;
            unsigned long long nw1 = tid + (int) blockDim.x < NW ? nsrc[tid + blockDim.x] : 0ull;
            switch (op.type) {
                case P_GEMV: {
                    const int b = op.slot;
                    const uint8_t * wb = smem + (size_t) b * P.wbuf_bytes;
                    const unsigned par = phase >> b & 1u;
                    const bool ok = op.nv == 1 ? gemv_slice<1>(op.g, cta, ncta, wb, work, mbar + b, par)
                                               : gemv_slice<2>(op.g, cta, ncta, wb, work, mbar + b, par);
                    if (!ok) {                          // block-uniform: a copy did not land in time
                        if (tid == 0) atomicExch(P.err, 2);
                        pk_drain(mbar, pending, phase);
                        return;
                    }
                    phase ^= 1u << b;
                    pending &= ~(1u << b);
                    break;
                }
                case P_ATTN: {
                    const int np = op.a.pos_ptr ? pos0 + f : op.a.pos_static;
                    if (op.a.warp_heads) {   // code-predictor step: warp 0 of CTAs 0 .. n_heads - 1
                        if (tid < 32)
                            for (int u = cta; u < op.a.n_heads; u += ncta) cp_step_attn_warp(op.a, u, np);
                        break;
                    }
                    for (int u = cta; u < op.a.n_heads * op.a.M; u += ncta) {
                        fused_attn_body(op.a, u, work, np, frame0 + f);
                        if (u + ncta < op.a.n_heads * op.a.M) __syncthreads();
                    }
                    break;
                }
                case P_SAMPLE:
                    if (cta == 0) {
                        const int frame = frame0 + f;
                        // earlier codes and table pointers for the talker input, loaded while sampling
                        int c_pre = 0;
                        const __half * t_pre = nullptr;
                        if (op.has_in && op.in.mode == IN_TALKER) {
                            if (tid < op.cb) c_pre = P.st->codes[tid];
                            if (tid >= 1 && tid < op.in.n_cb) t_pre = op.in.cp_embd[tid - 1];
                        }
                        const int tok = sample_body<8>(op.logits, op.V, op.cb, P.st, s_sp, frame);
                        if (tid == 0) sample_commit(tok, op.cb, P.st, s_sp, P.out_codes, P.out_cap, frame);
                        if (op.has_in) {
                            if (tid < op.cb) s_codes[tid] = c_pre;
                            if (tid == 0) s_codes[op.cb] = tok;
                            if (tid < QTTS_MAX_CB) s_tabs[tid] = t_pre;
                            __syncthreads();
                            frame_inputs_body(op.in, frame, s_codes, s_tabs, n_trailing);
                        }
                    }
                    break;
                case P_INPUT:   // inputs built right after a sampler: the program never emits it alone
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
            __syncthreads();   // everyone is done with desc[s & 1] and with the weight buffer of this op
            if (P.trace && tid == 0) {
                const unsigned long long t = globaltimer_ns();
                if (cta == 0) P.trace[PK_TRACE_SLOTS * s + 3] = t;
                atomicMax(P.trace + PK_TRACE_SLOTS * s + 4, t);
            }
            {
                unsigned long long * ndst = reinterpret_cast<unsigned long long *>(&desc[(s + 1) & 1]);
                if (tid < NW) ndst[tid] = nw0;
                if (tid + (int) blockDim.x < NW) ndst[tid + blockDim.x] = nw1;
            }
            // weight copies for the GEMV after next, L2 prefetches further ahead
            auto side = [&]() {
                if (op.issue) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue_gemv_slice(op.iA, op.iB, op.iG, smem + (size_t) op.issue_slot * P.wbuf_bytes,
                                     mbar + op.issue_slot, cta, ncta);
                }
                for (int k = 0; k < op.n_pf; ++k) {
                    prefetch_mat_slice(op.pfA[k], cta, ncta);
                    prefetch_mat_slice(op.pfB[k], cta, ncta);
                }
                if (P.trace && cta == 0) P.trace[PK_TRACE_SLOTS * s + 1] = globaltimer_ns();
            };
            if (op.issue) pending |= 1u << op.issue_slot;
            const int was_sample0 = op.type == P_SAMPLE && op.cb == 0;
            if (op.barrier) {
                if (!grid_barrier(P.flags, ++epoch, P.err, side)) { pk_drain(mbar, pending, phase); return; }
                if (was_sample0) {
                    if (tid == 0) s_done = *(volatile int *) &P.st->done;
                    __syncthreads();
                    if (s_done) { pk_drain(mbar, pending, phase); return; }
                }
            } else {
                if (tid == 32) side();
                __syncthreads();
            }
        }
    }
    pk_drain(mbar, pending, phase);
}

}  // namespace qtts
