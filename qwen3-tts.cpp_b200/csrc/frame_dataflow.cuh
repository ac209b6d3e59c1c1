// frame_dataflow.cuh — the codec frame as one cooperative launch whose ops hand
// activations to each other as tagged words.
//
// A frame of the batch-1 loop is a strict chain: every GEMV needs the whole
// output vector of the op before it.  On B200 one such all-to-all hand-off
// across the 148 SMs costs ~2.1 us whether it is a grid barrier followed by a
// load or a poll of the data itself, so the frame time is (hand-offs) x (that
// latency + the op's own work).  This kernel cuts both:
//
//   * activations travel as 64-bit words {F32 value, tag} (st_tagged): a
//     consumer polls its input words until they carry the tag of the write it
//     needs, so the data is the synchronisation (no barrier, no separate flag);
//   * every CTA runs the samplers itself (the same decision everywhere, from
//     the same logits and the same Philox draw) and builds the next input rows
//     from the sampled code, so sampling and embedding gathers cost no hand-off;
//   * the code-predictor step attention (<= 16 keys) runs as the O-projection's
//     prologue, one warp per query head, in every CTA: no hand-off either;
//   * each CTA keeps its own rows of the residual stream in shared memory (the
//     O and down projections write the rows they later add to).
//
// A frame is 15 code-predictor passes x (5 layers x 4 GEMVs + head) + 28 talker
// layers x (4 GEMVs + attention) + head = 456 hand-offs (548 launches in the
// CUDA-graph frame).  Arithmetic is the CUDA-graph path's, op for op (the same
// GEMV, attention, sampler and input-sum bodies, the same reduction orders), so
// both give the same bits.
//
// Tags: the write of op k in frame f of a launch carries tag_base + f * n_ops +
// k + 1; a tagged buffer has two slots, the w-th write of a frame going to slot
// (f * writes_per_frame + w) & 1.  A slot is rewritten only after every reader
// of its previous contents has finished: each GEMV uses all CTAs, so a CTA that
// writes version n + 2 has read version n + 1 in full, which every CTA wrote
// after reading version n.
//
// Every spin has an iteration limit; on expiry the kernel sets *err, waits
// (bounded) for its own bulk copies in flight and returns (no GPU trap).
#pragma once
#include "kernels.cuh"

namespace qtts {

constexpr int DF_THREADS = 512;

enum DfOpType : int { DF_GEMV = 1, DF_TATTN = 2 };

// Where a GEMV's activation rows come from.
enum DfPro : int {
    PRO_POLL = 0,      // tagged rows of in_buf
    PRO_CB0 = 1,       // sample codebook 0 (talker logits); rows [talker hidden, codec_embd[cb0]]
    PRO_CBG = 2,       // sample code-predictor codebook cb; row cp_embd[cb - 1][code]
    PRO_CBLAST = 3,    // sample the last codebook; row = the next talker step's input sum
    PRO_CPATTN2 = 4,   // code-predictor 2-row prefill attention (F32 K/V of this pass)
    PRO_CPATTN = 5,    // code-predictor step attention (1 row, F16 cache)
};

// Tagged buffers (two slots each).
enum DfBuf : int { DB_X = 0, DB_XCP, DB_QKV, DB_ATT, DB_H, DB_LCP, DB_LT, DB_N };

struct alignas(16) DfOp {
    int type, pro, nv;
    int in_buf, in_op, in_wr, in_row;   // tagged input: buffer, producer op (< 0: the previous frame's
                                        // op in_op + n_ops), the producer's write index, first row
    int out_buf, out_wr;                // tagged output and this op's write index of it in the frame
    int cb, layer, n_past;              // sampler codebook; attention table entry; CP position
    int slot, act, epi, head;           // weight buffer; activation mode; epilogue; 1: talker codec head
    DMat A, B;
    const float * norm_g;
    DMat iA, iB;                        // slice copied into `slot` once this op is done (iA.w: none)
    const float * iG;
    DMat pA, pB;                        // slice prefetched into L2 once this op is done (pA.w: none)
    const __half * iK, * iV;            // code-predictor K/V rows copied with that slice (iK: none)
    int i_kv_bytes, i_kv_off;           // bytes of each, their offset in the slot
    int kv_off, kv_bytes;               // this op's staged K/V rows (PRO_CPATTN; kv_off < 0: none)
};

struct DfArgs {
    const DfOp * ops;
    int n_ops, n_frames;
    unsigned tag_base;
    unsigned long long * buf[DB_N];     // tagged buffers, two slots each
    int buf_slot[DB_N];                 // words per slot
    int buf_w[DB_N];                    // writes per frame
    const FusedAttn * att;              // attention table: code-predictor layers, then talker layers
    int n_att;
    DevState * st;
    const SampleParams * sp;
    int * out_codes;
    int out_cap;
    int * err;
    const __half * codec_embd;
    const __half * const * cp_embd;     // device array of n_cb - 1 tables
    const float * trailing, * pad;
    const float * logits0;              // talker logits before the launch (frame 0's codebook-0 input)
    float * logits_out;                 // talker logits, written by every frame's head
    float * hidden;                     // talker hidden state: read at launch, written by every frame's head
    float eps;
    int H, n_cb, V0, V1;
    int wbuf_bytes, work_bytes;
    int first[2];                       // the frame's first two GEMV ops (slices copied at launch)
    int n_pf0;
    int pf0[8];                         // GEMV ops prefetched into L2 at launch
    unsigned long long * trace;         // optional [n_frames][n_ops][DF_TRACE] %globaltimer stamps
};
// Trace stamps per op (CTA 0 unless noted): start, input ready, latest input
// ready over the CTAs, weights ready, first output row stored, last output row
// stored, op done (thread 0), next slice copy and prefetches issued, past the
// first end-of-op barrier, past the second.
constexpr int DF_TRACE = 10;

__device__ __forceinline__ unsigned long long df_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void df_prefetch_l2(const void * p, size_t bytes) {
    const char * c = static_cast<const char *>(p);
    while (bytes > 0) {
        const unsigned n = (unsigned)(bytes > 65536 ? 65536 : bytes);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}

// This CTA's row slice of a weight matrix (the GEMV row split) into L2.
__device__ __forceinline__ void df_prefetch_slice(const DMat & M, int cta, int ncta) {
    if (!M.w) return;
    const int rpc = gemv_rpc(M.rows, ncta);
    const int r0 = cta * rpc, r1 = min(M.rows, r0 + rpc);
    if (r0 >= r1) return;
    const size_t es = M.type == W_F16 ? 2 : 1;
    df_prefetch_l2(static_cast<const char *>(M.w) + (size_t) r0 * M.cols * es, (size_t)(r1 - r0) * M.cols * es);
    if (M.type == W_Q8_0) df_prefetch_l2(M.d + (size_t) r0 * (M.cols / 32), (size_t)(r1 - r0) * (M.cols / 32) * 2);
}

__device__ __forceinline__ unsigned df_tag(const DfArgs & P, int f, int op) {
    return P.tag_base + (unsigned) f * (unsigned) P.n_ops + (unsigned) op + 1u;
}
__device__ __forceinline__ unsigned long long * df_slot(const DfArgs & P, int b, int f, int wr) {
    return P.buf[b] + (size_t)((unsigned)(f * P.buf_w[b] + wr) & 1u) * P.buf_slot[b];
}
// The op's tagged input in frame f: producer tag and slot.
__device__ __forceinline__ unsigned df_in_tag(const DfArgs & P, const DfOp & op, int f) {
    return op.in_op < 0 ? df_tag(P, f - 1, op.in_op + P.n_ops) : df_tag(P, f, op.in_op);
}
__device__ __forceinline__ const unsigned long long * df_in(const DfArgs & P, const DfOp & op, int f) {
    return df_slot(P, op.in_buf, op.in_op < 0 ? f - 1 : f, op.in_wr);
}

// Polls word pairs p = tid, tid + nt, ... < npairs of `src` (at most MAXP per
// thread, all in flight together) until both words carry `tag`, handing each
// pair to sink(p, v0, v1).  False when the limit ran out or another CTA
// reported an error.
template <int MAXP, class Addr, class Sink>
__device__ __forceinline__ bool df_poll_pairs_at(int npairs, unsigned tag, const Addr & addr, const Sink & sink,
                                                 const int * err) {
    const int tid = threadIdx.x, nt = blockDim.x;
    unsigned pend = 0u;
#pragma unroll
    for (int k = 0; k < MAXP; ++k)
        if (tid + k * nt < npairs) pend |= 1u << k;
    for (unsigned long long it = 0; pend && it < QTTS_SPIN_LIMIT; ++it) {
        unsigned long long a[MAXP], b[MAXP];
#pragma unroll
        for (int k = 0; k < MAXP; ++k)
            if (pend >> k & 1u) ld_tagged2(addr(tid + k * nt), a[k], b[k]);
#pragma unroll
        for (int k = 0; k < MAXP; ++k)
            if ((pend >> k & 1u) && tag_of(a[k]) == tag && tag_of(b[k]) == tag) {
                sink(tid + k * nt, val_of(a[k]), val_of(b[k]));
                pend &= ~(1u << k);
            }
        if ((it & 255u) == 255u && *(volatile const int *) err) break;
    }
    return pend == 0u;
}
template <int MAXP, class Sink>
__device__ __forceinline__ bool df_poll_pairs(const unsigned long long * src, int npairs, unsigned tag,
                                              const Sink & sink, const int * err) {
    return df_poll_pairs_at<MAXP>(npairs, tag, [&](int p) { return src + 2 * (size_t) p; }, sink, err);
}

// N float quads (two word pairs each) of one lane, all in flight together.
template <int N>
__device__ __forceinline__ bool df_poll_quads(const unsigned long long * const (&src)[N], int n, unsigned tag,
                                              float4 (&out)[N], const int * err) {
    unsigned pend = (1u << n) - 1u;
    for (unsigned long long it = 0; pend && it < QTTS_SPIN_LIMIT; ++it) {
        unsigned long long w[N][4];
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (pend >> k & 1u) {
                ld_tagged2(src[k], w[k][0], w[k][1]);
                ld_tagged2(src[k] + 2, w[k][2], w[k][3]);
            }
#pragma unroll
        for (int k = 0; k < N; ++k)
            if ((pend >> k & 1u) && tag_of(w[k][0]) == tag && tag_of(w[k][1]) == tag && tag_of(w[k][2]) == tag &&
                tag_of(w[k][3]) == tag) {
                out[k] = make_float4(val_of(w[k][0]), val_of(w[k][1]), val_of(w[k][2]), val_of(w[k][3]));
                pend &= ~(1u << k);
            }
        if ((it & 255u) == 255u && *(volatile const int *) err) break;
    }
    return pend == 0u;
}

// Rows [0, nv) of width cols (tagged) into the GEMV work area, two-plane layout.
__device__ __forceinline__ bool df_poll_rows(const unsigned long long * src, int cols, int nv, unsigned tag, float * xs,
                                             const int * err) {
    return df_poll_pairs<6>(src, nv * cols / 2, tag,
                            [&](int p, float v0, float v1) {
                                const int e = 2 * p, v = e / cols, c = e - v * cols;
                                *reinterpret_cast<float2 *>(xs + v * cols + xpos(c, cols)) = make_float2(v0, v1);
                            },
                            err);
}

// Output of a GEMV op: tagged words, optionally a plain copy, and this CTA's
// residual rows when the op advances the residual stream.
struct DfStore {
    unsigned long long * out;
    int ld;
    unsigned tag;
    float * plain;
    float (*res)[8];
    unsigned long long * stamp;   // trace: [0] first row stored, [1] latest row stored (or nullptr)
    __device__ __forceinline__ void operator()(int r, int rl, int v, float val) const {
        st_tagged(out + (size_t) v * ld + r, val, tag);
        if (plain) plain[(size_t) v * ld + r] = val;
        if (res) res[v][rl] = val;
        if (stamp) {
            const unsigned long long t = df_now();
            if (rl == 0 && v == 0) stamp[0] = t;
            atomicMax(stamp + 1, t);
        }
    }
};

// Code-predictor 2-row prefill attention of unit (query head hq, row i), one
// warp, the arithmetic of fused_attn_body in F32 mode for M = 2: rows 0..i of
// this pass are the keys; q and k get the per-head RMSNorm and NEOX RoPE of
// their positions; scores by 8-lane groups of 16 dims each (xor butterfly 4, 2,
// 1); softmax max / exp / double sum / e * (float)(1 / sum); P x V as position
// groups summed in order.  kv_write: append row i's K/V (F16) to the cache.
// Returns the output quad of dims 4 lane .. 4 lane + 3.
__device__ __forceinline__ float4 df_cp_prefill_unit(const FusedAttn & a, int hq, int i, int n_past, const float4 qv,
                                                     const float4 k0, const float4 v0, const float4 k1, const float4 v1,
                                                     bool kv_write) {
    const int lane = threadIdx.x & 31;
    const int NKV = a.n_kv_heads, g = hq / (a.n_heads / NKV);
    const size_t pstride = (size_t) NKV * QTTS_HD;
    float xq[4] = {qv.x, qv.y, qv.z, qv.w};
    head_norm_rope(xq, a.q_norm, a.eps, a.rope + (size_t)(n_past + i) * (QTTS_HD / 2), lane);
    float xk0[4] = {k0.x, k0.y, k0.z, k0.w}, xk1[4] = {k1.x, k1.y, k1.z, k1.w};
    head_norm_rope(xk0, a.k_norm, a.eps, a.rope + (size_t) n_past * (QTTS_HD / 2), lane);
    if (i == 1) head_norm_rope(xk1, a.k_norm, a.eps, a.rope + (size_t)(n_past + 1) * (QTTS_HD / 2), lane);
    if (kv_write) {
        const float4 vi = i == 0 ? v0 : v1;
        const float vq[4] = {vi.x, vi.y, vi.z, vi.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a.kc[(size_t)(n_past + i) * pstride + (size_t) g * QTTS_HD + lane * 4 + k] =
                __float2half_rn(i == 0 ? xk0[k] : xk1[k]);
            a.vc[(size_t)(n_past + i) * pstride + (size_t) g * QTTS_HD + lane * 4 + k] = __float2half_rn(vq[k]);
        }
    }
    // score of key j: the 8-lane group sub = lane & 7 chains dims 16 sub .. 16 sub + 15 (lanes 4 sub .. 4 sub + 3)
    const int sub = lane & 7;
    float sc0, sc1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        float s = 0.0f;
#pragma unroll 1
        for (int dq = 0; dq < 4; ++dq) {   // dims 16 sub + 4 dq + e, in order
            const int src = 4 * sub + dq;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float qd = __shfl_sync(0xffffffffu, xq[e], src);
                const float kd = __shfl_sync(0xffffffffu, j == 0 ? xk0[e] : xk1[e], src);
                s = fmaf(kd, qd, s);
            }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (j == 0) sc0 = __fmul_rn(s, a.scale);
        else sc1 = __fmul_rn(s, a.scale);
    }
    const int n = i + 1;
    const float mx = n == 2 ? fmaxf(sc0, sc1) : sc0;
    const float e0 = qtts_expf(__fsub_rn(sc0, mx));
    const float e1 = n == 2 ? qtts_expf(__fsub_rn(sc1, mx)) : 0.0f;
    const double sum = n == 2 ? (double) e0 + (double) e1 : (double) e0;
    const float inv = (float)(1.0 / sum);
    const float p0 = __fmul_rn(e0, inv), p1 = __fmul_rn(e1, inv);
    const float va[4] = {v0.x, v0.y, v0.z, v0.w}, vb[4] = {v1.x, v1.y, v1.z, v1.w};
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float part0 = fmaf(p0, va[k], 0.0f);
        const float part1 = n == 2 ? fmaf(p1, vb[k], 0.0f) : 0.0f;
        float s = __fadd_rn(0.0f, part0);
        s = __fadd_rn(s, part1);
        o[k] = __fadd_rn(s, 0.0f);   // the position groups with no key
    }
    return make_float4(o[0], o[1], o[2], o[3]);
}

// Waits (bounded) for the copies still in flight into either weight buffer.
__device__ __forceinline__ void df_drain(uint64_t * mbar, unsigned pending, unsigned phase) {
    if (threadIdx.x != 0) return;
    for (int b = 0; b < 2; ++b)
        if (pending >> b & 1u) mbar_wait(mbar + b, phase >> b & 1u);
}

// ---- per-CTA state of the kernel (shared memory).  Everything the stages
// keep per thread lives in registers: with ~215 KB of shared memory per SM the
// L1 cache left for local memory is small, and a spilled register or a stack
// frame would cost an L2 round trip per access.
__shared__ DfArgs df_P;                  // the launch arguments
__shared__ DfOp df_desc[3];              // ring: this op's descriptor, the next one's, and the one
                                         // before, which the issuing warp may still be reading
__shared__ __align__(8) uint64_t df_mbar[2];
__shared__ DevState df_st;               // this CTA's frame state (presence set, codes)
__shared__ SampleParams df_sp;
__shared__ float df_res[2][8];           // this CTA's rows of the residual stream
__shared__ const __half * df_tab[QTTS_MAX_CB];
__shared__ int df_bad;
__shared__ GemvArgs df_gemv;             // this op's GEMV arguments (built by thread 0)
extern __shared__ __align__(128) uint8_t df_smem[];

__device__ __forceinline__ uint8_t * df_work() { return df_smem + 2 * (size_t) df_P.wbuf_bytes; }
__device__ __forceinline__ FusedAttn * df_att() { return reinterpret_cast<FusedAttn *>(df_work() + df_P.work_bytes); }
__device__ __forceinline__ float * df_hid() { return reinterpret_cast<float *>(df_att() + df_P.n_att); }

// The op's activation rows from a tagged buffer.
__device__ __forceinline__ bool df_stage_poll(const DfOp & op, int f, float * xs) {
    const int cols = op.A.cols;
    return df_poll_rows(df_in(df_P, op, f) + (size_t) op.in_row * cols, cols, op.nv, df_in_tag(df_P, op, f), xs,
                        df_P.err);
}

// Sampler prologue: sample codebook op.cb (every CTA, the same decision), then
// the pass's input rows into xs and this CTA's residual rows.  Returns 1 when
// codebook 0 sampled EOS (the launch ends), -1 when an input did not arrive.
__device__ __forceinline__ int df_stage_sample(const DfOp & op, int f, int frame, float * xs) {
    const DfArgs & P = df_P;
    const int tid = threadIdx.x, nt = blockDim.x, cta = blockIdx.x;
    const int cb = op.cb, V = cb == 0 ? P.V0 : P.V1, H = P.H;
    int tok;
    if (cb == 0 && f == 0) {
        tok = sample_body_l<8>(
            [&](float * l) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int i = tid * 8 + e;
                    l[e] = i < V ? __ldcg(P.logits0 + i) : -INFINITY;
                }
            },
            V, cb, &df_st, df_sp, frame);
    } else {
        const unsigned long long * src = df_in(P, op, f);
        const unsigned tag = df_in_tag(P, op, f);
        tok = sample_body_l<8>(
            [&](float * l) {
#pragma unroll
                for (int e = 0; e < 8; ++e) l[e] = -INFINITY;
                const int np = max(0, min(4, (V - tid * 8) / 2));
                unsigned pend = (1u << np) - 1u;
                for (unsigned long long it = 0; pend && it < QTTS_SPIN_LIMIT; ++it) {
                    unsigned long long a[4], b[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if (pend >> q & 1u) ld_tagged2(src + tid * 8 + 2 * q, a[q], b[q]);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        if ((pend >> q & 1u) && tag_of(a[q]) == tag && tag_of(b[q]) == tag) {
                            l[2 * q] = val_of(a[q]);
                            l[2 * q + 1] = val_of(b[q]);
                            pend &= ~(1u << q);
                        }
                    if ((it & 255u) == 255u && *(volatile const int *) P.err) break;
                }
                if (pend) df_bad = 1;
            },
            V, cb, &df_st, df_sp, frame);
    }
    __syncthreads();
    if (df_bad) return -1;
    if (cb == 0 && tok == df_sp.eos_id) {
        if (cta == 0 && tid == 0) sample_commit(tok, 0, P.st, df_sp, P.out_codes, P.out_cap, frame);
        return 1;
    }
    if (tid == 0) {
        df_st.codes[cb] = tok;
        if (cb == 0) df_st.presence[tok >> 5] |= 1u << (tok & 31);
        if (cta == 0) sample_commit(tok, cb, P.st, df_sp, P.out_codes, P.out_cap, frame);
    }
    __syncthreads();
    // input rows of the pass (same values and sums as frame_inputs_body)
    const int rpc_h = gemv_rpc(H, gridDim.x), r0_h = cta * rpc_h;
    const int nrow_h = max(0, min(H, r0_h + rpc_h) - r0_h);
    const float * hid = df_hid();
    const int n_tr = df_st.n_trailing;
    for (int c = tid; c < H; c += nt) {
        float x0, x1 = 0.0f;
        if (op.pro == PRO_CB0) {
            x0 = hid[c];
            x1 = __half2float(P.codec_embd[(size_t) tok * H + c]);
        } else if (op.pro == PRO_CBG) {
            x0 = __half2float(df_tab[cb][(size_t) tok * H + c]);
        } else {
            float s = __half2float(P.codec_embd[(size_t) df_st.codes[0] * H + c]);
            for (int q = 1; q < P.n_cb; ++q) s = __fadd_rn(s, __half2float(df_tab[q][(size_t) df_st.codes[q] * H + c]));
            const float t = frame < n_tr ? P.trailing[(size_t) frame * H + c] : P.pad[c];
            x0 = __fadd_rn(s, t);
        }
        xs[xpos(c, H)] = x0;
        if (op.nv == 2) xs[H + xpos(c, H)] = x1;
        const int rl = c - r0_h;
        if (rl >= 0 && rl < nrow_h) {
            df_res[0][rl] = x0;
            df_res[1][rl] = x1;
        }
    }
    return 0;
}

// Code-predictor attention into the O-projection's input rows (xs, QD columns):
// steps one warp per query head, the 2-row prefill one warp per (head, row).
// CTA 0 appends the new K/V rows to the cache.  False when an input did not arrive.
__device__ __forceinline__ bool df_stage_cp_attn(const DfOp & op, int f, float * xs, unsigned parity) {
    const DfArgs & P = df_P;
    const FusedAttn & a = df_att()[op.layer];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int NH = a.n_heads, G = NH / a.n_kv_heads;
    const int QD = NH * QTTS_HD, KD = a.n_kv_heads * QTTS_HD;
    const unsigned long long * q = df_in(P, op, f);
    const unsigned tag = df_in_tag(P, op, f);
    bool wrote = false, ok = true;
    if (op.pro == PRO_CPATTN) {
        // the cached K/V rows arrived with this op's weight slice (same mbarrier phase)
        uint8_t * wb = df_smem + (size_t) op.slot * P.wbuf_bytes;
        const bool landed = threadIdx.x != 0 || mbar_wait(df_mbar + op.slot, parity);
        float4 in[3];
        int hq = warp;
        bool got = true;
        if (hq < NH) {
            const int g = hq / G;
            const unsigned long long * const srcs[3] = {q + (size_t) hq * QTTS_HD + lane * 4,
                                                        q + QD + (size_t) g * QTTS_HD + lane * 4,
                                                        q + QD + KD + (size_t) g * QTTS_HD + lane * 4};
            got = __all_sync(0xffffffffu, df_poll_quads<3>(srcs, 3, tag, in, P.err));
        }
        if (__syncthreads_or(!landed || !got)) return false;
        for (; hq < NH; hq += nw) {
            const int g = hq / G;
            if (hq != warp) {   // more heads than warps: poll this head's rows now
                const unsigned long long * const srcs[3] = {q + (size_t) hq * QTTS_HD + lane * 4,
                                                            q + QD + (size_t) g * QTTS_HD + lane * 4,
                                                            q + QD + KD + (size_t) g * QTTS_HD + lane * 4};
                if (!__all_sync(0xffffffffu, df_poll_quads<3>(srcs, 3, tag, in, P.err))) { ok = false; break; }
            }
            CpStepRegs R;
            const float2 * rp = a.rope + (size_t) op.n_past * (QTTS_HD / 2);
            head_params(a.q_norm, rp, lane, R.gq, R.cs);
            head_params(a.k_norm, rp, lane, R.gk, R.cs);
            const CpKvSmem kv{reinterpret_cast<const __half *>(wb + op.kv_off),
                              reinterpret_cast<const __half *>(wb + op.kv_off + op.kv_bytes), g, a.n_kv_heads};
            const bool w = blockIdx.x == 0 && hq % G == 0;
            const float4 o = cp_step_compute_kv(a, hq, op.n_past, R, kv, in[0], in[1], in[2], w);
            wrote |= w;
            *reinterpret_cast<float4 *>(xs + xpos(hq * QTTS_HD + lane * 4, QD)) = o;
        }
    } else {
        const int QKVD = QD + 2 * KD;
        for (int u = warp; u < 2 * NH; u += nw) {
            const int hq = u % NH, i = u / NH, g = hq / G;
            const unsigned long long * const srcs[5] = {q + (size_t) i * QKVD + (size_t) hq * QTTS_HD + lane * 4,
                                                        q + QD + (size_t) g * QTTS_HD + lane * 4,
                                                        q + QD + KD + (size_t) g * QTTS_HD + lane * 4,
                                                        q + QKVD + QD + (size_t) g * QTTS_HD + lane * 4,
                                                        q + QKVD + QD + KD + (size_t) g * QTTS_HD + lane * 4};
            float4 in[5] = {};
            if (!__all_sync(0xffffffffu, df_poll_quads<5>(srcs, i == 0 ? 3 : 5, tag, in, P.err))) { ok = false; break; }
            const bool w = blockIdx.x == 0 && hq % G == 0;
            const float4 o = df_cp_prefill_unit(a, hq, i, op.n_past, in[0], in[1], in[2], in[3], in[4], w);
            wrote |= w;
            *reinterpret_cast<float4 *>(xs + i * QD + xpos(hq * QTTS_HD + lane * 4, QD)) = o;
        }
    }
    if (wrote) __threadfence();   // the cache rows before this CTA's tagged outputs
    return ok;
}

// Talker attention, one query head per CTA (CTAs 0 .. n_heads - 1): the head's q
// and its group's k / v into a full-row staging area, then the fused unit with a
// tagged output.  Returns false when an input did not arrive.
__device__ __forceinline__ bool df_stage_talker_attn(const DfOp & op, int f, int k, int n_past, int frame) {
    const DfArgs & P = df_P;
    const FusedAttn & a0 = df_att()[op.layer];
    const int NH = a0.n_heads, G = NH / a0.n_kv_heads;
    const int QD = NH * QTTS_HD, KD = a0.n_kv_heads * QTTS_HD;
    const int hq = blockIdx.x, g = hq / G;
    __syncthreads();   // everyone has read the entry's sizes before thread 0 updates it
    uint8_t * work = df_work();
    float * stage = reinterpret_cast<float *>(work);
    const unsigned long long * q = df_in(P, op, f);
    // pair p < 64: q of head hq; 64..127: k of group g; 128..191: v of group g
    auto off = [&](int p) {
        const int part = p / (QTTS_HD / 2), c = 2 * (p % (QTTS_HD / 2));
        return (part == 0 ? hq * QTTS_HD : QD + (part == 2 ? KD : 0) + g * QTTS_HD) + c;
    };
    const bool ok = df_poll_pairs_at<1>(3 * QTTS_HD / 2, df_in_tag(P, op, f), [&](int p) { return q + off(p); },
                                        [&](int p, float v0, float v1) {
                                            *reinterpret_cast<float2 *>(stage + off(p)) = make_float2(v0, v1);
                                        },
                                        P.err);
    fence_acq_rel_gpu();   // the cached K/V rows other CTAs appended are read after this
    // this CTA's own copy of the table entry takes the staging area and the tagged output
    // (a local copy of the struct would live in local memory)
    FusedAttn & a = df_att()[op.layer];
    if (threadIdx.x == 0) {
        a.qkv = stage;
        a.fout = df_slot(P, op.out_buf, f, op.out_wr);
        a.ftag = df_tag(P, f, k);
    }
    if (__syncthreads_or(!ok)) return false;
    fused_attn_body(a, hq, work + ((size_t)(QD + 2 * KD) * 4 + 127) / 128 * 128, n_past, frame);
    return true;
}

// The op's GEMV with its activation rows in xs: residual rows from df_res,
// tagged outputs (the talker head also writes the plain logits, the hidden
// state in every CTA's df_hid and, in CTA 0, the plain hidden state).
template <int NV>
__device__ __forceinline__ bool df_stage_gemv(const DfOp & op, int f, int k, unsigned parity,
                                           unsigned long long * ready_stamp) {
    const DfArgs & P = df_P;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x, nt = blockDim.x;
    const int rpc = gemv_rpc(op.A.rows, ncta);
    const GemvWork W = gemv_work<NV>(df_work(), op.A.cols, rpc, op.A.type == W_Q8_0);
    if (op.epi == EPI_RESID) {
        const int H = P.H, r0 = cta * rpc, nrow = max(0, min(H, r0 + rpc) - r0);
        const int rstride = (rpc + 3) & ~3;
        for (int t = tid; t < NV * nrow; t += nt) W.rs[(t / nrow) * rstride + t % nrow] = df_res[t / nrow][t % nrow];
    }
    GemvArgs & g = df_gemv;   // in shared memory: a local copy of the struct would live in local memory
    if (tid == 0) {
        g = GemvArgs{};
        g.A = op.A;
        g.B = op.B;
        g.nv = NV;
        g.norm_g = op.norm_g;
        g.eps = P.eps;
        g.act = op.act;
        g.epi = op.epi;
        g.xn_out = op.head == 1 ? P.hidden : nullptr;   // CTA 0: the plain talker hidden state
        g.ldxn = P.H;
    }
    __syncthreads();
    const DfStore store{df_slot(P, op.out_buf, f, op.out_wr), op.A.rows, df_tag(P, f, k),
                        op.head == 1 ? P.logits_out : nullptr, op.epi == EPI_RESID ? df_res : nullptr,
                        ready_stamp ? ready_stamp + 1 : nullptr};
    const int b = op.slot;
    return gemv_compute<NV>(g, cta, ncta, df_smem + (size_t) b * P.wbuf_bytes, df_work(), df_mbar + b, parity, store,
                            op.head == 1 ? df_hid() : nullptr, ready_stamp);
}

__shared__ int df_pos0, df_frame0;     // frame state at launch

// Trace stamps of op k in frame f (nullptr when tracing is off).  Recomputed at
// each use so no register holds it across a stage.
__device__ __forceinline__ unsigned long long * df_tr(int f, int k) {
    return df_P.trace ? df_P.trace + ((size_t) f * df_P.n_ops + k) * DF_TRACE : nullptr;
}
__device__ __forceinline__ void df_stamp(int f, int k, int slot) {
    unsigned long long * tr = df_tr(f, k);
    if (tr && blockIdx.x == 0 && threadIdx.x == 0) tr[slot] = df_now();
}

// Loop state is kept to a few registers (frame, op, weight-buffer phases, two
// flags): every stage below gets the rest of the 128 a thread has.
__global__ void __launch_bounds__(DF_THREADS, 1) k_frame_dataflow(DfArgs Pk) {
    constexpr int NW = (int)(sizeof(DfOp) / 8);
    static_assert(sizeof(DfOp) % 8 == 0 && NW <= DF_THREADS, "descriptor copy");
    static_assert(sizeof(FusedAttn) % 8 == 0 && sizeof(DfArgs) % 8 == 0, "table copies");
    {
        const unsigned long long * src = reinterpret_cast<const unsigned long long *>(&Pk);
        for (int w = threadIdx.x; w < (int)(sizeof(DfArgs) / 8); w += blockDim.x)
            reinterpret_cast<unsigned long long *>(&df_P)[w] = src[w];
    }
    if (threadIdx.x == 0) {
        mbar_init(&df_mbar[0], 1);
        mbar_init(&df_mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        df_sp = *Pk.sp;
        if (blockIdx.x != 0) df_sp.record_logits = 0;   // CTA 0 records the debug logits
        df_bad = 0;
    }
    if (threadIdx.x < NW)
        reinterpret_cast<unsigned long long *>(&df_desc[0])[threadIdx.x] = reinterpret_cast<const unsigned long long *>(Pk.ops)[threadIdx.x];
    __syncthreads();
    {
        const DfArgs & P = df_P;
        const int tid = threadIdx.x, nt = blockDim.x;
        const int n8 = P.n_att * (int)(sizeof(FusedAttn) / 8);
        for (int w = tid; w < n8; w += nt)
            reinterpret_cast<unsigned long long *>(df_att())[w] = reinterpret_cast<const unsigned long long *>(P.att)[w];
        for (int i = tid; i < (int)(sizeof(DevState) / 4); i += nt)
            reinterpret_cast<int *>(&df_st)[i] = reinterpret_cast<const volatile int *>(P.st)[i];
        for (int c = tid; c < P.H; c += nt) df_hid()[c] = __ldcg(P.hidden + c);
        if (tid >= 1 && tid < P.n_cb) df_tab[tid] = P.cp_embd[tid - 1];
        __syncthreads();
        if (tid == 0) {
            df_pos0 = df_st.pos;
            df_frame0 = df_st.frame;
            for (int k = 0; k < P.n_pf0; ++k) {
                df_prefetch_slice(P.ops[P.pf0[k]].A, blockIdx.x, gridDim.x);
                df_prefetch_slice(P.ops[P.pf0[k]].B, blockIdx.x, gridDim.x);
            }
            for (int b = 0; b < 2; ++b) {
                const DfOp & g = P.ops[P.first[b]];
                issue_gemv_slice(g.A, g.B, g.norm_g, df_smem + (size_t) g.slot * P.wbuf_bytes, df_mbar + g.slot,
                                 blockIdx.x, gridDim.x);
            }
        }
        __syncthreads();
    }
    unsigned phase = 0u, pending = 3u;
    bool stop = false, failed = false;

    unsigned seq = 0;   // ops run so far in this launch (descriptor ring position)
    for (int f = 0; f < df_P.n_frames && !stop && !failed; ++f) {
        for (int k = 0; k < df_P.n_ops; ++k, ++seq) {
            const DfOp & op = df_desc[seq % 3];
            df_stamp(f, k, 0);
            // The next op's descriptor goes to the slot of op k - 2: every warp, the
            // issuing warp included, finished with it before op k - 1's end barrier.
            if (threadIdx.x < NW) {
                const int nx = k + 1 < df_P.n_ops ? k + 1 : 0;
                reinterpret_cast<unsigned long long *>(&df_desc[(seq + 1) % 3])[threadIdx.x] =
                    reinterpret_cast<const unsigned long long *>(df_P.ops + nx)[threadIdx.x];
            }
            if (op.type == DF_GEMV) {
                float * xs = reinterpret_cast<float *>(df_work());
                int rc = 0;
                if (op.pro == PRO_POLL) rc = df_stage_poll(op, f, xs) ? 0 : -1;
                else if (op.pro == PRO_CPATTN || op.pro == PRO_CPATTN2)
                    rc = df_stage_cp_attn(op, f, xs, phase >> op.slot & 1u) ? 0 : -1;
                else rc = df_stage_sample(op, f, df_frame0 + f, xs);
                if (__syncthreads_or(rc < 0)) {
                    failed = true;
                } else if (rc == 1) {
                    stop = true;
                } else {
                    unsigned long long * tr = df_tr(f, k);
                    if (tr && threadIdx.x == 0) {
                        const unsigned long long t = df_now();
                        if (blockIdx.x == 0) tr[1] = t;
                        atomicMax(tr + 2, t);
                    }
                    const int b = op.slot;
                    unsigned long long * rs = tr && blockIdx.x == 0 ? tr + 3 : nullptr;
                    const bool gok = op.nv == 1 ? df_stage_gemv<1>(op, f, k, phase >> b & 1u, rs)
                                                : df_stage_gemv<2>(op, f, k, phase >> b & 1u, rs);
                    if (!gok) failed = true;
                    phase ^= 1u << b;
                    pending &= ~(1u << b);
                }
            } else if ((int) blockIdx.x < df_att()[op.layer].n_heads) {   // DF_TATTN: CTAs 0 .. n_heads - 1
                if (!df_stage_talker_attn(op, f, k, df_pos0 + f, df_frame0 + f)) failed = true;
            }
            if (failed) {
                if (threadIdx.x == 0) atomicExch(df_P.err, 2);
                break;
            }
            if (stop) break;
            df_stamp(f, k, 6);
            __syncthreads();   // everyone is done with op k's descriptor and weight buffer
            df_stamp(f, k, 8);
            // The last warp issues the next copies into op k's buffer and then joins op k + 1;
            // the others start op k + 1 at once (its descriptor was stored before this barrier,
            // and it uses the other buffer and mbarrier).
            if (op.type == DF_GEMV && threadIdx.x == blockDim.x - 32) {
                if (op.iA.w) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    uint8_t * wb = df_smem + (size_t) op.slot * df_P.wbuf_bytes;
                    issue_gemv_slice(op.iA, op.iB, op.iG, wb, df_mbar + op.slot, blockIdx.x, gridDim.x,
                                     op.iK ? 2u * (unsigned) op.i_kv_bytes : 0u);
                    if (op.iK) {   // the next op's code-predictor K/V rows, behind its slice
                        bulk_g2s(wb + op.i_kv_off, op.iK, (unsigned) op.i_kv_bytes, df_mbar + op.slot);
                        bulk_g2s(wb + op.i_kv_off + op.i_kv_bytes, op.iV, (unsigned) op.i_kv_bytes, df_mbar + op.slot);
                    }
                }
                df_prefetch_slice(op.pA, blockIdx.x, gridDim.x);
                df_prefetch_slice(op.pB, blockIdx.x, gridDim.x);
                unsigned long long * tr = df_tr(f, k);
                if (tr && blockIdx.x == 0) tr[7] = df_now();
            }
            if (op.type == DF_GEMV && op.iA.w) pending |= 1u << op.slot;
        }
        if (failed || stop) break;
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            df_P.st->pos = df_pos0 + f + 1;
            df_P.st->frame = df_frame0 + f + 1;
            df_P.st->n_out += 1;
        }
    }
    __syncthreads();   // the issuing warp's last copies are posted before thread 0 waits for them
    df_drain(df_mbar, pending, phase);
}

}  // namespace qtts
