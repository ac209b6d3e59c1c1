// batch_engine.cuh — the frame loop for B independent utterances on one GPU
// (BASELINE configs 4 and 5: batched F16 serving, paged F16 KV cache).
//
// One frame for all B sequences is one CUDA graph: every projection is a
// tcgen05 tensor-core GEMM over the B (or 2B) activation rows (gemm_tc.cuh),
// the code predictor's attention runs the fused unit per (sequence, head,
// row), the talker's attention streams each sequence's KV pages through shared
// memory with bulk copies (one CTA per (sequence, kv head), exact two-pass
// softmax as ggml_soft_max), and samplers / input builders run one CTA per
// sequence.  Sequences keep their own frame state (position, codes, presence
// set, EOS flag), so they may have different prompt lengths and stop at
// different frames; a finished sequence's rows are still multiplied (the GEMM
// is one pass over the weights either way) but its attention, sampling and
// state are frozen.
//
// KV pages: BP_PAGE positions of every talker layer, laid out
// [page][layer][K|V][kv_head][BP_PAGE][128] F16, so one (page, layer, head)
// block of K or V is 16 KB contiguous (one bulk copy).  A sequence's pages come
// from a pool through its row of the page table.  This file is included into
// engine.cu after the Engine definition (it shares the Engine's weights).
#pragma once

namespace qtts {

constexpr int BP_PAGE = 64;           // positions per KV page
constexpr int PA_THREADS = 256;
constexpr int PA_RING = 4;            // page blocks in flight per CTA (two CTAs per SM)

__host__ __device__ inline size_t bp_page_elems(int n_layers, int nkv) {
    return (size_t) n_layers * 2 * nkv * BP_PAGE * QTTS_HD;
}
__host__ __device__ inline size_t bp_off(int page, int layer, int kv, int head, int p, int n_layers, int nkv) {
    return ((((size_t) page * n_layers + layer) * 2 + kv) * nkv + head) * (size_t) BP_PAGE * QTTS_HD +
           (size_t) p * QTTS_HD;
}

// ---- talker attention over paged KV ---------------------------------------
struct PagedAttnArgs {
    float * qkv;              // [B][ldq] raw q|k|v rows
    int ldq;
    int n_heads, n_kv_heads, n_layers, layer;
    const float * q_norm, * k_norm;
    float eps;
    const float2 * rope;      // [pos][64]
    __half * pool;
    const int * page_table;   // [B][max_pages]
    int max_pages;
    const DevState * st;      // [B]
    float scale;
    float * out;              // [B][ldo]
    int ldo;
    int n_max;                // capacity of the score buffer (positions of one CTA's page range)
    uint8_t * xt;             // optional: output also as F16 tiles (row b) for the O-projection GEMM
    int xt_np;
    int nsplit;               // CTAs per (sequence, kv head) along the pages (1: one CTA, exact softmax)
    float * part;             // nsplit > 1: [B][NKV][nsplit][G][PA_PART] = max, sum, unnormalised P x V
};
constexpr int PA_PART = QTTS_HD + 2;

__device__ __forceinline__ void mbar_arrive_one(uint64_t * m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(m)) : "memory");
}
// OR of a predicate over the compute warps (named barrier 1, PA_THREADS threads).
__device__ __forceinline__ bool pa_sync_or(bool p) {
    unsigned r;
    asm volatile("{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred o, 1, %2, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
                 : "=r"(r) : "r"((unsigned) p), "r"(PA_THREADS) : "memory");
    return r != 0;
}
constexpr int PA_MAX_SPLIT = 16;

__host__ __device__ inline size_t paged_attn_smem(int n_max, int G) {
    return (size_t) PA_RING * BP_PAGE * QTTS_HD * 2 + (size_t) G * ((n_max + 3) & ~3) * 4 + (size_t) G * QTTS_HD * 4 +
           2 * QTTS_HD * 4 + (size_t)(PA_THREADS / 64) * G * QTTS_HD * 4 + 256;
}

// One CTA per (sequence b, kv head g), or per (b, g, page range) when split
// (a.nsplit > 1, long contexts at small batches): the G query heads of the
// group share every K/V load.  Item i of the stream is page pg0 + (i mod npr)
// of K (i < npr) or V.  Unsplit: exact two-pass softmax as ggml_soft_max
// (global max, exp, double sum, p = e * (float)(1/sum) rounded to F16, P x V).
// Split (flash-decoding): each range writes its local max m, sum l of
// e = exp(s - m) and the unnormalised sum of e * V; k_attn_combine merges the
// ranges in order (no F16 rounding of p there).
//
// Pipeline: warp PA_WARPS (the producer) keeps PA_RING page blocks in flight
// through full / empty mbarriers; the eight compute warps wait on a slot's full
// barrier themselves and release it with one arrival each, so no block-wide
// barrier sits between pages (named barrier 1 joins the compute warps only
// where the softmax needs every score).  Each lane keeps its 16 query dims of
// the G heads in registers.
constexpr int PA_WARPS = PA_THREADS / 32;          // compute warps
constexpr int PA_BLOCK = PA_THREADS + 32;          // + the producer warp

__device__ __forceinline__ void pa_sync_compute() { asm volatile("bar.sync 1, %0;" ::"r"(PA_THREADS) : "memory"); }

template <int G>
__device__ __forceinline__ void attn_paged_body(const PagedAttnArgs & a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[PA_RING], empty[PA_RING];
    __shared__ float s_ml[ATT_MAX_GROUP][2];
    __shared__ int s_bad;
    const int NKV = a.n_kv_heads, NS = a.nsplit > 1 ? a.nsplit : 1;
    const int b = blockIdx.x / (NKV * NS), g = (blockIdx.x / NS) % NKV, sp = blockIdx.x % NS;
    const DevState & S = a.st[b];
    if (S.done) return;
    const int pos = S.pos, n = pos + 1, np_all = (n + BP_PAGE - 1) / BP_PAGE;
    const int chunk = (np_all + NS - 1) / NS;
    const int pg0 = min(np_all, sp * chunk), npr = min(np_all, pg0 + chunk) - pg0;   // this CTA's pages
    const int j0 = pg0 * BP_PAGE;                                                    // first position
    const int n_loc = min(n, (pg0 + npr) * BP_PAGE) - j0;                            // positions here
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nk4 = (n_loc + 3) & ~3;
    const bool has_pos = pos >= j0 && pos < j0 + n_loc;                              // the new row is here
    if (NS > 1 && npr <= 0) {   // an empty range: a neutral partial
        for (int t = tid; t < G * PA_PART; t += blockDim.x) {
            const int h = t / PA_PART, e = t % PA_PART;
            a.part[((((size_t) b * NKV + g) * NS + sp) * G + h) * PA_PART + e] = e == 0 ? -INFINITY : 0.0f;
        }
        return;
    }
    const int np = npr, nitems = 2 * np;
    __half * ring = reinterpret_cast<__half *>(smem);
    float * sc = reinterpret_cast<float *>(smem + (size_t) PA_RING * BP_PAGE * QTTS_HD * 2);   // [G][nk4]
    float * qs = sc + G * ((a.n_max + 3) & ~3);                                                  // [G][128]
    float * kcur = qs + G * QTTS_HD;                                                             // [128]
    float * vcur = kcur + QTTS_HD;                                                               // [128]
    float * part = vcur + QTTS_HD;                                                               // [4][G][128]
    const int * pt = a.page_table + (size_t) b * a.max_pages;
    const int QD = a.n_heads * QTTS_HD, KD = NKV * QTTS_HD;
    const unsigned blk = BP_PAGE * QTTS_HD * 2;
    if (tid == 0) {
        for (int s = 0; s < PA_RING; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], PA_WARPS); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_bad = 0;
    }
    __syncthreads();

    if (warp == PA_WARPS) {
        // producer: page blocks of K then V through the ring
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nitems; ++i) {
                const int s = i % PA_RING;
                if (i >= PA_RING) {
                    if (!mbar_wait(&empty[s], ((i / PA_RING) - 1) & 1)) { s_bad = 1; break; }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
                const int kv = i >= np, page = pg0 + i % np;
                mbar_expect_tx(&full[s], blk);
                bulk_g2s(ring + (size_t) s * BP_PAGE * QTTS_HD,
                         a.pool + bp_off(pt[page], a.layer, kv, g, 0, a.n_layers, NKV), blk, &full[s]);
                issued = i + 1;
            }
            // no copy may be in flight when the CTA exits: wait (bounded) for the last ones
            for (int i = issued > PA_RING ? issued - PA_RING : 0; i < issued; ++i)
                mbar_wait(&full[i % PA_RING], (i / PA_RING) & 1);
        }
        return;
    }

    // q heads and the new k/v row (the row is also appended to its page)
    const float * row = a.qkv + (size_t) b * a.ldq;
    if (warp < G) {
        const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
        const float4 q4 = *reinterpret_cast<const float4 *>(row + (size_t)(g * G + warp) * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.q_norm, rp, lane, gv, cs);
        float x[4] = {q4.x, q4.y, q4.z, q4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) qs[warp * QTTS_HD + lane * 4 + k] = round_f16(x[k]);
    } else if (warp == G && has_pos) {
        const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
        const float4 k4 = *reinterpret_cast<const float4 *>(row + QD + g * QTTS_HD + lane * 4);
        const float4 v4 = *reinterpret_cast<const float4 *>(row + QD + KD + g * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.k_norm, rp, lane, gv, cs);
        float x[4] = {k4.x, k4.y, k4.z, k4.w};
        const float v[4] = {v4.x, v4.y, v4.z, v4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
        const int pg = pt[pos / BP_PAGE], p = pos % BP_PAGE;
        __half * kd = a.pool + bp_off(pg, a.layer, 0, g, p, a.n_layers, NKV) + lane * 4;
        __half * vd = a.pool + bp_off(pg, a.layer, 1, g, p, a.n_layers, NKV) + lane * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half kh = __float2half_rn(x[k]), vh = __float2half_rn(v[k]);
            kd[k] = kh;
            vd[k] = vh;
            kcur[lane * 4 + k] = __half2float(kh);
            vcur[lane * 4 + k] = __half2float(vh);
        }
    }
    pa_sync_compute();

    // scores: per page, 8 lanes per position (16 dims each), 4 positions per warp step
    const int sub = lane & 7, slot = lane >> 3;
    float qr[G][16];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 16; ++d) qr[h][d] = qs[h * QTTS_HD + sub * 16 + d];
    bool ok = true;
    for (int i = 0; i < np; ++i) {
        const int s = i % PA_RING;
        bool got = true;
        if (lane == 0) got = mbar_wait(&full[s], (i / PA_RING) & 1);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (!got) { ok = false; break; }
        const __half * kb = ring + (size_t) s * BP_PAGE * QTTS_HD;
        for (int p0 = warp * 4; p0 < BP_PAGE; p0 += PA_WARPS * 4) {
            const int p = p0 + slot, j = i * BP_PAGE + p;   // j: position within this CTA's range
            float kv[16];
            if (j + j0 == pos) {
#pragma unroll
                for (int d = 0; d < 16; ++d) kv[d] = kcur[sub * 16 + d];
            } else {
                const uint4 * kp = reinterpret_cast<const uint4 *>(kb + (size_t) p * QTTS_HD + sub * 16);
#pragma unroll
                for (int h8 = 0; h8 < 2; ++h8) {
                    const uint4 u = kp[h8];
                    const __half2 * hp = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = __half22float2(hp[k]);
                        kv[8 * h8 + 2 * k] = f.x;
                        kv[8 * h8 + 2 * k + 1] = f.y;
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float acc = 0.0f;
#pragma unroll
                for (int d = 0; d < 16; ++d) acc = fmaf(kv[d], qr[h][d], acc);
                acc += __shfl_xor_sync(0xffffffffu, acc, 4);
                acc += __shfl_xor_sync(0xffffffffu, acc, 2);
                acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                if (sub == 0 && j < n_loc) sc[h * nk4 + j] = __fmul_rn(acc, a.scale);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_one(&empty[s]);   // this warp is done with slot s
    }
    // softmax per head: max, expf, double sum, e * (float)(1/sum), rounded to F16
    // (split: the range's max and sum go to the partial, e stays unnormalised)
    ok = !pa_sync_or(!ok);
    if (ok && warp < G) {
        float * r = sc + warp * nk4;
        float mx = -INFINITY;
        for (int j = lane; j < n_loc; j += 32) mx = fmaxf(mx, r[j]);
        mx = warp_max(mx);
        double sum = 0.0;
        for (int j = lane; j < n_loc; j += 32) {
            const float e = qtts_expf(__fsub_rn(r[j], mx));
            r[j] = e;
            sum += (double) e;
        }
        sum = warp_sum_d(sum);
        if (NS > 1) {
            if (lane == 0) { s_ml[warp][0] = mx; s_ml[warp][1] = (float) sum; }
        } else {
            const float inv = (float)(1.0 / sum);
            for (int j = lane; j < n_loc; j += 32) r[j] = round_f16(__fmul_rn(r[j], inv));
        }
    }
    pa_sync_compute();
    // P x V: thread (position group pq, dims 2 d2 .. 2 d2 + 1) for all G heads
    const int pq = tid >> 6, d2 = tid & 63;
    float acc[G][2];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = 0.0f;
    for (int i = np; ok && i < nitems; ++i) {
        const int s = i % PA_RING, page = i - np;
        bool got = true;
        if (lane == 0) got = mbar_wait(&full[s], (i / PA_RING) & 1);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (!got) { ok = false; break; }
        const __half * vb = ring + (size_t) s * BP_PAGE * QTTS_HD;
        for (int p = pq; p < BP_PAGE; p += PA_THREADS / 64) {
            const int j = page * BP_PAGE + p;   // position within this CTA's range
            if (j >= n_loc) break;
            float2 v;
            if (j + j0 == pos) v = make_float2(vcur[2 * d2], vcur[2 * d2 + 1]);
            else v = __half22float2(*reinterpret_cast<const __half2 *>(vb + (size_t) p * QTTS_HD + 2 * d2));
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pj = sc[h * nk4 + j];
                acc[h][0] = fmaf(pj, v.x, acc[h][0]);
                acc[h][1] = fmaf(pj, v.y, acc[h][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_one(&empty[s]);
    }
    ok = !pa_sync_or(!ok);
    if (!ok) return;   // (the producer drains the copies still in flight)
#pragma unroll
    for (int h = 0; h < G; ++h) {
        part[(pq * G + h) * QTTS_HD + 2 * d2] = acc[h][0];
        part[(pq * G + h) * QTTS_HD + 2 * d2 + 1] = acc[h][1];
    }
    pa_sync_compute();
    for (int t = tid; t < G * QTTS_HD; t += PA_THREADS) {
        float s = 0.0f;
        for (int q = 0; q < PA_THREADS / 64; ++q) s = __fadd_rn(s, part[q * G * QTTS_HD + t]);
        if (NS > 1) {
            const int h = t / QTTS_HD, d = t % QTTS_HD;
            float * pp = a.part + ((((size_t) b * NKV + g) * NS + sp) * G + h) * PA_PART;
            pp[2 + d] = s;
            if (d == 0) { pp[0] = s_ml[h][0]; pp[1] = s_ml[h][1]; }
            continue;
        }
        a.out[(size_t) b * a.ldo + (size_t)(g * G) * QTTS_HD + t] = s;
        if (a.xt) *reinterpret_cast<__half *>(a.xt + tc_x_off(b, g * G * QTTS_HD + t, a.xt_np)) = __float2half_rn(s);
    }
}

__global__ void __launch_bounds__(PA_BLOCK, 2) k_attn_paged(PagedAttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int G = a.n_heads / a.n_kv_heads;
    if (G == 1) attn_paged_body<1>(a);
    else if (G == 2) attn_paged_body<2>(a);
    else attn_paged_body<4>(a);
}

// Merge of the page ranges of a split paged attention, one CTA per (sequence,
// kv head), thread d = dim: M = max of the ranges' maxima, then in range order
// w = exp(m - M), L += l * w (double), O += o * w; out = O * (float)(1 / L).
__global__ void __launch_bounds__(QTTS_HD) k_attn_combine(PagedAttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int NKV = a.n_kv_heads, G = a.n_heads / NKV, NS = a.nsplit;
    const int b = blockIdx.x / NKV, g = blockIdx.x % NKV, d = threadIdx.x;
    if (a.st[b].done) return;
    for (int h = 0; h < G; ++h) {
        const float * pp = a.part + (((size_t) b * NKV + g) * NS * G + h) * PA_PART;
        float M = -INFINITY;
        for (int s = 0; s < NS; ++s) M = fmaxf(M, pp[(size_t) s * G * PA_PART]);
        double L = 0.0;
        float O = 0.0f;
        for (int s = 0; s < NS; ++s) {
            const float * q = pp + (size_t) s * G * PA_PART;
            if (q[0] == -INFINITY) continue;   // an empty range
            const float w = qtts_expf(__fsub_rn(q[0], M));
            L += (double) q[1] * (double) w;
            O = fmaf(q[2 + d], w, O);
        }
        const float o = __fmul_rn(O, (float)(1.0 / L));
        a.out[(size_t) b * a.ldo + (size_t)(g * G + h) * QTTS_HD + d] = o;
        if (a.xt) *reinterpret_cast<__half *>(a.xt + tc_x_off(b, (g * G + h) * QTTS_HD + d, a.xt_np)) = __float2half_rn(o);
    }
}

// ---- code-predictor attention for B sequences ------------------------------
// Code-predictor attention with one warp per (sequence b, query head, row i)
// unit.  Steps (one row, keys from the cache) run cp_step_attn_body, the
// batch-1 engine's per-head order.  The 2-token prefill (F32 K/V of the call):
// at most 17 keys, so lane j scores key j over all 128 dims (q broadcast
// from shared memory), the softmax is a warp reduction (max, expf, double sum,
// e * (float)(1/sum), F16-rounded in cache mode), and lane l accumulates dims
// 4l..4l+3 of P x V.  Arithmetic as the fused unit (per-head q/k RMSNorm,
// NEOX RoPE, F16 q / K / V / p in cache mode, F32 K / V of this call in the
// 2-token prefill); the warp of the first query head of a kv group appends the
// group's new K/V row to the sequence's cache.
constexpr int CPW_WARPS = 16;

__global__ void __launch_bounds__(CPW_WARPS * 32) k_cp_attn_warp(FusedAttn a, size_t cache_stride, const DevState * st,
                                                                 int B) {
    __shared__ float sq[CPW_WARPS][QTTS_HD];
    __shared__ float sk[CPW_WARPS][2][QTTS_HD];
    __shared__ float sv[CPW_WARPS][2][QTTS_HD];
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NH = a.n_heads, NKV = a.n_kv_heads, G = NH / NKV, M = a.M;
    const int unit = blockIdx.x * CPW_WARPS + warp;
    if (unit >= B * NH * M) return;
    const int b = unit / (NH * M), r = unit % (NH * M), i = r / NH, hq = r % NH, g = hq / G;
    if (st[b].done) return;
    const bool f32 = a.f32_mode != 0;
    if (!f32 && M == 1) {   // code-predictor step: the batch-1 engine's per-head order
        FusedAttn s = a;
        s.qkv = a.qkv + (size_t) b * a.ldq;
        s.kc = a.kc + (size_t) b * cache_stride;
        s.vc = a.vc + (size_t) b * cache_stride;
        s.out = a.out + (size_t) b * a.ldo;
        cp_step_attn_body(s, hq, a.pos_static, b);
        return;
    }
    const int n_past = a.pos_static, pos = n_past + i;
    const int n = f32 ? i + 1 : n_past + 1, nc = f32 ? 0 : n_past;
    const int QD = NH * QTTS_HD, KD = NKV * QTTS_HD;
    const size_t pstride = (size_t) NKV * QTTS_HD;
    const float * qkv = a.qkv + (size_t) b * M * a.ldq;
    __half * kc = a.kc + (size_t) b * cache_stride;
    __half * vc = a.vc + (size_t) b * cache_stride;

    // q head of row i
    {
        const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
        const float4 q4 = *reinterpret_cast<const float4 *>(qkv + (size_t) i * a.ldq + (size_t) hq * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.q_norm, rp, lane, gv, cs);
        float x[4] = {q4.x, q4.y, q4.z, q4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) sq[warp][lane * 4 + k] = f32 ? x[k] : round_f16(x[k]);
    }
    // k/v rows computed here: rows 0..i of this call (prefill) or the current row
    const int nrow = f32 ? i + 1 : 1;
    for (int rr = 0; rr < nrow; ++rr) {
        const int j = f32 ? rr : i;
        const float2 * rp = a.rope + (size_t)(n_past + j) * (QTTS_HD / 2);
        const float4 k4 = *reinterpret_cast<const float4 *>(qkv + (size_t) j * a.ldq + QD + g * QTTS_HD + lane * 4);
        const float4 v4 = *reinterpret_cast<const float4 *>(qkv + (size_t) j * a.ldq + QD + KD + g * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.k_norm, rp, lane, gv, cs);
        float x[4] = {k4.x, k4.y, k4.z, k4.w};
        const float v[4] = {v4.x, v4.y, v4.z, v4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half kh = __float2half_rn(x[k]), vh = __float2half_rn(v[k]);
            sk[warp][rr][lane * 4 + k] = f32 ? x[k] : __half2float(kh);
            sv[warp][rr][lane * 4 + k] = f32 ? v[k] : __half2float(vh);
            if (j == i && hq % G == 0) {
                kc[(size_t)(n_past + j) * pstride + g * QTTS_HD + lane * 4 + k] = kh;
                vc[(size_t)(n_past + j) * pstride + g * QTTS_HD + lane * 4 + k] = vh;
            }
        }
    }
    __syncwarp();
    // scores: lane j <-> key j
    float sj = -INFINITY;
    if (lane < n) {
        float acc = 0.0f;
        if (lane < nc) {
            const uint4 * kp = reinterpret_cast<const uint4 *>(kc + (size_t) lane * pstride + g * QTTS_HD);
#pragma unroll 4
            for (int c = 0; c < QTTS_HD / 8; ++c) {
                const uint4 u = kp[c];
                const __half2 * hp = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(hp[k]);
                    acc = fmaf(f.x, sq[warp][c * 8 + 2 * k], acc);
                    acc = fmaf(f.y, sq[warp][c * 8 + 2 * k + 1], acc);
                }
            }
        } else {
            const float * kr = sk[warp][f32 ? lane : 0];
            for (int d = 0; d < QTTS_HD; ++d) acc = fmaf(kr[d], sq[warp][d], acc);
        }
        sj = __fmul_rn(acc, a.scale);
    }
    const float mx = warp_max(sj);
    const float e = lane < n ? qtts_expf(__fsub_rn(sj, mx)) : 0.0f;
    const double sum = warp_sum_d(lane < n ? (double) e : 0.0);
    const float inv = (float)(1.0 / sum);
    float p = __fmul_rn(e, inv);
    if (!f32) p = round_f16(p);
    // P x V: lane owns dims 4 lane .. 4 lane + 3
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = 0; j < n; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        float v[4];
        if (j < nc) {
            const uint2 u = *reinterpret_cast<const uint2 *>(vc + (size_t) j * pstride + g * QTTS_HD + lane * 4);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
            v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
        } else {
            const float * vr = sv[warp][f32 ? j : 0];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = vr[lane * 4 + k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = fmaf(pj, v[k], o[k]);
    }
    const int row = b * M + i;
    *reinterpret_cast<float4 *>(a.out + (size_t) row * a.ldo + (size_t) hq * QTTS_HD + lane * 4) =
        make_float4(o[0], o[1], o[2], o[3]);
    if (a.xt) {
        __align__(8) __half h4[4] = {__float2half_rn(o[0]), __float2half_rn(o[1]), __float2half_rn(o[2]),
                                      __float2half_rn(o[3])};
        *reinterpret_cast<uint2 *>(a.xt + tc_x_off(row, hq * QTTS_HD + lane * 4, a.xt_np)) =
            *reinterpret_cast<const uint2 *>(h4);
    }
}

// ---- per-sequence samplers, inputs and frame end ---------------------------
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_batch(const float * logits, int ldl, int V, int cb,
                                                                 DevState * st, const SampleParams * sp,
                                                                 int * out_codes, int out_cap) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    DevState * s = st + b;
    if (s->done) return;
    SampleParams P = *sp;
    P.seed += 0x9E3779B97F4A7C15ull * (unsigned long long) b;   // independent Philox stream per sequence
    P.record_logits = 0;
    const int frame = s->frame;
    const int tok = sample_body<SAMPLE_PER_T>(logits + (size_t) b * ldl, V, cb, s, P, frame);
    if (threadIdx.x == 0) sample_commit(tok, cb, s, P, out_codes + (size_t) b * out_cap * P.n_cb, out_cap, frame);
}

struct BatchInputArgs {
    int mode, g, H, n_cb;
    const __half * codec_embd;
    const __half * const * cp_embd;
    const float * hidden;        // [B][H]
    const float * trailing;      // [B][trail_cap][H]
    int trail_cap;
    const float * pad;           // [H]
    float * out;
    const DevState * st;
};

__global__ void k_inputs_batch(BatchInputArgs a) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x;
    const DevState & S = a.st[b];
    if (S.done) return;
    const int H = a.H;
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        if (a.mode == IN_CP_PREFILL) {
            a.out[(size_t)(2 * b) * H + h] = a.hidden[(size_t) b * H + h];
            a.out[(size_t)(2 * b + 1) * H + h] = __half2float(a.codec_embd[(size_t) S.codes[0] * H + h]);
        } else if (a.mode == IN_CP_STEP) {
            a.out[(size_t) b * H + h] = __half2float(a.cp_embd[a.g - 1][(size_t) S.codes[a.g] * H + h]);
        } else {
            float s = __half2float(a.codec_embd[(size_t) S.codes[0] * H + h]);
            for (int cb = 1; cb < a.n_cb; ++cb)
                s = __fadd_rn(s, __half2float(a.cp_embd[cb - 1][(size_t) S.codes[cb] * H + h]));
            const float * tr = S.frame < S.n_trailing ? a.trailing + ((size_t) b * a.trail_cap + S.frame) * H : a.pad;
            a.out[(size_t) b * H + h] = __fadd_rn(s, tr[h]);
        }
    }
}

// End of a batched frame: every live sequence advances one position.  A
// sequence that has emitted its max_len frames stops here (done = 1), so its
// position never passes the prompt + max_len rows its pages and RoPE rows were
// sized for, and its code rows stay inside the max_frames buffer.
__global__ void k_frame_end_batch(DevState * st, int B, const int * max_len) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B && !st[b].done) {
        st[b].pos += 1;
        st[b].frame += 1;
        st[b].n_out += 1;
        if (st[b].n_out >= max_len[b]) st[b].done = 1;
    }
}

// Copy a prefill's KV rows [0, n) from the contiguous cache [layer][ctx][NKV][128]
// into the sequence's pages.
__global__ void k_kv_to_pages(const __half * kc, const __half * vc, int ctx, int n, int n_layers, int nkv,
                              const int * pt, __half * pool) {
    const int j = blockIdx.x, layer = blockIdx.y;
    if (j >= n) return;
    const size_t src = ((size_t) layer * ctx + j) * nkv * QTTS_HD;
    for (int t = threadIdx.x; t < nkv * QTTS_HD; t += blockDim.x) {
        const int h = t / QTTS_HD, d = t % QTTS_HD;
        pool[bp_off(pt[j / BP_PAGE], layer, 0, h, j % BP_PAGE, n_layers, nkv) + d] = kc[src + t];
        pool[bp_off(pt[j / BP_PAGE], layer, 1, h, j % BP_PAGE, n_layers, nkv) + d] = vc[src + t];
    }
}

}  // namespace qtts
