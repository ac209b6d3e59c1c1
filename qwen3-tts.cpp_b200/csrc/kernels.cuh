// kernels.cuh — sm_100a kernels of the per-frame codec-token loop.
//
// Each kernel restates one group of ggml ops of src/tts_transformer.cpp with
// the same dtype semantics (see the oracle for the CPU statement):
//   k_gemv          ggml_rms_norm+ggml_mul prologue, ggml_mul_mat (F16 or Q8_0
//                   weights), ggml_add residual / ggml_silu+ggml_mul epilogues
//                   (:1656-1661, :1732-1750, :1755-1760)
//   k_qk_rope_store per-head rms_norm q/k, NEOX rope, F16 KV append
//                   (:1667-1699)
//   k_attention     KQ, scale, causal mask, softmax, KQV with GQA (:1703-1730)
//   k_sample        codebook-0 and code-predictor sampling (:2750-2788,
//                   :3108-3191)
//   k_frame_inputs  embedding gathers for the code predictor and the next
//                   talker step (:2091, :2791, :3264-3295)
#pragma once
#include "common.cuh"

namespace qtts {

enum Epi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2 };
enum Act : int { ACT_F16 = 0, ACT_F32 = 1 };

struct GemvArgs {
    DMat A, B;              // B.w != nullptr: dual matrix (gate, up) with SwiGLU epilogue
    const float * x;        // input rows [nv][ldx]
    int ldx, nv;
    const float * norm_g;   // RMSNorm gain over the input (nullptr: no norm)
    float eps;
    int act;                // F16 weights: ACT_F16 rounds the activation, ACT_F32 keeps it
    float * y;              // output rows [nv][ldy]
    int ldy;
    const float * resid;    // EPI_RESID: y = acc + resid (resid may alias y)
    int ldr;
    int epi;
    float * xn_out;         // the CTA owning row 0 writes the normalised input rows here (F32)
    int ldxn;
    const int * done;       // frame-loop stop flag (skip when *done)
    int * block_dots;       // Q8_0 test hook: per-block int32 dots [nv][rows][cols/32] (nullptr: off)
};

constexpr size_t QTTS_GEMV_SMEM_MAX = 200 * 1024;   // dynamic shared memory of a stand-alone k_gemv

// Rows [r0, r1) of a GEMV belong to CTA `cta` of `ncta` (rpc = ceil(rows / ncta)).
__host__ __device__ inline int gemv_rpc(int rows, int ncta) { return (rows + ncta - 1) / ncta; }

// A CTA's weight slice as staged in shared memory:
//   A rows | B rows | A scales | B scales | RMSNorm gain (F32, cols)
struct SliceLayout {
    size_t bA, bS, gain_off, total;
};
__host__ __device__ inline SliceLayout slice_layout(const DMat & A, bool dual, bool has_gain, int nrow) {
    SliceLayout L;
    const bool q8 = A.type == W_Q8_0;
    L.bA = (size_t) nrow * A.cols * (q8 ? 1 : 2);
    L.bS = q8 ? (size_t) nrow * (A.cols / 32) * 2 : 0;
    const int nm = dual ? 2 : 1;
    L.gain_off = nm * (L.bA + L.bS);
    L.total = L.gain_off + (has_gain ? (size_t) A.cols * 4 : 0);
    return L;
}

// Shared-memory work area of a GEMV: x [NV][cols] F32, residuals [NV][rpc],
// Q8_0: activation quants [NV][cols] and scales [NV][cols/32].
__host__ __device__ inline size_t gemv_work_bytes(int type, int cols, int nv, int rpc) {
    size_t b = (size_t) nv * cols * 4 + (size_t) nv * ((rpc + 3) & ~3) * 4;
    if (type == W_Q8_0) b += (size_t) nv * cols + (size_t) nv * (cols / 32) * 4;
    return b;
}

// One thread: copy the CTA's slice of (A, B) and the norm gain into `buf`,
// completing on mbarrier m (expect_tx covers every byte, so the phase completes
// even when this CTA owns no rows).
// extra_bytes: further bulk copies the caller issues on the same mbarrier phase.
__device__ __forceinline__ void issue_gemv_slice(const DMat & A, const DMat & B, const float * gain, uint8_t * buf,
                                                 uint64_t * m, int cta, int ncta, unsigned extra_bytes = 0) {
    const int rpc = gemv_rpc(A.rows, ncta);
    const int r0 = cta * rpc, r1 = min(A.rows, r0 + rpc);
    const int nrow = r1 > r0 ? r1 - r0 : 0;
    const bool dual = B.w != nullptr;
    const SliceLayout L = slice_layout(A, dual, gain != nullptr, nrow);
    mbar_expect_tx(m, (nrow ? (unsigned) L.total : 0u) + extra_bytes);
    if (!nrow) return;
    const size_t es = A.type == W_Q8_0 ? 1 : 2;
    for (int k = 0; k < (dual ? 2 : 1); ++k) {
        const DMat & M = k ? B : A;   // (no array of pointers: it would live in local memory)
        const char * src = static_cast<const char *>(M.w) + (size_t) r0 * A.cols * es;
        for (size_t o = 0; o < L.bA; o += 32768) {
            const unsigned n = (unsigned)(L.bA - o < 32768 ? L.bA - o : 32768);
            bulk_g2s(buf + k * L.bA + o, src + o, n, m);
        }
        if (L.bS)
            bulk_g2s(buf + (dual ? 2 : 1) * L.bA + k * L.bS, M.d + (size_t) r0 * (A.cols / 32), (unsigned) L.bS, m);
    }
    if (gain) bulk_g2s(buf + L.gain_off, gain, (unsigned)(A.cols * 4), m);
}

// Epilogue of output row rl (local) of activation row v: SwiGLU, residual add or store.
__device__ __forceinline__ float gemv_epi(const GemvArgs & a, int v, float accA, float accB, const float * rs, int rl,
                                          int rstride) {
    if (a.epi == EPI_SWIGLU) return __fmul_rn(silu(accA), accB);
    if (a.epi == EPI_RESID) return __fadd_rn(accA, rs[v * rstride + rl]);
    return accA;
}

// Plain output store of a stand-alone or CUDA-graph GEMV: y[v][r] (the pointer
// and stride are read from the kernel arguments at the store).
struct GemvStorePlain {
    const GemvArgs & g;
    __device__ __forceinline__ void operator()(int r, int, int v, float out) const { g.y[(size_t) v * g.ldy + r] = out; }
};

// Activation rows live in shared memory in a two-plane layout per row: column
// c = 8*k + w sits at (w / 4) * cols/2 + 4*k + w % 4, so the lane that owns the
// 8-column chunk k reads two conflict-free float4 (plane 0 and plane 1).
__device__ __forceinline__ int xpos(int c, int cols) { return ((c & 7) >> 2) * (cols >> 1) + ((c >> 3) << 2) + (c & 3); }

// Shared-memory work area of a GEMV (gemv_work_bytes): activation rows xs in the
// two-plane layout, residual rows rs, then (Q8_0) activation quants and scales.
struct GemvWork {
    float * xs, * rs;
    int8_t * qa;
    float * da;
};
template <int NV>
__device__ __forceinline__ GemvWork gemv_work(uint8_t * work, int cols, int rpc, bool q8) {
    GemvWork w;
    w.xs = reinterpret_cast<float *>(work);
    w.rs = w.xs + NV * cols;
    w.qa = reinterpret_cast<int8_t *>(w.rs + NV * ((rpc + 3) & ~3));
    w.da = reinterpret_cast<float *>(w.qa + (q8 ? NV * cols : 0));
    return w;
}

// Activation loaders, run by gemv_compute ahead of its first block barrier (in
// the same function body: a separate load phase before the call measured ~3 %
// slower per frame on B200).  GemvLoadNone: the caller filled the work area.
constexpr int GEMV_RPT = 6;   // activation values per thread held in registers (one row, cols <= 6 x threads)

// Column of planar position p of the two-plane layout (see xpos).
__device__ __forceinline__ int planar_col(int p, int cols) {
    const int half = cols >> 1;
    const int q = p >= half ? p - half : p;
    return ((q >> 2) << 3) + (p >= half ? 4 : 0) + (q & 3);
}

struct GemvLoadNone {
    static constexpr bool active = false, regs_ok = false;
    __device__ __forceinline__ void operator()(const GemvWork &, int, int, int) const {}
    __device__ __forceinline__ void regs(float (&)[GEMV_RPT], const GemvWork &, int, int, int) const {}
};
// Activation rows from global memory into the two-plane layout (float4 i =
// columns 4i..4i+3 -> plane i & 1, chunk i >> 1) and this CTA's residual rows.
template <int NV>
struct GemvLoadGlobal {
    static constexpr bool active = true, regs_ok = NV == 1;
    const GemvArgs & a;
    // One row, cols <= GEMV_RPT x threads: thread t loads the values of the
    // planar positions p = t + k * threads that it reduces and normalises
    // (column planar_col(p)) into xr[k], so the RMSNorm sum needs no block
    // barrier first; residual rows go to the work area as above.
    __device__ __forceinline__ void regs(float (&xr)[GEMV_RPT], const GemvWork & w, int r0, int nrow,
                                         int rstride) const {
        const int cols = a.A.cols, tid = threadIdx.x, nt = blockDim.x;
#pragma unroll
        for (int k = 0; k < GEMV_RPT; ++k) {
            const int p = tid + k * nt;
            xr[k] = p < cols ? a.x[planar_col(p, cols)] : 0.0f;
        }
        if (a.epi == EPI_RESID)
            for (int r = tid; r < nrow; r += nt) w.rs[r] = a.resid[(size_t) r0 + r];
    }
    __device__ __forceinline__ void operator()(const GemvWork & w, int r0, int nrow, int rstride) const {
        const int cols = a.A.cols, tid = threadIdx.x, nt = blockDim.x;
        const int c4 = cols >> 2, h8 = cols >> 3;
        const int nv = a.nv;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (v >= nv) break;
            const float4 * src = reinterpret_cast<const float4 *>(a.x + (size_t) v * a.ldx);
            float4 * dst = reinterpret_cast<float4 *>(w.xs + v * cols);
            for (int i = tid; i < c4; i += nt) dst[(i & 1) * h8 + (i >> 1)] = src[i];
        }
        if (a.epi == EPI_RESID)
            for (int v = 0; v < nv; ++v)
                for (int r = tid; r < nrow; r += nt) w.rs[v * rstride + r] = a.resid[(size_t) v * a.ldr + r0 + r];
    }
};

// GEMV over this CTA's rows [r0, r1) with the weight slice in shared memory
// (`wsm`, layout slice_layout; complete once mbarrier `m` reaches `parity`, or
// immediately when m == nullptr) and the activation rows in the work area
// (two-plane layout), written by `load` or, with GemvLoadNone, by the caller,
// who synchronises the block after filling it.  Latency-oriented: one warp per row, two block barriers.  The RMSNorm sum of
// squares is a double sum over the CTA (thread-strided partials, warp
// butterfly, then the 16 warp partials in order); normalisation and F16
// rounding happen once, in place.  Reduction order of a row: lane l
// accumulates the 8-column chunks l, l+32, ... in order (8 sequential FMAs per
// F16 chunk; one 32-block term per lane pair for Q8_0), then a butterfly over
// the 32 lanes.  Outputs go through `store(r, rl, v, value)`; xn_smem (optional)
// receives every CTA's unrounded normalised row 0 in column order.
template <int NV, class Store, class Load = GemvLoadNone>
__device__ __forceinline__ bool gemv_compute(const GemvArgs & a, const int cta, const int ncta, const uint8_t * wsm,
                                             uint8_t * work, uint64_t * m, unsigned parity, const Store & store,
                                             float * xn_smem = nullptr, unsigned long long * ready_stamp = nullptr,
                                             const Load & load = Load{}) {
    __shared__ double s_red[QTTS_WARPS][NV];
    const int cols = a.A.cols, rows = a.A.rows;
    const int rpc = gemv_rpc(rows, ncta);
    const int r0 = cta * rpc, r1 = min(rows, r0 + rpc);
    const int nrow = r1 > r0 ? r1 - r0 : 0;
    const bool q8 = a.A.type == W_Q8_0, dual = a.B.w != nullptr;
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    const int nv = a.nv;
    const int rstride = (rpc + 3) & ~3;
    const GemvWork W = gemv_work<NV>(work, cols, rpc, q8);
    float * xs = W.xs;
    const float * rs = W.rs;
    int8_t * qa = W.qa;
    float * da = W.da;
    const int h8 = cols >> 3;
    // inreg: this thread's activation values (planar positions tid + k nt) in xr.
    // With Q8_0 weights only without an RMSNorm: with one, the frame measured
    // slower (the quantiser reads the row back from shared memory in 32-column
    // blocks after the normalisation barrier).
    const bool inreg = Load::regs_ok && cols <= GEMV_RPT * nt && (!q8 || a.norm_g == nullptr);
    float xr[GEMV_RPT];
    if (inreg) {
        load.regs(xr, W, r0, nrow, rstride);
    } else if (Load::active) {
        load(W, r0, nrow, rstride);
        __syncthreads();
    }

    // 1. RMSNorm partial sums (positions p = tid, tid + nt, ... in order); thread 0
    // waits for the weight slice
    const bool has_norm = a.norm_g != nullptr;
    if (has_norm) {
        if (inreg) {
            double ss = 0.0;
#pragma unroll
            for (int k = 0; k < GEMV_RPT; ++k)
                if (tid + k * nt < cols) ss += (double) __fmul_rn(xr[k], xr[k]);
            ss = warp_sum_d(ss);
            if (lane == 0) s_red[warp][0] = ss;
        } else {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (v >= nv) break;
                double ss = 0.0;
                for (int p = tid; p < cols; p += nt) { const float t = xs[v * cols + p]; ss += (double) __fmul_rn(t, t); }
                ss = warp_sum_d(ss);
                if (lane == 0) s_red[warp][v] = ss;
            }
        }
    } else if (inreg) {   // no RMSNorm: the row goes to shared memory now, published by the barrier below
        const bool r16 = !q8 && a.act == ACT_F16;
#pragma unroll
        for (int k = 0; k < GEMV_RPT; ++k)
            if (tid + k * nt < cols) xs[tid + k * nt] = r16 ? round_f16(xr[k]) : xr[k];
    }
    bool ok = true;
    if (m && tid == 0) {
        ok = mbar_wait(m, parity);
        if (ok && ready_stamp) {   // diagnostics: latest weight arrival over the CTAs
            unsigned long long t;
            asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
            atomicMax(ready_stamp, t);
        }
    }
    if (__syncthreads_or(!ok)) return false;
    const SliceLayout L = slice_layout(a.A, dual, has_norm, nrow);
    const float * gain = has_norm ? reinterpret_cast<const float *>(wsm + L.gain_off) : nullptr;

    // 2. normalise (x * scale) * gain, round to F16 for F16 weights with an F16 activation
    const bool round16 = !q8 && a.act == ACT_F16;
    if (inreg ? (has_norm || a.xn_out != nullptr) : (has_norm || round16 || a.xn_out || xn_smem)) {
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (v >= nv) break;
            float scale = 1.0f;
            if (has_norm) {
                double ss = 0.0;
                for (int w = 0; w < nw; ++w) ss += s_red[w][v];
                scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(ss / (double) cols), a.eps)));
            }
            auto put = [&](const int p, float t) {
                const int c = planar_col(p, cols);
                if (has_norm) t = __fmul_rn(__fmul_rn(t, scale), gain[c]);
                if (a.xn_out && r0 == 0) a.xn_out[(size_t) v * a.ldxn + c] = t;   // hidden_states (post-norm, unrounded)
                if (xn_smem && v == 0) xn_smem[c] = t;
                xs[v * cols + p] = round16 ? round_f16(t) : t;
            };
            if (inreg) {
#pragma unroll
                for (int k = 0; k < GEMV_RPT; ++k)
                    if (tid + k * nt < cols) put(tid + k * nt, xr[k]);
            } else {
                for (int p = tid; p < cols; p += nt) put(p, xs[v * cols + p]);
            }
        }
        __syncthreads();
    }

    if (!q8) {
        const uint8_t * wa = wsm;
        const uint8_t * wb = wsm + L.bA;
        for (int rl = warp; rl < nrow; rl += nw) {
            float acc[NV], accb[NV];
#pragma unroll
            for (int v = 0; v < NV; ++v) acc[v] = accb[v] = 0.0f;
            const uint4 * ra = reinterpret_cast<const uint4 *>(wa + (size_t) rl * cols * 2);
            const uint4 * rb = reinterpret_cast<const uint4 *>(wb + (size_t) rl * cols * 2);
            for (int c = lane; c < h8; c += 32) {
                const uint4 w = ra[c];
                const uint4 w2 = dual ? rb[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    if (v >= nv) continue;
                    const float4 x0 = reinterpret_cast<const float4 *>(xs + v * cols)[c];
                    const float4 x1 = reinterpret_cast<const float4 *>(xs + v * cols)[h8 + c];
                    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    acc[v] = dot8(w, xv, acc[v]);
                    if (dual) accb[v] = dot8(w2, xv, accb[v]);
                }
            }
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (v >= nv) continue;
                const float s1 = warp_sum(acc[v]);
                const float s2 = dual ? warp_sum(accb[v]) : 0.0f;
                if (lane == 0) store(r0 + rl, rl, v, gemv_epi(a, v, s1, s2, rs, rl, rstride));
            }
        }
        return true;
    }

    // Q8_0: quantise the (normalised) activation once per 32-block, as
    // quantize_row_q8_0_ref: d = amax / 127, id = 1 / d, q = roundf(x * id).
    // Eight lanes per block (four consecutive columns each, one 16-byte load
    // from the two-plane layout), four blocks per warp pass.
    const int nb = cols / 32;
    {
        const int sub = lane & 7, grp = lane >> 3;
        for (int blk0 = warp * 4; blk0 < nv * nb; blk0 += nw * 4) {
            const int blk = blk0 + grp;
            const bool okb = blk < nv * nb;
            const int v = okb ? blk / nb : 0, b = okb ? blk % nb : 0;
            const int c = b * 32 + sub * 4;
            const float4 x4 = okb ? *reinterpret_cast<const float4 *>(xs + v * cols + xpos(c, cols))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float am = fmaxf(fmaxf(fabsf(x4.x), fabsf(x4.y)), fmaxf(fabsf(x4.z), fabsf(x4.w)));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
            const float d = __fdiv_rn(am, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            if (okb) {
                char4 q;
                q.x = (signed char) roundf(__fmul_rn(x4.x, id));
                q.y = (signed char) roundf(__fmul_rn(x4.y, id));
                q.z = (signed char) roundf(__fmul_rn(x4.z, id));
                q.w = (signed char) roundf(__fmul_rn(x4.w, id));
                *reinterpret_cast<char4 *>(qa + v * cols + c) = q;
                if (sub == 0) da[v * nb + b] = __half2float(__float2half_rn(d));
            }
        }
    }
    __syncthreads();
    const uint8_t * qwa = wsm;
    const uint8_t * qwb = wsm + L.bA;
    const __half * swa = reinterpret_cast<const __half *>(wsm + (dual ? 2 : 1) * L.bA);
    const __half * swb = reinterpret_cast<const __half *>(wsm + (dual ? 2 : 1) * L.bA + L.bS);
    const int nchunk = cols / 16;
    for (int rl = warp; rl < nrow; rl += nw) {
        float acc[NV], accb[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[v] = accb[v] = 0.0f;
        const int4 * ra = reinterpret_cast<const int4 *>(qwa + (size_t) rl * cols);
        const int4 * rb = reinterpret_cast<const int4 *>(qwb + (size_t) rl * cols);
        for (int c0 = 0; c0 < nchunk; c0 += 32) {      // uniform trip count: full-mask shuffles inside
            const int c = c0 + lane;
            const bool ok = c < nchunk;                   // uniform within a lane pair (nchunk is even)
            const int4 w = ok ? ra[c] : make_int4(0, 0, 0, 0);
            const int4 w2 = (ok && dual) ? rb[c] : make_int4(0, 0, 0, 0);
            const float dwa = ok ? __half2float(swa[rl * nb + (c >> 1)]) : 0.0f;
            const float dwb = (ok && dual) ? __half2float(swb[rl * nb + (c >> 1)]) : 0.0f;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                if (v >= nv) continue;
                const int4 xq = ok ? reinterpret_cast<const int4 *>(qa + v * cols)[c] : make_int4(0, 0, 0, 0);
                const float dx = ok ? da[v * nb + (c >> 1)] : 0.0f;
                int ia = __dp4a(w.x, xq.x, 0);
                ia = __dp4a(w.y, xq.y, ia);
                ia = __dp4a(w.z, xq.z, ia);
                ia = __dp4a(w.w, xq.w, ia);
                ia += __shfl_xor_sync(0xffffffffu, ia, 1);   // the 32-block int32 dot
                if (a.block_dots && ok && !(lane & 1))
                    a.block_dots[((size_t) v * rows + r0 + rl) * nb + (c >> 1)] = ia;
                if (ok && !(lane & 1)) acc[v] = __fadd_rn(acc[v], __fmul_rn((float) ia, __fmul_rn(dwa, dx)));
                if (dual) {
                    int ib = __dp4a(w2.x, xq.x, 0);
                    ib = __dp4a(w2.y, xq.y, ib);
                    ib = __dp4a(w2.z, xq.z, ib);
                    ib = __dp4a(w2.w, xq.w, ib);
                    ib += __shfl_xor_sync(0xffffffffu, ib, 1);
                    if (ok && !(lane & 1)) accb[v] = __fadd_rn(accb[v], __fmul_rn((float) ib, __fmul_rn(dwb, dx)));
                }
            }
        }
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (v >= nv) continue;
            const float s1 = warp_sum(acc[v]);
            const float s2 = dual ? warp_sum(accb[v]) : 0.0f;
            if (lane == 0) store(r0 + rl, rl, v, gemv_epi(a, v, s1, s2, rs, rl, rstride));
        }
    }
    return true;
}

// GEMV with activations and residuals read from global memory (GemvLoadGlobal)
// and outputs stored to a.y.
template <int NV>
__device__ __forceinline__ bool gemv_slice(const GemvArgs & a, const int cta, const int ncta, const uint8_t * wsm,
                                           uint8_t * work, uint64_t * m, unsigned parity) {
    return gemv_compute<NV>(a, cta, ncta, wsm, work, m, parity, GemvStorePlain{a}, nullptr, nullptr,
                            GemvLoadGlobal<NV>{a});
}

// Stand-alone GEMV launch (CUDA-graph path, prefill, kernel tests): thread 0
// stages this CTA's weight slice into shared memory with TMA bulk copies while
// all threads load the activations.  Launched with programmatic dependent
// launch, the copy starts while the previous kernel still runs.  Registers
// capped at 48: two 512-thread CTAs per SM then leave a quarter of the register
// file for the next kernel's CTAs (at 49-64 registers two CTAs take all of it,
// measured 4 % slower per frame).
template <int NV>
__global__ void __maxnreg__(48) k_gemv(GemvArgs a, size_t slice_bytes) {
    pdl_trigger();
    const int rpc = gemv_rpc(a.A.rows, gridDim.x);
    if ((int) blockIdx.x * rpc >= a.A.rows) return;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t mbar;
    if (threadIdx.x == 0) {   // the weight slice is read-only: its copy may start before the predecessor ends
        mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue_gemv_slice(a.A, a.B, a.norm_g, smem_raw, &mbar, blockIdx.x, gridDim.x);
    }
    __syncthreads();
    pdl_wait();               // activations, the stop flag and the outputs follow the predecessor
    if (a.done && *a.done) {
        if (threadIdx.x == 0) mbar_wait(&mbar, 0u);   // no bulk copy in flight at exit
        return;
    }
    if (!gemv_slice<NV>(a, blockIdx.x, gridDim.x, smem_raw, smem_raw + slice_bytes, &mbar, 0u)) {
        // the copy did not complete within the wait limit: wait once more (bounded) so
        // no bulk copy is in flight when the block exits, and leave the output unwritten
        if (threadIdx.x == 0) mbar_wait(&mbar, 0u);
    }
}

// ---------------------------------------------------------------------------
// q/k RMSNorm + NEOX RoPE + F16 KV append.  One CTA per token row, one warp per
// head (q heads first, then kv heads).  q is updated in place (F32); k is
// written to the F16 cache and, for F32 attention (code-predictor prefill), back
// in place as F32.  v is appended to the F16 cache as is.
struct QkArgs {
    float * qkv;             // [M][ldq]: q (NH*D) | k (NKV*D) | v (NKV*D)
    int ldq;
    int n_heads, n_kv_heads;
    const float * q_norm, * k_norm;
    float eps;
    const float2 * rope;     // [pos][D/2] (cos, sin)
    __half * kc, * vc;       // cache base of this layer: [n_ctx][NKV][D]
    const int * pos_ptr;     // n_past (device) or nullptr
    int pos_static;
    int keep_f32_k;          // write normalised+roped k back in place
    const int * done;
};

// Per-lane parameters of a head's RMSNorm + NEOX RoPE: lane owns dims
// 4*lane .. 4*lane+3; the rotation pairs dim d with d +- 64.
__device__ __forceinline__ void head_params(const float * g, const float2 * rp, int lane, float gv[4], float2 cs[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int d = lane * 4 + k;
        gv[k] = g ? g[d] : 1.0f;
        cs[k] = rp[lane < 16 ? d : d - 64];
    }
}

__device__ __forceinline__ void head_norm_rope_v(float x[4], const float gv[4], const float2 cs[4], float eps, int lane) {
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) ss += (double) __fmul_rn(x[k], x[k]);
    ss = warp_sum_d(ss);
    const float mean = (float)(ss / (double) QTTS_HD);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(__fmul_rn(x[k], scale), gv[k]);
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __shfl_xor_sync(0xffffffffu, x[k], 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (lane < 16) x[k] = __fsub_rn(__fmul_rn(x[k], cs[k].x), __fmul_rn(o[k], cs[k].y));   // x0 = x[d], x1 = x[d + 64]
        else x[k] = __fadd_rn(__fmul_rn(o[k], cs[k].y), __fmul_rn(x[k], cs[k].x));              // x0 = x[d - 64], x1 = x[d]
    }
}

__device__ __forceinline__ void head_norm_rope(float x[4], const float * g, float eps, const float2 * rp, int lane) {
    float gv[4];
    float2 cs[4];
    head_params(g, rp, lane, gv, cs);
    head_norm_rope_v(x, gv, cs, eps, lane);
}

__global__ void k_qk_rope_store(QkArgs a) {
    if (a.done && *a.done) return;
    const int i = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int pos = (a.pos_ptr ? *a.pos_ptr : a.pos_static) + i;
    const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
    float * row = a.qkv + (size_t) i * a.ldq;
    const int QD = a.n_heads * QTTS_HD, KD = a.n_kv_heads * QTTS_HD;
    if (w < a.n_heads) {
        float * qh = row + w * QTTS_HD + lane * 4;
        float x[4] = {qh[0], qh[1], qh[2], qh[3]};
        head_norm_rope(x, a.q_norm, a.eps, rp, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) qh[k] = x[k];
    } else if (w < a.n_heads + a.n_kv_heads) {
        const int kh = w - a.n_heads;
        float * kp = row + QD + kh * QTTS_HD + lane * 4;
        const float * vp = row + QD + KD + kh * QTTS_HD + lane * 4;
        float x[4] = {kp[0], kp[1], kp[2], kp[3]};
        head_norm_rope(x, a.k_norm, a.eps, rp, lane);
        __half * kdst = a.kc + ((size_t) pos * a.n_kv_heads + kh) * QTTS_HD + lane * 4;
        __half * vdst = a.vc + ((size_t) pos * a.n_kv_heads + kh) * QTTS_HD + lane * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            kdst[k] = __float2half_rn(x[k]);
            vdst[k] = __float2half_rn(vp[k]);
            if (a.keep_f32_k) kp[k] = x[k];
        }
    }
}

// ---------------------------------------------------------------------------
// Frame state in device memory: the frame graph reads positions and codes from
// here, so one captured graph serves every frame.
struct DevState {
    int pos;          // n_past for the next talker step
    int frame;        // frame index in the current generate call
    int done;         // codebook-0 EOS was sampled
    int n_out;        // frames emitted
    int n_trailing;   // trailing text rows (one per frame, then tts_pad)
    int codes[QTTS_MAX_CB];
    uint32_t presence[128];   // set of emitted codebook-0 tokens (vocab <= 4096)
};

// ---------------------------------------------------------------------------
// Attention for M query rows at positions n_past..n_past+M-1.  One CTA per
// (kv head, query row); the CTA serves the n_heads/n_kv_heads query heads of the
// group.  Two-pass softmax exactly as ggml_soft_max (global max, expf, double
// sum, y = e * (float)(1/sum)), then the KQV product.  Cache mode rounds q and
// the probabilities to F16 (the F16 K/V dots of the talker and code-predictor
// step graphs); F32 mode attends over this call's F32 K/V rows (code-predictor
// 2-token prefill, src/tts_transformer.cpp:2000-2011).
struct AttnArgs {
    const float * q;          // [M][ldq], head h at h*D (normalised + roped)
    int ldq;
    const __half * kc, * vc;  // cache base of this layer [n_ctx][NKV][D]
    const float * kf, * vf;   // F32 mode: K/V rows of this call [M][ldkv]
    int ldkv;
    int f32_mode;
    int n_heads, n_kv_heads;
    const int * pos_ptr;
    int pos_static;
    float scale;
    float * out;              // [M][ldo]
    int ldo;
    const int * done;
    float * dump;             // post-softmax rows [frame][n_heads][dump_stride] or nullptr
    int dump_stride;
    const DevState * st;      // frame index for the dump
};

constexpr int ATT_THREADS = 256;
constexpr int ATT_MAX_GROUP = 4;   // query heads per kv head

__host__ __device__ inline size_t attn_smem_bytes(int max_keys, int group) {
    return (size_t) group * max_keys * 4 + (size_t) group * QTTS_HD * 4 + 4 * (size_t) group * QTTS_HD * 4 + 512;
}

__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnArgs a) {
    if (a.done && *a.done) return;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int g = blockIdx.x, i = blockIdx.y;
    const int G = a.n_heads / a.n_kv_heads;
    const int n_past = a.pos_ptr ? *a.pos_ptr : a.pos_static;
    const int n = a.f32_mode ? (i + 1) : (n_past + i + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float * qs = reinterpret_cast<float *>(smem_raw);             // [G][D]
    float * part = qs + G * QTTS_HD;                               // [4][G][D]
    float * sc = part + 4 * G * QTTS_HD;                           // [G][n]
    __shared__ float redf[32];
    __shared__ double redd[32];

    for (int t = tid; t < G * QTTS_HD; t += blockDim.x) {
        const float v = a.q[(size_t) i * a.ldq + (size_t)(g * G) * QTTS_HD + t];
        qs[t] = a.f32_mode ? v : round_f16(v);
    }
    __syncthreads();

    // scores: 8-lane groups, each lane 16 dims
    // Every lane of a warp runs the same number of iterations (the 8-lane
    // groups' shuffles use the full mask); out-of-range keys compute on zeros.
    const int sub = lane & 7, slot = lane >> 3;
    for (int j0 = warp * 4; j0 < n; j0 += (ATT_THREADS / 32) * 4) {
        const int j = j0 + slot;
        const bool jv = j < n;
        float kv[16];
        if (!jv) {
#pragma unroll
            for (int d = 0; d < 16; ++d) kv[d] = 0.0f;
        } else if (a.f32_mode) {
            const float4 * kp = reinterpret_cast<const float4 *>(a.kf + (size_t) j * a.ldkv + g * QTTS_HD + sub * 16);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                float4 f = kp[q4];
                kv[4 * q4] = f.x; kv[4 * q4 + 1] = f.y; kv[4 * q4 + 2] = f.z; kv[4 * q4 + 3] = f.w;
            }
        } else {
            const uint4 * kp = reinterpret_cast<const uint4 *>(a.kc + ((size_t) j * a.n_kv_heads + g) * QTTS_HD + sub * 16);
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

    // softmax per head
    for (int h = 0; h < G; ++h) {
        float mx = -INFINITY;
        for (int j = tid; j < n; j += blockDim.x) mx = fmaxf(mx, sc[h * n + j]);
        mx = block_max(mx, redf);
        double sum = 0.0;
        for (int j = tid; j < n; j += blockDim.x) {
            const float e = qtts_expf(__fsub_rn(sc[h * n + j], mx));
            sc[h * n + j] = e;
            sum += (double) e;
        }
        sum = block_sum_d(sum, redd);
        const float inv = (float)(1.0 / sum);
        float * drow = a.dump ? a.dump + ((size_t) a.st->frame * a.n_heads + g * G + h) * a.dump_stride : nullptr;
        for (int j = tid; j < n; j += blockDim.x) {
            const float p = __fmul_rn(sc[h * n + j], inv);
            if (drow) drow[j] = p;
            sc[h * n + j] = a.f32_mode ? p : round_f16(p);
        }
        __syncthreads();
    }

    // KQV: 4 position groups x 64 threads, each thread 2 dims of all G heads
    const int pg = tid >> 6, d2 = tid & 63;
    float acc[ATT_MAX_GROUP][2];
#pragma unroll
    for (int h = 0; h < ATT_MAX_GROUP; ++h) acc[h][0] = acc[h][1] = 0.0f;
    for (int j = pg; j < n; j += 4) {
        float2 v;
        if (a.f32_mode) v = *reinterpret_cast<const float2 *>(a.vf + (size_t) j * a.ldkv + g * QTTS_HD + 2 * d2);
        else v = __half22float2(*reinterpret_cast<const __half2 *>(a.vc + ((size_t) j * a.n_kv_heads + g) * QTTS_HD + 2 * d2));
#pragma unroll
        for (int h = 0; h < ATT_MAX_GROUP; ++h) {
            if (h < G) {
                const float p = sc[h * n + j];
                acc[h][0] = fmaf(p, v.x, acc[h][0]);
                acc[h][1] = fmaf(p, v.y, acc[h][1]);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < ATT_MAX_GROUP; ++h)
        if (h < G) {
            part[(pg * G + h) * QTTS_HD + 2 * d2] = acc[h][0];
            part[(pg * G + h) * QTTS_HD + 2 * d2 + 1] = acc[h][1];
        }
    __syncthreads();
    for (int t = tid; t < G * QTTS_HD; t += blockDim.x) {
        const float s = __fadd_rn(__fadd_rn(part[t], part[G * QTTS_HD + t]),
                                  __fadd_rn(part[2 * G * QTTS_HD + t], part[3 * G * QTTS_HD + t]));
        a.out[(size_t) i * a.ldo + (size_t)(g * G) * QTTS_HD + t] = s;
    }
}

// ---------------------------------------------------------------------------
// Fused q/k RMSNorm + RoPE + KV append + attention for one (query head, query
// row) unit of a frame step (M = 1, F16 cache) or of the code-predictor 2-token
// prefill (M = 2, F32 K/V of this call; unit row i normalises k rows 0..i
// itself, so no unit reads another unit's output).  Same arithmetic as
// k_qk_rope_store + k_attention (src/tts_transformer.cpp:1660-1712 for the
// talker step, :2000-2011 / :2130-2160 for the code predictor), restructured
// for latency: one query head per CTA (the dependent chains of a unit are
// short), every global load of the unit (q/k/v rows, norm gains, RoPE row, the
// first FA_KPASS cached keys and values) issued before the first block
// barrier, four barriers in all.  The first query head of each kv group
// appends the group's new K/V row to the cache.
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
    int f32_mode;
    float scale;
    float * out;
    int ldo;
    float * dump;             // post-softmax rows [frame][n_heads][dump_stride] or nullptr
    int dump_stride;
    const int * done;         // stand-alone launch: skip when *done
    uint8_t * xt;             // optional: output also as F16 tiles for the O-projection GEMM (row xt_row0 + i)
    int xt_np, xt_row0;
};

constexpr int FA_THREADS = 512;
constexpr int FA_KIT = 2;                                 // key iterations per pass (16 warps x 4 keys each)
constexpr int FA_KPASS = FA_KIT * (FA_THREADS / 32) * 4;  // keys per pass: 128
constexpr int FA_NPG = FA_THREADS / 64;                   // PV position groups: 8
constexpr int FA_VIT = FA_KPASS / FA_NPG;                 // V rows per thread per pass: 16

// Shared memory of one unit: q head [128], new K/V rows [M][128] x 2, scores
// [n_max] and PV partial sums [FA_NPG][128] (F32).
__host__ __device__ inline size_t fused_attn_smem(int max_keys, int M) {
    const size_t nk = (size_t)((max_keys + 3) & ~3);
    return 4 * ((size_t) QTTS_HD + 2 * (size_t) M * QTTS_HD + nk + (size_t) FA_NPG * QTTS_HD) + 64;
}

// n_past: position of query row 0; frame: dump row.
__device__ __forceinline__ void fused_attn_body(const FusedAttn & a, const int unit, uint8_t * smem, const int n_past,
                                const int frame) {
    const int NKV = a.n_kv_heads, G = a.n_heads / a.n_kv_heads;
    const int hq = unit % a.n_heads, i = unit / a.n_heads, g = hq / G;
    const bool writer = hq % G == 0;                        // appends this group's K/V row
    const int pos = n_past + i;
    const int n = a.f32_mode ? (i + 1) : (n_past + 1);     // keys attended
    const int nc = a.f32_mode ? 0 : n_past;                 // keys read from the cache
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int QD = a.n_heads * QTTS_HD, KD = NKV * QTTS_HD;
    float * qs = reinterpret_cast<float *>(smem);           // [128]
    float * kn = qs + QTTS_HD;                              // [M][128] keys computed here
    float * vn = kn + a.M * QTTS_HD;                        // [M][128]
    float * sc = vn + a.M * QTTS_HD;                        // [n]
    float * part = sc + ((n + 3) & ~3);                     // [FA_NPG][128]
    const int jn0 = a.f32_mode ? 0 : n_past;                // first key held in kn/vn
    const __half * kbase = a.kc + (size_t) g * QTTS_HD;
    const __half * vbase = a.vc + (size_t) g * QTTS_HD;
    const size_t pstride = (size_t) NKV * QTTS_HD;          // cache elements per position

    // 1. loads: cached keys/values of the first pass go to registers
    const int sub = lane & 7, slot = lane >> 3;
    const int pg = tid >> 6, d2 = tid & 63;
    uint4 kr[FA_KIT][2];
#pragma unroll
    for (int it = 0; it < FA_KIT; ++it) {
        const int j = it * (FA_THREADS / 8) + warp * 4 + slot;
        if (j < nc) {
            const uint4 * kp = reinterpret_cast<const uint4 *>(kbase + (size_t) j * pstride + sub * 16);
            kr[it][0] = kp[0];
            kr[it][1] = kp[1];
        } else {
            kr[it][0] = kr[it][1] = make_uint4(0, 0, 0, 0);
        }
    }
    __half2 vr[FA_VIT];
    {
        const __half2 * vp = reinterpret_cast<const __half2 *>(vbase + (size_t) pg * pstride) + d2;
        const size_t vstep = (size_t) FA_NPG * pstride / 2;
#pragma unroll
        for (int t = 0; t < FA_VIT; ++t) vr[t] = pg + t * FA_NPG < nc ? vp[t * vstep] : __float2half2_rn(0.0f);
    }
    if (warp == 0) {
        const float2 * rp = a.rope + (size_t) pos * (QTTS_HD / 2);
        const float4 q4 = *reinterpret_cast<const float4 *>(a.qkv + (size_t) i * a.ldq + (size_t) hq * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.q_norm, rp, lane, gv, cs);            // all loads in flight together
        float x[4] = {q4.x, q4.y, q4.z, q4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) qs[lane * 4 + k] = a.f32_mode ? x[k] : round_f16(x[k]);
    } else if (warp <= (a.f32_mode ? i + 1 : 1)) {
        const int j = a.f32_mode ? warp - 1 : i;            // row of this call whose k/v this warp prepares
        const float2 * rp = a.rope + (size_t)(n_past + j) * (QTTS_HD / 2);
        const float4 k4 = *reinterpret_cast<const float4 *>(a.qkv + (size_t) j * a.ldq + QD + g * QTTS_HD + lane * 4);
        const float4 v4 = *reinterpret_cast<const float4 *>(a.qkv + (size_t) j * a.ldq + QD + KD + g * QTTS_HD + lane * 4);
        float gv[4];
        float2 cs[4];
        head_params(a.k_norm, rp, lane, gv, cs);
        float x[4] = {k4.x, k4.y, k4.z, k4.w};
        const float v[4] = {v4.x, v4.y, v4.z, v4.w};
        head_norm_rope_v(x, gv, cs, a.eps, lane);
        const int r = a.f32_mode ? j : 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half kh = __float2half_rn(x[k]), vh = __float2half_rn(v[k]);
            kn[r * QTTS_HD + lane * 4 + k] = a.f32_mode ? x[k] : __half2float(kh);
            vn[r * QTTS_HD + lane * 4 + k] = a.f32_mode ? v[k] : __half2float(vh);
            if (j == i && writer) {
                a.kc[(size_t) pos * pstride + g * QTTS_HD + lane * 4 + k] = kh;
                a.vc[(size_t) pos * pstride + g * QTTS_HD + lane * 4 + k] = vh;
            }
        }
    }
    __syncthreads();   // barrier 1: q head and new k/v rows are in shared memory

    // 2. scores; 8 lanes per key (16 dims each), 4 keys per warp per iteration
    float q16[16];
#pragma unroll
    for (int d = 0; d < 16; ++d) q16[d] = qs[sub * 16 + d];
    for (int p0 = 0; p0 < n; p0 += FA_KPASS) {
#pragma unroll
        for (int it = 0; it < FA_KIT; ++it) {
            const int j = p0 + it * (FA_THREADS / 8) + warp * 4 + slot;
            if (p0 > 0) {
                if (j < nc) {
                    const uint4 * kp = reinterpret_cast<const uint4 *>(kbase + (size_t) j * pstride + sub * 16);
                    kr[it][0] = kp[0];
                    kr[it][1] = kp[1];
                } else {
                    kr[it][0] = kr[it][1] = make_uint4(0, 0, 0, 0);
                }
            }
            float s = 0.0f;
            if (j < nc) {
#pragma unroll
                for (int h8 = 0; h8 < 2; ++h8) {
                    const __half2 * hp = reinterpret_cast<const __half2 *>(&kr[it][h8]);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = __half22float2(hp[k]);
                        s = fmaf(f.x, q16[8 * h8 + 2 * k], s);
                        s = fmaf(f.y, q16[8 * h8 + 2 * k + 1], s);
                    }
                }
            } else if (j < n) {
#pragma unroll
                for (int d = 0; d < 16; ++d) s = fmaf(kn[(j - jn0) * QTTS_HD + sub * 16 + d], q16[d], s);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            if (sub == 0 && j < n) sc[j] = __fmul_rn(s, a.scale);
        }
    }
    __syncthreads();   // barrier 2

    // 3. softmax (warp 0): max, expf, double sum, e * (float)(1/sum)
    if (warp == 0) {
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[j]);
        mx = warp_max(mx);
        double sum = 0.0;
        for (int j = lane; j < n; j += 32) {
            const float e = qtts_expf(__fsub_rn(sc[j], mx));
            sc[j] = e;
            sum += (double) e;
        }
        sum = warp_sum_d(sum);
        const float inv = (float)(1.0 / sum);
        float * drow = a.dump ? a.dump + ((size_t) frame * a.n_heads + hq) * a.dump_stride : nullptr;
        for (int j = lane; j < n; j += 32) {
            const float pj = __fmul_rn(sc[j], inv);
            if (drow) drow[j] = pj;
            sc[j] = a.f32_mode ? pj : round_f16(pj);
        }
    }
    __syncthreads();   // barrier 3

    // 4. P x V: position group pg takes keys pg, pg + 8, ...; thread d2 two dims
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int p0 = 0; p0 < n; p0 += FA_KPASS) {
        const __half2 * vp = reinterpret_cast<const __half2 *>(vbase + (size_t)(p0 + pg) * pstride) + d2;
        const size_t vstep = (size_t) FA_NPG * pstride / 2;
#pragma unroll
        for (int t = 0; t < FA_VIT; ++t) {
            const int j = p0 + pg + t * FA_NPG;
            float2 v;
            if (j < nc) {
                if (p0 > 0) vr[t] = vp[t * vstep];
                v = __half22float2(vr[t]);
            } else if (j < n) {
                v = make_float2(vn[(j - jn0) * QTTS_HD + 2 * d2], vn[(j - jn0) * QTTS_HD + 2 * d2 + 1]);
            } else {
                break;
            }
            const float pj = sc[j];
            acc0 = fmaf(pj, v.x, acc0);
            acc1 = fmaf(pj, v.y, acc1);
        }
    }
    part[pg * QTTS_HD + 2 * d2] = acc0;
    part[pg * QTTS_HD + 2 * d2 + 1] = acc1;
    __syncthreads();   // barrier 4
    if (tid < QTTS_HD) {
        float s = 0.0f;
#pragma unroll
        for (int q = 0; q < FA_NPG; ++q) s = __fadd_rn(s, part[q * QTTS_HD + tid]);
        a.out[(size_t) i * a.ldo + (size_t) hq * QTTS_HD + tid] = s;
        if (a.xt)
            *reinterpret_cast<__half *>(a.xt + tc_x_off(a.xt_row0 + i, hq * QTTS_HD + tid, a.xt_np)) = __float2half_rn(s);
    }
}

// Code-predictor step attention (one new row, at most 16 keys): query head hq
// by one warp, the order the oracle restates for these steps (forward_stack's
// cp_step branch).  The new row's q and k get the per-head RMSNorm and NEOX
// RoPE of the fused unit; k and v are rounded to F16 and appended to the cache
// by the group's first head.  Scores: key j belongs to lanes 2j, 2j + 1; lane
// 2j + h chains the 64 dims [64h, 64h + 64) in dim order with fused
// multiply-adds and the pair adds its halves.  Softmax: max, exp, a double sum
// of the even lanes' values over the xor butterfly, p = round_f16(e * (float)(1
// / sum)).  P x V: lane l owns dims 4l .. 4l + 3 and chains the keys in order.
// Every global load (the q|k|v row, gains, RoPE, the cached K halves and V
// quads) is issued before the first use; the new row's K/V stay in registers.
constexpr int CPA_MAX_KEYS = 16;

// xt_row >= 0 and a.xt set: the output row is also written as F16 tiles (row
// xt_row) for a tcgen05 O-projection.
__device__ __forceinline__ void cp_step_attn_body(const FusedAttn & a, const int hq, const int n_past,
                                                  const int xt_row = -1) {
    const int lane = threadIdx.x & 31;
    const int NKV = a.n_kv_heads, G = a.n_heads / NKV, g = hq / G;
    const int QD = a.n_heads * QTTS_HD, KD = NKV * QTTS_HD;
    const size_t pstride = (size_t) NKV * QTTS_HD;
    const int h = lane & 1, jk = lane >> 1;
    const float2 * rp = a.rope + (size_t) n_past * (QTTS_HD / 2);
    const float4 q4 = *reinterpret_cast<const float4 *>(a.qkv + (size_t) hq * QTTS_HD + lane * 4);
    const float4 k4 = *reinterpret_cast<const float4 *>(a.qkv + QD + (size_t) g * QTTS_HD + lane * 4);
    const float4 v4 = *reinterpret_cast<const float4 *>(a.qkv + QD + KD + (size_t) g * QTTS_HD + lane * 4);
    float gq[4], gk[4];
    float2 cs[4];
    head_params(a.q_norm, rp, lane, gq, cs);
    head_params(a.k_norm, rp, lane, gk, cs);
    uint4 kr[8];
    {
        const uint4 * kp = reinterpret_cast<const uint4 *>(a.kc + (size_t) jk * pstride + (size_t) g * QTTS_HD + 64 * h);
#pragma unroll
        for (int c = 0; c < 8; ++c) kr[c] = jk < n_past ? kp[c] : make_uint4(0, 0, 0, 0);
    }
    uint2 vr[CPA_MAX_KEYS];
    {
        const __half * vb = a.vc + (size_t) g * QTTS_HD + lane * 4;
#pragma unroll
        for (int j = 0; j < CPA_MAX_KEYS; ++j)
            vr[j] = j < n_past ? *reinterpret_cast<const uint2 *>(vb + (size_t) j * pstride) : make_uint2(0, 0);
    }
    float xq[4] = {q4.x, q4.y, q4.z, q4.w};
    float xk[4] = {k4.x, k4.y, k4.z, k4.w};
    head_norm_rope_v(xq, gq, cs, a.eps, lane);
    head_norm_rope_v(xk, gk, cs, a.eps, lane);
    float kn[4], vn[4];   // the new row's k, v (F16-rounded), dims 4 lane .. 4 lane + 3
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half kh = __float2half_rn(xk[k]), vh = __float2half_rn((&v4.x)[k]);
        xq[k] = round_f16(xq[k]);
        kn[k] = __half2float(kh);
        vn[k] = __half2float(vh);
        if (hq % G == 0) {
            a.kc[(size_t) n_past * pstride + (size_t) g * QTTS_HD + lane * 4 + k] = kh;
            a.vc[(size_t) n_past * pstride + (size_t) g * QTTS_HD + lane * 4 + k] = vh;
        }
    }
    // score of key jk over dims [64h, 64h + 64): q and the new k come from lanes 16h .. 16h + 15
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const __half2 * hp = reinterpret_cast<const __half2 *>(&kr[c]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int d = 8 * c + e, src = 16 * h + (d >> 2);     // lane holding dim 64h + d
            const float qd = __shfl_sync(0xffffffffu, xq[e & 3], src);
            const float kd_new = __shfl_sync(0xffffffffu, kn[e & 3], src);
            const float kd = jk < n_past ? (e & 1 ? __high2float(hp[e >> 1]) : __low2float(hp[e >> 1])) : kd_new;
            acc = fmaf(kd, qd, acc);
        }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    const int n = n_past + 1;
    const float s = jk < n ? __fmul_rn(acc, a.scale) : -INFINITY;
    const float mx = warp_max(s);
    const float e = jk < n ? qtts_expf(__fsub_rn(s, mx)) : 0.0f;
    const double sum = warp_sum_d(h ? 0.0 : (double) e);
    const float p = round_f16(__fmul_rn(e, (float)(1.0 / sum)));
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < CPA_MAX_KEYS + 1; ++j) {
        if (j >= n) break;
        const float pj = __shfl_sync(0xffffffffu, p, 2 * j);
        float v[4];
        if (j < n_past) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&vr[j < CPA_MAX_KEYS ? j : 0].x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&vr[j < CPA_MAX_KEYS ? j : 0].y));
            v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = vn[k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = fmaf(pj, v[k], o[k]);
    }
    *reinterpret_cast<float4 *>(a.out + (size_t) hq * QTTS_HD + lane * 4) = make_float4(o[0], o[1], o[2], o[3]);
    if (a.xt && xt_row >= 0) {
        __align__(8) __half h4[4] = {__float2half_rn(o[0]), __float2half_rn(o[1]), __float2half_rn(o[2]),
                                      __float2half_rn(o[3])};
        *reinterpret_cast<uint2 *>(a.xt + tc_x_off(xt_row, hq * QTTS_HD + lane * 4, a.xt_np)) =
            *reinterpret_cast<const uint2 *>(h4);
    }
}

// Stand-alone launch (CUDA-graph frame path): one 32-thread CTA per query head.
__global__ void __launch_bounds__(32) k_cp_step_attn(FusedAttn a) {
    pdl_trigger();
    pdl_wait();
    if (a.done && *a.done) return;
    cp_step_attn_body(a, blockIdx.x, a.pos_static);
}

// Stand-alone launch of the fused unit (CUDA-graph frame path): one CTA per unit.
__global__ void __launch_bounds__(FA_THREADS) k_fused_attention(FusedAttn a, const DevState * st) {
    pdl_trigger();
    pdl_wait();
    const int dn = a.done ? *a.done : 0;   // stop flag, position and frame: one round trip
    const int np = a.pos_ptr ? *a.pos_ptr : a.pos_static;
    const int frame = st->frame;
    if (dn) return;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    fused_attn_body(a, blockIdx.x, smem_raw, np, frame);
}

struct SampleParams {
    float temperature;
    int top_k;
    float rep_penalty;
    float eos_bias;
    int target_frames;
    int eos_id;
    int suppress_start;
    int record_logits;       // copy raw logits to the debug buffers
    unsigned long long seed;
    float * dbg_talker;      // [cap][V0]
    float * dbg_cp;          // [cap][n_cb-1][V1]
    int dbg_cap;
    int n_cb;
};

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_PER_T = 4;   // vocab <= SAMPLE_THREADS * SAMPLE_PER_T = 4096
constexpr int SAMPLE_MAX_V = 4096;

// k-th largest key among valid elements (radix select, 8 bits per pass).
template <int PT>
__device__ __forceinline__ uint32_t block_kth_largest(const uint32_t (&key)[PT], const bool (&valid)[PT], int k) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_k;
    const int tid = threadIdx.x;
    if (tid == 0) { s_prefix = 0; s_k = (uint32_t) k; }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int t = tid; t < 256; t += blockDim.x) hist[t] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        const uint32_t hi = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
#pragma unroll
        for (int e = 0; e < PT; ++e)
            if (valid[e] && ((key[e] & hi) == (prefix & hi))) atomicAdd(&hist[(key[e] >> shift) & 255u], 1u);
        __syncthreads();
        if (tid < 32) {
            // lane l owns digits 255-8l .. 248-8l (descending)
            uint32_t cnt[8], tot = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) { cnt[b] = hist[255 - 8 * tid - b]; tot += cnt[b]; }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += t;
            }
            const uint32_t excl = incl - tot;
            const uint32_t kk = s_k;
            if (excl < kk && kk <= incl) {
                uint32_t cum = excl;
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    if (cum + cnt[b] >= kk) {
                        s_prefix = prefix | ((uint32_t)(255 - 8 * tid - b) << shift);
                        s_k = kk - cum;
                        break;
                    }
                    cum += cnt[b];
                }
            }
        }
        __syncthreads();
    }
    return s_prefix;
}

// Exclusive block scan of doubles (one value per thread); *total receives the sum.
__device__ double block_exscan_d(double v, double * total) {
    __shared__ double wsum[32];
    __shared__ double wtot;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    double incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    __syncthreads();
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        double w = lane < nw ? wsum[lane] : 0.0, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            double t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < nw) wsum[lane] = wi - w;   // exclusive warp offsets
        if (lane == nw - 1) wtot = wi;
    }
    __syncthreads();
    *total = wtot;
    return wsum[warp] + (incl - v);
}

// One sampling decision by the whole block; every thread returns the token.
// cb == 0: codebook-0 rules of generate() (suppression, presence penalty, EOS
// bias ramp).  cb >= 1: code-predictor sample_or_argmax.  PT elements per thread
// (contiguous), blockDim.x * PT >= V.
// `load(l)` fills this thread's PT logits l[e] of indices tid * PT + e (< V).
template <int PT, class Load>
__device__ int sample_body_l(const Load & load, int V, int cb, const DevState * st, const SampleParams & P, int frame) {
    __shared__ float redf[32];
    __shared__ double redd[32];
    __shared__ unsigned long long best;
    __shared__ int pick;
    const int tid = threadIdx.x;
    float l[PT];
    bool valid[PT];
    load(l);
#pragma unroll
    for (int e = 0; e < PT; ++e) {
        const int i = tid * PT + e;
        valid[e] = i < V;
        if (!valid[e]) l[e] = -INFINITY;
        if (valid[e] && P.record_logits && frame < P.dbg_cap) {
            if (cb == 0) P.dbg_talker[(size_t) frame * V + i] = l[e];
            else P.dbg_cp[((size_t) frame * (P.n_cb - 1) + (cb - 1)) * V + i] = l[e];
        }
    }
    float eb = 0.0f;
    if (cb == 0) {
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            const int i = tid * PT + e;
            if (!valid[e]) continue;
            if (i >= P.suppress_start && i != P.eos_id) l[e] = -INFINITY;
            if (P.rep_penalty != 1.0f && (st->presence[i >> 5] >> (i & 31) & 1u))
                l[e] = l[e] > 0.0f ? __fdiv_rn(l[e], P.rep_penalty) : __fmul_rn(l[e], P.rep_penalty);
        }
        eb = P.eos_bias;
        if (P.target_frames > 0 && frame > P.target_frames) {
            eb = __fadd_rn(eb, __fmul_rn(0.1f, (float)(frame - P.target_frames)));
            if (eb > 6.0f) eb = 6.0f;
        }
    }
    int tok;
    if (P.temperature <= 0.0f) {
        if (cb == 0 && eb != 0.0f) {
#pragma unroll
            for (int e = 0; e < PT; ++e)
                if (valid[e] && tid * PT + e == P.eos_id) l[e] = __fadd_rn(l[e], eb);
        }
        // first index of the maximum (strict >): key = (orderable value, ~index)
        unsigned long long mine = 0ull;
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            if (!valid[e] || l[e] != l[e]) continue;
            const unsigned long long k = ((unsigned long long) f2key(l[e]) << 32) |
                                         (unsigned long long)(0xFFFFFFFFu - (uint32_t)(tid * PT + e));
            mine = k > mine ? k : mine;
        }
        // warp maximum first: one shared atomic per warp instead of one per thread
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, mine, o);
            mine = other > mine ? other : mine;
        }
        __syncthreads();
        if (tid == 0) best = 0ull;
        __syncthreads();
        if ((tid & 31) == 0) atomicMax(&best, mine);
        __syncthreads();
        tok = best == 0ull ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    } else {
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            if (!valid[e]) continue;
            l[e] = __fdiv_rn(l[e], P.temperature);
            if (cb == 0 && eb != 0.0f && tid * PT + e == P.eos_id) l[e] = __fadd_rn(l[e], eb);
        }
        if (P.top_k > 0 && P.top_k < V) {
            uint32_t key[PT];
#pragma unroll
            for (int e = 0; e < PT; ++e) key[e] = f2key(l[e]);
            const float thr = key2f(block_kth_largest<PT>(key, valid, P.top_k));
#pragma unroll
            for (int e = 0; e < PT; ++e)
                if (valid[e] && l[e] < thr) l[e] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < PT; ++e) if (valid[e]) mx = fmaxf(mx, l[e]);
        mx = block_max(mx, redf);
        float ev[PT];
        double s = 0.0;
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            ev[e] = valid[e] ? qtts_expf(__fsub_rn(l[e], mx)) : 0.0f;
            s += (double) ev[e];
        }
        const double sum = block_sum_d(s, redd);
        float p[PT];
        double loc = 0.0;
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            p[e] = valid[e] ? (float)((double) ev[e] / sum) : 0.0f;
            loc += (double) p[e];
        }
        double total;
        double cum = block_exscan_d(loc, &total);
        const double target = uniform01(P.seed, (uint32_t) frame, (uint32_t) cb) * total;
        if (tid == 0) pick = 0x7fffffff;
        __syncthreads();
        int cand = 0x7fffffff, lastpos = -1;
#pragma unroll
        for (int e = 0; e < PT; ++e) {
            cum += (double) p[e];
            if (p[e] > 0.0f) {
                lastpos = tid * PT + e;
                if (cum > target && cand == 0x7fffffff) cand = tid * PT + e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
        if ((tid & 31) == 0) atomicMin(&pick, cand);
        __syncthreads();
        if (pick == 0x7fffffff) {  // rounding pushed the target past the last bucket
            __syncthreads();
            if (tid == 0) pick = -1;
            __syncthreads();
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) lastpos = max(lastpos, __shfl_xor_sync(0xffffffffu, lastpos, o));
            if ((tid & 31) == 0) atomicMax(&pick, lastpos);
            __syncthreads();
        }
        tok = pick < 0 ? 0 : pick;
        __syncthreads();
    }
    return tok;
}

template <int PT>
__device__ __forceinline__ int sample_body(const float * logits, int V, int cb, const DevState * st,
                                           const SampleParams & P, int frame) {
    return sample_body_l<PT>(
        [&](float * l) {
#pragma unroll
            for (int e = 0; e < PT; ++e) {
                const int i = threadIdx.x * PT + e;
                l[e] = i < V ? logits[i] : -INFINITY;
            }
        },
        V, cb, st, P, frame);
}

// Records a sampled token in the frame state (thread 0 only).
__device__ __forceinline__ void sample_commit(int tok, int cb, DevState * st, const SampleParams & P, int * out_codes,
                                              int out_cap, int frame) {
    if (cb == 0) {
        if (tok == P.eos_id) {
            st->done = 1;
            return;
        }
        st->codes[0] = tok;
        st->presence[tok >> 5] |= 1u << (tok & 31);
    } else {
        st->codes[cb] = tok;
    }
    if (out_codes && frame < out_cap) out_codes[(size_t) frame * P.n_cb + cb] = tok;
}

__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample(const float * logits, int V, int cb, DevState * st,
                                                           const SampleParams * sp, int * out_codes, int out_cap) {
    pdl_trigger();
    pdl_wait();
    const int dn = st->done, frame = st->frame;   // loaded together with the parameters
    const SampleParams P = *sp;
    if (dn) return;
    const int tok = sample_body<SAMPLE_PER_T>(logits, V, cb, st, P, frame);
    if (threadIdx.x == 0) sample_commit(tok, cb, st, P, out_codes, out_cap, frame);
}

// ---------------------------------------------------------------------------
enum InMode : int { IN_CP_PREFILL = 0, IN_CP_STEP = 1, IN_TALKER = 2 };

struct InputArgs {
    int mode;
    int g;                        // IN_CP_STEP: codebook index 1..n_cb-2
    int H;
    const __half * codec_embd;    // [V0][H]
    const __half * const * cp_embd;  // device array of n_cb-1 pointers, each [V1][H]
    const float * hidden;         // talker post-norm hidden [H]
    const float * trailing;       // [st->n_trailing][H]
    const float * pad;            // tts_pad projection [H]
    float * out;                  // [rows][H]
    DevState * st;
    int n_cb;
    const __half * step_tab;      // IN_CP_STEP: cp_embd[g - 1]
};

// Inputs of the next pass, built by the sampling CTA right after it sampled:
// codes[0..cb] (shared memory) hold this frame's codes so far, tabs[1..n_cb-1] the
// code-predictor embedding tables, n_trailing the trailing text rows.  Same
// sums in the same order as k_frame_inputs.
__device__ void frame_inputs_body(const InputArgs & a, const int frame, const int * codes,
                                  const __half * const * tabs, const int n_trailing) {
    for (int h = threadIdx.x; h < a.H; h += blockDim.x) {
        if (a.mode == IN_CP_PREFILL) {
            a.out[h] = a.hidden[h];
            a.out[a.H + h] = __half2float(a.codec_embd[(size_t) codes[0] * a.H + h]);
        } else if (a.mode == IN_CP_STEP) {
            a.out[h] = __half2float(a.step_tab[(size_t) codes[a.g] * a.H + h]);
        } else {
            float e[QTTS_MAX_CB];
            e[0] = __half2float(a.codec_embd[(size_t) codes[0] * a.H + h]);
#pragma unroll
            for (int cb = 1; cb < QTTS_MAX_CB; ++cb)
                e[cb] = cb < a.n_cb ? __half2float(tabs[cb][(size_t) codes[cb] * a.H + h]) : 0.0f;
            const float * tr = frame < n_trailing ? a.trailing + (size_t) frame * a.H : a.pad;
            const float t = tr[h];
            float s = e[0];
#pragma unroll
            for (int cb = 1; cb < QTTS_MAX_CB; ++cb)
                if (cb < a.n_cb) s = __fadd_rn(s, e[cb]);
            a.out[h] = __fadd_rn(s, t);
        }
    }
}

// Sampler of codebook cb followed by the next input rows (CUDA-graph frame
// path): one launch instead of k_sample + k_frame_inputs, with the decisions of
// k_sample and the sums of frame_inputs_body.  `in.mode` IN_CP_PREFILL follows
// codebook 0, IN_CP_STEP (g = cb) a code-predictor codebook, IN_TALKER the last
// codebook of the frame.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_inputs(const float * logits, int V, int cb, DevState * st,
                                                                  const SampleParams * sp, int * out_codes,
                                                                  int out_cap, InputArgs in) {
    __shared__ int s_codes[QTTS_MAX_CB];
    __shared__ const __half * s_tabs[QTTS_MAX_CB];
    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x;
    // frame state, earlier codes and table pointers: loaded together, before the sampler needs them
    const int dn = st->done, frame = st->frame, n_trailing = st->n_trailing;
    const SampleParams P = *sp;
    int c_pre = 0;
    const __half * t_pre = nullptr;
    if (in.mode == IN_TALKER) {
        if (tid < cb) c_pre = st->codes[tid];
        if (tid >= 1 && tid < in.n_cb) t_pre = in.cp_embd[tid - 1];
    }
    if (dn) return;
    const int tok = sample_body<SAMPLE_PER_T>(logits, V, cb, st, P, frame);
    if (tid == 0) sample_commit(tok, cb, st, P, out_codes, out_cap, frame);
    if (tid < cb) s_codes[tid] = c_pre;
    if (tid == 0) s_codes[cb] = tok;
    if (tid < QTTS_MAX_CB) s_tabs[tid] = t_pre;
    __syncthreads();
    frame_inputs_body(in, frame, s_codes, s_tabs, n_trailing);
}

__global__ void k_frame_inputs(InputArgs a) {
    pdl_trigger();
    pdl_wait();
    if (a.st->done) return;
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

__global__ void k_frame_end(DevState * st) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0 && !st->done) {
        st->pos += 1;
        st->frame += 1;
        st->n_out += 1;
    }
}

// Row-wise RMSNorm * gain (F32 out), for hidden_states of all prefill rows.
__global__ void k_rmsnorm_rows(const float * x, int ldx, const float * g, float eps, int H, float * y, int ldy) {
    __shared__ double red[32];
    const float * xr = x + (size_t) blockIdx.x * ldx;
    double ss = 0.0;
    for (int c = threadIdx.x; c < H; c += blockDim.x) ss += (double) __fmul_rn(xr[c], xr[c]);
    ss = block_sum_d(ss, red);
    const float mean = (float)(ss / (double) H);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
    for (int c = threadIdx.x; c < H; c += blockDim.x)
        y[(size_t) blockIdx.x * ldy + c] = __fmul_rn(__fmul_rn(xr[c], scale), g[c]);
}

// F16 rows -> F32 (embedding gathers of the host API).
__global__ void k_gather_rows(const __half * table, int dim, const int * ids, int n, float * out) {
    const int r = blockIdx.x;
    if (r >= n) return;
    for (int c = threadIdx.x; c < dim; c += blockDim.x)
        out[(size_t) r * dim + c] = __half2float(table[(size_t) ids[r] * dim + c]);
}

// ICL reference-frame codec rows (build_prefill_graph_icl, src/tts_transformer.cpp:
// 1188-1472): row f = codec_embd[code(f, 0)], then += code_pred_embd[cb - 1]
// [code(f, cb)] for cb = 1 .. n_cb - 1, the host loop's F32 sums in codebook
// order.  codes: [n_frames][16].
__global__ void k_icl_codec_rows(const __half * codec_embd, const __half * const * cp_embd, const int * codes,
                                 int n_cb, int H, float * out) {
    const int f = blockIdx.x;
    const int * cf = codes + (size_t) f * 16;
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        float s = __half2float(codec_embd[(size_t) cf[0] * H + h]);
        for (int cb = 1; cb < n_cb; ++cb) s = __fadd_rn(s, __half2float(cp_embd[cb - 1][(size_t) cf[cb] * H + h]));
        out[(size_t) f * H + h] = s;
    }
}

// One row of the assembled prompt (prefill rows, trailing text rows, pad row):
// dst = a, or 0 + a, then + b when b is set, in that order (the reference
// builds these rows with ggml_add of the same terms,
// src/tts_transformer.cpp:1030-1472).
struct PromptRow {
    float * dst;
    const float * a, * b;
    int zero_first;
};

// One CTA per row; every term is already an F32 row in device memory.
__global__ void k_prompt_rows(const PromptRow * rows, int H) {
    const PromptRow r = rows[blockIdx.x];
    for (int d = threadIdx.x; d < H; d += blockDim.x) {
        float v = r.a[d];
        if (r.zero_first) v = __fadd_rn(0.0f, v);
        if (r.b) v = __fadd_rn(v, r.b[d]);
        r.dst[d] = v;
    }
}

// y = silu(x + b) in place (text projection fc1 epilogue).
__global__ void k_bias_silu(float * x, const float * b, int n, int ld, int rows) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * rows; i += gridDim.x * blockDim.x) {
        const int r = i / n, c = i % n;
        x[(size_t) r * ld + c] = silu(__fadd_rn(x[(size_t) r * ld + c], b[c]));
    }
}
__global__ void k_bias_add(float * x, const float * b, int n, int ld, int rows) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * rows; i += gridDim.x * blockDim.x) {
        const int r = i / n, c = i % n;
        x[(size_t) r * ld + c] = __fadd_rn(x[(size_t) r * ld + c], b[c]);
    }
}

}  // namespace qtts
