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
    float * xn_out;         // CTA 0 writes the normalised input rows here (F32)
    int ldxn;
    const int * done;       // frame-loop stop flag (skip when *done)
    int kslices;            // k-slices per row inside a CTA
    int * block_dots;       // Q8_0 test hook: per-block int32 dots [nv][rows][cols/32] (nullptr: off)
};

// Shared memory: float xs[NV][cols]; Q8_0 additionally int8 qa[NV][cols] and
// float da[NV][cols/32]; then the per-item partials float[rpc*kslices][NV][2].
__host__ __device__ inline size_t gemv_smem_bytes(int type, int cols, int nv, int rpc, int kslices) {
    size_t b = (size_t) nv * cols * 4;
    if (type == W_Q8_0) b += (size_t) nv * cols + (size_t) nv * (cols / 32) * 4;
    b += (size_t) rpc * kslices * nv * 2 * 4;
    return b;
}

template <int NV>
__device__ __forceinline__ void gemv_prologue(const GemvArgs & a, float * xs, int8_t * qa, float * da, const int cta) {
    __shared__ double red[32];
    const int cols = a.A.cols;
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int v = 0; v < NV; ++v) {
        float * xr = xs + (size_t) v * cols;
        if (v >= a.nv) {
            for (int c = tid; c < cols; c += nt) xr[c] = 0.0f;
            continue;
        }
        const float * src = a.x + (size_t) v * a.ldx;
        double ss = 0.0;
        for (int c = tid; c < cols; c += nt) {
            const float t = src[c];
            xr[c] = t;
            ss += (double) __fmul_rn(t, t);
        }
        if (a.norm_g) {
            ss = block_sum_d(ss, red);
            const float mean = (float)(ss / (double) cols);
            const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, a.eps)));
            for (int c = tid; c < cols; c += nt) xr[c] = __fmul_rn(__fmul_rn(xr[c], scale), a.norm_g[c]);
        }
        if (a.xn_out && cta == 0)
            for (int c = tid; c < cols; c += nt) a.xn_out[(size_t) v * a.ldxn + c] = xr[c];
    }
    __syncthreads();
    if (a.A.type == W_F16) {
        if (a.act == ACT_F16)
            for (int i = tid; i < NV * cols; i += nt) xs[i] = round_f16(xs[i]);
    } else {  // Q8_0: quantize_row_q8_0_ref per 32-block, one warp per block
        const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
        const int nb = cols / 32;
        for (int blk = warp; blk < NV * nb; blk += nw) {
            const int v = blk / nb, b = blk % nb;
            const float val = xs[(size_t) v * cols + b * 32 + lane];
            const float amax = warp_max(fabsf(val));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            qa[(size_t) v * cols + b * 32 + lane] = (int8_t) roundf(__fmul_rn(val, id));
            if (lane == 0) da[(size_t) v * nb + b] = __half2float(__float2half_rn(d));
        }
    }
    __syncthreads();
}

template <int NV>
__device__ __forceinline__ void gemv_store(const GemvArgs & a, int r, int v, float accA, float accB) {
    if (v >= a.nv) return;
    float out;
    if (a.epi == EPI_SWIGLU) out = __fmul_rn(silu(accA), accB);
    else if (a.epi == EPI_RESID) out = __fadd_rn(accA, a.resid[(size_t) v * a.ldr + r]);
    else out = accA;
    a.y[(size_t) v * a.ldy + r] = out;
}

// Rows of A (and B) are split into contiguous per-CTA ranges.  Inside a CTA
// the work items are (row, k-slice) pairs; a warp takes two items at a time
// and issues all 16-byte loads of an iteration before the math.  Per-item
// partial dots go to shared memory and are summed in slice order, so the
// result depends only on (rows, grid, kslices), never on scheduling.
// Where a CTA reads its weight rows from: global memory (streaming loads) or a
// shared-memory copy of its row slice [r0, r1) (persistent frame kernel).
struct WSrc {
    const uint8_t * a, * b;       // F16 halves or int8 quants, row stride cols * elem size
    const __half * sa, * sb;      // Q8_0 scales, row stride cols / 32
    int rbase;                    // first row held by the pointers (0 for global)
};

template <bool SMEM>
__device__ __forceinline__ uint4 ld_w16(const uint8_t * p) {
    if constexpr (SMEM) return *reinterpret_cast<const uint4 *>(p);
    else return ld_stream(p);
}

template <int NV, bool SMEM = false>
__device__ __forceinline__ void gemv_body(const GemvArgs & a, const int cta, const int ncta, uint8_t * smem_raw,
                                          const WSrc * wsrc = nullptr) {
    const int cols = a.A.cols, rows = a.A.rows;
    const int rpc = (rows + ncta - 1) / ncta;
    const int r0 = cta * rpc, r1 = min(rows, r0 + rpc);
    if (r0 >= r1) return;
    WSrc src;
    if (SMEM) src = *wsrc;
    else src = WSrc{static_cast<const uint8_t *>(a.A.w), static_cast<const uint8_t *>(a.B.w), a.A.d, a.B.d, 0};
    float * xs = reinterpret_cast<float *>(smem_raw);
    int8_t * qa = reinterpret_cast<int8_t *>(xs + (size_t) NV * cols);
    float * da = reinterpret_cast<float *>(qa + (size_t)(a.A.type == W_Q8_0 ? NV * cols : 0));
    float * part = da + (a.A.type == W_Q8_0 ? NV * (cols / 32) : 0);
    gemv_prologue<NV>(a, xs, qa, da, cta);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool dual = a.B.w != nullptr;
    const int S = a.kslices;
    const int nrow = r1 - r0, n_items = nrow * S;
    constexpr int IU = 2, KU = 4;

    if (a.A.type == W_F16) {
        const int nchunk = cols / 8;
        const int sl = (nchunk + S - 1) / S;
        for (int it0 = warp * IU; it0 < n_items; it0 += QTTS_WARPS * IU) {
            float accA[IU][NV], accB[IU][NV];
            int row[IU], cbeg[IU], cend[IU];
#pragma unroll
            for (int u = 0; u < IU; ++u) {
                const int it = it0 + u;
                const bool iv = it < n_items;
                row[u] = r0 + (iv ? it / S : 0);
                cbeg[u] = (iv ? it % S : 0) * sl;
                cend[u] = iv ? min(nchunk, cbeg[u] + sl) : 0;
#pragma unroll
                for (int v = 0; v < NV; ++v) accA[u][v] = accB[u][v] = 0.0f;
            }
            for (int cc = 0; cc < sl; cc += 32 * KU) {
                uint4 wa[IU][KU], wb[IU][KU];
#pragma unroll
                for (int u = 0; u < IU; ++u)
#pragma unroll
                    for (int k = 0; k < KU; ++k) {
                        const int c = cbeg[u] + cc + lane + 32 * k;
                        const bool ok = c < cend[u];
                        const size_t off = ((size_t)(row[u] - src.rbase) * cols + (size_t) c * 8) * 2;
                        wa[u][k] = ok ? ld_w16<SMEM>(src.a + off) : make_uint4(0, 0, 0, 0);
                        wb[u][k] = (ok && dual) ? ld_w16<SMEM>(src.b + off) : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                for (int u = 0; u < IU; ++u)
#pragma unroll
                    for (int k = 0; k < KU; ++k) {
                        const int c = cbeg[u] + cc + lane + 32 * k;
                        if (c >= cend[u]) continue;
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const float * xv = xs + (size_t) v * cols + (size_t) c * 8;
                            accA[u][v] = dot8(wa[u][k], xv, accA[u][v]);
                            if (dual) accB[u][v] = dot8(wb[u][k], xv, accB[u][v]);
                        }
                    }
            }
#pragma unroll
            for (int u = 0; u < IU; ++u)
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    const float sa = warp_sum(accA[u][v]);
                    const float sb = dual ? warp_sum(accB[u][v]) : 0.0f;
                    if (lane == 0 && it0 + u < n_items) {
                        part[((size_t)(it0 + u) * NV + v) * 2 + 0] = sa;
                        part[((size_t)(it0 + u) * NV + v) * 2 + 1] = sb;
                    }
                }
        }
    } else {  // Q8_0: 16 quants per lane-chunk, lane pairs form one 32-block
        const int nchunk = cols / 16, nb = cols / 32;
        const int sl = (((nchunk + S - 1) / S) + 1) & ~1;   // even: slices start on a block
        for (int it0 = warp * IU; it0 < n_items; it0 += QTTS_WARPS * IU) {
            float accA[IU][NV], accB[IU][NV];
            int row[IU], cbeg[IU], cend[IU];
#pragma unroll
            for (int u = 0; u < IU; ++u) {
                const int it = it0 + u;
                const bool iv = it < n_items;
                row[u] = r0 + (iv ? it / S : 0);
                cbeg[u] = (iv ? it % S : 0) * sl;
                cend[u] = iv ? min(nchunk, cbeg[u] + sl) : 0;
#pragma unroll
                for (int v = 0; v < NV; ++v) accA[u][v] = accB[u][v] = 0.0f;
            }
            for (int cc = 0; cc < sl; cc += 32 * KU) {
                uint4 wa[IU][KU], wb[IU][KU];
                float swa[IU][KU], swb[IU][KU];
#pragma unroll
                for (int u = 0; u < IU; ++u)
#pragma unroll
                    for (int k = 0; k < KU; ++k) {
                        const int c = cbeg[u] + cc + lane + 32 * k;
                        const bool ok = c < cend[u];
                        const size_t ro = (size_t)(row[u] - src.rbase);
                        wa[u][k] = ok ? ld_w16<SMEM>(src.a + ro * cols + (size_t) c * 16) : make_uint4(0, 0, 0, 0);
                        wb[u][k] = (ok && dual) ? ld_w16<SMEM>(src.b + ro * cols + (size_t) c * 16) : make_uint4(0, 0, 0, 0);
                        swa[u][k] = ok ? __half2float(src.sa[ro * nb + (c >> 1)]) : 0.0f;
                        swb[u][k] = (ok && dual) ? __half2float(src.sb[ro * nb + (c >> 1)]) : 0.0f;
                    }
#pragma unroll
                for (int u = 0; u < IU; ++u)
#pragma unroll
                    for (int k = 0; k < KU; ++k) {
                        const int c = cbeg[u] + cc + lane + 32 * k;
                        const bool okc = c < cend[u];   // uniform within a lane pair
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const int4 xq = okc ? *reinterpret_cast<const int4 *>(qa + (size_t) v * cols + (size_t) c * 16)
                                                : make_int4(0, 0, 0, 0);
                            const float dx = okc ? da[(size_t) v * nb + (c >> 1)] : 0.0f;
                            int ia = __dp4a((int) wa[u][k].x, xq.x, 0);
                            ia = __dp4a((int) wa[u][k].y, xq.y, ia);
                            ia = __dp4a((int) wa[u][k].z, xq.z, ia);
                            ia = __dp4a((int) wa[u][k].w, xq.w, ia);
                            ia += __shfl_xor_sync(0xffffffffu, ia, 1);   // 32-block int32 dot
                            if (a.block_dots && !(lane & 1) && okc && v < a.nv)
                                a.block_dots[((size_t) v * rows + row[u]) * nb + (c >> 1)] = ia;
                            if (!(lane & 1) && okc)
                                accA[u][v] = __fadd_rn(accA[u][v], __fmul_rn((float) ia, __fmul_rn(swa[u][k], dx)));
                            if (dual) {
                                int ib = __dp4a((int) wb[u][k].x, xq.x, 0);
                                ib = __dp4a((int) wb[u][k].y, xq.y, ib);
                                ib = __dp4a((int) wb[u][k].z, xq.z, ib);
                                ib = __dp4a((int) wb[u][k].w, xq.w, ib);
                                ib += __shfl_xor_sync(0xffffffffu, ib, 1);
                                if (!(lane & 1) && okc)
                                    accB[u][v] = __fadd_rn(accB[u][v], __fmul_rn((float) ib, __fmul_rn(swb[u][k], dx)));
                            }
                        }
                    }
            }
#pragma unroll
            for (int u = 0; u < IU; ++u)
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    const float s1 = warp_sum(accA[u][v]);
                    const float s2 = dual ? warp_sum(accB[u][v]) : 0.0f;
                    if (lane == 0 && it0 + u < n_items) {
                        part[((size_t)(it0 + u) * NV + v) * 2 + 0] = s1;
                        part[((size_t)(it0 + u) * NV + v) * 2 + 1] = s2;
                    }
                }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < nrow * NV; t += blockDim.x) {
        const int rl = t / NV, v = t % NV;
        float sa = 0.0f, sb = 0.0f;
        for (int s2 = 0; s2 < S; ++s2) {
            sa = __fadd_rn(sa, part[((size_t)(rl * S + s2) * NV + v) * 2 + 0]);
            sb = __fadd_rn(sb, part[((size_t)(rl * S + s2) * NV + v) * 2 + 1]);
        }
        gemv_store<NV>(a, r0 + rl, v, sa, sb);
    }
}

template <int NV>
__global__ void __launch_bounds__(QTTS_WARPS * 32) k_gemv(GemvArgs a) {
    if (a.done && *a.done) return;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    gemv_body<NV>(a, blockIdx.x, gridDim.x, smem_raw);
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

__device__ __forceinline__ void head_norm_rope(float x[4], const float * g, float eps, const float2 * rp, int lane) {
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) ss += (double) __fmul_rn(x[k], x[k]);
    ss = warp_sum_d(ss);
    const float mean = (float)(ss / (double) QTTS_HD);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, eps)));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float t = __fmul_rn(x[k], scale);
        x[k] = g ? __fmul_rn(t, g[lane * 4 + k]) : t;
    }
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __shfl_xor_sync(0xffffffffu, x[k], 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int d = lane * 4 + k;
        if (lane < 16) {  // first half: x0 = x[d], x1 = x[d + 64]
            const float2 cs = rp[d];
            x[k] = __fsub_rn(__fmul_rn(x[k], cs.x), __fmul_rn(o[k], cs.y));
        } else {          // second half: x0 = x[d - 64], x1 = x[d]
            const float2 cs = rp[d - 64];
            x[k] = __fadd_rn(__fmul_rn(o[k], cs.y), __fmul_rn(x[k], cs.x));
        }
    }
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
    extern __shared__ __align__(16) uint8_t smem_raw[];
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
            const float e = expf(__fsub_rn(sc[h * n + j], mx));
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
__device__ uint32_t block_kth_largest(const uint32_t * key, const bool * valid, int k) {
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
template <int PT>
__device__ int sample_body(const float * logits, int V, int cb, const DevState * st, const SampleParams & P, int frame) {
    __shared__ float redf[32];
    __shared__ double redd[32];
    __shared__ unsigned long long best;
    __shared__ int pick;
    const int tid = threadIdx.x;
    float l[PT];
    bool valid[PT];
#pragma unroll
    for (int e = 0; e < PT; ++e) {
        const int i = tid * PT + e;
        valid[e] = i < V;
        l[e] = valid[e] ? logits[i] : -INFINITY;
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
        __syncthreads();
        if (tid == 0) best = 0ull;
        __syncthreads();
        atomicMax(&best, mine);
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
            ev[e] = valid[e] ? expf(__fsub_rn(l[e], mx)) : 0.0f;
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
        atomicMin(&pick, cand);
        __syncthreads();
        if (pick == 0x7fffffff) {  // rounding pushed the target past the last bucket
            __syncthreads();
            if (tid == 0) pick = -1;
            __syncthreads();
            atomicMax(&pick, lastpos);
            __syncthreads();
        }
        tok = pick < 0 ? 0 : pick;
        __syncthreads();
    }
    return tok;
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
    if (st->done) return;
    const SampleParams P = *sp;
    const int frame = st->frame;
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
};

__global__ void k_frame_inputs(InputArgs a) {
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
