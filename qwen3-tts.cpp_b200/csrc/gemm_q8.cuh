// gemm_q8.cuh — Q8_0 GEMM on the tcgen05 tensor cores (kind::i8) for the
// batched frame loop: Y[m][r] = sum over 32-blocks b of
// (float) isum(W[r] block b, Xq[m] block b) * (d_w[r][b] * d_a[m][b]), the
// per-block integer dot of ggml's Q8_0 x Q8_0 vec_dot (quantize_row_q8_0 on the
// activation, int8 products summed in int32) scaled by the two block scales.
//
// One tcgen05.mma of kind::i8 has K = 32: exactly one Q8_0 block.  Each block's
// MMA writes its own TMEM columns (no accumulation in TMEM), so the tensor core
// delivers the exact int32 block dots; epilogue warps read them with
// tcgen05.ld while later blocks are multiplied (TMEM columns double-buffered per
// 128-byte k-tile) and accumulate in F32 in block order:
//   acc = 0; for b: acc = acc + (float) isum_b * (d_w_b * d_a_b)
// which is the reference's sequential Q8_0 row dot.  With a k-split over a
// cluster of S CTAs, CTA s sums its block range that way and the tile owner adds
// the S partials in rank order (0 + P_0 + P_1 + ...).
//
// Layout: int8 weights and activations in the no-swizzle K-major core-matrix
// tiles of k_gemm_tc, read as bytes: a tile of 128 rows x 128 int8 is 16
// groups of 8 rows x 128 bytes, each group eight 128-byte core matrices (8 rows
// x 16 bytes) in k order; block j of a k-tile is core matrices 2j, 2j + 1.
// Weight block scales are repacked as [row tile][k-tile][128 rows][4] F16.
//
// Roles (320 threads): warps 0-7 drain TMEM and run the epilogue (warp w reads
// lanes 32 (w % 4) .. 32 (w % 4) + 31 = weight rows, and the 16-column chunks
// w / 4, w / 4 + 2, ... of the activation columns), warp 8 lane 0 streams W and
// X tiles through a shared-memory ring, warp 9 allocates TMEM and its lane 0
// issues the MMAs.  Every wait is bounded.
#pragma once
#include "gemm_tc.cuh"

namespace qtts {

constexpr int Q8_BK = 128;          // int8 k per tile (four Q8_0 blocks)
constexpr int Q8_EPI_WARPS = 8;     // epilogue warps: two per TMEM lane quarter (column halves)
constexpr int Q8_PRODUCER = Q8_EPI_WARPS * 32;        // thread that streams the tiles
constexpr int Q8_MMA_WARP = Q8_EPI_WARPS + 1;         // warp that owns TMEM; its lane 0 issues the MMAs
constexpr int Q8_THREADS = (Q8_EPI_WARPS + 2) * 32;
constexpr int Q8_MAX_N = 128;       // activation rows (MMA N) per launch
constexpr int Q8_MAX_STAGES = 8;

// Byte offset of int8 element (row r, k) inside a 128-wide k-tile of `rows` rows.
__host__ __device__ inline size_t q8_tile_off(int r, int k) {
    return (size_t)(r >> 3) * 1024 + (size_t)((k & 127) >> 4) * 128 + (size_t)(r & 7) * 16 + (size_t)(k & 15);
}
__host__ __device__ inline size_t q8_w_off(int r, int k, int cols) {
    return ((size_t)(r / TC_BM) * (cols / Q8_BK) + (size_t)(k / Q8_BK)) * (TC_BM * Q8_BK) + q8_tile_off(r % TC_BM, k);
}
__host__ __device__ inline size_t q8_x_off(int m, int k, int np) {
    return (size_t)(k / Q8_BK) * np * 128 + q8_tile_off(m, k);
}
// Weight scale (row r, block b) in the repacked scale plane.
__host__ __device__ inline size_t q8_s_off(int r, int b, int cols) {
    return (((size_t)(r / TC_BM) * (cols / Q8_BK) + (size_t)(b / 4)) * TC_BM + (size_t)(r % TC_BM)) * 4 + (size_t)(b & 3);
}

// Repack split-plane Q8_0 W[rows][cols] (int8 plane + scale plane) into tiles.
// W2: the gate/up pair, interleaved in 64-row groups as k_tile_weights does.
__global__ void k_tile_q8(DMat W, DMat W2, int rows_w, uint8_t * out, __half * sout) {
    const int r = blockIdx.x, cols = W.cols, nb = cols / 32;
    int src_r = r;
    const DMat * src = &W;
    if (W2.w) {
        const int tn = r / TC_BM, rr = r % TC_BM;
        src_r = tn * (TC_BM / 2) + (rr & (TC_BM / 2 - 1));
        src = rr < TC_BM / 2 ? &W : &W2;
    }
    const int8_t * q = static_cast<const int8_t *>(src->w) + (size_t) src_r * cols;
    for (int k16 = threadIdx.x; k16 < cols / 16; k16 += blockDim.x)
        *reinterpret_cast<uint4 *>(out + q8_w_off(r, k16 * 16, cols)) = *reinterpret_cast<const uint4 *>(q + k16 * 16);
    for (int b = threadIdx.x; b < nb; b += blockDim.x) sout[q8_s_off(r, b, cols)] = src->d[(size_t) src_r * nb + b];
    (void) rows_w;
}

// Activation rows -> Q8_0 int8 tiles + block scales, as quantize_row_q8_0_ref
// (d = amax / 127 rounded to F16, q = roundf(x / d)); optional RMSNorm first
// (double sum, as k_pack_act).  Rows >= m_real are zero.  One CTA per padded row.
struct PackQ8Args {
    const float * x;
    int ldx;
    int m_real, np, cols;
    const float * gain;        // nullptr: no norm
    float eps;
    uint8_t * out;             // tiled [cols/128][np][128] int8
    float * dscale;            // [np][cols/32]: the F16 block scales as F32
};

__global__ void __launch_bounds__(256) k_pack_q8(PackQ8Args a) {
    __shared__ double red[8];
    __shared__ float s_scale;
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    const bool real = m < a.m_real;
    const float * row = a.x + (size_t) m * a.ldx;
    float scale = 1.0f;
    if (a.gain && real) {
        double ss = 0.0;
        for (int c = tid; c < a.cols; c += blockDim.x) { const float t = row[c]; ss += (double) __fmul_rn(t, t); }
        ss = warp_sum_d(ss);
        if (lane == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid == 0) {
            double t = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
            s_scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(t / (double) a.cols), a.eps)));
        }
        __syncthreads();
        scale = s_scale;
    }
    // a warp quantises one 32-block per pass: lane = column in the block
    const int nb = a.cols / 32;
    for (int b = tid >> 5; b < nb; b += blockDim.x >> 5) {
        const int c = b * 32 + lane;
        float t = real ? row[c] : 0.0f;
        if (a.gain && real) t = __fmul_rn(__fmul_rn(t, scale), a.gain[c]);
        float am = fabsf(t);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float d = __fdiv_rn(am, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        a.out[q8_x_off(m, c, a.np)] = (uint8_t)(int8_t) roundf(__fmul_rn(t, id));
        if (lane == 0) a.dscale[(size_t) m * nb + b] = __half2float(__float2half_rn(d));
    }
}

struct GemmQ8Args {
    const uint8_t * w;        // int8 weight tiles, rows_w x cols
    const __half * ws;        // weight block scales (q8_s_off)
    const uint8_t * x;        // int8 activation tiles, np x cols
    const float * xs;         // activation block scales [np][cols/32]
    int rows_w, cols, np;     // np: MMA N (multiple of 16, <= Q8_MAX_N)
    int m_real;
    int epi;                  // TC_EPI_STORE / TC_EPI_RESID / TC_EPI_SWIGLU (gate/up interleaved tiles)
    float * y;
    int ldy;
    const float * resid;
    int ldr;
    int * err;
    int ksplit;               // CTAs per weight tile along k (a cluster; 1 = no split)
};

__device__ __forceinline__ void mbar_arrive_cta(uint64_t * m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(m)) : "memory");
}

// kind::i8: S32 accumulator, signed int8 A and B, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t q8_idesc(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}
__device__ __forceinline__ void q8_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(0));
}
__device__ __forceinline__ void q8_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                   "=r"(v[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void q8_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                   "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                   "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
                   "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMEM: NBUF buffers of 4 blocks x np columns (one buffer per k-tile in flight).
__host__ __device__ inline int q8_nbuf(int np) {
    const int n = 512 / (4 * np);
    return n > 4 ? 4 : (n < 1 ? 1 : n);
}
__host__ __device__ inline size_t q8_stage_bytes(int np) { return (size_t) TC_BM * Q8_BK + (size_t) np * 128; }
// Activation scales in shared memory [np][cols / 32] (np is a multiple of 16,
// the epilogue's column chunk).
__host__ __device__ inline size_t q8_scale_bytes(int np, int cols) { return (size_t) np * (cols / 32) * 4; }
__host__ __device__ inline size_t q8_partial_bytes(int np, int m_real, int ksplit) {
    if (ksplit <= 1) return 0;
    const int pc = m_real < np ? m_real : np;
    return (size_t) TC_BM * (((pc + 3) & ~3) + 4) * 4;
}
__host__ __device__ inline int q8_stages(int np, int cols, size_t pbytes) {
    const long avail = 200L * 1024 - (long) pbytes - (long) q8_scale_bytes(np, cols) - 1024;
    const int n = (int)(avail / (long) q8_stage_bytes(np));
    return n > Q8_MAX_STAGES ? Q8_MAX_STAGES : n;
}
__host__ __device__ inline size_t q8_smem_bytes(int np, int cols, size_t pbytes) {
    return (size_t) q8_stages(np, cols, pbytes) * q8_stage_bytes(np) + q8_scale_bytes(np, cols) + pbytes + 1024;
}

template <int NACC>   // accumulator columns of the launch (>= np); a thread holds NACC / 2
__global__ void __launch_bounds__(Q8_THREADS, 1) k_gemm_q8(GemmQ8Args g) {
    constexpr int NA = NACC / 2;   // columns per epilogue thread: 16-column chunks h, h + 2, h + 4, ...
    extern __shared__ __align__(128) uint8_t q8_smem[];
    __shared__ __align__(8) uint64_t full[Q8_MAX_STAGES], empty[Q8_MAX_STAGES], accf[4], acce[4];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ float s_swg[2][TC_BM / 2][17];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = g.ksplit > 1 ? g.ksplit : 1;
    const int tn = blockIdx.x / S, rank = blockIdx.x % S;
    const int nk_all = g.cols / Q8_BK;
    const int k0 = rank * nk_all / S, nk = (rank + 1) * nk_all / S - k0;
    const size_t wtile = (size_t) TC_BM * Q8_BK, xtile = (size_t) g.np * 128;
    const size_t sbytes = wtile + xtile;
    const size_t pbytes = q8_partial_bytes(g.np, g.m_real, g.ksplit);
    const int NST = q8_stages(g.np, g.cols, pbytes);
    const int NBUF = q8_nbuf(g.np);
    const int nb = g.cols / 32;
    float * xsc = reinterpret_cast<float *>(q8_smem + NST * sbytes);          // activation scales [np][nb]
    float * P = reinterpret_cast<float *>(q8_smem + NST * sbytes + q8_scale_bytes(g.np, g.cols));   // k-split slots
    int ncols = 32;
    while (ncols < NBUF * 4 * g.np) ncols <<= 1;
    // epilogue warp (q, h): TMEM lane quarter q = warp % 4 (weight rows 32q .. 32q + 31), column half h
    const int q4 = warp & 3, hh = (warp >> 2) & 1;
    const int r_tile = q4 * 32 + lane;

    const uint8_t * wsrc = g.w + ((size_t) tn * nk_all + k0) * wtile;
    const uint8_t * xsrc = g.x + (size_t) k0 * xtile;
    int issued = 0;
    pdl_trigger();
    if (tid == Q8_PRODUCER) {
        for (int s = 0; s < NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 4; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], Q8_EPI_WARPS); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
        for (int i = 0; i < nk && i < NST; ++i) {   // weight tiles are read-only: copy before the predecessor ends
            mbar_expect_tx(&full[i], (unsigned) sbytes);
            bulk_g2s(q8_smem + i * sbytes, wsrc + (size_t) i * wtile, (unsigned) wtile, &full[i]);
            issued = i + 1;
        }
    }
    if (warp == Q8_MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_wait();   // activations, their scales, residuals and outputs follow the predecessor
    if (tid == Q8_PRODUCER)
        for (int i = 0; i < issued; ++i)
            bulk_g2s(q8_smem + i * sbytes + wtile, xsrc + (size_t) i * xtile, (unsigned) xtile, &full[i]);
    for (int i = tid; i < g.np * nb; i += Q8_THREADS) xsc[i] = g.xs[i];
    __syncthreads();

    const int pc = g.m_real < g.np ? g.m_real : g.np;   // output columns kept
    float acc[NA];
#pragma unroll
    for (int i = 0; i < NA; ++i) acc[i] = 0.0f;
    bool ok = true;
    if (tid == Q8_PRODUCER) {
        // producer: W tile and X k-tile into stage i % NST
        for (int i = issued; i < nk; ++i) {
            const int s = i % NST;
            if (!mbar_wait(&empty[s], ((i / NST) - 1) & 1)) { s_fail = 1; break; }
            uint8_t * dst = q8_smem + s * sbytes;
            mbar_expect_tx(&full[s], (unsigned) sbytes);
            bulk_g2s(dst, wsrc + (size_t) i * wtile, (unsigned) wtile, &full[s]);
            bulk_g2s(dst + wtile, xsrc + (size_t) i * xtile, (unsigned) xtile, &full[s]);
            issued = i + 1;
        }
    } else if (tid == Q8_MMA_WARP * 32) {
        // MMA issuer: block j of k-tile i into TMEM columns (i % NBUF) * 4 np + j np
        const uint32_t idesc = q8_idesc(g.np);
        for (int i = 0; i < nk; ++i) {
            const int s = i % NST, bf = i % NBUF;
            if (i >= NBUF && !mbar_wait(&acce[bf], ((i / NBUF) - 1) & 1)) { s_fail = 1; break; }
            if (!mbar_wait(&full[s], (i / NST) & 1)) { s_fail = 1; break; }
            tc_fence_after();
            const uint32_t a0 = smem_u32(q8_smem + s * sbytes), b0 = a0 + (uint32_t) wtile;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                q8_mma(tmem + (uint32_t)((bf * 4 + j) * g.np), tc_smem_desc(a0 + j * 256), tc_smem_desc(b0 + j * 256),
                       idesc);
            tc_commit(&empty[s]);
            tc_commit(&accf[bf]);
        }
    } else if (warp < Q8_EPI_WARPS) {
        // epilogue warps: block dots of k-tile i -> acc, in block order
        const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
        const __half * wsrow = g.ws + q8_s_off(tn * TC_BM + r_tile, k0 * 4, g.cols);   // [k-tile][128][4] F16
        uint2 wsn = __ldg(reinterpret_cast<const uint2 *>(wsrow));
        for (int i = 0; i < nk; ++i) {
            const int bf = i % NBUF;
            const uint2 wsc = wsn;
            if (i + 1 < nk) wsn = __ldg(reinterpret_cast<const uint2 *>(wsrow + (size_t)(i + 1) * TC_BM * 4));
            bool got = true;
            if (lane == 0) got = mbar_wait(&accf[bf], (i / NBUF) & 1);
            got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
            if (!got) { ok = false; break; }
            tc_fence_after();
            const __half2 d01 = *reinterpret_cast<const __half2 *>(&wsc.x), d23 = *reinterpret_cast<const __half2 *>(&wsc.y);
            const float dw[4] = {__low2float(d01), __high2float(d01), __low2float(d23), __high2float(d23)};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int b = (k0 + i) * 4 + j;
#pragma unroll
                for (int c = 0; c < NA / 16; ++c) {
                    const int col0 = (2 * c + hh) * 16;
                    if (col0 < g.np) {   // warp-uniform
                        int v[16];
                        q8_ld16(trow + (uint32_t)((bf * 4 + j) * g.np + col0), v);
#pragma unroll
                        for (int t = 0; t < 16; ++t)
                            acc[c * 16 + t] = __fadd_rn(acc[c * 16 + t],
                                                        __fmul_rn((float) v[t], __fmul_rn(dw[j], xsc[(col0 + t) * nb + b])));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&acce[bf]);
        }
    }
    const int bad = __syncthreads_or(!ok || s_fail);
    if (bad && tid == 0) atomicExch(g.err, 1);
    const bool epi = warp < Q8_EPI_WARPS;
    if (S > 1) {
        // k-split: the thread of TMEM row r pushes its partial columns into slot [rank] of
        // the row's owner; after the cluster barrier each owner sums its slots in rank order
        const bool swg = g.epi == TC_EPI_SWIGLU;
        const int pc4 = (pc + 3) & ~3, ps = pc4 + 4;
        const int rs = (swg ? TC_BM / 2 : TC_BM) / S;
        const int orows = swg ? 2 * rs : rs;
        if (!bad && epi) {
            const int gr = swg ? (r_tile & (TC_BM / 2 - 1)) : r_tile;
            const int owner = gr / rs;
            const int orow = (gr % rs) + (swg && r_tile >= TC_BM / 2 ? rs : 0);
            const uint32_t dst = smem_u32(P + ((size_t) rank * orows + orow) * ps);
            uint32_t rdst;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(dst), "r"((uint32_t) owner));
#pragma unroll
            for (int c = 0; c < NA / 16; ++c) {
                const int col0 = (2 * c + hh) * 16;
#pragma unroll
                for (int t = 0; t < 16; t += 4)
                    if (col0 + t < pc4)
                        asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(rdst + (uint32_t)(col0 + t) * 4),
                                     "f"(acc[c * 16 + t]), "f"(acc[c * 16 + t + 1]), "f"(acc[c * 16 + t + 2]),
                                     "f"(acc[c * 16 + t + 3])
                                     : "memory");
            }
        }
        cluster_sync_all();
        if (!bad) {
            const int nq = pc4 / 4;
            for (int idx = tid; idx < rs * nq; idx += Q8_THREADS) {
                const int rl = idx % rs, m0 = (idx / rs) * 4;
                const int rt = rank * rs + rl;
                float a4s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, u4s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int q = 0; q < S; ++q) {
                    const float4 a4 = *reinterpret_cast<const float4 *>(P + ((size_t) q * orows + rl) * ps + m0);
                    a4s[0] = __fadd_rn(a4s[0], a4.x); a4s[1] = __fadd_rn(a4s[1], a4.y);
                    a4s[2] = __fadd_rn(a4s[2], a4.z); a4s[3] = __fadd_rn(a4s[3], a4.w);
                    if (swg) {
                        const float4 u4 = *reinterpret_cast<const float4 *>(P + ((size_t) q * orows + rs + rl) * ps + m0);
                        u4s[0] = __fadd_rn(u4s[0], u4.x); u4s[1] = __fadd_rn(u4s[1], u4.y);
                        u4s[2] = __fadd_rn(u4s[2], u4.z); u4s[3] = __fadd_rn(u4s[3], u4.w);
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = m0 + j;
                    if (m >= pc) break;
                    if (swg) {
                        g.y[(size_t) m * g.ldy + tn * (TC_BM / 2) + rt] = __fmul_rn(silu(a4s[j]), u4s[j]);
                    } else {
                        const int row = tn * TC_BM + rt;
                        float o = a4s[j];
                        if (g.epi == TC_EPI_RESID) o = __fadd_rn(o, g.resid[(size_t) m * g.ldr + row]);
                        g.y[(size_t) m * g.ldy + row] = o;
                    }
                }
            }
        }
    } else if (!bad && epi) {
        if (g.epi == TC_EPI_SWIGLU) {
            // quarters 0-1 hold gate rows, 2-3 the matching up rows; one 16-column chunk per half at a time
#pragma unroll
            for (int c = 0; c < NA / 16; ++c) {
                const int col0 = (2 * c + hh) * 16;
                if (q4 >= 2)
#pragma unroll
                    for (int t = 0; t < 16; ++t) s_swg[hh][r_tile - TC_BM / 2][t] = acc[c * 16 + t];
                asm volatile("bar.sync 1, %0;" ::"r"(Q8_EPI_WARPS * 32) : "memory");
                if (q4 < 2) {
                    const int col = tn * (TC_BM / 2) + r_tile;
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int m = col0 + t;
                        if (m < pc) g.y[(size_t) m * g.ldy + col] = __fmul_rn(silu(acc[c * 16 + t]), s_swg[hh][r_tile][t]);
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"r"(Q8_EPI_WARPS * 32) : "memory");
            }
        } else {
            const int row = tn * TC_BM + r_tile;
#pragma unroll
            for (int c = 0; c < NA / 16; ++c) {
                const int col0 = (2 * c + hh) * 16;
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const int m = col0 + t;
                    if (m >= pc) continue;
                    float o = acc[c * 16 + t];
                    if (g.epi == TC_EPI_RESID) o = __fadd_rn(o, g.resid[(size_t) m * g.ldr + row]);
                    g.y[(size_t) m * g.ldy + row] = o;
                }
            }
        }
    }
    // after a timeout: wait (bounded) for the copies still in flight, then free TMEM
    if (tid == Q8_PRODUCER && bad)
        for (int j = issued > NST ? issued - NST : 0; j < issued; ++j) mbar_wait(&full[j % NST], (j / NST) & 1);
    tc_fence_before();
    __syncthreads();
    if (warp == Q8_MMA_WARP) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
}

// k-split: the smallest power of two giving >= 128 CTAs (at most n_sm CTAs, one
// per SM), at most 8 (clusters of 16 CTAs at one CTA per SM are not all
// resident at once on B200) and at most the k-tiles, while the ring and the
// partial slots fit.
inline int q8_choose_split(const GemmQ8Args & g, int n_sm = 148) {
    const int tiles = g.rows_w / TC_BM, nk = g.cols / Q8_BK;
    int S = 1;
    while (tiles * S < 128 && tiles * S * 2 <= n_sm && S < 8 && S * 2 <= nk &&
           q8_stages(g.np, g.cols, q8_partial_bytes(g.np, g.m_real, S * 2)) >= 2)
        S *= 2;
    return S;
}

inline cudaError_t q8_launch(const GemmQ8Args & g, cudaStream_t stream) {
    const int S = g.ksplit > 1 ? g.ksplit : 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((g.rows_w / TC_BM) * S));
    cfg.blockDim = dim3(Q8_THREADS);
    cfg.dynamicSmemBytes = q8_smem_bytes(g.np, g.cols, q8_partial_bytes(g.np, g.m_real, g.ksplit));
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned) S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (g.np <= 32) return cudaLaunchKernelEx(&cfg, k_gemm_q8<32>, g);
    if (g.np <= 64) return cudaLaunchKernelEx(&cfg, k_gemm_q8<64>, g);
    return cudaLaunchKernelEx(&cfg, k_gemm_q8<128>, g);
}

inline cudaError_t q8_set_attributes() {
    for (auto fn : {(const void *) k_gemm_q8<32>, (const void *) k_gemm_q8<64>, (const void *) k_gemm_q8<128>}) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace qtts
