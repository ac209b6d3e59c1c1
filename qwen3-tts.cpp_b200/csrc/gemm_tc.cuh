// gemm_tc.cuh — tcgen05 (5th-generation tensor core) GEMM for the batched and
// prefill paths: Y[m][n] = sum_k W[n][k] * X[m][k] with F16 operands, F32
// accumulation in tensor memory (TMEM), and the frame loop's epilogues.
//
// The weight matrix is the MMA's A operand (M = 128 weight rows per tile) and
// the activation rows are the B operand (N = padded row count, 16..256), so a
// small batch still fills the 128-row MMA.  Both operands live in HBM in the
// canonical no-swizzle K-major core-matrix layout that tcgen05.mma reads from
// shared memory: a tile of R rows x 64 k is R/8 groups of 1024 bytes, each group
// eight 128-byte core matrices (8 rows x 8 k, 16 bytes per row) in k order.
// A tile is therefore one contiguous block, copied into shared memory by a
// single 1-D cp.async.bulk (no tensor map, no swizzle); the matrix descriptor
// strides are LBO = 128 B (next core matrix along k) and SBO = 1024 B (next
// 8-row group).
//
// Roles (128 threads): thread 0 streams W and X tiles through a STAGES-deep
// shared-memory ring (mbarriers full/empty), thread 32 issues the MMAs
// (4 x K=16 per 64-k tile) and commits each stage back to the producer, and all
// four warps drain the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32w..32w+31 = weight rows) into the epilogue.  Every wait is bounded.
#pragma once
#include "common.cuh"
#include <utility>

namespace qtts {

constexpr int TC_MAX_STAGES = 8;   // shared-memory ring depth (as many as fit in ~200 KB)
constexpr int TC_THREADS = 128;
constexpr int TC_MAX_N = 256;       // activation rows (MMA N) per launch

// Tiled weight matrix: tile (tn, tk) of W[rows][cols] at ((tn * (cols/64)) + tk) * 16 KB.
__host__ __device__ inline size_t tc_w_off(int r, int k, int cols) {
    return ((size_t)(r / TC_BM) * (cols / TC_BK) + (size_t)(k / TC_BK)) * (TC_BM * TC_BK * 2) + tc_tile_off(r % TC_BM, k);
}

// Repack row-major F16 W[rows][cols] into tiles (rows % 128 == 0, cols % 64 == 0).
// `interleave` > 0 builds the gate/up pair for the SwiGLU epilogue: tile tn
// holds rows [64 tn, 64 tn + 64) of W (gate) in tile rows 0..63 and the same rows
// of W2 (up) in tile rows 64..127.
__global__ void k_tile_weights(const __half * W, const __half * W2, int rows, int cols, uint8_t * out) {
    const int r = blockIdx.x;                      // destination row
    int src_r = r;
    const __half * src = W;
    if (W2) {
        const int tn = r / TC_BM, rr = r % TC_BM;
        src_r = tn * (TC_BM / 2) + (rr & (TC_BM / 2 - 1));
        src = rr < TC_BM / 2 ? W : W2;
    }
    for (int k8 = threadIdx.x; k8 < cols / 8; k8 += blockDim.x) {
        const uint4 v = *reinterpret_cast<const uint4 *>(src + (size_t) src_r * cols + k8 * 8);
        *reinterpret_cast<uint4 *>(out + tc_w_off(r, k8 * 8, cols)) = v;
    }
    (void) rows;
}

enum TcAct : int { TC_ACT_F16 = 0, TC_ACT_SPLIT = 1 };

// Activation rows -> F16 tiles.  Optional RMSNorm (double sum over the row, as
// the GEMV path), then round to F16 (TC_ACT_F16), or split x = hi + lo with
// hi = f16(x), lo = f16(x - hi) into rows m and np/2 + m (TC_ACT_SPLIT: the
// F32-activation products of ffn_down to ~22 bits).  Rows >= m_real are zero.
// One CTA per (padded) row.
struct PackArgs {
    const float * x;
    int ldx;
    int m_real, np, cols;
    const float * gain;        // nullptr: no norm
    float eps;
    int act;
    uint8_t * out;             // tiled [cols/64][np][64] F16
    float * xn_out;            // optional: normalised rows (F32) [m_real][ldxn]
    int ldxn;
};

__global__ void __launch_bounds__(256) k_pack_act(PackArgs a) {
    __shared__ double red[8];
    __shared__ float s_scale;
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;                         // packed row (for TC_ACT_SPLIT: m < np/2)
    const int tid = threadIdx.x;
    const bool real = m < a.m_real;
    const float * row = a.x + (size_t) m * a.ldx;
    float scale = 1.0f;
    if (a.gain && real) {
        double ss = 0.0;
        for (int c = tid; c < a.cols; c += blockDim.x) { const float t = row[c]; ss += (double) __fmul_rn(t, t); }
        ss = warp_sum_d(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid == 0) {
            double t = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
            s_scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float)(t / (double) a.cols), a.eps)));
        }
        __syncthreads();
        scale = s_scale;
    }
    const int half = a.np / 2;
    for (int k8 = tid; k8 < a.cols / 8; k8 += blockDim.x) {
        __align__(16) __half hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float t = real ? row[k8 * 8 + e] : 0.0f;
            if (a.gain && real) t = __fmul_rn(__fmul_rn(t, scale), a.gain[k8 * 8 + e]);
            if (a.xn_out && real) a.xn_out[(size_t) m * a.ldxn + k8 * 8 + e] = t;
            hi[e] = __float2half_rn(t);
            lo[e] = __float2half_rn(__fsub_rn(t, __half2float(hi[e])));
        }
        *reinterpret_cast<uint4 *>(a.out + tc_x_off(m, k8 * 8, a.np)) = *reinterpret_cast<const uint4 *>(hi);
        if (a.act == TC_ACT_SPLIT)
            *reinterpret_cast<uint4 *>(a.out + tc_x_off(half + m, k8 * 8, a.np)) = *reinterpret_cast<const uint4 *>(lo);
    }
}

enum TcEpi : int { TC_EPI_STORE = 0, TC_EPI_RESID = 1, TC_EPI_SWIGLU = 2 };

struct GemmTcArgs {
    const uint8_t * w;        // tiled weights, rows_w x cols
    const uint8_t * x;        // tiled activations, np x cols
    int rows_w, cols, np;     // np: MMA N (multiple of 16, <= 256)
    int m_real;               // rows of Y written
    int split;                // TC_ACT_SPLIT input: Y = D[:, m] + D[:, np/2 + m]
    int epi;
    float * y;                // [m_real][ldy]; SwiGLU: column r of the pair tile (rows_w / 2 columns)
    int ldy;
    const float * resid;      // EPI_RESID (may alias y)
    int ldr;
    int * err;                // set on a wait timeout
    uint8_t * xt_out;         // SwiGLU: also write h as F16 hi/lo tiles (rows m, xt_np/2 + m) for the down GEMM
    int xt_np;
    int ksplit;               // CTAs per weight tile along k (a cluster of that size; 1 = no split)
};

__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t) 1 << 46);
}
// kind::f16, F32 accumulator, F16 A and B, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t tc_idesc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void tc_commit(uint64_t * m) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(m))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld16_nowait(uint32_t taddr, float * v) {
    uint32_t * r = reinterpret_cast<uint32_t *>(v);
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__host__ __device__ inline size_t tc_stage_bytes(int np) { return (size_t) TC_BM * TC_BK * 2 + (size_t) np * 128; }
// Split-K partial slots [128][ps] (F32) placed after the ring: ps = columns
// kept (m_real, at most the MMA columns of one half for hi/lo inputs) rounded to
// 4, plus 4 so that 16-byte lanes at a row stride hit distinct banks.
__host__ __device__ inline size_t tc_partial_bytes(int np, int split, int m_real, int ksplit) {
    if (ksplit <= 1) return 0;
    const int mcols = split ? np / 2 : np;
    const int pc = m_real < mcols ? m_real : mcols;
    return (size_t) TC_BM * (((pc + 3) & ~3) + 4) * 4;
}
__host__ __device__ inline int tc_stages(int np, size_t pbytes) {
    const int n = (int)((200 * 1024 - pbytes) / tc_stage_bytes(np));
    return n > TC_MAX_STAGES ? TC_MAX_STAGES : (n < 2 ? 2 : n);
}
__host__ __device__ inline size_t tc_smem_bytes(int np, size_t pbytes = 0) {
    return tc_stages(np, pbytes) * tc_stage_bytes(np) + pbytes + 1024;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One CTA per (128-row weight tile, k slice).  With ksplit S > 1 the S CTAs
// of a tile form a thread-block cluster: each accumulates its k slice in TMEM
// and pushes each partial row into the shared memory of the CTA that owns the
// row (distributed shared memory stores); after a cluster barrier CTA r sums
// its rows [r*128/S, (r+1)*128/S) over the S slots in rank order
// (deterministic) and runs the epilogue.
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(GemmTcArgs g) {
    extern __shared__ __align__(128) uint8_t tc_smem[];
    __shared__ __align__(8) uint64_t full[TC_MAX_STAGES], empty[TC_MAX_STAGES], done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ float s_swg[TC_BM / 2][33];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = g.ksplit > 1 ? g.ksplit : 1;
    const int tn = blockIdx.x / S, rank = blockIdx.x % S;
    const int nk_all = g.cols / TC_BK;
    const int k0 = rank * nk_all / S, nk = (rank + 1) * nk_all / S - k0;
    const size_t wtile = (size_t) TC_BM * TC_BK * 2, xtile = (size_t) g.np * 128;
    const size_t sbytes = wtile + xtile;
    const size_t pbytes = tc_partial_bytes(g.np, g.split, g.m_real, g.ksplit);
    const int NST = tc_stages(g.np, pbytes);
    int ncols = 32;
    while (ncols < g.np) ncols <<= 1;

    // thread 0: barriers, then the first NST copies at once (they overlap the TMEM allocation)
    int issued = 0;
    const uint8_t * wsrc = g.w + ((size_t) tn * nk_all + k0) * wtile;
    const uint8_t * xsrc = g.x + (size_t) k0 * xtile;
    pdl_trigger();
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
        // weight tiles are read-only: their copies start before the predecessor finishes
        for (int i = 0; i < nk && i < NST; ++i) {
            mbar_expect_tx(&full[i], (unsigned) sbytes);
            bulk_g2s(tc_smem + i * sbytes, wsrc + (size_t) i * wtile, (unsigned) wtile, &full[i]);
            issued = i + 1;
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_wait();   // activations, residuals and outputs follow the predecessor in stream order
    if (tid == 0)
        for (int i = 0; i < issued; ++i)
            bulk_g2s(tc_smem + i * sbytes + wtile, xsrc + (size_t) i * xtile, (unsigned) xtile, &full[i]);

    if (tid == 0) {
        // producer: W tile (tn, k) and X k-tile into stage k % NST
        for (int i = issued; i < nk; ++i) {
            const int s = i % NST;
            if (!mbar_wait(&empty[s], ((i / NST) - 1) & 1)) { s_fail = 1; break; }
            uint8_t * dst = tc_smem + s * sbytes;
            mbar_expect_tx(&full[s], (unsigned) sbytes);
            bulk_g2s(dst, wsrc + (size_t) i * wtile, (unsigned) wtile, &full[s]);
            bulk_g2s(dst + wtile, xsrc + (size_t) i * xtile, (unsigned) xtile, &full[s]);
            issued = i + 1;
        }
    } else if (tid == 32) {
        // MMA issuer
        const uint32_t idesc = tc_idesc(g.np);
        int i = 0;
        for (; i < nk; ++i) {
            const int s = i % NST;
            if (!mbar_wait(&full[s], (i / NST) & 1)) { s_fail = 1; break; }
            tc_fence_after();
            const uint32_t a0 = smem_u32(tc_smem + s * sbytes), b0 = a0 + (uint32_t) wtile;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk)
                tc_mma(tmem, tc_smem_desc(a0 + kk * 256), tc_smem_desc(b0 + kk * 256), idesc, (i | kk) != 0);
            tc_commit(&empty[s]);
        }
        tc_commit(&done);   // arrives once every MMA issued above has completed
    }
    // epilogue: wait for the accumulator
    bool ok = true;
    if (tid == 0) ok = mbar_wait(&done, 0);
    const int bad = __syncthreads_or(!ok || s_fail);
    tc_fence_after();
    if (bad && tid == 0) atomicExch(g.err, 1);
    if (S > 1) {
        // Every CTA of the cluster reaches both cluster barriers (a failed one skips
        // the work only).  Push: the thread holding TMEM row r stores its partial
        // into slot [my rank] of the row's owner (CTA r / rs) with remote 16-byte
        // stores; after the barrier each owner sums its S slots in rank order.
        const bool swg = g.epi == TC_EPI_SWIGLU;
        const int mcols = g.split ? g.np / 2 : g.np;
        const int pc = g.m_real < mcols ? g.m_real : mcols;     // partial columns kept
        const int pc4 = (pc + 3) & ~3;
        const int ps = pc4 + 4;                                      // row stride: 16-byte lanes hit distinct banks
        const int rs = (swg ? TC_BM / 2 : TC_BM) / S;                // rows (gate rows for SwiGLU) owned per CTA
        const int orows = swg ? 2 * rs : rs;                         // rows held per slot (gate + up for SwiGLU)
        float * P = reinterpret_cast<float *>(tc_smem + NST * sbytes);   // [S][orows][ps], after the ring
        if (!bad) {
            const int r_tile = warp * 32 + lane;
            const int gr = swg ? (r_tile & (TC_BM / 2 - 1)) : r_tile;  // gate-row index for SwiGLU
            const int owner = gr / rs;
            const int orow = (gr % rs) + (swg && r_tile >= TC_BM / 2 ? rs : 0);
            const uint32_t dst = smem_u32(P + ((size_t) rank * orows + orow) * ps);
            uint32_t rdst;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(dst), "r"((uint32_t) owner));
            const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
            const int grp = g.split ? 32 : 64;                       // columns per TMEM wait
            for (int c0 = 0; c0 < pc; c0 += grp) {
                float v[64];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int cc = g.split ? (q >> 1) * 16 + (q & 1) * (g.np / 2) : q * 16;
                    const bool want = g.split ? (q < 2 || c0 + 16 < pc) : (c0 + q * 16 < pc);   // warp-uniform
                    if (want) tc_ld16_nowait(trow + (uint32_t)(c0 + cc), v + 16 * q);
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (g.split) {   // v[0..15] + v[16..31] = hi + lo of columns c0..c0+15, v[32..] the next 16
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        v[j] = __fadd_rn(v[j], v[16 + j]);
                        v[16 + j] = __fadd_rn(v[32 + j], v[48 + j]);
                    }
                }
#pragma unroll
                for (int j = 0; j < 64; j += 4)
                    if (j < grp && c0 + j < pc4)
                        asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(rdst + (uint32_t)(c0 + j) * 4),
                                     "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]), "f"(v[j + 3])
                                     : "memory");
            }
        }
        cluster_sync_all();
        if (!bad) {
            // this CTA owns rows [rank*rs, (rank+1)*rs): a thread takes 4 consecutive columns of one row
            const int nq = pc4 / 4;
            for (int idx = tid; idx < rs * nq; idx += TC_THREADS) {
                const int rl = idx % rs, m0 = (idx / rs) * 4;
                const int rt = rank * rs + rl;
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, up[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int q = 0; q < S; ++q) {
                    const float4 a4 = *reinterpret_cast<const float4 *>(P + ((size_t) q * orows + rl) * ps + m0);
                    acc[0] = __fadd_rn(acc[0], a4.x); acc[1] = __fadd_rn(acc[1], a4.y);
                    acc[2] = __fadd_rn(acc[2], a4.z); acc[3] = __fadd_rn(acc[3], a4.w);
                    if (swg) {
                        const float4 u4 = *reinterpret_cast<const float4 *>(P + ((size_t) q * orows + rs + rl) * ps + m0);
                        up[0] = __fadd_rn(up[0], u4.x); up[1] = __fadd_rn(up[1], u4.y);
                        up[2] = __fadd_rn(up[2], u4.z); up[3] = __fadd_rn(up[3], u4.w);
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = m0 + j;
                    if (m >= pc) break;
                    if (swg) {
                        const float h = __fmul_rn(silu(acc[j]), up[j]);
                        g.y[(size_t) m * g.ldy + tn * (TC_BM / 2) + rt] = h;
                        if (g.xt_out) tc_store_split(g.xt_out, m, tn * (TC_BM / 2) + rt, g.xt_np, h);
                    } else {
                        const int row = tn * TC_BM + rt;
                        float o = acc[j];
                        if (g.epi == TC_EPI_RESID) o = __fadd_rn(o, g.resid[(size_t) m * g.ldr + row]);
                        g.y[(size_t) m * g.ldy + row] = o;
                    }
                }
            }
        }
        // (no second cluster barrier: after the first one no CTA touches a peer's memory)
    } else if (!bad) {
        const int r_tile = warp * 32 + lane;                    // TMEM lane = weight row in the tile
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        const int mcols = g.split ? g.np / 2 : g.np;
        for (int c0 = 0; c0 < mcols && c0 < g.m_real; c0 += 16) {
            float v[16];
            tc_ld16(trow + (uint32_t) c0, v);
            if (g.split) {
                float w2[16];
                tc_ld16(trow + (uint32_t)(g.np / 2 + c0), w2);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], w2[j]);
            }
            if (g.epi == TC_EPI_SWIGLU) {
                // warps 0-1 hold gate rows, warps 2-3 the matching up rows
                __syncwarp();
                if (warp >= 2)
                    for (int j = 0; j < 16; ++j) s_swg[r_tile - TC_BM / 2][j] = v[j];
                __syncthreads();
                if (warp < 2) {
                    const int col = tn * (TC_BM / 2) + r_tile;
                    for (int j = 0; j < 16; ++j) {
                        const int m = c0 + j;
                        if (m >= g.m_real) break;
                        const float h = __fmul_rn(silu(v[j]), s_swg[r_tile][j]);
                        g.y[(size_t) m * g.ldy + col] = h;
                        if (g.xt_out) tc_store_split(g.xt_out, m, col, g.xt_np, h);
                    }
                }
                __syncthreads();
            } else {
                const int row = tn * TC_BM + r_tile;
                for (int j = 0; j < 16; ++j) {
                    const int m = c0 + j;
                    if (m >= g.m_real) break;
                    float o = v[j];
                    if (g.epi == TC_EPI_RESID) o = __fadd_rn(o, g.resid[(size_t) m * g.ldr + row]);
                    g.y[(size_t) m * g.ldy + row] = o;
                }
            }
        }
    }
    // after a timeout: wait (bounded) for the copies still in flight, then free TMEM
    if (tid == 0 && bad)
        for (int j = issued > NST ? issued - NST : 0; j < issued; ++j)
            mbar_wait(&full[j % NST], (j / NST) & 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
}

// k-split of a GEMM: the smallest power of two giving >= 64 CTAs, at most 8
// (the portable cluster size), at most the 64-k tiles, and only while the ring
// plus the partial slots fit the 201 KB of dynamic shared memory.
inline int tc_choose_split(const GemmTcArgs & g) {
    const int tiles = g.rows_w / TC_BM, nk = g.cols / TC_BK;
    int S = 1;
    while (tiles * S < 64 && S < 8 && S * 2 <= nk &&
           tc_smem_bytes(g.np, tc_partial_bytes(g.np, g.split, g.m_real, S * 2)) <= 201 * 1024)
        S *= 2;
    return S;
}

// Launch k_gemm_tc with g.ksplit CTAs per weight tile as a cluster.
inline cudaError_t tc_launch(const GemmTcArgs & g, cudaStream_t stream) {
    const int S = g.ksplit > 1 ? g.ksplit : 1;
    const size_t smem = tc_smem_bytes(g.np, tc_partial_bytes(g.np, g.split, g.m_real, g.ksplit));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((g.rows_w / TC_BM) * S));
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
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
    return cudaLaunchKernelEx(&cfg, k_gemm_tc, g);
}

// Launch any kernel with programmatic stream serialization (see pdl_wait).
template <class... KArgs, class... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args &&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qtts
