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

namespace qtts {

constexpr int TC_BM = 128;          // weight rows per tile (MMA M)
constexpr int TC_BK = 64;           // k per tile (four K=16 MMAs)
constexpr int TC_STAGES = 4;
constexpr int TC_THREADS = 128;
constexpr int TC_MAX_N = 256;       // activation rows (MMA N) per launch

// Byte offset of element (row r, column k) inside a tile of `rows` x 64.
__host__ __device__ inline size_t tc_tile_off(int r, int k) {
    return (size_t)(r >> 3) * 1024 + (size_t)((k & 63) >> 3) * 128 + (size_t)(r & 7) * 16 + (size_t)(k & 7) * 2;
}

// Tiled weight matrix: tile (tn, tk) of W[rows][cols] at ((tn * (cols/64)) + tk) * 16 KB.
__host__ __device__ inline size_t tc_w_off(int r, int k, int cols) {
    return ((size_t)(r / TC_BM) * (cols / TC_BK) + (size_t)(k / TC_BK)) * (TC_BM * TC_BK * 2) + tc_tile_off(r % TC_BM, k);
}

// Tiled activation rows: k-tile tk of X[np][cols] at tk * np * 128 bytes.
__host__ __device__ inline size_t tc_x_off(int m, int k, int np) {
    return (size_t)(k / TC_BK) * np * 128 + tc_tile_off(m, k);
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
__host__ __device__ inline size_t tc_smem_bytes(int np) { return TC_STAGES * tc_stage_bytes(np) + 1024; }

// One CTA per 128-row weight tile, full K.
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(GemmTcArgs g) {
    extern __shared__ __align__(128) uint8_t tc_smem[];
    __shared__ __align__(8) uint64_t full[TC_STAGES], empty[TC_STAGES], done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ float s_swg[TC_BM / 2][33];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tn = blockIdx.x;
    const int nk = g.cols / TC_BK;
    const size_t wtile = (size_t) TC_BM * TC_BK * 2, xtile = (size_t) g.np * 128;
    const size_t sbytes = wtile + xtile;
    int ncols = 32;
    while (ncols < g.np) ncols <<= 1;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (tid == 32) {
        for (int s = 0; s < TC_STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    int issued = 0;
    if (tid == 0) {
        // producer: W tile (tn, k) and X k-tile into stage k % STAGES
        const uint8_t * wsrc = g.w + (size_t) tn * nk * wtile;
        for (int i = 0; i < nk; ++i) {
            const int s = i % TC_STAGES;
            if (i >= TC_STAGES && !mbar_wait(&empty[s], ((i / TC_STAGES) - 1) & 1)) { s_fail = 1; break; }
            uint8_t * dst = tc_smem + s * sbytes;
            mbar_expect_tx(&full[s], (unsigned) sbytes);
            bulk_g2s(dst, wsrc + (size_t) i * wtile, (unsigned) wtile, &full[s]);
            bulk_g2s(dst + wtile, g.x + (size_t) i * xtile, (unsigned) xtile, &full[s]);
            issued = i + 1;
        }
    } else if (tid == 32) {
        // MMA issuer
        const uint32_t idesc = tc_idesc(g.np);
        int i = 0;
        for (; i < nk; ++i) {
            const int s = i % TC_STAGES;
            if (!mbar_wait(&full[s], (i / TC_STAGES) & 1)) { s_fail = 1; break; }
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
    if (bad) {
        if (tid == 0) atomicExch(g.err, 1);
    } else {
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
        for (int j = issued > TC_STAGES ? issued - TC_STAGES : 0; j < issued; ++j)
            mbar_wait(&full[j % TC_STAGES], (j / TC_STAGES) & 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
}

}  // namespace qtts
