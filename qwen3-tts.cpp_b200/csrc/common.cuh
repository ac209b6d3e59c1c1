// common.cuh — device helpers shared by the frame-loop kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QTTS_HD 128          // head_dim: fixed for the Qwen3 talker and code predictor
#define QTTS_MAX_CB 16       // codebooks per frame
#define QTTS_WARPS 16        // warps per GEMV CTA
#define QTTS_MAX_NV 8        // activation rows per weight pass

namespace qtts {

enum WType : int { W_F32 = 0, W_F16 = 1, W_Q8_0 = 8 };

// ggml layout matrix: rows x cols, row-major (ne0 = cols contiguous).
// Trivially constructible (it is copied into shared memory); zero-initialise with {}.
struct DMat {
    int type;
    int rows, cols;
    const void * w;        // F16 [rows][cols] or int8 quants [rows][cols]
    const __half * d;      // Q8_0 block scales [rows][cols/32]
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide double sum; `red` is >= 32 doubles of shared memory.  All threads
// receive the total.
__device__ __forceinline__ double block_sum_d(double v, double * red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = lane < nw ? red[lane] : 0.0;
    t = warp_sum_d(t);
    return t;
}
__device__ __forceinline__ float block_max(float v, float * red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : -INFINITY;
    return warp_max(t);
}

// Streaming 16-byte load that bypasses L1 (weights are read once per pass).
__device__ __forceinline__ uint4 ld_stream(const void * p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// 8 F16 weights (one uint4) dotted with 8 F32 activations, F32 accumulate
// (each product of an F16 weight with an F16-representable activation is exact).
__device__ __forceinline__ float dot8(const uint4 & w, const float * x, float acc) {
    const __half2 * h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float2 f = __half22float2(h[k]);
        acc = fmaf(f.x, x[2 * k], acc);
        acc = fmaf(f.y, x[2 * k + 1], acc);
    }
    return acc;
}

// e^x by Cody-Waite range reduction and a Taylor polynomial: x = n ln2 + r with
// n = rint(x log2 e), ln2 split into a 16-bit head (n * head is exact) and a
// tail, |r| <= ln2/2; e^r = sum_{k<=7} r^k / k! by Horner (truncation error
// ~5e-9 relative, below half a float ulp); the result is P(r) * 2^n, scaled in
// two steps near the ends of the range so subnormal results round once.
// Every operation is an explicitly rounded IEEE operation, so the CPU oracle's
// restatement of the same method gives the same bits.  Accuracy: within 2 ulp
// of e^x (checked against float64 in the tests).
__device__ __forceinline__ float qtts_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412701138295233249664306640625e-04f;       // 1/7!
    p = __fmaf_rn(p, r, 1.38888892251998186111450195312500e-03f);   // 1/6!
    p = __fmaf_rn(p, r, 8.33333376795053482055664062500000e-03f);   // 1/5!
    p = __fmaf_rn(p, r, 4.16666679084300994873046875000000e-02f);   // 1/4!
    p = __fmaf_rn(p, r, 1.66666671633720397949218750000000e-01f);   // 1/3!
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int) n;
    if (ni > 127) { p = __fmul_rn(p, 2.0f); ni -= 1; }
    if (ni < -126) { p = __fmul_rn(p, 5.42101086242752217003726400434970855712890625e-20f); ni += 64; }   // 2^-64
    return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// SiLU as ggml's scalar definition: x / (1 + exp(-x)).
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, qtts_expf(-x))); }

// Philox4x32-10 (Salmon et al., SC'11).  Same function as the CPU oracle.
__device__ __forceinline__ void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
        const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
}
__device__ __forceinline__ double uniform01(uint64_t seed, uint32_t frame, uint32_t cb) {
    uint32_t c[4] = {frame, cb, 0x51a3u, 0u};
    philox(c, (uint32_t) seed, (uint32_t)(seed >> 32));
    const uint64_t bits = ((uint64_t) c[0] << 32) | c[1];
    return (double)(bits >> 11) * (1.0 / 9007199254740992.0);
}

// Order-preserving map float -> uint32 (ascending float = ascending key).
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

constexpr int TC_BM = 128;          // tcgen05 GEMM: weight rows per tile (MMA M)
constexpr int TC_BK = 64;           // k per tile (four K=16 MMAs)

// Byte offset of element (row r, column k) inside a tile of `rows` x 64.
__host__ __device__ inline size_t tc_tile_off(int r, int k) {
    return (size_t)(r >> 3) * 1024 + (size_t)((k & 63) >> 3) * 128 + (size_t)(r & 7) * 16 + (size_t)(k & 7) * 2;
}

// Tiled activation rows: k-tile tk of X[np][cols] at tk * np * 128 bytes.
__host__ __device__ inline size_t tc_x_off(int m, int k, int np) {
    return (size_t)(k / TC_BK) * np * 128 + tc_tile_off(m, k);
}

// One F32 activation as F16 hi + lo in the tiled layout (rows m and np/2 + m).
__device__ __forceinline__ void tc_store_split(uint8_t * xt, int m, int k, int np, float v) {
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    *reinterpret_cast<__half *>(xt + tc_x_off(m, k, np)) = hi;
    *reinterpret_cast<__half *>(xt + tc_x_off(np / 2 + m, k, np)) = lo;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while its predecessor runs; pdl_wait() returns once
// the predecessor grid has completed and its writes are visible (a no-op for a
// normal launch), pdl_trigger() lets the successor start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

constexpr unsigned long long QTTS_SPIN_LIMIT = 1ull << 22;   // polls before a bounded wait gives up

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
    for (unsigned long long it = 0; it < QTTS_SPIN_LIMIT; ++it)
        if (mbar_try_wait(m, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, unsigned bytes, uint64_t * m) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(m)) : "memory");
}

}  // namespace qtts
