// oracle.cpp — CPU restatement of the qwen3-tts.cpp TTSTransformer decode path.
//
// TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 engine:
// only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
// legs load it.  The product never links it.
//
// PARITY STATUS: unpinned against ggml.  The reference does all arithmetic in
// the ggml submodule, which is empty and unpinned in the reference tree, and the
// reference's PyTorch goldens (reference/det_*.bin) are absent.  This file
// restates, op for op, the graphs of src/tts_transformer.cpp with ggml-CPU's
// canonical (scalar) dtype semantics:
//   * F16-weight mul_mat: activation rounded to F16 (RNE), products exact, F32
//     accumulation.  ffn_down with F16 weights is cast to F32 first
//     (src/tts_transformer.cpp:1746-1748), so its activation is NOT rounded.
//   * Q8_0-weight mul_mat: activation quantised per 32-block exactly as
//     quantize_row_q8_0_ref (d = amax/127, id = 1/d, q = roundf(x*id), d stored
//     as F16), int32 dot per block, sum += isum * (d_w * d_a) in F32.
//   * rms_norm: sum of squares in double, scale = 1/sqrtf(mean + eps).
//   * softmax: max, exp(x - max), sum in double, y = e * (float)(1/sum).
//   * exp (softmax, SiLU): Cody-Waite reduction + degree-7 Taylor polynomial
//     (qexpf), the method the engine uses, so both give the same bits.
//   * Summation orders: by default every reduction (GEMV rows, RMSNorm sums,
//     attention scores, softmax sums, P x V) runs in the engine's order (see
//     g_eng), so engine and oracle agree before each F16 rounding and Q8_0
//     quantisation; ggml's own order depends on its SIMD path.  Code-predictor
//     steps (one row, at most 16 keys) follow the engine's one-warp-per-head
//     attention (forward_stack's cp_step branch).
//   * RoPE NEOX: theta_i = pos * s^i by repeated F32 multiplication,
//     s = powf(base, -2/n_dims) (ggml_rope_cache_init).
//   * KV caches F16; talker prefill/step and code-predictor steps read K/V from
//     the F16 cache (Q and probabilities rounded to F16 for the dots); the
//     code-predictor 2-token prefill attends over its F32 Kcur/Vcur
//     (src/tts_transformer.cpp:2000-2011).
// Pins that do exist: the Q8_0 block format and quantiser are checked against
// gguf-py 0.19.0 (the package the reference converter imports), the GGUF reader
// against gguf-py's reader, and the decoder-layer maths against an independent
// fp32 PyTorch restatement (tests/test_oracle_cpu.py).
//
// Sampling follows src/tts_transformer.cpp:2750-2788 (code predictor) and
// :3108-3184 (codebook 0).  The reference draws from std::mt19937 seeded by
// std::random_device (src/tts_transformer.h:403), which no caller can seed;
// here (as in the engine) the draw is inverse-CDF with a Philox4x32-10 uniform
// keyed by (seed) and countered by (frame, codebook).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_set>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <immintrin.h>
#include <omp.h>

namespace orc {

// ---------------------------------------------------------------- F16 helpers
static inline float h2f(uint16_t h) { return _cvtsh_ss(h); }
static inline uint16_t f2h(float f) { return _cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT); }
static inline float round_f16(float f) { return h2f(f2h(f)); }

// ---------------------------------------------------------------- GGUF reader
enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8 };

struct Tensor {
    std::string name;
    int type = -1;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const uint8_t * data = nullptr;
    size_t nbytes = 0;
};

struct GGUF {
    uint8_t * map = nullptr;
    size_t size = 0;
    std::map<std::string, uint64_t> u;   // integer-valued keys
    std::map<std::string, double> f;     // float-valued keys
    std::map<std::string, Tensor> tensors;
    std::string err;
    ~GGUF() { if (map) munmap(map, size); }

    bool open(const char * path) {
        int fd = ::open(path, O_RDONLY);
        if (fd < 0) { err = std::string("cannot open ") + path; return false; }
        struct stat st; fstat(fd, &st); size = (size_t) st.st_size;
        map = (uint8_t *) mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (map == MAP_FAILED) { map = nullptr; err = "mmap failed"; return false; }
        size_t p = 0;
        auto rd = [&](void * dst, size_t n) -> bool {
            if (p + n > size) return false;
            memcpy(dst, map + p, n); p += n; return true;
        };
        auto rstr = [&](std::string & s) -> bool {
            uint64_t n; if (!rd(&n, 8) || p + n > size) return false;
            s.assign((const char *) map + p, n); p += n; return true;
        };
        uint32_t magic, version; uint64_t nt, nkv;
        if (!rd(&magic, 4) || magic != 0x46554747u) { err = "bad magic"; return false; }
        if (!rd(&version, 4) || version < 2) { err = "unsupported version"; return false; }
        if (!rd(&nt, 8) || !rd(&nkv, 8)) { err = "truncated header"; return false; }
        static const int tsize[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        for (uint64_t i = 0; i < nkv; ++i) {
            std::string key; uint32_t ty;
            if (!rstr(key) || !rd(&ty, 4)) { err = "truncated kv"; return false; }
            if (ty == 8) { std::string s; if (!rstr(s)) return false; continue; }
            if (ty == 9) {
                uint32_t at; uint64_t n; if (!rd(&at, 4) || !rd(&n, 8)) return false;
                for (uint64_t k = 0; k < n; ++k) {
                    if (at == 8) { std::string s; if (!rstr(s)) return false; }
                    else if (at < 13 && tsize[at]) p += tsize[at];
                    else { err = "nested array"; return false; }
                }
                continue;
            }
            if (ty >= 13 || !tsize[ty]) { err = "bad kv type"; return false; }
            uint8_t buf[8] = {0}; if (!rd(buf, tsize[ty])) return false;
            switch (ty) {
                case 0: u[key] = buf[0]; break;
                case 1: u[key] = (uint64_t)(int64_t)(int8_t) buf[0]; break;
                case 2: { uint16_t v; memcpy(&v, buf, 2); u[key] = v; } break;
                case 3: { int16_t v; memcpy(&v, buf, 2); u[key] = (uint64_t)(int64_t) v; } break;
                case 4: { uint32_t v; memcpy(&v, buf, 4); u[key] = v; } break;
                case 5: { int32_t v; memcpy(&v, buf, 4); u[key] = (uint64_t)(int64_t) v; } break;
                case 6: { float v; memcpy(&v, buf, 4); f[key] = v; } break;
                case 7: u[key] = buf[0]; break;
                case 10: case 11: { uint64_t v; memcpy(&v, buf, 8); u[key] = v; } break;
                case 12: { double v; memcpy(&v, buf, 8); f[key] = v; } break;
            }
        }
        struct Info { std::string name; uint32_t nd; uint64_t ne[4]; uint32_t type; uint64_t off; };
        std::vector<Info> infos(nt);
        for (auto & ti : infos) {
            if (!rstr(ti.name) || !rd(&ti.nd, 4) || ti.nd > 4) { err = "bad tensor info"; return false; }
            for (uint32_t d = 0; d < 4; ++d) ti.ne[d] = 1;
            for (uint32_t d = 0; d < ti.nd; ++d) if (!rd(&ti.ne[d], 8)) return false;
            if (!rd(&ti.type, 4) || !rd(&ti.off, 8)) return false;
        }
        uint64_t align = u.count("general.alignment") ? u["general.alignment"] : 32;
        size_t data_off = (p + align - 1) / align * align;
        for (auto & ti : infos) {
            Tensor t; t.name = ti.name; t.type = (int) ti.type; t.n_dims = (int) ti.nd;
            int64_t n = 1;
            for (int d = 0; d < 4; ++d) { t.ne[d] = (int64_t) ti.ne[d]; n *= t.ne[d]; }
            if (t.type == T_F32) t.nbytes = n * 4;
            else if (t.type == T_F16) t.nbytes = n * 2;
            else if (t.type == T_Q8_0) t.nbytes = n / 32 * 34;
            else t.nbytes = 0;  // unsupported types are loadable only if unused
            t.data = map + data_off + ti.off;
            if (data_off + ti.off + t.nbytes > size) { err = "tensor out of file: " + t.name; return false; }
            tensors[t.name] = t;
        }
        return true;
    }
    int64_t geti(std::initializer_list<const char *> keys, int64_t dflt) const {
        for (auto k : keys) { auto it = u.find(k); if (it != u.end()) return (int64_t) it->second; }
        return dflt;
    }
    double getf(std::initializer_list<const char *> keys, double dflt) const {
        for (auto k : keys) { auto it = f.find(k); if (it != f.end()) return it->second; }
        return dflt;
    }
};

// ---------------------------------------------------------------- model
struct Config {  // src/tts_transformer.h:59-103, parse_config :228-377
    int text_vocab = 151936, text_dim = 2048, hidden = 1024, n_layers = 28, n_heads = 16,
        n_kv = 8, ffn = 3072, head_dim = 128;
    float eps = 1e-6f, theta = 1e6f;
    int codec_vocab = 3072, n_cb = 16, cp_layers = 5, cp_vocab = 2048, cp_hidden = 1024,
        cp_ffn = 3072;
    float cp_theta = 1e4f;
    int codec_pad = 2148, codec_bos = 2149, codec_eos = 2150, tts_bos = 151672,
        tts_eos = 151673, tts_pad = 151671, think = 2154, nothink = 2155, think_bos = 2156,
        think_eos = 2157, english = 2050;
};

struct Layer {
    const Tensor *attn_norm, *q, *k, *v, *o, *q_norm, *k_norm, *ffn_norm, *gate, *up, *down;
};

struct KV {
    int n_ctx = 0, n_layers = 0, n_kv = 0, D = 0;
    std::vector<uint16_t> k, v;  // [layer][pos][kvh][D] F16
    void init(int layers, int ctx, int nkv, int d) {
        n_layers = layers; n_ctx = ctx; n_kv = nkv; D = d;
        k.assign((size_t) layers * ctx * nkv * d, 0);
        v.assign((size_t) layers * ctx * nkv * d, 0);
    }
    uint16_t * K(int l, int pos) { return k.data() + (((size_t) l * n_ctx + pos) * n_kv) * D; }
    uint16_t * V(int l, int pos) { return v.data() + (((size_t) l * n_ctx + pos) * n_kv) * D; }
};

struct Model {
    GGUF g;
    Config c;
    const Tensor *text_embd, *fc1, *fc1_b, *fc2, *fc2_b, *codec_embd, *out_norm, *codec_head,
        *cp_out_norm;
    std::vector<Layer> L, CPL;
    std::vector<const Tensor *> cp_embd, cp_head;
    KV cache, cp_cache;
    std::vector<float> last_hidden;
    std::string err;
};

static const Tensor * need(Model & m, const std::string & name) {
    auto it = m.g.tensors.find(name);
    if (it == m.g.tensors.end()) { m.err = "missing tensor " + name; return nullptr; }
    return &it->second;
}

// ---------------------------------------------------------------- engine-order arithmetic
// The engine's reductions run in a fixed order (lanes, butterflies, thread
// strides).  With g_eng set (the default) the oracle performs every reduction
// in that same order, so engine and oracle agree bit for bit before every
// rounding and quantisation step (the Q8_0 activation quantiser turns a last-bit
// difference into a whole int8 level).  With g_eng clear it uses plain
// sequential / AVX2 orders (faster; the CPU baseline timing uses it).  Either
// order is a valid restatement of the reference's F32 accumulations, whose
// own order depends on ggml's SIMD path.
static bool g_eng = true;

// e^x by Cody-Waite reduction and a degree-7 Taylor polynomial: the method the
// engine's qtts_expf uses, with the same explicitly rounded operations.
static inline float qexpf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541015625f) return 0.0f;
    const float n = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412701138295233249664306640625e-04f;
    p = fmaf(p, r, 1.38888892251998186111450195312500e-03f);
    p = fmaf(p, r, 8.33333376795053482055664062500000e-03f);
    p = fmaf(p, r, 4.16666679084300994873046875000000e-02f);
    p = fmaf(p, r, 1.66666671633720397949218750000000e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int) n;
    if (ni > 127) { p = p * 2.0f; ni -= 1; }
    if (ni < -126) { p = p * 5.42101086242752217003726400434970855712890625e-20f; ni += 64; }
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float sc;
    memcpy(&sc, &bits, 4);
    return p * sc;
}

// Lane 0's value after the xor butterfly 16, 8, 4, 2, 1 over 32 lanes.
static inline float bfly0(const float * v) {
    float a[32];
    memcpy(a, v, sizeof(a));
    for (int o = 16; o > 0; o >>= 1) {
        float b[32];
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}
// Every lane's value after the same butterfly on doubles.
static inline void bfly_all_d(double * a) {
    for (int o = 16; o > 0; o >>= 1) {
        double b[32];
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
        memcpy(a, b, sizeof(b));
    }
}

// RMSNorm scale of a GEMV prologue (512 threads): thread t sums the squares at
// planar positions t, t+512, ... (the two-plane activation layout: position p
// holds column ((q >> 2) << 3) + 4 [p >= cols/2] + (q & 3), q = p mod cols/2),
// lane 0 of each warp keeps its butterfly sum, the 16 warp sums add in order.
static float gemv_norm_scale(const float * x, int cols, float eps) {
    const int half = cols / 2;
    double warp_sum[16];
    for (int w = 0; w < 16; ++w) {
        double lanes[32];
        for (int l = 0; l < 32; ++l) {
            double ss = 0.0;
            for (int p = w * 32 + l; p < cols; p += 512) {
                const int q = p >= half ? p - half : p;
                const int c = ((q >> 2) << 3) + (p >= half ? 4 : 0) + (q & 3);
                ss += (double)(x[c] * x[c]);
            }
            lanes[l] = ss;
        }
        bfly_all_d(lanes);
        warp_sum[w] = lanes[0];
    }
    double ss = 0.0;
    for (int w = 0; w < 16; ++w) ss += warp_sum[w];
    const float mean = (float)(ss / (double) cols);
    return 1.0f / sqrtf(mean + eps);
}

// GEMV row dot in the engine's order: lane l chains 8-column chunks l, l+32, ...
// (eight fused multiply-adds per chunk, in column order), then the butterfly.
static inline float dot_f16_eng(const uint16_t * w, const float * x, int cols) {
    float lanes[32];
    const int nch = cols / 8;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int c = l; c < nch; c += 32)
            for (int e = 0; e < 8; ++e) acc = fmaf(h2f(w[8 * c + e]), x[8 * c + e], acc);
        lanes[l] = acc;
    }
    return bfly0(lanes);
}
// Q8_0 row dot in the engine's order: lane 2j adds the 32-blocks j, j+16, ...
// (isum * (d_w * d_a) each), odd lanes hold 0, then the butterfly.
static inline float dot_q8_eng(const uint8_t * row, const int8_t * qa, const uint16_t * da, int nb) {
    float lanes[32] = {0.0f};
    for (int j = 0; j < 16; ++j) {
        float acc = 0.0f;
        for (int b = j; b < nb; b += 16) {
            uint16_t dw;
            memcpy(&dw, row + b * 34, 2);
            const int8_t * qw = (const int8_t *)(row + b * 34 + 2);
            int32_t isum = 0;
            for (int k = 0; k < 32; ++k) isum += (int32_t) qw[k] * (int32_t) qa[b * 32 + k];
            acc = acc + (float) isum * (h2f(dw) * h2f(da[b]));
        }
        lanes[2 * j] = acc;
    }
    return bfly0(lanes);
}

// Per-head RMSNorm of q / k as the engine's warp does it: lane l squares its 4
// dims (double, in order), the butterfly gives each lane its own sum, and each
// lane scales its dims with its own scale.
static void head_norm_eng(float * x, int D, float eps, const float * gain) {
    double ss[32];
    for (int l = 0; l < 32; ++l) {
        double t = 0.0;
        for (int k = 0; k < 4; ++k) t += (double)(x[l * 4 + k] * x[l * 4 + k]);
        ss[l] = t;
    }
    bfly_all_d(ss);
    for (int l = 0; l < 32; ++l) {
        const float mean = (float)(ss[l] / (double) D);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int k = 0; k < 4; ++k) {
            const float t = x[l * 4 + k] * scale;
            x[l * 4 + k] = gain ? t * gain[l * 4 + k] : t;
        }
    }
}

// QK score of one key in the engine's order: lanes of an 8-lane group chain 16
// dims each, combined ((s0+s4)+(s2+s6)) + ((s1+s5)+(s3+s7)).
static inline float score_eng(const float * k, const float * q) {
    float s[8];
    for (int g = 0; g < 8; ++g) {
        float a = 0.0f;
        for (int d = 0; d < 16; ++d) a = fmaf(k[g * 16 + d], q[g * 16 + d], a);
        s[g] = a;
    }
    return ((s[0] + s[4]) + (s[2] + s[6])) + ((s[1] + s[5]) + (s[3] + s[7]));
}

// ---------------------------------------------------------------- kernels
// y[r] = W[r,:] . x  for a weight matrix with ne0 = cols (input), ne1 = rows.
// mode: 0 = ggml F16 semantics (x rounded to F16); 1 = weight cast to F32 (x
// unrounded); Q8_0 weights quantise x per block.
struct QBlocks { std::vector<int8_t> q; std::vector<uint16_t> d; };

static void quantize_q8_0(const float * x, int n, QBlocks & out) {
    // quantize_row_q8_0_ref semantics (also gguf-py Q8_0.quantize_blocks).
    int nb = n / 32;
    out.q.resize(n); out.d.resize(nb);
    for (int b = 0; b < nb; ++b) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[b * 32 + j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        out.d[b] = f2h(d);
        for (int j = 0; j < 32; ++j) out.q[b * 32 + j] = (int8_t) roundf(x[b * 32 + j] * id);
    }
}

static inline float dot_f16_f32acc(const uint16_t * w, const float * xh, int n) {
    // products of F16 values are exact in F32; accumulate in F32.
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        __m256 w0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(w + i)));
        __m256 w1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(w + i + 8)));
        acc0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(xh + i), acc0);
        acc1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(xh + i + 8), acc1);
    }
    acc0 = _mm256_add_ps(acc0, acc1);
    alignas(32) float t[8]; _mm256_store_ps(t, acc0);
    float s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    for (; i < n; ++i) s += h2f(w[i]) * xh[i];
    return s;
}

static void mul_mat(const Tensor * W, const float * x, int n_vec, float * y, bool f32_cast = false) {
    const int cols = (int) W->ne[0], rows = (int) W->ne[1];
    if (W->type == T_F32) {
        const float * w = (const float *) W->data;
        #pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; ++r)
            for (int v = 0; v < n_vec; ++v) {
                float s = 0.0f;
                for (int c = 0; c < cols; ++c) s += w[(size_t) r * cols + c] * x[(size_t) v * cols + c];
                y[(size_t) v * rows + r] = s;
            }
        return;
    }
    if (W->type == T_F16) {
        std::vector<float> xh((size_t) n_vec * cols);
        for (size_t i = 0; i < xh.size(); ++i) xh[i] = f32_cast ? x[i] : round_f16(x[i]);
        const uint16_t * w = (const uint16_t *) W->data;
        #pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; ++r)
            for (int v = 0; v < n_vec; ++v)
                y[(size_t) v * rows + r] = g_eng ? dot_f16_eng(w + (size_t) r * cols, xh.data() + (size_t) v * cols, cols)
                                                 : dot_f16_f32acc(w + (size_t) r * cols, xh.data() + (size_t) v * cols, cols);
        return;
    }
    if (W->type == T_Q8_0) {
        const int nb = cols / 32;
        std::vector<QBlocks> qx(n_vec);
        for (int v = 0; v < n_vec; ++v) quantize_q8_0(x + (size_t) v * cols, cols, qx[v]);
        const uint8_t * w = W->data;
        #pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; ++r) {
            const uint8_t * row = w + (size_t) r * nb * 34;
            for (int v = 0; v < n_vec; ++v) {
                if (g_eng) {
                    y[(size_t) v * rows + r] = dot_q8_eng(row, qx[v].q.data(), qx[v].d.data(), nb);
                    continue;
                }
                float s = 0.0f;
                for (int b = 0; b < nb; ++b) {
                    uint16_t dw; memcpy(&dw, row + b * 34, 2);
                    const int8_t * qw = (const int8_t *)(row + b * 34 + 2);
                    const int8_t * qa = qx[v].q.data() + b * 32;
                    int32_t isum = 0;
                    for (int j = 0; j < 32; ++j) isum += (int32_t) qw[j] * (int32_t) qa[j];
                    s += (float) isum * (h2f(dw) * h2f(qx[v].d[b]));
                }
                y[(size_t) v * rows + r] = s;
            }
        }
        return;
    }
}

// ---- the engine's fused frame path (two clustered kernels per layer), restated
// for the frame loop of orc_generate when split mode is on (engine order only).
static bool g_split = false;      // orc_set_frame_split
static bool g_in_frame = false;   // inside orc_generate's frame loop

// FFN block shape: R intermediate rows per CTA (a Q8_0 32-block), N CTAs, and
// clusters of C CTAs (the largest power of two <= 16 dividing N and H).
static void ffn_split(int I, int H, bool q8, int & R, int & N, int & C) {
    R = q8 ? 32 : 16;
    N = I / R;
    C = 16;
    while (C > 1 && (N % C || H % C)) C /= 2;
}

// O-projection by kv group: partial g is the GEMV over the group's gc columns
// (lane order of dot_f16_eng / dot_q8_eng over that slice); out = ((P_0 + P_1)
// + ...) + P_{ng-1}.
static void mul_mat_o_split(const Tensor * W, const float * x, int n_vec, float * y, int gc) {
    const int cols = (int) W->ne[0], rows = (int) W->ne[1], ng = cols / gc;
    if (W->type == T_F16) {
        std::vector<float> xh((size_t) n_vec * cols);
        for (size_t i = 0; i < xh.size(); ++i) xh[i] = round_f16(x[i]);
        const uint16_t * w = (const uint16_t *) W->data;
        #pragma omp parallel for schedule(static)
        for (int r = 0; r < rows; ++r)
            for (int v = 0; v < n_vec; ++v) {
                float acc = 0.0f;
                for (int g = 0; g < ng; ++g) {
                    const float pg = dot_f16_eng(w + (size_t) r * cols + g * gc, xh.data() + (size_t) v * cols + g * gc, gc);
                    acc = g == 0 ? pg : acc + pg;
                }
                y[(size_t) v * rows + r] = acc;
            }
        return;
    }
    const int nb = cols / 32, nbg = gc / 32;
    std::vector<QBlocks> qx(n_vec);
    for (int v = 0; v < n_vec; ++v) quantize_q8_0(x + (size_t) v * cols, cols, qx[v]);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int v = 0; v < n_vec; ++v) {
            const uint8_t * row = W->data + (size_t) r * nb * 34;
            float acc = 0.0f;
            for (int g = 0; g < ng; ++g) {
                const float pg = dot_q8_eng(row + (size_t) g * nbg * 34, qx[v].q.data() + g * gc, qx[v].d.data() + g * nbg, nbg);
                acc = g == 0 ? pg : acc + pg;
            }
            y[(size_t) v * rows + r] = acc;
        }
}

// ffn_down by intermediate slice (F16 weight cast to F32, F32 activation; Q8_0
// quantises the activation per 32-block): CTA s of the FFN block owns rows
// [s R, s R + R) of h; its partial of output r chains fmaf(W[r][j], h[j], acc)
// over j in order (Q8_0: the block's isum x (d_w x d_a)); a cluster adds its
// CTAs' partials in rank order, the output adds the clusters' in order.
static void mul_mat_down_split(const Tensor * W, const float * h, int n_vec, float * y) {
    const int I = (int) W->ne[0], H = (int) W->ne[1];
    const bool q8 = W->type == T_Q8_0;
    int R, N, C;
    ffn_split(I, H, q8, R, N, C);
    std::vector<QBlocks> qx(q8 ? n_vec : 0);
    for (int v = 0; q8 && v < n_vec; ++v) quantize_q8_0(h + (size_t) v * I, I, qx[v]);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < H; ++r)
        for (int v = 0; v < n_vec; ++v) {
            float out = 0.0f;
            for (int cl = 0; cl < N / C; ++cl) {
                float q = 0.0f;
                for (int p = 0; p < C; ++p) {
                    const int sl = cl * C + p;
                    float d;
                    if (q8) {
                        const uint8_t * blk = W->data + ((size_t) r * (I / 32) + sl) * 34;
                        uint16_t dw; memcpy(&dw, blk, 2);
                        const int8_t * qw = (const int8_t *)(blk + 2);
                        int32_t isum = 0;
                        for (int k = 0; k < 32; ++k) isum += (int32_t) qw[k] * (int32_t) qx[v].q[(size_t) sl * 32 + k];
                        d = (float) isum * (h2f(dw) * h2f(qx[v].d[sl]));
                    } else {
                        const uint16_t * w = (const uint16_t *) W->data + (size_t) r * I;
                        d = 0.0f;
                        for (int j = sl * R; j < sl * R + R; ++j) d = fmaf(h2f(w[j]), h[(size_t) v * I + j], d);
                    }
                    q = p == 0 ? d : q + d;
                }
                out = cl == 0 ? q : out + q;
            }
            y[(size_t) v * H + r] = out;
        }
}

static void rms_norm(const float * x, int n, float eps, const float * gain, float * y) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) { float t = x[i] * scale; y[i] = gain ? t * gain[i] : t; }
}

static const float * f32p(const Tensor * t) { return (const float *) t->data; }

// RMSNorm of a GEMV input (attn_norm, ffn_norm, output norms): the engine
// computes it in the GEMV prologue, with gemv_norm_scale's summation order.
static void rms_norm_in(const float * x, int n, float eps, const float * gain, float * y) {
    if (!g_eng) { rms_norm(x, n, eps, gain, y); return; }
    const float scale = gemv_norm_scale(x, n, eps);
    for (int i = 0; i < n; ++i) { const float t = x[i] * scale; y[i] = gain ? t * gain[i] : t; }
}

// ggml_rope_cache_init with ext_factor 0, freq_scale 1, attn_factor 1.
static void rope_cache(int pos, int n_dims, float base, float * cs /*[n_dims] cos,sin pairs*/) {
    const float theta_scale = powf(base, -2.0f / (float) n_dims);
    float theta = (float) pos;
    for (int i0 = 0; i0 < n_dims; i0 += 2) {
        cs[i0 + 0] = cosf(theta);
        cs[i0 + 1] = sinf(theta);
        theta *= theta_scale;
    }
}

static void rope_neox(float * x, int D, const float * cs) {
    const int half = D / 2;
    for (int ic = 0; ic < half; ++ic) {
        const float c = cs[2 * ic], s = cs[2 * ic + 1];
        const float x0 = x[ic], x1 = x[ic + half];
        x[ic] = x0 * c - x1 * s;
        x[ic + half] = x0 * s + x1 * c;
    }
}

static inline float silu(float x) { return x / (1.0f + qexpf(-x)); }

// One decoder stack over M token rows X[M][H] at positions n_past..n_past+M-1.
// kv_from_cache: attention reads F16 K/V from the cache (talker graphs and the
// code-predictor step graph); otherwise attends over F32 Kcur/Vcur of this call
// (code-predictor 2-token prefill).
// Attention dump (set_attn_dump / write_attn_dump, src/tts_transformer.cpp:2978-3005
// and the attn_rows capture in build_step_graph): the post-softmax row of one
// talker layer per decode step, [row][n_heads][stride], before the F16
// rounding that feeds P x V.  Filled by talker steps (orc_forward_step) only.
static float * g_attn_buf = nullptr;
static int g_attn_cap = 0, g_attn_stride = 0, g_attn_layer = -1, g_attn_rows = 0;
static bool g_talker_step = false;

static void attn_dump_row(int il, int h, int NH, const float * p, int n) {
    if (!g_attn_buf || !g_talker_step || il != g_attn_layer || g_attn_rows >= g_attn_cap) return;
    float * row = g_attn_buf + ((size_t) g_attn_rows * NH + h) * g_attn_stride;
    for (int j = 0; j < n && j < g_attn_stride; ++j) row[j] = p[j];
}

static void forward_stack(Model & m, std::vector<Layer> & layers, KV & cache, float theta,
                          std::vector<float> & X, int M, int n_past, bool kv_from_cache,
                          int ffn, bool cp_step = false) {
    const Config & c = m.c;
    const int H = c.hidden, D = c.head_dim, NH = c.n_heads, NKV = c.n_kv;
    const int QD = NH * D, KD = NKV * D;
    const float kq_scale = 1.0f / sqrtf((float) D);
    std::vector<float> xn((size_t) M * H), q((size_t) M * QD), k((size_t) M * KD), v((size_t) M * KD),
        att((size_t) M * QD), o((size_t) M * H), gt((size_t) M * ffn), up((size_t) M * ffn),
        hh((size_t) M * ffn), dn((size_t) M * H);
    std::vector<float> cs((size_t) M * D);
    for (int i = 0; i < M; ++i) rope_cache(n_past + i, D, theta, cs.data() + (size_t) i * D);
    const int n_kv_tot = n_past + M;
    for (size_t il = 0; il < layers.size(); ++il) {
        const Layer & ly = layers[il];
        for (int i = 0; i < M; ++i) rms_norm_in(&X[(size_t) i * H], H, c.eps, f32p(ly.attn_norm), &xn[(size_t) i * H]);
        mul_mat(ly.q, xn.data(), M, q.data());
        mul_mat(ly.k, xn.data(), M, k.data());
        mul_mat(ly.v, xn.data(), M, v.data());
        for (int i = 0; i < M; ++i) {
            for (int h = 0; h < NH; ++h) {
                float * qh = &q[(size_t) i * QD + h * D];
                if (g_eng) head_norm_eng(qh, D, c.eps, ly.q_norm ? f32p(ly.q_norm) : nullptr);
                else rms_norm(qh, D, c.eps, ly.q_norm ? f32p(ly.q_norm) : nullptr, qh);
                rope_neox(qh, D, &cs[(size_t) i * D]);
            }
            for (int h = 0; h < NKV; ++h) {
                float * kh = &k[(size_t) i * KD + h * D];
                if (g_eng) head_norm_eng(kh, D, c.eps, ly.k_norm ? f32p(ly.k_norm) : nullptr);
                else rms_norm(kh, D, c.eps, ly.k_norm ? f32p(ly.k_norm) : nullptr, kh);
                rope_neox(kh, D, &cs[(size_t) i * D]);
            }
            uint16_t * kc = cache.K((int) il, n_past + i);
            uint16_t * vc = cache.V((int) il, n_past + i);
            for (int t = 0; t < KD; ++t) { kc[t] = f2h(k[(size_t) i * KD + t]); vc[t] = f2h(v[(size_t) i * KD + t]); }
        }
        // attention
        #pragma omp parallel for collapse(2) schedule(static)
        for (int i = 0; i < M; ++i)
            for (int h = 0; h < NH; ++h) {
                const int g = h / (NH / NKV);
                const int nk = kv_from_cache ? n_kv_tot : M;
                const int base = kv_from_cache ? 0 : n_past;  // row index offset for the mask
                std::vector<float> s(nk), p(nk), qh(D);
                const float * qsrc = &q[(size_t) i * QD + h * D];
                for (int d = 0; d < D; ++d) qh[d] = kv_from_cache ? round_f16(qsrc[d]) : qsrc[d];
                if (g_eng && cp_step) {
                    // the engine's code-predictor step: one warp per query head.  Key j on
                    // lanes 2j, 2j + 1, each chaining 64 dims, the pair adding its halves;
                    // double sum of the even lanes over the butterfly; P x V chains keys per dim.
                    const int nkey = n_past + 1;   // <= 16
                    std::vector<float> kf(D), e(16, 0.0f);
                    float mx = -INFINITY;
                    for (int j = 0; j < nkey; ++j) {
                        const uint16_t * kj = cache.K((int) il, j) + g * D;
                        for (int d = 0; d < D; ++d) kf[d] = h2f(kj[d]);
                        float a0 = 0.0f, a1 = 0.0f;
                        for (int d = 0; d < 64; ++d) a0 = fmaf(kf[d], qh[d], a0);
                        for (int d = 64; d < 128; ++d) a1 = fmaf(kf[d], qh[d], a1);
                        s[j] = (a0 + a1) * kq_scale;
                        mx = std::max(mx, s[j]);
                    }
                    for (int j = 0; j < nkey; ++j) e[j] = qexpf(s[j] - mx);
                    double lane[32];
                    for (int l = 0; l < 32; ++l) lane[l] = (l & 1) ? 0.0 : (double) e[l >> 1];
                    bfly_all_d(lane);
                    const float inv = (float)(1.0 / lane[0]);
                    for (int j = 0; j < nkey; ++j) p[j] = round_f16(e[j] * inv);
                    float * out = &att[(size_t) i * QD + h * D];
                    for (int d = 0; d < D; ++d) {
                        float acc = 0.0f;
                        for (int j = 0; j < nkey; ++j) acc = fmaf(p[j], h2f(cache.V((int) il, j)[g * D + d]), acc);
                        out[d] = acc;
                    }
                    continue;
                }
                if (g_eng) {
                    // the engine's fused unit (frame steps, the code-predictor prefill, one-row
                    // prefill chunks) or its prefill kernel (chunks of 2-8 rows)
                    const int chunk = std::min(8, M - (i / 8) * 8);
                    const bool fused = !kv_from_cache || M == 1 || chunk == 1;
                    const int nkey = kv_from_cache ? n_past + i + 1 : i + 1;
                    std::vector<float> kf(D);
                    for (int j = 0; j < nkey; ++j) {
                        if (kv_from_cache) {
                            const uint16_t * kj = cache.K((int) il, j) + g * D;
                            for (int d = 0; d < D; ++d) kf[d] = h2f(kj[d]);
                            s[j] = score_eng(kf.data(), qh.data()) * kq_scale;
                        } else {
                            s[j] = score_eng(&k[(size_t) j * KD + g * D], qh.data()) * kq_scale;
                        }
                    }
                    float mx = -INFINITY;
                    for (int j = 0; j < nkey; ++j) mx = std::max(mx, s[j]);
                    for (int j = 0; j < nkey; ++j) p[j] = qexpf(s[j] - mx);
                    double lane[32];
                    if (fused) {
                        for (int l = 0; l < 32; ++l) {
                            double t = 0.0;
                            for (int j = l; j < nkey; j += 32) t += (double) p[j];
                            lane[l] = t;
                        }
                        bfly_all_d(lane);
                    } else {
                        double red[32] = {0.0};
                        for (int w = 0; w < 8; ++w) {
                            double tl[32];
                            for (int l = 0; l < 32; ++l) {
                                double t = 0.0;
                                for (int j = w * 32 + l; j < nkey; j += 256) t += (double) p[j];
                                tl[l] = t;
                            }
                            bfly_all_d(tl);
                            red[w] = tl[0];
                        }
                        memcpy(lane, red, sizeof(lane));
                        bfly_all_d(lane);
                    }
                    for (int j = 0; j < nkey; ++j) {
                        const float inv = (float)(1.0 / lane[j & 31]);
                        p[j] = p[j] * inv;
                    }
                    if (M == 1) attn_dump_row((int) il, h, NH, p.data(), nkey);
                    if (kv_from_cache)
                        for (int j = 0; j < nkey; ++j) p[j] = round_f16(p[j]);
                    const int npg = fused ? 8 : 4;
                    float * out = &att[(size_t) i * QD + h * D];
                    for (int d = 0; d < D; ++d) {
                        float part[8];
                        for (int pg = 0; pg < npg; ++pg) {
                            float acc = 0.0f;
                            for (int j = pg; j < nkey; j += npg) {
                                const float vj = kv_from_cache ? h2f(cache.V((int) il, j)[g * D + d]) : v[(size_t) j * KD + g * D + d];
                                acc = fmaf(p[j], vj, acc);
                            }
                            part[pg] = acc;
                        }
                        if (fused) {
                            float t = 0.0f;
                            for (int pg = 0; pg < 8; ++pg) t = t + part[pg];
                            out[d] = t;
                        } else {
                            out[d] = (part[0] + part[1]) + (part[2] + part[3]);
                        }
                    }
                    continue;
                }
                float mx = -INFINITY;
                for (int j = 0; j < nk; ++j) {
                    float dot = 0.0f;
                    if (kv_from_cache) {
                        const uint16_t * kj = cache.K((int) il, j) + g * D;
                        dot = dot_f16_f32acc(kj, qh.data(), D);
                    } else {
                        const float * kj = &k[(size_t) j * KD + g * D];
                        for (int d = 0; d < D; ++d) dot += kj[d] * qh[d];
                    }
                    float sc = dot * kq_scale;
                    if (j + base > n_past + i) sc = -INFINITY;  // ggml_diag_mask_inf(n_past)
                    s[j] = sc;
                    mx = std::max(mx, sc);
                }
                double sum = 0.0;
                for (int j = 0; j < nk; ++j) { float e = qexpf(s[j] - mx); p[j] = e; sum += (double) e; }
                const float inv = (float)(1.0 / sum);
                for (int j = 0; j < nk; ++j) p[j] *= inv;
                if (M == 1) attn_dump_row((int) il, h, NH, p.data(), nk);
                float * out = &att[(size_t) i * QD + h * D];
                for (int d = 0; d < D; ++d) out[d] = 0.0f;
                for (int j = 0; j < nk; ++j) {
                    if (kv_from_cache) {
                        const float pj = round_f16(p[j]);
                        const uint16_t * vj = cache.V((int) il, j) + g * D;
                        for (int d = 0; d < D; ++d) out[d] += pj * h2f(vj[d]);
                    } else {
                        const float * vj = &v[(size_t) j * KD + g * D];
                        for (int d = 0; d < D; ++d) out[d] += p[j] * vj[d];
                    }
                }
            }
        const bool split = g_split && g_eng && g_in_frame;   // the engine's fused frame path
        if (split) mul_mat_o_split(ly.o, att.data(), M, o.data(), (NH / NKV) * D);
        else mul_mat(ly.o, att.data(), M, o.data());
        for (size_t t = 0; t < (size_t) M * H; ++t) X[t] = o[t] + X[t];
        for (int i = 0; i < M; ++i) rms_norm_in(&X[(size_t) i * H], H, c.eps, f32p(ly.ffn_norm), &xn[(size_t) i * H]);
        mul_mat(ly.gate, xn.data(), M, gt.data());
        mul_mat(ly.up, xn.data(), M, up.data());
        for (size_t t = 0; t < (size_t) M * ffn; ++t) hh[t] = silu(gt[t]) * up[t];
        if (split) mul_mat_down_split(ly.down, hh.data(), M, dn.data());
        else mul_mat(ly.down, hh.data(), M, dn.data(), /*f32_cast=*/true);
        for (size_t t = 0; t < (size_t) M * H; ++t) X[t] = dn[t] + X[t];
    }
}

// ---------------------------------------------------------------- Philox4x32-10
// Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3"
// (SC'11): 10 rounds, multipliers 0xD2511F53 / 0xCD9E8D57, key bumps
// 0x9E3779B9 / 0xBB67AE85.
static void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t) 0xD2511F53u * c[0];
        uint64_t p1 = (uint64_t) 0xCD9E8D57u * c[2];
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t) p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t) p1;
        uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
}
// Uniform double in [0,1) for sampling event (frame, codebook).
static double uniform01(uint64_t seed, uint32_t frame, uint32_t cb) {
    uint32_t c[4] = {frame, cb, 0x51a3u, 0u};
    philox(c, (uint32_t) seed, (uint32_t)(seed >> 32));
    uint64_t bits = ((uint64_t) c[0] << 32) | c[1];
    return (double)(bits >> 11) * (1.0 / 9007199254740992.0);
}

// Near-tie measure of a sampled decision on the scale of a greedy top-2 logit
// gap (a greedy pick flips once the logits move by half its gap).  Raw logits
// moved by at most delta move every temperature-scaled logit by delta / T, so
// they shift the inverse-CDF bucket edges by about 2 delta / T and the top-k
// threshold gap (in scaled units) by 2 delta / T: the decision can flip only if
// 2 delta >= T * min(distance of the draw from the nearest edge, threshold gap
// to the best excluded logit).
static double sampled_tie_measure(double edge_gap, double topk_gap, double temperature) {
    return temperature * std::min(edge_gap, topk_gap);
}

static int32_t argmax(const float * d, int n) {  // src/tts_transformer.cpp:2583-2593
    int32_t mi = 0; float mv = d[0];
    for (int i = 1; i < n; ++i) if (d[i] > mv) { mv = d[i]; mi = i; }
    return mi;
}

// temperature-scaled logits in place -> top-k mask -> softmax -> inverse-CDF
// draw.  Returns the token; *cdf_gap receives the distance of the draw from
// the nearest bucket edge (for the near-tie bookkeeping).
static int32_t sample_tok(float * lg, int n, float temperature, int top_k, double u,
                          bool scale_temp, float eos_bias, int eos_id, double * edge_gap,
                          double * topk_gap = nullptr) {
    if (scale_temp) for (int i = 0; i < n; ++i) lg[i] /= temperature;
    if (eos_bias != 0.0f && eos_id >= 0) lg[eos_id] += eos_bias;
    if (topk_gap) *topk_gap = 1e30;
    if (top_k > 0 && top_k < n) {
        std::vector<float> sv(lg, lg + n);
        std::nth_element(sv.begin(), sv.begin() + (top_k - 1), sv.end(), std::greater<float>());
        const float thr = sv[top_k - 1];
        if (topk_gap) {   // distance from the threshold to the best excluded logit
            float below = -INFINITY;
            for (int i = 0; i < n; ++i) if (lg[i] < thr) below = std::max(below, lg[i]);
            *topk_gap = (double) thr - (double) below;
        }
        for (int i = 0; i < n; ++i) if (lg[i] < thr) lg[i] = -INFINITY;
    }
    float mx = *std::max_element(lg, lg + n);
    std::vector<float> p(n);
    double sum = 0.0;
    for (int i = 0; i < n; ++i) { p[i] = qexpf(lg[i] - mx); sum += p[i]; }
    for (int i = 0; i < n; ++i) p[i] = (float)(p[i] / sum);
    double tot = 0.0;
    for (int i = 0; i < n; ++i) tot += (double) p[i];
    const double target = u * tot;
    double cum = 0.0; int pick = -1; double prev = 0.0;
    for (int i = 0; i < n; ++i) {
        prev = cum; cum += (double) p[i];
        if (p[i] > 0.0f && cum > target) { pick = i; break; }
    }
    if (pick < 0) { for (int i = n - 1; i >= 0; --i) if (p[i] > 0.0f) { pick = i; break; } prev = cum; }
    if (edge_gap) *edge_gap = std::min(target - prev, cum - target);
    return pick;
}

}  // namespace orc

using namespace orc;

// ================================================================ C API
extern "C" {

struct orc_gen_args {
    const int32_t * text; int32_t n_text;
    const int32_t * ref_text; int32_t n_ref_text;
    const int32_t * ref_codes; int32_t n_ref_frames;  // ICL when ref_codes != NULL
    const float * speaker;                              // may be NULL
    int32_t max_len; int32_t language_id;
    float rep_penalty; float temperature; int32_t top_k;
    const int32_t * instruct; int32_t n_instruct;
    float eos_bias; int32_t target_frames; int32_t rep_loop_detect;
    uint64_t seed;
    const int32_t * follow; int32_t n_follow;  // engine codes to follow at near-ties
    float tie_tol;
    int32_t * codes_out; int32_t codes_cap;     // capacity in frames
    float * talker_logits_out;                  // [cap][codec_vocab] raw step logits, or NULL
    float * cp_logits_out;                      // [cap][n_cb-1][cp_vocab] raw, or NULL
    float * prefill_out; int32_t prefill_cap;   // prefill rows [cap][H], or NULL
};

struct orc_gen_result {
    int32_t n_frames; int32_t prefill_len; int32_t n_mismatch; int32_t n_ties;
    int32_t first_mismatch; int32_t truncated; float max_tie_gap; float min_decision_gap;
    float max_mismatch_gap;
};

void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
// Attention dump of talker layer `layer` for the following decode steps: row r
// of buf [cap][n_heads][stride] holds step r's post-softmax rows (nullptr: off).
void orc_set_attn_dump(float * buf, int cap, int stride, int layer) {
    g_attn_buf = buf; g_attn_cap = cap; g_attn_stride = stride; g_attn_layer = layer; g_attn_rows = 0;
}
int orc_attn_rows() { return g_attn_rows; }
// 1 (default): every reduction in the engine's order; 0: plain sequential / AVX2 orders.
void orc_set_engine_order(int on) { g_eng = on != 0; }
void orc_set_frame_split(int on) { g_split = on != 0; }
float orc_expf(float x) { return qexpf(x); }
int orc_get_threads() { return omp_get_max_threads(); }

void * orc_load(const char * path, char * err, int errlen) {
    auto m = std::make_unique<Model>();
    auto fail = [&](const std::string & e) -> void * {
        if (err && errlen > 0) snprintf(err, errlen, "%s", e.c_str());
        return nullptr;
    };
    if (!m->g.open(path)) return fail(m->g.err);
    GGUF & g = m->g;
    Config & c = m->c;
    c.text_vocab = (int) g.geti({"qwen3-tts.text.vocab_size", "qwen3-tts.text_vocab_size"}, 151936);
    c.text_dim = (int) g.geti({"qwen3-tts.text.embedding_dim", "qwen3-tts.text_hidden_size"}, 2048);
    c.hidden = (int) g.geti({"qwen3-tts.talker.embedding_length", "qwen3-tts.embedding_length"}, 1024);
    c.n_layers = (int) g.geti({"qwen3-tts.talker.block_count", "qwen3-tts.block_count"}, 28);
    c.n_heads = (int) g.geti({"qwen3-tts.talker.attention.head_count", "qwen3-tts.attention.head_count"}, 16);
    c.n_kv = (int) g.geti({"qwen3-tts.talker.attention.head_count_kv", "qwen3-tts.attention.head_count_kv"}, 8);
    c.ffn = (int) g.geti({"qwen3-tts.talker.feed_forward_length", "qwen3-tts.feed_forward_length"}, 3072);
    c.head_dim = (int) g.geti({"qwen3-tts.talker.attention.key_length", "qwen3-tts.attention.key_length"}, 128);
    c.eps = (float) g.getf({"qwen3-tts.talker.attention.layer_norm_rms_epsilon", "qwen3-tts.attention.layer_norm_rms_epsilon"}, 1e-6);
    c.theta = (float) g.getf({"qwen3-tts.talker.rope.freq_base", "qwen3-tts.rope.freq_base"}, 1e6);
    c.codec_vocab = (int) g.geti({"qwen3-tts.talker.codec_vocab_size", "qwen3-tts.vocab_size"}, 3072);
    c.n_cb = (int) g.geti({"qwen3-tts.talker.num_codebooks", "qwen3-tts.num_code_groups"}, 16);
    c.cp_layers = (int) g.geti({"qwen3-tts.code_pred.layer_count", "qwen3-tts.code_predictor.layer_count"}, 5);
    c.cp_vocab = (int) g.geti({"qwen3-tts.code_pred.vocab_size", "qwen3-tts.code_predictor.vocab_size"}, 2048);
    c.cp_hidden = (int) g.geti({"qwen3-tts.code_pred.embedding_length", "qwen3-tts.code_predictor.embedding_length"}, 1024);
    c.cp_ffn = (int) g.geti({"qwen3-tts.code_pred.feed_forward_length", "qwen3-tts.code_predictor.feed_forward_length"}, 3072);
    c.cp_theta = (float) g.getf({"qwen3-tts.code_pred.rope.freq_base", "qwen3-tts.code_predictor.rope.freq_base"}, c.theta);
    c.codec_pad = (int) g.geti({"qwen3-tts.codec.pad_id"}, 2148);
    c.codec_bos = (int) g.geti({"qwen3-tts.codec.bos_id"}, 2149);
    c.codec_eos = (int) g.geti({"qwen3-tts.codec.eos_id", "qwen3-tts.codec.eos_token_id"}, 2150);
    c.tts_bos = (int) g.geti({"qwen3-tts.tts_bos_token_id", "qwen3-tts.tts.bos_token_id", "qwen3-tts.tts.bos_id"}, 151672);
    c.tts_eos = (int) g.geti({"qwen3-tts.tts_eos_token_id", "qwen3-tts.tts.eos_token_id", "qwen3-tts.tts.eos_id"}, 151673);
    c.tts_pad = (int) g.geti({"qwen3-tts.tts_pad_token_id", "qwen3-tts.tts.pad_token_id", "qwen3-tts.tts.pad_id"}, 151671);
    c.think = (int) g.geti({"qwen3-tts.codec.think_id", "qwen3-tts.codec_think_id"}, 2154);
    c.nothink = (int) g.geti({"qwen3-tts.codec.nothink_id", "qwen3-tts.codec_nothink_id"}, 2155);
    c.think_bos = (int) g.geti({"qwen3-tts.codec.think_bos_id", "qwen3-tts.codec_think_bos_id"}, 2156);
    c.think_eos = (int) g.geti({"qwen3-tts.codec.think_eos_id", "qwen3-tts.codec_think_eos_id"}, 2157);
    c.english = (int) g.geti({"qwen3-tts.language.english_id", "qwen3-tts.codec.language.english_id", "qwen3-tts.language_id"}, 2050);
    if (c.cp_hidden != c.hidden) return fail("code predictor width != talker width (mtp_proj not supported)");

    Model & M = *m;
    if (!(M.text_embd = need(M, "talker.text_embd.weight")) || !(M.fc1 = need(M, "talker.text_proj.fc1.weight")) ||
        !(M.fc1_b = need(M, "talker.text_proj.fc1.bias")) || !(M.fc2 = need(M, "talker.text_proj.fc2.weight")) ||
        !(M.fc2_b = need(M, "talker.text_proj.fc2.bias")) || !(M.codec_embd = need(M, "talker.codec_embd.weight")) ||
        !(M.out_norm = need(M, "talker.output_norm.weight")) || !(M.codec_head = need(M, "talker.codec_head.weight")) ||
        !(M.cp_out_norm = need(M, "code_pred.output_norm.weight")))
        return fail(M.err);
    auto load_layers = [&](const char * pfx, int n, std::vector<Layer> & out) -> bool {
        out.resize(n);
        for (int i = 0; i < n; ++i) {
            std::string p = std::string(pfx) + std::to_string(i) + ".";
            Layer & l = out[i];
            if (!(l.attn_norm = need(M, p + "attn_norm.weight")) || !(l.q = need(M, p + "attn_q.weight")) ||
                !(l.k = need(M, p + "attn_k.weight")) || !(l.v = need(M, p + "attn_v.weight")) ||
                !(l.o = need(M, p + "attn_output.weight")) || !(l.ffn_norm = need(M, p + "ffn_norm.weight")) ||
                !(l.gate = need(M, p + "ffn_gate.weight")) || !(l.up = need(M, p + "ffn_up.weight")) ||
                !(l.down = need(M, p + "ffn_down.weight")))
                return false;
            auto qn = M.g.tensors.find(p + "attn_q_norm.weight");
            auto kn = M.g.tensors.find(p + "attn_k_norm.weight");
            l.q_norm = qn == M.g.tensors.end() ? nullptr : &qn->second;
            l.k_norm = kn == M.g.tensors.end() ? nullptr : &kn->second;
        }
        return true;
    };
    if (!load_layers("talker.blk.", c.n_layers, M.L) || !load_layers("code_pred.blk.", c.cp_layers, M.CPL))
        return fail(M.err);
    M.cp_embd.resize(c.n_cb - 1); M.cp_head.resize(c.n_cb - 1);
    for (int gi = 0; gi < c.n_cb - 1; ++gi) {
        if (!(M.cp_embd[gi] = need(M, "code_pred.codec_embd." + std::to_string(gi) + ".weight")) ||
            !(M.cp_head[gi] = need(M, "code_pred.lm_head." + std::to_string(gi) + ".weight")))
            return fail(M.err);
    }
    return m.release();
}

void orc_free(void * h) { delete (Model *) h; }

// ints: text_vocab text_dim hidden n_layers n_heads n_kv ffn head_dim codec_vocab n_cb
//       cp_layers cp_vocab cp_hidden cp_ffn codec_pad codec_bos codec_eos tts_bos tts_eos
//       tts_pad think nothink think_bos think_eos english ; floats: eps theta cp_theta
int orc_config(void * h, int32_t * iv, float * fv) {
    Config & c = ((Model *) h)->c;
    int32_t a[] = {c.text_vocab, c.text_dim, c.hidden, c.n_layers, c.n_heads, c.n_kv, c.ffn, c.head_dim,
                   c.codec_vocab, c.n_cb, c.cp_layers, c.cp_vocab, c.cp_hidden, c.cp_ffn, c.codec_pad,
                   c.codec_bos, c.codec_eos, c.tts_bos, c.tts_eos, c.tts_pad, c.think, c.nothink,
                   c.think_bos, c.think_eos, c.english};
    memcpy(iv, a, sizeof(a));
    fv[0] = c.eps; fv[1] = c.theta; fv[2] = c.cp_theta;
    return (int)(sizeof(a) / sizeof(a[0]));
}

int orc_init_kv(void * h, int n_ctx) {
    Model & m = *(Model *) h;
    m.cache.init(m.c.n_layers, n_ctx, m.c.n_kv, m.c.head_dim);
    return 0;
}

// F16/F32 embedding row gather (src/tts_transformer.cpp:920-961).
// which: 0 = codec_embd, 1..n_cb-1 = code_pred.codec_embd[which-1], -1 = text_embd.
int orc_lookup_rows(void * h, int which, const int32_t * ids, int n, float * out) {
    Model & m = *(Model *) h;
    const Tensor * t = which == 0 ? m.codec_embd : which < 0 ? m.text_embd : m.cp_embd[which - 1];
    const int dim = (int) t->ne[0], vocab = (int) t->ne[1];
    for (int i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= vocab) return -1;
        const uint16_t * row = (const uint16_t *) t->data + (size_t) ids[i] * dim;
        for (int d = 0; d < dim; ++d) out[(size_t) i * dim + d] = h2f(row[d]);
    }
    return 0;
}

// project_text_tokens (src/tts_transformer.cpp:963-1028).
int orc_project_text(void * h, const int32_t * toks, int n, float * out) {
    Model & m = *(Model *) h;
    const int TD = m.c.text_dim, H = m.c.hidden;
    std::vector<float> e((size_t) n * TD), a((size_t) n * TD);
    if (orc_lookup_rows(h, -1, toks, n, e.data()) != 0) return -1;
    mul_mat(m.fc1, e.data(), n, a.data());
    for (int i = 0; i < n; ++i)
        for (int d = 0; d < TD; ++d) a[(size_t) i * TD + d] = silu(a[(size_t) i * TD + d] + f32p(m.fc1_b)[d]);
    mul_mat(m.fc2, a.data(), n, out);
    for (int i = 0; i < n; ++i)
        for (int d = 0; d < H; ++d) out[(size_t) i * H + d] += f32p(m.fc2_b)[d];
    return 0;
}

// forward_prefill (src/tts_transformer.cpp:2217-2347): hidden_out [n][H] post-norm,
// logits_out [codec_vocab] of the last row (either may be NULL).
int orc_forward_prefill(void * h, const float * embd, int n, int n_past, float * hidden_out, float * logits_out) {
    Model & m = *(Model *) h;
    const int H = m.c.hidden;
    if (m.cache.n_ctx == 0) orc_init_kv(h, std::max(256, n_past + n + 16));
    if (n_past + n > m.cache.n_ctx) return -1;
    std::vector<float> X(embd, embd + (size_t) n * H), hs((size_t) n * H);
    forward_stack(m, m.L, m.cache, m.c.theta, X, n, n_past, true, m.c.ffn);
    for (int i = 0; i < n; ++i) rms_norm_in(&X[(size_t) i * H], H, m.c.eps, f32p(m.out_norm), &hs[(size_t) i * H]);
    if (hidden_out) memcpy(hidden_out, hs.data(), hs.size() * 4);
    m.last_hidden.assign(hs.end() - H, hs.end());
    if (logits_out) mul_mat(m.codec_head, m.last_hidden.data(), 1, logits_out);
    return 0;
}

// forward_step (src/tts_transformer.cpp:2379-2509).
int orc_forward_step(void * h, const float * embd, int n_past, float * logits_out, float * hidden_out) {
    Model & m = *(Model *) h;
    if (m.cache.n_ctx == 0) orc_init_kv(h, std::max(256, n_past + 1 + 16));
    if (n_past + 1 > m.cache.n_ctx) return -1;
    const int H = m.c.hidden;
    std::vector<float> X(embd, embd + H);
    g_talker_step = true;
    forward_stack(m, m.L, m.cache, m.c.theta, X, 1, n_past, true, m.c.ffn);
    g_talker_step = false;
    if (g_attn_buf && g_attn_layer >= 0 && g_attn_layer < (int) m.L.size() && g_attn_rows < g_attn_cap) ++g_attn_rows;
    m.last_hidden.resize(H);
    rms_norm_in(X.data(), H, m.c.eps, f32p(m.out_norm), m.last_hidden.data());
    if (hidden_out) memcpy(hidden_out, m.last_hidden.data(), H * 4);
    if (logits_out) mul_mat(m.codec_head, m.last_hidden.data(), 1, logits_out);
    return 0;
}

// One code-predictor pass: prefill (gen_step 0, two rows) or step gen_step >= 1.
static void cp_pass(Model & m, int gen_step, const float * rows, float * logits) {
    const int H = m.c.hidden;
    const int M = gen_step == 0 ? 2 : 1;
    const int n_past = gen_step == 0 ? 0 : gen_step + 1;
    std::vector<float> X(rows, rows + (size_t) M * H), hn(H);
    forward_stack(m, m.CPL, m.cp_cache, m.c.cp_theta, X, M, n_past, /*kv_from_cache=*/gen_step != 0, m.c.cp_ffn,
                  /*cp_step=*/gen_step != 0);
    rms_norm_in(&X[(size_t)(M - 1) * H], H, m.c.eps, f32p(m.cp_out_norm), hn.data());
    mul_mat(m.cp_head[gen_step], hn.data(), 1, logits);
}

struct Decision { int pick; float gap; };

// predict_codes_autoregressive (src/tts_transformer.cpp:2711-2976) with
// optional following of externally produced codes.
static void predict_codes(Model & m, const float * hidden, int cb0, float temperature, int top_k,
                          uint64_t seed, uint32_t frame, int32_t * out, float * logits_dump,
                          const int32_t * follow, float tie_tol, orc_gen_result * res, int * dec_index) {
    const int H = m.c.hidden, V = m.c.cp_vocab, NG = m.c.n_cb - 1;
    if (m.cp_cache.n_ctx < 16) m.cp_cache.init(m.c.cp_layers, 16, m.c.n_kv, m.c.head_dim);
    std::vector<float> rows(2 * H), lg(V);
    memcpy(rows.data(), hidden, H * 4);
    orc_lookup_rows(&m, 0, &cb0, 1, rows.data() + H);
    for (int g = 0; g < NG; ++g) {
        if (g > 0) {
            int32_t prev = out[g - 1];
            orc_lookup_rows(&m, g, &prev, 1, rows.data());
        }
        cp_pass(m, g, rows.data(), lg.data());
        if (logits_dump) memcpy(logits_dump + (size_t) g * V, lg.data(), V * 4);
        int pick; double gap = 1e30, kgap = 1e30;
        std::vector<float> work(lg);
        if (temperature <= 0.0f) {
            pick = argmax(work.data(), V);
        } else {
            pick = sample_tok(work.data(), V, temperature, top_k, uniform01(seed, frame, (uint32_t)(g + 1)),
                              true, 0.0f, -1, &gap, &kgap);
            gap = sampled_tie_measure(gap, kgap, temperature);
        }
        if (temperature <= 0.0f) {  // record the top-2 gap of this decision
            float best = -INFINITY, second = -INFINITY;
            for (int i = 0; i < V; ++i) {
                if (work[i] > best) { second = best; best = work[i]; } else if (work[i] > second) second = work[i];
            }
            res->min_decision_gap = std::min(res->min_decision_gap, best - second);
        }
        if (follow && follow[g] != pick) {
            float d = temperature <= 0.0f ? work[pick] - work[follow[g]] : (float) gap;
            if (d <= tie_tol) { res->n_ties++; res->max_tie_gap = std::max(res->max_tie_gap, d); }
            else {
                if (res->first_mismatch < 0) res->first_mismatch = *dec_index;
                res->n_mismatch++;
                res->max_mismatch_gap = std::max(res->max_mismatch_gap, d);
            }
            pick = follow[g];
        }
        (*dec_index)++;
        out[g] = pick;
    }
}

int orc_predict_codes_ar(void * h, const float * hidden, int cb0, float temperature, int top_k, uint64_t seed,
                         uint32_t frame, int32_t * codes_out, float * cp_logits_out) {
    Model & m = *(Model *) h;
    orc_gen_result r{}; r.first_mismatch = -1; r.min_decision_gap = INFINITY;
    int di = 0;
    predict_codes(m, hidden, cb0, temperature, top_k, seed, frame, codes_out, cp_logits_out, nullptr, 0, &r, &di);
    return 0;
}

// build_prefill_graph (src/tts_transformer.cpp:1030-1186).
static int build_prefill(Model & m, const orc_gen_args * a, std::vector<float> & prefill,
                         std::vector<float> & trailing, std::vector<float> & pad) {
    const Config & c = m.c;
    const int H = c.hidden;
    if (!a->text || a->n_text < 4) return -1;
    int32_t special[3] = {c.tts_bos, c.tts_eos, c.tts_pad};
    std::vector<float> sp(3 * H), role(3 * H), first(H);
    orc_project_text(&m, special, 3, sp.data());
    const float * bos = sp.data(); const float * eos = sp.data() + H;
    pad.assign(sp.data() + 2 * H, sp.data() + 3 * H);
    orc_project_text(&m, a->text, 3, role.data());
    std::vector<int32_t> ctoks;
    if (a->language_id < 0) ctoks = {c.nothink, c.think_bos, c.think_eos};
    else ctoks = {c.think, c.think_bos, a->language_id, c.think_eos};
    std::vector<float> cpe(ctoks.size() * H);
    if (orc_lookup_rows(&m, 0, ctoks.data(), (int) ctoks.size(), cpe.data())) return -1;
    int32_t tail[2] = {c.codec_pad, c.codec_bos};
    std::vector<float> te(2 * H);
    orc_lookup_rows(&m, 0, tail, 2, te.data());
    const bool spk = a->speaker != nullptr;
    const int cin = (int) ctoks.size() + (spk ? 1 : 0) + 2;
    std::vector<float> ci((size_t) cin * H);
    memcpy(ci.data(), cpe.data(), cpe.size() * 4);
    int dst = (int) ctoks.size();
    if (spk) { memcpy(ci.data() + (size_t) dst * H, a->speaker, H * 4); ++dst; }
    memcpy(ci.data() + (size_t) dst * H, te.data(), te.size() * 4);
    const int ov = cin - 1;
    std::vector<float> cov((size_t) ov * H);
    for (int t = 0; t < ov; ++t) {
        const float * o = (t == ov - 1) ? bos : pad.data();
        for (int d = 0; d < H; ++d) cov[(size_t) t * H + d] = o[d] + ci[(size_t) t * H + d];
    }
    orc_project_text(&m, a->text + 3, 1, first.data());
    std::vector<float> fb(H);
    for (int d = 0; d < H; ++d) fb[d] = first[d] + ci[(size_t)(cin - 1) * H + d];
    std::vector<float> ins;
    int ilen = 0;
    if (a->instruct && a->n_instruct > 0) {
        ins.resize((size_t) a->n_instruct * H);
        orc_project_text(&m, a->instruct, a->n_instruct, ins.data());
        ilen = a->n_instruct;
    }
    const int plen = ilen + 3 + ov + 1;
    prefill.resize((size_t) plen * H);
    if (ilen) memcpy(prefill.data(), ins.data(), ins.size() * 4);
    memcpy(prefill.data() + (size_t) ilen * H, role.data(), role.size() * 4);
    memcpy(prefill.data() + (size_t)(ilen + 3) * H, cov.data(), cov.size() * 4);
    memcpy(prefill.data() + (size_t)(plen - 1) * H, fb.data(), H * 4);
    const int ntrail = std::max(0, a->n_text - 9);
    trailing.assign((size_t)(ntrail + 1) * H, 0.0f);
    if (ntrail > 0) orc_project_text(&m, a->text + 4, ntrail, trailing.data());
    memcpy(trailing.data() + (size_t) ntrail * H, eos, H * 4);
    return 0;
}

// build_prefill_graph_icl (src/tts_transformer.cpp:1188-1472).
static int build_prefill_icl(Model & m, const orc_gen_args * a, std::vector<float> & prefill,
                             std::vector<float> & trailing, std::vector<float> & pad) {
    const Config & c = m.c;
    const int H = c.hidden;
    if (!a->text || a->n_text < 4 || !a->ref_codes || a->n_ref_frames < 1) return -1;
    int32_t special[3] = {c.tts_bos, c.tts_eos, c.tts_pad};
    std::vector<float> sp(3 * H), role(3 * H);
    orc_project_text(&m, special, 3, sp.data());
    const float * bos = sp.data();
    pad.assign(sp.data() + 2 * H, sp.data() + 3 * H);
    orc_project_text(&m, a->text, 3, role.data());
    std::vector<int32_t> ctoks = {c.nothink, c.think_bos, c.think_eos};
    std::vector<float> cpe(3 * H), te(2 * H);
    orc_lookup_rows(&m, 0, ctoks.data(), 3, cpe.data());
    int32_t tail[2] = {c.codec_pad, c.codec_bos};
    orc_lookup_rows(&m, 0, tail, 2, te.data());
    const bool spk = a->speaker != nullptr;
    const int cin = 3 + (spk ? 1 : 0) + 2;
    std::vector<float> ci((size_t) cin * H);
    memcpy(ci.data(), cpe.data(), cpe.size() * 4);
    int dst = 3;
    if (spk) { memcpy(ci.data() + (size_t) dst * H, a->speaker, H * 4); ++dst; }
    memcpy(ci.data() + (size_t) dst * H, te.data(), te.size() * 4);
    const int ov = cin - 1;
    prefill.assign((size_t)(3 + ov) * H, 0.0f);
    memcpy(prefill.data(), role.data(), role.size() * 4);
    for (int t = 0; t < ov; ++t) {
        const float * o = (t == ov - 1) ? bos : pad.data();
        for (int d = 0; d < H; ++d) prefill[(size_t)(3 + t) * H + d] = o[d] + ci[(size_t) t * H + d];
    }
    int rs = 3, re = a->n_ref_text - 5; if (re < rs) re = rs;
    int ts = 3, tend = a->n_text - 5; if (tend < ts) tend = ts;
    std::vector<int32_t> comb;
    for (int i = rs; i < re && i < a->n_ref_text; ++i) comb.push_back(a->ref_text[i]);
    for (int i = ts; i < tend && i < a->n_text; ++i) comb.push_back(a->text[i]);
    comb.push_back(c.tts_eos);
    const int nct = a->n_ref_frames + 1;
    std::vector<float> cf((size_t) nct * H, 0.0f), row(H);
    int32_t cbos = c.codec_bos;
    orc_lookup_rows(&m, 0, &cbos, 1, cf.data());
    for (int f = 0; f < a->n_ref_frames; ++f) {
        float * d = cf.data() + (size_t)(f + 1) * H;
        int32_t t0 = a->ref_codes[(size_t) f * 16];
        if (orc_lookup_rows(&m, 0, &t0, 1, d)) return -1;
        for (int cb = 1; cb < 16 && cb < c.n_cb; ++cb) {
            int32_t t = a->ref_codes[(size_t) f * 16 + cb];
            if (orc_lookup_rows(&m, cb, &t, 1, row.data())) return -1;
            for (int k = 0; k < H; ++k) d[k] += row[k];
        }
    }
    const int nt = (int) comb.size();
    std::vector<float> tp((size_t) nt * H);
    orc_project_text(&m, comb.data(), nt, tp.data());
    const int icl = nct;
    std::vector<float> ie((size_t) icl * H, 0.0f);
    for (int i = 0; i < icl; ++i) {
        float * d = ie.data() + (size_t) i * H;
        const float * t = i < nt ? tp.data() + (size_t) i * H : pad.data();
        for (int k = 0; k < H; ++k) d[k] += t[k];
        const float * cr = cf.data() + (size_t) i * H;
        for (int k = 0; k < H; ++k) d[k] += cr[k];
    }
    const size_t base = prefill.size() / H;
    prefill.resize((base + icl) * H);
    memcpy(prefill.data() + base * H, ie.data(), ie.size() * 4);
    trailing.clear();
    if (nt > nct) trailing.assign(tp.data() + (size_t) nct * H, tp.data() + (size_t) nt * H);
    return 0;
}

// generate (src/tts_transformer.cpp:3007-3371) / generate_icl (:3373-3656).
int orc_generate(void * h, const orc_gen_args * a, orc_gen_result * r) {
    Model & m = *(Model *) h;
    const Config & c = m.c;
    const int H = c.hidden, V = c.codec_vocab, NCB = c.n_cb;
    memset(r, 0, sizeof(*r));
    r->first_mismatch = -1; r->min_decision_gap = INFINITY;
    if (a->max_len <= 0) return 0;
    std::vector<float> prefill, trailing, pad;
    int rc = a->ref_codes ? build_prefill_icl(m, a, prefill, trailing, pad) : build_prefill(m, a, prefill, trailing, pad);
    if (rc) return rc;
    const int plen = (int)(prefill.size() / H), tlen = (int)(trailing.size() / H);
    r->prefill_len = plen;
    if (a->prefill_out) memcpy(a->prefill_out, prefill.data(), (size_t) std::min(plen, a->prefill_cap) * H * 4);
    const int required = plen + a->max_len + 8;
    if (m.cache.n_ctx < required || m.cache.n_ctx > std::max(required * 2, 512)) orc_init_kv(h, required);
    std::vector<float> logits(V), hidden(H);
    orc_forward_prefill(h, prefill.data(), plen, 0, nullptr, logits.data());
    int n_past = plen;
    std::vector<int32_t> fc(NCB), out;
    std::unordered_set<int32_t> seen;
    std::vector<std::vector<int32_t>> rep;
    int run = 0, run_start = 0;
    const int sup = V - 1024;
    std::vector<float> step(H), row(H);
    int dec = 0;
    g_in_frame = true;
    for (int frame = 0; frame < a->max_len; ++frame) {
        if (a->talker_logits_out && frame < a->codes_cap) memcpy(a->talker_logits_out + (size_t) frame * V, logits.data(), V * 4);
        for (int i = sup; i < V; ++i) if (i != c.codec_eos) logits[i] = -INFINITY;
        if (a->rep_penalty != 1.0f) {
            for (int32_t t : seen) {
                if (t >= 0 && t < V) { if (logits[t] > 0.0f) logits[t] /= a->rep_penalty; else logits[t] *= a->rep_penalty; }
            }
        }
        float eb = a->eos_bias;
        if (a->target_frames > 0 && frame > a->target_frames) {
            eb += 0.1f * (float)(frame - a->target_frames);
            if (eb > 6.0f) eb = 6.0f;
        }
        int next; double gap = 1e30, kgap = 1e30;
        if (a->temperature <= 0.0f) {
            if (eb != 0.0f) logits[c.codec_eos] += eb;
            next = argmax(logits.data(), V);
        } else {
            next = sample_tok(logits.data(), V, a->temperature, a->top_k, uniform01(a->seed, (uint32_t) frame, 0u),
                              true, eb, c.codec_eos, &gap, &kgap);
            gap = sampled_tie_measure(gap, kgap, a->temperature);
        }
        const int32_t * fol = nullptr;
        if (a->follow) {
            int want = frame < a->n_follow ? a->follow[(size_t) frame * NCB] : c.codec_eos;
            if (frame < a->n_follow) fol = a->follow + (size_t) frame * NCB;
            if (want != next) {
                float d = a->temperature <= 0.0f ? logits[next] - logits[want] : (float) gap;
                if (d <= a->tie_tol) { r->n_ties++; r->max_tie_gap = std::max(r->max_tie_gap, d); }
                else {
                    if (r->first_mismatch < 0) r->first_mismatch = dec;
                    r->n_mismatch++;
                    r->max_mismatch_gap = std::max(r->max_mismatch_gap, d);
                }
                next = want;
            }
        }
        if (a->temperature <= 0.0f) {
            float best = -INFINITY, second = -INFINITY;
            for (int i = 0; i < V; ++i) {
                if (logits[i] > best) { second = best; best = logits[i]; } else if (logits[i] > second) second = logits[i];
            }
            r->min_decision_gap = std::min(r->min_decision_gap, best - second);
        }
        dec++;
        if (next == c.codec_eos) break;
        fc[0] = next;
        seen.insert(next);
        predict_codes(m, m.last_hidden.data(), fc[0], a->temperature, a->top_k, a->seed, (uint32_t) frame, fc.data() + 1,
                      a->cp_logits_out && frame < a->codes_cap ? a->cp_logits_out + (size_t) frame * (NCB - 1) * c.cp_vocab : nullptr,
                      fol ? fol + 1 : nullptr, a->tie_tol, r, &dec);
        for (int cb = 0; cb < NCB; ++cb) out.push_back(fc[cb]);
        if (a->rep_loop_detect) rep.emplace_back(fc.begin(), fc.end());
        {
            const size_t nf = rep.size();
            bool is_rep = false;
            for (int back = 1; back <= 6 && !is_rep && (size_t) back < nf; ++back) {
                int match = 0;
                for (int cb = 0; cb < NCB; ++cb) if (rep[nf - 1][cb] == rep[nf - 1 - back][cb]) ++match;
                if (match >= 10) is_rep = true;
            }
            if (is_rep) { if (run == 0) run_start = (int)(nf - 1); ++run; } else run = 0;
            if (run >= 5) { out.resize((size_t) run_start * NCB); r->truncated = 1; break; }
        }
        if (frame + 1 >= a->max_len) break;
        orc_lookup_rows(h, 0, &fc[0], 1, step.data());
        for (int cb = 1; cb < NCB; ++cb) {
            orc_lookup_rows(h, cb, &fc[cb], 1, row.data());
            for (int d = 0; d < H; ++d) step[d] += row[d];
        }
        const float * tr = frame < tlen ? trailing.data() + (size_t) frame * H : pad.data();
        for (int d = 0; d < H; ++d) step[d] += tr[d];
        orc_forward_step(h, step.data(), n_past, logits.data(), nullptr);
        n_past++;
    }
    g_in_frame = false;
    r->n_frames = (int)(out.size() / NCB);
    if (a->codes_out) memcpy(a->codes_out, out.data(), (size_t) std::min(r->n_frames, a->codes_cap) * NCB * 4);
    return 0;
}

// Stand-alone helpers used by the component tests.
int orc_quantize_q8_0(const float * x, int n, int8_t * q, uint16_t * d) {
    QBlocks b; quantize_q8_0(x, n, b);
    memcpy(q, b.q.data(), n); memcpy(d, b.d.data(), (n / 32) * 2);
    return 0;
}
int orc_rope_cache(int pos, int n_dims, float base, float * cs) { rope_cache(pos, n_dims, base, cs); return 0; }
double orc_uniform01(uint64_t seed, uint32_t frame, uint32_t cb) { return uniform01(seed, frame, cb); }
void orc_philox(uint32_t * c, uint32_t k0, uint32_t k1) { philox(c, k0, k1); }
int orc_sample(float * logits, int n, float temperature, int top_k, double u) {
    if (temperature <= 0.0f) return argmax(logits, n);
    return sample_tok(logits, n, temperature, top_k, u, true, 0.0f, -1, nullptr);
}
// One talker layer stack run on M rows (for the layer-maths pin), F32 in/out.
int orc_forward_talker_rows(void * h, float * X, int M, int n_past) {
    Model & m = *(Model *) h;
    if (m.cache.n_ctx < n_past + M) orc_init_kv(h, n_past + M + 16);
    std::vector<float> x(X, X + (size_t) M * m.c.hidden);
    forward_stack(m, m.L, m.cache, m.c.theta, x, M, n_past, true, m.c.ffn);
    memcpy(X, x.data(), x.size() * 4);
    return 0;
}

}  // extern "C"
