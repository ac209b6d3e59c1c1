// engine.cu — B200 engine for the TTSTransformer decode path, behind the C ABI
// of include/qwen3tts_b200.h.
//
// Layout in HBM (one engine per GPU):
//   * weights: one allocation.  Per layer the Q, K and V matrices are fused into
//     one [NH*D + 2*NKV*D, H] matrix; F16 matrices keep the GGUF row-major
//     layout; Q8_0 matrices are split at load time into an int8 quant plane
//     [rows][cols] and an F16 scale plane [rows][cols/32] (same 34 bytes per 32
//     weights, 16-byte aligned rows for vector loads).
//   * KV caches: F16 [layer][pos][kv_head][128] (the reference's
//     [head_dim, n_kv_heads, n_ctx] ggml tensors, src/tts_transformer.cpp:757-770).
//   * RoPE tables: (cos, sin) per position and pair index, computed once with the
//     ggml_rope_cache_init recurrence.
//   * frame state (positions, codes, EOS flag, codebook-0 presence set) lives in
//     device memory, so a single captured CUDA graph replays every frame: talker
//     cb0 sampling, the 2-token code-predictor prefill, 14 code-predictor steps
//     with on-device sampling, the next-step embedding sum and the 28-layer talker
//     step, with no host round trip inside a frame.
#include "../../include/qwen3tts_b200.h"
#include "gguf.hpp"
#include "frame_fused.cuh"
#include "gemm_q8.cuh"
#include "gemm_tc.cuh"
#include "batch_engine.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <thread>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace qtts {

#define QCHECK(call)                                                                   \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            err = std::string(#call) + ": " + cudaGetErrorString(e_);                  \
            return false;                                                              \
        }                                                                              \
    } while (0)

enum KernelClass { KC_GEMV = 0, KC_ATTN = 1, KC_SAMPLE = 2, KC_OTHER = 3, KC_N = 4 };

struct LayerW {
    DMat qkv, o, gate, up, down;
    const float * attn_norm = nullptr, * ffn_norm = nullptr, * q_norm = nullptr, * k_norm = nullptr;
};

struct GenSession {
    bool active = false;
    int max_len = 0, prefill_len = 0, trailing_len = 0, produced = 0;
    bool done = false;
    DevState st0{};   // frame state right after the prefill (rewind target)
};

// Recipe of a prompt (build_prefill_graph, src/tts_transformer.cpp:1030-1186, and
// build_prefill_graph_icl, :1188-1472), written on the host and carried out on
// the device: the text tokens to project, the codec rows to gather, the speaker
// row, the ICL reference frames, and each output row's terms in order.
struct PromptSrc {
    enum { NONE = 0, TEXT, CODEC, SPEAKER, ICL };
    int kind = NONE, idx = 0;
};
struct PromptPlan {
    std::vector<int32_t> text, codec, icl_codes;   // icl_codes: [n_icl][16]
    int n_icl = 0;
    const float * speaker = nullptr;               // host row, or nullptr
    enum { PREFILL = 0, TRAILING, PAD };
    struct Row { int dst, r; PromptSrc a, b; int zero_first; };
    std::vector<Row> rows;
    int plen = 0, tlen = 0;
    void add(int dst, int r, PromptSrc a, PromptSrc b = {}, int zero_first = 0) {
        rows.push_back({dst, r, a, b, zero_first});
        if (dst == PREFILL) plen = std::max(plen, r + 1);
        if (dst == TRAILING) tlen = std::max(tlen, r + 1);
    }
};

struct Engine;
struct PrefillTC;
constexpr int PREFILL_TC_ROWS = 128;   // prompt rows per tensor-core chunk (hi/lo ffn_down doubles MMA N to 256)
// Tensor-core talker prefill (defined with the batched path's host code).
bool prefill_tc_layers(Engine & E, float * X, int M, int n_past);
bool prefill_tc_check(Engine & E);   // after a sync: no GEMM reported an error
void prefill_tc_free(PrefillTC * p);

struct Engine {
    int dev = 0, n_sm = 148;
    cudaStream_t stream = nullptr;
    qtts_config cfg{};
    std::string err;

    // weights
    uint8_t * wbuf = nullptr;
    size_t wbytes = 0, wused = 0;
    std::vector<LayerW> L, CPL;
    const __half * text_embd = nullptr, * codec_embd = nullptr;
    std::vector<const __half *> cp_embd;
    const __half ** d_cp_embd = nullptr;
    DMat codec_head, fc1, fc2;
    std::vector<DMat> cp_head;
    const float * fc1_b = nullptr, * fc2_b = nullptr, * out_norm = nullptr, * cp_out_norm = nullptr;

    // rope tables and caches
    float2 * rope_t = nullptr, * rope_cp = nullptr;
    __half * kc = nullptr, * vc = nullptr;
    int n_ctx = 0, n_used = 0;
    __half * cpk = nullptr, * cpv = nullptr;
    int cp_ctx = 0;

    // activations (rows <= QTTS_MAX_NV)
    float * x = nullptr, * xcp = nullptr, * qkv = nullptr, * att = nullptr, * hbuf = nullptr;
    float * logits = nullptr, * cp_logits = nullptr, * hidden = nullptr;
    float * logits0 = nullptr, * hidden0 = nullptr;   // prefill outputs kept for rewind
    float * tmp_a = nullptr, * tmp_b = nullptr;
    float * d_ptext = nullptr;  // projected text rows of project_text [ptext_cap][H]
    int ptext_cap = 0;
    int * d_ids = nullptr;
    int ids_cap = 0;
    float * d_prow = nullptr;   // prefill rows [prow_cap][H]: assembled on the device, or uploaded
    int prow_cap = 0;
    float * d_asm = nullptr;    // prompt assembly terms: gathered codec rows, speaker row, ICL frame rows
    int asm_cap = 0;
    PromptRow * d_pops = nullptr;   // prompt row recipes for k_prompt_rows
    int pops_cap = 0;
    cudaEvent_t ev_asm0 = nullptr, ev_asm1 = nullptr;
    PrefillTC * ptc = nullptr;  // tensor-core prefill (created on first use)

    // frame state
    DevState * st = nullptr;
    SampleParams * sp = nullptr;
    int * d_codes = nullptr;
    int codes_cap = 0;
    float * trailing = nullptr;
    int trailing_cap = 0;
    float * pad = nullptr;
    float * dbg_t = nullptr, * dbg_cp = nullptr;
    int dbg_cap = 0;
    float * h_dbg_t = nullptr, * h_dbg_cp = nullptr;
    int h_dbg_cap = 0;
    float * d_attn = nullptr;
    size_t attn_cap = 0;
    bool attn_dump = false;
    int attn_layer = 27;
    std::vector<std::vector<float>> attn_rows;

    cudaGraphExec_t graph = nullptr;
    bool graph_ok = false;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    std::vector<float> last_hidden;
    uint64_t seed = 0;
    uint32_t api_calls = 0;
    qtts_timing timing{};
    int launches = 0;
    int launches_per_frame = 0;
    GenSession sess;
    // frame path: FM_GRAPH (one kernel per op, the default) or FM_FUSED (two
    // clustered kernels per layer; QTTS_FRAME_MODE=fused, where the model's shapes
    // allow it)
    enum { FM_GRAPH = 0, FM_FUSED = 1 };
    int frame_mode = FM_GRAPH;
    int * d_err = nullptr;        // set by a fused kernel whose bounded wait gave up
    size_t gemv_smem_floor = 0;   // dynamic shared memory floor of a GEMV launch (see alloc_activations)
    struct FfLayerW { DMat qkv_g, o_g, down_r; };
    std::vector<FfLayerW> ffL, ffCP;
    uint8_t * ffw = nullptr;      // repacked weights of the fused frame path
    float * ff_part_o = nullptr, * ff_part_d = nullptr, * ff_xres = nullptr, * ff_xmid = nullptr;
    int ff_CA = 16;               // attention block: CTAs per kv-group cluster
    struct FfStack { int R = 0, N = 0, C = 0; };   // FFN block: rows per CTA, CTAs, cluster size
    FfStack ffs_t, ffs_cp;
    size_t ff_head_smem_t = 0, ff_head_smem_cp = 0;
    int ff_max_keys = 0;          // the talker attention row length the captured frame serves
    int ff_pf_ahead = 1;          // launches whose weights each launch prefetches into L2 (QTTS_FF_PF)
    std::string ff_why;           // why the fused path is off (empty: on)
    unsigned long long * d_fftrace = nullptr;   // QTTS_FF_TRACE=1: stamps of frame 1's launches
    std::vector<int> ff_kinds;    // per launch of the frame: kind * 4 + (samples ? 2 : 0) + (nv - 1)
    // eager profiling: CUDA events around every launch, accumulated per kernel class
    bool profiling = false;
    struct ProfEv { int cls; int stage; double bytes; cudaEvent_t a, b; };
    // stage timing (qtts_set_stage_timing): frames run kernel by kernel with events,
    // each launch charged to the talker step, the code predictor or the samplers
    enum { STG_TALKER = 0, STG_CP = 1 };
    int prof_stage = STG_TALKER;
    bool stage_timing = false;
    qtts_stage_timing stages{};
    std::vector<ProfEv> prof_evs;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    cudaEvent_t pool_event() {
        if (ev_used == ev_pool.size()) { cudaEvent_t e; cudaEventCreate(&e); ev_pool.push_back(e); }
        return ev_pool[ev_used++];
    }
    void prof_begin(int cls, double bytes) {
        if (!profiling) return;
        ProfEv p{cls, prof_stage, bytes, pool_event(), pool_event()};
        cudaEventRecord(p.a, stream);
        prof_evs.push_back(p);
    }
    void prof_end() { if (profiling) cudaEventRecord(prof_evs.back().b, stream); }

    ~Engine() {
        for (auto e : ev_pool) cudaEventDestroy(e);
        release();
    }

    int QD() const { return cfg.n_attention_heads * QTTS_HD; }
    int KD() const { return cfg.n_key_value_heads * QTTS_HD; }
    int QKVD() const { return QD() + 2 * KD(); }

    void release() {
        if (dev >= 0) cudaSetDevice(dev);
        if (graph) { cudaGraphExecDestroy(graph); graph = nullptr; }
        if (ptc) { prefill_tc_free(ptc); ptc = nullptr; }
        if (d_prow) { cudaFree(d_prow); d_prow = nullptr; prow_cap = 0; }
        if (d_asm) { cudaFree(d_asm); d_asm = nullptr; asm_cap = 0; }
        if (d_pops) { cudaFree(d_pops); d_pops = nullptr; pops_cap = 0; }
        if (ev_asm0) { cudaEventDestroy(ev_asm0); ev_asm0 = nullptr; }
        if (ev_asm1) { cudaEventDestroy(ev_asm1); ev_asm1 = nullptr; }
        void * ptrs[] = {wbuf, d_cp_embd, rope_t, rope_cp, kc, vc, cpk, cpv, x, xcp, qkv, att, hbuf, logits,
                         cp_logits, hidden, tmp_a, tmp_b, d_ptext, d_ids, st, sp, d_codes, trailing, pad,
                         dbg_t, dbg_cp, d_attn, d_err, logits0, hidden0, ffw, ff_part_o, ff_part_d, ff_xres,
                         ff_xmid, d_fftrace};
        for (void * p : ptrs) if (p) cudaFree(p);
        wbuf = nullptr; d_cp_embd = nullptr; rope_t = rope_cp = nullptr; kc = vc = cpk = cpv = nullptr;
        x = xcp = qkv = att = hbuf = logits = cp_logits = hidden = tmp_a = tmp_b = d_ptext = nullptr;
        ptext_cap = 0;
        logits0 = hidden0 = nullptr;
        d_ids = nullptr; st = nullptr; sp = nullptr; d_codes = nullptr; trailing = pad = nullptr;
        dbg_t = dbg_cp = nullptr; d_attn = nullptr; d_err = nullptr;
        ffw = nullptr; ff_part_o = ff_part_d = ff_xres = ff_xmid = nullptr; d_fftrace = nullptr;
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        ev0 = ev1 = nullptr;
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
    }

    // ------------------------------------------------------------ loading
    bool load(const char * path, int device);
    bool upload_weights(const GgufFile & g);
    bool alloc_activations();
    bool init_kv(int ctx);
    bool init_cp_kv(int ctx);
    void build_rope(std::vector<float2> & t, int n_pos, float base);

    // ------------------------------------------------------------ launches
    bool gemv(const DMat & A, const DMat * B, const float * xin, int ldx, int nv, const float * norm, int act,
              float * y, int ldy, const float * resid, int ldr, int epi, float * xn_out, int ldxn, const int * done);
    bool layers(std::vector<LayerW> & Ls, __half * kbase, __half * vbase, int ctx, const float2 * rope, float * X,
                int M, const int * pos_ptr, int pos_static, bool f32_mode, const int * done, int ffn,
                float * dump = nullptr, int dump_layer = -1);
    FusedAttn fused_attn_args(const LayerW & l, __half * kc_l, __half * vc_l, const float2 * rope, int M,
                              const int * pos_ptr, int pos_static, bool f32, float * dump, int dump_stride);
    void prefill_attention(const LayerW & l, __half * kc_l, __half * vc_l, const float2 * rope, const float * q,
                           int ldq, int M, const int * pos_ptr, int pos_static, const int * done, float * out, int ldo,
                           float * dump, int dump_stride, size_t smem);
    bool enqueue_cp(bool sample_cb0, const InputArgs * last_in = nullptr);
    bool enqueue_talker_step(const int * pos_ptr, int pos_static, const int * done, bool with_dump);
    bool enqueue_frame();
    bool capture_graph();
    GemvArgs make_gemv(const DMat & A, const DMat * B, const float * xin, int ldx, int nv, const float * norm, int act,
                       float * y, int ldy, const float * resid, int ldr, int epi, float * xn_out, int ldxn,
                       const int * done, int * ncta_out, size_t * slice_out, size_t * smem_out);
    bool ff_prepare();                  // repacked weights, buffers and launch shapes of FM_FUSED
    bool enqueue_frame_ff();
    bool ff_layers(bool cp, int pass, const float * in_logits);
    bool sync(const char * what);

    // ------------------------------------------------------------ API pieces
    bool prefill(const float * rows_host, int n, int n_past, float * hidden_out, float * logits_out);
    bool project_text(const int32_t * toks, int n, std::vector<float> & out);
    bool lookup(int table, const int32_t * ids, int n, std::vector<float> & out);
    bool project_text_dev(const int * d_tok, int n);
    bool grow_rows(float ** buf, int * cap, int n, const char * what);
    bool plan_prompt(const qtts_generate_params * p, PromptPlan & P);
    bool assemble_prompt(const PromptPlan & P);
    int begin(const qtts_generate_params * p);
    int run_frames(int n, int32_t * codes_out);
    int rewind();
};

static thread_local std::string g_create_error;

void Engine::build_rope(std::vector<float2> & t, int n_pos, float base) {
    // ggml_rope_cache_init (ext_factor 0, freq_scale 1, attn_factor 1): theta for
    // pair i is pos * s^i accumulated by repeated F32 multiplication.
    const int half = QTTS_HD / 2;
    t.resize((size_t) n_pos * half);
    const float theta_scale = powf(base, -2.0f / (float) QTTS_HD);
    for (int p = 0; p < n_pos; ++p) {
        float theta = (float) p;
        for (int i = 0; i < half; ++i) {
            t[(size_t) p * half + i] = make_float2(cosf(theta), sinf(theta));
            theta *= theta_scale;
        }
    }
}

bool Engine::load(const char * path, int device) {
    if (device < 0) {
        const char * env = getenv("QWEN3_TTS_DEVICE");
        device = env && *env ? atoi(env) : 0;
    }
    dev = device;
    const auto t_load = std::chrono::steady_clock::now();
    QCHECK(cudaSetDevice(dev));
    QCHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    QCHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    QCHECK(cudaEventCreate(&ev0));
    QCHECK(cudaEventCreate(&ev1));

    GgufFile g;
    if (!g.open(path, err)) return false;
    // parse_config (src/tts_transformer.cpp:228-377), same aliases and defaults
    qtts_config & c = cfg;
    c.text_vocab_size = (int) g.get_int({"qwen3-tts.text.vocab_size", "qwen3-tts.text_vocab_size"}, 151936);
    c.text_embd_dim = (int) g.get_int({"qwen3-tts.text.embedding_dim", "qwen3-tts.text_hidden_size"}, 2048);
    c.hidden_size = (int) g.get_int({"qwen3-tts.talker.embedding_length", "qwen3-tts.embedding_length"}, 1024);
    c.n_layers = (int) g.get_int({"qwen3-tts.talker.block_count", "qwen3-tts.block_count"}, 28);
    c.n_attention_heads = (int) g.get_int({"qwen3-tts.talker.attention.head_count", "qwen3-tts.attention.head_count"}, 16);
    c.n_key_value_heads = (int) g.get_int({"qwen3-tts.talker.attention.head_count_kv", "qwen3-tts.attention.head_count_kv"}, 8);
    c.intermediate_size = (int) g.get_int({"qwen3-tts.talker.feed_forward_length", "qwen3-tts.feed_forward_length"}, 3072);
    c.head_dim = (int) g.get_int({"qwen3-tts.talker.attention.key_length", "qwen3-tts.attention.key_length"}, 128);
    c.rms_norm_eps = (float) g.get_float({"qwen3-tts.talker.attention.layer_norm_rms_epsilon", "qwen3-tts.attention.layer_norm_rms_epsilon"}, 1e-6);
    c.rope_theta = (float) g.get_float({"qwen3-tts.talker.rope.freq_base", "qwen3-tts.rope.freq_base"}, 1000000.0);
    c.mrope_section[0] = 24; c.mrope_section[1] = 20; c.mrope_section[2] = 20;
    c.codec_vocab_size = (int) g.get_int({"qwen3-tts.talker.codec_vocab_size", "qwen3-tts.vocab_size"}, 3072);
    c.n_codebooks = (int) g.get_int({"qwen3-tts.talker.num_codebooks", "qwen3-tts.num_code_groups"}, 16);
    c.code_pred_layers = (int) g.get_int({"qwen3-tts.code_pred.layer_count", "qwen3-tts.code_predictor.layer_count"}, 5);
    c.code_pred_vocab_size = (int) g.get_int({"qwen3-tts.code_pred.vocab_size", "qwen3-tts.code_predictor.vocab_size"}, 2048);
    c.code_pred_hidden_size = (int) g.get_int({"qwen3-tts.code_pred.embedding_length", "qwen3-tts.code_predictor.embedding_length"}, 1024);
    c.code_pred_intermediate_size = (int) g.get_int({"qwen3-tts.code_pred.feed_forward_length", "qwen3-tts.code_predictor.feed_forward_length"}, 3072);
    c.code_pred_rope_theta = (float) g.get_float({"qwen3-tts.code_pred.rope.freq_base", "qwen3-tts.code_predictor.rope.freq_base"}, c.rope_theta);
    c.codec_pad_id = (int) g.get_int({"qwen3-tts.codec.pad_id"}, 2148);
    c.codec_bos_id = (int) g.get_int({"qwen3-tts.codec.bos_id"}, 2149);
    c.codec_eos_id = (int) g.get_int({"qwen3-tts.codec.eos_id", "qwen3-tts.codec.eos_token_id"}, 2150);
    c.tts_bos_token_id = (int) g.get_int({"qwen3-tts.tts_bos_token_id", "qwen3-tts.tts.bos_token_id", "qwen3-tts.tts.bos_id"}, 151672);
    c.tts_eos_token_id = (int) g.get_int({"qwen3-tts.tts_eos_token_id", "qwen3-tts.tts.eos_token_id", "qwen3-tts.tts.eos_id"}, 151673);
    c.tts_pad_token_id = (int) g.get_int({"qwen3-tts.tts_pad_token_id", "qwen3-tts.tts.pad_token_id", "qwen3-tts.tts.pad_id"}, 151671);
    c.codec_think_id = (int) g.get_int({"qwen3-tts.codec.think_id", "qwen3-tts.codec_think_id"}, 2154);
    c.codec_nothink_id = (int) g.get_int({"qwen3-tts.codec.nothink_id", "qwen3-tts.codec_nothink_id"}, 2155);
    c.codec_think_bos_id = (int) g.get_int({"qwen3-tts.codec.think_bos_id", "qwen3-tts.codec_think_bos_id"}, 2156);
    c.codec_think_eos_id = (int) g.get_int({"qwen3-tts.codec.think_eos_id", "qwen3-tts.codec_think_eos_id"}, 2157);
    c.english_language_id = (int) g.get_int({"qwen3-tts.language.english_id", "qwen3-tts.codec.language.english_id", "qwen3-tts.language_id"}, 2050);

    if (c.head_dim != QTTS_HD) { err = "head_dim must be 128"; return false; }
    if (c.code_pred_hidden_size != c.hidden_size || g.find("code_pred.mtp_proj.weight")) {
        err = "code predictor width differs from the talker (mtp_proj layout) - not supported";
        return false;
    }
    if (c.n_codebooks < 2 || c.n_codebooks > QTTS_MAX_CB) { err = "n_codebooks out of range"; return false; }
    static_assert(QTTS_MAX_CB <= CPA_MAX_KEYS, "code-predictor step attention covers every codebook position");
    if (c.codec_vocab_size > SAMPLE_THREADS * SAMPLE_PER_T || c.code_pred_vocab_size > SAMPLE_THREADS * SAMPLE_PER_T) {
        err = "vocabulary larger than 4096 is not supported"; return false;
    }
    if (c.n_attention_heads % c.n_key_value_heads || c.n_attention_heads / c.n_key_value_heads > ATT_MAX_GROUP ||
        c.n_attention_heads + c.n_key_value_heads > 32) {
        err = "unsupported head configuration"; return false;
    }
    if (c.hidden_size % 256 || c.intermediate_size % 32 || c.code_pred_intermediate_size % 32 || c.text_embd_dim % 32) {
        err = "hidden/ffn/text widths must be multiples of 256/32/32"; return false;
    }
    if (!upload_weights(g)) return false;
    if (!alloc_activations()) return false;
    if (!init_cp_kv(16)) return false;
    const char * fm = getenv("QTTS_FRAME_MODE");
    if (fm && strcmp(fm, "fused") == 0 && !ff_prepare()) return false;
    timing.load_ms = (float) std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_load).count();
    return true;
}

// Q8_0 GGUF blocks (f16 d + 32 int8, 34 bytes) -> the engine's int8 plane
// [rows][cols] and scale plane [rows][cols/32]: one thread per block.
__global__ void k_split_q8(const uint8_t * blocks, size_t n_blocks, int8_t * q, __half * d) {
    for (size_t bi = (size_t) blockIdx.x * blockDim.x + threadIdx.x; bi < n_blocks; bi += (size_t) gridDim.x * blockDim.x) {
        const uint8_t * src = blocks + bi * 34;
        uint32_t w[8];
        for (int k = 0; k < 8; ++k)
            w[k] = (uint32_t) src[2 + 4 * k] | (uint32_t) src[3 + 4 * k] << 8 | (uint32_t) src[4 + 4 * k] << 16 |
                   (uint32_t) src[5 + 4 * k] << 24;
        uint4 * dst = reinterpret_cast<uint4 *>(q + bi * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        d[bi] = __ushort_as_half((unsigned short)(src[0] | src[1] << 8));
    }
}

bool Engine::upload_weights(const GgufFile & g) {
    const qtts_config & c = cfg;
    struct Need { std::string name; int rows, cols; bool matrix; };
    auto mat_bytes = [](const GgufTensor * t) -> size_t {
        const size_t n = (size_t) t->ne[0] * t->ne[1];
        return t->type == GGML_Q8_0 ? n + (n / 32) * 2 + 512 : t->nbytes + 256;
    };
    auto get = [&](const std::string & name, int ne0, int ne1, const GgufTensor *& out) -> bool {
        out = g.find(name);
        if (!out) { err = "missing tensor " + name; return false; }
        if (out->ne[0] != ne0 || out->ne[1] != ne1) { err = "unexpected shape for " + name; return false; }
        if (ne1 > 1 && out->type != GGML_F16 && out->type != GGML_Q8_0) {
            err = "unsupported weight type for " + name + " (F16 or Q8_0 expected)"; return false;
        }
        if (ne1 == 1 && out->type != GGML_F32) { err = "1-D tensor " + name + " must be F32"; return false; }
        return true;
    };
    // Pass 1: size.
    const int H = c.hidden_size, TD = c.text_embd_dim;
    std::vector<std::pair<std::string, std::pair<int, int>>> all;
    auto add = [&](const std::string & n, int ne0, int ne1) { all.push_back({n, {ne0, ne1}}); };
    add("talker.text_embd.weight", TD, c.text_vocab_size);
    add("talker.text_proj.fc1.weight", TD, TD);
    add("talker.text_proj.fc1.bias", TD, 1);
    add("talker.text_proj.fc2.weight", TD, H);
    add("talker.text_proj.fc2.bias", H, 1);
    add("talker.codec_embd.weight", H, c.codec_vocab_size);
    add("talker.codec_head.weight", H, c.codec_vocab_size);
    add("talker.output_norm.weight", H, 1);
    add("code_pred.output_norm.weight", H, 1);
    auto add_layers = [&](const char * pfx, int n, int ffn) {
        for (int i = 0; i < n; ++i) {
            std::string p = std::string(pfx) + std::to_string(i) + ".";
            add(p + "attn_norm.weight", H, 1);
            add(p + "attn_q.weight", H, QD());
            add(p + "attn_k.weight", H, KD());
            add(p + "attn_v.weight", H, KD());
            add(p + "attn_output.weight", QD(), H);
            add(p + "attn_q_norm.weight", QTTS_HD, 1);
            add(p + "attn_k_norm.weight", QTTS_HD, 1);
            add(p + "ffn_norm.weight", H, 1);
            add(p + "ffn_gate.weight", H, ffn);
            add(p + "ffn_up.weight", H, ffn);
            add(p + "ffn_down.weight", ffn, H);
        }
    };
    add_layers("talker.blk.", c.n_layers, c.intermediate_size);
    add_layers("code_pred.blk.", c.code_pred_layers, c.code_pred_intermediate_size);
    for (int gi = 0; gi < c.n_codebooks - 1; ++gi) {
        add("code_pred.codec_embd." + std::to_string(gi) + ".weight", H, c.code_pred_vocab_size);
        add("code_pred.lm_head." + std::to_string(gi) + ".weight", H, c.code_pred_vocab_size);
    }
    size_t total = 0;
    for (auto & n : all) {
        const GgufTensor * t;
        if (!get(n.first, n.second.first, n.second.second, t)) return false;
        total += mat_bytes(t);
    }
    for (auto & n : all)
        if (n.first.find("embd") != std::string::npos && g.find(n.first)->type != GGML_F16) {
            err = "embedding " + n.first + " must be F16"; return false;
        }
    QCHECK(cudaMalloc(&wbuf, total));
    wbytes = total; wused = 0;

    // The file mapping is registered as pinned host memory where the platform
    // allows it (read-only registration of a file mapping), so the uploads below
    // are direct DMA; otherwise the driver stages the pageable copies itself.
    // Q8_0 tensors go up as raw blocks and are split into planes on the device.
    const bool registered =
        cudaHostRegister(const_cast<uint8_t *>(g.map()), g.size(), cudaHostRegisterReadOnly) == cudaSuccess;
    if (!registered) cudaGetLastError();
    size_t q8_max = 0;
    for (auto & kv : g.tensors())
        if (kv.second.type == GGML_Q8_0) q8_max = std::max(q8_max, kv.second.nbytes);
    uint8_t * q8_stage = nullptr;
    if (q8_max && cudaMalloc(&q8_stage, q8_max) != cudaSuccess) { err = "alloc Q8_0 staging"; return false; }
    struct Cleanup {
        const GgufFile & g; bool reg; uint8_t * stage; cudaStream_t st;
        ~Cleanup() {
            cudaStreamSynchronize(st);
            if (stage) cudaFree(stage);
            if (reg) cudaHostUnregister(const_cast<uint8_t *>(g.map()));
        }
    } cleanup{g, registered, q8_stage, stream};
    auto alloc = [&](size_t bytes) -> uint8_t * {
        uint8_t * p = wbuf + wused;
        wused += (bytes + 255) & ~(size_t) 255;
        return p;
    };
    auto up_raw = [&](const GgufTensor * t) -> const void * {
        uint8_t * p = alloc(t->nbytes);
        if (cudaMemcpyAsync(p, t->data, t->nbytes, cudaMemcpyHostToDevice, stream) != cudaSuccess) return nullptr;
        return p;
    };
    // Matrix upload; several GGUF tensors may be stacked along rows (QKV fusion).
    auto up_mat = [&](std::initializer_list<const GgufTensor *> parts, DMat & m) -> bool {
        const GgufTensor * t0 = *parts.begin();
        m.type = t0->type == GGML_Q8_0 ? W_Q8_0 : W_F16;
        m.cols = (int) t0->ne[0];
        m.rows = 0;
        for (auto * t : parts) {
            if (t->type != t0->type || t->ne[0] != t0->ne[0]) { err = "mixed types in fused matrix " + t->name; return false; }
            m.rows += (int) t->ne[1];
        }
        if (m.type == W_F16) {
            uint8_t * p = alloc((size_t) m.rows * m.cols * 2);
            size_t off = 0;
            for (auto * t : parts) {
                if (cudaMemcpyAsync(p + off, t->data, t->nbytes, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
                    err = "upload failed"; return false;
                }
                off += t->nbytes;
            }
            m.w = p; m.d = nullptr;
        } else {
            const int nb = m.cols / 32;
            uint8_t * q = alloc((size_t) m.rows * m.cols);
            uint8_t * d = alloc((size_t) m.rows * nb * 2);
            size_t roff = 0;
            for (auto * t : parts) {
                const size_t rows = (size_t) t->ne[1], nblk = rows * nb;
                // stream order: this copy waits for the previous split's reads of the staging buffer
                if (cudaMemcpyAsync(q8_stage, t->data, t->nbytes, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
                    err = "upload failed"; return false;
                }
                k_split_q8<<<(unsigned) std::min<size_t>((nblk + 255) / 256, 4096), 256, 0, stream>>>(
                    q8_stage, nblk, reinterpret_cast<int8_t *>(q + roff * m.cols), reinterpret_cast<__half *>(d + roff * nb * 2));
                roff += rows;
            }
            m.w = q; m.d = reinterpret_cast<const __half *>(d);
        }
        return true;
    };
    auto T = [&](const std::string & n) { return g.find(n); };
    text_embd = (const __half *) up_raw(T("talker.text_embd.weight"));
    codec_embd = (const __half *) up_raw(T("talker.codec_embd.weight"));
    if (!up_mat({T("talker.text_proj.fc1.weight")}, fc1) || !up_mat({T("talker.text_proj.fc2.weight")}, fc2) ||
        !up_mat({T("talker.codec_head.weight")}, codec_head))
        return false;
    fc1_b = (const float *) up_raw(T("talker.text_proj.fc1.bias"));
    fc2_b = (const float *) up_raw(T("talker.text_proj.fc2.bias"));
    out_norm = (const float *) up_raw(T("talker.output_norm.weight"));
    cp_out_norm = (const float *) up_raw(T("code_pred.output_norm.weight"));
    auto load_layers = [&](const char * pfx, int n, std::vector<LayerW> & out) -> bool {
        out.resize(n);
        for (int i = 0; i < n; ++i) {
            std::string p = std::string(pfx) + std::to_string(i) + ".";
            LayerW & l = out[i];
            if (!up_mat({T(p + "attn_q.weight"), T(p + "attn_k.weight"), T(p + "attn_v.weight")}, l.qkv) ||
                !up_mat({T(p + "attn_output.weight")}, l.o) || !up_mat({T(p + "ffn_gate.weight")}, l.gate) ||
                !up_mat({T(p + "ffn_up.weight")}, l.up) || !up_mat({T(p + "ffn_down.weight")}, l.down))
                return false;
            if (l.gate.type != l.up.type) { err = "gate/up types differ"; return false; }
            l.attn_norm = (const float *) up_raw(T(p + "attn_norm.weight"));
            l.ffn_norm = (const float *) up_raw(T(p + "ffn_norm.weight"));
            l.q_norm = (const float *) up_raw(T(p + "attn_q_norm.weight"));
            l.k_norm = (const float *) up_raw(T(p + "attn_k_norm.weight"));
        }
        return true;
    };
    if (!load_layers("talker.blk.", c.n_layers, L) || !load_layers("code_pred.blk.", c.code_pred_layers, CPL)) return false;
    cp_embd.resize(c.n_codebooks - 1);
    cp_head.resize(c.n_codebooks - 1);
    for (int gi = 0; gi < c.n_codebooks - 1; ++gi) {
        cp_embd[gi] = (const __half *) up_raw(T("code_pred.codec_embd." + std::to_string(gi) + ".weight"));
        if (!up_mat({T("code_pred.lm_head." + std::to_string(gi) + ".weight")}, cp_head[gi])) return false;
    }
    cfg.weight_type = L[0].qkv.type;
    if (cudaStreamSynchronize(stream) != cudaSuccess || cudaGetLastError() != cudaSuccess) { err = "weight upload failed"; return false; }
    QCHECK(cudaMalloc(&d_cp_embd, sizeof(void *) * cp_embd.size()));
    QCHECK(cudaMemcpy(d_cp_embd, cp_embd.data(), sizeof(void *) * cp_embd.size(), cudaMemcpyHostToDevice));
    if (wused > wbytes) { err = "weight arena overflow"; return false; }
    return true;
}

bool Engine::alloc_activations() {
    const qtts_config & c = cfg;
    const int H = c.hidden_size, NV = QTTS_MAX_NV;
    const int FF = std::max(c.intermediate_size, c.code_pred_intermediate_size);
    QCHECK(cudaMalloc(&x, sizeof(float) * NV * H));
    QCHECK(cudaMalloc(&xcp, sizeof(float) * 2 * H));
    QCHECK(cudaMalloc(&qkv, sizeof(float) * NV * QKVD()));
    QCHECK(cudaMalloc(&att, sizeof(float) * NV * QD()));
    QCHECK(cudaMalloc(&hbuf, sizeof(float) * NV * std::max(FF, c.text_embd_dim)));
    QCHECK(cudaMalloc(&logits, sizeof(float) * c.codec_vocab_size));
    QCHECK(cudaMalloc(&cp_logits, sizeof(float) * c.code_pred_vocab_size * (c.n_codebooks - 1)));
    QCHECK(cudaMalloc(&hidden, sizeof(float) * H));
    QCHECK(cudaMalloc(&logits0, sizeof(float) * c.codec_vocab_size));
    QCHECK(cudaMalloc(&hidden0, sizeof(float) * H));
    QCHECK(cudaMalloc(&tmp_a, sizeof(float) * NV * std::max(H, c.text_embd_dim)));
    QCHECK(cudaMalloc(&tmp_b, sizeof(float) * NV * std::max(H, c.text_embd_dim)));
    QCHECK(cudaMalloc(&st, sizeof(DevState)));
    QCHECK(cudaMemset(st, 0, sizeof(DevState)));
    QCHECK(cudaMalloc(&sp, sizeof(SampleParams)));
    QCHECK(cudaMemset(sp, 0, sizeof(SampleParams)));
    QCHECK(cudaMalloc(&pad, sizeof(float) * H));
    ids_cap = 4096;
    QCHECK(cudaMalloc(&d_ids, sizeof(int) * ids_cap));
    // large dynamic shared memory for the GEMV instantiations
    QCHECK(cudaFuncSetAttribute(k_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX));
    QCHECK(cudaFuncSetAttribute(k_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX));
    QCHECK(cudaFuncSetAttribute(k_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX));
    QCHECK(cudaFuncSetAttribute(k_fused_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    // The GEMV grid is two 512-thread CTAs per SM.  At 40 registers or fewer a
    // third CTA would fit and the block scheduler packs three onto some SMs
    // (measured 15 % slower per frame); should the kernel ever compile that
    // small, a shared-memory floor keeps the residency at two.
    int nb = 0, smem_sm = 0;
    QCHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_gemv<1>, QTTS_WARPS * 32, 0));
    QCHECK(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    gemv_smem_floor = nb > 2 ? (size_t) smem_sm / 3 + 1024 : 0;
    return true;
}

bool Engine::init_kv(int ctx) {
    if (ctx <= 0) { err = "n_ctx must be > 0"; return false; }
    const qtts_config & c = cfg;
    if (kc) { cudaFree(kc); kc = nullptr; }
    if (vc) { cudaFree(vc); vc = nullptr; }
    if (rope_t) { cudaFree(rope_t); rope_t = nullptr; }
    const size_t per = (size_t) c.n_layers * ctx * c.n_key_value_heads * QTTS_HD;
    QCHECK(cudaMalloc(&kc, per * sizeof(__half)));
    QCHECK(cudaMalloc(&vc, per * sizeof(__half)));
    std::vector<float2> t;
    build_rope(t, ctx, c.rope_theta);
    QCHECK(cudaMalloc(&rope_t, t.size() * sizeof(float2)));
    QCHECK(cudaMemcpy(rope_t, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
    const size_t smem = attn_smem_bytes(ctx, c.n_attention_heads / c.n_key_value_heads);
    if (smem > 220 * 1024) { err = "context too long for the attention kernel"; return false; }
    QCHECK(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) std::max<size_t>(smem, 48 * 1024)));
    n_ctx = ctx;
    n_used = 0;
    graph_ok = false;
    return true;
}

bool Engine::init_cp_kv(int ctx) {
    const qtts_config & c = cfg;
    if (ctx < 16) ctx = 16;
    if (cpk) { cudaFree(cpk); cpk = nullptr; }
    if (cpv) { cudaFree(cpv); cpv = nullptr; }
    if (rope_cp) { cudaFree(rope_cp); rope_cp = nullptr; }
    const size_t per = (size_t) c.code_pred_layers * ctx * c.n_key_value_heads * QTTS_HD;
    QCHECK(cudaMalloc(&cpk, per * sizeof(__half)));
    QCHECK(cudaMalloc(&cpv, per * sizeof(__half)));
    std::vector<float2> t;
    build_rope(t, ctx, c.code_pred_rope_theta);
    QCHECK(cudaMalloc(&rope_cp, t.size() * sizeof(float2)));
    QCHECK(cudaMemcpy(rope_cp, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
    cp_ctx = ctx;
    graph_ok = false;
    return true;
}

// Waits for the engine stream with a time limit (QTTS_SYNC_TIMEOUT_S, default
// 300 s): a stream that never drains is reported as an error instead of
// blocking the caller forever.
bool Engine::sync(const char * what) {
    static const double limit_s = [] {
        const char * v = getenv("QTTS_SYNC_TIMEOUT_S");
        return v && *v ? atof(v) : 300.0;
    }();
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e;
    int spins = 0;
    while ((e = cudaStreamQuery(stream)) == cudaErrorNotReady) {
        if (++spins > 1000) std::this_thread::sleep_for(std::chrono::microseconds(50));
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit_s) {
            err = std::string(what) + ": GPU work did not complete within the sync time limit";
            return false;
        }
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { err = std::string(what) + ": " + cudaGetErrorString(e); return false; }
    return true;
}

// ---------------------------------------------------------------- launches
// Grid and shared memory of a stand-alone k_gemv launch: one CTA per SM while
// its weight slice and work area fit, more CTAs (smaller slices) otherwise.
static bool gemv_shape(const DMat & A, bool dual, bool has_gain, int nvt, int n_sm, int * ncta_out, size_t * slice_out,
                       size_t * smem_out) {
    int ncta = std::min(2 * n_sm, A.rows);   // two CTAs per SM: half the rows each, and room for the next kernel under PDL
    for (;;) {
        const int rpc = gemv_rpc(A.rows, ncta);
        const size_t slice = (slice_layout(A, dual, has_gain, rpc).total + 127) & ~(size_t) 127;
        const size_t smem = slice + gemv_work_bytes(A.type, A.cols, nvt, rpc);
        if (smem <= QTTS_GEMV_SMEM_MAX) {
            *ncta_out = (A.rows + rpc - 1) / rpc;
            *slice_out = slice;
            *smem_out = smem;
            return true;
        }
        if (ncta >= A.rows) return false;
        ncta = std::min(A.rows, ncta * 2);
    }
}

GemvArgs Engine::make_gemv(const DMat & A, const DMat * B, const float * xin, int ldx, int nv, const float * norm,
                           int act, float * y, int ldy, const float * resid, int ldr, int epi, float * xn_out,
                           int ldxn, const int * done, int * ncta_out, size_t * slice_out, size_t * smem_out) {
    GemvArgs a{};
    a.A = A;
    if (B) a.B = *B;
    a.x = xin; a.ldx = ldx; a.nv = nv;
    a.norm_g = norm; a.eps = cfg.rms_norm_eps; a.act = act;
    a.y = y; a.ldy = ldy; a.resid = resid; a.ldr = ldr; a.epi = epi;
    a.xn_out = xn_out; a.ldxn = ldxn; a.done = done;
    const int NVt = nv == 1 ? 1 : nv == 2 ? 2 : 8;
    if (!gemv_shape(A, B != nullptr, norm != nullptr, NVt, n_sm, ncta_out, slice_out, smem_out)) *ncta_out = 0;
    *smem_out = std::max(*smem_out, gemv_smem_floor);
    return a;
}

bool Engine::gemv(const DMat & A, const DMat * B, const float * xin, int ldx, int nv, const float * norm, int act,
                  float * y, int ldy, const float * resid, int ldr, int epi, float * xn_out, int ldxn,
                  const int * done) {
    int ncta;
    size_t slice, smem;
    GemvArgs a = make_gemv(A, B, xin, ldx, nv, norm, act, y, ldy, resid, ldr, epi, xn_out, ldxn, done, &ncta, &slice,
                           &smem);
    const int NVt = nv == 1 ? 1 : nv == 2 ? 2 : 8;
    if (nv > QTTS_MAX_NV || ncta == 0) { err = "gemv shape too large"; return false; }
    const double wb = A.type == W_F16 ? (double) A.rows * A.cols * 2.0 : (double) A.rows * A.cols * 34.0 / 32.0;
    prof_begin(KC_GEMV, wb * (B ? 2.0 : 1.0) + 4.0 * nv * ((double) A.cols + A.rows));
    if (NVt == 1) pdl_launch(k_gemv<1>, dim3(ncta), dim3(QTTS_WARPS * 32), smem, stream, a, slice);
    else if (NVt == 2) pdl_launch(k_gemv<2>, dim3(ncta), dim3(QTTS_WARPS * 32), smem, stream, a, slice);
    else pdl_launch(k_gemv<8>, dim3(ncta), dim3(QTTS_WARPS * 32), smem, stream, a, slice);
    prof_end();
    ++launches;
    return true;
}

FusedAttn Engine::fused_attn_args(const LayerW & l, __half * kc_l, __half * vc_l, const float2 * rope, int M,
                                  const int * pos_ptr, int pos_static, bool f32, float * dump, int dump_stride) {
    const qtts_config & c = cfg;
    FusedAttn a{};
    a.qkv = qkv; a.ldq = QKVD(); a.n_heads = c.n_attention_heads; a.n_kv_heads = c.n_key_value_heads;
    a.q_norm = l.q_norm; a.k_norm = l.k_norm; a.eps = c.rms_norm_eps; a.rope = rope;
    a.kc = kc_l; a.vc = vc_l;
    a.pos_ptr = pos_ptr; a.pos_static = pos_static; a.M = M; a.f32_mode = f32 ? 1 : 0;
    a.scale = 1.0f / sqrtf((float) QTTS_HD); a.out = att; a.ldo = QD();
    a.dump = dump; a.dump_stride = dump_stride;
    return a;
}

// Prefill attention over M rows (chunks of the prompt): q/k norm + RoPE + F16
// KV append for the rows, then causal attention over the cache.  q: the
// rows' q|k|v [M][ldq]; out: [M][ldo].
void Engine::prefill_attention(const LayerW & l, __half * kc_l, __half * vc_l, const float2 * rope, const float * q,
                               int ldq, int M, const int * pos_ptr, int pos_static, const int * done, float * out,
                               int ldo, float * dump, int dump_stride, size_t smem) {
    const qtts_config & c = cfg;
    const int NH = c.n_attention_heads, NKV = c.n_key_value_heads;
    QkArgs qa{};
    qa.qkv = const_cast<float *>(q); qa.ldq = ldq; qa.n_heads = NH; qa.n_kv_heads = NKV;
    qa.q_norm = l.q_norm; qa.k_norm = l.k_norm; qa.eps = c.rms_norm_eps; qa.rope = rope;
    qa.kc = kc_l; qa.vc = vc_l;
    qa.pos_ptr = pos_ptr; qa.pos_static = pos_static; qa.keep_f32_k = 0; qa.done = done;
    prof_begin(KC_OTHER, 0.0);
    k_qk_rope_store<<<M, 32 * (NH + NKV), 0, stream>>>(qa);
    prof_end();
    ++launches;
    AttnArgs aa{};
    aa.q = q; aa.ldq = ldq; aa.kc = kc_l; aa.vc = vc_l;
    aa.kf = q + QD(); aa.vf = q + QD() + KD(); aa.ldkv = ldq; aa.f32_mode = 0;
    aa.n_heads = NH; aa.n_kv_heads = NKV; aa.pos_ptr = pos_ptr; aa.pos_static = pos_static;
    aa.scale = 1.0f / sqrtf((float) QTTS_HD);
    aa.out = out; aa.ldo = ldo; aa.done = done;
    aa.dump = dump; aa.dump_stride = dump_stride; aa.st = st;
    prof_begin(KC_ATTN, 0.0);
    k_attention<<<dim3(NKV, M), ATT_THREADS, smem, stream>>>(aa);
    prof_end();
    ++launches;
}

bool Engine::layers(std::vector<LayerW> & Ls, __half * kbase, __half * vbase, int ctx, const float2 * rope, float * X,
                    int M, const int * pos_ptr, int pos_static, bool f32_mode, const int * done, int ffn,
                    float * dump, int dump_layer) {
    const qtts_config & c = cfg;
    const int H = c.hidden_size, NH = c.n_attention_heads, NKV = c.n_key_value_heads;
    const int G = NH / NKV;
    const size_t layer_elems = (size_t) ctx * NKV * QTTS_HD;
    const size_t att_smem = attn_smem_bytes(f32_mode ? M : ctx, G);
    // code-predictor steps (one row, at most 16 keys from the cache): one warp per query head
    const bool cp_step = &Ls == &CPL && M == 1 && !f32_mode && !pos_ptr;
    if (cp_step && pos_static + 1 > CPA_MAX_KEYS) { err = "code-predictor step beyond 16 positions"; return false; }
    for (size_t il = 0; il < Ls.size(); ++il) {
        LayerW & l = Ls[il];
        if (!gemv(l.qkv, nullptr, X, H, M, l.attn_norm, ACT_F16, qkv, QKVD(), nullptr, 0, EPI_STORE, nullptr, 0, done))
            return false;
        if (cp_step) {
            FusedAttn fa = fused_attn_args(l, kbase + il * layer_elems, vbase + il * layer_elems, rope, 1, nullptr,
                                           pos_static, false, nullptr, ctx);
            fa.done = done;
            prof_begin(KC_ATTN, 0.0);
            pdl_launch(k_cp_step_attn, dim3(NH), dim3(32), 0, stream, fa);
            prof_end();
            ++launches;
        } else if (f32_mode || M == 1) {
            // frame steps and the code-predictor 2-token prefill: one fused unit per (kv head, row)
            FusedAttn fa = fused_attn_args(l, kbase + il * layer_elems, vbase + il * layer_elems, rope, M, pos_ptr,
                                           pos_static, f32_mode, ((int) il == dump_layer) ? dump : nullptr, ctx);
            fa.done = done;
            const size_t fsm = fused_attn_smem(f32_mode ? M : ctx, M);
            if (fsm > 200 * 1024) { err = "context too long for the fused attention kernel"; return false; }
            prof_begin(KC_ATTN, 0.0);
            pdl_launch(k_fused_attention, dim3(NH * M), dim3(FA_THREADS), fsm, stream, fa, (const DevState *) st);
            prof_end();
            ++launches;
        } else {
            prefill_attention(l, kbase + il * layer_elems, vbase + il * layer_elems, rope, qkv, QKVD(), M, pos_ptr,
                              pos_static, done, att, QD(), ((int) il == dump_layer) ? dump : nullptr, ctx, att_smem);
        }
        if (!gemv(l.o, nullptr, att, QD(), M, nullptr, ACT_F16, X, H, X, H, EPI_RESID, nullptr, 0, done)) return false;
        if (!gemv(l.gate, &l.up, X, H, M, l.ffn_norm, ACT_F16, hbuf, ffn, nullptr, 0, EPI_SWIGLU, nullptr, 0, done))
            return false;
        // ffn_down: F16 weights are cast to F32 by the reference (F32 x F32 mul_mat)
        if (!gemv(l.down, nullptr, hbuf, ffn, M, nullptr, ACT_F32, X, H, X, H, EPI_RESID, nullptr, 0, done)) return false;
    }
    return true;
}

// Code predictor for the current frame state: 2-token prefill, head 0, then 14
// single-token steps.  Each sampler also builds the next pass's input rows
// (k_sample_inputs); last_in: the inputs after the last code-predictor sampler
// (the next talker step), or nullptr for a plain sampler.
bool Engine::enqueue_cp(bool sample_cb0, const InputArgs * last_in) {
    const qtts_config & c = cfg;
    prof_stage = STG_CP;
    const int H = c.hidden_size, V1 = c.code_pred_vocab_size, NG = c.n_codebooks - 1;
    const int * done = &st->done;
    InputArgs ia{};
    ia.H = H; ia.codec_embd = codec_embd; ia.cp_embd = d_cp_embd; ia.hidden = hidden;
    ia.trailing = trailing; ia.pad = pad; ia.out = xcp; ia.st = st; ia.n_cb = c.n_codebooks;
    ia.mode = IN_CP_PREFILL;
    auto sample = [&](const float * lg, int V, int cb, const InputArgs * in) {
        prof_begin(KC_SAMPLE, 0.0);
        if (in)
            pdl_launch(k_sample_inputs, dim3(1), dim3(SAMPLE_THREADS), 0, stream, lg, V, cb, st,
                       (const SampleParams *) sp, d_codes, codes_cap, *in);
        else
            pdl_launch(k_sample, dim3(1), dim3(SAMPLE_THREADS), 0, stream, lg, V, cb, st, (const SampleParams *) sp,
                       d_codes, codes_cap);
        prof_end();
        ++launches;
    };
    if (sample_cb0) {
        sample(logits, c.codec_vocab_size, 0, &ia);
    } else {
        pdl_launch(k_frame_inputs, dim3(1), dim3(256), 0, stream, ia);
        ++launches;
    }
    if (!layers(CPL, cpk, cpv, cp_ctx, rope_cp, xcp, 2, nullptr, 0, true, done, c.code_pred_intermediate_size)) return false;
    if (!gemv(cp_head[0], nullptr, xcp + H, H, 1, cp_out_norm, ACT_F16, cp_logits, V1, nullptr, 0, EPI_STORE, nullptr, 0, done))
        return false;
    for (int gstep = 1; gstep < NG; ++gstep) {
        ia.mode = IN_CP_STEP; ia.g = gstep; ia.step_tab = cp_embd[gstep - 1];
        sample(cp_logits, V1, gstep, &ia);   // codebook gstep, then the step's input row
        if (!layers(CPL, cpk, cpv, cp_ctx, rope_cp, xcp, 1, nullptr, gstep + 1, false, done, c.code_pred_intermediate_size))
            return false;
        if (!gemv(cp_head[gstep], nullptr, xcp, H, 1, cp_out_norm, ACT_F16, cp_logits, V1, nullptr, 0, EPI_STORE, nullptr, 0, done))
            return false;
    }
    sample(cp_logits, V1, NG, last_in);
    return true;
}

bool Engine::enqueue_talker_step(const int * pos_ptr, int pos_static, const int * done, bool with_dump) {
    const qtts_config & c = cfg;
    prof_stage = STG_TALKER;
    const int H = c.hidden_size;
    if (!layers(L, kc, vc, n_ctx, rope_t, x, 1, pos_ptr, pos_static, false, done, c.intermediate_size,
                with_dump && attn_dump ? d_attn : nullptr, attn_layer))
        return false;
    return gemv(codec_head, nullptr, x, H, 1, out_norm, ACT_F16, logits, c.codec_vocab_size, nullptr, 0, EPI_STORE,
                hidden, H, done);
}

bool Engine::enqueue_frame() {
    InputArgs ia{};
    ia.H = cfg.hidden_size; ia.codec_embd = codec_embd; ia.cp_embd = d_cp_embd; ia.hidden = hidden;
    ia.trailing = trailing; ia.pad = pad; ia.out = x; ia.st = st; ia.n_cb = cfg.n_codebooks;
    ia.mode = IN_TALKER;
    if (!enqueue_cp(true, &ia)) return false;
    if (!enqueue_talker_step(&st->pos, 0, &st->done, true)) return false;
    pdl_launch(k_frame_end, dim3(1), dim3(32), 0, stream, st);
    ++launches;
    return true;
}

bool Engine::capture_graph() {
    if (graph) { cudaGraphExecDestroy(graph); graph = nullptr; }
    cudaGraph_t gr = nullptr;
    QCHECK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    launches = 0;
    const bool ok = frame_mode == FM_FUSED ? enqueue_frame_ff() : enqueue_frame();
    cudaError_t ce = cudaStreamEndCapture(stream, &gr);
    if (!ok) { if (gr) cudaGraphDestroy(gr); return false; }
    if (ce != cudaSuccess) { err = std::string("graph capture: ") + cudaGetErrorString(ce); return false; }
    launches_per_frame = launches;
    ce = cudaGraphInstantiate(&graph, gr, 0);
    cudaGraphDestroy(gr);
    if (ce != cudaSuccess) { err = std::string("graph instantiate: ") + cudaGetErrorString(ce); return false; }
    graph_ok = true;
    return true;
}

// ---------------------------------------------------------------- fused frame path
static size_t ff_attn_smem(const DMat & qkv, const DMat & o, int H, int rows_g, int GD, int CA, int nv, int keys);
// Repacked weights (group-major q|k|v and O, ffn_down in the FFN block's slice
// order), partial-sum buffers and launch shapes of FM_FUSED.  Leaves frame_mode
// at FM_GRAPH, with the reason in ff_why, when the model's shapes do not fit.
bool Engine::ff_prepare() {
    const qtts_config & c = cfg;
    const int H = c.hidden_size, NH = c.n_attention_heads, NKV = c.n_key_value_heads;
    const int G = NH / NKV, GD = G * QTTS_HD, rows_g = GD + 2 * QTTS_HD, QD = NH * QTTS_HD;
    const bool q8 = L[0].qkv.type == W_Q8_0;
    const size_t es = q8 ? 1 : 2;
    auto stack = [&](int I, FfStack & S) -> bool {
        S.R = q8 ? 32 : 16;
        if (I % S.R) return false;
        S.N = I / S.R;
        S.C = FF_MAX_CLUSTER;
        while (S.C > 1 && (S.N % S.C || H % S.C)) S.C /= 2;
        return true;
    };
    ff_why.clear();
    if (!stack(c.intermediate_size, ffs_t) || !stack(c.code_pred_intermediate_size, ffs_cp)) ff_why = "ffn width";
    else if (rows_g % ff_CA || H % ff_CA || GD % 32) ff_why = "head layout";
    else if (c.n_codebooks > QTTS_MAX_CB || c.codec_vocab_size > 4096 || c.code_pred_vocab_size > 4096) ff_why = "vocabulary";
    else {
        for (auto * Ls : {&L, &CPL})
            for (auto & l : *Ls)
                if (l.qkv.type != l.o.type || l.o.type != l.down.type || l.gate.type != l.down.type) ff_why = "mixed weight types";
    }
    if (ff_why.empty() && (NKV > FF_MAX_PART || ffs_t.N / ffs_t.C > FF_MAX_PART || ffs_cp.N / ffs_cp.C > FF_MAX_PART))
        ff_why = "too many partial vectors";
    if (!ff_why.empty()) return true;
    // repacked copies
    auto mat_size = [&](const DMat & m) { return (size_t) m.rows * m.cols * es + (q8 ? (size_t) m.rows * (m.cols / 32) * 2 : 0); };
    size_t total = 0;
    for (auto * Ls : {&L, &CPL})
        for (auto & l : *Ls) total += mat_size(l.qkv) + mat_size(l.o) + mat_size(l.down) + 6 * 256;
    QCHECK(cudaMalloc(&ffw, total));
    size_t used = 0;
    auto alloc = [&](size_t b) { uint8_t * p = ffw + used; used += (b + 255) & ~(size_t) 255; return p; };
    auto fresh = [&](const DMat & src, int rows, int cols) {
        DMat m = src;
        m.rows = rows; m.cols = cols;
        m.w = alloc((size_t) rows * cols * es);
        m.d = q8 ? reinterpret_cast<const __half *>(alloc((size_t) rows * (cols / 32) * 2)) : nullptr;
        return m;
    };
    auto copy_rows = [&](const DMat & dst, int dr, const DMat & src, int sr, int n) -> bool {
        const size_t rb = (size_t) src.cols * es;
        if (cudaMemcpy((uint8_t *) dst.w + dr * rb, (const uint8_t *) src.w + sr * rb, n * rb, cudaMemcpyDeviceToDevice) != cudaSuccess) return false;
        if (q8) {
            const size_t sb = (size_t)(src.cols / 32) * 2;
            if (cudaMemcpy((uint8_t *) dst.d + dr * sb, (const uint8_t *) src.d + sr * sb, n * sb, cudaMemcpyDeviceToDevice) != cudaSuccess) return false;
        }
        return true;
    };
    for (int which = 0; which < 2; ++which) {
        std::vector<LayerW> & Ls = which ? CPL : L;
        std::vector<FfLayerW> & F = which ? ffCP : ffL;
        F.resize(Ls.size());
        for (size_t il = 0; il < Ls.size(); ++il) {
            const LayerW & l = Ls[il];
            FfLayerW & f = F[il];
            f.qkv_g = fresh(l.qkv, NKV * rows_g, H);
            f.o_g = fresh(l.o, NKV * H, GD);
            f.down_r = fresh(l.down, l.down.rows, l.down.cols);
            for (int g = 0; g < NKV; ++g) {
                const int d0 = g * rows_g;
                if (!copy_rows(f.qkv_g, d0, l.qkv, g * GD, GD) ||
                    !copy_rows(f.qkv_g, d0 + GD, l.qkv, QD + g * QTTS_HD, QTTS_HD) ||
                    !copy_rows(f.qkv_g, d0 + GD + QTTS_HD, l.qkv, QD + NKV * QTTS_HD + g * QTTS_HD, QTTS_HD)) {
                    err = "fused path: q|k|v regroup failed"; return false;
                }
                QCHECK(cudaMemcpy2D((uint8_t *) f.o_g.w + (size_t) g * H * GD * es, GD * es,
                                    (const uint8_t *) l.o.w + (size_t) g * GD * es, (size_t) QD * es, GD * es, H,
                                    cudaMemcpyDeviceToDevice));
                if (q8)
                    QCHECK(cudaMemcpy2D((uint8_t *) f.o_g.d + (size_t) g * H * (GD / 32) * 2, (GD / 32) * 2,
                                        (const uint8_t *) l.o.d + (size_t)(g * GD / 32) * 2, (size_t)(QD / 32) * 2,
                                        (GD / 32) * 2, H, cudaMemcpyDeviceToDevice));
            }
            k_ff_repack_down<<<1024, 256, 0, stream>>>(l.down, const_cast<void *>(f.down_r.w), const_cast<__half *>(f.down_r.d));
        }
    }
    QCHECK(cudaGetLastError());
    QCHECK(cudaStreamSynchronize(stream));
    const int ncl = std::max(ffs_t.N / ffs_t.C, ffs_cp.N / ffs_cp.C);
    QCHECK(cudaMalloc(&ff_part_o, sizeof(float) * NKV * 2 * H));
    QCHECK(cudaMalloc(&ff_part_d, sizeof(float) * ncl * 2 * H));
    QCHECK(cudaMalloc(&ff_xres, sizeof(float) * 2 * H));
    QCHECK(cudaMalloc(&ff_xmid, sizeof(float) * 2 * H));
    if (!d_err) QCHECK(cudaMalloc(&d_err, sizeof(int)));
    QCHECK(cudaMemset(d_err, 0, sizeof(int)));
    for (auto fn : {(const void *) k_ff_attn<1>, (const void *) k_ff_attn<2>, (const void *) k_ff_ffn<1>,
                    (const void *) k_ff_ffn<2>}) {
        QCHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        QCHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    }
    QCHECK(cudaFuncSetAttribute(k_ff_head, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX));
    if (const char * v = getenv("QTTS_FF_PF")) ff_pf_ahead = std::max(0, atoi(v));
    if (getenv("QTTS_FF_TRACE")) {
        const size_t n = (size_t) 256 * FF_TRACE_CTAS * FF_TRACE_N;
        QCHECK(cudaMalloc(&d_fftrace, n * sizeof(unsigned long long)));
        QCHECK(cudaMemset(d_fftrace, 0, n * sizeof(unsigned long long)));
    }
    // attention block: the largest cluster (CTAs per kv group) whose NKV clusters are
    // resident together at the talker's shared-memory size for 4096-key rows
    ff_CA = 0;
    for (int ca = FF_MAX_CLUSTER; ca >= 2 && !ff_CA; ca /= 2) {
        if (rows_g % ca || H % ca) continue;
        cudaLaunchConfig_t cl{};
        cl.gridDim = dim3(NKV * ca);
        cl.blockDim = dim3(FF_THREADS);
        cl.dynamicSmemBytes = ff_attn_smem(L[0].qkv, L[0].o, H, rows_g, GD, ca, 2, 4096);
        cudaLaunchAttribute at{};
        at.id = cudaLaunchAttributeClusterDimension;
        at.val.clusterDim.x = (unsigned) ca; at.val.clusterDim.y = 1; at.val.clusterDim.z = 1;
        cl.attrs = &at;
        cl.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_ff_attn<2>, &cl) == cudaSuccess && n >= NKV) ff_CA = ca;
        cudaGetLastError();
    }
    if (!ff_CA) { ff_why = "attention-block clusters do not fit"; return true; }
    frame_mode = FM_FUSED;
    return true;
}

// Shared-memory bytes of the two clustered kernels.
static size_t ff_attn_smem(const DMat & qkv, const DMat & o, int H, int rows_g, int GD, int CA, int nv, int keys) {
    DMat Qg = qkv; Qg.rows = rows_g; Qg.cols = H;
    DMat Og = o; Og.rows = H; Og.cols = GD;
    const size_t wq = (slice_layout(Qg, false, true, rows_g / CA).total + 127) & ~(size_t) 127;
    const size_t wo = (slice_layout(Og, false, false, H / CA).total + 127) & ~(size_t) 127;
    size_t work = std::max(gemv_work_bytes(qkv.type, H, nv, rows_g / CA), gemv_work_bytes(o.type, GD, nv, H / CA));
    work = std::max(work, fused_attn_smem(keys, nv));
    return std::max(wq, wo) + ((work + 127) & ~(size_t) 127);
}
static size_t ff_ffn_work(int type, int H, int nv, int R) {
    return (std::max(gemv_work_bytes(type, H, nv, R), (size_t) nv * H * 4) + 127) & ~(size_t) 127;
}
static size_t ff_ffn_smem(const DMat & gate, const DMat & down, int H, int nv, int R) {
    const size_t wb_gu = (slice_layout(gate, true, true, R).total + 127) & ~(size_t) 127;
    const size_t wb_dn = (ff_down_slice_bytes(down.type, R, H) + 127) & ~(size_t) 127;
    return wb_gu + wb_dn + ff_ffn_work(down.type, H, nv, R) + (size_t) nv * R * 4;
}

namespace {
struct FfLaunch {
    int kind;                      // 0 attention block, 1 FFN block, 2 head
    int nv, grid, cluster, stage;
    bool samples;                  // the launch samples the pass's codebook in its prologue
    size_t smem;
    double bytes;
    FfAttnArgs a;
    FfFfnArgs f;
    FfHeadArgs h;
    std::vector<std::pair<const void *, size_t>> w;   // weight regions (prefetched by earlier launches)
};
void ff_regions(std::vector<std::pair<const void *, size_t>> & w, const DMat & m) {
    const size_t es = m.type == W_Q8_0 ? 1 : 2;
    w.push_back({m.w, (size_t) m.rows * m.cols * es});
    if (m.type == W_Q8_0) w.push_back({m.d, (size_t) m.rows * (m.cols / 32) * 2});
}
}  // namespace

// The frame as clustered launches: the code-predictor passes (pass 0 samples
// codebook 0 from the talker logits, pass g codebook g), then the talker step
// (its first layer samples the last codebook) and the codec head, which also
// advances the frame state.
bool Engine::enqueue_frame_ff() {
    const qtts_config & c = cfg;
    const int H = c.hidden_size, NH = c.n_attention_heads, NKV = c.n_key_value_heads;
    const int G = NH / NKV, GD = G * QTTS_HD, rows_g = GD + 2 * QTTS_HD, NG = c.n_codebooks - 1;
    const int V1 = c.code_pred_vocab_size;
    FfFrame fr{};
    fr.st = st; fr.err = d_err; fr.sp = sp; fr.out_codes = d_codes; fr.out_cap = codes_cap;
    fr.codec_embd = codec_embd; fr.cp_embd = d_cp_embd; fr.hidden = hidden; fr.trailing = trailing; fr.pad = pad;
    fr.H = H; fr.n_cb = c.n_codebooks; fr.V0 = c.codec_vocab_size; fr.V1 = V1; fr.eps = c.rms_norm_eps;
    fr.trace = d_fftrace; fr.trace_frame = 1;
    std::vector<FfLaunch> Ls;
    const size_t cp_layer = (size_t) cp_ctx * NKV * QTTS_HD, t_layer = (size_t) n_ctx * NKV * QTTS_HD;
    const double es = L[0].qkv.type == W_Q8_0 ? 34.0 / 32.0 : 2.0;
    // one stack (code-predictor pass or talker step); in_mode/cb: the first layer's sampler
    auto stack = [&](bool cp, int pass, int in_mode, int cb, const float * in_logits) {
        std::vector<LayerW> & LW = cp ? CPL : L;
        std::vector<FfLayerW> & FW = cp ? ffCP : ffL;
        const FfStack & S = cp ? ffs_cp : ffs_t;
        const int nv = cp && pass == 0 ? 2 : 1;
        for (size_t il = 0; il < LW.size(); ++il) {
            const LayerW & l = LW[il];
            FfLaunch A{};
            A.kind = 0; A.nv = nv; A.grid = NKV * ff_CA; A.cluster = ff_CA; A.stage = cp ? STG_CP : STG_TALKER;
            A.samples = il == 0;
            FfAttnArgs & a = A.a;
            a.fr = fr;
            if (il == 0) { a.in.mode = in_mode; a.in.cb = cb; a.in.logits = in_logits; }
            else { a.in.mode = FIN_PART; a.in.base = ff_xmid; a.in.part = ff_part_d; a.in.np = S.N / S.C; }
            a.in.x_out = ff_xres;
            a.nv = nv; a.qkv = FW[il].qkv_g; a.attn_norm = l.attn_norm; a.o = FW[il].o_g;
            a.qkv_buf = qkv; a.att_buf = att; a.part_out = ff_part_o;
            if (cp) {
                a.att = fused_attn_args(l, cpk + il * cp_layer, cpv + il * cp_layer, rope_cp, nv, nullptr,
                                        pass == 0 ? 0 : pass + 1, pass == 0, nullptr, cp_ctx);
                a.att_kind = pass == 0 ? FF_ATT_UNIT : FF_ATT_CPSTEP;
                a.n_past = pass == 0 ? 0 : pass + 1;
            } else {
                a.att = fused_attn_args(l, kc + il * t_layer, vc + il * t_layer, rope_t, 1, &st->pos, 0, false,
                                        attn_dump && (int) il == attn_layer ? d_attn : nullptr, n_ctx);
                a.att_kind = FF_ATT_UNIT;
            }
            A.smem = ff_attn_smem(l.qkv, l.o, H, rows_g, GD, ff_CA, nv, cp ? 2 : ff_max_keys);
            a.work_bytes = 0;
            A.bytes = es * ((double) l.qkv.rows * l.qkv.cols + (double) l.o.rows * l.o.cols);
            ff_regions(A.w, FW[il].qkv_g);
            ff_regions(A.w, FW[il].o_g);
            Ls.push_back(A);
            FfLaunch B{};
            B.kind = 1; B.nv = nv; B.grid = S.N; B.cluster = S.C; B.stage = A.stage;
            FfFfnArgs & f = B.f;
            f.fr = fr;
            f.in.mode = FIN_PART; f.in.base = ff_xres; f.in.part = ff_part_o; f.in.np = NKV; f.in.x_out = ff_xmid;
            f.nv = nv; f.gate = l.gate; f.up = l.up; f.ffn_norm = l.ffn_norm; f.down = FW[il].down_r; f.R = S.R;
            f.part_out = ff_part_d;
            f.set_presence = cp && pass == 0 && il == 0;
            f.work_bytes = (int) ff_ffn_work(l.down.type, H, nv, S.R);
            B.smem = ff_ffn_smem(l.gate, l.down, H, nv, S.R);
            B.bytes = es * 3.0 * (double) l.gate.rows * l.gate.cols;
            ff_regions(B.w, l.gate);
            ff_regions(B.w, l.up);
            ff_regions(B.w, FW[il].down_r);
            Ls.push_back(B);
        }
        FfLaunch Hd{};
        Hd.kind = 2; Hd.nv = 1; Hd.cluster = 1; Hd.stage = cp ? STG_CP : STG_TALKER;
        FfHeadArgs & h = Hd.h;
        const DMat & hm = cp ? cp_head[pass] : codec_head;
        int ncta = 0;
        size_t slice = 0, smem = 0;
        h.g = make_gemv(hm, nullptr, nullptr, H, 1, cp ? cp_out_norm : out_norm, ACT_F16, cp ? cp_logits : logits,
                        hm.rows, nullptr, 0, EPI_STORE, cp ? nullptr : hidden, H, nullptr, &ncta, &slice, &smem);
        h.slice_bytes = slice;
        h.base = ff_xmid; h.part = ff_part_d; h.np = S.N / S.C; h.nv_in = nv; h.in_row = nv - 1;
        h.st = st; h.err = d_err; h.frame_end = cp ? 0 : 1;
        Hd.grid = ncta; Hd.smem = smem;
        Hd.bytes = (hm.type == W_Q8_0 ? 34.0 / 32.0 : 2.0) * (double) hm.rows * hm.cols;
        ff_regions(Hd.w, hm);
        Ls.push_back(Hd);
        return ncta > 0;
    };
    for (int g = 0; g < NG; ++g)
        if (!stack(true, g, g == 0 ? FIN_CB0 : FIN_CBG, g, g == 0 ? logits : cp_logits)) { err = "fused frame: head shape"; return false; }
    if (!stack(false, 0, FIN_TALKER, NG, cp_logits)) { err = "fused frame: head shape"; return false; }
    if (d_fftrace && Ls.size() > 256) { err = "fused frame: too many launches to trace"; return false; }
    ff_kinds.clear();
    for (size_t i = 0; i < Ls.size(); ++i) {
        Ls[i].a.launch_id = Ls[i].f.launch_id = Ls[i].h.launch_id = (int) i;
        Ls[i].h.fr = fr;
        ff_kinds.push_back(Ls[i].kind * 4 + (Ls[i].samples ? 2 : 0) + (Ls[i].nv - 1));
    }
    // each launch prefetches the weights of the next two into L2
    for (size_t i = 0; i < Ls.size(); ++i) {
        FfPrefetch pf{};
        for (size_t k = i + 1; k < Ls.size() && k <= i + (size_t) ff_pf_ahead; ++k)
            for (auto & r : Ls[k].w)
                if (pf.n < FF_MAX_PF) { pf.p[pf.n] = r.first; pf.bytes[pf.n] = r.second; ++pf.n; }
        if (Ls[i].kind == 0) Ls[i].a.pf = pf;
        else if (Ls[i].kind == 1) Ls[i].f.pf = pf;
        else Ls[i].h.pf = pf;
    }
    for (auto & X : Ls) {
        cudaLaunchConfig_t cfgl{};
        cfgl.gridDim = dim3(X.grid);
        cfgl.blockDim = dim3(FF_THREADS);
        cfgl.dynamicSmemBytes = X.smem;
        cfgl.stream = stream;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = (unsigned) X.cluster;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = 1;
        cfgl.attrs = at;
        cfgl.numAttrs = X.kind == 2 ? 1 : 2;
        prof_stage = X.stage;
        // profile classes: a launch that samples is charged to sampling (it also runs its
        // pass's first attention block), other attention blocks to attention, the rest to GEMV
        prof_begin(X.kind == 0 ? (X.samples ? KC_SAMPLE : KC_ATTN) : KC_GEMV, X.bytes);
        cudaError_t e;
        if (X.kind == 0) e = X.nv == 2 ? cudaLaunchKernelEx(&cfgl, k_ff_attn<2>, X.a) : cudaLaunchKernelEx(&cfgl, k_ff_attn<1>, X.a);
        else if (X.kind == 1) e = X.nv == 2 ? cudaLaunchKernelEx(&cfgl, k_ff_ffn<2>, X.f) : cudaLaunchKernelEx(&cfgl, k_ff_ffn<1>, X.f);
        else e = cudaLaunchKernelEx(&cfgl, k_ff_head, X.h);
        prof_end();
        if (e != cudaSuccess) { err = std::string("fused frame launch: ") + cudaGetErrorString(e); return false; }
        ++launches;
    }
    prof_stage = STG_TALKER;
    return true;
}

// ---------------------------------------------------------------- prefill & helpers
bool Engine::prefill(const float * rows_host, int n, int n_past, float * hidden_out, float * logits_out) {
    const qtts_config & c = cfg;
    const int H = c.hidden_size;
    if (n <= 0) { err = "n_tokens must be > 0"; return false; }
    if (n_ctx == 0 && !init_kv(std::max(256, n_past + n + 16))) return false;
    if (n_past + n > n_ctx) { err = "Context length exceeded"; return false; }
    // rows uploaded once (rows_host), or already assembled in d_prow (rows_host ==
    // nullptr, generate); chunks of 8 rows through the GEMV path, or of up to 128
    // rows through tcgen05 GEMMs (kind::f16 for F16 weights, kind::i8 for Q8_0;
    // QTTS_PREFILL=gemv|tc, default tc for prompts of more than 8 rows)
    if (!rows_host && n > prow_cap) { err = "prefill rows not assembled"; return false; }
    if (rows_host && !grow_rows(&d_prow, &prow_cap, n, "alloc prefill rows")) return false;
    const char * pm = getenv("QTTS_PREFILL");
    const bool tc = pm && *pm ? strcmp(pm, "tc") == 0 : n > QTTS_MAX_NV;
    const int chunk = tc ? PREFILL_TC_ROWS : QTTS_MAX_NV;
    QCHECK(cudaEventRecord(ev0, stream));
    if (rows_host)
        QCHECK(cudaMemcpyAsync(d_prow, rows_host, sizeof(float) * (size_t) n * H, cudaMemcpyHostToDevice, stream));
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int M = std::min(chunk, n - c0);
        float * X = d_prow + (size_t) c0 * H;
        if (tc) { if (!prefill_tc_layers(*this, X, M, n_past + c0)) return false; }
        else if (!layers(L, kc, vc, n_ctx, rope_t, X, M, nullptr, n_past + c0, false, nullptr, c.intermediate_size))
            return false;
    }
    // last row: output norm + codec head (the GEMV writes the normed row to `hidden`)
    if (!gemv(codec_head, nullptr, d_prow + (size_t)(n - 1) * H, H, 1, out_norm, ACT_F16, logits, c.codec_vocab_size,
              nullptr, 0, EPI_STORE, hidden, H, nullptr))
        return false;
    if (hidden_out) {   // every row's hidden state, normalised in place after the head has read the last row
        k_rmsnorm_rows<<<n, 256, 0, stream>>>(d_prow, H, out_norm, c.rms_norm_eps, H, d_prow, H);
        QCHECK(cudaMemcpyAsync(hidden_out, d_prow, sizeof(float) * (size_t) n * H, cudaMemcpyDeviceToHost, stream));
    }
    QCHECK(cudaEventRecord(ev1, stream));
    last_hidden.resize(H);
    QCHECK(cudaMemcpyAsync(last_hidden.data(), hidden, sizeof(float) * H, cudaMemcpyDeviceToHost, stream));
    if (logits_out)
        QCHECK(cudaMemcpyAsync(logits_out, logits, sizeof(float) * c.codec_vocab_size, cudaMemcpyDeviceToHost, stream));
    if (!sync("forward_prefill")) return false;
    if (tc && !prefill_tc_check(*this)) return false;
    cudaEventElapsedTime(&timing.prefill_ms, ev0, ev1);
    n_used = n_past + n;
    return true;
}

bool Engine::lookup(int table, const int32_t * ids, int n, std::vector<float> & out) {
    const qtts_config & c = cfg;
    if (n <= 0) { out.clear(); return true; }
    const __half * tab;
    int dim, vocab;
    if (table == 0) { tab = codec_embd; dim = c.hidden_size; vocab = c.codec_vocab_size; }
    else if (table < 0) { tab = text_embd; dim = c.text_embd_dim; vocab = c.text_vocab_size; }
    else if (table < c.n_codebooks) { tab = cp_embd[table - 1]; dim = c.hidden_size; vocab = c.code_pred_vocab_size; }
    else { err = "Embedding tensor not found"; return false; }
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= vocab) { err = "Embedding token ID out of range"; return false; }
    out.resize((size_t) n * dim);
    const int step = QTTS_MAX_NV;   // rows staged through tmp_a per round trip
    for (int c0 = 0; c0 < n; c0 += step) {
        const int m = std::min(step, n - c0);
        QCHECK(cudaMemcpyAsync(d_ids, ids + c0, sizeof(int) * m, cudaMemcpyHostToDevice, stream));
        k_gather_rows<<<m, 256, 0, stream>>>(tab, dim, d_ids, m, tmp_a);
        QCHECK(cudaMemcpyAsync(out.data() + (size_t) c0 * dim, tmp_a, sizeof(float) * m * dim, cudaMemcpyDeviceToHost, stream));
        if (!sync("lookup_embedding_rows")) return false;
    }
    return true;
}

// Grows a device row buffer [cap][H] to at least n rows (contents not kept).
bool Engine::grow_rows(float ** buf, int * cap, int n, const char * what) {
    if (n <= *cap) return true;
    if (*buf) cudaFree(*buf);
    *cap = std::max(n, 256);
    if (cudaMalloc(buf, sizeof(float) * (size_t) *cap * cfg.hidden_size) != cudaSuccess) {
        *buf = nullptr; *cap = 0; err = what; return false;
    }
    return true;
}

// project_text_tokens (src/tts_transformer.cpp:963-1028) of n ids already on the
// device into d_ptext rows [0, n): per 8-row chunk the gather, fc1 + bias + SiLU
// and fc2 + bias.  Each row's arithmetic is independent of the chunking.
bool Engine::project_text_dev(const int * d_tok, int n) {
    const qtts_config & c = cfg;
    const int TD = c.text_embd_dim, H = c.hidden_size;
    if (!grow_rows(&d_ptext, &ptext_cap, n, "alloc text rows")) return false;
    for (int c0 = 0; c0 < n; c0 += QTTS_MAX_NV) {
        const int m = std::min(QTTS_MAX_NV, n - c0);
        float * y = d_ptext + (size_t) c0 * H;
        k_gather_rows<<<m, 256, 0, stream>>>(text_embd, TD, d_tok + c0, m, tmp_a);
        if (!gemv(fc1, nullptr, tmp_a, TD, m, nullptr, ACT_F16, hbuf, TD, nullptr, 0, EPI_STORE, nullptr, 0, nullptr)) return false;
        k_bias_silu<<<32, 256, 0, stream>>>(hbuf, fc1_b, TD, TD, m);
        if (!gemv(fc2, nullptr, hbuf, TD, m, nullptr, ACT_F16, y, H, nullptr, 0, EPI_STORE, nullptr, 0, nullptr)) return false;
        k_bias_add<<<32, 256, 0, stream>>>(y, fc2_b, H, H, m);
    }
    return true;
}

// qtts_project_text: the projected rows back to the host (one upload, one copy back).
bool Engine::project_text(const int32_t * toks, int n, std::vector<float> & out) {
    const qtts_config & c = cfg;
    const int H = c.hidden_size;
    if (n <= 0) { out.clear(); return true; }
    for (int i = 0; i < n; ++i)
        if (toks[i] < 0 || toks[i] >= c.text_vocab_size) { err = "Embedding token ID out of range"; return false; }
    if (n > ids_cap) {
        if (d_ids) cudaFree(d_ids);
        ids_cap = std::max(n, 2 * ids_cap);
        if (cudaMalloc(&d_ids, sizeof(int) * ids_cap) != cudaSuccess) { d_ids = nullptr; ids_cap = 0; err = "alloc ids"; return false; }
    }
    out.resize((size_t) n * H);
    QCHECK(cudaMemcpyAsync(d_ids, toks, sizeof(int) * n, cudaMemcpyHostToDevice, stream));
    if (!project_text_dev(d_ids, n)) return false;
    QCHECK(cudaMemcpyAsync(out.data(), d_ptext, sizeof(float) * (size_t) n * H, cudaMemcpyDeviceToHost, stream));
    return sync("project_text_tokens");
}

// The prompt recipe of generate (build_prefill_graph, src/tts_transformer.cpp:
// 1030-1186) or generate_icl (build_prefill_graph_icl, :1188-1472): which text
// tokens are projected, which codec rows are gathered, and each row's terms in
// the reference's order.  Host-only; ids are checked here.
bool Engine::plan_prompt(const qtts_generate_params * p, PromptPlan & P) {
    const qtts_config & c = cfg;
    const bool icl = p->ref_codec_tokens != nullptr;
    using S = PromptSrc;
    auto text = [&](int i) { return S{S::TEXT, i}; };
    auto codec = [&](int i) { return S{S::CODEC, i}; };
    if (icl) {
        if (!p->text_tokens || p->n_tokens < 4) { err = "ICL: need at least 4 target text tokens"; return false; }
        if (!p->ref_codec_tokens || p->n_ref_frames < 1) { err = "ICL: need at least 1 reference codec frame"; return false; }
    } else {
        if (!p->text_tokens) { err = "text_tokens is null"; return false; }
        if (p->n_tokens < 4) { err = "Need at least 4 text tokens for prefill"; return false; }
    }
    // projected text rows: 0 tts_bos, 1 tts_eos, 2 tts_pad, 3-5 the role tokens, then per mode
    P.text = {c.tts_bos_token_id, c.tts_eos_token_id, c.tts_pad_token_id, p->text_tokens[0], p->text_tokens[1],
              p->text_tokens[2]};
    const S bos = text(0), eos = text(1), pad = text(2);
    // codec prefix: think tokens (language or not), [speaker], codec_pad, codec_bos
    if (icl || p->language_id < 0) P.codec = {c.codec_nothink_id, c.codec_think_bos_id, c.codec_think_eos_id};
    else P.codec = {c.codec_think_id, c.codec_think_bos_id, p->language_id, c.codec_think_eos_id};
    const int nthink = (int) P.codec.size();
    P.codec.push_back(c.codec_pad_id);
    P.codec.push_back(c.codec_bos_id);
    P.speaker = p->speaker_embd;
    std::vector<S> ci;
    for (int i = 0; i < nthink; ++i) ci.push_back(codec(i));
    if (P.speaker) ci.push_back(S{S::SPEAKER, 0});
    ci.push_back(codec(nthink));
    ci.push_back(codec(nthink + 1));
    const int cin = (int) ci.size(), ov = cin - 1;
    int r = 0;
    if (!icl) {
        int ilen = 0;
        if (p->instruct_tokens && p->n_instruct > 0) {
            ilen = p->n_instruct;
            for (int i = 0; i < ilen; ++i) {
                P.add(PromptPlan::PREFILL, r++, text((int) P.text.size()));
                P.text.push_back(p->instruct_tokens[i]);
            }
        }
        for (int k = 0; k < 3; ++k) P.add(PromptPlan::PREFILL, r++, text(3 + k));
        for (int t = 0; t < ov; ++t) P.add(PromptPlan::PREFILL, r++, t == ov - 1 ? bos : pad, ci[t]);
        P.add(PromptPlan::PREFILL, r++, text((int) P.text.size()), ci[cin - 1]);   // first text token + codec_bos
        P.text.push_back(p->text_tokens[3]);
        const int ntrail = std::max(0, p->n_tokens - 9);
        for (int i = 0; i < ntrail; ++i) {
            P.add(PromptPlan::TRAILING, i, text((int) P.text.size()));
            P.text.push_back(p->text_tokens[4 + i]);
        }
        P.add(PromptPlan::TRAILING, ntrail, eos);
    } else {
        for (int k = 0; k < 3; ++k) P.add(PromptPlan::PREFILL, r++, text(3 + k));
        for (int t = 0; t < ov; ++t) P.add(PromptPlan::PREFILL, r++, t == ov - 1 ? bos : pad, ci[t]);
        // reference text [3, n_ref_text - 5) + target text [3, n_tokens - 5) + tts_eos
        int rs = 3, re = p->n_ref_text - 5; if (re < rs) re = rs;
        int ts = 3, tend = p->n_tokens - 5; if (tend < ts) tend = ts;
        const int t0 = (int) P.text.size();
        for (int i = rs; i < re && i < p->n_ref_text; ++i) P.text.push_back(p->ref_text_tokens[i]);
        for (int i = ts; i < tend && i < p->n_tokens; ++i) P.text.push_back(p->text_tokens[i]);
        P.text.push_back(c.tts_eos_token_id);
        const int nt = (int) P.text.size() - t0;
        const int nct = p->n_ref_frames + 1;
        P.codec.push_back(c.codec_bos_id);   // codec row of ICL position 0
        const S cbos = codec((int) P.codec.size() - 1);
        // ICL rows: (0 + text or pad) + (codec_bos, then the summed reference frames)
        for (int i = 0; i < nct; ++i)
            P.add(PromptPlan::PREFILL, r++, i < nt ? text(t0 + i) : pad, i == 0 ? cbos : S{S::ICL, i - 1}, 1);
        for (int i = nct; i < nt; ++i) P.add(PromptPlan::TRAILING, i - nct, text(t0 + i));
        P.n_icl = p->n_ref_frames;
        P.icl_codes.assign(p->ref_codec_tokens, p->ref_codec_tokens + (size_t) p->n_ref_frames * 16);
        const int NCB = std::min(16, c.n_codebooks);
        for (int f = 0; f < P.n_icl; ++f)
            for (int cb = 0; cb < NCB; ++cb) {
                const int id = P.icl_codes[(size_t) f * 16 + cb];
                if (id < 0 || id >= (cb == 0 ? c.codec_vocab_size : c.code_pred_vocab_size)) {
                    err = "Embedding token ID out of range"; return false;
                }
            }
    }
    P.add(PromptPlan::PAD, 0, pad);
    for (int32_t id : P.text)
        if (id < 0 || id >= c.text_vocab_size) { err = "Embedding token ID out of range"; return false; }
    for (int32_t id : P.codec)
        if (id < 0 || id >= c.codec_vocab_size) { err = "Embedding token ID out of range"; return false; }
    return true;
}

// Carries out a prompt recipe on the device: one upload of every id, the text
// projection into d_ptext, the codec rows (k_gather_rows), the speaker row and
// the ICL frame rows (k_icl_codec_rows) into d_asm, then k_prompt_rows writes
// the prefill rows (d_prow), the trailing text rows and the pad row.  No row
// crosses PCIe; the buffers it writes must be sized by the caller for trailing.
bool Engine::assemble_prompt(const PromptPlan & P) {
    const qtts_config & c = cfg;
    const int H = c.hidden_size, NCB = std::min(16, c.n_codebooks);
    const int nT = (int) P.text.size(), nC = (int) P.codec.size(), nI = P.n_icl;
    const int nid = nT + nC + nI * 16;
    if (nid > ids_cap) {
        if (d_ids) cudaFree(d_ids);
        ids_cap = std::max(nid, 2 * ids_cap);
        if (cudaMalloc(&d_ids, sizeof(int) * ids_cap) != cudaSuccess) { d_ids = nullptr; ids_cap = 0; err = "alloc ids"; return false; }
    }
    if (!grow_rows(&d_asm, &asm_cap, nC + 1 + nI, "alloc prompt terms") ||
        !grow_rows(&d_prow, &prow_cap, P.plen, "alloc prefill rows"))
        return false;
    const int nr = (int) P.rows.size();
    if (nr > pops_cap) {
        if (d_pops) cudaFree(d_pops);
        pops_cap = std::max(nr, 256);
        if (cudaMalloc(&d_pops, sizeof(PromptRow) * pops_cap) != cudaSuccess) {
            d_pops = nullptr; pops_cap = 0; err = "alloc prompt recipe"; return false;
        }
    }
    float * codec_rows = d_asm, * spk_row = d_asm + (size_t) nC * H, * icl_rows = d_asm + (size_t)(nC + 1) * H;
    auto src = [&](const PromptSrc & s) -> const float * {
        switch (s.kind) {
            case PromptSrc::TEXT: return d_ptext + (size_t) s.idx * H;
            case PromptSrc::CODEC: return codec_rows + (size_t) s.idx * H;
            case PromptSrc::SPEAKER: return spk_row;
            case PromptSrc::ICL: return icl_rows + (size_t) s.idx * H;
            default: return nullptr;
        }
    };
    std::vector<int32_t> ids;
    ids.reserve(nid);
    ids.insert(ids.end(), P.text.begin(), P.text.end());
    ids.insert(ids.end(), P.codec.begin(), P.codec.end());
    ids.insert(ids.end(), P.icl_codes.begin(), P.icl_codes.end());
    if (!ev_asm0) { QCHECK(cudaEventCreate(&ev_asm0)); QCHECK(cudaEventCreate(&ev_asm1)); }
    QCHECK(cudaEventRecord(ev_asm0, stream));
    QCHECK(cudaMemcpyAsync(d_ids, ids.data(), sizeof(int) * nid, cudaMemcpyHostToDevice, stream));
    if (!project_text_dev(d_ids, nT)) return false;
    k_gather_rows<<<nC, 256, 0, stream>>>(codec_embd, H, d_ids + nT, nC, codec_rows);
    if (P.speaker) QCHECK(cudaMemcpyAsync(spk_row, P.speaker, sizeof(float) * H, cudaMemcpyHostToDevice, stream));
    if (nI) k_icl_codec_rows<<<nI, 256, 0, stream>>>(codec_embd, d_cp_embd, d_ids + nT + nC, NCB, H, icl_rows);
    // (ICL rows: codec_embd[cb0] then += code_pred_embd[cb-1][code] in codebook order)
    std::vector<PromptRow> ops(nr);
    for (int i = 0; i < nr; ++i) {
        const PromptPlan::Row & R = P.rows[i];
        float * dst = R.dst == PromptPlan::PREFILL ? d_prow + (size_t) R.r * H
                      : R.dst == PromptPlan::TRAILING ? trailing + (size_t) R.r * H : pad;
        ops[i] = PromptRow{dst, src(R.a), src(R.b), R.zero_first};
    }
    QCHECK(cudaMemcpyAsync(d_pops, ops.data(), sizeof(PromptRow) * nr, cudaMemcpyHostToDevice, stream));
    k_prompt_rows<<<nr, 256, 0, stream>>>(d_pops, H);
    QCHECK(cudaGetLastError());
    QCHECK(cudaEventRecord(ev_asm1, stream));
    return true;
}

int Engine::begin(const qtts_generate_params * p) {
    const qtts_config & c = cfg;
    const int H = c.hidden_size;
    sess = GenSession{};
    attn_rows.clear();
    PromptPlan plan;
    stages = qtts_stage_timing{};
    const auto t_build = std::chrono::steady_clock::now();
    if (!plan_prompt(p, plan)) return -1;
    const float plan_ms =
        (float) std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_build).count();
    const int plen = plan.plen, tlen = plan.tlen;
    const int required = plen + p->max_len + 8;
    if (n_ctx < required || n_ctx > std::max(required * 2, 512)) { if (!init_kv(required)) return -1; }
    n_used = 0;
    // device buffers sized for this call (re-capture when they grow)
    if (p->max_len > codes_cap) {
        if (d_codes) cudaFree(d_codes);
        codes_cap = std::max(p->max_len, 256);
        if (cudaMalloc(&d_codes, sizeof(int) * codes_cap * c.n_codebooks) != cudaSuccess) { err = "alloc codes"; return -1; }
        graph_ok = false;
    }
    if (std::max(tlen, 1) > trailing_cap) {
        if (trailing) cudaFree(trailing);
        trailing_cap = std::max(tlen, 256);
        if (cudaMalloc(&trailing, sizeof(float) * trailing_cap * H) != cudaSuccess) { err = "alloc trailing"; return -1; }
        graph_ok = false;
    }
    if (attn_dump) {
        const size_t need = (size_t) p->max_len * c.n_attention_heads * n_ctx;
        if (need > attn_cap) {
            if (d_attn) cudaFree(d_attn);
            attn_cap = need;
            if (cudaMalloc(&d_attn, sizeof(float) * attn_cap) != cudaSuccess) { err = "alloc attn dump"; return -1; }
            graph_ok = false;
        }
    }
    if (h_dbg_cap > 0 && (h_dbg_t || h_dbg_cp)) {
        const int cap = std::min(h_dbg_cap, p->max_len);
        if (cap > dbg_cap) {
            if (dbg_t) cudaFree(dbg_t);
            if (dbg_cp) cudaFree(dbg_cp);
            dbg_cap = cap;
            if (cudaMalloc(&dbg_t, sizeof(float) * dbg_cap * c.codec_vocab_size) != cudaSuccess ||
                cudaMalloc(&dbg_cp, sizeof(float) * dbg_cap * (c.n_codebooks - 1) * c.code_pred_vocab_size) != cudaSuccess) {
                err = "alloc debug logits"; return -1;
            }
        }
    }
    if (!assemble_prompt(plan)) return -1;   // prefill rows, trailing rows and the pad row, on the device
    if (!prefill(nullptr, plen, 0, nullptr, nullptr)) return -1;
    stages.prefill_forward_ms = timing.prefill_ms;
    float asm_ms = 0.0f;
    cudaEventElapsedTime(&asm_ms, ev_asm0, ev_asm1);   // complete: prefill() synchronised the stream
    stages.prefill_build_ms = plan_ms + asm_ms;
    DevState hs{};
    hs.pos = plen; hs.frame = 0; hs.done = 0; hs.n_out = 0; hs.n_trailing = tlen;
    SampleParams P{};
    P.temperature = p->temperature; P.top_k = p->top_k; P.rep_penalty = p->repetition_penalty;
    P.eos_bias = p->eos_bias; P.target_frames = p->target_frames; P.eos_id = c.codec_eos_id;
    P.suppress_start = c.codec_vocab_size - 1024; P.seed = p->seed ? p->seed : seed;
    P.record_logits = (h_dbg_cap > 0 && (h_dbg_t || h_dbg_cp)) ? 1 : 0;
    P.dbg_talker = dbg_t; P.dbg_cp = dbg_cp; P.dbg_cap = P.record_logits ? std::min(dbg_cap, p->max_len) : 0;
    P.n_cb = c.n_codebooks;
    if (cudaMemcpyAsync(st, &hs, sizeof(hs), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(sp, &P, sizeof(P), cudaMemcpyHostToDevice, stream) != cudaSuccess) {
        err = "upload state"; return -1;
    }
    if (cudaMemcpyAsync(logits0, logits, sizeof(float) * c.codec_vocab_size, cudaMemcpyDeviceToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(hidden0, hidden, sizeof(float) * H, cudaMemcpyDeviceToDevice, stream) != cudaSuccess) {
        err = "snapshot prefill outputs"; return -1;
    }
    if (d_err && cudaMemsetAsync(d_err, 0, sizeof(int), stream) != cudaSuccess) { err = "reset error flag"; return -1; }
    if (!sync("generate setup")) return -1;
    sess.st0 = hs;
    if (frame_mode == FM_FUSED) {
        const int keys = std::min(n_ctx, plen + p->max_len + 1);   // the talker attention's longest row
        if (keys > ff_max_keys) { ff_max_keys = std::max(keys, 512); graph_ok = false; }
    }
    if (!graph_ok && !capture_graph()) return -1;
    sess.active = true;
    sess.max_len = p->max_len;
    sess.prefill_len = plen;
    sess.trailing_len = tlen;
    timing.frames_ms = 0.0f;
    timing.frames = 0;
    timing.kernel_launches = launches_per_frame;
    return plen;
}

// Back to frame 0 of the active generation: the frame state and the
// prefill's logits and hidden row are restored; KV positions past the prefill
// are rewritten as frames are generated again.
int Engine::rewind() {
    if (!sess.active) { err = "no active generation"; return -1; }
    if (cudaMemcpyAsync(st, &sess.st0, sizeof(DevState), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(logits, logits0, sizeof(float) * cfg.codec_vocab_size, cudaMemcpyDeviceToDevice, stream) != cudaSuccess ||
        cudaMemcpyAsync(hidden, hidden0, sizeof(float) * cfg.hidden_size, cudaMemcpyDeviceToDevice, stream) != cudaSuccess) {
        err = "rewind state"; return -1;
    }
    sess.produced = 0;
    sess.done = false;
    n_used = sess.st0.pos;
    return 0;
}

int Engine::run_frames(int n, int32_t * codes_out) {
    const int NCB = cfg.n_codebooks;
    if (!sess.active) { err = "no active generation"; return -1; }
    if (sess.done) return 0;
    n = std::min(n, sess.max_len - sess.produced);
    if (n <= 0) return 0;
    if (cudaEventRecord(ev0, stream) != cudaSuccess) { err = "event"; return -1; }
    const bool staged = stage_timing;
    if (staged) {   // kernel by kernel, events around every launch
        profiling = true;
        prof_evs.clear();
        ev_used = 0;
        bool ok = true;
        for (int i = 0; i < n && ok; ++i) ok = frame_mode == FM_FUSED ? enqueue_frame_ff() : enqueue_frame();
        profiling = false;
        if (!ok) return -1;
    } else {
        for (int i = 0; i < n; ++i)
            if (cudaGraphLaunch(graph, stream) != cudaSuccess) { err = "graph launch failed"; return -1; }
    }
    if (cudaEventRecord(ev1, stream) != cudaSuccess) { err = "event"; return -1; }
    DevState hs;
    int kerr = 0;
    if (cudaMemcpyAsync(&hs, st, sizeof(hs), cudaMemcpyDeviceToHost, stream) != cudaSuccess) { err = "state readback"; return -1; }
    if (frame_mode == FM_FUSED && cudaMemcpyAsync(&kerr, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) {
        err = "error flag readback"; return -1;
    }
    if (!sync("frame loop")) return -1;
    if (kerr) { err = "fused frame kernels: a wait timed out"; sess.active = false; return -1; }
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    timing.frames_ms += ms;
    const int got = hs.n_out - sess.produced;
    timing.frames += got;
    if (staged) {
        for (auto & e : prof_evs) {
            float t = 0.0f;
            cudaEventElapsedTime(&t, e.a, e.b);
            if (e.cls == KC_SAMPLE) stages.sample_embed_ms += t;
            else if (e.stage == STG_CP) stages.code_pred_ms += t;
            else stages.talker_ms += t;
        }
        prof_evs.clear();
        stages.frames += got;
    }
    if (got > 0 && codes_out) {
        if (cudaMemcpy(codes_out, d_codes + (size_t) sess.produced * NCB, sizeof(int) * got * NCB, cudaMemcpyDeviceToHost) != cudaSuccess) {
            err = "codes readback"; return -1;
        }
    }
    if (attn_dump && got > 0) {
        const int NH = cfg.n_attention_heads;
        std::vector<float> buf((size_t) NH * n_ctx);
        for (int f = sess.produced; f < sess.produced + got; ++f) {
            if (cudaMemcpy(buf.data(), d_attn + (size_t) f * NH * n_ctx, sizeof(float) * buf.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
                err = "attn readback"; return -1;
            }
            const int nkv = sess.prefill_len + f + 1;
            std::vector<float> row((size_t) NH * nkv);
            for (int h = 0; h < NH; ++h) memcpy(row.data() + (size_t) h * nkv, buf.data() + (size_t) h * n_ctx, sizeof(float) * nkv);
            attn_rows.push_back(std::move(row));
        }
    }
    if (h_dbg_cap > 0 && got > 0) {
        const int f0 = sess.produced, f1 = std::min(sess.produced + got + (hs.done ? 1 : 0), std::min(dbg_cap, h_dbg_cap));
        if (f1 > f0) {
            if (h_dbg_t) cudaMemcpy(h_dbg_t + (size_t) f0 * cfg.codec_vocab_size, dbg_t + (size_t) f0 * cfg.codec_vocab_size,
                                    sizeof(float) * (f1 - f0) * cfg.codec_vocab_size, cudaMemcpyDeviceToHost);
            const size_t per = (size_t)(NCB - 1) * cfg.code_pred_vocab_size;
            if (h_dbg_cp) cudaMemcpy(h_dbg_cp + f0 * per, dbg_cp + f0 * per, sizeof(float) * (f1 - f0) * per, cudaMemcpyDeviceToHost);
        }
    }
    sess.produced = hs.n_out;
    sess.done = hs.done != 0;
    n_used = hs.pos;
    return got;
}

}  // namespace qtts

#include "batch_host.cuh"

using qtts::Engine;

// ================================================================ C ABI
extern "C" {

// ---------------------------------------------------------------- kernel-level entry points
// These run one engine kernel on caller-provided host data (device buffers are
// allocated per call); the parity tests use them to check a kernel in isolation.
int32_t qtts_op_gemm_q8(int32_t device, const uint8_t * w, const uint8_t * w_up, int32_t rows, int32_t cols,
                        const float * xin, int32_t m, const float * norm_gain, float eps, int32_t epi,
                        const float * resid, int32_t ksplit, float * y) {
    using namespace qtts;
    const bool swiglu = epi == TC_EPI_SWIGLU;
    const int rows_w = swiglu ? 2 * rows : rows;
    const int np = (m + 15) / 16 * 16, nb = cols / 32;
    if (!w || !xin || !y || m <= 0 || rows <= 0 || rows_w % TC_BM || cols % Q8_BK || np > Q8_MAX_N ||
        (swiglu && (!w_up || rows % (TC_BM / 2))) || (epi == TC_EPI_RESID && !resid) || epi < 0 || epi > 2 ||
        ksplit < 0 || ksplit > 8)
        return 0;
    if (cudaSetDevice(device) != cudaSuccess) return 0;
    void * dq = nullptr, * dd = nullptr, * dq2 = nullptr, * dd2 = nullptr, * dwt = nullptr, * dws = nullptr,
         * dx = nullptr, * dxq = nullptr, * dxs = nullptr, * dy = nullptr, * dg = nullptr, * derr = nullptr;
    bool ok = true;
    std::string why;
    auto chk = [&](cudaError_t e) {
        if (e != cudaSuccess && ok) { ok = false; why = cudaGetErrorString(e); }
    };
    // GGUF blocks (f16 d + 32 int8) -> the engine's split planes
    std::vector<int8_t> hq((size_t) rows * cols), hq2(swiglu ? (size_t) rows * cols : 0);
    std::vector<uint16_t> hd((size_t) rows * nb), hd2(swiglu ? (size_t) rows * nb : 0);
    for (int pass = 0; pass < (swiglu ? 2 : 1); ++pass) {
        const uint8_t * src = pass ? w_up : w;
        int8_t * q = pass ? hq2.data() : hq.data();
        uint16_t * d = pass ? hd2.data() : hd.data();
        for (size_t blk = 0; blk < (size_t) rows * nb; ++blk) {
            memcpy(d + blk, src + blk * 34, 2);
            memcpy(q + blk * 32, src + blk * 34 + 2, 32);
        }
    }
    chk(cudaMalloc(&dq, hq.size()));
    chk(cudaMalloc(&dd, hd.size() * 2));
    if (swiglu) { chk(cudaMalloc(&dq2, hq2.size())); chk(cudaMalloc(&dd2, hd2.size() * 2)); }
    chk(cudaMalloc(&dwt, (size_t) rows_w * cols));
    chk(cudaMalloc(&dws, (size_t) rows_w * nb * 2));
    chk(cudaMalloc(&dx, sizeof(float) * m * cols));
    chk(cudaMalloc(&dxq, (size_t) np * cols));
    chk(cudaMalloc(&dxs, sizeof(float) * np * nb));
    chk(cudaMalloc(&dy, sizeof(float) * m * rows));
    chk(cudaMalloc(&derr, sizeof(int)));
    if (norm_gain) chk(cudaMalloc(&dg, sizeof(float) * cols));
    int S = 0;
    if (ok) {
        chk(cudaMemcpy(dq, hq.data(), hq.size(), cudaMemcpyHostToDevice));
        chk(cudaMemcpy(dd, hd.data(), hd.size() * 2, cudaMemcpyHostToDevice));
        if (swiglu) {
            chk(cudaMemcpy(dq2, hq2.data(), hq2.size(), cudaMemcpyHostToDevice));
            chk(cudaMemcpy(dd2, hd2.data(), hd2.size() * 2, cudaMemcpyHostToDevice));
        }
        chk(cudaMemcpy(dx, xin, sizeof(float) * m * cols, cudaMemcpyHostToDevice));
        if (resid) chk(cudaMemcpy(dy, resid, sizeof(float) * m * rows, cudaMemcpyHostToDevice));
        if (norm_gain) chk(cudaMemcpy(dg, norm_gain, sizeof(float) * cols, cudaMemcpyHostToDevice));
        chk(cudaMemset(derr, 0, sizeof(int)));
    }
    if (ok) {
        DMat W{}, W2{};
        W.type = W_Q8_0; W.rows = rows; W.cols = cols; W.w = dq; W.d = (const __half *) dd;
        if (swiglu) { W2 = W; W2.w = dq2; W2.d = (const __half *) dd2; }
        k_tile_q8<<<rows_w, 128>>>(W, W2, rows_w, (uint8_t *) dwt, (__half *) dws);
        PackQ8Args pa{};
        pa.x = (const float *) dx; pa.ldx = cols; pa.m_real = m; pa.np = np; pa.cols = cols;
        pa.gain = (const float *) dg; pa.eps = eps; pa.out = (uint8_t *) dxq; pa.dscale = (float *) dxs;
        k_pack_q8<<<np, 256>>>(pa);
        GemmQ8Args g{};
        g.w = (const uint8_t *) dwt; g.ws = (const __half *) dws; g.x = (const uint8_t *) dxq; g.xs = (const float *) dxs;
        g.rows_w = rows_w; g.cols = cols; g.np = np; g.m_real = m; g.epi = epi; g.y = (float *) dy; g.ldy = rows;
        g.resid = (const float *) dy; g.ldr = rows; g.err = (int *) derr;
        g.ksplit = ksplit > 0 ? ksplit : q8_choose_split(g);
        if (g.ksplit > cols / Q8_BK || q8_stages(np, cols, q8_partial_bytes(np, m, g.ksplit)) < 2) {
            ok = false; why = "k-split does not fit";
        }
        S = g.ksplit;
        chk(q8_set_attributes());
        if (ok) chk(q8_launch(g, 0));
        chk(cudaGetLastError());
        chk(cudaDeviceSynchronize());
        int herr = 0;
        if (ok) chk(cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr && ok) { ok = false; why = "a bounded wait gave up (" + std::to_string(herr) + ")"; }
        if (ok) chk(cudaMemcpy(y, dy, sizeof(float) * m * rows, cudaMemcpyDeviceToHost));
    }
    void * all[] = {dq, dd, dq2, dd2, dwt, dws, dx, dxq, dxs, dy, dg, derr};
    for (void * p : all) if (p) cudaFree(p);
    if (!ok) qtts::g_create_error = "qtts_op_gemm_q8: " + why;
    return ok ? S : 0;
}

int32_t qtts_op_gemm_tc(int32_t device, const uint16_t * w, const uint16_t * w_up, int32_t rows, int32_t cols,
                        const float * xin, int32_t m, const float * norm_gain, float eps, int32_t act, int32_t epi,
                        const float * resid, float * y) {
    using namespace qtts;
    const bool swiglu = epi == TC_EPI_SWIGLU;
    const int rows_w = swiglu ? 2 * rows : rows;
    const int mp = (m + 15) / 16 * 16;
    const int np = act == TC_ACT_SPLIT ? 2 * mp : mp;
    if (!w || !xin || !y || m <= 0 || rows <= 0 || rows_w % TC_BM || cols % TC_BK || np > TC_MAX_N ||
        (swiglu && !w_up) || (epi == TC_EPI_RESID && !resid) || epi < 0 || epi > 2 || act < 0 || act > 1)
        return 0;
    if (cudaSetDevice(device) != cudaSuccess) return 0;
    void * dw = nullptr, * dw2 = nullptr, * dwt = nullptr, * dx = nullptr, * dxt = nullptr, * dy = nullptr,
         * dg = nullptr, * derr = nullptr;
    bool ok = true;
    auto chk = [&](cudaError_t e) { if (e != cudaSuccess) ok = false; };
    const size_t wb = (size_t) rows * cols * 2;
    const int ycols = rows;
    chk(cudaMalloc(&dw, wb));
    if (swiglu) chk(cudaMalloc(&dw2, wb));
    chk(cudaMalloc(&dwt, (size_t) rows_w * cols * 2));
    chk(cudaMalloc(&dx, sizeof(float) * m * cols));
    chk(cudaMalloc(&dxt, (size_t) np * cols * 2));
    chk(cudaMalloc(&dy, sizeof(float) * m * ycols));
    chk(cudaMalloc(&derr, sizeof(int)));
    if (norm_gain) chk(cudaMalloc(&dg, sizeof(float) * cols));
    if (ok) {
        chk(cudaMemcpy(dw, w, wb, cudaMemcpyHostToDevice));
        if (swiglu) chk(cudaMemcpy(dw2, w_up, wb, cudaMemcpyHostToDevice));
        chk(cudaMemcpy(dx, xin, sizeof(float) * m * cols, cudaMemcpyHostToDevice));
        if (resid) chk(cudaMemcpy(dy, resid, sizeof(float) * m * ycols, cudaMemcpyHostToDevice));
        if (norm_gain) chk(cudaMemcpy(dg, norm_gain, sizeof(float) * cols, cudaMemcpyHostToDevice));
        chk(cudaMemset(derr, 0, sizeof(int)));
    }
    if (ok) {
        k_tile_weights<<<rows_w, 128>>>((const __half *) dw, (const __half *) dw2, rows_w, cols, (uint8_t *) dwt);
        PackArgs pa{};
        pa.x = (const float *) dx; pa.ldx = cols; pa.m_real = m; pa.np = np; pa.cols = cols;
        pa.gain = (const float *) dg; pa.eps = eps; pa.act = act; pa.out = (uint8_t *) dxt;
        k_pack_act<<<act == TC_ACT_SPLIT ? np / 2 : np, 256>>>(pa);
        GemmTcArgs g{};
        g.w = (const uint8_t *) dwt; g.x = (const uint8_t *) dxt; g.rows_w = rows_w; g.cols = cols; g.np = np;
        g.m_real = m; g.split = act == TC_ACT_SPLIT; g.epi = epi; g.y = (float *) dy; g.ldy = ycols;
        g.resid = (const float *) dy; g.ldr = ycols; g.err = (int *) derr;
        g.ksplit = tc_choose_split(g);
        chk(cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024));
        chk(cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        if (ok) chk(tc_launch(g, 0));
        chk(cudaGetLastError());
        chk(cudaDeviceSynchronize());
        int herr = 0;
        if (ok) chk(cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost));
        if (herr) ok = false;
        if (ok) chk(cudaMemcpy(y, dy, sizeof(float) * m * ycols, cudaMemcpyDeviceToHost));
    }
    void * all[] = {dw, dw2, dwt, dx, dxt, dy, dg, derr};
    for (void * p : all) if (p) cudaFree(p);
    return ok ? 1 : 0;
}

int32_t qtts_op_gemv(int32_t device, int32_t wtype, const void * w, int32_t rows, int32_t cols, const float * xin,
                     int32_t nv, const float * norm_gain, float eps, int32_t act_f32, float * y, int32_t * block_dots) {
    using namespace qtts;
    if (!w || !xin || !y || rows <= 0 || cols <= 0 || nv <= 0 || nv > QTTS_MAX_NV) return 0;
    if (wtype != W_F16 && wtype != W_Q8_0) return 0;
    if ((wtype == W_F16 && cols % 8) || (wtype == W_Q8_0 && cols % 32)) return 0;
    if (cudaSetDevice(device) != cudaSuccess) return 0;
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device);
    const int nb = cols / 32;
    std::vector<uint8_t> q, d;
    DMat A; A.type = wtype; A.rows = rows; A.cols = cols;
    void * dw = nullptr, * dd = nullptr, * dx = nullptr, * dy = nullptr, * dg = nullptr, * dbd = nullptr;
    bool ok = true;
    auto chk = [&](cudaError_t e) { if (e != cudaSuccess) ok = false; };
    if (wtype == W_F16) {
        chk(cudaMalloc(&dw, (size_t) rows * cols * 2));
        chk(cudaMemcpy(dw, w, (size_t) rows * cols * 2, cudaMemcpyHostToDevice));
    } else {
        q.resize((size_t) rows * cols); d.resize((size_t) rows * nb * 2);
        const uint8_t * src = static_cast<const uint8_t *>(w);
        for (size_t r = 0; r < (size_t) rows; ++r)
            for (int b = 0; b < nb; ++b) {
                memcpy(&d[(r * nb + b) * 2], src + (r * nb + b) * 34, 2);
                memcpy(&q[r * cols + (size_t) b * 32], src + (r * nb + b) * 34 + 2, 32);
            }
        chk(cudaMalloc(&dw, q.size())); chk(cudaMalloc(&dd, d.size()));
        chk(cudaMemcpy(dw, q.data(), q.size(), cudaMemcpyHostToDevice));
        chk(cudaMemcpy(dd, d.data(), d.size(), cudaMemcpyHostToDevice));
    }
    A.w = dw; A.d = (const __half *) dd;
    chk(cudaMalloc(&dx, sizeof(float) * nv * cols));
    chk(cudaMalloc(&dy, sizeof(float) * nv * rows));
    chk(cudaMemcpy(dx, xin, sizeof(float) * nv * cols, cudaMemcpyHostToDevice));
    if (norm_gain) { chk(cudaMalloc(&dg, sizeof(float) * cols)); chk(cudaMemcpy(dg, norm_gain, sizeof(float) * cols, cudaMemcpyHostToDevice)); }
    if (block_dots && wtype == W_Q8_0) { chk(cudaMalloc(&dbd, sizeof(int) * nv * rows * nb)); chk(cudaMemset(dbd, 0, sizeof(int) * nv * rows * nb)); }
    if (ok) {
        GemvArgs a{};
        a.A = A; a.x = (const float *) dx; a.ldx = cols; a.nv = nv; a.norm_g = (const float *) dg; a.eps = eps;
        a.act = act_f32 ? ACT_F32 : ACT_F16; a.y = (float *) dy; a.ldy = rows; a.epi = EPI_STORE;
        a.block_dots = (int *) dbd;
        const int NVt = nv == 1 ? 1 : nv == 2 ? 2 : 8;
        int ncta = 0;
        size_t slice = 0, smem = 0;
        if (!gemv_shape(A, false, dg != nullptr, NVt, n_sm, &ncta, &slice, &smem)) ok = false;
        cudaFuncSetAttribute(k_gemv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX);
        cudaFuncSetAttribute(k_gemv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX);
        cudaFuncSetAttribute(k_gemv<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) QTTS_GEMV_SMEM_MAX);
        if (!ok) {}
        else if (NVt == 1) k_gemv<1><<<ncta, QTTS_WARPS * 32, smem>>>(a, slice);
        else if (NVt == 2) k_gemv<2><<<ncta, QTTS_WARPS * 32, smem>>>(a, slice);
        else k_gemv<8><<<ncta, QTTS_WARPS * 32, smem>>>(a, slice);
        chk(cudaGetLastError());
        chk(cudaDeviceSynchronize());
        if (ok) chk(cudaMemcpy(y, dy, sizeof(float) * nv * rows, cudaMemcpyDeviceToHost));
        if (ok && dbd) chk(cudaMemcpy(block_dots, dbd, sizeof(int) * nv * rows * nb, cudaMemcpyDeviceToHost));
    }
    void * all[] = {dw, dd, dx, dy, dg, dbd};
    for (void * p : all) if (p) cudaFree(p);
    return ok ? 1 : 0;
}

// One sampling decision with the engine's sampler (cb 0 = codebook-0 rules with
// suppression/penalty/EOS bias; cb >= 1 = code-predictor rules).  presence:
// optional [vocab] 0/1 set of earlier codebook-0 tokens.  Returns the token or
// -1 (EOS for cb 0 returns eos_id).
int32_t qtts_op_sample(int32_t device, const float * logits_in, int32_t V, int32_t cb, float temperature, int32_t top_k,
                       float rep_penalty, const int32_t * presence, float eos_bias, int32_t target_frames, int32_t frame,
                       int32_t eos_id, int32_t suppress_start, uint64_t seed) {
    using namespace qtts;
    if (!logits_in || V <= 0 || V > SAMPLE_THREADS * SAMPLE_PER_T) return -1;
    if (cudaSetDevice(device) != cudaSuccess) return -1;
    float * dl = nullptr; DevState * dst = nullptr; SampleParams * dsp = nullptr;
    DevState hs{};
    hs.frame = frame;
    if (presence) for (int i = 0; i < V; ++i) if (presence[i]) hs.presence[i >> 5] |= 1u << (i & 31);
    SampleParams P{};
    P.temperature = temperature; P.top_k = top_k; P.rep_penalty = rep_penalty; P.eos_bias = eos_bias;
    P.target_frames = target_frames; P.eos_id = eos_id; P.suppress_start = suppress_start; P.seed = seed; P.n_cb = 16;
    int tok = -1;
    if (cudaMalloc(&dl, sizeof(float) * V) == cudaSuccess && cudaMalloc(&dst, sizeof(DevState)) == cudaSuccess &&
        cudaMalloc(&dsp, sizeof(SampleParams)) == cudaSuccess) {
        cudaMemcpy(dl, logits_in, sizeof(float) * V, cudaMemcpyHostToDevice);
        cudaMemcpy(dst, &hs, sizeof(hs), cudaMemcpyHostToDevice);
        cudaMemcpy(dsp, &P, sizeof(P), cudaMemcpyHostToDevice);
        k_sample<<<1, SAMPLE_THREADS>>>(dl, V, cb, dst, dsp, nullptr, 0);
        if (cudaDeviceSynchronize() == cudaSuccess && cudaMemcpy(&hs, dst, sizeof(hs), cudaMemcpyDeviceToHost) == cudaSuccess)
            tok = (cb == 0 && hs.done) ? eos_id : hs.codes[cb];
    }
    if (dl) cudaFree(dl);
    if (dst) cudaFree(dst);
    if (dsp) cudaFree(dsp);
    return tok;
}

// ---------------------------------------------------------------- sampler without allocation
// Fixed device scratch for qtts_op_sample_noalloc: the sampler's frame state
// (presence set, stop flag, codes) lives here instead of in memory allocated per
// call.  Every GPU that loads the library holds this array until exit.
#define QTTS_NOALLOC_SCRATCH_BYTES 4096
#define QTTS_NOALLOC_MAX_VOCAB 4096
static __device__ __align__(256) unsigned char g_sample_scratch[QTTS_NOALLOC_SCRATCH_BYTES];
static_assert(sizeof(qtts::DevState) <= QTTS_NOALLOC_SCRATCH_BYTES, "sampler state exceeds the fixed scratch");

namespace qtts {
// Same decision as k_sample, with the frame state in the caller-independent
// scratch.  Clears the state first: the array keeps the previous call's bytes.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_noalloc(const float * logits, int V, int cb, int frame,
                                                                   DevState * st, SampleParams P,
                                                                   const int32_t * presence, int32_t * token_out) {
    for (int i = threadIdx.x; i < 128; i += blockDim.x) {
        uint32_t bits = 0;
        if (presence)
            for (int b = 0; b < 32; ++b) {
                const int t = i * 32 + b;
                if (t < V && presence[t]) bits |= 1u << b;
            }
        st->presence[i] = bits;
    }
    if (threadIdx.x < QTTS_MAX_CB) st->codes[threadIdx.x] = 0;
    if (threadIdx.x == 0) { st->done = 0; st->frame = frame; st->pos = 0; st->n_out = 0; st->n_trailing = 0; }
    __syncthreads();
    const int tok = sample_body<SAMPLE_PER_T>(logits, V, cb, st, P, frame);
    if (threadIdx.x == 0) {
        sample_commit(tok, cb, st, P, nullptr, 0, frame);
        *token_out = (cb == 0 && st->done) ? P.eos_id : st->codes[cb];
    }
}
}  // namespace qtts

// Device address of g_sample_scratch, resolved once per device (host code must
// not pass the symbol itself: on the host it is only a stand-in).
static std::mutex g_scratch_mu;
static void * g_scratch_ptr[64];

int32_t qtts_op_sample_noalloc(int32_t device, const float * logits, int32_t V, int32_t cb, float temperature,
                               int32_t top_k, float rep_penalty, const int32_t * presence, float eos_bias,
                               int32_t target_frames, int32_t frame, int32_t eos_id, int32_t suppress_start,
                               uint64_t seed, int32_t * token_out, void * stream) {
    using namespace qtts;
    if (V > QTTS_NOALLOC_MAX_VOCAB) {
        fprintf(stderr, "qtts_op_sample_noalloc: vocabulary %d exceeds the fixed scratch limit of %d tokens\n", V,
                QTTS_NOALLOC_MAX_VOCAB);
        return -2;
    }
    if (!logits || !token_out || V <= 0 || cb < 0 || cb >= QTTS_MAX_CB || device < 0 || device >= 64) return 0;
    if (cudaSetDevice(device) != cudaSuccess) return 0;
    void * scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (!g_scratch_ptr[device]) {
            // First call on this device: resolve the array's device address and
            // make the kernel's module resident now (under CUDA's lazy module
            // loading, loading a module allocates device memory and may
            // synchronise); later calls only launch.
            cudaFuncAttributes fa{};
            if (cudaGetSymbolAddress(&g_scratch_ptr[device], g_sample_scratch) != cudaSuccess ||
                cudaFuncGetAttributes(&fa, k_sample_noalloc) != cudaSuccess) {
                g_scratch_ptr[device] = nullptr;
                return 0;
            }
        }
        scratch = g_scratch_ptr[device];
    }
    SampleParams P{};
    P.temperature = temperature; P.top_k = top_k; P.rep_penalty = rep_penalty; P.eos_bias = eos_bias;
    P.target_frames = target_frames; P.eos_id = eos_id; P.suppress_start = suppress_start; P.seed = seed;
    P.n_cb = QTTS_MAX_CB;
    k_sample_noalloc<<<1, SAMPLE_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        logits, V, cb, frame, static_cast<DevState *>(scratch), P, presence, token_out);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

qtts_engine * qtts_create(const char * gguf_path, int32_t device) {
    qtts::g_create_error.clear();
    if (!gguf_path) { qtts::g_create_error = "gguf_path is null"; return nullptr; }
    auto e = std::make_unique<Engine>();
    if (!e->load(gguf_path, device)) {
        qtts::g_create_error = e->err;
        return nullptr;
    }
    return reinterpret_cast<qtts_engine *>(e.release());
}

const char * qtts_create_error(void) { return qtts::g_create_error.c_str(); }

void qtts_destroy(qtts_engine * h) { delete reinterpret_cast<Engine *>(h); }

const char * qtts_get_error(const qtts_engine * h) {
    return h ? reinterpret_cast<const Engine *>(h)->err.c_str() : "null engine";
}

int32_t qtts_get_config(const qtts_engine * h, qtts_config * out) {
    if (!h || !out) return 0;
    *out = reinterpret_cast<const Engine *>(h)->cfg;
    return 1;
}

void qtts_set_n_threads(qtts_engine *, int32_t) {}

#define ENG(h) Engine & E = *reinterpret_cast<Engine *>(h); cudaSetDevice(E.dev)

int32_t qtts_init_kv_cache(qtts_engine * h, int32_t n_ctx) { if (!h) return 0; ENG(h); return E.init_kv(n_ctx) ? 1 : 0; }
void qtts_clear_kv_cache(qtts_engine * h) { if (h) reinterpret_cast<Engine *>(h)->n_used = 0; }
int32_t qtts_init_code_pred_kv_cache(qtts_engine * h, int32_t n_ctx) { if (!h) return 0; ENG(h); return E.init_cp_kv(n_ctx) ? 1 : 0; }
void qtts_clear_code_pred_kv_cache(qtts_engine *) {}

int32_t qtts_forward_prefill(qtts_engine * h, const float * embd, int32_t n, int32_t n_past, float * hidden_out,
                             float * logits_out) {
    if (!h) return 0;
    ENG(h);
    if (!embd) { E.err = "prefill_embd is null"; return 0; }
    E.sess.active = false;
    return E.prefill(embd, n, n_past, hidden_out, logits_out) ? 1 : 0;
}

int32_t qtts_forward_step(qtts_engine * h, const float * embd, int32_t n_past, float * logits_out, float * hidden_out) {
    if (!h) return 0;
    ENG(h);
    if (!embd) { E.err = "step_embd is null"; return 0; }
    E.sess.active = false;
    if (E.n_ctx == 0 && !E.init_kv(std::max(256, n_past + 1 + 16))) return 0;
    if (n_past + 1 > E.n_ctx) { E.err = "Context length exceeded"; return 0; }
    const int H = E.cfg.hidden_size;
    if (cudaMemcpyAsync(E.x, embd, sizeof(float) * H, cudaMemcpyHostToDevice, E.stream) != cudaSuccess) { E.err = "upload"; return 0; }
    if (!E.enqueue_talker_step(nullptr, n_past, nullptr, false)) return 0;
    E.last_hidden.resize(H);
    cudaMemcpyAsync(E.last_hidden.data(), E.hidden, sizeof(float) * H, cudaMemcpyDeviceToHost, E.stream);
    if (logits_out) cudaMemcpyAsync(logits_out, E.logits, sizeof(float) * E.cfg.codec_vocab_size, cudaMemcpyDeviceToHost, E.stream);
    if (!E.sync("forward_step")) return 0;
    if (hidden_out) memcpy(hidden_out, E.last_hidden.data(), sizeof(float) * H);
    E.n_used = n_past + 1;
    return 1;
}

int32_t qtts_forward_text(qtts_engine * h, const int32_t * toks, int32_t n, const float * spk, int32_t n_past,
                          float * hidden_out) {
    if (!h) return 0;
    ENG(h);
    if (!toks) { E.err = "text_tokens is null"; return 0; }
    if (n <= 0) { E.err = "n_tokens must be > 0"; return 0; }
    std::vector<float> proj;
    if (!E.project_text(toks, n, proj)) return 0;
    const int H = E.cfg.hidden_size;
    if (spk)
        for (int t = 0; t < n; ++t)
            for (int d = 0; d < H; ++d) proj[(size_t) t * H + d] += spk[d];
    return qtts_forward_prefill(h, proj.data(), n, n_past, hidden_out, nullptr);
}

int32_t qtts_forward_codec(qtts_engine * h, int32_t tok, int32_t n_past, float * logits_out) {
    if (!h) return 0;
    ENG(h);
    std::vector<float> row;
    if (!E.lookup(0, &tok, 1, row)) return 0;
    return qtts_forward_step(h, row.data(), n_past, logits_out, nullptr);
}

int32_t qtts_get_hidden_states(const qtts_engine * h, float * out) {
    if (!h || !out) return 0;
    const Engine & E = *reinterpret_cast<const Engine *>(h);
    if (E.sess.active) {
        cudaSetDevice(E.dev);
        cudaMemcpy(out, E.hidden, sizeof(float) * E.cfg.hidden_size, cudaMemcpyDeviceToHost);
        return 1;
    }
    if (E.last_hidden.empty()) return 0;
    memcpy(out, E.last_hidden.data(), sizeof(float) * E.last_hidden.size());
    return 1;
}

int32_t qtts_predict_codes_autoregressive(qtts_engine * h, const float * hidden, int32_t cb0, float temperature,
                                          int32_t top_k, int32_t * codes_out) {
    if (!h) return 0;
    ENG(h);
    const qtts_config & c = E.cfg;
    if (!hidden || !codes_out) { E.err = "null argument"; return 0; }
    if (cb0 < 0 || cb0 >= c.codec_vocab_size) { E.err = "Embedding token ID out of range"; return 0; }
    E.sess.active = false;
    qtts::DevState hs{};
    hs.codes[0] = cb0;
    hs.frame = (int) E.api_calls++;
    qtts::SampleParams P{};
    P.temperature = temperature; P.top_k = top_k; P.rep_penalty = 1.0f; P.eos_id = c.codec_eos_id;
    P.suppress_start = c.codec_vocab_size; P.seed = E.seed; P.n_cb = c.n_codebooks;
    cudaMemcpyAsync(E.hidden, hidden, sizeof(float) * c.hidden_size, cudaMemcpyHostToDevice, E.stream);
    cudaMemcpyAsync(E.st, &hs, sizeof(hs), cudaMemcpyHostToDevice, E.stream);
    cudaMemcpyAsync(E.sp, &P, sizeof(P), cudaMemcpyHostToDevice, E.stream);
    int saved_cap = E.codes_cap;
    E.codes_cap = 0;   // no frame output rows
    const bool ok = E.enqueue_cp(false);
    E.codes_cap = saved_cap;
    if (!ok) return 0;
    cudaMemcpyAsync(&hs, E.st, sizeof(hs), cudaMemcpyDeviceToHost, E.stream);
    if (!E.sync("predict_codes_autoregressive")) return 0;
    for (int g = 1; g < c.n_codebooks; ++g) codes_out[g - 1] = hs.codes[g];
    return 1;
}

// Legacy non-autoregressive predictor (build_code_pred_graph,
// src/tts_transformer.cpp:1771-1899): one row, no RoPE, attention over itself
// (softmax of one score is exactly 1, so the output is V), no output norm, all
// heads on the final row.
int32_t qtts_predict_codes(qtts_engine * h, const float * hidden, const int32_t * prev_codes, float * logits_out) {
    if (!h) return 0;
    ENG(h);
    const qtts_config & c = E.cfg;
    const int H = c.hidden_size, NG = c.n_codebooks - 1, V1 = c.code_pred_vocab_size;
    if (!hidden || !logits_out) { E.err = "null argument"; return 0; }
    E.sess.active = false;
    std::vector<float> row(hidden, hidden + H), r;
    if (prev_codes)
        for (int cb = 0; cb < NG; ++cb) {
            if (!E.lookup(cb + 1, prev_codes + cb, 1, r)) return 0;
            for (int d = 0; d < H; ++d) row[d] += r[d];
        }
    cudaMemcpyAsync(E.xcp, row.data(), sizeof(float) * H, cudaMemcpyHostToDevice, E.stream);
    for (auto & l : E.CPL) {
        E.gemv(l.qkv, nullptr, E.xcp, H, 1, l.attn_norm, qtts::ACT_F16, E.qkv, E.QKVD(), nullptr, 0, qtts::EPI_STORE, nullptr, 0, nullptr);
        qtts::AttnArgs aa{};
        aa.q = E.qkv; aa.ldq = E.QKVD(); aa.kf = E.qkv + E.QD(); aa.vf = E.qkv + E.QD() + E.KD(); aa.ldkv = E.QKVD();
        aa.f32_mode = 1; aa.n_heads = c.n_attention_heads; aa.n_kv_heads = c.n_key_value_heads;
        aa.pos_static = 0; aa.scale = 1.0f / sqrtf(128.0f); aa.out = E.att; aa.ldo = E.QD(); aa.st = E.st;
        qtts::k_attention<<<dim3(c.n_key_value_heads, 1), qtts::ATT_THREADS,
                            qtts::attn_smem_bytes(1, c.n_attention_heads / c.n_key_value_heads), E.stream>>>(aa);
        E.gemv(l.o, nullptr, E.att, E.QD(), 1, nullptr, qtts::ACT_F16, E.xcp, H, E.xcp, H, qtts::EPI_RESID, nullptr, 0, nullptr);
        E.gemv(l.gate, &l.up, E.xcp, H, 1, l.ffn_norm, qtts::ACT_F16, E.hbuf, c.code_pred_intermediate_size, nullptr, 0,
               qtts::EPI_SWIGLU, nullptr, 0, nullptr);
        E.gemv(l.down, nullptr, E.hbuf, c.code_pred_intermediate_size, 1, nullptr, qtts::ACT_F32, E.xcp, H, E.xcp, H,
               qtts::EPI_RESID, nullptr, 0, nullptr);
    }
    for (int g = 0; g < NG; ++g)
        E.gemv(E.cp_head[g], nullptr, E.xcp, H, 1, nullptr, qtts::ACT_F16, E.cp_logits + (size_t) g * V1, V1, nullptr, 0,
               qtts::EPI_STORE, nullptr, 0, nullptr);
    cudaMemcpyAsync(logits_out, E.cp_logits, sizeof(float) * NG * V1, cudaMemcpyDeviceToHost, E.stream);
    return E.sync("predict_codes") ? 1 : 0;
}

int32_t qtts_project_text(qtts_engine * h, const int32_t * toks, int32_t n, float * out) {
    if (!h || !toks || !out) return 0;
    ENG(h);
    std::vector<float> v;
    if (!E.project_text(toks, n, v)) return 0;
    memcpy(out, v.data(), v.size() * 4);
    return 1;
}

int32_t qtts_lookup_embedding_rows(qtts_engine * h, int32_t table, const int32_t * ids, int32_t n, float * out) {
    if (!h || !ids || !out) return 0;
    ENG(h);
    std::vector<float> v;
    if (!E.lookup(table, ids, n, v)) return 0;
    memcpy(out, v.data(), v.size() * 4);
    return 1;
}

int32_t qtts_generate_begin(qtts_engine * h, const qtts_generate_params * p) {
    if (!h || !p) return -1;
    ENG(h);
    if (p->max_len <= 0) { E.err = ""; E.sess = qtts::GenSession{}; return 0; }
    return E.begin(p);
}

int32_t qtts_run_frames(qtts_engine * h, int32_t n, int32_t * codes_out) {
    if (!h) return -1;
    ENG(h);
    return E.run_frames(n, codes_out);
}

int32_t qtts_generate_rewind(qtts_engine * h) {
    if (!h) return -1;
    ENG(h);
    return E.rewind();
}

int32_t qtts_codes_device(qtts_engine * h, const int32_t ** codes_dev, int32_t * n_frames) {
    if (!h || !codes_dev) return -1;
    ENG(h);
    if (!E.d_codes) { E.err = "no generation has run"; return -1; }
    *codes_dev = E.d_codes;
    if (n_frames) *n_frames = E.sess.produced;
    return 0;
}

int32_t qtts_generate(qtts_engine * h, const qtts_generate_params * p, qtts_frame_callback on_frame, void * user,
                      int32_t * codes_out, int32_t * n_frames_out) {
    if (!h || !p) return 0;
    ENG(h);
    if (n_frames_out) *n_frames_out = 0;
    if (p->max_len <= 0) return 1;
    const int NCB = E.cfg.n_codebooks;
    const auto t_call = std::chrono::steady_clock::now();
    if (E.begin(p) < 0) return 0;
    std::vector<int32_t> out;
    out.reserve((size_t) p->max_len * NCB);
    std::vector<int32_t> chunk;
    std::vector<std::vector<int32_t>> rep;
    int run = 0, run_start = 0, emitted = 0;
    bool stop = false, eos = false;
    const int CH = 16;
    while (!stop && emitted < p->max_len) {
        chunk.resize((size_t) CH * NCB);
        const int got = E.run_frames(std::min(CH, p->max_len - emitted), chunk.data());
        if (got < 0) return 0;
        for (int f = 0; f < got && !stop; ++f) {
            const int32_t * fc = chunk.data() + (size_t) f * NCB;
            out.insert(out.end(), fc, fc + NCB);
            const int frame = emitted++;
            if (on_frame && !on_frame(fc, NCB, frame, user)) { stop = true; break; }
            // repetition-loop detection (src/tts_transformer.cpp:3217-3254)
            if (p->rep_loop_detect) rep.emplace_back(fc, fc + NCB);
            const size_t nf = rep.size();
            bool is_rep = false;
            for (int back = 1; back <= 6 && !is_rep && (size_t) back < nf; ++back) {
                int match = 0;
                for (int cb = 0; cb < NCB; ++cb) if (rep[nf - 1][cb] == rep[nf - 1 - back][cb]) ++match;
                if (match >= 10) is_rep = true;
            }
            if (is_rep) { if (run == 0) run_start = (int)(nf - 1); ++run; } else run = 0;
            if (run >= 5) {
                fprintf(stderr, "  Repetition loop detected at frame %d, truncating %d frames\n", (int)(nf - 1), run);
                out.resize((size_t) run_start * NCB);
                stop = true;
            }
        }
        if (E.sess.done) { eos = true; break; }
        if (got == 0) break;
    }
    // attention rows: one per talker step the reference would have run
    if (E.attn_dump) {
        const size_t keep = eos && !stop ? (size_t) emitted : (size_t) std::max(0, emitted - 1);
        if (E.attn_rows.size() > keep) E.attn_rows.resize(keep);
    }
    const int n = (int)(out.size() / NCB);
    if (codes_out) memcpy(codes_out, out.data(), out.size() * sizeof(int32_t));
    if (n_frames_out) *n_frames_out = n;
    E.sess.active = false;
    E.stages.total_ms = (float) std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_call).count();
    return 1;
}

void qtts_set_seed(qtts_engine * h, uint64_t s) { if (h) reinterpret_cast<Engine *>(h)->seed = s; }

int32_t qtts_set_debug_logits(qtts_engine * h, float * tl, float * cl, int32_t cap) {
    if (!h) return 0;
    Engine & E = *reinterpret_cast<Engine *>(h);
    E.h_dbg_t = tl; E.h_dbg_cp = cl; E.h_dbg_cap = cap > 0 ? cap : 0;
    return 1;
}

int32_t qtts_set_attn_dump(qtts_engine * h, int32_t enabled, int32_t layer) {
    if (!h) return 0;
    Engine & E = *reinterpret_cast<Engine *>(h);
    if (layer < 0 || layer >= E.cfg.n_layers) { E.err = "attn dump layer out of range"; return 0; }
    E.attn_dump = enabled != 0;
    E.attn_layer = layer;
    E.graph_ok = false;
    return 1;
}

int32_t qtts_attn_rows(const qtts_engine * h) { return h ? (int32_t) reinterpret_cast<const Engine *>(h)->attn_rows.size() : 0; }

int32_t qtts_attn_row(const qtts_engine * h, int32_t r, float * out, int32_t cap) {
    if (!h) return -1;
    const Engine & E = *reinterpret_cast<const Engine *>(h);
    if (r < 0 || r >= (int) E.attn_rows.size()) return -1;
    const auto & row = E.attn_rows[r];
    if (out) memcpy(out, row.data(), sizeof(float) * std::min<size_t>(row.size(), (size_t) std::max(cap, 0)));
    return (int32_t) row.size();
}

// Runs up to n frames of the active generation eagerly (no graph) with CUDA
// events around every launch; out[class] = {launches, total ms, algorithmic bytes}.
int32_t qtts_profile_frames(qtts_engine * h, int32_t n, qtts_kernel_stats * out, int32_t n_classes) {
    if (!h || !out) return -1;
    ENG(h);
    if (!E.sess.active) { E.err = "no active generation"; return -1; }
    n = std::min(n, E.sess.max_len - E.sess.produced);
    E.profiling = true;
    E.prof_evs.clear();
    E.ev_used = 0;
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) ok = E.frame_mode == Engine::FM_FUSED ? E.enqueue_frame_ff() : E.enqueue_frame();
    E.profiling = false;
    qtts::DevState hs;
    cudaMemcpyAsync(&hs, E.st, sizeof(hs), cudaMemcpyDeviceToHost, E.stream);
    if (!ok || !E.sync("profile frames")) return -1;
    for (int c = 0; c < n_classes; ++c) out[c] = qtts_kernel_stats{0, 0.0f, 0.0};
    for (auto & p : E.prof_evs) {
        if (p.cls >= n_classes) continue;
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, p.a, p.b);
        out[p.cls].launches += 1;
        out[p.cls].total_ms += ms;
        out[p.cls].bytes += p.bytes;
    }
    const int got = hs.n_out - E.sess.produced;
    E.sess.produced = hs.n_out;
    E.sess.done = hs.done != 0;
    return got;
}


int32_t qtts_frame_trace(const qtts_engine * h, unsigned long long * out, int32_t cap, int32_t * kinds, int32_t kcap) {
    if (!h) return -1;
    const Engine & E = *reinterpret_cast<const Engine *>(h);
    if (!E.d_fftrace) return 0;
    const int n = (int) E.ff_kinds.size();
    for (int i = 0; i < n && i < kcap; ++i) kinds[i] = E.ff_kinds[i];
    const size_t words = (size_t) n * qtts::FF_TRACE_CTAS * qtts::FF_TRACE_N;
    if (out && cap > 0) cudaMemcpy(out, E.d_fftrace, sizeof(unsigned long long) * std::min(words, (size_t) cap), cudaMemcpyDeviceToHost);
    return n;
}

int32_t qtts_get_frame_mode(const qtts_engine * h) {
    if (!h) return -1;
    return reinterpret_cast<const Engine *>(h)->frame_mode;
}

int32_t qtts_set_stage_timing(qtts_engine * h, int32_t enabled) {
    if (!h) return 0;
    reinterpret_cast<Engine *>(h)->stage_timing = enabled != 0;
    return 1;
}

int32_t qtts_get_stage_timing(const qtts_engine * h, qtts_stage_timing * out) {
    if (!h || !out) return 0;
    *out = reinterpret_cast<const Engine *>(h)->stages;
    return 1;
}

int32_t qtts_get_timing(const qtts_engine * h, qtts_timing * out) {
    if (!h || !out) return 0;
    *out = reinterpret_cast<const Engine *>(h)->timing;
    return 1;
}

}  // extern "C"

// ---------------------------------------------------------------- batched frame loop (configs 4, 5)
struct qtts_batch { qtts::BatchEngine be; };

qtts_batch * qtts_batch_create(qtts_engine * h, int32_t max_batch, int32_t max_positions, int32_t max_frames) {
    if (!h || max_positions <= 0 || max_frames <= 0) return nullptr;
    ENG(h);
    auto * b = new qtts_batch();
    if (!b->be.create(&E, max_batch, max_positions, max_frames)) {
        E.err = b->be.err;
        delete b;
        return nullptr;
    }
    return b;
}

int32_t qtts_batch_begin(qtts_batch * b, int32_t n, const qtts_generate_params * params) {
    if (!b || !params) return -1;
    cudaSetDevice(b->be.dev);
    return b->be.begin(n, params);
}

int32_t qtts_batch_run(qtts_batch * b, int32_t n_frames) {
    if (!b) return -1;
    cudaSetDevice(b->be.dev);
    return b->be.run(n_frames);
}

int32_t qtts_batch_codes(qtts_batch * b, int32_t * codes_out, int32_t * n_frames_out) {
    if (!b) return 0;
    cudaSetDevice(b->be.dev);
    return b->be.read_codes(codes_out, n_frames_out) ? 1 : 0;
}

int32_t qtts_batch_codes_device(qtts_batch * b, const int32_t ** codes_dev, int32_t * n_frames_out) {
    if (!b || !codes_dev || b->be.B <= 0) return -1;
    *codes_dev = b->be.codes;
    if (n_frames_out) for (int i = 0; i < b->be.B; ++i) n_frames_out[i] = b->be.produced[i];
    return 0;
}

int32_t qtts_batch_timing(const qtts_batch * b, float * frames_ms, int32_t * seq_frames, int32_t * launches_per_frame) {
    if (!b) return 0;
    if (frames_ms) *frames_ms = b->be.frames_ms;
    if (seq_frames) *seq_frames = b->be.seq_frames;
    if (launches_per_frame) *launches_per_frame = b->be.launches;
    return 1;
}

int32_t qtts_batch_profile(qtts_batch * b, int32_t n_frames, float * ms_per_frame, int32_t * launches_per_frame) {
    if (!b || n_frames <= 0 || !ms_per_frame || !launches_per_frame) return 0;
    cudaSetDevice(b->be.dev);
    return b->be.profile(n_frames, ms_per_frame, launches_per_frame) ? 1 : 0;
}

const char * qtts_batch_error(const qtts_batch * b) { return b ? b->be.err.c_str() : "null batch"; }

void qtts_batch_free(qtts_batch * b) { delete b; }
