// tts_transformer.cpp — qwen3_tts::TTSTransformer (drop-in for the reference's
// src/tts_transformer.cpp) implemented over the B200 engine's C ABI.  Error
// convention as the reference: bool return + get_error(), no exceptions.
#include "../../include/tts_transformer.h"
#include "../../include/qwen3tts_b200.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

namespace qwen3_tts {

TTSTransformer::TTSTransformer() { seed_ = ((uint64_t) std::random_device{}() << 32) | std::random_device{}(); }

TTSTransformer::~TTSTransformer() { unload_model(); }

void TTSTransformer::unload_model() {
    if (engine_) { qtts_destroy(engine_); engine_ = nullptr; }
    free_transformer_model(model_);
    free_tts_kv_cache(cache_);
    last_hidden_.clear();
}

bool TTSTransformer::load_model(const std::string & model_path) {
    unload_model();
    engine_ = qtts_create(model_path.c_str(), -1);
    if (!engine_) { error_msg_ = qtts_create_error(); return false; }
    qtts_config c{};
    qtts_get_config(engine_, &c);
    tts_transformer_config & m = model_.config;
    m.text_vocab_size = c.text_vocab_size; m.text_embd_dim = c.text_embd_dim;
    m.hidden_size = c.hidden_size; m.n_layers = c.n_layers; m.n_attention_heads = c.n_attention_heads;
    m.n_key_value_heads = c.n_key_value_heads; m.intermediate_size = c.intermediate_size; m.head_dim = c.head_dim;
    m.rms_norm_eps = c.rms_norm_eps; m.rope_theta = c.rope_theta;
    for (int i = 0; i < 3; ++i) m.mrope_section[i] = c.mrope_section[i];
    m.codec_vocab_size = c.codec_vocab_size; m.n_codebooks = c.n_codebooks;
    m.code_pred_layers = c.code_pred_layers; m.code_pred_vocab_size = c.code_pred_vocab_size;
    m.code_pred_hidden_size = c.code_pred_hidden_size; m.code_pred_intermediate_size = c.code_pred_intermediate_size;
    m.code_pred_rope_theta = c.code_pred_rope_theta;
    m.codec_pad_id = c.codec_pad_id; m.codec_bos_id = c.codec_bos_id; m.codec_eos_id = c.codec_eos_id;
    m.tts_bos_token_id = c.tts_bos_token_id; m.tts_eos_token_id = c.tts_eos_token_id; m.tts_pad_token_id = c.tts_pad_token_id;
    m.codec_think_id = c.codec_think_id; m.codec_nothink_id = c.codec_nothink_id;
    m.codec_think_bos_id = c.codec_think_bos_id; m.codec_think_eos_id = c.codec_think_eos_id;
    m.english_language_id = c.english_language_id;
    cache_.head_dim = c.head_dim; cache_.n_kv_heads = c.n_key_value_heads; cache_.n_layers = c.n_layers;
    qtts_set_seed(engine_, seed_);
    fprintf(stderr, "  TTSTransformer backend: B200 engine (%s weights)\n", c.weight_type == 8 ? "Q8_0" : "F16");
    return true;
}

void TTSTransformer::set_n_threads(int32_t n_threads) { if (engine_) qtts_set_n_threads(engine_, n_threads); }

void TTSTransformer::set_seed(uint64_t seed) { seed_ = seed; if (engine_) qtts_set_seed(engine_, seed); }

void TTSTransformer::set_attn_dump(const std::string & path, int layer) {
    attn_dump_ = !path.empty();
    attn_dump_path_ = path;
    attn_dump_layer_ = layer;
    if (engine_) qtts_set_attn_dump(engine_, attn_dump_ ? 1 : 0, layer);
}

#define NEED_MODEL() do { if (!engine_) { error_msg_ = "Model not loaded"; return false; } } while (0)

bool TTSTransformer::init_kv_cache(int32_t n_ctx) {
    NEED_MODEL();
    if (!qtts_init_kv_cache(engine_, n_ctx)) { error_msg_ = qtts_get_error(engine_); return false; }
    cache_.n_ctx = n_ctx; cache_.n_used = 0;
    return true;
}
void TTSTransformer::clear_kv_cache() { cache_.n_used = 0; if (engine_) qtts_clear_kv_cache(engine_); }
bool TTSTransformer::init_code_pred_kv_cache(int32_t n_ctx) {
    NEED_MODEL();
    if (!qtts_init_code_pred_kv_cache(engine_, n_ctx)) { error_msg_ = qtts_get_error(engine_); return false; }
    return true;
}
void TTSTransformer::clear_code_pred_kv_cache() { if (engine_) qtts_clear_code_pred_kv_cache(engine_); }

bool TTSTransformer::forward_text(const int32_t * text_tokens, int32_t n_tokens, const float * speaker_embd,
                                  int32_t n_past, std::vector<float> & output) {
    NEED_MODEL();
    if (!text_tokens) { error_msg_ = "text_tokens is null"; return false; }
    if (n_tokens <= 0) { error_msg_ = "n_tokens must be > 0"; return false; }
    output.resize((size_t) n_tokens * model_.config.hidden_size);
    if (!qtts_forward_text(engine_, text_tokens, n_tokens, speaker_embd, n_past, output.data())) {
        error_msg_ = qtts_get_error(engine_); return false;
    }
    last_hidden_.assign(output.end() - model_.config.hidden_size, output.end());
    return true;
}

bool TTSTransformer::forward_prefill(const float * prefill_embd, int32_t n_tokens, int32_t n_past,
                                     std::vector<float> & output, std::vector<float> * logits_out) {
    NEED_MODEL();
    if (!prefill_embd) { error_msg_ = "prefill_embd is null"; return false; }
    if (n_tokens <= 0) { error_msg_ = "n_tokens must be > 0"; return false; }
    output.resize((size_t) n_tokens * model_.config.hidden_size);
    if (logits_out) logits_out->resize(model_.config.codec_vocab_size);
    if (!qtts_forward_prefill(engine_, prefill_embd, n_tokens, n_past, output.data(),
                              logits_out ? logits_out->data() : nullptr)) {
        error_msg_ = qtts_get_error(engine_); return false;
    }
    last_hidden_.assign(output.end() - model_.config.hidden_size, output.end());
    cache_.n_used = n_past + n_tokens;
    return true;
}

bool TTSTransformer::forward_codec(int32_t codec_token, int32_t n_past, std::vector<float> & output) {
    NEED_MODEL();
    output.resize(model_.config.codec_vocab_size);
    if (!qtts_forward_codec(engine_, codec_token, n_past, output.data())) { error_msg_ = qtts_get_error(engine_); return false; }
    last_hidden_.resize(model_.config.hidden_size);
    qtts_get_hidden_states(engine_, last_hidden_.data());
    return true;
}

bool TTSTransformer::forward_step(const float * step_embd, int32_t n_past, std::vector<float> & output,
                                  std::vector<float> * hidden_out) {
    NEED_MODEL();
    if (!step_embd) { error_msg_ = "step_embd is null"; return false; }
    output.resize(model_.config.codec_vocab_size);
    last_hidden_.resize(model_.config.hidden_size);
    if (!qtts_forward_step(engine_, step_embd, n_past, output.data(), last_hidden_.data())) {
        error_msg_ = qtts_get_error(engine_); return false;
    }
    if (hidden_out) *hidden_out = last_hidden_;
    cache_.n_used = n_past + 1;
    return true;
}

bool TTSTransformer::get_hidden_states(std::vector<float> & hidden) const {
    if (last_hidden_.empty()) return false;
    hidden = last_hidden_;
    return true;
}

bool TTSTransformer::predict_codes(const float * hidden, const int32_t * prev_codes, std::vector<float> & output) {
    NEED_MODEL();
    output.resize((size_t)(model_.config.n_codebooks - 1) * model_.config.code_pred_vocab_size);
    if (!qtts_predict_codes(engine_, hidden, prev_codes, output.data())) { error_msg_ = qtts_get_error(engine_); return false; }
    return true;
}

bool TTSTransformer::predict_codes_autoregressive(const float * hidden, int32_t codebook_0_token,
                                                  std::vector<int32_t> & output, float temperature, int32_t top_k) {
    NEED_MODEL();
    output.resize(model_.config.n_codebooks - 1);
    if (!qtts_predict_codes_autoregressive(engine_, hidden, codebook_0_token, temperature, top_k, output.data())) {
        error_msg_ = qtts_get_error(engine_); return false;
    }
    return true;
}

namespace {
// Stage timing report: compiled in with QWEN3_TTS_TIMING as in the reference, or
// switched on at run time with the environment variable QWEN3_TTS_TIMING=1 (the
// library is prebuilt).
bool timing_requested() {
#ifdef QWEN3_TTS_TIMING
    return true;
#else
    const char * v = getenv("QWEN3_TTS_TIMING");
    return v && *v && strcmp(v, "0") != 0;
#endif
}

// The layout of the reference's report (src/tts_transformer.cpp:3311-3353).  The
// frame graph is captured once per session, so graph build and allocation cost
// nothing per frame; the device stage times are CUDA-event times.
void print_timing_report(const qtts_stage_timing & t) {
    const int nf = t.frames;
    auto per = [nf](double ms) { return nf > 0 ? ms / nf : 0.0; };
    fprintf(stderr, "\n=== Detailed Generation Timing (%d frames) ===\n", nf);
    fprintf(stderr, "\n  Prefill:\n");
    fprintf(stderr, "    Build graph:      %8.1f ms\n", (double) t.prefill_build_ms);
    fprintf(stderr, "    Forward total:    %8.1f ms\n", (double) t.prefill_forward_ms);
    fprintf(stderr, "      Graph build:    %8.1f ms\n", 0.0);
    fprintf(stderr, "      Graph alloc:    %8.1f ms\n", 0.0);
    fprintf(stderr, "      Compute:        %8.1f ms\n", (double) t.prefill_forward_ms);
    fprintf(stderr, "      Data I/O:       %8.1f ms\n", 0.0);
    fprintf(stderr, "\n  Talker forward_step (total / per-frame):\n");
    fprintf(stderr, "    Total:            %8.1f ms   (%.3f ms/frame)\n", (double) t.talker_ms, per(t.talker_ms));
    fprintf(stderr, "      Compute:        %8.1f ms   (%.3f ms/frame)\n", (double) t.talker_ms, per(t.talker_ms));
    fprintf(stderr, "\n  Code predictor (total / per-frame):\n");
    fprintf(stderr, "    Backend:          B200 engine\n");
    fprintf(stderr, "    Total:            %8.1f ms   (%.3f ms/frame)\n", (double) t.code_pred_ms, per(t.code_pred_ms));
    fprintf(stderr, "      Compute:        %8.1f ms   (%.3f ms/frame)\n", (double) t.code_pred_ms, per(t.code_pred_ms));
    fprintf(stderr, "\n  Embed lookups:      %8.1f ms   (%.3f ms/frame)  (with the samplers)\n",
            (double) t.sample_embed_ms, per(t.sample_embed_ms));
    const double accounted = (double) t.prefill_build_ms + t.prefill_forward_ms + t.talker_ms + t.code_pred_ms +
                             t.sample_embed_ms;
    fprintf(stderr, "  Other/overhead:     %8.1f ms\n", (double) t.total_ms - accounted);
    fprintf(stderr, "  -----------------------------------------\n");
    fprintf(stderr, "  Total generate:     %8.1f ms\n", (double) t.total_ms);
    if (nf > 0)
        fprintf(stderr, "  Throughput:         %8.3f ms/frame (%.1f frames/s)\n", t.total_ms / nf, 1000.0 * nf / t.total_ms);
}

struct CbCtx { const TTSTransformer::FrameCallback * cb; };
int32_t trampoline(const int32_t * codes, int32_t n, int32_t frame, void * user) {
    auto * c = static_cast<CbCtx *>(user);
    return (*c->cb)(codes, n, frame) ? 1 : 0;
}
}  // namespace

bool TTSTransformer::generate_impl(const void * vp, std::vector<int32_t> & output, const FrameCallback & on_frame) {
    const auto * p = static_cast<const qtts_generate_params *>(vp);
    attn_rows_.clear();
    if (p->max_len <= 0) { output.clear(); return true; }
    output.assign((size_t) p->max_len * model_.config.n_codebooks, 0);
    CbCtx ctx{&on_frame};
    int32_t n = 0;
    const bool timed = timing_requested();
    if (timed) qtts_set_stage_timing(engine_, 1);
    const bool ok = qtts_generate(engine_, p, on_frame ? trampoline : nullptr, &ctx, output.data(), &n) != 0;
    if (timed) {
        qtts_stage_timing t{};
        qtts_get_stage_timing(engine_, &t);
        qtts_set_stage_timing(engine_, 0);
        if (ok) print_timing_report(t);
    }
    if (!ok) {
        error_msg_ = qtts_get_error(engine_);
        output.clear();
        return false;
    }
    output.resize((size_t) n * model_.config.n_codebooks);
    last_hidden_.resize(model_.config.hidden_size);
    qtts_get_hidden_states(engine_, last_hidden_.data());
    if (attn_dump_) {
        const int32_t rows = qtts_attn_rows(engine_);
        for (int32_t r = 0; r < rows; ++r) {
            std::vector<float> row((size_t) qtts_attn_row(engine_, r, nullptr, 0));
            qtts_attn_row(engine_, r, row.data(), (int32_t) row.size());
            attn_rows_.push_back(std::move(row));
        }
    }
    write_attn_dump();
    return true;
}

bool TTSTransformer::generate(const int32_t * text_tokens, int32_t n_tokens, const float * speaker_embd, int32_t max_len,
                              std::vector<int32_t> & output, int32_t language_id, float repetition_penalty,
                              float temperature, int32_t top_k, const int32_t * instruct_tokens, int32_t n_instruct,
                              float eos_bias, int32_t target_frames, bool rep_loop_detect,
                              const FrameCallback & on_frame) {
    attn_rows_.clear();
    NEED_MODEL();
    if (!text_tokens) { error_msg_ = "text_tokens is null"; return false; }
    if (n_tokens < 4) { error_msg_ = "Need at least 4 text tokens for generation"; return false; }
    qtts_generate_params p{};
    p.text_tokens = text_tokens; p.n_tokens = n_tokens; p.speaker_embd = speaker_embd; p.max_len = max_len;
    p.language_id = language_id; p.repetition_penalty = repetition_penalty; p.temperature = temperature;
    p.top_k = top_k; p.instruct_tokens = instruct_tokens; p.n_instruct = n_instruct; p.eos_bias = eos_bias;
    p.target_frames = target_frames; p.rep_loop_detect = rep_loop_detect ? 1 : 0; p.seed = seed_;
    return generate_impl(&p, output, on_frame);
}

bool TTSTransformer::generate_icl(const int32_t * text_tokens, int32_t n_tokens, const int32_t * ref_text_tokens,
                                  int32_t n_ref_text, const int32_t * ref_codec_tokens, int32_t n_ref_frames,
                                  const float * speaker_embd, int32_t max_len, std::vector<int32_t> & output,
                                  int32_t language_id, float repetition_penalty, float temperature, int32_t top_k,
                                  float eos_bias, int32_t target_frames, bool rep_loop_detect,
                                  const FrameCallback & on_frame) {
    attn_rows_.clear();
    NEED_MODEL();
    if (!text_tokens || n_tokens < 4) { error_msg_ = "ICL: need at least 4 target text tokens"; return false; }
    if (!ref_codec_tokens || n_ref_frames < 1) { error_msg_ = "ICL: need at least 1 reference codec frame"; return false; }
    qtts_generate_params p{};
    p.text_tokens = text_tokens; p.n_tokens = n_tokens; p.ref_text_tokens = ref_text_tokens; p.n_ref_text = n_ref_text;
    p.ref_codec_tokens = ref_codec_tokens; p.n_ref_frames = n_ref_frames; p.speaker_embd = speaker_embd;
    p.max_len = max_len; p.language_id = language_id; p.repetition_penalty = repetition_penalty;
    p.temperature = temperature; p.top_k = top_k; p.eos_bias = eos_bias; p.target_frames = target_frames;
    p.rep_loop_detect = rep_loop_detect ? 1 : 0; p.seed = seed_;
    return generate_impl(&p, output, on_frame);
}

bool TTSTransformer::forward(const int32_t * tokens, int32_t n_tokens, int32_t n_past, std::vector<float> & output) {
    return forward_text(tokens, n_tokens, nullptr, n_past, output);
}

bool TTSTransformer::forward_with_audio(const int32_t * tokens, int32_t n_tokens, const float *, int32_t, int32_t,
                                        int32_t n_past, std::vector<float> & output) {
    return forward_text(tokens, n_tokens, nullptr, n_past, output);
}

// 'ATTD' dump format of src/tts_transformer.cpp:2978-3005.
bool TTSTransformer::write_attn_dump() {
    if (!attn_dump_ || attn_dump_path_.empty() || attn_rows_.empty()) return true;
    FILE * f = fopen(attn_dump_path_.c_str(), "wb");
    if (!f) { fprintf(stderr, "attn-dump: cannot open %s for writing\n", attn_dump_path_.c_str()); return false; }
    const int32_t n_head = model_.config.n_attention_heads;
    const uint32_t magic = 0x41545444u;
    const int32_t version = 1, n_rows = (int32_t) attn_rows_.size();
    fwrite(&magic, 4, 1, f); fwrite(&version, 4, 1, f); fwrite(&attn_dump_layer_, 4, 1, f);
    fwrite(&n_head, 4, 1, f); fwrite(&n_rows, 4, 1, f);
    for (const auto & row : attn_rows_) {
        const int32_t n_kv = (int32_t)(row.size() / n_head);
        fwrite(&n_kv, 4, 1, f);
        fwrite(row.data(), 4, row.size(), f);
    }
    fclose(f);
    return true;
}

void free_transformer_model(tts_transformer_model & model) { model.config = tts_transformer_config{}; }

void free_tts_kv_cache(tts_kv_cache & cache) { cache.n_ctx = 0; cache.n_used = 0; }

}  // namespace qwen3_tts
