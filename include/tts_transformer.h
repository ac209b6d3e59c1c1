// tts_transformer.h — drop-in replacement for the reference's
// src/tts_transformer.h (class qwen3_tts::TTSTransformer, lines 198-422).
//
// The public section is the reference's, member for member, with the same
// default arguments; the private section is a handle to the B200 engine
// (include/qwen3tts_b200.h) instead of ggml tensors, so this header needs no
// ggml include.  Qwen3TTS (src/qwen3_tts.cpp) and tests/test_transformer.cpp
// compile against it unchanged.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

struct qtts_engine;

namespace qwen3_tts {

#ifdef QWEN3_TTS_TIMING
struct tts_timing {  // src/tts_transformer.h:21-53
    double t_prefill_build_ms = 0, t_prefill_forward_ms = 0, t_prefill_graph_build_ms = 0,
           t_prefill_graph_alloc_ms = 0, t_prefill_compute_ms = 0, t_prefill_data_ms = 0;
    double t_talker_forward_ms = 0, t_talker_graph_build_ms = 0, t_talker_graph_alloc_ms = 0,
           t_talker_compute_ms = 0, t_talker_data_ms = 0;
    double t_code_pred_ms = 0, t_code_pred_init_ms = 0, t_code_pred_prefill_ms = 0, t_code_pred_steps_ms = 0,
           t_code_pred_graph_build_ms = 0, t_code_pred_graph_alloc_ms = 0, t_code_pred_compute_ms = 0,
           t_code_pred_data_ms = 0, t_code_pred_coreml_ms = 0;
    double t_embed_lookup_ms = 0;
    int32_t n_frames = 0;
    double t_generate_total_ms = 0;
};
#endif

#define QWEN3_TTS_MAX_NODES 16384

// src/tts_transformer.h:59-103, identical fields and defaults.
struct tts_transformer_config {
    int32_t text_vocab_size = 151936;
    int32_t text_embd_dim = 2048;
    int32_t hidden_size = 1024;
    int32_t n_layers = 28;
    int32_t n_attention_heads = 16;
    int32_t n_key_value_heads = 8;
    int32_t intermediate_size = 3072;
    int32_t head_dim = 128;
    float rms_norm_eps = 1e-6f;
    float rope_theta = 1000000.0f;
    int32_t mrope_section[3] = {24, 20, 20};
    int32_t codec_vocab_size = 3072;
    int32_t n_codebooks = 16;
    int32_t code_pred_layers = 5;
    int32_t code_pred_vocab_size = 2048;
    int32_t code_pred_hidden_size = 1024;
    int32_t code_pred_intermediate_size = 3072;
    float code_pred_rope_theta = 10000.0f;
    int32_t codec_pad_id = 2148;
    int32_t codec_bos_id = 2149;
    int32_t codec_eos_id = 2150;
    int32_t tts_bos_token_id = 151672;
    int32_t tts_eos_token_id = 151673;
    int32_t tts_pad_token_id = 151671;
    int32_t codec_think_id = 2154;
    int32_t codec_nothink_id = 2155;
    int32_t codec_think_bos_id = 2156;
    int32_t codec_think_eos_id = 2157;
    int32_t english_language_id = 2050;
};

// The reference's weight and cache holders carry ggml tensors; here the
// weights and caches live in the engine, and these keep only their metadata
// so free_transformer_model / free_tts_kv_cache stay callable.
struct tts_transformer_model {
    tts_transformer_config config;
};
struct tts_kv_cache {
    int32_t n_ctx = 0;
    int32_t n_used = 0;
    int32_t head_dim = 128;
    int32_t n_kv_heads = 8;
    int32_t n_layers = 28;
};

class TTSTransformer {
public:
    TTSTransformer();
    ~TTSTransformer();

    bool load_model(const std::string & model_path);
    void set_n_threads(int32_t n_threads);
    void unload_model();
    void set_debug_dump(bool enabled) { debug_dump_ = enabled; }
    void set_attn_dump(const std::string & path, int layer = 27);
    const std::vector<std::vector<float>> & attn_rows() const { return attn_rows_; }

    bool init_kv_cache(int32_t n_ctx);
    void clear_kv_cache();
    bool init_code_pred_kv_cache(int32_t n_ctx);
    void clear_code_pred_kv_cache();

    bool forward_text(const int32_t * text_tokens, int32_t n_tokens, const float * speaker_embd, int32_t n_past,
                      std::vector<float> & output);
    bool forward_prefill(const float * prefill_embd, int32_t n_tokens, int32_t n_past, std::vector<float> & output,
                         std::vector<float> * logits_out = nullptr);
    bool forward_codec(int32_t codec_token, int32_t n_past, std::vector<float> & output);
    bool forward_step(const float * step_embd, int32_t n_past, std::vector<float> & output,
                      std::vector<float> * hidden_out = nullptr);
    bool get_hidden_states(std::vector<float> & hidden) const;
    bool predict_codes(const float * hidden, const int32_t * prev_codes, std::vector<float> & output);
    bool predict_codes_autoregressive(const float * hidden, int32_t codebook_0_token, std::vector<int32_t> & output,
                                      float temperature = 0.9f, int32_t top_k = 50);

    using FrameCallback = std::function<bool(const int32_t *, int32_t, int32_t)>;

    bool generate(const int32_t * text_tokens, int32_t n_tokens, const float * speaker_embd, int32_t max_len,
                  std::vector<int32_t> & output, int32_t language_id = 2050, float repetition_penalty = 1.05f,
                  float temperature = 0.9f, int32_t top_k = 50, const int32_t * instruct_tokens = nullptr,
                  int32_t n_instruct = 0, float eos_bias = 0.0f, int32_t target_frames = 0,
                  bool rep_loop_detect = false, const FrameCallback & on_frame = nullptr);

    bool generate_icl(const int32_t * text_tokens, int32_t n_tokens, const int32_t * ref_text_tokens,
                      int32_t n_ref_text, const int32_t * ref_codec_tokens, int32_t n_ref_frames,
                      const float * speaker_embd, int32_t max_len, std::vector<int32_t> & output,
                      int32_t language_id = 2050, float repetition_penalty = 1.05f, float temperature = 0.9f,
                      int32_t top_k = 50, float eos_bias = 0.0f, int32_t target_frames = 0,
                      bool rep_loop_detect = true, const FrameCallback & on_frame = nullptr);

    const tts_transformer_config & get_config() const { return model_.config; }
    const std::string & get_error() const { return error_msg_; }

    bool forward(const int32_t * tokens, int32_t n_tokens, int32_t n_past, std::vector<float> & output);
    bool forward_with_audio(const int32_t * tokens, int32_t n_tokens, const float * audio_embd, int32_t n_audio,
                            int32_t audio_start_pos, int32_t n_past, std::vector<float> & output);

    // Extension (not in the reference): seed of the sampled-decoding stream.
    // The reference seeds std::mt19937 from std::random_device and has no setter.
    void set_seed(uint64_t seed);

private:
    bool generate_impl(const void * params, std::vector<int32_t> & output, const FrameCallback & on_frame);
    bool write_attn_dump();

    tts_transformer_model model_;
    tts_kv_cache cache_;
    ::qtts_engine * engine_ = nullptr;
    std::string error_msg_;
    std::vector<float> last_hidden_;
    uint64_t seed_ = 0;
    bool debug_dump_ = false;
    bool attn_dump_ = false;
    int attn_dump_layer_ = 27;
    std::string attn_dump_path_;
    std::vector<std::vector<float>> attn_rows_;
};

void free_transformer_model(tts_transformer_model & model);
void free_tts_kv_cache(tts_kv_cache & cache);

}  // namespace qwen3_tts
