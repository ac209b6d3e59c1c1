/* qwen3tts_b200.h — C ABI of the B200 codec-token engine.
 *
 * One engine = one GPU, one sequence at a time, exactly like the reference's
 * TTSTransformer (src/tts_transformer.h:198-422).  Every entry point below
 * replaces one TTSTransformer member; the C++ drop-in class in
 * tts_transformer.h forwards to these.  Conventions follow the reference:
 * functions return 1 (true) / 0 (false) where the reference returns bool, and
 * the message is read with qtts_get_error() (src/tts_transformer.h:328).
 * Buffers are plain host pointers owned by the caller; sizes are in elements.
 * No torch, CUDA or ggml type appears in any signature.
 */
#ifndef QWEN3TTS_B200_H
#define QWEN3TTS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qtts_engine qtts_engine;

/* Field-for-field copy of tts_transformer_config (src/tts_transformer.h:59-103)
 * plus the weight type of the layer matrices (1 = F16, 8 = Q8_0). */
typedef struct qtts_config {
    int32_t text_vocab_size, text_embd_dim;
    int32_t hidden_size, n_layers, n_attention_heads, n_key_value_heads, intermediate_size, head_dim;
    float rms_norm_eps, rope_theta;
    int32_t mrope_section[3];
    int32_t codec_vocab_size, n_codebooks;
    int32_t code_pred_layers, code_pred_vocab_size, code_pred_hidden_size, code_pred_intermediate_size;
    float code_pred_rope_theta;
    int32_t codec_pad_id, codec_bos_id, codec_eos_id;
    int32_t tts_bos_token_id, tts_eos_token_id, tts_pad_token_id;
    int32_t codec_think_id, codec_nothink_id, codec_think_bos_id, codec_think_eos_id;
    int32_t english_language_id;
    int32_t weight_type;
} qtts_config;

/* Arguments of TTSTransformer::generate / generate_icl
 * (src/tts_transformer.h:293-324).  ICL mode when ref_codec_tokens != NULL.
 * seed keys the Philox stream of sampled decoding (the reference's std::mt19937
 * has no seed setter, src/tts_transformer.h:403). */
typedef struct qtts_generate_params {
    const int32_t * text_tokens; int32_t n_tokens;
    const int32_t * ref_text_tokens; int32_t n_ref_text;
    const int32_t * ref_codec_tokens; int32_t n_ref_frames;   /* [n_ref_frames x 16] */
    const float * speaker_embd;                                /* [hidden] or NULL */
    int32_t max_len;
    int32_t language_id;
    float repetition_penalty;
    float temperature;
    int32_t top_k;
    const int32_t * instruct_tokens; int32_t n_instruct;
    float eos_bias;
    int32_t target_frames;
    int32_t rep_loop_detect;
    uint64_t seed;
} qtts_generate_params;

/* FrameCallback (src/tts_transformer.h:291): return 0 to stop generation. */
typedef int32_t (*qtts_frame_callback)(const int32_t * frame_codes, int32_t n_codebooks,
                                       int32_t frame_index, void * user_data);

/* Device-side timings of the last call (CUDA events on the engine stream). */
typedef struct qtts_timing {
    float prefill_ms;        /* forward_prefill of the last generate */
    float frames_ms;         /* frame loop of the last generate / run_frames */
    int32_t frames;          /* frames in frames_ms */
    int32_t kernel_launches; /* engine kernels launched per frame */
    float load_ms;           /* load_model: GGUF parse, staged weight upload, repacking */
} qtts_timing;

/* Stage timings of the last generate (no reference counterpart as an ABI; the
 * reference prints the same stages under QWEN3_TTS_TIMING, src/tts_transformer.h:
 * 20-54, src/tts_transformer.cpp:3311-3353).  With stage timing on, frames run
 * kernel by kernel with CUDA events around every launch (slower than the frame
 * graph), each launch charged to the talker step, the code predictor, or the
 * samplers with their next-input embedding sums. */
typedef struct qtts_stage_timing {
    float prefill_build_ms;   /* host recipe + device text projection and prompt row assembly */
    float prefill_forward_ms; /* device: forward_prefill */
    float talker_ms;          /* device: talker steps (layers + codec head) */
    float code_pred_ms;       /* device: code-predictor passes (layers + heads) */
    float sample_embed_ms;    /* device: samplers and next-input embedding sums (fused frame path:
                                 the launches that sample, each also running its pass's first
                                 attention block) */
    float total_ms;           /* host: the whole qtts_generate call */
    int32_t frames;
} qtts_stage_timing;

/* Per-kernel-class statistics of qtts_profile_frames (classes: 0 = GEMV,
 * 1 = attention, 2 = sampling, 3 = other). */
typedef struct qtts_kernel_stats {
    int32_t launches;
    float total_ms;
    double bytes;            /* algorithmic bytes (weights + activations) */
} qtts_kernel_stats;

/* TTSTransformer::load_model (src/tts_transformer.h:204; src/tts_transformer.cpp:68-173).
 * device < 0 selects QWEN3_TTS_DEVICE or 0.  Returns NULL on failure;
 * qtts_create_error() then holds the message (per thread). */
qtts_engine * qtts_create(const char * gguf_path, int32_t device);
const char * qtts_create_error(void);
/* TTSTransformer::unload_model + destructor (src/tts_transformer.cpp:21-51). */
void qtts_destroy(qtts_engine * e);
/* TTSTransformer::get_error (src/tts_transformer.h:328). */
const char * qtts_get_error(const qtts_engine * e);
/* TTSTransformer::get_config (src/tts_transformer.h:326). */
int32_t qtts_get_config(const qtts_engine * e, qtts_config * out);
/* TTSTransformer::set_n_threads (src/tts_transformer.h:208): accepted, no effect on a GPU engine. */
void qtts_set_n_threads(qtts_engine * e, int32_t n_threads);

/* KV caches (src/tts_transformer.h:230-239; src/tts_transformer.cpp:731-837). */
int32_t qtts_init_kv_cache(qtts_engine * e, int32_t n_ctx);
void qtts_clear_kv_cache(qtts_engine * e);
int32_t qtts_init_code_pred_kv_cache(qtts_engine * e, int32_t n_ctx);
void qtts_clear_code_pred_kv_cache(qtts_engine * e);

/* TTSTransformer::forward_prefill (src/tts_transformer.h:250; .cpp:2217-2347).
 * hidden_out: [n_tokens x hidden] post-norm rows or NULL; logits_out: [codec_vocab]
 * of the last row or NULL. */
int32_t qtts_forward_prefill(qtts_engine * e, const float * prefill_embd, int32_t n_tokens, int32_t n_past,
                             float * hidden_out, float * logits_out);
/* TTSTransformer::forward_step (src/tts_transformer.h:261; .cpp:2379-2509). */
int32_t qtts_forward_step(qtts_engine * e, const float * step_embd, int32_t n_past,
                          float * logits_out, float * hidden_out);
/* TTSTransformer::forward_text (src/tts_transformer.h:246; .cpp:2349-2377). */
int32_t qtts_forward_text(qtts_engine * e, const int32_t * text_tokens, int32_t n_tokens,
                          const float * speaker_embd, int32_t n_past, float * hidden_out);
/* TTSTransformer::forward_codec (src/tts_transformer.h:258; .cpp:2511-2521). */
int32_t qtts_forward_codec(qtts_engine * e, int32_t codec_token, int32_t n_past, float * logits_out);
/* TTSTransformer::get_hidden_states (src/tts_transformer.h:266; .cpp:2523-2529). */
int32_t qtts_get_hidden_states(const qtts_engine * e, float * hidden_out);
/* TTSTransformer::predict_codes (legacy, src/tts_transformer.h:272; .cpp:2531-2581).
 * logits_out: [(n_codebooks-1) x code_pred_vocab]. */
int32_t qtts_predict_codes(qtts_engine * e, const float * hidden, const int32_t * prev_codes, float * logits_out);
/* TTSTransformer::predict_codes_autoregressive (src/tts_transformer.h:279; .cpp:2711-2976).
 * codes_out: [n_codebooks-1]. */
int32_t qtts_predict_codes_autoregressive(qtts_engine * e, const float * hidden, int32_t codebook_0_token,
                                          float temperature, int32_t top_k, int32_t * codes_out);

/* project_text_tokens (src/tts_transformer.cpp:963-1028): out [n x hidden]. */
int32_t qtts_project_text(qtts_engine * e, const int32_t * tokens, int32_t n, float * out);
/* lookup_embedding_rows (src/tts_transformer.cpp:839-961).  table: 0 = talker
 * codec_embd, 1..n_codebooks-1 = code_pred.codec_embd[table-1], -1 = text_embd. */
int32_t qtts_lookup_embedding_rows(qtts_engine * e, int32_t table, const int32_t * ids, int32_t n, float * out);

/* TTSTransformer::generate / generate_icl (src/tts_transformer.h:293-324;
 * .cpp:3007-3656).  codes_out: [max_len x n_codebooks]; *n_frames_out frames
 * are valid.  on_frame may be NULL. */
int32_t qtts_generate(qtts_engine * e, const qtts_generate_params * p, qtts_frame_callback on_frame,
                      void * user_data, int32_t * codes_out, int32_t * n_frames_out);

/* Streaming pieces of qtts_generate: begin builds and runs the prefill and arms
 * the device frame state; run_frames then advances up to n frames on the device
 * (stopping at EOS) and copies their codes to codes_out ([n x n_codebooks]).
 * Returns the number of frames produced, -1 on error. */
int32_t qtts_generate_begin(qtts_engine * e, const qtts_generate_params * p);
int32_t qtts_run_frames(qtts_engine * e, int32_t n, int32_t * codes_out);
/* Rewinds the active generation to frame 0 (the state right after begin's
 * prefill) so an utterance can be replayed without running its prefill again;
 * KV positions past the prefill are rewritten as frames are regenerated.
 * Returns 0, or -1 with no active generation.  No counterpart in the
 * reference (benchmark and streaming-restart helper). */
int32_t qtts_generate_rewind(qtts_engine * e);
/* Codes -> vocoder handoff without a host copy (no reference counterpart; the
 * reference hands codes to the decoder in host vectors, src/qwen3_tts.cpp:
 * 271-316): *codes_dev = the engine's device buffer, frame f of the current (or
 * last) generation at row f, [max_len][n_codebooks] int32, valid until the
 * next generation starts; *n_frames = frames generated so far.  The pointer is
 * on the engine's device.  Returns 0, or -1 before any generation. */
int32_t qtts_codes_device(qtts_engine * e, const int32_t ** codes_dev, int32_t * n_frames);

/* Sampling seed of the Philox stream (sampled decoding is reproducible). */
void qtts_set_seed(qtts_engine * e, uint64_t seed);
/* Record the raw codebook-0 logits ([cap x codec_vocab]) and code-predictor
 * logits ([cap x (n_codebooks-1) x code_pred_vocab]) of each generated frame into
 * host buffers (either may be NULL; cap 0 disables). */
int32_t qtts_set_debug_logits(qtts_engine * e, float * talker_logits, float * cp_logits, int32_t cap_frames);
/* TTSTransformer::set_attn_dump (src/tts_transformer.h:224): keep the
 * post-softmax row of talker layer `layer` for every generated frame. */
int32_t qtts_set_attn_dump(qtts_engine * e, int32_t enabled, int32_t layer);
/* Number of attention rows kept and row r ([n_kv x n_head] values). */
int32_t qtts_attn_rows(const qtts_engine * e);
int32_t qtts_attn_row(const qtts_engine * e, int32_t r, float * out, int32_t cap);
int32_t qtts_get_timing(const qtts_engine * e, qtts_timing * out);
/* The frame path in use (no reference counterpart): 0 = one kernel per op (the
 * default), 1 = two clustered kernels per transformer layer (QTTS_FRAME_MODE=fused
 * at load time, where the model's shapes allow it). */
int32_t qtts_get_frame_mode(const qtts_engine * e);
/* Diagnostics of the fused frame path (no reference counterpart), on when
 * QTTS_FF_TRACE=1 at load time: per launch of frame 1 of a run and per CTA (up
 * to 256), eight %globaltimer stamps (start, dependency wait returned, input
 * built, first GEMV done, first cluster barrier passed, attention or ffn_down
 * partial done, second cluster barrier passed, end; 0 = not reached) into out
 * [launch][256][8] (cap words), and kinds[launch] = kind * 4 + (samples ? 2 : 0)
 * + rows - 1 (kind 0 attention block, 1 FFN block, 2 head).  Returns the number
 * of launches (0 when tracing is off). */
int32_t qtts_frame_trace(const qtts_engine * e, unsigned long long * out, int32_t cap, int32_t * kinds, int32_t kcap);
/* Stage timing on (1) / off (0) for the following generate calls; 1 on success. */
int32_t qtts_set_stage_timing(qtts_engine * e, int32_t enabled);
int32_t qtts_get_stage_timing(const qtts_engine * e, qtts_stage_timing * out);
/* Advance up to n frames of the active generation kernel by kernel (no CUDA
 * graph) with CUDA events around each launch; fills stats[0..n_classes).
 * Returns frames produced or -1.  For measurement only. */
int32_t qtts_profile_frames(qtts_engine * e, int32_t n, qtts_kernel_stats * stats, int32_t n_classes);

/* One Q8_0 GEMM on the tcgen05 tensor cores (kind::i8) as the batched path runs
 * it for Q8_0 models (test entry; no reference counterpart; replaces the Q8_0
 * ggml_mul_mat calls of src/tts_transformer.cpp:1659-1661, 1739-1750 for many
 * sequences at once).  w (and w_up for SwiGLU): GGUF Q8_0 blocks [rows][cols/32]
 * of 34 bytes (f16 d, 32 int8).  The activations x[m x cols] (optionally
 * RMSNorm-ed with norm_gain) are quantised per 32-block as quantize_row_q8_0;
 * y[m][r] = sum over blocks b in order of (float) isum_b * (d_w * d_a), the
 * k-split partials (ksplit CTAs per 128-row tile; 0 = the engine's choice) added
 * in rank order.  epi as qtts_op_gemm_tc.  rows (x2 for SwiGLU) % 128 == 0,
 * cols % 128 == 0, m <= 128.  Returns the k-split used (>= 1), 0 on failure. */
int32_t qtts_op_gemm_q8(int32_t device, const uint8_t * w, const uint8_t * w_up, int32_t rows, int32_t cols,
                        const float * xin, int32_t m, const float * norm_gain, float eps, int32_t epi,
                        const float * resid, int32_t ksplit, float * y);
/* One tcgen05 tensor-core GEMM as the batched and prefill paths run it
 * (test entry; no reference counterpart): y[m][r] = sum_k W[r][k] * a[m][k],
 * W F16 row-major [rows x cols] (host), activations a = x[m x cols] after an
 * optional RMSNorm with norm_gain, rounded to F16 (act 0) or split into F16
 * hi + lo parts (act 1, the F32-activation ffn_down semantics).  epi 0 stores,
 * 1 adds resid[m x rows], 2 is SwiGLU: y = silu(W a) * (w_up a) with w_up the up
 * matrix.  rows (x2 for SwiGLU) % 128 == 0, cols % 64 == 0, m <= 256 (128 with
 * act 1).  Returns 1 on success. */
int32_t qtts_op_gemm_tc(int32_t device, const uint16_t * w, const uint16_t * w_up, int32_t rows, int32_t cols,
                        const float * x, int32_t m, const float * norm_gain, float eps, int32_t act, int32_t epi,
                        const float * resid, float * y);

/* ---- Kernel-level entry points (one engine kernel on host data) ----------
 * ggml_mul_mat (+ optional ggml_rms_norm prologue) as the engine computes it,
 * src/tts_transformer.cpp:1656-1661: y[nv][rows] = W[rows][cols] . x[nv][cols].
 * wtype 1 = F16 (w: [rows][cols] halves), 8 = Q8_0 (w: GGUF blocks
 * [rows][cols/32] x 34 bytes).  act_f32 keeps x unrounded (the F32-cast
 * ffn_down of :1746-1748).  block_dots, if not NULL, receives the per-block
 * int32 Q8_0 dot products [nv][rows][cols/32]. */
int32_t qtts_op_gemv(int32_t device, int32_t wtype, const void * w, int32_t rows, int32_t cols, const float * x,
                     int32_t nv, const float * norm_gain, float eps, int32_t act_f32, float * y, int32_t * block_dots);
/* One sampling decision (src/tts_transformer.cpp:3108-3184 for cb 0, :2750-2788
 * for cb >= 1).  presence: optional [V] 0/1 set of earlier codebook-0 tokens.
 * Returns the token (eos_id when codebook 0 samples EOS), -1 on error. */
int32_t qtts_op_sample(int32_t device, const float * logits, int32_t V, int32_t cb, float temperature, int32_t top_k,
                       float rep_penalty, const int32_t * presence, float eos_bias, int32_t target_frames,
                       int32_t frame, int32_t eos_id, int32_t suppress_start, uint64_t seed);
/* The same sampling decision as qtts_op_sample, for callers that cannot
 * allocate device memory: a real-time streaming loop, where the device-wide
 * synchronisation of a cudaMalloc/cudaFree pair per call would stall audio
 * output, and host applications that own all device memory through their own
 * pool and do not let libraries allocate.  This entry point has no
 * counterpart in the reference.
 * Inputs and the output are DEVICE pointers owned by the caller: logits [V],
 * presence [V] (0/1, optional), token_out [1] (written on `stream`, which may be
 * NULL for the default stream).  The sampler's state lives in a fixed 4 KiB
 * __device__ array inside the library (every GPU that loads the library holds
 * it until exit), so V is limited to 4096: larger vocabularies return -2 with
 * a message on stderr.  No cudaMalloc, cudaFree or allocating routine is
 * called by the entry point itself.  The first call on a device looks up the
 * array's device address (with that device current) and makes the sampler's
 * kernel resident: under CUDA's lazy module loading that first call may load
 * the module, which allocates device memory and can synchronise.  Make one
 * call per device outside the real-time loop, before any stream capture.
 * All calls share the array: the kernel clears the state it reads at every
 * call, and calls that overlap on the GPU (concurrent streams) race.
 * Returns 1 on a successful launch, 0 on invalid arguments or a CUDA error. */
int32_t qtts_op_sample_noalloc(int32_t device, const float * logits, int32_t V, int32_t cb, float temperature,
                               int32_t top_k, float rep_penalty, const int32_t * presence, float eos_bias,
                               int32_t target_frames, int32_t frame, int32_t eos_id, int32_t suppress_start,
                               uint64_t seed, int32_t * token_out, void * stream);

/* ---- batched frame loop (B independent utterances on one GPU; no reference
 * counterpart: the reference serves one sequence per TTSTransformer).
 * Every projection of an F16 model is a tcgen05 tensor-core GEMM over the batch rows, the
 * talker KV lives in 64-position pages, and each sequence keeps its own frame
 * state.  Weights are shared with the engine (Q8_0 models: the layer
 * projections run as 8-row GEMV chunks instead of tensor-core GEMMs).
 *   create: max_batch <= 64 sequences, max_positions = prompt + frames capacity
 *           per sequence, max_frames = codes capacity per sequence; NULL on
 *           failure (qtts_get_error(e) holds the message).
 *   begin:  runs each sequence's prefill (params[i], as qtts_generate) and arms
 *           the batch; sampling parameters come from params[0].  0 / -1.
 *   run:    advances up to n_frames frames for the whole batch; returns the
 *           number of sequence-frames produced, -1 on error.
 *   codes:  codes_out [n][max_frames][n_codebooks], n_frames_out [n].
 *   timing: device time of all run calls since begin, sequence-frames, kernels
 *           launched per frame. */
typedef struct qtts_batch qtts_batch;
qtts_batch * qtts_batch_create(qtts_engine * e, int32_t max_batch, int32_t max_positions, int32_t max_frames);
int32_t qtts_batch_begin(qtts_batch * b, int32_t n, const qtts_generate_params * params);
int32_t qtts_batch_run(qtts_batch * b, int32_t n_frames);
int32_t qtts_batch_codes(qtts_batch * b, int32_t * codes_out, int32_t * n_frames_out);
/* The batch's device code buffer [n][max_frames][n_codebooks] int32 (valid
 * until the next begin) and, in n_frames_out [n], the frames each sequence has
 * produced: the batched codes -> vocoder handoff.  0 / -1. */
int32_t qtts_batch_codes_device(qtts_batch * b, const int32_t ** codes_dev, int32_t * n_frames_out);
int32_t qtts_batch_timing(const qtts_batch * b, float * frames_ms, int32_t * seq_frames, int32_t * launches_per_frame);
/* Runs n_frames frames eagerly with CUDA events around every launch (frames
 * advance as with run).  Per frame, for the 10 kernel classes (pack, GEMM
 * qkv / o / gate-up / down / heads, code-predictor attention, talker attention,
 * samplers, other): device ms into ms_per_frame[10], launches into
 * launches_per_frame[10]. */
int32_t qtts_batch_profile(qtts_batch * b, int32_t n_frames, float * ms_per_frame, int32_t * launches_per_frame);
const char * qtts_batch_error(const qtts_batch * b);
void qtts_batch_free(qtts_batch * b);

#ifdef __cplusplus
}
#endif

#endif /* QWEN3TTS_B200_H */
