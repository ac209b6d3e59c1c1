// A C++ caller of the drop-in qwen3_tts::TTSTransformer (include/tts_transformer.h),
// compiled and linked against libqwen3tts_b200.so by tests/test_gpu_dropin.py.
// It walks the reference's own transformer test (tests/test_transformer.cpp:169-355
// of the reference: load_model, init_kv_cache(4096), forward_prefill, generate with
// language 2050 / penalty 1.05 / temperature 0) and the rest of the public
// surface: generate_icl with an on_frame abort, the attention dump, forward_text,
// forward_codec, get_hidden_states and both code predictors.
//
//   dropin_driver MODEL.gguf DIR
// reads DIR/{text,ref_text,ref_codes}.i32 and DIR/{speaker,prefill}.f32, writes
// one raw little-endian file per result into DIR and a summary to stdout.
#include "tts_transformer.h"

#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

template <class T>
static std::vector<T> read_raw(const std::string & path) {
    std::vector<T> v;
    FILE * f = fopen(path.c_str(), "rb");
    if (!f) return v;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    v.resize((size_t) n / sizeof(T));
    if (fread(v.data(), sizeof(T), v.size(), f) != v.size()) v.clear();
    fclose(f);
    return v;
}

template <class T>
static bool write_raw(const std::string & path, const std::vector<T> & v) {
    FILE * f = fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = fwrite(v.data(), sizeof(T), v.size(), f) == v.size();
    fclose(f);
    return ok;
}

#define CHECK(cond, what)                                                          \
    do {                                                                           \
        if (!(cond)) {                                                             \
            printf("FAIL %s: %s\n", what, tts.get_error().c_str());                \
            return 1;                                                              \
        }                                                                          \
        printf("ok %s\n", what);                                                   \
    } while (0)

int main(int argc, char ** argv) {
    if (argc < 3) { fprintf(stderr, "usage: %s MODEL.gguf DIR\n", argv[0]); return 2; }
    const std::string model = argv[1], dir = std::string(argv[2]) + "/";
    const auto text = read_raw<int32_t>(dir + "text.i32");
    const auto ref_text = read_raw<int32_t>(dir + "ref_text.i32");
    const auto ref_codes = read_raw<int32_t>(dir + "ref_codes.i32");
    const auto speaker = read_raw<float>(dir + "speaker.f32");
    const auto prefill = read_raw<float>(dir + "prefill.f32");

    qwen3_tts::TTSTransformer tts;
    tts.set_seed(1);
    CHECK(tts.load_model(model), "load_model");
    const auto & cfg = tts.get_config();
    const int H = cfg.hidden_size, NCB = cfg.n_codebooks;
    printf("config hidden=%d layers=%d heads=%d kv_heads=%d codec_vocab=%d codebooks=%d cp_layers=%d\n", H,
           cfg.n_layers, cfg.n_attention_heads, cfg.n_key_value_heads, cfg.codec_vocab_size, NCB,
           cfg.code_pred_layers);
    CHECK(tts.init_kv_cache(4096), "init_kv_cache");
    CHECK(tts.init_code_pred_kv_cache(16), "init_code_pred_kv_cache");

    // reference test 4: forward_prefill of a prefill embedding, hidden rows + logits
    const int n_pre = (int)(prefill.size() / H);
    std::vector<float> hid, logits;
    tts.clear_kv_cache();
    CHECK(tts.forward_prefill(prefill.data(), n_pre, 0, hid, &logits), "forward_prefill");
    write_raw(dir + "prefill_hidden.f32", hid);
    write_raw(dir + "prefill_logits.f32", logits);
    std::vector<float> last;
    CHECK(tts.get_hidden_states(last) && (int) last.size() == H, "get_hidden_states");
    write_raw(dir + "prefill_last_hidden.f32", last);

    // reference test 5: generate (language 2050, penalty 1.05, greedy), EOS held off
    // so the frame count is fixed, with the talker attention dump of layer 1
    tts.clear_kv_cache();
    tts.set_attn_dump(dir + "attn.bin", 1);
    std::vector<int32_t> codes;
    CHECK(tts.generate(text.data(), (int32_t) text.size(), speaker.data(), 8, codes, 2050, 1.05f, 0.0f, 0, nullptr,
                       0, -1e9f),
          "generate");
    write_raw(dir + "gen_codes.i32", codes);
    printf("attn_rows %zu\n", tts.attn_rows().size());
    tts.set_attn_dump("", 1);

    // generate_icl, aborted by the frame callback after frame 3 (4 frames kept)
    std::vector<int32_t> icl;
    std::vector<int32_t> seen;
    auto cb = [&](const int32_t * c, int32_t n, int32_t frame) {
        if (n != NCB || !c) return false;
        seen.push_back(frame);
        return frame < 3;
    };
    CHECK(tts.generate_icl(text.data(), (int32_t) text.size(), ref_text.data(), (int32_t) ref_text.size(),
                           ref_codes.data(), (int32_t)(ref_codes.size() / NCB), speaker.data(), 12, icl, 2050,
                           1.05f, 0.0f, 0, -1e9f, 0, false, cb),
          "generate_icl");
    write_raw(dir + "icl_codes.i32", icl);
    printf("icl_callback_frames %zu\n", seen.size());

    // interface-only members: forward_text, forward_codec, both code predictors
    std::vector<float> th;
    tts.clear_kv_cache();
    CHECK(tts.forward_text(text.data(), 6, speaker.data(), 0, th), "forward_text");
    write_raw(dir + "text_hidden.f32", th);
    std::vector<float> cl;
    CHECK(tts.forward_codec(cfg.codec_bos_id, 6, cl), "forward_codec");
    write_raw(dir + "codec_logits.f32", cl);
    std::vector<float> ch;
    CHECK(tts.get_hidden_states(ch), "get_hidden_states after forward_codec");
    write_raw(dir + "codec_hidden.f32", ch);
    std::vector<int32_t> ar;
    CHECK(tts.predict_codes_autoregressive(ch.data(), 7, ar, 0.0f, 0), "predict_codes_autoregressive");
    write_raw(dir + "cp_ar_codes.i32", ar);
    std::vector<int32_t> prev(NCB - 1);
    for (int g = 0; g < NCB - 1; ++g) prev[g] = (17 * g + 3) % cfg.code_pred_vocab_size;
    std::vector<float> pc;
    CHECK(tts.predict_codes(ch.data(), prev.data(), pc), "predict_codes");
    write_raw(dir + "cp_legacy_logits.f32", pc);

    // error convention: bool + get_error, no exception
    std::vector<int32_t> none;
    const bool bad = tts.generate(text.data(), 2, nullptr, 4, none);
    printf("short_text_rejected %d error=\"%s\"\n", bad ? 0 : 1, tts.get_error().c_str());
    tts.unload_model();
    std::vector<float> after;
    printf("unloaded_forward_rejected %d\n", tts.forward_codec(0, 0, after) ? 0 : 1);
    printf("DONE\n");
    return 0;
}
