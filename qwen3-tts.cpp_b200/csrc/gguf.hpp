// gguf.hpp — minimal GGUF v2/v3 reader (mmap) for the engine's weight loader.
//
// Covers what TTSTransformer::load_model reads (src/tts_transformer.cpp:105-137,
// 228-377, 670-729): scalar metadata (with the reference's alias lists), tensor
// infos and data offsets.  Tensor payloads stay in the mapping until uploaded.
#pragma once
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace qtts {

enum GgmlType : int { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8 };

struct GgufTensor {
    std::string name;
    int type = -1;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    const uint8_t * data = nullptr;
    size_t nbytes = 0;
};

class GgufFile {
public:
    ~GgufFile() { if (map_) munmap(map_, size_); }

    bool open(const std::string & path, std::string & err) {
        int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) { err = "Failed to open GGUF file: " + path; return false; }
        struct stat st;
        if (fstat(fd, &st) != 0) { ::close(fd); err = "stat failed: " + path; return false; }
        size_ = (size_t) st.st_size;
        void * m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) { err = "mmap failed: " + path; return false; }
        map_ = (uint8_t *) m;
        return parse(err);
    }

    int64_t get_int(std::initializer_list<const char *> keys, int64_t dflt) const {
        for (const char * k : keys) { auto it = ints_.find(k); if (it != ints_.end()) return it->second; }
        return dflt;
    }
    double get_float(std::initializer_list<const char *> keys, double dflt) const {
        for (const char * k : keys) { auto it = floats_.find(k); if (it != floats_.end()) return it->second; }
        return dflt;
    }
    const GgufTensor * find(const std::string & name) const {
        auto it = tensors_.find(name);
        return it == tensors_.end() ? nullptr : &it->second;
    }
    const std::map<std::string, GgufTensor> & tensors() const { return tensors_; }
    const uint8_t * map() const { return map_; }
    size_t size() const { return size_; }

private:
    bool parse(std::string & err) {
        size_t p = 0;
        auto rd = [&](void * dst, size_t n) { if (p + n > size_) return false; memcpy(dst, map_ + p, n); p += n; return true; };
        auto rstr = [&](std::string & s) {
            uint64_t n; if (!rd(&n, 8) || p + n > size_) return false;
            s.assign((const char *) map_ + p, n); p += n; return true;
        };
        uint32_t magic = 0, version = 0; uint64_t nt = 0, nkv = 0;
        if (!rd(&magic, 4) || magic != 0x46554747u) { err = "not a GGUF file"; return false; }
        if (!rd(&version, 4) || version < 2 || version > 3) { err = "unsupported GGUF version"; return false; }
        if (!rd(&nt, 8) || !rd(&nkv, 8)) { err = "truncated GGUF header"; return false; }
        static const int tsize[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        for (uint64_t i = 0; i < nkv; ++i) {
            std::string key; uint32_t ty;
            if (!rstr(key) || !rd(&ty, 4)) { err = "truncated GGUF metadata"; return false; }
            if (ty == 8) { std::string v; if (!rstr(v)) { err = "truncated string"; return false; } continue; }
            if (ty == 9) {
                uint32_t at; uint64_t n;
                if (!rd(&at, 4) || !rd(&n, 8)) { err = "truncated array"; return false; }
                for (uint64_t k = 0; k < n; ++k) {
                    if (at == 8) { std::string v; if (!rstr(v)) { err = "truncated array"; return false; } }
                    else if (at < 13 && tsize[at]) { p += tsize[at]; if (p > size_) { err = "truncated array"; return false; } }
                    else { err = "unsupported nested GGUF array"; return false; }
                }
                continue;
            }
            if (ty >= 13 || !tsize[ty]) { err = "bad GGUF metadata type"; return false; }
            uint8_t b[8] = {0};
            if (!rd(b, tsize[ty])) { err = "truncated GGUF metadata"; return false; }
            int64_t iv = 0; double fv = 0; bool isf = false;
            switch (ty) {
                case 0: iv = b[0]; break;
                case 1: iv = (int8_t) b[0]; break;
                case 2: { uint16_t v; memcpy(&v, b, 2); iv = v; } break;
                case 3: { int16_t v; memcpy(&v, b, 2); iv = v; } break;
                case 4: { uint32_t v; memcpy(&v, b, 4); iv = v; } break;
                case 5: { int32_t v; memcpy(&v, b, 4); iv = v; } break;
                case 6: { float v; memcpy(&v, b, 4); fv = v; isf = true; } break;
                case 7: iv = b[0]; break;
                case 10: { uint64_t v; memcpy(&v, b, 8); iv = (int64_t) v; } break;
                case 11: { int64_t v; memcpy(&v, b, 8); iv = v; } break;
                case 12: { double v; memcpy(&v, b, 8); fv = v; isf = true; } break;
            }
            if (isf) floats_[key] = fv; else ints_[key] = iv;
        }
        struct Info { std::string name; uint32_t nd; uint64_t ne[4]; uint32_t type; uint64_t off; };
        std::vector<Info> infos(nt);
        for (auto & ti : infos) {
            if (!rstr(ti.name) || !rd(&ti.nd, 4) || ti.nd > 4) { err = "bad GGUF tensor info"; return false; }
            for (int d = 0; d < 4; ++d) ti.ne[d] = 1;
            for (uint32_t d = 0; d < ti.nd; ++d) if (!rd(&ti.ne[d], 8)) { err = "bad GGUF tensor info"; return false; }
            if (!rd(&ti.type, 4) || !rd(&ti.off, 8)) { err = "bad GGUF tensor info"; return false; }
        }
        const uint64_t align = (uint64_t) get_int({"general.alignment"}, 32);
        const size_t data_off = (p + align - 1) / align * align;
        for (auto & ti : infos) {
            GgufTensor t;
            t.name = ti.name; t.type = (int) ti.type; t.n_dims = (int) ti.nd;
            int64_t n = 1;
            for (int d = 0; d < 4; ++d) { t.ne[d] = (int64_t) ti.ne[d]; n *= t.ne[d]; }
            if (t.type == GGML_F32) t.nbytes = (size_t) n * 4;
            else if (t.type == GGML_F16) t.nbytes = (size_t) n * 2;
            else if (t.type == GGML_Q8_0) t.nbytes = (size_t)(n / 32) * 34;
            else t.nbytes = 0;
            t.data = map_ + data_off + ti.off;
            if (data_off + ti.off + t.nbytes > size_) { err = "tensor data out of file: " + t.name; return false; }
            tensors_[t.name] = t;
        }
        return true;
    }

    uint8_t * map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, int64_t> ints_;
    std::map<std::string, double> floats_;
    std::map<std::string, GgufTensor> tensors_;
};

}  // namespace qtts
