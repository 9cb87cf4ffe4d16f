// nf_safetensors.hpp -- a read-only safetensors checkpoint store for the C++
// host: the shards of a checkpoint directory mapped into memory and indexed
// by tensor name, handing out nf_host::TensorView for MoeLayer / DenseMlp
// bind_from_store.  It stands where the reference's Store does
// (src/text_forward.cpp:328-495): the shards listed in
// model.safetensors.index.json (or a single model.safetensors) are mapped
// PROT_READ / MAP_PRIVATE, each header's dtype / shape / data_offsets is
// parsed, the four kinds of the MoE path are accepted (BF16 'b', F32 'f',
// U8 'u', F8_E4M3 '8'), and failures carry the reference's messages
// ("missing model.safetensors.index.json", "cannot open shard <path>",
// "bad safetensors header", "unsupported dtype <d> for <name>", "missing
// tensor <name>").  Beyond the reference, every tensor's byte range is
// checked against its shard and its shape ("tensor data out of range for
// <name>", "tensor size mismatch for <name>"), so a truncated or corrupt
// shard fails at open instead of at the first read past the mapping.
// Header-only, POSIX.
#pragma once

#include "nf_moe_layer.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

namespace nf_host {

namespace st_detail {

// Minimal JSON reader over the subset safetensors headers and indexes use:
// objects, arrays, strings (with escapes), integers, and values skipped whole.
class Json {
public:
    explicit Json(const std::string& text, size_t pos = 0) : s_(text), i_(pos) {}
    char peek() {
        ws();
        if (i_ >= s_.size()) throw std::runtime_error("bad safetensors header");
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) throw std::runtime_error("bad safetensors header");
        ++i_;
    }
    bool maybe(char c) {
        if (peek() != c) return false;
        ++i_;
        return true;
    }
    std::string str() {
        expect('"');
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) break;
                const char e = s_[i_++];
                if (e == 'u') {  // names are ASCII in practice; keep the code point's low byte
                    if (i_ + 4 > s_.size()) break;
                    unsigned v = 0;
                    for (int k = 0; k < 4; ++k) {
                        const char h = s_[i_ + k];
                        const int digit = h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                          : h >= 'A' && h <= 'F' ? h - 'A' + 10 : -1;
                        if (digit < 0) throw std::runtime_error("bad safetensors header");
                        v = v * 16 + static_cast<unsigned>(digit);
                    }
                    c = static_cast<char>(v & 0xffu);
                    i_ += 4;
                } else {
                    c = e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == 'b' ? '\b' : e == 'f' ? '\f' : e;
                }
            }
            out.push_back(c);
        }
        if (i_ >= s_.size()) throw std::runtime_error("bad safetensors header");
        ++i_;
        return out;
    }
    int64_t integer() {
        ws();
        size_t j = i_;
        if (j < s_.size() && (s_[j] == '-' || s_[j] == '+')) ++j;
        const size_t digits = j;
        while (j < s_.size() && s_[j] >= '0' && s_[j] <= '9') ++j;
        if (j == digits || j - digits > 18) throw std::runtime_error("bad safetensors header");
        const int64_t v = std::stoll(s_.substr(i_, j - i_));
        i_ = j;
        return v;
    }
    void skip() {
        const char c = peek();
        if (c == '"') {
            str();
        } else if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++i_;
            if (maybe(close)) return;
            for (;;) {
                if (c == '{') {
                    str();
                    expect(':');
                }
                skip();
                if (maybe(',')) continue;
                expect(close);
                return;
            }
        } else {
            while (i_ < s_.size() && std::strchr(",}] \t\r\n", s_[i_]) == nullptr) ++i_;
        }
    }

private:
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\r' || s_[i_] == '\n')) ++i_;
    }
    const std::string& s_;
    size_t i_;
};

struct Mapping {
    void* addr = MAP_FAILED;
    size_t len = 0;
    int fd = -1;
    ~Mapping() {
        if (addr != MAP_FAILED) ::munmap(addr, len);
        if (fd >= 0) ::close(fd);
    }
};

inline size_t elem_bytes(char kind) { return kind == 'b' ? 2 : kind == 'f' ? 4 : 1; }

}  // namespace st_detail

class SafetensorsStore {
public:
    explicit SafetensorsStore(const std::string& directory) {
        const std::string dir = directory.empty() || directory.back() == '/' ? directory : directory + "/";
        std::vector<std::string> shards;
        std::ifstream index(dir + "model.safetensors.index.json", std::ios::binary);
        if (!index) {
            std::ifstream single(dir + "model.safetensors", std::ios::binary);
            if (!single) throw std::runtime_error("missing model.safetensors.index.json");
            shards.push_back("model.safetensors");
        } else {
            const std::string text{std::istreambuf_iterator<char>(index), std::istreambuf_iterator<char>()};
            if (text.empty()) throw std::runtime_error("empty safetensors index");
            const size_t at = text.find("\"weight_map\"");
            if (at == std::string::npos) throw std::runtime_error("index has no weight_map");
            st_detail::Json j(text, at);
            j.str();
            j.expect(':');
            j.expect('{');
            std::set<std::string> seen;
            if (!j.maybe('}')) {
                for (;;) {
                    j.str();
                    j.expect(':');
                    const std::string shard = j.str();
                    if (seen.insert(shard).second) shards.push_back(shard);
                    if (j.maybe(',')) continue;
                    j.expect('}');
                    break;
                }
            }
        }
        for (const std::string& shard : shards) open_shard(dir + shard);
    }
    SafetensorsStore(const SafetensorsStore&) = delete;
    SafetensorsStore& operator=(const SafetensorsStore&) = delete;

    // NULL when the name is absent (bind_from_store then throws "missing tensor <name>").
    const TensorView* find(const std::string& name) const {
        const auto it = tensors_.find(name);
        return it == tensors_.end() ? nullptr : &it->second;
    }
    const TensorView& get(const std::string& name) const {
        const TensorView* t = find(name);
        if (!t) throw std::runtime_error("missing tensor " + name);
        return *t;
    }
    StoreLookup lookup() const {
        return [this](const std::string& name) { return find(name); };
    }
    size_t tensor_count() const { return tensors_.size(); }
    size_t shard_count() const { return maps_.size(); }
    uint64_t data_bytes() const { return data_bytes_; }

private:
    void open_shard(const std::string& path) {
        auto m = std::make_unique<st_detail::Mapping>();
        m->fd = ::open(path.c_str(), O_RDONLY);
        if (m->fd < 0) throw std::runtime_error("cannot open shard " + path);
        struct stat info {};
        if (::fstat(m->fd, &info) != 0 || info.st_size <= 0) throw std::runtime_error("cannot stat shard " + path);
        m->len = static_cast<size_t>(info.st_size);
        m->addr = ::mmap(nullptr, m->len, PROT_READ, MAP_PRIVATE, m->fd, 0);
        if (m->addr == MAP_FAILED) throw std::runtime_error("cannot map shard " + path);
        const auto* bytes = static_cast<const unsigned char*>(m->addr);
        if (m->len < 8) throw std::runtime_error("short safetensors file");
        uint64_t hlen = 0;
        for (int i = 0; i < 8; ++i) hlen |= static_cast<uint64_t>(bytes[i]) << (8 * i);
        if (hlen == 0 || hlen > m->len - 8) throw std::runtime_error("bad safetensors header");
        const std::string header(reinterpret_cast<const char*>(bytes + 8), static_cast<size_t>(hlen));
        const unsigned char* data = bytes + 8 + hlen;
        const uint64_t data_len = m->len - 8 - hlen;
        st_detail::Json j(header);
        j.expect('{');
        if (!j.maybe('}')) {
            for (;;) {
                const std::string name = j.str();
                j.expect(':');
                if (name == "__metadata__") {
                    j.skip();
                } else {
                    parse_tensor(j, name, data, data_len);
                }
                if (j.maybe(',')) continue;
                j.expect('}');
                break;
            }
        }
        maps_.push_back(std::move(m));
    }

    void parse_tensor(st_detail::Json& j, const std::string& name, const unsigned char* data, uint64_t data_len) {
        TensorView t;
        int64_t begin = -1, end = -1;
        bool have_shape = false;
        j.expect('{');
        for (;;) {
            const std::string key = j.str();
            j.expect(':');
            if (key == "dtype") {
                const std::string d = j.str();
                if (d == "BF16") t.kind = 'b';
                else if (d == "F32") t.kind = 'f';
                else if (d == "U8") t.kind = 'u';
                else if (d == "F8_E4M3") t.kind = '8';
                else throw std::runtime_error("unsupported dtype " + d + " for " + name);
            } else if (key == "shape") {
                have_shape = true;
                j.expect('[');
                if (!j.maybe(']')) {
                    for (;;) {
                        if (t.shape.size() >= 8) throw std::runtime_error("rank above 8 for " + name);
                        const int64_t v = j.integer();
                        if (v < 0) throw std::runtime_error("negative dimension for " + name);
                        t.shape.push_back(v);
                        if (j.maybe(',')) continue;
                        j.expect(']');
                        break;
                    }
                }
            } else if (key == "data_offsets") {
                j.expect('[');
                begin = j.integer();
                j.expect(',');
                end = j.integer();
                j.expect(']');
            } else {
                j.skip();
            }
            if (j.maybe(',')) continue;
            j.expect('}');
            break;
        }
        if (t.kind == '?' || !have_shape || begin < 0) throw std::runtime_error("incomplete tensor header for " + name);
        if (end < begin || static_cast<uint64_t>(end) > data_len)
            throw std::runtime_error("tensor data out of range for " + name);
        // (below 2^60 elements the byte count cannot wrap: at most 4 bytes each)
        uint64_t count = 1;
        for (int64_t d : t.shape) {
            if (d > 0 && count > (uint64_t{1} << 60) / static_cast<uint64_t>(d))
                throw std::runtime_error("tensor size mismatch for " + name);  // larger than any shard
            count *= static_cast<uint64_t>(d);
        }
        if (count * st_detail::elem_bytes(t.kind) != static_cast<uint64_t>(end - begin))
            throw std::runtime_error("tensor size mismatch for " + name);
        t.data = data + begin;
        data_bytes_ += static_cast<uint64_t>(end - begin);
        tensors_[name] = std::move(t);
    }

    std::vector<std::unique_ptr<st_detail::Mapping>> maps_;
    std::map<std::string, TensorView> tensors_;
    uint64_t data_bytes_ = 0;
};

}  // namespace nf_host
