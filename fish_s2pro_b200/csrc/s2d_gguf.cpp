// s2d_gguf.cpp -- GGUF v3 reader (see s2d_gguf.h).
#include "s2d_gguf.h"

#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>

namespace s2d {

int64_t ggml_byte_len(uint32_t type, uint64_t n) {
    switch (type) {
    case 0: return (int64_t)(n * 4);                  // F32
    case 1: return (int64_t)(n * 2);                  // F16
    case 8: return (int64_t)((n + 31) / 32 * 34);     // Q8_0
    case 12: return (int64_t)((n + 255) / 256 * 144); // Q4_K
    }
    return -1;
}

namespace {

struct Reader {
    const uint8_t *p;
    size_t pos, size;
    bool bad = false;
    bool need(size_t n) {
        if (bad || n > size - pos) bad = true;
        return !bad;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p + pos, sizeof(T));
            pos += sizeof(T);
        }
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!need((size_t)len)) return {};
        std::string s(reinterpret_cast<const char *>(p + pos), (size_t)len);
        pos += (size_t)len;
        return s;
    }
};

bool skip_value(Reader &r, uint32_t type, int depth) {
    switch (type) {
    case 0: case 1: case 7: r.get<uint8_t>(); break;
    case 2: case 3: r.get<uint16_t>(); break;
    case 4: case 5: case 6: r.get<uint32_t>(); break;
    case 10: case 11: case 12: r.get<uint64_t>(); break;
    case 8: r.str(); break;
    case 9: {
        if (depth > 4) return false;
        const uint32_t et = r.get<uint32_t>();
        const uint64_t len = r.get<uint64_t>();
        for (uint64_t i = 0; i < len && !r.bad; ++i)
            if (!skip_value(r, et, depth + 1)) return false;
        break;
    }
    default: return false;
    }
    return !r.bad;
}

}  // namespace

Gguf::~Gguf() {
    if (map_ && map_ != MAP_FAILED) munmap(const_cast<uint8_t *>(map_), size_);
    if (fd_ >= 0) close(fd_);
}

bool Gguf::open(const std::string &path, std::string *err) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) {
        *err = "IO: " + path + ": " + strerror(errno);
        return false;
    }
    struct stat st;
    if (fstat(fd_, &st) != 0) {
        *err = std::string("IO: ") + strerror(errno);
        return false;
    }
    size_ = (size_t)st.st_size;
    if (size_ < 4) {
        *err = "not a GGUF file: " + path;
        return false;
    }
    map_ = static_cast<const uint8_t *>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
    if (map_ == MAP_FAILED) {
        map_ = nullptr;
        *err = std::string("IO: mmap: ") + strerror(errno);
        return false;
    }
    if (memcmp(map_, "GGUF", 4) != 0) {
        *err = "not a GGUF file: " + path;
        return false;
    }
    Reader r{map_, 4, size_};
    version = r.get<uint32_t>();
    const uint64_t nt = r.get<uint64_t>(), nm = r.get<uint64_t>();
    if (r.bad || nt > (1u << 24) || nm > (1u << 24)) {
        *err = "GGUF header truncated or implausible";
        return false;
    }
    for (uint64_t i = 0; i < nm; ++i) {
        std::string key = r.str();
        GgufMeta m;
        m.type = r.get<uint32_t>();
        switch (m.type) {
        case 0: m.u = r.get<uint8_t>(); m.i = (int64_t)m.u; break;
        case 1: m.i = r.get<int8_t>(); m.u = (uint64_t)m.i; break;
        case 2: m.u = r.get<uint16_t>(); m.i = (int64_t)m.u; break;
        case 3: m.i = r.get<int16_t>(); m.u = (uint64_t)m.i; break;
        case 4: m.u = r.get<uint32_t>(); m.i = (int64_t)m.u; break;
        case 5: m.i = r.get<int32_t>(); m.u = (uint64_t)m.i; break;
        case 6: m.f = r.get<float>(); break;
        case 7: m.b = r.get<uint8_t>() != 0; break;
        case 8: m.s = r.str(); break;
        case 10: m.u = r.get<uint64_t>(); m.i = (int64_t)m.u; break;
        case 11: m.i = r.get<int64_t>(); m.u = (uint64_t)m.i; break;
        case 12: m.f = r.get<double>(); break;
        case 9: {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t len = r.get<uint64_t>();
            for (uint64_t k = 0; k < len && !r.bad; ++k)
                if (!skip_value(r, et, 1)) {
                    *err = "GGUF metadata array malformed";
                    return false;
                }
            break;
        }
        default: *err = "unknown GGUF value type: " + std::to_string(m.type); return false;
        }
        if (r.bad) {
            *err = "GGUF metadata truncated";
            return false;
        }
        meta_[key] = m;
    }
    tensors.reserve((size_t)nt);
    for (uint64_t i = 0; i < nt; ++i) {
        GgufTensor t;
        t.name = r.str();
        const uint32_t rank = r.get<uint32_t>();
        if (r.bad || rank > 4) {
            *err = "GGUF tensor info truncated or rank > 4";
            return false;
        }
        uint64_t count = 1;
        for (uint32_t k = 0; k < rank; ++k) {
            const uint64_t d = r.get<uint64_t>();
            if (d && count > UINT64_MAX / d) {
                *err = "tensor element count overflow: " + t.name;
                return false;
            }
            count *= d;
            t.dims.push_back(d);
        }
        t.type = r.get<uint32_t>();
        t.rel_offset = r.get<uint64_t>();
        t.elements = count;
        const int64_t bl = ggml_byte_len(t.type, count);
        if (bl < 0) {
            *err = "unsupported GGML tensor type " + std::to_string(t.type) + " for " + t.name;
            return false;
        }
        t.bytes = (uint64_t)bl;
        tensors.push_back(std::move(t));
    }
    if (r.bad) {
        *err = "GGUF truncated";
        return false;
    }
    const uint64_t data_start = (r.pos + 31) / 32 * 32;
    for (size_t i = 0; i < tensors.size(); ++i) {
        GgufTensor &t = tensors[i];
        const uint64_t start = data_start + t.rel_offset, end = start + t.bytes;
        if (end < start || end > size_) {
            *err = "tensor " + t.name + " extends past file end: " + std::to_string(end) + " > " +
                   std::to_string(size_);
            return false;
        }
        t.data = map_ + start;
        if (!index_.count(t.name)) index_[t.name] = i;  // first match wins (gguf.rs:75-77)
    }
    return true;
}

const GgufTensor *Gguf::tensor(const std::string &name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors[it->second];
}

const GgufMeta *Gguf::meta(const std::string &key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? nullptr : &it->second;
}

bool Gguf::meta_u32(const std::string &key, uint32_t *out, std::string *err) const {
    const GgufMeta *m = meta(key);
    if (!m) return *err = "missing " + key, false;
    const bool is_int = m->type <= 5 || m->type == 10 || m->type == 11;
    if (!is_int || m->i < 0 || m->u > 0xffffffffull)
        return *err = "invalid u32 metadata " + key, false;
    *out = (uint32_t)m->u;
    return true;
}

bool Gguf::meta_f32(const std::string &key, float *out, std::string *err) const {
    const GgufMeta *m = meta(key);
    if (!m) return *err = "missing " + key, false;
    if (m->type == 6 || m->type == 12) *out = (float)m->f;
    else if (m->type <= 5 || m->type == 10 || m->type == 11) *out = (float)m->i;
    else return *err = "invalid f32 metadata " + key, false;
    return true;
}

bool Gguf::meta_bool(const std::string &key, bool *out, std::string *err) const {
    const GgufMeta *m = meta(key);
    if (!m) return *err = "missing " + key, false;
    if (m->type != 7) return *err = "invalid bool metadata " + key, false;
    *out = m->b;
    return true;
}

bool Gguf::meta_str(const std::string &key, std::string *out, std::string *err) const {
    const GgufMeta *m = meta(key);
    if (!m) return *err = "missing " + key, false;
    if (m->type != 8) return *err = "invalid string metadata " + key, false;
    *out = m->s;
    return true;
}

}  // namespace s2d
