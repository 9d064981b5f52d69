// cw_gguf.cpp -- GGUF v3 reader (chat-wgpu src/loader/gguf.rs:65-162).
#include "cw_gguf.h"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/chatcuda.h"
#include "cw_common.h"

namespace cw {

const char* ggml_type_name(uint32_t t) {
    switch (t) {
        case GGML_F32: return "F32";
        case GGML_F16: return "F16";
        case GGML_Q4_0: return "Q4_0";
        case GGML_Q4_1: return "Q4_1";
        case GGML_Q8_0: return "Q8_0";
        case GGML_Q4_K: return "Q4_K";
        case GGML_Q5_K: return "Q5_K";
        case GGML_Q6_K: return "Q6_K";
        case GGML_BF16: return "BF16";
        default: return "unknown";
    }
}

size_t ggml_row_bytes(uint32_t type, size_t n) {
    switch (type) {
        case GGML_F32: return n * 4;
        case GGML_F16: case GGML_BF16: return n * 2;
        case GGML_Q4_0: return n % 32 ? 0 : n / 32 * 18;
        case GGML_Q4_1: return n % 32 ? 0 : n / 32 * 20;
        case GGML_Q8_0: return n % 32 ? 0 : n / 32 * 34;
        case GGML_Q4_K: return n % 256 ? 0 : n / 256 * 144;
        case GGML_Q5_K: return n % 256 ? 0 : n / 256 * 176;
        case GGML_Q6_K: return n % 256 ? 0 : n / 256 * 210;
        default: return 0;
    }
}

namespace {
struct Cursor {
    const uint8_t* b;
    size_t n, p = 0;
    bool bad = false;
    bool need(size_t k) {
        if (bad || p + k > n || p + k < p) {
            bad = true;
            return false;
        }
        return true;
    }
    template <class T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, b + p, sizeof(T));
            p += sizeof(T);
        }
        return v;
    }
    std::string str() {
        uint64_t len = get<uint64_t>();
        if (!need(len)) return std::string();
        std::string s((const char*)b + p, (size_t)len);
        p += len;
        return s;
    }
    void skip(size_t k) {
        if (need(k)) p += k;
    }
};

// gguf.rs:153-162
void skip_scalar(Cursor& c, uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: c.skip(1); break;
        case 2: case 3: c.skip(2); break;
        case 4: case 5: case 6: c.skip(4); break;
        case 8: c.str(); break;
        case 10: case 11: case 12: c.skip(8); break;
        default: c.bad = true; break;  // unknown element type: cannot continue
    }
}
}  // namespace

GgufFile::~GgufFile() {
    if (map_) munmap(map_, map_len_);
}

int GgufFile::open(const std::string& path, std::string& err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return CW_ERR_NOT_FOUND;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        err = "not a GGUF file (too short): " + path;
        return CW_ERR_FORMAT;
    }
    void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) {
        err = "mmap failed: " + path;
        return CW_ERR_FORMAT;
    }
    map_ = p;
    map_len_ = (size_t)st.st_size;
    Cursor c{(const uint8_t*)p, map_len_};
    if (memcmp(p, "GGUF", 4) != 0) {
        err = "not a GGUF file";
        return CW_ERR_FORMAT;
    }
    c.skip(4);
    uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) {
        err = "unsupported GGUF version " + std::to_string(version);
        return CW_ERR_FORMAT;
    }
    uint64_t n_t = c.get<uint64_t>(), n_meta = c.get<uint64_t>();
    if (n_t > (1u << 24) || n_meta > (1u << 24)) {
        err = "implausible GGUF header counts";
        return CW_ERR_FORMAT;
    }
    // metadata: gguf.rs:77-82, value kinds :125-151
    for (uint64_t i = 0; i < n_meta && !c.bad; i++) {
        std::string key = c.str();
        uint32_t t = c.get<uint32_t>();
        GgufMeta m;
        switch (t) {
            case 0: m.kind = GgufMeta::U; m.u = c.get<uint8_t>(); break;
            case 1: m.kind = GgufMeta::U; m.u = (uint64_t)(int64_t)c.get<int8_t>(); break;
            case 2: m.kind = GgufMeta::U; m.u = c.get<uint16_t>(); break;
            case 3: m.kind = GgufMeta::U; m.u = (uint64_t)(int64_t)c.get<int16_t>(); break;
            case 4: m.kind = GgufMeta::U; m.u = c.get<uint32_t>(); break;
            case 5: m.kind = GgufMeta::U; m.u = (uint64_t)(int64_t)c.get<int32_t>(); break;
            case 6: m.kind = GgufMeta::F; m.f = c.get<float>(); break;
            case 7: m.kind = GgufMeta::U; m.u = c.get<uint8_t>(); break;
            case 8: m.kind = GgufMeta::S; m.s = c.str(); break;
            case 9: {
                uint32_t et = c.get<uint32_t>();
                uint64_t cnt = c.get<uint64_t>();
                for (uint64_t k = 0; k < cnt && !c.bad; k++) skip_scalar(c, et);
                break;
            }
            case 10: case 11: m.kind = GgufMeta::U; m.u = c.get<uint64_t>(); break;
            case 12: m.kind = GgufMeta::F; m.f = c.get<double>(); break;
            default: c.bad = true; break;
        }
        meta_[key] = m;
    }
    // tensor infos: gguf.rs:84-94
    tensors.reserve((size_t)n_t);
    for (uint64_t i = 0; i < n_t && !c.bad; i++) {
        GgufTensor t;
        t.name = c.str();
        uint32_t nd = c.get<uint32_t>();
        if (nd > 4) {
            c.bad = true;
            break;
        }
        // a zero or overflowing dimension would break the size arithmetic
        // below (rows = n_elems / dims[0], nbytes = row * rows)
        t.n_elems = 1;
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t v = c.get<uint64_t>();
            t.dims.push_back(v);
            if (v == 0 || __builtin_mul_overflow(t.n_elems, v, &t.n_elems)) {
                if (!c.bad) {
                    err = "tensor " + t.name + ": zero or overflowing dimension";
                    return CW_ERR_FORMAT;
                }
            }
        }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        tensors.push_back(std::move(t));
    }
    if (c.bad) {
        err = "truncated or malformed GGUF header";
        return CW_ERR_FORMAT;
    }
    // data section at the next `general.alignment` boundary (gguf.rs:96-102)
    uint64_t align = 32;
    if (const GgufMeta* a = meta("general.alignment"))
        if (a->kind == GgufMeta::U && a->u) align = a->u;
    size_t ds = (size_t)((c.p + align - 1) / align * align);
    if (ds > map_len_) {
        err = "GGUF data section out of range";
        return CW_ERR_FORMAT;
    }
    const uint8_t* data = (const uint8_t*)p + ds;
    size_t data_len = map_len_ - ds;
    data_bytes = data_len;
    for (size_t i = 0; i < tensors.size(); i++) {
        GgufTensor& t = tensors[i];
        size_t row = t.dims.empty() ? 0 : ggml_row_bytes(t.type, (size_t)t.dims[0]);
        size_t rows = t.dims.empty() ? 0 : (size_t)(t.n_elems / t.dims[0]);
        if (__builtin_mul_overflow(row, rows, &t.nbytes)) {
            err = "tensor " + t.name + ": byte size overflows";
            return CW_ERR_FORMAT;
        }
        if (t.nbytes && (t.offset > data_len || t.nbytes > data_len - t.offset)) {
            err = "tensor " + t.name + " extends past the end of the file";
            return CW_ERR_FORMAT;
        }
        t.data = data + t.offset;
        index_[t.name] = i;
    }
    return CW_OK;
}

const GgufMeta* GgufFile::meta(const std::string& key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? nullptr : &it->second;
}

uint32_t GgufFile::meta_u32(const std::string& key, uint32_t dflt) const {
    const GgufMeta* m = meta(key);
    if (m && m->kind == GgufMeta::U) return (uint32_t)m->u;
    if (m && m->kind == GgufMeta::F) return (uint32_t)m->f;
    return dflt;
}

float GgufFile::meta_f32(const std::string& key, float dflt) const {
    const GgufMeta* m = meta(key);
    if (m && m->kind == GgufMeta::F) return (float)m->f;
    if (m && m->kind == GgufMeta::U) return (float)m->u;
    return dflt;
}

std::string GgufFile::meta_str(const std::string& key) const {
    const GgufMeta* m = meta(key);
    return (m && m->kind == GgufMeta::S) ? m->s : std::string();
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors[it->second];
}

}  // namespace cw

extern "C" int cw_gguf_inspect(const char* path, size_t* n_tensors, uint64_t* data_bytes) {
    cw::clear_error();
    CW_CHECK(path, CW_ERR_INVALID_ARG, "cw_gguf_inspect: path is NULL");
    cw::GgufFile f;
    std::string err;
    const int rc = f.open(path, err);
    if (rc != CW_OK) return cw::set_error(rc, "%s", err.c_str());
    if (n_tensors) *n_tensors = f.tensors.size();
    if (data_bytes) *data_bytes = f.data_bytes;
    return CW_OK;
}
