#include "gguf.h"

#include <cstring>
#include <functional>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace dfh {

int64_t ggml_block_size(int32_t t) {
    switch (t) {
        case GT_Q8_0: return 32;
        case GT_Q4_K: case GT_Q6_K: return 256;
        default: return 1;
    }
}
int64_t ggml_type_size(int32_t t) {
    switch (t) {
        case GT_F32: return 4;
        case GT_F16: case GT_BF16: return 2;
        case GT_Q8_0: return 34;
        case GT_Q4_K: return 144;
        case GT_Q6_K: return 210;
        default: return 0;
    }
}
int64_t ggml_row_size(int32_t t, int64_t n) {
    const int64_t ts = ggml_type_size(t);
    return ts ? n / ggml_block_size(t) * ts : -1;
}
const char *ggml_type_name(int32_t t) {
    switch (t) {
        case GT_F32: return "f32";
        case GT_F16: return "f16";
        case GT_BF16: return "bf16";
        case GT_Q8_0: return "q8_0";
        case GT_Q4_K: return "q4_K";
        case GT_Q6_K: return "q6_K";
        default: return "?";
    }
}

GgufReader::~GgufReader() {
    if (map_) munmap(map_, size_);
}

bool GgufReader::open(const std::string &path, std::string *err) {
    auto fail = [&](const std::string &m) { if (err) *err = m; return false; };
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail("cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); return fail("cannot stat " + path); }
    size_ = (size_t)st.st_size;
    void *p = size_ ? mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    ::close(fd);
    if (p == MAP_FAILED) return fail("cannot map " + path);
    map_ = p;
    const uint8_t *cur = (const uint8_t *)map_, *end = cur + size_;
    auto rd = [&](void *dst, size_t n) {
        if ((size_t)(end - cur) < n) return false;
        memcpy(dst, cur, n);
        cur += n;
        return true;
    };
    auto rstr = [&](std::string &s) {
        uint64_t n;
        if (!rd(&n, 8) || (uint64_t)(end - cur) < n) return false;
        s.assign((const char *)cur, n);
        cur += n;
        return true;
    };
    uint32_t magic = 0, version = 0;
    uint64_t nt = 0, nkv = 0;
    if (!rd(&magic, 4) || magic != 0x46554747u) return fail(path + ": not a GGUF file");
    if (!rd(&version, 4) || version < 2 || version > 3) return fail(path + ": unsupported GGUF version");
    if (!rd(&nt, 8) || !rd(&nkv, 8) || nt > (1u << 24) || nkv > (1u << 24)) return fail(path + ": truncated header");
    static const int ssz[13] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -1, 8, 8, 8};
    std::function<bool(int32_t, GgufValue *)> rval = [&](int32_t t, GgufValue *v) -> bool {
        if (t == 8) { std::string s; if (!rstr(s)) return false; if (v) v->s = s; return true; }
        if (t == 9) {
            int32_t at; uint64_t n;
            if (!rd(&at, 4) || !rd(&n, 8)) return false;
            for (uint64_t i = 0; i < n; i++) if (!rval(at, nullptr)) return false;
            return true;
        }
        if (t < 0 || t > 12 || ssz[t] < 0) return false;
        uint8_t b[8] = {0};
        if (!rd(b, ssz[t])) return false;
        if (v) {
            switch (t) {
                case 0: case 7: v->u = b[0]; break;
                case 1: v->u = (uint64_t)(int64_t)(int8_t)b[0]; break;
                case 2: { uint16_t x; memcpy(&x, b, 2); v->u = x; } break;
                case 3: { int16_t x; memcpy(&x, b, 2); v->u = (uint64_t)(int64_t)x; } break;
                case 4: { uint32_t x; memcpy(&x, b, 4); v->u = x; } break;
                case 5: { int32_t x; memcpy(&x, b, 4); v->u = (uint64_t)(int64_t)x; } break;
                case 6: { float x; memcpy(&x, b, 4); v->f = x; } break;
                case 10: case 11: memcpy(&v->u, b, 8); break;
                case 12: memcpy(&v->f, b, 8); break;
            }
        }
        return true;
    };
    for (uint64_t i = 0; i < nkv; i++) {
        std::string key;
        int32_t t;
        GgufValue v;
        if (!rstr(key) || !rd(&t, 4)) return fail(path + ": truncated metadata");
        v.type = t;
        if (!rval(t, &v)) return fail(path + ": bad metadata value for " + key);
        kv_[key] = v;
    }
    tensors_.resize(nt);
    for (uint64_t i = 0; i < nt; i++) {
        GgufTensor &T = tensors_[i];
        uint32_t nd;
        if (!rstr(T.name) || !rd(&nd, 4) || nd == 0 || nd > 4) return fail(path + ": bad tensor info");
        T.n_dims = (int)nd;
        for (uint32_t d = 0; d < nd; d++) if (!rd(&T.ne[d], 8) || T.ne[d] < 0) return fail(path + ": bad tensor dims");
        if (!rd(&T.type, 4) || !rd(&T.offset, 8)) return fail(path + ": bad tensor info");
        if (ggml_type_size(T.type) == 0) return fail(path + ": tensor " + T.name + " has unsupported type " + std::to_string(T.type));
        if (T.ne[0] % ggml_block_size(T.type)) return fail(path + ": tensor " + T.name + " row not a whole number of blocks");
    }
    uint64_t align = 32;
    auto a = kv_.find("general.alignment");
    if (a != kv_.end() && a->second.u) align = a->second.u;
    uint64_t off = (uint64_t)(cur - (const uint8_t *)map_);
    off = (off + align - 1) / align * align;
    for (size_t i = 0; i < tensors_.size(); i++) {
        GgufTensor &T = tensors_[i];
        const int64_t rows = T.ne[1] * T.ne[2] * T.ne[3];
        T.nbytes = (size_t)(ggml_row_size(T.type, T.ne[0]) * rows);
        if (off + T.offset + T.nbytes > size_) return fail(path + ": tensor " + T.name + " data past end of file (truncated?)");
        T.data = (const uint8_t *)map_ + off + T.offset;
        index_[T.name] = i;
    }
    return true;
}

const GgufValue *GgufReader::find(const std::string &key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}
const GgufTensor *GgufReader::tensor(const std::string &name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

void GgufWriter::add_u32(const std::string &k, uint32_t v) { kv_.push_back({k, 4, v, 0, ""}); }
void GgufWriter::add_f32(const std::string &k, float v) { kv_.push_back({k, 6, 0, v, ""}); }
void GgufWriter::add_str(const std::string &k, const std::string &v) { kv_.push_back({k, 8, 0, 0, v}); }
void GgufWriter::add_tensor_info(const std::string &name, int32_t type, int n_dims, const int64_t *ne) {
    TI t{name, type, n_dims, {1, 1, 1, 1}, 0, 0};
    int64_t rows = 1;
    for (int d = 0; d < n_dims; d++) { t.ne[d] = ne[d]; if (d) rows *= ne[d]; }
    t.nbytes = (size_t)(ggml_row_size(type, ne[0]) * rows);
    t.offset = data_bytes_;
    data_bytes_ += (t.nbytes + 31) / 32 * 32;
    ti_.push_back(t);
}

bool GgufWriter::begin(const std::string &path, std::string *err) {
    f_ = fopen(path.c_str(), "wb");
    if (!f_) { if (err) *err = "cannot create " + path; return false; }
    auto w = [&](const void *p, size_t n) { fwrite(p, 1, n, f_); };
    auto ws = [&](const std::string &s) { uint64_t n = s.size(); w(&n, 8); w(s.data(), n); };
    const uint32_t magic = 0x46554747u, version = 3;
    const uint64_t nt = ti_.size(), nkv = kv_.size();
    w(&magic, 4); w(&version, 4); w(&nt, 8); w(&nkv, 8);
    for (auto &k : kv_) {
        ws(k.key);
        w(&k.type, 4);
        if (k.type == 4) w(&k.u, 4);
        else if (k.type == 6) w(&k.f, 4);
        else ws(k.s);
    }
    for (auto &t : ti_) {
        ws(t.name);
        const uint32_t nd = t.n_dims;
        w(&nd, 4);
        for (int d = 0; d < t.n_dims; d++) w(&t.ne[d], 8);
        w(&t.type, 4);
        w(&t.offset, 8);
    }
    const long pos = ftell(f_);
    static const uint8_t zeros[32] = {0};
    if (pos % 32) w(zeros, 32 - pos % 32);
    next_ = 0;
    return !ferror(f_);
}

bool GgufWriter::write_tensor_data(const void *data, size_t nbytes, std::string *err) {
    if (next_ >= ti_.size() || ti_[next_].nbytes != nbytes) {
        if (err) *err = "tensor data out of order or wrong size";
        return false;
    }
    fwrite(data, 1, nbytes, f_);
    static const uint8_t zeros[32] = {0};
    if (nbytes % 32) fwrite(zeros, 1, 32 - nbytes % 32, f_);
    next_++;
    return !ferror(f_);
}

bool GgufWriter::finish(std::string *err) {
    bool ok = f_ && next_ == ti_.size() && !ferror(f_);
    if (f_) ok = (fclose(f_) == 0) && ok;
    f_ = nullptr;
    if (!ok && err) *err = "incomplete GGUF write";
    return ok;
}

}  // namespace dfh
