// gguf_file.h: a reader of GGUF files (format versions 2 and 3) for the model loader (tr_gpu_moe_config_from_gguf,
// tr_gpu_moe_load_gguf): the header, the metadata's scalars and strings, the tensor directory, and each tensor's
// bytes through a read-only mapping of the file. Model files come from outside: every count, length, dimension and
// offset is checked against the file's size before it is used, and a malformed file is an error, never a read
// outside the mapping. Host code only.
//
// The format (little-endian): "GGUF", version u32, tensor count u64, metadata count u64; each metadata entry a
// string key, a u32 value type and the value (strings are a u64 length and the bytes; arrays a u32 element type, a
// u64 count and the elements); each tensor a string name, a u32 dimension count, that many u64 dimensions (ggml
// order: the first is the row length), a u32 ggml type and a u64 offset into the data section; the data section
// starts at the next multiple of general.alignment (32 when absent) after the directory.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

// ggml's block of a tensor type: elements and bytes (the format's table of type numbers); false for a number that
// is not a known type
inline bool trx_ggml_block(uint32_t type, uint32_t &elems, uint32_t &bytes) {
    struct B {
        uint32_t type, elems, bytes;
    };
    static const B table[] = {{0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},   {6, 32, 22},
                              {7, 32, 24},    {8, 32, 34},    {9, 32, 36},    {10, 256, 84}, {11, 256, 110},
                              {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292}, {24, 1, 1},
                              {25, 1, 2},     {26, 1, 4},     {27, 1, 8},     {28, 1, 8},    {30, 1, 2}};
    for (const B &b : table)
        if (b.type == type) {
            elems = b.elems;
            bytes = b.bytes;
            return true;
        }
    return false;
}

enum : uint32_t {
    TRX_GGUF_U8 = 0, TRX_GGUF_I8 = 1, TRX_GGUF_U16 = 2, TRX_GGUF_I16 = 3, TRX_GGUF_U32 = 4, TRX_GGUF_I32 = 5,
    TRX_GGUF_F32 = 6, TRX_GGUF_BOOL = 7, TRX_GGUF_STRING = 8, TRX_GGUF_ARRAY = 9, TRX_GGUF_U64 = 10,
    TRX_GGUF_I64 = 11, TRX_GGUF_F64 = 12
};

struct TrxGgufKv {
    uint32_t type = 0;
    uint64_t u = 0;   // unsigned integers and bool
    int64_t i = 0;    // signed integers
    double f = 0.0;   // floats
    std::string s;    // string
};

struct TrxGgufTensor {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0; // from the start of the file
    uint64_t n_bytes = 0;
};

class TrxGguf {
  public:
    TrxGguf() = default;
    TrxGguf(const TrxGguf &) = delete;
    TrxGguf &operator=(const TrxGguf &) = delete;
    ~TrxGguf() { close(); }

    bool open(const char *path, std::string &err) {
        close();
        fd_ = ::open(path, O_RDONLY | O_CLOEXEC);
        if (fd_ < 0) return fail(err, std::string("cannot open '") + path + "': " + strerror(errno));
        struct stat st;
        if (fstat(fd_, &st) != 0 || st.st_size <= 0) return fail(err, std::string("cannot size '") + path + "'");
        size_ = (size_t)st.st_size;
        void *p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p == MAP_FAILED) return fail(err, std::string("cannot map '") + path + "': " + strerror(errno));
        base_ = static_cast<const uint8_t *>(p);
        Cur c{base_, size_, 0, true};
        uint32_t magic = 0, version = 0;
        uint64_t n_tensors = 0, n_kv = 0;
        if (!c.u32(magic) || magic != 0x46554747u) return fail(err, "not a GGUF file");
        if (!c.u32(version) || (version != 2 && version != 3))
            return fail(err, "GGUF version " + std::to_string(version) + " not supported (2 or 3)");
        version_ = version;
        if (!c.u64(n_tensors) || !c.u64(n_kv)) return fail(err, "truncated header");
        // every entry takes at least 12 bytes (metadata) or 28 bytes (tensor): counts beyond that are malformed
        if (n_kv > (size_ - c.pos) / 12 || n_tensors > (size_ - c.pos) / 28) return fail(err, "counts beyond the file");
        for (uint64_t k = 0; k < n_kv; k++) {
            std::string key;
            TrxGgufKv v;
            if (!c.str(key) || !c.u32(v.type)) return fail(err, "truncated metadata entry " + std::to_string(k));
            if (!value(c, v)) return fail(err, "metadata '" + key + "': bad or truncated value");
            kvs_[key] = std::move(v);
        }
        uint64_t align = 32;
        if (const TrxGgufKv *a = kv("general.alignment")) {
            uint32_t a32 = 0;
            if (!as_u32(*a, a32) || a32 == 0 || (a32 & (a32 - 1)) != 0 || a32 > 65536)
                return fail(err, "general.alignment must be a power of two <= 65536");
            align = a32;
        }
        tensors_.resize((size_t)n_tensors);
        for (uint64_t t = 0; t < n_tensors; t++) {
            TrxGgufTensor &x = tensors_[(size_t)t];
            if (!c.str(x.name) || !c.u32(x.n_dims)) return fail(err, "truncated tensor entry " + std::to_string(t));
            if (x.n_dims < 1 || x.n_dims > 4) return fail(err, "tensor '" + x.name + "' has a bad dimension count");
            for (uint32_t d = 0; d < x.n_dims; d++)
                if (!c.u64(x.ne[d])) return fail(err, "tensor '" + x.name + "': truncated");
            if (!c.u32(x.type) || !c.u64(x.offset)) return fail(err, "tensor '" + x.name + "': truncated");
            if (index_.count(x.name)) return fail(err, "tensor '" + x.name + "' appears twice");
            index_[x.name] = (size_t)t;
        }
        const uint64_t data = (c.pos + align - 1) / align * align;
        for (TrxGgufTensor &x : tensors_) {
            uint32_t be = 0, bb = 0;
            if (!trx_ggml_block(x.type, be, bb))
                return fail(err, "tensor '" + x.name + "' has unknown type " + std::to_string(x.type));
            uint64_t n = 1;
            for (uint32_t d = 0; d < 4; d++) {
                if (x.ne[d] != 0 && n > (UINT64_C(1) << 62) / x.ne[d])
                    return fail(err, "tensor '" + x.name + "' is too large");
                n *= x.ne[d];
            }
            if (x.ne[0] % be != 0) return fail(err, "tensor '" + x.name + "': rows are not whole blocks");
            x.n_bytes = n / be * bb;
            if (x.offset % align != 0) return fail(err, "tensor '" + x.name + "' is not aligned");
            if (x.offset > size_ || data > size_ - x.offset || x.n_bytes > size_ - x.offset - data)
                return fail(err, "tensor '" + x.name + "' lies beyond the end of the file");
            x.offset += data;
        }
        return true;
    }

    void close() {
        if (base_) munmap(const_cast<uint8_t *>(base_), size_);
        if (fd_ >= 0) ::close(fd_);
        base_ = nullptr;
        fd_ = -1;
        size_ = 0;
        kvs_.clear();
        tensors_.clear();
        index_.clear();
    }

    uint32_t version() const { return version_; }
    const TrxGgufKv *kv(const std::string &key) const {
        auto it = kvs_.find(key);
        return it == kvs_.end() ? nullptr : &it->second;
    }
    const TrxGgufTensor *tensor(const std::string &name) const {
        auto it = index_.find(name);
        return it == index_.end() ? nullptr : &tensors_[it->second];
    }
    const uint8_t *bytes(const TrxGgufTensor &t) const { return base_ + t.offset; }

    // typed reads: false when the key is absent or its value does not fit (an integer of any type in range)
    bool get_u32(const std::string &key, uint32_t &out) const {
        const TrxGgufKv *v = kv(key);
        return v != nullptr && as_u32(*v, out);
    }
    bool get_f32(const std::string &key, float &out) const {
        const TrxGgufKv *v = kv(key);
        if (v == nullptr || (v->type != TRX_GGUF_F32 && v->type != TRX_GGUF_F64)) return false;
        out = (float)v->f;
        return true;
    }
    bool get_bool(const std::string &key, bool &out) const {
        const TrxGgufKv *v = kv(key);
        if (v == nullptr || v->type != TRX_GGUF_BOOL) return false;
        out = v->u != 0;
        return true;
    }
    bool get_str(const std::string &key, std::string &out) const {
        const TrxGgufKv *v = kv(key);
        if (v == nullptr || v->type != TRX_GGUF_STRING) return false;
        out = v->s;
        return true;
    }

  private:
    // a bounds-checked cursor over the mapping
    struct Cur {
        const uint8_t *p;
        size_t n, pos;
        bool ok;
        bool take(void *dst, size_t k) {
            if (!ok || k > n - pos) return ok = false;
            memcpy(dst, p + pos, k);
            pos += k;
            return true;
        }
        bool skip(uint64_t k) {
            if (!ok || k > n - pos) return ok = false;
            pos += (size_t)k;
            return true;
        }
        bool u32(uint32_t &v) { return take(&v, 4); }
        bool u64(uint64_t &v) { return take(&v, 8); }
        bool str(std::string &s) {
            uint64_t len = 0;
            if (!u64(len) || len > n - pos) return ok = false;
            s.assign(reinterpret_cast<const char *>(p + pos), (size_t)len);
            pos += (size_t)len;
            return true;
        }
    };

    static size_t scalar_bytes(uint32_t type) {
        switch (type) {
        case TRX_GGUF_U8: case TRX_GGUF_I8: case TRX_GGUF_BOOL: return 1;
        case TRX_GGUF_U16: case TRX_GGUF_I16: return 2;
        case TRX_GGUF_U32: case TRX_GGUF_I32: case TRX_GGUF_F32: return 4;
        case TRX_GGUF_U64: case TRX_GGUF_I64: case TRX_GGUF_F64: return 8;
        default: return 0;
        }
    }

    // one value of v.type at the cursor: scalars and strings kept, arrays checked and skipped (nested ones refused)
    static bool value(Cur &c, TrxGgufKv &v) {
        if (v.type == TRX_GGUF_STRING) return c.str(v.s);
        if (v.type == TRX_GGUF_ARRAY) {
            uint32_t et = 0;
            uint64_t cnt = 0;
            if (!c.u32(et) || !c.u64(cnt) || et == TRX_GGUF_ARRAY) return false;
            if (et == TRX_GGUF_STRING) {
                for (uint64_t i = 0; i < cnt; i++) {
                    uint64_t len = 0;
                    if (!c.u64(len) || !c.skip(len)) return false;
                }
                return true;
            }
            const size_t sb = scalar_bytes(et);
            return sb != 0 && cnt <= (c.n - c.pos) / sb && c.skip(cnt * sb);
        }
        const size_t sb = scalar_bytes(v.type);
        if (sb == 0) return false;
        uint8_t raw[8] = {0};
        if (!c.take(raw, sb)) return false;
        switch (v.type) {
        case TRX_GGUF_U8: case TRX_GGUF_BOOL: v.u = raw[0]; break;
        case TRX_GGUF_I8: v.i = (int8_t)raw[0]; break;
        case TRX_GGUF_U16: { uint16_t x; memcpy(&x, raw, 2); v.u = x; break; }
        case TRX_GGUF_I16: { int16_t x; memcpy(&x, raw, 2); v.i = x; break; }
        case TRX_GGUF_U32: { uint32_t x; memcpy(&x, raw, 4); v.u = x; break; }
        case TRX_GGUF_I32: { int32_t x; memcpy(&x, raw, 4); v.i = x; break; }
        case TRX_GGUF_F32: { float x; memcpy(&x, raw, 4); v.f = x; break; }
        case TRX_GGUF_U64: memcpy(&v.u, raw, 8); break;
        case TRX_GGUF_I64: memcpy(&v.i, raw, 8); break;
        case TRX_GGUF_F64: memcpy(&v.f, raw, 8); break;
        }
        return true;
    }

    static bool as_u32(const TrxGgufKv &v, uint32_t &out) {
        switch (v.type) {
        case TRX_GGUF_U8: case TRX_GGUF_U16: case TRX_GGUF_U32: case TRX_GGUF_U64:
            if (v.u > UINT32_MAX) return false;
            out = (uint32_t)v.u;
            return true;
        case TRX_GGUF_I8: case TRX_GGUF_I16: case TRX_GGUF_I32: case TRX_GGUF_I64:
            if (v.i < 0 || v.i > (int64_t)UINT32_MAX) return false;
            out = (uint32_t)v.i;
            return true;
        default: return false;
        }
    }

    bool fail(std::string &err, const std::string &msg) {
        err = msg;
        close();
        return false;
    }

    int fd_ = -1;
    const uint8_t *base_ = nullptr;
    size_t size_ = 0;
    uint32_t version_ = 0;
    std::unordered_map<std::string, TrxGgufKv> kvs_;
    std::vector<TrxGgufTensor> tensors_;
    std::unordered_map<std::string, size_t> index_;
};
