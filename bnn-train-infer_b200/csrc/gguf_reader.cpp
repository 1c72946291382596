// gguf_reader.cpp - see gguf_reader.h.
#include "gguf_reader.h"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace bnn {

namespace {

enum : uint32_t {
    kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64
};

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    bool need(size_t n) {
        if (!ok || (size_t)(end - p) < n)
            ok = false;
        return ok;
    }
    template <typename T>
    T get() {
        T v{};
        if (need(sizeof(T))) {
            std::memcpy(&v, p, sizeof(T));
            p += sizeof(T);
        }
        return v;
    }
    std::string str() {
        uint64_t n = get<uint64_t>();
        if (!need(n))
            return {};
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
    }
}

}  // namespace

GgufFile::~GgufFile() {
    if (map_)
        munmap(map_, map_bytes_);
}

bool GgufFile::fail(const std::string& why) {
    error_ = why;
    return false;
}

bool GgufFile::open(const char* path) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0)
        return fail(std::string(path) + ": cannot open GGUF file");
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        ::close(fd);
        return fail(std::string(path) + ": cannot stat GGUF file");
    }
    map_bytes_ = (size_t)st.st_size;
    void* m = mmap(nullptr, map_bytes_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        map_ = nullptr;
        return fail(std::string(path) + ": cannot mmap GGUF file");
    }
    map_ = static_cast<uint8_t*>(m);
    Cursor c{map_, map_ + map_bytes_};
    char magic[4];
    for (char& ch : magic)
        ch = (char)c.get<uint8_t>();
    uint32_t version = c.get<uint32_t>();
    uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (!c.ok || std::memcmp(magic, "GGUF", 4) != 0 || version != 3)
        return fail("unsupported GGUF header or version");
    if (n_kv > 65536 || n_tensors > (1u << 20))
        return fail("implausible GGUF table sizes");
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        uint32_t type = c.get<uint32_t>();
        Value v;
        if (type == kString) {
            v.kind = 3;
            v.s = c.str();
        } else if (type == kArray) {
            uint32_t et = c.get<uint32_t>();
            uint64_t n = c.get<uint64_t>();
            v.kind = 4;
            v.n = (size_t)n;
            v.elem = et;
            v.first = c.p;
            if (et == kString) {
                for (uint64_t j = 0; j < n && c.ok; ++j)
                    c.str();
            } else {
                size_t sz = scalar_size(et);
                if (!sz || n > (uint64_t)(c.end - c.p) / sz)
                    return fail("bad GGUF array");
                c.p += sz * n;
            }
        } else {
            size_t sz = scalar_size(type);
            if (!sz || !c.need(sz))
                return fail("bad GGUF metadata value");
            if (type == kF32) {
                v.kind = 2;
                v.f = c.get<float>();
            } else if (type == kF64) {
                v.kind = 2;
                v.f = c.get<double>();
            } else {
                v.kind = 1;
                uint64_t u = 0;
                std::memcpy(&u, c.p, sz);
                c.p += sz;
                if (type == kI8) u = (uint64_t)(int64_t)(int8_t)u;
                if (type == kI16) u = (uint64_t)(int64_t)(int16_t)u;
                if (type == kI32) u = (uint64_t)(int64_t)(int32_t)u;
                v.u = u;
            }
        }
        if (key == "general.alignment" && v.kind == 1)
            alignment = v.u;
        kv_[key] = std::move(v);
    }
    if (!c.ok || alignment == 0 || alignment > 4096)
        return fail("invalid GGUF metadata");
    std::vector<GgufTensor> list;
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        GgufTensor t;
        t.name = c.str();
        uint32_t rank = c.get<uint32_t>();
        if (rank == 0 || rank > 4)
            return fail("bad GGUF tensor rank");
        for (uint32_t d = 0; d < rank; ++d)
            t.dims.push_back(c.get<uint64_t>());
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        list.push_back(std::move(t));
    }
    if (!c.ok)
        return fail("truncated GGUF tensor table");
    const uint64_t info_end = (uint64_t)(c.p - map_);
    const uint64_t data = (info_end + alignment - 1) / alignment * alignment;
    if (data > map_bytes_)
        return fail("GGUF data section out of bounds");
    for (GgufTensor& t : list) {
        uint64_t count = 1;
        for (uint64_t d : t.dims) {
            if (d == 0 || count > UINT64_MAX / d)
                return fail("bad tensor shape " + t.name);
            count *= d;
        }
        if (t.type == 0)
            t.bytes = count * 4;
        else if (t.type == 1)
            t.bytes = count * 2;
        else if (t.type == 41) {
            if (t.dims.size() != 2 || t.dims[0] % 128 != 0)
                return fail("bad Q1_0 tensor " + t.name);
            t.bytes = count / 128 * 18;
        } else {
            return fail("unsupported tensor type in " + t.name);
        }
        if (t.offset > map_bytes_ - data || t.bytes > map_bytes_ - data - t.offset)
            return fail("tensor data out of bounds: " + t.name);
        t.data = map_ + data + t.offset;
        tensors_[t.name] = t;
    }
    return true;
}

bool GgufFile::has(const std::string& key) const { return kv_.count(key) != 0; }

bool GgufFile::get_u64(const std::string& key, uint64_t* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.kind != 1)
        return false;
    *out = it->second.u;
    return true;
}

bool GgufFile::get_f32(const std::string& key, float* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.kind != 2)
        return false;
    *out = (float)it->second.f;
    return true;
}

bool GgufFile::get_str(const std::string& key, std::string* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.kind != 3)
        return false;
    *out = it->second.s;
    return true;
}

size_t GgufFile::array_len(const std::string& key) const {
    auto it = kv_.find(key);
    return it == kv_.end() || it->second.kind != 4 ? 0 : it->second.n;
}

bool GgufFile::get_str_array(const std::string& key, std::vector<std::string_view>* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.kind != 4 || it->second.elem != kString)
        return false;
    // open() walked these elements with bounds checks, so the walk stays inside the map.
    const uint8_t* p = it->second.first;
    out->clear();
    out->reserve(it->second.n);
    for (size_t i = 0; i < it->second.n; ++i) {
        uint64_t len;
        std::memcpy(&len, p, 8);
        out->emplace_back(reinterpret_cast<const char*>(p + 8), (size_t)len);
        p += 8 + len;
    }
    return true;
}

bool GgufFile::get_u32_array(const std::string& key, std::vector<uint32_t>* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.kind != 4 || (it->second.elem != kI32 && it->second.elem != kU32))
        return false;
    out->resize(it->second.n);
    if (it->second.n)
        std::memcpy(out->data(), it->second.first, it->second.n * 4);
    return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace bnn
