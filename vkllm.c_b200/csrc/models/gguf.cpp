// GGUF v2/v3 reader over mmap. Format (little endian): "GGUF", u32 version, u64 n_tensors,
// u64 n_kv, then n_kv {string key, u32 type, value}, then n_tensors {string name, u32 n_dims,
// u64 dims[n_dims], u32 ggml_type, u64 offset}, then the data section aligned to
// general.alignment (default 32). Strings are u64 length + bytes.
#include "gguf.h"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace vkb
{

namespace
{

struct Cursor
{
    const uint8_t *p, *end;
    bool ok = true;
    template <typename T> T get()
    {
        T v{};
        if (p + sizeof(T) > end)
        {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str()
    {
        uint64_t n = get<uint64_t>();
        if (!ok || n > (uint64_t)(end - p))
        {
            ok = false;
            return std::string();
        }
        std::string s((const char *)p, (size_t)n);
        p += n;
        return s;
    }
};

// Bytes of one scalar of a GGUF value type (0 for strings, arrays and unknown types).
uint64_t scalar_size(uint32_t type)
{
    switch (type)
    {
    case GGUF_U8:
    case GGUF_I8:
    case GGUF_BOOL:
        return 1;
    case GGUF_U16:
    case GGUF_I16:
        return 2;
    case GGUF_U32:
    case GGUF_I32:
    case GGUF_F32:
        return 4;
    case GGUF_U64:
    case GGUF_I64:
    case GGUF_F64:
        return 8;
    default:
        return 0;
    }
}

bool read_scalar(Cursor &c, uint32_t type, GgufKV &kv)
{
    switch (type)
    {
    case GGUF_U8:
        kv.u = c.get<uint8_t>();
        kv.i = (int64_t)kv.u;
        kv.f = (double)kv.u;
        break;
    case GGUF_I8:
        kv.i = c.get<int8_t>();
        kv.u = (uint64_t)kv.i;
        kv.f = (double)kv.i;
        break;
    case GGUF_U16:
        kv.u = c.get<uint16_t>();
        kv.i = (int64_t)kv.u;
        kv.f = (double)kv.u;
        break;
    case GGUF_I16:
        kv.i = c.get<int16_t>();
        kv.u = (uint64_t)kv.i;
        kv.f = (double)kv.i;
        break;
    case GGUF_U32:
        kv.u = c.get<uint32_t>();
        kv.i = (int64_t)kv.u;
        kv.f = (double)kv.u;
        break;
    case GGUF_I32:
        kv.i = c.get<int32_t>();
        kv.u = (uint64_t)kv.i;
        kv.f = (double)kv.i;
        break;
    case GGUF_F32:
        kv.f = c.get<float>();
        break;
    case GGUF_BOOL:
        kv.u = c.get<uint8_t>() ? 1 : 0;
        kv.i = (int64_t)kv.u;
        break;
    case GGUF_STRING:
        kv.s = c.str();
        break;
    case GGUF_U64:
        kv.u = c.get<uint64_t>();
        kv.i = (int64_t)kv.u;
        kv.f = (double)kv.u;
        break;
    case GGUF_I64:
        kv.i = c.get<int64_t>();
        kv.u = (uint64_t)kv.i;
        kv.f = (double)kv.i;
        break;
    case GGUF_F64:
        kv.f = c.get<double>();
        break;
    default:
        return false;
    }
    return c.ok;
}

} // namespace

GgufFile::~GgufFile()
{
    if (map_)
        munmap(map_, map_len_);
}

std::string GgufFile::open(const char *path)
{
    int fd = ::open(path, O_RDONLY);
    if (fd < 0)
        return std::string("cannot open ") + path;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24)
    {
        ::close(fd);
        return "file too small for a GGUF header";
    }
    map_len_ = (size_t)st.st_size;
    map_ = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED)
    {
        map_ = nullptr;
        return "mmap failed";
    }
    const uint8_t *base = (const uint8_t *)map_;
    Cursor c{base, base + map_len_};
    if (memcmp(base, "GGUF", 4) != 0)
        return "bad magic (not a GGUF file)";
    c.p += 4;
    version_ = c.get<uint32_t>();
    if (version_ < 2 || version_ > 3)
        return "unsupported GGUF version " + std::to_string(version_);
    uint64_t n_tensors = c.get<uint64_t>();
    uint64_t n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24))
        return "corrupt GGUF header counts";
    uint64_t alignment = 32;
    for (uint64_t k = 0; k < n_kv; ++k)
    {
        GgufKV kv;
        kv.key = c.str();
        kv.type = c.get<uint32_t>();
        if (!c.ok)
            return "truncated metadata";
        if (kv.type == GGUF_ARRAY)
        {
            kv.arr_type = c.get<uint32_t>();
            uint64_t n = c.get<uint64_t>();
            // every element takes at least its scalar size (a string: its 8-byte length) of the
            // bytes left, which bounds what is reserved below
            const uint64_t left = (uint64_t)(c.end - c.p);
            const uint64_t esz = kv.arr_type == GGUF_STRING ? 8 : scalar_size(kv.arr_type);
            if (!c.ok || (esz > 0 && n > left / esz))
                return "corrupt array in metadata key " + kv.key;
            if (kv.arr_type == GGUF_STRING)
            {
                kv.arr_str.reserve((size_t)n);
                for (uint64_t j = 0; j < n && c.ok; ++j)
                    kv.arr_str.push_back(c.str());
            }
            else if (kv.arr_type == GGUF_ARRAY)
                return "nested arrays are not supported (key " + kv.key + ")";
            else
            {
                kv.arr_num.reserve((size_t)n);
                for (uint64_t j = 0; j < n && c.ok; ++j)
                {
                    GgufKV e;
                    if (!read_scalar(c, kv.arr_type, e))
                        return "corrupt array element in key " + kv.key;
                    kv.arr_num.push_back(kv.arr_type == GGUF_F32 || kv.arr_type == GGUF_F64 ? e.f : (double)e.i);
                }
            }
            if (!c.ok)
                return "truncated array in key " + kv.key;
        }
        else if (!read_scalar(c, kv.type, kv))
            return "corrupt value of metadata key " + kv.key;
        if (kv.key == "general.alignment" && kv.u > 0)
        {
            if (kv.u > (1u << 20) || kv.u % 8 != 0) // the format asks for a multiple of 8
                return "unsupported general.alignment " + std::to_string(kv.u);
            alignment = kv.u;
        }
        kvs_.push_back(std::move(kv));
    }
    for (uint64_t t = 0; t < n_tensors; ++t)
    {
        GgufTensor ti;
        ti.name = c.str();
        ti.n_dims = c.get<uint32_t>();
        if (!c.ok || ti.n_dims > 4)
            return "corrupt tensor descriptor";
        for (uint32_t d = 0; d < ti.n_dims; ++d)
            ti.dims[d] = c.get<uint64_t>();
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        if (!c.ok)
            return "truncated tensor descriptors";
        uint64_t n = 1;
        for (uint32_t d = 0; d < 4; ++d)
            if (ti.dims[d] > 0xffffffffull || __builtin_mul_overflow(n, ti.dims[d], &n))
                return "corrupt dimensions of tensor " + ti.name;
        if ((ti.type == GGML_F32 || ti.type == GGML_F16) && n > map_len_) // cannot fit in the file
            return "tensor " + ti.name + " is larger than the file";
        if (ti.type == GGML_F32)
            ti.bytes = n * 4;
        else if (ti.type == GGML_F16)
            ti.bytes = n * 2;
        else
            ti.bytes = 0; // quantised types are not supported by this path
        tensors_.push_back(ti);
    }
    uint64_t header = (uint64_t)(c.p - base);
    uint64_t data_start = (header + alignment - 1) / alignment * alignment;
    for (auto &ti : tensors_)
    {
        if (ti.bytes == 0)
            continue;
        if (data_start > map_len_ || ti.offset > map_len_ - data_start || ti.bytes > map_len_ - data_start - ti.offset)
            return "tensor " + ti.name + " extends past the end of the file";
        ti.data = base + data_start + ti.offset;
    }
    return std::string();
}

} // namespace vkb
