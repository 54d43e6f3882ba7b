// Minimal GGUF (v2/v3) reader: metadata key/values and tensor descriptors of a memory-mapped file.
// Stands in for the un-vendored gguf-tools library the reference links
// (thirdparty/gguf-tools/repo.bzl:7; call sites src/models/vkllm_models_llama2.c:185-392).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace vkb
{

enum GgufValueType : uint32_t
{
    GGUF_U8 = 0,
    GGUF_I8 = 1,
    GGUF_U16 = 2,
    GGUF_I16 = 3,
    GGUF_U32 = 4,
    GGUF_I32 = 5,
    GGUF_F32 = 6,
    GGUF_BOOL = 7,
    GGUF_STRING = 8,
    GGUF_ARRAY = 9,
    GGUF_U64 = 10,
    GGUF_I64 = 11,
    GGUF_F64 = 12,
};

enum GgmlType : uint32_t
{
    GGML_F32 = 0,
    GGML_F16 = 1,
};

struct GgufKV
{
    std::string key;
    uint32_t type = 0;
    // Scalars (widened); strings; arrays of strings / numbers.
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    uint32_t arr_type = 0;
    std::vector<std::string> arr_str;
    std::vector<double> arr_num;
};

struct GgufTensor
{
    std::string name;
    uint32_t n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1}; // ne0 first (innermost)
    uint32_t type = 0;
    uint64_t offset = 0; // relative to the data section
    uint64_t bytes = 0;
    const uint8_t *data = nullptr;
};

class GgufFile
{
  public:
    ~GgufFile();
    // Returns an empty string on success, else a description of the problem.
    std::string open(const char *path);
    const std::vector<GgufKV> &kvs() const
    {
        return kvs_;
    }
    const std::vector<GgufTensor> &tensors() const
    {
        return tensors_;
    }
    uint32_t version() const
    {
        return version_;
    }

  private:
    std::vector<GgufKV> kvs_;
    std::vector<GgufTensor> tensors_;
    uint32_t version_ = 0;
    void *map_ = nullptr;
    size_t map_len_ = 0;
};

} // namespace vkb
