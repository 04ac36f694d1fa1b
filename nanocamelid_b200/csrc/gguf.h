// GGUF reader / synthetic writer (host).  gguf.rs:454-551 read_file semantics:
// v2/v3 header, metadata, tensor table, data start aligned to general.alignment (32).
#pragma once
#include <stdint.h>
#include <string>
#include <vector>
#include "../../include/ncm.h"

namespace ncm {

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;   // dims[0] = columns (fastest), dims[1] = rows
    int type = 0;
    uint64_t offset = 0;          // relative to data_start
    uint64_t nbytes = 0;
};

struct GgufFile {
    const uint8_t* map = nullptr;
    size_t size = 0;
    uint64_t alignment = 32, data_start = 0;
    std::string arch;
    int ctx = 0, emb = 0, layers = 0, ffn = 0, heads = 0, kv_heads = 0, vocab = 0, head_dim = 0, rope_dim = 0;
    float rope_base = 10000.0f, eps = 1e-5f;
    std::vector<GgufTensor> tensors;
    bool open(const char* path, std::string& err);
    const GgufTensor* find(const std::string& name) const;
    const uint8_t* data(const GgufTensor& t) const { return map + data_start + t.offset; }
    ~GgufFile();
};

struct SynthTensor {
    std::string name;
    int type;
    int64_t rows, cols;
    bool ones;   // norm weights: F32 ones
};
std::vector<SynthTensor> synth_tensor_list(const ncm_synth_spec& s);

}  // namespace ncm
