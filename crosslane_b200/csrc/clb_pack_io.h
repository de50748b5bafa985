// Strata pack reader shared by the C ABI (clb_pack_io.cu) and the bank's loader
// (clb_bank.cu). A pack is crosslane's index over the model's GGUF shards
// (engine/strata/sycl/stage/wiring/weight_source.hpp:1-5, pack_source.cpp:144-185):
//   <pack>/ds4.txt      "key value" lines (model_dir, format, geometry)
//   <pack>/tensors.txt  "file <i> <shard>" and "t <name> <dtype> <file> <offset> <bytes> <shape...>"
// Tensor bytes are read exactly as stored (POSIX pread); no conversion happens here.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

struct clb_strata_pack;

namespace clb {

struct PackTensor {
    std::string dtype;           // as tensors.txt spells it: "IQ2_XXS", "F32", ...
    int file = -1;
    uint64_t offset = 0, bytes = 0;
    std::vector<int64_t> shape;  // tensors.txt order: shape[0] = rows (out), shape[1] = cols (in)
};

const PackTensor* pack_find(const clb_strata_pack* p, const std::string& name);
std::string pack_meta(const clb_strata_pack* p, const std::string& key);  // "" when absent
void pack_read(const clb_strata_pack* p, const PackTensor& t, uint64_t offset, void* dst, uint64_t bytes);  // throws
// ggml type id of an admitted expert dtype (16 IQ2_XXS, 17 IQ2_XS, 29 IQ1_M), else 0.
int pack_expert_type(const std::string& dtype);

}  // namespace clb
