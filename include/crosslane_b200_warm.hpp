// The CUDA lane as a crosslane WarmRedirect (engine/strata/warm/runtime.hpp:10-16).
//
// Header-only C++20 adapter over the C ABI in crosslane_b200.h. Build it inside
// crosslane's engine/strata (include path: engine/strata/warm for runtime.hpp, plus this
// directory) and link libcrosslane_b200.so. Registration, in the stage set-up that builds
// the HIP bank today (runtime.cpp:109):
//
//     static strata::wiring::CudaBank cuda(cfg);       // cfg: clb_bank_config_v1
//     cuda.load(layer, expert, role, type, bytes);      // per resident matrix (or
//                                                       // clb_bank_load_strata_pack)
//     strata::wiring::warm_register(&cuda, /*hip slot = lane 1*/ true);
//
// warm_execute (runtime.cpp:121-189) then partitions with warm_contains, calls
// warm_compute_many once per layer for this lane's picks (warm_grouped() is true), joins
// every lane and combines in ascending expert id, unchanged. Every ABI status other than
// CLB_OK becomes a std::runtime_error carrying the library's message, which warm_execute
// rethrows after all lanes have drained (runtime.cpp:167-174); a CUDA failure poisons the
// bank, so later calls fail with CLB_E_STATE (abi_backend_plugin.cpp:27-39's convention).
#pragma once
#include <cstddef>
#include <cstdint>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#include "crosslane_b200.h"
#include "runtime.hpp"

namespace strata::wiring {

class CudaBank final : public WarmRedirect {
public:
    explicit CudaBank(const clb_bank_config_v1& cfg) : dim_(cfg.dim) {
        clb_error_v1 e{};
        check(clb_bank_create(&cfg, &bank_, &e), e);
    }
    CudaBank(const CudaBank&) = delete;
    CudaBank& operator=(const CudaBank&) = delete;
    ~CudaBank() override { clb_bank_destroy(bank_); }

    // One resident matrix from its ggml bytes (WeightSource::read_all of
    // layers.L.ffn.experts.E.{w1,w3,w2}.weight): role 0 = w1 (gate), 1 = w3 (up),
    // 2 = w2 (down); type = the ggml id 16 (IQ2_XXS), 17 (IQ2_XS) or 29 (IQ1_M).
    void load(uint32_t layer, int expert, int role, int type, std::span<const std::byte> bytes) {
        clb_error_v1 e{};
        check(clb_bank_load_matrix(bank_, layer, expert, role, type, bytes.data(), bytes.size(), &e), e);
    }

    // The frozen warm placement (STRATA_WARM_PLACEMENT_V1 text): this bank then holds the
    // experts whose row names lane_id; apply before any load.
    void apply_placement(const std::string& text, int32_t lane_id) {
        int32_t nl = 0, ne = 0, dim = 0, ff = 0;
        check_geometry(nl, ne, dim, ff);
        std::vector<int32_t> lanes((size_t)nl * (size_t)ne);
        clb_error_v1 e{};
        check(clb_placement_parse(text.data(), text.size(), nl, ne, lanes.data(), nullptr, &e), e);
        check(clb_bank_apply_placement(bank_, lanes.data(), lane_id, &e), e);
    }

    bool warm_grouped() const override { return true; }
    bool warm_contains(uint32_t layer, int expert) const override {
        return clb_bank_contains(bank_, layer, expert) != 0;
    }
    std::vector<float> warm_compute(uint32_t layer, int expert, std::span<const float> x) override {
        require_dim(x.size());
        std::vector<float> y((size_t)dim_);
        clb_error_v1 e{};
        check(clb_bank_compute(bank_, layer, expert, x.data(), y.data(), &e), e);
        return y;
    }
    std::vector<std::vector<float>> warm_compute_many(uint32_t layer, std::span<const int> ids,
                                                      std::span<const float> x) override {
        require_dim(x.size());
        std::vector<float> flat(ids.size() * (size_t)dim_);
        clb_error_v1 e{};
        check(clb_bank_compute_many(bank_, layer, ids.data(), (int32_t)ids.size(), x.data(), flat.data(), &e), e);
        std::vector<std::vector<float>> rows;
        rows.reserve(ids.size());
        for (size_t i = 0; i < ids.size(); ++i)
            rows.emplace_back(flat.begin() + (std::ptrdiff_t)(i * (size_t)dim_),
                              flat.begin() + (std::ptrdiff_t)((i + 1) * (size_t)dim_));
        return rows;
    }

    clb_bank* handle() const { return bank_; }

private:
    static void check(int32_t rc, const clb_error_v1& e) {
        if (rc != CLB_OK) throw std::runtime_error(std::string("crosslane_b200: ") + e.message);
    }
    void check_geometry(int32_t& nl, int32_t& ne, int32_t& dim, int32_t& ff) const {
        if (clb_bank_geometry(bank_, &nl, &ne, &dim, &ff) != CLB_OK)
            throw std::runtime_error("crosslane_b200: bank geometry unavailable");
    }
    void require_dim(size_t n) const {
        if (n != (size_t)dim_) throw std::runtime_error("crosslane_b200: x has the wrong length");
    }
    clb_bank* bank_ = nullptr;
    int dim_;
};

}  // namespace strata::wiring
