// TEST INFRASTRUCTURE ONLY -- C-ABI driver around crosslane's OWN CPU arithmetic.
//
// Compiled by oracle/Makefile against the crosslane sources where they lie (never
// copied into this repository) into oracle/_ref/libref.so:
//   engine/strata/sycl/stage/wiring/q8k_core.hpp  Q8_K quant, lane dots, SwiGLU
//   engine/strata/sycl/moe/core.hpp               per-32 decoder
//   engine/strata/warm/other_combine.hpp          fixed-order combine
//   engine/strata/sycl/route/route.cpp            route_cpu (mode B)
// Used (a) to pin the C oracle (oracle.c) bit-for-bit, (b) to produce the committed
// golden vectors, and (c) as bench.py's timed reference CPU lane: the reference's
// q8k::dot per row, on a persistent team of host threads taking 64-row jobs like
// engine/strata/sycl/moe/row_team.hpp:35-44.
#include <array>
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <span>
#include <thread>
#include <vector>

#include "sycl/stage/wiring/q8k_core.hpp"
#include "sycl/moe/core.hpp"
#include "warm/other_combine.hpp"
#include "sycl/route/route.hpp"

#include "../crosslane_b200/csrc/synth.h"

namespace q8k = strata::wiring::q8k;
namespace moe = strata::ds4::moe;

namespace {
// Persistent row team: the owner and N-1 workers pull 64-row jobs from a counter.
class Team {
    std::vector<std::thread> threads_;
    std::mutex m_;
    std::condition_variable cv_, done_cv_;
    std::function<void(int, int)> fn_;
    int n_ = 0, jobs_ = 0, generation_ = 0, busy_ = 0;
    std::atomic<int> next_{0};
    bool stop_ = false;
    void drain() {
        for (int j; (j = next_.fetch_add(1)) < jobs_;) fn_(j * 64, std::min(n_, (j + 1) * 64));
    }

public:
    explicit Team(int threads) {
        for (int i = 1; i < threads; ++i)
            threads_.emplace_back([this] {
                int seen = 0;
                for (;;) {
                    {
                        std::unique_lock<std::mutex> l(m_);
                        cv_.wait(l, [&] { return stop_ || generation_ != seen; });
                        if (stop_) return;
                        seen = generation_;
                        ++busy_;
                    }
                    drain();
                    std::lock_guard<std::mutex> l(m_);
                    if (--busy_ == 0) done_cv_.notify_all();
                }
            });
    }
    ~Team() {
        {
            std::lock_guard<std::mutex> l(m_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    int size() const { return int(threads_.size()) + 1; }
    void rows(int n, std::function<void(int, int)> fn) {
        {
            std::lock_guard<std::mutex> l(m_);
            fn_ = std::move(fn);
            n_ = n;
            jobs_ = (n + 63) / 64;
            next_ = 0;
            ++generation_;
        }
        cv_.notify_all();
        drain();
        std::unique_lock<std::mutex> l(m_);
        done_cv_.wait(l, [&] { return busy_ == 0 && next_.load() >= jobs_; });
    }
};
Team* team = nullptr;
int team_threads = 0;
Team& get_team(int threads) {
    if (threads <= 0) threads = int(std::max(1u, std::thread::hardware_concurrency()));
    if (!team || team_threads != threads) {
        delete team;
        team = new Team(threads);
        team_threads = threads;
    }
    return *team;
}

void quantize(const float* x, int k, q8k::Block* out) {
    for (int b = 0; b < k / 256; ++b) q8k::quant_block(x + 256 * b, out[b]);
}

void mv(int t, const uint8_t* w, const q8k::Block* q, float* y, int n, int k, Team& tm) {
    const int nb = k / 256;
    const size_t row = size_t(nb) * size_t(q8k::block_bytes(t));
    tm.rows(n, [&](int lo, int hi) {
        for (int r = lo; r < hi; ++r) y[r] = q8k::dot(t, w + size_t(r) * row, q, nb);
    });
}
}  // namespace

extern "C" {
int ref_block_bytes(int t) { return q8k::block_bytes(t); }
void ref_quant_block(const float* x, void* y) { q8k::quant_block(x, *static_cast<q8k::Block*>(y)); }
float ref_dot(int t, const uint8_t* w, const void* a, int nb) {
    return q8k::dot(t, w, static_cast<const q8k::Block*>(a), nb);
}
void ref_integer_lane(int t, const uint8_t* w, const void* a, int lane, int* main, int* delta) {
    const auto v = q8k::integer_lane(t, w, *static_cast<const q8k::Block*>(a), lane);
    *main = v.main;
    *delta = v.delta;
}
float ref_swiglu(float g, float u, float lim) { return q8k::swiglu(g, u, lim); }
int ref_ksigns(int i) { return q8k::ksigns_iq2xs[i & 127]; }
uint64_t ref_grid(int t, int i) {
    return t == 29 ? q8k::iq1s_grid[i & 2047] : t == 17 ? q8k::iq2xs_grid[i & 511] : q8k::iq2xxs_grid[i & 255];
}
float ref_half(uint16_t h) { return q8k::half(h); }

void ref_decode_sub(int t, const uint8_t* block, int ib, int* q, float* d, int* s) {
    const auto type = t == 16 ? moe::Type::iq2_xxs : t == 17 ? moe::Type::iq2_xs : moe::Type::iq1_m;
    const auto sub = moe::decode(type, block, ib);
    for (int j = 0; j < 32; ++j) q[j] = sub.q[j];
    *d = sub.d;
    s[0] = sub.s[0];
    s[1] = sub.s[1];
}

int ref_combine(const int* ids, const float* w, int n, const float* rows, const float* shared, int dim,
                float* out) {
    using Results = std::array<std::vector<std::pair<size_t, std::vector<float>>>, 3>;
    Results results;
    for (int i = 0; i < n; ++i)
        results[size_t(i) % 3].emplace_back(size_t(i), std::vector<float>(rows + size_t(i) * dim, rows + size_t(i + 1) * dim));
    std::vector<float> zero(size_t(dim), 0.0f);
    const auto o = strata::wiring::other_combine(std::span<const int>(ids, size_t(n)), std::span<const float>(w, size_t(n)),
                                                 std::span<const float>(shared ? shared : zero.data(), size_t(dim)),
                                                 results, strata::wiring::OtherOptions{false});
    std::memcpy(out, o.data(), sizeof(float) * size_t(dim));
    return 0;
}

int ref_route_cpu(const float* logits, const float* bias, int n, int k, float scale, int* ids, float* w) {
    try {
        const auto r = strata::ds4::route_port::route_cpu(std::span<const float>(logits, size_t(n)), size_t(n),
                                                          std::span<const float>(bias, size_t(n)), 1, size_t(k), scale);
        for (int i = 0; i < k; ++i) {
            ids[i] = r.ids[size_t(i)];
            w[i] = r.weights[size_t(i)];
        }
        return 0;
    } catch (...) {
        return -1;
    }
}

// One expert through the reference arithmetic, rows on the team.
int ref_expert(int t, const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x, int dim,
               int ff, float lim, int threads, float* h_out, float* y) {
    Team& tm = get_team(threads);
    std::vector<q8k::Block> qx(static_cast<size_t>(dim / 256)), qh(static_cast<size_t>(ff / 256));
    std::vector<float> g(static_cast<size_t>(ff)), u(static_cast<size_t>(ff)), h(static_cast<size_t>(ff));
    quantize(x, dim, qx.data());
    mv(t, gate, qx.data(), g.data(), ff, dim, tm);
    mv(t, up, qx.data(), u.data(), ff, dim, tm);
    for (int i = 0; i < ff; ++i) h[size_t(i)] = q8k::swiglu(g[size_t(i)], u[size_t(i)], lim);
    quantize(h.data(), ff, qh.data());
    mv(t, down, qh.data(), y, dim, ff, tm);
    if (h_out) std::memcpy(h_out, h.data(), sizeof(float) * size_t(ff));
    return 0;
}

int ref_team_threads(int threads) { return get_team(threads).size(); }
}
