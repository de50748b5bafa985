// TEST INFRASTRUCTURE ONLY -- the timed CPU expert lane of bench.py (never on the CUDA
// path): crosslane's CPU-lane arithmetic, engine/strata/sycl/stage/wiring/q8k_core.hpp
// (itself a restatement of ggml's x86 AVX2 Q8_K IQ dots), vectorised with AVX2 the way
// ggml vectorises it, and batched like the reference lane's layer batch.
//
// Bit-identity with q8k_core.hpp (pinned in tests/test_oracle_pin.py against the compiled
// reference and against oracle.c): the reference keeps 8 accumulation lanes per row; lane L
// holds positions 4L..4L+3 of every 32-value chunk (q8k_core.hpp:41-69). One AVX2 register
// of 8 int32 is exactly those lanes: maddubs/sign give byte products, madd_epi16 adds
// adjacent pairs times the chunk's sub-scale (positions 4L..4L+3 land in int32 lane L), and
// per block the 8 float lanes take one fused multiply-add with d = half(w.d) * a.d in block
// order (q8k_core.hpp:76-85), then the fixed pairwise hsum (q8k_core.hpp:86-91). The
// integers are exact in any order; the float operations are the reference's, lane by lane.
//
// Batching (engine/strata/sycl/moe/cpu_lane.cpp:177-251, Lane::experts): Q8_K(x) is formed
// once per layer, each phase first runs every expert's rows [0, 64) on the calling thread,
// then the remaining 64-row jobs of all experts are interleaved (job j -> expert j % n)
// over a persistent team of threads pulling jobs from a counter
// (engine/strata/sycl/moe/row_team.hpp:35-44, 90-111); SwiGLU is applied per row inside
// the gate/up job, Q8_K(h) per expert between the phases.
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "../crosslane_b200/csrc/iq_tables.h"

namespace {

struct Q8K {  // crosslane's q8k::Block (q8k_core.hpp:13-14)
    float d;
    int8_t qs[256];
    int16_t bsums[16];
};
static_assert(sizeof(Q8K) == 292, "Q8_K block");

uint64_t g_sign8[128];  // ksigns (7 sign bits + parity) -> 8 bytes of +1 / -1
std::once_flag g_tables_once;
void init_tables() {
    for (int s = 0; s < 128; ++s) {
        const unsigned v = (unsigned)s | ((unsigned)__builtin_parity((unsigned)s) << 7);
        uint64_t m = 0;
        for (int j = 0; j < 8; ++j) m |= (uint64_t)((v >> j) & 1u ? 0xFFu : 0x01u) << (8 * j);
        g_sign8[s] = m;
    }
}

inline uint16_t u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
inline uint32_t u32(const uint8_t* p) { return (uint32_t)u16(p) | ((uint32_t)u16(p + 2) << 16); }

// fp16 bits -> float, exactly (every finite half is a binary32 value).
inline float half_to_float(uint16_t h) {
    const int e = (h >> 10) & 31;
    float v;
    if (!e) v = ldexpf((float)(h & 1023), -24);
    else if (e == 31) v = (h & 1023) ? NAN : INFINITY;
    else v = ldexpf((float)(1024 + (h & 1023)), e - 25);
    return (h & 32768) ? -v : v;
}

inline int nearest(float x) {
    float v = x + 12582912.0f;
    uint32_t u;
    std::memcpy(&u, &v, 4);
    return (int)(u & 0x007fffffu) - 0x00400000;
}

// q8k_core.hpp:30-38.
void quant_block(const float* x, Q8K& y) {
    float mx = 0, am = 0;
    for (int j = 0; j < 256; ++j) {
        const float a = fabsf(x[j]);
        if (a > am) {
            am = a;
            mx = x[j];
        }
    }
    if (am == 0) {
        std::memset(&y, 0, sizeof y);
        return;
    }
    const float is = -127.0f / mx;
    for (int j = 0; j < 256; ++j) {
        const int v = nearest(is * x[j]);
        y.qs[j] = (int8_t)(v < 127 ? v : 127);
    }
    for (int j = 0; j < 16; ++j) {
        int s = 0;
        for (int z = 0; z < 16; ++z) s += y.qs[16 * j + z];
        y.bsums[j] = (int16_t)s;
    }
    y.d = 1.0f / is;
}

inline int block_bytes(int t) { return t == 29 ? 56 : t == 17 ? 74 : 66; }

inline float block_scale(int t, const uint8_t* w) {
    if (t != 29) return half_to_float(u16(w));
    const uint16_t h = (uint16_t)((u16(w + 48) >> 12) | ((u16(w + 50) >> 8) & 0xf0) | ((u16(w + 52) >> 4) & 0xf00) |
                                  (u16(w + 54) & 0xf000));
    return half_to_float(h);
}

inline __m256i grid4(uint64_t a, uint64_t b, uint64_t c, uint64_t d) {
    return _mm256_set_epi64x((long long)d, (long long)c, (long long)b, (long long)a);
}

// Lane integers of one block: main[L] (and delta[L] for IQ1_M), L = 0..7.
template <int T>
inline void block_lanes(const uint8_t* w, const int8_t* q, __m256i& main, __m256i& delta) {
    main = _mm256_setzero_si256();
    delta = _mm256_setzero_si256();
    const __m256i ones8 = _mm256_set1_epi8(1);
    for (int c = 0; c < 8; ++c) {
        const __m256i qv = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(q + 32 * c));
        if (T == 16) {
            const uint8_t* chunk = w + 2 + 8 * c;
            const uint32_t hi = u32(chunk + 4);
            const __m256i mag = grid4(clb_iq2xxs_grid[chunk[0]], clb_iq2xxs_grid[chunk[1]], clb_iq2xxs_grid[chunk[2]],
                                      clb_iq2xxs_grid[chunk[3]]);
            const __m256i sgn = grid4(g_sign8[hi & 127], g_sign8[(hi >> 7) & 127], g_sign8[(hi >> 14) & 127],
                                      g_sign8[(hi >> 21) & 127]);
            const __m256i p16 = _mm256_maddubs_epi16(mag, _mm256_sign_epi8(qv, sgn));
            main = _mm256_add_epi32(main, _mm256_madd_epi16(p16, _mm256_set1_epi16((short)(2 * (hi >> 28) + 1))));
        } else if (T == 17) {
            const uint8_t* chunk = w + 2 + 8 * c;
            const uint16_t c0 = u16(chunk), c1 = u16(chunk + 2), c2 = u16(chunk + 4), c3 = u16(chunk + 6);
            const __m256i mag = grid4(clb_iq2xs_grid[c0 & 511], clb_iq2xs_grid[c1 & 511], clb_iq2xs_grid[c2 & 511],
                                      clb_iq2xs_grid[c3 & 511]);
            const __m256i sgn = grid4(g_sign8[c0 >> 9], g_sign8[c1 >> 9], g_sign8[c2 >> 9], g_sign8[c3 >> 9]);
            const uint8_t sb = w[66 + c];
            const __m256i sc = _mm256_set_m128i(_mm_set1_epi16((short)(2 * (sb >> 4) + 1)),
                                                _mm_set1_epi16((short)(2 * (sb & 15) + 1)));
            const __m256i p16 = _mm256_maddubs_epi16(mag, _mm256_sign_epi8(qv, sgn));
            main = _mm256_add_epi32(main, _mm256_madd_epi16(p16, sc));
        } else {
            const uint8_t h0 = w[32 + 2 * c], h1 = w[33 + 2 * c];
            const int g0 = w[4 * c] | ((h0 << 8) & 0x700), g1 = w[4 * c + 1] | ((h0 << 4) & 0x700);
            const int g2 = w[4 * c + 2] | ((h1 << 8) & 0x700), g3 = w[4 * c + 3] | ((h1 << 4) & 0x700);
            const __m256i code = grid4(clb_iq1s_grid[g0], clb_iq1s_grid[g1], clb_iq1s_grid[g2], clb_iq1s_grid[g3]);
            const uint16_t sw = u16(w + 48 + 2 * (c / 2));
            const int sh = 6 * (c % 2);
            const __m256i sc = _mm256_set_m128i(_mm_set1_epi16((short)(2 * ((sw >> (sh + 3)) & 7) + 1)),
                                                _mm_set1_epi16((short)(2 * ((sw >> sh) & 7) + 1)));
            // delta sign per 8-value group: bit 3 (even group) / bit 7 (odd group) of its qh byte
            const uint64_t m0 = (h0 & 8) ? 0xFFFFFFFFFFFFFFFFull : 0x0101010101010101ull;
            const uint64_t m1 = (h0 & 128) ? 0xFFFFFFFFFFFFFFFFull : 0x0101010101010101ull;
            const uint64_t m2 = (h1 & 8) ? 0xFFFFFFFFFFFFFFFFull : 0x0101010101010101ull;
            const uint64_t m3 = (h1 & 128) ? 0xFFFFFFFFFFFFFFFFull : 0x0101010101010101ull;
            const __m256i dsg = grid4(m0, m1, m2, m3);
            const __m256i pm = _mm256_maddubs_epi16(ones8, _mm256_sign_epi8(qv, code));
            const __m256i pd = _mm256_maddubs_epi16(ones8, _mm256_sign_epi8(qv, dsg));
            main = _mm256_add_epi32(main, _mm256_madd_epi16(pm, sc));
            delta = _mm256_add_epi32(delta, _mm256_madd_epi16(pd, sc));
        }
    }
}

inline float hsum8(__m256 v) {  // q8k_core.hpp:86: ((v0+v4)+(v2+v6))+((v1+v5)+(v3+v7))
    alignas(32) float m[8];
    _mm256_store_ps(m, v);
    return ((m[0] + m[4]) + (m[2] + m[6])) + ((m[1] + m[5]) + (m[3] + m[7]));
}

// q8k_core.hpp:87-91, one row.
template <int T>
float row_dot(const uint8_t* w, const Q8K* a, int nb) {
    __m256 sm = _mm256_setzero_ps(), sd = _mm256_setzero_ps();
    for (int b = 0; b < nb; ++b) {
        const uint8_t* p = w + (size_t)b * block_bytes(T);
        __m256i im, id;
        block_lanes<T>(p, a[b].qs, im, id);
        const __m256 d = _mm256_set1_ps(block_scale(T, p) * a[b].d);
        sm = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(im), sm);
        if (T == 29) sd = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(id), sd);
    }
    const float main = hsum8(sm);
    return T == 29 ? main + 0.125f * hsum8(sd) : 0.125f * main;
}

float dot(int t, const uint8_t* w, const Q8K* a, int nb) {
    if (t == 16) return row_dot<16>(w, a, nb);
    if (t == 17) return row_dot<17>(w, a, nb);
    return row_dot<29>(w, a, nb);
}

// q8k_core.hpp:92-95.
inline float swiglu(float g, float u, float limit) {
    if (limit > 0) {
        g = fminf(g, limit);
        u = fminf(fmaxf(u, -limit), limit);
    }
    return (g / (1.0f + expf(-g))) * u;
}

// Persistent team: the caller and N-1 workers pull jobs from a counter.
class Team {
    std::vector<std::thread> threads_;
    std::mutex m_;
    std::condition_variable cv_, done_;
    std::function<void(int)> fn_;
    int jobs_ = 0, generation_ = 0, busy_ = 0;
    std::atomic<int> next_{0};
    bool stop_ = false;
    void drain() {
        for (int j; (j = next_.fetch_add(1)) < jobs_;) fn_(j);
    }

public:
    explicit Team(int n) {
        for (int i = 1; i < n; ++i)
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
                    if (--busy_ == 0) done_.notify_all();
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
    int size() const { return (int)threads_.size() + 1; }
    void run(int jobs, std::function<void(int)> fn) {
        if (jobs <= 0) return;
        {
            std::lock_guard<std::mutex> l(m_);
            fn_ = std::move(fn);
            jobs_ = jobs;
            next_ = 0;
            ++generation_;
        }
        cv_.notify_all();
        drain();
        std::unique_lock<std::mutex> l(m_);
        done_.wait(l, [&] { return busy_ == 0 && next_.load() >= jobs_; });
    }
};
std::mutex g_team_mutex;
Team* g_team = nullptr;
Team& team(int threads) {
    if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
    if (!g_team || g_team->size() != threads) {
        delete g_team;
        g_team = new Team(threads);
    }
    return *g_team;
}

}  // namespace

extern "C" {

// One row: y = dot(w_row, Q8_K(x)) (q8k_core.hpp::dot); q: nb crosslane Q8_K blocks.
float lane_dot(int t, const uint8_t* w, const void* q, int nb) {
    std::call_once(g_tables_once, init_tables);
    return dot(t, w, static_cast<const Q8K*>(q), nb);
}

void lane_quantize(const float* x, int k, void* q) {
    for (int b = 0; b < k / 256; ++b) quant_block(x + 256 * b, static_cast<Q8K*>(q)[b]);
}

// n experts of one token-layer (Lane::experts): types[i], the ggml AoS matrices gate[i] /
// up[i] [ff][dim] and down[i] [dim][ff]; x [dim]; y [n][dim]. threads <= 0: every host
// thread. Returns the team size used.
int lane_experts(int n, const int* types, const uint8_t* const* gate, const uint8_t* const* up,
                 const uint8_t* const* down, const float* x, int dim, int ff, float limit, int threads, float* y) {
    std::call_once(g_tables_once, init_tables);
    std::lock_guard<std::mutex> lock(g_team_mutex);
    Team& tm = team(threads);
    const int nbx = dim / 256, nbh = ff / 256;
    std::vector<Q8K> qx((size_t)nbx), qh((size_t)n * nbh);
    std::vector<float> h((size_t)n * ff);
    lane_quantize(x, dim, qx.data());
    // a phase: rows [0, 64) of every expert on this thread, then 64-row jobs of all
    // experts interleaved over the team
    auto phase = [&](int rows, const std::function<void(int, int, int)>& fn) {
        for (int i = 0; i < n; ++i) fn(i, 0, std::min(rows, 64));
        const int chunks = (rows - 1) / 64;
        tm.run(chunks * n, [&](int task) {
            const int i = task % n, lo = (1 + task / n) * 64;
            fn(i, lo, std::min(rows, lo + 64));
        });
    };
    phase(ff, [&](int i, int lo, int hi) {
        const size_t row = (size_t)nbx * block_bytes(types[i]);
        for (int r = lo; r < hi; ++r) {
            const float g = dot(types[i], gate[i] + (size_t)r * row, qx.data(), nbx);
            const float u = dot(types[i], up[i] + (size_t)r * row, qx.data(), nbx);
            h[(size_t)i * ff + r] = swiglu(g, u, limit);
        }
    });
    for (int i = 0; i < n; ++i) lane_quantize(h.data() + (size_t)i * ff, ff, qh.data() + (size_t)i * nbh);
    phase(dim, [&](int i, int lo, int hi) {
        const size_t row = (size_t)nbh * block_bytes(types[i]);
        for (int r = lo; r < hi; ++r)
            y[(size_t)i * dim + r] = dot(types[i], down[i] + (size_t)r * row, qh.data() + (size_t)i * nbh, nbh);
    });
    return tm.size();
}

int lane_team_threads(int threads) {
    std::lock_guard<std::mutex> lock(g_team_mutex);
    return team(threads).size();
}
}
