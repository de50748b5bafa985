// Host side of the CUDA expert lane: bank, workspace, launches and the C ABI
// declared in include/crosslane_b200.h.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cctype>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/crosslane_b200.h"
#include "clb_host.h"
#include "clb_kernels.h"
#include "clb_pack_io.h"
#include "clb_pack.h"
#include "scale_table.h"

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

std::once_flag g_scale_once;
uint16_t g_scale_host[65536];

// Per-device one-time state: nibble tables uploaded and kernel attributes set.
std::mutex g_dev_mutex;
std::set<int> g_dev_ready;
void ensure_device_ready(int dev, cudaStream_t s) {
    std::lock_guard<std::mutex> l(g_dev_mutex);
    if (g_dev_ready.count(dev)) return;
    cuda_check(clb::upload_tables(s), "upload codebook tables");
    cuda_check(clb::set_smem_limits(), "kernel shared-memory limits");
    cuda_check(clb::set_v2_smem_limits(), "kernel shared-memory limits");
    g_dev_ready.insert(dev);
}

// Routing mode A (route.cpp, mode A): the k largest logits, ties to the lower id, in
// selection order (descending logit); w_i = sigmoid(l_i) / sum of the selected sigmoids
// taken in that order. One pass with an insertion-sorted top-k list gives the same
// order as k arg-max passes. Logits must be finite.
void route_sigmoid_host(const float* logits, int n, int k, int32_t* ids, float* w) {
    float tv[64];
    int ti[64], cnt = 0;
    for (int e = 0; e < n; ++e) {
        const float v = logits[e];
        if (cnt == k && !(v > tv[k - 1])) continue;
        int pos = cnt < k ? cnt++ : k - 1;
        while (pos > 0 && v > tv[pos - 1]) {
            tv[pos] = tv[pos - 1];
            ti[pos] = ti[pos - 1];
            --pos;
        }
        tv[pos] = v;
        ti[pos] = e;
    }
    float s[64], sum = 0.0f;
    for (int i = 0; i < k; ++i) {
        ids[i] = ti[i];
        s[i] = 1.0f / (1.0f + std::exp(-tv[i]));
        sum += s[i];
    }
    for (int i = 0; i < k; ++i) w[i] = s[i] / sum;
}

// Splits [0, n) over up to 16 host threads in chunks of at least `grain` (one thread below
// that): the host-side loops of batched calls (validation of tens of MB, copies into the
// pinned staging buffers) would otherwise dominate their end-to-end time.
template <class F>
void host_parallel(size_t n, size_t grain, F&& f) {
    const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    const size_t parts = std::min<size_t>(hw, (n + grain - 1) / grain);
    if (parts <= 1) {
        f((size_t)0, n);
        return;
    }
    const size_t chunk = (n + parts - 1) / parts;
    std::vector<std::thread> th;
    th.reserve(parts - 1);
    for (size_t p = 1; p < parts; ++p) {
        const size_t b = p * chunk, e = std::min(n, b + chunk);
        if (b < e) th.emplace_back([&f, b, e] { f(b, e); });
    }
    f((size_t)0, std::min(n, chunk));
    for (auto& t : th) t.join();
}

// NVTX range over one entry point ("clb:<call>"), visible in nsys / ncu timelines; a no-op
// unless a tool is attached.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

bool finite_span(const float* v, size_t b, size_t e) {
    uint32_t bad = 0;
    for (size_t i = b; i < e; ++i) {
        uint32_t u;
        std::memcpy(&u, v + i, 4);
        bad |= (uint32_t)((u & 0x7f800000u) == 0x7f800000u);  // exponent all ones: inf or nan
    }
    return bad == 0;
}

bool finite_all(const float* v, size_t n) {
    std::atomic<bool> ok{true};
    host_parallel(n, (size_t)1 << 20, [&](size_t b, size_t e) {
        if (!finite_span(v, b, e)) ok.store(false, std::memory_order_relaxed);
    });
    return ok.load();
}

void copy_parallel(void* dst, const void* src, size_t bytes) {
    host_parallel(bytes, (size_t)4 << 20, [&](size_t b, size_t e) {
        std::memcpy(static_cast<uint8_t*>(dst) + b, static_cast<const uint8_t*>(src) + b, e - b);
    });
}

}  // namespace

struct clb_bank {
    clb_bank_config_v1 cfg{};
    cudaStream_t stream = nullptr;
    cudaEvent_t t_ev0 = nullptr, t_ev1 = nullptr;  // CLB_BANK_TIMING spans
    clb_timing_v1 last_timing{};
    bool poisoned = false;
    std::mutex call_mutex;  // one caller at a time (crosslane's WarmWorker guarantee)

    std::vector<void*> allocations;
    uint64_t weight_bytes = 0;
    std::vector<clb::ExpertDesc> desc;  // [layer][expert]
    std::vector<uint8_t> resident;
    std::vector<uint8_t> placed;  // [layer][expert]: this bank is to hold it (owned range, or a placement)
    clb::ExpertDesc* d_desc = nullptr;
    uint16_t* d_scales = nullptr;

    // fixed workspace
    float *d_x = nullptr, *d_out = nullptr, *d_shared = nullptr, *d_h = nullptr, *d_yrows = nullptr, *d_w = nullptr;
    int8_t *d_xqs = nullptr, *d_hqs = nullptr;
    float *d_xd = nullptr, *d_hd = nullptr;
    int* d_ids = nullptr;
    int* d_err = nullptr;
    float* d_gu = nullptr;          // gate/up rows [pick][2][ff]
    int* d_cnt_h = nullptr;         // last-arriver counters per (pick, 256-row block of h)
    int* d_cnt_y = nullptr;         // last-arriver counters per output row group (16 or 32 rows)
    unsigned* d_bar = nullptr;      // grid barrier state of the persistent stack kernel
    bool persistent = false;        // stack decode runs as one persistent kernel
    // expert-ID sharding over GPUs: exchange region [2][k][dim] floats + kMaxPeers flags,
    // exported through a CUDA IPC handle; peers' regions opened by clb_bank_connect
    uint8_t* d_xchg = nullptr;
    size_t xchg_bytes = 0;
    clb::StackShard shard;
    clb::StackWork stk;             // fast-order workspace of the persistent stack kernel
    unsigned wait_limit = clb::kDefaultWaitLimit;  // polls before a stack kernel's bounded wait gives up
    std::vector<void*> opened_peers;
    float* d_logits = nullptr;
    int* d_route_ids = nullptr;
    float* d_route_w = nullptr;
    float *h_x = nullptr, *h_out = nullptr, *h_logits = nullptr, *h_yrows = nullptr;
    int32_t* h_route_ids = nullptr;  // host-routed stack: [layers][max_picks]
    float* h_route_w = nullptr;
    std::map<std::pair<uint32_t, int>, cudaGraphExec_t> graphs, device_graphs;
    const float* graph_dx = nullptr;
    // batched prefill (clb_prefill_*): grow-only device workspace and pinned host staging
    void* pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    float *pf_hx = nullptr, *pf_hw = nullptr, *pf_dx = nullptr, *pf_dw = nullptr, *pf_dout = nullptr;
    int32_t *pf_hids = nullptr, *pf_dids = nullptr;
    int pf_tokens = 0, pf_k = 0;
    // batched stack decode (clb_stack_batch): grow-only device workspace, h and routes, pinned staging
    void* sb_ws = nullptr;
    float *sb_dh = nullptr, *sb_dw = nullptr, *sb_hh = nullptr, *sb_hw = nullptr;
    int32_t *sb_dids = nullptr, *sb_hids = nullptr;
    int sb_tokens = 0, sb_layers = 0;

    size_t L() const { return (size_t)cfg.n_layers; }
    size_t E() const { return (size_t)cfg.n_experts; }
    bool owns(int e) const { return e >= cfg.expert_begin && e < cfg.expert_end; }
    bool fast() const { return (cfg.flags & CLB_BANK_EXACT_ORDER) == 0; }
    bool use_persistent() const { return persistent; }

    template <class T>
    T* dev_alloc(size_t count) {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 256));
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(CLB_E_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        }
        allocations.push_back(p);
        return static_cast<T*>(p);
    }
    template <class T>
    T* host_alloc(size_t count) {
        void* p = nullptr;
        cuda_check(cudaMallocHost(&p, std::max<size_t>(count * sizeof(T), 256)), "cudaMallocHost");
        host_allocations.push_back(p);
        return static_cast<T*>(p);
    }
    std::vector<void*> host_allocations;

    void check_usable() { require(!poisoned, CLB_E_STATE, "bank poisoned by an earlier device failure"); }

    // device_step of a synchronous host call, timed under CLB_BANK_TIMING: events on the bank
    // stream around everything f enqueues (f ends with its copies back), one JSON line.
    template <class F>
    void timed_step(const char* call, int layer, int layers, int picks, uint64_t h2d, uint64_t d2h, F&& f) {
        char name[48];
        std::snprintf(name, sizeof name, "clb:%s", call);
        NvtxRange range(name);
        if (!t_ev0) {
            device_step(f);
            return;
        }
        device_step([&] {
            cuda_check(cudaEventRecord(t_ev0, stream), "timing event");
            f();
            cuda_check(cudaEventRecord(t_ev1, stream), "timing event");
            cuda_check(cudaEventSynchronize(t_ev1), "timing sync");
            float ms = 0.0f;
            cuda_check(cudaEventElapsedTime(&ms, t_ev0, t_ev1), "timing");
            last_timing = clb_timing_v1{(uint64_t)((double)ms * 1e6), h2d, d2h, layer, layers, picks, 0};
            std::fprintf(stderr,
                         "{\"schema\":\"clb-cuda-timing-v1\",\"lane\":\"cuda\",\"device\":%d,\"call\":\"%s\","
                         "\"layer\":%d,\"layers\":%d,\"picks\":%d,\"h2d_bytes\":%llu,\"d2h_bytes\":%llu,"
                         "\"ns\":%llu}\n",
                         cfg.device, call, layer, layers, picks, (unsigned long long)h2d, (unsigned long long)d2h,
                         (unsigned long long)last_timing.ns);
        });
    }

    // Runs f; on a device failure the bank is poisoned (abi_backend_plugin.cpp:31-39 convention).
    template <class F>
    void device_step(F&& f) {
        try {
            f();
        } catch (const Error& e) {
            if (e.code == CLB_E_CUDA) poisoned = true;
            throw;
        }
    }

    void check_err_flag() {
        int flag = 0;
        cuda_check(cudaMemcpyAsync(&flag, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream), "error flag D2H");
        cuda_check(cudaStreamSynchronize(stream), "stream sync");
        if (flag) {
            cuda_check(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "error flag reset");
            if (flag == 2) throw Error(CLB_E_CUDA, "a bounded wait of the stack kernel ran out (a peer GPU or CTA never posted)");
            if (flag == 3) throw Error(CLB_E_CUDA, "a tensor-core pipeline wait of the prefill kernel timed out");
            throw Error(CLB_E_INVALID, "a picked expert is not resident or has a mismatched shape");
        }
    }

    // Weight types among the layer's resident experts (clb::kTypeBit* bits), which selects
    // the grouped GEMM's decoder instantiation.
    int layer_types(uint32_t layer) const {
        int m = 0;
        for (size_t e = 0; e < E(); ++e) {
            if (!resident[(size_t)layer * E() + e]) continue;
            const auto& d = desc[(size_t)layer * E() + e];
            for (int t : {d.gate.type, d.up.type, d.down.type})
                m |= t == CLB_IQ2_XXS ? clb::kTypeBitXXS : t == CLB_IQ2_XS ? clb::kTypeBitXS : clb::kTypeBitIQ1M;
        }
        return m ? m : clb::kTypeBitAll;
    }
    std::vector<int> layer_types(uint32_t first, int nl) const {
        std::vector<int> v((size_t)nl);
        for (int l = 0; l < nl; ++l) v[(size_t)l] = layer_types(first + (uint32_t)l);
        return v;
    }

    void validate_ids(uint32_t layer, const int32_t* ids, int n, bool need_resident) {
        require(layer < (uint32_t)cfg.n_layers, CLB_E_INVALID, "layer %u out of range", layer);
        require(n >= 1 && n <= cfg.max_picks, CLB_E_INVALID, "pick count %d outside [1, %d]", n, cfg.max_picks);
        std::set<int> seen;
        for (int i = 0; i < n; ++i) {
            require(ids[i] >= 0 && ids[i] < cfg.n_experts, CLB_E_INVALID, "expert id %d out of range", ids[i]);
            require(seen.insert(ids[i]).second, CLB_E_INVALID, "duplicate expert id %d", ids[i]);
            if (need_resident)
                require(resident[(size_t)layer * E() + (size_t)ids[i]], CLB_E_INVALID,
                        "expert (%u, %d) is not resident in this bank", layer, ids[i]);
        }
    }

    // norm: the stack's pre-norm x = RMSNorm(h) is fused into the quantisation of x.
    void enqueue_layer(uint32_t layer, const int* ids, const float* w, int n, const float* x, const float* shared,
                       const float* resid, float* out, float* yrows, cudaStream_t s, bool norm = false) {
        const int dim = cfg.dim, ff = cfg.ff;
        const clb::ExpertDesc* ex = d_desc + (size_t)layer * E();
        if (norm)
            cuda_check(clb::launch_norm_quant(x, dim, d_xqs, d_xd, nullptr, s), "norm + quantize x");
        else
            cuda_check(clb::launch_quant(x, dim / 256, d_xqs, d_xd, s), "quantize x");
        cuda_check(clb::launch_gateup2(ex, ids, n, d_xqs, d_xd, dim, ff, cfg.limit, d_gu, d_hqs, d_hd, d_cnt_h, d_err, fast(), s),
                   "gate/up + SwiGLU + quantize h");
        cuda_check(clb::launch_down2(ex, ids, w, n, d_hqs, d_hd, dim, ff, shared, resid, out, yrows ? yrows : d_yrows,
                                     d_cnt_y, d_err, fast(), s),
                   "down + combine");
    }

    void enqueue_phases(uint32_t layer, const int* ids, const float* w, int n, const float* x, float* out, int mask,
                        cudaStream_t s) {
        const int dim = cfg.dim, ff = cfg.ff;
        const clb::ExpertDesc* ex = d_desc + (size_t)layer * E();
        if (mask & 1) cuda_check(clb::launch_quant(x, dim / 256, d_xqs, d_xd, s), "quantize x");
        if (mask & 2)
            cuda_check(clb::launch_gateup2(ex, ids, n, d_xqs, d_xd, dim, ff, cfg.limit, d_gu, d_hqs, d_hd, d_cnt_h, d_err,
                                           fast(), s),
                       "gate/up + SwiGLU + quantize h");
        if (mask & 8)
            cuda_check(clb::launch_down2(ex, ids, w, n, d_hqs, d_hd, dim, ff, nullptr, nullptr, out, d_yrows, d_cnt_y,
                                         d_err, fast(), s),
                       "down + combine");
    }

    // dlogits == nullptr: d_route_ids / d_route_w already hold the routing of the range.
    void enqueue_stack(uint32_t first, int nl, float* dx, const float* dlogits, cudaStream_t s) {
        const int k = cfg.max_picks;
        if (dlogits)
            cuda_check(clb::launch_route_sigmoid(dlogits, cfg.n_experts, k, nl, d_route_ids, d_route_w, s), "route");
        if (persistent) {
            cuda_check(clb::launch_stack(d_desc, cfg.n_experts, (int)first, nl, k, d_route_ids, d_route_w, dx, dx,
                                         cfg.dim, cfg.ff, cfg.limit, d_gu, d_yrows, d_bar, d_err, fast(), shard, s,
                                         wait_limit, stk),
                       "persistent stack kernel");
            // layers run through the kernel: the parity and targets of the monotonic row-group
            // counters and exchange flags (every GPU runs the same launches)
            shard.epoch += (unsigned)nl;
            return;
        }
        for (int i = 0; i < nl; ++i)
            enqueue_layer(first + (uint32_t)i, d_route_ids + (size_t)i * k, d_route_w + (size_t)i * k, k, dx, nullptr,
                          dx, dx, nullptr, s, true);
    }

    void set_matrix(uint32_t layer, int e, int role, int type, uint8_t* base) {
        const int n = role == 2 ? cfg.dim : cfg.ff, k = role == 2 ? cfg.ff : cfg.dim;
        const PackedLayout l = clb_packed_layout(type, n, k);
        PackedMat m{};
        m.body = base + l.body;
        m.sc = base + l.sc;
        m.d = reinterpret_cast<const uint16_t*>(base + l.d);
        m.type = type;
        m.n = n;
        m.k = k;
        auto& d = desc[(size_t)layer * E() + (size_t)e];
        (role == 0 ? d.gate : role == 1 ? d.up : d.down) = m;
    }

    void refresh_resident(uint32_t layer, int e) {
        const auto& d = desc[(size_t)layer * E() + (size_t)e];
        resident[(size_t)layer * E() + (size_t)e] = d.gate.body && d.up.body && d.down.body;
    }

    void upload_desc() {
        cuda_check(cudaMemcpyAsync(d_desc, desc.data(), desc.size() * sizeof(clb::ExpertDesc), cudaMemcpyHostToDevice,
                                   stream),
                   "descriptor upload");
        cuda_check(cudaStreamSynchronize(stream), "descriptor sync");
    }

    void free_prefill() {
        for (void* p : {(void*)pf_ws, (void*)pf_dx, (void*)pf_dw, (void*)pf_dout, (void*)pf_dids})
            if (p) cudaFree(p);
        for (void* p : {(void*)pf_hx, (void*)pf_hw, (void*)pf_hids})
            if (p) cudaFreeHost(p);
        pf_ws = nullptr, pf_dx = pf_dw = pf_dout = nullptr, pf_dids = nullptr, pf_hx = pf_hw = nullptr;
        pf_hids = nullptr, pf_ws_bytes = 0, pf_tokens = pf_k = 0;
    }

    void free_stack_batch() {
        for (void* p : {(void*)sb_ws, (void*)sb_dh, (void*)sb_dw, (void*)sb_dids})
            if (p) cudaFree(p);
        for (void* p : {(void*)sb_hh, (void*)sb_hw, (void*)sb_hids})
            if (p) cudaFreeHost(p);
        sb_ws = nullptr, sb_dh = sb_dw = sb_hh = sb_hw = nullptr, sb_dids = sb_hids = nullptr;
        sb_tokens = sb_layers = 0;
    }

    ~clb_bank() {
        free_prefill();
        free_stack_batch();
        for (void* p : opened_peers) cudaIpcCloseMemHandle(p);
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);
        for (auto& g : device_graphs) cudaGraphExecDestroy(g.second);
        for (void* p : allocations) cudaFree(p);
        for (void* p : host_allocations) cudaFreeHost(p);
        if (t_ev0) cudaEventDestroy(t_ev0);
        if (t_ev1) cudaEventDestroy(t_ev1);
        if (stream) cudaStreamDestroy(stream);
    }
};

extern "C" {

int32_t clb_abi_version(void) { return CLB_ABI_VERSION; }

// ---- Q8_K primitives ----
size_t clb_q8k_activation_bytes(int32_t k) {
    return (k > 0 && k % 256 == 0) ? (size_t)(k / 256) * clb::kQ8KBlockBytes : 0;
}

int32_t clb_q8k_quantize(const float* x, void* q, int32_t k, void* stream) {
    if (!x || !q || !clb_q8k_activation_bytes(k)) return CLB_E_INVALID;
    return clb::launch_quant_blocks(x, k / 256, q, static_cast<cudaStream_t>(stream)) == cudaSuccess ? CLB_OK
                                                                                                      : CLB_E_CUDA;
}

int32_t clb_q8k_mv(int32_t type, const void* w, const void* q, float* y, int32_t n, int32_t k, void* stream) {
    if (!clb_type_supported(type) || !w || !q || !y || n <= 0 || !clb_q8k_activation_bytes(k) || k > 65536)
        return CLB_E_INVALID;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CLB_E_CUDA;
    try {
        ensure_device_ready(dev, static_cast<cudaStream_t>(stream));
    } catch (...) {
        return CLB_E_CUDA;
    }
    const PackedLayout l = clb_packed_layout(type, n, k);
    const uint8_t* base = static_cast<const uint8_t*>(w);
    PackedMat m{};
    m.body = base + l.body;
    m.sc = base + l.sc;
    m.d = reinterpret_cast<const uint16_t*>(base + l.d);
    m.type = type;
    m.n = n;
    m.k = k;
    return clb::launch_mv2(m, q, y, static_cast<cudaStream_t>(stream)) == cudaSuccess ? CLB_OK : CLB_E_CUDA;
}

int32_t clb_q8k_activate(const float* g, const float* u, float* h, int32_t n, float limit, void* stream) {
    if (!g || !u || !h || n <= 0 || !std::isfinite(limit)) return CLB_E_INVALID;
    return clb::launch_activate(g, u, h, n, limit, static_cast<cudaStream_t>(stream)) == cudaSuccess ? CLB_OK
                                                                                                      : CLB_E_CUDA;
}

size_t clb_decode_tables(uint32_t* out, size_t words) {
    if (!out || words < (size_t)clb::kTableWords) return 0;
    clb::host_tables(out);
    return (size_t)clb::kTableWords;
}

// ---- layout ----
size_t clb_packed_bytes(int32_t type, int32_t n, int32_t k) {
    if (!clb_type_supported(type) || n <= 0 || k <= 0 || k % 256) return 0;
    return clb_packed_layout(type, n, k).total;
}

int32_t clb_pack(int32_t type, int32_t n, int32_t k, const void* ggml, size_t ggml_bytes, void* packed,
                 size_t packed_bytes) {
    const size_t need = clb_packed_bytes(type, n, k);
    if (!need || !ggml || !packed) return CLB_E_INVALID;
    const int nb = k / 256, bb = clb_block_bytes(type);
    if (ggml_bytes != (size_t)n * nb * bb || packed_bytes < need) return CLB_E_INVALID;
    const PackedLayout l = clb_packed_layout(type, n, k);
    const uint8_t* src = static_cast<const uint8_t*>(ggml);
    for (size_t i = 0; i < (size_t)n * nb; ++i)
        if ((clb_block_half(type, src + i * bb) & 0x7c00u) == 0x7c00u) return CLB_E_NONFINITE;
    std::memset(packed, 0, need);
    for (int r = 0; r < n; ++r)
        for (int b = 0; b < nb; ++b)
            clb_pack_block(type, n, nb, r, b, src + ((size_t)r * nb + b) * bb, static_cast<uint8_t*>(packed), l);
    return CLB_OK;
}

int32_t clb_unpack(int32_t type, int32_t n, int32_t k, const void* packed, size_t packed_bytes, void* ggml,
                   size_t ggml_bytes) {
    const size_t need = clb_packed_bytes(type, n, k);
    if (!need || !ggml || !packed) return CLB_E_INVALID;
    const int nb = k / 256, bb = clb_block_bytes(type);
    if (ggml_bytes != (size_t)n * nb * bb || packed_bytes < need) return CLB_E_INVALID;
    const PackedLayout l = clb_packed_layout(type, n, k);
    for (int r = 0; r < n; ++r)
        for (int b = 0; b < nb; ++b)
            clb_unpack_block(type, n, nb, r, b, static_cast<const uint8_t*>(packed), l,
                             static_cast<uint8_t*>(ggml) + ((size_t)r * nb + b) * bb);
    return CLB_OK;
}

// ---- bank ----
int32_t clb_bank_create(const clb_bank_config_v1* cfg_in, clb_bank** out, clb_error_v1* err) {
    if (!cfg_in || !out) return fail(err, CLB_E_INVALID, "null config/out");
    *out = nullptr;
    clb_bank* bank = nullptr;
    int rc = guarded(err, [&] {
        clb_bank_config_v1 cfg = *cfg_in;
        if (cfg.expert_begin == 0 && cfg.expert_end == 0) cfg.expert_end = cfg.n_experts;
        require(cfg.n_layers > 0 && cfg.n_experts > 0 && cfg.n_experts <= clb::kMaxExperts, CLB_E_INVALID,
                "layers/experts out of range");
        require(cfg.dim > 0 && cfg.dim % 256 == 0 && cfg.ff > 0 && cfg.ff % 256 == 0 && cfg.dim <= 32768 &&
                    cfg.ff <= 16384,
                CLB_E_UNSUPPORTED, "dim and ff must be positive multiples of 256 (dim <= 32768, ff <= 16384)");
        require(cfg.max_picks >= 1 && cfg.max_picks <= clb::kMaxPicks && cfg.max_picks <= cfg.n_experts,
                CLB_E_INVALID, "max_picks must be in [1, min(16, n_experts)]");
        require(std::isfinite(cfg.limit) && cfg.limit >= 0, CLB_E_INVALID, "SwiGLU limit must be finite and >= 0");
        require((cfg.flags & ~(CLB_BANK_EXACT_ORDER | CLB_BANK_PER_LAYER_KERNELS | CLB_BANK_TIMING)) == 0,
                CLB_E_INVALID, "unknown bank flags 0x%x", cfg.flags);
        require(cfg.expert_begin >= 0 && cfg.expert_begin < cfg.expert_end && cfg.expert_end <= cfg.n_experts,
                CLB_E_INVALID, "owned expert range invalid");
        require((size_t)cfg.max_picks * (cfg.ff / 256) <= 256, CLB_E_UNSUPPORTED,
                "max_picks * ff / 256 must be <= 256 (the down kernel stages every pick's Q8_K(h) in shared memory)");
        int ndev = 0;
        cuda_check(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
        require(cfg.device >= 0 && cfg.device < ndev, CLB_E_INVALID, "device %d not present", cfg.device);
        DeviceGuard g(cfg.device);
        bank = new clb_bank();
        bank->cfg = cfg;
        cuda_check(cudaStreamCreateWithFlags(&bank->stream, cudaStreamNonBlocking), "stream");
        if (cfg.flags & CLB_BANK_TIMING) {
            cuda_check(cudaEventCreate(&bank->t_ev0), "timing event");
            cuda_check(cudaEventCreate(&bank->t_ev1), "timing event");
        }
        ensure_device_ready(cfg.device, bank->stream);
        bank->desc.assign(bank->L() * bank->E(), clb::ExpertDesc{});
        bank->resident.assign(bank->L() * bank->E(), 0);
        bank->placed.assign(bank->L() * bank->E(), 0);
        for (size_t l = 0; l < bank->L(); ++l)
            for (int e = bank->cfg.expert_begin; e < bank->cfg.expert_end; ++e) bank->placed[l * bank->E() + (size_t)e] = 1;
        bank->d_desc = bank->dev_alloc<clb::ExpertDesc>(bank->L() * bank->E());
        const size_t dim = (size_t)cfg.dim, ff = (size_t)cfg.ff, k = (size_t)cfg.max_picks;
        bank->d_x = bank->dev_alloc<float>(dim);
        bank->d_out = bank->dev_alloc<float>(dim);
        bank->d_shared = bank->dev_alloc<float>(dim);
        bank->d_xqs = bank->dev_alloc<int8_t>(dim);
        bank->d_xd = bank->dev_alloc<float>(dim / 256);
        bank->d_h = bank->dev_alloc<float>(k * ff);
        bank->d_hqs = bank->dev_alloc<int8_t>(k * ff);
        bank->d_hd = bank->dev_alloc<float>(k * ff / 256);
        bank->d_yrows = bank->dev_alloc<float>(k * dim);
        bank->d_gu = bank->dev_alloc<float>(k * 2 * ff);
        bank->d_cnt_h = bank->dev_alloc<int>(k * ff / 256);
        bank->d_cnt_y = bank->dev_alloc<int>((dim + 15) / 16);
        cuda_check(cudaMemsetAsync(bank->d_cnt_h, 0, sizeof(int) * k * ff / 256, bank->stream), "memset");
        cuda_check(cudaMemsetAsync(bank->d_cnt_y, 0, sizeof(int) * ((dim + 15) / 16), bank->stream), "memset");
        bank->d_bar = bank->dev_alloc<unsigned>(2);
        // exchange region: expert rows [2][k][dim], kMaxPeers peer counters, row-group counters [2][dim / 32]
        bank->xchg_bytes = 2 * k * dim * sizeof(float) + clb::kMaxPeers * sizeof(unsigned) + 2 * (dim / 32) * sizeof(unsigned);
        bank->d_xchg = bank->dev_alloc<uint8_t>(bank->xchg_bytes);
        cuda_check(cudaMemsetAsync(bank->d_xchg, 0, bank->xchg_bytes, bank->stream), "memset");
        bank->shard.own_begin = cfg.expert_begin;
        bank->shard.own_end = cfg.expert_end;
        bank->shard.yx = reinterpret_cast<float*>(bank->d_xchg);
        bank->shard.flags = reinterpret_cast<unsigned*>(bank->d_xchg + 2 * k * dim * sizeof(float));
        bank->shard.rgcnt = bank->shard.flags + clb::kMaxPeers;
        bank->persistent = (cfg.flags & CLB_BANK_PER_LAYER_KERNELS) == 0 &&
                           clb::stack_supported(cfg.dim, cfg.ff, cfg.max_picks, bank->fast());
        if (bank->persistent && bank->fast()) {
            bank->stk.hbuf = bank->dev_alloc<float>(2 * dim);
            bank->stk.ssbuf = bank->dev_alloc<float>(2 * (dim / 32));
            bank->stk.blk = bank->dev_alloc<unsigned>(clb::stack_block_words(cfg.n_layers, (int)k, (int)ff));
        }
        bank->d_ids = bank->dev_alloc<int>(k);
        bank->d_w = bank->dev_alloc<float>(k);
        bank->d_err = bank->dev_alloc<int>(1);
        bank->d_logits = bank->dev_alloc<float>(bank->L() * bank->E());
        bank->d_route_ids = bank->dev_alloc<int>(bank->L() * k);
        bank->d_route_w = bank->dev_alloc<float>(bank->L() * k);
        bank->h_x = bank->host_alloc<float>(dim);
        bank->h_out = bank->host_alloc<float>(dim);
        bank->h_yrows = bank->host_alloc<float>(k * dim);
        bank->h_logits = bank->host_alloc<float>(bank->L() * bank->E());
        bank->h_route_ids = bank->host_alloc<int32_t>(bank->L() * k);
        bank->h_route_w = bank->host_alloc<float>(bank->L() * k);
        cuda_check(cudaMemsetAsync(bank->d_err, 0, sizeof(int), bank->stream), "memset");
        bank->upload_desc();
    });
    if (rc != CLB_OK) {
        delete bank;
        return rc;
    }
    *out = bank;
    return CLB_OK;
}

void clb_bank_destroy(clb_bank* bank) {
    if (!bank) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(bank->cfg.device);
    if (bank->stream) cudaStreamSynchronize(bank->stream);
    delete bank;
    if (prev >= 0) cudaSetDevice(prev);
}

uint64_t clb_bank_weight_bytes(const clb_bank* bank) { return bank ? bank->weight_bytes : 0; }

// ---- frozen warm placement (STRATA_WARM_PLACEMENT_V1, frozen_placement.hpp:5-16) ----
int32_t clb_placement_parse(const char* text, size_t len, int32_t n_layers, int32_t n_experts, int32_t* lanes,
                            uint64_t* tag, clb_error_v1* err) {
    if (!text || !lanes || n_layers <= 0 || n_experts <= 0) return fail(err, CLB_E_INVALID, "null placement/output");
    return guarded(err, [&] {
        const char* p = text;
        const char* end = text + len;
        auto word = [&](std::string& w) {
            while (p < end && std::isspace((unsigned char)*p)) ++p;
            const char* b = p;
            while (p < end && !std::isspace((unsigned char)*p)) ++p;
            w.assign(b, (size_t)(p - b));
            return !w.empty();
        };
        auto number = [&](uint64_t& v) {
            std::string w;
            if (!word(w) || w.size() > 20) return false;
            for (char c : w)
                if (c < '0' || c > '9') return false;
            errno = 0;
            v = std::strtoull(w.c_str(), nullptr, 10);
            return errno == 0;
        };
        std::string version;
        uint64_t nl = 0, ne = 0, t = 0;
        require(word(version) && version == "STRATA_WARM_PLACEMENT_V1" && number(nl) && number(ne) && number(t) &&
                    nl == (uint64_t)n_layers && ne == (uint64_t)n_experts,
                CLB_E_INVALID, "warm placement header/profile mismatch");
        for (int32_t l = 0; l < n_layers; ++l)
            for (int32_t e = 0; e < n_experts; ++e) {
                uint64_t rl = 0, re = 0, lane = 0;
                require(number(rl) && number(re) && number(lane) && rl == (uint64_t)l && re == (uint64_t)e &&
                            lane <= (uint64_t)CLB_LANE_CUDA,
                        CLB_E_INVALID, "warm placement missing/duplicate/unsorted row at (%d, %d)", l, e);
                lanes[(size_t)l * (size_t)n_experts + (size_t)e] = (int32_t)lane;
            }
        std::string extra;
        require(!word(extra), CLB_E_INVALID, "extra/invalid warm placement data");
        if (tag) *tag = t;
    });
}

int32_t clb_bank_apply_placement(clb_bank* bank, const int32_t* lanes, int32_t lane_id, clb_error_v1* err) {
    if (!bank || !lanes) return fail(err, CLB_E_INVALID, "null bank/placement");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        require(lane_id >= 1 && lane_id <= CLB_LANE_CUDA, CLB_E_INVALID, "lane id %d is not a GPU lane", lane_id);
        require(bank->weight_bytes == 0, CLB_E_STATE, "placement must be applied before any weights are loaded");
        for (size_t l = 0; l < bank->L(); ++l)
            for (size_t e = 0; e < bank->E(); ++e) {
                const int32_t lane = lanes[l * bank->E() + e];
                require(lane >= 0 && lane <= CLB_LANE_CUDA, CLB_E_INVALID, "lane %d out of range", lane);
                require(lane != lane_id || bank->owns((int)e), CLB_E_INVALID,
                        "expert (%zu, %zu) is placed on this lane but outside the bank's owned range", l, e);
                bank->placed[l * bank->E() + e] = lane == lane_id ? 1 : 0;
            }
    });
}

int32_t clb_bank_placed(const clb_bank* bank, uint32_t layer, int32_t expert) {
    if (!bank || layer >= (uint32_t)bank->cfg.n_layers || expert < 0 || expert >= bank->cfg.n_experts) return 0;
    return bank->placed[(size_t)layer * bank->E() + (size_t)expert] ? 1 : 0;
}

int32_t clb_bank_contains(const clb_bank* bank, uint32_t layer, int32_t expert) {
    if (!bank || layer >= (uint32_t)bank->cfg.n_layers || expert < 0 || expert >= bank->cfg.n_experts) return 0;
    return bank->resident[(size_t)layer * bank->E() + (size_t)expert] ? 1 : 0;
}

int32_t clb_bank_stack_persistent(const clb_bank* bank) { return bank && bank->persistent ? 1 : 0; }

int32_t clb_bank_set_wait_limit(clb_bank* bank, uint32_t polls, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        require(polls >= 1, CLB_E_INVALID, "wait limit must be at least one poll");
        bank->wait_limit = polls;
    });
}

int32_t clb_bank_exchange_handle(clb_bank* bank, void* handle_out, clb_error_v1* err) {
    if (!bank || !handle_out) return fail(err, CLB_E_INVALID, "null bank/handle");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        DeviceGuard g(bank->cfg.device);
        cudaIpcMemHandle_t h;
        cuda_check(cudaIpcGetMemHandle(&h, bank->d_xchg), "cudaIpcGetMemHandle");
        static_assert(sizeof(h) == CLB_EXCHANGE_HANDLE_BYTES, "IPC handle size");
        std::memcpy(handle_out, &h, sizeof(h));
    });
}

int32_t clb_bank_connect(clb_bank* bank, int32_t rank, int32_t world, const void* handles, clb_error_v1* err) {
    if (!bank || !handles) return fail(err, CLB_E_INVALID, "null bank/handles");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        require(world >= 2 && world <= clb::kMaxPeers && rank >= 0 && rank < world, CLB_E_INVALID,
                "rank %d / world %d outside [0, %d)", rank, world, clb::kMaxPeers);
        require(bank->shard.world == 1, CLB_E_STATE, "bank already connected");
        require(bank->persistent, CLB_E_UNSUPPORTED,
                "expert-ID sharding runs in the persistent stack kernel (not available for this geometry/flags)");
        DeviceGuard g(bank->cfg.device);
        clb::StackShard sh = bank->shard;
        std::vector<void*> opened;
        try {
            for (int r = 0; r < world; ++r) {
                if (r == rank) continue;
                cudaIpcMemHandle_t h;
                std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * CLB_EXCHANGE_HANDLE_BYTES, sizeof(h));
                void* p = nullptr;
                cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
                opened.push_back(p);
                const size_t k = (size_t)bank->cfg.max_picks, dim = (size_t)bank->cfg.dim;
                sh.peer_yx[r] = static_cast<float*>(p);
                sh.peer_flags[r] = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(p) + 2 * k * dim * sizeof(float));
                sh.peer_rgcnt[r] = sh.peer_flags[r] + clb::kMaxPeers;
            }
        } catch (...) {
            for (void* p : opened) cudaIpcCloseMemHandle(p);
            throw;
        }
        sh.world = world;
        sh.rank = rank;
        sh.epoch = 0;
        bank->shard = sh;
        bank->opened_peers = opened;
    });
}

int32_t clb_bank_fill_synthetic(clb_bank* bank, uint64_t seed, int32_t policy, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        require(policy >= 0 && policy <= 4, CLB_E_INVALID, "type policy %d unknown", policy);
        DeviceGuard g(bank->cfg.device);
        std::call_once(g_scale_once, [] { clb_build_scale_table(g_scale_host); });
        bank->device_step([&] {
            if (!bank->d_scales) {
                bank->d_scales = bank->dev_alloc<uint16_t>(65536);
                cuda_check(cudaMemcpyAsync(bank->d_scales, g_scale_host, sizeof g_scale_host, cudaMemcpyHostToDevice,
                                           bank->stream),
                           "scale table upload");
            }
            const auto& c = bank->cfg;
            for (uint32_t layer = 0; layer < (uint32_t)c.n_layers; ++layer) {
                // one slab per layer, each matrix 256-byte aligned inside it
                size_t slab = 0;
                std::vector<size_t> offs;
                for (int e = c.expert_begin; e < c.expert_end; ++e) {
                    if (!bank->placed[(size_t)layer * bank->E() + (size_t)e]) continue;
                    const int t = clb_expert_type(policy, seed, layer, (uint32_t)e);
                    for (int role = 0; role < 3; ++role) {
                        offs.push_back(slab);
                        slab += clb_packed_layout(t, role == 2 ? c.dim : c.ff, role == 2 ? c.ff : c.dim).total;
                    }
                }
                if (slab == 0) continue;  // nothing placed in this layer
                uint8_t* base = bank->dev_alloc<uint8_t>(slab);
                bank->weight_bytes += slab;
                size_t i = 0;
                for (int e = c.expert_begin; e < c.expert_end; ++e) {
                    if (!bank->placed[(size_t)layer * bank->E() + (size_t)e]) continue;
                    const int t = clb_expert_type(policy, seed, layer, (uint32_t)e);
                    for (int role = 0; role < 3; ++role, ++i) {
                        const int n = role == 2 ? c.dim : c.ff, k = role == 2 ? c.ff : c.dim;
                        const PackedLayout l = clb_packed_layout(t, n, k);
                        cuda_check(clb::launch_synth_fill(base + offs[i], l, t, n, k, seed, layer, (uint32_t)e,
                                                          (uint32_t)role, bank->d_scales, bank->stream),
                                   "synthetic fill");
                        bank->set_matrix(layer, e, role, t, base + offs[i]);
                    }
                    bank->refresh_resident(layer, e);
                }
            }
            cuda_check(cudaStreamSynchronize(bank->stream), "fill sync");
            bank->upload_desc();
        });
    });
}

static void load_matrix_locked(clb_bank* bank, uint32_t layer, int32_t expert, int32_t role, int32_t type,
                               const void* ggml, size_t bytes, bool upload) {
    bank->check_usable();
    const auto& c = bank->cfg;
    require(layer < (uint32_t)c.n_layers && expert >= 0 && expert < c.n_experts && role >= 0 && role <= 2,
            CLB_E_INVALID, "matrix address out of range");
    require(bank->owns(expert), CLB_E_INVALID, "expert %d outside this bank's owned range", expert);
    require(bank->placed[(size_t)layer * bank->E() + (size_t)expert], CLB_E_INVALID,
            "expert (%u, %d) is not placed on this bank", layer, expert);
    require(clb_type_supported(type), CLB_E_UNSUPPORTED, "quant type %d has no kernel", type);
    const int n = role == 2 ? c.dim : c.ff, k = role == 2 ? c.ff : c.dim;
    require(ggml && bytes == (size_t)n * (k / 256) * clb_block_bytes(type), CLB_E_INVALID,
            "matrix byte extent %zu does not match [%d, %d] of type %d", bytes, n, k, type);
    auto& d = bank->desc[(size_t)layer * bank->E() + (size_t)expert];
    const PackedMat& cur = role == 0 ? d.gate : role == 1 ? d.up : d.down;
    require(cur.body == nullptr, CLB_E_INVALID, "matrix already loaded");
    DeviceGuard g(c.device);
    bank->device_step([&] {
        const PackedLayout l = clb_packed_layout(type, n, k);
        uint8_t* packed = bank->dev_alloc<uint8_t>(l.total);
        void* staging = nullptr;
        cuda_check(cudaMalloc(&staging, bytes), "staging alloc");
        int bad = 0;
        cudaError_t e = cudaMemcpyAsync(staging, ggml, bytes, cudaMemcpyHostToDevice, bank->stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(bank->d_err, 0, sizeof(int), bank->stream);
        if (e == cudaSuccess)
            e = clb::launch_pack(static_cast<const uint8_t*>(staging), packed, l, type, n, k, bank->d_err,
                                 bank->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&bad, bank->d_err, sizeof(int), cudaMemcpyDeviceToHost, bank->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(bank->stream);
        cudaFree(staging);
        cuda_check(e, "matrix upload/pack");
        if (bad) {
            cuda_check(cudaMemsetAsync(bank->d_err, 0, sizeof(int), bank->stream), "flag reset");
            throw Error(CLB_E_NONFINITE, "non-finite fp16 super-scale in matrix");
        }
        bank->weight_bytes += l.total;
        bank->set_matrix(layer, expert, role, type, packed);
        bank->refresh_resident(layer, expert);
        if (upload) bank->upload_desc();
    });
}

int32_t clb_bank_load_matrix(clb_bank* bank, uint32_t layer, int32_t expert, int32_t role, int32_t type,
                             const void* ggml, size_t bytes, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] { load_matrix_locked(bank, layer, expert, role, type, ggml, bytes, true); });
}

int32_t clb_bank_geometry(const clb_bank* bank, int32_t* n_layers, int32_t* n_experts, int32_t* dim, int32_t* ff) {
    if (!bank) return CLB_E_INVALID;
    if (n_layers) *n_layers = bank->cfg.n_layers;
    if (n_experts) *n_experts = bank->cfg.n_experts;
    if (dim) *dim = bank->cfg.dim;
    if (ff) *ff = bank->cfg.ff;
    return CLB_OK;
}

int32_t clb_bank_load_strata_pack(clb_bank* bank, const clb_strata_pack* pack, uint32_t first_layer, clb_error_v1* err) {
    if (!bank || !pack) return fail(err, CLB_E_INVALID, "null bank/pack");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        auto geo = [&](const char* key, long want) {
            const std::string v = clb::pack_meta(pack, key);
            require(v.empty() || std::strtol(v.c_str(), nullptr, 10) == want, CLB_E_INVALID,
                    "pack %s = %s, the bank has %ld", key, v.c_str(), want);
        };
        geo("hidden_size", c.dim);
        geo("moe_intermediate_size", c.ff);
        geo("n_routed_experts", c.n_experts);
        const std::string nh = clb::pack_meta(pack, "num_hidden_layers");
        require(nh.empty() || (long)first_layer + c.n_layers <= std::strtol(nh.c_str(), nullptr, 10), CLB_E_INVALID,
                "pack has %s layers, the bank spans %u..%u", nh.c_str(), first_layer, first_layer + c.n_layers - 1);
        const std::string lim = clb::pack_meta(pack, "swiglu_limit");
        require(lim.empty() || std::strtof(lim.c_str(), nullptr) == c.limit, CLB_E_INVALID,
                "pack swiglu_limit %s differs from the bank's %g", lim.c_str(), (double)c.limit);
        static const char* roles[3] = {"w1", "w3", "w2"};  // gate, up, down (cpu_lane.hpp:36)
        std::vector<uint8_t> buf;
        size_t loaded = 0;
        for (int l = 0; l < c.n_layers; ++l)
            for (int e = 0; e < c.n_experts; ++e) {
                if (!bank->placed[(size_t)l * bank->E() + (size_t)e]) continue;
                for (int role = 0; role < 3; ++role) {
                    const std::string name = "layers." + std::to_string(first_layer + (uint32_t)l) + ".ffn.experts." +
                                             std::to_string(e) + "." + roles[role] + ".weight";
                    const clb::PackTensor* t = clb::pack_find(pack, name);
                    require(t != nullptr, CLB_E_INVALID, "missing tensor %s", name.c_str());
                    const int type = clb::pack_expert_type(t->dtype);
                    require(type != 0, CLB_E_UNSUPPORTED, "%s: unadmitted dtype %s", name.c_str(), t->dtype.c_str());
                    const long n = role == 2 ? c.dim : c.ff, k = role == 2 ? c.ff : c.dim;
                    require(t->shape.size() < 2 || (t->shape[0] == n && t->shape[1] == k), CLB_E_INVALID,
                            "%s: shape %lld x %lld, expected %ld x %ld", name.c_str(),
                            (long long)(t->shape.size() ? t->shape[0] : 0), (long long)(t->shape.size() > 1 ? t->shape[1] : 0),
                            n, k);
                    buf.resize((size_t)t->bytes);
                    clb::pack_read(pack, *t, 0, buf.data(), t->bytes);
                    load_matrix_locked(bank, (uint32_t)l, e, role, type, buf.data(), buf.size(), false);
                    ++loaded;
                }
            }
        if (loaded) {
            DeviceGuard g(c.device);
            bank->device_step([&] { bank->upload_desc(); });
        }
    });
}

void* clb_bank_stream(clb_bank* bank) { return bank ? bank->stream : nullptr; }

int32_t clb_bank_last_timing(const clb_bank* bank, clb_timing_v1* out) {
    if (!bank || !out) return CLB_E_INVALID;
    *out = bank->last_timing;
    return CLB_OK;
}

int32_t clb_lane_config_parse(const char* text, clb_lane_config_v1* out, clb_error_v1* err) {
    return guarded(err, [&] {
        require(text && out, CLB_E_INVALID, "null lane config");
        clb_lane_config_v1 c{};
        std::set<std::string> seen;
        std::string all(text), line;
        size_t pos = 0;
        auto canonical_u64 = [](const std::string& v, uint64_t* r) {
            if (v.empty() || v.size() > 20) return false;
            for (char ch : v)
                if (ch < '0' || ch > '9') return false;
            errno = 0;
            const unsigned long long x = std::strtoull(v.c_str(), nullptr, 10);
            if (errno == ERANGE || std::to_string(x) != v) return false;
            *r = (uint64_t)x;
            return true;
        };
        while (pos <= all.size()) {
            const size_t nl = all.find('\n', pos);
            line = all.substr(pos, nl == std::string::npos ? std::string::npos : nl - pos);
            pos = nl == std::string::npos ? all.size() + 1 : nl + 1;
            if (line.empty() || line[0] == '#') continue;
            const size_t eq = line.find('=');
            require(eq != std::string::npos, CLB_E_INVALID, "lane config line without '=': %s", line.c_str());
            const std::string k = line.substr(0, eq), v = line.substr(eq + 1);
            require(seen.insert(k).second, CLB_E_INVALID, "duplicate lane config key: %s", k.c_str());
            if (k == "warm_cuda_experts") {
                require(v == "off" || v == "layer-batch-v1" || v == "stack-v1", CLB_E_INVALID,
                        "unknown warm_cuda_experts mode: %s", v.c_str());
                c.experts = v == "off" ? 0 : v == "layer-batch-v1" ? 1 : 2;
            } else if (k == "cuda_expert_math") {
                require(v == "fast-v1" || v == "cpu-q8k-v1", CLB_E_INVALID, "unknown cuda_expert_math: %s", v.c_str());
                c.exact_math = v == "cpu-q8k-v1";
            } else if (k == "warm_cuda_bytes") {
                require(canonical_u64(v, &c.bytes), CLB_E_INVALID, "invalid warm_cuda_bytes: %s", v.c_str());
            } else if (k == "cuda_devices") {
                const size_t dots = v.find("..");
                uint64_t a = 0, b = 0;
                const bool ok = dots == std::string::npos ? canonical_u64(v, &a) && (b = a, true)
                                                          : canonical_u64(v.substr(0, dots), &a) &&
                                                                canonical_u64(v.substr(dots + 2), &b);
                require(ok && a <= b && b < 64, CLB_E_INVALID, "cuda_devices must be a or a..b with a <= b < 64: %s",
                        v.c_str());
                c.device_first = (int32_t)a;
                c.device_last = (int32_t)b;
            } else if (k == "warm_cuda_timing") {
                require(v == "0" || v == "1", CLB_E_INVALID, "warm_cuda_timing must be 0 or 1");
                c.timing = v == "1";
            } else {
                throw Error(CLB_E_INVALID, "unknown lane config key: " + k);
            }
        }
        const bool lane_keys = seen.count("cuda_expert_math") || seen.count("warm_cuda_bytes") ||
                               seen.count("cuda_devices") || seen.count("warm_cuda_timing");
        require(c.experts != 0 || !lane_keys, CLB_E_INVALID,
                "cuda_expert_math, warm_cuda_bytes, cuda_devices and warm_cuda_timing need warm_cuda_experts on");
        c.bank_flags = (c.exact_math ? CLB_BANK_EXACT_ORDER : 0) | (c.experts == 1 ? CLB_BANK_PER_LAYER_KERNELS : 0) |
                       (c.timing ? CLB_BANK_TIMING : 0);
        *out = c;
    });
}

int32_t clb_bank_synchronize(clb_bank* bank, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        DeviceGuard g(bank->cfg.device);
        bank->device_step([&] { cuda_check(cudaStreamSynchronize(bank->stream), "sync"); });
    });
}

static void compute_rows(clb_bank* bank, uint32_t layer, const int32_t* ids, int32_t n, const float* x, float* y) {
    const auto& c = bank->cfg;
    require(x && y, CLB_E_INVALID, "null buffer");
    bank->validate_ids(layer, ids, n, true);
    require(finite_all(x, (size_t)c.dim), CLB_E_NONFINITE, "non-finite activation");
    DeviceGuard g(c.device);
    bank->timed_step("compute_many", (int)layer, 1, n, sizeof(float) * c.dim + (uint64_t)n * 4,
                     (uint64_t)n * c.dim * 4, [&] {
        std::memcpy(bank->h_x, x, sizeof(float) * c.dim);
        cuda_check(cudaMemcpyAsync(bank->d_x, bank->h_x, sizeof(float) * c.dim, cudaMemcpyHostToDevice, bank->stream),
                   "x H2D");
        cuda_check(cudaMemcpyAsync(bank->d_ids, ids, sizeof(int) * n, cudaMemcpyHostToDevice, bank->stream), "ids H2D");
        cuda_check(cudaMemsetAsync(bank->d_w, 0, sizeof(float) * n, bank->stream), "w memset");
        bank->enqueue_layer(layer, bank->d_ids, bank->d_w, n, bank->d_x, nullptr, nullptr, bank->d_out, bank->d_yrows,
                            bank->stream);
        cuda_check(cudaMemcpyAsync(bank->h_yrows, bank->d_yrows, sizeof(float) * (size_t)n * c.dim,
                                   cudaMemcpyDeviceToHost, bank->stream),
                   "rows D2H");
        bank->check_err_flag();
    });
    std::memcpy(y, bank->h_yrows, sizeof(float) * (size_t)n * c.dim);
    require(finite_all(y, (size_t)n * c.dim), CLB_E_NONFINITE, "non-finite expert output");
}

int32_t clb_bank_compute(clb_bank* bank, uint32_t layer, int32_t expert, const float* x, float* y,
                         clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        compute_rows(bank, layer, &expert, 1, x, y);
    });
}

int32_t clb_bank_compute_many(clb_bank* bank, uint32_t layer, const int32_t* ids, int32_t n, const float* x,
                              float* y, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        require(ids, CLB_E_INVALID, "null ids");
        compute_rows(bank, layer, ids, n, x, y);
    });
}

int32_t clb_layer_execute(clb_bank* bank, uint32_t layer, const int32_t* ids, const float* w, int32_t n,
                          const float* x, const float* shared, float* out, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(ids && w && x && out, CLB_E_INVALID, "null buffer");
        bank->validate_ids(layer, ids, n, true);
        require(finite_all(w, (size_t)n), CLB_E_NONFINITE, "non-finite route weight");
        require(finite_all(x, (size_t)c.dim), CLB_E_NONFINITE, "non-finite activation");
        require(!shared || finite_all(shared, (size_t)c.dim), CLB_E_NONFINITE, "non-finite shared output");
        DeviceGuard g(c.device);
        bank->timed_step("layer_execute", (int)layer, 1, n, sizeof(float) * c.dim * (shared ? 2 : 1) + (uint64_t)n * 8,
                         sizeof(float) * c.dim, [&] {
            std::memcpy(bank->h_x, x, sizeof(float) * c.dim);
            cuda_check(cudaMemcpyAsync(bank->d_x, bank->h_x, sizeof(float) * c.dim, cudaMemcpyHostToDevice,
                                       bank->stream),
                       "x H2D");
            if (shared)
                cuda_check(cudaMemcpyAsync(bank->d_shared, shared, sizeof(float) * c.dim, cudaMemcpyHostToDevice,
                                           bank->stream),
                           "shared H2D");
            cuda_check(cudaMemcpyAsync(bank->d_ids, ids, sizeof(int) * n, cudaMemcpyHostToDevice, bank->stream),
                       "ids H2D");
            cuda_check(cudaMemcpyAsync(bank->d_w, w, sizeof(float) * n, cudaMemcpyHostToDevice, bank->stream), "w H2D");
            bank->enqueue_layer(layer, bank->d_ids, bank->d_w, n, bank->d_x, shared ? bank->d_shared : nullptr,
                                nullptr, bank->d_out, nullptr, bank->stream);
            cuda_check(cudaMemcpyAsync(bank->h_out, bank->d_out, sizeof(float) * c.dim, cudaMemcpyDeviceToHost,
                                       bank->stream),
                       "out D2H");
            bank->check_err_flag();
        });
        std::memcpy(out, bank->h_out, sizeof(float) * c.dim);
        require(finite_all(out, (size_t)c.dim), CLB_E_NONFINITE, "non-finite layer output");
    });
}

int32_t clb_layer_forward_device(clb_bank* bank, uint32_t layer, const int32_t* d_ids, const float* d_w, int32_t n,
                                 const float* d_x, const float* d_shared, const float* d_resid, float* d_out,
                                 void* stream, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        require(layer < (uint32_t)bank->cfg.n_layers && n >= 1 && n <= bank->cfg.max_picks && d_ids && d_w && d_x &&
                    d_out,
                CLB_E_INVALID, "invalid device layer arguments");
        DeviceGuard g(bank->cfg.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] {
            bank->enqueue_layer(layer, d_ids, d_w, n, d_x, d_shared, d_resid, d_out, nullptr, s);
        });
    });
}

int32_t clb_layer_phases_device(clb_bank* bank, uint32_t layer, const int32_t* d_ids, const float* d_w, int32_t n,
                                const float* d_x, float* d_out, int32_t phase_mask, void* stream, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        require(layer < (uint32_t)bank->cfg.n_layers && n >= 1 && n <= bank->cfg.max_picks && d_ids && d_w && d_x &&
                    d_out && phase_mask > 0 && phase_mask < 16,
                CLB_E_INVALID, "invalid phase arguments");
        DeviceGuard g(bank->cfg.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] { bank->enqueue_phases(layer, d_ids, d_w, n, d_x, d_out, phase_mask, s); });
    });
}

int32_t clb_bank_expert_info(const clb_bank* bank, uint32_t layer, int32_t expert, int32_t* type,
                             uint64_t* payload_bytes) {
    if (!bank || !clb_bank_contains(bank, layer, expert)) return CLB_E_INVALID;
    const auto& d = bank->desc[(size_t)layer * bank->E() + (size_t)expert];
    const int t = d.gate.type;
    const uint64_t bb = (uint64_t)clb_block_bytes(t);
    const uint64_t gu = (uint64_t)d.gate.n * (uint64_t)(d.gate.k / 256) * bb;
    const uint64_t dn = (uint64_t)d.down.n * (uint64_t)(d.down.k / 256) * (uint64_t)clb_block_bytes(d.down.type);
    if (type) *type = t;
    if (payload_bytes) *payload_bytes = 2 * gu + dn;
    return CLB_OK;
}

int32_t clb_router_device(const float* d_x, int32_t tokens, int32_t dim, const float* d_gate_w, int32_t n_experts,
                          float* d_logits, void* stream) {
    if (!d_x || !d_gate_w || !d_logits || tokens <= 0 || dim <= 0 || dim % 4 != 0 || n_experts <= 0 ||
        n_experts > clb::kMaxExperts)
        return CLB_E_INVALID;
    return clb::launch_router_gemv(d_gate_w, d_x, n_experts, dim, tokens, d_logits,
                                   static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? CLB_OK
               : CLB_E_CUDA;
}

int32_t clb_route_b_device(const float* d_logits, const float* d_bias, int32_t n_experts, int32_t k, int32_t tokens,
                           float scale, int32_t* d_ids, float* d_w, int32_t* d_status, void* stream) {
    if (!d_logits || !d_bias || !d_ids || !d_w || !d_status || n_experts <= 0 || n_experts > clb::kMaxExperts ||
        k <= 0 || k > clb::kMaxPicks || k > n_experts || tokens <= 0 || !std::isfinite(scale) || scale < 0)
        return CLB_E_INVALID;
    return clb::launch_route_b(d_logits, d_bias, n_experts, k, tokens, scale, d_ids, d_w, d_status,
                               static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? CLB_OK
               : CLB_E_CUDA;
}

int32_t clb_moe_block_device(clb_bank* bank, uint32_t layer, const float* d_x, const float* d_gate_w,
                             const float* d_bias, float scale, const float* d_shared, const float* d_resid,
                             float* d_out, float* d_logits, int32_t* d_ids, float* d_w, void* stream,
                             clb_error_v1* err) {
    NvtxRange range("clb:moe_block_device");
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(layer < (uint32_t)c.n_layers && d_x && d_gate_w && d_bias && d_out && d_logits && d_ids && d_w,
                CLB_E_INVALID, "invalid MoE block arguments");
        require(std::isfinite(scale) && scale >= 0, CLB_E_INVALID, "route scale must be finite and >= 0");
        require(c.n_experts <= 1024, CLB_E_UNSUPPORTED, "device routing handles at most 1024 experts");
        DeviceGuard g(c.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] {
            // router logits, route_cpu's selection, the experts and the ascending-id combine:
            // one stream, no host round trip (the picks' residency is checked on the device)
            cuda_check(clb::launch_router_gemv(d_gate_w, d_x, c.n_experts, c.dim, 1, d_logits, s), "router");
            cuda_check(clb::launch_route_b(d_logits, d_bias, c.n_experts, c.max_picks, 1, scale, d_ids, d_w,
                                           bank->d_err, s),
                       "route");
            bank->enqueue_layer(layer, d_ids, d_w, c.max_picks, d_x, d_shared, d_resid, d_out, nullptr, s);
        });
    });
}

int32_t clb_route_device(int32_t mode, const float* d_logits, int32_t n_experts, int32_t k, int32_t tokens,
                         int32_t* d_ids, float* d_w, void* stream) {
    if (mode != 0 || !d_logits || !d_ids || !d_w || n_experts <= 0 || n_experts > clb::kMaxExperts || k <= 0 ||
        k > clb::kMaxPicks || k > n_experts || tokens <= 0)
        return CLB_E_INVALID;
    return clb::launch_route_sigmoid(d_logits, n_experts, k, tokens, d_ids, d_w, static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? CLB_OK
               : CLB_E_CUDA;
}

int32_t clb_route_host(int32_t mode, const float* logits, const float* bias, int32_t n, int32_t k, float scale,
                       int32_t* ids, float* w) {
    if (!logits || !ids || !w || n <= 0 || k <= 0 || k > n || k > 64) return CLB_E_INVALID;
    if (!finite_all(logits, (size_t)n)) return CLB_E_NONFINITE;
    if (mode == 0) {
        route_sigmoid_host(logits, n, k, ids, w);
        return CLB_OK;
    }
    if (mode != 1 || !bias) return CLB_E_INVALID;
    if (!finite_all(bias, (size_t)n) || !std::isfinite(scale) || scale < 0) return CLB_E_INVALID;
    std::vector<float> sc((size_t)n), bs((size_t)n);
    for (int e = 0; e < n; ++e) {
        const float l = logits[e];
        const float sp = l > 20.0f ? l : std::log1p(std::exp(l));
        sc[(size_t)e] = std::sqrt(sp);
        bs[(size_t)e] = sc[(size_t)e] + bias[e];
        if (!std::isfinite(bs[(size_t)e])) return CLB_E_NONFINITE;
    }
    float sum = 0.0f;
    for (int i = 0; i < k; ++i) {
        int best = 0;
        for (int e = 1; e < n; ++e)
            if (bs[(size_t)e] > bs[(size_t)best]) best = e;
        ids[i] = best;
        sum += sc[(size_t)best];
        bs[(size_t)best] = -std::numeric_limits<float>::max();
    }
    for (int i = 0; i < k; ++i) w[i] = sc[(size_t)ids[i]] / (sum + 1e-20f) * scale;
    return CLB_OK;
}

int32_t clb_stack_decode(clb_bank* bank, uint32_t first, int32_t nl, const float* x, const float* logits, float* out,
                         clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(x && logits && out, CLB_E_INVALID, "null buffer");
        require(nl >= 1 && first + (uint32_t)nl <= (uint32_t)c.n_layers, CLB_E_INVALID, "layer range out of bounds");
        require(bank->shard.world > 1 || (c.expert_begin == 0 && c.expert_end == c.n_experts), CLB_E_INVALID,
                "stack decode of a partial bank needs clb_bank_connect (expert-ID sharding over GPUs)");
        for (int l = 0; l < nl; ++l)
            for (int e = c.expert_begin; e < c.expert_end; ++e)
                require(bank->resident[(size_t)(first + l) * bank->E() + (size_t)e], CLB_E_INVALID,
                        "expert (%u, %d) not resident", first + l, e);
        DeviceGuard g(c.device);
        require(finite_all(logits, (size_t)nl * c.n_experts), CLB_E_NONFINITE, "non-finite router logits");
        bank->timed_step("stack_decode", (int)first, nl, nl * c.max_picks,
                         sizeof(float) * c.dim + (uint64_t)nl * c.max_picks * 8, sizeof(float) * c.dim, [&] {
            // Routing on the host (route.cpp's order and libm), then x and the routes go
            // up; one stack launch (or the captured per-layer graph) and h comes back.
            const int k = c.max_picks;
            std::memcpy(bank->h_x, x, sizeof(float) * c.dim);
            for (int l = 0; l < nl; ++l)
                route_sigmoid_host(logits + (size_t)l * c.n_experts, c.n_experts, k, bank->h_route_ids + (size_t)l * k,
                                   bank->h_route_w + (size_t)l * k);
            auto enqueue_all = [&] {
                cuda_check(cudaMemcpyAsync(bank->d_x, bank->h_x, sizeof(float) * c.dim, cudaMemcpyHostToDevice,
                                           bank->stream),
                           "x H2D");
                cuda_check(cudaMemcpyAsync(bank->d_route_ids, bank->h_route_ids, sizeof(int32_t) * (size_t)nl * k,
                                           cudaMemcpyHostToDevice, bank->stream),
                           "route ids H2D");
                cuda_check(cudaMemcpyAsync(bank->d_route_w, bank->h_route_w, sizeof(float) * (size_t)nl * k,
                                           cudaMemcpyHostToDevice, bank->stream),
                           "route weights H2D");
                bank->enqueue_stack(first, nl, bank->d_x, nullptr, bank->stream);
                cuda_check(cudaMemcpyAsync(bank->h_out, bank->d_x, sizeof(float) * c.dim, cudaMemcpyDeviceToHost,
                                           bank->stream),
                           "out D2H");
            };
            if (bank->persistent) {  // one kernel: no graph needed
                enqueue_all();
                bank->check_err_flag();
                return;
            }
            auto key = std::make_pair(first, nl);
            auto it = bank->graphs.find(key);
            if (it == bank->graphs.end()) {
                cudaGraph_t graph = nullptr;
                cuda_check(cudaStreamBeginCapture(bank->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
                try {
                    enqueue_all();
                } catch (...) {
                    cudaStreamEndCapture(bank->stream, &graph);
                    if (graph) cudaGraphDestroy(graph);
                    throw;
                }
                cuda_check(cudaStreamEndCapture(bank->stream, &graph), "end capture");
                cudaGraphExec_t exec = nullptr;
                cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
                cudaGraphDestroy(graph);
                cuda_check(e, "graph instantiate");
                it = bank->graphs.emplace(key, exec).first;
            }
            cuda_check(cudaGraphLaunch(it->second, bank->stream), "graph launch");
            bank->check_err_flag();
        });
        std::memcpy(out, bank->h_out, sizeof(float) * c.dim);
        require(finite_all(out, (size_t)c.dim), CLB_E_NONFINITE, "non-finite stack output");
    });
}

int32_t clb_stack_decode_device(clb_bank* bank, uint32_t first, int32_t nl, float* d_x, const float* d_logits,
                                clb_error_v1* err) {
    NvtxRange range("clb:stack_decode_device");
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(d_x && d_logits && nl >= 1 && first + (uint32_t)nl <= (uint32_t)c.n_layers, CLB_E_INVALID,
                "invalid stack arguments");
        require(bank->shard.world > 1 || (c.expert_begin == 0 && c.expert_end == c.n_experts), CLB_E_INVALID,
                "stack decode of a partial bank needs clb_bank_connect (expert-ID sharding over GPUs)");
        DeviceGuard g(c.device);
        bank->device_step([&] {
            if (bank->persistent) {
                bank->enqueue_stack(first, nl, d_x, d_logits, bank->stream);
                return;
            }
            // Graphs are keyed by layer range and bound to (d_x, d_logits) of their capture.
            auto key = std::make_pair(first, nl);
            auto it = bank->device_graphs.find(key);
            if (it != bank->device_graphs.end() && bank->graph_dx != d_x) {
                cudaGraphExecDestroy(it->second);
                bank->device_graphs.erase(it);
                it = bank->device_graphs.end();
            }
            if (it == bank->device_graphs.end()) {
                cudaGraph_t graph = nullptr;
                cuda_check(cudaStreamBeginCapture(bank->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
                try {
                    bank->enqueue_stack(first, nl, d_x, d_logits, bank->stream);
                } catch (...) {
                    cudaStreamEndCapture(bank->stream, &graph);
                    if (graph) cudaGraphDestroy(graph);
                    throw;
                }
                cuda_check(cudaStreamEndCapture(bank->stream, &graph), "end capture");
                cudaGraphExec_t exec = nullptr;
                cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
                cudaGraphDestroy(graph);
                cuda_check(e, "graph instantiate");
                it = bank->device_graphs.emplace(key, exec).first;
                bank->graph_dx = d_x;
            }
            cuda_check(cudaGraphLaunch(it->second, bank->stream), "graph launch");
        });
    });
}

// ---- batched prefill ----
static void prefill_check_layer(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k) {
    const auto& c = bank->cfg;
    require(layer < (uint32_t)c.n_layers, CLB_E_INVALID, "layer %u out of range", layer);
    require(tokens >= 1 && tokens <= (1 << 20) && k >= 1 && k <= c.max_picks && k <= c.n_experts &&
                (int64_t)tokens * k <= (1 << 24),
            CLB_E_INVALID, "invalid prefill size (%d tokens x %d picks)", tokens, k);
    require(clb::prefill_shape_supported(c.dim, c.ff), CLB_E_UNSUPPORTED, "prefill needs dim, ff multiples of 256");
}

uint64_t clb_prefill_workspace_bytes(const clb_bank* bank, int32_t tokens, int32_t k) {
    if (!bank || tokens < 1 || k < 1) return 0;
    return clb::prefill_workspace_bytes(tokens, k, bank->cfg.dim, bank->cfg.ff, bank->cfg.n_experts);
}

static int32_t prefill_device(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* d_ids,
                              const float* d_w, const float* d_x, const float* d_resid, float* d_out, void* d_ws,
                              uint64_t ws_bytes, int32_t phase_mask, void* stream, clb_error_v1* err) {
    NvtxRange range("clb:prefill_device");
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        prefill_check_layer(bank, layer, tokens, k);
        require(d_ids && d_w && d_x && d_out && d_ws, CLB_E_INVALID, "null device buffer");
        require(ws_bytes >= clb_prefill_workspace_bytes(bank, tokens, k), CLB_E_INVALID, "prefill workspace too small");
        require(phase_mask > 0 && phase_mask < 32, CLB_E_INVALID, "invalid phase mask");
        DeviceGuard g(bank->cfg.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] {
            const auto& c = bank->cfg;
            cuda_check(clb::launch_prefill(bank->d_desc + (size_t)layer * bank->E(), c.n_experts, d_x, d_ids, d_w,
                                           tokens, k, c.dim, c.ff, c.limit, d_resid, d_out, d_ws, bank->d_err,
                                           phase_mask, s, false, 0, -1, nullptr, bank->layer_types(layer)),
                       "prefill launch");
        });
    });
}

int32_t clb_prefill_layer_device(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* d_ids,
                                 const float* d_w, const float* d_x, const float* d_resid, float* d_out, void* d_ws,
                                 uint64_t ws_bytes, void* stream, clb_error_v1* err) {
    return prefill_device(bank, layer, tokens, k, d_ids, d_w, d_x, d_resid, d_out, d_ws, ws_bytes, 31, stream, err);
}

int32_t clb_prefill_phases_device(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* d_ids,
                                  const float* d_w, const float* d_x, float* d_out, void* d_ws, uint64_t ws_bytes,
                                  int32_t phase_mask, void* stream, clb_error_v1* err) {
    return prefill_device(bank, layer, tokens, k, d_ids, d_w, d_x, nullptr, d_out, d_ws, ws_bytes, phase_mask, stream,
                          err);
}

int32_t clb_prefill_reserve(clb_bank* bank, int32_t tokens, int32_t k, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(tokens >= 1 && k >= 1 && k <= c.max_picks, CLB_E_INVALID, "invalid prefill reservation");
        if (tokens <= bank->pf_tokens && k <= bank->pf_k) return;
        DeviceGuard g(c.device);
        cuda_check(cudaStreamSynchronize(bank->stream), "stream sync");
        const int T = std::max(tokens, bank->pf_tokens), K = std::max(k, bank->pf_k);
        bank->free_prefill();
        const size_t ws = clb::prefill_workspace_bytes(T, K, c.dim, c.ff, c.n_experts);
        auto dmal = [&](void** p, size_t n) {
            cudaError_t e = cudaMalloc(p, std::max<size_t>(n, 256));
            if (e != cudaSuccess) {
                cudaGetLastError();
                bank->free_prefill();
                throw Error(CLB_E_NOMEM, std::string("cudaMalloc (prefill): ") + cudaGetErrorString(e));
            }
        };
        dmal(&bank->pf_ws, ws);
        dmal(reinterpret_cast<void**>(&bank->pf_dx), (size_t)T * c.dim * 4);
        dmal(reinterpret_cast<void**>(&bank->pf_dout), (size_t)T * c.dim * 4);
        dmal(reinterpret_cast<void**>(&bank->pf_dw), (size_t)T * K * 4);
        dmal(reinterpret_cast<void**>(&bank->pf_dids), (size_t)T * K * 4);
        cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->pf_hx), (size_t)T * c.dim * 4), "cudaMallocHost");
        cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->pf_hw), (size_t)T * K * 4), "cudaMallocHost");
        cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->pf_hids), (size_t)T * K * 4), "cudaMallocHost");
        bank->pf_ws_bytes = ws;
        bank->pf_tokens = T;
        bank->pf_k = K;
    });
}

int32_t clb_prefill_layer(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* ids,
                          const float* w, const float* x, float* out, clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    if (tokens > bank->pf_tokens || k > bank->pf_k) {
        const int32_t rc = clb_prefill_reserve(bank, tokens, k, err);
        if (rc != CLB_OK) return rc;
    }
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        prefill_check_layer(bank, layer, tokens, k);
        require(ids && w && x && out, CLB_E_INVALID, "null buffer");
        for (int32_t t = 0; t < tokens; ++t) bank->validate_ids(layer, ids + (size_t)t * k, k, true);
        require(finite_all(w, (size_t)tokens * k), CLB_E_NONFINITE, "non-finite route weight");
        require(finite_all(x, (size_t)tokens * c.dim), CLB_E_NONFINITE, "non-finite activation");
        DeviceGuard g(c.device);
        const size_t nx = (size_t)tokens * c.dim, np = (size_t)tokens * k;
        bank->timed_step("prefill_layer", (int)layer, 1, (int)np, nx * 4 + np * 8, nx * 4, [&] {
            copy_parallel(bank->pf_hx, x, nx * 4);
            std::memcpy(bank->pf_hids, ids, np * 4);
            std::memcpy(bank->pf_hw, w, np * 4);
            cuda_check(cudaMemcpyAsync(bank->pf_dx, bank->pf_hx, nx * 4, cudaMemcpyHostToDevice, bank->stream), "x H2D");
            cuda_check(cudaMemcpyAsync(bank->pf_dids, bank->pf_hids, np * 4, cudaMemcpyHostToDevice, bank->stream),
                       "ids H2D");
            cuda_check(cudaMemcpyAsync(bank->pf_dw, bank->pf_hw, np * 4, cudaMemcpyHostToDevice, bank->stream), "w H2D");
            cuda_check(clb::launch_prefill(bank->d_desc + (size_t)layer * bank->E(), c.n_experts, bank->pf_dx,
                                           bank->pf_dids, bank->pf_dw, tokens, k, c.dim, c.ff, c.limit, nullptr,
                                           bank->pf_dout, bank->pf_ws, bank->d_err, 31, bank->stream, false, 0, -1,
                                           nullptr, bank->layer_types(layer)),
                       "prefill launch");
            cuda_check(cudaMemcpyAsync(bank->pf_hx, bank->pf_dout, nx * 4, cudaMemcpyDeviceToHost, bank->stream),
                       "out D2H");
            bank->check_err_flag();
        });
        copy_parallel(out, bank->pf_hx, nx * 4);
        require(finite_all(out, nx), CLB_E_NONFINITE, "non-finite prefill output");
    });
}

// ---- batched stack decode (T tokens through consecutive layers, grouped GEMMs per layer) ----
static void stack_batch_check(clb_bank* bank, uint32_t first, int32_t nl, int32_t tokens) {
    const auto& c = bank->cfg;
    require(nl >= 1 && first + (uint32_t)nl <= (uint32_t)c.n_layers, CLB_E_INVALID, "layer range out of bounds");
    require(tokens >= 1 && tokens <= (1 << 16) && (int64_t)tokens * c.max_picks <= (1 << 24), CLB_E_INVALID,
            "invalid batch size (%d tokens)", tokens);
    require(c.expert_begin == 0 && c.expert_end == c.n_experts, CLB_E_INVALID,
            "batched stack decode needs every expert of its layers on this bank");
    require(clb::prefill_shape_supported(c.dim, c.ff), CLB_E_UNSUPPORTED,
            "batched stack decode needs dim, ff multiples of 256 in [512, 8192]");
    for (int l = 0; l < nl; ++l)
        for (int e = 0; e < c.n_experts; ++e)
            require(bank->resident[(size_t)(first + l) * bank->E() + (size_t)e], CLB_E_INVALID,
                    "expert (%u, %d) not resident", first + l, e);
}

uint64_t clb_stack_batch_workspace_bytes(const clb_bank* bank, int32_t tokens) {
    if (!bank || tokens < 1) return 0;
    const auto& c = bank->cfg;
    return clb::stack_batch_workspace_bytes(tokens, c.max_picks, c.dim, c.ff, c.n_experts);
}

int32_t clb_stack_batch_device(clb_bank* bank, uint32_t first, int32_t nl, int32_t tokens, const float* d_logits,
                               float* d_h, void* d_ws, uint64_t ws_bytes, void* stream, clb_error_v1* err) {
    NvtxRange range("clb:stack_batch_device");
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        stack_batch_check(bank, first, nl, tokens);
        require(d_logits && d_h && d_ws, CLB_E_INVALID, "null device buffer");
        require(ws_bytes >= clb_stack_batch_workspace_bytes(bank, tokens), CLB_E_INVALID,
                "stack batch workspace too small");
        DeviceGuard g(bank->cfg.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] {
            const auto& c = bank->cfg;
            const std::vector<int> types = bank->layer_types(first, nl);
            cuda_check(clb::launch_stack_batch(bank->d_desc + (size_t)first * bank->E(), c.n_experts, nl, d_logits,
                                               nullptr, nullptr, d_h, tokens, c.max_picks, c.dim, c.ff, c.limit, d_ws,
                                               bank->d_err, s, types.data()),
                       "stack batch launch");
        });
    });
}

int32_t clb_stack_batch_layer_device(clb_bank* bank, uint32_t layer, int32_t tokens, const float* d_logits, float* d_h,
                                     float* d_rows, void* d_ws, uint64_t ws_bytes, int32_t phase_mask, void* stream,
                                     clb_error_v1* err) {
    NvtxRange range("clb:stack_batch_layer_device");
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        require(layer < (uint32_t)c.n_layers, CLB_E_INVALID, "layer %u out of range", layer);
        require(tokens >= 1 && tokens <= (1 << 16) && (int64_t)tokens * c.max_picks <= (1 << 24), CLB_E_INVALID,
                "invalid batch size (%d tokens)", tokens);
        require(clb::prefill_shape_supported(c.dim, c.ff), CLB_E_UNSUPPORTED,
                "batched stack decode needs dim, ff multiples of 256 in [512, 8192]");
        require(phase_mask >= 1 && phase_mask <= 3, CLB_E_INVALID, "invalid phase mask");
        require(d_logits && d_h && d_rows && d_ws, CLB_E_INVALID, "null device buffer");
        require(ws_bytes >= clb_stack_batch_workspace_bytes(bank, tokens), CLB_E_INVALID,
                "stack batch workspace too small");
        for (int e = c.expert_begin; e < c.expert_end; ++e)
            require(bank->resident[(size_t)layer * bank->E() + (size_t)e], CLB_E_INVALID, "expert (%u, %d) not resident",
                    layer, e);
        DeviceGuard g(c.device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : bank->stream;
        bank->device_step([&] {
            const int k = c.max_picks;
            int* ids = nullptr;
            float* w = nullptr;
            clb::stack_batch_routes(d_ws, tokens, k, c.dim, c.ff, c.n_experts, &ids, &w);
            const clb::ExpertDesc* desc = bank->d_desc + (size_t)layer * bank->E();
            if (phase_mask & 1) {  // route, RMSNorm + Q8_K, this bank's experts into d_rows
                cuda_check(clb::launch_route_sigmoid(d_logits, c.n_experts, k, tokens, ids, w, s), "route");
                cuda_check(clb::launch_prefill(desc, c.n_experts, d_h, ids, w, tokens, k, c.dim, c.ff, c.limit, d_h, d_h,
                                               d_ws, bank->d_err, 1 | 2 | 4 | 8, s, true, c.expert_begin, c.expert_end,
                                               d_rows, bank->layer_types(layer)),
                           "stack batch layer");
            }
            if (phase_mask & 2)  // h += ascending-id combine of every pick's row
                cuda_check(clb::launch_prefill(desc, c.n_experts, d_h, ids, w, tokens, k, c.dim, c.ff, c.limit, d_h, d_h,
                                               d_ws, bank->d_err, 16, s, true, c.expert_begin, c.expert_end, d_rows),
                           "stack batch combine");
        });
    });
}

int32_t clb_stack_batch(clb_bank* bank, uint32_t first, int32_t nl, int32_t tokens, const float* logits, float* h,
                        clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    std::lock_guard<std::mutex> lock(bank->call_mutex);
    return guarded(err, [&] {
        bank->check_usable();
        const auto& c = bank->cfg;
        stack_batch_check(bank, first, nl, tokens);
        require(logits && h, CLB_E_INVALID, "null buffer");
        const int k = c.max_picks;
        const size_t nh = (size_t)tokens * c.dim, nr = (size_t)nl * tokens * k;
        require(finite_all(logits, (size_t)nl * tokens * c.n_experts), CLB_E_NONFINITE, "non-finite router logits");
        require(finite_all(h, nh), CLB_E_NONFINITE, "non-finite activation");
        DeviceGuard g(c.device);
        if (tokens > bank->sb_tokens || nl > bank->sb_layers) {
            cuda_check(cudaStreamSynchronize(bank->stream), "stream sync");
            const int T = std::max(tokens, bank->sb_tokens), L = std::max(nl, bank->sb_layers);
            bank->free_stack_batch();
            auto dmal = [&](void** p, size_t n) {
                cudaError_t e = cudaMalloc(p, std::max<size_t>(n, 256));
                if (e != cudaSuccess) {
                    cudaGetLastError();
                    bank->free_stack_batch();
                    throw Error(CLB_E_NOMEM, std::string("cudaMalloc (stack batch): ") + cudaGetErrorString(e));
                }
            };
            const size_t R = (size_t)L * T * k;
            dmal(&bank->sb_ws, clb::stack_batch_workspace_bytes(T, k, c.dim, c.ff, c.n_experts));
            dmal(reinterpret_cast<void**>(&bank->sb_dh), (size_t)T * c.dim * 4);
            dmal(reinterpret_cast<void**>(&bank->sb_dw), R * 4);
            dmal(reinterpret_cast<void**>(&bank->sb_dids), R * 4);
            cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->sb_hh), (size_t)T * c.dim * 4), "cudaMallocHost");
            cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->sb_hw), R * 4), "cudaMallocHost");
            cuda_check(cudaMallocHost(reinterpret_cast<void**>(&bank->sb_hids), R * 4), "cudaMallocHost");
            bank->sb_tokens = T;
            bank->sb_layers = L;
        }
        bank->timed_step("stack_batch", (int)first, nl, (int)nr, nh * 4 + nr * 8, nh * 4, [&] {
            // routing on the host (route.cpp's order and libm, as clb_stack_decode), then h and
            // the routes go up, nl grouped layers run, and h comes back
            for (int l = 0; l < nl; ++l)
                for (int t = 0; t < tokens; ++t) {
                    const size_t r = ((size_t)l * tokens + t) * k;
                    route_sigmoid_host(logits + ((size_t)l * tokens + t) * c.n_experts, c.n_experts, k,
                                       bank->sb_hids + r, bank->sb_hw + r);
                }
            copy_parallel(bank->sb_hh, h, nh * 4);
            cuda_check(cudaMemcpyAsync(bank->sb_dh, bank->sb_hh, nh * 4, cudaMemcpyHostToDevice, bank->stream), "h H2D");
            cuda_check(cudaMemcpyAsync(bank->sb_dids, bank->sb_hids, nr * 4, cudaMemcpyHostToDevice, bank->stream),
                       "route ids H2D");
            cuda_check(cudaMemcpyAsync(bank->sb_dw, bank->sb_hw, nr * 4, cudaMemcpyHostToDevice, bank->stream),
                       "route weights H2D");
            const std::vector<int> types = bank->layer_types(first, nl);
            cuda_check(clb::launch_stack_batch(bank->d_desc + (size_t)first * bank->E(), c.n_experts, nl, nullptr,
                                               bank->sb_dids, bank->sb_dw, bank->sb_dh, tokens, k, c.dim, c.ff,
                                               c.limit, bank->sb_ws, bank->d_err, bank->stream, types.data()),
                       "stack batch launch");
            cuda_check(cudaMemcpyAsync(bank->sb_hh, bank->sb_dh, nh * 4, cudaMemcpyDeviceToHost, bank->stream),
                       "h D2H");
            bank->check_err_flag();
        });
        copy_parallel(h, bank->sb_hh, nh * 4);
        require(finite_all(h, nh), CLB_E_NONFINITE, "non-finite stack output");
    });
}

int32_t clb_warm_execute(clb_bank* bank, uint32_t layer, const int32_t* ids, const float* w, int32_t n,
                         const float* x, const float* shared, clb_host_expert_fn host_lane, void* host_ctx, float* out,
                         clb_error_v1* err) {
    if (!bank) return fail(err, CLB_E_INVALID, "null bank");
    return guarded(err, [&] {
        const auto& c = bank->cfg;
        require(ids && w && x && out && n >= 1 && n <= 64, CLB_E_INVALID, "invalid warm_execute arguments");
        require(layer < (uint32_t)c.n_layers, CLB_E_INVALID, "layer out of range");
        std::set<int> seen;
        for (int i = 0; i < n; ++i) {
            require(ids[i] >= 0 && ids[i] < c.n_experts && seen.insert(ids[i]).second && std::isfinite(w[i]),
                    CLB_E_INVALID, "invalid/duplicate route");
        }
        const size_t dim = (size_t)c.dim;
        std::vector<int> gpu_pick, host_pick;
        for (int i = 0; i < n; ++i) (clb_bank_contains(bank, layer, ids[i]) ? gpu_pick : host_pick).push_back(i);
        require(host_pick.empty() || host_lane, CLB_E_INVALID, "picks outside the bank but no host lane");
        require((int)gpu_pick.size() <= c.max_picks, CLB_E_INVALID, "more resident picks than the bank's max_picks");
        std::vector<float> rows((size_t)n * dim);
        // CUDA lane on a worker thread, host lane on the caller; both always joined.
        clb_error_v1 gpu_err{};
        int gpu_rc = CLB_OK;
        std::thread gpu([&] {
            if (gpu_pick.empty()) return;
            std::vector<int32_t> sel;
            for (int i : gpu_pick) sel.push_back(ids[i]);
            std::vector<float> y(sel.size() * dim);
            gpu_rc = clb_bank_compute_many(bank, layer, sel.data(), (int32_t)sel.size(), x, y.data(), &gpu_err);
            if (gpu_rc == CLB_OK)
                for (size_t j = 0; j < sel.size(); ++j)
                    std::memcpy(&rows[(size_t)gpu_pick[j] * dim], &y[j * dim], sizeof(float) * dim);
        });
        int host_rc = CLB_OK;
        std::string host_msg;
        for (int i : host_pick) {
            const int32_t rc = host_lane(host_ctx, layer, ids[i], x, c.dim, &rows[(size_t)i * dim]);
            if (rc != 0) {
                host_rc = CLB_E_LANE;
                host_msg = "host lane failed for expert " + std::to_string(ids[i]);
                break;
            }
            if (!finite_all(&rows[(size_t)i * dim], dim)) {
                host_rc = CLB_E_NONFINITE;
                host_msg = "host lane returned a non-finite row";
                break;
            }
        }
        gpu.join();
        if (gpu_rc != CLB_OK) throw Error(gpu_rc, std::string("CUDA lane: ") + gpu_err.message);
        if (host_rc != CLB_OK) throw Error(host_rc, host_msg);
        // Combine: ascending expert id, out = fmaf(w, y, out), then + shared (runtime.cpp:184-187).
        std::vector<int> order((size_t)n);
        for (int i = 0; i < n; ++i) order[(size_t)i] = i;
        std::sort(order.begin(), order.end(), [&](int a, int b) { return ids[a] < ids[b]; });
        std::vector<float> acc(dim, 0.0f);
        for (int i : order)
            for (size_t k = 0; k < dim; ++k) acc[k] = std::fma(w[i], rows[(size_t)i * dim + k], acc[k]);
        if (shared)
            for (size_t k = 0; k < dim; ++k) acc[k] += shared[k];
        std::memcpy(out, acc.data(), sizeof(float) * dim);
    });
}

}  // extern "C"
