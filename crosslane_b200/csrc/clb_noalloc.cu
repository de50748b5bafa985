// One expert FFN for callers that cannot allocate device memory.
//
// Some callers of this lane cannot call cudaMalloc: a serving loop that must not risk the
// implicit device synchronisation an allocation can cause, or a plugin whose process hands
// all device memory to another allocator (a pool it does not control). They
// bring their own weights, input and output buffers; this entry point supplies the only
// other memory it needs -- the quantised input, the hidden vector and its quantisation --
// from one fixed array compiled into the library. Every GPU that loads the library holds
// that array (kNoAllocScratchBytes) until the process exits.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "../../include/crosslane_b200.h"
#include "clb_device.cuh"
#include "clb_kernels.h"

namespace {

// Largest shapes the fixed scratch covers.
constexpr int kNoAllocMaxDim = 16384;
constexpr int kNoAllocMaxFF = 8192;
// Scratch layout (256-byte aligned pieces): Q8_K(x) qs [dim] | Q8_K(x) d [dim/256] |
// h [ff] floats | Q8_K(h) qs [ff] | Q8_K(h) d [ff/256].
constexpr size_t kOffXqs = 0;
constexpr size_t kOffXd = kOffXqs + kNoAllocMaxDim;
constexpr size_t kOffH = kOffXd + 256;
constexpr size_t kOffHqs = kOffH + 4 * (size_t)kNoAllocMaxFF;
constexpr size_t kOffHd = kOffHqs + kNoAllocMaxFF;
constexpr size_t kNoAllocScratchBytes = kOffHd + 256;  // 57,856 bytes
static_assert(kNoAllocScratchBytes == 57856, "the documented size of the fixed scratch array");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
uint8_t* g_scratch_ptr[kMaxDevices] = {};
const uint32_t* g_tables_ptr[kMaxDevices] = {};

int set_error(clb_error_v1* err, int code, const char* msg) {
    if (err) {
        err->code = code;
        std::snprintf(err->message, sizeof err->message, "%s", msg);
    }
    return code;
}

__device__ __forceinline__ clb::Tables tables_from(const uint32_t* g, uint32_t* smem) {
    for (int i = threadIdx.x; i < clb::kTableWords; i += blockDim.x) smem[i] = g[i];
    clb::Tables tb;
    tb.xxs = smem + clb::kTabXXS;
    tb.xs = smem + clb::kTabXS;
    tb.iq1 = smem + clb::kTabIQ1;
    tb.sign = smem + clb::kTabSign;
    return tb;
}

// Variant of k_gateup for one expert whose matrices arrive by value: 64 hidden rows per
// CTA, warps 0-3 gate, 4-7 up, h = swiglu(g, u) written to the scratch.
__global__ void __launch_bounds__(256) k_gateup_noalloc(PackedMat gate, PackedMat up, const uint32_t* __restrict__ tables,
                                                        uint8_t* __restrict__ scratch, int dim, int ff, float limit) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    int8_t* aqs = reinterpret_cast<int8_t*>(smem + clb::kTableWords * 4);
    float* ad = reinterpret_cast<float*>(smem + clb::kTableWords * 4 + (size_t)dim);
    float* gu = ad + (dim >> 8);
    const clb::Tables tb = tables_from(tables, tab);
    const int8_t* xqs = reinterpret_cast<const int8_t*>(scratch + kOffXqs);
    const float* xd = reinterpret_cast<const float*>(scratch + kOffXd);
    float* h = reinterpret_cast<float*>(scratch + kOffH);
    for (int i = threadIdx.x; i < (dim >> 2); i += blockDim.x)
        reinterpret_cast<uint32_t*>(aqs)[i] = reinterpret_cast<const uint32_t*>(xqs)[i];
    for (int b = threadIdx.x; b < (dim >> 8); b += blockDim.x) ad[b] = xd[b];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const PackedMat& m = warp < 4 ? gate : up;
    const int r0 = blockIdx.x * 64 + (warp & 3) * 16;
    float out[2] = {0.0f, 0.0f};
    if (r0 < ff) clb::tile_dot_any(m, r0, clb::ActView{aqs, ad}, tb, out);
    if (t == 0) {
        gu[(warp >> 2) * 64 + (warp & 3) * 16 + g] = out[0];
        gu[(warp >> 2) * 64 + (warp & 3) * 16 + g + 8] = out[1];
    }
    __syncthreads();
    if (threadIdx.x < 64) {
        const int row = blockIdx.x * 64 + threadIdx.x;
        if (row < ff) h[row] = clb::swiglu(gu[threadIdx.x], gu[64 + threadIdx.x], limit);
    }
}

// Variant of the down projection for one expert: y[dim] from Q8_K(h) in the scratch.
__global__ void __launch_bounds__(128) k_down_noalloc(PackedMat down, const uint32_t* __restrict__ tables,
                                                      const uint8_t* __restrict__ scratch, int ff, float* __restrict__ y) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    int8_t* aqs = reinterpret_cast<int8_t*>(smem + clb::kTableWords * 4);
    float* ad = reinterpret_cast<float*>(smem + clb::kTableWords * 4 + (size_t)ff);
    const clb::Tables tb = tables_from(tables, tab);
    const int8_t* hqs = reinterpret_cast<const int8_t*>(scratch + kOffHqs);
    const float* hd = reinterpret_cast<const float*>(scratch + kOffHd);
    for (int i = threadIdx.x; i < (ff >> 2); i += blockDim.x)
        reinterpret_cast<uint32_t*>(aqs)[i] = reinterpret_cast<const uint32_t*>(hqs)[i];
    for (int b = threadIdx.x; b < (ff >> 8); b += blockDim.x) ad[b] = hd[b];
    __syncthreads();
    const int r0 = (blockIdx.x * 4 + (threadIdx.x >> 5)) * 16;
    if (r0 >= down.n) return;
    float out[2];
    clb::tile_dot_any(down, r0, clb::ActView{aqs, ad}, tb, out);
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    if (t == 0) {
        if (r0 + g < down.n) y[r0 + g] = out[0];
        if (r0 + g + 8 < down.n) y[r0 + g + 8] = out[1];
    }
}

PackedMat view(int type, const void* w, int n, int k) {
    const PackedLayout l = clb_packed_layout(type, n, k);
    const uint8_t* base = static_cast<const uint8_t*>(w);
    PackedMat m{};
    m.body = base + l.body;
    m.sc = base + l.sc;
    m.d = reinterpret_cast<const uint16_t*>(base + l.d);
    m.type = type;
    m.n = n;
    m.k = k;
    return m;
}

// Once per device, with that device current: resolve the scratch array's device
// address, make sure the decode tables are resident and allow the kernels' shared memory.
int setup_device(int dev, cudaStream_t stream, clb_error_v1* err) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[dev]) return CLB_OK;
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return set_error(err, CLB_E_CUDA, cudaGetErrorString(e));
    const uint32_t* tables = nullptr;
    if ((e = clb::tables_device_ptr(&tables)) != cudaSuccess || (e = clb::upload_tables(stream)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(k_gateup_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024)) !=
            cudaSuccess ||
        (e = cudaFuncSetAttribute(k_down_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024)) !=
            cudaSuccess)
        return set_error(err, CLB_E_CUDA, cudaGetErrorString(e));
    g_tables_ptr[dev] = tables;
    g_scratch_ptr[dev] = static_cast<uint8_t*>(ptr);
    return CLB_OK;
}

}  // namespace

extern "C" int32_t clb_expert_forward_noalloc(int32_t type, const void* w_gate, const void* w_up, const void* w_down,
                                              const float* x, float* y, int32_t dim, int32_t ff, float limit,
                                              void* stream, clb_error_v1* err) {
    if (!clb_type_supported(type)) return set_error(err, CLB_E_UNSUPPORTED, "quant type has no kernel");
    if (!w_gate || !w_up || !w_down || !x || !y) return set_error(err, CLB_E_INVALID, "null pointer argument");
    if (dim <= 0 || ff <= 0 || dim % 256 || ff % 256)
        return set_error(err, CLB_E_INVALID, "dim and ff must be positive multiples of 256");
    if (dim > kNoAllocMaxDim || ff > kNoAllocMaxFF)
        return set_error(err, CLB_E_UNSUPPORTED,
                         "shape exceeds the fixed no-alloc scratch: dim <= 16384 and ff <= 8192");
    if (!std::isfinite(limit) || limit < 0) return set_error(err, CLB_E_INVALID, "SwiGLU limit must be finite, >= 0");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(err, CLB_E_CUDA, "no current CUDA device");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rc = setup_device(dev, s, err);
    if (rc != CLB_OK) return rc;
    uint8_t* scratch = g_scratch_ptr[dev];
    const uint32_t* tables = g_tables_ptr[dev];
    const PackedMat gate = view(type, w_gate, ff, dim), up = view(type, w_up, ff, dim), down = view(type, w_down, dim, ff);
    cudaError_t e = clb::launch_quant(x, dim / 256, reinterpret_cast<int8_t*>(scratch + kOffXqs),
                                      reinterpret_cast<float*>(scratch + kOffXd), s);
    if (e == cudaSuccess) {
        const size_t sm = clb::kTableWords * 4 + (size_t)dim + (size_t)(dim >> 8) * 4 + 2 * 64 * 4 + 16;
        k_gateup_noalloc<<<(ff + 63) / 64, 256, sm, s>>>(gate, up, tables, scratch, dim, ff, limit);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = clb::launch_quant(reinterpret_cast<const float*>(scratch + kOffH), ff / 256,
                              reinterpret_cast<int8_t*>(scratch + kOffHqs), reinterpret_cast<float*>(scratch + kOffHd), s);
    if (e == cudaSuccess) {
        const size_t sm = clb::kTableWords * 4 + (size_t)ff + (size_t)(ff >> 8) * 4 + 16;
        k_down_noalloc<<<(dim + 63) / 64, 128, sm, s>>>(down, tables, scratch, ff, y);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return set_error(err, CLB_E_CUDA, cudaGetErrorString(e));
    if (err) {
        err->code = CLB_OK;
        err->message[0] = 0;
    }
    return CLB_OK;
}
