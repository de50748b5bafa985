// sm_100a kernels of the routed-expert decode path. See clb_device.cuh for the
// arithmetic contract and clb_types.h for the packed weight layout.
#include <cuda_runtime.h>
#include <cfloat>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "clb_device.cuh"
#include "clb_kernels.h"
#include "clb_pack.h"
#include "iq_tables.h"

namespace clb {

// Nibble selector tables, derived once from the ggml codebooks (iq_tables.h).
__device__ uint32_t g_tables[kTableWords];

static uint32_t iq2_symbols(uint64_t grid) {
    uint32_t v = 0;
    for (int j = 0; j < 8; ++j) {
        const uint32_t m = (uint32_t)((grid >> (8 * j)) & 255u);
        const uint32_t s = m == 8 ? 0u : m == 25 ? 1u : 2u;  // 43
        v |= s << (4 * j);
    }
    return v;
}
static uint32_t iq1_symbols(uint64_t grid) {
    uint32_t v = 0;
    for (int j = 0; j < 8; ++j) {
        const int8_t m = (int8_t)(uint8_t)((grid >> (8 * j)) & 255u);
        const uint32_t s = (uint32_t)(m + 1);  // -1,0,1 -> 0,1,2
        v |= s << (4 * j);
    }
    return v;
}

void host_tables(uint32_t* out) {
    for (int i = 0; i < 256; ++i) out[kTabXXS + i] = iq2_symbols(clb_iq2xxs_grid[i]);
    for (int i = 0; i < 512; ++i) out[kTabXS + i] = iq2_symbols(clb_iq2xs_grid[i]);
    for (int i = 0; i < 2048; ++i) out[kTabIQ1 + i] = iq1_symbols(clb_iq1s_grid[i]);
    for (int s = 0; s < 128; ++s) {
        const uint32_t v = (uint32_t)s | ((uint32_t)__builtin_parity((unsigned)s) << 7);  // ksigns_iq2xs
        uint32_t nib = 0;
        for (int j = 0; j < 8; ++j)
            if (v & (1u << j)) nib |= 4u << (4 * j);
        out[kTabSign + s] = nib;
    }
}

cudaError_t upload_tables(cudaStream_t stream) {
    // filled once (threads setting up different devices share the read-only copy)
    static uint32_t host[kTableWords];
    static std::once_flag filled;
    std::call_once(filled, [] { host_tables(host); });
    cudaError_t e = cudaMemcpyToSymbolAsync(g_tables, host, sizeof(host), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

// Device address of the selector tables, for kernels compiled in other translation units.
cudaError_t tables_device_ptr(const uint32_t** out) {
    return cudaGetSymbolAddress(reinterpret_cast<void**>(const_cast<uint32_t**>(out)), g_tables);
}

__device__ __forceinline__ Tables load_tables(uint32_t* smem) {
    for (int i = threadIdx.x; i < kTableWords; i += blockDim.x) smem[i] = g_tables[i];
    Tables tb;
    tb.xxs = smem + kTabXXS;
    tb.xs = smem + kTabXS;
    tb.iq1 = smem + kTabIQ1;
    tb.sign = smem + kTabSign;
    return tb;
}

// ------------------------------------------------------------------------------
// Q8_K quantisation: one warp per 256-value block.
__global__ void __launch_bounds__(128) k_quant(const float* __restrict__ x, int nblocks, int8_t* __restrict__ qs,
                                               float* __restrict__ d) {
    const int b = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    warp_quant_block(x + (size_t)b * 256, qs + (size_t)b * 256, d + b, nullptr);
}

// Q8_K quantisation into crosslane's 292-byte block struct (d @0, qs @4, bsums @260).
__global__ void __launch_bounds__(128) k_quant_blocks(const float* __restrict__ x, int nblocks,
                                                      uint8_t* __restrict__ out) {
    const int b = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    __shared__ __align__(16) int8_t qs[4][256];
    __shared__ float dd[4];
    __shared__ int16_t bs[4][16];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    warp_quant_block(x + (size_t)b * 256, qs[w], &dd[w], bs[w]);
    __syncwarp();
    uint8_t* blk = out + (size_t)b * kQ8KBlockBytes;
    if (lane == 0) *reinterpret_cast<float*>(blk) = dd[w];
    for (int i = lane; i < 64; i += 32) reinterpret_cast<uint32_t*>(blk + 4)[i] = reinterpret_cast<uint32_t*>(qs[w])[i];
    if (lane < 16) reinterpret_cast<int16_t*>(blk + 260)[lane] = bs[w][lane];
}

// ------------------------------------------------------------------------------
// Stack pre-norm fused with Q8_K: x = h * (float)(1 / sqrt(mean(h^2) + 1e-6)), then
// Q8_K(x). One CTA of 1024 threads; the fp64 sum of squares has a fixed order so
// the CPU oracle reproduces it bit for bit: lane t sums (double)h[t + 1024 j]^2 over
// j in order, then lanes combine in a binary tree (stride 512, 256, ..., 1).
__global__ void __launch_bounds__(1024) k_norm_quant(const float* __restrict__ h, int dim, int8_t* __restrict__ qs,
                                                     float* __restrict__ d, float* __restrict__ xnorm) {
    __shared__ double part[1024];
    __shared__ float scale_s;
    const int t = threadIdx.x;
    double s = 0.0;
    for (int i = t; i < dim; i += 1024) {
        const double v = (double)h[i];
        s = __dadd_rn(s, __dmul_rn(v, v));
    }
    part[t] = s;
    __syncthreads();
    for (int stride = 512; stride > 0; stride >>= 1) {
        if (t < stride) part[t] = __dadd_rn(part[t], part[t + stride]);
        __syncthreads();
    }
    if (t == 0) {
        const double mean = __ddiv_rn(part[0], (double)dim);
        scale_s = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(mean, 1e-6)));
    }
    __syncthreads();
    const float sc = scale_s;
    extern __shared__ __align__(16) float xs[];
    for (int i = t; i < dim; i += 1024) {
        const float v = __fmul_rn(h[i], sc);
        xs[i] = v;
        if (xnorm) xnorm[i] = v;
    }
    __syncthreads();
    for (int b = t >> 5; b < (dim >> 8); b += 32) warp_quant_block(xs + (size_t)b * 256, qs + (size_t)b * 256, d + b, nullptr);
}

// ------------------------------------------------------------------------------
// y[n] = W . Q8_K(x) for one packed matrix; q is crosslane's 292-byte block array.
// CTA: 4 warps x 16 rows.
__global__ void __launch_bounds__(128) k_mv(PackedMat m, const uint8_t* __restrict__ q, float* __restrict__ y) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    const int nb = m.k >> 8;
    int8_t* aqs = reinterpret_cast<int8_t*>(smem + kTableWords * 4);
    float* ad = reinterpret_cast<float*>(smem + kTableWords * 4 + (size_t)m.k);
    const Tables tb = load_tables(tab);
    for (int i = threadIdx.x; i < nb * 64; i += blockDim.x) {
        const int b = i >> 6, w = i & 63;
        reinterpret_cast<uint32_t*>(aqs)[i] =
            *reinterpret_cast<const uint32_t*>(q + (size_t)b * kQ8KBlockBytes + 4 + 4 * w);
    }
    for (int b = threadIdx.x; b < nb; b += blockDim.x) ad[b] = *reinterpret_cast<const float*>(q + (size_t)b * kQ8KBlockBytes);
    __syncthreads();
    const int r0 = (blockIdx.x * 4 + (threadIdx.x >> 5)) * 16;
    if (r0 >= m.n) return;
    float out[2];
    tile_dot_any(m, r0, ActView{aqs, ad}, tb, out);
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    if (t == 0) {
        if (r0 + g < m.n) y[r0 + g] = out[0];
        if (r0 + g + 8 < m.n) y[r0 + g + 8] = out[1];
    }
}

__global__ void k_activate(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ h, int n,
                           float limit) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = swiglu(g[i], u[i], limit);
}

// ------------------------------------------------------------------------------
// Fused gate + up + SwiGLU for all picks of a layer.
// blockIdx.x = pick * tiles + tile; a CTA covers 64 hidden rows of one pick:
// warps 0-3 gate rows, warps 4-7 the same up rows. h[pick][row] = swiglu(g, u).
__global__ void __launch_bounds__(256) k_gateup(const ExpertDesc* __restrict__ experts, const int* __restrict__ ids,
                                                const int8_t* __restrict__ xqs, const float* __restrict__ xd, int dim,
                                                int ff, float limit, float* __restrict__ h, int* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    int8_t* aqs = reinterpret_cast<int8_t*>(smem + kTableWords * 4);
    float* ad = reinterpret_cast<float*>(smem + kTableWords * 4 + (size_t)dim);
    float* gu = ad + (dim >> 8);  // [2][64]
    const int tiles = (ff + 63) >> 6;
    const int pick = blockIdx.x / tiles, tile = blockIdx.x % tiles;
    const int e = ids[pick];
    const Tables tb = load_tables(tab);
    for (int i = threadIdx.x; i < (dim >> 2); i += blockDim.x)
        reinterpret_cast<uint32_t*>(aqs)[i] = reinterpret_cast<const uint32_t*>(xqs)[i];
    for (int b = threadIdx.x; b < (dim >> 8); b += blockDim.x) ad[b] = xd[b];
    __syncthreads();
    const ExpertDesc& ex = experts[e];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const PackedMat& m = warp < 4 ? ex.gate : ex.up;
    const bool valid = m.body != nullptr && m.k == dim && m.n == ff;
    if (!valid && lane == 0) atomicExch(err, 1);
    const int r0 = tile * 64 + (warp & 3) * 16;
    float out[2] = {0.0f, 0.0f};
    if (valid && r0 < ff) tile_dot_any(m, r0, ActView{aqs, ad}, tb, out);
    if (t == 0) {
        gu[(warp >> 2) * 64 + (warp & 3) * 16 + g] = out[0];
        gu[(warp >> 2) * 64 + (warp & 3) * 16 + g + 8] = out[1];
    }
    __syncthreads();
    if (threadIdx.x < 64) {
        const int row = tile * 64 + threadIdx.x;
        if (row < ff) h[(size_t)pick * ff + row] = swiglu(gu[threadIdx.x], gu[64 + threadIdx.x], limit);
    }
}

// ------------------------------------------------------------------------------
// Fused down projection + fixed-order combine for one 16-row output tile.
// Warp p computes y_p = down_p . Q8_K(h_p) for the tile; then
//   out = fma over picks in ascending expert id (w_i, y_i) [runtime.cpp:184-187],
//   out = out + shared (if given), x_next = resid + out (if resid given).
// y_rows (optional) receives the per-pick rows [pick][dim].
__global__ void __launch_bounds__(512) k_down_combine(const ExpertDesc* __restrict__ experts, const int* __restrict__ ids,
                                                      const float* __restrict__ wts, int npick,
                                                      const int8_t* __restrict__ hqs, const float* __restrict__ hd,
                                                      int dim, int ff, const float* __restrict__ shared,
                                                      const float* __restrict__ resid, float* __restrict__ out,
                                                      float* __restrict__ y_rows, int* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    int8_t* aqs = reinterpret_cast<int8_t*>(smem + kTableWords * 4);          // [npick][ff]
    float* ad = reinterpret_cast<float*>(smem + kTableWords * 4 + (size_t)npick * ff);  // [npick][ff/256]
    float* ys = ad + npick * (ff >> 8);                                        // [npick][16]
    const Tables tb = load_tables(tab);
    const int nqw = (npick * ff) >> 2;
    for (int i = threadIdx.x; i < nqw; i += blockDim.x)
        reinterpret_cast<uint32_t*>(aqs)[i] = reinterpret_cast<const uint32_t*>(hqs)[i];
    for (int i = threadIdx.x; i < npick * (ff >> 8); i += blockDim.x) ad[i] = hd[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int r0 = blockIdx.x * 16;
    if (warp < npick) {
        const PackedMat& m = experts[ids[warp]].down;
        if (m.body == nullptr || m.k != ff || m.n != dim) {
            if (lane == 0) atomicExch(err, 1);
            for (int i = lane; i < 16; i += 32) ys[warp * 16 + i] = 0.0f;
        } else {
            float y[2];
            tile_dot_any(m, r0, ActView{aqs + (size_t)warp * ff, ad + warp * (ff >> 8)}, tb, y);
            if (t == 0) {
                ys[warp * 16 + g] = y[0];
                ys[warp * 16 + g + 8] = y[1];
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        const int row = r0 + threadIdx.x;
        if (row < dim) {
            // ascending expert id; ids are unique (validated on the host or by routing)
            float acc = 0.0f;
            int last = -1;
            for (int o = 0; o < npick; ++o) {
                int best = -1;
                for (int p = 0; p < npick; ++p)
                    if (ids[p] > last && (best < 0 || ids[p] < ids[best])) best = p;
                if (best < 0) break;  // duplicate ids never reach here (validated); stay in bounds anyway
                last = ids[best];
                acc = __fmaf_rn(wts[best], ys[best * 16 + threadIdx.x], acc);
            }
            if (shared) acc = __fadd_rn(acc, shared[row]);
            if (resid) acc = __fadd_rn(resid[row], acc);
            out[row] = acc;
            if (y_rows)
                for (int p = 0; p < npick; ++p) y_rows[(size_t)p * dim + row] = ys[p * 16 + threadIdx.x];
        }
    }
}

// ------------------------------------------------------------------------------
// Routing mode A for `tokens` rows of logits: top-k by logit (ties to the lower id),
// w_i = sigmoid(l_i) / sum of the selected sigmoids taken in selection order.
__global__ void k_route_sigmoid(const float* __restrict__ logits, int n, int k, int tokens, int* __restrict__ ids,
                                float* __restrict__ w) {
    const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= tokens) return;
    const int lane = threadIdx.x & 31;
    const float* l = logits + (size_t)tok * n;
    uint32_t chosen[kMaxExperts / 32];
    for (int i = 0; i < kMaxExperts / 32; ++i) chosen[i] = 0;
    float s[kMaxPicks];
    float sum = 0.0f;
    int sel[kMaxPicks];
    for (int i = 0; i < k; ++i) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < n; e += 32) {
            if ((chosen[e >> 5] >> (e & 31)) & 1u) continue;
            const float v = l[e];
            if (bi == 0x7fffffff || v > best || (v == best && e < bi)) { best = v; bi = e; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ob > best || (ob == best && oi < bi))) { best = ob; bi = oi; }
        }
        chosen[bi >> 5] |= 1u << (bi & 31);
        sel[i] = bi;
        // exp evaluated in double and rounded once: the correctly rounded float, which is
        // what glibc's expf returns for all but ~0.06% of arguments (there 1 ulp apart)
        s[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)best)));
        sum = __fadd_rn(sum, s[i]);
    }
    if (lane == 0)
        for (int i = 0; i < k; ++i) {
            ids[(size_t)tok * k + i] = sel[i];
            w[(size_t)tok * k + i] = __fdiv_rn(s[i], sum);
        }
}

// ------------------------------------------------------------------------------
// Router logits on the device: logits[t][e] = gate_w[e] . x[t] in fp32, one warp per
// (token, expert): lane j accumulates float4 groups j, j + 32, ... with fused multiply-adds
// in order, then a butterfly sum over the lanes (fixed order: run-to-run identical).
__global__ void __launch_bounds__(256) k_router_gemv(const float* __restrict__ gw, const float* __restrict__ x, int n,
                                                     int dim, int tokens, float* __restrict__ logits) {
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (item >= n * tokens) return;
    const int t = item / n, e = item - t * n;
    const float4* wr = reinterpret_cast<const float4*>(gw + (size_t)e * dim);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * dim);
    float acc = 0.0f;
    for (int i = lane; i < (dim >> 2); i += 32) {
        const float4 a = __ldg(wr + i), v = __ldg(xr + i);
        acc = __fmaf_rn(a.x, v.x, acc);
        acc = __fmaf_rn(a.y, v.y, acc);
        acc = __fmaf_rn(a.z, v.z, acc);
        acc = __fmaf_rn(a.w, v.w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) logits[(size_t)t * n + e] = acc;
}

// Mode-B routing on the device (crosslane route_cpu, engine/strata/sycl/route/route.cpp:15-37):
// sc = sqrt(softplus(l)) with softplus(l) = l above 20, else log1p(exp(l)) as two float
// roundings (exp and log1p evaluated in double and rounded once each: the correctly rounded
// float results); selection by sc + bias, largest first, ties to the lower id; sum of the
// picks' sc in selection order; w = sc / (sum + 1e-20) * scale. One CTA per token, one
// thread per expert (n <= 1024). A non-finite score sets *err = 1.
__global__ void __launch_bounds__(1024) k_route_b(const float* __restrict__ logits, const float* __restrict__ bias, int n,
                                                  int k, float scale, int* __restrict__ ids, float* __restrict__ w,
                                                  int* __restrict__ err) {
    __shared__ float scs[1024];
    __shared__ float wbest[32];
    __shared__ int wi[32];
    __shared__ int pick[kMaxPicks];
    const int t = blockIdx.x, e = threadIdx.x, lane = e & 31, warp = e >> 5;
    float sc = 0.0f, bs = -FLT_MAX;
    if (e < n) {
        const float l = logits[(size_t)t * n + e];
        const float sp = l > 20.0f ? l : (float)log1p((double)(float)exp((double)l));
        sc = __fsqrt_rn(sp);
        bs = __fadd_rn(sc, bias[e]);
        if (!isfinite(bs)) atomicExch(err, 1);
        scs[e] = sc;
    }
    for (int i = 0; i < k; ++i) {
        float v = e < n ? bs : -INFINITY;
        int vi = e < n ? e : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, vi, o);
            if (ov > v || (ov == v && oi < vi)) v = ov, vi = oi;
        }
        if (lane == 0) wbest[warp] = v, wi[warp] = vi;
        __syncthreads();
        if (warp == 0) {
            const int nw = (blockDim.x + 31) >> 5;
            v = lane < nw ? wbest[lane] : -INFINITY;
            vi = lane < nw ? wi[lane] : 0x7fffffff;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, vi, o);
                if (ov > v || (ov == v && oi < vi)) v = ov, vi = oi;
            }
            if (lane == 0) pick[i] = vi;
        }
        __syncthreads();
        if (e == pick[i]) bs = -FLT_MAX;  // the host marks a chosen expert with the lowest float
    }
    if (e == 0) {
        float sum = 0.0f;
        for (int i = 0; i < k; ++i) sum = __fadd_rn(sum, scs[pick[i]]);
        const float den = __fadd_rn(sum, 1e-20f);
        for (int i = 0; i < k; ++i) {
            ids[(size_t)t * k + i] = pick[i];
            w[(size_t)t * k + i] = __fmul_rn(__fdiv_rn(scs[pick[i]], den), scale);
        }
    }
}

// ------------------------------------------------------------------------------
// Synthetic fill: one thread per ggml block, written straight into the packed layout.
__global__ void k_synth_fill(uint8_t* __restrict__ packed, PackedLayout l, int type, int n, int k, uint64_t seed,
                             uint32_t layer, uint32_t expert, uint32_t role, const uint16_t* __restrict__ scales) {
    const int nb = k >> 8;
    const size_t total = (size_t)n * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        uint8_t blk[80];
        clb_synth_block(type, clb_block_key(seed, layer, expert, role, (uint64_t)i), scales, blk);
        const int r = (int)(i / nb), b = (int)(i % nb);
        clb_pack_block(type, n, nb, r, b, blk, packed, l);
    }
}

// ggml AoS matrix -> packed layout; flags a non-finite fp16 super-scale.
__global__ void k_pack(const uint8_t* __restrict__ aos, uint8_t* __restrict__ packed, PackedLayout l, int type, int n,
                       int k, int* __restrict__ bad) {
    const int nb = k >> 8;
    const int bytes = clb_block_bytes(type);
    const size_t total = (size_t)n * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint8_t* src = aos + i * bytes;
        if ((clb_block_half(type, src) & 0x7c00u) == 0x7c00u) atomicExch(bad, 1);
        clb_pack_block(type, n, nb, (int)(i / nb), (int)(i % nb), src, packed, l);
    }
}

// ------------------------------------------------------------------------------
// Launch helpers.
size_t mv_smem(int k) { return kTableWords * 4 + (size_t)k + (size_t)(k >> 8) * 4 + 16; }
size_t gateup_smem(int dim) { return kTableWords * 4 + (size_t)dim + (size_t)(dim >> 8) * 4 + 2 * 64 * 4 + 16; }
size_t down_smem(int npick, int ff) {
    return kTableWords * 4 + (size_t)npick * ff + (size_t)npick * (ff >> 8) * 4 + (size_t)npick * 16 * 4 + 16;
}

cudaError_t set_smem_limits() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_mv, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024))) return e;
    if ((e = cudaFuncSetAttribute(k_norm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024))) return e;
    if ((e = cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024))) return e;
    if ((e = cudaFuncSetAttribute(k_down_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024))) return e;
    return cudaSuccess;
}

cudaError_t launch_quant(const float* x, int nblocks, int8_t* qs, float* d, cudaStream_t s) {
    k_quant<<<(nblocks + 3) / 4, 128, 0, s>>>(x, nblocks, qs, d);
    return cudaGetLastError();
}
cudaError_t launch_quant_blocks(const float* x, int nblocks, void* out, cudaStream_t s) {
    k_quant_blocks<<<(nblocks + 3) / 4, 128, 0, s>>>(x, nblocks, static_cast<uint8_t*>(out));
    return cudaGetLastError();
}
cudaError_t launch_norm_quant(const float* h, int dim, int8_t* qs, float* d, float* xnorm, cudaStream_t s) {
    k_norm_quant<<<1, 1024, (size_t)dim * 4, s>>>(h, dim, qs, d, xnorm);
    return cudaGetLastError();
}
cudaError_t launch_mv(const PackedMat& m, const void* q, float* y, cudaStream_t s) {
    k_mv<<<(m.n + 63) / 64, 128, mv_smem(m.k), s>>>(m, static_cast<const uint8_t*>(q), y);
    return cudaGetLastError();
}
cudaError_t launch_activate(const float* g, const float* u, float* h, int n, float limit, cudaStream_t s) {
    k_activate<<<(n + 255) / 256, 256, 0, s>>>(g, u, h, n, limit);
    return cudaGetLastError();
}
cudaError_t launch_gateup(const ExpertDesc* experts, const int* ids, int npick, const int8_t* xqs, const float* xd,
                          int dim, int ff, float limit, float* h, int* err, cudaStream_t s) {
    const int tiles = (ff + 63) / 64;
    k_gateup<<<npick * tiles, 256, gateup_smem(dim), s>>>(experts, ids, xqs, xd, dim, ff, limit, h, err);
    return cudaGetLastError();
}
cudaError_t launch_down_combine(const ExpertDesc* experts, const int* ids, const float* w, int npick,
                                const int8_t* hqs, const float* hd, int dim, int ff, const float* shared,
                                const float* resid, float* out, float* y_rows, int* err, cudaStream_t s) {
    k_down_combine<<<(dim + 15) / 16, 32 * npick, down_smem(npick, ff), s>>>(experts, ids, w, npick, hqs, hd, dim, ff,
                                                                          shared, resid, out, y_rows, err);
    return cudaGetLastError();
}
cudaError_t launch_route_sigmoid(const float* logits, int n, int k, int tokens, int* ids, float* w, cudaStream_t s) {
    k_route_sigmoid<<<(tokens + 3) / 4, 128, 0, s>>>(logits, n, k, tokens, ids, w);
    return cudaGetLastError();
}
cudaError_t launch_router_gemv(const float* gate_w, const float* x, int n, int dim, int tokens, float* logits,
                               cudaStream_t s) {
    k_router_gemv<<<(n * tokens + 7) / 8, 256, 0, s>>>(gate_w, x, n, dim, tokens, logits);
    return cudaGetLastError();
}
cudaError_t launch_route_b(const float* logits, const float* bias, int n, int k, int tokens, float scale, int* ids,
                           float* w, int* err, cudaStream_t s) {
    k_route_b<<<tokens, (n + 31) / 32 * 32, 0, s>>>(logits, bias, n, k, scale, ids, w, err);
    return cudaGetLastError();
}
cudaError_t launch_synth_fill(uint8_t* packed, const PackedLayout& l, int type, int n, int k, uint64_t seed,
                              uint32_t layer, uint32_t expert, uint32_t role, const uint16_t* scales, cudaStream_t s) {
    const size_t total = (size_t)n * (k >> 8);
    const int grid = (int)((total + 255) / 256 < 148 * 32 ? (total + 255) / 256 : 148 * 32);
    k_synth_fill<<<grid, 256, 0, s>>>(packed, l, type, n, k, seed, layer, expert, role, scales);
    return cudaGetLastError();
}
cudaError_t launch_pack(const uint8_t* aos, uint8_t* packed, const PackedLayout& l, int type, int n, int k, int* bad,
                        cudaStream_t s) {
    const size_t total = (size_t)n * (k >> 8);
    const int grid = (int)((total + 255) / 256 < 148 * 32 ? (total + 255) / 256 : 148 * 32);
    k_pack<<<grid, 256, 0, s>>>(aos, packed, l, type, n, k, bad);
    return cudaGetLastError();
}

}  // namespace clb

// ==============================================================================
// v2: row-per-thread decode (clb_rowdot.cuh), persistent CTAs, fused epilogues.
// ==============================================================================
#include "clb_v2.cuh"

namespace clb {

// ------------------------------------------------------------------------------
// Gate + up for all picks (one warp item = 8 rows of one matrix of one pick), then,
// in the last warp to finish each 256-row block of a pick, SwiGLU and Q8_K(h).
template <int MAXT, bool PF, bool FAST>
__global__ void __launch_bounds__(MAXT, 1)
    k_gateup2(const ExpertDesc* __restrict__ experts, const int* __restrict__ ids, int npick,
              const int8_t* __restrict__ xqs, const float* __restrict__ xd, int dim, int ff, float limit,
              float* __restrict__ gu, int8_t* __restrict__ hqs, float* __restrict__ hd, int* __restrict__ counters,
              int* __restrict__ err) {
    uint8_t* smem = clb_dyn_smem;
    const int nbx = dim >> 8;
    int8_t* aq = reinterpret_cast<int8_t*>(smem + kRowTableBytes);
    float* ad = reinterpret_cast<float*>(smem + kRowTableBytes + (size_t)nbx * kActStride);
    uint32_t* xch_all = reinterpret_cast<uint32_t*>(smem + kRowTableBytes + (size_t)nbx * kActStride + 4 * nbx);
    fill_row_tables(g_tables, xch_all);  // the exchange area doubles as the staging area
    stage_act(xqs, xd, nbx, aq, ad);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    uint32_t* xch = xch_all + warp * 32 * kXchWords;
    const int groups = ff >> 3;                       // 8-row groups per matrix
    const int items = npick * 2 * groups;
    const int hblocks = ff >> 8;
    for (int it = blockIdx.x * nwarps + warp; it < items; it += gridDim.x * nwarps) {
        const int pick = it / (2 * groups), rem = it % (2 * groups);
        const int group = rem >> 1, mat = rem & 1;       // gate/up of the same rows are adjacent
        const ExpertDesc& ex = experts[ids[pick]];
        const PackedMat& m = mat ? ex.up : ex.gate;
        const int row = group * 8 + (lane >> 2);
        float y = 0.0f;
        if (m.body != nullptr && m.k == dim && m.n == ff)
            y = FAST ? seg_row_dot_any<PF>(m, row, 4, aq, ad) : quad_row_dot_any<PF>(m, row, aq, ad, xch);
        else if (lane == 0) atomicExch(err, 1);
        if ((lane & 3) == 0) gu[((size_t)pick * 2 + mat) * ff + row] = y;
        // last arriver of this (pick, 256-row block) applies SwiGLU and quantises h
        __threadfence();
        __syncwarp();
        int last = 0;
        const int ci = pick * hblocks + (group >> 5);
        if (lane == 0) last = atomicAdd(&counters[ci], 1) == 63;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            const int hb = group >> 5;
            const float* g = gu + ((size_t)pick * 2) * ff + hb * 256;
            const float* u = gu + ((size_t)pick * 2 + 1) * ff + hb * 256;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = swiglu(__ldcg(g + lane * 8 + i), __ldcg(u + lane * 8 + i), limit);
            warp_quant_regs(v, hqs + (size_t)pick * ff + hb * 256, hd + pick * hblocks + hb);
            if (lane == 0) counters[ci] = 0;
        }
    }
}

// ------------------------------------------------------------------------------
// Down projection (one warp item = 32 rows of one pick, one thread per row), then, in
// the last warp to finish each 32-row group, the ascending-id fma combine
// (runtime.cpp:184-187), + shared, + residual.
template <int MAXT, bool PF, bool FAST>
__global__ void __launch_bounds__(MAXT, 1)
    k_down2(const ExpertDesc* __restrict__ experts, const int* __restrict__ ids, const float* __restrict__ wts, int npick,
            const int8_t* __restrict__ hqs, const float* __restrict__ hd, int dim, int ff,
            const float* __restrict__ shared, const float* __restrict__ resid, float* __restrict__ out,
            float* __restrict__ yrows, int* __restrict__ counters, int* __restrict__ err) {
    uint8_t* smem = clb_dyn_smem;
    const int nbh = ff >> 8;
    int8_t* aq = reinterpret_cast<int8_t*>(smem + kRowTableBytes);
    float* ad = reinterpret_cast<float*>(smem + kRowTableBytes + (size_t)npick * nbh * kActStride);
    fill_row_tables(g_tables, reinterpret_cast<uint32_t*>(ad + npick * nbh + 4));
    stage_act(hqs, hd, npick * nbh, aq, ad);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    // exact: one thread per row, 32 rows per item; fast: 2 threads per row, 16 rows
    constexpr int RPI = FAST ? 16 : 32;
    const int groups = (dim + RPI - 1) / RPI;
    const int items = npick * groups;
    for (int it = blockIdx.x * nwarps + warp; it < items; it += gridDim.x * nwarps) {
        const int group = it / npick, pick = it % npick;
        const PackedMat& m = experts[ids[pick]].down;
        const int row = group * RPI + (FAST ? lane >> 1 : lane);
        const int rowc = row < dim ? row : dim - 1;
        float y = 0.0f;
        if (m.body != nullptr && m.k == ff && m.n == dim)
            y = FAST ? seg_row_dot_any<PF>(m, rowc, 2, aq + (size_t)pick * nbh * kActStride, ad + pick * nbh)
                     : thread_row_dot_any<PF>(m, rowc, aq + (size_t)pick * nbh * kActStride, ad + pick * nbh);
        else if (lane == 0) atomicExch(err, 1);
        if (row < dim && (!FAST || (lane & 1) == 0)) yrows[(size_t)pick * dim + row] = y;
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&counters[group], 1) == npick - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last && row < dim && (!FAST || (lane & 1) == 0)) {
            __threadfence();
            float acc = 0.0f;
            int prev = -1;
            for (int o = 0; o < npick; ++o) {
                int best = -1;
                for (int p = 0; p < npick; ++p)
                    if (ids[p] > prev && (best < 0 || ids[p] < ids[best])) best = p;
                if (best < 0) break;
                prev = ids[best];
                acc = __fmaf_rn(wts[best], __ldcg(yrows + (size_t)best * dim + row), acc);
            }
            if (shared) acc = __fadd_rn(acc, shared[row]);
            if (resid) acc = __fadd_rn(resid[row], acc);
            out[row] = acc;
        }
        if (last && lane == 0) counters[group] = 0;
    }
}

// ------------------------------------------------------------------------------
// y[n] = W . q for one packed matrix (crosslane q8k::Block input), one thread per row.
__global__ void __launch_bounds__(kV2Threads, 1) k_mv2(PackedMat m, const uint8_t* __restrict__ q, float* __restrict__ y) {
    uint8_t* smem = clb_dyn_smem;
    const int nb = m.k >> 8;
    int8_t* aq = reinterpret_cast<int8_t*>(smem + kRowTableBytes);
    float* ad = reinterpret_cast<float*>(smem + kRowTableBytes + (size_t)nb * kActStride);
    fill_row_tables(g_tables, reinterpret_cast<uint32_t*>(ad + nb + 4));
    for (int i = threadIdx.x; i < nb * 64; i += blockDim.x) {
        const int b = i >> 6, w = i & 63;
        reinterpret_cast<uint32_t*>(aq + (size_t)b * kActStride)[w] =
            *reinterpret_cast<const uint32_t*>(q + (size_t)b * kQ8KBlockBytes + 4 + 4 * w);
    }
    for (int b = threadIdx.x; b < nb; b += blockDim.x) ad[b] = *reinterpret_cast<const float*>(q + (size_t)b * kQ8KBlockBytes);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int groups = (m.n + 31) >> 5;
    for (int g = blockIdx.x * nwarps + warp; g < groups; g += gridDim.x * nwarps) {
        const int row = g * 32 + lane;
        const float v = thread_row_dot_any<true>(m, row < m.n ? row : m.n - 1, aq, ad);
        if (row < m.n) y[row] = v;
    }
}

// The exchange area doubles as the 2944-word staging buffer of fill_row_tables, so it
// is never smaller than that, whatever the warp count.
size_t gateup2_smem(int dim, int warps) {
    size_t xch_words = (size_t)warps * 32 * kXchWords;
    if (xch_words < 2944) xch_words = 2944;
    return kRowTableBytes + (size_t)(dim >> 8) * kActStride + 4 * (size_t)(dim >> 8) + xch_words * 4 + 16;
}
size_t down2_smem(int npick, int ff) {
    return kRowTableBytes + (size_t)npick * (ff >> 8) * (kActStride + 4) + 16 + 2944 * 4;
}
size_t mv2_smem(int k) { return kRowTableBytes + (size_t)(k >> 8) * (kActStride + 4) + 16 + 2944 * 4; }

static int g_num_sms = 0;
static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

// One CTA per SM with just enough warps (<= max_warps) that every SM gets a share of
// the warp items; items per warp stay within one of each other.
static void spread(int items, int max_warps, int& grid, int& threads) {
    const int sms = num_sms();
    int warps = (items + sms - 1) / sms;
    warps = warps < 1 ? 1 : warps > max_warps ? max_warps : warps;
    grid = (items + warps - 1) / warps;
    if (grid > sms) grid = sms;
    threads = 32 * warps;
}

// Occupancy / prefetch variant of the v2 decode kernels, chosen once per process from
// CLB_V2_VARIANT (a tuning knob; every variant of a summation order computes identical
// results): 0 = 512 threads with register prefetch of the next block;
// 1 = 512 threads with L2 prefetch (default); 2 = 1024 threads with L2 prefetch.
static int v2_variant() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("CLB_V2_VARIANT");
        v = e ? atoi(e) : 1;
        if (v < 0 || v > 2) v = 1;
    }
    return v;
}
static int v2_max_threads() { return v2_variant() == 2 ? 1024 : 512; }

// The most dynamic shared memory the kernel can be launched with: the per-block opt-in
// limit less the kernel's static shared memory (the decode's prmt byte tables).
template <typename K>
static cudaError_t allow_smem(K kernel) {
    int dev = 0, optin = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) || (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)))
        return e;
    cudaFuncAttributes a{};
    if ((e = cudaFuncGetAttributes(&a, kernel))) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)a.sharedSizeBytes);
}
cudaError_t set_v2_smem_limits() {
    cudaError_t e;
    if ((e = allow_smem(k_gateup2<512, true, false>))) return e;
    if ((e = allow_smem(k_gateup2<512, false, false>))) return e;
    if ((e = allow_smem(k_gateup2<1024, false, false>))) return e;
    if ((e = allow_smem(k_gateup2<512, false, true>))) return e;
    if ((e = allow_smem(k_gateup2<512, true, true>))) return e;
    if ((e = allow_smem(k_gateup2<1024, false, true>))) return e;
    if ((e = allow_smem(k_down2<512, true, false>))) return e;
    if ((e = allow_smem(k_down2<512, false, false>))) return e;
    if ((e = allow_smem(k_down2<1024, false, false>))) return e;
    if ((e = allow_smem(k_down2<512, false, true>))) return e;
    if ((e = allow_smem(k_down2<512, true, true>))) return e;
    if ((e = allow_smem(k_down2<1024, false, true>))) return e;
    return allow_smem(k_mv2);
}

cudaError_t launch_gateup2(const ExpertDesc* experts, const int* ids, int npick, const int8_t* xqs, const float* xd,
                           int dim, int ff, float limit, float* gu, int8_t* hqs, float* hd, int* counters, int* err,
                           bool fast, cudaStream_t s) {
    const int items = npick * 2 * (ff >> 3);
    int grid, threads;
    spread(items, v2_max_threads() / 32, grid, threads);
    const size_t sm = gateup2_smem(dim, threads / 32);
#define CLB_GU_ARGS experts, ids, npick, xqs, xd, dim, ff, limit, gu, hqs, hd, counters, err
    const int v = v2_variant();
    if (fast) {
        if (v == 0) k_gateup2<512, true, true><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
        else if (v == 2) k_gateup2<1024, false, true><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
        else k_gateup2<512, false, true><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
    } else {
        if (v == 0) k_gateup2<512, true, false><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
        else if (v == 2) k_gateup2<1024, false, false><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
        else k_gateup2<512, false, false><<<grid, threads, sm, s>>>(CLB_GU_ARGS);
    }
#undef CLB_GU_ARGS
    return cudaGetLastError();
}
cudaError_t launch_down2(const ExpertDesc* experts, const int* ids, const float* w, int npick, const int8_t* hqs,
                         const float* hd, int dim, int ff, const float* shared, const float* resid, float* out,
                         float* yrows, int* counters, int* err, bool fast, cudaStream_t s) {
    const int items = npick * (fast ? (dim + 15) >> 4 : (dim + 31) >> 5);
    int grid, threads;
    spread(items, v2_max_threads() / 32, grid, threads);
    const size_t sm = down2_smem(npick, ff);
#define CLB_DN_ARGS experts, ids, w, npick, hqs, hd, dim, ff, shared, resid, out, yrows, counters, err
    const int v = v2_variant();
    if (fast) {
        if (v == 0) k_down2<512, true, true><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
        else if (v == 2) k_down2<1024, false, true><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
        else k_down2<512, false, true><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
    } else {
        if (v == 0) k_down2<512, true, false><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
        else if (v == 2) k_down2<1024, false, false><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
        else k_down2<512, false, false><<<grid, threads, sm, s>>>(CLB_DN_ARGS);
    }
#undef CLB_DN_ARGS
    return cudaGetLastError();
}
cudaError_t launch_mv2(const PackedMat& m, const void* q, float* y, cudaStream_t s) {
    const int groups = (m.n + 31) >> 5;
    int grid, threads;
    spread(groups, kV2Warps, grid, threads);
    k_mv2<<<grid, threads, mv2_smem(m.k), s>>>(m, static_cast<const uint8_t*>(q), y);
    return cudaGetLastError();
}

}  // namespace clb
