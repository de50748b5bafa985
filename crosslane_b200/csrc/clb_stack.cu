// Persistent whole-stack decode kernel: one CTA per SM runs every layer of a token, so
// the tables are staged once per token and no kernel launch or prologue sits between the
// phases.
//
// Fast summation order, per layer l (ids/w = the routing of layer l, fixed before the
// launch), one grid barrier per layer:
//   1. every CTA: h (h_in, or the previous layer's combine in global memory) and its
//      per-32-row-group sums of squares; x = RMSNorm(h) (fixed-order total), Q8_K(x) into
//      shared memory;
//   2. gate/up rows of every pick in CTA rounds (K segments per warp, added in order,
//      rows decoded with lane_row_roll), SwiGLU -> gu; each 32-row group counts its 256-row
//      block with a release add (no round trip on the producer side);
//   3. each CTA waits for (only) the blocks of the picks its down rounds touch, quantizes
//      each block's SwiGLU output to Q8_K(h) in shared memory itself, and decodes its down
//      rounds -> expert rows (also into every peer's slot of a sharded bank); one GPU: each
//      row group counts its rows; sharded: each CTA counts itself after one system-scope
//      fence, and the last CTA of the GPU publishes the layer number to every peer;
//   4. the owner warp of each 32-row group waits for the rows of all k picks (sharded: for
//      every local CTA and every peer's flag) and applies h += the ascending-id fma combine
//      (runtime.cpp:184-187), writing h and its sum of squares for the next layer (the last
//      layer: h_out);
//   -- grid barrier --
// Exact order (q8k_core's arithmetic, bit-identical to the CPU lane), per layer:
//   1. every CTA: h += ascending-id fma combine of the previous layer's expert rows,
//      x = RMSNorm(h) (fixed-order fp64 sum of squares, as k_norm_quant), Q8_K(x);
//   2. gate/up rows of every pick (4 threads per row) -> gu;   -- grid barrier --
//   3. every CTA serves one pick in the down phase: SwiGLU + Q8_K(h) of that pick into
//      shared memory, then its share of the pick's down rows -> yrows;   -- grid barrier --
// After the last layer the combine is applied once more and written to h_out.
#include <cuda_runtime.h>

#include "clb_device.cuh"
#include "clb_kernels.h"
#include "clb_sync.cuh"
#include "clb_v2.cuh"

namespace clb {

#ifdef CLB_FLOW_TRACE
// Phase stamps of the stack kernel per (layer, CTA), a build-time option (%globaltimer ns;
// python crosslane_b200/build.py --trace). Fast order: 0 layer start, 1 h and its sums of
// squares loaded, 2 RMSNorm + Q8_K(x) done, 3 = 4 gate/up rounds done, 5 Q8_K(h) staged,
// 6 down rounds done (sharded: and the CTA's signal), 7 combine + grid barrier passed.
// Exact order: 1 combine done, 2 norm done, 3 gate/up done, 4 first barrier passed, 5
// Q8_K(h) staged, 6 down rows done, 7 second barrier passed.
constexpr int kStTraceLayers = 64, kStTraceCtas = 160, kStTraceSlots = 8;
__device__ unsigned long long g_stack_trace[kStTraceLayers * kStTraceCtas * kStTraceSlots];
__device__ __forceinline__ void stack_stamp(int li, int slot) {
    if (threadIdx.x == 0 && li < kStTraceLayers && blockIdx.x < kStTraceCtas) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_stack_trace[(li * kStTraceCtas + blockIdx.x) * kStTraceSlots + slot] = t;
    }
}
#define STACK_STAMP(li, slot) stack_stamp((li), (slot))
#else
#define STACK_STAMP(li, slot) do { } while (0)
#endif


namespace {

constexpr int kErrBarrier = 2;                     // err flag value of a timed-out barrier or wait
constexpr unsigned kBlockReady = 8;                 // block counter: its 8 row groups of SwiGLU output stored

// Grid-wide barrier over gridDim.x co-resident CTAs (cooperative launch) on a counter
// that only grows: barrier number e (1, 2, ...) is passed once the counter reaches
// e * gridDim.x. Thread 0 of each CTA arrives with a release add (the CTA's writes,
// ordered before it by the preceding __syncthreads, become visible first) and polls
// with acquire loads. Bounded: after `limit` polls the CTA sets *err and
// every thread of it gets false, so the kernel can return instead of hanging.
// `overlap` runs on the threads other than thread 0 while thread 0 waits (work that needs
// no other CTA's results, e.g. staging the next layer's routing).
template <class F>
__device__ bool grid_barrier(unsigned* count, unsigned epoch, int* err, unsigned limit, F&& overlap) {
    __syncthreads();
    int ok = 1;
    if (threadIdx.x != 0) overlap();
    if (threadIdx.x == 0) {
        const unsigned target = epoch * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(count), "r"(1u) : "memory");
        unsigned v = 0, spins = 0;
        while (true) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
            if ((int)(v - target) >= 0) break;
            if (++spins > limit) {
                atomicExch(err, kErrBarrier);
                ok = 0;
                break;
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}
__device__ bool grid_barrier(unsigned* count, unsigned epoch, int* err, unsigned limit) {
    return grid_barrier(count, epoch, err, limit, [] {});
}

// At the end of a layer's down phase every CTA tells every peer that its part of this GPU's
// rows is in place: the CTA barrier orders its threads' peer stores before thread 0's
// system-scope release add on the peer's flag for this rank (the release is cumulative over
// the writes the barrier made it observe). No per-thread system fence.
__device__ void signal_peers(const StackShard& sh) {
    __syncthreads();
    if (threadIdx.x == 0)
        for (int r = 0; r < sh.world; ++r)
            if (r != sh.rank)
                asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(sh.peer_flags[r] + sh.rank), "r"(1u)
                             : "memory");
}

// After the grid barrier that ends a layer: every CTA waits until every peer's CTAs have
// signalled their rows of this layer (signal_peers). Flags only grow, by gridDim.x per layer
// (every GPU runs the same grid): layer li of the launch with `epoch` layers before it is
// complete at (epoch + li + 1) * gridDim.x, compared modulo 2^32. Bounded like grid_barrier.
__device__ bool exchange_rows(const StackShard& sh, int li, int* err, unsigned limit) {
    int ok = 1;
    if (threadIdx.x == 0) {
        const unsigned target = (sh.epoch + (unsigned)li + 1u) * gridDim.x;
        for (int r = 0; r < sh.world && ok; ++r) {
            if (r == sh.rank) continue;
            unsigned v = 0, spins = 0;
            while (true) {
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(sh.flags + r) : "memory");
                if ((int)(v - target) >= 0) break;
                if (++spins > limit) {
                    atomicExch(err, kErrBarrier);
                    ok = 0;
                    break;
                }
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// K segments of the fast-order phases for `kown` picks on `grid` CTAs of `nw` warps, chosen
// to minimise the blocks one thread decodes (CTA rounds x blocks per segment; the smaller
// count on ties). gate/up: SG divides nw / 2, a round = nw / (2 SG) row groups of 32 rows x 2
// matrices x SG segments. down: SD in {1, 2, 3, 4, 6, 8}, a round = nw / SD (pick, row
// group) pairs x SD segments (nw % SD warps idle). Every thread evaluates the same expression.
__host__ __device__ inline int gateup_segments(int kown, int ff, int nb, int grid, int nw) {
    int best = 1;
    long best_cost = -1;
    const int choices[8] = {1, 2, 3, 4, 6, 8, 12, 16};
    for (int i = 0; i < 8; ++i) {
        const int SG = choices[i];
        if ((nw / 2) % SG != 0) continue;
        const int rgr = nw / 2 / SG;
        const long rounds = ((long)kown * (ff / 32) + rgr - 1) / rgr;
        const long cost = (rounds + grid - 1) / grid * ((nb + SG - 1) / SG);
        if (best_cost < 0 || cost < best_cost) best_cost = cost, best = SG;
    }
    return best;
}
__host__ __device__ inline int down_segments(int kown, int dim, int nb, int grid, int nw) {
    int best = 1;
    long best_cost = -1;
    const int choices[6] = {1, 2, 3, 4, 6, 8};
    for (int i = 0; i < 6; ++i) {
        const int SD = choices[i];
        const int ppr = nw / SD;
        if (ppr < 1) continue;
        const long rounds = ((long)kown * (dim / 32) + ppr - 1) / ppr;
        const long cost = (rounds + grid - 1) / grid * ((nb + SD - 1) / SD);
        if (best_cost < 0 || cost < best_cost) best_cost = cost, best = SD;
    }
    return best;
}

// First CTA of pick p when gridDim.x CTAs are split over k picks (CTA c serves pick
// c * k / gridDim.x).
__device__ __forceinline__ int pick_cta_begin(int p, int k) { return (p * (int)gridDim.x + k - 1) / k; }

}  // namespace

struct StackParams {
    const ExpertDesc* desc;  // [bank layers][E]
    int E, first, nl, k;
    const int* route_ids;    // [nl][k]
    const float* route_w;    // [nl][k]
    const float* h_in;       // dim
    float* h_out;            // dim (may alias h_in)
    int dim, ff;
    float limit;
    float* gu;               // [k][2][ff]
    float* yrows;            // [k][dim]
    unsigned* bar;           // grid barrier counter, zero before the launch
    int* err;
    unsigned wait_limit;     // polls before a bounded wait gives up
    const uint32_t* tables;  // compact selector tables (kTableWords)
    StackShard sh;           // expert-ID sharding over GPUs (world == 1: none)
    StackWork w;             // fast order: h between layers, Q8_K(h), block counters
};

// Shared memory carve-up (bytes), shared by the kernel and the host size query.
// nt: threads per CTA.
struct StackSmem {
    size_t h, xq, xd, hq, hd, desc, ids, w, order, own, tree, xch, total;
    // Every region starts on a 16-byte boundary (the activation blocks are read as uint4).
    static __host__ __device__ size_t up16(size_t o) { return (o + 15) & ~(size_t)15; }
    __host__ __device__ StackSmem(int dim, int ff, int k, bool exact, int nt) {
        size_t o = kRowTableBytes;
        h = o;     o = up16(o + (size_t)dim * 4);
        xq = o;    o = up16(o + (size_t)(dim >> 8) * kActStride);
        xd = o;    o = up16(o + (size_t)(dim >> 8) * 4);
        hq = o;    o = up16(o + (size_t)k * (ff >> 8) * kActStride);  // fast order: every pick
        hd = o;    o = up16(o + (size_t)k * (ff >> 8) * 4);
        desc = o;  o = up16(o + (size_t)2 * k * sizeof(ExpertDesc));  // this and the next layer
        ids = o;   o = up16(o + (size_t)2 * kMaxPicks * 4);  // this and the previous layer
        w = o;     o = up16(o + (size_t)2 * kMaxPicks * 4);
        order = o; o = up16(o + (size_t)2 * kMaxPicks * 4);
        own = o;   o = up16(o + (size_t)2 * (kMaxPicks + 1) * 4);  // owned pick indices + count
        tree = o;  o = up16(o + (size_t)nt * 8);  // also the K-segment partials [warp][lane]
        // scratch: table staging (kTableWords), one pick's fp32 SwiGLU output (ff), and
        // in the exact order the quad exchange records of every warp
        xch = o;
        size_t words = (size_t)kTableWords > (size_t)ff ? (size_t)kTableWords : (size_t)ff;
        if (exact && (size_t)(nt / 32) * 32 * kXchWords > words) words = (size_t)(nt / 32) * 32 * kXchWords;
        total = o + words * 4 + 16;
    }
};

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// v[0..7] = p[0..7] from shared memory (p 16-byte aligned) as two 16-byte loads: a warp's
// lanes at a stride of 8 floats then hit at most 2-way bank conflicts, where 8 scalar
// loads would each be 8-way.
__device__ __forceinline__ void load8(const float* p, float v[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// Sum of (double)h[i]^2 over i = lane, lane + 1024, ... in order (one of 1024 lanes).
__device__ __forceinline__ double lane_sumsq(const float* hs, int dim, int lane) {
    double s = 0.0;
    for (int i = lane; i < dim; i += 1024) {
        const double v = (double)hs[i];
        s = __dadd_rn(s, __dmul_rn(v, v));
    }
    return s;
}

// MULTI: compiled with the expert-ID sharding exchange (peer stores, signals, waits); the
// one-GPU instantiation carries none of it.
template <bool FAST, int NT, bool MULTI>
__global__ void __launch_bounds__(NT, 1) k_stack(const StackParams P) {
    constexpr int NW = NT / 32;
    uint8_t* smem = clb_dyn_smem;
    const StackSmem L(P.dim, P.ff, P.k, !FAST, NT);
    float* hs = reinterpret_cast<float*>(smem + L.h);
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
    float* xd = reinterpret_cast<float*>(smem + L.xd);
    int8_t* hq = reinterpret_cast<int8_t*>(smem + L.hq);
    float* hd = reinterpret_cast<float*>(smem + L.hd);
    ExpertDesc* dsc = reinterpret_cast<ExpertDesc*>(smem + L.desc);
    int* sid = reinterpret_cast<int*>(smem + L.ids);      // [2][kMaxPicks], slot li & 1
    float* sw = reinterpret_cast<float*>(smem + L.w);
    int* sord = reinterpret_cast<int*>(smem + L.order);   // picks in ascending id order
    double* tree = reinterpret_cast<double*>(smem + L.tree);
    uint32_t* xch_all = reinterpret_cast<uint32_t*>(smem + L.xch);
    float* hf = reinterpret_cast<float*>(smem + L.xch);   // SwiGLU output of this CTA's pick
    float* part = reinterpret_cast<float*>(smem + L.tree);  // K-segment partials [warp][lane]
    int* sown = reinterpret_cast<int*>(smem + L.own);       // [2][kMaxPicks + 1]: picks this GPU owns, count last

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dim = P.dim, ff = P.ff, k = P.k;
    const int nbx = dim >> 8, nbh = ff >> 8;
    const int G = gridDim.x, W = G * NW, gw = blockIdx.x * NW + warp;
    const StackShard& sh = P.sh;
    const size_t yslot = (size_t)k * dim;  // one layer's expert rows
    // expert rows of layer li: the bank's buffer, or (sharded) the exchange slot of its parity
    auto ybuf = [&](int li) -> float* {
        return !MULTI || sh.world == 1 ? P.yrows : sh.yx + ((sh.epoch + li) & 1) * yslot;
    };

    fill_row_tables(P.tables, xch_all);
    for (int i = tid; i < dim; i += NT) hs[i] = __ldcg(P.h_in + i);

    // Routing of layer lj into slot lj & 1, by warp 1: ids and weights, the ascending-id order
    // of the picks, the picks whose expert this GPU holds (in pick order, count last) and
    // their descriptors. Layer 0 before the loop; layer l + 1 while the last grid barrier of
    // layer l is waited for, so the loads are off the critical path.
    auto load_routing = [&](int lj) {
        if (warp != 1) return;
        const int sl = lj & 1;
        int e = -1;
        if (lane < k) {
            e = __ldcg(P.route_ids + (size_t)lj * k + lane);
            sid[sl * kMaxPicks + lane] = e;
            sw[sl * kMaxPicks + lane] = __ldcg(P.route_w + (size_t)lj * k + lane);
        }
        int rank = 0;
        for (int p = 0; p < k; ++p) rank += __shfl_sync(0xffffffffu, e, p) < e;
        if (lane < k) sord[sl * kMaxPicks + rank] = lane;
        const bool mine = lane < k && e >= sh.own_begin && e < sh.own_end;
        const uint32_t m = __ballot_sync(0xffffffffu, mine);
        if (FAST) {
            // the picks computed here ordered by decode speed (IQ2_XXS, IQ2_XS, IQ1_M; pick
            // order within a type): the rounds are pick-major, so the slowest picks' gate/up
            // rounds feed the later down rounds. The order decides only which CTA computes
            // what, not any sum.
            int key = 0x7fffffff;
            if (mine) {
                const int t = __ldcg(&P.desc[(size_t)(P.first + lj) * P.E + e].gate.type);
                key = (t == CLB_IQ2_XXS ? 0 : t == CLB_IQ2_XS ? 1 : 2) * 32 + lane;
            }
            int pos = 0;
            for (int p = 0; p < k; ++p) pos += __shfl_sync(0xffffffffu, key, p) < key;
            if (mine) sown[sl * (kMaxPicks + 1) + pos] = lane;
        } else if (mine) {
            sown[sl * (kMaxPicks + 1) + __popc(m & ((1u << lane) - 1u))] = lane;
        }
        if (lane == 0) sown[sl * (kMaxPicks + 1) + kMaxPicks] = __popc(m);
        __syncwarp();
        constexpr int words = (int)(sizeof(ExpertDesc) / 4);
        for (int i = lane; i < k * words; i += 32) {
            const int p = i / words, wd = i - p * words;
            const uint32_t* src =
                reinterpret_cast<const uint32_t*>(P.desc + (size_t)(P.first + lj) * P.E + sid[sl * kMaxPicks + p]);
            reinterpret_cast<uint32_t*>(dsc + sl * k + p)[wd] = __ldcg(src + wd);
        }
    };
    if (P.nl > 0) load_routing(0);
    __syncthreads();

    for (int li = 0; li <= P.nl; ++li) {
        const int cur = li & 1, prev = cur ^ 1;
        const ExpertDesc* dl = dsc + cur * k;  // this layer's descriptors
        auto stage_next = [&] {
            if (li + 1 < P.nl) load_routing(li + 1);
        };

        STACK_STAMP(li, 0);
        // 1. (exact) h += combine of the previous layer (ascending expert id), in every CTA:
        //    four rows per thread and two such quads at a time, the rows of up to 3 picks of
        //    both loaded before the fma chains
        if (!FAST && li > 0) {
            const float* yr = ybuf(li - 1);
            const int nq = dim >> 2;
            for (int q0 = tid; q0 < nq; q0 += 2 * NT) {
                const int q1 = q0 + NT;
                float4 a0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), a1 = a0;
                for (int o0 = 0; o0 < k; o0 += 3) {
                    float4 v0[3], v1[3];
#pragma unroll
                    for (int j = 0; j < 3; ++j)
                        if (o0 + j < k) {
                            const float* y = yr + (size_t)sord[prev * kMaxPicks + o0 + j] * dim;
                            v0[j] = ldcg4(y + 4 * q0);
                            if (q1 < nq) v1[j] = ldcg4(y + 4 * q1);
                        }
#pragma unroll
                    for (int j = 0; j < 3; ++j)
                        if (o0 + j < k) {
                            const float wj = sw[prev * kMaxPicks + sord[prev * kMaxPicks + o0 + j]];
                            a0.x = __fmaf_rn(wj, v0[j].x, a0.x);
                            a0.y = __fmaf_rn(wj, v0[j].y, a0.y);
                            a0.z = __fmaf_rn(wj, v0[j].z, a0.z);
                            a0.w = __fmaf_rn(wj, v0[j].w, a0.w);
                            if (q1 < nq) {
                                a1.x = __fmaf_rn(wj, v1[j].x, a1.x);
                                a1.y = __fmaf_rn(wj, v1[j].y, a1.y);
                                a1.z = __fmaf_rn(wj, v1[j].z, a1.z);
                                a1.w = __fmaf_rn(wj, v1[j].w, a1.w);
                            }
                        }
                }
                float4 hv = reinterpret_cast<float4*>(hs)[q0];
                hv.x = __fadd_rn(hv.x, a0.x);
                hv.y = __fadd_rn(hv.y, a0.y);
                hv.z = __fadd_rn(hv.z, a0.z);
                hv.w = __fadd_rn(hv.w, a0.w);
                reinterpret_cast<float4*>(hs)[q0] = hv;
                if (q1 < nq) {
                    hv = reinterpret_cast<float4*>(hs)[q1];
                    hv.x = __fadd_rn(hv.x, a1.x);
                    hv.y = __fadd_rn(hv.y, a1.y);
                    hv.z = __fadd_rn(hv.z, a1.z);
                    hv.w = __fadd_rn(hv.w, a1.w);
                    reinterpret_cast<float4*>(hs)[q1] = hv;
                }
            }
            __syncthreads();
        }
        if (li == P.nl) break;
        if (FAST && li > 0) {  // h and its row-group sums of squares as the previous layer's owner warps wrote them
            const float4* hsrc = reinterpret_cast<const float4*>(P.w.hbuf + (size_t)(li & 1) * dim);
            float* ssp = reinterpret_cast<float*>(tree);
            for (int i = tid; i < (dim >> 2); i += NT) reinterpret_cast<float4*>(hs)[i] = __ldcg(hsrc + i);
            for (int rg = tid; rg < (dim >> 5); rg += NT) ssp[rg] = __ldcg(P.w.ssbuf + (size_t)(li & 1) * (dim >> 5) + rg);
            __syncthreads();
        }
        STACK_STAMP(li, 1);

        // x = RMSNorm(h), Q8_K(x). Exact order: lane t of 1024 sums h[t + 1024 j]^2 in j
        // order in fp64, then a binary tree over the lanes (k_norm_quant's order; with 512
        // threads, thread t holds lanes t and t + 512, the tree's first level). Fast order:
        // fp32 fma chains per thread, butterfly sums in each warp, then over the warps; every
        // CTA evaluates the same expression, so all get the same scale.
        if (FAST) {
            // per 32-row group sums of squares (layer 0 from h; later layers as the owner
            // warps wrote them, the same expression), then a fixed-order total that every
            // warp of every CTA evaluates identically
            float* ssp = reinterpret_cast<float*>(tree);
            const int nrg = dim >> 5;
            if (li == 0) {
                for (int rg = warp; rg < nrg; rg += NW) {
                    const float v = hs[rg * 32 + lane];
                    float s = __fmul_rn(v, v);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
                    if (lane == 0) ssp[rg] = s;
                }
                __syncthreads();
            }
            float t = 0.0f;
            for (int i = lane; i < nrg; i += 32) t = __fadd_rn(t, ssp[i]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)dim), 1e-6f)));
            for (int b = warp; b < nbx; b += NW) {
                float v[8];
                load8(hs + b * 256 + lane * 8, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], sc);
                warp_quant_regs(v, xq + (size_t)b * kActStride, xd + b);
            }
        } else {
            double s = lane_sumsq(hs, dim, tid);
            if (NT == 512) s = __dadd_rn(s, lane_sumsq(hs, dim, tid + 512));
            tree[tid] = s;
            __syncthreads();
            for (int stride = NT / 2; stride >= 32; stride >>= 1) {
                if (tid < stride) tree[tid] = __dadd_rn(tree[tid], tree[tid + stride]);
                __syncthreads();
            }
            if (warp == 0) {  // strides 16 .. 1 of the same tree, lane t += lane t + stride
                double v = tree[lane];
#pragma unroll
                for (int stride = 16; stride > 0; stride >>= 1) v = __dadd_rn(v, __shfl_down_sync(0xffffffffu, v, stride));
                if (lane == 0) tree[0] = v;
            }
            __syncthreads();
            const double mean = __ddiv_rn(tree[0], (double)dim);
            const float sc = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(mean, 1e-6)));
            for (int b = warp; b < nbx; b += NW) {
                float v[8];
                load8(hs + b * 256 + lane * 8, v);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], sc);
                warp_quant_regs(v, xq + (size_t)b * kActStride, xd + b);
            }
        }
        __syncthreads();

        STACK_STAMP(li, 2);
        if (FAST) {
            // 2. gate/up, one row per lane: a CTA round covers 8 / SG row groups of 32 rows of
            //    both matrices, each split into SG K segments (one warp each); the segments
            //    are added in order and SwiGLU(g, u) goes to hbuf [pick][ff]
            const int* own = sown + cur * (kMaxPicks + 1);
            const int kown = own[kMaxPicks];
            const int SG = gateup_segments(kown, ff, nbx, G, NW), RGR = NW / 2 / SG, rgpp = ff >> 5, nrg = kown * rgpp;
            const int seg = warp % SG, mat = (warp / SG) & 1, rgl = warp / (2 * SG);
            const int per = (nbx + SG - 1) / SG, b0 = min(nbx, seg * per), b1 = min(nbx, b0 + per);
            for (int q = blockIdx.x; q * RGR < nrg; q += G) {
                const int rg = q * RGR + rgl;
                float y = 0.0f;
                if (rg < nrg) {
                    const int pick = own[rg / rgpp], row = (rg % rgpp) * 32 + lane;
                    const PackedMat& m = mat ? dl[pick].up : dl[pick].gate;
                    if (m.body != nullptr && m.k == dim && m.n == ff) y = lane_row_roll_any(m, row, b0, b1, xq, xd);
                    else if (lane == 0) atomicExch(P.err, 1);
                }
                part[warp * 32 + lane] = y;
                __syncthreads();
                if (tid < RGR * 32) {
                    const int r2 = tid >> 5, rg2 = q * RGR + r2;
                    if (rg2 < nrg) {
                        float g = 0.0f, u = 0.0f;
                        for (int s2 = 0; s2 < SG; ++s2) {
                            g = __fadd_rn(g, part[((r2 * 2 + 0) * SG + s2) * 32 + lane]);
                            u = __fadd_rn(u, part[((r2 * 2 + 1) * SG + s2) * 32 + lane]);
                        }
                        const int slot = own[rg2 / rgpp], rgi = rg2 % rgpp, hb = rgi >> 3;
                        P.gu[(size_t)slot * ff + rgi * 32 + lane] = swiglu(g, u, P.limit);
                        // count the 256-row block (the consumers quantize it once all 8 row groups are in)
                        __syncwarp();
                        if (lane == 0) red_release_gpu(P.w.blk + 1 + ((size_t)li * k + slot) * nbh + hb, 1u);
                    }
                }
                __syncthreads();
            }
            STACK_STAMP(li, 3);
            STACK_STAMP(li, 4);

            // 3. Q8_K(h) of every pick, then the down rows: a CTA round covers 16 / SD
            //    (pick, 32-row group) pairs, each split into SD K segments (one warp each)
            const int SD = down_segments(kown, dim, nbh, G, NW), PPR = NW / SD, rgd = dim >> 5, npair = kown * rgd;
            uint32_t need = 0;  // picks whose rows this CTA's down rounds touch
            for (int q = blockIdx.x; q * PPR < npair; q += G)
                for (int j = 0; j < PPR && q * PPR + j < npair; ++j) need |= 1u << own[(q * PPR + j) / rgd];
            const int nneed = __popc(need);
            {  // Q8_K(h) of those picks: wait until each block's 8 row groups of SwiGLU output are
               // stored, quantize it into shared memory
                int ok = 1;
                for (int wi = warp; wi < nneed * nbh; wi += NW) {
                    const int nth = wi / nbh, b = wi - nth * nbh;  // block b of the nth set bit of `need`
                    uint32_t m = need;
                    for (int c = 0; c < nth; ++c) m &= m - 1;
                    const int slot = __ffs(m) - 1;
                    int got = 1;
                    if (lane == 0)
                        got = wait_reached<false>(P.w.blk + 1 + ((size_t)li * k + slot) * nbh + b, kBlockReady, P.err,
                                                  P.wait_limit, kErrBarrier)
                                  ? 1
                                  : 0;
                    if (!__shfl_sync(0xffffffffu, got, 0)) {
                        ok = 0;
                        break;
                    }
                    __syncwarp();  // the other lanes' loads after lane 0's acquire
                    const float4* src = reinterpret_cast<const float4*>(P.gu + (size_t)slot * ff + (size_t)b * 256 + lane * 8);
                    const float4 lo = __ldcg(src), hi = __ldcg(src + 1);
                    float v8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                    warp_quant_regs(v8, hq + ((size_t)slot * nbh + b) * kActStride, hd + slot * nbh + b);
                }
                if (!__syncthreads_and(ok)) return;
            }
            STACK_STAMP(li, 5);
            const int slot = warp / SD, dseg = warp % SD;
            const int dper = (nbh + SD - 1) / SD, d0 = min(nbh, dseg * dper), d1 = min(nbh, d0 + dper);
            // two CTA rounds per pass: a warp decodes both of its units back to back and the
            // segments are added once per pass
            for (int q0 = blockIdx.x; q0 * PPR < npair; q0 += 2 * G) {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int q = q0 + rr * G, pr = q * PPR + slot;
                    float y = 0.0f;
                    if (slot < PPR && pr < npair) {
                        const int pick = own[pr / rgd], row = (pr % rgd) * 32 + lane;
                        const PackedMat& m = dl[pick].down;
                        if (m.body != nullptr && m.k == ff && m.n == dim)
                            y = lane_row_roll_any(m, row, d0, d1, hq + (size_t)pick * nbh * kActStride, hd + pick * nbh);
                        else if (lane == 0) atomicExch(P.err, 1);
                    }
                    part[(rr * NW + warp) * 32 + lane] = y;
                }
                __syncthreads();
                if (tid < 2 * PPR * 32) {
                    const int rr = tid / (PPR * 32), s2 = (tid >> 5) % PPR, pr2 = (q0 + rr * G) * PPR + s2;
                    if (pr2 < npair) {
                        float t = 0.0f;
                        for (int j = 0; j < SD; ++j) t = __fadd_rn(t, part[(rr * NW + s2 * SD + j) * 32 + lane]);
                        const int rgi = pr2 % rgd;
                        const size_t o = (size_t)own[pr2 / rgd] * dim + rgi * 32 + lane;
                        ybuf(li)[o] = t;
                        for (int r = 0; MULTI && r < sh.world; ++r)  // the peers' copies of this layer's slot
                            if (r != sh.rank) sh.peer_yx[r][((sh.epoch + li) & 1) * yslot + o] = t;
                        // one GPU: count the row group's rows for its owner warp (a sharded bank
                        // counts whole CTAs after the pass instead, see below)
                        __syncwarp();
                        if (!MULTI && lane == 0) red_release_gpu(sh.rgcnt + (size_t)((sh.epoch + li) & 1) * rgd + rgi, 1u);
                    }
                }
                __syncthreads();
            }
            if (MULTI) {
                // Sharded: this CTA's rows (local slot and every peer's copy) are stored (the
                // CTA barrier above); one system-scope fence makes them visible to the peers, a
                // GPU-scope add counts the CTA, and the CTA completing the count publishes the
                // layer number in its flag on every peer (one writer per flag, no contended
                // address on the peers).
                if (tid == 0) {
                    fence_acq_rel_sys();
                    const unsigned old = atom_add_acq_rel_gpu(P.w.blk, 1u);
                    if (old + 1u == (unsigned)G * (unsigned)(li + 1)) {
                        fence_acq_rel_sys();
                        for (int r = 0; r < sh.world; ++r)
                            if (r != sh.rank) st_relaxed_sys(sh.peer_flags[r] + sh.rank, sh.epoch + (unsigned)li + 1u);
                    }
                }
            }
            STACK_STAMP(li, 6);
            {  // 4. owner warp of row group blockIdx.x + warp * G: combine once all k picks' rows are in
                const int rg = blockIdx.x + warp * G;
                int ok = 1;
                if (rg < rgd) {
                    const unsigned lg = sh.epoch + (unsigned)li;
                    if (MULTI && lane == 0) {  // every local CTA's rows, then every peer's
                        ok = wait_reached<false>(P.w.blk, (unsigned)G * (unsigned)(li + 1), P.err, P.wait_limit,
                                                 kErrBarrier)
                                 ? 1
                                 : 0;
                        for (int r = 0; ok && r < sh.world; ++r)
                            if (r != sh.rank)
                                ok = wait_reached<true>(sh.flags + r, lg + 1u, P.err, P.wait_limit, kErrBarrier) ? 1 : 0;
                    }
                    if (!MULTI && lane == 0) {  // one GPU: the k picks' rows of this row group
                        const unsigned* rc = sh.rgcnt + (size_t)(lg & 1u) * rgd + rg;
                        ok = wait_reached<false>(rc, (unsigned)k * ((lg >> 1) + 1u), P.err, P.wait_limit, kErrBarrier) ? 1
                                                                                                                    : 0;
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    __syncwarp();  // the other lanes' loads after lane 0's acquire
                    if (ok) {
                        const float* yr = ybuf(li);
                        const int* ord = sord + cur * kMaxPicks;
                        float yv[kMaxPicks];
#pragma unroll
                        for (int o2 = 0; o2 < kMaxPicks; ++o2)
                            if (o2 < k) yv[o2] = __ldcg(yr + (size_t)ord[o2] * dim + rg * 32 + lane);
                        float acc = 0.0f;
#pragma unroll
                        for (int o2 = 0; o2 < kMaxPicks; ++o2)
                            if (o2 < k) acc = __fmaf_rn(sw[cur * kMaxPicks + ord[o2]], yv[o2], acc);
                        const float hn = __fadd_rn(hs[rg * 32 + lane], acc);
                        if (li == P.nl - 1) {
                            P.h_out[rg * 32 + lane] = hn;
                        } else {
                            P.w.hbuf[(size_t)((li + 1) & 1) * dim + rg * 32 + lane] = hn;
                            float s2 = __fmul_rn(hn, hn);
#pragma unroll
                            for (int o2 = 16; o2 > 0; o2 >>= 1) s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o2));
                            if (lane == 0) P.w.ssbuf[(size_t)((li + 1) & 1) * rgd + rg] = s2;
                        }
                    }
                }
                if (!__syncthreads_and(ok)) return;
            }
        } else {
            // 2. gate/up rows (exact order: 4 threads per row, quad exchange) -> gu
            const int* own = sown + cur * (kMaxPicks + 1);
            const int kown = own[kMaxPicks];
            const int rpw = 8, groups = ff / rpw, items = kown * 2 * groups;
            uint32_t* xch = xch_all + warp * 32 * kXchWords;
            for (int it = gw; it < items; it += W) {
                const int pick = own[it / (2 * groups)], rem = it % (2 * groups);
                const int group = rem >> 1, mat = rem & 1;
                const PackedMat& m = mat ? dl[pick].up : dl[pick].gate;
                const int row = group * rpw + lane / 4;
                float y = 0.0f;
                if (m.body != nullptr && m.k == dim && m.n == ff) y = quad_row_dot_any<false>(m, row, xq, xd, xch);
                else if (lane == 0) atomicExch(P.err, 1);
                if (lane % 4 == 0) P.gu[((size_t)pick * 2 + mat) * ff + row] = y;
            }
            if (!grid_barrier(P.bar, 2 * li + 1, P.err, P.wait_limit)) return;

            // 3. SwiGLU of this CTA's pick over all threads, Q8_K(h) per 256-block, then the
            //    pick's down rows (one thread per row, the reference's lane chains) -> yrows
            // CTA c serves owned pick c * kown / G (none when this GPU owns no pick)
            const int mi = blockIdx.x * max(kown, 1) / G, my_pick = kown > 0 ? own[mi] : 0;
            const int pc0 = pick_cta_begin(mi, max(kown, 1)), pc1 = pick_cta_begin(mi + 1, max(kown, 1));
            const int pick_warps = (pc1 - pc0) * NW, pick_warp = (blockIdx.x - pc0) * NW + warp;
            const float* g = P.gu + ((size_t)my_pick * 2) * ff;
            for (int i = tid; i < ff; i += NT) hf[i] = swiglu(__ldcg(g + i), __ldcg(g + ff + i), P.limit);
            __syncthreads();
            for (int hb = warp; hb < nbh; hb += NW) {
                float v[8];
                load8(hf + hb * 256 + lane * 8, v);
                warp_quant_regs(v, hq + (size_t)hb * kActStride, hd + hb);
            }
            __syncthreads();
            const PackedMat& m = dl[my_pick].down;
            const int groups_d = dim >> 5;
            const bool ok = m.body != nullptr && m.k == ff && m.n == dim;
            if (kown > 0 && !ok && tid == 0) atomicExch(P.err, 1);
            for (int g2 = pick_warp; kown > 0 && g2 < groups_d; g2 += pick_warps) {
                const int row = g2 * 32 + lane;
                const float y = ok ? thread_row_dot_any<false>(m, row, hq, hd) : 0.0f;
                const size_t o = (size_t)my_pick * dim + row;
                ybuf(li)[o] = y;
                for (int r = 0; MULTI && r < sh.world; ++r)
                    if (r != sh.rank) sh.peer_yx[r][((sh.epoch + li) & 1) * yslot + o] = y;
            }
        }
        if (!FAST) STACK_STAMP(li, 6);
        if (!FAST && MULTI && sh.world > 1) signal_peers(sh);  // this CTA's peer stores, then one release per peer
        // barrier number: one per layer in the fast order, two in the exact order
        if (!grid_barrier(P.bar, FAST ? li + 1 : 2 * li + 2, P.err, P.wait_limit, stage_next)) return;
        STACK_STAMP(li, 7);
        if (!FAST && MULTI && sh.world > 1 && !exchange_rows(sh, li, P.err, P.wait_limit)) return;
    }
    // h after the last layer: each CTA writes its slice (the fast order's owner warps wrote it)
    if (FAST) return;
    const int per = (dim + G - 1) / G;
    for (int i = blockIdx.x * per + tid; i < min(dim, (blockIdx.x + 1) * per); i += NT) P.h_out[i] = hs[i];
}

// Threads per CTA of the persistent kernel (16 warps, up to 128 registers a thread).
#ifndef CLB_STACK_FAST_THREADS
#define CLB_STACK_FAST_THREADS 512
#endif
// Threads per CTA of the persistent kernel: the exact order 16 warps (up to 128 registers a
// thread); the fast order CLB_STACK_FAST_THREADS.
static int stack_threads(bool fast) { return fast ? CLB_STACK_FAST_THREADS : 512; }

size_t stack_smem(int dim, int ff, int k, bool fast) { return StackSmem(dim, ff, k, !fast, stack_threads(fast)).total; }

static int stack_grid() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

size_t stack_block_words(int nl_max, int k, int ff) { return 1 + (size_t)nl_max * k * (ff >> 8); }

bool stack_supported(int dim, int ff, int k, bool fast) {
    int dev = 0, optin = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop) return false;
    const size_t need = stack_smem(dim, ff, k, fast);
    return optin > 0 && need <= (size_t)optin && k <= stack_grid();
}

cudaError_t launch_stack(const ExpertDesc* desc, int E, int first, int nl, int k, const int* route_ids,
                         const float* route_w, const float* h_in, float* h_out, int dim, int ff, float limit, float* gu,
                         float* yrows, unsigned* bar, int* err, bool fast, const StackShard& shard, cudaStream_t s,
                         unsigned wait_limit, const StackWork& w) {
    const uint32_t* tables = nullptr;
    cudaError_t e = tables_device_ptr(&tables);
    if (e != cudaSuccess) return e;
    const int G = stack_grid();
    StackParams P{};
    P.desc = desc;
    P.E = E;
    P.first = first;
    P.nl = nl;
    P.k = k;
    P.route_ids = route_ids;
    P.route_w = route_w;
    P.h_in = h_in;
    P.h_out = h_out;
    P.dim = dim;
    P.ff = ff;
    P.limit = limit;
    P.gu = gu;
    P.yrows = yrows;
    P.bar = bar;
    P.err = err;
    P.wait_limit = wait_limit;
    P.tables = tables;
    P.sh = shard;
    P.w = w;
    if (fast && (w.hbuf == nullptr || w.ssbuf == nullptr || w.blk == nullptr ||
                 shard.rgcnt == nullptr))
        return cudaErrorInvalidValue;
    const int nt = stack_threads(fast);
    const size_t sm = stack_smem(dim, ff, k, fast);
    const bool multi = shard.world > 1;
    constexpr int FT = CLB_STACK_FAST_THREADS;
    void (*kern)(StackParams) = fast ? (multi ? k_stack<true, FT, true> : k_stack<true, FT, false>)
                                     : (multi ? k_stack<false, 512, true> : k_stack<false, 512, false>);
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm))) return e;
    if ((e = cudaMemsetAsync(bar, 0, sizeof(unsigned), s))) return e;
    if (fast && (e = cudaMemsetAsync(w.blk, 0, stack_block_words(nl, k, ff) * sizeof(unsigned), s))) return e;
    void* args[] = {&P};
    return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(G), dim3(nt), args, sm, s);
}

}  // namespace clb

#ifdef CLB_FLOW_TRACE
extern "C" int clb_stack_trace_read(void* host, size_t bytes) {
    if (bytes > sizeof(clb::g_stack_trace)) bytes = sizeof(clb::g_stack_trace);
    return (int)cudaMemcpyFromSymbol(host, clb::g_stack_trace, bytes);
}
#endif
