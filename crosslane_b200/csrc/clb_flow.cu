// Dataflow whole-stack decode kernel (fast summation order): one CTA of 16 warps per SM
// runs every layer of a token. Inside a layer the CTAs take work "rounds" from a counter
// in the order gate/up rounds, then down rounds, and hand results on through completion
// counters instead of meeting at grid barriers between the phases:
//
//   norm      every CTA: sum of squares of h (per 32-row group partials written by the
//             previous layer's combines, added in a fixed order), x = RMSNorm(h), Q8_K(x)
//             into shared memory;
//   gate/up   a round = RGR row groups of 32 rows x {gate, up} x SG K segments (one warp
//             each, one row per lane); the segments are added in order, SwiGLU(g, u) goes
//             to gu. The round that completes a 256-row block of a pick quantizes it to
//             Q8_K (hq, hd) and counts the pick's quantized blocks;
//   down      a round = PPR (pick, 32-row group) pairs x SD K segments; it waits for its
//             picks' Q8_K(h), reads them from global memory, and writes the expert rows
//             (to every GPU of a sharded bank) and counts each row group's rows;
//   combine   CTA c owns row groups c, c + G, ...: once all k picks' rows of a group are
//             in, h += the ascending-id fma combine of the rows (runtime.cpp:184-187),
//             its sum of squares is written, and the layer counter is bumped;
//   -- the next layer starts when every row group is combined (the one grid-wide wait).
//
// Rounds are grabbed two ahead, so the counter's round trip and the readiness of the next
// down round's picks are waited for behind the current round's decode.
//
// Every wait is bounded (kFlowSpinLimit polls): a wait that runs out sets *err = 2 and the
// CTA returns, so no launch can hang. Counters that other GPUs write (row groups, by layer
// parity) only grow; the per-launch ones are zeroed by launch_flow.
#include <cuda_runtime.h>

#include "clb_device.cuh"
#include "clb_kernels.h"
#include "clb_v2.cuh"

namespace clb {

namespace {

constexpr unsigned kFlowSpinLimit = 1u << 22;
constexpr int kFlowDecodeWarps = 15;              // warps that decode weights
constexpr int kFlowWarps = kFlowDecodeWarps + 1;  // + one service warp
constexpr int kFlowThreads = kFlowWarps * 32;
constexpr int kErrWait = 2;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait until *p has reached target (modulo 2^32). SYS: the writers include other
// GPUs. Polls with relaxed loads (an acquire load per poll would discard the SM's L1 lines
// each time, under the feet of the warps still decoding) and orders the caller's later
// reads after the writes it waited for with one fence once the target is seen (the
// relaxed-load + fence acquire pattern). Backs off after a few hundred polls.
template <bool SYS>
__device__ bool wait_reached(const unsigned* p, unsigned target, int* err) {
    for (unsigned spins = 0;; ++spins) {
        const unsigned v = SYS ? ld_relaxed_sys(p) : ld_relaxed_gpu(p);
        if ((int)(v - target) >= 0) {
            if (SYS) fence_acq_rel_sys();
            else fence_acq_rel_gpu();
            return true;
        }
        if (spins > kFlowSpinLimit) {
            atomicExch(err, kErrWait);
            return false;
        }
        if (spins > 256) __nanosleep(64);
    }
}

}  // namespace

// Round shapes of one layer for `kown` picks computed here on `grid` CTAs of
// kFlowDecodeWarps decoding warps: gate/up rgr x 2 x sg warps, down ppr x sd warps; chosen
// to minimise an estimate of the layer's block decodes per CTA (the work spread over the
// grid, at least a gate/up segment then a down segment on the critical path) plus one down
// round of tail.
struct FlowShape {
    int rgr, sg, ppr, sd, ngu, nd;
};
__host__ __device__ inline FlowShape flow_shape(int kown, int dim, int ff, int grid) {
    const int rgpp = ff >> 5, rgd = dim >> 5, nbx = dim >> 8, nbh = ff >> 8;
    FlowShape best{1, 1, 1, 1, 0, 0};
    int best_cost = -1;
    for (int rgr = 8; rgr >= 1; rgr >>= 1) {
        const int sg = kFlowDecodeWarps / 2 / rgr;
        if (sg < 1 || rgpp % rgr) continue;
        const int ngu = kown * rgpp / rgr, seg_gu = (nbx + sg - 1) / sg;
        for (int sd = 1; sd <= 8; ++sd) {
            const int ppr = kFlowDecodeWarps / sd;
            const int nd = (kown * rgd + ppr - 1) / ppr, seg_d = (nbh + sd - 1) / sd;
            int spread = (ngu * seg_gu + nd * seg_d + grid - 1) / grid;
            if (spread < seg_gu + seg_d) spread = seg_gu + seg_d;
            const int cost = spread + seg_d;
            if (best_cost < 0 || cost < best_cost) {
                best_cost = cost;
                best = FlowShape{rgr, sg, ppr, sd, ngu, nd};
            }
        }
    }
    return best;
}

struct FlowParams {
    const ExpertDesc* desc;  // [bank layers][E]
    int E, first, nl, k;
    const int* route_ids;    // [nl][k]
    const float* route_w;    // [nl][k]
    const float* h_in;
    float* h_out;            // may alias h_in
    int dim, ff;
    float limit;
    FlowWork w;
    int* err;
    const uint32_t* tables;
    StackShard sh;
};

// Per-layer control block in shared memory (written between CTA barriers).
struct FlowCtl {
    int ring[3];        // round indices, grabbed two ahead by the service warp
    int ready[3];       // down round: 2 when every pick was seen quantized and is staged in shared memory
    FlowShape f;
    int kown, rounds;
};

// Shared memory layout (bytes), fixed for dim <= kFlowMaxDim and k <= kMaxPicks so that
// every address is a constant (no registers held for it across the decode calls).
constexpr int kFlowMaxDim = 16384;
constexpr uint32_t kFoStage = kRowTableBytes;
constexpr uint32_t kFoXq = kFoStage + kTableWords * 4;
constexpr uint32_t kFoXd = kFoXq + (kFlowMaxDim / 256) * kActStride;
constexpr uint32_t kFoPart = kFoXd + (kFlowMaxDim / 256) * 4;  // [2][decode warps][32] floats
constexpr uint32_t kFoIds = kFoPart + 2 * kFlowDecodeWarps * 32 * 4;
constexpr uint32_t kFoW = kFoIds + kMaxPicks * 4;
constexpr uint32_t kFoOrd = kFoW + kMaxPicks * 4;       // pick slots in ascending expert id order
constexpr uint32_t kFoOwn = kFoOrd + kMaxPicks * 4;     // pick slots computed here, count last
constexpr uint32_t kFoOcnt = kFoOwn + (kMaxPicks + 4) * 4;  // per slot: layers of this launch computed here
constexpr uint32_t kFoDesc = kFoOcnt + kMaxPicks * 4;
constexpr int kStagePicks = 3, kStageBlocks = 16;  // down-round activations staged in shared memory (ff <= 4096)
constexpr uint32_t kFoStageH = kFoDesc + kMaxPicks * sizeof(ExpertDesc);  // [2][picks][blocks] padded Q8_K blocks
constexpr uint32_t kFoStageD = kFoStageH + 2 * kStagePicks * kStageBlocks * kActStride;  // [2][picks][blocks] scales
constexpr uint32_t kFoCtl = kFoStageD + 2 * kStagePicks * kStageBlocks * 4;
constexpr uint32_t kFoParams = (kFoCtl + (uint32_t)sizeof(FlowCtl) + 15u) & ~15u;
constexpr uint32_t kFlowSmemBytes = (kFoParams + (uint32_t)sizeof(FlowParams) + 15u) & ~15u;
static_assert(kFoXq % 16 == 0 && kFoPart % 16 == 0 && kFoDesc % 16 == 0, "16-byte aligned regions");
static_assert((kFlowMaxDim >> 5) <= 2 * kFlowDecodeWarps * 32, "the norm's partials fit the round-partial area");

template <class T>
__device__ __forceinline__ T* fsm(uint32_t off) {
    return reinterpret_cast<T*>(clb_dyn_smem + off);
}
__device__ __forceinline__ const FlowParams& fparams() { return *fsm<const FlowParams>(kFoParams); }
__device__ __forceinline__ FlowCtl& fctl() { return *fsm<FlowCtl>(kFoCtl); }

size_t flow_counter_words(int nl_max, int k, int ff) {
    return (size_t)nl_max + (size_t)k * (ff >> 8) + (size_t)k + 1;
}

// This warp's segment of round r (nullptr: idle): matrix, row and block range.
__device__ __forceinline__ const PackedMat* flow_segment(int r, int warp, int lane, int dim, int ff, int& row, int& b0,
                                                         int& b1) {
    const FlowCtl& c = fctl();
    const FlowShape& F = c.f;
    const int* own = fsm<int>(kFoOwn);
    const ExpertDesc* dsc = fsm<ExpertDesc>(kFoDesc);
    const int rgpp = ff >> 5, rgd = dim >> 5, nbx = dim >> 8, nbh = ff >> 8;
    if (r < F.ngu) {
        const int j = warp / (2 * F.sg), mat = (warp / F.sg) & 1, s = warp % F.sg;
        if (j >= F.rgr) return nullptr;
        const int rgl = r * F.rgr + j, pick = own[rgl / rgpp];
        row = (rgl % rgpp) * 32 + lane;
        const int per = (nbx + F.sg - 1) / F.sg;
        b0 = min(nbx, s * per);
        b1 = min(nbx, b0 + per);
        return mat ? &dsc[pick].up : &dsc[pick].gate;
    }
    if (r < c.rounds) {
        const int jp = warp / F.sd, s = warp % F.sd, pair = (r - F.ngu) * F.ppr + jp;
        if (jp >= F.ppr || pair >= c.kown * rgd) return nullptr;
        row = (pair % rgd) * 32 + lane;
        const int per = (nbh + F.sd - 1) / F.sd;
        b0 = min(nbh, s * per);
        b1 = min(nbh, b0 + per);
        return &dsc[own[pair / rgd]].down;
    }
    return nullptr;
}

#ifdef CLB_FLOW_TRACE
// Phase stamps (%globaltimer ns) per (layer, CTA), a build-time option for phase tables:
// 0 layer entry, 1 h ready, 2 norm done, 3 rounds done, 4 combine done, 5 gate/up rounds,
// 6 down rounds, 7 ns warp 0 waited for down-round activations.
constexpr int kTraceLayers = 64, kTraceCtas = 160;
__device__ unsigned long long g_flow_trace[kTraceLayers * kTraceCtas * 8];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define FLOW_TRACE(li, slot, v)                                                                             \
    do {                                                                                                   \
        if ((li) < kTraceLayers && blockIdx.x < kTraceCtas) g_flow_trace[((li) * kTraceCtas + blockIdx.x) * 8 + (slot)] = (v); \
    } while (0)
#define FLOW_TRACE_ADD(li, slot, v)                                                                         \
    do {                                                                                                   \
        if ((li) < kTraceLayers && blockIdx.x < kTraceCtas) g_flow_trace[((li) * kTraceCtas + blockIdx.x) * 8 + (slot)] += (v); \
    } while (0)
#else
#define FLOW_TRACE(li, slot, v) do { } while (0)
#define FLOW_TRACE_ADD(li, slot, v) do { } while (0)
#endif

// Pick-quantization counters: [k] after grab [nl] and the block counters [k][nbh].
__device__ __forceinline__ unsigned* flow_pickq(const FlowParams& P) {
    return P.w.cnt + P.nl + P.k * (P.ff >> 8);
}

// Decoding warps of layer li: one segment per round until the rounds run out. False: a
// bounded wait ran out (the error flag is set).
__device__ __forceinline__ bool flow_decode(int li) {
    const FlowParams& P = fparams();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = 0;; ++i) {
        __syncthreads();  // round i may start (ring, ready and the partial buffer are set)
        const FlowCtl& c = fctl();
        const int r = c.ring[i % 3];
        if (r >= c.rounds) {
#ifdef CLB_FLOW_TRACE
            if (warp == 0 && lane == 0) FLOW_TRACE(li, 3, gtimer());
#endif
            return true;
        }
#ifdef CLB_FLOW_TRACE
        if (warp == 0 && lane == 0) FLOW_TRACE_ADD(li, r < c.f.ngu ? 5 : 6, 1ull);
#endif
        const int dim = P.dim, ff = P.ff;
        int row = 0, b0 = 0, b1 = 0;
        const PackedMat* m = flow_segment(r, warp, lane, dim, ff, row, b0, b1);
        float y = 0.0f;
        if (m) {
            const bool gu = r < c.f.ngu;
            const bool shape_ok = m->body != nullptr && (gu ? (m->k == dim && m->n == ff) : (m->k == ff && m->n == dim));
            if (!shape_ok) {
                if (lane == 0) atomicExch(P.err, 1);
            } else if (gu) {
                y = lane_row_db_any<kActStride>(*m, row, b0, b1, fsm<int8_t>(kFoXq), fsm<float>(kFoXd));
            } else {
                const int nbh = ff >> 8, rgd = dim >> 5, q = r - c.f.ngu;
                const int pi = (q * c.f.ppr + warp / c.f.sd) / rgd, slot = fsm<int>(kFoOwn)[pi];
                const int ready = c.ready[i % 3], ps = pi - q * c.f.ppr / rgd, buf = i & 1;
                int8_t* aq = fsm<int8_t>(kFoStageH) + ((buf * kStagePicks + ps) * kStageBlocks) * kActStride;
                float* ad = fsm<float>(kFoStageD) + (buf * kStagePicks + ps) * kStageBlocks;
                if (ready != 2) {
                    // not seen quantized by the service warp: wait here (bounded), then stage
                    // this segment's blocks of the pick (warps of the same pick write the same bytes)
#ifdef CLB_FLOW_TRACE
                    const unsigned long long t0 = gtimer();
#endif
                    bool got = true;
                    if (lane == 0)
                        got = wait_reached<false>(flow_pickq(P) + slot, (unsigned)nbh * (unsigned)fsm<int>(kFoOcnt)[slot],
                                                  P.err);
                    if (!__shfl_sync(0xffffffffu, (int)got, 0)) return false;
#ifdef CLB_FLOW_TRACE
                    if (warp == 0 && lane == 0) FLOW_TRACE_ADD(li, 7, gtimer() - t0);
#endif
                    const uint4* sq = reinterpret_cast<const uint4*>(P.w.hq + (size_t)slot * ff);
                    for (int c2 = b0 * 16 + lane; c2 < b1 * 16; c2 += 32)
                        *reinterpret_cast<uint4*>(aq + (c2 >> 4) * kActStride + (c2 & 15) * 16) = __ldcg(sq + c2);
                    if (lane < b1 - b0) ad[b0 + lane] = __ldcg(P.w.hd + (size_t)slot * nbh + b0 + lane);
                    __syncwarp();
                }
                y = lane_row_db_any<kActStride>(*m, row, b0, b1, aq, ad);
            }
        }
        fsm<float>(kFoPart)[((i & 1) * kFlowDecodeWarps + warp) * 32 + lane] = y;
    }
}

// Service warp of layer li: while the decoding warps run round i it finishes round i - 1
// (epilogue), grabs round i + 2, prefetches round i + 1's first blocks into L2 and samples
// whether round i + 1's picks are quantized.
__device__ __noinline__ void flow_service(int li) {
    const FlowParams& P = fparams();
    FlowCtl& c = fctl();
    const int lane = threadIdx.x & 31;
    const int dim = P.dim, ff = P.ff, k = P.k, nbh = ff >> 8, nrg = dim >> 5, rgpp = ff >> 5;
    const FlowShape F = c.f;
    const int R = c.rounds, npair = c.kown * nrg;
    const int* own = fsm<int>(kFoOwn);
    const int* ocnt = fsm<int>(kFoOcnt);
    unsigned* blk = P.w.cnt + P.nl;
    unsigned* pickq = flow_pickq(P);
    const StackShard& sh = P.sh;
    const unsigned lg = sh.epoch + (unsigned)li;
    const int par = (int)(lg & 1u);
    float* ybuf = sh.yx + (size_t)par * k * dim;
    unsigned* rgc = sh.rgcnt + (size_t)par * nrg;
    unsigned* grab = P.w.cnt + li;

    // Down round r: 0 if a pick's Q8_K(h) is not complete yet; else (after one fence, the
    // acquire for the decoders' reads) 2 when its picks' blocks were copied into the stage
    // buffer `buf` of shared memory, 1 when they are read from global memory.
    auto down_ready = [&](int r, int buf) -> int {
        if (r < F.ngu || r >= R) return 0;
        const int q = r - F.ngu, p0 = q * F.ppr / nrg, p1 = min(npair - 1, q * F.ppr + F.ppr - 1) / nrg;
        int rdy = 1;
        for (int pi = p0; pi <= p1; ++pi) {
            const int slot = own[pi];
            unsigned v = 0;
            if (lane == 0) v = ld_relaxed_gpu(pickq + slot);
            v = __shfl_sync(0xffffffffu, v, 0);
            if ((int)(v - (unsigned)nbh * (unsigned)ocnt[slot]) < 0) rdy = 0;
        }
        if (!rdy) return 0;
        fence_acq_rel_gpu();
        for (int pi = p0; pi <= p1; ++pi) {
            const int slot = own[pi], ps = pi - p0;
            int8_t* dq = fsm<int8_t>(kFoStageH) + ((buf * kStagePicks + ps) * kStageBlocks) * kActStride;
            const uint4* sq = reinterpret_cast<const uint4*>(P.w.hq + (size_t)slot * ff);
            for (int c2 = lane; c2 < nbh * 16; c2 += 32)
                *reinterpret_cast<uint4*>(dq + (c2 >> 4) * kActStride + (c2 & 15) * 16) = __ldcg(sq + c2);
            if (lane < nbh)
                fsm<float>(kFoStageD)[(buf * kStagePicks + ps) * kStageBlocks + lane] = __ldcg(P.w.hd + (size_t)slot * nbh + lane);
        }
        return 2;
    };
    auto prefetch_round = [&](int r) {
        for (int w = 0; w < kFlowDecodeWarps; ++w) {
            int row = 0, b0 = 0, b1 = 0;
            const PackedMat* m = flow_segment(r, w, lane, dim, ff, row, b0, b1);
            if (m && m->body && b0 < b1) prefetch_row_block(*m, row, b0);
        }
    };
    {
        const int rdy = down_ready(c.ring[0], 0);
        if (lane == 0) c.ready[0] = rdy;
        prefetch_round(c.ring[0]);
    }
    int rprev = -1;
    for (int i = 0;; ++i) {
        __syncthreads();
        const int r = c.ring[i % 3], rn = c.ring[(i + 1) % 3];
        const float* pb = fsm<float>(kFoPart) + ((i - 1) & 1) * kFlowDecodeWarps * 32;
        if (rprev >= 0 && rprev < F.ngu) {
            // gate/up epilogue: add the segments in order, SwiGLU; the round that completes a
            // 256-row block of a pick quantizes it to Q8_K
            for (int j = 0; j < F.rgr; ++j) {
                const int rgl = rprev * F.rgr + j, slot = own[rgl / rgpp], rgi = rgl % rgpp;
                float g = 0.0f, u = 0.0f;
                for (int s2 = 0; s2 < F.sg; ++s2) {
                    g = __fadd_rn(g, pb[((j * 2 + 0) * F.sg + s2) * 32 + lane]);
                    u = __fadd_rn(u, pb[((j * 2 + 1) * F.sg + s2) * 32 + lane]);
                }
                P.w.gu[(size_t)slot * ff + rgi * 32 + lane] = swiglu(g, u, P.limit);
                __syncwarp();
                const int bqi = rgi >> 3;
                unsigned old = 0;
                if (lane == 0) old = atom_add_acq_rel_gpu(blk + slot * nbh + bqi, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                if ((old & 7u) == 7u) {  // the 8th row group of this block in this layer
                    const float4* src =
                        reinterpret_cast<const float4*>(P.w.gu + (size_t)slot * ff + (size_t)bqi * 256 + lane * 8);
                    const float4 lo = __ldcg(src), hi = __ldcg(src + 1);
                    float v8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                    warp_quant_regs(v8, P.w.hq + (size_t)slot * ff + (size_t)bqi * 256, P.w.hd + (size_t)slot * nbh + bqi);
                    __syncwarp();
                    if (lane == 0) red_release_gpu(pickq + slot, 1u);
                }
            }
        } else if (rprev >= 0) {
            // down epilogue: add each pair's segments in order, store the expert rows (also
            // into every peer's slot of this layer parity), count the row group
            for (int jp = 0; jp < F.ppr; ++jp) {
                const int pair = (rprev - F.ngu) * F.ppr + jp;
                if (pair >= npair) break;
                const int slot = own[pair / nrg], rgi = pair % nrg;
                float t = 0.0f;
                for (int s2 = 0; s2 < F.sd; ++s2) t = __fadd_rn(t, pb[(jp * F.sd + s2) * 32 + lane]);
                const size_t o = (size_t)slot * dim + rgi * 32 + lane;
                ybuf[o] = t;
                if (sh.world > 1)
                    for (int rr = 0; rr < sh.world; ++rr)
                        if (rr != sh.rank) sh.peer_yx[rr][(size_t)par * k * dim + o] = t;
                __syncwarp();
                if (lane == 0) {
                    red_release_gpu(rgc + rgi, 1u);
                    if (sh.world > 1)
                        for (int rr = 0; rr < sh.world; ++rr)
                            if (rr != sh.rank) red_release_sys(sh.peer_rgcnt[rr] + (size_t)par * nrg + rgi, 1u);
                }
            }
        }
        if (r >= R) return;
        unsigned nn = 0;
        if (lane == 0) nn = atomicAdd(grab, 1u);
        prefetch_round(rn);
        const int rdy = down_ready(rn, (i + 1) & 1);
        nn = __shfl_sync(0xffffffffu, nn, 0);
        if (lane == 0) {
            c.ring[(i + 2) % 3] = (int)nn;
            c.ready[(i + 1) % 3] = rdy;
        }
        rprev = r;
    }
}

// Start of layer li (all warps): wait until every row group of the previous layer is
// combined, load the routing (warp 1), RMSNorm + Q8_K(x) into shared memory. False: a
// bounded wait ran out.
__device__ __noinline__ bool flow_start(int li) {
    const FlowParams& P = fparams();
    FlowCtl& ctl = fctl();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dim = P.dim, ff = P.ff, k = P.k, nbx = dim >> 8, nrg = dim >> 5;
    const StackShard& sh = P.sh;
    unsigned* layer_cnt = P.w.cnt + P.nl + k * (ff >> 8) + k;
    const float* hsrc = li == 0 ? P.h_in : P.w.hbuf + (size_t)(li & 1) * dim;
    int8_t* xq = fsm<int8_t>(kFoXq);
    float* xd = fsm<float>(kFoXd);

    bool ok = true;
#ifdef CLB_FLOW_TRACE
    if (tid == 0) FLOW_TRACE(li, 0, gtimer());
#endif
    if (warp == kFlowDecodeWarps && lane == 0) {
        ctl.ring[0] = (int)atomicAdd(P.w.cnt + li, 1u);
        ctl.ring[1] = (int)atomicAdd(P.w.cnt + li, 1u);
        if (li > 0) ok = wait_reached<false>(layer_cnt, (unsigned)nrg * (unsigned)li, P.err);
    }
    if (!__syncthreads_and(ok)) return false;
#ifdef CLB_FLOW_TRACE
    if (tid == 0) FLOW_TRACE(li, 1, gtimer());
#endif

    if (warp == 1) {  // routing: ids, weights, ascending-id order, the picks computed here, descriptors
        int* sid = fsm<int>(kFoIds);
        int* sown = fsm<int>(kFoOwn);
        int* socnt = fsm<int>(kFoOcnt);
        int e = -1;
        if (lane < k) {
            e = __ldcg(P.route_ids + (size_t)li * k + lane);
            sid[lane] = e;
            fsm<float>(kFoW)[lane] = __ldcg(P.route_w + (size_t)li * k + lane);
        }
        int rank = 0;
        for (int p = 0; p < k; ++p) rank += __shfl_sync(0xffffffffu, e, p) < e;
        if (lane < k) fsm<int>(kFoOrd)[rank] = lane;
        const bool mine = lane < k && e >= sh.own_begin && e < sh.own_end;
        const uint32_t m = __ballot_sync(0xffffffffu, mine);
        if (mine) {
            sown[__popc(m & ((1u << lane) - 1u))] = lane;
            socnt[lane] += 1;
        }
        if (lane == 0) {
            const int kown = __popc(m);
            sown[kMaxPicks] = kown;
            ctl.kown = kown;
            ctl.f = flow_shape(kown, dim, ff, gridDim.x);
            ctl.rounds = ctl.f.ngu + ctl.f.nd;
        }
        __syncwarp();
        constexpr int words = (int)(sizeof(ExpertDesc) / 4);
        ExpertDesc* dsc = fsm<ExpertDesc>(kFoDesc);
        for (int i = lane; i < k * words; i += 32) {
            const int p = i / words, wd = i - p * words;
            const uint32_t* src = reinterpret_cast<const uint32_t*>(P.desc + (size_t)(P.first + li) * P.E + sid[p]);
            reinterpret_cast<uint32_t*>(dsc + p)[wd] = __ldcg(src + wd);
        }
    }
    // sum of squares: per 32-row group partials (layer 0 from h_in, in the combine's own
    // order; later layers as the combines wrote them), then a fixed-order total that every
    // warp of every CTA evaluates identically
    float* ssp = fsm<float>(kFoPart);  // [nrg] scratch (the round partials are not in use yet)
    if (li == 0) {
        for (int rg = warp; rg < nrg; rg += kFlowWarps) {
            const float v = __ldcg(hsrc + rg * 32 + lane);
            float s = __fmul_rn(v, v);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
            if (lane == 0) ssp[rg] = s;
        }
    } else {
        for (int rg = tid; rg < nrg; rg += kFlowThreads) ssp[rg] = __ldcg(P.w.ssbuf + (size_t)(li & 1) * nrg + rg);
    }
    // this warp's first Q8_K(x) block is loaded before the barrier (it does not need the scale)
    float v[8];
    const int b0 = warp;
    if (b0 < nbx) {
        const float4* src = reinterpret_cast<const float4*>(hsrc + (size_t)b0 * 256 + lane * 8);
        const float4 lo = __ldcg(src), hi = __ldcg(src + 1);
        v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w, v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
    }
    __syncthreads();
    float t = 0.0f;
    for (int i = lane; i < nrg; i += 32) t = __fadd_rn(t, ssp[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)dim), 1e-6f)));
    for (int b = b0; b < nbx; b += kFlowWarps) {
        if (b != b0) {
            const float4* src = reinterpret_cast<const float4*>(hsrc + (size_t)b * 256 + lane * 8);
            const float4 lo = __ldcg(src), hi = __ldcg(src + 1);
            v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w, v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], sc);
        warp_quant_regs(v, xq + (size_t)b * kActStride, xd + b);
    }
    __syncthreads();
#ifdef CLB_FLOW_TRACE
    if (tid == 0) FLOW_TRACE(li, 2, gtimer());
#endif
    return true;
}

// Combine of layer li (all warps): warp w of CTA c owns row group c + w * G; once the rows
// of all k picks are in (row-group counter of the layer parity), h += the ascending-id fma
// combine (runtime.cpp:184-187); the new h and its sum of squares go to the next layer's
// buffers (the last layer writes h_out), then the layer counter. False: a wait ran out.
template <bool MULTI>
__device__ __noinline__ bool flow_combine(int li) {
    const FlowParams& P = fparams();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dim = P.dim, k = P.k, nrg = dim >> 5, G = gridDim.x;
    const StackShard& sh = P.sh;
    unsigned* layer_cnt = P.w.cnt + P.nl + k * (P.ff >> 8) + k;
    const float* hsrc = li == 0 ? P.h_in : P.w.hbuf + (size_t)(li & 1) * dim;
    const unsigned lg = sh.epoch + (unsigned)li;
    const int par = (int)(lg & 1u);
    const float* ybuf = sh.yx + (size_t)par * k * dim;
    unsigned* rgc = sh.rgcnt + (size_t)par * nrg;
    const bool last = li == P.nl - 1;
    const unsigned tgt = (unsigned)k * ((lg >> 1) + 1u);
    const int* sord = fsm<int>(kFoOrd);
    const float* sw = fsm<float>(kFoW);
    int wok = 1;
    for (int rg = blockIdx.x + warp * G; rg < nrg; rg += kFlowWarps * G) {
        bool got = true;
        if (lane == 0) got = MULTI ? wait_reached<true>(rgc + rg, tgt, P.err) : wait_reached<false>(rgc + rg, tgt, P.err);
        if (!__shfl_sync(0xffffffffu, got, 0)) {
            wok = 0;
            break;
        }
        float acc = 0.0f;
        for (int o = 0; o < k; ++o) {
            const int p = sord[o];
            acc = __fmaf_rn(sw[p], __ldcg(ybuf + (size_t)p * dim + rg * 32 + lane), acc);
        }
        const float hn = __fadd_rn(__ldcg(hsrc + rg * 32 + lane), acc);
        if (last && P.nl > 1) {
            P.h_out[rg * 32 + lane] = hn;
        } else {
            P.w.hbuf[(size_t)((li + 1) & 1) * dim + rg * 32 + lane] = hn;
            float s = __fmul_rn(hn, hn);
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o2));
            if (lane == 0) P.w.ssbuf[(size_t)((li + 1) & 1) * nrg + rg] = s;
        }
        __syncwarp();
        if (lane == 0) red_release_gpu(layer_cnt, 1u);
    }
    const bool ok = __syncthreads_and(wok) != 0;
#ifdef CLB_FLOW_TRACE
    if (threadIdx.x == 0) FLOW_TRACE(li, 4, gtimer());
#endif
    return ok;
}

template <bool MULTI>
__global__ void __launch_bounds__(kFlowThreads, 1) k_flow(const FlowParams Pk) {
    const int tid = threadIdx.x;
    if (tid == 0) *fsm<FlowParams>(kFoParams) = Pk;
    fill_row_tables(Pk.tables, fsm<uint32_t>(kFoStage));
    if (tid < kMaxPicks) fsm<int>(kFoOcnt)[tid] = 0;
    __syncthreads();
    const int nl = Pk.nl;
    for (int li = 0; li < nl; ++li) {
        if (!flow_start(li)) return;
        if ((tid >> 5) == kFlowDecodeWarps) flow_service(li);
        else if (!flow_decode(li)) return;
        if (!flow_combine<MULTI>(li)) return;
    }
    if (nl == 1) {  // h_out may alias h_in: the result went to hbuf[1]; copy once all are in
        const FlowParams& P = fparams();
        const int dim = P.dim, G = gridDim.x;
        bool ok = true;
        if (tid == 0) ok = wait_reached<false>(P.w.cnt + P.nl + P.k * (P.ff >> 8) + P.k, (unsigned)(dim >> 5), P.err);
        if (!__syncthreads_and(ok)) return;
        for (int i = blockIdx.x * kFlowThreads + tid; i < dim; i += G * kFlowThreads) P.h_out[i] = __ldcg(P.w.hbuf + dim + i);
    }
}

size_t flow_smem(int dim, int ff, int k) {
    (void)dim;
    (void)ff;
    (void)k;
    return kFlowSmemBytes;
}

static int flow_grid() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

bool flow_supported(int dim, int ff, int k) {
    int dev = 0, optin = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop || optin <= 0) return false;
    // a down round's picks are staged in shared memory: at most kStageBlocks blocks of h each,
    // and the rounds' pairs (at most kFlowDecodeWarps) span at most kStagePicks picks
    if ((ff >> 8) > kStageBlocks || (dim >> 5) < kFlowDecodeWarps) return false;
    return dim <= kFlowMaxDim && ff >= 256 && k <= kMaxPicks && flow_smem(dim, ff, k) <= (size_t)optin;
}

cudaError_t launch_flow(const ExpertDesc* desc, int E, int first, int nl, int k, const int* route_ids,
                        const float* route_w, const float* h_in, float* h_out, int dim, int ff, float limit,
                        const FlowWork& w, int* err, const StackShard& shard, cudaStream_t s) {
    const uint32_t* tables = nullptr;
    cudaError_t e = tables_device_ptr(&tables);
    if (e != cudaSuccess) return e;
    FlowParams P{};
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
    P.w = w;
    P.err = err;
    P.tables = tables;
    P.sh = shard;
    const size_t sm = flow_smem(dim, ff, k);
    void (*kern)(FlowParams) = shard.world > 1 ? k_flow<true> : k_flow<false>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm))) return e;
    if ((e = cudaMemsetAsync(w.cnt, 0, flow_counter_words(nl, k, ff) * sizeof(unsigned), s))) return e;
    void* args[] = {&P};
    return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(flow_grid()), dim3(kFlowThreads), args, sm, s);
}

}  // namespace clb

#ifdef CLB_FLOW_TRACE
// Copies the phase stamps of the last launches ([64 layers][160 CTAs][8] u64) to host memory.
extern "C" int clb_flow_trace_read(void* host, size_t bytes) {
    if (bytes > sizeof(clb::g_flow_trace)) bytes = sizeof(clb::g_flow_trace);
    return (int)cudaMemcpyFromSymbol(host, clb::g_flow_trace, bytes);
}
extern "C" int clb_flow_trace_clear() {
    static unsigned long long zero[clb::kTraceLayers * clb::kTraceCtas * 8];
    return (int)cudaMemcpyToSymbol(clb::g_flow_trace, zero, sizeof(zero));
}
#endif
