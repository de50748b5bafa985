// Dataflow whole-stack decode kernel (fast summation order): one CTA of 16 warps per SM
// runs every layer of a token; 15 warps decode weights, one "service" warp keeps the
// books. Inside a layer the CTAs take work "rounds" from a counter, in an order fixed on
// the host (the round schedule), and hand results on through completion counters instead
// of meeting at grid barriers between the phases:
//
//   norm      every CTA: sum of squares of h (per 32-row group partials written by the
//             previous layer's combines, added in a fixed order), x = RMSNorm(h), Q8_K(x)
//             into shared memory;
//   gate/up   a round = RGR row groups of 32 rows x {gate, up} x SG K segments (one warp
//             each, one row per lane); the service warp adds the segments in order and
//             applies SwiGLU(g, u) -> gu; the round that completes a 256-row block of a pick
//             quantizes it to Q8_K (hq, hd) and counts the pick's quantized blocks;
//   down      a round = PPR (pick, 32-row group) pairs x SD K segments; the service warp
//             stages the picks' Q8_K(h) in shared memory once they are complete, then adds
//             the segments in order and writes the expert rows (to every GPU of a sharded
//             bank) and counts each row group's rows;
//   combine   CTA c owns row groups c, c + G, ...: once all k picks' rows of a group are
//             in, h += the ascending-id fma combine of the rows (runtime.cpp:184-187),
//             its sum of squares is written, and the layer counter is bumped;
//   -- the next layer starts when every row group is combined (the one grid-wide wait).
//
// While the decoding warps run round i, the service warp finishes round i - 1, grabs
// round i + 2 and prepares round i + 1. The routing of layer l + 1 (ids, weights, the
// experts' descriptors) is read during layer l's combine, off the layer's critical path.
//
// Every wait is bounded (the bank's wait limit, 2^22 polls unless set): a wait that runs
// out sets *err = 2 and the CTA returns, so no launch can hang. Counters that other GPUs
// write (row groups, by layer parity) only grow; the per-launch ones are zeroed by
// launch_flow.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "clb_device.cuh"
#include "clb_kernels.h"
#include "clb_v2.cuh"

namespace clb {

namespace {

constexpr int kFlowDecodeWarps = 15;              // warps that decode weights
constexpr int kFlowWarps = kFlowDecodeWarps + 1;  // + one service warp
constexpr int kFlowThreads = kFlowWarps * 32;
constexpr int kServiceWarp = kFlowDecodeWarps;
constexpr int kErrWait = 2;
constexpr uint32_t kRoundDown = 1u << 30;  // schedule entry: a down round (else gate/up)
constexpr int kNoRound = -1;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
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
__device__ __forceinline__ int ld_acquire_cta_shared(const int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta_shared(int* p, int v) {
    asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Bounded wait until *p has reached target (modulo 2^32). SYS: the writers include other
// GPUs. Polls with relaxed loads (an acquire load per poll would discard the SM's L1 lines
// each time, under the feet of the warps still decoding) and orders the caller's later
// reads after the writes it waited for with one fence once the target is seen (the
// relaxed-load + fence acquire pattern). Backs off after a few hundred polls.
template <bool SYS>
__device__ bool wait_reached(const unsigned* p, unsigned target, int* err, unsigned limit) {
    for (unsigned spins = 0;; ++spins) {
        const unsigned v = SYS ? ld_relaxed_sys(p) : ld_relaxed_gpu(p);
        if ((int)(v - target) >= 0) {
            if (SYS) fence_acq_rel_sys();
            else fence_acq_rel_gpu();
            return true;
        }
        if (spins > limit) {
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
// round of tail. Host only: launch_flow passes the shapes of every pick count.
static FlowShape flow_shape(int kown, int dim, int ff, int grid) {
    const int rgpp = ff >> 5, rgd = dim >> 5, nbx = dim >> 8, nbh = ff >> 8;
    FlowShape best{1, 1, 1, 1, 0, 0};
    long best_cost = -1;
    for (int rgr = 8; rgr >= 1; rgr >>= 1) {
        const int sg = kFlowDecodeWarps / 2 / rgr;
        if (sg < 1 || rgpp % rgr) continue;
        const long ngu = (long)kown * rgpp / rgr, seg_gu = (nbx + sg - 1) / sg;
        for (int sd = 1; sd <= 8; ++sd) {
            const int ppr = kFlowDecodeWarps / sd;
            const long nd = ((long)kown * rgd + ppr - 1) / ppr, seg_d = (nbh + sd - 1) / sd;
            long spread = (ngu * seg_gu + nd * seg_d + grid - 1) / grid;
            if (spread < seg_gu + seg_d) spread = seg_gu + seg_d;
            const long cost = spread + seg_d;
            if (best_cost < 0 || cost < best_cost) {
                best_cost = cost;
                best = FlowShape{rgr, sg, ppr, sd, (int)ngu, (int)nd};
            }
        }
    }
    return best;
}

// Round order of a layer with `kown` picks: every gate/up round (pick-major), with a down
// round moved in as soon as the gate/up rounds of its picks are at least `gap` rounds
// behind it (two waves of the grid: a gate/up round's epilogue runs during its CTA's next
// round), so that it rarely waits for their SwiGLU and Q8_K; the remaining down rounds
// last (the short rounds form the layer's tail).
static void flow_schedule(const FlowShape& F, int kown, int dim, int ff, int gap, std::vector<uint32_t>& out) {
    const int rgpp = ff >> 5, rgd = dim >> 5, npair = kown * rgd;
    std::vector<long> gu_end(kown > 0 ? kown : 1, 0);  // schedule position of each pick's last gate/up round
    std::vector<char> gu_done(kown > 0 ? kown : 1, 0);
    int g = 0, d = 0;
    const size_t base = out.size();
    while (g < F.ngu || d < F.nd) {
        bool take_d = false;
        if (d < F.nd) {
            if (g >= F.ngu) {
                take_d = true;
            } else {
                const int p1 = std::min(npair - 1, d * F.ppr + F.ppr - 1) / rgd;
                take_d = gu_done[p1] && (long)(out.size() - base) >= gu_end[p1] + gap;
            }
        }
        if (take_d) {
            out.push_back(kRoundDown | (uint32_t)d++);
        } else {
            const int last_pick = (g * F.rgr + F.rgr - 1) / rgpp;
            out.push_back((uint32_t)g++);
            if (g == F.ngu || ((g * F.rgr) / rgpp) != last_pick) {  // the pick's gate/up rounds end here
                gu_end[last_pick] = (long)(out.size() - base) - 1;
                gu_done[last_pick] = 1;
            }
        }
    }
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
    unsigned wait_limit;     // polls before a bounded wait gives up
    const uint32_t* tables;
    StackShard sh;
    FlowShape shapes[kMaxPicks + 1];  // round shapes by pick count
};

// Routing of one layer in shared memory (two slots: this layer's and the next's).
struct FlowRoute {
    int ids[kMaxPicks];
    float w[kMaxPicks];
    int ord[kMaxPicks];       // pick slots in ascending expert id order
    int own[kMaxPicks];       // pick slots computed here
    int ocnt[kMaxPicks];      // per slot: layers of this launch (up to this one) it was computed here
    int kown;
    int pad[3];
    ExpertDesc desc[kMaxPicks];
};

// Per-layer control block in shared memory.
struct FlowCtl {
    int ring[3];        // schedule entries of rounds i, i + 1, i + 2 (kNoRound: none left)
    int ready[3];       // down round: 2 when its picks' Q8_K(h) are staged in shared memory
    int dready[3];      // down round staged late by the service warp: (layer << 16) | (i + 1)
    int pad;
};

// Shared memory layout (bytes), fixed for dim <= kFlowMaxDim and k <= kMaxPicks so that
// every address is a constant.
constexpr int kFlowMaxDim = 16384;
constexpr int kStagePicks = 3, kStageBlocks = 16;  // down-round activations staged in shared memory (ff <= 4096)
constexpr uint32_t kFoStage = kRowTableBytes;
constexpr uint32_t kFoXq = kFoStage + kTableWords * 4;
constexpr uint32_t kFoXd = kFoXq + (kFlowMaxDim / 256) * kActStride;
constexpr uint32_t kFoPart = kFoXd + (kFlowMaxDim / 256) * 4;  // [2][decode warps][32] floats
constexpr uint32_t kFoRoute = kFoPart + 2 * kFlowDecodeWarps * 32 * 4;  // [2] FlowRoute
constexpr uint32_t kFoStageH = kFoRoute + 2 * (uint32_t)sizeof(FlowRoute);  // [2][picks][blocks] Q8_K blocks
constexpr uint32_t kFoStageD = kFoStageH + 2 * kStagePicks * kStageBlocks * kActStride;  // [2][picks][blocks]
constexpr uint32_t kFoCtl = kFoStageD + 2 * kStagePicks * kStageBlocks * 4;
constexpr uint32_t kFoParams = (kFoCtl + (uint32_t)sizeof(FlowCtl) + 15u) & ~15u;
constexpr uint32_t kFlowSmemBytes = (kFoParams + (uint32_t)sizeof(FlowParams) + 15u) & ~15u;
static_assert(kFoXq % 16 == 0 && kFoPart % 16 == 0 && kFoRoute % 16 == 0 && kFoStageH % 16 == 0,
              "16-byte aligned regions");
static_assert(sizeof(FlowRoute) % 16 == 0, "route slots stay aligned");
static_assert((kFlowMaxDim >> 5) <= 2 * kFlowDecodeWarps * 32, "the norm's partials fit the round-partial area");

template <class T>
__device__ __forceinline__ T* fsm(uint32_t off) {
    return reinterpret_cast<T*>(clb_dyn_smem + off);
}
__device__ __forceinline__ const FlowParams& fparams() { return *fsm<const FlowParams>(kFoParams); }
__device__ __forceinline__ FlowCtl& fctl() { return *fsm<FlowCtl>(kFoCtl); }
__device__ __forceinline__ FlowRoute& froute(int li) { return fsm<FlowRoute>(kFoRoute)[li & 1]; }

size_t flow_counter_words(int nl_max, int k, int ff) {
    return (size_t)nl_max + (size_t)k * (ff >> 8) + (size_t)k + 1;
}

#ifdef CLB_FLOW_TRACE
// Phase stamps (%globaltimer ns) per (layer, CTA), a build-time option for phase tables:
// 0 layer entry, 1 h ready, 2 norm done, 3 rounds done, 4 combine done, 5 gate/up rounds,
// 6 down rounds, 7 ns warp 0 waited for down-round activations, 8 ns warp 0 decoded,
// 9 ns the service warp worked per round (sum), 10 ns from round start to round start
// (sum, warp 0), 11 ns the service warp spent in gate/up epilogues.
constexpr int kTraceLayers = 64, kTraceCtas = 160, kTraceSlots = 16;
__device__ unsigned long long g_flow_trace[kTraceLayers * kTraceCtas * kTraceSlots];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define FLOW_TRACE(li, slot, v)                                                                                     \
    do {                                                                                                           \
        if ((li) < kTraceLayers && blockIdx.x < kTraceCtas)                                                        \
            g_flow_trace[((li) * kTraceCtas + blockIdx.x) * kTraceSlots + (slot)] = (v);                           \
    } while (0)
#define FLOW_TRACE_ADD(li, slot, v)                                                                                 \
    do {                                                                                                           \
        if ((li) < kTraceLayers && blockIdx.x < kTraceCtas)                                                        \
            g_flow_trace[((li) * kTraceCtas + blockIdx.x) * kTraceSlots + (slot)] += (v);                          \
    } while (0)
#else
#define FLOW_TRACE(li, slot, v) do { } while (0)
#define FLOW_TRACE_ADD(li, slot, v) do { } while (0)
#endif

// Pick-quantization counters: [k] after grab [nl] and the block counters [k][nbh].
__device__ __forceinline__ unsigned* flow_pickq(const FlowParams& P) {
    return P.w.cnt + P.nl + P.k * (P.ff >> 8);
}
__device__ __forceinline__ unsigned* flow_layer_cnt(const FlowParams& P) {
    return P.w.cnt + P.nl + P.k * (P.ff >> 8) + P.k;
}

// Schedule entry `seq` of a layer with `kown` picks here (kNoRound past the end).
__device__ __forceinline__ int flow_round(const FlowParams& P, int kown, unsigned seq) {
    const FlowShape& F = P.shapes[kown];
    if (seq >= (unsigned)(F.ngu + F.nd)) return kNoRound;
    return (int)__ldg(P.w.sched + P.w.sched_off[kown] + seq);
}

// This warp's segment of round entry `e` (nullptr: idle): matrix, row, blocks [b0, b1).
__device__ __forceinline__ const PackedMat* flow_segment(const FlowParams& P, const FlowRoute& rt, int e, int warp,
                                                         int lane, int& row, int& b0, int& b1) {
    if (e < 0) return nullptr;
    const FlowShape& F = P.shapes[rt.kown];
    const int rgpp = P.ff >> 5, rgd = P.dim >> 5, nbx = P.dim >> 8, nbh = P.ff >> 8;
    const int idx = e & (int)(kRoundDown - 1);
    if (!(e & (int)kRoundDown)) {
        const int j = warp / (2 * F.sg), mat = (warp / F.sg) & 1, s = warp % F.sg;
        if (j >= F.rgr) return nullptr;
        const int rgl = idx * F.rgr + j, pick = rt.own[rgl / rgpp];
        row = (rgl % rgpp) * 32 + lane;
        const int per = (nbx + F.sg - 1) / F.sg;
        b0 = min(nbx, s * per);
        b1 = min(nbx, b0 + per);
        return mat ? &rt.desc[pick].up : &rt.desc[pick].gate;
    }
    const int jp = warp / F.sd, s = warp % F.sd, pair = idx * F.ppr + jp;
    if (jp >= F.ppr || pair >= rt.kown * rgd) return nullptr;
    row = (pair % rgd) * 32 + lane;
    const int per = (nbh + F.sd - 1) / F.sd;
    b0 = min(nbh, s * per);
    b1 = min(nbh, b0 + per);
    return &rt.desc[rt.own[pair / rgd]].down;
}

// Picks p0..p1 (indices into own[]) of down round `idx`.
__device__ __forceinline__ void flow_down_picks(const FlowParams& P, const FlowRoute& rt, int idx, int& p0, int& p1) {
    const FlowShape& F = P.shapes[rt.kown];
    const int rgd = P.dim >> 5;
    p0 = idx * F.ppr / rgd;
    p1 = min(rt.kown * rgd - 1, idx * F.ppr + F.ppr - 1) / rgd;
}

// Routing of layer li into its slot (one warp): ids, weights, ascending-id order, the
// picks this GPU computes and their layer counts, the experts' descriptors.
__device__ void flow_load_routing(int li) {
    const FlowParams& P = fparams();
    FlowRoute& rt = froute(li);
    const FlowRoute& prev = froute(li + 1);  // the other slot: layer li - 1 (ignored for li == 0)
    const int lane = threadIdx.x & 31, k = P.k;
    const StackShard& sh = P.sh;
    int e = -1;
    if (lane < k) {
        e = __ldcg(P.route_ids + (size_t)li * k + lane);
        rt.ids[lane] = e;
        rt.w[lane] = __ldcg(P.route_w + (size_t)li * k + lane);
    }
    int rank = 0;
    for (int p = 0; p < k; ++p) rank += __shfl_sync(0xffffffffu, e, p) < e;
    if (lane < k) rt.ord[rank] = lane;
    const bool mine = lane < k && e >= sh.own_begin && e < sh.own_end;
    const uint32_t m = __ballot_sync(0xffffffffu, mine);
    if (mine) rt.own[__popc(m & ((1u << lane) - 1u))] = lane;
    if (lane < kMaxPicks) rt.ocnt[lane] = (li > 0 ? prev.ocnt[lane] : 0) + (mine ? 1 : 0);
    if (lane == 0) rt.kown = __popc(m);
    __syncwarp();
    constexpr int words = (int)(sizeof(ExpertDesc) / 4);
    for (int i = lane; i < k * words; i += 32) {
        const int p = i / words, wd = i - p * words;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(P.desc + (size_t)(P.first + li) * P.E + rt.ids[p]);
        reinterpret_cast<uint32_t*>(rt.desc + p)[wd] = __ldcg(src + wd);
    }
}

// Decoding warps of layer li: one segment per round until the rounds run out. False: a
// bounded wait ran out (the error flag is set).
__device__ __forceinline__ bool flow_decode(int li) {
    const FlowParams& P = fparams();
    const FlowRoute& rt = froute(li);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef CLB_FLOW_TRACE
    unsigned long long t_round = 0;
#endif
    for (int i = 0;; ++i) {
        __syncthreads();  // round i may start (ring, ready and the partial buffer are set)
        const FlowCtl& c = fctl();
        const int e = c.ring[i % 3];
#ifdef CLB_FLOW_TRACE
        const unsigned long long t_sync = gtimer();
        if (warp == 0 && lane == 0 && i > 0) FLOW_TRACE_ADD(li, 10, t_sync - t_round);
        t_round = t_sync;
#endif
        if (e < 0) {
#ifdef CLB_FLOW_TRACE
            if (warp == 0 && lane == 0) FLOW_TRACE(li, 3, gtimer());
#endif
            return true;
        }
        const bool down = (e & (int)kRoundDown) != 0;
#ifdef CLB_FLOW_TRACE
        if (warp == 0 && lane == 0) FLOW_TRACE_ADD(li, down ? 6 : 5, 1ull);
#endif
        int row = 0, b0 = 0, b1 = 0;
        const PackedMat* m = flow_segment(P, rt, e, warp, lane, row, b0, b1);
        if (down && c.ready[i % 3] != 2) {
            // the service warp stages this round's Q8_K(h) once it is complete: wait for it
#ifdef CLB_FLOW_TRACE
            const unsigned long long t0 = gtimer();
#endif
            const int want = (li << 16) | (i + 1);
            int got = 1;
            if (lane == 0)
                for (unsigned spins = 0; ld_acquire_cta_shared(&c.dready[i % 3]) != want; ++spins)
                    if (spins > P.wait_limit) {
                        atomicExch(P.err, kErrWait);
                        got = 0;
                        break;
                    }
            if (!__shfl_sync(0xffffffffu, got, 0)) return false;
#ifdef CLB_FLOW_TRACE
            if (warp == 0 && lane == 0) FLOW_TRACE_ADD(li, 7, gtimer() - t0);
#endif
        }
        {  // this warp's segment of the next round: its first block into L2 behind this round
            int nrow = 0, nb0 = 0, nb1 = 0;
            const PackedMat* nm = flow_segment(P, rt, c.ring[(i + 1) % 3], warp, lane, nrow, nb0, nb1);
            if (nm && nm->body && nb0 < nb1) prefetch_row_block(*nm, nrow, nb0);
        }
        float y = 0.0f;
        if (m) {
            const int dim = P.dim, ff = P.ff;
            const bool shape_ok = m->body != nullptr && (down ? (m->k == ff && m->n == dim) : (m->k == dim && m->n == ff));
            if (!shape_ok) {
                if (lane == 0) atomicExch(P.err, 1);
            } else if (!down) {
                y = lane_row_db_any<kActStride>(*m, row, b0, b1, fsm<int8_t>(kFoXq), fsm<float>(kFoXd));
            } else {
                const FlowShape& F = P.shapes[rt.kown];
                const int rgd = dim >> 5, idx = e & (int)(kRoundDown - 1);
                const int ps = (idx * F.ppr + warp / F.sd) / rgd - idx * F.ppr / rgd, buf = i & 1;
                y = lane_row_db_any<kActStride>(
                    *m, row, b0, b1, fsm<int8_t>(kFoStageH) + ((buf * kStagePicks + ps) * kStageBlocks) * kActStride,
                    fsm<float>(kFoStageD) + (buf * kStagePicks + ps) * kStageBlocks);
            }
        }
        fsm<float>(kFoPart)[((i & 1) * kFlowDecodeWarps + warp) * 32 + lane] = y;
#ifdef CLB_FLOW_TRACE
        if (warp == 0 && lane == 0) FLOW_TRACE_ADD(li, 8, gtimer() - t_sync);
#endif
    }
}

// Service warp of layer li: while the decoding warps run round i it finishes round i - 1
// (epilogue), stages round i's Q8_K(h) if that was not possible earlier, grabs round i + 2
// and stages round i + 1's Q8_K(h) if it is already complete. It issues no prefetches:
// its acquire and release operations would otherwise wait for them.
__device__ __noinline__ void flow_service(int li) {
    const FlowParams& P = fparams();
    const FlowRoute& rt = froute(li);
    FlowCtl& c = fctl();
    const int lane = threadIdx.x & 31;
    const int dim = P.dim, ff = P.ff, k = P.k, nbh = ff >> 8, nrg = dim >> 5, rgpp = ff >> 5;
    const FlowShape F = P.shapes[rt.kown];
    const int npair = rt.kown * nrg;
    unsigned* blk = P.w.cnt + P.nl;
    unsigned* pickq = flow_pickq(P);
    const StackShard& sh = P.sh;
    const unsigned lg = sh.epoch + (unsigned)li;
    const int par = (int)(lg & 1u);
    float* ybuf = sh.yx + (size_t)par * k * dim;
    unsigned* rgc = sh.rgcnt + (size_t)par * nrg;
    unsigned* grab = P.w.cnt + li;

    // Stage the Q8_K(h) blocks of down round entry e into stage buffer `buf`: if `wait`,
    // after waiting (bounded) until each pick is complete; else only if all are complete
    // already (one acquire sample each). Returns 2 when staged, 0 when not, -1 on a timeout.
    auto stage = [&](int e, int buf, bool wait) -> int {
        if (e < 0 || !(e & (int)kRoundDown)) return 0;
        int p0, p1;
        flow_down_picks(P, rt, e & (int)(kRoundDown - 1), p0, p1);
        for (int pi = p0; pi <= p1; ++pi) {
            const int slot = rt.own[pi];
            const unsigned target = (unsigned)nbh * (unsigned)rt.ocnt[slot];
            int ok = 1;
            if (lane == 0) {
                if (wait) ok = wait_reached<false>(pickq + slot, target, P.err, P.wait_limit) ? 1 : -1;
                else ok = (int)(ld_acquire_gpu(pickq + slot) - target) >= 0 ? 1 : 0;
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok <= 0) return ok;
        }
        for (int pi = p0; pi <= p1; ++pi) {
            const int slot = rt.own[pi], ps = pi - p0;
            int8_t* dq = fsm<int8_t>(kFoStageH) + ((buf * kStagePicks + ps) * kStageBlocks) * kActStride;
            const uint4* sq = reinterpret_cast<const uint4*>(P.w.hq + (size_t)slot * ff);
            for (int c2 = lane; c2 < nbh * 16; c2 += 32)
                *reinterpret_cast<uint4*>(dq + (c2 >> 4) * kActStride + (c2 & 15) * 16) = __ldcg(sq + c2);
            if (lane < nbh)
                fsm<float>(kFoStageD)[(buf * kStagePicks + ps) * kStageBlocks + lane] =
                    __ldcg(P.w.hd + (size_t)slot * nbh + lane);
        }
        return 2;
    };
    {
        const int rdy = stage(c.ring[0], 0, false);
        if (lane == 0) c.ready[0] = rdy;
    }
    int eprev = kNoRound;
    for (int i = 0;; ++i) {
        __syncthreads();
        const int e = c.ring[i % 3], en = c.ring[(i + 1) % 3];
        const float* pb = fsm<float>(kFoPart) + ((i - 1) & 1) * kFlowDecodeWarps * 32;
#ifdef CLB_FLOW_TRACE
        const unsigned long long t_sync = gtimer();
#endif
        if (eprev >= 0 && !(eprev & (int)kRoundDown)) {
            // gate/up epilogue: add the segments in order, SwiGLU; the round that completes a
            // 256-row block of a pick quantizes it to Q8_K
            const int idx = eprev;
            for (int j = 0; j < F.rgr; ++j) {
                const int rgl = idx * F.rgr + j, slot = rt.own[rgl / rgpp], rgi = rgl % rgpp;
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
#ifdef CLB_FLOW_TRACE
            if (lane == 0) FLOW_TRACE_ADD(li, 11, gtimer() - t_sync);
#endif
        } else if (eprev >= 0) {
            // down epilogue: add each pair's segments in order, store the expert rows (also
            // into every peer's slot of this layer parity), count the row group
            const int idx = eprev & (int)(kRoundDown - 1);
            for (int jp = 0; jp < F.ppr; ++jp) {
                const int pair = idx * F.ppr + jp;
                if (pair >= npair) break;
                const int slot = rt.own[pair / nrg], rgi = pair % nrg;
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
        if (e < 0) return;
        if ((e & (int)kRoundDown) && c.ready[i % 3] != 2) {
            // round i's picks were not complete when sampled: wait, stage, release the decoders
            if (stage(e, i & 1, true) < 0) return;  // timed out (error flag set): decoders time out too
            __syncwarp();
            if (lane == 0) st_release_cta_shared(&c.dready[i % 3], (li << 16) | (i + 1));
        }
        unsigned seq = 0;
        if (lane == 0) seq = atomicAdd(grab, 1u);
        const int rdy = stage(en, (i + 1) & 1, false);
        seq = __shfl_sync(0xffffffffu, seq, 0);
        if (lane == 0) {
            c.ring[(i + 2) % 3] = flow_round(P, rt.kown, seq);
            c.ready[(i + 1) % 3] = rdy;
#ifdef CLB_FLOW_TRACE
            FLOW_TRACE_ADD(li, 9, gtimer() - t_sync);
#endif
        }
        eprev = e;
    }
}

// Start of layer li (all warps): wait until every row group of the previous layer is
// combined, then RMSNorm + Q8_K(x) into shared memory (the routing is already in its
// slot). False: a bounded wait ran out.
__device__ __noinline__ bool flow_start(int li) {
    const FlowParams& P = fparams();
    FlowCtl& ctl = fctl();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int dim = P.dim, nbx = dim >> 8, nrg = dim >> 5;
    const float* hsrc = li == 0 ? P.h_in : P.w.hbuf + (size_t)(li & 1) * dim;
    int8_t* xq = fsm<int8_t>(kFoXq);
    float* xd = fsm<float>(kFoXd);

    int ok = 1;
#ifdef CLB_FLOW_TRACE
    if (tid == 0) FLOW_TRACE(li, 0, gtimer());
#endif
    if (warp == kServiceWarp && lane == 0) {
        const int kown = froute(li).kown;
        ctl.ring[0] = flow_round(P, kown, atomicAdd(P.w.cnt + li, 1u));
        ctl.ring[1] = flow_round(P, kown, atomicAdd(P.w.cnt + li, 1u));
        if (li > 0) ok = wait_reached<false>(flow_layer_cnt(P), (unsigned)nrg * (unsigned)li, P.err, P.wait_limit);
    }
    if (!__syncthreads_and(ok)) return false;
#ifdef CLB_FLOW_TRACE
    if (tid == 0) FLOW_TRACE(li, 1, gtimer());
#endif
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
// buffers (the last layer writes h_out), then the layer counter. Warp 1 then reads the
// next layer's routing into the other slot. False: a wait ran out.
template <bool MULTI>
__device__ __noinline__ bool flow_combine(int li) {
    const FlowParams& P = fparams();
    const FlowRoute& rt = froute(li);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dim = P.dim, k = P.k, nrg = dim >> 5, G = gridDim.x;
    const StackShard& sh = P.sh;
    const float* hsrc = li == 0 ? P.h_in : P.w.hbuf + (size_t)(li & 1) * dim;
    const unsigned lg = sh.epoch + (unsigned)li;
    const int par = (int)(lg & 1u);
    const float* ybuf = sh.yx + (size_t)par * k * dim;
    unsigned* rgc = sh.rgcnt + (size_t)par * nrg;
    const bool last = li == P.nl - 1;
    const unsigned tgt = (unsigned)k * ((lg >> 1) + 1u);
    int wok = 1;
    for (int rg = blockIdx.x + warp * G; rg < nrg; rg += kFlowWarps * G) {
        int got = 1;
        if (lane == 0)
            got = MULTI ? wait_reached<true>(rgc + rg, tgt, P.err, P.wait_limit)
                        : wait_reached<false>(rgc + rg, tgt, P.err, P.wait_limit);
        if (!__shfl_sync(0xffffffffu, got, 0)) {
            wok = 0;
            break;
        }
        float acc = 0.0f;
        for (int o = 0; o < k; ++o) {
            const int p = rt.ord[o];
            acc = __fmaf_rn(rt.w[p], __ldcg(ybuf + (size_t)p * dim + rg * 32 + lane), acc);
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
        if (lane == 0) red_release_gpu(flow_layer_cnt(P), 1u);
    }
    if (warp == 1 && wok && li + 1 < P.nl) flow_load_routing(li + 1);
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
    // shared memory keeps an earlier launch's bytes: stamps of that launch's (layer, round)
    // pairs must not read as this launch's
    if (tid < 3) fctl().dready[tid] = -1;
    fill_row_tables(Pk.tables, fsm<uint32_t>(kFoStage));
    __syncthreads();
    if ((tid >> 5) == 1) flow_load_routing(0);
    __syncthreads();
    const int nl = Pk.nl;
    for (int li = 0; li < nl; ++li) {
        if (!flow_start(li)) return;
        if ((tid >> 5) == kServiceWarp) flow_service(li);
        else if (!flow_decode(li)) return;
        if (!flow_combine<MULTI>(li)) return;
    }
    if (nl == 1) {  // h_out may alias h_in: the result went to hbuf[1]; copy once all are in
        const FlowParams& P = fparams();
        const int dim = P.dim, G = gridDim.x;
        int ok = 1;
        if (tid == 0) ok = wait_reached<false>(flow_layer_cnt(P), (unsigned)(dim >> 5), P.err, P.wait_limit);
        if (!__syncthreads_and(ok)) return;
        for (int i = blockIdx.x * kFlowThreads + tid; i < dim; i += G * kFlowThreads)
            P.h_out[i] = __ldcg(P.w.hbuf + dim + i);
    }
}

size_t flow_smem(int dim, int ff, int k) {
    (void)dim;
    (void)ff;
    (void)k;
    return kFlowSmemBytes;
}

int flow_grid() {
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
    // a down round's picks are staged in shared memory: at most kStageBlocks blocks of h
    // each, and the rounds' pairs (at most kFlowDecodeWarps) span at most kStagePicks picks
    if ((ff >> 8) > kStageBlocks || (dim >> 5) < kFlowDecodeWarps) return false;
    return dim <= kFlowMaxDim && ff >= 256 && k <= kMaxPicks && flow_smem(dim, ff, k) <= (size_t)optin;
}

std::vector<uint32_t> flow_schedule_table(int dim, int ff, int k, int grid, uint32_t* offsets) {
    std::vector<uint32_t> tab;
    for (int kown = 0; kown <= k; ++kown) {
        offsets[kown] = (uint32_t)tab.size();
        flow_schedule(flow_shape(kown, dim, ff, grid), kown, dim, ff, 2 * grid, tab);
    }
    offsets[k + 1] = (uint32_t)tab.size();
    return tab;
}

cudaError_t launch_flow(const ExpertDesc* desc, int E, int first, int nl, int k, const int* route_ids,
                        const float* route_w, const float* h_in, float* h_out, int dim, int ff, float limit,
                        const FlowWork& w, int* err, unsigned wait_limit, const StackShard& shard, cudaStream_t s) {
    const uint32_t* tables = nullptr;
    cudaError_t e = tables_device_ptr(&tables);
    if (e != cudaSuccess) return e;
    if (w.sched == nullptr) return cudaErrorInvalidValue;
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
    P.wait_limit = wait_limit;
    P.tables = tables;
    P.sh = shard;
    const int grid = flow_grid();
    for (int kown = 0; kown <= k; ++kown) P.shapes[kown] = flow_shape(kown, dim, ff, grid);
    const size_t sm = flow_smem(dim, ff, k);
    void (*kern)(FlowParams) = shard.world > 1 ? k_flow<true> : k_flow<false>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm))) return e;
    if ((e = cudaMemsetAsync(w.cnt, 0, flow_counter_words(nl, k, ff) * sizeof(unsigned), s))) return e;
    void* args[] = {&P};
    return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(grid), dim3(kFlowThreads), args, sm, s);
}

}  // namespace clb

#ifdef CLB_FLOW_TRACE
// Copies the phase stamps of the last launches ([64 layers][160 CTAs][16] u64) to host memory.
extern "C" int clb_flow_trace_read(void* host, size_t bytes) {
    if (bytes > sizeof(clb::g_flow_trace)) bytes = sizeof(clb::g_flow_trace);
    return (int)cudaMemcpyFromSymbol(host, clb::g_flow_trace, bytes);
}
extern "C" int clb_flow_trace_clear() {
    static unsigned long long zero[clb::kTraceLayers * clb::kTraceCtas * clb::kTraceSlots];
    return (int)cudaMemcpyToSymbol(clb::g_flow_trace, zero, sizeof(zero));
}
#endif
