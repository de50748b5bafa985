// Batched prefill through one routed-expert layer: the T x k picks of T tokens are grouped
// per expert and each expert's FFN runs as two grouped tensor-core GEMMs over its tokens
// (gate/up over Q8_K(x), then down over Q8_K(h)), followed by the per-token combine in
// ascending expert id (engine/strata/warm/runtime.cpp:184-187 applied to every token).
// Experts with at most kPfColdMax picks skip the GEMMs: their (expert, token) pairs run the
// decode kernels' one-row-per-lane row dots instead (k_pairs_*), which cost a third of the
// GEMM decoder per weight. The same layer serves the batched stack decode (T tokens, one per
// sequence, through consecutive layers: launch_stack_batch, with the stack's fixed-order
// RMSNorm fused into Q8_K of x) and its expert-ID shards (picks outside [e_begin, e_end)
// skipped, their rows zero, for a sum over the GPUs).
//
// Arithmetic. Per 256-value block b the reference forms exact integers
// sum_k w_int[k] * q[k] (q8k_core.hpp:43-91) with q the Q8_K activation (|q| <= 127, exact
// in fp16) and w_int an exact fp16 integer for every expert type:
//   IQ2_XXS  w_int = (2s+1) * sign * mag, mag in {8, 25, 43}, one s per 32 values (<= 1333);
//   IQ2_XS   the same with one s per 16 values (scale bytes of the sc plane);
//   IQ1_M    w_int = (2s+1) * (8 g + delta), g in {-1, 0, 1}, delta = +-1 per 8 values, one
//            3-bit s per 16 values (<= 135): the reference's main sum plus 1/8 of its delta
//            sum (q8k_core.hpp:79-84) is 1/8 of this integer's sum.
// tcgen05.mma (kind::f16, fp32 accumulators in tensor memory) forms that block sum for a
// 128-row x N-token tile (exactly while partial sums stay below 2^24, which the Q8_K value
// ranges of real activations keep them); the epilogue adds (d_w[row, b] * d_x[token, b]) *
// sum_b into fp32 registers block by block and scales by 1/8 at the end. Per (token, row)
// that is the decode kernels' fast order.
//
// Data layout. The picks are grouped by expert into a list of slots (t*k + p), each
// expert's run padded to a multiple of 16 entries; activations are gathered into list
// order once (fp16 Q8_K values [list][K], scales [K/256][list]), so the token rows of a
// tile are contiguous. Gate/up outputs and Q8_K(h) stay in list order; the down GEMM
// writes expert rows by slot for the combine. Padding entries are never written: a tile
// reads them into MMA columns (tokens) whose results it never stores, and the columns of
// an MMA do not mix.
//
// GEMM kernel: one CTA per SM, persistent over tiles (expert, 128 weight rows, up to 48
// list entries), warp-specialised around one pipeline of 256-value K blocks (4 stages of 64)
// that runs across tiles; roles hand blocks to each other through mbarriers, one wait and
// one arrival per block:
//  * weight warp: bulk copies (cp.async.bulk) of the packed weight pieces of a block
//    (16 B per row and piece, 4 pieces for IQ2, 3 for IQ1_M) and of the rows' block scales
//    (d plane, sc plane), two blocks ahead;
//  * B warp: the B operand of a block by TMA (2-D tensor map over the list-order
//    activations, 128-byte swizzle, box height = the tile's entries rounded up to 16), two
//    blocks deep, and each tile's activation scales;
//  * MMA warp: 16 tcgen05.mma per block (A from tensor memory, B from shared memory) into
//    one of kPfAcc block accumulators, then one commit that frees the block's operands and
//    one that hands the accumulator to the epilogue;
//  * 8 decoder warps: each thread turns one 32-weight chunk of one row per stage into exact
//    fp16 integers and stores them to the A operand in tensor memory (tcgen05.st, row m in
//    lane m, values k, k+1 in one column; two blocks of buffers), two 32-column stores per
//    block; the matrix type is uniform per warp (a warp's 32 rows are all gate, all up or
//    all down rows of one expert);
//  * 8 epilogue warps (tensor-memory lane quarter x 32 columns): per block, D * d_w * d_x
//    added into running tile sums that also live in tensor memory; the tile's last block
//    writes the rows out.
// Tile information (types; first entry, entries, row tile; MMA width) reaches the consumer
// roles through 16-byte shared-memory headers released by the same mbarrier arrive as the
// data, so no consumer warp loads from global memory per tile. The kernel is instantiated
// per set of weight types present in the layer (TYPES), so a single-type layer decodes
// without a type dispatch.
// Control loops keep ring positions as counters (no divisions in the per-block path).
// Waits sleep in mbarrier.try_wait (suspend hint) rather than spin, and are bounded in time:
// on time-out the CTA flags *err and an abort flag that ends every loop, lets copies in
// flight land, waits (bounded) for its MMAs and frees its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "clb_device.cuh"
#include "clb_kernels.h"
#include "clb_v2.cuh"

namespace clb {

namespace {

constexpr int kPfDecWarps = 8;                // warp w: TMEM lane quarter w & 3, 32-value chunk w >> 2 of a stage
constexpr int kPfEpiWarps = 8;                // warp kPfDecWarps + w: lane quarter w & 3, 32 columns from 32 (w >> 2)
constexpr int kPfEpiWarp0 = kPfDecWarps;
constexpr int kPfProducerWarp = kPfDecWarps + kPfEpiWarps, kPfMmaWarp = kPfProducerWarp + 1, kPfBWarp = kPfProducerWarp + 2;
constexpr int kPfThreads = 32 * (kPfDecWarps + kPfEpiWarps + 3);
constexpr int kPfMaxN = 48;                   // list entries per tile (MMA N <= 48)
constexpr int kPfStageK = 64;                 // K values per stage (4 MMAs of K = 16); 4 stages per block
constexpr int kPfRawStage = 128 * 16;         // one 16-byte piece per weight row
constexpr int kPfRawSc = 4 * kPfRawStage;     // then the rows' 8 sc bytes (IQ2_XS, IQ1_M)
constexpr int kPfRawHdr = kPfRawSc + 128 * 8; // then a 16-byte header: the tile's packed types (word 0)
constexpr int kPfRawBlock = kPfRawHdr + 128;  // ~9 KB per block, 128-byte aligned (IQ1_M fills 3 of the 4 piece slots)
constexpr int kPfBStage = kPfMaxN * 128;      // 48 rows x 64 fp16, 128-byte swizzled
constexpr int kPfBBlock = 4 * kPfBStage;
constexpr int kPfMaxNb = 32;                  // K <= 8192
constexpr int kPfAcc = 3;                     // block accumulators (64 columns each, from column 0)
constexpr int kPfAccCols = 64;
constexpr int kPfDxsStride = 64;              // floats per block row of a tile's activation scales
constexpr int kPfDwRing = 8;                  // row-scale ring (blocks)
constexpr int kPfDwHdr = 256 + 128 * 8;       // per block: fp16 d of 128 rows, 8 sc bytes per row (IQ1_M),
constexpr int kPfDwSlot = kPfDwHdr + 128;     // then a header {first, entries, mt, types} of the block's tile
constexpr int kPfTmemCols = 512;
constexpr uint32_t kPfRCol = kPfAcc * kPfAccCols;       // running tile sums (64 columns)
constexpr uint32_t kPfACol = 256;                       // A operand: 2 blocks x 128 columns
// A operand of a block: the 16-value slice j (0-3) of stage q (0-3) sits at columns 32 j + 8 q, so
// the four stages of one slice are 32 contiguous columns (one tcgen05.st per decoder thread).
static_assert(kPfMaxN <= kPfAccCols && kPfMaxN <= kPfDxsStride && kPfMaxN % 16 == 0, "tile width");
static_assert(kPfRCol + kPfAccCols <= kPfACol && kPfACol + 8 * 32 <= kPfTmemCols, "tensor memory budget");
constexpr uint32_t kPfSpin = 1u << 22;        // drain wait polls
constexpr uint32_t kPfSuspendNs = 20000;      // try_wait suspend hint
constexpr uint64_t kPfTimeoutNs = 1000000000; // 1 s: a pipeline wait longer than this is an error
constexpr int kErrPrefillWait = 3;
constexpr int kPfColdMax = 2;                 // experts with at most this many picks take the row-dot path

// Values biased by +128 so that 0x64XX = 1024 + XX as fp16. IQ2: +8, +25, +43 and -8, -25, -43
// (selector nibble: symbol, bit 2 the sign). IQ1_M: 8 g + delta for g = -1, 0, +1 (symbol
// 0, 1, 2) with delta = +1 (kIq1Pos) or -1 (kIq1Neg).
constexpr uint32_t kPos2b = 0x00AB9988u;
constexpr uint32_t kNeg2b = 0x00556778u;
constexpr uint32_t kIq1Pos = 0x00898179u;
constexpr uint32_t kIq1Neg = 0x00877F77u;

// mbarriers; operand rings hold two blocks, each synchronised once per block
enum : int {
    kRawFull = 0,                      // [2] weight pieces of a block landed
    kRawEmpty = kRawFull + 2,          // [2] decoded
    kDwFull = kRawEmpty + 2,           // [kPfDwRing] row scales of a block landed
    kDwEmpty = kDwFull + kPfDwRing,    // [kPfDwRing] read by the epilogue
    kBFull = kDwEmpty + kPfDwRing,     // [2] B operand of a block landed
    kAFull = kBFull + 2,               // [2] A operand of a block stored
    kBlockDone = kAFull + 2,           // [2] MMAs of a block complete: its A and B buffers are free
    kAccFull = kBlockDone + 2,         // [kPfAcc]
    kAccEmpty = kAccFull + kPfAcc,     // [kPfAcc]
    kDxsFull = kAccEmpty + kPfAcc,     // [2] a tile's activation scales landed
    kDxsEmpty = kDxsFull + 2,          // [2]
    kDrain = kDxsEmpty + 2,
    kNumBars = kDrain + 1
};
__host__ __device__ constexpr uint32_t pf_bar_count(int i) {
    return ((i >= kRawEmpty && i < kRawEmpty + 2) || (i >= kAFull && i < kAFull + 2)) ? kPfDecWarps
           : ((i >= kDwEmpty && i < kDwEmpty + kPfDwRing) || (i >= kAccEmpty && i < kAccEmpty + kPfAcc) ||
              (i >= kDxsEmpty && i < kDxsEmpty + 2))
               ? kPfEpiWarps
               : 1;
}

struct PfSmem {
    // [0, 128K) decode tables of the three types; the B ring starts at the first 1024-byte
    // boundary after them
    static constexpr uint32_t braw = kRowTableBytes;                       // + alignment pad
    static constexpr uint32_t raw = braw + 1024 + 2 * kPfBBlock;           // weight pieces, 2 blocks
    static constexpr uint32_t dw = raw + 2 * kPfRawBlock;                  // [kPfDwRing][kPfDwSlot] row scales
    static constexpr uint32_t dxs = dw + kPfDwRing * kPfDwSlot;            // [2][kPfMaxNb][kPfDxsStride] floats
    static constexpr uint32_t bhdr = dxs + 2 * kPfMaxNb * kPfDxsStride * 4;  // [2] MMA width of a B block
    static constexpr uint32_t bars = bhdr + 16;
    static constexpr uint32_t tslot = bars + kNumBars * 8;
    static constexpr uint32_t abort_flag = tslot + 4;
    static constexpr uint32_t total = abort_flag + 12;
};
static_assert(PfSmem::raw % 16 == 0 && PfSmem::dw % 16 == 0 && PfSmem::dxs % 16 == 0 && PfSmem::bars % 8 == 0,
              "aligned regions");
static_assert(kPfBStage % 1024 == 0 && 2944 * 4 <= 2 * kPfRawBlock, "swizzle atoms; table staging area");
static_assert(PfSmem::total + 16 <= 227 * 1024, "fits one CTA per SM with the 16 bytes of static prmt tables");

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t pf_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes or the hint
// elapses instead of spinning (spinning warps would take issue slots from the decoders).
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kPfSuspendNs)
        : "memory");
    return done != 0;
}
// Bounded wait (kPfTimeoutNs); gives up early once another thread has raised the abort flag.
__device__ __noinline__ bool pf_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    const uint64_t t0 = pf_now_ns();
    for (;;) {
        if (mbar_try_sleep(bar, parity)) return true;
        if (*abort_flag) return false;
        if (pf_now_ns() - t0 > kPfTimeoutNs) break;
    }
    atomicExch(err, kErrPrefillWait);
    *abort_flag = 1;
    return false;
}
__device__ __forceinline__ bool pf_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    return mbar_try(bar, parity) || pf_wait_slow(bar, parity, abort_flag, err);
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// D (+)= A . B^T with A in tensor memory and B described by a shared-memory descriptor.
template <bool ACCUMULATE>
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc) {
    if (ACCUMULATE)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
            "r"(a), "l"(bdesc), "r"(idesc)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
            "r"(a), "l"(bdesc), "r"(idesc)
            : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Four biased bytes (value + 128) -> four fp16 (value * scale), exact because |value * scale|
// <= 1333: (1024 + byte) * scale - 1152 * scale in one fused rounding (1152 * scale is exact
// in fp16 for every odd scale <= 31).
__device__ __forceinline__ void biased4_to_half(uint32_t w, __half2 s2, __half2 noff, uint32_t& h01, uint32_t& h23) {
    const uint32_t a = __byte_perm(w, 0x64646464u, 0x5140), b = __byte_perm(w, 0x64646464u, 0x7362);
    const __half2 ra = __hfma2(*reinterpret_cast<const __half2*>(&a), s2, noff);
    const __half2 rb = __hfma2(*reinterpret_cast<const __half2*>(&b), s2, noff);
    h01 = *reinterpret_cast<const uint32_t*>(&ra);
    h23 = *reinterpret_cast<const uint32_t*>(&rb);
}

// One block of a decoder thread: its 32-value chunk c = 2q + dc of each stage q as exact fp16
// integers, stored to the A operand as two 32-column slices (values 0-15 and 16-31 of the
// chunks). cw: IQ2 types, words 2c and 2c+1 of the block body per stage (cw[2q], cw[2q+1]);
// IQ1_M, the qs word of chunk c (cw[q]) and its 4 qh nibbles (cw[4 + q]). s2[q] / nf[q]:
// the odd sub-scales of values 0-15 (low half) and 16-31 (high half) of chunk c, and
// -1152 times them. lb = lane * 4 (the lane's copy in the replicated tables).
template <int T>
__device__ __forceinline__ void pf_decode_block(const uint32_t (&cw)[8], const __half2 (&s2)[4],
                                                const __half2 (&nf)[4], uint32_t lb, uint32_t taddr) {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        uint32_t v[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // IQ2_XXS: one scale for the chunk (both halves of s2 equal)
            const __half2 s = T == CLB_IQ2_XXS ? s2[q] : jj ? __high2half2(s2[q]) : __low2half2(s2[q]);
            const __half2 n = T == CLB_IQ2_XXS ? nf[q] : jj ? __high2half2(nf[q]) : __low2half2(nf[q]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t grp = 2 * jj + h;  // 8-value group of the chunk
                uint32_t lo, hi;
                if (T == CLB_IQ2_XXS) {
                    const uint32_t selj = 0x5504u | (grp << 4);  // byte grp * 256 + lb
                    const uint32_t sel = tab32(kRowTabXXS + prmt2(cw[2 * q], lb, selj)) |
                                         tab32(kRowTabXXS + 128 + prmt2(cw[2 * q + 1], lb, selj));
                    lo = prmt_sel(kPos2b, kNeg2b, sel);
                    hi = prmt_sel(kPos2b, kNeg2b, sel >> 16);
                } else if (T == CLB_IQ2_XS) {
                    const uint32_t w = cw[2 * q + jj];
                    const uint32_t code = h ? (w >> 16) : (w & 0xffffu);  // 9-bit grid index, 7-bit sign index
                    const uint32_t sel = tab32(kRowTabXS + (code & 511u) * 64u + (lb & 60u)) |
                                         tab32(kRowTabXXS + (code >> 9) * 256u + 128u + lb);
                    lo = prmt_sel(kPos2b, kNeg2b, sel);
                    hi = prmt_sel(kPos2b, kNeg2b, sel >> 16);
                } else {
                    const uint32_t nib = (cw[4 + q] >> (4 * grp)) & 15u;
                    const uint32_t idx = ((cw[q] >> (8 * grp)) & 0xffu) | ((nib & 7u) << 8);
                    const uint32_t sel = tab32(kRowTabIQ1 + idx * 16u + (lb & 12u));
                    const uint32_t src = (nib & 8u) ? kIq1Neg : kIq1Pos;
                    lo = prmt_sel(src, 0u, sel);
                    hi = prmt_sel(src, 0u, sel >> 16);
                }
                biased4_to_half(lo, s, n, v[8 * q + 4 * h], v[8 * q + 4 * h + 1]);
                biased4_to_half(hi, s, n, v[8 * q + 4 * h + 2], v[8 * q + 4 * h + 3]);
            }
        }
        tmem_st32(taddr + (uint32_t)jj * 32u, v);
    }
}

// fp16 block scale of an IQ1_M row from its four scale words (top nibbles), as a float.
__device__ __forceinline__ float iq1m_scale(uint2 sc) {
    const uint32_t h = ((sc.x & 0xffffu) >> 12) | ((sc.x >> 24) & 0xf0u) | (((sc.y & 0xffffu) >> 4) & 0xf00u) |
                       ((sc.y >> 16) & 0xf000u);
    return __half2float(__ushort_as_half((uint16_t)h));
}

__host__ __device__ constexpr int pf_type_bit(int type) {
    return type == CLB_IQ2_XXS ? kTypeBitXXS : type == CLB_IQ2_XS ? kTypeBitXS : type == CLB_IQ1_M ? kTypeBitIQ1M : 0;
}

// Type of the matrix that supplies a warp's 32 rows (lane quarter `quarter`) of a tile, from
// the tile's packed types (gate | up << 8 | down << 16).
__device__ __forceinline__ int pf_row_type(int types, int role, int quarter) {
    return (types >> (role == 0 ? (quarter < 2 ? 0 : 8) : 16)) & 0xff;
}

// Position in a ring of R slots: slot, the parity of the slot's current use, and how many
// times the ring has wrapped.
template <int R>
struct Ring {
    int slot = 0;
    uint32_t phase = 0;
    int round = 0;
    __device__ __forceinline__ void next() {
        if (++slot == R) {
            slot = 0;
            phase ^= 1u;
            ++round;
        }
    }
};

}  // namespace

struct PrefillGemm {
    CUtensorMap bmaps[kPfMaxN / 16];  // B rows of the activations [P][K] fp16, box 64 x 16(i+1)
    const ExpertDesc* desc;           // this layer's descriptors [E]
    int role;                         // 0: gate + up (64 rows of each per tile), 1: down (128 rows)
    const int4* tiles;                // (expert, first list entry, entries, 0) per chunk of an expert's run
    const int* ntiles;                // chunks
    const int* list;                  // slot (t * k + p) per list entry, -1 for padding
    const float* actd;                // activation Q8_K scales [K/256][P]
    int P;                            // list length (multiple of 16)
    int K, nrows, mtiles;             // K, rows of one weight matrix, 128-row tiles per chunk
    float* out;                       // role 0: [P][2][ff] in list order; role 1: [T*k][dim] by slot
    int* err;
    const uint32_t* tables;
};

struct PfTile {
    int e, mt, first, ntok;
};
__device__ __forceinline__ PfTile pf_tile(const PrefillGemm& G, int i) {  // CTA-local tile i
    const int t = blockIdx.x + i * gridDim.x;
    const int4 c = G.tiles[t / G.mtiles];
    return PfTile{c.x, t % G.mtiles, c.y, c.z};
}

// TYPES: the weight types this instantiation decodes (kTypeBitXXS | kTypeBitXS | kTypeBitIQ1M);
// a layer whose experts share one type runs the instantiation for that type alone.
template <int TYPES>
__global__ void __launch_bounds__(kPfThreads, 1) k_prefill_gemm(const __grid_constant__ PrefillGemm G) {
    uint8_t* sm = clb_dyn_smem;
    const uint32_t sbase = smem_u32(sm);
    const uint32_t sb0 = (sbase + PfSmem::braw + 1023u) & ~1023u;  // B ring (1024-byte aligned for the swizzle)
    const uint32_t sraw = sbase + PfSmem::raw, sdw = sbase + PfSmem::dw, sdxs = sbase + PfSmem::dxs;
    const uint32_t bar0 = sbase + PfSmem::bars;
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + PfSmem::abort_flag);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = G.K >> 8, S = nb * (256 / kPfStageK);
    const int ntot = *G.ntiles * G.mtiles;
    const int my_tiles = (int)blockIdx.x < ntot ? (ntot - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my_tiles * S;  // stages of this CTA

    fill_row_tables(G.tables, reinterpret_cast<uint32_t*>(sm + PfSmem::raw));  // staged in the weight ring
    if (tid == 0) {
        for (int i = 0; i < kNumBars; ++i) mbar_init(bar(i), pf_bar_count(i));
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + PfSmem::tslot),
                     "r"(kPfTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + PfSmem::tslot);

    const int nblk = total / 4;
    if (warp == kPfProducerWarp) {
        // ---------------- weight pieces and row scales, two blocks ahead ----------------
        if (lane == 0 && total > 0) {
            Ring<2> rr;
            Ring<kPfDwRing> dr;
            int tile = 0, b = 0;
            bool ok = false;
            const uint8_t *pa0 = nullptr, *pa1 = nullptr, *ps0 = nullptr, *ps1 = nullptr;
            const uint16_t *pd0 = nullptr, *pd1 = nullptr;
            int np0 = 4, np1 = 4;
            size_t plane = 0, n = 0;
            uint32_t raw_tx = 0, dw_tx = 0;
            int4 hdr = make_int4(0, 0, 0, 0);
            const bool split = G.role == 0;  // 64 gate rows + 64 up rows per tile
            const uint32_t rb = split ? 64u : 128u;
            auto fits = [&](const PackedMat& m) {
                return m.body && m.k == G.K && (pf_type_bit(m.type) & TYPES) &&
                       (m.type == CLB_IQ2_XXS ? m.d != nullptr
                        : m.type == CLB_IQ2_XS ? (m.d != nullptr && m.sc != nullptr)
                                               : (m.type == CLB_IQ1_M && m.sc != nullptr));
            };
            for (int blk = 0; blk < nblk; ++blk) {
                if (b == 0) {  // tile setup
                    const PfTile t = pf_tile(G, tile);
                    const ExpertDesc& ex = G.desc[t.e];
                    const PackedMat& m0 = split ? ex.gate : ex.down;
                    const PackedMat& m1 = split ? ex.up : ex.down;
                    const int row0 = (int)rb * t.mt;
                    ok = fits(m0) && fits(m1) && m0.n == m1.n && row0 + (int)rb <= m0.n;
                    if (!ok) atomicExch(G.err, 1);
                    hdr = make_int4(t.first, t.ntok, t.mt,
                                    (ex.gate.type & 0xff) | ((ex.up.type & 0xff) << 8) | ((ex.down.type & 0xff) << 16));
                    n = (size_t)m0.n;
                    plane = n * 16;
                    np0 = m0.type == CLB_IQ1_M ? 3 : 4;
                    np1 = m1.type == CLB_IQ1_M ? 3 : 4;
                    pa0 = m0.body + (size_t)row0 * 16;
                    pa1 = m1.body + (size_t)row0 * 16;
                    pd0 = ok && m0.type != CLB_IQ1_M ? m0.d + row0 : nullptr;
                    pd1 = ok && m1.type != CLB_IQ1_M ? m1.d + row0 : nullptr;
                    ps0 = ok && m0.type != CLB_IQ2_XXS ? m0.sc + (size_t)row0 * 8 : nullptr;
                    ps1 = ok && m1.type != CLB_IQ2_XXS ? m1.sc + (size_t)row0 * 8 : nullptr;
                    // weight ring: pieces, then sc bytes (decoders); scale ring: d, or for IQ1_M the
                    // sc bytes that carry its scale (epilogue)
                    raw_tx = 16u * rb * (uint32_t)np0 + (ps0 ? 8u * rb : 0u);
                    dw_tx = pd0 ? 2u * rb : 8u * rb;
                    if (split) {
                        raw_tx += 16u * rb * (uint32_t)np1 + (ps1 ? 8u * rb : 0u);
                        dw_tx += pd1 ? 2u * rb : 8u * rb;
                    }
                }
                if (rr.round > 0 && !pf_wait(bar(kRawEmpty + rr.slot), rr.phase ^ 1u, abort_flag, G.err)) break;
                const uint32_t full = bar(kRawFull + rr.slot), dst = sraw + (uint32_t)rr.slot * kPfRawBlock;
                // headers are plain shared stores that the arrive below releases to the waiting roles
                *reinterpret_cast<int*>(sm + PfSmem::raw + rr.slot * kPfRawBlock + kPfRawHdr) = hdr.w;
                if (!ok) {
                    mbar_arrive(full);
                } else {
                    // piece p of the block -> piece slot p; gate rows then up rows within a slot
                    mbar_expect_tx(full, raw_tx);
                    // piece by piece, gate and up rows of a piece together
                    const uint8_t* s0 = pa0 + (size_t)b * (size_t)np0 * plane;
                    const uint8_t* s1 = pa1 + (size_t)b * (size_t)np1 * plane;
                    for (int p = 0; p < 4; ++p) {
                        if (p < np0) bulk_g2s(dst + p * kPfRawStage, s0 + p * plane, 16u * rb, full);
                        if (split && p < np1) bulk_g2s(dst + p * kPfRawStage + 16u * rb, s1 + p * plane, 16u * rb, full);
                    }
                    if (ps0) bulk_g2s(dst + kPfRawSc, ps0 + (size_t)b * n * 8, 8u * rb, full);
                    if (split && ps1) bulk_g2s(dst + kPfRawSc + 8u * rb, ps1 + (size_t)b * n * 8, 8u * rb, full);
                }
                rr.next();
                if (dr.round > 0 && !pf_wait(bar(kDwEmpty + dr.slot), dr.phase ^ 1u, abort_flag, G.err)) break;
                const uint32_t dfull = bar(kDwFull + dr.slot), ddst = sdw + (uint32_t)dr.slot * kPfDwSlot;
                *reinterpret_cast<int4*>(sm + PfSmem::dw + dr.slot * kPfDwSlot + kPfDwHdr) = hdr;
                if (!ok) {
                    mbar_arrive(dfull);
                } else {
                    // fp16 d of the rows at [0, 256), IQ1_M rows' 8 scale bytes at [256, 1280)
                    mbar_expect_tx(dfull, dw_tx);
                    if (pd0)
                        bulk_g2s(ddst, pd0 + (size_t)b * n, 2u * rb, dfull);
                    else
                        bulk_g2s(ddst + 256, ps0 + (size_t)b * n * 8, 8u * rb, dfull);
                    if (split) {
                        if (pd1)
                            bulk_g2s(ddst + 2u * rb, pd1 + (size_t)b * n, 2u * rb, dfull);
                        else
                            bulk_g2s(ddst + 256 + 8u * rb, ps1 + (size_t)b * n * 8, 8u * rb, dfull);
                    }
                }
                dr.next();
                if (++b == nb) {
                    b = 0;
                    ++tile;
                }
            }
        }
    } else if (warp == kPfBWarp) {
        // ---------------- B operand (TMA, 4 stages per block) and the tiles' activation scales ----------------
        if (lane == 0 && total > 0) {
            Ring<2> br;
            int tile = 0, b = 0, first = 0, n = 16, x = 0;
            for (int blk = 0; blk < nblk; ++blk) {
                if (b == 0) {
                    const PfTile t = pf_tile(G, tile);
                    first = t.first;
                    n = (t.ntok + 15) & ~15;
                    x = 0;
                    const int xs = tile & 1;
                    if (tile >= 2 && !pf_wait(bar(kDxsEmpty + xs), ((tile >> 1) & 1) ^ 1u, abort_flag, G.err)) break;
                    const uint32_t dfull = bar(kDxsFull + xs);
                    mbar_expect_tx(dfull, (uint32_t)(nb * n * 4));
                    for (int bb = 0; bb < nb; ++bb)
                        bulk_g2s(sdxs + (uint32_t)(xs * kPfMaxNb + bb) * (kPfDxsStride * 4), G.actd + (size_t)bb * G.P + first,
                                 (uint32_t)n * 4, dfull);
                }
                if (br.round > 0 && !pf_wait(bar(kBlockDone + br.slot), br.phase ^ 1u, abort_flag, G.err)) break;
                const uint32_t full = bar(kBFull + br.slot);
                reinterpret_cast<int*>(sm + PfSmem::bhdr)[br.slot] = n;
                mbar_expect_tx(full, (uint32_t)n * 128 * 4);
                const CUtensorMap* map = &G.bmaps[(n >> 4) - 1];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    tma_2d(sb0 + (uint32_t)(br.slot * 4 + q) * kPfBStage, map, x + q * kPfStageK, first, full);
                x += 4 * kPfStageK;
                br.next();
                if (++b == nb) {
                    b = 0;
                    ++tile;
                }
            }
        }
    } else if (warp == kPfMmaWarp) {
        // ---------------- MMAs: 16 per block (4 stages x 4) into one of kPfAcc accumulators ----------------
        if (lane == 0 && total > 0) {
            // B descriptors: K-major, 128-byte swizzle, 8-row groups 1024 B apart
            const uint64_t bdesc0 = ((uint64_t)1 << 16) | ((uint64_t)64 << 32) | ((uint64_t)1 << 46) |
                                    ((uint64_t)2 << 61) | (uint64_t)((sb0 >> 4) & 0x3FFFu);
            Ring<2> ab;
            Ring<kPfAcc> acc;
            const volatile int* bhdr = reinterpret_cast<const volatile int*>(sm + PfSmem::bhdr);
            for (int blk = 0; blk < nblk; ++blk) {
                // B first (it runs ahead): its header read overlaps the wait for A
                if (!pf_wait(bar(kBFull + ab.slot), ab.phase, abort_flag, G.err)) break;
                const uint32_t idesc = (1u << 4) | ((uint32_t)(bhdr[ab.slot] >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
                if (!pf_wait(bar(kAFull + ab.slot), ab.phase, abort_flag, G.err)) break;
                if (acc.round > 0 && !pf_wait(bar(kAccEmpty + acc.slot), acc.phase ^ 1u, abort_flag, G.err)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint64_t bdesc = bdesc0 + (uint64_t)(ab.slot * 4 * (kPfBStage >> 4));
                const uint32_t dd = tmem + (uint32_t)acc.slot * kPfAccCols;
                const uint32_t da = tmem + kPfACol + (uint32_t)ab.slot * 128;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
#pragma unroll
                    for (int j = 0; j < kPfStageK / 16; ++j) {
                        const uint64_t db = bdesc + (uint64_t)(q * (kPfBStage >> 4) + 2 * j);
                        if (q == 0 && j == 0)
                            umma_ts<false>(dd, da, db, idesc);
                        else
                            umma_ts<true>(dd, da + (uint32_t)(j * 32 + 8 * q), db, idesc);
                    }
                }
                umma_commit(bar(kBlockDone + ab.slot));
                umma_commit(bar(kAccFull + acc.slot));
                ab.next();
                acc.next();
            }
        }
    } else if (warp >= kPfEpiWarp0) {
        // ---------------- epilogue (8 warps: lane quarter, 32-column half) ----------------
        // Block sums D are scaled and added into running tile sums R kept in tensor memory;
        // the last block of a tile writes 0.125 * R out instead.
        const int ew = warp - kPfEpiWarp0, quarter = ew & 3, c0 = 32 * (ew >> 2), row = 32 * quarter + lane;
        const uint32_t tlane = (uint32_t)(32 * quarter) << 16;
        auto uwait = [&](int b, uint32_t parity) {
            return __all_sync(0xffffffffu, pf_wait(bar(b), parity, abort_flag, G.err));
        };
        Ring<kPfDwRing> dr;
        Ring<kPfAcc> acc;
        int tile = 0, b = 0;
        for (int e = 0; e < nblk; ++e) {
            if (!uwait(kDwFull + dr.slot, dr.phase)) break;
            const uint8_t* slot = sm + PfSmem::dw + dr.slot * kPfDwSlot;
            const int4 hdr = *reinterpret_cast<const int4*>(slot + kPfDwHdr);  // {first, entries, mt, types}
            const int first = hdr.x, ntok = hdr.y, mt = hdr.z, type = pf_row_type(hdr.w, G.role, quarter);
            if (b == 0 && !uwait(kDxsFull + (tile & 1), (tile >> 1) & 1)) break;
            if (!uwait(kAccFull + acc.slot, acc.phase)) break;
            const bool last = b == nb - 1;
            if (c0 < ntok) {
                const bool iq1 = TYPES == kTypeBitIQ1M || (TYPES != kTypeBitXXS && TYPES != kTypeBitXS && type == CLB_IQ1_M);
                const float dw = iq1 ? iq1m_scale(*reinterpret_cast<const uint2*>(slot + 256 + row * 8))
                                     : __half2float(reinterpret_cast<const __half*>(slot)[row]);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");  // the previous block's R stores
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const float* dxs = reinterpret_cast<const float*>(sm + PfSmem::dxs) +
                                   ((tile & 1) * kPfMaxNb + b) * kPfDxsStride + c0;
                uint32_t d[32], r[32];
                tmem_ld32(tmem + tlane + (uint32_t)(acc.slot * kPfAccCols + c0), d);
                if (b > 0) tmem_ld32(tmem + tlane + kPfRCol + (uint32_t)c0, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 d4 = reinterpret_cast<const float4*>(dxs)[j4];
                    const float sc[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int j = 4 * j4 + u;
                        const float prev = b > 0 ? __uint_as_float(r[j]) : 0.0f;
                        r[j] = __float_as_uint(__fmaf_rn(__fmul_rn(dw, sc[u]), __uint_as_float(d[j]), prev));
                    }
                }
                if (!last) {
                    tmem_st32(tmem + tlane + kPfRCol + (uint32_t)c0, r);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = c0 + j;
                        if (n < ntok) {
                            const float v = __fmul_rn(0.125f, __uint_as_float(r[j]));
                            if (G.role == 0)
                                G.out[((size_t)(first + n) * 2 + (row >> 6)) * G.nrows + mt * 64 + (row & 63)] = v;
                            else
                                G.out[(size_t)G.list[first + n] * G.nrows + mt * 128 + row] = v;
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(kAccEmpty + acc.slot));
                mbar_arrive(bar(kDwEmpty + dr.slot));
                if (last) mbar_arrive(bar(kDxsEmpty + (tile & 1)));
            }
            dr.next();
            acc.next();
            if (++b == nb) {
                b = 0;
                ++tile;
            }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    } else {
        // ---------------- decoders (warps 0-7): one 32-value chunk of one row per stage ----------------
        // Per block: the raw words of the thread's chunk c = 2q + dc of the 4 stages and its
        // sub-scales, then two 32-column tensor-memory stores (pf_decode_block).
        const uint32_t lb = (uint32_t)lane * 4u;
        const int quarter = warp & 3, dr = 32 * quarter + lane, dc = warp >> 2;  // row, chunk of a stage
        const uint32_t tlane = (uint32_t)(32 * quarter) << 16;
        const __half2 off2 = __float2half2_rn(-1152.0f);
        auto uwait = [&](int b, uint32_t parity) {
            return __all_sync(0xffffffffu, pf_wait(bar(b), parity, abort_flag, G.err));
        };
        Ring<2> rr;
        // One block of type T, after its weight pieces landed; false when a wait gave up.
        // Specialised per type so that each path is straight-line code.
        auto block = [&](auto tt) -> bool {
            constexpr int T = decltype(tt)::value;
            const uint8_t* slotp = sm + PfSmem::raw + rr.slot * kPfRawBlock;
            const uint8_t* raw = slotp + dr * 16;
            uint32_t cw[8];
            uint2 scw = make_uint2(0u, 0u);
            if (T != CLB_IQ2_XXS) scw = *reinterpret_cast<const uint2*>(slotp + kPfRawSc + dr * 8);
            if (T == CLB_IQ1_M) {
                const uint4 p0 = *reinterpret_cast<const uint4*>(raw);
                const uint4 p1 = *reinterpret_cast<const uint4*>(raw + kPfRawStage);
                const uint4 p2 = *reinterpret_cast<const uint4*>(raw + 2 * kPfRawStage);
                cw[0] = dc ? p0.y : p0.x;  // qs word of chunk c (piece c / 4, word c % 4)
                cw[1] = dc ? p0.w : p0.z;
                cw[2] = dc ? p1.y : p1.x;
                cw[3] = dc ? p1.w : p1.z;
                const uint32_t hs = 16u * (uint32_t)dc;  // qh half-word c of piece 2
                cw[4] = (p2.x >> hs) & 0xffffu;
                cw[5] = (p2.y >> hs) & 0xffffu;
                cw[6] = (p2.z >> hs) & 0xffffu;
                cw[7] = (p2.w >> hs) & 0xffffu;
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint2 v = *reinterpret_cast<const uint2*>(raw + q * kPfRawStage + dc * 8);
                    cw[2 * q] = v.x;
                    cw[2 * q + 1] = v.y;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kRawEmpty + rr.slot));
            __half2 s2[4], nf[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t c = 2u * q + (uint32_t)dc;
                if (T == CLB_IQ2_XXS) {  // bits 28-31 of the aux word: s
                    const uint32_t sc = (((cw[2 * q + 1] & 0x80808080u) | 0x08000000u) * 0x00204081u) >> 27;  // 2s + 1
                    s2[q] = __float2half2_rn((float)sc);
                } else if (T == CLB_IQ2_XS) {  // scale byte c: low nibble values 0-15, high 16-31
                    const uint32_t scb = ((q < 2 ? scw.x : scw.y) >> (8u * (c & 3u))) & 0xffu;
                    s2[q] = __floats2half2_rn((float)(((scb & 15u) << 1) | 1u), (float)(((scb >> 4) << 1) | 1u));
                } else {  // scale word c / 2: 3-bit scales at bit 6 (c & 1) and 6 (c & 1) + 3
                    const uint32_t w = ((q < 2 ? scw.x : scw.y) >> (16u * (q & 1u))) >> (6u * (c & 1u));
                    s2[q] = __floats2half2_rn((float)(((w & 7u) << 1) | 1u), (float)((((w >> 3) & 7u) << 1) | 1u));
                }
                nf[q] = __hmul2(off2, s2[q]);
            }
            // this block's A buffers were last read by the MMAs of block blk - 2
            if (rr.round > 0 && !uwait(kBlockDone + rr.slot, rr.phase ^ 1u)) return false;
            pf_decode_block<T>(cw, s2, nf, lb,
                               tmem + tlane + kPfACol + (uint32_t)rr.slot * 128 + (uint32_t)(2 * dc) * 32);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kAFull + rr.slot));
            return true;
        };
        for (int blk = 0; blk < nblk; ++blk) {
            if (!uwait(kRawFull + rr.slot, rr.phase)) break;
            const int type =
                pf_row_type(*reinterpret_cast<const int*>(sm + PfSmem::raw + rr.slot * kPfRawBlock + kPfRawHdr),
                            G.role, quarter);
            bool ok;
            if (TYPES == kTypeBitXXS)
                ok = block(std::integral_constant<int, CLB_IQ2_XXS>());
            else if (TYPES == kTypeBitXS)
                ok = block(std::integral_constant<int, CLB_IQ2_XS>());
            else if (TYPES == kTypeBitIQ1M)
                ok = block(std::integral_constant<int, CLB_IQ1_M>());
            else
                ok = type == CLB_IQ2_XXS ? block(std::integral_constant<int, CLB_IQ2_XXS>())
                     : type == CLB_IQ2_XS ? block(std::integral_constant<int, CLB_IQ2_XS>())
                                          : block(std::integral_constant<int, CLB_IQ1_M>());
            if (!ok) break;
            rr.next();
        }
    }

    __syncthreads();
    if (*abort_flag) {  // let copies already in flight land before the shared memory is released
        uint64_t t0, t1;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        do {
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
        } while (t1 - t0 < 200000u);
    }
    // drain: every MMA this CTA issued has completed before the tensor memory is freed
    if (warp == kPfMmaWarp && lane == 0 && total > 0) {
        umma_commit(bar(kDrain));
        bool done = false;
        for (uint32_t it = 0; it < kPfSpin && !done; ++it) done = mbar_try(bar(kDrain), 0);
        if (!done) atomicExch(G.err, kErrPrefillWait);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
}

// ---------------------------------------------------------------------------------------
// Grouping of the T x k picks by expert (one CTA of 1024 threads). Experts with more than
// `cold_max` picks go to the GEMMs: list[] holds their slots t*k+p expert after expert, in
// slot order within an expert, each expert's run padded with -1 to a multiple of 16 entries;
// tiles[] one entry per chunk of at most kPfMaxN entries. The slots of the other experts go
// to pairs[] (*npairs of them, in no particular order) for the row-dot path, which decodes a
// weight for one token at a third of the GEMM decoder's cost per weight.
__global__ void __launch_bounds__(1024) k_prefill_group(const int* __restrict__ ids, int T, int k, int E, int P,
                                                        int e_begin, int e_end, int cold_max, int* __restrict__ list,
                                                        int4* __restrict__ tiles, int* __restrict__ ntiles,
                                                        int* __restrict__ pairs, int* __restrict__ npairs,
                                                        int* __restrict__ err) {
    __shared__ int cnt[kMaxExperts], off[kMaxExperts], toff[kMaxExperts];
    __shared__ int np_s;
    const int n = T * k;
    for (int p = threadIdx.x; p < P; p += blockDim.x) list[p] = -1;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    if (threadIdx.x == 0) np_s = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = ids[i];
        if (e < 0 || e >= E) atomicExch(err, 1);
        else if (e >= e_begin && e < e_end) atomicAdd(&cnt[e], 1);  // picks of other GPUs' experts are skipped
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0, to = 0;
        for (int e = 0; e < E; ++e) {
            off[e] = o, toff[e] = to;
            if (cnt[e] > cold_max) {
                o += (cnt[e] + 15) & ~15;
                to += (cnt[e] + kPfMaxN - 1) / kPfMaxN;
            }
        }
        *ntiles = to;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = ids[i];
        if (e >= e_begin && e < e_end && cnt[e] <= cold_max) pairs[atomicAdd(&np_s, 1)] = i;
    }
    // stable placement by one warp, 32 slots at a time: slot i goes after every smaller slot
    // of the same expert (rank among equal lanes from __match_any_sync)
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            const int e = i < n ? ids[i] : -1;
            const bool valid = e >= e_begin && e < e_end && cnt[e] > cold_max;
            const unsigned m = __match_any_sync(0xffffffffu, valid ? e : -1);
            const int rank = __popc(m & ((1u << lane) - 1u));
            const int base = valid ? off[e] : 0;
            __syncwarp();
            if (valid) {
                list[base + rank] = i;
                if (rank == 0) off[e] = base + __popc(m);
            }
            __syncwarp();
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *npairs = np_s;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        if (e < e_begin || e >= e_end || cnt[e] <= cold_max) continue;
        const int start = off[e] - cnt[e];
        for (int j = 0; j * kPfMaxN < cnt[e]; ++j)
            tiles[toff[e] + j] = make_int4(e, start + j * kPfMaxN, min(kPfMaxN, cnt[e] - j * kPfMaxN), 0);
    }
}

// ---------------------------------------------------------------------------------------
// Row-dot path of the sparsely picked experts (pairs[]: one slot = one token of one expert):
// the decode kernels' one-row-per-lane fast order (lane_row_partial) over whole rows, the
// token's Q8_K activation read from global memory (L1 broadcast), one warp per 32 rows.
// Persistent: one CTA of kPcThreads per SM, decode tables in shared memory.
constexpr int kPcThreads = 512;
constexpr size_t kPcSmem = kRowTableBytes + 2944 * 4;  // tables + their staging area

__global__ void __launch_bounds__(kPcThreads, 1)
    k_pairs_gateup(const ExpertDesc* __restrict__ desc, const int* __restrict__ ids, const int* __restrict__ pairs,
                   const int* __restrict__ npairs, int k, const int8_t* __restrict__ qx, const float* __restrict__ dx,
                   int dim, int ff, const uint32_t* __restrict__ tables, float* __restrict__ gu, int* __restrict__ err) {
    const int np = *npairs;
    if (np == 0) return;
    fill_row_tables(tables, reinterpret_cast<uint32_t*>(clb_dyn_smem + kRowTableBytes));
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int groups = ff >> 5, nb = dim >> 8;
    const int items = np * 2 * groups;
    for (int it = blockIdx.x * nw + warp; it < items; it += gridDim.x * nw) {
        const int pr = it / (2 * groups), rem = it - pr * 2 * groups;
        const int mat = rem & 1, row = (rem >> 1) * 32 + lane;  // gate and up of the same rows adjacent
        const int sl = pairs[pr], t = sl / k;
        const ExpertDesc& ex = desc[ids[sl]];
        const PackedMat& m = mat ? ex.up : ex.gate;
        float y = 0.0f;
        if (m.body != nullptr && m.k == dim && m.n == ff)
            y = lane_row_partial_any<256>(m, row, 0, nb, qx + (size_t)t * dim, dx + (size_t)t * nb);
        else if (lane == 0)
            atomicExch(err, 1);
        gu[((size_t)pr * 2 + mat) * ff + row] = y;
    }
}

// SwiGLU of a pair's gate/up rows and Q8_K(h) (unpadded rows); one warp per 256 values.
__global__ void __launch_bounds__(256) k_pairs_act(const int* __restrict__ npairs, int ff, float limit,
                                                   const float* __restrict__ gu, int8_t* __restrict__ qh,
                                                   float* __restrict__ dh) {
    const int nbr = ff >> 8;
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk >= *npairs * nbr) return;
    const int p = blk / nbr, b = blk % nbr;
    const float* g = gu + (size_t)p * 2 * ff + b * 256 + lane * 8;
    const float* u = g + ff;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = swiglu(g[i], u[i], limit);
    warp_quant_regs(v, qh + (size_t)p * ff + b * 256, dh + (size_t)p * nbr + b);
}

// Down rows of every pair into the slot-ordered expert rows y[slot][dim] that the combine reads.
__global__ void __launch_bounds__(kPcThreads, 1)
    k_pairs_down(const ExpertDesc* __restrict__ desc, const int* __restrict__ ids, const int* __restrict__ pairs,
                 const int* __restrict__ npairs, const int8_t* __restrict__ qh, const float* __restrict__ dh, int dim,
                 int ff, const uint32_t* __restrict__ tables, float* __restrict__ y, int* __restrict__ err) {
    const int np = *npairs;
    if (np == 0) return;
    fill_row_tables(tables, reinterpret_cast<uint32_t*>(clb_dyn_smem + kRowTableBytes));
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int groups = dim >> 5, nbh = ff >> 8;
    const int items = np * groups;
    for (int it = blockIdx.x * nw + warp; it < items; it += gridDim.x * nw) {
        const int pr = it / groups, row = (it - pr * groups) * 32 + lane;
        const int sl = pairs[pr];
        const PackedMat& m = desc[ids[sl]].down;
        float v = 0.0f;
        if (m.body != nullptr && m.k == ff && m.n == dim)
            v = lane_row_partial_any<256>(m, row, 0, nbh, qh + (size_t)pr * ff, dh + (size_t)pr * nbh);
        else if (lane == 0)
            atomicExch(err, 1);
        y[(size_t)sl * dim + row] = v;
    }
}

// Q8_K of 256 values held 8 per lane into int8 (qs), the scale (*d) and fp16 copies (q16).
__device__ __forceinline__ void quant_block_fp16(float v[8], int8_t* qs, float* d, __half* q16) {
    const int lane = threadIdx.x & 31;
    warp_quant_regs(v, qs, d);
    const uint2 w = *reinterpret_cast<const uint2*>(qs + lane * 8);
    const uint32_t ws[2] = {w.x, w.y};
    __align__(16) __half h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __int2half_rn((int)(int8_t)(ws[i >> 2] >> (8 * (i & 3))));
    *reinterpret_cast<uint4*>(q16 + lane * 8) = *reinterpret_cast<const uint4*>(h);
}

// Q8_K of the token rows (one warp per 256-value block).
__global__ void __launch_bounds__(256) k_prefill_quant(const float* __restrict__ x, int nrows, int cols,
                                                       int8_t* __restrict__ qs, float* __restrict__ d,
                                                       __half* __restrict__ q16) {
    const int nbr = cols >> 8;
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk >= nrows * nbr) return;
    const int row = blk / nbr, b = blk % nbr;
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)row * cols + b * 256 + lane * 8);
    const float4 lo = src[0], hi = src[1];
    float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    const size_t o = (size_t)row * cols + b * 256;
    quant_block_fp16(v, qs + o, d + blk, q16 + o);
}

// x = RMSNorm(h) fused with Q8_K of the token rows, for the batched stack: one CTA of 1024
// threads per token. The fp64 sum of squares has k_norm_quant's fixed order (lane t sums
// (double)h[t + 1024 j]^2 over j, then a binary tree over the lanes), so every token gets the
// single-token stack's scale bit for bit; x = h * (float)(1 / sqrt(mean + 1e-6)).
__global__ void __launch_bounds__(1024) k_prefill_norm_quant(const float* __restrict__ h, int cols,
                                                             int8_t* __restrict__ qs, float* __restrict__ d,
                                                             __half* __restrict__ q16) {
    __shared__ double part[1024];
    __shared__ float scale_s;
    const int t = threadIdx.x, row = blockIdx.x;
    const float* hr = h + (size_t)row * cols;
    double s = 0.0;
    for (int i = t; i < cols; i += 1024) {
        const double v = (double)hr[i];
        s = __dadd_rn(s, __dmul_rn(v, v));
    }
    part[t] = s;
    __syncthreads();
    for (int stride = 512; stride > 0; stride >>= 1) {
        if (t < stride) part[t] = __dadd_rn(part[t], part[t + stride]);
        __syncthreads();
    }
    if (t == 0) {
        const double mean = __ddiv_rn(part[0], (double)cols);
        scale_s = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(mean, 1e-6)));
    }
    __syncthreads();
    const float sc = scale_s;
    const int nbr = cols >> 8, warp = t >> 5, lane = t & 31;
    for (int b = warp; b < nbr; b += 32) {
        const float4* src = reinterpret_cast<const float4*>(hr + b * 256 + lane * 8);
        const float4 lo = src[0], hi = src[1];
        float v[8] = {__fmul_rn(lo.x, sc), __fmul_rn(lo.y, sc), __fmul_rn(lo.z, sc), __fmul_rn(lo.w, sc),
                      __fmul_rn(hi.x, sc), __fmul_rn(hi.y, sc), __fmul_rn(hi.z, sc), __fmul_rn(hi.w, sc)};
        const size_t o = (size_t)row * cols + b * 256;
        quant_block_fp16(v, qs + o, d + (size_t)row * nbr + b, q16 + o);
    }
}

// Token rows of Q8_K(x) into list order: xg16[p] = q16[token of list[p]], dxg[b][p] its scales.
// One warp per (entry, 256-value block).
__global__ void __launch_bounds__(256) k_prefill_gather(const int* __restrict__ list, int P, int k, int cols,
                                                        const __half* __restrict__ q16, const float* __restrict__ d,
                                                        __half* __restrict__ xg16, float* __restrict__ dxg) {
    const int nbr = cols >> 8;
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk >= P * nbr) return;
    const int p = blk / nbr, b = blk % nbr, sl = list[p];
    if (sl < 0) return;  // padding: the GEMM reads these rows into columns it never stores
    const int t = sl / k;
    *reinterpret_cast<uint4*>(xg16 + (size_t)p * cols + b * 256 + lane * 8) =
        *reinterpret_cast<const uint4*>(q16 + (size_t)t * cols + b * 256 + lane * 8);
    if (lane == 0) dxg[(size_t)b * P + p] = d[(size_t)t * nbr + b];
}

// SwiGLU of the gate/up rows (list order) and Q8_K of h: qh16[p] fp16 values, dhg[b][p]
// scales. One warp per (entry, 256-value block).
__global__ void __launch_bounds__(256) k_prefill_act(const int* __restrict__ list, int P, int ff, float limit,
                                                     const float* __restrict__ gu, int8_t* __restrict__ qh,
                                                     __half* __restrict__ qh16, float* __restrict__ dhg) {
    const int nbr = ff >> 8;
    const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (blk >= P * nbr) return;
    const int p = blk / nbr, b = blk % nbr;
    const size_t o = (size_t)p * ff + b * 256;
    if (list[p] < 0) return;  // padding (see k_prefill_gather)
    const float* g = gu + (size_t)p * 2 * ff + b * 256 + lane * 8;
    const float* u = g + ff;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = swiglu(g[i], u[i], limit);
    quant_block_fp16(v, qh + o, dhg + (size_t)b * P + p, qh16 + o);
}

// out[t] = fma over the token's picks in ascending expert id of (w, expert row), then
// + resid when given (runtime.cpp:184-187). One CTA per token, four columns per thread.
__global__ void __launch_bounds__(256) k_prefill_combine(const float* __restrict__ y, const int* __restrict__ ids,
                                                         const float* __restrict__ w, int k, int dim,
                                                         const float* __restrict__ resid, float* __restrict__ out) {
    __shared__ int order[kMaxPicks];
    __shared__ float wo[kMaxPicks];
    __shared__ int npk;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        const int* id = ids + (size_t)t * k;
        int prev = -1, n = 0;
        for (int o = 0; o < k; ++o) {
            int best = -1;
            for (int p = 0; p < k; ++p)
                if (id[p] > prev && (best < 0 || id[p] < id[best])) best = p;
            if (best < 0) break;
            prev = id[best];
            order[n] = best;
            wo[n++] = w[(size_t)t * k + best];
        }
        npk = n;
    }
    __syncthreads();
    const int n = npk, d4 = dim >> 2;
    const float4* y4 = reinterpret_cast<const float4*>(y) + (size_t)t * k * d4;
    for (int c = threadIdx.x; c < d4; c += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int o = 0; o < n; ++o) {
            const float4 v = y4[(size_t)order[o] * d4 + c];
            const float wt = wo[o];
            acc.x = __fmaf_rn(wt, v.x, acc.x);
            acc.y = __fmaf_rn(wt, v.y, acc.y);
            acc.z = __fmaf_rn(wt, v.z, acc.z);
            acc.w = __fmaf_rn(wt, v.w, acc.w);
        }
        if (resid) {
            const float4 r = reinterpret_cast<const float4*>(resid)[(size_t)t * d4 + c];
            acc.x = __fadd_rn(r.x, acc.x);
            acc.y = __fadd_rn(r.y, acc.y);
            acc.z = __fadd_rn(r.z, acc.z);
            acc.w = __fadd_rn(r.w, acc.w);
        }
        reinterpret_cast<float4*>(out)[(size_t)t * d4 + c] = acc;
    }
}

namespace {
struct PrefillWs {
    int P;
    int* list;
    int* pairs;
    int* npairs;
    float* pgu;
    int8_t* pqh;
    float* pdh;
    int4* tiles;
    int* ntiles;
    int8_t* qx;
    float* dx;
    __half* qx16;
    __half* xg16;
    float* dxg;
    float* gu;
    int8_t* qh;
    __half* qh16;
    float* dhg;
    float* y;
};

size_t carve(void* base, int T, int k, int dim, int ff, int E, PrefillWs* ws) {
    const size_t slots = (size_t)T * k;
    const size_t P = (slots + 15 * std::min<size_t>((size_t)E, slots) + 15) & ~(size_t)15;
    const size_t nbx = dim / 256, nbh = ff / 256;
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t r = off;
        off += (n + 255) & ~(size_t)255;
        return r;
    };
    const size_t o_list = take(P * 4), o_tiles = take(((size_t)E + slots / kPfMaxN + 1) * 16), o_nt = take(16);
    const size_t maxp = std::min<size_t>(slots, (size_t)E * kPfColdMax);  // row-dot pairs
    const size_t o_pairs = take(slots * 4), o_np = take(16), o_pgu = take(maxp * 2 * ff * 4), o_pqh = take(maxp * ff),
                 o_pdh = take(maxp * nbh * 4);
    const size_t o_qx = take((size_t)T * dim), o_dx = take((size_t)T * nbx * 4), o_qx16 = take((size_t)T * dim * 2);
    const size_t o_xg16 = take(P * dim * 2), o_dxg = take(nbx * P * 4), o_gu = take(P * 2 * ff * 4);
    const size_t o_qh = take(P * ff), o_qh16 = take(P * ff * 2), o_dhg = take(nbh * P * 4), o_y = take(slots * dim * 4);
    if (ws && base) {
        uint8_t* p = static_cast<uint8_t*>(base);
        ws->P = (int)P;
        ws->list = reinterpret_cast<int*>(p + o_list);
        ws->pairs = reinterpret_cast<int*>(p + o_pairs);
        ws->npairs = reinterpret_cast<int*>(p + o_np);
        ws->pgu = reinterpret_cast<float*>(p + o_pgu);
        ws->pqh = reinterpret_cast<int8_t*>(p + o_pqh);
        ws->pdh = reinterpret_cast<float*>(p + o_pdh);
        ws->tiles = reinterpret_cast<int4*>(p + o_tiles);
        ws->ntiles = reinterpret_cast<int*>(p + o_nt);
        ws->qx = reinterpret_cast<int8_t*>(p + o_qx);
        ws->dx = reinterpret_cast<float*>(p + o_dx);
        ws->qx16 = reinterpret_cast<__half*>(p + o_qx16);
        ws->xg16 = reinterpret_cast<__half*>(p + o_xg16);
        ws->dxg = reinterpret_cast<float*>(p + o_dxg);
        ws->gu = reinterpret_cast<float*>(p + o_gu);
        ws->qh = reinterpret_cast<int8_t*>(p + o_qh);
        ws->qh16 = reinterpret_cast<__half*>(p + o_qh16);
        ws->dhg = reinterpret_cast<float*>(p + o_dhg);
        ws->y = reinterpret_cast<float*>(p + o_y);
    }
    return off;
}
}  // namespace

size_t prefill_workspace_bytes(int T, int k, int dim, int ff, int E) { return carve(nullptr, T, k, dim, ff, E, nullptr); }

bool prefill_shape_supported(int dim, int ff) {
    return dim % 256 == 0 && ff % 256 == 0 && dim >= 512 && ff >= 512 && dim / 256 <= kPfMaxNb &&
           ff / 256 <= kPfMaxNb;
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor maps over B rows [P][K] fp16 (list order): box 64 values x 16 (i + 1) rows, 128-byte swizzle.
cudaError_t encode_bmaps(CUtensorMap* maps, const __half* base, int P, int K) {
    static EncodeTiledFn encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (!fn || q != cudaDriverEntryPointSuccess) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)P};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t es[2] = {1, 1};
    for (int i = 0; i < kPfMaxN / 16; ++i) {
        const cuuint32_t box[2] = {(cuuint32_t)kPfStageK, (cuuint32_t)(16 * (i + 1))};
        if (encode(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}
}  // namespace

cudaError_t launch_prefill(const ExpertDesc* desc, int E, const float* x, const int* ids, const float* w, int T, int k,
                           int dim, int ff, float limit, const float* resid, float* out, void* wsp, int* err,
                           int phase_mask, cudaStream_t s, bool norm_x, int e_begin, int e_end, float* rows,
                           int type_mask) {
    PrefillWs ws{};
    carve(wsp, T, k, dim, ff, E, &ws);
    if (e_end < 0) e_end = E;
    if (rows) ws.y = rows;
    const int P = ws.P;
    const uint32_t* tables = nullptr;
    cudaError_t e = tables_device_ptr(&tables);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    void (*gemm)(PrefillGemm) = type_mask == kTypeBitXXS    ? k_prefill_gemm<kTypeBitXXS>
                                : type_mask == kTypeBitXS  ? k_prefill_gemm<kTypeBitXS>
                                : type_mask == kTypeBitIQ1M ? k_prefill_gemm<kTypeBitIQ1M>
                                                            : k_prefill_gemm<kTypeBitAll>;
    if ((e = cudaFuncSetAttribute(gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PfSmem::total)) !=
        cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(k_pairs_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPcSmem)) !=
        cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(k_pairs_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPcSmem)) !=
        cudaSuccess)
        return e;
    const int nbx = dim / 256, nbh = ff / 256;
    if (phase_mask & 1) {
        k_prefill_group<<<1, 1024, 0, s>>>(ids, T, k, E, P, e_begin, e_end, kPfColdMax, ws.list, ws.tiles,
                                           ws.ntiles, ws.pairs, ws.npairs, err);
        // rows of other GPUs' picks stay zero, so a sum over the GPUs' row buffers is exact
        if ((e_begin > 0 || e_end < E) && (e = cudaMemsetAsync(ws.y, 0, (size_t)T * k * dim * 4, s)) != cudaSuccess)
            return e;
        if (norm_x)
            k_prefill_norm_quant<<<T, 1024, 0, s>>>(x, dim, ws.qx, ws.dx, ws.qx16);
        else
            k_prefill_quant<<<(T * nbx + 7) / 8, 256, 0, s>>>(x, T, dim, ws.qx, ws.dx, ws.qx16);
        k_prefill_gather<<<(P * nbx + 7) / 8, 256, 0, s>>>(ws.list, P, k, dim, ws.qx16, ws.dx, ws.xg16, ws.dxg);
    }
    PrefillGemm g{};
    g.desc = desc;
    g.tiles = ws.tiles;
    g.ntiles = ws.ntiles;
    g.list = ws.list;
    g.P = P;
    g.err = err;
    g.tables = tables;
    if (phase_mask & 2) {
        if ((e = encode_bmaps(g.bmaps, ws.xg16, P, dim)) != cudaSuccess) return e;
        g.role = 0;
        g.actd = ws.dxg;
        g.K = dim;
        g.nrows = ff;
        g.mtiles = ff / 64;
        g.out = ws.gu;
        gemm<<<sms, kPfThreads, PfSmem::total, s>>>(g);
        k_pairs_gateup<<<sms, kPcThreads, kPcSmem, s>>>(desc, ids, ws.pairs, ws.npairs, k, ws.qx, ws.dx, dim, ff,
                                                         tables, ws.pgu, err);
    }
    if (phase_mask & 4) {
        k_prefill_act<<<(P * nbh + 7) / 8, 256, 0, s>>>(ws.list, P, ff, limit, ws.gu, ws.qh, ws.qh16, ws.dhg);
        const int maxp = std::min(T * k, E * kPfColdMax);
        k_pairs_act<<<(maxp * nbh + 7) / 8, 256, 0, s>>>(ws.npairs, ff, limit, ws.pgu, ws.pqh, ws.pdh);
    }
    if (phase_mask & 8) {
        if ((e = encode_bmaps(g.bmaps, ws.qh16, P, ff)) != cudaSuccess) return e;
        g.role = 1;
        g.actd = ws.dhg;
        g.K = ff;
        g.nrows = dim;
        g.mtiles = dim / 128;
        g.out = ws.y;
        gemm<<<sms, kPfThreads, PfSmem::total, s>>>(g);
        k_pairs_down<<<sms, kPcThreads, kPcSmem, s>>>(desc, ids, ws.pairs, ws.npairs, ws.pqh, ws.pdh, dim, ff, tables,
                                                       ws.y, err);
    }
    if (phase_mask & 16) k_prefill_combine<<<T, 256, 0, s>>>(ws.y, ids, w, k, dim, resid, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Batched stack: T tokens through layers 0 .. nl-1 of `desc` ([nl][E]), each layer
// h <- h + layer(RMSNorm(h)) (the single-token stack's recurrence) with the layer as the
// grouped prefill above. Routes: [nl][T][k] ids and weights, or, when `logits` ([nl][T][E])
// is given, top-k by sigmoid per token on the device into the workspace.
size_t stack_batch_workspace_bytes(int T, int k, int dim, int ff, int E) {
    const size_t a = (prefill_workspace_bytes(T, k, dim, ff, E) + 255) & ~(size_t)255;
    const size_t r = ((size_t)T * k * 4 + 255) & ~(size_t)255;
    return a + 2 * r + (size_t)T * dim * 4;
}

void stack_batch_routes(void* wsp, int T, int k, int dim, int ff, int E, int** ids, float** w) {
    uint8_t* base = static_cast<uint8_t*>(wsp);
    const size_t a = (prefill_workspace_bytes(T, k, dim, ff, E) + 255) & ~(size_t)255;
    const size_t r = ((size_t)T * k * 4 + 255) & ~(size_t)255;
    *ids = reinterpret_cast<int*>(base + a);
    *w = reinterpret_cast<float*>(base + a + r);
}

cudaError_t launch_stack_batch(const ExpertDesc* desc, int E, int nl, const float* logits, const int* ids_all,
                               const float* w_all, float* h, int T, int k, int dim, int ff, float limit, void* wsp,
                               int* err, cudaStream_t s, const int* type_masks) {
    uint8_t* base = static_cast<uint8_t*>(wsp);
    const size_t a = (prefill_workspace_bytes(T, k, dim, ff, E) + 255) & ~(size_t)255;
    const size_t r = ((size_t)T * k * 4 + 255) & ~(size_t)255;
    int* rids = reinterpret_cast<int*>(base + a);
    float* rw = reinterpret_cast<float*>(base + a + r);
    float* h2 = reinterpret_cast<float*>(base + a + 2 * r);
    float *hin = h, *hout = h2;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < nl; ++l) {
        const int* ids = ids_all ? ids_all + (size_t)l * T * k : rids;
        const float* w = w_all ? w_all + (size_t)l * T * k : rw;
        if (!ids_all && (e = launch_route_sigmoid(logits + (size_t)l * T * E, E, k, T, rids, rw, s)) != cudaSuccess)
            return e;
        if ((e = launch_prefill(desc + (size_t)l * E, E, hin, ids, w, T, k, dim, ff, limit, hin, hout, wsp, err, 31, s,
                                true, 0, -1, nullptr, type_masks ? type_masks[l] : kTypeBitAll)) != cudaSuccess)
            return e;
        float* t = hin;
        hin = hout;
        hout = t;
    }
    if (hin != h) e = cudaMemcpyAsync(h, hin, (size_t)T * dim * 4, cudaMemcpyDeviceToDevice, s);
    return e;
}

}  // namespace clb
