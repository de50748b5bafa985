// Row-dot building blocks of the v2 decode kernels, shared by the per-layer kernels
// (clb_kernels.cu) and the persistent stack kernel (clb_stack.cu).
#pragma once
#include "clb_rowdot.cuh"


namespace clb {

constexpr int kV2Threads = 512;          // 16 warps per CTA, one CTA per SM
constexpr int kV2Warps = kV2Threads / 32;
constexpr int kActStride = 272;          // padded Q8_K block stride in shared memory
constexpr int kXchWords = 18;            // per (row, block-slot) exchange record

// Q8_K of 256 values held 8 per lane (lane i holds values 8i..8i+7), as warp_quant_block.
__device__ __forceinline__ void warp_quant_regs(float v[8], int8_t* qs, float* d) {
    const int lane = threadIdx.x & 31;
    float am = 0.0f;
    int ai = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > am) { am = a; ai = lane * 8 + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, am, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ai, o);
        if (oa > am || (oa == am && oi < ai)) { am = oa; ai = oi; }
    }
    if (am == 0.0f) {
        *reinterpret_cast<uint2*>(qs + lane * 8) = make_uint2(0u, 0u);
        if (lane == 0) *d = 0.0f;
        return;
    }
    float mine = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
        if ((ai & 7) == i) mine = v[i];
    const float mx = __shfl_sync(0xffffffffu, mine, (ai >> 3) & 31);
    const float is = __fdiv_rn(-127.0f, mx);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float z = __fadd_rn(__fmul_rn(is, v[i]), 12582912.0f);
        int r = (int)(__float_as_uint(z) & 0x007fffffu) - 0x00400000;
        r = r < 127 ? r : 127;
        packed[i >> 2] |= ((uint32_t)(uint8_t)(int8_t)r) << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(qs + lane * 8) = make_uint2(packed[0], packed[1]);
    if (lane == 0) *d = __fdiv_rn(1.0f, is);
}

// Gate/up item for one warp: 8 rows of one matrix; 4 threads per row split the blocks
// (thread k takes blocks k, k+4, ...). Per round the 4 threads exchange their blocks'
// lane integers through shared memory so that thread k folds lanes 2k, 2k+1 of all 4
// blocks in block order, exactly the reference chain. Returns the row value in k == 0.
// Not inlined: each quant type gets its own register allocation (inlined together the
// three paths exceed 128 registers); the call happens once per warp item.
// L2 prefetch of one row block (no registers held).
template <int T>
__device__ __forceinline__ void prefetch_raw(const PackedMat& m, int row, int b) {
    const size_t n = (size_t)m.n;
    const uint8_t* p = m.body + ((size_t)b * (T == CLB_IQ1_M ? 3 : 4) * n + (size_t)row) * 16;
    prefetch_l2(p);
    prefetch_l2(p + n * 16);
    prefetch_l2(p + n * 32);
    if (T != CLB_IQ1_M) prefetch_l2(p + n * 48);
}

template <int T, bool PF>
__device__ __noinline__ float quad_row_dot(const PackedMat& m, int row, const int8_t* act_qs, const float* act_d,
                                           uint32_t* xch) {
    const int lane = threadIdx.x & 31, k = lane & 3, rr = lane >> 2;
    const uint32_t lb = (uint32_t)lane * 4u;
    const int nb = m.k >> 8;
    const int rounds = (nb + 3) >> 2;
    float acc0 = 0.0f, acc1 = 0.0f, dacc0 = 0.0f, dacc1 = 0.0f;
    // One round: decode block b = 4i + k from `r`, exchange lane integers within the
    // row's 4 threads, fold blocks 4i..4i+3 in order into lanes 2k, 2k+1.
    auto round = [&](int i, const RowRaw& r) {
        const int b = 4 * i + k;
        int I[8], D[8];
        float dd = 0.0f;
        if (b < nb) {
            block_lanes<T>(r, act_qs + (size_t)b * kActStride, lb, I, D);
            dd = __fmul_rn(raw_scale<T>(r), act_d[b]);
        } else {
#pragma unroll
            for (int L = 0; L < 8; ++L) I[L] = D[L] = 0;
        }
        uint32_t* mine = xch + (rr * 4 + k) * kXchWords;
#pragma unroll
        for (int L = 0; L < 8; ++L) mine[L] = (uint32_t)I[L];
        mine[8] = __float_as_uint(dd);
        if (T == CLB_IQ1_M) {
#pragma unroll
            for (int L = 0; L < 8; ++L) mine[9 + L] = (uint32_t)D[L];
        }
        __syncwarp();
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            if (4 * i + s < nb) {
                const uint32_t* src = xch + (rr * 4 + s) * kXchWords;
                const float ds = __uint_as_float(src[8]);
                acc0 = __fmaf_rn(ds, (float)(int)src[2 * k], acc0);
                acc1 = __fmaf_rn(ds, (float)(int)src[2 * k + 1], acc1);
                if (T == CLB_IQ1_M) {
                    dacc0 = __fmaf_rn(ds, (float)(int)src[9 + 2 * k], dacc0);
                    dacc1 = __fmaf_rn(ds, (float)(int)src[9 + 2 * k + 1], dacc1);
                }
            }
        }
        __syncwarp();
    };
    if (PF) {
        // ping-pong: round i decodes buffer i%2 while the loads of round i+1 are in flight
        RowRaw ra, rb;
        if (k < nb) load_raw_early<T>(m, row, k, ra);
        for (int i = 0; i < rounds; i += 2) {
            if (4 * (i + 1) + k < nb) load_raw_early<T>(m, row, 4 * (i + 1) + k, rb);
            round(i, ra);
            if (i + 1 >= rounds) break;
            if (4 * (i + 2) + k < nb) load_raw_early<T>(m, row, 4 * (i + 2) + k, ra);
            round(i + 1, rb);
        }
    } else {
        RowRaw cur;
        for (int i = 0; i < rounds; ++i) {
            const int b = 4 * i + k;
            if (b + 4 < nb) prefetch_raw<T>(m, row, b + 4);
            if (b < nb) load_raw<T>(m, row, b, cur);
            round(i, cur);
        }
    }
    const float main = quad_hsum(acc0, acc1);
    if (T == CLB_IQ1_M) return __fadd_rn(main, __fmul_rn(0.125f, quad_hsum(dacc0, dacc1)));
    return __fmul_rn(0.125f, main);
}

template <int T, bool PF>
__device__ __noinline__ float thread_row_dot(const PackedMat& m, int row, const int8_t* act_qs, const float* act_d) {
    const uint32_t lb = (uint32_t)(threadIdx.x & 31) * 4u;
    const int nb = m.k >> 8;
    float acc[8], dacc[8];
#pragma unroll
    for (int L = 0; L < 8; ++L) acc[L] = dacc[L] = 0.0f;
    auto step = [&](int b, const RowRaw& r) {
        int I[8], D[8];
        block_lanes<T>(r, act_qs + (size_t)b * kActStride, lb, I, D);
        const float dd = __fmul_rn(raw_scale<T>(r), act_d[b]);
#pragma unroll
        for (int L = 0; L < 8; ++L) {
            acc[L] = __fmaf_rn(dd, (float)I[L], acc[L]);
            if (T == CLB_IQ1_M) dacc[L] = __fmaf_rn(dd, (float)D[L], dacc[L]);
        }
    };
    if (PF) {
        RowRaw ra, rb;
        load_raw_early<T>(m, row, 0, ra);
        for (int b = 0; b < nb; b += 2) {
            if (b + 1 < nb) load_raw_early<T>(m, row, b + 1, rb);
            step(b, ra);
            if (b + 1 >= nb) break;
            if (b + 2 < nb) load_raw_early<T>(m, row, b + 2, ra);
            step(b + 1, rb);
        }
    } else {
        RowRaw cur;
        for (int b = 0; b < nb; ++b) {
            if (b + 1 < nb) prefetch_raw<T>(m, row, b + 1);
            load_raw<T>(m, row, b, cur);
            step(b, cur);
        }
    }
    const float main = hsum8_rn(acc);
    if (T == CLB_IQ1_M) return __fadd_rn(main, __fmul_rn(0.125f, hsum8_rn(dacc)));
    return __fmul_rn(0.125f, main);
}

// One block of a fast-order row segment: block_sum's exact integers, scaled once by
// d_w * d_x and accumulated in fp32.
template <int T>
__device__ __forceinline__ void seg_block(const RowRaw& r, const int8_t* act_qs, const float* act_d, int b,
                                          uint32_t lb, float& acc, float& dacc) {
    int M, D;
    block_sum<T>(r, act_qs + (size_t)b * kActStride, lb, M, D);
    const float dd = __fmul_rn(raw_scale<T>(r), act_d[b]);
    acc = __fmaf_rn(dd, (float)M, acc);
    if (T == CLB_IQ1_M) dacc = __fmaf_rn(dd, (float)D, dacc);
}

// Fast math: the S threads of a row (lanes base..base+S-1, k = lane % S) each stream
// the contiguous block range [k*ceil(nb/S), (k+1)*ceil(nb/S)) and accumulate fp32
// partials acc += d_b * M_b (and the IQ1_M delta); the partials are then added in lane
// order p_0 + p_1 + ... + p_{S-1}, so results are run-to-run identical and differ from
// the reference's per-lane order only by fp32 reassociation. Every lane returns the row
// value. Lanes past the last full group of S compute a throw-away copy.
// PF: the next block is loaded into registers while the current one is decoded (two
// register buffers, alternating), with an L2 prefetch two blocks ahead; otherwise each
// block is loaded at the top of its iteration behind an L2 prefetch one block ahead.
template <int T, bool PF, int S>
__device__ __noinline__ float seg_row_dot(const PackedMat& m, int row, const int8_t* act_qs, const float* act_d) {
    const int lane = threadIdx.x & 31, k = lane % S, base = lane - k;
    const uint32_t lb = (uint32_t)lane * 4u;
    const int nb = m.k >> 8;
    const int per = (nb + S - 1) / S, b0 = k * per, b1 = min(nb, b0 + per);
    float acc = 0.0f, dacc = 0.0f;
    if (PF) {
        RowRaw ra, rb;
        if (b0 < b1) load_raw_early<T>(m, row, b0, ra);
        if (b0 + 1 < b1) prefetch_raw<T>(m, row, b0 + 1);
        for (int b = b0; b < b1; b += 2) {
            if (b + 1 < b1) load_raw_early<T>(m, row, b + 1, rb);
            if (b + 2 < b1) prefetch_raw<T>(m, row, b + 2);
            seg_block<T>(ra, act_qs, act_d, b, lb, acc, dacc);
            if (b + 1 >= b1) break;
            if (b + 2 < b1) load_raw_early<T>(m, row, b + 2, ra);
            if (b + 3 < b1) prefetch_raw<T>(m, row, b + 3);
            seg_block<T>(rb, act_qs, act_d, b + 1, lb, acc, dacc);
        }
    } else {
        for (int b = b0; b < b1; ++b) {
            if (b + 1 < b1) prefetch_raw<T>(m, row, b + 1);
            RowRaw r;
            load_raw<T>(m, row, b, r);
            seg_block<T>(r, act_qs, act_d, b, lb, acc, dacc);
        }
    }
    float tot = __shfl_sync(0xffffffffu, acc, base);
    float dtot = 0.0f;
    if (T == CLB_IQ1_M) dtot = __shfl_sync(0xffffffffu, dacc, base);
#pragma unroll
    for (int j = 1; j < S; ++j) {
        tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, acc, (base + j) & 31));
        if (T == CLB_IQ1_M) dtot = __fadd_rn(dtot, __shfl_sync(0xffffffffu, dacc, (base + j) & 31));
    }
    if (T == CLB_IQ1_M) return __fadd_rn(tot, __fmul_rn(0.125f, dtot));
    return __fmul_rn(0.125f, tot);
}
template <bool PF, int S>
__device__ __forceinline__ float seg_row_dot_t(const PackedMat& m, int row, const int8_t* aq, const float* ad) {
    if (m.type == CLB_IQ2_XXS) return seg_row_dot<CLB_IQ2_XXS, PF, S>(m, row, aq, ad);
    if (m.type == CLB_IQ2_XS) return seg_row_dot<CLB_IQ2_XS, PF, S>(m, row, aq, ad);
    return seg_row_dot<CLB_IQ1_M, PF, S>(m, row, aq, ad);
}
// ---- fast order, one row per lane ----
// All lanes of a warp decode the same blocks of 32 consecutive rows, so every read of
// the activation block is a warp-wide broadcast and every weight load is 32 rows x 16
// contiguous bytes. Returns the row's partial over blocks [b0, b1) in block order:
// IQ2: 0.125 * sum d_b M_b; IQ1_M: sum d_b M_b + 0.125 * sum d_b D_b (block_sum's
// integers, d_b = d_w * d_x). The caller adds the partials of a row's K segments in a
// fixed order. AS: byte stride of the activation's 256-value blocks (kActStride in shared
// memory; 256 for an unpadded Q8_K row read from global memory, where the warp-wide
// broadcast reads hit L1).
template <int T, int AS = kActStride>
__device__ __noinline__ float lane_row_partial(const PackedMat& m, int row, int b0, int b1, const int8_t* act_qs,
                                               const float* act_d) {
    constexpr int NP = T == CLB_IQ1_M ? 3 : 4;
    const uint32_t lb = (threadIdx.x & 31) * 4u;
    const size_t n = (size_t)m.n, pstride = n * 16, bstride = (size_t)NP * n * 16;
    const uint8_t* p = m.body + (size_t)b0 * bstride + (size_t)row * 16;
    const uint8_t* sc = T == CLB_IQ2_XXS ? nullptr : m.sc + ((size_t)b0 * n + (size_t)row) * 8;
    const uint16_t* dp = T == CLB_IQ1_M ? nullptr : m.d + (size_t)b0 * n + (size_t)row;
    float acc = 0.0f, dacc = 0.0f;
    for (int b = b0; b < b1; ++b) {
        if (b + 1 < b1) {
            const uint8_t* q = p + bstride;
            prefetch_l2(q);
            prefetch_l2(q + pstride);
            prefetch_l2(q + 2 * pstride);
            if (T != CLB_IQ1_M) prefetch_l2(q + 3 * pstride);
        }
        RowRaw r;
        r.b0 = __ldg(reinterpret_cast<const uint4*>(p));
        r.b1 = __ldg(reinterpret_cast<const uint4*>(p + pstride));
        r.b2 = __ldg(reinterpret_cast<const uint4*>(p + 2 * pstride));
        if (T != CLB_IQ1_M) r.b3 = __ldg(reinterpret_cast<const uint4*>(p + 3 * pstride));
        if (T != CLB_IQ2_XXS) r.sc = __ldg(reinterpret_cast<const uint2*>(sc));
        if (T != CLB_IQ1_M) r.d = __ldg(dp);
        int M, D;
        block_sum<T>(r, act_qs + (size_t)b * AS, lb, M, D);
        const float dd = __fmul_rn(raw_scale<T>(r), act_d[b]);
        acc = __fmaf_rn(dd, (float)M, acc);
        if (T == CLB_IQ1_M) dacc = __fmaf_rn(dd, (float)D, dacc);
        p += bstride;
        if (T != CLB_IQ2_XXS) sc += n * 8;
        if (T != CLB_IQ1_M) dp += n;
    }
    if (T == CLB_IQ1_M) return __fadd_rn(acc, __fmul_rn(0.125f, dacc));
    return __fmul_rn(0.125f, acc);
}
template <int AS = kActStride>
__device__ __forceinline__ float lane_row_partial_any(const PackedMat& m, int row, int b0, int b1, const int8_t* aq,
                                                      const float* ad) {
    if (m.type == CLB_IQ2_XXS) return lane_row_partial<CLB_IQ2_XXS, AS>(m, row, b0, b1, aq, ad);
    if (m.type == CLB_IQ2_XS) return lane_row_partial<CLB_IQ2_XS, AS>(m, row, b0, b1, aq, ad);
    return lane_row_partial<CLB_IQ1_M, AS>(m, row, b0, b1, aq, ad);
}

// ---- fast order, one row per lane, rolling register reload (the persistent stack kernel) ----
// block_sum's exact integers, except that IQ1_M folds its delta into the main sum: every
// weight becomes the integer 8q + delta (q in {-1, 0, 1}, delta = +-1 per 8-value group,
// |8q + delta| <= 9), taken straight from the byte pairs {-7, 1, 9} | {-9, -1, 7} with the
// group's delta sign as selector bit 2, so one dp4a per 4 weights gives
// 8 * main + delta (q8k_core.hpp:79-84 keeps them apart: main + delta / 8 is 1/8 of it).

// Streaming weight loads: read once, so they bypass L1 allocation and leave the L1 lines
// to the data that is reused (activations, the stack).
__device__ __forceinline__ uint4 ldg_v4_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_v2_stream(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16_stream(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

template <int T>
__device__ __forceinline__ void load_raw_at(const uint8_t* p, size_t pstride, const uint8_t* sc, const uint16_t* dp,
                                            RowRaw& r) {
    r.b0 = ldg_v4_stream(p);
    r.b1 = ldg_v4_stream(p + pstride);
    r.b2 = ldg_v4_stream(p + 2 * pstride);
    if (T != CLB_IQ1_M) r.b3 = ldg_v4_stream(p + 3 * pstride);
    if (T != CLB_IQ2_XXS) r.sc = ldg_v2_stream(sc);
    if (T != CLB_IQ1_M) r.d = ldg_u16_stream(dp);
}

// One 32-value chunk c of a block: the chunk's exact integer (IQ1_M: 8q + delta), from the
// chunk's 32 activations qv, with the IQ2_XS / IQ1_M scale bytes taken from scx (chunks
// 0-3) / scy (chunks 4-7).
template <int T>
__device__ __forceinline__ int chunk_sum8_q(const RowRaw& r, const uint32_t qv[8], uint32_t lb, int c, uint32_t scx,
                                            uint32_t scy) {
    if (T == CLB_IQ2_XXS) {
        const uint32_t gw = rw(r, 2 * c), sw = rw(r, 2 * c + 1);
        const int scale = (int)((((sw & 0x80808080u) | 0x08000000u) * 0x00204081u) >> 27);
        uint32_t sel[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sel_j = 0x5504u | ((uint32_t)j << 4);
            sel[j] = tab32(kRowTabXXS + prmt2(gw, lb, sel_j)) | tab32(kRowTabXXS + 128 + prmt2(sw, lb, sel_j));
        }
        int a = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            a = __dp4a((int)prmt_k<kPos2, kNeg2>(sel[j]), (int)qv[2 * j], a);
            a = __dp4a((int)prmt_k<kPos2, kNeg2>(sel[j] >> 16), (int)qv[2 * j + 1], a);
        }
        return scale * a;
    } else if (T == CLB_IQ2_XS) {
        const uint32_t scb = ((c < 4 ? scx : scy) >> (8 * (c & 3))) & 0xffu;
        const int s_lo = (int)((scb & 15u) << 1) | 1, s_hi = (int)((scb >> 4) << 1) | 1;
        uint32_t sel[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w = rw(r, 2 * c + (j >> 1));
            const uint32_t code = (j & 1) ? (w >> 16) : (w & 0xffffu);
            sel[j] = tab32(kRowTabXS + (code & 511u) * 64u + (lb & 60u)) |
                     tab32(kRowTabXXS + (code >> 9) * 256u + 128u + lb);
        }
        int alo = 0, ahi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int& a = j < 2 ? alo : ahi;
            a = __dp4a((int)prmt_k<kPos2, kNeg2>(sel[j]), (int)qv[2 * j], a);
            a = __dp4a((int)prmt_k<kPos2, kNeg2>(sel[j] >> 16), (int)qv[2 * j + 1], a);
        }
        return s_lo * alo + s_hi * ahi;
    } else {
        const uint32_t qsw = rw(r, c);
        const uint32_t qh16 = (rw(r, 8 + (c >> 1)) >> (16 * (c & 1))) & 0xffffu;
        const uint32_t scw = ((c < 4 ? scx : scy) >> (16 * ((c >> 1) & 1))) & 0xffffu;
        const int s_lo = (int)(((scw >> (6 * (c & 1))) & 7u) << 1) | 1;
        const int s_hi = (int)(((scw >> (6 * (c & 1) + 3)) & 7u) << 1) | 1;
        int alo = 0, ahi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t nib = (qh16 >> (4 * j)) & 15u;
            const uint32_t idx = ((qsw >> (8 * j)) & 0xffu) | ((nib & 7u) << 8);
            const uint32_t sel = tab32(kRowTabIQ1 + idx * 16u + (lb & 12u)) | ((nib & 8u) ? 0x44444444u : 0u);
            int& a = j < 2 ? alo : ahi;
            a = __dp4a((int)prmt_k<kIq1DeltaPos, kIq1DeltaNeg>(sel), (int)qv[2 * j], a);
            a = __dp4a((int)prmt_k<kIq1DeltaPos, kIq1DeltaNeg>(sel >> 16), (int)qv[2 * j + 1], a);
        }
        return s_lo * alo + s_hi * ahi;
    }
}
template <int T>
__device__ __forceinline__ int chunk_sum8(const RowRaw& r, const int8_t* q, uint32_t lb, int c, uint32_t scx,
                                          uint32_t scy) {
    const uint4 qa = *reinterpret_cast<const uint4*>(q + 32 * c);
    const uint4 qb = *reinterpret_cast<const uint4*>(q + 32 * c + 16);
    const uint32_t qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    return chunk_sum8_q<T>(r, qv, lb, c, scx, scy);
}

// Partial of one row over blocks [b0, b1): 0.125 * sum_b (d_w * d_x)_b * M_b with M_b the
// block's exact integer (the sum of chunk_sum8; for IQ1_M 8q + delta), blocks in order,
// fp32. AS: byte stride of the activation blocks (kActStride in shared memory).
// Rolling register reload: the next block's 16-byte pieces
// are loaded into the registers of the current block's pieces as soon as the chunks that
// read them are done (IQ2: piece p holds chunks 2p, 2p+1; IQ1_M: qs pieces 0 / 1 hold
// chunks 0-3 / 4-7, the qh piece all of them), and the scale bytes right after they are
// copied at the block start. Each load gets most of a block's decode time to land, at no
// register cost beyond the scale copies.
template <int T, int AS = kActStride>
__device__ __noinline__ float lane_row_roll(const PackedMat& m, int row, int b0, int b1, const int8_t* act_qs,
                                            const float* act_d) {
    constexpr int NP = T == CLB_IQ1_M ? 3 : 4;
    const uint32_t lb = (threadIdx.x & 31) * 4u;
    const size_t n = (size_t)m.n, pstride = n * 16, bstride = (size_t)NP * n * 16;
    const uint8_t* p = m.body + (size_t)b0 * bstride + (size_t)row * 16;
    const uint8_t* sc = T == CLB_IQ2_XXS ? nullptr : m.sc + ((size_t)b0 * n + (size_t)row) * 8;
    const uint16_t* dp = T == CLB_IQ1_M ? nullptr : m.d + (size_t)b0 * n + (size_t)row;
    float acc = 0.0f;
    if (b0 >= b1) return 0.0f;
    RowRaw r;
    load_raw_at<T>(p, pstride, sc, dp, r);
    for (int b = b0; b < b1; ++b) {
        const bool more = b + 1 < b1;
        p += bstride;
        if (T != CLB_IQ2_XXS) sc += n * 8;
        if (T != CLB_IQ1_M) dp += n;
        const float dd = __fmul_rn(raw_scale<T>(r), act_d[b]);
        const uint32_t scx = r.sc.x, scy = r.sc.y;
        if (more) {
            if (T != CLB_IQ2_XXS) r.sc = ldg_v2_stream(sc);
            if (T != CLB_IQ1_M) r.d = ldg_u16_stream(dp);
        }
        const int8_t* q = act_qs + (size_t)b * AS;
        int M = 0;
        if (T != CLB_IQ1_M) {
            M += chunk_sum8<T>(r, q, lb, 0, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 1, scx, scy);
            if (more) r.b0 = ldg_v4_stream(p);
            M += chunk_sum8<T>(r, q, lb, 2, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 3, scx, scy);
            if (more) r.b1 = ldg_v4_stream(p + pstride);
            M += chunk_sum8<T>(r, q, lb, 4, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 5, scx, scy);
            if (more) r.b2 = ldg_v4_stream(p + 2 * pstride);
            M += chunk_sum8<T>(r, q, lb, 6, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 7, scx, scy);
            if (more) r.b3 = ldg_v4_stream(p + 3 * pstride);
        } else {
            M += chunk_sum8<T>(r, q, lb, 0, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 1, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 2, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 3, scx, scy);
            if (more) r.b0 = ldg_v4_stream(p);
            M += chunk_sum8<T>(r, q, lb, 4, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 5, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 6, scx, scy);
            M += chunk_sum8<T>(r, q, lb, 7, scx, scy);
            if (more) {
                r.b1 = ldg_v4_stream(p + pstride);
                r.b2 = ldg_v4_stream(p + 2 * pstride);
            }
        }
        acc = __fmaf_rn(dd, (float)M, acc);
    }
    return __fmul_rn(0.125f, acc);
}
template <int AS = kActStride>
__device__ __forceinline__ float lane_row_roll_any(const PackedMat& m, int row, int b0, int b1, const int8_t* aq,
                                                   const float* ad) {
    if (m.type == CLB_IQ2_XXS) return lane_row_roll<CLB_IQ2_XXS, AS>(m, row, b0, b1, aq, ad);
    if (m.type == CLB_IQ2_XS) return lane_row_roll<CLB_IQ2_XS, AS>(m, row, b0, b1, aq, ad);
    return lane_row_roll<CLB_IQ1_M, AS>(m, row, b0, b1, aq, ad);
}

// S in {1, 2, 3, 4, 6, 8} (kSegChoices); anything else is treated as 1.
template <bool PF>
__device__ __forceinline__ float seg_row_dot_any(const PackedMat& m, int row, int S, const int8_t* aq,
                                                 const float* ad) {
    switch (S) {
        case 2: return seg_row_dot_t<PF, 2>(m, row, aq, ad);
        case 3: return seg_row_dot_t<PF, 3>(m, row, aq, ad);
        case 4: return seg_row_dot_t<PF, 4>(m, row, aq, ad);
        case 6: return seg_row_dot_t<PF, 6>(m, row, aq, ad);
        case 8: return seg_row_dot_t<PF, 8>(m, row, aq, ad);
        default: return seg_row_dot_t<PF, 1>(m, row, aq, ad);
    }
}

template <bool PF>
__device__ __forceinline__ float quad_row_dot_any(const PackedMat& m, int row, const int8_t* aq, const float* ad,
                                                  uint32_t* xch) {
    if (m.type == CLB_IQ2_XXS) return quad_row_dot<CLB_IQ2_XXS, PF>(m, row, aq, ad, xch);
    if (m.type == CLB_IQ2_XS) return quad_row_dot<CLB_IQ2_XS, PF>(m, row, aq, ad, xch);
    return quad_row_dot<CLB_IQ1_M, PF>(m, row, aq, ad, xch);
}
template <bool PF>
__device__ __forceinline__ float thread_row_dot_any(const PackedMat& m, int row, const int8_t* aq, const float* ad) {
    if (m.type == CLB_IQ2_XXS) return thread_row_dot<CLB_IQ2_XXS, PF>(m, row, aq, ad);
    if (m.type == CLB_IQ2_XS) return thread_row_dot<CLB_IQ2_XS, PF>(m, row, aq, ad);
    return thread_row_dot<CLB_IQ1_M, PF>(m, row, aq, ad);
}

// Shared-memory copy of Q8_K activations (qs int8 + d floats, from global) with the
// padded block stride.
__device__ __forceinline__ void stage_act(const int8_t* __restrict__ qs, const float* __restrict__ d, int nblocks,
                                          int8_t* aq, float* ad) {
    for (int i = threadIdx.x; i < nblocks * 16; i += blockDim.x) {
        const int b = i >> 4, p = i & 15;
        *reinterpret_cast<uint4*>(aq + (size_t)b * kActStride + 16 * p) =
            reinterpret_cast<const uint4*>(qs + (size_t)b * 256)[p];
    }
    for (int b = threadIdx.x; b < nblocks; b += blockDim.x) ad[b] = d[b];
}

}  // namespace clb
