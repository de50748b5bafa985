// Device building blocks of the routed-expert decode path (sm_100a).
//
// Arithmetic contract: bit-identical to crosslane's CPU-lane restatement
// engine/strata/sycl/stage/wiring/q8k_core.hpp:13-95 for quantisation and row dots:
//   * Q8_K(x): signed max-abs element -> -127, q = min(127, rne(is*x)), d = 1/is;
//   * a row dot keeps the reference's 8 accumulation lanes. Lane L holds positions
//     4L..4L+3 of every 32-value chunk; per block the exact integer lane sum I_L is
//     folded as acc_L = fmaf(half(w.d) * a.d, (float)I_L, acc_L), blocks in order;
//     the row is ((m0+m4)+(m2+m6))+((m1+m5)+(m3+m7)), times 0.125 (IQ2) or plus
//     0.125 * the same sum of the delta lanes (IQ1_M).
// Integer lane sums are computed on the tensor pipe: one mma.sync m16n8k32 s8 per
// 32-value chunk and 16 rows, with the MMA's 8 output columns being the 8 lanes (the
// activation operand is masked per lane), so the column sums ARE the reference's lane
// integers. Every float operation is an explicit _rn intrinsic: nothing is contracted.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "clb_types.h"

namespace clb {

// Activation blocks inside a kernel: qs (int8, 256 per block) and d (fp32 per block).
struct ActView {
    const int8_t* qs;  // shared memory
    const float* d;    // shared memory
};

// Nibble selector tables in shared memory (built by build_tables):
//   grid{XXS,XS,1}[i]: nibble j = symbol of value j of the codebook entry
//                      (IQ2: 8,25,43 -> 0,1,2; IQ1: -1,0,1 -> 0,1,2);
//   sign[s]: nibble j = 4 if sign bit j of ksigns(s) is set (selects the negated byte).
struct Tables {
    uint32_t* xxs;   // 256
    uint32_t* xs;    // 512
    uint32_t* iq1;   // 2048
    uint32_t* sign;  // 128
};

// PRMT sources: byte index 0..3 from `lo`, 4..7 from `hi`.
constexpr uint32_t kIq2Pos = 0x002B1908u;  // +8, +25, +43
constexpr uint32_t kIq2Neg = 0x00D5E7F8u;  // -8, -25, -43
constexpr uint32_t kIq1Val = 0x000100FFu;  // -1, 0, +1

__device__ __forceinline__ uint32_t prmt(uint32_t lo, uint32_t hi, uint32_t sel) { return __byte_perm(lo, hi, sel); }

// D(16x8 s32) = A(16x32 s8) * B(32x8 s8); C = 0.
__device__ __forceinline__ void mma_s8(const uint32_t a[4], uint32_t b0, uint32_t b1, int d[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ float half_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint4 ldg16(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ uint2 ldg8(const void* p) {
    return __ldg(reinterpret_cast<const uint2*>(p));
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// One row's raw data of one block, already in registers.
struct RowBlock {
    uint4 body[4];  // IQ2: 64 B = 8 chunks x 8 B; IQ1_M: qs(32) + qh(16) in body[0..2]
    uint2 sc;       // IQ2_XS scale bytes / IQ1_M scale words
    uint16_t d;     // IQ2 fp16 super-scale
};

template <int T>
__device__ __forceinline__ void load_row_block(const PackedMat& m, int row, int b, RowBlock& rb) {
    const size_t n = (size_t)m.n;
    const uint8_t* body = m.body + ((size_t)b * (T == CLB_IQ1_M ? 3 : 4) * n + row) * 16;
    rb.body[0] = ldg16(body);
    rb.body[1] = ldg16(body + n * 16);
    rb.body[2] = ldg16(body + n * 32);
    if (T != CLB_IQ1_M) rb.body[3] = ldg16(body + n * 48);
    if (T != CLB_IQ2_XXS) rb.sc = ldg8(m.sc + ((size_t)b * n + row) * 8);
    if (T != CLB_IQ1_M) rb.d = __ldg(m.d + (size_t)b * n + row);
}

__device__ __forceinline__ uint32_t word_of(const uint4* body, int w) {
    const uint4 v = body[w >> 2];
    const int s = w & 3;
    return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

// fp16 super-scale of a row block (q8k_core.hpp:70-74 for IQ1_M).
template <int T>
__device__ __forceinline__ float row_scale(const RowBlock& rb) {
    if (T != CLB_IQ1_M) return half_bits(rb.d);
    const uint32_t w01 = rb.sc.x, w23 = rb.sc.y;
    const uint32_t h = ((w01 & 0xffffu) >> 12) | (((w01 >> 16) >> 8) & 0xf0u) | (((w23 & 0xffffu) >> 4) & 0xf00u) |
                       ((w23 >> 16) & 0xf000u);
    return half_bits((uint16_t)h);
}

// Decode group t (8 values, lanes 2t and 2t+1) of chunk c of one row block into two
// int8x4 MMA words, and return the chunk's odd sub-scale for those lanes.
// IQ1_M also returns the group's delta sign (+1/-1).
template <int T>
__device__ __forceinline__ void decode_group(const RowBlock& rb, int c, int t, const Tables& tb, uint32_t& lo,
                                             uint32_t& hi, int& scale, int& delta) {
    if (T == CLB_IQ2_XXS) {
        // packed chunk: [4 grid bytes][4 sign bytes, bit 7 of byte j = sub-scale bit j]
        const uint32_t gw = word_of(rb.body, 2 * c), sw = word_of(rb.body, 2 * c + 1);
        const uint32_t gi = (gw >> (8 * t)) & 0xffu;
        const uint32_t si = (sw >> (8 * t)) & 0x7fu;
        const uint32_t sel = tb.xxs[gi] | tb.sign[si];
        lo = prmt(kIq2Pos, kIq2Neg, sel);
        hi = prmt(kIq2Pos, kIq2Neg, sel >> 16);
        scale = (int)((((sw & 0x80808080u) | 0x08000000u) * 0x00204081u) >> 27);
        delta = 0;
    } else if (T == CLB_IQ2_XS) {
        const uint32_t w = word_of(rb.body, 2 * c + (t >> 1));
        const uint32_t code = (w >> (16 * (t & 1))) & 0xffffu;
        const uint32_t sel = tb.xs[code & 511u] | tb.sign[code >> 9];
        lo = prmt(kIq2Pos, kIq2Neg, sel);
        hi = prmt(kIq2Pos, kIq2Neg, sel >> 16);
        const uint32_t sb = ((c < 4 ? rb.sc.x : rb.sc.y) >> (8 * (c & 3))) & 0xffu;
        scale = (int)(((sb >> (4 * (t >> 1))) & 15u) << 1) | 1;
        delta = 0;
    } else {
        // qs[4c+t] at body byte 4c+t; qh[2c + t/2] at body byte 32 + 2c + t/2.
        const uint32_t qsw = word_of(rb.body, c);
        const uint32_t qhw = word_of(rb.body, 8 + (c >> 1));
        const uint32_t qh = (qhw >> (8 * (2 * (c & 1) + (t >> 1)))) & 0xffu;
        const uint32_t nib = (qh >> (4 * (t & 1))) & 15u;
        const uint32_t idx = ((qsw >> (8 * t)) & 0xffu) | ((nib & 7u) << 8);
        const uint32_t sel = tb.iq1[idx];
        lo = prmt(kIq1Val, 0u, sel);
        hi = prmt(kIq1Val, 0u, sel >> 16);
        const uint32_t scw = (c < 4 ? rb.sc.x : rb.sc.y) >> (16 * ((c >> 1) & 1));
        scale = (int)(((scw >> (6 * (c & 1) + 3 * (t >> 1))) & 7u) << 1) | 1;
        delta = (nib & 8u) ? -1 : 1;
    }
}

// Lane sums and final hsum helpers -------------------------------------------------

// Thread (g = lane/4, t = lane%4) of a warp handles rows g and g+8 of a 16-row tile
// and reference lanes 2t, 2t+1. acc[0..1]: row g lanes 2t,2t+1; acc[2..3]: row g+8.
struct RowAcc {
    float m[4];
    float d[4];  // IQ1_M delta lanes
};

// hsum (q8k_core.hpp:86) across the quad: thread t holds lanes 2t (e) and 2t+1 (o).
__device__ __forceinline__ float quad_hsum(float e, float o) {
    // xor 2 pairs lanes {0,4},{1,5} (t=0 with t=2) and {2,6},{3,7} (t=1 with t=3).
    e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, 2));
    o = __fadd_rn(o, __shfl_xor_sync(0xffffffffu, o, 2));
    // xor 1: (m0+m4)+(m2+m6) and (m1+m5)+(m3+m7).
    e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, 1));
    o = __fadd_rn(o, __shfl_xor_sync(0xffffffffu, o, 1));
    return __fadd_rn(e, o);
}

// Dot of a 16-row tile [r0, r0+16) of matrix m with Q8_K activation `act` (nb blocks).
// Returns, in every thread of quad g, the results of rows r0+g (y[0]) and r0+g+8 (y[1]).
// Rows at or beyond m.n read row m.n-1 (in bounds) and are discarded by the caller.
template <int T>
__device__ __forceinline__ void tile_dot(const PackedMat& m, int r0, const ActView& act, const Tables& tb,
                                         float y[2]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nb = m.k >> 8;
    const int ra = min(r0 + g, m.n - 1), rbw = min(r0 + g + 8, m.n - 1);
    // Activation masks: thread (g,t) feeds B column g from k-slots 4t.. (lane 2t) and
    // 16+4t.. (lane 2t+1); a k-slot carries a value only in its own lane's column.
    const uint32_t mask0 = (g == 2 * t) ? 0xffffffffu : 0u;
    const uint32_t mask1 = (g == 2 * t + 1) ? 0xffffffffu : 0u;
    RowAcc acc;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc.m[i] = acc.d[i] = 0.0f;
    RowBlock cur[2], nxt[2];
    load_row_block<T>(m, ra, 0, cur[0]);
    load_row_block<T>(m, rbw, 0, cur[1]);
    for (int b = 0; b < nb; ++b) {
        if (b + 1 < nb) {
            load_row_block<T>(m, ra, b + 1, nxt[0]);
            load_row_block<T>(m, rbw, b + 1, nxt[1]);
        }
        int im[4] = {0, 0, 0, 0}, id[4] = {0, 0, 0, 0};
        const int8_t* qsb = act.qs + (size_t)b * 256;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint2 qv = *reinterpret_cast<const uint2*>(qsb + 32 * c + 8 * t);
            const uint32_t b0 = qv.x & mask0, b1 = qv.y & mask1;
            uint32_t a[4];
            int sa, sb, da, db;
            decode_group<T>(cur[0], c, t, tb, a[0], a[2], sa, da);
            decode_group<T>(cur[1], c, t, tb, a[1], a[3], sb, db);
            int dv[4];
            mma_s8(a, b0, b1, dv);
            im[0] += sa * dv[0];
            im[1] += sa * dv[1];
            im[2] += sb * dv[2];
            im[3] += sb * dv[3];
            if (T == CLB_IQ1_M) {
                // delta term: scale * delta * (sum of the lane's 4 activations)
                const int q0 = __dp4a((int)qv.x, 0x01010101, 0), q1 = __dp4a((int)qv.y, 0x01010101, 0);
                id[0] += sa * da * q0;
                id[1] += sa * da * q1;
                id[2] += sb * db * q0;
                id[3] += sb * db * q1;
            }
        }
        const float ad = act.d[b];
        const float da_ = __fmul_rn(row_scale<T>(cur[0]), ad);
        const float db_ = __fmul_rn(row_scale<T>(cur[1]), ad);
        acc.m[0] = __fmaf_rn(da_, (float)im[0], acc.m[0]);
        acc.m[1] = __fmaf_rn(da_, (float)im[1], acc.m[1]);
        acc.m[2] = __fmaf_rn(db_, (float)im[2], acc.m[2]);
        acc.m[3] = __fmaf_rn(db_, (float)im[3], acc.m[3]);
        if (T == CLB_IQ1_M) {
            acc.d[0] = __fmaf_rn(da_, (float)id[0], acc.d[0]);
            acc.d[1] = __fmaf_rn(da_, (float)id[1], acc.d[1]);
            acc.d[2] = __fmaf_rn(db_, (float)id[2], acc.d[2]);
            acc.d[3] = __fmaf_rn(db_, (float)id[3], acc.d[3]);
        }
        if (b + 1 < nb) {
            cur[0] = nxt[0];
            cur[1] = nxt[1];
        }
    }
    const float ma = quad_hsum(acc.m[0], acc.m[1]);
    const float mb = quad_hsum(acc.m[2], acc.m[3]);
    if (T == CLB_IQ1_M) {
        const float dsa = quad_hsum(acc.d[0], acc.d[1]);
        const float dsb = quad_hsum(acc.d[2], acc.d[3]);
        y[0] = __fadd_rn(ma, __fmul_rn(0.125f, dsa));
        y[1] = __fadd_rn(mb, __fmul_rn(0.125f, dsb));
    } else {
        y[0] = __fmul_rn(0.125f, ma);
        y[1] = __fmul_rn(0.125f, mb);
    }
}

// Dispatch on the (warp-uniform) matrix type.
__device__ __forceinline__ void tile_dot_any(const PackedMat& m, int r0, const ActView& act, const Tables& tb,
                                             float y[2]) {
    if (m.type == CLB_IQ2_XXS) tile_dot<CLB_IQ2_XXS>(m, r0, act, tb, y);
    else if (m.type == CLB_IQ2_XS) tile_dot<CLB_IQ2_XS>(m, r0, act, tb, y);
    else tile_dot<CLB_IQ1_M>(m, r0, act, tb, y);
}

// Q8_K quantisation of one 256-value block by one warp (q8k_core.hpp:30-38).
// Writes qs (256 int8), *d, and, if bsums != nullptr, 16 int16 sums.
__device__ __forceinline__ void warp_quant_block(const float* x, int8_t* qs, float* d, int16_t* bsums) {
    const int lane = threadIdx.x & 31;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[lane * 8 + i];
    // Signed element of largest magnitude; the first index wins ties.
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
#pragma unroll
        for (int i = 0; i < 8; ++i) qs[lane * 8 + i] = 0;
        if (lane == 0) *d = 0.0f;
        if (bsums && lane < 16) bsums[lane] = 0;
        return;
    }
    const float mx = __shfl_sync(0xffffffffu, v[ai & 7], (ai >> 3) & 31);
    const float is = __fdiv_rn(-127.0f, mx);
    int8_t q[8];
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float z = __fadd_rn(__fmul_rn(is, v[i]), 12582912.0f);
        const int r = (int)(__float_as_uint(z) & 0x007fffffu) - 0x00400000;
        q[i] = (int8_t)(r < 127 ? r : 127);
        s += q[i];
    }
    *reinterpret_cast<uint2*>(qs + lane * 8) =
        make_uint2((uint32_t)(uint8_t)q[0] | (uint32_t)(uint8_t)q[1] << 8 | (uint32_t)(uint8_t)q[2] << 16 |
                       (uint32_t)(uint8_t)q[3] << 24,
                   (uint32_t)(uint8_t)q[4] | (uint32_t)(uint8_t)q[5] << 8 | (uint32_t)(uint8_t)q[6] << 16 |
                       (uint32_t)(uint8_t)q[7] << 24);
    // 16-value sums: lanes 2j and 2j+1 cover values 16j..16j+15.
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (bsums && (lane & 1) == 0) bsums[lane >> 1] = (int16_t)s;
    if (lane == 0) *d = __fdiv_rn(1.0f, is);
}

// SwiGLU (q8k_core.hpp:92-95). exp(-g) is evaluated in double and rounded once to
// float, which is the correctly rounded float in all but vanishingly rare cases; the
// reference CPU lane's glibc expf is likewise within 0.502 ulp, so the two agree on
// nearly every input and otherwise by an ulp. The rest is the reference's float math.
__device__ __forceinline__ float swiglu(float g, float u, float limit) {
    if (limit > 0.0f) {
        g = fminf(g, limit);
        u = fminf(fmaxf(u, -limit), limit);
    }
    const float e = (float)exp(-(double)g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

}  // namespace clb
