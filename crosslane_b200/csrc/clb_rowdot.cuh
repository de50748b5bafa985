// Row-per-thread IQ decode (v2): one thread decodes whole 256-value blocks of one row
// and keeps all 8 of the reference's accumulation lanes in registers.
//
// Arithmetic (bit-identical to crosslane's q8k_core.hpp:43-91): for lane L (positions
// 4L..4L+3 of every 32-value chunk) the exact integer I_L = sum_c scale_c * dot4, and
// for IQ1_M the delta integer D_L = sum_c scale_c * delta_group * sum(q of lane L).
// dp4a forms each 4-value dot; the odd sub-scale multiplies it with an integer
// multiply-add, so every I_L is exact.
//
// Decode: a 32-bit "selector" per group of 8 values holds one nibble per value:
// bits 0-1 the magnitude symbol (IQ2: 8,25,43 -> 0,1,2; IQ1: -1,0,1 -> 0,1,2) and bit 2
// the sign; prmt.b32 turns 4 nibbles into 4 signed int8 from the byte pair
// {+8,+25,+43 | -8,-25,-43} (or {-1,0,+1}). Selectors come from shared-memory tables
// replicated per lane so that 32 random lookups hit 32 different banks.
//
// Shared-memory tables (kRowTableBytes = 128 KiB), filled by fill_row_tables():
//   [0, 64K)    256 slots x 256 B: slot i = 32 copies of the IQ2_XXS grid selector i,
//               then 32 copies of the sign selector ksigns(i & 127). A table address is
//               then byte*256 + lane*4, which one prmt builds from a data byte.
//   [64K, 96K)  IQ2_XS grid selectors, 512 x 16 copies (address idx*64 + (lane&15)*4).
//   [96K, 128K) IQ1_M grid selectors, 2048 x 4 copies (address idx*16 + (lane&3)*4).
// fill_row_tables() also writes the 16 bytes of static shared memory clb_prmt_k (the byte
// tables of the fast-order prmt decode); kernels that launch with the most dynamic shared
// memory subtract them from the opt-in limit.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "clb_types.h"

namespace clb {

constexpr uint32_t kRowTabXXS = 0;
constexpr uint32_t kRowTabXS = 64 * 1024;
constexpr uint32_t kRowTabIQ1 = 96 * 1024;
constexpr uint32_t kRowTableBytes = 128 * 1024;

constexpr uint32_t kPos2 = 0x002B1908u;  // +8, +25, +43
constexpr uint32_t kNeg2 = 0x00D5E7F8u;  // -8, -25, -43
constexpr uint32_t kVal1 = 0x000100FFu;  // -1, 0, +1
constexpr uint32_t kIq1DeltaPos = 0x000901F9u;  // -7, 1, 9 (IQ1_M 8q + delta, delta = +1)
constexpr uint32_t kIq1DeltaNeg = 0x0007FFF7u;  // -9, -1, 7 (delta = -1)

// Byte permute (PTX prmt.b32, default mode) through the intrinsic, so constant operands
// become immediates instead of registers the compiler re-materialises.
__device__ __forceinline__ uint32_t prmt2(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }
// The same permute with a run-time selector taken from the tables: every selector nibble
// there is 0..6 (bit 3 clear), where prmt.b32 and __byte_perm agree, so the instruction
// is issued as is (the intrinsic would first mask the selector to 3-bit nibbles).
__device__ __forceinline__ uint32_t prmt_sel(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// The byte tables of the prmt decode {kPos2, kNeg2, kIq1DeltaPos, kIq1DeltaNeg} in shared
// memory, written by fill_row_tables: the decode loads them once per call, so both prmt
// operands stay in registers (as immediates the compiler re-creates them with a move
// before every prmt, which doubled the FMA-pipe instructions of the decode).
__shared__ uint32_t clb_prmt_k[4];
// prmt_sel with the byte tables A (bytes 0-3) and B (bytes 4-7) of clb_prmt_k.
template <uint32_t A, uint32_t B>
__device__ __forceinline__ uint32_t prmt_k(uint32_t sel) {
    static_assert((A == kPos2 && B == kNeg2) || (A == kIq1DeltaPos && B == kIq1DeltaNeg), "a table of clb_prmt_k");
    const int i = A == kPos2 ? 0 : 2;
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(clb_prmt_k[i]), "r"(clb_prmt_k[i + 1]), "r"(sel));
    return d;
}
// Table word at byte offset `off` of the kernel's dynamic shared memory. Indexing the
// extern __shared__ array directly lets the compiler fold its base into the load's
// immediate and schedule the load early.
extern __shared__ __align__(16) uint8_t clb_dyn_smem[];
__device__ __forceinline__ uint32_t tab32(uint32_t off) {
    return *reinterpret_cast<const uint32_t*>(clb_dyn_smem + off);
}
__device__ __forceinline__ int dp4a_s(uint32_t a, uint32_t b) {
    return __dp4a((int)a, (int)b, 0);
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Compact selectors (256 + 512 + 2048 + 128 words, clb_kernels.h layout) -> replicated
// shared-memory tables, using `stage` (2944 words of shared memory past the tables) to
// read the compact copy from global memory once with independent loads. Called by every
// thread of the CTA; the caller syncs afterwards.
__device__ __forceinline__ void fill_row_tables(const uint32_t* __restrict__ compact, uint32_t* stage) {
    for (int i = threadIdx.x; i < 2944; i += blockDim.x) stage[i] = __ldg(compact + i);
    if (threadIdx.x < 4) clb_prmt_k[threadIdx.x] = threadIdx.x == 0 ? kPos2 : threadIdx.x == 1 ? kNeg2
                                                  : threadIdx.x == 2 ? kIq1DeltaPos : kIq1DeltaNeg;
    __syncthreads();
    uint4* a = reinterpret_cast<uint4*>(clb_dyn_smem + kRowTabXXS);
    for (int s = threadIdx.x; s < 4096; s += blockDim.x) {  // slot i: 8 x grid, 8 x sign
        const int slot = s >> 4, part = s & 15;
        const uint32_t v = part < 8 ? stage[slot] : stage[2816 + (slot & 127)];
        a[s] = make_uint4(v, v, v, v);
    }
    uint4* b = reinterpret_cast<uint4*>(clb_dyn_smem + kRowTabXS);
    for (int s = threadIdx.x; s < 2048; s += blockDim.x) {  // 512 entries x 16 copies
        const uint32_t v = stage[256 + (s >> 2)];
        b[s] = make_uint4(v, v, v, v);
    }
    uint4* c = reinterpret_cast<uint4*>(clb_dyn_smem + kRowTabIQ1);
    for (int s = threadIdx.x; s < 2048; s += blockDim.x) {  // 2048 entries x 4 copies
        const uint32_t v = stage[768 + s];
        c[s] = make_uint4(v, v, v, v);
    }
}

// Raw data of one row's block.
struct RowRaw {
    uint4 b0, b1, b2, b3;  // body pieces (IQ1_M uses b0..b2)
    uint2 sc;              // IQ2_XS scale bytes / IQ1_M scale words
    uint16_t d;            // IQ2 fp16 super-scale
};

// 128/64/16-bit global loads through the non-coherent path that the compiler may not
// move: a prefetch issued with them really starts a round ahead of its use.
__device__ __forceinline__ uint4 ldg_v4_early(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_v2_early(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16_early(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

template <int T>
__device__ __forceinline__ void load_raw_early(const PackedMat& m, int row, int b, RowRaw& r) {
    const size_t n = (size_t)m.n;
    const uint8_t* p = m.body + ((size_t)b * (T == CLB_IQ1_M ? 3 : 4) * n + (size_t)row) * 16;
    r.b0 = ldg_v4_early(p);
    r.b1 = ldg_v4_early(p + n * 16);
    r.b2 = ldg_v4_early(p + n * 32);
    if (T != CLB_IQ1_M) r.b3 = ldg_v4_early(p + n * 48);
    if (T != CLB_IQ2_XXS) r.sc = ldg_v2_early(m.sc + ((size_t)b * n + row) * 8);
    if (T != CLB_IQ1_M) r.d = ldg_u16_early(m.d + (size_t)b * n + row);
}

template <int T>
__device__ __forceinline__ void load_raw(const PackedMat& m, int row, int b, RowRaw& r) {
    const size_t n = (size_t)m.n;
    const uint8_t* p = m.body + ((size_t)b * (T == CLB_IQ1_M ? 3 : 4) * n + (size_t)row) * 16;
    r.b0 = __ldg(reinterpret_cast<const uint4*>(p));
    r.b1 = __ldg(reinterpret_cast<const uint4*>(p + n * 16));
    r.b2 = __ldg(reinterpret_cast<const uint4*>(p + n * 32));
    if (T != CLB_IQ1_M) r.b3 = __ldg(reinterpret_cast<const uint4*>(p + n * 48));
    if (T != CLB_IQ2_XXS) r.sc = __ldg(reinterpret_cast<const uint2*>(m.sc + ((size_t)b * n + row) * 8));
    if (T != CLB_IQ1_M) r.d = __ldg(m.d + (size_t)b * n + row);
}

__device__ __forceinline__ uint32_t rw(const RowRaw& r, int w) {  // body word w (static after unrolling)
    const uint4 v = w < 4 ? r.b0 : w < 8 ? r.b1 : w < 12 ? r.b2 : r.b3;
    const int s = w & 3;
    return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

template <int T>
__device__ __forceinline__ float raw_scale(const RowRaw& r) {
    if (T != CLB_IQ1_M) return __half2float(__ushort_as_half(r.d));
    const uint32_t w01 = r.sc.x, w23 = r.sc.y;
    const uint32_t h = ((w01 & 0xffffu) >> 12) | ((w01 >> 24) & 0xf0u) | (((w23 & 0xffffu) >> 4) & 0xf00u) |
                       ((w23 >> 16) & 0xf000u);
    return __half2float(__ushort_as_half((uint16_t)h));
}

// Lane integers of one block. q: the block's 256 activation int8 in shared memory (16 B
// aligned). Tables sit at offset 0 of the dynamic shared memory. lb = lane*4.
template <int T>
__device__ __forceinline__ void block_lanes(const RowRaw& r, const int8_t* q, uint32_t lb, int I[8], int D[8]) {
#pragma unroll
    for (int L = 0; L < 8; ++L) I[L] = D[L] = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 qa = *reinterpret_cast<const uint4*>(q + 32 * c);
        const uint4 qb = *reinterpret_cast<const uint4*>(q + 32 * c + 16);
        const uint32_t qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        if (T == CLB_IQ2_XXS) {
            // chunk = [4 grid bytes][4 sign bytes, bit 7 of byte j = bit j of the sub-scale]
            const uint32_t gw = rw(r, 2 * c), sw = rw(r, 2 * c + 1);
            const int scale = (int)((((sw & 0x80808080u) | 0x08000000u) * 0x00204081u) >> 27);  // 2s+1
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t sel_j = 0x5504u | ((uint32_t)j << 4);
                const uint32_t ga = prmt2(gw, lb, sel_j);  // grid byte * 256 + lane*4
                const uint32_t sa = prmt2(sw, lb, sel_j);  // sign byte * 256 + lane*4
                const uint32_t sel = (tab32(kRowTabXXS + ga) | tab32(kRowTabXXS + 128 + sa));
                const uint32_t lo = prmt_sel(kPos2, kNeg2, sel), hi = prmt_sel(kPos2, kNeg2, sel >> 16);
                I[2 * j] += scale * dp4a_s(lo, qv[2 * j]);
                I[2 * j + 1] += scale * dp4a_s(hi, qv[2 * j + 1]);
            }
        } else if (T == CLB_IQ2_XS) {
            const uint32_t scb = ((c < 4 ? r.sc.x : r.sc.y) >> (8 * (c & 3))) & 0xffu;
            const int s_lo = (int)((scb & 15u) << 1) | 1, s_hi = (int)((scb >> 4) << 1) | 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t w = rw(r, 2 * c + (j >> 1));
                const uint32_t code = (j & 1) ? (w >> 16) : (w & 0xffffu);
                const uint32_t ga = (code & 511u) * 64u + (lb & 60u);
                const uint32_t sa = (code >> 9) * 256u + 128u + lb;
                const uint32_t sel = tab32(kRowTabXS + ga) | tab32(kRowTabXXS + sa);
                const uint32_t lo = prmt_sel(kPos2, kNeg2, sel), hi = prmt_sel(kPos2, kNeg2, sel >> 16);
                const int s = j < 2 ? s_lo : s_hi;
                I[2 * j] += s * dp4a_s(lo, qv[2 * j]);
                I[2 * j + 1] += s * dp4a_s(hi, qv[2 * j + 1]);
            }
        } else {
            const uint32_t qsw = rw(r, c);
            const uint32_t qh16 = (rw(r, 8 + (c >> 1)) >> (16 * (c & 1))) & 0xffffu;
            const uint32_t scw = ((c < 4 ? r.sc.x : r.sc.y) >> (16 * ((c >> 1) & 1))) & 0xffffu;
            const int s_lo = (int)(((scw >> (6 * (c & 1))) & 7u) << 1) | 1;
            const int s_hi = (int)(((scw >> (6 * (c & 1) + 3)) & 7u) << 1) | 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t nib = (qh16 >> (4 * j)) & 15u;
                const uint32_t idx = ((qsw >> (8 * j)) & 0xffu) | ((nib & 7u) << 8);
                const uint32_t sel = tab32(kRowTabIQ1 + idx * 16u + (lb & 12u));
                const uint32_t lo = prmt_sel(kVal1, 0u, sel), hi = prmt_sel(kVal1, 0u, sel >> 16);
                const int s = j < 2 ? s_lo : s_hi;
                I[2 * j] += s * dp4a_s(lo, qv[2 * j]);
                I[2 * j + 1] += s * dp4a_s(hi, qv[2 * j + 1]);
                const int sd = (nib & 8u) ? -s : s;
                D[2 * j] += sd * __dp4a((int)qv[2 * j], 0x01010101, 0);
                D[2 * j + 1] += sd * __dp4a((int)qv[2 * j + 1], 0x01010101, 0);
            }
        }
    }
}

// Fast-math form of block_lanes: the same exact integers, summed over the 8 lanes before
// the sub-scale is applied (the scale is per chunk for IQ2_XXS, per chunk half for
// IQ2_XS / IQ1_M), so a block yields one main integer M and, for IQ1_M, one delta
// integer D. M = sum over lanes of the reference's I_L, D = sum of its delta lanes.
template <int T>
__device__ __forceinline__ void block_sum(const RowRaw& r, const int8_t* q, uint32_t lb, int& M, int& D) {
    M = 0;
    D = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 qa = *reinterpret_cast<const uint4*>(q + 32 * c);
        const uint4 qb = *reinterpret_cast<const uint4*>(q + 32 * c + 16);
        const uint32_t qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        if (T == CLB_IQ2_XXS) {
            // all four table lookups of the chunk first, then the decode (more loads in flight)
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
            M += scale * a;
        } else if (T == CLB_IQ2_XS) {
            const uint32_t scb = ((c < 4 ? r.sc.x : r.sc.y) >> (8 * (c & 3))) & 0xffu;
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
            M += s_lo * alo + s_hi * ahi;
        } else {
            const uint32_t qsw = rw(r, c);
            const uint32_t qh16 = (rw(r, 8 + (c >> 1)) >> (16 * (c & 1))) & 0xffffu;
            const uint32_t scw = ((c < 4 ? r.sc.x : r.sc.y) >> (16 * ((c >> 1) & 1))) & 0xffffu;
            const int s_lo = (int)(((scw >> (6 * (c & 1))) & 7u) << 1) | 1;
            const int s_hi = (int)(((scw >> (6 * (c & 1) + 3)) & 7u) << 1) | 1;
            int alo = 0, ahi = 0, dlo = 0, dhi = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t nib = (qh16 >> (4 * j)) & 15u;
                const uint32_t idx = ((qsw >> (8 * j)) & 0xffu) | ((nib & 7u) << 8);
                const uint32_t sel = tab32(kRowTabIQ1 + idx * 16u + (lb & 12u));
                int& a = j < 2 ? alo : ahi;
                a = __dp4a((int)prmt_sel(kVal1, 0u, sel), (int)qv[2 * j], a);
                a = __dp4a((int)prmt_sel(kVal1, 0u, sel >> 16), (int)qv[2 * j + 1], a);
                // delta: +-1 per group times the group's 8 activations
                const int qs8 = __dp4a((int)qv[2 * j], 0x01010101, __dp4a((int)qv[2 * j + 1], 0x01010101, 0));
                int& dd = j < 2 ? dlo : dhi;
                dd += (nib & 8u) ? -qs8 : qs8;
            }
            M += s_lo * alo + s_hi * ahi;
            D += s_lo * dlo + s_hi * dhi;
        }
    }
}

// Final row value from the 8 lane chains (q8k_core.hpp:86-91).
__device__ __forceinline__ float hsum8_rn(const float* v) {
    return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[2], v[6])),
                     __fadd_rn(__fadd_rn(v[1], v[5]), __fadd_rn(v[3], v[7])));
}

}  // namespace clb
