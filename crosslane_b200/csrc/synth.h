// Counter-based synthetic expert weights, identical on host (C/C++) and device (CUDA).
//
// Every ggml block of every matrix is a pure function of
//   (seed, layer, expert, role, block index) -> block bytes,
// so the 40-layer bank (~130 GB) is generated directly in HBM by a kernel and any
// single block can be regenerated on the host for the CPU oracle. Integer-only:
// the fp16 super-scales come from a 65,536-entry table of |N(0,1)|*0.01 fp16 bit
// patterns (built once on the host in float64, see clb_build_scale_table) indexed
// by 16 random bits, so no libm call differs between CPU and GPU.
//
// Block byte layouts follow ggml (crosslane engine/strata/sycl/moe/format.hpp:36-41,
// engine/strata/sycl/stage/wiring/q8k_core.hpp:48-60):
//   IQ2_XXS (type 16, 66 B): fp16 d @0, 8 x {4 grid bytes, u32 aux} @2
//   IQ2_XS  (type 17, 74 B): fp16 d @0, 32 x u16 code @2, 8 scale bytes @66
//   IQ1_M   (type 29, 56 B): 32 qs @0, 16 qh @32, 4 x u16 scales @48 whose top
//                            nibbles carry the fp16 super-scale
// Grid indices, sign bits and 4/3-bit sub-scales are uniform random bits.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define CLB_HD __host__ __device__ __forceinline__
#else
#define CLB_HD static inline
#endif

enum { CLB_IQ2_XXS = 16, CLB_IQ2_XS = 17, CLB_IQ1_M = 29 };
enum { CLB_ROLE_GATE = 0, CLB_ROLE_UP = 1, CLB_ROLE_DOWN = 2 };

CLB_HD int clb_block_bytes(int type) {
    return type == CLB_IQ2_XXS ? 66 : type == CLB_IQ2_XS ? 74 : type == CLB_IQ1_M ? 56 : 0;
}

// splitmix64 finaliser (Steele, Lea, Flood 2014).
CLB_HD uint64_t clb_mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

CLB_HD uint64_t clb_block_key(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t role,
                              uint64_t block) {
    uint64_t k = clb_mix64(seed ^ 0x6a09e667f3bcc909ull);
    k = clb_mix64(k ^ ((uint64_t)layer << 32 | expert));
    k = clb_mix64(k ^ ((uint64_t)role << 56) ^ block);
    return k;
}

// Quant type of (layer, expert) under a type policy:
//   policy 0: all IQ2_XXS; 1: experts [0,128) IQ2_XXS, [128,256) IQ2_XS, rest IQ1_M;
//   2: per (layer, expert) drawn from the seed; 3: all IQ2_XS; 4: all IQ1_M.
CLB_HD int clb_expert_type(int policy, uint64_t seed, uint32_t layer, uint32_t expert) {
    if (policy == 0) return CLB_IQ2_XXS;
    if (policy == 3) return CLB_IQ2_XS;
    if (policy == 4) return CLB_IQ1_M;
    if (policy == 1) return expert < 128 ? CLB_IQ2_XXS : expert < 256 ? CLB_IQ2_XS : CLB_IQ1_M;
    const uint64_t h = clb_mix64(clb_mix64(seed ^ 0xbb67ae8584caa73bull) ^ ((uint64_t)layer << 32 | expert));
    const uint32_t r = (uint32_t)(h >> 33) % 3u;
    return r == 0 ? CLB_IQ2_XXS : r == 1 ? CLB_IQ2_XS : CLB_IQ1_M;
}

// Writes the ggml (AoS) bytes of one block. `scales` is the 65,536-entry fp16 table.
CLB_HD void clb_synth_block(int type, uint64_t key, const uint16_t* scales, uint8_t* out) {
    const int bytes = clb_block_bytes(type);
    // 64-bit random words; byte i of the block body comes from word i/8.
    for (int w = 0; w * 8 < bytes; ++w) {
        const uint64_t r = clb_mix64(key + (uint64_t)(w + 1) * 0xd1b54a32d192ed03ull);
        for (int j = 0; j < 8 && w * 8 + j < bytes; ++j) out[w * 8 + j] = (uint8_t)(r >> (8 * j));
    }
    const uint16_t d = scales[(uint32_t)(clb_mix64(key ^ 0x510e527fade682d1ull) >> 48)];
    if (type == CLB_IQ1_M) {
        // fp16 super-scale nibbles go to the top nibble of each u16 scale word
        // (q8k_core.hpp:70-74): word j carries bits 4j..4j+3 of d.
        for (int j = 0; j < 4; ++j) {
            const uint16_t v = (uint16_t)((out[48 + 2 * j] | (out[49 + 2 * j] << 8)) & 0x0fff);
            const uint16_t s = (uint16_t)(v | (((d >> (4 * j)) & 15u) << 12));
            out[48 + 2 * j] = (uint8_t)s;
            out[49 + 2 * j] = (uint8_t)(s >> 8);
        }
    } else {
        out[0] = (uint8_t)d;
        out[1] = (uint8_t)(d >> 8);
    }
}
