// Block-level scatter/gather between ggml AoS blocks and the packed bank layout
// (see clb_types.h). Host and device share these functions; both directions are
// byte moves only, so pack followed by unpack is the identity.
#pragma once
#include <string.h>

#include "clb_types.h"

#if defined(__CUDACC__)
#define CLB_PACK_FN __host__ __device__ __forceinline__
#else
#define CLB_PACK_FN static inline
#endif

CLB_PACK_FN void clb_copy_bytes(uint8_t* dst, const uint8_t* src, int n) {
    for (int i = 0; i < n; ++i) dst[i] = src[i];
}

// IQ2_XXS chunk re-planing: the u32 `aux` (four 7-bit sign fields at bits 7j, 4-bit
// sub-scale at bits 28-31) becomes four sign bytes, byte j = sign field j | bit j of the
// sub-scale << 7, so a kernel can address a sign table with one byte permute.
CLB_PACK_FN uint32_t clb_aux_to_signbytes(uint32_t aux) {
    uint32_t out = 0;
    for (int j = 0; j < 4; ++j) out |= (((aux >> (7 * j)) & 127u) | (((aux >> (28 + j)) & 1u) << 7)) << (8 * j);
    return out;
}
CLB_PACK_FN uint32_t clb_signbytes_to_aux(uint32_t sb) {
    uint32_t aux = 0;
    for (int j = 0; j < 4; ++j) {
        const uint32_t b = (sb >> (8 * j)) & 255u;
        aux |= (b & 127u) << (7 * j);
        aux |= (b >> 7) << (28 + j);
    }
    return aux;
}
CLB_PACK_FN uint32_t clb_rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
CLB_PACK_FN void clb_wr32(uint8_t* p, uint32_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
    p[2] = (uint8_t)(v >> 16);
    p[3] = (uint8_t)(v >> 24);
}

// Block (row r, block b) of an n-row matrix with nb blocks per row.
CLB_PACK_FN void clb_pack_block(int t, int n, int nb, int r, int b, const uint8_t* src, uint8_t* packed,
                                PackedLayout l) {
    (void)nb;
    const int q_count = t == 29 ? 3 : 4;
    const int off0 = t == 29 ? 0 : 2;
    for (int q = 0; q < q_count; ++q) {
        uint8_t* dst = packed + l.body + (((size_t)b * q_count + q) * (size_t)n + (size_t)r) * 16;
        clb_copy_bytes(dst, src + off0 + 16 * q, 16);
        if (t == 16)
            for (int c = 0; c < 2; ++c) clb_wr32(dst + 8 * c + 4, clb_aux_to_signbytes(clb_rd32(dst + 8 * c + 4)));
    }
    if (t != 16) clb_copy_bytes(packed + l.sc + ((size_t)b * n + r) * 8, src + (t == 17 ? 66 : 48), 8);
    if (t != 29) clb_copy_bytes(packed + l.d + ((size_t)b * n + r) * 2, src, 2);
}

CLB_PACK_FN void clb_unpack_block(int t, int n, int nb, int r, int b, const uint8_t* packed, PackedLayout l,
                                  uint8_t* dst) {
    (void)nb;
    const int q_count = t == 29 ? 3 : 4;
    const int off0 = t == 29 ? 0 : 2;
    for (int q = 0; q < q_count; ++q) {
        uint8_t* o = dst + off0 + 16 * q;
        clb_copy_bytes(o, packed + l.body + (((size_t)b * q_count + q) * (size_t)n + (size_t)r) * 16, 16);
        if (t == 16)
            for (int c = 0; c < 2; ++c) clb_wr32(o + 8 * c + 4, clb_signbytes_to_aux(clb_rd32(o + 8 * c + 4)));
    }
    if (t != 16) clb_copy_bytes(dst + (t == 17 ? 66 : 48), packed + l.sc + ((size_t)b * n + r) * 8, 8);
    if (t != 29) clb_copy_bytes(dst, packed + l.d + ((size_t)b * n + r) * 2, 2);
}

// fp16 super-scale of an AoS block (IQ1_M: scattered over the scale words' top nibbles).
CLB_PACK_FN uint16_t clb_block_half(int t, const uint8_t* blk) {
    if (t != 29) return (uint16_t)(blk[0] | (blk[1] << 8));
    uint16_t w[4];
    for (int j = 0; j < 4; ++j) w[j] = (uint16_t)(blk[48 + 2 * j] | (blk[49 + 2 * j] << 8));
    return (uint16_t)((w[0] >> 12) | ((w[1] >> 8) & 0xf0) | ((w[2] >> 4) & 0xf00) | (w[3] & 0xf000));
}
