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

// Block (row r, block b) of an n-row matrix with nb blocks per row.
CLB_PACK_FN void clb_pack_block(int t, int n, int nb, int r, int b, const uint8_t* src, uint8_t* packed,
                                PackedLayout l) {
    (void)nb;
    const int q_count = t == 29 ? 3 : 4;
    const int off0 = t == 29 ? 0 : 2;
    for (int q = 0; q < q_count; ++q)
        clb_copy_bytes(packed + l.body + (((size_t)b * q_count + q) * (size_t)n + (size_t)r) * 16, src + off0 + 16 * q,
                       16);
    if (t != 16) clb_copy_bytes(packed + l.sc + ((size_t)b * n + r) * 8, src + (t == 17 ? 66 : 48), 8);
    if (t != 29) clb_copy_bytes(packed + l.d + ((size_t)b * n + r) * 2, src, 2);
}

CLB_PACK_FN void clb_unpack_block(int t, int n, int nb, int r, int b, const uint8_t* packed, PackedLayout l,
                                  uint8_t* dst) {
    (void)nb;
    const int q_count = t == 29 ? 3 : 4;
    const int off0 = t == 29 ? 0 : 2;
    for (int q = 0; q < q_count; ++q)
        clb_copy_bytes(dst + off0 + 16 * q, packed + l.body + (((size_t)b * q_count + q) * (size_t)n + (size_t)r) * 16,
                       16);
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
