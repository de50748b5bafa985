// Types shared by host C++ and device code.
//
// Packed HBM layout of one quantized matrix ("bank layout"): lossless, the same
// number of payload bytes as the ggml blocks (crosslane's own SoA bank reorders
// likewise, engine/strata/warm/mmvq_layout.hpp:19-43), re-planed for sm_100a:
// 16-byte pieces of a block are stored row-contiguous, so the 8 rows of a warp's
// quad-group read one 128-byte line per 128-bit load.
//
//   n rows, k columns, nb = k/256 blocks per row; AoS block bytes B[0..bytes).
//   IQ2_XXS: body [nb][4][n][16] = B[2+16q .. 2+16q+16)   (8 chunks x {grid4, aux})
//            d    [nb][n] u16   = B[0..2)
//   IQ2_XS:  body [nb][4][n][16] = B[2+16q ..)             (8 chunks x 4 u16 codes)
//            sc   [nb][n][8]    = B[66..74)
//            d    [nb][n] u16   = B[0..2)
//   IQ1_M:   body [nb][3][n][16] = B[16q ..)               (qs 32 B, qh 16 B)
//            sc   [nb][n][8]    = B[48..56)                (scales + fp16 nibbles)
// Planes start at 256-byte aligned offsets of the matrix allocation.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "synth.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const uint8_t* body;
    const uint8_t* sc;
    const uint16_t* d;
    int type;
    int n;
    int k;
    int pad;
} PackedMat;

// Offsets of the three planes inside a packed matrix, and its total size.
typedef struct {
    size_t body, sc, d, total;
} PackedLayout;

static inline size_t clb_align256(size_t v) { return (v + 255u) & ~(size_t)255u; }

static inline int clb_type_supported(int t) { return t == 16 || t == 17 || t == 29; }

static inline PackedLayout clb_packed_layout(int t, int n, int k) {
    PackedLayout l = {0, 0, 0, 0};
    const size_t blocks = (size_t)n * (size_t)(k / 256);
    const size_t body = blocks * (t == 29 ? 48u : 64u);
    l.body = 0;
    l.sc = clb_align256(body);
    const size_t sc = t == 16 ? 0 : blocks * 8u;
    l.d = clb_align256(l.sc + sc);
    const size_t d = t == 29 ? 0 : blocks * 2u;
    l.total = clb_align256(l.d + d);
    return l;
}

#ifdef __cplusplus
}
#endif
