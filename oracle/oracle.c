// TEST INFRASTRUCTURE ONLY -- CPU oracle (see oracle.h for scope and citations).
// Build with -ffp-contract=off -fno-fast-math: every float operation below is one
// IEEE-754 binary32 operation, exactly as written (crosslane builds its Q8_K HIP twin
// with the same flags, engine/strata/sycl/stage/wiring/hip.cmake:88).
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../crosslane_b200/csrc/iq_tables.h"
#include "../crosslane_b200/csrc/scale_table.h"
#include "../crosslane_b200/csrc/synth.h"

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) { return (uint32_t)rd16(p) | ((uint32_t)rd16(p + 2) << 16); }

// ggml ksigns_iq2xs[i] = i | parity(i) << 7: the 8th sign makes the sign count even.
static unsigned ksign(unsigned v) {
    v &= 127u;
    return v | ((unsigned)__builtin_parity(v) << 7);
}

// q8k_core.hpp:16-23
float orc_half(uint16_t h) {
    const int e = (h >> 10) & 31;
    float v;
    if (!e) v = ldexpf((float)(h & 1023), -24);
    else if (e == 31) v = (h & 1023) ? NAN : INFINITY;
    else v = ldexpf((float)(1024 + (h & 1023)), e - 25);
    return (h & 32768) ? -v : v;
}

// q8k_core.hpp:25-29 (ggml nearest_int: round half to even through the 1.5*2^23 bias).
int orc_nearest(float x) {
    union { float f; uint32_t u; } v;
    v.f = x + 12582912.0f;
    return (int)(v.u & 0x007fffff) - 0x00400000;
}

// q8k_core.hpp:30-38. The signed element of largest magnitude (first one on ties)
// maps to -127; d = 1/is.
void orc_quant_block(const float* x, orc_block* y) {
    float mx = 0, am = 0;
    for (int j = 0; j < 256; ++j) {
        const float a = fabsf(x[j]);
        if (a > am) { am = a; mx = x[j]; }
    }
    if (am == 0) {
        y->d = 0;
        memset(y->qs, 0, sizeof y->qs);
        memset(y->bsums, 0, sizeof y->bsums);
        return;
    }
    const float is = -127.0f / mx;
    for (int j = 0; j < 256; ++j) {
        const int v = orc_nearest(is * x[j]);
        y->qs[j] = (int8_t)(v < 127 ? v : 127);
    }
    for (int j = 0; j < 16; ++j) {
        int s = 0;
        for (int z = 0; z < 16; ++z) s += y->qs[16 * j + z];
        y->bsums[j] = (int16_t)s;
    }
    y->d = 1.0f / is;
}

void orc_quantize(const float* x, int k, orc_block* out) {
    for (int b = 0; b < k / 256; ++b) orc_quant_block(x + 256 * b, out + b);
}

int orc_block_bytes(int t) { return t == 29 ? 56 : t == 17 ? 74 : t == 16 ? 66 : 0; }

// q8k_core.hpp:43-69. Lane L covers positions 4L..4L+3 of each of the 8 32-value
// chunks; `main` and `delta` are exact integers.
void orc_integer_lane(int t, const uint8_t* w, const orc_block* a, int lane, int* main_out,
                      int* delta_out) {
    int main = 0, dsum = 0;
    for (int c = 0; c < 8; ++c) {
        const int local = 4 * lane, group = local / 8;
        int sign = 0, scale = 0, delta = 0;
        uint64_t tab = 0;
        if (t == 29) {
            const uint8_t hi = w[32 + 2 * c + group / 2];
            const int grid = w[4 * c + group] | (((int)hi << (8 - 4 * (group % 2))) & 0x700);
            tab = clb_iq1s_grid[grid];
            delta = (hi & (group % 2 ? 128 : 8)) ? -1 : 1;
            const uint16_t sc = rd16(w + 48 + 2 * (c / 2));
            scale = 2 * ((sc >> (6 * (c % 2) + 3 * (local / 16))) & 7) + 1;
        } else if (t == 17) {
            const uint16_t q = rd16(w + 2 + 8 * c + 2 * group);
            tab = clb_iq2xs_grid[q & 511];
            sign = (int)ksign(q >> 9);
            scale = 2 * ((w[66 + c] >> (4 * (local / 16))) & 15) + 1;
        } else {
            const uint8_t* chunk = w + 2 + 8 * c;
            const uint32_t hi = rd32(chunk + 4);
            tab = clb_iq2xxs_grid[chunk[group]];
            sign = (int)ksign((hi >> (7 * group)) & 127);
            scale = 2 * (int)(hi >> 28) + 1;
        }
        for (int j = local % 8; j < local % 8 + 4; ++j) {
            const int q = a->qs[32 * c + 8 * group + j];
            const int code = t == 29 ? (int)(int8_t)(uint8_t)(tab >> (8 * j))
                                     : (int)(uint8_t)(tab >> (8 * j)) * ((sign & (1 << j)) ? -1 : 1);
            main += scale * code * q;
            if (t == 29) dsum += scale * delta * q;
        }
    }
    *main_out = main;
    *delta_out = dsum;
}

// q8k_core.hpp:70-74: IQ1_M's fp16 super-scale is scattered over the scale words' top nibbles.
float orc_block_scale(int t, const uint8_t* w) {
    if (t != 29) return orc_half(rd16(w));
    const uint16_t h = (uint16_t)((rd16(w + 48) >> 12) | ((rd16(w + 50) >> 8) & 0xf0) |
                                  ((rd16(w + 52) >> 4) & 0xf00) | (rd16(w + 54) & 0xf000));
    return orc_half(h);
}

// q8k_core.hpp:86
static float hsum8(const float* v) {
    return ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
}

// q8k_core.hpp:76-91: per lane, blocks in order, s = fmaf(half(w.d) * a.d, int, s).
float orc_dot(int t, const uint8_t* w, const orc_block* a, int nb) {
    float m[8], d[8];
    const int bb = orc_block_bytes(t);
    for (int l = 0; l < 8; ++l) {
        float sm = 0, sd = 0;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* p = w + (size_t)b * bb;
            int vm, vd;
            orc_integer_lane(t, p, a + b, l, &vm, &vd);
            const float dd = orc_block_scale(t, p) * a[b].d;
            sm = fmaf(dd, (float)vm, sm);
            if (t == 29) sd = fmaf(dd, (float)vd, sd);
        }
        m[l] = sm;
        d[l] = sd;
    }
    const float main = hsum8(m);
    return t == 29 ? main + 0.125f * hsum8(d) : 0.125f * main;
}

// q8k_core.hpp:92-95
float orc_swiglu(float g, float u, float limit) {
    if (limit > 0) {
        g = fminf(g, limit);
        u = fminf(fmaxf(u, -limit), limit);
    }
    return (g / (1.0f + expf(-g))) * u;
}

void orc_mv(int t, const uint8_t* w, const orc_block* q, float* y, int n, int k) {
    const int nb = k / 256;
    const size_t row = (size_t)nb * orc_block_bytes(t);
#pragma omp parallel for schedule(static, 64)
    for (int r = 0; r < n; ++r) y[r] = orc_dot(t, w + (size_t)r * row, q, nb);
}

static int all_finite(const float* v, int n) {
    for (int i = 0; i < n; ++i)
        if (!isfinite(v[i])) return 0;
    return 1;
}

// cpu_lane.cpp:137-175: Q8_K(x) -> gate, up rows -> SwiGLU -> Q8_K(h) -> down rows.
int orc_expert(int tg, const uint8_t* gate, int tu, const uint8_t* up, int td, const uint8_t* down,
               const float* x, int dim, int ff, float limit, float* h_out, float* y) {
    if (dim <= 0 || ff <= 0 || dim % 256 || ff % 256 || !all_finite(x, dim)) return -1;
    orc_block* qx = (orc_block*)malloc(sizeof(orc_block) * (size_t)(dim / 256));
    orc_block* qh = (orc_block*)malloc(sizeof(orc_block) * (size_t)(ff / 256));
    float* g = (float*)malloc(sizeof(float) * (size_t)ff * 3);
    float* u = g + ff;
    float* h = u + ff;
    orc_quantize(x, dim, qx);
    orc_mv(tg, gate, qx, g, ff, dim);
    orc_mv(tu, up, qx, u, ff, dim);
    for (int i = 0; i < ff; ++i) h[i] = orc_swiglu(g[i], u[i], limit);
    orc_quantize(h, ff, qh);
    orc_mv(td, down, qh, y, dim, ff);
    if (h_out) memcpy(h_out, h, sizeof(float) * (size_t)ff);
    free(qx);
    free(qh);
    free(g);
    return all_finite(y, dim) ? 0 : -1;
}

// runtime.cpp:184-187 (byte-identical SIMD twin other_combine.hpp:51-75).
int orc_combine(const int* ids, const float* w, int n, const float* rows, const float* shared,
                int dim, float* out) {
    int order[64];
    if (n < 0 || n > 64) return -1;
    for (int i = 0; i < n; ++i) order[i] = i;
    for (int i = 1; i < n; ++i)  // insertion sort by expert id (ids are unique)
        for (int j = i; j > 0 && ids[order[j - 1]] > ids[order[j]]; --j) {
            const int tmp = order[j];
            order[j] = order[j - 1];
            order[j - 1] = tmp;
        }
    for (int k = 0; k < dim; ++k) out[k] = 0;
    for (int o = 0; o < n; ++o) {
        const int i = order[o];
        for (int k = 0; k < dim; ++k) out[k] = fmaf(w[i], rows[(size_t)i * dim + k], out[k]);
    }
    if (shared)
        for (int k = 0; k < dim; ++k) out[k] += shared[k];
    return 0;
}

// Mode A. Selection is on the logits (sigmoid is strictly increasing), larger first,
// ties to the lower id; weights are sigmoid(l_i) normalised by their sum taken in
// selection order.
int orc_route_sigmoid(const float* logits, int n, int k, int* ids, float* w) {
    if (n <= 0 || k <= 0 || k > n || k > 64) return -1;
    unsigned char used[4096];
    if (n > 4096) return -1;
    memset(used, 0, (size_t)n);
    float s[64], sum = 0;
    for (int i = 0; i < k; ++i) {
        int best = -1;
        for (int e = 0; e < n; ++e)
            if (!used[e] && (best < 0 || logits[e] > logits[best])) best = e;
        used[best] = 1;
        ids[i] = best;
        s[i] = 1.0f / (1.0f + expf(-logits[best]));
        sum += s[i];
    }
    for (int i = 0; i < k; ++i) w[i] = s[i] / sum;
    return 0;
}

// Mode B, route.cpp:15-37 for one token.
int orc_route_sqrt_softplus(const float* logits, const float* bias, int n, int k, float scale,
                            int* ids, float* w) {
    if (n <= 0 || k <= 0 || k > n || n > 4096) return -1;
    float sc[4096], bs[4096];
    for (int e = 0; e < n; ++e) {
        const float l = logits[e];
        const float sp = l > 20.0f ? l : log1pf(expf(l));
        sc[e] = sqrtf(sp);
        bs[e] = sc[e] + bias[e];
        if (!isfinite(bs[e])) return -1;
    }
    float sum = 0;
    for (int i = 0; i < k; ++i) {
        int best = 0;
        for (int e = 1; e < n; ++e)
            if (bs[e] > bs[best]) best = e;
        ids[i] = best;
        sum += sc[best];
        bs[best] = -FLT_MAX;
    }
    for (int i = 0; i < k; ++i) w[i] = sc[ids[i]] / (sum + 1e-20f) * scale;
    return 0;
}

// core.hpp:13-57, IQ2_XXS / IQ2_XS / IQ1_M branches.
void orc_decode_sub(int t, const uint8_t* b, int ib, int q[32], float* d, int s[2]) {
    if (t == 16 || t == 17) {
        const uint8_t* p = b + 2 + 8 * ib;
        const unsigned aux = rd32(p + 4);
        for (int l = 0; l < 4; ++l) {
            const unsigned v = rd16(p + 2 * l);
            const uint64_t grid = t == 16 ? clb_iq2xxs_grid[p[l]] : clb_iq2xs_grid[v & 511];
            const unsigned sg = ksign(t == 16 ? aux >> (7 * l) : v >> 9);
            for (int j = 0; j < 8; ++j) {
                const int m = (int)((grid >> (8 * j)) & 255);
                q[8 * l + j] = ((sg >> j) & 1) ? -m : m;
            }
        }
        *d = orc_half(rd16(b)) * 0.125f;
        if (t == 16) {
            s[0] = s[1] = 2 * (int)(aux >> 28) + 1;
        } else {
            s[0] = 2 * (int)(b[66 + ib] & 15) + 1;
            s[1] = 2 * (int)(b[66 + ib] >> 4) + 1;
        }
    } else {
        const unsigned sc = rd16(b + 48 + 2 * (ib >> 1));
        *d = orc_block_scale(29, b) * 0.125f;
        s[0] = 2 * (int)((sc >> (6 * (ib & 1))) & 7) + 1;
        s[1] = 2 * (int)((sc >> (6 * (ib & 1) + 3)) & 7) + 1;
        for (int l = 0; l < 4; ++l) {
            const unsigned h = b[32 + 2 * ib + l / 2];
            const unsigned idx = b[4 * ib + l] | ((h << ((l & 1) ? 4 : 8)) & 0x700);
            const uint64_t grid = clb_iq1s_grid[idx];
            const int delta = (h & ((l & 1) ? 128 : 8)) ? -1 : 1;
            for (int j = 0; j < 8; ++j) q[8 * l + j] = 8 * (int)(int8_t)(uint8_t)(grid >> (8 * j)) + delta;
        }
    }
}

void orc_scale_table(uint16_t* table) { clb_build_scale_table(table); }

int orc_expert_type(int policy, uint64_t seed, uint32_t layer, uint32_t expert) {
    return clb_expert_type(policy, seed, layer, expert);
}

void orc_synth_matrix(int t, uint64_t seed, uint32_t layer, uint32_t expert, uint32_t role, int n,
                      int k, const uint16_t* table, uint8_t* out) {
    const size_t blocks = (size_t)n * (size_t)(k / 256);
    const int bb = orc_block_bytes(t);
#pragma omp parallel for schedule(static, 1024)
    for (long long i = 0; i < (long long)blocks; ++i)
        clb_synth_block(t, clb_block_key(seed, layer, expert, role, (uint64_t)i), table,
                        out + (size_t)i * bb);
}

int orc_layer_synth(int policy, uint64_t seed, uint32_t layer, const int* ids, const float* w,
                    int npick, const float* x, const float* shared, int dim, int ff, float limit,
                    const uint16_t* table, int threads, float* y) {
    (void)threads;
    if (npick <= 0 || npick > 64) return -1;
    float* rows = (float*)malloc(sizeof(float) * (size_t)dim * (size_t)npick);
    int rc = 0;
    for (int i = 0; i < npick && !rc; ++i) {
        const int t = clb_expert_type(policy, seed, layer, (uint32_t)ids[i]);
        const size_t gu_bytes = (size_t)ff * (size_t)(dim / 256) * (size_t)orc_block_bytes(t);
        const size_t dn_bytes = (size_t)dim * (size_t)(ff / 256) * (size_t)orc_block_bytes(t);
        uint8_t* g = (uint8_t*)malloc(gu_bytes * 2 + dn_bytes);
        uint8_t* u = g + gu_bytes;
        uint8_t* d = u + gu_bytes;
        orc_synth_matrix(t, seed, layer, (uint32_t)ids[i], CLB_ROLE_GATE, ff, dim, table, g);
        orc_synth_matrix(t, seed, layer, (uint32_t)ids[i], CLB_ROLE_UP, ff, dim, table, u);
        orc_synth_matrix(t, seed, layer, (uint32_t)ids[i], CLB_ROLE_DOWN, dim, ff, table, d);
        rc = orc_expert(t, g, t, u, t, d, x, dim, ff, limit, NULL, rows + (size_t)i * dim);
        free(g);
    }
    if (!rc) rc = orc_combine(ids, w, npick, rows, shared, dim, y);
    free(rows);
    return rc;
}

void orc_rmsnorm(const float* h, int dim, float* out) {
    double part[1024];
    for (int t = 0; t < 1024; ++t) {
        double s = 0.0;
        for (int i = t; i < dim; i += 1024) {
            const double v = (double)h[i];
            s = s + v * v;
        }
        part[t] = s;
    }
    for (int stride = 512; stride > 0; stride >>= 1)
        for (int t = 0; t < stride; ++t) part[t] = part[t] + part[t + stride];
    const double mean = part[0] / (double)dim;
    const float sc = (float)(1.0 / sqrt(mean + 1e-6));
    for (int i = 0; i < dim; ++i) out[i] = h[i] * sc;
}
