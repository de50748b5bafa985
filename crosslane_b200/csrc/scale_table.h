// Host-only: the 65,536-entry table of fp16 super-scales |N(0,1)| * 0.01.
//
// Entry i is the (i + 0.5) / 65536 quantile of the half-normal distribution,
// z = sqrt(2) * erfinv(u), scaled by 0.01 and rounded to fp16 (round to nearest
// even, subnormals included). erfinv is found by bisection on libm's double erf,
// which is monotone, so the table is a deterministic function of erf alone.
// Indexing it with 16 uniform random bits draws |N(0,1)|*0.01 in fp16.
#pragma once
#include <math.h>
#include <stdint.h>

static inline uint16_t clb_f64_to_f16_rne(double v) {
    uint16_t sign = 0;
    if (v < 0) { sign = 0x8000; v = -v; }
    if (v == 0) return sign;
    if (v >= 65520.0) return (uint16_t)(sign | 0x7c00);
    if (v < 6.103515625e-05) {  // below 2^-14: subnormal, unit 2^-24 (exact scaling)
        const double m = rint(v * 16777216.0);
        return (uint16_t)(sign | (uint16_t)m);  // m == 1024 is the smallest normal
    }
    int e = 0;
    const double f = frexp(v, &e);          // v = f * 2^e, f in [0.5, 1)
    double m = rint(f * 2048.0);            // 11 significant bits, exact scaling
    if (m == 2048.0) { m = 1024.0; ++e; }
    const int eh = e - 1 + 15;
    if (eh >= 31) return (uint16_t)(sign | 0x7c00);
    return (uint16_t)(sign | (uint16_t)(eh << 10) | (uint16_t)((int)m - 1024));
}

static inline void clb_build_scale_table(uint16_t* table /* [65536] */) {
    for (int i = 0; i < 65536; ++i) {
        const double u = ((double)i + 0.5) / 65536.0;
        double lo = 0.0, hi = 8.0;
        for (int it = 0; it < 80; ++it) {
            const double mid = 0.5 * (lo + hi);
            if (erf(mid) < u) lo = mid; else hi = mid;
        }
        const double z = 1.4142135623730951 * 0.5 * (lo + hi);
        table[i] = clb_f64_to_f16_rne(z * 0.01);
    }
}
