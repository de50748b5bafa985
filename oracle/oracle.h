// TEST INFRASTRUCTURE ONLY -- the CPU oracle for crosslane's routed-expert decode path.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
// library, and only as the checker. The product (crosslane_b200) never links it.
//
// A plain-C restatement of crosslane's CPU expert-lane arithmetic:
//   * Q8_K activation quantisation, lane-structured exact-integer IQ dots, pairwise
//     hsum and SwiGLU: engine/strata/sycl/stage/wiring/q8k_core.hpp:13-95 (itself
//     crosslane's restatement of ggml 6b9ba4f2's x86 AVX2 Q8_K IQ dots);
//   * an independent per-32 decoder used to cross-check the integer sub-dots:
//     engine/strata/sycl/moe/core.hpp:13-57;
//   * one expert FFN (quant x, gate/up rows, SwiGLU, quant h, down rows):
//     engine/strata/sycl/moe/cpu_lane.cpp:137-175;
//   * the fixed-order combine: engine/strata/warm/runtime.cpp:184-187;
//   * routing mode B (sqrt-softplus + bias): engine/strata/sycl/route/route.cpp:15-37,
//     and the benchmark's mode A (top-k by sigmoid score, renormalised).
// Parity pin: tests compare this oracle with the reference's own q8k_core.hpp compiled
// from the crosslane sources into oracle/_ref (see oracle/Makefile) and with committed
// golden vectors produced from that build (tests/golden/).
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Q8_K block (q8k_core.hpp:13-14): fp32 d, 256 int8 qs, 16 int16 bsums; 292 bytes.
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} orc_block;

float orc_half(uint16_t h);
int orc_nearest(float x);
void orc_quant_block(const float* x, orc_block* y);
void orc_quantize(const float* x, int k, orc_block* out);
int orc_block_bytes(int type);
// Integer sums of lane `lane` (0..7) over one 256-value block (q8k_core.hpp:43-69).
void orc_integer_lane(int type, const uint8_t* w, const orc_block* a, int lane, int* main, int* delta);
float orc_block_scale(int type, const uint8_t* w);
// Row dot of a ggml (AoS) row of nb blocks against nb Q8_K blocks (q8k_core.hpp:76-91).
float orc_dot(int type, const uint8_t* w, const orc_block* a, int nb);
float orc_swiglu(float g, float u, float limit);
// y[n] = W[n, k] . Q8_K(x): rows of a ggml AoS matrix.
void orc_mv(int type, const uint8_t* w, const orc_block* q, float* y, int n, int k);
// One expert: gate/up [ff, dim], down [dim, ff], all ggml AoS. Writes h[ff] (may be
// NULL) and y[dim]. Returns 0, or -1 on a non-finite input/output.
int orc_expert(int tg, const uint8_t* gate, int tu, const uint8_t* up, int td, const uint8_t* down,
               const float* x, int dim, int ff, float limit, float* h, float* y);
// out[k] = fma over picks in ascending id of (w_i, rows[i][k]), then + shared[k].
int orc_combine(const int* ids, const float* w, int n, const float* rows /* [n][dim] */,
                const float* shared /* may be NULL: zeros */, int dim, float* out);
// Mode A: top-k by sigmoid(logit), ties by lower id; w = s / sum(s).
int orc_route_sigmoid(const float* logits, int n, int k, int* ids, float* w);
// Mode B: route.cpp:15-37 (sqrt(softplus(l)) + bias, top-k, sc / (sum + 1e-20) * scale).
int orc_route_sqrt_softplus(const float* logits, const float* bias, int n, int k, float scale,
                            int* ids, float* w);

// Independent per-32 decode of sub-block ib of one block (core.hpp:13-57):
// q[32] signed codes, d = half * 0.125, s[2] = odd sub-scales of the two 16-halves,
// delta (IQ1_M: the 8*(q-1)+delta form folds it in; q holds 8*code+delta there).
void orc_decode_sub(int type, const uint8_t* block, int ib, int q[32], float* d, int s[2]);

// Synthetic inputs (crosslane_b200/csrc/synth.h), exposed for tests.
void orc_scale_table(uint16_t* table /* [65536] */);
void orc_synth_matrix(int type, uint64_t seed, uint32_t layer, uint32_t expert, uint32_t role,
                      int n, int k, const uint16_t* table, uint8_t* out /* n*k/256 blocks, AoS */);
int orc_expert_type(int policy, uint64_t seed, uint32_t layer, uint32_t expert);

// One routed MoE layer on synthetic weights: expert weights generated on demand.
// Writes y[dim] = combine(picks) (+ shared if non-NULL). Uses `threads` host threads
// over the row dimension (0 = all online CPUs).
int orc_layer_synth(int policy, uint64_t seed, uint32_t layer, const int* ids, const float* w,
                    int npick, const float* x, const float* shared, int dim, int ff, float limit,
                    const uint16_t* table, int threads, float* y);

// Stack pre-norm: out = h * (float)(1 / sqrt(mean(h^2) + 1e-6)), fp64 sum of squares in
// the order of crosslane_b200's k_norm_quant (1024 strided lanes, then a binary tree).
void orc_rmsnorm(const float* h, int dim, float* out);

#ifdef __cplusplus
}
#endif
