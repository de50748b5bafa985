// Host-side declarations of the sm_100a kernels (clb_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "clb_types.h"

namespace clb {

constexpr int kTabXXS = 0;
constexpr int kTabXS = 256;
constexpr int kTabIQ1 = 768;
constexpr int kTabSign = 2816;
constexpr int kTableWords = 2944;     // 256 + 512 + 2048 + 128 nibble selectors
constexpr int kQ8KBlockBytes = 292;   // crosslane q8k::Block (q8k_core.hpp:13-14)
constexpr int kMaxExperts = 1024;     // per layer, for device routing
constexpr int kMaxPicks = 16;         // hipex::max_jobs (hip_experts.hpp:8)

// Device descriptor of one resident expert: gate (w1), up (w3), down (w2).
struct ExpertDesc {
    PackedMat gate, up, down;
};

void host_tables(uint32_t* out /* kTableWords */);
cudaError_t upload_tables(cudaStream_t stream);
cudaError_t tables_device_ptr(const uint32_t** out);
cudaError_t set_smem_limits();
size_t mv_smem(int k);
size_t gateup_smem(int dim);
size_t down_smem(int npick, int ff);

cudaError_t launch_quant(const float* x, int nblocks, int8_t* qs, float* d, cudaStream_t s);
cudaError_t launch_quant_blocks(const float* x, int nblocks, void* out, cudaStream_t s);
cudaError_t launch_norm_quant(const float* h, int dim, int8_t* qs, float* d, float* xnorm, cudaStream_t s);
cudaError_t launch_mv(const PackedMat& m, const void* q, float* y, cudaStream_t s);
cudaError_t launch_activate(const float* g, const float* u, float* h, int n, float limit, cudaStream_t s);
cudaError_t launch_gateup(const ExpertDesc* experts, const int* ids, int npick, const int8_t* xqs, const float* xd,
                          int dim, int ff, float limit, float* h, int* err, cudaStream_t s);
cudaError_t launch_down_combine(const ExpertDesc* experts, const int* ids, const float* w, int npick,
                                const int8_t* hqs, const float* hd, int dim, int ff, const float* shared,
                                const float* resid, float* out, float* y_rows, int* err, cudaStream_t s);
cudaError_t launch_route_sigmoid(const float* logits, int n, int k, int tokens, int* ids, float* w, cudaStream_t s);
// logits [tokens][n] = gate_w [n][dim] . x [tokens][dim] (fp32, fixed order); dim % 4 == 0.
cudaError_t launch_router_gemv(const float* gate_w, const float* x, int n, int dim, int tokens, float* logits,
                               cudaStream_t s);
// route_cpu (mode B) on the device; n <= 1024; *err = 1 on a non-finite score.
cudaError_t launch_route_b(const float* logits, const float* bias, int n, int k, int tokens, float scale, int* ids,
                           float* w, int* err, cudaStream_t s);
cudaError_t launch_synth_fill(uint8_t* packed, const PackedLayout& l, int type, int n, int k, uint64_t seed,
                              uint32_t layer, uint32_t expert, uint32_t role, const uint16_t* scales, cudaStream_t s);
cudaError_t launch_pack(const uint8_t* aos, uint8_t* packed, const PackedLayout& l, int type, int n, int k, int* bad,
                        cudaStream_t s);

// v2 (row-per-thread decode, persistent CTAs, fused SwiGLU+Q8_K(h) and combine)
cudaError_t set_v2_smem_limits();
size_t gateup2_smem(int dim, int warps);
size_t down2_smem(int npick, int ff);
cudaError_t launch_gateup2(const ExpertDesc* experts, const int* ids, int npick, const int8_t* xqs, const float* xd,
                           int dim, int ff, float limit, float* gu, int8_t* hqs, float* hd, int* counters, int* err,
                           bool fast, cudaStream_t s);
cudaError_t launch_down2(const ExpertDesc* experts, const int* ids, const float* w, int npick, const int8_t* hqs,
                         const float* hd, int dim, int ff, const float* shared, const float* resid, float* out,
                         float* yrows, int* counters, int* err, bool fast, cudaStream_t s);
cudaError_t launch_mv2(const PackedMat& m, const void* q, float* y, cudaStream_t s);

// batched prefill through one layer (clb_prefill.cu): grouped tcgen05 GEMMs over IQ2_XXS experts.
// phase_mask: 1 group + quantise x, 2 gate/up GEMM, 4 SwiGLU + quantise h, 8 down GEMM, 16 combine.
size_t prefill_workspace_bytes(int T, int k, int dim, int ff, int E);
bool prefill_shape_supported(int dim, int ff);
// norm_x: x <- RMSNorm(x) (the stack's fixed-order pre-norm) before Q8_K. Only picks of
// experts [e_begin, e_end) are computed (e_end < 0: all); with a partial range the expert
// rows of the other picks are zero. rows: caller-owned expert rows [T*k][dim] (slot order)
// instead of the workspace's.
// type_mask: the weight types among the layer's experts (kTypeBit*; a single type selects
// a kernel that decodes that type alone; experts of a type outside the mask raise *err = 1).
constexpr int kTypeBitXXS = 1, kTypeBitXS = 2, kTypeBitIQ1M = 4, kTypeBitAll = 7;
cudaError_t launch_prefill(const ExpertDesc* desc, int E, const float* x, const int* ids, const float* w, int T, int k,
                           int dim, int ff, float limit, const float* resid, float* out, void* ws, int* err,
                           int phase_mask, cudaStream_t s, bool norm_x = false, int e_begin = 0, int e_end = -1,
                           float* rows = nullptr, int type_mask = kTypeBitAll);
// The routing slots of the batched stack's workspace: ids [T][k] and weights [T][k].
void stack_batch_routes(void* ws, int T, int k, int dim, int ff, int E, int** ids, float** w);
// T tokens through nl layers (desc [nl][E]): h <- h + layer(RMSNorm(h)) per layer, in place.
// Routes from ids_all / w_all ([nl][T][k]) or, when those are null, from logits ([nl][T][E]).
size_t stack_batch_workspace_bytes(int T, int k, int dim, int ff, int E);
cudaError_t launch_stack_batch(const ExpertDesc* desc, int E, int nl, const float* logits, const int* ids_all,
                               const float* w_all, float* h, int T, int k, int dim, int ff, float limit, void* ws,
                               int* err, cudaStream_t s, const int* type_masks = nullptr);

// persistent whole-stack kernel (clb_stack.cu)
constexpr int kMaxPeers = 8;  // GPUs of one node
constexpr unsigned kDefaultWaitLimit = 1u << 22;  // polls of a bounded device wait (a few seconds)
// Expert-ID sharding of the stack over `world` GPUs: this GPU holds experts [own_begin,
// own_end) of every layer and computes only those picks; the expert rows of every layer
// go to all GPUs through peer stores into double-buffered slots (yx: [2][k][dim] floats,
// then `flags`: one counter per source GPU). world == 1: no sharding.
// The fast order also keeps per-row-group completion counters there (rgcnt: [2][dim / 32],
// one set per layer parity), which every GPU increments.
struct StackShard {
    int world = 1, rank = 0, own_begin = 0, own_end = 0x7fffffff;
    unsigned epoch = 0;               // layers this bank has run through a stack kernel before this launch
    float* yx = nullptr;
    unsigned* flags = nullptr;
    unsigned* rgcnt = nullptr;
    float* peer_yx[kMaxPeers] = {};
    unsigned* peer_flags[kMaxPeers] = {};
    unsigned* peer_rgcnt[kMaxPeers] = {};
};
// Fast-order workspace of the persistent kernel: hbuf [2][dim] h between layers, ssbuf
// [2][dim / 32] its per-32-row-group sums of squares, blk: stack_block_words(nl_max, k, ff)
// counters of the SwiGLU output's 256-row blocks (8 row groups each), zeroed by
// launch_stack. The row-group counters live in StackShard::rgcnt.
struct StackWork {
    float* hbuf = nullptr;
    float* ssbuf = nullptr;
    unsigned* blk = nullptr;
};
size_t stack_block_words(int nl_max, int k, int ff);
size_t stack_smem(int dim, int ff, int k, bool fast);
bool stack_supported(int dim, int ff, int k, bool fast);
cudaError_t launch_stack(const ExpertDesc* desc, int E, int first, int nl, int k, const int* route_ids,
                         const float* route_w, const float* h_in, float* h_out, int dim, int ff, float limit, float* gu,
                         float* yrows, unsigned* bar, int* err, bool fast, const StackShard& shard, cudaStream_t s,
                         unsigned wait_limit, const StackWork& w);

}  // namespace clb
