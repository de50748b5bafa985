/* crosslane_b200 -- B200-native (sm_100a) routed-expert decode lane for crosslane.
 *
 * Drop-in C ABI of the CUDA expert lane. Plain pointers and sizes only; every
 * function returns 0 on success or a CLB_E_* code. Functions taking a
 * `clb_error_v1*` also write a message there (may be NULL); this mirrors crosslane's
 * `strata_stage_error_v1 {int32 code; char message[512]}` convention
 * (engine/strata/sycl/stage/abi.h:19-22).
 *
 * Device-pointer primitives take a caller-owned CUDA stream (`void*` = cudaStream_t,
 * NULL = legacy default stream) and never allocate, like crosslane's Q8_K HIP API
 * (engine/strata/sycl/stage/wiring/hip_q8k.hpp:6-10).
 *
 * Quant types use ggml ids: 16 = IQ2_XXS, 17 = IQ2_XS, 29 = IQ1_M.
 * Matrices are [n rows, k columns], k % 256 == 0. Expert roles: 0 = gate (w1),
 * 1 = up (w3), 2 = down (w2), as in layers.L.ffn.experts.E.{w1,w3,w2}.weight
 * (engine/strata/sycl/stage/wiring/cpu_lane.hpp:36).
 */
#ifndef CROSSLANE_B200_H
#define CROSSLANE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLB_ABI_VERSION 1

enum {
    CLB_OK = 0,
    CLB_E_INVALID = 1,     /* bad argument, shape, type or duplicate id */
    CLB_E_CUDA = 2,        /* a CUDA call failed */
    CLB_E_NOMEM = 3,       /* device or host allocation failed */
    CLB_E_STATE = 4,       /* object unusable (earlier failure poisons it) */
    CLB_E_NONFINITE = 5,   /* non-finite input or output */
    CLB_E_UNSUPPORTED = 6, /* quant type or geometry without a kernel */
    CLB_E_LANE = 7,        /* another lane of warm_execute failed */
    CLB_E_NCCL = 8         /* a collective failed */
};

typedef struct clb_error_v1 {
    int32_t code;
    char message[512];
} clb_error_v1;

/* ABI version; lets a dlopen()ing host refuse a mismatched library. */
int32_t clb_abi_version(void);

/* ---- Q8_K activation primitives (device pointers, caller stream, no allocation) ---- */

/* Bytes of the Q8_K activation of a k-vector: k/256 crosslane q8k::Block structs
 * (292 B: fp32 d, int8 qs[256], int16 bsums[16]); 0 if k % 256 != 0.
 * Replaces q8k::activation_bytes (engine/strata/sycl/stage/wiring/hip_q8k.hpp:8). */
size_t clb_q8k_activation_bytes(int32_t k);

/* q[k/256 blocks] = Q8_K(x[k]). Replaces q8k::quantize (hip_q8k.hpp:9). */
int32_t clb_q8k_quantize(const float* x, void* q, int32_t k, void* stream);

/* y[n] = W . q for a matrix in the packed bank layout (clb_pack).
 * Bit-identical to crosslane's q8k::dot per row (q8k_core.hpp:76-91).
 * Replaces q8k::mv (hip_q8k.hpp:10). */
int32_t clb_q8k_mv(int32_t type, const void* w_packed, const void* q, float* y, int32_t n, int32_t k, void* stream);

/* h[i] = swiglu(g[i], u[i]) with clamp `limit` (0 = none).
 * Replaces q8k::activate (hip_q8k.hpp:11). */
int32_t clb_q8k_activate(const float* g, const float* u, float* h, int32_t n, float limit, void* stream);

/* Diagnostics: copies the decode kernels' nibble-selector tables (2944 u32: IQ2_XXS
 * grid 256, IQ2_XS grid 512, IQ1 grid 2048, sign masks 128) to `out`; returns the
 * number of words, or 0 if `words` is too small. No counterpart in crosslane; lets
 * host tests prove the byte-permute decode against the ggml codebooks. */
size_t clb_decode_tables(uint32_t* out, size_t words);

/* ---- packed bank layout (host memory) ---- */

/* Size of one matrix in the packed bank layout (>= the ggml bytes, planes 256 B
 * aligned); 0 for an unsupported type or geometry.
 * Replaces mmvq::extent (engine/strata/warm/mmvq_layout.hpp:12-15). */
size_t clb_packed_bytes(int32_t type, int32_t n, int32_t k);

/* ggml AoS bytes -> packed layout; rejects a non-finite fp16 super-scale.
 * Replaces mmvq::reorder (mmvq_layout.hpp:19-32). */
int32_t clb_pack(int32_t type, int32_t n, int32_t k, const void* ggml, size_t ggml_bytes, void* packed,
                 size_t packed_bytes);

/* packed layout -> ggml AoS bytes (exact inverse of clb_pack).
 * Replaces mmvq::restore (mmvq_layout.hpp:33-42). */
int32_t clb_unpack(int32_t type, int32_t n, int32_t k, const void* packed, size_t packed_bytes, void* ggml,
                   size_t ggml_bytes);

/* ---- expert bank: the resident CUDA lane ---- */

typedef struct clb_bank clb_bank;

typedef struct clb_bank_config_v1 {
    int32_t device;        /* CUDA ordinal */
    int32_t n_layers;      /* layers the bank spans (ids 0..n_layers-1) */
    int32_t n_experts;     /* routed experts per layer */
    int32_t dim;           /* hidden size (gate/up k, down n) */
    int32_t ff;            /* expert intermediate size */
    int32_t max_picks;     /* routed experts per token and layer, <= 16 */
    float limit;           /* SwiGLU clamp, 0 = none (crosslane's model uses 10) */
    int32_t expert_begin;  /* this bank owns experts [expert_begin, expert_end) of */
    int32_t expert_end;    /*   every layer (expert-ID sharding); 0,0 = all */
    int32_t flags;         /* CLB_BANK_* bits below; other bits must be 0 */
    int32_t reserved[6];
} clb_bank_config_v1;

/* Summation order of the routed-expert row dots.
 * Default (flag clear): each row's 256-value blocks are split into contiguous segments,
 *   one per thread, whose fp32 partials are added in a fixed tree. Results are
 *   run-to-run bit-identical and agree with the reference CPU lane to fp32
 *   reassociation (well inside 1e-3 relative L2).
 * CLB_BANK_EXACT_ORDER: the reference's own order (8 lane chains, per-block fma in block
 *   order, q8k_core.hpp:43-91), bit-identical to the CPU lane, at lower throughput. */
#define CLB_BANK_EXACT_ORDER 1
/* Stack decode (clb_stack_decode*) launches three kernels per layer instead of one
 * persistent kernel holding one CTA on every SM (for processes that share the GPU). */
#define CLB_BANK_PER_LAYER_KERNELS 2
/* Device timing of the synchronous host entry points (clb_layer_execute, clb_warm_execute,
 * clb_stack_decode, clb_prefill_layer, clb_stack_batch): CUDA events on the bank stream
 * around each call's copies and kernels; one JSON line per call on stderr,
 *   {"schema":"clb-cuda-timing-v1","lane":"cuda","device":D,"call":"...","layer":L,
 *    "layers":N,"picks":P,"h2d_bytes":B,"d2h_bytes":B,"ns":T}
 * and the last span through clb_bank_last_timing. */
#define CLB_BANK_TIMING 4

/* The last span recorded under CLB_BANK_TIMING (zeros before the first). */
typedef struct clb_timing_v1 {
    uint64_t ns;         /* device time from the first copy up to the last copy back */
    uint64_t h2d_bytes;  /* host -> device bytes of the call */
    uint64_t d2h_bytes;  /* device -> host bytes of the call */
    int32_t layer;       /* first layer */
    int32_t layers;      /* layers the call ran */
    int32_t picks;       /* routed (token, expert) picks the call computed */
    int32_t reserved;
} clb_timing_v1;
int32_t clb_bank_last_timing(const clb_bank* bank, clb_timing_v1* out);

/* ---- the CUDA lane's keys of the stage config ----
 * crosslane's stage config is "key=value" lines, parsed strictly: '#' comments and empty
 * lines skipped, a line without '=', a duplicate key or an unknown key is an error
 * (engine/strata/sycl/stage/wiring/common.hpp:55-125). The CUDA lane's keys:
 *   warm_cuda_experts = off | layer-batch-v1 | stack-v1   (default off)
 *       layer-batch-v1: the lane serves warm_execute's layer batches (per-layer kernels);
 *       stack-v1: the device-resident persistent stack kernel
 *   cuda_expert_math  = fast-v1 | cpu-q8k-v1              (default fast-v1)
 *       cpu-q8k-v1: the CPU lane's summation order, bit for bit (CLB_BANK_EXACT_ORDER)
 *   warm_cuda_bytes   = canonical decimal byte cap of the bank's payload (0 = none)
 *   cuda_devices      = a | a..b                          (default 0)
 *   warm_cuda_timing  = 0 | 1                             (CLB_BANK_TIMING)
 * A host whose own parser sees these keys forwards those lines here. cpu-q8k-v1 needs the
 * lane on; warm_cuda_bytes and cuda_devices need it on too. */
typedef struct clb_lane_config_v1 {
    int32_t experts;       /* 0 off, 1 layer-batch-v1, 2 stack-v1 */
    int32_t exact_math;    /* 1 for cpu-q8k-v1 */
    uint64_t bytes;        /* 0 = no cap */
    int32_t device_first;  /* cuda_devices range, inclusive */
    int32_t device_last;
    int32_t timing;        /* 1 = CLB_BANK_TIMING */
    int32_t bank_flags;    /* the CLB_BANK_* flags these keys imply */
    int32_t reserved[6];
} clb_lane_config_v1;
int32_t clb_lane_config_parse(const char* text, clb_lane_config_v1* out, clb_error_v1* err);

/* Creates a bank and its fixed workspace on `device` (no allocation afterwards).
 * Replaces the construction half of HipResidentBank::load
 * (engine/strata/sycl/stage/wiring/hip_resident_bank.hpp:38-96). */
int32_t clb_bank_create(const clb_bank_config_v1* cfg, clb_bank** out, clb_error_v1* err);
void clb_bank_destroy(clb_bank* bank);

/* Allocates and fills every placed matrix (the owned range, or the experts a placement
 * gave this bank: clb_bank_apply_placement) with the counter-based synthetic weights
 * (seed, layer, expert, role, block) -> bytes. type_policy: 0 all IQ2_XXS,
 * 1 experts 0-127 IQ2_XXS / 128-255 IQ2_XS / 256+ IQ1_M, 2 per (layer, expert) from
 * the seed, 3 all IQ2_XS, 4 all IQ1_M. */
int32_t clb_bank_fill_synthetic(clb_bank* bank, uint64_t seed, int32_t type_policy, clb_error_v1* err);

/* Uploads one matrix given as ggml AoS bytes (host memory) and packs it on device.
 * Replaces the per-matrix upload of HipResidentBank::load (hip_resident_bank.hpp:97-136). */
int32_t clb_bank_load_matrix(clb_bank* bank, uint32_t layer, int32_t expert, int32_t role, int32_t type,
                             const void* ggml, size_t bytes, clb_error_v1* err);

/* ---- Strata pack ingestion (crosslane's index over the model's GGUF shards) ----
 * A pack is <dir>/ds4.txt ("key value" lines: model_dir, format, geometry) and
 * <dir>/tensors.txt ("file <i> <shard>", "t <name> <dtype> <file> <offset> <bytes> <shape...>")
 * (weight_source.hpp:1-5; pack_source.cpp:144-185); a relative model_dir is taken
 * relative to <dir>. Expert matrices are layers.<l>.ffn.experts.<e>.w{1,3,2}.weight (gate,
 * up, down) in ggml block bytes. No GPU is involved in opening or reading a pack. */
typedef struct clb_strata_pack clb_strata_pack;
/* Opens a pack: the reference's checks (model_dir present, format "gguf", well-formed and
 * unique tensor lines, no shard gap, every extent inside its shard). */
int32_t clb_strata_pack_open(const char* dir, clb_strata_pack** out, clb_error_v1* err);
void clb_strata_pack_close(clb_strata_pack* pack);
/* ds4.txt value of `key` into value[cap] (NUL-terminated); CLB_E_INVALID if absent / too long. */
int32_t clb_strata_pack_meta(const clb_strata_pack* pack, const char* key, char* value, size_t cap);
/* dtype (as tensors.txt spells it), byte size and shape of tensor `name`; CLB_E_INVALID if absent. */
int32_t clb_strata_pack_tensor(const clb_strata_pack* pack, const char* name, char* dtype, size_t dtype_cap, uint64_t* bytes,
                        int64_t* shape, int32_t shape_cap, int32_t* ndim);
/* bytes of tensor `name` from byte `offset` into dst (pread semantics, thread-safe). */
int32_t clb_strata_pack_read(const clb_strata_pack* pack, const char* name, uint64_t offset, void* dst, uint64_t bytes,
                      clb_error_v1* err);
/* Loads every matrix placed on the bank (owned range or placement) from the pack's layers
 * first_layer .. first_layer + n_layers - 1 (bank layer l <- pack layer first_layer + l),
 * repacking them into the HBM layout. Checks the pack's hidden_size, moe_intermediate_size,
 * n_routed_experts, num_hidden_layers and swiglu_limit against the bank, each expert dtype
 * (IQ2_XXS / IQ2_XS / IQ1_M, else CLB_E_UNSUPPORTED) and shape. Replaces the file half of
 * HipResidentBank::load (hip_resident_bank.hpp:97-136) over crosslane's WeightSource. */
int32_t clb_bank_load_strata_pack(clb_bank* bank, const clb_strata_pack* pack, uint32_t first_layer, clb_error_v1* err);
/* The bank's geometry. */
int32_t clb_bank_geometry(const clb_bank* bank, int32_t* n_layers, int32_t* n_experts, int32_t* dim, int32_t* ff);

/* Device bytes held by expert matrices (sum of packed sizes). */
uint64_t clb_bank_weight_bytes(const clb_bank* bank);
/* 1 when stack decode runs as the persistent kernel, 0 for the per-layer kernels
 * (CLB_BANK_PER_LAYER_KERNELS, or a geometry / device the persistent kernel cannot hold). */
int32_t clb_bank_stack_persistent(const clb_bank* bank);

/* Polls a stack kernel's bounded waits (layer barrier, a down round's inputs, the expert
 * rows of peer GPUs) make before giving up; default 2^22 (a few seconds). When a wait runs
 * out the kernel returns, the call fails with CLB_E_CUDA and the bank is poisoned (later
 * calls: CLB_E_STATE) -- e.g. when a peer GPU of a sharded bank never runs its share.
 * No counterpart in crosslane (its lanes are host threads joined on the host). */
int32_t clb_bank_set_wait_limit(clb_bank* bank, uint32_t polls, clb_error_v1* err);

/* ---- expert-ID sharding over the GPUs of one node (one process or thread per GPU) ----
 * Each GPU's bank owns experts [expert_begin, expert_end) of every layer (contiguous
 * blocks, together covering all experts). In clb_stack_decode* every GPU routes the same
 * token, computes only the picks it owns, and stores their expert rows straight into every
 * peer's exchange slot over NVLink. Per layer, default (fast) order: every CTA makes its
 * stores visible system-wide with one fence and counts itself, and the last CTA of the GPU
 * writes the layer number into its flag on every peer (one writer per flag). Exact order: a
 * per-layer counter per peer that every CTA increments. Every wait is bounded. Every GPU then runs the same combine, so all GPUs keep bit-identical
 * residual streams. All GPUs must make the same stack calls in the same order. Replaces
 * the per-layer gather that runtime.cpp:121-189 does across lanes. */
#define CLB_EXCHANGE_HANDLE_BYTES 64
/* The bank's exchange region as a CUDA IPC handle (64 bytes) for the other processes. */
int32_t clb_bank_exchange_handle(clb_bank* bank, void* handle_out, clb_error_v1* err);
/* Opens the peers' regions: handles = world x 64 bytes, indexed by rank (own entry
 * ignored). world in [2, 8]; needs the persistent stack kernel. */
int32_t clb_bank_connect(clb_bank* bank, int32_t rank, int32_t world, const void* handles, clb_error_v1* err);

/* ---- frozen warm placement ----
 * crosslane freezes which lane serves each (layer, expert) in a text document
 * (frozen_placement.hpp:5-16): "STRATA_WARM_PLACEMENT_V1 <layers> <experts> <profile tag>"
 * followed by one "<layer> <expert> <lane>" row for every pair in order. Lanes 0 (CPU),
 * 1 (HIP) and 2 (SYCL) are the reference's; CLB_LANE_CUDA (3) names this lane, which a
 * document may also give lane 1 (the GPU-lane slot). */
#define CLB_LANE_CPU 0
#define CLB_LANE_HIP 1
#define CLB_LANE_SYCL 2
#define CLB_LANE_CUDA 3
/* Parses a placement document (no GPU involved): lanes[layers * experts] receive the lane of
 * each (layer, expert), *tag (may be NULL) the profile tag. The header must name
 * n_layers x n_experts; rows must be complete, sorted, unique, lanes in [0, 3], nothing
 * after the last row (the reference's checks); otherwise CLB_E_INVALID with the reason. */
int32_t clb_placement_parse(const char* text, size_t len, int32_t n_layers, int32_t n_experts, int32_t* lanes,
                            uint64_t* tag, clb_error_v1* err);
/* Restricts the bank to the experts that lanes[layers * experts] assigns to lane_id (1 or 3
 * for this lane): later fills and matrix loads cover exactly those (within the owned
 * range), and clb_bank_contains answers for them, so warm_execute sends every other pick to
 * its other lane. Only before any weights are loaded (else CLB_E_STATE). Replaces the HIP
 * half of apply_frozen_warm_placement (frozen_placement.hpp:5-37). */
int32_t clb_bank_apply_placement(clb_bank* bank, const int32_t* lanes, int32_t lane_id, clb_error_v1* err);
/* 1 if (layer, expert) is placed on this bank (resident or to be loaded), else 0. */
int32_t clb_bank_placed(const clb_bank* bank, uint32_t layer, int32_t expert);

/* 1 if (layer, expert) is resident in this bank, else 0. Const, allocation free.
 * Replaces WarmRedirect::warm_contains (engine/strata/warm/runtime.hpp:14). */
int32_t clb_bank_contains(const clb_bank* bank, uint32_t layer, int32_t expert);

/* y[dim] = expert(x) for one resident expert; host buffers, synchronous.
 * Replaces WarmRedirect::warm_compute (runtime.hpp:15). */
int32_t clb_bank_compute(clb_bank* bank, uint32_t layer, int32_t expert, const float* x, float* y,
                         clb_error_v1* err);

/* y[n][dim] = expert_i(x), one row per id in the given order; host buffers, one
 * batched launch per phase for all picks. Replaces WarmRedirect::warm_compute_many
 * (runtime.hpp:13) / HipResidentBank::enqueue_layer (hip_resident_bank.hpp:170-236). */
int32_t clb_bank_compute_many(clb_bank* bank, uint32_t layer, const int32_t* ids, int32_t n, const float* x,
                              float* y, clb_error_v1* err);

/* out[dim] = sum over picks in ascending expert id of fma(w_i, expert_i(x)), then
 * + shared (shared may be NULL = zeros); all picks resident; host buffers.
 * The device-side twin of warm_execute's combine (engine/strata/warm/runtime.cpp:121-189). */
int32_t clb_layer_execute(clb_bank* bank, uint32_t layer, const int32_t* ids, const float* w, int32_t n,
                          const float* x, const float* shared, float* out, clb_error_v1* err);

/* Device-pointer layer step on the bank's stream (or `stream` if non-NULL):
 * d_out = [d_resid +] (combine over d_ids/d_w of expert(d_x) [+ d_shared]).
 * d_ids/d_w live in device memory (e.g. written by clb_route_device). */
int32_t clb_layer_forward_device(clb_bank* bank, uint32_t layer, const int32_t* d_ids, const float* d_w,
                                 int32_t n, const float* d_x, const float* d_shared, const float* d_resid,
                                 float* d_out, void* stream, clb_error_v1* err);

/* Profiling form of clb_layer_forward_device: runs only the kernels selected by
 * phase_mask (1 quantise x, 2 gate/up + SwiGLU + quantise h, 8 down + combine; bit 4 is
 * accepted and does nothing: h is quantised inside the gate/up kernel).
 * Phases read what earlier phases left in the bank's workspace, so a phase may run
 * alone only after a full step has run with the same arguments. */
int32_t clb_layer_phases_device(clb_bank* bank, uint32_t layer, const int32_t* d_ids, const float* d_w, int32_t n,
                                const float* d_x, float* d_out, int32_t phase_mask, void* stream, clb_error_v1* err);

/* Quant type and ggml payload bytes (sum of its three matrices) of a resident expert;
 * returns CLB_E_INVALID if (layer, expert) is not resident. */
int32_t clb_bank_expert_info(const clb_bank* bank, uint32_t layer, int32_t expert, int32_t* type,
                             uint64_t* payload_bytes);

/* Routing on device. mode 0: top-k by sigmoid(logit) (ties to the lower id),
 * weights renormalised to sum 1. `tokens` rows of n_experts logits.
 * Host twin of mode 1 (crosslane route_cpu, engine/strata/sycl/route/route.cpp:15-37)
 * is clb_route_host. */
int32_t clb_route_device(int32_t mode, const float* d_logits, int32_t n_experts, int32_t k, int32_t tokens,
                         int32_t* d_ids, float* d_w, void* stream);

/* Router logits on the device: d_logits [tokens][n_experts] = d_gate_w [n_experts][dim] .
 * d_x [tokens][dim], fp32 with a fixed summation order (run-to-run identical); dim % 4 == 0.
 * Replaces the router gemv of the GPU stage's MoE block (hip_backend.cpp:640). */
int32_t clb_router_device(const float* d_x, int32_t tokens, int32_t dim, const float* d_gate_w, int32_t n_experts,
                          float* d_logits, void* stream);

/* Mode-1 routing (crosslane route_cpu, engine/strata/sycl/route/route.cpp:15-37) on the
 * device, `tokens` rows: sc = sqrt(softplus(l)), top-k of sc + d_bias (ties to the lower
 * id), w = sc / (sum of the picks' sc + 1e-20) * scale; exp and log1p are the correctly
 * rounded float results, IEEE sqrt, add and divide. The picks equal clb_route_host(1, ...);
 * a weight differs from it by an ulp or two where glibc's expf or log1pf is not correctly
 * rounded (about 1.4 % of the scores; each such score moves every weight of its token).
 * *d_status (device int) is set to 1 if a score is not finite. n_experts <= 1024. */
int32_t clb_route_b_device(const float* d_logits, const float* d_bias, int32_t n_experts, int32_t k, int32_t tokens,
                           float scale, int32_t* d_ids, float* d_w, int32_t* d_status, void* stream);

/* The whole routed-expert MoE block of one token on the device, no host round trip
 * (the GPU stage today reads route, x back to the host for warm_execute and copies the
 * result up, hip_backend.cpp:640-742): router logits (clb_router_device) into d_logits
 * [n_experts], route_cpu's picks (max_picks of them) into d_ids/d_w, then
 * d_out = [d_resid +] combine over the picks of expert(d_x) [+ d_shared]
 * (clb_layer_forward_device). Non-finite scores or non-resident picks surface as an
 * error on the bank's next synchronising call. */
int32_t clb_moe_block_device(clb_bank* bank, uint32_t layer, const float* d_x, const float* d_gate_w,
                             const float* d_bias, float scale, const float* d_shared, const float* d_resid,
                             float* d_out, float* d_logits, int32_t* d_ids, float* d_w, void* stream,
                             clb_error_v1* err);

/* Host routing for one token. mode 0 as above; mode 1 = route_cpu:
 * sqrt(softplus(l)) + bias, top-k, w = sc / (sum + 1e-20) * scale. */
int32_t clb_route_host(int32_t mode, const float* logits, const float* bias, int32_t n_experts, int32_t k,
                       float scale, int32_t* ids, float* w);

/* Decode of `n_layers` consecutive layers for one token, end to end from host
 * memory, with the pre-norm residual structure of a DeepSeek layer:
 *   x_l = RMSNorm(h_l) = h_l * (float)(1 / sqrt(mean(h_l^2) + 1e-6))  (unit weight),
 *   h_{l+1} = h_l + combine_l(route(logits_l), experts(x_l)).
 * The fp64 sum of squares has a fixed order (1024 strided lanes, then a binary
 * tree) so it is reproducible bit for bit on the CPU.
 * h: [dim] in, logits: [n_layers][n_experts] (finite), out: [dim]. Routing mode 0 runs
 * on the host (route.cpp's selection order and the host libm, as the CPU lane), only
 * x and the routes cross to the device. One persistent kernel runs the layer range
 * (CLB_BANK_PER_LAYER_KERNELS: a captured per-layer graph, replayed). */
int32_t clb_stack_decode(clb_bank* bank, uint32_t first_layer, int32_t n_layers, const float* x,
                         const float* logits, float* out, clb_error_v1* err);

/* Device-resident variant of clb_stack_decode on the bank's stream (no host copies,
 * no synchronisation): d_x [dim] is updated in place. Routing runs on the device
 * (clb_route_device): the same experts; each weight's sigmoid uses the correctly
 * rounded exp, which glibc's expf matches on all but ~0.06% of arguments (1 ulp). */
int32_t clb_stack_decode_device(clb_bank* bank, uint32_t first_layer, int32_t n_layers, float* d_x,
                                const float* d_logits, clb_error_v1* err);

/* ---- batched prefill through one layer (grouped tensor-core GEMMs) ----
 * For T tokens with k picks each: out[t] = [resid[t] +] sum over token t's picks in
 * ascending expert id of fma(w, expert(x[t])), i.e. clb_layer_execute applied to every
 * token (warm_execute's combine, runtime.cpp:184-187). The T*k picks are grouped by
 * expert; each expert's gate/up and down run as tcgen05 GEMMs with the weights (IQ2_XXS,
 * IQ2_XS or IQ1_M, mixed freely across experts and matrices) decoded once per 48 tokens
 * into exact fp16 integers and the Q8_K activations as fp16 integers, per-256-block scales
 * applied from fp32 tensor-memory accumulators. Results agree with the CPU lane to fp32
 * reassociation (not bit for bit). dim and ff multiples of 256, from 512 to 8192 (else
 * CLB_E_UNSUPPORTED). No counterpart in crosslane's lanes (they decode one token at a time). */

/* Device bytes of workspace clb_prefill_layer_device needs for `tokens` x `k` picks. */
uint64_t clb_prefill_workspace_bytes(const clb_bank* bank, int32_t tokens, int32_t k);

/* Device-pointer prefill on the bank's stream (or `stream`), no synchronisation:
 * d_ids/d_w [tokens][k] (distinct ids per token, all resident; an id out of range or not
 * resident sets the bank's error flag, reported by the next host-synchronising call),
 * d_x/d_out [tokens][dim], d_resid NULL or [tokens][dim], d_ws >= the workspace size. */
int32_t clb_prefill_layer_device(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* d_ids,
                                 const float* d_w, const float* d_x, const float* d_resid, float* d_out, void* d_ws,
                                 uint64_t ws_bytes, void* stream, clb_error_v1* err);

/* Profiling form: only the kernels in phase_mask (1 grouping + Q8_K(x), 2 gate/up GEMM,
 * 4 SwiGLU + Q8_K(h), 8 down GEMM, 16 combine); later phases read what earlier ones left
 * in d_ws, so a phase runs alone only after a full call with the same arguments. */
int32_t clb_prefill_phases_device(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* d_ids,
                                  const float* d_w, const float* d_x, float* d_out, void* d_ws, uint64_t ws_bytes,
                                  int32_t phase_mask, void* stream, clb_error_v1* err);

/* Allocates (grow-only) the bank's own prefill workspace and pinned staging for up to
 * `tokens` x `k`; clb_prefill_layer calls it when a call is larger than the reservation. */
int32_t clb_prefill_reserve(clb_bank* bank, int32_t tokens, int32_t k, clb_error_v1* err);

/* Host-buffer prefill, synchronous: ids/w [tokens][k], x/out [tokens][dim]. */
int32_t clb_prefill_layer(clb_bank* bank, uint32_t layer, int32_t tokens, int32_t k, const int32_t* ids,
                          const float* w, const float* x, float* out, clb_error_v1* err);

/* ---- batched stack decode: T tokens (one per sequence) through consecutive layers ----
 * For every token t and layer l = first .. first + n_layers - 1:
 *   h_t <- h_t + layer_l(RMSNorm(h_t))
 * with the layer routed from logits [n_layers][tokens][n_experts] (top max_picks by sigmoid,
 * renormalised, as clb_stack_decode) and computed as one grouped prefill layer over the
 * batch, so each picked expert's weights are decoded once per 48 of its tokens instead of
 * once per token. This is clb_stack_decode applied to each token, to fp32 reassociation.
 * The bank holds every expert of those layers (no sharding); dim and ff as for prefill.
 * No counterpart in crosslane's lanes (they decode one token at a time). */
uint64_t clb_stack_batch_workspace_bytes(const clb_bank* bank, int32_t tokens);

/* Device pointers, the bank's stream (or `stream`), no synchronisation; routing on the
 * device. d_h [tokens][dim] is updated in place. */
int32_t clb_stack_batch_device(clb_bank* bank, uint32_t first_layer, int32_t n_layers, int32_t tokens,
                               const float* d_logits, float* d_h, void* d_ws, uint64_t ws_bytes, void* stream,
                               clb_error_v1* err);

/* Host buffers, synchronous; routing on the host. h [tokens][dim] is updated in place. */
int32_t clb_stack_batch(clb_bank* bank, uint32_t first_layer, int32_t n_layers, int32_t tokens, const float* logits,
                        float* h, clb_error_v1* err);

/* One layer of the batched stack in two phases, for expert-ID sharding over GPUs (the bank
 * holds experts [expert_begin, expert_end) and the caller sums the GPUs' row buffers):
 *   phase bit 1: route d_logits [tokens][n_experts] on the device, RMSNorm + Q8_K of d_h,
 *                and this bank's picks into d_rows [tokens * max_picks][dim] (slot t*k+p;
 *                the rows of other banks' picks are zero);
 *   phase bit 2: d_h += the ascending-id combine of the rows of every pick.
 * Between the two, an element-wise sum of d_rows over the GPUs (e.g. an NCCL all-reduce)
 * gives every GPU every row exactly (each row is non-zero on one GPU only), so the GPUs'
 * residual streams stay identical. The workspace is clb_stack_batch_workspace_bytes and
 * must be kept between the phases of a layer. */
int32_t clb_stack_batch_layer_device(clb_bank* bank, uint32_t layer, int32_t tokens, const float* d_logits,
                                     float* d_h, float* d_rows, void* d_ws, uint64_t ws_bytes, int32_t phase_mask,
                                     void* stream, clb_error_v1* err);

/* The bank's CUDA stream (cudaStream_t) and a synchronisation helper. */
void* clb_bank_stream(clb_bank* bank);
int32_t clb_bank_synchronize(clb_bank* bank, clb_error_v1* err);

/* ---- one expert without any allocation ---- */

/* y[dim] = down(swiglu(gate(x), up(x))) for one expert whose three matrices are given
 * in the packed layout (device pointers w_gate/w_up [ff, dim], w_down [dim, ff]); x and y
 * are device buffers; runs on `stream` and returns without synchronising.
 * No counterpart in crosslane. For callers that cannot call cudaMalloc (a serving loop
 * that must not risk an allocation's implicit device synchronisation, a plugin whose
 * device memory belongs to another allocator): the quantised input, hidden vector and
 * its quantisation live in one fixed
 * 57,856-byte array inside the library, held by every GPU that loads it until exit.
 * Limits: dim <= 16384, ff <= 8192 (else CLB_E_UNSUPPORTED with a message). It calls no
 * cudaMalloc/cudaFree. The first call on a device resolves that array's address and
 * uploads the decode tables (a synchronising step): make it before any stream capture.
 * All calls share the array, so calls that overlap on the GPU (other streams, other
 * threads) race; serialise them on one stream. Results equal clb_bank_compute's. */
int32_t clb_expert_forward_noalloc(int32_t type, const void* w_gate, const void* w_up, const void* w_down,
                                   const float* x, float* y, int32_t dim, int32_t ff, float limit, void* stream,
                                   clb_error_v1* err);

/* ---- warm_execute: the three-lane join with this bank as the GPU lane ---- */

/* Host lane callback: compute y[dim] of one non-resident expert (crosslane's
 * CpuLane::expert, engine/strata/sycl/stage/wiring/cpu_lane.hpp:18). Return 0 on
 * success; nonzero fails the layer after every lane has drained. */
typedef int32_t (*clb_host_expert_fn)(void* ctx, uint32_t layer, int32_t expert, const float* x, int32_t dim,
                                      float* y);

/* Partitions the picks (resident -> this bank, else -> host lane), runs both lanes
 * concurrently, always joins both, then combines in ascending expert id with fmaf
 * and adds `shared`. Replaces warm_execute (engine/strata/warm/runtime.cpp:121-189). */
int32_t clb_warm_execute(clb_bank* bank, uint32_t layer, const int32_t* ids, const float* w, int32_t n,
                         const float* x, const float* shared, clb_host_expert_fn host_lane, void* host_ctx,
                         float* out, clb_error_v1* err);

#ifdef __cplusplus
}
#endif

#endif /* CROSSLANE_B200_H */
