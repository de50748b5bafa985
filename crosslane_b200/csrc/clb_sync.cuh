// Memory-model helpers of the persistent stack kernel: release/acquire counter operations
// at GPU scope (CTAs of one GPU) and system scope (peer GPUs of a sharded bank), and a
// bounded wait on a counter.
#pragma once
#include <cuda_runtime.h>

namespace clb {

__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait until *p has reached target (modulo 2^32). SYS: the writers include other
// GPUs. Polls with relaxed loads (an acquire load per poll would discard the SM's L1 lines
// each time, under the feet of the warps still decoding) and orders the caller's later
// reads after the writes it waited for with one fence once the target is seen (the
// relaxed-load + fence acquire pattern). Backs off after a few hundred polls. After
// `limit` polls it sets *err = code and returns false.
template <bool SYS>
__device__ bool wait_reached(const unsigned* p, unsigned target, int* err, unsigned limit, int code) {
    for (unsigned spins = 0;; ++spins) {
        const unsigned v = SYS ? ld_relaxed_sys(p) : ld_relaxed_gpu(p);
        if ((int)(v - target) >= 0) {
            if (SYS) fence_acq_rel_sys();
            else fence_acq_rel_gpu();
            return true;
        }
        if (spins > limit) {
            atomicExch(err, code);
            return false;
        }
        if (spins > 256) __nanosleep(64);
    }
}

}  // namespace clb
