// Host-side helpers shared by the C ABI translation units: the per-thread
// last-error record, the launch counter and profiling scope, and the
// per-device attribute cache.  Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/rsort_b200.h"

namespace rsort {

// Records the failure in the calling thread's rsort_last_error record and
// returns `s`.  `role` must be a static string.
rsort_status record_failure(rsort_status s, const char *role, size_t expected = 0,
                            size_t actual = 0);

// The kernels load and store keys and values as whole elements, so every
// buffer must be aligned to its element size: a misaligned address would
// fault the kernel and leave the context unusable.  Entry points reject it
// first.  `bits` is the OR of the buffers' addresses (null adds nothing);
// the error's expected/actual are the alignment and the address remainder.
inline rsort_status check_alignment(uintptr_t bits, size_t align, const char *role) {
    if (align > 1 && (bits & (align - 1)) != 0)
        return record_failure(RSORT_BAD_ARGUMENT, role, align, size_t(bits & (align - 1)));
    return RSORT_OK;
}

inline uintptr_t addr(const void *p) { return reinterpret_cast<uintptr_t>(p); }

// Kernel launch bookkeeping: counts the launch and, when profiling is on,
// brackets it with CUDA events on `stream` (rsort_profile_*).
struct LaunchScope {
    int kernel;
    cudaStream_t stream;
    bool on;
    void *rec;
    LaunchScope(int kernel, cudaStream_t s);
    ~LaunchScope();
};

// SM count of the current device; RSORT_UNSUPPORTED_TARGET unless it is an
// sm_100 part.
rsort_status current_sm_count(int *sm_count);

// Driver entry point of the current context (cuCtxGetCurrent), as an opaque
// handle; nullptr when there is none.
cudaError_t current_context(void **ctx);

}  // namespace rsort
