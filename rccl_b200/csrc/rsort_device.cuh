// Device-side building blocks of the B200 radix sort: order-preserving key
// transforms, digit extraction, warp/block ranking and the bounded decoupled
// look-back.  Everything here is hand-written SIMT code for sm_100a; sorting is
// not a contraction, so no tensor-core path exists.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace rsort {

enum KeyKind : int { KIND_UINT = 0, KIND_SINT = 1, KIND_FLOAT = 2 };

constexpr int RADIX = 256;
constexpr uint32_t INVALID_DIGIT = 256;

// Status word values written into the counters region.
constexpr int DEV_STATUS_TIMEOUT = 7;
constexpr int DEV_STATUS_BOUNDS = 8;

template <typename B> struct KeyBits;
template <> struct KeyBits<uint32_t> {
    using Signed = int32_t;
    static constexpr uint32_t SIGN = 0x80000000u;
    static constexpr int WIDTH = 32;
};
template <> struct KeyBits<uint64_t> {
    using Signed = int64_t;
    static constexpr uint64_t SIGN = 0x8000000000000000ull;
    static constexpr int WIDTH = 64;
};

// Per-launch description of the key transform.  `kind` and `desc` are uniform
// across the grid, so the branches below never diverge.
struct KeyXform {
    int kind;
    int desc;
};

// Order-preserving image of a raw key (rccl-cub/src/ordering_backend/radix.rs:75-235):
// uint identity, int flips the sign bit, float flips every bit of negatives and
// the sign bit of non-negatives; descending is the bitwise NOT of ascending.
template <typename B>
__device__ __forceinline__ B to_ordered(B raw, KeyXform x) {
    using T = KeyBits<B>;
    B o = raw;
    if (x.kind == KIND_FLOAT) {
        o ^= B(typename T::Signed(raw) >> (T::WIDTH - 1)) | T::SIGN;
    } else if (x.kind == KIND_SINT) {
        o ^= T::SIGN;
    }
    return x.desc ? B(~o) : o;
}

template <typename B>
__device__ __forceinline__ B from_ordered(B ordered, KeyXform x) {
    using T = KeyBits<B>;
    B a = x.desc ? B(~ordered) : ordered;
    if (x.kind == KIND_FLOAT) {
        // top bit set -> was non-negative: flip the sign bit; else flip all bits
        a ^= (a & T::SIGN) ? T::SIGN : B(~B(0));
    } else if (x.kind == KIND_SINT) {
        a ^= T::SIGN;
    }
    return a;
}

// The float digit functions fold the ordered image 0x7fff..ff (one of the two
// zeros) onto 0x8000..00 so that -0.0 and +0.0 are equal radix keys
// (rccl-cub/src/ordering_backend/radix.rs:257-337).
template <typename B>
__device__ __forceinline__ B fold_zero(B ordered, int kind) {
    using T = KeyBits<B>;
    return (kind == KIND_FLOAT && ordered == B(T::SIGN - 1)) ? B(T::SIGN) : ordered;
}

template <typename B>
__device__ __forceinline__ uint32_t digit_of(B ordered, int kind, uint32_t shift, uint32_t mask) {
    return uint32_t(fold_zero(ordered, kind) >> shift) & mask;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ uint32_t lanemask_gt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_gt;" : "=r"(m));
    return m;
}

// Streaming (read-once) global loads: no L1 allocation.
__device__ __forceinline__ uint32_t ld_stream(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint64_t ld_stream(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint64_t ld_relaxed_gpu(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_gpu(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// Decoupled look-back words (one 64-bit word per tile and digit):
//   bits 63..62  state: 0 = empty, 1 = tile aggregate, 2 = inclusive prefix
//   bits 61..48  pass tag (pass index + 1), so one zeroing per sort serves
//                every pass
//   bits 47..0   count
// ---------------------------------------------------------------------------
constexpr uint64_t LB_AGGREGATE = 1ull << 62;
constexpr uint64_t LB_INCLUSIVE = 2ull << 62;
constexpr uint64_t LB_VALUE_MASK = (1ull << 48) - 1;

__device__ __forceinline__ uint64_t lb_word(uint64_t state, uint32_t tag, uint64_t value) {
    return state | (uint64_t(tag & 0x3fff) << 48) | (value & LB_VALUE_MASK);
}

// Iteration bound of one look-back wait: with the back-off below this is
// roughly a second of wall time before the wait gives up.
constexpr uint32_t LOOKBACK_SPIN_LIMIT = 1u << 22;

// Number of predecessor words one look-back round reads in parallel.  A
// one-tile-at-a-time walk costs one L2 round trip per predecessor and, at
// B200 tile rates, has to step back past every tile still in its own
// look-back; reading a window of predecessors per round keeps the walk to
// one or two round trips.
constexpr int LOOKBACK_WINDOW = 16;

// Sums the per-digit counts of all tiles before `tile`: walks back in windows
// of LOOKBACK_WINDOW predecessors, adding aggregates until it meets an
// inclusive prefix.  A word that is not yet published is re-polled (bounded):
// on give-up the device status word is set and the (meaningless) partial sum
// is returned; the caller then skips its global writes.
__device__ __forceinline__ uint64_t lookback_exclusive(const uint64_t *lookback, int64_t tile,
                                                       uint32_t digit, uint32_t tag, int *status,
                                                       bool *gave_up) {
    uint64_t exclusive = 0;
    int64_t t = tile - 1;
    uint32_t spins = 0;
    const uint32_t want_tag = tag & 0x3fff;
    while (t >= 0) {
        uint64_t w[LOOKBACK_WINDOW];
#pragma unroll
        for (int k = 0; k < LOOKBACK_WINDOW; ++k)
            w[k] = (t - k >= 0) ? ld_relaxed_gpu(lookback + (t - k) * RADIX + digit)
                                : lb_word(LB_INCLUSIVE, want_tag, 0);
        bool stop = false, found = false;
        int consumed = 0;
#pragma unroll
        for (int k = 0; k < LOOKBACK_WINDOW; ++k) {
            if (!stop) {
                const uint64_t state = w[k] & (3ull << 62);
                const bool ready = state != 0 && uint32_t((w[k] >> 48) & 0x3fff) == want_tag;
                if (!ready) {
                    stop = true;
                } else {
                    exclusive += w[k] & LB_VALUE_MASK;
                    ++consumed;
                    if (state == LB_INCLUSIVE) found = stop = true;
                }
            }
        }
        if (found) return exclusive;
        t -= consumed;
        if (consumed == LOOKBACK_WINDOW) continue;
        // The word at `t` is not published yet: back off and re-poll.
        ++spins;
        if (spins > 8) __nanosleep(spins > 4096 ? 256 : 32);
        if ((spins & 255) == 0 && ld_relaxed_gpu(status) != 0) {
            *gave_up = true;
            return exclusive;
        }
        if (spins > LOOKBACK_SPIN_LIMIT) {
            atomicExch(status, DEV_STATUS_TIMEOUT);
            *gave_up = true;
            return exclusive;
        }
    }
    return exclusive;
}

// ---------------------------------------------------------------------------
// Warp-level stable multi-split rank.  Items are processed in warp-striped
// order (item j of lane l sits at segment position j*32 + l), so lane order
// within one step and step order across steps are both input order.
// `whist` is this warp's 256-entry running histogram in shared memory.
// Returns the item's rank among equal digits of this warp processed so far.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t warp_rank_step(uint32_t d, uint32_t *whist) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t before = __popc(peers & lanemask_lt());
    const bool last_peer = (peers & lanemask_gt()) == 0;
    uint32_t base = 0;
    if (d < RADIX) base = whist[d];
    __syncwarp();
    if (last_peer && d < RADIX) whist[d] = base + before + 1;
    __syncwarp();
    (void)lane;
    return base + before;
}

// Exclusive scan over 256 values held by threads 0..255 (one per thread).
// `warp_sums` needs 8 words.  Must be called by all threads of the block.
__device__ __forceinline__ uint32_t block_exclusive_scan_256(uint32_t v, uint32_t *warp_sums,
                                                             uint32_t *total) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t inc = v;
    if (tid < RADIX) {
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= uint32_t(off)) inc += y;
        }
        if (lane == 31) warp_sums[warp] = inc;
    }
    __syncthreads();
    uint32_t prefix = 0, all = 0;
#pragma unroll
    for (int w = 0; w < RADIX / 32; ++w) {
        const uint32_t s = warp_sums[w];
        if (uint32_t(w) < warp) prefix += s;
        all += s;
    }
    if (total) *total = all;
    return prefix + inc - v;
}

}  // namespace rsort
