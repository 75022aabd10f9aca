// Device-side building blocks of the B200 radix sort: order-preserving key
// transforms, digit extraction, warp/block ranking and the bounded decoupled
// look-back.  Everything here is hand-written SIMT code for sm_100a; sorting is
// not a contraction, so no tensor-core path exists.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace rsort {

// KIND_FLOAT_TOTAL: float keys in IEEE total order (Rust's total_cmp): the
// float bit transform without the zero fold, so -0.0 sorts before +0.0.  It
// serves the named-order merge sort entry points; the radix entry points use
// KIND_FLOAT (the reference's radix order, where -0.0 and +0.0 are equal).
enum KeyKind : int { KIND_UINT = 0, KIND_SINT = 1, KIND_FLOAT = 2, KIND_FLOAT_TOTAL = 3 };

__host__ __device__ constexpr bool is_float_kind(int kind) {
    return kind == KIND_FLOAT || kind == KIND_FLOAT_TOTAL;
}

constexpr int RADIX = 256;
constexpr uint32_t INVALID_DIGIT = 256;

// Status word values written into the counters region.
constexpr int DEV_STATUS_TIMEOUT = 7;
constexpr int DEV_STATUS_BOUNDS = 8;

template <typename B> struct KeyBits;
template <> struct KeyBits<uint8_t> {
    using Signed = int8_t;
    static constexpr uint8_t SIGN = 0x80u;
    static constexpr int WIDTH = 8;
};
template <> struct KeyBits<uint16_t> {
    using Signed = int16_t;
    static constexpr uint16_t SIGN = 0x8000u;
    static constexpr int WIDTH = 16;
};
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
    if (is_float_kind(x.kind)) {
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
    if (is_float_kind(x.kind)) {
        // top bit set -> was non-negative: flip the sign bit; else flip all bits
        a ^= (a & T::SIGN) ? T::SIGN : B(~B(0));
    } else if (x.kind == KIND_SINT) {
        a ^= T::SIGN;
    }
    return a;
}

// Compile-time-kind forms used by the onesweep pass: `dmask` is all ones for
// descending order and zero for ascending, so the direction costs one XOR.
template <int KIND, typename B>
__device__ __forceinline__ B to_ordered_k(B raw, B dmask) {
    using T = KeyBits<B>;
    if constexpr (is_float_kind(KIND))
        return raw ^ (B(typename T::Signed(raw) >> (T::WIDTH - 1)) | T::SIGN) ^ dmask;
    else if constexpr (KIND == KIND_SINT)
        return raw ^ T::SIGN ^ dmask;
    else
        return raw ^ dmask;
}

template <int KIND, typename B>
__device__ __forceinline__ B from_ordered_k(B ordered, B dmask) {
    using T = KeyBits<B>;
    const B a = ordered ^ dmask;
    if constexpr (is_float_kind(KIND))
        return a ^ (T::SIGN | B(~B(typename T::Signed(a) >> (T::WIDTH - 1))));
    else if constexpr (KIND == KIND_SINT)
        return a ^ T::SIGN;
    else
        return a;
}

template <int KIND, typename B>
__device__ __forceinline__ uint32_t digit_k(B ordered, uint32_t shift, uint32_t mask) {
    using T = KeyBits<B>;
    if constexpr (KIND == KIND_FLOAT) {
        if (ordered == B(T::SIGN - 1)) ordered = B(T::SIGN);
    }
    return uint32_t(ordered >> shift) & mask;
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
__device__ __forceinline__ uint8_t ld_stream(const uint8_t *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(v) : "l"(p));
    return uint8_t(v);
}
__device__ __forceinline__ uint16_t ld_stream(const uint16_t *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
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

// Number of predecessor words one look-back round reads in parallel.  A
// one-tile-at-a-time walk costs one L2 round trip per predecessor and, at
// B200 tile rates, has to step back past every tile still in its own
// look-back; reading a window of predecessors per round keeps the walk to
// one or two round trips.
constexpr int LOOKBACK_WINDOW = 16;

// Bound of one look-back wait: it gives up after LOOKBACK_TIMEOUT_NS of wall
// time (device %globaltimer), or after LOOKBACK_SPIN_LIMIT polls, whichever
// comes first.
constexpr uint64_t LOOKBACK_TIMEOUT_NS = 1000000000ull;
constexpr uint32_t LOOKBACK_SPIN_LIMIT = 1u << 24;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

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
    uint64_t wait_start = 0;
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
        // The word of tile `t` is not published yet: poll that word alone
        // (bounded, with back-off) and continue the walk once it is.
        for (;;) {
            const uint64_t x = ld_relaxed_gpu(lookback + t * RADIX + digit);
            const uint64_t state = x & (3ull << 62);
            if (state != 0 && uint32_t((x >> 48) & 0x3fff) == want_tag) {
                exclusive += x & LB_VALUE_MASK;
                if (state == LB_INCLUSIVE) return exclusive;
                --t;
                break;
            }
            if (spins == 0) wait_start = global_ns();
            ++spins;
            if (spins > 8) __nanosleep(spins > 4096 ? 256 : 32);
            if ((spins & 255) == 0) {
                if (ld_relaxed_gpu(status) != 0) {
                    *gave_up = true;
                    return exclusive;
                }
                if (global_ns() - wait_start > LOOKBACK_TIMEOUT_NS) {
                    atomicExch(status, DEV_STATUS_TIMEOUT);
                    *gave_up = true;
                    return exclusive;
                }
            }
            if (spins > LOOKBACK_SPIN_LIMIT) {
                atomicExch(status, DEV_STATUS_TIMEOUT);
                *gave_up = true;
                return exclusive;
            }
        }
    }
    return exclusive;
}

// ---------------------------------------------------------------------------
// Warp-level stable multi-split rank.  Items are processed in warp-striped
// order (item j of lane l sits at segment position j*32 + l), so lane order
// within one step and step order across steps are both input order.
// `whist` is this warp's 256-entry running histogram in shared memory.
// ---------------------------------------------------------------------------
// Pipelined form over a thread's items, RANK_GROUP items at a time: every
// match of the group is issued first, then the peer-group leaders (highest
// lane of each group) add the group size to the warp histogram with one
// shared atomic per group, then every lane fetches its group's base from the
// leader.  The atomics of one warp reach the shared-memory unit in program
// order, so item j sees the counts of items 0..j-1 exactly as a serial walk
// does.  Groups bound the live registers of the pipeline.
constexpr int RANK_GROUP = 4;

// Lanes of the warp holding the same 8-bit digit: one ballot per digit bit
// (eight votes and eight logic ops).  On sm_100 this is far cheaper than
// __match_any_sync for 8-bit labels (measured: a 16-item rank step took ~9 us
// per 8192-key tile with match.any).  Padding items carry INVALID_DIGIT; a
// ninth vote on validity keeps them out of real digits' groups.
__device__ __forceinline__ uint32_t match_digit(uint32_t d, bool check_valid) {
    uint32_t peers = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const bool set = (d >> b) & 1u;
        const uint32_t v = __ballot_sync(0xffffffffu, set);
        peers &= set ? v : ~v;
    }
    if (check_valid) {
        const bool valid = d < RADIX;
        const uint32_t v = __ballot_sync(0xffffffffu, valid);
        peers &= valid ? v : ~v;
    }
    return peers;
}

// Warp multi-split rank, one item per lane per step, steps in input order.
// Per step the lanes of each digit find their peer group through a shared
// atomicOr of lane bits into the warp's 256-word mask array; the group's
// leader (its highest lane) fetches the warp's running count for the digit and
// advances it by the group size with one shared atomicAdd, and every lane
// takes base + its rank among lower peers.  RANK_MASK_SETS mask arrays
// are used in rotation: item j ORs into set j % 3 and the leader of item j
// clears its word while item j + 1 runs, after the sync that orders it
// behind every read of it, so one __syncwarp per item orders everything.
// (__match_any_sync, an 8-ballot network, owner election by lane-id stores
// and a three-sync single-array form were all measured slower on sm_100.)
constexpr int RANK_MASK_SETS = 3;

// Runs of equal keys: after the first pass, equal keys lie next to each
// other, so with duplicate-heavy inputs most warp steps hold one digit in all
// 32 lanes, or two (a run boundary), and their atomicOrs to one mask word
// serialize.  In RANK_RUNS mode the groups of lane 0's and lane 31's digits
// take their peer masks from two shuffles and two ballots and touch no mask
// word; only lanes between two run boundaries use the mask words.  Measured
// on B200 (2^30 u32 keys, 90% Zipf(1.1) + 10% one constant, passes 1-3):
// 5.35 / 5.05 / 4.07 ms with whole-warp steps only, 4.21 / 4.11 / 4.42 ms
// with the two groups.
constexpr int RANK_PLAIN = 0;
constexpr int RANK_RUNS = 1;

// A pass whose digit histogram has one digit holding at least 1/HOT_SHARE
// of the keys (short of all of them) is "hot".  A pass after the first runs
// the RANK_RUNS kernel when it and the pass before are both hot: that is
// where long runs of equal keys come from.  Measured on B200 (2^30 u32
// keys, 90% Zipf(1.1) + 10% one constant, all passes hot).
constexpr uint32_t HOT_SHARE = 16;

// rank[j] = digit << 16 | rank of item j among the warp's items of its digit.
// ALL_VALID: no padding items (full tile), so no per-item validity tests.
// MODE: RANK_PLAIN or RANK_RUNS (ALL_VALID only).
template <int ITEMS, bool ALL_VALID, int MODE = RANK_PLAIN, typename DigitAt>
__device__ __forceinline__ void warp_rank_items_or3(DigitAt digit_at, uint32_t (&rank)[ITEMS],
                                                    uint32_t *whist, uint32_t *wmask) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t lt = lanemask_lt(), bit = 1u << lane;
    uint32_t prev_d = 0;
    bool prev_leader = false;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        uint32_t *m = wmask + (j % 3) * RADIX;
        const uint32_t d = digit_at(j);
        const bool valid = ALL_VALID || d < RADIX;
        // RANK_RUNS: the lanes holding lane 0's digit, and those holding lane
        // 31's, take their peer masks from one ballot each (a step inside a
        // run is one group; a step across a run boundary is two, or two plus
        // a few lanes in between that use the mask words).
        bool known = false;
        uint32_t known_peers = 0;
        if constexpr (MODE == RANK_RUNS) {
            static_assert(ALL_VALID, "runs are found in full tiles only");
            // (Testing for a whole-warp group first, and taking the second
            // ballot only when that fails, measured the same on config 4.)
            const uint32_t d_first = __shfl_sync(0xffffffffu, d, 0);
            const uint32_t d_last = __shfl_sync(0xffffffffu, d, 31);
            const uint32_t b_first = __ballot_sync(0xffffffffu, d == d_first);
            const uint32_t b_last = __ballot_sync(0xffffffffu, d == d_last);
            known = d == d_first || d == d_last;
            known_peers = d == d_first ? b_first : b_last;
        }
        const bool uniform = known;  // no mask word for this lane's group
        if (valid && !uniform) atomicOr(&m[d], bit);
        // Orders this item's ORs before the reads below, the previous item's
        // reads before its clear below, and the previous item's whist update
        // before this item's whist read.
        __syncwarp();
        if (prev_leader) wmask[((j + 2) % 3) * RADIX + prev_d] = 0u;
        const uint32_t peers = uniform ? known_peers : valid ? m[d] : 0u;
        const uint32_t leader = 31 - __clz(peers);
        const bool is_leader = valid && lane == leader;
        // One shared atomic per group: it returns the running count and
        // advances it (measured 2-5% faster per pass than a load and a store).
        uint32_t got = 0;
        if (is_leader) got = atomicAdd(&whist[d], __popc(peers));
        prev_leader = is_leader && !uniform;  // a uniform step set no mask word
        prev_d = d;
        // Packed (digit << 16 | rank): the rank within the warp is below
        // 32 * ITEMS < 2^16, and the scatter reads the digit back from here.
        rank[j] = (d << 16) | (__shfl_sync(0xffffffffu, got, leader & 31) + __popc(peers & lt));
        asm volatile("" : "+r"(rank[j]));
    }
    // The last item's mask word stays set: the scratch is re-zeroed before
    // the next tile uses it.
    __syncwarp();
}

// `digit_at(j)` returns item j's digit (INVALID_DIGIT for padding items).
template <int ITEMS, typename DigitAt>
__device__ __forceinline__ void warp_rank_items(DigitAt digit_at, uint32_t (&rank)[ITEMS],
                                                uint32_t *whist, bool partial) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t lt = lanemask_lt();
#pragma unroll
    for (int g = 0; g < ITEMS; g += RANK_GROUP) {
        constexpr int G = RANK_GROUP;
        uint32_t d[G], peers[G], got[G];
#pragma unroll
        for (int u = 0; u < G; ++u)
            if (g + u < ITEMS) {
                d[u] = digit_at(g + u);
                peers[u] = match_digit(d[u], partial);
            }
#pragma unroll
        for (int u = 0; u < G; ++u) {
            if (g + u < ITEMS) {
                const uint32_t leader = 31 - __clz(peers[u]);
                got[u] = 0;
                if (lane == leader && d[u] < RADIX)
                    got[u] = atomicAdd(&whist[d[u]], __popc(peers[u]));
            }
        }
#pragma unroll
        for (int u = 0; u < G; ++u) {
            if (g + u < ITEMS) {
                const uint32_t leader = 31 - __clz(peers[u]);
                rank[g + u] = __shfl_sync(0xffffffffu, got[u], leader) + __popc(peers[u] & lt);
            }
        }
    }
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
