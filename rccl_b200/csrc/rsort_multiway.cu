// Single-pass stable merge of W sorted runs (no reference counterpart: the
// last step of the multi-GPU sample sort, where every rank merges the W runs
// it received).  Ties keep the lower run first, so runs given in source-rank
// order merge into the global stable order.
//
// Partition.  Every run contributes a pivot every S items (its items 0, S,
// 2S, ...).  For a pivot x of run s, the number of items of run t that come
// before x in the merged order is a binary search in run t (items with an
// image <= x for t < s, < x for t > s; S*k for run s itself), and x's rank
// among all pivots is the sum over runs of ceil(count / S).  Row q of the
// pivot table holds these W counts for the q-th pivot in merged order; row P
// holds the run lengths.  Between two consecutive pivots each run contributes
// fewer than S items, so G consecutive intervals hold at most (W + G) * S
// items: one CTA merges them in shared memory.
//
// Merge.  A CTA loads its G intervals' W segments (row r0 to row r0 + G of
// the table) back to back into shared memory, merges them pairwise in
// log2(W) rounds between two shared buffers (merge path per thread, ties to
// the left segment), and writes its output range out coalesced.  The runs
// are read once and the output written once.
#include "../../include/rsort_b200.h"
#include "rsort_device.cuh"
#include "rsort_internal.cuh"
#include "rsort_multiway.cuh"

namespace rsort {

template <typename B>
__device__ __forceinline__ uint64_t mw_image(B raw, KeyXform xf) {
    return uint64_t(fold_zero(to_ordered(raw, xf), xf.kind));
}

// Items of run `t` (length len) that precede an item of image x from run s:
// image <= x when t < s (the lower run wins ties), image < x when t > s.
template <typename B>
__device__ __forceinline__ uint64_t mw_count_before(const B *run, uint64_t len, uint64_t x,
                                                    bool le, KeyXform xf) {
    uint64_t lo = 0, hi = len;
    while (lo < hi) {
        const uint64_t mid = lo + ((hi - lo) >> 1);
        const uint64_t v = mw_image(run[mid], xf);
        if (le ? v <= x : v < x)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Pivot p of the table: its run s, its index k*S, and the counts of every
// run's items before it.  MAXW > 0: the W - 1 binary searches advance level
// by level together, with one load per run in flight at a time (W <= MAXW,
// registers); MAXW == 0: one search after another (any W).
template <typename B, int MAXW>
__global__ void multiway_pivot_kernel(MultiwayArgs a) {
    const uint64_t p = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t W = a.runs;
    if (p == a.pivots) {
        for (uint32_t t = 0; t < W; ++t) a.table[p * W + t] = a.len[t];
        return;
    }
    if (p > a.pivots) return;
    uint32_t s = 0;
    while (p >= a.pivot_start[s + 1]) ++s;
    const uint64_t k = p - a.pivot_start[s];
    const KeyXform xf{a.kind, a.desc};
    const uint64_t x = mw_image(static_cast<const B *>(a.keys[s])[k * a.stride], xf);
    uint64_t q = k;
    if constexpr (MAXW > 0) {
        uint64_t lo[MAXW], hi[MAXW];
        const B *run[MAXW];
#pragma unroll
        for (int t = 0; t < MAXW; ++t) {
            lo[t] = 0;
            hi[t] = (uint32_t(t) < W && uint32_t(t) != s) ? a.len[t] : 0;
            run[t] = uint32_t(t) < W ? static_cast<const B *>(a.keys[t]) : nullptr;
        }
        for (;;) {
            bool any = false;
            uint64_t v[MAXW];
#pragma unroll
            for (int t = 0; t < MAXW; ++t)
                if (lo[t] < hi[t]) v[t] = mw_image(run[t][lo[t] + ((hi[t] - lo[t]) >> 1)], xf);
#pragma unroll
            for (int t = 0; t < MAXW; ++t) {
                if (lo[t] < hi[t]) {
                    const uint64_t mid = lo[t] + ((hi[t] - lo[t]) >> 1);
                    const bool before = uint32_t(t) < s ? v[t] <= x : v[t] < x;
                    if (before)
                        lo[t] = mid + 1;
                    else
                        hi[t] = mid;
                    any = true;
                }
            }
            if (!any) break;
        }
#pragma unroll
        for (int t = 0; t < MAXW; ++t) {
            if (uint32_t(t) >= W) break;
            const uint64_t c = uint32_t(t) == s ? k * a.stride : lo[t];
            if (uint32_t(t) != s) q += (c + a.stride - 1) / a.stride;
            lo[t] = c;
        }
#pragma unroll
        for (int t = 0; t < MAXW; ++t)
            if (uint32_t(t) < W) a.table[q * W + t] = lo[t];
    } else {
        uint64_t c[MW_MAX_RUNS];
        for (uint32_t t = 0; t < W; ++t) {
            if (t == s) {
                c[t] = k * a.stride;
                continue;
            }
            c[t] = mw_count_before(static_cast<const B *>(a.keys[t]), a.len[t], x, t < s, xf);
            q += (c[t] + a.stride - 1) / a.stride;
        }
        for (uint32_t t = 0; t < W; ++t) a.table[q * W + t] = c[t];
    }
}

template <int VB> struct MwValue;
template <> struct MwValue<0> { using type = uint8_t; };
template <> struct MwValue<1> { using type = uint8_t; };
template <> struct MwValue<2> { using type = uint16_t; };
template <> struct MwValue<4> { using type = uint32_t; };
template <> struct MwValue<8> { using type = uint64_t; };
template <> struct MwValue<16> { using type = uint4; };

template <typename B, int VB>
struct MwShape {
    static constexpr int ITEMS = mw_items(int(sizeof(B)), VB);
    static constexpr int CAP = MW_THREADS * ITEMS;
    static constexpr int VSIZE = VB > 0 ? VB : 1;
    // two buffers (keys, values each), then the segment bounds
    static constexpr size_t K0 = 0;
    static constexpr size_t K1 = K0 + size_t(CAP) * sizeof(B);
    static constexpr size_t V0 = K1 + size_t(CAP) * sizeof(B);
    static constexpr size_t V1 = V0 + (VB > 0 ? size_t(CAP) * VSIZE : 0);
    static constexpr size_t BND = (V1 + (VB > 0 ? size_t(CAP) * VSIZE : 0) + 15) / 16 * 16;
    static constexpr size_t BYTES = BND + size_t(2 * MW_MAX_RUNS) * 8 + size_t(MW_MAX_RUNS + 1) * 4;
};

template <typename B, int VB>
__global__ void __launch_bounds__(MW_THREADS) multiway_merge_kernel(MultiwayArgs a) {
    using S = MwShape<B, VB>;
    using VT = typename MwValue<VB>::type;
    constexpr int ITEMS = S::ITEMS;
    extern __shared__ __align__(16) uint8_t smem[];
    B *const kb0 = reinterpret_cast<B *>(smem + S::K0);
    B *const kb1 = reinterpret_cast<B *>(smem + S::K1);
    VT *const vb0 = reinterpret_cast<VT *>(smem + S::V0);
    VT *const vb1 = reinterpret_cast<VT *>(smem + S::V1);
    const B **kseg = reinterpret_cast<const B **>(smem + S::BND);          // [W] segment starts
    const VT **vseg = reinterpret_cast<const VT **>(kseg + MW_MAX_RUNS);    // [W]
    uint32_t *bnd = reinterpret_cast<uint32_t *>(vseg + MW_MAX_RUNS);       // [W + 1] offsets
    __shared__ uint64_t lo_row[MW_MAX_RUNS], len_row[MW_MAX_RUNS];
    __shared__ uint64_t out_base;
    const uint32_t W = a.runs, tid = threadIdx.x;
    const KeyXform xf{a.kind, a.desc};
    const uint64_t r0 = uint64_t(blockIdx.x) * a.group;
    const uint64_t r1 = r0 + a.group < a.pivots ? r0 + a.group : a.pivots;
    // The table rows are read by W threads at once; one thread then turns the
    // segment lengths into offsets.
    if (tid < W) {
        const uint64_t lo = a.table[r0 * W + tid], hi = a.table[r1 * W + tid];
        lo_row[tid] = lo;
        len_row[tid] = hi - lo;
        kseg[tid] = static_cast<const B *>(a.keys[tid]) + lo;
        vseg[tid] = VB > 0 ? static_cast<const VT *>(a.values[tid]) + lo : nullptr;
    }
    __syncthreads();
    if (tid == 0) {
        uint64_t base = 0;
        uint32_t off = 0;
        for (uint32_t t = 0; t < W; ++t) {
            bnd[t] = off;
            off += uint32_t(len_row[t]);
            base += lo_row[t];
        }
        bnd[W] = off;
        out_base = base;
    }
    __syncthreads();
    const uint32_t n = bnd[W];
    // The partition bounds n by (W + G) * S <= CAP; the test only keeps a
    // corrupt table from overrunning shared memory.
    if (n > uint32_t(S::CAP)) return;
    // Stage the W segments back to back.  Every load of a thread is issued
    // before its first shared store, so ITEMS loads per thread are in flight
    // at once (the runs may be a peer's memory, microseconds away).
    {
        B kr[ITEMS];
        VT vr[VB > 0 ? ITEMS : 1];
        uint32_t t = 0;
#pragma unroll
        for (int u = 0; u < ITEMS; ++u) {
            const uint32_t i = tid + uint32_t(u) * MW_THREADS;
            if (i < n) {
                while (i >= bnd[t + 1]) ++t;
                kr[u] = kseg[t][i - bnd[t]];
                if constexpr (VB > 0) vr[u] = vseg[t][i - bnd[t]];
            }
        }
#pragma unroll
        for (int u = 0; u < ITEMS; ++u) {
            const uint32_t i = tid + uint32_t(u) * MW_THREADS;
            if (i < n) {
                kb0[i] = kr[u];
                if constexpr (VB > 0) vb0[i] = vr[u];
            }
        }
    }
    __syncthreads();

    // Pairwise rounds: segments (0,1), (2,3), ... of the current buffer merge
    // into the other; an unpaired last segment is copied.
    int cur = 0;
    uint32_t segs = W;
    while (segs > 1) {
        const B *ik = cur ? kb1 : kb0;
        const VT *iv = cur ? vb1 : vb0;
        B *ok = cur ? kb0 : kb1;
        VT *ov = cur ? vb0 : vb1;
        const uint32_t o0 = tid * ITEMS;
        const uint32_t oend = o0 + ITEMS < n ? o0 + ITEMS : n;
        const uint32_t npairs = (segs + 1) >> 1;
        // Fast path: the thread's outputs lie in one merge pair, so the merge
        // is a fixed, unrolled ITEMS-step loop (as in the two-run merge).
        bool done = o0 >= n;
        if (!done) {
            uint32_t pr = 0;
            while (pr + 1 < npairs && bnd[2 * pr + 2] <= o0) ++pr;
            const uint32_t sa = 2 * pr;
            const uint32_t a0 = bnd[sa], a1 = bnd[sa + 1];
            const uint32_t b1 = sa + 1 < segs ? bnd[sa + 2] : a1;
            if (oend <= b1 && b1 > a1) {
                const uint32_t la = a1 - a0, lb = b1 - a1;
                const B *ta = ik + a0;
                const B *tb = ik + a1;
                const uint32_t diag = o0 - a0;
                uint32_t lo = diag > lb ? diag - lb : 0, hi = diag < la ? diag : la;
                while (lo < hi) {
                    const uint32_t mid = (lo + hi) >> 1;
                    if (mw_image(ta[mid], xf) <= mw_image(tb[diag - 1 - mid], xf))
                        lo = mid + 1;
                    else
                        hi = mid;
                }
                uint32_t ia = lo, ib = diag - lo;
                uint64_t ima = ia < la ? mw_image(ta[ia], xf) : 0;
                uint64_t imb = ib < lb ? mw_image(tb[ib], xf) : 0;
#pragma unroll
                for (int k = 0; k < ITEMS; ++k) {
                    const bool take_a = ib >= lb || (ia < la && ima <= imb);
                    const uint32_t src = take_a ? a0 + ia : a1 + ib;
                    if (o0 + k < oend) {
                        ok[o0 + k] = ik[src];
                        if constexpr (VB > 0) ov[o0 + k] = iv[src];
                    }
                    if (take_a) {
                        ++ia;
                        if (ia < la) ima = mw_image(ta[ia], xf);
                    } else {
                        ++ib;
                        if (ib < lb) imb = mw_image(tb[ib], xf);
                    }
                }
                done = true;
            }
        }
        // General path: outputs that cross a pair boundary, or a lone
        // segment's copy.
        uint32_t o = done ? oend : o0;
        while (o < oend) {
            // the pair (segments 2pr and 2pr + 1) holding output position o;
            // a lone last segment is a pair without a right side
            uint32_t pr = 0;
            while (pr + 1 < npairs && bnd[2 * pr + 2] <= o) ++pr;
            const uint32_t sa = 2 * pr;
            const uint32_t a0 = bnd[sa];
            const uint32_t a1 = bnd[sa + 1];
            const uint32_t b1 = sa + 1 < segs ? bnd[sa + 2] : a1;
            const uint32_t la = a1 - a0, lb = b1 - a1;
            const uint32_t stop = oend < b1 ? oend : b1;
            if (lb == 0) {  // unpaired segment: copy
                for (; o < stop; ++o) {
                    ok[o] = ik[o];
                    if constexpr (VB > 0) ov[o] = iv[o];
                }
                continue;
            }
            const B *ta = ik + a0;
            const B *tb = ik + a1;
            const uint32_t diag = o - a0;
            uint32_t lo = diag > lb ? diag - lb : 0, hi = diag < la ? diag : la;
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (mw_image(ta[mid], xf) <= mw_image(tb[diag - 1 - mid], xf))
                    lo = mid + 1;
                else
                    hi = mid;
            }
            uint32_t ia = lo, ib = diag - lo;
            uint64_t ima = ia < la ? mw_image(ta[ia], xf) : 0;
            uint64_t imb = ib < lb ? mw_image(tb[ib], xf) : 0;
            for (; o < stop; ++o) {
                const bool take_a = ib >= lb || (ia < la && ima <= imb);
                const uint32_t src = take_a ? a0 + ia : a1 + ib;
                ok[o] = ik[src];
                if constexpr (VB > 0) ov[o] = iv[src];
                if (take_a) {
                    ++ia;
                    if (ia < la) ima = mw_image(ta[ia], xf);
                } else {
                    ++ib;
                    if (ib < lb) imb = mw_image(tb[ib], xf);
                }
            }
        }
        __syncthreads();
        // merged pair p spans the old segments 2p and 2p + 1
        const uint32_t nsegs = (segs + 1) / 2;
        if (tid == 0) {
            for (uint32_t p = 1; p <= nsegs; ++p) bnd[p] = bnd[2 * p < segs ? 2 * p : segs];
        }
        __syncthreads();
        segs = nsegs;
        cur ^= 1;
    }

    B *outk = static_cast<B *>(a.out_keys) + out_base;
    VT *outv = VB > 0 ? static_cast<VT *>(a.out_values) + out_base : nullptr;
    const B *fk = cur ? kb1 : kb0;
    const VT *fv = cur ? vb1 : vb0;
    for (uint32_t i = tid; i < n; i += MW_THREADS) {
        outk[i] = fk[i];
        if constexpr (VB > 0) outv[i] = fv[i];
    }
}

namespace {

template <typename B, int VB>
cudaError_t multiway_t(MultiwayArgs &a, cudaStream_t s) {
    using S = MwShape<B, VB>;
    const uint32_t piv_blocks = uint32_t((a.pivots + 1 + 255) / 256);
    if (a.runs <= 2)
        multiway_pivot_kernel<B, 2><<<piv_blocks, 256, 0, s>>>(a);
    else if (a.runs <= 4)
        multiway_pivot_kernel<B, 4><<<piv_blocks, 256, 0, s>>>(a);
    else if (a.runs <= 8)
        multiway_pivot_kernel<B, 8><<<piv_blocks, 256, 0, s>>>(a);
    else
        multiway_pivot_kernel<B, 0><<<piv_blocks, 256, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto k = multiway_merge_kernel<B, VB>;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::BYTES));
    if (e != cudaSuccess) return e;
    const uint64_t groups = (a.pivots + a.group - 1) / a.group;
    if (groups == 0) return cudaSuccess;
    k<<<dim3(uint32_t(groups)), MW_THREADS, S::BYTES, s>>>(a);
    return cudaGetLastError();
}

template <typename B>
cudaError_t multiway_vb(int vb, MultiwayArgs &a, cudaStream_t s) {
    switch (vb) {
        case 0: return multiway_t<B, 0>(a, s);
        case 1: return multiway_t<B, 1>(a, s);
        case 2: return multiway_t<B, 2>(a, s);
        case 4: return multiway_t<B, 4>(a, s);
        case 8: return multiway_t<B, 8>(a, s);
        case 16: return multiway_t<B, 16>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_multiway(int key_bytes, int value_bytes, MultiwayArgs &a, cudaStream_t s) {
    return key_bytes == 8 ? multiway_vb<uint64_t>(value_bytes, a, s)
                          : multiway_vb<uint32_t>(value_bytes, a, s);
}

}  // namespace rsort

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {

using rsort::MultiwayArgs;
using rsort::record_failure;

int key_bytes_mw(rsort_key_t k) { return (k == RSORT_U64 || k == RSORT_I64 || k == RSORT_F64) ? 8 : 4; }
int key_kind_mw(rsort_key_t k) {
    return (k == RSORT_I32 || k == RSORT_I64) ? rsort::KIND_SINT
           : (k == RSORT_F32 || k == RSORT_F64) ? rsort::KIND_FLOAT
                                                : rsort::KIND_UINT;
}

// Pivot stride S (a power of two) and group G for `runs` runs: one CTA's
// G intervals hold at most (runs + G) * S <= CAP items.
void plan(unsigned runs, int kb, int vb, uint32_t *stride, uint32_t *group) {
    const uint32_t cap = uint32_t(rsort::MW_THREADS) * uint32_t(rsort::mw_items(kb, vb));
    uint32_t s = 1;
    while (s * 2 * 2 * runs <= cap) s *= 2;
    *stride = s;
    *group = runs;
}

uint64_t pivot_count(const size_t *len, unsigned runs, uint32_t stride) {
    uint64_t p = 0;
    for (unsigned t = 0; t < runs; ++t) p += (uint64_t(len[t]) + stride - 1) / stride;
    return p;
}

}  // namespace

extern "C" {

size_t rsort_multiway_scratch_bytes(rsort_key_t key, size_t value_bytes, unsigned runs,
                                    size_t total) {
    if (int(key) < RSORT_U32 || int(key) > RSORT_F64 || runs == 0 ||
        runs > unsigned(rsort::MW_MAX_RUNS))
        return 0;
    uint32_t stride = 0, group = 0;
    plan(runs, key_bytes_mw(key), int(value_bytes), &stride, &group);
    // at most total / S + runs pivots, plus the end row
    const uint64_t rows = uint64_t(total) / stride + runs + 1;
    return size_t(rows * runs * 8);
}

rsort_status rsort_merge_multiway(rsort_key_t key, int descending, unsigned runs,
                                  const void *const *run_keys, const void *const *run_values,
                                  const size_t *run_lengths, size_t value_bytes, void *out_keys,
                                  void *out_values, void *d_scratch, size_t scratch_bytes,
                                  rsort_stream_t stream) {
    if (int(key) < RSORT_U32 || int(key) > RSORT_F64)
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: key type (32/64-bit)");
    if (!(value_bytes == 0 || value_bytes == 1 || value_bytes == 2 || value_bytes == 4 ||
          value_bytes == 8 || value_bytes == 16))
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: value width");
    if (runs == 0 || runs > unsigned(rsort::MW_MAX_RUNS))
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: run count (1..64)");
    if (!run_lengths || !run_keys || (value_bytes && !run_values))
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: null argument");
    uint64_t total = 0;
    for (unsigned t = 0; t < runs; ++t) {
        if (run_lengths[t] && (!run_keys[t] || (value_bytes && !run_values[t])))
            return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: null run");
        total += run_lengths[t];
    }
    if (total == 0) return RSORT_OK;
    if (!out_keys || (value_bytes && !out_values))
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: null output");
    {
        uintptr_t kbits = rsort::addr(out_keys), vbits = rsort::addr(out_values);
        for (unsigned t = 0; t < runs; ++t) {
            kbits |= rsort::addr(run_keys[t]);
            if (value_bytes) vbits |= rsort::addr(run_values[t]);
        }
        rsort_status st = rsort::check_alignment(kbits, size_t(key_bytes_mw(key)),
                                                 "multiway merge: keys alignment");
        if (st == RSORT_OK)
            st = rsort::check_alignment(vbits, value_bytes, "multiway merge: values alignment");
        if (st != RSORT_OK) return st;
    }
    const size_t need = rsort_multiway_scratch_bytes(key, value_bytes, runs, total);
    if (!d_scratch || scratch_bytes < need)
        return record_failure(RSORT_WORKSPACE_TOO_SMALL, "multiway merge scratch", need,
                              scratch_bytes);
    if (reinterpret_cast<uintptr_t>(d_scratch) & 7)
        return record_failure(RSORT_BAD_ARGUMENT, "multiway merge: scratch alignment (8 bytes)");
    int sms = 0;
    rsort_status st = rsort::current_sm_count(&sms);
    if (st != RSORT_OK) return st;
    const int kb = key_bytes_mw(key);
    MultiwayArgs a{};
    plan(runs, kb, int(value_bytes), &a.stride, &a.group);
    a.runs = runs;
    uint64_t acc = 0;
    for (unsigned t = 0; t < runs; ++t) {
        a.keys[t] = run_keys[t];
        a.values[t] = value_bytes ? run_values[t] : nullptr;
        a.len[t] = run_lengths[t];
        a.pivot_start[t] = acc;
        acc += (uint64_t(run_lengths[t]) + a.stride - 1) / a.stride;
    }
    a.pivot_start[runs] = acc;
    a.pivots = pivot_count(run_lengths, runs, a.stride);
    a.table = static_cast<uint64_t *>(d_scratch);
    a.out_keys = out_keys;
    a.out_values = out_values;
    a.kind = key_kind_mw(key);
    a.desc = descending ? 1 : 0;
    if ((a.pivots + 1) / a.group + 1 > 0x7fffffffull)
        return record_failure(RSORT_SIZE_OVERFLOW, "multiway merge: tile count");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        rsort::LaunchScope scope(RSORT_KERNEL_MERGE, s);
        e = rsort::launch_multiway(kb, int(value_bytes), a, s);
    }
    return e == cudaSuccess ? RSORT_OK : record_failure(RSORT_CUDA_ERROR, "multiway merge launch");
}

}  // extern "C"
