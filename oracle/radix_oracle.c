/*
 * CPU restatement of the reference DeviceRadixSort ordering rules.
 * TEST INFRASTRUCTURE ONLY -- see radix_oracle.h.  Nothing in the product
 * library links or calls this file.
 */
#include "radix_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

unsigned orc_key_bytes(int key_type) { return key_type >= ORC_U64 ? 8u : 4u; }
unsigned orc_key_bits(int key_type) { return 8u * orc_key_bytes(key_type); }

static int is_float(int t) { return t == ORC_F32 || t == ORC_F64; }
static int is_signed(int t) { return t == ORC_I32 || t == ORC_I64; }

static uint64_t all_ones(int t) { return orc_key_bits(t) == 64 ? ~0ull : 0xffffffffull; }
static uint64_t sign_bit(int t) { return 1ull << (orc_key_bits(t) - 1); }

/* radix.rs:75-235: uint identity, int flips the sign bit, float flips all
 * bits of negatives and the sign bit of non-negatives; descending is the
 * bitwise NOT of the ascending image. */
uint64_t orc_to_ordered(int t, int descending, uint64_t raw) {
    const uint64_t ones = all_ones(t), sign = sign_bit(t);
    uint64_t o = raw & ones;
    if (is_signed(t)) {
        o ^= sign;
    } else if (is_float(t)) {
        o = (o & sign) ? (~o & ones) : (o ^ sign);
    }
    if (descending) o = ~o & ones;
    return o;
}

uint64_t orc_from_ordered(int t, int descending, uint64_t ordered) {
    const uint64_t ones = all_ones(t), sign = sign_bit(t);
    uint64_t o = ordered & ones;
    if (descending) o = ~o & ones;
    if (is_signed(t)) {
        o ^= sign;
    } else if (is_float(t)) {
        o = (o & sign) ? (o ^ sign) : (~o & ones);
    }
    return o;
}

/* radix.rs:257-337: 0x7fff..ff (the ordered image of one zero) -> 0x8000..00. */
uint64_t orc_fold(int t, uint64_t ordered) {
    if (is_float(t) && ordered == sign_bit(t) - 1) return sign_bit(t);
    return ordered;
}

/* workspace.rs:23-66 (radix_reg_bound with 19 nominal items, 256 threads). */
size_t orc_single_tile_items(unsigned key_bytes, unsigned value_bytes) {
    unsigned item = key_bytes > value_bytes ? key_bytes : value_bytes;
    unsigned divisor = item > 4 ? item : 4;
    unsigned items = 19u * 4u / divisor;
    if (items < 1) items = 1;
    return 256u * (size_t)items;
}

static uint64_t window_mask(unsigned width) {
    return width >= 64 ? ~0ull : ((1ull << width) - 1);
}

/* Onesweep route (ordering_kernels.rs:1309-1314): digits of
 * fold(to_ordered_DIR(key)) over [begin, end), ascending.
 * Single-tile route (ordering_kernels.rs:1229-1234 and
 * ordering_backend/radix.rs:413-420): digits of fold(to_ordered_ascending(key))
 * with the counter lanes reversed for descending, i.e. descending by the
 * ascending-space window. */
uint64_t orc_sort_key(int t, int descending, unsigned begin_bit, unsigned end_bit,
                      int single_tile_route, uint64_t raw) {
    const unsigned width = end_bit - begin_bit;
    const uint64_t mask = window_mask(width);
    if (width == 0) return 0;
    if (single_tile_route) {
        uint64_t w = (orc_fold(t, orc_to_ordered(t, 0, raw)) >> begin_bit) & mask;
        return descending ? (~w & mask) : w;
    }
    return (orc_fold(t, orc_to_ordered(t, descending, raw)) >> begin_bit) & mask;
}

/* ---------------------------------------------------------------------------
 * Stable LSD counting sort of (sort key, index) on host threads.
 * ------------------------------------------------------------------------- */

typedef struct {
    const uint64_t *src_key;
    const uint64_t *src_idx;
    uint64_t *dst_key;
    uint64_t *dst_idx;
    size_t begin, end;
    unsigned shift;
    size_t *hist;   /* 256 entries for this thread */
    int phase;      /* 0 = count, 1 = scatter */
} lsd_job;

static void *lsd_worker(void *arg) {
    lsd_job *j = (lsd_job *)arg;
    if (j->phase == 0) {
        memset(j->hist, 0, 256 * sizeof(size_t));
        for (size_t i = j->begin; i < j->end; ++i) j->hist[(j->src_key[i] >> j->shift) & 0xff]++;
    } else {
        for (size_t i = j->begin; i < j->end; ++i) {
            unsigned d = (unsigned)((j->src_key[i] >> j->shift) & 0xff);
            size_t o = j->hist[d]++;
            j->dst_key[o] = j->src_key[i];
            j->dst_idx[o] = j->src_idx[i];
        }
    }
    return NULL;
}

static void run_jobs(lsd_job *jobs, int threads) {
    if (threads == 1) {
        lsd_worker(&jobs[0]);
        return;
    }
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    for (int t = 0; t < threads; ++t) pthread_create(&tid[t], NULL, lsd_worker, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
}

void orc_stable_order(const uint64_t *sort_keys, size_t n, unsigned key_bits, int threads,
                      uint64_t *perm) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > n / 65536 + 1) threads = (int)(n / 65536 + 1);
    uint64_t *ka = (uint64_t *)malloc(sizeof(uint64_t) * (n ? n : 1));
    uint64_t *kb = (uint64_t *)malloc(sizeof(uint64_t) * (n ? n : 1));
    uint64_t *ib = (uint64_t *)malloc(sizeof(uint64_t) * (n ? n : 1));
    uint64_t *ia = perm;
    memcpy(ka, sort_keys, sizeof(uint64_t) * n);
    for (size_t i = 0; i < n; ++i) ia[i] = i;
    lsd_job *jobs = (lsd_job *)calloc((size_t)threads, sizeof(lsd_job));
    size_t *hist = (size_t *)calloc((size_t)threads * 256, sizeof(size_t));
    for (unsigned shift = 0; shift < key_bits; shift += 8) {
        for (int t = 0; t < threads; ++t) {
            jobs[t].src_key = ka; jobs[t].src_idx = ia;
            jobs[t].dst_key = kb; jobs[t].dst_idx = ib;
            jobs[t].begin = n * (size_t)t / (size_t)threads;
            jobs[t].end = n * (size_t)(t + 1) / (size_t)threads;
            jobs[t].shift = shift;
            jobs[t].hist = hist + 256 * (size_t)t;
            jobs[t].phase = 0;
        }
        run_jobs(jobs, threads);
        /* A digit shared by every key leaves the order unchanged: skip. */
        int trivial = 0;
        for (unsigned d = 0; d < 256 && !trivial; ++d) {
            size_t total = 0;
            for (int t = 0; t < threads; ++t) total += hist[256 * (size_t)t + d];
            if (total == n) trivial = 1;
        }
        if (trivial) continue;
        size_t running = 0;
        for (unsigned d = 0; d < 256; ++d) {
            for (int t = 0; t < threads; ++t) {
                size_t c = hist[256 * (size_t)t + d];
                hist[256 * (size_t)t + d] = running;
                running += c;
            }
        }
        for (int t = 0; t < threads; ++t) jobs[t].phase = 1;
        run_jobs(jobs, threads);
        uint64_t *tk = ka; ka = kb; kb = tk;
        uint64_t *ti = ia; ia = ib; ib = ti;
    }
    if (ia != perm) {
        memcpy(perm, ia, sizeof(uint64_t) * n);
        ib = ia;
    }
    free(ka); free(kb); free(ib); free(jobs); free(hist);
}

static uint64_t load_key(const void *keys, unsigned kb, size_t i) {
    if (kb == 4) return ((const uint32_t *)keys)[i];
    return ((const uint64_t *)keys)[i];
}

int orc_radix_sort(int t, int descending, void *keys, void *values, size_t n,
                   unsigned value_bytes, unsigned begin_bit, unsigned end_bit, int threads,
                   int *swaps) {
    const unsigned kb = orc_key_bytes(t), bits = orc_key_bits(t);
    if (swaps) *swaps = 0;
    if (t < ORC_U32 || t > ORC_F64) return ORC_BAD_ARGUMENT;
    /* radix.rs:370-376 */
    if (begin_bit > end_bit || end_bit > bits) return ORC_INVALID_BIT_RANGE;
    const unsigned passes = (end_bit - begin_bit + 7) / 8;
    /* radix.rs:467-469 */
    if (n == 0 || passes == 0) return ORC_OK;
    const int single = n <= orc_single_tile_items(kb, value_bytes);
    uint64_t *sk = (uint64_t *)malloc(sizeof(uint64_t) * n);
    uint64_t *perm = (uint64_t *)malloc(sizeof(uint64_t) * n);
    for (size_t i = 0; i < n; ++i)
        sk[i] = orc_sort_key(t, descending, begin_bit, end_bit, single, load_key(keys, kb, i));
    orc_stable_order(sk, n, end_bit - begin_bit, threads, perm);
    unsigned char *tmp = (unsigned char *)malloc(n * (kb > value_bytes ? kb : value_bytes));
    for (size_t i = 0; i < n; ++i)
        memcpy(tmp + i * kb, (const unsigned char *)keys + perm[i] * kb, kb);
    memcpy(keys, tmp, n * kb);
    if (value_bytes && values) {
        for (size_t i = 0; i < n; ++i)
            memcpy(tmp + i * value_bytes, (const unsigned char *)values + perm[i] * value_bytes,
                   value_bytes);
        memcpy(values, tmp, n * value_bytes);
    }
    free(tmp); free(perm); free(sk);
    /* radix.rs:470-492 (one swap) and :518-552 (one swap per pass). */
    if (swaps) *swaps = single ? 1 : (int)passes;
    return ORC_OK;
}

/* ---------------------------------------------------------------------------
 * Sample-sort partition restatement (rccl_b200 multi-GPU path; no reference
 * counterpart).  Elements are ordered by the composite (sort key, rank,
 * position in the rank's locally sorted shard), which equals the global
 * stable order because shards are contiguous slices of the input.
 * ------------------------------------------------------------------------- */

typedef struct { uint64_t key; uint64_t rank; uint64_t idx; } composite;

static int composite_less(const composite *a, const composite *b) {
    if (a->key != b->key) return a->key < b->key;
    if (a->rank != b->rank) return a->rank < b->rank;
    return a->idx < b->idx;
}

static int composite_cmp(const void *pa, const void *pb) {
    const composite *a = (const composite *)pa, *b = (const composite *)pb;
    if (composite_less(a, b)) return -1;
    if (composite_less(b, a)) return 1;
    return 0;
}

int orc_sample_partition(int t, int descending, const void *keys, const size_t *shard_sizes,
                         int world, unsigned samples_per_rank, int threads, size_t *out_counts) {
    const unsigned kb = orc_key_bytes(t), bits = orc_key_bits(t);
    if (world < 1 || samples_per_rank < 1) return ORC_BAD_ARGUMENT;
    const size_t S = samples_per_rank;
    composite *samples = (composite *)malloc(sizeof(composite) * S * (size_t)world);
    uint64_t **sorted_keys = (uint64_t **)calloc((size_t)world, sizeof(uint64_t *));
    size_t valid = 0, offset = 0;
    for (int r = 0; r < world; ++r) {
        const size_t m = shard_sizes[r];
        uint64_t *sk = (uint64_t *)malloc(sizeof(uint64_t) * (m ? m : 1));
        uint64_t *perm = (uint64_t *)malloc(sizeof(uint64_t) * (m ? m : 1));
        for (size_t i = 0; i < m; ++i)
            sk[i] = orc_sort_key(t, descending, 0, bits, 0, load_key(keys, kb, offset + i));
        orc_stable_order(sk, m, bits, threads, perm);
        uint64_t *sorted = (uint64_t *)malloc(sizeof(uint64_t) * (m ? m : 1));
        for (size_t i = 0; i < m; ++i) sorted[i] = sk[perm[i]];
        sorted_keys[r] = sorted;
        free(sk); free(perm);
        /* Regular samples at floor((i+1) * m / (S+1)) of the sorted shard. */
        if (m > 0) {
            for (size_t i = 0; i < S; ++i) {
                size_t p = (size_t)(((unsigned __int128)(i + 1) * m) / (S + 1));
                composite c = {sorted[p], (uint64_t)r, (uint64_t)p};
                samples[valid++] = c;
            }
        }
        offset += m;
    }
    qsort(samples, valid, sizeof(composite), composite_cmp);
    /* Splitter j (1 <= j < world) is sample floor(j * valid / world). */
    for (int q = 0; q < world; ++q) out_counts[q] = 0;
    for (int r = 0; r < world; ++r) {
        const size_t m = shard_sizes[r];
        size_t prev = 0;
        for (int j = 1; j <= world; ++j) {
            size_t bound = m;
            if (j < world && valid > 0) {
                const composite *sp = &samples[(size_t)j * valid / (size_t)world];
                /* lower bound: first local i with (key_i, r, i) >= splitter */
                size_t lo = 0, hi = m;
                while (lo < hi) {
                    size_t mid = lo + (hi - lo) / 2;
                    composite c = {sorted_keys[r][mid], (uint64_t)r, (uint64_t)mid};
                    if (composite_less(&c, sp)) lo = mid + 1; else hi = mid;
                }
                bound = lo;
            } else if (j < world) {
                bound = 0;
            }
            out_counts[j - 1] += bound - prev;
            prev = bound;
        }
    }
    for (int r = 0; r < world; ++r) free(sorted_keys[r]);
    free(sorted_keys);
    free(samples);
    return ORC_OK;
}
