// The whole multi-GPU sample sort behind one C call: rsort_dist_pairs (one
// host thread drives every GPU) and rsort_dist_pairs_rank (one process or
// thread per GPU).  No reference counterpart: the reference is single-GPU.
//
// Per rank:  local stable sort -> S regular samples -> NCCL all-gather ->
// W-1 splitters -> W+1 bucket bounds -> NCCL all-gather of the bounds ->
// (host reads the bounds: the receive sizes are data dependent) -> bucket
// exchange (grouped ncclSend/ncclRecv, or a copy kernel reading the peers'
// shards) -> stable merge of the W received runs.  Every device step is one
// of the library's own kernels; NCCL moves the samples, bounds and buckets.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/rsort_b200.h"
#include "rsort_internal.cuh"

namespace {

using rsort::record_failure;

// ---------------------------------------------------------------------------
// NCCL entry points, resolved at run time from the NCCL library already in
// the process (the caller created its communicators with it), else from
// libnccl.so.2 on the library path.
// ---------------------------------------------------------------------------
struct Nccl {
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
                         cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int *) = nullptr;
    bool ok = false;
};

std::once_flag g_nccl_once;
Nccl g_nccl;

const Nccl &nccl() {
    std::call_once(g_nccl_once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW);
        if (!h) return;
        Nccl n;
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
        n.send = reinterpret_cast<decltype(n.send)>(dlsym(h, "ncclSend"));
        n.recv = reinterpret_cast<decltype(n.recv)>(dlsym(h, "ncclRecv"));
        n.group_start = reinterpret_cast<decltype(n.group_start)>(dlsym(h, "ncclGroupStart"));
        n.group_end = reinterpret_cast<decltype(n.group_end)>(dlsym(h, "ncclGroupEnd"));
        n.comm_count = reinterpret_cast<decltype(n.comm_count)>(dlsym(h, "ncclCommCount"));
        n.comm_user_rank =
            reinterpret_cast<decltype(n.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
        n.ok = n.all_gather && n.send && n.recv && n.group_start && n.group_end && n.comm_count &&
               n.comm_user_rank;
        g_nccl = n;
    });
    return g_nccl;
}

rsort_status nccl_fail(ncclResult_t r, const char *role) {
    (void)r;
    return record_failure(RSORT_CUDA_ERROR, role);
}

// Regular samples per rank: 64 * W, capped so the world's sample set fits the
// one-CTA splitter kernel (RSORT_MAX_SPLITTER_SAMPLES).
unsigned samples_per_rank(unsigned world) {
    const unsigned cap = RSORT_MAX_SPLITTER_SAMPLES / world;
    const unsigned s = 64u * world < cap ? 64u * world : cap;
    return s ? s : 1u;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int key_bytes_of(rsort_key_t k) {
    return (k == RSORT_U64 || k == RSORT_I64 || k == RSORT_F64) ? 8 : 4;
}
bool wide_key(rsort_key_t k) { return int(k) >= RSORT_U32 && int(k) <= RSORT_F64; }
bool value_ok(size_t vb) { return vb == 0 || vb == 1 || vb == 2 || vb == 4 || vb == 8 || vb == 16; }

// Byte offsets of the regions of one rank's scratch.
struct Layout {
    // sort_keys / sort_values: the local sort's scratch, then the received
    // runs; parts: the merge-path partitions (nparts words)
    size_t sort_keys, sort_values, bins, lookback, counters, samples, gathered, splitters,
        bounds, all_bounds, parts, total;
    rsort_controls controls;
    size_t nparts;
    unsigned S;
};

bool layout(rsort_key_t key, size_t vb, size_t n_local, size_t cap, unsigned world, Layout *L) {
    if (!wide_key(key) || !value_ok(vb) || world == 0) return false;
    rsort_controls c{};
    if (rsort_controls_query(key, vb, n_local, &c) != RSORT_OK) return false;
    const size_t kb = size_t(key_bytes_of(key));
    const size_t items = n_local > cap ? n_local : cap;
    const unsigned S = samples_per_rank(world);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    L->sort_keys = take(items * kb);
    L->sort_values = take(items * vb);
    L->bins = take(8 * c.bins);
    L->lookback = take(4 * c.lookback);
    L->counters = take(4 * c.counters);
    L->samples = take(size_t(S) * RSORT_COMPOSITE_BYTES);
    L->gathered = take(size_t(S) * world * RSORT_COMPOSITE_BYTES);
    L->splitters = take(size_t(world > 1 ? world - 1 : 1) * RSORT_COMPOSITE_BYTES);
    L->bounds = take(8 * size_t(world + 2));
    L->all_bounds = take(8 * size_t(world + 2) * world);
    L->nparts = rsort_merge_partition_words(cap);
    L->parts = take(8 * (L->nparts ? L->nparts : 1));
    L->total = off;
    L->controls = c;
    L->S = S;
    return true;
}

// One rank's view of the call.
struct Rank {
    int rank = 0;
    int device = 0;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    char *keys = nullptr, *values = nullptr;
    size_t n = 0;
    char *out_keys = nullptr, *out_values = nullptr;
    size_t cap = 0;
    char *scratch = nullptr;
    Layout L{};
    std::vector<size_t> recv;  // items received from each rank
    std::vector<size_t> send_start;  // first item of the bucket sent to each rank
    size_t n_out = 0;
    uint64_t cap_word = 0;  // host copy of cap, gathered with the bounds
};

// The receive area of the exchange: the local sort's scratch, free again.
char *recv_keys(Rank &r) { return r.scratch + r.L.sort_keys; }
char *recv_values(Rank &r) { return r.scratch + r.L.sort_values; }

// Step 1: local stable sort in place, then this rank's regular samples.
rsort_status local_sort_and_samples(rsort_key_t key, int desc, size_t vb, unsigned world,
                                    Rank &r) {
    cudaStream_t s = r.stream;
    rsort_stream_t rs = reinterpret_cast<rsort_stream_t>(s);
    const Layout &L = r.L;
    uint64_t *bins = L.controls.bins ? reinterpret_cast<uint64_t *>(r.scratch + L.bins) : nullptr;
    int32_t *lb = L.controls.lookback ? reinterpret_cast<int32_t *>(r.scratch + L.lookback) : nullptr;
    int32_t *ctr = L.controls.counters ? reinterpret_cast<int32_t *>(r.scratch + L.counters) : nullptr;
    if (ctr && cudaMemsetAsync(ctr, 0, 4 * L.controls.counters, s) != cudaSuccess)
        return record_failure(RSORT_CUDA_ERROR, "dist sort: counters reset");
    rsort_status st;
    if (vb == 0)
        st = rsort_keys(key, desc, r.keys, r.scratch + L.sort_keys, r.n, r.n, bins,
                        L.controls.bins, lb, L.controls.lookback, ctr, L.controls.counters, rs);
    else
        st = rsort_pairs(key, desc, r.keys, r.values, vb, r.scratch + L.sort_keys, r.n,
                         r.scratch + L.sort_values, r.n, r.n, bins, L.controls.bins, lb,
                         L.controls.lookback, ctr, L.controls.counters, rs);
    if (st != RSORT_OK) return st;
    return rsort_dist_samples(key, desc, r.keys, r.n, unsigned(r.rank), L.S,
                              r.scratch + L.samples, rs);
}

rsort_status all_gather_samples(const Nccl &nc, Rank &r) {
    const size_t bytes = size_t(r.L.S) * RSORT_COMPOSITE_BYTES;
    const ncclResult_t e = nc.all_gather(r.scratch + r.L.samples, r.scratch + r.L.gathered, bytes,
                                         ncclUint8, r.comm, r.stream);
    return e == ncclSuccess ? RSORT_OK : nccl_fail(e, "dist sort: sample all-gather");
}

// Step 2: splitters from the gathered samples, then this rank's bucket bounds.
// The record each rank contributes to the second all-gather is its W+1
// bounds followed by its output capacity, so every rank learns whether every
// part fits and all ranks take the same branch.
rsort_status partition(rsort_key_t key, int desc, unsigned world, Rank &r) {
    rsort_stream_t rs = reinterpret_cast<rsort_stream_t>(r.stream);
    rsort_status st = rsort_dist_splitters(r.scratch + r.L.gathered, size_t(r.L.S) * world, world,
                                           r.scratch + r.L.splitters, rs);
    if (st != RSORT_OK) return st;
    st = rsort_dist_bounds(key, desc, r.keys, r.n, unsigned(r.rank), r.scratch + r.L.splitters,
                           world, reinterpret_cast<uint64_t *>(r.scratch + r.L.bounds), rs);
    if (st != RSORT_OK) return st;
    r.cap_word = uint64_t(r.cap);
    if (cudaMemcpyAsync(r.scratch + r.L.bounds + 8 * size_t(world + 1), &r.cap_word, 8,
                        cudaMemcpyHostToDevice, r.stream) != cudaSuccess)
        return record_failure(RSORT_CUDA_ERROR, "dist sort: capacity word");
    return RSORT_OK;
}

rsort_status all_gather_bounds(const Nccl &nc, unsigned world, Rank &r) {
    const ncclResult_t e = nc.all_gather(r.scratch + r.L.bounds, r.scratch + r.L.all_bounds,
                                         8 * size_t(world + 2), ncclUint8, r.comm, r.stream);
    return e == ncclSuccess ? RSORT_OK : nccl_fail(e, "dist sort: bounds all-gather");
}

// Host read of the gathered records (row q = rank q's W+1 bounds and its
// output capacity), then this rank's receive sizes and send starts.
rsort_status read_bounds(unsigned world, Rank &r, std::vector<uint64_t> *table) {
    table->assign(size_t(world) * (world + 2), 0);
    cudaError_t e = cudaMemcpyAsync(table->data(), r.scratch + r.L.all_bounds,
                                    8 * table->size(), cudaMemcpyDeviceToHost, r.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(r.stream);
    if (e != cudaSuccess) return record_failure(RSORT_CUDA_ERROR, "dist sort: bounds read");
    return RSORT_OK;
}

constexpr size_t row_words(unsigned world) { return size_t(world) + 2; }

// Whether every rank's part fits its capacity (same answer on every rank).
bool all_fit(unsigned world, const std::vector<uint64_t> &t) {
    for (unsigned r = 0; r < world; ++r) {
        uint64_t got = 0;
        for (unsigned q = 0; q < world; ++q)
            got += t[q * row_words(world) + r + 1] - t[q * row_words(world) + r];
        if (got > t[r * row_words(world) + world + 1]) return false;
    }
    return true;
}

void plan_from_table(unsigned world, const std::vector<uint64_t> &t, Rank &r) {
    auto row = [&](unsigned q) { return &t[size_t(q) * row_words(world)]; };
    r.recv.assign(world, 0);
    r.send_start.assign(world + 1, 0);
    r.n_out = 0;
    for (unsigned q = 0; q < world; ++q) {
        r.recv[q] = size_t(row(q)[r.rank + 1] - row(q)[r.rank]);
        r.n_out += r.recv[q];
    }
    for (unsigned q = 0; q <= world; ++q) r.send_start[q] = size_t(row(unsigned(r.rank))[q]);
}

// Step 3 (NCCL): the bucket a rank keeps is a device copy, issued before the
// NCCL group so that the group holds nothing but NCCL calls.
rsort_status exchange_keep(size_t kb, size_t vb, unsigned world, Rank &r) {
    size_t roff = 0;
    for (unsigned q = 0; q < unsigned(r.rank); ++q) roff += r.recv[q];
    const size_t keep = r.send_start[r.rank + 1] - r.send_start[r.rank];
    const size_t so = r.send_start[r.rank];
    (void)world;
    if (!keep) return RSORT_OK;
    cudaError_t e = cudaMemcpyAsync(recv_keys(r) + roff * kb, r.keys + so * kb, keep * kb,
                                    cudaMemcpyDeviceToDevice, r.stream);
    if (e == cudaSuccess && vb)
        e = cudaMemcpyAsync(recv_values(r) + roff * vb, r.values + so * vb, keep * vb,
                            cudaMemcpyDeviceToDevice, r.stream);
    return e == cudaSuccess ? RSORT_OK
                            : record_failure(RSORT_CUDA_ERROR, "dist sort: local bucket copy");
}

// This rank's sends and receives (keys, then values, per peer); must be
// issued inside an NCCL group (the caller's).
rsort_status exchange_nccl(const Nccl &nc, size_t kb, size_t vb, unsigned world, Rank &r) {
    size_t roff = 0;
    for (unsigned q = 0; q < world; ++q) {
        const size_t send = r.send_start[q + 1] - r.send_start[q];
        const size_t so = r.send_start[q];
        if (int(q) != r.rank) {
            ncclResult_t e = ncclSuccess;
            if (send) {
                e = nc.send(r.keys + so * kb, send * kb, ncclUint8, int(q), r.comm, r.stream);
                if (e == ncclSuccess && vb)
                    e = nc.send(r.values + so * vb, send * vb, ncclUint8, int(q), r.comm,
                                r.stream);
            }
            if (e == ncclSuccess && r.recv[q]) {
                e = nc.recv(recv_keys(r) + roff * kb, r.recv[q] * kb, ncclUint8, int(q), r.comm,
                            r.stream);
                if (e == ncclSuccess && vb)
                    e = nc.recv(recv_values(r) + roff * vb, r.recv[q] * vb, ncclUint8, int(q),
                                r.comm, r.stream);
            }
            if (e != ncclSuccess) return nccl_fail(e, "dist sort: bucket send/recv");
        }
        roff += r.recv[q];
    }
    return RSORT_OK;
}

// Step 3 (peer): one copy kernel per array pulls rank r's bucket out of every
// rank's sorted shard (peer memory over NVLink, the own shard from HBM).
rsort_status exchange_peer(size_t kb, size_t vb, unsigned world, std::vector<Rank> &ranks,
                           const std::vector<uint64_t> &table, Rank &r) {
    auto row = [&](unsigned q) { return &table[size_t(q) * row_words(world)]; };
    for (int which = 0; which < (vb ? 2 : 1); ++which) {
        const size_t w = which ? vb : kb;
        std::vector<const void *> src(world);
        std::vector<uint64_t> bytes(world);
        for (unsigned q = 0; q < world; ++q) {
            const size_t start = size_t(row(q)[r.rank]);
            bytes[q] = uint64_t(r.recv[q] * w);
            src[q] = bytes[q] ? (which ? ranks[q].values : ranks[q].keys) + start * w : nullptr;
        }
        const rsort_status st = rsort_gather_segments(world, src.data(), bytes.data(),
                                                      which ? recv_values(r) : recv_keys(r),
                                                      reinterpret_cast<rsort_stream_t>(r.stream));
        if (st != RSORT_OK) return st;
    }
    return RSORT_OK;
}

// Step 4: stable merge of the received runs (back to back in the receive
// area, in source-rank order; ties keep the lower rank) into the output:
// pairwise merge-path rounds between the receive area and the output, the
// last round landing in the output (one copy when the run count makes the
// rounds end in the receive area).  Measured faster on B200 than one W-way
// pass (rsort_merge_multiway) for these local runs.
rsort_status merge_received(rsort_key_t key, int desc, size_t kb, size_t vb, unsigned world,
                            Rank &r) {
    (void)world;
    if (r.n_out == 0) return RSORT_OK;
    rsort_stream_t rs = reinterpret_cast<rsort_stream_t>(r.stream);
    int in_scratch = 0;
    rsort_status st = rsort_merge_runs(
        key, desc, recv_keys(r), vb ? recv_values(r) : nullptr, vb, r.recv.data(), world,
        r.out_keys, vb ? r.out_values : nullptr, reinterpret_cast<uint64_t *>(r.scratch + r.L.parts),
        r.L.nparts, &in_scratch, rs);
    if (st != RSORT_OK) return st;
    if (!in_scratch) {  // the result is in the receive area
        cudaError_t e = cudaMemcpyAsync(r.out_keys, recv_keys(r), r.n_out * kb,
                                        cudaMemcpyDeviceToDevice, r.stream);
        if (e == cudaSuccess && vb)
            e = cudaMemcpyAsync(r.out_values, recv_values(r), r.n_out * vb,
                                cudaMemcpyDeviceToDevice, r.stream);
        if (e != cudaSuccess) return record_failure(RSORT_CUDA_ERROR, "dist sort: merge copy");
    }
    return RSORT_OK;
}

rsort_status check_rank_args(rsort_key_t key, size_t vb, const Rank &r, size_t scratch_bytes,
                             unsigned world) {
    if (!r.comm || (r.n && !r.keys) || (vb && r.n && !r.values) || (r.cap && !r.out_keys) ||
        (vb && r.cap && !r.out_values))
        return record_failure(RSORT_BAD_ARGUMENT, "dist sort: null buffer or communicator");
    if (r.n >= (size_t(1) << 40))
        return record_failure(RSORT_SIZE_OVERFLOW, "dist sort: shard size (2^40 items)");
    if (reinterpret_cast<uintptr_t>(r.scratch) & 255)
        return record_failure(RSORT_BAD_ARGUMENT, "dist sort: scratch alignment (256 bytes)");
    const size_t need = rsort_dist_scratch_bytes(key, vb, r.n, r.cap, world);
    if (!r.scratch || scratch_bytes < need)
        return record_failure(RSORT_WORKSPACE_TOO_SMALL, "dist sort scratch", need, scratch_bytes);
    return RSORT_OK;
}

rsort_status check_comm(const Nccl &nc, ncclComm_t comm, int rank, int world) {
    int count = 0, user = -1;
    if (nc.comm_count(comm, &count) != ncclSuccess || nc.comm_user_rank(comm, &user) != ncclSuccess)
        return record_failure(RSORT_CUDA_ERROR, "dist sort: communicator query");
    if (count != world || user != rank)
        return record_failure(RSORT_BAD_ARGUMENT,
                              "dist sort: communicator rank/size differ from rank/world");
    return RSORT_OK;
}

struct DeviceGuard {
    int saved = -1;
    DeviceGuard() { cudaGetDevice(&saved); }
    ~DeviceGuard() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};

}  // namespace

extern "C" {

size_t rsort_dist_scratch_bytes(rsort_key_t key, size_t value_bytes, size_t n_local,
                                size_t out_capacity, unsigned world) {
    Layout L{};
    return layout(key, value_bytes, n_local, out_capacity, world, &L) ? L.total : 0;
}

rsort_status rsort_dist_pairs(rsort_key_t key, int descending, size_t value_bytes, int world,
                              const int *devices, rsort_nccl_comm_t const *comms,
                              rsort_stream_t const *streams, void *const *d_keys,
                              void *const *d_values, const size_t *n_local,
                              void *const *d_out_keys, void *const *d_out_values,
                              const size_t *out_capacity, void *const *d_scratch,
                              const size_t *scratch_bytes, rsort_exchange_t exchange,
                              size_t *n_out) {
    if (!wide_key(key)) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: key type (32/64-bit)");
    if (!value_ok(value_bytes)) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: value width");
    if (world < 1 || world > 64) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: world size");
    if (exchange != RSORT_EXCHANGE_NCCL && exchange != RSORT_EXCHANGE_PEER)
        return record_failure(RSORT_BAD_ARGUMENT, "dist sort: exchange mode");
    if (!devices || !comms || !streams || !d_keys || !n_local || !d_out_keys || !out_capacity ||
        !d_scratch || !scratch_bytes || !n_out || (value_bytes && (!d_values || !d_out_values)))
        return record_failure(RSORT_BAD_ARGUMENT, "dist sort: null argument array");
    const unsigned W = unsigned(world);
    const size_t kb = size_t(key_bytes_of(key)), vb = value_bytes;
    std::vector<Rank> ranks(W);
    for (unsigned q = 0; q < W; ++q) {
        Rank &r = ranks[q];
        r.rank = int(q);
        r.device = devices[q];
        r.comm = reinterpret_cast<ncclComm_t>(comms[q]);
        r.stream = reinterpret_cast<cudaStream_t>(streams[q]);
        r.keys = static_cast<char *>(d_keys[q]);
        r.values = vb ? static_cast<char *>(d_values[q]) : nullptr;
        r.n = n_local[q];
        r.out_keys = static_cast<char *>(d_out_keys[q]);
        r.out_values = vb ? static_cast<char *>(d_out_values[q]) : nullptr;
        r.cap = out_capacity[q];
        r.scratch = static_cast<char *>(d_scratch[q]);
        rsort_status st = check_rank_args(key, vb, r, scratch_bytes[q], W);
        if (st != RSORT_OK) return st;
        layout(key, vb, r.n, r.cap, W, &r.L);
        n_out[q] = 0;
    }
    const Nccl &nc = nccl();
    if (!nc.ok) return record_failure(RSORT_UNSUPPORTED_TARGET, "dist sort: NCCL library not found");
    for (unsigned q = 0; q < W; ++q) {
        rsort_status st = check_comm(nc, ranks[q].comm, int(q), world);
        if (st != RSORT_OK) return st;
    }
    DeviceGuard guard;
    auto on = [&](Rank &r) {
        return cudaSetDevice(r.device) == cudaSuccess
                   ? RSORT_OK
                   : record_failure(RSORT_CUDA_ERROR, "dist sort: cudaSetDevice");
    };
    // Peer exchange needs every pair of devices to reach each other.
    bool peer = exchange == RSORT_EXCHANGE_PEER && W > 1;
    for (unsigned a = 0; peer && a < W; ++a) {
        for (unsigned b = 0; peer && b < W; ++b) {
            if (a == b || ranks[a].device == ranks[b].device) continue;
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, ranks[a].device, ranks[b].device) != cudaSuccess ||
                !can) {
                peer = false;
                break;
            }
            if (on(ranks[a]) != RSORT_OK) return RSORT_CUDA_ERROR;
            const cudaError_t e = cudaDeviceEnablePeerAccess(ranks[b].device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) return record_failure(RSORT_CUDA_ERROR, "dist sort: peer access");
        }
    }

    rsort_status st = RSORT_OK;
    for (auto &r : ranks) {
        if ((st = on(r)) != RSORT_OK) return st;
        if ((st = local_sort_and_samples(key, descending, vb, W, r)) != RSORT_OK) return st;
    }
    if (nc.group_start() != ncclSuccess) return nccl_fail(ncclSystemError, "dist sort: group");
    for (auto &r : ranks) {
        if ((st = on(r)) != RSORT_OK || (st = all_gather_samples(nc, r)) != RSORT_OK) break;
    }
    if (nc.group_end() != ncclSuccess && st == RSORT_OK)
        st = nccl_fail(ncclSystemError, "dist sort: sample all-gather group");
    if (st != RSORT_OK) return st;
    for (auto &r : ranks) {
        if ((st = on(r)) != RSORT_OK) return st;
        if ((st = partition(key, descending, W, r)) != RSORT_OK) return st;
    }
    if (nc.group_start() != ncclSuccess) return nccl_fail(ncclSystemError, "dist sort: group");
    for (auto &r : ranks) {
        if ((st = on(r)) != RSORT_OK || (st = all_gather_bounds(nc, W, r)) != RSORT_OK) break;
    }
    if (nc.group_end() != ncclSuccess && st == RSORT_OK)
        st = nccl_fail(ncclSystemError, "dist sort: bounds all-gather group");
    if (st != RSORT_OK) return st;
    // Every rank gathered the same table; rank 0's copy plans them all.
    std::vector<uint64_t> table;
    if ((st = on(ranks[0])) != RSORT_OK) return st;
    if ((st = read_bounds(W, ranks[0], &table)) != RSORT_OK) return st;
    for (auto &r : ranks) {
        plan_from_table(W, table, r);
        n_out[r.rank] = r.n_out;
    }
    if (!all_fit(W, table)) {
        for (auto &r : ranks)
            if (r.n_out > r.cap)
                return record_failure(RSORT_WORKSPACE_TOO_SMALL, "dist sort output", r.n_out, r.cap);
    }
    if (peer) {
        for (auto &r : ranks) {
            if ((st = on(r)) != RSORT_OK) return st;
            if ((st = exchange_peer(kb, vb, W, ranks, table, r)) != RSORT_OK) return st;
        }
    } else {
        for (auto &r : ranks) {
            if ((st = on(r)) != RSORT_OK) return st;
            if ((st = exchange_keep(kb, vb, W, r)) != RSORT_OK) return st;
        }
        if (nc.group_start() != ncclSuccess) return nccl_fail(ncclSystemError, "dist sort: group");
        for (auto &r : ranks) {
            if ((st = on(r)) != RSORT_OK || (st = exchange_nccl(nc, kb, vb, W, r)) != RSORT_OK)
                break;
        }
        if (nc.group_end() != ncclSuccess && st == RSORT_OK)
            st = nccl_fail(ncclSystemError, "dist sort: exchange group");
        if (st != RSORT_OK) return st;
    }
    for (auto &r : ranks) {
        if ((st = on(r)) != RSORT_OK) return st;
        if ((st = merge_received(key, descending, kb, vb, W, r)) != RSORT_OK) return st;
    }
    if (peer) {
        // The copy kernels read the peers' shards: none may outlive the call.
        for (auto &r : ranks) {
            if ((st = on(r)) != RSORT_OK) return st;
            if (cudaStreamSynchronize(r.stream) != cudaSuccess)
                return record_failure(RSORT_CUDA_ERROR, "dist sort: stream synchronize");
        }
    }
    return RSORT_OK;
}

rsort_status rsort_dist_pairs_rank(rsort_key_t key, int descending, size_t value_bytes,
                                   int rank, int world, rsort_nccl_comm_t comm,
                                   rsort_stream_t stream, void *d_keys, void *d_values,
                                   size_t n_local, void *d_out_keys, void *d_out_values,
                                   size_t out_capacity, void *d_scratch, size_t scratch_bytes,
                                   size_t *n_out) {
    if (!wide_key(key)) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: key type (32/64-bit)");
    if (!value_ok(value_bytes)) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: value width");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return record_failure(RSORT_BAD_ARGUMENT, "dist sort: rank / world size");
    if (!n_out) return record_failure(RSORT_BAD_ARGUMENT, "dist sort: null n_out");
    const unsigned W = unsigned(world);
    const size_t kb = size_t(key_bytes_of(key)), vb = value_bytes;
    Rank r;
    r.rank = rank;
    r.comm = reinterpret_cast<ncclComm_t>(comm);
    r.stream = reinterpret_cast<cudaStream_t>(stream);
    r.keys = static_cast<char *>(d_keys);
    r.values = vb ? static_cast<char *>(d_values) : nullptr;
    r.n = n_local;
    r.out_keys = static_cast<char *>(d_out_keys);
    r.out_values = vb ? static_cast<char *>(d_out_values) : nullptr;
    r.cap = out_capacity;
    r.scratch = static_cast<char *>(d_scratch);
    *n_out = 0;
    rsort_status st = check_rank_args(key, vb, r, scratch_bytes, W);
    if (st != RSORT_OK) return st;
    layout(key, vb, r.n, r.cap, W, &r.L);
    const Nccl &nc = nccl();
    if (!nc.ok) return record_failure(RSORT_UNSUPPORTED_TARGET, "dist sort: NCCL library not found");
    if ((st = check_comm(nc, r.comm, rank, world)) != RSORT_OK) return st;
    if ((st = local_sort_and_samples(key, descending, vb, W, r)) != RSORT_OK) return st;
    if ((st = all_gather_samples(nc, r)) != RSORT_OK) return st;
    if ((st = partition(key, descending, W, r)) != RSORT_OK) return st;
    if ((st = all_gather_bounds(nc, W, r)) != RSORT_OK) return st;
    std::vector<uint64_t> table;
    if ((st = read_bounds(W, r, &table)) != RSORT_OK) return st;
    plan_from_table(W, table, r);
    *n_out = r.n_out;
    // Every rank holds the same table, so when any part does not fit every
    // rank returns here and none is left waiting in the exchange.
    if (!all_fit(W, table))
        return record_failure(RSORT_WORKSPACE_TOO_SMALL, "dist sort output (some rank)", r.n_out,
                              r.cap);
    if ((st = exchange_keep(kb, vb, W, r)) != RSORT_OK) return st;
    if (nc.group_start() != ncclSuccess) return nccl_fail(ncclSystemError, "dist sort: group");
    st = exchange_nccl(nc, kb, vb, W, r);
    if (nc.group_end() != ncclSuccess && st == RSORT_OK)
        st = nccl_fail(ncclSystemError, "dist sort: exchange group");
    if (st != RSORT_OK) return st;
    return merge_received(key, descending, kb, vb, W, r);
}

}  // extern "C"
