// stream_cache.cpp -- an expert pool in pinned host memory streamed into a
// device cache (the oversubscribed configuration: more expert bytes than HBM).
//
// Reference: the tier lookup of wisp_expert_fetch (csrc/core/wisp_engine.c
// :891-1078) -- a VRAM LRU in front of a RAM tier -- and the transfer stream
// of the engine (wisp_engine.h:411-412).  The reference fills a miss with a
// synchronous copy per fetch; here a miss is one cudaMemcpyAsync of the tiled
// blob straight from the pinned pool into its cache slot, on one of two
// transfer streams used in turn, and the ordering is carried by events
// instead of host synchronisation:
//   * compute waits for the copies of the experts a layer routed (ensure);
//   * a copy into a slot waits for the last kernels that read the slot's
//     previous expert (layer_done records that point on the compute stream);
//   * prefetch starts copies for experts predicted for the next layer while
//     the current layer computes.
// The device tables (one pointer per expert and layer) are what the fused
// kernels read (WispMoeLayer.expert_blobs); a NULL entry means "not resident"
// and makes the kernels flag ST_EXPERT instead of reading.

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "internal.h"
#include "tiers.h"

struct WispStreamCache {
    int L = 0, E = 0, device = 0;
    size_t blob_bytes = 0;
    wb::SlotArena arena;
    wb::Lru lru;
    std::vector<const void*> pool;  // [L * E] pinned host blobs (tiled)
    void** d_tables = nullptr;      // [L * E] device
    std::vector<void*> h_tables;    // [L * E] host mirror
    cudaStream_t xfer[2] = {nullptr, nullptr};
    int xfer_next = 0;
    // per slot
    std::vector<cudaEvent_t> ready;   // recorded after the slot's fill
    std::vector<int> last_use;        // index into use_ev (-1: never read)
    std::vector<uint8_t> from_prefetch;
    // slots a layer's ensure handed to kernels not yet marked by its layer_done:
    // not evicted until then, whatever order the caller prefetches in
    std::vector<uint8_t> pending;
    std::vector<uint64_t> slot_key;   // (layer, expert) key of the slot's expert
    std::vector<cudaEvent_t> use_ev;  // ring of "layer kernels done" events
    int use_head = 0;
    std::vector<std::vector<int>> layer_slots;  // per layer: slots held until its layer_done
    uint64_t hits = 0, misses = 0, prefetched = 0, prefetch_used = 0, bytes = 0;
    std::mutex mu;

    int slot_index(const void* blob) const {
        return (int)((static_cast<const char*>(blob) - 8 - arena_base()) / arena.slot_bytes());
    }
    const char* arena_base() const { return base; }
    const char* base = nullptr;
};

namespace {

constexpr int kUseEvents = 64;

// Slot for (layer, expert): a free one, else the LRU victim outside `keep`
// (its table entry cleared; the next copy into it waits for its last reader).
void* take_slot(WispStreamCache* c, const std::vector<uint64_t>& keep, cudaStream_t s) {
    void* p = c->arena.alloc();
    if (p) return p;
    std::vector<uint64_t> hold = keep;
    for (size_t si = 0; si < c->pending.size(); ++si)
        if (c->pending[si]) hold.push_back(c->slot_key[si]);
    std::sort(hold.begin(), hold.end());
    wb::Lru::Entry v;
    if (!c->lru.evict_except(hold, &v)) return nullptr;
    // kernels already queued may still read the victim (through the table and
    // the slot): the transfer stream waits for them before touching either; and
    // the victim's own fill may still be in flight on the other transfer stream
    // (a prefetch nobody read yet): the new copy waits for it too
    const int si = c->slot_index(v.data);
    if (c->last_use[si] >= 0) cudaStreamWaitEvent(s, c->use_ev[c->last_use[si]], 0);
    cudaStreamWaitEvent(s, c->ready[si], 0);
    const size_t ti = (size_t)v.layer * c->E + v.expert;
    c->h_tables[ti] = nullptr;
    cudaMemcpyAsync(c->d_tables + ti, &c->h_tables[ti], sizeof(void*), cudaMemcpyHostToDevice, s);
    return v.data;
}

// Copy expert (layer, e) into a slot on the next transfer stream; returns the
// slot or nullptr (no slot could be freed).
void* fill(WispStreamCache* c, int layer, int e, const std::vector<uint64_t>& keep,
           bool prefetch, WispErrCtx* err) {
    cudaStream_t s = c->xfer[c->xfer_next];
    c->xfer_next ^= 1;
    void* slot = take_slot(c, keep, s);
    if (!slot) {
        WB_SET_ERR(err, WISP_ERR_OOM, "stream cache: every slot is needed by this layer");
        return nullptr;
    }
    const size_t ti = (size_t)layer * c->E + e;
    cudaError_t ce = cudaMemcpyAsync(slot, c->pool[ti], c->blob_bytes, cudaMemcpyHostToDevice, s);
    const int si = c->slot_index(slot);
    c->h_tables[ti] = slot;
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(c->d_tables + ti, &c->h_tables[ti], sizeof(void*),
                             cudaMemcpyHostToDevice, s);
    // ready = blob and table entry landed
    if (ce == cudaSuccess) ce = cudaEventRecord(c->ready[si], s);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "stream cache copy: %s", cudaGetErrorString(ce));
        c->arena.release(slot);
        return nullptr;
    }
    c->last_use[si] = -1;
    c->from_prefetch[si] = prefetch ? 1 : 0;
    c->slot_key[si] = wb::Lru::key((uint32_t)layer, (uint32_t)e);
    c->lru.put((uint32_t)layer, (uint32_t)e, slot, c->blob_bytes);
    c->bytes += c->blob_bytes;
    return slot;
}

bool check_ids(WispStreamCache* c, int layer, const int* ids, int n, WispErrCtx* err) {
    if (!c || layer < 0 || layer >= c->L || n < 0 || (n > 0 && !ids)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "stream cache: bad layer or ids");
        return false;
    }
    for (int i = 0; i < n; ++i)
        if (ids[i] >= c->E || (ids[i] >= 0 && !c->pool[(size_t)layer * c->E + ids[i]])) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "stream cache: expert %d of layer %d has no "
                       "registered host blob", ids[i], layer);
            return false;
        }
    return true;
}

std::vector<int> unique_ids(const int* ids, int n) {
    std::vector<int> u;
    for (int i = 0; i < n; ++i)
        if (ids[i] >= 0) u.push_back(ids[i]);
    std::sort(u.begin(), u.end());
    u.erase(std::unique(u.begin(), u.end()), u.end());
    return u;
}

}  // namespace

extern "C" WispStreamCache* wisp_stream_create(int n_layers, int n_experts, size_t blob_bytes,
                                               size_t n_slots, WispErrCtx* err) {
    if (n_layers <= 0 || n_experts <= 0 || blob_bytes < 128 || n_slots == 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "stream cache: bad sizes");
        return nullptr;
    }
    WispStreamCache* c = new WispStreamCache();
    c->L = n_layers;
    c->E = n_experts;
    c->blob_bytes = blob_bytes;
    cudaGetDevice(&c->device);
    cudaError_t ce = c->arena.init(blob_bytes, n_slots);
    if (ce == cudaSuccess && c->arena.n_slots() == n_slots) {
        void* first = c->arena.alloc();
        c->base = static_cast<const char*>(first) - 8;
        c->arena.release(first);
    } else if (ce == cudaSuccess) {
        ce = cudaErrorMemoryAllocation;
    }
    const size_t nt = (size_t)n_layers * n_experts;
    if (ce == cudaSuccess) ce = cudaMalloc(&c->d_tables, nt * sizeof(void*));
    if (ce == cudaSuccess) ce = cudaMemset(c->d_tables, 0, nt * sizeof(void*));
    for (int i = 0; i < 2 && ce == cudaSuccess; ++i)
        ce = cudaStreamCreateWithFlags(&c->xfer[i], cudaStreamNonBlocking);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_OOM, "stream cache (%zu slots of %zu bytes): %s", n_slots,
                   blob_bytes, cudaGetErrorString(ce));
        delete c;
        return nullptr;
    }
    c->lru.set_capacity((uint64_t)n_slots * blob_bytes);
    c->pool.assign(nt, nullptr);
    c->h_tables.assign(nt, nullptr);
    c->ready.assign(n_slots, nullptr);
    c->last_use.assign(n_slots, -1);
    c->from_prefetch.assign(n_slots, 0);
    c->pending.assign(n_slots, 0);
    c->slot_key.assign(n_slots, 0);
    for (size_t i = 0; i < n_slots; ++i) cudaEventCreateWithFlags(&c->ready[i], cudaEventDisableTiming);
    c->use_ev.assign(kUseEvents, nullptr);
    for (int i = 0; i < kUseEvents; ++i) cudaEventCreateWithFlags(&c->use_ev[i], cudaEventDisableTiming);
    c->layer_slots.assign(n_layers, {});
    return c;
}

extern "C" void wisp_stream_destroy(WispStreamCache* c) {
    if (!c) return;
    for (int i = 0; i < 2; ++i)
        if (c->xfer[i]) {
            cudaStreamSynchronize(c->xfer[i]);
            cudaStreamDestroy(c->xfer[i]);
        }
    for (cudaEvent_t e : c->ready)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : c->use_ev)
        if (e) cudaEventDestroy(e);
    if (c->d_tables) cudaFree(c->d_tables);
    delete c;
}

extern "C" WispError wisp_stream_register(WispStreamCache* c, int layer, int expert,
                                          const void* host_blob, WispErrCtx* err) {
    if (!c || layer < 0 || layer >= c->L || expert < 0 || expert >= c->E || !host_blob) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "stream register: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    if (reinterpret_cast<const uint32_t*>(host_blob)[1] != 2u) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "stream register: layer %d expert %d is not a tiled blob",
                   layer, expert);
        return WISP_ERR_MODEL;
    }
    std::lock_guard<std::mutex> g(c->mu);
    c->pool[(size_t)layer * c->E + expert] = host_blob;
    return WISP_OK;
}

extern "C" const void* const* wisp_stream_table(WispStreamCache* c, int layer) {
    if (!c || layer < 0 || layer >= c->L) return nullptr;
    return const_cast<const void* const*>(c->d_tables + (size_t)layer * c->E);
}

extern "C" WispError wisp_stream_ensure(WispStreamCache* c, int layer, const int* ids, int n,
                                        cudaStream_t compute, int* hits, int* misses,
                                        WispErrCtx* err) {
    if (!check_ids(c, layer, ids, n, err)) return WISP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    const std::vector<int> u = unique_ids(ids, n);
    std::vector<uint64_t> keep;
    for (int e : u) keep.push_back(wb::Lru::key((uint32_t)layer, (uint32_t)e));
    std::sort(keep.begin(), keep.end());
    int h = 0, m = 0;
    // the layer's slots stay held until its layer_done; an ensure repeated before it
    // adds to the held set instead of replacing it (the earlier call's kernels may be
    // queued already)
    std::vector<int>& used = c->layer_slots[layer];
    for (int e : u) {
        wb::Lru::Entry ent;
        void* slot = nullptr;
        if (c->lru.get((uint32_t)layer, (uint32_t)e, &ent)) {
            c->lru.touch((uint32_t)layer, (uint32_t)e);
            slot = ent.data;
            ++h;
            const int si = c->slot_index(slot);
            if (c->from_prefetch[si]) {
                c->prefetch_used++;
                c->from_prefetch[si] = 0;
            }
        } else {
            slot = fill(c, layer, e, keep, false, err);
            if (!slot) return err && err->code ? (WispError)err->code : WISP_ERR_OOM;
            ++m;
        }
        const int si = c->slot_index(slot);
        cudaStreamWaitEvent(compute, c->ready[si], 0);
        if (!c->pending[si]) used.push_back(si);
        c->pending[si] = 1;
    }
    c->hits += (uint64_t)h;
    c->misses += (uint64_t)m;
    if (hits) *hits = h;
    if (misses) *misses = m;
    return WISP_OK;
}

extern "C" WispError wisp_stream_prefetch(WispStreamCache* c, int layer, const int* ids, int n,
                                          int* issued, WispErrCtx* err) {
    if (!check_ids(c, layer, ids, n, err)) return WISP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> g(c->mu);
    const std::vector<int> u = unique_ids(ids, n);
    std::vector<uint64_t> keep;
    for (int e : u) keep.push_back(wb::Lru::key((uint32_t)layer, (uint32_t)e));
    std::sort(keep.begin(), keep.end());
    int k = 0;
    for (int e : u) {
        if (c->lru.get((uint32_t)layer, (uint32_t)e, nullptr)) continue;
        WispErrCtx fe{};
        if (!fill(c, layer, e, keep, true, &fe)) break;  // the cache is full of needed experts
        ++k;
    }
    c->prefetched += (uint64_t)k;
    if (issued) *issued = k;
    return WISP_OK;
}

extern "C" WispError wisp_stream_layer_done(WispStreamCache* c, int layer, cudaStream_t compute,
                                            WispErrCtx* err) {
    if (!c || layer < 0 || layer >= c->L) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "stream layer_done: bad layer");
        return WISP_ERR_INVALID_ARG;
    }
    std::lock_guard<std::mutex> g(c->mu);
    const int i = c->use_head;
    c->use_head = (c->use_head + 1) % kUseEvents;
    WB_CUDA_RET(cudaEventRecord(c->use_ev[i], compute), err);
    for (int si : c->layer_slots[layer]) {
        c->last_use[si] = i;
        c->pending[si] = 0;
    }
    c->layer_slots[layer].clear();
    return WISP_OK;
}

extern "C" void wisp_stream_reset(WispStreamCache* c) {
    if (!c) return;
    std::lock_guard<std::mutex> g(c->mu);
    // every queued reader and copy finishes before the slots are forgotten
    cudaDeviceSynchronize();
    c->lru.clear([&](const wb::Lru::Entry& v) { c->arena.release(v.data); });
    std::fill(c->h_tables.begin(), c->h_tables.end(), nullptr);
    cudaMemset(c->d_tables, 0, c->h_tables.size() * sizeof(void*));
    std::fill(c->last_use.begin(), c->last_use.end(), -1);
    std::fill(c->from_prefetch.begin(), c->from_prefetch.end(), 0);
    std::fill(c->pending.begin(), c->pending.end(), 0);
    for (auto& v : c->layer_slots) v.clear();
    c->hits = c->misses = c->prefetched = c->prefetch_used = c->bytes = 0;
}

extern "C" void wisp_stream_stats(WispStreamCache* c, uint64_t* out6) {
    if (!c || !out6) return;
    std::lock_guard<std::mutex> g(c->mu);
    out6[0] = c->hits;
    out6[1] = c->misses;
    out6[2] = c->prefetched;
    out6[3] = c->prefetch_used;
    out6[4] = c->bytes;
    out6[5] = c->arena.n_slots();
}
