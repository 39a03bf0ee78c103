// tiers.h -- host-side tier bookkeeping: an O(1) LRU keyed by (layer,
// expert), a fixed-slot device arena, and the pinned double buffer.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <condition_variable>
#include <list>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

namespace wb {

// LRU over (layer, expert) with byte capacity.  Semantics follow the
// reference's lru_cache.c (get/touch/put-replaces/evict-tail/remove/clear,
// a per-entry hit counter that gates VRAM promotion).  All calls lock.
class Lru {
public:
    struct Entry {
        uint32_t layer, expert;
        void* data;
        size_t bytes;
        uint32_t hits;
    };
    explicit Lru(uint64_t capacity = 0) : cap_(capacity) {}
    void set_capacity(uint64_t c) { cap_ = c; }
    uint64_t capacity() const { return cap_; }
    uint64_t used() const;
    size_t count() const;
    // Returns a copy of the entry (or false on a miss); does not touch.
    bool get(uint32_t layer, uint32_t expert, Entry* out) const;
    // Move to MRU and bump the hit counter; returns the new hit count.
    uint32_t touch(uint32_t layer, uint32_t expert);
    // Insert or replace (replace keeps the entry, refreshes recency).
    void put(uint32_t layer, uint32_t expert, void* data, size_t bytes);
    // Pop the least-recently-used entry; false when empty.
    bool evict(Entry* out);
    // Pop the LRU entry whose key is not in `keep` (sorted keys); false if none.
    bool evict_except(const std::vector<uint64_t>& keep, Entry* out);
    bool remove(uint32_t layer, uint32_t expert, Entry* out);
    bool would_overflow(size_t bytes) const;
    // Remove everything, handing each entry to `fn`.
    template <typename F>
    void clear(F fn) {
        std::lock_guard<std::mutex> g(mu_);
        for (auto& e : list_) fn(e);
        list_.clear();
        map_.clear();
        used_ = 0;
    }
    static uint64_t key(uint32_t l, uint32_t e) { return ((uint64_t)l << 32) | e; }

private:
    mutable std::mutex mu_;
    uint64_t cap_ = 0, used_ = 0;
    std::list<Entry> list_;  // front = MRU
    std::unordered_map<uint64_t, std::list<Entry>::iterator> map_;
};

// One device allocation cut into equal slots; each slot's usable address is
// slot_base + 8 so that a .bin blob stored there has its 120-byte header end
// on a 16-byte boundary (the packed/scales/zeros sections start aligned).
class SlotArena {
public:
    ~SlotArena();
    cudaError_t init(size_t slot_bytes, size_t n_slots);
    void* alloc();            // blob address, or nullptr when full
    void release(void* blob);
    size_t slot_bytes() const { return slot_bytes_; }
    size_t n_slots() const { return n_; }
    size_t n_free() const;

private:
    mutable std::mutex mu_;
    char* base_ = nullptr;
    size_t slot_bytes_ = 0, n_ = 0;
    std::vector<size_t> free_;
};

// Two pinned host buffers, one being filled by a producer while the
// consumer works from the other (reference: double_buffer.h:23-77; same
// reserve / fill_done / tick contract).
struct ExpertBatch {
    static constexpr int kMax = 64;
    uint32_t layer[kMax], expert[kMax];
    size_t offset[kMax], size[kMax];
    int count = 0;
};

class DoubleBuffer {
public:
    ~DoubleBuffer();
    cudaError_t init(size_t buf_bytes, cudaStream_t transfer, bool pinned = true);
    void* reserve(uint32_t layer, uint32_t expert, size_t bytes);
    void fill_done();
    // Waits for the producer and the in-flight transfer, swaps roles and
    // returns the batch the consumer may now read.
    ExpertBatch* tick(ExpertBatch* current, ExpertBatch* next);
    void* buffer(int i) const { return buf_[i]; }
    size_t bytes() const { return bytes_; }
    int active() const { return active_; }

private:
    std::mutex mu_;
    std::condition_variable cv_;
    void* buf_[2] = {nullptr, nullptr};
    bool pinned_ = true;
    size_t bytes_ = 0;
    int active_ = 0, filling_ = 1;
    bool fill_in_progress_ = false;
    ExpertBatch batch_[2];
    cudaStream_t transfer_ = nullptr;
    cudaEvent_t done_ = nullptr;
};

}  // namespace wb
