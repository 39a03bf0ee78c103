// tiers.cpp -- LRU, slot arena and double buffer (see tiers.h), plus the
// host-only self-tests the reference exposes (lru_cache.c:213-270,
// double_buffer.c:184-229): same scenarios, run against these classes.
#include "tiers.h"

#include <string.h>

#include <algorithm>
#include <thread>

#include "wisp_b200.h"

namespace wb {

uint64_t Lru::used() const {
    std::lock_guard<std::mutex> g(mu_);
    return used_;
}
size_t Lru::count() const {
    std::lock_guard<std::mutex> g(mu_);
    return list_.size();
}
bool Lru::get(uint32_t layer, uint32_t expert, Entry* out) const {
    std::lock_guard<std::mutex> g(mu_);
    auto it = map_.find(key(layer, expert));
    if (it == map_.end()) return false;
    if (out) *out = *it->second;
    return true;
}
uint32_t Lru::touch(uint32_t layer, uint32_t expert) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = map_.find(key(layer, expert));
    if (it == map_.end()) return 0;
    list_.splice(list_.begin(), list_, it->second);
    return ++it->second->hits;
}
void Lru::put(uint32_t layer, uint32_t expert, void* data, size_t bytes) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = map_.find(key(layer, expert));
    if (it != map_.end()) {
        used_ -= it->second->bytes;
        it->second->data = data;
        it->second->bytes = bytes;
        used_ += bytes;
        list_.splice(list_.begin(), list_, it->second);
        return;
    }
    list_.push_front(Entry{layer, expert, data, bytes, 0});
    map_[key(layer, expert)] = list_.begin();
    used_ += bytes;
}
bool Lru::evict(Entry* out) {
    std::lock_guard<std::mutex> g(mu_);
    if (list_.empty()) return false;
    Entry e = list_.back();
    map_.erase(key(e.layer, e.expert));
    list_.pop_back();
    used_ -= e.bytes;
    if (out) *out = e;
    return true;
}
bool Lru::evict_except(const std::vector<uint64_t>& keep, Entry* out) {
    std::lock_guard<std::mutex> g(mu_);
    for (auto it = list_.rbegin(); it != list_.rend(); ++it) {
        uint64_t k = key(it->layer, it->expert);
        if (std::binary_search(keep.begin(), keep.end(), k)) continue;
        Entry e = *it;
        map_.erase(k);
        list_.erase(std::next(it).base());
        used_ -= e.bytes;
        if (out) *out = e;
        return true;
    }
    return false;
}
bool Lru::remove(uint32_t layer, uint32_t expert, Entry* out) {
    std::lock_guard<std::mutex> g(mu_);
    auto it = map_.find(key(layer, expert));
    if (it == map_.end()) return false;
    if (out) *out = *it->second;
    used_ -= it->second->bytes;
    list_.erase(it->second);
    map_.erase(it);
    return true;
}
bool Lru::would_overflow(size_t bytes) const {
    std::lock_guard<std::mutex> g(mu_);
    return used_ + bytes > cap_;
}

// ---------------------------------------------------------------- arena
SlotArena::~SlotArena() {
    if (base_) cudaFree(base_);
}
cudaError_t SlotArena::init(size_t slot_bytes, size_t n_slots) {
    slot_bytes_ = (slot_bytes + 8 + 255) / 256 * 256;
    n_ = n_slots;
    if (n_ == 0) return cudaSuccess;
    cudaError_t e = cudaMalloc(&base_, slot_bytes_ * n_);
    if (e != cudaSuccess) {
        base_ = nullptr;
        n_ = 0;
        return e;
    }
    free_.reserve(n_);
    for (size_t i = n_; i > 0; --i) free_.push_back(i - 1);
    return cudaSuccess;
}
void* SlotArena::alloc() {
    std::lock_guard<std::mutex> g(mu_);
    if (free_.empty()) return nullptr;
    size_t i = free_.back();
    free_.pop_back();
    return base_ + i * slot_bytes_ + 8;
}
void SlotArena::release(void* blob) {
    if (!blob) return;
    std::lock_guard<std::mutex> g(mu_);
    size_t i = (size_t)(static_cast<char*>(blob) - 8 - base_) / slot_bytes_;
    free_.push_back(i);
}
size_t SlotArena::n_free() const {
    std::lock_guard<std::mutex> g(mu_);
    return free_.size();
}

// ---------------------------------------------------------- double buffer
DoubleBuffer::~DoubleBuffer() {
    for (int i = 0; i < 2; ++i)
        if (buf_[i]) {
            if (pinned_)
                cudaFreeHost(buf_[i]);
            else
                free(buf_[i]);
        }
    if (done_) cudaEventDestroy(done_);
}
cudaError_t DoubleBuffer::init(size_t buf_bytes, cudaStream_t transfer, bool pinned) {
    bytes_ = buf_bytes;
    transfer_ = transfer;
    pinned_ = pinned;
    for (int i = 0; i < 2; ++i) {
        if (pinned) {
            cudaError_t e = cudaHostAlloc(&buf_[i], buf_bytes, cudaHostAllocDefault);
            if (e != cudaSuccess) return e;
        } else {
            buf_[i] = malloc(buf_bytes);
            if (!buf_[i]) return cudaErrorMemoryAllocation;
        }
    }
    if (pinned) return cudaEventCreateWithFlags(&done_, cudaEventDisableTiming);
    return cudaSuccess;
}
void* DoubleBuffer::reserve(uint32_t layer, uint32_t expert, size_t bytes) {
    std::lock_guard<std::mutex> g(mu_);
    ExpertBatch& b = batch_[filling_];
    size_t used = b.count ? b.offset[b.count - 1] + b.size[b.count - 1] : 0;
    if (b.count >= ExpertBatch::kMax || used + bytes > bytes_) return nullptr;
    int i = b.count++;
    b.layer[i] = layer;
    b.expert[i] = expert;
    b.offset[i] = used;
    b.size[i] = bytes;
    fill_in_progress_ = true;
    return static_cast<char*>(buf_[filling_]) + used;
}
void DoubleBuffer::fill_done() {
    std::lock_guard<std::mutex> g(mu_);
    fill_in_progress_ = false;
    cv_.notify_all();
}
ExpertBatch* DoubleBuffer::tick(ExpertBatch* current, ExpertBatch* next) {
    std::unique_lock<std::mutex> g(mu_);
    cv_.wait(g, [&] { return !fill_in_progress_; });
    if (done_ && transfer_) {
        cudaEventRecord(done_, transfer_);
        cudaEventSynchronize(done_);
    }
    std::swap(active_, filling_);
    if (current) *current = batch_[active_];
    batch_[filling_].count = 0;
    if (next) *next = batch_[filling_];
    return &batch_[active_];
}

}  // namespace wb

// ------------------------------------------------------------- self-tests
// The scenario exercises what the engine relies on: a byte budget over blobs of
// different sizes, recency across two layers, the hit counter that drives RAM ->
// VRAM promotion, eviction that spares the current layer's experts, and a clear
// that hands every blob back to its owner.
extern "C" int wisp_selftest_lru(void) {
    using wb::Lru;
    static unsigned char blob[4][64];
    Lru c(160);
    c.put(2, 10, blob[0], 64);  // layer 2: two experts of 64 bytes
    c.put(2, 11, blob[1], 64);
    c.put(3, 40, blob[2], 16);  // layer 3: a small one
    if (c.count() != 3 || c.used() != 144) return 0;
    if (!c.would_overflow(32) || c.would_overflow(16)) return 0;
    // Hits counted per entry; the third one is the promotion threshold.
    if (c.touch(2, 10) != 1 || c.touch(2, 10) != 2 || c.touch(2, 10) != 3) return 0;
    if (c.touch(9, 9) != 0) return 0;  // a miss counts nothing
    // Recency (MRU first): (2,10), (3,40), (2,11).  Keeping layer 2's experts
    // skips (2,11) and takes (3,40).
    std::vector<uint64_t> keep = {Lru::key(2, 10), Lru::key(2, 11)};
    std::sort(keep.begin(), keep.end());
    Lru::Entry e;
    if (!c.evict_except(keep, &e) || e.layer != 3 || e.expert != 40 || e.bytes != 16) return 0;
    if (c.evict_except(keep, &e)) return 0;  // nothing left outside `keep`
    // Re-inserting a key replaces its blob, keeps one entry, refreshes recency.
    c.put(2, 11, blob[3], 32);
    if (c.count() != 2 || c.used() != 96) return 0;
    if (!c.get(2, 11, &e) || e.data != blob[3] || e.bytes != 32) return 0;
    if (!c.evict(&e) || e.expert != 10 || e.hits != 3) return 0;  // (2,10) is LRU now
    if (!c.remove(2, 11, &e) || c.remove(2, 11, &e) || c.count() != 0) return 0;
    c.put(5, 1, blob[0], 48);
    c.put(5, 2, blob[1], 48);
    size_t handed = 0, bytes = 0;
    c.clear([&](const Lru::Entry& x) { ++handed; bytes += x.bytes; });
    if (handed != 2 || bytes != 96 || c.count() != 0 || c.used() != 0) return 0;
    return c.get(5, 1, nullptr) ? 0 : 1;
}

// The scenario checks what the staging path relies on: reservations packed back to
// back up to the exact capacity and refused past it or past the entry limit, a tick
// handing the consumer the filled side intact while new reservations land in the
// other buffer, and, with a producer thread, batches that only ever hold whole
// rounds of fills with their bytes where the entries say.
extern "C" int wisp_selftest_double_buffer(void) {
    using wb::ExpertBatch;
    constexpr size_t kCap = 1024;
    wb::DoubleBuffer db;
    if (db.init(kCap, nullptr, /*pinned=*/false) != cudaSuccess) return 0;
    const size_t sizes[4] = {256, 512, 128, 128};
    char* base = nullptr;
    for (uint32_t e = 0; e < 4; ++e) {
        char* p = static_cast<char*>(db.reserve(3, e, sizes[e]));
        if (!p) return 0;
        if (e == 0) base = p;
        memset(p, 0x40 + (int)e, sizes[e]);
    }
    if (db.reserve(3, 9, 1) != nullptr) return 0;  // exactly full
    db.fill_done();
    const int before = db.active();
    ExpertBatch cur, nxt;
    ExpertBatch* got = db.tick(&cur, &nxt);
    if (db.active() == before || got->count != 4 || cur.count != 4 || nxt.count != 0) return 0;
    const size_t want_off[4] = {0, 256, 768, 896};
    for (int i = 0; i < 4; ++i) {
        if (got->layer[i] != 3 || got->expert[i] != (uint32_t)i || got->offset[i] != want_off[i] ||
            got->size[i] != sizes[i])
            return 0;
        const char* d = static_cast<const char*>(db.buffer(db.active())) + got->offset[i];
        for (size_t k = 0; k < got->size[i]; ++k)
            if (d[k] != (char)(0x40 + i)) return 0;
    }
    if (base != db.buffer(db.active())) return 0;
    // the next fill goes to the other buffer, outside what the consumer reads
    char* q = static_cast<char*>(db.reserve(4, 0, 64));
    const char* act = static_cast<const char*>(db.buffer(db.active()));
    if (!q || (q >= act && q < act + kCap)) return 0;
    for (int i = 1; i < ExpertBatch::kMax; ++i)
        if (!db.reserve(4, (uint32_t)i, 1)) return 0;
    if (db.reserve(4, 99, 1) != nullptr) return 0;  // entry limit
    db.fill_done();
    db.tick(nullptr, nullptr);
    db.tick(nullptr, nullptr);  // both sides empty again
    // producer thread: 6 rounds of 4 fills of 32 bytes, one layer per round
    constexpr int kRounds = 6, kPer = 4;
    constexpr size_t kSz = 32;
    std::thread producer([&] {
        for (int r = 0; r < kRounds; ++r) {
            for (int e = 0; e < kPer; ++e) {
                char* d = static_cast<char*>(db.reserve((uint32_t)r, (uint32_t)e, kSz));
                if (d) memset(d, r * kPer + e + 1, kSz);
            }
            db.fill_done();
        }
    });
    int seen = 0;
    bool ok = true;
    auto check = [&](const ExpertBatch* bt) {
        if (bt->count % kPer) ok = false;
        const char* buf = static_cast<const char*>(db.buffer(db.active()));
        for (int i = 0; i < bt->count; ++i) {
            if (bt->expert[i] != (uint32_t)(i % kPer) || bt->layer[i] != bt->layer[i - i % kPer])
                ok = false;
            const char want = (char)(bt->layer[i] * kPer + bt->expert[i] + 1);
            for (size_t k = 0; k < kSz; ++k)
                if (buf[bt->offset[i] + k] != want) ok = false;
        }
        seen += bt->count;
    };
    for (int r = 0; r < kRounds; ++r) check(db.tick(nullptr, nullptr));
    producer.join();
    check(db.tick(nullptr, nullptr));
    check(db.tick(nullptr, nullptr));
    return ok && seen == kRounds * kPer ? 1 : 0;
}
