// engine.cpp -- the engine ABI (reference: csrc/core/wisp_engine.h:472-543,
// wisp_engine.c:851-1177 and 1601-2367) over the fused B200 MoE kernels.
//
// Model directory: manifest.json (keys found by name anywhere in the file,
// as the reference's strstr scan does, wisp_engine.c:1601-1657),
// dense/model_dense.safetensors (fp16: layers.i.router, router_bias,
// post_norm, shared.{gate,up,down}; wisp_engine.c:1698-1813) and
// experts/L%03u_E%05u.bin blobs.  The shared expert is run in the form the
// reference converter writes it, fp16-dense layers.i.shared.*, unless this
// build's int4 copy experts/L%03u_shared.bin (same .bin layout, a quarter of
// the bytes) is present.  A layer without a router is a dense-MLP layer
// (wisp_engine.c:1757): its FFN is the fp16-dense shared.* SwiGLU alone
// (run_dense_mlp, :1524-1534).  A routed expert whose file cannot be read
// (WISP_ERR_IO) is skipped and the others are combined, as run_moe does
// (:1473-1477, 1502-1506).
//
// Expert tiers (policy of wisp_engine.c:920-1078): VRAM LRU (fixed slots in
// one device arena), RAM LRU (pinned host blobs), SSD files.  A RAM hit is
// served through a small scratch ring of device slots until it has been hit
// WISP_PROMOTE_HITS (3) times, then it earns a VRAM slot (evicting the VRAM
// LRU back to RAM).  A cold SSD read takes a VRAM slot only if one is free.
// Each layer keeps a device table [E] of blob pointers that the fused
// kernels read; when every expert of a layer is VRAM-resident the whole MoE
// block runs with no host synchronisation.

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <utility>
#include <vector>

#include "dense_ffn.h"
#include "internal.h"
#include "tiers.h"

namespace {

constexpr uint32_t kMagic = 0x57455850u;
constexpr int kPromoteHits = 3;
constexpr int kPrefetchRing = 1024;

uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

bool read_file(const std::string& path, std::vector<char>& out) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (n < 0) {
        fclose(f);
        return false;
    }
    out.resize((size_t)n + 1);
    size_t got = fread(out.data(), 1, (size_t)n, f);
    fclose(f);
    if (got != (size_t)n) return false;
    out[(size_t)n] = 0;
    out.resize((size_t)n);
    return true;
}

// Value after "key": anywhere in a JSON text (the reference's lookup rule).
const char* json_find(const char* js, const char* key) {
    std::string pat = std::string("\"") + key + "\"";
    const char* p = strstr(js, pat.c_str());
    if (!p) return nullptr;
    p += pat.size();
    while (*p && *p != ':') ++p;
    if (*p != ':') return nullptr;
    ++p;
    while (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r') ++p;
    return p;
}
double json_num(const char* js, const char* key, double dflt) {
    const char* p = json_find(js, key);
    return p ? strtod(p, nullptr) : dflt;
}
std::string json_str(const char* js, const char* key) {
    const char* p = json_find(js, key);
    if (!p || *p != '"') return std::string();
    const char* q = strchr(p + 1, '"');
    return q ? std::string(p + 1, q) : std::string();
}

// Minimal safetensors reader: locate a tensor by exact name in the header.
struct StTensor {
    uint64_t off = 0, bytes = 0;
    std::vector<int64_t> shape;
    bool f16 = false;
};
struct StFile {
    FILE* f = nullptr;
    std::string header;
    uint64_t data_start = 0;
    ~StFile() {
        if (f) fclose(f);
    }
    bool open(const std::string& path) {
        f = fopen(path.c_str(), "rb");
        if (!f) return false;
        uint8_t le[8];
        if (fread(le, 1, 8, f) != 8) return false;
        uint64_t n = 0;
        for (int i = 7; i >= 0; --i) n = (n << 8) | le[i];
        if (n == 0 || n > (1ull << 31)) return false;
        header.resize(n);
        if (fread(&header[0], 1, n, f) != n) return false;
        data_start = 8 + n;
        return true;
    }
    bool find(const std::string& name, StTensor* t) const {
        std::string pat = "\"" + name + "\":";
        size_t p = header.find(pat);
        if (p == std::string::npos) return false;
        size_t ob = header.find('{', p + pat.size());
        size_t cb = header.find('}', ob);
        if (ob == std::string::npos || cb == std::string::npos) return false;
        std::string obj = header.substr(ob, cb - ob + 1);
        t->f16 = obj.find("\"F16\"") != std::string::npos;
        size_t sp = obj.find("\"shape\"");
        if (sp != std::string::npos) {
            size_t lb = obj.find('[', sp), rb = obj.find(']', lb);
            const char* c = obj.c_str() + lb + 1;
            const char* end = obj.c_str() + rb;
            while (c < end) {
                char* nx;
                long long v = strtoll(c, &nx, 10);
                if (nx == c) break;
                t->shape.push_back(v);
                c = nx;
                while (c < end && (*c == ',' || *c == ' ')) ++c;
            }
        }
        size_t dp = obj.find("\"data_offsets\"");
        if (dp == std::string::npos) return false;
        const char* c = obj.c_str() + obj.find('[', dp) + 1;
        char* nx;
        unsigned long long a = strtoull(c, &nx, 10);
        while (*nx == ',' || *nx == ' ') ++nx;
        unsigned long long b = strtoull(nx, nullptr, 10);
        t->off = a;
        t->bytes = b - a;
        return true;
    }
    bool read(const StTensor& t, void* dst) const {
        if (fseeko(f, (off_t)(data_start + t.off), SEEK_SET) != 0) return false;
        return fread(dst, 1, t.bytes, f) == t.bytes;
    }
};

struct LayerDev {
    wisp_half* router = nullptr;
    wisp_half* router_bias = nullptr;
    wisp_half* post_norm = nullptr;
    void* shared_blob = nullptr;
    WispExpertMeta shared_meta{};
    // fp16-dense shared expert / dense-MLP weights (layers.i.shared.*)
    wisp_half* shared_gate = nullptr;
    wisp_half* shared_up = nullptr;
    wisp_half* shared_down = nullptr;
    int shared_inter = 0;
    bool dense_mlp = false;       // no router: the layer's FFN is shared.* alone
    // the decoder step's attention (layers.i.input_norm, attn.{q,k,v,o}_proj)
    wisp_half* input_norm = nullptr;
    wisp_half* q_proj = nullptr;
    wisp_half* k_proj = nullptr;
    wisp_half* v_proj = nullptr;
    wisp_half* o_proj = nullptr;
    void** d_table = nullptr;     // device [E]
    std::vector<void*> h_table;   // host mirror
    std::vector<uint8_t> in_vram; // expert is VRAM-resident (not ring-served)
    int n_vram = 0;
};

}  // namespace

struct WispEngine {
    std::string path;
    int n_layers = 0, E = 0, K = 0, H = 0, inter = 0, gs = 64;
    float eps = 1e-6f;
    size_t expert_bytes = 0, max_expert_bytes = 0;
    int device = 0;
    cudaStream_t compute = nullptr, transfer = nullptr;
    std::vector<LayerDev> L;
    std::vector<WispExpertMeta> meta;
    wb::Lru ram, vram;
    wb::SlotArena arena, ring_arena;
    size_t vram_budget = 0;
    std::vector<void*> ring;
    int ring_pos = 0;
    void* staging = nullptr;  // pinned SSD staging (one expert)
    char* d_stage = nullptr;  // device staging slot: .bin blobs are tiled from here
    size_t stage_cap = 0;     // its capacity (bytes)
    std::mutex fetch_mu;
    // workspace of the fused kernels
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // per-call device buffers of the miss path and the layer-by-layer stack,
    // grown on demand and kept: routing [T, K], xn and ffn [T, H], dense h
    int* d_idx = nullptr;
    float* d_w = nullptr;
    float* d_xn = nullptr;
    float* d_ffn = nullptr;
    float* d_dh = nullptr;
    size_t cap_route = 0, cap_rows = 0, cap_dh = 0;
    std::vector<int> h_idx;        // host copy of the routing (miss path)
    cudaEvent_t order_ev = nullptr;  // orders the compute stream before a caller's stream
    // expert uploads and VRAM write-backs run on the transfer stream without host
    // synchronisation: up_ev marks the last one issued, the expert kernels wait on
    // it, and a RAM-tier buffer is freed only after they have drained
    cudaEvent_t up_ev = nullptr;
    cudaEvent_t evict_ev = nullptr;  // compute work before a VRAM victim is copied out
    bool uploads_pending = false;
    // prefetch worker
    std::thread worker;
    std::mutex q_mu;
    std::condition_variable q_cv;
    std::deque<std::pair<uint32_t, uint32_t>> q;
    bool stop = false;
    // stats
    std::mutex stats_mu;
    uint64_t hits[3] = {0, 0, 0};
    std::vector<uint32_t> log;
    int log_head = 0, log_count = 0;
    uint64_t log_dropped = 0;
    uint64_t tok_ns[32] = {0};
    int tok_head = 0, tok_count = 0;
    // decoder step (GQA / MHA models whose dense file holds the attention
    // projections): embedding, final norm, lm_head and per-token buffers
    bool has_decoder = false;
    std::string no_decoder;  // why not, for the error message
    int vocab = 0, n_heads = 0, n_kv = 0, head_dim = 0;
    float rope_theta = 10000.f;
    wisp_half* embed = nullptr;
    wisp_half* final_norm = nullptr;
    wisp_half* lm_head = nullptr;
    float* d_x = nullptr;       // [H] the token's hidden state
    float* d_logits = nullptr;  // [vocab]
    float* d_lmws = nullptr;    // [H] normalised input of lm_head
};

struct WispKVCache {
    int max_seq = 0, len = 0;
    size_t layer_elems = 0;  // max_seq * n_kv * head_dim
    wisp_half* k = nullptr;  // [layers][max_seq][n_kv][head_dim]
    wisp_half* v = nullptr;
    void* ws = nullptr;      // attention workspace (wisp_attn_workspace_bytes)
    size_t ws_bytes = 0;
    int device = 0;
};

namespace {

void stat_hit(WispEngine* e, int tier, uint32_t layer, uint32_t expert) {
    std::lock_guard<std::mutex> g(e->stats_mu);
    e->hits[tier]++;
    if (!e->log.empty()) {
        e->log[e->log_head] = ((layer & 0xFFFFu) << 16) | (expert & 0xFFFFu);
        e->log_head = (e->log_head + 1) % (int)e->log.size();
        if (e->log_count < (int)e->log.size())
            e->log_count++;
        else
            e->log_dropped++;
    }
}

std::string expert_path(const WispEngine* e, uint32_t layer, uint32_t expert) {
    char buf[64];
    snprintf(buf, sizeof buf, "/experts/L%03u_E%05u.bin", layer, expert);
    return e->path + buf;
}

// Read an expert file into `dst` (capacity cap). Returns bytes, 0 on error.
// The SSD tier's miss path (the reference opens the file and freads it per miss,
// wisp_engine.c:351-380): the file is opened with O_DIRECT and read with large
// preads straight into the destination, bypassing the page cache, when the
// destination and its capacity allow it (4096-byte aligned address, capacity >=
// the size rounded up to 4096 -- the engine's pinned staging buffer does); a
// filesystem that refuses O_DIRECT (tmpfs, some overlays) or an unaligned
// destination gets plain sequential preads.  *direct reports which one ran.
size_t read_file_into(const char* p, void* dst, size_t cap, int* direct, WispErrCtx* err) {
    constexpr size_t kAlign = 4096, kChunk = (size_t)16 << 20;
    if (direct) *direct = 0;
    struct stat sb;
    if (!p || !dst || stat(p, &sb) != 0) {
        WB_SET_ERR(err, WISP_ERR_IO, "expert file missing: %s", p ? p : "(null)");
        return 0;
    }
    const size_t n = (size_t)sb.st_size;
    if (n == 0 || n > cap) {
        WB_SET_ERR(err, WISP_ERR_IO, "expert file %s size %zu exceeds staging %zu", p, n, cap);
        return 0;
    }
    const size_t padded = (n + kAlign - 1) / kAlign * kAlign;
    const bool can_direct = (reinterpret_cast<uintptr_t>(dst) % kAlign) == 0 && padded <= cap;
    int fd = -1;
    bool use_direct = false;
#ifdef O_DIRECT
    if (can_direct) {
        fd = open(p, O_RDONLY | O_DIRECT);
        use_direct = fd >= 0;
    }
#endif
    if (fd < 0) fd = open(p, O_RDONLY);
    if (fd < 0) {
        WB_SET_ERR(err, WISP_ERR_IO, "expert file missing: %s", p);
        return 0;
    }
    if (!use_direct) posix_fadvise(fd, 0, 0, POSIX_FADV_SEQUENTIAL);
    char* out = static_cast<char*>(dst);
    size_t got = 0;
    const size_t want = use_direct ? padded : n;
    while (got < want) {
        const size_t len = std::min(kChunk, want - got);
        const ssize_t r = pread(fd, out + got, len, (off_t)got);
        if (r < 0 && errno == EINTR) continue;
        if (r < 0 && use_direct && got == 0 && errno == EINVAL) {
            // O_DIRECT accepted at open but not for this read: buffered instead
            close(fd);
            fd = open(p, O_RDONLY);
            use_direct = false;
            if (fd < 0) break;
            continue;
        }
        if (r <= 0) break;
        got += (size_t)r;
        if (use_direct && got >= n) break;  // the last block ends at end of file
    }
    if (fd >= 0) close(fd);
    if (got < n) {
        WB_SET_ERR(err, WISP_ERR_IO, "short read on %s: %zu of %zu", p, got, n);
        return 0;
    }
    if (direct) *direct = use_direct ? 1 : 0;
    return n;
}

size_t read_expert(const std::string& p, void* dst, size_t cap, WispErrCtx* err) {
    return read_file_into(p.c_str(), dst, cap, nullptr, err);
}

bool sections_aligned(const WispExpertMeta& m) {
    for (int i = 0; i < 3; ++i)
        if ((m.packed_off[i] - 120) % 16 || (m.scales_off[i] - 120) % 16 ||
            (m.zeros_off[i] - 120) % 16)
            return false;
    return (m.total_bytes - 120) % 16 == 0;
}

void set_table(WispEngine* e, uint32_t layer, uint32_t expert, void* ptr, bool vram) {
    LayerDev& d = e->L[layer];
    if (d.in_vram[expert] && !vram) d.n_vram--;
    if (!d.in_vram[expert] && vram) d.n_vram++;
    d.in_vram[expert] = vram ? 1 : 0;
    d.h_table[expert] = ptr;
    cudaMemcpyAsync(d.d_table + expert, &d.h_table[expert], sizeof(void*),
                    cudaMemcpyHostToDevice, e->compute);
}

// Wait for the uploads and write-backs in flight (their host buffers may be
// about to be freed or reused).
void drain_uploads(WispEngine* e) {
    if (!e->uploads_pending) return;
    cudaStreamSynchronize(e->transfer);
    e->uploads_pending = false;
}

// Insert a pinned host blob into the RAM tier, evicting its least recently used
// entries, except the keys in `keep` (sorted), until it fits.  A blob that cannot
// fit is freed instead and false is returned: the caller must not use `data` then.
bool ram_put(WispEngine* e, uint32_t layer, uint32_t expert, void* data, size_t n,
             const std::vector<uint64_t>& keep = {}) {
    if (n <= e->ram.capacity()) {
        wb::Lru::Entry v;
        while (e->ram.would_overflow(n) && e->ram.evict_except(keep, &v)) {
            drain_uploads(e);  // an upload or write-back may still use the victim's buffer
            cudaFreeHost(v.data);
        }
        if (!e->ram.would_overflow(n)) {
            e->ram.put(layer, expert, data, n);
            return true;
        }
    }
    drain_uploads(e);  // a write-back into `data` may still be in flight
    cudaFreeHost(data);
    return false;
}

// Host blob -> device slot in the tiled layout the kernels stream, on the
// transfer stream, not waited for: `src` must stay valid until the transfer
// stream passes it (RAM-tier buffers are freed only after drain_uploads), and
// whoever runs kernels on the slot waits for up_ev first (wait_uploads).  A .bin
// blob is copied to the device staging slot and tiled into `dst` (the staging
// slot is reused in transfer-stream order); a blob that is already tiled (a VRAM
// victim written back to the RAM tier) is copied as is.
bool put_tiled(WispEngine* e, void* dst, const void* src, size_t n, WispErrCtx* err) {
    WispExpertMeta m{};
    if (wisp_expert_parse_header(src, n, &m, err) != WISP_OK) return false;
    cudaError_t ce;
    if (m.tiled) {
        ce = cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, e->transfer);
    } else if (n > e->stage_cap) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "expert blob of %zu bytes exceeds the staging slot (%zu)",
                   n, e->stage_cap);
        return false;
    } else {
        ce = cudaMemcpyAsync(e->d_stage, src, n, cudaMemcpyHostToDevice, e->transfer);
        if (ce == cudaSuccess && wisp_expert_tile(&m, e->d_stage, dst, e->transfer, err) != WISP_OK)
            return false;
    }
    if (ce == cudaSuccess) ce = cudaEventRecord(e->up_ev, e->transfer);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "expert upload failed: %s", cudaGetErrorString(ce));
        return false;
    }
    e->uploads_pending = true;
    return true;
}

// Kernels queued next on `s` see every upload issued so far.
void wait_uploads(WispEngine* e, cudaStream_t s) {
    if (e->uploads_pending) cudaStreamWaitEvent(s, e->up_ev, 0);
}

// Upload into a ring slot (cool experts: no cache insert, no eviction).
void* scratch_serve(WispEngine* e, const void* src, size_t n, WispErrCtx* err) {
    void* slot = e->ring[e->ring_pos];
    e->ring_pos = (e->ring_pos + 1) % (int)e->ring.size();
    return put_tiled(e, slot, src, n, err) ? slot : nullptr;
}

// A VRAM slot, evicting the VRAM LRU (copied back to the RAM tier) until
// one is free.  `keep` lists keys that must not be evicted (sorted); `ram_keep`
// lists RAM-tier entries the write-backs must not push out (sorted: the blob
// being promoted, whose buffer is the next upload's source).
void* vram_alloc_evicting(WispEngine* e, size_t n, const std::vector<uint64_t>& keep,
                          const std::vector<uint64_t>& ram_keep) {
    if (e->arena.n_slots() == 0) return nullptr;
    for (;;) {
        if (!e->vram.would_overflow(n)) {
            void* p = e->arena.alloc();
            if (p) return p;
        }
        wb::Lru::Entry v;
        if (!e->vram.evict_except(keep, &v)) return nullptr;
        // The victim is copied back to the RAM tier on the transfer stream after the
        // kernels already queued on the compute stream (they may read its slot); the
        // slot's next upload follows on the same stream, so it cannot overtake.
        cudaEventRecord(e->evict_ev, e->compute);
        cudaStreamWaitEvent(e->transfer, e->evict_ev, 0);
        if (!e->ram.get(v.layer, v.expert, nullptr)) {
            void* host = nullptr;
            if (cudaHostAlloc(&host, v.bytes, cudaHostAllocDefault) == cudaSuccess) {
                if (cudaMemcpyAsync(host, v.data, v.bytes, cudaMemcpyDeviceToHost, e->transfer) ==
                    cudaSuccess) {
                    cudaEventRecord(e->up_ev, e->transfer);
                    e->uploads_pending = true;
                    ram_put(e, v.layer, v.expert, host, v.bytes, ram_keep);
                } else {
                    cudaFreeHost(host);
                }
            }
        }
        set_table(e, v.layer, v.expert, nullptr, false);
        e->arena.release(v.data);
    }
}

WispError ensure_meta(WispEngine* e, uint32_t layer, const void* blob, size_t n,
                      WispErrCtx* err) {
    if (e->meta[layer].valid) return WISP_OK;
    WispError r = wisp_expert_parse_header(blob, n, &e->meta[layer], err);
    if (r != WISP_OK) return r;
    return WISP_OK;
}

// Parse a layer's blob layout from the first readable expert file's header
// (no tier insertion, no statistics).
WispError meta_from_file(WispEngine* e, uint32_t layer, WispErrCtx* err) {
    for (int x = 0; x < e->E; ++x) {
        FILE* f = fopen(expert_path(e, layer, (uint32_t)x).c_str(), "rb");
        if (!f) continue;
        char head[120];
        size_t got = fread(head, 1, sizeof head, f);
        fseek(f, 0, SEEK_END);
        long n = ftell(f);
        fclose(f);
        if (got != sizeof head || n <= 0) continue;
        return wisp_expert_parse_header(head, (size_t)n, &e->meta[layer], err);
    }
    WB_SET_ERR(err, WISP_ERR_IO, "layer %u: no readable expert file", layer);
    return WISP_ERR_IO;
}

void* fetch_locked(WispEngine* e, uint32_t layer, uint32_t expert,
                   const std::vector<uint64_t>& keep, WispErrCtx* err) {
    wb::Lru::Entry ent;
    // 1. VRAM hit
    if (e->vram.get(layer, expert, &ent)) {
        e->vram.touch(layer, expert);
        stat_hit(e, 0, layer, expert);
        return ent.data;
    }
    // 2. RAM hit: promote after kPromoteHits, else serve through the ring
    if (e->ram.get(layer, expert, &ent)) {
        uint32_t h = e->ram.touch(layer, expert);
        stat_hit(e, 1, layer, expert);
        if (ensure_meta(e, layer, ent.data, ent.bytes, err) != WISP_OK) return nullptr;
        if (h < (uint32_t)kPromoteHits) {
            void* p = scratch_serve(e, ent.data, ent.bytes, err);
            if (p) set_table(e, layer, expert, p, false);
            return p;
        }
        void* slot = vram_alloc_evicting(e, ent.bytes, keep, {wb::Lru::key(layer, expert)});
        if (!slot) {
            void* p = scratch_serve(e, ent.data, ent.bytes, err);
            if (p) set_table(e, layer, expert, p, false);
            return p;
        }
        if (!put_tiled(e, slot, ent.data, ent.bytes, err)) {
            e->arena.release(slot);
            return nullptr;
        }
        e->vram.put(layer, expert, slot, ent.bytes);
        set_table(e, layer, expert, slot, true);
        return slot;
    }
    // 3. SSD miss
    size_t n = read_expert(expert_path(e, layer, expert), e->staging, e->max_expert_bytes, err);
    if (n == 0) return nullptr;
    stat_hit(e, 2, layer, expert);
    if (ensure_meta(e, layer, e->staging, n, err) != WISP_OK) return nullptr;
    // the RAM-tier copy is the upload's source, so the staging buffer is free for
    // the next read at once; without one, the upload from staging is waited for
    void* host = nullptr;
    if (n <= e->ram.capacity() && cudaHostAlloc(&host, n, cudaHostAllocDefault) == cudaSuccess) {
        memcpy(host, e->staging, n);
        if (!ram_put(e, layer, expert, host, n)) host = nullptr;  // freed: upload from staging
    }
    const void* src = host ? host : e->staging;
    void* slot = nullptr;
    if (!e->vram.would_overflow(n)) slot = e->arena.alloc();
    if (!slot) {
        void* p = scratch_serve(e, src, n, err);
        if (p) set_table(e, layer, expert, p, false);
        if (!host) drain_uploads(e);
        return p;
    }
    const bool up = put_tiled(e, slot, src, n, err);
    if (!host) drain_uploads(e);
    if (!up) {
        e->arena.release(slot);
        return nullptr;
    }
    e->vram.put(layer, expert, slot, n);
    set_table(e, layer, expert, slot, true);
    return slot;
}

void prefetch_loop(WispEngine* e) {
    // the RAM-tier buffers this thread pins belong to the engine's device context
    // (a new thread starts on device 0)
    cudaSetDevice(e->device);
    std::vector<char> buf;
    for (;;) {
        std::pair<uint32_t, uint32_t> item;
        {
            std::unique_lock<std::mutex> g(e->q_mu);
            e->q_cv.wait(g, [&] { return e->stop || !e->q.empty(); });
            if (e->stop && e->q.empty()) return;
            item = e->q.front();
            e->q.pop_front();
        }
        if (e->vram.get(item.first, item.second, nullptr) ||
            e->ram.get(item.first, item.second, nullptr))
            continue;
        WispErrCtx err{};
        if (!read_file(expert_path(e, item.first, item.second), buf) || buf.empty()) continue;
        void* host = nullptr;
        if (cudaHostAlloc(&host, buf.size(), cudaHostAllocDefault) != cudaSuccess) continue;
        memcpy(host, buf.data(), buf.size());
        std::lock_guard<std::mutex> g(e->fetch_mu);
        if (!e->meta[item.first].valid)
            wisp_expert_parse_header(host, buf.size(), &e->meta[item.first], &err);
        if (e->ram.get(item.first, item.second, nullptr))
            cudaFreeHost(host);
        else
            ram_put(e, item.first, item.second, host, buf.size());
    }
}

WispError load_half(WispEngine* e, const StFile& st, const std::string& name, wisp_half** out,
                    bool required, WispErrCtx* err, std::vector<int64_t>* shape = nullptr) {
    StTensor t;
    if (!st.find(name, &t)) {
        if (required) {
            WB_SET_ERR(err, WISP_ERR_MODEL, "dense file missing tensor %s", name.c_str());
            return WISP_ERR_MODEL;
        }
        return WISP_OK;
    }
    if (!t.f16) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "tensor %s is not F16", name.c_str());
        return WISP_ERR_MODEL;
    }
    std::vector<char> host(t.bytes);
    if (!st.read(t, host.data())) {
        WB_SET_ERR(err, WISP_ERR_IO, "short read for tensor %s", name.c_str());
        return WISP_ERR_IO;
    }
    WB_CUDA_RET(cudaMalloc(out, t.bytes), err);
    WB_CUDA_RET(cudaMemcpy(*out, host.data(), t.bytes, cudaMemcpyHostToDevice), err);
    if (shape) *shape = t.shape;
    (void)e;
    return WISP_OK;
}

// The fp16-dense shared.{gate,up,down} of layer l (gate/up [si, H], down
// [H, si]; wisp_engine.c:1748-1756).  Absent tensors leave the pointers NULL.
WispError load_dense_shared(WispEngine* e, const StFile& st, int l, WispErrCtx* err) {
    LayerDev& d = e->L[l];
    const std::string p = "layers." + std::to_string(l) + ".shared.";
    std::vector<int64_t> sg, su, sd;
    WispError r = load_half(e, st, p + "gate", &d.shared_gate, false, err, &sg);
    if (r == WISP_OK) r = load_half(e, st, p + "up", &d.shared_up, false, err, &su);
    if (r == WISP_OK) r = load_half(e, st, p + "down", &d.shared_down, false, err, &sd);
    if (r != WISP_OK) return r;
    if (!d.shared_gate && !d.shared_up && !d.shared_down) return WISP_OK;
    const int si = sg.size() == 2 ? (int)sg[0] : 0;
    const bool ok = d.shared_gate && d.shared_up && d.shared_down && sg.size() == 2 &&
                    su.size() == 2 && sd.size() == 2 && sg[1] == e->H && su[0] == si &&
                    su[1] == e->H && sd[0] == e->H && sd[1] == si &&
                    wb::dense_ffn_shape_ok(d.shared_gate, d.shared_up, d.shared_down, si, e->H);
    if (!ok) {
        WB_SET_ERR(err, WISP_ERR_MODEL,
                   "layer %d: shared.{gate,up,down} must be fp16 [si,%d], [si,%d], [%d,si] with "
                   "si a multiple of 8",
                   l, e->H, e->H, e->H);
        return WISP_ERR_MODEL;
    }
    d.shared_inter = si;
    return WISP_OK;
}

WispError ensure_ws(WispEngine* e, const std::vector<WispMoeLayer>& layers, int T,
                    WispErrCtx* err) {
    size_t need = wisp_moe_workspace_bytes(layers.data(), (int)layers.size(), T);
    if (need <= e->ws_bytes) return WISP_OK;
    if (e->ws) {
        cudaStreamSynchronize(e->compute);
        cudaFree(e->ws);
        e->ws = nullptr;
    }
    WB_CUDA_RET(cudaMalloc(&e->ws, need), err);
    e->ws_bytes = need;
    return WISP_OK;
}

WispMoeLayer layer_desc(WispEngine* e, int l) {
    WispMoeLayer d{};
    d.meta = e->meta[l];
    d.meta.tiled = 1;  // device copies are tiled (put_tiled)
    d.expert_blobs = const_cast<const void* const*>(e->L[l].d_table);
    d.router_w = e->L[l].router;
    d.router_bias = e->L[l].router_bias;
    d.norm_w = e->L[l].post_norm;
    d.shared_blob = e->L[l].shared_blob;
    d.shared_meta = e->L[l].shared_meta;
    if (!d.shared_blob && e->L[l].shared_gate) {
        d.shared_gate = e->L[l].shared_gate;
        d.shared_up = e->L[l].shared_up;
        d.shared_down = e->L[l].shared_down;
        d.shared_inter = e->L[l].shared_inter;
    }
    d.n_experts = e->E;
    d.top_k = e->K;
    return d;
}

bool layer_resident(WispEngine* e, int l) {
    return !e->L[l].dense_mlp && e->meta[l].valid && e->L[l].n_vram == e->E;
}

// Grow the engine's per-call device buffers to T tokens.  A grown buffer
// replaces the old one after the device is idle (cudaFree synchronises).
WispError ensure_bufs(WispEngine* e, int T, int si, WispErrCtx* err) {
    const size_t route = (size_t)T * e->K, rows = (size_t)T * e->H, dh = (size_t)T * si;
    if (route > e->cap_route) {
        cudaFree(e->d_idx);
        cudaFree(e->d_w);
        e->d_idx = nullptr;
        e->d_w = nullptr;
        e->cap_route = 0;
        WB_CUDA_RET(cudaMalloc(&e->d_idx, route * sizeof(int)), err);
        WB_CUDA_RET(cudaMalloc(&e->d_w, route * sizeof(float)), err);
        e->cap_route = route;
    }
    if (rows > e->cap_rows) {
        cudaFree(e->d_xn);
        cudaFree(e->d_ffn);
        e->d_xn = e->d_ffn = nullptr;
        e->cap_rows = 0;
        WB_CUDA_RET(cudaMalloc(&e->d_xn, rows * sizeof(float)), err);
        WB_CUDA_RET(cudaMalloc(&e->d_ffn, rows * sizeof(float)), err);
        e->cap_rows = rows;
    }
    if (dh > e->cap_dh) {
        cudaFree(e->d_dh);
        e->d_dh = nullptr;
        e->cap_dh = 0;
        WB_CUDA_RET(cudaMalloc(&e->d_dh, dh * sizeof(float)), err);
        e->cap_dh = dh;
    }
    return WISP_OK;
}

// Work queued on the compute stream (expert-table updates) precedes what the
// caller queues next on `s`.
void order_after_compute(WispEngine* e, cudaStream_t s) {
    if (s == e->compute) return;
    cudaEventRecord(e->order_ev, e->compute);
    cudaStreamWaitEvent(s, e->order_ev, 0);
}

WispError load_shared(WispEngine* e, int l, WispErrCtx* err) {
    char buf[64];
    snprintf(buf, sizeof buf, "/experts/L%03d_shared.bin", l);
    std::vector<char> blob;
    if (!read_file(e->path + buf, blob)) return WISP_OK;  // no int4 shared expert
    WispExpertMeta m{};
    WispError r = wisp_expert_parse_header(blob.data(), blob.size(), &m, err);
    if (r != WISP_OK) return r;
    // the fused block runs an int4 shared expert as one more tile of the routed
    // experts' shape; a shared expert of another width runs from its fp16-dense
    // copy (layers.i.shared.*) instead
    if ((int)m.rows[0] != e->inter || (int)m.cols[0] != e->H) return WISP_OK;
    // the shared expert may be wider than the routed ones (manifest
    // expert_size_bytes): grow the staging slot to hold it (engine creation,
    // nothing else is in flight on the transfer stream)
    if (blob.size() > e->stage_cap) {
        WB_CUDA_RET(cudaStreamSynchronize(e->transfer), err);
        cudaFree(e->d_stage - 8);
        e->d_stage = nullptr;
        char* p = nullptr;
        WB_CUDA_RET(cudaMalloc(&p, blob.size() + 264), err);
        e->d_stage = p + 8;
        e->stage_cap = blob.size();
    }
    // place at (256-aligned) + 8 so the sections are 16-byte aligned
    char* base = nullptr;
    WB_CUDA_RET(cudaMalloc(&base, blob.size() + 264), err);
    void* dst = base + 8;
    if (!put_tiled(e, dst, blob.data(), blob.size(), err)) {
        cudaFree(base);
        return err->code ? err->code : WISP_ERR_CUDA;
    }
    drain_uploads(e);  // `blob` is freed on return
    m.tiled = 1;
    e->L[l].shared_blob = dst;
    e->L[l].shared_meta = m;
    return WISP_OK;
}

}  // namespace

// The decoder step's weights (load_dense, wisp_engine.c:1698-1760, GQA/MHA
// names): embed_tokens [vocab, H], final_norm [H], lm_head [vocab, H], and per
// layer input_norm [H], attn.q_proj [nh*hd, H], attn.k_proj / v_proj
// [nkv*hd, H], attn.o_proj [H, nh*hd] (hd = H / nh, as the reference derives
// it).  A model without them (or with MLA attention) still serves the MoE
// entry points; the decoder calls then report why.
static WispError load_decoder(WispEngine* e, const StFile& st, const char* manifest,
                              WispErrCtx* err) {
    const std::string attn = json_str(manifest, "attention_type");
    e->vocab = (int)json_num(manifest, "vocab_size", 0);
    e->n_heads = (int)json_num(manifest, "num_attention_heads", 128);
    e->n_kv = (int)json_num(manifest, "num_kv_heads", e->n_heads);
    e->rope_theta = (float)json_num(manifest, "rope_theta", 10000.0);
    if (attn != "GQA" && attn != "MHA") {
        e->no_decoder = "attention type '" + attn + "' (the decoder step supports GQA and MHA)";
        return WISP_OK;
    }
    if (e->n_heads <= 0 || e->n_kv <= 0 || e->n_heads % e->n_kv || e->H % e->n_heads ||
        e->vocab <= 0) {
        e->no_decoder = "manifest heads / kv heads / vocab do not describe a GQA model";
        return WISP_OK;
    }
    e->head_dim = e->H / e->n_heads;
    const int64_t H = e->H, nh = e->n_heads, nkv = e->n_kv, hd = e->head_dim;
    std::vector<int64_t> sh;
    auto want = [&](const std::string& name, wisp_half** out, std::vector<int64_t> shape) -> int {
        WispError r = load_half(e, st, name, out, false, err, &sh);
        if (r != WISP_OK) return -1;
        if (!*out) return 0;
        if (sh != shape) {
            cudaFree(*out);
            *out = nullptr;
            if (e->no_decoder.empty()) e->no_decoder = "tensor " + name + " has an unexpected shape";
            return 0;
        }
        return 1;
    };
    int ok = 1;
    for (auto [name, out, shape] : {std::make_tuple(std::string("embed_tokens"), &e->embed,
                                                    std::vector<int64_t>{e->vocab, H}),
                                    std::make_tuple(std::string("final_norm"), &e->final_norm,
                                                    std::vector<int64_t>{H}),
                                    std::make_tuple(std::string("lm_head"), &e->lm_head,
                                                    std::vector<int64_t>{e->vocab, H})}) {
        const int r = want(name, out, shape);
        if (r < 0) return err->code;
        ok &= r;
    }
    for (int l = 0; l < e->n_layers && ok; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        LayerDev& d = e->L[l];
        const std::pair<std::string, std::pair<wisp_half**, std::vector<int64_t>>> t[] = {
            {p + "input_norm", {&d.input_norm, {H}}},
            {p + "attn.q_proj", {&d.q_proj, {nh * hd, H}}},
            {p + "attn.k_proj", {&d.k_proj, {nkv * hd, H}}},
            {p + "attn.v_proj", {&d.v_proj, {nkv * hd, H}}},
            {p + "attn.o_proj", {&d.o_proj, {H, nh * hd}}}};
        for (const auto& it : t) {
            const int r = want(it.first, it.second.first, it.second.second);
            if (r < 0) return err->code;
            if (r == 0 && it.first != p + "input_norm") {
                ok = 0;
                if (e->no_decoder.empty()) e->no_decoder = "tensor " + it.first + " missing";
            }
        }
    }
    if (!ok) {
        if (e->no_decoder.empty()) e->no_decoder = "embed_tokens / final_norm / lm_head missing";
        return WISP_OK;
    }
    WB_CUDA_RET(cudaMalloc(&e->d_x, (size_t)H * sizeof(float)), err);
    WB_CUDA_RET(cudaMalloc(&e->d_lmws, (size_t)H * sizeof(float)), err);
    WB_CUDA_RET(cudaMalloc(&e->d_logits, (size_t)e->vocab * sizeof(float)), err);
    e->has_decoder = true;
    return WISP_OK;
}

extern "C" size_t wisp_read_expert_file(const char* path, void* dst, size_t cap, int* direct,
                                        WispErrCtx* err) {
    return read_file_into(path, dst, cap, direct, err);
}

// ====================================================================== ABI

extern "C" WispError wisp_expert_parse_header(const void* blob, size_t blob_size,
                                              WispExpertMeta* meta, WispErrCtx* err) {
    if (!blob || !meta) {
        WB_SET_ERR(err, WISP_ERR_OOM, "NULL pointer: expert_parse_header");
        return WISP_ERR_OOM;
    }
    if (blob_size < 120) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "expert blob too small: %zu bytes", blob_size);
        return WISP_ERR_MODEL;
    }
    uint32_t h[6];
    memcpy(h, blob, sizeof h);
    if (h[0] != kMagic || (h[1] != 1u && h[1] != 2u) || h[5] != 3u) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "expert blob corrupt: magic=%08x version=%u n_mats=%u",
                   h[0], h[1], h[5]);
        return WISP_ERR_MODEL;
    }
    const uint8_t* b = static_cast<const uint8_t*>(blob);
    size_t off = 120;
    for (int m = 0; m < 3; ++m) {
        uint32_t rc[2];
        uint64_t sz[3];
        memcpy(rc, b + 24 + 32 * m, 8);
        memcpy(sz, b + 24 + 32 * m + 8, 24);
        meta->rows[m] = rc[0];
        meta->cols[m] = rc[1];
        meta->packed_off[m] = off;
        off += sz[0];
        meta->scales_off[m] = off;
        off += sz[1];
        meta->zeros_off[m] = off;
        off += sz[2];
    }
    meta->group_size = h[4];
    meta->total_bytes = off;
    meta->valid = 1;
    meta->tiled = h[1] == 2u ? 1 : 0;
    if (off > blob_size) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "expert blob truncated: needs %zu, have %zu", off,
                   blob_size);
        meta->valid = 0;
        return WISP_ERR_MODEL;
    }
    return WISP_OK;
}

extern "C" WispError wisp_debug_expert_probe(const char* path, int mat, int n, float* out,
                                             WispExpertMeta* out_meta, WispErrCtx* err) {
    if (!path || !out) {
        WB_SET_ERR(err, WISP_ERR_OOM, "NULL pointer: debug_probe");
        return WISP_ERR_OOM;
    }
    if (mat < 0 || mat >= 3 || n <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "debug_probe: mat=%d n=%d", mat, n);
        return WISP_ERR_INVALID_ARG;
    }
    std::vector<char> blob;
    if (!read_file(path, blob)) {
        WB_SET_ERR(err, WISP_ERR_IO, "debug_probe: cannot read %s", path);
        return WISP_ERR_IO;
    }
    WispExpertMeta m{};
    WispError r = wisp_expert_parse_header(blob.data(), blob.size(), &m, err);
    if (r != WISP_OK) return r;
    size_t total = (size_t)m.rows[mat] * m.cols[mat];
    if ((size_t)n > total) n = (int)total;
    const uint8_t* packed = reinterpret_cast<const uint8_t*>(blob.data() + m.packed_off[mat]);
    const __half* sc = reinterpret_cast<const __half*>(blob.data() + m.scales_off[mat]);
    const __half* ze = reinterpret_cast<const __half*>(blob.data() + m.zeros_off[mat]);
    for (int i = 0; i < n; ++i) {
        int code = (i & 1) ? (packed[i >> 1] >> 4) : (packed[i >> 1] & 0xF);
        size_t g = (size_t)i / m.group_size;
        out[i] = (float)(code - 8) * __half2float(sc[g]) + __half2float(ze[g]);
    }
    if (out_meta) *out_meta = m;
    return WISP_OK;
}

extern "C" WispEngine* wisp_engine_create(const char* model_path, size_t vram_budget,
                                          size_t ram_budget, const int* gpu_indices,
                                          int gpu_count, int omp_threads, WispErrCtx* err) {
    (void)omp_threads;  // no CPU compute path in this engine
    if (!model_path || !err) return nullptr;
    err->code = WISP_OK;
    if (gpu_count <= 0 || !gpu_indices) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "engine_create: this engine runs on a GPU only (gpu_count=%d)", gpu_count);
        return nullptr;
    }
    std::unique_ptr<WispEngine> e(new WispEngine());
    e->path = model_path;
    e->device = gpu_indices[0];
    cudaError_t ce = cudaSetDevice(e->device);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "cudaSetDevice(%d): %s", e->device, cudaGetErrorString(ce));
        return nullptr;
    }
    std::vector<char> js;
    if (!read_file(e->path + "/manifest.json", js)) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "cannot read %s/manifest.json", model_path);
        return nullptr;
    }
    js.push_back(0);
    const char* j = js.data();
    e->n_layers = (int)json_num(j, "num_layers", 0);
    e->E = (int)json_num(j, "num_experts_per_layer", 0);
    e->K = (int)json_num(j, "top_k_routing", 8);
    e->H = (int)json_num(j, "hidden_size", 0);
    e->inter = (int)json_num(j, "moe_intermediate_size", 2048);
    e->eps = (float)json_num(j, "rms_norm_eps", 1e-6);
    e->gs = (int)json_num(j, "group_size", 64);
    e->expert_bytes = (size_t)json_num(j, "expert_size_bytes", 18350080);
    if (e->n_layers <= 0 || e->H <= 0 || e->E <= 0 || e->K <= 0 || e->K > e->E) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "manifest invalid: layers=%d hidden=%d experts=%d top_k=%d",
                   e->n_layers, e->H, e->E, e->K);
        return nullptr;
    }
    e->max_expert_bytes = e->expert_bytes + e->expert_bytes / 4 + 4096;
    ce = cudaStreamCreateWithFlags(&e->compute, cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&e->transfer, cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->order_ev, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->up_ev, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->evict_ev, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaHostAlloc(&e->staging, e->max_expert_bytes, 0);
    if (ce == cudaSuccess) ce = cudaMalloc(&e->d_stage, e->max_expert_bytes + 264);
    if (ce == cudaSuccess) e->d_stage += 8;  // blob at 8 (mod 16), like every slot
    e->stage_cap = e->max_expert_bytes;
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "stream/staging setup: %s", cudaGetErrorString(ce));
        wisp_engine_destroy(e.release());
        return nullptr;
    }
    // dense weights
    StFile st;
    if (!st.open(e->path + "/dense/model_dense.safetensors")) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "cannot open dense weights: %s/dense/model_dense.safetensors",
                   model_path);
        wisp_engine_destroy(e.release());
        return nullptr;
    }
    e->L.resize(e->n_layers);
    e->meta.assign(e->n_layers, WispExpertMeta{});
    for (int l = 0; l < e->n_layers; ++l) {
        std::string p = "layers." + std::to_string(l) + ".";
        LayerDev& d = e->L[l];
        if (load_half(e.get(), st, p + "router", &d.router, false, err) != WISP_OK ||
            load_half(e.get(), st, p + "router_bias", &d.router_bias, false, err) != WISP_OK ||
            load_half(e.get(), st, p + "post_norm", &d.post_norm, false, err) != WISP_OK) {
            wisp_engine_destroy(e.release());
            return nullptr;
        }
        d.dense_mlp = d.router == nullptr;
        // the int4 shared blob when this build's converter wrote one, else the
        // reference's fp16-dense shared.* (also the whole FFN of a dense-MLP layer)
        WispError sr = d.dense_mlp ? WISP_OK : load_shared(e.get(), l, err);
        if (sr == WISP_OK && !d.shared_blob) sr = load_dense_shared(e.get(), st, l, err);
        if (sr == WISP_OK && d.dense_mlp && !d.shared_gate) {
            WB_SET_ERR(err, WISP_ERR_MODEL, "layer %d: no router and no dense MLP weights", l);
            sr = WISP_ERR_MODEL;
        }
        if (sr != WISP_OK) {
            wisp_engine_destroy(e.release());
            return nullptr;
        }
        d.h_table.assign(e->E, nullptr);
        d.in_vram.assign(e->E, 0);
        ce = cudaMalloc(&d.d_table, (size_t)e->E * sizeof(void*));
        if (ce == cudaSuccess) ce = cudaMemset(d.d_table, 0, (size_t)e->E * sizeof(void*));
        if (ce != cudaSuccess) {
            WB_SET_ERR(err, WISP_ERR_CUDA, "expert table alloc: %s", cudaGetErrorString(ce));
            wisp_engine_destroy(e.release());
            return nullptr;
        }
    }
    if (load_decoder(e.get(), st, j, err) != WISP_OK) {
        wisp_engine_destroy(e.release());
        return nullptr;
    }
    // tiers
    e->ram.set_capacity(ram_budget);
    e->vram_budget = vram_budget;
    e->vram.set_capacity(vram_budget);
    size_t n_slots = e->max_expert_bytes ? vram_budget / e->max_expert_bytes : 0;
    ce = e->arena.init(e->max_expert_bytes, n_slots);
    int ring_n = std::min(e->E, std::max(e->K + 2, 16));
    if (ce == cudaSuccess) ce = e->ring_arena.init(e->max_expert_bytes, (size_t)ring_n);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_OOM, "VRAM expert arena (%zu slots): %s", n_slots,
                   cudaGetErrorString(ce));
        wisp_engine_destroy(e.release());
        return nullptr;
    }
    for (int i = 0; i < ring_n; ++i) e->ring.push_back(e->ring_arena.alloc());
    int cap = e->K * e->n_layers * 16;
    cap = std::max(4096, std::min(cap, 1 << 20));
    e->log.assign((size_t)cap, 0);
    WispEngine* raw = e.release();
    raw->worker = std::thread(prefetch_loop, raw);
    return raw;
}

extern "C" void wisp_engine_destroy(WispEngine* e) {
    if (!e) return;
    if (e->worker.joinable()) {
        {
            std::lock_guard<std::mutex> g(e->q_mu);
            e->stop = true;
        }
        e->q_cv.notify_all();
        e->worker.join();
    }
    if (e->compute) cudaStreamSynchronize(e->compute);
    if (e->transfer) cudaStreamSynchronize(e->transfer);
    e->ram.clear([](const wb::Lru::Entry& v) { cudaFreeHost(v.data); });
    e->vram.clear([](const wb::Lru::Entry&) {});
    for (auto& d : e->L) {
        cudaFree(d.router);
        cudaFree(d.router_bias);
        cudaFree(d.post_norm);
        if (d.shared_blob) cudaFree(static_cast<char*>(d.shared_blob) - 8);
        cudaFree(d.shared_gate);
        cudaFree(d.shared_up);
        cudaFree(d.shared_down);
        cudaFree(d.d_table);
        cudaFree(d.input_norm);
        cudaFree(d.q_proj);
        cudaFree(d.k_proj);
        cudaFree(d.v_proj);
        cudaFree(d.o_proj);
    }
    cudaFree(e->embed);
    cudaFree(e->final_norm);
    cudaFree(e->lm_head);
    cudaFree(e->d_x);
    cudaFree(e->d_lmws);
    cudaFree(e->d_logits);
    if (e->ws) cudaFree(e->ws);
    cudaFree(e->d_idx);
    cudaFree(e->d_w);
    cudaFree(e->d_xn);
    cudaFree(e->d_ffn);
    cudaFree(e->d_dh);
    if (e->order_ev) cudaEventDestroy(e->order_ev);
    if (e->up_ev) cudaEventDestroy(e->up_ev);
    if (e->evict_ev) cudaEventDestroy(e->evict_ev);
    if (e->staging) cudaFreeHost(e->staging);
    if (e->d_stage) cudaFree(e->d_stage - 8);
    if (e->compute) cudaStreamDestroy(e->compute);
    if (e->transfer) cudaStreamDestroy(e->transfer);
    delete e;
}

extern "C" void* wisp_expert_fetch(WispEngine* e, uint32_t layer, uint32_t expert,
                                   WispErrCtx* err) {
    if (!e || layer >= (uint32_t)e->n_layers || expert >= (uint32_t)e->E) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "expert_fetch: L%u/E%u out of range", layer,
                   expert);
        return nullptr;
    }
    cudaSetDevice(e->device);
    std::lock_guard<std::mutex> g(e->fetch_mu);
    void* p = fetch_locked(e, layer, expert, {}, err);
    // the reference's contract: the returned slot holds the expert
    drain_uploads(e);
    return p;
}

extern "C" void wisp_expert_prefetch_hint(WispEngine* e, int layer, const int* ids, int n) {
    if (!e || layer < 0 || layer >= e->n_layers || !ids) return;
    std::lock_guard<std::mutex> g(e->q_mu);
    for (int i = 0; i < n && (int)e->q.size() < kPrefetchRing; ++i) {
        if (ids[i] < 0 || ids[i] >= e->E) continue;
        e->q.emplace_back((uint32_t)layer, (uint32_t)ids[i]);
    }
    e->q_cv.notify_one();
}

extern "C" int wisp_engine_pin_experts(WispEngine* e, int layer0, int n, WispErrCtx* err) {
    if (!e) return 0;
    cudaSetDevice(e->device);
    std::lock_guard<std::mutex> g(e->fetch_mu);
    int resident = 0;
    for (int l = layer0; l < layer0 + n && l < e->n_layers; ++l) {
        if (e->L[l].dense_mlp) continue;  // no routed experts
        for (int x = 0; x < e->E; ++x) {
            if (e->L[l].in_vram[x]) {
                ++resident;
                continue;
            }
            WispErrCtx le{};
            wb::Lru::Entry ent;
            void* host = nullptr;
            size_t bytes = 0;
            if (e->ram.get(l, x, &ent)) {
                host = ent.data;
                bytes = ent.bytes;
            } else {
                bytes = read_expert(expert_path(e, l, x), e->staging, e->max_expert_bytes, &le);
                if (!bytes) {
                    if (err) *err = le;
                    continue;
                }
                host = e->staging;
            }
            if (ensure_meta(e, l, host, bytes, &le) != WISP_OK) {
                if (err) *err = le;
                continue;
            }
            if (e->vram.would_overflow(bytes)) return resident;
            void* slot = e->arena.alloc();
            if (!slot) return resident;
            const bool up = put_tiled(e, slot, host, bytes, &le);
            if (host == e->staging) drain_uploads(e);  // staging is read into next
            if (!up) {
                e->arena.release(slot);
                if (err) *err = le;
                return resident;
            }
            e->vram.put(l, x, slot, bytes);
            set_table(e, l, x, slot, true);
            ++resident;
        }
    }
    drain_uploads(e);
    cudaStreamSynchronize(e->compute);
    return resident;
}

extern "C" cudaStream_t wisp_engine_stream(WispEngine* e) { return e ? e->compute : nullptr; }

extern "C" void wisp_engine_dims(WispEngine* e, int* hidden, int* n_experts, int* top_k,
                                 int* n_layers) {
    if (!e) return;
    if (hidden) *hidden = e->H;
    if (n_experts) *n_experts = e->E;
    if (top_k) *top_k = e->K;
    if (n_layers) *n_layers = e->n_layers;
}

static WispError moe_forward_impl(WispEngine* e, int l, const float* x, float* y, int T,
                                  cudaStream_t s, WispErrCtx* err) {
    LayerDev& ld = e->L[l];
    if (ld.dense_mlp) {
        // run_dense_mlp (wisp_engine.c:1524-1534): the fp16-dense SwiGLU FFN alone
        WispError br = ensure_bufs(e, T, ld.shared_inter, err);
        if (br != WISP_OK) return br;
        WB_CUDA_RET(wb::launch_dense_ffn(reinterpret_cast<const __half*>(ld.shared_gate),
                                     reinterpret_cast<const __half*>(ld.shared_up),
                                     reinterpret_cast<const __half*>(ld.shared_down),
                                     ld.shared_inter, e->H, x, e->H, e->d_dh, y, e->H, T, s),
                    err);
        return WISP_OK;
    }
    if (!e->meta[l].valid) {
        // nothing of this layer parsed yet: the layout is in any blob's header
        std::lock_guard<std::mutex> g(e->fetch_mu);
        WispError hr = meta_from_file(e, (uint32_t)l, err);
        if (hr != WISP_OK) return hr;
    }
    if (!sections_aligned(e->meta[l])) {
        WB_SET_ERR(err, WISP_ERR_MODEL,
                   "layer %d: expert section sizes are not multiples of 16 bytes", l);
        return WISP_ERR_MODEL;
    }
    std::vector<WispMoeLayer> d{layer_desc(e, l)};
    WispError r = ensure_ws(e, d, T, err);
    if (r != WISP_OK) return r;
    if (layer_resident(e, l))
        return wisp_moe_block_forward(&d[0], x, y, T, nullptr, nullptr, e->ws, e->ws_bytes, s,
                                      err);
    // miss path: the fused router decides, the host fetches what it chose, then the
    // expert kernels run on that same plan
    r = ensure_bufs(e, T, 0, err);
    if (r != WISP_OK) return r;
    r = wisp_moe_block_route(&d[0], x, T, e->d_idx, e->d_w, e->ws, e->ws_bytes, s, err);
    if (r != WISP_OK) return r;
    std::vector<int>& idx = e->h_idx;
    idx.assign((size_t)T * e->K, -1);
    cudaError_t ce = cudaMemcpyAsync(idx.data(), e->d_idx, idx.size() * sizeof(int),
                                     cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "router readback: %s", cudaGetErrorString(ce));
        return WISP_ERR_CUDA;
    }
    std::vector<int> uniq;
    for (int v : idx)
        if (v >= 0) uniq.push_back(v);
    std::sort(uniq.begin(), uniq.end());
    uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
    std::vector<uint64_t> keep;
    for (int v : uniq) keep.push_back(wb::Lru::key((uint32_t)l, (uint32_t)v));
    std::vector<int> missing;
    {
        int ring_used = 0;
        std::lock_guard<std::mutex> g(e->fetch_mu);
        for (int v : uniq) {
            WispErrCtx fe{};
            void* p = fetch_locked(e, (uint32_t)l, (uint32_t)v, keep, &fe);
            if (!p) {
                // run_moe skips an expert whose file cannot be read and combines
                // the others (wisp_engine.c:1473-1477, 1502-1506)
                if (fe.code == WISP_ERR_IO) {
                    missing.push_back(v);
                    continue;
                }
                if (err) *err = fe;
                return fe.code == WISP_OK ? WISP_ERR_EXPERT_MISS : fe.code;
            }
            if (!e->L[l].in_vram[v] && ++ring_used > (int)e->ring.size()) {
                WB_SET_ERR(err, WISP_ERR_OOM,
                           "layer %d routes %zu cold experts for %d tokens; raise the VRAM "
                           "budget (scratch ring holds %zu)",
                           l, uniq.size(), T, e->ring.size());
                return WISP_ERR_OOM;
            }
        }
    }
    if (!missing.empty()) {
        // the skipped experts' slots leave the plan and the combine (index -1); the
        // other weights stay as routed, as in the reference
        for (int& v : idx)
            if (std::binary_search(missing.begin(), missing.end(), v)) v = -1;
        WB_CUDA_RET(cudaMemcpyAsync(e->d_idx, idx.data(), idx.size() * sizeof(int),
                                    cudaMemcpyHostToDevice, s),
                    err);
    }
    // table updates were queued on the compute stream, the uploads on the
    // transfer stream
    order_after_compute(e, s);
    wait_uploads(e, s);
    return wisp_moe_block_experts(&d[0], x, y, T, e->d_idx, e->d_w, e->ws, e->ws_bytes, s, err);
}

extern "C" WispError wisp_moe_forward(WispEngine* e, int layer, const float* x, float* y, int T,
                                      cudaStream_t stream, WispErrCtx* err) {
    if (!e || layer < 0 || layer >= e->n_layers || !x || !y || T <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_forward: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    cudaSetDevice(e->device);
    cudaStream_t s = stream ? stream : e->compute;
    // pending table updates on the compute stream and uploads must land first
    order_after_compute(e, s);
    wait_uploads(e, s);
    return moe_forward_impl(e, layer, x, y, T, s, err);
}

extern "C" WispError wisp_moe_decode(WispEngine* e, int layer, const float* x, float* y,
                                     cudaStream_t stream, WispErrCtx* err) {
    return wisp_moe_forward(e, layer, x, y, 1, stream, err);
}

// x <- x + FFN_l(rmsnorm(x; post_norm_l)) for the layers [layer0, layer0 + n) on
// stream s (the FFN half of decode_step, wisp_engine.c:1563-1570).  A run of
// VRAM-resident MoE layers is one fused stack (the norm in the router kernel, the
// residual in the final combine); a layer on the miss path or a dense MLP runs
// as norm, FFN and residual add.
static WispError ffn_layers(WispEngine* e, int layer0, int n, float* x, int T, cudaStream_t s,
                            WispErrCtx* err) {
    WispError r = WISP_OK;
    for (int l = layer0; l < layer0 + n && r == WISP_OK;) {
        // a run of VRAM-resident MoE layers: one fused stack, no host synchronisation
        int j = l;
        while (j < layer0 + n && layer_resident(e, j)) ++j;
        if (j > l) {
            std::vector<WispMoeLayer> d;
            for (int q = l; q < j; ++q) d.push_back(layer_desc(e, q));
            r = ensure_ws(e, d, T, err);
            if (r == WISP_OK)
                r = wisp_moe_stack_forward(d.data(), j - l, e->eps, x, T, nullptr, nullptr, e->ws,
                                           e->ws_bytes, s, err);
            l = j;
            continue;
        }
        // one layer with the miss path or a dense MLP: xn = rmsnorm(x); x += ffn(xn)
        r = ensure_bufs(e, T, 0, err);
        if (r != WISP_OK) break;
        WB_CUDA_RET(wb::launch_rmsnorm_rows(x, reinterpret_cast<const __half*>(e->L[l].post_norm),
                                        e->d_xn, e->H, e->eps, T, s),
                    err);
        r = moe_forward_impl(e, l, e->d_xn, e->d_ffn, T, s, err);
        if (r == WISP_OK) WB_CUDA_RET(wb::launch_add_rows(x, e->d_ffn, (size_t)T * e->H, s), err);
        ++l;
    }
    return r;
}

extern "C" WispError wisp_moe_stack(WispEngine* e, int layer0, int n, float* x, int T,
                                    cudaStream_t stream, WispErrCtx* err) {
    if (!e || layer0 < 0 || n <= 0 || layer0 + n > e->n_layers || !x || T <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_stack: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    cudaSetDevice(e->device);
    cudaStream_t s = stream ? stream : e->compute;
    order_after_compute(e, s);
    wait_uploads(e, s);
    const WispError r = ffn_layers(e, layer0, n, x, T, s, err);
    std::lock_guard<std::mutex> g(e->stats_mu);
    e->tok_ns[e->tok_head] = now_ns();
    e->tok_head = (e->tok_head + 1) % 32;
    if (e->tok_count < 32) e->tok_count++;
    return r;
}

extern "C" void wisp_cache_stats(WispEngine* e, uint64_t* v, uint64_t* r, uint64_t* s,
                                 double* rate) {
    uint64_t a, b, c;
    {
        std::lock_guard<std::mutex> g(e->stats_mu);
        a = e->hits[0];
        b = e->hits[1];
        c = e->hits[2];
    }
    if (v) *v = a;
    if (r) *r = b;
    if (s) *s = c;
    uint64_t tot = a + b + c;
    if (rate) *rate = tot ? (double)(a + b) / (double)tot : 0.0;
}

extern "C" void wisp_cache_clear_all(WispEngine* e) {
    std::lock_guard<std::mutex> g(e->fetch_mu);
    cudaStreamSynchronize(e->compute);
    drain_uploads(e);  // slots and host buffers about to be released may be in flight
    e->vram.clear([&](const wb::Lru::Entry& v) {
        set_table(e, v.layer, v.expert, nullptr, false);
        e->arena.release(v.data);
    });
    e->ram.clear([](const wb::Lru::Entry& v) { cudaFreeHost(v.data); });
    std::lock_guard<std::mutex> s(e->stats_mu);
    e->hits[0] = e->hits[1] = e->hits[2] = 0;
}

extern "C" int wisp_ram_trim(WispEngine* e, int count) {
    if (!e || count <= 0) return 0;
    std::lock_guard<std::mutex> g(e->fetch_mu);
    drain_uploads(e);  // the freed buffers may be sources of uploads in flight
    int freed = 0;
    wb::Lru::Entry v;
    while (freed < count && e->ram.evict(&v)) {
        cudaFreeHost(v.data);
        ++freed;
    }
    return freed;
}

extern "C" int wisp_drain_expert_log(WispEngine* e, uint32_t* out, int max_out,
                                     uint64_t* dropped) {
    if (!e || !out || max_out <= 0) return 0;
    std::lock_guard<std::mutex> g(e->stats_mu);
    int cap = (int)e->log.size();
    int n = std::min(e->log_count, max_out);
    int start = ((e->log_head - e->log_count) % cap + cap) % cap;
    for (int i = 0; i < n; ++i) out[i] = e->log[(start + i) % cap];
    if (dropped) *dropped = e->log_dropped;
    e->log_count = 0;
    e->log_head = 0;
    e->log_dropped = 0;
    return n;
}

extern "C" size_t wisp_vram_used(WispEngine* e) { return e ? (size_t)e->vram.used() : 0; }
extern "C" size_t wisp_ram_used(WispEngine* e) { return e ? (size_t)e->ram.used() : 0; }

extern "C" double wisp_tok_per_sec(WispEngine* e) {
    std::lock_guard<std::mutex> g(e->stats_mu);
    int n = e->tok_count;
    if (n < 2) return 0.0;
    int newest = (e->tok_head + 31) % 32, oldest = (e->tok_head + 32 - n) % 32;
    uint64_t span = e->tok_ns[newest] - e->tok_ns[oldest];
    return span ? (double)(n - 1) * 1e9 / (double)span : 0.0;
}

// wisp_b200_version() is generated at build time (wisp_b200/build.py): it carries
// a hash of the sources the library was built from.

// ------------------------------------------------------------------------
// The decoder step (decode_step, wisp_engine.c:1537-1595) on the device:
// embedding, per layer x += attention(rmsnorm(x)) (wisp_attn_decode) and
// x += FFN(rmsnorm(x)) (the MoE block through the tiers, or the dense MLP),
// then lm_head over rmsnorm(x) when logits are wanted.
// ------------------------------------------------------------------------
extern "C" int wisp_engine_vocab(WispEngine* e) { return e && e->has_decoder ? e->vocab : 0; }

static bool decoder_ready(WispEngine* e, WispErrCtx* err, const char* what) {
    if (!e) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "%s: NULL engine", what);
        return false;
    }
    if (!e->has_decoder) {
        WB_SET_ERR(err, WISP_ERR_MODEL, "%s: the model has no decoder step this build runs: %s",
                   what, e->no_decoder.c_str());
        return false;
    }
    return true;
}

static WispAttnLayer attn_desc(WispEngine* e, int l) {
    const LayerDev& d = e->L[l];
    WispAttnLayer a{};
    a.input_norm = d.input_norm;
    a.q_proj = d.q_proj;
    a.k_proj = d.k_proj;
    a.v_proj = d.v_proj;
    a.o_proj = d.o_proj;
    a.hidden = e->H;
    a.n_heads = e->n_heads;
    a.n_kv_heads = e->n_kv;
    a.head_dim = e->head_dim;
    a.rope_theta = e->rope_theta;
    a.rms_eps = e->eps;
    return a;
}

extern "C" WispKVCache* wisp_kv_cache_alloc(WispEngine* e, int max_seq_len, WispErrCtx* err) {
    if (!decoder_ready(e, err, "kv_cache_alloc")) return nullptr;
    if (max_seq_len <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "max_seq_len must be > 0, got %d", max_seq_len);
        return nullptr;
    }
    cudaSetDevice(e->device);
    std::unique_ptr<WispKVCache> kv(new WispKVCache());
    kv->max_seq = max_seq_len;
    kv->device = e->device;
    kv->layer_elems = (size_t)max_seq_len * e->n_kv * e->head_dim;
    const size_t bytes = (size_t)e->n_layers * kv->layer_elems * sizeof(wisp_half);
    const WispAttnLayer a = attn_desc(e, 0);
    kv->ws_bytes = wisp_attn_workspace_bytes(&a, max_seq_len);
    cudaError_t ce = cudaMalloc(&kv->k, bytes);
    if (ce == cudaSuccess) ce = cudaMalloc(&kv->v, bytes);
    if (ce == cudaSuccess) ce = cudaMalloc(&kv->ws, kv->ws_bytes);
    if (ce == cudaSuccess) ce = cudaMemset(kv->ws, 0, kv->ws_bytes);  // the split-K counters
    if (ce != cudaSuccess) {
        cudaFree(kv->k);
        cudaFree(kv->v);
        cudaFree(kv->ws);
        WB_SET_ERR(err, WISP_ERR_OOM, "kv cache of %d positions (%zu bytes): %s", max_seq_len,
                   2 * bytes, cudaGetErrorString(ce));
        return nullptr;
    }
    return kv.release();
}

extern "C" void wisp_kv_cache_free(WispEngine* e, WispKVCache* kv) {
    if (!kv) return;
    if (e && e->compute) cudaStreamSynchronize(e->compute);
    cudaFree(kv->k);
    cudaFree(kv->v);
    cudaFree(kv->ws);
    delete kv;
}

extern "C" void wisp_kv_cache_clear(WispEngine* e, WispKVCache* kv) {
    (void)e;
    if (kv) kv->len = 0;
}

extern "C" void wisp_kv_cache_rollback(WispEngine* e, WispKVCache* kv, int n_tokens) {
    (void)e;
    if (!kv || n_tokens <= 0) return;
    kv->len = kv->len >= n_tokens ? kv->len - n_tokens : 0;
}

extern "C" int wisp_kv_cache_len(const WispKVCache* kv) { return kv ? kv->len : 0; }

static WispError decode_step(WispEngine* e, WispKVCache* kv, int token, float* out_logits,
                             WispErrCtx* err) {
    if (!decoder_ready(e, err, "decode")) return err->code;
    if (!kv) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "decode: NULL kv cache");
        return WISP_ERR_INVALID_ARG;
    }
    if (token < 0 || token >= e->vocab) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "token id %d out of range [0, %d)", token, e->vocab);
        return WISP_ERR_INVALID_ARG;
    }
    if (kv->len >= kv->max_seq) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "KV cache full (%d tokens)", kv->max_seq);
        return WISP_ERR_INVALID_ARG;
    }
    cudaSetDevice(e->device);
    cudaStream_t s = e->compute;
    order_after_compute(e, s);
    wait_uploads(e, s);
    WispError r = ensure_bufs(e, 1, 0, err);
    if (r != WISP_OK) return r;
    wisp_gpu_embed_lookup(e->embed, token, e->d_x, e->H, s);
    WB_CUDA_RET(cudaGetLastError(), err);
    for (int l = 0; l < e->n_layers; ++l) {
        const WispAttnLayer a = attn_desc(e, l);
        r = wisp_attn_decode(&a, e->d_x, kv->k + (size_t)l * kv->layer_elems,
                             kv->v + (size_t)l * kv->layer_elems, kv->len, kv->max_seq, kv->ws,
                             kv->ws_bytes, s, err);
        if (r != WISP_OK) return r;
        r = ffn_layers(e, l, 1, e->d_x, 1, s, err);
        if (r != WISP_OK) return r;
    }
    kv->len++;
    if (out_logits) {
        r = wisp_lm_head_forward(e->final_norm, e->lm_head, e->d_x, e->d_logits, e->vocab, e->H,
                                 e->eps, e->d_lmws, (size_t)e->H * sizeof(float), s, err);
        if (r != WISP_OK) return r;
        WB_CUDA_RET(cudaMemcpyAsync(out_logits, e->d_logits, (size_t)e->vocab * sizeof(float),
                                    cudaMemcpyDeviceToHost, s),
                    err);
        WB_CUDA_RET(cudaStreamSynchronize(s), err);
    }
    std::lock_guard<std::mutex> g(e->stats_mu);
    e->tok_ns[e->tok_head] = now_ns();
    e->tok_head = (e->tok_head + 1) % 32;
    if (e->tok_count < 32) e->tok_count++;
    return WISP_OK;
}

extern "C" WispError wisp_decode_one(WispEngine* e, int token_id, WispKVCache* kv,
                                     float* out_logits, WispErrCtx* err) {
    return decode_step(e, kv, token_id, out_logits, err);
}

extern "C" WispError wisp_prefill(WispEngine* e, const int* token_ids, int n_tokens,
                                  WispKVCache* kv, float* out_logits, WispErrCtx* err) {
    if (!token_ids || n_tokens <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: empty prompt");
        return WISP_ERR_INVALID_ARG;
    }
    for (int i = 0; i < n_tokens; ++i) {
        const bool want = i == n_tokens - 1 && out_logits;
        const WispError r = decode_step(e, kv, token_ids[i], want ? out_logits : nullptr, err);
        if (r != WISP_OK) return r;
    }
    return WISP_OK;
}

extern "C" WispError wisp_verify_tokens(WispEngine* e, const int* token_ids, int n_tokens,
                                        WispKVCache* kv, float* out_logits, WispErrCtx* err) {
    if (!out_logits || !token_ids || n_tokens < 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "verify: NULL output buffer or tokens");
        return WISP_ERR_INVALID_ARG;
    }
    for (int i = 0; i < n_tokens; ++i) {
        const WispError r = decode_step(e, kv, token_ids[i],
                                        out_logits + (size_t)i * (e ? e->vocab : 0), err);
        if (r != WISP_OK) return r;
    }
    return WISP_OK;
}
