// moe_kernels.cu -- the fused MoE block for sm_100a.
//
// What one block computes (reference: csrc/core/wisp_engine.c:1411-1522 with
// the CPU branch's arithmetic, :520-579 and :1383-1409):
//
//   logits = W_r x + b ; p = softmax(logits) ; idx = k strict-argmax passes
//   (lowest index wins ties) ; w = p[idx] / sum(p[idx])
//   y = [shared(x)] + sum_j w_j * Down_j( silu(Gate_j x) * (Up_j x) )
//
// with every expert matrix int4 in the WISP .bin layout: code c, fp16 scale s
// and zero z per group of gs (64) row-major elements, weight = (c-8)*s + z.
//
// Launch sequence per layer (programmatic dependent launch throughout, so a
// kernel's prologue overlaps the previous kernel's tail; a stack step is one
// CUDA graph):
//   prep_kernel    one CTA per token: [combine the previous block + residual]
//                  [+ RMSNorm] + quantise the activations
//   router_kernel  partial logits per (expert, 1024-slice); the last CTA does
//                  softmax + top-k per token and builds the expert-tile plan
//   gateup_kernel  h = silu(G.x) * (U.x) per routed (expert, token tile)
//   down_kernel    ypart[part][assignment][row] = D.h over one K part (h is
//                  quantised by the consuming warps)
//   prep_kernel    (next layer, or the final combine) sum_j w_j * sum_parts
//
// Weight streaming (gate/up, down): experts are in the tiled device layout
// (expert_layout.cu).  Each CTA owns a contiguous range of units (two 8-row
// blocks over a K range); its producer thread fills a ring of shared-memory
// stages with four cp.async.bulk (TMA) copies per unit and stages each tile's
// activations, sixteen consumer warps split the unit's K range on the tensor
// cores, and a reducer warp sums their partials.
//
// Int4 arithmetic on the tensor cores.  Activations are split per quant
// group into two int8 digits, x ~= k*a + (k/254)*b (|a|,|b| <= 127,
// k = max|x|/127, residual <= 1.6e-5 * max|x|).  Weight codes (0..15) are
// exact int8, so mma.sync m16n8k32 s8 gives the exact integer sums A = sum
// c*a and B = sum c*b of one 32-element slice for 16 weight rows and up to
// 4 tokens x 2 digits at once.  A packed 32-bit word (8 codes) becomes an A
// fragment with two LOP3s and a shift; the k order inside a group is
// permuted (identically for weights and activations) so that each thread's
// codes come from contiguous bytes.  After the MMAs of a group one fp32
// epilogue applies that group's scale and zero:
//   row += s * (k/254 * (254*A + B) - 8*S) + z * S,   S = sum of x~ in group.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "dense_ffn.h"
#include "internal.h"
#include "route_common.cuh"

#include <cooperative_groups.h>

namespace wb {
namespace {

constexpr int kChunk = 32;      // elements per MMA k-slice (16 packed bytes)
constexpr int kMT = 4;          // tokens per MMA column quad
constexpr int kMaxTile = 8;     // tokens per expert tile: one or two column quads
constexpr int kWideMaxNg = 4;   // quant groups per consumer warp that two quads fit in registers
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxPlanAssign = 4096;  // T*k limit of the device plan builder
constexpr int kMaxKp = 8;             // max K parts of the down projection

enum { C_TOK_DONE = 0, C_NTILES = 1 };
constexpr int kCounters = 8;          // router CTAs done, tiles of the plan
enum { ST_ALIGN = 1, ST_EXPERT = 2, ST_PLAN = 4, ST_TIMEOUT = 8, ST_LAYOUT = 16 };

struct Tile {
    int expert;  // 0..E-1, or E for the shared expert
    int m;       // tokens in the tile (1..kMaxTile)
    int tok[kMaxTile];
    int asg[kMaxTile];  // assignment ids: t*K + j, or T*K + t for the shared expert
    const unsigned char* blob;  // the expert's tiled blob, NULL if unusable (status set)
};

struct MatOff {
    unsigned long long packed, scales, zeros;
};

struct LayerArgs {
    const void* const* blobs;
    const void* shared_blob;
    const __half* router_w;
    const __half* router_bias;
    const __half* norm_w;
    MatOff mat[3];
    MatOff smat[3];
    const __half* sg;  // fp16-dense shared expert (has_shared == 2): gate/up [si, H]
    const __half* su;
    const __half* sd;  // down [H, si]
    int si;
    int H, I, E, K, gs;
    int has_shared;  // 0 none, 1 int4 blob (a tile of the plan), 2 fp16 dense (dense_ffn.cu)
    int kp;   // K parts of the down projection
    int act_slots;  // token slots of the staged activation tile (min(T, kMT))
    int mt;         // tokens per expert tile of the plan (1, 4 or 8)
    int gating;     // WISP_GATING_* of the layer
    int tiles_hint; // the plan's likely tile count (exact for one token), so the
                    // streaming kernels can fetch their first tile record
                    // while the actual count is still in flight
};

struct Ws {
    int* status;
    int* counters;
    int* tok_cnt;
    float* logits;   // partial logits [T][E][slices]
    int* topk_idx;   // routing of the layer being run [T, K]
    float* topk_w;
    int* prev_idx;   // routing of the previous layer (combine in prep)
    float* prev_w;
    Tile* tiles;
    float* xn;
    uint4* xq;      // [T][H/32][4]  activation digits
    float4* xqp;    // [T][H/gs]     (k/254, sum of quantised x, 0, 0) per group
    float* h;       // [A][I]
    float* hs;      // [T][si] the fp16-dense shared expert's SwiGLU activations
    float* ypart;   // [kp][A][H]; a dense shared expert writes part 0 of its rows
    int A;          // assignment capacity
    int max_tiles;
};

// ------------------------------------------------------------------------
// small device helpers
// ------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Split cluster barrier (all threads of every CTA of the cluster).
// Atomic add with release (this CTA's earlier writes, ordered by a preceding
// __syncthreads, become visible with it) and acquire (the writes released by
// earlier adders become visible to this thread, and after a __syncthreads to
// its CTA): the "last CTA to finish" election without a separate fence.
__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
                 : "memory");
    return old;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Quantise activation blocks of gs elements (one quant group) into the
// two-digit int8 form.  Lane layout: each lane holds 4 consecutive elements;
// a block spans lpb = gs/4 consecutive lanes (8, 16 or 32).  Per 32-element
// chunk the digits are stored as 16 words matching the nibble split of the
// weights: for packed word w (elements 8w..8w+7) of the chunk, word [2w]
// holds the a-digits of elements 8w, 8w+2, 8w+4, 8w+6, word [2w+1] those of
// the odd elements, words [8+2w] / [8+2w+1] the same for the b-digits (so one
// 64-bit load gives an MMA B fragment).
__device__ __forceinline__ void quantize_block(const float4 v, int lpb, uint32_t* chunk_words,
                                               float4* block_param, bool block_leader) {
    const int lane = threadIdx.x & 31, q = lane & 7;
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    for (int o = 1; o < lpb; o <<= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
    const float k = m * (1.0f / 127.0f);
    const float k2 = k * (1.0f / 254.0f);
    const float inv = m > 0.f ? 127.0f / m : 0.f;
    const float inv2 = inv * 254.0f;
    const float e[4] = {v.x, v.y, v.z, v.w};
    int a[4], b[4], sa = 0, sb = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        a[i] = max(-127, min(127, __float2int_rn(e[i] * inv)));
        const float r = fmaf(-k, (float)a[i], e[i]);
        b[i] = max(-127, min(127, __float2int_rn(r * inv2)));
        sa += a[i];
        sb += b[i];
    }
    for (int o = 1; o < lpb; o <<= 1) {
        sa += __shfl_xor_sync(kFull, sa, o);
        sb += __shfl_xor_sync(kFull, sb, o);
    }
    // 16-bit halves of the four words this lane feeds (word q>>1, half q&1)
    const uint32_t ae = (a[0] & 0xff) | ((a[2] & 0xff) << 8);
    const uint32_t ao = (a[1] & 0xff) | ((a[3] & 0xff) << 8);
    const uint32_t be = (b[0] & 0xff) | ((b[2] & 0xff) << 8);
    const uint32_t bo = (b[1] & 0xff) | ((b[3] & 0xff) << 8);
    const uint32_t ae2 = __shfl_xor_sync(kFull, ae, 1), ao2 = __shfl_xor_sync(kFull, ao, 1);
    const uint32_t be2 = __shfl_xor_sync(kFull, be, 1), bo2 = __shfl_xor_sync(kFull, bo, 1);
    if ((q & 1) == 0) {
        const int w = q >> 1;
        reinterpret_cast<uint2*>(chunk_words)[w] = make_uint2(ae | (ae2 << 16), ao | (ao2 << 16));
        reinterpret_cast<uint2*>(chunk_words)[4 + w] =
            make_uint2(be | (be2 << 16), bo | (bo2 << 16));
    }
    if (block_leader)
        *block_param = make_float4(k2, fmaf(k, (float)sa, k2 * (float)sb), 0.f, 0.f);
}

// Quantise the n-element row `src` (n % gs == 0) with one warp per 128
// elements; warps and lanes past the end redo the last block (same data).
// `warp_id`/`n_warps` index the warps taking part.
__device__ __forceinline__ void quantize_row(const float4* src, int n, int gs, int warp_id,
                                             int n_warps, uint4* xq, float4* xqp) {
    const int lane = threadIdx.x & 31;
    const int lpb = gs / 4;
    const int nblk = n / gs;
    for (int base = warp_id * 128; base < n; base += n_warps * 128) {
        int blk = (base + 4 * lane) / gs;
        const int pos = (4 * lane) % gs;
        if (blk >= nblk) blk = nblk - 1;
        const int e = blk * gs + pos;
        const float4 v = src[e / 4];
        quantize_block(v, lpb, reinterpret_cast<uint32_t*>(xq + (e / kChunk) * 4),
                       xqp + blk, pos == 0);
    }
}

// ------------------------------------------------------------------------
// router: per-(expert, 1024-element slice) partial logits for every token,
// then the last CTA to finish sums the slices (fixed order), adds the bias,
// does softmax + top-k per token and builds the expert-tile plan.
// ------------------------------------------------------------------------
constexpr int kSlice = 1024;

// Softmax + top-k of token t from its logits lg[E] (without the bias), by one
// warp, into W.topk_idx / W.topk_w (rule: route_common.cuh); sp: [E] shared
// scratch of this warp; bias: the layer's bias as fp16 or as a float copy in
// shared memory, NULL for none.
template <typename BiasT>
__device__ wisp_route::TopkLane topk_token(const LayerArgs& L, const Ws& W, int t, int K,
                                           const float* lg, float* sp, const BiasT* bias) {
    return wisp_route::warp_topk(lg, bias, L.E, K, sp, W.topk_idx + t * K, W.topk_w + t * K,
                                 L.gating);
}

// The tiled blob of expert e (E = the shared expert), or NULL with the status
// flagged: ST_EXPERT for an index out of range or a NULL table entry,
// ST_LAYOUT for a blob whose header is not the tiled layout's (version 2).
constexpr uint32_t kTiledVersion = 2;
__device__ __forceinline__ const unsigned char* blob_ptr(const LayerArgs& L, int e) {
    const void* b = nullptr;
    if (e == L.E)
        b = L.shared_blob;
    else if (e >= 0 && e < L.E)
        b = L.blobs[e];
    return static_cast<const unsigned char*>(b);
}
// Check code of a blob pointer: 0, ST_EXPERT (NULL) or ST_LAYOUT.
__device__ __forceinline__ int blob_code(const unsigned char* b) {
    if (!b) return ST_EXPERT;
    return __ldg(reinterpret_cast<const uint32_t*>(b) + 1) != kTiledVersion ? ST_LAYOUT : 0;
}
// Loads kept where they are written (volatile asm): issued early, their
// results used much later, so their latency overlaps other work.
__device__ __forceinline__ uint32_t ld_early_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_early_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ const unsigned char* checked_blob(const LayerArgs& L, const Ws& W, int e) {
    const unsigned char* b = blob_ptr(L, e);
    const int code = blob_code(b);
    if (code) atomicOr(W.status, code);
    return code ? nullptr : b;
}

// Shared memory of the plan builder, in ints: the routing [NA] (kMaxPlanAssign
// slots), then per expert its count and its first tile (2E + 2), rounded up.
__host__ __device__ constexpr int plan_scratch_ints(int E) { return kMaxPlanAssign + 2 * E + 64; }

// Tiles of up to mt tokens per routed expert, in expert order, each expert's
// tokens in assignment order (then the shared expert's tiles).  pblob / pcode:
// the experts' blob pointers and check codes probed earlier (indices 0..E,
// E = the shared expert), or NULL to probe here.  s_idx: kMaxPlanAssign ints,
// s_cnt: 2E + 2 ints of shared memory.  Every step is spread over the block:
// one warp ranks each assignment within its expert (a match over 32
// assignments at a time, in order), one warp scans the experts' tile counts,
// and the tile records are written field by field by all threads.
__device__ void build_plan(const LayerArgs& L, const Ws& W, int T, int mt,
                           int* s_idx, int* s_cnt, const unsigned char* const* pblob = nullptr,
                           const int* pcode = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    const int K = L.K, E = L.E, NA = T * K;
    int* s_off = s_cnt + E + 1;  // [E + 1]: first tile of each expert, then the total
    for (int a = tid; a < NA; a += nthr) s_idx[a] = __ldcg(W.topk_idx + a);
    for (int e = tid; e <= E; e += nthr) s_cnt[e] = 0;
    __syncthreads();
    // rank of each assignment among its expert's (stable): s_idx[a] becomes
    // e | rank << 10, or -1 for a slot that routes nowhere
    if (warp == 0) {
        for (int c = 0; c < NA; c += 32) {
            const int a = c + lane;
            const int e = a < NA ? s_idx[a] : -1;
            const bool ok = e >= 0 && e < E;
            const unsigned grp = __match_any_sync(kFull, ok ? e : (1 << 20) + lane);
            const int leader = __ffs(grp) - 1;
            int base = 0;
            if (ok && lane == leader) {
                base = s_cnt[e];
                s_cnt[e] = base + __popc(grp);
            }
            base = __shfl_sync(kFull, base, leader);
            if (a < NA) s_idx[a] = ok ? (e | ((base + __popc(grp & ((1u << lane) - 1u))) << 10)) : -1;
            __syncwarp();
        }
    }
    __syncthreads();
    // first tile of each expert: exclusive scan of ceil(count / mt), experts
    // split into contiguous runs of `per` per lane
    if (warp == 0) {
        const int per = (E + 31) / 32, e0 = lane * per, e1 = min(E, e0 + per);
        int sum = 0;
        for (int e = e0; e < e1; ++e) sum += (s_cnt[e] + mt - 1) / mt;
        int inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(kFull, inc, o);
            if (lane >= o) inc += v;
        }
        int run = inc - sum;
        for (int e = e0; e < e1; ++e) {
            s_off[e] = run;
            run += (s_cnt[e] + mt - 1) / mt;
        }
        if (lane == 31) s_off[E] = inc;
    }
    __syncthreads();
    const int routed_tiles = s_off[E];
    const int shared_tiles = L.has_shared == 1 ? (T + mt - 1) / mt : 0;
    const int total = routed_tiles + shared_tiles;
    if (total > W.max_tiles) {
        if (tid == 0) {
            atomicOr(W.status, ST_PLAN);
            W.counters[C_NTILES] = 0;
        }
        return;
    }
    auto blob_of = [&](int e) -> const unsigned char* {
        if (pblob) {
            if (pcode[e]) atomicOr(W.status, pcode[e]);
            return pcode[e] ? nullptr : pblob[e];
        }
        return checked_blob(L, W, e);
    };
    // tile headers (expert, m, blob) of every expert with tokens
    for (int e = tid; e < E; e += nthr) {
        const int cnt = s_cnt[e];
        if (!cnt) continue;
        const unsigned char* bp = blob_of(e);
        for (int j = 0, ti = s_off[e]; j * mt < cnt; ++j, ++ti) {
            Tile* tl = W.tiles + ti;
            tl->expert = e;
            tl->m = min(mt, cnt - j * mt);
            tl->blob = bp;
        }
    }
    // each assignment into its slot
    for (int a = tid; a < NA; a += nthr) {
        const int v = s_idx[a];
        if (v < 0) continue;
        const int e = v & 1023, r = v >> 10;
        Tile* tl = W.tiles + s_off[e] + r / mt;
        tl->tok[r % mt] = a / K;
        tl->asg[r % mt] = a;
    }
    if (shared_tiles) {
        const unsigned char* bp = tid < shared_tiles ? blob_of(E) : nullptr;
        for (int s2 = tid; s2 < shared_tiles; s2 += nthr) {
            Tile* tl = W.tiles + routed_tiles + s2;
            tl->expert = E;
            tl->m = min(mt, T - s2 * mt);
            tl->blob = bp;
        }
        for (int t = tid; t < T; t += nthr) {
            Tile* tl = W.tiles + routed_tiles + t / mt;
            tl->tok[t % mt] = t;
            tl->asg[t % mt] = T * K + t;
        }
    }
    if (tid == 0) W.counters[C_NTILES] = total;
}

// The plan of a single token (T == 1, K + 1 <= 32), by one warp from the
// lanes' top-k results: one tile per routed slot j (lane j: token 0,
// assignment j), then the int4 shared expert's tile (assignment K).
__device__ void plan_one_token(const LayerArgs& L, const Ws& W, const wisp_route::TopkLane& r,
                               const unsigned char* const* pblob, const int* pcode) {
    const int lane = threadIdx.x & 31, K = L.K;
    int e = -1, asg = 0;
    if (lane < K) {
        e = r.i0;
        asg = lane;
    } else if (lane == K && L.has_shared == 1) {
        e = L.E;
        asg = K;
    }
    const unsigned live = __ballot_sync(kFull, e >= 0);
    if (e >= 0) {
        Tile tl;
        tl.expert = e;
        tl.m = 1;
#pragma unroll
        for (int i = 0; i < kMaxTile; ++i) tl.tok[i] = tl.asg[i] = 0;
        tl.asg[0] = asg;
        const int code = pcode[e];
        if (code) atomicOr(W.status, code);
        tl.blob = code ? nullptr : pblob[e];
        W.tiles[__popc(live & ((1u << lane) - 1u))] = tl;
    }
    if (lane == 0) W.counters[C_NTILES] = __popc(live);
}

// ------------------------------------------------------------------------
// prep: [combine the previous block's expert outputs + residual] [+ RMSNorm]
// + quantise the activations [+ router logits, softmax + top-k and the tile
// plan].  One thread-block cluster of cs CTAs per token; CTA r of a cluster
// owns the slice [r*H/cs, (r+1)*H/cs) of the token (a whole number of quant
// groups).  The RMSNorm sum of squares and the router logits are reduced
// across the cluster through distributed shared memory in rank order
// (deterministic).  With P_ROUTE, rank 0 of each cluster does the token's
// softmax + top-k and the last token to finish builds the expert-tile plan.
// ------------------------------------------------------------------------
enum { P_COMBINE = 1, P_RESID = 2, P_NORM = 4, P_QUANT = 8, P_ROUTE = 16 };
constexpr int kPrepThreads = 256;

// Shared memory of prep: the row slice, the cluster's partial logits [cs][E]
// (gathered in rank 0), the top-k / plan scratch, then (8-byte aligned) the
// probed blob pointers and check codes [E + 1] and the bias as floats [E].
__host__ __device__ inline size_t prep_tail_off(int H, int cs, int E) {
    const size_t o = (size_t)(H / cs) * sizeof(float) + (size_t)cs * E * sizeof(float) +
                     (size_t)(plan_scratch_ints(E) > 3 * E ? plan_scratch_ints(E) : 3 * E) * sizeof(int);
    return (o + 7) & ~size_t(7);
}
__host__ __device__ inline size_t prep_smem_bytes(int H, int cs, int E) {
    return prep_tail_off(H, cs, E) + (size_t)(E + 1) * (sizeof(void*) + sizeof(int)) +
           (size_t)E * sizeof(float);
}
constexpr int kProbeSlots = 5;  // experts 0..E (E <= 1024) over 256 threads

// Partial router logit of expert e over a CTA's slice of the row (n4 float4s
// in shared memory, starting at float4 i0 of the row), reduced over the warp.
// With `pre`, this lane's first two 16-byte words of the row are rw0 / rw1
// (loaded before the PDL wait).
__device__ __forceinline__ float router_dot(const LayerArgs& L, const float4* sx4, int n4, int i0,
                                            int e, int lane, bool pre, uint4 rw0, uint4 rw1) {
    const uint4* row =
        reinterpret_cast<const uint4*>(L.router_w) + ((size_t)e * L.H + (size_t)i0 * 4) / 8;
    float acc = 0.f;
    for (int c = lane; c < n4 / 2; c += 32) {
        const uint4 wv = pre && c < lane + 64 ? (c == lane ? rw0 : rw1) : __ldg(row + c);
        const float4 a = sx4[2 * c], b = sx4[2 * c + 1];
        const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
        float2 f = __half22float2(w2[0]);
        acc = fmaf(f.x, a.x, acc); acc = fmaf(f.y, a.y, acc);
        f = __half22float2(w2[1]);
        acc = fmaf(f.x, a.z, acc); acc = fmaf(f.y, a.w, acc);
        f = __half22float2(w2[2]);
        acc = fmaf(f.x, b.x, acc); acc = fmaf(f.y, b.y, acc);
        f = __half22float2(w2[3]);
        acc = fmaf(f.x, b.z, acc); acc = fmaf(f.y, b.w, acc);
    }
    return warp_sum(acc);
}

__global__ void __launch_bounds__(kPrepThreads)
prep_kernel(LayerArgs L, Ws W, int T, int flags, float* x, float* y, float eps, int prevK,
            int prev_shared, int prev_kp, int mt) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int cs = (int)cl.num_blocks(), rank = (int)cl.block_rank();
    const int t = blockIdx.x / cs;
    const int H = L.H, E = L.E;
    const int n4 = H / 4 / cs, i0 = rank * n4;  // this CTA's float4 range of the row
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nw = kPrepThreads / 32;
    extern __shared__ float4 smem4[];
    float4* sx4 = smem4;                                // [n4] the slice
    float* s_lg = reinterpret_cast<float*>(sx4 + n4);  // [cs][E] partial logits (rank 0)
    int* s_scr = reinterpret_cast<int*>(s_lg + cs * E); // top-k / plan scratch (rank 0)
    unsigned char* tail = reinterpret_cast<unsigned char*>(smem4) + prep_tail_off(H, cs, E);
    const unsigned char** s_blob = reinterpret_cast<const unsigned char**>(tail);  // [E + 1]
    int* s_bcode = reinterpret_cast<int*>(s_blob + E + 1);                          // [E + 1]
    float* s_bias = reinterpret_cast<float*>(s_bcode + E + 1);                      // [E]
    // Rank 0 of a routing prep with a plan: the layer's weights (bias) and the
    // expert table are not written by the kernels of this stream, so they are
    // read before the PDL wait; the blob headers are probed after it, while
    // the router runs, so the plan needs no dependent global loads.
    const bool planner = (flags & P_ROUTE) && rank == 0 && mt != 0;
    const unsigned char* pb[kProbeSlots];
    uint32_t phdr[kProbeSlots];
    if ((flags & P_ROUTE) && rank == 0 && L.router_bias)
        for (int e = tid; e < E; e += kPrepThreads) s_bias[e] = __half2float(L.router_bias[e]);
#pragma unroll
    for (int i = 0; i < kProbeSlots; ++i) {
        const int e = tid + i * kPrepThreads;
        pb[i] = (planner && e <= E) ? blob_ptr(L, e) : nullptr;
    }
    // The router rows of this warp's first expert (this CTA's slice, two
    // 16-byte words per lane) and the norm weights of this thread's first
    // float4 are static: in registers before the wait, so the previous
    // kernel's tail hides their latency.
    const uint4* wr_rows = reinterpret_cast<const uint4*>(L.router_w);
    uint4 rw0 = make_uint4(0, 0, 0, 0), rw1 = make_uint4(0, 0, 0, 0);
    if ((flags & P_ROUTE) && warp < E) {
        const uint4* row = wr_rows + ((size_t)warp * H + (size_t)i0 * 4) / 8;
        if (lane < n4 / 2) rw0 = ld_early_v4(row + lane);
        if (lane + 32 < n4 / 2) rw1 = ld_early_v4(row + lane + 32);
    }
    uint2 nwv = make_uint2(0, 0);
    if ((flags & P_NORM) && L.norm_w && tid < n4)
        nwv = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half2*>(L.norm_w) +
                                              2 * (i0 + tid));
    // Partial sums are pushed into the shared memory of the CTAs that read them
    // (distributed shared memory stores) before a cluster barrier, so no CTA
    // reads a peer's memory and none has to wait for its peers to finish
    // reading; the first remote store waits for this arrival of every CTA of
    // the cluster, i.e. for all of them to have started.
    const bool remote = cs > 1 && (flags & (P_NORM | P_ROUTE));
    // With the router, the norm's scale is applied after the router's dot
    // products and the quantisation after the one cluster barrier.
    const bool fold = (flags & P_ROUTE) != 0;
    const bool norm = (flags & P_NORM) != 0;
    if (remote) cluster_arrive_relaxed();
    pdl_wait();
#pragma unroll
    for (int i = 0; i < kProbeSlots; ++i)
        phdr[i] = pb[i] ? ld_early_u32(reinterpret_cast<const uint32_t*>(pb[i]) + 1) : 0u;
    pdl_launch();
    __shared__ float red[nw];
    __shared__ float s_ssv[8];  // partial sums of squares of the cluster, by rank
    __shared__ int s_last;
    float4* xt = reinterpret_cast<float4*>(x + (size_t)t * H) + i0;

    const size_t part_stride = (size_t)W.A * H;
    float ss = 0.f;
    for (int i = tid; i < n4; i += kPrepThreads) {
        float4 v = xt[i];
        if (flags & P_COMBINE) {
            // reference order: shared expert first (weight 1), then top-k order
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            // every part of an assignment is loaded before they are summed
            // (in part order)
            float4 yp[kMaxKp];
            if (prev_shared) {
                // int4 shared expert: one ypart per down K part; fp16-dense: part 0
                const size_t a = (size_t)T * prevK + t;
                const int np = prev_shared == 2 ? 1 : prev_kp;
#pragma unroll
                for (int p = 0; p < kMaxKp; ++p)
                    if (p < np)
                        yp[p] = reinterpret_cast<const float4*>(W.ypart + p * part_stride +
                                                                a * H)[i0 + i];
#pragma unroll
                for (int p = 0; p < kMaxKp; ++p)
                    if (p < np) {
                        acc.x += yp[p].x; acc.y += yp[p].y; acc.z += yp[p].z; acc.w += yp[p].w;
                    }
            }
            for (int j = 0; j < prevK; ++j) {
                // loads do not wait for the routing; an unrouted slot is skipped by a select
                const bool live = __ldg(W.prev_idx + t * prevK + j) >= 0;
                const float wj = __ldg(W.prev_w + t * prevK + j);
                const size_t a = (size_t)t * prevK + j;
#pragma unroll
                for (int p = 0; p < kMaxKp; ++p)
                    if (p < prev_kp)
                        yp[p] = reinterpret_cast<const float4*>(W.ypart + p * part_stride +
                                                                a * H)[i0 + i];
                float4 yj = yp[0];
#pragma unroll
                for (int p = 1; p < kMaxKp; ++p)
                    if (p < prev_kp) {
                        yj.x += yp[p].x; yj.y += yp[p].y; yj.z += yp[p].z; yj.w += yp[p].w;
                    }
                if (live) {
                    acc.x += wj * yj.x; acc.y += wj * yj.y; acc.z += wj * yj.z; acc.w += wj * yj.w;
                }
            }
            if (flags & P_RESID) {
                v.x += acc.x; v.y += acc.y; v.z += acc.z; v.w += acc.w;
                xt[i] = v;
            } else {
                v = acc;
            }
            if (y) reinterpret_cast<float4*>(y + (size_t)t * H)[i0 + i] = v;
        }
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        if (fold && norm && L.norm_w) {
            uint2 nv = nwv;  // prefetched for the first float4
            if (i != tid) nv = *reinterpret_cast<const uint2*>(
                              reinterpret_cast<const __half2*>(L.norm_w) + 2 * (i0 + i));
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&nv.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&nv.y));
            v.x *= a.x; v.y *= a.y; v.z *= b.x; v.w *= b.y;
        }
        sx4[i] = v;
    }
    if (!(flags & (P_NORM | P_QUANT | P_ROUTE))) return;
    if (fold) {
        // RMSNorm scales the whole row by one factor, so the router's partial
        // dot products are taken on the weighted, unscaled slice and scaled once
        // the sum of squares is known: both partial sums cross the cluster in
        // one barrier, and the slice is normalised and quantised after it.
        if (norm) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
        }
        __syncthreads();
        const float lgp = warp < E ? router_dot(L, sx4, n4, i0, warp, lane, true, rw0, rw1) : 0.f;
        if (remote) cluster_wait();  // peers started (the arrival at entry)
        if (norm && tid < cs) {
            float v = 0.f;
            for (int w = 0; w < nw; ++w) v += red[w];
            *cl.map_shared_rank(&s_ssv[rank], tid) = v;  // into CTA tid's copy
        }
        if (warp < E && lane == 0) *cl.map_shared_rank(&s_lg[rank * E + warp], 0) = lgp;
        for (int e = warp + nw; e < E; e += nw) {  // experts past the warp count
            const float v = router_dot(L, sx4, n4, i0, e, lane, false, rw0, rw1);
            if (lane == 0) *cl.map_shared_rank(&s_lg[rank * E + e], 0) = v;
        }
        cl.sync();  // every CTA holds every sum of squares, rank 0 every partial logit
        float sc = 1.f;
        if (norm) {
            float tot = 0.f;
            for (int r = 0; r < cs; ++r) tot += s_ssv[r];
            sc = 1.0f / sqrtf(tot / (float)H + eps);
        }
        if (rank == 0)
            for (int e = tid; e < E; e += kPrepThreads) {
                float v = 0.f;
                for (int r = 0; r < cs; ++r) v += s_lg[r * E + e];
                s_scr[2 * E + e] = __float_as_int(norm ? v * sc : v);
            }
        // the normalised slice and its two-digit form; rank 0 leaves warp 0 to
        // the top-k and the plan
        const int w0 = rank == 0 ? 1 : 0, nws = nw - w0;
        if (warp >= w0) {
            float4* xn = reinterpret_cast<float4*>(W.xn + (size_t)t * H) + i0;
            for (int base = (warp - w0) * 128; norm && base < n4 * 4; base += nws * 128) {
                const int i = base / 4 + lane;
                if (i < n4) {
                    float4 v = sx4[i];
                    v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
                    sx4[i] = v;
                    xn[i] = v;
                }
            }
            __syncwarp();
            if (flags & P_QUANT)
                quantize_row(sx4, n4 * 4, L.gs, warp - w0, nws,
                             W.xq + ((size_t)t * (H / kChunk) + (size_t)i0 * 4 / kChunk) * 4,
                             W.xqp + (size_t)t * (H / L.gs) + (size_t)i0 * 4 / L.gs);
        }
    } else if (flags & P_NORM) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (remote) cluster_wait();  // peers started (the arrival at entry)
        if (tid < cs) {
            float v = 0.f;
            for (int w = 0; w < nw; ++w) v += red[w];
            *cl.map_shared_rank(&s_ssv[rank], tid) = v;  // into CTA tid's copy
        }
        cl.sync();  // every CTA holds every partial sum of squares
        float tot = 0.f;
        for (int r = 0; r < cs; ++r) tot += s_ssv[r];
        const float sc = 1.0f / sqrtf(tot / (float)H + eps);
        float4* xn = reinterpret_cast<float4*>(W.xn + (size_t)t * H) + i0;
        const __half2* nw2 = reinterpret_cast<const __half2*>(L.norm_w) + 2 * i0;
        for (int i = tid; i < n4; i += kPrepThreads) {
            float4 v = sx4[i];
            v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
            if (L.norm_w) {
                uint2 nv = nwv;  // prefetched for the first float4
                if (i != tid) nv = *reinterpret_cast<const uint2*>(nw2 + 2 * i);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&nv.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&nv.y));
                v.x *= a.x; v.y *= a.y; v.z *= b.x; v.w *= b.y;
            }
            sx4[i] = v;
            xn[i] = v;
        }
    }
    if (!fold) {
        __syncthreads();
        if (flags & P_QUANT)  // the two-digit form of the slice for the gate/up stream
            quantize_row(sx4, n4 * 4, L.gs, warp, nw,
                         W.xq + ((size_t)t * (H / kChunk) + (size_t)i0 * 4 / kChunk) * 4,
                         W.xqp + (size_t)t * (H / L.gs) + (size_t)i0 * 4 / L.gs);
    }
    if (!(flags & P_ROUTE) || rank != 0) return;
    // With the router and at most 31 experts, warp 0 holds every logit and
    // every probe, so the top-k and a one-token plan do not wait for the other
    // warps (which are still writing the slice's two-digit form).
    const bool w0only = fold && E + 1 <= 32;
    if (planner && (!w0only || warp == 0)) {
#pragma unroll
        for (int i = 0; i < kProbeSlots; ++i) {
            const int e = tid + i * kPrepThreads;
            if (e <= E) {
                s_blob[e] = pb[i];
                s_bcode[e] = !pb[i] ? ST_EXPERT : (phdr[i] != kTiledVersion ? ST_LAYOUT : 0);
            }
        }
    }
    if (w0only)
        __syncwarp();
    else
        __syncthreads();
    const bool one = T == 1 && L.K + 1 <= 32;  // the one-token plan
    if (warp == 0) {
        const float* lg = reinterpret_cast<const float*>(s_scr + 2 * E);
        float* sp = reinterpret_cast<float*>(s_scr);
        const wisp_route::TopkLane r =
            L.router_bias ? topk_token(L, W, t, L.K, lg, sp, s_bias)
                          : topk_token(L, W, t, L.K, lg, sp, static_cast<const float*>(nullptr));
        if (mt != 0 && one) plan_one_token(L, W, r, s_blob, s_bcode);
    }
    if (mt == 0 || one) return;  // routing only, or the plan is written
    __syncthreads();
    if (tid == 0) s_last = T == 1 || atomic_add_acq_rel(W.counters + C_TOK_DONE, 1) == T - 1;
    __syncthreads();
    if (!s_last) return;
    build_plan(L, W, T, mt, s_scr, s_scr + kMaxPlanAssign, s_blob, s_bcode);
    if (tid == 0) W.counters[C_TOK_DONE] = 0;  // ready for the next layer
}

// Expert-tile plan from a routing the caller supplies (W.topk_idx / W.topk_w,
// [T, K]) instead of the router: the expert-parallel path routes on the tokens'
// home GPU and runs the experts where they live.
__global__ void __launch_bounds__(kThreads)
plan_kernel(LayerArgs L, Ws W, int T, int mt) {
    pdl_wait();
    pdl_launch();
    extern __shared__ int smem[];
    build_plan(L, W, T, mt, smem, smem + kMaxPlanAssign);
}

// The status word and counters of a workspace, zeroed in stream order (see
// launch_zero_words).
__global__ void __launch_bounds__(256) zero_words_kernel(int* p, int n) {
    pdl_wait();
    pdl_launch();
    for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = 0;
}

// y[t] += sum_j w[t,j] * rows[ridx[t,j]] in j order (ridx < 0: skipped); the
// combine of the expert-parallel path on the tokens' home GPU.
__global__ void __launch_bounds__(kPrepThreads)
ep_combine_kernel(float* y, const float* rows, const int* ridx, const float* w, int T, int K,
                  int H) {
    // y is the output of the previous kernel (the shared expert's combine),
    // which may have triggered this launch before finishing
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.x;
    if (t >= T) return;
    float4* yt = reinterpret_cast<float4*>(y + (size_t)t * H);
    for (int i = threadIdx.x; i < H / 4; i += kPrepThreads) {
        float4 acc = yt[i];
        for (int j = 0; j < K; ++j) {
            const int r = ridx[t * K + j];
            if (r < 0) continue;
            const float wj = w[t * K + j];
            const float4 v = reinterpret_cast<const float4*>(rows + (size_t)r * H)[i];
            acc.x += wj * v.x; acc.y += wj * v.y; acc.z += wj * v.z; acc.w += wj * v.w;
        }
        yt[i] = acc;
    }
}

__global__ void __launch_bounds__(kThreads)
router_kernel(LayerArgs L, Ws W, int T, int mt, const float* xin, int nsl) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int E = L.E, H = L.H;
    __shared__ int s_last;
    extern __shared__ int smem[];

    const int item = blockIdx.x * kWarps + warp;
    if (item < E * nsl) {
        const int e = item / nsl, sl = item - e * nsl;
        const int c0 = sl * kSlice, c1 = min(H, c0 + kSlice);
        const __half* row = L.router_w + (size_t)e * H;
        uint4 wv[kSlice / 256];
#pragma unroll
        for (int i = 0; i < kSlice / 256; ++i) {
            const int c = c0 + i * 256 + lane * 8;
            wv[i] = c < c1 ? *reinterpret_cast<const uint4*>(row + c) : make_uint4(0, 0, 0, 0);
        }
        for (int t = 0; t < T; ++t) {
            const float* xr = xin + (size_t)t * H;
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < kSlice / 256; ++i) {
                const int c = c0 + i * 256 + lane * 8;
                if (c < c1) {
                    const float4 x0 = *reinterpret_cast<const float4*>(xr + c);
                    const float4 x1 = *reinterpret_cast<const float4*>(xr + c + 4);
                    const __half2* w2 = reinterpret_cast<const __half2*>(&wv[i]);
                    float2 f = __half22float2(w2[0]);
                    acc = fmaf(f.x, x0.x, acc);
                    acc = fmaf(f.y, x0.y, acc);
                    f = __half22float2(w2[1]);
                    acc = fmaf(f.x, x0.z, acc);
                    acc = fmaf(f.y, x0.w, acc);
                    f = __half22float2(w2[2]);
                    acc = fmaf(f.x, x1.x, acc);
                    acc = fmaf(f.y, x1.y, acc);
                    f = __half22float2(w2[3]);
                    acc = fmaf(f.x, x1.z, acc);
                    acc = fmaf(f.y, x1.w, acc);
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) W.logits[((size_t)t * E + e) * nsl + sl] = acc;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0)
        s_last = atomic_add_acq_rel(W.counters + C_TOK_DONE, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    {
        float* sp = reinterpret_cast<float*>(smem) + (size_t)warp * 3 * E;
        float* lg = sp + 2 * E;
        for (int t = warp; t < T; t += kWarps) {
            for (int e = lane; e < E; e += 32) {
                const float* pp = W.logits + ((size_t)t * E + e) * nsl;
                float v = 0.f;
                for (int q = 0; q < nsl; ++q) v += __ldcg(pp + q);
                lg[e] = v;
            }
            __syncwarp();
            topk_token(L, W, t, L.K, lg, sp, L.router_bias);
            __syncwarp();
        }
    }
    __syncthreads();  // this CTA's top-k writes are visible to all its threads
    if (mt == 0) return;  // routing only, no plan
    build_plan(L, W, T, mt, smem, smem + kMaxPlanAssign);
    if (threadIdx.x == 0) W.counters[C_TOK_DONE] = 0;  // ready for the next layer
}

// ------------------------------------------------------------------------
// TMA-staged weight streaming (shared by gate/up and down)
//
// Experts are in the tiled device layout (expert_layout.cu): every 8-row
// block of a matrix is contiguous, codes ordered [group][row] and then the
// (scale, zero) pairs [group][row].  A unit is two 8-row blocks (MMA rows 0-7
// and 8-15) over a K range of ng quant groups: gate/up = gate block b + up
// block b over all of H; down = blocks 2j, 2j+1 over one K part.  One CTA per
// SM = 1 producer warp + kNcw consumer warps.  The producer walks the CTA's
// units (static round robin: unit = CTA + k * CTAs, so no atomics) and issues
// four cp.async.bulk copies per unit (codes and scale/zero pairs of each
// block) into a ring of shared-memory stages, each guarded by a "full"
// mbarrier (transaction bytes) and an "empty" mbarrier (one arrival per
// consumer warp).  Every wait is bounded by %globaltimer: on timeout the warp
// sets ST_TIMEOUT in the status word and leaves, and the producer drains the
// copies it issued (bounded too) before the CTA exits.
// ------------------------------------------------------------------------
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity to complete (the timer is
// read every 64 polls; each poll may itself suspend the thread briefly).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try(bar, parity)) return true;
        if ((n & 63u) == 0 && gtimer() - t0 > kWaitNs) return false;
    }
}
// Weights are read exactly once per kernel: their copies carry an L2
// evict-first policy so that streaming them does not push the small
// activation and partial-sum buffers the kernels share out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Plain bulk copy (activations: small, re-read by every CTA, left to the
// default L2 policy).
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 16-byte copies through the load/store path (cp.async), completion tracked
// by an mbarrier: the fp32 activation rows of the down projection take this
// path so that they do not queue in the copy engine behind the weight stages
// the CTA filled before its PDL wait.
__device__ __forceinline__ void ldgsts16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void ldgsts_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
// The warp copies `rows` fp32 rows of `bytes` each (src_row(t) -> dst + t *
// bytes) and makes `bar` (expected count 1) complete when they have landed.
template <typename SrcRow>
__device__ __forceinline__ void copy_rows_lsu(uint8_t* dst, uint32_t bytes, int rows,
                                              SrcRow src_row, uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    const int n16 = (int)(bytes / 16);
    for (int t = 0; t < rows; ++t) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(src_row(t));
        for (int i = lane; i < n16; i += 32) ldgsts16(dst + (size_t)t * bytes + i * 16, src + i * 16);
    }
    ldgsts_arrive(bar);  // every lane: one pending arrival, released when its copies land
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

// A streaming CTA: warp 0 = producer (lane 0), warp 1 = reducer, warps
// 2 .. kNcw+1 = tensor-core consumers.
constexpr int kNcw = 16;                          // consumer warps per CTA
constexpr int kStreamCta = 32 * (kNcw + 2);
constexpr int kMaxWarpK = 512;                    // K elements per consumer warp
constexpr int kMaxPartK = kNcw * kMaxWarpK;       // K elements per unit
constexpr int kSkip = 0x40000000;                 // unit flag: weights unusable, contribute 0

// Geometry of a unit's stage: block A (MMA rows 0-7) at 0, block B (rows
// 8-15) at bbytes; each block = codes [ng][8][gs/2] then pairs [ng][8].
struct Geo {
    int ng;           // quant groups in the K range
    uint32_t pbytes;  // code bytes of one block's range = ng * 4 * gs
    uint32_t bbytes;  // pbytes + ng * 32
};
__host__ __device__ inline Geo make_geo(int ng, int gs) {
    Geo g;
    g.ng = ng;
    g.pbytes = (uint32_t)ng * 4u * (uint32_t)gs;
    g.bbytes = g.pbytes + (uint32_t)ng * 32u;
    return g;
}
__host__ __device__ inline uint32_t stage_bytes_of(const Geo& g) {
    return (2 * g.bbytes + 127) / 128 * 128;
}
// Bytes of one 8-row block of a [rows, cols] matrix in the tiled layout.
__host__ __device__ inline size_t block_bytes_of(int cols, int gs) {
    return 4 * (size_t)cols + 32 * (size_t)(cols / gs);
}
// Activation tile of a K range of ng groups (NPG 32-element chunks each) for
// kMT token slots: one column quad of an expert tile at a time (a tile of
// more than kMT tokens stages its second quad once the first is in the
// consumers' registers).  Quantised (gate/up): the words [slot][chunk][64 B],
// then (k/254, S) per group [slot][group][16 B].  Float (down): the fp32
// rows [slot][ng * gs], quantised by the consumer warps themselves.
__host__ __device__ inline uint32_t act_row_bytes(int ng, int npg, bool f32) {
    return (uint32_t)ng * npg * (f32 ? 128u : 64u);
}
__host__ __device__ inline uint32_t act_bytes_of(int ng, int npg, bool f32, int slots) {
    return (uint32_t)slots * (act_row_bytes(ng, npg, f32) + (f32 ? 0u : (uint32_t)ng * 16u));
}

// Per-stage unit record written by the producer: unit id (| kSkip), or -1 at
// the end; the tile's token count, token and assignment ids (the reducer
// stores by assignment and stages a second column quad by either).
struct UnitInfo {
    int u, m, tile;  // tile: the tile whose m/asg the record holds
    int asg[kMaxTile];
    int tok[kMaxTile];
};


// Shared memory of a streaming CTA.
struct StreamSmem {
    uint8_t* stages;   // [n_stages][stage_bytes]
    float2* red;       // [n_stages][kNcw][32] consumer partials
    uint8_t* act;      // activation tile (act_bytes_of)
    float2* kp;        // [kNcw][NG][MT] (k/254, S) of each warp's groups
    UnitInfo* info;    // [n_stages]
    uint64_t* full;    // [n_stages] weights landed (tx)
    uint64_t* red_bar; // [n_stages] consumer partials written (kNcw arrivals)
    uint64_t* empty;   // [n_stages] stage reusable (reducer)
    uint64_t* act_full;   // first column quad of a tile staged (producer)
    uint64_t* act_empty;  // activation tile read (kNcw arrivals)
    uint64_t* act_mid;    // first quad read, second may be staged (kNcw arrivals)
    uint64_t* act_full2;  // second column quad staged (reducer)
    uint32_t stage_bytes, act_row, act_bytes;
    int act_slots;
    int n_stages;
};
// Per stage: consumer partials for the tile width's token quads.
__host__ __device__ constexpr size_t red_bytes_per_stage(int mt) {
    return (size_t)kNcw * 32 * 8 * (mt / 4);
}
// (k/254, S) pairs: each consumer warp's ng groups x the tile width.
__host__ __device__ constexpr size_t kp_bytes(int ng, int mt) {
    return (size_t)kNcw * ng * mt * 8;
}
__host__ __device__ inline size_t stream_smem_bytes(int n_stages, uint32_t stage_bytes,
                                                     uint32_t act_bytes, int mt, int ng) {
    return (size_t)n_stages * (stage_bytes + red_bytes_per_stage(mt) + sizeof(UnitInfo) + 24) +
           (act_bytes + 127) / 128 * 128 + kp_bytes(ng, mt) + 32 + 128;
}
// The float path (down) quantises its rows in place in the activation tile.
__device__ __forceinline__ StreamSmem stream_smem(uint8_t* base, int n_stages,
                                                  uint32_t stage_bytes, const Geo& geo, int npg,
                                                  bool f32, int slots, int mt, int ng) {
    StreamSmem s;
    s.stage_bytes = stage_bytes;
    s.n_stages = n_stages;
    s.act_row = act_row_bytes(geo.ng, npg, f32);
    s.act_bytes = act_bytes_of(geo.ng, npg, f32, slots);
    s.act_slots = slots;
    size_t o = 0;
    s.stages = base;
    o += (size_t)n_stages * stage_bytes;
    s.act = base + o;
    o += (s.act_bytes + 127) / 128 * 128;
    s.red = reinterpret_cast<float2*>(base + o);
    o += (size_t)n_stages * red_bytes_per_stage(mt);
    s.kp = reinterpret_cast<float2*>(base + o);
    o += kp_bytes(ng, mt);
    s.info = reinterpret_cast<UnitInfo*>(base + o);
    o += (size_t)n_stages * sizeof(UnitInfo);
    o = (o + 7) & ~size_t(7);
    s.full = reinterpret_cast<uint64_t*>(base + o);
    s.red_bar = s.full + n_stages;
    s.empty = s.red_bar + n_stages;
    s.act_full = s.empty + n_stages;
    s.act_empty = s.act_full + 1;
    s.act_mid = s.act_full + 2;
    s.act_full2 = s.act_full + 3;
    return s;
}
__device__ __forceinline__ void stream_init(const StreamSmem& S) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < S.n_stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.red_bar[s], kNcw);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(S.act_full, 1);
        mbar_init(S.act_empty, kNcw);
        mbar_init(S.act_mid, kNcw);
        mbar_init(S.act_full2, 1);
        for (int s = 0; s < S.n_stages; ++s) S.info[s].tile = -1;
        mbar_fence_init();
    }
    __syncthreads();
}

// A tile record as a streaming kernel built for MT-token tiles holds it: the
// plan's slots past MT are never used there, and not carrying them keeps the
// producer's copies of the current and next record small.
template <int MT>
struct TileView {
    int m;
    int tok[MT];
    int asg[MT];
    const unsigned char* blob;
};
template <int MT>
__device__ __forceinline__ void load_tile(const Tile* src, TileView<MT>& tl) {
    tl.m = __ldcg(&src->m);
#pragma unroll
    for (int i = 0; i < MT; ++i) {
        tl.tok[i] = __ldcg(&src->tok[i]);
        tl.asg[i] = __ldcg(&src->asg[i]);
    }
    tl.blob = reinterpret_cast<const unsigned char*>(
        __ldcg(reinterpret_cast<const unsigned long long*>(&src->blob)));
}

// Where the producer finds a tile's activations: quantised rows `xq`
// ([row][chunk][64 B], nchk chunks per row) and their per-group parameters
// `xqp` ([row][group] float4, ngrp groups per row), K range starting at
// group kg0; rows are token ids (gate/up) or assignment ids (down).
struct ActSrc {
    const uint8_t* xq;
    const float4* xqp;
    const float* xf;   // fp32 rows instead (float path), row_elems per row
    int nchk, ngrp, kg0, npg, gs, row_elems;
    bool by_asg;
};

// Producer (lane 0 of warp 0): for the units [u_begin, u_end) in order, fill
// the weight stages and, for each tile, the activation tile; then post a
// sentinel.  Unit u is unit r = u % upt of tile u / upt; blk(blob, r, c) gives
// the global address of its copy c (0: codes of block A, 1: pairs of block A,
// 2/3: block B).  The next tile's record is loaded one tile ahead.  With
// `act_after_pdl` the activations come from the previous kernel in the
// stream: the first tile's activation copies wait for it (griddepcontrol)
// but only after the weight stages have been filled.
// Global addresses of a unit's four copies (0: codes of block A, 1: pairs of
// block A, 2/3: block B): blob + off0 + r * ustride + coff[c] for unit r of a
// tile whose expert blob is `blob`.
struct UnitAddr {
    size_t off0, ustride;
    size_t coff[4];
};

// With `first_act_elsewhere` another warp loads the range's first
// activation tile (the down kernel's reducer, right after the PDL wait), and
// the producer issues only kPrePdlStages stages before it waits for the
// previous kernel itself: a full ring on every SM at that moment would queue
// the small activation loads behind ~28 MB of weight copies, and the down
// projection is bound by its consumers once h is complete, not by DRAM.
constexpr int kPrePdlStages = 2;
template <int MT>
__device__ void produce(const StreamSmem& S, const Ws& W, int u_begin, int u_end, int upt,
                        int ntiles, const Geo& geo, const ActSrc& as, bool act_after_pdl,
                        const UnitAddr& ua, bool first_act_elsewhere = false,
                        const TileView<MT>* pre = nullptr, int pre_ti = -1) {
    const int lane = threadIdx.x & 31;
    const uint32_t tx = 2 * geo.bbytes, zb = (uint32_t)geo.ng * 32u;
    const bool f32 = as.xf != nullptr;
    const uint32_t rowb = act_row_bytes(geo.ng, as.npg, f32);
    const uint32_t pb = f32 ? 0u : (uint32_t)geo.ng * 16u;
    const uint64_t pol = evict_first_policy();
    // this lane's copy: destination offset in a stage and size
    const uint32_t dst_off = (lane >> 1) * geo.bbytes + (lane & 1) * geo.pbytes;
    const uint32_t csize = (lane & 1) ? zb : geo.pbytes;
    const size_t coff = lane < 4 ? ua.coff[lane] : 0;
    int ti = u_begin / upt, r = u_begin - ti * upt;
    TileView<MT> cur, nxt;
    if (u_begin < u_end) {
        if (pre && pre_ti == ti)
            cur = *pre;
        else
            load_tile(W.tiles + ti, cur);
    }
    // with a pre-loaded first record (gate/up) the next one is read once the
    // first copies are on their way
    bool nxt_due = ti + 1 < ntiles;
    if (!pre && nxt_due) {
        load_tile(W.tiles + ti + 1, nxt);
        nxt_due = false;
    }
    const unsigned char* p = nullptr;
    bool tile_ok = false;
    // per tile: the lane's source pointer and whether the tile's copies are usable
    auto start_tile = [&]() {
        p = cur.blob ? cur.blob + ua.off0 + (size_t)r * ua.ustride + coff : nullptr;
        const bool mis = __any_sync(kFull, lane < 4 && p && !aligned16(p));
        tile_ok = cur.blob != nullptr && !mis;
        if (mis && lane == 0) atomicOr(W.status, ST_ALIGN);
    };
    if (u_begin < u_end) start_tile();
    int it = 0, tiles_done = 0, s = 0, issued = 0;
    uint32_t ph = 0;
    bool ok = true, act_due = true, waited_pdl = !act_after_pdl;
    if (first_act_elsewhere && u_begin < u_end) {
        act_due = false;
        tiles_done = 1;
    }
    // barrier waits by lane 0, result shared with the warp
    auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
        int v = 1;
        if (lane == 0) v = mbar_wait(bar, parity) ? 1 : 0;
        return __shfl_sync(kFull, v, 0) != 0;
    };
    // activation tile of `cur` (its first column quad), once the consumers
    // copied the previous one; one copy per lane
    auto issue_act = [&]() -> bool {
        if (!waited_pdl) {
            pdl_wait();
            waited_pdl = true;
        }
        if (tiles_done > 0 && !wait0(S.act_empty, (tiles_done - 1) & 1)) return false;
        const int m0 = min(cur.m, S.act_slots);
        if (f32) {
            copy_rows_lsu(S.act, rowb, m0, [&](int t) {
                const int row = as.by_asg ? cur.asg[t] : cur.tok[t];
                return as.xf + (size_t)row * as.row_elems + (size_t)as.kg0 * as.gs;
            }, S.act_full);
            ++tiles_done;
            act_due = false;
            return true;
        }
        if (lane == 0) mbar_expect_tx(S.act_full, (uint32_t)m0 * (rowb + pb));
        __syncwarp();
        const int t = lane / 2;
        if (t < m0) {
            const int row = as.by_asg ? cur.asg[t] : cur.tok[t];
            if ((lane & 1) == 0) {
                bulk_g2s_plain(S.act + t * rowb,
                               as.xq + ((size_t)row * as.nchk + (size_t)as.kg0 * as.npg) * 64,
                               rowb, S.act_full);
            } else {
                bulk_g2s_plain(S.act + S.act_slots * rowb + t * pb,
                               as.xqp + (size_t)row * as.ngrp + as.kg0, pb, S.act_full);
            }
        }
        ++tiles_done;
        act_due = false;
        return true;
    };
    for (int u = u_begin;; ++u, ++it) {
        if (!wait0(&S.empty[s], ph ^ 1)) {
            ok = false;
            break;
        }
        if (u >= u_end) {
            if (lane == 0) {
                S.info[s].u = -1;
                mbar_arrive(&S.full[s]);
            }
            break;
        }
        if (r == upt) {
            r = 0;
            ++ti;
            cur = nxt;
            if (ti + 1 < ntiles) load_tile(W.tiles + ti + 1, nxt);
            act_due = true;
            start_tile();
        }
        if (act_due && waited_pdl && !issue_act()) {
            ok = false;
            break;
        }
        if (lane == 0) {
            UnitInfo& inf = S.info[s];
            if (inf.tile != ti) {
                inf.tile = ti;
                inf.m = cur.m;
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    inf.asg[t] = cur.asg[t];
                    inf.tok[t] = cur.tok[t];
                }
            }
            inf.u = tile_ok ? u : (u | kSkip);
            if (tile_ok)
                mbar_expect_tx(&S.full[s], tx);
            else
                mbar_arrive(&S.full[s]);
        }
        __syncwarp();
        if (tile_ok && lane < 4)
            bulk_g2s(S.stages + (size_t)s * S.stage_bytes + dst_off, p, csize, &S.full[s], pol);
        ++issued;
        if (nxt_due) {
            load_tile(W.tiles + ti + 1, nxt);
            nxt_due = false;
        }
        p += ua.ustride;
        ++r;
        if (first_act_elsewhere && !waited_pdl && it + 1 >= kPrePdlStages) {
            pdl_wait();
            waited_pdl = true;
            // a tile that began before this point still needs its activations
            if (act_due && !issue_act()) {
                ok = false;
                break;
            }
        }
        // a deferred first activation tile: once the stages are full, or before
        // the tile or the range ends
        if (act_due && !waited_pdl &&
            (it + 1 >= S.n_stages || r == upt || u + 1 >= u_end) && !issue_act()) {
            ok = false;
            break;
        }
        if (++s == S.n_stages) {
            s = 0;
            ph ^= 1;
        }
    }
    if (!ok && lane == 0) {
        atomicOr(W.status, ST_TIMEOUT);
        // a consumer stopped early: let every issued copy land before exiting
        for (int k = 0; k < S.n_stages && k < issued; ++k) {
            const int j = issued - 1 - k;
            mbar_wait(&S.full[j % S.n_stages], (j / S.n_stages) & 1);
        }
        if (tiles_done > 0) mbar_wait(S.act_full, (tiles_done - 1) & 1);
    }
}

// Reducer (warp 1): per unit, once the consumers' partials are in, sum them in
// warp order (deterministic) and store the result; then release the stage.
// out(u, asg, g, sum) is called by lane (g, q) for token slot q < m.  At the
// first unit of a tile of more than kMT tokens it also stages the tile's
// second column quad (stage2(inf): copies into the activation tile that
// complete S.act_full2) once the consumers have read the first (S.act_mid):
// the weight producer keeps streaming meanwhile.
template <int MT, typename Out, typename Stage2>
__device__ void reduce_units(const StreamSmem& S, const Ws& W, Out out, Stage2 stage2) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    int s = 0, last_tile = -1, wide = 0;
    uint32_t ph = 0;
    for (;;) {
        if (!mbar_wait(&S.full[s], ph)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            break;
        }
        const UnitInfo& inf = S.info[s];
        const int u = *reinterpret_cast<const volatile int*>(&inf.u);
        if (u == -1) break;
        if constexpr (MT > kMT) {
            const int ti = *reinterpret_cast<const volatile int*>(&inf.tile);
            if (ti != last_tile) {
                last_tile = ti;
                if (inf.m > kMT) {
                    if (!mbar_wait(S.act_mid, wide & 1)) {
                        if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
                        break;
                    }
                    stage2(inf);
                    ++wide;
                }
            }
        }
        if (!mbar_wait(&S.red_bar[s], ph)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            break;
        }
        if (!(u & kSkip)) {
            const float2* red = S.red + (size_t)s * kNcw * 32 * (MT / 4);
#pragma unroll
            for (int h = 0; h < MT / 4; ++h) {
                if (4 * h + q < inf.m) {
                    float2 sum = make_float2(0.f, 0.f);
#pragma unroll
                    for (int w = 0; w < kNcw; ++w) {
                        const float2 v = red[(w * (MT / 4) + h) * 32 + lane];
                        sum.x += v.x;
                        sum.y += v.y;
                    }
                    out(u, inf.asg[4 * h + q], g, sum);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
        if (++s == S.n_stages) {
            s = 0;
            ph ^= 1;
        }
    }
    // copies of a second quad that no consumer waited for (error paths)
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// ------------------------------------------------------------------------
// Tensor-core consumers.  Consumer warp w owns the groups [g0, g0 + n) of the
// unit's K range (g0 = w*ng/kNcw) for every unit of the CTA, so the B
// fragments of its range (the quantised activations) are loaded into
// registers once per tile, from the activation tile the producer staged.
// Thread (g = lane/4, q = lane%4) accumulates MMA rows g (block A) and g+8
// (block B) for token slot q in fp32, and per unit writes its partial to the
// stage's reduction slot.
// ------------------------------------------------------------------------
// d += A.B (pure: not volatile, so the compiler may interleave the MMAs of
// independent groups).
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}

template <int NPG>
struct Words {
    uint32_t w[NPG];
};
template <int NPG>
__device__ __forceinline__ Words<NPG> lds_w(uint32_t a) {
    Words<NPG> r;
    if constexpr (NPG == 1) {
        r.w[0] = lds32(a);
    } else if constexpr (NPG == 2) {
        const uint2 v = lds64(a);
        r.w[0] = v.x;
        r.w[1] = v.y;
    } else {
        const uint4 v = lds128(a);
        r.w[0] = v.x;
        r.w[1] = v.y;
        r.w[2] = v.z;
        r.w[3] = v.w;
    }
    return r;
}

// B fragments of NG groups (registers).  A warp owns n <= NG groups of the
// unit's K range; the kernels are built for a few NG per NPG (ng_bucket) and
// the groups past n are masked (zero B fragments and (k/254, S) = 0, so they
// add exactly 0).  The (k/254, S) pairs of the warp's groups live in shared
// memory, NG x kMT per warp, written and read by the owning warp only.
template <int NPG, int NG, int MT>
struct WarpAct {
    uint2 b[NG][NPG][MT / 4];  // per token quad: slots 4h .. 4h+3
};

// Copy the warp's B fragments and (k/254, S) pairs of column quad QH of the
// current tile from the staged activation tile (slots t < m hold tokens
// 4*QH + t; the rest are zero).
template <int NPG, int NG, int MT, int QH>
__device__ __forceinline__ void load_act(WarpAct<NPG, NG, MT>& A, float2* kp_w,
                                         const StreamSmem& S, int g0, int n, int m) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int bd = g & 1;
    const int bt = g >> 1;
    const uint32_t base = smem_addr(S.act) + bt * S.act_row + bd * 32;
#pragma unroll
    for (int G = 0; G < NG; ++G) {
#pragma unroll
        for (int i = 0; i < NPG; ++i) {
            const int wi = q * NPG + i;
            const int chunk = (g0 + G) * NPG + (wi >> 2);
            A.b[G][i][QH] = (G < n && bt < m) ? lds64(base + chunk * 64 + (wi & 3) * 8)
                                              : make_uint2(0u, 0u);
        }
    }
    const float4* par = reinterpret_cast<const float4*>(S.act + S.act_slots * S.act_row);
    const int ngr = (int)(S.act_row / (64u * NPG));  // groups in the range
    for (int e = lane; e < NG * kMT; e += 32) {
        const int G = e / kMT, t = e - G * kMT;
        float2 v = make_float2(0.f, 0.f);
        if (G < n && t < m) {
            const float4 p = par[t * ngr + g0 + G];
            v = make_float2(p.x, p.y);
        }
        kp_w[G * MT + QH * kMT + t] = v;
    }
    __syncwarp();
}


// Float rows (down): the warp quantises its groups [g0, g0 + n) of the
// first `rows` rows of the activation tile in place, once per tile, right
// after they land -- a group's gs fp32 values (gs*4 bytes)
// become its NPG digit chunks (NPG*64 bytes) followed by its (k/254, S)
// float4.  Each (row, group) item takes gs/4 lanes; two passes of items are
// quantised together (independent shuffle chains); lanes past the last item
// redo it (same data, same bytes written).  Every read of a batch happens
// before the batch's writes, and items never overlap.
template <int NPG>
__device__ __forceinline__ void quant_rows_in_place(const StreamSmem& S, int rows, int g0,
                                                    int n) {
    constexpr int kGs = 32 * NPG, kLpb = kGs / 4, kPer = 32 / kLpb;
    const int lane = threadIdx.x & 31, pos = (lane % kLpb) * 4;
    const int items = rows * n;
    for (int i0 = 0; i0 < items; i0 += 2 * kPer) {
        const int ia = min(i0 + lane / kLpb, items - 1);
        const int ib = min(i0 + kPer + lane / kLpb, items - 1);
        const int ra = ia / n, rb = ib / n;
        uint8_t* ga = S.act + (size_t)ra * S.act_row + (size_t)(g0 + ia - ra * n) * (kGs * 4);
        uint8_t* gb = S.act + (size_t)rb * S.act_row + (size_t)(g0 + ib - rb * n) * (kGs * 4);
        const float4 va = *reinterpret_cast<const float4*>(ga + pos * 4);
        const float4 vb = *reinterpret_cast<const float4*>(gb + pos * 4);
        __syncwarp();
        quantize_block(va, kLpb, reinterpret_cast<uint32_t*>(ga + (pos / kChunk) * 64),
                       reinterpret_cast<float4*>(ga + NPG * 64), pos == 0);
        quantize_block(vb, kLpb, reinterpret_cast<uint32_t*>(gb + (pos / kChunk) * 64),
                       reinterpret_cast<float4*>(gb + NPG * 64), pos == 0);
        __syncwarp();
    }
}

// B fragments and (k/254, S) pairs of the warp's groups for column quad QH
// of a tile, whose m fp32 rows (slots 0..m-1 of the activation tile, tokens
// 4*QH + t) were quantised in place: group G of a slot at G * gs*4 bytes, its
// NPG digit chunks first, then its float4.
template <int NPG, int NG, int MT, int QH>
__device__ __forceinline__ void load_act_inplace(WarpAct<NPG, NG, MT>& A, float2* kp_w,
                                                 const StreamSmem& S, int g0, int n, int m) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int bd = g & 1;
    constexpr uint32_t kGstride = NPG * 128u;
    const uint32_t act = smem_addr(S.act);
    const int bt = g >> 1;
    const uint32_t base = act + (bt < m ? bt : 0) * S.act_row + bd * 32;
#pragma unroll
    for (int G = 0; G < NG; ++G) {
#pragma unroll
        for (int i = 0; i < NPG; ++i) {
            const int wi = q * NPG + i;
            A.b[G][i][QH] = (G < n && bt < m)
                                ? lds64(base + (g0 + G) * kGstride + (wi >> 2) * 64 + (wi & 3) * 8)
                                : make_uint2(0u, 0u);
        }
    }
    for (int e = lane; e < NG * kMT; e += 32) {
        const int G = e / kMT, t = e - G * kMT;
        float2 v = make_float2(0.f, 0.f);
        if (G < n && t < m) {
            const float4 p = *reinterpret_cast<const float4*>(
                S.act + (size_t)t * S.act_row + (size_t)(g0 + G) * kGstride + NPG * 64);
            v = make_float2(p.x, p.y);
        }
        kp_w[G * MT + QH * kMT + t] = v;
    }
    __syncwarp();
}

// This warp's partial dot products of a unit: acc[h].x = MMA row g (block A),
// acc[h].y = row g+8 (block B), for token slot 4h + q.  `st`: the stage
// (shared address); groups g0 .. g0+n-1 of the unit's range (n <= NG; the
// masked groups past n would add exactly 0 and are skipped); kp: shared
// address of this warp's (k/254, S) pairs.
template <int NPG, int NG, int MT, int NQ>
__device__ __forceinline__ void mma_unit(uint32_t st, const Geo& geo, int g0, int n,
                                         const WarpAct<NPG, NG, MT>& A, uint32_t kp,
                                         float2 (&acc)[MT / 4]) {
    static_assert(NQ >= 1 && NQ <= MT / 4, "active token quads");
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    constexpr uint32_t kGroupCode = 4u * 32u * NPG;  // 8 rows x gs/2 bytes
    const uint32_t a_lo = st + g * (16 * NPG) + q * (4 * NPG);
    const uint32_t z_lo = st + geo.pbytes + g * 4;
    const uint32_t kq = kp + q * 8;
#pragma unroll
    for (int h = 0; h < MT / 4; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll
    for (int G = 0; G < NG; ++G) {
        if (G >= n) break;  // warp-uniform
        const uint32_t gg = (uint32_t)(g0 + G);
        const Words<NPG> wl = lds_w<NPG>(a_lo + gg * kGroupCode);
        const Words<NPG> wh = lds_w<NPG>(a_lo + geo.bbytes + gg * kGroupCode);
        const uint32_t pl = lds32(z_lo + gg * 32), ph = lds32(z_lo + geo.bbytes + gg * 32);
        const float2 sl = __half22float2(*reinterpret_cast<const __half2*>(&pl));
        const float2 sh = __half22float2(*reinterpret_cast<const __half2*>(&ph));
        int d[NQ][4];
#pragma unroll
        for (int h = 0; h < NQ; ++h) d[h][0] = d[h][1] = d[h][2] = d[h][3] = 0;
#pragma unroll
        for (int i = 0; i < NPG; ++i) {
            uint32_t a[4];
            a[0] = wl.w[i] & 0x0F0F0F0Fu;
            a[1] = wh.w[i] & 0x0F0F0F0Fu;
            a[2] = (wl.w[i] >> 4) & 0x0F0F0F0Fu;
            a[3] = (wh.w[i] >> 4) & 0x0F0F0F0Fu;
            // the group's slices accumulate in the MMA; the groups are
            // independent chains the compiler interleaves
#pragma unroll
            for (int h = 0; h < NQ; ++h) mma_s8(d[h], a, A.b[G][i][h].x, A.b[G][i][h].y);
        }
        // row += s * (k/254 * (254*A + B) - 8*S) + z * S
#pragma unroll
        for (int h = 0; h < NQ; ++h) {
            const uint2 kv = lds64(kq + (G * MT + 4 * h) * 8);
            const float k2 = __uint_as_float(kv.x), S = __uint_as_float(kv.y);
            const float m8 = -8.0f * S;
            acc[h].x = fmaf(sl.x, fmaf(k2, (float)(d[h][0] * 254 + d[h][1]), m8),
                            fmaf(sl.y, S, acc[h].x));
            acc[h].y = fmaf(sh.x, fmaf(k2, (float)(d[h][2] * 254 + d[h][3]), m8),
                            fmaf(sh.y, S, acc[h].y));
        }
    }
}

// Consumer loop: `upt` units per tile; F32: the activation tile is fp32.
template <int NPG, int NG, int MT, bool F32>
__device__ void consume(const StreamSmem& S, const Ws& W, const Geo& geo, int upt) {
    const int lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 2;
    const int g0 = cw * geo.ng / kNcw, n = (cw + 1) * geo.ng / kNcw - g0;
    float2* kp_w = S.kp + cw * NG * MT;
    const uint32_t st0 = smem_addr(S.stages), kp = smem_addr(kp_w);
    WarpAct<NPG, NG, MT> A;
    int tile_end = -1, tiles = 0, wide = 0, s = 0, nq = 1;
    uint32_t ph = 0;
    for (;;) {
        if (!mbar_wait(&S.full[s], ph)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            break;
        }
        const UnitInfo& inf = S.info[s];
        const int uf = *reinterpret_cast<const volatile int*>(&inf.u);
        if (uf == -1) break;
        const int u = uf & ~kSkip;
        if (u >= tile_end) {  // first unit of a tile (units arrive in increasing order)
            tile_end = (u / upt + 1) * upt;
            if (!mbar_wait(S.act_full, tiles & 1)) {
                if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
                break;
            }
            const int m = inf.m, m0 = min(m, kMT);
            if constexpr (F32) {
                quant_rows_in_place<NPG>(S, m0, g0, n);
                load_act_inplace<NPG, NG, MT, 0>(A, kp_w, S, g0, n, m0);
            } else {
                load_act<NPG, NG, MT, 0>(A, kp_w, S, g0, n, m0);
            }
            nq = 1;
            if constexpr (MT > kMT) {
                if (m > kMT) {  // the second column quad, staged by the reducer
                    if (lane == 0) mbar_arrive(S.act_mid);
                    if (!mbar_wait(S.act_full2, wide & 1)) {
                        if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
                        break;
                    }
                    ++wide;
                    if constexpr (F32) {
                        quant_rows_in_place<NPG>(S, m - kMT, g0, n);
                        load_act_inplace<NPG, NG, MT, 1>(A, kp_w, S, g0, n, m - kMT);
                    } else {
                        load_act<NPG, NG, MT, 1>(A, kp_w, S, g0, n, m - kMT);
                    }
                    nq = 2;
                }
            }
            if (lane == 0) mbar_arrive(S.act_empty);
            ++tiles;
        }
        float2 part[MT / 4];
#pragma unroll
        for (int h = 0; h < MT / 4; ++h) part[h] = make_float2(0.f, 0.f);
        if (!(uf & kSkip)) {
            if constexpr (MT > kMT) {
                if (nq == 2)
                    mma_unit<NPG, NG, MT, 2>(st0 + s * S.stage_bytes, geo, g0, n, A, kp, part);
                else
                    mma_unit<NPG, NG, MT, 1>(st0 + s * S.stage_bytes, geo, g0, n, A, kp, part);
            } else {
                mma_unit<NPG, NG, MT, 1>(st0 + s * S.stage_bytes, geo, g0, n, A, kp, part);
            }
        }
        float2* red = S.red + ((size_t)s * kNcw + cw) * 32 * (MT / 4);
#pragma unroll
        for (int h = 0; h < MT / 4; ++h)
            if (h < nq) red[h * 32 + lane] = part[h];
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.red_bar[s]);
        if (++s == S.n_stages) {
            s = 0;
            ph ^= 1;
        }
    }
}

// ------------------------------------------------------------------------
// gate/up + SwiGLU: unit = gate block b + up block b (8 output rows) x all of H
// ------------------------------------------------------------------------
template <int NPG, int NG, int MT>
__global__ void __launch_bounds__(kStreamCta, 1)
gateup_kernel(LayerArgs L, Ws W, int n_stages, uint32_t stage_bytes) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int H = L.H, I = L.I, gs = L.gs;
    const Geo geo = make_geo(H / gs, gs);
    const StreamSmem S =
        stream_smem(smem_raw, n_stages, stage_bytes, geo, NPG, false, L.act_slots, MT, NG);
    stream_init(S);
    pdl_wait();
    pdl_launch();
    const int warp = threadIdx.x >> 5;
    const int rbs = I / 8;  // 8-row blocks per matrix
    const int ntiles = __ldcg(W.counters + C_NTILES);
    const long long total = (long long)ntiles * rbs;

    if (warp == 0) {
        {
            // the record of the first tile if the plan has tiles_hint tiles, read
            // alongside the tile count (both come from the previous kernel)
            TileView<MT> spec;
            int spec_ti = -1;
            if (L.tiles_hint > 0) {
                const long long th = (long long)L.tiles_hint * rbs;
                spec_ti = (int)(th * blockIdx.x / gridDim.x / rbs);
                if (spec_ti < W.max_tiles)
                    load_tile(W.tiles + spec_ti, spec);
                else
                    spec_ti = -1;
            }
            const int b = (int)(total * blockIdx.x / gridDim.x);
            const int e = (int)(total * (blockIdx.x + 1) / gridDim.x);
            const size_t bb = block_bytes_of(H, gs);
            const size_t off_g = L.mat[0].packed, off_u = L.mat[1].packed;
            const ActSrc as{reinterpret_cast<const uint8_t*>(W.xq), W.xqp, nullptr, H / kChunk,
                            H / gs, 0, NPG, gs, H, false};
            const UnitAddr ua{off_g, bb, {0, 4 * (size_t)H, off_u - off_g, off_u - off_g + 4 * (size_t)H}};
            produce<MT>(S, W, b, e, rbs, ntiles, geo, as, false, ua, false,
                        spec_ti >= 0 ? &spec : nullptr, spec_ti);
        }
        return;
    }
    if (warp == 1) {
        const int lane = threadIdx.x & 31;
        const uint32_t rowb = act_row_bytes(geo.ng, NPG, false), pb = (uint32_t)geo.ng * 16u;
        reduce_units<MT>(
            S, W,
            [&](int u, int asg, int g, float2 v) {
                const size_t row = (size_t)(u % rbs) * 8 + g;
                W.h[(size_t)asg * I + row] = v.x / (1.0f + expf(-v.x)) * v.y;
            },
            [&](const UnitInfo& inf) {  // tokens kMT.. of the tile: words, then (k/254, S)
                const int m2 = inf.m - kMT;
                for (int t = 0; t < m2; ++t) {
                    const int tok = inf.tok[kMT + t];
                    const uint8_t* xw = reinterpret_cast<const uint8_t*>(W.xq) +
                                        (size_t)tok * (H / kChunk) * 64;
                    const uint8_t* xp = reinterpret_cast<const uint8_t*>(W.xqp + (size_t)tok * (H / gs));
                    for (uint32_t i = lane; i < rowb / 16; i += 32)
                        ldgsts16(S.act + (size_t)t * rowb + i * 16, xw + i * 16);
                    for (uint32_t i = lane; i < pb / 16; i += 32)
                        ldgsts16(S.act + (size_t)S.act_slots * rowb + t * pb + i * 16, xp + i * 16);
                }
                ldgsts_arrive(S.act_full2);
                __syncwarp();
                if (lane == 0) mbar_arrive(S.act_full2);
            });
        return;
    }
    consume<NPG, NG, MT, false>(S, W, geo, rbs);
}

// ------------------------------------------------------------------------
// down projection: unit = blocks 2j, 2j+1 (16 output rows) x one of kp K
// parts.  CTA c serves part c % kp, with a contiguous range of the part's
// units.  Each part is written to its own ypart buffer and the combine adds
// them in fixed order (deterministic, no float atomics).
// ------------------------------------------------------------------------
template <int NPG, int NG, int MT>
__global__ void __launch_bounds__(kStreamCta, 1)
down_kernel(LayerArgs L, Ws W, int n_stages, uint32_t stage_bytes) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int kp = L.kp;
    const int H = L.H, I = L.I, gs = L.gs;
    const int ngp = I / gs / kp;  // groups per part
    const Geo geo = make_geo(ngp, gs);
    const StreamSmem S =
        stream_smem(smem_raw, n_stages, stage_bytes, geo, NPG, true, L.act_slots, MT, NG);
    stream_init(S);
    // Weights, the expert table and the tile plan (written by the router,
    // which completed before the gate/up kernel could start) do not depend on
    // the previous kernel (gate/up, which writes h): the producer waits for it
    // only before the first activation copy, so these CTAs start streaming
    // weights on SMs that gate/up's CTAs have already left.
    pdl_launch();
    const int warp = threadIdx.x >> 5;
    const int pi = blockIdx.x % kp;
    const int cpp = (gridDim.x - pi + kp - 1) / kp;  // CTAs serving this part
    const int upt = H / 16;
    const int ntiles = __ldcg(W.counters + C_NTILES);
    const long long total = (long long)ntiles * upt;

    if (warp == 0) {
        {
            const int j = blockIdx.x / kp;
            const int b = (int)(total * j / cpp), e = (int)(total * (j + 1) / cpp);
            const size_t bb = block_bytes_of(I, gs);
            const size_t z_off = 4 * (size_t)I + (size_t)pi * geo.ng * 32;
            const size_t p_off = (size_t)pi * geo.pbytes;
            const ActSrc as{nullptr, nullptr, W.h, I / kChunk, I / gs, pi * ngp, NPG, gs, I, true};
            const UnitAddr ua{L.mat[2].packed, 2 * bb, {p_off, z_off, bb + p_off, bb + z_off}};
            produce<MT>(S, W, b, e, upt, ntiles, geo, as, true, ua, true);
        }
        return;
    }
    if (warp == 1) {
        {
            // the first activation tile of the range, as soon as h is complete
            const int j = blockIdx.x / kp;
            const int b = (int)(total * j / cpp), e = (int)(total * (j + 1) / cpp);
            if (b < e) {
                TileView<kMT> tl;
                load_tile(W.tiles + b / upt, tl);
                pdl_wait();
                copy_rows_lsu(S.act, act_row_bytes(ngp, NPG, true), min(tl.m, S.act_slots),
                              [&](int t) {
                    return W.h + (size_t)tl.asg[t] * I + (size_t)pi * ngp * gs;
                }, S.act_full);
            }
        }
        reduce_units<MT>(
            S, W,
            [&](int u, int asg, int g, float2 v) {
                const size_t row = (size_t)(u % upt) * 16 + g;
                float* dst = W.ypart + ((size_t)pi * W.A + asg) * H + row;
                dst[0] = v.x;
                dst[8] = v.y;
            },
            [&](const UnitInfo& inf) {  // rows of assignments kMT.. of the tile
                copy_rows_lsu(S.act, act_row_bytes(ngp, NPG, true), inf.m - kMT, [&](int t) {
                    return W.h + (size_t)inf.asg[kMT + t] * I + (size_t)pi * ngp * gs;
                }, S.act_full2);
            });
        return;
    }
    consume<NPG, NG, MT, true>(S, W, geo, upt);
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------
struct Layout {
    size_t status, counters, tok_cnt, logits, topk_idx, topk_w, pidx, pw, tiles,
        xn, xq, xqp, h, hs, ypart, total;
    int A, max_tiles;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Layout make_layout(int T, int H, int I, int E, int K, bool shared, int si = 0) {
    Layout l{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    l.A = T * K + (shared ? T : 0);
    l.max_tiles = T * K + E + T + 1;
    l.status = take(4 * sizeof(int));
    l.counters = take(kCounters * sizeof(int));
    l.tok_cnt = take((size_t)T * sizeof(int));
    l.logits = take((size_t)T * E * ((H + kSlice - 1) / kSlice) * sizeof(float));
    l.topk_idx = take((size_t)T * K * sizeof(int));
    l.topk_w = take((size_t)T * K * sizeof(float));
    l.pidx = take((size_t)T * K * sizeof(int));
    l.pw = take((size_t)T * K * sizeof(float));
    l.tiles = take((size_t)l.max_tiles * sizeof(Tile));
    l.xn = take((size_t)T * H * sizeof(float));
    l.xq = take((size_t)T * (H / kChunk) * 64);
    l.xqp = take((size_t)T * (H / kChunk) * sizeof(float4));  // >= per-group params
    l.h = take((size_t)l.A * I * sizeof(float));
    l.hs = take((size_t)T * si * sizeof(float));
    l.ypart = take((size_t)kMaxKp * l.A * H * sizeof(float));
    l.total = o;
    return l;
}

Ws make_ws(void* base, const Layout& l) {
    char* b = static_cast<char*>(base);
    Ws w{};
    w.status = reinterpret_cast<int*>(b + l.status);
    w.counters = reinterpret_cast<int*>(b + l.counters);
    w.tok_cnt = reinterpret_cast<int*>(b + l.tok_cnt);
    w.logits = reinterpret_cast<float*>(b + l.logits);
    w.topk_idx = reinterpret_cast<int*>(b + l.topk_idx);
    w.topk_w = reinterpret_cast<float*>(b + l.topk_w);
    w.prev_idx = reinterpret_cast<int*>(b + l.pidx);
    w.prev_w = reinterpret_cast<float*>(b + l.pw);
    w.tiles = reinterpret_cast<Tile*>(b + l.tiles);
    w.xn = reinterpret_cast<float*>(b + l.xn);
    w.xq = reinterpret_cast<uint4*>(b + l.xq);
    w.xqp = reinterpret_cast<float4*>(b + l.xqp);
    w.h = reinterpret_cast<float*>(b + l.h);
    w.hs = reinterpret_cast<float*>(b + l.hs);
    w.ypart = reinterpret_cast<float*>(b + l.ypart);
    w.A = l.A;
    w.max_tiles = l.max_tiles;
    return w;
}

MatOff mat_off(const WispExpertMeta& m, int i) {
    return {(unsigned long long)m.packed_off[i], (unsigned long long)m.scales_off[i],
            (unsigned long long)m.zeros_off[i]};
}

// Group counts per consumer warp the streaming kernels are built for (per
// NPG = gs / 32); a warp's actual count is rounded up to the next one and the
// rest masked.
constexpr int kNgSet1[] = {1, 2, 4, 8, 16};
constexpr int kNgSet2[] = {1, 2, 4, 7, 8};
constexpr int kNgSet4[] = {1, 2};
template <size_t N>
int bucket_in(const int (&set)[N], int need) {
    for (size_t i = 0; i < N; ++i)
        if (set[i] >= need) return set[i];
    return 0;
}
int ng_bucket(int npg, int ng) {
    const int need = std::max(1, (ng + kNcw - 1) / kNcw);
    return npg == 1 ? bucket_in(kNgSet1, need) : npg == 2 ? bucket_in(kNgSet2, need)
                                                          : bucket_in(kNgSet4, need);
}

// Smallest split of the down projection's K (= I) into parts of whole quant
// groups, each at most kMaxPartK wide; 0 when none exists.
int min_down_parts(int I, int gs) {
    const int G = I / gs;
    for (int kp = 1; kp <= kMaxKp; ++kp)
        if (G % kp == 0 && (I / kp) <= kMaxPartK) return kp;
    return 0;
}

bool check_layer(const WispMoeLayer* ly, int T, WispErrCtx* err) {
    const WispExpertMeta& m = ly->meta;
    const int H = (int)m.cols[0], I = (int)m.rows[0], gs = (int)m.group_size;
    if (!m.valid || m.rows[1] != (uint32_t)I || m.cols[1] != (uint32_t)H ||
        m.rows[2] != (uint32_t)H || m.cols[2] != (uint32_t)I) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: expert meta invalid or not gate/up [I,H], down [H,I]");
        return false;
    }
    if (H % kChunk || I % kChunk || H % gs || I % gs || H % 16 || I % 8 ||
        (gs != 32 && gs != 64 && gs != 128)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: unsupported shape H=%d I=%d group_size=%d (need multiples "
                   "of 32, H of 16, group_size 32/64/128 dividing H and I)",
                   H, I, gs);
        return false;
    }
    if (ly->gating != WISP_GATING_SOFTMAX && ly->gating != WISP_GATING_SIGMOID) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe layer: unknown gating %d", ly->gating);
        return false;
    }
    if (ly->n_experts <= 0 || ly->n_experts > 1024 || ly->top_k <= 0 ||
        ly->top_k > ly->n_experts || ly->top_k > 64) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe layer: n_experts=%d top_k=%d",
                   ly->n_experts, ly->top_k);
        return false;
    }
    if (T <= 0 || T * ly->top_k > kMaxPlanAssign) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe layer: T=%d (T*top_k must be <= %d)", T,
                   kMaxPlanAssign);
        return false;
    }
    if (!ly->expert_blobs || !ly->router_w) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe layer: NULL expert table or router");
        return false;
    }
    if (ly->shared_gate || ly->shared_up || ly->shared_down) {
        if (ly->shared_blob ||
            !dense_ffn_shape_ok(ly->shared_gate, ly->shared_up, ly->shared_down,
                                ly->shared_inter, H)) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "moe layer: fp16-dense shared expert needs gate, up and down (16-byte "
                       "aligned), shared_inter a positive multiple of 8 (got %d), and no int4 "
                       "shared blob beside it",
                       ly->shared_inter);
            return false;
        }
    }
    if (ly->shared_blob) {
        const WispExpertMeta& s = ly->shared_meta;
        if (!s.valid || s.cols[0] != (uint32_t)H || s.rows[0] != (uint32_t)I ||
            s.group_size != (uint32_t)gs || !s.tiled) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "moe layer: shared expert must match the routed experts' shape, group "
                       "size and tiled layout");
            return false;
        }
    }
    if (!m.tiled) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: expert blobs must be in the tiled device layout (see "
                   "wisp_expert_tile); meta describes a .bin blob");
        return false;
    }
    if (H > kMaxPartK || !ng_bucket(gs / kChunk, H / gs)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe layer: hidden %d above the supported %d", H,
                   kMaxPartK);
        return false;
    }
    if (min_down_parts(I, gs) == 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: intermediate %d cannot be split into at most %d parts of whole "
                   "quant groups of at most %d elements",
                   I, kMaxKp, kMaxPartK);
        return false;
    }
    return true;
}

// Shared memory of a streaming CTA (one per SM): as many ring stages (each
// with its reduction slot) as fit, up to 8.
struct StreamCfg {
    int stages = 0, blocks = 0;
    uint32_t stage_bytes = 0;
    size_t smem = 0;
};

constexpr size_t kSmemPerCta = 227 * 1024;

// Stages: enough to keep about kInFlight bytes of weights in flight per SM
// (more only lengthens the DRAM queues every other load waits in), at least
// 2, at most 8, within the shared memory left after the activation tile.
constexpr size_t kInFlight = 192 * 1024;
constexpr int kMaxStages = 12;

StreamCfg plan_stream(const Geo& geo, int npg, bool f32, int slots, int mt) {
    StreamCfg c;
    c.stage_bytes = stage_bytes_of(geo);
    const uint32_t act = act_bytes_of(geo.ng, npg, f32, slots);
    const int ng = ng_bucket(npg, geo.ng);
    int want = (int)((kInFlight + c.stage_bytes / 2) / c.stage_bytes);
    want = std::max(2, std::min(kMaxStages, want));
    c.stages = 0;
    for (int st = want; st >= 2; --st)
        if (stream_smem_bytes(st, c.stage_bytes, act, mt, ng) <= kSmemPerCta) {
            c.stages = st;
            break;
        }
    c.smem = stream_smem_bytes(c.stages, c.stage_bytes, act, mt, ng);
    return c;
}

int down_parts(int I, int gs, long long units, int ctas, int slots, int mt);

LayerArgs layer_args(const WispMoeLayer* ly, int T, int ctas) {
    LayerArgs a{};
    a.blobs = ly->expert_blobs;
    a.shared_blob = ly->shared_blob;
    a.router_w = reinterpret_cast<const __half*>(ly->router_w);
    a.router_bias = reinterpret_cast<const __half*>(ly->router_bias);
    a.norm_w = reinterpret_cast<const __half*>(ly->norm_w);
    for (int i = 0; i < 3; ++i) {
        a.mat[i] = mat_off(ly->meta, i);
        a.smat[i] = ly->shared_blob ? mat_off(ly->shared_meta, i) : MatOff{0, 0, 0};
    }
    a.H = (int)ly->meta.cols[0];
    a.I = (int)ly->meta.rows[0];
    a.E = ly->n_experts;
    a.K = ly->top_k;
    a.gs = (int)ly->meta.group_size;
    a.has_shared = ly->shared_blob ? 1 : (ly->shared_gate ? 2 : 0);
    a.sg = reinterpret_cast<const __half*>(ly->shared_gate);
    a.su = reinterpret_cast<const __half*>(ly->shared_up);
    a.sd = reinterpret_cast<const __half*>(ly->shared_down);
    a.si = a.has_shared == 2 ? ly->shared_inter : 0;
    a.gating = ly->gating;
    // Tokens per expert tile: up to 4 (one MMA column quad) while no expert can
    // have more (T <= 4); beyond, up to 8, so an expert with 5..8 tokens
    // streams its weights once instead of twice.  The activation tile stages
    // one quad at a time either way.
    // (Two quads hold twice the B fragments in registers: past 4 groups per
    // consumer warp -- H above 64 quant groups -- they spill, and the layer
    // keeps 4-token tiles.)
    const int npg = a.gs / kChunk;
    a.mt = T > kMT && ng_bucket(npg, a.H / a.gs) <= kWideMaxNg ? kMaxTile : kMT;
    a.act_slots = std::min(T, kMT);
    const long long tiles = std::min<long long>((long long)ly->n_experts, (long long)T * a.K) +
                            (a.has_shared == 1 ? (T + a.mt - 1) / a.mt : 0);
    a.tiles_hint = (int)std::min<long long>(tiles, (long long)T * a.K + a.E + T + 1);
    a.kp = down_parts(a.I, a.gs, tiles * (a.H / 16), ctas, a.act_slots, a.mt);
    if (a.mt == kMaxTile && ng_bucket(npg, a.I / a.gs / a.kp) > kWideMaxNg) {
        a.mt = kMT;
        a.kp = down_parts(a.I, a.gs, tiles * (a.H / 16), ctas, a.act_slots, a.mt);
    }
    return a;
}

StreamCfg gateup_cfg(const LayerArgs& a) {
    return plan_stream(make_geo(a.H / a.gs, a.gs), a.gs / kChunk, false, a.act_slots, a.mt);
}

StreamCfg down_cfg(const LayerArgs& a) {
    return plan_stream(make_geo(a.I / a.gs / a.kp, a.gs), a.gs / kChunk, true, a.act_slots, a.mt);
}

// K parts of the down projection.  A part is a whole number of quant groups
// and at most kMaxPartK wide (the consumer warps hold its activations in
// registers).  Among the valid splits, pick the one that wastes least: masked
// groups (the per-warp group count rounded up to a built bucket), uneven
// units per CTA (`units` = down units of one part, tiles x H/16), and a small
// cost per extra part (the combine reads every part).
int down_parts(int I, int gs, long long units, int ctas, int slots, int mt) {
    const int G = I / gs, npg = gs / kChunk;
    int best = 0;
    double best_score = -1.0;
    for (int kp = 1; kp <= kMaxKp; ++kp) {
        if (G % kp || I / kp > kMaxPartK) continue;
        const int ngp = G / kp, ng = ng_bucket(npg, ngp);
        if (!ng) continue;
        const double eff = std::min(1.0, (double)ngp / (double)(ng * kNcw));
        const double per = (double)units * kp / (double)ctas;
        const double bal = per > 0 ? per / std::ceil(per) : 1.0;
        // a shallow ring (big stages) starves the consumers while a stage turns
        // over; small units pay the fixed per-unit cost (barriers, reduction)
        const Geo geo = make_geo(ngp, gs);
        const int st = plan_stream(geo, npg, true, slots, mt).stages;
        const double depth = std::min(1.0, st / 4.0);
        const double size = std::min(1.0, 2.0 * geo.bbytes / 32768.0);
        const double score = eff * bal * depth * size * (1.0 - 0.01 * kp);
        if (score > best_score + 1e-9) {
            best_score = score;
            best = kp;
        }
    }
    return best ? best : 1;
}

template <typename K>
cudaError_t finish_cfg(K kern, StreamCfg& c) {
    if (c.stages < 2) return cudaErrorInvalidConfiguration;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    c.blocks = sms;
    return cudaSuccess;
}

struct DevInfo {
    int sms = 0;
};

DevInfo dev_info() {
    static std::mutex mu;
    static DevInfo cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = cache[dev & 63];
    if (!d.sms) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    return d;
}

size_t router_smem(int E) {
    return std::max((size_t)plan_scratch_ints(E), (size_t)kWarps * 3 * E) * sizeof(int);
}
constexpr int kMaxHidden = 8192;

cudaError_t ensure_attrs(int H) {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (done[dev & 63]) return cudaSuccess;
    (void)H;
    cudaError_t e = cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)std::max(prep_smem_bytes(kMaxHidden, 1, 1024),
                                                       prep_smem_bytes(kMaxHidden, 8, 1024)));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)router_smem(1024));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)router_smem(1024));
    if (e != cudaSuccess) return e;
    done[dev & 63] = true;
    return cudaSuccess;
}

// CTAs per token in prep: the largest of 8/4/2/1 that splits the row into
// whole quant groups.
int prep_cluster(int H, int gs) {
    for (int cs = 8; cs > 1; cs >>= 1)
        if (H % (cs * gs) == 0) return cs;
    return 1;
}

// Router inside prep (every token's cluster reads the whole router matrix)
// unless that re-reads more than 32 MB; then the separate router kernel,
// which reads it once for all tokens.
bool route_in_prep(const LayerArgs& a, int T) {
    return (size_t)T * a.E * a.H * 2 <= ((size_t)32 << 20);
}

int plan_tokens(const LayerArgs& a, int T) { return T == 1 ? 1 : a.mt; }

// Optional profiling hook: when set, an event is recorded on the launch stream
// before every kernel of the fused path and once after the last, so a caller
// can read per-kernel durations (the events serialise the PDL overlap).
struct ProfileHook {
    cudaEvent_t* ev = nullptr;
    int cap = 0, n = 0;
};
thread_local ProfileHook g_hook;

void hook_mark(cudaStream_t s) {
    if (g_hook.ev && g_hook.n < g_hook.cap) cudaEventRecord(g_hook.ev[g_hook.n++], s);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args&&... args) {
    hook_mark(s);
    return launch_pdl(kern, grid, block, smem, s, std::forward<Args>(args)...);
}



template <int NPG, int NG, int MT>
cudaError_t launch_gateup(const LayerArgs& a, const Ws& W, cudaStream_t s) {
    StreamCfg c = gateup_cfg(a);
    cudaError_t e = finish_cfg(gateup_kernel<NPG, NG, MT>, c);
    if (e != cudaSuccess) return e;
    return launch(gateup_kernel<NPG, NG, MT>, dim3(c.blocks), dim3(kStreamCta), c.smem, s, a,
                  W, c.stages, c.stage_bytes);
}

template <int NPG, int NG, int MT>
cudaError_t launch_down(const LayerArgs& a, const Ws& W, cudaStream_t s) {
    StreamCfg c = down_cfg(a);
    cudaError_t e = finish_cfg(down_kernel<NPG, NG, MT>, c);
    if (e != cudaSuccess) return e;
    return launch(down_kernel<NPG, NG, MT>, dim3(c.blocks), dim3(kStreamCta), c.smem, s, a, W,
                  c.stages, c.stage_bytes);
}

cudaError_t launch_gateup_any(int npg, int ng, int mt, const LayerArgs& a, const Ws& W,
                              cudaStream_t s) {
    switch (mt * 1000 + npg * 100 + ng) {
        case 4101: return launch_gateup<1, 1, 4>(a, W, s);
        case 4102: return launch_gateup<1, 2, 4>(a, W, s);
        case 4104: return launch_gateup<1, 4, 4>(a, W, s);
        case 4108: return launch_gateup<1, 8, 4>(a, W, s);
        case 4116: return launch_gateup<1, 16, 4>(a, W, s);
        case 4201: return launch_gateup<2, 1, 4>(a, W, s);
        case 4202: return launch_gateup<2, 2, 4>(a, W, s);
        case 4204: return launch_gateup<2, 4, 4>(a, W, s);
        case 4207: return launch_gateup<2, 7, 4>(a, W, s);
        case 4208: return launch_gateup<2, 8, 4>(a, W, s);
        case 4401: return launch_gateup<4, 1, 4>(a, W, s);
        case 4402: return launch_gateup<4, 2, 4>(a, W, s);
        case 8101: return launch_gateup<1, 1, 8>(a, W, s);
        case 8102: return launch_gateup<1, 2, 8>(a, W, s);
        case 8104: return launch_gateup<1, 4, 8>(a, W, s);
        case 8108: return launch_gateup<1, 8, 8>(a, W, s);
        case 8116: return launch_gateup<1, 16, 8>(a, W, s);
        case 8201: return launch_gateup<2, 1, 8>(a, W, s);
        case 8202: return launch_gateup<2, 2, 8>(a, W, s);
        case 8204: return launch_gateup<2, 4, 8>(a, W, s);
        case 8207: return launch_gateup<2, 7, 8>(a, W, s);
        case 8208: return launch_gateup<2, 8, 8>(a, W, s);
        case 8401: return launch_gateup<4, 1, 8>(a, W, s);
        case 8402: return launch_gateup<4, 2, 8>(a, W, s);
        default: return cudaErrorInvalidConfiguration;
    }
}

cudaError_t launch_down_any(int npg, int ng, int mt, const LayerArgs& a, const Ws& W,
                            cudaStream_t s) {
    switch (mt * 1000 + npg * 100 + ng) {
        case 4101: return launch_down<1, 1, 4>(a, W, s);
        case 4102: return launch_down<1, 2, 4>(a, W, s);
        case 4104: return launch_down<1, 4, 4>(a, W, s);
        case 4108: return launch_down<1, 8, 4>(a, W, s);
        case 4116: return launch_down<1, 16, 4>(a, W, s);
        case 4201: return launch_down<2, 1, 4>(a, W, s);
        case 4202: return launch_down<2, 2, 4>(a, W, s);
        case 4204: return launch_down<2, 4, 4>(a, W, s);
        case 4207: return launch_down<2, 7, 4>(a, W, s);
        case 4208: return launch_down<2, 8, 4>(a, W, s);
        case 4401: return launch_down<4, 1, 4>(a, W, s);
        case 4402: return launch_down<4, 2, 4>(a, W, s);
        case 8101: return launch_down<1, 1, 8>(a, W, s);
        case 8102: return launch_down<1, 2, 8>(a, W, s);
        case 8104: return launch_down<1, 4, 8>(a, W, s);
        case 8108: return launch_down<1, 8, 8>(a, W, s);
        case 8116: return launch_down<1, 16, 8>(a, W, s);
        case 8201: return launch_down<2, 1, 8>(a, W, s);
        case 8202: return launch_down<2, 2, 8>(a, W, s);
        case 8204: return launch_down<2, 4, 8>(a, W, s);
        case 8207: return launch_down<2, 7, 8>(a, W, s);
        case 8208: return launch_down<2, 8, 8>(a, W, s);
        case 8401: return launch_down<4, 1, 8>(a, W, s);
        case 8402: return launch_down<4, 2, 8>(a, W, s);
        default: return cudaErrorInvalidConfiguration;
    }
}

cudaError_t launch_streams(const LayerArgs& a, const Ws& W, int T, cudaStream_t s) {
    const int npg = a.gs / kChunk;
    (void)T;
    cudaError_t e = launch_gateup_any(npg, ng_bucket(npg, a.H / a.gs), a.mt, a, W, s);
    if (e != cudaSuccess) return e;
    return launch_down_any(npg, ng_bucket(npg, a.I / a.gs / a.kp), a.mt, a, W, s);
}

cudaError_t launch_router(const LayerArgs& a, const Ws& W, int T, const float* xin,
                          cudaStream_t s, bool plan = true) {
    const int mt = plan ? plan_tokens(a, T) : 0;
    const int nsl = (a.H + kSlice - 1) / kSlice;
    const int blocks = (a.E * nsl + kWarps - 1) / kWarps;
    return launch(router_kernel, dim3(blocks), dim3(kThreads), router_smem(a.E), s, a, W, T, mt,
                  xin, nsl);
}

// The fp16-dense shared expert of a layer (has_shared == 2) on its input xin
// [T, H]: h into W.hs, the result into part 0 of the shared rows of ypart
// (assignments T*K + t), which the combine adds first with weight 1.
cudaError_t launch_dense_shared(const LayerArgs& a, const Ws& W, int T, const float* xin,
                                cudaStream_t s) {
    if (a.has_shared != 2) return cudaSuccess;
    return launch_dense_ffn(a.sg, a.su, a.sd, a.si, a.H, xin, a.H, W.hs,
                            W.ypart + (size_t)T * a.K * a.H, a.H, T, s, hook_mark);
}

// Run one layer's router + expert kernels.  The layer's input is already
// quantised in W.xq (and xin holds the router input).
// prep over T tokens (one cluster per token).  P_ROUTE is added when the
// router runs inside prep; otherwise the separate router kernel follows.
cudaError_t launch_prep(const LayerArgs& a, const Ws& W, int T, int flags, float* x, float* y,
                        float eps, int prevK, int prev_sh, int prev_kp, cudaStream_t s,
                        bool plan = true) {
    const int cs = prep_cluster(a.H, a.gs);
    hook_mark(s);
    return launch_pdl_cluster(prep_kernel, dim3(T * cs), dim3(kPrepThreads),
                              prep_smem_bytes(a.H, cs, a.E), s, cs, a, W, T, flags, x, y, eps,
                              prevK, prev_sh, prev_kp, plan ? plan_tokens(a, T) : 0);
}

// Routing of a layer whose input prep is about to quantise: the router in
// prep, or prep then the router kernel on `xin`.
cudaError_t launch_prep_route(const LayerArgs& a, const Ws& W, int T, int flags, float* x,
                              float eps, int prevK, int prev_sh, int prev_kp, const float* xin,
                              cudaStream_t s, bool plan = true) {
    const bool fused = route_in_prep(a, T);
    cudaError_t e = launch_prep(a, W, T, flags | (fused ? (int)P_ROUTE : 0), x, nullptr, eps,
                                prevK, prev_sh, prev_kp, s, plan);
    if (e != cudaSuccess || fused) return e;
    return launch_router(a, W, T, xin, s, plan);
}

}  // namespace

int sm_count() { return dev_info().sms; }

cudaError_t launch_zero_words(int* p, int n_words, cudaStream_t stream) {
    return launch_pdl(zero_words_kernel, dim3(1), dim3(256), 0, stream, p, n_words);
}

}  // namespace wb

using namespace wb;

extern "C" void wisp_moe_profile_events(void* events, int n_events) {
    g_hook.ev = static_cast<cudaEvent_t*>(events);
    g_hook.cap = events ? n_events : 0;
    g_hook.n = 0;
}

extern "C" int wisp_moe_profile_count(void) { return g_hook.n; }

extern "C" size_t wisp_moe_workspace_bytes(const WispMoeLayer* layers, int n_layers, int T) {
    size_t best = 0;
    for (int i = 0; i < n_layers; ++i) {
        const WispMoeLayer& l = layers[i];
        const bool dense_sh = l.shared_gate != nullptr;
        Layout lo = make_layout(T, (int)l.meta.cols[0], (int)l.meta.rows[0], l.n_experts,
                                l.top_k, l.shared_blob != nullptr || dense_sh,
                                dense_sh ? l.shared_inter : 0);
        best = std::max(best, lo.total);
    }
    return best;
}

extern "C" int wisp_moe_status(const void* workspace, cudaStream_t stream) {
    int v = 0;
    if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
        return -1;
    return v;
}

static WispError common_checks(const WispMoeLayer* layers, int n_layers, int T, void* ws,
                               size_t ws_bytes, WispErrCtx* err) {
    if (!layers || n_layers <= 0 || !ws) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe: NULL layers or workspace");
        return WISP_ERR_INVALID_ARG;
    }
    for (int i = 0; i < n_layers; ++i)
        if (!check_layer(&layers[i], T, err)) return WISP_ERR_INVALID_ARG;
    size_t need = wisp_moe_workspace_bytes(layers, n_layers, T);
    if (ws_bytes < need) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe: workspace %zu bytes < required %zu",
                   ws_bytes, need);
        return WISP_ERR_INVALID_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe: workspace must be 256-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    return WISP_OK;
}

static bool aligned_io(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// prep (quantise x) + router/top-k/plan for one layer.
static WispError block_route(const WispMoeLayer* layer, const float* x, int T, int* topk_idx,
                             float* topk_w, void* workspace, size_t workspace_bytes,
                             cudaStream_t stream, WispErrCtx* err, LayerArgs* a_out, Ws* w_out,
                             bool plan = true) {
    WispError ce = common_checks(layer, 1, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    if (!x || !aligned_io(x)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe block: x NULL or not 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    LayerArgs a = layer_args(layer, T, dev_info().sms);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared != 0, a.si);
    Ws W = make_ws(workspace, lo);
    if (topk_idx) W.topk_idx = topk_idx;
    if (topk_w) W.topk_w = topk_w;
    WB_CUDA_RET(ensure_attrs(a.H), err);
    WB_CUDA_RET(launch_zero_words(static_cast<int*>(workspace),
                                  (int)((lo.counters + kCounters * sizeof(int)) / 4), stream),
                err);
    WB_CUDA_RET(launch_prep_route(a, W, T, (int)P_QUANT, const_cast<float*>(x), 0.f, 0, 0, 1, x,
                                  stream, plan),
                err);
    *a_out = a;
    *w_out = W;
    return WISP_OK;
}

// gate/up + down + combine, on the plan the preceding route left in the workspace.
static WispError block_experts(const LayerArgs& a, const Ws& W, int T, const float* x, float* y,
                               cudaStream_t stream, WispErrCtx* err) {
    WB_CUDA_RET(launch_dense_shared(a, W, T, x, stream), err);
    WB_CUDA_RET(launch_streams(a, W, T, stream), err);
    Ws Wc = W;
    Wc.prev_idx = W.topk_idx;
    Wc.prev_w = W.topk_w;
    WB_CUDA_RET(launch_prep(a, Wc, T, (int)P_COMBINE, const_cast<float*>(x), y, 0.f, a.K,
                            a.has_shared, a.kp, stream),
                err);
    hook_mark(stream);
    return WISP_OK;
}

extern "C" WispError wisp_moe_block_forward(const WispMoeLayer* layer, const float* x, float* y,
                                            int T, int* topk_idx, float* topk_w,
                                            void* workspace, size_t workspace_bytes,
                                            cudaStream_t stream, WispErrCtx* err) {
    if (!y || x == y || !aligned_io(y)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe_block_forward: y NULL, aliased with x, or not 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    LayerArgs a;
    Ws W;
    WispError r = block_route(layer, x, T, topk_idx, topk_w, workspace, workspace_bytes, stream,
                              err, &a, &W);
    if (r != WISP_OK) return r;
    return block_experts(a, W, T, x, y, stream, err);
}

extern "C" WispError wisp_moe_block_route(const WispMoeLayer* layer, const float* x, int T,
                                          int* topk_idx, float* topk_w, void* workspace,
                                          size_t workspace_bytes, cudaStream_t stream,
                                          WispErrCtx* err) {
    // routing only: the expert plan is built by wisp_moe_block_experts once the
    // caller has made the routed experts resident
    LayerArgs a;
    Ws W;
    WispError r = block_route(layer, x, T, topk_idx, topk_w, workspace, workspace_bytes, stream,
                              err, &a, &W, /*plan=*/false);
    if (r == WISP_OK) hook_mark(stream);
    return r;
}

extern "C" WispError wisp_moe_block_experts(const WispMoeLayer* layer, const float* x, float* y,
                                            int T, int* topk_idx, float* topk_w,
                                            void* workspace, size_t workspace_bytes,
                                            cudaStream_t stream, WispErrCtx* err) {
    WispError ce = common_checks(layer, 1, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    if (!x || !y || x == y || !aligned_io(x) || !aligned_io(y)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_block_experts: bad x/y");
        return WISP_ERR_INVALID_ARG;
    }
    LayerArgs a = layer_args(layer, T, dev_info().sms);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared != 0, a.si);
    Ws W = make_ws(workspace, lo);
    if (topk_idx) W.topk_idx = topk_idx;
    if (topk_w) W.topk_w = topk_w;
    WB_CUDA_RET(ensure_attrs(a.H), err);
    WB_CUDA_RET(launch(plan_kernel, dim3(1), dim3(kThreads), router_smem(a.E), stream, a, W, T,
                       plan_tokens(a, T)),
                err);
    return block_experts(a, W, T, x, y, stream, err);
}

extern "C" WispError wisp_moe_stack_forward(const WispMoeLayer* layers, int n_layers, float eps,
                                            float* x, int T, int* topk_idx, float* topk_w,
                                            void* workspace, size_t workspace_bytes,
                                            cudaStream_t stream, WispErrCtx* err) {
    WispError ce = common_checks(layers, n_layers, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    if (!x || !aligned_io(x)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_stack_forward: x NULL or not 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    for (int l = 1; l < n_layers; ++l) {
        if (layers[l].meta.cols[0] != layers[0].meta.cols[0]) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_stack_forward: hidden size differs");
            return WISP_ERR_INVALID_ARG;
        }
    }
    // the workspace layout is sized for the largest layer; all layers share it
    int maxI = 0, maxE = 0, maxK = 0, maxSI = 0;
    bool anysh = false;
    for (int l = 0; l < n_layers; ++l) {
        maxI = std::max(maxI, (int)layers[l].meta.rows[0]);
        maxE = std::max(maxE, layers[l].n_experts);
        maxK = std::max(maxK, layers[l].top_k);
        anysh = anysh || layers[l].shared_blob || layers[l].shared_gate;
        if (layers[l].shared_gate) maxSI = std::max(maxSI, layers[l].shared_inter);
    }
    const int H = (int)layers[0].meta.cols[0];
    WB_CUDA_RET(ensure_attrs(H), err);
    {
        const Layout lo0 = make_layout(T, H, maxI, maxE, maxK, anysh, maxSI);
        WB_CUDA_RET(launch_zero_words(static_cast<int*>(workspace),
                                      (int)((lo0.counters + kCounters * sizeof(int)) / 4), stream),
                    err);
    }
    int prevK = 0, prev_sh = 0, prev_kp = 1;
    for (int l = 0; l < n_layers; ++l) {
        LayerArgs a = layer_args(&layers[l], T, dev_info().sms);
        Layout lo = make_layout(T, H, maxI, maxE, maxK, anysh, maxSI);
        Ws W = make_ws(workspace, lo);
        // the previous layer's routing is read (per token, before this
        // layer's routing of the same token is written) by prep's combine
        Ws Wp = W;
        if (l > 0) {
            Wp.prev_idx = topk_idx ? topk_idx + (size_t)(l - 1) * T * prevK : W.topk_idx;
            Wp.prev_w = topk_w ? topk_w + (size_t)(l - 1) * T * prevK : W.topk_w;
        }
        if (topk_idx) W.topk_idx = Wp.topk_idx = topk_idx + (size_t)l * T * a.K;
        if (topk_w) W.topk_w = Wp.topk_w = topk_w + (size_t)l * T * a.K;
        const int flags = (l > 0 ? (P_COMBINE | P_RESID) : 0) | P_NORM | P_QUANT;
        WB_CUDA_RET(launch_prep_route(a, Wp, T, flags, x, eps, prevK, prev_sh, prev_kp, W.xn,
                                      stream),
                    err);
        WB_CUDA_RET(launch_dense_shared(a, W, T, W.xn, stream), err);
        WB_CUDA_RET(launch_streams(a, W, T, stream), err);
        prevK = a.K;
        prev_sh = a.has_shared;
        prev_kp = a.kp;
        if (l == n_layers - 1) {
            Ws Wf = W;
            Wf.prev_idx = W.topk_idx;
            Wf.prev_w = W.topk_w;
            WB_CUDA_RET(launch_prep(a, Wf, T, (int)(P_COMBINE | P_RESID), x, nullptr, eps, prevK,
                                    prev_sh, prev_kp, stream),
                        err);
        }
    }
    hook_mark(stream);
    return WISP_OK;
}

// ------------------------------------------------------------------------
// Expert-parallel building blocks: experts on a supplied routing, and the
// weighted combine of rows returned by the expert owners.
// ------------------------------------------------------------------------
extern "C" WispError wisp_moe_experts_routed(const WispMoeLayer* layer, const float* x,
                                             float* y, int T, const int* topk_idx,
                                             const float* topk_w, void* workspace,
                                             size_t workspace_bytes, cudaStream_t stream,
                                             WispErrCtx* err) {
    if (!layer || !x || !y || x == y || !topk_idx || !topk_w || !aligned_io(x) ||
        !aligned_io(y)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_experts_routed: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    // the router is not used: check the layer with a stand-in router pointer
    WispMoeLayer chk = *layer;
    if (!chk.router_w) chk.router_w = reinterpret_cast<const wisp_half*>(x);
    WispError ce = common_checks(&chk, 1, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    LayerArgs a = layer_args(layer, T, dev_info().sms);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared != 0, a.si);
    Ws W = make_ws(workspace, lo);
    W.topk_idx = const_cast<int*>(topk_idx);
    W.topk_w = const_cast<float*>(topk_w);
    WB_CUDA_RET(ensure_attrs(a.H), err);
    WB_CUDA_RET(launch_zero_words(static_cast<int*>(workspace),
                                  (int)((lo.counters + kCounters * sizeof(int)) / 4), stream),
                err);
    WB_CUDA_RET(launch_prep(a, W, T, (int)P_QUANT, const_cast<float*>(x), nullptr, 0.f, 0, 0, 1,
                            stream),
                err);
    WB_CUDA_RET(launch(plan_kernel, dim3(1), dim3(kThreads), router_smem(a.E), stream, a, W, T,
                       plan_tokens(a, T)),
                err);
    return block_experts(a, W, T, x, y, stream, err);
}

extern "C" WispError wisp_moe_route(const WispMoeLayer* layer, const float* x, int T,
                                    int* topk_idx, float* topk_w, void* workspace,
                                    size_t workspace_bytes, cudaStream_t stream,
                                    WispErrCtx* err) {
    if (!layer || !x || !topk_idx || !topk_w || !aligned_io(x)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_route: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    // the experts are not used: check the layer with a stand-in table pointer
    WispMoeLayer chk = *layer;
    if (!chk.expert_blobs) chk.expert_blobs = reinterpret_cast<const void* const*>(x);
    WispError ce = common_checks(&chk, 1, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    LayerArgs a = layer_args(&chk, T, dev_info().sms);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared != 0, a.si);
    Ws W = make_ws(workspace, lo);
    W.topk_idx = topk_idx;
    W.topk_w = topk_w;
    WB_CUDA_RET(ensure_attrs(a.H), err);
    WB_CUDA_RET(launch_zero_words(static_cast<int*>(workspace),
                                  (int)((lo.counters + kCounters * sizeof(int)) / 4), stream),
                err);
    const int cs = prep_cluster(a.H, a.gs);
    const bool fused = route_in_prep(a, T);
    hook_mark(stream);
    WB_CUDA_RET(launch_pdl_cluster(prep_kernel, dim3(T * cs), dim3(kPrepThreads),
                                   prep_smem_bytes(a.H, cs, a.E), stream, cs, a, W, T,
                                   (int)(P_QUANT | (fused ? P_ROUTE : 0)),
                                   const_cast<float*>(x), (float*)nullptr, 0.f, 0, 0, 1, 0),
                err);
    if (!fused) {
        const int nsl = (a.H + kSlice - 1) / kSlice;
        const int blocks = (a.E * nsl + kWarps - 1) / kWarps;
        WB_CUDA_RET(launch(router_kernel, dim3(blocks), dim3(kThreads), router_smem(a.E), stream,
                           a, W, T, 0, x, nsl),
                    err);
    }
    return WISP_OK;
}

extern "C" WispError wisp_moe_ep_combine(float* y, const float* rows, const int* row_idx,
                                         const float* weights, int T, int K, int H,
                                         cudaStream_t stream, WispErrCtx* err) {
    if (!y || !row_idx || !weights || T <= 0 || K <= 0 || H <= 0 || H % 4 || !aligned_io(y) ||
        (rows && !aligned_io(rows))) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_ep_combine: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    WB_CUDA_RET(launch(ep_combine_kernel, dim3(T), dim3(kPrepThreads), 0, stream, y, rows,
                       row_idx, weights, T, K, H),
                err);
    return WISP_OK;
}

// ------------------------------------------------------------------------
// Fixed-scratch variant of wisp_moe_block_forward.
//
// Some callers cannot hand the library a device workspace: a host that binds
// this library through a plain C FFI and owns no device allocator, or a
// serving loop that reserved all device memory before it started and may not
// allocate per step (a cudaMalloc there can fail under memory pressure in the
// middle of a decode, and it synchronises the device).  For them the block
// runs in a file-scope device array instead: no cudaMalloc, cudaFree or
// allocating library routine is called.
//
// Limits: the array holds kStaticScratchBytes (8 MiB), enough for a
// Mixtral-shaped layer (hidden 4096, intermediate 14336, top-2) up to T = 16;
// larger requests are rejected with WISP_ERR_INVALID_ARG before any GPU work.
// Every call on a device shares the one array, so two calls whose kernels
// overlap on the GPU (different streams, or different host threads without
// ordering) race and corrupt each other's results.  Each call clears what
// must start at zero (the status word and the kernels' counters) with a
// one-CTA zeroing kernel on the call's stream, as wisp_moe_block_forward does
// for a caller's workspace.
// ------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_block_scratch[kStaticScratchBytes];

// Device address of the array on the current device, looked up once per device
// (the first call on a device does this look-up).
static void* block_scratch(WispErrCtx* err) {
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess || dev < 0 || dev >= 64) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "moe_block_forward_static: no usable device (%s)",
                   cudaGetErrorString(ce));
        return nullptr;
    }
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        ce = cudaGetSymbolAddress(&p, g_block_scratch);
        if (ce != cudaSuccess || !p) {
            WB_SET_ERR(err, WISP_ERR_CUDA,
                       "moe_block_forward_static: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(ce));
            return nullptr;
        }
        addr[dev] = p;
    }
    return addr[dev];
}

extern "C" WispError wisp_moe_block_forward_static(const WispMoeLayer* layer, const float* x,
                                                   float* y, int T, int* topk_idx,
                                                   float* topk_w, cudaStream_t stream,
                                                   WispErrCtx* err) {
    if (!layer) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe_block_forward_static: NULL layer");
        return WISP_ERR_INVALID_ARG;
    }
    if (!check_layer(layer, T, err)) return WISP_ERR_INVALID_ARG;
    const size_t need = wisp_moe_workspace_bytes(layer, 1, T);
    if (need > kStaticScratchBytes) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe_block_forward_static: T=%d needs %zu bytes of scratch but the fixed "
                   "scratch holds %zu; use wisp_moe_block_forward with a workspace",
                   T, need, kStaticScratchBytes);
        return WISP_ERR_INVALID_ARG;
    }
    void* ws = block_scratch(err);
    if (!ws) return WISP_ERR_CUDA;
    return wisp_moe_block_forward(layer, x, y, T, topk_idx, topk_w, ws, kStaticScratchBytes,
                                  stream, err);
}

// Status word of the last wisp_moe_block_forward_static call on the current
// device (the first int of the fixed array; bits as wisp_moe_status).  A caller
// of the static entry has no workspace pointer to hand wisp_moe_status, so this
// reads it through the array's cached address.  Synchronises `stream`; -1 when
// the read fails.
extern "C" int wisp_moe_block_static_status(cudaStream_t stream) {
    WispErrCtx err{};
    void* ws = block_scratch(&err);
    if (!ws) return -1;
    return wisp_moe_status(ws, stream);
}
