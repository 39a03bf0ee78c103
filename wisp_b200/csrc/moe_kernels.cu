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
// and zero z per group of 64 row-major elements, weight = (c-8)*s + z.
//
// Launch sequence per layer (each launch uses programmatic dependent launch,
// so one kernel's prologue overlaps the previous one's tail):
//   prep_kernel     one CTA per token: [combine previous layer + residual]
//                   [+ RMSNorm] + quantise the activations (see below)
//   router_kernel   logits, then the last CTA of each token does softmax/top-k
//                   and the last token builds the expert-tile plan
//   gateup_kernel   persistent, one warp per (tile, row) task taken from an
//                   atomic counter: h = silu(G.x) * (U.x); the warp finishing
//                   the last row of a 32-row chunk of h quantises that chunk
//   down_kernel     persistent, one warp per (tile, row, K-half):
//                   ypart[half][assignment][row] = D.h over that half
//   prep_kernel     (next layer or final): y = sum_j w_j (ypart0 + ypart1)
//
// Arithmetic of the int4 dot products.  Activations are split per 32-element
// chunk into two int8 digits, x ~= k*a + (k/254)*b with |a|,|b| <= 127 and
// k = max|x|/127 (residual error <= max|x| * 1.6e-5).  A 16-byte load of
// packed weights is 32 codes; two LOP3s and a shift split them into the even
// and odd codes as bytes, and four dp4a per 8 codes give the exact integer
// sums A = sum c*a and B = sum c*b.  The chunk's contribution to a row is
//   s * (k/254) * (254*A + B) + (z - 8*s) * sum(x~)
// -- exact integer accumulation, 0.9 instructions per weight element, so the
// kernels stay bound by HBM bandwidth rather than by issue.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "internal.h"

namespace wb {
namespace {

constexpr int kChunk = 32;      // elements per 16-byte packed load
constexpr int kMT = 4;          // max tokens per expert tile
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxPlanAssign = 4096;  // T*k limit of the device plan builder

enum { C_GU_TASK = 0, C_DN_TASK = 1, C_TOK_DONE = 2, C_NTILES = 3, C_COUNT = 8 };
enum { ST_ALIGN = 1, ST_EXPERT = 2, ST_PLAN = 4 };

struct Tile {
    int expert;  // 0..E-1, or E for the shared expert
    int m;       // tokens in the tile (1..kMT)
    int tok[kMT];
    int asg[kMT];  // assignment ids: t*K + j, or T*K + t for the shared expert
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
    int H, I, E, K, gs, has_shared;
};

struct Ws {
    int* status;
    int* counters;
    int* tok_cnt;
    float* logits;
    int* topk_idx;  // routing of the layer being run [T, K]
    float* topk_w;
    int* prev_idx;  // routing of the previous layer (combine in prep)
    float* prev_w;
    Tile* tiles;
    float* xn;
    uint4* xq;  // [T][H/32][4]
    float2* xqp;
    float* h;   // [A][I]
    uint4* hq;  // [A][I/32][4]
    float2* hqp;
    int* hcnt;      // [A][I/32]
    float* ypart;   // [2][A][H]
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

// Streaming 16-byte load of weights: read-only path, no L1 allocation, and a
// 256-byte L2 fetch granule so neighbouring lanes' sectors arrive together.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile(
        "ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_half(const __half* p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Quantise one 32-element chunk held one element per lane into the two-digit
// int8 form and store it: 16 words + (k/254, sum of the quantised values).
// Word layout (matches the nibble split of a 16-byte weight load): for weight
// word w (elements 8w..8w+7), word [w] holds a of elements 8w,8w+2,8w+4,8w+6,
// word [4+w] holds a of the odd ones, [8+w] / [12+w] the same for b.
__device__ __forceinline__ void quantize_chunk_warp(float v, uint4* dst_q,
                                                    float2* dst_p) {
    const int lane = threadIdx.x & 31;
    float mx = warp_max(fabsf(v));
    float k = mx * (1.0f / 127.0f);
    float inv = mx > 0.f ? 127.0f / mx : 0.f;
    int a = __float2int_rn(v * inv);
    a = max(-127, min(127, a));
    float r = fmaf(-k, (float)a, v);
    int b = __float2int_rn(r * (inv * 254.0f));
    b = max(-127, min(127, b));
    float k2 = k * (1.0f / 254.0f);
    int sa = warp_sum_i(a), sb = warp_sum_i(b);
    // gather the 16 words: lane L < 16 builds word L
    const int kind = (lane >> 3) & 1;  // 0: a, 1: b
    const int odd = (lane >> 2) & 1;
    const int w = lane & 3;
    uint32_t word = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        int src = 8 * w + 2 * p + odd;
        int va = __shfl_sync(kFull, a, src);
        int vb = __shfl_sync(kFull, b, src);
        word |= (uint32_t)((kind ? vb : va) & 0xff) << (8 * p);
    }
    if (lane < 16) reinterpret_cast<uint32_t*>(dst_q)[lane] = word;
    if (lane == 0) *dst_p = make_float2(k2, fmaf(k, (float)sa, k2 * (float)sb));
}

struct XChunk {
    uint4 q[4];
    float k2, xs;
};

__device__ __forceinline__ void load_xchunk(XChunk& x, const uint4* q,
                                            const float2* p) {
    x.q[0] = q[0];
    x.q[1] = q[1];
    x.q[2] = q[2];
    x.q[3] = q[3];
    float2 pp = *p;
    x.k2 = pp.x;
    x.xs = pp.y;
}

struct Nib {
    int lo[4], hi[4];
};
__device__ __forceinline__ void split_nibbles(const uint4& w, Nib& n) {
    const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        n.lo[i] = (int)(v[i] & 0x0F0F0F0Fu);
        n.hi[i] = (int)((v[i] >> 4) & 0x0F0F0F0Fu);
    }
}
__device__ __forceinline__ float chunk_dot(const Nib& n, const XChunk& x,
                                           float s, float z) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(x.q);
    int A = 0, B = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        A = __dp4a(n.lo[i], (int)q[i], A);
        A = __dp4a(n.hi[i], (int)q[4 + i], A);
        B = __dp4a(n.lo[i], (int)q[8 + i], B);
        B = __dp4a(n.hi[i], (int)q[12 + i], B);
    }
    int C = A * 254 + B;
    return fmaf(s * x.k2, (float)C, fmaf(-8.0f, s, z) * x.xs);
}

__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

struct MatPtr {
    const uint8_t* packed;
    const __half* scales;
    const __half* zeros;
};
__device__ __forceinline__ MatPtr mat_ptr(const void* blob, const MatOff& o) {
    const uint8_t* b = static_cast<const uint8_t*>(blob);
    return {b + o.packed, reinterpret_cast<const __half*>(b + o.scales),
            reinterpret_cast<const __half*>(b + o.zeros)};
}

// ------------------------------------------------------------------------
// prep: combine + residual + RMSNorm + activation quantisation (per token)
// ------------------------------------------------------------------------
enum { P_COMBINE = 1, P_RESID = 2, P_NORM = 4, P_QUANT = 8 };

__global__ void __launch_bounds__(kThreads)
prep_kernel(LayerArgs L, Ws W, int T, int flags, float* x, float* y,
            float eps, int prevK, int prev_shared) {
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.x;
    const int H = L.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float red[kWarps];
    __shared__ float s_scale;
    extern __shared__ float sx[];  // [H] working copy of this token
    float* xt = x + (size_t)t * H;

    if (tid == 0) W.tok_cnt[t] = 0;
    if (t == 0 && tid == 0) W.counters[C_TOK_DONE] = 0;

    // 1. combine the previous block's expert outputs (reference order: shared
    //    expert first with weight 1, then routed experts in top-k order).
    for (int i = tid; i < H; i += kThreads) {
        float v = xt[i];
        if (flags & P_COMBINE) {
            float acc = 0.f;
            const size_t half_stride = (size_t)W.A * H;
            if (prev_shared) {
                size_t a = (size_t)T * prevK + t;
                acc += W.ypart[a * H + i] + W.ypart[half_stride + a * H + i];
            }
            for (int j = 0; j < prevK; ++j) {
                int e = W.prev_idx[t * prevK + j];
                if (e < 0) continue;
                size_t a = (size_t)t * prevK + j;
                float yj = W.ypart[a * H + i] + W.ypart[half_stride + a * H + i];
                acc += W.prev_w[t * prevK + j] * yj;
            }
            v = (flags & P_RESID) ? v + acc : acc;
            if (y) y[(size_t)t * H + i] = v;
            if (flags & P_RESID) xt[i] = v;
        }
        sx[i] = v;
    }
    if (!(flags & (P_NORM | P_QUANT))) return;
    __syncthreads();

    // 2. RMSNorm: y = x / sqrt(mean(x^2) + eps) * w
    if (flags & P_NORM) {
        float ss = 0.f;
        for (int i = tid; i < H; i += kThreads) ss += sx[i] * sx[i];
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = lane < kWarps ? red[lane] : 0.f;
            v = warp_sum(v);
            if (lane == 0) s_scale = 1.0f / sqrtf(v / (float)H + eps);
        }
        __syncthreads();
        const float sc = s_scale;
        for (int i = tid; i < H; i += kThreads) {
            float v = sx[i] * sc;
            if (L.norm_w) v *= __half2float(L.norm_w[i]);
            sx[i] = v;
            W.xn[(size_t)t * H + i] = v;
        }
        __syncthreads();
    }

    // 3. quantise the router/expert input, one warp per 32-element chunk
    if (flags & P_QUANT) {
        const int nch = H / kChunk;
        for (int c = warp; c < nch; c += kWarps) {
            float v = sx[c * kChunk + lane];
            size_t o = (size_t)t * nch + c;
            quantize_chunk_warp(v, W.xq + o * 4, W.xqp + o);
        }
    }
}

// ------------------------------------------------------------------------
// router: logits, then softmax + top-k, then the expert-tile plan
// ------------------------------------------------------------------------
__device__ void topk_token(const LayerArgs& L, const Ws& W, int t, int K,
                           float* sp, int* staken) {
    // one warp; sp: [E] shared scratch
    const int lane = threadIdx.x & 31;
    const int E = L.E;
    float mx = -1e30f;
    for (int e = lane; e < E; e += 32) {
        float v = __ldcg(W.logits + (size_t)t * E + e);
        sp[e] = v;
        staken[e] = 0;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    float den = 0.f;
    for (int e = lane; e < E; e += 32) {
        float v = expf(sp[e] - mx);
        sp[e] = v;
        den += v;
    }
    den = warp_sum(den);
    for (int e = lane; e < E; e += 32) sp[e] = sp[e] / den;
    __syncwarp();
    float wsum = 0.f;
    float wsel[64];
    int isel[64];
    for (int j = 0; j < K; ++j) {
        float bv = -1.f;
        int be = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            float v = sp[e];
            if (!staken[e] && v > bv) { bv = v; be = e; }
        }
        // warp argmax: larger value wins, equal values -> lower index
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(kFull, bv, o);
            int oe = __shfl_xor_sync(kFull, be, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
        }
        if (bv < 0.f) be = -1;  // fewer candidates than k (E < K)
        if (lane == 0 && be >= 0) staken[be] = 1;
        __syncwarp();
        wsel[j] = bv;
        isel[j] = be;
        if (be >= 0) wsum += bv;
    }
    if (lane == 0) {
        for (int j = 0; j < K; ++j) {
            float wj = isel[j] >= 0 ? wsel[j] : 0.f;
            if (wsum > 0.f) wj = wj / wsum;
            W.topk_idx[t * K + j] = isel[j];
            W.topk_w[t * K + j] = wj;
        }
    }
}

__device__ void build_plan(const LayerArgs& L, const Ws& W, int T, int mt,
                           int* s_idx, int* s_cnt) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = L.K, E = L.E, NA = T * K;
    for (int a = tid; a < NA; a += kThreads) s_idx[a] = __ldcg(W.topk_idx + a);
    __syncthreads();
    // tiles per expert; experts e = tid, tid + 256, ... (E <= 1024)
    int my_tiles[4] = {0, 0, 0, 0};
    int local = 0;
    for (int r = 0; r < 4; ++r) {
        int e = tid + r * kThreads;
        if (e < E) {
            int cnt = 0;
            for (int a = 0; a < NA; ++a) cnt += (s_idx[a] == e);
            my_tiles[r] = (cnt + mt - 1) / mt;
            local += my_tiles[r];
        }
    }
    // block exclusive scan of `local` (experts ordered by thread, then round:
    // tile order does not affect any result, each row is per-token).
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_cnt[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int v = lane < kWarps ? s_cnt[lane] : 0;
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int u = __shfl_up_sync(kFull, inc, o);
            if (lane >= o) inc += u;
        }
        if (lane < kWarps) s_cnt[kWarps + lane] = inc - v;  // exclusive
        if (lane == kWarps - 1) s_cnt[2 * kWarps] = inc;      // routed total
    }
    __syncthreads();
    int base = s_cnt[kWarps + warp] + incl - local;
    const int routed_tiles = s_cnt[2 * kWarps];
    const int shared_tiles = L.has_shared ? (T + mt - 1) / mt : 0;
    const int total = routed_tiles + shared_tiles;
    if (total > W.max_tiles) {
        if (tid == 0) {
            atomicOr(W.status, ST_PLAN);
            W.counters[C_NTILES] = 0;
        }
        return;
    }
    for (int r = 0; r < 4; ++r) {
        int e = tid + r * kThreads;
        if (e >= E || my_tiles[r] == 0) continue;
        Tile tl;
        tl.expert = e;
        tl.m = 0;
        int ti = base;
        for (int a = 0; a < NA; ++a) {
            if (s_idx[a] != e) continue;
            tl.tok[tl.m] = a / K;
            tl.asg[tl.m] = a;
            if (++tl.m == mt) {
                W.tiles[ti++] = tl;
                tl.m = 0;
            }
        }
        if (tl.m) W.tiles[ti++] = tl;
        base = ti;
    }
    for (int s = tid; s < shared_tiles; s += kThreads) {
        Tile tl;
        tl.expert = E;
        tl.m = 0;
        for (int t = s * mt; t < T && tl.m < mt; ++t) {
            tl.tok[tl.m] = t;
            tl.asg[tl.m] = T * K + t;
            tl.m++;
        }
        W.tiles[routed_tiles + s] = tl;
    }
    const int nchunk_h = L.I / kChunk;
    for (int i = tid; i < W.A * nchunk_h; i += kThreads) W.hcnt[i] = 0;
    if (tid == 0) {
        W.counters[C_NTILES] = total;
        W.counters[C_GU_TASK] = 0;
        W.counters[C_DN_TASK] = 0;
    }
}

__global__ void __launch_bounds__(kThreads)
router_kernel(LayerArgs L, Ws W, int T, int mt, const float* xin) {
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int E = L.E, H = L.H;
    __shared__ int s_last;
    extern __shared__ int smem[];

    const int e = blockIdx.x * kWarps + warp;
    if (e < E) {
        const __half* row = L.router_w + (size_t)e * H;
        const float* xr = xin + (size_t)t * H;
        float acc = 0.f;
        for (int c = lane * 8; c < H; c += 32 * 8) {
            uint4 wv = *reinterpret_cast<const uint4*>(row + c);
            const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
            float4 x0 = *reinterpret_cast<const float4*>(xr + c);
            float4 x1 = *reinterpret_cast<const float4*>(xr + c + 4);
            float2 f;
            f = __half22float2(w2[0]);
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
        acc = warp_sum(acc);
        if (lane == 0) {
            float b = L.router_bias ? __half2float(L.router_bias[e]) : 0.f;
            W.logits[(size_t)t * E + e] = acc + b;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(W.tok_cnt + t, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (warp == 0) {
        float* sp = reinterpret_cast<float*>(smem);
        int* staken = smem + E;
        topk_token(L, W, t, L.K, sp, staken);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(W.counters + C_TOK_DONE, 1) == T - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    build_plan(L, W, T, mt, smem, smem + kMaxPlanAssign);
}

// ------------------------------------------------------------------------
// gate/up + SwiGLU
// ------------------------------------------------------------------------
template <int M>
__device__ __forceinline__ void gateup_row(const LayerArgs& L, const Ws& W,
                                           const Tile& tl, MatPtr g, MatPtr u,
                                           int row) {
    const int lane = threadIdx.x & 31;
    const int H = L.H, I = L.I, gs = L.gs;
    const int nch = H / kChunk;
    const uint8_t* gp = g.packed + (size_t)row * (H / 2);
    const uint8_t* up = u.packed + (size_t)row * (H / 2);
    const size_t srow = (size_t)row * (H / gs);
    float ag[M], au[M];
#pragma unroll
    for (int j = 0; j < M; ++j) ag[j] = au[j] = 0.f;

#pragma unroll 2
    for (int c = lane; c < nch; c += 32) {
        uint4 wg = ld_stream(gp + (size_t)c * 16);
        uint4 wu = ld_stream(up + (size_t)c * 16);
        const size_t gi = srow + (size_t)(c * kChunk) / gs;
        float sg = ld_half(g.scales + gi), zg = ld_half(g.zeros + gi);
        float su = ld_half(u.scales + gi), zu = ld_half(u.zeros + gi);
        Nib ng, nu;
        split_nibbles(wg, ng);
        split_nibbles(wu, nu);
#pragma unroll
        for (int j = 0; j < M; ++j) {
            XChunk x;
            size_t o = (size_t)tl.tok[j] * nch + c;
            load_xchunk(x, W.xq + o * 4, W.xqp + o);
            ag[j] += chunk_dot(ng, x, sg, zg);
            au[j] += chunk_dot(nu, x, su, zu);
        }
    }
    float hv = 0.f;
    int asg = -1;
#pragma unroll
    for (int j = 0; j < M; ++j) {
        float gv = warp_sum(ag[j]);
        float uv = warp_sum(au[j]);
        if (lane == j) {
            hv = gv / (1.0f + expf(-gv)) * uv;
            asg = tl.asg[j];
        }
    }
    const int nchunk_h = I / kChunk;
    bool done = false;
    if (lane < M) {
        W.h[(size_t)asg * I + row] = hv;
        __threadfence();
        int old = atomicAdd(W.hcnt + (size_t)asg * nchunk_h + row / kChunk, 1);
        done = (old == kChunk - 1);
    }
    unsigned mask = __ballot_sync(kFull, done);
    while (mask) {
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        const int a = __shfl_sync(kFull, asg, src);
        __threadfence();
        const int hc = row / kChunk;
        float v = __ldcg(W.h + (size_t)a * I + hc * kChunk + lane);
        size_t o = (size_t)a * nchunk_h + hc;
        quantize_chunk_warp(v, W.hq + o * 4, W.hqp + o);
    }
}

__device__ __forceinline__ bool tile_mats(const LayerArgs& L, const Ws& W,
                                          const Tile& tl, int m0, int m1,
                                          MatPtr& a, MatPtr& b) {
    const void* blob;
    const MatOff* off;
    if (tl.expert == L.E) {
        blob = L.shared_blob;
        off = L.smat;
    } else if (tl.expert >= 0 && tl.expert < L.E) {
        blob = L.blobs[tl.expert];
        off = L.mat;
    } else {
        if ((threadIdx.x & 31) == 0) atomicOr(W.status, ST_EXPERT);
        return false;
    }
    a = mat_ptr(blob, off[m0]);
    bool ok = aligned16(a.packed) && aligned16(a.scales) && aligned16(a.zeros);
    if (m1 >= 0) {
        b = mat_ptr(blob, off[m1]);
        ok = ok && aligned16(b.packed);
    }
    if (!ok && (threadIdx.x & 31) == 0) atomicOr(W.status, ST_ALIGN);
    return ok;
}

__device__ __forceinline__ void load_tile(const Tile* src, Tile& tl) {
    const int* s = reinterpret_cast<const int*>(src);
    int* d = reinterpret_cast<int*>(&tl);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(Tile) / 4); ++i) d[i] = __ldcg(s + i);
}

template <int MTMAX>
__global__ void __launch_bounds__(kThreads)
gateup_kernel(LayerArgs L, Ws W) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int I = L.I;
    const long long total = (long long)__ldcg(W.counters + C_NTILES) * I;
    int task = 0;
    if (lane == 0) task = atomicAdd(W.counters + C_GU_TASK, 1);
    task = __shfl_sync(kFull, task, 0);
    int cur = -1;
    bool ok = false;
    Tile tl;
    MatPtr g, u;
    while (task < total) {
        int next = 0;
        if (lane == 0) next = atomicAdd(W.counters + C_GU_TASK, 1);
        const int ti = task / I, row = task - ti * I;
        if (ti != cur) {
            load_tile(W.tiles + ti, tl);
            ok = tile_mats(L, W, tl, 0, 1, g, u) && aligned16(u.scales) &&
                 aligned16(u.zeros);
            cur = ti;
        }
        if (ok) {
            if (MTMAX == 1 || tl.m == 1) {
                gateup_row<1>(L, W, tl, g, u, row);
            } else if (MTMAX > 1) {
                switch (tl.m) {
                    case 2: gateup_row<2>(L, W, tl, g, u, row); break;
                    case 3: gateup_row<3>(L, W, tl, g, u, row); break;
                    default: gateup_row<4>(L, W, tl, g, u, row); break;
                }
            }
        }
        task = __shfl_sync(kFull, next, 0);
    }
}

// ------------------------------------------------------------------------
// down projection (two K-halves per row, written separately: deterministic)
// ------------------------------------------------------------------------
template <int M>
__device__ __forceinline__ void down_row(const LayerArgs& L, const Ws& W,
                                         const Tile& tl, MatPtr d, int row,
                                         int half) {
    const int lane = threadIdx.x & 31;
    const int H = L.H, I = L.I, gs = L.gs;
    const int nch = I / kChunk;
    const int per = (nch + 1) / 2;
    const int c0 = half * per, c1 = min(nch, c0 + per);
    const uint8_t* dp = d.packed + (size_t)row * (I / 2);
    const size_t srow = (size_t)row * (I / gs);
    float acc[M];
#pragma unroll
    for (int j = 0; j < M; ++j) acc[j] = 0.f;
#pragma unroll 2
    for (int c = c0 + lane; c < c1; c += 32) {
        uint4 wd = ld_stream(dp + (size_t)c * 16);
        const size_t gi = srow + (size_t)(c * kChunk) / gs;
        float s = ld_half(d.scales + gi), z = ld_half(d.zeros + gi);
        Nib nd;
        split_nibbles(wd, nd);
#pragma unroll
        for (int j = 0; j < M; ++j) {
            XChunk x;
            size_t o = (size_t)tl.asg[j] * nch + c;
            load_xchunk(x, W.hq + o * 4, W.hqp + o);
            acc[j] += chunk_dot(nd, x, s, z);
        }
    }
#pragma unroll
    for (int j = 0; j < M; ++j) {
        float v = warp_sum(acc[j]);
        if (lane == j)
            W.ypart[((size_t)half * W.A + tl.asg[j]) * H + row] = v;
    }
}

template <int MTMAX>
__global__ void __launch_bounds__(kThreads)
down_kernel(LayerArgs L, Ws W) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int H = L.H;
    const long long total = (long long)__ldcg(W.counters + C_NTILES) * H * 2;
    int task = 0;
    if (lane == 0) task = atomicAdd(W.counters + C_DN_TASK, 1);
    task = __shfl_sync(kFull, task, 0);
    int cur = -1;
    bool ok = false;
    Tile tl;
    MatPtr d, unused;
    while (task < total) {
        int next = 0;
        if (lane == 0) next = atomicAdd(W.counters + C_DN_TASK, 1);
        const int ti = task / (2 * H);
        const int rem = task - ti * 2 * H;
        const int row = rem >> 1, half = rem & 1;
        if (ti != cur) {
            load_tile(W.tiles + ti, tl);
            ok = tile_mats(L, W, tl, 2, -1, d, unused);
            cur = ti;
        }
        if (ok) {
            if (MTMAX == 1 || tl.m == 1) {
                down_row<1>(L, W, tl, d, row, half);
            } else if (MTMAX > 1) {
                switch (tl.m) {
                    case 2: down_row<2>(L, W, tl, d, row, half); break;
                    case 3: down_row<3>(L, W, tl, d, row, half); break;
                    default: down_row<4>(L, W, tl, d, row, half); break;
                }
            }
        }
        task = __shfl_sync(kFull, next, 0);
    }
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------
struct Layout {
    size_t status, counters, tok_cnt, logits, topk_idx, topk_w, pidx, pw, tiles,
        xn, xq, xqp, h, hq, hqp, hcnt, ypart, total;
    int A, max_tiles;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Layout make_layout(int T, int H, int I, int E, int K, bool shared) {
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
    l.counters = take(C_COUNT * sizeof(int));
    l.tok_cnt = take((size_t)T * sizeof(int));
    l.logits = take((size_t)T * E * sizeof(float));
    l.topk_idx = take((size_t)T * K * sizeof(int));
    l.topk_w = take((size_t)T * K * sizeof(float));
    l.pidx = take((size_t)T * K * sizeof(int));
    l.pw = take((size_t)T * K * sizeof(float));
    l.tiles = take((size_t)l.max_tiles * sizeof(Tile));
    l.xn = take((size_t)T * H * sizeof(float));
    l.xq = take((size_t)T * (H / kChunk) * 64);
    l.xqp = take((size_t)T * (H / kChunk) * sizeof(float2));
    l.h = take((size_t)l.A * I * sizeof(float));
    l.hq = take((size_t)l.A * (I / kChunk) * 64);
    l.hqp = take((size_t)l.A * (I / kChunk) * sizeof(float2));
    l.hcnt = take((size_t)l.A * (I / kChunk) * sizeof(int));
    l.ypart = take((size_t)2 * l.A * H * sizeof(float));
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
    w.xqp = reinterpret_cast<float2*>(b + l.xqp);
    w.h = reinterpret_cast<float*>(b + l.h);
    w.hq = reinterpret_cast<uint4*>(b + l.hq);
    w.hqp = reinterpret_cast<float2*>(b + l.hqp);
    w.hcnt = reinterpret_cast<int*>(b + l.hcnt);
    w.ypart = reinterpret_cast<float*>(b + l.ypart);
    w.A = l.A;
    w.max_tiles = l.max_tiles;
    return w;
}

MatOff mat_off(const WispExpertMeta& m, int i) {
    return {(unsigned long long)m.packed_off[i], (unsigned long long)m.scales_off[i],
            (unsigned long long)m.zeros_off[i]};
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
    if (H % kChunk || I % kChunk || gs % kChunk || H % gs || I % gs || H % 8 || I % 8) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: unsupported shape H=%d I=%d group_size=%d (need multiples "
                   "of 32, group_size | H and I, group_size %% 32 == 0)",
                   H, I, gs);
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
    if (ly->shared_blob) {
        const WispExpertMeta& s = ly->shared_meta;
        if (!s.valid || s.cols[0] != (uint32_t)H || s.rows[0] != (uint32_t)I ||
            s.group_size != (uint32_t)gs) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "moe layer: shared expert must match the routed experts' shape "
                       "and group size");
            return false;
        }
    }
    return true;
}

LayerArgs layer_args(const WispMoeLayer* ly) {
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
    a.has_shared = ly->shared_blob != nullptr;
    return a;
}

struct DevInfo {
    int sms = 0, gu_blocks[2] = {0, 0}, dn_blocks[2] = {0, 0};
};

DevInfo dev_info() {
    static std::mutex mu;
    static DevInfo cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = cache[dev & 63];
    if (!d.sms) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        int b = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gateup_kernel<1>, kThreads, 0);
        d.gu_blocks[0] = std::max(1, b) * d.sms;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, gateup_kernel<kMT>, kThreads, 0);
        d.gu_blocks[1] = std::max(1, b) * d.sms;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, down_kernel<1>, kThreads, 0);
        d.dn_blocks[0] = std::max(1, b) * d.sms;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, down_kernel<kMT>, kThreads, 0);
        d.dn_blocks[1] = std::max(1, b) * d.sms;
    }
    return d;
}

size_t prep_smem(int H) { return (size_t)H * sizeof(float); }
size_t router_smem() { return (size_t)(kMaxPlanAssign + 2 * 1024 + 64) * sizeof(int); }

cudaError_t ensure_attrs(int H) {
    static std::mutex mu;
    static int done_H[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (done_H[dev & 63] >= H) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)prep_smem(std::max(H, 8192)));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)router_smem());
    if (e != cudaSuccess) return e;
    done_H[dev & 63] = std::max(H, 8192);
    return cudaSuccess;
}

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

// Run one layer's router + expert kernels.  The layer's input is already
// quantised in W.xq (and xin holds the router input).
cudaError_t run_layer_experts(const LayerArgs& a, const Ws& W, int T, const float* xin,
                              cudaStream_t s) {
    const DevInfo d = dev_info();
    const int mt = T == 1 ? 1 : kMT;
    const int neb = (a.E + kWarps - 1) / kWarps;
    cudaError_t e = launch(router_kernel, dim3(neb, T), dim3(kThreads), router_smem(), s, a,
                               W, T, mt, xin);
    if (e != cudaSuccess) return e;
    if (mt == 1) {
        e = launch(gateup_kernel<1>, dim3(d.gu_blocks[0]), dim3(kThreads), 0, s, a, W);
        if (e != cudaSuccess) return e;
        return launch(down_kernel<1>, dim3(d.dn_blocks[0]), dim3(kThreads), 0, s, a, W);
    }
    e = launch(gateup_kernel<kMT>, dim3(d.gu_blocks[1]), dim3(kThreads), 0, s, a, W);
    if (e != cudaSuccess) return e;
    return launch(down_kernel<kMT>, dim3(d.dn_blocks[1]), dim3(kThreads), 0, s, a, W);
}

}  // namespace

int sm_count() { return dev_info().sms; }

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
        Layout lo = make_layout(T, (int)l.meta.cols[0], (int)l.meta.rows[0], l.n_experts,
                                l.top_k, l.shared_blob != nullptr);
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
                             cudaStream_t stream, WispErrCtx* err, LayerArgs* a_out, Ws* w_out) {
    WispError ce = common_checks(layer, 1, T, workspace, workspace_bytes, err);
    if (ce != WISP_OK) return ce;
    if (!x || !aligned_io(x)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "moe block: x NULL or not 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    LayerArgs a = layer_args(layer);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared);
    Ws W = make_ws(workspace, lo);
    if (topk_idx) W.topk_idx = topk_idx;
    if (topk_w) W.topk_w = topk_w;
    WB_CUDA_RET(ensure_attrs(a.H), err);
    WB_CUDA_RET(cudaMemsetAsync(W.status, 0, sizeof(int), stream), err);
    WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kThreads), prep_smem(a.H), stream, a, W, T,
                       (int)P_QUANT, const_cast<float*>(x), (float*)nullptr, 0.f, 0, 0),
                err);
    const int mt = T == 1 ? 1 : kMT;
    const int neb = (a.E + kWarps - 1) / kWarps;
    WB_CUDA_RET(launch(router_kernel, dim3(neb, T), dim3(kThreads), router_smem(), stream, a, W, T,
                       mt, x),
                err);
    *a_out = a;
    *w_out = W;
    return WISP_OK;
}

// gate/up + down + combine, on the plan the preceding route left in the workspace.
static WispError block_experts(const LayerArgs& a, const Ws& W, int T, const float* x, float* y,
                               cudaStream_t stream, WispErrCtx* err) {
    const DevInfo d = dev_info();
    if (T == 1) {
        WB_CUDA_RET(launch(gateup_kernel<1>, dim3(d.gu_blocks[0]), dim3(kThreads), 0, stream, a, W),
                    err);
        WB_CUDA_RET(launch(down_kernel<1>, dim3(d.dn_blocks[0]), dim3(kThreads), 0, stream, a, W),
                    err);
    } else {
        WB_CUDA_RET(launch(gateup_kernel<kMT>, dim3(d.gu_blocks[1]), dim3(kThreads), 0, stream, a,
                           W),
                    err);
        WB_CUDA_RET(launch(down_kernel<kMT>, dim3(d.dn_blocks[1]), dim3(kThreads), 0, stream, a, W),
                    err);
    }
    Ws Wc = W;
    Wc.prev_idx = W.topk_idx;
    Wc.prev_w = W.topk_w;
    WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kThreads), prep_smem(a.H), stream, a, Wc, T,
                       (int)P_COMBINE, const_cast<float*>(x), y, 0.f, a.K, a.has_shared),
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
    LayerArgs a;
    Ws W;
    WispError r = block_route(layer, x, T, topk_idx, topk_w, workspace, workspace_bytes, stream,
                              err, &a, &W);
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
    LayerArgs a = layer_args(layer);
    Layout lo = make_layout(T, a.H, a.I, a.E, a.K, a.has_shared);
    Ws W = make_ws(workspace, lo);
    if (topk_idx) W.topk_idx = topk_idx;
    if (topk_w) W.topk_w = topk_w;
    WB_CUDA_RET(ensure_attrs(a.H), err);
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
    int maxI = 0, maxE = 0, maxK = 0;
    bool anysh = false;
    for (int l = 0; l < n_layers; ++l) {
        maxI = std::max(maxI, (int)layers[l].meta.rows[0]);
        maxE = std::max(maxE, layers[l].n_experts);
        maxK = std::max(maxK, layers[l].top_k);
        anysh = anysh || layers[l].shared_blob;
    }
    const int H = (int)layers[0].meta.cols[0];
    WB_CUDA_RET(ensure_attrs(H), err);
    WB_CUDA_RET(cudaMemsetAsync(workspace, 0, sizeof(int), stream), err);
    int prevK = 0, prev_sh = 0;
    for (int l = 0; l < n_layers; ++l) {
        LayerArgs a = layer_args(&layers[l]);
        Layout lo = make_layout(T, H, maxI, maxE, maxK, anysh);
        Ws W = make_ws(workspace, lo);
        // previous layer's routing lives in the "current" slots until this
        // layer's router overwrites them; prep reads it first (stream order)
        Ws Wp = W;
        if (l > 0) {
            Wp.prev_idx = topk_idx ? topk_idx + (size_t)(l - 1) * T * prevK : W.topk_idx;
            Wp.prev_w = topk_w ? topk_w + (size_t)(l - 1) * T * prevK : W.topk_w;
        }
        const int flags = (l > 0 ? (P_COMBINE | P_RESID) : 0) | P_NORM | P_QUANT;
        WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kThreads), prep_smem(H), stream, a, Wp,
                               T, flags, x, (float*)nullptr, eps, prevK, prev_sh),
                    err);
        if (topk_idx) W.topk_idx = topk_idx + (size_t)l * T * a.K;
        if (topk_w) W.topk_w = topk_w + (size_t)l * T * a.K;
        WB_CUDA_RET(run_layer_experts(a, W, T, W.xn, stream), err);
        prevK = a.K;
        prev_sh = a.has_shared;
        if (l == n_layers - 1) {
            Ws Wf = W;
            Wf.prev_idx = W.topk_idx;
            Wf.prev_w = W.topk_w;
            WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kThreads), prep_smem(H), stream, a,
                                   Wf, T, (int)(P_COMBINE | P_RESID), x, (float*)nullptr, eps,
                                   prevK, prev_sh),
                        err);
        }
    }
    hook_mark(stream);
    return WISP_OK;
}
