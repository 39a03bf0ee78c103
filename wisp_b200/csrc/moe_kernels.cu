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
//   hquant_kernel  quantise h
//   down_kernel    ypart[part][assignment][row] = D.h over one K part
//   prep_kernel    (next layer, or the final combine) sum_j w_j * sum_parts
//
// Weight streaming (gate/up, down): a producer warp hands (tile, row block)
// units from an atomic counter to a ring of shared-memory stages filled by
// cp.async.bulk (TMA) copies; eight consumer warps split the unit's K range.
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
#include <mutex>

#include "internal.h"

namespace wb {
namespace {

constexpr int kChunk = 32;      // elements per MMA k-slice (16 packed bytes)
constexpr int kMT = 4;          // max tokens per expert tile (= MMA N / 2)
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxPlanAssign = 4096;  // T*k limit of the device plan builder
constexpr int kMaxKp = 32;            // max K parts of the down projection

enum { C_GU_TASK = 0, C_TOK_DONE = 2, C_NTILES = 3, C_DN_BASE = 8 };
constexpr int kCounters = C_DN_BASE + kMaxKp;  // gate/up units, tokens, tiles, down units per part
enum { ST_ALIGN = 1, ST_EXPERT = 2, ST_PLAN = 4, ST_TIMEOUT = 8 };

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
    int kp;   // K parts of the down projection
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
    float2* xqp;    // [T][H/gs]     (k/254, sum of quantised x) per group
    float* h;       // [A][I]
    uint4* hq;      // [A][I/32][4]
    float2* hqp;    // [A][I/gs]
    int* hcnt;      // unused
    float* ypart;   // [kp][A][H]
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
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
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
                                               float2* block_param, bool block_leader) {
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
    if (block_leader) *block_param = make_float2(k2, fmaf(k, (float)sa, k2 * (float)sb));
}

// Quantise the n-element row `src` (n % gs == 0) with one warp per 128
// elements; warps and lanes past the end redo the last block (same data).
// `warp_id`/`n_warps` index the warps taking part.
__device__ __forceinline__ void quantize_row(const float4* src, int n, int gs, int warp_id,
                                             int n_warps, uint4* xq, float2* xqp) {
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
// prep: combine + residual + RMSNorm + activation quantisation (per token)
// ------------------------------------------------------------------------
enum { P_COMBINE = 1, P_RESID = 2, P_NORM = 4, P_QUANT = 8 };
constexpr int kPrepThreads = 1024;

// One CTA per token, 1024 threads, float4 granules.
__global__ void __launch_bounds__(kPrepThreads)
prep_kernel(LayerArgs L, Ws W, int T, int flags, float* x, float* y, float eps, int prevK,
            int prev_shared, int prev_kp) {
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.x;
    const int H = L.H, n4 = H / 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float red[32];
    __shared__ float s_scale;
    __shared__ float s_w[64];
    __shared__ int s_i[64];
    extern __shared__ float4 sx4[];  // [H/4]
    float4* xt = reinterpret_cast<float4*>(x + (size_t)t * H);

    if (t == 0 && tid == 0) W.counters[C_TOK_DONE] = 0;
    if (flags & P_COMBINE) {
        if (tid < prevK) {
            s_i[tid] = W.prev_idx[t * prevK + tid];
            s_w[tid] = W.prev_w[t * prevK + tid];
        }
        __syncthreads();
    }
    const size_t part_stride = (size_t)W.A * H;
    float ss = 0.f;
    for (int i = tid; i < n4; i += kPrepThreads) {
        float4 v = xt[i];
        if (flags & P_COMBINE) {
            // reference order: shared expert first (weight 1), then top-k order
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (prev_shared) {
                const size_t a = (size_t)T * prevK + t;
                for (int p = 0; p < prev_kp; ++p) {
                    const float4 yv =
                        reinterpret_cast<const float4*>(W.ypart + p * part_stride + a * H)[i];
                    acc.x += yv.x; acc.y += yv.y; acc.z += yv.z; acc.w += yv.w;
                }
            }
            for (int j = 0; j < prevK; ++j) {
                if (s_i[j] < 0) continue;
                const size_t a = (size_t)t * prevK + j;
                float4 yj = reinterpret_cast<const float4*>(W.ypart + a * H)[i];
                for (int p = 1; p < prev_kp; ++p) {
                    const float4 yv =
                        reinterpret_cast<const float4*>(W.ypart + p * part_stride + a * H)[i];
                    yj.x += yv.x; yj.y += yv.y; yj.z += yv.z; yj.w += yv.w;
                }
                const float wj = s_w[j];
                acc.x += wj * yj.x; acc.y += wj * yj.y; acc.z += wj * yj.z; acc.w += wj * yj.w;
            }
            if (flags & P_RESID) {
                v.x += acc.x; v.y += acc.y; v.z += acc.z; v.w += acc.w;
                xt[i] = v;
            } else {
                v = acc;
            }
            if (y) reinterpret_cast<float4*>(y + (size_t)t * H)[i] = v;
        }
        sx4[i] = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    if (!(flags & (P_NORM | P_QUANT))) return;
    if (flags & P_NORM) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = red[lane];
            v = warp_sum(v);
            if (lane == 0) s_scale = 1.0f / sqrtf(v / (float)H + eps);
        }
        __syncthreads();
        const float sc = s_scale;
        float4* xn = reinterpret_cast<float4*>(W.xn + (size_t)t * H);
        const __half2* nw = reinterpret_cast<const __half2*>(L.norm_w);
        for (int i = tid; i < n4; i += kPrepThreads) {
            float4 v = sx4[i];
            v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
            if (nw) {
                const float2 a = __half22float2(nw[2 * i]), b = __half22float2(nw[2 * i + 1]);
                v.x *= a.x; v.y *= a.y; v.z *= b.x; v.w *= b.y;
            }
            sx4[i] = v;
            xn[i] = v;
        }
    }
    __syncthreads();
    if (flags & P_QUANT)
        quantize_row(sx4, H, L.gs, warp, kPrepThreads / 32, W.xq + (size_t)t * (H / kChunk) * 4,
                     W.xqp + (size_t)t * (H / L.gs));
}

// ------------------------------------------------------------------------
// router: per-(expert, 1024-element slice) partial logits for every token,
// then the last CTA to finish sums the slices (fixed order), adds the bias,
// does softmax + top-k per token and builds the expert-tile plan.
// ------------------------------------------------------------------------
constexpr int kSlice = 1024;

__device__ void topk_token(const LayerArgs& L, const Ws& W, int t, int K, int nsl, float* sp,
                           int* staken) {
    // one warp; sp/staken: [E] shared scratch of this warp
    const int lane = threadIdx.x & 31;
    const int E = L.E;
    float mx = -1e30f;
    for (int e = lane; e < E; e += 32) {
        const float* pp = W.logits + ((size_t)t * E + e) * nsl;
        float v = 0.f;
        for (int s = 0; s < nsl; ++s) v += __ldcg(pp + s);
        if (L.router_bias) v += __half2float(L.router_bias[e]);
        sp[e] = v;
        staken[e] = 0;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    float den = 0.f;
    for (int e = lane; e < E; e += 32) {
        const float v = expf(sp[e] - mx);
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
            const float v = sp[e];
            if (!staken[e] && v > bv) {
                bv = v;
                be = e;
            }
        }
        // warp argmax: larger value wins, equal values -> lower index
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(kFull, bv, o);
            const int oe = __shfl_xor_sync(kFull, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (bv < 0.f) be = -1;
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
    if (tid == 0) {
        W.counters[C_NTILES] = total;
        W.counters[C_GU_TASK] = 0;
        for (int p = 0; p < kMaxKp; ++p) W.counters[C_DN_BASE + p] = 0;
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
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(W.counters + C_TOK_DONE, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    {
        float* sp = reinterpret_cast<float*>(smem) + (size_t)warp * 2 * E;
        int* staken = smem + (size_t)warp * 2 * E + E;
        for (int t = warp; t < T; t += kWarps) topk_token(L, W, t, L.K, nsl, sp, staken);
    }
    __syncthreads();
    __threadfence();
    build_plan(L, W, T, mt, smem, smem + kMaxPlanAssign);
}

// ------------------------------------------------------------------------
// TMA-staged weight streaming (shared by gate/up and down)
//
// One CTA = 1 producer warp + the consumer warps.  The producer takes
// units (tile, block of 8 rows[, K part]) from an atomic counter and issues
// cp.async.bulk global->shared copies of the unit's packed rows and fp16
// scales/zeros into a ring of shared-memory stages, each guarded by a "full"
// mbarrier (transaction bytes) and an "empty" mbarrier (one arrival per
// consumer warp).  Consumer warp w computes row 8*rb + w of the unit from
// shared memory.  Every wait is bounded by %globaltimer: on timeout the warp
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
// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > kWaitNs) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// One bulk copy request of a unit: up to 48 per unit (gate/up: 6; down with a
// K split: 3 per row).
struct Copy {
    const void* src;
    uint32_t dst_off, bytes;
};

__host__ __device__ constexpr size_t ring_extra_bytes(int stages) {
    return (size_t)stages * 20 + 64;  // full + empty barriers, unit ids, slack
}

struct StreamSmem {
    uint8_t* stages;
    uint64_t* full;
    uint64_t* empty;
    int* unit;
    uint32_t stage_bytes;
    int n_stages;
};

__device__ __forceinline__ StreamSmem stream_smem(uint8_t* base, int n_stages,
                                                  uint32_t stage_bytes) {
    StreamSmem s;
    s.stages = base;
    s.full = reinterpret_cast<uint64_t*>(base + (size_t)n_stages * stage_bytes);
    s.empty = s.full + n_stages;
    s.unit = reinterpret_cast<int*>(s.empty + n_stages);
    s.stage_bytes = stage_bytes;
    s.n_stages = n_stages;
    return s;
}

__device__ __forceinline__ void load_tile(const Tile* src, Tile& tl) {
    const int* s = reinterpret_cast<const int*>(src);
    int* d = reinterpret_cast<int*>(&tl);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(Tile) / 4); ++i) d[i] = __ldcg(s + i);
}

__device__ __forceinline__ const void* tile_blob(const LayerArgs& L, int expert,
                                                 const MatOff*& off) {
    if (expert == L.E) {
        off = L.smat;
        return L.shared_blob;
    }
    off = L.mat;
    return (expert >= 0 && expert < L.E) ? L.blobs[expert] : nullptr;
}

// Stage layout of a unit of 16 rows x K range (see UnitGeom); `padded`
// when every row can be its own 16-byte-multiple copy.
struct StageLayout {
    uint32_t rb, sb;    // row bytes of the range: packed, scales
    uint32_t rbp, sbp;  // strides in the stage
    bool padded;
    uint32_t bytes;
};
__host__ __device__ inline StageLayout stage_layout(int k_range, int gs) {
    StageLayout s;
    s.rb = (uint32_t)k_range / 2;
    s.sb = (uint32_t)(k_range / gs) * 2;
    s.padded = (s.rb % 16 == 0) && (s.sb % 16 == 0);
    s.rbp = s.padded ? s.rb + 16 : s.rb;
    s.sbp = s.padded ? s.sb + 16 : s.sb;
    s.bytes = 16 * s.rbp + 32 * s.sbp;
    return s;
}

// Producer warp: fill stages until the units run out, then post a sentinel.
// The next unit id is fetched from the counter one unit ahead, so the atomic's
// latency overlaps the current unit's copies.  Lane r < 16 owns MMA row r of
// the unit: `rowsrc(u, r, p, sc, ze)` gives the global addresses of its packed
// bytes, scales and zeros (false = unusable unit, status already flagged).
// Padded layout: every lane < 16 copies its own row's three sections;
// otherwise lanes 0 and 8 copy 8 contiguous rows each.
template <typename RowSrc>
__device__ void produce(const StreamSmem& S, const Ws& W, int* counter, long long total,
                        const StageLayout& sl, RowSrc rowsrc) {
    const int lane = threadIdx.x & 31;
    const uint32_t soff = 16 * sl.rbp, zoff = soff + 16 * sl.sbp;
    const uint32_t tx = 16 * (sl.rb + 2 * sl.sb);
    int u_next = 0;
    if (lane == 0) u_next = atomicAdd(counter, 1);
    u_next = __shfl_sync(kFull, u_next, 0);
    int it = 0;
    bool ok = true;
    for (;; ++it) {
        const int s = it % S.n_stages;
        int waited = 1;
        if (lane == 0) waited = mbar_wait(&S.empty[s], ((it / S.n_stages) & 1) ^ 1) ? 1 : 0;
        if (!__shfl_sync(kFull, waited, 0)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            ok = false;
            break;
        }
        const int u = u_next;
        if (u >= total) {
            if (lane == 0) {
                S.unit[s] = -1;
                mbar_arrive(&S.full[s]);
            }
            break;
        }
        if (lane == 0) u_next = atomicAdd(counter, 1);
        const uint8_t *p = nullptr, *sc = nullptr, *ze = nullptr;
        bool good = true;
        if (lane < 16) good = rowsrc(u, lane, p, sc, ze);
        int n = 0;
        Copy c[3];
        if (sl.padded) {
            if (lane < 16) {
                c[0] = Copy{p, lane * sl.rbp, sl.rb};
                c[1] = Copy{sc, soff + lane * sl.sbp, sl.sb};
                c[2] = Copy{ze, zoff + lane * sl.sbp, sl.sb};
                n = 3;
            }
        } else if (lane == 0 || lane == 8) {
            const uint32_t h = lane / 8;
            c[0] = Copy{p, 8 * h * sl.rb, 8 * sl.rb};
            c[1] = Copy{sc, soff + 8 * h * sl.sb, 8 * sl.sb};
            c[2] = Copy{ze, zoff + 8 * h * sl.sb, 8 * sl.sb};
            n = 3;
        }
        for (int i = 0; i < n; ++i)
            good = good && aligned16(c[i].src) && !(c[i].bytes & 15u) && !(c[i].dst_off & 15u);
        const bool all = __all_sync(kFull, good);
        if (lane == 0) {
            S.unit[s] = all ? u : -2;
            if (all) {
                mbar_expect_tx(&S.full[s], tx);
            } else {
                atomicOr(W.status, ST_ALIGN);
                mbar_arrive(&S.full[s]);
            }
        }
        __syncwarp();
        if (all) {
            uint8_t* dst = S.stages + (size_t)s * S.stage_bytes;
            for (int i = 0; i < n; ++i) bulk_g2s(dst + c[i].dst_off, c[i].src, c[i].bytes, &S.full[s]);
        }
        u_next = __shfl_sync(kFull, u_next, 0);
    }
    __syncwarp();
    if (!ok && lane == 0) {
        // a consumer stopped early: let every issued copy land before exiting
        for (int k = 0; k < S.n_stages && k < it; ++k) {
            const int j = it - 1 - k;
            mbar_wait(&S.full[j % S.n_stages], (j / S.n_stages) & 1);
        }
    }
}

// ------------------------------------------------------------------------
// Tensor-core consumers.  A unit is 16 MMA rows over a K range of ng quant
// groups (gate/up: rows 0-7 = gate rows, 8-15 = up rows of 8 output rows;
// down: 16 output rows of one K part).  kNcw consumer warps split the K range
// into contiguous runs of group pairs; thread (g = lane/4, q = lane%4)
// accumulates rows g and g+8 for token q in fp32.
//
// Shared memory of a streaming CTA: the stage ring, then the activation tile
// (the B fragments of every MMA of the K range in per-lane order, and the
// per-group (k/254, S) of each token slot) -- written once per tile (and
// part) by the consumers, so the steady state reads only shared memory --
// then the cross-warp reduction scratch.
// ------------------------------------------------------------------------
constexpr int kNcw = 16;                          // consumer warps per CTA
constexpr int kStreamCta = 32 * (kNcw + 1);       // + 1 producer warp

struct UnitGeom {
    int ng;         // quant groups in the unit's K range
    uint32_t rbp;   // packed row stride in the stage
    uint32_t sbp;   // scale/zero row stride in the stage
    uint32_t zoff;  // offset of the zero rows from the scale rows
};

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
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
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
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

// Stage the activation tile of a K range: for each group G and MMA i, the
// (b0, b1) of every lane, and (k/254, S) of each token slot.  xw/xp point at
// the range's first chunk/group of token row 0; rows are nchk chunks / ngrp
// groups apart.  Executed by all consumer threads.
template <int NPG>
__device__ __forceinline__ void stage_xtile(uint2* xt, float2* xtp, int ng, const uint4* xw,
                                            const float2* xp, int nchk, int ngrp,
                                            const int* xrow, int m_tok) {
    const int ct = threadIdx.x - 32, nct = kNcw * 32;
    const uint2* xw2 = reinterpret_cast<const uint2*>(xw);
    const int nent = ng * NPG * 32;
    for (int e = ct; e < nent; e += nct) {
        const int l = e & 31, gi = e >> 5;  // gi = G*NPG + i
        const int G = gi / NPG, i = gi - G * NPG;
        const int g = l >> 2, q = l & 3;
        const int bt = g >> 1, bd = g & 1;
        uint2 v = make_uint2(0u, 0u);
        if (bt < m_tok) {
            const int wi = q * NPG + i;
            const int chunk = G * NPG + (wi >> 2);
            v = __ldg(xw2 + (size_t)xrow[bt] * nchk * 8 + (size_t)chunk * 8 + bd * 4 + (wi & 3));
        }
        xt[e] = v;
    }
    for (int e = ct; e < ng * kMT; e += nct) {
        const int G = e / kMT, t = e - G * kMT;
        xtp[e] = t < m_tok ? __ldg(xp + (size_t)xrow[t] * ngrp + G) : make_float2(0.f, 0.f);
    }
}

// Operands of a pair of groups (2P, 2P+1), loaded one pair ahead of use.
template <int NPG>
struct PairFrag {
    Words<NPG> wl[2], wh[2];  // packed words of rows g, g+8
    uint2 b[2][NPG];          // B fragments
    float2 kp[2];             // (k/254, S) of token q
    uint32_t s_lo, z_lo, s_hi, z_hi;  // half2 scales/zeros of rows g, g+8
    bool two;                         // the pair's second group exists
};

// Partial dot products of one unit for this thread: acc[0] = row g, acc[1] =
// row g+8, token q.  `xt`/`xtp`: the staged activation tile (shared memory).
template <int NPG>
__device__ __forceinline__ void mma_unit(const uint8_t* st, const UnitGeom& geo, uint32_t xt,
                                         uint32_t xtp, float (&acc)[2]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int cw = (threadIdx.x >> 5) - 1;  // consumer warp
    const int npair = (geo.ng + 1) >> 1;
    const int p0 = (cw * npair) / kNcw, p1 = ((cw + 1) * npair) / kNcw;
    if (p0 >= p1) return;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(st);
    const uint32_t a_lo = sbase + g * geo.rbp + q * (NPG * 4);
    const uint32_t a_hi = a_lo + 8 * geo.rbp;
    const uint32_t s_lo = sbase + 16 * geo.rbp + g * geo.sbp;
    const uint32_t s_hi = s_lo + 8 * geo.sbp;
    const bool s_al = (geo.sbp & 3) == 0;  // scale rows allow half2 loads
    const uint32_t xtl = xt + lane * 8, xtq = xtp + q * 8;
    const int ng = geo.ng;
    auto ld2 = [&](uint32_t a) -> uint32_t {
        return s_al ? lds32(a) : (lds16(a) | (lds16(a + 2) << 16));
    };
    auto load = [&](int P, PairFrag<NPG>& f) {
        const int G = 2 * P;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int Gh = min(G + h, ng - 1);  // a missing odd group reads group ng-1 with kp = 0
            f.wl[h] = lds_w<NPG>(a_lo + Gh * (NPG * 16));
            f.wh[h] = lds_w<NPG>(a_hi + Gh * (NPG * 16));
#pragma unroll
            for (int i = 0; i < NPG; ++i) f.b[h][i] = lds64(xtl + (Gh * NPG + i) * 256);
            const uint2 kv = lds64(xtq + Gh * (kMT * 8));
            f.kp[h] = G + h < ng ? make_float2(__uint_as_float(kv.x), __uint_as_float(kv.y))
                                 : make_float2(0.f, 0.f);
        }
        f.two = G + 1 < ng;
        f.s_lo = ld2(s_lo + 2 * G);
        f.z_lo = ld2(s_lo + geo.zoff + 2 * G);
        f.s_hi = ld2(s_hi + 2 * G);
        f.z_hi = ld2(s_hi + geo.zoff + 2 * G);
    };
    auto compute = [&](const PairFrag<NPG>& f) {
        const float2 slo = __half22float2(*reinterpret_cast<const __half2*>(&f.s_lo));
        const float2 zlo = __half22float2(*reinterpret_cast<const __half2*>(&f.z_lo));
        const float2 shi = __half22float2(*reinterpret_cast<const __half2*>(&f.s_hi));
        const float2 zhi = __half22float2(*reinterpret_cast<const __half2*>(&f.z_hi));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < NPG; ++i) {
                uint32_t a[4];
                a[0] = f.wl[h].w[i] & 0x0F0F0F0Fu;
                a[1] = f.wh[h].w[i] & 0x0F0F0F0Fu;
                a[2] = (f.wl[h].w[i] >> 4) & 0x0F0F0F0Fu;
                a[3] = (f.wh[h].w[i] >> 4) & 0x0F0F0F0Fu;
                mma_s8(d, a, f.b[h][i].x, f.b[h][i].y);
            }
            // kp = 0 (absent group or token) makes the contribution 0
            const float m8 = -8.0f * f.kp[h].y;
            const float c_lo = (float)(d[0] * 254 + d[1]);
            const float c_hi = (float)(d[2] * 254 + d[3]);
            // an absent second group (odd count) has kp = 0 and may have read
            // scale bytes past the row end: use 0 so they cannot make a NaN
            const bool live = h == 0 || f.two;
            const float sl = live ? (h ? slo.y : slo.x) : 0.f, zl = live ? (h ? zlo.y : zlo.x) : 0.f;
            const float sh = live ? (h ? shi.y : shi.x) : 0.f, zh = live ? (h ? zhi.y : zhi.x) : 0.f;
            acc[0] = fmaf(sl, fmaf(f.kp[h].x, c_lo, m8), fmaf(zl, f.kp[h].y, acc[0]));
            acc[1] = fmaf(sh, fmaf(f.kp[h].x, c_hi, m8), fmaf(zh, f.kp[h].y, acc[1]));
        }
    };
    PairFrag<NPG> fa, fb;
    load(p0, fa);
    for (int P = p0; P < p1; P += 2) {
        if (P + 1 < p1) load(P + 1, fb);
        compute(fa);
        if (P + 1 >= p1) break;
        if (P + 2 < p1) load(P + 2, fa);
        compute(fb);
    }
}

// Sum the consumer warps' partials (fixed order).  Returns, for the threads
// of consumer warp 0, the unit sums of rows g and g+8 for token q.
__device__ __forceinline__ bool unit_reduce(const float (&acc)[2], float2* part,
                                            float (&out)[2]) {
    const int lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 1;
    part[cw * 32 + lane] = make_float2(acc[0], acc[1]);
    asm volatile("bar.sync 1, %0;" ::"r"(kNcw * 32) : "memory");
    if (cw != 0) return false;
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int w = 0; w < kNcw; ++w) {
        const float2 v = part[w * 32 + lane];
        a += v.x;
        b += v.y;
    }
    out[0] = a;
    out[1] = b;
    return true;
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kNcw * 32) : "memory");
}

// Dynamic shared memory of a streaming CTA (see the section comment).
struct StreamLayout {
    uint8_t* ring;
    uint2* xt;
    float2* xtp;
    float2* red;  // [2][kNcw*32]
};
__device__ __forceinline__ StreamLayout stream_layout(uint8_t* base, int n_stages,
                                                      uint32_t stage_bytes, int ng, int npg) {
    StreamLayout s;
    s.ring = base;
    size_t o = (size_t)n_stages * stage_bytes + ring_extra_bytes(n_stages);
    o = (o + 127) & ~size_t(127);
    s.xt = reinterpret_cast<uint2*>(base + o);
    o += (size_t)ng * npg * 32 * sizeof(uint2);
    s.xtp = reinterpret_cast<float2*>(base + o);
    o += (size_t)ng * kMT * sizeof(float2);
    o = (o + 15) & ~size_t(15);
    s.red = reinterpret_cast<float2*>(base + o);
    return s;
}

// ------------------------------------------------------------------------
// gate/up + SwiGLU: unit = 8 output rows (gate rows + up rows) x all of H
// ------------------------------------------------------------------------
template <int NPG>
__global__ void __launch_bounds__(kStreamCta, 1)
gateup_kernel(LayerArgs L, Ws W, int n_stages, uint32_t stage_bytes) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const StreamSmem S = stream_smem(smem_raw, n_stages, stage_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = L.H, I = L.I, gs = L.gs;
    const StreamLayout X = stream_layout(smem_raw, n_stages, stage_bytes, H / gs, NPG);
    if (threadIdx.x == 0) {
        for (int s = 0; s < n_stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kNcw);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_launch();
    const int rbs = I / 8;  // 8-row blocks per tile
    const long long total = (long long)__ldcg(W.counters + C_NTILES) * rbs;
    const StageLayout sl = stage_layout(H, gs);

    if (warp == 0) {
        int ctile = -1;
        const uint8_t* cblob = nullptr;
        const MatOff* coff = nullptr;
        produce(S, W, W.counters + C_GU_TASK, total, sl,
                [&](int u, int r, const uint8_t*& p, const uint8_t*& sc,
                    const uint8_t*& ze) -> bool {
                    const int ti = u / rbs;
                    if (ti != ctile) {
                        Tile tl;
                        load_tile(W.tiles + ti, tl);
                        cblob = static_cast<const uint8_t*>(tile_blob(L, tl.expert, coff));
                        ctile = ti;
                    }
                    if (!cblob) {
                        atomicOr(W.status, ST_EXPERT);
                        return false;
                    }
                    const MatOff& o = coff[r < 8 ? 0 : 1];
                    const size_t row = (size_t)(u % rbs) * 8 + (r & 7);
                    p = cblob + o.packed + row * sl.rb;
                    sc = cblob + o.scales + row * sl.sb;
                    ze = cblob + o.zeros + row * sl.sb;
                    return true;
                });
        return;
    }
    const UnitGeom geo{H / gs, sl.rbp, sl.sbp, 16 * sl.sbp};
    const uint32_t xt = (uint32_t)__cvta_generic_to_shared(X.xt);
    const uint32_t xtp = (uint32_t)__cvta_generic_to_shared(X.xtp);
    int cur = -1;
    Tile tl;
    for (int it = 0;; ++it) {
        const int s = it % n_stages;
        if (!mbar_wait(&S.full[s], (it / n_stages) & 1)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            break;
        }
        const int u = *reinterpret_cast<volatile int*>(&S.unit[s]);
        if (u == -1) break;
        if (u < 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
            continue;
        }
        const int ti = u / rbs;
        if (ti != cur) {
            // every consumer is past the previous unit's reduction barrier
            load_tile(W.tiles + ti, tl);
            stage_xtile<NPG>(X.xt, X.xtp, H / gs, W.xq, W.xqp, H / kChunk, H / gs, tl.tok, tl.m);
            consumers_sync();
            cur = ti;
        }
        float acc[2] = {0.f, 0.f};
        mma_unit<NPG>(S.stages + (size_t)s * stage_bytes, geo, xt, xtp, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);  // the stage is no longer read
        float out[2];
        if (unit_reduce(acc, X.red + (it & 1) * kNcw * 32, out)) {
            const int g = lane >> 2, q = lane & 3;
            if (q < tl.m) {
                const int row = (u % rbs) * 8 + g;
                W.h[(size_t)tl.asg[q] * I + row] = out[0] / (1.0f + expf(-out[0])) * out[1];
            }
        }
    }
}

// ------------------------------------------------------------------------
// h quantiser: every quant group of h (all assignments), 128 elements per
// warp.
// ------------------------------------------------------------------------
__global__ void __launch_bounds__(kPrepThreads)
hquant_kernel(LayerArgs L, Ws W) {
    pdl_wait();
    pdl_launch();
    const int I = L.I;
    const int warps = kPrepThreads / 32;
    const int per_a = (I + 127) / 128;  // warps per assignment row
    const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
    const int a = gw / per_a;
    if (a >= W.A) return;
    const int wi = gw % per_a;
    quantize_row(reinterpret_cast<const float4*>(W.h + (size_t)a * I), I, L.gs, wi, per_a,
                 W.hq + (size_t)a * (I / kChunk) * 4, W.hqp + (size_t)a * (I / L.gs));
}

// ------------------------------------------------------------------------
// down projection: unit = 16 output rows x one of kp K parts.  A CTA serves
// one part (blockIdx.x % kp), so its activation tile changes only with the
// expert tile; units of a part come from that part's counter.  Each part is
// written to its own ypart buffer and the combine adds them in fixed order
// (deterministic, no float atomics).
// ------------------------------------------------------------------------
template <int NPG>
__global__ void __launch_bounds__(kStreamCta, 1)
down_kernel(LayerArgs L, Ws W, int n_stages, uint32_t stage_bytes) {
    const int kp = L.kp;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const StreamSmem S = stream_smem(smem_raw, n_stages, stage_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = L.H, I = L.I, gs = L.gs;
    const int kr = I / kp;  // K range of a part
    const StreamLayout X = stream_layout(smem_raw, n_stages, stage_bytes, kr / gs, NPG);
    if (threadIdx.x == 0) {
        for (int s = 0; s < n_stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kNcw);
        }
        mbar_fence_init();
    }
    __syncthreads();
    // The producer streams weights before the previous kernel (the h
    // quantiser) has finished: weights, the expert table and the tile plan
    // (written by the router, which completed before the gate/up kernel that
    // precedes the quantiser could start) do not depend on it.  Consumers wait
    // for it before reading the quantised h.
    pdl_launch();
    const int pi = blockIdx.x % kp;
    const int rbs = H / 16;
    const long long total = (long long)__ldcg(W.counters + C_NTILES) * rbs;
    const StageLayout sl = stage_layout(kr, gs);

    if (warp == 0) {
        int ctile = -1;
        const uint8_t* cblob = nullptr;
        const MatOff* coff = nullptr;
        const size_t rowb = I / 2, rows = (size_t)(I / gs) * 2;
        produce(S, W, W.counters + C_DN_BASE + pi, total, sl,
                [&](int u, int r, const uint8_t*& p, const uint8_t*& sc,
                    const uint8_t*& ze) -> bool {
                    const int ti = u / rbs;
                    if (ti != ctile) {
                        Tile tl;
                        load_tile(W.tiles + ti, tl);
                        cblob = static_cast<const uint8_t*>(tile_blob(L, tl.expert, coff));
                        ctile = ti;
                    }
                    if (!cblob) {
                        atomicOr(W.status, ST_EXPERT);
                        return false;
                    }
                    const size_t row = (size_t)(u % rbs) * 16 + r;
                    p = cblob + coff[2].packed + row * rowb + pi * sl.rb;
                    sc = cblob + coff[2].scales + row * rows + pi * sl.sb;
                    ze = cblob + coff[2].zeros + row * rows + pi * sl.sb;
                    return true;
                });
        return;
    }
    pdl_wait();
    const UnitGeom geo{kr / gs, sl.rbp, sl.sbp, 16 * sl.sbp};
    const uint32_t xt = (uint32_t)__cvta_generic_to_shared(X.xt);
    const uint32_t xtp = (uint32_t)__cvta_generic_to_shared(X.xtp);
    int cur = -1;
    Tile tl;
    for (int it = 0;; ++it) {
        const int s = it % n_stages;
        if (!mbar_wait(&S.full[s], (it / n_stages) & 1)) {
            if (lane == 0) atomicOr(W.status, ST_TIMEOUT);
            break;
        }
        const int u = *reinterpret_cast<volatile int*>(&S.unit[s]);
        if (u == -1) break;
        if (u < 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
            continue;
        }
        const int ti = u / rbs;
        if (ti != cur) {
            load_tile(W.tiles + ti, tl);
            // activations of this part: chunks [pi*kr/32, ...), groups [pi*kr/gs, ...)
            stage_xtile<NPG>(X.xt, X.xtp, kr / gs, W.hq + (size_t)pi * (kr / kChunk) * 4,
                             W.hqp + (size_t)pi * (kr / gs), I / kChunk, I / gs, tl.asg, tl.m);
            consumers_sync();
            cur = ti;
        }
        float acc[2] = {0.f, 0.f};
        mma_unit<NPG>(S.stages + (size_t)s * stage_bytes, geo, xt, xtp, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
        float out[2];
        if (unit_reduce(acc, X.red + (it & 1) * kNcw * 32, out)) {
            const int g = lane >> 2, q = lane & 3;
            if (q < tl.m) {
                const int row = (u % rbs) * 16 + g;
                float* dst = W.ypart + ((size_t)pi * W.A + tl.asg[q]) * H + row;
                dst[0] = out[0];
                dst[8] = out[1];
            }
        }
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
    l.xqp = take((size_t)T * (H / kChunk) * sizeof(float2));  // >= per-group params
    l.h = take((size_t)l.A * I * sizeof(float));
    l.hq = take((size_t)l.A * (I / kChunk) * 64);
    l.hqp = take((size_t)l.A * (I / kChunk) * sizeof(float2));
    l.hcnt = take((size_t)l.A * (I / kChunk) * sizeof(int));
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
    if (H % kChunk || I % kChunk || H % gs || I % gs || H % 16 || I % 8 ||
        (gs != 32 && gs != 64 && gs != 128)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "moe layer: unsupported shape H=%d I=%d group_size=%d (need multiples "
                   "of 32, H of 16, group_size 32/64/128 dividing H and I)",
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

// K parts of the down projection: the smallest split whose part is at most
// 2048 wide and still splits into whole quant groups with padded stage rows.
int down_parts(int I, int gs) {
    for (int kp = 1; kp <= kMaxKp; ++kp) {
        if (I % kp) continue;
        const int kr = I / kp;
        if (kr % kChunk || kr % gs) continue;
        if (kp > 1 && (kr / gs) % 8) continue;
        if (kr <= 2048) return kp;
    }
    return 1;
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
    a.kp = down_parts(a.I, a.gs);
    return a;
}

// Shared memory of a streaming CTA (one per SM): the activation tile of its
// K range and the reduction scratch, and as many ring stages as fit (up to 8).
struct StreamCfg {
    int stages = 0, blocks = 0;
    uint32_t stage_bytes = 0;
    size_t smem = 0;
};

constexpr size_t kSmemPerCta = 227 * 1024;

StreamCfg plan_stream(uint32_t unit_bytes, int ng, int npg) {
    StreamCfg c;
    c.stage_bytes = (unit_bytes + 127) / 128 * 128;
    const size_t xtile = (size_t)ng * npg * 32 * 8 + (size_t)ng * kMT * 8 + 256;
    const size_t red = (size_t)2 * kNcw * 32 * 8;
    const size_t fixed = xtile + red + 1024;
    c.stages = 0;
    for (int st = 8; st >= 2; --st)
        if ((size_t)st * c.stage_bytes + ring_extra_bytes(st) + fixed <= kSmemPerCta) {
            c.stages = st;
            break;
        }
    c.smem = (size_t)c.stages * c.stage_bytes + ring_extra_bytes(c.stages) + fixed;
    return c;
}

StreamCfg gateup_cfg(const LayerArgs& a) {
    return plan_stream(stage_layout(a.H, a.gs).bytes, a.H / a.gs, a.gs / kChunk);
}

StreamCfg down_cfg(const LayerArgs& a) {
    const int kr = a.I / a.kp;
    return plan_stream(stage_layout(kr, a.gs).bytes, kr / a.gs, a.gs / kChunk);
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

size_t prep_smem(int H) { return (size_t)H * sizeof(float); }
size_t router_smem(int E) {
    return std::max((size_t)(kMaxPlanAssign + 64), (size_t)kWarps * 2 * E) * sizeof(int);
}

cudaError_t ensure_attrs(int H) {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (done[dev & 63] && H <= 16384) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)prep_smem(std::max(H, 16384)));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)router_smem(1024));
    if (e != cudaSuccess) return e;
    done[dev & 63] = true;
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


cudaError_t launch_hquant(const LayerArgs& a, const Ws& W, cudaStream_t s) {
    const int per_a = (a.I + 127) / 128;
    const int warps = W.A * per_a;
    const int wpc = kPrepThreads / 32;
    return launch(hquant_kernel, dim3((warps + wpc - 1) / wpc), dim3(kPrepThreads), 0, s, a, W);
}

template <int NPG>
cudaError_t launch_streams_npg(const LayerArgs& a, const Ws& W, cudaStream_t s) {
    StreamCfg gu = gateup_cfg(a), dn = down_cfg(a);
    cudaError_t e = finish_cfg(gateup_kernel<NPG>, gu);
    if (e != cudaSuccess) return e;
    if ((e = finish_cfg(down_kernel<NPG>, dn)) != cudaSuccess) return e;
    e = launch(gateup_kernel<NPG>, dim3(gu.blocks), dim3(kStreamCta), gu.smem, s, a, W,
               gu.stages, gu.stage_bytes);
    if (e == cudaSuccess) e = launch_hquant(a, W, s);
    if (e != cudaSuccess) return e;
    return launch(down_kernel<NPG>, dim3(dn.blocks), dim3(kStreamCta), dn.smem, s, a, W,
                  dn.stages, dn.stage_bytes);
}

cudaError_t launch_streams(const LayerArgs& a, const Ws& W, int T, cudaStream_t s) {
    (void)T;
    switch (a.gs / kChunk) {
        case 1: return launch_streams_npg<1>(a, W, s);
        case 2: return launch_streams_npg<2>(a, W, s);
        default: return launch_streams_npg<4>(a, W, s);
    }
}

cudaError_t launch_router(const LayerArgs& a, const Ws& W, int T, const float* xin,
                          cudaStream_t s) {
    const int mt = T == 1 ? 1 : kMT;
    const int nsl = (a.H + kSlice - 1) / kSlice;
    const int blocks = (a.E * nsl + kWarps - 1) / kWarps;
    return launch(router_kernel, dim3(blocks), dim3(kThreads), router_smem(a.E), s, a, W, T, mt,
                  xin, nsl);
}

// Run one layer's router + expert kernels.  The layer's input is already
// quantised in W.xq (and xin holds the router input).
cudaError_t run_layer_experts(const LayerArgs& a, const Ws& W, int T, const float* xin,
                              cudaStream_t s) {
    cudaError_t e = launch_router(a, W, T, xin, s);
    if (e != cudaSuccess) return e;
    return launch_streams(a, W, T, s);
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
    WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kPrepThreads), prep_smem(a.H), stream, a, W, T,
                       (int)P_QUANT, const_cast<float*>(x), (float*)nullptr, 0.f, 0, 0, 1),
                err);
    WB_CUDA_RET(launch_router(a, W, T, x, stream), err);
    *a_out = a;
    *w_out = W;
    return WISP_OK;
}

// gate/up + down + combine, on the plan the preceding route left in the workspace.
static WispError block_experts(const LayerArgs& a, const Ws& W, int T, const float* x, float* y,
                               cudaStream_t stream, WispErrCtx* err) {
    WB_CUDA_RET(launch_streams(a, W, T, stream), err);
    Ws Wc = W;
    Wc.prev_idx = W.topk_idx;
    Wc.prev_w = W.topk_w;
    WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kPrepThreads), prep_smem(a.H), stream, a, Wc,
                       T, (int)P_COMBINE, const_cast<float*>(x), y, 0.f, a.K, a.has_shared, a.kp),
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
    int prevK = 0, prev_sh = 0, prev_kp = 1;
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
        WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kPrepThreads), prep_smem(H), stream, a, Wp,
                           T, flags, x, (float*)nullptr, eps, prevK, prev_sh, prev_kp),
                    err);
        if (topk_idx) W.topk_idx = topk_idx + (size_t)l * T * a.K;
        if (topk_w) W.topk_w = topk_w + (size_t)l * T * a.K;
        WB_CUDA_RET(run_layer_experts(a, W, T, W.xn, stream), err);
        prevK = a.K;
        prev_sh = a.has_shared;
        prev_kp = a.kp;
        if (l == n_layers - 1) {
            Ws Wf = W;
            Wf.prev_idx = W.topk_idx;
            Wf.prev_w = W.topk_w;
            WB_CUDA_RET(launch(prep_kernel, dim3(T), dim3(kPrepThreads), prep_smem(H), stream, a,
                               Wf, T, (int)(P_COMBINE | P_RESID), x, (float*)nullptr, eps, prevK,
                               prev_sh, prev_kp),
                        err);
        }
    }
    hook_mark(stream);
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
// Mixtral-shaped layer (hidden 4096, intermediate 14336, top-2) up to T = 6;
// larger requests are rejected with WISP_ERR_INVALID_ARG before any GPU work.
// Every call on a device shares the one array, so two calls whose kernels
// overlap on the GPU (different streams, or different host threads without
// ordering) race and corrupt each other's results.  Each call clears the only
// word that must start at zero (the status word, by cudaMemsetAsync on the
// call's stream); the kernels reset their own counters.
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
