// route_common.cuh -- the gating rule shared by the decode and prefill routers.
//
// Reference: router_topk_kernel (csrc/cuda/router.cu:60-120) and its CPU twin
// cpu_router_topk (csrc/core/wisp_engine.c:520-556): p = softmax(logits + bias),
// then k passes of argmax with a strict '>' (the lowest index wins a tie,
// chosen experts are skipped), and w_j = p_j / sum of the selected p.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace wisp_route {

constexpr unsigned kAll = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kAll, v, o);
    return v;
}
// Order-preserving map of floats to unsigned integers (and back), so a
// single redux.sync finds a warp maximum.
__device__ __forceinline__ uint32_t float_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ float warp_max(float v) {
    return key_float(__reduce_max_sync(kAll, float_key(v)));
}

// Gating rules (WispMoeLayer.gating): 0 the reference's softmax(+bias); 1
// sigmoid scores, selection on score + bias, weights = selected scores
// renormalised (DeepSeek-V3 style; no reference implementation).
constexpr int kGatingSoftmax = 0;
constexpr int kGatingSigmoid = 1;

__device__ __forceinline__ float sigmoid_score(float v) { return 1.0f / (1.0f + expf(-v)); }

// Result of warp_topk held by each lane: the selections of slots `lane` and
// `lane + 32` (index -1 and weight 0 for a slot no expert could fill, or
// past K), weights already normalised.
struct TopkLane {
    int i0, i1;
    float w0, w1;
};

__device__ __forceinline__ float bias_at(const __half* b, int e) { return __half2float(b[e]); }
__device__ __forceinline__ float bias_at(const float* b, int e) { return b[e]; }

// Weights of the selected slots normalised by their sum, and the optional
// out_idx[K] / out_w[K] stores (the end of both forms of warp_topk).
__device__ __forceinline__ TopkLane topk_finish(TopkLane r, float wsum, int K, int* out_idx,
                                                float* out_w) {
    const int lane = threadIdx.x & 31;
    r.w0 = r.i0 >= 0 ? r.w0 : 0.f;
    r.w1 = r.i1 >= 0 ? r.w1 : 0.f;
    if (wsum > 0.f) {
        r.w0 = r.w0 / wsum;
        r.w1 = r.w1 / wsum;
    }
    if (out_idx) {
        if (lane < K) {
            out_idx[lane] = r.i0;
            out_w[lane] = r.w0;
        }
        if (lane + 32 < K) {
            out_idx[lane + 32] = r.i1;
            out_w[lane + 32] = r.w1;
        }
    }
    return r;
}

// Softmax gating with at most 32 experts: lane e holds expert e's
// probability in a register, so the passes need no shared memory.  The same
// operations in the same order as the general form below (max, exp, the
// butterfly sum, one division per expert, strict '>' with the lowest index
// winning), so the selections and weights are identical.
template <typename BiasT>
__device__ inline TopkLane warp_topk_small(const float* lg, const BiasT* bias, int E, int K,
                                           int* out_idx, float* out_w) {
    const int lane = threadIdx.x & 31;
    const bool live = lane < E;
    float v = -1e30f;
    if (live) {
        v = lg[lane];
        if (bias) v += bias_at(bias, lane);
    }
    const float mx = warp_max(v);
    float p = live ? expf(v - mx) : 0.f;
    const float den = warp_sum(p);
    p = live ? p / den : -1.f;
    bool taken = false;
    float wsum = 0.f;
    TopkLane r{-1, -1, 0.f, 0.f};
    for (int j = 0; j < K; ++j) {
        const bool cand = live && !taken && p > -1.f;  // (a NaN is never selected)
        const uint32_t key = float_key(cand ? p : -1.f), kmax = __reduce_max_sync(kAll, key);
        int be = (int)__reduce_min_sync(
            kAll, key == kmax && cand ? (uint32_t)lane : 0x7fffffffu);
        const float bv = key_float(kmax);
        if (bv < 0.f) be = -1;
        if (be == lane) taken = true;
        if (j == lane) {
            r.i0 = be;
            r.w0 = bv;
        } else if (j == lane + 32) {
            r.i1 = be;
            r.w1 = bv;
        }
        if (be >= 0) wsum += bv;
    }
    return topk_finish(r, wsum, K, out_idx, out_w);
}

// One token by one warp.  lg[E]: logits without the bias; bias: [E] fp16 or
// fp32 (NULL: none); sp: [E] scratch of this warp (shared memory).  The
// selected experts are tracked in a per-lane bit mask (element lane + 32 i
// is bit i, so E <= 1024) and each slot's result stays in the registers of
// lane slot % 32, so no per-thread arrays are needed.  When out_idx is not
// NULL the lanes write out_idx[K] / out_w[K].  K <= 64.
template <typename BiasT>
__device__ inline TopkLane warp_topk(const float* lg, const BiasT* bias, int E, int K, float* sp,
                                     int* out_idx, float* out_w, int gating = kGatingSoftmax) {
    const int lane = threadIdx.x & 31;
    const bool sig = gating == kGatingSigmoid;
    if (!sig && E <= 32) return warp_topk_small(lg, bias, E, K, out_idx, out_w);
    if (sig) {
        // selection scores; the weights come from the scores without the bias
        for (int e = lane; e < E; e += 32) {
            float v = sigmoid_score(lg[e]);
            if (bias) v += bias_at(bias, e);
            sp[e] = v;
        }
    } else {
        float mx = -1e30f;
        for (int e = lane; e < E; e += 32) {
            float v = lg[e];
            if (bias) v += bias_at(bias, e);
            sp[e] = v;
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
    }
    __syncwarp();
    uint32_t taken = 0u;
    float wsum = 0.f;
    TopkLane r{-1, -1, 0.f, 0.f};
    for (int j = 0; j < K; ++j) {
        float bv = sig ? -INFINITY : -1.f;
        int be = 0x7fffffff;
        int i = 0;
        for (int e = lane; e < E; e += 32, ++i) {
            const float v = sp[e];
            if (!((taken >> i) & 1u) && v > bv) {
                bv = v;
                be = e;
            }
        }
        // warp argmax: the largest value (one redux over an order-preserving
        // integer image of the floats), and among the lanes holding it the
        // lowest expert index (a second redux) -- the strict '>' rule
        const uint32_t key = float_key(bv), kmax = __reduce_max_sync(kAll, key);
        be = (int)__reduce_min_sync(kAll, key == kmax ? (uint32_t)be : 0x7fffffffu);
        bv = key_float(kmax);
        if (sig ? be == 0x7fffffff : bv < 0.f) be = -1;
        if (be >= 0 && (be & 31) == lane) taken |= 1u << (be >> 5);
        const float wv = sig ? (be >= 0 ? sigmoid_score(lg[be]) : 0.f) : bv;
        if (j == lane) {
            r.i0 = be;
            r.w0 = wv;
        } else if (j == lane + 32) {
            r.i1 = be;
            r.w1 = wv;
        }
        if (be >= 0) wsum += wv;  // every lane holds the same sum, in slot order
    }
    return topk_finish(r, wsum, K, out_idx, out_w);
}

}  // namespace wisp_route
