// route_common.cuh -- the gating rule shared by the decode and prefill routers.
//
// Reference: router_topk_kernel (csrc/cuda/router.cu:60-120) and its CPU twin
// cpu_router_topk (csrc/core/wisp_engine.c:520-556): p = softmax(logits + bias),
// then k passes of argmax with a strict '>' (the lowest index wins a tie,
// chosen experts are skipped), and w_j = p_j / sum of the selected p.
#pragma once

#include <cuda_fp16.h>

namespace wisp_route {

constexpr unsigned kAll = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kAll, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kAll, v, o));
    return v;
}

// Gating rules (WispMoeLayer.gating): 0 the reference's softmax(+bias); 1
// sigmoid scores, selection on score + bias, weights = selected scores
// renormalised (DeepSeek-V3 style; no reference implementation).
constexpr int kGatingSoftmax = 0;
constexpr int kGatingSigmoid = 1;

__device__ __forceinline__ float sigmoid_score(float v) { return 1.0f / (1.0f + expf(-v)); }

// One token by one warp.  lg[E]: logits without the bias; sp/staken: [E]
// scratch of this warp (shared memory).  Lane 0 writes out_idx[K] / out_w[K]
// (-1 / 0 for a slot no expert could fill).  K <= 64.
__device__ inline void warp_topk(const float* lg, const __half* bias, int E, int K, float* sp,
                                 int* staken, int* out_idx, float* out_w,
                                 int gating = kGatingSoftmax) {
    const int lane = threadIdx.x & 31;
    const bool sig = gating == kGatingSigmoid;
    if (sig) {
        // selection scores; the weights come from the scores without the bias
        for (int e = lane; e < E; e += 32) {
            float v = sigmoid_score(lg[e]);
            if (bias) v += __half2float(bias[e]);
            sp[e] = v;
            staken[e] = 0;
        }
    } else {
        float mx = -1e30f;
        for (int e = lane; e < E; e += 32) {
            float v = lg[e];
            if (bias) v += __half2float(bias[e]);
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
    }
    __syncwarp();
    float wsum = 0.f;
    float wsel[64];
    int isel[64];
    for (int j = 0; j < K; ++j) {
        float bv = sig ? -INFINITY : -1.f;
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
            const float ov = __shfl_xor_sync(kAll, bv, o);
            const int oe = __shfl_xor_sync(kAll, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (sig ? be == 0x7fffffff : bv < 0.f) be = -1;
        if (lane == 0 && be >= 0) staken[be] = 1;
        __syncwarp();
        const float wv = sig ? (be >= 0 ? sigmoid_score(lg[be]) : 0.f) : bv;
        wsel[j] = wv;
        isel[j] = be;
        if (be >= 0) wsum += wv;
    }
    if (lane == 0) {
        for (int j = 0; j < K; ++j) {
            float wj = isel[j] >= 0 ? wsel[j] : 0.f;
            if (wsum > 0.f) wj = wj / wsum;
            out_idx[j] = isel[j];
            out_w[j] = wj;
        }
    }
}

}  // namespace wisp_route
