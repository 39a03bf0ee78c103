// decoder.cu -- the decoder step around the MoE block: the token embedding,
// GQA attention over an fp16 KV cache (its projections, rotary embedding and
// cache append), and the logits.  With the fused MoE block these make the
// engine's wisp_decode_one a whole device-side decoder step.
//
// Reference (the CPU twins the parity tests pin against):
//   decode_step          csrc/core/wisp_engine.c:1537-1595
//   run_attention (GQA)  csrc/core/wisp_engine.c:1328-1348
//   cpu_attention        csrc/core/wisp_engine.c:465-505  (two-pass softmax)
//   cpu_rope             csrc/core/wisp_engine.c:446-460  (neox pairs i, i+d/2)
//   cpu_kv_append        csrc/core/wisp_engine.c:507-518  (fp16 cache)
//   cpu_embed_lookup     csrc/core/wisp_engine.c:439-443
//   cpu_rmsnorm          csrc/core/wisp_engine.c:415-422  (double sum of squares)
//   cpu_gemv_f16         csrc/core/wisp_engine.c:389-400
//
// Kernels (all HBM- or latency-bound at one token; every one waits on its
// predecessor with griddepcontrol.wait before reading its output):
//   embed_kernel        x = fp32(embed[token])
//   proj_split_kernel   q / k / v (with the RMSNorm, the rotation and the fp16
//                       cache stores) and o_proj (with the residual) on the
//                       tensor cores, each 16-row tile split over column slices
//                       (see the comment at the kernel)
//   attn_part_kernel    flash-decoding: CTA (kv head, up to 8 of its query heads,
//                       a chunk of positions): scores with one lane per position
//                       (the K row read once for all the CTA's heads), the
//                       chunk's max and sum, and P.V with one thread per output
//                       dimension (V rows read coalesced)
//   attn_merge_kernel   the chunks' (max, sum, output) merged per head
//   rows_gemv_kernel    y = W x or y += W x, warp per row (lm_head; o_proj of
//                       shapes the split kernel does not take)
//   qkv_rope_kernel     q / k / v warp per rotary row pair (shapes the split
//                       kernel does not take)

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "dense_ffn.h"
#include "internal.h"

namespace wb {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kAttnHeads = 8;     // query heads per attention CTA
constexpr int kAttnChunk = 256;   // positions per attention CTA (at least)
constexpr int kMaxHeadDim = 576;  // k_dim / v_dim limit of the attention kernels

__device__ __forceinline__ void dec_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dec_pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Warm L2 with `bytes` (a multiple of 16) at the 16-byte aligned p: issued
// before griddepcontrol.wait for weights and cache rows this kernel will
// read, so their DRAM reads overlap the previous kernel's tail.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float dot8(const uint4& wv, const float* x) {
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(w2[i]);
        acc = fmaf(f.x, x[2 * i], acc);
        acc = fmaf(f.y, x[2 * i + 1], acc);
    }
    return acc;
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

// x[i] = fp32(table[token][i])
__global__ void __launch_bounds__(kDecThreads)
embed_kernel(const __half* __restrict__ table, int token, float* __restrict__ x, int H) {
    dec_pdl_wait();
    dec_pdl_launch();
    const int i = blockIdx.x * kDecThreads + threadIdx.x;
    if (i < H) x[i] = __half2float(table[(size_t)token * H + i]);
}

// y = x * rsqrt(mean(x^2) + eps) * w into shared memory (w NULL: ones), the
// sum of squares in double as cpu_rmsnorm accumulates it.
__device__ void norm_to_smem(const float* __restrict__ x, const __half* __restrict__ w, int H,
                             float eps, float* xs) {
    __shared__ double red[kDecWarps];
    __shared__ float s_scale;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = x[i];
        xs[i] = v;
        ss += (double)v * (double)v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double v = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v += red[i];
        s_scale = (float)(1.0 / sqrt(v / (double)H + (double)eps));
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        xs[i] = xs[i] * sc * (w ? __half2float(w[i]) : 1.0f);
    __syncthreads();
}

// One warp's dot products of rows r0 and r1 of W [*, H] with xs (shared).
__device__ __forceinline__ float2 row_pair_dot(const __half* __restrict__ W, int r0, int r1, int H,
                                               const float* xs) {
    const int lane = threadIdx.x & 31;
    const uint4* a = reinterpret_cast<const uint4*>(W + (size_t)r0 * H);
    const uint4* b = reinterpret_cast<const uint4*>(W + (size_t)r1 * H);
    // kLoads 16-byte loads of each row in flight per lane before any is used
    constexpr int kLoads = 4;
    const int n = H / 8;
    float s0 = 0.f, s1 = 0.f;
    for (int c0 = lane; c0 < n; c0 += 32 * kLoads) {
        uint4 wa[kLoads], wb[kLoads];
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int c = c0 + 32 * u;
            wa[u] = c < n ? __ldg(a + c) : make_uint4(0, 0, 0, 0);
            wb[u] = c < n ? __ldg(b + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int c = min(c0 + 32 * u, n - 1);
            s0 += dot8(wa[u], xs + c * 8);
            s1 += dot8(wb[u], xs + c * 8);
        }
    }
    return make_float2(warp_sum(s0), warp_sum(s1));
}

// Rotation of the pair (a, b) = (v[i], v[i + d/2]) at position pos (cpu_rope).
__device__ __forceinline__ float2 rope_pair(float a, float b, int i, int d, int pos, float theta) {
    const float freq = powf(theta, -2.0f * (float)i / (float)d);
    const float ang = (float)pos * freq;
    float s, c;
    sincosf(ang, &s, &c);
    return make_float2(a * c - b * s, b * c + a * s);
}

// Heads 0..nh-1: q (rotated, fp32 into q_out); nh..nh+nkv-1: k (rotated,
// fp16 into K at pos); then v (fp16 into V at pos).  CTA: head blockIdx.y,
// rotary pairs [blockIdx.x * kDecWarps, ...), one pair per warp.  Dynamic
// shared memory: H floats (the normalised input).
__global__ void __launch_bounds__(kDecThreads)
qkv_rope_kernel(const float* __restrict__ x, const __half* __restrict__ norm_w, float eps,
                const __half* __restrict__ Wq, const __half* __restrict__ Wk,
                const __half* __restrict__ Wv, float* __restrict__ q_out, __half* __restrict__ Kc,
                __half* __restrict__ Vc, int pos, int nh, int nkv, int hd, int H, float theta) {
    extern __shared__ __align__(16) float xs[];
    dec_pdl_wait();
    dec_pdl_launch();
    norm_to_smem(x, norm_w, H, eps, xs);
    const int head = blockIdx.y, half = hd / 2;
    const int i = blockIdx.x * kDecWarps + (threadIdx.x >> 5);
    if (i >= half) return;
    const int lane = threadIdx.x & 31;
    if (head < nh) {
        const float2 v = row_pair_dot(Wq, head * hd + i, head * hd + i + half, H, xs);
        if (lane == 0) {
            const float2 r = rope_pair(v.x, v.y, i, hd, pos, theta);
            q_out[head * hd + i] = r.x;
            q_out[head * hd + i + half] = r.y;
        }
    } else if (head < nh + nkv) {
        const int kh = head - nh;
        const float2 v = row_pair_dot(Wk, kh * hd + i, kh * hd + i + half, H, xs);
        if (lane == 0) {
            const float2 r = rope_pair(v.x, v.y, i, hd, pos, theta);
            __half* dst = Kc + ((size_t)pos * nkv + kh) * hd;
            dst[i] = __float2half_rn(r.x);
            dst[i + half] = __float2half_rn(r.y);
        }
    } else {
        const int vh = head - nh - nkv;
        const float2 v = row_pair_dot(Wv, vh * hd + i, vh * hd + i + half, H, xs);
        if (lane == 0) {
            __half* dst = Vc + ((size_t)pos * nkv + vh) * hd;
            dst[i] = __float2half_rn(v.x);
            dst[i + half] = __float2half_rn(v.y);
        }
    }
}

// acc += x . w over 8 elements, in element order (the reference's sequential
// sum, one rounding per fused multiply-add).
__device__ __forceinline__ float dot8_chain(const uint4& wv, const float* x, float acc) {
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(w2[i]);
        acc = fmaf(x[2 * i], f.x, acc);
        acc = fmaf(x[2 * i + 1], f.y, acc);
    }
    return acc;
}

// Attention of up to kAttnHeads query heads sharing kv head `kvh` over the
// positions [t0, t0 + chunk) of the cache.  Grid: x = nkv * hblocks (kv
// head, block of its query heads), y = chunk index.  K [seq][nkv][k_dim],
// V [seq][nkv][v_stride] fp16 (V == K with v_stride = k_dim: the value is
// the first v_dim dims of the key).  One chunk: the normalised output goes
// to out [nh][v_dim]; several: the chunk's max, sum and unnormalised output
// go to part_ml [nh][nsplit][2] / part_o [nh][nsplit][v_dim] for the merge.
// Dynamic shared memory: kAttnHeads * (k_dim + chunk) floats.
__global__ void __launch_bounds__(kDecThreads)
attn_part_kernel(const float* __restrict__ q, const __half* __restrict__ Kc,
                 const __half* __restrict__ Vc, float* __restrict__ out,
                 float* __restrict__ part_o, float* __restrict__ part_ml, int seq, int nh,
                 int nkv, int k_dim, int v_dim, int v_stride, float scale, int chunk) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[kDecWarps][kAttnHeads];
    __shared__ float s_m[kAttnHeads], s_l[kAttnHeads];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int group = nh / nkv, hblocks = (group + kAttnHeads - 1) / kAttnHeads;
    const int kvh = blockIdx.x / hblocks, hb = blockIdx.x % hblocks;
    const int h0 = kvh * group + hb * kAttnHeads;
    const int ng = min(kAttnHeads, group - hb * kAttnHeads);
    const int nsplit = gridDim.y, split = blockIdx.y;
    const int t0 = split * chunk, tn = min(seq, t0 + chunk) - t0;
    float* qs = sm;                        // [kAttnHeads][k_dim]
    float* sc = sm + kAttnHeads * k_dim;   // [kAttnHeads][chunk]
    if (hb == 0) {  // one CTA of the kv head's query-head blocks warms the chunk's rows
        // (value rows only when they are 16-byte aligned pieces of whole 16 bytes)
        const bool v_ok = Vc != Kc && v_stride % 8 == 0 && v_dim % 8 == 0 &&
                          (reinterpret_cast<uintptr_t>(Vc) & 15u) == 0;
        for (int t = tid; t < tn; t += kDecThreads) {
            prefetch_l2(Kc + ((size_t)(t0 + t) * nkv + kvh) * k_dim, (uint32_t)k_dim * 2);
            if (v_ok)
                prefetch_l2(Vc + ((size_t)(t0 + t) * nkv + kvh) * v_stride, (uint32_t)v_dim * 2);
        }
    }
    dec_pdl_wait();
    dec_pdl_launch();
    for (int i = tid; i < ng * k_dim; i += kDecThreads) qs[i] = q[(size_t)h0 * k_dim + i];
    __syncthreads();
    // scores: one thread per position, the key row read once for all heads
    float mloc[kAttnHeads];
#pragma unroll
    for (int g = 0; g < kAttnHeads; ++g) mloc[g] = -1e30f;
    for (int t = tid; t < tn; t += kDecThreads) {
        const uint4* kr = reinterpret_cast<const uint4*>(Kc + ((size_t)(t0 + t) * nkv + kvh) * k_dim);
        float acc[kAttnHeads];
#pragma unroll
        for (int g = 0; g < kAttnHeads; ++g) acc[g] = 0.f;
        constexpr int kLoads = 8;  // the key row's 16-byte pieces in flight together
        for (int c0 = 0; c0 < k_dim / 8; c0 += kLoads) {
            uint4 kv[kLoads];
#pragma unroll
            for (int u = 0; u < kLoads; ++u)
                kv[u] = c0 + u < k_dim / 8 ? __ldg(kr + c0 + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                if (c0 + u >= k_dim / 8) break;
#pragma unroll
                for (int g = 0; g < kAttnHeads; ++g)
                    if (g < ng) acc[g] = dot8_chain(kv[u], qs + g * k_dim + (c0 + u) * 8, acc[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < kAttnHeads; ++g)
            if (g < ng) {
                const float s = acc[g] * scale;
                sc[g * chunk + t] = s;
                mloc[g] = fmaxf(mloc[g], s);
            }
    }
#pragma unroll
    for (int g = 0; g < kAttnHeads; ++g) {
        const float m = warp_max(mloc[g]);
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
    if (tid < kAttnHeads) {
        float m = -1e30f;
        for (int w = 0; w < kDecWarps; ++w) m = fmaxf(m, red[w][tid]);
        s_m[tid] = m;
    }
    __syncthreads();
    float lloc[kAttnHeads];
#pragma unroll
    for (int g = 0; g < kAttnHeads; ++g) lloc[g] = 0.f;
    for (int t = tid; t < tn; t += kDecThreads) {
#pragma unroll
        for (int g = 0; g < kAttnHeads; ++g)
            if (g < ng) {
                const float p = expf(sc[g * chunk + t] - s_m[g]);
                sc[g * chunk + t] = p;
                lloc[g] += p;
            }
    }
#pragma unroll
    for (int g = 0; g < kAttnHeads; ++g) {
        const float l = warp_sum(lloc[g]);
        if (lane == 0) red[warp][g] = l;
    }
    __syncthreads();
    if (tid < kAttnHeads) {
        float l = 0.f;
        for (int w = 0; w < kDecWarps; ++w) l += red[w][tid];
        s_l[tid] = l;
    }
    __syncthreads();
    // P.V: one thread per (head, output dimension); V rows read coalesced
    for (int i = tid; i < ng * v_dim; i += kDecThreads) {
        const int g = i / v_dim, d = i - g * v_dim;
        const float* p = sc + g * chunk;
        const __half* vcol = Vc + (size_t)kvh * v_stride + d;
        const size_t vstep = (size_t)nkv * v_stride;
        float acc = 0.f;
#pragma unroll 8
        for (int t = 0; t < tn; ++t) acc = fmaf(p[t], __half2float(vcol[(size_t)(t0 + t) * vstep]), acc);
        const int h = h0 + g;
        if (nsplit == 1) {
            const float l = s_l[g];
            out[(size_t)h * v_dim + d] = acc * (1.f / (l > 0.f ? l : 1.f));
        } else {
            part_o[((size_t)h * nsplit + split) * v_dim + d] = acc;
        }
    }
    if (nsplit > 1 && tid < ng) {
        part_ml[((size_t)(h0 + tid) * nsplit + split) * 2] = s_m[tid];
        part_ml[((size_t)(h0 + tid) * nsplit + split) * 2 + 1] = s_l[tid];
    }
}

// out[h] = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M) over the chunks.
__global__ void __launch_bounds__(kDecThreads)
attn_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                  float* __restrict__ out, int nsplit, int v_dim) {
    extern __shared__ float s_e[];  // [nsplit] e^(m_i - M)
    __shared__ float s_inv;
    const int h = blockIdx.x;
    dec_pdl_wait();
    dec_pdl_launch();
    const float* ml = part_ml + (size_t)h * nsplit * 2;
    if (threadIdx.x < 32) {
        float M = -1e30f;
        for (int i = threadIdx.x; i < nsplit; i += 32) M = fmaxf(M, ml[2 * i]);
        M = warp_max(M);
        float L = 0.f;
        for (int i = threadIdx.x; i < nsplit; i += 32) {
            const float e = expf(ml[2 * i] - M);
            s_e[i] = e;
            L += ml[2 * i + 1] * e;
        }
        L = warp_sum(L);
        if (threadIdx.x == 0) s_inv = 1.f / (L > 0.f ? L : 1.f);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int d = threadIdx.x; d < v_dim; d += kDecThreads) {
        const float* po = part_o + (size_t)h * nsplit * v_dim + d;
        float acc = 0.f;
#pragma unroll 8
        for (int i = 0; i < nsplit; ++i) acc = fmaf(po[(size_t)i * v_dim], s_e[i], acc);
        out[(size_t)h * v_dim + d] = acc * inv;
    }
}

// ------------------------------------------------------------------------
// q / k / v and o projections on the tensor cores, split over the columns.
// A CTA computes one 16-row tile (one rotary tile pair for q / k / v) over a
// 1/J slice of the columns: the layer's weights spread over many small CTAs,
// each warp with a single round of 16-byte loads in flight.  mma.sync
// m16n8k16 (fp16 x fp16 -> fp32) takes the weights as A; the input vector is
// split into fp16 hi and lo parts (x ~= hi + lo to about 2^-22) in columns 0
// and 1 of B, so the products carry fp32-level precision and row r's result
// is column 0 + column 1; the 16 rows of a tile share every input fragment.
// Each lane loads 16 contiguous bytes of its two rows per 32-column block;
// the K order inside a block is permuted identically for the weights and the
// input (a dot product is order-free).  The J partial tiles are summed in
// slice order by the last CTA to finish (a counter per tile, left at zero),
// which also applies the rotation and the cache stores, or the residual.
// With `norm`, each CTA computes cpu_rmsnorm's scale over the whole input
// and applies it on the way in.
// ------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
                 : "memory");
    return old;
}

struct ProjArgs {
    const __half* W[3];    // q, k, v projections (QKV) or the matrix
    const float* x;        // fp32 input [K] (written by the previous kernel)
    const __half* norm_w;  // with `norm`: the input is rmsnorm(x; norm_w, eps) (NULL: ones)
    float eps;
    int norm;
    float* part;    // [tiles][J][32] partial rows
    int* counters;  // [tiles], zero on entry, left zero
    int K, J, rows;
    int nh, nkv, hd;  // QKV
    float* y;         // rows mode: y[r] += W[r] . x
    float* q_out;     // QKV outputs
    __half* Kc;
    __half* Vc;
    int pos;
    float theta;
};

// 8 consecutive inputs at k (normalised when `norm`: (x * scale) * w, as
// cpu_rmsnorm rounds it) as the fp16 hi or lo part: this lane's B pieces.
__device__ __forceinline__ uint4 x_frag(const float* __restrict__ x, int k, bool lo, bool norm,
                                        float scale, const __half* __restrict__ w) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(x + k));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(x + k + 4));
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (norm) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = v[i] * scale * (w ? __half2float(w[k + i]) : 1.0f);
    }
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half h0 = __float2half_rn(v[2 * i]), h1 = __float2half_rn(v[2 * i + 1]);
        if (lo) {
            h0 = __float2half_rn(v[2 * i] - __half2float(h0));
            h1 = __float2half_rn(v[2 * i + 1] - __half2float(h1));
        }
        const __half2 h2 = __halves2half2(h0, h1);
        r[i] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
}

template <bool QKV>
__global__ void __launch_bounds__(kDecThreads)
proj_split_kernel(ProjArgs P) {
    __shared__ float part[kDecWarps][2][32][4];
    __shared__ int s_last;
    __shared__ double s_red[kDecWarps];
    __shared__ float s_scale;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int j = blockIdx.x, u = blockIdx.y, J = P.J, K = P.K;
    const __half* W = P.W[0];
    int rA, rB = 0, rows;
    if (QKV) {
        const int per = P.hd / 32, head = u / per, t = u - head * per, half = P.hd / 2;
        int r0;
        if (head < P.nh) {
            r0 = head * P.hd;
        } else if (head < P.nh + P.nkv) {
            W = P.W[1];
            r0 = (head - P.nh) * P.hd;
        } else {
            W = P.W[2];
            r0 = (head - P.nh - P.nkv) * P.hd;
        }
        rA = r0 + t * 16;
        rB = r0 + half + t * 16;
        rows = r0 + P.hd;
    } else {
        rA = u * 16;
        rows = P.rows;
    }
    constexpr int kT = QKV ? 2 : 1;
    constexpr int kU = 4;
    const int ks = K / J, kc0 = j * ks;
    const int kw = ks / kDecWarps, k0 = kc0 + warp * kw, k1 = k0 + kw;
    const int ra[2] = {min(rA + g, rows - 1), min(rB + g, rows - 1)};
    const int rb[2] = {min(rA + g + 8, rows - 1), min(rB + g + 8, rows - 1)};
    uint4 wa[kT][kU], wb[kT][kU];
    // this lane's 16-byte weight pieces of kU 32-column blocks from kb on
    auto load_w = [&](int kb) {
#pragma unroll
        for (int tt = 0; tt < kT; ++tt)
#pragma unroll
            for (int v = 0; v < kU; ++v) {
                const bool in = kb + 32 * v < k1;
                const size_t c = (size_t)(kb + 32 * v) + 8 * q;
                wa[tt][v] = in ? __ldg(reinterpret_cast<const uint4*>(W + (size_t)ra[tt] * K + c))
                               : make_uint4(0, 0, 0, 0);
                wb[tt][v] = in ? __ldg(reinterpret_cast<const uint4*>(W + (size_t)rb[tt] * K + c))
                               : make_uint4(0, 0, 0, 0);
            }
    };
    if (kw > 32 * kU && threadIdx.x < 16 * kT) {  // a slice longer than one round: warm it
        const int r = threadIdx.x < 16 ? rA + threadIdx.x : rB + threadIdx.x - 16;
        if (r < rows) prefetch_l2(W + (size_t)r * K + kc0, (uint32_t)ks * 2);
    }
    // the weights do not depend on the previous kernel: the first round of loads
    // is in flight through the dependency wait and the RMSNorm
    load_w(k0);
    dec_pdl_wait();
    dec_pdl_launch();
    float scale = 1.f;
    if (P.norm) {
        double ss = 0.0;
        for (int i = threadIdx.x; i < K; i += kDecThreads) {
            const double v = (double)__ldcg(P.x + i);
            ss += v * v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int i = 0; i < kDecWarps; ++i) t += s_red[i];
            s_scale = (float)(1.0 / sqrt(t / (double)K + (double)P.eps));
        }
        __syncthreads();
        scale = s_scale;
    }
    float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int kb = k0; kb < k1; kb += 32 * kU) {
        if (kb != k0) load_w(kb);
#pragma unroll
        for (int v = 0; v < kU; ++v) {
            if (kb + 32 * v >= k1) break;
            const uint4 xv = g < 2 ? x_frag(P.x, kb + 32 * v + 8 * q, g == 1, P.norm != 0, scale,
                                            P.norm_w)
                                   : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int tt = 0; tt < kT; ++tt) {
                mma_f16(d[tt], wa[tt][v].x, wb[tt][v].x, wa[tt][v].y, wb[tt][v].y, xv.x, xv.y);
                mma_f16(d[tt], wa[tt][v].z, wb[tt][v].z, wa[tt][v].w, wb[tt][v].w, xv.z, xv.w);
            }
        }
    }
#pragma unroll
    for (int tt = 0; tt < kT; ++tt)
#pragma unroll
        for (int i = 0; i < 4; ++i) part[warp][tt][lane][i] = d[tt][i];
    __syncthreads();
    // this slice's rows, summed over the warps in order, to the slice record
    if (warp == 0 && q == 0) {
#pragma unroll
        for (int tt = 0; tt < kT; ++tt) {
            float a = 0.f, b = 0.f;
            for (int w = 0; w < kDecWarps; ++w) {
                a += part[w][tt][lane][0] + part[w][tt][lane][1];
                b += part[w][tt][lane][2] + part[w][tt][lane][3];
            }
            float* dst = P.part + ((size_t)u * J + j) * 32 + tt * 16;
            dst[g] = a;
            dst[g + 8] = b;
        }
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomic_add_acq_rel(P.counters + u, 1) == J - 1;
    __syncthreads();
    if (!s_last) return;
    // the last slice: the tile's rows over all slices in order, then the epilogue
    if (threadIdx.x < 16) {
        const int i = threadIdx.x;
        float a = 0.f, b = 0.f;
        for (int jj = 0; jj < J; ++jj) {
            const float* src = P.part + ((size_t)u * J + jj) * 32;
            a += __ldcg(src + i);
            if (QKV) b += __ldcg(src + 16 + i);
        }
        if (QKV) {
            const int per = P.hd / 32, head = u / per, t = u - head * per, half = P.hd / 2;
            const int pi = t * 16 + i;  // rotary pair (pi, pi + half)
            if (head < P.nh) {
                const float2 r = rope_pair(a, b, pi, P.hd, P.pos, P.theta);
                P.q_out[head * P.hd + pi] = r.x;
                P.q_out[head * P.hd + pi + half] = r.y;
            } else if (head < P.nh + P.nkv) {
                const float2 r = rope_pair(a, b, pi, P.hd, P.pos, P.theta);
                __half* dst = P.Kc + ((size_t)P.pos * P.nkv + (head - P.nh)) * P.hd;
                dst[pi] = __float2half_rn(r.x);
                dst[pi + half] = __float2half_rn(r.y);
            } else {
                __half* dst = P.Vc + ((size_t)P.pos * P.nkv + (head - P.nh - P.nkv)) * P.hd;
                dst[pi] = __float2half_rn(a);
                dst[pi + half] = __float2half_rn(b);
            }
        } else if (rA + i < rows) {
            P.y[rA + i] += a;
        }
    }
    if (threadIdx.x == 0) P.counters[u] = 0;  // ready for the next call
}

// y[r] (= or +=) W[r] . x for rows r, one warp per row; x staged in dynamic
// shared memory (cols floats).  cols % 8 == 0, W rows 16-byte aligned.
template <bool ACC>
__global__ void __launch_bounds__(kDecThreads)
rows_gemv_kernel(const __half* __restrict__ W, const float* __restrict__ x, float* __restrict__ y,
                 int rows, int cols) {
    extern __shared__ __align__(16) float xs[];
    dec_pdl_wait();
    dec_pdl_launch();
    for (int i = threadIdx.x; i < cols; i += kDecThreads) xs[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * kDecWarps + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint4* w = reinterpret_cast<const uint4*>(W + (size_t)r * cols);
    constexpr int kLoads = 8;  // 16-byte loads in flight per lane
    const int n = cols / 8;
    float s = 0.f;
    for (int c0 = lane; c0 < n; c0 += 32 * kLoads) {
        uint4 wv[kLoads];
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            const int c = c0 + 32 * u;
            wv[u] = c < n ? __ldg(w + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kLoads; ++u) s += dot8(wv[u], xs + min(c0 + 32 * u, n - 1) * 8);
    }
    s = warp_sum(s);
    if (lane == 0) y[r] = ACC ? y[r] + s : s;
}

// fp32 -> fp16 rows into the cache at pos (cpu_kv_append)
__global__ void __launch_bounds__(kDecThreads)
kv_append_kernel(__half* __restrict__ K, __half* __restrict__ V, const float* __restrict__ k,
                 const float* __restrict__ v, int pos, int nk, int nv) {
    dec_pdl_wait();
    dec_pdl_launch();
    const int i = blockIdx.x * kDecThreads + threadIdx.x;
    if (i < nk) K[(size_t)pos * nk + i] = __float2half_rn(k[i]);
    if (V && v && i < nv) V[(size_t)pos * nv + i] = __float2half_rn(v[i]);
}

// cpu_rope on x [n_heads][head_stride], window [rope_off, rope_off + rope_dim)
__global__ void __launch_bounds__(kDecThreads)
rope_kernel(float* __restrict__ x, int n_heads, int head_stride, int rope_off, int rope_dim,
            int pos, float theta) {
    dec_pdl_wait();
    dec_pdl_launch();
    const int half = rope_dim / 2;
    const int j = blockIdx.x * kDecThreads + threadIdx.x;
    if (j >= n_heads * half) return;
    const int h = j / half, i = j - h * half;
    float* v = x + (size_t)h * head_stride + rope_off;
    const float2 r = rope_pair(v[i], v[i + half], i, rope_dim, pos, theta);
    v[i] = r.x;
    v[i + half] = r.y;
}

}  // namespace
}  // namespace wb

namespace wb {
namespace {

// Positions per attention chunk: at least kAttnChunk, and at least twice a
// partial result (v_dim + 2 floats), so the reference launcher's score
// scratch ([n_heads][seq] floats) holds every chunk's partials.
int attn_chunk(int v_dim) { return std::max(kAttnChunk, 2 * (v_dim + 2)); }

// Chunk of the fused decode (its own workspace, sized for chunks of at least
// kMinChunk): enough chunks for about two CTAs per SM, 32-position multiples,
// at most kMaxChunk positions (shared memory).
constexpr int kMinChunk = 32, kMaxChunk = 4096;
int decode_chunk(int seq, int ctas_per_chunk) {
    const int want = std::max(1, (2 * sm_count() + ctas_per_chunk - 1) / ctas_per_chunk);
    int c = (seq + want - 1) / want;
    c = (std::max(c, kMinChunk) + 31) / 32 * 32;
    return std::min(c, kMaxChunk);
}
size_t attn_smem(int k_dim, int chunk) { return (size_t)kAttnHeads * (k_dim + chunk) * sizeof(float); }

// Dynamic shared memory above the 48 KB default needs the kernel's opt-in
// (per call: cheap, and right on whichever device is current).
bool set_smem_once(const void* kern, size_t bytes) {
    if (bytes <= 48 * 1024) return true;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
           cudaSuccess;
}

}  // namespace

cudaError_t launch_attention(const float* q, const __half* K, const __half* V, float* out,
                             float* part_o, float* part_ml, int seq, int nh, int nkv, int k_dim,
                             int v_dim, int v_stride, float scale, int chunk, cudaStream_t s) {
    const int nsplit = (seq + chunk - 1) / chunk;
    const int group = nh / nkv, hblocks = (group + kAttnHeads - 1) / kAttnHeads;
    const size_t smem = attn_smem(k_dim, chunk);
    if (!set_smem_once(reinterpret_cast<const void*>(attn_part_kernel), smem))
        return cudaErrorInvalidConfiguration;
    cudaError_t e = launch_pdl(attn_part_kernel, dim3(nkv * hblocks, nsplit), dim3(kDecThreads), smem,
                               s, q, K, V, out, part_o, part_ml, seq, nh, nkv, k_dim, v_dim,
                               v_stride, scale, chunk);
    if (e != cudaSuccess || nsplit == 1) return e;
    return launch_pdl(attn_merge_kernel, dim3(nh), dim3(kDecThreads), (size_t)nsplit * 4, s,
                      (const float*)part_o, (const float*)part_ml, out, nsplit, v_dim);
}

}  // namespace wb

using namespace wb;

namespace {
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Column slices of a split projection: the most of 4 / 2 / 1 that leaves each
// warp a whole number of 32-column blocks.
int split_of(int K) {
    for (int J = 4; J > 1; J /= 2)
        if (K % (256 * J) == 0) return J;
    return 1;
}

struct AttnWs {
    float *q, *attn, *part_ml, *part_o, *pq, *po;
    int* counters;
    bool split;          // tensor-core split projections (else warp-per-row kernels)
    int jq, jo, uq, uo;  // slices and tiles of the q/k/v and o projections
    size_t bytes;
};
AttnWs attn_ws_layout(const WispAttnLayer* L, int max_seq, void* base) {
    const int nh = L->n_heads, nkv = L->n_kv_heads, hd = L->head_dim, H = L->hidden;
    const int nsplit = (max_seq + kMinChunk - 1) / kMinChunk;
    auto up = [](size_t v) { return (v + 63) / 64 * 64; };
    AttnWs w{};
    w.split = H % 256 == 0 && hd % 32 == 0 && (nh * hd) % 256 == 0;
    w.jq = split_of(H);
    w.jo = split_of(nh * hd);
    w.uq = (nh + 2 * nkv) * (hd / 32);
    w.uo = (H + 15) / 16;
    size_t o = 0;
    char* b = static_cast<char*>(base);
    w.q = reinterpret_cast<float*>(b + o);
    o += up((size_t)nh * hd * 4);
    w.attn = reinterpret_cast<float*>(b + o);
    o += up((size_t)nh * hd * 4);
    w.part_ml = reinterpret_cast<float*>(b + o);
    o += up((size_t)nh * nsplit * 2 * 4);
    w.part_o = reinterpret_cast<float*>(b + o);
    o += up((size_t)nh * nsplit * hd * 4);
    w.pq = reinterpret_cast<float*>(b + o);
    o += up((size_t)w.uq * w.jq * 32 * 4);
    w.po = reinterpret_cast<float*>(b + o);
    o += up((size_t)w.uo * w.jo * 32 * 4);
    w.counters = reinterpret_cast<int*>(b + o);
    o += up((size_t)(w.uq + w.uo) * 4);
    w.bytes = o;
    return w;
}
}  // namespace

// Launchers with the reference's signatures (void, as in csrc/cuda/*.cu).
extern "C" void wisp_gpu_embed_lookup(const wisp_half* table, int token, float* x, int hidden,
                                      cudaStream_t s) {
    launch_pdl(embed_kernel, dim3((hidden + kDecThreads - 1) / kDecThreads), dim3(kDecThreads), 0,
               s, reinterpret_cast<const __half*>(table), token, x, hidden);
}

extern "C" void wisp_gpu_rope(float* x, int n_heads, int head_stride, int rope_off, int rope_dim,
                              int pos, float theta, cudaStream_t s) {
    const int n = n_heads * (rope_dim / 2);
    if (n <= 0) return;
    launch_pdl(rope_kernel, dim3((n + kDecThreads - 1) / kDecThreads), dim3(kDecThreads), 0, s, x,
               n_heads, head_stride, rope_off, rope_dim, pos, theta);
}

extern "C" void wisp_gpu_kv_append(wisp_half* K, wisp_half* V, const float* k, const float* v,
                                   int pos, int kv_heads, int k_dim, int v_dim, cudaStream_t s) {
    const int nk = kv_heads * k_dim, nv = V && v ? kv_heads * v_dim : 0;
    const int n = std::max(nk, nv);
    if (n <= 0) return;
    launch_pdl(kv_append_kernel, dim3((n + kDecThreads - 1) / kDecThreads), dim3(kDecThreads), 0, s,
               reinterpret_cast<__half*>(K), reinterpret_cast<__half*>(V), k, v, pos, nk, nv);
}

extern "C" void wisp_gpu_attention(const float* q, const wisp_half* Kcache, const wisp_half* Vcache,
                                   float* out, float* score_scratch, int seq_len, int n_heads,
                                   int kv_heads, int k_dim, int v_dim, float scale,
                                   cudaStream_t s) {
    if (seq_len <= 0 || n_heads <= 0 || kv_heads <= 0 || n_heads % kv_heads || k_dim % 8 ||
        k_dim > kMaxHeadDim || v_dim > kMaxHeadDim || !al16(Kcache))
        return;
    const int chunk = attn_chunk(v_dim);
    const int nsplit = (seq_len + chunk - 1) / chunk;
    float* part_ml = score_scratch;
    float* part_o = score_scratch + (size_t)n_heads * nsplit * 2;
    const bool same = Vcache == Kcache || Vcache == nullptr;
    launch_attention(q, reinterpret_cast<const __half*>(Kcache),
                     reinterpret_cast<const __half*>(same ? Kcache : Vcache), out, part_o, part_ml,
                     seq_len, n_heads, kv_heads, k_dim, v_dim, same ? k_dim : v_dim, scale, chunk,
                     s);
}

extern "C" size_t wisp_attn_workspace_bytes(const WispAttnLayer* layer, int max_seq) {
    if (!layer || max_seq <= 0) return 0;
    return attn_ws_layout(layer, max_seq, nullptr).bytes;
}

extern "C" WispError wisp_attn_decode(const WispAttnLayer* L, float* x, wisp_half* k_cache,
                                      wisp_half* v_cache, int pos, int max_seq, void* workspace,
                                      size_t workspace_bytes, cudaStream_t s, WispErrCtx* err) {
    if (!L || !x || !k_cache || !v_cache || !workspace || pos < 0 || pos >= max_seq ||
        !L->q_proj || !L->k_proj || !L->v_proj || !L->o_proj) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "attn_decode: NULL argument or pos %d outside [0, %d)",
                   pos, max_seq);
        return WISP_ERR_INVALID_ARG;
    }
    const int H = L->hidden, nh = L->n_heads, nkv = L->n_kv_heads, hd = L->head_dim;
    if (H <= 0 || H % 8 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || hd % 16 ||
        hd > kMaxHeadDim || (nh * hd) % 8) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "attn_decode: unsupported shape hidden=%d heads=%d kv_heads=%d head_dim=%d "
                   "(hidden a multiple of 8, heads a multiple of kv_heads, head_dim a multiple of "
                   "16 up to %d)",
                   H, nh, nkv, hd, kMaxHeadDim);
        return WISP_ERR_INVALID_ARG;
    }
    if (!al16(x) || !al16(k_cache) || !al16(v_cache) || !al16(L->q_proj) || !al16(L->k_proj) ||
        !al16(L->v_proj) || !al16(L->o_proj) || !al16(workspace)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "attn_decode: pointers must be 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    const AttnWs w = attn_ws_layout(L, max_seq, workspace);
    if (workspace_bytes < w.bytes) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "attn_decode: workspace %zu bytes, need %zu",
                   workspace_bytes, w.bytes);
        return WISP_ERR_INVALID_ARG;
    }
    const __half* Kc = reinterpret_cast<const __half*>(k_cache);
    const __half* Vc = reinterpret_cast<const __half*>(v_cache);
    // q / k / v: tensor-core split-K projections when the shapes split evenly
    // (H and the head width multiples of 256, head_dim of 32), else warp-per-row
    // fused multiply-adds
    if (w.split) {
        ProjArgs P{};
        P.W[0] = reinterpret_cast<const __half*>(L->q_proj);
        P.W[1] = reinterpret_cast<const __half*>(L->k_proj);
        P.W[2] = reinterpret_cast<const __half*>(L->v_proj);
        P.x = x;
        P.norm = 1;
        P.norm_w = reinterpret_cast<const __half*>(L->input_norm);
        P.eps = L->rms_eps;
        P.part = w.pq;
        P.counters = w.counters;
        P.K = H;
        P.J = w.jq;
        P.nh = nh;
        P.nkv = nkv;
        P.hd = hd;
        P.q_out = w.q;
        P.Kc = reinterpret_cast<__half*>(k_cache);
        P.Vc = reinterpret_cast<__half*>(v_cache);
        P.pos = pos;
        P.theta = L->rope_theta;
        WB_CUDA_RET(launch_pdl(proj_split_kernel<true>, dim3(w.jq, w.uq), dim3(kDecThreads), 0, s, P),
                    err);
    } else {
        if (!set_smem_once(reinterpret_cast<const void*>(qkv_rope_kernel), (size_t)H * 4)) {
            WB_SET_ERR(err, WISP_ERR_CUDA, "attn_decode: shared memory attribute refused");
            return WISP_ERR_CUDA;
        }
        WB_CUDA_RET(launch_pdl(qkv_rope_kernel, dim3((hd / 2 + kDecWarps - 1) / kDecWarps, nh + 2 * nkv),
                               dim3(kDecThreads), (size_t)H * 4, s, (const float*)x,
                               reinterpret_cast<const __half*>(L->input_norm), L->rms_eps,
                               reinterpret_cast<const __half*>(L->q_proj),
                               reinterpret_cast<const __half*>(L->k_proj),
                               reinterpret_cast<const __half*>(L->v_proj), w.q,
                               reinterpret_cast<__half*>(k_cache),
                               reinterpret_cast<__half*>(v_cache), pos, nh, nkv, hd, H,
                               L->rope_theta),
                    err);
    }
    const int hblocks = (nh / nkv + kAttnHeads - 1) / kAttnHeads;
    WB_CUDA_RET(launch_attention(w.q, Kc, Vc, w.attn, w.part_o, w.part_ml, pos + 1, nh, nkv, hd, hd,
                                 hd, 1.0f / sqrtf((float)hd), decode_chunk(pos + 1, nkv * hblocks),
                                 s),
                err);
    if (w.split) {
        ProjArgs P{};
        P.W[0] = reinterpret_cast<const __half*>(L->o_proj);
        P.x = w.attn;
        P.part = w.po;
        P.counters = w.counters + w.uq;
        P.K = nh * hd;
        P.J = w.jo;
        P.rows = H;
        P.y = x;
        WB_CUDA_RET(launch_pdl(proj_split_kernel<false>, dim3(w.jo, w.uo), dim3(kDecThreads), 0, s, P),
                    err);
    } else {
        if (!set_smem_once(reinterpret_cast<const void*>(rows_gemv_kernel<true>), (size_t)nh * hd * 4)) {
            WB_SET_ERR(err, WISP_ERR_CUDA, "attn_decode: shared memory attribute refused");
            return WISP_ERR_CUDA;
        }
        WB_CUDA_RET(launch_pdl(rows_gemv_kernel<true>, dim3((H + kDecWarps - 1) / kDecWarps),
                               dim3(kDecThreads), (size_t)nh * hd * 4, s,
                               reinterpret_cast<const __half*>(L->o_proj), (const float*)w.attn, x,
                               H, nh * hd),
                    err);
    }
    return WISP_OK;
}

extern "C" WispError wisp_lm_head_forward(const wisp_half* final_norm, const wisp_half* lm_head,
                                          const float* x, float* logits, int vocab, int hidden,
                                          float eps, void* workspace, size_t workspace_bytes,
                                          cudaStream_t s, WispErrCtx* err) {
    if (!lm_head || !x || !logits || !workspace || vocab <= 0 || hidden <= 0 || hidden % 8 ||
        workspace_bytes < (size_t)hidden * sizeof(float) || !al16(lm_head) || !al16(workspace)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "lm_head_forward: bad arguments (hidden a multiple of 8, workspace of hidden "
                   "floats, 16-byte aligned weights)");
        return WISP_ERR_INVALID_ARG;
    }
    float* xn = static_cast<float*>(workspace);
    if (!set_smem_once(reinterpret_cast<const void*>(rows_gemv_kernel<false>), (size_t)hidden * 4)) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "lm_head_forward: shared memory attribute refused");
        return WISP_ERR_CUDA;
    }
    WB_CUDA_RET(launch_rmsnorm_rows(x, reinterpret_cast<const __half*>(final_norm), xn, hidden, eps, 1,
                                    s),
                err);
    WB_CUDA_RET(launch_pdl(rows_gemv_kernel<false>, dim3((vocab + kDecWarps - 1) / kDecWarps),
                           dim3(kDecThreads), (size_t)hidden * 4, s,
                           reinterpret_cast<const __half*>(lm_head), (const float*)xn, logits, vocab,
                           hidden),
                err);
    return WISP_OK;
}
