// ref_launchers.cu -- the reference's kernel-launcher ABI for the MoE path,
// same C signatures as csrc/core/wisp_engine.h:549-612, written for sm_100a.
//
// These are the building blocks the reference engine composes one launch at
// a time (router, dequant, fp16 GEMV, SwiGLU, combine, RMSNorm, residual).
// The engine in this library does not use them on its hot path -- it runs
// the fused kernels of moe_kernels.cu -- but a caller built against the
// reference launchers links against these unchanged.
//
// Differences from the reference that a caller can observe: none in the
// contract.  Internally the GEMVs are warp-per-row with 16-byte loads and
// shuffle reductions, the dequant writes 8 fp16 per thread, and the router
// keeps its device staging per device (the reference's process-wide buffer,
// router.cu:152-158, is unsafe across devices).

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "internal.h"

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// dot of an fp16 row with an fp32 vector, one warp
__device__ __forceinline__ float row_dot(const __half* row, const float* x, int cols) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    const bool vec = ((cols & 7) == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    if (vec) {
        for (int c = lane * 8; c < cols; c += 256) {
            uint4 wv = *reinterpret_cast<const uint4*>(row + c);
            const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
            float4 a = *reinterpret_cast<const float4*>(x + c);
            float4 b = *reinterpret_cast<const float4*>(x + c + 4);
            float2 f0 = __half22float2(w2[0]), f1 = __half22float2(w2[1]);
            float2 f2 = __half22float2(w2[2]), f3 = __half22float2(w2[3]);
            acc = fmaf(f0.x, a.x, acc);
            acc = fmaf(f0.y, a.y, acc);
            acc = fmaf(f1.x, a.z, acc);
            acc = fmaf(f1.y, a.w, acc);
            acc = fmaf(f2.x, b.x, acc);
            acc = fmaf(f2.y, b.y, acc);
            acc = fmaf(f3.x, b.z, acc);
            acc = fmaf(f3.y, b.w, acc);
        }
    } else {
        for (int c = lane; c < cols; c += 32) acc = fmaf(__half2float(row[c]), x[c], acc);
    }
    return wsum(acc);
}

__global__ void gemv_rows_kernel(const __half* W, const float* x, float* y, int rows, int cols) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float v = row_dot(W + (size_t)r * cols, x, cols);
    if ((threadIdx.x & 31) == 0) y[r] = v;
}

__global__ void gemv_t_kernel(const __half* W, const float* x, float* y, int rows, int cols) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    float acc = 0.f;
    for (int r = 0; r < rows; ++r) acc = fmaf(__half2float(W[(size_t)r * cols + c]), x[r], acc);
    y[c] = acc;
}

__global__ void swiglu_ffn_kernel(const __half* Wg, const __half* Wu, const float* x, float* h,
                                  int inter, int cols) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= inter) return;
    float g = row_dot(Wg + (size_t)r * cols, x, cols);
    float u = row_dot(Wu + (size_t)r * cols, x, cols);
    if ((threadIdx.x & 31) == 0) h[r] = g / (1.0f + expf(-g)) * u;
}

__global__ void rmsnorm_kernel(const float* x, const __half* w, float* y, int n, float eps) {
    __shared__ float red[32];
    __shared__ float s_scale;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = wsum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = wsum(v);
        if (threadIdx.x == 0) s_scale = 1.0f / sqrtf(v / (float)n + eps);
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * sc * __half2float(w[i]);
}

__global__ void residual_kernel(float* x, const float* d, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += d[i];
}

__global__ void swiglu_kernel(const float* g, const float* u, float* o, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float gv = g[i];
        o[i] = gv / (1.0f + expf(-gv)) * u[i];
    }
}

__global__ void scale_accum_kernel(float* acc, const float* x, float w, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) acc[i] = fmaf(w, x[i], acc[i]);
}

// router: logits (warp per expert), then one warp does softmax + top-k
__global__ void router_logits_kernel(const __half* W, const __half* bias, const float* x,
                                     float* logits, int E, int H) {
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= E) return;
    float v = row_dot(W + (size_t)e * H, x, H);
    if ((threadIdx.x & 31) == 0) logits[e] = v + (bias ? __half2float(bias[e]) : 0.f);
}

__global__ void router_select_kernel(const float* logits, int E, int K, int* out_idx,
                                     float* out_w) {
    extern __shared__ float sp[];
    int* taken = reinterpret_cast<int*>(sp + E);
    const int lane = threadIdx.x;
    float mx = -1e30f;
    for (int e = lane; e < E; e += 32) {
        sp[e] = logits[e];
        taken[e] = 0;
        mx = fmaxf(mx, sp[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    float den = 0.f;
    for (int e = lane; e < E; e += 32) {
        sp[e] = expf(sp[e] - mx);
        den += sp[e];
    }
    den = wsum(den);
    for (int e = lane; e < E; e += 32) sp[e] = sp[e] / den;
    __syncwarp();
    float sum = 0.f;
    for (int j = 0; j < K; ++j) {
        float bv = -1.f;
        int be = 0x7fffffff;
        for (int e = lane; e < E; e += 32)
            if (!taken[e] && sp[e] > bv) {
                bv = sp[e];
                be = e;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(kFull, bv, o);
            int oe = __shfl_xor_sync(kFull, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (bv < 0.f) be = -1;
        if (lane == 0) {
            out_idx[j] = be;
            out_w[j] = be >= 0 ? bv : 0.f;
            if (be >= 0) taken[be] = 1;
        }
        if (be >= 0) sum += bv;
        __syncwarp();
    }
    if (lane == 0 && sum > 0.f)
        for (int j = 0; j < K; ++j) out_w[j] = out_w[j] / sum;
}

// int4 -> fp16, 8 elements per thread (one packed 32-bit word)
__global__ void dequant8_kernel(const uint32_t* packed, const __half* scales, const __half* zeros,
                                __half* out, long long n8, int gs) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    uint32_t w = packed[i];
    long long e0 = i * 8;
    __align__(16) __half o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        long long g = (e0 + k) / gs;
        float s = __half2float(scales[g]), z = __half2float(zeros[g]);
        int code = (w >> (4 * k)) & 0xF;
        o[k] = __float2half_rn(fmaf((float)(code - 8), s, z));
    }
    *reinterpret_cast<uint4*>(out + e0) = *reinterpret_cast<uint4*>(o);
}

__global__ void dequant1_kernel(const uint8_t* packed, const __half* scales, const __half* zeros,
                                __half* out, int n, int gs) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint8_t b = packed[i >> 1];
    int code = (i & 1) ? (b >> 4) : (b & 0xF);
    int g = i / gs;
    out[i] = __float2half_rn(fmaf((float)(code - 8), __half2float(scales[g]),
                                  __half2float(zeros[g])));
}

int rows_grid(int rows, int warps) { return (rows + warps - 1) / warps; }

struct RouterStaging {
    int* idx = nullptr;
    float* w = nullptr;
};

}  // namespace

extern "C" void wisp_gpu_gemv_f16(const wisp_half* W, const float* x, float* y, int rows,
                                  int cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    gemv_rows_kernel<<<rows_grid(rows, 8), 256, 0, s>>>((const __half*)W, x, y, rows, cols);
}

extern "C" void wisp_gpu_gemv_t_f16(const wisp_half* W, const float* x, float* y, int rows,
                                    int cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    gemv_t_kernel<<<(cols + 255) / 256, 256, 0, s>>>((const __half*)W, x, y, rows, cols);
}

extern "C" void wisp_gpu_rmsnorm(const float* x, const wisp_half* w, float* y, int n, float eps,
                                 cudaStream_t s) {
    if (n <= 0) return;
    rmsnorm_kernel<<<1, 1024, 0, s>>>(x, (const __half*)w, y, n, eps);
}

extern "C" void wisp_gpu_residual_add(float* x, const float* d, int n, cudaStream_t s) {
    if (n <= 0) return;
    residual_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, d, n);
}

extern "C" void wisp_gpu_swiglu(const float* g, const float* u, float* o, int n, cudaStream_t s) {
    if (n <= 0) return;
    swiglu_kernel<<<(n + 255) / 256, 256, 0, s>>>(g, u, o, n);
}

extern "C" void wisp_gpu_swiglu_ffn(const wisp_half* Wg, const wisp_half* Wu, const float* x,
                                    float* h, int inter, int cols, cudaStream_t s) {
    if (inter <= 0 || cols <= 0) return;
    swiglu_ffn_kernel<<<rows_grid(inter, 8), 256, 0, s>>>((const __half*)Wg, (const __half*)Wu,
                                                          x, h, inter, cols);
}

extern "C" void wisp_gpu_scale_accum(float* acc, const float* x, float w, int n, cudaStream_t s) {
    if (n <= 0) return;
    scale_accum_kernel<<<(n + 255) / 256, 256, 0, s>>>(acc, x, w, n);
}

extern "C" void wisp_gpu_router_topk(const wisp_half* W, const wisp_half* bias, const float* x,
                                     float* logits_scratch, int n_experts, int hidden, int top_k,
                                     int* out_idx, float* out_w, cudaStream_t s) {
    constexpr int kMaxTopK = 64;
    if (n_experts <= 0 || top_k <= 0) return;
    if (top_k > kMaxTopK) top_k = kMaxTopK;
    static std::mutex mu;
    static RouterStaging staging[64];
    int dev = 0;
    cudaGetDevice(&dev);
    RouterStaging* st;
    {
        std::lock_guard<std::mutex> g(mu);
        st = &staging[dev & 63];
        if (!st->idx) {
            if (cudaMalloc(&st->idx, kMaxTopK * sizeof(int)) != cudaSuccess ||
                cudaMalloc(&st->w, kMaxTopK * sizeof(float)) != cudaSuccess) {
                st->idx = nullptr;
                return;
            }
        }
    }
    router_logits_kernel<<<rows_grid(n_experts, 8), 256, 0, s>>>(
        (const __half*)W, (const __half*)bias, x, logits_scratch, n_experts, hidden);
    router_select_kernel<<<1, 32, (size_t)n_experts * 8, s>>>(logits_scratch, n_experts, top_k,
                                                             st->idx, st->w);
    cudaMemcpyAsync(out_idx, st->idx, (size_t)top_k * sizeof(int), cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(out_w, st->w, (size_t)top_k * sizeof(float), cudaMemcpyDeviceToHost, s);
}

extern "C" cudaError_t launch_dequant_expert(const uint8_t* d_packed, const wisp_half* d_scales,
                                             const wisp_half* d_zeros, wisp_half* d_output,
                                             int n_elements, int group_size,
                                             cudaStream_t stream) {
    if (n_elements <= 0 || group_size <= 0) return cudaErrorInvalidValue;
    const bool vec = (n_elements % 8 == 0) &&
                     ((reinterpret_cast<uintptr_t>(d_packed) & 3) == 0) &&
                     ((reinterpret_cast<uintptr_t>(d_output) & 15) == 0);
    if (vec) {
        long long n8 = n_elements / 8;
        dequant8_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, stream>>>(
            reinterpret_cast<const uint32_t*>(d_packed), (const __half*)d_scales,
            (const __half*)d_zeros, (__half*)d_output, n8, group_size);
    } else {
        dequant1_kernel<<<(n_elements + 255) / 256, 256, 0, stream>>>(
            d_packed, (const __half*)d_scales, (const __half*)d_zeros, (__half*)d_output,
            n_elements, group_size);
    }
    return cudaGetLastError();
}

extern "C" cudaError_t async_load_expert(const uint8_t* h_packed, const wisp_half* h_scales,
                                         const wisp_half* h_zeros, uint8_t* d_packed_tmp,
                                         wisp_half* d_scales_tmp, wisp_half* d_zeros_tmp,
                                         wisp_half* d_output, int n_elements, int group_size,
                                         cudaStream_t stream) {
    if (n_elements <= 0 || group_size <= 0) return cudaErrorInvalidValue;
    const size_t n_groups = ((size_t)n_elements + group_size - 1) / group_size;
    const size_t packed_bytes = ((size_t)n_elements + 1) / 2;
    cudaError_t e = cudaMemcpyAsync(d_packed_tmp, h_packed, packed_bytes, cudaMemcpyHostToDevice,
                                    stream);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(d_scales_tmp, h_scales, n_groups * 2, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(d_zeros_tmp, h_zeros, n_groups * 2, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    return launch_dequant_expert(d_packed_tmp, d_scales_tmp, d_zeros_tmp, d_output, n_elements,
                                 group_size, stream);
}
