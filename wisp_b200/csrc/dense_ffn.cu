// dense_ffn.cu -- the fp16-dense SwiGLU FFN of the reference's model directories.
//
// The reference converter stores a layer's shared expert, and the whole MLP of
// a router-less ("dense MLP") layer, as fp16 tensors layers.{i}.shared.{gate,
// up,down} in the dense safetensors file (gate/up [si, H], down [H, si];
// loader wisp_engine.c:1748-1757).  run_moe adds the shared expert with
// weight 1 before the routed experts (wisp_engine.c:1443-1450); run_dense_mlp
// is the same FFN alone (:1524-1534):
//
//   h = silu(Wg x) * (Wu x),   y = Wd h        (fp16 weights, fp32 math)
//
// These are HBM-bound GEMVs for the decode batch sizes: one warp per output
// row streams the row with 16-byte loads, up to 8 tokens share each load (the
// tokens' input slice is staged in shared memory per 1024 columns), and a
// shuffle reduction finishes each row.  Launched with programmatic dependent
// launch like the rest of the block: every kernel waits (griddepcontrol.wait)
// before reading its input.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "dense_ffn.h"
#include "internal.h"

namespace wb {
namespace {

constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kDenseThreads = 256;
constexpr int kDenseRows = kDenseThreads / 32;  // one output row per warp
constexpr int kDenseTok = 8;                    // tokens per pass over the weights
constexpr int kDenseCols = 1024;                // input columns staged per step

__device__ __forceinline__ void dense_pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void dense_pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fma8(float& acc, const uint4& wv, const float4& a,
                                     const float4& b) {
    const __half2* w2 = reinterpret_cast<const __half2*>(&wv);
    float2 f = __half22float2(w2[0]);
    acc = fmaf(f.x, a.x, acc);
    acc = fmaf(f.y, a.y, acc);
    f = __half22float2(w2[1]);
    acc = fmaf(f.x, a.z, acc);
    acc = fmaf(f.y, a.w, acc);
    f = __half22float2(w2[2]);
    acc = fmaf(f.x, b.x, acc);
    acc = fmaf(f.y, b.y, acc);
    f = __half22float2(w2[3]);
    acc = fmaf(f.x, b.z, acc);
    acc = fmaf(f.y, b.w, acc);
}

// out[t*ldo + r] = PAIR ? silu(W0[r].x_t) * (W1[r].x_t) : W0[r].x_t for rows r
// of this CTA and tokens t < T.  W0/W1 [rows, cols] fp16 row-major; x [T, ldx]
// fp32.  cols % 8 == 0; rows, x and out 16-byte aligned (checked on the host).
template <bool PAIR>
__global__ void __launch_bounds__(kDenseThreads)
dense_rows_kernel(const __half* __restrict__ W0, const __half* __restrict__ W1,
                  const float* __restrict__ x, int ldx, float* __restrict__ out, int ldo,
                  int rows, int cols, int T) {
    __shared__ __align__(16) float xs[kDenseTok][kDenseCols];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = blockIdx.x * kDenseRows + warp;
    dense_pdl_wait();
    dense_pdl_launch();
    const __half* row0 = W0 + (size_t)(r < rows ? r : 0) * cols;
    const __half* row1 = PAIR ? W1 + (size_t)(r < rows ? r : 0) * cols : nullptr;
    for (int t0 = 0; t0 < T; t0 += kDenseTok) {
        const int tt = min(kDenseTok, T - t0);
        float a0[kDenseTok], a1[kDenseTok];
#pragma unroll
        for (int t = 0; t < kDenseTok; ++t) a0[t] = a1[t] = 0.f;
        for (int c0 = 0; c0 < cols; c0 += kDenseCols) {
            const int cw = min(kDenseCols, cols - c0);
            __syncthreads();  // the previous step's readers are done
            for (int i = tid; i < tt * (kDenseCols / 4); i += kDenseThreads) {
                const int t = i / (kDenseCols / 4), j = (i % (kDenseCols / 4)) * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (j < cw)
                    v = *reinterpret_cast<const float4*>(x + (size_t)(t0 + t) * ldx + c0 + j);
                *reinterpret_cast<float4*>(&xs[t][j]) = v;
            }
            __syncthreads();
            if (r < rows) {
                uint4 w0[kDenseCols / 256], w1[kDenseCols / 256];
#pragma unroll
                for (int i = 0; i < kDenseCols / 256; ++i) {
                    const int c = i * 256 + lane * 8;
                    w0[i] = c < cw ? __ldg(reinterpret_cast<const uint4*>(row0 + c0 + c))
                                   : make_uint4(0, 0, 0, 0);
                    if (PAIR)
                        w1[i] = c < cw ? __ldg(reinterpret_cast<const uint4*>(row1 + c0 + c))
                                       : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int i = 0; i < kDenseCols / 256; ++i) {
                    const int c = i * 256 + lane * 8;
#pragma unroll
                    for (int t = 0; t < kDenseTok; ++t) {
                        if (t < tt) {
                            const float4 a = *reinterpret_cast<const float4*>(&xs[t][c]);
                            const float4 b = *reinterpret_cast<const float4*>(&xs[t][c + 4]);
                            fma8(a0[t], w0[i], a, b);
                            if (PAIR) fma8(a1[t], w1[i], a, b);
                        }
                    }
                }
            }
        }
        if (r < rows) {
#pragma unroll
            for (int t = 0; t < kDenseTok; ++t) {
                if (t >= tt) break;
                float g = a0[t], u = a1[t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    g += __shfl_xor_sync(kFullMask, g, o);
                    if (PAIR) u += __shfl_xor_sync(kFullMask, u, o);
                }
                if (lane == 0)
                    out[(size_t)(t0 + t) * ldo + r] = PAIR ? g / (1.0f + expf(-g)) * u : g;
            }
        }
    }
}

// RMSNorm of T rows (one CTA per row): y = x * rsqrt(mean(x^2) + eps) * w, the
// sum of squares accumulated in double as the reference's CPU path does
// (cpu_rmsnorm, wisp_engine.c:415-422).  w may be NULL (ones).
__global__ void __launch_bounds__(kDenseThreads)
rmsnorm_rows_kernel(const float* __restrict__ x, const __half* __restrict__ w,
                    float* __restrict__ y, int H, float eps) {
    __shared__ double red[kDenseThreads / 32];
    __shared__ float s_scale;
    dense_pdl_wait();
    dense_pdl_launch();
    const float* xr = x + (size_t)blockIdx.x * H;
    float* yr = y + (size_t)blockIdx.x * H;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += kDenseThreads) ss += (double)xr[i] * (double)xr[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFullMask, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double v = 0.0;
        for (int i = 0; i < kDenseThreads / 32; ++i) v += red[i];
        s_scale = (float)(1.0 / sqrt(v / (double)H + (double)eps));
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < H; i += kDenseThreads)
        yr[i] = xr[i] * sc * (w ? __half2float(w[i]) : 1.0f);
}

// x += d over n elements.
__global__ void __launch_bounds__(kDenseThreads)
add_rows_kernel(float* __restrict__ x, const float* __restrict__ d, size_t n) {
    dense_pdl_wait();
    dense_pdl_launch();
    for (size_t i = (size_t)blockIdx.x * kDenseThreads + threadIdx.x; i < n;
         i += (size_t)gridDim.x * kDenseThreads)
        x[i] += d[i];
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool dense_ffn_shape_ok(const void* gate, const void* up, const void* down, int inter, int H) {
    return gate && up && down && inter > 0 && H > 0 && inter % 8 == 0 && H % 8 == 0 &&
           al16(gate) && al16(up) && al16(down);
}

cudaError_t launch_dense_ffn(const __half* gate, const __half* up, const __half* down, int inter,
                             int H, const float* x, int ldx, float* h, float* y, int ldy, int T,
                             cudaStream_t s, void (*mark)(cudaStream_t)) {
    if (mark) mark(s);
    cudaError_t e = launch_pdl(dense_rows_kernel<true>, dim3((inter + kDenseRows - 1) / kDenseRows),
                               dim3(kDenseThreads), 0, s, gate, up, x, ldx, h, inter, inter, H, T);
    if (e != cudaSuccess) return e;
    if (mark) mark(s);
    return launch_pdl(dense_rows_kernel<false>, dim3((H + kDenseRows - 1) / kDenseRows),
                      dim3(kDenseThreads), 0, s, down, (const __half*)nullptr, (const float*)h,
                      inter, y, ldy, H, inter, T);
}

cudaError_t launch_rmsnorm_rows(const float* x, const __half* w, float* y, int H, float eps,
                                int T, cudaStream_t s) {
    return launch_pdl(rmsnorm_rows_kernel, dim3(T), dim3(kDenseThreads), 0, s, x, w, y, H, eps);
}

cudaError_t launch_add_rows(float* x, const float* d, size_t n, cudaStream_t s) {
    const size_t blocks = std::min<size_t>((n + kDenseThreads - 1) / kDenseThreads, 148 * 8);
    return launch_pdl(add_rows_kernel, dim3((unsigned)std::max<size_t>(blocks, 1)),
                      dim3(kDenseThreads), 0, s, x, d, n);
}

}  // namespace wb

using namespace wb;

extern "C" size_t wisp_dense_ffn_workspace_bytes(int inter, int T) {
    return (size_t)(inter > 0 ? inter : 0) * (size_t)(T > 0 ? T : 0) * sizeof(float);
}

extern "C" WispError wisp_dense_ffn_forward(const wisp_half* gate, const wisp_half* up,
                                            const wisp_half* down, int inter, int hidden,
                                            const float* x, float* y, int T, void* workspace,
                                            size_t workspace_bytes, cudaStream_t stream,
                                            WispErrCtx* err) {
    if (!dense_ffn_shape_ok(gate, up, down, inter, hidden)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "dense_ffn: NULL or unaligned weights, or inter=%d / hidden=%d not positive "
                   "multiples of 8",
                   inter, hidden);
        return WISP_ERR_INVALID_ARG;
    }
    if (T <= 0 || !x || !y || x == y || !al16(x) || !al16(y) || !workspace || !al16(workspace) ||
        workspace_bytes < wisp_dense_ffn_workspace_bytes(inter, T)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "dense_ffn: T=%d, x/y NULL, aliased or unaligned, or workspace %zu < %zu", T,
                   workspace_bytes, wisp_dense_ffn_workspace_bytes(inter, T));
        return WISP_ERR_INVALID_ARG;
    }
    WB_CUDA_RET(launch_dense_ffn(reinterpret_cast<const __half*>(gate),
                                 reinterpret_cast<const __half*>(up),
                                 reinterpret_cast<const __half*>(down), inter, hidden, x, hidden,
                                 static_cast<float*>(workspace), y, hidden, T, stream),
                err);
    return WISP_OK;
}
