// quantize.cu -- the reference converter's int4 quantiser on the GPU.
//
// Restates quantize_int4 (wisp/converter/quantizer.py:46-86) bit for bit on fp32
// input: per group of `gs` consecutive elements of the row-major matrix,
//   zero  = (max + min) / 2,  scale = max((max - min) / 15, 1e-8)   (fp32)
//   q     = clamp(round_half_even((x - zero) / scale) + 8, 0, 15)
// codes packed two per byte (low nibble = even element), scale and zero stored
// as fp16 (round to nearest even).  The divisions are IEEE round-to-nearest
// (__fdiv_rn) and the rounding is rintf (round half to even), which is what
// torch computes on the CPU and on CUDA tensors, so the bytes are identical.
// Used to build large expert pools on the device (a 58-layer DeepSeek-shaped
// pool is 654 G elements) without a host round trip.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace {

constexpr unsigned kAll = 0xffffffffu;

// One warp per group; lane j handles elements j, j + 32, ... of the group, and
// the byte of each even/odd pair is assembled with a shuffle.
__global__ void __launch_bounds__(256)
quantize_int4_kernel(const float* __restrict__ w, long long n_groups, int gs,
                     uint8_t* __restrict__ packed, __half* __restrict__ scales,
                     __half* __restrict__ zeros) {
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long g = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
         g < n_groups; g += warps) {
        const float* x = w + g * gs;
        float mx = -INFINITY, mn = INFINITY;
        for (int i = lane; i < gs; i += 32) {
            const float v = x[i];
            mx = fmaxf(mx, v);
            mn = fminf(mn, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, o));
            mn = fminf(mn, __shfl_xor_sync(kAll, mn, o));
        }
        const float zero = __fdiv_rn(__fadd_rn(mx, mn), 2.0f);
        const float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), 15.0f), 1e-8f);
        for (int i0 = 0; i0 < gs; i0 += 64) {
            // lane j: elements i0 + 2j, i0 + 2j + 1 -> byte i0/2 + j
            const int i = i0 + 2 * lane;
            if (i < gs) {
                uint32_t b = 0;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float q = rintf(__fdiv_rn(__fsub_rn(x[i + h], zero), scale)) + 8.0f;
                    q = fminf(fmaxf(q, 0.0f), 15.0f);
                    b |= (uint32_t)q << (4 * h);
                }
                packed[g * (gs / 2) + i / 2] = (uint8_t)b;
            }
        }
        if (lane == 0) {
            scales[g] = __float2half_rn(scale);
            zeros[g] = __float2half_rn(zero);
        }
    }
}

}  // namespace

extern "C" WispError wisp_quantize_int4(const float* w, int rows, int cols, int group_size,
                                        uint8_t* packed, void* scales, void* zeros,
                                        cudaStream_t stream, WispErrCtx* err) {
    const long long n = (long long)rows * cols;
    if (!w || !packed || !scales || !zeros || rows <= 0 || cols <= 0 || group_size <= 0 ||
        group_size % 2 || n % group_size) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "quantize_int4: bad arguments (rows %d cols %d group %d; the element count "
                   "must be a multiple of an even group size)",
                   rows, cols, group_size);
        return WISP_ERR_INVALID_ARG;
    }
    const long long groups = n / group_size;
    const int sms = wb::sm_count();
    const long long want = (groups + 7) / 8;
    const int blocks = (int)(want < 32LL * sms ? want : 32LL * sms);
    quantize_int4_kernel<<<blocks, 256, 0, stream>>>(w, groups, group_size, packed,
                                                     static_cast<__half*>(scales),
                                                     static_cast<__half*>(zeros));
    WB_CUDA_RET(cudaGetLastError(), err);
    return WISP_OK;
}
