// dense_ffn.h -- launchers of the fp16-dense SwiGLU FFN (dense_ffn.cu), shared
// by the fused block (shared expert stored fp16-dense) and the engine
// (router-less dense-MLP layers).  Not part of the ABI.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace wb {

// gate/up [inter, H], down [H, inter] fp16, 16-byte aligned, inter and H
// multiples of 8.
bool dense_ffn_shape_ok(const void* gate, const void* up, const void* down, int inter, int H);

// y[t*ldy + :H] = down . (silu(gate . x_t) * (up . x_t)) for t < T, with h
// [T, inter] fp32 scratch.  Two PDL launches on `s`; `mark` (optional) is
// called with `s` before each.
cudaError_t launch_dense_ffn(const __half* gate, const __half* up, const __half* down, int inter,
                             int H, const float* x, int ldx, float* h, float* y, int ldy, int T,
                             cudaStream_t s, void (*mark)(cudaStream_t) = nullptr);

// y = rmsnorm(x; w, eps) row by row (T rows of H), double sum of squares.
cudaError_t launch_rmsnorm_rows(const float* x, const __half* w, float* y, int H, float eps,
                                int T, cudaStream_t s);

// x += d (n floats).
cudaError_t launch_add_rows(float* x, const float* d, size_t n, cudaStream_t s);

}  // namespace wb
