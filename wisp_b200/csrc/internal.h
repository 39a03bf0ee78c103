// internal.h -- shared helpers of the wisp_b200 sources (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <utility>

#include "wisp_b200.h"

#define WB_SET_ERR(ctx, c, ...)                                   \
    do {                                                          \
        if (ctx) {                                                \
            (ctx)->code = (c);                                    \
            snprintf((ctx)->message, sizeof((ctx)->message),      \
                     __VA_ARGS__);                                \
            (ctx)->file = __FILE__;                               \
            (ctx)->line = __LINE__;                               \
        }                                                         \
    } while (0)

#define WB_CUDA_RET(call, ctx)                                            \
    do {                                                                  \
        cudaError_t _e = (call);                                          \
        if (_e != cudaSuccess) {                                          \
            WB_SET_ERR(ctx, WISP_ERR_CUDA, "CUDA error: %s (%s)",         \
                       cudaGetErrorString(_e), #call);                    \
            return WISP_ERR_CUDA;                                         \
        }                                                                 \
    } while (0)

namespace wb {

// Number of SMs of the current device (cached per device id).
int sm_count();

// Zero n_words 32-bit words at p (the status word and counters of a
// workspace) on `stream` with a one-CTA kernel launched like every other
// kernel of this library (programmatic dependent launch, griddepcontrol.wait
// before the stores).  A cudaMemsetAsync is not a grid that a following
// kernel's griddepcontrol.wait waits for, so it is not used for state that
// the next kernels read.
cudaError_t launch_zero_words(int* p, int n_words, cudaStream_t stream);

// Launch `kern` with programmatic dependent launch enabled, so its prologue
// may overlap the tail of the previous kernel on `stream`; the kernel must
// call griddepcontrol.wait before touching its predecessor's outputs.
// `cluster` > 1 launches thread-block clusters of that many CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, int cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int n = 1;
    if (cluster > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)cluster;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t stream, Args&&... args) {
    return launch_pdl_cluster(kern, grid, block, smem, stream, 1, std::forward<Args>(args)...);
}

}  // namespace wb
