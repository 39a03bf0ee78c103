// expert_layout.cu -- the tiled device layout of an int4 expert blob.
//
// On disk an expert is a WISP .bin blob (writer: wisp/converter/partitioner.py
// :45-89; parser: csrc/core/wisp_engine.c:268-303): a 120-byte header, then per
// matrix (gate [I,H], up [I,H], down [H,I]) the packed codes of every row, the
// fp16 scales and the fp16 zeros, each row-major.
//
// The fused kernels stream a matrix in blocks of 8 rows, and their tensor-core
// fragments read, for one quant group, the same 8 rows side by side.  In the
// tiled layout every 8-row block is one contiguous run, stored in that order:
//
//   block b (rows 8b .. 8b+7), G = cols / gs groups per row:
//     packed[g][j]  g < G, j < 8 : the gs/2 code bytes of row 8b+j, group g
//     sz[g][j]      g < G, j < 8 : scale and zero of row 8b+j, group g (2 x fp16)
//   block bytes = 8 * cols / 2 + 8 * G * 4 = 4 * cols + 32 * G
//
// so one block is a single bulk copy, any range of groups of a block is two
// (codes, then scale/zero pairs), and a warp's reads of one group of 8 rows
// touch one contiguous 4*gs-byte run (no shared-memory bank conflicts).  A
// matrix's region keeps its place and size in the blob (packed + scales + zeros
// bytes), and the header is the .bin header with version = 2, so the section
// sizes and offsets parse exactly as before.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace {

constexpr uint32_t kTiledVersion = 2;

// One thread per 32-bit output word of a matrix: first the code words of
// every block, then the (scale, zero) words.
__global__ void tile_matrix_kernel(const uint32_t* __restrict__ src_packed,
                                   const uint16_t* __restrict__ src_scales,
                                   const uint16_t* __restrict__ src_zeros,
                                   uint8_t* __restrict__ dst, int rows, int cols, int gs,
                                   const uint32_t* header_src, uint32_t* header_dst) {
    const long long G = cols / gs;
    const long long block_bytes = 4LL * cols + 32LL * G;
    const long long code_words = (long long)rows * cols / 8;
    const long long sz_words = (long long)rows * G;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (header_dst && tid < 30) header_dst[tid] = tid == 1 ? kTiledVersion : header_src[tid];
    const int wpg = gs / 8;  // code words per (row, group)
    for (long long w = tid; w < code_words; w += stride) {
        const long long b = w / cols, r = w - b * cols;  // a block holds `cols` code words
        const long long g = r / gs, rem = r - g * gs;    // a group of a block: gs words
        const long long j = rem / wpg, i = rem - j * wpg;
        const long long row = 8 * b + j;
        const uint32_t v = src_packed[(row * (cols / 2) + g * (gs / 2)) / 4 + i];
        *reinterpret_cast<uint32_t*>(dst + b * block_bytes + 4 * r) = v;
    }
    for (long long w = tid; w < sz_words; w += stride) {
        const long long b = w / (8 * G), r = w - b * 8 * G;
        const long long g = r / 8, j = r - g * 8;
        const long long src = (8 * b + j) * G + g;
        const uint32_t v = (uint32_t)src_scales[src] | ((uint32_t)src_zeros[src] << 16);
        *reinterpret_cast<uint32_t*>(dst + b * block_bytes + 4LL * cols + 4 * r) = v;
    }
}

}  // namespace

extern "C" WispError wisp_expert_tile(const WispExpertMeta* meta, const void* src_blob,
                                      void* dst_blob, cudaStream_t stream, WispErrCtx* err) {
    if (!meta || !src_blob || !dst_blob || src_blob == dst_blob) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "expert_tile: NULL or in-place arguments");
        return WISP_ERR_INVALID_ARG;
    }
    if (!meta->valid || meta->tiled) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "expert_tile: source must be a parsed .bin blob (valid=%d tiled=%d)",
                   meta->valid, meta->tiled);
        return WISP_ERR_INVALID_ARG;
    }
    const int gs = (int)meta->group_size;
    const uint8_t* src = static_cast<const uint8_t*>(src_blob);
    uint8_t* dst = static_cast<uint8_t*>(dst_blob);
    if ((reinterpret_cast<uintptr_t>(src) - 120) % 16 || (reinterpret_cast<uintptr_t>(dst) - 120) % 16) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "expert_tile: blobs must start at an address = 8 (mod 16)");
        return WISP_ERR_INVALID_ARG;
    }
    for (int m = 0; m < WISP_EXPERT_NMATS; ++m) {
        const long long R = meta->rows[m], Cc = meta->cols[m];
        if (gs <= 0 || gs % 8 || R % 8 || Cc % gs || Cc % 8 ||
            meta->scales_off[m] - meta->packed_off[m] != (size_t)(R * Cc / 2) ||
            meta->zeros_off[m] - meta->scales_off[m] != (size_t)(R * (Cc / gs) * 2) ||
            (meta->packed_off[m] - 120) % 16) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "expert_tile: matrix %d [%lld x %lld] group %d cannot be tiled (rows must "
                       "be a multiple of 8, cols of group_size and 8, group_size of 8)",
                       m, R, Cc, gs);
            return WISP_ERR_INVALID_ARG;
        }
    }
    for (int m = 0; m < WISP_EXPERT_NMATS; ++m) {
        const long long R = meta->rows[m], Cc = meta->cols[m];
        const long long words = R * Cc / 8 + R * (Cc / gs);
        const int threads = 256;
        const long long want = (words + threads - 1) / threads;
        const int blocks = (int)(want < 4096 ? want : 4096);
        tile_matrix_kernel<<<blocks, threads, 0, stream>>>(
            reinterpret_cast<const uint32_t*>(src + meta->packed_off[m]),
            reinterpret_cast<const uint16_t*>(src + meta->scales_off[m]),
            reinterpret_cast<const uint16_t*>(src + meta->zeros_off[m]), dst + meta->packed_off[m],
            (int)R, (int)Cc, gs, reinterpret_cast<const uint32_t*>(src),
            m == 0 ? reinterpret_cast<uint32_t*>(dst) : nullptr);
        WB_CUDA_RET(cudaGetLastError(), err);
    }
    return WISP_OK;
}
