// prefill.cu -- the MoE block for batched and prefill tokens on the 5th-generation
// tensor cores (tcgen05 + TMA).
//
// Semantics are the reference's run_moe (csrc/core/wisp_engine.c:1411-1522) per
// token -- the reference has no batch, a batch of T tokens is T independent
// calls -- with the router rule of router.cu:60-120 / wisp_engine.c:520-556
// (route_common.cuh), the int4 rule of quantizer.py:89-105 (weight =
// (q - 8) * scale + zero, scale and zero fp16), SwiGLU h = silu(g) * u
// (matmul.cu:169-205) and the combine y = shared(x) + sum_j w_j * down_j(h_j)
// (wisp_engine.c:1443-1522).  Like the reference's GPU dequant
// (expert_loader.cu:23-43) the weights are rounded to fp16 before the matmul;
// the activations are rounded to fp16 too, and every product is accumulated in
// fp32 (TMEM).
//
// One block, all on one stream, no host synchronisation:
//   router_logits_kernel  logits [T, E] in fp32 on the CUDA cores
//   route_topk_kernel     top-k under the layer's gating rule, one warp per token
//   prefill_plan_kernel   one CTA: the (token, slot) assignments grouped by
//                         expert into rows, the tile lists, and the per-expert
//                         TMA descriptors (a host-encoded template whose global
//                         address is replaced on the device, so experts may sit
//                         anywhere: resident arena, cache slots, scratch ring)
//   prefill_scatter_kernel xs[row] = fp16(x[token(row)]) for every row; y = 0
//   grouped_gemm<2>       gate/up: hs[row] = silu(Wg xs[row]) * (Wu xs[row])
//   grouped_gemm<1>       down:    y[token(row)] += w(row) * (Wd hs[row])
//
// The grouped GEMM puts the weights on the MMA's M side (128 weight rows per
// tile) and the tokens of one expert on N (16..128 per tile), so an expert with
// few tokens wastes little of the tensor core.  A persistent CTA per SM walks
// the tile list (static round robin) with warp-specialised roles:
//   warps 0-3   epilogue: tcgen05.ld of the fp32 accumulators (warp q reads
//               TMEM lanes 32q..32q+31), SwiGLU / gate-weighted combine
//   warp 4      weight producer: two 3-D TMA loads per matrix and K block
//               (the codes and the scale/zero pairs of 16 tiled 8-row blocks)
//   warp 5      MMA issuer (one thread): tcgen05.mma kind::f16, M=128, K=16,
//               A from tensor memory, B from shared memory
//   warp 6      activation producer: 2-D TMA loads, 128-byte swizzle
//   warps 7-22  dequantisers: int4 codes -> fp16, written straight into
//               tensor memory with tcgen05.st (TMEM lane = weight row), so the
//               dequantised weights never round-trip through shared memory
// TMEM (512 columns): accumulators in [0, 256), dequantised A stages above.
// Shared-memory rings with mbarriers connect the roles; every wait is bounded
// (2 s of %globaltimer) and a timeout sets ST_TIMEOUT in the status word, makes
// every role leave, drains the copies and MMAs in flight and frees TMEM.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "dense_ffn.h"
#include "internal.h"
#include "route_common.cuh"

namespace {

enum { ST_ALIGN = 1, ST_EXPERT = 2, ST_PLAN = 4, ST_TIMEOUT = 8, ST_LAYOUT = 16 };
constexpr uint32_t kTiledVersion = 2;
constexpr unsigned kFull = 0xffffffffu;

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBK = 64;         // K per stage: one quant group
constexpr int kNT = 128;        // max tokens per tile (MMA N)
constexpr int kWProdWarp = 4, kMmaWarp = 5, kBProdWarp = 6, kDqWarp0 = 7, kDqWarps = 16;
constexpr int kGemmThreads = (kDqWarp0 + kDqWarps) * 32;  // 736
constexpr int kMaps = 6;        // per expert: (gate, up, down) x (codes, scale/zero)
constexpr int kBoxes = 4;       // activation boxes of 16, 32, 64, 128 rows
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr int kPlanThreads = 1024;
constexpr int kRouteTile = 64;
constexpr int kRouterTcMinT = 64;  // tokens from which the router runs on the tensor cores
constexpr uint32_t kAcol0 = 256;  // TMEM: accumulators in columns [0, 256), A stages above

constexpr int kBTile = kNT * 128;          // 128 rows x 64 fp16 (16 KB)
constexpr int kWCodes = 16 * 8 * 32;       // 16 blocks x 8 rows x 32 code bytes
constexpr int kWStage = kWCodes + 16 * 32;  // + 16 blocks x 8 (scale, zero) pairs

struct PTile {
    int e, mt, row0, n;  // expert (E = shared), weight-row tile, first row, tokens
};

struct BMaps {
    CUtensorMap box[kBoxes];  // box i: 64 columns x (16 << i) rows
};
struct WTemplates {
    CUtensorMap m[kMaps];  // global address replaced per expert on the device
};

struct PArgs {
    const void* const* blobs;
    const void* shared_blob;
    const __half* router_w;
    const __half* router_bias;
    unsigned long long mat_off[3];  // packed_off of gate, up, down in a blob
    int H, I, E, K, has_shared;
    int gating; // WISP_GATING_* of the layer
};

struct PWs {
    int* status;
    int* counters;    // [0] gate/up tiles, [1] down tiles
    float* logits;    // [T, E]
    int* idx;         // [T, K]
    float* w;         // [T, K]
    int* cnt;         // [E + 1] rows per expert (E = shared)
    int* seg;         // [E + 2] first row per expert
    int* row_tok;     // [R]
    float* row_w;     // [R]
    int* row_of;      // [T * K]
    PTile* tiles_gu;  // [max_gu]
    PTile* tiles_dn;  // [max_dn]
    CUtensorMap* wmaps;  // [(E + 1) * kMaps]
    __half* xs;       // [R, H]
    __half* hs;       // [R, I]
    int R, max_gu, max_dn;
};

// A stage covers KG quant groups (K = 64 * KG).  Ring depths in stages -- WS:
// weight staging (smem); BS: activation tiles (smem, deep: their loads are the
// longest-latency step); S: dequantised weight tiles in TMEM (NMAT * KG * 32
// columns each); NACC: accumulator buffers (TMEM, 128 columns per matrix).
// TMEM: 256 accumulator columns + S * NMAT * KG * 32 = 256 A columns.  Every
// stage carries a fixed cost (the issuing thread's polls, fence and commits, the
// dequantisers' TMEM-store wait and arrivals), so stages are as large as TMEM
// allows: gate/up 2 groups (two matrices), down 4 groups when its K has a
// multiple of 4 groups and the expert tiles are thin, else 2.  kKG is the
// gate/up stage size.
constexpr int kKG = 2;
template <int NMAT, int KG>
struct GCfg;
template <>
struct GCfg<2, 2> {  // gate + up
    static constexpr int WS = 4, BS = 4, S = 2, NACC = 1;
};
template <>
struct GCfg<1, 2> {  // down, K of 2 (mod 4) groups
    static constexpr int WS = 8, BS = 4, S = 4, NACC = 2;
};
template <>
struct GCfg<1, 4> {  // down
    static constexpr int WS = 4, BS = 2, S = 2, NACC = 2;
};

template <int NMAT, int KG>
constexpr size_t gemm_smem_bytes() {
    using C = GCfg<NMAT, KG>;
    return 1024 + (size_t)C::BS * KG * kBTile + (size_t)C::WS * NMAT * KG * kWStage + 1024;
}

// ------------------------------------------------------------------------
// device helpers
// ------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ uint32_t saddr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait of one thread; false on timeout (sets the abort flag and
// ST_TIMEOUT) or when another role aborted.
__device__ __forceinline__ bool wait1(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                      int* status) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 63) {
            if (*abort_flag) return false;
            const uint64_t t = gtimer();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > kWaitNs) {
                *abort_flag = 1;
                atomicOr(status, ST_TIMEOUT);
                return false;
            }
        }
    }
}
// The same for a whole warp, with a warp-uniform result.
__device__ __forceinline__ bool wait_warp(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                          int* status) {
    const int lane = threadIdx.x & 31;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(kFull, mbar_try(b, parity))) return true;
        if ((it & 63) == 63) {
            int stop = 0;
            if (lane == 0) {
                if (*abort_flag) {
                    stop = 1;
                } else {
                    const uint64_t t = gtimer();
                    if (t0 == 0) {
                        t0 = t;
                    } else if (t - t0 > kWaitNs) {
                        *abort_flag = 1;
                        atomicOr(status, ST_TIMEOUT);
                        stop = 1;
                    }
                }
            }
            if (__shfl_sync(kFull, stop, 0)) return false;
        }
    }
}
// Waits of the roles that are not latency-critical (producers refilling deep
// rings, the epilogue waiting for a whole tile): after a few polls they back
// off with __nanosleep so they do not take issue slots from the MMA thread
// and the dequantisers.
__device__ __forceinline__ bool wait1_lazy(uint64_t* b, uint32_t parity,
                                           volatile int* abort_flag, int* status) {
    for (int i = 0; i < 8; ++i)
        if (mbar_try(b, parity)) return true;
    uint64_t t0 = gtimer();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(b, parity)) return true;
        __nanosleep(64);
        if ((it & 15) == 15) {
            if (*abort_flag) return false;
            if (gtimer() - t0 > kWaitNs) {
                *abort_flag = 1;
                atomicOr(status, ST_TIMEOUT);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool wait_warp_lazy(uint64_t* b, uint32_t parity,
                                               volatile int* abort_flag, int* status) {
    const int lane = threadIdx.x & 31;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(kFull, mbar_try(b, parity))) return true;
        __nanosleep(256);
        if ((it & 15) == 15) {
            int stop = 0;
            if (lane == 0) {
                if (*abort_flag) {
                    stop = 1;
                } else {
                    const uint64_t t = gtimer();
                    if (t0 == 0) {
                        t0 = t;
                    } else if (t - t0 > kWaitNs) {
                        *abort_flag = 1;
                        atomicOr(status, ST_TIMEOUT);
                        stop = 1;
                    }
                }
            }
            if (__shfl_sync(kFull, stop, 0)) return false;
        }
    }
}
// Drain wait: ignores the abort flag, bounded by time only.
__device__ __forceinline__ void wait_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = gtimer();
    while (!mbar_try(b, parity))
        if (gtimer() - t0 > kWaitNs) return;
}

__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                      uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(saddr(bar))
        : "memory");
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                      uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(saddr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(saddr(bar))
        : "memory");
}
__device__ __forceinline__ void tmap_acquire(const CUtensorMap* map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(
                     reinterpret_cast<uint64_t>(map))
                 : "memory");
}

// tcgen05 ------------------------------------------------------------------
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 B (stride byte offset 1024, leading byte offset unused = 16 B),
// descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator, both
// K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}
// D (TMEM) += A (TMEM, 128 lanes x 8 columns of fp16 pairs) * B (smem descriptor)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(id), "r"(acc), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            saddr(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16};" ::"r"(addr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// K order inside every 8-element chunk of the MMA operands: position 2i holds
// element i and position 2i+1 element i+4 (i < 4), the order in which one
// 32-bit word of int4 codes unpacks into fp16 pairs without byte permutes.
// The activation rows (xs, hs) are written in the same order.
__device__ __forceinline__ int kperm(int f) { return (f & ~7) | ((f & 3) << 1) | ((f >> 2) & 1); }

// Eight int4 codes (one 32-bit word, low nibble = even element) with their
// group's fp16 scale and zero -> four TMEM columns of fp16 weight pairs
// (e0,e4) (e1,e5) (e2,e6) (e3,e7), each weight (q - 8) * s + z rounded once
// (fused multiply-add on the exact q - 8): 1024 + q is built in the fp16 bit
// pattern (0x6400 | q) and 1032 subtracted exactly.
__device__ __forceinline__ void dequant_cols(uint32_t v, __half2 s2, __half2 z2, uint32_t* o) {
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6408u));  // 1032
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t t = ((v >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&t), off);
        const __half2 w = __hfma2(q, s2, z2);
        o[i] = *reinterpret_cast<const uint32_t*>(&w);
    }
}

// ------------------------------------------------------------------------
// routing
// ------------------------------------------------------------------------

// logits[t][e] = sum_h x[t][h] * W[e][h] in fp32.  CTA tile 64 tokens x 64
// experts, 256 threads of 4 x 4 outputs, K in chunks of 32.
__global__ void __launch_bounds__(256)
router_logits_kernel(const float* __restrict__ x, const __half* __restrict__ Wr,
                     float* __restrict__ lg, int T, int E, int H) {
    pdl_wait();
    pdl_launch();
    __shared__ float xs[32][kRouteTile + 4];
    __shared__ float ws[32][kRouteTile + 4];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int t0 = blockIdx.x * kRouteTile, e0 = blockIdx.y * kRouteTile;
    float acc[4][4] = {};
    for (int h0 = 0; h0 < H; h0 += 32) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int id = tid + 256 * i, r = id >> 5, k = id & 31;
            const int t = t0 + r, e = e0 + r;
            xs[k][r] = t < T ? x[(size_t)t * H + h0 + k] : 0.f;
            ws[k][r] = e < E ? __half2float(Wr[(size_t)e * H + h0 + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[k][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&ws[k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < E) lg[(size_t)t * E + e] = acc[i][j];
        }
    }
}

// x [T, H] fp32 -> hi = fp16(x), lo = fp16(x - hi): the router GEMM on the
// tensor cores sums W*hi + W*lo, which carries x to ~2^-22 relative precision
// (fp16 x fp16 products are exact in the fp32 accumulator).
__global__ void __launch_bounds__(256)
split_hilo_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo,
                  long long n4) {
    pdl_wait();
    pdl_launch();
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n4; i += (long long)gridDim.x * 256) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        const __half2 l0 = __floats2half2_rn(v.x - f0.x, v.y - f0.y);
        const __half2 l1 = __floats2half2_rn(v.z - f1.x, v.w - f1.y);
        uint2 a, b;
        a.x = *reinterpret_cast<const uint32_t*>(&h0);
        a.y = *reinterpret_cast<const uint32_t*>(&h1);
        b.x = *reinterpret_cast<const uint32_t*>(&l0);
        b.y = *reinterpret_cast<const uint32_t*>(&l1);
        reinterpret_cast<uint2*>(hi)[i] = a;
        reinterpret_cast<uint2*>(lo)[i] = b;
    }
}

// Router logits on the tensor cores: logits[t][e] = W[e] . (hi[t] + lo[t]).
// One CTA per (128 experts x 128 tokens) tile; warp 4 loads W, hi and lo tiles
// (64-wide K blocks, 128-byte swizzle) into a 4-stage ring, warp 5 issues
// eight kind::f16 MMAs per K block into one fp32 accumulator (128 TMEM
// columns), warps 0-3 write the logits.  Rows past E and tokens past T are
// zero-filled by TMA and not stored.
struct RouterMaps {
    CUtensorMap w, hi, lo;
};
constexpr int kRtStages = 4;
constexpr int kRtTile = 128 * 128;  // bytes of one 128 x 64 fp16 tile
constexpr size_t kRouterSmem = 1024 + (size_t)kRtStages * 3 * kRtTile + 256;

__global__ void __launch_bounds__(192, 1)
router_tc_kernel(const __grid_constant__ RouterMaps rm, float* __restrict__ lg, int T, int E,
                 int H, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kRtStages * 3 * kRtTile);
    uint64_t* empty = full + kRtStages;
    uint64_t* done = empty + kRtStages;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e0 = blockIdx.x * 128, t0 = blockIdx.y * 128;
    const int KB = H / kBK;
    if (tid == 0) {
        for (int i = 0; i < kRtStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(
                         saddr(s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    pdl_wait();
    pdl_launch();
    if (warp == 4) {
        if (lane == 0) {
            uint32_t i = 0;
            for (int kb = 0; kb < KB; ++kb, ++i) {
                const int s = i % kRtStages;
                if (!wait1_lazy(&empty[s], ((i / kRtStages) & 1) ^ 1, s_abort, status)) break;
                mbar_expect_tx(&full[s], 3 * kRtTile);
                uint8_t* st = base + s * 3 * kRtTile;
                tma2d(st, &rm.w, kb * kBK, e0, &full[s]);
                tma2d(st + kRtTile, &rm.hi, kb * kBK, t0, &full[s]);
                tma2d(st + 2 * kRtTile, &rm.lo, kb * kBK, t0, &full[s]);
            }
            const uint32_t first = i > (uint32_t)kRtStages ? i - kRtStages : 0;
            for (uint32_t j = first; j < i; ++j) wait_drain(&full[j % kRtStages], (j / kRtStages) & 1);
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t id = idesc_f16(128);
            bool ok = true;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % kRtStages;
                if (!wait1(&full[s], (kb / kRtStages) & 1, s_abort, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = saddr(base + s * 3 * kRtTile);
                const uint64_t wd = sdesc(st), hd = sdesc(st + kRtTile), ld = sdesc(st + 2 * kRtTile);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                        "l"(wd + 2 * k), "l"(hd + 2 * k), "r"(id), "r"((kb | k) ? 1u : 0u)
                        : "memory");
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                        "l"(wd + 2 * k), "l"(ld + 2 * k), "r"(id), "r"(1u)
                        : "memory");
                }
                mma_commit(&empty[s]);
            }
            (void)ok;
            mma_commit(done);  // also the drain: every MMA of this CTA has completed
            wait_drain(done, 0);
        }
    } else {
        // warps 0-3: TMEM lane = expert row of the tile, column = token
        if (wait_warp_lazy(done, 0, s_abort, status)) {
            tc_fence_after();
            const int e = e0 + warp * 32 + lane;
            const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
            for (int c = 0; c < 128; c += 16) {
                float v[16];
                tmem_ld16(lb + c, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + c + j;
                    if (e < E && t < T) lg[(size_t)t * E + e] = v[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem)
                     : "memory");
    }
}

// top-k per token under the layer's gating rule (softmax(+bias) or sigmoid
// scores), one warp per token.
__global__ void __launch_bounds__(256)
route_topk_kernel(const float* __restrict__ lg, const __half* bias, int T, int E, int K,
                  int* idx, float* w, int gating) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float rs[];
    const int warp = threadIdx.x >> 5;
    float* sp = rs + (size_t)warp * 2 * E;
    for (int t = blockIdx.x * 8 + warp; t < T; t += gridDim.x * 8) {
        wisp_route::warp_topk(lg + (size_t)t * E, bias, E, K, sp, idx + (size_t)t * K,
                              w + (size_t)t * K, gating);
        __syncwarp();
    }
}

// ------------------------------------------------------------------------
// plan: rows grouped by expert, tiles, TMA descriptors
// ------------------------------------------------------------------------
__device__ const void* blob_of(const PArgs& P, int e) {
    return e == P.E ? P.shared_blob : P.blobs[e];
}

__global__ void __launch_bounds__(kPlanThreads)
prefill_plan_kernel(PArgs P, PWs W, int T, const __grid_constant__ WTemplates tmpl) {
    pdl_wait();
    pdl_launch();
    extern __shared__ int ps[];
    __shared__ alignas(128) CUtensorMap s_map[kPlanThreads / 32];
    const int E = P.E, K = P.K, NE = E + 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int* s_cnt = ps;               // [E + 1]
    int* s_fill = s_cnt + NE;      // [E + 1]
    int* s_seg = s_fill + NE;      // [E + 2]
    int* s_tgu = s_seg + NE + 1;   // [E + 2]
    int* s_tdn = s_tgu + NE + 1;   // [E + 2]
    const int mt_gu = P.I / kBM, mt_dn = P.H / kBM;
    for (int e = tid; e < NE; e += kPlanThreads) {
        s_cnt[e] = 0;
        s_fill[e] = 0;
    }
    __syncthreads();
    for (int a = tid; a < T * K; a += kPlanThreads) {
        const int e = W.idx[a];
        if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
    }
    if (tid == 0) s_cnt[E] = P.has_shared ? T : 0;
    __syncthreads();
    // the experts that have rows must be present, tiled and 16-byte aligned
    for (int e = tid; e < NE; e += kPlanThreads) {
        if (s_cnt[e] == 0) continue;
        const void* b = blob_of(P, e);
        int bad = 0;
        if (!b)
            bad = ST_EXPERT;
        else if ((reinterpret_cast<uintptr_t>(b) & 15) != 8)
            bad = ST_ALIGN;
        else if (__ldg(reinterpret_cast<const uint32_t*>(b) + 1) != kTiledVersion)
            bad = ST_LAYOUT;
        if (bad) {
            atomicOr(W.status, bad);
            s_cnt[e] = 0;
        }
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0, tg = 0, td = 0;
        for (int e = 0; e < NE; ++e) {
            s_seg[e] = run;
            s_tgu[e] = tg;
            s_tdn[e] = td;
            const int nt = (s_cnt[e] + kNT - 1) / kNT;
            run += s_cnt[e];
            tg += nt * mt_gu;
            td += nt * mt_dn;
        }
        s_seg[NE] = run;
        s_tgu[NE] = tg;
        s_tdn[NE] = td;
        if (run > W.R || tg > W.max_gu || td > W.max_dn) {
            atomicOr(W.status, ST_PLAN);
            tg = td = 0;
        }
        W.counters[0] = tg;
        W.counters[1] = td;
    }
    __syncthreads();
    for (int e = tid; e < NE; e += kPlanThreads) {
        W.cnt[e] = s_cnt[e];
        W.seg[e] = s_seg[e];
    }
    if (tid == 0) W.seg[NE] = s_seg[NE];
    for (int a = tid; a < T * K; a += kPlanThreads) {
        const int e = W.idx[a];
        int r = -1;
        if (e >= 0 && e < E && s_cnt[e] > 0 && s_seg[e] + s_cnt[e] <= W.R) {
            r = s_seg[e] + atomicAdd(&s_fill[e], 1);
            W.row_tok[r] = a / K;
            W.row_w[r] = W.w[a];
        }
        W.row_of[a] = r;
    }
    if (s_cnt[E] > 0 && s_seg[E] + T <= W.R)
        for (int t = tid; t < T; t += kPlanThreads) {
            W.row_tok[s_seg[E] + t] = t;
            W.row_w[s_seg[E] + t] = 1.f;
        }
    // tile lists, ordered (expert, token tile, weight-row tile)
    const int ntg = W.counters[0] ? s_tgu[NE] : 0, ntd = W.counters[1] ? s_tdn[NE] : 0;
    for (int pass = 0; pass < 2; ++pass) {
        const int* base = pass ? s_tdn : s_tgu;
        const int n = pass ? ntd : ntg, mt_per = pass ? mt_dn : mt_gu;
        PTile* out = pass ? W.tiles_dn : W.tiles_gu;
        for (int i = tid; i < n; i += kPlanThreads) {
            int lo = 0, hi = NE;  // last e with base[e] <= i
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (base[mid] <= i) lo = mid; else hi = mid;
            }
            // experts with no tiles share a base: take the one that has tiles
            int e = lo;
            while (e + 1 < NE && base[e + 1] <= i) ++e;
            const int local = i - base[e], nt = local / mt_per;
            PTile tl;
            tl.e = e;
            tl.mt = local - nt * mt_per;
            tl.row0 = s_seg[e] + nt * kNT;
            tl.n = min(kNT, s_cnt[e] - nt * kNT);
            out[i] = tl;
        }
    }
    // TMA descriptors of the experts with rows: one warp per descriptor
    for (int j = warp; j < NE * kMaps; j += kPlanThreads / 32) {
        const int e = j / kMaps, m = j - e * kMaps;
        if (s_cnt[e] == 0) continue;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&tmpl.m[m]);
        reinterpret_cast<uint32_t*>(&s_map[warp])[lane] = src[lane];
        __syncwarp();
        if (lane == 0) {
            const int mat = m >> 1;
            const unsigned long long cols = mat == 2 ? (unsigned long long)P.I : P.H;
            const unsigned long long addr = reinterpret_cast<unsigned long long>(blob_of(P, e)) +
                                            P.mat_off[mat] + ((m & 1) ? 4ull * cols : 0ull);
            asm volatile("tensormap.replace.tile.global_address.shared::cta.b1024.b64 [%0], %1;"
                         ::"r"(saddr(&s_map[warp])), "l"(addr)
                         : "memory");
        }
        __syncwarp();
        asm volatile(
            "tensormap.cp_fenceproxy.global.shared::cta.tensormap::generic.release.gpu.sync."
            "aligned [%0], [%1], 128;" ::"l"(reinterpret_cast<uint64_t>(W.wmaps + j)),
            "r"(saddr(&s_map[warp]))
            : "memory");
        __syncwarp();
    }
}

// xs[row] = fp16(x[token]) for each row of token t (routed slots + shared);
// y[t] = 0 (the down GEMM accumulates into it).
__global__ void __launch_bounds__(256)
prefill_scatter_kernel(PArgs P, PWs W, int T, const float* __restrict__ x, float* __restrict__ y) {
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.x, K = P.K, H = P.H;
    __shared__ int rows[65];
    if (threadIdx.x < K) rows[threadIdx.x] = W.row_of[t * K + threadIdx.x];
    // the shared expert's rows exist only with one (the plan writes its count
    // and segment only then; a routing-given call has none)
    if (threadIdx.x == 0) rows[K] = P.has_shared && W.cnt[P.E] > 0 ? W.seg[P.E] + t : -1;
    __syncthreads();
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * H);
    float4* yr = reinterpret_cast<float4*>(y + (size_t)t * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
        const float4 a = xr[2 * c], b = xr[2 * c + 1];
        // the operands' K order inside a chunk: x0 x4 x1 x5 x2 x6 x3 x7 (kperm)
        const __half2 h0 = __floats2half2_rn(a.x, b.x), h1 = __floats2half2_rn(a.y, b.y);
        const __half2 h2 = __floats2half2_rn(a.z, b.z), h3 = __floats2half2_rn(a.w, b.w);
        uint4 v;
        v.x = *reinterpret_cast<const uint32_t*>(&h0);
        v.y = *reinterpret_cast<const uint32_t*>(&h1);
        v.z = *reinterpret_cast<const uint32_t*>(&h2);
        v.w = *reinterpret_cast<const uint32_t*>(&h3);
        for (int j = 0; j <= K; ++j) {
            const int r = rows[j];
            if (r >= 0) reinterpret_cast<uint4*>(W.xs + (size_t)r * H)[c] = v;
        }
        yr[2 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
        yr[2 * c + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Between stacked blocks (the FFN half of decode_step, csrc/core/wisp_engine.c
// :1563-1570, attention = identity): x[t] += y[t] (the previous block's
// output, when `add`), then xn[t] = rmsnorm(x[t]) * w (cpu_rmsnorm,
// wisp_engine.c:415-422), when `norm`.  One CTA per token.
__global__ void __launch_bounds__(256)
prefill_norm_kernel(float* __restrict__ x, const float* __restrict__ y,
                    const __half* __restrict__ w, float* __restrict__ xn, int H, float eps,
                    int add, int norm) {
    pdl_wait();
    pdl_launch();
    const int t = blockIdx.x, tid = threadIdx.x;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)t * H);
    const float4* yr = reinterpret_cast<const float4*>(y + (size_t)t * H);
    __shared__ float red[8];
    float ss = 0.f;
    for (int i = tid; i < H / 4; i += 256) {
        float4 v = xr[i];
        if (add) {
            const float4 d = yr[i];
            v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
            xr[i] = v;
        }
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    if (!norm) return;
    ss = wisp_route::warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float sc = 1.0f / sqrtf(tot / (float)H + eps);
    float4* on = reinterpret_cast<float4*>(xn + (size_t)t * H);
    const __half2* w2 = reinterpret_cast<const __half2*>(w);
    for (int i = tid; i < H / 4; i += 256) {
        float4 v = xr[i];
        v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
        if (w) {
            const float2 a = __half22float2(w2[2 * i]), b = __half22float2(w2[2 * i + 1]);
            v.x *= a.x; v.y *= a.y; v.z *= b.x; v.w *= b.y;
        }
        on[i] = v;
    }
}

__device__ __forceinline__ PTile tiles_at(const PTile* tiles, int t) {
    const int4 v = __ldcg(reinterpret_cast<const int4*>(tiles) + t);
    return PTile{v.x, v.y, v.z, v.w};
}

// ------------------------------------------------------------------------
// the grouped GEMM
// ------------------------------------------------------------------------
template <int NMAT, int KG>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_kernel(PArgs P, PWs W, const __grid_constant__ BMaps bm, float* __restrict__ y) {
    using C = GCfg<NMAT, KG>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~(uintptr_t)1023);
    uint8_t* sB = base;
    uint8_t* sW = sB + C::BS * KG * kBTile;
    uint64_t* w_full = reinterpret_cast<uint64_t*>(sW + C::WS * NMAT * KG * kWStage);
    uint64_t* w_empty = w_full + C::WS;
    uint64_t* a_full = w_empty + C::WS;   // dequantised tile in TMEM
    uint64_t* a_empty = a_full + C::S;
    uint64_t* b_full = a_empty + C::S;    // activation tile in smem
    uint64_t* b_empty = b_full + C::BS;
    uint64_t* acc_full = b_empty + C::BS;
    uint64_t* acc_empty = acc_full + C::NACC;
    uint64_t* drain = acc_empty + C::NACC;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < C::WS; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], kDqWarps);
        }
        for (int i = 0; i < C::S; ++i) {
            mbar_init(&a_full[i], kDqWarps);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < C::BS; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < C::NACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(drain, 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         saddr(s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    pdl_wait();
    pdl_launch();
    const int ntiles = __ldcg(W.counters + (NMAT == 2 ? 0 : 1));
    const PTile* tiles = NMAT == 2 ? W.tiles_gu : W.tiles_dn;
    const int KS = (NMAT == 2 ? P.H : P.I) / (kBK * KG);  // stages per tile
    int* status = W.status;

    if (warp == kWProdWarp) {
        if (lane == 0) {
            uint32_t wi = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                const PTile tl = tiles[t];
                const CUtensorMap* maps[NMAT][2];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const int mat = NMAT == 2 ? m : 2;
                    maps[m][0] = W.wmaps + tl.e * kMaps + mat * 2;
                    maps[m][1] = maps[m][0] + 1;
                    tmap_acquire(maps[m][0]);
                    tmap_acquire(maps[m][1]);
                }
                for (int ks = 0; ks < KS; ++ks, ++wi) {
                    const int s = wi % C::WS;
                    if (!wait1_lazy(&w_empty[s], ((wi / C::WS) & 1) ^ 1, s_abort, status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&w_full[s], NMAT * KG * kWStage);
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        // [16 blocks][KG groups] of codes, then of scale/zero pairs
                        uint8_t* dst = sW + (s * NMAT + m) * KG * kWStage;
                        tma3d(dst, maps[m][0], 0, ks * KG, tl.mt * 16, &w_full[s]);
                        tma3d(dst + KG * kWCodes, maps[m][1], 0, ks * KG, tl.mt * 16, &w_full[s]);
                    }
                }
            }
            const uint32_t first = wi > (uint32_t)C::WS ? wi - C::WS : 0;
            for (uint32_t i = first; i < wi; ++i) wait_drain(&w_full[i % C::WS], (i / C::WS) & 1);
        }
    } else if (warp == kBProdWarp) {
        if (lane == 0) {
            uint32_t bi = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                const PTile tl = tiles[t];
                const int nmma = (tl.n + 15) & ~15;
                for (int ks = 0; ks < KS; ++ks, ++bi) {
                    const int s = bi % C::BS;
                    if (!wait1_lazy(&b_empty[s], ((bi / C::BS) & 1) ^ 1, s_abort, status)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&b_full[s], (uint32_t)(KG * nmma * 128));
#pragma unroll
                    for (int g = 0; g < KG; ++g) {
                        int off = 0;
#pragma unroll
                        for (int i = kBoxes - 1; i >= 0; --i) {
                            const int h = 16 << i;
                            if ((nmma - off) >= h) {
                                tma2d(sB + (s * KG + g) * kBTile + off * 128, &bm.box[i],
                                      (ks * KG + g) * kBK, tl.row0 + off, &b_full[s]);
                                off += h;
                            }
                        }
                    }
                }
            }
            const uint32_t first = bi > (uint32_t)C::BS ? bi - C::BS : 0;
            for (uint32_t i = first; i < bi; ++i) wait_drain(&b_full[i % C::BS], (i / C::BS) & 1);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t si = 0, ci = 0;
            bool ok = true;
            const uint64_t bdesc0 = sdesc(saddr(sB));
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++ci) {
                const PTile tl = tiles[t];
                const int nmma = (tl.n + 15) & ~15;
                const uint32_t id = idesc_f16(nmma);
                const int buf = ci % C::NACC;
                if (!wait1(&acc_empty[buf], ((ci / C::NACC) & 1) ^ 1, s_abort, status)) break;
                tc_fence_after();
                const uint32_t d0 = tmem + (uint32_t)((NMAT == 2 ? 0 : buf) * kNT);
                for (int ks = 0; ks < KS; ++ks, ++si) {
                    const int s = si % C::S, sb = si % C::BS;
                    if (!wait1(&a_full[s], (si / C::S) & 1, s_abort, status) ||
                        !wait1(&b_full[sb], (si / C::BS) & 1, s_abort, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bd = bdesc0 + (uint64_t)(sb * KG * (kBTile >> 4));
                    const uint32_t at = tmem + kAcol0 + (uint32_t)(s * NMAT * KG * 32);
#pragma unroll
                    for (int g = 0; g < KG; ++g)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
#pragma unroll
                            for (int m = 0; m < NMAT; ++m)
                                mma_ts(d0 + (uint32_t)(m * kNT),
                                       at + (uint32_t)((m * KG + g) * 32 + k * 8),
                                       bd + (uint64_t)(g * (kBTile >> 4) + 2 * k), id,
                                       (ks | g | k) ? 1u : 0u);
                    mma_commit(&a_empty[s]);
                    mma_commit(&b_empty[sb]);
                }
                if (ok) mma_commit(&acc_full[buf]);
            }
            mma_commit(drain);
            wait_drain(drain, 0);
        }
    } else if (warp < 4) {
        // epilogue: warp q owns TMEM lanes (weight rows) 32q .. 32q+31
        const int q = warp;
        uint32_t ci = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++ci) {
            const PTile tl = tiles[t];
            const int nmma = (tl.n + 15) & ~15;
            const int buf = ci % C::NACC;
            if (!wait_warp_lazy(&acc_full[buf], (ci / C::NACC) & 1, s_abort, status)) break;
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
            const int f = tl.mt * kBM + q * 32 + lane;  // output feature of this thread
            for (int c = 0; c < nmma; c += 16) {
                if (NMAT == 2) {
                    float g[16], u[16];
                    tmem_ld16(lane_base + c, g);
                    tmem_ld16(lane_base + kNT + c, u);
                    tmem_ld_wait();
                    const int fp = kperm(f);  // hs is the down GEMM's operand: K order
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (c + j < tl.n) {
                            const float h = g[j] / (1.0f + expf(-g[j])) * u[j];
                            W.hs[(size_t)(tl.row0 + c + j) * P.I + fp] = __float2half_rn(h);
                        }
                    }
                } else {
                    float v[16];
                    tmem_ld16(lane_base + buf * kNT + c, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (c + j < tl.n) {
                            const int r = tl.row0 + c + j;
                            const int tok = __ldg(W.row_tok + r);
                            const float wr = __ldg(W.row_w + r);
                            atomicAdd(y + (size_t)tok * P.H + f, wr * v[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    } else {
        // dequantisers: warp (g, q) writes TMEM lanes 32q..32q+31 (weight rows) of
        // part g of each group of the stage: gate/up -> matrix g/2, half g%2 of the
        // 64-wide group (16 columns); down -> quarter g (8 columns)
        const int dw = warp - kDqWarp0, q = warp & 3, gw = dw >> 2;
        const int r = q * 32 + lane;
        const int mat = NMAT == 2 ? (gw >> 1) : 0;
        constexpr int PW = NMAT == 2 ? 4 : 2;  // code words per thread and group
        const int part = NMAT == 2 ? (gw & 1) : gw;
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + kAcol0 +
                                   (uint32_t)(mat * KG * 32 + part * PW * 4);
        // smem staging of one matrix: [16 blocks][KG groups][8 rows][8 code words],
        // then [16 blocks][KG groups][8 rows] (scale, zero) words
        const int cw0 = ((r >> 3) * KG) * 64 + (r & 7) * 8 + part * PW;
        const int sw0 = KG * kWCodes / 4 + ((r >> 3) * KG) * 8 + (r & 7);
        uint32_t wi = 0, ai = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
            for (int ks = 0; ks < KS; ++ks, ++wi, ++ai) {
                const int ws = wi % C::WS, as = ai % C::S;
                if (!wait_warp(&w_full[ws], (wi / C::WS) & 1, s_abort, status) ||
                    !wait_warp(&a_empty[as], ((ai / C::S) & 1) ^ 1, s_abort, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t* st = reinterpret_cast<const uint32_t*>(
                    sW + (ws * NMAT + mat) * KG * kWStage);
#pragma unroll
                for (int g = 0; g < KG; ++g) {
                    const uint32_t szw = st[sw0 + g * 8];
                    const __half2 s2 =
                        __half2half2(__ushort_as_half((unsigned short)(szw & 0xFFFFu)));
                    const __half2 z2 = __half2half2(__ushort_as_half((unsigned short)(szw >> 16)));
                    const uint32_t ta = lane_addr + (uint32_t)((as * NMAT * KG + g) * 32);
                    if (PW == 4) {
                        const uint4 c4 = *reinterpret_cast<const uint4*>(st + cw0 + g * 64);
                        uint32_t o[16];
                        dequant_cols(c4.x, s2, z2, o);
                        dequant_cols(c4.y, s2, z2, o + 4);
                        dequant_cols(c4.z, s2, z2, o + 8);
                        dequant_cols(c4.w, s2, z2, o + 12);
                        tmem_st16(ta, o);
                    } else {
                        const uint2 c2 = *reinterpret_cast<const uint2*>(st + cw0 + g * 64);
                        uint32_t o[8];
                        dequant_cols(c2.x, s2, z2, o);
                        dequant_cols(c2.y, s2, z2, o + 4);
                        tmem_st8(ta, o);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[as]);
                    mbar_arrive(&w_empty[ws]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem)
                     : "memory");
    }
}

// ------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

size_t al(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct PLayout {
    size_t status, counters, logits, idx, w, cnt, seg, row_tok, row_w, row_of, tiles_gu, tiles_dn,
        wmaps, xs, hs, dh, dy, total;
    int R, max_gu, max_dn;
};

// si > 0: the layer's shared expert is fp16-dense (dense_ffn.cu), with its
// SwiGLU activations dh [T, si] and output dy [T, H] (fp32) in the workspace.
PLayout make_playout(int T, int H, int I, int E, int K, int si = 0) {
    PLayout L{};
    const int R = T * K + T;
    const int nt_max = (R + kNT - 1) / kNT + E + 2;  // token tiles over all experts
    L.R = R;
    L.max_gu = nt_max * (I / kBM);
    L.max_dn = nt_max * (H / kBM);
    size_t o = 0;
    L.status = o; o += 256;
    L.counters = o; o += 256;
    L.logits = o; o = al(o + (size_t)T * E * 4, 256);
    L.idx = o; o = al(o + (size_t)T * K * 4, 256);
    L.w = o; o = al(o + (size_t)T * K * 4, 256);
    L.cnt = o; o = al(o + (size_t)(E + 1) * 4, 256);
    L.seg = o; o = al(o + (size_t)(E + 2) * 4, 256);
    L.row_tok = o; o = al(o + (size_t)R * 4, 256);
    L.row_w = o; o = al(o + (size_t)R * 4, 256);
    L.row_of = o; o = al(o + (size_t)T * K * 4, 256);
    L.tiles_gu = o; o = al(o + (size_t)L.max_gu * sizeof(PTile), 256);
    L.tiles_dn = o; o = al(o + (size_t)L.max_dn * sizeof(PTile), 256);
    L.wmaps = o; o = al(o + (size_t)(E + 1) * kMaps * sizeof(CUtensorMap), 1024);
    L.xs = o; o = al(o + (size_t)R * H * 2, 1024);
    L.hs = o; o = al(o + (size_t)R * I * 2, 1024);
    L.dh = o; o = al(o + (size_t)T * si * 4, 1024);
    L.dy = o; o = al(o + (size_t)(si ? T : 0) * H * 4, 1024);
    L.total = o;
    return L;
}

PWs make_pws(void* ws, const PLayout& L) {
    char* b = static_cast<char*>(ws);
    PWs W;
    W.status = reinterpret_cast<int*>(b + L.status);
    W.counters = reinterpret_cast<int*>(b + L.counters);
    W.logits = reinterpret_cast<float*>(b + L.logits);
    W.idx = reinterpret_cast<int*>(b + L.idx);
    W.w = reinterpret_cast<float*>(b + L.w);
    W.cnt = reinterpret_cast<int*>(b + L.cnt);
    W.seg = reinterpret_cast<int*>(b + L.seg);
    W.row_tok = reinterpret_cast<int*>(b + L.row_tok);
    W.row_w = reinterpret_cast<float*>(b + L.row_w);
    W.row_of = reinterpret_cast<int*>(b + L.row_of);
    W.tiles_gu = reinterpret_cast<PTile*>(b + L.tiles_gu);
    W.tiles_dn = reinterpret_cast<PTile*>(b + L.tiles_dn);
    W.wmaps = reinterpret_cast<CUtensorMap*>(b + L.wmaps);
    W.xs = reinterpret_cast<__half*>(b + L.xs);
    W.hs = reinterpret_cast<__half*>(b + L.hs);
    W.R = L.R;
    W.max_gu = L.max_gu;
    W.max_dn = L.max_dn;
    return W;
}

// The layer's geometry must suit the tensor-core tiles: tiled int4 experts with
// 64-element groups, 128-row tiles of every matrix, a shared expert (if any) of
// the routed experts' shape.
WispError check_prefill_layer(const WispMoeLayer* l, int T, WispErrCtx* err, bool route = true) {
    const WispExpertMeta& m = l->meta;
    const int H = (int)m.cols[0], I = (int)m.rows[0];
    if (!l->expert_blobs || (route && !l->router_w) || !m.valid || T <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: missing layer pointers or T <= 0");
        return WISP_ERR_INVALID_ARG;
    }
    if (l->gating != WISP_GATING_SOFTMAX && l->gating != WISP_GATING_SIGMOID) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: unknown gating %d", l->gating);
        return WISP_ERR_INVALID_ARG;
    }
    if (!m.tiled || m.group_size != 64 || H % kBM || I % kBM || m.rows[1] != (uint32_t)I ||
        m.cols[1] != (uint32_t)H || m.rows[2] != (uint32_t)H || m.cols[2] != (uint32_t)I) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "prefill: needs tiled experts with group_size 64 and hidden/intermediate "
                   "multiples of 128 (got tiled=%d gs=%u H=%d I=%d)",
                   m.tiled, m.group_size, H, I);
        return WISP_ERR_INVALID_ARG;
    }
    for (int i = 0; i < 3; ++i)
        if ((m.packed_off[i] - 120) % 16) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: matrix %d not 16-byte aligned", i);
            return WISP_ERR_INVALID_ARG;
        }
    if (l->n_experts <= 0 || l->n_experts > 1024 || l->top_k <= 0 || l->top_k > 64 ||
        l->top_k > l->n_experts) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: n_experts %d / top_k %d out of range",
                   l->n_experts, l->top_k);
        return WISP_ERR_INVALID_ARG;
    }
    if (l->shared_gate || l->shared_up || l->shared_down) {
        if (l->shared_blob ||
            !wb::dense_ffn_shape_ok(l->shared_gate, l->shared_up, l->shared_down,
                                    l->shared_inter, H)) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "prefill: fp16-dense shared expert needs gate, up and down (16-byte "
                       "aligned), shared_inter a positive multiple of 8, and no int4 shared "
                       "blob beside it");
            return WISP_ERR_INVALID_ARG;
        }
    }
    if (l->shared_blob) {
        const WispExpertMeta& s = l->shared_meta;
        for (int i = 0; i < 3; ++i)
            if (s.rows[i] != m.rows[i] || s.cols[i] != m.cols[i] ||
                s.packed_off[i] != m.packed_off[i] || !s.tiled || s.group_size != m.group_size) {
                WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                           "prefill: the shared expert must have the routed experts' layout");
                return WISP_ERR_INVALID_ARG;
            }
    }
    return WISP_OK;
}

PArgs make_pargs(const WispMoeLayer* l) {
    PArgs P;
    P.blobs = l->expert_blobs;
    P.shared_blob = l->shared_blob;
    P.router_w = static_cast<const __half*>(l->router_w);
    P.router_bias = static_cast<const __half*>(l->router_bias);
    for (int i = 0; i < 3; ++i) P.mat_off[i] = l->meta.packed_off[i];
    P.H = (int)l->meta.cols[0];
    P.I = (int)l->meta.rows[0];
    P.E = l->n_experts;
    P.K = l->top_k;
    P.has_shared = l->shared_blob ? 1 : 0;
    P.gating = l->gating;
    return P;
}

bool encode(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* addr, const cuuint64_t* dims,
            const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint32_t es[3] = {1, 1, 1};
    return fn(map, dt, (cuuint32_t)rank, addr, dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Templates of the weight descriptors: codes [16 blocks][8 rows x 32 B] and
// (scale, zero) pairs [16 blocks][8 x 4 B] of one quant group, as 32-bit words
// over (word, group, 8-row block).  `anchor`: any 16-byte aligned device address
// (replaced per expert on the device).
// The boxes span one stage's groups: kKG for gate/up, `kg_down` for down.
bool weight_templates(const PArgs& P, const WispExpertMeta& m, void* anchor, WTemplates* t,
                      int kg_down) {
    for (int mat = 0; mat < 3; ++mat) {
        const cuuint64_t rows = m.rows[mat], cols = m.cols[mat];
        const cuuint64_t G = cols / 64, nblk = rows / 8, block_bytes = 4 * cols + 32 * G;
        const cuuint32_t kg = (cuuint32_t)(mat == 2 ? kg_down : kKG);
        const cuuint64_t dc[3] = {64, G, nblk}, sc[2] = {256, block_bytes};
        const cuuint32_t bc[3] = {64, kg, 16};
        const cuuint64_t ds[3] = {8, G, nblk}, ss[2] = {32, block_bytes};
        const cuuint32_t bs[3] = {8, kg, 16};
        if (!encode(&t->m[mat * 2], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, anchor, dc, sc, bc,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !encode(&t->m[mat * 2 + 1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, anchor, ds, ss, bs,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
            return false;
    }
    (void)P;
    return true;
}

// Activation rows [R][cols] fp16, boxes of 64 columns x (16 << i) rows, with the
// 128-byte swizzle tcgen05 reads.
bool row_maps(__half* rows_base, int R, int cols, BMaps* b) {
    const cuuint64_t d[2] = {(cuuint64_t)cols, (cuuint64_t)R}, s[1] = {(cuuint64_t)cols * 2};
    for (int i = 0; i < kBoxes; ++i) {
        const cuuint32_t box[2] = {64, (cuuint32_t)(16 << i)};
        if (!encode(&b->box[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows_base, d, s, box,
                    CU_TENSOR_MAP_SWIZZLE_128B))
            return false;
    }
    return true;
}

cudaError_t ensure_gemm_attrs() {
    static cudaError_t e = [] {
        cudaError_t r = cudaFuncSetAttribute(grouped_gemm_kernel<2, 2>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)gemm_smem_bytes<2, 2>());
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(grouped_gemm_kernel<1, 2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)gemm_smem_bytes<1, 2>());
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(grouped_gemm_kernel<1, 4>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)gemm_smem_bytes<1, 4>());
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(prefill_plan_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 5 * 1026 * 4);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kRouterSmem);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(route_topk_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 2 * 1024 * 4);
        return r;
    }();
    return e;
}

// Route x, then run the experts; x [T, H] fp32 is the MoE input (normalised).
// One block.  route: run the router (else topk_idx/topk_w [T, K] are the caller's
// routing, K = k_override, and the shared expert is left out: the expert-parallel
// owner of routed rows).
WispError prefill_block(const WispMoeLayer* layer, const float* x, float* y, int T,
                        int* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                        bool reset_status, cudaStream_t stream, WispErrCtx* err,
                        bool route = true, int k_override = 0) {
    WispError ce = check_prefill_layer(layer, T, err, route);
    if (ce != WISP_OK) return ce;
    PArgs P = make_pargs(layer);
    if (!route) {
        if (!topk_idx || !topk_w || k_override <= 0 || k_override > 64) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                       "prefill_routed: routing arrays and 1 <= K <= 64 required");
            return WISP_ERR_INVALID_ARG;
        }
        P.K = k_override;
        P.has_shared = 0;
    }
    // fp16-dense shared expert: CUDA-core GEMVs after the routed experts (dense_ffn.cu)
    const int dense_si = route && layer->shared_gate ? layer->shared_inter : 0;
    const PLayout L = make_playout(T, P.H, P.I, P.E, P.K, dense_si);
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 1023)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "prefill: workspace %zu bytes (need %zu, 1024-byte aligned)", workspace_bytes,
                   L.total);
        return WISP_ERR_INVALID_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: x and y must be 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    PWs W = make_pws(workspace, L);
    if (topk_idx) W.idx = topk_idx;
    if (topk_w) W.w = topk_w;
    WTemplates wt;
    BMaps bx, bh;
    // down stages of 4 groups when its K (= I) has a multiple of 4 groups and the
    // experts' tiles are thin (<= 96 rows per expert on average): measured on the
    // DeepSeek layer, 4 groups take -4.3% at 18 rows per expert (512 tokens) and
    // -3.3% at 36 (1024), +0.5% at 143 (4096), and +3.7% in a 32-expert layer at
    // 280 rows (ncu), where the shallower activation ring shows.
    const int nexp = P.E + (P.has_shared ? 1 : 0);
    const long long rows_per_expert = (long long)T * (P.K + (P.has_shared ? 1 : 0)) / nexp;
    const bool kg4_ok = (P.I / 64) % 4 == 0;
    int kg_down = kg4_ok && rows_per_expert <= 96 ? 4 : 2;
    if (!weight_templates(P, layer->meta, W.xs, &wt, kg_down) || !row_maps(W.xs, L.R, P.H, &bx) ||
        !row_maps(W.hs, L.R, P.I, &bh)) {
        WB_SET_ERR(err, WISP_ERR_CUDA, "prefill: cuTensorMapEncodeTiled failed or unavailable");
        return WISP_ERR_CUDA;
    }
    WB_CUDA_RET(ensure_gemm_attrs(), err);
    // the plan kernel rewrites the tile counters; the status word accumulates
    // over the blocks of a stack
    if (reset_status) WB_CUDA_RET(wb::launch_zero_words(W.status, 1, stream), err);
    const int sms = wb::sm_count();
    if (!route) {
        // routing given: straight to the plan
    } else if (T >= kRouterTcMinT) {
        // hi/lo halves of x live in the (not yet used) activation-row buffer
        __half* hi = W.xs;
        __half* lo = W.xs + (size_t)T * P.H;
        RouterMaps rm;
        const cuuint64_t dw[2] = {(cuuint64_t)P.H, (cuuint64_t)P.E}, sw[1] = {(cuuint64_t)P.H * 2};
        const cuuint64_t dx[2] = {(cuuint64_t)P.H, (cuuint64_t)T};
        const cuuint32_t box[2] = {64, 128};
        if (!encode(&rm.w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(P.router_w), dw,
                    sw, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode(&rm.hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, hi, dx, sw, box,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode(&rm.lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, lo, dx, sw, box,
                    CU_TENSOR_MAP_SWIZZLE_128B)) {
            WB_SET_ERR(err, WISP_ERR_CUDA, "prefill: router tensor maps could not be encoded");
            return WISP_ERR_CUDA;
        }
        const long long n4 = (long long)T * P.H / 4;
        WB_CUDA_RET(wb::launch_pdl(split_hilo_kernel,
                                   dim3((unsigned)std::min<long long>((n4 + 255) / 256, 8 * sms)),
                                   dim3(256), 0, stream, x, hi, lo, n4),
                    err);
        WB_CUDA_RET(wb::launch_pdl(router_tc_kernel, dim3((P.E + 127) / 128, (T + 127) / 128),
                                   dim3(192), kRouterSmem, stream, rm, W.logits, T, P.E, P.H,
                                   W.status),
                    err);
    } else {
        const dim3 rg((T + kRouteTile - 1) / kRouteTile, (P.E + kRouteTile - 1) / kRouteTile);
        WB_CUDA_RET(wb::launch_pdl(router_logits_kernel, rg, dim3(256), 0, stream, x, P.router_w,
                                   W.logits, T, P.E, P.H),
                    err);
    }
    if (route)
        WB_CUDA_RET(wb::launch_pdl(route_topk_kernel, dim3(std::min((T + 7) / 8, 4 * sms)),
                                   dim3(256), (size_t)8 * 2 * P.E * 4, stream,
                                   (const float*)W.logits, P.router_bias, T, P.E, P.K, W.idx,
                                   W.w, P.gating),
                    err);
    WB_CUDA_RET(wb::launch_pdl(prefill_plan_kernel, dim3(1), dim3(kPlanThreads),
                               (size_t)5 * (P.E + 2) * 4, stream, P, W, T, wt),
                err);
    WB_CUDA_RET(wb::launch_pdl(prefill_scatter_kernel, dim3(T), dim3(256), 0, stream, P, W, T, x,
                               y),
                err);
    WB_CUDA_RET(wb::launch_pdl(grouped_gemm_kernel<2, 2>, dim3(sms), dim3(kGemmThreads),
                               gemm_smem_bytes<2, 2>(), stream, P, W, bx, y),
                err);
    if (kg_down == 4)
        WB_CUDA_RET(wb::launch_pdl(grouped_gemm_kernel<1, 4>, dim3(sms), dim3(kGemmThreads),
                                   gemm_smem_bytes<1, 4>(), stream, P, W, bh, y),
                    err);
    else
        WB_CUDA_RET(wb::launch_pdl(grouped_gemm_kernel<1, 2>, dim3(sms), dim3(kGemmThreads),
                                   gemm_smem_bytes<1, 2>(), stream, P, W, bh, y),
                    err);
    if (dense_si) {
        char* b = static_cast<char*>(workspace);
        float* dy = reinterpret_cast<float*>(b + L.dy);
        WB_CUDA_RET(wb::launch_dense_ffn(static_cast<const __half*>(layer->shared_gate),
                                         static_cast<const __half*>(layer->shared_up),
                                         static_cast<const __half*>(layer->shared_down),
                                         dense_si, P.H, x, P.H, reinterpret_cast<float*>(b + L.dh),
                                         dy, P.H, T, stream),
                    err);
        WB_CUDA_RET(wb::launch_add_rows(y, dy, (size_t)T * P.H, stream), err);
    }
    return WISP_OK;
}

// Workspace of the stack: one block's workspace, then xn and y [T, H] fp32.
size_t stack_ws_bytes(const WispMoeLayer* l, int T, size_t* block_bytes) {
    const WispExpertMeta& m = l->meta;
    const size_t b = al(make_playout(T, (int)m.cols[0], (int)m.rows[0], l->n_experts,
                                     l->top_k, l->shared_gate ? l->shared_inter : 0).total,
                        1024);
    if (block_bytes) *block_bytes = b;
    return b + 2 * al((size_t)T * m.cols[0] * sizeof(float), 1024);
}

}  // namespace

extern "C" size_t wisp_moe_prefill_workspace_bytes(const WispMoeLayer* layer, int T) {
    if (!layer || T <= 0) return 0;
    const WispExpertMeta& m = layer->meta;
    return make_playout(T, (int)m.cols[0], (int)m.rows[0], layer->n_experts, layer->top_k,
                        layer->shared_gate ? layer->shared_inter : 0)
        .total;
}

extern "C" size_t wisp_moe_prefill_stack_workspace_bytes(const WispMoeLayer* layers, int n_layers,
                                                         int T) {
    if (!layers || n_layers <= 0 || T <= 0) return 0;
    size_t best = 0;
    for (int i = 0; i < n_layers; ++i) best = std::max(best, stack_ws_bytes(&layers[i], T, nullptr));
    return best;
}

extern "C" WispError wisp_moe_prefill_stack_forward(const WispMoeLayer* layers, int n_layers,
                                                    float eps, float* x, int T, int* topk_idx,
                                                    float* topk_w, void* workspace,
                                                    size_t workspace_bytes, cudaStream_t stream,
                                                    WispErrCtx* err) {
    if (!layers || n_layers <= 0 || !x || T <= 0) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill_stack: bad arguments");
        return WISP_ERR_INVALID_ARG;
    }
    const int H = (int)layers[0].meta.cols[0];
    for (int l = 0; l < n_layers; ++l)
        if ((int)layers[l].meta.cols[0] != H) {
            WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill_stack: layers differ in hidden size");
            return WISP_ERR_INVALID_ARG;
        }
    // one block's workspace sized for the largest layer, then xn and y
    size_t bb = 0, need = 0;
    for (int l = 0; l < n_layers; ++l) {
        size_t b = 0;
        need = std::max(need, stack_ws_bytes(&layers[l], T, &b));
        bb = std::max(bb, b);
    }
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 1023)) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG,
                   "prefill_stack: workspace %zu bytes (need %zu, 1024-byte aligned)",
                   workspace_bytes, need);
        return WISP_ERR_INVALID_ARG;
    }
    if (reinterpret_cast<uintptr_t>(x) & 15) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill_stack: x must be 16-byte aligned");
        return WISP_ERR_INVALID_ARG;
    }
    char* ws = static_cast<char*>(workspace);
    float* xn = reinterpret_cast<float*>(ws + bb);
    float* y = reinterpret_cast<float*>(ws + bb + al((size_t)T * H * sizeof(float), 1024));
    const int K = layers[0].top_k;
    for (int l = 0; l < n_layers; ++l) {
        WB_CUDA_RET(wb::launch_pdl(prefill_norm_kernel, dim3(T), dim3(256), 0, stream, x,
                                   (const float*)y,
                                   static_cast<const __half*>(layers[l].norm_w), xn, H, eps,
                                   l > 0 ? 1 : 0, 1),
                    err);
        WispError r = prefill_block(&layers[l], xn, y, T,
                                    topk_idx ? topk_idx + (size_t)l * T * K : nullptr,
                                    topk_w ? topk_w + (size_t)l * T * K : nullptr, workspace, bb,
                                    l == 0, stream, err);
        if (r != WISP_OK) return r;
    }
    WB_CUDA_RET(wb::launch_pdl(prefill_norm_kernel, dim3(T), dim3(256), 0, stream, x,
                               (const float*)y, (const __half*)nullptr, xn, H, eps, 1, 0),
                err);
    return WISP_OK;
}

extern "C" size_t wisp_moe_prefill_routed_workspace_bytes(const WispMoeLayer* layer, int T,
                                                          int K) {
    if (!layer || T <= 0 || K <= 0) return 0;
    const WispExpertMeta& m = layer->meta;
    return make_playout(T, (int)m.cols[0], (int)m.rows[0], layer->n_experts, K).total;
}

extern "C" WispError wisp_moe_prefill_routed(const WispMoeLayer* layer, const float* x, float* y,
                                             int T, int K, const int* topk_idx,
                                             const float* topk_w, void* workspace,
                                             size_t workspace_bytes, cudaStream_t stream,
                                             WispErrCtx* err) {
    if (!layer || !x || !y) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill_routed: NULL layer, x or y");
        return WISP_ERR_INVALID_ARG;
    }
    return prefill_block(layer, x, y, T, const_cast<int*>(topk_idx), const_cast<float*>(topk_w),
                         workspace, workspace_bytes, true, stream, err, /*route=*/false, K);
}

extern "C" WispError wisp_moe_prefill_forward(const WispMoeLayer* layer, const float* x, float* y,
                                              int T, int* topk_idx, float* topk_w,
                                              void* workspace, size_t workspace_bytes,
                                              cudaStream_t stream, WispErrCtx* err) {
    if (!layer || !x || !y) {
        WB_SET_ERR(err, WISP_ERR_INVALID_ARG, "prefill: NULL layer, x or y");
        return WISP_ERR_INVALID_ARG;
    }
    return prefill_block(layer, x, y, T, topk_idx, topk_w, workspace, workspace_bytes, true,
                         stream, err);
}
