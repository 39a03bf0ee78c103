/*
 * wisp_b200.h -- C ABI of the B200-native WISP MoE-block library
 * (libwisp_b200.so, built for sm_100a).
 *
 * Three groups of entry points:
 *
 *  1. The reference's kernel-launcher ABI for the MoE path, with identical C
 *     signatures (reference: csrc/core/wisp_engine.h:549-665).  Each
 *     declaration names the reference launcher it replaces.
 *  2. The fused MoE block (new): router + top-k + int4 gate/up/SwiGLU +
 *     int4 down + gate-weighted combine for T tokens, with no host
 *     synchronisation, on caller-owned device buffers.  The stacked form
 *     adds the RMSNorm + residual between blocks (the FFN half of
 *     decode_step, csrc/core/wisp_engine.c:1563-1570, attention = identity).
 *  3. The engine ABI (reference: csrc/core/wisp_engine.h:472-543): engine
 *     lifecycle on a converted model directory, the 3-tier expert fetch,
 *     cache statistics, the expert access log, prefetch hints, self-tests
 *     and the byte-layout probe; plus the new wisp_moe_forward.
 *
 * Conventions (same as the reference): functions that can fail return
 * WispError and fill a caller-provided WispErrCtx; device buffers are owned
 * by the caller; every launcher takes the stream it runs on.  No entry point
 * falls back to the CPU: without a CUDA device they return WISP_ERR_CUDA.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>
#ifdef __cplusplus
#include <cuda_fp16.h>
typedef __half wisp_half;
#else
typedef uint16_t wisp_half; /* raw fp16 bits; same size/layout as __half */
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------- *
 * Errors -- same codes and context struct as the reference
 * (csrc/core/wisp_engine.h:50-67).
 * ---------------------------------------------------------------------- */
typedef enum {
    WISP_OK = 0,
    WISP_ERR_OOM = 1,
    WISP_ERR_IO = 2,
    WISP_ERR_CUDA = 3,
    WISP_ERR_INVALID_ARG = 4,
    WISP_ERR_EXPERT_MISS = 5,
    WISP_ERR_MODEL = 6,
    WISP_ERR_TIMEOUT = 7,
} WispError;

typedef struct {
    WispError code;
    char message[512];
    const char* file;
    int line;
} WispErrCtx;

/* Expert blob layout, parsed from the 120-byte .bin header
 * (reference: csrc/core/wisp_engine.h:241-251).  `tiled` is set for a blob in
 * the device layout wisp_expert_tile writes (header version 2). */
#define WISP_EXPERT_NMATS 3
typedef struct {
    size_t packed_off[WISP_EXPERT_NMATS];
    size_t scales_off[WISP_EXPERT_NMATS];
    size_t zeros_off[WISP_EXPERT_NMATS];
    uint32_t rows[WISP_EXPERT_NMATS];
    uint32_t cols[WISP_EXPERT_NMATS];
    uint32_t group_size;
    size_t total_bytes;
    int valid;
    int tiled;
} WispExpertMeta;

/* Replaces wisp_expert_parse_header (csrc/core/wisp_engine.c:268-303);
 * also accepts version 2 (tiled) headers. */
WispError wisp_expert_parse_header(const void* blob, size_t blob_size,
                                   WispExpertMeta* meta, WispErrCtx* err);

/* New.  Rewrite a .bin expert blob (device memory, `meta` parsed from its
 * header) into the tiled device layout the fused kernels stream, at dst_blob
 * (device, not overlapping).  Each matrix keeps its place and size; inside it,
 * every 8-row block is contiguous: for each quant group g, the g-th gs/2 code
 * bytes of the block's 8 rows, then for each g the 8 rows' (scale, zero)
 * fp16 pairs.  The header is copied with version 2.  Both blobs start at an
 * address = 8 (mod 16); rows must be multiples of 8.  Asynchronous on
 * `stream`. */
WispError wisp_expert_tile(const WispExpertMeta* meta, const void* src_blob,
                           void* dst_blob, cudaStream_t stream,
                           WispErrCtx* err);

/* ====================================================================== *
 * 1. Reference kernel-launcher ABI (identical signatures)
 * ====================================================================== */

/* Replaces csrc/cuda/matmul.cu:56-62 (wisp_engine.h:552). y = W x. */
void wisp_gpu_gemv_f16(const wisp_half* W, const float* x, float* y,
                       int rows, int cols, cudaStream_t s);
/* Replaces matmul.cu:80-86 (wisp_engine.h:554). y = W^T x. */
void wisp_gpu_gemv_t_f16(const wisp_half* W, const float* x, float* y,
                         int rows, int cols, cudaStream_t s);
/* Replaces matmul.cu:112-117 (wisp_engine.h:556). In-place safe. */
void wisp_gpu_rmsnorm(const float* x, const wisp_half* w, float* y, int n,
                      float eps, cudaStream_t s);
/* Replaces matmul.cu:125-130 (wisp_engine.h:558). x += d. */
void wisp_gpu_residual_add(float* x, const float* delta, int n,
                           cudaStream_t s);
/* Replaces matmul.cu:144-148 (wisp_engine.h:560). out = silu(g)*u. */
void wisp_gpu_swiglu(const float* gate, const float* up, float* out, int n,
                     cudaStream_t s);
/* Replaces matmul.cu:207-213 (wisp_engine.h:562). h = silu(Wg x)*(Wu x). */
void wisp_gpu_swiglu_ffn(const wisp_half* Wg, const wisp_half* Wu,
                         const float* x, float* h, int inter, int cols,
                         cudaStream_t s);
/* Replaces matmul.cu:157-161 (wisp_engine.h:565). acc += w*x. */
void wisp_gpu_scale_accum(float* acc, const float* x, float w, int n,
                          cudaStream_t s);
/* Replaces csrc/cuda/router.cu:140-171 (wisp_engine.h:587).  logits = W x +
 * bias, softmax, k strict-argmax passes, renormalised weights.  out_idx /
 * out_w are HOST pointers, valid after the caller synchronises `s`. */
void wisp_gpu_router_topk(const wisp_half* W, const wisp_half* bias,
                          const float* x, float* logits_scratch,
                          int n_experts, int hidden, int top_k,
                          int* out_idx, float* out_w, cudaStream_t s);
/* Replaces csrc/cuda/expert_loader.cu:46-63 (wisp_engine.h:598).
 * out[i] = fp16((nib(i)-8)*scale[i/gs] + zero[i/gs]). */
cudaError_t launch_dequant_expert(const uint8_t* d_packed,
                                  const wisp_half* d_scales,
                                  const wisp_half* d_zeros,
                                  wisp_half* d_output, int n_elements,
                                  int group_size, cudaStream_t stream);
/* Replaces expert_loader.cu:67-97 (wisp_engine.h:604): 3 H2D copies on
 * `stream`, then dequant. */
cudaError_t async_load_expert(const uint8_t* h_packed,
                              const wisp_half* h_scales,
                              const wisp_half* h_zeros, uint8_t* d_packed_tmp,
                              wisp_half* d_scales_tmp, wisp_half* d_zeros_tmp,
                              wisp_half* d_output, int n_elements,
                              int group_size, cudaStream_t stream);

/* ====================================================================== *
 * 2. Fused MoE block (new; no reference counterpart -- replaces the body of
 *    run_moe, csrc/core/wisp_engine.c:1411-1522, for the all-resident case)
 * ====================================================================== */

/* One MoE layer as the kernels see it.  All pointers are DEVICE pointers
 * except where noted.  Every expert blob of the layer is in the tiled device
 * layout (wisp_expert_tile; meta.tiled set) and has the same shape, described
 * by `meta` (host copy, parsed from any blob's header).  Blobs start at an
 * address = 8 (mod 16), so every section is 16-byte aligned (the engine's
 * VRAM slots do this).  Shape limits: hidden a multiple of 32 and at most
 * 8192, inter a multiple of 32; group_size 32, 64 or 128 dividing both. */
typedef struct {
    WispExpertMeta meta;               /* host copy                        */
    const void* const* expert_blobs;   /* device array [n_experts]         */
    const wisp_half* router_w;         /* [n_experts, hidden] fp16         */
    const wisp_half* router_bias;      /* [n_experts] fp16 or NULL         */
    const wisp_half* norm_w;           /* [hidden] RMSNorm weight (stacks) */
    const void* shared_blob;           /* int4 shared expert blob or NULL  */
    WispExpertMeta shared_meta;        /* host copy; used when shared_blob */
    int n_experts;
    int top_k;
    int gating;                        /* WISP_GATING_* (0 = the reference's) */
    /* The shared expert in the form the reference converter writes it:
     * fp16-dense layers.{i}.shared.{gate,up,down} (gate/up [shared_inter, H],
     * down [H, shared_inter], row-major, 16-byte aligned; shared_inter a
     * multiple of 8), run always-on with weight 1 before the routed experts
     * (csrc/core/wisp_engine.c:1443-1450).  NULL when absent; set at most one
     * of shared_blob and shared_gate. */
    const wisp_half* shared_gate;
    const wisp_half* shared_up;
    const wisp_half* shared_down;
    int shared_inter;
} WispMoeLayer;

/* Gating rules of WispMoeLayer.gating.
 *  SOFTMAX: the reference's (router.cu:60-120, wisp_engine.c:520-556):
 *           p = softmax(logits + bias), k strict-argmax passes (lowest index
 *           wins ties), w_j = p_j / sum of the selected p.
 *  SIGMOID: DeepSeek-V3-style scores, s = sigmoid(logits); the experts are
 *           chosen on s + bias (the bias steers selection only), k strict-argmax
 *           passes as above, w_j = s_j / sum of the selected s.  No reference
 *           implementation exists: parity unpinned, tested against its own
 *           restatement. */
#define WISP_GATING_SOFTMAX 0
#define WISP_GATING_SIGMOID 1

/* Bytes of device workspace wisp_moe_block_forward / wisp_moe_stack_forward
 * need for T tokens (max over the layers passed). */
size_t wisp_moe_workspace_bytes(const WispMoeLayer* layers, int n_layers,
                                int T);

/* y[T,H] = MoE(x[T,H]) for one layer.  x is the block input (the
 * reference's buf_norm); y may not alias x.  topk_idx / topk_w (device,
 * [T, top_k], optional) receive the routing.  workspace: device, at least
 * wisp_moe_workspace_bytes(); contents need no initialisation. */
WispError wisp_moe_block_forward(const WispMoeLayer* layer, const float* x,
                                 float* y, int T, int* topk_idx,
                                 float* topk_w, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream,
                                 WispErrCtx* err);

/* The two halves of wisp_moe_block_forward, for callers that must see the
 * routing on the host between them (e.g. to fetch the routed experts into
 * the table first): _route quantises x and runs router + top-k (the expert
 * table is not read); _experts builds the expert-tile plan from that routing
 * -- reading the table then, after the caller's fetch -- and runs gate/up,
 * down and the combine, in the SAME workspace (same x, T, layer shape,
 * stream; topk_idx/topk_w the same buffers or both NULL). */
WispError wisp_moe_block_route(const WispMoeLayer* layer, const float* x,
                               int T, int* topk_idx, float* topk_w,
                               void* workspace, size_t workspace_bytes,
                               cudaStream_t stream, WispErrCtx* err);
WispError wisp_moe_block_experts(const WispMoeLayer* layer, const float* x,
                                 float* y, int T, int* topk_idx,
                                 float* topk_w, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream,
                                 WispErrCtx* err);

/* New: the experts of one layer on a routing the caller supplies (device
 * topk_idx [T, top_k] of expert indices of THIS layer descriptor, or -1, and
 * topk_w [T, top_k]): y[t] = [shared(x[t])] + sum_j w[t,j] * E_idx[t,j](x[t]).
 * router_w may be NULL.  The expert-parallel path runs each GPU's experts on the
 * token rows dispatched to it (layer->top_k = 1, weights 1). */
WispError wisp_moe_experts_routed(const WispMoeLayer* layer, const float* x,
                                  float* y, int T, const int* topk_idx,
                                  const float* topk_w, void* workspace,
                                  size_t workspace_bytes, cudaStream_t stream,
                                  WispErrCtx* err);
/* New: routing only -- router logits (+bias), softmax and the k strict-argmax
 * passes for T tokens into device topk_idx / topk_w [T, top_k]; the layer's
 * expert table may be NULL.  The expert-parallel path routes on the tokens'
 * home GPU with the full router. */
WispError wisp_moe_route(const WispMoeLayer* layer, const float* x, int T,
                         int* topk_idx, float* topk_w, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream,
                         WispErrCtx* err);
/* New: y[t] += sum_j weights[t,j] * rows[row_idx[t,j]] for j in order
 * (row_idx < 0: skipped) -- the expert-parallel combine on the tokens' home GPU.
 * y [T,H], rows [*,H] fp32 device buffers, row_idx/weights [T,K] device. */
WispError wisp_moe_ep_combine(float* y, const float* rows, const int* row_idx,
                              const float* weights, int T, int K, int H,
                              cudaStream_t stream, WispErrCtx* err);

/* Replaces run_dense_mlp (csrc/core/wisp_engine.c:1524-1534) and the dense
 * shared-expert FFN of run_moe (:1443-1450, op_swiglu_ffn + op_gemv): for T
 * tokens, y[t] = down . (silu(gate . x[t]) * (up . x[t])) with the fp16-dense
 * weights the reference converter writes as layers.{i}.shared.{gate,up,down}
 * (gate/up [inter, hidden], down [hidden, inter], row-major), fp32 math.
 * x, y [T, hidden] fp32 device (16-byte aligned, not aliased); inter and
 * hidden multiples of 8.  workspace: wisp_dense_ffn_workspace_bytes(inter, T)
 * device bytes (the SwiGLU activations).  Launch-only. */
size_t wisp_dense_ffn_workspace_bytes(int inter, int T);
WispError wisp_dense_ffn_forward(const wisp_half* gate, const wisp_half* up,
                                 const wisp_half* down, int inter, int hidden,
                                 const float* x, float* y, int T, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream,
                                 WispErrCtx* err);

/* New: the converter's int4 quantiser on the GPU (wisp/converter/quantizer.py
 * :46-86, bit-identical on fp32 input): w [rows, cols] fp32 device, row-major;
 * per group of group_size consecutive elements zero = (max+min)/2, scale =
 * max((max-min)/15, 1e-8), codes clamp(round_half_even((x-zero)/scale)+8, 0,
 * 15) packed low nibble first into packed [rows*cols/2]; scales, zeros fp16
 * [rows*cols/group_size].  rows*cols must be a multiple of an even group size.
 * Launch-only. */
WispError wisp_quantize_int4(const float* w, int rows, int cols, int group_size,
                             uint8_t* packed, void* scales, void* zeros,
                             cudaStream_t stream, WispErrCtx* err);

/* Multi-GPU helpers of the reference (csrc/cuda/multi_gpu.cu:37-160, declared in
 * csrc/core/wisp_engine.h:656-665), same signatures and codes (0 ok, -1 failure):
 * a single-process NCCL pipeline -- init builds one communicator per GPU of
 * gpu_indices (stage i = gpu_indices[i]); send/recv move n fp32 values between
 * the current device's stage and peer_stage on stream s (issue a matching
 * send and receive from different host threads) -- and 2-GPU peer access /
 * peer copies.  NCCL is loaded at first use; without it wisp_nccl_available()
 * is 0 and the pipeline calls return -1. */
int  wisp_nccl_available(void);
int  wisp_pipeline_init(const int* gpu_indices, int n);
void wisp_pipeline_shutdown(void);
int  wisp_pipeline_send_activation(const float* x, int n, int peer_stage,
                                   cudaStream_t s);
int  wisp_pipeline_recv_activation(float* x, int n, int peer_stage,
                                   cudaStream_t s);
int  wisp_peer_enable(int dev_a, int dev_b);
int  wisp_peer_copy_async(void* dst, int dst_dev, const void* src,
                          int src_dev, size_t n, cudaStream_t s);

/* New: the block for batched / prefill tokens on the tensor cores (tcgen05).
 * Same contract as wisp_moe_block_forward -- x [T,H] fp32 MoE input (already
 * normalised), y [T,H] fp32 output (overwritten), optional device
 * topk_idx/topk_w [T, top_k] -- for T independent tokens of run_moe
 * (csrc/core/wisp_engine.c:1411-1522): the tokens are grouped by expert and
 * every expert runs as one GEMM over its tokens, int4 dequantised to fp16 in
 * shared memory, fp32 accumulation.  Needs tiled experts with group_size 64,
 * hidden and intermediate sizes multiples of 128, and a shared expert (if any)
 * of the routed experts' layout.  Launch-only; the status word (offset 0 of
 * the workspace, wisp_moe_status) reports missing or misaligned experts and
 * timeouts.  workspace: wisp_moe_prefill_workspace_bytes(layer, T) bytes,
 * 1024-byte aligned. */
size_t wisp_moe_prefill_workspace_bytes(const WispMoeLayer* layer, int T);
WispError wisp_moe_prefill_forward(const WispMoeLayer* layer, const float* x,
                                   float* y, int T, int* topk_idx, float* topk_w,
                                   void* workspace, size_t workspace_bytes,
                                   cudaStream_t stream, WispErrCtx* err);

/* New: the routed experts only, on the tensor-core path, for a routing the
 * caller supplies -- y[t] = sum_j w[t,j] * expert_{idx[t,j]}(x[t]) over K slots
 * (idx < 0: skipped), no router, no shared expert.  The expert-parallel owner of
 * dispatched rows calls it with K = 1 and w = 1 (the counterpart of
 * wisp_moe_experts_routed for many rows per expert).  workspace:
 * wisp_moe_prefill_routed_workspace_bytes(layer, T, K), 1024-byte aligned. */
size_t wisp_moe_prefill_routed_workspace_bytes(const WispMoeLayer* layer, int T, int K);
WispError wisp_moe_prefill_routed(const WispMoeLayer* layer, const float* x, float* y,
                                  int T, int K, const int* topk_idx, const float* topk_w,
                                  void* workspace, size_t workspace_bytes,
                                  cudaStream_t stream, WispErrCtx* err);

/* New: stack of n_layers blocks on the prefill path -- per layer l,
 * x <- x + MoE_l(rmsnorm(x; norm_w_l, eps)) (the FFN half of decode_step,
 * csrc/core/wisp_engine.c:1563-1570, attention = identity), each block by
 * wisp_moe_prefill_forward's kernels.  x [T,H] fp32 device, in place;
 * topk_idx/topk_w optional device [n_layers, T, top_k].  Launch-only.
 * workspace: wisp_moe_prefill_stack_workspace_bytes bytes, 1024-byte aligned;
 * its first word is the status word (wisp_moe_status), accumulated over the
 * layers. */
size_t wisp_moe_prefill_stack_workspace_bytes(const WispMoeLayer* layers,
                                              int n_layers, int T);
WispError wisp_moe_prefill_stack_forward(const WispMoeLayer* layers, int n_layers,
                                         float eps, float* x, int T, int* topk_idx,
                                         float* topk_w, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream,
                                         WispErrCtx* err);

/* New: an expert pool in pinned host memory streamed into a device cache of
 * n_slots slots under LRU (the oversubscribed configuration).  Replaces the
 * synchronous VRAM fill of wisp_expert_fetch (csrc/core/wisp_engine.c
 * :891-1078) for a pool held in RAM: a miss is one cudaMemcpyAsync of the
 * tiled blob from the pool into its slot on one of two transfer streams, and
 * events order everything (no host synchronisation):
 *   ensure     -- make ids[n] of `layer` resident; `compute` waits for their
 *                 copies; *hits / *misses of this call;
 *   prefetch   -- start copies for experts predicted for a later layer;
 *   layer_done -- the layer's kernels are queued on `compute`: slots they read
 *                 are not overwritten before those kernels finish.
 * wisp_stream_table(layer) is the device pointer table [n_experts] to put in
 * WispMoeLayer.expert_blobs (NULL entries: not resident).  Host blobs must be
 * tiled (wisp_expert_tile layout), stay valid and pinned while registered.
 * stats: hits, misses, prefetched, prefetched-then-used, bytes copied, slots. */
typedef struct WispStreamCache WispStreamCache;
WispStreamCache* wisp_stream_create(int n_layers, int n_experts, size_t blob_bytes,
                                    size_t n_slots, WispErrCtx* err);
void wisp_stream_destroy(WispStreamCache* c);
WispError wisp_stream_register(WispStreamCache* c, int layer, int expert,
                               const void* host_blob, WispErrCtx* err);
const void* const* wisp_stream_table(WispStreamCache* c, int layer);
WispError wisp_stream_ensure(WispStreamCache* c, int layer, const int* ids, int n,
                             cudaStream_t compute, int* hits, int* misses,
                             WispErrCtx* err);
WispError wisp_stream_prefetch(WispStreamCache* c, int layer, const int* ids, int n,
                               int* issued, WispErrCtx* err);
WispError wisp_stream_layer_done(WispStreamCache* c, int layer, cudaStream_t compute,
                                 WispErrCtx* err);
void wisp_stream_stats(WispStreamCache* c, uint64_t* out6);
/* Forget every resident expert and zero the statistics (a cold cache), after
 * the device is idle.  A layer's slots handed out by ensure stay out of
 * eviction until its layer_done, whatever the caller prefetches in between. */
void wisp_stream_reset(WispStreamCache* c);

/* No counterpart in the reference.  wisp_moe_block_forward without a
 * workspace argument, for callers that cannot allocate device memory: a host
 * binding the library through a plain C FFI with no device allocator of its
 * own, or a serving loop that reserved all device memory up front and must
 * not allocate per step.  The block runs in a fixed 8 MiB device array inside
 * the library (enough for a Mixtral-shaped layer up to T = 16); larger requests
 * fail with WISP_ERR_INVALID_ARG before any GPU work.  Nothing is allocated.
 * The first call on a device looks up the array's address; make that first
 * call before any stream capture.  All calls on a device share the array:
 * calls whose kernels overlap on the GPU race. */
WispError wisp_moe_block_forward_static(const WispMoeLayer* layer,
                                        const float* x, float* y, int T,
                                        int* topk_idx, float* topk_w,
                                        cudaStream_t stream, WispErrCtx* err);
/* The device-side status word (bits as wisp_moe_status) that the last
 * wisp_moe_block_forward_static call on the current device left in the fixed
 * array: a caller of that entry has no workspace pointer to pass to
 * wisp_moe_status.  Synchronises `stream` (the stream of that call); -1 when the
 * read fails.  Allocates nothing. */
int wisp_moe_block_static_status(cudaStream_t stream);

/* Stack of n_layers blocks: per layer l, x <- x + MoE_l(rmsnorm(x; norm_w_l,
 * eps)).  x [T,H] is updated in place.  topk_idx/topk_w optional, device
 * [n_layers, T, top_k].  Launch-only (capturable into a CUDA graph). */
WispError wisp_moe_stack_forward(const WispMoeLayer* layers, int n_layers,
                                 float eps, float* x, int T, int* topk_idx,
                                 float* topk_w, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream,
                                 WispErrCtx* err);

/* Device-side status word the kernels set instead of faulting (bit 0: a
 * weight section was not 16-byte aligned; bit 1: an expert index was out of
 * range or its table entry NULL; bit 2: a plan overflowed; bit 3: a bounded
 * wait timed out; bit 4: a blob was not in the tiled layout).  Synchronises
 * `stream`. */
int wisp_moe_status(const void* workspace, cudaStream_t stream);

/* Profiling hook (new): while `events` is set, the calling thread's
 * block/stack forwards record events[i] on the launch stream before each
 * kernel they launch and one after the last (so n kernels -> n+1 events,
 * durations by cudaEventElapsedTime of neighbours).  The records sit between
 * launches and remove the programmatic overlap, so time the headline
 * without them.  NULL turns the hook off; the count restarts at 0. */
void wisp_moe_profile_events(void* events, int n_events);
/* Events recorded since the hook was set. */
int wisp_moe_profile_count(void);

/* ====================================================================== *
 * 2c. The decoder step's kernels (decoder.cu)
 * ====================================================================== */
/* Replace the launchers of csrc/cuda/attention.cu, kv_cache.cu and the
 * embedding (wisp_engine.h:567-595), same signatures and semantics:
 * embedding row -> fp32; neox rotary on [n_heads][head_stride] at rope_off;
 * fp32 -> fp16 cache rows at pos; softmax(q.K * scale).V over seq_len
 * positions, K [seq][kv_heads][k_dim], V [seq][kv_heads][v_dim] (V == K or
 * NULL: the first v_dim dims of the key), score_scratch [n_heads][seq_len]
 * floats (holds the per-chunk partial results). */
void wisp_gpu_embed_lookup(const wisp_half* table, int token, float* x, int hidden,
                           cudaStream_t s);
void wisp_gpu_rope(float* x, int n_heads, int head_stride, int rope_off, int rope_dim,
                   int pos, float theta, cudaStream_t s);
void wisp_gpu_kv_append(wisp_half* K, wisp_half* V, const float* k, const float* v,
                        int pos, int kv_heads, int k_dim, int v_dim, cudaStream_t s);
void wisp_gpu_attention(const float* q, const wisp_half* Kcache, const wisp_half* Vcache,
                        float* out, float* score_scratch, int seq_len, int n_heads,
                        int kv_heads, int k_dim, int v_dim, float scale, cudaStream_t s);

/* New: one GQA attention block fused for one token (run_attention's GQA
 * branch, wisp_engine.c:1328-1348, with the RMSNorm before it and the
 * residual after it): x[H] += o_proj(attn(rope(q), cache)) with q, k, v the
 * projections of rmsnorm(x; input_norm), k and v stored at `pos` of the
 * layer's cache [max_seq][n_kv_heads][head_dim] (fp16) first.  Weights
 * fp16 row-major, 16-byte aligned; head_dim a multiple of 16 (<= 576);
 * hidden a multiple of 8.  The workspace (wisp_attn_workspace_bytes) must be
 * zero-filled before its first use: it holds the counters of the split
 * projections, which every call leaves at zero. */
typedef struct WispAttnLayer {
    const wisp_half* input_norm; /* [H] (NULL: ones) */
    const wisp_half* q_proj;     /* [n_heads * head_dim, H] */
    const wisp_half* k_proj;     /* [n_kv_heads * head_dim, H] */
    const wisp_half* v_proj;     /* [n_kv_heads * head_dim, H] */
    const wisp_half* o_proj;     /* [H, n_heads * head_dim] */
    int hidden, n_heads, n_kv_heads, head_dim;
    float rope_theta, rms_eps;
} WispAttnLayer;
size_t wisp_attn_workspace_bytes(const WispAttnLayer* layer, int max_seq);
WispError wisp_attn_decode(const WispAttnLayer* layer, float* x, wisp_half* k_cache,
                           wisp_half* v_cache, int pos, int max_seq, void* workspace,
                           size_t workspace_bytes, cudaStream_t s, WispErrCtx* err);
/* New: logits[vocab] = lm_head . rmsnorm(x; final_norm) (decode_step's tail,
 * wisp_engine.c:1575-1579); workspace of hidden floats. */
WispError wisp_lm_head_forward(const wisp_half* final_norm, const wisp_half* lm_head,
                               const float* x, float* logits, int vocab, int hidden, float eps,
                               void* workspace, size_t workspace_bytes, cudaStream_t s,
                               WispErrCtx* err);

/* ====================================================================== *
 * 3. Engine ABI (reference: csrc/core/wisp_engine.h:472-543)
 * ====================================================================== */
typedef struct WispEngine WispEngine;

/* Replaces wisp_engine_create (wisp_engine.c:1914-2094).  Loads
 * manifest.json and dense/model_dense.safetensors from model_path; expert
 * blobs stream from experts/ through the RAM and VRAM LRU tiers.  Requires
 * a GPU (gpu_count >= 1); the first index is the device used. */
WispEngine* wisp_engine_create(const char* model_path,
                               size_t vram_expert_budget_bytes,
                               size_t ram_expert_budget_bytes,
                               const int* gpu_indices, int gpu_count,
                               int omp_threads, WispErrCtx* err);
/* Replaces wisp_engine_destroy (wisp_engine.c:2096-2187). */
void wisp_engine_destroy(WispEngine* eng);

/* Replaces wisp_expert_fetch (wisp_engine.c:920-1078): returns a device
 * pointer to the expert's blob (VRAM tier, or a scratch-ring slot for
 * experts that have not earned a VRAM slot), NULL + err on failure
 * (WISP_ERR_IO = file missing/short; callers skip the expert). */
void* wisp_expert_fetch(WispEngine* eng, uint32_t layer_id,
                        uint32_t expert_id, WispErrCtx* err);
/* New: read a whole expert file into `dst` (capacity `cap`) the way the SSD
 * tier's miss path does (replaces the fopen/fread of wisp_engine.c:351-380):
 * O_DIRECT preads straight into `dst` when it is 4096-byte aligned and `cap`
 * holds the size rounded up to 4096 (a pinned staging buffer), else buffered
 * sequential preads.  Returns the file size, 0 on error (WISP_ERR_IO in `err`);
 * *direct (if non-NULL) = 1 when O_DIRECT was used. */
size_t wisp_read_expert_file(const char* path, void* dst, size_t cap, int* direct,
                             WispErrCtx* err);
/* Replaces wisp_expert_prefetch_hint (wisp_engine.c:1162-1177). */
void wisp_expert_prefetch_hint(WispEngine* eng, int layer_idx,
                               const int* expert_ids, int n);

/* New: one MoE layer on device buffers x/y [T,H] on the engine's compute
 * stream (or `stream` when non-NULL).  If every expert of the layer is
 * VRAM-resident the whole block runs without a host sync; otherwise the
 * router runs first, the host fetches the routed experts through the
 * tiers, then the expert kernels run. */
WispError wisp_moe_forward(WispEngine* eng, int layer, const float* x,
                           float* y, int T, cudaStream_t stream,
                           WispErrCtx* err);
/* New: the decode form of wisp_moe_forward: one token, y[H] = MoE_l(x[H]).
 * With the layer's experts VRAM-resident it enqueues the fused block with no
 * host synchronisation (graph-capturable); otherwise it takes the miss path of
 * wisp_moe_forward. */
WispError wisp_moe_decode(WispEngine* eng, int layer, const float* x, float* y,
                          cudaStream_t stream, WispErrCtx* err);
/* New: x <- x + MoE_l(rmsnorm(x)) for layers [layer0, layer0+n). */
WispError wisp_moe_stack(WispEngine* eng, int layer0, int n_layers, float* x,
                         int T, cudaStream_t stream, WispErrCtx* err);
/* New: load every expert of layers [layer0, layer0+n) into the VRAM tier
 * (until the budget is full).  Returns the number of experts resident. */
int wisp_engine_pin_experts(WispEngine* eng, int layer0, int n_layers,
                            WispErrCtx* err);
/* New: the device stream the engine computes on. */
cudaStream_t wisp_engine_stream(WispEngine* eng);
/* New: hidden size, experts per layer, top-k, layers (for callers). */
void wisp_engine_dims(WispEngine* eng, int* hidden, int* n_experts,
                      int* top_k, int* n_layers);

/* ---------------------------------------------------------------------- *
 * The decoder step around the MoE block (GQA models).  The engine loads the
 * dense file's embed_tokens, final_norm, lm_head and per-layer input_norm /
 * attn.{q,k,v,o}_proj (loader wisp_engine.c:1698-1760); MLA and KDA models
 * are refused by these calls (WISP_ERR_MODEL).
 * ---------------------------------------------------------------------- */
typedef struct WispKVCache WispKVCache;

/* Replaces wisp_kv_cache_alloc (wisp_engine.c:2191-2232): an fp16 K and V
 * cache of max_seq_len positions per layer on the engine's device, layout
 * [layer][pos][n_kv_heads][head_dim]. */
WispKVCache* wisp_kv_cache_alloc(WispEngine* eng, int max_seq_len, WispErrCtx* err);
/* Replace wisp_kv_cache_free / _clear / _rollback (wisp_engine.c:2234-2259). */
void wisp_kv_cache_free(WispEngine* eng, WispKVCache* kv);
void wisp_kv_cache_clear(WispEngine* eng, WispKVCache* kv);
void wisp_kv_cache_rollback(WispEngine* eng, WispKVCache* kv, int n_tokens);
/* New: positions held by the cache. */
int wisp_kv_cache_len(const WispKVCache* kv);

/* Replace wisp_prefill / wisp_decode_one / wisp_verify_tokens
 * (wisp_engine.c:2263-2303) and their decode_step (:1537-1595): embed the
 * token, per layer x += attention(rmsnorm(x)) and x += FFN(rmsnorm(x)) (the
 * MoE block through the tiers, or the dense MLP), then the logits of
 * rmsnorm(x) through lm_head, copied to the host array out_logits [vocab]
 * (prefill: the last token's; verify: one row per token).  Tokens out of
 * [0, vocab) and a full cache are refused with WISP_ERR_INVALID_ARG. */
WispError wisp_prefill(WispEngine* eng, const int* token_ids, int n_tokens,
                       WispKVCache* kv, float* out_logits, WispErrCtx* err);
WispError wisp_decode_one(WispEngine* eng, int token_id, WispKVCache* kv,
                          float* out_logits, WispErrCtx* err);
WispError wisp_verify_tokens(WispEngine* eng, const int* token_ids, int n_tokens,
                             WispKVCache* kv, float* out_logits, WispErrCtx* err);
/* New: vocabulary size of the engine's model (0 without a decoder). */
int wisp_engine_vocab(WispEngine* eng);

/* Replace wisp_cache_stats / wisp_cache_clear_all / wisp_ram_trim /
 * wisp_drain_expert_log / wisp_vram_used / wisp_ram_used / wisp_tok_per_sec
 * (wisp_engine.c:872-889, 2305-2367), same semantics. */
void wisp_cache_stats(WispEngine* eng, uint64_t* vram_hits,
                      uint64_t* ram_hits, uint64_t* ssd_hits,
                      double* hit_rate);
void wisp_cache_clear_all(WispEngine* eng);
int wisp_ram_trim(WispEngine* eng, int count);
int wisp_drain_expert_log(WispEngine* eng, uint32_t* out, int max_out,
                          uint64_t* dropped_out);
size_t wisp_vram_used(WispEngine* eng);
size_t wisp_ram_used(WispEngine* eng);
double wisp_tok_per_sec(WispEngine* eng);

/* Replace the self-tests (lru_cache.c:213-270, double_buffer.c:184-229):
 * host-only, return 1 on success. */
int wisp_selftest_lru(void);
int wisp_selftest_double_buffer(void);

/* Replaces wisp_debug_expert_probe (wisp_engine.c:311-349): parse a .bin
 * and dequantise the first n values of matrix `mat` (host arithmetic, the
 * byte-layout cross-check the reference's tests call). */
WispError wisp_debug_expert_probe(const char* path, int mat, int n,
                                  float* out_values, WispExpertMeta* out_meta,
                                  WispErrCtx* err);

/* Library identity: "wisp_b200 <version> sm_100a". */
const char* wisp_b200_version(void);

#ifdef __cplusplus
}
#endif
