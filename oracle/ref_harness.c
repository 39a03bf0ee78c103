/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Builds the reference WISP engine's own CPU MoE forward from its unmodified
 * sources and exposes it through a tiny C ABI, so tests and the CPU baseline
 * can call the reference's `run_moe` (csrc/core/wisp_engine.c:1411-1522) on a
 * converted-model directory.  The reference file is textually included because
 * `run_moe` and `cpu_rmsnorm` are `static` there; nothing of it is copied.
 *
 * Compiled by oracle/build.py with -DWISP_NO_CUDA -fopenmp into
 * oracle/_ref/libwisp_ref.so.  The engine runs in CPU mode (gpu_count = 0):
 * router = cpu_router_topk (wisp_engine.c:520-556), experts = cpu_expert_ffn
 * (:1383-1409) reading RAM-tier blobs fetched by wisp_expert_fetch (:920-1078).
 */
#include "wisp_engine.c"

#include <stdlib.h>

/* Open a converted model directory in CPU mode. Returns NULL on failure and
 * writes the reference's error text to errbuf. */
void* ref_open(const char* model_dir, unsigned long long ram_budget_bytes,
               int threads, char* errbuf, int errlen) {
    WispErrCtx err;
    memset(&err, 0, sizeof(err));
    WispEngine* eng = wisp_engine_create(model_dir, 0, (size_t)ram_budget_bytes,
                                         NULL, 0, threads, &err);
    if (!eng && errbuf && errlen > 0)
        snprintf(errbuf, (size_t)errlen, "[%d] %s", (int)err.code, err.message);
    return eng;
}

void ref_close(void* h) { wisp_engine_destroy((WispEngine*)h); }

int ref_hidden(void* h) { return ((WispEngine*)h)->cfg.hidden; }
int ref_top_k(void* h) { return ((WispEngine*)h)->cfg.top_k; }

/* The FFN of one layer as decode_step runs it (wisp_engine.c:1564-1568):
 * run_dense_mlp for a router-less layer, else run_moe. */
static WispError ref_ffn(WispEngine* eng, int layer, WispErrCtx* err) {
    if (eng->layers[layer].is_dense_mlp) return run_dense_mlp(eng, layer);
    return run_moe(eng, layer, err);
}

/* One MoE block on T tokens (T sequential run_moe calls: the reference has
 * no batched path; a dense-MLP layer runs run_dense_mlp and leaves idx/w
 * at -1/0).  x: [T,H] normalised input; y: [T,H] block output (buf_ffn);
 * idx/w: [T,k] routing (host_topk_*).  Returns WispError. */
int ref_moe(void* h, int layer, const float* x, int T, float* y, int* idx,
            float* w) {
    WispEngine* eng = (WispEngine*)h;
    int H = eng->cfg.hidden, K = eng->cfg.top_k;
    for (int t = 0; t < T; t++) {
        WispErrCtx err;
        memset(&err, 0, sizeof(err));
        memcpy(eng->buf_norm, x + (size_t)t * H, (size_t)H * sizeof(float));
        WispError e = ref_ffn(eng, layer, &err);
        if (e != WISP_OK) return (int)e;
        memcpy(y + (size_t)t * H, eng->buf_ffn, (size_t)H * sizeof(float));
        const int dense = eng->layers[layer].is_dense_mlp;
        for (int j = 0; j < K; j++) {
            if (idx) idx[(size_t)t * K + j] = dense ? -1 : eng->host_topk_idx[j];
            if (w) w[(size_t)t * K + j] = dense ? 0.f : eng->host_topk_w[j];
        }
    }
    return 0;
}

/* The FFN half of decode_step (wisp_engine.c:1563-1570) over a layer range
 * with attention taken as identity: per layer x <- x + run_moe(rmsnorm(x)).
 * Dense-MLP layers run run_dense_mlp, as decode_step does.
 * x: [T,H] updated in place. idx/w (optional): [T, n_layers, k]. */
int ref_stack(void* h, int layer0, int n_layers, float* x, int T, int* idx,
              float* w) {
    WispEngine* eng = (WispEngine*)h;
    WispModelConfig* c = &eng->cfg;
    int H = c->hidden, K = c->top_k;
    for (int t = 0; t < T; t++) {
        float* xt = x + (size_t)t * H;
        for (int l = 0; l < n_layers; l++) {
            int layer = layer0 + l;
            WispErrCtx err;
            memset(&err, 0, sizeof(err));
            cpu_rmsnorm(xt, eng->layers[layer].post_norm, eng->buf_norm, H,
                        c->rms_eps);
            WispError e = ref_ffn(eng, layer, &err);
            if (e != WISP_OK) return (int)e;
            cpu_residual_add(xt, eng->buf_ffn, H);
            size_t o = ((size_t)t * n_layers + l) * K;
            const int dense = eng->layers[layer].is_dense_mlp;
            for (int j = 0; j < K; j++) {
                if (idx) idx[o + j] = dense ? -1 : eng->host_topk_idx[j];
                if (w) w[o + j] = dense ? 0.f : eng->host_topk_w[j];
            }
        }
    }
    return 0;
}

/* Expert-fetch tier statistics of the reference engine. */
void ref_cache_stats(void* h, unsigned long long* out3) {
    uint64_t v, r, s;
    double rate;
    wisp_cache_stats((WispEngine*)h, &v, &r, &s, &rate);
    out3[0] = v; out3[1] = r; out3[2] = s;
}

/* The reference's byte-layout probe (wisp_engine.c:311-349). */
int ref_probe(const char* path, int mat, int n, float* out) {
    WispErrCtx err;
    WispExpertMeta meta;
    memset(&err, 0, sizeof(err));
    return (int)wisp_debug_expert_probe(path, mat, n, out, &meta, &err);
}

/* The reference's whole decoder step (decode_step, wisp_engine.c:1537-1595)
 * for n tokens from an empty KV cache of max_seq positions: logits [n][vocab]
 * (wisp_verify_tokens, :2288-2303).  Returns the WispError code. */
int ref_vocab(void* h) { return ((WispEngine*)h)->cfg.vocab; }

int ref_decode(void* h, const int* tokens, int n, int max_seq, float* logits) {
    WispEngine* eng = (WispEngine*)h;
    WispErrCtx err;
    memset(&err, 0, sizeof(err));
    WispKVCache* kv = wisp_kv_cache_alloc(eng, max_seq, &err);
    if (!kv) return (int)err.code;
    WispError e = wisp_verify_tokens(eng, tokens, n, kv, logits, &err);
    wisp_kv_cache_free(eng, kv);
    return (int)e;
}
