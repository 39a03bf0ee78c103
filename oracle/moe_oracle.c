/*
 * moe_oracle.c -- TEST INFRASTRUCTURE ONLY: a CPU restatement of the WISP MoE
 * block forward, used as the checker for the CUDA path and as the "port"
 * CPU baseline.  Nothing in the product links or calls this file.
 *
 * Every function restates the reference's CPU arithmetic in the same order,
 * so that (compiled with the same flags, no FMA contraction) it reproduces the
 * reference harness (oracle/ref_harness.c) bit for bit:
 *
 *   half_to_float     -- IEEE binary16 -> binary32 (wisp_engine.c:53-75)
 *   router_topk       -- fp16 GEMV + bias, softmax with expf, k argmax passes
 *                        with strict '>' (lowest index wins), renormalise
 *                        (wisp_engine.c:520-556)
 *   gemv_int4         -- y[r] = sum_c ((nib-8)*s_g + z_g) * x[c], low nibble =
 *                        even flat index, g = flat/gs (wisp_engine.c:560-579)
 *   swiglu            -- g/(1+expf(-g)) * u (wisp_engine.c:428-433)
 *   gemv_f16          -- dense fp16 GEMV for the shared expert (:389-400)
 *   moe_block         -- run_moe's CPU branch: router, zero acc, shared expert
 *                        (w = 1), routed experts in top-k order; an expert
 *                        whose blob is absent (file unreadable: fetch gives
 *                        WISP_ERR_IO) is skipped (wisp_engine.c:1411-1493,
 *                        1473-1477, 1383-1409)
 *   dense_ffn         -- run_dense_mlp: the fp16-dense SwiGLU FFN of a
 *                        router-less layer (wisp_engine.c:1524-1534)
 *   rmsnorm           -- double sum of squares, float scale (:415-422)
 *   stack             -- x += ffn(rmsnorm(x)) per layer, ffn = dense_ffn for
 *                        a router-less layer else moe_block (decode_step's
 *                        FFN half, :1563-1570, attention taken as identity)
 *
 * Expert blobs are in the .bin layout (wisp/converter/partitioner.py:11-26):
 * 120-byte header, then packed|scales|zeros for gate, up, down.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define HDR_BYTES 120

static float half_to_float(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31;
    int e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu;
    uint32_t out;
    if (e == 31) {
        out = s | 0x7F800000u | (m << 13);
    } else if (e == 0) {
        if (m == 0) {
            out = s;
        } else {
            /* subnormal: renormalise the mantissa */
            int shift = 0;
            while ((m & 0x400u) == 0) { m <<= 1; shift++; }
            m &= 0x3FFu;
            out = s | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (m << 13);
        }
    } else {
        out = s | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &out, sizeof f);
    return f;
}

typedef struct {
    uint32_t rows, cols;
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* zeros;
} QView;

/* Views of the three matrices of a blob; returns group size, 0 on a bad blob. */
static uint32_t blob_views(const uint8_t* blob, QView v[3]) {
    uint32_t hdr[6];
    memcpy(hdr, blob, sizeof hdr);
    if (hdr[0] != 0x57455850u || hdr[1] != 1u || hdr[5] != 3u) return 0;
    size_t off = HDR_BYTES;
    for (int m = 0; m < 3; m++) {
        const uint8_t* rec = blob + 24 + 32 * m;
        uint32_t rc[2];
        uint64_t sz[3];
        memcpy(rc, rec, 8);
        memcpy(sz, rec + 8, 24);
        v[m].rows = rc[0];
        v[m].cols = rc[1];
        v[m].packed = blob + off;
        v[m].scales = (const uint16_t*)(blob + off + sz[0]);
        v[m].zeros = (const uint16_t*)(blob + off + sz[0] + sz[1]);
        off += sz[0] + sz[1] + sz[2];
    }
    return hdr[4];
}

static void gemv_int4(const QView* q, uint32_t gs, const float* x, float* y) {
    long rows = (long)q->rows;
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; r++) {
        size_t base = (size_t)r * q->cols;
        float acc = 0.f;
        for (uint32_t c = 0; c < q->cols; c++) {
            size_t i = base + c;
            uint8_t b = q->packed[i >> 1];
            int code = (i & 1) ? (b >> 4) : (b & 0x0F);
            size_t g = i / gs;
            float s = half_to_float(q->scales[g]);
            float z = half_to_float(q->zeros[g]);
            acc += ((float)(code - 8) * s + z) * x[c];
        }
        y[r] = acc;
    }
}

static void gemv_f16(const uint16_t* W, const float* x, float* y, int rows,
                     int cols) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const uint16_t* row = W + (size_t)r * cols;
        float acc = 0.f;
        for (int c = 0; c < cols; c++) acc += half_to_float(row[c]) * x[c];
        y[r] = acc;
    }
}

static void swiglu(const float* g, const float* u, float* h, int n) {
    for (int i = 0; i < n; i++) h[i] = g[i] / (1.f + expf(-g[i])) * u[i];
}

/* Router: logits, softmax, k strict-argmax passes, renormalise. */
void oracle_router_topk(const uint16_t* W, const uint16_t* bias,
                        const float* x, int E, int H, int k, int* idx,
                        float* w, float* probs_out) {
    float* p = (float*)malloc((size_t)E * sizeof(float));
    gemv_f16(W, x, p, E, H);
    if (bias)
        for (int e = 0; e < E; e++) p[e] += half_to_float(bias[e]);
    float mx = -1e30f;
    for (int e = 0; e < E; e++)
        if (p[e] > mx) mx = p[e];
    float den = 0.f;
    for (int e = 0; e < E; e++) {
        p[e] = expf(p[e] - mx);
        den += p[e];
    }
    for (int e = 0; e < E; e++) p[e] /= den;
    float sum = 0.f;
    for (int j = 0; j < k; j++) {
        int best = -1;
        float bv = -1.f;
        for (int e = 0; e < E; e++) {
            int used = 0;
            for (int i = 0; i < j; i++) used |= (idx[i] == e);
            if (!used && p[e] > bv) { bv = p[e]; best = e; }
        }
        idx[j] = best;
        w[j] = bv;
        sum += bv;
    }
    if (sum > 0.f)
        for (int j = 0; j < k; j++) w[j] /= sum;
    if (probs_out) memcpy(probs_out, p, (size_t)E * sizeof(float));
    free(p);
}

/* One MoE block for T tokens.  blobs[e] = expert e's .bin blob; shared_* =
 * fp16 dense shared expert (NULL = none; shared_inter rows).  y: [T,H]. */
int oracle_moe_block(const uint16_t* router_w, const uint16_t* router_bias,
                     int E, int H, int k, const uint8_t* const* blobs,
                     const uint16_t* shared_gate, const uint16_t* shared_up,
                     const uint16_t* shared_down, int shared_inter,
                     const float* x, int T, float* y, int* idx, float* w,
                     int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    int max_i = shared_inter;
    for (int e = 0; e < E; e++) {
        QView v[3];
        if (!blobs[e]) continue; /* absent file: skipped when routed */
        if (!blob_views(blobs[e], v)) return 6;
        if ((int)v[0].rows > max_i) max_i = (int)v[0].rows;
    }
    float* g = (float*)malloc((size_t)max_i * sizeof(float));
    float* u = (float*)malloc((size_t)max_i * sizeof(float));
    float* h = (float*)malloc((size_t)max_i * sizeof(float));
    float* yy = (float*)malloc((size_t)H * sizeof(float));
    int* ti = (int*)malloc((size_t)k * sizeof(int));
    float* tw = (float*)malloc((size_t)k * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * H;
        float* acc = y + (size_t)t * H;
        oracle_router_topk(router_w, router_bias, xt, E, H, k, ti, tw, NULL);
        memset(acc, 0, (size_t)H * sizeof(float));
        if (shared_gate && shared_up && shared_down) {
            gemv_f16(shared_gate, xt, g, shared_inter, H);
            gemv_f16(shared_up, xt, u, shared_inter, H);
            swiglu(g, u, h, shared_inter);
            gemv_f16(shared_down, h, yy, H, shared_inter);
            for (int i = 0; i < H; i++) acc[i] += 1.0f * yy[i];
        }
        for (int j = 0; j < k; j++) {
            if (ti[j] < 0 || !blobs[ti[j]]) continue; /* run_moe: IO miss -> skip */
            QView v[3];
            uint32_t gs = blob_views(blobs[ti[j]], v);
            gemv_int4(&v[0], gs, xt, g);
            gemv_int4(&v[1], gs, xt, u);
            swiglu(g, u, h, (int)v[0].rows);
            gemv_int4(&v[2], gs, h, yy);
            for (int i = 0; i < H; i++) acc[i] += tw[j] * yy[i];
        }
        if (idx) memcpy(idx + (size_t)t * k, ti, (size_t)k * sizeof(int));
        if (w) memcpy(w + (size_t)t * k, tw, (size_t)k * sizeof(float));
    }
    free(g); free(u); free(h); free(yy); free(ti); free(tw);
    return 0;
}

/* The expert half of run_moe on a given routing (idx/w [T,k]; idx < 0 or an
 * absent blob: skipped): zero acc, fp16 shared expert (w = 1), then the routed
 * experts in slot order -- the same arithmetic as oracle_moe_block, used to
 * check a token whose routing differs from the reference's only by a near-tie
 * against the experts it was actually routed to. */
int oracle_experts_routed(int E, int H, int k, const uint8_t* const* blobs,
                          const uint16_t* shared_gate, const uint16_t* shared_up,
                          const uint16_t* shared_down, int shared_inter,
                          const float* x, int T, const int* idx, const float* w,
                          float* y, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    int max_i = shared_inter;
    for (int e = 0; e < E; e++) {
        QView v[3];
        if (!blobs[e]) continue;
        if (!blob_views(blobs[e], v)) return 6;
        if ((int)v[0].rows > max_i) max_i = (int)v[0].rows;
    }
    float* g = (float*)malloc((size_t)max_i * sizeof(float));
    float* u = (float*)malloc((size_t)max_i * sizeof(float));
    float* h = (float*)malloc((size_t)max_i * sizeof(float));
    float* yy = (float*)malloc((size_t)H * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * H;
        float* acc = y + (size_t)t * H;
        memset(acc, 0, (size_t)H * sizeof(float));
        if (shared_gate && shared_up && shared_down) {
            gemv_f16(shared_gate, xt, g, shared_inter, H);
            gemv_f16(shared_up, xt, u, shared_inter, H);
            swiglu(g, u, h, shared_inter);
            gemv_f16(shared_down, h, yy, H, shared_inter);
            for (int i = 0; i < H; i++) acc[i] += 1.0f * yy[i];
        }
        for (int j = 0; j < k; j++) {
            const int e = idx[(size_t)t * k + j];
            if (e < 0 || e >= E || !blobs[e]) continue;
            QView v[3];
            uint32_t gs = blob_views(blobs[e], v);
            gemv_int4(&v[0], gs, xt, g);
            gemv_int4(&v[1], gs, xt, u);
            swiglu(g, u, h, (int)v[0].rows);
            gemv_int4(&v[2], gs, h, yy);
            const float wj = w[(size_t)t * k + j];
            for (int i = 0; i < H; i++) acc[i] += wj * yy[i];
        }
    }
    free(g); free(u); free(h); free(yy);
    return 0;
}

/* run_dense_mlp for T tokens: y = down . (silu(gate . x) * (up . x)), gate/up
 * [inter, H], down [H, inter] fp16 bits. */
int oracle_dense_ffn(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                     int inter, int H, const float* x, int T, float* y, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    float* g = (float*)malloc((size_t)inter * sizeof(float));
    float* u = (float*)malloc((size_t)inter * sizeof(float));
    float* h = (float*)malloc((size_t)inter * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * H;
        gemv_f16(gate, xt, g, inter, H);
        gemv_f16(up, xt, u, inter, H);
        swiglu(g, u, h, inter);
        gemv_f16(down, h, y + (size_t)t * H, H, inter);
    }
    free(g); free(u); free(h);
    return 0;
}

void oracle_rmsnorm(const float* x, const uint16_t* wn, float* y, int n,
                    float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * x[i];
    float sc = (float)(1.0 / sqrt(ss / n + eps));
    for (int i = 0; i < n; i++) y[i] = x[i] * sc * half_to_float(wn[i]);
}

/* Stack: per layer l, x <- x + moe_l(rmsnorm(x; norm_w[l])).  Arrays of
 * per-layer pointers; blobs is [L][E] flattened.  x: [T,H] in place. */
int oracle_stack(int L, const uint16_t* const* router_w,
                 const uint16_t* const* router_bias,
                 const uint16_t* const* norm_w, float eps, int E, int H, int k,
                 const uint8_t* const* blobs, const float* x_in, float* x,
                 int T, int* idx, float* w, int threads) {
    float* xn = (float*)malloc((size_t)H * sizeof(float));
    float* f = (float*)malloc((size_t)H * sizeof(float));
    if (x != x_in) memcpy(x, x_in, (size_t)T * H * sizeof(float));
    for (int t = 0; t < T; t++) {
        float* xt = x + (size_t)t * H;
        for (int l = 0; l < L; l++) {
            oracle_rmsnorm(xt, norm_w[l], xn, H, eps);
            size_t o = ((size_t)t * L + l) * k;
            int rc = oracle_moe_block(router_w[l], router_bias ? router_bias[l] : NULL,
                                      E, H, k, blobs + (size_t)l * E, NULL, NULL,
                                      NULL, 0, xn, 1, f, idx ? idx + o : NULL,
                                      w ? w + o : NULL, threads);
            if (rc) { free(xn); free(f); return rc; }
            for (int i = 0; i < H; i++) xt[i] += f[i];
        }
    }
    free(xn);
    free(f);
    return 0;
}

/* Stack over layers of any kind: router_w[l] NULL = a dense-MLP layer whose FFN
 * is shared_*[l] alone; else an MoE layer with the fp16 shared expert
 * shared_*[l] (NULL = none).  blobs [L][E] flattened (NULL = absent file).
 * idx/w (optional) [T, L, k]; a dense layer leaves -1 / 0 there. */
int oracle_stack_layers(int L, const uint16_t* const* router_w,
                        const uint16_t* const* router_bias,
                        const uint16_t* const* norm_w, float eps, int E, int H, int k,
                        const uint8_t* const* blobs, const uint16_t* const* shared_gate,
                        const uint16_t* const* shared_up,
                        const uint16_t* const* shared_down, const int* shared_inter,
                        const float* x_in, float* x, int T, int* idx, float* w,
                        int threads) {
    float* xn = (float*)malloc((size_t)H * sizeof(float));
    float* f = (float*)malloc((size_t)H * sizeof(float));
    if (x != x_in) memcpy(x, x_in, (size_t)T * H * sizeof(float));
    for (int t = 0; t < T; t++) {
        float* xt = x + (size_t)t * H;
        for (int l = 0; l < L; l++) {
            oracle_rmsnorm(xt, norm_w[l], xn, H, eps);
            size_t o = ((size_t)t * L + l) * k;
            int rc;
            const int si = shared_inter ? shared_inter[l] : 0;
            if (!router_w[l]) {
                rc = oracle_dense_ffn(shared_gate[l], shared_up[l], shared_down[l], si, H, xn,
                                      1, f, threads);
                for (int j = 0; j < k; j++) {
                    if (idx) idx[o + j] = -1;
                    if (w) w[o + j] = 0.f;
                }
            } else {
                rc = oracle_moe_block(router_w[l], router_bias ? router_bias[l] : NULL, E, H,
                                      k, blobs + (size_t)l * E,
                                      si ? shared_gate[l] : NULL, si ? shared_up[l] : NULL,
                                      si ? shared_down[l] : NULL, si, xn, 1, f,
                                      idx ? idx + o : NULL, w ? w + o : NULL, threads);
            }
            if (rc) { free(xn); free(f); return rc; }
            for (int i = 0; i < H; i++) xt[i] += f[i];
        }
    }
    free(xn);
    free(f);
    return 0;
}

/* Dequantise the first n values of matrix `mat` of a blob (fp32). */
int oracle_dequant(const uint8_t* blob, int mat, long n, float* out) {
    QView v[3];
    uint32_t gs = blob_views(blob, v);
    if (!gs || mat < 0 || mat > 2) return 4;
    for (long i = 0; i < n; i++) {
        uint8_t b = v[mat].packed[i >> 1];
        int code = (i & 1) ? (b >> 4) : (b & 0x0F);
        long g = i / gs;
        out[i] = (float)(code - 8) * half_to_float(v[mat].scales[g]) +
                 half_to_float(v[mat].zeros[g]);
    }
    return 0;
}
