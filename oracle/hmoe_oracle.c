/*
 * hmoe_oracle.c -- CPU restatement of the HyperMoE sparse-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path in
 * hypermoe-engine_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product never calls it and
 * has no CPU fallback that could route through it.
 *
 * Every function restates one function of the reference (paths are relative
 * to the HyperMoE source tree) with the same floating-point operation order,
 * so that results are bit-identical to the reference's CPU backend:
 *
 *   hmo_route_batch     src/router/CpuRouterBackend.cpp:35-91 (routeToken)
 *                       and :125-160 (routeBatch grouping)
 *   hmo_int8_matmul     src/tensor/backend/CpuTensorBackend.cpp:133-190
 *   hmo_silu            src/tensor/activation/Activation.cpp:44
 *   hmo_expert_mlp      src/experts/ExpertExecutor.cpp:43-138
 *   hmo_moe_layer[_threads]
 *                       src/core/runtime/MoERuntime.cpp:58-349 (CPU branch:
 *                       host gather :288-298, combine :311-325)
 *   hmo_quantize_int8   src/tensor/quantization/Quantization.cpp:45-79
 *
 * Parity pin: tests/test_oracle_golden.py checks these functions against
 * fixtures produced by the unmodified reference sources (oracle/_ref, built
 * by oracle/Makefile) and against the reference tests' known answers.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (see oracle/Makefile).
 * -ffp-contract=off keeps a*b+c as two roundings, as the reference's x86-64
 * build does (no FMA in the baseline ISA).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HMO_OK 0
#define HMO_INVALID 1
#define HMO_NON_FINITE 2

/* ---------------------------------------------------------------- router */

/* One token: logits, softmax, top-k by (score desc, id asc), renorm.
 * Restates CpuRouterBackend.cpp:35-91.  `bias` (may be NULL) is a build
 * addition used by the Zipf-skewed configurations: it enters the logit as
 * the final term of the double accumulation, which is exactly what the
 * reference computes when the hidden row is extended by a constant 1 and
 * the router weight by a bias row. */
static int route_token(const float *hidden, const float *weights,
                       const float *bias, size_t H, size_t E, size_t k,
                       int softmax, int renorm, float *scores_scratch,
                       uint32_t *order_scratch, uint32_t *ids, float *out) {
    for (size_t e = 0; e < E; ++e) {
        double s = 0.0;
        for (size_t i = 0; i < H; ++i)
            s += (double)hidden[i] * (double)weights[i * E + e];
        if (bias) s += 1.0 * (double)bias[e];
        if (!isfinite(s)) return HMO_NON_FINITE;
        scores_scratch[e] = (float)s;
    }
    if (softmax) {
        float m = scores_scratch[0];
        for (size_t e = 1; e < E; ++e)
            if (scores_scratch[e] > m) m = scores_scratch[e];
        double den = 0.0;
        for (size_t e = 0; e < E; ++e) {
            scores_scratch[e] = expf(scores_scratch[e] - m);
            den += scores_scratch[e];
        }
        if (!isfinite(den) || den <= 0.0) return HMO_NON_FINITE;
        for (size_t e = 0; e < E; ++e)
            scores_scratch[e] = (float)((double)scores_scratch[e] / den);
    }
    /* partial_sort with comparator (score desc, id asc): the first k of a
     * strict total order, so a selection sort gives the same sequence. */
    for (size_t e = 0; e < E; ++e) order_scratch[e] = (uint32_t)e;
    for (size_t r = 0; r < k; ++r) {
        size_t best = r;
        for (size_t j = r + 1; j < E; ++j) {
            uint32_t a = order_scratch[j], b = order_scratch[best];
            float sa = scores_scratch[a], sb = scores_scratch[b];
            if (sa == sb ? a < b : sa > sb) best = j;
        }
        uint32_t t = order_scratch[r];
        order_scratch[r] = order_scratch[best];
        order_scratch[best] = t;
    }
    for (size_t r = 0; r < k; ++r) {
        ids[r] = order_scratch[r];
        out[r] = scores_scratch[order_scratch[r]];
    }
    if (renorm) {
        double sum = 0.0; /* std::accumulate(..., 0.0) */
        for (size_t r = 0; r < k; ++r) sum += out[r];
        if (!isfinite(sum) || sum == 0.0) return HMO_NON_FINITE;
        for (size_t r = 0; r < k; ++r) out[r] = (float)((double)out[r] / sum);
    }
    return HMO_OK;
}

/* Batch routing + expert grouping (CpuRouterBackend.cpp:125-160).
 * ids/scores: [T,k] in rank order.  Grouping is returned in CSR form:
 * offsets[E+1]; group e holds tokens in ascending order (tokens are visited
 * in order and appended), with the token's routing score for that expert.
 * Groups of unselected experts are empty; the reference's group list sorted
 * by expert id is the list of non-empty groups in e order. */
int hmo_route_batch(const float *hidden, const float *weights,
                    const float *bias, size_t T, size_t H, size_t E,
                    size_t k, int softmax, int renorm, uint32_t *ids,
                    float *scores, int32_t *offsets, uint32_t *group_tokens,
                    float *group_scores, uint32_t *group_slots) {
    if (E == 0 || k == 0 || k > E || H == 0) return HMO_INVALID;
    float *sc = (float *)malloc(E * sizeof(float));
    uint32_t *ord = (uint32_t *)malloc(E * sizeof(uint32_t));
    int status = HMO_OK;
    for (size_t t = 0; t < T && status == HMO_OK; ++t)
        status = route_token(hidden + t * H, weights, bias, H, E, k, softmax,
                             renorm, sc, ord, ids + t * k, scores + t * k);
    free(sc);
    free(ord);
    if (status != HMO_OK) return status;
    if (offsets) {
        for (size_t e = 0; e <= E; ++e) offsets[e] = 0;
        for (size_t a = 0; a < T * k; ++a) offsets[ids[a] + 1]++;
        for (size_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
        int32_t *fill = (int32_t *)malloc(E * sizeof(int32_t));
        for (size_t e = 0; e < E; ++e) fill[e] = offsets[e];
        for (size_t t = 0; t < T; ++t)
            for (size_t r = 0; r < k; ++r) {
                uint32_t e = ids[t * k + r];
                int32_t pos = fill[e]++;
                if (group_tokens) group_tokens[pos] = (uint32_t)t;
                if (group_scores) group_scores[pos] = scores[t * k + r];
                if (group_slots) group_slots[pos] = (uint32_t)r;
            }
        free(fill);
    }
    return HMO_OK;
}

/* ------------------------------------------------------------ expert MLP */

/* out[r,c] = sum_k left[r,k] * (float(q[k,c] - zp) * scale), serial FP32 in
 * k order (CpuTensorBackend.cpp:173-186).  The loop nest is row, k, column
 * with one accumulator per column: each output still sees exactly the same
 * sequence of roundings as the reference's row, column, k nest. */
void hmo_int8_matmul(const float *left, const int8_t *q, float *out,
                     size_t rows, size_t K, size_t N, float scale,
                     int32_t zp) {
    float *acc = (float *)malloc(N * sizeof(float));
    float *w = (float *)malloc(N * sizeof(float));
    for (size_t r = 0; r < rows; ++r) {
        for (size_t c = 0; c < N; ++c) acc[c] = 0.0f;
        for (size_t i = 0; i < K; ++i) {
            const float x = left[r * K + i];
            const int8_t *qrow = q + i * N;
            for (size_t c = 0; c < N; ++c)
                w[c] = (float)((int32_t)qrow[c] - zp) * scale;
            for (size_t c = 0; c < N; ++c) acc[c] += x * w[c];
        }
        memcpy(out + r * N, acc, N * sizeof(float));
    }
    free(acc);
    free(w);
}

/* Activation.cpp:44 */
float hmo_silu(float v) { return v / (1.0f + expf(-v)); }

/* The host libm's expf over an array (the exponential of the reference's
 * softmax, CpuRouterBackend.cpp:54), for tests that look for inputs it
 * rounds differently from the correctly rounded exponential. */
void hmo_expf_array(const float *x, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = expf(x[i]);
}

/* RMSNorm::execute, CPU branch (src/transformer/norm/RMSNorm.cpp:64-77):
 * squares summed sequentially in double, inverse RMS in double, one rounding
 * to float per output. */
void hmo_rms_norm(const float *x, const float *w, float *out, size_t T, size_t H, float eps) {
    for (size_t t = 0; t < T; ++t) {
        double ss = 0.0;
        for (size_t i = 0; i < H; ++i) {
            const float v = x[t * H + i];
            ss += (double)v * v;
        }
        const double inv = 1.0 / sqrt(ss / (double)H + eps);
        for (size_t i = 0; i < H; ++i) out[t * H + i] = (float)(x[t * H + i] * inv * w[i]);
    }
}

/* down(SiLU(x*Wg) (.) (x*Wu)), ExpertExecutor.cpp:118-131 with the CPU
 * backend: two INT8 GEMMs, elementwise SiLU, elementwise multiply
 * (CpuTensorBackend.cpp:207-220), INT8 GEMM. */
void hmo_expert_mlp(const float *x, size_t rows, size_t H, size_t I,
                    const int8_t *gate, const int8_t *up, const int8_t *down,
                    const float scale[3], const int32_t zp[3], float *y) {
    float *g = (float *)malloc(rows * I * sizeof(float));
    float *u = (float *)malloc(rows * I * sizeof(float));
    hmo_int8_matmul(x, gate, g, rows, H, I, scale[0], zp[0]);
    hmo_int8_matmul(x, up, u, rows, H, I, scale[1], zp[1]);
    for (size_t i = 0; i < rows * I; ++i) {
        const float a = hmo_silu(g[i]);
        g[i] = a * u[i];
    }
    hmo_int8_matmul(g, down, y, rows, I, H, scale[2], zp[2]);
    free(g);
    free(u);
}

/* Whole MoE layer, CPU branch of MoERuntime::executeBatch.
 *
 * Expert weights live in one arena with a uniform per-expert stride
 * (ExpertPacker's experts.bin layout: expert blob = gate|up|down, blob start
 * 4096-aligned).  expert e's projections are at
 *   arena + e*stride + {gate_off, up_off, down_off}
 * with quantisation parameters qscale[3e+p], qzp[3e+p] (p = gate, up, down).
 * n_shared always-on experts follow the routed ones (ids E..E+S-1); they see
 * every token with weight 1.0 and are combined after the routed experts, so
 * the combine order stays ascending expert id.  The reference has no shared
 * experts (PackedModelRuntime.cpp:267-270 rejects them); this is the
 * build's definition for the Qwen1.5-MoE configuration.
 *
 * hmo_moe_layer_threads computes the experts' MLPs on `threads` host
 * threads (each expert's rows are independent: gather, three INT8 GEMMs,
 * SiLU and multiply see exactly the numbers and order of the sequential
 * loop), then combines `out[tok] += w * y` in ascending expert id on one
 * thread (MoERuntime.cpp:311-325).  The result is bit-identical for any
 * thread count.
 *
 * Optional outputs (may be NULL): ids/scores [T,k], offsets [E+1]. */
typedef struct {
    const float *x;
    size_t T, H, I, E;
    const int8_t *arena;
    size_t stride, gate_off, up_off, down_off;
    const float *qscale;
    const int32_t *qzp;
    const int32_t *off;
    const uint32_t *gt;
    const size_t *row0; /* first row of expert e in yall */
    float *yall;
    size_t total;
    size_t next; /* work counter (guarded by lock) */
    pthread_mutex_t lock;
} hmo_layer_job;

static size_t expert_rows(const hmo_layer_job *j, size_t e) {
    return e < j->E ? (size_t)(j->off[e + 1] - j->off[e]) : j->T;
}

static void *layer_worker(void *arg) {
    hmo_layer_job *j = (hmo_layer_job *)arg;
    float *xin = NULL;
    size_t cap = 0;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        const size_t e = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (e >= j->total) break;
        const size_t n = expert_rows(j, e);
        if (n == 0) continue;
        if (n > cap) {
            free(xin);
            cap = n;
            xin = (float *)malloc(cap * j->H * sizeof(float));
        }
        const uint32_t *toks = e < j->E ? j->gt + j->off[e] : NULL;
        for (size_t r = 0; r < n; ++r) {
            const size_t tok = toks ? toks[r] : r;
            memcpy(xin + r * j->H, j->x + tok * j->H, j->H * sizeof(float));
        }
        const int8_t *blob = j->arena + e * j->stride;
        hmo_expert_mlp(xin, n, j->H, j->I, blob + j->gate_off, blob + j->up_off,
                       blob + j->down_off, j->qscale + 3 * e, j->qzp + 3 * e,
                       j->yall + j->row0[e] * j->H);
    }
    free(xin);
    return NULL;
}

int hmo_moe_layer_threads(const float *x, size_t T, size_t H, size_t I,
                          size_t E, size_t k, int softmax, int renorm,
                          const float *router_w, const float *router_bias,
                          size_t n_shared, const int8_t *arena, size_t stride,
                          size_t gate_off, size_t up_off, size_t down_off,
                          const float *qscale, const int32_t *qzp, float *out,
                          uint32_t *ids_out, float *scores_out,
                          int32_t *offsets_out, int threads) {
    uint32_t *ids = (uint32_t *)malloc(T * k * sizeof(uint32_t));
    float *scores = (float *)malloc(T * k * sizeof(float));
    int32_t *off = (int32_t *)malloc((E + 1) * sizeof(int32_t));
    uint32_t *gt = (uint32_t *)malloc(T * k * sizeof(uint32_t));
    float *gs = (float *)malloc(T * k * sizeof(float));
    int st = hmo_route_batch(x, router_w, router_bias, T, H, E, k, softmax,
                             renorm, ids, scores, off, gt, gs, NULL);
    if (st == HMO_OK) {
        const size_t total = E + n_shared;
        hmo_layer_job j;
        memset(&j, 0, sizeof(j));
        j.x = x; j.T = T; j.H = H; j.I = I; j.E = E;
        j.arena = arena; j.stride = stride;
        j.gate_off = gate_off; j.up_off = up_off; j.down_off = down_off;
        j.qscale = qscale; j.qzp = qzp; j.off = off; j.gt = gt;
        j.total = total;
        size_t *row0 = (size_t *)malloc((total + 1) * sizeof(size_t));
        row0[0] = 0;
        for (size_t e = 0; e < total; ++e) row0[e + 1] = row0[e] + expert_rows(&j, e);
        j.row0 = row0;
        j.yall = (float *)malloc((row0[total] ? row0[total] : 1) * H * sizeof(float));
        pthread_mutex_init(&j.lock, NULL);
        int nt = threads < 1 ? 1 : threads;
        if ((size_t)nt > total) nt = (int)total;
        pthread_t *tid = (pthread_t *)malloc((size_t)nt * sizeof(pthread_t));
        int started = 0;
        for (int i = 1; i < nt; ++i)
            if (pthread_create(&tid[started], NULL, layer_worker, &j) == 0) ++started;
        layer_worker(&j);
        for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
        pthread_mutex_destroy(&j.lock);
        free(tid);
        memset(out, 0, T * H * sizeof(float));
        for (size_t e = 0; e < total; ++e) {
            const size_t n = expert_rows(&j, e);
            const uint32_t *toks = e < E ? gt + off[e] : NULL;
            const float *w = e < E ? gs + off[e] : NULL;
            const float *yout = j.yall + row0[e] * H;
            for (size_t r = 0; r < n; ++r) {
                const size_t tok = toks ? toks[r] : r;
                const float wt = w ? w[r] : 1.0f;
                for (size_t h = 0; h < H; ++h)
                    out[tok * H + h] += wt * yout[r * H + h];
            }
        }
        free(j.yall);
        free(row0);
        if (ids_out) memcpy(ids_out, ids, T * k * sizeof(uint32_t));
        if (scores_out) memcpy(scores_out, scores, T * k * sizeof(float));
        if (offsets_out) memcpy(offsets_out, off, (E + 1) * sizeof(int32_t));
    }
    free(ids);
    free(scores);
    free(off);
    free(gt);
    free(gs);
    return st;
}

int hmo_moe_layer(const float *x, size_t T, size_t H, size_t I, size_t E,
                  size_t k, int softmax, int renorm, const float *router_w,
                  const float *router_bias, size_t n_shared,
                  const int8_t *arena, size_t stride, size_t gate_off,
                  size_t up_off, size_t down_off, const float *qscale,
                  const int32_t *qzp, float *out, uint32_t *ids_out,
                  float *scores_out, int32_t *offsets_out) {
    return hmo_moe_layer_threads(x, T, H, I, E, k, softmax, renorm, router_w,
                                 router_bias, n_shared, arena, stride,
                                 gate_off, up_off, down_off, qscale, qzp, out,
                                 ids_out, scores_out, offsets_out, 1);
}

/* ---------------------------------------------------------- quantisation */

/* Symmetric per-tensor INT8 (Quantization.cpp:45-79): scale = max|w|/127
 * (1 when all zero), q = clamp(round(w/scale), -127, 127), zero point 0. */
int hmo_quantize_int8(const float *w, size_t n, int8_t *q, float *scale,
                      int32_t *zp, float *max_err) {
    if (n == 0) return HMO_INVALID;
    float m = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        if (!isfinite(w[i])) return HMO_INVALID;
        const float a = fabsf(w[i]);
        if (a > m) m = a;
    }
    const float s = m == 0.0f ? 1.0f : m / 127.0f;
    float err = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float r = roundf(w[i] / s);
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        const int8_t v = (int8_t)r;
        q[i] = v;
        const float rec = (float)((int32_t)v - 0) * s;
        const float d = fabsf(w[i] - rec);
        if (d > err) err = d;
    }
    *scale = s;
    *zp = 0;
    if (max_err) *max_err = err;
    return HMO_OK;
}
