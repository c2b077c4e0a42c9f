/*
 * moe_oracle.c - TEST INFRASTRUCTURE ONLY: a plain-C restatement of the
 * reference runtime's MoE block, used as the parity checker for the CUDA path.
 * Never linked into the product library.
 *
 * Follows moe_forward, c/src/model.c:1281-1405, step by step:
 *   router logits      model.c:1301   (gemm_bf16 -> canonical dot, below)
 *   top-k              model.c:1303   (kernel_topk_indices, kernel.c:114-150)
 *   softmax over the k model.c:1305-1318
 *   unique expert set  model.c:1321-1332 (first-appearance order)
 *   per-expert gather  model.c:1354-1367
 *   gate/up, SiLU x up model.c:1368-1374 (fp32 dequantised weights, as the
 *                                          reference's expert cache holds them,
 *                                          model.c:643-651)
 *   down + combine     model.c:1375-1386
 *   shared expert      model.c:1388-1395 (gemm_q4, kernel.c:230-309, group 64)
 *   shared gate        model.c:1396-1402 (sigmoid of a 1-row bf16 product)
 *
 * Two points are defined here, where the reference leaves them open:
 *  1. Router arithmetic. The reference calls Apple's closed BNNSMatMul
 *     (kernel.c:190-228). The canonical definition used by this oracle, by the
 *     Accelerate shim of oracle/_ref and by the GPU router kernel is
 *     oracle_router_dot below: exact bf16 x fp32 products summed in fp64 in a
 *     fixed order, rounded once to fp32.
 *  2. Top-k order. kth_largest (kernel.c:114-138) leaves the order inside the
 *     k and the choice among equal values unspecified. Here the k are chosen
 *     by (value desc, index asc) and reported in that order; parity compares
 *     selections as sets, and a token with an exact tie at the k boundary is
 *     reported separately by the tests.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* bf16 -> fp32 widening, as c/src/util.h:56-61 */
static float bf16f(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/*
 * Canonical router dot product (defines gemm_bf16 for this project).
 * 32 "lanes"; lane l owns the elements k = 256*i + 8*l + j (j = 0..7) and keeps
 * eight fp64 partial sums a[j], each accumulated over i in ascending order.
 * Every product bf16 * fp32 is exact in fp64. The lane total is
 * ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)); the 32 lane totals are combined by a
 * butterfly: for off = 16, 8, 4, 2, 1: s[l] = s[l] + s[l ^ off]. The fp64
 * result is rounded once to fp32.
 */
float oracle_router_dot(const float *x, const uint16_t *w, int K) {
    double s[32];
    for (int l = 0; l < 32; l++) {
        double a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int base = 0; base < K; base += 256) {
            for (int j = 0; j < 8; j++) {
                int k = base + 8 * l + j;
                if (k < K) a[j] += (double)x[k] * (double)bf16f(w[k]);
            }
        }
        s[l] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    }
    for (int off = 16; off >= 1; off >>= 1) {
        double t[32];
        for (int l = 0; l < 32; l++) t[l] = s[l] + s[l ^ off];
        memcpy(s, t, sizeof(t));
    }
    return (float)s[0];
}

/* kernel_dequant_q4, c/src/kernel.c:152-173: low nibble first, 8 per word,
 * groups along the row. */
void oracle_dequant_q4(const uint32_t *q, const float *scales,
                       const float *biases, int rows, int cols, int group,
                       float *out) {
    int words = cols / 8, groups = cols / group;
    for (int r = 0; r < rows; r++) {
        for (int c = 0; c < cols; c++) {
            uint32_t wv = q[(size_t)r * words + c / 8];
            float qv = (float)((wv >> (4 * (c % 8))) & 0xF);
            out[(size_t)r * cols + c] =
                qv * scales[(size_t)r * groups + c / group] +
                biases[(size_t)r * groups + c / group];
        }
    }
}

/* dequantise rows with bf16 scales/biases (dequant_raw, model.c:424-472,
 * widens them to fp32 first) */
static void dequant_bf16sb(const uint32_t *q, const uint16_t *s,
                           const uint16_t *b, int rows, int cols, int group,
                           float *out) {
    int groups = cols / group;
    float *fs = malloc((size_t)rows * groups * sizeof(float));
    float *fb = malloc((size_t)rows * groups * sizeof(float));
    for (size_t i = 0; i < (size_t)rows * groups; i++) {
        fs[i] = bf16f(s[i]);
        fb[i] = bf16f(b[i]);
    }
    oracle_dequant_q4(q, fs, fb, rows, cols, group, out);
    free(fs);
    free(fb);
}

/* C[M,N] = A[M,K] . W[N,K]^T in fp32, k ascending (gemm_fp32, kernel.c:181) */
static void gemm_f32(int M, int N, int K, const float *A, const float *W,
                     float *C) {
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const float *a = A + (size_t)m * K, *w = W + (size_t)n * K;
            float acc = 0.0f;
            for (int k = 0; k < K; k++) acc += a[k] * w[k];
            C[(size_t)m * N + n] = acc;
        }
}

/* gemm_q4, kernel.c:230-309: per group, acc += s*sum(x*q) + b*sum(x) */
static void gemm_q4_f(int M, int N, int K, const float *A, const uint32_t *W,
                      const uint16_t *S, const uint16_t *B, int group,
                      float *C) {
    int groups = K / group, wpg = group / 8;
    float *xsum = malloc((size_t)groups * sizeof(float));
    for (int m = 0; m < M; m++) {
        const float *a = A + (size_t)m * K;
        for (int g = 0; g < groups; g++) {
            float s = 0;
            for (int i = 0; i < group; i++) s += a[g * group + i];
            xsum[g] = s;
        }
        for (int n = 0; n < N; n++) {
            const uint32_t *w = W + (size_t)n * (K / 8);
            float acc = 0;
            for (int g = 0; g < groups; g++) {
                float xq = 0;
                const float *ag = a + (size_t)g * group;
                for (int wd = 0; wd < wpg; wd++) {
                    uint32_t v = w[g * wpg + wd];
                    for (int i = 0; i < 8; i++)
                        xq += ag[wd * 8 + i] * (float)((v >> (4 * i)) & 0xF);
                }
                float s = bf16f(S[(size_t)n * groups + g]);
                float b = B ? bf16f(B[(size_t)n * groups + g]) : 0.0f; /* absent: zeros */
                acc += s * xq + b * xsum[g];
            }
            C[(size_t)m * N + n] = acc;
        }
    }
    free(xsum);
}

static float silu1(float v) { return v / (1.0f + expf(-v)); } /* kernel.c:38-43 */

/* top-k by (value desc, index asc) */
static void topk_canon(const float *v, int E, int k, int32_t *idx) {
    for (int s = 0; s < k; s++) {
        int best = -1;
        for (int e = 0; e < E; e++) {
            int taken = 0;
            for (int t = 0; t < s; t++)
                if (idx[t] == e) { taken = 1; break; }
            if (taken) continue;
            if (best < 0 || v[e] > v[best]) best = e;
        }
        idx[s] = best;
    }
}

int oracle_route(const oracle_layer *L, const float *x, int n, int32_t *idx,
                 float *wts, float *logits) {
    int d = L->d, E = L->E, k = L->k;
    float *lg = malloc((size_t)E * sizeof(float));
    for (int t = 0; t < n; t++) {
        const float *xt = x + (size_t)t * d;
        for (int e = 0; e < E; e++) {
            float v = oracle_router_dot(xt, L->router + (size_t)e * d, d);
            /* workload bias, added to the fp32 logit after rounding */
            if (L->logit_bias) v = v + L->logit_bias[e];
            lg[e] = v;
        }
        if (logits) memcpy(logits + (size_t)t * E, lg, (size_t)E * sizeof(float));
        int32_t *it = idx + (size_t)t * k;
        topk_canon(lg, E, k, it);
        /* softmax over the selected k, model.c:1305-1318 */
        float mx = -1e30f;
        for (int s = 0; s < k; s++)
            if (lg[it[s]] > mx) mx = lg[it[s]];
        float sum = 0, ev[64];
        for (int s = 0; s < k; s++) {
            ev[s] = expf(lg[it[s]] - mx);
            sum += ev[s];
        }
        for (int s = 0; s < k; s++) wts[(size_t)t * k + s] = ev[s] / sum;
    }
    free(lg);
    return 0;
}

int oracle_moe_forward(const oracle_layer *L, const float *x, int n,
                       float *out, int32_t *idx_out, float *wts_out,
                       float *logits) {
    int d = L->d, E = L->E, k = L->k, I = L->I, g = L->g;
    if (n < 0 || k > 64 || k > E || d % g || I % g || g % 8) return -1;
    int32_t *idx = malloc((size_t)(n ? n : 1) * k * sizeof(int32_t));
    float *wts = malloc((size_t)(n ? n : 1) * k * sizeof(float));
    oracle_route(L, x, n, idx, wts, logits);
    memset(out, 0, (size_t)n * d * sizeof(float));

    /* unique experts in first-appearance order, model.c:1321-1332 */
    int *uniq = malloc((size_t)(n ? n : 1) * k * sizeof(int));
    int nu = 0;
    for (int t = 0; t < n; t++)
        for (int s = 0; s < k; s++) {
            int e = idx[(size_t)t * k + s], seen = 0;
            for (int u = 0; u < nu; u++)
                if (uniq[u] == e) { seen = 1; break; }
            if (!seen) uniq[nu++] = e;
        }

    size_t gsz = (size_t)I * d;
    float *w = malloc(3 * gsz * sizeof(float));
    int *tok = malloc((size_t)(n ? n : 1) * sizeof(int));
    float *xs = malloc((size_t)(n ? n : 1) * d * sizeof(float));
    float *go = malloc((size_t)(n ? n : 1) * I * sizeof(float));
    float *uo = malloc((size_t)(n ? n : 1) * I * sizeof(float));
    float *ro = malloc((size_t)(n ? n : 1) * d * sizeof(float));
    for (int u = 0; u < nu; u++) {
        int e = uniq[u];
        size_t qo = (size_t)e * I * (d / 8), so = (size_t)e * I * (d / g);
        size_t dqo = (size_t)e * d * (I / 8), dso = (size_t)e * d * (I / g);
        dequant_bf16sb(L->gq + qo, L->gs + so, L->gb + so, I, d, g, w);
        dequant_bf16sb(L->uq + qo, L->us + so, L->ub + so, I, d, g, w + gsz);
        dequant_bf16sb(L->dq + dqo, L->ds + dso, L->db + dso, d, I, g, w + 2 * gsz);
        int nt = 0;
        for (int t = 0; t < n; t++)
            for (int s = 0; s < k; s++)
                if (idx[(size_t)t * k + s] == e) { tok[nt++] = t; break; }
        if (!nt) continue;
        for (int i = 0; i < nt; i++)
            memcpy(xs + (size_t)i * d, x + (size_t)tok[i] * d, (size_t)d * sizeof(float));
        gemm_f32(nt, I, d, xs, w, go);
        gemm_f32(nt, I, d, xs, w + gsz, uo);
        for (size_t i = 0; i < (size_t)nt * I; i++) go[i] = silu1(go[i]) * uo[i];
        gemm_f32(nt, d, I, go, w + 2 * gsz, ro);
        for (int i = 0; i < nt; i++) {
            int t = tok[i];
            for (int s = 0; s < k; s++)
                if (idx[(size_t)t * k + s] == e) {
                    float wg = wts[(size_t)t * k + s];
                    for (int j = 0; j < d; j++)
                        out[(size_t)t * d + j] += wg * ro[(size_t)i * d + j];
                }
        }
    }
    free(w); free(tok); free(xs); free(go); free(uo); free(ro); free(uniq);

    /* shared expert and its sigmoid gate, model.c:1388-1402 */
    float *sh = malloc((size_t)(n ? n : 1) * I * sizeof(float));
    float *su = malloc((size_t)(n ? n : 1) * I * sizeof(float));
    float *so = malloc((size_t)(n ? n : 1) * d * sizeof(float));
    gemm_q4_f(n, I, d, x, L->sgq, L->sgs, L->sgb, g, sh);
    gemm_q4_f(n, I, d, x, L->suq, L->sus, L->sub, g, su);
    for (size_t i = 0; i < (size_t)n * I; i++) sh[i] = silu1(sh[i]) * su[i];
    gemm_q4_f(n, d, I, sh, L->sdq, L->sds, L->sdb, g, so);
    for (int t = 0; t < n; t++) {
        float gv = oracle_router_dot(x + (size_t)t * d, L->shared_gate, d);
        float gs = 1.0f / (1.0f + expf(-gv));
        for (int j = 0; j < d; j++) out[(size_t)t * d + j] += gs * so[(size_t)t * d + j];
    }
    free(sh); free(su); free(so);

    if (idx_out) memcpy(idx_out, idx, (size_t)n * k * sizeof(int32_t));
    if (wts_out) memcpy(wts_out, wts, (size_t)n * k * sizeof(float));
    free(idx);
    free(wts);
    return 0;
}

/* ------------------------------------------------ hyper connections */

/* kernel_rmsnorm_grouped, c/src/kernel.c:22-36: groups of `group` values,
 * weight row (g % groups_per_row) */
static void rmsnorm_grouped(const float *x, const float *w, size_t n, size_t group, size_t rows,
                            float eps, float *y) {
    size_t groups = n / group, per_row = rows ? groups / rows : groups;
    for (size_t g = 0; g < groups; g++) {
        const float *xg = x + g * group;
        float ss = 0;
        for (size_t i = 0; i < group; i++) ss += xg[i] * xg[i];
        float r = 1.0f / sqrtf(ss / (float)group + eps);
        const float *wg = w ? w + (g % per_row) * group : NULL;
        for (size_t i = 0; i < group; i++) y[g * group + i] = xg[i] * r * (wg ? wg[i] : 1.0f);
    }
}

static float sigmoid1(float v) { return 1.0f / (1.0f + expf(-v)); } /* kernel.c:45-47 */

/* linear_forward (model.c:194-202) with group 64, as gated_residual calls it
 * (model.c:753, :757): q4 through gemm_q4, else bf16 through gemm_bf16 */
static void hc_linear(const uint32_t *q, const uint16_t *s, const uint16_t *b, const uint16_t *bf,
                      int M, int N, int K, const float *A, float *C) {
    if (q) {
        gemm_q4_f(M, N, K, A, q, s, b, 64, C);
        return;
    }
    for (int m = 0; m < M; m++)
        for (int nn = 0; nn < N; nn++)
            C[(size_t)m * N + nn] = oracle_router_dot(A + (size_t)m * K, bf + (size_t)nn * K, K);
}

int oracle_gated_residual(const oracle_hc *H, const float *h, int n, float *mixed,
                          float *inject) {
    const int hc = H->hc, d = H->d, lr = H->lowrank, hd = hc * d;
    if (n < 0 || hc < 1 || d < 1 || lr < 1 || (!H->down_q && !H->down_bf16) ||
        (!H->up_q && !H->up_bf16) || (inject && !H->inject))
        return -1;
    if (!n) return 0;
    float *normed = malloc((size_t)n * hd * sizeof(float));
    float *w = malloc((size_t)n * lr * sizeof(float));
    float *tmp = malloc((size_t)n * hd * sizeof(float));
    if (!normed || !w || !tmp) {
        free(normed);
        free(w);
        free(tmp);
        return -1;
    }
    /* normed = rmsnorm over each stream's d values (model.c:733) */
    rmsnorm_grouped(h, H->norm, (size_t)n * hd, (size_t)d, (size_t)n, 1e-6f, normed);
    /* w = silu(down(normed) / hc) (model.c:752-755) */
    hc_linear(H->down_q, H->down_s, H->down_b, H->down_bf16, n, lr, hd, normed, w);
    for (size_t i = 0; i < (size_t)n * lr; i++) w[i] = silu1(w[i] * (1.0f / hc));
    /* tmp = sigmoid(up(w)) (model.c:756-758) */
    hc_linear(H->up_q, H->up_s, H->up_b, H->up_bf16, n, hd, lr, w, tmp);
    for (size_t i = 0; i < (size_t)n * hd; i++) tmp[i] = sigmoid1(tmp[i]);
    /* mixed = mean over the streams of tmp * normed (model.c:773-783) */
    for (int t = 0; t < n; t++)
        for (int i = 0; i < d; i++) {
            float acc = 0;
            for (int c = 0; c < hc; c++)
                acc += tmp[(size_t)t * hd + (size_t)c * d + i] * normed[(size_t)t * hd + (size_t)c * d + i];
            mixed[(size_t)t * d + i] = acc / hc;
        }
    /* inject = 2 * sigmoid(block_inject(normed) / hc) (model.c:784-791) */
    if (inject)
        for (int t = 0; t < n; t++)
            for (int c = 0; c < hc; c++) {
                float v = oracle_router_dot(normed + (size_t)t * hd, H->inject + (size_t)c * hd, hd);
                inject[(size_t)t * hc + c] = sigmoid1(v * (1.0f / hc)) * 2.0f;
            }
    free(normed);
    free(w);
    free(tmp);
    return 0;
}

int oracle_hc_moe_step(const oracle_hc *H, const oracle_layer *L, float *h, int n) {
    const int hc = H->hc, d = H->d;
    if (d != L->d) return -1;
    if (!n) return 0;
    float *mixed = malloc((size_t)n * d * sizeof(float));
    float *inj = malloc((size_t)n * hc * sizeof(float));
    float *y = malloc((size_t)n * d * sizeof(float));
    int rc = -1;
    if (mixed && inj && y && !oracle_gated_residual(H, h, n, mixed, inj) &&
        !oracle_moe_forward(L, mixed, n, y, NULL, NULL, NULL)) {
        /* the inject-add after the block (model.c:1723-1731) */
        for (int t = 0; t < n; t++)
            for (int c = 0; c < hc; c++) {
                const float a = inj[(size_t)t * hc + c];
                for (int j = 0; j < d; j++) h[((size_t)t * hc + c) * d + j] += a * y[(size_t)t * d + j];
            }
        rc = 0;
    }
    free(mixed);
    free(inj);
    free(y);
    return rc;
}
