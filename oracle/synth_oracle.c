/*
 * synth_oracle.c - TEST INFRASTRUCTURE ONLY.
 *
 * The seeded synthetic workload (layers and tokens), generated on the CPU
 * without the product library, so that the reference arm of the benchmark
 * and the CPU baselines build their inputs from checker code alone. It is a
 * restatement of the published generator every workload config uses:
 *
 *   - stream key  = mix(mix(seed ^ 0x5851F42D4C957F2D) + (layer << 16) + tensor)
 *   - i-th draw   = mix(key + (i + 1) * 0x9E3779B97F4A7C15)  (splitmix64's
 *                   counter form; mix is the splitmix64 finaliser that the
 *                   reference's cache hashes keys with, c/src/cache.c:15-21)
 *   - q4 words    = low 32 bits of one draw per word
 *   - normals     = Box-Muller in fp64 on draws 2i and 2i + 1 (53-bit
 *                   uniforms centred in their bins), rounded once to fp32
 *   - scales      = bf16(|N(0,1) * 0.02|), biases bf16(-8 * scale)
 *   - router, shared gate = bf16(N(0,1) * 0.02); tokens bf16(N(0,1)) as fp32
 *   - Zipf bias   = -s * ln(1 + pi(e)), pi a Fisher-Yates permutation whose
 *                   i-th swap partner is draw(i) mod (i + 1)
 *
 * bf16 rounding is round-to-nearest-even as f32_to_bf16 (c/src/util.h:63-71).
 * Tensor stream ids: router 0, shared gate 1, gate q/s 2/3, up q/s 4/5,
 * down q/s 6/7, shared gate q/s 8/9, shared up q/s 10/11, shared down q/s
 * 12/13, permutation 20; tokens use layer 0xFFFF and tensor 0x1000 + stream.
 *
 * Pinned by the SHA-256 digests of every input tensor stored with the golden
 * fixtures (tests/golden/moe_cfg0.npz, moe_cfg1_tokens.npz), which the
 * reference's own moe_forward consumed when it wrote them.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

#include "oracle.h"

enum {
    T_ROUTER = 0, T_SHGATE = 1, T_GQ = 2, T_GS = 3, T_UQ = 4, T_US = 5, T_DQ = 6, T_DS = 7,
    T_SGQ = 8, T_SGS = 9, T_SUQ = 10, T_SUS = 11, T_SDQ = 12, T_SDS = 13, T_PERM = 20
};

static uint64_t fin(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t nth(uint64_t key, uint64_t i) { return fin(key + (i + 1) * 0x9E3779B97F4A7C15ull); }

static uint64_t key_of(uint64_t seed, uint64_t layer, uint64_t tensor) {
    return fin(fin(seed ^ 0x5851F42D4C957F2Dull) + (layer << 16) + tensor);
}

static double u01(uint64_t r) { return ((double)(r >> 11) + 0.5) / 9007199254740992.0; }

static float gauss(uint64_t key, uint64_t i) {
    const double a = u01(nth(key, 2 * i)), b = u01(nth(key, 2 * i + 1));
    return (float)(sqrt(-2.0 * log(a)) * cos(6.283185307179586 * b));
}

static uint16_t bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    uint32_t hi = u >> 16;
    const uint32_t lo = u & 0xFFFFu;
    if (lo > 0x8000u || (lo == 0x8000u && (hi & 1u))) hi++;
    return (uint16_t)hi;
}

static float bf16_val(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* One tensor stream's work: words (q), or scale/bias pairs (s, b), or bf16
 * normals (o), for elements [first, first + n) of the stream written to
 * element 0 of the given buffers. Split over host threads by element range;
 * every element depends only on its own index, so the split changes nothing. */
typedef struct {
    uint64_t key;
    size_t first, n;
    uint32_t *q;
    uint16_t *s, *b, *o;
} job;

typedef struct {
    const job *j;
    size_t lo, hi;
} span;

static void run_span(const job *j, size_t lo, size_t hi) {
    for (size_t i = lo; i < hi; i++) {
        const size_t at = j->first + i;
        if (j->q) {
            j->q[i] = (uint32_t)nth(j->key, at);
        } else if (j->o) {
            j->o[i] = bf16_rne(gauss(j->key, at) * 0.02f);
        } else {
            const uint16_t v = bf16_rne(fabsf(gauss(j->key, at) * 0.02f));
            if (j->s) j->s[i] = v;
            if (j->b) j->b[i] = bf16_rne(-8.0f * bf16_val(v));
        }
    }
}

static void *span_main(void *arg) {
    const span *sp = arg;
    run_span(sp->j, sp->lo, sp->hi);
    return NULL;
}

static void run(const job *j) {
    if (!j->q && !j->s && !j->b && !j->o) return;
    long nc = sysconf(_SC_NPROCESSORS_ONLN);
    int nt = nc < 1 ? 1 : (nc > 64 ? 64 : (int)nc);
    if (j->n < (size_t)1 << 16) nt = 1;
    pthread_t th[64];
    span sp[64];
    for (int t = 0; t < nt; t++) {
        sp[t].j = j;
        sp[t].lo = j->n * (size_t)t / (size_t)nt;
        sp[t].hi = j->n * (size_t)(t + 1) / (size_t)nt;
        if (t > 0 && pthread_create(&th[t], NULL, span_main, &sp[t]) != 0) {
            run_span(j, sp[t].lo, sp[t].hi); /* no thread: do it here */
            sp[t].j = NULL;
        }
    }
    run_span(j, sp[0].lo, sp[0].hi);
    for (int t = 1; t < nt; t++)
        if (sp[t].j) pthread_join(th[t], NULL);
}

static void words(uint64_t key, uint32_t *q, size_t first, size_t n) {
    const job j = {key, first, n, q, NULL, NULL, NULL};
    run(&j);
}

static void scales(uint64_t key, uint16_t *s, uint16_t *b, size_t first, size_t n) {
    const job j = {key, first, n, NULL, s, b, NULL};
    run(&j);
}

static void normals_bf16(uint64_t key, uint16_t *o, size_t n) {
    const job j = {key, 0, n, NULL, NULL, NULL, o};
    run(&j);
}

int oracle_synth_layer(oracle_layer *L, uint64_t seed, int layer, int e0, int e1) {
    if (!L || L->d <= 0 || L->I <= 0 || L->g <= 0 || L->d % L->g || L->I % L->g || L->g % 8) return -1;
    const size_t d = (size_t)L->d, I = (size_t)L->I, g = (size_t)L->g;
    if (e1 <= e0) {
        e0 = 0;
        e1 = L->E;
    }
    if (e0 < 0 || e1 > L->E) return -1;
    const uint64_t l = (uint64_t)layer;
    normals_bf16(key_of(seed, l, T_ROUTER), (uint16_t *)L->router, (size_t)L->E * d);
    normals_bf16(key_of(seed, l, T_SHGATE), (uint16_t *)L->shared_gate, d);
    /* routed experts: rows of experts [e0, e1) of the stacked tensors; the
     * buffers hold all E experts and the slice is written in place */
    const size_t gq = I * (d / 8), gs = I * (d / g), dq = d * (I / 8), ds = d * (I / g);
    const size_t a = (size_t)e0, n = (size_t)(e1 - e0);
#define PART(Q, S, B, TQ, TS, PQ, PS)                                                           \
    do {                                                                                        \
        words(key_of(seed, l, TQ), L->Q ? (uint32_t *)L->Q + a * PQ : NULL, a * PQ, n * PQ);    \
        scales(key_of(seed, l, TS), L->S ? (uint16_t *)L->S + a * PS : NULL,                   \
               L->B ? (uint16_t *)L->B + a * PS : NULL, a * PS, n * PS);                        \
    } while (0)
    PART(gq, gs, gb, T_GQ, T_GS, gq, gs);
    PART(uq, us, ub, T_UQ, T_US, gq, gs);
    PART(dq, ds, db, T_DQ, T_DS, dq, ds);
#undef PART
    words(key_of(seed, l, T_SGQ), (uint32_t *)L->sgq, 0, gq);
    scales(key_of(seed, l, T_SGS), (uint16_t *)L->sgs, (uint16_t *)L->sgb, 0, gs);
    words(key_of(seed, l, T_SUQ), (uint32_t *)L->suq, 0, gq);
    scales(key_of(seed, l, T_SUS), (uint16_t *)L->sus, (uint16_t *)L->sub, 0, gs);
    words(key_of(seed, l, T_SDQ), (uint32_t *)L->sdq, 0, dq);
    scales(key_of(seed, l, T_SDS), (uint16_t *)L->sds, (uint16_t *)L->sdb, 0, ds);
    return 0;
}

void oracle_synth_tokens(uint64_t seed, uint64_t stream, int n, int d, float *x) {
    const uint64_t key = key_of(seed, 0xFFFF, 0x1000 + stream);
    const size_t total = (size_t)n * (size_t)d;
    for (size_t i = 0; i < total; i++) x[i] = bf16_val(bf16_rne(gauss(key, i)));
}

int oracle_synth_zipf_bias(uint64_t seed, int layer, int E, double s, float *bias) {
    if (E <= 0 || E > 65536 || !bias) return -1;
    const uint64_t key = key_of(seed, (uint64_t)layer, T_PERM);
    int perm[65536];
    for (int i = 0; i < E; i++) perm[i] = i;
    for (int i = E - 1; i > 0; i--) {
        const int j = (int)(nth(key, (uint64_t)i) % (uint64_t)(i + 1));
        const int t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
    }
    for (int e = 0; e < E; e++) bias[e] = (float)(-s * log(1.0 + (double)perm[e]));
    return 0;
}

/* RMSNorm of each row with unit weight, as the stack configs apply it
 * before every layer: kernel_rmsnorm (c/src/kernel.c:10-20) with the sum of
 * squares accumulated in fp64. */
void oracle_rmsnorm_rows(const float *x, int n, int d, float eps, float *y) {
    for (int t = 0; t < n; t++) {
        const float *r = x + (size_t)t * d;
        double ss = 0.0;
        for (int i = 0; i < d; i++) ss += (double)r[i] * (double)r[i];
        const float inv = 1.0f / sqrtf((float)ss / (float)d + eps);
        for (int i = 0; i < d; i++) y[(size_t)t * d + i] = r[i] * inv;
    }
}
