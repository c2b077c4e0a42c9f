/*
 * qmoe_synth.c - seeded synthetic MoE layers and tokens (host C).
 *
 * Inputs for benchmarks and tests in the reference checkpoint layout
 * (c/src/model.c:555-557, :1902-1923). Every value comes from a counter-based
 * splitmix64 stream keyed by (seed, layer, tensor), so any subset of experts
 * can be generated independently and identically. The splitmix64 finaliser
 * is the same mixer the reference's cache hashes keys with
 * (c/src/cache.c:15-21).
 *
 * Distributions: nibbles uniform over 0..15 (one 32-bit draw per word);
 * scales bf16(|N(0, 0.02)|) and biases bf16(-8 * scale), so a weight is
 * exactly (q - 8) * scale; router and shared gate bf16(N(0, 0.02));
 * tokens bf16(N(0, 1)) delivered as fp32. Normals use Box-Muller in fp64,
 * rounded once to fp32 and then to bf16 by round-to-nearest-even
 * (f32_to_bf16, c/src/util.h:63-71).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/qmoe.h"
#include "qmoe_internal.h"

#define GOLDEN 0x9E3779B97F4A7C15ull

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* i-th output of the splitmix64 sequence whose state starts at key */
static inline uint64_t draw(uint64_t key, uint64_t i) {
    return mix64(key + (i + 1) * GOLDEN);
}

uint64_t qk_stream_key(uint64_t seed, uint64_t layer, uint64_t tensor) {
    return mix64(mix64(seed ^ 0x5851F42D4C957F2Dull) + (layer << 16) + tensor);
}

static double unit(uint64_t r) { return ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

static float normal(uint64_t key, uint64_t i) {
    double u1 = unit(draw(key, 2 * i)), u2 = unit(draw(key, 2 * i + 1));
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

static uint16_t to_bf16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    uint32_t r = b >> 16, rem = b & 0xFFFF;
    if (rem > 0x8000 || (rem == 0x8000 && (r & 1))) r++;
    return (uint16_t)r;
}

static float from_bf16(uint16_t h) {
    uint32_t b = (uint32_t)h << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}


static void fill_words(uint64_t key, uint32_t *q, size_t off, size_t n) {
    for (size_t i = 0; i < n; i++) q[off + i] = (uint32_t)draw(key, off + i);
}

static void fill_scales(uint64_t key, uint16_t *s, uint16_t *b, size_t off,
                        size_t n) {
    for (size_t i = 0; i < n; i++) {
        uint16_t sv = to_bf16(fabsf(normal(key, off + i) * 0.02f));
        if (s) s[off + i] = sv;
        if (b) b[off + i] = to_bf16(-8.0f * from_bf16(sv));
    }
}

int qmoe_synth_sizes(const qmoe_config *c, qmoe_synth_size *o) {
    if (!c || !o || c->hidden <= 0 || c->moe_inter <= 0 || c->group_size <= 0 ||
        c->hidden % c->group_size || c->moe_inter % c->group_size || c->group_size % 8)
        return -1;
    size_t d = (size_t)c->hidden, E = (size_t)c->num_experts, I = (size_t)c->moe_inter,
           g = (size_t)c->group_size;
    o->router = E * d;
    o->shared_gate = d;
    o->expert_q = E * I * (d / 8);
    o->expert_sb = E * I * (d / g);
    o->down_q = E * d * (I / 8);
    o->down_sb = E * d * (I / g);
    o->sh_q = I * (d / 8);
    o->sh_sb = I * (d / g);
    o->sh_down_q = d * (I / 8);
    o->sh_down_sb = d * (I / g);
    return 0;
}

int qmoe_synth_layer(const qmoe_config *c, uint64_t seed, int layer,
                     qmoe_layer_weights *w, int e0, int e1) {
    qmoe_synth_size sz;
    if (qmoe_synth_sizes(c, &sz) || !w) return -1;
    size_t d = (size_t)c->hidden, I = (size_t)c->moe_inter, g = (size_t)c->group_size;
    int E = c->num_experts;
    if (e1 <= e0) { e0 = 0; e1 = E; }
    if (e0 < 0 || e1 > E) return -1;
    uint64_t L = (uint64_t)layer;
    if (w->router) {
        uint64_t key = qk_stream_key(seed, L, QK_T_ROUTER);
        uint16_t *r = (uint16_t *)w->router;
        for (size_t i = 0; i < sz.router; i++) r[i] = to_bf16(normal(key, i) * 0.02f);
    }
    if (w->shared_gate) {
        uint64_t key = qk_stream_key(seed, L, QK_T_SHGATE);
        uint16_t *r = (uint16_t *)w->shared_gate;
        for (size_t i = 0; i < sz.shared_gate; i++) r[i] = to_bf16(normal(key, i) * 0.02f);
    }
    /* routed experts: [e0, e1) slices of the stacked tensors */
    size_t gq_pe = I * (d / 8), gs_pe = I * (d / g), dq_pe = d * (I / 8), ds_pe = d * (I / g);
    size_t e0s = (size_t)e0, ne = (size_t)(e1 - e0);
    struct { const qmoe_q4 *t; int tq, ts; size_t q_pe, s_pe; } parts[3] = {
        {&w->gate, QK_T_GQ, QK_T_GS, gq_pe, gs_pe},
        {&w->up, QK_T_UQ, QK_T_US, gq_pe, gs_pe},
        {&w->down, QK_T_DQ, QK_T_DS, dq_pe, ds_pe},
    };
    for (int p = 0; p < 3; p++) {
        const qmoe_q4 *t = parts[p].t;
        if (t->q)
            fill_words(qk_stream_key(seed, L, parts[p].tq), (uint32_t *)t->q,
                       e0s * parts[p].q_pe, ne * parts[p].q_pe);
        if (t->scales || t->biases)
            fill_scales(qk_stream_key(seed, L, parts[p].ts), (uint16_t *)t->scales,
                        (uint16_t *)t->biases, e0s * parts[p].s_pe, ne * parts[p].s_pe);
    }
    struct { const qmoe_q4 *t; int tq, ts; size_t nq, ns; } sh[3] = {
        {&w->sh_gate, QK_T_SGQ, QK_T_SGS, sz.sh_q, sz.sh_sb},
        {&w->sh_up, QK_T_SUQ, QK_T_SUS, sz.sh_q, sz.sh_sb},
        {&w->sh_down, QK_T_SDQ, QK_T_SDS, sz.sh_down_q, sz.sh_down_sb},
    };
    for (int p = 0; p < 3; p++) {
        const qmoe_q4 *t = sh[p].t;
        if (t->q) fill_words(qk_stream_key(seed, L, sh[p].tq), (uint32_t *)t->q, 0, sh[p].nq);
        if (t->scales || t->biases)
            fill_scales(qk_stream_key(seed, L, sh[p].ts), (uint16_t *)t->scales,
                        (uint16_t *)t->biases, 0, sh[p].ns);
    }
    return 0;
}

void qmoe_synth_tokens(uint64_t seed, uint64_t stream, int n, int d, float *x) {
    uint64_t key = qk_stream_key(seed, 0xFFFF, 0x1000 + stream);
    for (size_t i = 0; i < (size_t)n * (size_t)d; i++)
        x[i] = from_bf16(to_bf16(normal(key, i)));
}

void qmoe_synth_zipf_bias(uint64_t seed, int layer, int E, double s,
                          float *bias) {
    uint64_t key = qk_stream_key(seed, (uint64_t)layer, QK_T_PERM);
    int perm[4096];
    if (E > 4096) return;
    for (int i = 0; i < E; i++) perm[i] = i;
    for (int i = E - 1; i > 0; i--) {
        int j = (int)(draw(key, (uint64_t)i) % (uint64_t)(i + 1));
        int t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
    }
    for (int e = 0; e < E; e++) bias[e] = (float)(-s * log(1.0 + (double)perm[e]));
}
