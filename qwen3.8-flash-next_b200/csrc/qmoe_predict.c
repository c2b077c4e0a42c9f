/*
 * qmoe_predict.c - route statistics and prefetch prediction of the
 * streaming pool (host only).
 *
 * The bookkeeping of ExpertStore (src/colibri_runtime/streaming.py):
 *   record_route           :400-413  per-layer routed counts, the previous
 *                                    step's selected set, transition counts
 *                                    previous -> selected, hot marks (count >= 4)
 *   prefetch_predictions   :415-435  candidates from the transitions of the
 *                                    selected experts (else the layer's counts)
 *                                    plus twice the next layer's counts; the
 *                                    prefetch_count best for this layer and the
 *                                    next layer's prefetch_count most routed
 *   snapshot               :445-453  the 20 most routed (layer, expert)
 *
 * Ranking is that of Counter.most_common: by count, ties in the order the
 * keys were first inserted. Every counter therefore keeps its keys' insertion
 * order next to the counts (a list per counter), and the candidate counter of
 * a prediction is built in the order the reference's updates insert into it.
 * Transition tables are allocated per layer on first use (E x E counts and
 * orders).
 */
#include <stdlib.h>
#include <string.h>

#include "../../include/qmoe.h"

typedef struct {
    uint32_t *count; /* [E * E]: count[old * E + e] */
    uint16_t *order; /* [E * E]: row old lists its keys in insertion order */
    uint16_t *n;     /* [E] keys in row old */
} trans_layer;

struct qmoe_predictor {
    int L, E;
    uint64_t *freq;       /* [L * E] routed count (token assignments) */
    uint16_t *freq_order; /* [L * E] experts of a layer in first-routed order */
    int *freq_n;          /* [L] */
    int32_t *last;        /* [L * E] previous step's selected set, ascending */
    int *last_n;          /* [L] */
    trans_layer *trans;   /* [L] */
    int *layer_seq;       /* [L] order in which a layer's counter was created, -1 before */
    int next_seq;
    uint64_t routes;
};

qmoe_predictor *qmoe_predictor_new(int num_layers, int num_experts) {
    if (num_layers < 1 || num_experts < 1 || num_experts > 65535) return NULL;
    qmoe_predictor *p = calloc(1, sizeof(*p));
    if (!p) return NULL;
    const size_t LE = (size_t)num_layers * (size_t)num_experts;
    p->L = num_layers;
    p->E = num_experts;
    p->freq = calloc(LE, sizeof(uint64_t));
    p->freq_order = calloc(LE, sizeof(uint16_t));
    p->freq_n = calloc((size_t)num_layers, sizeof(int));
    p->last = calloc(LE, sizeof(int32_t));
    p->last_n = calloc((size_t)num_layers, sizeof(int));
    p->trans = calloc((size_t)num_layers, sizeof(trans_layer));
    p->layer_seq = malloc((size_t)num_layers * sizeof(int));
    if (!p->freq || !p->freq_order || !p->freq_n || !p->last || !p->last_n || !p->trans ||
        !p->layer_seq) {
        qmoe_predictor_free(p);
        return NULL;
    }
    for (int l = 0; l < num_layers; l++) p->layer_seq[l] = -1;
    return p;
}

void qmoe_predictor_free(qmoe_predictor *p) {
    if (!p) return;
    if (p->trans)
        for (int l = 0; l < p->L; l++) {
            free(p->trans[l].count);
            free(p->trans[l].order);
            free(p->trans[l].n);
        }
    free(p->trans);
    free(p->freq);
    free(p->freq_order);
    free(p->freq_n);
    free(p->last);
    free(p->last_n);
    free(p->layer_seq);
    free(p);
}

/* the reference's per-layer counters live in a defaultdict: a layer's counter
 * exists from its first access, which fixes the layer order of snapshot ties */
static void touch(qmoe_predictor *p, int layer) {
    if (p->layer_seq[layer] < 0) p->layer_seq[layer] = p->next_seq++;
}

/* A layer's transition tables, allocated on first use and written through at
 * once: a sequential fill maps every page now, where the lazily mapped zero
 * pages of calloc would fault one row at a time on the streaming path (tens of
 * microseconds a decode step until every row was touched). */
static trans_layer *trans_of(qmoe_predictor *p, int layer) {
    trans_layer *t = &p->trans[layer];
    if (!t->count) {
        const size_t EE = (size_t)p->E * (size_t)p->E;
        t->count = malloc(EE * sizeof(uint32_t));
        t->order = malloc(EE * sizeof(uint16_t));
        t->n = calloc((size_t)p->E, sizeof(uint16_t));
        if (!t->count || !t->order || !t->n) {
            free(t->count);
            free(t->order);
            free(t->n);
            memset(t, 0, sizeof(*t));
            return NULL;
        }
        memset(t->count, 0, EE * sizeof(uint32_t));
        memset(t->order, 0, EE * sizeof(uint16_t));
    }
    return t;
}

int qmoe_predictor_record(qmoe_predictor *p, qmoe_cache *cache, int layer, const int32_t *experts,
                          size_t n, int32_t *selected_out) {
    if (!p || layer < 0 || layer >= p->L || (n && !experts)) return -1;
    const int E = p->E;
    for (size_t i = 0; i < n; i++)
        if (experts[i] < 0 || experts[i] >= E) return -1; /* validated first, :403 */
    unsigned char *mark = calloc((size_t)E, 1);
    int32_t *sel = malloc((size_t)E * sizeof(int32_t));
    if (!mark || !sel) {
        free(mark);
        free(sel);
        return -1;
    }
    for (size_t i = 0; i < n; i++) mark[experts[i]] = 1;
    int ns = 0;
    for (int e = 0; e < E; e++)
        if (mark[e]) sel[ns++] = e;
    free(mark);
    /* transitions previous -> selected, then the counts, then the new
     * previous set (:406-410) */
    const int np = p->last_n[layer];
    const int32_t *prev = p->last + (size_t)layer * E;
    trans_layer *t = np && ns ? trans_of(p, layer) : NULL;
    if (np && ns && !t) {
        free(sel);
        return -1;
    }
    for (int a = 0; t && a < np; a++) { /* t is NULL when either set is empty */
        uint32_t *crow = t->count + (size_t)prev[a] * E;
        uint16_t *orow = t->order + (size_t)prev[a] * E;
        unsigned keys = t->n[prev[a]];
        for (int s = 0; s < ns; s++) {
            const int e = sel[s];
            if (!crow[e]++) orow[keys++] = (uint16_t)e;
        }
        t->n[prev[a]] = (uint16_t)keys;
    }
    touch(p, layer);
    uint64_t *f = p->freq + (size_t)layer * E;
    uint16_t *fo = p->freq_order + (size_t)layer * E;
    for (size_t i = 0; i < n; i++)
        if (!f[experts[i]]++) fo[p->freq_n[layer]++] = (uint16_t)experts[i];
    memcpy(p->last + (size_t)layer * E, sel, (size_t)ns * sizeof(int32_t));
    p->last_n[layer] = ns;
    p->routes += n;
    /* hot marks of the selected experts (:412-413) */
    if (cache)
        for (int s = 0; s < ns; s++)
            qmoe_cache_mark_hot(cache, ((uint64_t)(uint32_t)layer << 32) | (uint32_t)sel[s],
                                f[sel[s]] >= 4);
    if (selected_out) memcpy(selected_out, sel, (size_t)ns * sizeof(int32_t));
    free(sel);
    return ns;
}

/* the `want` best of keys[0..nk) by score, ties to the earlier key (the
 * stable ranking of Counter.most_common) */
static int most_common(const uint16_t *keys, int nk, const uint64_t *score, int want, int64_t *out) {
    int got = 0;
    unsigned char *taken = calloc((size_t)(nk ? nk : 1), 1);
    if (!taken) return 0;
    while (got < want) {
        int best = -1;
        for (int i = 0; i < nk; i++)
            if (!taken[i] && (best < 0 || score[keys[i]] > score[keys[best]])) best = i;
        if (best < 0) break;
        taken[best] = 1;
        out[got++] = keys[best];
    }
    free(taken);
    return got;
}

int qmoe_predictor_predict(qmoe_predictor *p, int layer, const int32_t *selected, size_t n, int depth,
                           int64_t *pick, int *npick, int64_t *next, int *nnext) {
    if (npick) *npick = 0;
    if (nnext) *nnext = 0;
    if (!p || layer < 0 || layer >= p->L || (n && !selected)) return -1;
    const int E = p->E;
    for (size_t i = 0; i < n; i++)
        if (selected[i] < 0 || selected[i] >= E) return -1; /* :418 */
    if (depth <= 0) return 0;                               /* :419-420 */
    if (!pick || !npick || !next || !nnext) return -1;
    uint64_t *cand = calloc((size_t)E, sizeof(uint64_t));
    uint16_t *order = malloc((size_t)E * sizeof(uint16_t));
    if (!cand || !order) {
        free(cand);
        free(order);
        return -1;
    }
    int nc = 0;
    const trans_layer *t = &p->trans[layer];
    if (t->count)
        for (size_t i = 0; i < n; i++) { /* :423-424 */
            const uint32_t *crow = t->count + (size_t)selected[i] * E;
            const uint16_t *orow = t->order + (size_t)selected[i] * E;
            const int keys = t->n[selected[i]];
            for (int j = 0; j < keys; j++) {
                const uint16_t e = orow[j];
                if (!cand[e]) order[nc++] = e;
                cand[e] += crow[e];
            }
        }
    if (!nc) { /* :425-426 */
        touch(p, layer);
        const uint64_t *f = p->freq + (size_t)layer * E;
        const uint16_t *fo = p->freq_order + (size_t)layer * E;
        for (int j = 0; j < p->freq_n[layer]; j++) {
            if (!cand[fo[j]]) order[nc++] = fo[j];
            cand[fo[j]] += f[fo[j]];
        }
    }
    const int has_next = layer + 1 < p->L;
    if (has_next) { /* :427-428 */
        touch(p, layer + 1);
        const uint64_t *f = p->freq + (size_t)(layer + 1) * E;
        const uint16_t *fo = p->freq_order + (size_t)(layer + 1) * E;
        for (int j = 0; j < p->freq_n[layer + 1]; j++) {
            if (!cand[fo[j]]) order[nc++] = fo[j];
            cand[fo[j]] += 2 * f[fo[j]];
        }
    }
    *npick = most_common(order, nc, cand, depth, pick); /* :429-430 */
    if (has_next)                                        /* :431-435 */
        *nnext = most_common(p->freq_order + (size_t)(layer + 1) * E, p->freq_n[layer + 1],
                             p->freq + (size_t)(layer + 1) * E, depth, next);
    free(cand);
    free(order);
    return 0;
}

uint64_t qmoe_predictor_count(const qmoe_predictor *p, int layer, int expert) {
    if (!p || layer < 0 || layer >= p->L || expert < 0 || expert >= p->E) return 0;
    return p->freq[(size_t)layer * p->E + expert];
}

uint64_t qmoe_predictor_routes(const qmoe_predictor *p) { return p ? p->routes : 0; }

int qmoe_predictor_frequent(const qmoe_predictor *p, int want, int32_t *layer, int32_t *expert,
                            uint64_t *count) {
    if (!p || want < 0 || (want && (!layer || !expert || !count))) return -1;
    /* (layer, expert) keys in the reference's insertion order: layers as
     * their counters were created, experts as first routed */
    int *lorder = malloc((size_t)p->L * sizeof(int));
    if (!lorder) return -1;
    int nl = 0;
    for (int s = 0; s < p->next_seq; s++)
        for (int l = 0; l < p->L; l++)
            if (p->layer_seq[l] == s) lorder[nl++] = l;
    int got = 0;
    uint64_t last = UINT64_MAX;
    int last_pos = -1; /* position of the last pick in insertion order */
    while (got < want) {
        int bl = -1, be = -1, bpos = -1, pos = 0;
        uint64_t bc = 0;
        for (int a = 0; a < nl; a++) {
            const int l = lorder[a];
            const uint64_t *f = p->freq + (size_t)l * p->E;
            const uint16_t *fo = p->freq_order + (size_t)l * p->E;
            for (int j = 0; j < p->freq_n[l]; j++, pos++) {
                const uint64_t c = f[fo[j]];
                /* the next key in (count desc, position asc) after the last pick */
                if (c > last || (c == last && pos <= last_pos)) continue;
                if (bl < 0 || c > bc) {
                    bl = l, be = fo[j], bc = c, bpos = pos;
                }
            }
        }
        if (bl < 0) break;
        layer[got] = bl;
        expert[got] = be;
        count[got] = bc;
        got++;
        last = bc;
        last_pos = bpos;
    }
    free(lorder);
    return got;
}
