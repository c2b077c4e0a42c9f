/*
 * qmoe_cache.c - byte-budgeted expert cache bookkeeping (host C).
 *
 * Behaviour follows the reference's cache (c/src/cache.c, c/src/cache.h):
 *  - keys are (layer << 32) | expert, the high half is the partition
 *    (cache.h:15, cache.c:76-78);
 *  - put rejects an entry larger than the budget, replaces an existing key
 *    (keeping its pin and hot flags, dropping it first), then evicts until the
 *    new entry fits; when nothing is evictable the put is rejected
 *    (cache.c:221-266);
 *  - victim choice (cache.c:99-163): pinned entries are never chosen; when
 *    partitions > 0 and some unpinned entry's partition holds more than
 *    budget/partitions bytes, only over-share partitions are candidates;
 *    cold entries beat hot ones; among equals LRU takes the least recently
 *    touched, LFU the lowest frequency and ADAPTIVE the lowest
 *    (freq + 4*hot) / nbytes, ties to the least recently touched. The
 *    reference's scan restarts its score at 0 when it moves from a hot
 *    candidate to a cold one; that is kept, so results match it;
 *  - get counts a hit (frequency + 1, recency refreshed) or a miss; peek
 *    touches nothing (cache.c:185-209).
 * Recency uses a logical clock instead of CLOCK_MONOTONIC nanoseconds, so
 * equal timestamps cannot occur.
 *
 * The structure is a chained hash table plus an intrusive recency list and a
 * per-partition byte tally (no O(n^2) partition scan). Values are opaque
 * 64-bit tokens; the GPU context stores HBM slot numbers in them.
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/qmoe.h"
#include "qmoe_internal.h"

typedef struct node {
    uint64_t key, value, nbytes, freq, touched;
    int pinned, hot;
    struct node *hnext;        /* hash chain */
    struct node *prev, *next;  /* recency: head = most recent */
} node;

typedef struct part {
    uint32_t id;
    uint64_t bytes;
    struct part *next;
} part;

struct qmoe_cache {
    uint64_t max_bytes;
    int policy, partitions;
    node **buckets;
    size_t nbuckets, count;
    node *head, *tail;
    part **pbuckets; /* partition tallies, 256 chains */
    uint64_t clock;
    uint64_t bytes, peak_bytes, hits, misses, evictions, rejected, pinned_count;
    pthread_mutex_t lock;
};

static size_t hidx(const qmoe_cache *c, uint64_t key) {
    uint64_t z = key * 0x9E3779B97F4A7C15ull;
    return (size_t)(z >> 20) & (c->nbuckets - 1);
}

static node *find(const qmoe_cache *c, uint64_t key) {
    for (node *n = c->buckets[hidx(c, key)]; n; n = n->hnext)
        if (n->key == key) return n;
    return NULL;
}

static part *part_of(qmoe_cache *c, uint32_t id, int create) {
    part **b = &c->pbuckets[id & 255];
    for (part *p = *b; p; p = p->next)
        if (p->id == id) return p;
    if (!create) return NULL;
    part *p = calloc(1, sizeof(part));
    if (!p) return NULL;
    p->id = id;
    p->next = *b;
    *b = p;
    return p;
}

static uint64_t part_bytes(qmoe_cache *c, uint64_t key) {
    part *p = part_of(c, (uint32_t)(key >> 32), 0);
    return p ? p->bytes : 0;
}

static void unlink_lru(qmoe_cache *c, node *n) {
    if (n->prev) n->prev->next = n->next; else c->head = n->next;
    if (n->next) n->next->prev = n->prev; else c->tail = n->prev;
    n->prev = n->next = NULL;
}

static void push_front(qmoe_cache *c, node *n) {
    n->prev = NULL;
    n->next = c->head;
    if (c->head) c->head->prev = n;
    c->head = n;
    if (!c->tail) c->tail = n;
}

static void grow(qmoe_cache *c) {
    size_t nb = c->nbuckets * 2;
    node **b = calloc(nb, sizeof(node *));
    if (!b) return;
    node **old = c->buckets;
    size_t on = c->nbuckets;
    c->buckets = b;
    c->nbuckets = nb;
    for (size_t i = 0; i < on; i++) {
        node *n = old[i];
        while (n) {
            node *nx = n->hnext;
            size_t h = hidx(c, n->key);
            n->hnext = b[h];
            b[h] = n;
            n = nx;
        }
    }
    free(old);
}

static void drop(qmoe_cache *c, node *n) {
    node **pp = &c->buckets[hidx(c, n->key)];
    while (*pp != n) pp = &(*pp)->hnext;
    *pp = n->hnext;
    unlink_lru(c, n);
    c->bytes -= n->nbytes;
    part *p = part_of(c, (uint32_t)(n->key >> 32), 0);
    if (p) p->bytes -= n->nbytes;
    if (n->pinned) c->pinned_count--;
    c->count--;
    free(n);
}

static node *pick_victim(qmoe_cache *c) {
    uint64_t fair = c->partitions > 0 ? c->max_bytes / (uint64_t)c->partitions : 0;
    int any_over = 0;
    if (c->partitions > 0)
        for (node *e = c->tail; e; e = e->prev)
            if (!e->pinned && part_bytes(c, e->key) > fair) { any_over = 1; break; }
    node *best = NULL;
    double best_score = 0;
    uint64_t best_touched = 0;
    for (node *e = c->tail; e; e = e->prev) {
        if (e->pinned) continue;
        if (c->partitions > 0 && any_over && part_bytes(c, e->key) <= fair) continue;
        if (best && !e->hot && best->hot) {
            best = e;
            best_score = 0;
            best_touched = e->touched;
            continue;
        }
        if (best && e->hot && !best->hot) continue;
        double score;
        if (c->policy == QMOE_POLICY_LRU) score = 0;
        else if (c->policy == QMOE_POLICY_LFU) score = (double)e->freq;
        else score = (double)(e->freq + (e->hot ? 4 : 0)) / (double)(e->nbytes ? e->nbytes : 1);
        int better;
        if (!best) better = 1;
        else if (c->policy == QMOE_POLICY_LRU) better = e->touched < best_touched;
        else better = score < best_score || (score == best_score && e->touched < best_touched);
        if (better) {
            best = e;
            best_score = score;
            best_touched = e->touched;
        }
    }
    return best;
}

qmoe_cache *qmoe_cache_new(uint64_t max_bytes, int policy, int partitions) {
    qmoe_cache *c = calloc(1, sizeof(*c));
    if (!c) return NULL;
    c->max_bytes = max_bytes;
    c->policy = policy;
    c->partitions = partitions;
    c->nbuckets = 1024;
    c->buckets = calloc(c->nbuckets, sizeof(node *));
    c->pbuckets = calloc(256, sizeof(part *));
    if (!c->buckets || !c->pbuckets) {
        free(c->buckets);
        free(c->pbuckets);
        free(c);
        return NULL;
    }
    pthread_mutex_init(&c->lock, NULL);
    return c;
}

void qmoe_cache_free(qmoe_cache *c) {
    if (!c) return;
    node *n = c->head;
    while (n) {
        node *nx = n->next;
        free(n);
        n = nx;
    }
    for (int i = 0; i < 256; i++) {
        part *p = c->pbuckets[i];
        while (p) {
            part *nx = p->next;
            free(p);
            p = nx;
        }
    }
    free(c->pbuckets);
    free(c->buckets);
    pthread_mutex_destroy(&c->lock);
    free(c);
}

int qmoe_cache_peek(qmoe_cache *c, uint64_t key, uint64_t *value) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    if (n && value) *value = n->value;
    pthread_mutex_unlock(&c->lock);
    return n != NULL;
}

int qmoe_cache_get(qmoe_cache *c, uint64_t key, uint64_t *value) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    if (n) {
        n->freq++;
        n->touched = ++c->clock;
        unlink_lru(c, n);
        push_front(c, n);
        c->hits++;
        if (value) *value = n->value;
    } else {
        c->misses++;
    }
    pthread_mutex_unlock(&c->lock);
    return n != NULL;
}

static void note(uint64_t v, uint64_t *ev, size_t cap, size_t *nev) {
    if (ev && *nev < cap) ev[*nev] = v;
    (*nev)++;
}

int qmoe_cache_put(qmoe_cache *c, uint64_t key, uint64_t value,
                   uint64_t nbytes, int pin, int hot, uint64_t *evicted,
                   size_t max_evicted, size_t *n_evicted) {
    size_t nev = 0;
    pthread_mutex_lock(&c->lock);
    int ok = 0;
    if (c->max_bytes > 0 && nbytes > c->max_bytes) {
        c->rejected++;
        goto out;
    }
    node *old = find(c, key);
    if (old) {
        pin = pin || old->pinned;
        hot = hot || old->hot;
        note(old->value, evicted, max_evicted, &nev);
        drop(c, old);
    }
    uint64_t nvict = 0;
    while (c->max_bytes > 0 && c->bytes + nbytes > c->max_bytes) {
        node *v = pick_victim(c);
        if (!v) {
            /* as cache.c:236-242: victims already dropped are not counted */
            c->rejected++;
            goto out;
        }
        note(v->value, evicted, max_evicted, &nev);
        drop(c, v);
        nvict++;
    }
    node *n = calloc(1, sizeof(node));
    part *p = part_of(c, (uint32_t)(key >> 32), 1);
    if (!n || !p) {
        free(n);
        c->rejected++;
        c->evictions += nvict;
        goto out;
    }
    if (c->count + 1 > c->nbuckets * 3 / 4) grow(c);
    n->key = key;
    n->value = value;
    n->nbytes = nbytes;
    n->pinned = pin;
    n->hot = hot;
    n->freq = 1;
    n->touched = ++c->clock;
    size_t h = hidx(c, key);
    n->hnext = c->buckets[h];
    c->buckets[h] = n;
    push_front(c, n);
    p->bytes += nbytes;
    c->bytes += nbytes;
    if (c->bytes > c->peak_bytes) c->peak_bytes = c->bytes;
    c->count++;
    if (pin) c->pinned_count++;
    c->evictions += nvict;
    ok = 1;
out:
    pthread_mutex_unlock(&c->lock);
    if (n_evicted) *n_evicted = nev;
    return ok;
}

int qmoe_cache_pin(qmoe_cache *c, uint64_t key) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    int ok = 0;
    if (n && !n->pinned) {
        n->pinned = 1;
        c->pinned_count++;
        ok = 1;
    }
    pthread_mutex_unlock(&c->lock);
    return ok;
}

int qmoe_cache_unpin(qmoe_cache *c, uint64_t key) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    int ok = 0;
    if (n && n->pinned) {
        n->pinned = 0;
        c->pinned_count--;
        ok = 1;
    }
    pthread_mutex_unlock(&c->lock);
    return ok;
}

int qmoe_cache_mark_hot(qmoe_cache *c, uint64_t key, int hot) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    if (n) n->hot = hot;
    pthread_mutex_unlock(&c->lock);
    return n != NULL;
}

int qmoe_cache_erase(qmoe_cache *c, uint64_t key, uint64_t *value) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    if (n) {
        if (value) *value = n->value;
        drop(c, n);
    }
    pthread_mutex_unlock(&c->lock);
    return n != NULL;
}

int qmoe__cache_set_value(qmoe_cache *c, uint64_t key, uint64_t value) {
    pthread_mutex_lock(&c->lock);
    node *n = find(c, key);
    if (n) n->value = value;
    pthread_mutex_unlock(&c->lock);
    return n != NULL;
}

qmoe_cache_stats qmoe_cache_stats_get(qmoe_cache *c) {
    qmoe_cache_stats s;
    memset(&s, 0, sizeof(s));
    pthread_mutex_lock(&c->lock);
    s.hits = c->hits;
    s.misses = c->misses;
    s.evictions = c->evictions;
    s.rejected = c->rejected;
    s.pinned = c->pinned_count;
    s.bytes = c->bytes;
    s.peak_bytes = c->peak_bytes;
    s.size = c->count;
    for (node *n = c->head; n; n = n->next)
        if (n->hot) s.hot++;
    pthread_mutex_unlock(&c->lock);
    return s;
}
