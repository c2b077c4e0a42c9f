/*
 * The C port's side of the drop-in, checked by the compiler and the linker:
 * this file includes the reference's own c/src/model.c (unmodified) together
 * with qmoe.h and writes the integration the way a maintainer of the port
 * would (config from qcfg, the layer upload from the checkpoint directory, the
 * MoE call of model_forward, the counters). It runs without a GPU: main only
 * reports that the pieces resolved.
 */
#include "model.c"

#include <stddef.h>

#include "qmoe.h"

/* the port passes its err_t straight through (c/src/util.h:11-13) */
_Static_assert(sizeof(err_t) == sizeof(qmoe_err), "err_t and qmoe_err differ in size");
_Static_assert(offsetof(err_t, msg) == offsetof(qmoe_err, msg), "err_t.msg moved");
_Static_assert(sizeof(((err_t *)0)->msg) == sizeof(((qmoe_err *)0)->msg), "msg sizes differ");

static qmoe_ctx *port_ctx;

/* model_load: replaces cache_init(&m->expert_cache, ...) (model.c:1806) */
static int port_create(const qmodel *m, uint64_t expert_budget, err_t *err) {
    const qcfg *c = &m->cfg;
    qmoe_config qc = {0};
    qc.hidden = c->hidden_size;
    qc.num_experts = c->num_experts;
    qc.top_k = c->num_experts_per_tok;
    qc.moe_inter = c->moe_intermediate_size;
    qc.group_size = c->group_size;
    qc.bits = c->bits;
    qc.num_layers = c->num_layers;
    qc.max_tokens = 4096;
    qc.pool_bytes = expert_budget;
    qc.policy = QMOE_POLICY_ADAPTIVE;
    qc.prefetch_depth = 2;
    port_ctx = qmoe_create(&qc, (qmoe_err *)err);
    return port_ctx ? 0 : -1;
}

/* model_load, after the layers: every MoE layer from the checkpoint files */
static int port_upload(const char *dir, int io_workers, int n_layers, err_t *err) {
    qmoe_ckpt *ck = qmoe_ckpt_open(dir, io_workers, (qmoe_err *)err);
    if (!ck) return -1;
    int rc = 0;
    for (int i = 0; i < n_layers && rc == 0; i++)
        rc = qmoe_upload_layer_ckpt(port_ctx, i, ck, i, (qmoe_err *)err);
    qmoe_ckpt_close(ck);
    return rc;
}

/* model_forward, model.c:1712: moe_forward's arguments, the scratch unused */
static int port_moe(qmodel *m, qlayer *l, const float *x, int n, float *out, float *scratch,
                    err_t *err) {
    (void)scratch;
    return qmoe_forward(port_ctx, (int)(l - m->layers), x, n, out, (qmoe_err *)err);
}

/* the port's counters (c/src/model.h:18-24) */
static void port_stats(qstats *s) {
    qmoe_stats q;
    if (qmoe_stats_get(port_ctx, &q) != 0) return;
    s->expert_loads = q.expert_loads;
    s->expert_bytes = q.expert_bytes;
    s->expert_wait_seconds = q.expert_wait_seconds;
    s->prefill_calls = q.prefill_calls;
    s->decode_calls = q.decode_calls;
}

typedef int (*moe_fn)(qmodel *, qlayer *, const float *, int, float *, float *, err_t *);

int main(void) {
    /* the replacement has moe_forward's exact type */
    moe_fn ref = moe_forward, ours = port_moe;
    int (*create)(const qmodel *, uint64_t, err_t *) = port_create;
    int (*upload)(const char *, int, int, err_t *) = port_upload;
    void (*stats)(qstats *) = port_stats;
    printf("drop-in resolved: %d %s\n", ref != ours && create && upload && stats, qmoe_version());
    return 0;
}
