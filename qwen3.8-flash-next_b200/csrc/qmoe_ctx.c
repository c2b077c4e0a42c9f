/*
 * qmoe_ctx.c - host side of the B200 MoE layer (C, CUDA runtime API).
 *
 * Replaces, for one GPU:
 *   moe_forward   c/src/model.c:1281-1405  -> qmoe_forward / qmoe_forward_dev
 *   experts_load  c/src/model.c:539-674    -> qmoe_experts_load (pinned host
 *                                             store -> HBM slot copies instead
 *                                             of pread + fp32 dequant)
 *   expert cache  c/src/cache.c            -> qmoe_cache over HBM slot numbers
 *   route stats / prefetch, streaming.py:400-435 -> qmoe_record_route,
 *                                             qmoe_prefetch_predictions (the
 *                                             predictor is qmoe_predict.c)
 *
 * The context owns every device buffer: router, shared gate and shared
 * expert per layer, the expert pool (fixed-size slots), the expert -> slot
 * table the kernels read, and workspaces sized for cfg.max_tokens at create
 * time, so a forward call allocates nothing.
 */
#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../include/qmoe.h"
#include "qmoe_internal.h"

#define NO_OWNER UINT64_MAX

typedef struct {
    cudaGraphExec_t tok_graph; /* host-pointer single-token call, captured once */
    uint16_t *router;     /* [E, d] */
    uint16_t *shgate;     /* [d] */
    float *bias;          /* [E] or NULL */
    uint8_t *shared_slot; /* slot layout */
    float router_wmax;    /* max_e |router row e|_2, rounded up */
    int ready;
    qk_hc_dev hc;         /* the hyper connection around the block (hc.hc == 0: none) */
} layer_dev;

struct qmoe_ctx {
    qmoe_config cfg;
    qk_layout L;
    int num_sms;
    cudaStream_t stream, copy_stream;
    cudaEvent_t copy_done;
    cudaEvent_t compute_mark; /* streaming: recorded on the compute stream before a fill */
    int pf_outstanding;       /* prefetched experts neither routed to nor evicted yet */
    /* hyper-connection workspaces, [max_tokens] rows of hc_lr / hc_n / d values */
    float *hc_W, *hc_R, *hc_INJ, *hc_mixed, *hc_y;
    unsigned long long *hc_sync; /* the one-token pre-pass's grid-barrier counter */
    void *hc_dsync;              /* the decode kernel's counter and exchange area in hc_pre launches */
    int hc_lr, hc_n;
    int max_speculative;      /* their cap (ExpertStore._max_speculative) */
    /* device error word and output share one allocation (err at 0, out at
       256) so a host-pointer forward reads both back with one copy; the
       pinned mirror has the same layout */
    uint8_t *io_dev, *io_pin;
    int *err_dev;
    int *err_host;
    /* single-token host calls: completions counted by the report kernel at
     * io + 4 (device counter, pinned mirror); tok_seq = the count expected */
    unsigned *tok_ctr_dev, *tok_ctr_host;
    unsigned tok_seq;
    void *dsync;     /* launch counter + exchange area of the single-launch decode kernel */
    layer_dev *layers;
    /* expert pool */
    uint8_t *pool;
    int nslots;
    int resident_all;
    int32_t *slot_of_dev;  /* [num_layers * E] */
    int32_t *slot_of_host; /* [num_layers * E] */
    uint64_t *slot_owner;  /* [nslots] */
    int *free_slots;
    int nfree;
    qmoe_cache *cache;
    uint8_t *host_store;   /* pinned [num_layers][local experts] slots when streaming */
    /* the pool holds nslots routed slots followed by one shared-expert slot
       per layer (slot nslots + layer), so TMA descriptors cover both */
    qk_prefill *prefill;   /* tcgen05 multi-token path, NULL if the shape is not covered */
    /* workspaces */
    float *x_dev, *out_dev, *logits, *wts, *sgate, *h;
    int32_t *idx;
    float *x_pin, *out_pin;
    int32_t *idx_pin;
    uint8_t *wave_pin;      /* streaming: [E + 1] expert mask of one wave */
    int last_T;
    qmoe_stats stats;
    /* route statistics and prediction (streaming.py:400-435) */
    qmoe_predictor *pred;
    int32_t *sel_buf;       /* [E] one step's selected experts */
    unsigned char *pf_mark; /* [num_layers * E] filled by a prefetch, not yet routed to */
    /* diagnostics: per-kernel event timing (qmoe_profile_forward) */
    int profile;
    int prof_kernels; /* kernels of the last forward: 1 (single launch) or 4 */
    cudaEvent_t pev[8];
    pthread_mutex_t lock;
    /* expert parallelism */
    int ep_world, ep_rank, ep_lo, ep_hi; /* experts [ep_lo, ep_hi) are local */
    ncclComm_t ep_comm;
    int ep_p2p; /* the exchanges go through peer memory (qk_ep_*_p2p) */
    int32_t *ep_recv_pin;  /* streaming: pinned copy of the received rows' expert ids */
    /* MoE-only stack: the normalised layer input and the layer output */
    float *stk_xn, *stk_y; /* fp32 [max_tokens, d] each */
};

static int check_dev_err(qmoe_ctx *c, cudaStream_t st, qmoe_err *err);
static int report_dev_err(qmoe_ctx *c, int code, cudaStream_t st, qmoe_err *err);

static void seterr(qmoe_err *err, const char *fmt, ...) {
    if (!err) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err->msg, sizeof(err->msg), fmt, ap);
    va_end(ap);
}

#define CK(call)                                                                 \
    do {                                                                         \
        cudaError_t e_ = (call);                                                 \
        if (e_ != cudaSuccess) {                                                 \
            seterr(err, "%s:%d %s: %s", __FILE__, __LINE__, #call,               \
                   cudaGetErrorString(e_));                                      \
            goto fail;                                                           \
        }                                                                        \
    } while (0)

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* ------------------------------------------------------------------ layout */

int qk_layout_init(qk_layout *L, int d, int E, int k, int I, int g) {
    if (d <= 0 || E <= 0 || k <= 0 || I <= 0 || g <= 0) return -1;
    if (g % 32 || d % g || I % g || d % 256 || I % 32) return -1;
    int units = I / 32;
    if (units > 32 || (units & (units - 1))) return -1; /* down: lanes per row */
    if (k > 32 || k > E || E > 1024) return -1;
    L->d = d; L->E = E; L->k = k; L->I = I; L->g = g;
    L->gu_row = d / 2 + d / 2 + (d / g) * 8;
    int drow = I / 2 + (I / g) * 4;
    L->d_row = (drow + 15) / 16 * 16;
    L->gu_bytes = (size_t)I * (size_t)L->gu_row;
    size_t s = L->gu_bytes + (size_t)d * (size_t)L->d_row;
    L->slot_bytes = (s + 255) / 256 * 256;
    if (L->gu_row % 16) return -1;
    return 0;
}

size_t qmoe_slot_bytes(const qmoe_config *cfg) {
    qk_layout L;
    if (!cfg || qk_layout_init(&L, cfg->hidden, cfg->num_experts, cfg->top_k, cfg->moe_inter,
                               cfg->group_size))
        return 0;
    return L.slot_bytes;
}

void qk_pack_expert(const qk_layout *L, const uint32_t *gq, const uint16_t *gs,
                    const uint16_t *gb, const uint32_t *uq, const uint16_t *us,
                    const uint16_t *ub, const uint32_t *dq, const uint16_t *ds,
                    const uint16_t *db, uint8_t *slot) {
    int d = L->d, I = L->I, g = L->g, G = d / g, Gd = I / g;
    for (int n = 0; n < I; n++) {
        uint8_t *row = slot + (size_t)n * L->gu_row;
        memcpy(row, gq + (size_t)n * (d / 8), (size_t)d / 2);
        memcpy(row + d / 2, uq + (size_t)n * (d / 8), (size_t)d / 2);
        uint16_t *quad = (uint16_t *)(row + d);
        for (int j = 0; j < G; j++) {
            quad[4 * j + 0] = gs[(size_t)n * G + j];
            quad[4 * j + 1] = gb[(size_t)n * G + j];
            quad[4 * j + 2] = us[(size_t)n * G + j];
            quad[4 * j + 3] = ub[(size_t)n * G + j];
        }
    }
    uint8_t *dsec = slot + L->gu_bytes;
    for (int n = 0; n < d; n++) {
        uint8_t *row = dsec + (size_t)n * L->d_row;
        memset(row, 0, (size_t)L->d_row);
        memcpy(row, dq + (size_t)n * (I / 8), (size_t)I / 2);
        uint16_t *pair = (uint16_t *)(row + I / 2);
        for (int j = 0; j < Gd; j++) {
            pair[2 * j + 0] = ds[(size_t)n * Gd + j];
            pair[2 * j + 1] = db[(size_t)n * Gd + j];
        }
    }
    size_t used = L->gu_bytes + (size_t)d * L->d_row;
    if (used < L->slot_bytes) memset(slot + used, 0, L->slot_bytes - used);
}

static void pack_routed(const qmoe_ctx *c, const qmoe_layer_weights *w, int e, uint8_t *slot) {
    const qk_layout *L = &c->L;
    size_t d = (size_t)L->d, I = (size_t)L->I, g = (size_t)L->g;
    size_t qo = (size_t)e * I * (d / 8), so = (size_t)e * I * (d / g);
    size_t dqo = (size_t)e * d * (I / 8), dso = (size_t)e * d * (I / g);
    qk_pack_expert(L, w->gate.q + qo, w->gate.scales + so, w->gate.biases + so, w->up.q + qo,
                   w->up.scales + so, w->up.biases + so, w->down.q + dqo, w->down.scales + dso,
                   w->down.biases + dso, slot);
}

/* ---------------------------------------------------------------- NCCL */

/* NCCL is resolved at run time (dlopen of libnccl.so.2): a process that
 * already loaded it (PyTorch does) shares that copy, and contexts that never
 * use expert parallelism need no NCCL at all. */
typedef struct {
    int ok;
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*group_start)(void);
    ncclResult_t (*group_end)(void);
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char *(*error_string)(ncclResult_t);
} nccl_fns;

static nccl_fns g_nccl;
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    *(void **)&g_nccl.get_unique_id = dlsym(h, "ncclGetUniqueId");
    *(void **)&g_nccl.comm_init_rank = dlsym(h, "ncclCommInitRank");
    *(void **)&g_nccl.comm_destroy = dlsym(h, "ncclCommDestroy");
    *(void **)&g_nccl.group_start = dlsym(h, "ncclGroupStart");
    *(void **)&g_nccl.group_end = dlsym(h, "ncclGroupEnd");
    *(void **)&g_nccl.send = dlsym(h, "ncclSend");
    *(void **)&g_nccl.recv = dlsym(h, "ncclRecv");
    *(void **)&g_nccl.error_string = dlsym(h, "ncclGetErrorString");
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy &&
                g_nccl.group_start && g_nccl.group_end && g_nccl.send && g_nccl.recv &&
                g_nccl.error_string;
}

static const nccl_fns *nccl_api(void) {
    pthread_once(&g_nccl_once, nccl_load);
    return &g_nccl;
}

/* ----------------------------------------------------------------- create */

static void hc_free(qk_hc_dev *w) {
    cudaFree(w->norm);
    cudaFree(w->down_q);
    cudaFree(w->down_s);
    cudaFree(w->down_b);
    cudaFree(w->down_bf);
    cudaFree(w->up_q);
    cudaFree(w->up_s);
    cudaFree(w->up_b);
    cudaFree(w->up_bf);
    cudaFree(w->inject);
    memset(w, 0, sizeof(*w));
}

void qmoe_destroy(qmoe_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    if (c->layers) {
        for (int l = 0; l < c->cfg.num_layers; l++) {
            if (c->layers[l].tok_graph) cudaGraphExecDestroy(c->layers[l].tok_graph);
            cudaFree(c->layers[l].router);
            cudaFree(c->layers[l].shgate);
            cudaFree(c->layers[l].bias);
            hc_free(&c->layers[l].hc);
        }
        free(c->layers);
    }
    cudaFree(c->pool);
    cudaFree(c->slot_of_dev);
    cudaFree(c->io_dev);
    cudaFree(c->dsync);
    cudaFree(c->x_dev);
    cudaFree(c->logits);
    cudaFree(c->idx);
    cudaFree(c->wts);
    cudaFree(c->sgate);
    cudaFree(c->h);
    cudaFree(c->stk_xn);
    cudaFree(c->stk_y);
    cudaFree(c->hc_W);
    cudaFree(c->hc_R);
    cudaFree(c->hc_INJ);
    cudaFree(c->hc_mixed);
    cudaFree(c->hc_y);
    cudaFree(c->hc_sync);
    cudaFree(c->hc_dsync);
    cudaFreeHost(c->x_pin);
    cudaFreeHost(c->idx_pin);
    cudaFreeHost(c->wave_pin);
    cudaFreeHost(c->io_pin);
    cudaFreeHost(c->host_store);
    free(c->slot_of_host);
    free(c->slot_owner);
    free(c->free_slots);
    qmoe_predictor_free(c->pred);
    free(c->sel_buf);
    free(c->pf_mark);
    if (c->cache) qmoe_cache_free(c->cache);
    qk_prefill_destroy(c->prefill);
    if (c->ep_comm) nccl_api()->comm_destroy(c->ep_comm);
    cudaFreeHost(c->ep_recv_pin);
    if (c->copy_done) cudaEventDestroy(c->copy_done);
    if (c->compute_mark) cudaEventDestroy(c->compute_mark);
    for (int i = 0; i < 8; i++)
        if (c->pev[i]) cudaEventDestroy(c->pev[i]);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    pthread_mutex_destroy(&c->lock);
    free(c);
}

qmoe_ctx *qmoe_create(const qmoe_config *cfg, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!cfg) {
        seterr(err, "qmoe_create: NULL config");
        return NULL;
    }
    if (cfg->bits != 4) {
        seterr(err, "qmoe_create: only 4-bit experts are supported (bits=%d)", cfg->bits);
        return NULL;
    }
    if (cfg->num_layers < 1 || cfg->max_tokens < 1) {
        seterr(err, "qmoe_create: num_layers and max_tokens must be positive");
        return NULL;
    }
    qmoe_ctx *c = calloc(1, sizeof(*c));
    if (!c) {
        seterr(err, "qmoe_create: out of host memory");
        return NULL;
    }
    pthread_mutex_init(&c->lock, NULL);
    c->cfg = *cfg;
    if (qk_layout_init(&c->L, cfg->hidden, cfg->num_experts, cfg->top_k, cfg->moe_inter,
                       cfg->group_size)) {
        seterr(err,
               "qmoe_create: unsupported shape d=%d E=%d k=%d I=%d g=%d (need d %% 256 == 0, "
               "g %% 32 == 0, I/32 a power of two <= 32, k <= 32, E <= 1024)",
               cfg->hidden, cfg->num_experts, cfg->top_k, cfg->moe_inter, cfg->group_size);
        free(c);
        return NULL;
    }
    const int Lz = cfg->num_layers, E = cfg->num_experts, T = cfg->max_tokens;
    const qk_layout *L = &c->L;
    c->ep_world = cfg->ep_world > 1 ? cfg->ep_world : 1;
    c->ep_rank = c->ep_world > 1 ? cfg->ep_rank : 0;
    if (c->ep_world > 1 && (E % c->ep_world || c->ep_rank < 0 || c->ep_rank >= c->ep_world ||
                            c->ep_world > 64)) {
        seterr(err, "qmoe_create: expert parallelism needs E %% ep_world == 0 and "
                    "0 <= ep_rank < ep_world <= 64");
        free(c);
        return NULL;
    }
    c->ep_lo = c->ep_rank * (E / c->ep_world);
    c->ep_hi = c->ep_lo + E / c->ep_world;
    CK(cudaSetDevice(cfg->device));
    CK(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, cfg->device));
    {
        int major = 0, minor = 0;
        CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cfg->device));
        CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, cfg->device));
        if (major != 10 || minor != 0) {
            seterr(err, "qmoe_create: device %d is sm_%d%d; this library is built for sm_100a only",
                   cfg->device, major, minor);
            goto fail;
        }
    }
    CK((cudaError_t)qk_prepare_kernels());
    for (int i = 0; i < 8; i++) CK(cudaEventCreate(&c->pev[i]));
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&c->copy_done, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&c->compute_mark, cudaEventDisableTiming));
    {
        const size_t io = 256 + (size_t)T * L->d * sizeof(float);
        CK(cudaMalloc((void **)&c->io_dev, io));
        CK(cudaMemset(c->io_dev, 0, 256));
        CK(cudaMallocHost((void **)&c->io_pin, io));
        memset(c->io_pin, 0, 256);
        c->err_dev = (int *)c->io_dev;
        c->err_host = (int *)c->io_pin;
        c->tok_ctr_dev = (unsigned *)(c->io_dev + 4);
        c->tok_ctr_host = (unsigned *)(c->io_pin + 4);
        c->out_dev = (float *)(c->io_dev + 256);
        c->out_pin = (float *)(c->io_pin + 256);
    }
    CK(cudaMalloc(&c->dsync, qk_decode_sync_bytes(L)));
    CK(cudaMemset(c->dsync, 0, qk_decode_sync_bytes(L)));
    c->layers = calloc((size_t)Lz, sizeof(layer_dev));
    if (!c->layers) {
        seterr(err, "qmoe_create: out of host memory");
        goto fail;
    }
    /* pool */
    {
        uint64_t total = (uint64_t)Lz * (uint64_t)E;
        uint64_t local = (uint64_t)Lz * (uint64_t)(c->ep_hi - c->ep_lo);
        uint64_t want = cfg->pool_bytes ? cfg->pool_bytes / L->slot_bytes : local;
        if (want > local) want = local;
        if (want < (uint64_t)cfg->top_k) {
            seterr(err, "qmoe_create: pool_bytes holds %llu slots, fewer than top_k=%d",
                   (unsigned long long)want, cfg->top_k);
            goto fail;
        }
        c->nslots = (int)want;
        c->resident_all = want == local;
        /* prefetches in flight: min(cache slots, max(2 workers, prefetch_count
         * x layers)) as ExpertStore sizes it (streaming.py:115), with the
         * copy stream as the one I/O worker */
        {
            const long spec = (long)(cfg->prefetch_depth > 0 ? cfg->prefetch_depth : 0) * Lz;
            c->max_speculative = (int)(spec > 2 ? (spec < c->nslots ? spec : c->nslots)
                                               : (2 < c->nslots ? 2 : c->nslots));
        }
        CK(cudaMalloc((void **)&c->pool, ((size_t)c->nslots + Lz) * L->slot_bytes));
        for (int l = 0; l < Lz; l++)
            c->layers[l].shared_slot = c->pool + ((size_t)c->nslots + l) * L->slot_bytes;
        CK(cudaMalloc((void **)&c->slot_of_dev, (size_t)total * sizeof(int32_t)));
        CK(cudaMemset(c->slot_of_dev, 0xff, (size_t)total * sizeof(int32_t)));
        c->slot_of_host = malloc((size_t)total * sizeof(int32_t));
        c->slot_owner = malloc((size_t)c->nslots * sizeof(uint64_t));
        c->free_slots = malloc((size_t)c->nslots * sizeof(int));
        c->pred = qmoe_predictor_new(Lz, E);
        c->sel_buf = malloc((size_t)E * sizeof(int32_t));
        c->pf_mark = calloc((size_t)total, 1);
        if (!c->slot_of_host || !c->slot_owner || !c->free_slots || !c->pred || !c->sel_buf ||
            !c->pf_mark) {
            seterr(err, "qmoe_create: out of host memory");
            goto fail;
        }
        memset(c->slot_of_host, 0xff, (size_t)total * sizeof(int32_t));
        for (int s = 0; s < c->nslots; s++) {
            c->slot_owner[s] = NO_OWNER;
            c->free_slots[s] = c->nslots - 1 - s; /* pop order 0, 1, 2, ... */
        }
        c->nfree = c->nslots;
        c->cache = qmoe_cache_new((uint64_t)c->nslots * L->slot_bytes, cfg->policy,
                                  c->resident_all ? 0 : Lz);
        if (!c->cache) {
            seterr(err, "qmoe_create: out of host memory");
            goto fail;
        }
        if (!c->resident_all) { /* the local experts only */
            size_t hs = (size_t)local * L->slot_bytes;
            CK(cudaHostAlloc((void **)&c->host_store, hs, cudaHostAllocPortable));
        }
    }
    /* workspaces for max_tokens */
    CK(cudaMalloc((void **)&c->x_dev, (size_t)T * L->d * sizeof(float)));
    CK(cudaMalloc((void **)&c->logits, (size_t)T * (E + 1) * sizeof(float)));
    CK(cudaMalloc((void **)&c->idx, (size_t)T * L->k * sizeof(int32_t)));
    CK(cudaMalloc((void **)&c->wts, (size_t)T * L->k * sizeof(float)));
    CK(cudaMalloc((void **)&c->sgate, (size_t)T * sizeof(float)));
    CK(cudaMalloc((void **)&c->h, (size_t)T * (L->k + 1) * L->I * sizeof(float)));
    CK(cudaMalloc((void **)&c->stk_xn, (size_t)T * L->d * sizeof(float)));
    CK(cudaMalloc((void **)&c->stk_y, (size_t)T * L->d * sizeof(float)));
    CK(cudaMallocHost((void **)&c->x_pin, (size_t)T * L->d * sizeof(float)));
    CK(cudaMallocHost((void **)&c->idx_pin, (size_t)T * L->k * sizeof(int32_t)));
    CK(cudaMallocHost((void **)&c->wave_pin, (size_t)L->E + 1));
    if (c->ep_world > 1) {
        /* the experts pass holds the own T tokens and at most T tokens from
         * every rank */
        char msg[256] = {0};
        c->prefill = qk_prefill_create(L, T * (c->ep_world + 1), c->pool, c->nslots + Lz,
                                       c->num_sms, msg, sizeof(msg));
        if (!c->prefill) {
            seterr(err, "qmoe_create: expert parallelism needs the grouped path: %s", msg);
            goto fail;
        }
        CK((cudaError_t)qk_ep_alloc(c->prefill, T, c->ep_world));
        if (!c->resident_all)
            CK(cudaMallocHost((void **)&c->ep_recv_pin,
                              (size_t)c->ep_world * T * L->k * sizeof(int32_t)));
    } else if (T > 1) {
        char msg[256] = {0};
        c->prefill = qk_prefill_create(L, T, c->pool, c->nslots + Lz, c->num_sms, msg, sizeof(msg));
        /* NULL: shape outside the grouped-GEMM kernels; the per-token path runs */
    }
    return c;
fail:
    qmoe_destroy(c);
    return NULL;
}

/* ------------------------------------------------------------- pool fills */

static uint64_t ekey(int layer, int e) { return ((uint64_t)(uint32_t)layer << 32) | (uint32_t)e; }

/* A local expert's slot in the pinned host store (streaming contexts). */
static uint8_t *store_slot(const qmoe_ctx *c, int layer, int e) {
    const size_t el = (size_t)(c->ep_hi - c->ep_lo);
    return c->host_store + ((size_t)layer * el + (size_t)(e - c->ep_lo)) * c->L.slot_bytes;
}

/* Assigns a slot to (layer, e) in the bookkeeping; evicted owners lose their
 * table entries. Returns the slot or -1 when the cache rejects the entry (all
 * candidates pinned). Caller holds c->lock. */
static int claim_slot(qmoe_ctx *c, int layer, int e, int pin) {
    uint64_t key = ekey(layer, e);
    uint64_t ev[64];
    size_t nev = 0;
    int slot = c->nfree > 0 ? c->free_slots[c->nfree - 1] : -1;
    /* an expert routed at least four times enters hot (streaming.py:396-397) */
    const int hot = qmoe_predictor_count(c->pred, layer, e) >= 4;
    const int ok = qmoe_cache_put(c->cache, key, slot >= 0 ? (uint64_t)slot : NO_OWNER,
                                  c->L.slot_bytes, pin, hot, ev, 64, &nev);
    if (ok && slot >= 0) c->nfree--;
    /* victims leave the pool even when the put is then rejected (the cache
     * does not restore them, as cache.c:236-242): their slots are free */
    for (size_t i = 0; i < nev && i < 64; i++) {
        if (ev[i] == NO_OWNER) continue;
        int s = (int)ev[i];
        uint64_t owner = c->slot_owner[s];
        if (owner != NO_OWNER) {
            const size_t m = (size_t)(owner >> 32) * (size_t)c->L.E + (uint32_t)owner;
            c->slot_of_host[m] = -1;
            c->slot_owner[s] = NO_OWNER;
            if (c->pf_mark[m]) { /* prefetched, never routed to */
                c->pf_mark[m] = 0;
                c->pf_outstanding--;
                c->stats.prefetch_wasted++;
            }
        }
        c->free_slots[c->nfree++] = s;
    }
    if (!ok) return -1;
    if (slot < 0) {
        if (c->nfree == 0) {
            uint64_t dummy;
            qmoe_cache_erase(c->cache, key, &dummy);
            return -1;
        }
        slot = c->free_slots[--c->nfree];
        qmoe__cache_set_value(c->cache, key, (uint64_t)slot);
    }
    c->slot_owner[slot] = key;
    c->slot_of_host[(size_t)layer * c->L.E + e] = slot;
    return slot;
}

/* Fill of the uncached experts in ids (experts_load semantics: present
 * entries are skipped without touching their stats). While the call runs,
 * every listed expert is pinned so that filling one cannot evict another the
 * same call needs; pins the call added are dropped at the end.
 *   st == NULL  synchronous: the host waits for the copies; the caller makes
 *               sure no queued kernel still reads a slot that may be evicted
 *               (the compute stream is idle).
 *   st != NULL  asynchronous: the copy stream first waits for everything
 *               already queued on st (a victim slot may still be read there),
 *               then copies; nothing waits on the host. The copies complete
 *               before whatever the caller queues on st after a later
 *               mark_fills_ready(c, st). */
static int fill_experts(qmoe_ctx *c, int layer, const int64_t *ids, size_t n, cudaStream_t st,
                        qmoe_err *err) {
    const qk_layout *L = &c->L;
    double t0 = now_s();
    int loaded = 0, rc = 0;
    if (n > (size_t)c->nslots) {
        seterr(err, "qmoe_experts_load: %zu experts requested, the pool has %d slots", n,
               c->nslots);
        return -1;
    }
    unsigned char *ours = calloc(n ? n : 1, 1);
    if (!ours) {
        seterr(err, "qmoe_experts_load: out of host memory");
        return -1;
    }
    if (st) {
        cudaError_t ce = cudaEventRecord(c->compute_mark, st);
        if (ce == cudaSuccess) ce = cudaStreamWaitEvent(c->copy_stream, c->compute_mark, 0);
        if (ce != cudaSuccess) {
            free(ours);
            seterr(err, "qmoe_experts_load: %s", cudaGetErrorString(ce));
            return -1;
        }
    }
    pthread_mutex_lock(&c->lock);
    for (size_t i = 0; i < n; i++) {
        int e = (int)ids[i];
        if (e < 0 || e >= L->E) {
            seterr(err, "qmoe_experts_load: expert %lld out of range", (long long)ids[i]);
            rc = -1;
            break;
        }
        if (e < c->ep_lo || e >= c->ep_hi) {
            seterr(err, "qmoe_experts_load: expert %d is not one of this rank's [%d, %d)", e,
                   c->ep_lo, c->ep_hi);
            rc = -1;
            break;
        }
        if (qmoe_cache_peek(c->cache, ekey(layer, e), NULL)) {
            ours[i] = (unsigned char)qmoe_cache_pin(c->cache, ekey(layer, e));
            continue;
        }
        if (!c->host_store) {
            seterr(err, "qmoe_experts_load: expert %d of layer %d was never uploaded", e, layer);
            rc = -1;
            break;
        }
        int slot = claim_slot(c, layer, e, 1);
        if (slot < 0) {
            seterr(err, "qmoe_experts_load: pool full of pinned experts (layer %d expert %d)",
                   layer, e);
            rc = -1;
            break;
        }
        ours[i] = 1;
        const uint8_t *src = store_slot(c, layer, e);
        cudaError_t ce = cudaMemcpyAsync(c->pool + (size_t)slot * L->slot_bytes, src,
                                         L->slot_bytes, cudaMemcpyHostToDevice, c->copy_stream);
        if (ce != cudaSuccess) {
            seterr(err, "qmoe_experts_load: %s", cudaGetErrorString(ce));
            rc = -1;
            break;
        }
        loaded++;
    }
    for (size_t i = 0; i < n; i++)
        if (ours[i]) qmoe_cache_unpin(c->cache, ekey(layer, (int)ids[i]));
    free(ours);
    /* the layer's slot table (from pageable memory: staged by the call, so
     * the host may change it again at once) */
    cudaError_t ce = cudaSuccess;
    if (loaded || !st)
        ce = cudaMemcpyAsync(c->slot_of_dev + (size_t)layer * L->E, c->slot_of_host + (size_t)layer * L->E,
                             (size_t)L->E * sizeof(int32_t), cudaMemcpyHostToDevice, c->copy_stream);
    if (ce == cudaSuccess && !st) ce = cudaStreamSynchronize(c->copy_stream);
    pthread_mutex_unlock(&c->lock);
    if (rc) return rc;
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_experts_load: %s", cudaGetErrorString(ce));
        return -1;
    }
    c->stats.expert_loads += (uint64_t)loaded;
    c->stats.expert_bytes += (uint64_t)loaded * L->slot_bytes;
    c->stats.expert_wait_seconds += now_s() - t0;
    return 0;
}

/* Whatever the caller queues on st after this waits for every copy queued
 * so far on the copy stream (the layer's fills and earlier prefetches). */
static int mark_fills_ready(qmoe_ctx *c, cudaStream_t st, qmoe_err *err) {
    cudaError_t ce = cudaEventRecord(c->copy_done, c->copy_stream);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(st, c->copy_done, 0);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

/* ----------------------------------------------------------------- upload */

/* Largest 2-norm of a router row (bf16), in fp64, rounded up to fp32 with a
 * margin: the error bound of the tensor-core routing scales with it. */
static float router_wmax(const uint16_t *router, int E, int d) {
    double best = 0.0;
    for (int e = 0; e < E; e++) {
        double ss = 0.0;
        for (int i = 0; i < d; i++) {
            uint32_t b = (uint32_t)router[(size_t)e * d + i] << 16;
            float f;
            memcpy(&f, &b, 4);
            ss += (double)f * (double)f;
        }
        if (ss > best) best = ss;
    }
    float r = (float)(sqrt(best) * (1.0 + 1e-6));
    return isfinite(r) ? nextafterf(r, INFINITY) : INFINITY;
}

static int upload_shared(qmoe_ctx *c, layer_dev *ld, const qmoe_layer_weights *w, qmoe_err *err) {
    const qk_layout *L = &c->L;
    uint8_t *buf = malloc(L->slot_bytes);
    if (!buf) {
        seterr(err, "qmoe_upload_layer: out of host memory");
        return -1;
    }
    qk_pack_expert(L, w->sh_gate.q, w->sh_gate.scales, w->sh_gate.biases, w->sh_up.q,
                   w->sh_up.scales, w->sh_up.biases, w->sh_down.q, w->sh_down.scales,
                   w->sh_down.biases, buf);
    cudaError_t ce = cudaMemcpy(ld->shared_slot, buf, L->slot_bytes, cudaMemcpyHostToDevice);
    free(buf);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_upload_layer: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

int qmoe_upload_layer(qmoe_ctx *c, int layer, const qmoe_layer_weights *w, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !w || layer < 0 || layer >= c->cfg.num_layers) {
        seterr(err, "qmoe_upload_layer: bad arguments (layer %d)", layer);
        return -1;
    }
    const qmoe_q4 *ts[6] = {&w->gate, &w->up, &w->down, &w->sh_gate, &w->sh_up, &w->sh_down};
    for (int i = 0; i < 6; i++)
        if (!ts[i]->q || !ts[i]->scales || !ts[i]->biases) {
            seterr(err, "qmoe_upload_layer: missing q4 tensor %d", i);
            return -1;
        }
    if (!w->router || !w->shared_gate) {
        seterr(err, "qmoe_upload_layer: missing router or shared gate");
        return -1;
    }
    const qk_layout *L = &c->L;
    layer_dev *ld = &c->layers[layer];
    uint8_t *stage = NULL;
    if (ld->tok_graph) { /* it holds this layer's old pointers */
        cudaGraphExecDestroy(ld->tok_graph);
        ld->tok_graph = NULL;
    }
    const int batch = 16;
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaStreamSynchronize(c->stream));
    if (!ld->router) CK(cudaMalloc((void **)&ld->router, (size_t)L->E * L->d * 2));
    if (!ld->shgate) CK(cudaMalloc((void **)&ld->shgate, (size_t)L->d * 2));
    CK(cudaMemcpy(ld->router, w->router, (size_t)L->E * L->d * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ld->shgate, w->shared_gate, (size_t)L->d * 2, cudaMemcpyHostToDevice));
    if (w->logit_bias) {
        if (!ld->bias) CK(cudaMalloc((void **)&ld->bias, (size_t)L->E * sizeof(float)));
        CK(cudaMemcpy(ld->bias, w->logit_bias, (size_t)L->E * sizeof(float), cudaMemcpyHostToDevice));
    } else if (ld->bias) {
        cudaFree(ld->bias);
        ld->bias = NULL;
    }
    if (upload_shared(c, ld, w, err)) return -1;
    ld->router_wmax = router_wmax(w->router, L->E, L->d);
    if (c->resident_all) {
        CK(cudaMallocHost((void **)&stage, (size_t)batch * L->slot_bytes));
        for (int e0 = c->ep_lo; e0 < c->ep_hi; e0 += batch) {
            int nb = c->ep_hi - e0 < batch ? c->ep_hi - e0 : batch;
            CK(cudaStreamSynchronize(c->copy_stream));
            for (int i = 0; i < nb; i++) pack_routed(c, w, e0 + i, stage + (size_t)i * L->slot_bytes);
            pthread_mutex_lock(&c->lock);
            int first = -1, contiguous = 1;
            for (int i = 0; i < nb; i++) {
                int e = e0 + i;
                int slot = c->slot_of_host[(size_t)layer * L->E + e];
                if (slot < 0) slot = claim_slot(c, layer, e, 0);
                if (i == 0) first = slot;
                else if (slot != first + i) contiguous = 0;
                if (slot < 0) contiguous = -1;
            }
            pthread_mutex_unlock(&c->lock);
            if (contiguous < 0) {
                seterr(err, "qmoe_upload_layer: pool bookkeeping failed");
                goto fail;
            }
            if (contiguous) {
                CK(cudaMemcpyAsync(c->pool + (size_t)first * L->slot_bytes, stage,
                                   (size_t)nb * L->slot_bytes, cudaMemcpyHostToDevice, c->copy_stream));
            } else {
                for (int i = 0; i < nb; i++) {
                    int slot = c->slot_of_host[(size_t)layer * L->E + e0 + i];
                    CK(cudaMemcpyAsync(c->pool + (size_t)slot * L->slot_bytes,
                                       stage + (size_t)i * L->slot_bytes, L->slot_bytes,
                                       cudaMemcpyHostToDevice, c->copy_stream));
                }
            }
        }
        CK(cudaStreamSynchronize(c->copy_stream));
        CK(cudaMemcpy(c->slot_of_dev + (size_t)layer * L->E, c->slot_of_host + (size_t)layer * L->E,
                      (size_t)L->E * sizeof(int32_t), cudaMemcpyHostToDevice));
        cudaFreeHost(stage);
        stage = NULL;
    } else {
        /* streaming: experts stay in the pinned host store; drop stale slots */
        pthread_mutex_lock(&c->lock);
        for (int e = 0; e < L->E; e++) {
            uint64_t v;
            if (qmoe_cache_erase(c->cache, ekey(layer, e), &v) && v != NO_OWNER) {
                c->slot_owner[v] = NO_OWNER;
                c->free_slots[c->nfree++] = (int)v;
            }
            c->slot_of_host[(size_t)layer * L->E + e] = -1;
            if (e >= c->ep_lo && e < c->ep_hi) pack_routed(c, w, e, store_slot(c, layer, e));
        }
        pthread_mutex_unlock(&c->lock);
        CK(cudaMemcpy(c->slot_of_dev + (size_t)layer * L->E, c->slot_of_host + (size_t)layer * L->E,
                      (size_t)L->E * sizeof(int32_t), cudaMemcpyHostToDevice));
    }
    ld->ready = 1;
    return 0;
fail:
    if (stage) cudaFreeHost(stage);
    return -1;
}

/* The seeded synthetic layer of qmoe_synth_layer, generated on the device:
 * the local experts straight into the pool (resident contexts) or, through a
 * device staging buffer, into the pinned host store (streaming contexts,
 * whose cached copies of the layer are dropped); the shared slot, the
 * router and the shared gate on the device; the Zipf bias (zipf_s > 0) made
 * on the host. */
int qmoe_synth_layer_dev(qmoe_ctx *c, int layer, uint64_t seed, double zipf_s, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || layer < 0 || layer >= c->cfg.num_layers) {
        seterr(err, "qmoe_synth_layer_dev: bad arguments (layer %d)", layer);
        return -1;
    }
    const qk_layout *L = &c->L;
    layer_dev *ld = &c->layers[layer];
    cudaStream_t st = c->copy_stream;
    uint16_t *router_host = NULL;
    float *bias_host = NULL;
    uint8_t *stage = NULL;            /* streaming: device staging slots */
    const int stage_slots = 32;
    const uint64_t Ly = (uint64_t)layer;
    const uint64_t rk[6] = {qk_stream_key(seed, Ly, QK_T_GQ), qk_stream_key(seed, Ly, QK_T_GS),
                            qk_stream_key(seed, Ly, QK_T_UQ), qk_stream_key(seed, Ly, QK_T_US),
                            qk_stream_key(seed, Ly, QK_T_DQ), qk_stream_key(seed, Ly, QK_T_DS)};
    const uint64_t sk[6] = {qk_stream_key(seed, Ly, QK_T_SGQ), qk_stream_key(seed, Ly, QK_T_SGS),
                            qk_stream_key(seed, Ly, QK_T_SUQ), qk_stream_key(seed, Ly, QK_T_SUS),
                            qk_stream_key(seed, Ly, QK_T_SDQ), qk_stream_key(seed, Ly, QK_T_SDS)};
    if (ld->tok_graph) { /* it holds this layer's old pointers */
        cudaGraphExecDestroy(ld->tok_graph);
        ld->tok_graph = NULL;
    }
    ld->ready = 0;
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaStreamSynchronize(c->stream));
    if (!ld->router) CK(cudaMalloc((void **)&ld->router, (size_t)L->E * L->d * 2));
    if (!ld->shgate) CK(cudaMalloc((void **)&ld->shgate, (size_t)L->d * 2));
    CK((cudaError_t)qk_synth_bf16_normal(ld->router, (size_t)L->E * L->d,
                                         qk_stream_key(seed, Ly, QK_T_ROUTER), st));
    CK((cudaError_t)qk_synth_bf16_normal(ld->shgate, (size_t)L->d,
                                         qk_stream_key(seed, Ly, QK_T_SHGATE), st));
    CK((cudaError_t)qk_synth_slot(L, ld->shared_slot, 0, sk, st));
    if (c->resident_all) {
        for (int e = c->ep_lo; e < c->ep_hi; e++) {
            pthread_mutex_lock(&c->lock);
            int slot = c->slot_of_host[(size_t)layer * L->E + e];
            if (slot < 0) slot = claim_slot(c, layer, e, 0);
            pthread_mutex_unlock(&c->lock);
            if (slot < 0) {
                seterr(err, "qmoe_synth_layer_dev: pool bookkeeping failed");
                goto fail;
            }
            CK((cudaError_t)qk_synth_slot(L, c->pool + (size_t)slot * L->slot_bytes, e, rk, st));
        }
    } else {
        /* streaming: the layer's cached copies are stale */
        pthread_mutex_lock(&c->lock);
        for (int e = 0; e < L->E; e++) {
            uint64_t v;
            if (qmoe_cache_erase(c->cache, ekey(layer, e), &v) && v != NO_OWNER) {
                c->slot_owner[v] = NO_OWNER;
                c->free_slots[c->nfree++] = (int)v;
            }
            c->slot_of_host[(size_t)layer * L->E + e] = -1;
        }
        pthread_mutex_unlock(&c->lock);
        CK(cudaMalloc((void **)&stage, (size_t)stage_slots * L->slot_bytes));
        for (int e0 = c->ep_lo; e0 < c->ep_hi; e0 += stage_slots) {
            const int nb = c->ep_hi - e0 < stage_slots ? c->ep_hi - e0 : stage_slots;
            for (int i = 0; i < nb; i++)
                CK((cudaError_t)qk_synth_slot(L, stage + (size_t)i * L->slot_bytes, e0 + i, rk, st));
            CK(cudaMemcpyAsync(store_slot(c, layer, e0), stage, (size_t)nb * L->slot_bytes,
                               cudaMemcpyDeviceToHost, st));
            CK(cudaStreamSynchronize(st));
        }
        cudaFree(stage);
        stage = NULL;
    }
    if (zipf_s > 0) {
        bias_host = malloc((size_t)L->E * sizeof(float));
        if (!bias_host) {
            seterr(err, "qmoe_synth_layer_dev: out of host memory");
            goto fail;
        }
        qmoe_synth_zipf_bias(seed, layer, L->E, zipf_s, bias_host);
        if (!ld->bias) CK(cudaMalloc((void **)&ld->bias, (size_t)L->E * sizeof(float)));
        CK(cudaMemcpy(ld->bias, bias_host, (size_t)L->E * sizeof(float), cudaMemcpyHostToDevice));
    } else if (ld->bias) {
        cudaFree(ld->bias);
        ld->bias = NULL;
    }
    router_host = malloc((size_t)L->E * L->d * 2);
    if (!router_host) {
        seterr(err, "qmoe_synth_layer_dev: out of host memory");
        goto fail;
    }
    CK(cudaMemcpyAsync(router_host, ld->router, (size_t)L->E * L->d * 2, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    ld->router_wmax = router_wmax(router_host, L->E, L->d);
    CK(cudaMemcpy(c->slot_of_dev + (size_t)layer * L->E, c->slot_of_host + (size_t)layer * L->E,
                  (size_t)L->E * sizeof(int32_t), cudaMemcpyHostToDevice));
    free(router_host);
    free(bias_host);
    ld->ready = 1;
    return 0;
fail:
    if (stage) cudaFree(stage);
    free(router_host);
    free(bias_host);
    return -1;
}

/* ---------------------------------------------------------------- forward */

static void fill_fwd(qmoe_ctx *c, int layer, const void *x, int x_bf16, int n, float *out,
                     qk_fwd *f) {
    layer_dev *ld = &c->layers[layer];
    memset(f, 0, sizeof(*f));
    f->L = c->L;
    f->T = n;
    f->x = x;
    f->x_bf16 = x_bf16;
    f->router = ld->router;
    f->shared_gate = ld->shgate;
    f->logit_bias = ld->bias;
    f->pool = c->pool;
    f->slot_of = c->slot_of_dev + (size_t)layer * c->L.E;
    f->shared_slot = ld->shared_slot;
    f->logits = c->logits;
    f->idx = c->idx;
    f->wts = c->wts;
    f->sgate = c->sgate;
    f->h = c->h;
    f->out = out;
    f->err = c->err_dev;
    f->num_sms = c->num_sms;
}

static int kerr(int rc, const char *what, qmoe_err *err) {
    if (rc != 0) {
        seterr(err, "%s launch failed: %s", what, cudaGetErrorString((cudaError_t)rc));
        return -1;
    }
    return 0;
}

/* Routing (idx, wts, sgate) of f->T tokens: the tensor-core path with exact
 * re-ranking for multi-token calls when the plan covers the shape, else the
 * fp64 router and the one-warp top-k. mid: NULL or an event recorded
 * between the two kernels of either path. */
static int route(qmoe_ctx *c, int layer, qk_fwd *f, cudaStream_t st, int pdl, cudaEvent_t mid,
                 qmoe_err *err) {
    if (c->prefill && f->T > 1) {
        int rc = qk_launch_route(c->prefill, f, c->layers[layer].router_wmax, st, mid);
        if (rc != QK_ROUTE_UNFIT) return kerr(rc, "route", err);
    }
    if (kerr(qk_launch_router(f, st, pdl), "router", err)) return -1;
    if (mid) cudaEventRecordWithFlags(mid, st, cudaEventRecordExternal);
    return kerr(qk_launch_topk(f, st, pdl), "topk", err);
}

/* streaming mode: route first, make the selected experts resident. When the
 * call routes to more distinct experts than the pool has slots, nothing is
 * filled: *over receives the distinct experts (first-appearance order, the
 * caller frees it) and *n_over their count, for a pass in waves. */
static int stream_in(qmoe_ctx *c, int layer, qk_fwd *f, cudaStream_t st, int64_t **over,
                     size_t *n_over, qmoe_err *err) {
    *over = NULL;
    *n_over = 0;
    int n = f->T, k = c->L.k;
    if (route(c, layer, f, st, 0, NULL, err)) return -1;
    cudaError_t ce = cudaMemcpyAsync(c->idx_pin, c->idx, (size_t)n * k * sizeof(int32_t),
                                     cudaMemcpyDeviceToHost, st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
        return -1;
    }
    int64_t *uniq = calloc((size_t)n * k, sizeof(int64_t));
    unsigned char *seen = calloc((size_t)c->L.E, 1);
    if (!uniq || !seen) {
        free(uniq);
        free(seen);
        seterr(err, "qmoe_forward: out of host memory");
        return -1;
    }
    size_t nu = 0;
    for (int i = 0; i < n * k; i++) {
        int e = c->idx_pin[i];
        if (e >= 0 && e < c->L.E && !seen[e]) {
            seen[e] = 1;
            uniq[nu++] = e;
            const int resident = qmoe_cache_peek(c->cache, ekey(layer, e), NULL);
            c->stats.routed_lookups++;
            c->stats.routed_hits += (uint64_t)resident;
            /* a prefetched expert routed to while still in the pool */
            unsigned char *pm = c->pf_mark + (size_t)layer * c->L.E + e;
            if (*pm) {
                if (resident) c->stats.prefetch_hits++;
                *pm = 0;
                c->pf_outstanding--;
            }
        }
    }
    free(seen);
    if (nu > (size_t)c->nslots) {
        *over = uniq;
        *n_over = nu;
        return 0;
    }
    /* the misses are copied behind the routing on the copy stream; the
     * layer's kernels, queued next on st, wait for them (and for any
     * prefetch still in flight) */
    int rc = fill_experts(c, layer, uniq, nu, st, err);
    if (rc == 0) rc = mark_fills_ready(c, st, err);
    if (rc == 0) {
        pthread_mutex_lock(&c->lock);
        for (size_t i = 0; i < nu; i++) qmoe_cache_get(c->cache, ekey(layer, (int)uniq[i]), NULL);
        pthread_mutex_unlock(&c->lock);
    }
    free(uniq);
    return rc;
}

/* A streaming call whose distinct experts exceed the pool (the reference
 * reloads evicted experts inside its expert loop, model.c:1341-1349): rows
 * grouped once, then the experts in waves of at most the pool's slots, each
 * wave filled and run through the grouped GEMMs over its own tiles, then one
 * combine. Each output row is computed by exactly one wave and combined in
 * the one-pass order, so the result equals a pool that holds them all. */
static int forward_waves(qmoe_ctx *c, int layer, qk_fwd *f, cudaStream_t st, const int64_t *ids,
                         size_t nu, qmoe_err *err) {
    if (!c->prefill || f->T < 2) {
        seterr(err, "qmoe_forward: %zu distinct experts routed, the pool has %d slots (a "
                    "single-token call needs them at once)", nu, c->nslots);
        return -1;
    }
    const int E = c->L.E, shared = c->nslots + layer;
    if (kerr(qk_prefill_plan(c->prefill, f, shared, st), "prefill plan", err)) return -1;
    uint8_t *mask_dev = qk_prefill_wave_mask(c->prefill);
    for (size_t w0 = 0; w0 < nu; w0 += (size_t)c->nslots) {
        const size_t nw = nu - w0 < (size_t)c->nslots ? nu - w0 : (size_t)c->nslots;
        /* the previous wave's GEMMs read slots this wave's fills may evict,
         * and its mask copy reads wave_pin */
        cudaError_t ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
            return -1;
        }
        if (fill_experts(c, layer, ids + w0, nw, NULL, err)) return -1;
        pthread_mutex_lock(&c->lock);
        for (size_t i = 0; i < nw; i++) qmoe_cache_get(c->cache, ekey(layer, (int)ids[w0 + i]), NULL);
        pthread_mutex_unlock(&c->lock);
        memset(c->wave_pin, 0, (size_t)E + 1);
        c->wave_pin[0] = w0 == 0; /* the shared expert runs with the first wave */
        for (size_t i = 0; i < nw; i++) c->wave_pin[ids[w0 + i] + 1] = 1;
        ce = cudaMemcpyAsync(mask_dev, c->wave_pin, (size_t)E + 1, cudaMemcpyHostToDevice, st);
        if (ce != cudaSuccess) {
            seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
            return -1;
        }
        if (kerr(qk_prefill_wave(c->prefill, f, shared, st), "prefill wave", err)) return -1;
        c->stats.expert_waves++;
    }
    return kerr(qk_prefill_combine(c->prefill, f, st), "combine", err);
}

int qmoe_forward_dev(qmoe_ctx *c, int layer, const void *x, int x_dtype, int n, float *out,
                     void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !x || !out || layer < 0 || layer >= c->cfg.num_layers) {
        seterr(err, "qmoe_forward: bad arguments (layer %d)", layer);
        return -1;
    }
    if (!c->layers[layer].ready) {
        seterr(err, "qmoe_forward: layer %d was not uploaded", layer);
        return -1;
    }
    if (n < 0 || n > c->cfg.max_tokens) {
        seterr(err, "qmoe_forward: n=%d outside [0, max_tokens=%d]", n, c->cfg.max_tokens);
        return -1;
    }
    if (x_dtype != QMOE_F32 && x_dtype != QMOE_BF16) {
        seterr(err, "qmoe_forward: unknown x dtype %d", x_dtype);
        return -1;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (n == 0) return 0;
    qk_fwd f;
    fill_fwd(c, layer, x, x_dtype == QMOE_BF16, n, out, &f);
    c->last_T = n;
    if (n == 1) c->stats.decode_calls++;
    else c->stats.prefill_calls++;
    /* profiling (inside a capture): external event records between kernels,
     * so they are real timestamps in the graph; no programmatic overlap */
    const int prof = c->profile;
#define PEV(i) \
    if (prof) cudaEventRecordWithFlags(c->pev[i], st, cudaEventRecordExternal)
    if (c->resident_all && n == 1) {
        /* one persistent launch for the whole layer */
        PEV(0);
        int rc = qk_launch_decode_fused(&f, c->dsync, st, !prof);
        if (rc == 0) {
            PEV(1);
            c->prof_kernels = 1;
            return 0;
        }
        if (rc != QK_FUSED_UNFIT) return kerr(rc, "decode_fused", err);
    }
    c->prof_kernels = 4;
    if (!c->resident_all) {
        int64_t *over = NULL;
        size_t n_over = 0;
        if (stream_in(c, layer, &f, st, &over, &n_over, err)) return -1;
        if (over) {
            const int rc = forward_waves(c, layer, &f, st, over, n_over, err);
            free(over);
            c->prof_kernels = 6;
            return rc;
        }
    } else {
        PEV(0);
        if (route(c, layer, &f, st, !prof, prof ? c->pev[1] : NULL, err)) return -1;
        PEV(2);
    }
    if (c->prefill && n > 1) {
        /* grouped tcgen05 path: grouping + gather, gate/up, down, combine */
        void *ev[4] = {c->pev[3], c->pev[4], c->pev[5], c->pev[6]};
        int rc = qk_launch_prefill(c->prefill, &f, c->nslots + layer, st, prof ? ev : NULL);
        if (rc) return kerr(rc, "prefill", err);
        c->prof_kernels = 6;
        return 0;
    }
    if (kerr(qk_launch_decode_gateup(&f, st, !prof), "decode_gateup", err)) return -1;
    PEV(3);
    if (kerr(qk_launch_decode_down(&f, st, !prof), "decode_down", err)) return -1;
    PEV(4);
#undef PEV
    return 0;
}

/* ------------------------------------------------------------- graphs */

struct qmoe_graph {
    cudaGraphExec_t exec;
    cudaStream_t stream;
};

int qmoe_capture_begin(qmoe_ctx *c, void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !c->resident_all) {
        seterr(err, "qmoe_capture_begin: needs a context with every expert resident");
        return -1;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    cudaError_t ce = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_capture_begin: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

qmoe_graph *qmoe_capture_end(qmoe_ctx *c, void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c) return NULL;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    cudaGraph_t g = NULL;
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_capture_end: %s", cudaGetErrorString(ce));
        return NULL;
    }
    qmoe_graph *q = calloc(1, sizeof(*q));
    if (!q) {
        cudaGraphDestroy(g);
        seterr(err, "qmoe_capture_end: out of host memory");
        return NULL;
    }
    ce = cudaGraphInstantiate(&q->exec, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) {
        free(q);
        seterr(err, "qmoe_capture_end: instantiate: %s", cudaGetErrorString(ce));
        return NULL;
    }
    q->stream = st;
    return q;
}

int qmoe_graph_launch(qmoe_graph *g, void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!g) return -1;
    cudaError_t ce = cudaGraphLaunch(g->exec, stream ? (cudaStream_t)stream : g->stream);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_graph_launch: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

void qmoe_graph_free(qmoe_graph *g) {
    if (!g) return;
    cudaGraphExecDestroy(g->exec);
    free(g);
}

/* Diagnostics (not in the public header): one single-token forward through the
 * single-launch kernel with per-CTA phase timestamps; out_ns receives
 * [grid][16] %globaltimer values. Returns the grid size, or -1. */
/* Diagnostics (not in the public header): n_tokens single-token qmoe_forward
 * calls made from C, token t from x + t d into out + t d, as the reference's
 * C caller makes them (one moe_forward per token). */
int qmoe__forward_tokens(qmoe_ctx *c, int layer, const float *x, int n_tokens, float *out,
                         qmoe_err *err) {
    if (!c || n_tokens < 0) return -1;
    const size_t d = (size_t)c->L.d;
    for (int t = 0; t < n_tokens; t++)
        if (qmoe_forward(c, layer, x + (size_t)t * d, 1, out + (size_t)t * d, err)) return -1;
    return 0;
}

int qmoe__phase_times(qmoe_ctx *c, int layer, const void *x, int x_dtype, float *out,
                      unsigned long long *out_ns, int max_ctas) {
    if (!c || !c->resident_all || !c->layers[layer].ready) return -1;
    unsigned long long *buf = NULL;
    size_t bytes = (size_t)c->num_sms * 32 * sizeof(unsigned long long);
    if (cudaMalloc((void **)&buf, bytes) != cudaSuccess) return -1;
    cudaMemset(buf, 0, bytes);
    qk_fwd f;
    fill_fwd(c, layer, x, x_dtype == QMOE_BF16, 1, out, &f);
    f.ptimes = buf;
    int rc = qk_launch_decode_fused(&f, c->dsync, c->stream, 0);
    if (rc == 0) rc = cudaStreamSynchronize(c->stream);
    if (rc == 0) {
        int n = max_ctas < c->num_sms ? max_ctas : c->num_sms;
        rc = cudaMemcpy(out_ns, buf, (size_t)n * 32 * sizeof(unsigned long long),
                        cudaMemcpyDeviceToHost);
    }
    cudaFree(buf);
    return rc == 0 ? c->num_sms : -1;
}

/* Diagnostics (not in the public header): n_tokens single-token launches of
 * the single-launch kernel back to back on the context's stream with
 * programmatic dependent launch, as a captured decode step runs them, token t
 * from x + t d (x_dtype) into out + t d, each with per-CTA phase timestamps:
 * out_ns receives [n_tokens][max_ctas][32] values. Returns the grid size, or
 * -1. */
int qmoe__phase_times_seq(qmoe_ctx *c, int layer, const void *x, int x_dtype, float *out,
                          int n_tokens, unsigned long long *out_ns, int max_ctas) {
    if (!c || !c->resident_all || !c->layers[layer].ready || n_tokens < 1) return -1;
    const size_t per = (size_t)c->num_sms * 32;
    unsigned long long *buf = NULL;
    if (cudaMalloc((void **)&buf, per * n_tokens * sizeof(unsigned long long)) != cudaSuccess)
        return -1;
    int rc = cudaMemset(buf, 0, per * n_tokens * sizeof(unsigned long long));
    const size_t xb = (size_t)c->L.d * (x_dtype == QMOE_BF16 ? 2 : 4);
    for (int t = 0; rc == 0 && t < n_tokens; t++) {
        qk_fwd f;
        fill_fwd(c, layer, (const char *)x + t * xb, x_dtype == QMOE_BF16, 1,
                 out + (size_t)t * c->L.d, &f);
        f.ptimes = buf + per * t;
        rc = qk_launch_decode_fused(&f, c->dsync, c->stream, t > 0);
    }
    if (rc == 0) rc = cudaStreamSynchronize(c->stream);
    const int n = max_ctas < c->num_sms ? max_ctas : c->num_sms;
    for (int t = 0; rc == 0 && t < n_tokens; t++)
        rc = cudaMemcpy(out_ns + (size_t)t * max_ctas * 32, buf + per * t,
                        (size_t)n * 32 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(buf);
    return rc == 0 ? c->num_sms : -1;
}

int qmoe_profile_forward(qmoe_ctx *c, int layer, const void *x, int x_dtype, int n, float *out,
                         int reps, double *kernel_us, int max_kernels, int *kernels,
                         qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || reps < 1 || !kernel_us) {
        seterr(err, "qmoe_profile_forward: bad arguments");
        return -1;
    }
    if (qmoe_capture_begin(c, NULL, err)) return -1;
    c->profile = 1;
    int rc = qmoe_forward_dev(c, layer, x, x_dtype, n, out, NULL, err);
    c->profile = 0;
    qmoe_graph *g = qmoe_capture_end(c, NULL, rc ? NULL : err);
    if (rc || !g) {
        qmoe_graph_free(g);
        return -1;
    }
    const int nk = c->prof_kernels;
    double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < reps; r++) {
        if (qmoe_graph_launch(g, NULL, err)) {
            qmoe_graph_free(g);
            return -1;
        }
        cudaError_t ce = cudaStreamSynchronize(c->stream);
        if (ce != cudaSuccess) {
            qmoe_graph_free(g);
            seterr(err, "qmoe_profile_forward: %s", cudaGetErrorString(ce));
            return -1;
        }
        for (int i = 0; i < nk; i++) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, c->pev[i], c->pev[i + 1]);
            acc[i] += ms;
        }
    }
    qmoe_graph_free(g);
    for (int i = 0; i < max_kernels && i < nk && i < 8; i++) kernel_us[i] = 1e3 * acc[i] / reps;
    if (kernels) *kernels = nk;
    return check_dev_err(c, c->stream, err);
}

static int check_dev_err(qmoe_ctx *c, cudaStream_t st, qmoe_err *err) {
    cudaError_t ce = cudaMemcpyAsync(c->err_host, c->err_dev, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe: CUDA error: %s", cudaGetErrorString(ce));
        return -1;
    }
    return report_dev_err(c, *c->err_host, st, err);
}

/* code: the error word as read back (0: no error). On an error, clears the
 * word and the decode kernel's barrier and exchange area. */
static int report_dev_err(qmoe_ctx *c, int code, cudaStream_t st, qmoe_err *err) {
    if (code) {
        /* clear the sticky word and the decode kernel's counter and exchange
         * area (a launch that gave up may have left its barrier unfinished) */
        cudaMemsetAsync(c->err_dev, 0, sizeof(int), st);
        cudaMemsetAsync(c->dsync, 0, qk_decode_sync_bytes(&c->L), st);
        cudaStreamSynchronize(st);
        seterr(err, "qmoe: device reported error 0x%x (%s%s%s%s)", code,
               code & QK_ERR_TIMEOUT_COPY ? "copy wait timed out; " : "",
               code & QK_ERR_NOT_RESIDENT ? "routed expert not resident; " : "",
               code & QK_ERR_BAD_ROUTE ? "top-k selection failed; " : "",
               code & QK_ERR_TIMEOUT_GRID ? "grid barrier or exchange timed out" : "");
        return -1;
    }
    return 0;
}

int qmoe_sync(qmoe_ctx *c, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c) return -1;
    return check_dev_err(c, c->stream, err);
}

int qmoe_forward(qmoe_ctx *c, int layer, const float *x, int n, float *out, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || (n > 0 && (!x || !out))) {
        seterr(err, "qmoe_forward: bad arguments");
        return -1;
    }
    if (n < 0 || n > c->cfg.max_tokens) {
        seterr(err, "qmoe_forward: n=%d outside [0, max_tokens=%d]", n, c->cfg.max_tokens);
        return -1;
    }
    if (n == 0) return 0;
    double t0 = now_s();
    size_t bytes = (size_t)n * c->L.d * sizeof(float);
    memcpy(c->x_pin, x, bytes);
    if (n == 1 && c->resident_all && layer >= 0 && layer < c->cfg.num_layers &&
        c->layers[layer].ready) {
        /* one token: x read by a small kernel from pinned memory (the decode
         * kernel's prologue overlaps it), the output written straight into
         * pinned memory, the error word copied back by a dependent launch;
         * no copy-engine transfers. The three launches are captured once per
         * layer as a graph (fixed buffers) and replayed. */
        layer_dev *ld = &c->layers[layer];
        if (!ld->tok_graph) {
            cudaGraph_t g = NULL;
            int ok = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
            if (ok) {
                int rc = qk_launch_copy_in(c->x_pin, c->x_dev, bytes, c->stream) ||
                         qmoe_forward_dev(c, layer, c->x_dev, QMOE_F32, n, c->out_pin, c->stream,
                                          err) ||
                         qk_launch_report(c->err_dev, c->err_host, c->tok_ctr_dev,
                                          c->tok_ctr_host, c->stream);
                cudaError_t ee = cudaStreamEndCapture(c->stream, &g);
                ok = rc == 0 && ee == cudaSuccess && g &&
                     cudaGraphInstantiate(&ld->tok_graph, g, 0) == cudaSuccess;
                if (g) cudaGraphDestroy(g);
            }
            if (!ok) {
                cudaGetLastError();
                ld->tok_graph = NULL;
                seterr(err, "qmoe_forward: could not capture the single-token call");
                return -1;
            }
            c->stats.decode_calls--; /* counted below, once per call */
        }
        c->stats.decode_calls++;
        c->last_T = 1;
        if (cudaGraphLaunch(ld->tok_graph, c->stream) != cudaSuccess) {
            seterr(err, "qmoe_forward: graph launch failed");
            return -1;
        }
        /* wait for the report kernel's count in pinned memory (no driver
         * call on the way); after 2 s, or on a count out of step, the stream
         * is synchronised, which also surfaces a failed launch */
        const unsigned want = ++c->tok_seq;
        volatile const unsigned *done = c->tok_ctr_host;
        int seen = 0;
        double tw = 0.0;
        for (unsigned spin = 0;; spin++) {
            if (*done == want) {
                seen = 1;
                break;
            }
            if ((spin & 1023u) == 1023u) {
                const double tn = now_s();
                if (tw == 0.0) tw = tn;
                else if (tn - tw > 2.0) break;
            }
        }
        if (!seen) {
            cudaError_t se = cudaStreamSynchronize(c->stream);
            if (se != cudaSuccess) {
                seterr(err, "qmoe_forward: %s", cudaGetErrorString(se));
                return -1;
            }
            c->tok_seq = *done;
        }
        if (report_dev_err(c, *(volatile int *)c->err_host, c->stream, err)) return -1;
        memcpy(out, c->out_pin, bytes);
        c->stats.forward_seconds += now_s() - t0;
        return 0;
    }
    cudaError_t ce = cudaMemcpyAsync(c->x_dev, c->x_pin, bytes, cudaMemcpyHostToDevice, c->stream);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
        return -1;
    }
    if (qmoe_forward_dev(c, layer, c->x_dev, QMOE_F32, n, c->out_dev, c->stream, err)) return -1;
    /* the error word and the output in one copy */
    ce = cudaMemcpyAsync(c->io_pin, c->io_dev, 256 + bytes, cudaMemcpyDeviceToHost, c->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->stream);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_forward: %s", cudaGetErrorString(ce));
        return -1;
    }
    if (report_dev_err(c, *c->err_host, c->stream, err)) return -1;
    memcpy(out, c->out_pin, bytes);
    c->stats.forward_seconds += now_s() - t0;
    return 0;
}

int qmoe_last_routing(qmoe_ctx *c, int32_t *idx, float *weights, float *shared_gate,
                      qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c) return -1;
    int n = c->last_T, k = c->L.k;
    cudaError_t ce = cudaStreamSynchronize(c->stream);
    if (ce == cudaSuccess && idx && n)
        ce = cudaMemcpy(idx, c->idx, (size_t)n * k * sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (ce == cudaSuccess && weights && n)
        ce = cudaMemcpy(weights, c->wts, (size_t)n * k * sizeof(float), cudaMemcpyDeviceToHost);
    if (ce == cudaSuccess && shared_gate && n)
        ce = cudaMemcpy(shared_gate, c->sgate, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_last_routing: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

/* -------------------------------------------------------- cache hooks */

int qmoe_expert_peek(qmoe_ctx *c, int layer, int e) {
    uint64_t v;
    if (!c || !qmoe_cache_peek(c->cache, ekey(layer, e), &v) || v == NO_OWNER) return -1;
    return (int)v;
}

int qmoe_expert_get(qmoe_ctx *c, int layer, int e) {
    uint64_t v;
    if (!c || !qmoe_cache_get(c->cache, ekey(layer, e), &v) || v == NO_OWNER) return -1;
    return (int)v;
}

int qmoe_experts_load(qmoe_ctx *c, int layer, const int64_t *ids, size_t n, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || layer < 0 || layer >= c->cfg.num_layers || (n && !ids)) {
        seterr(err, "qmoe_experts_load: bad arguments");
        return -1;
    }
    /* slots may be read by queued kernels: let them finish before reuse */
    cudaError_t ce = cudaStreamSynchronize(c->stream);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_experts_load: %s", cudaGetErrorString(ce));
        return -1;
    }
    return fill_experts(c, layer, ids, n, NULL, err);
}

int qmoe_expert_pin(qmoe_ctx *c, int layer, int e) {
    return c ? qmoe_cache_pin(c->cache, ekey(layer, e)) : 0;
}
int qmoe_expert_unpin(qmoe_ctx *c, int layer, int e) {
    return c ? qmoe_cache_unpin(c->cache, ekey(layer, e)) : 0;
}
int qmoe_expert_mark_hot(qmoe_ctx *c, int layer, int e, int hot) {
    return c ? qmoe_cache_mark_hot(c->cache, ekey(layer, e), hot) : 0;
}

int qmoe_cache_snapshot(qmoe_ctx *c, qmoe_cache_stats *out) {
    if (!c || !out) return -1;
    *out = qmoe_cache_stats_get(c->cache);
    return 0;
}

int qmoe_stats_get(qmoe_ctx *c, qmoe_stats *out) {
    if (!c || !out) return -1;
    *out = c->stats;
    return 0;
}

/* ------------------------------------------------------ prefetch hooks */

/* Prefetch fills ordered after the work queued on st (see qmoe_prefetch). */
static int prefetch_on(qmoe_ctx *c, int layer, const int64_t *ids, size_t n, cudaStream_t st) {
    if (!c || layer < 0 || layer >= c->cfg.num_layers || c->resident_all || (n && !ids)) return 0;
    qmoe_err e;
    int queued = 0;
    for (size_t i = 0; i < n; i++) {
        int ex = (int)ids[i];
        if (ex < c->ep_lo || ex >= c->ep_hi) continue; /* not this rank's */
        if (qmoe_cache_peek(c->cache, ekey(layer, ex), NULL)) continue;
        /* speculative fills in flight are capped (streaming.py:115, :235-241) */
        if (c->pf_outstanding >= c->max_speculative) break;
        int64_t one = ex;
        /* asynchronous: the copy waits, on the device, for the kernels
         * already queued on the compute stream (a victim slot may still be
         * read there) and never blocks the host */
        if (fill_experts(c, layer, &one, 1, st, &e) == 0) {
            queued++;
            c->pf_mark[(size_t)layer * c->L.E + ex] = 1;
            c->pf_outstanding++;
        }
    }
    c->stats.prefetch_issued += (uint64_t)queued;
    return queued;
}

int qmoe_prefetch(qmoe_ctx *c, int layer, const int64_t *ids, size_t n) {
    return c ? prefetch_on(c, layer, ids, n, c->stream) : 0;
}

void qmoe_record_route(qmoe_ctx *c, int layer, const int32_t *experts, size_t n) {
    if (!c || layer < 0 || layer >= c->cfg.num_layers) return;
    pthread_mutex_lock(&c->lock);
    qmoe_predictor_record(c->pred, c->cache, layer, experts, n, NULL);
    pthread_mutex_unlock(&c->lock);
}

static int prefetch_predictions_on(qmoe_ctx *c, int layer, const int32_t *selected, size_t n,
                                   cudaStream_t st) {
    if (!c || layer < 0 || layer >= c->cfg.num_layers || c->cfg.prefetch_depth <= 0) return 0;
    const int P = c->cfg.prefetch_depth < 64 ? c->cfg.prefetch_depth : 64;
    int64_t pick[64], next[64];
    int npick = 0, nnext = 0;
    pthread_mutex_lock(&c->lock);
    int rc = qmoe_predictor_predict(c->pred, layer, selected, n, P, pick, &npick, next, &nnext);
    pthread_mutex_unlock(&c->lock);
    if (rc) return 0;
    int q = prefetch_on(c, layer, pick, (size_t)npick, st);
    if (nnext) q += prefetch_on(c, layer + 1, next, (size_t)nnext, st);
    return q;
}

int qmoe_prefetch_predictions(qmoe_ctx *c, int layer, const int32_t *selected, size_t n) {
    return c ? prefetch_predictions_on(c, layer, selected, n, c->stream) : 0;
}

const qmoe_predictor *qmoe_ctx_predictor(const qmoe_ctx *c) { return c ? c->pred : NULL; }

int qmoe_upload_layer_ckpt(qmoe_ctx *c, int layer, qmoe_ckpt *ck, int ckpt_layer,
                           qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !ck) {
        seterr(err, "qmoe_upload_layer_ckpt: no context or checkpoint");
        return -1;
    }
    const size_t nb = qmoe_ckpt_layer_bytes(&c->cfg);
    void *buf = nb ? malloc(nb) : NULL;
    if (!buf) {
        seterr(err, "qmoe_upload_layer_ckpt: out of host memory (%zu bytes)", nb);
        return -1;
    }
    qmoe_layer_weights w;
    int rc = qmoe_ckpt_read_layer(ck, &c->cfg, ckpt_layer, buf, nb, &w, err);
    if (rc == 0) rc = qmoe_upload_layer(c, layer, &w, err);
    free(buf);
    return rc;
}

const char *qmoe_version(void) { return "qmoe-b200 0.1 (sm_100a)"; }

/* ------------------------------------------------- hyper connection */

static int dev_copy(void **dst, const void *src, size_t bytes, qmoe_err *err) {
    *dst = NULL;
    if (!src) return 0;
    cudaError_t ce = cudaMalloc(dst, bytes);
    if (ce == cudaSuccess) ce = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        seterr(err, "qmoe_upload_hc: %s", cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

int qmoe_upload_hc(qmoe_ctx *c, int layer, const qmoe_hc_weights *w, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !w || layer < 0 || layer >= c->cfg.num_layers) {
        seterr(err, "qmoe_upload_hc: bad arguments (layer %d)", layer);
        return -1;
    }
    const int d = c->L.d, hc = w->hc, lr = w->lowrank;
    const size_t hd = (size_t)hc * d;
    if (hc < 1 || hc > 8 || lr < 1 || !w->norm || !w->inject) {
        seterr(err, "qmoe_upload_hc: need 1 <= hc <= 8, lowrank >= 1, norm and inject (hc=%d lowrank=%d)",
               hc, lr);
        return -1;
    }
    if (w->down.q ? (!w->down.scales || hd % 64) : !w->down_bf16) {
        seterr(err, "qmoe_upload_hc: down mixer: q4 needs scales and hc*d %% 64 == 0, else dense bf16");
        return -1;
    }
    if (w->up.q ? (!w->up.scales || lr % 64) : !w->up_bf16) {
        seterr(err, "qmoe_upload_hc: up mixer: q4 needs scales and lowrank %% 64 == 0 (lowrank=%d), else "
                    "dense bf16", lr);
        return -1;
    }
    if (!qk_hc_smem_ok(d, hc)) {
        seterr(err, "qmoe_upload_hc: hc*d = %zu values do not fit the kernel's shared memory", hd);
        return -1;
    }
    if (cudaSetDevice(c->cfg.device) != cudaSuccess || cudaStreamSynchronize(c->stream) != cudaSuccess ||
        qk_hc_prepare(d, hc) != 0) {
        seterr(err, "qmoe_upload_hc: device set-up failed");
        return -1;
    }
    qk_hc_dev *h = &c->layers[layer].hc;
    hc_free(h);
    const size_t ngd = hd / 64, ngu = (size_t)lr / 64;
    int rc = dev_copy((void **)&h->norm, w->norm, hd * sizeof(float), err);
    if (!rc && w->down.q) {
        rc = dev_copy((void **)&h->down_q, w->down.q, (size_t)lr * hd / 2, err);
        if (!rc) rc = dev_copy((void **)&h->down_s, w->down.scales, (size_t)lr * ngd * 2, err);
        if (!rc) rc = dev_copy((void **)&h->down_b, w->down.biases, (size_t)lr * ngd * 2, err);
    } else if (!rc) {
        rc = dev_copy((void **)&h->down_bf, w->down_bf16, (size_t)lr * hd * 2, err);
    }
    if (!rc && w->up.q) {
        rc = dev_copy((void **)&h->up_q, w->up.q, hd * (size_t)lr / 2, err);
        if (!rc) rc = dev_copy((void **)&h->up_s, w->up.scales, hd * ngu * 2, err);
        if (!rc) rc = dev_copy((void **)&h->up_b, w->up.biases, hd * ngu * 2, err);
    } else if (!rc) {
        rc = dev_copy((void **)&h->up_bf, w->up_bf16, hd * (size_t)lr * 2, err);
    }
    if (!rc) rc = dev_copy((void **)&h->inject, w->inject, (size_t)hc * hd * 2, err);
    if (rc) {
        hc_free(h);
        return -1;
    }
    h->d = d;
    h->hc = hc;
    h->lowrank = lr;
    /* workspaces for max_tokens rows, grown to the widest layer */
    const size_t T = (size_t)c->cfg.max_tokens;
    if (!c->hc_mixed) {
        if (cudaMalloc((void **)&c->hc_mixed, T * d * sizeof(float)) != cudaSuccess ||
            cudaMalloc((void **)&c->hc_y, T * d * sizeof(float)) != cudaSuccess ||
            cudaMalloc((void **)&c->hc_sync, sizeof(unsigned long long)) != cudaSuccess ||
            cudaMemset(c->hc_sync, 0, sizeof(unsigned long long)) != cudaSuccess ||
            cudaMalloc(&c->hc_dsync, qk_decode_sync_bytes(&c->L)) != cudaSuccess ||
            cudaMemset(c->hc_dsync, 0, qk_decode_sync_bytes(&c->L)) != cudaSuccess) {
            seterr(err, "qmoe_upload_hc: out of device memory");
            return -1;
        }
    }
    if (lr > c->hc_lr) {
        cudaFree(c->hc_W);
        c->hc_W = NULL;
        if (cudaMalloc((void **)&c->hc_W, T * lr * sizeof(float)) != cudaSuccess) {
            seterr(err, "qmoe_upload_hc: out of device memory");
            return -1;
        }
        c->hc_lr = lr;
    }
    if (hc > c->hc_n) {
        cudaFree(c->hc_R);
        cudaFree(c->hc_INJ);
        c->hc_R = c->hc_INJ = NULL;
        if (cudaMalloc((void **)&c->hc_R, T * hc * sizeof(float)) != cudaSuccess ||
            cudaMalloc((void **)&c->hc_INJ, T * hc * sizeof(float)) != cudaSuccess) {
            seterr(err, "qmoe_upload_hc: out of device memory");
            return -1;
        }
        c->hc_n = hc;
    }
    return 0;
}

/* The one-token hyper-connection step as one decode-kernel launch
 * (QK_FUSED_UNFIT when the kernel's plan does not cover the shape). */
static int launch_hc_fused(qmoe_ctx *c, int layer, float *h, cudaStream_t st, unsigned long long *ptimes,
                           int pdl) {
    const qk_hc_dev *w = &c->layers[layer].hc;
    qk_fwd f;
    fill_fwd(c, layer, c->hc_mixed, 0, 1, c->hc_y, &f);
    f.ptimes = ptimes;
    f.hc_h = h;
    f.hc_inj = c->hc_INJ;
    f.hc_n = w->hc;
    f.hc_pre = 1;
    f.hc_lr = w->lowrank;
    f.hc_norm = w->norm;
    f.hc_down_q = w->down_q;
    f.hc_down_s = w->down_s;
    f.hc_down_b = w->down_b;
    f.hc_down_bf = w->down_bf;
    f.hc_up_q = w->up_q;
    f.hc_up_s = w->up_s;
    f.hc_up_b = w->up_b;
    f.hc_up_bf = w->up_bf;
    f.hc_inject = w->inject;
    f.hc_w = c->hc_W;
    f.hc_mixed = c->hc_mixed;
    return qk_launch_decode_fused(&f, c->hc_dsync, st, pdl);
}

/* Diagnostics: the phase timestamps of n_tokens back-to-back one-token
 * hyper-connection steps on h [n_tokens, hc*d] (as qmoe__phase_times_seq). */
int qmoe__phase_times_hc(qmoe_ctx *c, int layer, float *h, int n_tokens, unsigned long long *out_ns,
                         int max_ctas) {
    if (!c || !c->resident_all || layer < 0 || layer >= c->cfg.num_layers || !c->layers[layer].ready ||
        !c->layers[layer].hc.hc || n_tokens < 1)
        return -1;
    const size_t per = (size_t)c->num_sms * 32;
    const size_t row = (size_t)c->layers[layer].hc.hc * c->L.d;
    unsigned long long *buf = NULL;
    if (cudaMalloc((void **)&buf, per * n_tokens * sizeof(unsigned long long)) != cudaSuccess) return -1;
    int rc = cudaMemset(buf, 0, per * n_tokens * sizeof(unsigned long long));
    for (int t = 0; rc == 0 && t < n_tokens; t++)
        rc = launch_hc_fused(c, layer, h + row * t, c->stream, buf + per * t, t > 0);
    if (rc == 0) rc = cudaStreamSynchronize(c->stream);
    const int n = max_ctas < c->num_sms ? max_ctas : c->num_sms;
    for (int t = 0; rc == 0 && t < n_tokens; t++)
        rc = cudaMemcpy(out_ns + (size_t)t * max_ctas * 32, buf + per * t,
                        (size_t)n * 32 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(buf);
    return rc == 0 ? c->num_sms : -1;
}

int qmoe_forward_hc(qmoe_ctx *c, int layer, float *h, int n, void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !h || layer < 0 || layer >= c->cfg.num_layers) {
        seterr(err, "qmoe_forward_hc: bad arguments (layer %d)", layer);
        return -1;
    }
    const qk_hc_dev *w = &c->layers[layer].hc;
    if (!w->hc) {
        seterr(err, "qmoe_forward_hc: layer %d has no hyper connection (qmoe_upload_hc)", layer);
        return -1;
    }
    if (n < 0 || n > c->cfg.max_tokens) {
        seterr(err, "qmoe_forward_hc: n=%d outside [0, max_tokens=%d]", n, c->cfg.max_tokens);
        return -1;
    }
    if (!c->layers[layer].ready) {
        seterr(err, "qmoe_forward_hc: layer %d was not uploaded", layer);
        return -1;
    }
    if (n == 0) return 0;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (n == 1 && c->resident_all) {
        /* one token: gated_residual in the decode kernel's prologue and the
         * inject-add in its combine, one launch */
        const int rc = launch_hc_fused(c, layer, h, st, NULL, 1);
        if (rc == 0) {
            c->last_T = 1;
            c->stats.decode_calls++;
            return 0;
        }
        if (rc != QK_FUSED_UNFIT) return kerr(rc, "decode_fused", err);
    }
    if (kerr(qk_launch_hc_pre(w, h, n, c->hc_W, c->hc_R, c->hc_INJ, c->hc_mixed, c->hc_sync, c->err_dev,
                              c->num_sms, st),
             "hc pre", err))
        return -1;
    if (n == 1 && c->resident_all && c->layers[layer].ready) {
        /* one token: the decode kernel adds inject x its output to h itself */
        qk_fwd f;
        fill_fwd(c, layer, c->hc_mixed, 0, 1, c->hc_y, &f);
        f.hc_h = h;
        f.hc_inj = c->hc_INJ;
        f.hc_n = w->hc;
        const int rc = qk_launch_decode_fused(&f, c->dsync, st, 1);
        if (rc == 0) {
            c->last_T = 1;
            c->stats.decode_calls++;
            return 0;
        }
        if (rc != QK_FUSED_UNFIT) return kerr(rc, "decode_fused", err);
    }
    if (qmoe_forward_dev(c, layer, c->hc_mixed, QMOE_F32, n, c->hc_y, st, err)) return -1;
    return kerr(qk_launch_hc_inject(h, c->hc_INJ, c->hc_y, n, w->hc, w->d, st), "hc inject", err);
}

/* ------------------------------------------------- expert parallelism */

#define NCK(call, what)                                                                   \
    do {                                                                                  \
        ncclResult_t r_ = (call);                                                         \
        if (r_ != ncclSuccess) {                                                          \
            seterr(err, "%s: NCCL %s", what, nccl_api()->error_string(r_));               \
            return -1;                                                                    \
        }                                                                                 \
    } while (0)

int qmoe_ep_unique_id(unsigned char id[QMOE_EP_ID_BYTES], qmoe_err *err) {
    if (err) err->msg[0] = 0;
    const nccl_fns *n = nccl_api();
    if (!n->ok) {
        seterr(err, "qmoe_ep_unique_id: libnccl.so.2 could not be loaded");
        return -1;
    }
    ncclUniqueId u;
    NCK(n->get_unique_id(&u), "qmoe_ep_unique_id");
    memcpy(id, u.internal, QMOE_EP_ID_BYTES);
    return 0;
}

/* Every rank's bytes [len] at slot rank of all [W][len] (device), over the
 * communicator. */
static int ep_allgather(qmoe_ctx *c, const unsigned char *mine, unsigned char *all, size_t len, qmoe_err *err) {
    const nccl_fns *n = nccl_api();
    const int W = c->ep_world, me = c->ep_rank;
    unsigned char *dev = NULL;
    cudaError_t ce = cudaMalloc((void **)&dev, (size_t)W * len);
    if (ce == cudaSuccess) ce = cudaMemcpy(dev + (size_t)me * len, mine, len, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        cudaFree(dev);
        seterr(err, "qmoe_ep_connect: %s", cudaGetErrorString(ce));
        return -1;
    }
    ncclResult_t r = n->group_start();
    for (int p = 0; p < W && r == ncclSuccess; p++) {
        if (p == me) continue;
        r = n->send(dev + (size_t)me * len, len, ncclUint8, p, c->ep_comm, c->stream);
        if (r == ncclSuccess) r = n->recv(dev + (size_t)p * len, len, ncclUint8, p, c->ep_comm, c->stream);
    }
    const ncclResult_t r2 = n->group_end();
    if (r == ncclSuccess) r = r2;
    ce = cudaStreamSynchronize(c->stream);
    if (r == ncclSuccess && ce == cudaSuccess) ce = cudaMemcpy(all, dev, (size_t)W * len, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (r != ncclSuccess || ce != cudaSuccess) {
        seterr(err, "qmoe_ep_connect: exchange failed (%s)",
               r != ncclSuccess ? n->error_string(r) : cudaGetErrorString(ce));
        return -1;
    }
    return 0;
}

/* The peer-memory exchange when every rank can map every other rank's
 * buffers (another GPU with peer access; QMOE_EP_P2P=0 keeps NCCL): the IPC
 * handles and device ordinals travel over the communicator, then every
 * rank reports whether it mapped all of them, and the ranks use peer memory
 * only if all did (they must take the same path). Collective. */
static int ep_try_p2p(qmoe_ctx *c, qmoe_err *err) {
    enum { LEN = 5 * 64 + 8 };
    const int W = c->ep_world, me = c->ep_rank;
    const char *pv = getenv("QMOE_EP_P2P");
    unsigned char mine[LEN];
    memset(mine, 0, sizeof(mine));
    int want = !(pv && strcmp(pv, "0") == 0) && c->prefill != NULL;
    if (want && qk_ep_ipc_handles(c->prefill, mine) != 0) {
        cudaGetLastError();
        want = 0;
    }
    memcpy(mine + 320, &c->cfg.device, 4);
    memcpy(mine + 324, &want, 4);
    unsigned char *all = calloc((size_t)W, LEN);
    if (!all) {
        seterr(err, "qmoe_ep_connect: out of host memory");
        return -1;
    }
    if (ep_allgather(c, mine, all, LEN, err)) {
        free(all);
        return -1;
    }
    int ok = 1;
    for (int p = 0; p < W; p++) {
        int dev, w;
        memcpy(&dev, all + (size_t)p * LEN + 320, 4);
        memcpy(&w, all + (size_t)p * LEN + 324, 4);
        if (!w) ok = 0;
        if (p == me) continue;
        int can = 0;
        if (dev == c->cfg.device || cudaDeviceCanAccessPeer(&can, c->cfg.device, dev) != cudaSuccess || !can)
            ok = 0;
    }
    cudaGetLastError();
    if (ok) {
        unsigned char *h = calloc((size_t)W, 5 * 64);
        if (!h) ok = 0;
        for (int p = 0; h && p < W; p++) memcpy(h + (size_t)p * 5 * 64, all + (size_t)p * LEN, 5 * 64);
        if (ok && qk_ep_p2p_open(c->prefill, h, me) != 0) {
            cudaGetLastError();
            ok = 0;
        }
        free(h);
    }
    free(all);
    /* every rank's outcome: peer memory only if all mapped everything */
    unsigned char okb[8] = {0};
    memcpy(okb, &ok, 4);
    unsigned char *oks = calloc((size_t)W, 8);
    if (!oks) {
        seterr(err, "qmoe_ep_connect: out of host memory");
        return -1;
    }
    if (ep_allgather(c, okb, oks, 8, err)) {
        free(oks);
        return -1;
    }
    int all_ok = 1;
    for (int p = 0; p < W; p++) {
        int v;
        memcpy(&v, oks + (size_t)p * 8, 4);
        if (!v) all_ok = 0;
    }
    free(oks);
    if (!all_ok) qk_ep_p2p_close(c->prefill);
    c->ep_p2p = all_ok;
    return 0;
}

/* Diagnostics: 1 when this context's exchanges go through peer memory. */
int qmoe__ep_p2p(const qmoe_ctx *c) { return c ? c->ep_p2p : 0; }

int qmoe_ep_connect(qmoe_ctx *c, const unsigned char id[QMOE_EP_ID_BYTES], qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || c->ep_world < 2) {
        seterr(err, "qmoe_ep_connect: the context was created without ep_world > 1");
        return -1;
    }
    const nccl_fns *n = nccl_api();
    if (!n->ok) {
        seterr(err, "qmoe_ep_connect: libnccl.so.2 could not be loaded");
        return -1;
    }
    if (c->ep_comm) return 0;
    ncclUniqueId u;
    memcpy(u.internal, id, QMOE_EP_ID_BYTES);
    if (cudaSetDevice(c->cfg.device) != cudaSuccess) {
        seterr(err, "qmoe_ep_connect: cudaSetDevice failed");
        return -1;
    }
    NCK(n->comm_init_rank(&c->ep_comm, c->ep_world, u, c->ep_rank), "qmoe_ep_connect");
    return ep_try_p2p(c, err);
}

/* One collective forward: every rank calls it for the same layer with its
 * own n tokens. Route locally; send every rank a block of max_tokens rows in
 * which row t is token t when that rank owns one of its experts (x as given,
 * slot expert ids and weights) and a row of expert ids -1 otherwise; one
 * grouped pass runs the shared expert on the own tokens and this rank's
 * experts on the rows received, combining each received row's local slots;
 * those partial rows go back; add them (rank order) and the shared expert's
 * rows. No host synchronisation: the call can be captured in a graph. */
int qmoe_forward_ep(qmoe_ctx *c, int layer, const void *x, int x_dtype, int n, float *out,
                    void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !c->ep_comm) {
        seterr(err, "qmoe_forward_ep: no expert-parallel communicator (qmoe_ep_connect)");
        return -1;
    }
    if (layer < 0 || layer >= c->cfg.num_layers || !c->layers[layer].ready) {
        seterr(err, "qmoe_forward_ep: layer %d is not uploaded", layer);
        return -1;
    }
    if (n < 0 || n > c->cfg.max_tokens || (n > 0 && (!x || !out))) {
        seterr(err, "qmoe_forward_ep: n=%d outside [0, max_tokens=%d] or missing buffers", n,
               c->cfg.max_tokens);
        return -1;
    }
    if (x_dtype != QMOE_F32 && x_dtype != QMOE_BF16) {
        seterr(err, "qmoe_forward_ep: unknown x dtype %d", x_dtype);
        return -1;
    }
    const nccl_fns *nc = nccl_api();
    const int W = c->ep_world, d = c->L.d, k = c->L.k;
    const size_t cap = (size_t)c->cfg.max_tokens;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    if (cudaSetDevice(c->cfg.device) != cudaSuccess) {
        seterr(err, "qmoe_forward_ep: cudaSetDevice failed");
        return -1;
    }
    qk_fwd f;
    fill_fwd(c, layer, x, x_dtype == QMOE_BF16, n, out, &f);
    c->last_T = n;
    c->stats.prefill_calls++;
    qk_ep_bufs b;
    qk_ep_buffers(c->prefill, &b);
    if (n > 0 && route(c, layer, &f, st, 0, NULL, err)) return -1;
    /* the receive buffer: the own tokens in rows [0, cap), rank p's rows
     * from cap + p cap on; x travels as given (bf16 or fp32: every rank
     * passes the same dtype) */
    const size_t own = cap, row = (size_t)d * (x_dtype == QMOE_BF16 ? 2 : 4);
    if (c->ep_p2p) {
        /* peer memory: rows written straight into their destinations */
        if (kerr(qk_ep_dispatch_p2p(c->prefill, &f, c->ep_rank, st), "ep dispatch", err) ||
            kerr(qk_ep_wait(c->prefill, 0, c->err_dev, st), "ep wait", err))
            return -1;
    } else {
    if (kerr(qk_ep_dispatch(c->prefill, &f, st), "ep dispatch", err)) return -1;
    NCK(nc->group_start(), "qmoe_forward_ep");
    for (int p = 0; p < W; p++) {
        const size_t so = (size_t)p * cap, ro = own + (size_t)p * cap;
        NCK(nc->send((const uint8_t *)b.send_x + so * row, cap * row, ncclUint8, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
        NCK(nc->send(b.send_e + so * k, cap * k, ncclInt32, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
        NCK(nc->send(b.send_w + so * k, cap * k, ncclFloat32, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
        NCK(nc->recv((uint8_t *)b.recv_x + ro * row, cap * row, ncclUint8, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
        NCK(nc->recv(b.recv_e + ro * k, cap * k, ncclInt32, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
        NCK(nc->recv(b.recv_w + ro * k, cap * k, ncclFloat32, p, c->ep_comm, st),
            "qmoe_forward_ep dispatch");
    }
    NCK(nc->group_end(), "qmoe_forward_ep");
    }
    if (!c->resident_all) {
        /* streaming pool: the rows received name this rank's experts; fill
         * the missing ones before the grouped pass reads the pool */
        const size_t nr = (size_t)W * cap * k;
        cudaError_t ce = cudaMemcpyAsync(c->ep_recv_pin, b.recv_e + own * k, nr * sizeof(int32_t),
                                         cudaMemcpyDeviceToHost, st);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            seterr(err, "qmoe_forward_ep: %s", cudaGetErrorString(ce));
            return -1;
        }
        int64_t *uniq = calloc(nr ? nr : 1, sizeof(int64_t));
        unsigned char *seen = calloc((size_t)c->L.E, 1);
        if (!uniq || !seen) {
            free(uniq);
            free(seen);
            seterr(err, "qmoe_forward_ep: out of host memory");
            return -1;
        }
        size_t nu = 0;
        for (size_t i = 0; i < nr; i++) {
            const int e = c->ep_recv_pin[i];
            if (e < 0 || e >= c->L.E || seen[e]) continue;
            seen[e] = 1;
            uniq[nu++] = e;
            const int resident = qmoe_cache_peek(c->cache, ekey(layer, e), NULL);
            c->stats.routed_lookups++;
            c->stats.routed_hits += (uint64_t)resident;
            unsigned char *pm = c->pf_mark + (size_t)layer * c->L.E + e;
            if (*pm) {
                if (resident) c->stats.prefetch_hits++;
                *pm = 0;
                c->pf_outstanding--;
            }
        }
        free(seen);
        int rc = fill_experts(c, layer, uniq, nu, st, err);
        if (rc == 0) rc = mark_fills_ready(c, st, err);
        if (rc == 0) {
            pthread_mutex_lock(&c->lock);
            for (size_t i = 0; i < nu; i++) qmoe_cache_get(c->cache, ekey(layer, (int)uniq[i]), NULL);
            pthread_mutex_unlock(&c->lock);
        }
        free(uniq);
        if (rc) return -1;
    }
    /* this rank's experts over the rows it received, combined per row */
    if (c->ep_p2p) {
        /* partial rows written straight into their owners' return rows */
        if (kerr(qk_ep_experts_p2p(c->prefill, &f, c->nslots + layer, c->ep_rank, st), "ep experts", err) ||
            kerr(qk_ep_wait(c->prefill, 1, c->err_dev, st), "ep wait", err))
            return -1;
        if (n > 0 && kerr(qk_ep_finish(c->prefill, &f, st), "ep finish", err)) return -1;
        return 0;
    }
    if (kerr(qk_ep_experts(c->prefill, &f, c->nslots + layer, st), "ep experts", err)) return -1;
    /* partial rows back to the ranks that own the tokens */
    NCK(nc->group_start(), "qmoe_forward_ep");
    for (int p = 0; p < W; p++) {
        const size_t o = (size_t)p * cap;
        NCK(nc->send(b.ret + o * d, cap * d, ncclFloat32, p, c->ep_comm, st),
            "qmoe_forward_ep combine");
        NCK(nc->recv(b.back + o * d, cap * d, ncclFloat32, p, c->ep_comm, st),
            "qmoe_forward_ep combine");
    }
    NCK(nc->group_end(), "qmoe_forward_ep");
    if (n > 0 && kerr(qk_ep_finish(c->prefill, &f, st), "ep finish", err)) return -1;
    return 0;
}

/* MoE-only stack over layers [l0, l1): h_{l+1} = h_l + MoE_l(RMSNorm(h_l)),
 * RMSNorm with unit weight and eps; each layer through qmoe_forward_ep on an
 * expert-parallel context, else qmoe_forward_dev. h: fp32 [n, d] device
 * rows, updated in place. With every expert resident it is stream-ordered
 * only (no host synchronisation), so a whole stack can be captured in a
 * graph; a streaming context waits for each layer's routing on the host to
 * fill its experts, then records the route and queues the predicted
 * prefetches. */
int qmoe_forward_stack(qmoe_ctx *c, int l0, int l1, float *h, int n, float eps, void *stream,
                       qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!c || !h || l0 < 0 || l1 > c->cfg.num_layers || l0 > l1 || n < 0 ||
        n > c->cfg.max_tokens) {
        seterr(err, "qmoe_forward_stack: bad arguments (layers [%d, %d), n=%d)", l0, l1, n);
        return -1;
    }
    if (c->ep_world > 1 && !c->ep_comm) {
        seterr(err, "qmoe_forward_stack: no expert-parallel communicator (qmoe_ep_connect)");
        return -1;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const int d = c->L.d;
    for (int l = l0; l < l1; l++) {
        int rc = qk_launch_residual_norm(h, l > l0 ? c->stk_y : NULL, c->stk_xn, n, d, eps, st);
        if (kerr(rc, "residual_norm", err)) return -1;
        if (c->ep_world > 1) rc = qmoe_forward_ep(c, l, c->stk_xn, QMOE_F32, n, c->stk_y, st, err);
        else rc = n > 0 ? qmoe_forward_dev(c, l, c->stk_xn, QMOE_F32, n, c->stk_y, st, err) : 0;
        if (rc) return -1;
        if (!c->resident_all && n > 0) {
            /* streaming: route statistics and predicted prefetches follow the
             * layer's routing (on the host already, or read back here on an
             * expert-parallel context), as model.py:458-459 calls
             * record_route and prefetch_predictions */
            const size_t nk = (size_t)n * c->L.k;
            if (c->ep_world > 1) {
                cudaError_t ce = cudaMemcpyAsync(c->idx_pin, c->idx, nk * sizeof(int32_t),
                                                 cudaMemcpyDeviceToHost, st);
                if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
                if (ce != cudaSuccess) {
                    seterr(err, "qmoe_forward_stack: layer %d failed on the device", l);
                    return -1;
                }
            }
            /* (single GPU: idx_pin already holds the layer's routing, read
             * before its fills; no wait for the layer's kernels here, since a
             * prefetch's copies wait for them on the device) */
            /* record every assignment; predict from the distinct experts in
             * ascending order (np.unique at model.py:432) */
            pthread_mutex_lock(&c->lock);
            const int ns = qmoe_predictor_record(c->pred, c->cache, l, c->idx_pin, nk, c->sel_buf);
            pthread_mutex_unlock(&c->lock);
            if (ns > 0) prefetch_predictions_on(c, l, c->sel_buf, (size_t)ns, st);
        }
    }
    if (l1 > l0 && kerr(qk_launch_residual_norm(h, c->stk_y, NULL, n, d, eps, st), "residual_norm", err))
        return -1;
    return 0;
}

int qmoe_ep_plan_host(const int32_t *idx, int n, int k, int E, int W, int cap, int *counts,
                      int *pos) {
    if (!idx || !counts || n < 0 || cap < n || k < 1 || W < 1 || W > 64 || E % W) return -1;
    const int e_per = E / W;
    for (int g = 0; g < W; g++) counts[g] = 0;
    for (int t = 0; t < n; t++) {
        unsigned long long m = 0;
        for (int s = 0; s < k; s++) {
            int e = idx[(size_t)t * k + s];
            if (e < 0 || e >= E) return -1;
            m |= 1ull << (e / e_per);
        }
        for (int g = 0; g < W; g++) {
            const int live = (int)((m >> g) & 1ull);
            counts[g] += live;
            if (pos) pos[(size_t)g * n + t] = live ? g * cap + t : -1;
        }
    }
    return 0;
}
