/*
 * qmoe.h - C ABI of the B200 mixture-of-experts layer.
 *
 * Drop-in for the MoE path of the reference runtime's C port:
 *   moe_forward      c/src/model.c:1281-1405 (called at model.c:1712)
 *   experts_load     c/src/model.c:539-674
 *   the expert cache c/src/cache.h:38-60 (instance at model.c:1806)
 *   prefetch hooks   src/colibri_runtime/streaming.py:226-435 (the C port
 *                    parses --expert-prefetch but never uses it,
 *                    c/src/main.c:65,:99,:264)
 *
 * All entry points are plain C: pointers, sizes and integers. CUDA streams
 * are passed as void * (a cudaStream_t). Every call returns 0 on success and
 * -1 on failure with a message in *err, the reference's convention
 * (err_t, c/src/util.h:11-19; -1 returns as at model.c:552, :1351).
 *
 * One context drives one GPU. A context is not re-entrant: calls on one
 * context must not overlap. The expert-cache bookkeeping is internally
 * locked, as the reference's cache is (c/src/cache.c:186-208).
 */
#ifndef QMOE_H
#define QMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same size and meaning as the reference's err_t (c/src/util.h:11-13); a
 * caller holding an err_t may pass it here by pointer cast. */
typedef struct {
    char msg[512];
} qmoe_err;

/* Expert cache policies, c/src/cache.h:8-10. */
enum { QMOE_POLICY_LRU = 0, QMOE_POLICY_LFU = 1, QMOE_POLICY_ADAPTIVE = 2 };

/* Element type of device-resident activations passed to qmoe_forward_dev. */
enum { QMOE_F32 = 0, QMOE_BF16 = 1 };

typedef struct {
    int hidden;          /* d: hidden_size */
    int num_experts;     /* E: num_experts (<= 1024) */
    int top_k;           /* k: num_experts_per_tok (<= 32) */
    int moe_inter;       /* I: moe_intermediate_size; the shared expert uses it
                            too, as model.c:1391-1392 does */
    int group_size;      /* quantization.group_size (64) */
    int bits;            /* quantization.bits (4) */
    int num_layers;      /* layers this context serves */
    int max_tokens;      /* largest n of one forward call (sizes workspaces) */
    uint64_t pool_bytes; /* HBM expert pool budget in bytes; 0 = room for every
                            expert of every layer (all resident). A streaming
                            pool must hold at least top_k slots. A multi-token
                            call whose distinct routed experts of a layer do
                            not fit runs them in waves of at most a pool each
                            (filled, then computed; one combine at the end),
                            with the result of a pool that holds them all, as
                            the reference reloads evicted experts inside its
                            expert loop (model.c:1341-1349). Expert-parallel
                            streaming calls need a rank's experts of a call to
                            fit at once. */
    int policy;          /* QMOE_POLICY_* for the pool (reference: ADAPTIVE) */
    int prefetch_depth;  /* prefetch_count of streaming.py (2) */
    int device;          /* CUDA device ordinal */
    int ep_rank;         /* expert parallelism: this context's rank ... */
    int ep_world;        /* ... of ep_world (0 or 1: no expert parallelism). Rank
                            g holds experts [g E/W, (g+1) E/W) of every layer
                            (E % W == 0) and serves qmoe_forward_ep;
                            max_tokens is the per-rank token count of one
                            call. With pool_bytes below the rank's share the
                            rank streams its own experts from a pinned host
                            store of those experts only */
} qmoe_config;

/* One affine 4-bit tensor in the reference checkpoint layout: `rows` rows of
 * `cols` values; q holds cols/8 u32 words per row, low nibble first; scales
 * and biases hold cols/group bf16 values per row (dequant: q*s + b,
 * c/src/kernel.c:152-173). For the routed experts the E tensors are stacked
 * ([E, rows, cols/8] etc., model.c:555-557). */
typedef struct {
    const uint32_t *q;
    const uint16_t *scales;
    const uint16_t *biases;
} qmoe_q4;

/* Host tensors of one MoE layer (tensor names as model.c:1902-1923 and
 * model.c:541-546). */
typedef struct {
    const uint16_t *router;      /* bf16 [E, d]   mlp.gate.weight */
    const uint16_t *shared_gate; /* bf16 [1, d]   mlp.shared_expert_gate.weight */
    const float *logit_bias;     /* fp32 [E] added to the router logits, or NULL */
    qmoe_q4 gate, up;            /* switch_mlp.{gate,up}_proj  [E, I, d] */
    qmoe_q4 down;                /* switch_mlp.down_proj       [E, d, I] */
    qmoe_q4 sh_gate, sh_up;      /* shared_expert.{gate,up}_proj [I, d] */
    qmoe_q4 sh_down;             /* shared_expert.down_proj      [d, I] */
} qmoe_layer_weights;

/* Cache counters, c/src/cache.h:55-58. */
typedef struct {
    uint64_t hits, misses, evictions, rejected, pinned;
    uint64_t bytes, peak_bytes, size, hot;
} qmoe_cache_stats;

/* Runtime counters, mirroring qstats (c/src/model.h:18-24). */
typedef struct {
    uint64_t expert_loads, expert_bytes;   /* host -> HBM slot fills */
    double expert_wait_seconds;            /* host time blocked on fills */
    uint64_t prefill_calls, decode_calls;
    double forward_seconds;                /* host wall time inside qmoe_forward */
    uint64_t prefetch_issued, prefetch_hits;
    /* streaming: distinct experts a call's routing selected per layer, and
     * how many of them were already in the pool before its fills */
    uint64_t routed_lookups, routed_hits;
    /* prefetched experts evicted before any routing reached them
     * (StreamStats.prefetch_wasted, streaming.py:346-349) */
    uint64_t prefetch_wasted;
    /* streaming: waves run by calls that routed to more distinct experts of
     * a layer than the pool has slots (each wave fills at most a pool) */
    uint64_t expert_waves;
} qmoe_stats;

typedef struct qmoe_ctx qmoe_ctx;

/* ---- context (replaces model_load's MoE part, c/src/model.h:27-28) ---- */

qmoe_ctx *qmoe_create(const qmoe_config *cfg, qmoe_err *err);
void qmoe_destroy(qmoe_ctx *ctx);

/* Bytes of one expert slot in HBM (the packed q4 expert, rows padded to 16
 * bytes): 1,769,472 at d=2048, I=512. */
size_t qmoe_slot_bytes(const qmoe_config *cfg);

/* Copies one layer's tensors (host memory, reference layout) into the
 * context: router, shared gate, shared expert and bias to HBM; routed experts
 * to the HBM pool when they fit, and to the pinned host store otherwise. */
int qmoe_upload_layer(qmoe_ctx *ctx, int layer, const qmoe_layer_weights *w,
                      qmoe_err *err);

/* ---- forward (replaces moe_forward, c/src/model.c:1281) ----
 * x: host fp32 [n, d]; out: host fp32 [n, d], overwritten. Synchronous. */
int qmoe_forward(qmoe_ctx *ctx, int layer, const float *x, int n, float *out,
                 qmoe_err *err);

/* Device-resident variant: x is a device pointer of QMOE_F32 or QMOE_BF16
 * elements [n, d]; out a device fp32 [n, d]. Enqueued on `stream` (NULL = the
 * context's stream); returns without waiting when every routed expert of the
 * layer is resident in HBM. Device-side wait timeouts are reported by the
 * next qmoe_sync / qmoe_forward call. */
int qmoe_forward_dev(qmoe_ctx *ctx, int layer, const void *x, int x_dtype,
                     int n, float *out, void *stream, qmoe_err *err);

/* Waits for the context's work and reports any device-side error. */
int qmoe_sync(qmoe_ctx *ctx, qmoe_err *err);

/* MoE-only layer stack (the workload's 76-layer configuration; attention
 * replaced by the identity): for l in [l0, l1)
 *   h <- h + MoE_l(RMSNorm(h)),  RMSNorm unit weight, eps (1e-6 there),
 * RMSNorm as kernel_rmsnorm (c/src/kernel.c:10-20). h: device fp32 [n, d],
 * updated in place. Each layer is qmoe_forward_dev, or qmoe_forward_ep on an
 * expert-parallel context (then collective: every rank calls it for the same
 * layers). Enqueued on `stream` without any host synchronisation, so the
 * whole stack can be captured in one CUDA graph. No reference counterpart:
 * the reference calls moe_forward once per layer from model_forward
 * (c/src/model.c:1712). */
int qmoe_forward_stack(qmoe_ctx *ctx, int l0, int l1, float *h, int n, float eps,
                       void *stream, qmoe_err *err);

/* ---- one decode token without any allocation (no counterpart in the
 *      reference runtime) ----
 * For callers that cannot call cudaMalloc: code that must run inside a
 * device-memory budget or arena owned by someone else, or on a path where an
 * allocation could block, fail or be forbidden at run time. qmoe_create
 * allocates its workspaces; this entry point allocates nothing. The caller
 * passes every input and output in device memory, including the experts
 * already packed in the slot layout:
 *   slot = GU section (I rows) then D section (d rows), zero-padded to
 *   qmoe_slot_bytes(cfg);
 *   GU row n = gate q row (d/2 bytes) | up q row (d/2 bytes) |
 *              per group j < d/g: gate scale, gate bias, up scale, up bias
 *              (4 bf16);
 *   D row n  = down q row (I/2 bytes) | per group j < I/g: scale, bias
 *              (2 bf16) | zeros to a multiple of 16 bytes;
 *   q rows are the checkpoint rows verbatim (u32 words, low nibble first).
 * The call's intermediates (routing, the router logits and gate/up
 * activations that the kernel's thread blocks exchange, a grid-barrier
 * counter and an error word) live in one device array of QMOE_NOALLOC_SCRATCH_BYTES
 * defined inside the library; every GPU that loads the library holds it until
 * the process exits. A shape needing more than that (at most
 * 4 * (E + 4 + (k + 1) * I) + 768 bytes) is rejected with an error, as is a
 * shape the single-launch decode kernel does not cover.
 * The first call on a device looks up the array's device address and sets
 * kernel attributes, with that device current; make that first call before
 * any stream capture. All calls share the array and each call starts by
 * clearing its error word, barrier counter and exchange area, so calls that
 * overlap on the GPU race; serialise them. x, out, router, shared_gate, pool,
 * slot_of and shared_slot must be 16-byte aligned (the kernel moves them with
 * 16-byte vector loads and bulk copies; slots are multiples of 16 bytes), and
 * logit_bias 4-byte aligned: other addresses are refused before any launch.
 * Before returning, the call synchronises `stream` (NULL = the legacy default
 * stream) and reads the error word back with a blocking copy; it returns 0,
 * or -1 with a message. */
#define QMOE_NOALLOC_SCRATCH_BYTES (64u * 1024u)
typedef struct {
    int hidden, num_experts, top_k, moe_inter, group_size;
    const void *x;               /* [1, d] device, QMOE_F32 or QMOE_BF16 */
    int x_dtype;
    float *out;                  /* [1, d] device fp32, overwritten */
    const uint16_t *router;      /* [E, d] bf16 device */
    const uint16_t *shared_gate; /* [d] bf16 device */
    const float *logit_bias;     /* [E] device, or NULL */
    const uint8_t *pool;         /* device base of the packed expert slots */
    const int32_t *slot_of;      /* [E] device: slot index of each expert */
    const uint8_t *shared_slot;  /* device: the packed shared expert */
} qmoe_token_args;
int qmoe_forward_token_noalloc(const qmoe_token_args *a, void *stream,
                               qmoe_err *err);

/* ---- the MoE side's hyper connection around the block ----
 * The C port's layer wraps the MoE block in a hyper connection
 * (mlp_hyper_connection.*, c/src/model.c:1945-1964): the residual state of a
 * token is hc streams of d values, h [n, hc*d]. qmoe_forward_hc runs, on the
 * device, gated_residual (c/src/model.c:728-796: each stream RMS-normalised
 * with eps 1e-6 and scaled by norm; w = silu(down(normed) / hc);
 * tmp = sigmoid(up(w)); mixed = the streams' mean of tmp * normed;
 * inject = 2 sigmoid(inject(normed) / hc)), the MoE block of `layer` on
 * mixed (as qmoe_forward_dev), and the inject-add after it
 * (c/src/model.c:1723-1731: h[t, c, :] += inject[t, c] * moe[t, :]), in
 * stream order, without host waits on a resident context. The mixers are q4
 * with group 64 (absent biases read as zeros; up needs lowrank % 64 == 0) or
 * dense bf16 (q NULL); dense bf16 products and inject use the canonical dot
 * of the router. */
typedef struct {
    int hc;                      /* hc_count: streams (1..8) */
    int lowrank;                 /* hc_lowrank */
    const float *norm;           /* [hc*d] hc_norm.weight, widened to fp32 */
    qmoe_q4 down;                /* input_mix_weight_down [lowrank, hc*d] */
    const uint16_t *down_bf16;   /* or dense bf16 [lowrank, hc*d] when down.q is NULL */
    qmoe_q4 up;                  /* input_mix_weight_up [hc*d, lowrank] */
    const uint16_t *up_bf16;     /* or dense bf16 [hc*d, lowrank] when up.q is NULL */
    const uint16_t *inject;      /* block_inject_weight bf16 [hc, hc*d] */
} qmoe_hc_weights;
/* Copies one layer's hyper-connection weights to the device (host pointers).
 * Returns 0, or -1 with a message (shapes the kernels do not cover included). */
int qmoe_upload_hc(qmoe_ctx *ctx, int layer, const qmoe_hc_weights *w, qmoe_err *err);
/* h: device fp32 [n, hc*d], updated in place; n <= max_tokens. */
int qmoe_forward_hc(qmoe_ctx *ctx, int layer, float *h, int n, void *stream, qmoe_err *err);

/* Expert parallelism over ep_world GPUs, one context (and one process or
 * thread) per GPU, created with qmoe_config.ep_rank / ep_world. Experts are
 * partitioned as in a config-2/3 expert-parallel run: rank g owns experts
 * [g E/W, (g+1) E/W) of every layer; the router and the shared expert are on
 * every rank. Rank 0 makes an id (qmoe_ep_unique_id), the caller hands it to
 * every rank, and each rank calls qmoe_ep_connect (collective; NCCL is
 * loaded at run time from libnccl.so.2).
 * qmoe_forward_ep is a collective replacement of qmoe_forward_dev for the
 * rank's own n tokens (device pointers, n may differ between ranks and may
 * be 0; x_dtype the same on every rank): local routing; each token sent
 * once (x as given, bf16 or fp32, with its k slots) to
 * every rank that owns one of its experts; the owners' grouped GEMMs and a
 * weighted combine of each token's local slots; one fp32 partial row per
 * (token, rank) sent back; on the token's rank the partials (in rank order)
 * plus the shared expert. Transfers have a fixed size, max_tokens rows
 * between every pair of ranks (token t in row t, rows of tokens not bound
 * for a rank carrying expert ids -1), so the call never waits on the host
 * and can be captured in a CUDA graph; size max_tokens to the tokens per
 * rank actually used. No reference counterpart: the C port runs on one
 * device. */
#define QMOE_EP_ID_BYTES 128
int qmoe_ep_unique_id(unsigned char id[QMOE_EP_ID_BYTES], qmoe_err *err);
int qmoe_ep_connect(qmoe_ctx *ctx, const unsigned char id[QMOE_EP_ID_BYTES], qmoe_err *err);
int qmoe_forward_ep(qmoe_ctx *ctx, int layer, const void *x_dev, int x_dtype, int n,
                    float *out_dev, void *stream, qmoe_err *err);
/* Host form of qmoe_forward_ep's dispatch plan, the same arithmetic as its
 * device kernels: for the routing idx [n, k] of one rank, counts[g] = tokens
 * sent to rank g (of W <= 64, E % W == 0: those with at least one expert in
 * [g E/W, (g+1) E/W)) and, if pos is not NULL, pos[g * n + t] = the send
 * row of token t for rank g, g * cap + t, or -1 when t is not sent there
 * (cap >= n: the rows per rank, max_tokens in qmoe_forward_ep). Returns 0,
 * or -1 on bad arguments. */
int qmoe_ep_plan_host(const int32_t *idx, int n, int k, int E, int W, int cap, int *counts,
                      int *pos);

/* Routing of the last forward call (waits for it): idx [n, k] in
 * (logit desc, expert asc) order, weights [n, k] (softmax renormalised over
 * the k, model.c:1305-1318), shared-gate sigmoid [n]. Any pointer may be NULL. */
int qmoe_last_routing(qmoe_ctx *ctx, int32_t *idx, float *weights,
                      float *shared_gate, qmoe_err *err);

/* ---- CUDA graphs of forward calls (no reference counterpart: the
 *      reference runs eagerly on the CPU) ----
 * qmoe_capture_begin starts capturing the qmoe_forward_dev calls issued on
 * `stream` (NULL = the context's stream) into a CUDA graph; qmoe_capture_end
 * instantiates it. Only contexts whose experts are all resident can be
 * captured (streaming forwards wait on the host). Replaying the graph with
 * qmoe_graph_launch reruns the captured calls with the same pointers. */
typedef struct qmoe_graph qmoe_graph;
int qmoe_capture_begin(qmoe_ctx *ctx, void *stream, qmoe_err *err);
qmoe_graph *qmoe_capture_end(qmoe_ctx *ctx, void *stream, qmoe_err *err);
int qmoe_graph_launch(qmoe_graph *g, void *stream, qmoe_err *err);
void qmoe_graph_free(qmoe_graph *g);

/* ---- diagnostics (no reference counterpart; the reference's qstats only
 *      time whole forwards, c/src/model.c:1756-1761) ----
 * Captures one forward of n tokens with CUDA events between its kernels,
 * replays it `reps` times and returns the mean device time of each kernel
 * launch in microseconds, in launch order (router, top-k, gate/up, down);
 * *kernels receives the count. Kernels run back to back without
 * programmatic overlap while profiled. Resident contexts only. */
int qmoe_profile_forward(qmoe_ctx *ctx, int layer, const void *x, int x_dtype,
                         int n, float *out, int reps, double *kernel_us,
                         int max_kernels, int *kernels, qmoe_err *err);

/* ---- expert cache hooks (cache.h:38-53 keyed (layer << 32) | expert,
 *      model.c:594) ---- */

/* Slot index of a resident expert or -1; no stats or recency (cache_peek). */
int qmoe_expert_peek(qmoe_ctx *ctx, int layer, int expert);
/* As peek, but counts a hit or miss and refreshes recency (cache_get). */
int qmoe_expert_get(qmoe_ctx *ctx, int layer, int expert);
/* Makes the listed experts resident, filling misses from the pinned host
 * store; returns when the copies are done (experts_load, model.c:539). */
int qmoe_experts_load(qmoe_ctx *ctx, int layer, const int64_t *ids, size_t n,
                      qmoe_err *err);
int qmoe_expert_pin(qmoe_ctx *ctx, int layer, int expert);
int qmoe_expert_unpin(qmoe_ctx *ctx, int layer, int expert);
int qmoe_expert_mark_hot(qmoe_ctx *ctx, int layer, int expert, int hot);
int qmoe_cache_snapshot(qmoe_ctx *ctx, qmoe_cache_stats *out);
int qmoe_stats_get(qmoe_ctx *ctx, qmoe_stats *out);

/* ---- prefetch hooks (streaming.py:271-284, :400-435) ---- */

/* Queues fills of the listed experts that are not in the pool on the copy
 * stream and returns at once (ExpertStore.request(prefetch=True) futures):
 * the copies wait, on the device, for the work already queued on the
 * context's own stream (a fill may evict a slot its kernels read; a caller
 * that runs forwards on a stream of its own synchronises that stream first,
 * or prefetches through qmoe_forward_stack, which orders them after its
 * stream), and the next forward's kernels wait for them. Prefetched experts
 * neither routed to nor evicted yet are capped at min(pool slots,
 * max(2, prefetch_depth x layers)) (ExpertStore._max_speculative,
 * streaming.py:115). Returns the number queued; 0 on a resident context. */
int qmoe_prefetch(qmoe_ctx *ctx, int layer, const int64_t *ids, size_t n);
/* Records one step's routing, every token's k experts (ExpertStore.record_route,
 * streaming.py:400-413, called with idx.reshape(-1) at model.py:458): the
 * context's predictor (qmoe_predictor_record) with the pool as the cache whose
 * hot marks it sets. */
void qmoe_record_route(qmoe_ctx *ctx, int layer, const int32_t *experts,
                       size_t n);
/* Predicts and queues prefetches (as qmoe_prefetch) for this layer and the
 * next from the route statistics (ExpertStore.prefetch_predictions,
 * streaming.py:415-435, called with the step's distinct experts in ascending
 * order at model.py:459). Returns the number queued. */
int qmoe_prefetch_predictions(qmoe_ctx *ctx, int layer,
                              const int32_t *selected, size_t n);

/* ---- host-side expert cache object (cache.c semantics over opaque values),
 *      usable without a GPU; the context's pool bookkeeping is built on it.
 *      Mirrors cache_init/put/get/peek/pin/unpin/mark_hot/snapshot,
 *      c/src/cache.h:38-60; values are 64-bit tokens (slot numbers). ---- */

typedef struct qmoe_cache qmoe_cache;
qmoe_cache *qmoe_cache_new(uint64_t max_bytes, int policy, int partitions);
void qmoe_cache_free(qmoe_cache *c);
/* returns 1 and stores the value on a hit, 0 on a miss */
int qmoe_cache_peek(qmoe_cache *c, uint64_t key, uint64_t *value);
int qmoe_cache_get(qmoe_cache *c, uint64_t key, uint64_t *value);
/* 1 when inserted. Each evicted value is appended to evicted[] (capacity
 * max_evicted, may be NULL) and counted in *n_evicted (may be NULL). */
int qmoe_cache_put(qmoe_cache *c, uint64_t key, uint64_t value,
                   uint64_t nbytes, int pin, int hot, uint64_t *evicted,
                   size_t max_evicted, size_t *n_evicted);
int qmoe_cache_pin(qmoe_cache *c, uint64_t key);
int qmoe_cache_unpin(qmoe_cache *c, uint64_t key);
int qmoe_cache_mark_hot(qmoe_cache *c, uint64_t key, int hot);
/* removes the entry; 1 if it existed */
int qmoe_cache_erase(qmoe_cache *c, uint64_t key, uint64_t *value);
qmoe_cache_stats qmoe_cache_stats_get(qmoe_cache *c);

/* ---- host-side route predictor (ExpertStore's route statistics,
 *      streaming.py:400-435 and :445-453), usable without a GPU; a streaming
 *      context owns one (qmoe_record_route / qmoe_prefetch_predictions).
 *      Rankings are Counter.most_common's: by count, ties to the key inserted
 *      first. Not internally locked. ---- */
typedef struct qmoe_predictor qmoe_predictor;
qmoe_predictor *qmoe_predictor_new(int num_layers, int num_experts);
void qmoe_predictor_free(qmoe_predictor *p);
/* One step's routed experts (all token assignments, duplicates counted):
 * transitions from the layer's previous selected set to this one, the routed
 * counts, the new selected set (its distinct experts, ascending, also
 * written to selected_out when not NULL, capacity num_experts), and, when
 * cache is not NULL, the hot mark of each selected key ((layer << 32) | e)
 * set to count >= 4. Returns the number selected, or -1 (nothing changed)
 * for an expert out of range. */
int qmoe_predictor_record(qmoe_predictor *p, qmoe_cache *cache, int layer,
                          const int32_t *experts, size_t n, int32_t *selected_out);
/* The predicted prefetches after a step of `layer` that selected
 * selected[0..n): up to depth experts of this layer (pick) and up to depth of
 * the next layer (next), each in rank order. depth <= 0 predicts nothing. */
int qmoe_predictor_predict(qmoe_predictor *p, int layer, const int32_t *selected, size_t n,
                           int depth, int64_t *pick, int *npick, int64_t *next, int *nnext);
uint64_t qmoe_predictor_count(const qmoe_predictor *p, int layer, int expert);
/* token assignments recorded (StreamStats.routes) */
uint64_t qmoe_predictor_routes(const qmoe_predictor *p);
/* the `want` most routed (layer, expert) pairs (snapshot's frequent_experts);
 * returns how many were written */
int qmoe_predictor_frequent(const qmoe_predictor *p, int want, int32_t *layer,
                            int32_t *expert, uint64_t *count);
/* The context's predictor (NULL on a resident context), for reading. */
const qmoe_predictor *qmoe_ctx_predictor(const qmoe_ctx *ctx);

/* ---- seeded synthetic layers (host; benchmark and test inputs) ----
 * Counter-based splitmix64 streams keyed by (seed, layer, tensor). Nibbles
 * uniform 0..15; scales bf16(|N(0, 0.02)|), biases bf16(-8 * scale); router
 * and shared gate bf16(N(0, 0.02)). Buffers are caller-owned, reference
 * layout, sized by qmoe_synth_sizes. */
typedef struct {
    size_t router, shared_gate;           /* bf16 elements */
    size_t expert_q, expert_sb;           /* per stacked gate/up tensor: words, bf16 */
    size_t down_q, down_sb;               /* stacked down tensor */
    size_t sh_q, sh_sb, sh_down_q, sh_down_sb;
} qmoe_synth_size;

int qmoe_synth_sizes(const qmoe_config *cfg, qmoe_synth_size *out);
/* Fills every non-NULL pointer of w (cast away const: the buffers are the
 * caller's). Experts [e0, e1) only are written when e1 > e0 (others untouched);
 * e0 = e1 = 0 writes all. */
int qmoe_synth_layer(const qmoe_config *cfg, uint64_t seed, int layer,
                     qmoe_layer_weights *w, int e0, int e1);
/* bf16(N(0,1)) activations as fp32 [n, d]; stream selects the token set. */
void qmoe_synth_tokens(uint64_t seed, uint64_t stream, int n, int d, float *x);
/* Zipf logit bias: bias[e] = -s * ln(1 + pi(e)) for a seeded permutation pi. */
void qmoe_synth_zipf_bias(uint64_t seed, int layer, int E, double s,
                          float *bias);
/* The same layer generated on the device straight into a context with every
 * local expert resident: its experts (the rank's share on an
 * expert-parallel context), shared expert, router, shared gate, and the Zipf
 * bias when zipf_s > 0. For stacks too large to build on the host (76 layers
 * of 512 experts: 68.9 GB). Nibble words equal the host streams bit for
 * bit; the normals use the device's log and cos, which may differ from the
 * host's in the last place, so a scale or router weight may differ from
 * qmoe_synth_layer's by one bf16 unit in rare elements. */
int qmoe_synth_layer_dev(qmoe_ctx *ctx, int layer, uint64_t seed, double zipf_s,
                         qmoe_err *err);

/* ---- checkpoint reader: safetensors files straight into the pools ----
 * The reference's storage layer on the MoE path (c/src/safetensors.h:1-76,
 * c/src/reader.c:11-112, src/colibri_runtime/storage.py:69-291): every
 * *.safetensors file of a directory is indexed at open, with the same
 * validation (header length, JSON, dtype, shape, offsets matching the size
 * and inside the file, no duplicate names, no overlapping ranges) and the
 * same name normalisation (a leading "language_model." is dropped; a lookup
 * of "model.x" also tries "language_model.model.x"). Reads are pread(2) on
 * io_workers threads. The index is read-only after open: reads may run
 * from several threads at once. */
typedef struct qmoe_ckpt qmoe_ckpt;

/* safetensors dtypes, in the order of st_dtype (c/src/safetensors.h:10-25) */
enum {
    QMOE_ST_BOOL, QMOE_ST_U8, QMOE_ST_I8, QMOE_ST_U16, QMOE_ST_I16, QMOE_ST_U32, QMOE_ST_I32,
    QMOE_ST_U64, QMOE_ST_I64, QMOE_ST_F16, QMOE_ST_BF16, QMOE_ST_F32, QMOE_ST_F64, QMOE_ST_COUNT
};

typedef struct {
    int dtype;         /* QMOE_ST_* */
    int ndim;
    int64_t shape[8];
    uint64_t nbytes;
    uint64_t row_bytes; /* nbytes / shape[0]; 0 for a scalar or empty tensor */
    int file;          /* index of its file, files in name order */
    uint64_t offset;   /* byte offset of its data in that file */
} qmoe_tensor_info;

/* I/O counters, as IOStats (storage.py:60-66) and st_index's counters
 * (c/src/safetensors.h:43-48): pread_calls counts system calls; bytes_read
 * the bytes those reads returned (a row read once however often it was
 * requested); rows_read the rows requested; tensors_read the whole tensors. */
typedef struct {
    uint64_t pread_calls, bytes_read, rows_read, tensors_read;
    double read_seconds;
} qmoe_io_stats;

/* st_index_open / st_index_close (c/src/safetensors.h:54-58) */
qmoe_ckpt *qmoe_ckpt_open(const char *dir, int io_workers, qmoe_err *err);
void qmoe_ckpt_close(qmoe_ckpt *ck);
/* tensors in name order (normalised names) */
size_t qmoe_ckpt_count(const qmoe_ckpt *ck);
const char *qmoe_ckpt_name(const qmoe_ckpt *ck, size_t i);
/* st_find (c/src/safetensors.h:60): 0 and *out, or -1 when absent */
int qmoe_ckpt_find(const qmoe_ckpt *ck, const char *name, qmoe_tensor_info *out);
/* st_read_tensor (c/src/safetensors.h:63): the whole tensor into out */
int qmoe_ckpt_read_tensor(qmoe_ckpt *ck, const char *name, void *out, size_t out_bytes,
                          qmoe_err *err);
/* st_read_rows (c/src/safetensors.h:67-68): rows of dimension 0 into out in
 * request order; repeated rows are read once; contiguous rows share a read */
int qmoe_ckpt_read_rows(qmoe_ckpt *ck, const char *name, const int64_t *rows, size_t n,
                        void *out, size_t out_bytes, qmoe_err *err);
int qmoe_ckpt_io_stats(const qmoe_ckpt *ck, qmoe_io_stats *out);

/* Bytes of the host buffer qmoe_ckpt_read_layer fills for one layer. */
size_t qmoe_ckpt_layer_bytes(const qmoe_config *cfg);
/* One MoE layer's tensors (model.layers.<layer>.mlp.{gate, shared_expert_gate,
 * switch_mlp.*, shared_expert.*}, c/src/model.c:1902-1923, :541-585) read
 * into buf and *w pointed at them, ready for qmoe_upload_layer. The router
 * and the shared gate must be dense BF16 (model.c:262-265), weights U32 and
 * scales/biases BF16 of the configured shapes; a missing biases tensor of the
 * shared expert reads as zeros (model.c:251-257). logit_bias is NULL. */
int qmoe_ckpt_read_layer(qmoe_ckpt *ck, const qmoe_config *cfg, int layer, void *buf,
                         size_t buf_bytes, qmoe_layer_weights *w, qmoe_err *err);
/* The rows of experts ids[0..n) of one layer (the nine rows experts_load
 * reads, c/src/model.c:603-629) packed into n consecutive slots of
 * qmoe_slot_bytes each, the layout of the HBM pool. */
int qmoe_ckpt_pack_experts(qmoe_ckpt *ck, const qmoe_config *cfg, int layer,
                           const int64_t *ids, size_t n, void *slots, size_t slots_bytes,
                           qmoe_err *err);
/* One expert of host weights packed into a slot (expert -1: the shared
 * expert); the packing qmoe_upload_layer does. */
int qmoe_pack_expert(const qmoe_config *cfg, const qmoe_layer_weights *w, int expert,
                     void *slot);
/* qmoe_ckpt_read_layer of checkpoint layer ckpt_layer, then
 * qmoe_upload_layer into the context's layer `layer`. */
int qmoe_upload_layer_ckpt(qmoe_ctx *ctx, int layer, qmoe_ckpt *ck, int ckpt_layer,
                           qmoe_err *err);

const char *qmoe_version(void);

#ifdef __cplusplus
}
#endif

#endif
