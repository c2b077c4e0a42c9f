/*
 * qmoe_internal.h - layouts and kernel launchers shared by the host C code
 * and the CUDA translation units. Not part of the public ABI.
 */
#ifndef QMOE_INTERNAL_H
#define QMOE_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Expert slot layout in HBM (one routed expert, or the shared expert):
 *
 *   GU section, I rows of gu_row bytes; h-row n holds
 *     [ gate q: d/2 bytes ][ up q: d/2 bytes ][ d/g quads (gs, gb, us, ub) bf16 ]
 *   D section, d rows of d_row bytes; output row n holds
 *     [ down q: I/2 bytes ][ I/g pairs (ds, db) bf16 ][ pad to 16 bytes ]
 *
 * Nibble order inside the q bytes is the checkpoint's (low nibble first,
 * c/src/kernel.c:163-166), so a row's q bytes are the checkpoint row verbatim.
 * Gate and up rows of the same h-row sit side by side so one contiguous read
 * feeds SiLU(gate) * up, and scales ride with their row.
 */
typedef struct {
    int d, E, k, I, g;
    int gu_row;        /* bytes per GU row */
    int d_row;         /* bytes per D row (16-byte multiple) */
    size_t gu_bytes;   /* I * gu_row */
    size_t slot_bytes; /* gu_bytes + d * d_row, rounded up to 256 */
} qk_layout;

int qk_layout_init(qk_layout *L, int d, int E, int k, int I, int g);

/* Host-side repack of one expert from checkpoint layout into a slot. */
void qk_pack_expert(const qk_layout *L, const uint32_t *gq, const uint16_t *gs,
                    const uint16_t *gb, const uint32_t *uq, const uint16_t *us,
                    const uint16_t *ub, const uint32_t *dq, const uint16_t *ds,
                    const uint16_t *db, uint8_t *slot);

/* Device error word bits (set by kernels, read by the host after a sync). */
enum {
    QK_ERR_TIMEOUT_COPY = 1,  /* bulk-copy completion wait gave up */
    QK_ERR_NOT_RESIDENT = 2,  /* a routed expert had no HBM slot */
    QK_ERR_BAD_ROUTE = 4,     /* top-k found fewer than k finite logits */
    QK_ERR_TIMEOUT_GRID = 8,  /* grid barrier or cross-CTA exchange wait gave up */
};

/* Everything one forward call needs on the device. */
typedef struct {
    qk_layout L;
    int T;                       /* tokens */
    const void *x;               /* [T, d] fp32 or bf16 */
    int x_bf16;
    const uint16_t *router;      /* [E, d] bf16 */
    const uint16_t *shared_gate; /* [d] bf16 */
    const float *logit_bias;     /* [E] or NULL */
    const uint8_t *pool;         /* slot 0 of the HBM pool */
    const int32_t *slot_of;      /* [E] slot of each expert of this layer, -1 absent */
    const uint8_t *shared_slot;  /* the shared expert, slot layout */
    float *logits;               /* [T, E + 1]; column E is the shared-gate logit */
    int32_t *idx;                /* [T, k] */
    float *wts;                  /* [T, k] */
    float *sgate;                /* [T] sigmoid(shared-gate logit) */
    float *h;                    /* [T, k + 1, I] */
    float *out;                  /* [T, d] */
    int *err;                    /* device error word */
    int num_sms;
    unsigned long long *ptimes;  /* diagnostics: per-CTA phase timestamps
                                    [grid][32] (%globaltimer ns), or NULL */
    /* the hyper connection's inject-add in the decode kernel's combine
     * (T = 1): hc_h[c, :] += hc_inj[c] * out for c < hc_n; hc_h NULL: none */
    float *hc_h;
    float *hc_inj;
    int hc_n;
    /* hc_pre: the decode kernel also computes gated_residual from hc_h
     * first (its prologue, two more grid barriers, a counter of its own):
     * the inject weights into hc_inj, the low-rank w into hc_w and the block
     * input into x (= hc_mixed, fp32). The layer's device weights: */
    int hc_pre, hc_lr;
    const float *hc_norm;
    const uint32_t *hc_down_q, *hc_up_q;
    const uint16_t *hc_down_s, *hc_down_b, *hc_down_bf, *hc_up_s, *hc_up_b, *hc_up_bf, *hc_inject;
    float *hc_w, *hc_mixed;
} qk_fwd;

/* Kernel launchers (qmoe_kernels.cu). Each returns a cudaError_t as int.
 * stream is a cudaStream_t. pdl != 0 launches with programmatic stream
 * serialization so the kernel's prologue overlaps its predecessor. */
/* One-time per-device kernel attributes (dynamic shared memory limits), so
 * launches never call cudaFuncSetAttribute (safe under stream capture). */
int qk_prepare_kernels(void);
int qk_launch_router(const qk_fwd *f, void *stream, int pdl);
int qk_launch_topk(const qk_fwd *f, void *stream, int pdl);
int qk_launch_decode_gateup(const qk_fwd *f, void *stream, int pdl);
int qk_launch_decode_down(const qk_fwd *f, void *stream, int pdl);

/* Host-pointer single-token calls: copy `bytes` (a multiple of 16) of x from
 * pinned host memory to the device with one CTA that lets its dependents
 * launch at once; after the layer, a dependent launch copies the error word
 * to pinned host memory and, when ctr is not NULL, increments the device
 * counter ctr and writes its new value to ctr_host (pinned). */
int qk_launch_copy_in(const void *src_host, void *dst, size_t bytes, void *stream);
int qk_launch_report(const int *err, int *err_host, unsigned *ctr, unsigned *ctr_host,
                     void *stream);

/* Single-launch decode (T == 1): router, top-k, gate/up and down+combine in
 * one persistent kernel with one CTA per SM and grid barriers between the
 * phases. sync: qk_decode_sync_bytes(L) bytes of device memory owned by the
 * caller (the grid-barrier counter, then the logits and h the CTAs
 * exchange), zeroed before the first launch and again after a launch that
 * reported an error; successive launches on it must be stream-ordered.
 * Only idx, wts, sgate and out of f are written (not logits or h).
 * Returns QK_FUSED_UNFIT (no launch) when the shape's per-CTA working set does
 * not fit in shared memory; the caller then uses the four-kernel path. */
#define QK_FUSED_UNFIT (-7)
size_t qk_decode_sync_bytes(const qk_layout *L);
int qk_launch_decode_fused(const qk_fwd *f, void *sync, void *stream, int pdl);

/* Prefill / multi-token path (qmoe_prefill.cu): tokens grouped by expert, a
 * tcgen05 grouped GEMM for gate/up (SiLU x up epilogue) and for down, and a
 * gather-combine. The plan owns its workspaces (sized for max_tokens) and
 * the TMA descriptors over the pool; created once per context. */
typedef struct qk_prefill qk_prefill;
/* pool: base of pool_slots slots (routed slots and one shared slot per layer) */
qk_prefill *qk_prefill_create(const qk_layout *L, int max_tokens, const uint8_t *pool,
                              int pool_slots, int num_sms, char *msg, size_t msg_len);
void qk_prefill_destroy(qk_prefill *p);
/* Runs everything after routing (f->idx, f->wts, f->sgate must be ready in
 * stream order); shared_slot_index: the pool slot of this layer's shared
 * expert. events: NULL, or 4 cudaEvent_t recorded after grouping+gather,
 * gate/up GEMM, down GEMM and combine (diagnostics). */
int qk_launch_prefill(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream,
                      void **events);
/* The same pass in waves, for a call whose distinct experts exceed the pool:
 * qk_prefill_plan groups and gathers every row once (as qk_launch_prefill);
 * then per wave the caller fills the wave's experts, writes the wave's
 * expert mask (qk_prefill_wave_mask: [E + 1] bytes on the device, index 0
 * the shared expert, e + 1 expert e) and calls qk_prefill_wave, which runs
 * the two GEMMs over that wave's tiles only (each output row is written by
 * exactly one wave, at the row the plan gave it); qk_prefill_combine then
 * combines every row once, in the fixed order of qk_launch_prefill, so the
 * result is the one-pass result bit for bit. */
int qk_prefill_plan(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream);
uint8_t *qk_prefill_wave_mask(qk_prefill *p);
int qk_prefill_wave(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream);
int qk_prefill_combine(qk_prefill *p, const qk_fwd *f, void *stream);

/* Routing of a multi-token call on the tensor cores (approximate logits)
 * with an exact re-ranking of each token's candidates: writes f->idx, f->wts
 * and f->sgate, identical to qk_launch_router + qk_launch_topk (f->logits is
 * not written). wmax: max over experts of the router row's 2-norm, rounded
 * up. mid_event: NULL, or a cudaEvent_t recorded between the two halves.
 * Returns QK_ROUTE_UNFIT (no launch) when the plan does not cover the shape. */
#define QK_ROUTE_UNFIT (-8)
int qk_launch_route(qk_prefill *p, const qk_fwd *f, float wmax, void *stream, void *mid_event);

/* The MoE side's hyper connection (qmoe_hc.cu), device copies of one layer's
 * weights: gated_residual before the block, the inject-add after it. */
typedef struct {
    int d, hc, lowrank;
    float *norm;                          /* [hc*d] */
    uint32_t *down_q;                     /* [lowrank, hc*d/8] or NULL: down_bf */
    uint16_t *down_s, *down_b, *down_bf;  /* [lowrank, hc*d/64] (b may be NULL), [lowrank, hc*d] */
    uint32_t *up_q;                       /* [hc*d, lowrank/8] or NULL: up_bf */
    uint16_t *up_s, *up_b, *up_bf;        /* [hc*d, lowrank/64] (b may be NULL), [hc*d, lowrank] */
    uint16_t *inject;                     /* [hc, hc*d] */
} qk_hc_dev;
int qk_hc_smem_ok(int d, int hc);
int qk_hc_prepare(int d, int hc);
/* gated_residual of n tokens h [n, hc*d]: mixed [n, d] (the block's input),
 * INJ [n, hc]; W [n, lowrank] and R [n, hc] are its workspaces. One token
 * takes a single launch of num_sms CTAs with a grid barrier on the zeroed,
 * only-growing counter ctr (timeouts set QK_ERR_TIMEOUT_GRID in err); more
 * tokens take two launches. */
int qk_launch_hc_pre(const qk_hc_dev *w, const float *h, int n, float *W, float *R, float *INJ,
                     float *mixed, unsigned long long *ctr, int *err, int num_sms, void *stream);
/* h[t, c, :] += INJ[t, c] * y[t, :] */
int qk_launch_hc_inject(float *h, const float *INJ, const float *y, int n, int hc, int d,
                        void *stream);

/* Expert parallelism (qmoe_prefill.cu). Rank g of G owns experts
 * [g E/G, (g+1) E/G). A token travels once to every rank that owns one of
 * its experts (x as given, bf16 or fp32, plus its k slots, other ranks' slots
 * as expert id -1),
 * that rank combines its slots' outputs with the routing weights, and one
 * fp32 partial row per (token, rank) comes back. Transfers have a fixed
 * size: cap rows (the plan's tokens per rank) between every pair of ranks,
 * token t in row t of its destination's block, so nothing waits for counts
 * on the host and a whole call can be captured in a graph; rows of tokens
 * not bound for a rank carry only expert ids -1.
 *   qk_ep_alloc     buffers for cap tokens per rank and G ranks
 *   qk_ep_dispatch  after routing: the G cap send rows (rank-major) and the
 *                   own tokens as the leading rows of the receive buffer
 *   qk_ep_experts   one grouped pass: the own T tokens through the shared
 *                   expert, the G cap received rows (after the own tokens)
 *                   through this rank's experts, then the expert-side combine
 *                   into one partial row each
 *   qk_ep_finish    the sum of the returned partials (rank order) and the
 *                   shared expert into out
 * The transfers between them are the caller's (NCCL send/recv on the
 * buffers of qk_ep_buffers), or the peer-memory path below. The receive
 * buffer holds the own tokens in rows [0, cap) and rank g's rows from
 * cap + g cap on. */
typedef struct {
    void *send_x, *recv_x;       /* [rows, d] x as given: bf16 or fp32 (same on every rank) */
    int32_t *send_e, *recv_e;    /* [rows, k] */
    float *send_w, *recv_w;      /* [rows, k] */
    float *ret, *back;           /* fp32 [G cap, d]: partials in received order / send order */
} qk_ep_bufs;
int qk_ep_alloc(qk_prefill *p, int cap, int G);
/* Peer-memory exchange instead of the caller's transfers (every pair of
 * ranks with peer access, one process per GPU): each rank's receive rows,
 * return rows and flags mapped into every rank through CUDA IPC.
 *   qk_ep_ipc_handles   the 5 handles of this rank (5 x 64 bytes)
 *   qk_ep_p2p_open      maps every rank's handles (all: G x 5 x 64 bytes)
 *   qk_ep_dispatch_p2p  the dispatch written into the destinations' receive
 *                       rows, then the destinations' flags raised
 *   qk_ep_wait          waits (bounded) for every rank's flag `which`
 *                       (0: dispatch, 1: return; the return wait ends the call)
 *   qk_ep_experts_p2p   qk_ep_experts with each partial row written into its
 *                       owner's return row, then the owners' flags raised */
int qk_ep_ipc_handles(qk_prefill *p, unsigned char *out);
int qk_ep_p2p_open(qk_prefill *p, const unsigned char *all, int rank);
void qk_ep_p2p_close(qk_prefill *p);
int qk_ep_dispatch_p2p(qk_prefill *p, const qk_fwd *f, int rank, void *stream);
int qk_ep_wait(qk_prefill *p, int which, int *err, void *stream);
int qk_ep_experts_p2p(qk_prefill *p, const qk_fwd *f, int shared_slot_index, int rank, void *stream);
void qk_ep_buffers(qk_prefill *p, qk_ep_bufs *b);
int qk_ep_dispatch(qk_prefill *p, const qk_fwd *f, void *stream);
int qk_ep_experts(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream);
int qk_ep_finish(qk_prefill *p, const qk_fwd *f, void *stream);

/* Seeded synthetic weights (qmoe_synth.c on the host, qmoe_synth_dev.cu on
 * the device). Stream of tensor `tensor` of layer `layer`: a splitmix64
 * counter sequence keyed by qk_stream_key. */
enum {
    QK_T_ROUTER = 0, QK_T_SHGATE, QK_T_GQ, QK_T_GS, QK_T_UQ, QK_T_US, QK_T_DQ, QK_T_DS,
    QK_T_SGQ, QK_T_SGS, QK_T_SUQ, QK_T_SUS, QK_T_SDQ, QK_T_SDS, QK_T_PERM = 20
};
uint64_t qk_stream_key(uint64_t seed, uint64_t layer, uint64_t tensor);
/* One expert straight into its slot: keys = the streams of gate q, gate
 * scales, up q, up scales, down q, down scales; e = the expert's index in
 * those (stacked) streams, 0 for the shared expert. */
int qk_synth_slot(const qk_layout *L, uint8_t *slot, int e, const uint64_t keys[6], void *stream);
/* bf16(N(0, 1) * 0.02) for elements [0, n) of a stream */
int qk_synth_bf16_normal(uint16_t *out, size_t n, uint64_t key, void *stream);

/* Residual stream of the MoE-only stack (qmoe_stack.cu), h fp32 [n, d]:
 * y != NULL: h += y; xn != NULL: xn = RMSNorm(h) (unit weight, eps). */
int qk_launch_residual_norm(float *h, const float *y, float *xn, int n, int d, float eps,
                            void *stream);

/* internal cache helper: replace the value of an existing key */
struct qmoe_cache;
int qmoe__cache_set_value(struct qmoe_cache *c, uint64_t key, uint64_t value);

#ifdef __cplusplus
}
#endif

#endif
