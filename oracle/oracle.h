/*
 * oracle.h - TEST INFRASTRUCTURE ONLY.
 *
 * CPU checkers for the MoE layer. Two implementations share this interface:
 *   - oracle_moe_forward (oracle/moe_oracle.c): a plain-C restatement of the
 *     reference runtime's MoE block, moe_forward in c/src/model.c:1281-1405;
 *   - ref_moe_forward (oracle/ref_harness.c, built into oracle/_ref/): the
 *     reference's own moe_forward compiled unmodified from its sources.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may call these. The product library never links them.
 *
 * Tensor layout is the reference checkpoint layout for one layer
 * (c/src/model.c:555-557 for the routed experts, :1902-1923 for the router,
 * shared expert and shared gate): q4 words u32 with 8 nibbles each, low nibble
 * first; scales and biases bf16, one per group of `g` values along the row.
 */
#ifndef QMOE_ORACLE_H
#define QMOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

typedef struct {
    int d;  /* hidden_size */
    int E;  /* num_experts */
    int k;  /* num_experts_per_tok */
    int I;  /* moe_intermediate_size (routed and shared, c/src/model.c:1391-1392) */
    int g;  /* quantization group size */
    const uint16_t *router;      /* bf16 [E, d]  mlp.gate.weight */
    const uint16_t *shared_gate; /* bf16 [d]     mlp.shared_expert_gate.weight */
    const float *logit_bias;     /* fp32 [E] added to router logits, or NULL */
    /* switch_mlp experts: gate/up [E, I, d/8] words, [E, I, d/g] scales/biases;
       down [E, d, I/8] words, [E, d, I/g] scales/biases */
    const uint32_t *gq, *uq, *dq;
    const uint16_t *gs, *gb, *us, *ub, *ds, *db;
    /* shared expert: gate/up [I, d/8], [I, d/g]; down [d, I/8], [d, I/g] */
    const uint32_t *sgq, *suq, *sdq;
    const uint16_t *sgs, *sgb, *sus, *sub, *sds, *sdb;
} oracle_layer;

/* Restatement (moe_oracle.c). out: fp32 [n, d], overwritten. idx/wts
 * (optional, [n, k]) receive the routing in (value desc, index asc) order.
 * logits (optional, [n, E]) receives the biased router logits. */
int oracle_moe_forward(const oracle_layer *L, const float *x, int n,
                       float *out, int32_t *idx, float *wts, float *logits);

/* Router + top-k + renormalised softmax only (model.c:1301-1319). */
int oracle_route(const oracle_layer *L, const float *x, int n, int32_t *idx,
                 float *wts, float *logits);

/* Canonical router dot product: see moe_oracle.c. */
float oracle_router_dot(const float *x, const uint16_t *w, int K);

/* The MoE side's hyper connection of one layer (mlp_hyper_connection.*,
 * c/src/model.c:1945-1964; the checkpoint's hc_count streams of d values).
 * The two mixer weights are q4 when their words are given (u32 [rows,
 * cols/8], bf16 scales/biases [rows, cols/64], biases may be NULL = zeros),
 * else dense bf16 [rows, cols] (mw_load, model.c:215-266). */
typedef struct {
    int d, hc, lowrank;
    const float *norm;           /* fp32 [hc*d]   hc_norm.weight (model.c:1946) */
    const uint32_t *down_q;      /* input_mix_weight_down [lowrank, hc*d] */
    const uint16_t *down_s, *down_b, *down_bf16;
    const uint32_t *up_q;        /* input_mix_weight_up   [hc*d, lowrank] */
    const uint16_t *up_s, *up_b, *up_bf16;
    const uint16_t *inject;      /* bf16 [hc, hc*d] block_inject_weight */
} oracle_hc;

/* gated_residual restated (model.c:728-796): h fp32 [n, hc*d] -> mixed
 * [n, d] and, when inject is not NULL, inject [n, hc]. */
int oracle_gated_residual(const oracle_hc *H, const float *h, int n, float *mixed,
                          float *inject);
/* One layer's MoE step with its hyper connection (model.c:1708-1731):
 * gated_residual, moe_forward of the mixed rows, then
 * h[t, c, :] += inject[t, c] * moe[t, :]. h is updated in place. */
int oracle_hc_moe_step(const oracle_hc *H, const oracle_layer *L, float *h, int n);
/* The same two through the reference's own code (ref_harness.c). */
int ref_gated_residual(const oracle_hc *H, const float *h, int n, float *mixed, float *inject);
int ref_hc_moe_step(const oracle_hc *H, const oracle_layer *L, float *h, int n);

/* The reference's safetensors index and row reader (ref_harness.c, oracle/_ref
 * only): st_index_open / st_find / st_read_rows behind opaque handles. */
void *ref_st_open(const char *dir, int workers, char *msg, int msgcap);
void ref_st_close(void *h);
int ref_st_count(void *h);
const char *ref_st_name(void *h, int i);
int ref_st_info(void *h, const char *name, int *dtype, int *ndim, int64_t *shape,
                uint64_t *offset, uint64_t *nbytes);
int ref_st_read_rows(void *h, const char *name, const int64_t *rows, size_t n, void *out);
uint64_t ref_st_rows_read(void *h);

/* Known-answer helper: kernel_dequant_q4 restated (c/src/kernel.c:152-173). */
void oracle_dequant_q4(const uint32_t *q, const float *scales,
                       const float *biases, int rows, int cols, int group,
                       float *out);

/* The reference compiled unmodified (ref_harness.c, oracle/_ref only). The
 * harness reports the reference's selection order in idx (unspecified within
 * the k, c/src/kernel.h:44-46). threads: BLAS threads for cblas_sgemm. */
int ref_moe_forward(const oracle_layer *L, const float *x, int n, float *out,
                    int32_t *idx, float *wts);
void ref_set_threads(int threads);
/* Drops the harness's dequantised expert cache (fp32, 12*d*I bytes each). */
void ref_reset_cache(void);

/* The seeded synthetic workload (synth_oracle.c): writes the tensors L points
 * at (the pointers are written through although declared const), for experts
 * [e0, e1) of the routed tensors (e1 <= e0: all), the router, shared gate and
 * shared expert. Buffers hold all E experts. Returns 0, or -1 on a bad shape. */
int oracle_synth_layer(oracle_layer *L, uint64_t seed, int layer, int e0, int e1);
void oracle_synth_tokens(uint64_t seed, uint64_t stream, int n, int d, float *x);
int oracle_synth_zipf_bias(uint64_t seed, int layer, int E, double s, float *bias);
/* Unit-weight RMSNorm of n rows of d (sum of squares in fp64). */
void oracle_rmsnorm_rows(const float *x, int n, int d, float eps, float *y);

#endif
