// qmoe_decode_fused.cu - one-launch MoE layer for a single decode token.
//
// The whole of moe_forward (c/src/model.c:1281-1405) for T == 1 in one
// persistent kernel: one CTA of 16 warps per SM, three phases split by grid
// barriers (one arrive per CTA, fire-and-forget, and one polling thread).
//
//   prologue  bulk-copy what does not depend on routing into shared memory:
//             this CTA's router rows (mlp.gate plus the shared-gate row), its
//             rows of the shared expert (gate/up and down) and the layer's
//             expert -> slot table. Issued before griddepcontrol.wait.
//   phase 1   x -> fp64 in shared memory; router rows -> logits; while the
//             grid barrier is pending, x -> 16-bit integers (quant_word) for
//             the experts.                                     [grid barrier]
//   phase 2   every CTA takes all logits as order keys and computes the same
//             exact top-k (block-wide threshold, then one warp ranks the
//             candidates), looks the k experts up in the staged slot table
//             and issues its share of their gate/up rows (in chunks of <= 16
//             rows, one mbarrier each) and of their down rows (all k experts
//             at once). Meanwhile the warps that do not share warp 0's
//             scheduler compute the shared expert's gate/up rows. Then all
//             warps compute the routed gate/up rows
//             chunk by chunk as they land -> h.              [grid barrier]
//   phase 3   h -> 24-bit integers in shared memory (every h load of a
//             thread issued before it quantizes); this CTA's output rows with
//             one warp per expert: the expert's h units stay in registers
//             while the warp walks the rows, one partial per row step in
//             registers, the row reductions (shuffles) batched at the end;
//             per-expert partials are combined in a fixed expert order with
//             the routing weights and the shared gate; each output written
//             once.
//
// With f.hc_pre (the hyper connection around the block, one token) the
// kernel first computes gated_residual: every CTA stages the normed hc
// streams (each stream's RMS in fp64) in its routed gate/up area, which is
// idle until phase 2; CTA r < lowrank computes down-mixer row r (16 warps
// over word ranges for q4, the canonical order's eight per-lane sums for
// bf16), the next hc CTAs the inject weights; [grid barrier] every CTA then
// computes the up-mixer rows and the stream mean of its d / G columns into
// f.x; [grid barrier] phase 1 reads x from there. The combine adds inject x
// output to every stream. These launches count four barriers and use a
// counter of their own.
//
// The q4 products are the integer dot products of qmoe_dev.cuh (quant_word,
// dot_unit_q): four dp4a per q4 word for x, six for h. The router dot keeps
// the canonical fp64 order (router_lane) with x staged once as doubles.
//
// Per CTA at d=2048, E=512, k=10, I=512 on 148 SMs: 16 KB router, 9 KB shared
// gate/up, 81 KB routed gate/up, 44 KB down rows, so every byte the CTA needs
// for the token is requested at once. Dependents are triggered only after the
// second grid barrier, when every CTA of this grid is resident, so a waiting
// next launch can never take an SM this grid still needs.

#include "qmoe_dev.cuh"

using namespace qk;

cudaError_t qk_launch_raw(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream,
                          int pdl, void **args);

namespace {

constexpr int kThreads = 512;   // 16 warps, one CTA per SM
constexpr int kWarps = kThreads / 32;
constexpr int kChunkRows = 16;  // routed gate/up rows per bulk copy / mbarrier (one per warp)
constexpr int kMaxChunks = 12;  // chunks per CTA (checked by make_plan)
constexpr int kXB = 2;          // byte planes of x
constexpr int kHB = 3;          // byte planes of h
constexpr int kSyncWords = 32;  // 64-bit words before the exchange area
constexpr int kHW = 2;          // h words (8 values) quantized per thread in phase 3
constexpr int kRowSteps = 8;    // phase 3: output row steps per expert warp (checked by make_plan)

struct Plan {
    int G;       // CTAs, one per SM
    int rr_max;  // router rows per CTA (of E + 1)
    int sr_max;  // shared gate/up rows per CTA (of I)
    int gr_max;  // routed gate/up rows per CTA (of k * I)
    int or_max;  // output rows per CTA (of d)
    int off_router, off_sgu, off_rgu, off_down, off_xq, off_x, total;
};

__device__ __forceinline__ int part(int c, int n, int G) { return (c * n) / G; }

// x (bf16 or fp32) word t: elements 8t .. 8t + 7
template <bool HC>
__device__ __forceinline__ void load_x_word(const qk_fwd &f, int t, float (&v)[8]) {
    if (f.x_bf16) {
        const uint4 w = reinterpret_cast<const uint4 *>(f.x)[t];
        v[0] = bf16lo(w.x); v[1] = bf16hi(w.x); v[2] = bf16lo(w.y); v[3] = bf16hi(w.y);
        v[4] = bf16lo(w.z); v[5] = bf16hi(w.z); v[6] = bf16lo(w.w); v[7] = bf16hi(w.w);
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(f.x) + 2 * t;
        // written by this launch's CTAs (hc_pre): past L1
        const float4 a = HC ? __ldcg(p) : p[0], b = HC ? __ldcg(p + 1) : p[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

constexpr int kHcVals = 16;  // hc_pre: h values per thread (hc*d <= 16 * kThreads, d % kThreads == 0)

// Up-mixer row `row` (lowrank 64, one q4 group: the words and the group's
// scale and bias already in registers) times w: the arithmetic of
// qmoe_hc.cu's up_row for one group.
__device__ __forceinline__ float hc_up1(uint4 qa, uint4 qb, float sg, float bg, bool has_b,
                                        const float *s_w) {
    const uint32_t uw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    float xq = 0.f, xs = 0.f;
    for (int i2 = 0; i2 < 64; ++i2) xs += s_w[i2];
#pragma unroll
    for (int wd = 0; wd < 8; ++wd)
#pragma unroll
        for (int bb = 0; bb < 8; ++bb)
            xq = fmaf(s_w[8 * wd + bb], static_cast<float>((uw[wd] >> (4 * bb)) & 0xFu), xq);
    float u = fmaf(sg, xq, 0.f);
    if (has_b) u = fmaf(bg, xs, u);
    return u;
}

// One h-row of gate/up from a staged slot row: h = SiLU(gate . x) * (up . x).
// Lane l owns the 32-element units l, l + 32, ... of x (UPL of them).
template <int UPL>
__device__ __forceinline__ float gateup_row(const uint8_t *row, const qk_layout &L,
                                            const uint2 (&xw)[UPL][kXB][4], const float (&xsc)[UPL],
                                            const float (&xsm)[UPL], int lane) {
    const int nunits = L.d / 32, half = L.d / 2;
    float pg = 0.f, pu = 0.f;
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        if (u < nunits) {
            const uint4 gw = *reinterpret_cast<const uint4 *>(row + 16 * u);
            const uint4 uw = *reinterpret_cast<const uint4 *>(row + half + 16 * u);
            const uint2 sb = *reinterpret_cast<const uint2 *>(row + L.d + 8 * ((32 * u) / L.g));
            const float ag = dot_unit_q<kXB>(gw, xw[i]) * xsc[i];
            const float au = dot_unit_q<kXB>(uw, xw[i]) * xsc[i];
            pg += fmaf(bf16lo(sb.x), ag, bf16hi(sb.x) * xsm[i]);
            pu += fmaf(bf16lo(sb.y), au, bf16hi(sb.y) * xsm[i]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        pg += __shfl_xor_sync(QK_FULL, pg, off);
        pu += __shfl_xor_sync(QK_FULL, pu, off);
    }
    return (pg / (1.0f + expf(-pg))) * pu;
}

template <int UPL, int LPR, bool HC>
__global__ void __launch_bounds__(kThreads, 1) k_decode_fused(qk_fwd f, Plan p,
                                                              unsigned long long *sync) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[2 + kMaxChunks];  // 0: prologue, 1: down rows, 2..: chunks
    __shared__ uint64_t s_hcbar;              // hc_pre: the down-mixer row or inject stream
    __shared__ int s_ok;
    __shared__ int s_chunk0[kMaxChunks + 1];  // first routed row (CTA-local) of each chunk
    __shared__ int s_nchunks;
    __shared__ uint32_t s_key[32];
    __shared__ int s_idx[32];
    __shared__ float s_ev[32];
    __shared__ int r_idx[32];
    __shared__ float r_w[33];
    __shared__ float s_gl;
    __shared__ uint32_t s_wmax[kWarps];
    __shared__ int s_cnt;
    __shared__ unsigned long long s_base;
    __shared__ double s_rpart[kWarps][32];  // router: per-warp partial sums
    __shared__ const uint8_t *s_slotp[32];  // slot of each routed expert
    __shared__ __align__(16) int32_t s_slots[1024];  // this layer's expert -> slot table
    __shared__ uint32_t s_keys[1024];                // staged top-k keys

    const qk_layout &L = f.L;
    const int c = blockIdx.x, G = p.G;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int d = L.d, E = L.E, k = L.k, I = L.I, S = k + 1;
    const int rr0 = part(c, E + 1, G), rr1 = part(c + 1, E + 1, G);
    const int sr0 = part(c, I, G), sr1 = part(c + 1, I, G);
    const int gr0 = part(c, k * I, G), gr1 = part(c + 1, k * I, G);
    const int or0 = part(c, d, G), or1 = part(c + 1, d, G);
    const int xwn = d / 8;  // words of x
    uint8_t *sm_router = smem + p.off_router;
    uint8_t *sm_sgu = smem + p.off_sgu;
    uint8_t *sm_rgu = smem + p.off_rgu;
    uint8_t *sm_down = smem + p.off_down;
    uint2 *xq = reinterpret_cast<uint2 *>(smem + p.off_xq);   // kXB planes of d / 8 words
    float *xusc = reinterpret_cast<float *>(xq + kXB * xwn);  // [d / 32] unit scales
    float *xusm = xusc + d / 32;                              // [d / 32] unit sums
    double2 *rx = reinterpret_cast<double2 *>(smem + p.off_x);  // x staged for the router

    // diagnostics: phase timestamps of this CTA (thread 0, %globaltimer),
    // kept in shared memory and written out when the CTA ends, so the probe
    // adds no global stores along the way
    __shared__ unsigned long long s_stamp[32];
#define STAMP(i)                                   \
    do {                                           \
        if (f.ptimes && tid == 0) s_stamp[(i)] = gtimer(); \
    } while (0)
    if (f.ptimes && tid < 32) s_stamp[tid] = 0ull;
    STAMP(0);
    if (f.ptimes && tid == 0) s_stamp[30] = clock64();
    const uint32_t b_router = static_cast<uint32_t>((rr1 - rr0) * d * 2);
    const uint32_t b_sgu = static_cast<uint32_t>((sr1 - sr0) * L.gu_row);
    const uint32_t b_sdown = static_cast<uint32_t>((or1 - or0) * L.d_row);
    const uint32_t b_slots = static_cast<uint32_t>(E * 4);
    if (tid < 2 + kMaxChunks) mbar_init(&bar[tid], 1);
    if (tid == kThreads - 1) mbar_init(&s_hcbar, 1);
    // the prologue barrier's byte count before any of its copies is issued
    if (tid == 0) mbar_expect_tx(&bar[0], b_router + b_sgu + b_sdown + b_slots);
    __syncthreads();

    // ---- prologue: what does not depend on routing. Five bulk copies, each
    // issued by lane 0 of its own warp among the last six (a TMA issue costs
    // ~0.1 us; the warps issue in parallel), while the sixth plans the routed
    // gate/up chunks; the first warps, which stage x, go straight on to it.
    {
        const int re = min(rr1, E);
        const int q = warp - (kWarps - 6);  // 0..5 for the last six warps
        if (q == 0 && lane == 0) {
            if (re > rr0)
                bulk_load(sm_router, f.router + static_cast<size_t>(rr0) * d,
                          static_cast<uint32_t>((re - rr0) * d * 2), &bar[0]);
        } else if (q == 1 && lane == 0) {
            if (rr1 > E)
                bulk_load(sm_router + static_cast<size_t>(E - rr0) * d * 2, f.shared_gate,
                          static_cast<uint32_t>(d * 2), &bar[0]);
        } else if (q == 2 && lane == 0) {
            bulk_load(s_slots, f.slot_of, b_slots, &bar[0]);
        } else if (q == 3 && lane == 0) {
            if (sr1 > sr0)
                bulk_load(sm_sgu, f.shared_slot + static_cast<size_t>(sr0) * L.gu_row, b_sgu, &bar[0]);
        } else if (q == 4 && lane == 0) {
            if (or1 > or0)
                bulk_load(sm_down + static_cast<size_t>(k) * p.or_max * L.d_row,
                          f.shared_slot + L.gu_bytes + static_cast<size_t>(or0) * L.d_row, b_sdown,
                          &bar[0]);
        } else if (q == 5 && lane == 0) {
            // routed gate/up chunk boundaries: runs within one expert, <= 16 rows
            int n = 0, r = gr0;
            while (r < gr1 && n < kMaxChunks) {
                const int end = min(min(gr1, (r / I + 1) * I), r + kChunkRows);
                s_chunk0[n++] = r - gr0;
                r = end;
            }
            s_chunk0[n] = gr1 - gr0;
            s_nchunks = n;
        }
    }
    // hc_pre: this CTA's down-mixer row or inject stream into shared memory
    // (after the normed streams), and the up-mixer words of its columns into
    // registers, before waiting for the previous kernel
    const int hd = HC ? f.hc_n * d : 0;
    float *hc_x = reinterpret_cast<float *>(sm_rgu);  // [hd] normed streams
    uint8_t *hc_row = sm_rgu + static_cast<size_t>(hd) * 4;
    const bool hc_q4 = HC && c < f.hc_lr && f.hc_down_q;
    const bool hc_canon = HC && !hc_q4 && c < f.hc_lr + f.hc_n;
    const int hc_i0 = part(c, d, G), hc_nc = part(c + 1, d, G) - hc_i0;
    const bool hc_urow = HC && tid < f.hc_n * hc_nc;
    const int hc_uc = hc_urow ? tid / hc_nc : 0;
    const size_t hc_ui = static_cast<size_t>(hc_uc) * d + hc_i0 + (hc_urow ? tid - hc_uc * hc_nc : 0);
    uint4 hc_ua = make_uint4(0u, 0u, 0u, 0u), hc_ub = hc_ua;
    uint16_t hc_usb = 0, hc_ubb = 0;
    float hc_nv[kHcVals];
    if constexpr (HC) {
        STAMP(18);
        if (tid == 0 && (hc_q4 || hc_canon)) {
            uint32_t bytes;
            if (hc_q4) {
                const uint32_t qb = static_cast<uint32_t>(hd / 2), sb = static_cast<uint32_t>(hd / 32);
                bytes = qb + sb + (f.hc_down_b ? sb : 0u);
                mbar_expect_tx(&s_hcbar, bytes);
                bulk_load(hc_row, f.hc_down_q + static_cast<size_t>(c) * (hd / 8), qb, &s_hcbar);
                bulk_load(hc_row + qb, f.hc_down_s + static_cast<size_t>(c) * (hd / 64), sb, &s_hcbar);
                if (f.hc_down_b)
                    bulk_load(hc_row + qb + sb, f.hc_down_b + static_cast<size_t>(c) * (hd / 64), sb, &s_hcbar);
            } else {
                const uint16_t *src = c >= f.hc_lr ? f.hc_inject + static_cast<size_t>(c - f.hc_lr) * hd
                                                   : f.hc_down_bf + static_cast<size_t>(c) * hd;
                bytes = static_cast<uint32_t>(hd * 2);
                mbar_expect_tx(&s_hcbar, bytes);
                bulk_load(hc_row, src, bytes, &s_hcbar);
            }
        }
        if (hc_urow && f.hc_up_q) {
            hc_ua = *reinterpret_cast<const uint4 *>(f.hc_up_q + hc_ui * 8);
            hc_ub = *reinterpret_cast<const uint4 *>(f.hc_up_q + hc_ui * 8 + 4);
            hc_usb = f.hc_up_s[hc_ui];  // converted after the wait: no use of a load before it
            hc_ubb = f.hc_up_b ? f.hc_up_b[hc_ui] : 0;
        }
#pragma unroll
        for (int u = 0; u < kHcVals; ++u) {
            const int kk = u * kThreads + tid;
            hc_nv[u] = kk < hd ? f.hc_norm[kk] : 0.f;
        }
    }
    STAMP(24);
    pdl_wait();
    // Grid barriers: every launch adds nb G to the counter (each CTA arrives
    // nb times: 2, or 4 with hc_pre, whose launches use a counter of their
    // own), so it starts at a multiple of nb G; when this CTA reads it, at
    // most G - 1 arrivals of this launch can have happened (the first
    // barrier needs this CTA), so rounding down gives the launch's base.
    // (Read by the last thread, which stages no x: x's loads go out at once.)
    const unsigned long long nbG = (HC ? 4ull : 2ull) * G;
    const unsigned long long boff = HC ? 2ull * G : 0ull;  // the decode barriers' offset
    if (tid == kThreads - 1) s_base = ld_acquire64(sync) / nbG * nbG;
    float *lg = reinterpret_cast<float *>(sync + kSyncWords);  // [E + 1] logits
    float *hf = lg + ((E + 1 + 3) & ~3);                       // [S * I] h
    STAMP(1);

    if constexpr (HC) {
        // ---- gated_residual: h -> each stream's 1/rms (fp64 sum of squares,
        // the thread's values in ascending order, then the warps in order)
        double *s_ss = reinterpret_cast<double *>(hc_row + 16384 + 1024);  // [kWarps][8]
        double *s_acc = s_ss + kWarps * 8;                                  // [8][32]
        float *s_part = reinterpret_cast<float *>(s_acc + 8 * 32);          // [kWarps]
        float *s_r = s_part + kWarps;                                       // [8]
        float *s_w = s_r + 8;                                               // [lowrank]
        float *s_m = s_w + f.hc_lr;                                         // [8][32]
        // d = 4 kThreads (make_plan): values u = 4 sc .. 4 sc + 3 of a thread
        // belong to stream sc (hc <= 4)
        float hv[kHcVals];
#pragma unroll
        for (int u = 0; u < kHcVals; ++u) {
            const int kk = u * kThreads + tid;
            hv[u] = kk < hd ? f.hc_h[kk] : 0.f;
        }
        double ss[4];
#pragma unroll
        for (int sc = 0; sc < 4; ++sc) {
            ss[sc] = 0.0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const double v = f32_to_f64(hv[4 * sc + j]);
                ss[sc] = fma(v, v, ss[sc]);
            }
        }
        STAMP(19);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int sc = 0; sc < 4; ++sc) ss[sc] += __shfl_xor_sync(QK_FULL, ss[sc], off);
        if (lane == 0)
#pragma unroll
            for (int sc = 0; sc < 4; ++sc) s_ss[warp * 8 + sc] = ss[sc];
        __syncthreads();
        STAMP(22);
        if (tid < f.hc_n) {
            double tot = 0.0;
            for (int w = 0; w < kWarps; w += 2) tot += s_ss[w * 8 + tid] + s_ss[(w + 1) * 8 + tid];
            s_r[tid] = 1.0f / sqrtf(static_cast<float>(tot) / static_cast<float>(d) + 1e-6f);
        }
        __syncthreads();
#pragma unroll
        for (int sc = 0; sc < 4; ++sc) {
            if (sc < f.hc_n) {
                const float rc = s_r[sc];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    hc_x[(4 * sc + j) * kThreads + tid] = hv[4 * sc + j] * rc * hc_nv[4 * sc + j];
            }
        }
        STAMP(27);
        bool okh = true;
        if ((hc_q4 || hc_canon) && !mbar_wait(&s_hcbar, 0)) okh = false;
        okh = __syncthreads_and(okh) != 0;
        if (!okh && tid == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
        STAMP(23);
        const float inv_hc = 1.0f / static_cast<float>(f.hc_n);
        if (okh && hc_q4) {
            // down-mixer row c: warp w takes words [w nw / 16, (w + 1) nw / 16)
            const int nw = hd / 8;
            const uint32_t *q = reinterpret_cast<const uint32_t *>(hc_row);
            const uint16_t *scl = reinterpret_cast<const uint16_t *>(hc_row + hd / 2);
            const uint16_t *bia = f.hc_down_b ? scl + hd / 64 : nullptr;
            float acc = 0.f;
            for (int wi = warp * nw / kWarps + lane; wi < (warp + 1) * nw / kWarps; wi += 32) {
                const uint32_t v = q[wi];
                const float4 x0 = *reinterpret_cast<const float4 *>(hc_x + 8 * wi);
                const float4 x1 = *reinterpret_cast<const float4 *>(hc_x + 8 * wi + 4);
                const float xs8[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                float xq = 0.f, xs = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    xq = fmaf(xs8[i], static_cast<float>((v >> (4 * i)) & 0xFu), xq);
                    xs += xs8[i];
                }
                acc = fmaf(bf16lo(static_cast<uint32_t>(scl[wi / 8])), xq, acc);
                if (bia) acc = fmaf(bf16lo(static_cast<uint32_t>(bia[wi / 8])), xs, acc);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(QK_FULL, acc, off);
            if (lane == 0) s_part[warp] = acc;
            __syncthreads();
            if (tid == 0) {
                float v = 0.f;
                for (int w = 0; w < kWarps; ++w) v += s_part[w];
                v *= inv_hc;
                f.hc_w[c] = v / (1.0f + expf(-v));
            }
        } else if (okh && hc_canon) {
            // inject weights (or a dense bf16 down row): fp32 products, each
            // thread's over k = tid + 512 m in order, then the lanes' tree
            // and the warps in order (within the tolerance of the oracle's
            // canonical fp64 dot, which took about 3 us on eight warps here)
            const uint16_t *wr = reinterpret_cast<const uint16_t *>(hc_row);
            float acc = 0.f;
            for (int kk = tid; kk < hd; kk += kThreads) acc = fmaf(hc_x[kk], bf16lo(wr[kk]), acc);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(QK_FULL, acc, off);
            if (lane == 0) s_part[warp] = acc;
            __syncthreads();
            if (warp == 0) {
                float v = 0.f;
                for (int w = 0; w < kWarps; ++w) v += s_part[w];
                if (lane == 0) {
                    if (c >= f.hc_lr) {
                        f.hc_inj[c - f.hc_lr] = 2.0f / (1.0f + expf(-(v * inv_hc)));
                    } else {
                        const float u = v * inv_hc;
                        f.hc_w[c] = u / (1.0f + expf(-u));
                    }
                }
            }
        }
        STAMP(17);
        const unsigned long long hbase = s_base;  // (read after the CTA barriers above)
        grid_arrive(sync);
        grid_wait(sync, hbase + G, f.err);
        STAMP(28);
        // ---- the up-mixer rows and the stream mean of columns [i0, i0 + nc)
        for (int j = tid; j < f.hc_lr; j += kThreads) s_w[j] = __ldcg(f.hc_w + j);
        __syncthreads();
        if (hc_urow) {
            // (make_plan: a q4 up mixer with lowrank 64)
            const float u = hc_up1(hc_ua, hc_ub, bf16lo(hc_usb), bf16lo(hc_ubb), f.hc_up_b != nullptr, s_w);
            const float tmp = 1.0f / (1.0f + expf(-u));
            s_m[hc_uc * 32 + (tid - hc_uc * hc_nc)] = tmp * hc_x[hc_ui];
        }
        __syncthreads();
        if (tid < hc_nc) {
            float acc = 0.f;
            for (int sc = 0; sc < f.hc_n; ++sc) acc += s_m[sc * 32 + tid];
            f.hc_mixed[hc_i0 + tid] = acc / static_cast<float>(f.hc_n);
        }
        grid_arrive(sync);
        grid_wait(sync, hbase + 2ull * G, f.err);
        STAMP(29);
    }

    // ---- phase 1: x -> fp64 in shared memory for the router; thread t owns
    // the q4 word position t (elements 8t .. 8t + 7) and keeps its 8 values
    // in registers for the integer planes, which are made after the router
    // while the first grid barrier is pending (make_plan: d / 8 <= threads)
    float xv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = 0.f;
    if (tid < xwn) {
        load_x_word<HC>(f, tid, xv);
        rx_store(rx, tid, xv);
    }
    __syncthreads();
    const unsigned long long base = s_base;
    STAMP(21);
    const bool ok0 = __syncthreads_and(mbar_wait(&bar[0], 0)) != 0;  // CTA-uniform
    STAMP(2);
    if (!ok0 && tid == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
    const int nrr = rr1 - rr0;
    const int wpr = nrr * 4 <= kWarps ? 4 : (nrr * 2 <= kWarps ? 2 : 1);  // warps per router row
    if (ok0 && wpr > 1) {
        // each row split over wpr warps (2 or 4 of the eight sums per lane),
        // the parts folded in the canonical order, then one butterfly
        const int rl = warp / wpr, q = warp % wpr;
        if (rl < nrr) {
            const uint16_t *w =
                reinterpret_cast<const uint16_t *>(sm_router + static_cast<size_t>(rl) * d * 2);
            s_rpart[warp][lane] = wpr == 4 ? router_lane_part<2>(w, rx, d, lane, 2 * q)
                                           : router_lane_part<4>(w, rx, d, lane, 4 * q);
        }
        __syncthreads();
        if (warp < nrr) {
            const double *pp = &s_rpart[warp * wpr][lane];
            const double a = wpr == 4 ? (pp[0] + pp[32]) + (pp[64] + pp[96]) : pp[0] + pp[32];
            const double s = warp_sum_butterfly(a);
            STAMP(15);
            if (lane == 0) {
                const int r = rr0 + warp;
                float v = static_cast<float>(s);
                if (r < E && f.logit_bias) v = v + f.logit_bias[r];
                lg[r] = v;
            }
        }
    } else if (ok0) {
        for (int r = rr0 + warp; r < rr1; r += kWarps) {
            const uint16_t *w =
                reinterpret_cast<const uint16_t *>(sm_router + static_cast<size_t>(r - rr0) * d * 2);
            const double s = warp_sum_butterfly(router_lane(w, rx, d, lane));
            STAMP(15);
            if (lane == 0) {
                float v = static_cast<float>(s);
                if (r < E && f.logit_bias) v = v + f.logit_bias[r];
                lg[r] = v;
            }
        }
    }
    STAMP(3);
    grid_arrive(sync);
    // the experts' x: 16-bit integer planes, unit scales and sums
    {
        uint2 pl[kXB];
        float usum;
        const float sc = quant_word<kXB>(xv, pl, &usum);
        if (tid < xwn) {
            store_word<kXB>(xq, xwn, tid, pl);
            if ((tid & 3) == 0) {
                xusc[tid >> 2] = sc;
                xusm[tid >> 2] = usum;
            }
        }
    }
    __syncthreads();
    // every lane: its x units in registers
    uint2 xw[UPL][kXB][4];
    float xsc[UPL], xsm[UPL];
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        if (u < d / 32) {
            load_unit<kXB>(xq, xwn, u, xw[i]);
            xsc[i] = xusc[u];
            xsm[i] = xusm[u];
        } else {
#pragma unroll
            for (int pp = 0; pp < kXB; ++pp)
#pragma unroll
                for (int q = 0; q < 4; ++q) xw[i][pp][q] = make_uint2(0u, 0u);
            xsc[i] = 0.f;
            xsm[i] = 0.f;
        }
    }
    STAMP(13);
    grid_wait(sync, base + boff + G, f.err);
    STAMP(4);

    // ---- phase 2: top-k over the whole CTA. Every warp's largest key goes to
    // s_wmax; tau = the k-th largest of those maxima, so at least k keys are
    // >= tau and the keys >= tau hold the top-k and everything tied with or
    // above its members. They are gathered (in any order: the ranking
    // compares indices) and ranked by warp 0 (topk_rank_softmax), which
    // gives the result of topk_warp. When fewer than k warps hold keys, or
    // more than 32 keys reach tau, warp 0 runs topk_warp on all keys.
    const int nE = (E + 31) / 32 * 32;
    const bool block_topk = min(kWarps, nE / 32) >= k;
    {
        uint32_t mine[2] = {0u, 0u};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = tid + h * kThreads;
            if (e < nE) {
                mine[h] = e < E ? fkey(__ldcg(lg + e)) : 0u;
                s_keys[e] = mine[h];
            }
        }
        if (tid == 0) {
            s_gl = __ldcg(lg + E);
            s_cnt = 0;
        }
        const uint32_t wm = __reduce_max_sync(QK_FULL, max(mine[0], mine[1]));
        if (lane == 0) s_wmax[warp] = wm;
        __syncthreads();
        if (block_topk) {
            const uint32_t mv = lane < kWarps ? s_wmax[lane] : 0u;
            int r = 0;
#pragma unroll
            for (int j = 0; j < kWarps; ++j) {
                const uint32_t o = __shfl_sync(QK_FULL, mv, j);
                r += (o > mv || (o == mv && j < lane)) ? 1 : 0;
            }
            const uint32_t tau = __shfl_sync(QK_FULL, mv, __ffs(__ballot_sync(QK_FULL, r == k - 1)) - 1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int e = tid + h * kThreads;
                if (e < E && mine[h] >= tau && mine[h] != 0u) {
                    const int pos = atomicAdd(&s_cnt, 1);
                    if (pos < 32) {
                        s_key[pos] = mine[h];
                        s_idx[pos] = e;
                    }
                }
            }
        }
        __syncthreads();
    }
    STAMP(6);
    if (warp == 0) {
        STAMP(20);
        const int C = s_cnt;
        bool okk;
        if (block_topk && C >= k && C <= 32) {
            topk_rank_softmax(C, k, s_key, s_idx, s_ev, r_idx, r_w);
            okk = true;
        } else {
            okk = topk_warp(s_keys, E, k, s_key, s_idx, s_ev, r_idx, r_w);
        }
        STAMP(7);
        const uint8_t *sp = nullptr;
        if (okk && lane < k) {
            const int e = r_idx[lane];
            const int slot = (e >= 0 && e < E) ? s_slots[e] : -1;
            if (slot >= 0) sp = f.pool + static_cast<size_t>(slot) * L.slot_bytes;
        }
        const bool resident = __all_sync(QK_FULL, lane >= k || sp != nullptr);
        STAMP(25);
        const bool good = okk && resident && ok0;  // no copies in flight on error paths
        const int nch = s_nchunks;
        if (good && lane < nch)  // expect_tx before any copy of that barrier is issued
            mbar_expect_tx(&bar[2 + lane],
                           static_cast<uint32_t>((s_chunk0[lane + 1] - s_chunk0[lane]) * L.gu_row));
        if (lane < k) s_slotp[lane] = sp;
        if (lane == 0) {
            r_w[k] = 1.0f / (1.0f + expf(-s_gl));
            if (!okk) atomicOr(f.err, QK_ERR_BAD_ROUTE);
            else if (!resident) atomicOr(f.err, QK_ERR_NOT_RESIDENT);
            s_ok = good ? 1 : 0;
        }
        STAMP(26);
        __syncwarp();
        // the routed gate/up rows: one bulk copy per chunk (nch <= 12), from
        // the chunk's lane; the down rows follow below as 16-byte
        // asynchronous copies by every thread
        if (good) {
            if (lane < nch) {
                const int lo = gr0 + s_chunk0[lane], hi = gr0 + s_chunk0[lane + 1];
                const int sx = lo / I;
                bulk_load(sm_rgu + static_cast<size_t>(lo - gr0) * L.gu_row,
                          s_slotp[sx] + static_cast<size_t>(lo - sx * I) * L.gu_row,
                          static_cast<uint32_t>((hi - lo) * L.gu_row), &bar[2 + lane]);
            }
        }
        STAMP(14);
        if (c == 0 && okk) {
            if (lane < k) {
                f.idx[lane] = r_idx[lane];
                f.wts[lane] = r_w[lane];
            }
            if (lane == 0) f.sgate[0] = r_w[k];
        }
    } else if (ok0 && warp % 4 != 0) {
        // the shared expert's gate/up rows while warp 0 routes, on the warps
        // that do not share warp 0's scheduler (warp w issues on scheduler
        // w % 4): warp 0's top-k is on the critical path
        const int helper = warp - 1 - warp / 4, helpers = kWarps - kWarps / 4;
        for (int i = helper; i < sr1 - sr0; i += helpers) {
            const float hv =
                gateup_row<UPL>(sm_sgu + static_cast<size_t>(i) * L.gu_row, L, xw, xsc, xsm, lane);
            if (lane == 0) hf[static_cast<size_t>(k) * I + sr0 + i] = hv;
        }
    }
    __syncthreads();
    STAMP(5);
    const bool live = s_ok != 0;
    if (live) {
        // this CTA's down rows of the k routed experts -> sm_down (expert s
        // at s * or_max rows), 16 bytes per copy, spread over every thread
        const int per = (or1 - or0) * (L.d_row / 16);
        for (int i = tid; i < k * per; i += kThreads) {
            const int sx = i / per, rem = i - sx * per;
            cp_async16(sm_down + static_cast<size_t>(sx) * p.or_max * L.d_row + 16 * static_cast<size_t>(rem),
                       s_slotp[sx] + L.gu_bytes + static_cast<size_t>(or0) * L.d_row + 16 * static_cast<size_t>(rem));
        }
        cp_async_commit();
    }
    bool ok1 = true;
    if (live) {
        // routed rows, each after its chunk has landed
        const int nr = gr1 - gr0;
        int ch = 0;
        for (int i = warp; i < nr; i += kWarps) {
            while (ch + 1 < s_nchunks && s_chunk0[ch + 1] <= i) ++ch;
            if (!mbar_wait(&bar[2 + ch], 0)) {
                ok1 = false;
                break;
            }
            const float hv =
                gateup_row<UPL>(sm_rgu + static_cast<size_t>(i) * L.gu_row, L, xw, xsc, xsm, lane);
            // slot (gr0+i)/I, row (gr0+i)%I
            if (lane == 0) hf[gr0 + i] = hv;
        }
        // every chunk has landed before sm_rgu is reused for h
        for (int q = 0; q < s_nchunks && ok1; ++q) ok1 = mbar_wait(&bar[2 + q], 0);
        if (!ok1 && lane == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
    }
    ok1 = __syncthreads_and(ok1) != 0;  // CTA-uniform from here on
    STAMP(8);
    grid_arrive_wait(sync, base + boff + 2ull * G, f.err);  // every CTA, on every path
    STAMP(9);
    // every CTA of this grid has arrived, so all of them are resident: a
    // dependent launch may take SMs as they free up
    pdl_trigger();
    if (!live) return;

    // ---- phase 3: h -> 24-bit integers (kHB planes of S * I / 8 words, one
    // scale and sum per 32-element unit); a thread's kHW words are all loaded
    // before it quantizes, so the L2 round trip is paid once
    const int hwn = S * (I / 8), upe = I / 32;
    uint2 *hq = reinterpret_cast<uint2 *>(sm_rgu);
    float *husc = reinterpret_cast<float *>(hq + kHB * hwn);
    float *husm = husc + S * upe;
    {
        float4 hl[kHW][2];
#pragma unroll
        for (int r = 0; r < kHW; ++r) {
            const int w = tid + r * kThreads;
            if (w < hwn) {
                const float4 *hp = reinterpret_cast<const float4 *>(hf) + 2 * w;
                hl[r][0] = __ldcg(hp);
                hl[r][1] = __ldcg(hp + 1);
            } else {
                hl[r][0] = make_float4(0.f, 0.f, 0.f, 0.f);
                hl[r][1] = hl[r][0];
            }
        }
#pragma unroll
        for (int r = 0; r < kHW; ++r) {
            if (r * kThreads >= hwn) break;  // CTA-uniform
            const int w = tid + r * kThreads;
            const float v[8] = {hl[r][0].x, hl[r][0].y, hl[r][0].z, hl[r][0].w,
                                hl[r][1].x, hl[r][1].y, hl[r][1].z, hl[r][1].w};
            uint2 pl[kHB];
            float usum;
            const float sc = quant_word<kHB>(v, pl, &usum);
            if (w < hwn) {
                store_word<kHB>(hq, hwn, w, pl);
                if ((w & 3) == 0) {
                    husc[w >> 2] = sc;
                    husm[w >> 2] = usum;
                }
            }
        }
    }
    cp_async_wait_all();  // this thread's down-row copies (none when !live)
    __syncthreads();
    STAMP(10);
    if (!ok1) return;
    STAMP(11);
    // down: warp w takes expert s = w (and w + 16, ...): its h units stay in
    // registers (lane j holds unit j % LPR) while it walks the CTA's output
    // rows, RPW rows per step, keeping one partial per row step in registers;
    // each row's LPR lanes then reduce by shuffles (all row steps at once) into
    // partial[s][row]. The combine sums the partials in expert order with the
    // routing weights (the shared gate last); each output is written once.
    constexpr int RPW = 32 / LPR;
    const int nrows = or1 - or0;
    const int nsteps = (nrows + RPW - 1) / RPW;  // <= kRowSteps (make_plan)
    const int j = lane % LPR;
    const int grp = (32 * j) / L.g;
    float *partial = husm + S * upe;  // [S][or_max]
    for (int s = warp; s < S; s += kWarps) {
        uint2 hv[kHB][4];
        load_unit<kHB>(hq, hwn, s * upe + j, hv);
        const float hsc = husc[s * upe + j], hsm = husm[s * upe + j];
        const uint8_t *rows = sm_down + static_cast<size_t>(s) * p.or_max * L.d_row;
        float part[kRowSteps];
#pragma unroll
        for (int q = 0; q < kRowSteps; ++q) {
            part[q] = 0.f;
            const int rl = q * RPW + lane / LPR;
            if (q < nsteps && rl < nrows) {
                const uint8_t *row = rows + static_cast<size_t>(rl) * L.d_row;
                const uint4 w = *reinterpret_cast<const uint4 *>(row + 16 * j);
                const uint32_t sb = *reinterpret_cast<const uint32_t *>(row + I / 2 + 4 * grp);
                part[q] = fmaf(bf16lo(sb), dot_unit_q<kHB>(w, hv) * hsc, bf16hi(sb) * hsm);
            }
        }
#pragma unroll
        for (int off = LPR / 2; off >= 1; off >>= 1)
#pragma unroll
            for (int q = 0; q < kRowSteps; ++q) part[q] += __shfl_xor_sync(QK_FULL, part[q], off);
#pragma unroll
        for (int q = 0; q < kRowSteps; ++q) {
            const int rl = q * RPW + lane / LPR;
            if (j == 0 && q < nsteps && rl < nrows) partial[s * p.or_max + rl] = part[q];
        }
    }
    __syncthreads();
    STAMP(16);
    // combine in expert order: out = sum_s w_s * partial_s (shared gate last)
    for (int rl = tid; rl < nrows; rl += kThreads) {
        float acc = 0.f;
        for (int s = 0; s < S; ++s) acc = fmaf(r_w[s], partial[s * p.or_max + rl], acc);
        f.out[or0 + rl] = acc;
        if (f.hc_h) {  // the hyper connection's inject-add (k_hc_inject's arithmetic)
            for (int sc = 0; sc < f.hc_n; ++sc) {
                float *hp = f.hc_h + static_cast<size_t>(sc) * L.d + or0 + rl;
                *hp = fmaf(__ldcg(f.hc_inj + sc), acc, *hp);
            }
        }
    }
    STAMP(12);
    if (f.ptimes && tid == 0) {
        s_stamp[31] = clock64();
        for (int i = 0; i < 32; ++i) f.ptimes[static_cast<size_t>(c) * 32 + i] = s_stamp[i];
    }
#undef STAMP
}

constexpr int kFusedSmemMax = 200 * 1024;  // + ~10 KB static stays under 227 KB

int align128(int v) { return (v + 127) / 128 * 128; }

bool make_plan(const qk_fwd *f, Plan *p) {
    const qk_layout &L = f->L;
    const int G = f->num_sms > 0 ? f->num_sms : 148;
    const int S = L.k + 1;
    p->G = G;
    p->rr_max = (L.E + 1 + G - 1) / G;
    p->sr_max = (L.I + G - 1) / G;
    p->gr_max = (L.k * L.I + G - 1) / G;
    p->or_max = (L.d + G - 1) / G;
    // chunk count bound: every expert boundary inside the range adds one
    const int chunks = (p->gr_max + kChunkRows - 1) / kChunkRows + (p->gr_max + L.I - 1) / L.I + 1;
    if (chunks > kMaxChunks) return false;
    if (f->hc_pre) {
        // gated_residual in the prologue: h values per thread, one item per
        // CTA, columns per CTA, a q4 up mixer of one group, the staging in
        // the routed gate/up area (normed streams, the item's row, scratch)
        const int hd = f->hc_n * L.d;
        if (f->hc_n < 1 || f->hc_n > 4 || L.d != 4 * kThreads) return false;
        if (G < f->hc_lr + f->hc_n || L.d > 32 * G || !f->hc_up_q || f->hc_lr != 64) return false;
        const int need = hd * 4 + 16384 + 1024 + kWarps * 8 * 8 + 8 * 32 * 8 + kWarps * 4 + 8 * 4 +
                         f->hc_lr * 4 + 8 * 32 * 4;
        if (hd * 2 > 16384 || need > ((L.k * L.I + G - 1) / G) * L.gu_row) return false;
    }
    int off = 0;
    p->off_router = off;
    off = align128(off + p->rr_max * L.d * 2);
    p->off_sgu = off;
    off = align128(off + p->sr_max * L.gu_row);
    p->off_rgu = off;
    // after phase 2 the routed gate/up area holds h (planes, unit scales and
    // sums) and the per-expert partial outputs
    const int h_bytes = kHB * S * (L.I / 8) * 8 + 2 * S * (L.I / 32) * 4 + S * p->or_max * 4;
    if (S * (L.I / 8) > kHW * kThreads) return false;  // phase 3's h words per thread
    if (L.d / 8 > kThreads) return false;              // phase 1: one x word per thread
    if ((p->or_max + 32 / (L.I / 32) - 1) / (32 / (L.I / 32)) > kRowSteps) return false;
    off = align128(off + (p->gr_max * L.gu_row > h_bytes ? p->gr_max * L.gu_row : h_bytes));
    p->off_down = off;
    off = align128(off + S * p->or_max * L.d_row);
    p->off_xq = off;
    off = align128(off + kXB * (L.d / 8) * 8 + 2 * (L.d / 32) * 4);
    p->off_x = off;
    off = align128(off + L.d * 8);
    p->total = off;
    return off <= kFusedSmemMax;
}

template <int UPL, int LPR, bool HC = false>
const void *fused_fn() {
    return reinterpret_cast<const void *>(&k_decode_fused<UPL, LPR, HC>);
}

// instantiated shapes: d in (1024, 2048] with I = 512, and d <= 1024 with
// I = 128 (E <= 1024, group 64 for both)
// (the gated_residual prologue, hc_pre, is instantiated for the first shape)
const void *pick(const qk_layout &L, bool hc) {
    const int nunits = L.d / 32, lpr = L.I / 32;
    if (L.E > 1024 || L.g != 64) return nullptr;
    if (nunits <= 64 && nunits > 32 && lpr == 16) return hc ? fused_fn<2, 16, true>() : fused_fn<2, 16>();
    if (nunits <= 32 && lpr == 4 && !hc) return fused_fn<1, 4>();
    return nullptr;
}

}  // namespace

int qk_prepare_fused() {
    const void *fns[] = {fused_fn<2, 16>(), fused_fn<1, 4>(), fused_fn<2, 16, true>()};
    for (const void *fn : fns) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmemMax);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

extern "C" size_t qk_decode_sync_bytes(const qk_layout *L) {
    return 8 * kSyncWords + 4 * static_cast<size_t>((L->E + 1 + 3) & ~3) +
           4 * static_cast<size_t>(L->k + 1) * L->I;
}

extern "C" int qk_launch_decode_fused(const qk_fwd *f, void *sync, void *stream, int pdl) {
    if (f->T != 1) return QK_FUSED_UNFIT;
    Plan p;
    const void *fn = pick(f->L, f->hc_pre != 0);
    if (!fn || !make_plan(f, &p) || (f->L.E & 3)) return QK_FUSED_UNFIT;
    qk_fwd a = *f;
    unsigned long long *ctr = static_cast<unsigned long long *>(sync);
    void *args[] = {&a, &p, &ctr};
    return qk_launch_raw(fn, dim3(p.G), dim3(kThreads), static_cast<size_t>(p.total), stream, pdl,
                         args);
}
