// qmoe_decode_fused.cu - one-launch MoE layer for a single decode token.
//
// The whole of moe_forward (c/src/model.c:1281-1405) for T == 1 in one
// persistent kernel: one CTA per SM, three phases split by grid barriers.
//
//   prologue  bulk-copy the weights that do not depend on routing into shared
//             memory: this CTA's router rows (mlp.gate, plus the shared-gate
//             row) and its rows of the shared expert (gate/up and down).
//             Issued before griddepcontrol.wait, so they overlap the previous
//             kernel in the stream.
//   phase 1   x -> registers / shared memory; router rows -> logits (global);
//             shared-expert gate/up rows -> h (global).       [grid barrier]
//   phase 2   every CTA computes the same exact top-k from the 512 logits,
//             then bulk-copies its share of the routed experts' gate/up rows
//             AND its share of their down rows (all k experts at once), and
//             computes its gate/up rows -> h.                 [grid barrier]
//   phase 3   h -> shared memory; this CTA's output rows for all k+1 experts
//             (down weights already resident), weighted combine in registers.
//
// Per CTA at d=2048, E=512, k=10, I=512 on 148 SMs: 16 KB router, 9 KB shared
// gate/up, 81 KB routed gate/up, 44 KB down rows: every byte the CTA needs for
// the token is in flight at once. Dependents are triggered only after the
// second grid barrier, when every CTA of this grid is resident, so a waiting
// next launch can never take an SM this grid still needs.

#include "qmoe_dev.cuh"

using namespace qk;

cudaError_t qk_launch_raw(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream,
                          int pdl, void **args);

namespace {

struct Plan {
    int G;       // CTAs, one per SM
    int rr_max;  // router rows per CTA (of E + 1)
    int sr_max;  // shared gate/up rows per CTA (of I)
    int gr_max;  // routed gate/up rows per CTA (of k * I)
    int or_max;  // output rows per CTA (of d)
    int off_router, off_sgu, off_rgu, off_down, total;
};

__device__ __forceinline__ int part(int c, int n, int G) {
    return static_cast<int>((static_cast<long long>(c) * n) / G);
}

__device__ __forceinline__ void load_x_unit(const qk_fwd &f, int u, float *xr) {
    if (f.x_bf16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(f.x) + 32 * u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 v = p[q];
            xr[8 * q + 0] = bf16lo(v.x); xr[8 * q + 1] = bf16hi(v.x);
            xr[8 * q + 2] = bf16lo(v.y); xr[8 * q + 3] = bf16hi(v.y);
            xr[8 * q + 4] = bf16lo(v.z); xr[8 * q + 5] = bf16hi(v.z);
            xr[8 * q + 6] = bf16lo(v.w); xr[8 * q + 7] = bf16hi(v.w);
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(f.x) + 32 * u);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = p[q];
            xr[4 * q + 0] = v.x; xr[4 * q + 1] = v.y; xr[4 * q + 2] = v.z; xr[4 * q + 3] = v.w;
        }
    }
}

// One h-row of gate/up from a staged slot row: h = SiLU(gate . x) * (up . x).
template <int UPL>
__device__ __forceinline__ float gateup_row(const uint8_t *row, const qk_layout &L,
                                            const float (&xr)[UPL][32], const float (&xs)[UPL],
                                            int lane) {
    const int nunits = L.d / 32, half = L.d / 2;
    float pg = 0.f, pu = 0.f;
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        if (u < nunits) {
            const uint4 gw = *reinterpret_cast<const uint4 *>(row + 16 * u);
            const uint4 uw = *reinterpret_cast<const uint4 *>(row + half + 16 * u);
            const int grp = (32 * u) / L.g;
            const uint2 sb = *reinterpret_cast<const uint2 *>(row + L.d + 8 * grp);
            const float ag = dot_unit(gw, xr[i]);
            const float au = dot_unit(uw, xr[i]);
            pg += fmaf(bf16lo(sb.x), 16.f * (ag - xs[i]), bf16hi(sb.x) * xs[i]);
            pu += fmaf(bf16lo(sb.y), 16.f * (au - xs[i]), bf16hi(sb.y) * xs[i]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        pg += __shfl_xor_sync(QK_FULL, pg, off);
        pu += __shfl_xor_sync(QK_FULL, pu, off);
    }
    return (pg / (1.0f + expf(-pg))) * pu;
}

template <int UPL, int LPR>
__global__ void __launch_bounds__(256, 1) k_decode_fused(qk_fwd f, Plan p,
                                                         unsigned long long *gbar) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[3];
    __shared__ int s_ok;
    __shared__ uint32_t s_key[32];
    __shared__ int s_idx[32];
    __shared__ float s_ev[32];
    __shared__ int r_idx[32];
    __shared__ float r_w[33];
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
    uint8_t *sm_router = smem + p.off_router;
    uint8_t *sm_sgu = smem + p.off_sgu;
    uint8_t *sm_rgu = smem + p.off_rgu;
    uint8_t *sm_down = smem + p.off_down;
    float *sm_x = reinterpret_cast<float *>(smem + p.total) - d;  // last d floats

    // diagnostics: phase timestamps of this CTA (thread 0)
#define STAMP(i)                                                              \
    do {                                                                      \
        if (f.ptimes && tid == 0) f.ptimes[static_cast<size_t>(c) * 16 + (i)] = gtimer(); \
    } while (0)
    STAMP(0);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 1);
    }
    __syncthreads();

    // ---- prologue: weights independent of routing
    if (tid == 0) {
        const uint32_t b_router = static_cast<uint32_t>((rr1 - rr0) * d * 2);
        const uint32_t b_sgu = static_cast<uint32_t>((sr1 - sr0) * L.gu_row);
        const uint32_t b_sdown = static_cast<uint32_t>((or1 - or0) * L.d_row);
        const uint32_t b_slots = static_cast<uint32_t>(E * 4);
        mbar_expect_tx(&bar[0], b_router + b_sgu + b_sdown + b_slots);
        bulk_load(s_slots, f.slot_of, b_slots, &bar[0]);
        const int re = min(rr1, E);
        if (re > rr0)
            bulk_load(sm_router, f.router + static_cast<size_t>(rr0) * d,
                      static_cast<uint32_t>((re - rr0) * d * 2), &bar[0]);
        if (rr1 > E)
            bulk_load(sm_router + static_cast<size_t>(E - rr0) * d * 2, f.shared_gate,
                      static_cast<uint32_t>(d * 2), &bar[0]);
        if (sr1 > sr0)
            bulk_load(sm_sgu, f.shared_slot + static_cast<size_t>(sr0) * L.gu_row, b_sgu, &bar[0]);
        if (or1 > or0)
            bulk_load(sm_down + static_cast<size_t>(k) * p.or_max * L.d_row,
                      f.shared_slot + L.gu_bytes + static_cast<size_t>(or0) * L.d_row, b_sdown,
                      &bar[0]);
    }
    pdl_wait();
    STAMP(1);

    // ---- phase 1: x, router rows, shared gate/up rows
    for (int i = tid; i < d; i += blockDim.x)
        sm_x[i] = f.x_bf16
                      ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t *>(f.x)[i]) << 16)
                      : static_cast<const float *>(f.x)[i];
    float xr[UPL][32];
    float xs[UPL];
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        xs[i] = 0.f;
        if (u < d / 32) {
            load_x_unit(f, u, xr[i]);
#pragma unroll
            for (int q = 0; q < 32; ++q) xs[i] += xr[i][q];
        }
    }
    __syncthreads();
    const bool ok0 = mbar_wait(&bar[0], 0);
    STAMP(2);
    if (!ok0 && tid == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
    if (ok0) {
        for (int r = rr0 + warp; r < rr1; r += 8) {
            const uint16_t *w =
                reinterpret_cast<const uint16_t *>(sm_router + static_cast<size_t>(r - rr0) * d * 2);
            const double s = warp_sum_butterfly(router_lane(w, sm_x, d, lane));
            if (lane == 0) {
                float v = static_cast<float>(s);
                if (r < E && f.logit_bias) v = v + f.logit_bias[r];
                f.logits[r] = v;
            }
        }
    }
    STAMP(3);
    grid_sync(gbar, G, f.err);
    STAMP(4);

    // ---- phase 2: top-k, routed copies, routed gate/up rows. Warp 0 does
    // the top-k, looks the experts up in the staged slot table and issues
    // every routed copy, one copy per lane.
    topk_stage_keys<true>(f.logits, E, s_keys, tid, blockDim.x);
    __syncthreads();
    if (warp == 0) {
        const bool okk = topk_warp(s_keys, E, k, s_key, s_idx, s_ev, r_idx, r_w);
        const float gl = __ldcg(f.logits + E);
        const uint8_t *sp = nullptr;
        if (okk && lane < k) {
            const int e = r_idx[lane];
            const int slot = (e >= 0 && e < E) ? s_slots[e] : -1;
            if (slot >= 0) sp = f.pool + static_cast<size_t>(slot) * L.slot_bytes;
        }
        const bool resident = __all_sync(QK_FULL, lane >= k || sp != nullptr);
        const bool good = okk && resident && ok0;  // no copies in flight on error paths
        if (lane == 0) {
            r_w[k] = 1.0f / (1.0f + expf(-gl));
            if (!okk) atomicOr(f.err, QK_ERR_BAD_ROUTE);
            else if (!resident) atomicOr(f.err, QK_ERR_NOT_RESIDENT);
            s_ok = good ? 1 : 0;
            if (good) {
                mbar_expect_tx(&bar[1], static_cast<uint32_t>((gr1 - gr0) * L.gu_row));
                mbar_expect_tx(&bar[2], static_cast<uint32_t>(k * (or1 - or0) * L.d_row));
            }
        }
        __syncwarp();
        if (good) {
            const int s0 = gr0 / I;
            const int npieces = gr1 > gr0 ? (gr1 - 1) / I - s0 + 1 : 0;
            const int ndown = or1 > or0 ? k : 0;
            for (int q = 0; q < npieces + ndown; q += 32) {
                const int my = q + lane;
                const int s = my < npieces ? s0 + my : my - npieces;
                const uint8_t *src = reinterpret_cast<const uint8_t *>(
                    __shfl_sync(QK_FULL, reinterpret_cast<uintptr_t>(sp), s & 31));
                if (my < npieces) {
                    const int lo = max(gr0, s * I), hi = min(gr1, (s + 1) * I);
                    bulk_load(sm_rgu + static_cast<size_t>(lo - gr0) * L.gu_row,
                              src + static_cast<size_t>(lo - s * I) * L.gu_row,
                              static_cast<uint32_t>((hi - lo) * L.gu_row), &bar[1]);
                } else if (my < npieces + ndown) {
                    bulk_load(sm_down + static_cast<size_t>(s) * p.or_max * L.d_row,
                              src + L.gu_bytes + static_cast<size_t>(or0) * L.d_row,
                              static_cast<uint32_t>((or1 - or0) * L.d_row), &bar[2]);
                }
            }
        }
        if (c == 0 && okk) {
            if (lane < k) {
                f.idx[lane] = r_idx[lane];
                f.wts[lane] = r_w[lane];
            }
            if (lane == 0) f.sgate[0] = r_w[k];
        }
    }
    __syncthreads();
    STAMP(5);
    const bool live = s_ok != 0;
    bool ok1 = true;
    STAMP(6);
    if (live) {
        // The shared expert's rows (staged since the prologue) first, while
        // the routed copies fly, then the routed rows; one loop, so the
        // unrolled row code exists once.
        const int ns = sr1 - sr0, nr = gr1 - gr0;
        bool waited = false;
        for (int i = warp; i < ns + nr; i += 8) {
            const uint8_t *row;
            size_t hi;
            if (i < ns) {
                row = sm_sgu + static_cast<size_t>(i) * L.gu_row;
                hi = static_cast<size_t>(k) * I + sr0 + i;
            } else {
                if (!waited) {
                    ok1 = mbar_wait(&bar[1], 0);
                    waited = true;
                    if (!ok1) break;
                }
                row = sm_rgu + static_cast<size_t>(i - ns) * L.gu_row;
                hi = static_cast<size_t>(gr0 + i - ns);  // slot (gr0+i-ns)/I, row %I
            }
            const float hv = gateup_row<UPL>(row, L, xr, xs, lane);
            if (lane == 0) f.h[hi] = hv;
        }
        if (!waited) ok1 = mbar_wait(&bar[1], 0);
        STAMP(7);
        if (!ok1 && lane == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
    }
    STAMP(8);
    grid_sync(gbar, G, f.err);
    STAMP(9);
    pdl_trigger();

    // ---- phase 3: h -> shared memory, down rows + weighted combine
    float4 *hs4 = reinterpret_cast<float4 *>(sm_rgu);
    float *hsum = reinterpret_cast<float *>(hs4 + S * (I / 4));
    const int q4 = I / 4, units = I / 32;
    const float4 *hg = reinterpret_cast<const float4 *>(f.h);
    for (int i = tid; i < S * q4; i += blockDim.x) {
        const int s = i / q4, cc = i % q4, j = cc >> 3, q = cc & 7;
        hs4[s * q4 + 8 * j + (q ^ (j & 7))] = __ldcg(hg + i);
    }
    __syncthreads();
    for (int i = tid; i < S * units; i += blockDim.x) {
        const int j = i % units;
        const float4 *pp = hs4 + (i / units) * q4 + 8 * j;
        float a = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = pp[q ^ (j & 7)];
            a += v.x; a += v.y; a += v.z; a += v.w;
        }
        hsum[i] = a;
    }
    __syncthreads();
    STAMP(10);
    if (!live || !ok1) return;
    if (!mbar_wait(&bar[2], 0)) {
        if (tid == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
        mbar_wait(&bar[2], 0);
        return;
    }
    STAMP(11);
    constexpr int RPW = 32 / LPR;
    const int j = lane % LPR;
    for (int base = 0; base < or1 - or0; base += 8 * RPW) {
        const int rl = base + warp * RPW + lane / LPR;
        const bool on = rl < or1 - or0;
        const int rlc = on ? rl : 0;
        float acc = 0.f;
        for (int s = 0; s < S; ++s) {
            const uint8_t *row = sm_down + (static_cast<size_t>(s) * p.or_max + rlc) * L.d_row;
            const uint4 w = *reinterpret_cast<const uint4 *>(row + 16 * j);
            const int grp = (32 * j) / L.g;
            const uint32_t sb = *reinterpret_cast<const uint32_t *>(row + I / 2 + 4 * grp);
            float hv[32];
            const float4 *hb = hs4 + s * q4 + 8 * j;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = hb[q ^ (j & 7)];
                hv[4 * q + 0] = v.x; hv[4 * q + 1] = v.y; hv[4 * q + 2] = v.z; hv[4 * q + 3] = v.w;
            }
            const float hsu = hsum[s * units + j];
            const float a = dot_unit(w, hv);
            float part_ = fmaf(bf16lo(sb), 16.f * (a - hsu), bf16hi(sb) * hsu);
#pragma unroll
            for (int off = LPR / 2; off >= 1; off >>= 1)
                part_ += __shfl_xor_sync(QK_FULL, part_, off);
            acc = fmaf(r_w[s], part_, acc);
        }
        if (on && j == 0) f.out[or0 + rl] = acc;
    }
    STAMP(12);  // thread 0's own rows done
#undef STAMP
}

// dynamic shared memory cap; with ~9 KB of static shared memory this stays
// under the 227 KB a CTA may use
constexpr int kFusedSmemMax = 200 * 1024;

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
    int off = 0;
    p->off_router = off;
    off = align128(off + p->rr_max * L.d * 2);
    p->off_sgu = off;
    off = align128(off + p->sr_max * L.gu_row);
    p->off_rgu = off;
    const int h_bytes = S * L.I * 4 + S * (L.I / 32) * 4;
    off = align128(off + (p->gr_max * L.gu_row > h_bytes ? p->gr_max * L.gu_row : h_bytes));
    p->off_down = off;
    off = align128(off + S * p->or_max * L.d_row);
    off = align128(off + L.d * 4);  // x (fp32) at the end
    p->total = off;
    return off <= kFusedSmemMax;
}

template <int UPL, int LPR>
const void *fused_fn() {
    return reinterpret_cast<const void *>(&k_decode_fused<UPL, LPR>);
}

// instantiated shapes: d in (1024, 2048] with I = 512, and d <= 1024 with
// I = 128 (E <= 1024 for both)
const void *pick(const qk_layout &L) {
    const int nunits = L.d / 32, lpr = L.I / 32;
    if (L.E > 1024) return nullptr;
    if (nunits <= 64 && nunits > 32 && lpr == 16) return fused_fn<2, 16>();
    if (nunits <= 32 && lpr == 4) return fused_fn<1, 4>();
    return nullptr;
}

}  // namespace

int qk_prepare_fused() {
    const void *fns[] = {fused_fn<2, 16>(), fused_fn<1, 4>()};
    for (const void *fn : fns) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmemMax);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

extern "C" int qk_launch_decode_fused(const qk_fwd *f, unsigned *gbar, void *stream, int pdl) {
    if (f->T != 1) return QK_FUSED_UNFIT;
    Plan p;
    const void *fn = pick(f->L);
    if (!fn || !make_plan(f, &p) || (f->L.E & 3)) return QK_FUSED_UNFIT;
    qk_fwd a = *f;
    unsigned long long *ctr = reinterpret_cast<unsigned long long *>(gbar);
    void *args[] = {&a, &p, &ctr};
    return qk_launch_raw(fn, dim3(p.G), dim3(256), static_cast<size_t>(p.total), stream, pdl, args);
}
