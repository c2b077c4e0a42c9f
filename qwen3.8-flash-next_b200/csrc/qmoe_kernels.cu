// qmoe_kernels.cu - router, top-k and decode expert kernels for sm_100a.
//
// Reference path: moe_forward, c/src/model.c:1281-1405.
//   k_router        router logits + shared-gate logit   (model.c:1301, :1396)
//   k_topk          exact top-k, renormalised softmax,   (model.c:1303-1318,
//                   shared-gate sigmoid                   :1398)
//   k_decode_gateup gate/up dequant-GEMV, SiLU(g)*u      (model.c:1368-1374,
//                   for the k routed experts + shared     :1391-1394)
//   k_decode_down   down dequant-GEMV and the weighted   (model.c:1375-1386,
//                   combine with the sigmoid-gated shared :1395-1402)
//                   expert, reduced in registers (no atomics, no scatter)
//
// Weights stream HBM -> shared memory with cp.async.bulk (one bulk copy per
// contiguous row range, completion on an mbarrier), so every CTA has its whole
// share of bytes in flight at once. Waits on the mbarrier are bounded by
// %globaltimer and report QK_ERR_TIMEOUT_COPY instead of hanging.
// Consecutive kernels use programmatic dependent launch (griddepcontrol):
// each kernel triggers its dependents only after its own griddepcontrol.wait,
// so a kernel's prologue may read the outputs of the kernel two launches back.

#include <cuda_runtime.h>
#include <stdint.h>

#include "qmoe_internal.h"

#define DEV __device__ __forceinline__
#define FULL 0xffffffffu

namespace {

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s bound on copy waits

DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

DEV float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
DEV float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

DEV uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

DEV uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of bar; false when it timed out.
DEV bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (gtimer() - t0 > kWaitNs) return false;
    }
}

// Global -> shared bulk copy; dst, src and bytes are 16-byte multiples.
DEV void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Dot product of 32 nibbles (one 16-byte unit, low nibble first) with x:
// returns sum_i x_i * (1 + q_i / 16). The caller recovers sum x_i q_i as
// 16 * (result - sum x_i). Building 1 + q/16 costs one shift and one LOP3
// (exponent 127 OR'd over the nibble placed at mantissa bits 19..22), so each
// weight is one FFMA with no int->float conversion.
DEV float dot_unit(uint4 w, const float *x) {
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int sh = 19 - 4 * i;
            const uint32_t b = sh >= 0 ? (wd[j] << sh) : (wd[j] >> (-sh));
            const float fq = __uint_as_float((b & 0x00780000u) | 0x3F800000u);
            if (i & 1)
                a1 = fmaf(x[8 * j + i], fq, a1);
            else
                a0 = fmaf(x[8 * j + i], fq, a0);
        }
    }
    return a0 + a1;
}

DEV const uint8_t *expert_slot(const qk_fwd &f, int t, int s) {
    if (s == f.L.k) return f.shared_slot;
    const int e = f.idx[t * f.L.k + s];
    if (e < 0 || e >= f.L.E) return nullptr;
    const int slot = f.slot_of[e];
    if (slot < 0) return nullptr;
    return f.pool + static_cast<size_t>(slot) * f.L.slot_bytes;
}

DEV void load_x32(const qk_fwd &f, int t, int u, float *xr) {
    const int d = f.L.d;
    if (f.x_bf16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(
            static_cast<const uint16_t *>(f.x) + static_cast<size_t>(t) * d + 32 * u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 v = p[q];
            xr[8 * q + 0] = bf16lo(v.x); xr[8 * q + 1] = bf16hi(v.x);
            xr[8 * q + 2] = bf16lo(v.y); xr[8 * q + 3] = bf16hi(v.y);
            xr[8 * q + 4] = bf16lo(v.z); xr[8 * q + 5] = bf16hi(v.z);
            xr[8 * q + 6] = bf16lo(v.w); xr[8 * q + 7] = bf16hi(v.w);
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(
            static_cast<const float *>(f.x) + static_cast<size_t>(t) * d + 32 * u);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = p[q];
            xr[4 * q + 0] = v.x; xr[4 * q + 1] = v.y; xr[4 * q + 2] = v.z; xr[4 * q + 3] = v.w;
        }
    }
}

// ---------------------------------------------------------------------------
// Router: one warp per (row, token). Rows 0..E-1 are mlp.gate, row E is the
// shared-expert gate. Canonical order (identical to the CPU oracle's
// oracle_router_dot): lane l owns k = 256*i + 8*l + j, keeps eight fp64 sums
// a[j] accumulated over i ascending (the bf16 x fp32 products are exact in
// fp64, so the FMA equals the oracle's multiply-then-add), folds them as
// ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)), then a butterfly over lanes 16..1,
// and rounds once to fp32.
__global__ void __launch_bounds__(256) k_router(qk_fwd f) {
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = f.L.d, E = f.L.E;
    const int r = blockIdx.x * 8 + warp;
    const int t = blockIdx.y;
    if (r > E) return;
    const uint16_t *w = r < E ? f.router + static_cast<size_t>(r) * d : f.shared_gate;
    double a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = 0.0;
    for (int base = 0; base < d; base += 256) {
        const int k0 = base + 8 * lane;
        if (k0 < d) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(w + k0);
            float xv[8];
            if (f.x_bf16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(
                    static_cast<const uint16_t *>(f.x) + static_cast<size_t>(t) * d + k0);
                xv[0] = bf16lo(v.x); xv[1] = bf16hi(v.x); xv[2] = bf16lo(v.y); xv[3] = bf16hi(v.y);
                xv[4] = bf16lo(v.z); xv[5] = bf16hi(v.z); xv[6] = bf16lo(v.w); xv[7] = bf16hi(v.w);
            } else {
                const float4 *p = reinterpret_cast<const float4 *>(
                    static_cast<const float *>(f.x) + static_cast<size_t>(t) * d + k0);
                const float4 v0 = p[0], v1 = p[1];
                xv[0] = v0.x; xv[1] = v0.y; xv[2] = v0.z; xv[3] = v0.w;
                xv[4] = v1.x; xv[5] = v1.y; xv[6] = v1.z; xv[7] = v1.w;
            }
            const float wf[8] = {bf16lo(wv.x), bf16hi(wv.x), bf16lo(wv.y), bf16hi(wv.y),
                                 bf16lo(wv.z), bf16hi(wv.z), bf16lo(wv.w), bf16hi(wv.w)};
#pragma unroll
            for (int j = 0; j < 8; ++j)
                a[j] = fma(static_cast<double>(xv[j]), static_cast<double>(wf[j]), a[j]);
        }
    }
    double s = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = s + __shfl_xor_sync(FULL, s, off);
    if (lane == 0) {
        float v = static_cast<float>(s);
        if (r < E && f.logit_bias) v = v + f.logit_bias[r];
        f.logits[static_cast<size_t>(t) * (E + 1) + r] = v;
    }
}

// ---------------------------------------------------------------------------
// Top-k: one warp per token. Logits map to order-preserving u32 keys (-0 is
// folded onto +0). The k-th largest key is found MSB-first: at each bit the
// warp counts keys >= prefix|bit with one redux.sync; the search stops early
// as soon as exactly k keys qualify. Ties at the threshold are filled in
// ascending expert order, so the selection is (value desc, index asc), and
// the k are written in that order. Softmax over the k as model.c:1305-1318.
DEV uint32_t fkey(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b << 1) == 0) b = 0;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int VPL>
__global__ void __launch_bounds__(256) k_topk(qk_fwd f) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t s_key[8][32];
    __shared__ int s_idx[8][32];
    __shared__ float s_ev[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= f.T) return;
    const int E = f.L.E, k = f.L.k;
    const float *lg = f.logits + static_cast<size_t>(t) * (E + 1);
    uint32_t key[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        const int e = j * 32 + lane;
        key[j] = e < E ? fkey(lg[e]) : 0u;
    }
    uint32_t prefix = 0;
    bool exact = false;
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = prefix | (1u << bit);
        int c = 0;
#pragma unroll
        for (int j = 0; j < VPL; ++j) c += key[j] >= cand ? 1 : 0;
        const int cnt = static_cast<int>(__reduce_add_sync(FULL, static_cast<unsigned>(c)));
        if (cnt >= k) {
            prefix = cand;
            if (cnt == k) {
                exact = true;
                break;
            }
        }
    }
    // gather the selected (key, index) pairs into shared memory
    int base = 0;
    int need_eq = 0;
    if (!exact) {
        int c = 0;
#pragma unroll
        for (int j = 0; j < VPL; ++j) c += key[j] > prefix ? 1 : 0;
        need_eq = k - static_cast<int>(__reduce_add_sync(FULL, static_cast<unsigned>(c)));
    }
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        bool sel;
        if (exact) {
            sel = key[j] >= prefix;
        } else {
            const bool gt = key[j] > prefix;
            const bool eq = key[j] == prefix;
            const unsigned eqm = __ballot_sync(FULL, eq);
            const int before = __popc(eqm & ((1u << lane) - 1u));
            sel = gt || (eq && before < need_eq);
            need_eq -= min(__popc(eqm), need_eq);
        }
        const unsigned m = __ballot_sync(FULL, sel);
        if (sel) {
            const int pos = base + __popc(m & ((1u << lane) - 1u));
            if (pos < 32) {
                s_key[warp][pos] = key[j];
                s_idx[warp][pos] = j * 32 + lane;
            }
        }
        base += __popc(m);
    }
    __syncwarp();
    if (base != k) {
        if (lane == 0) atomicOr(f.err, QK_ERR_BAD_ROUTE);
        return;
    }
    // rank inside the k: value desc, index asc
    int rank = 0;
    uint32_t mk = 0;
    int mi = 0;
    if (lane < k) {
        mk = s_key[warp][lane];
        mi = s_idx[warp][lane];
        for (int m = 0; m < k; ++m) {
            const uint32_t ok = s_key[warp][m];
            const int oi = s_idx[warp][m];
            rank += (ok > mk || (ok == mk && oi < mi)) ? 1 : 0;
        }
    }
    __syncwarp();
    float v = 0.f;
    if (lane < k) {
        v = lg[mi];
        s_idx[warp][rank] = mi;
        s_key[warp][rank] = __float_as_uint(v);
    }
    __syncwarp();
    const float mx = __uint_as_float(s_key[warp][0]);  // rank 0 holds the max
    float ev = 0.f;
    if (lane < k) {
        ev = expf(v - mx);
        s_ev[warp][rank] = ev;
    }
    __syncwarp();
    float sum = 0.f;
    for (int m = 0; m < k; ++m) sum += s_ev[warp][m];
    if (lane < k) {
        f.idx[static_cast<size_t>(t) * k + rank] = mi;
        f.wts[static_cast<size_t>(t) * k + rank] = ev / sum;
    }
    if (lane == 0) {
        const float gl = lg[E];
        f.sgate[t] = 1.0f / (1.0f + expf(-gl));
    }
}

// ---------------------------------------------------------------------------
// Decode gate/up: rows r in [0, (k+1)*I) enumerate (expert slot s = r / I,
// h-row n = r % I); slot k is the shared expert. A CTA streams its contiguous
// row range into shared memory (one bulk copy per expert it touches) while its
// lanes load their slice of x into registers: lane l owns the 32-element units
// u = l, l + 32, ... (UPL units). One warp per h-row reduces the gate and up
// partial dots and writes h = SiLU(g) * u (fp32; model.c:1373-1374).
template <int UPL>
__global__ void __launch_bounds__(256, 1) k_decode_gateup(qk_fwd f, int rows_per_cta) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int ok;
    const qk_layout &L = f.L;
    const int t = blockIdx.y;
    const int total = (L.k + 1) * L.I;
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(total, r0 + rows_per_cta);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (r0 >= total) return;
    if (threadIdx.x == 0) {
        int good = 1;
        for (int r = r0; r < r1;) {
            const int s = r / L.I, n = r % L.I;
            const int cnt = min(r1 - r, L.I - n);
            if (!expert_slot(f, t, s)) good = 0;
            r += cnt;
        }
        ok = good;
        if (!good) {
            atomicOr(f.err, QK_ERR_NOT_RESIDENT);
        } else {
            mbar_expect_tx(&bar, static_cast<uint32_t>((r1 - r0) * L.gu_row));
            for (int r = r0; r < r1;) {
                const int s = r / L.I, n = r % L.I;
                const int cnt = min(r1 - r, L.I - n);
                bulk_load(smem + static_cast<size_t>(r - r0) * L.gu_row,
                          expert_slot(f, t, s) + static_cast<size_t>(n) * L.gu_row,
                          static_cast<uint32_t>(cnt * L.gu_row), &bar);
                r += cnt;
            }
        }
    }
    // x slice and unit sums into registers while the copies fly
    const int nunits = L.d / 32;
    float xr[UPL][32];
    float xs[UPL];
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        xs[i] = 0.f;
        if (u < nunits) {
            load_x32(f, t, u, xr[i]);
#pragma unroll
            for (int q = 0; q < 32; ++q) xs[i] += xr[i][q];
        }
    }
    __syncthreads();
    if (!ok) return;
    if (!mbar_wait(&bar, 0)) {
        if (threadIdx.x == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
        mbar_wait(&bar, 0);
        return;
    }
    const int half = L.d / 2;
    for (int r = r0 + warp; r < r1; r += 8) {
        const uint8_t *row = smem + static_cast<size_t>(r - r0) * L.gu_row;
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
            pg += __shfl_xor_sync(FULL, pg, off);
            pu += __shfl_xor_sync(FULL, pu, off);
        }
        if (lane == 0) {
            const int s = r / L.I, n = r % L.I;
            const float sg = pg / (1.0f + expf(-pg));
            f.h[(static_cast<size_t>(t) * (L.k + 1) + s) * L.I + n] = sg * pu;
        }
    }
}

// ---------------------------------------------------------------------------
// Decode down + combine: a CTA owns output rows [n0, n0 + R2) of one token
// and computes them for all k+1 experts, so the weighted combine
//   out[n] = sum_s w_s * (Wd_s . h_s)[n] + sigmoid(g) * (Wd_sh . h_sh)[n]
// happens in registers and each output is written once. LPR lanes share one
// row (one 32-element unit each); h sits in shared memory with its 16-byte
// chunks XOR-swizzled so the lanes' unit reads are bank-conflict free.
template <int LPR>
__global__ void __launch_bounds__(256, 1) k_decode_down(qk_fwd f) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int ok;
    constexpr int RPW = 32 / LPR;
    constexpr int R2 = 8 * RPW;
    const qk_layout &L = f.L;
    const int t = blockIdx.y;
    const int n0 = blockIdx.x * R2;
    const int nrows = min(R2, L.d - n0);
    const int S = L.k + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *wsm = smem;
    float4 *hs4 = reinterpret_cast<float4 *>(smem + static_cast<size_t>(S) * R2 * L.d_row);
    float *hsum = reinterpret_cast<float *>(hs4 + S * (L.I / 4));
    float *ws = hsum + S * (L.I / 32);
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    // Routing is two launches back and complete (see the file comment), so
    // the weight copies start before waiting for h.
    if (threadIdx.x == 0) {
        int good = 1;
        for (int s = 0; s < S; ++s)
            if (!expert_slot(f, t, s)) good = 0;
        ok = good;
        if (!good) {
            atomicOr(f.err, QK_ERR_NOT_RESIDENT);
        } else {
            mbar_expect_tx(&bar, static_cast<uint32_t>(S * nrows * L.d_row));
            for (int s = 0; s < S; ++s)
                bulk_load(wsm + static_cast<size_t>(s) * R2 * L.d_row,
                          expert_slot(f, t, s) + L.gu_bytes + static_cast<size_t>(n0) * L.d_row,
                          static_cast<uint32_t>(nrows * L.d_row), &bar);
        }
    }
    pdl_wait();
    pdl_trigger();
    // h of this token -> shared memory (swizzled), unit sums, combine weights
    const float4 *hg = reinterpret_cast<const float4 *>(f.h + static_cast<size_t>(t) * S * L.I);
    const int q4 = L.I / 4;
    for (int c = threadIdx.x; c < S * q4; c += blockDim.x) {
        const int s = c / q4, cc = c % q4, j = cc >> 3, q = cc & 7;
        hs4[s * q4 + 8 * j + (q ^ (j & 7))] = hg[c];
    }
    const int units = L.I / 32;
    for (int c = threadIdx.x; c < S * units; c += blockDim.x) {
        const float *p = f.h + (static_cast<size_t>(t) * S + c / units) * L.I + 32 * (c % units);
        float a = 0.f;
        for (int q = 0; q < 32; ++q) a += p[q];
        hsum[c] = a;
    }
    if (threadIdx.x < S)
        ws[threadIdx.x] = threadIdx.x < L.k ? f.wts[static_cast<size_t>(t) * L.k + threadIdx.x]
                                            : f.sgate[t];
    __syncthreads();
    if (!ok) return;
    if (!mbar_wait(&bar, 0)) {
        if (threadIdx.x == 0) atomicOr(f.err, QK_ERR_TIMEOUT_COPY);
        mbar_wait(&bar, 0);
        return;
    }
    const int rl = warp * RPW + lane / LPR;
    const int j = lane % LPR;
    const bool live = rl < nrows;
    const int rlc = live ? rl : 0;
    float acc = 0.f;
    for (int s = 0; s < S; ++s) {
        const uint8_t *row = wsm + (static_cast<size_t>(s) * R2 + rlc) * L.d_row;
        const uint4 w = *reinterpret_cast<const uint4 *>(row + 16 * j);
        const int grp = (32 * j) / L.g;
        const uint32_t sb = *reinterpret_cast<const uint32_t *>(row + L.I / 2 + 4 * grp);
        float hv[32];
        const float4 *hb = hs4 + s * q4 + 8 * j;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = hb[q ^ (j & 7)];
            hv[4 * q + 0] = v.x; hv[4 * q + 1] = v.y; hv[4 * q + 2] = v.z; hv[4 * q + 3] = v.w;
        }
        const float hsu = hsum[s * units + j];
        const float a = dot_unit(w, hv);
        float part = fmaf(bf16lo(sb), 16.f * (a - hsu), bf16hi(sb) * hsu);
#pragma unroll
        for (int off = LPR / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(FULL, part, off);
        acc = fmaf(ws[s], part, acc);
    }
    if (live && j == 0) f.out[static_cast<size_t>(t) * L.d + n0 + rl] = acc;
}

// ---------------------------------------------------------------------------

cudaError_t launch(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream, int pdl,
                   void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

int gateup_rows_per_cta(const qk_fwd *f) {
    const int total = (f->L.k + 1) * f->L.I;
    int ctas = f->num_sms > 0 ? f->num_sms : 148;
    if (f->T > 1) ctas = (ctas + f->T - 1) / f->T * 2;
    int r = (total + ctas - 1) / ctas;
    const int max_rows = (200 * 1024) / f->L.gu_row;
    if (r > max_rows) r = max_rows;
    if (r < 1) r = 1;
    return r;
}

constexpr int kMaxDynSmem = 200 * 1024;

const void *gateup_fn(int nunits) {
    if (nunits <= 32) return reinterpret_cast<const void *>(&k_decode_gateup<1>);
    if (nunits <= 64) return reinterpret_cast<const void *>(&k_decode_gateup<2>);
    return reinterpret_cast<const void *>(&k_decode_gateup<4>);
}

const void *down_fn(int lpr) {
    switch (lpr) {
        case 1: return reinterpret_cast<const void *>(&k_decode_down<1>);
        case 2: return reinterpret_cast<const void *>(&k_decode_down<2>);
        case 4: return reinterpret_cast<const void *>(&k_decode_down<4>);
        case 8: return reinterpret_cast<const void *>(&k_decode_down<8>);
        case 16: return reinterpret_cast<const void *>(&k_decode_down<16>);
        case 32: return reinterpret_cast<const void *>(&k_decode_down<32>);
        default: return nullptr;
    }
}

}  // namespace

extern "C" int qk_prepare_kernels(void) {
    const void *fns[] = {gateup_fn(32), gateup_fn(64), gateup_fn(128), down_fn(1), down_fn(2),
                         down_fn(4),    down_fn(8),    down_fn(16),    down_fn(32)};
    for (const void *fn : fns) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

extern "C" int qk_launch_router(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    void *args[] = {&a};
    dim3 grid((f->L.E + 1 + 7) / 8, f->T);
    return launch(reinterpret_cast<const void *>(&k_router), grid, dim3(256), 0, stream, pdl, args);
}

extern "C" int qk_launch_topk(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    void *args[] = {&a};
    dim3 grid((f->T + 7) / 8);
    const void *fn;
    if (f->L.E <= 64) fn = reinterpret_cast<const void *>(&k_topk<2>);
    else if (f->L.E <= 256) fn = reinterpret_cast<const void *>(&k_topk<8>);
    else if (f->L.E <= 512) fn = reinterpret_cast<const void *>(&k_topk<16>);
    else fn = reinterpret_cast<const void *>(&k_topk<32>);
    return launch(fn, grid, dim3(256), 0, stream, pdl, args);
}

extern "C" int qk_launch_decode_gateup(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    int rows = gateup_rows_per_cta(f);
    void *args[] = {&a, &rows};
    const int total = (f->L.k + 1) * f->L.I;
    dim3 grid((total + rows - 1) / rows, f->T);
    const size_t smem = static_cast<size_t>(rows) * f->L.gu_row;
    if (smem > static_cast<size_t>(kMaxDynSmem) || f->L.d / 32 > 128) return cudaErrorInvalidValue;
    return launch(gateup_fn(f->L.d / 32), grid, dim3(256), smem, stream, pdl, args);
}

extern "C" int qk_launch_decode_down(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    void *args[] = {&a};
    const int units = f->L.I / 32;
    const int lpr = units;  // one 32-element unit per lane
    const int R2 = 8 * (32 / lpr);
    const int S = f->L.k + 1;
    dim3 grid((f->L.d + R2 - 1) / R2, f->T);
    const size_t smem = static_cast<size_t>(S) * R2 * f->L.d_row +
                        static_cast<size_t>(S) * f->L.I * 4 + static_cast<size_t>(S) * units * 4 +
                        static_cast<size_t>(S) * 4;
    const void *fn = down_fn(lpr);
    if (!fn || smem > static_cast<size_t>(kMaxDynSmem)) return cudaErrorInvalidValue;
    return launch(fn, grid, dim3(256), smem, stream, pdl, args);
}
