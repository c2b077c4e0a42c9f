// qmoe_kernels.cu - router, top-k and per-token expert kernels for sm_100a
// (the multi-token path; T == 1 uses the single-launch kernel in
// qmoe_decode_fused.cu).
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
// contiguous row range, completion on an mbarrier). Consecutive kernels use
// programmatic dependent launch: each kernel triggers its dependents only
// after its own griddepcontrol.wait, so a kernel's prologue may read the
// outputs of the kernel two launches back.

#include "qmoe_dev.cuh"

using namespace qk;

namespace {

__device__ const uint8_t *slot_of_token(const qk_fwd &f, int t, int s) {
    if (s == f.L.k) return f.shared_slot;
    const int e = f.idx[t * f.L.k + s];
    if (e < 0 || e >= f.L.E) return nullptr;
    const int slot = f.slot_of[e];
    if (slot < 0) return nullptr;
    return f.pool + static_cast<size_t>(slot) * f.L.slot_bytes;
}

// Elements 8w .. 8w + 7 of token t's x (bf16 or fp32).
__device__ void load_x8(const qk_fwd &f, int t, int w, float *v) {
    const int d = f.L.d;
    if (f.x_bf16) {
        const uint4 q = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(f.x) +
                                                        static_cast<size_t>(t) * d)[w];
        v[0] = bf16lo(q.x); v[1] = bf16hi(q.x); v[2] = bf16lo(q.y); v[3] = bf16hi(q.y);
        v[4] = bf16lo(q.z); v[5] = bf16hi(q.z); v[6] = bf16lo(q.w); v[7] = bf16hi(q.w);
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(f.x) +
                                                           static_cast<size_t>(t) * d) + 2 * w;
        const float4 a = p[0], b = p[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

// ---------------------------------------------------------------------------
// Router: a CTA stages one token's x as fp32 in shared memory, then each warp
// computes one row (rows 0..E-1 are mlp.gate, row E is the shared-expert
// gate) in the canonical order of router_lane, identical to the CPU oracle.
__global__ void __launch_bounds__(256) k_router(qk_fwd f) {
    extern __shared__ __align__(16) double2 rx[];
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = f.L.d, E = f.L.E;
    const int t = blockIdx.y;
    // 8 elements per thread per step, loads before stores
    for (int i0 = 8 * threadIdx.x; i0 < d; i0 += 8 * blockDim.x) {
        float v[8];
        if (f.x_bf16) {
            const uint4 w = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(f.x) +
                                                             static_cast<size_t>(t) * d + i0);
            v[0] = bf16lo(w.x); v[1] = bf16hi(w.x); v[2] = bf16lo(w.y); v[3] = bf16hi(w.y);
            v[4] = bf16lo(w.z); v[5] = bf16hi(w.z); v[6] = bf16lo(w.w); v[7] = bf16hi(w.w);
        } else {
            const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(f.x) +
                                                               static_cast<size_t>(t) * d + i0);
            const float4 a = p[0], b = p[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        rx_store(rx, i0 / 8, v);
    }
    __syncthreads();
    for (int r = blockIdx.x * 8 + warp; r <= E; r += gridDim.x * 8) {
        const uint16_t *w = r < E ? f.router + static_cast<size_t>(r) * d : f.shared_gate;
        const double s = warp_sum_butterfly(router_lane(w, rx, d, lane));
        if (lane == 0) {
            float v = static_cast<float>(s);
            if (r < E && f.logit_bias) v = v + f.logit_bias[r];
            f.logits[static_cast<size_t>(t) * (E + 1) + r] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// Top-k: one warp per token (topk_warp on keys staged in shared memory),
// plus the shared-gate sigmoid.
__global__ void __launch_bounds__(256) k_topk(qk_fwd f) {
    extern __shared__ uint32_t keys_all[];  // [8][(E+31)/32*32]
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
    uint32_t *keys = keys_all + warp * ((E + 31) / 32 * 32);
    topk_stage_keys<false>(lg, E, keys, lane, 32);
    __syncwarp();
    if (!topk_warp(keys, E, k, s_key[warp], s_idx[warp], s_ev[warp],
                   f.idx + static_cast<size_t>(t) * k, f.wts + static_cast<size_t>(t) * k)) {
        if (lane == 0) atomicOr(f.err, QK_ERR_BAD_ROUTE);
        return;
    }
    if (lane == 0) f.sgate[t] = 1.0f / (1.0f + expf(-lg[E]));
}

// ---------------------------------------------------------------------------
// Gate/up: rows r in [0, (k+1)*I) enumerate (expert slot s = r / I, h-row
// n = r % I); slot k is the shared expert. A CTA streams its contiguous row
// range into shared memory (one bulk copy per expert it touches) while its
// threads put x into 16-bit integers (quant_word) and each lane takes its
// slice into registers: lane l owns the 32-element units u = l, l + 32, ...
// (UPL units). One warp per h-row reduces the gate and up partial dots and
// writes h = SiLU(g) * u (fp32; model.c:1373-1374). The arithmetic is the
// single-launch decode kernel's, so both give the same bits.
constexpr int kMaxD = 4096;  // largest hidden size of the per-token kernels

template <int UPL>
__global__ void __launch_bounds__(256, 1) k_decode_gateup(qk_fwd f, int rows_per_cta) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int ok;
    __shared__ __align__(16) uint2 xq[2 * (kMaxD / 8)];
    __shared__ float xusc[kMaxD / 32], xusm[kMaxD / 32];
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
            if (!slot_of_token(f, t, s)) good = 0;
            r += min(r1 - r, L.I - n);
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
                          slot_of_token(f, t, s) + static_cast<size_t>(n) * L.gu_row,
                          static_cast<uint32_t>(cnt * L.gu_row), &bar);
                r += cnt;
            }
        }
    }
    const int nunits = L.d / 32, xwn = L.d / 8;
    for (int w0 = 0; w0 < xwn; w0 += blockDim.x) {
        const int w = w0 + threadIdx.x;
        float v[8];
        if (w < xwn) {
            load_x8(f, t, w, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.f;
        }
        uint2 pl[2];
        float usum;
        const float sc = quant_word<2>(v, pl, &usum);
        if (w < xwn) {
            store_word<2>(xq, xwn, w, pl);
            if ((w & 3) == 0) {
                xusc[w >> 2] = sc;
                xusm[w >> 2] = usum;
            }
        }
    }
    __syncthreads();
    uint2 xw[UPL][2][4];
    float xsc[UPL], xsm[UPL];
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = lane + 32 * i;
        const int uc = u < nunits ? u : 0;
        load_unit<2>(xq, xwn, uc, xw[i]);
        xsc[i] = u < nunits ? xusc[uc] : 0.f;
        xsm[i] = u < nunits ? xusm[uc] : 0.f;
    }
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
                const float ag = dot_unit_q<2>(gw, xw[i]) * xsc[i];
                const float au = dot_unit_q<2>(uw, xw[i]) * xsc[i];
                pg += fmaf(bf16lo(sb.x), ag, bf16hi(sb.x) * xsm[i]);
                pu += fmaf(bf16lo(sb.y), au, bf16hi(sb.y) * xsm[i]);
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            pg += __shfl_xor_sync(QK_FULL, pg, off);
            pu += __shfl_xor_sync(QK_FULL, pu, off);
        }
        if (lane == 0) {
            const int s = r / L.I, n = r % L.I;
            const float sg = pg / (1.0f + expf(-pg));
            f.h[(static_cast<size_t>(t) * (L.k + 1) + s) * L.I + n] = sg * pu;
        }
    }
}

// ---------------------------------------------------------------------------
// Down + combine: a CTA owns output rows [n0, n0 + R2) of one token and
// computes them for all k+1 experts, so the weighted combine
//   out[n] = sum_s w_s * (Wd_s . h_s)[n] + sigmoid(g) * (Wd_sh . h_sh)[n]
// happens in registers and each output is written once. LPR lanes share one
// row (one 32-element unit each); h sits in shared memory as 24-bit integers
// (quant_word), as in the single-launch decode kernel.
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
    const int hwn = S * (L.I / 8), upe = L.I / 32;  // words of h, units per expert
    uint8_t *wsm = smem;
    uint2 *hq = reinterpret_cast<uint2 *>(smem + static_cast<size_t>(S) * R2 * L.d_row);
    float *husc = reinterpret_cast<float *>(hq + 3 * hwn);
    float *husm = husc + S * upe;
    float *ws = husm + S * upe;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    // Routing is two launches back and complete, so the weight copies start
    // before waiting for h.
    if (threadIdx.x == 0) {
        int good = 1;
        for (int s = 0; s < S; ++s)
            if (!slot_of_token(f, t, s)) good = 0;
        ok = good;
        if (!good) {
            atomicOr(f.err, QK_ERR_NOT_RESIDENT);
        } else {
            mbar_expect_tx(&bar, static_cast<uint32_t>(S * nrows * L.d_row));
            for (int s = 0; s < S; ++s)
                bulk_load(wsm + static_cast<size_t>(s) * R2 * L.d_row,
                          slot_of_token(f, t, s) + L.gu_bytes + static_cast<size_t>(n0) * L.d_row,
                          static_cast<uint32_t>(nrows * L.d_row), &bar);
        }
    }
    pdl_wait();
    pdl_trigger();
    const float4 *hg = reinterpret_cast<const float4 *>(f.h + static_cast<size_t>(t) * S * L.I);
    for (int w0 = 0; w0 < hwn; w0 += blockDim.x) {
        const int w = w0 + threadIdx.x;
        float v[8];
        if (w < hwn) {
            const float4 a = hg[2 * w], b = hg[2 * w + 1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.f;
        }
        uint2 pl[3];
        float usum;
        const float sc = quant_word<3>(v, pl, &usum);
        if (w < hwn) {
            store_word<3>(hq, hwn, w, pl);
            if ((w & 3) == 0) {
                husc[w >> 2] = sc;
                husm[w >> 2] = usum;
            }
        }
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
        uint2 hv[3][4];
        load_unit<3>(hq, hwn, s * upe + j, hv);
        float part = fmaf(bf16lo(sb), dot_unit_q<3>(w, hv) * husc[s * upe + j],
                          bf16hi(sb) * husm[s * upe + j]);
#pragma unroll
        for (int off = LPR / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(QK_FULL, part, off);
        acc = fmaf(ws[s], part, acc);
    }
    if (live && j == 0) f.out[static_cast<size_t>(t) * L.d + n0 + rl] = acc;
}

// ---------------------------------------------------------------------------
// Host-pointer single-token calls: x is read from pinned host memory by one
// CTA (its dependents may launch at once, so the decode kernel's weight
// prologue overlaps the PCIe read), and after the layer the error word is
// copied to pinned host memory by a dependent launch (the output itself is
// written to pinned host memory by the decode kernel).
__global__ void k_copy_in(const float4 *src, float4 *dst, int n4) {
    pdl_trigger();
    for (int i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = src[i];
}

// After the layer: the error word to pinned memory, then (ctr != NULL) a
// completion count, so the host can wait by watching pinned memory instead
// of synchronising the stream. The layer's output writes completed with its
// grid, before pdl_wait returns here.
__global__ void k_report(const int *err, volatile int *err_host, unsigned *ctr,
                         volatile unsigned *ctr_host) {
    pdl_wait();
    if (threadIdx.x == 0) {
        *err_host = *err;
        if (ctr) {
            const unsigned v = *ctr + 1u;
            *ctr = v;
            __threadfence_system();
            *ctr_host = v;
        }
    }
}

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

cudaError_t qk_launch_raw(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream,
                          int pdl, void **args) {
    return launch(fn, grid, block, smem, stream, pdl, args);
}

int qk_prepare_fused();

extern "C" int qk_prepare_kernels(void) {
    const void *fns[] = {gateup_fn(32), gateup_fn(64), gateup_fn(128), down_fn(1), down_fn(2),
                         down_fn(4),    down_fn(8),    down_fn(16),    down_fn(32)};
    for (const void *fn : fns) {
        cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
        if (e != cudaSuccess) return e;
    }
    return qk_prepare_fused();
}

extern "C" int qk_launch_router(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    void *args[] = {&a};
    const int per_token = (f->L.E + 1 + 7) / 8;
    dim3 grid(per_token < 64 ? per_token : 64, f->T);
    return launch(reinterpret_cast<const void *>(&k_router), grid, dim3(256),
                  static_cast<size_t>(f->L.d) * sizeof(double), stream, pdl, args);
}

extern "C" int qk_launch_copy_in(const void *src_host, void *dst, size_t bytes, void *stream) {
    if (bytes % 16) return cudaErrorInvalidValue;
    const float4 *s = static_cast<const float4 *>(src_host);
    float4 *d = static_cast<float4 *>(dst);
    int n4 = static_cast<int>(bytes / 16);
    void *args[] = {&s, &d, &n4};
    return launch(reinterpret_cast<const void *>(&k_copy_in), dim3(1), dim3(512), 0, stream, 0,
                  args);
}

extern "C" int qk_launch_report(const int *err, int *err_host, unsigned *ctr, unsigned *ctr_host,
                                void *stream) {
    volatile int *h = err_host;
    volatile unsigned *ch = ctr_host;
    void *args[] = {&err, &h, &ctr, &ch};
    return launch(reinterpret_cast<const void *>(&k_report), dim3(1), dim3(32), 0, stream, 1, args);
}

extern "C" int qk_launch_topk(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    void *args[] = {&a};
    dim3 grid((f->T + 7) / 8);
    const size_t smem = static_cast<size_t>(8) * ((f->L.E + 31) / 32 * 32) * sizeof(uint32_t);
    return launch(reinterpret_cast<const void *>(&k_topk), grid, dim3(256), smem, stream, pdl,
                  args);
}

extern "C" int qk_launch_decode_gateup(const qk_fwd *f, void *stream, int pdl) {
    qk_fwd a = *f;
    int rows = gateup_rows_per_cta(f);
    void *args[] = {&a, &rows};
    const int total = (f->L.k + 1) * f->L.I;
    dim3 grid((total + rows - 1) / rows, f->T);
    const size_t smem = static_cast<size_t>(rows) * f->L.gu_row;
    if (smem > static_cast<size_t>(kMaxDynSmem) || f->L.d > kMaxD) return cudaErrorInvalidValue;
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
                        3 * static_cast<size_t>(S) * (f->L.I / 8) * 8 +
                        2 * static_cast<size_t>(S) * units * 4 + static_cast<size_t>(S) * 4;
    const void *fn = down_fn(lpr);
    if (!fn || smem > static_cast<size_t>(kMaxDynSmem)) return cudaErrorInvalidValue;
    return launch(fn, grid, dim3(256), smem, stream, pdl, args);
}
