// qmoe_hc.cu - the MoE side's hyper connection of one layer, around the MoE
// block: gated_residual before it and the inject-add after it
// (c/src/model.c:728-796, :1708-1731).
//
// The residual state of a token is hc streams of d values, h [hc * d]. Per
// token:
//   normed = RMSNorm of each stream's d values (eps 1e-6) x hc_norm
//   w      = silu(down(normed) / hc)                 down [lowrank, hc*d]
//   tmp    = sigmoid(up(w))                          up   [hc*d, lowrank]
//   mixed  = mean over the streams of tmp * normed   -> the MoE block's x
//   inject = 2 sigmoid(block_inject(normed) / hc)    block_inject [hc, hc*d]
//   h[c, :] += inject[c] * moe(mixed)                for every stream c
// The mixers are q4 with group 64 (linear_forward -> gemm_q4: per group
// s * sum x q + b * sum x, absent biases read as zeros) or dense bf16; dense
// bf16 products and block_inject use the canonical router dot (exact products
// summed in fp64 in a fixed order, one rounding), as gemm_bf16 is defined for
// this project.
//
//   k_hc_down    grid (lowrank / 4 + 1, tokens): a CTA stages the token's
//                normed streams in shared memory (sum of squares in fp64);
//                warp w of CTA j computes w[4j + w]; the last CTA computes
//                inject and the streams' norms for k_hc_up.
//   k_hc_up      grid (d / 128, tokens): thread i of CTA b owns column
//                128 b + i of every stream: tmp of its hc up-rows, and mixed.
//   k_hc_pre1    one token (decode): both of the above in one launch of one
//                CTA per SM with one grid barrier. Every CTA stages the
//                normed streams; CTA b takes down rows / inject streams
//                b, b + G, ... (eight warps per row: q4 rows split into
//                eight word ranges, dense rows into the canonical order's
//                eight per-lane sums); after the barrier CTA b computes the
//                up rows and mixed values of its d / G columns.
//   k_hc_inject  grid (hc*d / 1024, tokens): h += inject x the block's
//                output, launched as a programmatic dependent of the block.

#include "qmoe_dev.cuh"

using namespace qk;

namespace {

struct HcArgs {
    int d, hc, lr;
    const float *norm;                 // [hc*d]
    const uint32_t *down_q;            // [lr, hc*d/8] or NULL (dense)
    const uint16_t *down_s, *down_b;   // [lr, hc*d/64]; b may be NULL
    const uint16_t *down_bf;           // [lr, hc*d]
    const uint32_t *up_q;              // [hc*d, lr/8] or NULL (dense)
    const uint16_t *up_s, *up_b;       // [hc*d, lr/64]; b may be NULL
    const uint16_t *up_bf;             // [hc*d, lr]
    const uint16_t *inject;            // [hc, hc*d]
    const float *h;                    // [n, hc*d]
    float *W;                          // [n, lr]
    float *R;                          // [n, hc] 1/rms of each stream
    float *INJ;                        // [n, hc]
    float *mixed;                      // [n, d]
};

QK_DEV float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

// The canonical dot over K values (x fp32 in shared memory, w bf16): lane l
// owns k = 256 i + 8 l + j, eight fp64 sums over i ascending, folded
// ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)), then a butterfly 16..1; every lane
// returns the fp64 total.
QK_DEV double canon_dot(const float *x, const uint16_t *w, int K, int lane) {
    double a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = 0.0;
    for (int base = 0; base < K; base += 256) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = base + 8 * lane + j;
            if (k < K) a[j] = fma(static_cast<double>(x[k]), bf16_to_f64(w[k]), a[j]);
        }
    }
    return warp_sum_butterfly(((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7])));
}

// One q4 row times x (K values in shared memory): per 8-value word,
// s * sum x q + b * sum x with the word's group scale and bias, summed over
// the lane's words and then over the warp. Returns the total on every lane.
QK_DEV float q4_dot(const float *x, const uint32_t *q, const uint16_t *s, const uint16_t *b, int K,
                    int lane) {
    float acc = 0.f;
    for (int wi = lane; wi < K / 8; wi += 32) {
        const uint32_t v = q[wi];
        float xq = 0.f, xs = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float xv = x[8 * wi + i];
            xq = fmaf(xv, static_cast<float>((v >> (4 * i)) & 0xFu), xq);
            xs += xv;
        }
        const int g = wi / 8;
        acc = fmaf(bf16f(s[g]), xq, acc);
        if (b) acc = fmaf(bf16f(b[g]), xs, acc);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(QK_FULL, acc, off);
    return acc;
}

__global__ void __launch_bounds__(128) k_hc_down(HcArgs a, int nb) {
    extern __shared__ float s_x[];  // [hc*d] normed
    __shared__ double s_ss[4][8];
    __shared__ float s_r[8];
    const int t = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = a.hc * a.d;
    const float *h = a.h + static_cast<size_t>(t) * hd;
    // sum of squares of each stream in fp64 (exact squares; order fixed)
    for (int c = 0; c < a.hc; ++c) {
        double ss = 0.0;
        for (int i = threadIdx.x; i < a.d; i += blockDim.x) {
            const double v = h[static_cast<size_t>(c) * a.d + i];
            ss = fma(v, v, ss);
        }
        ss = warp_sum_butterfly(ss);
        if (lane == 0) s_ss[warp][c & 7] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            const double tot = (s_ss[0][c & 7] + s_ss[1][c & 7]) + (s_ss[2][c & 7] + s_ss[3][c & 7]);
            s_r[c & 7] = 1.0f / sqrtf(static_cast<float>(tot) / static_cast<float>(a.d) + 1e-6f);
        }
        __syncthreads();
        const float r = s_r[c & 7];
        for (int i = threadIdx.x; i < a.d; i += blockDim.x) {
            const size_t k = static_cast<size_t>(c) * a.d + i;
            s_x[k] = h[k] * r * a.norm[k];
        }
        if (blockIdx.x == nb && threadIdx.x == 0) a.R[static_cast<size_t>(t) * a.hc + c] = r;
    }
    __syncthreads();
    const float inv_hc = 1.0f / static_cast<float>(a.hc);
    if (blockIdx.x < nb) {
        const int j = 4 * blockIdx.x + warp;
        if (j < a.lr) {
            float v;
            if (a.down_q) {
                const size_t ng = static_cast<size_t>(hd) / 64;
                v = q4_dot(s_x, a.down_q + static_cast<size_t>(j) * (hd / 8), a.down_s + j * ng,
                           a.down_b ? a.down_b + j * ng : nullptr, hd, lane);
            } else {
                v = static_cast<float>(canon_dot(s_x, a.down_bf + static_cast<size_t>(j) * hd, hd, lane));
            }
            v *= inv_hc;
            if (lane == 0) a.W[static_cast<size_t>(t) * a.lr + j] = v / (1.0f + expf(-v));
        }
    } else {
        // inject = 2 sigmoid(block_inject(normed) / hc), one warp per stream
        for (int c = warp; c < a.hc; c += 4) {
            const float v = static_cast<float>(canon_dot(s_x, a.inject + static_cast<size_t>(c) * hd, hd, lane));
            if (lane == 0) a.INJ[static_cast<size_t>(t) * a.hc + c] = 2.0f / (1.0f + expf(-(v * inv_hc)));
        }
    }
}

// Up-mixer row `row` times w (lowrank values in shared memory), computed by
// one thread: q4 rows with gemm_q4's per-group sums, groups in order; dense
// rows in the canonical order for K = lowrank.
QK_DEV float up_row(const HcArgs &a, size_t row, const float *s_w) {
        float u;
        if (a.up_q) {
            // one thread per up-row: gemm_q4's per-group sums, groups in order
            const uint32_t *q = a.up_q + row * (a.lr / 8);
            const int ng = a.lr / 64;
            u = 0.f;
            for (int g = 0; g < ng; ++g) {
                // the group's eight words and its scale and bias loaded
                // before any arithmetic (one memory latency per group)
                const uint4 qa = *reinterpret_cast<const uint4 *>(q + 8 * g);
                const uint4 qb = *reinterpret_cast<const uint4 *>(q + 8 * g + 4);
                const float sg = bf16f(a.up_s[row * ng + g]);
                const float bg = a.up_b ? bf16f(a.up_b[row * ng + g]) : 0.f;
                const uint32_t wds[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                float xq = 0.f, xs = 0.f;
                for (int i2 = 0; i2 < 64; ++i2) xs += s_w[64 * g + i2];
#pragma unroll
                for (int wd = 0; wd < 8; ++wd) {
                    const uint32_t v = wds[wd];
#pragma unroll
                    for (int b = 0; b < 8; ++b)
                        xq = fmaf(s_w[64 * g + 8 * wd + b], static_cast<float>((v >> (4 * b)) & 0xFu), xq);
                }
                u = fmaf(sg, xq, u);
                if (a.up_b) u = fmaf(bg, xs, u);
            }
        } else {
            // the canonical order for K = lowrank, computed by one thread
            const uint16_t *w = a.up_bf + row * a.lr;
            double lanes[32];
            for (int l = 0; l < 32; ++l) {
                double p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int base = 0; base < a.lr; base += 256)
                    for (int j = 0; j < 8; ++j) {
                        const int k = base + 8 * l + j;
                        if (k < a.lr) p[j] = fma(static_cast<double>(s_w[k]), bf16_to_f64(w[k]), p[j]);
                    }
                lanes[l] = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
            }
            for (int off = 16; off >= 1; off >>= 1) {
                double nx[32];
                for (int l = 0; l < 32; ++l) nx[l] = lanes[l] + lanes[l ^ off];
                for (int l = 0; l < 32; ++l) lanes[l] = nx[l];
            }
            u = static_cast<float>(lanes[0]);
        }
        return u;
}

__global__ void __launch_bounds__(128) k_hc_up(HcArgs a) {
    extern __shared__ float s_w[];  // [lr]
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    const int hd = a.hc * a.d;
    for (int j = threadIdx.x; j < a.lr; j += blockDim.x) s_w[j] = a.W[static_cast<size_t>(t) * a.lr + j];
    __syncthreads();
    if (i >= a.d) return;
    const float *h = a.h + static_cast<size_t>(t) * hd;
    float acc = 0.f;
    for (int c = 0; c < a.hc; ++c) {
        const size_t row = static_cast<size_t>(c) * a.d + i;
        const float u = up_row(a, row, s_w);
        const float tmp = 1.0f / (1.0f + expf(-u));
        const float nv = h[row] * a.R[static_cast<size_t>(t) * a.hc + c] * a.norm[row];
        acc += tmp * nv;
    }
    a.mixed[static_cast<size_t>(t) * a.d + i] = acc / static_cast<float>(a.hc);
}

// One CTA per 1024 values of a token's hc*d, 256 consecutive values per
// pass (h is the caller's buffer: no alignment beyond 4 bytes is assumed).
// Waits for the block that wrote y.
__global__ void __launch_bounds__(256) k_hc_inject(float *h, const float *inj, const float *y, int hc, int d) {
    pdl_wait();
    const int t = blockIdx.y, hd = hc * d;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int e = blockIdx.x * 1024 + p * 256 + threadIdx.x;
        if (e < hd) {
            const int c = e / d;
            const float s = inj[static_cast<size_t>(t) * hc + c];
            float *hp = h + static_cast<size_t>(t) * hd + e;
            *hp = fmaf(s, y[static_cast<size_t>(t) * d + (e - c * d)], *hp);
        }
    }
}

constexpr int kPreThreads = 256;  // k_hc_pre1: eight warps
constexpr int kPreCols = 32;      // k_hc_pre1: most d columns per CTA
constexpr int kPreWords = 4;      // k_hc_pre1: most q4 words of a down row per lane
constexpr int kPreH = 32;         // k_hc_pre1: h values per thread (hc*d <= 8192)

__global__ void __launch_bounds__(kPreThreads) k_hc_pre1(HcArgs a, unsigned long long *ctr, int *err) {
    extern __shared__ float s_x[];  // [hc*d] normed, then [lr] w
    __shared__ double s_ss[8][8];   // [warp][stream]
    __shared__ double s_acc[8][32];
    __shared__ float s_part[8];
    __shared__ float s_r[8];
    __shared__ float s_m[8][kPreCols];
    __shared__ unsigned long long s_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = a.hc * a.d, G = gridDim.x;
    const int nh = hd / kPreThreads;    // h values of this thread: k = 256 u + tid
    const int upc = a.d / kPreThreads;  // of them per stream (the launcher checks d % 256 == 0)
    float *s_w = s_x + hd;
    const float inv_hc = 1.0f / static_cast<float>(a.hc);

    // ---- every weight this thread will use, loaded before anything waits:
    // they do not depend on the previous kernel, so their latency overlaps
    // its end and the loads of h
    const int r = blockIdx.x;  // this CTA's item: r < lr a down row, then the inject streams
    const bool q4item = r < a.lr && a.down_q;
    const bool canon_item = !q4item && r < a.lr + a.hc;
    const int nw = hd / 8;
    const int w0 = warp * nw / 8, w1 = (warp + 1) * nw / 8;
    uint32_t qv[kPreWords];
    float sv[kPreWords], bv[kPreWords];
    uint16_t wv[kPreH];
    if (q4item) {
        const int ng = hd / 64;
        const uint32_t *q = a.down_q + static_cast<size_t>(r) * nw;
        const uint16_t *sc = a.down_s + static_cast<size_t>(r) * ng;
        const uint16_t *bi = a.down_b ? a.down_b + static_cast<size_t>(r) * ng : nullptr;
#pragma unroll
        for (int m = 0; m < kPreWords; ++m) {
            const int wi = w0 + lane + 32 * m;
            qv[m] = wi < w1 ? q[wi] : 0u;
            sv[m] = wi < w1 ? bf16f(sc[wi / 8]) : 0.f;
            bv[m] = wi < w1 && bi ? bf16f(bi[wi / 8]) : 0.f;
        }
    } else if (canon_item) {
        // lane's canonical sum number `warp`: k = 256 u + 8 lane + warp
        const uint16_t *wr = r >= a.lr ? a.inject + static_cast<size_t>(r - a.lr) * hd
                                       : a.down_bf + static_cast<size_t>(r) * hd;
#pragma unroll
        for (int u = 0; u < kPreH; ++u) {
            const int k = 256 * u + 8 * lane + warp;
            wv[u] = k < hd ? wr[k] : 0;
        }
    }
    const int i0 = blockIdx.x * a.d / G, nc = (blockIdx.x + 1) * a.d / G - i0;
    const bool urow = tid < a.hc * nc;
    const int uc = urow ? tid / nc : 0, ucol = urow ? tid - uc * nc : 0;
    const size_t urow_i = static_cast<size_t>(uc) * a.d + i0 + ucol;
    const bool up1 = a.up_q && a.lr == 64;  // one q4 group per up row: prefetched
    uint32_t uw[8];
    float usg = 0.f, ubg = 0.f;
    if (urow && up1) {
        const uint4 qa = *reinterpret_cast<const uint4 *>(a.up_q + urow_i * 8);
        const uint4 qb = *reinterpret_cast<const uint4 *>(a.up_q + urow_i * 8 + 4);
        uw[0] = qa.x, uw[1] = qa.y, uw[2] = qa.z, uw[3] = qa.w;
        uw[4] = qb.x, uw[5] = qb.y, uw[6] = qb.z, uw[7] = qb.w;
        usg = bf16f(a.up_s[urow_i]);
        ubg = a.up_b ? bf16f(a.up_b[urow_i]) : 0.f;
    }
    float nv[kPreH];
#pragma unroll
    for (int u = 0; u < kPreH; ++u) nv[u] = u < nh ? a.norm[256 * u + tid] : 0.f;

    pdl_wait();     // h comes from the previous kernel
    pdl_trigger();  // the block may be scheduled: it waits for this grid before reading mixed
    // every launch adds G to the counter, so it starts at a multiple of G and
    // at most G - 1 of this launch's arrivals precede this read
    if (tid == 0) s_base = ld_acquire64(ctr) / G * G;
    float hv[kPreH];
#pragma unroll
    for (int u = 0; u < kPreH; ++u) hv[u] = u < nh ? a.h[256 * u + tid] : 0.f;

    // sum of squares of each stream in fp64: the thread's values of the
    // stream in ascending order, then the warp and the eight warps
    for (int c = 0; c < a.hc; ++c) {
        double ss = 0.0;
#pragma unroll
        for (int u = 0; u < kPreH; ++u)
            if (u >= c * upc && u < (c + 1) * upc) ss = fma(static_cast<double>(hv[u]), static_cast<double>(hv[u]), ss);
        ss = warp_sum_butterfly(ss);
        if (lane == 0) s_ss[warp][c] = ss;
    }
    __syncthreads();
    if (tid < a.hc) {
        const double tot = ((s_ss[0][tid] + s_ss[1][tid]) + (s_ss[2][tid] + s_ss[3][tid])) +
                           ((s_ss[4][tid] + s_ss[5][tid]) + (s_ss[6][tid] + s_ss[7][tid]));
        s_r[tid] = 1.0f / sqrtf(static_cast<float>(tot) / static_cast<float>(a.d) + 1e-6f);
    }
    __syncthreads();
    for (int c = 0; c < a.hc; ++c) {
        const float rc = s_r[c];
#pragma unroll
        for (int u = 0; u < kPreH; ++u)
            if (u >= c * upc && u < (c + 1) * upc) s_x[256 * u + tid] = hv[u] * rc * nv[u];
    }
    __syncthreads();

    // ---- this CTA's down row (w) or inject stream
    if (q4item) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < kPreWords; ++m) {
            const int wi = w0 + lane + 32 * m;
            if (wi < w1) {
                const uint32_t v = qv[m];
                const float4 x0 = *reinterpret_cast<const float4 *>(s_x + 8 * wi);
                const float4 x1 = *reinterpret_cast<const float4 *>(s_x + 8 * wi + 4);
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                float xq = 0.f, xs = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    xq = fmaf(xv[i], static_cast<float>((v >> (4 * i)) & 0xFu), xq);
                    xs += xv[i];
                }
                acc = fmaf(sv[m], xq, acc);
                if (a.down_b) acc = fmaf(bv[m], xs, acc);
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(QK_FULL, acc, off);
        if (lane == 0) s_part[warp] = acc;
        __syncthreads();
        if (tid == 0) {
            float v = 0.f;
            for (int w = 0; w < 8; ++w) v += s_part[w];
            v *= inv_hc;
            a.W[r] = v / (1.0f + expf(-v));
        }
    } else if (canon_item) {
        double acc = 0.0;
#pragma unroll
        for (int u = 0; u < kPreH; ++u) {
            const int k = 256 * u + 8 * lane + warp;
            if (k < hd) acc = fma(static_cast<double>(s_x[k]), bf16_to_f64(wv[u]), acc);
        }
        s_acc[warp][lane] = acc;
        __syncthreads();
        if (warp == 0) {
            const double f = ((s_acc[0][lane] + s_acc[1][lane]) + (s_acc[2][lane] + s_acc[3][lane])) +
                             ((s_acc[4][lane] + s_acc[5][lane]) + (s_acc[6][lane] + s_acc[7][lane]));
            const float v = static_cast<float>(warp_sum_butterfly(f));
            if (lane == 0) {
                if (r >= a.lr) {
                    a.INJ[r - a.lr] = 2.0f / (1.0f + expf(-(v * inv_hc)));
                } else {
                    const float u = v * inv_hc;
                    a.W[r] = u / (1.0f + expf(-u));
                }
            }
        }
    }

    grid_arrive(ctr);
    grid_wait(ctr, s_base + G, err);

    // ---- up rows and mixed for columns [i0, i1)
    for (int j = tid; j < a.lr; j += kPreThreads) s_w[j] = __ldcg(a.W + j);
    __syncthreads();
    if (urow) {
        float u;
        if (up1) {
            // up_row's arithmetic for one group
            float xq = 0.f, xs = 0.f;
            for (int i2 = 0; i2 < 64; ++i2) xs += s_w[i2];
#pragma unroll
            for (int wd = 0; wd < 8; ++wd)
#pragma unroll
                for (int bb = 0; bb < 8; ++bb)
                    xq = fmaf(s_w[8 * wd + bb], static_cast<float>((uw[wd] >> (4 * bb)) & 0xFu), xq);
            u = fmaf(usg, xq, 0.f);
            if (a.up_b) u = fmaf(ubg, xs, u);
        } else {
            u = up_row(a, urow_i, s_w);
        }
        const float tmp = 1.0f / (1.0f + expf(-u));
        s_m[uc][ucol] = tmp * s_x[urow_i];
    }
    __syncthreads();
    if (tid < nc) {
        float acc = 0.f;
        for (int c = 0; c < a.hc; ++c) acc += s_m[c][tid];
        a.mixed[i0 + tid] = acc / static_cast<float>(a.hc);
    }
}

}  // namespace

// Weights and workspaces of one layer's hyper connection (device pointers).
extern "C" int qk_hc_smem_ok(int d, int hc) {
    return static_cast<size_t>(hc) * d * sizeof(float) <= 200 * 1024 ? 1 : 0;
}

extern "C" int qk_hc_prepare(int d, int hc) {
    const size_t smem = static_cast<size_t>(hc) * d * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void *>(&k_hc_down),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(reinterpret_cast<const void *>(&k_hc_pre1),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem + 1024 * sizeof(float)));
    return e;
}

cudaError_t qk_launch_raw(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream,
                          int pdl, void **args);

extern "C" int qk_launch_hc_pre(const qk_hc_dev *w, const float *h, int n, float *W, float *R,
                                float *INJ, float *mixed, unsigned long long *ctr, int *err,
                                int num_sms, void *stream) {
    if (n <= 0) return 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    HcArgs a;
    a.d = w->d;
    a.hc = w->hc;
    a.lr = w->lowrank;
    a.norm = w->norm;
    a.down_q = w->down_q;
    a.down_s = w->down_s;
    a.down_b = w->down_b;
    a.down_bf = w->down_bf;
    a.up_q = w->up_q;
    a.up_s = w->up_s;
    a.up_b = w->up_b;
    a.up_bf = w->up_bf;
    a.inject = w->inject;
    a.h = h;
    a.W = W;
    a.R = R;
    a.INJ = INJ;
    a.mixed = mixed;
    const size_t smem = static_cast<size_t>(a.hc) * a.d * sizeof(float);
    if (n == 1 && ctr && num_sms >= a.lr + a.hc && a.hc <= 8 && a.lr <= 1024 &&
        a.d <= kPreCols * num_sms && a.d % kPreThreads == 0 && a.hc * a.d <= kPreThreads * kPreH &&
        a.hc * ((a.d + num_sms - 1) / num_sms) <= kPreThreads) {
        void *args[] = {&a, &ctr, &err};
        return qk_launch_raw(reinterpret_cast<const void *>(&k_hc_pre1), dim3(num_sms), dim3(kPreThreads),
                             smem + static_cast<size_t>(a.lr) * sizeof(float), st, 1, args);
    }
    const int nb = (a.lr + 3) / 4;
    k_hc_down<<<dim3(nb + 1, n), 128, smem, st>>>(a, nb);
    k_hc_up<<<dim3((a.d + 127) / 128, n), 128, a.lr * sizeof(float), st>>>(a);
    return cudaGetLastError();
}

extern "C" int qk_launch_hc_inject(float *h, const float *INJ, const float *y, int n, int hc, int d,
                                   void *stream) {
    if (n <= 0) return 0;
    void *args[] = {&h, &INJ, &y, &hc, &d};
    return qk_launch_raw(reinterpret_cast<const void *>(&k_hc_inject), dim3((hc * d + 1023) / 1024, n),
                         dim3(256), 0, stream, 1, args);
}
