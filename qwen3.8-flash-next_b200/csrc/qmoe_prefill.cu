// qmoe_prefill.cu - the multi-token MoE layer on the 5th-generation tensor
// cores (tcgen05, accumulators in tensor memory).
//
// Reference path: moe_forward, c/src/model.c:1281-1405, for n > 1 tokens.
// After routing (router + top-k kernels in qmoe_kernels.cu):
//   k_count      per-expert token counts                 (model.c:1321-1332)
//   k_plan       row offsets of each expert group and the M-tile list
//   k_place      token -> row permutation per expert (warp-aggregated
//                atomics; model.c:1354-1367 gathers the same rows)
//   k_gather     x rows -> fp16 A operand, grouped by expert; the shared
//                expert's group is every token in order
//   k_gemm<GU>   H = SiLU(X_e Wg_e^T) * (X_e Wu_e^T)           (model.c:1371-1374)
//   k_gemm<DN>   Y = H_e Wd_e^T                                (model.c:1375)
//   k_combine    out[t] = sum_s w[t,s] Y[row(t,s)] + sigmoid(g_t) Y_sh[t]
//                in a fixed order (model.c:1376-1386, :1396-1402)
//
// Grouped GEMM (one persistent kernel, one CTA per SM, 14 warps):
//   warp 0       TMA producer: the A tile (128 rows x 64 fp16, 128-byte
//                swizzle) and the packed q4 rows + scales of the B tile
//   warp 1       allocates 512 TMEM columns; one thread issues tcgen05.mma
//                (M=128, N=256, K=16 x 4 per K step) and tcgen05.commit
//   warps 2-9    dequantise q4 -> fp16 into the canonical K-major 128-byte
//                swizzled layout (w = q*s + b, exact for b = -8s), one B row
//                per thread; two warps per scheduler hide each other's latency
//   warps 10-13  epilogue: tcgen05.ld of the accumulator (double-buffered in
//                TMEM); gate/up: SiLU(g)*u stored as fp16 (the down GEMM's A
//                operand); down: fp32 stores (keeps the combine at fp32)
// Measured per K step on config 2 before the dequantisers were doubled: the
// MMA issue ran at the tensor pipe's full rate and waited 31% of the time for
// dequantised B tiles and 17% for TMA data. Every wait is bounded.
//
// Inside each 8-element chunk along K, the fp16 operands use the element
// order [0,4,1,5,2,6,3,7]: the dequantiser then builds two fp16 values per
// LOP3 (nibbles i and i+4 of a q4 word). X and H are written in the same
// order, so the products pair up as in the natural order.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qmoe_dev.cuh"

using namespace qk;

cudaError_t qk_launch_raw(const void *fn, dim3 grid, dim3 block, size_t smem, void *stream,
                          int pdl, void **args);

namespace {

constexpr int BM = 128;           // token rows per tile
constexpr int BK = 64;            // K per stage: one 128-byte swizzle row of fp16
constexpr int BN = 256;           // accumulator columns (gate|up, or down outputs)
constexpr int kThreads = 448;     // 14 warps
constexpr int kDeqWarps = 8;      // warps 2 .. 9
constexpr int kA = BM * BK * 2;   // 16 KB
constexpr int kBf = BN * BK * 2;  // 32 KB
constexpr int kBq = BN * 32;      // 8 KB packed q4
constexpr int kBs = BN * 16;      // 4 KB scales
// Two rings in shared memory. The raw ring takes the TMA loads of one K step
// (A tile, packed q4 rows, scales) and is released by the MMA; the Bf ring
// holds two dequantised B tiles, written by the dequantisers and released by
// the MMA too, so dequantisation runs ahead of the MMA while the raw ring
// prefetches further. The down GEMM's A operand is H as an fp16 hi/lo pair
// (H = hi + lo to about 22 significant bits): two A tiles per raw stage and
// two MMAs per K step against the same dequantised B tile.
// MODE 2 is the router: A = x as a bf16 hi/lo pair, B = the bf16 router rows
// loaded by TMA straight into the swizzled layout (no dequantisation): its
// raw stage holds A and B, and there is no Bf ring.
// MODE 3 is gate/up for fp32 activations: A = x as an fp16 hi/lo pair (two
// MMAs per K step, as the down GEMM); MODE 0 takes activations that fp16
// holds exactly (bf16 or fp16 inputs) as one plane.
constexpr int kMaxNR = 5;
template <int MODE>
struct Cfg {
    static constexpr bool GU = MODE == 0 || MODE == 3;  // gate/up (SiLU x up epilogue)
    static constexpr int A = MODE ? 2 * kA : kA;
    static constexpr int Raw = MODE == 2 ? A + kBf : A + kBq + kBs;
    static constexpr int NR = MODE == 0 ? 5 : 3;
    static constexpr int Smem = NR * Raw + (MODE == 2 ? 0 : 2 * kBf) + (GU ? 0 : 4 * 4096) +
                                1024;  // + alignment slack
};

struct MTile {
    int m0;    // first row in the grouped buffers
    int rows;  // valid rows (<= 128)
    int slot;  // pool slot of the expert
    int ex;    // the expert (-1: the shared expert)
};

struct GemmArgs {
    int mode;   // 0: gate/up, 1: down, 2: router
    int KB;     // K / 64
    int ksplit; // router only: K split over this many tiles (0 or 1: none)
    int NT;     // N-tiles per M-tile
    int ld_out; // output row length (elements)
    int n_cols; // fp32 outputs: columns that exist (a multiple of 16)
    int d, I;
    const MTile *tiles;
    const int *n_mtiles;
    int rows_max;       // rows of one plane of the grouped buffers
    size_t lo_plane;    // gate/up: element offset of H's lo plane
    __half *out;   // gate/up: H (fp16 hi and lo planes, permuted chunks)
    float *outf;   // down: Y (fp32)
    int *err;
};

QK_DEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
QK_DEV __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// One q4 word (8 nibbles, k = 8c..8c+7) -> 8 fp16 in the order
// [0,4,1,5,2,6,3,7], each w = q*s + b (one rounding; exact when b = -8s).
QK_DEV uint4 dequant_word(uint32_t w, __half2 s2, __half2 b2) {
    const __half2 k1024 = u2h(0x64006400u);   // {1024, 1024}
    const __half2 k16th = u2h(0x2C002C00u);   // {1/16, 1/16}
    const __half2 km64 = u2h(0xD400D400u);    // {-64, -64}
    const uint32_t w8 = w >> 8;
    const __half2 q04 = __hsub2(u2h((w & 0x000F000Fu) | 0x64006400u), k1024);
    const __half2 q15 = __hfma2(u2h((w & 0x00F000F0u) | 0x64006400u), k16th, km64);
    const __half2 q26 = __hsub2(u2h((w8 & 0x000F000Fu) | 0x64006400u), k1024);
    const __half2 q37 = __hfma2(u2h((w8 & 0x00F000F0u) | 0x64006400u), k16th, km64);
    uint4 o;
    o.x = h2u(__hfma2(q04, s2, b2));
    o.y = h2u(__hfma2(q15, s2, b2));
    o.z = h2u(__hfma2(q26, s2, b2));
    o.w = h2u(__hfma2(q37, s2, b2));
    return o;
}

// Row r of a K-major, 128-byte-swizzled tile: 16-byte chunk c lives at
// (r / 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) * 16).
QK_DEV uint32_t sw128(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

QK_DEV void dequant_row(const uint8_t *q32, float s, float b, uint8_t *bf, int r) {
    const uint4 qa = *reinterpret_cast<const uint4 *>(q32);
    const uint4 qb = *reinterpret_cast<const uint4 *>(q32 + 16);
    const __half2 s2 = __float2half2_rn(s), b2 = __float2half2_rn(b);
    const uint32_t wd[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4 *>(bf + sw128(r, c)) = dequant_word(wd[c], s2, b2);
}

// The 16 values v (natural order, columns j0..j0+15) -> two 16-byte chunks
// in the order [0,4,1,5,2,6,3,7].
QK_DEV void pack_perm16(const float *v, uint4 *o) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float *p = v + 8 * h;
        o[h].x = h2u(__floats2half2_rn(p[0], p[4]));
        o[h].y = h2u(__floats2half2_rn(p[1], p[5]));
        o[h].z = h2u(__floats2half2_rn(p[2], p[6]));
        o[h].w = h2u(__floats2half2_rn(p[3], p[7]));
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
           const __grid_constant__ CUtensorMap tmS, GemmArgs g) {
    constexpr int NR = Cfg<MODE>::NR;
    constexpr int kAm = Cfg<MODE>::A;
    constexpr int kRaw = Cfg<MODE>::Raw;
    constexpr bool kDeq = MODE != 2;
    constexpr bool kGU = Cfg<MODE>::GU;
    extern __shared__ uint8_t smem_raw[];
    // raw ring: TMA in, released by the MMA; Bf ring: dequantised B tiles
    __shared__ uint64_t raw_full[kMaxNR], raw_empty[kMaxNR], bf_full[2], bf_empty[2];
    __shared__ uint64_t acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag_;
    volatile int &abort_flag = abort_flag_;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *bf_base = smem + NR * kRaw;  // two dequantised B tiles (MODE 0, 1)
    // fp32 epilogue staging (MODE 1, 2): 4 KB per epilogue warp
    uint8_t *stg_base = bf_base + (MODE == 2 ? 0 : 2 * kBf);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < NR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bf_full[b], kDeqWarps);
            mbar_init(&bf_empty[b], 1);
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(&drain, 1);
        abort_flag = 0;
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    // the router (MODE 2) may split K over KS tiles that add into zeroed outputs
    const int KS = (MODE == 2 && g.ksplit > 1) ? g.ksplit : 1;
    const int ntiles = *g.n_mtiles * g.NT * KS;
    const int KB = g.KB / KS;

    if (warp == 0) {
        // ---------------- TMA producer: the raw ring
        if (lane == 0) {
            int it = 0;
            int last_it[kMaxNR];
            for (int s = 0; s < NR; ++s) last_it[s] = -1;
            for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x) {
                const MTile mt = g.tiles[tile / (g.NT * KS)];
                const int nt = (tile / KS) % g.NT;
                const int kb0 = (tile % KS) * KB;
                for (int kb = kb0; kb < kb0 + KB; ++kb, ++it) {
                    const int s = it % NR;
                    const uint32_t ph = (it / NR) & 1;
                    if (!mbar_wait(&raw_empty[s], ph ^ 1)) {
                        atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                        abort_flag = 1;
                        break;
                    }
                    uint8_t *A = smem + s * kRaw;
                    uint8_t *Bq = A + kAm, *Bs = Bq + kBq;
                    if (kGU) {
                        mbar_expect_tx(&raw_full[s], kAm + 2 * (128 * 32) + 128 * 16);
                        tma_load_2d(A, &tmA, kb * BK, mt.m0, &raw_full[s]);  // (hi)
                        if (MODE == 3)
                            tma_load_2d(A + kA, &tmA, kb * BK, g.rows_max + mt.m0, &raw_full[s]);  // lo
                        tma_load_3d(Bq, &tmQ, kb * 32, nt * 128, mt.slot, &raw_full[s]);
                        tma_load_3d(Bq + 128 * 32, &tmQ, g.d / 2 + kb * 32, nt * 128, mt.slot,
                                    &raw_full[s]);
                        tma_load_3d(Bs, &tmS, g.d + 16 * (kb >> 1), nt * 128, mt.slot, &raw_full[s]);
                    } else if (MODE == 1) {
                        mbar_expect_tx(&raw_full[s], 2 * kA + 256 * 32 + 256 * 16);
                        tma_load_2d(A, &tmA, kb * BK, mt.m0, &raw_full[s]);                   // hi
                        tma_load_2d(A + kA, &tmA, kb * BK, g.rows_max + mt.m0, &raw_full[s]);  // lo
                        tma_load_3d(Bq, &tmQ, kb * 32, nt * 256, mt.slot, &raw_full[s]);
                        tma_load_3d(Bs, &tmS, g.I / 2 + 16 * (kb >> 2), nt * 256, mt.slot,
                                    &raw_full[s]);
                    } else {
                        mbar_expect_tx(&raw_full[s], 2 * kA + kBf);
                        tma_load_2d(A, &tmA, kb * BK, mt.m0, &raw_full[s]);                   // hi
                        tma_load_2d(A + kA, &tmA, kb * BK, g.rows_max + mt.m0, &raw_full[s]);  // lo
                        tma_load_2d(A + kAm, &tmQ, kb * BK, nt * 256, &raw_full[s]);         // router rows
                    }
                    last_it[s] = it;
                }
            }
            // every load this thread issued has landed before the CTA exits
            for (int s = 0; s < NR; ++s)
                if (last_it[s] >= 0) mbar_wait(&raw_full[s], (last_it[s] / NR) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        const uint32_t idesc = idesc_f16(BM, BN, MODE == 2);
        int it = 0, lt = 0;
        for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x, ++lt) {
            const int buf = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&acc_empty[buf], aph ^ 1)) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const uint32_t dt = tmem + buf * BN;
            bool ok = true;
            for (int kb = 0; kb < KB; ++kb, ++it) {  // (kb counts from the split's first step)
                const int s = it % NR, b = it & 1;
                const uint32_t ph = (it / NR) & 1, bph = (it >> 1) & 1;
                if (!mbar_wait(&raw_full[s], ph) || (kDeq && !mbar_wait(&bf_full[b], bph))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a0 = smem_addr(smem + s * kRaw);
                    const uint32_t b0 = kDeq ? smem_addr(bf_base + b * kBf) : a0 + kAm;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        umma_f16(dt, sdesc_sw128(a0 + kk * 32), sdesc_sw128(b0 + kk * 32), idesc,
                                 (kb | kk) != 0);
                        if (MODE != 0)  // lo plane of the A operand, same B
                            umma_f16(dt, sdesc_sw128(a0 + kA + kk * 32), sdesc_sw128(b0 + kk * 32),
                                     idesc, 1u);
                    }
                    umma_commit(&raw_empty[s]);
                    if (kDeq) umma_commit(&bf_empty[b]);
                }
                __syncwarp();
            }
            if (!ok) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            if (lane == 0) umma_commit(&acc_full[buf]);
            __syncwarp();
        }
        // every MMA this thread issued has completed before TMEM is freed
        if (lane == 0) {
            umma_commit(&drain);
            mbar_wait(&drain, 0);
        }
        __syncwarp();
    } else if (warp < 2 + kDeqWarps) {
        // ---------------- dequantisers: 256 threads, B row t each, from raw
        // stage s into Bf tile b (the router's B tile arrives ready)
        const int t = tid - 64;
        const int dq_tiles = kDeq ? ntiles : 0;
        int it = 0;
        for (int tile = blockIdx.x; tile < dq_tiles && !abort_flag; tile += gridDim.x) {
            bool ok = true;
            for (int kb = 0; kb < KB; ++kb, ++it) {
                const int s = it % NR, b = it & 1;
                const uint32_t ph = (it / NR) & 1, bph = (it >> 1) & 1;
                if (!mbar_wait(&raw_full[s], ph) || !mbar_wait(&bf_empty[b], bph ^ 1)) {
                    ok = false;
                    break;
                }
                uint8_t *Bq = smem + s * kRaw + kAm, *Bs = Bq + kBq;
                uint8_t *Bf = bf_base + b * kBf;
                if (kGU) {
                    // gate row r -> B row r, up row r -> B row 128 + r; the 16
                    // scale bytes of row r hold the quads of groups 2j and 2j+1
                    const int r = t & 127;
                    const uint2 quad = *reinterpret_cast<const uint2 *>(Bs + r * 16 + 8 * (kb & 1));
                    const uint32_t sb = t < 128 ? quad.x : quad.y;
                    dequant_row(Bq + t * 32, bf16lo(sb), bf16hi(sb), Bf, t);
                } else {
                    const uint32_t pr = *reinterpret_cast<const uint32_t *>(Bs + t * 16 + 4 * (kb & 3));
                    dequant_row(Bq + t * 32, bf16lo(pr), bf16hi(pr), Bf, t);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bf_full[b]);
            }
            if (!ok) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
        }
    } else {
        // ---------------- epilogue: 128 threads = 128 accumulator rows
        const int q = warp & 3;  // TMEM lanes [32q, 32q + 32)
        const int row = 32 * q + lane;
        int lt = 0;
        for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x, ++lt) {
            const MTile mt = g.tiles[tile / (g.NT * KS)];
            const int nt = (tile / KS) % g.NT;
            const int buf = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&acc_full[buf], aph)) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * BN;
            const bool live = row < mt.rows;
            const size_t orow_i = static_cast<size_t>(mt.m0 + (live ? row : 0)) * g.ld_out;
            if (kGU) {
                __half *orow = g.out + orow_i;
                for (int c = 0; c < 128; c += 16) {
                    float gv[16], uv[16], hv[16];
                    tmem_ld16(tbase + c, gv);
                    tmem_ld16(tbase + 128 + c, uv);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i) hv[i] = (gv[i] / (1.0f + expf(-gv[i]))) * uv[i];
                    // hi = fp16(h), lo = fp16(h - hi): the pair carries h to ~22 bits
                    float lv[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) lv[i] = hv[i] - __half2float(__float2half_rn(hv[i]));
                    uint4 o[2], ol[2];
                    pack_perm16(hv, o);
                    pack_perm16(lv, ol);
                    if (live) {
                        uint4 *dst = reinterpret_cast<uint4 *>(orow + nt * 128 + c);
                        dst[0] = o[0];
                        dst[1] = o[1];
                        uint4 *dl = reinterpret_cast<uint4 *>(orow + g.lo_plane + nt * 128 + c);
                        dl[0] = ol[0];
                        dl[1] = ol[1];
                    }
                }
            } else {
                // fp32 out, 32 columns at a time through this warp's 4 KB of
                // shared memory (float4 index XOR row % 8: no bank conflicts),
                // so each store instruction writes 4 full 128-byte row pieces
                float4 *stg = reinterpret_cast<float4 *>(stg_base + q * 4096);
                for (int c = 0; c < 256; c += 32) {
                    float yv[32];
                    tmem_ld16(tbase + c, yv);
                    tmem_ld16(tbase + c + 16, yv + 16);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        stg[lane * 8 + (j ^ (lane & 7))] =
                            make_float4(yv[4 * j], yv[4 * j + 1], yv[4 * j + 2], yv[4 * j + 3]);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = 4 * i + (lane >> 3), j = lane & 7;
                        const int col = nt * 256 + c + 4 * j;
                        const float4 v = stg[r * 8 + (j ^ (r & 7))];
                        if (32 * q + r < mt.rows && col < g.n_cols) {
                            float *o = g.outf + static_cast<size_t>(mt.m0 + 32 * q + r) * g.ld_out + col;
                            if (KS > 1) {
                                atomicAdd(o, v.x);
                                atomicAdd(o + 1, v.y);
                                atomicAdd(o + 2, v.z);
                                atomicAdd(o + 3, v.w);
                            } else {
                                *reinterpret_cast<float4 *>(o) = v;
                            }
                        }
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    // drain: let every issued TMA load and MMA finish before TMEM and shared
    // memory go away (bounded)
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// Grouped GEMM for small groups (at most NS = 32 rows per tile): the operands
// swap roles. A = 128 dequantised weight rows (gate, up or down rows, the B
// tile of k_gemm), kept in tensor memory; B = the group's token rows (x or
// H) from shared memory, the hi and lo planes side by side in N (one plane:
// N = the rows). Per 16-wide K slice and half of the 256-row weight tile
// one MMA of M=128 x N x K=16; D[weight row][token] sits in TMEM lanes =
// weight rows and the epilogue writes it transposed (token rows of H or Y),
// adding the hi and lo columns. Keeping the weights out of shared memory
// matters here: with them there, the operand reads of these small MMAs and
// the dequantisers' stores took the shared-memory bandwidth and set the
// pace. TMEM: accumulators in columns [0, 256) (2 buffers x 2 halves x 64),
// four dequantised weight buffers in [256, 512) (2 halves x 32 columns).
//
// A raw stage holds KS = 4 K steps. The packed q4 words of its 256 weight
// rows arrive as one 128-byte-wide box per 128 rows (128-byte swizzle, so
// the dequantisers' reads of 32 bytes per row and step spread over the
// banks) and the scales as one 32-byte box: 2 + 1 loads for 4 steps,
// where one box per step and per row block cost a TMA row request for
// every 32 (or 16) bytes. Tiles of at most 8 rows (most groups at batch
// decode sizes) load 8-row token boxes and run N = 16 (8 hi + 8 lo
// columns), so their token traffic is a quarter of a 32-row tile's.
// Warp roles and bounded waits as k_gemm; MODE 0 / 3 gate/up (x one plane /
// hi+lo), 1 down (H hi+lo).
constexpr int NS = 32;                    // token rows per small tile
constexpr int NS8 = 8;                    // rows of a narrow tile (8-row token boxes)
constexpr int kSmallMax = 2 * NS;         // largest group planned as small tiles
constexpr int kXs = NS * BK * 2;          // 4 KB: one plane of the token tile, one K step
constexpr int kNbT = 4;                   // dequantised weight buffers in TMEM
constexpr int kThreadsSw = kThreads + 32; // a second MMA-issuing warp (warp 14)
constexpr int KS = 4;                     // K steps per raw stage
template <int MODE>
struct CfgS {
    static constexpr bool GU = MODE != 1;
    static constexpr int Xr = KS * 2 * kXs;  // 32 KB: KS steps x (hi, lo) planes x 32 rows
    static constexpr int Qr = 256 * 128;     // 32 KB: 256 weight rows x 128 bytes (KS steps of q4)
    static constexpr int Sr = 256 * 32;      // 8 KB: scales of KS steps (GU: 128 rows x 32 B)
    static constexpr int Raw = Xr + Qr + Sr; // 72 KB (1024-aligned)
    static constexpr int NR = 3;
    static constexpr int Smem = NR * Raw + 1024;
};

template <int MODE>
__global__ void __launch_bounds__(kThreadsSw, 1)
    k_gemm_sw(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmX8,
              const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmS,
              GemmArgs g) {
    constexpr int NR = CfgS<MODE>::NR;
    constexpr int kRaw = CfgS<MODE>::Raw;
    constexpr int kXr = CfgS<MODE>::Xr, kQr = CfgS<MODE>::Qr;
    constexpr bool kGU = CfgS<MODE>::GU;
    constexpr bool kLo = MODE != 0;
    extern __shared__ uint8_t smem_raw[];
    // raw_full[s] / raw_free[s]: stage s loaded / its last step's MMAs done
    // (one commit from each issuer); wfree[b]: the MMAs that read weight
    // buffer b completed (one commit from each issuer); bf_full[b]: weight
    // buffer b written by the eight dequantising warps
    __shared__ uint64_t raw_full[NR], raw_free[NR], wfree[kNbT], bf_full[kNbT];
    __shared__ uint64_t acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag_;
    volatile int &abort_flag = abort_flag_;
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < NR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_free[s], 2);
        }
        for (int b = 0; b < kNbT; ++b) {
            mbar_init(&bf_full[b], kDeqWarps);
            mbar_init(&wfree[b], 2);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 2);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(&drain, 2);
        abort_flag = 0;
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    const uint32_t tmem_w = tmem + 256;  // dequantised weight buffers
    const int ntiles = *g.n_mtiles * g.NT;
    const int KB = g.KB;
    const int nst = (KB + KS - 1) / KS;  // stages per tile

    if (warp == 0) {
        // ---------------- TMA producer: one raw stage per KS K steps
        if (lane == 0) {
            int sg = 0;
            int last_sg[NR];
            for (int s = 0; s < NR; ++s) last_sg[s] = -1;
            for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x) {
                const MTile mt = g.tiles[tile / g.NT];
                const int nt = tile % g.NT;
                const bool narrow = mt.rows <= NS8;
                const uint32_t xbox = (narrow ? NS8 : NS) * BK * 2;
                const int lo_off = narrow ? NS8 * 128 : kXs;  // lo plane right after the hi rows
                for (int st = 0; st < nst; ++st, ++sg) {
                    const int s = sg % NR;
                    if (!mbar_wait(&raw_free[s], ((sg / NR) & 1) ^ 1)) {
                        atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                        abort_flag = 1;
                        break;
                    }
                    const int kb0 = st * KS, nk = min(KS, KB - kb0);
                    uint8_t *X = smem + s * kRaw, *Q = X + kXr, *S = Q + kQr;
                    mbar_expect_tx(&raw_full[s], nk * xbox * (kLo ? 2 : 1) + 256 * 128 + (kGU ? 128 : 256) * 32);
                    for (int kk = 0; kk < nk; ++kk) {
                        uint8_t *Xk = X + kk * 2 * kXs;
                        const int kb = kb0 + kk;
                        tma_load_2d(Xk, narrow ? &tmX8 : &tmX, kb * BK, mt.m0, &raw_full[s]);  // (hi)
                        if (kLo)
                            tma_load_2d(Xk + lo_off, narrow ? &tmX8 : &tmX, kb * BK, g.rows_max + mt.m0,
                                        &raw_full[s]);
                    }
                    if (kGU) {
                        tma_load_3d(Q, &tmQ, kb0 * 32, nt * 128, mt.slot, &raw_full[s]);                    // gate
                        tma_load_3d(Q + 128 * 128, &tmQ, g.d / 2 + kb0 * 32, nt * 128, mt.slot, &raw_full[s]);  // up
                        tma_load_3d(S, &tmS, g.d + 8 * kb0, nt * 128, mt.slot, &raw_full[s]);
                    } else {
                        tma_load_3d(Q, &tmQ, kb0 * 32, nt * 256, mt.slot, &raw_full[s]);
                        tma_load_3d(Q + 128 * 128, &tmQ, kb0 * 32, nt * 256 + 128, mt.slot, &raw_full[s]);
                        tma_load_3d(S, &tmS, g.I / 2, nt * 256, mt.slot, &raw_full[s]);
                    }
                    last_sg[s] = sg;
                }
            }
            for (int s = 0; s < NR; ++s)
                if (last_sg[s] >= 0) mbar_wait(&raw_full[s], (last_sg[s] / NR) & 1);
        }
    } else if (warp == 1 || warp == kThreads / 32) {
        // ---------------- MMA issuers: warp 1 the first 128 weight rows, the
        // last warp the second (one issuing thread runs small MMAs at about
        // half the tensor pipe's rate; two keep it busy)
        const int hh = warp == 1 ? 0 : 1;
        int it = 0, sg = 0, lt = 0;
        for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x, ++lt) {
            const MTile mt = g.tiles[tile / g.NT];
            const bool narrow = mt.rows <= NS8;
            const int ns = narrow ? NS8 : NS;
            const uint32_t idesc = idesc_f16(BM, kLo ? 2 * ns : (narrow ? 16 : NS));
            const int buf = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&acc_empty[buf], aph ^ 1)) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const uint32_t dt = tmem + buf * 128;
            bool ok = true;
            for (int st = 0; st < nst && ok; ++st, ++sg) {
                const int s = sg % NR;
                const int nk = min(KS, KB - st * KS);
                if (!mbar_wait(&raw_full[s], (sg / NR) & 1)) {
                    ok = false;
                    break;
                }
                for (int kk = 0; kk < nk; ++kk, ++it) {
                    const int b = it % kNbT;
                    if (!mbar_wait(&bf_full[b], (it / kNbT) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t x0 = smem_addr(smem + s * kRaw + kk * 2 * kXs);
                        const uint32_t w0 = tmem_w + b * 64;
#pragma unroll
                        for (int kq = 0; kq < BK / 16; ++kq)
                            umma_f16_ts(dt + hh * 64, w0 + hh * 32 + kq * 8, sdesc_sw128(x0 + kq * 32), idesc,
                                        (st | kk | kq) != 0);
                        umma_commit(&wfree[b]);
                        if (kk == nk - 1) umma_commit(&raw_free[s]);
                    }
                    __syncwarp();
                }
            }
            if (!ok) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            if (lane == 0) umma_commit(&acc_full[buf]);
            __syncwarp();
        }
        if (lane == 0) {
            umma_commit(&drain);
            mbar_wait(&drain, 0);
        }
        __syncwarp();
    } else if (warp < 2 + kDeqWarps) {
        // ---------------- dequantisers: weight row r of the 256-row tile =
        // TMEM lane 32 q + lane of half h (warp w reaches lanes 32 (w % 4)..)
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int r = h * 128 + 32 * q + lane;
        const int rr = r & 127;
        const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
        int it = 0, sg = 0;
        for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x) {
            bool ok = true;
            for (int st = 0; st < nst && ok; ++st, ++sg) {
                const int s = sg % NR;
                const int nk = min(KS, KB - st * KS);
                if (!mbar_wait(&raw_full[s], (sg / NR) & 1)) {
                    ok = false;
                    break;
                }
                const uint8_t *Qrow = smem + s * kRaw + kXr + r * 128;  // 128-byte swizzled row
                const uint8_t *S = smem + s * kRaw + kXr + kQr;
                for (int kk = 0; kk < nk; ++kk, ++it) {
                    const int b = it % kNbT;
                    // weight buffer b is free once the MMAs of step it - kNbT are done
                    const int pv = it - kNbT;
                    if (pv >= 0 && !mbar_wait(&wfree[b], (pv / kNbT) & 1)) {
                        ok = false;
                        break;
                    }
                    uint32_t sb;
                    if (kGU) {
                        const uint2 quad = *reinterpret_cast<const uint2 *>(S + rr * 32 + 8 * kk);
                        sb = h == 0 ? quad.x : quad.y;
                    } else {
                        sb = *reinterpret_cast<const uint32_t *>(S + r * 32 + 4 * (st * KS + kk));
                    }
                    const uint4 qa = *reinterpret_cast<const uint4 *>(Qrow + (((2 * kk) ^ (r & 7)) << 4));
                    const uint4 qb = *reinterpret_cast<const uint4 *>(Qrow + (((2 * kk + 1) ^ (r & 7)) << 4));
                    const __half2 s2 = __float2half2_rn(bf16lo(sb)), b2 = __float2half2_rn(bf16hi(sb));
                    const uint32_t wd[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    uint32_t v[32];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint4 o = dequant_word(wd[c], s2, b2);
                        v[4 * c] = o.x;
                        v[4 * c + 1] = o.y;
                        v[4 * c + 2] = o.z;
                        v[4 * c + 3] = o.w;
                    }
                    tc_fence_after();  // the MMAs that read this buffer before have completed
                    tmem_st32(tmem_w + lane_off + b * 64 + h * 32, v);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bf_full[b]);
                }
            }
            if (!ok) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
        }
    } else if (warp < kThreads / 32) {
        // ---------------- epilogue (warps 10-13): thread = weight row 32q + lane of each
        // half; token columns c (hi) and ns + c (lo)
        const int q = warp & 3;
        const int wr = 32 * q + lane;
        int lt = 0;
        for (int tile = blockIdx.x; tile < ntiles && !abort_flag; tile += gridDim.x, ++lt) {
            const MTile mt = g.tiles[tile / g.NT];
            const int nt = tile % g.NT;
            const bool narrow = mt.rows <= NS8;
            const int buf = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!mbar_wait(&acc_full[buf], aph)) {
                if (lane == 0) {
                    atomicOr(g.err, QK_ERR_TIMEOUT_COPY);
                    abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const uint32_t tb = tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * 128;
            float v0[NS], v1[NS];
            if (narrow) {
                // columns [0, 8) hi and [8, 16) lo (one plane: [0, 8))
                float a0[16], a1[16];
                tmem_ld16(tb, a0);
                tmem_ld16(tb + 64, a1);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < NS8; ++c) {
                    v0[c] = kLo ? a0[c] + a0[NS8 + c] : a0[c];
                    v1[c] = kLo ? a1[c] + a1[NS8 + c] : a1[c];
                }
#pragma unroll
                for (int c = NS8; c < NS; ++c) v0[c] = v1[c] = 0.f;
            } else {
                tmem_ld16(tb, v0);
                tmem_ld16(tb + 16, v0 + 16);
                tmem_ld16(tb + 64, v1);
                tmem_ld16(tb + 64 + 16, v1 + 16);
                tmem_wait_ld();
                if (kLo) {
                    float l0[NS], l1[NS];
                    tmem_ld16(tb + NS, l0);
                    tmem_ld16(tb + NS + 16, l0 + 16);
                    tmem_ld16(tb + 64 + NS, l1);
                    tmem_ld16(tb + 64 + NS + 16, l1 + 16);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < NS; ++c) {
                        v0[c] += l0[c];
                        v1[c] += l1[c];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);  // TMEM free: values are in registers
            if (kGU) {
                // H[token][f], f = nt*128 + wr, fp16 hi/lo at the chunk
                // position of f ([0,4,1,5,2,6,3,7] inside 8-element chunks)
                const int f = nt * 128 + wr, j = f & 7;
                const int col = (f & ~7) + (j < 4 ? 2 * j : 2 * (j - 4) + 1);
#pragma unroll
                for (int c = 0; c < NS; ++c) {
                    if (c < mt.rows) {
                        const float gv = v0[c], uv = v1[c];
                        const float hv = (gv / (1.0f + expf(-gv))) * uv;
                        const __half hi = __float2half_rn(hv);
                        const __half lo = __float2half_rn(hv - __half2float(hi));
                        __half *orow = g.out + static_cast<size_t>(mt.m0 + c) * g.ld_out + col;
                        orow[0] = hi;
                        orow[g.lo_plane] = lo;
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < NS; ++c) {
                    if (c < mt.rows) {
                        float *orow = g.outf + static_cast<size_t>(mt.m0 + c) * g.ld_out + nt * 256;
                        orow[wr] = v0[c];
                        orow[128 + wr] = v1[c];
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

constexpr int kSbThreads = 512;
constexpr int kSbBatch = 8;     // most rows (tokens) of a tile on the CUDA cores
constexpr int kSbGuRows = 32;   // gate/up rows per unit (one 32-element unit of h)
constexpr int kSbDnRows = 128;  // down rows per unit
constexpr int kSbMaxRows = 4;   // default: tiles of more rows stay on the tensor cores

// x of a token: two 8-bit planes of d / 8 words in group-major 16-byte
// chunks (store_word_gx), then {scale, sum} per 64-element group
__host__ __device__ constexpr int sb_xrow(int d) { return (d / 8) * 16 + (d / 64) * 8; }
__host__ __device__ constexpr int sb_hrow(int I) { return (I / 8) * 24 + (I / 32) * 8; }

struct SbArgs {
    const MTile *tiles;       // the light tiles (at most kSbBatch rows of one group)
    const int *n_tiles;
    int nsh;                  // rows [0, nsh) are tokens [0, nsh) (the shared expert)
    const int *perm_tok;      // row -> token for the other rows
    const uint8_t *pool;
    qk_layout L;
    const uint8_t *xq;        // [tokens][sb_xrow(d)]
    uint8_t *hq;              // [rows][sb_hrow(I)]
    float *Y;                 // [rows][d]
    int *ctr;                 // [2]: next unit to take, CTAs done (both 0 between launches)
    int *err;
};

// The staged x and h vectors interleave each plane's words by unit: the 16
// bytes of words 4u, 4u + 1 of every unit u first, then those of words
// 4u + 2, 4u + 3, so that lanes reading consecutive units read consecutive
// 16-byte pieces (no shared-memory bank conflicts). n words a plane.
template <int NB>
QK_DEV void store_word_il(uint2 *planes, int n, int w, const uint2 (&pl)[NB]) {
    const int q = w & 3;
    const size_t pos = static_cast<size_t>(q >> 1) * (n / 2) + 2 * (w >> 2) + (q & 1);
#pragma unroll
    for (int p = 0; p < NB; ++p) planes[static_cast<size_t>(p) * n + pos] = pl[p];
}

template <int NB>
QK_DEV void load_unit_il(const uint2 *planes, int n, int u, uint2 (&v)[NB][4]) {
#pragma unroll
    for (int p = 0; p < NB; ++p) {
        const uint2 *base = planes + static_cast<size_t>(p) * n;
        const uint4 a = reinterpret_cast<const uint4 *>(base)[u];
        const uint4 b = reinterpret_cast<const uint4 *>(base + n / 2)[u];
        v[p][0] = make_uint2(a.x, a.y);
        v[p][1] = make_uint2(a.z, a.w);
        v[p][2] = make_uint2(b.x, b.y);
        v[p][3] = make_uint2(b.z, b.w);
    }
}

// Group-major chunks of a plane of n words (gate/up's x): chunk (q, g), 16
// bytes at (q * n / 8 + g) * 16, holds words 8 g + 2 q and 8 g + 2 q + 1, so
// the lane of group g reads its 8 words as 4 chunks, consecutive lanes
// consecutive chunks.
template <int NB>
QK_DEV void store_word_gx(uint2 *planes, int n, int w, const uint2 (&pl)[NB]) {
    const int g = w >> 3, q = (w & 7) >> 1;
    const size_t pos = (static_cast<size_t>(q) * (n / 8) + g) * 2 + (w & 1);
#pragma unroll
    for (int p = 0; p < NB; ++p) planes[static_cast<size_t>(p) * n + pos] = pl[p];
}

// a (4 unsigned bytes) . b (4 signed bytes) + c
QK_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// sum(q_k x_k) over one 64-element group: q the 8 q4 words w0 (words 0-3),
// w1 (4-7); x 16-bit as a signed hi and an unsigned lo plane, chunk q of each
// holding words 2q, 2q + 1 as {even bytes, odd bytes}. The odd nibbles are
// used in place (w & 0xF0F0F0F0, 16 q) and their sums shifted back once.
// Exact in 32 bits (|sum| < 64 * 15 * 2^15).
QK_DEV int dot_group_x16(const uint4 &w0, const uint4 &w1, const uint4 (&xh)[4], const uint4 (&xl)[4]) {
    const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    int he = 0, ho = 0;
    unsigned le = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t ev = wd[i] & 0x0F0F0F0Fu, oh = wd[i] & 0xF0F0F0F0u;
        const uint4 &ch = xh[i >> 1], &cl = xl[i >> 1];
        const uint32_t hev = (i & 1) ? ch.z : ch.x, hod = (i & 1) ? ch.w : ch.y;
        const uint32_t lev = (i & 1) ? cl.z : cl.x, lod = (i & 1) ? cl.w : cl.y;
        he = __dp4a(static_cast<int>(ev), static_cast<int>(hev), he);
        ho = dp4a_us(oh, hod, ho);
        le = __dp4a(ev, lev, le);
        lo = __dp4a(oh, lod, lo);
    }
    return (he + (ho >> 4)) * 256 + static_cast<int>(le + (lo >> 4));
}

// sum(q_k h_k) over one 16-byte unit (32 nibbles) for 24-bit h (signed hi,
// unsigned mid and lo planes), in units of the scale; the odd nibbles used in
// place as in dot_group_x16. The same value as dot_unit_q<3>.
QK_DEV float dot_unit_h24(const uint4 &w, const uint2 (&v)[3][4]) {
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    int he = 0, ho = 0;
    unsigned me = 0, mo = 0, le = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t ev = wd[i] & 0x0F0F0F0Fu, oh = wd[i] & 0xF0F0F0F0u;
        he = __dp4a(static_cast<int>(ev), static_cast<int>(v[0][i].x), he);
        ho = dp4a_us(oh, v[0][i].y, ho);
        me = __dp4a(ev, v[1][i].x, me);
        mo = __dp4a(oh, v[1][i].y, mo);
        le = __dp4a(ev, v[2][i].x, le);
        lo = __dp4a(oh, v[2][i].y, lo);
    }
    const int hi = he + (ho >> 4);
    const unsigned mid = me + (mo >> 4), low = le + (lo >> 4);
    return fmaf(static_cast<float>(hi), 65536.f, static_cast<float>(mid * 256u + low));
}

// Sums each of v[0 .. N) over an aligned group of W lanes, halving the
// values at each of the first log2 N levels (a lane keeps one half and
// sends the other): log2 N + ... shuffles in all instead of N log2 W. On
// return lane l holds the sum of value (l % W) / (W / N).
template <int N, int W>
QK_DEV float group_sum_tr(float (&v)[N], int lane) {
    constexpr int kLevels = N >= 32 ? 5 : N >= 16 ? 4 : N >= 8 ? 3 : N >= 4 ? 2 : N >= 2 ? 1 : 0;
    static_assert((1 << kLevels) == N && N <= W, "N a power of two, at most W");
#pragma unroll
    for (int lv = 0; lv < kLevels; ++lv) {
        const int c = N >> lv, off = W >> (lv + 1);
        const bool hi = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < c / 2; ++i) {
            const float send = hi ? v[i] : v[i + c / 2];
            const float keep = hi ? v[i + c / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(QK_FULL, send, off);
        }
    }
    float r = v[0];
#pragma unroll
    for (int off = W / N / 2; off >= 1; off >>= 1) r += __shfl_xor_sync(QK_FULL, r, off);
    return r;
}

// NT tokens (jj0 .. jj0 + NT of the staged batch) of the warp's two gate/up
// rows il and il + 16; lane l on the 64-element group l (lanes past the
// groups contribute 0): each token's x is read once for both rows; the 4 NT
// sums (token, row, gate/up) reduced together.
template <int NT>
QK_DEV void sb_gu_tokens(const uint8_t *xs, int xrow, int n, bool act, int lane, int jj0,
                         const uint4 (&gw)[2][2], const uint4 (&uw)[2][2], const uint2 (&sb)[2],
                         float *hbuf, int il) {
    constexpr int N = 4 * NT;
    float v[N];
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = 0.f;
    if (act) {
        const int ng = n / 8;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const uint8_t *xr = xs + (jj0 + t) * xrow;
            const uint4 *ph = reinterpret_cast<const uint4 *>(xr);
            const uint4 *pl = reinterpret_cast<const uint4 *>(xr + n * 8);
            uint4 xh[4], xl[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                xh[q] = ph[q * ng + lane];
                xl[q] = pl[q * ng + lane];
            }
            const float2 xs2 = reinterpret_cast<const float2 *>(xr + n * 16)[lane];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const float dg = static_cast<float>(dot_group_x16(gw[rr][0], gw[rr][1], xh, xl));
                const float du = static_cast<float>(dot_group_x16(uw[rr][0], uw[rr][1], xh, xl));
                v[(t * 2 + rr) * 2] = fmaf(bf16lo(sb[rr].x), dg * xs2.x, bf16hi(sb[rr].x) * xs2.y);
                v[(t * 2 + rr) * 2 + 1] = fmaf(bf16lo(sb[rr].y), du * xs2.x, bf16hi(sb[rr].y) * xs2.y);
            }
        }
    }
    // value k = (t * 2 + row) * 2 + gate/up sits on lanes k (32 / N) ..
    constexpr int kSpan = 32 / N;
    const float r = group_sum_tr<N, 32>(v, lane);
    const float up = __shfl_down_sync(QK_FULL, r, kSpan);
    const int k = lane / kSpan;
    if (lane % kSpan == 0 && (k & 1) == 0) {
        const int t = k >> 2, rr = (k >> 1) & 1;
        hbuf[(jj0 + t) * 32 + il + 16 * rr] = (r / (1.0f + expf(-r))) * up;
    }
}

// NT tile rows of the lane group's P down rows (LPR lanes, lane j on h unit
// j): each row of h read once for the P rows, the P NT sums reduced together.
template <int NT, int P, int LPR>
QK_DEV void sb_dn_tokens(const uint8_t *hs, int hrow, int hn, int upe, int j, int lane, int jj0,
                         const uint4 (&w)[P], const uint32_t (&sb)[P], float *ys, const int (&r)[P]) {
    constexpr int N = NT * P;
    float v[N];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t *hr = hs + (jj0 + t) * hrow;
        uint2 hv[3][4];
        load_unit_il<3>(reinterpret_cast<const uint2 *>(hr), hn, j, hv);
        const float *hsf = reinterpret_cast<const float *>(hr + hn * 24);
        const float hsc = hsf[j], hsm = hsf[upe + j];
#pragma unroll
        for (int p = 0; p < P; ++p)
            v[t * P + p] = fmaf(bf16lo(sb[p]), dot_unit_h24(w[p], hv) * hsc, bf16hi(sb[p]) * hsm);
    }
    constexpr int kSpan = LPR / N;
    const float s = group_sum_tr<N, LPR>(v, lane);
    if (j % kSpan == 0) {
        const int k = j / kSpan, t = k / P, p = k % P;
        int rp = r[0];
#pragma unroll
        for (int q = 1; q < P; ++q)
            if (p == q) rp = r[q];
        if (rp < kSbDnRows) ys[(jj0 + t) * kSbDnRows + rp] = s;
    }
}

// Gate/up: unit = (small tile of at most kSbBatch rows, 32 gate/up rows). A
// stage holds the unit's weight rows and the x of the tile's tokens, both by
// bulk copies on one barrier, the next unit's stage in flight while this one
// computes. Tile descriptors are read two units ahead and the tokens one
// unit ahead, so a unit's copies are issued without a dependent global load.
// Warp w takes rows w and w + 16 (weights in registers), lane l the
// 64-element scale group l (d <= 2048); each token's x is read once for both
// rows (integer dots on 16-bit block fixed point x, as in the decode kernel's
// gateup_row). h goes through one of two buffers, so warp 0 quantises it
// while the others go on.
__host__ __device__ int sb_gu_stage(const qk_layout &L) { return kSbGuRows * L.gu_row + kSbBatch * sb_xrow(L.d); }
int sb_gu_smem(const qk_layout &L) { return 2 * sb_gu_stage(L) + 2 * kSbBatch * 32 * 4; }

// Units are taken in request order from a counter (a.ctr[0]), four ahead of
// the one computing, so CTAs that start late (the SMs of a tensor-core
// kernel running beside this one) take fewer. Unit k's index is requested at
// the top of iteration k - 4 and published in s_u before that iteration's
// block barrier. The last CTA to finish zeroes the counters.
QK_DEV void sb_take_first(int *ctr, int *s_u) {
    if (threadIdx.x == 0)
        for (int i = 0; i < 4; ++i) s_u[i] = atomicAdd(ctr, 1);
    __syncthreads();
}

QK_DEV void sb_finish(int *ctr) {
    if (threadIdx.x == 0 && atomicAdd(ctr + 1, 1) == static_cast<int>(gridDim.x) - 1) {
        atomicExch(ctr, 0);
        atomicExch(ctr + 1, 0);
    }
}

__global__ void __launch_bounds__(kSbThreads, 1) k_sb_gu(SbArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t sbar[2];
    __shared__ int s_u[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const qk_layout &L = a.L;
    const int d = L.d, n = d / 8, xrow = sb_xrow(d), hrow = sb_hrow(L.I);
    const bool act = lane < d / 64;  // lane l: 64-element group l
    const uint32_t wbytes = static_cast<uint32_t>(kSbGuRows * L.gu_row);
    const size_t stage = static_cast<size_t>(sb_gu_stage(L));
    float *hbuf0 = reinterpret_cast<float *>(smem + 2 * stage);  // 2 x [kSbBatch][32]
    if (tid == 0) {
        mbar_init(&sbar[0], 1);
        mbar_init(&sbar[1], 1);
    }
    const int rb_n = L.I / kSbGuRows;
    const int nu = *a.n_tiles * rb_n;
    sb_take_first(a.ctr, s_u);  // (its barrier also publishes the barrier inits)
    auto tile_of = [&](int u) {
        MTile m = {0, 0, 0, 0};
        if (u < nu) m = a.tiles[u / rb_n];
        return m;
    };
    // warp 0 lane l: the token of the tile's row l
    auto tok_of = [&](const MTile &m) {
        int t = 0;
        if (warp == 0 && lane < m.rows) {
            const int r = m.m0 + lane;
            t = r < a.nsh ? r : a.perm_tok[r];
        }
        return t;
    };
    // warp 0: the unit's weights and its tokens' x into stage s
    auto issue = [&](int u, int s, const MTile &mt, int tok) {
        uint8_t *dst = smem + s * stage;
        if (lane == 0) {
            mbar_expect_tx(&sbar[s], wbytes + static_cast<uint32_t>(mt.rows * xrow));
            bulk_load(dst, a.pool + static_cast<size_t>(mt.slot) * L.slot_bytes +
                               static_cast<size_t>(u % rb_n) * kSbGuRows * L.gu_row,
                      wbytes, &sbar[s]);
        }
        __syncwarp();
        if (lane < mt.rows)
            bulk_load(dst + wbytes + lane * xrow, a.xq + static_cast<size_t>(tok) * xrow,
                      static_cast<uint32_t>(xrow), &sbar[s]);
    };
    // units u0 (computing), u1 (its stage in flight), u2 (descriptor and
    // tokens read), u3 (descriptor read)
    int u0 = s_u[0], u1 = s_u[1], u2 = s_u[2], u3 = s_u[3];
    MTile m0 = tile_of(u0), m1 = tile_of(u1), m2 = tile_of(u2);
    int t1 = tok_of(m1);
    if (warp == 0 && u0 < nu) issue(u0, 0, m0, tok_of(m0));
    bool ok = true;
    for (int it = 0; u0 < nu; ++it) {
        const int s = it & 1;
        const MTile mt = m0;
        const int rb = u0 % rb_n;
        if (warp == 0 && u1 < nu) issue(u1, s ^ 1, m1, t1);
        int grab = 0;
        if (tid == 0) grab = atomicAdd(a.ctr, 1);  // unit it + 4
        {
            const MTile m3 = tile_of(u3);
            t1 = tok_of(m2);
            m0 = m1;
            m1 = m2;
            m2 = m3;
        }
        if (!mbar_wait(&sbar[s], (it >> 1) & 1)) ok = false;
        const uint8_t *W = smem + s * stage;
        const uint8_t *xs = W + wbytes;
        const int nb = mt.rows;
        float *hbuf = hbuf0 + (it & 1) * kSbBatch * 32;
        {
            // warp w: rows w and w + 16, the lane's group of each in registers
            // (the prefill path's scale groups are 64 wide)
            uint4 gw[2][2], uw[2][2];
            uint2 sb[2];
            const int gc = act ? lane : 0;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const uint8_t *row = W + static_cast<size_t>(warp + 16 * rr) * L.gu_row;
                const uint4 *gq = reinterpret_cast<const uint4 *>(row + 32 * gc);
                const uint4 *uq = reinterpret_cast<const uint4 *>(row + d / 2 + 32 * gc);
                gw[rr][0] = gq[0];
                gw[rr][1] = gq[1];
                uw[rr][0] = uq[0];
                uw[rr][1] = uq[1];
                sb[rr] = *reinterpret_cast<const uint2 *>(row + d + 8 * gc);
            }
            // one token at a time (two would hold 64 registers of x; an
            // unrolled loop predicated on nb would issue all kSbBatch tokens'
            // work)
            for (int jj = 0; jj < nb; ++jj) sb_gu_tokens<1>(xs, xrow, n, act, lane, jj, gw, uw, sb, hbuf, warp);
        }
        // the stage is refilled two units on, after the next unit's barrier
        if (tid == 0) s_u[it & 3] = grab;
        __syncthreads();
        u0 = u1;
        u1 = u2;
        u2 = u3;
        u3 = s_u[it & 3];
        // h of the tile's rows over this unit's 32 rows -> 24-bit planes with
        // their own scale (lanes 4 jj .. 4 jj + 3: token jj's words); the
        // next unit writes the other buffer
        if (warp == 0) {
            const int jj = lane >> 2, w = lane & 3;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = jj < nb ? hbuf[jj * 32 + 8 * w + i] : 0.f;
            uint2 pl[3];
            float usum;
            const float sc = quant_word<3, 4>(v, pl, &usum);
            if (jj < nb) {
                uint8_t *hr = a.hq + static_cast<size_t>(mt.m0 + jj) * hrow;
                store_word_il<3>(reinterpret_cast<uint2 *>(hr), L.I / 8, rb * 4 + w, pl);
                if (w == 0) {
                    float *hs = reinterpret_cast<float *>(hr + (L.I / 8) * 24);
                    hs[rb] = sc;
                    hs[L.I / 32 + rb] = usum;
                }
            }
        }
    }
    if (!ok && tid == 0) atomicOr(a.err, QK_ERR_TIMEOUT_COPY);
    sb_finish(a.ctr);
}

// Down: unit = (small tile of at most kSbBatch rows, 128 down rows). A stage
// holds the unit's weight rows and the h of the tile's rows (one bulk copy
// each, one barrier); three stages, two units in flight while one computes,
// the descriptors read a unit before their copies are issued. LPR lanes per
// down row (one 32-element unit of h each); a lane group holds P rows'
// weights in registers and reads each row of h once for them. Y is staged in
// one of two shared buffers and written a row piece at a time while the next
// unit computes into the other.
__host__ __device__ int sb_dn_stage(const qk_layout &L) { return kSbDnRows * L.d_row + kSbBatch * sb_hrow(L.I); }
int sb_dn_smem(const qk_layout &L) { return 3 * sb_dn_stage(L) + 2 * kSbBatch * kSbDnRows * 4; }

template <int LPR>
__global__ void __launch_bounds__(kSbThreads, 1) k_sb_dn(SbArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t sbar[3];
    __shared__ int s_u[4];
    constexpr int RPW = 32 / LPR;                                  // rows a warp holds at once
    constexpr int P = kSbDnRows / ((kSbThreads / 32) * RPW) > 0    // rows a lane group holds
                          ? kSbDnRows / ((kSbThreads / 32) * RPW) : 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const qk_layout &L = a.L;
    const int d = L.d, hn = L.I / 8, upe = L.I / 32, hrow = sb_hrow(L.I);
    const uint32_t wbytes = static_cast<uint32_t>(kSbDnRows * L.d_row);
    const size_t stage = static_cast<size_t>(sb_dn_stage(L));
    float *ys0 = reinterpret_cast<float *>(smem + 3 * stage);  // 2 x [kSbBatch][kSbDnRows]
    if (tid == 0) {
        mbar_init(&sbar[0], 1);
        mbar_init(&sbar[1], 1);
        mbar_init(&sbar[2], 1);
    }
    const int db_n = d / kSbDnRows;
    const int nu = *a.n_tiles * db_n;
    sb_take_first(a.ctr, s_u);  // (its barrier also publishes the barrier inits)
    auto tile_of = [&](int u) {
        MTile m = {0, 0, 0, 0};
        if (u < nu) m = a.tiles[u / db_n];
        return m;
    };
    auto issue = [&](int u, int s, const MTile &mt) {
        uint8_t *dst = smem + s * stage;
        mbar_expect_tx(&sbar[s], wbytes + static_cast<uint32_t>(mt.rows * hrow));
        bulk_load(dst, a.pool + static_cast<size_t>(mt.slot) * L.slot_bytes + L.gu_bytes +
                           static_cast<size_t>(u % db_n) * kSbDnRows * L.d_row,
                  wbytes, &sbar[s]);
        bulk_load(dst + wbytes, a.hq + static_cast<size_t>(mt.m0) * hrow,
                  static_cast<uint32_t>(mt.rows * hrow), &sbar[s]);
    };
    // units u0 (computing), u1 and u2 (stages in flight), u3 (descriptor read)
    int u0 = s_u[0], u1 = s_u[1], u2 = s_u[2], u3 = s_u[3];
    MTile m0 = tile_of(u0), m1 = tile_of(u1), m2 = tile_of(u2);
    if (tid == 0) {
        if (u0 < nu) issue(u0, 0, m0);
        if (u1 < nu) issue(u1, 1, m1);
    }
    bool ok = true;
    for (int it = 0; u0 < nu; ++it) {
        const int s = it % 3;
        const MTile mt = m0;
        const int db = u0 % db_n;
        int grab = 0;
        if (tid == 0) {
            if (u2 < nu) issue(u2, (it + 2) % 3, m2);
            grab = atomicAdd(a.ctr, 1);  // unit it + 4
        }
        {
            const MTile m3 = tile_of(u3);
            m0 = m1;
            m1 = m2;
            m2 = m3;
        }
        if (!mbar_wait(&sbar[s], (it / 3) & 1)) ok = false;
        const uint8_t *W = smem + s * stage;
        const uint8_t *hs = W + wbytes;
        float *ys = ys0 + (it & 1) * kSbBatch * kSbDnRows;
        const int j = lane % LPR;
        if (warp * RPW < kSbDnRows) {
            // the lane group's P rows, weights in registers (scale group of
            // unit j: j / 2, the prefill path's groups being 64 wide)
            int r[P];
            uint4 w[P];
            uint32_t sb[P];
#pragma unroll
            for (int q = 0; q < P; ++q) {
                r[q] = warp * RPW + lane / LPR + q * (kSbThreads / 32) * RPW;
                const uint8_t *row = W + static_cast<size_t>(r[q] < kSbDnRows ? r[q] : 0) * L.d_row;
                w[q] = *reinterpret_cast<const uint4 *>(row + 16 * j);
                sb[q] = *reinterpret_cast<const uint32_t *>(row + L.I / 2 + 4 * (j >> 1));
            }
            int jj = 0;
            for (; jj + 2 <= mt.rows; jj += 2) sb_dn_tokens<2, P, LPR>(hs, hrow, hn, upe, j, lane, jj, w, sb, ys, r);
            if (jj < mt.rows) sb_dn_tokens<1, P, LPR>(hs, hrow, hn, upe, j, lane, jj, w, sb, ys, r);
        }
        // one barrier a unit: the stage and this ys buffer are reused only
        // after later barriers
        if (tid == 0) s_u[it & 3] = grab;
        __syncthreads();
        u0 = u1;
        u1 = u2;
        u2 = u3;
        u3 = s_u[it & 3];
        for (int i = tid; i < mt.rows * kSbDnRows; i += kSbThreads)
            a.Y[static_cast<size_t>(mt.m0 + i / kSbDnRows) * d + db * kSbDnRows + i % kSbDnRows] = ys[i];
    }
    if (!ok && tid == 0) atomicOr(a.err, QK_ERR_TIMEOUT_COPY);
    sb_finish(a.ctr);
}

// The small tiles split in list order by one CTA: those of at most max_rows
// rows (k_sb_*) and the others (k_gemm_sw). s_cnt: 2 x 32 ints of shared
// memory.
QK_DEV void split_tiles(const MTile *tiles, int n, int max_rows, MTile *light, int *n_light,
                        MTile *heavy, int *n_heavy, int *s_cnt) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    int base_l = 0, base_h = 0;
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
        const int i = i0 + tid;
        MTile m = {0, 0, 0, 0};
        if (i < n) m = tiles[i];
        const bool hv = i < n && m.rows > max_rows, lt = i < n && !hv;
        const unsigned bh = __ballot_sync(QK_FULL, hv), bl = __ballot_sync(QK_FULL, lt);
        if (lane == 0) {
            s_cnt[warp] = __popc(bl);
            s_cnt[32 + warp] = __popc(bh);
        }
        __syncthreads();
        int before_l = 0, before_h = 0, total_l = 0, total_h = 0;
        for (int w = 0; w < nw; ++w) {
            before_l += w < warp ? s_cnt[w] : 0;
            before_h += w < warp ? s_cnt[32 + w] : 0;
            total_l += s_cnt[w];
            total_h += s_cnt[32 + w];
        }
        const unsigned below = (1u << lane) - 1u;
        if (lt) light[base_l + before_l + __popc(bl & below)] = m;
        if (hv) heavy[base_h + before_h + __popc(bh & below)] = m;
        base_l += total_l;
        base_h += total_h;
        __syncthreads();
    }
    if (tid == 0) {
        *n_light = base_l;
        *n_heavy = base_h;
    }
}

__global__ void k_split_tiles(const MTile *tiles, const int *n_tiles, int max_rows, MTile *light,
                              int *n_light, MTile *heavy, int *n_heavy) {
    __shared__ int s_cnt[64];
    split_tiles(tiles, *n_tiles, max_rows, light, n_light, heavy, n_heavy, s_cnt);
}

// ---------------------------------------------------------------------------
// routing -> groups

// Slots with a negative expert id (owned by another rank) are skipped. Lanes
// of a warp with the same expert add together (one atomic per expert per
// warp: hot experts would otherwise serialise on one counter).
__global__ void k_count(const int32_t *idx, int nk, int *counts) {
    const int lane = threadIdx.x & 31;
    for (int a0 = blockIdx.x * blockDim.x; a0 < nk; a0 += gridDim.x * blockDim.x) {
        const int a = a0 + threadIdx.x;
        const int e = a < nk ? idx[a] : -1;
        const unsigned same = __match_any_sync(QK_FULL, e);
        if (e >= 0 && lane == __ffs(same) - 1) atomicAdd(counts + e, __popc(same));
    }
}

// One CTA (1024 threads, E + 1 <= 1024 groups). Group 0 is the shared expert
// (rows [0, nsh): every token, or none); group 1 + e is routed expert e.
// Writes the first row of each routed expert and the tile lists: groups of
// at most small_max rows as NS-row tiles (stiles, k_gemm_sw), larger groups
// as BM-row tiles (tiles, k_gemm).
struct PlanOut {
    int small_max;
    MTile *tiles, *stiles;
    int *n_tiles, *n_stiles, *n_rows;
};

QK_DEV void plan_group(int rows, int slot, int ex, int r0, const PlanOut &o, int t0, int u0) {
    const bool small = rows <= o.small_max;
    const int mt = small ? 0 : (rows + BM - 1) / BM;
    const int st = small ? (rows + NS - 1) / NS : 0;
    for (int i = 0; i < mt; ++i) o.tiles[t0 + i] = MTile{r0 + BM * i, min(BM, rows - BM * i), slot, ex};
    for (int i = 0; i < st; ++i) o.stiles[u0 + i] = MTile{r0 + NS * i, min(NS, rows - NS * i), slot, ex};
}

// Inclusive block scans (1024 threads) of the rows and the two tile counts
// of group g; returns the exclusive starts through the pointers.
QK_DEV void plan_scan(int g, int rows, const PlanOut &o, int *s_a, int *s_b, int *s_c, int *r0,
                      int *t0, int *u0) {
    const bool small = rows <= o.small_max;
    const int mt = small ? 0 : (rows + BM - 1) / BM;
    const int st = small ? (rows + NS - 1) / NS : 0;
    s_a[g] = rows;
    s_b[g] = mt;
    s_c[g] = st;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        const int a = g >= off ? s_a[g - off] : 0;
        const int b = g >= off ? s_b[g - off] : 0;
        const int c = g >= off ? s_c[g - off] : 0;
        __syncthreads();
        s_a[g] += a;
        s_b[g] += b;
        s_c[g] += c;
        __syncthreads();
    }
    *r0 = s_a[g] - rows;
    *t0 = s_b[g] - mt;
    *u0 = s_c[g] - st;
    if (g == 1023) {
        *o.n_tiles = s_b[1023];
        *o.n_stiles = s_c[1023];
        *o.n_rows = s_a[1023];
    }
}

__global__ void __launch_bounds__(1024) k_plan(const int *counts, int E, int nsh,
                                               const int32_t *slot_of, int shared_slot, int *row0,
                                               PlanOut o) {
    __shared__ int s_a[1024], s_b[1024], s_c[1024];
    const int g = threadIdx.x;
    const int rows = g == 0 ? nsh : (g <= E ? counts[g - 1] : 0);
    int r0, t0, u0;
    plan_scan(g, rows, o, s_a, s_b, s_c, &r0, &t0, &u0);
    if (g >= 1 && g <= E) row0[g - 1] = r0;
    const int slot = g == 0 ? shared_slot : (g <= E ? slot_of[g - 1] : -1);
    plan_group(rows, slot, g - 1, r0, o, t0, u0);
}

// Small calls (at most kPlanSmall slots): counting, planning and placing in
// one CTA, the counters in shared memory (k_count + k_plan + k_place in one
// launch). Same tile lists and row layout as those three.
constexpr int kPlanSmall = 4096;
__global__ void __launch_bounds__(1024) k_plan_small(const int32_t *idx, int nk, int k, int E,
                                                     int nsh, const int32_t *slot_of,
                                                     int shared_slot, PlanOut o, int *inv,
                                                     int *perm_tok) {
    __shared__ int s_cnt[1024], s_a[1024], s_b[1024], s_c[1024], s_row0[1024];
    const int g = threadIdx.x;
    s_cnt[g] = 0;
    __syncthreads();
    for (int a = g; a < nk; a += 1024) {
        const int e = idx[a];
        if (e >= 0) atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    const int rows = g == 0 ? nsh : (g <= E ? s_cnt[g - 1] : 0);
    int r0, t0, u0;
    plan_scan(g, rows, o, s_a, s_b, s_c, &r0, &t0, &u0);
    s_row0[g] = r0;
    const int slot = g == 0 ? shared_slot : (g <= E ? slot_of[g - 1] : -1);
    plan_group(rows, slot, g - 1, r0, o, t0, u0);
    s_cnt[g] = 0;  // now the placement cursors
    __syncthreads();
    for (int a = g; a < nk; a += 1024) {
        const int e = idx[a];
        if (e >= 0) {
            const int pos = s_row0[e + 1] + atomicAdd(&s_cnt[e], 1);
            inv[a] = pos;
            perm_tok[pos] = a / k;
        }
    }
}

// Row of each (token, slot) within its expert's group: row0[e] plus a place
// taken from the expert's cursor (warp-aggregated atomics). The order of the
// rows inside a group varies from call to call, the results do not: every
// row's products and sums are the same wherever the row sits in a tile.
__global__ void k_place(const int32_t *idx, int nk, int k, const int *row0, int *cursor, int *inv,
                        int *perm_tok) {
    const int lane = threadIdx.x & 31;
    for (int a0 = blockIdx.x * blockDim.x; a0 < nk; a0 += gridDim.x * blockDim.x) {
        const int a = a0 + threadIdx.x;
        const int e = a < nk ? idx[a] : -1;
        const unsigned same = __match_any_sync(QK_FULL, e);
        const int leader = __ffs(same) - 1;
        int base = 0;
        if (e >= 0 && lane == leader) base = atomicAdd(cursor + e, __popc(same));
        base = __shfl_sync(QK_FULL, base, leader);
        if (e >= 0) {
            const int pos = row0[e] + base + __popc(same & ((1u << lane) - 1u));
            inv[a] = pos;
            perm_tok[pos] = a / k;
        }
    }
}

// The tiles of one wave of a call whose experts exceed the pool (the
// experts of wave[ex + 1] != 0, the shared expert at wave[0]): copies of the
// plan's tiles with the slots the experts hold now. The order of the copies
// varies from call to call, the results do not (every tile is independent).
__global__ void __launch_bounds__(1024) k_wave_tiles(const MTile *tiles, const int *n_tiles,
                                                     const MTile *stiles, const int *n_stiles,
                                                     const uint8_t *wave, const int32_t *slot_of,
                                                     MTile *wt, int *n_wt, MTile *wst, int *n_wst) {
    __shared__ int c0, c1;
    if (threadIdx.x == 0) c0 = c1 = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < *n_tiles; i += blockDim.x) {
        MTile m = tiles[i];
        if (wave[m.ex + 1]) {
            if (m.ex >= 0) m.slot = slot_of[m.ex];
            wt[atomicAdd(&c0, 1)] = m;
        }
    }
    for (int i = threadIdx.x; i < *n_stiles; i += blockDim.x) {
        MTile m = stiles[i];
        if (wave[m.ex + 1]) {
            if (m.ex >= 0) m.slot = slot_of[m.ex];
            wst[atomicAdd(&c1, 1)] = m;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *n_wt = c0;
        *n_wst = c1;
    }
}

// x element types of the grouped path
enum { XK_F32 = 0, XK_BF16 = 1, XK_F16 = 2 };

// ---------------------------------------------------------------------------
// Small groups on the CUDA cores (calls whose groups all have at most 64
// rows: batched decode and the stack): the integer dot products of the
// single-launch decode kernel, each expert's weight rows streamed once for
// all of its rows (tokens). The tensor-core path dequantises a 256-row weight
// tile per K step whatever the group's few tokens; here every q4 word is
// multiplied with each token's 16-bit x (four dp4a a token).
//   k_sb_xq   every token's x -> 16-bit planes, one scale and sum per
//             32-element unit (XROW bytes a token)
//   k_sb_gu   unit = (small tile, 32 gate/up rows): the rows by one bulk copy
//             (two-unit ring), the tile's tokens' x in batches of 8; h of the
//             32 rows per token -> 24-bit planes with its own unit scale
//             (HROW bytes a grouped row)
//   k_sb_dn   unit = (small tile, 64 down rows): Y[row][d0 .. d0 + 64) fp32
// k_combine then runs as on the tensor-core path.
// One CTA per token, one thread per q4 word position (d / 8 <= 1024).
// It also writes the token's rows of the grouped fp16 A operand of the
// tensor-core kernels (as k_gather: row t for t < nsh, the row inv[t, s] of
// each slot with an expert id >= 0; the lo plane for fp32 x). With
// tiles != nullptr the grid has one block more, block T, which splits the
// call's small tiles into the light and heavy lists.
__global__ void k_sb_xq(const void *x, int x_kind, int d, int T, uint8_t *xq, const MTile *tiles,
                        const int *n_tiles, int max_rows, MTile *light, int *n_light, MTile *heavy,
                        int *n_heavy, const int32_t *idx, int k, int nsh, const int *inv, __half *xp,
                        size_t lo_plane) {
    __shared__ int s_cnt[64];
    __shared__ int s_row[33];  // the token's rows of the grouped operand (-1: none)
    const int t = blockIdx.x, w = threadIdx.x, n = d / 8;
    if (t == T) {
        split_tiles(tiles, *n_tiles, max_rows, light, n_light, heavy, n_heavy, s_cnt);
        return;
    }
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (w < n) {
        if (x_kind == XK_BF16) {
            const uint4 q = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + static_cast<size_t>(t) * d)[w];
            v[0] = bf16lo(q.x); v[1] = bf16hi(q.x); v[2] = bf16lo(q.y); v[3] = bf16hi(q.y);
            v[4] = bf16lo(q.z); v[5] = bf16hi(q.z); v[6] = bf16lo(q.w); v[7] = bf16hi(q.w);
        } else if (x_kind == XK_F16) {
            const uint4 q = reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) + static_cast<size_t>(t) * d)[w];
            const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f2 = __half22float2(u2h(qq[i]));
                v[2 * i] = f2.x;
                v[2 * i + 1] = f2.y;
            }
        } else {
            const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(x) + static_cast<size_t>(t) * d) + 2 * w;
            const float4 a = p[0], b = p[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
    }
    for (int i = w; i <= k; i += blockDim.x) {
        int r = -1;
        if (i == k) r = t < nsh ? t : -1;
        else if (idx[static_cast<size_t>(t) * k + i] >= 0) r = inv[static_cast<size_t>(t) * k + i];
        s_row[i] = r;
    }
    uint2 pl[2];
    float usum;
    const float sc = quant_word<2>(v, pl, &usum);  // one scale per 64-element group
    const float gsum = usum + __shfl_xor_sync(QK_FULL, usum, 4);
    uint8_t *row = xq + static_cast<size_t>(t) * sb_xrow(d);
    if (w < n) {
        store_word_gx<2>(reinterpret_cast<uint2 *>(row), n, w, pl);
        if ((w & 7) == 0) reinterpret_cast<float2 *>(row + n * 16)[w >> 3] = make_float2(sc, gsum);
    }
    uint4 o = make_uint4(0u, 0u, 0u, 0u), ol = make_uint4(0u, 0u, 0u, 0u);
    if (w < n) {
        o.x = h2u(__floats2half2_rn(v[0], v[4]));
        o.y = h2u(__floats2half2_rn(v[1], v[5]));
        o.z = h2u(__floats2half2_rn(v[2], v[6]));
        o.w = h2u(__floats2half2_rn(v[3], v[7]));
        if (x_kind == XK_F32) {
            // lo = fp16(x - hi): the pair carries x to about 22 bits
            const float2 h0 = __half22float2(u2h(o.x)), h1 = __half22float2(u2h(o.y)),
                         h2 = __half22float2(u2h(o.z)), h3 = __half22float2(u2h(o.w));
            ol.x = h2u(__floats2half2_rn(v[0] - h0.x, v[4] - h0.y));
            ol.y = h2u(__floats2half2_rn(v[1] - h1.x, v[5] - h1.y));
            ol.z = h2u(__floats2half2_rn(v[2] - h2.x, v[6] - h2.y));
            ol.w = h2u(__floats2half2_rn(v[3] - h3.x, v[7] - h3.y));
        }
    }
    __syncthreads();
    if (w < n) {
        for (int sl = 0; sl <= k; ++sl) {
            const int r = s_row[sl];
            if (r < 0) continue;
            __half *dst = xp + static_cast<size_t>(r) * d;
            reinterpret_cast<uint4 *>(dst)[w] = o;
            if (x_kind == XK_F32) reinterpret_cast<uint4 *>(dst + lo_plane)[w] = ol;
        }
    }
}


// Grouped fp16 A operand: row r holds token r (r < nsh, the shared group) or
// perm_tok[r]; each 8-element chunk in the order [0,4,1,5,2,6,3,7].
__global__ void k_gather(const void *x, int x_kind, int d, int nsh, int rows, const int *n_rows,
                         const int *perm_tok, __half *xp, size_t lo_plane) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows || warp >= *n_rows) return;
    const int tok = warp < nsh ? warp : perm_tok[warp];
    __half *dst = xp + static_cast<size_t>(warp) * d;
    for (int c = lane; c < d / 8; c += 32) {
        float v[8];
        if (x_kind == XK_F16) {
            const uint4 w = reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) +
                                                            static_cast<size_t>(tok) * d)[c];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 p = __half22float2(u2h(ww[i]));
                v[2 * i] = p.x;
                v[2 * i + 1] = p.y;
            }
        } else if (x_kind == XK_BF16) {
            const uint4 w = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) +
                                                            static_cast<size_t>(tok) * d)[c];
            v[0] = bf16lo(w.x); v[1] = bf16hi(w.x); v[2] = bf16lo(w.y); v[3] = bf16hi(w.y);
            v[4] = bf16lo(w.z); v[5] = bf16hi(w.z); v[6] = bf16lo(w.w); v[7] = bf16hi(w.w);
        } else {
            const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(x) +
                                                               static_cast<size_t>(tok) * d) + 2 * c;
            const float4 a = p[0], b = p[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        uint4 o;
        o.x = h2u(__floats2half2_rn(v[0], v[4]));
        o.y = h2u(__floats2half2_rn(v[1], v[5]));
        o.z = h2u(__floats2half2_rn(v[2], v[6]));
        o.w = h2u(__floats2half2_rn(v[3], v[7]));
        reinterpret_cast<uint4 *>(dst)[c] = o;
        if (x_kind == XK_F32) {
            // lo = fp16(x - hi): the pair carries x to about 22 bits
            float l[8];
            const float2 h0 = __half22float2(u2h(o.x)), h1 = __half22float2(u2h(o.y)),
                         h2 = __half22float2(u2h(o.z)), h3 = __half22float2(u2h(o.w));
            l[0] = v[0] - h0.x; l[4] = v[4] - h0.y; l[1] = v[1] - h1.x; l[5] = v[5] - h1.y;
            l[2] = v[2] - h2.x; l[6] = v[6] - h2.y; l[3] = v[3] - h3.x; l[7] = v[7] - h3.y;
            uint4 ol;
            ol.x = h2u(__floats2half2_rn(l[0], l[4]));
            ol.y = h2u(__floats2half2_rn(l[1], l[5]));
            ol.z = h2u(__floats2half2_rn(l[2], l[6]));
            ol.w = h2u(__floats2half2_rn(l[3], l[7]));
            reinterpret_cast<uint4 *>(dst + lo_plane)[c] = ol;
        }
    }
}

// out[t] = sum_s w[t,s] * Yr[inv[t,s]] + sigmoid(g_t) * Ysh[t], fixed
// order; one CTA per token, 4 columns per thread, all row loads of a thread
// issued before the sums.
// Threads per token: a small call (fewer tokens than about two per SM) gets
// one thread per 4 columns, up to 512, so each thread's loads are one group;
// a large call 256 (measured faster at 4096 tokens).
int combine_threads(int T, int d) { return T <= 256 ? min(512, (d / 4 + 31) / 32 * 32) : 256; }

__global__ void k_combine(const float *Yr, const float *Ysh, const int *inv, const float *wts,
                          const float *sgate, int k, int d, float *out) {
    // the token's k + 1 row pointers and weights first, so that a thread's
    // row loads go out together (8 at a time), summed in slot order
    __shared__ const float *s_y[33];
    __shared__ float s_w[33];
    const int t = blockIdx.x;
    for (int s = threadIdx.x; s <= k; s += blockDim.x) {
        s_y[s] = s < k ? Yr + static_cast<size_t>(inv[t * k + s]) * d : Ysh + static_cast<size_t>(t) * d;
        s_w[s] = s < k ? wts[t * k + s] : sgate[t];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < d / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 <= k; s0 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (s0 + u <= k) v[u] = reinterpret_cast<const float4 *>(s_y[s0 + u])[c];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (s0 + u <= k) {
                    const float w = s_w[s0 + u];
                    acc.x = fmaf(w, v[u].x, acc.x);
                    acc.y = fmaf(w, v[u].y, acc.y);
                    acc.z = fmaf(w, v[u].z, acc.z);
                    acc.w = fmaf(w, v[u].w, acc.w);
                }
            }
        }
        reinterpret_cast<float4 *>(out + static_cast<size_t>(t) * d)[c] = acc;
    }
}

// ---------------------------------------------------------------------------
// expert-parallel dispatch and return (one rank per GPU; rank g owns experts
// [g * E_per, (g + 1) * E_per))

// Each token goes once to every rank that owns one of its experts; its
// other slots travel with it as expert id -1. The bit mask of destinations
// of token t: mask[t].
__global__ void k_ep_mask(const int32_t *idx, int T, int k, int e_per, unsigned long long *mask) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        unsigned long long m = 0;
        for (int s = 0; s < k; ++s) m |= 1ull << (idx[t * k + s] / e_per);
        mask[t] = m;
    }
}

// Fixed-capacity send rows: rank g's rows are [g cap, (g + 1) cap), token t
// in row g cap + t. A row carries x[t] as given (row_bytes: bf16 or fp32,
// copied verbatim) and the token's k slots, expert ids of other ranks
// replaced by -1 (weights 0); rows of tokens not bound for g, and rows
// t >= T, carry only k ids -1 (x is not written). One warp per row.
__global__ void k_ep_pack(const uint8_t *x, int row_bytes, int T, int cap, int k, int e_per,
                          int G, const int32_t *idx, const float *wts,
                          const unsigned long long *mask, uint8_t *send_x, int32_t *send_e,
                          float *send_w) {
    const int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wi >= G * cap) return;
    const int g = wi / cap, t = wi % cap;
    const size_t p = static_cast<size_t>(wi);
    const bool live = t < T && ((mask[t] >> g) & 1ull);
    if (lane < k) {
        const int e = live ? idx[t * k + lane] : -1;
        const bool own = live && e / e_per == g;
        send_e[p * k + lane] = own ? e : -1;
        send_w[p * k + lane] = own ? wts[t * k + lane] : 0.f;
    }
    if (!live) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(send_x + p * row_bytes);
    for (int c = lane; c < row_bytes / 16; c += 32) dst[c] = src[c];
}

// The rank's own tokens as the leading rows of the receive buffer (x as
// given; rows [T, cap) carry only ids), no routed slots (the experts pass
// gives them only the shared expert).
__global__ void k_ep_own(const uint8_t *x, int row_bytes, int T, int cap, int k, uint8_t *recv_x,
                         int32_t *recv_e) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= cap) return;
    if (lane < k) recv_e[static_cast<size_t>(t) * k + lane] = -1;
    if (t >= T) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(recv_x + static_cast<size_t>(t) * row_bytes);
    for (int c = lane; c < row_bytes / 16; c += 32) dst[c] = src[c];
}

// Expert-side combine of the received rows: part[r] = sum over the row's
// local slots (expert id >= 0) of w * Y[inv[r, s]], in slot order.
__global__ void k_ep_partial(const float *Y, const int *inv, const int32_t *e_of, const float *w,
                             int k, int d, float *part) {
    const int r = blockIdx.x;
    for (int c = threadIdx.x; c < d / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < k; ++s) {
            const size_t a = static_cast<size_t>(r) * k + s;
            if (e_of[a] < 0) continue;
            const float4 v = reinterpret_cast<const float4 *>(Y + static_cast<size_t>(inv[a]) * d)[c];
            const float ws = w[a];
            acc.x = fmaf(ws, v.x, acc.x);
            acc.y = fmaf(ws, v.y, acc.y);
            acc.z = fmaf(ws, v.z, acc.z);
            acc.w = fmaf(ws, v.w, acc.w);
        }
        reinterpret_cast<float4 *>(part + static_cast<size_t>(r) * d)[c] = acc;
    }
}

// Token side: out[t] = sum over the destination ranks in rank order of the
// returned partial rows (row g cap + t from rank g) + sigmoid(g_t) * Ysh[t].
__global__ void k_ep_final(const float *back, const unsigned long long *mask, int T, int cap,
                           int G, const float *Ysh, const float *sgate, int d, float *out) {
    const int t = blockIdx.x;
    const unsigned long long m = mask[t];
    for (int c = threadIdx.x; c < d / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int g = 0; g < G; ++g) {
            if (!((m >> g) & 1ull)) continue;
            const size_t p = static_cast<size_t>(g) * cap + t;
            const float4 v = reinterpret_cast<const float4 *>(back + p * d)[c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float sg = sgate[t];
        const float4 v = reinterpret_cast<const float4 *>(Ysh + static_cast<size_t>(t) * d)[c];
        acc.x = fmaf(sg, v.x, acc.x);
        acc.y = fmaf(sg, v.y, acc.y);
        acc.z = fmaf(sg, v.z, acc.z);
        acc.w = fmaf(sg, v.w, acc.w);
        reinterpret_cast<float4 *>(out + static_cast<size_t>(t) * d)[c] = acc;
    }
}

// ---------------------------------------------------------------------------
// routing of a multi-token call (model.c:1301-1318, :1396-1398)
//
// The canonical router logit of (token t, expert e) is one fp32 rounding of
// an fp64 sum in a fixed order (router_lane); the top-k and its softmax
// follow from those values. Computing all T x E of them in fp64 is the cost
// of the whole layer at prefill sizes, so the call runs in three steps:
//   k_route_split   x -> bf16 pair (hi = bf16(x), lo = bf16(x - hi)), the
//                   2-norm of each token
//   k_gemm<2>       approximate logits a[t, e] = (hi + lo) . w_e on the
//                   tensor cores (fp32 accumulation)
//   k_route_exact   per token: with a bound |a - logit| <= beta, every
//                   member of the exact top-k (and every expert tied with
//                   one) has a >= a_(k) - 2 beta, a_(k) the k-th largest
//                   approximate value. The exact logits of that candidate
//                   set (typically 11-16 experts) are computed in the
//                   canonical order and ranked exactly, so the selection,
//                   order and weights are those of the full exact top-k.
// beta = 2^-10 |x_t| max_e |w_e| + 2^-20 max_e |a[t, e]|: the first term is
// twice the worst case of 4096 products (hi and lo) summed in fp32 with
// truncation at every step, |x - hi - lo| <= 2^-18 |x| included, over
// sum_i |x_i w_i| <= |x| |w| (Cauchy-Schwarz); the second covers the fp32
// additions of the logit bias. The candidate threshold uses 3 beta. A token
// whose candidate set exceeds 32, or with a non-finite value, gets every
// logit exactly instead (the one-warp path of k_topk).

// warps per token (CTA) of k_route_exact: 4 at prefill sizes, 16 for small
// calls (fewer tokens than SMs: the candidates' dots run in parallel)
constexpr int kRW = 4, kRWsmall = 16;

__global__ void k_route_split(const void *x, int x_bf16, int d, int T, int Tpad,
                              __nv_bfloat16 *xr, float *xnorm, MTile *tiles, int *n_mtiles) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (blockIdx.x == 0) {
        const int nm = (T + BM - 1) / BM;
        for (int i = threadIdx.x; i < nm; i += blockDim.x) {
            MTile m;
            m.m0 = BM * i;
            m.rows = min(BM, T - BM * i);
            m.slot = 0;
            m.ex = 0;
            tiles[i] = m;
        }
        if (threadIdx.x == 0) *n_mtiles = nm;
    }
    if (warp >= T) return;
    double ss = 0.0;
    for (int c = lane; c < d / 8; c += 32) {
        float v[8];
        if (x_bf16) {
            const uint4 w = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) +
                                                            static_cast<size_t>(warp) * d)[c];
            v[0] = bf16lo(w.x); v[1] = bf16hi(w.x); v[2] = bf16lo(w.y); v[3] = bf16hi(w.y);
            v[4] = bf16lo(w.z); v[5] = bf16hi(w.z); v[6] = bf16lo(w.w); v[7] = bf16hi(w.w);
        } else {
            const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(x) +
                                                               static_cast<size_t>(warp) * d) + 2 * c;
            const float4 a = p[0], b = p[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            const float2 hf = __bfloat1622float2(h);
            const __nv_bfloat162 l = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
            hi[i] = *reinterpret_cast<const uint32_t *>(&h);
            lo[i] = *reinterpret_cast<const uint32_t *>(&l);
            ss = fma(static_cast<double>(v[2 * i]), static_cast<double>(v[2 * i]), ss);
            ss = fma(static_cast<double>(v[2 * i + 1]), static_cast<double>(v[2 * i + 1]), ss);
        }
        reinterpret_cast<uint4 *>(xr + static_cast<size_t>(warp) * d)[c] =
            make_uint4(hi[0], hi[1], hi[2], hi[3]);
        reinterpret_cast<uint4 *>(xr + static_cast<size_t>(Tpad + warp) * d)[c] =
            make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    ss = warp_sum_butterfly(ss);
    if (lane == 0) xnorm[warp] = __double2float_ru(sqrt(ss));
}

// Small calls (T <= kRouteSmallT): the approximate logits on the CUDA cores
// in fp32, in place of k_route_split + k_gemm<2>. CTA (32 experts, 8 tokens),
// 8 warps; the CTA's router rows come in by one bulk copy, x of its tokens is
// staged as fp32. Warp w takes experts e0 + 4w .. e0 + 4w + 3 for the 8
// tokens, lane l the elements 4l + 128i + (0..3) (consecutive lanes read
// consecutive 16-byte pieces), the 32 sums reduced by a halving butterfly.
// Along any path an fp32 sum here meets at most 69 roundings, far inside the
// bound k_route_exact allows for (2^-10 |x| max|w|), so its candidate sets
// still hold the exact top-k. The first expert block also writes the tokens'
// 2-norms exactly as k_route_split does.
constexpr int kRouteSmallT = 64, kRaTok = 8, kRaExp = 32, kRaEw = 4, kRaThreads = kRaExp / kRaEw * 32;
int route_approx_smem(int d) { return kRaExp * d * 2 + kRaTok * d * 4; }
constexpr int kRaSmemMax = 200 * 1024;  // larger d: k_route_split + k_gemm<2>

__global__ void __launch_bounds__(kRaThreads) k_route_approx(const void *x, int x_bf16, int d, int T, int E,
                                                       const uint16_t *router, float *lga, float *xnorm,
                                                       int *err) {
    // dynamic shared memory: the CTA's 32 router rows (bf16, one bulk copy),
    // then x of its 8 tokens as fp32
    extern __shared__ __align__(128) uint8_t rsa[];
    __shared__ uint64_t rbar;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * kRaExp, t0 = blockIdx.y * kRaTok;
    const int nt = min(kRaTok, T - t0), ne = min(kRaExp, E - e0);
    const uint16_t *wr = reinterpret_cast<const uint16_t *>(rsa);
    float *xsa = reinterpret_cast<float *>(rsa + static_cast<size_t>(kRaExp) * d * 2);
    const uint32_t rbytes = static_cast<uint32_t>(ne) * d * 2;
    if (threadIdx.x == 0) {
        mbar_init(&rbar, 1);
        mbar_expect_tx(&rbar, rbytes);
        bulk_load(rsa, router + static_cast<size_t>(e0) * d, rbytes, &rbar);
    }
    // x of the 8 tokens: every load of a thread issued before its stores
    constexpr int kMaxPer = 8;  // chunks per thread (d <= 2048 at 256 threads)
    const int per = (kRaTok * (d / 8) + blockDim.x - 1) / blockDim.x;
    float4 va[kMaxPer], vb[kMaxPer];
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
        va[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        vb[j] = va[j];
        const int i = threadIdx.x + j * blockDim.x;
        const int tt = i / (d / 8), c = i % (d / 8);
        if (j < per && tt < nt) {
            if (x_bf16) {
                const uint4 w = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) +
                                                                static_cast<size_t>(t0 + tt) * d)[c];
                va[j] = make_float4(bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y));
                vb[j] = make_float4(bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w));
            } else {
                const float4 *q = reinterpret_cast<const float4 *>(static_cast<const float *>(x) +
                                                                   static_cast<size_t>(t0 + tt) * d) + 2 * c;
                va[j] = q[0];
                vb[j] = q[1];
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (j < per && i < kRaTok * (d / 8)) {
            float4 *dst = reinterpret_cast<float4 *>(xsa + static_cast<size_t>(i / (d / 8)) * d) + 2 * (i % (d / 8));
            dst[0] = va[j];
            dst[1] = vb[j];
        }
    }
    __syncthreads();
    // the tokens' 2-norms (first expert block), from the staged values in
    // k_route_split's order
    if (blockIdx.x == 0 && warp < nt) {
        double ss = 0.0;
        const float *xr = xsa + static_cast<size_t>(warp) * d;
        for (int c = lane; c < d / 8; c += 32)
#pragma unroll
            for (int i = 0; i < 8; ++i)
                ss = fma(static_cast<double>(xr[8 * c + i]), static_cast<double>(xr[8 * c + i]), ss);
        ss = warp_sum_butterfly(ss);
        if (lane == 0) xnorm[t0 + warp] = __double2float_ru(sqrt(ss));
    }
    // (a copy that never lands: NaN logits, which send the tokens to the
    // all-exact ranking, and the error word)
    const bool ok = mbar_wait(&rbar, 0);
    if (!ok && threadIdx.x == 0) atomicOr(err, QK_ERR_TIMEOUT_COPY);
    const int el = kRaEw * warp;  // experts e0 + el .. e0 + el + 3
    float acc[kRaEw * kRaTok];
#pragma unroll
    for (int i = 0; i < kRaEw * kRaTok; ++i) acc[i] = 0.f;
    for (int k0 = 4 * lane; k0 < d; k0 += 128) {
        float w[kRaEw][4];
#pragma unroll
        for (int j = 0; j < kRaEw; ++j) {
            const uint2 q = el + j < ne ? *reinterpret_cast<const uint2 *>(wr + static_cast<size_t>(el + j) * d + k0)
                                        : make_uint2(0u, 0u);
            w[j][0] = bf16lo(q.x); w[j][1] = bf16hi(q.x); w[j][2] = bf16lo(q.y); w[j][3] = bf16hi(q.y);
        }
#pragma unroll
        for (int tt = 0; tt < kRaTok; ++tt) {
            const float4 a = *reinterpret_cast<const float4 *>(xsa + static_cast<size_t>(tt) * d + k0);
#pragma unroll
            for (int j = 0; j < kRaEw; ++j) {
                float &c = acc[j * kRaTok + tt];
                c = fmaf(a.x, w[j][0], c);
                c = fmaf(a.y, w[j][1], c);
                c = fmaf(a.z, w[j][2], c);
                c = fmaf(a.w, w[j][3], c);
            }
        }
    }
    // lane l: the sum of value l = (expert e0 + el + l / 8, token l % 8)
    const float sum = group_sum_tr<kRaEw * kRaTok, 32>(acc, lane);
    const int ee = el + lane / kRaTok, tt = lane % kRaTok;
    if (tt < nt && ee < ne) lga[static_cast<size_t>(t0 + tt) * E + e0 + ee] = ok ? sum : NAN;
}

struct RouteArgs {
    const void *x;
    int x_bf16, d, E, k, T;
    const uint16_t *router, *shared_gate;
    const float *bias;   // [E] or NULL
    const float *lga;    // [T, E] approximate logits (without the bias)
    const float *xnorm;  // [T]
    float wmax;          // max_e |w_e|, rounded up
    int32_t *idx;
    float *wts, *sgate;
    int *err;
};

// The k-th largest of E staged keys (keys past E are 0; k <= 32, k <= E),
// or a lower bound of it when more than 32 keys reach the k-th largest of
// the 32 lane maxima. One warp.
QK_DEV uint32_t kth_key(const uint32_t *keys, int E, int k, uint32_t *s_key) {
    const int lane = threadIdx.x & 31;
    const int nj = (E + 31) / 32;
    uint32_t mxk = 0;
    for (int j = 0; j < nj; ++j) mxk = max(mxk, keys[j * 32 + lane]);
    int r = 0;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const uint32_t o = __shfl_sync(QK_FULL, mxk, j);
        r += (o > mxk || (o == mxk && j < lane)) ? 1 : 0;
    }
    const uint32_t tau = __shfl_sync(QK_FULL, mxk, __ffs(__ballot_sync(QK_FULL, r == k - 1)) - 1);
    int own = 0;
    for (int j = 0; j < nj; ++j) own += keys[j * 32 + lane] >= tau ? 1 : 0;
    int incl = own;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(QK_FULL, incl, off);
        if (lane >= off) incl += t;
    }
    const int C = __shfl_sync(QK_FULL, incl, 31);
    if (C > 32) return tau;
    int pos = incl - own;
    for (int j = 0; j < nj; ++j) {
        const uint32_t kk = keys[j * 32 + lane];
        if (kk >= tau) s_key[pos++] = kk;
    }
    __syncwarp();
    const uint32_t mk = lane < C ? s_key[lane] : 0u;
    int rank = 0;
    for (int m = 0; m < C; ++m) {
        const uint32_t o = __shfl_sync(QK_FULL, mk, m);
        rank += (o > mk || (o == mk && m < lane)) ? 1 : 0;
    }
    const unsigned hit = __ballot_sync(QK_FULL, lane < C && rank == k - 1);
    const uint32_t res = __shfl_sync(QK_FULL, mk, __ffs(hit) - 1);
    __syncwarp();
    return res;
}

QK_DEV float exact_logit(const RouteArgs &a, const double2 *xs, int e, int lane) {
    const double s = warp_sum_butterfly(router_lane(a.router + static_cast<size_t>(e) * a.d, xs, a.d, lane));
    float v = static_cast<float>(s);
    if (a.bias) v = v + a.bias[e];
    return v;
}

// One CTA of kRW warps per token; dynamic shared memory: x staged as d
// doubles, then E keys. Warp 0 finds the candidate set; the candidates'
// canonical logits are spread over the warps (each dot is a chain of L2
// loads, so several in flight per token matter); warp 0 ranks them.
template <int kRW>
__global__ void __launch_bounds__(kRW * 32) k_route_exact(RouteArgs a) {
    extern __shared__ __align__(16) float rsm[];
    __shared__ uint32_t s_key[32];
    __shared__ int s_idx[32];
    __shared__ float s_ev[32];
    __shared__ float s_wmax[kRW];
    __shared__ int s_C, s_fast, s_fin;
    __shared__ float s_sg;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x;
    const int d = a.d, E = a.E, k = a.k, nE = (E + 31) / 32 * 32;
    double2 *xs = reinterpret_cast<double2 *>(rsm);
    uint32_t *keys = reinterpret_cast<uint32_t *>(rsm + static_cast<size_t>(d) * 2);
    for (int c = threadIdx.x; c < d / 8; c += kRW * 32) {
        float v[8];
        if (a.x_bf16) {
            const uint4 w = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.x) +
                                                            static_cast<size_t>(t) * d)[c];
            v[0] = bf16lo(w.x); v[1] = bf16hi(w.x); v[2] = bf16lo(w.y); v[3] = bf16hi(w.y);
            v[4] = bf16lo(w.z); v[5] = bf16hi(w.z); v[6] = bf16lo(w.w); v[7] = bf16hi(w.w);
        } else {
            const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) +
                                                               static_cast<size_t>(t) * d) + 2 * c;
            const float4 u = p[0], w = p[1];
            v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; v[4] = w.x; v[5] = w.y; v[6] = w.z; v[7] = w.w;
        }
        rx_store(xs, c, v);
    }
    // approximate logits (+ bias, as the canonical logit adds it) -> keys
    const float *lr = a.lga + static_cast<size_t>(t) * E;
    bool finite = isfinite(a.xnorm[t]);
    float maxabs = 0.f;
    for (int e = threadIdx.x; e < nE; e += kRW * 32) {
        uint32_t key = 0u;
        if (e < E) {
            float v = lr[e];
            if (a.bias) v = v + a.bias[e];
            finite = finite && isfinite(v);
            maxabs = fmaxf(maxabs, fabsf(v));
            key = fkey(v);
        }
        keys[e] = key;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) maxabs = fmaxf(maxabs, __shfl_xor_sync(QK_FULL, maxabs, off));
    if (lane == 0) s_wmax[warp] = maxabs;
    finite = __syncthreads_and(finite) != 0;
    if (warp == 0) {
        float m = lane < kRW ? s_wmax[lane] : 0.f;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(QK_FULL, m, off));
        bool fast = finite;
        int C = 0;
        if (fast) {
            const float vk = key_value(kth_key(keys, E, k, s_key));
            const float beta = __fmaf_ru(__fmul_ru(0x1p-10f, a.xnorm[t]), a.wmax, __fmul_ru(0x1p-20f, m));
            const uint32_t tk = fkey(__fsub_rd(vk, __fmul_ru(3.0f, beta)));
            int own = 0;
            for (int e = lane; e < E; e += 32) own += keys[e] >= tk ? 1 : 0;
            int incl = own;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int u = __shfl_up_sync(QK_FULL, incl, off);
                if (lane >= off) incl += u;
            }
            C = __shfl_sync(QK_FULL, incl, 31);
            fast = C >= k && C <= 32;
            if (fast) {
                int pos = incl - own;
                for (int e = lane; e < E; e += 32)
                    if (keys[e] >= tk) s_idx[pos++] = e;
            }
        }
        if (lane == 0) {
            s_C = C;
            s_fast = fast ? 1 : 0;
            s_fin = 1;
        }
    } else if (warp == kRW - 1) {  // the shared gate, canonical order, beside warp 0's selection
        const double sg = warp_sum_butterfly(router_lane(a.shared_gate, xs, d, lane));
        if (lane == 0) s_sg = 1.0f / (1.0f + expf(-static_cast<float>(sg)));
    }
    __syncthreads();
    const bool fast = s_fast != 0;
    const int C = s_C;
    if (fast) {
        // exact logits of the candidates, canonical order, spread over warps
        for (int m = warp; m < C; m += kRW) {
            const float v = exact_logit(a, xs, s_idx[m], lane);
            if (lane == 0) {
                s_key[m] = fkey(v);
                if (!isfinite(v)) s_fin = 0;
            }
        }
    }
    __syncthreads();
    if (fast && s_fin) {
        if (warp == 0)
            topk_rank_softmax(C, k, s_key, s_idx, s_ev, a.idx + static_cast<size_t>(t) * k,
                              a.wts + static_cast<size_t>(t) * k);
    } else {
        // every logit exactly (rare)
        for (int e = warp; e < E; e += kRW) {
            const float v = exact_logit(a, xs, e, lane);
            if (lane == 0) keys[e] = fkey(v);
        }
        __syncthreads();
        if (warp == 0 && !topk_warp(keys, E, k, s_key, s_idx, s_ev, a.idx + static_cast<size_t>(t) * k,
                                    a.wts + static_cast<size_t>(t) * k)) {
            if (lane == 0) atomicOr(a.err, QK_ERR_BAD_ROUTE);
            return;
        }
    }
    if (threadIdx.x == 0) a.sgate[t] = s_sg;
}

// ---------------------------------------------------------------------------
// host side

typedef CUresult (*encode_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                              const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                              const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

encode_fn get_encode() {
    static encode_fn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<encode_fn>(p);
    }
    return fn;
}

// Row-major [rows, cols] of 16-bit elements, boxes of 64 x box_rows with the
// 128-byte swizzle (the K-major operand layout of the MMA).
bool map_2d_16(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, bool bf16,
               uint32_t box_rows = BM) {
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {BK, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return get_encode()(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void *>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool map_3d_u8(CUtensorMap *m, const void *base, uint64_t row_bytes, uint64_t rows,
               uint64_t slots, uint64_t slot_stride, uint32_t box_x, uint32_t box_y,
               bool swizzle128 = false) {
    const cuuint64_t dims[3] = {row_bytes, rows, slots};
    const cuuint64_t strides[2] = {row_bytes, slot_stride};
    const cuuint32_t box[3] = {box_x, box_y, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return get_encode()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Every rank's receive-side buffers as mapped in this process (peer
// exchange).
struct EpPeers {
    uint8_t *recv_x[64];
    int32_t *recv_e[64];
    float *recv_w[64];
    float *back[64];
    unsigned long long *flags[64];
};

struct qk_prefill {
    qk_layout L;
    int max_tokens, num_sms, pool_slots, rows_max, tiles_max;
    int small_max;                  // groups of at most this many rows use k_gemm_sw
    int sb;                         // small tiles on the CUDA cores (k_sb_*) instead of k_gemm_sw
    int sb_max_rows;                // ... those of at most this many rows; k_gemm_sw the others
    uint8_t *sb_xq, *sb_hq;         // their quantised x per token, h per grouped row
    MTile *ltiles, *htiles;         // the small tiles of at most / more than sb_max_rows rows
    int *n_ltiles, *n_htiles;
    int *sb_ctr;                    // [4]: k_sb_gu's and k_sb_dn's unit counters (0 between launches)
    cudaStream_t st2;               // k_gemm_sw on the heavy tiles, beside k_sb_* ...
    cudaEvent_t ev_fork, ev_join;   // ... forked from and joined back into the call's stream
    const uint8_t *pool;            // the weight pool the expert slots index
    int *counts, *cursor, *row0, *inv, *perm_tok, *n_mtiles, *n_stiles, *n_rows;
    MTile *tiles, *stiles;          // BM-row tiles (k_gemm), NS-row tiles (k_gemm_sw)
    // waves of a call whose experts exceed the pool: the wave's tiles and the
    // expert mask ([E + 1], shared expert first)
    MTile *wtiles, *wstiles;
    int *n_wtiles;                  // [2]: tiles, small tiles
    uint8_t *wave;
    __half *xp, *H;
    float *Y;
    CUtensorMap tmX, tmH, tmQgu, tmSgu, tmQdn, tmSdn;
    CUtensorMap tmXs, tmHs;         // the same planes in NS-row boxes
    CUtensorMap tmXs8, tmHs8;       // and in NS8-row boxes (narrow small tiles)
    // k_gemm_sw's weight boxes: q4 words of KS K steps (128 bytes, swizzled)
    // per row, the scales of KS steps (GU) or of the whole row (down)
    CUtensorMap tmQgu4, tmSgu4, tmQdn4, tmSdn4;
    // routing: x as a bf16 pair [2 * Tpad, d], token norms, approximate
    // logits [max_tokens, E], the router's M-tile list
    int route_ok, Tpad;
    size_t route_smem;
    __nv_bfloat16 *xr;
    float *xnorm, *lga;
    MTile *rtiles;
    int *rn;
    CUtensorMap tmXr;
    // expert parallelism: one row per (token, destination rank)
    int ep_T, ep_G;                 // rows per rank pair (capacity), ranks
    unsigned long long *ep_mask;    // [ep_T] destination ranks of each token
    int32_t *ep_send_e, *ep_recv_e; // [rows * k] slot expert ids (-1: another rank's)
    float *ep_send_w, *ep_recv_w;   // [rows * k] slot weights
    uint8_t *ep_send_x, *ep_recv_x; // [rows, d] x as given (bf16 or fp32)
    float *ep_ret, *ep_back;        // [rows, d] fp32 partial outputs: received / send order
    unsigned long long *ep_flags;   // [2][64] peer-exchange flags (written by the peers)
    unsigned long long *ep_epoch;   // calls completed (peer exchange)
    unsigned *ep_done;              // [2] CTAs done, dispatch / return grids
    EpPeers ep_peers;               // every rank's buffers as mapped here
    EpPeers *ep_peers_dev;
    int ep_p2p;                     // the peer table is open
};

extern "C" void qk_prefill_destroy(qk_prefill *p) {
    if (!p) return;
    cudaFree(p->counts);  // cursor lives in the same allocation
    cudaFree(p->row0);
    cudaFree(p->inv);
    cudaFree(p->perm_tok);
    cudaFree(p->n_mtiles);
    cudaFree(p->n_stiles);
    cudaFree(p->n_rows);
    cudaFree(p->tiles);
    cudaFree(p->stiles);
    cudaFree(p->sb_xq);
    cudaFree(p->sb_hq);
    cudaFree(p->htiles);
    cudaFree(p->n_htiles);
    cudaFree(p->ltiles);
    cudaFree(p->n_ltiles);
    cudaFree(p->sb_ctr);
    if (p->st2) cudaStreamDestroy(p->st2);
    if (p->ev_fork) cudaEventDestroy(p->ev_fork);
    if (p->ev_join) cudaEventDestroy(p->ev_join);
    cudaFree(p->xp);
    cudaFree(p->H);
    cudaFree(p->Y);
    cudaFree(p->xr);
    cudaFree(p->xnorm);
    cudaFree(p->lga);
    cudaFree(p->rtiles);
    cudaFree(p->rn);
    cudaFree(p->ep_mask);
    cudaFree(p->ep_send_e);
    cudaFree(p->ep_recv_e);
    cudaFree(p->ep_send_w);
    cudaFree(p->ep_recv_w);
    cudaFree(p->ep_send_x);
    cudaFree(p->ep_recv_x);
    cudaFree(p->ep_ret);
    qk_ep_p2p_close(p);
    cudaFree(p->ep_flags);
    cudaFree(p->ep_epoch);
    cudaFree(p->ep_done);
    cudaFree(p->ep_peers_dev);
    cudaFree(p->ep_back);
    cudaFree(p->wtiles);
    cudaFree(p->wstiles);
    cudaFree(p->n_wtiles);
    cudaFree(p->wave);
    delete p;
}

extern "C" qk_prefill *qk_prefill_create(const qk_layout *L, int max_tokens, const uint8_t *pool,
                                         int pool_slots, int num_sms, char *msg, size_t msg_len) {
    // shapes the kernels cover: I a multiple of 128, d a multiple of 256
    if (L->I % 128 || L->d % 256 || L->g != 64 || L->E + 1 > 1024) {
        snprintf(msg, msg_len, "prefill path needs I %% 128 == 0, d %% 256 == 0, g == 64, E < 1024");
        return nullptr;
    }
    if (!get_encode()) {
        snprintf(msg, msg_len, "cuTensorMapEncodeTiled unavailable");
        return nullptr;
    }
    qk_prefill *p = new qk_prefill();
    memset(p, 0, sizeof(*p));
    p->L = *L;
    p->max_tokens = max_tokens;
    p->num_sms = num_sms;
    p->pool_slots = pool_slots;
    p->pool = pool;
    p->rows_max = max_tokens * (L->k + 1);
    // tuning knob: QMOE_GROUP_SMALL_ROWS in [0, 64] (0: k_gemm_sw never used)
    p->small_max = kSmallMax;
    if (const char *v = getenv("QMOE_GROUP_SMALL_ROWS")) {
        const int n = atoi(v);
        if (n >= 0 && n <= kSmallMax) p->small_max = n;
    }
    // tuning knob: QMOE_SMALL_PATH=tc keeps small groups on the tensor cores
    // (k_gemm_sw); the CUDA-core path covers d <= 2048 and I / 32 in {4, 16}
    p->sb = L->d <= 2048 && L->d % 256 == 0 && (L->I == 128 || L->I == 512) && L->g % 32 == 0;
    if (const char *v = getenv("QMOE_SMALL_PATH")) p->sb = p->sb && strcmp(v, "tc") != 0;
    // tuning knob: QMOE_SB_MAX_ROWS in [1, 8], the largest tile on the CUDA
    // cores (a token more costs them a pass over the unit; k_gemm_sw's cost
    // hardly depends on the rows)
    p->sb_max_rows = kSbMaxRows;
    if (const char *v = getenv("QMOE_SB_MAX_ROWS")) {
        const int m = atoi(v);
        if (m >= 1 && m <= kSbBatch) p->sb_max_rows = m;
    }
    p->tiles_max = p->rows_max / BM + L->E + 2;
    const size_t R = static_cast<size_t>(p->rows_max);
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = cudaMalloc(&p->counts, sizeof(int) * 2 * (L->E + 1));
    if (e == cudaSuccess) p->cursor = p->counts + (L->E + 1);
    if (e == cudaSuccess) e = cudaMalloc(&p->row0, sizeof(int) * (L->E + 1));
    if (e == cudaSuccess) e = cudaMalloc(&p->inv, sizeof(int) * static_cast<size_t>(max_tokens) * L->k);
    if (e == cudaSuccess) e = cudaMalloc(&p->perm_tok, sizeof(int) * R);
    if (e == cudaSuccess) e = cudaMalloc(&p->n_mtiles, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&p->n_stiles, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&p->n_rows, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&p->tiles, sizeof(MTile) * p->tiles_max);
    // groups of at most kSmallMax rows: at most kSmallMax / NS tiles each
    if (e == cudaSuccess) e = cudaMalloc(&p->stiles, sizeof(MTile) * (L->E + 1) * (kSmallMax / NS));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->sb_xq, static_cast<size_t>(max_tokens) * sb_xrow(L->d));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->sb_hq, R * sb_hrow(L->I));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->htiles, sizeof(MTile) * (L->E + 1) * (kSmallMax / NS));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->n_htiles, sizeof(int));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->ltiles, sizeof(MTile) * (L->E + 1) * (kSmallMax / NS));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->n_ltiles, sizeof(int));
    if (e == cudaSuccess && p->sb) e = cudaMalloc(&p->sb_ctr, 4 * sizeof(int));
    if (e == cudaSuccess && p->sb) e = cudaMemset(p->sb_ctr, 0, 4 * sizeof(int));
    if (e == cudaSuccess && p->sb) e = cudaStreamCreateWithFlags(&p->st2, cudaStreamNonBlocking);
    if (e == cudaSuccess && p->sb) e = cudaEventCreateWithFlags(&p->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess && p->sb) e = cudaEventCreateWithFlags(&p->ev_join, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&p->wtiles, sizeof(MTile) * p->tiles_max);
    if (e == cudaSuccess) e = cudaMalloc(&p->wstiles, sizeof(MTile) * (L->E + 1) * (kSmallMax / NS));
    if (e == cudaSuccess) e = cudaMalloc(&p->n_wtiles, 2 * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&p->wave, L->E + 1);
    if (e == cudaSuccess) e = cudaMalloc(&p->xp, 2 * R * L->d * sizeof(__half));  // hi, lo planes
    if (e == cudaSuccess) e = cudaMalloc(&p->H, 2 * R * L->I * sizeof(__half));  // hi, lo planes
    if (e == cudaSuccess) e = cudaMalloc(&p->Y, R * L->d * sizeof(float));
    if (e != cudaSuccess) {
        snprintf(msg, msg_len, "prefill workspace: %s", cudaGetErrorString(e));
        qk_prefill_destroy(p);
        return nullptr;
    }
    bool ok = map_2d_16(&p->tmX, p->xp, L->d, 2 * R, false) &&
              map_2d_16(&p->tmH, p->H, L->I, 2 * R, false) &&
              map_2d_16(&p->tmXs, p->xp, L->d, 2 * R, false, NS) &&
              map_2d_16(&p->tmHs, p->H, L->I, 2 * R, false, NS) &&
              map_2d_16(&p->tmXs8, p->xp, L->d, 2 * R, false, NS8) &&
              map_2d_16(&p->tmHs8, p->H, L->I, 2 * R, false, NS8) &&
              map_3d_u8(&p->tmQgu4, pool, L->gu_row, L->I, pool_slots, L->slot_bytes, 128, 128, true) &&
              map_3d_u8(&p->tmSgu4, pool, L->gu_row, L->I, pool_slots, L->slot_bytes, 32, 128) &&
              map_3d_u8(&p->tmQdn4, pool + L->gu_bytes, L->d_row, L->d, pool_slots, L->slot_bytes, 128, 128,
                        true) &&
              map_3d_u8(&p->tmSdn4, pool + L->gu_bytes, L->d_row, L->d, pool_slots, L->slot_bytes, 32, 256) &&
              map_3d_u8(&p->tmQgu, pool, L->gu_row, L->I, pool_slots, L->slot_bytes, 32, 128) &&
              map_3d_u8(&p->tmSgu, pool, L->gu_row, L->I, pool_slots, L->slot_bytes, 16, 128) &&
              map_3d_u8(&p->tmQdn, pool + L->gu_bytes, L->d_row, L->d, pool_slots, L->slot_bytes, 32,
                        256) &&
              map_3d_u8(&p->tmSdn, pool + L->gu_bytes, L->d_row, L->d, pool_slots, L->slot_bytes, 16,
                        256);
    if (!ok) {
        snprintf(msg, msg_len, "prefill: tensor map encoding failed");
        qk_prefill_destroy(p);
        return nullptr;
    }
    // tensor-core routing: E a multiple of 16 (whole 16-column epilogue
    // chunks; router rows past E read as zeros), the shapes' workspace
    const int nE = (L->E + 31) / 32 * 32;
    p->Tpad = (max_tokens + BM - 1) / BM * BM;
    p->route_smem = (2 * static_cast<size_t>(L->d) + nE) * 4;
    p->route_ok = L->E % 16 == 0 && L->k <= 32 && p->route_smem <= 200 * 1024;
    if (p->route_ok) {
        const size_t Tp = static_cast<size_t>(p->Tpad);
        e = cudaMalloc(&p->xr, 2 * Tp * L->d * sizeof(__nv_bfloat16));
        if (e == cudaSuccess) e = cudaMalloc(&p->xnorm, Tp * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&p->lga, static_cast<size_t>(max_tokens) * L->E * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&p->rtiles, sizeof(MTile) * (Tp / BM));
        if (e == cudaSuccess) e = cudaMalloc(&p->rn, sizeof(int));
        if (e != cudaSuccess) {
            snprintf(msg, msg_len, "prefill routing workspace: %s", cudaGetErrorString(e));
            qk_prefill_destroy(p);
            return nullptr;
        }
        CUtensorMap probe;  // the per-call router map, encoded once here as a check
        p->route_ok = map_2d_16(&p->tmXr, p->xr, L->d, 2 * Tp, true) &&
                      map_2d_16(&probe, p->xr, L->d, L->E, true, 256);
    }
    const void *fns[9] = {reinterpret_cast<const void *>(&k_gemm<0>),
                          reinterpret_cast<const void *>(&k_gemm<1>),
                          reinterpret_cast<const void *>(&k_gemm<3>),
                          reinterpret_cast<const void *>(&k_gemm_sw<0>),
                          reinterpret_cast<const void *>(&k_gemm_sw<1>),
                          reinterpret_cast<const void *>(&k_gemm_sw<3>),
                          reinterpret_cast<const void *>(&k_gemm<2>),
                          reinterpret_cast<const void *>(&k_route_exact<kRW>),
                          reinterpret_cast<const void *>(&k_route_exact<kRWsmall>)};
    const int smem[9] = {Cfg<0>::Smem, Cfg<1>::Smem, Cfg<3>::Smem, CfgS<0>::Smem, CfgS<1>::Smem,
                         CfgS<3>::Smem, Cfg<2>::Smem, static_cast<int>(p->route_smem),
                         static_cast<int>(p->route_smem)};
    for (int i = 0; i < (p->route_ok ? 9 : 6); ++i) {
        e = cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize, smem[i]);
        if (e != cudaSuccess) {
            snprintf(msg, msg_len, "prefill: %s", cudaGetErrorString(e));
            qk_prefill_destroy(p);
            return nullptr;
        }
    }
    if (p->route_ok && route_approx_smem(L->d) <= kRaSmemMax) {
        e = cudaFuncSetAttribute(reinterpret_cast<const void *>(&k_route_approx),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, route_approx_smem(L->d));
        if (e != cudaSuccess) {
            snprintf(msg, msg_len, "prefill: %s", cudaGetErrorString(e));
            qk_prefill_destroy(p);
            return nullptr;
        }
    }
    if (p->sb) {
        const void *sfn[3] = {reinterpret_cast<const void *>(&k_sb_gu), reinterpret_cast<const void *>(&k_sb_dn<4>),
                              reinterpret_cast<const void *>(&k_sb_dn<16>)};
        const int ssm[3] = {sb_gu_smem(*L), sb_dn_smem(*L), sb_dn_smem(*L)};
        for (int i = 0; i < 3; ++i) {
            e = cudaFuncSetAttribute(sfn[i], cudaFuncAttributeMaxDynamicSharedMemorySize, ssm[i]);
            if (e != cudaSuccess) {
                snprintf(msg, msg_len, "prefill: %s", cudaGetErrorString(e));
                qk_prefill_destroy(p);
                return nullptr;
            }
        }
    }
    return p;
}

namespace {

// Grouping, gather and the two grouped GEMMs for T "tokens" (rows of x) with
// k routed slots each (idx [T, k], global expert ids with a slot in
// slot_of; -1 for none), plus the shared expert over the first nsh rows.
// Leaves the down outputs in p->Y (shared rows first) and the row of each
// (token, slot) in p->inv. events: NULL or 3 events (after grouping+gather,
// gate/up, down).
// phases: 1 = grouping and gather, 2 = the two GEMMs (both by default).
// wave != 0: the GEMMs take the wave tile lists (p->wtiles, p->wstiles).
cudaError_t grouped(qk_prefill *p, const void *x, int x_kind, int T, const int32_t *idx, int k,
                    int nsh, int routed_max, const int32_t *slot_of, int shared_slot_index,
                    int *err, cudaStream_t st, void **events, int phases = 3, int wave = 0) {
    const qk_layout &L = p->L;
    const int E = L.E;
    const int nk = T * k;
    const int rows = nsh + nk;
    if (rows > p->rows_max || nk > p->max_tokens * L.k) return cudaErrorInvalidValue;
    auto mark = [&](int i) {
        if (events) cudaEventRecordWithFlags(static_cast<cudaEvent_t>(events[i]), st,
                                             cudaEventRecordExternal);
    };
    // No group can exceed the small-tile limit (each token is in a group at
    // most once): every group runs on k_gemm_sw. Otherwise every group runs
    // on k_gemm (a second, small-tile launch beside it measured slower on the
    // prefill workload).
    const bool all_small = nsh <= p->small_max && routed_max <= p->small_max;
    const bool lo = x_kind == XK_F32;  // x as an fp16 hi/lo pair
    PlanOut po;
    po.small_max = all_small ? p->small_max : 0;
    po.tiles = p->tiles;
    po.stiles = p->stiles;
    po.n_tiles = p->n_mtiles;
    po.n_stiles = p->n_stiles;
    po.n_rows = p->n_rows;
    cudaError_t e = cudaSuccess;
    if (!(phases & 1)) {
        // GEMMs only (a wave of an earlier plan)
    } else if (nk <= kPlanSmall) {
        k_plan_small<<<1, 1024, 0, st>>>(idx, nk, k, E, nsh, slot_of, shared_slot_index, po, p->inv,
                                         p->perm_tok);
    } else {
        // counts and cursors in one allocation, cleared together
        e = cudaMemsetAsync(p->counts, 0, sizeof(int) * 2 * (E + 1), st);
        if (e != cudaSuccess) return e;
        k_count<<<(nk + 255) / 256, 256, 0, st>>>(idx, nk, p->counts);
        k_plan<<<1, 1024, 0, st>>>(p->counts, E, nsh, slot_of, shared_slot_index, p->row0, po);
        k_place<<<(nk + 255) / 256, 256, 0, st>>>(idx, nk, k, p->row0, p->cursor, p->inv,
                                                 p->perm_tok);
    }
    // small groups on the CUDA cores: x quantised per token (by the plan
    // phase; the waves of a call read it) instead of the grouped fp16 rows
    const bool sb = all_small && p->sb;
    const bool xq_split = sb && (phases & 1) && !wave && T > 0;  // xq's block 0 splits the tiles
    if (sb && (phases & 1) && T > 0)
        k_sb_xq<<<T + (xq_split ? 1 : 0), (L.d / 8 + 31) / 32 * 32, 0, st>>>(x, x_kind, L.d, T, p->sb_xq,
                                                       xq_split ? p->stiles : nullptr, p->n_stiles,
                                                       p->sb_max_rows, p->ltiles, p->n_ltiles,
                                                       p->htiles, p->n_htiles, idx, k, nsh, p->inv,
                                                       p->xp, static_cast<size_t>(p->rows_max) * L.d);
    else if ((phases & 1) && rows > 0)
        k_gather<<<(rows * 32 + 255) / 256, 256, 0, st>>>(x, x_kind, L.d, nsh, rows, p->n_rows,
                                                         p->perm_tok, p->xp,
                                                         static_cast<size_t>(p->rows_max) * L.d);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    mark(0);
    if (!(phases & 2)) return cudaSuccess;
    MTile *tl = wave ? p->wtiles : p->tiles, *stl = wave ? p->wstiles : p->stiles;
    int *ntl = wave ? p->n_wtiles : p->n_mtiles, *nstl = wave ? p->n_wtiles + 1 : p->n_stiles;

    auto launch = [&](const void *fn, int smem, const CUtensorMap *a, const CUtensorMap *q,
                      const CUtensorMap *sc, GemmArgs *ga, int threads) {
        void *args[] = {const_cast<CUtensorMap *>(a), const_cast<CUtensorMap *>(q),
                        const_cast<CUtensorMap *>(sc), ga};
        return qk_launch_raw(fn, dim3(p->num_sms), dim3(threads), smem, st, 0, args);
    };
    auto fn = [](auto f) { return reinterpret_cast<const void *>(f); };
    auto launch_sw = [&](const void *f, int smem, const CUtensorMap *a, const CUtensorMap *a8,
                         const CUtensorMap *q, const CUtensorMap *sc, GemmArgs *ga,
                         cudaStream_t on = nullptr) {
        void *args[] = {const_cast<CUtensorMap *>(a), const_cast<CUtensorMap *>(a8),
                        const_cast<CUtensorMap *>(q), const_cast<CUtensorMap *>(sc), ga};
        return qk_launch_raw(f, dim3(p->num_sms), dim3(kThreadsSw), smem, on ? on : st, 0, args);
    };
    GemmArgs gu;
    memset(&gu, 0, sizeof(gu));
    gu.mode = lo ? 3 : 0;
    gu.KB = L.d / BK;
    gu.ld_out = L.I;
    gu.n_cols = L.I;
    gu.d = L.d;
    gu.I = L.I;
    gu.rows_max = p->rows_max;
    gu.lo_plane = static_cast<size_t>(p->rows_max) * L.I;
    gu.out = p->H;
    gu.outf = nullptr;
    gu.err = err;
    GemmArgs dn = gu;
    dn.mode = 1;
    dn.KB = L.I / BK;
    dn.ld_out = L.d;
    dn.n_cols = L.d;
    dn.out = nullptr;
    dn.outf = p->Y;
    if (sb) {
        if (!xq_split) {
            k_split_tiles<<<1, 1024, 0, st>>>(stl, nstl, p->sb_max_rows, p->ltiles, p->n_ltiles, p->htiles,
                                              p->n_htiles);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        // the heavy tiles on the tensor cores, on the second stream beside
        // k_sb_* (which take their units from a counter, so they fill the
        // SMs k_gemm_sw leaves)
        e = cudaEventRecord(p->ev_fork, st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->st2, p->ev_fork, 0);
        if (e != cudaSuccess) return e;
        gu.NT = L.I / 128;
        gu.tiles = p->htiles;
        gu.n_mtiles = p->n_htiles;
        e = lo ? launch_sw(fn(&k_gemm_sw<3>), CfgS<3>::Smem, &p->tmXs, &p->tmXs8, &p->tmQgu4, &p->tmSgu4, &gu, p->st2)
               : launch_sw(fn(&k_gemm_sw<0>), CfgS<0>::Smem, &p->tmXs, &p->tmXs8, &p->tmQgu4, &p->tmSgu4, &gu, p->st2);
        if (e != cudaSuccess) return e;
        dn.NT = L.d / 256;
        dn.tiles = p->htiles;
        dn.n_mtiles = p->n_htiles;
        e = launch_sw(fn(&k_gemm_sw<1>), CfgS<1>::Smem, &p->tmHs, &p->tmHs8, &p->tmQdn4, &p->tmSdn4, &dn, p->st2);
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_join, p->st2);
        if (e != cudaSuccess) return e;
        SbArgs sa;
        sa.tiles = p->ltiles;
        sa.n_tiles = p->n_ltiles;
        sa.nsh = nsh;
        sa.perm_tok = p->perm_tok;
        sa.pool = p->pool;
        sa.L = L;
        sa.xq = p->sb_xq;
        sa.hq = p->sb_hq;
        sa.Y = p->Y;
        sa.ctr = p->sb_ctr;
        sa.err = err;
        void *args[] = {&sa};
        e = qk_launch_raw(reinterpret_cast<const void *>(&k_sb_gu), dim3(p->num_sms), dim3(kSbThreads),
                          sb_gu_smem(L), st, 0, args);
        if (e != cudaSuccess) return e;
        mark(1);
        sa.ctr = p->sb_ctr + 2;
        const void *dfn = L.I == 128 ? reinterpret_cast<const void *>(&k_sb_dn<4>)
                                     : reinterpret_cast<const void *>(&k_sb_dn<16>);
        e = qk_launch_raw(dfn, dim3(p->num_sms), dim3(kSbThreads), sb_dn_smem(L), st, 0, args);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, p->ev_join, 0);
        if (e != cudaSuccess) return e;
    } else if (all_small) {
        gu.NT = L.I / 128;
        gu.tiles = stl;
        gu.n_mtiles = nstl;
        e = lo ? launch_sw(fn(&k_gemm_sw<3>), CfgS<3>::Smem, &p->tmXs, &p->tmXs8, &p->tmQgu4, &p->tmSgu4, &gu)
               : launch_sw(fn(&k_gemm_sw<0>), CfgS<0>::Smem, &p->tmXs, &p->tmXs8, &p->tmQgu4, &p->tmSgu4, &gu);
        if (e != cudaSuccess) return e;
        mark(1);
        dn.NT = L.d / 256;
        dn.tiles = stl;
        dn.n_mtiles = nstl;
        e = launch_sw(fn(&k_gemm_sw<1>), CfgS<1>::Smem, &p->tmHs, &p->tmHs8, &p->tmQdn4, &p->tmSdn4, &dn);
        if (e != cudaSuccess) return e;
    } else {
        gu.NT = L.I / 128;
        gu.tiles = tl;
        gu.n_mtiles = ntl;
        e = lo ? launch(fn(&k_gemm<3>), Cfg<3>::Smem, &p->tmX, &p->tmQgu, &p->tmSgu, &gu, kThreads)
               : launch(fn(&k_gemm<0>), Cfg<0>::Smem, &p->tmX, &p->tmQgu, &p->tmSgu, &gu, kThreads);
        if (e != cudaSuccess) return e;
        mark(1);
        dn.NT = L.d / 256;
        dn.tiles = tl;
        dn.n_mtiles = ntl;
        e = launch(fn(&k_gemm<1>), Cfg<1>::Smem, &p->tmH, &p->tmQdn, &p->tmSdn, &dn, kThreads);
        if (e != cudaSuccess) return e;
    }
    mark(2);
    return cudaSuccess;
}

}  // namespace

extern "C" int qk_launch_prefill(qk_prefill *p, const qk_fwd *f, int shared_slot_index,
                                 void *stream, void **events) {
    const qk_layout &L = p->L;
    const int T = f->T, k = L.k;
    if (T > p->max_tokens) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // diagnostics: events[0..3] bracket grouping+gather, gate/up, down, combine
    cudaError_t e = grouped(p, f->x, f->x_bf16 ? XK_BF16 : XK_F32, T, f->idx, k, T, T, f->slot_of,
                            shared_slot_index, f->err, st, events);
    if (e != cudaSuccess) return e;
    k_combine<<<T, combine_threads(T, L.d), 0, st>>>(p->Y, p->Y, p->inv, f->wts, f->sgate, k, L.d, f->out);
    if (events) cudaEventRecordWithFlags(static_cast<cudaEvent_t>(events[3]), st, cudaEventRecordExternal);
    return cudaGetLastError();
}

extern "C" uint8_t *qk_prefill_wave_mask(qk_prefill *p) { return p->wave; }

extern "C" int qk_prefill_plan(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream) {
    const int T = f->T;
    if (T > p->max_tokens) return cudaErrorInvalidValue;
    return grouped(p, f->x, f->x_bf16 ? XK_BF16 : XK_F32, T, f->idx, p->L.k, T, T, f->slot_of,
                   shared_slot_index, f->err, static_cast<cudaStream_t>(stream), nullptr, 1);
}

extern "C" int qk_prefill_wave(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    k_wave_tiles<<<1, 1024, 0, st>>>(p->tiles, p->n_mtiles, p->stiles, p->n_stiles, p->wave,
                                     f->slot_of, p->wtiles, p->n_wtiles, p->wstiles, p->n_wtiles + 1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int T = f->T;
    return grouped(p, f->x, f->x_bf16 ? XK_BF16 : XK_F32, T, f->idx, p->L.k, T, T, f->slot_of,
                   shared_slot_index, f->err, st, nullptr, 2, 1);
}

extern "C" int qk_prefill_combine(qk_prefill *p, const qk_fwd *f, void *stream) {
    const int T = f->T;
    k_combine<<<T, combine_threads(T, p->L.d), 0, static_cast<cudaStream_t>(stream)>>>(
        p->Y, p->Y, p->inv, f->wts, f->sgate, p->L.k, p->L.d, f->out);
    return cudaGetLastError();
}

// ---- peer-memory exchange: every rank's receive-side buffers mapped into
// every rank (CUDA IPC), so rows go straight into their destination's
// buffers over NVLink; per-rank flags [2][64] (dispatch, return; indexed by
// the writing rank) carry the call's epoch (this rank's counter + 1: every
// rank runs the same calls, so the counters advance in step).

QK_DEV void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
QK_DEV unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// After a CTA's peer writes: every thread fences them at system scope, the
// CTA counts itself done, and the last CTA of the grid raises flag slot
// `which` of this rank on every destination (dst_mask bit g: rank g).
QK_DEV void ep_signal(const EpPeers *peers, int which, int me, int G, unsigned long long e, unsigned *done) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(done, 1u) == gridDim.x - 1) {
        *done = 0;  // the next call's count (stream-ordered after this grid)
        __threadfence_system();
        for (int g = 0; g < G; ++g) st_release_sys(peers->flags[g] + which * 64 + me, e);
    }
}

// The dispatch of k_ep_pack, written into rank g's receive rows
// cap + me * cap + t (its rows [0, cap) are its own tokens).
__global__ void k_ep_pack_p2p(const uint8_t *x, int row_bytes, int T, int cap, int k, int e_per, int G, int me,
                              const int32_t *idx, const float *wts, const unsigned long long *mask,
                              const EpPeers *peers, const unsigned long long *epoch, unsigned *done) {
    const int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wi < G * cap) {
        const int g = wi / cap, t = wi % cap;
        const size_t row = static_cast<size_t>(cap) * (1 + me) + t;
        const bool live = t < T && ((mask[t] >> g) & 1ull);
        if (lane < k) {
            const int e = live ? idx[t * k + lane] : -1;
            const bool own = live && e / e_per == g;
            peers->recv_e[g][row * k + lane] = own ? e : -1;
            peers->recv_w[g][row * k + lane] = own ? wts[t * k + lane] : 0.f;
        }
        if (live) {
            const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * row_bytes);
            uint4 *dst = reinterpret_cast<uint4 *>(peers->recv_x[g] + row * row_bytes);
            for (int c = lane; c < row_bytes / 16; c += 32) dst[c] = src[c];
        }
    }
    ep_signal(peers, 0, me, G, *epoch + 1, done);
}

// Waits (one thread per source rank, bounded) until every rank's flag
// `which` carries this call's epoch; the return wait then advances the
// epoch for the next call.
__global__ void k_ep_wait(const unsigned long long *flags, int which, int G, unsigned long long *epoch, int *err) {
    const unsigned long long e = *epoch + 1;
    const int g = threadIdx.x;
    if (g < G) {
        const unsigned long long *fl = flags + which * 64 + g;
        if (ld_acquire_sys(fl) < e) {
            const uint64_t t0 = gtimer();
            while (ld_acquire_sys(fl) < e) {
                if (gtimer() - t0 > kWaitNs) {
                    atomicOr(err, QK_ERR_TIMEOUT_GRID);
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (which == 1 && threadIdx.x == 0) *epoch = e;
}

// The expert-side combine of k_ep_partial for received row j (source rank
// j / cap, its token j % cap), written into the source's return row
// me * cap + t; rows that carry none of this rank's experts are not sent
// (their owner does not read them).
__global__ void k_ep_partial_p2p(const float *Y, const int *inv, const int32_t *e_of, const float *w, int k,
                                 int d, int cap, int G, int me, const EpPeers *peers,
                                 const unsigned long long *epoch, unsigned *done) {
    const int r = blockIdx.x;
    bool live = false;
    for (int s = 0; s < k; ++s) live |= e_of[static_cast<size_t>(r) * k + s] >= 0;
    if (live) {
        float *dst = peers->back[r / cap] + (static_cast<size_t>(me) * cap + r % cap) * d;
        for (int c = threadIdx.x; c < d / 4; c += blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s = 0; s < k; ++s) {
                const size_t a = static_cast<size_t>(r) * k + s;
                if (e_of[a] < 0) continue;
                const float4 v = reinterpret_cast<const float4 *>(Y + static_cast<size_t>(inv[a]) * d)[c];
                const float ws = w[a];
                acc.x = fmaf(ws, v.x, acc.x);
                acc.y = fmaf(ws, v.y, acc.y);
                acc.z = fmaf(ws, v.z, acc.z);
                acc.w = fmaf(ws, v.w, acc.w);
            }
            reinterpret_cast<float4 *>(dst)[c] = acc;
        }
    }
    ep_signal(peers, 1, me, G, *epoch + 1, done);
}

extern "C" int qk_ep_alloc(qk_prefill *p, int T, int G) {
    const qk_layout &L = p->L;
    const size_t rows = static_cast<size_t>(T) * G;  // both directions: at most T per pair
    // the receive side holds the own T tokens first, then up to T per rank
    if (G > 64 || rows + T > static_cast<size_t>(p->max_tokens)) return cudaErrorInvalidValue;
    p->ep_T = T;
    p->ep_G = G;
    const size_t d = static_cast<size_t>(L.d), k = static_cast<size_t>(L.k);
    cudaError_t e = cudaMalloc(&p->ep_mask, sizeof(unsigned long long) * T);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_send_e, sizeof(int32_t) * rows * k);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_recv_e, sizeof(int32_t) * (rows + T) * k);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_send_w, sizeof(float) * rows * k);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_recv_w, sizeof(float) * (rows + T) * k);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_send_x, sizeof(float) * rows * d);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_recv_x, sizeof(float) * (rows + T) * d);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_ret, sizeof(float) * rows * d);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_back, sizeof(float) * rows * d);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_flags, sizeof(unsigned long long) * 2 * 64);
    if (e == cudaSuccess) e = cudaMemset(p->ep_flags, 0, sizeof(unsigned long long) * 2 * 64);
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_epoch, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(p->ep_epoch, 0, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_done, 2 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(p->ep_done, 0, 2 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMalloc(&p->ep_peers_dev, sizeof(EpPeers));
    return e;
}

extern "C" int qk_ep_ipc_handles(qk_prefill *p, unsigned char *out) {
    void *bufs[5] = {p->ep_recv_x, p->ep_recv_e, p->ep_recv_w, p->ep_back, p->ep_flags};
    for (int i = 0; i < 5; ++i) {
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, bufs[i]);
        if (e != cudaSuccess) return e;
        memcpy(out + 64 * i, &h, 64);
    }
    return cudaSuccess;
}

extern "C" void qk_ep_p2p_close(qk_prefill *p) {
    if (!p->ep_p2p) return;
    for (int g = 0; g < p->ep_G; ++g)
        if (p->ep_peers.back[g] != p->ep_back) {
            cudaIpcCloseMemHandle(p->ep_peers.recv_x[g]);
            cudaIpcCloseMemHandle(p->ep_peers.recv_e[g]);
            cudaIpcCloseMemHandle(p->ep_peers.recv_w[g]);
            cudaIpcCloseMemHandle(p->ep_peers.back[g]);
            cudaIpcCloseMemHandle(p->ep_peers.flags[g]);
        }
    p->ep_p2p = 0;
}

extern "C" int qk_ep_p2p_open(qk_prefill *p, const unsigned char *all, int rank) {
    EpPeers pe;
    memset(&pe, 0, sizeof(pe));
    cudaError_t e = cudaSuccess;
    for (int g = 0; g < p->ep_G && e == cudaSuccess; ++g) {
        if (g == rank) {
            pe.recv_x[g] = p->ep_recv_x;
            pe.recv_e[g] = p->ep_recv_e;
            pe.recv_w[g] = p->ep_recv_w;
            pe.back[g] = p->ep_back;
            pe.flags[g] = p->ep_flags;
            continue;
        }
        void *ptr[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
        for (int i = 0; i < 5 && e == cudaSuccess; ++i) {
            cudaIpcMemHandle_t h;
            memcpy(&h, all + (static_cast<size_t>(g) * 5 + i) * 64, 64);
            e = cudaIpcOpenMemHandle(&ptr[i], h, cudaIpcMemLazyEnablePeerAccess);
        }
        if (e != cudaSuccess) {
            for (int i = 0; i < 5; ++i)
                if (ptr[i]) cudaIpcCloseMemHandle(ptr[i]);
            break;
        }
        pe.recv_x[g] = static_cast<uint8_t *>(ptr[0]);
        pe.recv_e[g] = static_cast<int32_t *>(ptr[1]);
        pe.recv_w[g] = static_cast<float *>(ptr[2]);
        pe.back[g] = static_cast<float *>(ptr[3]);
        pe.flags[g] = static_cast<unsigned long long *>(ptr[4]);
    }
    if (e != cudaSuccess) {
        for (int g = 0; g < p->ep_G; ++g)
            if (g != rank && pe.back[g]) {
                cudaIpcCloseMemHandle(pe.recv_x[g]);
                cudaIpcCloseMemHandle(pe.recv_e[g]);
                cudaIpcCloseMemHandle(pe.recv_w[g]);
                cudaIpcCloseMemHandle(pe.back[g]);
                cudaIpcCloseMemHandle(pe.flags[g]);
            }
        cudaGetLastError();
        return e;
    }
    e = cudaMemcpy(p->ep_peers_dev, &pe, sizeof(pe), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return e;
    p->ep_peers = pe;
    p->ep_p2p = 1;
    return cudaSuccess;
}

extern "C" void qk_ep_buffers(qk_prefill *p, qk_ep_bufs *b) {
    b->send_x = p->ep_send_x;
    b->send_e = p->ep_send_e;
    b->send_w = p->ep_send_w;
    b->recv_x = p->ep_recv_x;
    b->recv_e = p->ep_recv_e;
    b->recv_w = p->ep_recv_w;
    b->ret = p->ep_ret;
    b->back = p->ep_back;
}

extern "C" int qk_ep_dispatch(qk_prefill *p, const qk_fwd *f, void *stream) {
    const qk_layout &L = p->L;
    const int T = f->T, G = p->ep_G, cap = p->ep_T;
    if (T > cap || L.E % G) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int e_per = L.E / G;
    if (T > 0)
        k_ep_mask<<<(T + 255) / 256, 256, 0, st>>>(f->idx, T, L.k, e_per, p->ep_mask);
    const int row_bytes = L.d * (f->x_bf16 ? 2 : 4);
    const uint8_t *x = static_cast<const uint8_t *>(f->x);
    k_ep_pack<<<(G * cap * 32 + 255) / 256, 256, 0, st>>>(x, row_bytes, T, cap, L.k, e_per, G,
                                                         f->idx, f->wts, p->ep_mask, p->ep_send_x,
                                                         p->ep_send_e, p->ep_send_w);
    // this rank's own tokens lead the receive buffer (rows [0, cap): shared
    // expert only)
    k_ep_own<<<(cap * 32 + 255) / 256, 256, 0, st>>>(x, row_bytes, T, cap, L.k, p->ep_recv_x, p->ep_recv_e);
    return cudaGetLastError();
}

extern "C" int qk_ep_dispatch_p2p(qk_prefill *p, const qk_fwd *f, int rank, void *stream) {
    const qk_layout &L = p->L;
    const int T = f->T, G = p->ep_G, cap = p->ep_T;
    if (!p->ep_p2p || T > cap || L.E % G) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int e_per = L.E / G;
    if (T > 0)
        k_ep_mask<<<(T + 255) / 256, 256, 0, st>>>(f->idx, T, L.k, e_per, p->ep_mask);
    const int row_bytes = L.d * (f->x_bf16 ? 2 : 4);
    const uint8_t *x = static_cast<const uint8_t *>(f->x);
    k_ep_own<<<(cap * 32 + 255) / 256, 256, 0, st>>>(x, row_bytes, T, cap, L.k, p->ep_recv_x, p->ep_recv_e);
    k_ep_pack_p2p<<<(G * cap * 32 + 255) / 256, 256, 0, st>>>(x, row_bytes, T, cap, L.k, e_per, G, rank,
                                                             f->idx, f->wts, p->ep_mask, p->ep_peers_dev,
                                                             p->ep_epoch, p->ep_done);
    return cudaGetLastError();
}

extern "C" int qk_ep_wait(qk_prefill *p, int which, int *err, void *stream) {
    k_ep_wait<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(p->ep_flags, which, p->ep_G, p->ep_epoch, err);
    return cudaGetLastError();
}

// The experts pass over rows [0, cap + rows): the own tokens (rows [0, T))
// through the shared expert, the received rows (from cap on) through this
// rank's experts; then each received row's partial, kept here (the caller
// returns it) or, with the peer table, written into its owner's return row.
static int ep_experts(qk_prefill *p, const qk_fwd *f, int shared_slot_index, int rank, bool p2p,
                      void *stream) {
    const qk_layout &L = p->L;
    const int T = f->T, cap = p->ep_T, rows = cap * p->ep_G;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = grouped(p, p->ep_recv_x, f->x_bf16 ? XK_BF16 : XK_F32, cap + rows, p->ep_recv_e,
                            L.k, T, rows, f->slot_of, shared_slot_index, f->err, st, nullptr);
    if (e != cudaSuccess) return e;
    const size_t o = static_cast<size_t>(cap) * L.k;
    if (p2p)
        k_ep_partial_p2p<<<rows, 256, 0, st>>>(p->Y, p->inv + o, p->ep_recv_e + o, p->ep_recv_w + o, L.k,
                                               L.d, cap, p->ep_G, rank, p->ep_peers_dev, p->ep_epoch,
                                               p->ep_done + 1);
    else
        k_ep_partial<<<rows, 256, 0, st>>>(p->Y, p->inv + o, p->ep_recv_e + o, p->ep_recv_w + o, L.k, L.d,
                                           p->ep_ret);
    return cudaGetLastError();
}

extern "C" int qk_ep_experts(qk_prefill *p, const qk_fwd *f, int shared_slot_index, void *stream) {
    return ep_experts(p, f, shared_slot_index, 0, false, stream);
}

extern "C" int qk_ep_experts_p2p(qk_prefill *p, const qk_fwd *f, int shared_slot_index, int rank,
                                 void *stream) {
    if (!p->ep_p2p) return cudaErrorInvalidValue;
    return ep_experts(p, f, shared_slot_index, rank, true, stream);
}

extern "C" int qk_ep_finish(qk_prefill *p, const qk_fwd *f, void *stream) {
    const qk_layout &L = p->L;
    const int T = f->T;
    if (T == 0) return cudaSuccess;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the shared rows are Y[0, T) of the experts pass
    k_ep_final<<<T, 256, 0, st>>>(p->ep_back, p->ep_mask, T, p->ep_T, p->ep_G, p->Y, f->sgate,
                                  L.d, f->out);
    return cudaGetLastError();
}

static int route_exact(qk_prefill *p, const qk_fwd *f, float wmax, cudaStream_t st, void *mid_event);

extern "C" int qk_launch_route(qk_prefill *p, const qk_fwd *f, float wmax, void *stream,
                               void *mid_event) {
    if (!p->route_ok) return QK_ROUTE_UNFIT;
    const qk_layout &L = p->L;
    const int T = f->T, E = L.E;
    if (T > p->max_tokens) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (T <= kRouteSmallT && route_approx_smem(L.d) <= kRaSmemMax) {
        k_route_approx<<<dim3((E + kRaExp - 1) / kRaExp, (T + kRaTok - 1) / kRaTok), kRaThreads,
                         route_approx_smem(L.d), st>>>(f->x, f->x_bf16, L.d, T, E, f->router, p->lga,
                                                       p->xnorm, f->err);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        return route_exact(p, f, wmax, st, mid_event);
    }
    k_route_split<<<(T * 32 + 255) / 256, 256, 0, st>>>(f->x, f->x_bf16, L.d, T, p->Tpad, p->xr,
                                                       p->xnorm, p->rtiles, p->rn);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap tmR;
    if (!map_2d_16(&tmR, f->router, L.d, E, true, 256)) return cudaErrorInvalidValue;
    GemmArgs ra;
    memset(&ra, 0, sizeof(ra));
    ra.mode = 2;
    ra.KB = L.d / BK;
    ra.NT = (E + BN - 1) / BN;
    ra.ld_out = E;
    ra.n_cols = E;
    ra.d = L.d;
    ra.I = L.I;
    ra.tiles = p->rtiles;
    ra.n_mtiles = p->rn;
    ra.rows_max = p->Tpad;
    ra.outf = p->lga;
    ra.err = f->err;
    // small calls: split K so that more SMs share the router's 2 MiB (the
    // approximate logits then add up in a different order, which the bound
    // below allows: any order of the same fp32 additions stays within it)
    int ks = 1;
    if (T <= 512)
        while (ks * 2 <= ra.KB / 2 && (T + BM - 1) / BM * ra.NT * ks * 2 <= p->num_sms) ks *= 2;
    ra.ksplit = ks;
    if (ks > 1) {
        e = cudaMemsetAsync(p->lga, 0, sizeof(float) * static_cast<size_t>(T) * E, st);
        if (e != cudaSuccess) return e;
    }
    const int ntiles = (T + BM - 1) / BM * ra.NT * ks;
    {
        void *args[] = {&p->tmXr, &tmR, &tmR, &ra};
        e = qk_launch_raw(reinterpret_cast<const void *>(&k_gemm<2>),
                          dim3(ntiles < p->num_sms ? ntiles : p->num_sms), dim3(kThreads),
                          Cfg<2>::Smem, stream, 0, args);
        if (e != cudaSuccess) return e;
    }
    return route_exact(p, f, wmax, st, mid_event);
}

// The exact re-ranking of the approximate logits in p->lga (after either
// approximate pass).
static int route_exact(qk_prefill *p, const qk_fwd *f, float wmax, cudaStream_t st, void *mid_event) {
    const qk_layout &L = p->L;
    const int T = f->T, E = L.E;
    if (mid_event) cudaEventRecordWithFlags(static_cast<cudaEvent_t>(mid_event), st, cudaEventRecordExternal);
    RouteArgs a;
    a.x = f->x;
    a.x_bf16 = f->x_bf16;
    a.d = L.d;
    a.E = E;
    a.k = L.k;
    a.T = T;
    a.router = f->router;
    a.shared_gate = f->shared_gate;
    a.bias = f->logit_bias;
    a.lga = p->lga;
    a.xnorm = p->xnorm;
    a.wmax = wmax;
    a.idx = f->idx;
    a.wts = f->wts;
    a.sgate = f->sgate;
    a.err = f->err;
    if (T < p->num_sms)
        k_route_exact<kRWsmall><<<T, kRWsmall * 32, p->route_smem, st>>>(a);
    else
        k_route_exact<kRW><<<T, kRW * 32, p->route_smem, st>>>(a);
    return cudaGetLastError();
}
