// qmoe_dev.cuh - device helpers shared by the MoE kernels (sm_100a).
//
// mbarrier + cp.async.bulk staging with %globaltimer-bounded waits, the
// programmatic-dependent-launch controls, a bounded grid barrier, and the
// arithmetic building blocks that define the layer's results:
//   router_dot_smem / router_dot_lane  canonical fp64 router dot
//   quant_word / dot_unit_q            integer q4 dot products
//   topk_warp                          exact top-k + renormalised softmax
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "qmoe_internal.h"

#define QK_DEV __device__ __forceinline__
#define QK_FULL 0xffffffffu

namespace qk {

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s bound on every device wait

QK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QK_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

QK_DEV float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
QK_DEV float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

QK_DEV uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

QK_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

QK_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

QK_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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

QK_DEV uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of bar; false when it timed out.
QK_DEV bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (gtimer() - t0 > kWaitNs) return false;
    }
}

// Global -> shared bulk copy; dst, src and bytes are 16-byte multiples.
QK_DEV void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---- tensor-memory accelerator (TMA) tiled loads, each to this CTA only ----
QK_DEV void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

QK_DEV void tma_load_3d(void *dst, const void *tmap, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only); completion per
// thread with cp_async_wait_all.
QK_DEV void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst_smem)), "l"(src)
                 : "memory");
}
QK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
QK_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

QK_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Generic-proxy shared-memory writes made visible to the async proxy (the
// tensor cores read operands through it).
QK_DEV void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 (5th-generation tensor cores, accumulators in TMEM) ----
QK_DEV void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
QK_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
QK_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
QK_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QK_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16/bf16 operands,
// fp32 accumulation). Issued by one thread.
QK_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, A read from tensor
// memory (M rows in the lanes, K packed two 16-bit elements per 32-bit
// column). Issued by one thread.
QK_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                        uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp w reaches
// lanes [32 (w % 4), 32 (w % 4) + 32)).
QK_DEV void tmem_st32(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
QK_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives once on bar when all previously issued tcgen05.mma of this thread
// have completed.
QK_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
QK_DEV void tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
QK_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B
// (64 16-bit elements), 8-row atoms of 1024 B at stride 1024 B. Start
// address in 16-byte units; version 1 (sm_100).
QK_DEV uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused here)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride byte offset: 8-row atom
    d |= static_cast<uint64_t>(1) << 46;                 // descriptor version
    d |= static_cast<uint64_t>(2) << 61;                 // layout: SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::f16: fp16 (or bf16) A and B, both
// K-major, fp32 D. A and B always share one type.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16 = false) {
    return (1u << 4)                                   // D format f32
           | ((bf16 ? 1u : 0u) << 7)                   // A format: f16 0, bf16 1
           | ((bf16 ? 1u : 0u) << 10)                  // B format: same as A
           | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

QK_DEV unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

QK_DEV void st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

QK_DEV unsigned long long atom_add_release(unsigned long long *p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

QK_DEV unsigned long long ld_acquire64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Arrives at a grid barrier and waits for it: the CTA's writes so far are
// released (__syncthreads, then one red.release), then one thread polls the
// counter (acquire) until it reaches `target`. The caller knows the target
// (its launch's base plus the number of CTAs times the barrier's ordinal),
// so the arrive needs no reply. Bounded: on timeout QK_ERR_TIMEOUT_GRID is
// set and the CTA goes on (that launch's results are invalid).
QK_DEV void grid_arrive_wait(unsigned long long *ctr, unsigned long long target, int *err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
        if (ld_acquire64(ctr) < target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire64(ctr) < target) {
                if (gtimer() - t0 > kWaitNs) {
                    atomicOr(err, QK_ERR_TIMEOUT_GRID);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// The two halves of grid_arrive_wait, so that work that the barrier does not
// order can run between them: grid_arrive publishes the CTA's writes so far
// and arrives (fire-and-forget); grid_wait waits (bounded) for `target`.
QK_DEV void grid_arrive(unsigned long long *ctr) {
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
}
QK_DEV void grid_wait(unsigned long long *ctr, unsigned long long target, int *err) {
    if (threadIdx.x == 0 && ld_acquire64(ctr) < target) {
        const uint64_t t0 = gtimer();
        while (ld_acquire64(ctr) < target) {
            if (gtimer() - t0 > kWaitNs) {
                atomicOr(err, QK_ERR_TIMEOUT_GRID);
                break;
            }
        }
    }
    __syncthreads();
}

// Grid-wide barrier for a grid whose CTAs are all resident. `ctr` is a 64-bit
// counter that only grows: each CTA adds 1 with release semantics and waits
// (acquire) until the counter reaches the next multiple of the grid size,
// computed from the value its own add returned. No reset is needed between
// barriers or launches as long as every launch of the same grid size uses
// it. The spin is bounded: on timeout it sets QK_ERR_TIMEOUT_GRID and returns
// false (that call's results are then invalid, but the kernel ends).
QK_DEV bool grid_sync(unsigned long long *ctr, unsigned nctas, int *err) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned long long old = atom_add_release(ctr, 1ull);
        const unsigned long long target = (old / nctas + 1) * nctas;
        if (ld_acquire64(ctr) < target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire64(ctr) < target) {
                if (gtimer() - t0 > kWaitNs) {
                    atomicOr(err, QK_ERR_TIMEOUT_GRID);
                    ok = 0;
                    break;
                }
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// Integer q4 dot products. A q4 row times a vector v is, per 64-element
// group, s * sum(q_i v_i) + b * sum(v_i) (w = q s + b, the dequantised
// weights of model.c:1371-1375). v is stored once as integers
// v_i = round(v_i * 2^e), one power-of-two scale per 64 elements, in NB byte
// planes (plane 0 the signed high byte, the others unsigned): NB = 2 keeps 15
// significant bits of the group's largest |v| (used for x), NB = 3 keeps 22
// (used for h, whose groups have a much wider range). A q4 word w (8
// nibbles, low first) gives its even nibbles as the bytes of w & 0x0F0F0F0F
// and its odd ones as the bytes of (w >> 4) & 0x0F0F0F0F, so sum(q_i v_i)
// over the word is 2 NB dp4a (even/odd per plane), exact in int32: 0.9 (NB=2)
// or 1.1 (NB=3) instructions per weight against about 3 for a float
// dequantise-and-FMA. Each plane of a word is a uint2 {even bytes, odd
// bytes}; a vector of n words stores plane p at [p * n, (p + 1) * n).

// 2^e for e in [-126, 127]
QK_DEV float pow2i(int e) { return __int_as_float((127 + e) << 23); }

// Quantises the 8 values of one q4 word position into NB planes. The calling
// thread is lane 8a + r (r < 8) of a group of 8 consecutive lanes that
// together hold one 64-element group; every lane of the warp calls (inactive
// lanes pass zeros). Returns the group's scale 2^-e; *usum gets the unit's
// (4 words, 32 elements) sum of the quantised values, scaled back. A group
// with a non-finite value gets a NaN scale, so its dot products come out NaN
// as the float ones would.
// GL = 4 makes the scale per 32-element unit (four lanes) instead.
template <int NB, int GL = 8>
QK_DEV float quant_word(const float (&v)[8], uint2 (&pl)[NB], float *usum) {
    constexpr int kBits = NB == 2 ? 15 : 22;  // largest |v| 2^e in [2^(kBits-1), 2^kBits)
    constexpr int kMax = (1 << (8 * NB - 1)) - 1;
    float m = 0.f;
    bool fin = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m = fmaxf(m, fabsf(v[i]));
        fin = fin && isfinite(v[i]);
    }
#pragma unroll
    for (int off = 1; off < GL; off <<= 1) m = fmaxf(m, __shfl_xor_sync(QK_FULL, m, off));
    const unsigned bad = __ballot_sync(QK_FULL, !fin);
    const int lane = threadIdx.x & 31;
    const bool gfin = ((bad >> (lane & ~(GL - 1))) & ((1u << GL) - 1u)) == 0u;
    int ex = 0;
    frexpf(m, &ex);  // m = f 2^ex, f in [0.5, 1)
    int e = m > 0.f ? kBits - ex : 0;
    e = min(max(e, -126), 126);
    const float up = pow2i(e);
#pragma unroll
    for (int p = 0; p < NB; ++p) pl[p] = make_uint2(0u, 0u);
    int isum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = gfin ? min(__float2int_rn(v[i] * up), kMax) : 0;
        isum += q;
        const int sh = 8 * (i >> 1);
#pragma unroll
        for (int p = 0; p < NB; ++p) {
            const uint32_t b = (static_cast<uint32_t>(q >> (8 * (NB - 1 - p))) & 0xFFu) << sh;
            if (i & 1) pl[p].y |= b;
            else pl[p].x |= b;
        }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) isum += __shfl_xor_sync(QK_FULL, isum, off);
    const float scale = gfin ? pow2i(-e) : __int_as_float(0x7fc00000);
    *usum = static_cast<float>(isum) * scale;
    return scale;
}

// Stores one quantised word (NB planes) at word w of a vector of n words.
template <int NB>
QK_DEV void store_word(uint2 *planes, int n, int w, const uint2 (&pl)[NB]) {
#pragma unroll
    for (int p = 0; p < NB; ++p) planes[static_cast<size_t>(p) * n + w] = pl[p];
}

// The 4 words of unit u (NB planes) of a quantised vector of n words.
template <int NB>
QK_DEV void load_unit(const uint2 *planes, int n, int u, uint2 (&v)[NB][4]) {
#pragma unroll
    for (int p = 0; p < NB; ++p) {
        const uint4 *s = reinterpret_cast<const uint4 *>(planes + static_cast<size_t>(p) * n + 4 * u);
        const uint4 a = s[0], b = s[1];
        v[p][0] = make_uint2(a.x, a.y);
        v[p][1] = make_uint2(a.z, a.w);
        v[p][2] = make_uint2(b.x, b.y);
        v[p][3] = make_uint2(b.z, b.w);
    }
}

// sum(q_i v_i) over one 16-byte unit (32 nibbles), in units of the scale:
// exact for NB = 2 (below 2^24), one fp32 rounding for NB = 3.
template <int NB>
QK_DEV float dot_unit_q(const uint4 &w, const uint2 (&v)[NB][4]) {
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    int hi = 0;
    unsigned mid = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t ev = wd[i] & 0x0F0F0F0Fu, od = (wd[i] >> 4) & 0x0F0F0F0Fu;
        hi = __dp4a(static_cast<int>(ev), static_cast<int>(v[0][i].x), hi);
        hi = __dp4a(static_cast<int>(od), static_cast<int>(v[0][i].y), hi);
        if (NB == 3) {
            mid = __dp4a(ev, v[1][i].x, mid);
            mid = __dp4a(od, v[1][i].y, mid);
        }
        lo = __dp4a(ev, v[NB - 1][i].x, lo);
        lo = __dp4a(od, v[NB - 1][i].y, lo);
    }
    if (NB == 2) return static_cast<float>(hi * 256 + static_cast<int>(lo));
    return fmaf(static_cast<float>(hi), 65536.f, static_cast<float>(mid * 256u + lo));
}

// bf16 bits (low 16 bits of b) -> double, exactly. Normal numbers are
// rebuilt with integer operations (sign; exponent + 1023 - 127; the 7
// mantissa bits on top of the double's); zero, subnormals, infinities and
// NaN take the conversion instruction, which on this GPU issues at a small
// fraction of the rate of the integer path. (A branch-free form that builds
// every case with integer operations and selects measured slower: the router
// phase of the decode kernel went from 0.9 to 1.7 us.)
QK_DEV double bf16_to_f64(uint32_t b) {
    const uint32_t e = (b >> 7) & 0xFFu;
    if (e - 1u >= 254u) return static_cast<double>(__uint_as_float(b << 16));
    const uint32_t hi = ((b & 0x8000u) << 16) | (((b & 0x7FFFu) << 13) + (896u << 20));
    return __hiloint2double(static_cast<int>(hi), 0);
}

// fp32 -> fp64 by rebuilding the IEEE fields with integer operations
// (exponent + 1023 - 127, fraction shifted up by 29) for normal numbers;
// zero, subnormals, infinities and NaN take the conversion instruction.
QK_DEV double f32_to_f64(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t e = (u >> 23) & 0xFFu;
    if (e - 1u >= 254u) return static_cast<double>(x);
    const uint32_t hi = (u & 0x80000000u) | (((u & 0x7FFFFFFFu) >> 3) + (896u << 20));
    return __hiloint2double(static_cast<int>(hi), static_cast<int>(u << 29));
}

// Staged x for the canonical router dot: element k = 256 i + 8 l + j (lane
// l, j < 8) sits in double2 slot (4 i + j / 2) * 32 + l, so each lane's
// 128-bit reads are consecutive across the warp. rx_slot gives the slot of
// the pair (8 t + 2 q, 8 t + 2 q + 1) for word t = 32 i + l.
QK_DEV int rx_slot(int t, int q) { return ((t >> 5) * 4 + q) * 32 + (t & 31); }

// Stores x word t (8 values) into the staged layout.
QK_DEV void rx_store(double2 *rx, int t, const float (&v)[8]) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
        rx[rx_slot(t, q)] = make_double2(static_cast<double>(v[2 * q]), static_cast<double>(v[2 * q + 1]));
}

// Lane part of the canonical router dot (see oracle/moe_oracle.c,
// oracle_router_dot): lane l owns k = 256*i + 8*l + j; eight fp64 sums a[j]
// over i ascending; exact products; folded ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)).
// The caller finishes with a butterfly over lanes 16..1 and one rounding.
// w: d bf16 values; rx: x staged by rx_store (d a multiple of 256).
QK_DEV double router_lane(const uint16_t *w, const double2 *rx, int d, int lane) {
    double a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = 0.0;
#pragma unroll 4
    for (int i = 0; i < d / 256; ++i) {
        const uint4 wv = *reinterpret_cast<const uint4 *>(w + 256 * i + 8 * lane);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const double2 xv = rx[(4 * i + q) * 32 + lane];
            a[2 * q] = fma(xv.x, bf16_to_f64(ww[q] & 0xFFFFu), a[2 * q]);
            a[2 * q + 1] = fma(xv.y, bf16_to_f64(ww[q] >> 16), a[2 * q + 1]);
        }
    }
    return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// The same dot split across warps: this lane's sums a[j] for the NJ values
// j0 .. j0 + NJ - 1 (NJ = 2 or 4, j0 a multiple of NJ), folded as the
// canonical fold folds them, so combining the warps' parts as
//   NJ = 2: (p0 + p1) + (p2 + p3),  NJ = 4: P0 + P1
// gives router_lane's value bit for bit.
template <int NJ>
QK_DEV double router_lane_part(const uint16_t *w, const double2 *rx, int d, int lane, int j0) {
    double a[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) a[j] = 0.0;
#pragma unroll 4
    for (int i = 0; i < d / 256; ++i) {
#pragma unroll
        for (int q2 = 0; q2 < NJ / 2; ++q2) {
            const int q = j0 / 2 + q2;
            const uint32_t wv = *reinterpret_cast<const uint32_t *>(w + 256 * i + 8 * lane + 2 * q);
            const double2 xv = rx[(4 * i + q) * 32 + lane];
            a[2 * q2] = fma(xv.x, bf16_to_f64(wv & 0xFFFFu), a[2 * q2]);
            a[2 * q2 + 1] = fma(xv.y, bf16_to_f64(wv >> 16), a[2 * q2 + 1]);
        }
    }
    if (NJ == 2) return a[0] + a[1];
    return (a[0] + a[1]) + (a[2 % NJ] + a[3 % NJ]);
}

QK_DEV double warp_sum_butterfly(double s) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = s + __shfl_xor_sync(QK_FULL, s, off);
    return s;
}

// Order-preserving u32 key of a logit (-0 folded onto +0).
QK_DEV uint32_t fkey(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b << 1) == 0) b = 0;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

QK_DEV float key_value(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key ^ 0x80000000u) : ~key);
}

// Slow path of topk_warp: gathers the canonical top-k into s_key/s_idx
// (unordered) by finding the k-th largest key MSB-first (one redux.sync count
// per bit, early exit when exactly k keys qualify); ties at the threshold go
// to the lower expert ids. keys: nj*32 staged keys (0 = absent). Returns the
// number gathered (k on success).
QK_DEV int topk_gather_radix(const uint32_t *keys, int nj, int k, uint32_t *s_key, int *s_idx) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0;
    bool exact = false;
#pragma unroll 1
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = prefix | (1u << bit);
        int c = 0;
#pragma unroll 4
        for (int j = 0; j < nj; ++j) c += keys[j * 32 + lane] >= cand ? 1 : 0;
        const int cnt = static_cast<int>(__reduce_add_sync(QK_FULL, static_cast<unsigned>(c)));
        if (cnt >= k) {
            prefix = cand;
            if (cnt == k) {
                exact = true;
                break;
            }
        }
    }
    int base = 0, need_eq = 0;
    if (!exact) {
        int c = 0;
#pragma unroll 4
        for (int j = 0; j < nj; ++j) c += keys[j * 32 + lane] > prefix ? 1 : 0;
        need_eq = k - static_cast<int>(__reduce_add_sync(QK_FULL, static_cast<unsigned>(c)));
    }
#pragma unroll 1
    for (int j = 0; j < nj; ++j) {
        const uint32_t kk = keys[j * 32 + lane];
        bool sel;
        if (exact) {
            sel = kk >= prefix;
        } else {
            const bool eq = kk == prefix;
            const unsigned eqm = __ballot_sync(QK_FULL, eq);
            const int before = __popc(eqm & ((1u << lane) - 1u));
            sel = kk > prefix || (eq && before < need_eq);
            need_eq -= min(__popc(eqm), need_eq);
        }
        const unsigned m = __ballot_sync(QK_FULL, sel);
        if (sel) {
            const int pos = base + __popc(m & ((1u << lane) - 1u));
            if (pos < 32) {
                s_key[pos] = kk;
                s_idx[pos] = j * 32 + lane;
            }
        }
        base += __popc(m);
    }
    __syncwarp();
    return base;
}

// Global (L2) -> shared copy of n float4 by `nthreads` threads, with all of a
// thread's loads of a batch issued before its stores: a plain load/store
// loop costs one memory round trip per iteration, since the compiler cannot
// prove the global source and the shared destination do not alias.
QK_DEV void copy_f4_l2_to_smem(float4 *dst, const float4 *src, int n, int t, int nthreads) {
    constexpr int B = 8;
    for (int base = t; base < n; base += B * nthreads) {
        float4 v[B];
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int i = base + u * nthreads;
            if (i < n) v[u] = __ldcg(src + i);
        }
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int i = base + u * nthreads;
            if (i < n) dst[i] = v[u];
        }
    }
}

// Stages the order-preserving keys of E logits into keys[0, nj*32) (zero
// past E), shared by the calling group of `nthreads` threads (t = index in
// the group); loads are batched before stores. Callers synchronise before
// topk_warp.
template <bool CG>
QK_DEV void topk_stage_keys(const float *lg, int E, uint32_t *keys, int t, int nthreads) {
    constexpr int B = 8;
    const int n = (E + 31) / 32 * 32;
    for (int base = t; base < n; base += B * nthreads) {
        float v[B];
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int e = base + u * nthreads;
            v[u] = e < E ? (CG ? __ldcg(lg + e) : lg[e]) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < B; ++u) {
            const int e = base + u * nthreads;
            if (e < n) keys[e] = e < E ? fkey(v[u]) : 0u;
        }
    }
}

// Ranks C candidates (keys in s_key, expert ids in s_idx, C <= 32) by
// (value desc, index asc), writes the first k in that order to idx_out and
// the softmax over their logits to w_out (model.c:1305-1318). Any candidate
// set that contains every key ranked above a member of the top-k gives the
// same result as the full key array.
QK_DEV void topk_rank_softmax(int C, int k, uint32_t *s_key, int *s_idx, float *s_ev,
                              int *idx_out, float *w_out) {
    const int lane = threadIdx.x & 31;
    int rank = 0, mi = 0;
    uint32_t mk = 0;
    if (lane < C) {
        mk = s_key[lane];
        mi = s_idx[lane];
    }
    // rank among the candidates: lane m's (key, index) arrive by shuffle
#pragma unroll 4
    for (int m = 0; m < C; ++m) {
        const uint32_t ok = __shfl_sync(QK_FULL, mk, m);
        const int oi = __shfl_sync(QK_FULL, mi, m);
        rank += (ok > mk || (ok == mk && oi < mi)) ? 1 : 0;
    }
    const bool mine = lane < C && rank < k;
    float v = 0.f;
    if (mine) {
        v = key_value(mk);
        s_idx[rank] = mi;
        s_key[rank] = __float_as_uint(v);
    }
    __syncwarp();
    const float mx = __uint_as_float(s_key[0]);
    float ev = 0.f;
    if (mine) {
        ev = expf(v - mx);
        s_ev[rank] = ev;
    }
    __syncwarp();
    // the sum in rank order (the order of model.c:1311-1316), read by shuffles
    const float evr = lane < k ? s_ev[lane] : 0.f;
    float sum = 0.f;
    for (int m = 0; m < k; ++m) sum += __shfl_sync(QK_FULL, evr, m);
    if (mine) {
        idx_out[rank] = mi;
        w_out[rank] = ev / sum;
    }
    __syncwarp();
}

// Exact top-k of E staged keys by one warp (k <= 32), selection by
// (value desc, index asc), written in that order; w is the softmax over the
// selected logits (model.c:1305-1318).
//   1. tau = the k-th largest of the 32 lane maxima. At least k keys are
//      >= tau, so every member of the top-k (and every key tied with its
//      k-th value) is >= tau: the keys >= tau are a complete candidate set,
//      typically 10-20 of them.
//   2. The candidates are compacted in index order and each is ranked among
//      the candidates by (key desc, index asc); rank < k is the answer.
// When more than 32 keys qualify the radix path gathers the set instead.
// keys: (E+31)/32*32 staged keys; s_key/s_idx/s_ev: 32-entry scratch of this
// warp. Returns false if fewer than k keys exist.
// (out of line: the fallback of the decode kernel's top-k, kept apart from
// its hot code)
static __device__ __noinline__ bool topk_warp(const uint32_t *keys, int E, int k, uint32_t *s_key, int *s_idx,
                      float *s_ev, int *idx_out, float *w_out) {
    const int lane = threadIdx.x & 31;
    const int nj = (E + 31) / 32;
    uint32_t mxk = 0;
#pragma unroll 4
    for (int j = 0; j < nj; ++j) mxk = max(mxk, keys[j * 32 + lane]);
    int r = 0;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const uint32_t o = __shfl_sync(QK_FULL, mxk, j);
        r += (o > mxk || (o == mxk && j < lane)) ? 1 : 0;
    }
    const unsigned bm = __ballot_sync(QK_FULL, r == k - 1);
    const uint32_t tau = __shfl_sync(QK_FULL, mxk, __ffs(bm) - 1);
    // compaction: per-lane count, warp prefix sum, per-lane writes (the
    // candidate order is irrelevant: ranking compares indices explicitly)
    int own = 0;
#pragma unroll 4
    for (int j = 0; j < nj; ++j) {
        const uint32_t kk = keys[j * 32 + lane];
        own += (j * 32 + lane < E && kk >= tau && kk != 0u) ? 1 : 0;
    }
    int incl = own;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(QK_FULL, incl, off);
        if (lane >= off) incl += t;
    }
    const int C0 = __shfl_sync(QK_FULL, incl, 31);
    int C = C0;
    if (C0 <= 32) {
        int pos = incl - own;
#pragma unroll 4
        for (int j = 0; j < nj; ++j) {
            const int e = j * 32 + lane;
            const uint32_t kk = keys[e];
            if (e < E && kk >= tau && kk != 0u) {
                s_key[pos] = kk;
                s_idx[pos] = e;
                ++pos;
            }
        }
    }
    __syncwarp();
    if (C > 32) C = topk_gather_radix(keys, nj, k, s_key, s_idx);
    if (C < k || C > 32) return false;
    topk_rank_softmax(C, k, s_key, s_idx, s_ev, idx_out, w_out);
    return true;
}

}  // namespace qk
