// qmoe_synth_dev.cu - the seeded synthetic layers of qmoe_synth.c, generated
// on the device straight into the slot layout.
//
// Large benchmark stacks (76 layers of 512 experts, 69 GB) cannot be made on
// the host and uploaded in the time a benchmark has. The streams are the
// host generator's (counter-based splitmix64 keyed by seed, layer, tensor):
// nibble words are bit-identical; the normals (scales, router) use the same
// Box-Muller in fp64 with the device's log and cos, which may differ from the
// host libm in the last place and, rarely, move a bf16 rounding by one unit.
// The parity tests therefore use host-generated layers; these are for
// measurement.

#include <stdint.h>

#include "qmoe_internal.h"

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t draw(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * kGolden); }

__device__ __forceinline__ double unit(uint64_t r) {
    return (static_cast<double>(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ float normal(uint64_t key, uint64_t i) {
    const double u1 = unit(draw(key, 2 * i)), u2 = unit(draw(key, 2 * i + 1));
    return static_cast<float>(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

__device__ __forceinline__ uint32_t to_bf16(float f) {
    const uint32_t b = __float_as_uint(f);
    uint32_t r = b >> 16;
    const uint32_t rem = b & 0xFFFFu;
    if (rem > 0x8000u || (rem == 0x8000u && (r & 1u))) ++r;
    return r & 0xFFFFu;
}

// (scale, bias) of element i of a scales stream, packed as bf16 (s | b << 16)
__device__ __forceinline__ uint32_t scale_pair(uint64_t key, uint64_t i) {
    const uint32_t s = to_bf16(fabsf(normal(key, i) * 0.02f));
    const uint32_t b = to_bf16(-8.0f * __uint_as_float(s << 16));
    return s | (b << 16);
}

struct SlotKeys {
    uint64_t gq, gs, uq, us, dq, ds;
};

// One 4-byte word of expert e's slot per thread (layout: qmoe_internal.h).
__global__ void k_synth_slot(uint32_t *slot, qk_layout L, int e, SlotKeys kk) {
    const size_t words = L.slot_bytes / 4;
    const size_t d = L.d, I = L.I, g = L.g;
    for (size_t w = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; w < words;
         w += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t off = 4 * w;
        uint32_t v = 0;
        if (off < L.gu_bytes) {
            const size_t n = off / L.gu_row, col = off % L.gu_row;
            const size_t row = e * I + n;
            if (col < d / 2) {
                v = static_cast<uint32_t>(draw(kk.gq, row * (d / 8) + col / 4));
            } else if (col < d) {
                v = static_cast<uint32_t>(draw(kk.uq, row * (d / 8) + (col - d / 2) / 4));
            } else {
                const size_t q = col - d, j = q / 8;
                v = scale_pair((q % 8) < 4 ? kk.gs : kk.us, row * (d / g) + j);
            }
        } else if (off < L.gu_bytes + d * L.d_row) {
            const size_t o2 = off - L.gu_bytes, n = o2 / L.d_row, col = o2 % L.d_row;
            const size_t row = e * d + n;
            if (col < I / 2)
                v = static_cast<uint32_t>(draw(kk.dq, row * (I / 8) + col / 4));
            else if (col < I / 2 + 4 * (I / g))
                v = scale_pair(kk.ds, row * (I / g) + (col - I / 2) / 4);
        }
        slot[w] = v;
    }
}

// bf16(N(0, 0.02)) vector of n elements
__global__ void k_synth_bf16_normal(uint16_t *out, size_t n, uint64_t key) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = static_cast<uint16_t>(to_bf16(normal(key, i) * 0.02f));
}

}  // namespace

extern "C" int qk_synth_slot(const qk_layout *L, uint8_t *slot, int e, const uint64_t keys[6],
                             void *stream) {
    SlotKeys kk{keys[0], keys[1], keys[2], keys[3], keys[4], keys[5]};
    k_synth_slot<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<uint32_t *>(slot),
                                                                     *L, e, kk);
    return cudaGetLastError();
}

extern "C" int qk_synth_bf16_normal(uint16_t *out, size_t n, uint64_t key, void *stream) {
    k_synth_bf16_normal<<<296, 256, 0, static_cast<cudaStream_t>(stream)>>>(out, n, key);
    return cudaGetLastError();
}
