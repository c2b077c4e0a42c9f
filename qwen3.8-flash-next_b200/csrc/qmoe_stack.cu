// qmoe_stack.cu - the residual stream of a MoE-only layer stack:
//   h_{l+1} = h_l + MoE_l(RMSNorm(h_l)),  RMSNorm with unit weight.
// RMSNorm follows kernel_rmsnorm (c/src/kernel.c:10-20): r = 1 / sqrt(ss / n
// + eps) in fp32, y = x * r. The sum of squares is taken in fp64 (each fp32
// square is exact there), so it is closer to the exact value than the
// reference's sequential fp32 sum; the two differ by far less than the
// layer's output tolerance.

#include <stdint.h>

#include "qmoe_internal.h"

namespace {

constexpr int kThreads = 256;

// One CTA per token row. y != NULL: h += y first. xn != NULL: xn = RMSNorm(h).
__global__ void __launch_bounds__(kThreads) k_residual_norm(float *h, const float *y, float *xn,
                                                            int d, float eps) {
    __shared__ double s_part[kThreads / 32];
    const size_t row = static_cast<size_t>(blockIdx.x) * d;
    float4 *hr = reinterpret_cast<float4 *>(h + row);
    const float4 *yr = y ? reinterpret_cast<const float4 *>(y + row) : nullptr;
    double ss = 0.0;
    for (int c = threadIdx.x; c < d / 4; c += kThreads) {
        float4 v = hr[c];
        if (yr) {
            const float4 u = yr[c];
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
            hr[c] = v;
        }
        ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y +
              static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
    }
    if (!xn) return;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) tot += s_part[w];
    const float r = 1.0f / sqrtf(static_cast<float>(tot) / static_cast<float>(d) + eps);
    float4 *xr = reinterpret_cast<float4 *>(xn + row);
    for (int c = threadIdx.x; c < d / 4; c += kThreads) {
        const float4 v = hr[c];
        xr[c] = make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
    }
}

}  // namespace

extern "C" int qk_launch_residual_norm(float *h, const float *y, float *xn, int n, int d, float eps,
                                       void *stream) {
    if (n <= 0) return 0;
    if (d % 4) return cudaErrorInvalidValue;
    k_residual_norm<<<n, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(h, y, xn, d, eps);
    return cudaGetLastError();
}
