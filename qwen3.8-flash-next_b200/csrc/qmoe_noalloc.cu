// qmoe_noalloc.cu - qmoe_forward_token_noalloc: one decode token through the
// single-launch kernel with no allocation at all.
//
// Who this is for: callers that cannot call cudaMalloc, such as code running
// inside another framework's fixed device-memory arena or budget, or on a path
// where an allocation may block, fail or is not allowed. They pass every
// input and output; the intermediates of the call live in g_scratch below, a
// file-scope device array of QMOE_NOALLOC_SCRATCH_BYTES that each GPU loading
// the library holds until the process exits.
//
// Host code never dereferences or passes `g_scratch` itself: on the host that
// name is only a stand-in symbol. Its device address is looked up once per
// device (cudaGetSymbolAddress, with that device current) on the first call
// for that device, and that address is what the kernel receives. Make that
// first call before any stream capture. All calls share the array: each call
// clears the error word and the kernel's barrier counter and exchange area
// first, and calls that overlap on the GPU race on it.

#include <cuda_runtime.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/qmoe.h"
#include "qmoe_internal.h"

// The one scratch array (device memory, zero-initialised at module load).
static __device__ __align__(256) unsigned char g_scratch[QMOE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
unsigned char *g_scratch_dev[kMaxDevices];  // device address of g_scratch, per device
int g_num_sms[kMaxDevices];

void seterr(qmoe_err *err, const char *msg) {
    if (err) snprintf(err->msg, sizeof(err->msg), "%s", msg);
}

size_t up16(size_t v) { return (v + 15) / 16 * 16; }

bool misaligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

// Per-device set-up on the first call: device address of the array, kernel
// attributes, SM count. Runs with `dev` current.
int setup(int dev, qmoe_err *err) {
    pthread_mutex_lock(&g_lock);
    int rc = 0;
    if (!g_scratch_dev[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        int sms = 0;
        if (e == cudaSuccess) e = static_cast<cudaError_t>(qk_prepare_kernels());
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || !p) {
            char m[256];
            snprintf(m, sizeof(m), "qmoe_forward_token_noalloc: set-up on device %d failed: %s", dev,
                     cudaGetErrorString(e));
            seterr(err, m);
            rc = -1;
        } else {
            g_num_sms[dev] = sms;
            g_scratch_dev[dev] = static_cast<unsigned char *>(p);
        }
    }
    pthread_mutex_unlock(&g_lock);
    return rc;
}

}  // namespace

extern "C" int qmoe_forward_token_noalloc(const qmoe_token_args *a, void *stream, qmoe_err *err) {
    if (err) err->msg[0] = 0;
    if (!a || !a->x || !a->out || !a->router || !a->shared_gate || !a->pool || !a->slot_of ||
        !a->shared_slot) {
        seterr(err, "qmoe_forward_token_noalloc: missing device pointer");
        return -1;
    }
    if (a->x_dtype != QMOE_F32 && a->x_dtype != QMOE_BF16) {
        seterr(err, "qmoe_forward_token_noalloc: unknown x dtype");
        return -1;
    }
    // the kernel reads x, the router rows, the shared gate, the slot table and
    // the slots with 16-byte vector loads and bulk copies, which need 16-byte
    // aligned addresses: refuse others here rather than fault on the GPU
    {
        const struct { const void *p; const char *name; } ptrs[] = {
            {a->x, "x"}, {a->out, "out"}, {a->router, "router"}, {a->shared_gate, "shared_gate"},
            {a->pool, "pool"}, {a->slot_of, "slot_of"}, {a->shared_slot, "shared_slot"}};
        for (const auto &q : ptrs)
            if (misaligned(q.p, 16)) {
                char m[160];
                snprintf(m, sizeof(m),
                         "qmoe_forward_token_noalloc: %s (%p) is not 16-byte aligned", q.name, q.p);
                seterr(err, m);
                return -1;
            }
        if (a->logit_bias && misaligned(a->logit_bias, 4)) {
            seterr(err, "qmoe_forward_token_noalloc: logit_bias is not 4-byte aligned");
            return -1;
        }
    }
    qk_layout L;
    if (qk_layout_init(&L, a->hidden, a->num_experts, a->top_k, a->moe_inter, a->group_size)) {
        seterr(err, "qmoe_forward_token_noalloc: unsupported shape");
        return -1;
    }
    // scratch layout: [0,4) error word; from 256 idx [k], weights [k], shared
    // gate [1]; then the kernel's counter and exchange area
    const size_t off_idx = 256;
    const size_t off_wts = off_idx + up16(4 * static_cast<size_t>(L.k));
    const size_t off_sg = off_wts + up16(4 * static_cast<size_t>(L.k));
    const size_t off_sync = (off_sg + 16 + 255) / 256 * 256;
    const size_t sync_bytes = qk_decode_sync_bytes(&L);
    const size_t need = off_sync + sync_bytes;
    if (need > QMOE_NOALLOC_SCRATCH_BYTES) {
        char m[256];
        snprintf(m, sizeof(m),
                 "qmoe_forward_token_noalloc: this shape needs %zu bytes of scratch; the "
                 "library's array holds %u (QMOE_NOALLOC_SCRATCH_BYTES)",
                 need, QMOE_NOALLOC_SCRATCH_BYTES);
        seterr(err, m);
        return -1;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        seterr(err, "qmoe_forward_token_noalloc: no usable current device");
        return -1;
    }
    if (setup(dev, err)) return -1;
    unsigned char *base = g_scratch_dev[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    qk_fwd f;
    memset(&f, 0, sizeof(f));
    f.L = L;
    f.T = 1;
    f.x = a->x;
    f.x_bf16 = a->x_dtype == QMOE_BF16;
    f.router = a->router;
    f.shared_gate = a->shared_gate;
    f.logit_bias = a->logit_bias;
    f.pool = a->pool;
    f.slot_of = a->slot_of;
    f.shared_slot = a->shared_slot;
    f.idx = reinterpret_cast<int32_t *>(base + off_idx);
    f.wts = reinterpret_cast<float *>(base + off_wts);
    f.sgate = reinterpret_cast<float *>(base + off_sg);
    f.out = a->out;
    f.err = reinterpret_cast<int *>(base);
    f.num_sms = g_num_sms[dev];

    // what must start at zero: the error word, and the kernel's barrier
    // counter and exchange area (an earlier call may have left them set)
    e = cudaMemsetAsync(base, 0, 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(base + off_sync, 0, sync_bytes, st);
    if (e != cudaSuccess) {
        seterr(err, cudaGetErrorString(e));
        return -1;
    }
    const int rc = qk_launch_decode_fused(&f, base + off_sync, st, 0);
    if (rc == QK_FUSED_UNFIT) {
        seterr(err, "qmoe_forward_token_noalloc: shape not covered by the single-launch kernel");
        return -1;
    }
    if (rc != 0) {
        seterr(err, cudaGetErrorString(static_cast<cudaError_t>(rc)));
        return -1;
    }
    int code = 0;
    e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaMemcpy(&code, base, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        seterr(err, cudaGetErrorString(e));
        return -1;
    }
    if (code) {
        char m[128];
        snprintf(m, sizeof(m), "qmoe_forward_token_noalloc: device reported error 0x%x", code);
        seterr(err, m);
        return -1;
    }
    return 0;
}
