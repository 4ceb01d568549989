// zwg_attention_dev_noalloc: the split-K decode attention with its scratch in a
// library-owned device array instead of caller-provided workspace.
//
// Who needs this: hosts that cannot call cudaMalloc for the workspace. One case is an
// embedding that reaches the engine only through this C ABI, from a runtime with no
// binding for CUDA's allocator (a Zig or Rust host linking the library as the reference's
// host code links libzwhisper.a). Another is a streaming decode thread with a per-token
// latency budget: cudaMalloc and cudaFree may synchronize the whole device and stall for
// milliseconds, so such a thread must not allocate between tokens.
//
// The scratch is a file-scope __device__ array of a fixed size (kNoAllocScratchBytes,
// 4 MiB). Every GPU that loads this library holds that much memory until the process
// exits. Host code cannot use the array's name as a device address (on the host it names a
// stand-in object), so the device address is looked up with cudaGetSymbolAddress once per
// device, with that device current, on the first call made on that device. Make that first
// call on each device before any stream capture begins. The address is remembered together
// with the CUDA context it belongs to: after a device reset (cudaDeviceReset, or a reset of
// the primary context by other code in the process) the module is loaded again and the
// array may move, so the next call sees a new context and looks the address up again.
//
// All calls on a device share the one array, and the array keeps whatever the previous
// call left in it. Nothing in it has to start at zero: each call writes every partial slot
// it reads before the combine kernel reads it, in stream order. Two calls that overlap on
// the GPU (different streams, or different host threads without a synchronization between
// them) use the same array and race; issue calls for one device on one stream, or order
// them.
#include "../../include/zwgpu.h"
#include "api_internal.h"
#include "common.cuh"
#include "kernels.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocScratchFloats = kNoAllocScratchBytes / sizeof(float);

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (no link against libcuda).
CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (CtxGetCurrentFn)p;
    });
    return fn;
}

struct ScratchSlot {
    CUcontext ctx = nullptr;
    float* ptr = nullptr;
};

std::mutex g_mu;
ScratchSlot g_slots[64];

// Device address of the array in the current device's current context; looked up on the
// first call in that context.
int scratch_for_current_device(int dev, float** out) {
    if (dev < 0 || dev >= 64) return zwg::set_last_error("device index out of range");
    CtxGetCurrentFn get = ctx_get_current_fn();
    if (!get) return zwg::set_last_error("cuCtxGetCurrent is not available from the driver");
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return zwg::set_last_error("cuCtxGetCurrent failed");
    if (!ctx) {
        // nothing has used the device on this thread yet: cudaSetDevice makes its primary
        // context current (it allocates no memory)
        cudaError_t e = cudaSetDevice(dev);
        if (e != cudaSuccess) return zwg::set_last_error_cuda("cudaSetDevice", e);
        if (get(&ctx) != CUDA_SUCCESS || !ctx) return zwg::set_last_error("no current CUDA context");
    }
    std::lock_guard<std::mutex> lk(g_mu);
    ScratchSlot& slot = g_slots[dev];
    if (slot.ctx != ctx || !slot.ptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return zwg::set_last_error_cuda("cudaGetSymbolAddress(scratch)", e);
        slot.ctx = ctx;
        slot.ptr = static_cast<float*>(p);
    }
    *out = slot.ptr;
    return ZWG_OK;
}

}  // namespace

extern "C" int zwg_attention_dev_noalloc(const zwg_attn_shape* sh, const zwg_batch* b, const float* q,
                                         const float* k, const float* v, float* out, void* stream) {
    // the checks every attention entry point makes (the reference's asserts), then this
    // entry point's own limits
    int rc = zwg::capi::check_shape(sh);
    if (rc) return rc;
    const size_t rows = sh->n_q * (sh->n_head / sh->n_head_kv);
    if (!zwg::decode_supported(sh->d, rows, sh->kt_stride))
        return zwg::set_last_error("zwg_attention_dev_noalloc takes decode shapes only: d in {32, 64, 128}, "
                                   "n_q * n_head / n_head_kv <= 8, kt_stride a multiple of 4");
    const size_t nb = b ? b->n_batch : 1;
    if (nb == 0 || sh->n_q == 0) return ZWG_OK;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) return zwg::set_last_error("q, k, v must be 16-byte aligned");
    if ((sh->kv_stride | sh->q_stride) % 4) return zwg::set_last_error("strides must be multiples of 4");
    if (b && (b->q_batch_stride % 4 || b->k_batch_stride % 4 || b->v_batch_stride % 4))
        return zwg::set_last_error("batch strides must be multiples of 4");

    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return zwg::set_last_error_cuda("cudaGetDevice", e);
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || sms <= 0) return zwg::set_last_error_cuda("cudaDeviceGetAttribute(SM count)", e);
    int n_splits = 1, chunk = 0;
    zwg::decode_plan(nb, sh->n_head_kv, sh->n_kv, sh->kt_stride != 0, sms, &n_splits, &chunk);
    const size_t need = zwg::decode_workspace_floats(nb, sh->n_head_kv, rows, n_splits, sh->d);
    if (need > kNoAllocScratchFloats)
        return zwg::set_last_error("zwg_attention_dev_noalloc: this call needs more scratch than the built-in "
                                   "4 MiB array holds; split the batch or use zwg_attention_dev");
    float* scratch = nullptr;
    rc = scratch_for_current_device(dev, &scratch);
    if (rc) return rc;

    zwg::DecodeParams p{};
    p.q = q; p.k = k; p.v = v; p.out = out; p.ws = scratch;
    p.n_q = sh->n_q; p.n_kv = sh->n_kv; p.n_head = sh->n_head; p.n_head_kv = sh->n_head_kv; p.d = sh->d;
    p.q_stride = sh->q_stride; p.kv_stride = sh->kv_stride; p.out_stride = sh->out_stride;
    p.kt_stride = sh->kt_stride; p.causal = sh->causal ? 1 : 0;
    p.n_splits = n_splits; p.chunk = chunk;
    if (b) { p.q_bs = b->q_batch_stride; p.k_bs = b->k_batch_stride; p.v_bs = b->v_batch_stride; p.out_bs = b->out_batch_stride; }
    if (zwg::decode_f32_launch(p, nb, (cudaStream_t)stream)) {
        e = cudaGetLastError();
        if (e == cudaSuccess) return zwg::set_last_error("zwg_attention_dev_noalloc: no decode kernel for this shape");
        return zwg::set_last_error_cuda("decode kernel launch", e);
    }
    return ZWG_OK;
}
