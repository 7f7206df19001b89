// glmx_moe_forward_noalloc: the routed-expert forward with its scratch in a fixed device array of this library, for
// callers that cannot hand in a workspace and must not allocate device memory per call:
//   * a host in another language (a cgo / JNI / N-API binding) that has no device allocator of its own to make one;
//   * a serving loop whose HBM is held in full by its own allocator (expert bank + KV cache) so that a cudaMalloc
//     here would fail or fragment it, and where cudaMalloc / cudaFree would also synchronise the device mid-step.
// The work and the results are those of glmx_moe_forward: this file only supplies the workspace.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "glmx.h"
#include "glmx_internal.h"

namespace {

// The scratch. 48 MiB holds the workspace of up to 8 tokens x top-8 (+ a shared expert) at H = 6144, I = 1536 in
// either mode on a 148-SM B200; larger calls are rejected with GLMX_E_WORKSPACE. It is created with the module (no
// allocation call at run time) and, being a __device__ array, starts zeroed; nothing in it has to start at zero per
// call anyway: the only words a call needs cleared (the split-K arrival counters and the device error word) are
// cleared by the call's own first kernel (the split) on the call's stream before any later kernel reads them.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GLMX_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch on device `dev`, resolved once per device (this is the set-up the first call on each
// device performs; the symbol lookup may load this module on that device, so that first call belongs outside stream
// capture). The caller has checked that `dev` is the current device.
int scratch_for_device(int dev, void** ptr)
{
    if (dev < 0 || dev >= kMaxDevices)
    {
        glmx::set_error("glmx_moe_forward_noalloc: device index out of range");
        return GLMX_E_ARG;
    }
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev])
    {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
        {
            glmx::set_error(std::string("glmx_moe_forward_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            return GLMX_E_CUDA;
        }
        g_scratch_ptr[dev] = p;
    }
    *ptr = g_scratch_ptr[dev];
    return GLMX_OK;
}

// The layer's device, which must be the current device (checked before anything touches the scratch, so a call on
// the wrong device neither loads the module there nor resolves its array).
int layer_device(const glmx_layer* layer, const char* who, int* dev)
{
    const int ldev = glmx_layer_device(layer);
    int cur = -1;
    const cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess)
    {
        glmx::set_error(std::string(who) + ": cudaGetDevice: " + cudaGetErrorString(e));
        return GLMX_E_CUDA;
    }
    if (ldev < 0 || cur != ldev)
    {
        glmx::set_error(std::string(who) + ": current device differs from the layer's device");
        return GLMX_E_ARG;
    }
    *dev = ldev;
    return GLMX_OK;
}

}  // namespace

extern "C" int glmx_moe_forward_noalloc(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                                        int sel_dtype, const void* w, int w_dtype, int topk, int mode, void* out,
                                        int out_dtype, int accumulate, void* stream)
{
    if (!layer)
    {
        glmx::set_error("glmx_moe_forward_noalloc: null layer");
        return GLMX_E_ARG;
    }
    if (ntok < 0 || topk < 0)
    {
        glmx::set_error("glmx_moe_forward_noalloc: ntok >= 0 and topk >= 0 required");
        return GLMX_E_ARG;
    }
    const size_t need = glmx_workspace_bytes(layer, ntok, topk);
    if (need > (size_t) GLMX_NOALLOC_SCRATCH_BYTES)
    {
        glmx::set_error("glmx_moe_forward_noalloc: this call needs " + std::to_string(need) +
                        " bytes of scratch but the built-in scratch holds " + std::to_string((size_t) GLMX_NOALLOC_SCRATCH_BYTES) +
                        " (ntok=" + std::to_string(ntok) + ", topk=" + std::to_string(topk) +
                        "); split the batch or call glmx_moe_forward with a caller-owned workspace");
        return GLMX_E_WORKSPACE;
    }
    int dev = -1;
    int rc = layer_device(layer, "glmx_moe_forward_noalloc", &dev);
    if (rc != GLMX_OK) return rc;
    void* scratch = nullptr;
    rc = scratch_for_device(dev, &scratch);
    if (rc != GLMX_OK) return rc;
    return glmx_moe_forward(layer, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, out, out_dtype, accumulate,
                            scratch, (size_t) GLMX_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int glmx_check_noalloc(const glmx_layer* layer, int ntok, int topk, void* stream, int* flags)
{
    if (!layer || ntok < 0 || topk < 0)
    {
        glmx::set_error("glmx_check_noalloc: bad argument");
        return GLMX_E_ARG;
    }
    int dev = -1;
    int rc = layer_device(layer, "glmx_check_noalloc", &dev);
    if (rc != GLMX_OK) return rc;
    void* scratch = nullptr;
    rc = scratch_for_device(dev, &scratch);
    if (rc != GLMX_OK) return rc;
    return glmx_check(layer, ntok, topk, scratch, stream, flags);
}
