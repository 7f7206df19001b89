// Expert-parallel return over peer memory (NVLink / NVSwitch), the combine side's counterpart.
//
// Every rank runs the layer over all ranks' gathered rows with its shard of the experts; its combine kernels store
// token t's fp32 partial row directly into the owner rank's receive buffer (recv[seq & 1][source rank][t % rpr]) and
// their last CTA publishes flag [seq & 1][source rank] = seq on every rank (combine kernels, PeerOut). Here the owner
// waits for all world flags of this call (bounded: after WAIT_TIMEOUT_NS it records ERR_TIMEOUT_PEER and writes nothing)
// and sums the world partial rows in rank order. This replaces a reduce-scatter of the partials: the transfer happens
// inside the combine, row by row, as the partials are produced. Two buffers alternate by call parity; a rank can only
// reuse one after the next call's collective dispatch, which no rank passes before every owner finished reading it.
//
// The buffers are shared between processes with CUDA IPC handles: glmx_ipc_alloc makes each one its own allocation, so
// the mapping glmx_ipc_open returns in another process starts at the buffer itself.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "glmx.h"
#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

__global__ void __launch_bounds__(256) peer_reduce_kernel(const float* recv, const int* flags, int world, int rpr, int H,
                                                          int seq, void* out, int out_dtype, int* err)
{
    __shared__ int s_ok;
    if (threadIdx.x == 0)
    {
        int ok = 1;
        const uint64_t t0 = globaltimer();
        for (int s = 0; s < world && ok; ++s)
            while (ld_acquire_sys(flags + (seq & 1) * world + s) != seq)
                if (globaltimer() - t0 > (uint64_t) WAIT_TIMEOUT_NS)
                {
                    atomicOr(err, ERR_TIMEOUT_PEER);
                    ok = 0;
                    break;
                }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    const size_t n4 = (size_t) rpr * H / 4;
    const float4* base = reinterpret_cast<const float4*>(recv + (size_t) (seq & 1) * world * rpr * H);
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t) gridDim.x * blockDim.x)
    {
        float4 v = __ldcg(base + i);
        for (int s = 1; s < world; ++s)
        {
            const float4 u = __ldcg(base + (size_t) s * n4 + i);
            v.x = __fadd_rn(v.x, u.x); v.y = __fadd_rn(v.y, u.y); v.z = __fadd_rn(v.z, u.z); v.w = __fadd_rn(v.w, u.w);
        }
        if (out_dtype == GLMX_F32) reinterpret_cast<float4*>(out)[i] = v;
        else
        {
            __half2* o = reinterpret_cast<__half2*>(out) + 2 * i;
            o[0] = __floats2half2_rn(v.x, v.y);
            o[1] = __floats2half2_rn(v.z, v.w);
        }
    }
}

// The shard's picks of every gathered row: route [rows][2k] int32 = global ids (k) then the fp32 weight bits (k), as
// the dispatch gathers them. loc [rows][k + extra]: ids first .. first + n - 1 become local 0 .. n - 1, others -1 (weight
// 0); extra = 1 adds local id n (the shared expert, weight 1) on rows [own0, own1) and -1 / 0 elsewhere.
__global__ void __launch_bounds__(256) ep_split_kernel(const int* route, int rows, int k, int first, int n, int extra,
                                                       int own0, int own1, int* loc, float* wl)
{
    const int kk = k + extra;
    const long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long) rows * kk) return;
    const int r = (int) (i / kk), j = (int) (i % kk);
    int id = -1;
    float wt = 0.0f;
    if (j < k)
    {
        const int g = route[(size_t) r * 2 * k + j] - first;
        if (g >= 0 && g < n) { id = g; wt = __int_as_float(route[(size_t) r * 2 * k + k + j]); }
    }
    else if (r >= own0 && r < own1) { id = n; wt = 1.0f; }
    loc[i] = id;
    wl[i] = wt;
}

int fail(int code, const std::string& msg)
{
    set_error(msg);
    return code;
}

}  // namespace

}  // namespace glmx

using namespace glmx;

extern "C" int glmx_peer_reduce(const float* recv, const int* flags, int world, int rows_per_rank, int hidden, int seq, void* out,
                                int out_dtype, int* err, void* stream)
{
    if (!recv || !flags || !out || !err) return fail(GLMX_E_ARG, "glmx_peer_reduce: null argument");
    if (world < 1 || world > 64 || rows_per_rank < 0 || hidden <= 0 || hidden % 4 || seq <= 0)
        return fail(GLMX_E_ARG, "glmx_peer_reduce: world in [1, 64], rows_per_rank >= 0, hidden a multiple of 4, seq > 0");
    if (out_dtype != GLMX_F32 && out_dtype != GLMX_F16) return fail(GLMX_E_ARG, "glmx_peer_reduce: out dtype must be fp32 or fp16");
    if (rows_per_rank == 0) return GLMX_OK;
    const size_t n4 = (size_t) rows_per_rank * hidden / 4;
    const unsigned grid = (unsigned) ((n4 + 255) / 256 < 148 * 4 ? (n4 + 255) / 256 : 148 * 4);
    peer_reduce_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(recv, flags, world, rows_per_rank, hidden, seq, out,
                                                                              out_dtype, err);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_peer_reduce: launch: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ep_split(const int* route, int rows, int topk, int first, int n, int shared, int own_begin, int own_end,
                             int* loc, float* w, void* stream)
{
    if (rows < 0 || topk < 1 || topk > 64 || n < 1 || (rows > 0 && (!route || !loc || !w)))
        return fail(GLMX_E_ARG, "glmx_ep_split: rows >= 0, 1 <= topk <= 64, n >= 1 and non-null arrays required");
    if (rows == 0) return GLMX_OK;
    const int kk = topk + (shared ? 1 : 0);
    const long long total = (long long) rows * kk;
    ep_split_kernel<<<(unsigned) ((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        route, rows, topk, first, n, shared ? 1 : 0, own_begin, own_end, loc, w);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ep_split: launch: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ipc_alloc(size_t bytes, void** dev_ptr)
{
    if (!dev_ptr || bytes == 0) return fail(GLMX_E_ARG, "glmx_ipc_alloc: null pointer or zero size");
    cudaError_t e = cudaMalloc(dev_ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*dev_ptr, 0, bytes);
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ipc_alloc: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ipc_free(void* dev_ptr)
{
    if (!dev_ptr) return GLMX_OK;
    const cudaError_t e = cudaFree(dev_ptr);
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ipc_free: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ipc_handle(const void* dev_ptr, void* handle)
{
    if (!dev_ptr || !handle) return fail(GLMX_E_ARG, "glmx_ipc_handle: null argument");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ipc_handle: ") + cudaGetErrorString(e));
    static_assert(sizeof(h) == GLMX_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return GLMX_OK;
}

extern "C" int glmx_ipc_open(const void* handle, void** dev_ptr)
{
    if (!handle || !dev_ptr) return fail(GLMX_E_ARG, "glmx_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ipc_open: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ipc_close(void* dev_ptr)
{
    if (!dev_ptr) return fail(GLMX_E_ARG, "glmx_ipc_close: null argument");
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ipc_close: ") + cudaGetErrorString(e));
    return GLMX_OK;
}
