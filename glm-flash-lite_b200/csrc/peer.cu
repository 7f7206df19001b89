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

// ---- expert-parallel dispatch / return as an all-to-all over the ranks ---------------------------------------------
// ep_pack_kernel (one CTA): for each destination rank d (the owner of experts [d n, (d + 1) n)), the tokens with at least
// one pick there, ascending: their order in the send buffer is (d, token). Writes counts[d], the send rows' token
// index, their routing for d (local ids of d's shard, other picks -1 with weight 0, then the fp32 weight bits) and
// pos[d][t] = send row of (d, t) or -1. total[0] = the number of send rows.
constexpr int EP_T = 1024;

__device__ int ep_block_scan(int v, int* warp_sums, int* total)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
    {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[wid] = x;
    __syncthreads();
    if (wid == 0)
    {
        int s = lane < (int) (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;
    }
    __syncthreads();
    const int before = (wid ? warp_sums[wid - 1] : 0) + x - v;
    *total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before;
}

__global__ void __launch_bounds__(EP_T) ep_pack_kernel(const int* sel, const float* w, int B, int k, int n, int world,
                                                       int* counts, int* total, int* send_tok, int* send_route, int* pos)
{
    __shared__ int warp_sums[32];
    int off = 0;
    for (int d = 0; d < world; ++d)
    {
        const int lo = d * n, hi = lo + n;
        for (int t0 = 0; t0 < B; t0 += EP_T)
        {
            const int t = t0 + threadIdx.x;
            int has = 0;
            if (t < B)
                for (int j = 0; j < k; ++j)
                {
                    const int e = sel[(size_t) t * k + j];
                    has |= (e >= lo && e < hi);
                }
            int cnt;
            const int before = ep_block_scan(has, warp_sums, &cnt);
            if (t < B)
            {
                const int r = off + before;
                pos[(size_t) d * B + t] = has ? r : -1;
                if (has)
                {
                    send_tok[r] = t;
                    for (int j = 0; j < k; ++j)
                    {
                        const int e = sel[(size_t) t * k + j];
                        const bool mine = e >= lo && e < hi;
                        send_route[(size_t) r * 2 * k + j] = mine ? e - lo : -1;
                        send_route[(size_t) r * 2 * k + k + j] = mine ? __float_as_int(w[(size_t) t * k + j]) : 0;
                    }
                }
            }
            off += cnt;
        }
        if (threadIdx.x == 0) counts[d] = off;          // end offset of d for now
        __syncthreads();
    }
    // counts[d] so far holds the running end offset of d: turn it into the per-destination count
    if (threadIdx.x == 0)
    {
        int prev = 0;
        for (int d = 0; d < world; ++d) { const int end = counts[d]; counts[d] = end - prev; prev = end; }
        *total = off;
    }
}

// send_x[r] = x[send_tok[r]] for r < *total (rows of `row_bytes` bytes, 16-byte multiples)
__global__ void __launch_bounds__(256) ep_gather_kernel(const uint4* x, int row16, const int* send_tok, const int* total,
                                                        uint4* send_x, int max_rows)
{
    const int n = min(*total, max_rows);
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < (long long) n * row16;
         i += (long long) gridDim.x * blockDim.x)
    {
        const int r = (int) (i / row16), c = (int) (i % row16);
        send_x[i] = x[(size_t) send_tok[r] * row16 + c];
    }
}

// out[t] += ret[pos[0][t]] + ... + ret[pos[world-1][t]] (rows present only), added in rank order
__global__ void __launch_bounds__(256) ep_unpack_add_kernel(const float4* ret, const int* pos, int B, int world, int H4,
                                                            float4* out)
{
    for (long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x; i < (long long) B * H4;
         i += (long long) gridDim.x * blockDim.x)
    {
        const int t = (int) (i / H4), c = (int) (i % H4);
        float4 v = out[i];
        for (int d = 0; d < world; ++d)
        {
            const int r = pos[(size_t) d * B + t];
            if (r < 0) continue;
            const float4 u = ret[(size_t) r * H4 + c];
            v.x = __fadd_rn(v.x, u.x); v.y = __fadd_rn(v.y, u.y); v.z = __fadd_rn(v.z, u.z); v.w = __fadd_rn(v.w, u.w);
        }
        out[i] = v;
    }
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

extern "C" int glmx_ep_pack(const int* sel, const float* w, int B, int topk, int experts_per_rank, int world, const void* x,
                            int row_bytes, int* counts, int* total, int* send_tok, int* send_route, int* pos, void* send_x,
                            void* stream)
{
    if (B < 0 || topk < 1 || topk > 64 || experts_per_rank < 1 || world < 1 || world > 64 || row_bytes <= 0 || row_bytes % 16 ||
        !counts || !total || (B > 0 && (!sel || !w || !x || !send_tok || !send_route || !pos || !send_x)))
        return fail(GLMX_E_ARG, "glmx_ep_pack: B >= 0, 1 <= topk <= 64, world in [1, 64], row_bytes a positive multiple of 16, "
                                "non-null arrays");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send_x)) & 15u)
        return fail(GLMX_E_ARG, "glmx_ep_pack: x and send_x must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ep_pack_kernel<<<1, EP_T, 0, st>>>(sel, w, B, topk, experts_per_rank, world, counts, total, send_tok, send_route, pos);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && B > 0)
    {
        const int row16 = row_bytes / 16;
        const long long work = (long long) B * world * row16;
        const unsigned grid = (unsigned) ((work + 255) / 256 < 148 * 8 ? (work + 255) / 256 : 148 * 8);
        ep_gather_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(x), row16, send_tok, total, static_cast<uint4*>(send_x),
                                               B * world);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ep_pack: launch: ") + cudaGetErrorString(e));
    return GLMX_OK;
}

extern "C" int glmx_ep_unpack_add(const float* ret, const int* pos, int B, int world, int hidden, float* out, void* stream)
{
    if (B < 0 || world < 1 || world > 64 || hidden <= 0 || hidden % 4 || (B > 0 && (!ret || !pos || !out)))
        return fail(GLMX_E_ARG, "glmx_ep_unpack_add: B >= 0, world in [1, 64], hidden a multiple of 4, non-null arrays");
    if (B == 0) return GLMX_OK;
    const int H4 = hidden / 4;
    const long long work = (long long) B * H4;
    const unsigned grid = (unsigned) ((work + 255) / 256 < 148 * 8 ? (work + 255) / 256 : 148 * 8);
    ep_unpack_add_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<const float4*>(ret), pos, B, world,
                                                                                H4, reinterpret_cast<float4*>(out));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("glmx_ep_unpack_add: launch: ") + cudaGetErrorString(e));
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
