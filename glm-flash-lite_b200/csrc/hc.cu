// Hyper-connection site kernels of GLM-5.3 (hc_mult 4) around the MoE sublayer, as the reference fuses them for
// decode (glm53/k_hcfuse.py):
//   hc_apply_partials_kernel   hc_apply of the pending site (x_g <- post_g y + sum_h comb[h][g] x_h, in place) and
//                              hc_mix_partials of the next site (k_hcfuse.py:41-126)
//   hc_finalize_kernel         hc_mix_finalize (pre / post / Sinkhorn comb) + the site's RMSNorm of the collapsed row
//                              (k_hcfuse.py:129-294)
// The results are bit-identical to the reference's kernels: this file is compiled with --use_fast_math as the reference
// compiles them (k_hcfuse.py:363), and every value is formed by the same expressions, in the same order, over the same
// thread mapping (the warp reduction trees fix the summation order).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int NS = 4;           // streams
constexpr int NMIX = 24;        // mix rows of fn: 4 pre + 4 post + 16 comb (hc_mix_warp)
constexpr int NACC = NMIX + 1;  // + the sum of squares

__device__ __forceinline__ float sigm(float v) { return 1.0f / (1.0f + __expf(-v)); }

__device__ __forceinline__ float4 load_y4(const void* y, int y_half, size_t i4)
{
    if (y_half)
    {
        const __half2* p = reinterpret_cast<const __half2*>(y) + 2 * i4;
        const float2 a = __half22float2(p[0]), b = __half22float2(p[1]);
        return make_float4(a.x, a.y, b.x, b.y);
    }
    return reinterpret_cast<const float4*>(y)[i4];
}

}  // namespace

namespace {

// grid (D / 128, R), 128 threads: warp g = stream, lane = column quad jb * 32 + lane of that stream
__global__ void __launch_bounds__(128) hc_apply_partials_kernel(float* x, const void* y, int y_half, const float* post,
                                                                const float* comb, const __half* fn, float* part, int D,
                                                                int apply)
{
    const int r = blockIdx.y, jb = blockIdx.x;
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D4 = D / 4, q = jb * 32 + lane;
    float4* x4 = reinterpret_cast<float4*>(x + (size_t) r * NS * D);
    float4 s;
    if (apply)
    {
        const float pg = post[(size_t) r * NS + g];
        float cg[NS];
#pragma unroll
        for (int h = 0; h < NS; ++h) cg[h] = comb[((size_t) r * NS + h) * NS + g];
        float4 xv[NS];
#pragma unroll
        for (int h = 0; h < NS; ++h) xv[h] = x4[(size_t) h * D4 + q];
        const float4 yv = load_y4(y, y_half, (size_t) r * D4 + q);
        float4 o = make_float4(pg * yv.x, pg * yv.y, pg * yv.z, pg * yv.w);
#pragma unroll
        for (int h = 0; h < NS; ++h)
        {
            o.x = fmaf(cg[h], xv[h].x, o.x);
            o.y = fmaf(cg[h], xv[h].y, o.y);
            o.z = fmaf(cg[h], xv[h].z, o.z);
            o.w = fmaf(cg[h], xv[h].w, o.w);
        }
        __syncthreads();                      // all four streams of these quads are read before any is rewritten
        x4[(size_t) g * D4 + q] = o;
        s = o;
    }
    else
        s = x4[(size_t) g * D4 + q];
    if (!part) return;
    const size_t nb = D / 128;
    hc_mix_warp(s, fn + (size_t) g * D + 4 * (size_t) q, (size_t) NS * D,
                part + (((size_t) r * NS + g) * nb + jb) * NACC, lane);
}

// grid (2, R): block x = 0 collapses and normalises row r, block x = 1 forms its post and Sinkhorn comb on warp 0 (so
// the norm's block reduction never waits on the Sinkhorn chain). blockDim = min(1024, D/4 rounded up to 32) threads.
template <typename W_T>
__global__ void __launch_bounds__(1024) hc_finalize_kernel(const float* x, const float* part, const float* base,
                                                           const float* scale, float* post, float* comb, const W_T* nw,
                                                           __half* out, int D, float rms_eps, float hc_eps, int iters,
                                                           float n_eps, float cbias, float cscale)
{
    const bool sink = blockIdx.x == 1;
    const int r = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row_len = NS * D, chunks = NS * D / 256;
    if (sink && warp >= 8) return;
    __shared__ float mix[NACC];
    __shared__ float pre[NS];
    __shared__ float wsum[8][NACC];
    if (warp < 8 && lane < NACC)
    {
        // chunk c = (0 + half 2c) + half 2c+1; warp w adds its chunks w, w + 8, ... in order
        const float* p = part + (size_t) r * 2 * chunks * NACC + lane;
        float v = 0.0f;
        for (int c = warp; c < chunks; c += 8)
        {
            float cv = 0.0f;
            cv += p[(size_t) (2 * c) * NACC];
            cv += p[(size_t) (2 * c + 1) * NACC];
            v += cv;
        }
        wsum[warp][lane] = v;
    }
    if (sink) asm volatile("bar.sync 1, 256;" ::: "memory"); else __syncthreads();
    if (tid < NACC)
    {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += wsum[w][tid];
        mix[tid] = v;
    }
    if (sink) asm volatile("bar.sync 1, 256;" ::: "memory"); else __syncthreads();
    const float rmr = rsqrtf(mix[NMIX] / (float) row_len + rms_eps);

    if (sink)
    {
        if (warp != 0) return;
        if (tid < NS) post[(size_t) r * NS + tid] = 2.0f * sigm(fmaf(mix[NS + tid] * rmr, scale[1], base[NS + tid]));
        if (tid < NS * NS)
        {
            // lane t = h * 4 + g: softmax over g within row h, then column (over h) and row normalisation rounds
            const unsigned m16 = 0xffffu;
            float v = fmaf(mix[2 * NS + tid] * rmr, scale[2], base[2 * NS + tid]);
            float m = v;
            for (int o = 1; o < NS; o <<= 1) m = fmaxf(m, __shfl_xor_sync(m16, m, o));
            v = __expf(v - m);
            float sr = v;
            for (int o = 1; o < NS; o <<= 1) sr += __shfl_xor_sync(m16, sr, o);
            v = __fdividef(v, sr) + hc_eps;
            float sc = v;
            for (int o = NS; o < NS * NS; o <<= 1) sc += __shfl_xor_sync(m16, sc, o);
            v = __fdividef(v, sc + hc_eps);
            for (int it = 1; it < iters; ++it)
            {
                sr = v;
                for (int o = 1; o < NS; o <<= 1) sr += __shfl_xor_sync(m16, sr, o);
                v = __fdividef(v, sr + hc_eps);
                sc = v;
                for (int o = NS; o < NS * NS; o <<= 1) sc += __shfl_xor_sync(m16, sc, o);
                v = __fdividef(v, sc + hc_eps);
            }
            comb[(size_t) r * NS * NS + tid] = v;
        }
        return;
    }

    if (tid < NS) pre[tid] = sigm(fmaf(mix[tid] * rmr, scale[0], base[tid])) + hc_eps;
    __syncthreads();
    float pr[NS];
#pragma unroll
    for (int h = 0; h < NS; ++h) pr[h] = pre[h];
    const int quads = D / 4;
    const float4* s4 = reinterpret_cast<const float4*>(x + (size_t) r * row_len);
    // collapsed quads of this thread (one per thread when D <= 4096), kept for the normalisation pass
    constexpr int MAXQ = 4;
    float4 cq[MAXQ];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXQ; ++i)
    {
        const int q = tid + i * blockDim.x;
        cq[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (q < quads)
        {
            float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int h = 0; h < NS; ++h)
            {
                const float4 s = s4[(size_t) h * quads + q];
                o.x = fmaf(pr[h], s.x, o.x);
                o.y = fmaf(pr[h], s.y, o.y);
                o.z = fmaf(pr[h], s.z, o.z);
                o.w = fmaf(pr[h], s.w, o.w);
            }
            const __half2 a = __floats2half2_rn(o.x, o.y), b = __floats2half2_rn(o.z, o.w);
            const float lim = 65504.0f;
            cq[i].x = fmaxf(-lim, fminf(__half2float(__low2half(a)), lim));
            cq[i].y = fmaxf(-lim, fminf(__half2float(__high2half(a)), lim));
            cq[i].z = fmaxf(-lim, fminf(__half2float(__low2half(b)), lim));
            cq[i].w = fmaxf(-lim, fminf(__half2float(__high2half(b)), lim));
            sum = fmaf(cq[i].x, cq[i].x, sum);
            sum = fmaf(cq[i].y, cq[i].y, sum);
            sum = fmaf(cq[i].z, cq[i].z, sum);
            sum = fmaf(cq[i].w, cq[i].w, sum);
        }
    }
    // block reduction: xor tree in each warp, warp totals gathered and reduced again by every warp
    __shared__ float sums[32];
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const int nw_ = blockDim.x / 32;
    if (nw_ > 1)
    {
        if (lane == 0) sums[warp] = sum;
        __syncthreads();
        sum = lane < nw_ ? sums[lane] : 0.0f;
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    }
    const float rmf = rsqrtf(sum / (float) D + n_eps) * cscale;
#pragma unroll
    for (int i = 0; i < MAXQ; ++i)
    {
        const int q = tid + i * blockDim.x;
        if (q >= quads) continue;
        float4 w4;
        if constexpr (std::is_same_v<W_T, __nv_bfloat16>)
        {
            const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(nw + 4 * (size_t) q);
            const __nv_bfloat162 w01 = wp[0], w23 = wp[1];
            w4 = make_float4(__bfloat162float(__low2bfloat16(w01)), __bfloat162float(__high2bfloat16(w01)),
                             __bfloat162float(__low2bfloat16(w23)), __bfloat162float(__high2bfloat16(w23)));
        }
        else
        {
            const __half2* wp = reinterpret_cast<const __half2*>(nw + 4 * (size_t) q);
            const __half2 w01 = wp[0], w23 = wp[1];
            w4 = make_float4(__half2float(__low2half(w01)), __half2float(__high2half(w01)), __half2float(__low2half(w23)),
                             __half2float(__high2half(w23)));
        }
        if (cbias != 0.0f) { w4.x += cbias; w4.y += cbias; w4.z += cbias; w4.w += cbias; }
        const float4 c = cq[i];
        __half2* o2 = reinterpret_cast<__half2*>(out + (size_t) r * D + 4 * (size_t) q);
        o2[0] = __halves2half2(__float2half_rn(c.x * w4.x * rmf), __float2half_rn(c.y * w4.y * rmf));
        o2[1] = __halves2half2(__float2half_rn(c.z * w4.z * rmf), __float2half_rn(c.w * w4.w * rmf));
    }
}

}  // namespace

cudaError_t launch_hc_apply_partials(float* x, const void* y, int y_half, const float* post, const float* comb,
                                     const __half* fn, float* part, int R, int D, int apply, cudaStream_t st)
{
    if (R <= 0) return cudaSuccess;
    hc_apply_partials_kernel<<<dim3(D / 128, R), 128, 0, st>>>(x, y, y_half, post, comb, fn, part, D, apply);
    return cudaGetLastError();
}

cudaError_t launch_hc_finalize(const float* x, const float* part, const float* base, const float* scale, float* post,
                               float* comb, const void* nw, int nw_bf16, __half* out, int R, int D, float rms_eps,
                               float hc_eps, int iters, float n_eps, float cbias, float cscale, cudaStream_t st)
{
    if (R <= 0) return cudaSuccess;
    const int q = D / 4;
    const int threads = q >= 1024 ? 1024 : ((q + 31) / 32) * 32 < 256 ? 256 : ((q + 31) / 32) * 32;
    const dim3 grid(2, R);
    if (nw_bf16)
        hc_finalize_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(x, part, base, scale, post, comb,
            static_cast<const __nv_bfloat16*>(nw), out, D, rms_eps, hc_eps, iters, n_eps, cbias, cscale);
    else
        hc_finalize_kernel<__half><<<grid, threads, 0, st>>>(x, part, base, scale, post, comb,
            static_cast<const __half*>(nw), out, D, rms_eps, hc_eps, iters, n_eps, cbias, cscale);
    return cudaGetLastError();
}

}  // namespace glmx
