// Top-k token split: expert-major grouping of the router's picks (one CTA).
//
// Reference behaviour: moe_forward builds jobs by walking tokens in order and, per token, its picks in order,
// appending (token, weight) to the expert's current job and opening a new job once it holds MAXM = 8 tokens
// (kernels/cpu_avx2/ft_core.h:1344-1349). tier_forward skips picks with sel < 0 (ft_tier_ext.cpp:896-898).
// Here the rows are laid out expert-major (expert ascending, pick index ascending = token order), which is the
// canonical order of the reference's grouped rows, and jobs are consecutive runs of <= 8 rows of one expert, so
// each job holds exactly the tokens of the corresponding reference job.
//
// The stable scatter processes the picks in chunks of 1024: __match_any_sync gives each pick its rank among equal
// experts in its warp, a per-(warp, expert) count table gives the rank across warps, a running base per expert
// carries ranks across chunks. This is the warp-ballot prefix of ft_split_fast (kernels/k110/ft_split_fast.cu:153-175)
// generalised from one warp to the whole block.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int RT = 1024;   // threads of the route CTA

struct RouteArgs
{
    const void* sel; int sel_i64;
    const void* w; int w_dtype;
    int ntok, topk, E, has_shared;
    int first;                // global id of local expert 0
    int maxm;                 // rows per job (EXACT GEMV 8, I16 4, GEMM 128)
    int nb_gu, nb_d;          // n-blocks of 128 of the gate/up and down kernels
    int kq_gu, kq_d;          // GEMV pipeline stages per full K of gate/up and down
    int cost_gu, cost_d;      // an item's fixed cost in those stages
    int grid_ctas;
    long long part_bytes;     // room for EXACT split-K partials: splits x rows x matrices x columns x 8 bytes
    Plan* plan;
    int* offsets; int* row_token; int* row_expert; int* row_pick; float* row_weight; int* pick_row; int4* jobs; int* row_job;
    int* cnt_gu; int* cnt_d; int* err;
};

// local expert id of pick p: sel - first; anything outside [0, E) (masked picks, other shards' experts) is skipped
__device__ __forceinline__ int load_sel(const RouteArgs& a, int p)
{
    const long long g = a.sel_i64 ? reinterpret_cast<const long long*>(a.sel)[p] : (long long) reinterpret_cast<const int*>(a.sel)[p];
    if (g < 0) return -1;
    const long long e = g - a.first;
    return (e >= 0 && e < a.E) ? (int) e : -1;
}

__device__ __forceinline__ float load_w(const RouteArgs& a, int p)
{
    if (a.w_dtype == GLMX_F16) return __half2float(reinterpret_cast<const __half*>(a.w)[p]);
    if (a.w_dtype == GLMX_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.w)[p]);
    return reinterpret_cast<const float*>(a.w)[p];
}

// exclusive scan of one int per thread (RT threads); returns the exclusive prefix, *total = sum
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total)
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
        int s = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;   // inclusive over warps
    }
    __syncthreads();
    const int before = (wid ? warp_sums[wid - 1] : 0) + x - v;
    *total = warp_sums[31];
    __syncthreads();
    return before;
}

// K splits of a GEMV with `units` (job, column block) items of `stages` pipeline stages on `target` resident CTAs:
// the divisor d of stages with the shortest critical path, ceil(units * d / target) waves of stages / d + item_cost
// stages each (an item's fixed cost - the split hand-off, the epilogue - measured at about two 128-input steps), the
// smaller d on ties, and d within the room for partial sums, max_split
__device__ int pick_split(long long units, int stages, int target, long long max_split, int item_cost)
{
    if (units <= 0) return 1;
    int best = 1;
    long long best_cost = ((units + target - 1) / target) * (stages + item_cost);
    for (int d = 2; d <= stages; ++d)
    {
        if (stages % d) continue;
        if (d > max_split) break;
        const long long cost = ((units * d + target - 1) / target) * (stages / d + item_cost);
        if (cost < best_cost) { best_cost = cost; best = d; }
    }
    return best;
}

__global__ void __launch_bounds__(RT) route_kernel(RouteArgs a)
{
    pdl_enter();
    extern __shared__ int sm[];
    const int E = a.E;
    int* cnt = sm;                                   // [E]
    int* base = cnt + E;                             // [E]
    int* jbase = base + E;                           // [E] first job of each expert
    unsigned short* wcnt = reinterpret_cast<unsigned short*>(jbase + E);  // [32][E]
    __shared__ int warp_sums[32];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int n = a.ntok * a.topk;

    for (int e = tid; e < E; e += RT) cnt[e] = 0;
    for (int i = tid; i < 32 * E; i += RT) wcnt[i] = 0;
    __syncthreads();
    for (int p = tid; p < n; p += RT)
    {
        const int e = load_sel(a, p);
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();

    // offsets and jobs (E <= RT: one expert per thread)
    const int c = tid < E ? cnt[tid] : 0;
    int P;
    const int off = block_exclusive_scan(c, warp_sums, &P);
    const int maxm = a.maxm;
    const int nj = (c + maxm - 1) / maxm;
    int Jr;
    const int joff = block_exclusive_scan(nj, warp_sums, &Jr);
    if (tid < E)
    {
        a.offsets[tid] = off;
        base[tid] = off;
        cnt[tid] = off;                              // from here on cnt holds the expert's first row
        jbase[tid] = joff;
        for (int q = 0; q < nj; ++q)
        {
            const int r0 = off + q * maxm, m = min(maxm, c - q * maxm);
            a.jobs[joff + q] = make_int4(tid, r0, m, 0);
        }
    }
    if (tid == 0) a.offsets[E] = P;
    const int nsh = a.has_shared ? a.ntok : 0;
    const int Jsh = (nsh + maxm - 1) / maxm;
    for (int q = tid; q < Jsh; q += RT)
    {
        const int r0 = P + q * maxm, m = min(maxm, nsh - q * maxm);
        a.jobs[Jr + q] = make_int4(E, r0, m, 0);
    }
    for (int t = tid; t < nsh; t += RT)
    {
        a.row_token[P + t] = t; a.row_expert[P + t] = E; a.row_pick[P + t] = -1; a.row_weight[P + t] = 1.0f;
        a.row_job[P + t] = Jr + t / maxm;
    }
    __syncthreads();

    // stable scatter, chunks of RT picks
    const unsigned lt = (1u << lane) - 1u;
    for (int c0 = 0; c0 < n; c0 += RT)
    {
        const int p = c0 + tid;
        int e = -1;
        float wt = 0.0f;
        if (p < n)
        {
            e = load_sel(a, p);
            wt = load_w(a, p);
            if (e < 0 || e >= E) { a.pick_row[p] = -1; e = -1; }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int lrank = __popc(peers & lt);
        if (e >= 0 && lrank == 0) wcnt[wid * E + e] = (unsigned short) __popc(peers);
        __syncthreads();
        if (e >= 0)
        {
            int pre = 0;
            for (int w2 = 0; w2 < wid; ++w2) pre += wcnt[w2 * E + e];
            const int r = base[e] + pre + lrank;
            a.row_token[r] = p / a.topk; a.row_expert[r] = e; a.row_pick[r] = p; a.row_weight[r] = wt;
            a.row_job[r] = jbase[e] + (r - cnt[e]) / maxm;
            a.pick_row[p] = r;
        }
        __syncthreads();
        for (int e2 = tid; e2 < E; e2 += RT)
        {
            int s = 0;
            for (int w2 = 0; w2 < 32; ++w2) { s += wcnt[w2 * E + e2]; wcnt[w2 * E + e2] = 0; }
            base[e2] += s;
        }
        __syncthreads();
    }

    const int J = Jr + Jsh;
    for (int i = tid; i < J * a.nb_gu; i += RT) a.cnt_gu[i] = 0;
    for (int i = tid; i < J * a.nb_d; i += RT) a.cnt_d[i] = 0;
    if (tid == 0)
    {
        Plan pl;
        pl.P = P; pl.R = P + nsh; pl.J = J;
        // partial sums of split k: [k][row][matrix][column]: gate/up 2 x I columns per row, down H
        const long long R = P + nsh > 0 ? P + nsh : 1;
        pl.S_gu = pick_split((long long) J * a.nb_gu, a.kq_gu, a.grid_ctas, a.part_bytes / (R * 2 * 128 * a.nb_gu * 8), a.cost_gu);
        pl.S_d = pick_split((long long) J * a.nb_d, a.kq_d, a.grid_ctas, a.part_bytes / (R * 128 * a.nb_d * 8), a.cost_d);
        pl.ntok = a.ntok; pl.topk = a.topk; pl.pad = 0;
        pl.next_gu = 0; pl.next_d = 0;
        *a.plan = pl;
        *a.err = 0;
    }
}

}  // namespace

cudaError_t launch_route(const Layer& L, const void* sel, int sel_i64, const void* w, int w_dtype, int ntok, int topk,
                         int maxm, uint8_t* ws, const WsLayout& lay, int grid_ctas, cudaStream_t st)
{
    RouteArgs a;
    a.maxm = maxm;
    a.sel = sel; a.sel_i64 = sel_i64; a.w = w; a.w_dtype = w_dtype;
    a.ntok = ntok; a.topk = topk; a.E = L.E; a.has_shared = L.has_shared; a.first = L.first;
    a.nb_gu = L.I / 128; a.nb_d = L.H / 128;
    // the EXACT GEMV's stages may hold two 128-input blocks; the I16 GEMV's hold one
    const int hb_gu = maxm == EXACT_MAXM ? exact_stage_blocks(L, 0) : 1, hb_d = maxm == EXACT_MAXM ? exact_stage_blocks(L, 2) : 1;
    a.kq_gu = L.H / (128 * hb_gu); a.kq_d = L.I / (128 * hb_d);
    a.cost_gu = 2 / hb_gu; a.cost_d = 2 / hb_d;
    a.grid_ctas = grid_ctas;
    a.part_bytes = (long long) lay.part_bytes;
    a.plan = reinterpret_cast<Plan*>(ws + lay.plan);
    a.offsets = reinterpret_cast<int*>(ws + lay.offsets);
    a.row_token = reinterpret_cast<int*>(ws + lay.row_token);
    a.row_expert = reinterpret_cast<int*>(ws + lay.row_expert);
    a.row_pick = reinterpret_cast<int*>(ws + lay.row_pick);
    a.row_weight = reinterpret_cast<float*>(ws + lay.row_weight);
    a.pick_row = reinterpret_cast<int*>(ws + lay.pick_row);
    a.jobs = reinterpret_cast<int4*>(ws + lay.jobs);
    a.row_job = reinterpret_cast<int*>(ws + lay.row_job);
    a.cnt_gu = reinterpret_cast<int*>(ws + lay.cnt_gu);
    a.cnt_d = reinterpret_cast<int*>(ws + lay.cnt_d);
    a.err = reinterpret_cast<int*>(ws + lay.err);
    const size_t smem = sizeof(int) * 3 * L.E + sizeof(unsigned short) * 32 * L.E + 16;
    static bool attr_set[64] = {};
    if (L.device < 0 || L.device >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[L.device])
    {
        cudaError_t e = cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[L.device] = true;
    }
    return launch_chained(route_kernel, dim3(1), dim3(RT), smem, st, a);
}

}  // namespace glmx
