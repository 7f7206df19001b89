// Routed-expert MoE layer, decode-sized batches: grouped EXL3 dequant-GEMV on sm_100a.
//
// Pipeline of one forward call (all on one stream):
//   route   (route.cu)        picks -> expert-major rows, jobs of <= 8 rows
//   prep                      per row: xt = fp16(had128(x * suh) * HAD) for gate and up   (ft_core.h:96-102)
//   gemv<gate+up>             per (job, 128-col block, k-split): trellis tiles streamed by the bulk-copy engine into a
//                             shared-memory ring, decoded in registers straight into mma.m16n8k16 A fragments, fp32
//                             accumulation; epilogue: out_block (ft_core.h:104-110) of g and u, a = fp16(silu(g) * u)
//                             (ft_core.h:123-132, 980), then the down projection's input transform for that block
//   gemv<down>                same main loop over the down matrix; epilogue out_block -> per-row fp32 y
//   combine                   out[t] = sum over t's picks in pick order of w * y (+ shared expert), fp32
//                             (ft_core.h:1020-1033; ft_combine's add, ft_tier_cu.cu:226-233)
//
// Work split of the GEMV kernels: a CTA of 8 consumer warps + 1 producer warp processes items (job, n-block of 128
// outputs, k-split); consumer warp w owns n-tile w of the block for the whole item (no cross-warp reduction), the
// producer warp's lane 0 issues cp.async.bulk copies of the item's k-rows (8 tiles = 8*32*K contiguous bytes per k-row
// in the native layout) and of the rows' activations into a NST-deep ring guarded by full/empty mbarriers.
// Split-K partials are summed in a fixed order by the last CTA of a (job, block), so results are deterministic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int RB = 8;        // k-rows (16 inputs each) per pipeline stage = one 128-input block
constexpr int NCW = 8;       // consumer warps = n-tiles per 128-output block
constexpr int NTHR = (NCW + 1) * 32;
constexpr int XROW = 272;    // bytes per staged activation row: 128 fp16 + 16 bytes pad (conflict-free B loads)
#ifndef GLMX_EXACT_CTAS
#define GLMX_EXACT_CTAS 3
#endif
constexpr int CTAS_PER_SM = GLMX_EXACT_CTAS;
constexpr int RING_BYTES = (CTAS_PER_SM >= 3 ? 64 : 96) * 1024;    // per CTA; CTAS_PER_SM rings share an SM

template <int K0, int K1, int NMAT>
struct Cfg
{
    static constexpr int TB0 = 32 * K0, TB1 = 32 * K1;
    static constexpr int ROW0 = 8 * TB0, ROW1 = 8 * TB1;
    static constexpr int MAT0 = RB * ROW0, MAT1 = NMAT > 1 ? RB * ROW1 : 0;
    static constexpr int XS = MAXM * XROW;
    static constexpr int STAGE = (MAT0 + MAT1 + NMAT * XS + 127) / 128 * 128;   // tensor copies land 128-byte aligned
    static constexpr int NST = RING_BYTES / STAGE < 3 ? 3 : (RING_BYTES / STAGE > 12 ? 12 : RING_BYTES / STAGE);
    static constexpr int RED = NMAT * MAXM * 128 * 4;
    static constexpr int SMEM = NST * STAGE + RED + 2 * NST * 8;
    static_assert(STAGE % 128 == 0 && MAT0 % 128 == 0 && (MAT0 + MAT1) % 16 == 0, "stage alignment");
};

struct GemvArgs
{
    const Plan* plan;
    const int4* jobs;
    const uint64_t* trellis;     // [E_total][3]
    const CUtensorMap* tmaps;    // [E_total][3]: each trellis tensor as rows of k-tiles (boxes of 8 rows x 8 tiles)
    int proj0;                   // projection index of matrix 0 (0 = gate, 2 = down)
    int kt, ntn;                 // k-tiles and n-tiles of the matrix
    int kdim, ndim;              // K and N
    const __half* xin0; const __half* xin1;       // staged activation rows [R][kdim]
    const __half* svh0; const __half* svh1;       // [E_total][ndim]
    const __half* suh_next;                       // gate/up: suh of down [E_total][ndim]
    __half* xd;                                   // gate/up epilogue output [R][ndim]
    float* y;                                     // down epilogue output [R][ndim]
    float* partials; int* counters; int* err;
    float act_limit;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }

__device__ __forceinline__ float h2f(const __half* p) { return __half2float(*p); }

template <int K0, int K1, int NMAT, bool GATEUP>
__global__ void __launch_bounds__(NTHR, CTAS_PER_SM) gemv_kernel(GemvArgs a)
{
    using C = Cfg<K0, K1, NMAT>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float* red = reinterpret_cast<float*>(smem + C::NST * C::STAGE);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NST * C::STAGE + C::RED);
    uint64_t* empty = full + C::NST;
    __shared__ int s_last;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0)
    {
        for (int s = 0; s < C::NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], NCW); }
        s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const Plan pl = *a.plan;
    const int nb = a.ntn / 8;
    const int S = GATEUP ? pl.S_gu : pl.S_d;
    const int kqs = (a.kt / RB) / S;                        // stages per item
    const long long items = (long long) pl.J * nb * S;

    if (warp == NCW)
    {
        // ---------------- producer ----------------
        if (lane != 0) return;
        long long it = 0;
        for (long long item = blockIdx.x; item < items && !s_abort; item += gridDim.x)
        {
            const int ks = (int) (item % S);
            const long long jn = item / S;
            const int nbi = (int) (jn % nb), j = (int) (jn / nb);
            const int4 job = a.jobs[j];
            const CUtensorMap* m0 = a.tmaps + job.x * 3 + a.proj0;
            const uint32_t bytes = (uint32_t) (C::MAT0 + C::MAT1 + NMAT * job.z * 256);
            for (int q = 0; q < kqs; ++q, ++it)
            {
                const int s = (int) (it % C::NST);
                const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
                if (!s_abort && !mbar_wait_bounded(&empty[s], ph ^ 1u)) { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; }
                if (s_abort) break;
                const int kr = (ks * kqs + q) * RB;
                uint8_t* st = ring + s * C::STAGE;
                mbar_arrive_expect_tx(&full[s], bytes);
                // the stage's RB k-tile rows x 8 tiles of each matrix: one tensor copy (x in 32-bit words)
                tma_load_2d(st, m0, nbi * 8 * C::TB0 / 4, kr, &full[s]);
                if (NMAT > 1) tma_load_2d(st + C::MAT0, m0 + 1, nbi * 8 * C::TB1 / 4, kr, &full[s]);
                uint8_t* xs = st + C::MAT0 + C::MAT1;
                for (int i = 0; i < job.z; ++i)
                    bulk_g2s(xs + i * XROW, a.xin0 + (size_t) (job.y + i) * a.kdim + kr * 16, 256, &full[s]);
                if (NMAT > 1)
                    for (int i = 0; i < job.z; ++i)
                        bulk_g2s(xs + C::XS + i * XROW, a.xin1 + (size_t) (job.y + i) * a.kdim + kr * 16, 256, &full[s]);
            }
        }
        // drain: every issued stage must have landed before the CTA may exit
        const long long first = it > C::NST ? it - C::NST : 0;
        for (long long k = first; k < it; ++k)
            if (!mbar_wait_bounded(&full[k % C::NST], (uint32_t) ((k / C::NST) & 1))) { atomicOr(a.err, ERR_TIMEOUT_FULL); break; }
        return;
    }

    // ---------------- consumers ----------------
    LaneDecode<K0> L0;
    L0.init(lane);
    LaneDecode<K1> L1;
    L1.init(lane);
    OnesFrag ones;
    ones.init(lane);
    const int g = lane >> 2, tq = lane & 3;
    // per-lane offsets inside a stage: this warp's tile of k-row 0 and this lane's B-fragment words
    const int t0_off = warp * C::TB0, t1_off = C::MAT0 + warp * C::TB1;
    const int x_off = C::MAT0 + C::MAT1 + g * XROW + tq * 4;
    long long it = 0;
    for (long long item = blockIdx.x; item < items; item += gridDim.x)
    {
        const long long jn = item / S;
        const int nbi = (int) (jn % nb), j = (int) (jn / nb);
        const int4 job = a.jobs[j];
        // Accumulation: one tensor-core chain per 128-input block (a pipeline stage), then the block sum is added into
        // a (hi, lo) fp32 pair with Fast2Sum, so rounding errors do not grow with the chain length.
        float acc[NMAT][4], lo[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[m][v] = lo[m][v] = 0.0f;

        for (int q = 0; q < kqs; ++q, ++it)
        {
            const int s = (int) (it % C::NST);
            const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
            if (!s_abort && !mbar_wait_bounded(&full[s], ph)) { atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; }
            const uint8_t* st = ring + s * C::STAGE;
            float blk[NMAT][4];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) blk[m][0] = blk[m][1] = blk[m][2] = blk[m][3] = 0.0f;
#pragma unroll
            for (int r = 0; r < RB; ++r)
            {
                uint32_t af[4];
                decode_frag_tc<K0>(st + t0_off + r * C::ROW0, L0, ones, af);
                mma16816(blk[0], af, lds32(st + x_off + r * 32), lds32(st + x_off + r * 32 + 16));
                if (NMAT > 1)
                {
                    uint32_t bf[4];
                    decode_frag_tc<K1>(st + t1_off + r * C::ROW1, L1, ones, bf);
                    mma16816(blk[NMAT - 1], bf, lds32(st + x_off + C::XS + r * 32), lds32(st + x_off + C::XS + r * 32 + 16));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int v = 0; v < 4; ++v)
                {
                    const float sum = __fadd_rn(acc[m][v], blk[m][v]);
                    const float big = fabsf(acc[m][v]) >= fabsf(blk[m][v]) ? acc[m][v] : blk[m][v];
                    const float small = fabsf(acc[m][v]) >= fabsf(blk[m][v]) ? blk[m][v] : acc[m][v];
                    lo[m][v] = __fadd_rn(lo[m][v], __fsub_rn(small, __fsub_rn(sum, big)));
                    acc[m][v] = sum;
                }
        }
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[m][v] = __fadd_rn(acc[m][v], lo[m][v]);

        // ---- epilogue: fragments -> red[mat][token][128] ----
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
        {
            float* rm = red + m * MAXM * 128;
            const int o = warp * 16 + g;
            rm[(2 * tq) * 128 + o] = acc[m][0];
            rm[(2 * tq + 1) * 128 + o] = acc[m][1];
            rm[(2 * tq) * 128 + o + 8] = acc[m][2];
            rm[(2 * tq + 1) * 128 + o + 8] = acc[m][3];
        }
        consumer_sync();
        if (S > 1)
        {
            constexpr int NV = NMAT * MAXM * 128;
            float* part = a.partials + (size_t) item * NV;
            for (int i = tid; i < NV; i += NCW * 32) __stcg(part + i, red[i]);
            __threadfence();
            consumer_sync();
            if (tid == 0)
            {
                const int old = atomicAdd(&a.counters[jn], 1);
                s_last = old == S - 1;
            }
            consumer_sync();
            if (!s_last) continue;
            __threadfence();
            const float* p0 = a.partials + (size_t) (jn * S) * NV;
            for (int i = tid; i < NV; i += NCW * 32)
            {
                float v = 0.0f;
                for (int k = 0; k < S; ++k) v += __ldcg(p0 + (size_t) k * NV + i);
                red[i] = v;
            }
            consumer_sync();
        }

        if (warp < job.z)
        {
            const int i = warp, row = job.y + i, e = job.x;
            const size_t cb = (size_t) e * a.ndim + nbi * 128;
            if (GATEUP)
            {
                float gv[4], uv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    gv[q] = r16(red[i * 128 + lane + 32 * q]);
                    uv[q] = r16(red[MAXM * 128 + i * 128 + lane + 32 * q]);
                }
                had128_warp(gv, lane);
                had128_warp(uv, lane);
                float av[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    const int c = lane + 32 * q;
                    const float gq = r16(__fmul_rn(__fmul_rn(gv[q], HAD), h2f(a.svh0 + cb + c)));
                    const float uq = r16(__fmul_rn(__fmul_rn(uv[q], HAD), h2f(a.svh1 + cb + c)));
                    av[q] = __fmul_rn(r16(act_mul(gq, uq, a.act_limit)), h2f(a.suh_next + cb + c));
                }
                had128_warp(av, lane);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    const int c = lane + 32 * q;     // stored in PERM16 order inside each 16-row tile (decode_frag_tc)
                    a.xd[(size_t) row * a.ndim + nbi * 128 + (c & ~15) + perm16_inv(c & 15)] = __float2half_rn(__fmul_rn(av[q], HAD));
                }
            }
            else
            {
                float yv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) yv[q] = r16(red[i * 128 + lane + 32 * q]);
                had128_warp(yv, lane);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    const int c = lane + 32 * q;
                    a.y[(size_t) row * a.ndim + nbi * 128 + c] = r16(__fmul_rn(__fmul_rn(yv[q], HAD), h2f(a.svh0 + cb + c)));
                }
            }
        }
        consumer_sync();
    }
}

// ---- prep: xt = fp16(had128(x * suh) * HAD) per row and projection (gate, up) ----
// One warp per (token, 128-input block, projection): the token's x block is loaded once and transformed for every row
// of the token (its routed picks, then the shared expert's row), each with that row's expert's suh.
struct PrepArgs
{
    const Plan* plan;
    const void* x; int x_dtype; int H;
    int ntok, topk, has_shared, E;
    const int* pick_row; const int* row_expert;
    const __half* suh_g; const __half* suh_u;
    __half* xg; __half* xu;
    int natural;          // 1: natural input order (tensor-core GEMM), 0: PERM16 order inside 16-row tiles (GEMV)
};

__device__ __forceinline__ float load_x(const void* x, int dt, size_t i)
{
    if (dt == GLMX_F16) return __half2float(reinterpret_cast<const __half*>(x)[i]);
    if (dt == GLMX_BF16) return r16(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]));
    return reinterpret_cast<const float*>(x)[i];
}

__global__ void __launch_bounds__(256) prep_kernel(PrepArgs a)
{
    const int nbk = a.H / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int t = (int) (wid / (2 * nbk));
    if (t >= a.ntok) return;
    const int rem = (int) (wid % (2 * nbk)), p = rem / nbk, b = rem % nbk;
    float xv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = load_x(a.x, a.x_dtype, (size_t) t * a.H + b * 128 + lane + 32 * q);
    const __half* suh_p = p ? a.suh_u : a.suh_g;
    __half* out_p = p ? a.xu : a.xg;
    const int nk = a.topk + (a.has_shared ? 1 : 0);
    for (int k = 0; k < nk; ++k)
    {
        int r, e;
        if (k < a.topk)
        {
            r = a.pick_row[(size_t) t * a.topk + k];
            if (r < 0) continue;
            e = a.row_expert[r];
        }
        else { r = a.plan->P + t; e = a.E; }
        const __half* suh = suh_p + (size_t) e * a.H + b * 128;
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = __fmul_rn(xv[q], __half2float(suh[lane + 32 * q]));
        had128_warp(v, lane);
        __half* out = out_p + (size_t) r * a.H + b * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const int c = lane + 32 * q;         // GEMV: PERM16 order inside each 16-row tile (decode_frag_tc)
            out[a.natural ? c : (c & ~15) + perm16_inv(c & 15)] = __float2half_rn(__fmul_rn(v[q], HAD));
        }
    }
}

// ---- combine: out[t] = sum_k w * y[row(t,k)] (+ shared), fp32, pick order ----
struct CombineArgs
{
    const Plan* plan;
    const int* pick_row; const float* row_weight; const float* y;
    int H, ntok, topk, has_shared;
    void* out; int out_dtype; int accumulate;
    HcOut hc;                           // hc.x != nullptr: hyper-connection epilogue instead of writing out
};

__device__ __forceinline__ void combine_cols(const CombineArgs& a, int t, int c)
{
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < a.topk; ++k)
    {
        const int r = a.pick_row[t * a.topk + k];
        if (r < 0) continue;
        const float w = a.row_weight[r];
        const float4 y = *reinterpret_cast<const float4*>(a.y + (size_t) r * a.H + c);
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, y.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, y.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, y.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, y.w));
    }
    if (a.has_shared)
    {
        const int r = a.plan->P + t;
        const float4 y = *reinterpret_cast<const float4*>(a.y + (size_t) r * a.H + c);
        acc.x = __fadd_rn(acc.x, y.x); acc.y = __fadd_rn(acc.y, y.y); acc.z = __fadd_rn(acc.z, y.z); acc.w = __fadd_rn(acc.w, y.w);
    }
    if (a.hc.peer.recv)
    {
        const PeerOut& p = a.hc.peer;
        *reinterpret_cast<float4*>(peer_row(p.recv, p.rank, p.world, p.rpr, p.seq, t, a.H) + c) = acc;
        return;
    }
    if (a.hc.x)
    {
        const float v[4] = { acc.x, acc.y, acc.z, acc.w };
#pragma unroll
        for (int i = 0; i < 4; ++i)
            hc_apply_col(a.hc.x + (size_t) t * 4 * a.H, a.H, c + i, a.hc.y_half ? __half2float(__float2half_rn(v[i])) : v[i],
                         a.hc.post + (size_t) t * 4, a.hc.comb + (size_t) t * 16);
        return;
    }
    const size_t o = (size_t) t * a.H + c;
    if (a.out_dtype == GLMX_F32)
    {
        float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + o);
        if (a.accumulate)
        {
            const float4 v = *p;
            acc.x = __fadd_rn(v.x, acc.x); acc.y = __fadd_rn(v.y, acc.y); acc.z = __fadd_rn(v.z, acc.z); acc.w = __fadd_rn(v.w, acc.w);
        }
        *p = acc;
    }
    else
    {
        __half* p = reinterpret_cast<__half*>(a.out) + o;
        float v[4] = { acc.x, acc.y, acc.z, acc.w };
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = __float2half_rn(a.accumulate ? __fadd_rn(__half2float(p[i]), v[i]) : v[i]);
    }
}

__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a)
{
    const int t = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c < a.H) combine_cols(a, t, c);
    if (a.hc.peer.recv) peer_done(a.hc.peer.recv, a.hc.peer.flags, a.hc.peer.counter, a.hc.peer.rank, a.hc.peer.world, a.hc.peer.seq);
}

// ---- known-answer decode of whole tiles (the GEMV's own decode_frag_tc, rows un-permuted on the way out) ----
template <int K>
__global__ void decode_tiles_kernel(const uint8_t* tiles, int ntiles, uint16_t* out)
{
    __shared__ __align__(16) uint8_t tile[8][32 * 4];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + w;
    if (t >= ntiles) return;        // warp-uniform
    for (int i = lane; i < 32 * K; i += 32) tile[w][i] = tiles[(size_t) t * 32 * K + i];
    __syncwarp();
    LaneDecode<K> L;
    L.init(lane);
    OnesFrag ones;
    ones.init(lane);
    uint32_t a[4];
    decode_frag_tc<K>(tile[w], L, ones, a);
    const int g = lane >> 2, tq = lane & 3;
    // a[0] = rows (perm16(2tq), perm16(2tq+1)) of column g, a[1] the same rows of column g+8, a[2] / a[3] those rows + 8
    const int r0 = perm16(2 * tq), r1 = perm16(2 * tq + 1);
    uint16_t* o = out + (size_t) t * 256;
    o[r0 * 16 + g] = a[0] & 0xffff;             o[r1 * 16 + g] = a[0] >> 16;
    o[r0 * 16 + g + 8] = a[1] & 0xffff;         o[r1 * 16 + g + 8] = a[1] >> 16;
    o[(r0 + 8) * 16 + g] = a[2] & 0xffff;       o[(r1 + 8) * 16 + g] = a[2] >> 16;
    o[(r0 + 8) * 16 + g + 8] = a[3] & 0xffff;   o[(r1 + 8) * 16 + g + 8] = a[3] >> 16;
}

template <int K0, int K1, int NMAT, bool GATEUP>
cudaError_t launch_gemv(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    using C = Cfg<K0, K1, NMAT>;
    static bool attr_set[64] = {};
    if (!attr_set[L.device])
    {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<K0, K1, NMAT, GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[L.device] = true;
    }
    gemv_kernel<K0, K1, NMAT, GATEUP><<<grid, NTHR, C::SMEM, st>>>(a);
    return cudaGetLastError();
}

template <int K0>
cudaError_t launch_gateup_k0(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    switch (L.bits[1])
    {
        case 2: return launch_gemv<K0, 2, 2, true>(L, a, grid, st);
        case 3: return launch_gemv<K0, 3, 2, true>(L, a, grid, st);
        default: return launch_gemv<K0, 4, 2, true>(L, a, grid, st);
    }
}

cudaError_t launch_gateup(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    switch (L.bits[0])
    {
        case 2: return launch_gateup_k0<2>(L, a, grid, st);
        case 3: return launch_gateup_k0<3>(L, a, grid, st);
        default: return launch_gateup_k0<4>(L, a, grid, st);
    }
}

cudaError_t launch_down(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    switch (L.bits[2])
    {
        case 2: return launch_gemv<2, 2, 1, false>(L, a, grid, st);
        case 3: return launch_gemv<3, 3, 1, false>(L, a, grid, st);
        default: return launch_gemv<4, 4, 1, false>(L, a, grid, st);
    }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

int gemv_sm_count(const Layer& L)
{
    static int sms[64] = {};
    if (!sms[L.device])
    {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, L.device) != cudaSuccess || v <= 0) v = 148;
        sms[L.device] = v;
    }
    return sms[L.device];
}

int gemv_grid_ctas(const Layer& L)
{
    return gemv_sm_count(L) * CTAS_PER_SM;   // CTAS_PER_SM CTAs (9 warps, <= 64 KB ring each) per SM
}

WsLayout ws_layout(const Layer& L, int ntok, int topk, int grid_ctas)
{
    WsLayout w;
    const int n = ntok * topk;
    const int rows = n + (L.has_shared ? ntok : 0);
    const int jobs = rows + 1;                       // each job holds >= 1 row
    const int nmax = (L.H > L.I ? L.H : L.I);
    w.rows_max = rows; w.jobs_max = jobs; w.part_slots = 2 * grid_ctas;
    size_t o = 0;
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + (bytes ? bytes : 1)); return at; };
    w.plan = take(sizeof(Plan));
    w.err = take(sizeof(int));
    w.offsets = take(sizeof(int) * (size_t) (L.E + 1));
    w.row_token = take(sizeof(int) * (size_t) rows);
    w.row_expert = take(sizeof(int) * (size_t) rows);
    w.row_pick = take(sizeof(int) * (size_t) rows);
    w.row_weight = take(sizeof(float) * (size_t) rows);
    w.pick_row = take(sizeof(int) * (size_t) n);
    w.jobs = take(sizeof(int4) * (size_t) jobs);
    w.row_job = take(sizeof(int) * (size_t) rows);
    w.cnt_gu = take(sizeof(int) * (size_t) jobs * (L.I / 128));
    w.cnt_d = take(sizeof(int) * (size_t) jobs * (L.H / 128));
    w.xg = take(sizeof(__half) * (size_t) rows * L.H);
    w.xu = take(sizeof(__half) * (size_t) rows * L.H);
    w.xd = take(sizeof(__half) * (size_t) rows * L.I);
    w.yrow = take(sizeof(float) * (size_t) rows * L.H);
    w.partials = take(sizeof(float) * (size_t) w.part_slots * 2 * MAXM * 128 + 0 * nmax);
    // raw fp32 gate/up outputs (I16 GEMV: one slice; prefill GEMM: one slice per K split)
    w.yraw_gu = take(sizeof(float) * (size_t) PF_KSPLIT * rows * 2 * L.I);
    // I16 mode (decode-sized calls only): jobs of <= I16_MAXM rows of one expert: at most rows/4 + one partial job per
    // expert
    const int ji = rows <= I16_MAX_ROWS ? (rows < (rows + 3) / 4 + L.E_total ? rows : (rows + 3) / 4 + L.E_total) : 0;
    w.jobs_max_i16 = ji;
    const int BH = L.H / 128, BI = L.I / 128;
    w.actb_gu = take((size_t) ji * BH * i16_rec_bytes(2));
    w.psum_gu = take(sizeof(float) * (size_t) (ji ? rows : 0) * 2 * BH);
    w.actb_d = take((size_t) ji * BI * i16_rec_bytes(1));
    w.psum_d = take(sizeof(float) * (size_t) (ji ? rows : 0) * BI);
    // K-split class sums of the I16 gate/up GEMV for calls of at most I16_SPLIT_MAX_ROWS rows
    w.isum_gu = take(ji && rows <= I16_SPLIT_MAX_ROWS ? sizeof(int) * 4 * (size_t) rows * 2 * BH * L.I : 0);
    w.total = o;
    return w;
}

cudaError_t launch_prep_exact(const Layer& L, const void* x, int x_dtype, int ntok, int topk, uint8_t* ws, const WsLayout& lay,
                              cudaStream_t st, bool natural)
{
    if (ntok <= 0) return cudaSuccess;
    PrepArgs p;
    p.plan = reinterpret_cast<const Plan*>(ws + lay.plan); p.x = x; p.x_dtype = x_dtype; p.H = L.H;
    p.ntok = ntok; p.topk = topk; p.has_shared = L.has_shared; p.E = L.E;
    p.pick_row = reinterpret_cast<const int*>(ws + lay.pick_row);
    p.row_expert = reinterpret_cast<const int*>(ws + lay.row_expert);
    p.suh_g = reinterpret_cast<const __half*>(L.suh[0]);
    p.suh_u = reinterpret_cast<const __half*>(L.suh[1]);
    p.xg = reinterpret_cast<__half*>(ws + lay.xg);
    p.xu = reinterpret_cast<__half*>(ws + lay.xu);
    p.natural = natural ? 1 : 0;
    const long long warps = (long long) ntok * 2 * (L.H / 128);
    prep_kernel<<<(unsigned) ((warps + 7) / 8), 256, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_decode_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, int mode, void* out,
                                  int out_dtype, int accumulate, uint8_t* ws, const WsLayout& lay, int grid, cudaStream_t st,
                                  void* const* events, const HcOut* hc)
{
    (void) mode;
    auto mark = [&](int i) -> cudaError_t {
        if (events && events[i]) return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
        return cudaSuccess;
    };
    const Plan* plan = reinterpret_cast<const Plan*>(ws + lay.plan);
    const int rows = lay.rows_max;
    cudaError_t e;
    if (rows > 0)
    {
        if ((e = launch_prep_exact(L, x, x_dtype, ntok, topk, ws, lay, st, false)) != cudaSuccess) return e;
        if ((e = mark(2)) != cudaSuccess) return e;

        GemvArgs g;
        g.plan = plan;
        g.jobs = reinterpret_cast<const int4*>(ws + lay.jobs);
        g.trellis = L.d_trellis;
        g.tmaps = L.d_tmaps;
        g.err = reinterpret_cast<int*>(ws + lay.err);
        g.partials = reinterpret_cast<float*>(ws + lay.partials);
        g.act_limit = L.act_limit;
        // gate + up
        g.proj0 = 0; g.kt = L.H / 16; g.ntn = L.I / 16; g.kdim = L.H; g.ndim = L.I;
        g.xin0 = reinterpret_cast<const __half*>(ws + lay.xg); g.xin1 = reinterpret_cast<const __half*>(ws + lay.xu);
        g.svh0 = reinterpret_cast<const __half*>(L.svh[0]);
        g.svh1 = reinterpret_cast<const __half*>(L.svh[1]);
        g.suh_next = reinterpret_cast<const __half*>(L.suh[2]);
        g.xd = reinterpret_cast<__half*>(ws + lay.xd);
        g.y = nullptr;
        g.counters = reinterpret_cast<int*>(ws + lay.cnt_gu);
        if ((e = launch_gateup(L, g, grid, st)) != cudaSuccess) return e;
        if ((e = mark(3)) != cudaSuccess) return e;
        // down
        g.proj0 = 2; g.kt = L.I / 16; g.ntn = L.H / 16; g.kdim = L.I; g.ndim = L.H;
        g.xin0 = g.xd; g.xin1 = nullptr;
        g.svh0 = reinterpret_cast<const __half*>(L.svh[2]);
        g.svh1 = nullptr; g.suh_next = nullptr;
        g.y = reinterpret_cast<float*>(ws + lay.yrow);
        g.counters = reinterpret_cast<int*>(ws + lay.cnt_d);
        if ((e = launch_down(L, g, grid, st)) != cudaSuccess) return e;
        if ((e = mark(4)) != cudaSuccess) return e;
    }
    else
    {
        for (int i = 2; i <= 4; ++i)
            if ((e = mark(i)) != cudaSuccess) return e;
    }
    if (ntok > 0)
    {
        CombineArgs c;
        c.plan = plan;
        c.pick_row = reinterpret_cast<const int*>(ws + lay.pick_row);
        c.row_weight = reinterpret_cast<const float*>(ws + lay.row_weight);
        c.y = reinterpret_cast<const float*>(ws + lay.yrow);
        c.H = L.H; c.ntok = ntok; c.topk = topk; c.has_shared = L.has_shared;
        c.out = out; c.out_dtype = out_dtype; c.accumulate = accumulate;
        c.hc = hc ? *hc : HcOut{ nullptr, nullptr, nullptr, 0 };
        dim3 grd((unsigned) ((L.H / 4 + 255) / 256), (unsigned) ntok);
        combine_kernel<<<grd, 256, 0, st>>>(c);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return mark(5);
}

cudaError_t launch_decode_tiles(const uint8_t* tiles, int bits, int ntiles, uint16_t* out, cudaStream_t st)
{
    if (ntiles <= 0) return cudaSuccess;
    const unsigned grid = (unsigned) ((ntiles + 7) / 8);
    if (bits == 2) decode_tiles_kernel<2><<<grid, 256, 0, st>>>(tiles, ntiles, out);
    else if (bits == 3) decode_tiles_kernel<3><<<grid, 256, 0, st>>>(tiles, ntiles, out);
    else decode_tiles_kernel<4><<<grid, 256, 0, st>>>(tiles, ntiles, out);
    return cudaGetLastError();
}

}  // namespace glmx
