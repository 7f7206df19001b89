// Routed-expert MoE layer for prefill-sized batches (many rows per expert), EXACT mode: a grouped GEMM on the
// 5th-generation tensor cores. Per (job of <= 128 rows of one expert, column block of TN = 256 (else 128) outputs,
// projection, K split) tile:
//
//   A  = the rows' transformed activations (fp16, natural input order), [128 x 64] per stage,
//        loaded by the tensor-memory-access unit from the row-major activation buffer with the 128-byte swizzle
//   B  = the expert's trellis tiles for the stage (4 k-rows x TN/16 tiles), bulk-copied to shared memory, decoded by
//        8 warps into fp16 (integer byte sums with dp4a + codebook FMA, decode_frag_nat: a lane's 8 stream weights are
//        exactly its m16n8k16 fragment of the transposed tile) and written with stmatrix into the K-major interleaved
//        layout the MMA reads. The byte sums stay off the tensor pipe, which the tcgen05 MMAs keep busy
//   D  = fp32 accumulators in tensor memory (tcgen05.mma kind::f16, M=128, N=TN, K=16 per instruction). Long K sums
//        are kept short: gate/up split K=6144 over 3 tiles (partial sums added in order in fp32 by the epilogue
//        kernel), and inside a tile 128-input block b accumulates into chain b % (512 / TN) of tensor memory, the chains
//        added in order in fp32 by the epilogue warps. With chains of at most 64 MMAs the tensor-core rounding stays
//        within the EXACT-mode accuracy of the reference's fp32 kernel.
//
// Warp roles: 0 producer (one lane issues the TMA / bulk copies), 1 MMA issuer (one lane) and tensor-memory owner,
// 2.. decoders (16 with TN = 256, 8 with TN = 128; warp d decodes tiles d, d + NDEC, ... of the stage's 4 x TN/16),
// then 8 epilogue warps (two per tensor-memory lane quarter, each draining half of the columns: raw fp32 D rows to
// global). Every wait is bounded; a timeout sets the workspace error word and all roles leave their loops,
// drain their asynchronous work and free the tensor memory.
//
// The numbers are those of the EXACT GEMV path (ft_core.h:313-387 with fp16 weights, fp32 accumulation); the
// transforms around the GEMMs (out_block, SiLU*up, the down input transform, the combine) are the same kernels'
// arithmetic (ft_core.h:96-132, 980, 1020-1033).
#include <cuda.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int PM = 128;                  // rows per tile (UMMA M)
constexpr int PK = 64;                   // k per stage (4 UMMA K16 steps, 4 trellis k-rows)
constexpr int NEPI = 8;
constexpr int W_PROD = 0, W_MMA = 1, W_DEC0 = 2;
constexpr int SMEM_MAX = 227 * 1024;
// kind::f16 instruction descriptor: D f32 (bit 4), A = B = f16, both K-major, N >> 3 at bit 17, M >> 4 at bit 24
__host__ __device__ constexpr uint32_t idesc_f16(int n) { return (1u << 4) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (PM >> 4) << 24); }

// TN: output columns per tile (UMMA N): 256 where the projection's width allows it (each activation tile read from
// L2 then feeds 256 FLOP per byte), else 128
template <int K, int TN>
struct CfgP
{
    static constexpr int NT = TN / 16;                  // trellis n-tiles per column block
    static constexpr int TA = PM * PK * 2;              // A tile bytes
    static constexpr int TB = TN * PK * 2;              // decoded B tile bytes
    static constexpr int TT = 4 * NT * 32 * K;          // trellis bytes per stage: 4 k-rows x NT tiles
    static constexpr int STAGE = TA + TB + TT;
    static constexpr int BAR_BYTES = 512;
    static constexpr int NST_FIT = (SMEM_MAX - 1024 - BAR_BYTES) / STAGE;
    static constexpr int NST = NST_FIT > 8 ? 8 : NST_FIT;
    static constexpr int SMEM = 1024 + NST * STAGE + BAR_BYTES;   // 1024: alignment slack of the swizzled A tiles
    static constexpr int TMEM_COLS = 512;
    static constexpr int CH = TMEM_COLS / TN;                      // accumulator chains
    // decoder warps: 16 with TN = 256 (4 tiles each per stage); 8 with TN = 128, whose epilogue needs the registers
    static constexpr int NDEC = TN == 256 ? 16 : 8;
    static constexpr int W_EPI0 = W_DEC0 + NDEC;
    static constexpr int THREADS = (W_EPI0 + NEPI) * 32;
    static_assert(STAGE % 1024 == 0, "A tiles must stay 1024-byte aligned");
    static_assert(NST >= 2, "at least two stages");
    static_assert(SMEM <= SMEM_MAX, "shared memory");
};

struct PfArgs
{
    const Plan* plan;
    const int4* jobs;
    const uint64_t* trellis;
    int proj0;           // first projection (0 = gate, 2 = down); tiles cover projections proj0 .. proj0 + nproj - 1
    int nproj;           // 2 for gate + up (activations tmA0 / tmA1), 1 for down or for one of gate / up
    int nslot, slot0;    // yraw row holds nslot projections; projection p of this launch goes to slot slot0 + p
    int kt;              // k-tiles of the projection (K / 16)
    int ntn;             // n-tiles of the projection (N / 16)
    int ndim;            // N
    int ksplit;          // K splits per (job, projection, column block); split s writes its partial sums to slice s
    size_t split_stride; // floats between the slices of yraw
    float* yraw;         // [ksplit][R][nslot][ndim] raw fp32 GEMM partial outputs
    int* err;
};

// ---- tcgen05 / TMA primitives -------------------------------------------------------------------------------------

// shared-memory matrix descriptor: start, leading / stride byte offsets, Blackwell version 1, swizzle mode
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swizzle)
{
    return (uint64_t) ((saddr & 0x3FFFFu) >> 4) | ((uint64_t) (lbo >> 4) << 16) | ((uint64_t) (sbo >> 4) << 32) |
           (1ull << 46) | ((uint64_t) swizzle << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc));
}

// arrive on `bar` once every tcgen05.mma this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's tensor-memory lane (32x32b shape: warp quarter q reads lanes 32q..32q+31)
// (the registers are valid after tmem_wait_ld)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// four 8x8 b16 matrices (the registers of an m16n8k16 A fragment) to shared memory, one 16-byte row per lane address
__device__ __forceinline__ void stmatrix_x4(uint32_t saddr, const uint32_t a[4])
{
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(a[0]), "r"(a[1]),
                 "r"(a[2]), "r"(a[3])
                 : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// tile t -> (job, column block, projection, K split); the split varies fastest, then the projection
struct PfTile
{
    int job, nb, p, ks;
};
__device__ __forceinline__ PfTile pf_tile(long long t, int NB, int NP, int KS)
{
    PfTile r;
    r.ks = (int) (t % KS);
    t /= KS;
    r.p = (int) (t % NP);
    t /= NP;
    r.nb = (int) (t % NB);
    r.job = (int) (t / NB);
    return r;
}

template <int K, int TN>
__global__ void __launch_bounds__(CfgP<K, TN>::THREADS, 1)
    gemm_pf_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1, PfArgs a)
{
    using C = CfgP<K, TN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NST * C::STAGE);
    uint64_t* dec = full + C::NST;
    uint64_t* empty = dec + C::NST;
    uint64_t* tfull = empty + C::NST;
    uint64_t* tempty = tfull + 1;
    uint64_t* fin = tempty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0)
    {
        for (int s = 0; s < C::NST; ++s) { mbar_init(&full[s], 1); mbar_init(&dec[s], C::NDEC); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        mbar_init(tempty, NEPI);
        mbar_init(fin, 1);
        s_abort = 0;
        fence_barrier_init();
    }
    if (warp == W_MMA)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t) C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int J = a.plan->J;
    const int NB = a.ndim / TN, NP = a.nproj, KS = a.ksplit;
    const long long ntiles = (long long) J * NB * NP * KS;
    const int nks = a.kt / 4 / KS;            // stages per tile (this tile's share of K)
    auto stage = [&](int s) { return smem + (size_t) s * C::STAGE; };
    // stage layout: A | B | T

    if (warp == W_PROD)
    {
        if (lane == 0)
        {
            long long it = 0;
            for (long long t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x)
            {
                const PfTile tl = pf_tile(t, NB, NP, KS);
                const int4 job = a.jobs[tl.job];
                const uint8_t* b = reinterpret_cast<const uint8_t*>(a.trellis[job.x * 3 + a.proj0 + tl.p]);
                const CUtensorMap* map = tl.p ? &tmA1 : &tmA0;
                for (int ks = 0; ks < nks; ++ks, ++it)
                {
                    const int s = (int) (it % C::NST);
                    const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1u)) { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; }
                    if (s_abort) break;
                    uint8_t* st = stage(s);
                    const int kg = tl.ks * nks + ks;              // stage index along the whole K
                    mbar_arrive_expect_tx(&full[s], (uint32_t) (C::TA + C::TT));
                    tma_load_2d(st, map, kg * PK, job.y, &full[s]);
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        bulk_g2s(st + C::TA + C::TB + r * C::NT * 32 * K,
                                 b + ((size_t) (kg * 4 + r) * a.ntn + tl.nb * C::NT) * (32 * K), C::NT * 32 * K, &full[s]);
                }
            }
            // every issued copy lands before the CTA may exit
            const long long first = it > C::NST ? it - C::NST : 0;
            for (long long k = first; k < it; ++k)
                if (!mbar_wait_bounded(&full[k % C::NST], (uint32_t) ((k / C::NST) & 1))) { atomicOr(a.err, ERR_TIMEOUT_FULL); break; }
        }
    }
    else if (warp == W_MMA)
    {
        if (lane == 0)
        {
            long long it = 0;
            int lt = 0;
            for (long long t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x, ++lt)
            {
                if (!mbar_wait_bounded(tempty, (uint32_t) ((lt & 1) ^ 1))) { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; break; }
                tc_fence_after();
                bool ok = true;
                for (int ks = 0; ks < nks; ++ks, ++it)
                {
                    const int s = (int) (it % C::NST);
                    const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
                    if (!mbar_wait_bounded(&full[s], ph) || !mbar_wait_bounded(&dec[s], ph))
                    {
                        atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; ok = false; break;
                    }
                    tc_fence_after();
                    uint8_t* st = stage(s);
                    // 128-input block b of the tile accumulates into chain b % CH; its first stage starts the chain
                    const int blk = ks >> 1, ch = blk % C::CH;
                    const bool acc = blk >= C::CH || (ks & 1);
                    const uint32_t sa = smem_u32(st), sb = smem_u32(st + C::TA);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16(tmem + (uint32_t) (ch * TN), umma_desc(sa + kk * 32, 16, 1024, 2),
                                 umma_desc(sb + kk * 256, 128, 1024, 0), idesc_f16(TN), acc || kk != 0);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(tfull);
            }
            // all issued MMAs complete before the tensor memory is released
            umma_commit(fin);
            if (!mbar_wait_bounded(fin, 0)) atomicOr(a.err, ERR_TIMEOUT_FULL);
        }
    }
    else if (warp < C::W_EPI0)
    {
        // decoders: warp d owns n-tiles d, d + 8, ... of the column block; per stage it decodes their 4 k-tiles
        constexpr int TPW = 4 * C::NT / C::NDEC;       // tiles per decoder warp and stage: tile u = d + NDEC i
        static_assert(TPW >= 1 && (4 * C::NT) % C::NDEC == 0, "decoder split");
        const int d = warp - W_DEC0;
        LaneDecode<K> L;
        L.init(lane);
        // stmatrix row address of this lane: matrix j = lane / 8 (0: n 0-7 k 0-7, 1: n 8-15 k 0-7, 2: n 0-7 k 8-15,
        // 3: n 8-15 k 8-15), row = lane % 8; K-major interleaved B: 8-row groups 1024 B apart, 16-byte k-chunks 128 B,
        // the stage's k-tile kt 256 B further
        const int j = lane >> 3;
        uint32_t boff[TPW], toff[TPW];
#pragma unroll
        for (int i = 0; i < TPW; ++i)
        {
            const int u = d + C::NDEC * i, nt = u % C::NT, kt = u / C::NT;
            const int n = 16 * nt + (lane & 7) + 8 * (j & 1);
            boff[i] = (uint32_t) ((n >> 3) * 1024 + (j >> 1) * 128 + (n & 7) * 16 + kt * 256);
            toff[i] = (uint32_t) ((kt * C::NT + nt) * (32 * K));
        }
        long long it = 0;
        for (long long t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x)
        {
            for (int ks = 0; ks < nks; ++ks, ++it)
            {
                const int s = (int) (it % C::NST);
                const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
                if (!mbar_wait_bounded(&full[s], ph)) { atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; }
                if (s_abort) break;
                uint8_t* st = stage(s);
                const uint8_t* tr = st + C::TA + C::TB;
                const uint32_t sb = smem_u32(st + C::TA);
                // all loads first, then independent decode chains, then the stores
                uint32_t hw[TPW], lw[TPW], frag[TPW][4];
#pragma unroll
                for (int i = 0; i < TPW; ++i)
                {
                    hw[i] = lds32(tr + toff[i] + L.off_hi);
                    lw[i] = lds32(tr + toff[i] + L.off_lo);
                }
#pragma unroll
                for (int i = 0; i < TPW; ++i) decode_frag_nat<K>(hw[i], lw[i], L, frag[i]);
#pragma unroll
                for (int i = 0; i < TPW; ++i) stmatrix_x4(sb + boff[i], frag[i]);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&dec[s]);
            }
        }
    }
    else
    {
        const int q = warp & 3;              // tensor-memory lane quarter this warp may read
        const int half = (warp - C::W_EPI0) >> 2;   // two warps per quarter, each drains half of the columns
        const int chains = nks / 2 < C::CH ? nks / 2 : C::CH;
        int lt = 0;
        for (long long t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x, ++lt)
        {
            if (!mbar_wait_bounded(tfull, (uint32_t) (lt & 1))) { atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; break; }
            tc_fence_after();
            const PfTile tl = pf_tile(t, NB, NP, KS);
            const int4 job = a.jobs[tl.job];
            float* yout = a.yraw + (size_t) tl.ks * a.split_stride;
            const int r = 32 * q + lane;
            const bool valid = r < job.z;
            const size_t row = (size_t) job.y + r;
            const uint32_t tq = tmem + ((uint32_t) (32 * q) << 16);
            for (int c = half * (TN / 32); c < (half + 1) * (TN / 32); ++c)
            {
                // the chains' 16 columns are loaded together and waited for once, then added in chain order
                uint32_t v[C::CH][16];
#pragma unroll
                for (int ch = 0; ch < C::CH; ++ch)
                    if (ch < chains) tmem_ld16(tq + (uint32_t) (ch * TN + c * 16), v[ch]);
                tmem_wait_ld();
                float f[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) f[u] = __uint_as_float(v[0][u]);
#pragma unroll
                for (int ch = 1; ch < C::CH; ++ch)
                    if (ch < chains)
                    {
#pragma unroll
                        for (int u = 0; u < 16; ++u) f[u] = __fadd_rn(f[u], __uint_as_float(v[ch][u]));
                    }
                if (valid)
                {
                    float4* dst = reinterpret_cast<float4*>(yout + (row * a.nslot + a.slot0 + tl.p) * a.ndim + tl.nb * TN + c * 16);
#pragma unroll
                    for (int u = 0; u < 4; ++u) dst[u] = make_float4(f[4 * u], f[4 * u + 1], f[4 * u + 2], f[4 * u + 3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t) C::TMEM_COLS) : "memory");
    }
}

// ---- gate/up epilogue: raw g, u -> out_block, SiLU*up, down input transform (fp16, natural order) ----
struct EpiPfArgs
{
    const Plan* plan;
    int I;
    const int* row_expert;
    const float* yraw;                  // [ksplit][R][2][I] partial sums of the K splits
    int ksplit; size_t split_stride;
    const __half* svh_g; const __half* svh_u; const __half* suh_d;
    float act_limit;
    __half* xd;                         // [R][I]
};

__global__ void __launch_bounds__(256) epi_pf_kernel(EpiPfArgs a)
{
    const int nbk = a.I / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int row = (int) (wid / nbk);
    if (row >= a.plan->R) return;
    const int nb = (int) (wid % nbk);
    const int e = a.row_expert[row];
    const size_t cb = (size_t) e * a.I + nb * 128;
    // every partial is read once: issue all the loads (streaming), then add the splits in order
    float gp[PF_KSPLIT][4], up[PF_KSPLIT][4];
#pragma unroll
    for (int s = 0; s < PF_KSPLIT; ++s)
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const size_t o = s * a.split_stride + (size_t) row * 2 * a.I + nb * 128 + lane + 32 * q;
            gp[s][q] = s < a.ksplit ? __ldcs(a.yraw + o) : 0.0f;
            up[s][q] = s < a.ksplit ? __ldcs(a.yraw + o + a.I) : 0.0f;
        }
    float gv[4], uv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        float g = gp[0][q], u = up[0][q];
#pragma unroll
        for (int s = 1; s < PF_KSPLIT; ++s)
            if (s < a.ksplit) { g = __fadd_rn(g, gp[s][q]); u = __fadd_rn(u, up[s][q]); }
        gv[q] = r16(g);
        uv[q] = r16(u);
    }
    had128_warp(gv, lane);
    had128_warp(uv, lane);
    float av[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        const int c = lane + 32 * q;
        const float gq = r16(__fmul_rn(__fmul_rn(gv[q], HAD), __half2float(a.svh_g[cb + c])));
        const float uq = r16(__fmul_rn(__fmul_rn(uv[q], HAD), __half2float(a.svh_u[cb + c])));
        av[q] = __fmul_rn(r16(act_mul(gq, uq, a.act_limit)), __half2float(a.suh_d[cb + c]));
    }
    had128_warp(av, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        const int c = lane + 32 * q;
        a.xd[(size_t) row * a.I + nb * 128 + c] = __float2half_rn(__fmul_rn(av[q], HAD));
    }
}

// ---- host side ------------------------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn)
    {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// row-major fp16 [rows, kdim] activations, boxes of 64 k x 128 rows with the 128-byte swizzle
cudaError_t act_map(CUtensorMap* m, const void* base, int kdim, int rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = { (cuuint64_t) kdim, (cuuint64_t) (rows > 0 ? rows : 1) };
    const cuuint64_t strides[1] = { (cuuint64_t) kdim * 2 };
    const cuuint32_t box[2] = { (cuuint32_t) PK, (cuuint32_t) PM };
    const cuuint32_t es[2] = { 1, 1 };
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

// The GEMV kernels' view of one trellis tensor [k x n]: rows of k-tiles, each ntn tiles of 32 * bits bytes, as 32-bit
// words; boxes of 8 consecutive k-tile rows x 8 tiles (one stage of one 128-column item).
cudaError_t trellis_map(CUtensorMap* m, const void* base, int k, int n, int bits)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int tb = 32 * bits, ntn = n / 16, kt = k / 16;
    const cuuint64_t dims[2] = { (cuuint64_t) ntn * tb / 4, (cuuint64_t) kt };
    const cuuint64_t strides[1] = { (cuuint64_t) ntn * tb };
    const cuuint32_t box[2] = { (cuuint32_t) (8 * tb / 4), 8u };
    const cuuint32_t es[2] = { 1, 1 };
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {

template <int K, int TN>
cudaError_t launch_gemm_pf(const Layer& L, const CUtensorMap& m0, const CUtensorMap& m1, const PfArgs& a, long long max_tiles,
                           cudaStream_t st)
{
    using C = CfgP<K, TN>;
    static bool attr_set[64] = {};
    static int sms[64] = {};
    if (!attr_set[L.device])
    {
        cudaError_t e = cudaFuncSetAttribute(gemm_pf_kernel<K, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (cudaDeviceGetAttribute(&sms[L.device], cudaDevAttrMultiProcessorCount, L.device) != cudaSuccess || sms[L.device] <= 0)
            sms[L.device] = 148;
        attr_set[L.device] = true;
    }
    const long long grid = max_tiles < sms[L.device] ? max_tiles : sms[L.device];
    if (grid <= 0) return cudaSuccess;
    gemm_pf_kernel<K, TN><<<(unsigned) grid, C::THREADS, C::SMEM, st>>>(m0, m1, a);
    return cudaGetLastError();
}

// tile width for a projection of width n
int pf_tile_n(int n) { return n % 256 == 0 ? 256 : 128; }

// one launch over jobs_max x (ndim / TN) x per_job tiles (per_job: projections x K splits)
cudaError_t launch_gemm_pf_bits(const Layer& L, int bits, const CUtensorMap& m0, const CUtensorMap& m1, const PfArgs& a,
                                long long jobs_max, long long per_job, cudaStream_t st)
{
    const int tn = pf_tile_n(a.ndim);
    const long long mt = jobs_max * (a.ndim / tn) * per_job;
    if (tn == 256)
        switch (bits)
        {
            case 2: return launch_gemm_pf<2, 256>(L, m0, m1, a, mt, st);
            case 3: return launch_gemm_pf<3, 256>(L, m0, m1, a, mt, st);
            default: return launch_gemm_pf<4, 256>(L, m0, m1, a, mt, st);
        }
    switch (bits)
    {
        case 2: return launch_gemm_pf<2, 128>(L, m0, m1, a, mt, st);
        case 3: return launch_gemm_pf<3, 128>(L, m0, m1, a, mt, st);
        default: return launch_gemm_pf<4, 128>(L, m0, m1, a, mt, st);
    }
}

}  // namespace

cudaError_t launch_prefill_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, void* out, int out_dtype,
                                   int accumulate, uint8_t* ws, const WsLayout& lay, cudaStream_t st, void* const* events,
                                   const HcOut* hc)
{
    auto mark = [&](int i) -> cudaError_t {
        if (events && events[i]) return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
        return cudaSuccess;
    };
    const Plan* plan = reinterpret_cast<const Plan*>(ws + lay.plan);
    const int rows = lay.rows_max;
    cudaError_t e;
    if (rows > 0)
    {
        if ((e = launch_prep_exact(L, x, x_dtype, ntok, topk, ws, lay, st, true)) != cudaSuccess) return e;
        if ((e = mark(2)) != cudaSuccess) return e;

        // upper bound of the jobs of <= 128 rows: every expert may end with a partial job
        const long long jobs_max = (long long) rows / PM + L.E_total;
        CUtensorMap mg, mu, md;
        if ((e = act_map(&mg, ws + lay.xg, L.H, rows)) != cudaSuccess) return e;
        if ((e = act_map(&mu, ws + lay.xu, L.H, rows)) != cudaSuccess) return e;
        if ((e = act_map(&md, ws + lay.xd, L.I, rows)) != cudaSuccess) return e;

        PfArgs g;
        g.plan = plan;
        g.jobs = reinterpret_cast<const int4*>(ws + lay.jobs);
        g.trellis = L.d_trellis;
        g.err = reinterpret_cast<int*>(ws + lay.err);
        g.proj0 = 0; g.nproj = 2; g.nslot = 2; g.slot0 = 0; g.kt = L.H / 16; g.ntn = L.I / 16; g.ndim = L.I;
        // split K (at most PF_KSPLIT ways) so that every split holds a whole number of 128-input blocks per accumulator
        // chain (2 chains at TN = 256, 4 at TN = 128): the most splits that divide, the shortest tensor-core chains
        const int nblk = L.H / 128, nch = pf_tile_n(L.I) == 256 ? 2 : 4;
        g.ksplit = 1;
        for (int ks = PF_KSPLIT; ks > 1; --ks)
            if (nblk % (ks * nch) == 0) { g.ksplit = ks; break; }
        g.split_stride = (size_t) rows * 2 * L.I;
        g.yraw = reinterpret_cast<float*>(ws + lay.yraw_gu);
        if (L.bits[0] == L.bits[1])
        {
            if ((e = launch_gemm_pf_bits(L, L.bits[0], mg, mu, g, jobs_max, 2 * g.ksplit, st)) != cudaSuccess) return e;
        }
        else
        {   // gate and up at different trellis widths: one launch each
            PfArgs g1 = g;
            g1.nproj = 1;
            if ((e = launch_gemm_pf_bits(L, L.bits[0], mg, mg, g1, jobs_max, g.ksplit, st)) != cudaSuccess) return e;
            g1.proj0 = 1; g1.slot0 = 1;
            if ((e = launch_gemm_pf_bits(L, L.bits[1], mu, mu, g1, jobs_max, g.ksplit, st)) != cudaSuccess) return e;
        }

        EpiPfArgs q;
        q.plan = plan; q.I = L.I;
        q.row_expert = reinterpret_cast<const int*>(ws + lay.row_expert);
        q.yraw = g.yraw; q.ksplit = g.ksplit; q.split_stride = g.split_stride;
        q.svh_g = reinterpret_cast<const __half*>(L.svh[0]);
        q.svh_u = reinterpret_cast<const __half*>(L.svh[1]);
        q.suh_d = reinterpret_cast<const __half*>(L.suh[2]);
        q.act_limit = L.act_limit;
        q.xd = reinterpret_cast<__half*>(ws + lay.xd);
        const long long w2 = (long long) rows * (L.I / 128);
        epi_pf_kernel<<<(unsigned) ((w2 + 7) / 8), 256, 0, st>>>(q);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if ((e = mark(3)) != cudaSuccess) return e;

        PfArgs d = g;
        d.proj0 = 2; d.nproj = 1; d.nslot = 1; d.slot0 = 0; d.kt = L.I / 16; d.ntn = L.H / 16; d.ndim = L.H;
        d.ksplit = 1; d.split_stride = 0;
        d.yraw = reinterpret_cast<float*>(ws + lay.yrow);
        if ((e = launch_gemm_pf_bits(L, L.bits[2], md, md, d, jobs_max, 1, st)) != cudaSuccess) return e;
        if ((e = mark(4)) != cudaSuccess) return e;
    }
    else
    {
        for (int i = 2; i <= 4; ++i)
            if ((e = mark(i)) != cudaSuccess) return e;
    }
    if (ntok > 0)
        if ((e = launch_combine_raw(L, reinterpret_cast<const float*>(ws + lay.yrow), ntok, topk, out, out_dtype, accumulate, ws,
                                    lay, st, hc)) != cudaSuccess)
            return e;
    return mark(5);
}

}  // namespace glmx
