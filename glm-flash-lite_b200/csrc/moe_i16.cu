// Routed-expert MoE layer in I16 mode: the reference's int16-activation decode mode (kernels/cpu_avx2/ft_core.h:418-598,
// the mode tier_forward / local_forward pick for decode, ft_tier_ext.cpp:396, 899-901), bit-identical to it.
//
// Arithmetic of one linear (restated from quant_block_i16, tile_accum_i16 and gemv_block_i16):
//   per 128-input block b: xt = fp16(had128(x * suh) * HAD); sc_b = amax / 16383; xi = nearbyint(xt / sc_b) (|xi| <= 16383);
//   sumx = ((0 + float(sum xi_0) * sc_0) + float(sum xi_1) * sc_1) + ...
//   per output column n and tile-row class c in {rows 0,2,4,6 | 1,3,5,7 | 8,10,12,14 | 9,11,13,15} of every 16-row tile:
//     I_{b,c} = sum over block b's rows of class c of bytesum(state) * xi (exact int32)
//     a_c = fma(float(I_{b,c}), sc_b, a_c) for b = 0, 1, ...          (one fp32 FMA chain per class, in block order)
//   y_n = KINV * ((a_0 + a_1) + (a_2 + a_3)) + CAFF * sumx            (KINV * lo and CAFF * sumx rounded separately)
//
// On the GPU the integer sums run on the tensor cores: one mma.m16n8k32 (u8 x s8 -> s32) per class and pair of tiles,
// A = the lane's product words x_j = state * MUL1 (their 4 bytes sum to bytesum), B = the activation's two signed
// byte planes (xi = 256 * hi + lo) replicated over the 4 bytes of the matching word, N = 4 tokens x 2 planes so a lane
// gets (hi, lo) of its own token and recombines them exactly. Every float operation is the reference's, in its order.
//
// Kernels: prep_i16 (input transform + quantisation into the replicated B layout), gemv_i16<gate+up> -> raw y,
// epi_gu_i16 (out_block, SiLU*up, down input transform + quantisation), gemv_i16<down> -> raw y, combine_i16 (down
// out_block + weighted sum in pick order + shared expert).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int RB = 8;                  // tile rows per stage = one 128-input block
constexpr int NW = 8;                  // consumer warps = 16-column n-tiles per item (128 columns)
constexpr int NTHR = (NW + 1) * 32;
#ifndef GLMX_I16_CTAS
#define GLMX_I16_CTAS 2
#endif
#ifndef GLMX_I16_RING_KB
#define GLMX_I16_RING_KB (GLMX_I16_CTAS >= 3 ? 64 : 96)
#endif
// Two CTAs of 9 warps per SM: up to 113 registers a thread (no spills in the consumer loop) and a 4-stage gate+up ring;
// three CTAs (72 registers) measured 6 % slower on the gate+up GEMV at B = 64.
constexpr int CTAS = GLMX_I16_CTAS;                 // CTAs per SM
constexpr int RING = GLMX_I16_RING_KB * 1024;       // ring bytes per CTA

template <int K0, int K1, int NMAT>
struct CfgI
{
    static constexpr int TB0 = 32 * K0, TB1 = 32 * K1;
    static constexpr int ROW0 = NW * TB0, ROW1 = NW * TB1;
    static constexpr int MAT0 = RB * ROW0, MAT1 = NMAT > 1 ? RB * ROW1 : 0;
    static constexpr int ACT = NMAT * I16_ACT_BYTES;
    static constexpr int SC = NMAT * 16;
    static constexpr int BYTES = MAT0 + MAT1 + ACT + SC;                  // bytes copied into a stage
    static constexpr int STAGE = (BYTES + 127) / 128 * 128;                 // tensor copies land 128-byte aligned
    static constexpr int NST = RING / STAGE < 2 ? 2 : (RING / STAGE > 8 ? 8 : RING / STAGE);
    static constexpr int SMEM = NST * STAGE + 2 * NST * 8;
    static_assert(STAGE % 128 == 0 && MAT0 % 128 == 0 && (MAT0 + MAT1) % 16 == 0, "stage alignment");
};

struct GemvI16Args
{
    const Plan* plan;
    const int4* jobs;
    const uint64_t* trellis;
    const CUtensorMap* tmaps;       // [E_total][3]: each trellis tensor as rows of k-tiles (boxes of 8 rows x 8 tiles)
    int proj0, nmat;
    int kt, ntn, ndim;              // k-tiles, n-tiles, output dim
    const uint8_t* actb;            // [J][kt/8] records of i16_rec_bytes(nmat): planes of each projection, then scales
    const float* psum;              // [R][nmat][kt/8]
    float* yraw;                    // [R][nmat][ndim]
    int* err;
    // K split of small calls (gate+up, at most I16_SPLIT_MAX_ROWS rows): each split stores its exact int32 class sums
    // per 128-input block, isum [R][nmat][kt/8][ndim][4 classes]; the last split of a (job, column block) to arrive
    // (counters [J][ndim/128], cleared by the route kernel) runs the per-class fp32 chains in block order
    int* isum;
    int* counters;
    int* next;                      // item counter (zeroed by the route kernel): CTAs take items as they free up
};

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory"); }

// y of one (row, projection, column) from its exact block sums: the four class chains a_c = fma(float(I_b,c), sc_b,
// a_c) in block order, then KINV * ((a0 + a1) + (a2 + a3)) + CAFF * sumx, as the unsplit kernel does
__device__ __forceinline__ float i16_finish(float a0, float a1, float a2, float a3, const float* ps, int nkb)
{
    const float kinv = __half2float(__ushort_as_half(KINV_BITS));
    const float caff = 1024.0f * kinv + __half2float(__ushort_as_half(KBIAS_BITS));
    float sumx = 0.0f;
    for (int kb0 = 0; kb0 < nkb; kb0 += 8)
    {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = kb0 + u < nkb ? __ldg(ps + kb0 + u) : 0.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (kb0 + u < nkb) sumx = __fadd_rn(sumx, v[u]);
    }
    const float lo = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    return __fadd_rn(__fmul_rn(kinv, lo), __fmul_rn(caff, sumx));
}

// The last split of a (job, column block): every (row slot, projection, column) of the block from the stored block
// sums. Kept out of line so its registers do not weigh on the main loop's allocation.
__device__ __noinline__ void i16_chain_item(const GemvI16Args& a, int4 job, int j, int nbi, int nmat, int nkb, int tid)
{
    for (int idx = tid; idx < job.z * nmat * 128; idx += NW * 32)
    {
        const int slot = idx / (nmat * 128), m = (idx / 128) % nmat, col = nbi * 128 + idx % 128;
        const int row = job.y + slot;
        const int4* src = reinterpret_cast<const int4*>(a.isum) + (((size_t) row * nmat + m) * nkb) * a.ndim + col;
        const size_t rec = i16_rec_bytes(nmat);
        const float* scl = reinterpret_cast<const float*>(a.actb + (size_t) j * nkb * rec + nmat * I16_ACT_BYTES) + m * 4 + slot;
        float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
        for (int kb0 = 0; kb0 < nkb; kb0 += 4)
        {
            int4 v[4];
            float sc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (kb0 + u < nkb) { v[u] = __ldcg(src + (size_t) (kb0 + u) * a.ndim); sc[u] = __ldg(scl + (kb0 + u) * (rec / 4)); }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (kb0 + u < nkb)
                {
                    c0 = __fmaf_rn(__int2float_rn(v[u].x), sc[u], c0);
                    c1 = __fmaf_rn(__int2float_rn(v[u].y), sc[u], c1);
                    c2 = __fmaf_rn(__int2float_rn(v[u].z), sc[u], c2);
                    c3 = __fmaf_rn(__int2float_rn(v[u].w), sc[u], c3);
                }
        }
        a.yraw[((size_t) row * nmat + m) * a.ndim + col] = i16_finish(c0, c1, c2, c3, a.psum + ((size_t) row * nmat + m) * nkb, nkb);
    }
}

template <int K0, int K1, int NMAT, bool SPLIT>
__global__ void __launch_bounds__(NTHR, CTAS) gemv_i16_kernel(GemvI16Args a)
{
    pdl_enter();
    using C = CfgI<K0, K1, NMAT>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NST * C::STAGE);
    uint64_t* empty = full + C::NST;
    __shared__ volatile int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0)
    {
        for (int s = 0; s < C::NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], NW); }
        s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const Plan pl = *a.plan;
    const int nb = a.ntn / NW;
    const int nkb = a.kt / RB;
    const int S = SPLIT ? pl.S_gu : 1;                                       // K splits (item = (job, block, split))
    const int kbs = nkb / S;                                                 // blocks per split
    const long long items = (long long) pl.J * nb * S;
    __shared__ int s_last;
    // Items are taken from a global counter as CTAs free up (the co-resident CTAs of an SM progress at unequal rates,
    // so a fixed share per CTA leaves stragglers); the producer writes each item's id into the slot of its first stage
    // and, after the last item, an end marker (-1) in one more slot completed with a plain arrival.
    __shared__ int s_item[C::NST];

    if (warp == NW)
    {
        if (lane != 0) return;
        long long it = 0;
        for (;;)
        {
            const long long item = s_abort ? items : (long long) atomicAdd(a.next, 1);
            if (item >= items) break;
            const int ks = (int) (item % S);
            const long long jn = item / S;
            const int nbi = (int) (jn % nb), j = (int) (jn / nb);
            const int4 job = a.jobs[j];
            const CUtensorMap* m0 = a.tmaps + job.x * 3 + a.proj0;
            for (int kb = ks * kbs; kb < (ks + 1) * kbs; ++kb, ++it)
            {
                const int s = (int) (it % C::NST);
                const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
                if (!s_abort && !mbar_wait_bounded(&empty[s], ph ^ 1u)) { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; }
                if (s_abort) break;
                uint8_t* st = ring + s * C::STAGE;
                s_item[s] = (int) item;
                mbar_arrive_expect_tx(&full[s], (uint32_t) C::BYTES);
                // the stage's RB k-tile rows x NW tiles of each matrix: one tensor copy (x in 32-bit words)
                tma_load_2d(st, m0, nbi * NW * C::TB0 / 4, kb * RB, &full[s]);
                if (NMAT > 1) tma_load_2d(st + C::MAT0, m0 + 1, nbi * NW * C::TB1 / 4, kb * RB, &full[s]);
                // the block's activation record (every projection's planes, then their scales): one copy
                bulk_g2s(st + C::MAT0 + C::MAT1, a.actb + ((size_t) j * nkb + kb) * (C::ACT + C::SC), C::ACT + C::SC, &full[s]);
            }
        }
        if (!s_abort)
        {
            const int s = (int) (it % C::NST);
            if (mbar_wait_bounded(&empty[s], (uint32_t) (((it / C::NST) & 1) ^ 1)))
            {
                s_item[s] = -1;
                mbar_arrive(&full[s]);
                ++it;
            }
            else { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; }
        }
        const long long first = it > C::NST ? it - C::NST : 0;
        for (long long k = first; k < it; ++k)
            if (!mbar_wait_bounded(&full[k % C::NST], (uint32_t) ((k / C::NST) & 1))) { atomicOr(a.err, ERR_TIMEOUT_FULL); break; }
        return;
    }

    LaneDecode<K0> L0;
    L0.init(lane);
    LaneDecode<K1> L1;
    L1.init(lane);
    const int g = lane >> 2, tq = lane & 3;
    long long it = 0;
    for (;;)
    {
        // the next item: its id is in the slot of its first stage
        {
            const int s = (int) (it % C::NST);
            if (!s_abort && !mbar_wait_bounded(&full[s], (uint32_t) ((it / C::NST) & 1))) { atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; }
        }
        if (s_abort) break;
        const int item_id = s_item[it % C::NST];
        if (item_id < 0) break;
        const long long item = item_id;
        const int ks = (int) (item % S);
        const long long jn = item / S;
        const int nbi = (int) (jn % nb), j = (int) (jn / nb);
        const int4 job = a.jobs[j];
        float accf[NMAT][4][2];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int c = 0; c < 4; ++c) accf[m][c][0] = accf[m][c][1] = 0.0f;

        for (int kb = ks * kbs; kb < (ks + 1) * kbs; ++kb, ++it)
        {
            const int s = (int) (it % C::NST);
            const uint32_t ph = (uint32_t) ((it / C::NST) & 1);
            if (kb != ks * kbs && !s_abort && !mbar_wait_bounded(&full[s], ph)) { atomicOr(a.err, ERR_TIMEOUT_FULL); s_abort = 1; }
            const uint8_t* st = ring + s * C::STAGE;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
            {
                const uint8_t* mat = st + (m == 0 ? 0 : C::MAT0);
                const int row_bytes = m == 0 ? C::ROW0 : C::ROW1;
                const int tb = m == 0 ? C::TB0 : C::TB1;
                const uint8_t* act = st + C::MAT0 + C::MAT1 + m * I16_ACT_BYTES + lane * 16;
                int acc[4][4];
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0;
#pragma unroll
                for (int p = 0; p < 4; ++p)
                {
                    uint32_t xa[8], xb[8];
                    if (m == 0)
                    {
                        decode_words<K0>(mat + (2 * p) * row_bytes + warp * tb, L0, xa);
                        decode_words<K0>(mat + (2 * p + 1) * row_bytes + warp * tb, L0, xb);
                    }
                    else
                    {
                        decode_words<K1>(mat + (2 * p) * row_bytes + warp * tb, L1, xa);
                        decode_words<K1>(mat + (2 * p + 1) * row_bytes + warp * tb, L1, xb);
                    }
#pragma unroll
                    for (int ch = 0; ch < 2; ++ch)
                    {
                        // the B fragments of classes 2ch and 2ch + 1: one 16-byte load
                        const uint4 bb = *reinterpret_cast<const uint4*>(act + (p * 2 + ch) * 512);
                        imma_u8s8(acc[2 * ch], xa[2 * ch], xa[2 * ch + 4], xb[2 * ch], xb[2 * ch + 4], bb.x, bb.y);
                        imma_u8s8(acc[2 * ch + 1], xa[2 * ch + 1], xa[2 * ch + 5], xb[2 * ch + 1], xb[2 * ch + 5], bb.z, bb.w);
                    }
                }
                if (SPLIT)      // also for S = 1: one epilogue form per variant keeps the split variant's registers low
                {
                    // exact class sums of this block for row slot tq, columns g and g + 8 of the warp's n-tile
                    if (tq < job.z)
                    {
                        int* dst = a.isum + ((((size_t) (job.y + tq) * NMAT + m) * nkb + kb) * a.ndim + nbi * 128 + warp * 16 + g) * 4;
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            __stcg(reinterpret_cast<int4*>(dst + 32 * h),
                                   make_int4(acc[0][2 * h] * 256 + acc[0][2 * h + 1], acc[1][2 * h] * 256 + acc[1][2 * h + 1],
                                             acc[2][2 * h] * 256 + acc[2][2 * h + 1], acc[3][2 * h] * 256 + acc[3][2 * h + 1]));
                    }
                }
                else
                {
                    const float sc = *reinterpret_cast<const float*>(st + C::MAT0 + C::MAT1 + C::ACT + m * 16 + tq * 4);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                        {
                            const int v = acc[c][2 * h] * 256 + acc[c][2 * h + 1];     // exact: |v| < 2^30
                            accf[m][c][h] = __fmaf_rn(__int2float_rn(v), sc, accf[m][c][h]);
                        }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (SPLIT)
        {
            // the last split of this (job, column block) to arrive chains every block's sums, in block order
            __threadfence();
            consumers_sync();
            if (tid == 0) s_last = atomicAdd(a.counters + jn, 1) == S - 1;
            consumers_sync();
            if (!s_last) continue;
            __threadfence();
            i16_chain_item(a, job, j, nbi, NMAT, nkb, tid);
            continue;
        }
        if (tq < job.z)
        {
            const int row = job.y + tq;
            const float kinv = __half2float(__ushort_as_half(KINV_BITS));
            const float caff = 1024.0f * kinv + __half2float(__ushort_as_half(KBIAS_BITS));
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
            {
                const float* ps = a.psum + ((size_t) row * NMAT + m) * nkb;
                float sumx = 0.0f;
                // the loads are independent: fetch 8 at a time, then fold them in block order
                for (int kb0 = 0; kb0 < nkb; kb0 += 8)
                {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = kb0 + u < nkb ? __ldg(ps + kb0 + u) : 0.0f;
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (kb0 + u < nkb) sumx = __fadd_rn(sumx, v[u]);
                }
                const float t1 = __fmul_rn(caff, sumx);
#pragma unroll
                for (int h = 0; h < 2; ++h)
                {
                    const float lo = __fadd_rn(__fadd_rn(accf[m][0][h], accf[m][1][h]), __fadd_rn(accf[m][2][h], accf[m][3][h]));
                    a.yraw[((size_t) row * NMAT + m) * a.ndim + nbi * 128 + warp * 16 + g + 8 * h] = __fadd_rn(__fmul_rn(kinv, lo), t1);
                }
            }
        }
    }
}

// ---- quantisation of one 128-block held by a warp (v[q] = element lane + 32 q) into the replicated B layout ----
// Layout of one (job, projection, block): [pair p 0..3][class pair c / 2][lane 0..31][class c % 2][b0, b1] 32-bit words
// (a lane's fragments of two classes are one 16-byte load); lane
// (g, tq) holds, for token slot g/2 and plane g%2 (0 = hi, 1 = lo), the plane byte of block row 16*(2p + b) + 2tq + off_c
// (off = 0, 1, 8, 9) replicated into the four bytes of word b.
__device__ __forceinline__ void quantise_block(float v[4], int lane, int slot, uint8_t* actb_blk, float* sc_slot, float* psum_out)
{
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = amax > 0.0f ? __fdiv_rn(amax, 16383.0f) : 1.0f;
    const float rs = __fdiv_rn(1.0f, sc);
    int si = 0;
    uint32_t* words = reinterpret_cast<uint32_t*>(actb_blk);
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        const int xi = __float2int_rn(__fmul_rn(v[q], rs));
        si += xi;
        const int lo = ((xi + 128) & 255) - 128;
        const int hi = (xi - lo) >> 8;
        const int rb = lane + 32 * q;                      // row within the block
        const int tt = rb >> 4, r = rb & 15;
        const int p = tt >> 1, b = tt & 1;
        const int c = (r & 1) | ((r >> 3) << 1);
        const int tqd = (r & 7) >> 1;
        const int l_hi = (2 * slot) * 4 + tqd, l_lo = (2 * slot + 1) * 4 + tqd;
        words[(((p * 2 + (c >> 1)) * 32 + l_hi) * 2 + (c & 1)) * 2 + b] = ((uint32_t) hi & 0xffu) * 0x01010101u;
        words[(((p * 2 + (c >> 1)) * 32 + l_lo) * 2 + (c & 1)) * 2 + b] = ((uint32_t) lo & 0xffu) * 0x01010101u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) si += __shfl_xor_sync(0xffffffffu, si, o);
    if (lane == 0)
    {
        *sc_slot = sc;
        *psum_out = __fmul_rn((float) si, sc);
    }
}

struct PrepI16Args
{
    const Plan* plan;
    const void* x; int x_dtype; int H;
    const int* row_token; const int* row_expert; const int* row_job; const int4* jobs;
    const __half* suh_g; const __half* suh_u;
    uint8_t* actb; float* psum;
};

__device__ __forceinline__ float load_x(const void* x, int dt, size_t i)
{
    if (dt == GLMX_F16) return __half2float(reinterpret_cast<const __half*>(x)[i]);
    if (dt == GLMX_BF16) return r16(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]));
    return reinterpret_cast<const float*>(x)[i];
}

__global__ void __launch_bounds__(256) prep_i16_kernel(PrepI16Args a)
{
    pdl_enter();
    const int nbk = a.H / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int row = (int) (wid / (2 * nbk));
    if (row >= a.plan->R) return;
    const int rem = (int) (wid % (2 * nbk)), proj = rem / nbk, kb = rem % nbk;
    const int t = a.row_token[row], e = a.row_expert[row], j = a.row_job[row];
    const int slot = row - a.jobs[j].y;
    const __half* suh = (proj ? a.suh_u : a.suh_g) + (size_t) e * a.H + kb * 128;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        const int c = lane + 32 * q;
        v[q] = __fmul_rn(load_x(a.x, a.x_dtype, (size_t) t * a.H + kb * 128 + c), __half2float(suh[c]));
    }
    had128_warp(v, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = r16(__fmul_rn(v[q], HAD));
    uint8_t* rec = a.actb + ((size_t) j * nbk + kb) * i16_rec_bytes(2);
    quantise_block(v, lane, slot, rec + proj * I16_ACT_BYTES, reinterpret_cast<float*>(rec + 2 * I16_ACT_BYTES) + proj * 4 + slot,
                   a.psum + ((size_t) row * 2 + proj) * nbk + kb);
}

struct EpiGuArgs
{
    const Plan* plan;
    int I;
    const int* row_expert; const int* row_job; const int4* jobs;
    const float* yraw;                  // [R][2][I]
    const __half* svh_g; const __half* svh_u; const __half* suh_d;
    float act_limit;
    uint8_t* actb; float* psum;                  // down input: records [J][I/128] of i16_rec_bytes(1)
};

__global__ void __launch_bounds__(256) epi_gu_i16_kernel(EpiGuArgs a)
{
    pdl_enter();
    const int nbk = a.I / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int row = (int) (wid / nbk);
    if (row >= a.plan->R) return;
    const int nb = (int) (wid % nbk);
    const int e = a.row_expert[row], j = a.row_job[row];
    const int slot = row - a.jobs[j].y;
    const size_t cb = (size_t) e * a.I + nb * 128;
    float gv[4], uv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        gv[q] = r16(a.yraw[((size_t) row * 2 + 0) * a.I + nb * 128 + lane + 32 * q]);
        uv[q] = r16(a.yraw[((size_t) row * 2 + 1) * a.I + nb * 128 + lane + 32 * q]);
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
    for (int q = 0; q < 4; ++q) av[q] = r16(__fmul_rn(av[q], HAD));
    uint8_t* rec = a.actb + ((size_t) j * nbk + nb) * i16_rec_bytes(1);
    quantise_block(av, lane, slot, rec, reinterpret_cast<float*>(rec + I16_ACT_BYTES) + slot, a.psum + (size_t) row * nbk + nb);
}

struct CombineI16Args
{
    const Plan* plan;
    const int* pick_row; const float* row_weight; const int* row_expert;
    const float* yraw;                  // [R][H] raw down outputs
    const __half* svh_d;
    int H, ntok, topk, has_shared, E;
    void* out; int out_dtype; int accumulate;
    HcOut hc;                           // hc.x != nullptr: hyper-connection epilogue instead of writing out
};

// the combined value of token t, columns hb*128 + lane + 32q: hyper-connection update, expert-parallel return to the
// token's owner rank, or (accumulating) store
__device__ __forceinline__ void combine_store(const CombineI16Args& a, int t, int hb, int lane, const float acc[4])
{
    if (a.hc.peer.recv)
    {
        const PeerOut& p = a.hc.peer;
        float* dst = peer_row(p.recv, p.rank, p.world, p.rpr, p.seq, t, a.H) + hb * 128 + lane;
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[32 * q] = acc[q];
        return;
    }
    if (a.hc.x)
    {
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const float y = a.hc.y_half ? __half2float(__float2half_rn(acc[q])) : acc[q];
            hc_apply_col(a.hc.x + (size_t) t * 4 * a.H, a.H, hb * 128 + lane + 32 * q, y, a.hc.post + (size_t) t * 4,
                         a.hc.comb + (size_t) t * 16);
        }
        return;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
    {
        const size_t o = (size_t) t * a.H + hb * 128 + lane + 32 * q;
        if (a.out_dtype == GLMX_F32)
        {
            float* p = reinterpret_cast<float*>(a.out) + o;
            *p = a.accumulate ? __fadd_rn(*p, acc[q]) : acc[q];
        }
        else
        {
            __half* p = reinterpret_cast<__half*>(a.out) + o;
            *p = __float2half_rn(a.accumulate ? __fadd_rn(__half2float(*p), acc[q]) : acc[q]);
        }
    }
}

// one warp per (token, 128-output block): down out_block per pick, weighted sum in pick order (+ shared)
__global__ void __launch_bounds__(256) combine_i16_kernel(CombineI16Args a)
{
    pdl_enter();
    const int nbk = a.H / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int t = (int) (wid / nbk);
    const int hb = (int) (wid % nbk);
    float acc[4] = { 0.f, 0.f, 0.f, 0.f };
    const int nk = t < a.ntok ? a.topk + (a.has_shared ? 1 : 0) : 0;
    for (int k = 0; k < nk; ++k)
    {
        int r;
        float w;
        if (k < a.topk)
        {
            r = a.pick_row[t * a.topk + k];
            if (r < 0) continue;
            w = a.row_weight[r];
        }
        else { r = a.plan->P + t; w = 1.0f; }
        const int e = k < a.topk ? a.row_expert[r] : a.E;
        float y[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) y[q] = r16(a.yraw[(size_t) r * a.H + hb * 128 + lane + 32 * q]);
        had128_warp(y, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const int c = hb * 128 + lane + 32 * q;
            const float yq = r16(__fmul_rn(__fmul_rn(y[q], HAD), __half2float(a.svh_d[(size_t) e * a.H + c])));
            acc[q] = k < a.topk ? __fadd_rn(acc[q], __fmul_rn(w, yq)) : __fadd_rn(acc[q], yq);
        }
    }
    if (t < a.ntok) combine_store(a, t, hb, lane, acc);
    if (a.hc.peer.recv) peer_done(a.hc.peer.recv, a.hc.peer.flags, a.hc.peer.counter, a.hc.peer.rank, a.hc.peer.world, a.hc.peer.seq);
}

// Small batches: one CTA per (token, 128-output block), one warp per pick computing its weighted down out_block into
// shared memory; warp 0 then adds the picks in pick order (the same fp32 operations as combine_i16_kernel, in the
// same order), so the picks' transforms run side by side instead of one after another.
constexpr int COMBINE_MAXK = 65;           // topk <= 64, plus the shared expert
constexpr int COMBINE_WIDE_MAX_TOKENS = 32;
__global__ void __launch_bounds__(256) combine_wide_kernel(CombineI16Args a)
{
    pdl_enter();
    __shared__ float ys[COMBINE_MAXK][128];
    __shared__ int valid[COMBINE_MAXK];
    const int nbk = a.H / 128;
    const int t = blockIdx.x / nbk, hb = blockIdx.x % nbk;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = a.topk + (a.has_shared ? 1 : 0);
    for (int k = warp; k < nk; k += 8)
    {
        int r;
        float w = 1.0f;
        if (k < a.topk)
        {
            r = a.pick_row[t * a.topk + k];
            if (r < 0)
            {
                if (lane == 0) valid[k] = 0;
                continue;
            }
            w = a.row_weight[r];
        }
        else r = a.plan->P + t;
        const int e = k < a.topk ? a.row_expert[r] : a.E;
        float y[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) y[q] = r16(a.yraw[(size_t) r * a.H + hb * 128 + lane + 32 * q]);
        had128_warp(y, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const int c = hb * 128 + lane + 32 * q;
            const float yq = r16(__fmul_rn(__fmul_rn(y[q], HAD), __half2float(a.svh_d[(size_t) e * a.H + c])));
            ys[k][lane + 32 * q] = k < a.topk ? __fmul_rn(w, yq) : yq;
        }
        if (lane == 0) valid[k] = 1;
    }
    __syncthreads();
    if (warp == 0)
    {
        float acc[4] = { 0.f, 0.f, 0.f, 0.f };
        for (int k = 0; k < nk; ++k)
            if (valid[k])
            {
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[q] = __fadd_rn(acc[q], ys[k][lane + 32 * q]);
            }
        combine_store(a, t, hb, lane, acc);
    }
    if (a.hc.peer.recv) peer_done(a.hc.peer.recv, a.hc.peer.flags, a.hc.peer.counter, a.hc.peer.rank, a.hc.peer.world, a.hc.peer.seq);
}

// the combine for ntok tokens: the wide form at decode sizes, one warp per (token, block) above
cudaError_t launch_combine(const CombineI16Args& c, int ntok, int H, cudaStream_t st)
{
    if (ntok <= COMBINE_WIDE_MAX_TOKENS)
        return launch_chained(combine_wide_kernel, dim3((unsigned) (ntok * (H / 128))), dim3(256), 0, st, c);
    else
    {
        const long long w3 = (long long) ntok * (H / 128);
        return launch_chained(combine_i16_kernel, dim3((unsigned) ((w3 + 7) / 8)), dim3(256), 0, st, c);
    }
}

}  // namespace

int i16_grid_ctas(const Layer& L)
{
    return gemv_sm_count(L) * CTAS;
}

namespace {

template <int K0, int K1, int NMAT, bool SPLIT>
cudaError_t launch_gemv_i16_v(const Layer& L, const GemvI16Args& a, cudaStream_t st)
{
    using C = CfgI<K0, K1, NMAT>;
    static bool attr_set[64] = {};
    if (!attr_set[L.device])
    {
        cudaError_t e = cudaFuncSetAttribute(gemv_i16_kernel<K0, K1, NMAT, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[L.device] = true;
    }
    return launch_chained(gemv_i16_kernel<K0, K1, NMAT, SPLIT>, dim3(i16_grid_ctas(L)), dim3(NTHR), C::SMEM, st, a);
}

// the K-split form only where its sums buffer exists (gate/up of calls with at most I16_SPLIT_MAX_ROWS rows)
template <int K0, int K1, int NMAT>
cudaError_t launch_gemv_i16(const Layer& L, const GemvI16Args& a, cudaStream_t st)
{
    if (NMAT == 2 && a.isum) return launch_gemv_i16_v<K0, K1, NMAT, NMAT == 2>(L, a, st);
    return launch_gemv_i16_v<K0, K1, NMAT, false>(L, a, st);
}

template <int K0>
cudaError_t launch_gu_i16_k0(const Layer& L, const GemvI16Args& a, cudaStream_t st)
{
    switch (L.bits[1])
    {
        case 2: return launch_gemv_i16<K0, 2, 2>(L, a, st);
        case 3: return launch_gemv_i16<K0, 3, 2>(L, a, st);
        default: return launch_gemv_i16<K0, 4, 2>(L, a, st);
    }
}

}  // namespace

cudaError_t launch_combine_raw(const Layer& L, const float* yraw, int ntok, int topk, void* out, int out_dtype, int accumulate,
                               uint8_t* ws, const WsLayout& lay, cudaStream_t st, const HcOut* hc)
{
    if (ntok <= 0) return cudaSuccess;
    CombineI16Args c;
    c.plan = reinterpret_cast<const Plan*>(ws + lay.plan);
    c.pick_row = reinterpret_cast<const int*>(ws + lay.pick_row);
    c.row_weight = reinterpret_cast<const float*>(ws + lay.row_weight);
    c.row_expert = reinterpret_cast<const int*>(ws + lay.row_expert);
    c.yraw = yraw;
    c.svh_d = reinterpret_cast<const __half*>(L.svh[2]);
    c.H = L.H; c.ntok = ntok; c.topk = topk; c.has_shared = L.has_shared; c.E = L.E;
    c.out = out; c.out_dtype = out_dtype; c.accumulate = accumulate;
    c.hc = hc ? *hc : HcOut{ nullptr, nullptr, nullptr, 0 };
    return launch_combine(c, ntok, L.H, st);
}

cudaError_t launch_i16_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, void* out, int out_dtype,
                               int accumulate, uint8_t* ws, const WsLayout& lay, cudaStream_t st, void* const* events,
                               const HcOut* hc)
{
    auto mark = [&](int i) -> cudaError_t {
        if (events && events[i]) return cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
        return cudaSuccess;
    };
    const Plan* plan = reinterpret_cast<const Plan*>(ws + lay.plan);
    const int rows = lay.rows_max;
    const int* row_token = reinterpret_cast<const int*>(ws + lay.row_token);
    const int* row_expert = reinterpret_cast<const int*>(ws + lay.row_expert);
    const int* row_job = reinterpret_cast<const int*>(ws + lay.row_job);
    const int4* jobs = reinterpret_cast<const int4*>(ws + lay.jobs);
    cudaError_t e;
    if (rows > 0)
    {
        PrepI16Args p;
        p.plan = plan; p.x = x; p.x_dtype = x_dtype; p.H = L.H;
        p.row_token = row_token; p.row_expert = row_expert; p.row_job = row_job; p.jobs = jobs;
        p.suh_g = reinterpret_cast<const __half*>(L.suh[0]);
        p.suh_u = reinterpret_cast<const __half*>(L.suh[1]);
        p.actb = ws + lay.actb_gu;
        p.psum = reinterpret_cast<float*>(ws + lay.psum_gu);
        const long long w1 = (long long) rows * 2 * (L.H / 128);
        if ((e = launch_chained(prep_i16_kernel, dim3((unsigned) ((w1 + 7) / 8)), dim3(256), 0, st, p)) != cudaSuccess) return e;
        if ((e = mark(2)) != cudaSuccess) return e;

        GemvI16Args g;
        g.plan = plan; g.jobs = jobs; g.trellis = L.d_trellis; g.tmaps = L.d_tmaps; g.err = reinterpret_cast<int*>(ws + lay.err);
        g.proj0 = 0; g.nmat = 2; g.kt = L.H / 16; g.ntn = L.I / 16; g.ndim = L.I;
        g.actb = ws + lay.actb_gu;
        g.psum = reinterpret_cast<const float*>(ws + lay.psum_gu);
        g.yraw = reinterpret_cast<float*>(ws + lay.yraw_gu);
        g.isum = rows <= I16_SPLIT_MAX_ROWS ? reinterpret_cast<int*>(ws + lay.isum_gu) : nullptr;
        g.counters = reinterpret_cast<int*>(ws + lay.cnt_gu);
        g.next = reinterpret_cast<int*>(ws + lay.plan + offsetof(Plan, next_gu));
        switch (L.bits[0])
        {
            case 2: e = launch_gu_i16_k0<2>(L, g, st); break;
            case 3: e = launch_gu_i16_k0<3>(L, g, st); break;
            default: e = launch_gu_i16_k0<4>(L, g, st); break;
        }
        if (e != cudaSuccess) return e;

        EpiGuArgs q;
        q.plan = plan; q.I = L.I; q.row_expert = row_expert; q.row_job = row_job; q.jobs = jobs;
        q.yraw = g.yraw;
        q.svh_g = reinterpret_cast<const __half*>(L.svh[0]);
        q.svh_u = reinterpret_cast<const __half*>(L.svh[1]);
        q.suh_d = reinterpret_cast<const __half*>(L.suh[2]);
        q.act_limit = L.act_limit;
        q.actb = ws + lay.actb_d;
        q.psum = reinterpret_cast<float*>(ws + lay.psum_d);
        const long long w2 = (long long) rows * (L.I / 128);
        if ((e = launch_chained(epi_gu_i16_kernel, dim3((unsigned) ((w2 + 7) / 8)), dim3(256), 0, st, q)) != cudaSuccess) return e;
        if ((e = mark(3)) != cudaSuccess) return e;

        GemvI16Args d = g;
        d.proj0 = 2; d.nmat = 1; d.kt = L.I / 16; d.ntn = L.H / 16; d.ndim = L.H;
        d.actb = ws + lay.actb_d;
        d.psum = reinterpret_cast<const float*>(ws + lay.psum_d);
        d.yraw = reinterpret_cast<float*>(ws + lay.yrow);
        d.isum = nullptr;                       // the down GEMV has J x H/128 column blocks: enough items unsplit
        d.counters = nullptr;
        d.next = reinterpret_cast<int*>(ws + lay.plan + offsetof(Plan, next_d));
        switch (L.bits[2])
        {
            case 2: e = launch_gemv_i16<2, 2, 1>(L, d, st); break;
            case 3: e = launch_gemv_i16<3, 3, 1>(L, d, st); break;
            default: e = launch_gemv_i16<4, 4, 1>(L, d, st); break;
        }
        if (e != cudaSuccess) return e;
        if ((e = mark(4)) != cudaSuccess) return e;
    }
    else
    {
        for (int i = 2; i <= 4; ++i)
            if ((e = mark(i)) != cudaSuccess) return e;
    }
    if (ntok > 0)
    {
        CombineI16Args c;
        c.plan = plan;
        c.pick_row = reinterpret_cast<const int*>(ws + lay.pick_row);
        c.row_weight = reinterpret_cast<const float*>(ws + lay.row_weight);
        c.row_expert = row_expert;
        c.yraw = reinterpret_cast<const float*>(ws + lay.yrow);
        c.svh_d = reinterpret_cast<const __half*>(L.svh[2]);
        c.H = L.H; c.ntok = ntok; c.topk = topk; c.has_shared = L.has_shared; c.E = L.E;
        c.out = out; c.out_dtype = out_dtype; c.accumulate = accumulate;
        c.hc = hc ? *hc : HcOut{ nullptr, nullptr, nullptr, 0 };
        if ((e = launch_combine(c, ntok, L.H, st)) != cudaSuccess) return e;
    }
    return mark(5);
}

}  // namespace glmx
