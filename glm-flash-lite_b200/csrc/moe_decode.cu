// Routed-expert MoE layer, decode-sized batches: grouped EXL3 dequant-GEMV on sm_100a.
//
// Pipeline of one forward call (all on one stream):
//   route   (route.cu)        picks -> expert-major rows, jobs of <= 8 rows
//   prep                      per row: xt = fp16(had128(x * suh) * HAD) for gate and up   (ft_core.h:96-102)
//   gemv<gate+up>             per (job, 128-col block, k-split): trellis tiles streamed by the tensor-copy engine into
//                             a shared-memory ring, decoded in registers straight into mma.m16n8k16 A fragments (chains
//                             of 4 tile MMAs from zero, chain sums added in fp32, compensated per block); epilogue: out_block (ft_core.h:104-110) of g and u, a = fp16(silu(g) * u)
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

constexpr int RB = 8;        // k-rows (16 inputs each) per 128-input block
constexpr int NCW = 8;       // consumer warps = n-tiles per 128-output block
constexpr int NTHR = (NCW + 1) * 32;
constexpr int XBLK = 256;    // bytes of one staged activation row per 128-input block (fp16, lane order of gemv_xpos)
#ifndef GLMX_EXACT_CTAS
#define GLMX_EXACT_CTAS 3
#endif
constexpr int CTAS_PER_SM = GLMX_EXACT_CTAS;
constexpr int RING_BYTES = (CTAS_PER_SM >= 3 ? 56 : 88) * 1024;    // per CTA; CTAS_PER_SM rings share an SM

// One pipeline stage holds HB 128-input blocks (HB * RB k-tile rows x 8 tiles) of ONE matrix (an item of the gate/up
// kernel runs all stages of gate, then all stages of up) and the job's activation rows for them. Two blocks per stage
// halve the per-stage costs (the ring's waits and arrivals, the addressing); the block sums stay per 128 inputs.
template <int K0, int K1, int NMAT, int HB>
struct Cfg
{
    static constexpr int TB0 = 32 * K0, TB1 = 32 * K1;
    static constexpr int ROW0 = 8 * TB0, ROW1 = 8 * TB1;
    static constexpr int MAT = HB * RB * (ROW0 > ROW1 ? ROW0 : ROW1);
    static constexpr int XROW = HB * XBLK;   // bytes per staged activation row
    // stride of the staged activation rows: lane (g, tq) reads row g, and a stride of 64 mod 128 bytes puts the two
    // rows of each quarter-warp's 16-byte loads in different bank halves
    static constexpr int XSTR = XROW + 64;
    static constexpr int XS = EXACT_MAXM * XSTR;
    static constexpr int STAGE = (MAT + XS + 127) / 128 * 128;   // tensor copies land 128-byte aligned
    static constexpr int NST = RING_BYTES / STAGE < 3 ? 3 : (RING_BYTES / STAGE > 12 ? 12 : RING_BYTES / STAGE);
    static constexpr int RED = NMAT * EXACT_MAXM * 128 * 8;      // (hi, lo) pairs
    static constexpr int SMEM = NST * STAGE + RED + 2 * NST * 8;
    static_assert(STAGE % 128 == 0 && MAT % 128 == 0, "stage alignment");
    static_assert(EXACT_MAXM == 8, "EXACT GEMV jobs of up to 8 rows: the 8 token columns of one MMA");
    static_assert(HB == 1 || HB == 2, "one or two 128-input blocks per stage");
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
    const __half* xin0; const __half* xin1;       // staged activation rows [R][kdim] (gemv_xpos order per block)
    const __half* svh0; const __half* svh1;       // [E_total][ndim]
    const __half* suh_next;                       // gate/up: suh of down [E_total][ndim]
    __half* xd;                                   // gate/up epilogue output [R][ndim]
    float* y;                                     // down epilogue output [R][ndim]
    float2* partials; int* counters; int* err;
    float act_limit;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }

__device__ __forceinline__ float h2f(const __half* p) { return __half2float(*p); }

// m16n8k16 f16 x f16 -> f32 with C = 0: one 16-input tile of 16 outputs against 8 tokens, the start of a chain
__device__ __forceinline__ void hmma0(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// the same MMA accumulating onto d
__device__ __forceinline__ void hmma_acc(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Tiles per accumulation chain inside the MMA. The MMA aligns its addends (the 16 products and C) to the largest and
// drops the bits below about 24 bits of it, so a long chain, whose C outgrows the products, is shortened toward zero
// step after step; chains of 4 tiles (64 inputs), added in fp32 and compensated per 128-input block, measured closer
// to the fp64 restatement than single tiles (and than chains of 8, which are not).
constexpr int TCHAIN = 4;
static_assert(RB % TCHAIN == 0 && TCHAIN % 2 == 0, "chains of whole tile pairs within a block");

// One pipeline stage of one matrix, tensor-core form: lane (g, tq) of consumer warp w decodes its A fragments of tiles
// (2rp, w) and (2rp + 1, w), loads token g's activations of both tiles (one 16-byte load: B fragments of the two MMAs)
// and chains the two MMAs - outputs (g, g + 8) x tokens (2tq, 2tq + 1) - into the current TCHAIN-tile chain.
template <int K>
__device__ __forceinline__ void stage_tc(const uint8_t* st, int row_bytes, int t_off, int x_off, const LaneDecode<K>& L,
                                         const OnesFrag& ones, float blk[4])
{
    float ch[4];
#pragma unroll
    for (int rp = 0; rp < RB / 2; ++rp)
    {
        uint32_t a[4], b[4];
        decode_frag_tc<K>(st + t_off + (2 * rp) * row_bytes, L, ones, a);
        decode_frag_tc<K>(st + t_off + (2 * rp + 1) * row_bytes, L, ones, b);
        const uint4 xv = *reinterpret_cast<const uint4*>(st + x_off + rp * 64);
        // chains of TCHAIN tiles inside the MMA accumulator (the first from zero), each added to the block sum in fp32
        if ((2 * rp) % TCHAIN == 0) hmma0(ch, a, xv.x, xv.y);
        else hmma_acc(ch, a, xv.x, xv.y);
        hmma_acc(ch, b, xv.z, xv.w);
        if ((2 * rp + 2) % TCHAIN == 0)
#pragma unroll
            for (int c = 0; c < 4; ++c) blk[c] = __fadd_rn(blk[c], ch[c]);
    }
}

// The k-stages of one item, tensor-core form (any job of <= 8 rows): per lane 4 (output, token) block sums, each fed
// once per 128-input block into a (hi, lo) pair by Fast2Sum; the pairs go to red[mat][token][col].
template <int K0, int K1, int NMAT, int HB>
__device__ __forceinline__ void item_consume_tc(uint8_t* ring, uint64_t* full, uint64_t* empty, float2* red, int kqs,
                                                int& s, uint32_t& ph, volatile int* s_abort, int* err, int warp, int lane,
                                                const LaneDecode<K0>& L0, const LaneDecode<K1>& L1, const OnesFrag& ones)
{
    using C = Cfg<K0, K1, NMAT, HB>;
    const int g = lane >> 2, tq = lane & 3;
    const int x_off = C::MAT + g * C::XSTR + tq * 16;
#pragma unroll 1
    for (int m = 0; m < NMAT; ++m)
    {
        float hi[4] = {0.0f, 0.0f, 0.0f, 0.0f}, lo[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
        for (int q = 0; q < kqs; ++q)
        {
            if (!*s_abort && !mbar_wait_bounded(&full[s], ph)) { atomicOr(err, ERR_TIMEOUT_FULL); *s_abort = 1; }
            const uint8_t* st = ring + s * C::STAGE;
#pragma unroll 1
            for (int hb = 0; hb < HB; ++hb)
            {
                // block hb: its tiles RB * hb k-rows in, its activations XBLK * hb bytes into each staged row
                float blk[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (NMAT == 1 || m == 0)
                    stage_tc<K0>(st + hb * RB * C::ROW0, C::ROW0, warp * C::TB0, x_off + hb * (XBLK - RB * C::ROW0), L0, ones, blk);
                else
                    stage_tc<K1>(st + hb * RB * C::ROW1, C::ROW1, warp * C::TB1, x_off + hb * (XBLK - RB * C::ROW1), L1, ones, blk);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                {
                    const float sum = __fadd_rn(hi[c], blk[c]);
                    lo[c] = __fadd_rn(lo[c], __fsub_rn(blk[c], __fsub_rn(sum, hi[c])));
                    hi[c] = sum;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == C::NST) { s = 0; ph ^= 1u; }
        }
        float2* rm = red + m * EXACT_MAXM * 128;
        const int o = warp * 16 + g;
#pragma unroll
        for (int c = 0; c < 4; ++c) rm[(2 * tq + (c & 1)) * 128 + o + 8 * (c >> 1)] = make_float2(hi[c], lo[c]);
    }
}

// EXACT-mode GEMV (one persistent kernel per phase). Items (job of <= 8 rows, 128-column block, K split); per item the
// producer warp's lane 0 streams the stages of HB 128-input blocks (trellis: one 2-D tensor copy per block;
// activations: one bulk copy per row), the 8 consumer warps decode (byte sums on the integer tensor pipe, codebook by HFMA2) and form each 16x16 tile's
// products with m16n8k16 MMAs against the job's 8 token columns in chains of TCHAIN tiles started from zero
// (stage_tc); the chain sums are added on the CUDA cores, block sums compensated (Fast2Sum, TwoSum across K splits).
template <int K0, int K1, int NMAT, bool GATEUP, int HB>
__global__ void __maxnreg__(CTAS_PER_SM >= 3 ? 72 : 112) gemv_kernel(GemvArgs a)
{
    using C = Cfg<K0, K1, NMAT, HB>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float2* red = reinterpret_cast<float2*>(smem + C::NST * C::STAGE);
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

    pdl_enter();                  // the split's plan and jobs and the staged activations come from earlier kernels
    const Plan pl = *a.plan;
    const int nb = a.ntn / 8;
    const int S = GATEUP ? pl.S_gu : pl.S_d;
    const int kqs = (a.kt / (HB * RB)) / S;                 // stages per item and matrix
    const int items = pl.J * nb * S;                        // < 2^31: J <= rows + 1, nb <= 64, S <= 64

    if (warp == NCW)
    {
        // ---------------- producer ----------------
        if (lane != 0) return;
        int s = 0, issued = 0;
        uint32_t ph = 0;
        for (int item = blockIdx.x; item < items && !s_abort; item += gridDim.x)
        {
            const int ks = item % S;
            const int jn = item / S;
            const int nbi = jn % nb, j = jn / nb;
            const int4 job = a.jobs[j];
            for (int m = 0; m < NMAT && !s_abort; ++m)
            {
                const CUtensorMap* map = a.tmaps + job.x * 3 + a.proj0 + m;
                const int tb = m ? C::TB1 : C::TB0, rowb = m ? C::ROW1 : C::ROW0;
                const __half* xin = m ? a.xin1 : a.xin0;
                const uint32_t bytes = (uint32_t) (HB * RB * rowb + job.z * C::XROW);
                for (int q = 0; q < kqs; ++q)
                {
                    if (!s_abort && !mbar_wait_bounded(&empty[s], ph ^ 1u)) { atomicOr(a.err, ERR_TIMEOUT_EMPTY); s_abort = 1; }
                    if (s_abort) break;
                    const int kr = (ks * kqs + q) * HB * RB;
                    uint8_t* st = ring + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], bytes);
                    // the stage's HB x RB k-tile rows x 8 tiles of the matrix: one tensor copy (x in 32-bit words) per
                    // block of RB rows
                    for (int hb = 0; hb < HB; ++hb)
                        tma_load_2d(st + hb * RB * rowb, map, nbi * 8 * tb / 4, kr + hb * RB, &full[s]);
                    for (int i = 0; i < job.z; ++i)
                        bulk_g2s(st + C::MAT + i * C::XSTR, xin + (size_t) (job.y + i) * a.kdim + kr * 16, C::XROW, &full[s]);
                    ++issued;
                    if (++s == C::NST) { s = 0; ph ^= 1u; }
                }
            }
        }
        // drain: every issued stage must have landed before the CTA may exit (the last min(issued, NST) stages, in
        // issue order, each with the phase it was issued in)
        const int nd = issued < C::NST ? issued : C::NST;
        int ds = s - nd, dph = (int) ph;
        if (ds < 0) { ds += C::NST; dph ^= 1; }
        for (int k = 0; k < nd; ++k)
        {
            if (!mbar_wait_bounded(&full[ds], (uint32_t) dph)) { atomicOr(a.err, ERR_TIMEOUT_FULL); break; }
            if (++ds == C::NST) { ds = 0; dph ^= 1; }
        }
        return;
    }

    // ---------------- consumers ----------------
    LaneDecode<K0> L0;
    L0.init(lane);
    LaneDecode<K1> L1;
    L1.init(lane);
    OnesFrag ones;
    ones.init(lane);
    int s = 0;
    uint32_t ph = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x)
    {
        const int jn = item / S;
        const int nbi = jn % nb, j = jn / nb;
        const int4 job = a.jobs[j];
        item_consume_tc<K0, K1, NMAT, HB>(ring, full, empty, red, kqs, s, ph, &s_abort, a.err, warp, lane, L0, L1, ones);
        consumer_sync();
        if (S > 1)
        {
            // split-K: each piece stores its (hi, lo) pairs; the last to arrive adds them in split order (TwoSum on the
            // hi parts, lo parts added), so the split does not round the partial sums to fp32
            // the job's rows only, at [split][row][matrix][column]: entry v of its NMAT x job.z x 128 values is
            // red[m][i][c]
            const int ks = item - jn * S;
            const int zr = job.z * 128, nvj = NMAT * zr;
            const size_t kstride = (size_t) pl.R * NMAT * a.ndim;
            auto slot = [&](int v) { const int m = v / zr, r = v - m * zr; return m * EXACT_MAXM * 128 + r; };
            auto gidx = [&](int v) {
                const int m = v / zr, r = v - m * zr, i = r >> 7, c = r & 127;
                return ((size_t) (job.y + i) * NMAT + m) * a.ndim + nbi * 128 + c;
            };
            for (int v = tid; v < nvj; v += NCW * 32) __stcg(a.partials + ks * kstride + gidx(v), red[slot(v)]);
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
            for (int v = tid; v < nvj; v += NCW * 32)
            {
                const int i = slot(v);
                const float2* p0 = a.partials + gidx(v);
                float h = 0.0f, l = 0.0f;
                for (int k = 0; k < S; ++k)
                {
                    const float2 pv = __ldcg(p0 + k * kstride);
                    const float sum = __fadd_rn(h, pv.x);
                    const float bb = __fsub_rn(sum, h);
                    const float e = __fadd_rn(__fsub_rn(h, __fsub_rn(sum, bb)), __fsub_rn(pv.x, bb));
                    l = __fadd_rn(__fadd_rn(l, pv.y), e);
                    h = sum;
                }
                red[i] = make_float2(h, l);
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
                    const float2 gp = red[i * 128 + lane + 32 * q], up = red[EXACT_MAXM * 128 + i * 128 + lane + 32 * q];
                    gv[q] = r16(__fadd_rn(gp.x, gp.y));
                    uv[q] = r16(__fadd_rn(up.x, up.y));
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
                    const int c = lane + 32 * q;     // the down GEMV reads its input in the gemv_xpos lane order
                    a.xd[(size_t) row * a.ndim + nbi * 128 + gemv_xpos(c)] = __float2half_rn(__fmul_rn(av[q], HAD));
                }
            }
            else
            {
                float yv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                {
                    const float2 yp = red[i * 128 + lane + 32 * q];
                    yv[q] = r16(__fadd_rn(yp.x, yp.y));
                }
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
// One warp per (token, 128-input block, projection) and row group: the token's x block is loaded once per warp and
// transformed for the token's rows of its group (its routed picks, then the shared expert's row), each with that row's
// expert's suh. Small batches give every row its own warp (groups = rows per token); large ones one warp per block.
struct PrepArgs
{
    const Plan* plan;
    const void* x; int x_dtype; int H;
    int ntok, topk, has_shared, E;
    const int* pick_row; const int* row_expert;
    const __half* suh_g; const __half* suh_u;
    __half* xg; __half* xu;
    int natural;          // 1: natural input order (tensor-core GEMM), 0: PERM16 order inside 16-row tiles (GEMV)
    int groups;           // warps per (token, block, projection): warp g transforms the token's rows g, g + groups, ...
};

__device__ __forceinline__ float load_x(const void* x, int dt, size_t i)
{
    if (dt == GLMX_F16) return __half2float(reinterpret_cast<const __half*>(x)[i]);
    if (dt == GLMX_BF16) return r16(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]));
    return reinterpret_cast<const float*>(x)[i];
}

__global__ void __launch_bounds__(256) prep_kernel(PrepArgs a)
{
    pdl_enter();
    const int nbk = a.H / 128;
    const long long wid = ((long long) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int t = (int) (wid / (2 * nbk * a.groups));
    if (t >= a.ntok) return;
    const int rem = (int) (wid % (2 * nbk * a.groups)), grp = rem % a.groups, pb = rem / a.groups;
    const int p = pb / nbk, b = pb % nbk;
    float xv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = load_x(a.x, a.x_dtype, (size_t) t * a.H + b * 128 + lane + 32 * q);
    const __half* suh_p = p ? a.suh_u : a.suh_g;
    __half* out_p = p ? a.xu : a.xg;
    const int nk = a.topk + (a.has_shared ? 1 : 0);
    for (int k = grp; k < nk; k += a.groups)
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
            const int c = lane + 32 * q;         // GEMV: the lane order of gemv_xpos
            out[a.natural ? c : gemv_xpos(c)] = __float2half_rn(__fmul_rn(v[q], HAD));
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
        float* xr = a.hc.x + (size_t) t * 4 * a.H;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            hc_apply_col(xr, a.H, c + i, a.hc.y_half ? __half2float(__float2half_rn(v[i])) : v[i],
                         a.hc.post + (size_t) t * 4, a.hc.comb + (size_t) t * 16);
        if (a.hc.fn)
        {
            // the next site's mix partials of the updated stack: this warp's 32 quads are 128-column block c / 128
            const size_t nb = a.H / 128, jb = c / 128;
#pragma unroll
            for (int g = 0; g < 4; ++g)
                hc_mix_warp(*reinterpret_cast<const float4*>(xr + (size_t) g * a.H + c), a.hc.fn + (size_t) g * a.H + c,
                            (size_t) 4 * a.H, a.hc.part + (((size_t) t * 4 + g) * nb + jb) * 25, threadIdx.x & 31);
        }
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
    pdl_enter();
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

template <int K0, int K1, int NMAT, bool GATEUP, int HB>
cudaError_t launch_gemv_hb(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    using C = Cfg<K0, K1, NMAT, HB>;
    static bool attr_set[64] = {};
    if (!attr_set[L.device])
    {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<K0, K1, NMAT, GATEUP, HB>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[L.device] = true;
    }
    return launch_chained(gemv_kernel<K0, K1, NMAT, GATEUP, HB>, dim3(grid), dim3(NTHR), C::SMEM, st, a);
}

// the stage form the split plan was made for (exact_stage_blocks); two-block stages exist for bitrates up to 3 only
template <int K0, int K1, int NMAT, bool GATEUP>
cudaError_t launch_gemv(const Layer& L, const GemvArgs& a, int grid, cudaStream_t st)
{
    if constexpr (K0 <= 3 && K1 <= 3)
        if (exact_stage_blocks(L, GATEUP ? 0 : 2) == 2) return launch_gemv_hb<K0, K1, NMAT, GATEUP, 2>(L, a, grid, st);
    return launch_gemv_hb<K0, K1, NMAT, GATEUP, 1>(L, a, grid, st);
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

int exact_stage_blocks(const Layer& L, int proj)
{
    const int kdim = proj == 0 ? L.H : L.I;
    const bool low = proj == 0 ? (L.bits[0] <= 3 && L.bits[1] <= 3) : L.bits[2] <= 3;
    return low && kdim % 256 == 0 ? 2 : 1;
}

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
    w.rows_max = rows; w.jobs_max = jobs;
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
    // EXACT split-K (hi, lo) pairs: room for as many splits as 2 x grid_ctas items of a full job would fill
    w.part_bytes = sizeof(float2) * (size_t) 2 * grid_ctas * 2 * EXACT_MAXM * 128;
    w.partials = take(w.part_bytes);
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
    // small batches: one warp per row of a token block (the token's rows in parallel); large ones: one warp per token
    // block serving all its rows (the block loaded once)
    p.groups = ntok <= 16 ? topk + (L.has_shared ? 1 : 0) : 1;
    const long long warps = (long long) ntok * 2 * (L.H / 128) * p.groups;
    return launch_chained(prep_kernel, dim3((unsigned) ((warps + 7) / 8)), dim3(256), 0, st, p);
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
        g.partials = reinterpret_cast<float2*>(ws + lay.partials);
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
        if ((e = launch_chained(combine_kernel, grd, dim3(256), 0, st, c)) != cudaSuccess) return e;
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
