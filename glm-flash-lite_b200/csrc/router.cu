// Router of the MoE site, in front of the split: gate linear, sigmoid, score-correction bias, group-limited top-k and
// renormalised weights. This is the GLM-4 MoE routing the reference takes from exllamav3's router through its
// routing_fn hook (glm53/cpu_tier.py:305-335: sel [bsz, k] and w [bsz, k] come out of it), as the published model
// code states it (transformers' Glm4MoeTopkRouter.forward and Glm4MoeMoE.route_tokens_to_experts,
// models/glm4_moe/modeling_glm4_moe.py:302-305 and 389-412):
//   logits = fp32(z) . fp32(W)^T                                      [ntok, E]
//   s = sigmoid(logits);  c = s + bias                                 (c decides, s weighs)
//   group score = sum of the two largest c of each of n_group equal groups; keep the topk_group best groups and set c
//   of the others to 0.0; picks = the topk largest c; w = s[picks]; norm: w /= (sum w + 1e-20); w *= scale.
//
// Conventions where the published code leaves the order open (torch.topk with sorted=False): picks come out in
// descending c, equal values in ascending expert id; the normalising sum adds the weights in pick order. sigmoid is
// 1 / (1 + e^-x) with e^-x from a fixed sequence of fp32 operations (exp_cw below), so the value does not depend on
// one platform's exp.
//
// Kernels: router_gate_kernel computes a 16-token x 8-expert block of logits per CTA on the tensor cores (exact
// products, fp32 sums); router_select_kernel runs the selection, one token per warp, as a programmatic dependent
// launch behind the gate kernel (or alone when the caller passes logits).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

constexpr int SEL_WARPS = 8;

struct RouterArgs
{
    const void* z; int z_dtype; int ntok, H;
    const void* gw; int gw_dtype;
    const float* bias; int E, n_group, topk_group, topk, norm; float scale;
    float* logits; void* sel; int sel_i64; void* w; int w_dtype;
};

// (v, i) ranks before (u, j): larger value first, equal values by smaller index
__device__ __forceinline__ bool better(float v, int i, float u, int j) { return v > u || (v == u && i < j); }

// 2^k as an fp32 (k in [-149, 127]; below that 0)
__device__ __forceinline__ float pow2i(int k)
{
    if (k >= -126) return __int_as_float((k + 127) << 23);
    return k >= -149 ? __int_as_float(1 << (k + 149)) : 0.0f;
}

// e^y in fp32 by Cody and Waite's argument reduction (y = n ln2 + r, |r| <= ln2 / 2, ln2 split into a 16-bit head and
// a tail so n * head is exact) and the degree-8 Taylor polynomial of e^r in Horner form with fused multiply-adds; 2^n
// is applied in two halves so every intermediate stays finite until the last product. Every step is one IEEE fp32
// operation, so any platform with fp32 FMA and round-to-nearest gets the same bits (the C restatement does).
__device__ __forceinline__ float exp_cw(float y)
{
    if (y != y) return y;
    y = fminf(fmaxf(y, -175.0f), 175.0f);
    const float n = rintf(__fmul_rn(y, 1.44269502162933349609375f));
    float r = __fmaf_rn(n, -0.693145751953125f, y);
    r = __fmaf_rn(n, -1.428606765330187045037746429443359375e-06f, r);
    float p = 2.4801587301587302e-05f;
    p = __fmaf_rn(p, r, 1.9841269841269841e-04f);
    p = __fmaf_rn(p, r, 1.3888888888888889e-03f);
    p = __fmaf_rn(p, r, 8.3333333333333332e-03f);
    p = __fmaf_rn(p, r, 4.1666666666666664e-02f);
    p = __fmaf_rn(p, r, 1.6666666666666666e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int) n, n1 = ni / 2, n2 = ni - n1;
    return __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(n2));
}

__device__ __forceinline__ float sigmoid_cw(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cw(-x))); }

constexpr int SEL_SLOTS = GLMX_ROUTER_MAX_EXPERTS / 32;    // experts per lane: lane + 32 i

// Selection for one token by one warp, all in registers. row = the token's E logits (written by other CTAs of this
// launch: read through L2).
__device__ void select_token(const RouterArgs& a, int t, const float* row, float* s_buf, int lane)
{
    const int E = a.E;
    float s[SEL_SLOTS], c[SEL_SLOTS];
    // every load first (clamped ids, so none waits behind a bounds check), then the arithmetic
#pragma unroll
    for (int i = 0; i < SEL_SLOTS; ++i)
    {
        const int e = min(lane + 32 * i, E - 1);
        s[i] = __ldcg(row + e);
        c[i] = a.bias ? __ldg(a.bias + e) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < SEL_SLOTS; ++i)
    {
        s[i] = sigmoid_cw(s[i]);
        if (a.bias) c[i] = __fadd_rn(s[i], c[i]);
        else c[i] = s[i];
    }
    if (a.n_group > 1)
    {
        // group score = largest + second largest c of the group (torch.topk(2).sum of two values: order-free)
        const int G = E / a.n_group;
        float gs = -INFINITY;                 // lane g keeps group g's score
        for (int g = 0; g < a.n_group; ++g)
        {
            float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
            for (int i = 0; i < SEL_SLOTS; ++i)
            {
                const int e = lane + 32 * i;
                if (e < E && e / G == g)
                {
                    if (c[i] > m1) { m2 = m1; m1 = c[i]; }
                    else if (c[i] > m2) m2 = c[i];
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
            {
                const float o1 = __shfl_xor_sync(0xffffffffu, m1, o), o2 = __shfl_xor_sync(0xffffffffu, m2, o);
                const float hi = fmaxf(m1, o1), lo = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
                m1 = hi; m2 = lo;
            }
            if (lane == g) gs = __fadd_rn(m1, m2);
        }
        int rank = 0;                          // rank of group `lane` among the n_group scores
        for (int h = 0; h < a.n_group; ++h)
        {
            const float v = __shfl_sync(0xffffffffu, gs, h);
            if (lane < a.n_group && better(v, h, gs, lane)) ++rank;
        }
        const unsigned keep = __ballot_sync(0xffffffffu, lane < a.n_group && rank < a.topk_group);
#pragma unroll
        for (int i = 0; i < SEL_SLOTS; ++i)
        {
            const int e = lane + 32 * i;
            if (e < E && !((keep >> (e / G)) & 1u)) c[i] = 0.0f;      // masked_fill(~mask, 0.0)
        }
    }
#pragma unroll
    for (int i = 0; i < SEL_SLOTS; ++i)
        if (lane + 32 * i < E) s_buf[lane + 32 * i] = s[i];
    __syncwarp();
    // top-k on 64-bit order keys: high word = the order-preserving bits of c, low word = ~id (equal c: smaller id
    // ranks first); free slots hold key 0, below every real key (a NaN c ranks above everything, as in torch.topk).
    // Each lane sorts its keys once (bitonic network, descending); per round two redux.sync max operations find the
    // warp's best head, and the lane that owned it shifts its list by one.
    unsigned long long k[SEL_SLOTS];
#pragma unroll
    for (int i = 0; i < SEL_SLOTS; ++i)
    {
        const int e = lane + 32 * i;
        const uint32_t b = __float_as_uint(c[i]);
        const uint32_t hi = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        k[i] = e < E ? ((unsigned long long) hi << 32) | (uint32_t) ~(uint32_t) e : 0ull;
    }
#pragma unroll
    for (int size = 2; size <= SEL_SLOTS; size <<= 1)
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
            for (int i = 0; i < SEL_SLOTS; ++i)
            {
                const int j = i ^ stride;
                if (j > i)
                {
                    const bool desc = (i & size) == 0;
                    const unsigned long long x = k[i], y = k[j];
                    const bool sw = desc ? x < y : x > y;
                    k[i] = sw ? y : x;
                    k[j] = sw ? x : y;
                }
            }
    int pick = -1;
    float wsum = 0.0f, wv = 0.0f;
    for (int r = 0; r < a.topk; ++r)
    {
        const uint32_t bh = (uint32_t) (k[0] >> 32), bl = (uint32_t) k[0];
        const uint32_t mh = __reduce_max_sync(0xffffffffu, bh);
        const uint32_t ml = __reduce_max_sync(0xffffffffu, bh == mh ? bl : 0u);
        const int id = (int) ~ml;
        const float sv = s_buf[id];
        wsum = __fadd_rn(wsum, sv);
        if (lane == r) { pick = id; wv = sv; }
        if ((id & 31) == lane)
        {
#pragma unroll
            for (int i = 0; i + 1 < SEL_SLOTS; ++i) k[i] = k[i + 1];
            k[SEL_SLOTS - 1] = 0ull;
        }
    }
    __syncwarp();
    if (lane < a.topk)
    {
        float v = wv;
        if (a.norm) v = __fdiv_rn(v, __fadd_rn(wsum, 1e-20f));
        v = __fmul_rn(v, a.scale);
        const size_t o = (size_t) t * a.topk + lane;
        if (a.sel_i64) reinterpret_cast<long long*>(a.sel)[o] = pick;
        else reinterpret_cast<int*>(a.sel)[o] = pick;
        if (a.w_dtype == GLMX_F16) reinterpret_cast<__half*>(a.w)[o] = __float2half_rn(v);
        else if (a.w_dtype == GLMX_BF16) reinterpret_cast<__nv_bfloat16*>(a.w)[o] = __float2bfloat16_rn(v);
        else reinterpret_cast<float*>(a.w)[o] = v;
    }
}

// ---- gate linear on the tensor cores ----
//
// logits[t][e] = sum_k z[t][k] W[e][k] with mma.m16n8k16 (bf16 x bf16 -> fp32): a 16-token x 8-expert tile per warp,
// 32 inputs (two MMAs) per step. Every operand is split exactly into bf16 parts (bf16: itself; fp16: hi + lo, the
// 11-bit significand in 8 + 3 bits; fp32: hi + mid + lo, 8 + 8 + 8 bits), so every product the tensor core forms is
// exact; each MMA starts from zero and its 16-product sum is added to the fp32 accumulator with an IEEE add, in input
// order. Lane (g, tq) loads 8 consecutive inputs 8tq .. 8tq+7 of token rows g and g+8 and of expert row g; inside an
// MMA the k slots {2tq, 2tq+1, 2tq+8, 2tq+9} take inputs {0,1,2,3} (first MMA) or {4,5,6,7} (second) of that run, for
// A and B alike, so each product pairs the same input index. The 8 warps of a CTA take consecutive eighths of K; their
// partial tiles are added in warp order in shared memory.

// bf16x2 words (4 per part) of 8 consecutive values of type T
template <typename T> struct Parts;
template <> struct Parts<__nv_bfloat16>
{
    static constexpr int P = 1;
    uint4 raw;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { raw = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void split(uint32_t w[P][4]) const { w[0][0] = raw.x; w[0][1] = raw.y; w[0][2] = raw.z; w[0][3] = raw.w; }
};

__device__ __forceinline__ uint32_t bf2_bits(float x, float y)
{
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 bf2_float(uint32_t w)
{
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
// v = hi + (rest): hi = the bf16 rounding of v, rest exact in fp32
__device__ __forceinline__ uint32_t split_step(float2& v)
{
    const uint32_t hi = bf2_bits(v.x, v.y);
    const float2 h = bf2_float(hi);
    v.x = __fsub_rn(v.x, h.x);
    v.y = __fsub_rn(v.y, h.y);
    return hi;
}

template <> struct Parts<__half>
{
    static constexpr int P = 2;
    uint4 raw;
    __device__ __forceinline__ void load(const __half* p) { raw = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void split(uint32_t w[P][4]) const
    {
        const uint32_t r[4] = { raw.x, raw.y, raw.z, raw.w };
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            float2 v = __half22float2(*reinterpret_cast<const __half2*>(&r[j]));
            w[0][j] = split_step(v);
            w[1][j] = bf2_bits(v.x, v.y);              // <= 3 significant bits: exact
        }
    }
};

template <> struct Parts<float>
{
    static constexpr int P = 3;
    float4 lo4, hi4;
    __device__ __forceinline__ void load(const float* p)
    {
        lo4 = __ldg(reinterpret_cast<const float4*>(p));
        hi4 = __ldg(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void split(uint32_t w[P][4]) const
    {
        float2 v[4] = { make_float2(lo4.x, lo4.y), make_float2(lo4.z, lo4.w), make_float2(hi4.x, hi4.y), make_float2(hi4.z, hi4.w) };
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            w[0][j] = split_step(v[j]);
            w[1][j] = split_step(v[j]);
            w[2][j] = bf2_bits(v[j].x, v[j].y);        // <= 8 significant bits left: exact
        }
    }
};

__device__ __forceinline__ void mma_bf16_zero(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

constexpr int GATE_TT = 16;    // tokens per CTA (MMA rows)
constexpr int GATE_TE = 8;     // experts per CTA (MMA columns)
constexpr int GATE_WARPS = 8;  // K eighths

template <typename TZ, typename TW>
__global__ void __launch_bounds__(GATE_WARPS * 32, Parts<TZ>::P * Parts<TW>::P > 1 ? 1 : 2) router_gate_kernel(RouterArgs a)
{
    constexpr int D = (sizeof(TZ) == 4 || sizeof(TW) == 4) ? 4 : 8;     // 32-input steps loaded ahead
    constexpr int PZ = Parts<TZ>::P, PW = Parts<TW>::P;
    __shared__ float red[GATE_WARPS][GATE_TT][GATE_TE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    const int e0 = blockIdx.x * GATE_TE, t0 = blockIdx.y * GATE_TT;
    const int nt = min(GATE_TT, a.ntok - t0);
    const TZ* z = reinterpret_cast<const TZ*>(a.z);
    const TZ* za = z + (size_t) (t0 + min(g, nt - 1)) * a.H + 8 * tq;
    const TZ* zb = z + (size_t) (t0 + min(g + 8, nt - 1)) * a.H + 8 * tq;
    const TW* wr = reinterpret_cast<const TW*>(a.gw) + (size_t) min(e0 + g, a.E - 1) * a.H + 8 * tq;
    const int nch = a.H / 32, cpw = (nch + GATE_WARPS - 1) / GATE_WARPS;
    const int c_beg = warp * cpw, c_end = min(nch, c_beg + cpw);
    float acc[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
    for (int c0 = c_beg; c0 < c_end; c0 += D)
    {
        Parts<TZ> A0[D], A1[D];
        Parts<TW> B[D];
#pragma unroll
        for (int j = 0; j < D; ++j)
            if (c0 + j < c_end)
            {
                const int k = (c0 + j) * 32;
                A0[j].load(za + k);
                A1[j].load(zb + k);
                B[j].load(wr + k);
            }
#pragma unroll
        for (int j = 0; j < D; ++j)
            if (c0 + j < c_end)
            {
                uint32_t a0[PZ][4], a1[PZ][4], b[PW][4];
                A0[j].split(a0);
                A1[j].split(a1);
                B[j].split(b);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int pz = 0; pz < PZ; ++pz)
#pragma unroll
                        for (int pw = 0; pw < PW; ++pw)
                        {
                            float d[4];
                            mma_bf16_zero(d, a0[pz][2 * h], a1[pz][2 * h], a0[pz][2 * h + 1], a1[pz][2 * h + 1],
                                          b[pw][2 * h], b[pw][2 * h + 1]);
#pragma unroll
                            for (int q = 0; q < 4; ++q) acc[q] = __fadd_rn(acc[q], d[q]);
                        }
            }
    }
    red[warp][g][2 * tq] = acc[0];
    red[warp][g][2 * tq + 1] = acc[1];
    red[warp][g + 8][2 * tq] = acc[2];
    red[warp][g + 8][2 * tq + 1] = acc[3];
    __syncthreads();
    if (threadIdx.x < GATE_TT * GATE_TE)
    {
        const int t = threadIdx.x / GATE_TE, n = threadIdx.x % GATE_TE;
        float v = red[0][t][n];
#pragma unroll
        for (int w = 1; w < GATE_WARPS; ++w) v = __fadd_rn(v, red[w][t][n]);
        if (t < nt && e0 + n < a.E) a.logits[(size_t) (t0 + t) * a.E + e0 + n] = v;
    }
    // the selection kernel behind this one (programmatic dependent launch) may start its launch now; it waits for
    // this grid's completion and memory flush before reading any logit
    asm volatile("griddepcontrol.launch_dependents;");
}

__global__ void __launch_bounds__(SEL_WARPS * 32) router_select_kernel(RouterArgs a)
{
    __shared__ float s_buf[SEL_WARPS][GLMX_ROUTER_MAX_EXPERTS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * SEL_WARPS + warp;
    asm volatile("griddepcontrol.wait;" ::: "memory");     // the gate kernel's logits (no-op without one)
    if (t >= a.ntok) return;
    select_token(a, t, a.logits + (size_t) t * a.E, s_buf[warp], lane);
}

int gate_token_blocks(int ntok) { return (ntok + GATE_TT - 1) / GATE_TT; }

template <typename TZ>
cudaError_t launch_gate(const RouterArgs& a, cudaStream_t st)
{
    const dim3 grid((a.E + GATE_TE - 1) / GATE_TE, gate_token_blocks(a.ntok));
    if (a.gw_dtype == GLMX_F32) router_gate_kernel<TZ, float><<<grid, GATE_WARPS * 32, 0, st>>>(a);
    else if (a.gw_dtype == GLMX_BF16) router_gate_kernel<TZ, __nv_bfloat16><<<grid, GATE_WARPS * 32, 0, st>>>(a);
    else router_gate_kernel<TZ, __half><<<grid, GATE_WARPS * 32, 0, st>>>(a);
    return cudaGetLastError();
}

// selection, one token per warp; after the gate kernel it is a programmatic dependent launch, so its launch overlaps
// the gate kernel's tail
cudaError_t launch_select(const RouterArgs& a, bool after_gate, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.ntok + SEL_WARPS - 1) / SEL_WARPS);
    cfg.blockDim = dim3(SEL_WARPS * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = after_gate ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, router_select_kernel, a);
}

bool dtype_float(int d) { return d == GLMX_F16 || d == GLMX_F32 || d == GLMX_BF16; }

int fail(int code, const std::string& msg)
{
    set_error("glmx_router: " + msg);
    return code;
}

}  // namespace

}  // namespace glmx

using namespace glmx;

extern "C" int glmx_router(const void* z, int z_dtype, int ntok, int hidden, const void* gate_w, int gate_dtype,
                           const float* bias, int n_experts, int n_group, int topk_group, int topk, int norm, float scale,
                           float* logits, void* sel, int sel_dtype, void* w, int w_dtype, void* stream)
{
    if (ntok < 0) return fail(GLMX_E_ARG, "ntok must be >= 0");
    if (n_experts < 1 || n_experts > GLMX_ROUTER_MAX_EXPERTS) return fail(GLMX_E_ARG, "n_experts must be in [1, 512]");
    if (n_group < 1 || n_experts % n_group || n_group > 32) return fail(GLMX_E_ARG, "n_group must divide n_experts (<= 32 groups)");
    if (n_group > 1 && n_experts / n_group < 2) return fail(GLMX_E_ARG, "groups need at least 2 experts each");
    if (topk_group < 1 || topk_group > n_group) return fail(GLMX_E_ARG, "topk_group must be in [1, n_group]");
    if (topk < 1 || topk > 32 || topk > topk_group * (n_experts / n_group))
        return fail(GLMX_E_ARG, "topk must be in [1, 32] and at most topk_group * n_experts / n_group");
    if (!logits || !sel || !w) return fail(GLMX_E_ARG, "logits, sel and w are required");
    if (sel_dtype != GLMX_I32 && sel_dtype != GLMX_I64) return fail(GLMX_E_ARG, "sel_dtype must be GLMX_I32 or GLMX_I64");
    if (!dtype_float(w_dtype)) return fail(GLMX_E_ARG, "w_dtype must be GLMX_F16, GLMX_F32 or GLMX_BF16");
    if (gate_w)
    {
        if (!z) return fail(GLMX_E_ARG, "z is required with gate_w");
        if (!dtype_float(z_dtype) || !dtype_float(gate_dtype)) return fail(GLMX_E_ARG, "z_dtype and gate_dtype must be float types");
        if (hidden < 32 || hidden % 32) return fail(GLMX_E_ARG, "hidden must be a positive multiple of 32");
        if ((reinterpret_cast<uintptr_t>(z) & 15u) || (reinterpret_cast<uintptr_t>(gate_w) & 15u))
            return fail(GLMX_E_ARG, "z and gate_w must be 16-byte aligned");
    }
    if (ntok == 0) return GLMX_OK;
    RouterArgs a{};
    a.z = z; a.z_dtype = z_dtype; a.ntok = ntok; a.H = hidden;
    a.gw = gate_w; a.gw_dtype = gate_dtype;
    a.bias = bias; a.E = n_experts; a.n_group = n_group; a.topk_group = topk_group; a.topk = topk; a.norm = norm ? 1 : 0;
    a.scale = scale;
    a.logits = logits; a.sel = sel; a.sel_i64 = sel_dtype == GLMX_I64; a.w = w; a.w_dtype = w_dtype;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (gate_w)
    {
        if (z_dtype == GLMX_F32) e = launch_gate<float>(a, st);
        else if (z_dtype == GLMX_BF16) e = launch_gate<__nv_bfloat16>(a, st);
        else e = launch_gate<__half>(a, st);
        if (e == cudaSuccess) e = launch_select(a, true, st);
    }
    else
        e = launch_select(a, false, st);
    if (e != cudaSuccess) return fail(GLMX_E_CUDA, std::string("launch: ") + cudaGetErrorString(e));
    return GLMX_OK;
}
