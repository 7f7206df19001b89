// Shared device helpers of the routed-expert MoE path (sm_100a).
//
// EXL3 "MUL1" trellis tiles (restated from nkeilar/glm-flash-lite kernels/cpu_avx2/ft_core.h:28-83):
//   a 16x16 tile of K-bit weights is a circular bit stream of 256*K bits stored as little-endian 32-bit words,
//   most significant bit first inside each word. Weight i's 16-bit state is the window ending at bit i*K+K
//   (ft_core.h:65-73); its value is fp16(fma(1024 + bytesum(state * 0x83DCD12D), KINV, KBIAS)) (ft_core.h:75-83).
//   Stream weights 8t..8t+7 sit at the tile positions the mma.m16n8k16 A fragment gives lane t when A = W^T
//   (PERM, ft_core.h:48-61), so one lane decodes exactly its own fragment.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace glmx {

constexpr uint32_t MUL1 = 0x83DCD12Du;
constexpr float HAD = 0.088388347648f;          // 1/sqrt(128) as the reference writes it (ft_core.h:29)
constexpr uint16_t KINV_BITS = 0x1eee;          // ft_core.h:38
constexpr uint16_t KBIAS_BITS = 0xc931;         // ft_core.h:39
constexpr int MAXM = 8;                         // tokens per job (ft_core.h:32)
constexpr int WAIT_TIMEOUT_NS = 2000000000;     // bounded device waits: 2 s

// error bits written to the workspace error word
enum : int { ERR_TIMEOUT_FULL = 1, ERR_TIMEOUT_EMPTY = 2, ERR_BAD_EXPERT = 4, ERR_BAD_SHAPE = 8, ERR_TIMEOUT_PEER = 16 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier + bulk async copy (TMA engine, no tensor map) -----------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and the caller records an error and leaves its loop) once timeout_ns passed.
__device__ __forceinline__ bool mbar_wait_bounded_ns(uint64_t* bar, uint32_t parity, uint64_t timeout_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true)
    {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > timeout_ns) return false;
    }
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity)
{
    return mbar_wait_bounded_ns(bar, parity, (uint64_t) WAIT_TIMEOUT_NS);
}

// 2-D tiled tensor copy global -> shared (the innermost coordinate x times the element size a multiple of 16 bytes),
// completion counted on `bar`
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes and addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ---- programmatic dependent launch -----------------------------------------------------------------------------------
// Kernels of a layer call launched with launch_chained start with pdl_enter(): wait until the previous kernel of the
// stream has completed and its memory is visible (a no-op without a chained launch), then allow the next kernel to be
// launched while this one runs (its CTAs are placed as resources free up and wait in their own pdl_enter()).
__device__ __forceinline__ void pdl_enter()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
}

// ---- expert-parallel return over peer memory ------------------------------------------------------------------------

__device__ __forceinline__ void st_release_sys(int* p, int v)
{
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p)
{
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Destination of token t's combined row in the peer return (see PeerOut).
__device__ __forceinline__ float* peer_row(float* const* recv, int rank, int world, int rpr, int seq, int t, int H)
{
    const int owner = t / rpr, tl = t % rpr;
    return recv[owner] + ((size_t) ((seq & 1) * world + rank) * rpr + tl) * H;
}

// Called by every thread of every CTA of a combine launch after its peer stores: the last CTA to arrive (arrival
// counter, no waiting) publishes flag [seq & 1][rank] = seq on every rank and clears the counter.
__device__ __forceinline__ void peer_done(float* const* recv, int* const* flags, int* counter, int rank, int world, int seq)
{
    (void) recv;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && threadIdx.y == 0)
    {
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        if ((unsigned) atomicAdd(counter, 1) == total - 1)
        {
            __threadfence_system();
            for (int d = 0; d < world; ++d) st_release_sys(flags[d] + (seq & 1) * world + rank, seq);
            atomicExch(counter, 0);
        }
    }
}

// ---- trellis tile decode ---------------------------------------------------------------------------------------------

// Per-lane constants for decoding lane `lane`'s 8 stream weights of a K-bit tile: the two 32-bit words holding its
// (7K+16)-bit window and the right shift `pre` of (hi:lo) that brings the window to bits [0, 7K+16). State j then sits
// at the compile-time shift K * (7 - j), so no per-state shift is held in registers. pre is in [0, 32] for the tile
// layouts of K = 2, 3, 4 (K = 2 lanes whose window lies wholly in the hi word need 32).
template <int K>
struct LaneDecode
{
    static_assert(K >= 2 && K <= 4, "trellis bitrates 2..4");
    uint32_t off_hi, off_lo, pre;
    __device__ __forceinline__ void init(int lane)
    {
        constexpr int bits = 256 * K, words = 8 * K;
        const int start = (8 * lane * K + K - 16 + bits) % bits;     // first bit of weight 8*lane's window
        const int wa = start / 32, rs = start % 32;
        off_hi = 4u * wa;
        off_lo = 4u * ((wa + 1) % words);
        pre = uint32_t(48 - rs - 7 * K);                              // state 0 starts at bit 48 - rs of (hi:lo)
    }
};

// Shared-memory word load as an ordinary C++ load, so the compiler may schedule it freely between the (memory-
// clobbering) mbarrier waits.
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// fp16 pair (lo = a, hi = b) of codebook weights from two byte sums, one fp16 rounding (hfma), ft_core.h:81-83.
// sa, sb are 0x6400 + s (< 2^16), so the pack is an exact multiply-add (FMA pipe; the integer ALU pipe is the scarcer).
__device__ __forceinline__ uint32_t codebook_pair(uint32_t sa, uint32_t sb)
{
    const uint32_t hb = sb * 65536u + sa;                            // half(1024+sa) | half(1024+sb) << 16
    __half2 h = *reinterpret_cast<const __half2*>(&hb);
    const __half2 kinv = __halves2half2(__ushort_as_half(KINV_BITS), __ushort_as_half(KINV_BITS));
    const __half2 kbias = __halves2half2(__ushort_as_half(KBIAS_BITS), __ushort_as_half(KBIAS_BITS));
    h = __hfma2(h, kinv, kbias);
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---- decode with the byte sums on the tensor pipe --------------------------------------------------------------------
//
// The 8 product words x_j = state_j * MUL1 of a lane go into two mma.m16n8k32 u8 x u8 -> s32 as A operands; B is a
// constant 0/1 pattern selecting the 4 bytes of one word per output (B[k][n] = 1 iff k/4 == n) and C = 0x6400, so
// D[m][n] = 0x6400 + bytesum(word (m, n)): the fp16 bit pattern of 1024 + s. Word (m, n) is slot a0 (n < 4) / a2 (n >= 4)
// of lane (m % 8, n % 4) for m < 8, a1 / a3 for m >= 8. With IMMA #1 fed (x0, x4, x1, x5) and IMMA #2 fed
// (x2, x6, x3, x7), lane (g, tq) receives the sums of tile positions (rows rho(2tq), rho(2tq+1) [+8 for IMMA #2],
// columns g and g+8), rho(n) = 2n for n < 4, 2(n-4)+1 otherwise. Output columns stay the lane's own (g, g+8); the
// tile rows arrive permuted, so the activations (B operand of the following f16 MMA) are stored with the rows of each
// 16-row tile in the order PERM16 below: B-fragment k-slot h holds input row PERM16[h].
//   PERM16 = {0, 2, 4, 6, 1, 3, 5, 7, 8, 10, 12, 14, 9, 11, 13, 15}
__host__ __device__ constexpr int perm16(int h) { return (h & 8) | ((h & 4) ? (((h & 3) << 1) | 1) : ((h & 3) << 1)); }
// position h of input row r within its 16-row tile (inverse of perm16)
__host__ __device__ constexpr int perm16_inv(int r) { return (r & 8) | ((r & 1) ? (4 | ((r & 7) >> 1)) : ((r & 7) >> 1)); }

// Position (in fp16 elements) of input k (0..127) of a 128-input block in the EXACT GEMV's activation layout: for each
// pair of 16-row tile rows (r = 2 rp, 2 rp + 1) and each lane quad tq, the 8 values that lane (g, tq) multiplies with its
// decode_frag_tc weights: rows PERM16(2tq), PERM16(2tq+1), PERM16(2tq)+8, PERM16(2tq+1)+8 of tile row 2 rp, then of
// tile row 2 rp + 1. A lane reads them with one 16-byte load; the four quads read one contiguous 64-byte run.
__host__ __device__ constexpr int gemv_xpos(int k)
{
    return (k >> 5) * 32 + (((perm16_inv(k & 15) & 7) >> 1) * 8) + (((k >> 4) & 1) * 4) + ((perm16_inv(k & 15) & 1) |
           ((perm16_inv(k & 15) >> 3) << 1));
}

__device__ __forceinline__ void imma_bytesum(uint32_t d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1, uint32_t c)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}

struct OnesFrag
{
    uint32_t b0, b1;
    __device__ __forceinline__ void init(int lane)
    {
        const int g = lane >> 2, tq = lane & 3;
        b0 = (g == tq) ? 0x01010101u : 0u;
        b1 = (g == 4 + tq) ? 0x01010101u : 0u;
    }
};

// The 8 product words x_j = state_j * MUL1 (mod 2^32) of a lane's stream weights from its two stream words (hi = word at
// off_hi, lo = word at off_lo); the codebook value of weight j is a function of bytesum(x_j) (ft_core.h:75-83). The
// window is first shifted to bit 0 (clamped funnel shifts: pre may be 32); states that lie in the low word then need
// a plain shift (none for j = 7), the others a funnel shift.
template <int K>
__device__ __forceinline__ void decode_words_from(uint32_t hi, uint32_t lo, const LaneDecode<K>& L, uint32_t x[8])
{
    const uint32_t lo2 = __funnelshift_rc(lo, hi, L.pre);
    const uint32_t hi2 = __funnelshift_rc(hi, 0u, L.pre);
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        const int sh = K * (7 - j);
        const uint32_t st = sh == 0 ? lo2 : (sh + 16 <= 32 ? lo2 >> sh : __funnelshift_r(lo2, hi2, sh));
        x[j] = (st & 0xffffu) * MUL1;
    }
}

// decode_words_from reading the lane's two words of the tile at `tile` (shared memory)
template <int K>
__device__ __forceinline__ void decode_words(const uint8_t* tile, const LaneDecode<K>& L, uint32_t x[8])
{
    decode_words_from<K>(lds32(tile + L.off_hi), lds32(tile + L.off_lo), L, x);
}

// mma.m16n8k32, A = product bytes (u8), B = activation planes (s8), exact int32 accumulation
__device__ __forceinline__ void imma_u8s8(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same A fragment as decode_frag but with the rows of the tile permuted by PERM16 (see above).
template <int K>
__device__ __forceinline__ void decode_frag_tc(const uint8_t* tile, const LaneDecode<K>& L, const OnesFrag& ones, uint32_t a[4])
{
    uint32_t x[8];
    decode_words<K>(tile, L, x);
    uint32_t d1[4], d2[4];
    imma_bytesum(d1, x[0], x[4], x[1], x[5], ones.b0, ones.b1, 0x6400u);
    imma_bytesum(d2, x[2], x[6], x[3], x[7], ones.b0, ones.b1, 0x6400u);
    a[0] = codebook_pair(d1[0], d1[1]);
    a[1] = codebook_pair(d1[2], d1[3]);
    a[2] = codebook_pair(d2[0], d2[1]);
    a[3] = codebook_pair(d2[2], d2[3]);
}

// Decoded fp16 weights of one tile as an m16n8k16 A fragment of the transposed tile (rows = output columns n, columns =
// inputs k) in NATURAL input order: the trellis stream order is that fragment layout (ft_core.h:48-61 PERM: lane
// (g, tq)'s stream weights 8*lane .. 8*lane+7 sit at (k, n) = (2tq, g), (2tq+1, g), (2tq+8, g), (2tq+9, g), then the
// same k at n = g+8). Byte sums on the integer pipe (dp4a against 0x01010101, accumulated onto 0x6400 so each sum is
// the fp16 pattern of 1024 + s), then the codebook FMA per pair.
template <int K>
__device__ __forceinline__ void decode_frag_nat(uint32_t hi, uint32_t lo, const LaneDecode<K>& L, uint32_t a[4])
{
    uint32_t x[8];
    decode_words_from<K>(hi, lo, L, x);
    uint32_t s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = (uint32_t) __dp4a(x[j], 0x01010101u, 0x6400u);
    a[0] = codebook_pair(s[0], s[1]);     // n = g,     k = 2tq, 2tq+1
    a[1] = codebook_pair(s[4], s[5]);     // n = g + 8, k = 2tq, 2tq+1
    a[2] = codebook_pair(s[2], s[3]);     // n = g,     k = 2tq+8, 2tq+9
    a[3] = codebook_pair(s[6], s[7]);     // n = g + 8, k = 2tq+8, 2tq+9
}

// ---- hyper-connection update of one column (exllamav3 hc_apply; glm53/k_hcfuse.py:62-91) --------------------------
// x_row: the row's 4 streams [4][D]; x_g <- post_g * y + comb[0][g] * x_0 + ... + comb[3][g] * x_3, the products
// accumulated by fma in stream order h = 0..3 starting from post_g * y (the reference's expressions and order).
__device__ __forceinline__ void hc_apply_col(float* x_row, int D, int c, float y, const float* post, const float* comb)
{
    float xv[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) xv[h] = x_row[(size_t) h * D + c];
#pragma unroll
    for (int g = 0; g < 4; ++g)
    {
        float o = __fmul_rn(post[g], y);
#pragma unroll
        for (int h = 0; h < 4; ++h) o = __fmaf_rn(comb[h * 4 + g], xv[h], o);
        x_row[(size_t) g * D + c] = o;
    }
}

// hc_mix_partials of one (row, stream, 128-column block) on a warp whose lane l holds the updated column quad
// jb * 32 + l of that stream (glm53/k_hcfuse.py:92-126): per lane the sum of squares (fma chain from 0) and s . fn_j for
// the 24 mix rows (fma chain from s.w * w.w, added to 0), then the warp's shfl_down tree; lane 0 stores the 25 sums at
// part[0..24]. fn_q points at the quad's 4 weights of mix row 0, rows fn_row elements apart. All 32 lanes must be active.
__device__ __forceinline__ void hc_mix_warp(float4 s, const __half* fn_q, size_t fn_row, float* part, int lane)
{
    float acc[25];
    acc[24] = 0.0f;
    acc[24] = fmaf(s.x, s.x, acc[24]);
    acc[24] = fmaf(s.y, s.y, acc[24]);
    acc[24] = fmaf(s.z, s.z, acc[24]);
    acc[24] = fmaf(s.w, s.w, acc[24]);
#pragma unroll
    for (int j = 0; j < 24; ++j)
    {
        const uint2 pk = *reinterpret_cast<const uint2*>(fn_q + (size_t) j * fn_row);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&pk.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&pk.y));
        acc[j] = 0.0f + fmaf(s.x, lo.x, fmaf(s.y, lo.y, fmaf(s.z, hi.x, __fmul_rn(s.w, hi.y))));
    }
#pragma unroll
    for (int k = 0; k < 25; ++k)
    {
        float v = acc[k];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
        if (lane == 0) part[k] = v;
    }
}

// ---- 128-point transforms on one warp (lane holds v[q] = element lane + 32 q) ------------------------------------------

// Unnormalised Walsh-Hadamard butterfly in the reference's stage order w = 1, 2, ..., 64 (ft_core.h:89-94):
// v[i] = a + c, v[i + w] = a - c with a = v[i], c = v[i + w]. Same fp32 operations, same order.
__device__ __forceinline__ void had128_warp(float v[4], int lane)
{
#pragma unroll
    for (int w = 1; w < 32; w <<= 1)
    {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int q = 0; q < 4; ++q)
        {
            const float o = __shfl_xor_sync(0xffffffffu, v[q], w);
            v[q] = upper ? (o - v[q]) : (v[q] + o);
        }
    }
    {   // w = 32: pairs (q0, q1), (q2, q3)
        const float a0 = v[0], c0 = v[1], a1 = v[2], c1 = v[3];
        v[0] = a0 + c0; v[1] = a0 - c0; v[2] = a1 + c1; v[3] = a1 - c1;
    }
    {   // w = 64: pairs (q0, q2), (q1, q3)
        const float a0 = v[0], c0 = v[2], a1 = v[1], c1 = v[3];
        v[0] = a0 + c0; v[2] = a0 - c0; v[1] = a1 + c1; v[3] = a1 - c1;
    }
}

__device__ __forceinline__ float r16(float f) { return __half2float(__float2half_rn(f)); }

// silu(g) * u with the reference's optional clamp (ft_core.h:122-132). exp is evaluated in double and rounded, so the
// fp32 value matches a correctly rounded expf.
__device__ __forceinline__ float act_mul(float g, float u, float limit)
{
    const float e = (float) exp(-(double) g);
    float x = g / (1.0f + e);
    if (limit != 0.0f) { u = fminf(fmaxf(u, -limit), limit); x = fminf(x, limit); }
    return x * u;
}

}  // namespace glmx
