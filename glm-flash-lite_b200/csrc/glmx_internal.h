// Internal (non-ABI) declarations shared by the .cu files of libglmx.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "glmx.h"

namespace glmx {

// Registered layer: device pointer tables of an HBM-resident expert bank (one entry per expert; the shared expert,
// when present, is the last entry).
struct Layer
{
    int H = 0, I = 0, E = 0, E_total = 0, has_shared = 0;
    int bits[3] = { 3, 3, 3 };
    float act_limit = 0.0f;
    int first = 0;                     // global id of routed expert 0 (expert-parallel shards)
    int device = 0;
    uint64_t* d_trellis = nullptr;     // device [E_total][3] addresses (gate, up, down)
    const uint16_t* suh[3] = {};       // device fp16 [E_total][k]
    const uint16_t* svh[3] = {};       // device fp16 [E_total][n]
    CUtensorMap* d_tmaps = nullptr;    // device [E_total][3] tensor maps of the trellis tensors (GEMV stage boxes)
};

// tensor map of one trellis tensor [k x n] at `base` for the GEMV kernels (boxes of 8 k-tile rows x 8 tiles)
cudaError_t trellis_map(CUtensorMap* m, const void* base, int k, int n, int bits);

// Per-call routing plan, written by the route kernel and read by the later kernels.
struct Plan
{
    int P;       // valid routed picks (rows 0..P-1, expert-major)
    int R;       // rows including the shared expert's rows
    int J;       // jobs (<= MAXM rows of one expert)
    int S_gu;    // split-K of the gate/up kernel
    int S_d;     // split-K of the down kernel
    int ntok, topk, pad;
    int next_gu, next_d;   // item counters of the I16 gate/up and down GEMVs (zeroed here, taken by their CTAs)
};

// Workspace layout of one forward call (byte offsets from the workspace base, 256-byte aligned).
struct WsLayout
{
    size_t plan, err, offsets, row_token, row_expert, row_pick, row_weight, pick_row, jobs, row_job;
    size_t cnt_gu, cnt_d, xg, xu, xd, yrow, partials;
    // I16 mode
    size_t actb_gu, psum_gu, yraw_gu, actb_d, psum_d, isum_gu;
    size_t total;
    int rows_max, jobs_max, jobs_max_i16;
    size_t part_bytes;        // EXACT split-K partial sums: [split][row][matrix][column] (hi, lo) pairs
};

WsLayout ws_layout(const Layer& L, int ntok, int topk, int grid_ctas);

// grid size of the persistent GEMV kernels on the current device
int gemv_grid_ctas(const Layer& L);   // resident CTAs of the EXACT GEMV grid
int gemv_sm_count(const Layer& L);
int i16_grid_ctas(const Layer& L);    // resident CTAs of the I16 GEMV grid

void set_error(const std::string& msg);

// Hyper-connection epilogue of the combine (exllamav3 hc_apply as glm53/k_hcfuse.py:62-91 restates it): instead of
// writing the layer output y, update the row's stream stack in place, x_g <- post_g * y + sum_h comb[h][g] * x_h.
// Expert-parallel return (glmx_peer_out of glmx.h): instead of writing out, the combine stores token t's fp32 row into
// rank t / rpr's receive buffer, slot [seq & 1][rank][t % rpr], over peer memory; the combine's last CTA then sets
// flag [seq & 1][rank] = seq on every rank.
struct PeerOut
{
    float* const* recv;    // device array [world]: each rank's float [2][world][rpr][H]
    int* const* flags;     // device array [world]: each rank's int [2][world]
    int* counter;          // this rank's arrival counter (zero between calls)
    int rank, world, rpr, seq;
};

struct HcOut
{
    float* x;              // [ntok][4][H] fp32 stream stack, updated in place
    const float* post;     // [ntok][4]
    const float* comb;     // [ntok][4][4], comb[h][g]
    int y_half;            // 1: y is rounded to fp16 first (an fp16 sublayer output), 0: fp32
    PeerOut peer;          // peer.recv != nullptr (and x == nullptr): expert-parallel return instead of out
    const __half* fn;      // != nullptr: also the next site's hc_mix_partials of the updated stack: fn [24][4H] fp16
    float* part;           // [ntok][4H/128][25] fp32 mix partial sums
};

// A kernel launch that may overlap the previous kernel of the stream (programmatic dependent launch); the kernel must
// begin with pdl_enter().
template <typename... P, typename... A>
cudaError_t launch_chained(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// 128-input blocks per pipeline stage of the EXACT GEMV of projection proj (0: gate/up over H, 2: down over I): 2 where
// the matrices' bitrates are at most 3 and K is a multiple of 256 (a stage of two blocks fits the ring three times),
// else 1. The split plan counts K splits in these stages.
int exact_stage_blocks(const Layer& L, int proj);

// launchers (return cudaError_t of the launch)
cudaError_t launch_route(const Layer& L, const void* sel, int sel_i64, const void* w, int w_dtype, int ntok, int topk,
                         int maxm, uint8_t* ws, const WsLayout& lay, int grid_ctas, cudaStream_t st);
cudaError_t launch_decode_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, int mode, void* out,
                                  int out_dtype, int accumulate, uint8_t* ws, const WsLayout& lay, int grid_ctas,
                                  cudaStream_t st, void* const* events, const HcOut* hc = nullptr);
cudaError_t launch_i16_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, void* out, int out_dtype,
                               int accumulate, uint8_t* ws, const WsLayout& lay, cudaStream_t st, void* const* events,
                               const HcOut* hc = nullptr);
cudaError_t launch_decode_tiles(const uint8_t* tiles, int bits, int ntiles, uint16_t* out, cudaStream_t st);
// prefill path (tensor-core GEMM, EXACT mode) and the two kernels it shares with the GEMV paths
cudaError_t launch_prefill_forward(const Layer& L, const void* x, int x_dtype, int ntok, int topk, void* out, int out_dtype,
                                   int accumulate, uint8_t* ws, const WsLayout& lay, cudaStream_t st, void* const* events,
                                   const HcOut* hc = nullptr);
// EXACT input transform of every row (xg, xu: fp16 [R][H]; PERM16 order inside 16-row tiles for the GEMV kernels,
// natural order for the tensor-core GEMM)
cudaError_t launch_prep_exact(const Layer& L, const void* x, int x_dtype, int ntok, int topk, uint8_t* ws, const WsLayout& lay,
                              cudaStream_t st, bool natural);
// down out_block of raw fp32 rows [R][H] + weighted sum in pick order (+ shared expert) into out
cudaError_t launch_combine_raw(const Layer& L, const float* yraw, int ntok, int topk, void* out, int out_dtype, int accumulate,
                               uint8_t* ws, const WsLayout& lay, cudaStream_t st, const HcOut* hc = nullptr);

// hyper-connection site kernels (hc.cu): hc_apply (apply != 0) + hc_mix_partials (part != nullptr) over R rows of
// [4][D] stream stacks; hc_mix_finalize + RMSNorm
cudaError_t launch_hc_apply_partials(float* x, const void* y, int y_half, const float* post, const float* comb,
                                     const __half* fn, float* part, int R, int D, int apply, cudaStream_t st);
cudaError_t launch_hc_finalize(const float* x, const float* part, const float* base, const float* scale, float* post,
                               float* comb, const void* nw, int nw_bf16, __half* out, int R, int D, float rms_eps,
                               float hc_eps, int iters, float n_eps, float cbias, float cscale, cudaStream_t st);

constexpr int I16_MAXM = 4;            // rows per job in I16 mode (one 4-token activation set)
constexpr int EXACT_MAXM = 8;         // rows per job of the EXACT decode GEMV (the 8 token columns of one MMA)
constexpr int I16_ACT_BYTES = 4096;    // replicated activation planes of one (job, projection, 128-input block)
// one (job, 128-input block) record of the I16 activations, laid out as a GEMV stage holds it: the nmat projections'
// planes, then their 4 scales (16 bytes each)
__host__ __device__ constexpr size_t i16_rec_bytes(int nmat) { return (size_t) nmat * (I16_ACT_BYTES + 16); }
constexpr int I16_MAX_ROWS = 8192;     // I16 is the decode mode: its activation layout is sized for up to this many rows
constexpr int I16_SPLIT_MAX_ROWS = 16; // calls this small split the I16 gate/up GEMV along K (exact int32 block sums)
constexpr int PF_MAXM = 128;           // rows per job of the prefill GEMM (one tensor-core tile)
constexpr int PF_AUTO_ROWS_PER_EXPERT = 12;   // EXACT mode takes the GEMM path from this many rows per expert on average
constexpr int PF_KSPLIT = 3;           // K splits of the prefill gate/up GEMM (partial sums added in order in fp32)

}  // namespace glmx
