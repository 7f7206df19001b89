/* Test infrastructure only: CPU restatement of the reference's routed-expert path.
 *
 * This is the checker for the CUDA product in glm-flash-lite_b200/. Only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline leg of bench.py may load it. Nothing in the product links it.
 *
 * Every function restates code from nkeilar/glm-flash-lite kernels/cpu_avx2/ft_core.h (cited per function).
 * The trellis bit width K is a parameter here; the reference fixes K=3 (ft_core.h:30-31). K=2/4 follow the
 * same formula with K substituted and are not pinned by anything in the reference tree.
 */
#ifndef FT_ORACLE_H
#define FT_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* PERM table, ft_core.h:48-61 (stream index -> r*16 + c inside the 16x16 tile) */
void fto_init(void);
int fto_perm(int i);

/* ft_core.h:65-73 with BITS -> K: 16-bit trellis state of stream weight t of one tile (32*K bytes) */
uint16_t fto_state(const uint8_t* tile, int K, int t);
/* ft_core.h:75-79 */
int fto_bytesum(uint16_t st);
/* ft_core.h:81-83: fp16 bits of fp16(fma(1024 + s, KINV, KBIAS)) */
uint16_t fto_codebook_h(int s);

/* one tile -> 256 fp16 bit patterns in (r, c) row-major order, r = input row, c = output column */
void fto_decode_tile(const uint8_t* tile, int K, uint16_t* w16);
/* ft_core.h:1657-1672 dense_weights: [k][n] fp32 (fp16-valued) from a native-layout trellis tensor */
void fto_dense(const uint8_t* tr, int K, int k, int n, float* W);

/* fp16 helpers (IEEE binary16, round to nearest even) */
uint16_t fto_f2h(float f);
float fto_h2f(uint16_t h);

/* ft_core.h:89-110 transforms on one 128-block */
void fto_had128(float* v);
void fto_prep_block(const float* x, const uint16_t* suh, float* xt);
void fto_out_block(float* y, const uint16_t* svh);
/* ft_core.h:122-132 act_mul; limit 0 = off */
float fto_act_mul(float g, float u, float limit);

/* One EXL3 linear in the reference's "GPU-exact weights, fp64 accumulation" form (ft_core.h:1674-1682).
 * mode 1 = EXACT (fp16-rounded codebook weights), mode 0 = AFFINE (unrounded codebook KINV*(1024+s)+KBIAS).
 * x: [m][k] fp16-valued fp32, y: [m][n]. W may be NULL (decoded on the fly) or a dense [k][n] array that
 * matches the mode. */
void fto_linear(const uint8_t* tr, int K, const uint16_t* suh, const uint16_t* svh, int k, int n,
                const float* W, int mode, const float* x, int m, float* y);

/* ft_core.h:1684-1691 ref_expert for m tokens: y[m][H] from x[m][H] (fp16-valued fp32) */
typedef struct {
    const uint8_t* tr[3];        /* gate, up, down trellis, native layout */
    const uint16_t* suh[3];      /* fp16 [k] per projection */
    const uint16_t* svh[3];      /* fp16 [n] per projection */
    int K[3];                    /* bits per weight per projection */
} fto_expert_t;
void fto_expert(const fto_expert_t* ex, int H, int I, int mode, float act_limit, const float* x, int m, float* y);

/* Expert-major grouping of the routed picks (ft_core.h:1344-1349 job rule, canonical expert-ascending form).
 * sel/w: [ntok][topk]; picks with sel < 0 or sel >= E are skipped.
 * outputs: offsets[E+1], row_token[P], row_weight[P], row_pick[P] (pick index t*topk+kk), pick_row[ntok*topk]
 * (-1 for skipped picks). Returns P (number of valid picks). */
int fto_group(const int32_t* sel, const float* w, int ntok, int topk, int E,
              int32_t* offsets, int32_t* row_token, float* row_weight, int32_t* row_pick, int32_t* pick_row);

/* The reference's own job list (ft_core.h:1344-1349): first-touch expert order, <= maxm tokens per job.
 * job_e/job_m: [njobs], job_tok/job_w: [njobs][maxm]. Returns njobs. */
int fto_jobs_ref(const int32_t* sel, const float* w, int ntok, int topk, int E, int maxm,
                 int32_t* job_e, int32_t* job_m, int32_t* job_tok, float* job_w);

/* I16 mode (the reference's mode 2, ft_core.h:418-598): per 128-input block the transformed activations are quantised
 * to int16 with scale amax / 16383 (quant_block_i16, ft_core.h:583-598); each output column keeps four fp32
 * accumulators, one per tile-row class {0,2,4,6}, {1,3,5,7}, {8,10,12,14}, {9,11,13,15} (the four AVX lanes of
 * tile_accum_i16), each fed once per block with fma(float(exact int32 block sum of bytesum * xi), scale, acc)
 * (gemv_block_i16, ft_core.h:497-541); out = KINV * ((a0 + a1) + (a2 + a3)) + CAFF * sumx. Weights are unrounded
 * codebook values (AFFINE). Same algorithm as the reference at any H; the reference's own scratch is sized for
 * H / 128 <= 32 blocks (ft_core.h:1353), this restatement is not. */
void fto_expert_i16(const fto_expert_t* ex, int H, int I, float act_limit, const float* x, int m, float* y);

/* Whole layer: out[t] = sum over token t's picks in pick order of w * expert(x[t]) (fp32, ft_core.h:1020-1033
 * with the sum taken in pick order), plus the shared expert (weight 1) when shared != NULL. */
/* mode 0 AFFINE, 1 EXACT (fp64 accumulation), 2 I16 */
void fto_moe_forward(const fto_expert_t* experts, int E, const fto_expert_t* shared, int H, int I, int mode,
                     float act_limit, const float* x, int ntok, const int32_t* sel, const float* w, int topk, float* out);

/* Hyper-connection update after the MoE sublayer (exllamav3 hc_apply as glm53/k_hcfuse.py:62-91 restates it):
 * x [R][4][D] fp32 updated in place, y [R][D] the sublayer output (already in the precision the model feeds it),
 * post [R][4], comb [R][4][4] (comb[h][g]): x_g <- fma(comb[3][g], x_3, ... fma(comb[0][g], x_0, post_g * y)). */
void fto_hc_apply(float* x, const float* y, int R, int D, const float* post, const float* comb);

/* hc_mix_partials of the next site (glm53/k_hcfuse.py:92-126): for row r, stream g and 128-column block jb, the 25
 * sums over the block's 32 column quads (lane l = quad jb*32 + l) of s.fn_j (j < 24, fn [24][4D] fp16, 4-term fma
 * chain from s.w*w.w) and of s.s (fma chain from 0), each reduced over the 32 lanes by the warp's shfl_down tree.
 * part [R][4 D/128][25], index (r * 4 D/128 + g * D/128 + jb) * 25 + k. */
void fto_hc_mix_partials(const float* x, const uint16_t* fn, int R, int D, float* part);

/* hc_mix_finalize + RMSNorm of the collapsed row (glm53/k_hcfuse.py:129-294), in plain fp32 math (expf, 1/sqrtf,
 * IEEE division: the reference's fast intrinsics are not restated, so this is a tolerance check): mix = the chunk sums
 * of part (chunk k = (0 + half 2k) + half 2k+1, warp w sums chunks w, w+8, ..., then the 8 warps in order);
 * rmr = 1/sqrt(mix[24] / 4D + rms_eps); post = 2 sigmoid(mix[4+g] rmr scale[1] + base[4+g]); comb = Sinkhorn
 * (softmax over g per h, + hc_eps, column-normalised, iters - 1 more row/column rounds) of mix[8+4h+g] rmr scale[2] +
 * base[8+4h+g]; pre = sigmoid(mix[h] rmr scale[0] + base[h]) + hc_eps; out = fp16(c * (nw + cbias) * rmf) with
 * c = clamp(fp16(sum_h pre_h x_h)) and rmf = cscale / sqrt(sum c^2 / D + n_eps). nw fp32 values [D]. */
void fto_hc_finalize_norm(const float* x, const float* part, int R, int D, const float* base, const float* scale,
                          const float* nw, float rms_eps, float hc_eps, int iters, float n_eps, float cbias, float cscale,
                          float* post, float* comb, uint16_t* out);

/* Router in front of the split: the GLM-4 MoE routing of exllamav3's router (un-vendored third-party code), as the
 * published model code states it (transformers, models/glm4_moe/modeling_glm4_moe.py:302-305 and 389-412).
 * fto_router_gate: logits[t][e] = sum_h z[t][h] * W[e][h], accumulated in fp64 and rounded once (the reference
 * accumulates in fp32 in an order of its own; this is the exact value it approximates).
 * fto_router_select: s = sigmoid(logit) = 1 / (1 + e^-logit) with e^y from a fixed fp32 sequence (Cody-Waite reduction,
 * degree-8 Taylor polynomial; fto_router_sigmoid exposes it), c = s + bias; n_group > 1: group score = sum of
 * the two largest c of each group, c = 0 outside the topk_group best groups; picks = topk largest c in descending
 * order (equal values: smaller id first); w = s[pick], norm: w / (sum in pick order + 1e-20), then * scale. */
void fto_router_gate(const float* z, int ntok, int H, const float* W, int E, float* logits);
void fto_router_sigmoid(const float* x, int n, float* out);
void fto_router_select(const float* logits, int ntok, int E, const float* bias, int n_group, int topk_group, int topk,
                       int norm, float scale, int32_t* sel, float* w);

#ifdef __cplusplus
}
#endif
#endif
