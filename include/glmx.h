/* glmx - B200 (sm_100a) routed-expert MoE layer over EXL3 trellis-coded experts.
 *
 * C ABI of libglmx.so. Plain pointers and sizes; every device pointer is a CUDA device address on the current
 * device, `stream` is a cudaStream_t (NULL = the legacy default stream). Every entry point returns 0 on success and
 * a negative GLMX_E_* code on failure; glmx_last_error() then describes the failure (thread-local).
 * Nothing here allocates device memory except glmx_layer_create (the layer's pointer tables). Scratch memory of a
 * forward call is the caller's workspace (glmx_workspace_bytes).
 *
 * Each entry point names the reference interface it replaces (nkeilar/glm-flash-lite, file:line).
 */
#ifndef GLMX_H
#define GLMX_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLMX_ABI_VERSION 2

#if defined(__GNUC__)
#define GLMX_API __attribute__((visibility("default")))
#else
#define GLMX_API
#endif

#define GLMX_OK 0
#define GLMX_E_ARG -1       /* invalid argument or shape */
#define GLMX_E_CUDA -2      /* CUDA runtime error (launch or memory) */
#define GLMX_E_DEVICE -3    /* a device-side check failed (bounded wait expired, bad expert id): see glmx_check */
#define GLMX_E_WORKSPACE -4 /* workspace too small */

/* dtypes */
#define GLMX_F16 0
#define GLMX_F32 1
#define GLMX_BF16 2
#define GLMX_I32 3
#define GLMX_I64 4

/* numeric modes, same numbering as the reference's moe_forward (kernels/cpu_avx2/ft_core.h:822-823) */
#define GLMX_MODE_EXACT 1   /* fp16-rounded codebook weights, fp16 x fp16 products accumulated in fp32 (decode GEMV:
                               one tensor-core MMA per 16x16 tile started from zero, tile sums added in fp32 with
                               compensated block sums; prefill GEMM: short tensor-memory accumulation chains) */
#define GLMX_MODE_I16 2     /* int16 activations per 128-block, exact integer tensor-core sums, the reference's fp32
                               flush order (ft_core.h:418-598): bit-identical to the reference's I16 mode. The decode
                               mode: at most 8192 rows (picks + shared-expert rows) per call */
/* Path selection, OR'ed into the mode (EXACT only; default: chosen from the batch): GEMV = the decode kernels (one pass
 * over each expert's trellis per job of <= 8 rows); GEMM = the prefill kernels (tcgen05 tensor-core GEMM over jobs of
 * <= 128 rows, trellis decoded into shared memory once per 128-row tile), the default once the call has >= 12 rows per
 * expert on average. The reference's large-batch schedule is moe_forward_band (ft_core.h:1617-1651). */
#define GLMX_PATH_GEMV 0x100
#define GLMX_PATH_GEMM 0x200

typedef struct glmx_layer glmx_layer;

/* One MoE layer's routed experts (+ optional shared expert as the last entry), HBM-resident, native EXL3 layout:
 * tile (tk, tn) of a [k x n] projection at byte (tk * (n/16) + tn) * 32 * bits. Replaces the registration of
 * tier_add_layer(li, ptrs int64 [E,3], suh_g, svh_g, suh_u, svh_u, suh_d, svh_d) (kernels/cpu_avx2/ft_tier_ext.cpp:160-183)
 * and the per-expert pointer tables exllamav3 keeps (ptrs_trellis, glm53/expert_cache.py:603-616). */
typedef struct
{
    int hidden;                       /* H, multiple of 128 */
    int intermediate;                 /* I, multiple of 128 */
    int n_experts;                    /* routed experts E (<= 1024) */
    int has_shared;                   /* 1: a shared expert is stored as entry E */
    int bits[3];                      /* trellis bits per weight of gate, up, down: 2, 3 or 4 */
    const uint64_t* trellis;          /* HOST array [(E + has_shared) * 3] of device addresses (gate, up, down), 16-byte aligned */
    const void* suh[3];               /* device fp16 [(E + has_shared), k] input sign/scale vectors per projection */
    const void* svh[3];               /* device fp16 [(E + has_shared), n] output scale vectors per projection */
    float act_limit;                  /* SwiGLU clamp (0 = off), tier_set_act_limit (ft_tier_ext.cpp:635) */
    int first_expert;                 /* global id of routed expert 0 of this layer (an expert-parallel shard holds
                                         ids [first_expert, first_expert + n_experts)); picks are read as
                                         sel - first_expert. ft_split's `first` / the module's `routing_first`
                                         (kernels/cpu_avx2/ft_tier_cu.cu:22, glm53/cpu_tier.py:293-299) */
} glmx_layer_desc;

/* No counterpart: the ABI version (GLMX_ABI_VERSION-checked by the Python loader) and the calling thread's last error
 * message. The reference raises its argument errors as TORCH_CHECK RuntimeErrors (kernels/cpu_avx2/ft_tier_ext.cpp:143,
 * 166); here every entry returns a GLMX_E_* status and leaves the message for glmx_last_error. */
GLMX_API int glmx_version(void);
GLMX_API const char* glmx_last_error(void);

/* tier_add_layer (kernels/cpu_avx2/ft_tier_ext.cpp:160-183): registers one layer's expert pointer table and scales.
 * The trellis tensors stay the caller's (borrowed, as the reference keeps them alive with T->keep, 154, 184). */
GLMX_API int glmx_layer_create(const glmx_layer_desc* desc, glmx_layer** out);
/* The per-layer part of tier_stop (kernels/cpu_avx2/ft_tier_ext.cpp:837): frees the layer's device table and tensor maps. */
GLMX_API int glmx_layer_destroy(glmx_layer* layer);
/* No counterpart (the reference's tier is one process-wide CPU pool): the CUDA device index the layer was created on
 * (the current device at glmx_layer_create), or GLMX_E_ARG for a null layer. */
GLMX_API int glmx_layer_device(const glmx_layer* layer);
/* tier_set_act_limit (kernels/cpu_avx2/ft_tier_ext.cpp:635) */
GLMX_API int glmx_layer_set_act_limit(glmx_layer* layer, float limit);

/* Bytes of caller-provided device workspace a forward over `ntok` tokens with `topk` picks each needs. No counterpart:
 * tier_forward allocates its output per call (torch::zeros, kernels/cpu_avx2/ft_tier_ext.cpp:895); here the caller owns
 * all device memory, allocated once and reused, so a forward allocates nothing. */
GLMX_API size_t glmx_workspace_bytes(const glmx_layer* layer, int ntok, int topk);

/* Top-k token split: expert-major grouping of the picks into the workspace (offsets [E+1], rows sorted by
 * (expert, token), pick -> row map, jobs of <= 8 rows; glmx_moe_forward uses jobs of <= 8 rows on its EXACT decode
 * path, <= 4 in I16 mode, <= 128 on the GEMM path). Replaces ft_split (kernels/cpu_avx2/ft_tier_cu.cu:238-271,
 * kernels/k110/ft_split_fast.cu:200-235) and the job grouping of moe_forward (kernels/cpu_avx2/ft_core.h:1344-1349).
 * sel: device [ntok, topk] int32 or int64 (sel_dtype GLMX_I32 / GLMX_I64) of global expert ids; ids outside
 * [first_expert, first_expert + E) are skipped (negative ids mask a pick).
 * w: device [ntok, topk] fp32 / fp16 / bf16. */
GLMX_API int glmx_route(const glmx_layer* layer, const void* sel, int sel_dtype, const void* w, int w_dtype, int ntok, int topk,
               void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart (the split's outputs in the reference are ft_split's sel_out / w_out / hpicks,
 * kernels/cpu_avx2/ft_tier_cu.cu:238-271). Locate one routing array inside a workspace filled by glmx_route (for tests
 * and callers that reuse the split):
 * which = 0 offsets int32 [E+1], 1 row_token int32 [R], 2 row_weight fp32 [R], 3 pick_row int32 [ntok*topk],
 * 4 jobs int32x4 [J] (expert, row0, m, 0), 5 plan int32 [8] (P, R, J, S_gu, S_d, ntok, topk, 0; two internal item
 * counters of the I16 GEMVs follow), 6 row_pick int32 [R]. */
GLMX_API int glmx_workspace_array(const glmx_layer* layer, int ntok, int topk, int which, size_t* offset_bytes);

/* Whole routed-MoE layer on the GPU: split -> gate/up dequant-GEMV + SiLU*up -> down dequant-GEMV -> weighted
 * combine (+ shared expert, weight 1). out [ntok, H] (fp32 or fp16) = sum over token picks of w * expert(x) + shared(x);
 * accumulate = 1 adds into out instead (ft_combine's `out += partial`, kernels/cpu_avx2/ft_tier_cu.cu:226-233).
 * Replaces tier_forward(li, x fp32 [m,H], sel int32 [m,k], w fp32 [m,k], mode) (kernels/cpu_avx2/ft_tier_ext.cpp:865-904)
 * and the GPU expert path it stands beside (exllamav3 BlockSparseMLP experts). x: device [ntok, H] fp16 / fp32 / bf16. */
GLMX_API int glmx_moe_forward(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                     const void* w, int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate,
                     void* workspace, size_t workspace_bytes, void* stream);

/* The per-phase timers of tier_stats (kernels/cpu_avx2/ft_tier_ext.cpp:906-914) as CUDA events:
 * glmx_moe_forward that also records `events` (GLMX_PHASES cudaEvent_t, or NULL entries to skip) on `stream` before the
 * split, after the split, after the input transform, after gate/up, after down and after the combine, so a caller
 * can time each kernel on the launching stream. */
#define GLMX_PHASES 6
GLMX_API int glmx_moe_forward_timed(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                     int sel_dtype, const void* w, int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate,
                     void* workspace, size_t workspace_bytes, void* stream, void* const* events);

/* glmx_moe_forward followed, in the combine kernel itself, by the hyper-connection update that comes right after the
 * MoE sublayer in GLM-5.3 (exllamav3 hc_apply, fused by the reference into k_apply_partials: glm53/k_hcfuse.py:62-91):
 * for every token t and column c, with y the layer output (rounded to fp16 first when y_dtype is GLMX_F16, as an fp16
 * sublayer output is) and x the token's 4-stream stack,
 *     x[t][g][c] <- post[t][g] * y + comb[t][0][g] * x[t][0][c] + ... + comb[t][3][g] * x[t][3][c]   (g = 0..3)
 * with the products added by fma in stream order (the reference's expressions). hc_x: device fp32 [ntok][4][H],
 * updated in place; hc_post: fp32 [ntok][4]; hc_comb: fp32 [ntok][4][4] (comb[h][g]). The layer output itself is not
 * written. Same modes, paths and workspace as glmx_moe_forward. */
GLMX_API int glmx_moe_forward_hc(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                     int sel_dtype, const void* w, int w_dtype, int topk, int mode, float* hc_x, const float* hc_post,
                     const float* hc_comb, int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* glmx_moe_forward_hc followed by the next site's hc_mix_partials of the updated stream stack, as the reference's
 * k_apply_partials does after its hc_apply (glm53/k_hcfuse.py:92-126; replaces ext().apply_partials(x, y, post, comb,
 * fn, partials) with y = this layer's output, glm53/k_hcfuse.py:296-320, called at 427-428): fn fp16 [24][4H] (16-byte aligned), partials fp32
 * [ntok][4H/128][25]: for row t, stream g and 128-column block b the 25 sums at (t*4H/128 + g*H/128 + b)*25 - the 24
 * products s.fn_j and s.s over the block's updated values, bit-identical to the reference's reduction tree. On the EXACT
 * GEMV path this runs inside the combine kernel; the I16 and GEMM paths add one pass over the updated stack. */
GLMX_API int glmx_moe_forward_hc_mix(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                     int sel_dtype, const void* w, int w_dtype, int topk, int mode, float* hc_x, const float* hc_post,
                     const float* hc_comb, int y_dtype, const uint16_t* fn, float* partials, void* workspace,
                     size_t workspace_bytes, void* stream);

/* The reference's fused site kernels on their own (replace ext().apply_partials and ext().finalize_norm,
 * glm53/k_hcfuse.py:296-344, called at 427-432). glmx_hc_apply_partials: with y (fp16 or fp32 [R][D]) the hc_apply update of x fp32
 * [R][4][D] in place (post [R][4], comb [R][4][4]), then the mix partials of the (updated) stack into partials
 * [R][4D/128][25]; y == NULL computes only the partials. D a multiple of 128. Bit-identical to the reference. */
GLMX_API int glmx_hc_apply_partials(float* x, const void* y, int y_dtype, const float* post, const float* comb,
                     const uint16_t* fn, float* partials, int R, int D, void* stream);

/* hc_mix_finalize + the site's RMSNorm (glm53/k_hcfuse.py:129-294): from the partials of glmx_hc_apply_partials, per
 * row the 25 mix sums, rmr = rsqrt(mix[24] / 4D + rms_eps), post [R][4] = 2 sigmoid(mix[4+g] rmr scale[1] + base[4+g]),
 * comb [R][4][4] by Sinkhorn (iters rounds, hc_eps) of mix[8+..] rmr scale[2] + base[8+..], and out fp16 [R][D] = the
 * collapsed row sum_h (sigmoid(mix[h] rmr scale[0] + base[h]) + hc_eps) x_h (rounded to fp16, clamped) normalised by
 * its RMS (n_eps) times cscale and (nw + cbias); nw fp16 or bf16 [D]. D a multiple of 512, at most 16384; for
 * D = 4096 (the size the reference builds it for) bit-identical to the reference. */
GLMX_API int glmx_hc_finalize_norm(const float* x, const float* partials, int R, int D, const float* base,
                     const float* scale, float* post, float* comb, const void* nw, int nw_dtype, uint16_t* out,
                     float rms_eps, float hc_eps, int iters, float n_eps, float cbias, float cscale, void* stream);

/* Known-answer entry for the trellis decode: `ntiles` tiles of 32*bits bytes (device) -> fp16 bit patterns
 * [ntiles, 16, 16] (row r = input index, column c = output index), as dense_weights (kernels/cpu_avx2/ft_core.h:1657-1672). */
GLMX_API int glmx_decode_tiles(const uint8_t* tiles, int bits, int ntiles, uint16_t* out, void* stream);

/* Synchronise `stream` and read the device error word of a workspace (bounded waits that expired, bad expert ids):
 * returns GLMX_OK or GLMX_E_DEVICE; *flags receives the raw bits. The reference surfaces device failures through
 * sticky ctrl words and stats (kernels/cpu_avx2/ft_tier_cu.cu:33-52, 176-193). */
GLMX_API int glmx_check(const glmx_layer* layer, int ntok, int topk, void* workspace, void* stream, int* flags);

/* Failure-detection self-test (no counterpart in the reference, whose device waits also give up after a limit,
 * kernels/cpu_avx2/ft_tier_cu.cu:176-193): launches one warp that runs the library's bounded mbarrier wait on a
 * barrier nothing completes; after timeout_us (1 .. 1e7) it gives up and ORs the timeout bit into the device int
 * *flag (the bit glmx_check reports for a stalled forward). The kernel returns normally; the context stays usable. */
GLMX_API int glmx_selftest_bounded_wait(int timeout_us, int* flag, void* stream);

/* No counterpart (the reference runs every expert of a layer on one GPU and its CPU tier; expert sharding over GPUs is
 * this library's). Expert-parallel return over peer memory. A rank of `world` holds a shard of the experts (first_expert, n_experts)
 * and runs the layer over all ranks' gathered rows, rows_per_rank consecutive rows per rank (ntok = world *
 * rows_per_rank). glmx_moe_forward_peer computes like glmx_moe_forward but, instead of writing `out`, its combine stores
 * token t's fp32 row into rank (t / rows_per_rank)'s receive buffer at [seq & 1][rank][t % rows_per_rank], through the
 * peer mappings, then sets that rank's flag [seq & 1][rank] = seq. glmx_peer_reduce, on the owner, waits for all world
 * flags of call `seq` (bounded: on expiry it ORs 16 into *err and writes nothing) and writes out[r] = the sum of the
 * world rows in rank order. It replaces the reduce-scatter of a plain expert-parallel layer (the reference has no
 * multi-GPU mode). Calls of the same buffers must alternate parity (seq, seq + 1, ...), and a rank may start call seq + 2
 * only after a collective that every owner enters after its call-seq reduce (the next call's dispatch does). */
typedef struct glmx_peer_out {
    void* const* recv;  /* device array [world]: rank d's receive buffer, float [2][world][rows_per_rank][hidden] */
    int* const* flags;  /* device array [world]: rank d's flags, int [2][world], zero before the first call */
    int* counter;       /* this rank's device int, zero before the first call (left zero after each call) */
    int rank, world, rows_per_rank, seq;
} glmx_peer_out;
GLMX_API int glmx_moe_forward_peer(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                                   int sel_dtype, const void* w, int w_dtype, int topk, int mode, const glmx_peer_out* peer,
                                   void* workspace, size_t workspace_bytes, void* stream);
GLMX_API int glmx_peer_reduce(const float* recv, const int* flags, int world, int rows_per_rank, int hidden, int seq,
                              void* out, int out_dtype, int* err, void* stream);
/* No counterpart (expert parallelism). The shard's picks of the gathered rows, one kernel: route int32 [rows][2 * topk] = global expert ids then the fp32
 * weights' bits; loc int32 / w fp32 [rows][topk + (shared ? 1 : 0)]: ids in [first, first + n) become 0 .. n - 1 with
 * their weight, others -1 with weight 0; with shared, a last column of local id n (weight 1) on rows
 * [own_begin, own_end) (the rank's own rows) and -1 elsewhere. */
GLMX_API int glmx_ep_split(const int* route, int rows, int topk, int first, int n, int shared, int own_begin, int own_end,
                           int* loc, float* w, void* stream);
/* No counterpart (expert parallelism). The all-to-all form of the dispatch and return (glmx.ep, exchange "a2a"): every
 * rank sends each token row only to the ranks that own at least one of its picks, and gets back only those rows' partial
 * results. glmx_ep_pack, on the token owner: sel int32 / w fp32 [B][topk] (global ids; rank d owns ids
 * [d * experts_per_rank, (d + 1) * experts_per_rank), others and negative ids are skipped) and x [B] rows of row_bytes
 * bytes -> counts int32 [world] (rows for each rank), *total (their sum), send_tok int32 [B * world] (each send row's
 * token), send_route int32 [B * world][2 * topk] (the row's picks in the destination's local ids, -1 with weight 0
 * elsewhere, then the weights' fp32 bits), pos int32 [world][B] (send row of (rank, token) or -1) and send_x
 * [B * world] rows (x gathered), all in (destination, token) order. glmx_ep_unpack_add, after the return: out fp32
 * [B][hidden] += the returned rows ret fp32 [*total][hidden] (in send order) of each token, added in rank order. */
GLMX_API int glmx_ep_pack(const int* sel, const float* w, int B, int topk, int experts_per_rank, int world, const void* x,
                          int row_bytes, int* counts, int* total, int* send_tok, int* send_route, int* pos, void* send_x,
                          void* stream);
GLMX_API int glmx_ep_unpack_add(const float* ret, const int* pos, int B, int world, int hidden, float* out, void* stream);
/* No counterpart (expert parallelism). CUDA IPC for those buffers: glmx_ipc_alloc makes a zeroed device allocation of its own (the mapping in another
 * process then starts at the buffer), glmx_ipc_handle its handle (GLMX_IPC_HANDLE_BYTES bytes), glmx_ipc_open maps a
 * peer's handle, glmx_ipc_close / glmx_ipc_free undo them. */
#define GLMX_IPC_HANDLE_BYTES 64
GLMX_API int glmx_ipc_alloc(size_t bytes, void** dev_ptr);
GLMX_API int glmx_ipc_free(void* dev_ptr);
GLMX_API int glmx_ipc_handle(const void* dev_ptr, void* handle);
GLMX_API int glmx_ipc_open(const void* handle, void** dev_ptr);
GLMX_API int glmx_ipc_close(void* dev_ptr);

/* Router of the MoE site, in front of the split: the GLM-4 MoE routing that exllamav3's router produces for the
 * reference's routing_fn hook (glm53/cpu_tier.py:305-335, sel [bsz, k] and w [bsz, k]). With gate_w (E x hidden,
 * row-major, dtype gate_dtype) the logits are computed first, logits[t][e] = sum_h z[t][h] * gate_w[e][h] with exact
 * products and fp32 sums (z: [ntok][hidden], dtype z_dtype; hidden a multiple of 32; both pointers 16-byte aligned),
 * and written to `logits`; with gate_w == NULL, `logits` (fp32 [ntok][n_experts]) is the input. Then per token:
 * s = sigmoid(logit), c = s + bias (bias fp32 [n_experts] or NULL); with n_group > 1 the topk_group groups of largest
 * (top-2 sum of c) stay and c is 0 elsewhere; picks = the topk largest c, in descending order, equal values by smaller
 * id; w = s[pick], if norm w / (sum of the picks' s + 1e-20), then * scale. sel: [ntok][topk] GLMX_I32 or GLMX_I64;
 * w: [ntok][topk] float dtype w_dtype. Limits: n_experts <= GLMX_ROUTER_MAX_EXPERTS, n_group <= 32 dividing n_experts,
 * topk <= 32. Two kernels on `stream`, nothing allocated. */
#define GLMX_ROUTER_MAX_EXPERTS 512
GLMX_API int glmx_router(const void* z, int z_dtype, int ntok, int hidden, const void* gate_w, int gate_dtype,
                         const float* bias, int n_experts, int n_group, int topk_group, int topk, int norm, float scale,
                         float* logits, void* sel, int sel_dtype, void* w, int w_dtype, void* stream);

/* Size of the scratch built into the library for glmx_moe_forward_noalloc: 48 MiB, which holds the workspace of up
 * to 8 tokens x top-8 (+ a shared expert) at H = 6144, I = 1536, in either mode, on a GPU of up to 148 SMs (B200; the
 * split-K partial sums of the workspace grow with the SM count, so a part with more SMs may take fewer tokens). */
#define GLMX_NOALLOC_SCRATCH_BYTES (48u << 20)

/* glmx_moe_forward without a workspace argument, for callers that cannot allocate device memory for one: a host in
 * another language with no device allocator of its own (cgo, JNI, N-API), or a serving loop whose HBM is already
 * held in full by its own allocator, where a cudaMalloc would fail and would also synchronise the device mid-step.
 * No counterpart in the reference (its CPU tier owns its buffers); same arguments, work and results as
 * glmx_moe_forward, minus the workspace.
 *   - Scratch is a fixed device array inside the library (GLMX_NOALLOC_SCRATCH_BYTES per device); nothing is
 *     allocated. A call whose workspace (glmx_workspace_bytes) would exceed it returns GLMX_E_WORKSPACE and runs
 *     nothing.
 *   - The first call on each device resolves that array's device address (one-time set-up per device, which may
 *     load the library's device code); make that first call before any stream capture.
 *   - All calls on one device share the one scratch: calls that overlap in time (different streams, or host threads
 *     whose work is in flight together) race and corrupt each other's results. Calls queued on one stream are safe.
 *   - Device-side error flags of these calls stay in the library's scratch: glmx_check_noalloc reads them. */
GLMX_API int glmx_moe_forward_noalloc(const glmx_layer* layer, const void* x, int x_dtype, int ntok, const void* sel,
                     int sel_dtype, const void* w, int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate,
                     void* stream);

/* glmx_check for glmx_moe_forward_noalloc: synchronises `stream` and reads the device error word of the built-in
 * scratch for a call of (ntok, topk) (the same word glmx_check reads in a caller's workspace). No counterpart in the
 * reference. The layer's device must be current. */
GLMX_API int glmx_check_noalloc(const glmx_layer* layer, int ntok, int topk, void* stream, int* flags);

#ifdef __cplusplus
}
#endif
#endif
