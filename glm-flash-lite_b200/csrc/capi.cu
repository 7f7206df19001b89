// extern "C" entry points of libglmx.so (declared in include/glmx.h).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "glmx_common.cuh"
#include "glmx_internal.h"

struct glmx_layer
{
    glmx::Layer L;
};

namespace glmx {

static thread_local std::string g_err;

void set_error(const std::string& msg) { g_err = msg; }

static int fail(int code, const std::string& msg)
{
    set_error(msg);
    return code;
}

static int cuda_fail(cudaError_t e, const char* what)
{
    return fail(GLMX_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace glmx

using namespace glmx;

extern "C" {

int glmx_version(void) { return GLMX_ABI_VERSION; }

const char* glmx_last_error(void) { return g_err.c_str(); }

int glmx_layer_create(const glmx_layer_desc* d, glmx_layer** out)
{
    if (!d || !out) return fail(GLMX_E_ARG, "glmx_layer_create: null argument");
    *out = nullptr;
    if (d->hidden <= 0 || d->intermediate <= 0 || d->hidden % 128 || d->intermediate % 128)
        return fail(GLMX_E_ARG, "glmx_layer_create: hidden and intermediate must be positive multiples of 128");
    if (d->n_experts < 1 || d->n_experts > 1024) return fail(GLMX_E_ARG, "glmx_layer_create: n_experts must be in [1, 1024]");
    for (int p = 0; p < 3; ++p)
    {
        if (d->bits[p] < 2 || d->bits[p] > 4) return fail(GLMX_E_ARG, "glmx_layer_create: bits must be 2, 3 or 4");
        if (!d->suh[p] || !d->svh[p]) return fail(GLMX_E_ARG, "glmx_layer_create: null suh/svh");
    }
    if (!d->trellis) return fail(GLMX_E_ARG, "glmx_layer_create: null trellis table");
    const int et = d->n_experts + (d->has_shared ? 1 : 0);
    for (int i = 0; i < et * 3; ++i)
    {
        if (!d->trellis[i]) return fail(GLMX_E_ARG, "glmx_layer_create: null trellis pointer at entry " + std::to_string(i));
        if (d->trellis[i] & 15u) return fail(GLMX_E_ARG, "glmx_layer_create: trellis pointer not 16-byte aligned at entry " + std::to_string(i));
    }
    glmx_layer* l = new glmx_layer();
    Layer& L = l->L;
    L.H = d->hidden; L.I = d->intermediate; L.E = d->n_experts; L.has_shared = d->has_shared ? 1 : 0; L.E_total = et;
    for (int p = 0; p < 3; ++p)
    {
        L.bits[p] = d->bits[p];
        L.suh[p] = static_cast<const uint16_t*>(d->suh[p]);
        L.svh[p] = static_cast<const uint16_t*>(d->svh[p]);
    }
    L.act_limit = d->act_limit;
    L.first = d->first_expert;
    cudaError_t e = cudaGetDevice(&L.device);
    if (e != cudaSuccess) { delete l; return cuda_fail(e, "glmx_layer_create: cudaGetDevice"); }
    if (L.device >= 64) { delete l; return fail(GLMX_E_ARG, "glmx_layer_create: device index >= 64"); }
    e = cudaMalloc(&L.d_trellis, sizeof(uint64_t) * et * 3);
    if (e != cudaSuccess) { delete l; return cuda_fail(e, "glmx_layer_create: cudaMalloc"); }
    e = cudaMemcpy(L.d_trellis, d->trellis, sizeof(uint64_t) * et * 3, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { cudaFree(L.d_trellis); delete l; return cuda_fail(e, "glmx_layer_create: cudaMemcpy"); }
    // the GEMV kernels' tensor maps, one per (expert, projection)
    {
        std::vector<CUtensorMap> maps((size_t) et * 3);
        for (int i = 0; i < et * 3 && e == cudaSuccess; ++i)
        {
            const int p = i % 3;
            e = trellis_map(&maps[i], reinterpret_cast<const void*>(d->trellis[i]), p < 2 ? L.H : L.I, p < 2 ? L.I : L.H, L.bits[p]);
        }
        if (e == cudaSuccess) e = cudaMalloc(&L.d_tmaps, sizeof(CUtensorMap) * maps.size());
        if (e == cudaSuccess) e = cudaMemcpy(L.d_tmaps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess)
        {
            if (L.d_tmaps) cudaFree(L.d_tmaps);
            cudaFree(L.d_trellis);
            delete l;
            return cuda_fail(e, "glmx_layer_create: trellis tensor maps");
        }
    }
    *out = l;
    return GLMX_OK;
}

int glmx_layer_destroy(glmx_layer* l)
{
    if (!l) return GLMX_OK;
    if (l->L.d_trellis) cudaFree(l->L.d_trellis);
    if (l->L.d_tmaps) cudaFree(l->L.d_tmaps);
    delete l;
    return GLMX_OK;
}

int glmx_layer_device(const glmx_layer* l) { return l ? l->L.device : GLMX_E_ARG; }

int glmx_layer_set_act_limit(glmx_layer* l, float limit)
{
    if (!l) return fail(GLMX_E_ARG, "glmx_layer_set_act_limit: null layer");
    l->L.act_limit = limit;
    return GLMX_OK;
}

size_t glmx_workspace_bytes(const glmx_layer* l, int ntok, int topk)
{
    if (!l || ntok < 0 || topk < 0) return 0;
    return ws_layout(l->L, ntok, topk, gemv_grid_ctas(l->L)).total;
}

int glmx_workspace_array(const glmx_layer* l, int ntok, int topk, int which, size_t* offset)
{
    if (!l || !offset || ntok < 0 || topk < 0) return fail(GLMX_E_ARG, "glmx_workspace_array: bad argument");
    const WsLayout w = ws_layout(l->L, ntok, topk, gemv_grid_ctas(l->L));
    switch (which)
    {
        case 0: *offset = w.offsets; break;
        case 1: *offset = w.row_token; break;
        case 2: *offset = w.row_weight; break;
        case 3: *offset = w.pick_row; break;
        case 4: *offset = w.jobs; break;
        case 5: *offset = w.plan; break;
        case 6: *offset = w.row_pick; break;
        default: return fail(GLMX_E_ARG, "glmx_workspace_array: unknown array");
    }
    return GLMX_OK;
}

static int check_common(const glmx_layer* l, int ntok, int topk, int sel_dtype, int w_dtype, void* ws, size_t ws_bytes,
                        WsLayout* lay, int* grid, const char* who)
{
    if (!l) return fail(GLMX_E_ARG, std::string(who) + ": null layer");
    if (ntok < 0 || topk < 0 || topk > 64) return fail(GLMX_E_ARG, std::string(who) + ": ntok >= 0 and 0 <= topk <= 64 required");
    if ((long long) ntok * topk > (1LL << 24)) return fail(GLMX_E_ARG, std::string(who) + ": too many picks");
    if (sel_dtype != GLMX_I32 && sel_dtype != GLMX_I64) return fail(GLMX_E_ARG, std::string(who) + ": sel dtype must be int32 or int64");
    if (w_dtype != GLMX_F32 && w_dtype != GLMX_F16 && w_dtype != GLMX_BF16)
        return fail(GLMX_E_ARG, std::string(who) + ": w dtype must be fp32, fp16 or bf16");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, who);
    if (dev != l->L.device) return fail(GLMX_E_ARG, std::string(who) + ": current device differs from the layer's device");
    *grid = gemv_grid_ctas(l->L);
    *lay = ws_layout(l->L, ntok, topk, *grid);
    if (!ws || ws_bytes < lay->total)
        return fail(GLMX_E_WORKSPACE, std::string(who) + ": workspace needs " + std::to_string(lay->total) + " bytes, got " + std::to_string(ws_bytes));
    if (!aligned16(ws)) return fail(GLMX_E_ARG, std::string(who) + ": workspace must be 16-byte aligned");
    return GLMX_OK;
}

int glmx_route(const glmx_layer* l, const void* sel, int sel_dtype, const void* w, int w_dtype, int ntok, int topk,
               void* ws, size_t ws_bytes, void* stream)
{
    WsLayout lay;
    int grid;
    int rc = check_common(l, ntok, topk, sel_dtype, w_dtype, ws, ws_bytes, &lay, &grid, "glmx_route");
    if (rc) return rc;
    if (ntok * topk > 0 && (!sel || !w)) return fail(GLMX_E_ARG, "glmx_route: null sel/w");
    cudaError_t e = launch_route(l->L, sel, sel_dtype == GLMX_I64, w, w_dtype, ntok, topk, MAXM, static_cast<uint8_t*>(ws), lay,
                                 grid, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "glmx_route: launch");
    return GLMX_OK;
}

int glmx_moe_forward(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype, const void* w,
                     int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate, void* ws, size_t ws_bytes,
                     void* stream)
{
    return glmx_moe_forward_timed(l, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, out, out_dtype, accumulate, ws,
                                  ws_bytes, stream, nullptr);
}

}  // extern "C"

// the forward of glmx_moe_forward_timed and glmx_moe_forward_hc (hc: hyper-connection epilogue instead of `out`)
static int forward_impl(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                        const void* w, int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate, void* ws,
                        size_t ws_bytes, void* stream, void* const* events, const HcOut* hc)
{
    WsLayout lay;
    int grid;
    int rc = check_common(l, ntok, topk, sel_dtype, w_dtype, ws, ws_bytes, &lay, &grid, "glmx_moe_forward");
    if (rc) return rc;
    const int base = mode & 0xff, path = mode & (GLMX_PATH_GEMV | GLMX_PATH_GEMM);
    if ((base != GLMX_MODE_EXACT && base != GLMX_MODE_I16) || (mode & ~(0xff | GLMX_PATH_GEMV | GLMX_PATH_GEMM)) ||
        path == (GLMX_PATH_GEMV | GLMX_PATH_GEMM))
        return fail(GLMX_E_ARG, "glmx_moe_forward: mode must be GLMX_MODE_EXACT (1) or GLMX_MODE_I16 (2), optionally with one "
                                "of GLMX_PATH_GEMV / GLMX_PATH_GEMM");
    if (base == GLMX_MODE_I16 && path == GLMX_PATH_GEMM)
        return fail(GLMX_E_ARG, "glmx_moe_forward: the tensor-core GEMM path is EXACT mode only");
    if (base == GLMX_MODE_I16 && lay.rows_max > I16_MAX_ROWS)
        return fail(GLMX_E_ARG, "glmx_moe_forward: I16 is the decode mode (at most " + std::to_string(I16_MAX_ROWS) +
                                " rows = picks + shared-expert rows per call); use GLMX_MODE_EXACT for larger batches");
    const bool gemm = base == GLMX_MODE_EXACT &&
                      (path == GLMX_PATH_GEMM || (path == 0 && lay.rows_max >= PF_AUTO_ROWS_PER_EXPERT * l->L.E_total));
    if (x_dtype != GLMX_F16 && x_dtype != GLMX_F32 && x_dtype != GLMX_BF16)
        return fail(GLMX_E_ARG, "glmx_moe_forward: x dtype must be fp16, fp32 or bf16");
    if (out_dtype != GLMX_F16 && out_dtype != GLMX_F32) return fail(GLMX_E_ARG, "glmx_moe_forward: out dtype must be fp16 or fp32");
    if (ntok > 0 && (!x || (!out && !hc))) return fail(GLMX_E_ARG, "glmx_moe_forward: null x/out");
    if (ntok * topk > 0 && (!sel || !w)) return fail(GLMX_E_ARG, "glmx_moe_forward: null sel/w");
    if (out && !aligned16(out)) return fail(GLMX_E_ARG, "glmx_moe_forward: out must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    cudaError_t e = cudaSuccess;
    if (events && events[0]) e = cudaEventRecord(static_cast<cudaEvent_t>(events[0]), st);
    const int maxm = base == GLMX_MODE_I16 ? I16_MAXM : gemm ? PF_MAXM : EXACT_MAXM;
    // the K-split plan is made for the grid of the GEMV that follows
    const int plan_grid = base == GLMX_MODE_I16 ? i16_grid_ctas(l->L) : grid;
    if (e == cudaSuccess) e = launch_route(l->L, sel, sel_dtype == GLMX_I64, w, w_dtype, ntok, topk, maxm, wsb, lay, plan_grid, st);
    if (e == cudaSuccess && events && events[1]) e = cudaEventRecord(static_cast<cudaEvent_t>(events[1]), st);
    if (e != cudaSuccess) return cuda_fail(e, "glmx_moe_forward: route launch");
    if (base == GLMX_MODE_I16)
        e = launch_i16_forward(l->L, x, x_dtype, ntok, topk, out, out_dtype, accumulate, wsb, lay, st, events, hc);
    else if (gemm)
        e = launch_prefill_forward(l->L, x, x_dtype, ntok, topk, out, out_dtype, accumulate, wsb, lay, st, events, hc);
    else
        e = launch_decode_forward(l->L, x, x_dtype, ntok, topk, base, out, out_dtype, accumulate, wsb, lay, grid, st, events, hc);
    // the next site's mix partials: fused into the EXACT GEMV path's combine, a pass over the updated stack otherwise
    if (e == cudaSuccess && hc && hc->fn && (base == GLMX_MODE_I16 || gemm))
        e = launch_hc_apply_partials(hc->x, nullptr, 0, nullptr, nullptr, hc->fn, hc->part, ntok, l->L.H, 0, st);
    if (e != cudaSuccess) return cuda_fail(e, "glmx_moe_forward: launch");
    return GLMX_OK;
}

extern "C" {

int glmx_moe_forward_timed(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                           const void* w, int w_dtype, int topk, int mode, void* out, int out_dtype, int accumulate, void* ws,
                           size_t ws_bytes, void* stream, void* const* events)
{
    return forward_impl(l, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, out, out_dtype, accumulate, ws, ws_bytes,
                        stream, events, nullptr);
}

int glmx_moe_forward_hc(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                        const void* w, int w_dtype, int topk, int mode, float* hc_x, const float* hc_post,
                        const float* hc_comb, int y_dtype, void* ws, size_t ws_bytes, void* stream)
{
    if (ntok > 0 && (!hc_x || !hc_post || !hc_comb)) return fail(GLMX_E_ARG, "glmx_moe_forward_hc: null stream stack / post / comb");
    if (y_dtype != GLMX_F16 && y_dtype != GLMX_F32) return fail(GLMX_E_ARG, "glmx_moe_forward_hc: y dtype must be fp16 or fp32");
    const HcOut hc{ hc_x, hc_post, hc_comb, y_dtype == GLMX_F16 ? 1 : 0 };
    return forward_impl(l, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, nullptr, GLMX_F32, 0, ws, ws_bytes, stream,
                        nullptr, &hc);
}

int glmx_moe_forward_hc_mix(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                            const void* w, int w_dtype, int topk, int mode, float* hc_x, const float* hc_post,
                            const float* hc_comb, int y_dtype, const uint16_t* fn, float* partials, void* ws, size_t ws_bytes,
                            void* stream)
{
    if (ntok > 0 && (!hc_x || !hc_post || !hc_comb || !fn || !partials))
        return fail(GLMX_E_ARG, "glmx_moe_forward_hc_mix: null stream stack / post / comb / fn / partials");
    if (y_dtype != GLMX_F16 && y_dtype != GLMX_F32) return fail(GLMX_E_ARG, "glmx_moe_forward_hc_mix: y dtype must be fp16 or fp32");
    if (!aligned16(hc_x) || !aligned16(fn)) return fail(GLMX_E_ARG, "glmx_moe_forward_hc_mix: x and fn must be 16-byte aligned");
    HcOut hc{ hc_x, hc_post, hc_comb, y_dtype == GLMX_F16 ? 1 : 0 };
    hc.fn = reinterpret_cast<const __half*>(fn);
    hc.part = partials;
    return forward_impl(l, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, nullptr, GLMX_F32, 0, ws, ws_bytes, stream,
                        nullptr, &hc);
}

int glmx_hc_apply_partials(float* x, const void* y, int y_dtype, const float* post, const float* comb, const uint16_t* fn,
                           float* partials, int R, int D, void* stream)
{
    if (R < 0 || D <= 0 || D % 128) return fail(GLMX_E_ARG, "glmx_hc_apply_partials: R >= 0 rows, D a multiple of 128");
    if (R == 0) return GLMX_OK;
    if (!x || !fn || !partials) return fail(GLMX_E_ARG, "glmx_hc_apply_partials: null x / fn / partials");
    if (y && (!post || !comb || (y_dtype != GLMX_F16 && y_dtype != GLMX_F32)))
        return fail(GLMX_E_ARG, "glmx_hc_apply_partials: y needs post, comb and an fp16 or fp32 dtype");
    if (!aligned16(x) || !aligned16(fn) || (y && !aligned16(y)))
        return fail(GLMX_E_ARG, "glmx_hc_apply_partials: x, y and fn must be 16-byte aligned");
    const cudaError_t e = launch_hc_apply_partials(x, y, y_dtype == GLMX_F16, post, comb, reinterpret_cast<const __half*>(fn),
                                                   partials, R, D, y ? 1 : 0, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GLMX_OK : cuda_fail(e, "glmx_hc_apply_partials: launch");
}

int glmx_hc_finalize_norm(const float* x, const float* partials, int R, int D, const float* base, const float* scale,
                          float* post, float* comb, const void* nw, int nw_dtype, uint16_t* out, float rms_eps, float hc_eps,
                          int iters, float n_eps, float cbias, float cscale, void* stream)
{
    if (R < 0 || D <= 0 || D % 512 || D > 16384)
        return fail(GLMX_E_ARG, "glmx_hc_finalize_norm: D a multiple of 512 up to 16384 (8 warps of partial chunks)");
    if (R == 0) return GLMX_OK;
    if (!x || !partials || !base || !scale || !post || !comb || !nw || !out)
        return fail(GLMX_E_ARG, "glmx_hc_finalize_norm: null argument");
    if (nw_dtype != GLMX_F16 && nw_dtype != GLMX_BF16) return fail(GLMX_E_ARG, "glmx_hc_finalize_norm: norm weight fp16 or bf16");
    if (iters < 1) return fail(GLMX_E_ARG, "glmx_hc_finalize_norm: iters >= 1");
    if (!aligned16(x) || !aligned16(out)) return fail(GLMX_E_ARG, "glmx_hc_finalize_norm: x and out must be 16-byte aligned");
    const cudaError_t e = launch_hc_finalize(x, partials, base, scale, post, comb, nw, nw_dtype == GLMX_BF16,
                                             reinterpret_cast<__half*>(out), R, D, rms_eps, hc_eps, iters, n_eps, cbias,
                                             cscale, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GLMX_OK : cuda_fail(e, "glmx_hc_finalize_norm: launch");
}

int glmx_moe_forward_peer(const glmx_layer* l, const void* x, int x_dtype, int ntok, const void* sel, int sel_dtype,
                          const void* w, int w_dtype, int topk, int mode, const glmx_peer_out* peer, void* ws, size_t ws_bytes,
                          void* stream)
{
    if (!peer || !peer->recv || !peer->flags || !peer->counter) return fail(GLMX_E_ARG, "glmx_moe_forward_peer: null peer table");
    if (peer->world < 1 || peer->world > 64 || peer->rank < 0 || peer->rank >= peer->world || peer->rows_per_rank <= 0 ||
        peer->seq <= 0 || (long long) peer->world * peer->rows_per_rank != ntok)
        return fail(GLMX_E_ARG, "glmx_moe_forward_peer: need 0 <= rank < world <= 64, seq > 0 and ntok = world * rows_per_rank > 0");
    HcOut hc{};
    hc.peer = PeerOut{ reinterpret_cast<float* const*>(peer->recv), peer->flags, peer->counter, peer->rank, peer->world,
                       peer->rows_per_rank, peer->seq };
    return forward_impl(l, x, x_dtype, ntok, sel, sel_dtype, w, w_dtype, topk, mode, nullptr, GLMX_F32, 0, ws, ws_bytes, stream,
                        nullptr, &hc);
}

int glmx_decode_tiles(const uint8_t* tiles, int bits, int ntiles, uint16_t* out, void* stream)
{
    if (bits < 2 || bits > 4) return fail(GLMX_E_ARG, "glmx_decode_tiles: bits must be 2, 3 or 4");
    if (ntiles < 0 || (ntiles > 0 && (!tiles || !out))) return fail(GLMX_E_ARG, "glmx_decode_tiles: bad arguments");
    cudaError_t e = launch_decode_tiles(tiles, bits, ntiles, out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "glmx_decode_tiles: launch");
    return GLMX_OK;
}

int glmx_check(const glmx_layer* l, int ntok, int topk, void* ws, void* stream, int* flags)
{
    if (!l || !ws) return fail(GLMX_E_ARG, "glmx_check: null argument");
    const WsLayout lay = ws_layout(l->L, ntok, topk, gemv_grid_ctas(l->L));
    int v = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&v, static_cast<uint8_t*>(ws) + lay.err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "glmx_check");
    if (flags) *flags = v;
    if (v) return fail(GLMX_E_DEVICE, "glmx_check: device error flags " + std::to_string(v));
    return GLMX_OK;
}

}  // extern "C"
