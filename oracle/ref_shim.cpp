// Test infrastructure only: a C-ABI shim over the reference's own CPU tier, kernels/cpu_avx2/ft_core.h of
// nkeilar/glm-flash-lite, compiled from the reference tree where it lies (include path given by the Makefile).
// It is used (a) to pin the restatement in ft_oracle.c against the real reference and to generate the golden
// fixtures under tests/golden/, and (b) as the timed CPU baseline of bench.py. Nothing here is product code.
#include "ft_core.h"

#include <sched.h>

namespace {
Pool g_pool;
bool g_pool_on = false;

// Builds the reference's route vector (ft_tier_ext.cpp:896-898 tier_forward: picks with sel < 0 skipped)
std::vector<std::vector<std::pair<int, float>>> make_route(const int32_t* sel, const float* w, int ntok, int topk, int E)
{
    std::vector<std::vector<std::pair<int, float>>> route(ntok);
    for (int t = 0; t < ntok; ++t)
        for (int k = 0; k < topk; ++k)
        {
            const int e = sel[t * topk + k];
            if (e >= 0 && e < E) route[t].push_back({ e, w[t * topk + k] });
        }
    return route;
}
}  // namespace

extern "C" {

int ftref_init()
{
    init_perm();
    init_tables();
    return 0;
}

void ftref_set_act_limit(float limit) { ACT_LIMIT = limit; }

// dense_weights (ft_core.h:1657-1672) of one native-layout K=3 tensor [k][n]
void ftref_dense(const uint8_t* tr, int k, int n, float* W)
{
    Mat m; m.tr = tr; m.suh = nullptr; m.svh = nullptr; m.k = k; m.n = n; m.swz = 0;
    std::vector<float> d = dense_weights(m);
    std::memcpy(W, d.data(), sizeof(float) * d.size());
}

// A Layer over caller-owned memory. tr/suh/svh: [E][3] pointers (gate, up, down).
void* ftref_layer_new(int H, int I, int E, const uint8_t* const* tr, const uint16_t* const* suh, const uint16_t* const* svh)
{
    Layer* L = new Layer();
    L->H = H; L->I = I; L->ex.resize(E);
    for (int e = 0; e < E; ++e)
    {
        L->ex[e].g = { tr[e * 3 + 0], suh[e * 3 + 0], svh[e * 3 + 0], H, I };
        L->ex[e].u = { tr[e * 3 + 1], suh[e * 3 + 1], svh[e * 3 + 1], H, I };
        L->ex[e].d = { tr[e * 3 + 2], suh[e * 3 + 2], svh[e * 3 + 2], I, H };
    }
    return L;
}

void ftref_layer_free(void* L) { delete static_cast<Layer*>(L); }

// Pool::start pins the calling thread to cpus[0]; the caller's affinity is restored afterwards
// (the same dance as ft_tier_ext.cpp:146-148).
int ftref_pool_start(int threads, const int* cpus, int ncpus)
{
    if (g_pool_on) return 1;
    std::vector<int> c(cpus, cpus + ncpus);
    cpu_set_t saved; sched_getaffinity(0, sizeof(saved), &saved);
    g_pool.start(threads, c);
    sched_setaffinity(0, sizeof(saved), &saved);
    g_pool_on = true;
    return 0;
}

void ftref_pool_stop()
{
    if (!g_pool_on) return;
    g_pool.stop();
    g_pool.th.clear();
    g_pool.quit = false;
    g_pool_on = false;
}

// moe_forward (ft_core.h:1338-1407); mode 0 AFFINE, 1 EXACT (mode 2 is invalid at H > 4096, see ft_core.h:1353)
int ftref_moe_forward(void* L, const float* x, int ntok, const int32_t* sel, const float* w, int topk, float* out, int mode)
{
    if (!g_pool_on) return -1;
    Layer* Lp = static_cast<Layer*>(L);
    auto route = make_route(sel, w, ntok, topk, int(Lp->ex.size()));
    moe_forward(g_pool, *Lp, x, ntok, route, out, mode);
    return 0;
}

// moe_forward_band (ft_core.h:1617-1651)
int ftref_moe_forward_band(void* L, const float* x, int ntok, const int32_t* sel, const float* w, int topk, float* out, int mode)
{
    if (!g_pool_on) return -1;
    Layer* Lp = static_cast<Layer*>(L);
    auto route = make_route(sel, w, ntok, topk, int(Lp->ex.size()));
    moe_forward_band(g_pool, *Lp, x, ntok, route, out, mode);
    return 0;
}

// ref_expert (ft_core.h:1684-1691): fp64-accumulated single-token expert on GPU-exact weights. Valid for I <= 2048.
void ftref_expert_fp64(void* L, int e, const float* x, float* y)
{
    Layer* Lp = static_cast<Layer*>(L);
    const Expert& E = Lp->ex[e];
    std::vector<float> W[3] = { dense_weights(E.g), dense_weights(E.u), dense_weights(E.d) };
    ref_expert(E, W, x, y);
}

}  // extern "C"
