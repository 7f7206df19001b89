/* Test infrastructure only: CPU restatement of the reference's routed-expert path (see ft_oracle.h).
 * Plain C11, scalar, single-threaded. Reference: nkeilar/glm-flash-lite kernels/cpu_avx2/ft_core.h. */
#include "ft_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ft_core.h:28-40 */
#define MUL1 0x83DCD12Du
static const float HAD = 0.088388347648f;

static int PERM[256];
static float CODEBOOK_EXACT[1021];   /* s -> fp16-rounded weight (as fp32) */
static float CODEBOOK_AFFINE[1021];  /* s -> unrounded fma(1024+s, KINV, KBIAS), exact in fp32 */
static uint16_t BYTESUM[65536];     /* st -> bytesum(st * MUL1), a cache of fto_bytesum */
static float KINV, KBIAS;
static int inited = 0;

uint16_t fto_f2h(float f) { _Float16 h = (_Float16) f; uint16_t b; memcpy(&b, &h, 2); return b; }
float fto_h2f(uint16_t b) { _Float16 h; memcpy(&h, &b, 2); return (float) h; }
static float r16(float f) { return fto_h2f(fto_f2h(f)); }

/* ft_core.h:48-61 init_perm */
void fto_init(void)
{
    if (inited) return;
    for (int t = 0; t < 32; ++t) {
        const int r0 = (t % 4) * 2, r1 = r0 + 1, r2 = r0 + 8, r3 = r0 + 9;
        const int c0 = t / 4, c1 = c0 + 8;
        const int rc[8] = { r0 * 16 + c0, r1 * 16 + c0, r2 * 16 + c0, r3 * 16 + c0,
                            r0 * 16 + c1, r1 * 16 + c1, r2 * 16 + c1, r3 * 16 + c1 };
        for (int j = 0; j < 8; ++j) PERM[t * 8 + j] = rc[j];
    }
    KINV = fto_h2f(0x1eee);
    KBIAS = fto_h2f(0xc931);
    for (int s = 0; s <= 1020; ++s) {
        CODEBOOK_AFFINE[s] = fmaf((float) (1024 + s), KINV, KBIAS);
        CODEBOOK_EXACT[s] = r16(CODEBOOK_AFFINE[s]);
    }
    for (int st = 0; st < 65536; ++st) BYTESUM[st] = (uint16_t) fto_bytesum((uint16_t) st);
    inited = 1;
}

int fto_perm(int i) { fto_init(); return PERM[i]; }

/* little-endian 32-bit word i of the tile (ft_core.h:63 ld32) */
static uint32_t ld32(const uint8_t* p, int i)
{
    return (uint32_t) p[4 * i] | ((uint32_t) p[4 * i + 1] << 8) | ((uint32_t) p[4 * i + 2] << 16) | ((uint32_t) p[4 * i + 3] << 24);
}

/* ft_core.h:65-73 state_scalar with BITS = K */
uint16_t fto_state(const uint8_t* tile, int K, int t)
{
    const int words32 = K * 256 / 32;
    const int b0 = t * K + K - 16 + 256 * K;
    const int b1 = b0 + 16;
    const int shift = ((b1 - 1) / 32 + 1) * 32 - b1;
    const uint64_t merged = ((uint64_t) ld32(tile, (b0 / 32) % words32) << 32) | ld32(tile, ((b1 - 1) / 32) % words32);
    return (uint16_t) (merged >> shift);
}

/* ft_core.h:75-79 */
int fto_bytesum(uint16_t st)
{
    const uint32_t x = (uint32_t) st * MUL1;
    return (int) ((x & 0xff) + ((x >> 8) & 0xff) + ((x >> 16) & 0xff) + (x >> 24));
}

/* ft_core.h:81-83 w_gpu_s */
uint16_t fto_codebook_h(int s) { fto_init(); return fto_f2h(CODEBOOK_EXACT[s]); }

void fto_decode_tile(const uint8_t* tile, int K, uint16_t* w16)
{
    fto_init();
    for (int i = 0; i < 256; ++i) w16[PERM[i]] = fto_f2h(CODEBOOK_EXACT[fto_bytesum(fto_state(tile, K, i))]);
}

/* ft_core.h:1657-1672 dense_weights (mode 1) and the unrounded codebook (mode 0) */
static void dense_mode(const uint8_t* tr, int K, int k, int n, int mode, float* W)
{
    fto_init();
    const float* cb = mode == 0 ? CODEBOOK_AFFINE : CODEBOOK_EXACT;
    const int tn = n / 16, tb = 32 * K;
    for (int tk = 0; tk < k / 16; ++tk)
        for (int t = 0; t < tn; ++t) {
            const uint8_t* tile = tr + ((size_t) tk * tn + t) * tb;
            for (int i = 0; i < 256; ++i) {
                const int rc = PERM[i];
                W[(size_t) (tk * 16 + rc / 16) * n + t * 16 + rc % 16] = cb[BYTESUM[fto_state(tile, K, i)]];
            }
        }
}

void fto_dense(const uint8_t* tr, int K, int k, int n, float* W) { dense_mode(tr, K, k, n, 1, W); }

/* ft_core.h:89-94 */
void fto_had128(float* v)
{
    for (int w = 1; w < 128; w *= 2)
        for (int b = 0; b < 128; b += 2 * w)
            for (int i = 0; i < w; ++i) { const float a = v[b + i], c = v[b + w + i]; v[b + i] = a + c; v[b + w + i] = a - c; }
}

/* ft_core.h:96-102 */
void fto_prep_block(const float* x, const uint16_t* suh, float* xt)
{
    for (int i = 0; i < 128; ++i) xt[i] = x[i] * fto_h2f(suh[i]);
    fto_had128(xt);
    for (int i = 0; i < 128; ++i) xt[i] = r16(xt[i] * HAD);
}

/* ft_core.h:104-110 */
void fto_out_block(float* y, const uint16_t* svh)
{
    for (int i = 0; i < 128; ++i) y[i] = r16(y[i]);
    fto_had128(y);
    for (int i = 0; i < 128; ++i) { const float t = y[i] * HAD; y[i] = r16(t * fto_h2f(svh[i])); }
}

/* ft_core.h:122-132 */
float fto_act_mul(float g, float u, float limit)
{
    float x = g / (1.0f + expf(-g));
    if (limit != 0.0f) { u = fminf(fmaxf(u, -limit), limit); x = fminf(x, limit); }
    return x * u;
}

/* ft_core.h:1674-1682 ref_linear, m tokens at once (fp64 accumulation) */
void fto_linear(const uint8_t* tr, int K, const uint16_t* suh, const uint16_t* svh, int k, int n,
                const float* W, int mode, const float* x, int m, float* y)
{
    float* Wl = NULL;
    if (!W) { Wl = (float*) malloc(sizeof(float) * (size_t) k * n); dense_mode(tr, K, k, n, mode, Wl); W = Wl; }
    float* xt = (float*) malloc(sizeof(float) * (size_t) k);
    double* acc = (double*) malloc(sizeof(double) * (size_t) n);
    for (int t = 0; t < m; ++t) {
        const float* xr = x + (size_t) t * k;
        float* yr = y + (size_t) t * n;
        for (int b = 0; b < k / 128; ++b) fto_prep_block(xr + b * 128, suh + b * 128, xt + b * 128);
        for (int j = 0; j < n; ++j) acc[j] = 0.0;
        for (int kk = 0; kk < k; ++kk) {
            const double xv = xt[kk];
            const float* wr = W + (size_t) kk * n;
            for (int j = 0; j < n; ++j) acc[j] += xv * wr[j];
        }
        for (int j = 0; j < n; ++j) yr[j] = (float) acc[j];
        for (int b = 0; b < n / 128; ++b) fto_out_block(yr + b * 128, svh + b * 128);
    }
    free(acc); free(xt); free(Wl);
}

/* ft_core.h:1684-1691 ref_expert (generic I; activation rounding point of ft_core.h:980) */
void fto_expert(const fto_expert_t* ex, int H, int I, int mode, float act_limit, const float* x, int m, float* y)
{
    float* g = (float*) malloc(sizeof(float) * (size_t) m * I);
    float* u = (float*) malloc(sizeof(float) * (size_t) m * I);
    fto_linear(ex->tr[0], ex->K[0], ex->suh[0], ex->svh[0], H, I, NULL, mode, x, m, g);
    fto_linear(ex->tr[1], ex->K[1], ex->suh[1], ex->svh[1], H, I, NULL, mode, x, m, u);
    for (size_t i = 0; i < (size_t) m * I; ++i) g[i] = r16(fto_act_mul(g[i], u[i], act_limit));
    fto_linear(ex->tr[2], ex->K[2], ex->suh[2], ex->svh[2], I, H, NULL, mode, g, m, y);
    free(g); free(u);
}

/* ---- I16 mode ---------------------------------------------------------------------------------------------- */

/* ft_core.h:583-598 quant_block_i16 (values only; the reference's duplicated/permuted register layout is not needed) */
static float quant_block_i16(const float* xt, int32_t* xi, float* sum)
{
    float amax = 0.0f;
    for (int r = 0; r < 128; ++r) { const float a = fabsf(xt[r]); amax = amax < a ? a : amax; }
    const float sc = amax > 0 ? amax / 16383.0f : 1.0f, rs = 1.0f / sc;
    long long si = 0;
    for (int r = 0; r < 128; ++r) { const float v = xt[r] * rs; xi[r] = (int32_t) nearbyintf(v); si += xi[r]; }
    const float add = (float) si * sc;
    *sum = *sum + add;
    return sc;
}

/* byte sums of a native-layout tensor [k][n] */
static void dense_bytesum(const uint8_t* tr, int K, int k, int n, uint16_t* S)
{
    fto_init();
    const int tn = n / 16, tb = 32 * K;
    for (int tk = 0; tk < k / 16; ++tk)
        for (int t = 0; t < tn; ++t) {
            const uint8_t* tile = tr + ((size_t) tk * tn + t) * tb;
            for (int i = 0; i < 256; ++i) {
                const int rc = PERM[i];
                S[(size_t) (tk * 16 + rc / 16) * n + t * 16 + rc % 16] = BYTESUM[fto_state(tile, K, i)];
            }
        }
}

/* ft_core.h:497-541 gemv_block_i16 for all output columns of one token: xi [k] int16 values, sc [k/128] */
static void gemv_i16(const uint16_t* S, int k, int n, const int32_t* xi, const float* sc, float sumx, float* y)
{
    static const int off[4] = { 0, 1, 8, 9 };
    float* acc = (float*) calloc((size_t) n * 4, sizeof(float));
    long long* blk = (long long*) malloc(sizeof(long long) * (size_t) n * 4);
    for (int b = 0; b < k / 128; ++b) {
        for (size_t i = 0; i < (size_t) n * 4; ++i) blk[i] = 0;
        for (int tk = b * 8; tk < b * 8 + 8; ++tk)
            for (int cl = 0; cl < 4; ++cl)
                for (int q = 0; q < 4; ++q) {
                    const int row = tk * 16 + 2 * q + off[cl];
                    const long long xv = xi[row];
                    const uint16_t* Sr = S + (size_t) row * n;
                    for (int c = 0; c < n; ++c) blk[(size_t) c * 4 + cl] += (long long) Sr[c] * xv;
                }
        for (int c = 0; c < n; ++c)
            for (int cl = 0; cl < 4; ++cl) {
                float* a = &acc[(size_t) c * 4 + cl];
                *a = fmaf((float) (int32_t) blk[(size_t) c * 4 + cl], sc[b], *a);
            }
    }
    const float kinv = KINV, caff = 1024.0f * KINV + KBIAS;
    for (int c = 0; c < n; ++c) {
        const float* a = &acc[(size_t) c * 4];
        const float lo = (a[0] + a[1]) + (a[2] + a[3]);
        const float t0 = kinv * lo, t1 = caff * sumx;
        y[c] = t0 + t1;
    }
    free(blk); free(acc);
}

void fto_expert_i16(const fto_expert_t* ex, int H, int I, float act_limit, const float* x, int m, float* y)
{
    fto_init();
    uint16_t* Sg = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) H * I);
    uint16_t* Su = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) H * I);
    uint16_t* Sd = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) I * H);
    dense_bytesum(ex->tr[0], ex->K[0], H, I, Sg);
    dense_bytesum(ex->tr[1], ex->K[1], H, I, Su);
    dense_bytesum(ex->tr[2], ex->K[2], I, H, Sd);
    const int BH = H / 128, BI = I / 128;
    int32_t* xg = (int32_t*) malloc(sizeof(int32_t) * (size_t) H);
    int32_t* xu = (int32_t*) malloc(sizeof(int32_t) * (size_t) H);
    int32_t* xd = (int32_t*) malloc(sizeof(int32_t) * (size_t) I);
    float* scg = (float*) malloc(sizeof(float) * (size_t) BH);
    float* scu = (float*) malloc(sizeof(float) * (size_t) BH);
    float* scd = (float*) malloc(sizeof(float) * (size_t) BI);
    float* sdb = (float*) malloc(sizeof(float) * (size_t) BI);
    float* g = (float*) malloc(sizeof(float) * (size_t) I);
    float* u = (float*) malloc(sizeof(float) * (size_t) I);
    float xt[128];
    for (int t = 0; t < m; ++t) {
        const float* xr = x + (size_t) t * H;
        float sg = 0.0f, su = 0.0f;                    /* ft_core.h:886-897 phase 0 */
        for (int b = 0; b < BH; ++b) {
            fto_prep_block(xr + b * 128, ex->suh[0] + b * 128, xt);
            scg[b] = quant_block_i16(xt, xg + b * 128, &sg);
            fto_prep_block(xr + b * 128, ex->suh[1] + b * 128, xt);
            scu[b] = quant_block_i16(xt, xu + b * 128, &su);
        }
        gemv_i16(Sg, H, I, xg, scg, sg, g);            /* phase 1 (ft_core.h:899-955) */
        gemv_i16(Su, H, I, xu, scu, su, u);
        for (int b = 0; b < BI; ++b) {
            fto_out_block(g + b * 128, ex->svh[0] + b * 128);
            fto_out_block(u + b * 128, ex->svh[1] + b * 128);
            float a[128];
            for (int r = 0; r < 128; ++r) a[r] = r16(fto_act_mul(g[b * 128 + r], u[b * 128 + r], act_limit));
            fto_prep_block(a, ex->suh[2] + b * 128, xt);
            float s = 0.0f;
            scd[b] = quant_block_i16(xt, xd + b * 128, &s);
            sdb[b] = s;
        }
        float sd = 0.0f;                                /* phase 2 (ft_core.h:997-1003): block sums in order */
        for (int b = 0; b < BI; ++b) sd = sd + sdb[b];
        float* yr = y + (size_t) t * H;
        gemv_i16(Sd, I, H, xd, scd, sd, yr);
        for (int b = 0; b < BH; ++b) fto_out_block(yr + b * 128, ex->svh[2] + b * 128);
    }
    free(u); free(g); free(sdb); free(scd); free(scu); free(scg); free(xd); free(xu); free(xg); free(Sd); free(Su); free(Sg);
}

/* Expert-major grouping: rows sorted by (expert asc, pick index asc). Within an expert the pick index order
 * is token order, which is the order ft_core.h:1344-1349 appends tokens to an expert's jobs. */
int fto_group(const int32_t* sel, const float* w, int ntok, int topk, int E,
              int32_t* offsets, int32_t* row_token, float* row_weight, int32_t* row_pick, int32_t* pick_row)
{
    const int n = ntok * topk;
    for (int e = 0; e <= E; ++e) offsets[e] = 0;
    for (int p = 0; p < n; ++p) if (sel[p] >= 0 && sel[p] < E) offsets[sel[p] + 1]++;
    for (int e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    int32_t* fill = (int32_t*) calloc((size_t) (E > 0 ? E : 0) + 1, sizeof(int32_t));
    for (int p = 0; p < n; ++p) {
        const int e = sel[p];
        if (e < 0 || e >= E) { pick_row[p] = -1; continue; }
        const int r = offsets[e] + fill[e]++;
        row_token[r] = p / topk; row_weight[r] = w[p]; row_pick[r] = p; pick_row[p] = r;
    }
    free(fill);
    return offsets[E];
}

/* ft_core.h:1344-1349 */
int fto_jobs_ref(const int32_t* sel, const float* w, int ntok, int topk, int E, int maxm,
                 int32_t* job_e, int32_t* job_m, int32_t* job_tok, float* job_w)
{
    int32_t* jid = (int32_t*) malloc(sizeof(int32_t) * ((size_t) (E > 0 ? E : 0) + 1));
    for (int e = 0; e < E; ++e) jid[e] = -1;
    int nj = 0;
    for (int t = 0; t < ntok; ++t)
        for (int kk = 0; kk < topk; ++kk) {
            const int e = sel[t * topk + kk];
            if (e < 0 || e >= E) continue;
            if (jid[e] < 0 || job_m[jid[e]] == maxm) { jid[e] = nj; job_e[nj] = e; job_m[nj] = 0; ++nj; }
            const int j = jid[e];
            job_tok[j * maxm + job_m[j]] = t; job_w[j * maxm + job_m[j]] = w[t * topk + kk]; job_m[j]++;
        }
    free(jid);
    return nj;
}

void fto_moe_forward(const fto_expert_t* experts, int E, const fto_expert_t* shared, int H, int I, int mode,
                     float act_limit, const float* x, int ntok, const int32_t* sel, const float* w, int topk, float* out)
{
    const int n = ntok * topk;
    int32_t* offsets = (int32_t*) malloc(sizeof(int32_t) * ((size_t) (E > 0 ? E : 0) + 1));
    int32_t* row_token = (int32_t*) malloc(sizeof(int32_t) * (size_t) (n > 0 ? n : 1));
    float* row_weight = (float*) malloc(sizeof(float) * (size_t) (n > 0 ? n : 1));
    int32_t* row_pick = (int32_t*) malloc(sizeof(int32_t) * (size_t) (n > 0 ? n : 1));
    int32_t* pick_row = (int32_t*) malloc(sizeof(int32_t) * (size_t) (n > 0 ? n : 1));
    const int P = fto_group(sel, w, ntok, topk, E, offsets, row_token, row_weight, row_pick, pick_row);
    float* yrow = (float*) malloc(sizeof(float) * (size_t) (P > 0 ? P : 1) * H);
    float* xs = (float*) malloc(sizeof(float) * (size_t) (P > 0 ? P : 1) * H);   /* one expert can take every pick */
    for (int e = 0; e < E; ++e) {
        const int r0 = offsets[e], m = offsets[e + 1] - r0;
        if (!m) continue;
        for (int i = 0; i < m; ++i) memcpy(xs + (size_t) i * H, x + (size_t) row_token[r0 + i] * H, sizeof(float) * H);
        if (mode == 2) fto_expert_i16(&experts[e], H, I, act_limit, xs, m, yrow + (size_t) r0 * H);
        else fto_expert(&experts[e], H, I, mode, act_limit, xs, m, yrow + (size_t) r0 * H);
    }
    float* ysh = NULL;
    if (shared && ntok) {
        ysh = (float*) malloc(sizeof(float) * (size_t) ntok * H);
        if (mode == 2) fto_expert_i16(shared, H, I, act_limit, x, ntok, ysh);
        else fto_expert(shared, H, I, mode, act_limit, x, ntok, ysh);
    }
    for (int t = 0; t < ntok; ++t) {
        float* o = out + (size_t) t * H;
        for (int c = 0; c < H; ++c) o[c] = 0.0f;
        for (int kk = 0; kk < topk; ++kk) {
            const int r = pick_row[t * topk + kk];
            if (r < 0) continue;
            const float wt = row_weight[r];
            const float* y = yrow + (size_t) r * H;
            for (int c = 0; c < H; ++c) o[c] += wt * y[c];
        }
        if (ysh) { const float* y = ysh + (size_t) t * H; for (int c = 0; c < H; ++c) o[c] += y[c]; }
    }
    free(ysh); free(xs); free(yrow); free(pick_row); free(row_pick); free(row_weight); free(row_token); free(offsets);
}

/* glm53/k_hcfuse.py:62-91 (k_apply_partials, APPLY leg): o = post_g * y, then o = fmaf(comb[h][g], x_h, o), h = 0..3 */
void fto_hc_apply(float* x, const float* y, int R, int D, const float* post, const float* comb)
{
    for (int r = 0; r < R; ++r)
        for (int c = 0; c < D; ++c)
        {
            float* xr = x + (size_t) r * 4 * D;
            float xv[4];
            for (int h = 0; h < 4; ++h) xv[h] = xr[(size_t) h * D + c];
            const float yv = y[(size_t) r * D + c];
            for (int g = 0; g < 4; ++g)
            {
                float o = post[r * 4 + g] * yv;
                for (int h = 0; h < 4; ++h) o = fmaf(comb[(r * 4 + h) * 4 + g], xv[h], o);
                xr[(size_t) g * D + c] = o;
            }
        }
}

/* ---- hc_mix_partials (glm53/k_hcfuse.py:92-126): per-lane terms, then the warp's shfl_down tree ---- */
void fto_hc_mix_partials(const float* x, const uint16_t* fn, int R, int D, float* part)
{
    const int nb = D / 128, nhalf = 4 * nb;
    for (int r = 0; r < R; ++r)
        for (int g = 0; g < 4; ++g)
            for (int jb = 0; jb < nb; ++jb)
            {
                float v[32][25];
                for (int l = 0; l < 32; ++l)
                {
                    const int q = jb * 32 + l;
                    const float* s = x + (size_t) r * 4 * D + (size_t) g * D + 4 * q;
                    float a = 0.0f;
                    for (int i = 0; i < 4; ++i) a = fmaf(s[i], s[i], a);
                    v[l][24] = a;
                    for (int j = 0; j < 24; ++j)
                    {
                        const uint16_t* w = fn + (size_t) j * 4 * D + (size_t) g * D + 4 * q;
                        const float d = fmaf(s[0], fto_h2f(w[0]), fmaf(s[1], fto_h2f(w[1]),
                                             fmaf(s[2], fto_h2f(w[2]), s[3] * fto_h2f(w[3]))));
                        v[l][j] = 0.0f + d;
                    }
                }
                for (int off = 16; off > 0; off >>= 1)
                    for (int l = 0; l < off; ++l)
                        for (int k = 0; k < 25; ++k) v[l][k] = v[l][k] + v[l + off][k];
                for (int k = 0; k < 25; ++k) part[((size_t) r * nhalf + (size_t) g * nb + jb) * 25 + k] = v[0][k];
            }
}

static float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

void fto_hc_finalize_norm(const float* x, const float* part, int R, int D, const float* base, const float* scale,
                          const float* nw, float rms_eps, float hc_eps, int iters, float n_eps, float cbias, float cscale,
                          float* post, float* comb, uint16_t* out)
{
    const int chunks = 4 * D / 256, per = chunks / 8;
    for (int r = 0; r < R; ++r)
    {
        const float* p = part + (size_t) r * 2 * chunks * 25;
        float mix[25];
        for (int k = 0; k < 25; ++k)
        {
            float tot = 0.0f;
            for (int w = 0; w < 8; ++w)
            {
                float v = 0.0f;
                for (int i = 0; i < per; ++i)
                {
                    const int c = w + 8 * i;
                    v += (0.0f + p[(size_t) 2 * c * 25 + k]) + p[(size_t) (2 * c + 1) * 25 + k];
                }
                tot += v;
            }
            mix[k] = tot;
        }
        const float rmr = 1.0f / sqrtf(mix[24] / (float) (4 * D) + rms_eps);
        for (int g = 0; g < 4; ++g) post[r * 4 + g] = 2.0f * sigmoid_f(fmaf(mix[4 + g] * rmr, scale[1], base[4 + g]));
        float v[16];
        for (int t = 0; t < 16; ++t) v[t] = fmaf(mix[8 + t] * rmr, scale[2], base[8 + t]);
        for (int h = 0; h < 4; ++h)
        {
            float m = v[h * 4];
            for (int g = 1; g < 4; ++g) m = fmaxf(m, v[h * 4 + g]);
            float s = 0.0f;
            for (int g = 0; g < 4; ++g) { v[h * 4 + g] = expf(v[h * 4 + g] - m); s += v[h * 4 + g]; }
            for (int g = 0; g < 4; ++g) v[h * 4 + g] = v[h * 4 + g] / s + hc_eps;
        }
        for (int it = 0; it < iters; ++it)
        {
            if (it > 0)
                for (int h = 0; h < 4; ++h)
                {
                    float rs = 0.0f;
                    for (int g = 0; g < 4; ++g) rs += v[h * 4 + g];
                    for (int g = 0; g < 4; ++g) v[h * 4 + g] /= rs + hc_eps;
                }
            for (int g = 0; g < 4; ++g)
            {
                float cs = 0.0f;
                for (int h = 0; h < 4; ++h) cs += v[h * 4 + g];
                for (int h = 0; h < 4; ++h) v[h * 4 + g] /= cs + hc_eps;
            }
        }
        memcpy(comb + (size_t) r * 16, v, sizeof v);
        float pre[4];
        for (int h = 0; h < 4; ++h) pre[h] = sigmoid_f(fmaf(mix[h] * rmr, scale[0], base[h])) + hc_eps;
        float* col = malloc(sizeof(float) * (size_t) D);
        double ss = 0.0;
        for (int c = 0; c < D; ++c)
        {
            float o = 0.0f;
            for (int h = 0; h < 4; ++h) o = fmaf(pre[h], x[(size_t) r * 4 * D + (size_t) h * D + c], o);
            o = r16(o);
            o = fmaxf(-65504.0f, fminf(o, 65504.0f));
            col[c] = o;
            ss += (double) o * o;
        }
        const float rmf = 1.0f / sqrtf((float) ss / (float) D + n_eps) * cscale;
        for (int c = 0; c < D; ++c) out[(size_t) r * D + c] = fto_f2h(col[c] * (nw[c] + cbias) * rmf);
        free(col);
    }
}

/* ---- router in front of the split (the GLM-4 MoE routing of exllamav3's router, as transformers states it in
 * models/glm4_moe/modeling_glm4_moe.py:302-305 (gate) and 389-412 (route_tokens_to_experts)) ---- */

/* 2^k as an fp32 (k in [-149, 127]; below that 0) */
static float pow2i_f(int k)
{
    uint32_t b;
    float f;
    if (k >= -126) b = (uint32_t) (k + 127) << 23;
    else if (k >= -149) b = 1u << (k + 149);
    else return 0.0f;
    memcpy(&f, &b, sizeof f);
    return f;
}

/* e^y in fp32: Cody and Waite's argument reduction (y = n ln2 + r, ln2 split into a 16-bit head and a tail) and the
 * degree-8 Taylor polynomial of e^r in Horner form with fused multiply-adds, 2^n applied in two halves. The same fp32
 * operation sequence as the GPU router's, so both give the same bits. */
static float exp_cw(float y)
{
    if (y != y) return y;
    y = fminf(fmaxf(y, -175.0f), 175.0f);
    const float n = rintf(y * 1.44269502162933349609375f);
    float r = fmaf(n, -0.693145751953125f, y);
    r = fmaf(n, -1.428606765330187045037746429443359375e-06f, r);
    float p = 2.4801587301587302e-05f;
    p = fmaf(p, r, 1.9841269841269841e-04f);
    p = fmaf(p, r, 1.3888888888888889e-03f);
    p = fmaf(p, r, 8.3333333333333332e-03f);
    p = fmaf(p, r, 4.1666666666666664e-02f);
    p = fmaf(p, r, 1.6666666666666666e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int) n, n1 = ni / 2, n2 = ni - n1;
    return (p * pow2i_f(n1)) * pow2i_f(n2);
}

static float router_sigmoid(float x) { return 1.0f / (1.0f + exp_cw(-x)); }

void fto_router_sigmoid(const float* x, int n, float* out)
{
    for (int i = 0; i < n; ++i) out[i] = router_sigmoid(x[i]);
}

/* (v, i) before (u, j): larger value first, equal values by smaller index */
static int router_better(float v, int i, float u, int j) { return v > u || (v == u && i < j); }

void fto_router_gate(const float* z, int ntok, int H, const float* W, int E, float* logits)
{
    for (int t = 0; t < ntok; ++t)
        for (int e = 0; e < E; ++e)
        {
            double s = 0.0;
            for (int h = 0; h < H; ++h) s += (double) z[(size_t) t * H + h] * (double) W[(size_t) e * H + h];
            logits[(size_t) t * E + e] = (float) s;
        }
}

void fto_router_select(const float* logits, int ntok, int E, const float* bias, int n_group, int topk_group, int topk,
                       int norm, float scale, int32_t* sel, float* w)
{
    float* s = (float*) malloc(sizeof(float) * (size_t) E);
    float* c = (float*) malloc(sizeof(float) * (size_t) E);
    unsigned char* taken = (unsigned char*) malloc((size_t) E);
    const int G = E / n_group;
    for (int t = 0; t < ntok; ++t)
    {
        for (int e = 0; e < E; ++e)
        {
            s[e] = router_sigmoid(logits[(size_t) t * E + e]);
            c[e] = bias ? s[e] + bias[e] : s[e];
            taken[e] = 0;
        }
        if (n_group > 1)
        {
            float gs[64];
            for (int g = 0; g < n_group; ++g)
            {
                float m1 = -INFINITY, m2 = -INFINITY;
                for (int e = g * G; e < (g + 1) * G; ++e)
                {
                    if (c[e] > m1) { m2 = m1; m1 = c[e]; }
                    else if (c[e] > m2) m2 = c[e];
                }
                gs[g] = m1 + m2;
            }
            for (int g = 0; g < n_group; ++g)
            {
                int rank = 0;
                for (int h = 0; h < n_group; ++h) rank += router_better(gs[h], h, gs[g], g);
                if (rank >= topk_group)
                    for (int e = g * G; e < (g + 1) * G; ++e) c[e] = 0.0f;
            }
        }
        float wsum = 0.0f;
        for (int r = 0; r < topk; ++r)
        {
            int bi = -1;
            for (int e = 0; e < E; ++e)
                if (!taken[e] && (bi < 0 || router_better(c[e], e, c[bi], bi))) bi = e;
            taken[bi] = 1;
            sel[(size_t) t * topk + r] = bi;
            w[(size_t) t * topk + r] = s[bi];
            wsum += s[bi];
        }
        for (int r = 0; r < topk; ++r)
        {
            float v = w[(size_t) t * topk + r];
            if (norm) v = v / (wsum + 1e-20f);
            w[(size_t) t * topk + r] = v * scale;
        }
    }
    free(s);
    free(c);
    free(taken);
}
