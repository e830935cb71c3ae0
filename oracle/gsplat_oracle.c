/*
 * gsplat_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, fp32 restatement of the reference renderer of bigwolfeman/gaussian-2d-splat-encoder, used
 * as the parity checker for the CUDA path (tests/, __graft_entry__.smoke(), bench.py's CPU baseline).
 * The product never links, loads or calls this file.
 *
 * What it restates (paths inside the reference project):
 *   activate_scale                       gaussian_splat_encoder/params.py:18-28
 *   _build_tiles (tile CSR)              gaussian_splat_encoder/render_triton.py:351-409
 *   _render_fwd_cull_kernel              gaussian_splat_encoder/render_triton.py:423-517
 *   _render_bwd_cull_kernel              gaussian_splat_encoder/render_triton.py:602-720
 *   _backward_cull / _backward_cull_fields (per-pair -> per-splat sum)  render_triton.py:723-810
 *   _upsample_field (bilinear, align_corners=False) and its adjoint     render_triton.py:864-876
 *   render_alpha_multires                render_triton.py:879-922
 *   _octave_of / render_alpha_octave     render_triton.py:925-980
 *   _render_fwd_kernel / _render_bwd_kernel (exact path)                render_triton.py:58-303
 *   the composite and its autograd backward (torch ops in the wrappers) render_triton.py:918-921,976-979
 *
 * Build with -ffp-contract=off: the tile-rectangle arithmetic must round like the reference's separate
 * fp32 torch ops for the binning to be bit-exact.  Within a tile the reference sorts with an unstable
 * argsort; this oracle emits ascending splat id (a stable counting sort), which is the canonical order
 * the parity tests compare against.
 *
 * Multi-threaded with OpenMP over tiles (forward) and over tiles with per-thread gradient buffers
 * (backward), so it doubles as the timed CPU baseline.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ALPHA_MAX (1.0f - 1e-4f)

/* ------------------------------------------------------------------ splat views */
typedef struct {
    int n, C;
    const float *muy, *mux, *sy, *sx, *th, *op, *col; /* col: [n][C]; th may be NULL */
} splats_t;

typedef struct {
    float *muy, *mux, *sy, *sx, *th, *op, *col; /* per-splat grads (local index), th may be NULL */
} sgrads_t;

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* params.py:28 -- softplus(x) (torch: threshold 20, beta 1) + SCALE_EPS */
static inline float softplus_eps(float x) { return (x > 20.0f ? x : log1pf(expf(x))) + 1e-4f; }
static inline float softplus_grad(float x) {
    if (x > 20.0f) return 1.0f;
    float z = expf(x);
    return z / (z + 1.0f);
}

void orc_activate_scale(const float *ls, float *sc, long n) {
    for (long i = 0; i < n; i++) sc[i] = softplus_eps(ls[i]);
}

/* render_triton.py:925-932 + 950-952 */
int orc_octave_of(float sy, float sx, float rep, float base_texels, int max_octaves) {
    float sp = fmaxf(sy, sx) * rep;
    float q = sp / base_texels;
    if (!(q >= 1e-6f)) q = 1e-6f;
    float o = ceilf(log2f(q));
    if (o < 0.0f) o = 0.0f;
    if (o > (float)max_octaves) o = (float)max_octaves;
    return (int)o;
}

/* render_triton.py:362-377: the clamped tile rectangle of one splat */
static inline void tile_rect(float muy, float mux, float sy, float sx, int H, int W, int TILE, float cutoff,
                             int *tx0, int *tx1, int *ty0, int *ty1) {
    int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE;
    float cx = mux * (float)W;
    float cy = muy * (float)H;
    float r = cutoff * fmaxf(sy, sx);
    float rx = r * (float)W;
    float ry = r * (float)H;
    float a = floorf((cx - rx) / (float)TILE), b = floorf((cx + rx) / (float)TILE);
    float c = floorf((cy - ry) / (float)TILE), d = floorf((cy + ry) / (float)TILE);
    a = fminf(fmaxf(a, 0.0f), (float)(ntx - 1));
    b = fminf(fmaxf(b, 0.0f), (float)(ntx - 1));
    c = fminf(fmaxf(c, 0.0f), (float)(nty - 1));
    d = fminf(fmaxf(d, 0.0f), (float)(nty - 1));
    *tx0 = (int)a; *tx1 = (int)b; *ty0 = (int)c; *ty1 = (int)d;
}

/* Count the (tile, splat) pairs of a splat group at (H,W). */
long orc_count_pairs(const splats_t *s, int H, int W, int TILE, float cutoff) {
    long tot = 0;
    for (int i = 0; i < s->n; i++) {
        int x0, x1, y0, y1;
        tile_rect(s->muy[i], s->mux[i], s->sy[i], s->sx[i], H, W, TILE, cutoff, &x0, &x1, &y0, &y1);
        tot += (long)(x1 - x0 + 1) * (long)(y1 - y0 + 1);
    }
    return tot;
}

/* _build_tiles: CSR sorted by tile, ascending local splat id inside a tile.  starts has nt+1 entries,
 * gid has room for the pair count (orc_count_pairs). */
void orc_build_tiles(const splats_t *s, int H, int W, int TILE, float cutoff, int *starts, int *gid) {
    int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE, nt = ntx * nty;
    int *cnt = (int *)calloc((size_t)nt + 1, sizeof(int));
    for (int i = 0; i < s->n; i++) {
        int x0, x1, y0, y1;
        tile_rect(s->muy[i], s->mux[i], s->sy[i], s->sx[i], H, W, TILE, cutoff, &x0, &x1, &y0, &y1);
        for (int ty = y0; ty <= y1; ty++)
            for (int tx = x0; tx <= x1; tx++) cnt[ty * ntx + tx]++;
    }
    starts[0] = 0;
    for (int t = 0; t < nt; t++) starts[t + 1] = starts[t] + cnt[t];
    for (int t = 0; t < nt; t++) cnt[t] = starts[t];
    for (int i = 0; i < s->n; i++) {
        int x0, x1, y0, y1;
        tile_rect(s->muy[i], s->mux[i], s->sy[i], s->sx[i], H, W, TILE, cutoff, &x0, &x1, &y0, &y1);
        for (int ty = y0; ty <= y1; ty++)
            for (int tx = x0; tx <= x1; tx++) gid[cnt[ty * ntx + tx]++] = i;
    }
    free(cnt);
}

/* per-pair geometry shared by forward and backward (render_triton.py:468-492) */
typedef struct {
    float ry, rx, inv_sy, inv_sx, f, fo, a, cth, sth;
} geom_t;

static inline void pair_geom(const splats_t *s, int g, float py, float px, geom_t *o) {
    float dy = py - s->muy[g], dx = px - s->mux[g];
    if (s->th) {
        o->cth = cosf(s->th[g]);
        o->sth = sinf(s->th[g]);
        o->ry = o->cth * dy + o->sth * dx;
        o->rx = -o->sth * dy + o->cth * dx;
    } else {
        o->cth = 1.0f; o->sth = 0.0f;
        o->ry = dy; o->rx = dx;
    }
    o->inv_sy = 1.0f / s->sy[g];
    o->inv_sx = 1.0f / s->sx[g];
    float maha = (o->ry * o->ry) * (o->inv_sy * o->inv_sy) + (o->rx * o->rx) * (o->inv_sx * o->inv_sx);
    o->f = expf(-0.5f * maha);
    o->fo = o->f * s->op[g];
    o->a = fminf(o->fo, ALPHA_MAX);
}

/* _render_fwd_cull_kernel (FIELDS=True): raw sums per pixel.  slog/sa: [H*W]; sac: [H*W][C]. */
void orc_fields_fwd(const splats_t *s, int H, int W, int TILE, const int *starts, const int *gid, int odds,
                    float *slog, float *sa, float *sac) {
    int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE, nt = ntx * nty, C = s->C;
    memset(slog, 0, sizeof(float) * (size_t)H * W);
    memset(sa, 0, sizeof(float) * (size_t)H * W);
    memset(sac, 0, sizeof(float) * (size_t)H * W * C);
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < nt; t++) {
        int tx = t % ntx, ty = t / ntx;
        for (int ly = 0; ly < TILE; ly++) {
            int yp = ty * TILE + ly;
            if (yp >= H) continue;
            float py = ((float)yp + 0.5f) / (float)H;
            for (int lx = 0; lx < TILE; lx++) {
                int xp = tx * TILE + lx;
                if (xp >= W) continue;
                float px = ((float)xp + 0.5f) / (float)W;
                float Sl = 0.0f, Sa = 0.0f, Sc[8] = {0};
                for (int k = starts[t]; k < starts[t + 1]; k++) {
                    int g = gid[k];
                    geom_t q;
                    pair_geom(s, g, py, px, &q);
                    Sl += logf(1.0f - q.a);
                    float w = odds ? q.a / (1.0f - q.a) : q.a;
                    Sa += w;
                    for (int c = 0; c < C; c++) Sc[c] += w * s->col[(size_t)g * C + c];
                }
                size_t p = (size_t)yp * W + xp;
                slog[p] = Sl;
                sa[p] = Sa;
                for (int c = 0; c < C; c++) sac[p * C + c] = Sc[c];
            }
        }
    }
}

/* one pixel-pair of _render_bwd_cull_kernel (render_triton.py:661-720), accumulated into grads */
static inline void pair_bwd(const splats_t *s, int g, float py, float px, float dSl, float dSa, const float *dSc,
                            int odds, sgrads_t *gr) {
    int C = s->C;
    geom_t q;
    pair_geom(s, g, py, px, &q);
    float inv1ma = 1.0f / (1.0f - q.a);
    float col_term = 0.0f;
    for (int c = 0; c < C; c++) col_term += dSc[c] * s->col[(size_t)g * C + c];
    float da, cw;
    if (odds) {
        da = dSl * (-inv1ma) + (dSa + col_term) * (inv1ma * inv1ma);
        cw = q.a * inv1ma;
    } else {
        da = dSl * (-inv1ma) + dSa + col_term;
        cw = q.a;
    }
    for (int c = 0; c < C; c++) gr->col[(size_t)g * C + c] += cw * dSc[c];
    float da_fo = (q.fo < ALPHA_MAX) ? da : 0.0f;
    gr->op[g] += da_fo * q.f;
    float gm = (da_fo * s->op[g]) * (-0.5f * q.f);
    gr->sy[g] += gm * (-2.0f * q.ry * q.ry) * (q.inv_sy * q.inv_sy * q.inv_sy);
    gr->sx[g] += gm * (-2.0f * q.rx * q.rx) * (q.inv_sx * q.inv_sx * q.inv_sx);
    float gry = gm * (2.0f * q.ry) * (q.inv_sy * q.inv_sy);
    float grx = gm * (2.0f * q.rx) * (q.inv_sx * q.inv_sx);
    if (s->th) {
        gr->th[g] += gry * q.rx - grx * q.ry;
        gr->muy[g] += -(gry * q.cth - grx * q.sth);
        gr->mux[g] += -(gry * q.sth + grx * q.cth);
    } else {
        gr->muy[g] += -gry;
        gr->mux[g] += -grx;
    }
}

static void grads_alloc(sgrads_t *g, int n, int C, int has_th) {
    g->muy = (float *)calloc((size_t)n, sizeof(float));
    g->mux = (float *)calloc((size_t)n, sizeof(float));
    g->sy = (float *)calloc((size_t)n, sizeof(float));
    g->sx = (float *)calloc((size_t)n, sizeof(float));
    g->op = (float *)calloc((size_t)n, sizeof(float));
    g->th = has_th ? (float *)calloc((size_t)n, sizeof(float)) : NULL;
    g->col = (float *)calloc((size_t)n * C, sizeof(float));
}

static void grads_free(sgrads_t *g) {
    free(g->muy); free(g->mux); free(g->sy); free(g->sx); free(g->op); free(g->th); free(g->col);
}

static void grads_add(sgrads_t *dst, const sgrads_t *src, int n, int C) {
    for (int i = 0; i < n; i++) {
        dst->muy[i] += src->muy[i]; dst->mux[i] += src->mux[i];
        dst->sy[i] += src->sy[i]; dst->sx[i] += src->sx[i];
        dst->op[i] += src->op[i];
        if (dst->th) dst->th[i] += src->th[i];
    }
    for (long i = 0; i < (long)n * C; i++) dst->col[i] += src->col[i];
}

/* _render_bwd_cull_kernel with FIELDS=True: dS fields in, per-splat grads accumulated (the per-pair
 * values summed per splat, which is what the reference's index_add_ does). */
void orc_fields_bwd(const splats_t *s, int H, int W, int TILE, const int *starts, const int *gid, int odds,
                    const float *dslog, const float *dsa, const float *dsac, sgrads_t *out) {
    int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE, nt = ntx * nty, C = s->C;
    int nth = orc_num_threads();
    sgrads_t *part = (sgrads_t *)calloc((size_t)nth, sizeof(sgrads_t));
    for (int i = 0; i < nth; i++) grads_alloc(&part[i], s->n, C, s->th != NULL);
#pragma omp parallel
    {
        int tid = 0;
#ifdef _OPENMP
        tid = omp_get_thread_num();
#endif
        sgrads_t *gr = &part[tid];
#pragma omp for schedule(dynamic, 4)
        for (int t = 0; t < nt; t++) {
            int tx = t % ntx, ty = t / ntx;
            for (int ly = 0; ly < TILE; ly++) {
                int yp = ty * TILE + ly;
                if (yp >= H) continue;
                float py = ((float)yp + 0.5f) / (float)H;
                for (int lx = 0; lx < TILE; lx++) {
                    int xp = tx * TILE + lx;
                    if (xp >= W) continue;
                    float px = ((float)xp + 0.5f) / (float)W;
                    size_t p = (size_t)yp * W + xp;
                    for (int k = starts[t]; k < starts[t + 1]; k++)
                        pair_bwd(s, gid[k], py, px, dslog[p], dsa[p], dsac + p * C, odds, gr);
                }
            }
        }
    }
    for (int i = 0; i < nth; i++) {
        grads_add(out, &part[i], s->n, C);
        grads_free(&part[i]);
    }
    free(part);
}

/* ------------------------------------------------------------------ bilinear (torch semantics) */
static inline void lin_index(int d, int in_size, int out_size, int *i0, int *i1, float *l0, float *l1) {
    float scale = (float)in_size / (float)out_size;
    float src = scale * ((float)d + 0.5f) - 0.5f;
    if (src < 0.0f) src = 0.0f;
    int i = (int)src;
    if (i > in_size - 1) i = in_size - 1;
    int ip = (i < in_size - 1) ? 1 : 0;
    float lam = src - (float)i;
    lam = fminf(fmaxf(lam, 0.0f), 1.0f);
    *i0 = i; *i1 = i + ip; *l1 = lam; *l0 = 1.0f - lam;
}

/* out[Ho*Wo][C] += bilinear(in[Hi*Wi][C]) */
void orc_upsample_add(const float *in, int Hi, int Wi, int C, float *out, int Ho, int Wo) {
#pragma omp parallel for
    for (int y = 0; y < Ho; y++) {
        int y0, y1; float h0, h1;
        lin_index(y, Hi, Ho, &y0, &y1, &h0, &h1);
        for (int x = 0; x < Wo; x++) {
            int x0, x1; float w0, w1;
            lin_index(x, Wi, Wo, &x0, &x1, &w0, &w1);
            for (int c = 0; c < C; c++) {
                float v = h0 * (w0 * in[((size_t)y0 * Wi + x0) * C + c] + w1 * in[((size_t)y0 * Wi + x1) * C + c]) +
                          h1 * (w0 * in[((size_t)y1 * Wi + x0) * C + c] + w1 * in[((size_t)y1 * Wi + x1) * C + c]);
                out[((size_t)y * Wo + x) * C + c] += v;
            }
        }
    }
}

/* gin[Hi*Wi][C] += adjoint of the bilinear upsample applied to gout[Ho*Wo][C] */
void orc_upsample_adjoint_add(const float *gout, int Ho, int Wo, int C, float *gin, int Hi, int Wi) {
    for (int y = 0; y < Ho; y++) {
        int y0, y1; float h0, h1;
        lin_index(y, Hi, Ho, &y0, &y1, &h0, &h1);
        for (int x = 0; x < Wo; x++) {
            int x0, x1; float w0, w1;
            lin_index(x, Wi, Wo, &x0, &x1, &w0, &w1);
            for (int c = 0; c < C; c++) {
                float g = gout[((size_t)y * Wo + x) * C + c];
                gin[((size_t)y0 * Wi + x0) * C + c] += h0 * w0 * g;
                gin[((size_t)y0 * Wi + x1) * C + c] += h0 * w1 * g;
                gin[((size_t)y1 * Wi + x0) * C + c] += h1 * w0 * g;
                gin[((size_t)y1 * Wi + x1) * C + c] += h1 * w1 * g;
            }
        }
    }
}

/* ------------------------------------------------------------------ composite (torch autograd) */
/* img[C][P] (one image, planar) from summed fields; render_triton.py:976-979 */
static void composite_fwd(int P, int C, const float *slog, const float *sa, const float *sac, const float *bg,
                          float *img) {
    for (int p = 0; p < P; p++) {
        float asum = fmaxf(sa[p], 1e-8f);
        float T = expf(slog[p]);
        for (int c = 0; c < C; c++) {
            float fg = sac[(size_t)p * C + c] / asum;
            img[(size_t)c * P + p] = (1.0f - T) * fg + T * bg[c];
        }
    }
}

/* autograd of the composite: g[C][P] -> dslog, dsa, dsac; gbg += sum_p g*T.  clamp_min passes the
 * gradient where sa >= 1e-8 (torch's clamp_min backward). */
static void composite_bwd(int P, int C, const float *slog, const float *sa, const float *sac, const float *bg,
                          const float *g, float *dslog, float *dsa, float *dsac, float *gbg, int clamp_mask) {
    for (int c = 0; c < C; c++) {
        double acc = 0.0;
        for (int p = 0; p < P; p++) acc += (double)g[(size_t)c * P + p] * (double)expf(slog[p]);
        gbg[c] += (float)acc;
    }
    for (int p = 0; p < P; p++) {
        float asum = fmaxf(sa[p], 1e-8f);
        float T = expf(slog[p]);
        float dT = 0.0f, dasum = 0.0f;
        for (int c = 0; c < C; c++) {
            float gc = g[(size_t)c * P + p];
            float fg = sac[(size_t)p * C + c] / asum;
            dT += gc * (bg[c] - fg);
            float dfg = gc * (1.0f - T);
            dsac[(size_t)p * C + c] = dfg / asum;
            dasum += dfg * fg;
        }
        dslog[p] = dT * T;
        float d = -dasum / asum;
        dsa[p] = (clamp_mask && !(sa[p] >= 1e-8f)) ? 0.0f : d;
    }
}

/* ------------------------------------------------------------------ group render helpers */
typedef struct {
    int H, W, n;
    int *starts, *gid;
    float *slog, *sa, *sac;
} group_t;

static int group_bin(group_t *G, const splats_t *s, int H, int W, int TILE, float cutoff, long max_pairs) {
    int ntx = (W + TILE - 1) / TILE, nty = (H + TILE - 1) / TILE, nt = ntx * nty;
    long tot = orc_count_pairs(s, H, W, TILE, cutoff);
    if (max_pairs >= 0 && tot > max_pairs) return 1;
    G->H = H; G->W = W; G->n = s->n;
    G->starts = (int *)malloc(sizeof(int) * ((size_t)nt + 1));
    G->gid = (int *)malloc(sizeof(int) * (size_t)(tot > 0 ? tot : 1));
    orc_build_tiles(s, H, W, TILE, cutoff, G->starts, G->gid);
    G->slog = (float *)malloc(sizeof(float) * (size_t)H * W);
    G->sa = (float *)malloc(sizeof(float) * (size_t)H * W);
    G->sac = (float *)malloc(sizeof(float) * (size_t)H * W * s->C);
    return 0;
}

static void group_free(group_t *G) {
    free(G->starts); free(G->gid); free(G->slog); free(G->sa); free(G->sac);
    memset(G, 0, sizeof(*G));
}

/* gather a subset (idx) of image b's splats into contiguous per-component arrays */
typedef struct {
    splats_t s;
    float *buf;
} subset_t;

static void subset_make(subset_t *S, int C, int has_th, const float *mu, const float *sc, const float *col,
                        const float *op, const float *th, const int *idx, int n) {
    S->buf = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * (7 + C));
    float *b = S->buf;
    float *muy = b, *mux = b + n, *sy = b + 2 * n, *sx = b + 3 * n, *opp = b + 4 * n, *thh = b + 5 * n,
          *cc = b + 7 * n;
    for (int k = 0; k < n; k++) {
        int i = idx ? idx[k] : k;
        muy[k] = mu[2 * i]; mux[k] = mu[2 * i + 1];
        sy[k] = sc[2 * i]; sx[k] = sc[2 * i + 1];
        opp[k] = op[i];
        thh[k] = has_th ? th[i] : 0.0f;
        for (int c = 0; c < C; c++) cc[(size_t)k * C + c] = col[(size_t)i * C + c];
    }
    S->s.n = n; S->s.C = C;
    S->s.muy = muy; S->s.mux = mux; S->s.sy = sy; S->s.sx = sx; S->s.op = opp;
    S->s.th = has_th ? thh : NULL;
    S->s.col = cc;
}

/* scatter subset grads back to the image's per-splat grads (scale grads chained through softplus) */
static void subset_scatter(const sgrads_t *g, const int *idx, int n, int C, const float *ls, float *gmu, float *gls,
                           float *gcol, float *gop, float *gth) {
    for (int k = 0; k < n; k++) {
        int i = idx ? idx[k] : k;
        gmu[2 * i] += g->muy[k];
        gmu[2 * i + 1] += g->mux[k];
        gls[2 * i] += g->sy[k] * softplus_grad(ls[2 * i]);
        gls[2 * i + 1] += g->sx[k] * softplus_grad(ls[2 * i + 1]);
        gop[i] += g->op[k];
        if (gth && g->th) gth[i] += g->th[k];
        for (int c = 0; c < C; c++) gcol[(size_t)i * C + c] += g->col[(size_t)k * C + c];
    }
}

/* ------------------------------------------------------------------ public entry points
 * Layouts follow the reference API: mu [B][N][2] (y,x); log_scale [B][N][2]; color [B][N][C];
 * opacity [B][N]; bg [B][C]; theta [B][N] or NULL; out/gC [B][C][H][W].  Grad outputs (NULL gC ->
 * forward only) are overwritten.  Return 0, or 1 when a (image, group) pair count exceeds max_pairs
 * (PairBudgetExceeded; max_pairs < 0 disables the check). */

/* render_alpha_octave (render_triton.py:935-980); with groups = octaves.  mode 0 = octave routing;
 * mode 1 = multires split (render_triton.py:879-922, n_coarse / coarse_factor). */
static int render_groups(int mode, int B, int N, int C, const float *mu, const float *ls, const float *col,
                         const float *op, const float *bg, const float *th, int H, int W, float cutoff, int TILE,
                         float base_texels, int max_octaves, int n_coarse, int coarse_factor, long max_pairs,
                         int odds, float *out, const float *gC, float *gmu, float *gls, float *gcol, float *gop,
                         float *gbg, float *gth, const float *l2_target, float l2_scale, float *l2_grad,
                         double *l2_loss) {
    int P = H * W, has_th = th != NULL;
    if (l2_target) gC = l2_grad;
    float *sc = (float *)malloc(sizeof(float) * (size_t)B * N * 2);
    orc_activate_scale(ls, sc, (long)B * N * 2);
    if (gC) {
        memset(gmu, 0, sizeof(float) * (size_t)B * N * 2);
        memset(gls, 0, sizeof(float) * (size_t)B * N * 2);
        memset(gcol, 0, sizeof(float) * (size_t)B * N * C);
        memset(gop, 0, sizeof(float) * (size_t)B * N);
        memset(gbg, 0, sizeof(float) * (size_t)B * C);
        if (gth) memset(gth, 0, sizeof(float) * (size_t)B * N);
    }
    int status = 0;
    int *idx = (int *)malloc(sizeof(int) * (size_t)(N > 0 ? N : 1));
    float *slog = (float *)malloc(sizeof(float) * (size_t)P);
    float *sa = (float *)malloc(sizeof(float) * (size_t)P);
    float *sac = (float *)malloc(sizeof(float) * (size_t)P * C);
    for (int b = 0; b < B && !status; b++) {
        const float *mub = mu + (size_t)b * N * 2, *scb = sc + (size_t)b * N * 2, *lsb = ls + (size_t)b * N * 2;
        const float *colb = col + (size_t)b * N * C, *opb = op + (size_t)b * N, *thb = has_th ? th + (size_t)b * N : NULL;
        memset(slog, 0, sizeof(float) * P);
        memset(sa, 0, sizeof(float) * P);
        memset(sac, 0, sizeof(float) * (size_t)P * C);
        int ngroups;
        int *gof = (int *)malloc(sizeof(int) * (size_t)(N > 0 ? N : 1));
        if (mode == 0) {
            float rep = (float)(H < W ? H : W);
            for (int i = 0; i < N; i++) gof[i] = orc_octave_of(scb[2 * i], scb[2 * i + 1], rep, base_texels, max_octaves);
            ngroups = max_octaves + 1;
        } else {
            for (int i = 0; i < N; i++) gof[i] = (n_coarse > 0 && n_coarse < N && i < n_coarse) ? 0 : 1;
            ngroups = 2;
        }
        group_t *G = (group_t *)calloc((size_t)ngroups, sizeof(group_t));
        subset_t *S = (subset_t *)calloc((size_t)ngroups, sizeof(subset_t));
        int **gidx = (int **)calloc((size_t)ngroups, sizeof(int *));
        int *gn = (int *)calloc((size_t)ngroups, sizeof(int));
        for (int o = 0; o < ngroups && !status; o++) {
            int n = 0;
            for (int i = 0; i < N; i++)
                if (gof[i] == o) idx[n++] = i;
            gn[o] = n;
            if (n == 0) continue;
            int Ho, Wo;
            if (mode == 0) {
                Ho = (H >> o) > 8 ? (H >> o) : 8;
                Wo = (W >> o) > 8 ? (W >> o) : 8;
            } else if (o == 0) {
                int m = (H < W ? H : W) / 8;
                int cf = coarse_factor < (m > 1 ? m : 1) ? coarse_factor : (m > 1 ? m : 1);
                Ho = H / cf > 1 ? H / cf : 1;
                Wo = W / cf > 1 ? W / cf : 1;
            } else {
                Ho = H; Wo = W;
            }
            gidx[o] = (int *)malloc(sizeof(int) * (size_t)n);
            memcpy(gidx[o], idx, sizeof(int) * (size_t)n);
            subset_make(&S[o], C, has_th, mub, scb, colb, opb, thb, gidx[o], n);
            if (group_bin(&G[o], &S[o].s, Ho, Wo, TILE, cutoff, max_pairs)) { status = 1; break; }
            orc_fields_fwd(&S[o].s, Ho, Wo, TILE, G[o].starts, G[o].gid, odds, G[o].slog, G[o].sa, G[o].sac);
            if (Ho == H && Wo == W) {
                for (int p = 0; p < P; p++) { slog[p] += G[o].slog[p]; sa[p] += G[o].sa[p]; }
                for (long p = 0; p < (long)P * C; p++) sac[p] += G[o].sac[p];
            } else {
                orc_upsample_add(G[o].slog, Ho, Wo, 1, slog, H, W);
                orc_upsample_add(G[o].sa, Ho, Wo, 1, sa, H, W);
                orc_upsample_add(G[o].sac, Ho, Wo, C, sac, H, W);
            }
        }
        if (!status) {
            composite_fwd(P, C, slog, sa, sac, bg + (size_t)b * C, out + (size_t)b * C * P);
            if (l2_target) { /* the fitting loss l2_scale * sum (out - target)^2 and its gradient */
                const float *ob = out + (size_t)b * C * P, *tb = l2_target + (size_t)b * C * P;
                float *gb = l2_grad + (size_t)b * C * P;
                double acc = 0.0;
                for (long i = 0; i < (long)C * P; i++) {
                    float d = ob[i] - tb[i];
                    gb[i] = 2.0f * l2_scale * d;
                    acc += (double)d * d;
                }
                *l2_loss += (double)l2_scale * acc;
            }
            if (gC) {
                float *dslog = (float *)malloc(sizeof(float) * P), *dsa = (float *)malloc(sizeof(float) * P);
                float *dsac = (float *)malloc(sizeof(float) * (size_t)P * C);
                composite_bwd(P, C, slog, sa, sac, bg + (size_t)b * C, gC + (size_t)b * C * P, dslog, dsa, dsac,
                              gbg + (size_t)b * C, 1);
                for (int o = 0; o < ngroups; o++) {
                    if (gn[o] == 0) continue;
                    int Ho = G[o].H, Wo = G[o].W;
                    float *gl = dslog, *ga = dsa, *gc = dsac;
                    if (!(Ho == H && Wo == W)) {
                        gl = (float *)calloc((size_t)Ho * Wo, sizeof(float));
                        ga = (float *)calloc((size_t)Ho * Wo, sizeof(float));
                        gc = (float *)calloc((size_t)Ho * Wo * C, sizeof(float));
                        orc_upsample_adjoint_add(dslog, H, W, 1, gl, Ho, Wo);
                        orc_upsample_adjoint_add(dsa, H, W, 1, ga, Ho, Wo);
                        orc_upsample_adjoint_add(dsac, H, W, C, gc, Ho, Wo);
                    }
                    sgrads_t g;
                    grads_alloc(&g, gn[o], C, has_th);
                    orc_fields_bwd(&S[o].s, Ho, Wo, TILE, G[o].starts, G[o].gid, odds, gl, ga, gc, &g);
                    subset_scatter(&g, gidx[o], gn[o], C, lsb, gmu + (size_t)b * N * 2, gls + (size_t)b * N * 2,
                                   gcol + (size_t)b * N * C, gop + (size_t)b * N, gth ? gth + (size_t)b * N : NULL);
                    grads_free(&g);
                    if (gl != dslog) { free(gl); free(ga); free(gc); }
                }
                free(dslog); free(dsa); free(dsac);
            }
        }
        for (int o = 0; o < ngroups; o++) {
            if (gidx[o]) { free(gidx[o]); free(S[o].buf); }
            if (G[o].starts) group_free(&G[o]);
        }
        free(G); free(S); free(gidx); free(gn); free(gof);
    }
    free(idx); free(slog); free(sa); free(sac); free(sc);
    return status;
}

int orc_render_octave(int B, int N, int C, const float *mu, const float *ls, const float *col, const float *op,
                      const float *bg, const float *th, int H, int W, float cutoff, int TILE, float base_texels,
                      int max_octaves, long max_pairs, int odds, float *out, const float *gC, float *gmu, float *gls,
                      float *gcol, float *gop, float *gbg, float *gth) {
    return render_groups(0, B, N, C, mu, ls, col, op, bg, th, H, W, cutoff, TILE, base_texels, max_octaves, 0, 0,
                         max_pairs, odds, out, gC, gmu, gls, gcol, gop, gbg, gth, NULL, 0.0f, NULL, NULL);
}

/* One fitting step's render: forward, loss = scale * sum (out - target)^2 (scale = 1/out.numel() is
 * mse_loss), its gradient into gC_out, and the backward of that gradient -- the forward runs once, as
 * in the reference's autograd (render_triton.py:935-980 forward, its Function's backward). */
int orc_render_octave_l2(int B, int N, int C, const float *mu, const float *ls, const float *col, const float *op,
                         const float *bg, const float *th, int H, int W, float cutoff, int TILE, float base_texels,
                         int max_octaves, long max_pairs, int odds, const float *target, float scale, float *out,
                         float *gC_out, double *loss, float *gmu, float *gls, float *gcol, float *gop, float *gbg,
                         float *gth) {
    *loss = 0.0;
    return render_groups(0, B, N, C, mu, ls, col, op, bg, th, H, W, cutoff, TILE, base_texels, max_octaves, 0, 0,
                         max_pairs, odds, out, NULL, gmu, gls, gcol, gop, gbg, gth, target, scale, gC_out, loss);
}

int orc_render_multires(int B, int N, int C, const float *mu, const float *ls, const float *col, const float *op,
                        const float *bg, const float *th, int H, int W, int n_coarse, int coarse_factor, float cutoff,
                        int TILE, long max_pairs, int odds, float *out, const float *gC, float *gmu, float *gls,
                        float *gcol, float *gop, float *gbg, float *gth) {
    return render_groups(1, B, N, C, mu, ls, col, op, bg, th, H, W, cutoff, TILE, 0.0f, 0, n_coarse, coarse_factor,
                         max_pairs, odds, out, gC, gmu, gls, gcol, gop, gbg, gth, NULL, 0.0f, NULL, NULL);
}

/* render_alpha_full_triton(cull=True): one group at (H,W), composite inside the kernel; the backward
 * derives dS from (T, asum, fg) WITHOUT the clamp_min mask (render_triton.py:644-654). */
int orc_render_cull(int B, int N, int C, const float *mu, const float *ls, const float *col, const float *op,
                    const float *bg, const float *th, int H, int W, int TILE, float cutoff, int odds, float *out,
                    const float *gC, float *gmu, float *gls, float *gcol, float *gop, float *gbg, float *gth) {
    int P = H * W, has_th = th != NULL;
    float *sc = (float *)malloc(sizeof(float) * (size_t)B * N * 2);
    orc_activate_scale(ls, sc, (long)B * N * 2);
    if (gC) {
        memset(gmu, 0, sizeof(float) * (size_t)B * N * 2); memset(gls, 0, sizeof(float) * (size_t)B * N * 2);
        memset(gcol, 0, sizeof(float) * (size_t)B * N * C); memset(gop, 0, sizeof(float) * (size_t)B * N);
        memset(gbg, 0, sizeof(float) * (size_t)B * C);
        if (gth) memset(gth, 0, sizeof(float) * (size_t)B * N);
    }
    for (int b = 0; b < B; b++) {
        subset_t S;
        subset_make(&S, C, has_th, mu + (size_t)b * N * 2, sc + (size_t)b * N * 2, col + (size_t)b * N * C,
                    op + (size_t)b * N, has_th ? th + (size_t)b * N : NULL, NULL, N);
        group_t G;
        group_bin(&G, &S.s, H, W, TILE, cutoff, -1);
        orc_fields_fwd(&S.s, H, W, TILE, G.starts, G.gid, odds, G.slog, G.sa, G.sac);
        composite_fwd(P, C, G.slog, G.sa, G.sac, bg + (size_t)b * C, out + (size_t)b * C * P);
        if (gC) {
            float *dslog = (float *)malloc(sizeof(float) * P), *dsa = (float *)malloc(sizeof(float) * P);
            float *dsac = (float *)malloc(sizeof(float) * (size_t)P * C);
            composite_bwd(P, C, G.slog, G.sa, G.sac, bg + (size_t)b * C, gC + (size_t)b * C * P, dslog, dsa, dsac,
                          gbg + (size_t)b * C, 0);
            sgrads_t g;
            grads_alloc(&g, N, C, has_th);
            orc_fields_bwd(&S.s, H, W, TILE, G.starts, G.gid, odds, dslog, dsa, dsac, &g);
            subset_scatter(&g, NULL, N, C, ls + (size_t)b * N * 2, gmu + (size_t)b * N * 2, gls + (size_t)b * N * 2,
                           gcol + (size_t)b * N * C, gop + (size_t)b * N, gth ? gth + (size_t)b * N : NULL);
            grads_free(&g);
            free(dslog); free(dsa); free(dsac);
        }
        group_free(&G);
        free(S.buf);
    }
    free(sc);
    return 0;
}

/* torch.linspace(0.5/n, 1-0.5/n, n) in fp32 (render.py:61-65) */
static void pixel_centers(int n, float *v) {
    float start = (float)(0.5 / n), end = (float)(1.0 - 0.5 / n);
    if (n == 1) { v[0] = start; return; }
    float step = (end - start) / (float)(n - 1);
    int half = n / 2;
    for (int i = 0; i < n; i++) v[i] = i < half ? start + step * (float)i : end - step * (float)(n - 1 - i);
}

/* render_alpha_full_triton(cull=False): every pixel x every splat, alpha mode (render_triton.py:58-303) */
int orc_render_exact(int B, int N, int C, const float *mu, const float *ls, const float *col, const float *op,
                     const float *bg, const float *th, int H, int W, float *out, const float *gC, float *gmu,
                     float *gls, float *gcol, float *gop, float *gbg, float *gth) {
    int P = H * W, has_th = th != NULL;
    float *sc = (float *)malloc(sizeof(float) * (size_t)B * N * 2);
    orc_activate_scale(ls, sc, (long)B * N * 2);
    float *pyv = (float *)malloc(sizeof(float) * H), *pxv = (float *)malloc(sizeof(float) * W);
    pixel_centers(H, pyv);
    pixel_centers(W, pxv);
    if (gC) {
        memset(gmu, 0, sizeof(float) * (size_t)B * N * 2); memset(gls, 0, sizeof(float) * (size_t)B * N * 2);
        memset(gcol, 0, sizeof(float) * (size_t)B * N * C); memset(gop, 0, sizeof(float) * (size_t)B * N);
        memset(gbg, 0, sizeof(float) * (size_t)B * C);
        if (gth) memset(gth, 0, sizeof(float) * (size_t)B * N);
    }
    float *slog = (float *)malloc(sizeof(float) * P), *sa = (float *)malloc(sizeof(float) * P);
    float *sac = (float *)malloc(sizeof(float) * (size_t)P * C);
    for (int b = 0; b < B; b++) {
        subset_t S;
        subset_make(&S, C, has_th, mu + (size_t)b * N * 2, sc + (size_t)b * N * 2, col + (size_t)b * N * C,
                    op + (size_t)b * N, has_th ? th + (size_t)b * N : NULL, NULL, N);
#pragma omp parallel for
        for (int p = 0; p < P; p++) {
            float py = pyv[p / W], px = pxv[p % W];
            float Sl = 0.0f, Sa = 0.0f, Sc[8] = {0};
            for (int g = 0; g < N; g++) {
                geom_t q;
                pair_geom(&S.s, g, py, px, &q);
                Sl += logf(1.0f - q.a);
                Sa += q.a;
                for (int c = 0; c < C; c++) Sc[c] += q.a * S.s.col[(size_t)g * C + c];
            }
            slog[p] = Sl; sa[p] = Sa;
            for (int c = 0; c < C; c++) sac[(size_t)p * C + c] = Sc[c];
        }
        composite_fwd(P, C, slog, sa, sac, bg + (size_t)b * C, out + (size_t)b * C * P);
        if (gC) {
            float *dslog = (float *)malloc(sizeof(float) * P), *dsa = (float *)malloc(sizeof(float) * P);
            float *dsac = (float *)malloc(sizeof(float) * (size_t)P * C);
            composite_bwd(P, C, slog, sa, sac, bg + (size_t)b * C, gC + (size_t)b * C * P, dslog, dsa, dsac,
                          gbg + (size_t)b * C, 0);
            int nth = orc_num_threads();
            sgrads_t *part = (sgrads_t *)calloc((size_t)nth, sizeof(sgrads_t));
            for (int i = 0; i < nth; i++) grads_alloc(&part[i], N, C, has_th);
#pragma omp parallel
            {
                int tid = 0;
#ifdef _OPENMP
                tid = omp_get_thread_num();
#endif
#pragma omp for
                for (int p = 0; p < P; p++)
                    for (int g = 0; g < N; g++)
                        pair_bwd(&S.s, g, pyv[p / W], pxv[p % W], dslog[p], dsa[p], dsac + (size_t)p * C, 0,
                                 &part[tid]);
            }
            sgrads_t g;
            grads_alloc(&g, N, C, has_th);
            for (int i = 0; i < nth; i++) { grads_add(&g, &part[i], N, C); grads_free(&part[i]); }
            free(part);
            subset_scatter(&g, NULL, N, C, ls + (size_t)b * N * 2, gmu + (size_t)b * N * 2, gls + (size_t)b * N * 2,
                           gcol + (size_t)b * N * C, gop + (size_t)b * N, gth ? gth + (size_t)b * N : NULL);
            grads_free(&g);
            free(dslog); free(dsa); free(dsac);
        }
        free(S.buf);
    }
    free(slog); free(sa); free(sac); free(sc); free(pyv); free(pxv);
    return 0;
}

/* Binning of one image for the octave path, for bit-exact comparison with the CUDA binning:
 * oct[N] receives each splat's octave; for each octave o the CSR (local-to-octave starts over that
 * octave's tiles, ids are GLOBAL splat ids, ascending within a tile) is written at
 * starts + soff[o] / gid + goff[o], where soff/goff are filled by this call (soff has max_octaves+2
 * entries, goff likewise).  Call first with gid == NULL to get the sizes. */
long orc_bin_octave(int N, const float *mu, const float *sc, int H, int W, float cutoff, int TILE, float base_texels,
                    int max_octaves, int *oct, long *soff, long *goff, int *starts, int *gid) {
    float rep = (float)(H < W ? H : W);
    for (int i = 0; i < N; i++) oct[i] = orc_octave_of(sc[2 * i], sc[2 * i + 1], rep, base_texels, max_octaves);
    int *idx = (int *)malloc(sizeof(int) * (size_t)(N > 0 ? N : 1));
    long so = 0, go = 0;
    for (int o = 0; o <= max_octaves; o++) {
        int Ho = (H >> o) > 8 ? (H >> o) : 8, Wo = (W >> o) > 8 ? (W >> o) : 8;
        int ntx = (Wo + TILE - 1) / TILE, nty = (Ho + TILE - 1) / TILE, nt = ntx * nty;
        int n = 0;
        for (int i = 0; i < N; i++)
            if (oct[i] == o) idx[n++] = i;
        soff[o] = so; goff[o] = go;
        subset_t S;
        subset_make(&S, 1, 0, mu, sc, sc, sc, NULL, idx, n);
        long tot = orc_count_pairs(&S.s, Ho, Wo, TILE, cutoff);
        if (gid) {
            orc_build_tiles(&S.s, Ho, Wo, TILE, cutoff, starts + so, gid + go);
            for (long k = 0; k < tot; k++) gid[go + k] = idx[gid[go + k]];
        }
        free(S.buf);
        so += nt + 1;
        go += tot;
    }
    soff[max_octaves + 1] = so;
    goff[max_octaves + 1] = go;
    free(idx);
    return go;
}
