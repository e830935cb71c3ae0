// Shared device helpers for the gsplat_b200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define GS_MAX_GROUPS 8

// Hardware approximations (PTX ex2.approx / rcp.approx; rel. error ~2^-22).
__device__ __forceinline__ float gs_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gs_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte vector reduction into global memory (sm_90+): one L2 atomic op for four floats.
__device__ __forceinline__ void gs_red_add_v4(float *addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// softplus(x) + SCALE_EPS with torch's threshold 20 (params.py:28; torch F.softplus defaults).
__device__ __forceinline__ float gs_softplus_eps(float x) { return (x > 20.0f ? x : log1pf(expf(x))) + 1e-4f; }
__device__ __forceinline__ float gs_softplus_grad(float x) {
    if (x > 20.0f) return 1.0f;
    float z = expf(x);
    return z / (z + 1.0f);
}

// Geometry of one render group (an octave, the coarse/fine multires group, or the single
// resolution of the cull/exact paths).
struct GroupGeom {
    int H, W;      // group resolution
    int ntx, nty;  // tiles
    int tile_off;  // first tile of this group inside an image's tile range
    int fld_off;   // first float of this group's 5 planar fields inside an image's field block
    int ty_lo, ty_hi;  // tile rows this call needs (the native row band's bilinear footprint)
    float up_sy, up_sx;  // bilinear source-index scales group/native, (float)Hg / (float)H as torch computes
    int adj_off;         // first texel of this group in the adjoint launch (coarse groups only), -1 if none
    int prior_grp;       // group of a prior render whose fields this group reuses, -1 if none
    int prior_off;       // first float of that group's fields inside the prior's per-image block
    int pad;
};

struct RenderGeom {
    int mode, B, N, C, H, W, tile, odds, has_theta, max_oct, n_coarse, ngroups;
    int y0, y1;  // native row band
    float cutoff, base_texels, rep;
    int tiles_per_image;
    long long fld_per_image;  // floats of group fields per image
    long long cap;            // pair capacity of the workspace
    int order[GS_MAX_GROUPS]; // summation order of groups in the composite (the reference's order)
    // reuse of a prior render's group fields: splats [0, skip_n) of each image whose octave at the prior's
    // representative size prior_rep is the prior group mapped to their group here are not binned; the
    // prior group's fields are added to this group's fields instead
    int skip_n;
    float prior_rep;
    GroupGeom g[GS_MAX_GROUPS];
};

// One splat, pre-transformed for rendering: 48 bytes, 16-byte aligned.
//   a = {mu_y, mu_x, A, Bc}   u = A*dy + Bc*dx  (= K * rotated_y / sigma_y)
//   b = {Cc, D, op, log2(op)} v = Cc*dy + D*dx  (= K * rotated_x / sigma_x)
//   c = {col0, col1, col2, dead}; dead = 1 when op <= 1/32 (odds weight by series, no rcp)
// with K^2 = 0.5*log2(e) so exp(-maha/2) = 2^-(u^2+v^2).
struct __align__(16) SplatRec {
    float4 a, b, c;
};

#define GS_K 0.84932180028801907f        // sqrt(0.5 * log2(e))
#define GS_ALPHA_MAX (1.0f - 1e-4f)      // render_triton.py:491
#define GS_LN2 0.69314718055994531f
#define GS_DEAD_OP (1.0f / 32.0f)
