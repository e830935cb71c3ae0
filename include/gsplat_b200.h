/*
 * gsplat_b200.h -- C ABI of libgsplat_b200.so, the B200 (sm_100a) kernels behind the
 * gaussian_2d_splat_encoder_b200 Python package.
 *
 * The reference (bigwolfeman/gaussian-2d-splat-encoder) exposes this hot path as Python functions on
 * torch tensors; these entry points are what its wrappers would bind through ctypes/cffi instead of
 * launching Triton kernels.  Each declaration names the reference interface it replaces.
 *
 * Conventions for every entry point:
 *   - pointers are DEVICE pointers (fp32 unless stated), tightly packed in the reference's layouts:
 *       mu [B][N][2] as (y,x) in normalised [0,1] image units; log_scale [B][N][2] pre-softplus;
 *       color [B][N][C]; opacity [B][N] in (0,1); theta [B][N] (may be NULL); bg [B][C];
 *       images [B][C][H][W].
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).  Every call only
 *     enqueues work on that stream; none synchronises it except gs_render_count.
 *   - the return value is a gs_status; nothing aborts the process.
 *   - workspaces are caller-owned device memory of at least the size the matching *_workspace_size
 *     query returns; their contents are private to the library and must stay untouched between a
 *     forward and its backward.
 */
#ifndef GSPLAT_B200_H
#define GSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    GS_OK = 0,
    GS_ERR_PAIR_BUDGET = 1,  /* reference: PairBudgetExceeded (render_triton.py:51-54) */
    GS_ERR_BAD_ARGUMENT = 2, /* reference: ValueError / NotImplementedError / assert */
    GS_ERR_TIMEOUT = 3,      /* a bounded device wait gave up */
    GS_ERR_CUDA = 4,         /* a CUDA runtime call failed (see gs_last_error) */
    GS_ERR_WORKSPACE = 5     /* workspace smaller than the size query asked for */
} gs_status;

/* Render modes: which reference entry point a descriptor describes. */
typedef enum {
    GS_MODE_OCTAVE = 0,   /* render_alpha_octave            render_triton.py:935-980 */
    GS_MODE_CULL = 1,     /* render_alpha_full_triton(cull=True)  render_triton.py:326-347, 538-567 */
    GS_MODE_MULTIRES = 2, /* render_alpha_multires          render_triton.py:879-922 */
    GS_MODE_EXACT = 3     /* render_alpha_full_triton(cull=False) / render.render_alpha_full */
} gs_render_mode;

typedef struct {
    int32_t mode;          /* gs_render_mode */
    int32_t B, N, C;       /* images, splats per image, colour channels (1..3) */
    int32_t H, W;          /* output resolution */
    int32_t tile;          /* TILE: 4, 8 or 16 (reference default 8) */
    int32_t odds;          /* 1: odds weights w = a/(1-a) (render_triton.py:494-499) */
    int32_t has_theta;     /* 0: theta pointer ignored (axis-aligned splats) */
    int32_t max_octaves;   /* octave mode (reference default 6) */
    int32_t n_coarse;      /* multires mode; <=0 or >=N -> single full-resolution group */
    int32_t coarse_factor; /* multires mode (reference default 8) */
    float cutoff;          /* bbox radius in sigmas (reference default 3.0) */
    float base_texels;     /* octave mode (reference default 8.0) */
    int64_t max_pairs;     /* per (image, group) pair budget; < 0 disables the check.  gs_render_fwd refuses a
                              render with more pairs in one (image, group) (GS_ERR_PAIR_BUDGET), as the
                              reference's _build_tiles does (render_triton.py:378-385) */
    int64_t pair_capacity; /* pairs the workspace holds for the whole batch; 0 -> gs_render_pair_bound.  A
                              capacity below the bound makes gs_render_fwd count first and refuse a render
                              that would not fit (GS_ERR_WORKSPACE); pairs are never silently dropped */
    int32_t row_begin;     /* native row band [row_begin, row_end) this call renders (tile-row sharding); */
    int32_t row_end;       /* row_end <= 0 -> all rows.  Output rows outside the band are not written and
                              the backward reads grad_out only inside it. */
} gs_render_desc;

/* Upper bound on the (tile, splat) pairs of the whole batch, computed on the host from the
 * descriptor alone (no device access).  Replaces the pair-count .item() sync of _build_tiles
 * (render_triton.py:378-391) whenever the bound is within budget. */
int64_t gs_render_pair_bound(const gs_render_desc *d);

/* Workspace bytes for a forward (with_backward = 0) or a forward + backward (with_backward = 1); 0 for
 * an invalid descriptor or a pair capacity of 2^31 or more (pair positions are 32-bit; split the batch). */
size_t gs_render_workspace_size(const gs_render_desc *d, int with_backward);

/* Forward render without any caller-provided workspace (no counterpart in the reference).  For callers
 * that cannot allocate device memory -- a host whose device memory belongs to an allocator it cannot
 * call, or a latency-critical path that must not pay for cudaMalloc's implicit synchronisation -- the
 * workspace of gs_render_fwd is taken from a fixed array inside the library instead.  Same arguments
 * and result as gs_render_fwd minus the workspace.  Limits: a render whose forward workspace
 * (gs_render_workspace_size(d, 0)) exceeds GS_NOALLOC_SCRATCH_BYTES is refused with
 * GS_ERR_WORKSPACE before any launch; every GPU that loads the library holds the array until exit;
 * all calls on a device share it, so calls that overlap on the GPU (other streams or threads) race and
 * must be serialised by the caller; the first call on a device looks up the array's address and
 * should come before any stream capture (the address is cached for the process's life, so a
 * cudaDeviceReset needs a reload of the library).  The pair checks of gs_render_fwd apply unchanged.
 * There is no backward variant. */
#define GS_NOALLOC_SCRATCH_BYTES (32u << 20)
int gs_render_fwd_noalloc(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                          const float *opacity, const float *bg, const float *theta, float *out, void *stream);

/* Exact pair counts per (image, group) into counts_host[B * groups] (groups = max_octaves + 1 in octave
 * mode, 2 in multires mode, 1 otherwise); *groups_out receives the group count.  Runs the
 * preprocessing kernel and SYNCHRONISES the stream: the analogue of _build_tiles's budget check
 * (render_triton.py:378-385), used only when the host bound exceeds the budget. */
int gs_render_count(const gs_render_desc *d, const float *mu, const float *log_scale, void *workspace,
                    size_t workspace_bytes, int64_t *counts_host, int32_t *groups_out, void *stream);

/* Forward render: out [B][C][H][W].  Replaces _forward_cull / _forward_cull_fields + the octave loop
 * of render_alpha_octave / render_alpha_multires + the exact _forward (render_triton.py:128-157,
 * 538-600, 879-980).  Keeps the state its backward needs in the workspace.
 * Pair checks: when the host bound (gs_render_pair_bound, per group) cannot rule out a (image, group)
 * count above max_pairs, or pair_capacity is below the bound, the call reads the exact counts back first
 * (one synchronisation of `stream`, like the reference's .item()) and returns GS_ERR_PAIR_BUDGET
 * (budget) or GS_ERR_WORKSPACE (capacity) without rendering.  That read-back is not possible while
 * `stream` is being captured: such a call returns GS_ERR_BAD_ARGUMENT (capture with pair_capacity = 0
 * and a budget the bound satisfies).  The kernels themselves never write past the pair capacity. */
int gs_render_fwd(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                  const float *opacity, const float *bg, const float *theta, float *out, void *workspace,
                  size_t workspace_bytes, void *stream);

/* Backward of gs_render_fwd for upstream gradient grad_out [B][C][H][W]: gradients of all six
 * leaves (g_theta may be NULL).  Replaces _backward / _backward_cull / _backward_cull_fields and the
 * torch autograd of the upsample + composite (render_triton.py:269-303, 723-810, 864-980). */
int gs_render_bwd(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                  const float *opacity, const float *bg, const float *theta, const float *grad_out, float *g_mu,
                  float *g_log_scale, float *g_color, float *g_opacity, float *g_bg, float *g_theta,
                  void *workspace, size_t workspace_bytes, void *stream);

/* Pixel-list render: replaces render_alpha_subsampled (render.py:68-87) and the torch autograd of its
 * alpha_composite (render.py:47-65).  All N splats of image b are composited (alpha mode, no binning) at
 * the P pixels px_idx[b][0..P) (flat indices y*W + x, int64, as torch.randint returns them).
 * d->mode must be GS_MODE_EXACT and d->odds 0; tile, cutoff and the octave fields are ignored.
 * out is [B][C][P].  The forward keeps the per-pixel sums in the workspace for the backward, which
 * takes grad_out [B][C][P] and writes the gradients of the six leaves (g_theta may be NULL). */
size_t gs_render_points_workspace_size(const gs_render_desc *d, int32_t P, int with_backward);
int gs_render_points_fwd(const gs_render_desc *d, int32_t P, const int64_t *px_idx, const float *mu,
                         const float *log_scale, const float *color, const float *opacity, const float *bg,
                         const float *theta, float *out, void *workspace, size_t workspace_bytes, void *stream);
int gs_render_points_bwd(const gs_render_desc *d, int32_t P, const int64_t *px_idx, const float *log_scale,
                         const float *bg, const float *theta, const float *grad_out, float *g_mu,
                         float *g_log_scale, float *g_color, float *g_opacity, float *g_bg, float *g_theta,
                         void *workspace, size_t workspace_bytes, void *stream);

/* Debug/parity accessors for the binning held in a forward's workspace (octave/cull/multires):
 * copies (SYNCHRONOUSLY) the total pair count, the per-group geometry and the sorted CSR so tests can
 * compare it bit-exactly with the reference's _build_tiles (render_triton.py:351-409).
 * tile_ranges_host receives [B * tiles_per_image][2] (begin, end); splat_ids_host receives
 * [total_pairs] global splat ids (b * N + i); geom_host receives per group
 * {H, W, ntx, nty, tile_offset}. Any output pointer may be NULL. */
int gs_render_debug_bins(const gs_render_desc *d, const void *workspace, int64_t *total_pairs,
                         int32_t *tiles_per_image, int32_t *geom_host, int32_t *tile_ranges_host,
                         int32_t *splat_ids_host, int32_t *octave_host);

/* One encoder convolution on the tensor cores: NHWC bf16 input [B][H][W][Cin], packed bf16 weights
 * [Cout][kh*kw*Cin] (tap-major, channel-minor), fp32 bias, NHWC bf16 output [B][Ho][Wo][Cout] with
 * bias + (optional) GELU applied (erf form, |error| < 7e-7 before the bf16 rounding); when gn_stats
 * is non-NULL the GroupNorm(8) partial sums (sum, sum of squares) of the output are ADDED to
 * gn_stats[B][8][2].  kind 0: Cin a multiple of 64,
 * stride 1 or 2; kind 1: the encoder's first layer expressed on its space-to-depth input (Cin = 16,
 * 4x4 taps, stride 1, pad 2, output Ho x Wo given explicitly).  Cout in {64, 128, 256}.  err_flag
 * (device int, may be NULL) receives a non-zero code if a bounded device wait gave up.
 * Replaces nn.Conv2d + nn.GELU of the reference encoder (efficient_encoder.py:53-58, 86-87). */
typedef struct {
    int32_t B, H, W, Cin;
    int32_t Cout, kh, kw, stride, pad;
    int32_t Ho, Wo; /* 0 -> derived from the standard formula */
    int32_t gelu;
    int32_t kind;
} gs_conv_desc;

int gs_conv2d(const gs_conv_desc *d, const void *in_bf16, const void *w_bf16, const float *bias, void *out_bf16,
              double *gn_stats, int *err_flag, void *stream);

/* EfficientGaussianEncoder, variant 'adaptive' (efficient_encoder.py:200-378) with d_feature 256,
 * stride 8, fine_stride 4, GroupNorm, gradient input: the released checkpoint's architecture. */
typedef struct {
    int32_t B, H, W;           /* image batch [B][3][H][W], H and W multiples of 8 */
    int32_t d;                 /* d_feature (256) */
    int32_t M, Mf;             /* coarse / fine splats per cell (1..2) */
    int32_t residual_grid;     /* resolution of the internal coarse render */
    int32_t odds;              /* odds compositing of the internal render */
    int32_t use_rotation;      /* theta heads present */
    float coarse_ls_floor;     /* softplus^-1(coarse_min_scale), or -inf for none */
    float coarse_offset, fine_offset; /* offset_cells of the two heads */
    float coarse_min_opacity;  /* coarse opacity floor */
} gs_encoder_desc;

/* Device pointers of the packed weights (see gaussian_2d_splat_encoder_b200/efficient_encoder.py):
 * w1 bf16 [64][256] (first layer on the space-to-depth input), w2 bf16 [128][576], w3 bf16 [256][1152],
 * w4 bf16 [128][3456] (decoder), fp32 biases and GroupNorm affine parameters, bg head [3][256] + [3],
 * coarse head [9*M][257] + [9*M], fine head [9*Mf][133] + [9*Mf] (rows: mu, scale, colour, opacity,
 * theta). */
typedef struct {
    const void *w1, *w2, *w3, *w4;
    const float *b1, *b2, *b3, *b4;
    const float *gn1_w, *gn1_b, *gn2_w, *gn2_b, *gn3_w, *gn3_b, *gn4_w, *gn4_b;
    const float *bg_w, *bg_b, *hc_w, *hc_b, *hf_w, *hf_b;
} gs_encoder_weights;

size_t gs_encoder_workspace_size(const gs_encoder_desc *e);

/* Encoder forward of a batch: outputs in the reference's layouts with N = 2*(H/8)(W/8)*M/2... precisely
 * N = (H/8)(W/8)M + (H/4)(W/4)Mf splats per image ordered [coarse | fine], cell-major then slot:
 * mu [B][N][2], log_scale [B][N][2], color [B][N][3], opacity [B][N], theta [B][N] (if use_rotation),
 * bg [B][3]; features (optional) receives backbone_features as NHWC fp32 [B][H/8][W/8][256]; latents
 * (optional) receives the normalised fine-decoder features, NHWC fp32 [B][H/4][W/4][128]
 * (splat_features of forward(return_latents=True)).
 * Replaces EfficientGaussianEncoder.forward (efficient_encoder.py:306-378), including its internal
 * render_alpha_octave call. */
int gs_encoder_fwd(const gs_encoder_desc *e, const gs_encoder_weights *w, const float *image, float *mu,
                   float *log_scale, float *color, float *opacity, float *theta, float *bg, float *features,
                   float *latents, void *workspace, size_t workspace_bytes, void *stream);

/* Encoder forward followed by render_alpha_octave of its splats at the image size, in one call: the
 * pipeline of examples/encode_and_render.py:31-38 with render_alpha_octave's defaults (TILE 8, cutoff 3,
 * base_texels 8, max_octaves 6, max_pairs 48e6, odds = the encoder's odds).  Outputs as gs_encoder_fwd,
 * plus the reconstruction out [B][3][H][W].  When H = W = 2 * residual_grid the coarse splats fall on the
 * same texel grids in both of the path's renders (octave k of the encoder's internal coarse render is
 * octave k + 1 of the final one), so the final render adds those octaves' fields from the internal render
 * instead of binning and compositing the coarse splats again (sums are regrouped: results agree with the
 * two separate calls to fp32 rounding).  The workspace holds the encoder's and the render's. */
size_t gs_encode_render_workspace_size(const gs_encoder_desc *e);
int gs_encode_render_fwd(const gs_encoder_desc *e, const gs_encoder_weights *w, const float *image, float *mu,
                         float *log_scale, float *color, float *opacity, float *theta, float *bg, float *features,
                         float *latents, float *out, void *workspace, size_t workspace_bytes, void *stream);

/* Debug accessor of a gs_encode_render_fwd workspace (SYNCHRONOUS, like gs_render_debug_bins): pairs[0] =
 * (tile, splat) pairs of the encoder's internal coarse render, pairs[1] = pairs the final render binned
 * (the coarse splats whose fields it reused from the internal render are not binned again). */
int gs_encode_render_debug_pairs(const gs_encoder_desc *e, const void *workspace, int64_t *pairs);

/* Reads (synchronously) the bounded-wait error flag left in an encoder workspace (0 = none). */
int gs_encoder_error_flag(const gs_encoder_desc *e, const void *workspace, int *flag_host);

/* Fused L2 loss of a fitting step over rows [row_begin, row_end) (row_end <= 0: all rows) of `planes`
 * H x W fp32 images: grad = 2*scale*(out - target) inside the band (other rows untouched) and
 * *loss = scale * sum (out - target)^2 (loss is a device float, zeroed by the call).  With
 * scale = 1/(planes*H*W) this is mse_loss and its gradient (the loss of the reference's fitting
 * configurations); with a band it is that band's share. */
int gs_l2_loss_grad(const float *out, const float *target, int64_t planes, int32_t H, int32_t W, int32_t row_begin,
                    int32_t row_end, float scale, float *grad, float *loss, void *stream);

/* activate_scale (params.py:18-28): out = softplus(log_scale) + 1e-4, n elements. */
int gs_activate_scale(const float *log_scale, float *out, int64_t n, void *stream);

/* Text of the last CUDA error seen by the calling thread (empty when none). */
const char *gs_last_error(void);

/* Number of kernels (memsets included) this library has enqueued since it was loaded; benchmarks
 * read it before and after a timed region to report their launch count. */
uint64_t gs_kernel_launches(void);

/* Device-time profiling of library stages.  While enabled, the entry points record CUDA events on
 * their stream around each stage; gs_profile_collect waits for them and returns per-stage totals (ms)
 * and call counts (arrays of 16): 0 binning (preprocess..tile ranges), 1 fields forward, 2 composite,
 * 3 composite backward + upsample adjoint, 4 fields backward, 5 finalize, 6 binning and 7 fields forward
 * of the encoder's internal coarse render, 8 encoder input preparation,
 * 9..12 encoder convolutions 1..4, 13 encoder heads, 14 encoder GroupNorm/concat/cond, 15 the
 * encoder's internal coarse render. */
void gs_profile_enable(int on);
int gs_profile_collect(double *ms_out, int64_t *count_out);
/* As gs_profile_collect; keep != 0 leaves the event slots assigned (for a captured CUDA graph that
 * records them on every replay). */
int gs_profile_collect2(double *ms_out, int64_t *count_out, int keep);

/* Library version and the compute capability it was built for (100 = sm_100a). */
int gs_build_arch(void);

#ifdef __cplusplus
}
#endif

#endif /* GSPLAT_B200_H */
