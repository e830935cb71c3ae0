// Internal interface between the renderer (gs_render.cu) and the encoder (gs_encoder.cu): a forward render
// that reuses the group fields of an earlier render of a subset of its splats.
#pragma once
#include <cuda_runtime.h>

#include "../../include/gsplat_b200.h"
#include "gs_common.cuh"

struct GsPrior {
    const float *fields;         // the earlier render's group fields, [B][fld_per_image] (its workspace)
    long long fld_per_image;
    int skip_n;                  // splats [0, skip_n) of every image are the earlier render's splats
    float rep;                   // min(H, W) of the earlier render (its octave routing size)
    int grp[GS_MAX_GROUPS];      // group of this render -> group of the earlier one (-1: none)
    int off[GS_MAX_GROUPS];      // that group's first float inside the earlier render's per-image fields
};

// Map the groups of render `d` onto those of the earlier octave render `prior_d` of its first n_prior
// splats (per image) whose workspace is `prior_ws`.  Group k here takes prior group k - 1 when every
// splat the earlier render routed to k - 1 routes to k here with the same texel grid (min(H, W) exactly
// twice the earlier one, both renders with the same tile, cutoff, base texels, octave count and weight
// form, k - 1 neither the first nor the clamped last octave).  Returns the number of mapped groups.
int gs_render_prior_map(const gs_render_desc *prior_d, const void *prior_ws, const gs_render_desc *d, int n_prior,
                        GsPrior *out);

// gs_render_fwd with a prior (NULL: plain gs_render_fwd).
int gs_render_fwd_prior(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                        const float *opacity, const float *bg, const float *theta, float *out, const GsPrior *prior,
                        void *workspace, size_t workspace_bytes, void *stream);

// Sets the text gs_last_error returns to the calling thread.
void gs_set_last_error(const char *msg);
