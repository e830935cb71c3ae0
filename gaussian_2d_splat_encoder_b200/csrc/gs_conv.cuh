// Internal interface of the tcgen05 convolution (gs_conv.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/gsplat_b200.h"

struct ConvArgs {
    int B, Hi, Wi, Ci, Co;
    int KH, KW, stride, pad;  // pad: rows (and columns unless padw says otherwise)
    int padw;                 // column padding
    int Ho, Wo;
    int TX, TY, tiles_x, tiles_y;
    int nchunks, nkb;
    int nchunks1;  // input-channel chunks read from the first input (the rest from the second)
    int gelu;
    const float *bias;
    __nv_bfloat16 *out;
    double *stats;  // [B][8][2] GroupNorm partial sums (sum, sum of squares), accumulated
    int *err;       // set to a non-zero stage code when a bounded wait gives up
    // halo form (stride 1, one input-channel chunk): per item one window of hrows x hcols pixels per 8-channel
    // slice (hslice bytes apart), every tap an offset view of it; hbreg bytes of weights loaded once per CTA
    int hrows, hcols, hslice, hbreg;
};

void gs_conv_pick_tile(int Ho, int Wo, int MT, int *TX, int *TY);
int gs_conv_run(const gs_conv_desc *d, const void *in, const void *w, const float *bias, void *out, double *stats,
                int *err, cudaStream_t st);
// The same convolution over the channel concatenation [in (Cin1 channels), in2 (d->Cin - Cin1 channels)],
// both NHWC with the same B, H, W; neither is copied.
// padw >= 0 overrides the column padding (d->pad stays the row padding).
int gs_conv_run2(const gs_conv_desc *d, const void *in, int Cin1, const void *in2, const void *w, const float *bias,
                 void *out, double *stats, int *err, cudaStream_t st, int padw = -1);
