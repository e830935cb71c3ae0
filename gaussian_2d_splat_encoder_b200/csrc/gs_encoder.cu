// gs_encoder.cu -- EfficientGaussianEncoder('adaptive') forward on B200 (reference:
// bigwolfeman/gaussian-2d-splat-encoder, gaussian_splat_encoder/efficient_encoder.py:306-378).
//
//   k_prep        grey, Sobel/4, gradient magnitude (efficient_encoder.py:123-130) and the
//                 space-to-depth bf16 input of the first convolution
//   k_pool48      4x4 and 8x8 pooled gradients in one pass
//   conv1..3      tcgen05 implicit GEMM (gs_conv.cu): 7x7/2 (on the space-to-depth tensor as 4x4/1),
//                 3x3/2, 3x3/2, bias + GELU + GroupNorm statistics fused (efficient_encoder.py:53-58)
//   k_gn_apply    GroupNorm(8) normalise + affine in place (NHWC bf16); the last one also sums the
//                 channels for the background head
//   k_bg          sigmoid(Linear(mean_hw(s8)))               (efficient_encoder.py:267-268)
//   k_head        1x1 head + activations of one splat group   (efficient_encoder.py:170-197, 340-342)
//   coarse render render_alpha_octave at residual_grid^2 with odds (gs_render.cu)
//   k_cond        bilinear(image -> grid), |target - render|, mean(render)   (efficient_encoder.py:349-351)
//   k_upsample    bilinear(s8 -> s4 size)  (the _UpBlock input is [this, s4], efficient_encoder.py:89-91)
//   conv4         3x3/1 384->128 decoder convolution on the tensor cores, reading [up, s4] in place
//   k_head (fine) GroupNorm applied on the fly, [fine_feat, pooled gradient, bilinear(cond)] 1x1 head
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../include/gsplat_b200.h"
#include "gs_conv.cuh"
#include "gs_prof.cuh"
#include "gs_render_internal.cuh"

namespace {

__device__ __forceinline__ void lin_idx(int d, int in_size, int out_size, int &i0, int &i1, float &l0, float &l1) {
    float scale = (float)in_size / (float)out_size;
    float src = scale * ((float)d + 0.5f) - 0.5f;
    if (src < 0.0f) src = 0.0f;
    int i = (int)src;
    if (i > in_size - 1) i = in_size - 1;
    int ip = (i < in_size - 1) ? 1 : 0;
    float lam = fminf(fmaxf(src - (float)i, 0.0f), 1.0f);
    i0 = i;
    i1 = i + ip;
    l1 = lam;
    l0 = 1.0f - lam;
}

// torch.linspace(0.5/n, 1-0.5/n, n)[i] in fp32 (efficient_encoder.py:174-175)
__device__ __forceinline__ float lin_center(int i, int n) {
    float start = 0.5f / (float)n, end = 1.0f - 0.5f / (float)n;
    if (n == 1) return start;
    float step = (end - start) / (float)(n - 1);
    return i < n / 2 ? start + step * (float)i : end - step * (float)(n - 1 - i);
}

// grad [B][H][W] fp32 and the space-to-depth bf16 input Z[B][H/2][W/2][16],
// Z[p][q][(dy*2+dx)*4 + c] = X[2p+dy][2q+dx][c], X = (R, G, B, grad).
// A block = 32 x 8 Z cells (64 x 16 pixels) of one image (grid = (ceil(W/64), ceil(H/16), B)): the grey
// values of the tile and its one-pixel halo (zero outside the image, the convolution's padding) are
// computed once into shared memory, then each thread takes the 4x4 grey neighbourhood of its 2x2 pixels.
#define PREP_TX 32
#define PREP_TY 8
__global__ void __launch_bounds__(256) k_prep(const float *__restrict__ image, int B, int H, int W,
                                              float *__restrict__ grad, __nv_bfloat16 *__restrict__ Z) {
    constexpr int GW = 2 * PREP_TX + 2, GH = 2 * PREP_TY + 2;
    __shared__ float gs[GH][GW + 1];
    __shared__ uint2 rgb[GH - 2][GW - 2];  // the tile's own pixels as bf16 (R, G, B, 0) for Z
    const int b = blockIdx.z;
    const int Hz = H / 2, Wz = W / 2;
    const float *img = image + (long long)b * 3 * H * W;
    const long long P = (long long)H * W;
    const int y0 = 2 * PREP_TY * blockIdx.y - 1, x0 = 2 * PREP_TX * blockIdx.x - 1;
    for (int k = threadIdx.x; k < GH * GW; k += blockDim.x) {
        const int a = k / GW, c = k - a * GW;
        const int y = y0 + a, x = x0 + c;
        float v = 0.0f, r = 0.f, g = 0.f, bl = 0.f;
        if (y >= 0 && y < H && x >= 0 && x < W) {
            const long long pp = (long long)y * W + x;
            r = img[pp];
            g = img[P + pp];
            bl = img[2 * P + pp];
            v = (r + g + bl) / 3.0f;
        }
        gs[a][c] = v;
        if (a >= 1 && a <= GH - 2 && c >= 1 && c <= GW - 2) {
            const __nv_bfloat162 rg = __floats2bfloat162_rn(r, g), b0 = __floats2bfloat162_rn(bl, 0.f);
            rgb[a - 1][c - 1] = make_uint2(*reinterpret_cast<const uint32_t *>(&rg), *reinterpret_cast<const uint32_t *>(&b0));
        }
    }
    __syncthreads();
    const int tx = threadIdx.x % PREP_TX, ty = threadIdx.x / PREP_TX;
    const int q = blockIdx.x * PREP_TX + tx, p = blockIdx.y * PREP_TY + ty;
    if (p >= Hz || q >= Wz) return;
    // 4x4 grey neighbourhood of the 2x2 block: rows 2p-1 .. 2p+2, columns 2q-1 .. 2q+2
    float g[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) g[a][c] = gs[2 * ty + a][2 * tx + c];
    __align__(16) __nv_bfloat16 z[16];
    float gmv[2][2];
#pragma unroll
    for (int dy = 0; dy < 2; dy++)
#pragma unroll
        for (int dx = 0; dx < 2; dx++) {
            // F.conv2d with kx = [[-1,0,1],[-2,0,2],[-1,0,1]]/4, ky = kx^T (cross-correlation, zero pad)
            float gx = 0.f, gy = 0.f;
            const float k[3][3] = {{-1.f, 0.f, 1.f}, {-2.f, 0.f, 2.f}, {-1.f, 0.f, 1.f}};
#pragma unroll
            for (int u = 0; u < 3; u++)
#pragma unroll
                for (int v = 0; v < 3; v++) {
                    float gv = g[dy + u][dx + v];
                    gx += (k[u][v] / 4.0f) * gv;
                    gy += (k[v][u] / 4.0f) * gv;
                }
            const float gm = sqrtf(gx * gx + gy * gy + 1e-6f);
            gmv[dy][dx] = gm;
            const int base = (dy * 2 + dx) * 4;
            const uint2 c3 = rgb[2 * ty + dy][2 * tx + dx];
            const __nv_bfloat16 *e3 = reinterpret_cast<const __nv_bfloat16 *>(&c3);
            z[base + 0] = e3[0];
            z[base + 1] = e3[1];
            z[base + 2] = e3[2];
            z[base + 3] = __float2bfloat16_rn(gm);
        }
#pragma unroll
    for (int dy = 0; dy < 2; dy++)
        *reinterpret_cast<float2 *>(grad + (long long)b * P + (long long)(2 * p + dy) * W + 2 * q) =
            make_float2(gmv[dy][0], gmv[dy][1]);
    uint4 *dst = reinterpret_cast<uint4 *>(Z + (((long long)b * Hz + p) * Wz + q) * 16);
    dst[0] = reinterpret_cast<uint4 *>(z)[0];
    dst[1] = reinterpret_cast<uint4 *>(z)[1];
}

// adaptive_avg_pool2d of grad to (H/4, W/4) and (H/8, W/8) (H, W multiples of 8): eight consecutive
// lanes own one 8x8 block, lane a loading row a with two 16-byte loads; row sums meet by shuffles.
__global__ void __launch_bounds__(256) k_pool48(const float *__restrict__ grad, int B, int H, int W,
                                                float *__restrict__ out4, float *__restrict__ out8) {
    const int H8 = H / 8, W8 = W / 8;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = t >> 3, a = t & 7;
    const bool live = i < B * H8 * W8;
    const int ii = live ? i : 0;
    const int b = ii / (H8 * W8);
    const int r = ii - b * H8 * W8;
    const int y = r / W8, x = r - y * W8;
    const float *g = grad + (long long)b * H * W + (long long)(8 * y + a) * W + 8 * x;
    const float4 lo = *reinterpret_cast<const float4 *>(g);
    const float4 hi = *reinterpret_cast<const float4 *>(g + 4);
    float sl = ((lo.x + lo.y) + lo.z) + lo.w, sh = ((hi.x + hi.y) + hi.z) + hi.w;
    // 4-row sums (rows 0-3 or 4-7 of the block), then the whole block
    sl += __shfl_xor_sync(0xffffffffu, sl, 1);
    sh += __shfl_xor_sync(0xffffffffu, sh, 1);
    sl += __shfl_xor_sync(0xffffffffu, sl, 2);
    sh += __shfl_xor_sync(0xffffffffu, sh, 2);
    float s8 = sl + sh;
    s8 += __shfl_xor_sync(0xffffffffu, s8, 4);
    if (!live) return;
    const int W4 = W / 4;
    if ((a & 3) == 0) {
        float *o4 = out4 + (long long)b * (H / 4) * W4 + (long long)(2 * y + (a >> 2)) * W4 + 2 * x;
        o4[0] = sl / 16.0f;
        o4[1] = sh / 16.0f;
    }
    if (a == 0) out8[i] = s8 / 64.0f;
}

// GroupNorm(8) of channel c of image b as y * sc + sh, from the (sum, sum of squares) statistics
__device__ __forceinline__ void gn_affine(const double *__restrict__ stats, const float *__restrict__ gamma,
                                          const float *__restrict__ beta, int b, int c, int C, long long HW,
                                          float &sc, float &sh) {
    const int g = c / (C / 8);
    const double n = (double)HW * (C / 8);
    const double mean = stats[(b * 8 + g) * 2] / n;
    double var = stats[(b * 8 + g) * 2 + 1] / n - mean * mean;
    if (var < 0) var = 0;
    const float rstd = (float)(1.0 / sqrt(var + 1e-5));
    sc = gamma[c] * rstd;
    sh = beta[c] - (float)mean * gamma[c] * rstd;
}

// GroupNorm(8) apply in place on NHWC bf16 [B][HW][C]; chsum (optional) receives this block's per-channel
// sums of the normalised values, chsum[b][blockIdx.x][C] (k_bg reduces them in a fixed order, so the
// background colour is reproducible bit for bit).  Each thread handles 8-channel vectors of one fixed
// channel octet (the grid stride in channels, gridDim.x * 256 * 8, is a multiple of C), so its
// scale/shift and its channel sums stay in registers.
// With apply = 0 the tensor is only read and chsum receives the sums of the raw values.
__global__ void __launch_bounds__(256) k_gn_apply(__nv_bfloat16 *__restrict__ x, int HW, int C,
                                                  const double *__restrict__ stats, const float *__restrict__ gamma,
                                                  const float *__restrict__ beta, float *__restrict__ chsum,
                                                  int apply) {
    __shared__ float red[256][9];
    const int b = blockIdx.y;
    const int nvec = HW * (C / 8);
    const int stride = gridDim.x * blockDim.x;
    int v = blockIdx.x * blockDim.x + threadIdx.x;
    const int c0 = (v * 8) % C;
    const int g = c0 / (C / 8);
    const double n = (double)HW * (C / 8);
    const double mean = stats[(b * 8 + g) * 2] / n;
    double var = stats[(b * 8 + g) * 2 + 1] / n - mean * mean;
    if (var < 0) var = 0;
    const float rstd = (float)(1.0 / sqrt(var + 1e-5));
    float sc[8], sh[8], cs[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        sc[k] = gamma[c0 + k] * rstd;
        sh[k] = beta[c0 + k] - (float)mean * gamma[c0 + k] * rstd;
        cs[k] = 0.f;
    }
    uint4 *xb = reinterpret_cast<uint4 *>(x + (long long)b * HW * C);
    auto norm = [&](uint4 &u) {
        __nv_bfloat16 *e = reinterpret_cast<__nv_bfloat16 *>(&u);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (apply) e[k] = __float2bfloat16_rn(fmaf(__bfloat162float(e[k]), sc[k], sh[k]));
            cs[k] += __bfloat162float(e[k]);
        }
    };
    // four vectors in flight per thread, then two, then one (the sums keep the order of the vectors)
    for (; v + 3 * stride < nvec; v += 4 * stride) {
        uint4 u0 = xb[v], u1 = xb[v + stride], u2 = xb[v + 2 * stride], u3 = xb[v + 3 * stride];
        norm(u0);
        norm(u1);
        norm(u2);
        norm(u3);
        if (apply) {
            xb[v] = u0;
            xb[v + stride] = u1;
            xb[v + 2 * stride] = u2;
            xb[v + 3 * stride] = u3;
        }
    }
    if (v + stride < nvec) {
        uint4 u0 = xb[v], u1 = xb[v + stride];
        norm(u0);
        norm(u1);
        if (apply) {
            xb[v] = u0;
            xb[v + stride] = u1;
        }
        v += 2 * stride;
    }
    if (v < nvec) {
        uint4 u0 = xb[v];
        norm(u0);
        if (apply) xb[v] = u0;
    }
    if (chsum) {
        // threads t, t + C/8, t + 2C/8, ... share a channel octet: sum their registers in thread order
#pragma unroll
        for (int k = 0; k < 8; k++) red[threadIdx.x][k] = cs[k];
        __syncthreads();
        const int oct = C / 8;
        for (int c = threadIdx.x; c < C; c += blockDim.x) {
            float t = 0.f;
            for (int j = c / 8; j < (int)blockDim.x; j += oct) t += red[j][c % 8];
            chsum[((long long)b * gridDim.x + blockIdx.x) * C + c] = t;
        }
    }
}

// bg = sigmoid(W * mean_hw(s8) + b) (efficient_encoder.py:308-309); one block of C threads per image: thread
// c sums channel c's nblk block partials in order, then the three dot products reduce over the block
__global__ void __launch_bounds__(1024) k_bg(const float *__restrict__ chsum, int nblk, int C, long long HW,
                                             const float *__restrict__ w, const float *__restrict__ bias,
                                             const double *__restrict__ gn_stats, const float *__restrict__ gn_gamma,
                                             const float *__restrict__ gn_beta, float2 *__restrict__ gn_table,
                                             float *__restrict__ bg) {
    // 4 threads per channel (C <= 256), each a quarter of the nblk partials with 4 independent running
    // sums (loads in flight together), combined in a fixed order: reproducible
    __shared__ float part[4][256];
    __shared__ float red[3][8];
    const int b = blockIdx.x, c = threadIdx.x & 255, pq = threadIdx.x >> 8;
    if (c < C) {
        const int k0 = pq * nblk / 4, k1 = (pq + 1) * nblk / 4;
        const float *src = chsum + (long long)b * nblk * C + c;
        float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
        int k = k0;
        for (; k + 4 <= k1; k += 4) {
            t0 += src[(long long)k * C];
            t1 += src[(long long)(k + 1) * C];
            t2 += src[(long long)(k + 2) * C];
            t3 += src[(long long)(k + 3) * C];
        }
        for (; k < k1; k++) t0 += src[(long long)k * C];
        part[pq][c] = (t0 + t1) + (t2 + t3);
    }
    __syncthreads();
    if (threadIdx.x >= 256) return;
    const int lane = c & 31, warp = c >> 5;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    if (c < C) {
        float t = (part[0][c] + part[1][c]) + (part[2][c] + part[3][c]);
        float m = t / (float)HW;
        if (gn_stats) {  // the sums are of the raw values: mean of the normalised = scale * mean + shift
            float sc, sh;
            gn_affine(gn_stats, gn_gamma, gn_beta, b, c, C, HW, sc, sh);
            m = fmaf(m, sc, sh);
            gn_table[b * C + c] = make_float2(sc, sh);  // for the other consumers of the raw tensor
        }
        s0 = w[c] * m;
        s1 = w[C + c] * m;
        s2 = w[2 * C + c] * m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
        red[0][warp] = s0;
        red[1][warp] = s1;
        red[2][warp] = s2;
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the first 256 threads only
    if (c < 3) {
        float s = bias[c];
        for (int k = 0; k < 8; k++) s += red[c][k];
        bg[b * 3 + c] = 1.0f / (1.0f + expf(-s));
    }
}

#define GN_BG_BLOCKS 128  // blocks of the GroupNorm launch that also sums channels for the background head

#define HEAD_NP 20     // head outputs (9 per splat, 2 splats per cell) padded to a multiple of 4
#define HEAD_CELLS 32  // cells per warp of k_head

struct HeadArgs {
    int B, fH, fW, M;          // grid and splats per cell
    int Cfeat;                 // feature channels read from `feat` (NHWC bf16)
    const __nv_bfloat16 *feat;
    const double *gn_stats;    // if non-NULL, feat is pre-GroupNorm: normalise on the fly
    const float *gn_gamma, *gn_beta;
    const float *gpool;        // [B][fH][fW] pooled gradient (extra channel Cfeat)
    const float *cond;         // [B][rg][rg][4] or NULL: bilinear-sampled extra channels Cfeat+1..+4
    int rg;
    const float *w, *b;        // [nout][Cin], [nout]; rows: mu(2M), scale(2M), colour(3M), opacity(M), theta(M)
    int Cin, nout;
    float off_scale, ls_floor, min_op;
    int use_rot;
    // outputs: API tensors [B][Ntot][...] at splat offset n0, plus optional contiguous copies
    int Ntot, n0;
    float *mu, *ls, *col, *op, *th;
    float *cmu, *cls, *ccol, *cop, *cth;  // contiguous [B][fH*fW*M] copies (coarse render input)
    // k_head_tc operands (k_head_prep): B fragments and bias' per image, the extra channels' weights
    const uint4 *frag;
    const float *fbias, *wext;
};

// acc += the extra input channels of a head: the pooled gradient (channel Cfeat) and, for the fine
// head, the bilinear-sampled cond map (Cfeat+1..+4); wext = their weights, [Cin - Cfeat][HEAD_NP]
__device__ __forceinline__ void head_extra(const HeadArgs &a, const float *wext, long long cell, int b, int y, int x,
                                           float (&acc)[HEAD_NP]) {
    auto fma_row = [&](int e, float v) {
        const float4 *wc = reinterpret_cast<const float4 *>(wext + e * HEAD_NP);
#pragma unroll
        for (int q = 0; q < HEAD_NP / 4; q++) {
            const float4 w4 = wc[q];
            acc[4 * q + 0] = fmaf(w4.x, v, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(w4.y, v, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(w4.z, v, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(w4.w, v, acc[4 * q + 3]);
        }
    };
    fma_row(0, a.gpool[cell]);
    if (a.cond) {
        int y0, y1, x0, x1;
        float h0, h1, w0, w1;
        lin_idx(y, a.rg, a.fH, y0, y1, h0, h1);
        lin_idx(x, a.rg, a.fW, x0, x1, w0, w1);
        const float *cb = a.cond + (long long)b * a.rg * a.rg * 4;
        const float4 c00 = *reinterpret_cast<const float4 *>(cb + ((long long)y0 * a.rg + x0) * 4);
        const float4 c01 = *reinterpret_cast<const float4 *>(cb + ((long long)y0 * a.rg + x1) * 4);
        const float4 c10 = *reinterpret_cast<const float4 *>(cb + ((long long)y1 * a.rg + x0) * 4);
        const float4 c11 = *reinterpret_cast<const float4 *>(cb + ((long long)y1 * a.rg + x1) * 4);
        fma_row(1, h0 * (w0 * c00.x + w1 * c01.x) + h1 * (w0 * c10.x + w1 * c11.x));
        fma_row(2, h0 * (w0 * c00.y + w1 * c01.y) + h1 * (w0 * c10.y + w1 * c11.y));
        fma_row(3, h0 * (w0 * c00.z + w1 * c01.z) + h1 * (w0 * c10.z + w1 * c11.z));
        fma_row(4, h0 * (w0 * c00.w + w1 * c01.w) + h1 * (w0 * c10.w + w1 * c11.w));
    }
}

// activations and stores of cell (b, r = y * fW + x) of a head (efficient_encoder.py:170-197): the splat
// slots m with m % NFIN == part.  Channel layout of acc: (m, component) per parameter block.
// M (splats per cell) is a template parameter so every acc[] index is static and acc stays in registers.
template <int M, int NFIN>
__device__ __forceinline__ void head_activate(const HeadArgs &a, int part, int b, int r, int y, int x,
                                              const float (&acc)[HEAD_NP]) {
    const float by = lin_center(y, a.fH), bx = lin_center(x, a.fW);
#pragma unroll
    for (int m = 0; m < M; m++) {
        if (m % NFIN != part) continue;
        const long long nl = (long long)r * M + m;  // splat index inside the group (cell-major, then slot)
        const long long n = (long long)b * a.Ntot + a.n0 + nl;
        float muy = by + tanhf(acc[m * 2 + 0]) * a.off_scale;
        float mux = bx + tanhf(acc[m * 2 + 1]) * a.off_scale;
        muy = fminf(fmaxf(muy, 0.005f), 0.995f);
        mux = fminf(fmaxf(mux, 0.005f), 0.995f);
        float ly = acc[2 * M + m * 2 + 0], lx = acc[2 * M + m * 2 + 1];
        ly = fmaxf(ly, a.ls_floor);
        lx = fmaxf(lx, a.ls_floor);
        float cc[3];
#pragma unroll
        for (int c = 0; c < 3; c++) cc[c] = 1.0f / (1.0f + expf(-acc[4 * M + m * 3 + c]));
        float o = 1.0f / (1.0f + expf(-acc[7 * M + m]));
        if (a.min_op > 0.f) o = a.min_op + (1.0f - a.min_op) * o;
        float t = a.use_rot ? tanhf(acc[8 * M + m]) * 1.5707963267948966f : 0.f;
        a.mu[n * 2] = muy; a.mu[n * 2 + 1] = mux;
        a.ls[n * 2] = ly; a.ls[n * 2 + 1] = lx;
#pragma unroll
        for (int c = 0; c < 3; c++) a.col[n * 3 + c] = cc[c];
        a.op[n] = o;
        if (a.use_rot && a.th) a.th[n] = t;
        if (a.cmu) {
            const long long q = (long long)b * a.fH * a.fW * M + nl;
            a.cmu[q * 2] = muy; a.cmu[q * 2 + 1] = mux;
            a.cls[q * 2] = ly; a.cls[q * 2 + 1] = lx;
#pragma unroll
            for (int c = 0; c < 3; c++) a.ccol[q * 3 + c] = cc[c];
            a.cop[q] = o;
            if (a.cth) a.cth[q] = t;
        }
    }
}

// 1x1 convolution of the head + activations (efficient_encoder.py:170-197).  A block takes HEAD_CELLS
// feature cells (lane = cell) and PARTS warps, each warp accumulating its slice of the feature channels;
// with PARTS > 1 the partial sums meet in shared memory; then warp w < min(PARTS, M) adds the extra
// channels (pooled gradient, bilinear cond) and applies the activations of the splat slots m with
// m % min(PARTS, M) == w.  PARTS = 1 (each warp 32 cells, all channels; WPB such warps per block share
// one staging of the weights and GroupNorm table) suits many cells; a channel split (PARTS = 4) gives
// small grids enough warps.  Weights sit transposed in shared memory, [Cin][20] (18 outputs padded to
// 20), so one input channel is 5 broadcast 16-byte loads for 18 FMAs.
template <int M, int PARTS, int WPB = 1>
__global__ void __launch_bounds__(32 * PARTS * WPB) k_head(HeadArgs a) {
    static_assert(PARTS == 1 || WPB == 1, "a channel split works on one group of 32 cells");
    // wT [Cin][20], bias [20], gn scale/shift [2][Cfeat], partial sums [PARTS][HEAD_CELLS][20] (PARTS > 1)
    extern __shared__ __align__(16) float shw[];
    float *wT = shw, *sb = shw + a.Cin * HEAD_NP, *gsc = sb + HEAD_NP, *gsh = gsc + a.Cfeat;
    float *red = gsh + a.Cfeat;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int part = PARTS > 1 ? warp : 0;  // channel slice of this warp
    const int cw = PARTS > 1 ? 0 : warp;    // group of 32 cells of this warp inside the block
    const long long cell0 = (long long)blockIdx.x * (HEAD_CELLS * WPB);
    const long long ncell = (long long)a.B * a.fH * a.fW;
    const int b0 = (int)(cell0 / ((long long)a.fH * a.fW));
    // w [nout][Cin] -> wT [Cin][20]: row k, channels strided over the block (coalesced, no divisions),
    // four rows' loads in flight per thread; outputs nout..19 are zero
    for (int k0 = 0; k0 < HEAD_NP; k0 += 4) {
        for (int c = threadIdx.x; c < a.Cin; c += blockDim.x) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = k0 + u < a.nout ? __ldg(a.w + (k0 + u) * a.Cin + c) : 0.f;
            *reinterpret_cast<float4 *>(wT + c * HEAD_NP + k0) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    for (int i = threadIdx.x; i < HEAD_NP; i += blockDim.x) sb[i] = i < a.nout ? a.b[i] : 0.f;
    // GroupNorm scale/shift of the block's image (blocks never straddle images: the caller requires
    // fH*fW to be a multiple of HEAD_CELLS when gn_stats is used, and launch_head takes WPB > 1 only when
    // fH*fW is a multiple of the block's HEAD_CELLS * WPB cells)
    if (a.gn_stats) {
        const double n = (double)a.fH * a.fW * (a.Cfeat / 8);
        for (int c = threadIdx.x; c < a.Cfeat; c += blockDim.x) {
            int g = c / (a.Cfeat / 8);
            double mean = a.gn_stats[(b0 * 8 + g) * 2] / n;
            double var = a.gn_stats[(b0 * 8 + g) * 2 + 1] / n - mean * mean;
            if (var < 0) var = 0;
            float rstd = (float)(1.0 / sqrt(var + 1e-5));
            gsc[c] = a.gn_gamma[c] * rstd;
            gsh[c] = a.gn_beta[c] - (float)mean * a.gn_gamma[c] * rstd;
        }
    }
    __syncthreads();
    const long long cell = cell0 + cw * HEAD_CELLS + lane;
    const bool live = cell < ncell;
    float acc[HEAD_NP];
#pragma unroll
    for (int k = 0; k < HEAD_NP; k++) acc[k] = 0.f;
    auto fma_channel = [&](int c, float v) {
        const float4 *wc = reinterpret_cast<const float4 *>(wT + c * HEAD_NP);
#pragma unroll
        for (int q = 0; q < HEAD_NP / 4; q++) {
            const float4 w4 = wc[q];
            acc[4 * q + 0] = fmaf(w4.x, v, acc[4 * q + 0]);
            acc[4 * q + 1] = fmaf(w4.y, v, acc[4 * q + 1]);
            acc[4 * q + 2] = fmaf(w4.z, v, acc[4 * q + 2]);
            acc[4 * q + 3] = fmaf(w4.w, v, acc[4 * q + 3]);
        }
    };
    const int per = ((a.Cfeat / 8 + PARTS - 1) / PARTS) * 8;
    const int c_lo = part * per, c_hi = min(a.Cfeat, c_lo + per);
    if (live) {
        // the warp's slice, up to 4 vectors of 8 channels at a time, loaded before any arithmetic
        const __nv_bfloat16 *fp = a.feat + cell * a.Cfeat;
        for (int c1 = c_lo; c1 < c_hi; c1 += 32) {
            uint4 u[4];
#pragma unroll
            for (int q = 0; q < 4; q++)
                if (c1 + 8 * q < c_hi) u[q] = __ldg(reinterpret_cast<const uint4 *>(fp + c1 + 8 * q));
#pragma unroll
            for (int q = 0; q < 4; q++) {
                if (c1 + 8 * q >= c_hi) break;
                const int c = c1 + 8 * q;
                const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&u[q]);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float v = __bfloat162float(e[j]);
                    if (a.gn_stats) v = fmaf(v, gsc[c + j], gsh[c + j]);
                    fma_channel(c + j, v);
                }
            }
        }
    }
    constexpr int NFIN = PARTS < M ? PARTS : M;  // warps that finish the cells
    if (PARTS > 1) {
        {
            float4 *rp = reinterpret_cast<float4 *>(red + (warp * HEAD_CELLS + lane) * HEAD_NP);
#pragma unroll
            for (int q = 0; q < HEAD_NP / 4; q++)
                rp[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        }
        __syncthreads();
        if (warp >= NFIN || !live) return;
#pragma unroll
        for (int k = 0; k < HEAD_NP; k++) acc[k] = 0.f;
#pragma unroll
        for (int p = 0; p < PARTS; p++) {  // partials summed in a fixed order
            const float4 *rp = reinterpret_cast<const float4 *>(red + (p * HEAD_CELLS + lane) * HEAD_NP);
#pragma unroll
            for (int q = 0; q < HEAD_NP / 4; q++) {
                const float4 t = rp[q];
                acc[4 * q] += t.x;
                acc[4 * q + 1] += t.y;
                acc[4 * q + 2] += t.z;
                acc[4 * q + 3] += t.w;
            }
        }
    } else if (!live) {
        return;
    }
#pragma unroll
    for (int k = 0; k < HEAD_NP; k++) acc[k] += sb[k];
    const int b = (int)(cell / ((long long)a.fH * a.fW));
    const int r = (int)(cell - (long long)b * a.fH * a.fW);
    const int y = r / a.fW, x = r - y * a.fW;
    head_extra(a, wT + a.Cfeat * HEAD_NP, cell, b, y, x, acc);
    head_activate<M, NFIN>(a, part, b, r, y, x, acc);
}

// ---- the heads on the tensor cores ----
// The head is a [cells x Cfeat] x [Cfeat x 18] contraction: far too narrow (N = 18) for a tcgen05 tile, and
// bound by reading its bf16 features, so it runs on the warp-level mma.sync (m16n8k16, bf16 in, fp32
// accumulate).  The features are exact bf16 operands; GroupNorm folds into the weights of the block's
// image, w'[o][c] = w[o][c] * sc[c] and bias'[o] = b[o] + sum_c w[o][c] * sh[c], and w' enters as three bf16
// terms (hi + mid + lo, together exact to ~2^-24 of |w'|), so the products match fp32 arithmetic.
__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void split3_bf16(float w, __nv_bfloat16 &h, __nv_bfloat16 &m, __nv_bfloat16 &l) {
    h = __float2bfloat16_rn(w);
    float r = w - __bfloat162float(h);  // exact
    m = __float2bfloat16_rn(r);
    r -= __bfloat162float(m);           // exact
    l = __float2bfloat16_rn(r);
}

__device__ __forceinline__ uint32_t pack_bf16(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// Per-image operands of k_head_tc, written by k_head_prep: the B fragments
// frag[b][Cfeat/32 chunks][3 terms][3 n-tiles][32 lanes] (16 bytes: lane (g, t) holds outputs 8j + g at
// channels 32 chunk + 8t .. +8 of one term) and bias'[b][24].
size_t head_frag_bytes(int Cfeat) { return (size_t)(Cfeat / 32) * 9 * 32 * 16; }

// grid = (ceil(Cfeat/32 * 96 / 128), B): one (chunk, n-tile, lane) item per thread; block x = 0 also sums
// bias' (each warp six outputs at once: lane-strided sums, then a fixed xor tree).  The GroupNorm scale/shift are the
// ones k_head applies on the fly (same float/double arithmetic).
__global__ void __launch_bounds__(128) k_head_prep(HeadArgs a, uint4 *__restrict__ frag, float *__restrict__ fbias,
                                                   float *__restrict__ wext) {
    __shared__ double gmean[8];
    __shared__ float grstd[8];
    const int b = blockIdx.y;
    const int nch = a.Cfeat / 32, cpg = a.Cfeat / 8;
    if (threadIdx.x < 8 && a.gn_stats) {
        const double n = (double)a.fH * a.fW * cpg;
        const double mean = a.gn_stats[(b * 8 + threadIdx.x) * 2] / n;
        double var = a.gn_stats[(b * 8 + threadIdx.x) * 2 + 1] / n - mean * mean;
        if (var < 0) var = 0;
        gmean[threadIdx.x] = mean;
        grstd[threadIdx.x] = (float)(1.0 / sqrt(var + 1e-5));
    }
    __syncthreads();
    auto scale = [&](int c) { return a.gn_stats ? a.gn_gamma[c] * grstd[c / cpg] : 1.f; };
    auto shift = [&](int c) {
        return a.gn_stats ? a.gn_beta[c] - (float)gmean[c / cpg] * a.gn_gamma[c] * grstd[c / cpg] : 0.f;
    };
    const int it = blockIdx.x * blockDim.x + threadIdx.x;
    if (it < nch * 96) {
        const int ln = it & 31, j = (it >> 5) % 3, ch = it / 96;
        const int o = 8 * j + (ln >> 2), c0 = ch * 32 + 8 * (ln & 3);
        uint32_t hv[4], mv[4], lv[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            float w0 = 0.f, w1 = 0.f;
            if (o < a.nout) {
                w0 = __ldg(a.w + o * a.Cin + c0 + e) * scale(c0 + e);
                w1 = __ldg(a.w + o * a.Cin + c0 + e + 1) * scale(c0 + e + 1);
            }
            __nv_bfloat16 h0, m0, l0, h1, m1, l1;
            split3_bf16(w0, h0, m0, l0);
            split3_bf16(w1, h1, m1, l1);
            hv[e >> 1] = pack_bf16(h0, h1);
            mv[e >> 1] = pack_bf16(m0, m1);
            lv[e >> 1] = pack_bf16(l0, l1);
        }
        uint4 *fr = frag + (size_t)b * nch * 9 * 32;
        fr[(ch * 9 + 0 + j) * 32 + ln] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        fr[(ch * 9 + 3 + j) * 32 + ln] = make_uint4(mv[0], mv[1], mv[2], mv[3]);
        fr[(ch * 9 + 6 + j) * 32 + ln] = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
    if (blockIdx.x == 0) {
        if (b == 0)  // the extra channels' weights, [Cin - Cfeat][HEAD_NP]
            for (int i = threadIdx.x; i < (a.Cin - a.Cfeat) * HEAD_NP; i += blockDim.x) {
                const int e = i / HEAD_NP, o = i - e * HEAD_NP;
                wext[i] = o < a.nout ? __ldg(a.w + o * a.Cin + a.Cfeat + e) : 0.f;
            }
        // warp w sums outputs w, w + 4, ..., w + 20 at once: lane-strided channel sums (all six outputs'
        // loads of a channel in flight together), then a fixed xor tree per output
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        float sum[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c = lane; c < a.Cfeat; c += 32) {
            const float shc = shift(c);
#pragma unroll
            for (int k = 0; k < 6; k++) {
                const int o = warp + 4 * k;
                if (o < a.nout) sum[k] = fmaf(__ldg(a.w + o * a.Cin + c), shc, sum[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < 6; k++) {
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], m);
            const int o = warp + 4 * k;
            if (lane == 0) fbias[b * 24 + o] = o < a.nout ? a.b[o] + sum[k] : 0.f;
        }
    }
}

// One block = 4 warps over 64 consecutive cells of one image (grid = (fH*fW / 64, B)); each warp takes one
// m-tile of 16 cells.  Lane (g, t) = (lane / 4, lane % 4) loads channels [32 ch + 8t, +8) of its rows g and
// g + 8 with one 16-byte load each and feeds them as the k-slots (2t, 2t+1 | 2t+8, 2t+9) of the chunk's two
// k-steps; k_head_prep laid the B fragments out with the same channel permutation, so the sum over k is the
// sum over channels.  All NCH = Cfeat/32 chunks of the warp's features are loaded up front (2-4 KB per warp
// in flight: the head is bound by reading its features), the B fragments (9 x 512 bytes per chunk, shared by
// every warp of the image) come through L1.
// Epilogue: the accumulators go through shared memory so that lanes l and l + 16 own cell l of the warp:
// both add bias' and the extra channels in fp32 (head_extra), each applies the activations of half of the
// cell's splat slots (head_activate).
template <int M, int NCH>
__global__ void __launch_bounds__(128) k_head_tc(HeadArgs a) {
    __shared__ float stage[4][16][25];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.y;
    const int HW = a.fH * a.fW;
    const int cw = blockIdx.x * 64 + warp * 16;  // the warp's first cell inside image b
    const int g = lane >> 2, t = lane & 3;
    const __nv_bfloat16 *fb = a.feat + ((long long)b * HW + cw + g) * (NCH * 32) + 8 * t;
    uint4 ar[NCH][2];
#pragma unroll
    for (int ch = 0; ch < NCH; ch++)
#pragma unroll
        for (int q = 0; q < 2; q++)
            ar[ch][q] = __ldg(reinterpret_cast<const uint4 *>(fb + q * 8 * (NCH * 32) + ch * 32));
    const uint4 *fr = a.frag + (size_t)b * NCH * 9 * 32 + lane;
    float acc[3][4];
#pragma unroll
    for (int j = 0; j < 3; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[j][e] = 0.f;
#pragma unroll
    for (int ch = 0; ch < NCH; ch++) {
        const uint4 &r0 = ar[ch][0], &r1 = ar[ch][1];  // rows g, g + 8
#pragma unroll
        for (int k = 0; k < 9; k++) {
            const uint4 bv = __ldg(fr + (ch * 9 + k) * 32);
            const int j = k % 3;
            mma_16816_bf16(acc[j], r0.x, r1.x, r0.y, r1.y, bv.x, bv.y);
            mma_16816_bf16(acc[j], r0.z, r1.z, r0.w, r1.w, bv.z, bv.w);
        }
    }
    // epilogue: C fragment (row g | g + 8, outputs 8j + 2t, +1) -> stage[cell][output] -> lane = cell
    float(*sw)[25] = stage[warp];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int o = 8 * j + 2 * t;
        sw[g][o] = acc[j][0];
        sw[g][o + 1] = acc[j][1];
        sw[g + 8][o] = acc[j][2];
        sw[g + 8][o + 1] = acc[j][3];
    }
    __syncwarp();
    // lane = (splat slot half, cell): both half-warps finish the 16 cells, half h the slots m with m % 2 == h
    constexpr int NFIN = M < 2 ? M : 2;
    const int lc = lane & 15, part = lane >> 4;
    if (part >= NFIN) return;
    float v[HEAD_NP];
    const float *fbias = a.fbias + b * 24;
#pragma unroll
    for (int k = 0; k < HEAD_NP; k++) v[k] = sw[lc][k] + __ldg(fbias + k);
    const int r = cw + lc;
    const int y = r / a.fW, x = r - y * a.fW;
    const long long cell = (long long)b * HW + r;
    head_extra(a, a.wext, cell, b, y, x, v);
    head_activate<M, NFIN>(a, part, b, r, y, x, v);
}

// cond[B][rg][rg][4] = (|bilinear(image) - render|, mean_c(render)) (efficient_encoder.py:349-351)
// grid = (ceil(rg^2 / 256), B)
__global__ void k_cond(const float *__restrict__ image, int B, int H, int W, const float *__restrict__ render, int rg,
                       float *__restrict__ cond) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rg * rg) return;
    const int b = blockIdx.y;
    const long long i = (long long)b * rg * rg + r;
    int y = r / rg, x = r - y * rg;
    int y0, y1, x0, x1;
    float h0, h1, w0, w1;
    lin_idx(y, H, rg, y0, y1, h0, h1);
    lin_idx(x, W, rg, x0, x1, w0, w1);
    const long long P = (long long)H * W, R = (long long)rg * rg;
    float msum = 0.f;
    for (int c = 0; c < 3; c++) {
        const float *im = image + ((long long)b * 3 + c) * P;
        float t = h0 * (w0 * im[(long long)y0 * W + x0] + w1 * im[(long long)y0 * W + x1]) +
                  h1 * (w0 * im[(long long)y1 * W + x0] + w1 * im[(long long)y1 * W + x1]);
        float rv = render[((long long)b * 3 + c) * R + r];
        cond[i * 4 + c] = fabsf(t - rv);
        msum += rv;
    }
    cond[i * 4 + 3] = msum / 3.0f;
}

// up[B][H4][W4][Cu] = bilinear(s8 -> H4 x W4) (the upsampled half of the _UpBlock input,
// efficient_encoder.py:89-91; the decoder convolution reads [up, s4] as two inputs, so the
// concatenation is never materialised).  grid = (row blocks, H4, B); one thread per 8-channel vector.
__global__ void __launch_bounds__(256) k_upsample(const __nv_bfloat16 *__restrict__ s8, int H8, int W8, int Cu,
                                                  int H4, int W4, const float2 *__restrict__ gn_table,
                                                  __nv_bfloat16 *__restrict__ up) {
    const int nv = Cu / 8;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= W4 * nv) return;
    const int y = blockIdx.y, b = blockIdx.z;
    const int x = i / nv, c0 = (i - x * nv) * 8;
    int y0, y1, x0, x1;
    float h0, h1, w0, w1;
    lin_idx(y, H8, H4, y0, y1, h0, h1);
    lin_idx(x, W8, W4, x0, x1, w0, w1);
    const __nv_bfloat16 *sb = s8 + (long long)b * H8 * W8 * Cu + c0;
    const uint4 a00 = *reinterpret_cast<const uint4 *>(sb + (y0 * W8 + x0) * Cu);
    const uint4 a01 = *reinterpret_cast<const uint4 *>(sb + (y0 * W8 + x1) * Cu);
    const uint4 a10 = *reinterpret_cast<const uint4 *>(sb + (y1 * W8 + x0) * Cu);
    const uint4 a11 = *reinterpret_cast<const uint4 *>(sb + (y1 * W8 + x1) * Cu);
    const __nv_bfloat16 *p00 = reinterpret_cast<const __nv_bfloat16 *>(&a00);
    const __nv_bfloat16 *p01 = reinterpret_cast<const __nv_bfloat16 *>(&a01);
    const __nv_bfloat16 *p10 = reinterpret_cast<const __nv_bfloat16 *>(&a10);
    const __nv_bfloat16 *p11 = reinterpret_cast<const __nv_bfloat16 *>(&a11);
    // s8 may be the raw convolution output: GroupNorm is a per-channel affine map, so it is applied after
    // the interpolation (the bilinear weights sum to one)
    float sc[8], sh[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        sc[k] = 1.f;
        sh[k] = 0.f;
    }
    if (gn_table) {
        const float4 *t = reinterpret_cast<const float4 *>(gn_table + (long long)b * Cu + c0);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float4 v = t[k];
            sc[2 * k] = v.x;
            sh[2 * k] = v.y;
            sc[2 * k + 1] = v.z;
            sh[2 * k + 1] = v.w;
        }
    }
    uint4 res;
    __nv_bfloat16 *e = reinterpret_cast<__nv_bfloat16 *>(&res);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float f = h0 * (w0 * __bfloat162float(p00[k]) + w1 * __bfloat162float(p01[k])) +
                  h1 * (w0 * __bfloat162float(p10[k]) + w1 * __bfloat162float(p11[k]));
        e[k] = __float2bfloat16_rn(fmaf(f, sc[k], sh[k]));
    }
    *reinterpret_cast<uint4 *>(up + (((long long)b * H4 + y) * W4 + x) * Cu + c0) = res;
}

// k_upsample for an exact 2x upsample (H4 = 2 H8, W4 = 2 W8), one thread per 2x2 output block of one
// 8-channel vector: output rows 2p and 2p+1 read source rows p-1, p, p+1 (clamped) and likewise the
// columns, so 9 vector loads serve 4 outputs and the horizontal blends of the middle source row serve both
// output rows.  Even outputs take source slots (0, 1), odd ones (1, 2); at a border the clamped slot holds
// the same row or column as its neighbour and the weight from lin_idx is 1/0 there, so every output is
// the same torch bilinear (align_corners=False) value as k_upsample's.
__global__ void __launch_bounds__(256) k_upsample2x(const __nv_bfloat16 *__restrict__ s8, int H8, int W8, int Cu,
                                                    const float2 *__restrict__ gn_table,
                                                    __nv_bfloat16 *__restrict__ up) {
    const int nv = Cu / 8;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= W8 * nv) return;
    const int p = blockIdx.y, b = blockIdx.z;
    const int q = i / nv, c0 = (i - q * nv) * 8;
    const int H4 = 2 * H8, W4 = 2 * W8;
    // weights of output rows 2p, 2p+1 and columns 2q, 2q+1 (slots as above)
    float hy[2][2], wx[2][2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        int i0, i1;
        lin_idx(2 * p + t, H8, H4, i0, i1, hy[t][0], hy[t][1]);
        lin_idx(2 * q + t, W8, W4, i0, i1, wx[t][0], wx[t][1]);
    }
    const __nv_bfloat16 *sb = s8 + (long long)b * H8 * W8 * Cu + c0;
    uint4 v[3][3];
#pragma unroll
    for (int r = 0; r < 3; r++) {
        const int yy = min(max(p - 1 + r, 0), H8 - 1);
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const int xx = min(max(q - 1 + c, 0), W8 - 1);
            v[r][c] = __ldg(reinterpret_cast<const uint4 *>(sb + ((long long)yy * W8 + xx) * Cu));
        }
    }
    float sc[8], sh[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        sc[k] = 1.f;
        sh[k] = 0.f;
    }
    if (gn_table) {
        const float4 *t = reinterpret_cast<const float4 *>(gn_table + (long long)b * Cu + c0);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float4 g = t[k];
            sc[2 * k] = g.x;
            sh[2 * k] = g.y;
            sc[2 * k + 1] = g.z;
            sh[2 * k + 1] = g.w;
        }
    }
    // channel pairs: one bf16x2 -> float2 unpack per source word, one packed rounding per output pair
    uint32_t res[2][2][4];
#pragma unroll
    for (int k2 = 0; k2 < 4; k2++) {
        float2 f[3][3];
#pragma unroll
        for (int r = 0; r < 3; r++)
#pragma unroll
            for (int c = 0; c < 3; c++) f[r][c] = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162 *>(&v[r][c])[k2]);
        // horizontal blends of the three source rows at the two output columns
        float2 hb[3][2];
#pragma unroll
        for (int r = 0; r < 3; r++)
#pragma unroll
            for (int t = 0; t < 2; t++) {
                hb[r][t].x = wx[t][0] * f[r][t].x + wx[t][1] * f[r][t + 1].x;
                hb[r][t].y = wx[t][0] * f[r][t].y + wx[t][1] * f[r][t + 1].y;
            }
#pragma unroll
        for (int ty = 0; ty < 2; ty++)
#pragma unroll
            for (int tx = 0; tx < 2; tx++) {
                const float ox = hy[ty][0] * hb[ty][tx].x + hy[ty][1] * hb[ty + 1][tx].x;
                const float oy = hy[ty][0] * hb[ty][tx].y + hy[ty][1] * hb[ty + 1][tx].y;
                const __nv_bfloat162 pk =
                    __floats2bfloat162_rn(fmaf(ox, sc[2 * k2], sh[2 * k2]), fmaf(oy, sc[2 * k2 + 1], sh[2 * k2 + 1]));
                res[ty][tx][k2] = *reinterpret_cast<const uint32_t *>(&pk);
            }
    }
#pragma unroll
    for (int ty = 0; ty < 2; ty++)
#pragma unroll
        for (int tx = 0; tx < 2; tx++)
            *reinterpret_cast<uint4 *>(up + (((long long)b * H4 + 2 * p + ty) * W4 + 2 * q + tx) * Cu + c0) =
                make_uint4(res[ty][tx][0], res[ty][tx][1], res[ty][tx][2], res[ty][tx][3]);
}

// per-channel GroupNorm(8) scale and shift, table[b][c] = (sc, sh) with normalised = raw * sc + sh
__global__ void __launch_bounds__(256) k_gn_table(const double *__restrict__ stats, const float *__restrict__ gamma,
                                                  const float *__restrict__ beta, int C, long long HW,
                                                  float2 *__restrict__ table) {
    const int b = blockIdx.x;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float sc, sh;
        gn_affine(stats, gamma, beta, b, c, C, HW, sc, sh);
        table[b * C + c] = make_float2(sc, sh);
    }
}

// GroupNorm(8) applied to NHWC bf16 [B][HW][C] written as NHWC fp32, 8 channels per thread, from a
// scale/shift table (the fine decoder's normalised features for return_latents; the backbone features
// when s8 stays raw)
// grid = (ceil(HW * C / 8 / 256), B): 32-bit index arithmetic inside one image
__global__ void __launch_bounds__(256) k_gn_to_f32(const __nv_bfloat16 *__restrict__ x, int B, long long HW, int C,
                                                   const float2 *__restrict__ table, float *__restrict__ out) {
    const int nv = C / 8;
    const int nvi = (int)HW * nv;  // vectors of 8 channels per image
    const int iv = blockIdx.x * blockDim.x + threadIdx.x;
    if (iv >= nvi) return;
    const int b = blockIdx.y;
    const int c0 = (iv % nv) * 8;
    const long long i = (long long)b * nvi + iv;
    const float4 *t = reinterpret_cast<const float4 *>(table + (long long)b * C + c0);
    const float4 t0 = t[0], t1 = t[1], t2 = t[2], t3 = t[3];
    const uint4 u = reinterpret_cast<const uint4 *>(x)[i];
    const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&u);
    float4 *o = reinterpret_cast<float4 *>(out) + 2 * i;
    o[0] = make_float4(fmaf(__bfloat162float(e[0]), t0.x, t0.y), fmaf(__bfloat162float(e[1]), t0.z, t0.w),
                       fmaf(__bfloat162float(e[2]), t1.x, t1.y), fmaf(__bfloat162float(e[3]), t1.z, t1.w));
    o[1] = make_float4(fmaf(__bfloat162float(e[4]), t2.x, t2.y), fmaf(__bfloat162float(e[5]), t2.z, t2.w),
                       fmaf(__bfloat162float(e[6]), t3.x, t3.y), fmaf(__bfloat162float(e[7]), t3.z, t3.w));
}

// NHWC bf16 -> NHWC fp32 (backbone_features output), 8 elements per thread (n a multiple of 8)
__global__ void k_bf16_to_f32(const __nv_bfloat16 *__restrict__ in, float *__restrict__ out, long long n) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i * 8 >= n) return;
    uint4 u = reinterpret_cast<const uint4 *>(in)[i];
    const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&u);
    float4 *o = reinterpret_cast<float4 *>(out) + 2 * i;
    o[0] = make_float4(__bfloat162float(e[0]), __bfloat162float(e[1]), __bfloat162float(e[2]), __bfloat162float(e[3]));
    o[1] = make_float4(__bfloat162float(e[4]), __bfloat162float(e[5]), __bfloat162float(e[6]), __bfloat162float(e[7]));
}

// channel split for the head: 4 warps per 32 cells for grids under ~16k cells, else one warp
int head_parts(long long ncell) { return ncell < 16384 ? 4 : 1; }

size_t head_smem(const HeadArgs &h, long long ncell) {
    const int parts = head_parts(ncell);
    return ((size_t)h.Cin * HEAD_NP + HEAD_NP + 2 * h.Cfeat + (parts > 1 ? parts * HEAD_CELLS * HEAD_NP : 0)) * 4;
}

template <int M, int NCH>
void launch_head_tc(const HeadArgs &h, cudaStream_t s) {
    dim3 grid((unsigned)(h.fH * h.fW / 64), (unsigned)h.B);
    k_head_tc<M, NCH><<<grid, 128, 0, s>>>(h);
}

// k_head_tc takes heads whose image block is a multiple of 64 cells with 128 or 256 feature channels, up
// to 5 extra channels and at most 2 splats per cell
bool head_tc_ok(const HeadArgs &h) {
    return ((long long)h.fH * h.fW) % 64 == 0 && (h.Cfeat == 128 || h.Cfeat == 256) && h.Cin > h.Cfeat &&
           h.Cin - h.Cfeat <= 5 && h.nout <= HEAD_NP && (h.M == 1 || h.M == 2);
}

// workspace of the tensor-core head's per-image operands
size_t head_tc_ws(int B, int Cfeat) { return (size_t)B * head_frag_bytes(Cfeat) + (size_t)B * 24 * 4 + 5 * HEAD_NP * 4; }

// k_head_prep for head h into ws (head_tc_ws bytes, 16-byte aligned); sets h's operand pointers.  Returns the
// number of launches (0 when the head takes the SIMT kernel).
int launch_head_prep(HeadArgs &h, void *ws, cudaStream_t s) {
    if (!head_tc_ok(h)) return 0;
    uint4 *frag = reinterpret_cast<uint4 *>(ws);
    float *fbias = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + (size_t)h.B * head_frag_bytes(h.Cfeat));
    float *wext = fbias + h.B * 24;
    dim3 grid((unsigned)((h.Cfeat / 32 * 96 + 127) / 128), (unsigned)h.B);
    k_head_prep<<<grid, 128, 0, s>>>(h, frag, fbias, wext);
    h.frag = frag;
    h.fbias = fbias;
    h.wext = wext;
    return 1;
}

void launch_head(const HeadArgs &h, long long ncell, cudaStream_t s) {
    if (h.frag) {
        if (h.Cfeat == 128) h.M == 1 ? launch_head_tc<1, 4>(h, s) : launch_head_tc<2, 4>(h, s);
        else h.M == 1 ? launch_head_tc<1, 8>(h, s) : launch_head_tc<2, 8>(h, s);
        return;
    }
    const size_t smem = head_smem(h, ncell);
    if (head_parts(ncell) == 4) {
        const unsigned grid = (unsigned)((ncell + HEAD_CELLS - 1) / HEAD_CELLS);
        if (h.M == 1) k_head<1, 4><<<grid, 128, smem, s>>>(h);
        else k_head<2, 4><<<grid, 128, smem, s>>>(h);
    } else if (((long long)h.fH * h.fW) % (HEAD_CELLS * 8) == 0) {
        // 8 warps of 32 cells per block: one weight staging for 256 cells
        const unsigned grid = (unsigned)((ncell + HEAD_CELLS * 8 - 1) / (HEAD_CELLS * 8));
        if (h.M == 1) k_head<1, 1, 8><<<grid, 256, smem, s>>>(h);
        else k_head<2, 1, 8><<<grid, 256, smem, s>>>(h);
    } else {
        const unsigned grid = (unsigned)((ncell + HEAD_CELLS - 1) / HEAD_CELLS);
        if (h.M == 1) k_head<1, 1><<<grid, 32, smem, s>>>(h);
        else k_head<2, 1><<<grid, 32, smem, s>>>(h);
    }
}

size_t al(size_t x) { return (x + 255) & ~(size_t)255; }

struct EncPlan {
    int B, H, W, H2, W2, H4, W4, H8, W8, d, Nc, Nf, N, rg;
    size_t o_Z, o_y1, o_y2, o_y3, o_cat, o_y4, o_grad, o_g4, o_g8, o_stats, o_chsum, o_gtab, o_err, o_ht3, o_ht4,
        o_c[5], o_render, o_cond, o_rws, total;
    gs_render_desc rd;
    size_t rws;
};

int enc_plan(const gs_encoder_desc *e, EncPlan &p) {
    if (!e || e->B < 1 || e->H < 16 || e->W < 16 || e->H % 8 || e->W % 8) return GS_ERR_BAD_ARGUMENT;
    if (e->d != 256 || e->M < 1 || e->M > 2 || e->Mf < 1 || e->Mf > 2) return GS_ERR_BAD_ARGUMENT;
    if (e->residual_grid < 8) return GS_ERR_BAD_ARGUMENT;
    // the fine head's thread blocks (64 cells) must not straddle two images
    if (((long long)(e->H / 4) * (e->W / 4)) % 64 != 0) return GS_ERR_BAD_ARGUMENT;
    memset(&p, 0, sizeof(p));
    p.B = e->B; p.H = e->H; p.W = e->W; p.d = e->d; p.rg = e->residual_grid;
    p.H2 = p.H / 2; p.W2 = p.W / 2; p.H4 = p.H / 4; p.W4 = p.W / 4; p.H8 = p.H / 8; p.W8 = p.W / 8;
    p.Nc = p.H8 * p.W8 * e->M;
    p.Nf = p.H4 * p.W4 * e->Mf;
    p.N = p.Nc + p.Nf;
    const size_t B = p.B;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o = al(o + bytes); return r; };
    p.o_Z = take(B * p.H2 * p.W2 * 16 * 2);
    p.o_y1 = take(B * p.H2 * p.W2 * 64 * 2);
    p.o_y2 = take(B * p.H4 * p.W4 * 128 * 2);
    p.o_y3 = take(B * p.H8 * p.W8 * 256 * 2);
    p.o_cat = take(B * p.H4 * p.W4 * 256 * 2);  // bilinear(s8) at the s4 size, the decoder's first input
    p.o_y4 = take(B * p.H4 * p.W4 * 128 * 2);
    p.o_grad = take(B * p.H * p.W * 4);
    p.o_g4 = take(B * p.H4 * p.W4 * 4);
    p.o_g8 = take(B * p.H8 * p.W8 * 4);
    p.o_stats = take(4 * B * 16 * sizeof(double));
    p.o_chsum = take(B * GN_BG_BLOCKS * 256 * 4);  // per-block channel sums of the normalised s8
    p.o_gtab = take(B * (256 + 128) * 8);            // GroupNorm scale/shift tables: s8, decoder output
    p.o_err = take(64);
    p.o_ht3 = take(head_tc_ws(p.B, 256));  // tensor-core head operands: coarse head, fine head
    p.o_ht4 = take(head_tc_ws(p.B, 128));
    const size_t nc = B * p.Nc;
    p.o_c[0] = take(nc * 2 * 4);
    p.o_c[1] = take(nc * 2 * 4);
    p.o_c[2] = take(nc * 3 * 4);
    p.o_c[3] = take(nc * 4);
    p.o_c[4] = take(nc * 4);
    p.o_render = take(B * 3 * p.rg * p.rg * 4);
    p.o_cond = take(B * p.rg * p.rg * 4 * 4);
    gs_render_desc &rd = p.rd;
    memset(&rd, 0, sizeof(rd));
    rd.mode = GS_MODE_OCTAVE; rd.B = p.B; rd.N = p.Nc; rd.C = 3; rd.H = p.rg; rd.W = p.rg; rd.tile = 8;
    rd.odds = e->odds; rd.has_theta = e->use_rotation; rd.max_octaves = 6; rd.cutoff = 3.0f; rd.base_texels = 8.0f;
    rd.max_pairs = -1; rd.pair_capacity = 0;
    p.rws = gs_render_workspace_size(&rd, 0);
    if (p.rws == 0) return GS_ERR_BAD_ARGUMENT;
    p.o_rws = take(p.rws);
    p.total = o;
    return GS_OK;
}

template <typename T>
T *W(void *ws, size_t off) { return reinterpret_cast<T *>(reinterpret_cast<char *>(ws) + off); }

// A second stream per (host thread, device) for the fine decoder, which needs only the backbone: it runs
// while the internal coarse render -- a latency-bound chain that keeps a fraction of the SMs busy --
// proceeds on the caller's stream.  Fork and join are event edges, so a CUDA graph capture of the
// caller's stream records the two branches as parallel graph nodes.  Per thread, so concurrent callers
// never re-record each other's events.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

// *out stays NULL (the caller runs both branches on its own stream) when the side stream does not exist
// yet and `main` is being captured: the stream and events are only ever created outside a capture.
int side_stream(cudaStream_t main, SideStream **out) {
    static thread_local std::vector<SideStream> per_dev;  // index: device ordinal (never destroyed)
    *out = nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GS_ERR_CUDA;
    if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1);
    SideStream &ss = per_dev[dev];
    if (!ss.s) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(main, &cs) != cudaSuccess) return GS_ERR_CUDA;
        if (cs != cudaStreamCaptureStatusNone) return GS_OK;
        if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess) return GS_ERR_CUDA;
        if (cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess) return GS_ERR_CUDA;
        if (cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) return GS_ERR_CUDA;
    }
    *out = &ss;
    return GS_OK;
}

// Forks `side` from `main` on construction; joins it back (once) on join() or on scope exit, so an early
// error return never leaves a capture with an unjoined branch.
struct Fork {
    SideStream *ss;
    cudaStream_t main;
    bool joined = false;
    Fork(SideStream *x, cudaStream_t m) : ss(x), main(m) {
        if (!ss) return;
        cudaEventRecord(ss->fork, main);
        cudaStreamWaitEvent(ss->s, ss->fork, 0);
    }
    cudaStream_t side() const { return ss ? ss->s : main; }
    void join() {
        if (joined || !ss) return;
        cudaEventRecord(ss->join, ss->s);
        cudaStreamWaitEvent(main, ss->join, 0);
        joined = true;
    }
    ~Fork() { join(); }
};

}  // namespace

extern "C" size_t gs_encoder_workspace_size(const gs_encoder_desc *e) {
    EncPlan p;
    if (enc_plan(e, p) != GS_OK) return 0;
    return p.total;
}

extern "C" int gs_encoder_fwd(const gs_encoder_desc *e, const gs_encoder_weights *w, const float *image, float *mu,
                              float *log_scale, float *color, float *opacity, float *theta, float *bg,
                              float *features, float *latents, void *workspace, size_t workspace_bytes,
                              void *stream) {
    EncPlan p;
    int st = enc_plan(e, p);
    if (st != GS_OK) return st;
    if (!w || !image || !mu || !log_scale || !color || !opacity || !bg || (e->use_rotation && !theta))
        return GS_ERR_BAD_ARGUMENT;
    if (!workspace || workspace_bytes < p.total) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    void *ws = workspace;
    const int B = p.B;
    cudaMemsetAsync(W<char>(ws, p.o_stats), 0, p.o_err + 64 - p.o_stats, s);  // stats, chsum, err
    double *stats = W<double>(ws, p.o_stats);
    int *err = W<int>(ws, p.o_err);
    float *grad = W<float>(ws, p.o_grad);
    // 1. input preparation
    {
        ProfScope ps(PR_ENC_PREP, s);
        dim3 pg((unsigned)((p.W2 + PREP_TX - 1) / PREP_TX), (unsigned)((p.H2 + PREP_TY - 1) / PREP_TY), (unsigned)B);
        k_prep<<<pg, PREP_TX * PREP_TY, 0, s>>>(image, B, p.H, p.W, grad, W<__nv_bfloat16>(ws, p.o_Z));
        long long n8 = (long long)B * p.H8 * p.W8 * 8;
        k_pool48<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(grad, B, p.H, p.W, W<float>(ws, p.o_g4),
                                                             W<float>(ws, p.o_g8));
    }
    // 2. backbone: conv -> GELU -> GroupNorm, three stages
    auto gn = [&](void *x, long long HW, int C, const double *stt, const float *gamma, const float *beta, float *chsum,
                  int apply) {
        // with channel sums every block ends in C global atomics: keep the grid small for that launch
        // with channel sums the grid is fixed (GN_BG_BLOCKS per image): k_bg reduces exactly that many partials
        dim3 grid((unsigned)(chsum ? GN_BG_BLOCKS : std::min<long long>(1024, (HW * C / 8 + 255) / 256)), (unsigned)B);
        k_gn_apply<<<grid, 256, 0, s>>>((__nv_bfloat16 *)x, (int)HW, C, stt, gamma, beta, chsum, apply);
    };
    gs_conv_desc cd;
    memset(&cd, 0, sizeof(cd));
    cd.B = B; cd.H = p.H2; cd.W = p.W2; cd.Cin = 16; cd.Cout = 64; cd.kh = 4; cd.kw = 4; cd.stride = 1; cd.pad = 2;
    cd.Ho = p.H2; cd.Wo = p.W2; cd.gelu = 1; cd.kind = 1;
    {
        ProfScope ps(PR_CONV1, s);
        if ((st = gs_conv_run(&cd, W<void>(ws, p.o_Z), w->w1, w->b1, W<void>(ws, p.o_y1), stats, err, s))) return st;
    }
    gn(W<void>(ws, p.o_y1), (long long)p.H2 * p.W2, 64, stats, w->gn1_w, w->gn1_b, nullptr, 1);
    memset(&cd, 0, sizeof(cd));
    cd.B = B; cd.H = p.H2; cd.W = p.W2; cd.Cin = 64; cd.Cout = 128; cd.kh = 3; cd.kw = 3; cd.stride = 2; cd.pad = 1;
    cd.gelu = 1;
    {
        ProfScope ps(PR_CONV2, s);
        if ((st = gs_conv_run(&cd, W<void>(ws, p.o_y1), w->w2, w->b2, W<void>(ws, p.o_y2), stats + B * 16, err, s)))
            return st;
    }
    gn(W<void>(ws, p.o_y2), (long long)p.H4 * p.W4, 128, stats + B * 16, w->gn2_w, w->gn2_b, nullptr, 1);
    memset(&cd, 0, sizeof(cd));
    cd.B = B; cd.H = p.H4; cd.W = p.W4; cd.Cin = 128; cd.Cout = 256; cd.kh = 3; cd.kw = 3; cd.stride = 2; cd.pad = 1;
    cd.gelu = 1;
    {
        ProfScope ps(PR_CONV3, s);
        if ((st = gs_conv_run(&cd, W<void>(ws, p.o_y2), w->w3, w->b3, W<void>(ws, p.o_y3), stats + 2 * B * 16, err,
                              s)))
            return st;
    }
    float *chsum = W<float>(ws, p.o_chsum);
    // GroupNorm of s8: applied on the fly by its consumers (upsample, coarse head, features, background
    // head) when the coarse head's 32-cell blocks cannot straddle images; else in place as for s2, s4
    const double *gn3 = stats + 2 * B * 16;
    const bool gn3_fly = ((long long)p.H8 * p.W8) % HEAD_CELLS == 0;
    gn(W<void>(ws, p.o_y3), (long long)p.H8 * p.W8, 256, gn3, w->gn3_w, w->gn3_b, chsum, gn3_fly ? 0 : 1);
    float2 *gtab = W<float2>(ws, p.o_gtab);
    k_bg<<<B, 1024, 0, s>>>(chsum, GN_BG_BLOCKS, 256, (long long)p.H8 * p.W8, w->bg_w, w->bg_b,
                           gn3_fly ? gn3 : nullptr, w->gn3_w, w->gn3_b, gtab, bg);
    // fork: the fine decoder (5.) on the side stream, the coarse head and render (3., 4.) on the caller's.
    // With stage profiling on, both run on the caller's stream so each stage's events time its own kernels.
    SideStream *side = nullptr;
    if (!gs_prof_on() && (st = side_stream(s, &side))) return st;
    Fork fork(side, s);
    const cudaStream_t s2 = fork.side();
    // 5. fine decoder: bilinear(s8) || s4 -> 3x3 conv 384->128 (+GELU, GN stats)
    {
        ProfScope ps(PR_ENC_MISC, s2);
        if (p.H4 == 2 * p.H8 && p.W4 == 2 * p.W8) {
            dim3 ug((unsigned)((p.W8 * (256 / 8) + 255) / 256), (unsigned)p.H8, (unsigned)B);
            k_upsample2x<<<ug, 256, 0, s2>>>(W<__nv_bfloat16>(ws, p.o_y3), p.H8, p.W8, 256, gn3_fly ? gtab : nullptr,
                                             W<__nv_bfloat16>(ws, p.o_cat));
        } else {
            dim3 ug((unsigned)((p.W4 * (256 / 8) + 255) / 256), (unsigned)p.H4, (unsigned)B);
            k_upsample<<<ug, 256, 0, s2>>>(W<__nv_bfloat16>(ws, p.o_y3), p.H8, p.W8, 256, p.H4, p.W4,
                                           gn3_fly ? gtab : nullptr, W<__nv_bfloat16>(ws, p.o_cat));
        }
    }
    memset(&cd, 0, sizeof(cd));
    cd.B = B; cd.H = p.H4; cd.W = p.W4; cd.Cin = 384; cd.Cout = 128; cd.kh = 3; cd.kw = 3; cd.stride = 1; cd.pad = 1;
    cd.gelu = 1;
    {
        ProfScope ps(PR_CONV4, s2);
        if ((st = gs_conv_run2(&cd, W<void>(ws, p.o_cat), 256, W<void>(ws, p.o_y2), w->w4, w->b4,
                               W<void>(ws, p.o_y4), stats + 3 * B * 16, err, s2)))
            return st;
    }
    // the fine head's arguments; its tensor-core operands (GroupNorm folded into the weights) are prepared
    // on the side stream as soon as the decoder's statistics exist
    HeadArgs hf;
    memset(&hf, 0, sizeof(hf));
    hf.B = B; hf.fH = p.H4; hf.fW = p.W4; hf.M = e->Mf; hf.Cfeat = 128; hf.feat = W<__nv_bfloat16>(ws, p.o_y4);
    hf.gn_stats = stats + 3 * B * 16; hf.gn_gamma = w->gn4_w; hf.gn_beta = w->gn4_b;
    hf.gpool = W<float>(ws, p.o_g4); hf.cond = W<float>(ws, p.o_cond); hf.rg = p.rg;
    hf.w = w->hf_w; hf.b = w->hf_b; hf.Cin = 133; hf.nout = (e->use_rotation ? 9 : 8) * e->Mf;
    hf.off_scale = e->fine_offset / (float)std::max(p.H4, p.W4);
    hf.ls_floor = -INFINITY; hf.min_op = 0.f; hf.use_rot = e->use_rotation;
    hf.Ntot = p.N; hf.n0 = p.Nc; hf.mu = mu; hf.ls = log_scale; hf.col = color; hf.op = opacity; hf.th = theta;
    int nprep = launch_head_prep(hf, W<void>(ws, p.o_ht4), s2);
    // 3. coarse head (writes the API tensors and a contiguous copy for the coarse render)
    HeadArgs h;
    memset(&h, 0, sizeof(h));
    h.B = B; h.fH = p.H8; h.fW = p.W8; h.M = e->M; h.Cfeat = 256; h.feat = W<__nv_bfloat16>(ws, p.o_y3);
    if (gn3_fly) {
        h.gn_stats = gn3; h.gn_gamma = w->gn3_w; h.gn_beta = w->gn3_b;
    }
    h.gpool = W<float>(ws, p.o_g8); h.w = w->hc_w; h.b = w->hc_b; h.Cin = 257; h.nout = (e->use_rotation ? 9 : 8) * e->M;
    h.off_scale = e->coarse_offset / (float)std::max(p.H8, p.W8);
    h.ls_floor = e->coarse_ls_floor; h.min_op = e->coarse_min_opacity; h.use_rot = e->use_rotation;
    h.Ntot = p.N; h.n0 = 0; h.mu = mu; h.ls = log_scale; h.col = color; h.op = opacity; h.th = theta;
    h.cmu = W<float>(ws, p.o_c[0]); h.cls = W<float>(ws, p.o_c[1]); h.ccol = W<float>(ws, p.o_c[2]);
    h.cop = W<float>(ws, p.o_c[3]); h.cth = e->use_rotation ? W<float>(ws, p.o_c[4]) : nullptr;
    {
        ProfScope ps(PR_HEADS, s);
        long long ncell = (long long)B * p.H8 * p.W8;
        nprep += launch_head_prep(h, W<void>(ws, p.o_ht3), s);
        launch_head(h, ncell, s);
    }
    // 4. coarse render at residual_grid^2 (odds) -> cond map
    {
        ProfScope ps(PR_ENC_RENDER, s);
        float *bgws = bg;
        gs_prof_set_internal(1);
        st = gs_render_fwd(&p.rd, h.cmu, h.cls, h.ccol, h.cop, bgws, h.cth, W<float>(ws, p.o_render),
                           W<void>(ws, p.o_rws), p.rws, stream);
        gs_prof_set_internal(0);
        if (st != GS_OK) return st;
        k_cond<<<dim3((unsigned)((p.rg * p.rg + 255) / 256), (unsigned)B), 256, 0, s>>>(
            image, B, p.H, p.W, W<float>(ws, p.o_render), p.rg, W<float>(ws, p.o_cond));
    }
    // join: the fine head needs the decoder's output and statistics and the coarse render's cond map
    fork.join();
    // 6. fine head: GN on the fly (or folded into its tensor-core operands), + pooled gradient + bilinear(cond)
    {
        ProfScope ps(PR_HEADS, s);
        long long ncell = (long long)B * p.H4 * p.W4;
        launch_head(hf, ncell, s);
    }
    if (latents) {
        float2 *gtab4 = W<float2>(ws, p.o_gtab) + B * 256;
        k_gn_table<<<B, 128, 0, s>>>(stats + 3 * B * 16, w->gn4_w, w->gn4_b, 128, (long long)p.H4 * p.W4, gtab4);
        dim3 tg((unsigned)(((long long)p.H4 * p.W4 * 16 + 255) / 256), (unsigned)B);
        k_gn_to_f32<<<tg, 256, 0, s>>>(W<__nv_bfloat16>(ws, p.o_y4), B, (long long)p.H4 * p.W4, 128, gtab4, latents);
        gs_count_launch(2);
    }
    if (features) {
        long long n = (long long)B * p.H8 * p.W8 * 256;
        if (gn3_fly)
            k_gn_to_f32<<<dim3((unsigned)(((long long)p.H8 * p.W8 * 32 + 255) / 256), (unsigned)B), 256, 0, s>>>(
                W<__nv_bfloat16>(ws, p.o_y3), B, (long long)p.H8 * p.W8, 256, gtab, features);
        else
            k_bf16_to_f32<<<(unsigned)((n / 8 + 255) / 256), 256, 0, s>>>(W<__nv_bfloat16>(ws, p.o_y3), features, n);
    }
    // memset, prep, pool, 4 convs, 3 GN applies, bg, 2 heads, cond, upsample, optional feature copy
    gs_count_launch(16 + (features ? 1 : 0) + nprep);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
        fprintf(stderr, "gs_encoder_fwd: %s\n", cudaGetErrorString(ce));
        return GS_ERR_CUDA;
    }
    return GS_OK;
}

// The final render of gs_encode_render_fwd: render_alpha_octave's defaults at the image size.
static int final_render_desc(const gs_encoder_desc *e, const EncPlan &p, gs_render_desc &fd) {
    memset(&fd, 0, sizeof(fd));
    fd.mode = GS_MODE_OCTAVE; fd.B = p.B; fd.N = p.N; fd.C = 3; fd.H = p.H; fd.W = p.W; fd.tile = 8;
    fd.odds = e->odds; fd.has_theta = e->use_rotation; fd.max_octaves = 6; fd.cutoff = 3.0f; fd.base_texels = 8.0f;
    fd.n_coarse = -1; fd.coarse_factor = 8; fd.max_pairs = 48000000;
    const int64_t bound = gs_render_pair_bound(&fd);
    if (bound < 0) return GS_ERR_BAD_ARGUMENT;
    // the reference checks the budget per image and octave; the host bound is per image here
    if (bound / p.B > fd.max_pairs) return GS_ERR_PAIR_BUDGET;
    fd.pair_capacity = std::max<int64_t>(bound, 1);
    return GS_OK;
}

extern "C" size_t gs_encode_render_workspace_size(const gs_encoder_desc *e) {
    EncPlan p;
    if (enc_plan(e, p) != GS_OK) return 0;
    gs_render_desc fd;
    if (final_render_desc(e, p, fd) != GS_OK) return 0;
    const size_t r = gs_render_workspace_size(&fd, 0);
    return r ? al(p.total) + r : 0;
}

extern "C" int gs_encode_render_fwd(const gs_encoder_desc *e, const gs_encoder_weights *w, const float *image,
                                    float *mu, float *log_scale, float *color, float *opacity, float *theta,
                                    float *bg, float *features, float *latents, float *out, void *workspace,
                                    size_t workspace_bytes, void *stream) {
    EncPlan p;
    int st = enc_plan(e, p);
    if (st != GS_OK) return st;
    gs_render_desc fd;
    if ((st = final_render_desc(e, p, fd)) != GS_OK) return st;
    if (!out) return GS_ERR_BAD_ARGUMENT;
    const size_t rws = gs_render_workspace_size(&fd, 0);
    if (!workspace || workspace_bytes < al(p.total) + rws) return GS_ERR_WORKSPACE;
    st = gs_encoder_fwd(e, w, image, mu, log_scale, color, opacity, theta, bg, features, latents, workspace, p.total,
                        stream);
    if (st != GS_OK) return st;
    // the coarse splats' octave fields of the encoder's internal render carry over when the texel grids agree
    GsPrior prior;
    const int mapped = gs_render_prior_map(&p.rd, W<void>(workspace, p.o_rws), &fd, p.Nc, &prior);
    return gs_render_fwd_prior(&fd, mu, log_scale, color, opacity, bg, theta, out, mapped ? &prior : nullptr,
                               W<void>(workspace, al(p.total)), rws, stream);
}

extern "C" int gs_encode_render_debug_pairs(const gs_encoder_desc *e, const void *workspace, int64_t *pairs) {
    EncPlan p;
    int st = enc_plan(e, p);
    if (st != GS_OK) return st;
    gs_render_desc fd;
    if ((st = final_render_desc(e, p, fd)) != GS_OK) return st;
    if (!workspace || !pairs) return GS_ERR_BAD_ARGUMENT;
    int64_t a = 0, b = 0;
    st = gs_render_debug_bins(&p.rd, W<void>(const_cast<void *>(workspace), p.o_rws), &a, nullptr, nullptr, nullptr,
                              nullptr, nullptr);
    if (st != GS_OK) return st;
    st = gs_render_debug_bins(&fd, W<void>(const_cast<void *>(workspace), al(p.total)), &b, nullptr, nullptr, nullptr,
                              nullptr, nullptr);
    pairs[0] = a;
    pairs[1] = b;
    return st;
}

extern "C" int gs_encoder_error_flag(const gs_encoder_desc *e, const void *workspace, int *flag_host) {
    EncPlan p;
    int st = enc_plan(e, p);
    if (st != GS_OK) return st;
    cudaError_t ce = cudaMemcpy(flag_host, W<int>(const_cast<void *>(workspace), p.o_err), sizeof(int),
                                cudaMemcpyDeviceToHost);
    return ce == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}
