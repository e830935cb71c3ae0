// gs_conv.cu -- implicit-GEMM convolution on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes a 128-pixel x Cout output tile (M = 128 output pixels laid out as TY rows x TX
// columns of one image, N = Cout <= 256, fp32 accumulator in TMEM).  The K loop runs over
// (tap, input-channel chunk): for each k-block TMA brings the A tile (128 input pixels x KC channels,
// NHWC bf16, zero fill outside the image = the convolution's zero padding) and the B tile (Cout x KC
// slice of the packed weight matrix) into a STAGES-deep shared-memory ring; one thread issues
// tcgen05.mma (kind::f16, bf16 x bf16 -> f32) and commits each stage back to the producer.  The
// epilogue reads TMEM with tcgen05.ld (one output pixel per thread), adds the bias, applies the exact
// GELU, accumulates the GroupNorm(8) partial sums of the tile and stores bf16 NHWC.
//
// Stride-2 convolutions read their input through a 5-D view (C, x parity, x/2, y, image) so the
// 128 output pixels of a row map to TX consecutive elements of the x/2 axis; stride-1 convolutions
// read a TY x TX box directly.  Replaces nn.Conv2d + nn.GELU (+ the statistics pass of nn.GroupNorm)
// of the reference encoder (efficient_encoder.py:53-58, 86-87).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>

#include "../../include/gsplat_b200.h"
#include "gs_conv.cuh"
#include "gs_tc.cuh"

using namespace gs_tc;

namespace {

template <int BN, int KC, int STAGES>
__global__ void __launch_bounds__(128, 1) k_conv_tc(const __grid_constant__ CUtensorMap tmA,
                                                    const __grid_constant__ CUtensorMap tmB, ConvArgs a) {
    constexpr uint32_t A_BYTES = 128u * KC * 2u;
    constexpr uint32_t B_BYTES = (uint32_t)BN * KC * 2u;
    constexpr uint32_t STAGE = A_BYTES + B_BYTES;
    constexpr uint32_t LAYOUT = KC == 64 ? 2u : 6u;       // SWIZZLE_128B : SWIZZLE_32B
    constexpr uint32_t SBO = KC == 64 ? 1024u : 256u;     // 8 rows x row pitch
    constexpr int CPG = BN / 8;                           // channels per GroupNorm group
    extern __shared__ uint8_t dsmem[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], done;
    __shared__ uint32_t tmem_base;
    __shared__ float gsum[4][8], gsq[4][8];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int t = blockIdx.x;
    const int tx = t % a.tiles_x;
    t /= a.tiles_x;
    const int ty = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int x0 = tx * a.TX, y0 = ty * a.TY;

    if (warp == 0) {
        tmem_alloc(&tmem_base, BN < 32 ? 32 : BN);
        tmem_relinquish();
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        fence_barrier_init();
    }
    if (threadIdx.x == 64) {
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // TMA producer
            for (int kb = 0; kb < a.nkb; kb++) {
                const int s = kb % STAGES;
                if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, a.err, 1)) break;
                mbar_arrive_expect_tx(&full[s], STAGE);
                uint8_t *sa = smem + s * STAGE;
                uint8_t *sb = sa + A_BYTES;
                const int tap = kb / a.nchunks, chunk = kb - tap * a.nchunks;
                const int kh = tap / a.KW, kw = tap - kh * a.KW;
                const int c0 = chunk * KC;
                if (a.stride == 1) {
                    tma_load_4d(sa, &tmA, &full[s], c0, x0 + kw - a.pad, y0 + kh - a.pad, b);
                } else {
                    const int xin = 2 * x0 + kw - a.pad;
                    const int xp = xin & 1;
                    const int xh = (xin - xp) / 2;
                    for (int r = 0; r < a.TY; r++)
                        tma_load_5d(sa + r * a.TX * KC * 2, &tmA, &full[s], c0, xp, xh, 2 * (y0 + r) + kh - a.pad,
                                    b);
                }
                tma_load_2d(sb, &tmB, &full[s], kb * KC, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer
            constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
            for (int kb = 0; kb < a.nkb; kb++) {
                const int s = kb % STAGES;
                if (!mbar_wait(&full[s], (kb / STAGES) & 1, a.err, 2)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * STAGE);
                const uint32_t sb = sa + A_BYTES;
#pragma unroll
                for (int k = 0; k < KC / 16; k++)
                    mma_bf16(tbase, sdesc(sa + 32u * k, SBO, LAYOUT), sdesc(sb + 32u * k, SBO, LAYOUT), idesc,
                             (kb | k) != 0 ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            mma_commit(&done);
        }
    }
    __syncwarp();

    // epilogue: thread = one output pixel (TMEM lane), BN channels in chunks of 16
    const bool ok = mbar_wait(&done, 0, a.err, 3);
    tc_fence_after();
    const int m = warp * 32 + lane;
    const int yy = y0 + m / a.TX, xx = x0 + m % a.TX;
    const bool valid = ok && yy < a.Ho && xx < a.Wo;
    float gs[8], gq[8];
#pragma unroll
    for (int g = 0; g < 8; g++) {
        gs[g] = 0.f;
        gq[g] = 0.f;
    }
    __nv_bfloat16 *dst = a.out + (((long long)b * a.Ho + yy) * a.Wo + xx) * BN;
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            float x = v[i] + a.bias[c0 + i];
            if (a.gelu) x = 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
            v[i] = x;
            const int g = (c0 + i) / CPG;
            gs[g] += x;
            gq[g] += x * x;
        }
        if (valid) {
            uint4 p0, p1;
            uint32_t *q0 = &p0.x, *q1 = &p1.x;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                __nv_bfloat162 h0 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 + 2 * i], v[8 + 2 * i + 1]);
                q0[i] = *reinterpret_cast<uint32_t *>(&h0);
                q1[i] = *reinterpret_cast<uint32_t *>(&h1);
            }
            reinterpret_cast<uint4 *>(dst + c0)[0] = p0;
            reinterpret_cast<uint4 *>(dst + c0)[1] = p1;
        }
    }
    if (a.stats) {
#pragma unroll
        for (int g = 0; g < 8; g++) {
            float s = valid ? gs[g] : 0.f, q = valid ? gq[g] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                s += __shfl_xor_sync(0xffffffffu, s, o);
                q += __shfl_xor_sync(0xffffffffu, q, o);
            }
            if (lane == 0) {
                gsum[warp][g] = s;
                gsq[warp][g] = q;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (a.stats && threadIdx.x < 16) {
        const int g = threadIdx.x >> 1, which = threadIdx.x & 1;
        float v = 0.f;
        for (int w = 0; w < 4; w++) v += which ? gsq[w][g] : gsum[w][g];
        atomicAdd(&a.stats[(b * 8 + g) * 2 + which], (double)v);
    }
    if (warp == 0) tmem_dealloc(tbase, BN < 32 ? 32 : BN);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

int make_map(CUtensorMap *tm, const void *base, int rank, const uint64_t *dims, const uint64_t *strides_bytes,
             const uint32_t *box, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return GS_ERR_CUDA;
    uint32_t es[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void *>(base),
                    (const cuuint64_t *)dims, (const cuuint64_t *)strides_bytes, (const cuuint32_t *)box,
                    (const cuuint32_t *)es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GS_OK : GS_ERR_BAD_ARGUMENT;
}

template <int BN, int KC, int STAGES>
int launch(const CUtensorMap &tA, const CUtensorMap &tB, const ConvArgs &a, int nblocks, cudaStream_t st) {
    constexpr size_t SMEM = (size_t)STAGES * (128 * KC * 2 + BN * KC * 2) + 1024;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(k_conv_tc<BN, KC, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
        configured = true;
    }
    k_conv_tc<BN, KC, STAGES><<<nblocks, 128, SMEM, st>>>(tA, tB, a);
    return cudaGetLastError() == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

}  // namespace

// Choose the TY x TX output tile (TX * TY = 128) that wastes the fewest pixels.
void gs_conv_pick_tile(int Ho, int Wo, int *TX, int *TY) {
    long long best = -1;
    int btx = 128;
    for (int tx = 128; tx >= 8; tx >>= 1) {
        int ty = 128 / tx;
        long long cover = (long long)((Wo + tx - 1) / tx) * tx * ((Ho + ty - 1) / ty) * ty;
        long long waste = cover - (long long)Wo * Ho;
        if (best < 0 || waste < best) {
            best = waste;
            btx = tx;
        }
    }
    *TX = btx;
    *TY = 128 / btx;
}

int gs_conv_run(const gs_conv_desc *d, const void *in, const void *w, const float *bias, void *out, double *stats,
                int *err, cudaStream_t st) {
    if (!d || !in || !w || !bias || !out) return GS_ERR_BAD_ARGUMENT;
    const int B = d->B, Hi = d->H, Wi = d->W, Ci = d->Cin, Co = d->Cout;
    if (!(Co == 64 || Co == 128 || Co == 256)) return GS_ERR_BAD_ARGUMENT;
    const int KC = d->kind == 1 ? 16 : 64;
    if (Ci % KC != 0) return GS_ERR_BAD_ARGUMENT;
    if (d->stride == 2 && (Wi % 2 != 0)) return GS_ERR_BAD_ARGUMENT;
    if (d->stride != 1 && d->stride != 2) return GS_ERR_BAD_ARGUMENT;
    ConvArgs a;
    a.B = B; a.Hi = Hi; a.Wi = Wi; a.Ci = Ci; a.Co = Co;
    a.KH = d->kh; a.KW = d->kw; a.stride = d->stride; a.pad = d->pad;
    a.Ho = d->Ho > 0 ? d->Ho : (Hi + 2 * d->pad - d->kh) / d->stride + 1;
    a.Wo = d->Wo > 0 ? d->Wo : (Wi + 2 * d->pad - d->kw) / d->stride + 1;
    gs_conv_pick_tile(a.Ho, a.Wo, &a.TX, &a.TY);
    a.tiles_x = (a.Wo + a.TX - 1) / a.TX;
    a.tiles_y = (a.Ho + a.TY - 1) / a.TY;
    a.nchunks = Ci / KC;
    a.nkb = d->kh * d->kw * a.nchunks;
    a.gelu = d->gelu;
    a.bias = bias;
    a.out = reinterpret_cast<__nv_bfloat16 *>(out);
    a.stats = stats;
    a.err = err;
    CUtensorMap tA, tB;
    CUtensorMapSwizzle swz = KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B;
    int s;
    if (d->stride == 1) {
        uint64_t dims[4] = {(uint64_t)Ci, (uint64_t)Wi, (uint64_t)Hi, (uint64_t)B};
        uint64_t str[3] = {(uint64_t)Ci * 2, (uint64_t)Wi * Ci * 2, (uint64_t)Hi * Wi * Ci * 2};
        uint32_t box[4] = {(uint32_t)KC, (uint32_t)a.TX, (uint32_t)a.TY, 1};
        s = make_map(&tA, in, 4, dims, str, box, swz);
    } else {
        uint64_t dims[5] = {(uint64_t)Ci, 2, (uint64_t)(Wi / 2), (uint64_t)Hi, (uint64_t)B};
        uint64_t str[4] = {(uint64_t)Ci * 2, (uint64_t)Ci * 4, (uint64_t)Wi * Ci * 2, (uint64_t)Hi * Wi * Ci * 2};
        uint32_t box[5] = {(uint32_t)KC, 1, (uint32_t)a.TX, 1, 1};
        s = make_map(&tA, in, 5, dims, str, box, swz);
    }
    if (s != GS_OK) return s;
    const int K = d->kh * d->kw * Ci;
    {
        uint64_t dims[2] = {(uint64_t)K, (uint64_t)Co};
        uint64_t str[1] = {(uint64_t)K * 2};
        uint32_t box[2] = {(uint32_t)KC, (uint32_t)Co};
        s = make_map(&tB, w, 2, dims, str, box, swz);
    }
    if (s != GS_OK) return s;
    const int nblocks = B * a.tiles_x * a.tiles_y;
    if (KC == 16) return launch<64, 16, 8>(tA, tB, a, nblocks, st);
    if (Co == 64) return launch<64, 64, 4>(tA, tB, a, nblocks, st);
    if (Co == 128) return launch<128, 64, 4>(tA, tB, a, nblocks, st);
    return launch<256, 64, 4>(tA, tB, a, nblocks, st);
}

extern "C" int gs_conv2d(const gs_conv_desc *d, const void *in_bf16, const void *w_bf16, const float *bias,
                         void *out_bf16, double *gn_stats, int *err_flag, void *stream) {
    return gs_conv_run(d, in_bf16, w_bf16, bias, out_bf16, gn_stats, err_flag, (cudaStream_t)stream);
}
