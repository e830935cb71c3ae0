// gs_conv.cu -- implicit-GEMM convolution on the 5th-generation tensor cores (sm_100a).
//
// The output is cut into work items of MT vertically stacked M-tiles (each 128 output pixels laid out
// as TY rows x TX columns of one image) times a BN-wide slice of the output channels; a persistent grid
// strides over the items.  The K loop of an item runs over (tap, input-channel chunk): for each k-block
// TMA brings the MT A tiles (128 input pixels x KC channels, NHWC bf16, zero fill outside the image =
// the convolution's zero padding) and the B tile (BN x KC slice of the packed weight matrix) into a
// STAGES-deep shared-memory ring; one thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32) into
// TMEM and commits each stage back to the producer.  Accumulators are double-buffered in TMEM, so the
// epilogue warps (tcgen05.ld, bias, GELU, GroupNorm(8) partial sums, bf16 NHWC store) of one
// item run while the tensor cores work on the next.
//
// Stride-2 convolutions read their input through a 5-D view (C, x parity, x/2, y, image) so the
// TX output pixels of a row map to TX consecutive elements of the x/2 axis; stride-1 convolutions
// read a TY x TX box directly.  Replaces nn.Conv2d + nn.GELU (+ the statistics pass of nn.GroupNorm)
// of the reference encoder (efficient_encoder.py:53-58, 86-87).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>

#include <algorithm>

#include "../../include/gsplat_b200.h"
#include "gs_conv.cuh"
#include "gs_tc.cuh"

using namespace gs_tc;

namespace {

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU(x) = 0.5 x (1 + erf(x / sqrt 2)) with erf from the rational approximation of Abramowitz &
// Stegun, Handbook of Mathematical Functions, formula 7.1.26: for z >= 0,
// erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z), |error| <= 1.5e-7.
// 1 + erf(x / sqrt 2) is formed as 2 - q (x >= 0) or q (x < 0), q = t (...) exp(-z^2), so the negative
// tail keeps its relative accuracy.  In fp32 the GELU error stays below 7e-7 absolute over [-12, 12],
// far under the bf16 rounding of the stored activation.
__device__ __forceinline__ float gelu_erf(float x) {
    const float z = fabsf(x) * 0.70710678118654752f;
    const float t = rcp_approx(fmaf(0.3275911f, z, 1.0f));
    float q = fmaf(1.061405429f, t, -1.453152027f);
    q = fmaf(q, t, 1.421413741f);
    q = fmaf(q, t, -0.284496736f);
    q = fmaf(q, t, 0.254829592f);
    q *= t * ex2_approx(-(z * z) * 1.4426950408889634f);
    return 0.5f * x * (x >= 0.f ? 2.0f - q : q);
}

// Persistent, warp-specialised convolution.  Work item = MT vertically stacked 128-pixel M-tiles x
// one BN-wide slice of the output channels; CTAs stride over the items.
//   warp 0        TMA producer (one lane): A tiles of the MT M-tiles + the B slice, STAGES-deep ring
//   warp 1        TMEM owner + MMA issuer (one lane): MT accumulators of 128 x BN fp32 per item,
//                 double-buffered in TMEM so the epilogue of item i overlaps the K loop of item i+1
//   warps 2..     4*MT*CS epilogue warps: warp w drains TMEM lanes 32*(w%4).. of one accumulator, one of
//                 CS column slices --
//                 bias, GELU (gelu_erf), GroupNorm(8) partial sums, bf16 NHWC store
// Every wait is bounded; a wait that gives up records its stage in *err and raises a CTA-wide abort
// flag so the other roles stop issuing, then the CTA drains its copies and MMAs and frees TMEM.
template <int BN, int KC, int STAGES, int MT, int CPG, int MINB, int CS, bool HALO>
__global__ void __launch_bounds__(64 + 128 * MT * CS, MINB)
    k_conv_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
              const __grid_constant__ CUtensorMap tmB, ConvArgs a) {
    constexpr int NEPI = 4 * MT * CS;  // epilogue warps: 4 lane quarters x MT accumulators x CS column slices
    constexpr int BNS = BN / CS;        // columns drained by one epilogue warp
    static_assert(BNS % 16 == 0 && BNS % CPG == 0, "column slices hold whole chunks and GroupNorm groups");
    constexpr uint32_t A_BYTES = 128u * KC * 2u;
    constexpr uint32_t B_BYTES = (uint32_t)BN * KC * 2u;
    constexpr uint32_t STAGE = MT * A_BYTES + B_BYTES;
    constexpr uint32_t LAYOUT = KC == 64 ? 2u : 6u;    // SWIZZLE_128B : SWIZZLE_32B
    constexpr uint32_t SBO = KC == 64 ? 1024u : 256u;  // 8 rows x row pitch
    constexpr uint32_t ACC = (uint32_t)MT * BN;        // TMEM columns of one accumulator buffer
    constexpr uint32_t TCOLS = 2 * ACC < 32 ? 32 : 2 * ACC;
    static_assert((TCOLS & (TCOLS - 1)) == 0 && TCOLS <= 512, "TMEM columns");
    static_assert(CPG % 8 == 0 && (CPG >= 16 ? CPG % 16 == 0 : true), "GroupNorm channels per group");
    extern __shared__ uint8_t dsmem[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], mdone, bfull;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ int issued, consumed, b_issued;
    __shared__ __align__(16) float sbias[256];
    __shared__ float sacc[NEPI][16];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nsplit = a.Co / BN;
    const int n_items = a.B * a.tiles_y * a.tiles_x * nsplit;

    for (int i = threadIdx.x; i < a.Co; i += blockDim.x) sbias[i] = a.bias[i];
    for (int i = threadIdx.x; i < NEPI * 16; i += blockDim.x) (&sacc[0][0])[i] = 0.f;
    if (warp == 1) {
        tmem_alloc(&tmem_base, TCOLS);
        tmem_relinquish();
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int j = 0; j < 2; j++) {
            mbar_init(&tfull[j], 1);
            mbar_init(&tempty[j], NEPI);
        }
        mbar_init(&mdone, 1);
        mbar_init(&bfull, 1);
        abort_flag = 0;
        issued = 0;
        consumed = 0;
        b_issued = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        if (a.nchunks1 < a.nchunks) prefetch_tensormap(&tmA2);
        prefetch_tensormap(&tmB);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base;

    // halo form: [weights, hbreg bytes][STAGES windows of KC/8 slices]
    uint8_t *const hwin = smem + a.hbreg;
    const uint32_t hstage = (uint32_t)(KC / 8) * (uint32_t)a.hslice;
    if (HALO && warp == 0) {
        if (lane == 0) {
            // every (tap, 8-channel slice) of the BN weight rows once: [tap][slice][BN rows][16 B]
            mbar_arrive_expect_tx(&bfull, (uint32_t)a.hbreg);
            const int ntap = a.KH * a.KW;
            for (int t = 0; t < ntap; t++)
#pragma unroll
                for (int sl = 0; sl < KC / 8; sl++)
                    tma_load_2d(smem + (t * (KC / 8) + sl) * BN * 16, &tmB, &bfull, t * KC + sl * 8, 0);
            b_issued = 1;
            int it = 0;
            for (int item = blockIdx.x; item < n_items && !abort_flag; item += gridDim.x, it++) {
                int t = item;
                t /= nsplit;
                const int tx = t % a.tiles_x;
                t /= a.tiles_x;
                const int ty = t % a.tiles_y;
                const int b = t / a.tiles_y;
                const int x0 = tx * a.TX, y0 = ty * MT;  // TX = 128, TY = 1
                const int s = it % STAGES;
                if (it >= STAGES && !mbar_wait_or_abort(&empty[s], ((it / STAGES) - 1) & 1, &abort_flag, a.err, 1))
                    break;
                if (abort_flag) break;
                // (the boxes' bytes: the slices are padded to 128-byte multiples in shared memory only)
                mbar_arrive_expect_tx(&full[s], (uint32_t)(KC / 8) * 16u * (uint32_t)(a.hcols * a.hrows));
#pragma unroll
                for (int sl = 0; sl < KC / 8; sl++)
                    tma_load_4d(hwin + s * hstage + sl * a.hslice, &tmA, &full[s], sl * 8, x0 - a.padw, y0 - a.pad, b);
                issued = it + 1;
            }
        }
    } else if (HALO && warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
            const uint32_t sbw = smem_u32(smem), sw0 = smem_u32(hwin);
            const uint32_t rowb = (uint32_t)a.hcols * 16u;
            bool ok = mbar_wait_or_abort(&bfull, 0, &abort_flag, a.err, 7);
            int it = 0, tc = 0;
            for (int item = blockIdx.x; ok && item < n_items && !abort_flag; item += gridDim.x, tc++, it++) {
                const int buf = tc & 1;
                if (tc >= 2 && !mbar_wait_or_abort(&tempty[buf], ((tc >> 1) - 1) & 1, &abort_flag, a.err, 2)) break;
                tc_fence_after();
                const uint32_t dcol = tbase + (uint32_t)buf * ACC;
                const int s = it % STAGES;
                if (!mbar_wait_or_abort(&full[s], (it / STAGES) & 1, &abort_flag, a.err, 3)) break;
                tc_fence_after();
                const uint32_t win = sw0 + (uint32_t)s * hstage;
                // tap (kh, kw) of output row mt: the window from row mt + kh, column kw (a 16-byte offset per
                // pixel in the unswizzled layout); K = 16 per instruction = two 8-channel slices (LBO apart)
                for (int kh = 0; kh < a.KH; kh++)
                    for (int kw = 0; kw < a.KW; kw++) {
                        const uint32_t tap = (uint32_t)(kh * a.KW + kw);
#pragma unroll
                        for (int k = 0; k < KC / 16; k++) {
                            const uint64_t bd = sdesc_ns(sbw + (tap * (KC / 8) + 2 * k) * BN * 16, BN * 16, 128);
#pragma unroll
                            for (int mt = 0; mt < MT; mt++) {
                                const uint32_t aa = win + 2u * k * (uint32_t)a.hslice + (uint32_t)(mt + kh) * rowb +
                                                    (uint32_t)kw * 16u;
                                mma_bf16(dcol + (uint32_t)(mt * BN), sdesc_ns(aa, (uint32_t)a.hslice, 128), bd, idesc,
                                         (tap | k) != 0 ? 1u : 0u);
                            }
                        }
                    }
                mma_commit(&empty[s]);
                consumed = it + 1;
                mma_commit(&tfull[buf]);
            }
            mma_commit(&mdone);
            mbar_wait(&mdone, 0, a.err, 4);
        }
    } else if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int item = blockIdx.x; item < n_items && !abort_flag; item += gridDim.x) {
                int t = item;
                const int nb = t % nsplit;
                t /= nsplit;
                const int tx = t % a.tiles_x;
                t /= a.tiles_x;
                const int ty = t % a.tiles_y;
                const int b = t / a.tiles_y;
                const int x0 = tx * a.TX, y0 = ty * a.TY * MT;
                // (kh, kw, chunk) of k-block kb, stepped without divisions
                int kh = 0, kw = 0, chunk = 0;
                for (int kb = 0; kb < a.nkb; kb++, it++) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait_or_abort(&empty[s], ((it / STAGES) - 1) & 1, &abort_flag, a.err, 1))
                        break;
                    if (abort_flag) break;
                    mbar_arrive_expect_tx(&full[s], STAGE);
                    uint8_t *sa = smem + s * STAGE;
                    uint8_t *sb = sa + MT * A_BYTES;
                    // input channels [0, nchunks1*KC) come from tmA, the rest from tmA2 (a concatenation
                    // the convolution reads in place)
                    const bool first = chunk < a.nchunks1;
                    const CUtensorMap *ma = first ? &tmA : &tmA2;
                    const int c0 = (first ? chunk : chunk - a.nchunks1) * KC;
#pragma unroll
                    for (int mt = 0; mt < MT; mt++) {
                        const int ym = y0 + mt * a.TY;
                        if (a.stride == 1) {
                            tma_load_4d(sa + mt * A_BYTES, ma, &full[s], c0, x0 + kw - a.padw, ym + kh - a.pad, b);
                        } else {
                            const int xin = 2 * x0 + kw - a.padw;
                            const int xp = xin & 1;
                            const int xh = (xin - xp) / 2;
                            for (int r = 0; r < a.TY; r++)
                                tma_load_5d(sa + mt * A_BYTES + r * a.TX * KC * 2, ma, &full[s], c0, xp, xh,
                                            2 * (ym + r) + kh - a.pad, b);
                        }
                    }
                    tma_load_2d(sb, &tmB, &full[s], kb * KC, nb * BN);
                    issued = it + 1;
                    if (++chunk == a.nchunks) {
                        chunk = 0;
                        if (++kw == a.KW) {
                            kw = 0;
                            ++kh;
                        }
                    }
                }
                if (abort_flag) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
            int it = 0, tc = 0;
            for (int item = blockIdx.x; item < n_items && !abort_flag; item += gridDim.x, tc++) {
                const int buf = tc & 1;
                if (tc >= 2 && !mbar_wait_or_abort(&tempty[buf], ((tc >> 1) - 1) & 1, &abort_flag, a.err, 2)) break;
                tc_fence_after();
                const uint32_t dcol = tbase + (uint32_t)buf * ACC;
                bool ok = true;
                for (int kb = 0; kb < a.nkb; kb++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait_or_abort(&full[s], (it / STAGES) & 1, &abort_flag, a.err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * STAGE);
                    const uint32_t sb = sa + MT * A_BYTES;
#pragma unroll
                    for (int k = 0; k < KC / 16; k++) {
                        const uint64_t bd = sdesc(sb + 32u * k, SBO, LAYOUT);
#pragma unroll
                        for (int mt = 0; mt < MT; mt++)
                            mma_bf16(dcol + (uint32_t)(mt * BN), sdesc(sa + mt * A_BYTES + 32u * k, SBO, LAYOUT), bd,
                                     idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                    consumed = it + 1;
                }
                if (!ok) break;
                mma_commit(&tfull[buf]);
            }
            // all MMAs of this CTA (also those of an aborted item) have finished once mdone flips
            mma_commit(&mdone);
            mbar_wait(&mdone, 0, a.err, 4);
        }
    } else {
        // epilogue
        const int e = warp - 2;
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int mt = (e >> 2) % MT, cs = (e >> 2) / MT;
        const int clo = cs * BNS, chi = clo + BNS;
        const int m = q * 32 + lane;
        float *acc = sacc[e];
        int cur_b = -1, tc = 0;
        // per-lane GroupNorm sums of the warp's NG = BNS / CPG groups for the current (image, slice)
        constexpr int NG = BNS / CPG;
        float ls[NG], lq[NG];
#pragma unroll
        for (int k = 0; k < NG; k++) ls[k] = lq[k] = 0.f;
        int lane_b = -1, lane_nb = 0;
        // the lanes' sums of (lane_b, lane_nb) into the warp's accumulators, in a fixed xor-tree order
        auto fold_lanes = [&]() {
            if (lane_b < 0) return;
#pragma unroll
            for (int k = 0; k < NG; k++) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    ls[k] += __shfl_xor_sync(0xffffffffu, ls[k], o);
                    lq[k] += __shfl_xor_sync(0xffffffffu, lq[k], o);
                }
                if (lane == 0) {
                    const int g = (lane_nb * BN + clo) / CPG + k;
                    acc[2 * g] += ls[k];
                    acc[2 * g + 1] += lq[k];
                }
                ls[k] = lq[k] = 0.f;
            }
            __syncwarp();
        };
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, tc++) {
            int t = item;
            const int nb = t % nsplit;
            t /= nsplit;
            const int tx = t % a.tiles_x;
            t /= a.tiles_x;
            const int ty = t % a.tiles_y;
            const int b = t / a.tiles_y;
            const int yy = ty * a.TY * MT + mt * a.TY + m / a.TX, xx = tx * a.TX + m % a.TX;
            const bool valid = yy < a.Ho && xx < a.Wo;
            const int buf = tc & 1;
            if (!mbar_wait_or_abort(&tfull[buf], (tc >> 1) & 1, &abort_flag, a.err, 5)) break;
            tc_fence_after();
            // the lanes' sums of the previous (image, slice) reach the warp's accumulators first
            if (a.stats && (b != lane_b || nb != lane_nb)) {
                fold_lanes();
                lane_b = b;
                lane_nb = nb;
            }
            if (a.stats && b != cur_b) {
                if (cur_b >= 0 && lane < 16) {
                    atomicAdd(&a.stats[cur_b * 16 + lane], (double)acc[lane]);
                    acc[lane] = 0.f;
                }
                cur_b = b;
                __syncwarp();
            }
            const int n0 = nb * BN;
            __nv_bfloat16 *dst = a.out + (((long long)b * a.Ho + yy) * a.Wo + xx) * a.Co + n0;
            const uint32_t taddr = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)buf * ACC + (uint32_t)(mt * BN);
            // one 16-column chunk: TMEM -> bias, GELU, bf16 store; its GroupNorm partial sums (two groups of
            // 8 channels for CPG = 8, else one slice of a group) in s0/q0 (and s1/q1)
            auto process = [&](int c0, float &s0, float &q0, float &s1, float &q1) {
                float v[16];
                tmem_ld16(taddr + (uint32_t)c0, v);
                if (c0 + 16 == chi) {
                    // the accumulator buffer is drained: hand it back to the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[buf]);
                }
                s0 = q0 = s1 = q1 = 0.f;
                const float4 *bb = reinterpret_cast<const float4 *>(sbias + n0 + c0);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 bj = bb[j];
                    v[4 * j] += bj.x;
                    v[4 * j + 1] += bj.y;
                    v[4 * j + 2] += bj.z;
                    v[4 * j + 3] += bj.w;
                }
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    float x = v[i];
                    if (a.gelu) x = gelu_erf(x);
                    v[i] = x;
                    if (CPG == 8 && i >= 8) {
                        s1 += x;
                        q1 += x * x;
                    } else {
                        s0 += x;
                        q0 += x * x;
                    }
                }
                if (valid) {
                    uint4 p0, p1;
                    uint32_t *w0 = &p0.x, *w1 = &p1.x;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 + 2 * i], v[8 + 2 * i + 1]);
                        w0[i] = *reinterpret_cast<uint32_t *>(&h0);
                        w1[i] = *reinterpret_cast<uint32_t *>(&h1);
                    }
                    reinterpret_cast<uint4 *>(dst + c0)[0] = p0;
                    reinterpret_cast<uint4 *>(dst + c0)[1] = p1;
                }
            };
            // GroupNorm sums stay in the lane's registers across chunks and items (ls/lq, folded into the
            // warp's shared accumulators when the image or channel slice changes, above): no warp
            // reduction per chunk
#pragma unroll
            for (int ci = 0; ci < BNS / 16; ci++) {
                float s0, q0, s1, q1;
                process(clo + 16 * ci, s0, q0, s1, q1);
                if (a.stats && valid) {
                    if (CPG == 8) {
                        ls[2 * ci] += s0;
                        lq[2 * ci] += q0;
                        ls[2 * ci + 1] += s1;
                        lq[2 * ci + 1] += q1;
                    } else {
                        ls[ci * 16 / CPG] += s0;
                        lq[ci * 16 / CPG] += q0;
                    }
                }
            }
        }
        __syncwarp();
        if (a.stats) fold_lanes();
        __syncwarp();
        if (a.stats && cur_b >= 0 && lane < 16) atomicAdd(&a.stats[cur_b * 16 + lane], (double)acc[lane]);
    }

    tc_fence_before();
    __syncthreads();
    if (abort_flag && threadIdx.x == 0) {
        // copies that were issued but never consumed still land in shared memory: wait for them
        for (int j = consumed; j < issued; j++) mbar_wait(&full[j % STAGES], (j / STAGES) & 1, a.err, 6);
        if (HALO && b_issued) mbar_wait(&bfull, 0, a.err, 8);
    }
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, TCOLS);
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

int sm_count() {
    static int n[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!n[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n[dev] = v > 0 ? v : 148;
    }
    return n[dev];
}

template <int BN, int KC, int STAGES, int MT, int CPG, int MINB, int CS, bool HALO = false>
int launch(const CUtensorMap &tA, const CUtensorMap &tA2, const CUtensorMap &tB, const ConvArgs &a,
           cudaStream_t st) {
    const size_t SMEM = HALO ? (size_t)a.hbreg + (size_t)STAGES * (KC / 8) * a.hslice + 1024
                             : (size_t)STAGES * (MT * 128 * KC * 2 + BN * KC * 2) + 1024;
    auto kern = k_conv_tc<BN, KC, STAGES, MT, CPG, MINB, CS, HALO>;
    static size_t configured = 0;
    if (configured < SMEM) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
        configured = SMEM;
    }
    const long long items = (long long)a.B * a.tiles_y * a.tiles_x * (a.Co / BN);
    const long long slots = (long long)sm_count() * MINB;
    const int grid = (int)(items < slots ? items : slots);
    kern<<<grid, 64 + 128 * MT * CS, SMEM, st>>>(tA, tA2, tB, a);
    return cudaGetLastError() == cudaSuccess ? GS_OK : GS_ERR_CUDA;
}

}  // namespace

// Choose the TY x TX M-tile (TX * TY = 128) whose MT-stacked cover of the output wastes the fewest
// pixels; ties go to the wider tile.
void gs_conv_pick_tile(int Ho, int Wo, int MT, int *TX, int *TY) {
    long long best = -1;
    int btx = 128;
    for (int tx = 128; tx >= 8; tx >>= 1) {
        int ty = (128 / tx) * MT;
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
    return gs_conv_run2(d, in, d ? d->Cin : 0, nullptr, w, bias, out, stats, err, st);
}

int gs_conv_run2(const gs_conv_desc *d, const void *in, int Cin1, const void *in2, const void *w, const float *bias,
                 void *out, double *stats, int *err, cudaStream_t st, int padw) {
    if (!d || !in || !w || !bias || !out) return GS_ERR_BAD_ARGUMENT;
    const int B = d->B, Hi = d->H, Wi = d->W, Ci = d->Cin, Co = d->Cout;
    const int Ci2 = Ci - Cin1;
    if (Cin1 <= 0 || Ci2 < 0 || (Ci2 > 0 && !in2)) return GS_ERR_BAD_ARGUMENT;
    if (B <= 0 || Hi <= 0 || Wi <= 0 || d->kh <= 0 || d->kw <= 0 || d->pad < 0) return GS_ERR_BAD_ARGUMENT;
    if (!(Co == 64 || Co == 128 || Co == 256)) return GS_ERR_BAD_ARGUMENT;
    const int KC = d->kind == 1 ? 16 : 64;
    if (Ci % KC != 0 || Cin1 % KC != 0) return GS_ERR_BAD_ARGUMENT;
    if (d->kind == 1 && Co != 64) return GS_ERR_BAD_ARGUMENT;
    if (d->stride == 2 && (Wi % 2 != 0)) return GS_ERR_BAD_ARGUMENT;
    if (d->stride != 1 && d->stride != 2) return GS_ERR_BAD_ARGUMENT;
    // kernel shape per layer: MT stacked M-tiles per work item, BN output channels per item.  The 3x3
    // layers at Cout 128 / 256 take single 128-pixel tiles (and 64-channel slices at 256) with 3 stages, so
    // two or three CTAs share an SM: a layer at 768^2 has only ~150 items of MT = 2, one per SM, whose TMA +
    // MMA latency chain and epilogue then ran back to back with nothing to overlap them
    const int MT = (KC == 64 && Co >= 128) ? 1 : 2;
    int BN = Co == 256 ? 64 : Co;
    ConvArgs a;
    memset(&a, 0, sizeof(a));
    a.B = B; a.Hi = Hi; a.Wi = Wi; a.Ci = Ci; a.Co = Co;
    a.KH = d->kh; a.KW = d->kw; a.stride = d->stride; a.pad = d->pad; a.padw = padw >= 0 ? padw : d->pad;
    a.Ho = d->Ho > 0 ? d->Ho : (Hi + 2 * d->pad - d->kh) / d->stride + 1;
    a.Wo = d->Wo > 0 ? d->Wo : (Wi + 2 * a.padw - d->kw) / d->stride + 1;
    if (a.Ho <= 0 || a.Wo <= 0) return GS_ERR_BAD_ARGUMENT;
    // Cout 256: 128-channel slices (each A tile read twice instead of four times) once the layer has items
    // enough for two CTAs per SM
    if (Co == 256 && KC == 64 && (long long)B * a.Ho * a.Wo / 128 * 2 >= 2LL * sm_count()) BN = 128;

    gs_conv_pick_tile(a.Ho, a.Wo, MT, &a.TX, &a.TY);
    a.tiles_x = (a.Wo + a.TX - 1) / a.TX;
    a.tiles_y = (a.Ho + a.TY * MT - 1) / (a.TY * MT);
    a.nchunks = Ci / KC;
    a.nchunks1 = Cin1 / KC;
    a.nkb = d->kh * d->kw * a.nchunks;
    a.gelu = d->gelu;
    a.bias = bias;
    a.out = reinterpret_cast<__nv_bfloat16 *>(out);
    a.stats = stats;
    a.err = err;
    CUtensorMap tA, tA2, tB;
    CUtensorMapSwizzle swz = KC == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B;
    // NHWC input with Cm channels: a 4-D box for stride 1, a 5-D (C, x parity, x/2, y, image) view for stride 2
    auto input_map = [&](CUtensorMap *tm, const void *ptr, int Cm) {
        if (d->stride == 1) {
            uint64_t dims[4] = {(uint64_t)Cm, (uint64_t)Wi, (uint64_t)Hi, (uint64_t)B};
            uint64_t str[3] = {(uint64_t)Cm * 2, (uint64_t)Wi * Cm * 2, (uint64_t)Hi * Wi * Cm * 2};
            uint32_t box[4] = {(uint32_t)KC, (uint32_t)a.TX, (uint32_t)a.TY, 1};
            return make_map(tm, ptr, 4, dims, str, box, swz);
        }
        uint64_t dims[5] = {(uint64_t)Cm, 2, (uint64_t)(Wi / 2), (uint64_t)Hi, (uint64_t)B};
        uint64_t str[4] = {(uint64_t)Cm * 2, (uint64_t)Cm * 4, (uint64_t)Wi * Cm * 2, (uint64_t)Hi * Wi * Cm * 2};
        uint32_t box[5] = {(uint32_t)KC, 1, (uint32_t)a.TX, 1, 1};
        return make_map(tm, ptr, 5, dims, str, box, swz);
    };
    int s = input_map(&tA, in, Cin1);
    if (s != GS_OK) return s;
    if (Ci2 > 0) {
        s = input_map(&tA2, in2, Ci2);
        if (s != GS_OK) return s;
    } else {
        tA2 = tA;
    }
    const int K = d->kh * d->kw * Ci;
    {
        uint64_t dims[2] = {(uint64_t)K, (uint64_t)Co};
        uint64_t str[1] = {(uint64_t)K * 2};
        uint32_t box[2] = {(uint32_t)KC, (uint32_t)BN};
        s = make_map(&tB, w, 2, dims, str, box, swz);
    }
    if (s != GS_OK) return s;
    // halo form for the stride-1 layer on one 16-channel chunk (the first convolution): one window per item
    // (MT + KH - 1 rows x 128 + KW - 1 pixels, two 8-channel slices, unswizzled) serves all KH x KW taps,
    // and the layer's weights stay in shared memory for the CTA's whole life: 2 TMA copies per item
    // instead of 3 per tap
    const char *hv = getenv("GS_CONV_HALO");
    if (KC == 16 && d->stride == 1 && Ci == KC && Ci2 == 0 && a.TX == 128 && a.TY == 1 && BN == Co && MT == 2 &&
        d->kw <= 129 && MT + d->kh - 1 <= 256 && !(hv && hv[0] == '0')) {
        a.hcols = 128 + d->kw - 1;
        a.hrows = MT + d->kh - 1;
        a.hslice = (16 * a.hcols * a.hrows + 127) & ~127;
        a.hbreg = d->kh * d->kw * (KC / 8) * BN * 16;
        CUtensorMap hA, hB;
        uint64_t dims[4] = {(uint64_t)Ci, (uint64_t)Wi, (uint64_t)Hi, (uint64_t)B};
        uint64_t str[3] = {(uint64_t)Ci * 2, (uint64_t)Wi * Ci * 2, (uint64_t)Hi * Wi * Ci * 2};
        uint32_t box[4] = {8, (uint32_t)a.hcols, (uint32_t)a.hrows, 1};
        if ((s = make_map(&hA, in, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)) != GS_OK) return s;
        uint64_t wd[2] = {(uint64_t)K, (uint64_t)Co};
        uint64_t ws[1] = {(uint64_t)K * 2};
        uint32_t wb[2] = {8, (uint32_t)BN};
        if ((s = make_map(&hB, w, 2, wd, ws, wb, CU_TENSOR_MAP_SWIZZLE_NONE)) != GS_OK) return s;
        return launch<64, 16, 3, 2, 8, 2, 1, true>(hA, hA, hB, a, st);
    }
    // one column slice per accumulator: doubling the epilogue warps (CS = 2) measured slower on B200
    if (KC == 16) return launch<64, 16, 8, 2, 8, 2, 1>(tA, tA2, tB, a, st);
    if (Co == 64) return launch<64, 64, 5, 2, 8, 1, 1>(tA, tA2, tB, a, st);
    // (Cout 128 in two-M-tile items at 4 stages, one CTA per SM, measured no faster at four images per launch)
    if (Co == 128) return launch<128, 64, 3, 1, 16, 2, 1>(tA, tA2, tB, a, st);
    return BN == 128 ? launch<128, 64, 3, 1, 32, 2, 1>(tA, tA2, tB, a, st)
                     : launch<64, 64, 3, 1, 32, 3, 1>(tA, tA2, tB, a, st);
}

extern "C" int gs_conv2d(const gs_conv_desc *d, const void *in_bf16, const void *w_bf16, const float *bias,
                         void *out_bf16, double *gn_stats, int *err_flag, void *stream) {
    return gs_conv_run(d, in_bf16, w_bf16, bias, out_bf16, gn_stats, err_flag, (cudaStream_t)stream);
}
