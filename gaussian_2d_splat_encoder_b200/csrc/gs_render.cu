// gs_render.cu -- tile-binned, order-independent ("odds"/alpha) splat renderer for sm_100a.
//
// Replaces the reference's render path (bigwolfeman/gaussian-2d-splat-encoder,
// gaussian_splat_encoder/render_triton.py): the octave routing + per-octave _build_tiles +
// _gather_pairs + _render_fwd_cull_kernel + _upsample_field + composite (forward), and
// _render_bwd_cull_kernel + index_add_ + the autograd of the upsample/composite (backward).
//
// Forward, one launch sequence for the whole batch and all octaves (no host sync):
//   k_preprocess   per splat: softplus scale, octave, clamped tile rectangle, 48-byte render record; the
//                  rectangle rows into a difference array of per-tile pair counts
//   k_tile_scan    tile counts -> every tile's [begin, end) in the pair list, a cursor per tile, the total
//   k_scatter      every (tile, splat) pair placed at its tile's cursor (load-balanced per 256 splats)
//   k_fields_fwd   one CTA per tile: raw sums S_log, S_w, S_wc of every group (octave) at its own
//                  resolution; splat records staged per warp in shared memory
//   k_composite    bilinear upsample of every present group to native resolution, sum, composite
// Backward:
//   k_composite_bwd  dS fields at native resolution, bg gradient
//   k_adjoint_*      adjoint of the bilinear upsample -> dS fields of every coarse group (direct gather for
//                    upsampling factors <= 8, separable row/column passes for deeper octaves)
//   k_fields_bwd     one CTA per tile, one lane per (tile, splat) pair looping over the tile's
//                    pixels; 9 per-splat sums leave through 3 vector atomics per pair
//   k_finalize       per-splat chain rule (rotation, scale, softplus) into the leaf gradients
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "../../include/gsplat_b200.h"
#include "gs_common.cuh"

static thread_local char g_last_error[512] = "";
static unsigned long long g_launches = 0;  // kernels enqueued by this library (all threads)

#define GS_COUNT(n) __atomic_fetch_add(&g_launches, (unsigned long long)(n), __ATOMIC_RELAXED)

#include <memory>
#include <mutex>
#include <vector>

#include "gs_prof.cuh"
#include "gs_render_internal.cuh"

namespace {
struct ProfEvent {
    int region;
    cudaEvent_t a, b;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfEvent> g_prof_pool;  // pre-created events
size_t g_prof_used = 0;
}  // namespace

bool gs_prof_on() { return g_prof_on; }
static thread_local int g_prof_internal = 0;
void gs_prof_set_internal(int on) { g_prof_internal = on; }
int gs_prof_internal() { return g_prof_internal; }
void gs_prof_take(int region, cudaEvent_t *a, cudaEvent_t *b) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_used >= g_prof_pool.size()) {
        *a = *b = nullptr;
        return;
    }
    ProfEvent &e = g_prof_pool[g_prof_used++];
    e.region = region;
    *a = e.a;
    *b = e.b;
}
void gs_count_launch(unsigned long long n) { GS_COUNT(n); }

void gs_set_last_error(const char *msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : ""); }

static int set_cuda_error(cudaError_t e, const char *where) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, cudaGetErrorString(e));
    return GS_ERR_CUDA;
}

#define GS_CHECK_LAUNCH(where)                                   \
    do {                                                         \
        GS_COUNT(1);                                             \
        cudaError_t _e = cudaGetLastError();                     \
        if (_e != cudaSuccess) return set_cuda_error(_e, where); \
    } while (0)

// ----------------------------------------------------------------------------------------------------
// block-wide helpers

template <int NT, typename T = int>
__device__ __forceinline__ T block_excl_scan(T v, T *warp_sums, T *total) {
    constexpr int NWARP = NT / 32;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        T s = lane < NWARP ? warp_sums[lane] : (T)0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            T y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < NWARP) warp_sums[lane] = s;  // inclusive
    }
    __syncthreads();
    T warp_prefix = warp > 0 ? warp_sums[warp - 1] : (T)0;
    if (total) *total = warp_sums[NWARP - 1];
    T r = warp_prefix + x - v;
    __syncthreads();
    return r;
}

// ----------------------------------------------------------------------------------------------------
// geometry of a splat (render_triton.py:362-377 and 925-952), fp32 with no contraction so the tile
// rectangle is bit-identical to the reference's separate torch ops.

__device__ __forceinline__ int octave_of(float sy, float sx, float rep, float bt, int maxo) {
    float sp = __fmul_rn(fmaxf(sy, sx), rep);
    float q = __fdiv_rn(sp, bt);
    q = fmaxf(q, 1e-6f);
    float o = ceilf(log2f(q));
    o = fminf(fmaxf(o, 0.0f), (float)maxo);
    return (int)o;
}

__device__ __forceinline__ void tile_rect(float muy, float mux, float sy, float sx, int Hg, int Wg, int T,
                                          float cutoff, int ntx, int nty, int &x0, int &x1, int &y0, int &y1) {
    float cx = __fmul_rn(mux, (float)Wg);
    float cy = __fmul_rn(muy, (float)Hg);
    float r = __fmul_rn(cutoff, fmaxf(sy, sx));
    float rx = __fmul_rn(r, (float)Wg);
    float ry = __fmul_rn(r, (float)Hg);
    float fT = (float)T;
    float a = floorf(__fdiv_rn(__fsub_rn(cx, rx), fT));
    float b = floorf(__fdiv_rn(__fadd_rn(cx, rx), fT));
    float c = floorf(__fdiv_rn(__fsub_rn(cy, ry), fT));
    float d = floorf(__fdiv_rn(__fadd_rn(cy, ry), fT));
    float mx = (float)(ntx - 1), my = (float)(nty - 1);
    x0 = (int)fminf(fmaxf(a, 0.0f), mx);
    x1 = (int)fminf(fmaxf(b, 0.0f), mx);
    y0 = (int)fminf(fmaxf(c, 0.0f), my);
    y1 = (int)fminf(fmaxf(d, 0.0f), my);
}

__device__ __forceinline__ int group_of_splat(const RenderGeom &G, int i, float sy, float sx) {
    if (G.mode == GS_MODE_OCTAVE) return octave_of(sy, sx, G.rep, G.base_texels, G.max_oct);
    if (G.mode == GS_MODE_MULTIRES) return (G.n_coarse > 0 && G.n_coarse < G.N && i < G.n_coarse) ? 0 : 1;
    return 0;
}

// ----------------------------------------------------------------------------------------------------
// forward: preprocessing

// Render record of splat s (activate_scale of params.py:18-28, the rotation of render.py:21-26 and the
// opacity), with the activated scales returned in sy, sx.
__device__ __forceinline__ SplatRec make_rec(long long s, int C, int has_theta, const float *__restrict__ mu,
                                             const float *__restrict__ ls, const float *__restrict__ col,
                                             const float *__restrict__ op, const float *__restrict__ th, float &sy,
                                             float &sx) {
    float2 m = reinterpret_cast<const float2 *>(mu)[s];  // (y, x)
    float2 l = reinterpret_cast<const float2 *>(ls)[s];
    sy = gs_softplus_eps(l.x);
    sx = gs_softplus_eps(l.y);
    float o = op[s];
    float cth = 1.0f, sth = 0.0f;
    if (has_theta) sincosf(th[s], &sth, &cth);
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
    if (C > 0) c0 = col[s * C + 0];
    if (C > 1) c1 = col[s * C + 1];
    if (C > 2) c2 = col[s * C + 2];
    float iy = GS_K / sy, ix = GS_K / sx;
    SplatRec r;
    r.a = make_float4(m.x, m.y, cth * iy, sth * iy);
    r.b = make_float4(-sth * ix, cth * ix, o, log2f(o));
    r.c = make_float4(c0, c1, c2, o <= GS_DEAD_OP ? 1.0f : 0.0f);
    return r;
}

// ----------------------------------------------------------------------------------------------------
// binning: per tile, the list of splats whose tile rectangle covers it (render_triton.py:351-409), as a
// counting sort of the (tile, splat) pairs by global tile id:
//
//   k_preprocess  per splat as above; each rectangle row [a, a + w) of global tile ids adds +1 at a and
//                 -1 at a + w of a difference array over all tiles (equal addresses of a warp summed
//                 first; the pairs themselves are not enumerated)
//   k_tile_scan   one block: tile counts = prefix of the differences, tile starts = exclusive prefix of
//                 the counts -> every tile's [begin, end), a cursor at its begin, the pair total, and the
//                 list of deep tiles (more than FW_DEEP pairs) for the 16-warp field kernel
//   k_scatter     the pairs enumerated in splat order, load-balanced per block of 256 splats, counted per
//                 tile in a shared-memory hash table and placed with one cursor atomic per (chunk, tile)
//
// Within a tile the splats therefore come in the order their groups reach the cursor, not by splat id:
// the forward fields are sums (alpha compositing of the octave/odds path is a commutative monoid), so the
// order only changes floating-point rounding, as the reference's own unstable argsort does.

// Layout of the 64-byte status block of a render workspace (zeroed before every forward).
#define MISC_TOTAL 0   // long long: pairs of the whole call
#define MISC_STATUS 8  // int: bit 0 set when the pairs exceed the workspace's pair capacity
#define MISC_NEFF 16   // long long: pairs the field kernels process (0 after an overflow)
#define MISC_NDEEP 24  // int: tiles in the deep-tile list
#define FW_DEEP 256    // pairs above which a TILE 8 tile is composited by 16 warps

__device__ __forceinline__ void red_add_i32(int *p, int v) {
    asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// meta = {global tile id of the rectangle's top-left, width | group << 24, ntx of the group, count}
// tdiff: tile difference array (zeroed beforehand; nullptr when only the counts are wanted).
__global__ void __launch_bounds__(256) k_preprocess(RenderGeom G, const float *__restrict__ mu,
                                                    const float *__restrict__ ls, const float *__restrict__ col,
                                                    const float *__restrict__ op, const float *__restrict__ th,
                                                    SplatRec *__restrict__ rec, int4 *__restrict__ meta,
                                                    int *__restrict__ counts, unsigned long long *__restrict__ gpairs,
                                                    int *__restrict__ gsplats, int *__restrict__ tdiff) {
    __shared__ unsigned long long s_pairs[4 * GS_MAX_GROUPS];
    __shared__ int s_spl[4 * GS_MAX_GROUPS];
    if (threadIdx.x < 4 * GS_MAX_GROUPS) {
        s_pairs[threadIdx.x] = 0ull;
        s_spl[threadIdx.x] = 0;
    }
    __syncthreads();
    const int b0 = G.N > 0 ? (int)(((long long)blockIdx.x * blockDim.x) / G.N) : 0;
    long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    int count = 0;
    int skey = -1;
    int row0 = 0, rstep = 0, rw = 1, nrows = 0;  // the rectangle's rows in global tile ids
    if (s < (long long)G.B * G.N) {
        int b = (int)(s / G.N), i = (int)(s - (long long)b * G.N);
        float2 m = reinterpret_cast<const float2 *>(mu)[s];  // (y, x)
        float sy, sx;
        rec[s] = make_rec(s, G.C, G.has_theta, mu, ls, col, op, th, sy, sx);
        int g = group_of_splat(G, i, sy, sx);
        int4 mt = make_int4(0, 0, 1, 0);
        if (G.mode != GS_MODE_EXACT) {
            GroupGeom gg = G.g[g];
            int x0, x1, y0, y1;
            tile_rect(m.x, m.y, sy, sx, gg.H, gg.W, G.tile, G.cutoff, gg.ntx, gg.nty, x0, x1, y0, y1);
            y0 = max(y0, gg.ty_lo);
            y1 = min(y1, gg.ty_hi);
            int w = x1 - x0 + 1;
            count = y1 >= y0 ? w * (y1 - y0 + 1) : 0;
            // a splat whose contribution arrives with a prior render's fields is not binned again
            if (i < G.skip_n && gg.prior_grp >= 0 &&
                octave_of(sy, sx, G.prior_rep, G.base_texels, G.max_oct) == gg.prior_grp)
                count = 0;
            mt = make_int4(b * G.tiles_per_image + gg.tile_off + y0 * gg.ntx + x0, w | (g << 24), gg.ntx, count);
        } else {
            mt.y = g << 24;
        }
        meta[s] = mt;
        counts[s] = count;
        skey = b * GS_MAX_GROUPS + g;
        row0 = mt.x;
        rstep = mt.z;
        rw = mt.y & 0xffffff;
        nrows = count > 0 ? count / rw : 0;
    }
    if (tdiff) {
        // rectangle rows into the difference array; neighbouring splats (the encoder emits them cell by
        // cell) often share a row's first or past-the-end tile, so equal addresses of a warp are summed
        // before one reduction each
        int rmax = nrows;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rmax = max(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
        const unsigned lt = (1u << (threadIdx.x & 31)) - 1u;
        for (int q = 0; q < rmax; q++) {
            const bool on = q < nrows;
            const int a = on ? row0 + q * rstep : -1;
            unsigned peers = __match_any_sync(0xffffffffu, a);
            if (on && (peers & lt) == 0u) red_add_i32(tdiff + a, __popc(peers));
            const int e = on ? a + rw : -1;
            peers = __match_any_sync(0xffffffffu, e);
            if (on && (peers & lt) == 0u) red_add_i32(tdiff + e, -(int)__popc(peers));
        }
    }
    {
        // aggregate per warp over lanes with the same (image, group), then per block in shared memory
        const unsigned peers = __match_any_sync(0xffffffffu, skey);
        const int npeer = __popc(peers);
        const unsigned psum = __reduce_add_sync(peers, (unsigned)count);
        const bool leader = (peers & ((1u << (threadIdx.x & 31)) - 1u)) == 0u;
        if (leader && skey >= 0) {
            const int b = skey / GS_MAX_GROUPS, g = skey % GS_MAX_GROUPS;
            if (b - b0 < 4) {
                atomicAdd(&s_pairs[(b - b0) * GS_MAX_GROUPS + g], (unsigned long long)psum);
                atomicAdd(&s_spl[(b - b0) * GS_MAX_GROUPS + g], npeer);
            } else {
                atomicAdd(&gpairs[b * G.ngroups + g], (unsigned long long)psum);
                atomicAdd(&gsplats[b * G.ngroups + g], npeer);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < 4 * GS_MAX_GROUPS && s_spl[threadIdx.x] > 0) {
        int bb = b0 + threadIdx.x / GS_MAX_GROUPS, gg = threadIdx.x % GS_MAX_GROUPS;
        atomicAdd(&gpairs[bb * G.ngroups + gg], s_pairs[threadIdx.x]);
        atomicAdd(&gsplats[bb * G.ngroups + gg], s_spl[threadIdx.x]);
    }
}

// One block of 1024 threads over the nt = B * tiles_per_image tiles, TS_PER consecutive tiles per thread
// per round: count = prefix of tdiff, begin = exclusive prefix of count (64-bit), ranges = [begin, begin +
// count), cursor = begin; tiles with more than FW_DEEP pairs go to dlist (order of arrival; at most
// cap / (FW_DEEP + 1) of them); misc gets the total, the overflow status, the effective pair count and
// the deep-tile count.  After an overflow (total > cap: rare, the ranges then point past the pair
// buffer) a second sweep empties every range and the lists, and k_scatter places nothing.
#define TS_THREADS 1024
#define TS_PER 16
// Exclusive block scan of non-negative values with the sum saturating at TS_SAT (associative for
// non-negative inputs, so the saturation only marks an overflowing total).
#define TS_SAT 0x7fffffffu
template <int NT>
__device__ __forceinline__ unsigned block_excl_scan_sat(unsigned v, unsigned *warp_sums, unsigned *total) {
    constexpr int NWARP = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x = min(x + y, TS_SAT);
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        unsigned s = lane < NWARP ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s = min(s + y, TS_SAT);
        }
        if (lane < NWARP) warp_sums[lane] = s;  // inclusive
    }
    __syncthreads();
    const unsigned wp = warp > 0 ? warp_sums[warp - 1] : 0u;
    if (total) *total = warp_sums[NWARP - 1];
    const unsigned r = min(wp + x, TS_SAT) - v;  // (exact whenever the inclusive sum did not saturate)
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(TS_THREADS) k_tile_scan(const int *__restrict__ tdiff, long long nt, long long cap,
                                                          int2 *__restrict__ ranges, int *__restrict__ cursor,
                                                          int *__restrict__ dlist, int dcap,
                                                          unsigned char *__restrict__ misc) {
    __shared__ int wsum_d[32];
    __shared__ unsigned wsum_c[32];
    const int tid = threadIdx.x;
    // 32-bit throughout: a tile's count (a prefix of the differences) is at most the splats of one image,
    // and the begin offsets saturate at 2^31 - 1 > cap, which then reads as an overflow
    int carry_d = 0;
    unsigned carry_c = 0u;
    for (long long base = 0; base < nt; base += (long long)TS_THREADS * TS_PER) {
        const long long lo = base + (long long)tid * TS_PER;
        // 16-byte loads: the difference array is zeroed and allocated in whole 256-byte blocks
        int dl[TS_PER];
#pragma unroll
        for (int k = 0; k < TS_PER; k += 4) {
            const int4 v = lo + k < nt ? *reinterpret_cast<const int4 *>(tdiff + lo + k) : make_int4(0, 0, 0, 0);
            dl[k] = v.x;
            dl[k + 1] = v.y;
            dl[k + 2] = v.z;
            dl[k + 3] = v.w;
        }
        int sd = 0;
#pragma unroll
        for (int k = 0; k < TS_PER; k++) {
            if (lo + k >= nt) dl[k] = 0;
            sd += dl[k];
        }
        int td;
        const int pd = carry_d + block_excl_scan<TS_THREADS, int>(sd, wsum_d, &td);
        // counts of this thread's tiles (past the last tile the running prefix is not a count)
        int run = pd;
        unsigned sc = 0u;
        int cnt[TS_PER];
#pragma unroll
        for (int k = 0; k < TS_PER; k++) {
            run += dl[k];
            cnt[k] = lo + k < nt ? run : 0;
            sc = min(sc + (unsigned)cnt[k], TS_SAT);
        }
        unsigned tc;
        unsigned beg = min(carry_c + block_excl_scan_sat<TS_THREADS>(sc, wsum_c, &tc), TS_SAT);
        int bg[TS_PER];
#pragma unroll
        for (int k = 0; k < TS_PER; k++) {
            bg[k] = (int)beg;
            beg = min(beg + (unsigned)cnt[k], TS_SAT);
            if (cnt[k] > FW_DEEP) {
                const int i = atomicAdd(reinterpret_cast<int *>(misc + MISC_NDEEP), 1);
                if (i < dcap) dlist[i] = (int)(lo + k);
            }
        }
        if (lo + TS_PER <= nt) {  // a whole run of 16 tiles: 16-byte stores
#pragma unroll
            for (int k = 0; k < TS_PER; k += 2)
                *reinterpret_cast<int4 *>(ranges + lo + k) =
                    make_int4(bg[k], bg[k] + cnt[k], bg[k + 1], bg[k + 1] + cnt[k + 1]);
#pragma unroll
            for (int k = 0; k < TS_PER; k += 4)
                *reinterpret_cast<int4 *>(cursor + lo + k) = make_int4(bg[k], bg[k + 1], bg[k + 2], bg[k + 3]);
        } else {
#pragma unroll
            for (int k = 0; k < TS_PER; k++)
                if (lo + k < nt) {
                    ranges[lo + k] = make_int2(bg[k], bg[k] + cnt[k]);
                    cursor[lo + k] = bg[k];
                }
        }
        carry_d += td;
        carry_c = min(carry_c + tc, TS_SAT);
    }
    const long long total = (long long)carry_c;  // (TS_SAT: at least 2^31 - 1 pairs, more than any capacity)
    const bool ok = total <= cap && carry_c < TS_SAT;
    if (tid == 0) {
        *reinterpret_cast<long long *>(misc + MISC_TOTAL) = total;
        if (!ok) *reinterpret_cast<int *>(misc + MISC_STATUS) |= 1;
        *reinterpret_cast<long long *>(misc + MISC_NEFF) = ok ? total : 0;
    }
    if (!ok) {
        __syncthreads();  // (after every thread's writes above)
        for (long long i = tid; i < nt; i += TS_THREADS) ranges[i] = make_int2(0, 0);
        if (tid == 0) *reinterpret_cast<int *>(misc + MISC_NDEEP) = 0;
    }
}

// Every pair of the call placed at its tile's cursor.  Splat block j (256 splats, the preprocessing block)
// is shared by `parts` scatter blocks, part p taking pairs [min(p*c, tot_j), min((p+1)*c, tot_j)) of the
// block's pairs in splat order, c = ceil(tot_j / parts).  A block works in chunks of SC_CHUNK pairs: each
// thread lists its own splat's pairs of the chunk (tile ids stepped along the rectangle's rows, one
// division per splat and chunk), then every pair is counted per tile in a shared-memory hash table (the
// rank of each pair inside its tile's group), each tile's group is reserved with ONE global atomic, and
// the pairs are written.  Deep tiles (a coarse octave tile under a thousand splats of neighbouring encoder
// cells) otherwise serialise on their cursor.
#define SC_CHUNK 2048
#define SC_HASH 4096  // >= 2 * SC_CHUNK: a probe sequence always ends
__global__ void __launch_bounds__(256) k_scatter(RenderGeom G, const int4 *__restrict__ meta,
                                                 const int *__restrict__ counts, int parts,
                                                 int *__restrict__ cursor, int *__restrict__ vals,
                                                 const unsigned char *__restrict__ misc) {
    __shared__ int wsum[8];
    __shared__ int soff[257];
    __shared__ int4 smeta[256];
    __shared__ int hkey[SC_HASH];
    __shared__ int hval[SC_HASH];               // per tile: pairs in the chunk, then their global start
    __shared__ int ptile[SC_CHUNK];             // per pair: its tile, then (hash slot | rank << 16)
    __shared__ unsigned char psplat[SC_CHUNK];  // per pair: splat of the block
    // after a capacity overflow (k_tile_scan) nothing is scattered
    if (*reinterpret_cast<const int *>(misc + MISC_STATUS) != 0) return;
    const int tid = threadIdx.x;
    const int j = blockIdx.x / parts, part = blockIdx.x - j * parts;
    const long long s0 = (long long)j * 256;
    const long long s = s0 + tid;
    int c = 0;
    int4 mt = make_int4(0, 1, 1, 0);
    if (s < (long long)G.B * G.N) {
        c = counts[s];
        mt = meta[s];
    }
    int tot;
    const int off = block_excl_scan<256>(c, wsum, &tot);
    soff[tid] = off;
    smeta[tid] = mt;
    if (tid == 0) soff[256] = tot;
    __syncthreads();
    const int chunk = (tot + parts - 1) / parts;
    const int e_lo = min(part * chunk, tot), e_hi = min(e_lo + chunk, tot);
    const long long cap = G.cap;
    for (int c0 = e_lo; c0 < e_hi; c0 += SC_CHUNK) {  // block-uniform
        const int n = min(SC_CHUNK, e_hi - c0);
        // a table of the next power of two >= 2n slots (at least 64): short chunks clear a short table
        const int hbits = max(6, 32 - __clz(2 * n - 1));  // <= 12 (n <= SC_CHUNK)
        const int hsize = 1 << hbits;
        for (int i = tid; i < hsize; i += 256) {
            hkey[i] = -1;
            hval[i] = 0;
        }
        {
            // this thread's splat: its pairs [e0, e1) of the chunk, row by row of its tile rectangle
            const int e0 = max(soff[tid], c0), e1 = min(soff[tid + 1], c0 + n);
            if (e0 < e1) {
                const int4 m = smeta[tid];
                const int w = m.y & 0xffffff;
                const int r = e0 - soff[tid];
                const int q = r / w;
                int col = r - q * w, rowbase = m.x + q * m.z;
                for (int e = e0; e < e1; e++) {
                    ptile[e - c0] = rowbase + col;
                    psplat[e - c0] = (unsigned char)tid;
                    if (++col == w) {
                        col = 0;
                        rowbase += m.z;
                    }
                }
            }
        }
        __syncthreads();
        for (int jj = tid; jj < n; jj += 256) {
            const int tile = ptile[jj];
            unsigned h = ((unsigned)tile * 2654435761u) >> (32 - hbits);
            for (int probe = 0; probe < hsize; probe++) {
                const int k = atomicCAS(&hkey[h], -1, tile);
                if (k == -1 || k == tile) break;
                h = (h + 1) & (unsigned)(hsize - 1);
            }
            ptile[jj] = (int)h | (atomicAdd(&hval[h], 1) << 16);
        }
        __syncthreads();
        {
            // every slot's cursor atomic issued before any result is used (up to 16 in flight per thread)
            constexpr int HJ = SC_HASH / 256;
            int res[HJ];
#pragma unroll
            for (int jj = 0; jj < HJ; jj++) {
                const int i = tid + jj * 256;
                res[jj] = 0;
                if (i < hsize) {
                    const int k = hkey[i];
                    if (k >= 0) res[jj] = atomicAdd(cursor + k, hval[i]);
                }
            }
#pragma unroll
            for (int jj = 0; jj < HJ; jj++) {
                const int i = tid + jj * 256;
                if (i < hsize && hkey[i] >= 0) hval[i] = res[jj];
            }
        }
        __syncthreads();
        for (int jj = tid; jj < n; jj += 256) {
            const int sr = ptile[jj];
            const int pos = hval[sr & 0xffff] + (sr >> 16);
            if (pos >= 0 && pos < cap) vals[pos] = (int)(s0 + psplat[jj]);  // (always: the counts bound the cursors)
        }
        __syncthreads();
    }
}

// ----------------------------------------------------------------------------------------------------
// forward: per-tile field sums (render_triton.py:423-517 with FIELDS=True)

__device__ __forceinline__ int group_of_tile(const RenderGeom &G, int lt) {
    int g = 0;
#pragma unroll
    for (int k = 0; k < GS_MAX_GROUPS; k++)
        if (k < G.ngroups && lt >= G.g[k].tile_off && lt < G.g[k].tile_off + G.g[k].ntx * G.g[k].nty) g = k;
    return g;
}

__device__ __forceinline__ void renorm(float &P, int &E) {
    int bits = __float_as_int(P);
    E += ((bits >> 23) & 0xff) - 126;
    P = __int_as_float((bits & 0x807fffff) | 0x3f000000);
}

// One splat record of opacity 0: composites to nothing (pads a batch to a multiple of 8).
__device__ __forceinline__ SplatRec null_rec() {
    SplatRec z;
    z.a = make_float4(0.f, 0.f, 0.f, 0.f);
    z.b = make_float4(0.f, 0.f, 0.f, -INFINITY);  // log2 opacity: alpha = 2^-inf = 0
    z.c = make_float4(0.f, 0.f, 0.f, 0.f);
    return z;
}

// Composite the staged records into the lane's PPL pixels, all in one column (x terms once per splat), the
// two half-warps on alternate records: half h takes sr[h], sr[h + 2], ... (nb even: blocks of 16 records
// unrolled, each half renormalising after its 8, then the batch's tail of fewer than 8 per half).  alpha = min(2^(log2 op - u^2 - v^2), 1 - 1e-4) and the
// weight sums (w = alpha / (1 - alpha) for odds).  Alpha mode keeps the running product P of (1 - alpha);
// odds mode forms the weight without alpha itself: r = 2^(u^2 + v^2 - log2 op) = 1 / alpha, w = 1 / (r - 1)
// with r - 1 clamped below at (1 - AMAX) / AMAX (exactly the clamped alpha's odds), and keeps
// P = prod (1 + w) = 1 / prod (1 - alpha) instead -- one multiply per pixel-pair less.  Both products are
// renormalised every 8 splats (P stays within 2^+-128: at most 1e4^8 growth or 1e-32 decay in between).
#define GS_ODDS_TMIN ((1.0f - GS_ALPHA_MAX) / GS_ALPHA_MAX)
template <int PPL, bool ODDS>
__device__ __forceinline__ void fields_sweep16h(const SplatRec *__restrict__ sr, int nb, int h, const float (&py)[PPL],
                                                float pxl, float (&P)[PPL], int (&E)[PPL], float (&Sw)[PPL],
                                                float (&S0)[PPL], float (&S1)[PPL], float (&S2)[PPL]) {
    auto one = [&](int k) {
        const SplatRec &r = sr[k];
        const float4 A = r.a, Bv = r.b, Cv = r.c;
        const float dx = pxl - A.y;
        const float ux = A.w * dx, vx = Bv.y * dx;
#pragma unroll
        for (int j = 0; j < PPL; j++) {
            const float dy = py[j] - A.x;
            const float u = fmaf(A.z, dy, ux);
            const float v = fmaf(Bv.x, dy, vx);
            float w;
            if (ODDS) {
                const float narg = fmaf(u, u, fmaf(v, v, -Bv.w));
                w = gs_rcp(fmaxf(gs_ex2(narg) - 1.0f, GS_ODDS_TMIN));
                P[j] = fmaf(P[j], w, P[j]);
            } else {
                const float arg = fmaf(-u, u, fmaf(-v, v, Bv.w));
                w = fminf(gs_ex2(arg), GS_ALPHA_MAX);
                P[j] *= 1.0f - w;
            }
            Sw[j] += w;
            S0[j] = fmaf(w, Cv.x, S0[j]);
            S1[j] = fmaf(w, Cv.y, S1[j]);
            S2[j] = fmaf(w, Cv.z, S2[j]);
        }
    };
    int i = 0;
    for (; i + 16 <= nb; i += 16) {
#pragma unroll
        for (int ii = 0; ii < 8; ii++) one(i + 2 * ii + h);
#pragma unroll
        for (int j = 0; j < PPL; j++) renorm(P[j], E[j]);
    }
    if (i < nb) {
        // the batch's last (nb - i) / 2 < 8 records of each half (nb even)
#pragma unroll 1
        for (int k = i + h; k < nb; k += 2) one(k);
#pragma unroll
        for (int j = 0; j < PPL; j++) renorm(P[j], E[j]);
    }
}

// Stage the records [base, base + 32) of a warp's list (splat ids ids[0, n)) in sr, padded with null
// records to a multiple of 8; the next batch is fetched into `nxt` meanwhile.  Returns the padded count.
template <int PAD = 8>
__device__ __forceinline__ int stage_batch(SplatRec *__restrict__ sr, SplatRec &nxt, const SplatRec *__restrict__ rec,
                                           const int *__restrict__ ids, int base, int n, int lane) {
    const int nb = min(32, n - base), nb8 = (nb + PAD - 1) & ~(PAD - 1);
    if (lane < nb) sr[lane] = nxt;
    else if (lane < nb8) sr[lane] = null_rec();
    __syncwarp();
    const int kb = base + 32 + lane;
    if (kb < n) nxt = rec[ids[kb]];
    return nb8;
}

// (1, 2 and 4 tiles per CTA measured within 1% of each other at four images per launch)
#define FW_W8_WPB 4
// TILE 8, binned modes: one WARP per tile (FW_W8_WPB tiles per CTA), 2 pixels per lane in one column, so there
// is no cross-warp reduction and one set-up per tile and lane; each lane writes its pixels' five sums.
// Tiles with more than FW_DEEP pairs are left to k_fields_deep8.
template <bool ODDS, int WPB>
__global__ void __launch_bounds__(WPB * 32) k_fields_w8(RenderGeom G, const SplatRec *__restrict__ rec,
                                                        const int2 *__restrict__ ranges, const int *__restrict__ vals,
                                                        float *__restrict__ fields, int nt) {
    __shared__ SplatRec srec[WPB][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = lane >> 4, hl = lane & 15;  // half-warp; pixels (column hl & 7, rows (hl >> 3) + 2j)
    const int gt = blockIdx.x * WPB + warp;
    if (gt >= nt) return;  // (warp-uniform; the kernel synchronises warps only)
    const int2 rg = ranges[gt];  // empty tile: begin == end
    const int p0 = rg.y > rg.x ? rg.x : 0;
    const int n = rg.y > rg.x ? rg.y - rg.x : 0;
    if (n > FW_DEEP) return;
    const int b = gt / G.tiles_per_image;
    const int lt = gt - b * G.tiles_per_image;
    const int g = group_of_tile(G, lt);
    const int Hg = G.g[g].H, Wg = G.g[g].W, ntx = G.g[g].ntx;
    const int t = lt - G.g[g].tile_off;
    const int tx = t % ntx, ty = t / ntx;
    float py[4];
#pragma unroll
    for (int j = 0; j < 4; j++) py[j] = __fdiv_rn((float)(ty * 8 + (hl >> 3) + 2 * j) + 0.5f, (float)Hg);
    const float pxl = __fdiv_rn((float)(tx * 8 + (hl & 7)) + 0.5f, (float)Wg);
    float P[4] = {1.f, 1.f, 1.f, 1.f}, Sw[4] = {0.f, 0.f, 0.f, 0.f}, S0[4] = {0.f, 0.f, 0.f, 0.f},
          S1[4] = {0.f, 0.f, 0.f, 0.f}, S2[4] = {0.f, 0.f, 0.f, 0.f};
    int E[4] = {0, 0, 0, 0};
    const int *ids = vals + p0;
    SplatRec nxt;
    if (lane < n) nxt = rec[ids[lane]];
    for (int base = 0; base < n; base += 32) {
        const int nb2 = stage_batch<2>(srec[warp], nxt, rec, ids, base, n, lane);
        fields_sweep16h<4, ODDS>(srec[warp], nb2, h, py, pxl, P, E, Sw, S0, S1, S2);
        __syncwarp();
    }
    // lanes l and l + 16 hold the same pixels: the halves' sums combine (log form for the transmittance)
    float *fb = fields + (long long)b * G.fld_per_image + G.g[g].fld_off;
    const long long plane = (long long)Hg * Wg;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        renorm(P[j], E[j]);
        float sl = __logf(P[j]) + (float)E[j] * GS_LN2;
        if (ODDS) sl = -sl;  // P = 1 / transmittance
        sl += __shfl_xor_sync(0xffffffffu, sl, 16);
        const float sw = Sw[j] + __shfl_xor_sync(0xffffffffu, Sw[j], 16);
        const float s0 = S0[j] + __shfl_xor_sync(0xffffffffu, S0[j], 16);
        const float s1 = S1[j] + __shfl_xor_sync(0xffffffffu, S1[j], 16);
        const float s2 = S2[j] + __shfl_xor_sync(0xffffffffu, S2[j], 16);
        const int yp = ty * 8 + (hl >> 3) + 2 * j, xp = tx * 8 + (hl & 7);
        if (h == 0 && yp < Hg && xp < Wg) {
            float *f = fb + (long long)yp * Wg + xp;
            f[0] = sl;
            f[plane] = sw;
            f[2 * plane] = s0;
            f[3 * plane] = s1;
            f[4 * plane] = s2;
        }
    }
}

// TILE 8 deep tiles (more than FW_DEEP pairs, listed by k_tile_scan): a persistent grid over the list,
// FW_DEEP_NW warps per tile splitting its list (half-warps on alternate splats, 4 pixels per lane as in
// k_fields_w8), combined in shared memory in fixed warp order.  The encoder's internal coarse render puts
// ~1,250 splats on each of its busy tiles.
#define FW_DEEP_NW 8
template <bool ODDS>
__global__ void __launch_bounds__(FW_DEEP_NW * 32) k_fields_deep8(RenderGeom G, const SplatRec *__restrict__ rec,
                                                                 const int2 *__restrict__ ranges,
                                                                 const int *__restrict__ vals,
                                                                 const int *__restrict__ dlist,
                                                                 const unsigned char *__restrict__ misc,
                                                                 float *__restrict__ fields) {
    constexpr int NW = FW_DEEP_NW;
    __shared__ SplatRec srec[NW][32];
    __shared__ float red[NW][5][64];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = lane >> 4, hl = lane & 15;
    const int nwork = *reinterpret_cast<const volatile int *>(misc + MISC_NDEEP);
    for (int wi = blockIdx.x; wi < nwork; wi += gridDim.x) {
        const int gt = dlist[wi];
        const int2 rg = ranges[gt];
        const int p0 = rg.x, n = rg.y - rg.x;  // (> FW_DEEP: listed tiles are not empty)
        const int b = gt / G.tiles_per_image;
        const int lt = gt - b * G.tiles_per_image;
        const int g = group_of_tile(G, lt);
        const int Hg = G.g[g].H, Wg = G.g[g].W, ntx = G.g[g].ntx;
        const int t = lt - G.g[g].tile_off;
        const int tx = t % ntx, ty = t / ntx;
        float py[4];
#pragma unroll
        for (int j = 0; j < 4; j++) py[j] = __fdiv_rn((float)(ty * 8 + (hl >> 3) + 2 * j) + 0.5f, (float)Hg);
        const float pxl = __fdiv_rn((float)(tx * 8 + (hl & 7)) + 0.5f, (float)Wg);
        float P[4] = {1.f, 1.f, 1.f, 1.f}, Sw[4] = {0.f, 0.f, 0.f, 0.f}, S0[4] = {0.f, 0.f, 0.f, 0.f},
              S1[4] = {0.f, 0.f, 0.f, 0.f}, S2[4] = {0.f, 0.f, 0.f, 0.f};
        int E[4] = {0, 0, 0, 0};
        const int s_lo = (int)(((long long)n * warp) / NW), s_hi = (int)(((long long)n * (warp + 1)) / NW);
        const int *ids = vals + p0 + s_lo;
        const int m = s_hi - s_lo;
        SplatRec nxt;
        if (lane < m) nxt = rec[ids[lane]];
        for (int base = 0; base < m; base += 32) {
            const int nb2 = stage_batch<2>(srec[warp], nxt, rec, ids, base, m, lane);
            fields_sweep16h<4, ODDS>(srec[warp], nb2, h, py, pxl, P, E, Sw, S0, S1, S2);
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            renorm(P[j], E[j]);
            float sl = __logf(P[j]) + (float)E[j] * GS_LN2;
            if (ODDS) sl = -sl;  // P = 1 / transmittance
            sl += __shfl_xor_sync(0xffffffffu, sl, 16);
            const float sw = Sw[j] + __shfl_xor_sync(0xffffffffu, Sw[j], 16);
            const float s0 = S0[j] + __shfl_xor_sync(0xffffffffu, S0[j], 16);
            const float s1 = S1[j] + __shfl_xor_sync(0xffffffffu, S1[j], 16);
            const float s2 = S2[j] + __shfl_xor_sync(0xffffffffu, S2[j], 16);
            if (h == 0) {
                const int q = ((hl >> 3) + 2 * j) * 8 + (hl & 7);
                red[warp][0][q] = sl;
                red[warp][1][q] = sw;
                red[warp][2][q] = s0;
                red[warp][3][q] = s1;
                red[warp][4][q] = s2;
            }
        }
        __syncthreads();
        float *fb = fields + (long long)b * G.fld_per_image + G.g[g].fld_off;
        const long long plane = (long long)Hg * Wg;
        for (int i = threadIdx.x; i < 5 * 64; i += NW * 32) {
            const int c = i >> 6, pq = i & 63;
            const int yp = ty * 8 + (pq >> 3), xp = tx * 8 + (pq & 7);
            float sacc = 0.f;
#pragma unroll
            for (int w = 0; w < NW; w++) sacc += red[w][c][pq];
            if (yp < Hg && xp < Wg) fb[c * plane + (long long)yp * Wg + xp] = sacc;
        }
        __syncthreads();  // (srec and red are reused by the next listed tile)
    }
}

// Generic form (TILE 4 and 16, and the dense EXACT mode): one CTA of NW warps per tile, the warps
// splitting the tile's list.
template <int TILE, int NW, bool ODDS>
__global__ void __launch_bounds__(NW * 32) k_fields_fwd(RenderGeom G, const SplatRec *__restrict__ rec,
                                                        const int2 *__restrict__ ranges,
                                                        const int *__restrict__ vals, float *__restrict__ fields) {
    constexpr int NPIX = TILE * TILE;
    constexpr int PPL = NPIX >= 32 ? NPIX / 32 : 1;
    __shared__ SplatRec srec[NW][32];
    __shared__ float red[NW][5][NPIX];
    const int gt = blockIdx.x;
    const int b = gt / G.tiles_per_image;
    const int lt = gt - b * G.tiles_per_image;
    const int g = group_of_tile(G, lt);
    const int Hg = G.g[g].H, Wg = G.g[g].W, ntx = G.g[g].ntx;
    const int t = lt - G.g[g].tile_off;
    const int tx = t % ntx, ty = t / ntx;
    int p0, p1;
    const bool dense = G.mode == GS_MODE_EXACT;
    if (dense) {
        p0 = 0;
        p1 = G.N;
    } else {
        const int2 rg = ranges[gt];  // empty tile: begin == end
        p0 = rg.y > rg.x ? rg.x : 0;
        p1 = rg.y > rg.x ? rg.y : 0;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the PPL pixels of a lane share one column (32 is a multiple of TILE), so the x terms of the
    // quadratic form are computed once per splat and lane
    static_assert(NPIX < 32 || 32 % TILE == 0, "lane pixels must share a column");
    float py[PPL];
#pragma unroll
    for (int j = 0; j < PPL; j++) {
        int q = lane + 32 * j;
        py[j] = __fdiv_rn((float)(ty * TILE + q / TILE) + 0.5f, (float)Hg);
    }
    const float pxl = __fdiv_rn((float)(tx * TILE + lane % TILE) + 0.5f, (float)Wg);
    float P[PPL], Sw[PPL], S0[PPL], S1[PPL], S2[PPL];
    int E[PPL];
#pragma unroll
    for (int j = 0; j < PPL; j++) {
        P[j] = 1.0f; E[j] = 0; Sw[j] = 0.f; S0[j] = 0.f; S1[j] = 0.f; S2[j] = 0.f;
    }
    const int n = p1 - p0;
    // one splat at the lane's PPL pixels; the weight form (alpha, odds by rcp, odds by series for dead
    // splats) is chosen once per splat; the record is the same for every lane, and the warp vote makes
    // that branch uniform for the compiler too
    auto step = [&](const SplatRec &r) {
        const float4 A = r.a, Bv = r.b, Cv = r.c;
        const float dx = pxl - A.y;
        const float ux = A.w * dx, vx = Bv.y * dx;
        auto body = [&](auto weight) {
#pragma unroll
            for (int j = 0; j < PPL; j++) {
                float dy = py[j] - A.x;
                float u = fmaf(A.z, dy, ux);
                float v = fmaf(Bv.x, dy, vx);
                float arg = fmaf(-u, u, fmaf(-v, v, Bv.w));
                float a = fminf(gs_ex2(arg), GS_ALPHA_MAX);
                float om = 1.0f - a;
                P[j] *= om;
                float w = weight(a, om);
                Sw[j] += w;
                S0[j] = fmaf(w, Cv.x, S0[j]);
                S1[j] = fmaf(w, Cv.y, S1[j]);
                S2[j] = fmaf(w, Cv.z, S2[j]);
            }
        };
        if (!ODDS) body([](float a, float) { return a; });
        else if (__all_sync(0xffffffffu, Cv.w != 0.0f))
            body([](float a, float) { return a * fmaf(a, fmaf(a, fmaf(a, 1.0f, 1.0f), 1.0f), 1.0f); });
        else body([](float a, float om) { return a * gs_rcp(om); });
    };
    // warp w takes the w-th quarter of the tile's list (even split: short lists keep all warps busy), in
    // batches of 32 records; the next batch is fetched into registers while the current one is composited
    const int s_lo = (int)(((long long)n * warp) / NW), s_hi = (int)(((long long)n * (warp + 1)) / NW);
    SplatRec nxt;
    int kb = s_lo + lane;
    if (kb < s_hi) nxt = rec[dense ? b * G.N + kb : vals[p0 + kb]];
    for (int base = s_lo; base < s_hi; base += 32) {
        if (base + lane < s_hi) srec[warp][lane] = nxt;
        __syncwarp();
        kb = base + 32 + lane;
        if (kb < s_hi) nxt = rec[dense ? b * G.N + kb : vals[p0 + kb]];
        const int nb = min(32, s_hi - base);
        int i = 0;
        // (1 - a) >= 1e-4, so 8 factors stay normal in fp32: renormalise after every 8 splats
        for (; i + 8 <= nb; i += 8) {
#pragma unroll
            for (int ii = 0; ii < 8; ii++) step(srec[warp][i + ii]);
#pragma unroll
            for (int j = 0; j < PPL; j++) renorm(P[j], E[j]);
        }
        for (; i < nb; ++i) step(srec[warp][i]);
#pragma unroll
        for (int j = 0; j < PPL; j++) renorm(P[j], E[j]);
        __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < PPL; j++) {
        int q = lane + 32 * j;
        if (q < NPIX) {
            red[warp][0][q] = logf(P[j]) + (float)E[j] * GS_LN2;
            red[warp][1][q] = Sw[j];
            red[warp][2][q] = S0[j];
            red[warp][3][q] = S1[j];
            red[warp][4][q] = S2[j];
        }
    }
    __syncthreads();
    float *fb = fields + (long long)b * G.fld_per_image + G.g[g].fld_off;
    const long long plane = (long long)Hg * Wg;
    for (int q = threadIdx.x; q < 5 * NPIX; q += NW * 32) {
        int c = q / NPIX, pq = q - c * NPIX;
        int yp = ty * TILE + pq / TILE, xp = tx * TILE + pq % TILE;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) s += red[w][c][pq];
        if (yp < Hg && xp < Wg) fb[c * plane + (long long)yp * Wg + xp] = s;
    }
}

// ----------------------------------------------------------------------------------------------------
// bilinear upsample with torch's align_corners=False source-index rule

__device__ __forceinline__ void lin_index_s(int d, int in_size, float scale, int &i0, int &i1, float &l0, float &l1) {
    float src = __fsub_rn(__fmul_rn(scale, __fadd_rn((float)d, 0.5f)), 0.5f);
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

__device__ __forceinline__ void lin_index(int d, int in_size, int out_size, int &i0, int &i1, float &l0, float &l1) {
    float scale = __fdiv_rn((float)in_size, (float)out_size);
    float src = __fsub_rn(__fmul_rn(scale, __fadd_rn((float)d, 0.5f)), 0.5f);
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

__device__ __forceinline__ bool group_native(const RenderGeom &G, int g) { return G.g[g].H == G.H && G.g[g].W == G.W; }

// S[0..4] = the five raw sums at native pixel (y, x) of image b: every present group's field, bilinearly
// upsampled to native resolution (torch align_corners=False), added in the reference's order
// (render_triton.py:959-972, 914-916).
__device__ __forceinline__ void gather_sums(const RenderGeom &G, const float *__restrict__ fields,
                                            const int *__restrict__ gsplats, int b, int y, int x, float S[5]) {
    // y is uniform over the block (one native row per block), so the row weights of each group are
    // computed once in uniform registers; offsets are 32-bit inside one image's field block
#pragma unroll
    for (int c = 0; c < 5; c++) S[c] = 0.f;
    const float *fimg = fields + (long long)b * G.fld_per_image;
#pragma unroll
    for (int k = 0; k < GS_MAX_GROUPS; k++) {
        if (k >= G.ngroups) break;
        const int g = G.order[k];
        if (gsplats[b * G.ngroups + g] == 0) continue;
        const float *f = fimg + G.g[g].fld_off;
        const int Hg = G.g[g].H, Wg = G.g[g].W;
        const int plane = Hg * Wg;
        if (Hg == G.H && Wg == G.W) {
            const int p = y * Wg + x;
#pragma unroll
            for (int c = 0; c < 5; c++) S[c] += f[c * plane + p];
        } else {
            int y0, y1, x0, x1;
            float h0, h1, w0, w1;
            lin_index_s(y, Hg, G.g[g].up_sy, y0, y1, h0, h1);
            lin_index_s(x, Wg, G.g[g].up_sx, x0, x1, w0, w1);
            const int r0 = y0 * Wg, r1 = y1 * Wg;
#pragma unroll
            for (int c = 0; c < 5; c++) {
                const float *fc = f + c * plane;
                S[c] += h0 * (w0 * fc[r0 + x0] + w1 * fc[r0 + x1]) + h1 * (w0 * fc[r1 + x0] + w1 * fc[r1 + x1]);
            }
        }
    }
}

// one native pixel per thread, one native row per block row (grid = (ceil(W / 128), band rows, B)): sum
// the present groups' fields and composite (render_triton.py:976-979)
__global__ void __launch_bounds__(128) k_composite(RenderGeom G, const float *__restrict__ fields,
                                                   const int *__restrict__ gsplats, const float *__restrict__ bg,
                                                   float *__restrict__ out) {
    const int b = blockIdx.z;
    const int y = G.y0 + blockIdx.y;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= G.W) return;
    const long long P = (long long)G.H * G.W;
    const long long p = (long long)y * G.W + x;
    float S[5];
    gather_sums(G, fields, gsplats, b, y, x, S);
    float asum = fmaxf(S[1], 1e-8f);
    float T = expf(S[0]);
    float *ob = out + (long long)b * G.C * P;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        if (c < G.C) {
            float fg = S[2 + c] / asum;
            ob[c * P + p] = (1.0f - T) * fg + T * bg[b * G.C + c];
        }
    }
}

// One upsampled group's contribution at the four pixels x0..x0+3 of a row (x0 % 4 == 0) for an exact
// 1/2^K column scale (W = Wg << K, K >= 1).  The pixels' column taps then fall in NC source columns, a fixed
// pattern per K: K = 1 uses columns (2m-1 .. 2m+2) of x0 = 4m, taps at slots (0,1) (1,2) (1,2) (2,3);
// K = 2 columns (m-1 .. m+1), slots (0,1) (0,1) (1,2) (1,2); K >= 3 the two taps of pixel x0 for all four.
// Columns are loaded clamped to the plane, so at a border the slot holds the same column as its
// neighbour while lin_index_s gives that pixel the weights (1, 0) or a tap pair with equal columns: every
// pixel gets gather_sums' value with the same taps and weights (the row blend of each source column is
// formed first, so the rounding differs from gather_sums' column-then-row order by an ulp or so).
template <int K>
__device__ __forceinline__ void up_group4(const float *__restrict__ f, int plane, int Wg, float usx, int ra, int rb,
                                          float h0, float h1, int x0, float (&S)[5][4]) {
    constexpr int NC = K == 1 ? 4 : (K == 2 ? 3 : 2);
    // lin_index_s's weights without its index clamps: with usx = 2^-K the source coordinate
    // (x + 0.5) usx - 0.5 is exact, stays below Wg - 1/2 (so its floor is a valid column) and is clamped at 0
    float w0[4], w1[4];
    int first = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float src = fmaxf(__fsub_rn(__fmul_rn(usx, __fadd_rn((float)(x0 + j), 0.5f)), 0.5f), 0.0f);
        const float fl = floorf(src);
        w1[j] = src - fl;
        w0[j] = 1.0f - w1[j];
        if (j == 0) first = (int)fl;
    }
    const int cl = K >= 3 ? first : (x0 >> K) - 1;
    int col[NC];
#pragma unroll
    for (int s = 0; s < NC; s++) col[s] = min(max(cl + s, 0), Wg - 1);
    // separable: the row blend of each source column once, then two FMAs per pixel (the same bilinear
    // value as gather_sums' row-then-column order up to float rounding)
#pragma unroll
    for (int c = 0; c < 5; c++) {
        const float *fc = f + c * plane;
        float vc[NC];
#pragma unroll
        for (int s = 0; s < NC; s++) vc[s] = fmaf(h1, __ldg(fc + rb + col[s]), h0 * __ldg(fc + ra + col[s]));
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int s0 = K == 1 ? (j + 1) >> 1 : (K == 2 ? j >> 1 : 0);
            S[c][j] = fmaf(w1[j], vc[s0 + 1], fmaf(w0[j], vc[s0], S[c][j]));
        }
    }
}

// k_composite with four neighbouring pixels of a row per thread (W % 4 == 0, output 16-byte aligned):
// float4 loads of a native-resolution group's fields and float4 stores, exact power-of-two groups through
// up_group4 (2-4 source columns per four pixels instead of 2 per pixel), others per pixel as gather_sums.
// grid = (ceil(W / 256), band rows, B), 64 threads.
__global__ void __launch_bounds__(64) k_composite4(RenderGeom G, const float *__restrict__ fields,
                                                   const int *__restrict__ gsplats, const float *__restrict__ bg,
                                                   float *__restrict__ out) {
    const int b = blockIdx.z;
    const int y = G.y0 + blockIdx.y;
    const int x0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (x0 >= G.W) return;
    float S[5][4];
#pragma unroll
    for (int c = 0; c < 5; c++)
#pragma unroll
        for (int j = 0; j < 4; j++) S[c][j] = 0.f;
    const float *fimg = fields + (long long)b * G.fld_per_image;
#pragma unroll 1
    for (int k = 0; k < G.ngroups; k++) {
        const int g = G.order[k];
        if (gsplats[b * G.ngroups + g] == 0) continue;
        const float *f = fimg + G.g[g].fld_off;
        const int Hg = G.g[g].H, Wg = G.g[g].W;
        const int plane = Hg * Wg;
        if (Hg == G.H && Wg == G.W) {
            const int p = y * Wg + x0;
            if ((reinterpret_cast<uintptr_t>(f) & 15) == 0) {
#pragma unroll
                for (int c = 0; c < 5; c++) {
                    const float4 v = __ldg(reinterpret_cast<const float4 *>(f + c * plane + p));
                    S[c][0] += v.x;
                    S[c][1] += v.y;
                    S[c][2] += v.z;
                    S[c][3] += v.w;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 5; c++)
#pragma unroll
                    for (int j = 0; j < 4; j++) S[c][j] += f[c * plane + p + j];
            }
            continue;
        }
        int y0, y1;
        float h0, h1;
        lin_index_s(y, Hg, G.g[g].up_sy, y0, y1, h0, h1);
        const int ra = y0 * Wg, rb = y1 * Wg;
        const float usx = G.g[g].up_sx;
        if ((Wg << 1) == G.W) {
            up_group4<1>(f, plane, Wg, usx, ra, rb, h0, h1, x0, S);
        } else if ((Wg << 2) == G.W) {
            up_group4<2>(f, plane, Wg, usx, ra, rb, h0, h1, x0, S);
        } else if (Wg < G.W && (G.W % Wg) == 0 && __popc(G.W / Wg) == 1) {
            up_group4<3>(f, plane, Wg, usx, ra, rb, h0, h1, x0, S);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int xa, xb;
                float w0, w1;
                lin_index_s(x0 + j, Wg, usx, xa, xb, w0, w1);
#pragma unroll
                for (int c = 0; c < 5; c++) {
                    const float *fc = f + c * plane;
                    S[c][j] += h0 * (w0 * fc[ra + xa] + w1 * fc[ra + xb]) + h1 * (w0 * fc[rb + xa] + w1 * fc[rb + xb]);
                }
            }
        }
    }
    float T[4], ra[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        ra[j] = 1.0f / fmaxf(S[1][j], 1e-8f);
        T[j] = expf(S[0][j]);
    }
    const long long P = (long long)G.H * G.W;
    float *ob = out + (long long)b * G.C * P + (long long)y * G.W + x0;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        if (c < G.C) {
            const float bgc = bg[b * G.C + c];
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; j++) o[j] = (1.0f - T[j]) * (S[2 + c][j] * ra[j]) + T[j] * bgc;
            *reinterpret_cast<float4 *>(ob + c * P) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

// fields[b][lo + i] += prior[b][plo + i] for i < n (n % 4 == 0, both offsets multiples of 4): the mapped
// groups when they are consecutive here and in the prior (the octaves k >= 2 of the encoder's final render
// map to the prior's k - 1), one flat float4 pass; grid = (ceil(n / 1024), B)
__global__ void __launch_bounds__(256) k_add_prior_flat(const float *__restrict__ prior, long long prior_per_image,
                                                        long long plo, float *__restrict__ fields,
                                                        long long fld_per_image, long long lo, int n4) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const int b = blockIdx.y;
    const float4 p = reinterpret_cast<const float4 *>(prior + b * prior_per_image + plo)[i];
    float4 *f = reinterpret_cast<float4 *>(fields + b * fld_per_image + lo) + i;
    float4 v = *f;
    v.x += p.x;
    v.y += p.y;
    v.z += p.z;
    v.w += p.w;
    *f = v;
}

// fields of group g += the mapped prior group's fields (every group with prior_off >= 0, all images);
// grid = (texel blocks, groups, images)
__global__ void __launch_bounds__(256) k_add_prior(RenderGeom G, const float *__restrict__ prior,
                                                   long long prior_per_image, float *__restrict__ fields) {
    const GroupGeom &gg = G.g[blockIdx.y];
    if (gg.prior_off < 0) return;
    const long long n = 5LL * gg.H * gg.W;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int b = blockIdx.z;
    fields[(long long)b * G.fld_per_image + gg.fld_off + i] += prior[(long long)b * prior_per_image + gg.prior_off + i];
}

// ----------------------------------------------------------------------------------------------------
// backward

// dS at native resolution from dL/dimage (torch autograd of render_triton.py:976-979; the cull and
// exact paths skip the clamp_min mask, render_triton.py:644-654); bg gradient sum_p g * T.
__global__ void __launch_bounds__(128) k_composite_bwd(RenderGeom G, const float *__restrict__ fields,
                                                       const int *__restrict__ gsplats,
                                                       const float *__restrict__ bg,
                                                       const float *__restrict__ gout, float *__restrict__ Gn,
                                                       float *__restrict__ gbg, int clamp_mask) {
    __shared__ float red[3][4];
    const int b = blockIdx.z;
    const long long P = (long long)G.H * G.W;
    const int y = G.y0 + blockIdx.y;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const long long p = (long long)y * G.W + x;
    float gT[3] = {0.f, 0.f, 0.f};
    if (x < G.W) {
        float S[5];
        gather_sums(G, fields, gsplats, b, y, x, S);
        const float Sl = S[0], Sw = S[1];
        float asum = fmaxf(Sw, 1e-8f);
        float T = expf(Sl);
        float dT = 0.f, dasum = 0.f, dsc[3] = {0.f, 0.f, 0.f};
        const float *gb = gout + (long long)b * G.C * P;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            if (c < G.C) {
                float gc = gb[c * P + p];
                float fg = S[2 + c] / asum;
                dT += gc * (bg[b * G.C + c] - fg);
                float dfg = gc * (1.0f - T);
                dsc[c] = dfg / asum;
                dasum += dfg * fg;
                gT[c] = gc * T;
            }
        }
        float dsw = -dasum / asum;
        if (clamp_mask && !(Sw >= 1e-8f)) dsw = 0.0f;
        float *Gb = Gn + (long long)b * 5 * P;
        Gb[p] = dT * T;
        Gb[P + p] = dsw;
        Gb[2 * P + p] = dsc[0];
        Gb[3 * P + p] = dsc[1];
        Gb[4 * P + p] = dsc[2];
    }
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        float v = gT[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[c][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < 3 && threadIdx.x < G.C) {
        float v = 0.f;
        for (int w = 0; w < 4; w++) v += red[threadIdx.x][w];
        atomicAdd(&gbg[b * 4 + threadIdx.x], v);
    }
}

// Adjoint of the bilinear upsample (align_corners=False) for every coarse group, as two separable passes:
//   X: T[g][c][y][j] = sum_x wx(x, j) * dS[c][y][x]      native rows y of the band, coarse columns j
//   Y: dF[g][c][i][j] = sum_y wy(y, i) * T[g][c][y][j]   coarse rows i
// Each output gathers the O(native/coarse) inputs whose taps touch it, in a fixed order; the deepest
// octaves (upsampling factor 64 and up) give each output a 32-lane team that splits the inputs and reduces
// with shuffles in a fixed tree, so the result is deterministic and the work linear in the image size.
struct AdjPlan {
    long long uD[GS_MAX_GROUPS + 1];                          // direct-gather texel offsets per group
    long long uX[GS_MAX_GROUPS + 1], uY[GS_MAX_GROUPS + 1];  // work-unit offsets per group (multiples of 32)
    long long tOff[GS_MAX_GROUPS];                            // first float of the group's T block (per image)
    long long tPerImage;
    int teamX[GS_MAX_GROUPS], teamY[GS_MAX_GROUPS];
};

__device__ __forceinline__ int adj_group(const long long *off, long long u) {
    int g = -1;
#pragma unroll
    for (int k = 0; k < GS_MAX_GROUPS; k++)
        if (u >= off[k] && u < off[k + 1]) g = k;
    return g;
}

__device__ __forceinline__ void team_reduce5(float acc[5], int team) {
    if (team == 32) {
#pragma unroll
        for (int c = 0; c < 5; c++)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], o);
    }
}

// Shallow groups (upsampling factor <= 8, at most 19 x 19 native taps per texel) gather directly, one
// thread per texel; texels of tiles without pairs are never read by the backward and are skipped, which
// keeps sparsely populated octaves cheap.
__global__ void __launch_bounds__(256) k_adjoint_direct(RenderGeom G, AdjPlan A, const int *__restrict__ gsplats,
                                                        const int2 *__restrict__ ranges, const float *__restrict__ Gn,
                                                        float *__restrict__ gfields) {
    const int b = blockIdx.y;
    const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int g = adj_group(A.uD, u);
    if (g < 0 || gsplats[b * G.ngroups + g] == 0) return;
    const long long q = u - A.uD[g];
    const int Hg = G.g[g].H, Wg = G.g[g].W;
    if (q >= (long long)Hg * Wg) return;
    const int i = (int)(q / Wg), j = (int)(q - (long long)i * Wg);
    const int tile = G.g[g].tile_off + (i / G.tile) * G.g[g].ntx + (j / G.tile);
    const int2 rg = ranges[(long long)b * G.tiles_per_image + tile];
    if (rg.y <= rg.x) return;
    const long long P = (long long)G.H * G.W;
    const float inv_sy = (float)G.H / (float)Hg, inv_sx = (float)G.W / (float)Wg;
    const int ylo = max(G.y0, (int)ceilf((i - 0.5f) * inv_sy - 0.5f) - 1);
    const int yhi = min(G.y1 - 1, (int)floorf((i + 1.5f) * inv_sy - 0.5f) + 1);
    const int xlo = max(0, (int)ceilf((j - 0.5f) * inv_sx - 0.5f) - 1);
    const int xhi = min(G.W - 1, (int)floorf((j + 1.5f) * inv_sx - 0.5f) + 1);
    const float usy = G.g[g].up_sy, usx = G.g[g].up_sx;
    constexpr int MAXW = 20;  // 2 * factor + 3 <= 19 for the groups this kernel takes
    float wx[MAXW];
    const int nx = min(xhi - xlo + 1, MAXW);
#pragma unroll
    for (int t = 0; t < MAXW; t++) {
        wx[t] = 0.f;
        if (t < nx) {
            int x0, x1;
            float w0, w1;
            lin_index_s(xlo + t, Wg, usx, x0, x1, w0, w1);
            wx[t] = (x0 == j ? w0 : 0.f) + (x1 == j ? w1 : 0.f);
        }
    }
    float acc5[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    const float *Gb = Gn + (long long)b * 5 * P;
    for (int y = ylo; y <= yhi; y++) {
        int y0, y1;
        float h0, h1;
        lin_index_s(y, Hg, usy, y0, y1, h0, h1);
        const float wy = (y0 == i ? h0 : 0.f) + (y1 == i ? h1 : 0.f);
        if (wy == 0.f) continue;
        const long long rowp = (long long)y * G.W + xlo;
#pragma unroll
        for (int t = 0; t < MAXW; t++) {
            const float w = wy * wx[t];
            if (t >= nx || w == 0.f) continue;
#pragma unroll
            for (int c = 0; c < 5; c++) acc5[c] += w * Gb[c * P + rowp + t];
        }
    }
    float *gf = gfields + (long long)b * G.fld_per_image + G.g[g].fld_off;
    const long long plane = (long long)Hg * Wg;
#pragma unroll
    for (int c = 0; c < 5; c++) gf[c * plane + q] = acc5[c];
}

__global__ void __launch_bounds__(256) k_adjoint_x(RenderGeom G, AdjPlan A, const int *__restrict__ gsplats,
                                                   const float *__restrict__ Gn, float *__restrict__ T) {
    const int b = blockIdx.y;
    const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int g = adj_group(A.uX, u);
    if (g < 0 || gsplats[b * G.ngroups + g] == 0) return;  // uniform over the warp (groups padded to 32)
    const int team = A.teamX[g];
    const long long local = u - A.uX[g];
    const long long out = local / team;
    const int lt = (int)(local - out * team);
    const int Wg = G.g[g].W;
    const int rows = G.y1 - G.y0;
    if (out >= (long long)rows * Wg) return;  // padding units: whole warps when team == 32
    const int y = G.y0 + (int)(out / Wg), j = (int)(out % Wg);
    const float inv_sx = (float)G.W / (float)Wg;
    const int xlo = max(0, (int)ceilf((j - 0.5f) * inv_sx - 0.5f) - 1);
    const int xhi = min(G.W - 1, (int)floorf((j + 1.5f) * inv_sx - 0.5f) + 1);
    const float usx = G.g[g].up_sx;
    const long long P = (long long)G.H * G.W;
    const float *row = Gn + (long long)b * 5 * P + (long long)y * G.W;
    float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    for (int x = xlo + lt; x <= xhi; x += team) {
        int x0, x1;
        float w0, w1;
        lin_index_s(x, Wg, usx, x0, x1, w0, w1);
        const float w = (x0 == j ? w0 : 0.f) + (x1 == j ? w1 : 0.f);
        if (w == 0.f) continue;
#pragma unroll
        for (int c = 0; c < 5; c++) acc[c] += w * row[c * P + x];
    }
    team_reduce5(acc, team);
    if (lt == 0) {
        float *t = T + (long long)b * A.tPerImage + A.tOff[g];
        const long long plane = (long long)rows * Wg;
#pragma unroll
        for (int c = 0; c < 5; c++) t[c * plane + out] = acc[c];
    }
}

__global__ void __launch_bounds__(256) k_adjoint_y(RenderGeom G, AdjPlan A, const int *__restrict__ gsplats,
                                                   const float *__restrict__ T, float *__restrict__ gfields) {
    const int b = blockIdx.y;
    const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int g = adj_group(A.uY, u);
    if (g < 0 || gsplats[b * G.ngroups + g] == 0) return;
    const int team = A.teamY[g];
    const long long local = u - A.uY[g];
    const long long out = local / team;
    const int lt = (int)(local - out * team);
    const int Hg = G.g[g].H, Wg = G.g[g].W;
    if (out >= (long long)Hg * Wg) return;
    const int i = (int)(out / Wg), j = (int)(out % Wg);
    const float inv_sy = (float)G.H / (float)Hg;
    const int ylo = max(G.y0, (int)ceilf((i - 0.5f) * inv_sy - 0.5f) - 1);
    const int yhi = min(G.y1 - 1, (int)floorf((i + 1.5f) * inv_sy - 0.5f) + 1);
    const float usy = G.g[g].up_sy;
    const int rows = G.y1 - G.y0;
    const long long tplane = (long long)rows * Wg;
    const float *t = T + (long long)b * A.tPerImage + A.tOff[g];
    float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    for (int y = ylo + lt; y <= yhi; y += team) {
        int y0, y1;
        float h0, h1;
        lin_index_s(y, Hg, usy, y0, y1, h0, h1);
        const float w = (y0 == i ? h0 : 0.f) + (y1 == i ? h1 : 0.f);
        if (w == 0.f) continue;
        const long long r = (long long)(y - G.y0) * Wg + j;
#pragma unroll
        for (int c = 0; c < 5; c++) acc[c] += w * t[c * tplane + r];
    }
    team_reduce5(acc, team);
    if (lt == 0) {
        float *gf = gfields + (long long)b * G.fld_per_image + G.g[g].fld_off;
        const long long plane = (long long)Hg * Wg;
#pragma unroll
        for (int c = 0; c < 5; c++) gf[c * plane + out] = acc[c];
    }
}

// one CTA per tile; lane = one (tile, splat) pair looping over the tile's pixels
// (render_triton.py:602-720 with FIELDS=True; the index_add_ of render_triton.py:757-761/803-807
// becomes three 16-byte vector atomics per pair into the per-splat sums).
template <int TILE, int NW, bool ODDS>
__global__ void __launch_bounds__(NW * 32) k_fields_bwd(RenderGeom G, const SplatRec *__restrict__ rec,
                                                        const int2 *__restrict__ ranges,
                                                        const int *__restrict__ vals, const float *__restrict__ Gn,
                                                        const float *__restrict__ gfields,
                                                        float *__restrict__ acc) {
    constexpr int NPIX = TILE * TILE;
    __shared__ float4 dsa[NPIX];
    __shared__ float dsb[NPIX];
    __shared__ float spy[TILE], spx[TILE];
    const int gt = blockIdx.x;
    const int b = gt / G.tiles_per_image;
    const int lt = gt - b * G.tiles_per_image;
    const int g = group_of_tile(G, lt);
    const int Hg = G.g[g].H, Wg = G.g[g].W, ntx = G.g[g].ntx;
    const int t = lt - G.g[g].tile_off;
    const int tx = t % ntx, ty = t / ntx;
    int p0, p1;
    const bool dense = G.mode == GS_MODE_EXACT;
    if (dense) {
        p0 = 0;
        p1 = G.N;
    } else {
        const int2 rg = ranges[gt];  // empty tile: begin == end
        p0 = rg.y > rg.x ? rg.x : 0;
        p1 = rg.y > rg.x ? rg.y : 0;
    }
    if (p1 <= p0) return;
    const float *src;
    long long plane = (long long)Hg * Wg;
    if (group_native(G, g)) src = Gn + (long long)b * 5 * plane;
    else src = gfields + (long long)b * G.fld_per_image + G.g[g].fld_off;
    for (int q = threadIdx.x; q < NPIX; q += NW * 32) {
        int yp = ty * TILE + q / TILE, xp = tx * TILE + q % TILE;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        float v4 = 0.f;
        const bool inband = !group_native(G, g) || (yp >= G.y0 && yp < G.y1);
        if (yp < Hg && xp < Wg && inband) {
            long long p = (long long)yp * Wg + xp;
            v = make_float4(src[p], src[plane + p], src[2 * plane + p], src[3 * plane + p]);
            v4 = src[4 * plane + p];
        }
        dsa[q] = v;
        dsb[q] = v4;
    }
    if (threadIdx.x < TILE) {
        spy[threadIdx.x] = __fdiv_rn((float)(ty * TILE + threadIdx.x) + 0.5f, (float)Hg);
        spx[threadIdx.x] = __fdiv_rn((float)(tx * TILE + threadIdx.x) + 0.5f, (float)Wg);
    }
    __syncthreads();
    const int n = p1 - p0;
    for (int k = threadIdx.x; k < ((n + 31) & ~31); k += NW * 32) {
        if (k >= n) continue;  // whole-warp granularity: tail lanes idle
        const int sid = dense ? b * G.N + k : vals[p0 + k];
        const SplatRec r = rec[sid];
        const float muy = r.a.x, mux = r.a.y, A = r.a.z, Bc = r.a.w;
        const float Cc = r.b.x, D = r.b.y, op = r.b.z;
        const float c0 = r.c.x, c1 = r.c.y, c2 = r.c.z;
        float ux[TILE], vx[TILE];
#pragma unroll
        for (int lx = 0; lx < TILE; lx++) {
            float dx = spx[lx] - mux;
            ux[lx] = Bc * dx;
            vx[lx] = D * dx;
        }
        float Su = 0.f, Sv = 0.f, Suu = 0.f, Svv = 0.f, Suv = 0.f, Sf = 0.f, Sc0 = 0.f, Sc1 = 0.f, Sc2 = 0.f;
        // alpha = min(op f, 1 - 1e-4) with f <= 1: when every splat of the warp has op below the clamp, no
        // pixel clamps and the clamp's compare / select drop out of the loop (CLAMP = false)
        auto sweep = [&](auto clamp_tag) {
            constexpr bool CLAMP = decltype(clamp_tag)::value;
            // rows rolled, columns unrolled: the loop body stays small enough for the instruction cache
#pragma unroll 1
            for (int ly = 0; ly < TILE; ly++) {
                const float dy = spy[ly] - muy;
                const float uy = A * dy, vy = Cc * dy;
#pragma unroll
                for (int lx = 0; lx < TILE; lx++) {
                    const int q = ly * TILE + lx;
                    const float4 d4 = dsa[q];
                    const float dS2 = dsb[q];
                    const float u = uy + ux[lx];
                    const float v = vy + vx[lx];
                    const float f = gs_ex2(-fmaf(u, u, v * v));
                    const float fo = op * f;
                    const float a = CLAMP ? fminf(fo, GS_ALPHA_MAX) : fo;
                    const float om = 1.0f - a;
                    const float rr = gs_rcp(om);
                    const float col_term = fmaf(d4.z, c0, fmaf(d4.w, c1, dS2 * c2));
                    float da, cw;
                    if (ODDS) {
                        da = fmaf(d4.y + col_term, rr, -d4.x) * rr;
                        cw = a * rr;
                    } else {
                        da = fmaf(-d4.x, rr, d4.y + col_term);
                        cw = a;
                    }
                    Sc0 = fmaf(cw, d4.z, Sc0);
                    Sc1 = fmaf(cw, d4.w, Sc1);
                    Sc2 = fmaf(cw, dS2, Sc2);
                    const float dafo = (!CLAMP || fo < GS_ALPHA_MAX) ? da : 0.0f;
                    Sf = fmaf(dafo, f, Sf);
                    const float Gm = dafo * fo;
                    const float Gu = Gm * u, Gv = Gm * v;
                    Su += Gu;
                    Sv += Gv;
                    Suu = fmaf(Gu, u, Suu);
                    Svv = fmaf(Gv, v, Svv);
                    Suv = fmaf(Gu, v, Suv);
                }
            }
        };
        if (__all_sync(__activemask(), op < GS_ALPHA_MAX)) sweep(std::false_type());
        else sweep(std::true_type());
        float *ap = acc + (long long)sid * 12;
        gs_red_add_v4(ap, Su, Sv, Suu, Svv);
        gs_red_add_v4(ap + 4, Suv, Sf, Sc0, Sc1);
        gs_red_add_v4(ap + 8, Sc2, 0.f, 0.f, 0.f);
    }
}

// per-splat chain rule from the 9 sums (u = K*rotated_y/sigma_y, v = K*rotated_x/sigma_x,
// Gm = dL/da * a on unclamped pairs) to the reference's leaf gradients.
__global__ void __launch_bounds__(256) k_finalize(RenderGeom G, const float *__restrict__ ls,
                                                  const float *__restrict__ th, const float *__restrict__ acc,
                                                  const float *__restrict__ gbg_ws, float *__restrict__ g_mu,
                                                  float *__restrict__ g_ls, float *__restrict__ g_col,
                                                  float *__restrict__ g_op, float *__restrict__ g_bg,
                                                  float *__restrict__ g_th) {
    long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s < (long long)G.B * G.C && g_bg) {
        int b = (int)(s / G.C), c = (int)(s - (long long)b * G.C);
        g_bg[s] = gbg_ws[b * 4 + c];
    }
    if (s >= (long long)G.B * G.N) return;
    const float4 a0 = reinterpret_cast<const float4 *>(acc)[s * 3 + 0];
    const float4 a1 = reinterpret_cast<const float4 *>(acc)[s * 3 + 1];
    const float4 a2 = reinterpret_cast<const float4 *>(acc)[s * 3 + 2];
    const float Su = a0.x, Sv = a0.y, Suu = a0.z, Svv = a0.w, Suv = a1.x, Sf = a1.y;
    float2 l = reinterpret_cast<const float2 *>(ls)[s];
    float sy = gs_softplus_eps(l.x), sx = gs_softplus_eps(l.y);
    float cth = 1.0f, sth = 0.0f;
    if (G.has_theta) sincosf(th[s], &sth, &cth);
    const float invK = 1.0f / GS_K, invK2 = invK * invK;
    float gsy = Suu * invK2 / sy;
    float gsx = Svv * invK2 / sx;
    float gmuy = (cth / sy * Su - sth / sx * Sv) * invK;
    float gmux = (sth / sy * Su + cth / sx * Sv) * invK;
    reinterpret_cast<float2 *>(g_mu)[s] = make_float2(gmuy, gmux);
    reinterpret_cast<float2 *>(g_ls)[s] = make_float2(gsy * gs_softplus_grad(l.x), gsx * gs_softplus_grad(l.y));
    g_op[s] = Sf;
    if (G.C > 0) g_col[s * G.C + 0] = a1.z;
    if (G.C > 1) g_col[s * G.C + 1] = a1.w;
    if (G.C > 2) g_col[s * G.C + 2] = a2.x;
    if (G.has_theta && g_th) g_th[s] = -(sx / sy - sy / sx) * Suv * invK2;
}

// ----------------------------------------------------------------------------------------------------
// pixel-list render (render.py:68-87, render_alpha_subsampled): alpha compositing of all N splats of an
// image at P listed pixels (flat indices y*W + x), dense (no binning), alpha mode, autograd of
// render.py:47-65 including the clamp_min(1e-8) mask.  CTA = PT_PIX pixels x one slice of the splats.

#define PT_PIX 64
#define PT_SLICE 2048

__device__ __forceinline__ void point_coords(const long long *__restrict__ px_idx, int P, int W, int H, int b, int p,
                                             float &py, float &px) {
    long long idx = p < P ? px_idx[(long long)b * P + p] : 0;
    long long y = idx / W, x = idx - y * W;
    py = __fdiv_rn((float)y + 0.5f, (float)H);  // ((idx // W) + 0.5) / H as torch computes it
    px = __fdiv_rn((float)x + 0.5f, (float)W);
}

// partial sums (log T, S_w, S_c[3]) of splats [slice*PT_SLICE, ...) at the CTA's pixels:
// part[slice][b][5][P]
template <int NW>
__global__ void __launch_bounds__(NW * 32) k_points_fwd(int N, int H, int W, int P,
                                                        const long long *__restrict__ px_idx,
                                                        const SplatRec *__restrict__ rec, float *__restrict__ part) {
    constexpr int PPL = PT_PIX / 32;
    __shared__ SplatRec srec[NW][32];
    __shared__ float red[NW][5][PT_PIX];
    const int b = blockIdx.z, slice = blockIdx.y;
    const int pbase = blockIdx.x * PT_PIX;
    const int n0 = slice * PT_SLICE, n1 = min(N, n0 + PT_SLICE);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float py[PPL], px[PPL], Pp[PPL], Sw[PPL], S0[PPL], S1[PPL], S2[PPL];
    int E[PPL];
#pragma unroll
    for (int j = 0; j < PPL; j++) {
        point_coords(px_idx, P, W, H, b, pbase + lane + 32 * j, py[j], px[j]);
        Pp[j] = 1.0f; E[j] = 0; Sw[j] = 0.f; S0[j] = 0.f; S1[j] = 0.f; S2[j] = 0.f;
    }
    const SplatRec *rb = rec + (long long)b * N;
    for (int base = n0 + warp * 32; base < n1; base += NW * 32) {
        if (base + lane < n1) srec[warp][lane] = rb[base + lane];
        __syncwarp();
        const int nb = min(32, n1 - base);
        for (int i = 0; i < nb; ++i) {
            const float4 A = srec[warp][i].a, Bv = srec[warp][i].b, Cv = srec[warp][i].c;
#pragma unroll
            for (int j = 0; j < PPL; j++) {
                float dy = py[j] - A.x, dx = px[j] - A.y;
                float u = fmaf(A.z, dy, A.w * dx);
                float v = fmaf(Bv.x, dy, Bv.y * dx);
                float a = fminf(gs_ex2(fmaf(-u, u, fmaf(-v, v, Bv.w))), GS_ALPHA_MAX);
                Pp[j] *= 1.0f - a;
                Sw[j] += a;
                S0[j] = fmaf(a, Cv.x, S0[j]);
                S1[j] = fmaf(a, Cv.y, S1[j]);
                S2[j] = fmaf(a, Cv.z, S2[j]);
            }
            if ((i & 7) == 7) {
#pragma unroll
                for (int j = 0; j < PPL; j++) renorm(Pp[j], E[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < PPL; j++) renorm(Pp[j], E[j]);
        __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < PPL; j++) {
        const int q = lane + 32 * j;
        red[warp][0][q] = logf(Pp[j]) + (float)E[j] * GS_LN2;
        red[warp][1][q] = Sw[j];
        red[warp][2][q] = S0[j];
        red[warp][3][q] = S1[j];
        red[warp][4][q] = S2[j];
    }
    __syncthreads();
    const int B = gridDim.z;
    for (int t = threadIdx.x; t < 5 * PT_PIX; t += NW * 32) {
        const int c = t / PT_PIX, q = t - c * PT_PIX, p = pbase + q;
        if (p >= P) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) v += red[w][c][q];
        part[(((long long)slice * B + b) * 5 + c) * P + p] = v;
    }
}

// fields[b][5][p] = sum over slices (fixed order), then the composite of render.py:47-65:
// out[b][c][p] = (1 - T) * S_c / max(S_w, 1e-8) + T * bg[b][c]
__global__ void __launch_bounds__(256) k_points_composite(int B, int C, int P, int nslices,
                                                          const float *__restrict__ part,
                                                          const float *__restrict__ bg, float *__restrict__ fields,
                                                          float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * P) return;
    const int b = (int)(i / P), p = (int)(i - (long long)b * P);
    float S[5];
#pragma unroll
    for (int c = 0; c < 5; c++) {
        float v = 0.f;
        for (int sl = 0; sl < nslices; sl++) v += part[(((long long)sl * B + b) * 5 + c) * P + p];
        S[c] = v;
        fields[((long long)b * 5 + c) * P + p] = v;
    }
    const float T = expf(S[0]);
    const float asum = fmaxf(S[1], 1e-8f);
#pragma unroll
    for (int c = 0; c < 3; c++)
        if (c < C) out[((long long)b * C + c) * P + p] = (1.0f - T) * (S[2 + c] / asum) + T * bg[b * C + c];
}

// backward: the composite's adjoint for the CTA's pixels (fused), then lane = splat of the slice looping
// over the pixels; the per-splat sums are those of k_fields_bwd, finished by k_finalize.
template <int NW>
__global__ void __launch_bounds__(NW * 32) k_points_bwd(int N, int C, int H, int W, int P,
                                                        const long long *__restrict__ px_idx,
                                                        const SplatRec *__restrict__ rec,
                                                        const float *__restrict__ fields, const float *__restrict__ bg,
                                                        const float *__restrict__ gout, float *__restrict__ acc,
                                                        float *__restrict__ gbg) {
    __shared__ float4 sxy[PT_PIX];  // (py, px, dS_c2, -)
    __shared__ float4 sds[PT_PIX];  // (dS_log, dS_w, dS_c0, dS_c1)
    __shared__ float red[3][NW];
    const int b = blockIdx.z, slice = blockIdx.y;
    const int pbase = blockIdx.x * PT_PIX;
    float gT[3] = {0.f, 0.f, 0.f};
    if (threadIdx.x < PT_PIX) {
        const int q = threadIdx.x, p = pbase + q;
        float py, px;
        point_coords(px_idx, P, W, H, b, p, py, px);
        float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
        float d2 = 0.f;
        if (p < P) {
            float S[5];
#pragma unroll
            for (int c = 0; c < 5; c++) S[c] = fields[((long long)b * 5 + c) * P + p];
            const float Sw = S[1], asum = fmaxf(Sw, 1e-8f), T = expf(S[0]);
            float dT = 0.f, dasum = 0.f, dsc[3] = {0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 3; c++) {
                if (c < C) {
                    const float gc = gout[((long long)b * C + c) * P + p];
                    const float fg = S[2 + c] / asum;
                    dT += gc * (bg[b * C + c] - fg);
                    const float dfg = gc * (1.0f - T);
                    dsc[c] = dfg / asum;
                    dasum += dfg * fg;
                    gT[c] = gc * T;
                }
            }
            const float dsw = Sw >= 1e-8f ? -dasum / asum : 0.0f;  // clamp_min(1e-8) passes no gradient
            d = make_float4(dT * T, dsw, dsc[0], dsc[1]);
            d2 = dsc[2];
        }
        sxy[q] = make_float4(py, px, d2, 0.f);
        sds[q] = d;
    }
    if (slice == 0) {  // the background gradient, once per pixel
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            float v = gT[c];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[c][warp] = v;
        }
    }
    __syncthreads();
    if (slice == 0 && threadIdx.x < 3 && threadIdx.x < C) {
        float v = 0.f;
        for (int w = 0; w < NW; w++) v += red[threadIdx.x][w];
        atomicAdd(&gbg[b * 4 + threadIdx.x], v);
    }
    const int npix = min(PT_PIX, P - pbase);
    const int n0 = slice * PT_SLICE, n1 = min(N, n0 + PT_SLICE);
    for (int k = n0 + threadIdx.x; k < n1; k += NW * 32) {
        const long long sid = (long long)b * N + k;
        const SplatRec r = rec[sid];
        const float muy = r.a.x, mux = r.a.y, A = r.a.z, Bc = r.a.w;
        const float Cc = r.b.x, D = r.b.y, op = r.b.z;
        const float c0 = r.c.x, c1 = r.c.y, c2 = r.c.z;
        float Su = 0.f, Sv = 0.f, Suu = 0.f, Svv = 0.f, Suv = 0.f, Sf = 0.f, Sc0 = 0.f, Sc1 = 0.f, Sc2 = 0.f;
        for (int q = 0; q < npix; q++) {
            const float4 xy = sxy[q];
            const float4 d4 = sds[q];
            const float dy = xy.x - muy, dx = xy.y - mux;
            const float u = fmaf(A, dy, Bc * dx);
            const float v = fmaf(Cc, dy, D * dx);
            const float f = gs_ex2(-fmaf(u, u, v * v));
            const float fo = op * f;
            const float a = fminf(fo, GS_ALPHA_MAX);
            const float rr = gs_rcp(1.0f - a);
            const float col_term = fmaf(d4.z, c0, fmaf(d4.w, c1, xy.z * c2));
            const float da = fmaf(-d4.x, rr, d4.y + col_term);
            Sc0 = fmaf(a, d4.z, Sc0);
            Sc1 = fmaf(a, d4.w, Sc1);
            Sc2 = fmaf(a, xy.z, Sc2);
            const float dafo = fo < GS_ALPHA_MAX ? da : 0.0f;
            Sf = fmaf(dafo, f, Sf);
            const float Gm = dafo * fo;
            const float Gu = Gm * u, Gv = Gm * v;
            Su += Gu;
            Sv += Gv;
            Suu = fmaf(Gu, u, Suu);
            Svv = fmaf(Gv, v, Svv);
            Suv = fmaf(Gu, v, Suv);
        }
        float *ap = acc + sid * 12;
        gs_red_add_v4(ap, Su, Sv, Suu, Svv);
        gs_red_add_v4(ap + 4, Suv, Sf, Sc0, Sc1);
        gs_red_add_v4(ap + 8, Sc2, 0.f, 0.f, 0.f);
    }
}

// L2 loss of a [planes][H][W] image against a target over rows [y0, y1): grad = 2*scale*(out - target)
// inside the band (rows outside are not written), loss += scale * sum (out - target)^2.
__global__ void __launch_bounds__(256) k_l2_grad(const float *__restrict__ out, const float *__restrict__ target,
                                                 long long planes, int H, int W, int y0, int y1, float scale,
                                                 float *__restrict__ grad, float *__restrict__ loss) {
    __shared__ float red[8];
    const long long per = (long long)(y1 - y0) * W;
    float acc = 0.f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < planes * per;
         i += (long long)gridDim.x * blockDim.x) {
        const long long pl = i / per, r = i - pl * per;
        const long long idx = pl * H * W + (long long)y0 * W + r;
        const float d = out[idx] - target[idx];
        grad[idx] = 2.0f * scale * d;
        acc = fmaf(d, d, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
        atomicAdd(loss, t * scale);
    }
}

__global__ void k_activate_scale(const float *__restrict__ ls, float *__restrict__ out, long long n) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = gs_softplus_eps(ls[i]);
}

// ----------------------------------------------------------------------------------------------------
// host side: geometry, bounds, workspace plan

namespace {

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Plan {
    RenderGeom G;
    int ngroups;
    long long cap;
    int nblk_pre;
    int scatter_parts;  // scatter blocks per preprocessing block (>= 4 blocks per SM of 148 in all)
    int dcap;           // deep-tile list capacity
    size_t o_rec, o_meta, o_counts, o_zero, o_gpairs, o_gsplats, o_misc, o_tdiff, z_len;
    size_t o_ranges, o_cursor, o_dlist, o_vals, o_fields, fwd_bytes;
    size_t o_G, o_gfields, o_adjT, o_bzero, o_acc, o_gbg, bz_len, total_bytes;
    AdjPlan adj;
};

int validate(const gs_render_desc *d) {
    if (!d) return GS_ERR_BAD_ARGUMENT;
    if (d->mode < 0 || d->mode > 3) return GS_ERR_BAD_ARGUMENT;
    if (d->B < 1 || d->N < 0 || d->C < 1 || d->C > 3 || d->H < 1 || d->W < 1) return GS_ERR_BAD_ARGUMENT;
    if (!(d->tile == 4 || d->tile == 8 || d->tile == 16)) return GS_ERR_BAD_ARGUMENT;
    if (d->mode == GS_MODE_OCTAVE && (d->max_octaves < 0 || d->max_octaves > GS_MAX_GROUPS - 1))
        return GS_ERR_BAD_ARGUMENT;
    if (d->mode == GS_MODE_EXACT && d->odds) return GS_ERR_BAD_ARGUMENT;
    if (!(d->cutoff > 0.0f)) return GS_ERR_BAD_ARGUMENT;
    if ((long long)d->B * d->N >= (1LL << 31)) return GS_ERR_BAD_ARGUMENT;
    if (d->row_end > 0 && (d->row_begin < 0 || d->row_begin >= d->row_end || d->row_end > d->H))
        return GS_ERR_BAD_ARGUMENT;
    return GS_OK;
}

void make_geom(const gs_render_desc *d, RenderGeom &G) {
    memset(&G, 0, sizeof(G));
    G.mode = d->mode; G.B = d->B; G.N = d->N; G.C = d->C; G.H = d->H; G.W = d->W; G.tile = d->tile;
    G.odds = d->odds; G.has_theta = d->has_theta; G.max_oct = d->max_octaves;
    G.n_coarse = d->n_coarse; G.cutoff = d->cutoff; G.base_texels = d->base_texels;
    G.rep = (float)std::min(d->H, d->W);
    int T = d->tile;
    int res[GS_MAX_GROUPS][2];
    int ng;
    if (d->mode == GS_MODE_OCTAVE) {
        ng = d->max_octaves + 1;
        for (int o = 0; o < ng; o++) {
            res[o][0] = std::max(8, d->H >> o);
            res[o][1] = std::max(8, d->W >> o);
        }
        for (int k = 0; k < ng; k++) G.order[k] = k;  // octave 0 first (render_triton.py:959-972)
    } else if (d->mode == GS_MODE_MULTIRES) {
        ng = 2;
        int m = std::min(d->H, d->W) / 8;
        int cf = std::min(d->coarse_factor, std::max(1, m));
        res[0][0] = std::max(1, d->H / cf);
        res[0][1] = std::max(1, d->W / cf);
        res[1][0] = d->H;
        res[1][1] = d->W;
        G.order[0] = 1;  // fine + upsampled coarse (render_triton.py:914-916)
        G.order[1] = 0;
    } else {
        ng = 1;
        res[0][0] = d->H;
        res[0][1] = d->W;
        G.order[0] = 0;
    }
    G.ngroups = ng;
    // tile numbering: coarsest group first so the deep (long) tiles are scheduled early
    int toff = 0;
    long long foff = 0;
    for (int k = ng - 1; k >= 0; k--) {
        GroupGeom &gg = G.g[k];
        gg.H = res[k][0];
        gg.W = res[k][1];
        gg.ntx = (gg.W + T - 1) / T;
        gg.nty = (gg.H + T - 1) / T;
        gg.tile_off = toff;
        toff += gg.ntx * gg.nty;
    }
    for (int k = 0; k < ng; k++) {
        G.g[k].fld_off = (int)foff;
        foff += 5LL * G.g[k].H * G.g[k].W;
        G.g[k].prior_grp = -1;
        G.g[k].prior_off = -1;
    }
    G.tiles_per_image = toff;
    G.fld_per_image = foff;
    {
        long long adj = 0;
        for (int k = 0; k < ng; k++) {
            GroupGeom &gg = G.g[k];
            gg.up_sy = (float)gg.H / (float)d->H;
            gg.up_sx = (float)gg.W / (float)d->W;
            if (gg.H == d->H && gg.W == d->W) {
                gg.adj_off = -1;
            } else {
                gg.adj_off = (int)adj;
                adj += (long long)gg.H * gg.W;
            }
        }
    }
    G.y0 = std::max(0, d->row_begin);
    G.y1 = d->row_end > 0 ? std::min(d->H, d->row_end) : d->H;
    for (int k = 0; k < ng; k++) {
        GroupGeom &gg = G.g[k];
        int lo, hi;  // texel rows of group k sampled by native rows [y0, y1) (+1 row of margin)
        if (gg.H == d->H) {
            lo = G.y0;
            hi = G.y1 - 1;
        } else {
            double sc = (double)gg.H / (double)d->H;
            lo = (int)std::floor(sc * (G.y0 + 0.5) - 0.5) - 1;
            hi = (int)std::floor(sc * (G.y1 - 1 + 0.5) - 0.5) + 2;
        }
        lo = std::max(0, lo);
        hi = std::min(gg.H - 1, hi);
        gg.ty_lo = lo / T;
        gg.ty_hi = hi >= lo ? hi / T : -1;
    }
}

// per-splat upper bound on the tiles of group g (see gs_render_pair_bound)
long long group_tile_bound(const gs_render_desc *d, const RenderGeom &G, int g) {
    const GroupGeom &gg = G.g[g];
    long long nt = (long long)gg.ntx * gg.nty;
    if (d->mode != GS_MODE_OCTAVE || g == d->max_octaves) return nt;
    // octave o < max: ceil(log2(sigma_px / base_texels)) <= o  =>  sigma <= base_texels * 2^o / min(H, W)
    double smax = (double)d->base_texels * (double)(1LL << g) / (double)std::min(d->H, d->W);
    smax *= 1.0 + 1e-5;
    double r = (double)d->cutoff * smax;
    double rx = r * gg.W, ry = r * gg.H;
    long long sx = std::min<long long>(gg.ntx, (long long)(2.0 * rx / d->tile) + 2);
    long long sy = std::min<long long>(gg.nty, (long long)(2.0 * ry / d->tile) + 2);
    return std::min(nt, sx * sy);
}

long long pair_bound(const gs_render_desc *d, const RenderGeom &G) {
    if (d->mode == GS_MODE_EXACT) return 0;
    long long worst = 0;
    for (int g = 0; g < G.ngroups; g++) worst = std::max(worst, group_tile_bound(d, G, g));
    if (d->mode == GS_MODE_MULTIRES && d->n_coarse > 0 && d->n_coarse < d->N) {
        long long b0 = group_tile_bound(d, G, 0) * d->n_coarse + group_tile_bound(d, G, 1) * (d->N - d->n_coarse);
        return b0 * d->B;
    }
    return worst * (long long)d->N * d->B;
}

// Splats of one image that group g may hold: every splat in octave mode (routing is by scale), the
// head split in multires mode.
long long group_splats(const gs_render_desc *d, int g) {
    if (d->mode == GS_MODE_MULTIRES && d->n_coarse > 0 && d->n_coarse < d->N) return g == 0 ? d->n_coarse : d->N - d->n_coarse;
    return d->N;
}

void make_plan(const gs_render_desc *d, Plan &pl) {
    memset(&pl, 0, sizeof(pl));
    make_geom(d, pl.G);
    pl.ngroups = pl.G.ngroups;
    long long cap = d->pair_capacity > 0 ? d->pair_capacity : pair_bound(d, pl.G);
    if (d->mode == GS_MODE_EXACT) cap = 0;
    pl.cap = cap;
    pl.G.cap = cap;
    long long BN = (long long)d->B * d->N;
    pl.nblk_pre = (int)std::max<long long>(1, (BN + 255) / 256);
    pl.scatter_parts = std::min(8, std::max(1, (4 * 148 + pl.nblk_pre - 1) / pl.nblk_pre));
    const long long ntiles = (long long)d->B * pl.G.tiles_per_image;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o = align256(o + bytes); return r; };
    pl.o_rec = take(sizeof(SplatRec) * (size_t)std::max<long long>(BN, 1));
    pl.o_meta = take(sizeof(int4) * (size_t)std::max<long long>(BN, 1));
    pl.o_counts = take(sizeof(int) * (size_t)std::max<long long>(BN, 1));
    // zeroed block (memset): group stats, misc (total pairs as int64 + status), the tile difference array
    pl.o_zero = o;
    pl.o_gpairs = take(sizeof(unsigned long long) * (size_t)d->B * pl.ngroups);
    pl.o_gsplats = take(sizeof(int) * (size_t)d->B * pl.ngroups);
    pl.o_misc = take(64);
    pl.o_tdiff = take(sizeof(int) * (size_t)(ntiles + 1));
    pl.z_len = o - pl.o_zero;
    pl.o_ranges = take(sizeof(int2) * (size_t)ntiles);  // written whole by k_tile_scan
    pl.o_cursor = take(sizeof(int) * (size_t)ntiles);
    pl.dcap = (int)std::min<long long>(ntiles, cap / (FW_DEEP + 1) + 1);
    pl.o_dlist = take(sizeof(int) * (size_t)std::max(pl.dcap, 1));
    pl.o_vals = take(sizeof(int) * (size_t)std::max<long long>(cap, 1));
    pl.o_fields = take(sizeof(float) * (size_t)d->B * pl.G.fld_per_image);
    pl.fwd_bytes = o;
    pl.o_G = take(sizeof(float) * 5 * (size_t)d->B * d->H * d->W);
    pl.o_gfields = take(sizeof(float) * (size_t)d->B * pl.G.fld_per_image);
    {
        // separable adjoint: per coarse group, X outputs (band rows x coarse columns) and Y outputs (coarse
        // texels), thread-per-output or a 32-lane team when an output gathers more than ~24 inputs
        AdjPlan &A = pl.adj;
        memset(&A, 0, sizeof(A));
        const RenderGeom &G = pl.G;
        const long long rows = std::max(0, G.y1 - G.y0);
        long long ud = 0, ux = 0, uy = 0, toff = 0;
        for (int k = 0; k < GS_MAX_GROUPS; k++) {
            A.uD[k] = ud;
            A.uX[k] = ux;
            A.uY[k] = uy;
            A.teamX[k] = A.teamY[k] = 1;
            if (k >= G.ngroups || G.g[k].adj_off < 0) continue;
            const long long Hg = G.g[k].H, Wg = G.g[k].W;
            if ((d->W + Wg - 1) / Wg <= 8 && (d->H + Hg - 1) / Hg <= 8) {  // shallow: direct gather
                ud += Hg * Wg;
                continue;
            }
            // a 32-lane team only where one output gathers more than ~100 taps (factor >= 64): a team
            // multiplies the launch 32-fold, which costs even when the group turns out empty on the device
            A.teamX[k] = 2 * (d->W + Wg - 1) / Wg + 3 > 100 ? 32 : 1;
            A.teamY[k] = 2 * (d->H + Hg - 1) / Hg + 3 > 100 ? 32 : 1;
            ux += (rows * Wg * A.teamX[k] + 31) / 32 * 32;
            uy += (Hg * Wg * A.teamY[k] + 31) / 32 * 32;
            A.tOff[k] = toff;
            toff += 5 * rows * Wg;
        }
        A.uD[GS_MAX_GROUPS] = ud;
        A.uX[GS_MAX_GROUPS] = ux;
        A.uY[GS_MAX_GROUPS] = uy;
        A.tPerImage = toff;
    }
    pl.o_adjT = take(sizeof(float) * (size_t)std::max<long long>(1, d->B * pl.adj.tPerImage));
    pl.o_bzero = o;
    pl.o_acc = take(sizeof(float) * 12 * (size_t)std::max<long long>(BN, 1));
    pl.o_gbg = take(sizeof(float) * 4 * (size_t)d->B);
    pl.bz_len = o - pl.o_bzero;
    pl.total_bytes = o;
}

// The pair counts must be read back (one stream sync) before the pairs are emitted when the host bound
// cannot rule out (a) a (image, group) pair count above the budget max_pairs -- the reference's
// _build_tiles refusal, render_triton.py:378-385 -- or (b) more pairs than the workspace's pair capacity
// (a capacity set below gs_render_pair_bound).
bool needs_exact_check(const gs_render_desc *d, const Plan &pl) {
    if (d->mode == GS_MODE_EXACT || d->N <= 0) return false;
    if (pl.cap < pair_bound(d, pl.G)) return true;
    if (d->max_pairs < 0) return false;
    for (int g = 0; g < pl.G.ngroups; g++)
        if (group_tile_bound(d, pl.G, g) * group_splats(d, g) > d->max_pairs) return true;
    return false;
}

template <typename T>
T *at(void *ws, size_t off) { return reinterpret_cast<T *>(reinterpret_cast<char *>(ws) + off); }

int launch_fields_fwd(const Plan &pl, void *ws, cudaStream_t st) {
    const RenderGeom &G = pl.G;
    dim3 grid((unsigned)((long long)G.B * G.tiles_per_image));
    auto rec = at<SplatRec>(ws, pl.o_rec);
    auto rng = at<int2>(ws, pl.o_ranges);
    const int *vals = at<int>(ws, pl.o_vals);
    auto fld = at<float>(ws, pl.o_fields);
    if (G.tile == 8 && G.mode != GS_MODE_EXACT) {
        // deep tiles (more than FW_DEEP pairs) first, FW_DEEP_NW warps each on a persistent grid (three
        // CTAs per SM); then one warp per remaining tile
        const int *dl = at<int>(ws, pl.o_dlist);
        const unsigned char *misc = at<unsigned char>(ws, pl.o_misc);
        const unsigned dgrid = (unsigned)std::max(1, std::min(pl.dcap, 148 * 3));
        const int nt = (int)((long long)G.B * G.tiles_per_image);
        constexpr int WPB = FW_W8_WPB;
        const unsigned wgrid = (unsigned)((nt + WPB - 1) / WPB);
        if (G.odds) {
            k_fields_deep8<true><<<dgrid, FW_DEEP_NW * 32, 0, st>>>(G, rec, rng, vals, dl, misc, fld);
            k_fields_w8<true, WPB><<<wgrid, WPB * 32, 0, st>>>(G, rec, rng, vals, fld, nt);
        } else {
            k_fields_deep8<false><<<dgrid, FW_DEEP_NW * 32, 0, st>>>(G, rec, rng, vals, dl, misc, fld);
            k_fields_w8<false, WPB><<<wgrid, WPB * 32, 0, st>>>(G, rec, rng, vals, fld, nt);
        }
        GS_COUNT(1);
        GS_CHECK_LAUNCH("k_fields_w8");
        return GS_OK;
    }
    // 4 warps per tile (8 measured slower: the per-warp staging and the cross-warp reduction dominate
    // short lists)
    if (G.odds) {
        if (G.tile == 8) k_fields_fwd<8, 4, true><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
        else if (G.tile == 16) k_fields_fwd<16, 4, true><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
        else k_fields_fwd<4, 4, true><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
    } else {
        if (G.tile == 8) k_fields_fwd<8, 4, false><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
        else if (G.tile == 16) k_fields_fwd<16, 4, false><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
        else k_fields_fwd<4, 4, false><<<grid, 128, 0, st>>>(G, rec, rng, vals, fld);
    }
    GS_CHECK_LAUNCH("k_fields_fwd");
    return GS_OK;
}

// with_bins: the workspace holds the binning buffers (not so for gs_render_count's short one)
int run_preprocess(const Plan &pl, const float *mu, const float *ls, const float *col, const float *op,
                   const float *th, void *ws, cudaStream_t st, bool with_bins = true) {
    const RenderGeom &G = pl.G;
    cudaError_t e = cudaMemsetAsync(at<char>(ws, pl.o_zero), 0, pl.z_len, st);
    GS_COUNT(1);
    if (e != cudaSuccess) return set_cuda_error(e, "memset");
    const bool bins = with_bins && G.mode != GS_MODE_EXACT;
    k_preprocess<<<pl.nblk_pre, 256, 0, st>>>(G, mu, ls, col, op, G.has_theta ? th : nullptr, at<SplatRec>(ws, pl.o_rec),
                                              at<int4>(ws, pl.o_meta), at<int>(ws, pl.o_counts),
                                              at<unsigned long long>(ws, pl.o_gpairs), at<int>(ws, pl.o_gsplats),
                                              bins ? at<int>(ws, pl.o_tdiff) : nullptr);
    GS_CHECK_LAUNCH("k_preprocess");
    return GS_OK;
}

// Exact check after k_preprocess (its per-(image, group) pair counts are in the workspace): copies them to
// the host, synchronising the stream.  GS_ERR_PAIR_BUDGET when one (image, group) exceeds d->max_pairs,
// GS_ERR_WORKSPACE when the call's pairs exceed the pair capacity; refused during stream capture, where a
// synchronisation is not possible (size the capacity from gs_render_pair_bound or gs_render_count then).
int exact_check(const gs_render_desc *d, const Plan &pl, void *ws, cudaStream_t s) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone) {
        snprintf(g_last_error, sizeof(g_last_error),
                 "gs_render_fwd: the pair budget / pair capacity check needs the exact pair counts (a stream "
                 "synchronisation), which stream capture does not allow; capture with pair_capacity = 0 and a "
                 "budget the host bound satisfies");
        return GS_ERR_BAD_ARGUMENT;
    }
    const int n = d->B * pl.ngroups;
    std::vector<unsigned long long> cnt((size_t)n);
    cudaError_t e = cudaMemcpyAsync(cnt.data(), at<unsigned long long>(ws, pl.o_gpairs),
                                    sizeof(unsigned long long) * (size_t)n, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return set_cuda_error(e, "gs_render_fwd (pair check)");
    unsigned long long worst = 0, total = 0;
    for (int i = 0; i < n; i++) {
        worst = std::max(worst, cnt[(size_t)i]);
        total += cnt[(size_t)i];
    }
    if (d->max_pairs >= 0 && worst > (unsigned long long)d->max_pairs) {
        snprintf(g_last_error, sizeof(g_last_error),
                 "%llu (tile, splat) pairs in one (image, group) exceed the %lld budget @ %dx%d TILE=%d cutoff=%g "
                 "N=%d; refusing to render", worst, (long long)d->max_pairs, d->H, d->W, d->tile, (double)d->cutoff,
                 d->N);
        return GS_ERR_PAIR_BUDGET;
    }
    if (total > (unsigned long long)pl.cap) {
        snprintf(g_last_error, sizeof(g_last_error),
                 "%llu (tile, splat) pairs exceed the workspace's pair capacity %lld", total, (long long)pl.cap);
        return GS_ERR_WORKSPACE;
    }
    return GS_OK;
}

// ---- pixel-list render (render_alpha_subsampled)

__global__ void __launch_bounds__(256) k_points_prep(long long BN, int C, int has_theta, const float *__restrict__ mu,
                                                     const float *__restrict__ ls, const float *__restrict__ col,
                                                     const float *__restrict__ op, const float *__restrict__ th,
                                                     SplatRec *__restrict__ rec) {
    const long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= BN) return;
    float sy, sx;
    rec[s] = make_rec(s, C, has_theta, mu, ls, col, op, th, sy, sx);
}

struct PointsPlan {
    int nslices;
    size_t o_rec, o_part, o_fields, o_acc, o_gbg, fwd_bytes, total_bytes;
};

int points_validate(const gs_render_desc *d, int P) {
    int st = validate(d);
    if (st != GS_OK) return st;
    if (d->mode != GS_MODE_EXACT || d->odds || P < 1) return GS_ERR_BAD_ARGUMENT;
    if ((long long)d->B * P >= (1LL << 31)) return GS_ERR_BAD_ARGUMENT;
    return GS_OK;
}

void points_plan(const gs_render_desc *d, int P, PointsPlan &pp) {
    const long long BN = (long long)d->B * d->N;
    pp.nslices = (int)std::max<long long>(1, (d->N + PT_SLICE - 1) / PT_SLICE);
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o = align256(o + bytes); return r; };
    pp.o_rec = take(sizeof(SplatRec) * (size_t)std::max<long long>(BN, 1));
    pp.o_part = take(sizeof(float) * 5 * (size_t)pp.nslices * d->B * P);
    pp.o_fields = take(sizeof(float) * 5 * (size_t)d->B * P);
    pp.fwd_bytes = o;
    pp.o_acc = take(sizeof(float) * 12 * (size_t)std::max<long long>(BN, 1));
    pp.o_gbg = take(sizeof(float) * 4 * (size_t)d->B);
    pp.total_bytes = o;
}

}  // namespace

// ----------------------------------------------------------------------------------------------------
// C ABI

extern "C" {

int64_t gs_render_pair_bound(const gs_render_desc *d) {
    if (validate(d) != GS_OK) return -1;
    RenderGeom G;
    make_geom(d, G);
    return pair_bound(d, G);
}

// Pair positions and tile ranges are 32-bit: one call holds fewer than 2^31 (tile, splat) pairs.
static bool pairs_fit(const Plan &pl) { return pl.cap < (1LL << 31); }

size_t gs_render_workspace_size(const gs_render_desc *d, int with_backward) {
    if (validate(d) != GS_OK) return 0;
    Plan pl;
    make_plan(d, pl);
    if (!pairs_fit(pl)) return 0;
    return with_backward ? pl.total_bytes : pl.fwd_bytes;
}

int gs_render_count(const gs_render_desc *d, const float *mu, const float *log_scale, void *workspace,
                    size_t workspace_bytes, int64_t *counts_host, int32_t *groups_out, void *stream) {
    int st = validate(d);
    if (st != GS_OK) return st;
    if (!mu || !log_scale || !counts_host) return GS_ERR_BAD_ARGUMENT;
    gs_render_desc dd = *d;
    dd.pair_capacity = 1;
    Plan pl;
    make_plan(&dd, pl);
    if (workspace_bytes < pl.o_ranges) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    // colour/opacity are not needed for counting: point them at the positions (any readable floats)
    const float *dummy = mu;
    pl.G.C = 1;
    pl.G.has_theta = 0;
    st = run_preprocess(pl, mu, log_scale, dummy, dummy, nullptr, workspace, s, false);
    if (st != GS_OK) return st;
    int n = d->B * pl.ngroups;
    unsigned long long *tmp = new unsigned long long[n];
    cudaError_t e = cudaMemcpyAsync(tmp, at<unsigned long long>(workspace, pl.o_gpairs), sizeof(unsigned long long) * n,
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        delete[] tmp;
        return set_cuda_error(e, "gs_render_count");
    }
    for (int i = 0; i < n; i++) counts_host[i] = (int64_t)tmp[i];
    delete[] tmp;
    if (groups_out) *groups_out = pl.ngroups;
    return GS_OK;
}

int gs_render_fwd(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                  const float *opacity, const float *bg, const float *theta, float *out, void *workspace,
                  size_t workspace_bytes, void *stream) {
    return gs_render_fwd_prior(d, mu, log_scale, color, opacity, bg, theta, out, nullptr, workspace,
                               workspace_bytes, stream);
}

}  // extern "C"

int gs_render_prior_map(const gs_render_desc *prior_d, const void *prior_ws, const gs_render_desc *d, int n_prior,
                        GsPrior *out) {
    if (!out) return 0;
    memset(out, 0, sizeof(*out));
    for (int k = 0; k < GS_MAX_GROUPS; k++) out->grp[k] = out->off[k] = -1;
    if (validate(prior_d) != GS_OK || validate(d) != GS_OK || !prior_ws) return 0;
    if (prior_d->mode != GS_MODE_OCTAVE || d->mode != GS_MODE_OCTAVE) return 0;
    if (prior_d->B != d->B || prior_d->tile != d->tile || prior_d->cutoff != d->cutoff ||
        prior_d->base_texels != d->base_texels || prior_d->max_octaves != d->max_octaves ||
        prior_d->odds != d->odds || prior_d->has_theta != d->has_theta || prior_d->C != d->C)
        return 0;
    if (n_prior <= 0 || n_prior != prior_d->N || n_prior > d->N || prior_d->row_end > 0 || d->row_end > 0) return 0;
    const int rep_p = std::min(prior_d->H, prior_d->W), rep = std::min(d->H, d->W);
    if (rep != 2 * rep_p) return 0;  // the octave index then shifts by exactly one
    Plan pp;
    make_plan(prior_d, pp);
    RenderGeom G;
    make_geom(d, G);
    int mapped = 0;
    for (int k = 2; k <= d->max_octaves; k++) {
        const int kp = k - 1;
        if (kp >= prior_d->max_octaves) continue;  // the prior's clamped last octave also holds larger splats
        if (G.g[k].H != pp.G.g[kp].H || G.g[k].W != pp.G.g[kp].W) continue;
        out->grp[k] = kp;
        out->off[k] = pp.G.g[kp].fld_off;
        mapped++;
    }
    if (!mapped) return 0;
    out->fields = reinterpret_cast<const float *>(reinterpret_cast<const char *>(prior_ws) + pp.o_fields);
    out->fld_per_image = pp.G.fld_per_image;
    out->skip_n = n_prior;
    out->rep = (float)rep_p;
    return mapped;
}

int gs_render_fwd_prior(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                        const float *opacity, const float *bg, const float *theta, float *out, const GsPrior *prior,
                        void *workspace, size_t workspace_bytes, void *stream) {
    int st = validate(d);
    if (st != GS_OK) return st;
    if (!bg || !out) return GS_ERR_BAD_ARGUMENT;
    if (d->N > 0 && (!mu || !log_scale || !color || !opacity || (d->has_theta && !theta))) return GS_ERR_BAD_ARGUMENT;
    Plan pl;
    make_plan(d, pl);
    if (!pairs_fit(pl)) return GS_ERR_BAD_ARGUMENT;
    if (!workspace || workspace_bytes < pl.fwd_bytes) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    if (prior && prior->fields) {
        pl.G.skip_n = prior->skip_n;
        pl.G.prior_rep = prior->rep;
        for (int k = 0; k < pl.G.ngroups; k++) {
            pl.G.g[k].prior_grp = prior->grp[k];
            pl.G.g[k].prior_off = prior->off[k];
        }
    }
    const RenderGeom &G = pl.G;
    std::unique_ptr<ProfScope> bin_scope(new ProfScope(gs_prof_internal() ? PR_ENC_BIN : PR_BIN, s));
    st = run_preprocess(pl, mu, log_scale, color, opacity, theta, workspace, s);
    if (st != GS_OK) return st;
    unsigned char *misc = at<unsigned char>(workspace, pl.o_misc);
    if (d->mode != GS_MODE_EXACT) {
        if (d->N > 0 && needs_exact_check(d, pl)) {
            st = exact_check(d, pl, workspace, s);
            if (st != GS_OK) return st;
        }
        // (with no splats the scan still runs: it writes every tile's range empty)
        const long long nt = (long long)d->B * G.tiles_per_image;
        int *cursor = at<int>(workspace, pl.o_cursor);
        k_tile_scan<<<1, TS_THREADS, 0, s>>>(at<int>(workspace, pl.o_tdiff), nt, pl.cap, at<int2>(workspace, pl.o_ranges),
                                             cursor, at<int>(workspace, pl.o_dlist), pl.dcap, misc);
        GS_CHECK_LAUNCH("k_tile_scan");
        if (d->N > 0) {
            k_scatter<<<pl.nblk_pre * pl.scatter_parts, 256, 0, s>>>(G, at<int4>(workspace, pl.o_meta),
                                                                     at<int>(workspace, pl.o_counts),
                                                                     pl.scatter_parts, cursor,
                                                                     at<int>(workspace, pl.o_vals), misc);
            GS_CHECK_LAUNCH("k_scatter");
        }
    }
    bin_scope.reset();
    {
        ProfScope ps(gs_prof_internal() ? PR_ENC_FIELDS_FWD : PR_FIELDS_FWD, s);
        st = launch_fields_fwd(pl, workspace, s);
        if (st != GS_OK) return st;
        if (G.skip_n > 0) {
            long long big = 0;
            for (int k = 0; k < G.ngroups; k++)
                if (G.g[k].prior_off >= 0) big = std::max(big, 5LL * G.g[k].H * G.g[k].W);
            // the mapped groups as one range when they are consecutive in both layouts
            int k0 = -1, k1 = -1;
            bool flat = true;
            for (int k = 0; k < G.ngroups; k++) {
                if (G.g[k].prior_off < 0) continue;
                if (k0 < 0) k0 = k;
                else if (k != k1 + 1 || G.g[k].prior_off - G.g[k1].prior_off != (long long)G.g[k].fld_off - G.g[k1].fld_off)
                    flat = false;
                k1 = k;
            }
            const long long lo = k0 >= 0 ? G.g[k0].fld_off : 0, plo = k0 >= 0 ? G.g[k0].prior_off : 0;
            const long long n = k0 >= 0 ? (long long)G.g[k1].fld_off + 5LL * G.g[k1].H * G.g[k1].W - lo : 0;
            float *fl = at<float>(workspace, pl.o_fields);
            if (flat && n > 0 && n % 4 == 0 && lo % 4 == 0 && plo % 4 == 0 && G.fld_per_image % 4 == 0 &&
                prior->fld_per_image % 4 == 0 && (reinterpret_cast<uintptr_t>(prior->fields) & 15) == 0 &&
                (reinterpret_cast<uintptr_t>(fl) & 15) == 0 && n / 4 < (1LL << 31)) {
                dim3 pg((unsigned)((n / 4 + 255) / 256), (unsigned)d->B);
                k_add_prior_flat<<<pg, 256, 0, s>>>(prior->fields, prior->fld_per_image, plo, fl, G.fld_per_image, lo,
                                                    (int)(n / 4));
            } else {
                dim3 pg((unsigned)((big + 255) / 256), (unsigned)G.ngroups, (unsigned)d->B);
                k_add_prior<<<pg, 256, 0, s>>>(G, prior->fields, prior->fld_per_image, fl);
            }
            GS_CHECK_LAUNCH("k_add_prior");
        }
    }
    if (G.y1 > G.y0) {
        ProfScope ps(PR_COMPOSITE, s);
        const unsigned rows = (unsigned)std::max(1, G.y1 - G.y0);
        if (d->W % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
            dim3 cg((unsigned)((d->W / 4 + 63) / 64), rows, (unsigned)d->B);
            k_composite4<<<cg, 64, 0, s>>>(G, at<float>(workspace, pl.o_fields), at<int>(workspace, pl.o_gsplats), bg,
                                           out);
        } else {
            dim3 cg((unsigned)((d->W + 127) / 128), rows, (unsigned)d->B);
            k_composite<<<cg, 128, 0, s>>>(G, at<float>(workspace, pl.o_fields), at<int>(workspace, pl.o_gsplats), bg,
                                           out);
        }
        GS_CHECK_LAUNCH("k_composite");
    }
    return GS_OK;
}

extern "C" {

int gs_render_bwd(const gs_render_desc *d, const float *mu, const float *log_scale, const float *color,
                  const float *opacity, const float *bg, const float *theta, const float *grad_out, float *g_mu,
                  float *g_log_scale, float *g_color, float *g_opacity, float *g_bg, float *g_theta,
                  void *workspace, size_t workspace_bytes, void *stream) {
    int st = validate(d);
    if (st != GS_OK) return st;
    if (!grad_out || !g_bg) return GS_ERR_BAD_ARGUMENT;
    if (d->N > 0 && (!g_mu || !g_log_scale || !g_color || !g_opacity || !log_scale)) return GS_ERR_BAD_ARGUMENT;
    (void)mu; (void)color; (void)opacity;
    Plan pl;
    make_plan(d, pl);
    if (!workspace || workspace_bytes < pl.total_bytes) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const RenderGeom &G = pl.G;
    cudaError_t e = cudaMemsetAsync(at<char>(workspace, pl.o_bzero), 0, pl.bz_len, s);
    GS_COUNT(1);
    if (e != cudaSuccess) return set_cuda_error(e, "memset");
    dim3 cg((unsigned)((d->W + 127) / 128), (unsigned)std::max(1, G.y1 - G.y0), (unsigned)d->B);
    int clamp_mask = (d->mode == GS_MODE_OCTAVE || d->mode == GS_MODE_MULTIRES) ? 1 : 0;
    std::unique_ptr<ProfScope> cb_scope(new ProfScope(PR_COMPOSITE_BWD, s));
    k_composite_bwd<<<cg, 128, 0, s>>>(G, at<float>(workspace, pl.o_fields), at<int>(workspace, pl.o_gsplats), bg,
                                       grad_out, at<float>(workspace, pl.o_G), at<float>(workspace, pl.o_gbg),
                                       clamp_mask);
    GS_CHECK_LAUNCH("k_composite_bwd");
    bool any_coarse = false;
    for (int g = 0; g < G.ngroups; g++)
        if (!(G.g[g].H == G.H && G.g[g].W == G.W)) any_coarse = true;
    if (any_coarse) {
        const AdjPlan &A = pl.adj;
        const long long ud = A.uD[GS_MAX_GROUPS], ux = A.uX[GS_MAX_GROUPS], uy = A.uY[GS_MAX_GROUPS];
        if (ud > 0) {
            dim3 gd((unsigned)((ud + 255) / 256), (unsigned)d->B);
            k_adjoint_direct<<<gd, 256, 0, s>>>(G, A, at<int>(workspace, pl.o_gsplats),
                                                at<int2>(workspace, pl.o_ranges), at<float>(workspace, pl.o_G),
                                                at<float>(workspace, pl.o_gfields));
            GS_CHECK_LAUNCH("k_adjoint_direct");
        }
        if (ux > 0) {
            dim3 gx((unsigned)((ux + 255) / 256), (unsigned)d->B);
            k_adjoint_x<<<gx, 256, 0, s>>>(G, A, at<int>(workspace, pl.o_gsplats), at<float>(workspace, pl.o_G),
                                           at<float>(workspace, pl.o_adjT));
            GS_CHECK_LAUNCH("k_adjoint_x");
        }
        if (uy > 0) {
            dim3 gy((unsigned)((uy + 255) / 256), (unsigned)d->B);
            k_adjoint_y<<<gy, 256, 0, s>>>(G, A, at<int>(workspace, pl.o_gsplats), at<float>(workspace, pl.o_adjT),
                                           at<float>(workspace, pl.o_gfields));
            GS_CHECK_LAUNCH("k_adjoint_y");
        }
    }
    cb_scope.reset();
    dim3 grid((unsigned)((long long)G.B * G.tiles_per_image));
    auto rec = at<SplatRec>(workspace, pl.o_rec);
    auto rng = at<int2>(workspace, pl.o_ranges);
    const int *vals = at<int>(workspace, pl.o_vals);
    auto Gn = at<float>(workspace, pl.o_G);
    auto gf = at<float>(workspace, pl.o_gfields);
    auto acc = at<float>(workspace, pl.o_acc);
    if (d->N > 0) {
        ProfScope ps(PR_FIELDS_BWD, s);
        if (G.odds) {
            if (G.tile == 8) k_fields_bwd<8, 4, true><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
            else if (G.tile == 16) k_fields_bwd<16, 4, true><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
            else k_fields_bwd<4, 4, true><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
        } else {
            if (G.tile == 8) k_fields_bwd<8, 4, false><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
            else if (G.tile == 16) k_fields_bwd<16, 4, false><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
            else k_fields_bwd<4, 4, false><<<grid, 128, 0, s>>>(G, rec, rng, vals, Gn, gf, acc);
        }
        GS_CHECK_LAUNCH("k_fields_bwd");
    }
    long long nfin = std::max<long long>((long long)d->B * d->N, (long long)d->B * d->C);
    ProfScope ps(PR_FINALIZE, s);
    k_finalize<<<(unsigned)((nfin + 255) / 256), 256, 0, s>>>(G, log_scale, d->has_theta ? theta : nullptr, acc,
                                                              at<float>(workspace, pl.o_gbg), g_mu, g_log_scale,
                                                              g_color, g_opacity, g_bg, g_theta);
    GS_CHECK_LAUNCH("k_finalize");
    return GS_OK;
}

int gs_render_debug_bins(const gs_render_desc *d, const void *workspace, int64_t *total_pairs,
                         int32_t *tiles_per_image, int32_t *geom_host, int32_t *tile_ranges_host,
                         int32_t *splat_ids_host, int32_t *octave_host) {
    int st = validate(d);
    if (st != GS_OK) return st;
    Plan pl;
    make_plan(d, pl);
    void *ws = const_cast<void *>(workspace);
    long long tot = 0;
    cudaError_t e = cudaMemcpy(&tot, at<long long>(ws, pl.o_misc), sizeof(long long), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_cuda_error(e, "debug_bins");
    if (total_pairs) *total_pairs = tot;
    if (tiles_per_image) *tiles_per_image = pl.G.tiles_per_image;
    if (geom_host)
        for (int g = 0; g < pl.ngroups; g++) {
            geom_host[g * 5 + 0] = pl.G.g[g].H;
            geom_host[g * 5 + 1] = pl.G.g[g].W;
            geom_host[g * 5 + 2] = pl.G.g[g].ntx;
            geom_host[g * 5 + 3] = pl.G.g[g].nty;
            geom_host[g * 5 + 4] = pl.G.g[g].tile_off;
        }
    if (tile_ranges_host) {
        e = cudaMemcpy(tile_ranges_host, at<int2>(ws, pl.o_ranges), sizeof(int2) * (size_t)d->B * pl.G.tiles_per_image,
                       cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return set_cuda_error(e, "debug_bins");
    }
    if (splat_ids_host && tot > 0) {
        const int *vals = at<int>(ws, pl.o_vals);
        e = cudaMemcpy(splat_ids_host, vals, sizeof(int) * (size_t)std::min<long long>(tot, pl.cap),
                       cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return set_cuda_error(e, "debug_bins");
    }
    if (octave_host) {
        long long BN = (long long)d->B * d->N;
        int4 *m = new int4[std::max<long long>(BN, 1)];
        e = cudaMemcpy(m, at<int4>(ws, pl.o_meta), sizeof(int4) * (size_t)BN, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess)
            for (long long i = 0; i < BN; i++) octave_host[i] = m[i].y >> 24;
        delete[] m;
        if (e != cudaSuccess) return set_cuda_error(e, "debug_bins");
    }
    int status = 0;
    e = cudaMemcpy(&status, at<int>(ws, pl.o_misc + 8), sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_cuda_error(e, "debug_bins");
    return status ? GS_ERR_PAIR_BUDGET : GS_OK;
}

int gs_l2_loss_grad(const float *out, const float *target, int64_t planes, int32_t H, int32_t W, int32_t row_begin,
                    int32_t row_end, float scale, float *grad, float *loss, void *stream) {
    if (!out || !target || !grad || !loss || planes < 0 || H < 1 || W < 1) return GS_ERR_BAD_ARGUMENT;
    int y0 = std::max(0, row_begin), y1 = row_end > 0 ? std::min(H, row_end) : H;
    if (y1 <= y0) return GS_ERR_BAD_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(loss, 0, sizeof(float), s);
    GS_COUNT(1);
    if (e != cudaSuccess) return set_cuda_error(e, "gs_l2_loss_grad");
    long long n = planes * (long long)(y1 - y0) * W;
    unsigned grid = (unsigned)std::min<long long>(148 * 8, std::max<long long>(1, (n + 255) / 256));
    k_l2_grad<<<grid, 256, 0, s>>>(out, target, planes, H, W, y0, y1, scale, grad, loss);
    GS_CHECK_LAUNCH("k_l2_grad");
    return GS_OK;
}

int gs_activate_scale(const float *log_scale, float *out, int64_t n, void *stream) {
    if (!log_scale || !out || n < 0) return GS_ERR_BAD_ARGUMENT;
    if (n == 0) return GS_OK;
    k_activate_scale<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(log_scale, out, n);
    GS_CHECK_LAUNCH("k_activate_scale");
    return GS_OK;
}

size_t gs_render_points_workspace_size(const gs_render_desc *d, int32_t P, int with_backward) {
    if (points_validate(d, P) != GS_OK) return 0;
    PointsPlan pp;
    points_plan(d, P, pp);
    return with_backward ? pp.total_bytes : pp.fwd_bytes;
}

int gs_render_points_fwd(const gs_render_desc *d, int32_t P, const int64_t *px_idx, const float *mu,
                         const float *log_scale, const float *color, const float *opacity, const float *bg,
                         const float *theta, float *out, void *workspace, size_t workspace_bytes, void *stream) {
    int st = points_validate(d, P);
    if (st != GS_OK) return st;
    if (!px_idx || !bg || !out) return GS_ERR_BAD_ARGUMENT;
    if (d->N > 0 && (!mu || !log_scale || !color || !opacity || (d->has_theta && !theta))) return GS_ERR_BAD_ARGUMENT;
    PointsPlan pp;
    points_plan(d, P, pp);
    if (!workspace || workspace_bytes < pp.fwd_bytes) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const long long BN = (long long)d->B * d->N;
    auto rec = at<SplatRec>(workspace, pp.o_rec);
    auto part = at<float>(workspace, pp.o_part);
    const long long *idx = reinterpret_cast<const long long *>(px_idx);
    if (BN > 0) {
        k_points_prep<<<(unsigned)((BN + 255) / 256), 256, 0, s>>>(BN, d->C, d->has_theta, mu, log_scale, color,
                                                                  opacity, d->has_theta ? theta : nullptr, rec);
        GS_CHECK_LAUNCH("k_points_prep");
        dim3 grid((unsigned)((P + PT_PIX - 1) / PT_PIX), (unsigned)pp.nslices, (unsigned)d->B);
        k_points_fwd<4><<<grid, 128, 0, s>>>(d->N, d->H, d->W, P, idx, rec, part);
        GS_CHECK_LAUNCH("k_points_fwd");
    } else {
        cudaError_t e = cudaMemsetAsync(part, 0, sizeof(float) * 5 * (size_t)pp.nslices * d->B * P, s);
        GS_COUNT(1);
        if (e != cudaSuccess) return set_cuda_error(e, "memset");
    }
    const long long n = (long long)d->B * P;
    k_points_composite<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d->B, d->C, P, pp.nslices, part, bg,
                                                                   at<float>(workspace, pp.o_fields), out);
    GS_CHECK_LAUNCH("k_points_composite");
    return GS_OK;
}

int gs_render_points_bwd(const gs_render_desc *d, int32_t P, const int64_t *px_idx, const float *log_scale,
                         const float *bg, const float *theta, const float *grad_out, float *g_mu,
                         float *g_log_scale, float *g_color, float *g_opacity, float *g_bg, float *g_theta,
                         void *workspace, size_t workspace_bytes, void *stream) {
    int st = points_validate(d, P);
    if (st != GS_OK) return st;
    if (!px_idx || !bg || !grad_out || !g_bg) return GS_ERR_BAD_ARGUMENT;
    if (d->N > 0 && (!g_mu || !g_log_scale || !g_color || !g_opacity || !log_scale)) return GS_ERR_BAD_ARGUMENT;
    PointsPlan pp;
    points_plan(d, P, pp);
    if (!workspace || workspace_bytes < pp.total_bytes) return GS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(at<char>(workspace, pp.o_acc), 0, pp.total_bytes - pp.o_acc, s);
    GS_COUNT(1);
    if (e != cudaSuccess) return set_cuda_error(e, "memset");
    const long long *idx = reinterpret_cast<const long long *>(px_idx);
    dim3 grid((unsigned)((P + PT_PIX - 1) / PT_PIX), (unsigned)pp.nslices, (unsigned)d->B);
    k_points_bwd<4><<<grid, 128, 0, s>>>(d->N, d->C, d->H, d->W, P, idx, at<SplatRec>(workspace, pp.o_rec),
                                         at<float>(workspace, pp.o_fields), bg, grad_out,
                                         at<float>(workspace, pp.o_acc), at<float>(workspace, pp.o_gbg));
    GS_CHECK_LAUNCH("k_points_bwd");
    RenderGeom G;
    make_geom(d, G);
    long long nfin = std::max<long long>((long long)d->B * d->N, (long long)d->B * d->C);
    k_finalize<<<(unsigned)((nfin + 255) / 256), 256, 0, s>>>(G, log_scale, d->has_theta ? theta : nullptr,
                                                              at<float>(workspace, pp.o_acc),
                                                              at<float>(workspace, pp.o_gbg), g_mu, g_log_scale,
                                                              g_color, g_opacity, g_bg, g_theta);
    GS_CHECK_LAUNCH("k_finalize");
    return GS_OK;
}

const char *gs_last_error(void) { return g_last_error; }

uint64_t gs_kernel_launches(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

void gs_profile_enable(int on) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (on && g_prof_pool.empty()) {
        g_prof_pool.resize(4096);
        for (auto &e : g_prof_pool) {
            cudaEventCreate(&e.a);
            cudaEventCreate(&e.b);
            e.region = -1;
        }
    }
    g_prof_on = on != 0;
}

// Durations of the events recorded since the last collect (or, for events recorded by a CUDA graph,
// of its last replay); the pool is then recycled unless `keep` is set, in which case the same event
// slots stay assigned so a captured graph can be replayed and collected again.
int gs_profile_collect2(double *ms_out, int64_t *count_out, int keep) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (int r = 0; r < PR_N; r++) {
        if (ms_out) ms_out[r] = 0.0;
        if (count_out) count_out[r] = 0;
    }
    int st = GS_OK;
    for (size_t i = 0; i < g_prof_used; i++) {
        ProfEvent &e = g_prof_pool[i];
        float ms = 0.f;
        cudaError_t err = cudaEventSynchronize(e.b);
        if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e.a, e.b);
        if (err != cudaSuccess) {
            st = set_cuda_error(err, "gs_profile_collect");
            continue;
        }
        if (e.region >= 0 && e.region < PR_N) {
            if (ms_out) ms_out[e.region] += ms;
            if (count_out) count_out[e.region] += 1;
        }
    }
    if (!keep) g_prof_used = 0;
    return st;
}

int gs_profile_collect(double *ms_out, int64_t *count_out) { return gs_profile_collect2(ms_out, count_out, 0); }

int gs_build_arch(void) { return 100; }

}  // extern "C"
