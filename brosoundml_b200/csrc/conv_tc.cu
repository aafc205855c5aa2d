// tcgen05 implicit-GEMM convolution kernels (sm_100a).
//
// Forward-like form (conv fwd, conv input gradient with flipped/transposed
// weights, ConvTranspose1d stride phases):
//   D[co, o] = sum_{t, ci} W_t[co, ci] * X[b, (o + o_base) + t*d - p, ci]
// Persistent kernel, one 128 (co) x NP (positions, 192..256) fp32 tile at a time.
// K runs over 128-byte chunks of input channels; for each chunk the CTA loads one
// activation window of NP + (taps-1)*d rows and reuses it for every tap: tap
// t's operand is the same window shifted by t*d rows (a descriptor offset, not
// a new load). Only the per-tap weight tiles stream through their own ring.
// A launch with fewer tiles than half the SMs also splits each tile's K loop
// (chunk ranges) over the idle SMs; the partial tiles are summed in a fixed
// order by a reduce pass that applies the epilogue.
//
// Weight-gradient form (stride-1 convs):
//   D[co, ci] (tap t) = sum_{b, o} dY[b, o, co] * X[b, o + t*d - p, ci]
// K runs over chunks of positions; both operands are MN-major (positions are
// rows, channels contiguous), staged as 128-byte-wide column blocks. A CTA
// computes two taps from one dY chunk and one X window. Split-K over position
// chunks writes fp32 partial tiles, reduced in double afterwards.
//
// Warp roles: warp 0 issues TMA, warp 1 owns TMEM and one thread issues
// tcgen05.mma, the remaining warps read the accumulator (each warp its 32-lane
// quarter of TMEM) and run the epilogue.
//
// Promotion (TF32x3): the tensor core's in-TMEM fp32 accumulation is not
// round-to-nearest, and its error grows with K. The MMA warp alternates between
// two TMEM accumulators, PG K steps each, and the epilogue warps fold every
// finished partial into fp32 registers, so each TMEM sum spans only 12*PG
// instructions and the long sum is formed with ordinary fp32 adds. In the
// persistent forward kernel the same two buffers carry on into the next tile,
// so the epilogue's stores of one tile overlap the next tile's MMAs.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "conv_tc.h"
#include "kernels.h"
#include "planes.cuh"
#include "tc_ptx.cuh"

namespace bsml {

namespace {

__device__ int g_tc_err = 0;

constexpr int TILE_BYTES = 16384;   // 128 rows x 128 bytes
// promoted accumulation: K steps summed in TMEM before the epilogue folds them into registers
#ifndef BSML_PG
#define BSML_PG 2
#endif
constexpr int PG = BSML_PG;
constexpr int SMEM_OPTIN = 232448;  // opt-in dynamic shared memory per block on sm_100

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ── forward-like kernel ──────────────────────────────────────────────────────
// Operand format of a mode: fp32 containers read by tf32 MMAs (TF32X3, planes hi +
// lo) or bf16 (BF16: one plane; BF16X3: hi + lo planes). Two planes issue the three
// products hi*hi + hi*lo + lo*hi per K step.
template <int MODE>
struct Fmt {
    static constexpr bool F32 = MODE == TC_TF32X3;
    static constexpr bool LO = MODE != TC_BF16;
    static constexpr int PLANES = LO ? 2 : 1;
    static constexpr int BKE = F32 ? 32 : 64;             // elements per 128-byte row
    static constexpr uint32_t KIND = F32 ? 2u : 1u;       // instruction-descriptor A/B format
};

template <int MODE, int NP, int NH_>
struct FCfg {
    static constexpr int BKE = Fmt<MODE>::BKE;            // channels per 128-byte row
    static constexpr int PLANES = Fmt<MODE>::PLANES;
    static constexpr int NPOS = NP;                        // positions per tile (MMA N): 256, 224 or 192
    static constexpr int NH = NH_;                         // column groups per TMEM lane quarter (2 or 4)
    static constexpr int HALF = NP / NH;                   // columns per epilogue warp (multiple of 8)
    static constexpr int WT_BYTES = PLANES * TILE_BYTES;   // one weight stage: 128 co x 128 B per plane
    static constexpr int NEPI = 4 * NH;                    // epilogue warps: 4 lane quarters x NH column groups
    static constexpr int THREADS = 64 + NEPI * 32;
    static constexpr int MAX_SW = 8;
};

struct FArgs {
    int No, o_base, p, d, taps, kchunks, Co;
    int n_co, n_pt, n_tiles;
    int wbox;        // rows per window box; a window is two boxes (2 * wbox rows)
    int win_bytes;   // one window stage, all planes
    int sw;          // weight stages
    float* y; int64_t y_bs; int y_ld; int orow_mul, orow_off, y_rows;
    const float* bias;
    const float* r; int64_t r_bs; int r_ld; int r_shift;
    float alpha; int accum;
    double* stats;   // per-(b, co) sum and sum of squares of the stored outputs (nullable)
    // split-K: work item i = tile (i % n_tiles) over chunk range (i / n_tiles) of ksplit;
    // with ksplit > 1 the epilogue stores raw fp32 partials part[split][b][o][co]
    int ksplit, nb;
    float* part;
};

// Input-channel chunks [lo, hi) of split `s` of `ks` (near-equal ranges).
__device__ __forceinline__ int split_lo(int s, int ks, int kchunks) { return (int)((int64_t)s * kchunks / ks); }

// 2 + 4*NH warps. NH = 2: 320 threads, 168 registers per thread at most (3 warps
// per SM sub-partition); NH = 4: 576 threads, 96 registers (5 warps per
// sub-partition). More epilogue warps shorten each warp's share of the tile-end
// stores, which must finish before the MMAs, two promotion groups ahead, need its
// buffer; fewer, with more registers, fold faster when a tile has many K steps.
template <int MODE, int NPT, int NH>
__global__ void __launch_bounds__(FCfg<MODE, NPT, NH>::THREADS, 1)
    conv_fwd_tc_kernel(const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                       const __grid_constant__ CUtensorMap mXh, const __grid_constant__ CUtensorMap mXl,
                       const FArgs a) {
    using F = FCfg<MODE, NPT, NH>;
    constexpr bool LO = Fmt<MODE>::LO, F32E = Fmt<MODE>::F32;
    constexpr int NP = F::NPOS, HC = F::HALF;
    constexpr uint32_t TCOLS = 512;   // two promotion buffers of NP fp32 columns (allocation: a power of 2)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* win = smem;                          // [2 stages][PLANES][2 * wbox rows][128 B]
    uint8_t* wst = smem + 2 * a.win_bytes;        // [sw][PLANES][128 rows][128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(wst + a.sw * F::WT_BYTES);
    uint64_t* wfull = bars;                       // [MAX_SW]
    uint64_t* wempty = bars + F::MAX_SW;          // [MAX_SW]
    uint64_t* xfull = bars + 2 * F::MAX_SW;       // [2]
    uint64_t* xempty = xfull + 2;                 // [2]
    uint64_t* accf = xempty + 2;                  // [2]
    uint64_t* acce = accf + 2;                    // [2]
    uint64_t* mdone = acce + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + 1);
    int* err = &g_tc_err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = a.n_tiles * a.ksplit;
    const int plane_bytes = 2 * a.wbox * 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.sw; ++s) {
            tc::mbar_init(&wfull[s], 1);
            tc::mbar_init(&wempty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&xfull[s], 1);
            tc::mbar_init(&xempty[s], 1);
            tc::mbar_init(&accf[s], 1);
            tc::mbar_init(&acce[s], F::NEPI);
        }
        tc::mbar_init(mdone, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&mWh);
        tc::prefetch_tmap(&mXh);
        if (LO) {
            tc::prefetch_tmap(&mWl);
            tc::prefetch_tmap(&mXl);
        }
    }
    if (warp == 1) {
        tc::tmem_alloc(tslot, TCOLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            // ── TMA producer: per chunk one window, then one weight tile per tap
            int kit = 0, cw = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const int tile = it % a.n_tiles, ks = it / a.n_tiles;
                const int ct = tile % a.n_co, rest = tile / a.n_co;
                const int pt = rest % a.n_pt, b = rest / a.n_pt;
                const int m0 = ct * 128, row0 = pt * NP + a.o_base - a.p;
                const int c_hi = split_lo(ks + 1, a.ksplit, a.kchunks);
                for (int c = split_lo(ks, a.ksplit, a.kchunks); ok && c < c_hi; ++c) {
                    const int kx = c * F::BKE;
                    const int xs = cw & 1;
                    if (!tc::mbar_wait(&xempty[xs], ((cw >> 1) & 1) ^ 1, err, tc::TC_ERR_WAIT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t* wb = win + xs * a.win_bytes;
                    tc::mbar_arrive_expect_tx(&xfull[xs], a.win_bytes);
                    tc::tma_load_3d(wb, &mXh, &xfull[xs], kx, row0, b);
                    tc::tma_load_3d(wb + a.wbox * 128, &mXh, &xfull[xs], kx, row0 + a.wbox, b);
                    if (LO) {
                        tc::tma_load_3d(wb + plane_bytes, &mXl, &xfull[xs], kx, row0, b);
                        tc::tma_load_3d(wb + plane_bytes + a.wbox * 128, &mXl, &xfull[xs], kx, row0 + a.wbox, b);
                    }
                    ++cw;
                    for (int t = 0; t < a.taps; ++t) {
                        const int s = kit % a.sw;
                        if (!tc::mbar_wait(&wempty[s], ((kit / a.sw) & 1) ^ 1, err, tc::TC_ERR_WAIT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        uint8_t* ws = wst + s * F::WT_BYTES;
                        tc::mbar_arrive_expect_tx(&wfull[s], F::WT_BYTES);
                        tc::tma_load_3d(ws, &mWh, &wfull[s], kx, m0, t);
                        if (LO) tc::tma_load_3d(ws + TILE_BYTES, &mWl, &wfull[s], kx, m0, t);
                        ++kit;
                    }
                }
            }
            if (!ok) {   // drain: copies issued into the rings may still be in flight
                for (int i = kit - a.sw < 0 ? 0 : kit - a.sw; i < kit; ++i)
                    tc::mbar_wait(&wfull[i % a.sw], (i / a.sw) & 1, nullptr, tc::TC_ERR_DRAIN);
                for (int i = cw - 2 < 0 ? 0 : cw - 2; i < cw; ++i)
                    tc::mbar_wait(&xfull[i & 1], (i >> 1) & 1, nullptr, tc::TC_ERR_DRAIN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ── MMA issuer
            constexpr uint32_t idesc = tc::make_idesc(Fmt<MODE>::KIND, 0u, 0u, 128, NP);
            int kit = 0, cw = 0, G = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const int ks = it / a.n_tiles;
                const int c_lo = split_lo(ks, a.ksplit, a.kchunks), c_hi = split_lo(ks + 1, a.ksplit, a.kchunks);
                const int n_iters = a.taps * (c_hi - c_lo);        // K steps of this item
                const int n_groups = (n_iters + PG - 1) / PG;      // its promotion groups
                for (int c = c_lo; ok && c < c_hi; ++c) {
                    const int xs = cw & 1;
                    if (!tc::mbar_wait(&xfull[xs], (cw >> 1) & 1, err, tc::TC_ERR_WAIT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t xh = tc::smem_u32(win + xs * a.win_bytes);
                    const uint32_t xl = xh + plane_bytes;
                    for (int t = 0; t < a.taps; ++t) {
                        const int li = (c - c_lo) * a.taps + t;
                        const bool g_first = (li % PG) == 0;
                        const bool g_last = (li % PG) == PG - 1 || li == n_iters - 1;
                        const int g = G + li / PG;
                        const int buf = g & 1;
                        if (g_first && g >= 2 &&
                            !tc::mbar_wait(&acce[buf], ((g >> 1) - 1) & 1, err, tc::TC_ERR_WAIT_ACC)) {
                            ok = false;
                            break;
                        }
                        const int s = kit % a.sw;
                        if (!tc::mbar_wait(&wfull[s], (kit / a.sw) & 1, err, tc::TC_ERR_WAIT_FULL)) {
                            ok = false;
                            break;
                        }
                        tc::tc_fence_after();
                        const uint32_t wa = tc::smem_u32(wst + s * F::WT_BYTES);
                        const uint32_t roff = (uint32_t)(t * a.d) * 128u;   // tap shift inside the window
                        const uint32_t d_tmem = tbase + (uint32_t)(buf * NP);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t dAh = tc::desc_kmajor_sw128(wa + kk * 32);
                            const uint64_t dBh = tc::desc_kmajor_sw128(xh + roff + kk * 32);
                            const uint32_t acc = (g_first && kk == 0) ? 0u : 1u;
                            tc::umma<F32E>(d_tmem, dAh, dBh, idesc, acc);
                            if (LO) {
                                const uint64_t dAl = tc::desc_kmajor_sw128(wa + TILE_BYTES + kk * 32);
                                const uint64_t dBl = tc::desc_kmajor_sw128(xl + roff + kk * 32);
                                tc::umma<F32E>(d_tmem, dAh, dBl, idesc, 1u);
                                tc::umma<F32E>(d_tmem, dAl, dBh, idesc, 1u);
                            }
                        }
                        tc::umma_commit(&wempty[s]);   // frees the weight stage once these MMAs have read it
                        ++kit;
                        if (g_last) tc::umma_commit(&accf[buf]);
                    }
                    if (!ok) break;
                    tc::umma_commit(&xempty[xs]);      // frees the window after its last tap
                    ++cw;
                }
                G += n_groups;
            }
            // every issued MMA has completed before TMEM is released
            tc::umma_commit(mdone);
            tc::mbar_wait(mdone, 0, nullptr, tc::TC_ERR_DRAIN);
        }
    } else {
        // ── epilogue: warp (q, h) folds lanes 32q..32q+31, columns HC*h..HC*h+HC-1
        const int ew = warp - 2;
        const int q = warp & 3;   // the TMEM lane quarter this warp may access
        const int h = ew >> 2;
        const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * HC);
        int G = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
            const int tile = it % a.n_tiles, ks = it / a.n_tiles;
            const int n_iters = a.taps * (split_lo(ks + 1, a.ksplit, a.kchunks) - split_lo(ks, a.ksplit, a.kchunks));
            const int n_groups = (n_iters + PG - 1) / PG;
            const int ct = tile % a.n_co, rest = tile / a.n_co;
            const int pt = rest % a.n_pt, b = rest / a.n_pt;
            const int mrow = ct * 128 + q * 32 + lane;   // co
            const int o0 = pt * NP + h * HC;
            // columns j in [jlo, jhi) map to output rows inside y: row(j) = row0 + j*orow_mul
            const int row0 = (o0 + a.o_base) * a.orow_mul + a.orow_off;
            const int jlo = row0 >= 0 ? 0 : (-row0 + a.orow_mul - 1) / a.orow_mul;
            int jhi = min(HC, a.No - o0);
            jhi = a.y_rows > row0 ? min(jhi, (a.y_rows - row0 + a.orow_mul - 1) / a.orow_mul) : 0;
            if (mrow >= a.Co) jhi = 0;
            const float* rb = (a.r && a.ksplit == 1) ? a.r + (int64_t)b * a.r_bs + mrow : nullptr;
            float* yb = a.y + (int64_t)b * a.y_bs + mrow;
            // the prior-output rows an accumulating tile reads at its end go to L2 now,
            // while its MMAs run (a warp's 32 lanes share each 128-byte line)
            if (a.accum && a.ksplit == 1)
                for (int j = jlo; j < jhi; ++j) tc::prefetch_l2(yb + (row0 + j * a.orow_mul) * a.y_ld);
            // the residual starts the sum: its loads complete under the tile's first
            // MMAs instead of stalling the tile-end stores
            float R[HC];
#pragma unroll
            for (int j = 0; j < HC; ++j)
                R[j] = (rb && j >= jlo && j < jhi) ? rb[((row0 + j * a.orow_mul) >> a.r_shift) * a.r_ld] : 0.f;
            for (int gi = 0; gi < n_groups; ++gi) {
                const int g = G + gi, buf = g & 1;
                bool w = true;
                if (lane == 0) w = tc::mbar_wait(&accf[buf], (g >> 1) & 1, err, tc::TC_ERR_WAIT_ACC);
                ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (int c16 = 0; c16 + 16 <= HC; c16 += 16) {
                    uint32_t v[16];
                    tc::tmem_ld16_nowait(trow + (uint32_t)(buf * NP + c16), v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) R[c16 + j] += __uint_as_float(v[j]);
                }
                if (HC % 16 == 8) {
                    constexpr int c8 = HC - 8;
                    uint32_t v[8];
                    tc::tmem_ld8_nowait(trow + (uint32_t)(buf * NP + c8), v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j) R[c8 + j] += __uint_as_float(v[j]);
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&acce[buf]);
            }
            G += n_groups;
            if (!ok || *(volatile int*)err != tc::TC_OK) break;
            if (a.ksplit > 1) {   // raw partial sums; the reduce pass applies the epilogue
                if (mrow < a.Co) {
                    const int nrow = min(HC, a.No - o0);
                    float* pp = a.part + (((int64_t)ks * a.nb + b) * a.No + o0) * a.Co + mrow;
#pragma unroll
                    for (int jj = 0; jj < HC; ++jj)
                        if (jj < nrow) pp[(int64_t)jj * a.Co] = R[jj];
                }
                continue;
            }
            if (mrow < a.Co) {
                const float bv = a.bias ? a.bias[mrow] : 0.f;
                // ST: also the output statistics. They are summed in fp32 about a shift c
                // (this thread's first column), so the sums stay at the scale of the
                // spread rather than of the mean, and moved to double once per tile: per
                // output one subtract and two fp32 adds, no float-to-double conversion
                // (those run on the narrow XU pipe and throttled the epilogue). Without
                // statistics no such work is issued at all.
                auto store = [&](auto st_tag) {
                    constexpr bool ST = decltype(st_tag)::value;
                    const float c = (R[0] + bv) * a.alpha;
                    float g1 = 0.f, g2 = 0.f;
                    auto emit = [&](int jj, float val) {
                        yb[(row0 + jj * a.orow_mul) * a.y_ld] = val;
                        if (ST) {
                            const float dv = val - c;
                            g1 += dv;
                            g2 = fmaf(dv, dv, g2);
                        }
                    };
                    if (!a.accum) {
#pragma unroll
                        for (int jj = 0; jj < HC; ++jj)
                            if (jj >= jlo && jj < jhi) emit(jj, (R[jj] + bv) * a.alpha);
                    } else {
                        // EB columns at a time: their reads are all issued before their stores
                        constexpr int EB = 8;
#pragma unroll
                        for (int c16 = 0; c16 < HC; c16 += EB) {
                            float u[EB];
#pragma unroll
                            for (int j = 0; j < EB; ++j) {
                                const int jj = c16 + j;
                                u[j] = (jj >= jlo && jj < jhi) ? yb[(row0 + jj * a.orow_mul) * a.y_ld] : 0.f;
                            }
#pragma unroll
                            for (int j = 0; j < EB; ++j) {
                                const int jj = c16 + j;
                                if (jj >= jlo && jj < jhi) emit(jj, (R[jj] + bv) * a.alpha + u[j]);
                            }
                        }
                    }
                    if (ST) {
                        // sum (v) = sum (v - c) + n c;  sum (v^2) = sum (v - c)^2 + 2 c sum (v - c) + n c^2
                        const double n = (double)max(jhi - jlo, 0), cd = c, d1 = g1;
                        atomicAdd(&a.stats[((int64_t)b * a.Co + mrow) * 2], d1 + n * cd);
                        atomicAdd(&a.stats[((int64_t)b * a.Co + mrow) * 2 + 1], (double)g2 + cd * (2.0 * d1 + n * cd));
                    }
                };
                if (a.stats)
                    store(std::true_type{});
                else
                    store(std::false_type{});
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, TCOLS);
    }
}

// Split-K epilogue: sums the ksplit partial tiles of each output element in a
// fixed order and applies the forward kernel's epilogue (bias, residual, scale,
// accumulation, output statistics). One thread per output channel over a strip
// of FR_ROWS positions, whose loads are all issued before the first store.
constexpr int FR_ROWS = 8;
__global__ void __launch_bounds__(128) fwd_split_reduce_kernel(const FArgs a) {
    const int co = blockIdx.y * 128 + threadIdx.x, b = blockIdx.z;
    if (co >= a.Co) return;
    const int o0 = blockIdx.x * FR_ROWS;
    const int64_t sstride = (int64_t)a.nb * a.No * a.Co;
    const float* __restrict__ pb = a.part + ((int64_t)b * a.No + o0) * a.Co + co;
    float acc[FR_ROWS], t[FR_ROWS], u[FR_ROWS];
    int row[FR_ROWS];
    bool in[FR_ROWS];
#pragma unroll
    for (int r = 0; r < FR_ROWS; ++r) {
        row[r] = (o0 + r + a.o_base) * a.orow_mul + a.orow_off;
        in[r] = o0 + r < a.No && row[r] >= 0 && row[r] < a.y_rows;
        acc[r] = 0.f;
    }
    for (int k = 0; k < a.ksplit; ++k)
#pragma unroll
        for (int r = 0; r < FR_ROWS; ++r)
            if (in[r]) acc[r] += pb[k * sstride + (int64_t)r * a.Co];
    const float bv = a.bias ? a.bias[co] : 0.f;
    const float* rb = a.r ? a.r + (int64_t)b * a.r_bs + co : nullptr;
    float* yb = a.y + (int64_t)b * a.y_bs + co;
#pragma unroll
    for (int r = 0; r < FR_ROWS; ++r) {
        t[r] = (rb && in[r]) ? rb[(int64_t)(row[r] >> a.r_shift) * a.r_ld] : 0.f;
        u[r] = (a.accum && in[r]) ? yb[(int64_t)row[r] * a.y_ld] : 0.f;
    }
    double s1 = 0.0, s2 = 0.0;
#pragma unroll
    for (int r = 0; r < FR_ROWS; ++r) {
        if (!in[r]) continue;
        const float val = (acc[r] + bv + t[r]) * a.alpha + u[r];
        yb[(int64_t)row[r] * a.y_ld] = val;
        s1 += val;
        s2 = fma((double)val, (double)val, s2);
    }
    if (a.stats) {
        atomicAdd(&a.stats[((int64_t)b * a.Co + co) * 2], s1);
        atomicAdd(&a.stats[((int64_t)b * a.Co + co) * 2 + 1], s2);
    }
}

// ── weight-gradient kernel ───────────────────────────────────────────────────
// One CTA: a 128 (co) x 128 (ci) tile for a pair of taps (t0, t0+1) over a split
// of the position chunks. Per K step it stages one dY chunk (KROWS positions) and
// one X window of KROWS + d rows: tap t0 + u reads the window shifted by u*d rows
// (a descriptor offset), so the dY chunk and the X rows serve both taps.
constexpr int BM = 128, BN = 128;

template <int MODE>
struct WCfg {
    static constexpr int PLANES = Fmt<MODE>::PLANES;
    static constexpr int BKE = Fmt<MODE>::BKE;        // elements per 128-byte row
    // positions (K rows) per stage; one MMA consumes 32 bytes of K = 8 (tf32)
    // or 16 (bf16) rows; 128-byte column blocks per 128-wide operand
    static constexpr int KROWS = Fmt<MODE>::F32 ? 32 : 64;
    static constexpr int MN_BLOCKS = 128 / BKE;
    static constexpr int A_BYTES = PLANES * MN_BLOCKS * KROWS * 128;   // dY chunk, all planes
    static constexpr int NEPI = 8;                                      // 4 lane quarters x 2 taps
    static constexpr int THREADS = 64 + NEPI * 32;
    static constexpr int MAX_S = 8;
};

struct WArgs {
    int taps, p, d, Co, Ci;
    // Ci tiles, tap pairs, chunks per clip, total chunks, chunks per split
    int n_ci_tiles, n_pairs, chunks_pc, chunks_total, chunks_per_split;
    int wrows;        // X window rows per column block (KROWS + d, rounded up to 8)
    int stage_bytes;  // A_BYTES + X window (all planes)
    int stages;
    float* part;      // [split][tap][Ci][Co]
};

template <int MODE>
__global__ void __launch_bounds__(WCfg<MODE>::THREADS, 1)
    conv_wgrad_tc_kernel(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                         const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl,
                         const WArgs a) {
    using C = WCfg<MODE>;
    constexpr bool LO = Fmt<MODE>::LO, F32E = Fmt<MODE>::F32;
    constexpr uint32_t TCOLS = 4 * BN;   // 2 taps x 2 promotion buffers
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.stages * a.stage_bytes);
    uint64_t* empty = full + C::MAX_S;
    uint64_t* accf = empty + C::MAX_S;   // [2]
    uint64_t* acce = accf + 2;           // [2]
    uint64_t* mdone = acce + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + 1);
    int* err = &g_tc_err;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM;                              // co
    const int pair = blockIdx.y / a.n_ci_tiles;
    const int n0 = (blockIdx.y - pair * a.n_ci_tiles) * BN;      // ci
    const int t0 = 2 * pair;
    const int ntap = min(2, a.taps - t0);
    // A lone last tap (odd tap count > 1) still issues the second tap's MMAs (into a
    // TMEM buffer nobody reads): every CTA then runs at the same pace, so the CTAs
    // of one split stream the same dY / X rows together and share them in L2.
    const int nmma = a.taps > 1 ? 2 : 1;
    const int it0 = blockIdx.z * a.chunks_per_split;
    const int it1 = min(a.chunks_total, it0 + a.chunks_per_split);
    const int n_iters = it1 > it0 ? it1 - it0 : 0;
    const int xplane = C::MN_BLOCKS * a.wrows * 128;             // one X plane in a stage

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(&accf[0], 1);
        tc::mbar_init(&accf[1], 1);
        tc::mbar_init(&acce[0], C::NEPI);
        tc::mbar_init(&acce[1], C::NEPI);
        tc::mbar_init(mdone, 1);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&mAh);
        tc::prefetch_tmap(&mBh);
        if (LO) {
            tc::prefetch_tmap(&mAl);
            tc::prefetch_tmap(&mBl);
        }
    }
    if (warp == 1) {
        tc::tmem_alloc(tslot, TCOLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            // ── TMA producer
            int issued = 0;
            bool ok = true;
            for (int it = 0; it < n_iters; ++it) {
                const int s = it % a.stages;
                const uint32_t ph = (it / a.stages) & 1;
                if (!tc::mbar_wait(&empty[s], ph ^ 1, err, tc::TC_ERR_WAIT_EMPTY)) { ok = false; break; }
                uint8_t* st = smem + s * a.stage_bytes;
                uint8_t* sB = st + C::A_BYTES;
                tc::mbar_arrive_expect_tx(&full[s], a.stage_bytes);
                const int q = it0 + it;
                const int bb = q / a.chunks_pc;
                const int orow = (q - bb * a.chunks_pc) * C::KROWS;
                const int xrow = orow + t0 * a.d - a.p;
#pragma unroll
                for (int j = 0; j < C::MN_BLOCKS; ++j) {
                    tc::tma_load_3d(st + j * C::KROWS * 128, &mAh, &full[s], m0 + j * C::BKE, orow, bb);
                    tc::tma_load_3d(sB + j * a.wrows * 128, &mBh, &full[s], n0 + j * C::BKE, xrow, bb);
                    if (LO) {
                        tc::tma_load_3d(st + C::A_BYTES / 2 + j * C::KROWS * 128, &mAl, &full[s], m0 + j * C::BKE,
                                        orow, bb);
                        tc::tma_load_3d(sB + xplane + j * a.wrows * 128, &mBl, &full[s], n0 + j * C::BKE, xrow, bb);
                    }
                }
                issued = it + 1;
            }
            if (!ok) {   // drain: the last issued stages may still have copies in flight
                for (int it = issued - a.stages < 0 ? 0 : issued - a.stages; it < issued; ++it)
                    tc::mbar_wait(&full[it % a.stages], (it / a.stages) & 1, nullptr, tc::TC_ERR_DRAIN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ── MMA issuer
            constexpr uint32_t idesc = tc::make_idesc(Fmt<MODE>::KIND, 1u, 1u, BM, BN);
            const uint32_t lbo_a = C::KROWS * 128, lbo_b = (uint32_t)a.wrows * 128;
            for (int it = 0; it < n_iters; ++it) {
                const int s = it % a.stages;
                const uint32_t ph = (it / a.stages) & 1;
                const int g = it / PG;                          // promotion group
                const bool g_first = (it % PG) == 0;
                const bool g_last = (it % PG) == PG - 1 || it == n_iters - 1;
                const int buf = g & 1;
                if (g_first && g >= 2 &&
                    !tc::mbar_wait(&acce[buf], ((g >> 1) - 1) & 1, err, tc::TC_ERR_WAIT_ACC))
                    break;
                if (!tc::mbar_wait(&full[s], ph, err, tc::TC_ERR_WAIT_FULL)) break;
                tc::tc_fence_after();
                const uint32_t base = tc::smem_u32(smem + s * a.stage_bytes);
                const uint32_t aH = base, aL = base + C::A_BYTES / 2;
                const uint32_t bH = base + C::A_BYTES, bL = bH + xplane;
                for (int u = 0; u < nmma; ++u) {
                    const uint32_t d_tmem = tbase + (uint32_t)((u * 2 + buf) * BN);
                    const uint32_t bshift = (uint32_t)(u * a.d) * 128u;   // tap t0 + u: window shifted by u*d rows
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        // +32 bytes of K = 8 rows (tf32) or 16 rows (bf16) = 1024 / 2048 B
                        const uint32_t off = kk * (F32E ? 1024 : 2048);
                        const uint64_t dAh = tc::desc_mnmajor(aH + off, lbo_a, F32E);
                        const uint64_t dBh = tc::desc_mnmajor(bH + bshift + off, lbo_b, F32E);
                        const uint32_t acc = (g_first && kk == 0) ? 0u : 1u;
                        tc::umma<F32E>(d_tmem, dAh, dBh, idesc, acc);
                        if (LO) {
                            const uint64_t dAl = tc::desc_mnmajor(aL + off, lbo_a, F32E);
                            const uint64_t dBl = tc::desc_mnmajor(bL + bshift + off, lbo_b, F32E);
                            tc::umma<F32E>(d_tmem, dAh, dBl, idesc, 1u);
                            tc::umma<F32E>(d_tmem, dAl, dBh, idesc, 1u);
                        }
                    }
                }
                tc::umma_commit(&empty[s]);           // frees the stage once these MMAs have read it
                if (g_last) tc::umma_commit(&accf[buf]);
            }
            tc::umma_commit(mdone);
            tc::mbar_wait(mdone, 0, nullptr, tc::TC_ERR_DRAIN);
        }
    } else {
        // ── epilogue: warp (q, u) folds lanes 32q..32q+31 of tap t0 + u
        const int q = warp & 3;
        const int u = (warp - 2) >> 2;
        const int mrow = m0 + q * 32 + lane;   // co
        const uint32_t trow = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(u * 2 * BN);
        float R[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) R[j] = 0.f;
        bool ok = true;
        const int n_groups = (n_iters + PG - 1) / PG;
        for (int g = 0; g < n_groups; ++g) {
            const int buf = g & 1;
            bool w = true;
            if (lane == 0) w = tc::mbar_wait(&accf[buf], (g >> 1) & 1, err, tc::TC_ERR_WAIT_ACC);
            ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc::tc_fence_after();
            if (u < ntap) {
#pragma unroll
                for (int c16 = 0; c16 < BN; c16 += 16) {
                    uint32_t v[16];
                    tc::tmem_ld16_nowait(trow + (uint32_t)(buf * BN + c16), v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) R[c16 + j] += __uint_as_float(v[j]);
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acce[buf]);
        }
        const bool valid = ok && *(volatile int*)err == tc::TC_OK;
        if (valid && u < ntap && mrow < a.Co) {
            // partials [split][tap][ci][co]: a warp's 32 lanes (consecutive co) store
            // one 128-byte line per column; the reduce reorders into dW
            float* pp = a.part + (((int64_t)blockIdx.z * a.taps + t0 + u) * a.Ci + n0) * a.Co + mrow;
#pragma unroll
            for (int j = 0; j < BN; ++j)
                if (n0 + j < a.Ci) pp[(int64_t)j * a.Co] = R[j];
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, TCOLS);
    }
}

// ── operand planes

// v as the operand planes of MODE at element o
template <int MODE>
__device__ __forceinline__ void put_planes(void* hi, void* lo, int64_t o, float v) {
    if (MODE == TC_TF32X3) {
        const float h = tf32_rna(v);
        static_cast<float*>(hi)[o] = h;
        static_cast<float*>(lo)[o] = v - h;
    } else if (MODE == TC_BF16X3) {
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        static_cast<__nv_bfloat16*>(hi)[o] = h;
        static_cast<__nv_bfloat16*>(lo)[o] = __float2bfloat16_rn(v - __bfloat162float(h));
    } else {
        static_cast<__nv_bfloat16*>(hi)[o] = __float2bfloat16_rn(v);
    }
}

template <int MODE>
__global__ void act_planes_kernel(Act x, void* hi, void* lo, int ld) {
    const int64_t n = x.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % x.C);
        const int64_t r = i / x.C;
        const int l = (int)(r % x.L), b = (int)(r / x.L);
        const float v = x.row(b, l)[c];
        const int64_t o = ((int64_t)b * x.L + l) * ld + c;
        put_planes<MODE>(hi, lo, o, v);
    }
}

// Element (t, m, kk) of one packed weight [tap][M][Kp] (zero padding of K to Kp).
__device__ __forceinline__ float pack_value(const float* W, int kind, int Co, int Ci, int k, int s, int r, int taps,
                                            int K, int t, int m, int kk) {
    if (kk >= K) return 0.f;
    if (kind == PACK_CONV_FWD) return W[((int64_t)m * Ci + kk) * k + t];                 // m = co, kk = ci
    if (kind == PACK_CONV_DGRAD) return W[((int64_t)kk * Ci + m) * k + (k - 1 - t)];     // m = ci, kk = co
    if (kind == PACK_CONVT_PHASE) {                                                       // m = co, kk = ci
        const int tt = r + (taps - 1 - t) * s;
        return W[((int64_t)kk * Co + m) * k + tt];
    }
    if (kind == PACK_CONV_STRIDED) {   // row-packed strided conv: m = co, kk = j*ld + ci (ld = r)
        const int j = kk / r, ci = kk - j * r;
        const int tt = t * s + j;
        return (ci < Ci && tt < k) ? W[((int64_t)m * Ci + ci) * k + tt] : 0.f;
    }
    // convT dgrad, row-packed: m = ci, kk = j*Co + co
    const int u_min = -((r + s - 1) / s);
    const int j = kk / Co, co = kk - j * Co;
    const int tt = (t + u_min) * s + j + r;
    return (tt >= 0 && tt < k) ? W[((int64_t)m * Co + co) * k + tt] : 0.f;
}

// Item i = m*Kp + kk of one packed weight: every tap of (m, kk). A thread's taps come
// from one source row of the weight (k consecutive floats for a conv), so a warp's
// loads cover a contiguous span instead of striding by k per lane; each tap's stores
// are consecutive kk across the warp.
template <int MODE>
__device__ __forceinline__ void pack_item(const float* W, int kind, int Co, int Ci, int k, int s, int r, int taps,
                                          int M, int K, int Kp, void* hi, void* lo, int64_t i) {
    const int kk = (int)(i % Kp);
    const int m = (int)(i / Kp);
    for (int t = 0; t < taps; ++t)
        put_planes<MODE>(hi, lo, ((int64_t)t * M + m) * Kp + kk, pack_value(W, kind, Co, Ci, k, s, r, taps, K, t, m, kk));
}

template <int MODE>
__global__ void pack_w_kernel(const float* W, int kind, int Co, int Ci, int k, int s, int r, int taps, int M, int K,
                              int Kp, void* hi, void* lo) {
    const int64_t n = (int64_t)M * Kp;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        pack_item<MODE>(W, kind, Co, Ci, k, s, r, taps, M, K, Kp, hi, lo, i);
}

// All jobs of a batch over one flat index space; each thread finds its job by
// binary search over the jobs' starts (held in shared memory).
template <int MODE>
__global__ void pack_w_batch_kernel(const float* params, const PackJob* jobs, int n_jobs, int64_t total) {
    __shared__ int64_t start[PACK_MAX_JOBS];
    for (int j = threadIdx.x; j < n_jobs; j += blockDim.x) start[j] = jobs[j].start;
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int lo = 0, hi = n_jobs - 1;
        while (lo < hi) {   // last job whose start <= i
            const int mid = (lo + hi + 1) >> 1;
            if (start[mid] <= i) lo = mid;
            else hi = mid - 1;
        }
        const PackJob& J = jobs[lo];
        pack_item<MODE>(params + J.w_off, J.kind, J.Co, J.Ci, J.k, J.s, J.r, J.taps, J.M, J.K, J.Kp, J.hi, J.lo,
                        i - start[lo]);
    }
}

// dW[(co*Ci + ci)*k + t] (+)= sum_split part[split][t][ci][co]; threads run in
// partial order (coalesced reads of the large partials, scattered writes of dW)
__global__ void wgrad_reduce_kernel(const float* part, int splits, int taps, int Co, int Ci, float* dW, int accum) {
    const int64_t n = (int64_t)Co * Ci * taps;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(i % Co);
        const int64_t q = i / Co;
        const int ci = (int)(q % Ci), t = (int)(q / Ci);
        const double s = sum_strided(part + i, n, splits);
        const int64_t o = ((int64_t)co * Ci + ci) * taps + t;
        dW[o] = (float)(accum ? dW[o] + s : s);
    }
}

// dW[co][ci][u*s + j] = dW2[co][j*ld + ci][u]   (strided conv, row-packed form)
__global__ void wgrad_unpack_strided_kernel(const float* dW2, int Co, int Ci, int k, int s, int ld, int U,
                                            float* dW) {
    const int64_t n = (int64_t)Co * Ci * k;
    const int K2 = s * ld;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i % k);
        const int64_t q = i / k;
        const int ci = (int)(q % Ci), co = (int)(q / Ci);
        const int u = t / s, j = t - u * s;
        dW[i] = dW2[((int64_t)co * K2 + j * ld + ci) * U + u];
    }
}

// ConvTranspose1d weight gradient from the row-packed partials:
// dW[(ci*CoT + co)*k + t] (+)= sum_split part[split][tau][j*CoT + co][ci], t - p = (tau + u_min)*s + j.
// Threads run in partial order; (tau, j) pairs whose t falls outside [0, k) carry no weight.
__global__ void wgrad_reduce_convT_kernel(const float* part, int splits, int taps, int M, int N, int CoT, int k, int s,
                                          int p, int u_min, float* dW, int accum) {
    const int64_t n = (int64_t)taps * N * M;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i % M);
        const int64_t q = i / M;
        const int nn = (int)(q % N), tau = (int)(q / N);
        const int j = nn / CoT, co = nn - j * CoT;
        const int t = (tau + u_min) * s + j + p;
        if (t < 0 || t >= k) continue;
        const double acc = sum_strided(part + i, n, splits);
        const int64_t o = ((int64_t)m * CoT + co) * k + t;
        dW[o] = (float)(accum ? dW[o] + acc : acc);
    }
}

inline int grid_for(int64_t n, int threads = 256) {
    int64_t g = ceil_div(n, threads);
    if (g > 148 * 32) g = 148 * 32;
    return (int)(g < 1 ? 1 : g);
}

// ── tensor maps
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) fail("conv_tc", "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// 3-D map over [d2][d1][d0] (d0 contiguous), box {box0, box1, 1}, 128-byte swizzle
// span (16-byte chunks, or 32-byte chunks for MN-major tf32 operands).
CUtensorMap make_map(const void* base, int mode, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t pitch0_elems,
                     uint64_t d1_elems_per_d2, uint32_t box0, uint32_t box1, bool atom32 = false) {
    CUtensorMap m;
    const uint64_t es = (uint64_t)tc_esize(mode);
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {pitch0_elems * es, pitch0_elems * d1_elems_per_d2 * es};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt =
        mode == TC_TF32X3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) fail("conv_tc", "operand base not 16-byte aligned");
    if (box0 * es != 128) fail("conv_tc", "box inner extent must be 128 bytes");
    const CUresult rc = get_encode()(&m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                                     atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) fail("conv_tc", "cuTensorMapEncodeTiled failed (" + std::to_string((int)rc) + ")");
    return m;
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        BSML_CUDA(cudaGetDevice(&dev));
        BSML_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    }
    return n;
}

// Tile width: the widest of 256 / 224 / 192 positions whose activation windows
// (two stages) still leave room for three weight stages.
struct FwdGeom {
    int np, wbox, win_bytes, sw, smem;
};
FwdGeom fwd_geom(int planes, int halo) {
    const int wt = planes * TILE_BYTES, fixed = 1024 + 256;
    FwdGeom g{};
    for (int np : {256, 224, 192}) {
        g.np = np;
        g.wbox = (int)round_up(ceil_div(np + halo, 2), 8);
        g.win_bytes = planes * 2 * g.wbox * 128;
        g.sw = std::min(8, (SMEM_OPTIN - fixed - 2 * g.win_bytes) / wt);
        if (g.wbox <= 256 && g.sw >= 3) break;
    }
    if (g.wbox > 256) fail("conv_fwd_tc", "tap span too large for the activation window");
    if (g.sw < 2) fail("conv_fwd_tc", "activation window too large for shared memory");
    g.smem = 2 * g.win_bytes + g.sw * wt + fixed;
    return g;
}

// K splits of a forward-like launch: only when its output tiles fill less than half
// of the SMs, at most one input-channel chunk range per idle SM, and within the
// caller's scratch (`cap` floats for ksplit x B x No x Co partials).
int fwd_ksplit(const TcConvFwd& c, int mode, int np, int64_t cap) {
    const int kchunks = (int)ceil_div(c.Ci, mode == TC_TF32X3 ? 32 : 64);
    const int64_t tiles = ceil_div(c.Co, 128) * ceil_div(c.No, np) * (int64_t)c.B;
    const int sms = sm_count();
    if (tiles * 2 > sms || kchunks < 2) return 1;
    int64_t ks = std::min<int64_t>(kchunks, sms / tiles);
    const int64_t per = (int64_t)c.B * c.No * c.Co;
    ks = std::min<int64_t>(ks, cap / std::max<int64_t>(per, 1));
    return ks >= 2 ? (int)ks : 1;
}

template <int MODE, int NPT, int NH>
void launch_fwd_np(const TcConvFwd& c, int mode, const FwdGeom& g, cudaStream_t st) {
    using F = FCfg<MODE, NPT, NH>;
    constexpr bool LO = Fmt<MODE>::LO;
    static bool attr = false;
    if (!attr) {
        BSML_CUDA(cudaFuncSetAttribute(conv_fwd_tc_kernel<MODE, NPT, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_OPTIN));
        attr = true;
    }
    FArgs a{};
    a.wbox = g.wbox;
    a.win_bytes = g.win_bytes;
    a.sw = g.sw;
    const uint32_t bke = F::BKE;
    const CUtensorMap mWh = make_map(c.w.hi, mode, c.Ci, c.Co, c.taps, c.w.ld, c.Co, bke, 128);
    const CUtensorMap mWl = LO ? make_map(c.w.lo, mode, c.Ci, c.Co, c.taps, c.w.ld, c.Co, bke, 128) : mWh;
    const CUtensorMap mXh = make_map(c.x.hi, mode, c.Ci, c.L_in, c.B, c.x.ld, c.L_in, bke, a.wbox);
    const CUtensorMap mXl = LO ? make_map(c.x.lo, mode, c.Ci, c.L_in, c.B, c.x.ld, c.L_in, bke, a.wbox) : mXh;
    a.No = c.No; a.o_base = c.o_base; a.p = c.p; a.d = c.d; a.taps = c.taps;
    a.kchunks = (int)ceil_div(c.Ci, F::BKE);
    a.Co = c.Co;
    a.n_co = (int)ceil_div(c.Co, 128);
    a.n_pt = (int)ceil_div(c.No, F::NPOS);
    const int64_t tiles = (int64_t)a.n_co * a.n_pt * c.B;
    if (tiles > (1ll << 30)) fail("conv_fwd_tc", "too many tiles");
    a.n_tiles = (int)tiles;
    a.y = c.y.p; a.y_bs = c.y.bstride; a.y_ld = c.y.ld; a.orow_mul = c.orow_mul; a.orow_off = c.orow_off;
    a.y_rows = c.y.L;
    a.bias = c.bias;
    a.r = c.r ? c.r->p : nullptr; a.r_bs = c.r ? c.r->bstride : 0; a.r_ld = c.r ? c.r->ld : 0; a.r_shift = c.r_shift;
    a.alpha = c.alpha; a.accum = c.accum ? 1 : 0;
    a.stats = c.stats;
    a.nb = c.B;
    a.part = c.part;
    a.ksplit = c.part ? fwd_ksplit(c, mode, F::NPOS, c.part_cap) : 1;
    if (c.stats && c.accum) fail("conv_fwd_tc", "output statistics need a non-accumulating output");
    // the epilogue forms in-clip offsets (row * ld) in 32 bits
    if ((int64_t)c.y.L * c.y.ld >= (1ll << 31) || (c.r && (int64_t)c.r->L * c.r->ld >= (1ll << 31)))
        fail("conv_fwd_tc", "clip too long for 32-bit row offsets");
    const int grid = (int)std::min<int64_t>(tiles * a.ksplit, sm_count());
    ::bsml::count_launch();
    conv_fwd_tc_kernel<MODE, NPT, NH><<<grid, F::THREADS, g.smem, st>>>(mWh, mWl, mXh, mXl, a);
    BSML_LAUNCH("conv_fwd_tc");
    if (a.ksplit > 1) {
        ::bsml::count_launch();
        fwd_split_reduce_kernel<<<dim3((unsigned)ceil_div(c.No, FR_ROWS), (unsigned)ceil_div(c.Co, 128), (unsigned)c.B),
                                  128, 0, st>>>(a);
        BSML_LAUNCH("fwd_split_reduce");
    }
}

template <int MODE, int NH>
void launch_fwd_nh(const TcConvFwd& c, int mode, const FwdGeom& g, cudaStream_t st) {
    if (g.np == 256)
        launch_fwd_np<MODE, 256, NH>(c, mode, g, st);
    else if (g.np == 224)
        launch_fwd_np<MODE, 224, NH>(c, mode, g, st);
    else
        launch_fwd_np<MODE, 192, NH>(c, mode, g, st);
}

// Epilogue width by the K steps of a work item (taps x input-channel chunks, after
// any split): up to 32 steps the tile-end stores recur often enough to stall the
// MMAs and 16 epilogue warps win (measured: C128 k3 -8 %, k7 -2 %, BF16x3 k7 -8 %);
// longer K loops keep 8 warps with more registers (C128 k11 d5 and C1024 k3 lose
// 1-4 % with 16).
constexpr int NH4_MAX_KSTEPS = 32;

template <int MODE>
void launch_fwd(const TcConvFwd& c, int mode, cudaStream_t st) {
    const FwdGeom g = fwd_geom(Fmt<MODE>::PLANES, (c.taps - 1) * c.d);
    const int kchunks = (int)ceil_div(c.Ci, Fmt<MODE>::BKE);
    const int ks = c.part ? fwd_ksplit(c, mode, g.np, c.part_cap) : 1;
    const int64_t ksteps = (int64_t)c.taps * ceil_div(kchunks, ks);
    if (ksteps <= NH4_MAX_KSTEPS)
        launch_fwd_nh<MODE, 4>(c, mode, g, st);
    else
        launch_fwd_nh<MODE, 2>(c, mode, g, st);
}

template <int MODE>
void launch_wgrad(const TcConvWgrad& c, int mode, float* part, int64_t part_cap, cudaStream_t st) {
    using CF = WCfg<MODE>;
    constexpr bool LO = Fmt<MODE>::LO, F32E = Fmt<MODE>::F32;
    static bool attr = false;
    if (!attr) {
        BSML_CUDA(cudaFuncSetAttribute(conv_wgrad_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_OPTIN));
        attr = true;
    }
    WArgs a{};
    a.taps = c.taps; a.p = c.p; a.d = c.d; a.Co = c.Co; a.Ci = c.Ci;
    // X window: KROWS positions plus the second tap's shift
    a.wrows = (int)round_up(CF::KROWS + (c.taps > 1 ? c.d : 0), 8);
    if (a.wrows > 256) fail("conv_wgrad_tc", "dilation too large for the position window");
    a.stage_bytes = CF::A_BYTES + CF::PLANES * CF::MN_BLOCKS * a.wrows * 128;
    const int fixed = 1024 + 256;
    a.stages = std::min(CF::MAX_S, (SMEM_OPTIN - fixed) / a.stage_bytes);
    if (a.stages < 2) fail("conv_wgrad_tc", "stage too large for shared memory");
    const int smem = a.stages * a.stage_bytes + fixed;
    const uint32_t bke = CF::BKE, kr = CF::KROWS;
    // A: dY planes [B][Lo][ld] (M = Co along the contiguous dim); B: X planes (N = Ci)
    const CUtensorMap mAh = make_map(c.dy.hi, mode, c.Co, c.Lo, c.B, c.dy.ld, c.Lo, bke, kr, F32E);
    const CUtensorMap mAl = LO ? make_map(c.dy.lo, mode, c.Co, c.Lo, c.B, c.dy.ld, c.Lo, bke, kr, F32E) : mAh;
    const CUtensorMap mBh = make_map(c.x.hi, mode, c.Ci, c.L_in, c.B, c.x.ld, c.L_in, bke, a.wrows, F32E);
    const CUtensorMap mBl =
        LO ? make_map(c.x.lo, mode, c.Ci, c.L_in, c.B, c.x.ld, c.L_in, bke, a.wrows, F32E) : mBh;
    a.n_ci_tiles = (int)ceil_div(c.Ci, BN);
    a.n_pairs = (int)ceil_div(c.taps, 2);
    a.chunks_pc = (int)ceil_div(c.Lo, CF::KROWS);
    a.chunks_total = a.chunks_pc * c.B;
    // one full wave of equal CTAs (one per SM: a second wave repeats each CTA's pipeline
    // fill and epilogue, measured 2-9 % slower), each with >= 8 chunks of K, within the
    // partial budget
    const int64_t tiles = ceil_div(c.Co, BM) * a.n_ci_tiles * a.n_pairs;
    int64_t splits = std::max<int64_t>(1, sm_count() / tiles);
    splits = std::min<int64_t>(splits, ceil_div(a.chunks_total, 8));
    splits = std::min<int64_t>(splits, part_cap / ((int64_t)c.taps * c.Co * c.Ci));
    if (splits < 1) fail("conv_wgrad_tc", "split-K partial buffer too small");
    a.chunks_per_split = (int)ceil_div(a.chunks_total, splits);
    splits = ceil_div(a.chunks_total, a.chunks_per_split);
    a.part = part;
    dim3 grid((unsigned)ceil_div(c.Co, BM), (unsigned)(a.n_ci_tiles * a.n_pairs), (unsigned)splits);
    ::bsml::count_launch();
    conv_wgrad_tc_kernel<MODE><<<grid, CF::THREADS, smem, st>>>(mAh, mAl, mBh, mBl, a);
    BSML_LAUNCH("conv_wgrad_tc");
    ::bsml::count_launch();
    if (c.ct_s > 0) {
        const ConvTPack pk = convT_pack(c.ct_k, c.ct_s, c.ct_p);
        if (pk.taps != c.taps || c.Ci != c.ct_s * c.ct_Co) fail("conv_wgrad_tc", "inconsistent ConvTranspose1d packing");
        wgrad_reduce_convT_kernel<<<grid_for((int64_t)c.taps * c.Ci * c.Co), 256, 0, st>>>(
            part, (int)splits, c.taps, c.Co, c.Ci, c.ct_Co, c.ct_k, c.ct_s, c.ct_p, pk.u_min, c.dW, c.accum ? 1 : 0);
    } else {
        wgrad_reduce_kernel<<<grid_for((int64_t)c.Co * c.Ci * c.taps), 256, 0, st>>>(part, (int)splits, c.taps, c.Co,
                                                                                        c.Ci, c.dW, c.accum ? 1 : 0);
    }
    BSML_LAUNCH("wgrad_reduce");
}

}  // namespace

void make_act_planes(const Act& x, int mode, void* hi, void* lo, cudaStream_t st) {
    const int ld = tc_pitch(x.C, mode);
    if ((reinterpret_cast<uintptr_t>(x.p) & 15) == 0 && (x.ld & 3) == 0 && (x.bstride & 3) == 0) {
        PlaneOut po;
        po.hi = hi; po.lo = lo; po.ld = ld; po.mode = mode;
        scale_out_v(x, 1.f, nullptr, &po, nullptr, st);
        return;
    }
    ::bsml::count_launch();
    if (mode == TC_TF32X3)
        act_planes_kernel<TC_TF32X3><<<grid_for(x.numel()), 256, 0, st>>>(x, hi, lo, ld);
    else if (mode == TC_BF16X3)
        act_planes_kernel<TC_BF16X3><<<grid_for(x.numel()), 256, 0, st>>>(x, hi, lo, ld);
    else
        act_planes_kernel<TC_BF16><<<grid_for(x.numel()), 256, 0, st>>>(x, hi, lo, ld);
    BSML_LAUNCH("make_act_planes");
}

void wgrad_unpack_strided(const float* dW2, int Co, int Ci, int k, int s, int ld, float* dW, cudaStream_t st) {
    ::bsml::count_launch();
    wgrad_unpack_strided_kernel<<<grid_for((int64_t)Co * Ci * k), 256, 0, st>>>(dW2, Co, Ci, k, s, ld,
                                                                                 (k + s - 1) / s, dW);
    BSML_LAUNCH("wgrad_unpack_strided");
}

PackJob make_pack_job(int64_t w_off, int kind, int Co, int Ci, int k, int s, int r, void* hi, void* lo) {
    PackJob J;
    J.w_off = w_off; J.kind = kind; J.Co = Co; J.Ci = Ci; J.k = k; J.s = s; J.r = r; J.hi = hi; J.lo = lo;
    J.taps = k; J.M = Co; J.K = Ci;
    if (kind == PACK_CONV_DGRAD) { J.M = Ci; J.K = Co; }
    if (kind == PACK_CONVT_PHASE) J.taps = (k - r + s - 1) / s;
    if (kind == PACK_CONVT_DGRAD) {
        if (r < 0) fail("pack_w_tc", "negative ConvTranspose1d padding");
        J.M = Ci; J.K = s * Co; J.taps = convT_pack(k, s, r).taps;
    }
    if (kind == PACK_CONV_STRIDED) {
        if (r < Ci || s < 1) fail("pack_w_tc", "bad row-packed strided conv");
        J.K = s * r; J.taps = (k + s - 1) / s;
    }
    J.Kp = (int)round_up(J.K, 8);
    J.n = (int64_t)J.taps * J.M * J.Kp;
    J.items = (int64_t)J.M * J.Kp;
    return J;
}

void pack_w_tc_batch(const float* params, const PackJob* jobs, int n_jobs, int64_t total, int mode, cudaStream_t st) {
    if (n_jobs <= 0 || total <= 0) return;
    if (n_jobs > PACK_MAX_JOBS) fail("pack_w_tc_batch", "too many jobs in one batch");
    ::bsml::count_launch();
    if (mode == TC_TF32X3)
        pack_w_batch_kernel<TC_TF32X3><<<grid_for(total), 256, 0, st>>>(params, jobs, n_jobs, total);
    else if (mode == TC_BF16X3)
        pack_w_batch_kernel<TC_BF16X3><<<grid_for(total), 256, 0, st>>>(params, jobs, n_jobs, total);
    else
        pack_w_batch_kernel<TC_BF16><<<grid_for(total), 256, 0, st>>>(params, jobs, n_jobs, total);
    BSML_LAUNCH("pack_w_tc_batch");
}

void pack_w_tc(const float* W, int kind, int Co, int Ci, int k, int s, int r, int mode, void* hi, void* lo,
               cudaStream_t st) {
    int taps = k, M = Co, K = Ci;
    if (kind == PACK_CONV_DGRAD) { M = Ci; K = Co; }
    if (kind == PACK_CONVT_PHASE) taps = (k - r + s - 1) / s;
    if (kind == PACK_CONVT_DGRAD) {
        if (r < 0) fail("pack_w_tc", "negative ConvTranspose1d padding");
        M = Ci; K = s * Co; taps = convT_pack(k, s, r).taps;
    }
    const int Kp = (int)round_up(K, 8);
    const int64_t n = (int64_t)M * Kp;
    ::bsml::count_launch();
    if (mode == TC_TF32X3)
        pack_w_kernel<TC_TF32X3><<<grid_for(n), 256, 0, st>>>(W, kind, Co, Ci, k, s, r, taps, M, K, Kp, hi, lo);
    else if (mode == TC_BF16X3)
        pack_w_kernel<TC_BF16X3><<<grid_for(n), 256, 0, st>>>(W, kind, Co, Ci, k, s, r, taps, M, K, Kp, hi, lo);
    else
        pack_w_kernel<TC_BF16><<<grid_for(n), 256, 0, st>>>(W, kind, Co, Ci, k, s, r, taps, M, K, Kp, hi, lo);
    BSML_LAUNCH("pack_w_tc");
}

int64_t conv_fwd_tc_part_floats(const TcConvFwd& c, int mode) {
    const int planes = mode == TC_BF16 ? 1 : 2;
    const int np = fwd_geom(planes, (c.taps - 1) * c.d).np;
    const int ks = fwd_ksplit(c, mode, np, INT64_MAX);
    return ks > 1 ? (int64_t)ks * c.B * c.No * c.Co : 0;
}

void conv_fwd_tc(const TcConvFwd& c, int mode, cudaStream_t st) {
    if (c.No <= 0) return;
    if (mode == TC_TF32X3)
        launch_fwd<TC_TF32X3>(c, mode, st);
    else if (mode == TC_BF16X3)
        launch_fwd<TC_BF16X3>(c, mode, st);
    else
        launch_fwd<TC_BF16>(c, mode, st);
}

void conv_wgrad_tc(const TcConvWgrad& c, int mode, float* part, int64_t part_cap, cudaStream_t st) {
    if (c.Lo <= 0) return;
    if (mode == TC_TF32X3)
        launch_wgrad<TC_TF32X3>(c, mode, part, part_cap, st);
    else if (mode == TC_BF16X3)
        launch_wgrad<TC_BF16X3>(c, mode, part, part_cap, st);
    else
        launch_wgrad<TC_BF16>(c, mode, part, part_cap, st);
}

// One thread waits, through the same bounded wait every tensor-core kernel uses,
// on an mbarrier phase that nothing completes: after the limit it leaves
// TC_ERR_WAIT_FULL in the error word and returns (nothing in flight).
__global__ void wait_selftest_kernel() {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    tc::mbar_wait(&bar, 0, &g_tc_err, tc::TC_ERR_WAIT_FULL);
}

void tc_wait_selftest(cudaStream_t st) {
    count_launch();
    wait_selftest_kernel<<<1, 32, 0, st>>>();
    BSML_LAUNCH("wait_selftest_kernel");
}

int tc_error_flag() {
    int v = 0, zero = 0;
    BSML_CUDA(cudaDeviceSynchronize());
    BSML_CUDA(cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(int)));
    BSML_CUDA(cudaMemcpyToSymbol(g_tc_err, &zero, sizeof(int)));
    return v;
}

}  // namespace bsml
