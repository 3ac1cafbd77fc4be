// gemm.cu -- tcgen05 GEMM engine for the corpus's fp16 and int8 GEMMs.
//
// out[M,N] = epilogue( A[M,K] . B[K,N] ), A and B^T both staged K-major.
//
// Persistent, warp-specialised kernel, one CTA per SM (320 threads):
//   warp 0      TMA producer: 128 x 128-byte A box + BN x 128-byte B box per
//               stage (128-byte swizzle), kStages-deep ring of full/empty
//               mbarriers;
//   warp 1      allocates 2*BN TMEM columns (two fp32/s32 accumulators) and,
//               from one elected lane, issues tcgen05.mma (M=128, N=BN, 32 B
//               of K per instruction: K=16 f16 or K=32 int8), releasing each
//               smem stage with tcgen05.commit;
//   warps 2..9  epilogue, two warps per TMEM lane quarter (one per half of
//               the tile's columns): tcgen05.ld 32 lanes x 32 columns at a
//               time, apply the fp16 rounding or the fixed-point requant
//               (per-column parameters staged in shared memory), store to HBM,
//               then hand the accumulator back to the MMA warp.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile
// i+1.  Tiles are walked in groups sized from the L2 capacity (pick_raster):
// a panel of one operand stays resident in L2 while the other streams past it
// once per group, and the CTAs of a wave share the streamed blocks.  When
// the last wave would leave most CTAs idle, the integer GEMMs cut its tiles
// into K parts run by separate CTAs (tail split, unit_of).  A CTA-pair
// variant (gemm_tc2_kernel, cta_group::2) computes 256 x 256 tiles on two SMs.
//
// Operand preparation (HBM-bound pre-passes, only where needed): a row-major
// B[K,N] whose rows TMA can address is read in place as an MN-major operand,
// else transposed into a K-major copy; the zero-point GEMMs' int32 column
// sums of B come from a separate read of B (or from the transpose pass); an
// A whose row pitch is not a multiple of 16 bytes is copied into a padded
// buffer, because TMA rows must start on 16-byte boundaries.
//
// Every mbarrier wait is bounded (tc::mbar_wait); on expiry the kernel raises
// a CTA-wide abort flag, records the device error word, drains its own
// outstanding TMA loads and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "ew_launch.cuh"
#include "hx_internal.h"
#include "requant.cuh"
#include "tc_common.cuh"

namespace hx {
namespace {

using tc::MmaKind;

constexpr int kBM = 128;             // rows of A per tile (UMMA M)
constexpr int kBKBytes = 128;        // K extent of one stage, in bytes
constexpr int kStages = 4;
constexpr int kThreads = 320;      // TMA warp, MMA warp, 8 epilogue warps
constexpr int kColParamBytes = 6 * 32 * 4;   // one epilogue warp's ColParams
constexpr int kStoreStageBytes = 32 * 64;    // 32 rows x 64 B, one epilogue warp

enum EpiKind { kEpiF16 = 0, kEpiRequant = 1, kEpiHmx = 2, kEpiF16Ex = 3 };

// Activations of the HMX epilogue used only by the FFN compositions below
// (the public entries accept HEXCUDA_HMX_ACT_* only): an arithmetic right
// shift by post_shift after the bias, with ReLU (v > 0 ? v >> s : 0) or
// without it.
constexpr int kActReluShr = 16, kActShr = 17;

struct EpiParams {
    void *out;
    int64_t ldo;               // output row pitch, elements
    int M, N;
    // requant epilogue (int8 GEMMs):
    //   acc32  = rawdot - zpA * colsum[j]      (int32 wrap, as the C reference)
    //   x      = (int64) acc32 + bias[j]
    //   q      = sat(round_half_away(x * mult_j >> shift_j) + zp, lo, hi)
    const int32_t *colsum;     // null: no zero-point term
    int32_t zpA;
    const int32_t *bias;       // null: no bias
    const int32_t *mult_pc;    // null: scalar mult / shift
    const int *shift_pc;
    int32_t mult;
    int shift;
    int zp;
    int lo, hi;
    int relu_pre;              // requant: x = max(x, 0) after the bias add
    // HMX-convention epilogue (kEpiHmx): acc32 as above, then
    //   v = sx12((acc32 * 17 + 8) >> 4)    (int32 wrap, arithmetic shift)
    //   v += bias[j] (null: 0); v += res[i][j] (res_kind 1 int32, 2 int8,
    //   row-major [M, N]); activation; store (HEXCUDA_HMX_STORE_* of
    //   hexcuda.h); col_major stores out[j * ldo + i].  All adds wrap.
    int hmx_store, hmx_act, res_kind, col_major;
    int post_shift;            // kActReluShr / kActShr
    const void *res;
    const void *lut;
    // hmx_raw: the raw accumulator instead of the sx12 field, with the bias,
    // residual and activation in int64 before the store's saturation (the
    // int8 GEMM callers that widen to int64 before they saturate)
    int hmx_raw;
    // requant epilogue: int8 residual [M, N] added with int8 saturation
    // after the requant's clamp (null: none)
    const int8_t *rq_res;
    // fp16 post-ops (kEpiF16Ex), in the corpus's order: v = acc + res[i][j]
    // (fp16 [M, N] or null) + bias[j] (fp16 or null); preround: v = fp16(v);
    // activation (HEXCUDA_F16_ACT_*); v *= scale; out = fp16(v)
    const __half *f16_bias, *f16_res;
    int f16_act, f16_preround;
    float f16_scale;
};

struct GemmArgs {
    int tiles_m, tiles_n, num_kb;
    // rasterisation: consecutive tiles walk `group` blocks of one dimension
    // (M-blocks when group_n_major == 0, N-blocks otherwise) before moving
    // along the other, so the group's panel of that operand stays in L2
    int group, group_n_major;
    // work units (unit_of): tiles [0, dp_tiles) whole, then `split` K parts
    // of each remaining tile; part_flag / part_ws hold the parts' arrival
    // flags and raw accumulators, ticket is this launch's serial number
    int units, dp_tiles, split;
    uint32_t ticket;
    int *part_flag;
    int32_t *part_ws;
    int *err_word;
    EpiParams epi;
};

template <int BN>
struct Smem {
    static constexpr int kABytes = kBM * kBKBytes;        // 16 KB
    static constexpr int kBBytes = BN * kBKBytes;         // 16 or 32 KB
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kBarOffset = kStages * kStageBytes;
    // full[S], empty[S], tfull[2], tempty[2], drain
    static constexpr int kNumBars = 2 * kStages + 5;
    // per epilogue warp: the requant parameters of its current 32 columns,
    // read with 16-byte loads, so the region starts on a 128-byte boundary
    static constexpr int kParamOffset = (kBarOffset + kNumBars * 8 + 16 + 127) / 128 * 128;
    static constexpr int kParamBytes = 8 * kColParamBytes;
    // per epilogue warp: a 2 KB staging block for coalesced 4-byte stores
    static constexpr int kStoreOffset = kParamOffset + kParamBytes;
    static constexpr int kTotal = kStoreOffset + 8 * kStoreStageBytes + 1024;  // + align slack
};

// Tile t -> (M-block, N-block): groups of `group` blocks of the resident
// dimension, walked across the other dimension; inside a group the resident
// dimension varies fastest, so the CTAs of a wave share the streamed operand's
// blocks too.
__device__ __forceinline__ void tile_coords(int t, const GemmArgs &a, int &mb, int &nb) {
    const int along = a.group_n_major ? a.tiles_n : a.tiles_m;   // resident dimension
    const int across = a.group_n_major ? a.tiles_m : a.tiles_n;
    const int per_group = a.group * across;
    const int g = t / per_group;
    const int first = g * a.group;
    const int gsize = min(along - first, a.group);
    const int r = t - g * per_group;
    const int res = first + r % gsize, str = r / gsize;
    mb = a.group_n_major ? str : res;
    nb = a.group_n_major ? res : str;
}

// Work units of the persistent kernels.  Tiles [0, dp_tiles) run whole; each
// remaining tile (the last, partial wave) is cut into `split` K ranges that
// different CTAs (CTA pairs) run at the same time.  Part 0 owns the tile: its
// epilogue warps wait until parts 1..split-1 have left their raw accumulators
// in the workspace, add them and run the epilogue.  A part p >= 1 stores its
// accumulator and sets its flag (one per epilogue warp) to the launch's
// ticket.  The host makes dp_tiles a multiple of the grid and the parts at
// most one grid, so every part is its CTA's last unit: a part p >= 1 never
// waits, and the CTAs that run them have only whole tiles before them.
struct Unit {
    int t;          // tile
    int kb0, kb1;   // K blocks [kb0, kb1)
    int part;       // -1: whole tile; else this unit's K part of tile t
};

__device__ __forceinline__ Unit unit_of(int u, const GemmArgs &a) {
    Unit w;
    if (u < a.dp_tiles) {
        w.t = u;
        w.kb0 = 0;
        w.kb1 = a.num_kb;
        w.part = -1;
        return w;
    }
    const int i = u - a.dp_tiles;
    w.t = a.dp_tiles + i / a.split;
    w.part = i % a.split;
    w.kb0 = (int)((int64_t)w.part * a.num_kb / a.split);
    w.kb1 = (int)((int64_t)(w.part + 1) * a.num_kb / a.split);
    return w;
}

// Flag / workspace slot of (split tile, part p >= 1, CTA rank of the pair,
// epilogue warp); a workspace slot holds one epilogue warp's 32 rows x
// `cols` columns of int32 as [cols / 32][8][lane][4]: the warp's 32 lanes
// store (and the owner's lanes load) 512 contiguous bytes per instruction.
__device__ __forceinline__ size_t part_slot(const GemmArgs &a, int t, int p, int rank,
                                            int nranks, int warp_slot) {
    return (((size_t)(t - a.dp_tiles) * (a.split - 1) + (p - 1)) * nranks + rank) * 8 + warp_slot;
}

__device__ __forceinline__ void part_store(int32_t *ws, int chunk, int lane,
                                           const uint32_t (&r)[32]) {
    int4 *dst = reinterpret_cast<int4 *>(ws) + (size_t)chunk * 256 + lane;
#pragma unroll
    for (int e = 0; e < 8; e++)
        dst[e * 32] =
            make_int4((int)r[4 * e], (int)r[4 * e + 1], (int)r[4 * e + 2], (int)r[4 * e + 3]);
}

// r += the stored part (int32 wrap-around, or fp32 for the fp16 GEMMs); the
// loads bypass L1, whose lines are not kept coherent with other SMs' stores
template <bool F32>
__device__ __forceinline__ void part_add(const int32_t *ws, int chunk, int lane, uint32_t (&r)[32]) {
    const int4 *src = reinterpret_cast<const int4 *>(ws) + (size_t)chunk * 256 + lane;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int4 v = __ldcg(src + e * 32);
        const int w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t &x = r[4 * e + i];
            x = F32 ? __float_as_uint(__uint_as_float(x) + __int_as_float(w[i]))
                    : x + (uint32_t)w[i];
        }
    }
}

__device__ __forceinline__ void part_flag_set(int *f, uint32_t ticket) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(ticket) : "memory");
}

// Bounded wait for a part's flag to reach this launch's ticket (kWaitBudgetNs;
// on expiry the device error word gets kErrWaitPart and the CTA aborts).
__device__ __forceinline__ bool part_flag_wait(const int *f, uint32_t ticket, volatile int *abort,
                                               int *err_word) {
    const uint64_t t0 = tc::globaltimer();
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (v == ticket) return true;
        if (*abort) return false;
        if (tc::globaltimer() - t0 > kWaitBudgetNs) {
            atomicOr(err_word, kErrWaitPart);
            *abort = 1;
            return false;
        }
        __nanosleep(128);
    }
}

// Owner of a split tile: adds the `nparts` other parts of this epilogue
// warp's 32 rows x COLS columns (the first at ws, the next `stride` words on)
// into its accumulator in TMEM (taddr = the warp's lane quarter and first
// column), before the ordinary epilogue reads it.
template <bool F32, int COLS>
__device__ __forceinline__ void merge_parts(const int32_t *ws, size_t stride, int nparts,
                                            uint32_t taddr, int lane) {
#pragma unroll 1
    for (int c = 0; c < COLS; c += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(taddr + (uint32_t)c, r);
        tc::tmem_ld_wait(r);
#pragma unroll 1
        for (int p = 0; p < nparts; p++) part_add<F32>(ws + p * stride, c / 32, lane, r);
        tc::tmem_st_32x32b_x32(taddr + (uint32_t)c, r);
    }
    tc::tmem_st_wait();
}

// Requant parameters of one epilogue warp's current 32 columns; half is the
// rounding term 2^(shift-1) (0 for shift 0) as two 32-bit words.
struct ColParams {
    int32_t corr[32], bias[32], mult[32], shift[32];
    uint32_t half_lo[32], half_hi[32];
};
static_assert(sizeof(ColParams) == kColParamBytes, "per-warp parameter slice");

// Rounded magnitudes at or above kMagCap saturate every clamp of the requant
// epilogue (the host keeps |zp|, |lo|, |hi| below 2^19), so the magnitude is
// capped there and the zero point and clamps run in 32 bits.
constexpr uint32_t kMagCap = 1u << 20;

// 32 requantised columns of one row -> 8 words of packed 8-bit outputs:
//   x = (int64)(acc32 - corr_j) + bias_j; RELU: x = max(x, 0)
//   v = x * mult_j (int64 wrap); q = sign(v) ((|v| + half_j) >> shift_j)
//   out = clamp(q + zp, lo, hi)   (upper clamp first, as the reference)
template <bool RELU>
__device__ __forceinline__ void requant_chunk(const EpiParams &ep, const uint32_t (&r)[32],
                                              const ColParams *cp, uint32_t (&w)[8]) {
#pragma unroll
    for (int i4 = 0; i4 < 8; i4++) {
        const int4 c4 = *reinterpret_cast<const int4 *>(&cp->corr[4 * i4]);
        const int4 b4 = *reinterpret_cast<const int4 *>(&cp->bias[4 * i4]);
        const int4 m4 = *reinterpret_cast<const int4 *>(&cp->mult[4 * i4]);
        const int4 s4 = *reinterpret_cast<const int4 *>(&cp->shift[4 * i4]);
        const uint4 hl4 = *reinterpret_cast<const uint4 *>(&cp->half_lo[4 * i4]);
        const uint4 hh4 = *reinterpret_cast<const uint4 *>(&cp->half_hi[4 * i4]);
        const int cc[4] = {c4.x, c4.y, c4.z, c4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
        const int mm[4] = {m4.x, m4.y, m4.z, m4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
        const uint32_t hl[4] = {hl4.x, hl4.y, hl4.z, hl4.w}, hh[4] = {hh4.x, hh4.y, hh4.z, hh4.w};
        uint32_t q[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int32_t a32 = (int32_t)(r[4 * i4 + u] - (uint32_t)cc[u]);
            int64_t xb = (int64_t)a32 + bb[u];
            if (RELU && xb < 0) xb = 0;
            const int64_t v = (int64_t)((uint64_t)xb * (uint64_t)(int64_t)mm[u]);
            const uint64_t av = v < 0 ? 0ull - (uint64_t)v : (uint64_t)v;
            const uint64_t mag = (av + (((uint64_t)hh[u] << 32) | hl[u])) >> ss[u];
            const int32_t m32 = mag >= kMagCap ? (int32_t)kMagCap : (int32_t)mag;
            int32_t x = (v < 0 ? -m32 : m32) + ep.zp;
            x = x > ep.hi ? ep.hi : x;
            x = x < ep.lo ? ep.lo : x;
            q[u] = (uint32_t)x;
        }
        w[i4] = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const EpiParams &ep, const uint32_t (&r)[32],
                                               int row, int col0, const ColParams *cp,
                                               uint4 *stage) {
    if constexpr (EPI == kEpiF16) {
        const int lane = threadIdx.x & 31;
        __half *o0 = reinterpret_cast<__half *>(ep.out) + (size_t)(row - lane) * ep.ldo + col0;
        if (col0 + 32 <= ep.N && (ep.ldo & 7) == 0 && (reinterpret_cast<uintptr_t>(o0) & 15u) == 0) {
            // warp-uniform: the warp's 32 rows x 32 fp16 through the staging block
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; i++) {
                __half2 h = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                w[i] = *reinterpret_cast<uint32_t *>(&h);
            }
            tc::store_block_coalesced(w, stage, reinterpret_cast<uint8_t *>(o0), (size_t)ep.ldo * 2,
                                  min(32, ep.M - (row - lane)));
            return;
        }
        if (row >= ep.M) return;
        __half *o = reinterpret_cast<__half *>(ep.out) + (size_t)row * ep.ldo + col0;
        if (col0 + 32 <= ep.N && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
            uint4 v[4];
            uint32_t *w = reinterpret_cast<uint32_t *>(v);
#pragma unroll
            for (int i = 0; i < 16; i++) {
                __half2 h = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
                w[i] = *reinterpret_cast<uint32_t *>(&h);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(o);
#pragma unroll
            for (int i = 0; i < 4; i++) dst[i] = v[i];
        } else {
            for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = __float2half_rn(__uint_as_float(r[i]));
        }
    } else if constexpr (EPI == kEpiF16Ex) {
        // rows past M compute on (unused) accumulators and store nothing
        const __half *rr =
            (ep.f16_res && row < ep.M) ? ep.f16_res + (size_t)row * ep.N + col0 : nullptr;
        __half hv[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int j = col0 + i;
            float v = __uint_as_float(r[i]);
            if (ep.f16_preround == HEXCUDA_F16_PREROUND_ACC) v = __half2float(__float2half_rn(v));
            if (j < ep.N) {
                if (rr) v += __half2float(rr[i]);
                if (ep.f16_bias) v += __half2float(ep.f16_bias[j]);
            }
            if (ep.f16_preround == HEXCUDA_F16_PREROUND_SUM) v = __half2float(__float2half_rn(v));
            if (ep.f16_act == HEXCUDA_F16_ACT_RELU) {
                v = v > 0.0f ? v : 0.0f;
            } else if (ep.f16_act == HEXCUDA_F16_ACT_LEAKY) {
                v = v > 0.0f ? v : v * 0.125f;
            } else if (ep.f16_act == HEXCUDA_F16_ACT_GELU) {
                const float c = 0.7978845608f * (v + 0.044715f * v * v * v);
                v = 0.5f * v * (1.0f + tanhf(c));
            } else if (ep.f16_act == HEXCUDA_F16_ACT_SIGMOID) {
                v = 1.0f / (1.0f + expf(-v));
            } else if (ep.f16_act == HEXCUDA_F16_ACT_TANH) {
                v = tanhf(v);
            }
            hv[i] = __float2half_rn(v * ep.f16_scale);
        }
        const int lane = threadIdx.x & 31;
        __half *o0 = reinterpret_cast<__half *>(ep.out) + (size_t)(row - lane) * ep.ldo + col0;
        if (col0 + 32 <= ep.N && (ep.ldo & 7) == 0 && (reinterpret_cast<uintptr_t>(o0) & 15u) == 0) {
            // warp-uniform: the warp's 32 rows x 32 fp16 through the staging block
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; i++) w[i] = reinterpret_cast<const uint32_t *>(hv)[i];
            tc::store_block_coalesced(w, stage, reinterpret_cast<uint8_t *>(o0), (size_t)ep.ldo * 2,
                                  min(32, ep.M - (row - lane)));
            return;
        }
        if (row >= ep.M) return;
        __half *o = reinterpret_cast<__half *>(ep.out) + (size_t)row * ep.ldo + col0;
        if (col0 + 32 <= ep.N && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
            const uint4 *src = reinterpret_cast<const uint4 *>(hv);
            uint4 *dst = reinterpret_cast<uint4 *>(o);
#pragma unroll
            for (int i = 0; i < 4; i++) dst[i] = src[i];
        } else {
            for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = hv[i];
        }
    } else if constexpr (EPI == kEpiHmx) {
        // residual of this row's 32 columns (rows past M are never stored)
        int32_t rv[32];
#pragma unroll
        for (int i = 0; i < 32; i++) rv[i] = 0;
        const bool full = col0 + 32 <= ep.N;
        if (ep.res_kind != 0 && row < ep.M) {
            const size_t base = (size_t)row * ep.N + col0;
            if (ep.res_kind == 1) {
                const int32_t *rp = reinterpret_cast<const int32_t *>(ep.res) + base;
                if (full && (reinterpret_cast<uintptr_t>(rp) & 15u) == 0) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int4 t = __ldg(reinterpret_cast<const int4 *>(rp) + i);
                        rv[4 * i] = t.x, rv[4 * i + 1] = t.y, rv[4 * i + 2] = t.z, rv[4 * i + 3] = t.w;
                    }
                } else {
                    for (int i = 0; i < 32 && col0 + i < ep.N; i++) rv[i] = __ldg(rp + i);
                }
            } else {
                const int8_t *rp = reinterpret_cast<const int8_t *>(ep.res) + base;
                for (int i = 0; i < 32 && col0 + i < ep.N; i++) rv[i] = __ldg(rp + i);
            }
        }
        int32_t v[32];
#pragma unroll
        for (int i4 = 0; i4 < 8; i4++) {
            const int4 c4 = *reinterpret_cast<const int4 *>(&cp->corr[4 * i4]);
            const int4 b4 = *reinterpret_cast<const int4 *>(&cp->bias[4 * i4]);
            const int cc[4] = {c4.x, c4.y, c4.z, c4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t a32 = r[4 * i4 + u] - (uint32_t)cc[u];
                if (ep.hmx_raw) {
                    int64_t x = (int64_t)(int32_t)a32 + bb[u] + rv[4 * i4 + u];
                    if (ep.hmx_act == HEXCUDA_HMX_ACT_RELU) x = x > 0 ? x : 0;
                    else if (ep.hmx_act == HEXCUDA_HMX_ACT_LEAKY_SHR3) x = x >= 0 ? x : (x >> 3);
                    switch (ep.hmx_store) {
                    case HEXCUDA_HMX_STORE_I8_SAT: x = x > 127 ? 127 : (x < -128 ? -128 : x); break;
                    case HEXCUDA_HMX_STORE_U8_SAT: x = x > 255 ? 255 : (x < 0 ? 0 : x); break;
                    case HEXCUDA_HMX_STORE_U16_FIELD: x &= 0xFFF; break;
                    case HEXCUDA_HMX_STORE_LUT_I32:
                        x = __ldg(reinterpret_cast<const int32_t *>(ep.lut) +
                                  (x + 128 > 255 ? 255 : (x + 128 < 0 ? 0 : x + 128)));
                        break;
                    case HEXCUDA_HMX_STORE_LUT_I8:
                        x = __ldg(reinterpret_cast<const int8_t *>(ep.lut) +
                                  ((x > 127 ? 127 : (x < -128 ? -128 : x)) + 128));
                        break;
                    default: break;
                    }
                    v[4 * i4 + u] = (int32_t)x;
                    continue;
                }
                const int32_t f = (int32_t)(a32 * 17u + 8u) >> 4;
                uint32_t xu = (uint32_t)((int32_t)((uint32_t)f << 20) >> 20);  // sx12
                if (ep.hmx_store == HEXCUDA_HMX_STORE_ACC_I32) xu = a32;     // raw accumulator
                xu += (uint32_t)bb[u] + (uint32_t)rv[4 * i4 + u];
                int32_t x = (int32_t)xu;
                if (ep.hmx_act == HEXCUDA_HMX_ACT_RELU) x = max(x, 0);
                else if (ep.hmx_act == HEXCUDA_HMX_ACT_LEAKY_SHR3) x = x >= 0 ? x : (x >> 3);
                else if (ep.hmx_act == kActReluShr) x = x > 0 ? (x >> ep.post_shift) : 0;
                else if (ep.hmx_act == kActShr) x >>= ep.post_shift;
                switch (ep.hmx_store) {
                case HEXCUDA_HMX_STORE_I8_SAT: x = min(max(x, -128), 127); break;
                case HEXCUDA_HMX_STORE_U8_SAT: x = min(max(x, 0), 255); break;
                case HEXCUDA_HMX_STORE_U16_FIELD: x &= 0xFFF; break;
                case HEXCUDA_HMX_STORE_LUT_I32:
                    x = __ldg(reinterpret_cast<const int32_t *>(ep.lut) + min(max(x + 128, 0), 255));
                    break;
                case HEXCUDA_HMX_STORE_LUT_I8:
                    x = __ldg(reinterpret_cast<const int8_t *>(ep.lut) + (min(max(x, -128), 127) + 128));
                    break;
                default: break;  // I32; I8_LOW keeps the low byte at the store
                }
                v[4 * i4 + u] = x;
            }
        }
        const int es = (ep.hmx_store == HEXCUDA_HMX_STORE_I32 ||
                        ep.hmx_store == HEXCUDA_HMX_STORE_LUT_I32 ||
                        ep.hmx_store == HEXCUDA_HMX_STORE_ACC_I32) ? 4
                       : ep.hmx_store == HEXCUDA_HMX_STORE_U16_FIELD ? 2 : 1;
        const int lane = threadIdx.x & 31;
        int32_t *o0 = reinterpret_cast<int32_t *>(ep.out) + (size_t)(row - lane) * ep.ldo + col0;
        // (warp-uniform: col0, the row block and the pointers are the same in
        // every lane of the warp)
        if (es == 4 && !ep.col_major && full && (ep.ldo & 3) == 0 &&
            (reinterpret_cast<uintptr_t>(o0) & 15u) == 0) {
            // 32 rows x 32 int32: two 64-byte halves through the staging block
            const int nrows = min(32, ep.M - (row - lane));
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; i++) w[i] = (uint32_t)v[16 * half + i];
                tc::store_block_coalesced(w, stage, reinterpret_cast<uint8_t *>(o0 + 16 * half),
                                      (size_t)ep.ldo * 4, nrows);
            }
            return;
        }
        uint8_t *ob0 = reinterpret_cast<uint8_t *>(ep.out) + ((size_t)(row - lane) * ep.ldo + col0) * es;
        if (es < 4 && !ep.col_major && full && ((ep.ldo * es) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(ob0) & 15u) == 0) {
            const int nrows = min(32, ep.M - (row - lane));
            if (es == 2) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; i++)
                    w[i] = ((uint32_t)v[2 * i] & 0xFFFFu) | ((uint32_t)v[2 * i + 1] << 16);
                tc::store_block_coalesced(w, stage, ob0, (size_t)ep.ldo * 2, nrows);
            } else {
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; i++)
                    w[i] = ((uint32_t)v[4 * i] & 0xFFu) | (((uint32_t)v[4 * i + 1] & 0xFFu) << 8) |
                           (((uint32_t)v[4 * i + 2] & 0xFFu) << 16) | ((uint32_t)v[4 * i + 3] << 24);
                tc::store_block32_coalesced(w, stage, ob0, (size_t)ep.ldo, nrows);
            }
            return;
        }
        if (row >= ep.M) return;
        if (ep.col_major) {
            // lanes are consecutive rows: each column's store is one
            // contiguous run across the warp
            for (int i = 0; i < 32 && col0 + i < ep.N; i++) {
                const size_t o = (size_t)(col0 + i) * ep.ldo + row;
                if (es == 4) reinterpret_cast<int32_t *>(ep.out)[o] = v[i];
                else if (es == 2) reinterpret_cast<uint16_t *>(ep.out)[o] = (uint16_t)v[i];
                else reinterpret_cast<uint8_t *>(ep.out)[o] = (uint8_t)v[i];
            }
        } else if (es == 4) {
            int32_t *o = reinterpret_cast<int32_t *>(ep.out) + (size_t)row * ep.ldo + col0;
            if (full && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
                uint4 *dst = reinterpret_cast<uint4 *>(o);
#pragma unroll
                for (int i = 0; i < 8; i++)
                    dst[i] = make_uint4((uint32_t)v[4 * i], (uint32_t)v[4 * i + 1],
                                        (uint32_t)v[4 * i + 2], (uint32_t)v[4 * i + 3]);
            } else {
                for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = v[i];
            }
        } else if (es == 2) {
            uint16_t *o = reinterpret_cast<uint16_t *>(ep.out) + (size_t)row * ep.ldo + col0;
            if (full && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
                uint4 *dst = reinterpret_cast<uint4 *>(o);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    uint32_t w[4];
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        w[k] = ((uint32_t)v[8 * i + 2 * k] & 0xFFFFu) |
                               ((uint32_t)v[8 * i + 2 * k + 1] << 16);
                    dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            } else {
                for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = (uint16_t)v[i];
            }
        } else {
            uint8_t *o = reinterpret_cast<uint8_t *>(ep.out) + (size_t)row * ep.ldo + col0;
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                w[i] = ((uint32_t)v[4 * i] & 0xFFu) | (((uint32_t)v[4 * i + 1] & 0xFFu) << 8) |
                       (((uint32_t)v[4 * i + 2] & 0xFFu) << 16) | ((uint32_t)v[4 * i + 3] << 24);
            if (full && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
                uint4 *dst = reinterpret_cast<uint4 *>(o);
                dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
                for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = (uint8_t)v[i];
            }
        }
    } else {
        // requant: the 32 columns' parameters were staged in `cp` by this warp
        uint8_t *o = reinterpret_cast<uint8_t *>(ep.out) + (size_t)row * ep.ldo + col0;
        uint32_t w[8];
        if (ep.relu_pre)
            requant_chunk<true>(ep, r, cp, w);
        else
            requant_chunk<false>(ep, r, cp, w);
        if (ep.rq_res && row < ep.M) {
            // q = sat8(q + res[i][j]): one signed saturating byte add per 4
            const int8_t *rp = ep.rq_res + (size_t)row * ep.N + col0;
#pragma unroll
            for (int i4 = 0; i4 < 8; i4++) {
                uint32_t rw = 0;
                for (int u = 0; u < 4 && col0 + 4 * i4 + u < ep.N; u++)
                    rw |= (uint32_t)(uint8_t)__ldg(rp + 4 * i4 + u) << (8 * u);
                w[i4] = __vaddss4(w[i4], rw);
            }
        }
        const int lane = threadIdx.x & 31;
        uint8_t *o0 = o - (size_t)lane * ep.ldo;
        if (col0 + 32 <= ep.N && (ep.ldo & 15) == 0 && (reinterpret_cast<uintptr_t>(o0) & 15u) == 0) {
            // warp-uniform: the warp's 32 rows x 32 bytes through the staging block
            tc::store_block32_coalesced(w, stage, o0, (size_t)ep.ldo, min(32, ep.M - (row - lane)));
            return;
        }
        if (row >= ep.M) return;
        if (col0 + 32 <= ep.N && ((reinterpret_cast<uintptr_t>(o) & 15u) == 0)) {
            uint4 *dst = reinterpret_cast<uint4 *>(o);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
            for (int i = 0; i < 32 && col0 + i < ep.N; i++) o[i] = (uint8_t)(w[i >> 2] >> (8 * (i & 3)));
        }
    }
}

// Stage the requant parameters of columns col0..col0+31 (lane = column) into
// the warp's shared-memory slice: zpA * colsum[j] (int32 wrap), bias[j],
// mult[j], shift[j] clamped to 0..63 (the C reference is undefined beyond)
// and its rounding term.
__device__ __forceinline__ void stage_params(const EpiParams &ep, ColParams *cp, int col0,
                                             int lane) {
    const int j = col0 + lane;
    int32_t c = 0, b = 0, m = ep.mult, sh = ep.shift;
    if (j < ep.N) {
        if (ep.colsum) c = (int32_t)((uint32_t)ep.zpA * (uint32_t)__ldg(ep.colsum + j));
        if (ep.bias) b = __ldg(ep.bias + j);
        if (ep.mult_pc) m = __ldg(ep.mult_pc + j);
        if (ep.shift_pc) sh = __ldg(ep.shift_pc + j);
    }
    sh = sh < 0 ? 0 : (sh > 63 ? 63 : sh);
    const uint64_t half = sh > 0 ? 1ull << (sh - 1) : 0ull;
    cp->corr[lane] = c;
    cp->bias[lane] = b;
    cp->mult[lane] = m;
    cp->shift[lane] = sh;
    cp->half_lo[lane] = (uint32_t)half;
    cp->half_hi[lane] = (uint32_t)(half >> 32);
}

template <MmaKind KIND, int BN, int EPI, bool A_SIGNED, bool B_SIGNED, bool B_MN = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
    // B_MN: B is read straight from its row-major [K, N] layout as an MN-major
    // operand: per stage BN/(128/esize) boxes of (128 bytes of N) x (one K
    // block of rows), each box a column of 128-byte swizzle atoms.
    constexpr int kEsize = KIND == MmaKind::F16 ? 2 : 1;
    constexpr int kKElems = kBKBytes / kEsize;          // K rows per stage
    constexpr int kNBox = 128 / kEsize;                 // N elements per box
    constexpr int kBoxBytes = kKElems * 128;            // one MN-major box
    using L = Smem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + kStages;
    uint64_t *tfull = bars + 2 * kStages;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr uint32_t kTmemCols = 2 * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 8);   // one arrive per epilogue warp
        }
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch_desc(&tmA);
        tc::tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0;    // bit s: stage s has a load in flight we may need to drain
            uint32_t armed_phase = 0;
            for (int u = blockIdx.x; u < args.units && !*abort_flag; u += gridDim.x) {
                const Unit w = unit_of(u, args);
                int mb, nb;
                tile_coords(w.t, args, mb, nb);
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err_word,
                                       kErrWaitEmpty))
                        break;
                    uint8_t *sa = smem + stage * L::kStageBytes;
                    uint8_t *sb = sa + L::kABytes;
                    tc::mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
                    const int kx = kb * (KIND == MmaKind::F16 ? kBKBytes / 2 : kBKBytes);
                    tc::tma_load_2d(sa, &tmA, &full[stage], kx, mb * kBM);
                    if constexpr (B_MN) {
#pragma unroll
                        for (int c = 0; c < BN / kNBox; c++)
                            tc::tma_load_2d(sb + c * kBoxBytes, &tmB, &full[stage],
                                            nb * BN + c * kNBox, kx);
                    } else {
                        tc::tma_load_2d(sb, &tmB, &full[stage], kx, nb * BN);
                    }
                    armed |= 1u << stage;
                    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain: every load this thread issued must land before the CTA
            // exits (normally all were consumed already and this is a no-op).
            for (int s = 0; s < kStages; s++)
                if (armed & (1u << s)) {
                    const uint64_t t0 = tc::globaltimer();
                    while (!tc::mbar_try_wait(&full[s], (armed_phase >> s) & 1u) &&
                           tc::globaltimer() - t0 < kWaitBudgetNs) {
                    }
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            constexpr uint32_t idesc = (KIND == MmaKind::F16)
                                           ? tc::idesc_f16_f32(kBM, BN, B_MN)
                                           : tc::idesc_i8_s32(kBM, BN, A_SIGNED, B_SIGNED, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool issued = false;
            for (int u = blockIdx.x; u < args.units && !*abort_flag; u += gridDim.x, local++) {
                const Unit w = unit_of(u, args);
                const int buf = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!tc::mbar_wait(&tempty[buf], aphase ^ 1, abort_flag, args.err_word,
                                   kErrWaitAccum))
                    break;
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!tc::mbar_wait(&full[stage], phase, abort_flag, args.err_word,
                                       kErrWaitFull))
                        break;
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * L::kStageBytes);
                    const uint32_t sb = sa + L::kABytes;
#pragma unroll
                    for (int k = 0; k < kBKBytes / 32; k++) {
                        const uint64_t ad = tc::sdesc_kmajor_sw128(sa + k * 32);
                        // one MMA consumes 32 bytes of K: 32 bytes of each
                        // K-major row, or 32/esize rows of an MN-major box
                        const uint64_t bd =
                            B_MN ? tc::sdesc_mnmajor_sw128(sb + k * (32 / kEsize) * 128, kBoxBytes, 1024)
                                 : tc::sdesc_kmajor_sw128(sb + k * 32);
                        tc::mma_ss<KIND>(d_tmem, ad, bd, idesc, (kb != w.kb0 || k != 0) ? 1u : 0u);
                    }
                    issued = true;
                    tc::mma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit(&tfull[buf]);
            }
            // Drain: wait until every MMA issued by this thread has finished.
            if (issued) {
                tc::mma_commit(drain);
                const uint64_t t0 = tc::globaltimer();
                while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < kWaitBudgetNs) {
                }
            }
        }
    } else {
        // The column sums come from the kernel launched just before this one,
        // which may still be running (programmatic dependent launch): wait
        // for it before the first epilogue (a no-op without a prerequisite).
        if (args.epi.colsum) tc::grid_dependency_wait();
        // ---------------- epilogue warps 2..9: TMEM lane quarter = warp % 4,
        // column half = (warp - 2) / 4.  Every decision below is warp-uniform
        // (__all_sync / __any_sync), so the .sync.aligned TMEM loads always run
        // with the full warp.
        const int q = warp & 3;
        const int chalf = (warp - 2) >> 2;
        ColParams *cp = reinterpret_cast<ColParams *>(smem + L::kParamOffset) + (warp - 2);
        uint4 *stage = reinterpret_cast<uint4 *>(smem + L::kStoreOffset + (warp - 2) * kStoreStageBytes);
        const int wslot = warp - 2;
        constexpr size_t kPartWords = (size_t)(BN / 2) * 32;
        int local = 0;
        for (int u = blockIdx.x; u < args.units && !__any_sync(0xffffffffu, *abort_flag);
             u += gridDim.x, local++) {
            const Unit w = unit_of(u, args);
            int mb, nb;
            tile_coords(w.t, args, mb, nb);
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            bool ok = tc::mbar_wait(&tfull[buf], aphase, abort_flag, args.err_word, kErrWaitAccum);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc::tc_fence_after();
            const int row = mb * kBM + q * 32 + lane;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
            if (w.part >= 1) {
                // a K part of a split tile: raw accumulator to the workspace
                const size_t ps = part_slot(args, w.t, w.part, 0, 1, wslot);
                int32_t *ws = args.part_ws + ps * kPartWords;
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 32) {
                    uint32_t r[32];
                    tc::tmem_ld_32x32b_x32(taddr + (uint32_t)(chalf * (BN / 2) + c), r);
                    tc::tmem_ld_wait(r);
                    part_store(ws, c / 32, lane, r);
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) part_flag_set(args.part_flag + ps, args.ticket);
            } else {
                if (w.part == 0) {
                    // owner of a split tile: the other parts' accumulators are
                    // added into this warp's TMEM columns first
                    for (int p = 1; p < args.split && ok; p++)
                        ok = part_flag_wait(args.part_flag + part_slot(args, w.t, p, 0, 1, wslot),
                                            args.ticket, abort_flag, args.err_word);
                    if (!__all_sync(0xffffffffu, ok)) break;
                    merge_parts<KIND == MmaKind::F16, BN / 2>(
                        args.part_ws + part_slot(args, w.t, 1, 0, 1, wslot) * kPartWords,
                        8 * kPartWords, args.split - 1, taddr + (uint32_t)(chalf * (BN / 2)), lane);
                }
#pragma unroll 1
                for (int c = chalf * (BN / 2); c < (chalf + 1) * (BN / 2); c += 32) {
                    uint32_t r[32];
                    if constexpr (EPI == kEpiRequant || EPI == kEpiHmx) {
                        stage_params(args.epi, cp, nb * BN + c, lane);
                    }
                    __syncwarp();
                    tc::tmem_ld_32x32b_x32(taddr + (uint32_t)c, r);
                    tc::tmem_ld_wait(r);
                    epilogue_chunk<EPI>(args.epi, r, row, nb * BN + c, cp, stage);
                    __syncwarp();
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[buf]);
        }
    }

    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tc::tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------- CTA-pair kernel (cta_group::2)
//
// Same roles and epilogues as gemm_tc_kernel, on 256 x 256 output tiles
// computed by a cluster of two CTAs on two SMs.  CTA r of the pair stages
// rows [256 mb + 128 r, +128) of A and columns [256 nb + 128 r, +128) of B;
// the even CTA's MMA thread issues M = 256, N = 256 MMAs that read both
// CTAs' stages and leave rows 128 r.. of the tile in CTA r's tensor memory.
// Per SM a stage is 32 KB for the same MMA time that a 48 KB stage of the
// 128 x 256 tile feeds, so operand traffic per SM drops by a third and six
// stages fit in shared memory.
//
// Barriers: full[s] lives in the even CTA (both CTAs' TMA loads count their
// bytes there; its producer arms it with both halves); empty[s] and tfull[b]
// live in both CTAs and are signalled by the even CTA's MMA commits;
// tempty[b] lives in the even CTA and collects one arrival per epilogue warp
// of both CTAs.
constexpr int kStages2 = 6;

struct Smem2 {
    static constexpr int kABytes = 128 * kBKBytes;        // this CTA's 128 rows of A
    static constexpr int kBBytes = 128 * kBKBytes;        // this CTA's 128 columns of B
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kBarOffset = kStages2 * kStageBytes;
    // full[S], empty[S], tfull[2], tempty[2], drain
    static constexpr int kNumBars = 2 * kStages2 + 5;
    static constexpr int kParamOffset = (kBarOffset + kNumBars * 8 + 16 + 127) / 128 * 128;
    static constexpr int kParamBytes = 8 * kColParamBytes;
    static constexpr int kStoreOffset = kParamOffset + kParamBytes;
    static constexpr int kTotal = kStoreOffset + 8 * kStoreStageBytes + 1024;
};
static_assert(Smem2::kTotal <= 227 * 1024, "pair-kernel shared memory");


template <MmaKind KIND, int EPI, bool A_SIGNED, bool B_SIGNED, bool B_MN = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmArgs args) {
    constexpr int kEsize = KIND == MmaKind::F16 ? 2 : 1;
    constexpr int kKElems = kBKBytes / kEsize;
    constexpr int kNBox = 128 / kEsize;
    constexpr int kBoxBytes = kKElems * 128;
    constexpr int kTileN = 256;
    constexpr uint32_t kTmemCols = 512;               // two 256-column accumulators
    using L = Smem2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + kStages2;
    uint64_t *tfull = bars + 2 * kStages2;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + L::kNumBars);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_ctarank();
    const bool even = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages2; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 16);   // one arrive per epilogue warp of the pair
        }
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::tma_prefetch_desc(&tmA);
        tc::tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tc::tmem_alloc_pair(tmem_slot, kTmemCols);
        tc::tmem_relinquish_pair();
    }
    // barriers of both CTAs initialised and the allocation visible before
    // any load, commit or remote arrive of the pair
    tc::tc_fence_before();
    tc::cluster_sync_all();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs)
            const uint32_t full_even = tc::mapa_shared(tc::smem_u32(full), 0);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_phase = 0;
            for (int u = pair; u < args.units && !*abort_flag; u += npairs) {
                const Unit w = unit_of(u, args);
                int mb, nb;
                tile_coords(w.t, args, mb, nb);
                const int row0 = mb * 256 + (int)rank * 128;
                const int col0 = nb * kTileN + (int)rank * 128;
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!tc::mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err_word,
                                       kErrWaitEmpty))
                        break;
                    uint8_t *sa = smem + stage * L::kStageBytes;
                    uint8_t *sb = sa + L::kABytes;
                    if (even) tc::mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
                    const uint32_t fb = full_even + (uint32_t)stage * 8u;
                    const int kx = kb * kKElems;
                    tc::tma_load_2d_pair(sa, &tmA, fb, kx, row0);
                    if constexpr (B_MN) {
#pragma unroll
                        for (int c = 0; c < 128 / kNBox; c++)
                            tc::tma_load_2d_pair(sb + c * kBoxBytes, &tmB, fb, col0 + c * kNBox, kx);
                    } else {
                        tc::tma_load_2d_pair(sb, &tmB, fb, kx, col0);
                    }
                    armed |= 1u << stage;
                    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages2) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain (even CTA): the full barriers count both CTAs' bytes, so
            // once the armed phases complete no load of the pair is in flight.
            if (even)
                for (int s = 0; s < kStages2; s++)
                    if (armed & (1u << s)) {
                        const uint64_t t0 = tc::globaltimer();
                        while (!tc::mbar_try_wait(&full[s], (armed_phase >> s) & 1u) &&
                               tc::globaltimer() - t0 < kWaitBudgetNs) {
                        }
                    }
        }
    } else if (warp == 1) {
        if (lane == 0 && even) {
            // ---------------- MMA issuer (even CTA only)
            constexpr uint32_t idesc = (KIND == MmaKind::F16)
                                           ? tc::idesc_f16_f32(256, kTileN, B_MN)
                                           : tc::idesc_i8_s32(256, kTileN, A_SIGNED, B_SIGNED, B_MN);
            const uint32_t empty_own = tc::smem_u32(empty);
            const uint32_t empty_odd = tc::mapa_shared(empty_own, 1);
            const uint32_t tfull_own = tc::smem_u32(tfull);
            const uint32_t tfull_odd = tc::mapa_shared(tfull_own, 1);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool issued = false;
            for (int u = pair; u < args.units && !*abort_flag; u += npairs, local++) {
                const Unit w = unit_of(u, args);
                const int buf = local & 1;
                const uint32_t aphase = (local >> 1) & 1;
                if (!tc::mbar_wait_cluster(&tempty[buf], aphase ^ 1, abort_flag, args.err_word,
                                           kErrWaitAccum))
                    break;
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kTileN);
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!tc::mbar_wait(&full[stage], phase, abort_flag, args.err_word,
                                       kErrWaitFull))
                        break;
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(smem + stage * L::kStageBytes);
                    const uint32_t sb = sa + L::kABytes;
#pragma unroll
                    for (int k = 0; k < kBKBytes / 32; k++) {
                        const uint64_t ad = tc::sdesc_kmajor_sw128(sa + k * 32);
                        const uint64_t bd =
                            B_MN ? tc::sdesc_mnmajor_sw128(sb + k * (32 / kEsize) * 128, kBoxBytes, 1024)
                                 : tc::sdesc_kmajor_sw128(sb + k * 32);
                        tc::mma_ss_pair<KIND>(d_tmem, ad, bd, idesc,
                                              (kb != w.kb0 || k != 0) ? 1u : 0u);
                    }
                    issued = true;
                    tc::mma_commit_pair(empty_own + (uint32_t)stage * 8u);
                    tc::mma_commit_pair(empty_odd + (uint32_t)stage * 8u);
                    if (++stage == kStages2) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                tc::mma_commit_pair(tfull_own + (uint32_t)buf * 8u);
                tc::mma_commit_pair(tfull_odd + (uint32_t)buf * 8u);
            }
            if (issued) {
                tc::mma_commit_pair(tc::smem_u32(drain));
                const uint64_t t0 = tc::globaltimer();
                while (!tc::mbar_try_wait(drain, 0) && tc::globaltimer() - t0 < kWaitBudgetNs) {
                }
            }
        }
    } else {
        // The column sums come from the kernel launched just before this one,
        // which may still be running (programmatic dependent launch): wait
        // for it before the first epilogue (a no-op without a prerequisite).
        if (args.epi.colsum) tc::grid_dependency_wait();
        // ---------------- epilogue warps 2..9 of both CTAs: this CTA's 128
        // rows of the tile, all 256 columns (warp halves as gemm_tc_kernel)
        const int q = warp & 3;
        const int chalf = (warp - 2) >> 2;
        ColParams *cp = reinterpret_cast<ColParams *>(smem + L::kParamOffset) + (warp - 2);
        uint4 *stage = reinterpret_cast<uint4 *>(smem + L::kStoreOffset + (warp - 2) * kStoreStageBytes);
        const uint32_t tempty_even = tc::mapa_shared(tc::smem_u32(tempty), 0);
        const int wslot = warp - 2;
        constexpr size_t kPartWords = (size_t)(kTileN / 2) * 32;
        int local = 0;
        for (int u = pair; u < args.units && !__any_sync(0xffffffffu, *abort_flag);
             u += npairs, local++) {
            const Unit w = unit_of(u, args);
            int mb, nb;
            tile_coords(w.t, args, mb, nb);
            const int buf = local & 1;
            const uint32_t aphase = (local >> 1) & 1;
            bool ok = tc::mbar_wait(&tfull[buf], aphase, abort_flag, args.err_word, kErrWaitAccum);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc::tc_fence_after();
            const int row = mb * 256 + (int)rank * 128 + q * 32 + lane;
            const uint32_t taddr =
                tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kTileN);
            if (w.part >= 1) {
                // a K part of a split tile: this CTA's raw accumulator rows to
                // the workspace
                const size_t ps = part_slot(args, w.t, w.part, (int)rank, 2, wslot);
                int32_t *ws = args.part_ws + ps * kPartWords;
#pragma unroll 1
                for (int c = 0; c < kTileN / 2; c += 32) {
                    uint32_t r[32];
                    tc::tmem_ld_32x32b_x32(taddr + (uint32_t)(chalf * (kTileN / 2) + c), r);
                    tc::tmem_ld_wait(r);
                    part_store(ws, c / 32, lane, r);
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) part_flag_set(args.part_flag + ps, args.ticket);
            } else {
                if (w.part == 0) {
                    for (int p = 1; p < args.split && ok; p++)
                        ok = part_flag_wait(
                            args.part_flag + part_slot(args, w.t, p, (int)rank, 2, wslot),
                            args.ticket, abort_flag, args.err_word);
                    if (!__all_sync(0xffffffffu, ok)) break;
                    merge_parts<KIND == MmaKind::F16, kTileN / 2>(
                        args.part_ws + part_slot(args, w.t, 1, (int)rank, 2, wslot) * kPartWords,
                        16 * kPartWords, args.split - 1, taddr + (uint32_t)(chalf * (kTileN / 2)),
                        lane);
                }
#pragma unroll 1
                for (int c = chalf * (kTileN / 2); c < (chalf + 1) * (kTileN / 2); c += 32) {
                    uint32_t r[32];
                    if constexpr (EPI == kEpiRequant || EPI == kEpiHmx) {
                        stage_params(args.epi, cp, nb * kTileN + c, lane);
                    }
                    __syncwarp();
                    tc::tmem_ld_32x32b_x32(taddr + (uint32_t)c, r);
                    tc::tmem_ld_wait(r);
                    epilogue_chunk<EPI>(args.epi, r, row, nb * kTileN + c, cp, stage);
                    __syncwarp();
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_remote(tempty_even + (uint32_t)buf * 8u);
        }
    }

    // Both CTAs stay resident until the pair's last MMA, commit and remote
    // arrive are done; then each frees its half of the allocation.
    __syncwarp();
    tc::tc_fence_before();
    tc::cluster_sync_all();
    tc::tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tc::tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------- pre-pass kernels

// Bt[n][k] = B[k][n] for k < K, 0 for K <= k < Kp (Kp a multiple of 64);
// optionally colsum[n] += sum_k B[k][n] (int8 only; colsum pre-zeroed).
template <typename T, bool COLSUM>
__global__ void __launch_bounds__(256) transpose_pack_kernel(const T *__restrict__ B,
                                                              T *__restrict__ Bt,
                                                              int32_t *__restrict__ colsum, int K,
                                                              int N, int64_t ldb, int64_t Kp) {
    __shared__ T tile[64][64 + 4];
    const int k0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    // load: thread (kr, nc) reads 16 consecutive n of row k
    {
        const int kr = threadIdx.x >> 2, nc = (threadIdx.x & 3) * 16;
        const int k = k0 + kr;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int n = n0 + nc + i;
            tile[kr][nc + i] = (k < K && n < N) ? B[(size_t)k * ldb + n] : T(0);
        }
    }
    __syncthreads();
    if (COLSUM && threadIdx.x < 64) {
        const int n = n0 + threadIdx.x;
        int32_t s = 0;
        for (int kr = 0; kr < 64; kr++) s += (int32_t)(int8_t)tile[kr][threadIdx.x];
        if (n < N) atomicAdd(colsum + n, s);
    }
    // store: thread (nr, kc) writes 16 consecutive k of column n
    {
        const int nr = threadIdx.x >> 2, kc = (threadIdx.x & 3) * 16;
        const int n = n0 + nr;
        if (n < N && k0 + kc < Kp) {
            T v[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = tile[kc + i][nr];
            uint4 *dst = reinterpret_cast<uint4 *>(Bt + (size_t)n * Kp + k0 + kc);
            const uint4 *src = reinterpret_cast<const uint4 *>(v);
#pragma unroll
            for (int i = 0; i < (int)(16 * sizeof(T) / 16); i++) dst[i] = src[i];
        }
    }
}

// dst[r][k] = src[r][k] for k < K, 0 for K <= k < ldd (never reads src when
// K == 0).
template <typename T>
__global__ void __launch_bounds__(256) pad_rows_kernel(const T *__restrict__ src, int64_t lds,
                                                        T *__restrict__ dst, int64_t ldd, int rows,
                                                        int K) {
    const int64_t total = (int64_t)rows * ldd;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ldd, k = i % ldd;
        dst[i] = k < K ? src[r * lds + k] : T(0);
    }
}

// colsum[n] += sum_{k in this block's rows} B[k][n] for a row-major int8 B
// [K, N] (N a multiple of 16, rows 16-byte aligned; colsum pre-zeroed).
// A block of 8 warps covers 512 columns (16 per lane) and kColsumRows rows
// at most; warp w reads rows w, w + 8, ..., four rows per loop trip so that
// 64 bytes per thread are in flight (the pass is bound by HBM latency
// otherwise).  Bytes are summed as unsigned (b + 128) in packed 16-bit lanes
// (even and odd bytes of each word; at most kColsumRows / 8 = 256 rows per
// thread, so a lane stays below 65536) and unbiased at the end; the 8 warps'
// sums meet in shared memory and each column takes one atomic per block.
constexpr int kColsumRows = 2048;

__global__ void __launch_bounds__(256) colsum_kernel(const int8_t *__restrict__ B,
                                                     int32_t *__restrict__ colsum, int K, int N,
                                                     int kchunk) {
    tc::launch_dependents();
    __shared__ int32_t red[8][512];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = blockIdx.x * 512;
    const int n0 = nblk + lane * 16;
    const int k0 = blockIdx.y * kchunk, k1 = min(K, k0 + kchunk);
    uint32_t ev[4] = {0, 0, 0, 0}, od[4] = {0, 0, 0, 0};
    int rows = 0;
    if (n0 < N) {
        const int8_t *col = B + n0;
        auto add = [&](const int4 v) {
            const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t x = w[j] ^ 0x80808080u;
                ev[j] += x & 0x00FF00FFu;
                od[j] += (x >> 8) & 0x00FF00FFu;
            }
        };
        int k = k0 + warp;
        for (; k + 24 < k1; k += 32) {
            int4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                v[u] = __ldg(reinterpret_cast<const int4 *>(col + (size_t)(k + 8 * u) * N));
#pragma unroll
            for (int u = 0; u < 4; u++) add(v[u]);
            rows += 4;
        }
        for (; k < k1; k += 8) {
            add(__ldg(reinterpret_cast<const int4 *>(col + (size_t)k * N)));
            rows++;
        }
    }
    // column 4j + 0 / 4j + 2 in the low / high half of ev[j]; 4j + 1 / 4j + 3 of od[j]
    const int bias = 128 * rows;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        red[warp][lane * 16 + 4 * j + 0] = (int32_t)(ev[j] & 0xFFFFu) - bias;
        red[warp][lane * 16 + 4 * j + 1] = (int32_t)(od[j] & 0xFFFFu) - bias;
        red[warp][lane * 16 + 4 * j + 2] = (int32_t)(ev[j] >> 16) - bias;
        red[warp][lane * 16 + 4 * j + 3] = (int32_t)(od[j] >> 16) - bias;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int c = threadIdx.x * 2 + h;
        int32_t sum = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) sum += red[w][c];
        if (nblk + c < N) atomicAdd(colsum + nblk + c, sum);
    }
}

// colsum[n] = sum_k Bt[n][k] for a K-major int8 Bt [N, K] (pitch ldb): one
// warp per row, 16-byte loads where the row allows them (four in flight per
// lane), each word's four signed bytes summed by one dp4a against ones.
__global__ void __launch_bounds__(256) rowsum_i8_kernel(const int8_t *__restrict__ Bt,
                                                        int64_t ldb, int32_t *__restrict__ colsum,
                                                        int N, int K, int vec) {
    tc::launch_dependents();
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const int8_t *row = Bt + (size_t)n * ldb;
    int32_t s = 0;
    int k0 = 0;
    if (vec) {
        constexpr int kOnes = 0x01010101;
        const int kv = K & ~15;
        auto add = [&](const int4 q) {
            s = __dp4a(q.x, kOnes, s);
            s = __dp4a(q.y, kOnes, s);
            s = __dp4a(q.z, kOnes, s);
            s = __dp4a(q.w, kOnes, s);
        };
        int k = lane * 16;
        for (; k + 3 * 512 < kv; k += 4 * 512) {
            int4 q[4];
#pragma unroll
            for (int u = 0; u < 4; u++) q[u] = __ldg(reinterpret_cast<const int4 *>(row + k + u * 512));
#pragma unroll
            for (int u = 0; u < 4; u++) add(q[u]);
        }
        for (; k < kv; k += 512) add(__ldg(reinterpret_cast<const int4 *>(row + k)));
        k0 = kv;
    }
    for (int k = k0 + lane; k < K; k += 32) s += row[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) colsum[n] = s;
}

// ------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2D K-major operand map: rows x K elements, row pitch `pitch_bytes`, box
// 128 bytes of K x box_rows rows, 128-byte swizzle, zero fill out of bounds.
int make_kmajor_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int esize,
                    int64_t K, int64_t rows, int64_t pitch_bytes, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(HEXCUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(kBKBytes / esize), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(HEXCUDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): K=%lld rows=%lld pitch=%lld",
                    (int)r, (long long)K, (long long)rows, (long long)pitch_bytes);
    return HEXCUDA_OK;
}

// Row-major B [K, N] read as an MN-major operand: boxes of 128 bytes of N x
// k_rows rows of K, 128-byte swizzle, zero fill out of bounds.
int make_mnmajor_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int esize,
                     int64_t N, int64_t K, int k_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(HEXCUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)(N * esize)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / esize), (cuuint32_t)k_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(HEXCUDA_ERR_CUDA, "cuTensorMapEncodeTiled (MN-major B) failed (%d): N=%lld K=%lld",
                    (int)r, (long long)N, (long long)K);
    return HEXCUDA_OK;
}

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// The rasterisation group from L2 capacity: hold a panel of one operand
// (group blocks x K) resident in L2 while the other streams past it once per
// group.  DRAM reads are then about   resident + streamed x groups;  the
// orientation and group size minimising that, with the panel within
// kL2PanelBytes (a share of the 126 MB L2 that leaves room for the streamed
// operand and the output), are chosen.  Measured DRAM reads of the
// 16384 x 8192 x 8192 u8 x s8 GEMM per panel budget: 24 MB 474 MB, 32 MB
// 406, 40 MB 401 (modelled 384), 48 MB 488-509 (modelled 320: the panel is
// no longer kept), 64 MB 1506; the time is flat from 24 to 48 MB.
// HEXCUDA_GEMM_L2_PANEL_MB overrides the panel budget (a tuning knob).
constexpr int64_t kL2PanelBytes = 40ll << 20;

void pick_raster(GemmArgs &a, int64_t bm, int64_t bn, int64_t kbytes) {
    static int64_t budget = -1;
    if (budget < 0) {
        const char *e = getenv("HEXCUDA_GEMM_L2_PANEL_MB");
        budget = e ? (int64_t)atoi(e) << 20 : kL2PanelBytes;
    }
    const int64_t a_blk = bm * kbytes, b_blk = bn * kbytes;
    auto cost = [&](int64_t along, int64_t blk, int64_t across_bytes, int64_t own_bytes,
                    int &g) {
        g = (int)std::max<int64_t>(1, std::min<int64_t>(along, budget / std::max<int64_t>(blk, 1)));
        const int64_t groups = (along + g - 1) / g;
        // spread the blocks evenly over the groups
        g = (int)((along + groups - 1) / groups);
        return own_bytes + across_bytes * groups;
    };
    int gm = 1, gn = 1;
    const int64_t a_bytes = a_blk * a.tiles_m, b_bytes = b_blk * a.tiles_n;
    const int64_t cm = cost(a.tiles_m, a_blk, b_bytes, a_bytes, gm);
    const int64_t cn = cost(a.tiles_n, b_blk, a_bytes, b_bytes, gn);
    a.group_n_major = cn < cm ? 1 : 0;
    a.group = cn < cm ? gn : gm;
}

// Tail split (see unit_of): when the last wave of a persistent launch over
// `slots` CTAs (or CTA pairs) would leave at least half of them idle, its
// tiles are cut into K parts, up to kMaxSplit and at least kMinSplitKb K
// blocks each, so that the wave keeps the idle slots busy and takes about
// 1 / split of a tile's time.  The partial accumulators (part_bytes per
// part) and arrival flags (flags_per_part per part) live in scratch slot
// kSlotSplit: a fixed kSplitFlagBytes of flags, zeroed once per buffer and
// afterwards written only with launch tickets, then the workspace.  Sets the
// unit fields of `a` and the grid in slots.  single_wave_only: split only
// when every tile is in the one, partial wave.  HEXCUDA_GEMM_SPLIT=0 turns
// the split off (a tuning knob).  Measured on the 2048 x 8192 x 8192 u8 x s8
// GEMM (the row shard of an 8-GPU run; 50 launches, two runs): 0.1271 ->
// 0.1242 ms.
constexpr int kMaxSplit = 4;
constexpr int kMinSplitKb = 8;
constexpr size_t kSplitFlagBytes = 64 << 10;
std::atomic<uint32_t> g_split_ticket{0};

int plan_tail_split(Dev *d, GemmArgs &a, int slots, size_t part_bytes, int flags_per_part,
                    int &grid, bool allowed = true, bool single_wave_only = false) {
    static int enabled = -1;
    if (enabled < 0) {
        const char *e = getenv("HEXCUDA_GEMM_SPLIT");
        enabled = (e && atoi(e) == 0) ? 0 : 1;
    }
    const int tiles = a.tiles_m * a.tiles_n;
    a.dp_tiles = tiles;
    a.split = 1;
    a.units = tiles;
    a.ticket = 0;
    a.part_flag = nullptr;
    a.part_ws = nullptr;
    grid = std::min(tiles, slots);
    const int rem = tiles % slots;        // tiles of the last wave
    if (!enabled || !allowed || rem == 0 || (single_wave_only && tiles > slots)) return HEXCUDA_OK;
    const int split = std::min(std::min(slots / rem, a.num_kb / kMinSplitKb), kMaxSplit);
    const size_t nparts = (size_t)rem * (size_t)(split - 1);
    if (split < 2 || nparts * flags_per_part * sizeof(int) > kSplitFlagBytes) return HEXCUDA_OK;
    uint8_t *buf =
        reinterpret_cast<uint8_t *>(scratch(d, kSlotSplit, kSplitFlagBytes + nparts * part_bytes));
    if (!buf) return hexcuda_last_error();
    if (d->split_zeroed != buf || d->split_zeroed_bytes < kSplitFlagBytes) {
        if (int rc = check(cudaMemsetAsync(buf, 0, kSplitFlagBytes, d->stream), "memset split flags"))
            return rc;
        d->split_zeroed = buf;
        d->split_zeroed_bytes = kSplitFlagBytes;
    }
    uint32_t ticket = ++g_split_ticket;
    if (ticket == 0) ticket = ++g_split_ticket;
    a.dp_tiles = tiles - rem;
    a.split = split;
    a.units = a.dp_tiles + rem * split;
    a.ticket = ticket;
    a.part_flag = reinterpret_cast<int *>(buf);
    a.part_ws = reinterpret_cast<int32_t *>(buf + kSplitFlagBytes);
    grid = a.dp_tiles > 0 ? slots : rem * split;
    return HEXCUDA_OK;
}

template <MmaKind KIND, int BN, int EPI, bool AS, bool BS, bool BMN = false>
int launch_gemm_kernel(Dev *d, const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K,
                       const EpiParams &ep, bool pdl = false, bool allow_split = true) {
    using L = Smem<BN>;
    auto kern = gemm_tc_kernel<KIND, BN, EPI, AS, BS, BMN>;
    static bool attr_done[64] = {};
    const int dev_slot = d->ordinal & 63;
    if (!attr_done[dev_slot]) {
        if (int rc = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                L::kTotal),
                           "cudaFuncSetAttribute(gemm smem)"))
            return rc;
        attr_done[dev_slot] = true;
    }
    GemmArgs args;
    args.tiles_m = (M + kBM - 1) / kBM;
    args.tiles_n = (N + BN - 1) / BN;
    const int kelems = KIND == MmaKind::F16 ? kBKBytes / 2 : kBKBytes;
    args.num_kb = (K + kelems - 1) / kelems;
    args.err_word = d->err_word;
    args.epi = ep;
    pick_raster(args, kBM, BN, (int64_t)args.num_kb * kBKBytes);
    int grid = 0;
    // integer GEMMs only: int32 parts add exactly, so the result does not
    // depend on the split (an fp16 GEMM's would, by its fp32 rounding, and
    // with it on how the caller's rows were cut into launches)
    if (int rc = plan_tail_split(d, args, d->sms, (size_t)kBM * BN * 4, 8, grid,
                                 allow_split && KIND == MmaKind::I8))
        return rc;
    if (pdl) {
        // a programmatic dependent of the column-sum pass launched just before
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = L::kTotal;
        cfg.stream = d->stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (int rc = check(cudaLaunchKernelEx(&cfg, kern, ta, tb, args), "launch gemm kernel"))
            return rc;
    } else {
        kern<<<grid, kThreads, L::kTotal, d->stream>>>(ta, tb, args);
    }
    note_mech(kMechTcgen05 | kMechTma);
    return HEXCUDA_OK;
}

// The CTA-pair kernel, persistent over as many pairs as the device keeps
// resident at once.  Returns HEXCUDA_OK with *launched = false (nothing
// launched) when the device reports no resident pair, so the caller takes
// the one-SM kernel.
template <MmaKind KIND, int EPI, bool AS, bool BS, bool BMN = false>
int launch_gemm2_kernel(Dev *d, const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K,
                        const EpiParams &ep, bool *launched, bool pdl = false) {
    using L = Smem2;
    auto kern = gemm_tc2_kernel<KIND, EPI, AS, BS, BMN>;
    static int pairs_resident[64] = {};     // 0: not queried yet, -1: none
    const int dev_slot = d->ordinal & 63;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // optionally a programmatic dependent of the column-sum pass before it
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = d->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    *launched = false;
    if (pairs_resident[dev_slot] == 0) {
        if (int rc = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                L::kTotal),
                           "cudaFuncSetAttribute(gemm pair smem)"))
            return rc;
        cfg.gridDim = dim3(2, 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = -1;
        }
        pairs_resident[dev_slot] = n;
    }
    if (pairs_resident[dev_slot] < 0) return HEXCUDA_OK;
    GemmArgs args;
    args.tiles_m = (M + 255) / 256;
    args.tiles_n = (N + 255) / 256;
    const int kelems = KIND == MmaKind::F16 ? kBKBytes / 2 : kBKBytes;
    args.num_kb = (K + kelems - 1) / kelems;
    args.err_word = d->err_word;
    args.epi = ep;
    pick_raster(args, 256, 256, (int64_t)args.num_kb * kBKBytes);
    int pairs = 0;
    // integer GEMMs only (as the one-SM kernel), and only when all tiles fit
    // in one wave: behind full waves the split tail measured slower here
    // (HMX int32 out, 2048 x 8192 x 8192: 0.139 -> 0.149 ms), the previous
    // tile's heavy epilogue delaying the parts' hand-over
    if (int rc = plan_tail_split(d, args, pairs_resident[dev_slot], (size_t)256 * 256 * 4, 16,
                                 pairs, KIND == MmaKind::I8, true))
        return rc;
    cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
    cfg.numAttrs = pdl ? 2 : 1;
    if (int rc = check(cudaLaunchKernelEx(&cfg, kern, ta, tb, args), "launch gemm pair kernel"))
        return rc;
    note_mech(kMechTcgen05 | kMechTma);
    *launched = true;
    return HEXCUDA_OK;
}

// The CTA-pair kernel serves the 256-column launches with at least two row
// tiles of the fp16 and HMX-convention epilogues (measured 0-5 % faster than
// the one-SM kernel there); the per-channel requant epilogue measured ~3 %
// faster on the one-SM kernel (u8 x s8 16384 x 8192 x 8192), so it stays
// there.  HEXCUDA_GEMM_PAIR=0 / =1 in the environment forces either kernel.
template <int EPI>
bool gemm_pair_enabled(int M, int N) {
    if (M <= kBM || N <= 128) return false;
    const char *e = getenv("HEXCUDA_GEMM_PAIR");
    if (e && e[0] == '0') return false;
    if (e && e[0] == '1') return true;
    return EPI != kEpiRequant;
}

// 128-column tiles for N <= 128, 256-column ones otherwise.  (On a
// 2048 x 8192 x 8192 row shard, where 256-column tiles leave the last of four
// waves half empty, 128-column tiles measured 23 % slower all the same: they
// reuse each A stage half as often.)  HEXCUDA_GEMM_BN=128 / 256 forces either
// (a tuning knob).
bool narrow_tiles(int N) {
    static int force = -1;
    if (force < 0) {
        const char *e = getenv("HEXCUDA_GEMM_BN");
        force = e ? atoi(e) : 0;
    }
    if (force == 128 || force == 256) return force == 128;
    return N <= 128;
}

// Common driver: A [M,K] K-major (pitch lda elements), B given either as
// Bt [N,K] K-major (b_kmajor) or as row-major B [K,N] (transposed here).
// Operands whose rows are not 16-byte aligned, or shorter than one 128-byte
// K block, are copied into zero-padded [rows, Kp] buffers (Kp * esize a
// multiple of 128 bytes); TMA zero-fills every other out-of-range element.
template <MmaKind KIND, int EPI, bool AS, bool BS>
int run_gemm(int dev, const void *A, int64_t lda, const void *B, bool b_kmajor, int M, int N,
             int K, EpiParams ep, bool want_colsum, const char *name) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "%s: bad shape %dx%dx%d", name, M, N, K);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if ((K > 0 && (!A || !B)) || !ep.out) return fail(HEXCUDA_ERR_ARG, "%s: null pointer", name);
    if (EPI == kEpiRequant &&
        (ep.zp <= -(1 << 19) || ep.zp >= (1 << 19) || ep.lo <= -(1 << 19) || ep.hi >= (1 << 19)))
        return fail(HEXCUDA_ERR_ARG, "%s: zero point / clamp out of range", name);
    constexpr int esize = KIND == MmaKind::F16 ? 2 : 1;
    constexpr int kelems = kBKBytes / esize;
    constexpr CUtensorMapDataType dt =
        KIND == MmaKind::F16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    using T = typename std::conditional<KIND == MmaKind::F16, uint16_t, uint8_t>::type;
    const int64_t Kp = round_up(K > 0 ? K : 1, kelems);
    const bool short_k = K < kelems;

    launch_begin(d);
    int nl = 0;
    // The GEMM may start as a programmatic dependent (its mainloop overlapping
    // the previous kernel) only when that kernel is the column-sum pass, whose
    // output it reads in the epilogue, after griddepcontrol.wait.
    bool pdl = false;
    // ---- B operand
    const T *bt = reinterpret_cast<const T *>(B);
    int64_t bt_pitch = (int64_t)K * esize, b_kdim = K;
    int32_t *colsum = nullptr;
    if (want_colsum) {
        colsum = reinterpret_cast<int32_t *>(scratch(d, 1, sizeof(int32_t) * (size_t)N));
        if (!colsum) return HEXCUDA_ERR_OOM;
        if (int rc = check(cudaMemsetAsync(colsum, 0, sizeof(int32_t) * (size_t)N, d->stream),
                           "memset colsum"))
            return rc;
    }
    if (want_colsum && b_kmajor) {
        // column sums of B = row sums of the K-major Bt, from the caller's copy
        const bool vec = aligned16(B) && (K % 16) == 0;
        rowsum_i8_kernel<<<(unsigned)((N + 7) / 8), 256, 0, d->stream>>>(
            reinterpret_cast<const int8_t *>(B), K, colsum, N, K, vec ? 1 : 0);
        nl++;
        pdl = true;
    }
    // row-major B that TMA can read in place: MN-major operand, no copy
    const bool b_mn = !b_kmajor && ((int64_t)N * esize) % 16 == 0 && aligned16(B) &&
                      (int64_t)N * esize >= 128 && K >= kelems;
    if (b_mn) {
        if (want_colsum) {
            // about four 256-thread blocks per SM, each at most kColsumRows rows
            const int nblk = (N + 511) / 512;
            const int splits = std::max(1, (4 * d->sms + nblk - 1) / nblk);
            int kchunk = (K + splits - 1) / splits;
            kchunk = std::min(kColsumRows, std::max(32, (kchunk + 31) / 32 * 32));
            dim3 g((unsigned)nblk, (unsigned)((K + kchunk - 1) / kchunk));
            colsum_kernel<<<g, 256, 0, d->stream>>>(reinterpret_cast<const int8_t *>(B), colsum, K,
                                                     N, kchunk);
            nl++;
            pdl = true;
        }
    } else if (!b_kmajor) {
        T *tmp = reinterpret_cast<T *>(scratch(d, 0, (size_t)N * Kp * esize));
        if (!tmp) return HEXCUDA_ERR_OOM;
        dim3 g((unsigned)((N + 63) / 64), (unsigned)(Kp / 64));
        if (want_colsum)
            transpose_pack_kernel<T, true><<<g, 256, 0, d->stream>>>(
                reinterpret_cast<const T *>(B), tmp, colsum, K, N, N, Kp);
        else
            transpose_pack_kernel<T, false><<<g, 256, 0, d->stream>>>(
                reinterpret_cast<const T *>(B), tmp, nullptr, K, N, N, Kp);
        nl++;
        pdl = false;
        bt = tmp;
        bt_pitch = Kp * esize;
        b_kdim = Kp;
    } else if ((bt_pitch % 16) != 0 || !aligned16(B) || short_k) {
        T *tmp = reinterpret_cast<T *>(scratch(d, 0, (size_t)N * Kp * esize));
        if (!tmp) return HEXCUDA_ERR_OOM;
        pad_rows_kernel<T><<<(unsigned)std::min<int64_t>((N * Kp + 255) / 256, 4096), 256, 0,
                             d->stream>>>(reinterpret_cast<const T *>(B), K, tmp, Kp, N, K);
        nl++;
        pdl = false;
        bt = tmp;
        bt_pitch = Kp * esize;
        b_kdim = Kp;
    }
    // ---- A operand
    const T *a = reinterpret_cast<const T *>(A);
    int64_t a_pitch = lda * esize, a_kdim = K;
    if ((a_pitch % 16) != 0 || !aligned16(A) || short_k) {
        T *tmp = reinterpret_cast<T *>(scratch(d, 2, (size_t)M * Kp * esize));
        if (!tmp) return HEXCUDA_ERR_OOM;
        pad_rows_kernel<T><<<(unsigned)std::min<int64_t>((M * Kp + 255) / 256, 4096), 256, 0,
                             d->stream>>>(reinterpret_cast<const T *>(A), lda, tmp, Kp, M, K);
        nl++;
        pdl = false;
        a = tmp;
        a_pitch = Kp * esize;
        a_kdim = Kp;
    }
    // Overlapping the column-sum pass pays on short GEMMs (a 2048 x 8192 x
    // 8192 row shard: 0.152 -> 0.144 ms) and costs on long ones, whose early
    // CTAs then compete with the pass for DRAM and hold their first
    // accumulators until it ends (16384 x 8192 x 8192: 0.784 -> 0.800 ms):
    // only GEMMs of at most 8 waves of 128 x 256 tiles take it.
    if (pdl && (int64_t)((M + kBM - 1) / kBM) * ((N + 255) / 256) > 8ll * d->sms) pdl = false;
    CUtensorMap ta, tb;
    if (int rc = make_kmajor_map(&ta, a, dt, esize, a_kdim, M, a_pitch, kBM)) return rc;
    ep.colsum = colsum;
    ep.M = M;
    ep.N = N;
    const int kdim = (int)std::max(a_kdim, b_kdim);
    int rc;
    if (gemm_pair_enabled<EPI>(M, N)) {
        bool launched = false;
        if (b_mn) {
            if ((rc = make_mnmajor_map(&tb, B, dt, esize, N, K, kelems))) return rc;
            rc = launch_gemm2_kernel<KIND, EPI, AS, BS, true>(d, ta, tb, M, N, kdim, ep, &launched,
                                                              pdl);
        } else {
            if ((rc = make_kmajor_map(&tb, bt, dt, esize, b_kdim, N, bt_pitch, 128))) return rc;
            rc = launch_gemm2_kernel<KIND, EPI, AS, BS>(d, ta, tb, M, N, kdim, ep, &launched, pdl);
        }
        if (rc) return rc;
        if (launched) return launch_end(d, name, nl + 1);
    }
    const bool narrow = narrow_tiles(N);
    if (b_mn) {
        if ((rc = make_mnmajor_map(&tb, B, dt, esize, N, K, kelems))) return rc;
        if (narrow)
            rc = launch_gemm_kernel<KIND, 128, EPI, AS, BS, true>(d, ta, tb, M, N, kdim, ep, pdl);
        else
            rc = launch_gemm_kernel<KIND, 256, EPI, AS, BS, true>(d, ta, tb, M, N, kdim, ep, pdl);
    } else if (narrow) {
        if ((rc = make_kmajor_map(&tb, bt, dt, esize, b_kdim, N, bt_pitch, 128))) return rc;
        rc = launch_gemm_kernel<KIND, 128, EPI, AS, BS>(d, ta, tb, M, N, kdim, ep, pdl);
    } else {
        if ((rc = make_kmajor_map(&tb, bt, dt, esize, b_kdim, N, bt_pitch, 256))) return rc;
        rc = launch_gemm_kernel<KIND, 256, EPI, AS, BS>(d, ta, tb, M, N, kdim, ep, pdl);
    }
    if (rc) return rc;
    return launch_end(d, name, nl + 1);
}

EpiParams requant_epi(void *out, int N, int32_t mult, int shift, int zp, int lo, int hi) {
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    ep.mult = mult;
    ep.shift = shift;
    ep.zp = zp;
    ep.lo = lo;
    ep.hi = hi;
    return ep;
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_gemm_f16_nt(int dev, const uint16_t *A, const uint16_t *Bt, uint16_t *out,
                                  int M, int N, int K) {
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    return run_gemm<MmaKind::F16, kEpiF16, false, false>(dev, A, K, Bt, true, M, N, K, ep, false,
                                                         "gemm_f16_nt");
}

HX_EXPORT int hexcuda_gemm_f16_nn(int dev, const uint16_t *A, const uint16_t *B, uint16_t *out,
                                  int M, int N, int K) {
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    return run_gemm<MmaKind::F16, kEpiF16, false, false>(dev, A, K, B, false, M, N, K, ep, false,
                                                         "gemm_f16_nn");
}

HX_EXPORT int hexcuda_gemm_i8_requant(int dev, const int8_t *A, const int8_t *B, int8_t *out,
                                      int M, int N, int K, int32_t mult, int shift, int8_t zp) {
    if (shift < 0 || shift > 63) return fail(HEXCUDA_ERR_ARG, "gemm_i8_requant: shift %d", shift);
    EpiParams ep = requant_epi(out, N, mult, shift, zp, -128, 127);
    return run_gemm<MmaKind::I8, kEpiRequant, true, true>(dev, A, K, B, false, M, N, K, ep, false,
                                                          "gemm_i8_requant");
}

HX_EXPORT int hexcuda_gemm_i8_bias_requant(int dev, const int8_t *A, const int8_t *B,
                                           const int32_t *bias, int8_t *out, int M, int N, int K,
                                           int32_t mult, int shift, int8_t zp) {
    if (shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_bias_requant: shift %d", shift);
    if (!bias && N > 0) return fail(HEXCUDA_ERR_ARG, "gemm_i8_bias_requant: null bias");
    EpiParams ep = requant_epi(out, N, mult, shift, zp, -128, 127);
    ep.bias = bias;
    return run_gemm<MmaKind::I8, kEpiRequant, true, true>(dev, A, K, B, false, M, N, K, ep, false,
                                                          "gemm_i8_bias_requant");
}

HX_EXPORT int hexcuda_gemm_i8_zp(int dev, const int8_t *A, const int8_t *B, int8_t *out, int M,
                                 int N, int K, int32_t zpA, int32_t scale_mult, int scale_shift) {
    if (scale_shift < 0 || scale_shift > 63)
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_zp: shift %d", scale_shift);
    EpiParams ep = requant_epi(out, N, scale_mult, scale_shift, 0, -128, 127);
    ep.zpA = zpA;
    return run_gemm<MmaKind::I8, kEpiRequant, true, true>(dev, A, K, B, false, M, N, K, ep,
                                                          zpA != 0, "gemm_i8_zp");
}

HX_EXPORT int hexcuda_gemm_u8s8_pc(int dev, const uint8_t *A, const int8_t *B, const int32_t *bias,
                                   uint8_t *out, int M, int N, int K, int32_t zpA,
                                   const int32_t *mult, const int *shift, uint8_t zp_out) {
    if ((!bias || !mult || !shift) && N > 0)
        return fail(HEXCUDA_ERR_ARG, "gemm_u8s8_pc: null bias/mult/shift");
    EpiParams ep = requant_epi(out, N, 0, 0, zp_out, 0, 255);
    ep.zpA = zpA;
    ep.bias = bias;
    ep.mult_pc = mult;
    ep.shift_pc = shift;
    return run_gemm<MmaKind::I8, kEpiRequant, false, true>(dev, A, K, B, false, M, N, K, ep,
                                                           zpA != 0, "gemm_u8s8_pc");
}

// HMX-convention u8 x s8 GEMM (the corpus's hmx_matmul_i8_* family and
// i8_gemm_bias_relu_requant_hmx): acc = A.B - zpA * colsum(B) in int32, then
// sx12((acc * 17 + 8) >> 4) and, by out_kind, int32 / int8-clamp /
// u8 bias-ReLU-clamp.  B is row-major [K, N] or, with b_transposed, K-major
// Bt [N, K] (hmx_matmul_i8_transposeB).
HX_EXPORT int hexcuda_gemm_f16_ex(int dev, const uint16_t *A, const uint16_t *B, int b_transposed,
                                  const uint16_t *bias, const uint16_t *res, uint16_t *out, int act,
                                  int preround, float scale, int M, int N, int K) {
    if (act < HEXCUDA_F16_ACT_NONE || act > HEXCUDA_F16_ACT_TANH)
        return fail(HEXCUDA_ERR_ARG, "gemm_f16_ex: activation %d", act);
    if (preround < HEXCUDA_F16_PREROUND_NONE || preround > HEXCUDA_F16_PREROUND_ACC)
        return fail(HEXCUDA_ERR_ARG, "gemm_f16_ex: preround %d", preround);
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    ep.f16_bias = reinterpret_cast<const __half *>(bias);
    ep.f16_res = reinterpret_cast<const __half *>(res);
    ep.f16_act = act;
    ep.f16_preround = preround;
    ep.f16_scale = scale;
    return run_gemm<MmaKind::F16, kEpiF16Ex, false, false>(dev, A, K, B, b_transposed != 0, M, N, K,
                                                           ep, false, "gemm_f16_ex");
}

HX_EXPORT int hexcuda_gemm_i8_rq_ex(int dev, const int8_t *A, const int8_t *B, int b_transposed,
                                    const int32_t *bias, const int8_t *res, int8_t *out, int M,
                                    int N, int K, int32_t mult, int shift, int8_t zp, int relu) {
    if (shift < 0 || shift > 63) return fail(HEXCUDA_ERR_ARG, "gemm_i8_rq_ex: shift %d", shift);
    EpiParams ep = requant_epi(out, N, mult, shift, zp, -128, 127);
    ep.bias = bias;
    ep.relu_pre = relu ? 1 : 0;
    ep.rq_res = res;
    return run_gemm<MmaKind::I8, kEpiRequant, true, true>(dev, A, K, B, b_transposed != 0, M, N, K,
                                                          ep, false, "gemm_i8_rq_ex");
}

HX_EXPORT int hexcuda_gemm_i8_acc(int dev, const void *A, int a_signed, const int8_t *B,
                                  int b_transposed, const int32_t *bias, const void *res,
                                  int res_kind, const void *lut, void *out, int store, int act,
                                  int M, int N, int K) {
    if (store < HEXCUDA_HMX_STORE_I32 || store > HEXCUDA_HMX_STORE_ACC_I32)
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_acc: store kind %d", store);
    if (act < HEXCUDA_HMX_ACT_NONE || act > HEXCUDA_HMX_ACT_LEAKY_SHR3)
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_acc: activation %d", act);
    if (res_kind < HEXCUDA_HMX_RES_NONE || res_kind > HEXCUDA_HMX_RES_I8 || (res_kind && !res))
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_acc: residual kind %d", res_kind);
    if ((store == HEXCUDA_HMX_STORE_LUT_I32 || store == HEXCUDA_HMX_STORE_LUT_I8) && !lut)
        return fail(HEXCUDA_ERR_ARG, "gemm_i8_acc: table store without a table");
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    ep.bias = bias;
    ep.res = res;
    ep.res_kind = res_kind;
    ep.lut = lut;
    ep.hmx_store = store;
    ep.hmx_act = act;
    ep.hmx_raw = 1;
    if (a_signed)
        return run_gemm<MmaKind::I8, kEpiHmx, true, true>(dev, A, K, B, b_transposed != 0, M, N, K,
                                                          ep, false, "gemm_i8_acc");
    return run_gemm<MmaKind::I8, kEpiHmx, false, true>(dev, A, K, B, b_transposed != 0, M, N, K, ep,
                                                       false, "gemm_i8_acc");
}

// scratch slot of the FFN's hidden activations (device entries own 0..7)
constexpr int kSlotFfnHidden = 19;

HX_EXPORT int hexcuda_ffn_relu_i8(int dev, const int8_t *A, const int8_t *W1, const int32_t *b1,
                                  const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K,
                                  int V, int D, int32_t mult, int shift, int8_t zp) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "ffn_relu_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    int8_t *hid = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHidden, (size_t)M * (V > 0 ? V : 1)));
    if (!hid) return HEXCUDA_ERR_OOM;
    if (V > 0) {
        if (int rc = hexcuda_gemm_i8_acc(dev, A, 1, W1, 0, b1, nullptr, HEXCUDA_HMX_RES_NONE, nullptr,
                                         hid, HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_RELU, M, V, K))
            return rc;
    }
    return hexcuda_gemm_i8_rq_ex(dev, hid, W2, 0, b2, nullptr, out, M, D, V, mult, shift, zp, 0);
}

HX_EXPORT int hexcuda_ffn_lut_i8(int dev, const int8_t *A, const int8_t *W1, const int32_t *b1,
                                 const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                                 int8_t *out, int M, int K, int V, int D, int32_t mult, int shift,
                                 int8_t zp) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "ffn_lut_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (!act_lut) return fail(HEXCUDA_ERR_ARG, "ffn_lut_i8: null table");
    int8_t *hid = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHidden, (size_t)M * (V > 0 ? V : 1)));
    if (!hid) return HEXCUDA_ERR_OOM;
    if (V > 0) {
        if (int rc = hexcuda_gemm_i8_acc(dev, A, 1, W1, 0, b1, nullptr, HEXCUDA_HMX_RES_NONE, act_lut,
                                         hid, HEXCUDA_HMX_STORE_LUT_I8, HEXCUDA_HMX_ACT_NONE, M, V, K))
            return rc;
    }
    return hexcuda_gemm_i8_rq_ex(dev, hid, W2, 0, b2, nullptr, out, M, D, V, mult, shift, zp, 0);
}

HX_EXPORT int hexcuda_gemm_hmx_s8u8(int dev, const int8_t *A, const uint8_t *B, void *out, int store,
                                    int M, int N, int K) {
    if (store < HEXCUDA_HMX_STORE_I32 || store > HEXCUDA_HMX_STORE_ACC_I32 ||
        store == HEXCUDA_HMX_STORE_LUT_I32 || store == HEXCUDA_HMX_STORE_LUT_I8)
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx_s8u8: store kind %d", store);
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    ep.hmx_store = store;
    return run_gemm<MmaKind::I8, kEpiHmx, true, false>(dev, A, K, B, false, M, N, K, ep, false,
                                                       "gemm_hmx_s8u8");
}

HX_EXPORT int hexcuda_gemm_hmx_ex(int dev, const uint8_t *A, const int8_t *B, int b_transposed,
                                  const int32_t *bias, const void *res, int res_kind,
                                  const void *lut, void *out, int store, int act, int col_major,
                                  int M, int N, int K, int32_t zpA) {
    if (store < HEXCUDA_HMX_STORE_I32 || store > HEXCUDA_HMX_STORE_ACC_I32)
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx: store kind %d", store);
    if (act < HEXCUDA_HMX_ACT_NONE || act > HEXCUDA_HMX_ACT_LEAKY_SHR3)
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx: activation %d", act);
    if (res_kind < HEXCUDA_HMX_RES_NONE || res_kind > HEXCUDA_HMX_RES_I8)
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx: residual kind %d", res_kind);
    if (M > 0 && N > 0 && ((res_kind != HEXCUDA_HMX_RES_NONE && !res) ||
                           ((store == HEXCUDA_HMX_STORE_LUT_I32 || store == HEXCUDA_HMX_STORE_LUT_I8) &&
                            !lut)))
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx: null residual or table");
    EpiParams ep{};
    ep.out = out;
    ep.ldo = col_major ? M : N;
    ep.zpA = zpA;
    ep.bias = bias;
    ep.hmx_store = store;
    ep.hmx_act = act;
    ep.res_kind = res_kind;
    ep.res = res;
    ep.lut = lut;
    ep.col_major = col_major ? 1 : 0;
    return run_gemm<MmaKind::I8, kEpiHmx, false, true>(dev, A, K, B, b_transposed != 0, M, N, K,
                                                       ep, zpA != 0, "gemm_hmx");
}

namespace hx {
namespace {
// u8 A x s8 B [K,N] HMX-field GEMM + bias, shift activation, int8 saturation
int hmx_shift_gemm(int dev, const uint8_t *A, const int8_t *B, const int32_t *bias, int8_t *out,
                   int M, int N, int K, int act, int shift, const char *name) {
    EpiParams ep{};
    ep.out = out;
    ep.ldo = N;
    ep.bias = bias;
    ep.hmx_store = HEXCUDA_HMX_STORE_I8_SAT;
    ep.hmx_act = act;
    ep.post_shift = shift;
    return run_gemm<MmaKind::I8, kEpiHmx, false, true>(dev, A, K, B, false, M, N, K, ep, false, name);
}

// Hu = (u8)(clamp((lut[g + 128] u) >> sh, -zp, zp - 1) + zp), lut read as int8
// (i8_ffn_swiglu_block/kernel_api.h: sw_gate, sw_hu)
__global__ void __launch_bounds__(256) swiglu_gate_kernel(const int8_t *__restrict__ g,
                                                          const int8_t *__restrict__ u,
                                                          const uint8_t *__restrict__ lut,
                                                          uint8_t *__restrict__ hu, int64_t n,
                                                          int sh, int zp) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int s = (int)(int8_t)__ldg(lut + (int)g[i] + 128);
        int h = (s * (int)u[i]) >> sh;
        h = h > zp - 1 ? zp - 1 : (h < -zp ? -zp : h);
        hu[i] = (uint8_t)(h + zp);
    }
}
}  // namespace
}  // namespace hx

// ---------------------------------------------------------------- int16 GEMM
//
// i16_gemm/reference.c:2-11: C = A B with int16 operands and an int32
// accumulator (modulo 2^32).  Each operand is split into a signed high byte
// and a signed low byte, x - 128 = 256 xh + xl' (xh = x >> 8, xl' =
// (x & 255) - 128), so one kind::i8 GEMM of [Ah; Al'] (2M x K) by
// [Bh | Bl'] (K x 2N) gives the four byte products, and
//   sum a b = 65536 hh + 256 (hl + lh) + ll + 128 rowsum(A - 128)
//             + 128 colsum(B - 128) + 16384 K            (all modulo 2^32).
namespace hx {
namespace {
constexpr int kSlotI16A = 19, kSlotI16B = 20, kSlotI16T = 21, kSlotI16Sums = 22;

__global__ void __launch_bounds__(256) i16_split_a_kernel(const int16_t *__restrict__ A,
                                                          int8_t *__restrict__ As,
                                                          int32_t *__restrict__ rs, int M, int K) {
    __shared__ uint32_t part[8];
    const int i = blockIdx.x;
    uint32_t s = 0;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int x = A[(size_t)i * K + k];
        As[(size_t)i * K + k] = (int8_t)(x >> 8);
        As[(size_t)(M + i) * K + k] = (int8_t)((x & 255) - 128);
        s += (uint32_t)(x - 128);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
        rs[i] = (int32_t)t;
    }
}

// one thread per column j and chunk of 64 rows; column sums by atomic adds
// (integer, so the order does not matter)
__global__ void __launch_bounds__(256) i16_split_b_kernel(const int16_t *__restrict__ B,
                                                          int8_t *__restrict__ Bs,
                                                          int32_t *__restrict__ cs, int K, int N) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int k0 = blockIdx.y * 64;
    if (j >= N) return;
    uint32_t s = 0;
    for (int k = k0; k < min(k0 + 64, K); k++) {
        const int x = B[(size_t)k * N + j];
        Bs[(size_t)k * 2 * N + j] = (int8_t)(x >> 8);
        Bs[(size_t)k * 2 * N + N + j] = (int8_t)((x & 255) - 128);
        s += (uint32_t)(x - 128);
    }
    atomicAdd(reinterpret_cast<unsigned *>(cs) + j, s);
}

__global__ void __launch_bounds__(256) i16_combine_kernel(const int32_t *__restrict__ T,
                                                          const int32_t *__restrict__ rs,
                                                          const int32_t *__restrict__ cs,
                                                          int32_t *__restrict__ C, int M, int N,
                                                          uint32_t kterm) {
    const int64_t n = (int64_t)M * N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride) {
        const int i = (int)(t / N), j = (int)(t % N);
        const size_t r0 = (size_t)i * 2 * N, r1 = (size_t)(M + i) * 2 * N;
        const uint32_t hh = (uint32_t)T[r0 + j], hl = (uint32_t)T[r0 + N + j];
        const uint32_t lh = (uint32_t)T[r1 + j], ll = (uint32_t)T[r1 + N + j];
        C[t] = (int32_t)((hh << 16) + ((hl + lh) << 8) + ll + 128u * (uint32_t)rs[i] +
                         128u * (uint32_t)cs[j] + kterm);
    }
}
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_gemm_i16(int dev, const int16_t *A, const int16_t *B, int32_t *C, int M, int N,
                               int K) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || N < 0 || K < 0 || (int64_t)M * 2 > INT32_MAX || (int64_t)N * 2 > INT32_MAX)
        return fail(HEXCUDA_ERR_ARG, "gemm_i16: bad shape %dx%dx%d", M, N, K);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if ((K > 0 && (!A || !B)) || !C) return fail(HEXCUDA_ERR_ARG, "gemm_i16: null pointer");
    const size_t kk = (size_t)(K > 0 ? K : 1);
    int8_t *As = reinterpret_cast<int8_t *>(scratch(d, kSlotI16A, 2 * (size_t)M * kk));
    int8_t *Bs = reinterpret_cast<int8_t *>(scratch(d, kSlotI16B, 2 * (size_t)N * kk));
    int32_t *T = reinterpret_cast<int32_t *>(scratch(d, kSlotI16T, 16 * (size_t)M * N));
    int32_t *sums = reinterpret_cast<int32_t *>(scratch(d, kSlotI16Sums, 4 * ((size_t)M + N)));
    if (!As || !Bs || !T || !sums) return HEXCUDA_ERR_OOM;
    int32_t *rs = sums, *cs = sums + M;
    launch_begin(d);
    if (int rc = check(cudaMemsetAsync(sums, 0, 4 * ((size_t)M + N), d->stream), "memset i16 sums"))
        return rc;
    if (K > 0) {
        i16_split_a_kernel<<<M, 256, 0, d->stream>>>(A, As, rs, M, K);
        i16_split_b_kernel<<<dim3((unsigned)((N + 255) / 256), (unsigned)((K + 63) / 64)), 256, 0,
                             d->stream>>>(B, Bs, cs, K, N);
    }
    if (int rc = launch_end(d, "gemm_i16 (split)")) return rc;
    if (int rc = hexcuda_gemm_i8_acc(dev, As, 1, Bs, 0, nullptr, nullptr, HEXCUDA_HMX_RES_NONE, nullptr,
                                     T, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 2 * M, 2 * N, K))
        return rc;
    launch_begin(d);
    constexpr auto kern = i16_combine_kernel;
    kern<<<resident_blocks<kern>(d, (int64_t)M * N), 256, 0, d->stream>>>(
        T, rs, cs, C, M, N, 16384u * (uint32_t)K);
    return launch_end(d, "gemm_i16 (combine)");
}

// ------------------------------------------------- mixer blocks and RNN cell
namespace hx {
namespace {
constexpr int kSlotMixQ = 19, kSlotMixY = 20, kSlotMixT = 21, kSlotMixX = 22, kSlotMixXt = 23;

// out [C][R] = in [R][C] (int8), 32 x 32 tiles through shared memory
__global__ void __launch_bounds__(256) transpose_i8_kernel(const int8_t *__restrict__ in,
                                                           int8_t *__restrict__ out, int R, int C) {
    __shared__ int8_t t[32][33];
    const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    for (int k = threadIdx.x; k < 32 * 32; k += blockDim.x) {
        const int r = k / 32, c = k % 32;
        if (r0 + r < R && c0 + c < C) t[r][c] = in[(size_t)(r0 + r) * C + c0 + c];
    }
    __syncthreads();
    for (int k = threadIdx.x; k < 32 * 32; k += blockDim.x) {
        const int c = k / 32, r = k % 32;
        if (r0 + r < R && c0 + c < C) out[(size_t)(c0 + c) * R + r0 + r] = t[r][c];
    }
}

int transpose_i8(Dev *d, const int8_t *in, int8_t *out, int R, int C) {
    launch_begin(d);
    transpose_i8_kernel<<<dim3((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32)), 256, 0,
                          d->stream>>>(in, out, R, C);
    return launch_end(d, "transpose_i8");
}
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_mix_mlp_i8(int dev, const int8_t *X, const int8_t *W1, const int32_t *b1,
                                 const int8_t *lut, const int8_t *W2, const int32_t *b2, int8_t *out,
                                 int M, int K, int V, int D, int32_t mult1, int shift1,
                                 int32_t mult2, int shift2) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "mix_mlp_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    const size_t n = (size_t)M * (V > 0 ? V : 1);
    int8_t *q = reinterpret_cast<int8_t *>(scratch(d, kSlotMixQ, n));
    int8_t *y = reinterpret_cast<int8_t *>(scratch(d, kSlotMixY, n));
    if (!q || !y) return HEXCUDA_ERR_OOM;
    if (V > 0) {
        if (int rc = hexcuda_gemm_i8_rq_ex(dev, X, W1, 1, b1, nullptr, q, M, V, K, mult1, shift1, 0, 0))
            return rc;
        if (lut) {
            // y = lut[(uint8)(q + 128)]: q + 128 lies in [0, 255]
            if (int rc = hexcuda_requant_ew(dev, q, 1, nullptr, 0, y, (int64_t)M * V, HEXCUDA_RQ_PRE_A, 0,
                                            1, 0, 128, 0, 0, 255, 0, 255, lut))
                return rc;
        } else {
            y = q;
        }
    }
    return hexcuda_gemm_i8_rq_ex(dev, y, W2, 1, b2, nullptr, out, M, D, V, mult2, shift2, 0, 0);
}

HX_EXPORT int hexcuda_token_mix_i8(int dev, const int8_t *X, const int8_t *W, const int32_t *b,
                                   const int8_t *W2, const int32_t *b2, int8_t *out, int T, int C,
                                   int DM, int32_t mult1, int shift1, int32_t mult2, int shift2) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (T < 0 || C < 0 || DM < 0) return fail(HEXCUDA_ERR_ARG, "token_mix_i8: bad shape");
    if (T == 0 || C == 0) return HEXCUDA_OK;
    if (!X || !out) return fail(HEXCUDA_ERR_ARG, "token_mix_i8: null pointer");
    int8_t *xt = reinterpret_cast<int8_t *>(scratch(d, kSlotMixXt, (size_t)T * C));
    int8_t *ot = reinterpret_cast<int8_t *>(scratch(d, kSlotMixT, (size_t)T * C));
    if (!xt || !ot) return HEXCUDA_ERR_OOM;
    // mixing along the tokens is the channel MLP of X^T (channels as rows)
    if (int rc = transpose_i8(d, X, xt, T, C)) return rc;
    if (int rc = hexcuda_mix_mlp_i8(dev, xt, W, b, nullptr, W2, b2, ot, C, T, DM, T, mult1, shift1,
                                    mult2, shift2))
        return rc;
    return transpose_i8(d, ot, out, C, T);
}

HX_EXPORT int hexcuda_rnn_cell_i8(int dev, const int8_t *Wx, const int8_t *Wh, const int32_t *b,
                                  const int8_t *x, const int8_t *h_prev, int8_t *h_t, int H, int I,
                                  int32_t mult, int shift, int8_t zp, const int8_t *tanh_lut) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (H < 0 || I < 0) return fail(HEXCUDA_ERR_ARG, "rnn_cell_i8: H %d I %d", H, I);
    if (H == 0) return HEXCUDA_OK;
    if (!Wh || !b || !h_prev || !h_t || !tanh_lut || (I > 0 && (!Wx || !x)))
        return fail(HEXCUDA_ERR_ARG, "rnn_cell_i8: null pointer");
    const int KK = I + H;
    int8_t *W = reinterpret_cast<int8_t *>(scratch(d, kSlotMixT, (size_t)H * KK));
    int8_t *xh = reinterpret_cast<int8_t *>(scratch(d, kSlotMixX, (size_t)KK));
    int8_t *q = reinterpret_cast<int8_t *>(scratch(d, kSlotMixQ, (size_t)H));
    if (!W || !xh || !q) return HEXCUDA_ERR_OOM;
    // [Wx | Wh] (H x (I + H)) and [x, h_prev]: one matrix-vector product
    launch_begin(d);
    int rc = HEXCUDA_OK;
    if (I > 0) {
        rc = check(cudaMemcpy2DAsync(W, KK, Wx, I, I, H, cudaMemcpyDeviceToDevice, d->stream), "copy Wx");
        if (!rc) rc = check(cudaMemcpyAsync(xh, x, I, cudaMemcpyDeviceToDevice, d->stream), "copy x");
    }
    if (!rc) rc = check(cudaMemcpy2DAsync(W + I, KK, Wh, H, H, H, cudaMemcpyDeviceToDevice, d->stream),
                        "copy Wh");
    if (!rc) rc = check(cudaMemcpyAsync(xh + I, h_prev, H, cudaMemcpyDeviceToDevice, d->stream),
                        "copy h_prev");
    if (rc) return rc;
    if ((rc = launch_end(d, "rnn_cell_i8 (pack)", 0))) return rc;
    if ((rc = hexcuda_gemm_i8_rq_ex(dev, xh, W, 1, b, nullptr, q, 1, H, KK, mult, shift, zp, 0)))
        return rc;
    // h_t = tanh_lut[(uint8) q]
    return hexcuda_requant_ew(dev, q, 1, nullptr, 0, h_t, H, HEXCUDA_RQ_PRE_A, 0, 1, 0, 0, 0,
                              -128, 127, -128, 127, tanh_lut);
}

// ------------------------------------------------ HMX-convention convolution
//
// out[co][p] = epilogue(sum_{ci, kh, kw} W[co][ci][kh][kw] in[ci][window(p)])
// as the HMX-convention GEMM of the window matrix (rows = output positions,
// u8) by W^T (W row-major [c_out][c_in kh kw] is its K-major Bt), stored
// column-major so that out is [c_out][positions].
namespace hx {
namespace {
constexpr int kSlotConvCol = 23;

__global__ void __launch_bounds__(256) im2col_u8_kernel(const uint8_t *__restrict__ in,
                                                        uint8_t *__restrict__ col, int C, int IH,
                                                        int IW, int KH, int KW, int stride, int OW,
                                                        int64_t n) {
    const int kk = C * KH * KW;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += step) {
        const int p = (int)(t / kk), r = (int)(t % kk);
        const int ci = r / (KH * KW), kh = (r / KW) % KH, kw = r % KW;
        const int oh = p / OW, ow = p % OW;
        col[t] = in[((size_t)ci * IH + oh * stride + kh) * IW + ow * stride + kw];
    }
}
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_conv2d_hmx(int dev, const uint8_t *in, const int8_t *W, const int32_t *bias,
                                 void *out, int store, int act, int c_in, int ih, int iw, int c_out,
                                 int kh, int kw, int stride) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (c_in < 1 || c_out < 1 || kh < 1 || kw < 1 || stride < 1 || ih < kh || iw < kw)
        return fail(HEXCUDA_ERR_ARG, "conv2d_hmx: c_in %d %dx%d c_out %d kernel %dx%d stride %d", c_in, ih,
                    iw, c_out, kh, kw, stride);
    if (store != HEXCUDA_HMX_STORE_I32 && store != HEXCUDA_HMX_STORE_I8_SAT &&
        store != HEXCUDA_HMX_STORE_U16_FIELD)
        return fail(HEXCUDA_ERR_ARG, "conv2d_hmx: store kind %d", store);
    if (!in || !W || !out) return fail(HEXCUDA_ERR_ARG, "conv2d_hmx: null pointer");
    const int oh = (ih - kh) / stride + 1, ow = (iw - kw) / stride + 1;
    const int P = oh * ow, KK = c_in * kh * kw;
    uint8_t *col = reinterpret_cast<uint8_t *>(scratch(d, kSlotConvCol, (size_t)P * KK));
    if (!col) return HEXCUDA_ERR_OOM;
    launch_begin(d);
    constexpr auto kern = im2col_u8_kernel;
    kern<<<resident_blocks<kern>(d, (int64_t)P * KK), 256, 0, d->stream>>>(
        in, col, c_in, ih, iw, kh, kw, stride, ow, (int64_t)P * KK);
    if (int rc = launch_end(d, "conv2d_hmx (im2col)")) return rc;
    return hexcuda_gemm_hmx_ex(dev, col, W, 1, bias, nullptr, HEXCUDA_HMX_RES_NONE, nullptr, out, store,
                               act, 1, P, c_out, KK, 0);
}

HX_EXPORT int hexcuda_ffn_hmx_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                 const int8_t *W2, const int32_t *b2, int8_t *out, int M, int D,
                                 int Dff, int sh1, int sh2) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || D < 0 || Dff < 0 || sh1 < 0 || sh1 > 31 || sh2 < 0 || sh2 > 31)
        return fail(HEXCUDA_ERR_ARG, "ffn_hmx_i8: M %d D %d Dff %d shifts %d / %d", M, D, Dff, sh1, sh2);
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (!X || !W1 || !b1 || !W2 || !b2 || !out) return fail(HEXCUDA_ERR_ARG, "ffn_hmx_i8: null pointer");
    int8_t *hid = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHidden, (size_t)M * (Dff > 0 ? Dff : 1)));
    if (!hid) return HEXCUDA_ERR_OOM;
    if (int rc = hmx_shift_gemm(dev, X, W1, b1, hid, M, Dff, D, kActReluShr, sh1, "ffn_hmx_i8 (up)"))
        return rc;
    // hid is in [0, 127]: its bytes read the same as u8
    return hmx_shift_gemm(dev, reinterpret_cast<const uint8_t *>(hid), W2, b2, out, M, D, Dff, kActShr,
                          sh2, "ffn_hmx_i8 (down)");
}

HX_EXPORT int hexcuda_ffn_swiglu_hmx_i8(int dev, const uint8_t *X, const int8_t *Wg,
                                        const int8_t *Wu, const int8_t *Wd, const int32_t *bd,
                                        const uint8_t *silu_lut, int8_t *out, int M, int D, int Dff,
                                        int sg, int su, int sh, int zp, int so) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || D < 0 || Dff < 0 || sg < 0 || sg > 31 || su < 0 || su > 31 || sh < 0 || sh > 31 ||
        so < 0 || so > 31 || zp < 1 || zp > 128)
        return fail(HEXCUDA_ERR_ARG, "ffn_swiglu_hmx_i8: M %d D %d Dff %d sg %d su %d sh %d zp %d so %d",
                    M, D, Dff, sg, su, sh, zp, so);
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (!X || !Wg || !Wu || !Wd || !bd || !silu_lut || !out)
        return fail(HEXCUDA_ERR_ARG, "ffn_swiglu_hmx_i8: null pointer");
    const size_t n = (size_t)M * (Dff > 0 ? Dff : 1);
    int8_t *g = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHidden, n));
    int8_t *u = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHidden + 1, n));
    uint8_t *hu = reinterpret_cast<uint8_t *>(scratch(d, kSlotFfnHidden + 2, n));
    if (!g || !u || !hu) return HEXCUDA_ERR_OOM;
    if (Dff > 0) {
        if (int rc = hmx_shift_gemm(dev, X, Wg, nullptr, g, M, Dff, D, kActShr, sg, "ffn_swiglu (gate)"))
            return rc;
        if (int rc = hmx_shift_gemm(dev, X, Wu, nullptr, u, M, Dff, D, kActShr, su, "ffn_swiglu (up)"))
            return rc;
        launch_begin(d);
        constexpr auto kern = swiglu_gate_kernel;
        kern<<<resident_blocks<kern>(d, (int64_t)M * Dff), 256, 0, d->stream>>>(
            g, u, silu_lut, hu, (int64_t)M * Dff, sh, zp);
        if (int rc = launch_end(d, "ffn_swiglu (gate x up)")) return rc;
    }
    return hmx_shift_gemm(dev, hu, Wd, bd, out, M, D, Dff, kActShr, so, "ffn_swiglu (down)");
}

HX_EXPORT int hexcuda_gemm_hmx(int dev, const uint8_t *A, const int8_t *B, int b_transposed,
                               const int32_t *bias, void *out, int out_kind, int M, int N, int K,
                               int32_t zpA) {
    if (out_kind < HEXCUDA_HMX_OUT_I32 || out_kind > HEXCUDA_HMX_OUT_U8_BIAS_RELU)
        return fail(HEXCUDA_ERR_ARG, "gemm_hmx: out_kind %d", out_kind);
    if (out_kind == HEXCUDA_HMX_OUT_U8_BIAS_RELU) {
        if (!bias && N > 0) return fail(HEXCUDA_ERR_ARG, "gemm_hmx: null bias");
        return hexcuda_gemm_hmx_ex(dev, A, B, b_transposed, bias, nullptr, HEXCUDA_HMX_RES_NONE,
                                   nullptr, out, HEXCUDA_HMX_STORE_U8_SAT, HEXCUDA_HMX_ACT_RELU, 0,
                                   M, N, K, zpA);
    }
    return hexcuda_gemm_hmx_ex(dev, A, B, b_transposed, nullptr, nullptr, HEXCUDA_HMX_RES_NONE,
                               nullptr, out,
                               out_kind == HEXCUDA_HMX_OUT_I32 ? HEXCUDA_HMX_STORE_I32
                                                               : HEXCUDA_HMX_STORE_I8_SAT,
                               HEXCUDA_HMX_ACT_NONE, 0, M, N, K, zpA);
}

// ------------------------------------------------ no-allocation u8 x s8 GEMM
//
// hexcuda_gemm_u8s8_pc_noalloc: the u8 x s8 per-channel GEMM for callers that
// must not have the library allocate device memory -- a runtime that reserved
// the GPU's memory up front for its own arena, where a library cudaMalloc
// would fail or fragment it, or a latency-bound caller that cannot take the
// implicit device synchronisation of cudaMalloc / cudaFree.  The regular entry
// keeps its K-major copy of B and the column sums in grow-only scratch it
// allocates on first use; this one uses a fixed region compiled into the
// library instead (every GPU that loads libhexcuda holds it until exit):
//   g_na_bt      K-major copy of B, at most kNoAllocBtBytes bytes
//                (round_up(K, 128) * N <= 16 MiB);
//   g_na_colsum  column sums of B, N <= kNoAllocMaxN.
// A is read in place, so its rows must start on 16 bytes (K % 16 == 0, K >= 128).
// Larger or unaligned problems are rejected with HEXCUDA_ERR_ARG.  With
// zpA == 0 the column sums are not needed and neither cleared nor computed
// (the transpose pass then only copies B), as in the regular entry.
namespace hx {
namespace {

constexpr size_t kNoAllocBtBytes = 16u << 20;
constexpr int kNoAllocMaxN = 16384;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_na_bt[kNoAllocBtBytes];
static __device__ __align__(256) int32_t g_na_colsum[kNoAllocMaxN];

struct NoAllocPtrs {
    std::once_flag once;
    int rc = HEXCUDA_OK;
    uint8_t *bt = nullptr;
    int32_t *colsum = nullptr;
};

// Device addresses of the fixed region on device `d` (current).  In host code
// the arrays' names are host-side stand-ins, not device addresses; the real
// addresses come from cudaGetSymbolAddress, queried once per device (once even
// when two host threads make their first call at the same time).
int noalloc_ptrs(Dev *d, NoAllocPtrs **out) {
    static NoAllocPtrs per_dev[kNoAllocMaxDevices];
    if (d->ordinal < 0 || d->ordinal >= kNoAllocMaxDevices)
        return fail(HEXCUDA_ERR_ARG, "gemm_u8s8_pc_noalloc: device ordinal %d >= %d", d->ordinal,
                    kNoAllocMaxDevices);
    NoAllocPtrs &p = per_dev[d->ordinal];
    std::call_once(p.once, [&] {
        p.rc = check(cudaGetSymbolAddress(reinterpret_cast<void **>(&p.bt), g_na_bt),
                     "cudaGetSymbolAddress(g_na_bt)");
        if (!p.rc)
            p.rc = check(cudaGetSymbolAddress(reinterpret_cast<void **>(&p.colsum), g_na_colsum),
                         "cudaGetSymbolAddress(g_na_colsum)");
    });
    if (p.rc) return p.rc;
    *out = &p;
    return HEXCUDA_OK;
}

}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_gemm_u8s8_pc_noalloc(int dev, const uint8_t *A, const int8_t *B,
                                           const int32_t *bias, uint8_t *out, int M, int N, int K,
                                           int32_t zpA, const int32_t *mult, const int *shift,
                                           uint8_t zp_out) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || N < 0 || K < 0)
        return fail(HEXCUDA_ERR_ARG, "gemm_u8s8_pc_noalloc: bad shape %dx%dx%d", M, N, K);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (!A || !B || !bias || !mult || !shift || !out)
        return fail(HEXCUDA_ERR_ARG, "gemm_u8s8_pc_noalloc: null pointer");
    const int64_t Kp = round_up(K, kBKBytes);
    if (N > kNoAllocMaxN || Kp * (int64_t)N > (int64_t)kNoAllocBtBytes)
        return fail(HEXCUDA_ERR_ARG,
                    "gemm_u8s8_pc_noalloc: N=%d K=%d exceeds the fixed scratch (N <= %d, "
                    "round_up(K,128)*N <= %zu bytes); use hexcuda_gemm_u8s8_pc",
                    N, K, kNoAllocMaxN, kNoAllocBtBytes);
    if (K < kBKBytes || (K % 16) != 0 || !aligned16(A))
        return fail(HEXCUDA_ERR_ARG,
                    "gemm_u8s8_pc_noalloc: A rows must be 16-byte aligned with K >= 128 and "
                    "K %% 16 == 0 (K=%d)",
                    K);
    NoAllocPtrs *np = nullptr;
    if (int rc = noalloc_ptrs(d, &np)) return rc;

    EpiParams ep = requant_epi(out, N, 0, 0, zp_out, 0, 255);
    ep.zpA = zpA;
    ep.bias = bias;
    ep.mult_pc = mult;
    ep.shift_pc = shift;
    ep.colsum = zpA ? np->colsum : nullptr;
    ep.M = M;
    ep.N = N;

    launch_begin(d);
    dim3 g((unsigned)((N + 63) / 64), (unsigned)(Kp / 64));
    if (zpA) {
        // the column sums accumulate atomically: clear them first (every call
        // shares this region; calls that overlap on the GPU race on it)
        if (int rc = check(cudaMemsetAsync(np->colsum, 0, sizeof(int32_t) * (size_t)N, d->stream),
                           "memset colsum"))
            return rc;
        transpose_pack_kernel<uint8_t, true><<<g, 256, 0, d->stream>>>(
            reinterpret_cast<const uint8_t *>(B), np->bt, np->colsum, K, N, N, Kp);
    } else {
        transpose_pack_kernel<uint8_t, false><<<g, 256, 0, d->stream>>>(
            reinterpret_cast<const uint8_t *>(B), np->bt, nullptr, K, N, N, Kp);
    }
    CUtensorMap ta, tb;
    if (int rc = make_kmajor_map(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, kBM)) return rc;
    int rc;
    if (N <= 128) {
        if ((rc = make_kmajor_map(&tb, np->bt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Kp, N, Kp, 128)))
            return rc;
        // no tail split: its workspace would be allocated scratch
        rc = launch_gemm_kernel<MmaKind::I8, 128, kEpiRequant, false, true>(d, ta, tb, M, N,
                                                                            (int)Kp, ep, false,
                                                                            false);
    } else {
        if ((rc = make_kmajor_map(&tb, np->bt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Kp, N, Kp, 256)))
            return rc;
        rc = launch_gemm_kernel<MmaKind::I8, 256, kEpiRequant, false, true>(d, ta, tb, M, N,
                                                                            (int)Kp, ep, false,
                                                                            false);
    }
    if (rc) return rc;
    return launch_end(d, "gemm_u8s8_pc_noalloc", 2);
}
