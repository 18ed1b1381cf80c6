// sm_100a kernels of the FP8 E4M3 quantized-linear hot path.
//
//   fp8_gemm_kernel      tcgen05 kind::f8f6f4 GEMM, TMA-fed mbarrier ring, fp32
//                        accumulators in TMEM (double buffered), fused epilogue
//                        (per-channel scale, fp16 bias, fp16-edge GELU, fp16 out
//                        and/or E4M3 codes for the next linear), TMA stores.
//   skinny_kernel        small-M (m <= 32, decoder step) linear on tensor cores:
//                        swap-AB tcgen05 MMAs over streamed weight tiles, cluster
//                        split-K reduced through distributed shared memory.
//   quantize kernels     fp16 -> E4M3 with a scalar or per-row scale.
//   scale kernels        per-row weight scales, dynamic activation amax/448.
//   fp16 projections     sm_100a rebuild of the reference plugins' fc1/qkv/bias.
//
// Semantics follow the reference's TensorRT graph: cpp/src/network_graph.cpp
// :115-159 (Q/DQ + MatMul + bias) and :168-180 (GELU with fp16 edges), and the
// fp16 plugin kernels of cpp/kernels.cu:10-78.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <tuple>
#include <type_traits>
#include <set>
#include <utility>
#include <vector>

#include "launch.h"
#include "lffw_fp8.h"
#include "ptx.cuh"

#include "erf_table.inc"

namespace lffw {

namespace {
std::atomic<uint64_t> g_launches{0};
}

// Device copy of the fp16 erf table (see erf_table.inc); copied into shared
// memory by the GELU epilogue at kernel start.  Padded to a whole number of
// 32-bit words.
__device__ __align__(16) const uint16_t g_erf_table[(LFFW_ERF_TABLE_SIZE + 1) / 2 * 2] = {LFFW_ERF_TABLE_VALUES};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// Scalar helpers.  Explicit .rn on the f16 ops keeps ptxas from contracting a
// multiply and an add into one fma: every fp16 graph edge rounds on its own.

__device__ __forceinline__ float h2f(uint16_t h)
{
    float f;
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return f;
}

__device__ __forceinline__ uint16_t f2h_rn(float f)
{
    uint16_t h;
    asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
    return h;
}

__device__ __forceinline__ uint16_t hadd_rn(uint16_t a, uint16_t b)
{
    uint16_t r;
    asm("add.rn.f16 %0, %1, %2;" : "=h"(r) : "h"(a), "h"(b));
    return r;
}

__device__ __forceinline__ uint16_t hmul_rn(uint16_t a, uint16_t b)
{
    uint16_t r;
    asm("mul.rn.f16 %0, %1, %2;" : "=h"(r) : "h"(a), "h"(b));
    return r;
}

// GELU with the reference graph's fp16 edges: (x*0.5)*(1+erf(x*fp16(2^-1/2))).
__device__ __forceinline__ uint16_t gelu_fp16_edges(uint16_t x)
{
    constexpr uint16_t kInvSqrt2 = 0x39A8; // 0.70703125 = fp16(2^-0.5)
    constexpr uint16_t kHalf = 0x3800;
    constexpr uint16_t kOne = 0x3C00;
    uint16_t scaled = hmul_rn(x, kInvSqrt2);
    uint16_t erf16 = f2h_rn(erff(h2f(scaled)));
    uint16_t left = hmul_rn(x, kHalf);
    uint16_t right = hadd_rn(kOne, erf16);
    return hmul_rn(left, right);
}

// 16 bytes read once: non-coherent, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream16(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Two fp32 values -> two E4M3 codes (round to nearest even, saturate finite);
// `lo` lands in the low byte.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi)
{
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Q of one fp16 value: fp32 IEEE quotient, then E4M3.
__device__ __forceinline__ float q_quotient(uint16_t h, float scale)
{
    return __fdiv_rn(h2f(h), scale);
}

__device__ __forceinline__ uint64_t f2_bits(float lo, float hi)
{
    return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}

// Two E4M3 codes (low byte = low half) of the packed fp16 pair h2 divided by
// `scale`, with y = RN(1/scale): the division-free quotient below on f32x2.
// Zero and infinite inputs keep q0 (= +-0 or +-inf, whose codes are +-0 and
// +-448), NaN stays NaN; everything else takes the corrected quotient.
__device__ __forceinline__ uint32_t e4m3x2_quotient(uint32_t h2, uint64_t scale2_neg, uint64_t recip2)
{
    const uint64_t x = f2_bits(h2f(static_cast<uint16_t>(h2 & 0xFFFFu)), h2f(static_cast<uint16_t>(h2 >> 16)));
    uint64_t q0, r, q1;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q0) : "l"(x), "l"(recip2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(scale2_neg), "l"(q0), "l"(x));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(q1) : "l"(r), "l"(recip2), "l"(q0));
    const float q0l = __uint_as_float(static_cast<uint32_t>(q0)), q0h = __uint_as_float(static_cast<uint32_t>(q0 >> 32));
    const float q1l = __uint_as_float(static_cast<uint32_t>(q1)), q1h = __uint_as_float(static_cast<uint32_t>(q1 >> 32));
    const float ql = (fabsf(q0l) == 0.0f || fabsf(q0l) == __int_as_float(0x7F800000)) ? q0l : q1l;
    const float qh = (fabsf(q0h) == 0.0f || fabsf(q0h) == __int_as_float(0x7F800000)) ? q0h : q1h;
    return e4m3x2(ql, qh);
}

// Scales for which the lean quotient below is exact: 65504 / 128 > 448, so a
// magnitude clamped to 65504 (an infinity) still saturates, and
// 65504 * 2^110 < 2^128, so no product overflows.
__host__ __device__ __forceinline__ bool lean_scale(float scale)
{
    return scale >= 0x1p-110f && scale <= 128.0f;
}

// E4M3 codes of |h2| / scale (sign bits clear) for a lean scale: the magnitude
// is clamped to 65504 with min.NaN (NaN stays NaN), then takes the same
// corrected quotient as e4m3x2_quotient; zero needs no special case.
__device__ __forceinline__ uint32_t e4m3x2_magnitude(uint32_t h2, uint64_t scale2_neg, uint64_t recip2)
{
    uint32_t a;
    asm("min.NaN.f16x2 %0, %1, %2;" : "=r"(a) : "r"(h2 & 0x7FFF7FFFu), "r"(0x7BFF7BFFu));
    const uint64_t x = f2_bits(h2f(static_cast<uint16_t>(a & 0xFFFFu)), h2f(static_cast<uint16_t>(a >> 16)));
    uint64_t q0, r, q1;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q0) : "l"(x), "l"(recip2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(scale2_neg), "l"(q0), "l"(x));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(q1) : "l"(r), "l"(recip2), "l"(q0));
    return e4m3x2(__uint_as_float(static_cast<uint32_t>(q1)), __uint_as_float(static_cast<uint32_t>(q1 >> 32)));
}

// Four E4M3 codes (byte i = half i of h01, h23) for a lean scale: magnitudes,
// then each input's sign bit copied onto its code (prmt replicates the sign
// of bytes 1, 3, 5, 7 -- the fp16 sign bits -- across result bytes 0-3).
__device__ __forceinline__ uint32_t e4m3x4_lean(uint32_t h01, uint32_t h23, uint64_t scale2_neg, uint64_t recip2)
{
    const uint32_t lo = e4m3x2_magnitude(h01, scale2_neg, recip2);
    const uint32_t hi = e4m3x2_magnitude(h23, scale2_neg, recip2);
    uint32_t q, sign;
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(q) : "r"(lo), "r"(hi));
    asm("prmt.b32 %0, %1, %2, 0xFDB9;" : "=r"(sign) : "r"(h01), "r"(h23));
    return q | (sign & 0x80808080u);
}

// Four codes by whichever quotient the scale admits (`lean` is uniform).
__device__ __forceinline__ uint32_t e4m3x4(uint32_t h01, uint32_t h23, bool lean, uint64_t scale2_neg, uint64_t recip2)
{
    if (lean)
        return e4m3x4_lean(h01, h23, scale2_neg, recip2);
    return e4m3x2_quotient(h01, scale2_neg, recip2) | (e4m3x2_quotient(h23, scale2_neg, recip2) << 16);
}


// ---------------------------------------------------------------------------
// FP8 GEMM (tcgen05)
//
// Persistent, warp-specialized: warp 0 issues TMA loads into a ring of shared
// memory stages, warp 1 issues tcgen05.mma (one thread) into one of two TMEM
// accumulators, warps 2-17 drain the other accumulator through the epilogue.
// Each epilogue warp owns 32 TMEM lanes (rows) x a quarter of the tile's
// columns and stores its own 32 x 32 sub-blocks with TMA from a private
// staging buffer, so no epilogue warp ever waits for another; four warps per
// lane quarter keep the scale / GELU / quotient arithmetic latency hidden.

namespace gemm {

constexpr int kBM = 128;       // tile rows (TMEM lanes)
constexpr int kBK = 128;       // K bytes per stage = one 128B swizzle row
constexpr int kUmmaK = 32;     // K of one kind::f8f6f4 MMA
constexpr int kEpiWarps = 16;             // 4 per TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreads = 64 + kEpiThreads; // warp 0 TMA, warp 1 MMA, warps 2-17 epilogue
constexpr int kSub = 32;                   // columns per epilogue store

enum : int {
    kEpiGelu = 1,
    kEpiY = 2,
    kEpiCodes = 4,
    // Operands are fp16 (kind::f16 MMAs, 64 elements per 128-byte K block) and
    // the per-channel scale is 1: the encoder's fp16 convolutions.
    kEpiF16In = 8,
    // y = fp16(acc * scale + bias) with the bias added in fp32 (one rounding),
    // a convolution layer's own bias, instead of the linear's fp16 bias edge.
    kEpiBiasF32 = 16,
    // After the GELU: y = fp16(y + pos[t]), the positional embedding of row t
    // of its segment (network_graph.cpp:280-282).  Without kEpiSeg, pos is an
    // [m, pos_ld] tensor read at the output's own row: the residual add of
    // network_graph.cpp:285-287 after a linear's bias.
    kEpiPos = 32,
    // Rows form segments (streams) of p.seg_rows: tiles never straddle two
    // segments; A is read through 3-D maps (k, row, segment), one per
    // convolution tap, and outputs are stored through 3-D maps.
    kEpiSeg = 64,
    // The fp16 output is stored split by heads: column c of row t of segment s
    // lands at [c / (64 H)][s][(c / 64) % H][t][c % 64] (requires kEpiSeg).
    kEpiHeads = 128,
};

// kPair: a cluster of two CTAs computes a 256 x BN tile with cta_group::2 MMAs.
// Each CTA loads its 128 rows of A and its BN/2 rows of B (the pair's B tile is
// split along N), holds its 128 rows of the accumulator in its own TMEM, and
// runs its own epilogue.  Per SM that halves the B operand traffic.
template <int BN, int EPI, bool kPair>
struct Cfg {
    static constexpr bool kGelu = (EPI & kEpiGelu) != 0;
    static constexpr bool kY = (EPI & kEpiY) != 0;
    static constexpr bool kCodes = (EPI & kEpiCodes) != 0;
    static constexpr bool kF16In = (EPI & kEpiF16In) != 0;
    static constexpr bool kBiasF32 = (EPI & kEpiBiasF32) != 0;
    static constexpr bool kPos = (EPI & kEpiPos) != 0;
    static constexpr bool kSeg = (EPI & kEpiSeg) != 0;
    static constexpr bool kHeads = (EPI & kEpiHeads) != 0;
    static_assert(!kHeads || (kSeg && kY && !kCodes), "head-split stores: segmented fp16 output only");
    static constexpr int kKElems = kF16In ? kBK / 2 : kBK; // elements per 128-byte K block
    static constexpr int kTileM = kPair ? 2 * kBM : kBM;
    static constexpr int kBRows = kPair ? BN / 2 : BN; // B rows this CTA loads
    static constexpr int kABytes = kBM * kBK;
    static constexpr int kBBytes = kBRows * kBK;
    static constexpr int kStageBytes = kABytes + kBBytes;                // per CTA
    static constexpr int kTxBytes = kPair ? 2 * kStageBytes : kStageBytes; // counted on the leader
    static constexpr int kYBuf = 32 * kSub * 2; // 32 rows x 64 B (fp16), 64B swizzle
    static constexpr int kCBuf = 32 * kSub;     // 32 rows x 32 B (E4M3), 32B swizzle
    static constexpr int kWarpStaging = (kY ? kYBuf : 0) + (kCodes ? kCBuf : 0);
    static constexpr int kStagingBytes = kEpiWarps * kWarpStaging;
    // GELU with E4M3 codes as the only output: the codes are a function of the
    // 16-bit pre-GELU value alone, so the epilogue reads them from a 64 KB
    // table (one code per fp16 bit pattern) built per launch.  Otherwise the
    // GELU reads fp16(erf) from a table of the non-negative fp16 inputs.
    static constexpr bool kCodeTable = kGelu && kCodes && !kY;
    static constexpr int kTableBytes =
        kCodeTable ? 65536 : (kGelu ? (LFFW_ERF_TABLE_SIZE * 2 + 1023) / 1024 * 1024 : 0);
    static constexpr int kBarBytes = 256;
    static constexpr int kBudget = 232448 - 1024; // opt-in maximum minus base alignment slack
    static constexpr int kFit = (kBudget - kStagingBytes - kTableBytes - kBarBytes) / kStageBytes;
    static constexpr int kStages = kFit > 6 ? 6 : kFit;
    static constexpr int kOffB = kStages * kABytes;
    static constexpr int kOffStaging = kOffB + kStages * kBBytes;
    static constexpr int kOffTable = kOffStaging + kStagingBytes;
    static constexpr int kOffBar = kOffTable + kTableBytes;
    static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512; // two accumulators, allocated as a power of two
    static constexpr int kSubs = BN / kSub;                      // 32-column store boxes per tile
    static_assert(BN % kSub == 0 && kSubs <= 8, "tile width: a multiple of 32, at most 256");
    static constexpr int kAccEmptyArrivals = kPair ? 2 * kEpiWarps : kEpiWarps;
    static_assert(kStages >= 3, "pipeline depth");
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert((2 * kStages + 5) * 8 + 8 <= kBarBytes, "barrier area");
    static_assert(2 * BN <= kTmemCols, "TMEM columns");
    static_assert(kY || kCodes, "an output is required");
};

struct Params {
    int m, n, k;
    int m_tiles, num_tiles, num_kb;
    int n_tiles, group_m;    // raster: see tile_coords
    int seg_rows, seg_tiles; // kEpiSeg: rows per segment, tiles per segment
    int kb_per_tap;          // kEpiSeg: K blocks per A map (convolution tap)
    int heads;               // kEpiHeads: H
    const uint16_t *pos;     // kEpiPos: fp16 [seg_rows, pos_ld] (segmented) or [m, pos_ld] (residual)
    int pos_ld;
    float act_scale;
    const float *act_scale_ptr;
    const float *w_scales;
    const uint16_t *bias;
    float next_scale;
    float next_recip; // RN(1 / next_scale)
    int next_lean;    // lean_scale(next_scale)
};

// fp16(erf(x)) of two packed fp16 values, rounded to nearest even: one table
// read per value.  The table covers every non-negative fp16 input up to
// 0x4131, whose entry is 1.0 like erf of every larger input; NaN inputs read
// 1.0 too, which leaves GELU's result NaN through its x*0.5 factor.
__device__ __forceinline__ uint32_t erf_fp16x2(uint32_t s2, const uint16_t *table)
{
    uint32_t idx;
    asm("min.u16x2 %0, %1, %2;" : "=r"(idx) : "r"(s2 & 0x7FFF7FFFu), "r"(LFFW_ERF_TABLE_HI * 0x10001u));
    const uint32_t lo = table[idx & 0xFFFFu];
    const uint32_t hi = table[idx >> 16];
    return (lo | (hi << 16)) | (s2 & 0x80008000u);
}

__device__ __forceinline__ uint32_t cvt_f16x2(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t hadd2_rn(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b)
{
    uint64_t x, y, z;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
    float2 r;
    memcpy(&r, &z, 8);
    return r;
}

// GELU on two fp16 values with every graph edge rounded to fp16.
__device__ __forceinline__ uint32_t gelu_fp16x2(uint32_t x, const uint16_t *table)
{
    const uint32_t scaled = hmul2_rn(x, 0x39A839A8u); // x * fp16(2^-1/2)
    const uint32_t e = erf_fp16x2(scaled, table);
    const uint32_t left = hmul2_rn(x, 0x38003800u);   // x * 0.5
    const uint32_t right = hadd2_rn(0x3C003C00u, e);  // 1 + erf
    return hmul2_rn(left, right);
}

template <int BN, int EPI, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_c,
                    const __grid_constant__ CUtensorMap tm_a1, const __grid_constant__ CUtensorMap tm_a2,
                    const Params p)
{
    using C = Cfg<BN, EPI, kPair>;
    // Segment and first row (within the segment, or of the whole matrix) of this
    // CTA's 128 rows of tile t.
    // Tile t -> (M tile, N tile).  group_m = 0 walks the tiles column by column
    // (M fastest).  Otherwise tiles go in groups of group_m M tiles, each group
    // column by column, so that the waves in flight share a few A row panels and
    // every panel is reused from L2 by all N tiles instead of being read once per
    // column (an A operand larger than L2 is otherwise re-read from DRAM for every
    // column).  A function of t alone: the producer, MMA and epilogue agree.
    auto tile_coords = [&](int t) {
        if (p.group_m <= 0)
            return int2{t % p.m_tiles, t / p.m_tiles};
        const int per_group = p.group_m * p.n_tiles;
        const int g = t / per_group;
        const int first = g * p.group_m;
        const int rows = min(p.group_m, p.m_tiles - first);
        const int r = t - g * per_group;
        return int2{first + r % rows, r / rows};
    };
    auto tile_rows = [&](int t, uint32_t r) {
        const int mt = tile_coords(t).x;
        if (C::kSeg)
            return int2{mt / p.seg_tiles, (mt % p.seg_tiles) * C::kTileM + static_cast<int>(r) * kBM};
        return int2{0, mt * C::kTileM + static_cast<int>(r) * kBM};
    };
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u; // 0 = leader of the pair
    const bool leader = rank == 0;
    const int tile_step = kPair ? static_cast<int>(gridDim.x / 2) : static_cast<int>(gridDim.x);
    const int tile_first = kPair ? static_cast<int>(blockIdx.x / 2) : static_cast<int>(blockIdx.x);
    const uint32_t bar_full = sbase + C::kOffBar;
    const uint32_t bar_empty = bar_full + 8 * C::kStages;
    const uint32_t bar_acc_full = bar_empty + 8 * C::kStages;
    const uint32_t bar_acc_empty = bar_acc_full + 16;
    const uint32_t bar_drain = bar_acc_empty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kOffBar + (2 * C::kStages + 5) * 8);
    uint16_t *erf_table = reinterpret_cast<uint16_t *>(smem + C::kOffTable);

    if (threadIdx.x == 0) {
        // The next kernel on the stream may launch now; it waits for this grid
        // to complete before it reads this grid's outputs.
        griddepcontrol_launch_dependents();
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_acc_full + 8 * a, 1);
            mbar_init(bar_acc_empty + 8 * a, C::kAccEmptyArrivals);
        }
        mbar_init(bar_drain, 1);
        fence_barrier_init();
        prefetch_tensor_map(&tm_a);
        prefetch_tensor_map(&tm_b);
        if (C::kSeg && p.num_kb > p.kb_per_tap) {
            prefetch_tensor_map(&tm_a1);
            prefetch_tensor_map(&tm_a2);
        }
        if (C::kY)
            prefetch_tensor_map(&tm_y);
        if (C::kCodes)
            prefetch_tensor_map(&tm_c);
    }
    if (C::kGelu && !C::kCodeTable) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(g_erf_table);
        uint32_t *dst = reinterpret_cast<uint32_t *>(erf_table);
        for (int i = threadIdx.x; i < (LFFW_ERF_TABLE_SIZE + 1) / 2; i += kThreads)
            dst[i] = src[i];
    }
    if (warp == 1) {
        if (kPair) {
            tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (kPair)
        cluster_sync(); // the peer's barriers exist before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (one thread) ----------------
        if (lane == 0) {
            uint32_t used_mask = 0, parity_mask = 0;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            // The weights do not come from the previous kernel: the first stages'
            // B tiles are requested before waiting for it (stages start empty).
            const int pre = tile_first < p.num_tiles ? (p.num_kb < C::kStages ? p.num_kb : C::kStages) : 0;
            // Arms stage `stage` for a full stage and loads its B (weight) rows; in a
            // pair both CTAs' bytes complete on the leader's barrier, armed by the leader.
            auto arm_and_load_b = [&](int stage, int kb, int n0) {
                const uint32_t full = bar_full + 8 * stage;
                if (kPair) {
                    if (leader)
                        mbar_arrive_expect_tx(full, C::kTxBytes);
                    tma_load_2d_pair(sbase + C::kOffB + stage * C::kBBytes, &tm_b, map_to_rank(full, 0),
                                     kb * C::kKElems, n0);
                } else {
                    mbar_arrive_expect_tx(full, C::kTxBytes);
                    tma_load_2d(sbase + C::kOffB + stage * C::kBBytes, &tm_b, full, kb * C::kKElems, n0);
                }
            };
            // The activation rows of K block kb; segmented A has one 3-D map per tap.
            auto load_a = [&](int stage, int kb, int seg, int r0) {
                const uint32_t full = bar_full + 8 * stage;
                const uint32_t dst = sbase + stage * C::kABytes;
                if (C::kSeg) {
                    const int tap = kb / p.kb_per_tap;
                    const CUtensorMap *map = tap == 0 ? &tm_a : (tap == 1 ? &tm_a1 : &tm_a2);
                    const int x = (kb - tap * p.kb_per_tap) * C::kKElems;
                    if (kPair)
                        tma_load_3d_pair(dst, map, map_to_rank(full, 0), x, r0, seg);
                    else
                        tma_load_3d(dst, map, full, x, r0, seg);
                } else if (kPair) {
                    tma_load_2d_pair(dst, &tm_a, map_to_rank(full, 0), kb * C::kKElems, r0);
                } else {
                    tma_load_2d(dst, &tm_a, full, kb * C::kKElems, r0);
                }
            };
            for (int kb = 0; kb < pre; ++kb)
                arm_and_load_b(kb, kb, tile_coords(tile_first).y * BN + static_cast<int>(rank) * C::kBRows);
            griddepcontrol_wait();
            int issued = 0;
            for (int t = tile_first; ok && t < p.num_tiles; t += tile_step) {
                // In a pair each CTA loads half of the tile's B rows.
                const auto rows = tile_rows(t, rank);
                const int n0 = tile_coords(t).y * BN + static_cast<int>(rank) * C::kBRows;
                for (int kb = 0; kb < p.num_kb; ++kb, ++issued) {
                    if (issued < pre) {
                        // Armed with its B tile above: only the activations remain.
                        load_a(s, kb, rows.x, rows.y);
                    } else {
                        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, kSiteProducerEmpty)) {
                            ok = false;
                            break;
                        }
                        arm_and_load_b(s, kb, n0);
                        load_a(s, kb, rows.x, rows.y);
                    }
                    used_mask |= 1u << s;
                    parity_mask = (parity_mask & ~(1u << s)) | (ph << s);
                    if (++s == C::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            // Every issued load must land before shared memory is released.  In a
            // pair the leader's full barriers count both CTAs' loads.
            if (leader)
                for (int i = 0; i < C::kStages; ++i)
                    if (used_mask & (1u << i)) {
                        const uint32_t par = (parity_mask >> i) & 1u;
                        for (int tries = 0; tries < (1 << 22) && !mbar_try_wait(bar_full + 8 * i, par); ++tries) {
                        }
                    }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread of the leader) ----------------
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = C::kF16In ? idesc_f16_f32<C::kTileM, BN>() : idesc_e4m3_f32<C::kTileM, BN>();
            int s = 0;
            uint32_t ph = 0;
            int local = 0;
            bool ok = true;
            for (int t = tile_first; ok && t < p.num_tiles; t += tile_step, ++local) {
                const uint32_t a = local & 1;
                const uint32_t acc_ph = (local >> 1) & 1;
                if (!mbar_wait(bar_acc_empty + 8 * a, acc_ph ^ 1u, kSiteMmaAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + a * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(bar_full + 8 * s, ph, kSiteMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = sbase + s * C::kABytes;
                    const uint32_t b_addr = sbase + C::kOffB + s * C::kBBytes;
#pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        const uint64_t da = smem_desc_k_sw128(a_addr + k * kUmmaK);
                        const uint64_t db = smem_desc_k_sw128(b_addr + k * kUmmaK);
                        // One MMA covers 32 bytes of K: 32 E4M3 or 16 fp16 elements.
                        if (C::kF16In) {
                            if (kPair)
                                mma_f16_pair(d_tmem, da, db, idesc, (kb | k) != 0);
                            else
                                mma_f16(d_tmem, da, db, idesc, (kb | k) != 0);
                        } else if (kPair) {
                            mma_f8f6f4_pair(d_tmem, da, db, idesc, (kb | k) != 0);
                        } else {
                            mma_f8f6f4(d_tmem, da, db, idesc, (kb | k) != 0);
                        }
                    }
                    // Frees the stage (in both CTAs of a pair) once these MMAs finish.
                    if (kPair)
                        mma_commit_pair_both(bar_empty + 8 * s);
                    else
                        mma_commit(bar_empty + 8 * s);
                    if (++s == C::kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (ok) {
                    if (kPair)
                        mma_commit_pair_both(bar_acc_full + 8 * a);
                    else
                        mma_commit(bar_acc_full + 8 * a);
                }
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            if (kPair)
                mma_commit_pair_local(bar_drain);
            else
                mma_commit(bar_drain);
            for (int tries = 0; tries < (1 << 22) && !mbar_try_wait(bar_drain, 0); ++tries) {
            }
        }
    } else {
        // ---------------- Epilogue: 16 independent warps ----------------
        const int ew = warp - 2;
        const int quarter = warp & 3; // the TMEM lane quarter this warp may access
        const int slice = ew >> 2;    // this warp's 32-column stores: tile subs slice and slice + 4
        const uint64_t neg_scale2 = f2_bits(-p.next_scale, -p.next_scale);
        const uint64_t recip2 = f2_bits(p.next_recip, p.next_recip);
        uint8_t *code_table = smem + C::kOffTable;
        if (C::kCodeTable) {
            // code_table[z] = Q(GELU(z) / next_scale) for every fp16 bit pattern z,
            // by the same functions the direct path uses; four patterns per step.
            // It depends on kernel parameters only, so it is built while the
            // previous kernel may still run, and while the first tile's MMAs do.
            for (int i = static_cast<int>(threadIdx.x) - 64; i < 16384; i += kEpiThreads) {
                const uint32_t z01 = static_cast<uint32_t>(4 * i) | (static_cast<uint32_t>(4 * i + 1) << 16);
                const uint32_t z23 = static_cast<uint32_t>(4 * i + 2) | (static_cast<uint32_t>(4 * i + 3) << 16);
                reinterpret_cast<uint32_t *>(code_table)[i] =
                    e4m3x4(gelu_fp16x2(z01, g_erf_table), gelu_fp16x2(z23, g_erf_table), p.next_lean != 0,
                           neg_scale2, recip2);
            }
            named_barrier_sync(1, kEpiThreads);
        }
        // A dynamic scale, and the buffers this grid writes, belong to the
        // previous kernel until it completes.
        griddepcontrol_wait();
        const float act_scale = p.act_scale_ptr ? *p.act_scale_ptr : p.act_scale;
        // Accumulator release goes to the leader's barriers (cluster addresses in a pair).
        const uint32_t acc_empty_base = kPair ? map_to_rank(bar_acc_empty, 0) : bar_acc_empty;
        uint8_t *staging = smem + C::kOffStaging + ew * C::kWarpStaging;
        const uint32_t staging_s = smem_u32(staging);
        int local = 0;
        const int row_limit = C::kSeg ? p.seg_rows : p.m;
        for (int t = tile_first; t < p.num_tiles; t += tile_step, ++local) {
            const auto rows = tile_rows(t, rank);
            const int seg = rows.x;
            const int m0 = rows.y;
            const int n0 = tile_coords(t).y * BN;
            const uint32_t a = local & 1;
            const uint32_t acc_ph = (local >> 1) & 1;
            // This warp's columns: lane i holds columns 2(i % 16) and 2(i % 16) + 1 of
            // sub slice + 4(i / 16) (combined scale act * w and the fp16 bias pair),
            // read before the accumulator wait.
            float2 my_cs = make_float2(0.0f, 0.0f);
            uint32_t my_b = 0u;
            {
                const int c = n0 + (slice + 4 * (lane >> 4)) * kSub + 2 * (lane & 15);
                if (c < p.n) {
                    if (C::kF16In) {
                        my_cs = make_float2(1.0f, 1.0f); // fp16 operands carry no scales
                    } else {
                        const float2 w = __ldg(reinterpret_cast<const float2 *>(p.w_scales + c));
                        my_cs = make_float2(act_scale * w.x, act_scale * w.y);
                    }
                    if (p.bias)
                        my_b = __ldg(reinterpret_cast<const uint32_t *>(p.bias + c));
                }
            }
            const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full + 8 * a, acc_ph, kSiteEpilogueAccFull));
            if (!ok)
                break;
            tc_fence_after();
            // Active subs are a prefix: sub k is tile sub slice + 4k, columns increase with k.
            int subs = 0;
            while (subs < 2 && slice + 4 * subs < C::kSubs && n0 + (slice + 4 * subs) * kSub < p.n)
                ++subs;
            const int row0 = m0 + quarter * 32;
            if (row0 >= row_limit)
                subs = 0; // every row of this warp is padding: nothing to load or store
            const uint32_t t_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
#pragma unroll 1
            for (int sub = 0; sub < subs; ++sub) {
                const int tsub = slice + 4 * sub;
                const int col0 = n0 + tsub * kSub;
                // The previous store from this warp's staging buffer has read it.
                if (lane == 0)
                    bulk_wait_group_read0();
                __syncwarp();
                // Two 16-column halves keep the live registers low.
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint32_t v[16];
                    tmem_ld_32x32b_x16(t_base + tsub * kSub + hf * 16, v);
                    tmem_wait_ld();
                    if (sub == subs - 1 && hf == 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            if (kPair)
                                mbar_arrive_cluster(acc_empty_base + 8 * a);
                            else
                                mbar_arrive(acc_empty_base + 8 * a);
                        }
                    }
                    // Scale, round to fp16, bias, GELU: two columns per packed op; the
                    // pair's scale and bias come from lane (column offset / 2).
                    uint32_t h[8];
                    uint4 pos_lo = make_uint4(0u, 0u, 0u, 0u), pos_hi = pos_lo;
                    if (C::kPos) {
                        // This lane's row of the positional table (padding rows read the
                        // last row; the store clips them).
                        const int prow = min(row0 + lane, row_limit - 1);
                        const uint16_t *pp = p.pos + static_cast<size_t>(prow) * p.pos_ld + col0 + hf * 16;
                        pos_lo = __ldg(reinterpret_cast<const uint4 *>(pp));
                        pos_hi = __ldg(reinterpret_cast<const uint4 *>(pp + 8));
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int src = sub * (kSub / 2) + hf * 8 + i;
                        const float2 cs = make_float2(__shfl_sync(0xffffffffu, my_cs.x, src),
                                                      __shfl_sync(0xffffffffu, my_cs.y, src));
                        const float2 acc = make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
                        uint32_t z;
                        if (C::kBiasF32) {
                            const uint32_t b2 = __shfl_sync(0xffffffffu, my_b, src);
                            const float2 y = make_float2(
                                fmaf(acc.x, cs.x, h2f(static_cast<uint16_t>(b2 & 0xFFFFu))),
                                fmaf(acc.y, cs.y, h2f(static_cast<uint16_t>(b2 >> 16))));
                            z = cvt_f16x2(y.x, y.y);
                        } else {
                            const float2 y = fmul2(acc, cs);
                            z = cvt_f16x2(y.x, y.y);
                            if (p.bias)
                                z = hadd2_rn(z, __shfl_sync(0xffffffffu, my_b, src));
                        }
                        if (C::kGelu && !C::kCodeTable)
                            z = gelu_fp16x2(z, erf_table);
                        if (C::kPos) {
                            const uint32_t pw = i < 4 ? (&pos_lo.x)[i] : (&pos_hi.x)[i - 4];
                            z = hadd2_rn(z, pw);
                        }
                        h[i] = z;
                    }
                    if (C::kY) {
                        // 32 rows x 64 B, 64B swizzle: 16B chunk j of row r at chunk j ^ ((r >> 1) & 3).
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) {
                            const uint32_t j = static_cast<uint32_t>(2 * hf + jj);
                            const uint32_t pos = j ^ ((static_cast<uint32_t>(lane) >> 1) & 3u);
                            *reinterpret_cast<uint4 *>(staging + lane * 64 + pos * 16) =
                                make_uint4(h[4 * jj], h[4 * jj + 1], h[4 * jj + 2], h[4 * jj + 3]);
                        }
                    }
                    if (C::kCodes) {
                        // 32 rows x 32 B, 32B swizzle: chunk j of row r at chunk j ^ ((r >> 2) & 1).
                        uint8_t *cbuf = staging + (C::kY ? C::kYBuf : 0);
                        uint32_t q[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            if (C::kCodeTable) {
                                // h holds pre-GELU fp16 pairs: one table byte per value.
                                const uint32_t c0 = code_table[h[2 * i] & 0xFFFFu];
                                const uint32_t c1 = code_table[h[2 * i] >> 16];
                                const uint32_t c2 = code_table[h[2 * i + 1] & 0xFFFFu];
                                const uint32_t c3 = code_table[h[2 * i + 1] >> 16];
                                q[i] = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
                            } else {
                                q[i] = e4m3x4(h[2 * i], h[2 * i + 1], p.next_lean != 0, neg_scale2, recip2);
                            }
                        }
                        const uint32_t pos = static_cast<uint32_t>(hf) ^ ((static_cast<uint32_t>(lane) >> 2) & 1u);
                        *reinterpret_cast<uint4 *>(cbuf + lane * 32 + pos * 16) = make_uint4(q[0], q[1], q[2], q[3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (C::kHeads) {
                        const int head_cols = 64 * p.heads;
                        tma_store_5d(&tm_y, staging_s, col0 % 64, row0, (col0 / 64) % p.heads, seg, col0 / head_cols);
                    } else if (C::kSeg) {
                        if (C::kY)
                            tma_store_3d(&tm_y, staging_s, col0, row0, seg);
                        if (C::kCodes)
                            tma_store_3d(&tm_c, staging_s + (C::kY ? C::kYBuf : 0), col0, row0, seg);
                    } else {
                        if (C::kY)
                            tma_store_2d(&tm_y, staging_s, col0, row0);
                        if (C::kCodes)
                            tma_store_2d(&tm_c, staging_s + (C::kY ? C::kYBuf : 0), col0, row0);
                    }
                    bulk_commit_group();
                }
            }
            if (subs == 0) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (kPair)
                        mbar_arrive_cluster(acc_empty_base + 8 * a);
                    else
                        mbar_arrive(acc_empty_base + 8 * a);
                }
            }
        }
        if (lane == 0)
            bulk_wait_group0();
    }

    tc_fence_before();
    __syncthreads();
    if (kPair)
        cluster_sync(); // neither CTA leaves while its peer may still touch its barriers or TMEM
    if (warp == 1) {
        tc_fence_after();
        if (kPair)
            tmem_dealloc_pair(tmem_base, C::kTmemCols);
        else
            tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

} // namespace gemm

// ---------------------------------------------------------------------------
// Skinny linear (decoder step, m <= 32) on tensor cores.
//
// Swap-AB: 128 weight rows are the MMA's M side and the (zero-padded) 32
// activation rows its N side, D[n, m] = sum_k W[n, k] x[m, k] in TMEM (32
// fp32 columns).  A cluster of S CTAs shares one 128-row block and splits K;
// partial sums meet in distributed shared memory, each CTA reduces 128/S rows
// in a fixed order (deterministic) and runs the epilogue for them.  Weights
// stream through a TMA ring; the kernel arms its weight loads before waiting
// on the previous grid (programmatic dependent launch), so back-to-back
// linears overlap their weight streaming with the previous kernel's tail.

namespace skinny {

constexpr int kThreads = 128;
constexpr int kRows = 128;  // weight rows per cluster (MMA M)
constexpr int kAct = 32;    // activation rows per MMA (MMA N); m <= 32
constexpr int kBK = 128;    // K bytes per stage
constexpr int kWBytes = kRows * kBK;
constexpr int kXBytes = kAct * kBK;
constexpr int kStageBytes = kWBytes + kXBytes;

// Split-K exchange buffer: row r of sender rank q lands at float offset
// (q * 128 / S + r % (128 / S)) * stride, its activation rows m contiguous;
// stride = 4 * ceil(m / 4) + 4 floats (16-byte rows, padded against bank
// conflicts).  Separate from the ring: peers may write it while this CTA still
// loads and multiplies.
__host__ __device__ constexpr int recv_stride(int m) { return (m + 3) / 4 * 4 + 4; }
__host__ __device__ constexpr int recv_bytes(int m) { return kRows * recv_stride(m) * 4; }

// Shared-memory ring of ST stages.  Two stages and small CTAs (four per SM)
// stream fastest when there are many CTAs (measured on B200: more independent
// weight streams per SM beat deeper rings); a deep ring is used when the grid
// is small and each CTA owns more K blocks than two stages hold, so that all
// of a CTA's weights are requested before it waits for the previous kernel.
// Five deep stages hold the decoder fc2's share (5120 -> 1280 over clusters of
// 8: five 16 KB tiles per CTA) at ~113 KB, small enough to become resident
// beside the previous links' CTAs (measured: 6 stages, 142 KB, made the C3
// step 3.6% slower).  The split-K exchange buffer (sized by m at launch)
// follows the barriers.
template <int ST>
struct Ring {
    static constexpr int kStages = ST;
    static constexpr int kOffX = ST * kWBytes;
    static constexpr int kRingBytes = kOffX + ST * kXBytes;
    static constexpr int kOffBar = kRingBytes;
    static constexpr int kOffRecv = kOffBar + 128;
    static constexpr int kSmemBase = kOffRecv + 1024; // + recv_bytes(m) when S > 1
    static_assert(kRingBytes % 1024 == 0, "swizzled stages stay 1024-byte aligned");
    static_assert((2 * ST + 3) * 8 <= 128, "barrier area");
};
constexpr int kShallow = 2;
constexpr int kDeep = 5;
static_assert(Ring<kShallow>::kSmemBase + recv_bytes(20) <= 56 * 1024, "four CTAs per SM at the decoder's m");
static_assert(Ring<kDeep>::kSmemBase + recv_bytes(kAct) <= 227 * 1024, "shared memory budget");
constexpr int kMaxCluster = 8;

enum : int { kKindE4M3 = 0, kKindF16 = 1 };

struct Params {
    int m, n, num_kb;
    int cluster; // CTAs per 128-row block (power of two, <= kMaxCluster)
    float act_scale;
    const float *act_scale_ptr;
    const float *w_scales; // nullptr: unit scales (fp16 weights)
    const uint16_t *bias;
    uint16_t *y;
    float next_scale, next_recip;
    uint8_t *next_codes;
    const uint8_t *w_packed; // non-null: weights in pre-swizzled 16 KB tiles (pack_kernel)
};

// Split-K sums over a cluster of S CTAs.  Each CTA finishes 128 / S of the
// 128 weight rows; a thread owns one of them (local index `r_local`) and the
// activation rows m = g + j*S (j < 32 / S) below m_count, where
// g = threadIdx.x / (128 / S).  The S partials of a row are added in rank
// order: slot q of `recv` holds CTA q's, and `own` this CTA's (rank `rank`).
template <int S>
__device__ __forceinline__ void sum_rows(const float *recv, const float *own, int rank, int stride, int r_local,
                                         int m_count, float (&acc)[kAct / 2])
{
    constexpr int kPer = kAct / S; // activation rows per thread
    constexpr int kRowsPer = kRows / S;
    const int g = static_cast<int>(threadIdx.x) / kRowsPer;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int m = g + j * S;
        float sum = 0.0f;
        if (m < m_count) {
#pragma unroll
            for (int q = 0; q < S; ++q)
                sum += (q == rank ? own : recv + q * kRowsPer * stride)[r_local * stride + m];
        }
        acc[j] = sum;
    }
}

template <int KIND, int EPI, int ST>
__global__ void __launch_bounds__(kThreads)
    skinny_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, const Params p)
{
    constexpr int kStages = Ring<ST>::kStages;
    constexpr int kOffX = Ring<ST>::kOffX;
    constexpr int kOffBar = Ring<ST>::kOffBar;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int S = p.cluster;
    const int rank = static_cast<int>(blockIdx.x) % S;
    const int n0 = (static_cast<int>(blockIdx.x) / S) * kRows;
    const int kb_begin = static_cast<int>((static_cast<int64_t>(p.num_kb) * rank) / S);
    const int kb_end = static_cast<int>((static_cast<int64_t>(p.num_kb) * (rank + 1)) / S);
    const int nkb = kb_end - kb_begin;
    const uint32_t bar_full = sbase + kOffBar;
    const uint32_t bar_empty = bar_full + 8 * kStages;
    const uint32_t bar_acc = bar_empty + 8 * kStages;
    const uint32_t bar_recv = bar_acc + 8; // split-K partials from the peers have landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8 * (2 * kStages + 2));
    const uint32_t recv = sbase + Ring<ST>::kOffRecv;
    const int stride = recv_stride(p.m);
    const int nvec = (p.m + 3) / 4; // 16-byte pieces of a row's partials

    if (threadIdx.x == 0) {
        griddepcontrol_launch_dependents();
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_acc, 1);
        mbar_init(bar_recv, 1);
        // The one local arrival, and the bytes the S - 1 peers will send.
        if (S > 1)
            mbar_arrive_expect_tx(bar_recv, static_cast<uint32_t>((S - 1) * (kRows / S) * stride * 4));
        fence_barrier_init();
        prefetch_tensor_map(&tm_w);
        prefetch_tensor_map(&tm_x);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Peers may send partials into this CTA once every CTA of the cluster has
    // initialised its barriers: arrive now, wait just before the first send.
    if (S > 1)
        cluster_arrive();

    // The output row this thread finishes (its own TMEM lane when S == 1, else
    // row `threadIdx.x % (128 / S)` of this CTA's share of the reduction) and
    // that row's weight scale and bias: constants of the layer, so they are
    // read before waiting for the previous kernel.
    const int my_row = S == 1 ? static_cast<int>(threadIdx.x)
                              : rank * (kRows / S) + static_cast<int>(threadIdx.x) % (kRows / S);
    const int my_n = n0 + my_row;
    float my_ws = 1.0f;
    uint16_t my_bias = 0;
    if (my_n < p.n) {
        if (p.w_scales)
            my_ws = __ldg(p.w_scales + my_n);
        if (p.bias)
            my_bias = __ldg(p.bias + my_n);
    }

    if (warp == 0 && lane == 0) {
        // Weights do not depend on the previous kernel: arm the first stages now.
        // Packed weights: tile (row block, k block) is one contiguous 16 KB image.
        const uint8_t *tiles =
            p.w_packed ? p.w_packed + (static_cast<size_t>(n0 / kRows) * p.num_kb) * kWBytes : nullptr;
        auto load_w = [&](int s, int kb) {
            if (p.w_packed)
                bulk_load(sbase + s * kWBytes, tiles + static_cast<size_t>(kb) * kWBytes, kWBytes, bar_full + 8 * s);
            else
                tma_load_2d(sbase + s * kWBytes, &tm_w, bar_full + 8 * s, kb * kBK / (KIND == kKindF16 ? 2 : 1), n0);
        };
        const int first = nkb < kStages ? nkb : kStages;
        for (int i = 0; i < first; ++i) {
            mbar_arrive_expect_tx(bar_full + 8 * i, kStageBytes);
            load_w(i, kb_begin + i);
        }
        griddepcontrol_wait();
        for (int i = 0; i < first; ++i)
            tma_load_2d(sbase + kOffX + i * kXBytes, &tm_x, bar_full + 8 * i, (kb_begin + i) * kBK / (KIND == kKindF16 ? 2 : 1), 0);
        for (int j = first; j < nkb; ++j) {
            const int s = j % kStages;
            const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
            if (!mbar_wait(bar_empty + 8 * s, ph ^ 1u, kSiteProducerEmpty))
                break;
            const int xk = (kb_begin + j) * kBK / (KIND == kKindF16 ? 2 : 1);
            mbar_arrive_expect_tx(bar_full + 8 * s, kStageBytes);
            load_w(s, kb_begin + j);
            tma_load_2d(sbase + kOffX + s * kXBytes, &tm_x, bar_full + 8 * s, xk, 0);
        }
        // Drain: every issued load lands before shared memory is released.
        for (int j = (nkb > kStages ? nkb - kStages : 0); j < nkb; ++j) {
            const uint32_t par = static_cast<uint32_t>(j / kStages) & 1u;
            for (int tries = 0; tries < (1 << 22) && !mbar_try_wait(bar_full + 8 * (j % kStages), par); ++tries) {
            }
        }
    } else {
        // Outputs of this grid may be inputs of the previous one: no global
        // access before that grid is complete.
        griddepcontrol_wait();
    }
    if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = KIND == kKindF16 ? idesc_f16_f32<kRows, kAct>() : idesc_e4m3_f32<kRows, kAct>();
        bool ok = true;
        for (int j = 0; ok && j < nkb; ++j) {
            const int s = j % kStages;
            const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
            if (!mbar_wait(bar_full + 8 * s, ph, kSiteMmaFull)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k) {
                const uint64_t da = smem_desc_k_sw128(sbase + s * kWBytes + k * 32);
                const uint64_t db = smem_desc_k_sw128(sbase + kOffX + s * kXBytes + k * 32);
                if (KIND == kKindF16)
                    mma_f16(tmem_base, da, db, idesc, (j | k) != 0);
                else
                    mma_f8f6f4(tmem_base, da, db, idesc, (j | k) != 0);
            }
            mma_commit(bar_empty + 8 * s);
        }
        mma_commit(bar_acc);
    }

    // Read the accumulator: thread (warp w, lane) holds weight row 32w + lane,
    // one fp32 per activation row.
    const float act_scale = p.act_scale_ptr ? *p.act_scale_ptr : p.act_scale;
    uint32_t v[kAct];
    const bool ok = nkb == 0 || __all_sync(0xffffffffu, mbar_wait(bar_acc, 0, kSiteEpilogueAccFull));
    if (nkb > 0 && ok) {
        tc_fence_after();
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(warp * 32) << 16), v);
        tmem_wait_ld();
    } else {
#pragma unroll
        for (int i = 0; i < kAct; ++i)
            v[i] = 0u; // this CTA's K slice is empty
    }
    const float cs = p.w_scales ? act_scale * my_ws : 1.0f;
    const uint64_t neg_scale2 = f2_bits(-p.next_scale, -p.next_scale);
    const uint64_t recip2 = f2_bits(p.next_recip, p.next_recip);
    // The epilogue of C values acc[j] (activation row rows(j)): scale, round to
    // fp16, bias, then GELU on pairs -- every table lookup is issued before any
    // store, so the lookups share one memory round trip -- then the stores.
    auto finish = [&](const auto &acc, auto rows, auto count) {
        constexpr int C = decltype(count)::value;
        uint32_t z[C];
#pragma unroll
        for (int j = 0; j < C; ++j) {
            z[j] = f2h_rn(acc[j] * cs);
            if (p.bias)
                z[j] = hadd_rn(static_cast<uint16_t>(z[j]), my_bias);
        }
        if (EPI & 1) {
#pragma unroll
            for (int j = 0; j < C; j += 2) {
                const uint32_t g = gemm::gelu_fp16x2(z[j] | (z[j + 1] << 16), g_erf_table);
                z[j] = g & 0xFFFFu;
                z[j + 1] = g >> 16;
            }
        }
#pragma unroll
        for (int j = 0; j < C; ++j) {
            const int m = rows(j);
            if (m < p.m) {
                const size_t o = static_cast<size_t>(m) * p.n + my_n;
                if (p.y)
                    p.y[o] = static_cast<uint16_t>(z[j]);
                if (p.next_codes)
                    p.next_codes[o] = static_cast<uint8_t>(e4m3x2_quotient(z[j], neg_scale2, recip2) & 0xFFu);
            }
        }
    };
    if (S == 1) {
        if (my_n < p.n) {
            float acc[kAct];
#pragma unroll
            for (int m = 0; m < kAct; ++m)
                acc[m] = __uint_as_float(v[m]);
            finish(acc, [](int j) { return j; }, std::integral_constant<int, kAct>{});
        }
    } else {
        // Split-K exchange.  Each thread stages its row (TMEM lane threadIdx.x)
        // in the ring, idle now that every MMA has completed: row R at float
        // offset R * stride, so the rows a peer finishes form one contiguous run.
        // Lane 0 of each warp then copies the warp's 32 rows, one bulk copy per
        // owner (two when S = 8), into slot `rank` of the owner's receive buffer;
        // each copy completes its bytes on the owner's bar_recv (a few barrier
        // updates instead of one per 16 bytes, and no CTA-wide barrier first).
        const int rows_per = kRows / S;
#pragma unroll
        for (int i = 0; i < kAct / 4; ++i)
            if (i < nvec)
                st_shared_v4(sbase + static_cast<uint32_t>((threadIdx.x * stride + 4 * i) * 4),
                             make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
        fence_proxy_async_smem(); // the bulk copies (async proxy) read these stores
        cluster_wait();           // every peer's bar_recv is initialised
        __syncwarp();
        if (lane == 0) {
            const int r0 = warp * 32;
            const int span = rows_per < 32 ? rows_per : 32;
            for (int r = r0; r < r0 + 32; r += span) {
                const int q = r / rows_per;
                if (q != rank) {
                    const uint32_t dst = recv + static_cast<uint32_t>(((rank * rows_per + r % rows_per) * stride) * 4);
                    bulk_copy_to_peer(map_to_rank(dst, static_cast<uint32_t>(q)),
                                      sbase + static_cast<uint32_t>(r * stride * 4),
                                      static_cast<uint32_t>(span * stride * 4),
                                      map_to_rank(bar_recv, static_cast<uint32_t>(q)));
                }
            }
        }
        // A bounded wait that gives up sets the error word; the sums still run.
        mbar_wait_cluster(bar_recv, 0, kSiteClusterExchange);
        __syncthreads(); // this CTA's own staged rows, written by other warps
        // This CTA has everything it was sent: arrive on the exit barrier, which
        // keeps every CTA's staged runs (the copies' sources) alive until all
        // peers have received theirs.  Every copy into a CTA has completed
        // before it arrives, so the arrival orders nothing: relaxed.
        cluster_arrive_relaxed();
        const float *rbuf = reinterpret_cast<const float *>(smem + Ring<ST>::kOffRecv);
        const float *own = reinterpret_cast<const float *>(smem) + rank * rows_per * stride;
        const int r_local = static_cast<int>(threadIdx.x) % rows_per;
        float acc[kAct / 2];
        if (my_n < p.n) {
            switch (S) {
            case 2: sum_rows<2>(rbuf, own, rank, stride, r_local, p.m, acc); break;
            case 4: sum_rows<4>(rbuf, own, rank, stride, r_local, p.m, acc); break;
            default: sum_rows<8>(rbuf, own, rank, stride, r_local, p.m, acc); break;
            }
            const int g = static_cast<int>(threadIdx.x) / rows_per;
            switch (S) {
            case 2: finish(acc, [g](int j) { return g + 2 * j; }, std::integral_constant<int, kAct / 2>{}); break;
            case 4: finish(acc, [g](int j) { return g + 4 * j; }, std::integral_constant<int, kAct / 4>{}); break;
            default: finish(acc, [g](int j) { return g + 8 * j; }, std::integral_constant<int, kAct / 8>{}); break;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 32);
    }
    if (S > 1)
        cluster_wait();
}

// Re-lays a row-major [n, row_bytes] weight as 16 KB tiles: tile (rb, kb)
// holds rows [128 rb, 128 rb + 128) x bytes [128 kb, 128 kb + 128), each row's
// 16-byte chunk c stored at chunk c ^ (row & 7) -- exactly the shared-memory
// image a 128B-swizzled TMA load of that box produces.  Out-of-range rows and
// bytes are zero.  One thread per 16-byte chunk.
__global__ void __launch_bounds__(256)
    pack_kernel(const uint8_t *__restrict__ w, int64_t n, int64_t row_bytes, int64_t num_kb,
                uint8_t *__restrict__ packed)
{
    const int64_t chunk = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    const int64_t tiles = (n + kRows - 1) / kRows * num_kb;
    if (chunk >= tiles * (kWBytes / 16))
        return;
    const int64_t tile = chunk / (kWBytes / 16);
    const int within = static_cast<int>(chunk % (kWBytes / 16));
    const int r = within / 8, c = within % 8;
    const int64_t row = (tile / num_kb) * kRows + r;
    const int64_t col = (tile % num_kb) * kBK + c * 16;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < n && col < row_bytes)
        v = *reinterpret_cast<const uint4 *>(w + row * row_bytes + col);
    *reinterpret_cast<uint4 *>(packed + tile * kWBytes + r * 128 + ((c ^ (r & 7)) * 16)) = v;
}

} // namespace skinny

// ---------------------------------------------------------------------------
// Chain of small-M linears in one persistent launch (a decoder step's linears).
// The per-launch skinny kernel pays, for every dependent linear, the grid's exit
// and the next grid's release; here clusters of kCS CTAs stay resident and walk
// the links in order.  Each cluster takes the 128-row blocks b = cluster,
// cluster + clusters, ... of a link, splits K over its CTAs and reduces the
// partials through DSMEM as the skinny kernel does.  When a cluster has finished
// its blocks of link i, its leader adds their count to done[i] (release, after
// a cluster barrier that orders every rank's stores); a link's activations are
// loaded only after done[i - 1] reaches the previous link's block count
// (acquire), so each link sees all of its predecessor's outputs and no link
// overwrites a buffer an earlier link still reads.  The next unit's weight tiles
// are requested before that wait.  Every wait is bounded.

namespace chain {

// Persistent chain of small-m linears.  One CTA per SM owns a fixed list of
// units in chain order; a unit is one 128-row block of one link's weights over
// a K slice of at most kMaxUnitKb 16 KB tiles.  Each role walks the same list:
//   warp 0: loads a unit's weight tiles as soon as the previous unit's MMAs
//           are done -- normally a layer before the unit's activations exist;
//   warp 1: loads a unit's activations once every row block of the previous
//           link is complete (a release/acquire counter per link);
//   warp 2: issues the unit's MMAs into one of two TMEM accumulators;
//   warps 3-6: epilogue.  An unsplit unit finishes its rows directly; the K
//           slices of a split unit write fp32 partials and the last slice to
//           arrive (an atomic counter per row block) sums them in slice order.
// Each buffer is one unit long and each handoff is one mbarrier phase per unit
// (a completed-phase wait still costs ~100 cycles, so per-tile barriers would
// dominate a unit's critical path).  Nothing waits on another CTA except
// through the link counters, so the only requirement is that all CTAs are
// resident (one per SM).
using skinny::kAct;
using skinny::kBK;
using skinny::kRows;
using skinny::kWBytes;
using skinny::kXBytes;
constexpr int kMaxUnitKb = 10; // 160 KB of weights per unit
constexpr int kEpiWarp0 = 3;
constexpr int kEpiThreads = 128;
constexpr int kThreads = 32 * kEpiWarp0 + kEpiThreads;
constexpr int kOffX = kMaxUnitKb * kWBytes;
constexpr int kOffBar = kOffX + kMaxUnitKb * kXBytes;
constexpr int kBars = 9; // w_full, x_full[2] (the unit's two halves), acc_full[2], acc_empty[2], drain
constexpr int kSmemBytes = kOffBar + 128 + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");
// Distinct activation tensor maps passed as kernel parameters (TMA reads a
// parameter-space descriptor without a global fetch per load); chains with
// more distinct activation buffers keep them in global memory.
constexpr int kParamMaps = 48;

struct Link {
    const uint8_t *w; // packed 16 KB tiles (lffw_pack_skinny_weights)
    const float *w_scales;
    const uint16_t *bias;
    const float *act_scale_ptr;
    uint16_t *y;
    uint8_t *codes;
    float *partials;        // split links: [blocks][split][kAct][kRows] fp32
    unsigned int *arrivals; // split links: K slices finished, per row block
    int n, num_kb, split, slice_kb, gelu, map; // map: index of the link's activation tensor map
    float act_scale, next_scale, next_recip, pad1;
};

struct Unit {
    int link, block, k0, k1;
};

struct Params {
    CUtensorMap maps[kParamMaps]; // activation codes [m, k], 128-byte x 32-row boxes, SW128
    const CUtensorMap *global_maps; // used instead when non-null
    const Link *links;
    const Unit *units;         // CTA c's units are units[first[c] .. first[c + 1])
    const int *first;
    unsigned int *done; // per link: row blocks finished
    int m;
};

__device__ __forceinline__ unsigned int blocks_of(const Link &l) { return (l.n + kRows - 1) / kRows; }

__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ Params p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t w_full = sbase + kOffBar;
    const uint32_t x_full = w_full + 8; // [2]: K blocks [0, h) and [h, nkb), h = (nkb + 1) / 2
    const uint32_t acc_full = x_full + 16;
    const uint32_t acc_empty = acc_full + 16;
    const uint32_t drain = acc_empty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8 * kBars);
    volatile int *last_flag = reinterpret_cast<volatile int *>(smem + kOffBar + 8 * kBars + 4);
    const int u_begin = p.first[blockIdx.x];
    const int u_end = p.first[blockIdx.x + 1];

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        mbar_init(x_full, 1);
        mbar_init(x_full + 8, 1);
        for (int a = 0; a < 2; ++a) {
            mbar_init(acc_full + 8 * a, 1);
            mbar_init(acc_empty + 8 * a, kEpiThreads / 32);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(smem_u32(tmem_slot), 2 * kAct);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // The previous unit's MMAs are complete (its buffers are free): acc_full
    // of unit local - 1, waited on by the producers as well as the epilogue.
    auto previous_done = [&](int local) {
        return local == 0 || mbar_wait(acc_full + 8 * ((local - 1) & 1), ((local - 1) >> 1) & 1u, kSiteProducerEmpty);
    };

    if (warp == 0) {
        // ---------------- weight producer ----------------
        if (lane == 0) {
            int issued = 0; // units whose loads were issued
            for (int i = u_begin, local = 0; i < u_end; ++i, ++local) {
                if (!previous_done(local))
                    break;
                const Unit un = p.units[i];
                const uint8_t *tiles = p.links[un.link].w + static_cast<size_t>(un.block) * p.links[un.link].num_kb * kWBytes;
                mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(un.k1 - un.k0) * kWBytes);
                for (int kb = un.k0; kb < un.k1; ++kb)
                    bulk_load(sbase + (kb - un.k0) * kWBytes, tiles + static_cast<size_t>(kb) * kWBytes, kWBytes, w_full);
                issued = local + 1;
            }
            // A load still in flight (only after an abandoned wait) lands before exit.
            if (issued > 0)
                for (int t = 0; t < (1 << 20) && !mbar_try_wait(w_full, (issued - 1) & 1u); ++t) {
                }
        }
    } else if (warp == 1) {
        // ---------------- activation producer ----------------
        if (lane == 0) {
            int issued = 0;
            int ready = 0; // links [0, ready) are complete
            for (int i = u_begin, local = 0; i < u_end; ++i, ++local) {
                const Unit un = p.units[i];
                const int mi = p.links[un.link].map;
                const CUtensorMap *map = p.global_maps ? p.global_maps + mi : &p.maps[mi];
                prefetch_tensor_map(map);
                if (!previous_done(local))
                    break;
                if (un.link > ready) {
                    const unsigned int need = blocks_of(p.links[un.link - 1]);
                    const uint64_t start = global_timer_ns();
                    bool ok = true;
                    for (uint32_t spin = 0; ld_acquire_gpu(p.done + un.link - 1) < need; ++spin)
                        if ((spin & 63u) == 63u &&
                            (device_error_raised() || global_timer_ns() - start > 2000000000ull)) {
                            atomicCAS(&g_device_error, 0, kSiteChainDependency);
                            ok = false;
                            break;
                        }
                    if (!ok)
                        break;
                    // The previous links' outputs were written by generic stores; TMA reads them.
                    fence_proxy_async_global();
                    ready = un.link;
                }
                // Two halves, so that the MMAs start while the second half lands.
                const int nkb = un.k1 - un.k0, h = (nkb + 1) / 2;
                mbar_arrive_expect_tx(x_full, static_cast<uint32_t>(h) * kXBytes);
                mbar_arrive_expect_tx(x_full + 8, static_cast<uint32_t>(nkb - h) * kXBytes);
                for (int j = 0; j < nkb; ++j)
                    tma_load_2d(sbase + kOffX + j * kXBytes, map, x_full + (j < h ? 0 : 8), (un.k0 + j) * kBK, 0);
                issued = local + 1;
            }
            for (int half = 0; issued > 0 && half < 2; ++half)
                for (int t = 0; t < (1 << 20) && !mbar_try_wait(x_full + 8 * half, (issued - 1) & 1u); ++t) {
                }
        }
    } else if (warp == 2) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_e4m3_f32<kRows, kAct>();
            for (int i = u_begin, local = 0; i < u_end; ++i, ++local) {
                const Unit un = p.units[i];
                const uint32_t a = local & 1;
                if (!mbar_wait(acc_empty + 8 * a, ((local >> 1) & 1u) ^ 1u, kSiteMmaAccEmpty) ||
                    !mbar_wait(w_full, local & 1u, kSiteMmaFull))
                    break;
                const uint32_t d = tmem_base + a * kAct;
                const int nkb = un.k1 - un.k0, h = (nkb + 1) / 2;
                bool ok = true;
                for (int half = 0; ok && half < 2; ++half) {
                    if (!mbar_wait(x_full + 8 * half, local & 1u, kSiteMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kb = half ? h : 0; kb < (half ? nkb : h); ++kb)
#pragma unroll
                        for (int k = 0; k < kBK / 32; ++k)
                            mma_f8f6f4(d, smem_desc_k_sw128(sbase + kb * kWBytes + k * 32),
                                       smem_desc_k_sw128(sbase + kOffX + kb * kXBytes + k * 32), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                }
                if (!ok)
                    break;
                mma_commit(acc_full + 8 * a);
            }
            // Every MMA of this thread completes before TMEM is freed.
            mma_commit(drain);
            for (int tries = 0; tries < (1 << 22) && !mbar_try_wait(drain, 0); ++tries) {
            }
        }
    } else {
        // ---------------- epilogue: 4 warps, one accumulator row per thread ----------------
        // Every epilogue thread walks all units, even after a wait has given up
        // (waits then return at once), so the named barriers always match.
        const int et = static_cast<int>(threadIdx.x) - 32 * kEpiWarp0;
        const int row = 32 * (warp & 3) + lane; // TMEM lane = weight row in the block
        for (int i = u_begin, local = 0; i < u_end; ++i, ++local) {
            const Unit un = p.units[i];
            const Link l = p.links[un.link]; // a copy: the stores below cannot alias it
            const int n = un.block * kRows + row;
            float ws = 0.0f;
            uint16_t bias = 0;
            if (n < l.n) {
                ws = __ldg(l.w_scales + n);
                if (l.bias)
                    bias = __ldg(l.bias + n);
            }
            const uint32_t a = local & 1;
            bool ok = true;
            if (lane == 0)
                ok = mbar_wait(acc_full + 8 * a, (local >> 1) & 1u, kSiteEpilogueAccFull);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            tc_fence_after();
            uint32_t v[kAct];
            tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + a * kAct, v);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(acc_empty + 8 * a);
            float acc[kAct];
#pragma unroll
            for (int m = 0; m < kAct; ++m)
                acc[m] = ok ? __uint_as_float(v[m]) : 0.0f;
            bool finish = true;
            if (l.split > 1) {
                const int slice = un.k0 / l.slice_kb;
                float *mine = l.partials + (static_cast<size_t>(un.block) * l.split + slice) * (kAct * kRows);
#pragma unroll
                for (int m = 0; m < kAct; ++m)
                    if (m < p.m)
                        mine[m * kRows + row] = acc[m];
                __threadfence();
                named_barrier_sync(1, kEpiThreads);
                if (et == 0)
                    *last_flag = static_cast<int>(atomicAdd(l.arrivals + un.block, 1u));
                named_barrier_sync(1, kEpiThreads);
                finish = *last_flag == l.split - 1;
                if (finish) {
                    // The other slices' partials are visible: each was fenced before its arrival.
                    __threadfence();
                    // Sum in slice order; the loads of up to four slices are in flight together.
                    const float *all = l.partials + static_cast<size_t>(un.block) * l.split * (kAct * kRows) + row;
#pragma unroll
                    for (int m = 0; m < kAct; ++m)
                        acc[m] = 0.0f;
                    for (int q0 = 0; q0 < l.split; q0 += 4) {
                        float t[4][kAct];
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int m = 0; m < kAct; ++m)
                                t[j][m] = q0 + j < l.split && m < p.m
                                              ? __ldcg(all + (static_cast<size_t>(q0 + j) * kAct + m) * kRows)
                                              : 0.0f;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (q0 + j < l.split)
#pragma unroll
                                for (int m = 0; m < kAct; ++m)
                                    acc[m] += t[j][m];
                    }
                }
            }
            if (finish) {
                const float act_scale = l.act_scale_ptr ? *l.act_scale_ptr : l.act_scale;
                const float cs = act_scale * ws;
                const uint64_t neg_scale2 = f2_bits(-l.next_scale, -l.next_scale);
                const uint64_t recip2 = f2_bits(l.next_recip, l.next_recip);
                if (n < l.n) {
                    // Rows in pairs, every row's chain independent (fully unrolled,
                    // predicated): the GELU table reads of all rows overlap.
#pragma unroll
                    for (int m = 0; m < kAct; m += 2) {
                        if (m < p.m) {
                            uint32_t z = f2h_rn(acc[m] * cs) | (static_cast<uint32_t>(f2h_rn(acc[m + 1] * cs)) << 16);
                            if (l.bias)
                                z = gemm::hadd2_rn(z, static_cast<uint32_t>(bias) * 0x10001u);
                            if (l.gelu)
                                z = gemm::gelu_fp16x2(z, g_erf_table);
                            const size_t o = static_cast<size_t>(m) * l.n + n;
                            const bool second = m + 1 < p.m;
                            if (l.y) {
                                l.y[o] = static_cast<uint16_t>(z & 0xFFFFu);
                                if (second)
                                    l.y[o + l.n] = static_cast<uint16_t>(z >> 16);
                            }
                            if (l.codes) {
                                const uint32_t q2 = e4m3x2_quotient(z, neg_scale2, recip2);
                                l.codes[o] = static_cast<uint8_t>(q2 & 0xFFu);
                                if (second)
                                    l.codes[o + l.n] = static_cast<uint8_t>((q2 >> 8) & 0xFFu);
                            }
                        }
                    }
                }
                // Later links read these codes with TMA: the reader orders its
                // async-proxy loads after its acquire with a proxy fence.
                named_barrier_sync(1, kEpiThreads);
                if (et == 0) {
                    fence_gpu();
                    red_release_gpu_add(p.done + un.link, 1u);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * kAct);
    }
}

} // namespace chain

// ---------------------------------------------------------------------------
// Quantize / scale kernels.

namespace quant {

constexpr int kThreads = 256;



// A warp converts 1024 halves per iteration: four coalesced 512-byte loads
// per lane group (16 bytes per lane each), four coalesced 256-byte stores,
// streaming cache hints (the activations are read once).  The next chunk's
// loads are issued before the current chunk is converted, so each warp keeps
// 4 KB in flight while its arithmetic runs.
constexpr int64_t kQuantChunk = 1024;

__device__ __forceinline__ void load_chunk(uint4 (&h)[4], const uint16_t *x, int64_t c, int lane)
{
    const uint16_t *src = x + c * kQuantChunk + lane * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        h[i] = ld_stream16(src + 256 * i);
}

__global__ void __launch_bounds__(kThreads)
    quantize_kernel(const uint16_t *__restrict__ x, int64_t count, float scale_value, float recip_value,
                    const float *scale_ptr, uint8_t *__restrict__ codes)
{
    // Programmatic dependent launch: the next kernel may start its prologue
    // now; this one waits for the previous kernel before reading its output.
    if (threadIdx.x == 0)
        griddepcontrol_launch_dependents();
    griddepcontrol_wait();
    const float scale = scale_ptr ? *scale_ptr : scale_value;
    const float recip = scale_ptr ? __frcp_rn(scale) : recip_value;
    const bool lean = lean_scale(scale);
    const uint64_t neg_scale2 = f2_bits(-scale, -scale), recip2 = f2_bits(recip, recip);
    const int lane = threadIdx.x % 32;
    const int64_t chunks = count / kQuantChunk;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
    int64_t c = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + threadIdx.x / 32;
    uint4 cur[4], next[4];
    if (c < chunks)
        load_chunk(cur, x, c, lane);
    for (; c < chunks; c += warps) {
        if (c + warps < chunks)
            load_chunk(next, x, c + warps, lane);
        uint8_t *dst = codes + c * kQuantChunk + lane * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = e4m3x4(cur[i].x, cur[i].y, lean, neg_scale2, recip2);
            const uint32_t hi = e4m3x4(cur[i].z, cur[i].w, lean, neg_scale2, recip2);
            asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(dst + 256 * i), "r"(lo), "r"(hi) : "memory");
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
            cur[i] = next[i];
    }
    // Tail (count % 1024), handled by block 0.
    if (blockIdx.x == 0)
        for (int64_t i = chunks * kQuantChunk + threadIdx.x; i < count; i += kThreads)
            codes[i] = static_cast<uint8_t>(e4m3x2(q_quotient(x[i], scale), 0.0f) & 0xFF);
}

// codes[r, :] = Q(w[r, :] / scales[r]); grid.x = row, grid.y strides the row.
__global__ void __launch_bounds__(kThreads)
    quantize_rows_kernel(const uint16_t *__restrict__ w, int64_t cols, const float *__restrict__ scales,
                         uint8_t *__restrict__ codes)
{
    const int64_t r = blockIdx.x;
    const float scale = scales[r];
    const uint16_t *src = w + r * cols;
    uint8_t *dst = codes + r * cols;
    for (int64_t c = static_cast<int64_t>(blockIdx.y) * kThreads + threadIdx.x; c < cols;
         c += static_cast<int64_t>(gridDim.y) * kThreads)
        dst[c] = static_cast<uint8_t>(e4m3x2(q_quotient(src[c], scale), 0.0f) & 0xFF);
}

__device__ __forceinline__ float block_max(float v)
{
    __shared__ float partial[kThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off /= 2)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (threadIdx.x % 32 == 0)
        partial[threadIdx.x / 32] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < kThreads / 32 ? partial[threadIdx.x] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off /= 2)
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    }
    return v;
}

// One block per weight row: scale = max|w| / 448 (IEEE division), <= 0 -> 1.
__global__ void __launch_bounds__(kThreads)
    weight_scales_kernel(const uint16_t *__restrict__ w, int64_t cols, float *__restrict__ scales)
{
    const uint16_t *row = w + static_cast<int64_t>(blockIdx.x) * cols;
    float best = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads)
        best = fmaxf(best, fabsf(h2f(row[c]))); // fmaxf drops NaN
    best = block_max(best);
    if (threadIdx.x == 0) {
        const float s = __fdiv_rn(best, 448.0f);
        scales[blockIdx.x] = s > 0.0f ? s : 1.0f;
    }
}

// amax over the whole tensor into *bits (non-negative float bit patterns order as ints).
__global__ void __launch_bounds__(kThreads)
    amax_kernel(const uint16_t *__restrict__ x, int64_t count, int *bits)
{
    float best = 0.0f;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < count; i += stride)
        best = fmaxf(best, fabsf(h2f(x[i])));
    best = block_max(best);
    if (threadIdx.x == 0)
        atomicMax(bits, __float_as_int(best));
}

__global__ void finalize_scale_kernel(float *scale, float *amax_out)
{
    const float amax = *scale; // holds the amax bits written by amax_kernel
    if (amax_out)
        *amax_out = amax;
    *scale = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
}

} // namespace quant

// ---------------------------------------------------------------------------
// LayerNorm producer (cpp/src/network_graph.cpp:160-166, with the residual add
// of :285-287): the fp16 residual sum, the fp16 LayerNorm output and/or its E4M3
// codes for the next linear, in one pass over the row.

namespace norm {

constexpr int kThreads = 256; // one row per warp
constexpr int kRowsPerBlock = kThreads / 32;

struct Params {
    int rows, cols;
    const uint16_t *x, *residual;
    uint16_t *sum_out;
    const float *gamma, *beta;
    float eps;
    uint16_t *y;
    float code_scale, code_recip;
    const float *code_scale_ptr;
    uint8_t *codes;
};

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off /= 2)
        v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// KV: 16-byte vectors (8 halves) per lane; the row (cols / 8 vectors) is spread
// over the lanes, vector v on lane v % 32, held in registers between passes.
// Warps loop over rows (grid-stride).  gamma and beta are staged once per block
// in shared memory (dynamic, 8 bytes per column): every row reads them again.
// kCodesOnly: x in (no residual), E4M3 codes out only (no sum, no fp16 y), the
// form that follows a GEMM epilogue which already added the residual.

template <int KV, bool kCodesOnly>
__global__ void __launch_bounds__(kThreads, KV <= 5 ? 4 : 1) layer_norm_kernel(const Params p)
{
    extern __shared__ __align__(16) float gb_s[]; // gamma [cols], beta [cols]
    if (threadIdx.x == 0)
        griddepcontrol_launch_dependents();
    for (int i = threadIdx.x; i < p.cols / 4; i += kThreads) { // layer constants: before the wait
        reinterpret_cast<float4 *>(gb_s)[i] = __ldg(reinterpret_cast<const float4 *>(p.gamma) + i);
        reinterpret_cast<float4 *>(gb_s + p.cols)[i] = __ldg(reinterpret_cast<const float4 *>(p.beta) + i);
    }
    __syncthreads();
    griddepcontrol_wait();
    const float *gamma_s = gb_s, *beta_s = gb_s + p.cols;
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int vecs = p.cols / 8;
    const int stride = static_cast<int>(gridDim.x) * kRowsPerBlock;
    for (int row = blockIdx.x * kRowsPerBlock + warp; row < p.rows; row += stride) {
    const size_t base = static_cast<size_t>(row) * p.cols;
    uint4 v[KV];
#pragma unroll
    for (int j = 0; j < KV; ++j) {
        const int c = lane + 32 * j;
        v[j] = make_uint4(0u, 0u, 0u, 0u);
        if (c < vecs) {
            v[j] = ld_stream16(p.x + base + 8 * c);
            if (!kCodesOnly && p.residual) {
                const uint4 r = ld_stream16(p.residual + base + 8 * c);
                v[j] = make_uint4(gemm::hadd2_rn(v[j].x, r.x), gemm::hadd2_rn(v[j].y, r.y),
                                  gemm::hadd2_rn(v[j].z, r.z), gemm::hadd2_rn(v[j].w, r.w));
            }
            if (!kCodesOnly && p.sum_out)
                *reinterpret_cast<uint4 *>(p.sum_out + base + 8 * c) = v[j];
        }
    }
    // Two-pass statistics in fp32 over the row held in registers.
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < KV; ++j) {
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            acc += h2f(static_cast<uint16_t>(w[i] & 0xFFFFu)) + h2f(static_cast<uint16_t>(w[i] >> 16));
    }
    const float inv_cols = 1.0f / static_cast<float>(p.cols);
    const float mean = warp_sum(acc) * inv_cols;
    acc = 0.0f;
#pragma unroll
    for (int j = 0; j < KV; ++j) {
        if (lane + 32 * j < vecs) {
            const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float d0 = h2f(static_cast<uint16_t>(w[i] & 0xFFFFu)) - mean;
                const float d1 = h2f(static_cast<uint16_t>(w[i] >> 16)) - mean;
                acc += d0 * d0 + d1 * d1;
            }
        }
    }
    const float rstd = __frsqrt_rn(warp_sum(acc) * inv_cols + p.eps);
    const float scale = p.code_scale_ptr ? *p.code_scale_ptr : p.code_scale;
    const float recip = p.code_scale_ptr ? __frcp_rn(scale) : p.code_recip;
    const bool lean = lean_scale(scale);
    const uint64_t neg_scale2 = f2_bits(-scale, -scale), recip2 = f2_bits(recip, recip);
#pragma unroll
    for (int j = 0; j < KV; ++j) {
        const int c = lane + 32 * j;
        if (c >= vecs)
            continue;
        const float4 g0 = reinterpret_cast<const float4 *>(gamma_s + 8 * c)[0];
        const float4 g1 = reinterpret_cast<const float4 *>(gamma_s + 8 * c)[1];
        const float4 b0 = reinterpret_cast<const float4 *>(beta_s + 8 * c)[0];
        const float4 b1 = reinterpret_cast<const float4 *>(beta_s + 8 * c)[1];
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        uint32_t out[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float y0 = fmaf((h2f(static_cast<uint16_t>(w[i] & 0xFFFFu)) - mean) * rstd, g[2 * i], b[2 * i]);
            const float y1 = fmaf((h2f(static_cast<uint16_t>(w[i] >> 16)) - mean) * rstd, g[2 * i + 1], b[2 * i + 1]);
            out[i] = gemm::cvt_f16x2(y0, y1);
        }
        if (!kCodesOnly && p.y)
            *reinterpret_cast<uint4 *>(p.y + base + 8 * c) = make_uint4(out[0], out[1], out[2], out[3]);
        if (kCodesOnly || p.codes) {
            const uint32_t lo = e4m3x4(out[0], out[1], lean, neg_scale2, recip2);
            const uint32_t hi = e4m3x4(out[2], out[3], lean, neg_scale2, recip2);
            asm volatile("st.global.v2.u32 [%0], {%1, %2};" ::"l"(p.codes + base + 8 * c), "r"(lo), "r"(hi) : "memory");
        }
    }
    }
}

} // namespace norm

// ---------------------------------------------------------------------------
// Decoder cross-attention over the cached encoder K/V (cpp/src/network_graph.cpp
// :235-244 `attend`, with the cross-K/V cache of :401-404).  A cluster of S CTAs
// serves one (stream, head); all query rows (beams) of the stream share one pass
// over the head's K and V, each CTA over a contiguous range of the keys.
// Pass 1 streams K and forms fp16 scores with m16n8k16 MMAs.  The softmax is
// over all keys: in one exchange through distributed shared memory the CTAs
// share each row's local max m_r and local sum of exp(s - m_r); every CTA then
// forms the global max M and sum L = sum_r l_r exp(m_r - M) in rank order, so
// every probability is half(exp(s - M) / L).  Pass 2 streams V and
// forms each CTA's part of P.V; the parts are summed in rank order by the CTA
// owning each group of output columns.  K/V tiles arrive by TMA (128B-swizzled,
// so the ldmatrix fragment reads are conflict-free) through a ring fed by one
// producer warp.  Peers push values into each other's shared memory and arrive
// on each other's mbarriers, so only the consumer warps take part in exchanges.

namespace attn {

constexpr int kDim = 64;         // head dimension
constexpr int kChunk = 128;      // keys per stage: one 128-row x 128-byte box
constexpr int kMaxStages = 4; // ring depth is chosen per launch (3 or 4)
constexpr int kStageBytes = kChunk * kDim * 2;
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32; // + the producer warp
constexpr int kMaxQueries = 16;           // MMA M
constexpr int kMaxCluster = 8;
// Exchange area: row maxima and sums from every rank, then the P.V parts each
// rank sends to the owner of its columns ([source rank][query row][64 columns]).
constexpr int kXMax = 0;
constexpr int kXSum = kXMax + kMaxCluster * kMaxQueries * 4;
constexpr int kXOut = kXSum + kMaxCluster * kMaxQueries * 4;

struct Params {
    int streams, queries, heads, keys;
    int cluster; // CTAs per (stream, head)
    int kpc;     // keys per CTA (multiple of 16); CTA r takes [r*kpc, min(keys, (r+1)*kpc))
    int pstride; // fp16 elements per score row: kpc + 8 (conflict-free ldmatrix rows)
    int stages;      // K/V ring depth
    int score_bytes; // queries score rows, then a 16-byte zero block (the MMA's padding rows)
    int xch_bytes;
    const uint16_t *q;
    uint16_t *out;
    uint32_t scale2; // fp16 head_dim^-0.25 in both halves
    float code_scale, code_recip;
    const float *code_scale_ptr;
    uint8_t *codes;
};

// Score rows exist for the real query rows only; the MMA's rows past them read
// a 16-byte zero block that follows the rows.
__host__ __device__ constexpr int score_bytes(int queries, int pstride) { return (queries * pstride * 2 + 31) / 16 * 16; }
__host__ __device__ constexpr int xch_bytes(int queries, int cluster) { return kXOut + cluster * queries * kDim * 4; }
__host__ __device__ constexpr int smem_bytes(int stages, int queries, int pstride, int cluster)
{
    return 1024 + stages * kStageBytes + score_bytes(queries, pstride) + xch_bytes(queries, cluster) + 128;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int off = 16; off > 0; off /= 2)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__global__ void __launch_bounds__(kThreads, 1)
    cross_attention_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                           const Params p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t ring = sbase;
    const int depth = p.stages; // ring stages
    uint16_t *scores = reinterpret_cast<uint16_t *>(smem + depth * kStageBytes);
    const uint32_t scores_s = smem_u32(scores);
    const uint32_t zero_s = scores_s + static_cast<uint32_t>(p.score_bytes) - 16;
    float *xch = reinterpret_cast<float *>(smem + depth * kStageBytes + p.score_bytes);
    const uint32_t xch_s = smem_u32(xch);
    const uint32_t bar_full = xch_s + p.xch_bytes;
    const uint32_t bar_empty = bar_full + 8 * depth;
    const uint32_t bar_stats = bar_empty + 8 * depth; // S arrivals: every rank's maxima and sums are here
    const uint32_t bar_out = bar_stats + 8;            // S arrivals: every rank's parts of my columns
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int S = p.cluster;
    const int rank = static_cast<int>(blockIdx.x) % S;
    const int sh = static_cast<int>(blockIdx.x) / S;
    const int head = sh % p.heads;
    const int stream = sh / p.heads;
    const int width = p.heads * kDim;
    const int kbeg = rank * p.kpc;
    const int kend = kbeg + p.kpc < p.keys ? kbeg + p.kpc : p.keys;
    const int lk = kend > kbeg ? kend - kbeg : 0; // this CTA's keys
    const int nchunks = (lk + kChunk - 1) / kChunk;

    if (threadIdx.x == 0) {
        griddepcontrol_launch_dependents();
        for (int i = 0; i < depth; ++i) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, kConsumerWarps);
        }
        mbar_init(bar_stats, S);
        mbar_init(bar_out, S);
        fence_barrier_init();
        prefetch_tensor_map(&tm_k);
        prefetch_tensor_map(&tm_v);
    }
    // Scores start at zero: keys past the last 16-key step stay zero, and so does
    // the zero block the padding rows read, so they add nothing to P.V.
    for (int i = threadIdx.x; i < p.score_bytes / 16; i += kThreads)
        reinterpret_cast<uint4 *>(scores)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    if (S > 1)
        cluster_sync(); // every rank's barriers exist before any peer arrives on them
    griddepcontrol_wait(); // q, K and V are written by earlier kernels

    const int row0 = sh * p.keys + kbeg; // first K/V row of this CTA
    const int total = 2 * nchunks;       // K chunks, then V chunks

    if (warp == kConsumerWarps) {
        // ---------------- producer (one thread) ----------------
        if (lane == 0) {
            int issued = 0;
            for (int c = 0; c < total; ++c, ++issued) {
                const int st = c % depth;
                if (!mbar_wait(bar_empty + 8 * st, ((c / depth) & 1u) ^ 1u, kSiteProducerEmpty))
                    break;
                mbar_arrive_expect_tx(bar_full + 8 * st, kStageBytes);
                const int kc = c < nchunks ? c : c - nchunks;
                tma_load_2d(ring + st * kStageBytes, c < nchunks ? &tm_k : &tm_v, bar_full + 8 * st, 0,
                            row0 + kc * kChunk);
            }
            // Every issued load lands before shared memory is released.
            for (int c = issued > depth ? issued - depth : 0; c < issued; ++c)
                for (int tries = 0; tries < (1 << 22) &&
                                    !mbar_try_wait(bar_full + 8 * (c % depth), (c / depth) & 1u);
                     ++tries) {
                }
        }
    } else {
        const int g = lane >> 2, tig = lane & 3;
        // Q' = half(q * c) as MMA A fragments (rows = query rows, K = 64 dims in 4 steps).
        uint32_t qa[4][4];
        {
            const uint16_t *q0 = p.q + static_cast<size_t>(stream * p.queries + g) * width + head * kDim;
            const uint16_t *q8 = q0 + static_cast<size_t>(8) * width;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const int col = ks * 16 + 2 * tig;
                qa[ks][0] = g < p.queries ? *reinterpret_cast<const uint32_t *>(q0 + col) : 0u;
                qa[ks][1] = g + 8 < p.queries ? *reinterpret_cast<const uint32_t *>(q8 + col) : 0u;
                qa[ks][2] = g < p.queries ? *reinterpret_cast<const uint32_t *>(q0 + col + 8) : 0u;
                qa[ks][3] = g + 8 < p.queries ? *reinterpret_cast<const uint32_t *>(q8 + col + 8) : 0u;
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    qa[ks][r] = gemm::hmul2_rn(qa[ks][r], p.scale2);
            }
        }
        bool ok = true;
        // ---------------- pass 1: scores = half(Q' K'^T) over this CTA's keys ----------------
        for (int c = 0; c < nchunks; ++c) {
            const int st = c % depth;
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar_full + 8 * st, (c / depth) & 1u, kSiteMmaFull));
            const int kc = lk - c * kChunk < kChunk ? lk - c * kChunk : kChunk;
            const uint32_t stage = ring + st * kStageBytes;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int kb = warp * 16 + nt * 8; // first key of this 8-key n-tile
                if (!ok || kb >= kc)
                    continue;
                uint32_t b[8];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    // matrices (k-step 2*half + (i >> 1), 8-dim chunk i & 1) for lanes 8i..8i+7
                    const int mi = lane >> 3, key = kb + (lane & 7);
                    const int chunk16 = 2 * (2 * half + (mi >> 1)) + (mi & 1);
                    uint32_t r[4];
                    ldmatrix_x4(stage + key * 128 + ((chunk16 ^ (key & 7)) << 4), r);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        b[4 * half + i] = gemm::hmul2_rn(r[i], p.scale2); // K' = half(k * c)
                }
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    mma_m16n8k16_f16_f32(acc, qa[ks], b[2 * ks], b[2 * ks + 1]);
                const int key = c * kChunk + kb + 2 * tig;
                const uint32_t lo = gemm::cvt_f16x2(acc[0], acc[1]), hi = gemm::cvt_f16x2(acc[2], acc[3]);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    if (key + e >= lk)
                        continue;
                    if (g < p.queries)
                        scores[g * p.pstride + key + e] = static_cast<uint16_t>(lo >> (16 * e));
                    if (g + 8 < p.queries)
                        scores[(g + 8) * p.pstride + key + e] = static_cast<uint16_t>(hi >> (16 * e));
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(bar_empty + 8 * st);
        }
        named_barrier_sync(1, kConsumers);
        // ---------------- softmax over all keys of the head ----------------
        if (S == 1) {
            // The CTA holds every key: p = half(exp(s - max) / sum) from its own rows.
            for (int row = warp; row < p.queries; row += kConsumerWarps) {
                uint16_t *sr = scores + row * p.pstride;
                float mx = -INFINITY;
                for (int j = lane; j < lk; j += 32)
                    mx = fmaxf(mx, h2f(sr[j]));
                mx = warp_max(mx);
                float sum = 0.0f;
                for (int j = lane; j < lk; j += 32)
                    sum += expf(h2f(sr[j]) - mx);
                sum = norm::warp_sum(sum);
                for (int j = lane; j < lk; j += 32)
                    sr[j] = f2h_rn(__fdiv_rn(expf(h2f(sr[j]) - mx), sum));
            }
        } else {
        // Row max m_r and sum of exp(s - m_r) over this CTA's keys, pushed to
        // every rank: xch[kXMax][rank][row] and xch[kXSum][rank][row].
        for (int row = warp; row < kMaxQueries; row += kConsumerWarps) {
            float mx = -INFINITY;
            if (row < p.queries)
                for (int j = lane; j < lk; j += 32)
                    mx = fmaxf(mx, h2f(scores[row * p.pstride + j]));
            mx = warp_max(mx);
            float sum = 0.0f;
            if (row < p.queries && mx != -INFINITY)
                for (int j = lane; j < lk; j += 32)
                    sum += expf(h2f(scores[row * p.pstride + j]) - mx);
            sum = norm::warp_sum(sum);
            if (lane < S) {
                st_shared_cluster_f32(map_to_rank(xch_s + kXMax + (rank * kMaxQueries + row) * 4, lane), mx);
                st_shared_cluster_f32(map_to_rank(xch_s + kXSum + (rank * kMaxQueries + row) * 4, lane), sum);
            }
        }
        fence_cluster();
        named_barrier_sync(1, kConsumers);
        if (threadIdx.x < S)
            mbar_arrive_cluster(map_to_rank(bar_stats, threadIdx.x));
        ok = ok && __all_sync(0xffffffffu, mbar_wait_cluster(bar_stats, 0, kSiteClusterExchange));
        // p = half(exp(s - M) / L): M the max over ranks, L = sum_r l_r exp(m_r - M)
        // taken in rank order (a rank without keys adds nothing).
        for (int row = warp; row < p.queries; row += kConsumerWarps) {
            float mx = -INFINITY, sum = 0.0f;
            for (int r = 0; r < S; ++r)
                mx = fmaxf(mx, xch[kXMax / 4 + r * kMaxQueries + row]);
            for (int r = 0; r < S; ++r) {
                const float mr = xch[kXMax / 4 + r * kMaxQueries + row];
                if (mr != -INFINITY)
                    sum += xch[kXSum / 4 + r * kMaxQueries + row] * expf(mr - mx);
            }
            for (int j = lane; j < lk; j += 32)
                scores[row * p.pstride + j] =
                    f2h_rn(__fdiv_rn(expf(h2f(scores[row * p.pstride + j]) - mx), sum));
        }
        }
        named_barrier_sync(1, kConsumers);
        // ---------------- pass 2: this CTA's P.V, warp w owns columns 8w..8w+7 ----------------
        float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int c = 0; c < nchunks; ++c) {
            const int seq = nchunks + c, st = seq % depth;
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar_full + 8 * st, (seq / depth) & 1u, kSiteMmaFull));
            const int kc = lk - c * kChunk < kChunk ? lk - c * kChunk : kChunk;
            const uint32_t stage = ring + st * kStageBytes;
            const int steps = ok ? (kc + 15) / 16 : 0;
            for (int ks = 0; ks < steps; ++ks) {
                uint32_t a[4], bv[2];
                {
                    const int mi = lane >> 3, r = lane & 7;
                    const int row = r + (mi & 1) * 8, key = c * kChunk + ks * 16 + (mi >> 1) * 8;
                    ldmatrix_x4(row < p.queries ? scores_s + static_cast<uint32_t>((row * p.pstride + key) * 2) : zero_s, a);
                }
                {
                    const int key = ks * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
                    ldmatrix_x2_trans(stage + key * 128 + ((warp ^ (key & 7)) << 4), bv);
                }
                mma_m16n8k16_f16_f32(o, a, bv[0], bv[1]);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(bar_empty + 8 * st);
        }
        const float scale = p.code_scale_ptr ? *p.code_scale_ptr : p.code_scale;
        const float recip = p.code_scale_ptr ? __frcp_rn(scale) : p.code_recip;
        const uint64_t neg_scale2 = f2_bits(-scale, -scale), recip2 = f2_bits(recip, recip);
        auto store_pair = [&](int row, int col, float v0, float v1) {
            const uint32_t pair = gemm::cvt_f16x2(v0, v1);
            const size_t idx = static_cast<size_t>(stream * p.queries + row) * width + head * kDim + col;
            if (p.out)
                *reinterpret_cast<uint32_t *>(p.out + idx) = pair;
            if (p.codes)
                *reinterpret_cast<uint16_t *>(p.codes + idx) =
                    static_cast<uint16_t>(e4m3x2_quotient(pair, neg_scale2, recip2));
        };
        if (S == 1) {
#pragma unroll
            for (int e = 0; e < 2; ++e)
                if (ok && g + 8 * e < p.queries)
                    store_pair(g + 8 * e, warp * 8 + 2 * tig, o[2 * e], o[2 * e + 1]);
        } else {
        // Parts of P.V go to the owner of their columns: rank r owns 64/S columns.
        const int cols_per = kDim / S;
        const int owner = (warp * 8) / cols_per;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int row = g + 8 * e;
            const int col = warp * 8 + 2 * tig;
            if (row >= p.queries)
                continue;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const uint32_t dst = xch_s + kXOut + ((rank * p.queries + row) * kDim + col + i) * 4;
                st_shared_cluster_f32(map_to_rank(dst, static_cast<uint32_t>(owner)), o[2 * e + i]);
            }
        }
        fence_cluster();
        named_barrier_sync(1, kConsumers);
        if (threadIdx.x < S)
            mbar_arrive_cluster(map_to_rank(bar_out, threadIdx.x));
        ok = ok && __all_sync(0xffffffffu, mbar_wait_cluster(bar_out, 0, kSiteClusterExchange));
        // My columns [rank*cols_per, +cols_per) for every query row: sum the parts in rank order.
        for (int e = threadIdx.x; ok && e < p.queries * (cols_per / 2); e += kConsumers) {
            const int row = e / (cols_per / 2);
            const int col = rank * cols_per + 2 * (e % (cols_per / 2));
            float s0 = 0.0f, s1 = 0.0f;
            for (int r = 0; r < S; ++r) {
                s0 += xch[kXOut / 4 + (r * p.queries + row) * kDim + col];
                s1 += xch[kXOut / 4 + (r * p.queries + row) * kDim + col + 1];
            }
            store_pair(row, col, s0, s1);
        }
        }
    }
    __syncthreads();
    if (S > 1)
        cluster_sync(); // no CTA leaves while stores to its peers may be in flight
}

} // namespace attn

// ---------------------------------------------------------------------------
// Encoder self-attention (cpp/src/network_graph.cpp:235-247 `attention`: `attend`
// on the layer's own q/k/v projections, no mask) with the graph's fp16 edges:
// q' = half(q c), k' = half(k c), scores half(q'.k'), p = half(softmax_fp32),
// out = half(p.v).  A CTA takes 128 query rows of one (stream, head): eight MMA
// warps of 16 rows and a producer warp.  Pass 1 streams K and keeps each row's
// running max and sum of exp; pass 2 streams K and V again, recomputes the same
// fp16 scores and forms p = half(exp(s - max) / sum) with the final max and sum,
// straight from the score accumulators into the A fragments of P.V.  The
// exponentials use the hardware's approximate 2^x (relative error about 2^-22),
// far below the fp16 rounding of p.  q, k and v
// are read in place from the projections' rows (for instance the fused QKV
// output), through 128B-swizzled TMA boxes.

namespace sattn {

// Shared by the self-attention kernel (namespace fattn) and its launcher.
constexpr int kDim = 64;
constexpr int kBQ = 128;    // query rows per CTA
constexpr int kChunk = 128; // keys per tile

struct Params {
    int streams, tokens, heads;
    int qblocks; // ceil(tokens / kBQ)
    int qpairs;  // ceil(qblocks / 2): items per (stream, head), two query tiles each
    int nchunks; // ceil(tokens / kChunk)
    uint16_t *out;
    uint32_t scale2; // fp16 head_dim^-0.25 in both halves
    float code_scale, code_recip;
    const float *code_scale_ptr;
    uint8_t *codes;
};

// 2^x by the hardware's approximate exponential (relative error about 2^-22), and
// log2(x) likewise: exp(s - m) = 2^(s log2(e) - m log2(e)).
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float fast_log2(float x)
{
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;

} // namespace sattn

// ---------------------------------------------------------------------------
// Encoder self-attention on tcgen05 with the graph's fp16 edges (q' = half(q c),
// k' = half(k c), s = half(q'.k'), out = half(sum_j p_j v_j)) and a one-pass
// (online) softmax.  An item is two 128-query tiles (slots A and B) of one
// (stream, head), which share every K and V tile:
//   warp 0: TMA producer (an item's two Q tiles; K and V tiles once each);
//   warp 1: MMA issuer.  Per key tile, S_A = Q'_A K'^T and S_B = Q'_B K'^T
//           (kind::f16 128 x 128 x 16, one TMEM region per slot), then the
//           previous tile's O_X += P_X V (128 x 64 x 16) with P_X read from
//           TMEM and V MN-major straight from its TMA tile;
//   warps 2-3: rescale Q and each K tile in shared memory (half(x c)) before
//           the MMA reads it, half of the tile each;
//   warps 4-7 / 8-11: softmax of slot A / B, one thread per query row with
//           all 128 key columns of a tile, so the row maximum and sum need no
//           exchange between threads.  Each row keeps a running maximum m
//           raised only when a tile's maximum exceeds it by more than 2^8 in
//           exp (then O and the row sum are rescaled in place).
//           P = half(exp(s - m)) is stored as fp16 pairs into the slot's TMEM
//           P region, and out = half(O / sum) at the end of the item.
// Against the graph's p = half(exp(s - max) / sum) the probabilities round once
// each at another scale: the output moves by at most 2^-10 sum_j p_j |v_j| (first
// order), which the tests add to the fp16 bound.
// The two slots' softmax run on different warps while the tensor core works on
// the other slot's tile.  The kernel is persistent: one CTA per SM walks
// (stream, head, query-tile pair) items, its rings and barrier phases running on
// across items; Q is double-buffered by item parity, so the next item's Q and
// first K tiles load and scale while the current item finishes.
namespace fattn {

using sattn::kLog2e;
using sattn::fast_exp2;
constexpr int kDim = 64;
constexpr int kBQ = 128;  // query rows per slot
constexpr int kBK = 128;  // keys per tile
constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr int kTile = kBK * kDim * 2; // one Q, K or V tile: 16 KB
constexpr int kQBytes = 2 * kTile;    // an item's two Q tiles
constexpr int kScaleWarp0 = 2;
constexpr int kScaleWarps = 2;
constexpr int kSoftWarp0 = 4; // slot A: warps 4-7, slot B: 8-11 (warp % 4 = TMEM lane quarter)
constexpr int kSlotThreads = 4 * 32;
constexpr int kThreads = 12 * 32;
constexpr uint32_t kTurnBar0 = 1; // named barriers 1 (slot A's turn) and 2 (slot B's)
constexpr int kOffK = 2 * kQBytes; // Q double-buffered by item parity
constexpr int kOffV = kOffK + kKStages * kTile;
constexpr int kOffRowMax = kOffV + kVStages * kTile; // float [slot][row]
constexpr int kOffBar = kOffRowMax + 2 * kBQ * 4;
constexpr int kBars = 6 + 3 * kKStages + 2 * kVStages + 12 + 1;
constexpr int kSmemBytes = kOffBar + 8 * kBars + 16 + 1024;
// The running maximum is raised only when a tile's maximum exceeds it by more than
// 2^kLazy in exp: P = exp(s - m) then stays below 2^kLazy, exact in fp16 range.
constexpr float kLazy = 8.0f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;   // S of slot X: columns X * 128 .. + 127 (fp32)
constexpr uint32_t kTmemP = 256; // P of slot X: X * 64 .. + 63 (fp16 pairs)
constexpr uint32_t kTmemO = 384; // O of slot X: X * 64 .. + 63 (fp32)
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Packed fp16 maximum (a NaN operand yields the other operand, like fmaxf).
__device__ __forceinline__ uint32_t max_f16x2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// (lo - c, hi - c) of a packed fp16 pair as fp32, one rounding each: the mixed-
// precision add takes the fp16 operand as is, with no separate conversion.
__device__ __forceinline__ void sub_f16x2_f32(uint32_t h2, float c, float &lo, float &hi)
{
    asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.f16 %0, l, %3;\n\tadd.rn.f32.f16 %1, h, %3;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(h2), "f"(-c));
}

// Packed fp32 pairs (low lane = first value): one instruction rounds each lane as
// the scalar mul.rn / add.rn would.
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float lo_f32(uint64_t x) { return __uint_as_float(static_cast<uint32_t>(x)); }
__device__ __forceinline__ float hi_f32(uint64_t x) { return __uint_as_float(static_cast<uint32_t>(x >> 32)); }

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const sattn::Params p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sb = smem_u32(smem);
    const uint32_t sQ = sb, sK = sb + kOffK, sV = sb + kOffV;
    const uint32_t q_full = sb + kOffBar; // [2] by item parity, like q_ready and q_empty
    const uint32_t q_ready = q_full + 16;
    const uint32_t q_empty = q_ready + 16; // the item's Q is read by no later MMA
    const uint32_t k_full = q_empty + 16;
    const uint32_t k_ready = k_full + 8 * kKStages;
    const uint32_t k_empty = k_ready + 8 * kKStages;
    const uint32_t v_full = k_empty + 8 * kKStages;
    const uint32_t v_empty = v_full + 8 * kVStages;
    const uint32_t s_full = v_empty + 8 * kVStages; // [2] by slot, like the five below
    const uint32_t s_empty = s_full + 16;           // the slot's S has been read
    const uint32_t p_full = s_empty + 16;           // the slot's P is in TMEM
    const uint32_t p_empty = p_full + 16;           // the slot's P.V MMAs are done
    const uint32_t o_full = p_empty + 16;           // the item's last P.V is done
    const uint32_t o_empty = o_full + 16;           // the slot's O has been read
    const uint32_t drain = o_empty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8 * kBars);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int nt = p.nchunks;
    const int items = p.streams * p.heads * p.qpairs;
    struct Item {
        int head, row_base, q0; // q0: slot A's first query; slot B's is q0 + kBQ
    };
    auto item_of = [&](int it) {
        const int qp = it % p.qpairs;
        const int sh = it / p.qpairs;
        return Item{sh % p.heads, (sh / p.heads) * p.tokens, qp * 2 * kBQ};
    };

    if (threadIdx.x == 0) {
        griddepcontrol_launch_dependents();
        for (int b = 0; b < 2; ++b) {
            mbar_init(q_full + 8 * b, 1);
            mbar_init(q_ready + 8 * b, kScaleWarps);
            mbar_init(q_empty + 8 * b, 1);
            mbar_init(s_full + 8 * b, 1);
            mbar_init(s_empty + 8 * b, 4);
            mbar_init(p_full + 8 * b, 4);
            mbar_init(p_empty + 8 * b, 1);
            mbar_init(o_full + 8 * b, 1);
            mbar_init(o_empty + 8 * b, 4);
        }
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(k_full + 8 * s, 1);
            mbar_init(k_ready + 8 * s, kScaleWarps);
            mbar_init(k_empty + 8 * s, 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(v_full + 8 * s, 1);
            mbar_init(v_empty + 8 * s, 1);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        prefetch_tensor_map(&tm_q);
        prefetch_tensor_map(&tm_k);
        prefetch_tensor_map(&tm_v);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddepcontrol_wait(); // q, k and v are written by earlier kernels

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int k_issued = 0, v_issued = 0, q_issued = 0;
            bool ok = true;
            for (int it = blockIdx.x, local = 0; ok && it < items; it += gridDim.x, ++local) {
                const Item w = item_of(it);
                const uint32_t qb = local & 1;
                if (!mbar_wait(q_empty + 8 * qb, ((local >> 1) & 1u) ^ 1u, kSiteProducerEmpty))
                    break;
                mbar_arrive_expect_tx(q_full + 8 * qb, kQBytes);
                tma_load_2d(sQ + qb * kQBytes, &tm_q, q_full + 8 * qb, w.head * kDim, w.row_base + w.q0);
                tma_load_2d(sQ + qb * kQBytes + kTile, &tm_q, q_full + 8 * qb, w.head * kDim, w.row_base + w.q0 + kBQ);
                ++q_issued;
                for (int j = 0; j < nt; ++j) {
                    const int s = k_issued % kKStages;
                    if (!mbar_wait(k_empty + 8 * s, ((k_issued / kKStages) & 1u) ^ 1u, kSiteProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(k_full + 8 * s, kTile);
                    tma_load_2d(sK + s * kTile, &tm_k, k_full + 8 * s, w.head * kDim, w.row_base + j * kBK);
                    ++k_issued;
                    const int vs = v_issued % kVStages;
                    if (!mbar_wait(v_empty + 8 * vs, ((v_issued / kVStages) & 1u) ^ 1u, kSiteProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(v_full + 8 * vs, kTile);
                    tma_load_2d(sV + vs * kTile, &tm_v, v_full + 8 * vs, w.head * kDim, w.row_base + j * kBK);
                    ++v_issued;
                }
            }
            // Loads still in flight (only after an abandoned wait) land before exit.
            for (int j = k_issued > kKStages ? k_issued - kKStages : 0; j < k_issued; ++j)
                for (int t = 0; t < (1 << 20) && !mbar_try_wait(k_full + 8 * (j % kKStages), (j / kKStages) & 1u); ++t) {
                }
            for (int c = v_issued > kVStages ? v_issued - kVStages : 0; c < v_issued; ++c)
                for (int t = 0; t < (1 << 20) && !mbar_try_wait(v_full + 8 * (c % kVStages), (c / kVStages) & 1u); ++t) {
                }
            for (int q = q_issued > 2 ? q_issued - 2 : 0; q < q_issued; ++q)
                for (int t = 0; t < (1 << 20) && !mbar_try_wait(q_full + 8 * (q & 1), (q >> 1) & 1u); ++t) {
                }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16_f32<kBQ, kBK>();
            constexpr uint32_t id_o = idesc_f16_f32<kBQ, kDim>() | (1u << 16); // B (V) MN-major
            bool ok = true;
            int u = 0, cc = 0; // score tiles and P tiles issued over all items (per slot)
            int local = 0;
            // Descriptors are computed once: a tile's descriptor is the base one plus
            // the tile's byte offset / 16 (the start-address field), so each MMA
            // issues with one add per operand.  The issuing thread shares its SMSP
            // with softmax warps, and every instruction it saves shortens the
            // tensor core's wait for work.
            const uint64_t d_q = smem_desc_k_sw128(sQ), d_k = smem_desc_k_sw128(sK), d_v = smem_desc_mn_sw128(sV);
            auto pv_mma = [&](int first) { // P.V of P tile cc for both slots
                const int vs = cc % kVStages;
                ok = ok && mbar_wait(v_full + 8 * vs, (cc / kVStages) & 1u, kSiteMmaFull);
                const uint64_t b0 = d_v + static_cast<uint64_t>(vs * (kTile >> 4));
                for (int x = 0; x < 2 && ok; ++x) {
                    if (first)
                        ok = mbar_wait(o_empty + 8 * x, (local & 1u) ^ 1u, kSiteMmaAccEmpty);
                    ok = ok && mbar_wait(p_full + 8 * x, cc & 1u, kSiteMmaFull);
                    if (!ok)
                        break;
                    tc_fence_after();
                    const uint32_t d = tmem + kTmemO + x * kDim, a = tmem + kTmemP + x * (kBK / 2);
                    if (first)
                        mma_f16_ts_c<0>(d, a, b0, id_o);
                    else
                        mma_f16_ts_c<1>(d, a, b0, id_o);
#pragma unroll
                    for (int k = 1; k < kBK / 16; ++k) // 16 keys: 8 TMEM columns of P, 16 rows (2 KB) of V
                        mma_f16_ts_c<1>(d, a + k * 8, b0 + static_cast<uint64_t>(k * (2048 >> 4)), id_o);
                    mma_commit(p_empty + 8 * x);
                }
                if (ok)
                    mma_commit(v_empty + 8 * vs);
                ++cc;
            };
            for (int it = blockIdx.x; ok && it < items; it += gridDim.x, ++local) {
                const uint32_t qb = local & 1;
                ok = mbar_wait(q_ready + 8 * qb, (local >> 1) & 1u, kSiteMmaFull);
                for (int c = 0; ok && c < nt; ++c) {
                    const int ks = u % kKStages;
                    ok = mbar_wait(k_ready + 8 * ks, (u / kKStages) & 1u, kSiteMmaFull);
                    for (int x = 0; x < 2 && ok; ++x) {
                        ok = mbar_wait(s_empty + 8 * x, (u & 1u) ^ 1u, kSiteMmaAccEmpty);
                        if (!ok)
                            break;
                        tc_fence_after();
                        const uint32_t d = tmem + kTmemS + x * kBK;
                        const uint64_t a = d_q + static_cast<uint64_t>((qb * kQBytes + x * kTile) >> 4);
                        const uint64_t b = d_k + static_cast<uint64_t>(ks * (kTile >> 4));
                        mma_f16_c<0>(d, a, b, id_s);
#pragma unroll
                        for (int k = 1; k < kDim / 16; ++k) // 16 dims: 32 bytes along the 128-byte rows
                            mma_f16_c<1>(d, a + 2 * k, b + 2 * k, id_s);
                        mma_commit(s_full + 8 * x);
                    }
                    if (!ok)
                        break;
                    mma_commit(k_empty + 8 * ks);
                    if (c == nt - 1)
                        mma_commit(q_empty + 8 * qb);
                    ++u;
                    if (c > 0)
                        pv_mma(c == 1);
                }
                if (!ok)
                    break;
                pv_mma(nt == 1);
                if (ok) {
                    mma_commit(o_full);
                    mma_commit(o_full + 8);
                }
            }
            // Every MMA of this thread completes before TMEM is freed.
            mma_commit(drain);
            for (int t = 0; t < (1 << 22) && !mbar_try_wait(drain, 0); ++t) {
            }
        }
    } else if (warp >= kScaleWarp0 && warp < kScaleWarp0 + kScaleWarps) {
        // ---------------- operand scaling: x' = half(x c), in place ----------------
        const int part = warp - kScaleWarp0; // this warp's share of each tile
        auto scale_tile = [&](uint32_t tile) {
#pragma unroll 4
            for (int i = 0; i < kTile / 16 / 32 / kScaleWarps; ++i) {
                const uint32_t a = tile + part * (kTile / kScaleWarps) + (i * 32 + lane) * 16;
                uint32_t v0, v1, v2, v3;
                asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3) : "r"(a));
                v0 = gemm::hmul2_rn(v0, p.scale2);
                v1 = gemm::hmul2_rn(v1, p.scale2);
                v2 = gemm::hmul2_rn(v2, p.scale2);
                v3 = gemm::hmul2_rn(v3, p.scale2);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v0), "r"(v1), "r"(v2), "r"(v3)
                             : "memory");
            }
        };
        bool ok = true;
        int k_scaled = 0;
        for (int it = blockIdx.x, local = 0; ok && it < items; it += gridDim.x, ++local) {
            const uint32_t qb = local & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(q_full + 8 * qb, (local >> 1) & 1u, kSiteMmaFull));
            if (!ok)
                break;
            scale_tile(sQ + qb * kQBytes);
            scale_tile(sQ + qb * kQBytes + kTile);
            fence_proxy_async_smem(); // the MMA (async proxy) reads what these stores wrote
            __syncwarp();
            if (lane == 0)
                mbar_arrive(q_ready + 8 * qb);
            for (int j = 0; ok && j < nt; ++j, ++k_scaled) {
                const int s = k_scaled % kKStages;
                ok = __all_sync(0xffffffffu, mbar_wait(k_full + 8 * s, (k_scaled / kKStages) & 1u, kSiteMmaFull));
                if (!ok)
                    break;
                scale_tile(sK + s * kTile);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(k_ready + 8 * s);
            }
        }
    } else if (warp >= kSoftWarp0) {
        // ---------------- softmax: one thread per query row of a slot ----------------
        const int x = (warp - kSoftWarp0) >> 2; // slot
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t s_base = tmem + lanes + kTmemS + x * kBK;
        const uint32_t p_base = tmem + lanes + kTmemP + x * (kBK / 2);
        const uint32_t o_base = tmem + lanes + kTmemO + x * kDim;
        // The two slots take turns at the exponentials: slot x waits for its turn
        // barrier (the other slot's arrival) before its exponentials and hands the
        // turn over after them, so one slot's score loads, maxima and hand-overs
        // run while the other keeps the MUFU busy.  Slot A takes the first turn.
        const uint32_t my_turn = kTurnBar0 + x, their_turn = kTurnBar0 + (x ^ 1);
        const uint32_t m_slot = sb + kOffRowMax + (x * kBQ + row) * 4; // this row's running maximum
        bool ok = true;
        // Every lane polls the barrier (one shared word, the same answer for all
        // lanes); the warp reconverges before the warp-wide TMEM instructions.
        // After a wait has given up, later waits return at once, but every warp
        // still walks every tile (its TMEM accesses stay inside this CTA's
        // allocation) so that the turn barriers always pair up.
        auto wait_all = [&](uint32_t bar, uint32_t parity, int site) {
            ok = ok && mbar_wait(bar, parity, site);
            __syncwarp();
        };
        const uint64_t log2e2 = f2_bits(kLog2e, kLog2e);
        int u = 0, cc = 0;
        for (int it = blockIdx.x, local = 0; it < items; it += gridDim.x, ++local) {
            const Item w = item_of(it);
            float m = -INFINITY; // the row's running maximum
            float l = 0.0f;      // the row's sum of exp(s - m)
            for (int c = 0; c < nt; ++c, ++u, ++cc) {
                // The row's 128 scores of tile c, rounded to fp16 (the MatMul edge);
                // keys past the stream's tokens are -inf.  Frees the slot's S.
                wait_all(s_full + 8 * x, u & 1u, kSiteEpilogueAccFull);
                tc_fence_after();
                uint32_t h[kBK / 2];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t v[64];
                    tmem_ld_32x32b_x32(s_base + half * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
                    tmem_ld_32x32b_x32(s_base + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 64; i += 2)
                        h[half * 32 + i / 2] = gemm::cvt_f16x2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(s_empty + 8 * x);
                const int valid = min(max(p.tokens - c * kBK, 0), kBK);
                if (valid < kBK) // the last tile only: fp16 -inf past the stream's keys
#pragma unroll
                    for (int i = 0; i < kBK; i += 2) {
                        if (i >= valid)
                            h[i / 2] = (h[i / 2] & 0xFFFF0000u) | 0xFC00u;
                        if (i + 1 >= valid)
                            h[i / 2] = (h[i / 2] & 0x0000FFFFu) | 0xFC000000u;
                    }
                // Tile maximum: packed fp16 maxima over eight independent chains.
                uint32_t pm[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    pm[j] = h[j];
#pragma unroll
                for (int i = 8; i < kBK / 2; ++i)
                    pm[i & 7] = max_f16x2(pm[i & 7], h[i]);
                const uint32_t m2 = max_f16x2(max_f16x2(max_f16x2(pm[0], pm[1]), max_f16x2(pm[2], pm[3])),
                                              max_f16x2(max_f16x2(pm[4], pm[5]), max_f16x2(pm[6], pm[7])));
                const float tm = fmaxf(h2f(static_cast<uint16_t>(m2 & 0xFFFFu)), h2f(static_cast<uint16_t>(m2 >> 16)));
                // Raise the running maximum on the first tile, or when the tile's
                // maximum exceeds it by more than 2^kLazy in exp; alpha rescales what
                // was summed (and accumulated in O) against the old maximum.
                float alpha = 1.0f;
                bool raised = false;
                if (m == -INFINITY || (tm - m) * kLog2e > kLazy) {
                    raised = m != -INFINITY;
                    alpha = raised ? fast_exp2((m - tm) * kLog2e) : 0.0f;
                    l *= alpha;
                    m = tm;
                }
                // P.V of the previous tile is done: P is free and O holds this item's
                // tiles 0 .. c - 1 against the old maximum.
                wait_all(p_empty + 8 * x, (cc & 1u) ^ 1u, kSiteProducerEmpty);
                if (ok && c > 0 && __any_sync(0xffffffffu, raised)) {
                    // Scale the raised rows of O (the other rows by 1: the TMEM
                    // access is warp-wide).
                    tc_fence_after();
                    uint32_t o[kDim];
                    tmem_ld_32x32b_x32(o_base, *reinterpret_cast<uint32_t(*)[32]>(o));
                    tmem_ld_32x32b_x32(o_base + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
                    tmem_wait_ld();
                    const float f = raised ? alpha : 1.0f;
#pragma unroll
                    for (int i = 0; i < kDim; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                    tmem_st_32x32b_x32(o_base, *reinterpret_cast<const uint32_t(*)[32]>(o));
                    tmem_st_32x32b_x32(o_base + 32, *reinterpret_cast<const uint32_t(*)[32]>(o + 32));
                }
                // The exponentials read m back from shared memory after the turn
                // barrier, so no compiler stage can hoist them above it; the hand-over
                // waits for the P stores, so none can sink below it.
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(m_slot), "f"(m) : "memory");
                if (x == 1 || u > 0)
                    turn_wait(my_turn, 2 * kSlotThreads);
                asm volatile("ld.volatile.shared.f32 %0, [%1];" : "=f"(m) : "r"(m_slot) : "memory");
                // P = half(exp(s - m)) with packed fp32 pairs; the row sum takes the
                // unrounded exponentials (four partial pairs keep the chains short).
                uint64_t ps[4] = {0, 0, 0, 0};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float d0, d1;
                        sub_f16x2_f32(h[q * 16 + i], m, d0, d1);
                        const uint64_t e = mul_f32x2(f2_bits(d0, d1), log2e2);
                        const float e0 = fast_exp2(lo_f32(e)), e1 = fast_exp2(hi_f32(e));
                        ps[i & 3] = add_f32x2(ps[i & 3], f2_bits(e0, e1));
                        pk[i] = gemm::cvt_f16x2(e0, e1);
                    }
                    tmem_st_32x32b_x16(p_base + q * 16, pk);
                }
                tmem_wait_st();
                turn_pass(their_turn, 2 * kSlotThreads);
                l += ((lo_f32(ps[0]) + hi_f32(ps[0])) + (lo_f32(ps[1]) + hi_f32(ps[1]))) +
                     ((lo_f32(ps[2]) + hi_f32(ps[2])) + (lo_f32(ps[3]) + hi_f32(ps[3])));
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(p_full + 8 * x);
            }
            // ---- epilogue: out = half(O / sum) for the row's 64 dims ----
            const float inv = __frcp_rn(l);
            wait_all(o_full + 8 * x, local & 1u, kSiteEpilogueAccFull);
            tc_fence_after();
            uint32_t o[kDim];
            tmem_ld_32x32b_x32(o_base, *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld_32x32b_x32(o_base + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(o_empty + 8 * x); // the next item's P.V MMAs may overwrite O
            const int token = w.q0 + x * kBQ + row;
            if (ok && token < p.tokens) {
                const size_t idx = static_cast<size_t>(w.row_base + token) * (p.heads * kDim) + w.head * kDim;
                uint32_t hy[kDim / 2];
                const uint64_t inv2 = f2_bits(inv, inv);
#pragma unroll
                for (int i = 0; i < kDim / 2; ++i) {
                    const uint64_t y = mul_f32x2(f2_bits(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2);
                    hy[i] = gemm::cvt_f16x2(lo_f32(y), hi_f32(y));
                }
                if (p.out) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + idx);
#pragma unroll
                    for (int j = 0; j < kDim / 8; ++j)
                        dst[j] = make_uint4(hy[4 * j], hy[4 * j + 1], hy[4 * j + 2], hy[4 * j + 3]);
                }
                if (p.codes) {
                    const float scale = p.code_scale_ptr ? *p.code_scale_ptr : p.code_scale;
                    const float recip = p.code_scale_ptr ? __frcp_rn(scale) : p.code_recip;
                    const uint64_t neg_scale2 = f2_bits(-scale, -scale), recip2 = f2_bits(recip, recip);
                    uint32_t qc[kDim / 4];
#pragma unroll
                    for (int j = 0; j < kDim / 4; ++j)
                        qc[j] = (e4m3x2_quotient(hy[2 * j], neg_scale2, recip2) & 0xFFFFu) |
                                (e4m3x2_quotient(hy[2 * j + 1], neg_scale2, recip2) << 16);
                    uint4 *dst = reinterpret_cast<uint4 *>(p.codes + idx);
#pragma unroll
                    for (int j = 0; j < kDim / 16; ++j)
                        dst[j] = make_uint4(qc[4 * j], qc[4 * j + 1], qc[4 * j + 2], qc[4 * j + 3]);
                }
            }
        }
        // Slot A takes slot B's last hand-over, so both turn barriers end complete.
        if (x == 0 && u > 0)
            turn_wait(my_turn, 2 * kSlotThreads);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

} // namespace fattn

// ---------------------------------------------------------------------------
// fp16 single-token projections (the reference plugins' kernels on sm_100a).

namespace proj {

constexpr int kThreads = 256;

// Slab kernel geometry.  Each CTA owns a contiguous run of weight rows (one CTA
// per SM for the plugins' shapes) and pulls the whole run into shared memory
// with bulk copies at kernel start, so every byte of the weight is in flight
// after one DRAM latency and the next launch's copies can start (programmatic
// dependent launch) while this one finishes its sums.
constexpr int kSlabThreads = 256;
constexpr int kSlabMaxBytes = 96 * 1024; // weight rows per CTA
constexpr int kSlabMaxWidth = 4096;      // DEPTH <= 4096: 128 values per lane
constexpr int kSlabChunks = 16;          // one mbarrier per chunk of rows
constexpr int kSlabSmemBytes = kSlabMaxBytes;

// fp32 fma of two fp16 operands: RN(a*b + c) with the product exact (sm_100
// mixed-precision fma), so fma16(a, b, -0) is the exact product, signed zero
// included, and fma16(a, b, c) equals fadd(a*b, c) for any c.
__device__ __forceinline__ float fma16(uint16_t a, uint16_t b, float c)
{
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint16_t half_of(const uint2 &v, int e)
{
    const uint32_t word = e < 2 ? v.x : v.y;
    return static_cast<uint16_t>((e & 1) ? word >> 16 : word & 0xFFFFu);
}

// Two fp32 adds in one packed instruction: (a0 + b0, a1 + b1), each rounded
// to nearest as a scalar add would be.
__device__ __forceinline__ float2 add2(float2 a, float2 b)
{
    uint64_t d;
    const uint64_t ua = (static_cast<uint64_t>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x);
    const uint64_t ub = (static_cast<uint64_t>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(ua), "l"(ub));
    return make_float2(__uint_as_float(static_cast<uint32_t>(d)), __uint_as_float(static_cast<uint32_t>(d >> 32)));
}

// x . w for one row in the reference plugins' summation order
// (cpp/kernels.cu:27-49).  With DEPTH = max(128, the power of two >= width) and
// V = DEPTH / 32, lane L holds the products for columns (i/4)*128 + 4L + i%4,
// i < V, and +0 past the width.  The V values are folded by halving strides
// (p[i] += p[i + s] for s = V/2, ..., 1), then across lanes by shfl_down with
// offsets 16, ..., 1; lane 0 holds the row's sum.  fp16 x fp16 products are
// exact in fp32, so this order alone fixes every rounding and the result equals
// the reference kernel's bit for bit.  The first fold is one fma16 pair per
// value: p[i] + p[i + V/2] = fma16(x_i, w_i, fma16(x_j, w_j, -0)); the later
// folds add neighbouring pairs with one packed instruction.  Columns past the
// width carry x = w = 0, whose product +0 is the reference's padding value
// (and +0 + -0 = +0 as in its fold).  G > 0 states at compile time that the
// width is G * 128 (every lane's first G column groups in, the rest out), so
// padding products become the constant +0; G = 0 tests each group against the
// runtime width.  xg holds the lane's x groups, ws is the row in shared memory.
template <int V, int G>
__device__ __forceinline__ float tree_dot(const uint2 (&xg)[V / 4], const uint16_t *ws, int width, int lane)
{
    constexpr int kGroups = G > 0 ? G : V / 4;
    uint2 wg[V / 4];
#pragma unroll
    for (int g = 0; g < V / 4; ++g) {
        const int col = g * 128 + 4 * lane;
        // width % 8 == 0: a lane's four columns are all in or all out
        const bool in = G > 0 ? g < G : col < width;
        wg[g] = in ? *reinterpret_cast<const uint2 *>(ws + col) : make_uint2(0u, 0u);
    }
    float p[V / 2];
#pragma unroll
    for (int i = 0; i < V / 2; ++i) {
        const int j = i + V / 2;
        if (i / 4 >= kGroups) {
            p[i] = 0.0f; // +0 + +0
        } else {
            const float pj =
                j / 4 < kGroups ? fma16(half_of(xg[j / 4], j % 4), half_of(wg[j / 4], j % 4), -0.0f) : 0.0f;
            p[i] = fma16(half_of(xg[i / 4], i % 4), half_of(wg[i / 4], i % 4), pj);
        }
    }
#pragma unroll
    for (int s = V / 4; s > 1; s /= 2) {
#pragma unroll
        for (int i = 0; i < s; i += 2) {
            const float2 r = add2(make_float2(p[i], p[i + 1]), make_float2(p[i + s], p[i + s + 1]));
            p[i] = r.x;
            p[i + 1] = r.y;
        }
    }
    float r = V / 2 > 1 ? __fadd_rn(p[0], p[1]) : p[0];
#pragma unroll
    for (int off = 16; off > 0; off /= 2)
        r = __fadd_rn(r, __shfl_down_sync(0xffffffffu, r, off));
    return r;
}

// The row's bias bits as staged in shared memory: fc1 keeps bias[r] in the low
// half; qkv keeps q_bias[r] (rows < width) low and v_bias[r - 2 width] (rows >=
// 2 width) high, +0 where the row has none, as the reference's `q`/`v` terms.
template <bool kFc1>
__device__ __forceinline__ uint32_t projection_bias(int gr, int width, const uint16_t *__restrict__ b0,
                                                    const uint16_t *__restrict__ b1)
{
    if (kFc1)
        return b0[gr];
    const uint32_t q = gr < width ? b0[gr] : 0u;
    const uint32_t v = gr >= 2 * width ? b1[gr - 2 * width] : 0u;
    return q | (v << 16);
}

template <bool kFc1>
__device__ __forceinline__ uint16_t projection_out(float acc, uint32_t bias)
{
    if (kFc1)
        return gelu_fp16_edges(hadd_rn(f2h_rn(acc), static_cast<uint16_t>(bias)));
    const float q = h2f(static_cast<uint16_t>(bias & 0xFFFFu));
    const float v = h2f(static_cast<uint16_t>(bias >> 16));
    return f2h_rn(__fadd_rn(__fadd_rn(acc, q), v));
}

// y = the plugin projection of x (fc1 or qkv) for rows_per_cta weight rows per
// CTA.  Thread 0 issues the CTA's weight rows as up to kSlabChunks bulk copies,
// each completing on its own mbarrier, and the CTA stages its rows' biases in
// shared memory, all before griddepcontrol.wait (weights and biases are layer
// constants); x is read after it, straight into each lane's registers.  Warp w
// sums rows w, w + 8, ... two at a time as their chunks land.  Waits are
// bounded; a CTA that gave up still waits (bounded) for its copies before it
// exits.
template <int V, int G, bool kFc1>
__global__ void __launch_bounds__(kSlabThreads)
    fp16_projection_slab_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                                const uint16_t *__restrict__ b0, const uint16_t *__restrict__ b1,
                                uint16_t *__restrict__ y, int rows, int width, int rows_per_cta, int chunk_rows)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[kSlabChunks];
    constexpr int kWarps = kSlabThreads / 32;
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int row0 = blockIdx.x * rows_per_cta;
    const int nrows = min(rows_per_cta, rows - row0);
    const int nchunks = (nrows + chunk_rows - 1) / chunk_rows;
    const uint32_t row_bytes = static_cast<uint32_t>(width) * 2;
    const uint16_t *ws = reinterpret_cast<const uint16_t *>(smem);
    uint32_t *bias_s = reinterpret_cast<uint32_t *>(smem + static_cast<size_t>(rows_per_cta) * row_bytes);
    const uint32_t bar0 = smem_u32(bars);

    if (threadIdx.x == 0) {
        for (int c = 0; c < nchunks; ++c)
            mbar_init(bar0 + 8 * c, 1);
        fence_barrier_init();
        for (int c = 0; c < nchunks; ++c) {
            const int r = c * chunk_rows;
            const uint32_t bytes = static_cast<uint32_t>(min(chunk_rows, nrows - r)) * row_bytes;
            mbar_arrive_expect_tx(bar0 + 8 * c, bytes);
            bulk_load(smem_u32(smem) + static_cast<uint32_t>(r) * row_bytes,
                      w + static_cast<size_t>(row0 + r) * width, bytes, bar0 + 8 * c);
        }
    }
    for (int r = threadIdx.x; r < nrows; r += kSlabThreads)
        bias_s[r] = projection_bias<kFc1>(row0 + r, width, b0, b1);
    griddepcontrol_launch_dependents();
    griddepcontrol_wait(); // x is written by the previous kernel
    uint2 xg[V / 4];
#pragma unroll
    for (int g = 0; g < V / 4; ++g) {
        const int col = g * 128 + 4 * lane;
        xg[g] = col < width ? __ldg(reinterpret_cast<const uint2 *>(x + col)) : make_uint2(0u, 0u);
    }
    __syncthreads(); // barrier inits and staged biases are visible to every warp

    bool ok = true;
    for (int r = warp; r < nrows; r += 2 * kWarps) {
        const int r2 = r + kWarps;
        const bool two = r2 < nrows;
        ok = __all_sync(0xffffffffu, mbar_wait(bar0 + 8 * (r / chunk_rows), 0, kSiteMmaFull) &&
                                         (!two || mbar_wait(bar0 + 8 * (r2 / chunk_rows), 0, kSiteMmaFull)));
        if (!ok)
            break;
        const float acc = tree_dot<V, G>(xg, ws + static_cast<size_t>(r) * width, width, lane);
        const float acc2 = two ? tree_dot<V, G>(xg, ws + static_cast<size_t>(r2) * width, width, lane) : 0.0f;
        if (lane == 0) {
            y[row0 + r] = projection_out<kFc1>(acc, bias_s[r]);
            if (two)
                y[row0 + r2] = projection_out<kFc1>(acc2, bias_s[r2]);
        }
    }
    if (__syncthreads_or(!ok) && threadIdx.x == 0) {
        for (int c = 0; c < nchunks; ++c)
            mbar_wait(bar0 + 8 * c, 0, kSiteDrain);
    }
}

// One warp per output row; each lane streams 8 halves per 128-bit load.  Used
// for widths above kSlabMaxWidth (sequential per-lane order, then xor shuffles).
template <bool kFc1>
__global__ void __launch_bounds__(kThreads)
    fp16_projection_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w,
                           const uint16_t *__restrict__ b0, const uint16_t *__restrict__ b1,
                           uint16_t *__restrict__ y, int rows, int width)
{
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int chunks = width / 8;
    for (int r = blockIdx.x * (kThreads / 32) + warp; r < rows; r += gridDim.x * (kThreads / 32)) {
        const uint16_t *wrow = w + static_cast<size_t>(r) * width;
        float acc = 0.0f;
        for (int c = lane; c < chunks; c += 32) {
            const uint4 wv = ld_stream16(wrow + c * 8);
            const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(x) + c);
            uint16_t wh[8], xh[8];
            memcpy(wh, &wv, 16);
            memcpy(xh, &xv, 16);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                acc = fmaf(h2f(xh[i]), h2f(wh[i]), acc); // fp16 x fp16 products are exact in fp32
        }
#pragma unroll
        for (int off = 16; off > 0; off /= 2)
            acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) {
            if (kFc1) {
                const uint16_t value = hadd_rn(f2h_rn(acc), b0[r]);
                y[r] = gelu_fp16_edges(value);
            } else {
                const float q = r < width ? h2f(b0[r]) : 0.0f;
                const float v = r >= 2 * width ? h2f(b1[r - 2 * width]) : 0.0f;
                y[r] = f2h_rn(__fadd_rn(__fadd_rn(acc, q), v));
            }
        }
    }
}

// Elementwise GELU with fp16 edges (graph::gelu, network_graph.cpp:168-180),
// through the same erf path as the GEMM epilogue (table read from global).
__global__ void __launch_bounds__(kThreads)
    fp16_gelu_kernel(const uint16_t *__restrict__ x, uint16_t *__restrict__ y, int64_t count)
{
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < count; i += stride)
        y[i] = static_cast<uint16_t>(gemm::gelu_fp16x2(x[i], g_erf_table) & 0xFFFFu);
}

__global__ void __launch_bounds__(kThreads)
    fp16_bias_kernel(const uint16_t *__restrict__ x, uint16_t bias, uint16_t *__restrict__ y,
                     uint32_t count)
{
    const float b = h2f(bias);
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < count; i += gridDim.x * kThreads)
        y[i] = f2h_rn(__fadd_rn(h2f(x[i]), b));
}

} // namespace proj

// ---------------------------------------------------------------------------
// Encoder front end: the fp32 log-mel cast to fp16 (network_graph.cpp:257,
// `half(mel)`) and transposed to the time-major, zero-padded rows the
// convolution reads, and the convolution weights re-laid tap-major.

namespace front {

constexpr int kTile = 32;

// mel fp32 [streams, mels, frames] -> x fp16 [streams, frames + 2, mels] with
// x[s][t + 1][c] = half(mel[s][c][t]) and rows 0, frames + 1 zero.  A 32 x 32
// tile goes through shared memory so both the read (along frames) and the
// write (along mels) are coalesced.
__global__ void __launch_bounds__(kTile * 8)
    mel_frames_kernel(const float *__restrict__ mel, int mels, int frames, uint16_t *__restrict__ x)
{
    __shared__ uint16_t tile[kTile][kTile + 2];
    const int s = blockIdx.z;
    const int t0 = blockIdx.x * kTile;
    const int c0 = blockIdx.y * kTile;
    const float *src = mel + static_cast<size_t>(s) * mels * frames;
    uint16_t *dst = x + static_cast<size_t>(s) * (frames + 2) * mels;
    for (int r = threadIdx.y; r < kTile; r += 8) {
        const int c = c0 + r, t = t0 + threadIdx.x;
        tile[r][threadIdx.x] = (c < mels && t < frames) ? f2h_rn(src[static_cast<size_t>(c) * frames + t]) : 0;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < kTile; r += 8) {
        const int t = t0 + r, c = c0 + threadIdx.x;
        if (t < frames && c < mels)
            dst[static_cast<size_t>(t + 1) * mels + c] = tile[threadIdx.x][r];
    }
    if (blockIdx.x == 0) // the two padding rows of this stream's column range
        for (int i = threadIdx.y * kTile + threadIdx.x; i < kTile; i += kTile * 8)
            if (c0 + i < mels) {
                dst[c0 + i] = 0;
                dst[static_cast<size_t>(frames + 1) * mels + c0 + i] = 0;
            }
}

// w [c_out, c_in, 3] -> out [c_out, 3, c_in]: out[o][j][i] = w[o][i][j].
__global__ void __launch_bounds__(256)
    conv_weight_layout_kernel(const uint16_t *__restrict__ w, int64_t c_out, int64_t c_in, uint16_t *__restrict__ out)
{
    const int64_t total = c_out * c_in * 3;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * 256) {
        const int64_t o = e / (3 * c_in);
        const int64_t rem = e - o * 3 * c_in;
        const int64_t j = rem / c_in;
        const int64_t i = rem - j * c_in;
        out[e] = w[(o * c_in + i) * 3 + j];
    }
}

} // namespace front

// ---------------------------------------------------------------------------
// Decoder step pieces (network_graph.cpp:378-416): the token + position
// embedding, self-attention over the fp16 KV cache with the step's own key and
// value appended, and the greedy token choice.  Lengths (cached keys per stream,
// which is also the new token's position) live in device memory, so one CUDA
// graph of a step serves every step of a decode.

namespace dec {

// Sticky error word of the decoder kernels (1: token or position outside its
// table, 2: cache full); read and cleared by read_and_clear_decoder_error.
__device__ int g_decoder_error = 0;

constexpr int kDim = 64;
constexpr int kAttnThreads = 128;
constexpr int kMaxCache = 512;                        // keys per (stream, head), the new one included
constexpr int kKeysPerThread = kMaxCache / kAttnThreads;
constexpr int kGroups = kAttnThreads / 16;            // P.V: 16 threads x 4 dims cover a row

// x[s] = half(token_table[tokens[s]] + position_table[lengths[s]]), 8 halves per thread.
__global__ void __launch_bounds__(256)
    embed_kernel(const int32_t *__restrict__ tokens, const int32_t *__restrict__ lengths,
                 const uint16_t *__restrict__ token_table, const uint16_t *__restrict__ position_table, int width,
                 int vocab, int positions, uint16_t *__restrict__ x)
{
    griddepcontrol_wait(); // tokens and lengths come from the previous step
    const int s = blockIdx.x;
    const int tok = tokens[s], pos = lengths[s];
    if (tok < 0 || tok >= vocab || pos < 0 || pos >= positions) {
        if (threadIdx.x == 0)
            atomicExch(&g_decoder_error, 1);
        return;
    }
    const uint4 *a = reinterpret_cast<const uint4 *>(token_table + static_cast<size_t>(tok) * width);
    const uint4 *b = reinterpret_cast<const uint4 *>(position_table + static_cast<size_t>(pos) * width);
    uint4 *y = reinterpret_cast<uint4 *>(x + static_cast<size_t>(s) * width);
    for (int i = threadIdx.x; i < width / 8; i += blockDim.x) {
        const uint4 u = __ldg(a + i), v = __ldg(b + i);
        y[i] = make_uint4(gemm::hadd2_rn(u.x, v.x), gemm::hadd2_rn(u.y, v.y), gemm::hadd2_rn(u.z, v.z),
                          gemm::hadd2_rn(u.w, v.w));
    }
}

struct AttnParams {
    int heads, capacity;
    const uint16_t *qkv;   // [streams, qkv_ld]: q | k | v columns of the step's QKV linear
    int64_t qkv_ld;
    uint16_t *cache_k;     // [streams, heads, capacity, 64]
    uint16_t *cache_v;
    const int32_t *lengths; // cached keys per stream before this step
    uint32_t scale2;        // fp16 head_dim^-0.25 in both halves
    uint16_t *out;          // [streams, heads * 64] or null
    uint8_t *codes;         // [streams, heads * 64] or null
    float code_scale, code_recip;
};

// One CTA per (stream, head): append the step's k and v at row `length` of the
// cache, then attend q over rows 0 .. length with the graph's fp16 edges:
// q' = half(q c), k' = half(k c), s = half(q'.k'), p = half(exp(s - max) / sum),
// out = half(sum_j p_j v_j).  The scores stay in registers, so the exact
// normalised p costs no second pass over K.
__global__ void __launch_bounds__(kAttnThreads)
    self_attention_kernel(const AttnParams p)
{
    __shared__ __align__(16) uint16_t q_s[kDim];
    __shared__ float p_s[kMaxCache];
    __shared__ float red[kAttnThreads / 32];
    __shared__ __align__(16) float part[kGroups][kDim];
    const int sh = blockIdx.x;
    const int s = sh / p.heads, h = sh % p.heads;
    const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    griddepcontrol_wait(); // the QKV linear and the previous step wrote what is read here
    const int n0 = p.lengths[s];
    if (n0 < 0 || n0 >= p.capacity) {
        if (tid == 0)
            atomicExch(&g_decoder_error, 2);
        return;
    }
    const int n = n0 + 1;
    const uint16_t *row = p.qkv + static_cast<size_t>(s) * p.qkv_ld;
    const size_t base = (static_cast<size_t>(s) * p.heads + h) * p.capacity * kDim;
    uint16_t *ck = p.cache_k + base;
    uint16_t *cv = p.cache_v + base;
    const int width = p.heads * kDim;
    // the step's k and v rows -> cache row n0; q' -> shared memory
    if (tid < 8) {
        reinterpret_cast<uint4 *>(ck + static_cast<size_t>(n0) * kDim)[tid] =
            reinterpret_cast<const uint4 *>(row + width + h * kDim)[tid];
    } else if (tid < 16) {
        reinterpret_cast<uint4 *>(cv + static_cast<size_t>(n0) * kDim)[tid - 8] =
            reinterpret_cast<const uint4 *>(row + 2 * width + h * kDim)[tid - 8];
    } else if (tid < 24) {
        uint4 v = reinterpret_cast<const uint4 *>(row + h * kDim)[tid - 16];
        v = make_uint4(gemm::hmul2_rn(v.x, p.scale2), gemm::hmul2_rn(v.y, p.scale2), gemm::hmul2_rn(v.z, p.scale2),
                       gemm::hmul2_rn(v.w, p.scale2));
        reinterpret_cast<uint4 *>(q_s)[tid - 16] = v;
    }
    __syncthreads(); // the appended rows and q' are visible to the whole block
    uint32_t q2[kDim / 2];
#pragma unroll
    for (int i = 0; i < kDim / 8; ++i) {
        const uint4 v = reinterpret_cast<const uint4 *>(q_s)[i];
        q2[4 * i] = v.x;
        q2[4 * i + 1] = v.y;
        q2[4 * i + 2] = v.z;
        q2[4 * i + 3] = v.w;
    }
    // scores: thread t takes keys t, t + 128, ...
    float sc[kKeysPerThread];
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kKeysPerThread; ++r) {
        const int j = tid + r * kAttnThreads;
        sc[r] = -INFINITY;
        if (j < n) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(ck + static_cast<size_t>(j) * kDim);
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < kDim / 8; ++i) {
                const uint4 v = kr[i];
                const uint32_t w[4] = {gemm::hmul2_rn(v.x, p.scale2), gemm::hmul2_rn(v.y, p.scale2),
                                       gemm::hmul2_rn(v.z, p.scale2), gemm::hmul2_rn(v.w, p.scale2)};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t a = q2[4 * i + e], b = w[e];
                    acc = fmaf(h2f(static_cast<uint16_t>(a & 0xFFFFu)), h2f(static_cast<uint16_t>(b & 0xFFFFu)), acc);
                    acc = fmaf(h2f(static_cast<uint16_t>(a >> 16)), h2f(static_cast<uint16_t>(b >> 16)), acc);
                }
            }
            sc[r] = h2f(f2h_rn(acc)); // the MatMul's fp16 edge
            mx = fmaxf(mx, sc[r]);
        }
    }
    mx = attn::warp_max(mx);
    if (lane == 0)
        red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float sum = 0.0f;
#pragma unroll
    for (int r = 0; r < kKeysPerThread; ++r) {
        sc[r] = tid + r * kAttnThreads < n ? __expf(sc[r] - mx) : 0.0f;
        sum += sc[r];
    }
#pragma unroll
    for (int off = 16; off > 0; off /= 2)
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0)
        red[warp] = sum;
    __syncthreads();
    sum = (red[0] + red[1]) + (red[2] + red[3]);
#pragma unroll
    for (int r = 0; r < kKeysPerThread; ++r) {
        const int j = tid + r * kAttnThreads;
        if (j < n)
            p_s[j] = h2f(f2h_rn(__fdiv_rn(sc[r], sum))); // p = half(softmax)
    }
    __syncthreads();
    // P.V: thread t sums dims 4 (t % 16) .. + 3 over keys j = t / 16 (mod kGroups)
    const int d0 = 4 * (tid % 16), g = tid / 16;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = g; j < n; j += kGroups) {
        const uint2 v = *reinterpret_cast<const uint2 *>(cv + static_cast<size_t>(j) * kDim + d0);
        const float pj = p_s[j];
        o[0] = fmaf(pj, h2f(static_cast<uint16_t>(v.x & 0xFFFFu)), o[0]);
        o[1] = fmaf(pj, h2f(static_cast<uint16_t>(v.x >> 16)), o[1]);
        o[2] = fmaf(pj, h2f(static_cast<uint16_t>(v.y & 0xFFFFu)), o[2]);
        o[3] = fmaf(pj, h2f(static_cast<uint16_t>(v.y >> 16)), o[3]);
    }
    *reinterpret_cast<float4 *>(&part[g][d0]) = make_float4(o[0], o[1], o[2], o[3]);
    __syncthreads();
    if (tid < kDim / 2) { // two output dims per thread, key groups summed in order
        float a = 0.0f, b = 0.0f;
#pragma unroll
        for (int k = 0; k < kGroups; ++k) {
            a += part[k][2 * tid];
            b += part[k][2 * tid + 1];
        }
        const uint32_t h2 = gemm::cvt_f16x2(a, b);
        const size_t idx = static_cast<size_t>(s) * width + h * kDim + 2 * tid;
        if (p.out)
            *reinterpret_cast<uint32_t *>(p.out + idx) = h2;
        if (p.codes) {
            const uint64_t neg_scale2 = f2_bits(-p.code_scale, -p.code_scale);
            const uint64_t recip2 = f2_bits(p.code_recip, p.code_recip);
            *reinterpret_cast<uint16_t *>(p.codes + idx) =
                static_cast<uint16_t>(e4m3x2_quotient(h2, neg_scale2, recip2) & 0xFFFFu);
        }
    }
}

// Greedy choice per stream (network_graph.cpp:332-339 select_token):
// score = fp32(logits) + suppression; token = the smallest index whose score
// equals the maximum.  Then the stream's length grows by one (the step's key and
// value are in the cache now).
constexpr int kSelectThreads = 1024;
__global__ void __launch_bounds__(kSelectThreads)
    select_kernel(const uint16_t *__restrict__ logits, int64_t logits_ld, const float *__restrict__ suppression,
                  int64_t suppression_ld, int vocab, int32_t *__restrict__ tokens, int32_t *__restrict__ lengths)
{
    __shared__ float best_v[kSelectThreads / 32];
    __shared__ int best_i[kSelectThreads / 32];
    griddepcontrol_wait();
    const int s = blockIdx.x;
    const uint16_t *row = logits + static_cast<size_t>(s) * logits_ld;
    const float *sup = suppression + static_cast<size_t>(s) * suppression_ld;
    float bv = -INFINITY;
    int bi = vocab;
    for (int i = threadIdx.x; i < vocab; i += kSelectThreads) {
        const float v = h2f(row[i]) + sup[i];
        if (v > bv) { // increasing i per thread: the first index of a tie stays
            bv = v;
            bi = i;
        }
    }
    // (value, index) maximum with ties to the smaller index, over the warp then the block
#pragma unroll
    for (int off = 16; off > 0; off /= 2) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (threadIdx.x % 32 == 0) {
        best_v[threadIdx.x / 32] = bv;
        best_i[threadIdx.x / 32] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = best_v[threadIdx.x];
        bi = best_i[threadIdx.x];
#pragma unroll
        for (int off = 16; off > 0; off /= 2) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (threadIdx.x == 0) {
            tokens[s] = bi < vocab ? bi : vocab; // vocab: every score was NaN (the graph's sentinel)
            if (lengths)
                lengths[s] += 1;
        }
    }
}

} // namespace dec

namespace proj {

} // namespace proj

// ---------------------------------------------------------------------------
// Host side.

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult status{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
                cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// 2-D row-major tensor [rows, cols] with `elem` bytes per element.
// 2-D tensor map over [rows, cols] elements whose rows are `ld` elements apart
// (ld >= cols: a column window of a wider matrix).
bool make_map_ld(CUtensorMap *map, CUtensorMapDataType type, int elem, const void *base, int64_t rows,
                 int64_t cols, int64_t ld, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn)
        return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem)};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estrides[2] = {1, 1};
    return fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estrides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map(CUtensorMap *map, CUtensorMapDataType type, int elem, const void *base, int64_t rows,
              int64_t cols, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn)
        return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * elem)};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estrides[2] = {1, 1};
    return fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estrides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// N-d tensor map (rank <= 5): dims[0] is the contiguous axis, strides_bytes[i]
// the byte step of axis i + 1.
bool make_map_nd(CUtensorMap *map, CUtensorMapDataType type, int rank, const void *base, const int64_t *dims,
                 const int64_t *strides_bytes, const uint32_t *box, CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn || rank < 1 || rank > 5)
        return false;
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = static_cast<cuuint64_t>(dims[i]);
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank)
            st[i] = static_cast<cuuint64_t>(strides_bytes[i]);
    }
    return fn(map, type, static_cast<cuuint32_t>(rank), const_cast<void *>(base), d, st, b, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kMaxDevices = 64;

int current_device()
{
    int device = 0;
    cudaGetDevice(&device);
    return device >= 0 && device < kMaxDevices ? device : 0;
}

int sm_count()
{
    static std::atomic<int> cache[kMaxDevices];
    const int device = current_device();
    int count = cache[device].load(std::memory_order_relaxed);
    if (count <= 0) {
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        count = count > 0 ? count : 148;
        cache[device].store(count, std::memory_order_relaxed);
    }
    return count;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
// Keyed by the kernel's address: template instances share a pointer type.
template <class Kernel>
cudaError_t ensure_smem(Kernel kernel, int bytes)
{
    static std::mutex lock;
    static std::set<std::pair<const void *, int>> done;
    const std::pair<const void *, int> key{reinterpret_cast<const void *>(kernel), current_device()};
    std::lock_guard<std::mutex> guard(lock);
    if (done.count(key))
        return cudaSuccess;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess)
        done.insert(key);
    return err;
}

// Launches fp8_gemm_kernel<BN, EPI, kPair> over p.num_tiles tiles with
// persistent CTAs (pairs).  maps: A, B, Y, codes, A of tap 1, A of tap 2.
template <int BN, int EPI, bool kPair>
cudaError_t launch_gemm_kernel(const CUtensorMap (&maps)[6], const gemm::Params &p, cudaStream_t stream)
{
    using C = gemm::Cfg<BN, EPI, kPair>;
    const int units = kPair ? sm_count() / 2 : sm_count(); // persistent CTAs (pairs)
    auto kernel = gemm::fp8_gemm_kernel<BN, EPI, kPair>;
    const cudaError_t attr = ensure_smem(kernel, C::kSmemBytes);
    if (attr != cudaSuccess)
        return attr;
    const int grid = std::min(p.num_tiles, units) * (kPair ? 2 : 1);
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(grid));
    config.blockDim = dim3(gemm::kThreads);
    config.dynamicSmemBytes = C::kSmemBytes;
    config.stream = stream;
    cudaLaunchAttribute attrs[2];
    int count = 0;
    attrs[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
    if (kPair) {
        attrs[count].id = cudaLaunchAttributeClusterDimension;
        attrs[count].val.clusterDim.x = 2;
        attrs[count].val.clusterDim.y = 1;
        attrs[count].val.clusterDim.z = 1;
        ++count;
    }
    config.attrs = attrs;
    config.numAttrs = count;
    const cudaError_t err =
        cudaLaunchKernelEx(&config, kernel, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

// M tiles per raster group of a plain linear (tile_coords).  Measured on B200:
// groups of 8 make the encoder's fc2 (A = 123 MB of codes per 16-stream slice,
// about the size of L2) 4% faster in the C4 forward and fc2 at M = 12000 (61 MB)
// 1% faster, but the linears whose A fits in L2 comfortably (15-31 MB) 2-3%
// slower; so only an A operand above 48 MB is grouped.  LFFW_GEMM_GROUP (tuning)
// forces a group size for every linear (0 = column by column), read once.
int gemm_group_m(int64_t a_bytes)
{
    static const int forced = [] {
        const char *v = std::getenv("LFFW_GEMM_GROUP");
        const int g = v ? std::atoi(v) : -1;
        return g >= 0 && g <= 1024 ? g : -1;
    }();
    if (forced >= 0)
        return forced;
    return a_bytes > (int64_t{48} << 20) ? 8 : 0;
}

template <int BN, int EPI, bool kPair>
cudaError_t run_gemm(const LinearLaunch &L, cudaStream_t stream)
{
    using C = gemm::Cfg<BN, EPI, kPair>;
    CUtensorMap maps[6] = {};
    CUtensorMap &tm_a = maps[0], &tm_b = maps[1], &tm_y = maps[2], &tm_c = maps[3];
    if (!make_map(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.x_codes, L.m, L.k, gemm::kBK, gemm::kBM,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.w_codes, L.n, L.k, gemm::kBK, C::kBRows,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    // Epilogue stores: one 32-row x 32-column box per warp and sub-chunk.
    if (C::kY && !make_map(&tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.y, L.m, L.n, gemm::kSub, 32,
                           CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    if (C::kCodes && !make_map(&tm_c, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.next_codes, L.m, L.n, gemm::kSub,
                               32, CU_TENSOR_MAP_SWIZZLE_32B))
        return cudaErrorInvalidValue;
    gemm::Params p{};
    p.m = static_cast<int>(L.m);
    p.n = static_cast<int>(L.n);
    p.k = static_cast<int>(L.k);
    p.m_tiles = static_cast<int>((L.m + C::kTileM - 1) / C::kTileM);
    const int n_tiles = static_cast<int>((L.n + BN - 1) / BN);
    p.num_tiles = p.m_tiles * n_tiles;
    p.n_tiles = n_tiles;
    p.group_m = gemm_group_m(L.m * L.k * (C::kF16In ? 2 : 1));
    p.num_kb = static_cast<int>((L.k + gemm::kBK - 1) / gemm::kBK);
    p.act_scale = L.act_scale;
    p.act_scale_ptr = L.act_scale_ptr;
    p.w_scales = L.w_scales;
    p.bias = L.bias;
    p.next_scale = L.next_scale;
    // Correctly rounded reciprocal: binary64 quotient, one rounding to binary32
    // (innocuous double rounding for division since 53 >= 2*24 + 2).
    p.next_recip = L.next_codes ? static_cast<float>(1.0 / static_cast<double>(L.next_scale)) : 0.0f;
    p.next_lean = L.next_codes && lean_scale(L.next_scale) ? 1 : 0;
    p.kb_per_tap = p.num_kb;
    if (C::kPos) {
        p.pos = L.residual;
        p.pos_ld = static_cast<int>(L.n);
    }
    return launch_gemm_kernel<BN, EPI, kPair>(maps, p, stream);
}

// Encoder convolution on fp16 tensor cores (see ConvLaunch).
template <bool kPair, bool kPos>
cudaError_t run_conv(const ConvLaunch &L, cudaStream_t stream)
{
    using namespace gemm;
    constexpr int BN = 256;
    constexpr int EPI = kEpiF16In | kEpiBiasF32 | kEpiGelu | kEpiY | kEpiSeg | (kPos ? kEpiPos : 0);
    using C = Cfg<BN, EPI, kPair>;
    const int64_t t_out = L.t_in / L.stride;
    const int64_t in_rows = static_cast<int64_t>(L.t_in) + 2;
    CUtensorMap maps[6] = {};
    // Tap j of output row t reads padded input row stride * t + j (row 0 and
    // row t_in + 1 of each stream are the zero padding).
    for (int j = 0; j < 3; ++j) {
        const int64_t dims[3] = {L.c_in, t_out, L.streams};
        const int64_t strides[2] = {static_cast<int64_t>(L.stride) * L.c_in * 2, in_rows * L.c_in * 2};
        const uint32_t box[3] = {static_cast<uint32_t>(C::kKElems), static_cast<uint32_t>(kBM), 1u};
        if (!make_map_nd(&maps[j == 0 ? 0 : 3 + j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                         L.x + static_cast<int64_t>(j) * L.c_in, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
    }
    if (!make_map(&maps[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.w, L.c_out, 3 * static_cast<int64_t>(L.c_in),
                  C::kKElems, C::kBRows, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    {
        const int64_t dims[3] = {L.c_out, t_out, L.streams};
        const int64_t strides[2] = {static_cast<int64_t>(L.c_out) * 2, static_cast<int64_t>(L.y_rows) * L.c_out * 2};
        const uint32_t box[3] = {static_cast<uint32_t>(kSub), 32u, 1u};
        if (!make_map_nd(&maps[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                         L.y + static_cast<int64_t>(L.y_row0) * L.c_out, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
    }
    Params p{};
    p.m = static_cast<int>(t_out * L.streams);
    p.n = L.c_out;
    p.k = 3 * L.c_in;
    p.seg_rows = static_cast<int>(t_out);
    p.seg_tiles = static_cast<int>((t_out + C::kTileM - 1) / C::kTileM);
    p.m_tiles = p.seg_tiles * L.streams;
    p.num_tiles = p.m_tiles * ((L.c_out + BN - 1) / BN);
    p.kb_per_tap = L.c_in / C::kKElems;
    p.num_kb = 3 * p.kb_per_tap;
    p.act_scale = 1.0f;
    p.bias = L.bias;
    p.pos = L.pos;
    p.pos_ld = L.c_out;
    return launch_gemm_kernel<BN, EPI, kPair>(maps, p, stream);
}

// FP8 linear with a head-split fp16 output (see HeadsLinearLaunch).
template <bool kPair>
cudaError_t run_linear_heads(const HeadsLinearLaunch &L, cudaStream_t stream)
{
    using namespace gemm;
    constexpr int BN = 256;
    constexpr int EPI = kEpiY | kEpiSeg | kEpiHeads;
    using C = Cfg<BN, EPI, kPair>;
    CUtensorMap maps[6] = {};
    {
        const int64_t dims[3] = {L.k, L.tokens, L.streams};
        const int64_t strides[2] = {L.k, static_cast<int64_t>(L.tokens) * L.k};
        const uint32_t box[3] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(kBM), 1u};
        if (!make_map_nd(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, L.x_codes, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
    }
    if (!make_map(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.w_codes, L.n, L.k, kBK, C::kBRows,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    {
        const int64_t groups = L.n / (64 * static_cast<int64_t>(L.heads));
        const int64_t dims[5] = {64, L.tokens, L.heads, L.streams, groups};
        const int64_t head = static_cast<int64_t>(L.tokens) * 64 * 2;
        const int64_t strides[4] = {128, head, head * L.heads, head * L.heads * L.y_streams};
        const uint32_t box[5] = {static_cast<uint32_t>(kSub), 32u, 1u, 1u, 1u};
        if (!make_map_nd(&maps[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, L.y, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
    }
    Params p{};
    p.m = L.tokens * L.streams;
    p.n = static_cast<int>(L.n);
    p.k = static_cast<int>(L.k);
    p.seg_rows = L.tokens;
    p.seg_tiles = (L.tokens + C::kTileM - 1) / C::kTileM;
    p.m_tiles = p.seg_tiles * L.streams;
    p.num_tiles = p.m_tiles * static_cast<int>((L.n + BN - 1) / BN);
    p.num_kb = static_cast<int>((L.k + kBK - 1) / kBK);
    p.kb_per_tap = p.num_kb;
    p.heads = L.heads;
    p.act_scale = L.act_scale;
    p.act_scale_ptr = L.act_scale_ptr;
    p.w_scales = L.w_scales;
    p.bias = L.bias;
    return launch_gemm_kernel<BN, EPI, kPair>(maps, p, stream);
}

template <int BN, bool kPair>
cudaError_t run_gemm_epilogue(const LinearLaunch &L, cudaStream_t stream)
{
    using namespace gemm;
    const int epi = (L.gelu ? kEpiGelu : 0) | (L.y ? kEpiY : 0) | (L.next_codes ? kEpiCodes : 0) |
                    (L.residual ? kEpiPos : 0);
    switch (epi) {
    case kEpiY: return run_gemm<BN, kEpiY, kPair>(L, stream);
    case kEpiY | kEpiPos: return run_gemm<BN, kEpiY | kEpiPos, kPair>(L, stream);
    case kEpiCodes: return run_gemm<BN, kEpiCodes, kPair>(L, stream);
    case kEpiY | kEpiCodes: return run_gemm<BN, kEpiY | kEpiCodes, kPair>(L, stream);
    case kEpiGelu | kEpiY: return run_gemm<BN, kEpiGelu | kEpiY, kPair>(L, stream);
    case kEpiGelu | kEpiCodes: return run_gemm<BN, kEpiGelu | kEpiCodes, kPair>(L, stream);
    case kEpiGelu | kEpiY | kEpiCodes: return run_gemm<BN, kEpiGelu | kEpiY | kEpiCodes, kPair>(L, stream);
    default: return cudaErrorInvalidValue;
    }
}


} // namespace

// LFFW_GEMM_TILE overrides the tile choice (tuning): "1x256", "1x128",
// "2x256", "2x128" = CTAs per tile x tile width.  Read once per process.
int tile_override()
{
    static const int mode = [] {
        const char *v = std::getenv("LFFW_GEMM_TILE");
        if (v == nullptr)
            return 0;
        const std::string s(v);
        return s == "1x256" ? 1 : s == "1x128" ? 2 : s == "2x256" ? 3 : s == "2x128" ? 4 : 0;
    }();
    return mode;
}

cudaError_t launch_conv_gelu(const ConvLaunch &L, cudaStream_t stream)
{
    // CTA pairs for long K (the 1280-channel convolution, K = 3840), as for the linears.
    const bool pair = 3 * static_cast<int64_t>(L.c_in) >= 1024 && static_cast<int64_t>(L.t_in) * L.streams >= 512;
    if (pair)
        return L.pos ? run_conv<true, true>(L, stream) : run_conv<true, false>(L, stream);
    return L.pos ? run_conv<false, true>(L, stream) : run_conv<false, false>(L, stream);
}

cudaError_t launch_fp8_linear_heads(const HeadsLinearLaunch &L, cudaStream_t stream)
{
    const bool pair = L.k >= 1024 && static_cast<int64_t>(L.tokens) * L.streams >= 512;
    return pair ? run_linear_heads<true>(L, stream) : run_linear_heads<false>(L, stream);
}

cudaError_t launch_fp8_gemm(const LinearLaunch &L, cudaStream_t stream)
{
    switch (tile_override()) {
    case 1: return run_gemm_epilogue<256, false>(L, stream);
    case 2: return run_gemm_epilogue<128, false>(L, stream);
    case 3: return run_gemm_epilogue<256, true>(L, stream);
    case 4: return run_gemm_epilogue<128, true>(L, stream);
    default: break;
    }
    // Measured on B200 (C2 shapes, M = 12000): 256-wide tiles beat 128-wide ones
    // by ~30% even where 128 would fill the last wave better.  CTA pairs (256-row
    // tiles, half the B traffic per SM, six stages instead of four) feed the MMA
    // better: +12% for K = 5120, +3-4% for K = 1280 with fp16 outputs.  Not for the
    // GELU code-table epilogue (E4M3 codes as the only output): there the faster
    // main loop leaves the MMA waiting on the epilogue (-5%).
    const bool code_table = L.gelu && L.next_codes != nullptr && L.y == nullptr;
    const bool pair = L.m >= 512 && L.k >= 1024 && !code_table;
    // Tile width 224 or 256: fewer, fuller waves at a narrower tile.  A tile's time
    // is ~0.44 fixed + 0.56 x width/256 of a 256-wide one (measured from 128- and
    // 256-wide tiles), so the estimate is waves x that.  N = 1280 (out_proj, fc2):
    // 470 tiles = 3.18 waves at 256, 564 = 3.81 waves at 224.
    const int64_t units = pair ? sm_count() / 2 : sm_count();
    const int64_t m_tiles = (L.m + (pair ? 255 : 127)) / (pair ? 256 : 128);
    auto cost = [&](int bn) {
        const int64_t tiles = m_tiles * ((L.n + bn - 1) / bn);
        return static_cast<double>((tiles + units - 1) / units) * (0.44 + 0.56 * bn / 256.0);
    };
    const bool narrow = cost(224) < cost(256);
    if (pair)
        return narrow ? run_gemm_epilogue<224, true>(L, stream) : run_gemm_epilogue<256, true>(L, stream);
    return narrow ? run_gemm_epilogue<224, false>(L, stream) : run_gemm_epilogue<256, false>(L, stream);
}

namespace {

// Cluster size (CTAs sharing one 128-row block, splitting K): enough CTAs for
// about two per SM, a power of two, at most `max_cluster` and at most the
// number of K blocks.
int skinny_cluster(int64_t n, int num_kb, int max_cluster)
{
    const int64_t blocks = (n + skinny::kRows - 1) / skinny::kRows;
    const int64_t want = (2 * static_cast<int64_t>(sm_count()) + blocks - 1) / blocks;
    int s = 1;
    while (s < want && s * 2 <= max_cluster && s * 2 <= num_kb)
        s *= 2;
    return s;
}

// Largest cluster size the skinny kernel uses: 8 (measured on B200, 16-CTA
// clusters reduce slower than they stream), or the LFFW_SKINNY_MAX_CLUSTER
// tuning override (1 to 8), read once.
int skinny_max_cluster()
{
    static const int value = [] {
        const char *cap = std::getenv("LFFW_SKINNY_MAX_CLUSTER");
        const int v = cap ? std::atoi(cap) : 0;
        return v >= 1 && v <= skinny::kMaxCluster ? v : skinny::kMaxCluster;
    }();
    return value;
}

template <int KIND, int EPI>
cudaError_t run_skinny(const void *x, const void *w, int64_t m, int64_t n, int64_t k, const LinearLaunch &L,
                       cudaStream_t stream, bool packed)
{
    const int elem = KIND == skinny::kKindF16 ? 2 : 1;
    const CUtensorMapDataType type = KIND == skinny::kKindF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUtensorMap tm_w{}, tm_x{};
    if ((!packed && !make_map(&tm_w, type, elem, w, n, k, skinny::kBK / elem, skinny::kRows,
                              CU_TENSOR_MAP_SWIZZLE_128B)) ||
        !make_map(&tm_x, type, elem, x, m, k, skinny::kBK / elem, skinny::kAct, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    skinny::Params p{};
    p.m = static_cast<int>(m);
    p.n = static_cast<int>(n);
    p.num_kb = static_cast<int>((k * elem + skinny::kBK - 1) / skinny::kBK);
    p.cluster = skinny_cluster(n, p.num_kb, skinny_max_cluster());
    p.act_scale = L.act_scale;
    p.act_scale_ptr = L.act_scale_ptr;
    p.w_scales = L.w_scales;
    p.bias = L.bias;
    p.y = L.y;
    p.next_scale = L.next_scale;
    p.next_recip = L.next_codes ? static_cast<float>(1.0 / static_cast<double>(L.next_scale)) : 0.0f;
    p.next_codes = L.next_codes;
    p.w_packed = packed ? static_cast<const uint8_t *>(w) : nullptr;
    const int64_t blocks = (n + skinny::kRows - 1) / skinny::kRows;
    const int64_t grid = blocks * p.cluster;
    const int per_cta = (p.num_kb + p.cluster - 1) / p.cluster;
    // A grid of at most one CTA per SM whose CTAs own more K blocks than the
    // shallow ring holds takes the deep ring.
    const bool deep = grid <= sm_count() && per_cta > skinny::kShallow;
    auto kernel = deep ? skinny::skinny_kernel<KIND, EPI, skinny::kDeep> : skinny::skinny_kernel<KIND, EPI, skinny::kShallow>;
    const int base = deep ? skinny::Ring<skinny::kDeep>::kSmemBase : skinny::Ring<skinny::kShallow>::kSmemBase;
    const int smem = base + (p.cluster > 1 ? skinny::recv_bytes(p.m) : 0);
    const cudaError_t attr = ensure_smem(kernel, base + skinny::recv_bytes(skinny::kAct));
    if (attr != cudaSuccess)
        return attr;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(grid));
    config.blockDim = dim3(skinny::kThreads);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attrs[2];
    int count = 0;
    attrs[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
    if (p.cluster > 1) {
        attrs[count].id = cudaLaunchAttributeClusterDimension;
        attrs[count].val.clusterDim.x = static_cast<unsigned>(p.cluster);
        attrs[count].val.clusterDim.y = 1;
        attrs[count].val.clusterDim.z = 1;
        ++count;
    }
    config.attrs = attrs;
    config.numAttrs = count;
    const cudaError_t err = cudaLaunchKernelEx(&config, kernel, tm_w, tm_x, p);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

} // namespace

cudaError_t launch_fp8_skinny(const LinearLaunch &L, cudaStream_t stream)
{
    if (L.gelu)
        return run_skinny<skinny::kKindE4M3, 1>(L.x_codes, L.w_codes, L.m, L.n, L.k, L, stream, L.w_packed);
    return run_skinny<skinny::kKindE4M3, 0>(L.x_codes, L.w_codes, L.m, L.n, L.k, L, stream, L.w_packed);
}

cudaError_t launch_fp16_skinny(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y, int64_t m,
                               int64_t n, int64_t k, bool packed, cudaStream_t stream)
{
    LinearLaunch L{};
    L.m = m;
    L.n = n;
    L.k = k;
    L.bias = bias;
    L.y = y;
    return run_skinny<skinny::kKindF16, 0>(x, w, m, n, k, L, stream, packed);
}

int64_t skinny_packed_bytes(int64_t n, int64_t row_bytes)
{
    const int64_t blocks = (n + skinny::kRows - 1) / skinny::kRows;
    const int64_t kbs = (row_bytes + skinny::kBK - 1) / skinny::kBK;
    return blocks * kbs * skinny::kWBytes;
}

cudaError_t launch_pack_skinny(const void *w, int64_t n, int64_t row_bytes, void *packed, cudaStream_t stream)
{
    const int64_t kbs = (row_bytes + skinny::kBK - 1) / skinny::kBK;
    const int64_t chunks = skinny_packed_bytes(n, row_bytes) / 16;
    skinny::pack_kernel<<<static_cast<unsigned>((chunks + 255) / 256), 256, 0, stream>>>(
        static_cast<const uint8_t *>(w), n, row_bytes, kbs, static_cast<uint8_t *>(packed));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize(const uint16_t *x, int64_t count, float scale, const float *scale_ptr,
                            uint8_t *codes, cudaStream_t stream)
{
    const int64_t chunks = count / quant::kQuantChunk;
    const int64_t warps_per_block = quant::kThreads / 32;
    int64_t blocks = (chunks + warps_per_block - 1) / warps_per_block;
    // Four blocks (32 warps) per SM, each warp looping over chunks with the next
    // chunk's loads in flight.
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(sm_count()) * 4));
    const float recip = static_cast<float>(1.0 / static_cast<double>(scale));
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(blocks));
    config.blockDim = dim3(quant::kThreads);
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, quant::quantize_kernel, x, count, scale, recip, scale_ptr, codes);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_layer_norm(const LayerNormLaunch &L, cudaStream_t stream)
{
    norm::Params p{};
    p.rows = static_cast<int>(L.rows);
    p.cols = static_cast<int>(L.cols);
    p.x = L.x;
    p.residual = L.residual;
    p.sum_out = L.sum_out;
    p.gamma = L.gamma;
    p.beta = L.beta;
    p.eps = L.eps;
    p.y = L.y;
    p.code_scale = L.code_scale;
    p.code_recip = L.codes && !L.code_scale_ptr ? static_cast<float>(1.0 / static_cast<double>(L.code_scale)) : 0.0f;
    p.code_scale_ptr = L.code_scale_ptr;
    p.codes = L.codes;
    const int per_lane = static_cast<int>((L.cols / 8 + 31) / 32);
    cudaLaunchConfig_t config{};
    const int64_t row_blocks = (L.rows + norm::kRowsPerBlock - 1) / norm::kRowsPerBlock;
    config.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(row_blocks, static_cast<int64_t>(sm_count()) * 4)));
    config.blockDim = dim3(norm::kThreads);
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    config.dynamicSmemBytes = static_cast<size_t>(L.cols) * 8; // gamma and beta
    const bool codes_only = L.residual == nullptr && L.sum_out == nullptr && L.y == nullptr && L.codes != nullptr;
    auto launch = [&](auto kernel) {
        cudaError_t e = ensure_smem(kernel, 4096 * 8);
        return e != cudaSuccess ? e : cudaLaunchKernelEx(&config, kernel, p);
    };
    cudaError_t err;
    if (per_lane <= 2)
        err = codes_only ? launch(norm::layer_norm_kernel<2, true>) : launch(norm::layer_norm_kernel<2, false>);
    else if (per_lane <= 5)
        err = codes_only ? launch(norm::layer_norm_kernel<5, true>) : launch(norm::layer_norm_kernel<5, false>);
    else if (per_lane <= 8)
        err = codes_only ? launch(norm::layer_norm_kernel<8, true>) : launch(norm::layer_norm_kernel<8, false>);
    else
        err = codes_only ? launch(norm::layer_norm_kernel<16, true>) : launch(norm::layer_norm_kernel<16, false>);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_cross_attention(const CrossAttentionLaunch &L, cudaStream_t stream)
{
    attn::Params p{};
    p.streams = L.streams;
    p.queries = L.queries;
    p.heads = L.heads;
    p.keys = L.keys;
    // CTAs per (stream, head) and ring depth: the most CTAs (each keeping at
    // least 128 keys) that run in one wave given how many fit an SM's shared
    // memory, the deeper ring when both depths fit.
    const int pairs = L.streams * L.heads;
    auto kpc_for = [&](int cl) { return ((L.keys + cl - 1) / cl + 15) / 16 * 16; };
    auto per_sm = [&](int cl, int st) {
        const int bytes = attn::smem_bytes(st, L.queries, kpc_for(cl) + 8, cl) + 1024; // + the per-CTA reserve
        return std::max(1, 233472 / bytes);
    };
    int S = 1, stages = attn::kMaxStages;
    for (int cl = 1; cl <= attn::kMaxCluster; cl *= 2) {
        if (cl > 1 && (L.keys + cl - 1) / cl < attn::kChunk)
            break;
        if (kpc_for(cl) > kAttentionMaxKeysPerCta)
            continue;
        for (int st = attn::kMaxStages; st >= 3; --st)
            if (static_cast<int64_t>(pairs) * cl <= static_cast<int64_t>(per_sm(cl, st)) * sm_count()) {
                S = cl;
                stages = st;
                break;
            }
    }
    while (kpc_for(S) > kAttentionMaxKeysPerCta && S < attn::kMaxCluster)
        S *= 2;
    p.cluster = S;
    p.stages = stages;
    p.kpc = ((L.keys + S - 1) / S + 15) / 16 * 16;
    p.pstride = p.kpc + 8;
    p.score_bytes = attn::score_bytes(L.queries, p.pstride);
    p.xch_bytes = attn::xch_bytes(L.queries, S);
    p.q = L.q;
    p.out = L.out;
    const uint16_t c = __half_as_ushort(__float2half_rn(static_cast<float>(std::pow(double(attn::kDim), -0.25))));
    p.scale2 = static_cast<uint32_t>(c) * 0x10001u;
    p.code_scale = L.code_scale;
    p.code_recip = L.codes && !L.code_scale_ptr ? static_cast<float>(1.0 / static_cast<double>(L.code_scale)) : 0.0f;
    p.code_scale_ptr = L.code_scale_ptr;
    p.codes = L.codes;
    const int64_t rows = static_cast<int64_t>(L.streams) * L.heads * L.keys;
    CUtensorMap tm_k{}, tm_v{};
    if (!make_map(&tm_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.k, rows, attn::kDim, attn::kDim, attn::kChunk,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tm_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.v, rows, attn::kDim, attn::kDim, attn::kChunk,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const int smem = attn::smem_bytes(p.stages, L.queries, p.pstride, S);
    // The attribute is set once, for the largest shared memory the launcher picks.
    constexpr int kMaxSmem =
        attn::smem_bytes(attn::kMaxStages, attn::kMaxQueries, kAttentionMaxKeysPerCta + 8, attn::kMaxCluster);
    static_assert(kMaxSmem <= 232448, "shared memory budget");
    const cudaError_t attr = ensure_smem(attn::cross_attention_kernel, kMaxSmem);
    if (attr != cudaSuccess)
        return attr;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(pairs * S));
    config.blockDim = dim3(attn::kThreads);
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attrs[2];
    int count = 0;
    attrs[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
    if (S > 1) {
        attrs[count].id = cudaLaunchAttributeClusterDimension;
        attrs[count].val.clusterDim.x = static_cast<unsigned>(S);
        attrs[count].val.clusterDim.y = 1;
        attrs[count].val.clusterDim.z = 1;
        ++count;
    }
    config.attrs = attrs;
    config.numAttrs = count;
    const cudaError_t err = cudaLaunchKernelEx(&config, attn::cross_attention_kernel, tm_k, tm_v, p);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_self_attention(const SelfAttentionLaunch &L, cudaStream_t stream)
{
    sattn::Params p{};
    p.streams = L.streams;
    p.tokens = L.tokens;
    p.heads = L.heads;
    p.qblocks = (L.tokens + sattn::kBQ - 1) / sattn::kBQ;
    p.qpairs = (p.qblocks + 1) / 2;
    p.nchunks = (L.tokens + sattn::kChunk - 1) / sattn::kChunk;
    p.out = L.out;
    const uint16_t c = __half_as_ushort(__float2half_rn(static_cast<float>(std::pow(double(sattn::kDim), -0.25))));
    p.scale2 = static_cast<uint32_t>(c) * 0x10001u;
    p.code_scale = L.code_scale;
    p.code_recip = L.codes && !L.code_scale_ptr ? static_cast<float>(1.0 / static_cast<double>(L.code_scale)) : 0.0f;
    p.code_scale_ptr = L.code_scale_ptr;
    p.codes = L.codes;
    const int64_t rows = static_cast<int64_t>(L.streams) * L.tokens;
    const int64_t width = static_cast<int64_t>(L.heads) * sattn::kDim;
    CUtensorMap tm_q{}, tm_k{}, tm_v{};
    if (!make_map_ld(&tm_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.q, rows, width, L.q_ld, sattn::kDim, sattn::kBQ,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_ld(&tm_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.k, rows, width, L.k_ld, sattn::kDim,
                     sattn::kChunk, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_ld(&tm_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, L.v, rows, width, L.v_ld, sattn::kDim,
                     sattn::kChunk, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const cudaError_t attr = ensure_smem(fattn::attention_kernel, fattn::kSmemBytes);
    if (attr != cudaSuccess)
        return attr;
    cudaLaunchConfig_t config{};
    // Persistent: one CTA per SM walks the (stream, head, query-tile pair) items.
    const int64_t items = static_cast<int64_t>(L.streams) * L.heads * p.qpairs;
    config.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(items, sm_count())));
    config.blockDim = dim3(fattn::kThreads);
    config.dynamicSmemBytes = fattn::kSmemBytes;
    config.stream = stream;
    cudaLaunchAttribute attr_pdl[1];
    attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr_pdl;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, fattn::attention_kernel, tm_q, tm_k, tm_v, p);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

struct ChainPlan {
    void *device = nullptr; // [global maps][links][units][first][counters][partials]
    std::vector<CUtensorMap> maps; // distinct activation maps
    const CUtensorMap *global_maps = nullptr; // set when there are more than kParamMaps
    const chain::Link *links = nullptr;
    const chain::Unit *units = nullptr;
    const int *first = nullptr;
    unsigned int *counters = nullptr; // done per link, then arrivals per split row block
    size_t counter_bytes = 0;
    int count = 0, m = 0, ctas = 0, device_id = 0;
};

cudaError_t chain_create(const LinearLaunch *links, int count, ChainPlan **plan)
{
    using chain::kAct;
    using chain::kRows;
    *plan = nullptr;
    std::vector<CUtensorMap> maps; // one per distinct (activation buffer, m, k)
    std::vector<std::tuple<const void *, int64_t, int64_t>> map_keys;
    std::vector<chain::Link> host(static_cast<size_t>(count));
    std::vector<chain::Unit> all;
    size_t arrivals = 0, partial_floats = 0;
    for (int i = 0; i < count; ++i) {
        const LinearLaunch &L = links[i];
        const auto key = std::make_tuple(static_cast<const void *>(L.x_codes), L.m, L.k);
        int map = static_cast<int>(std::find(map_keys.begin(), map_keys.end(), key) - map_keys.begin());
        if (map == static_cast<int>(map_keys.size())) {
            CUtensorMap tm{};
            if (!make_map(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, L.x_codes, L.m, L.k, skinny::kBK, skinny::kAct,
                          CU_TENSOR_MAP_SWIZZLE_128B))
                return cudaErrorInvalidValue;
            map_keys.push_back(key);
            maps.push_back(tm);
        }
        chain::Link &c = host[i];
        c.map = map;
        c.w = L.w_codes;
        c.w_scales = L.w_scales;
        c.bias = L.bias;
        c.act_scale_ptr = L.act_scale_ptr;
        c.y = L.y;
        c.codes = L.next_codes;
        c.n = static_cast<int>(L.n);
        c.num_kb = static_cast<int>((L.k + skinny::kBK - 1) / skinny::kBK);
        // K slices of at most kMaxUnitKb tiles, none empty.
        const int want = (c.num_kb + chain::kMaxUnitKb - 1) / chain::kMaxUnitKb;
        c.slice_kb = (c.num_kb + want - 1) / want;
        c.split = (c.num_kb + c.slice_kb - 1) / c.slice_kb;
        c.gelu = L.gelu ? 1 : 0;
        c.act_scale = L.act_scale;
        c.next_scale = L.next_scale;
        c.next_recip = L.next_codes ? static_cast<float>(1.0 / static_cast<double>(L.next_scale)) : 0.0f;
        const int blocks = (c.n + kRows - 1) / kRows;
        if (c.split > 1) {
            arrivals += static_cast<size_t>(blocks);
            // One workspace for every split link: link i's slices run only after
            // every earlier link has finished reading its partials.
            partial_floats = std::max(partial_floats, static_cast<size_t>(blocks) * c.split * kAct * kRows);
        }
        for (int b = 0; b < blocks; ++b)
            for (int s = 0; s < c.split; ++s)
                all.push_back(chain::Unit{i, b, s * c.slice_kb, std::min((s + 1) * c.slice_kb, c.num_kb)});
    }
    cudaError_t err = ensure_smem(chain::chain_kernel, chain::kSmemBytes);
    if (err != cudaSuccess)
        return err;
    // One CTA per SM, all resident: a CTA waits only for units of earlier links,
    // which sit earlier in every CTA's list.
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain::chain_kernel, chain::kThreads,
                                                        chain::kSmemBytes);
    if (err != cudaSuccess || per_sm < 1)
        return err != cudaSuccess ? err : cudaErrorInvalidConfiguration;
    const int ctas = static_cast<int>(std::min<size_t>(static_cast<size_t>(sm_count()), all.size()));
    // Round-robin in chain order: CTA c takes units c, c + ctas, ...
    std::vector<chain::Unit> units;
    units.reserve(all.size());
    std::vector<int> first(static_cast<size_t>(ctas) + 1, 0);
    for (int c = 0; c < ctas; ++c) {
        first[c] = static_cast<int>(units.size());
        for (size_t u = static_cast<size_t>(c); u < all.size(); u += static_cast<size_t>(ctas))
            units.push_back(all[u]);
    }
    first[ctas] = static_cast<int>(units.size());
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = (off + bytes + 255) / 256 * 256;
        return at;
    };
    const bool param_maps = maps.size() <= static_cast<size_t>(chain::kParamMaps);
    const size_t o_maps = take(param_maps ? 0 : sizeof(CUtensorMap) * maps.size());
    const size_t o_links = take(sizeof(chain::Link) * host.size());
    const size_t o_units = take(sizeof(chain::Unit) * units.size());
    const size_t o_first = take(sizeof(int) * first.size());
    const size_t counter_bytes = sizeof(unsigned int) * (static_cast<size_t>(count) + arrivals);
    const size_t o_counters = take(counter_bytes);
    const size_t o_partials = take(sizeof(float) * partial_floats);
    auto *plan_ptr = new (std::nothrow) ChainPlan();
    if (!plan_ptr)
        return cudaErrorMemoryAllocation;
    err = cudaMalloc(&plan_ptr->device, off);
    if (err != cudaSuccess) {
        delete plan_ptr;
        return err;
    }
    auto *base = static_cast<uint8_t *>(plan_ptr->device);
    auto *counters = reinterpret_cast<unsigned int *>(base + o_counters);
    size_t next_arrival = static_cast<size_t>(count);
    for (chain::Link &c : host)
        if (c.split > 1) {
            c.partials = reinterpret_cast<float *>(base + o_partials);
            c.arrivals = counters + next_arrival;
            next_arrival += static_cast<size_t>((c.n + kRows - 1) / kRows);
        }
    if (!param_maps)
        err = cudaMemcpy(base + o_maps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(base + o_links, host.data(), sizeof(chain::Link) * host.size(), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(base + o_units, units.data(), sizeof(chain::Unit) * units.size(), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(base + o_first, first.data(), sizeof(int) * first.size(), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(plan_ptr->device);
        delete plan_ptr;
        return err;
    }
    plan_ptr->maps = std::move(maps);
    plan_ptr->global_maps = param_maps ? nullptr : reinterpret_cast<const CUtensorMap *>(base + o_maps);
    plan_ptr->links = reinterpret_cast<const chain::Link *>(base + o_links);
    plan_ptr->units = reinterpret_cast<const chain::Unit *>(base + o_units);
    plan_ptr->first = reinterpret_cast<const int *>(base + o_first);
    plan_ptr->counters = counters;
    plan_ptr->counter_bytes = counter_bytes;
    plan_ptr->count = count;
    plan_ptr->m = static_cast<int>(links[0].m);
    plan_ptr->ctas = ctas;
    plan_ptr->device_id = current_device();
    *plan = plan_ptr;
    return cudaSuccess;
}

cudaError_t chain_run(const ChainPlan *plan, cudaStream_t stream)
{
    if (current_device() != plan->device_id)
        return cudaErrorInvalidDevice; // descriptors live on the creating device
    cudaError_t err = cudaMemsetAsync(plan->counters, 0, plan->counter_bytes, stream);
    if (err != cudaSuccess)
        return err;
    chain::Params p{};
    if (plan->global_maps == nullptr)
        std::copy(plan->maps.begin(), plan->maps.end(), p.maps);
    p.global_maps = plan->global_maps;
    p.links = plan->links;
    p.units = plan->units;
    p.first = plan->first;
    p.done = plan->counters;
    p.m = plan->m;
    // CTAs wait on each other's completion counters, so all of them must be
    // resident at once: a cooperative launch guarantees that, or fails with
    // cudaErrorCooperativeLaunchTooLarge instead of stalling on a CTA that
    // never becomes resident (another context holding SMs, for example).
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(plan->ctas));
    config.blockDim = dim3(chain::kThreads);
    config.dynamicSmemBytes = chain::kSmemBytes;
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    err = cudaLaunchKernelEx(&config, chain::chain_kernel, p);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

void chain_destroy(ChainPlan *plan)
{
    if (!plan)
        return;
    cudaFree(plan->device);
    delete plan;
}

cudaError_t launch_quantize_rows(const uint16_t *w, int64_t rows, int64_t cols, const float *scales,
                                 uint8_t *codes, cudaStream_t stream)
{
    const int64_t yblocks = std::min<int64_t>((cols + quant::kThreads - 1) / quant::kThreads, 16);
    const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(yblocks));
    quant::quantize_rows_kernel<<<grid, quant::kThreads, 0, stream>>>(w, cols, scales, codes);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_weight_scales(const uint16_t *w, int64_t rows, int64_t cols, float *scales,
                                 cudaStream_t stream)
{
    quant::weight_scales_kernel<<<static_cast<unsigned>(rows), quant::kThreads, 0, stream>>>(w, cols, scales);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_dynamic_scale(const uint16_t *x, int64_t count, float *scale, float *amax_out,
                                 cudaStream_t stream)
{
    cudaError_t err = cudaMemsetAsync(scale, 0, sizeof(float), stream);
    if (err != cudaSuccess)
        return err;
    int64_t blocks = (count + quant::kThreads - 1) / quant::kThreads;
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(sm_count()) * 4));
    quant::amax_kernel<<<static_cast<unsigned>(blocks), quant::kThreads, 0, stream>>>(
        x, count, reinterpret_cast<int *>(scale));
    count_launch();
    quant::finalize_scale_kernel<<<1, 1, 0, stream>>>(scale, amax_out);
    count_launch();
    return cudaGetLastError();
}

// The slab kernel for the plugins' projections: `rows` weight rows of `width`
// halves split into one run per SM (fewer rows per CTA when a run would exceed
// kSlabMaxBytes), launched with programmatic stream serialisation.
template <bool kFc1>
cudaError_t launch_projection_slab(const uint16_t *x, const uint16_t *w, const uint16_t *b0, const uint16_t *b1,
                                   uint16_t *y, int64_t rows, int64_t width, cudaStream_t stream)
{
    const int64_t row_bytes = width * 2;
    const int64_t cap = proj::kSlabMaxBytes / (row_bytes + 4); // weight row + staged bias word
    // About three CTAs per SM: more warps hide the fold's latency, and smaller
    // CTAs leave room for the next launch's copies.
    const int64_t ctas = 3 * static_cast<int64_t>(sm_count());
    const int64_t per_cta = std::max<int64_t>(1, std::min<int64_t>(cap, (rows + ctas - 1) / ctas));
    const int64_t chunk_rows = (per_cta + proj::kSlabChunks - 1) / proj::kSlabChunks;
    const unsigned grid = static_cast<unsigned>((rows + per_cta - 1) / per_cta);
    const int smem = static_cast<int>(per_cta * (row_bytes + 4));
    int depth = 128;
    while (depth < width)
        depth *= 2;
    auto pick = [&](auto kernel) -> cudaError_t {
        cudaError_t err = ensure_smem(kernel, proj::kSlabSmemBytes);
        if (err != cudaSuccess)
            return err;
        cudaLaunchConfig_t config{};
        config.gridDim = dim3(grid);
        config.blockDim = dim3(proj::kSlabThreads);
        config.dynamicSmemBytes = static_cast<size_t>(smem);
        config.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        config.attrs = attr;
        config.numAttrs = 1;
        err = cudaLaunchKernelEx(&config, kernel, x, w, b0, b1, y, static_cast<int>(rows), static_cast<int>(width),
                                 static_cast<int>(per_cta), static_cast<int>(chunk_rows));
        count_launch();
        return err != cudaSuccess ? err : cudaGetLastError();
    };
    // Whisper's widths (384, 512, 768, 1024, 1280) have every column group full.
    switch (width) {
    case 384: return pick(proj::fp16_projection_slab_kernel<16, 3, kFc1>);
    case 512: return pick(proj::fp16_projection_slab_kernel<16, 4, kFc1>);
    case 768: return pick(proj::fp16_projection_slab_kernel<32, 6, kFc1>);
    case 1024: return pick(proj::fp16_projection_slab_kernel<32, 8, kFc1>);
    case 1280: return pick(proj::fp16_projection_slab_kernel<64, 10, kFc1>);
    default: break;
    }
    switch (depth) {
    case 128: return pick(proj::fp16_projection_slab_kernel<4, 0, kFc1>);
    case 256: return pick(proj::fp16_projection_slab_kernel<8, 0, kFc1>);
    case 512: return pick(proj::fp16_projection_slab_kernel<16, 0, kFc1>);
    case 1024: return pick(proj::fp16_projection_slab_kernel<32, 0, kFc1>);
    case 2048: return pick(proj::fp16_projection_slab_kernel<64, 0, kFc1>);
    default: return pick(proj::fp16_projection_slab_kernel<128, 0, kFc1>);
    }
}

cudaError_t launch_fp16_fc1(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                            int64_t rows, int64_t width, cudaStream_t stream)
{
    if (width <= proj::kSlabMaxWidth)
        return launch_projection_slab<true>(x, w, bias, nullptr, y, rows, width, stream);
    const int64_t per_block = proj::kThreads / 32;
    const unsigned blocks = static_cast<unsigned>((rows + per_block - 1) / per_block);
    proj::fp16_projection_kernel<true><<<blocks, proj::kThreads, 0, stream>>>(
        x, w, bias, nullptr, y, static_cast<int>(rows), static_cast<int>(width));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_fp16_qkv(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                            const uint16_t *v_bias, uint16_t *y, int64_t width, cudaStream_t stream)
{
    const int64_t rows = 3 * width;
    if (width <= proj::kSlabMaxWidth)
        return launch_projection_slab<false>(x, w, q_bias, v_bias, y, rows, width, stream);
    const int64_t per_block = proj::kThreads / 32;
    const unsigned blocks = static_cast<unsigned>((rows + per_block - 1) / per_block);
    proj::fp16_projection_kernel<false><<<blocks, proj::kThreads, 0, stream>>>(
        x, w, q_bias, v_bias, y, static_cast<int>(rows), static_cast<int>(width));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_fp16_bias(const uint16_t *x, uint16_t bias, uint16_t *y, int64_t count,
                             cudaStream_t stream)
{
    int64_t blocks = (count + proj::kThreads - 1) / proj::kThreads;
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(sm_count()) * 16));
    proj::fp16_bias_kernel<<<static_cast<unsigned>(blocks), proj::kThreads, 0, stream>>>(
        x, bias, y, static_cast<uint32_t>(count));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_mel_frames(const float *mel, int streams, int mels, int frames, uint16_t *x, cudaStream_t stream)
{
    const dim3 grid(static_cast<unsigned>((frames + front::kTile - 1) / front::kTile),
                    static_cast<unsigned>((mels + front::kTile - 1) / front::kTile), static_cast<unsigned>(streams));
    front::mel_frames_kernel<<<grid, dim3(front::kTile, 8), 0, stream>>>(mel, mels, frames, x);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_conv_weight_layout(const uint16_t *w, int64_t c_out, int64_t c_in, uint16_t *out,
                                      cudaStream_t stream)
{
    const int64_t total = c_out * c_in * 3;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4 * 148));
    front::conv_weight_layout_kernel<<<blocks, 256, 0, stream>>>(w, c_out, c_in, out);
    count_launch();
    return cudaGetLastError();
}

// Launches with programmatic stream serialisation: the kernel waits for the
// previous grid (griddepcontrol.wait) before reading anything it wrote.
template <class Kernel, class... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, cudaStream_t stream, Args... args)
{
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, kernel, args...);
    count_launch();
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_decoder_embed(const int32_t *tokens, const int32_t *lengths, const uint16_t *token_table,
                                 const uint16_t *position_table, int streams, int width, int vocab, int positions,
                                 uint16_t *x, cudaStream_t stream)
{
    return launch_pdl(dec::embed_kernel, dim3(static_cast<unsigned>(streams)), dim3(256), stream, tokens, lengths,
                      token_table, position_table, width, vocab, positions, x);
}

cudaError_t launch_decoder_self_attention(const DecoderAttentionLaunch &L, cudaStream_t stream)
{
    dec::AttnParams p{};
    p.heads = L.heads;
    p.capacity = L.capacity;
    p.qkv = L.qkv;
    p.qkv_ld = L.qkv_ld;
    p.cache_k = L.cache_k;
    p.cache_v = L.cache_v;
    p.lengths = L.lengths;
    const uint16_t c = __half_as_ushort(__float2half_rn(static_cast<float>(std::pow(64.0, -0.25))));
    p.scale2 = static_cast<uint32_t>(c) * 0x10001u;
    p.out = L.out;
    p.codes = L.codes;
    p.code_scale = L.code_scale;
    p.code_recip = L.codes ? static_cast<float>(1.0 / static_cast<double>(L.code_scale)) : 0.0f;
    return launch_pdl(dec::self_attention_kernel, dim3(static_cast<unsigned>(L.streams * L.heads)),
                      dim3(dec::kAttnThreads), stream, p);
}

cudaError_t launch_greedy_select(const uint16_t *logits, int64_t logits_ld, const float *suppression,
                                 int64_t suppression_ld, int streams, int vocab, int32_t *tokens, int32_t *lengths,
                                 cudaStream_t stream)
{
    return launch_pdl(dec::select_kernel, dim3(static_cast<unsigned>(streams)), dim3(dec::kSelectThreads), stream,
                      logits, logits_ld, suppression, suppression_ld, vocab, tokens, lengths);
}

int read_and_clear_decoder_error()
{
    int value = 0;
    if (cudaMemcpyFromSymbol(&value, dec::g_decoder_error, sizeof(int)) != cudaSuccess)
        return -1;
    const int zero = 0;
    if (value != 0 && cudaMemcpyToSymbol(dec::g_decoder_error, &zero, sizeof(int)) != cudaSuccess)
        return -1;
    return value;
}

cudaError_t launch_fp16_gelu(const uint16_t *x, uint16_t *y, int64_t count, cudaStream_t stream)
{
    int64_t blocks = (count + proj::kThreads - 1) / proj::kThreads;
    blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(sm_count()) * 16));
    proj::fp16_gelu_kernel<<<static_cast<unsigned>(blocks), proj::kThreads, 0, stream>>>(x, y, count);
    count_launch();
    return cudaGetLastError();
}

cudaError_t read_and_clear_device_error(int *site)
{
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess)
        return err;
    int value = 0;
    err = cudaMemcpyFromSymbol(&value, g_device_error, sizeof(int));
    if (err != cudaSuccess)
        return err;
    if (value != 0) {
        const int zero = 0;
        err = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    }
    if (site)
        *site = value;
    return err;
}

} // namespace lffw

// ---------------------------------------------------------------------------
// Allocation-free FP8 linear on fp16 activations (lffw_fp8_linear_half_static).
//
// The E4M3 codes of the activations live in this fixed device buffer instead
// of memory the caller allocates, for callers that cannot allocate device
// memory (see include/lffw_fp8.h).  Each GPU that loads the library holds one
// copy until the process exits.  Nothing in it needs to start at zero: every
// call first writes the m * k codes it then reads.

static __device__ __align__(256) uint8_t g_static_scratch[LFFW_STATIC_SCRATCH_BYTES];

namespace {

// Device address of g_static_scratch on `device` (the current device), looked
// up once per device.  The symbol's name in host code is only a host-side
// handle.  Ordinals beyond the cache are refused rather than sharing a slot.
cudaError_t static_scratch_address(int device, uint8_t **out)
{
    static std::mutex lock;
    static uint8_t *addresses[lffw::kMaxDevices] = {};
    if (device < 0 || device >= lffw::kMaxDevices)
        return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(lock);
    if (addresses[device] == nullptr) {
        void *p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_static_scratch);
        if (err != cudaSuccess)
            return err;
        addresses[device] = static_cast<uint8_t *>(p);
    }
    *out = addresses[device];
    return cudaSuccess;
}

bool static_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

} // namespace

extern "C" LFFW_FP8_API lffw_status lffw_fp8_linear_half_static(const uint16_t *x, int64_t m, int64_t n, int64_t k,
                                                                float act_scale, const uint8_t *w_codes,
                                                                const float *w_scales, const uint16_t *bias,
                                                                int32_t epilogue, uint16_t *y, void *stream) noexcept
{
    if (x == nullptr || w_codes == nullptr || w_scales == nullptr || y == nullptr || m < 1 || n < 1 || k < 1 ||
        k % 16 != 0 || n % 16 != 0 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
        return LFFW_INVALID_ARGUMENT;
    if (!static_aligned16(x) || !static_aligned16(w_codes) || !static_aligned16(w_scales) ||
        !static_aligned16(bias) || !static_aligned16(y))
        return LFFW_INVALID_ARGUMENT;
    if (!(std::isfinite(act_scale) && act_scale >= 0x1p-125f && act_scale <= 0x1p125f))
        return LFFW_INVALID_ARGUMENT;
    if (epilogue != LFFW_EPILOGUE_NONE && epilogue != LFFW_EPILOGUE_GELU)
        return LFFW_INVALID_ARGUMENT;
    if (m * k > static_cast<int64_t>(LFFW_STATIC_SCRATCH_BYTES))
        return LFFW_SCRATCH_TOO_SMALL;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return LFFW_CUDA_ERROR;
    }
    const lffw_status gate = lffw_device_supported(device);
    if (gate != LFFW_SUCCESS)
        return gate;
    uint8_t *codes = nullptr;
    if (static_scratch_address(device, &codes) != cudaSuccess) {
        cudaGetLastError();
        return LFFW_CUDA_ERROR;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (lffw::launch_quantize(x, m * k, act_scale, nullptr, codes, st) != cudaSuccess)
        return LFFW_CUDA_ERROR;
    lffw::LinearLaunch L{};
    L.m = m;
    L.n = n;
    L.k = k;
    L.x_codes = codes;
    L.act_scale = act_scale;
    L.w_codes = w_codes;
    L.w_scales = w_scales;
    L.bias = bias;
    L.gelu = epilogue == LFFW_EPILOGUE_GELU;
    L.y = y;
    const bool small = m <= lffw::kSmallMaxRows;
    const cudaError_t err = small ? lffw::launch_fp8_skinny(L, st) : lffw::launch_fp8_gemm(L, st);
    return err == cudaSuccess ? LFFW_SUCCESS : LFFW_CUDA_ERROR;
}
