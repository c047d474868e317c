// Tensor-core grouped GEMM for sm_100a: TMA tile loads into 128B-swizzled shared memory,
// tcgen05.mma (kind::tf32) with the fp32 accumulator in tensor memory, tcgen05.ld epilogue.
//
// Precision modes
//   1  TF32: one MMA per k-step on the operands as stored (about 1e-3 relative per product).
//      Tiles 128 x 128, A and B from shared memory, K stages spread over 4 accumulators.
//   2  3xTF32: each fp32 operand x is split into hi = x with the low 13 mantissa bits cleared and
//      lo = x - hi (exact); C += A_hi B_hi + A_hi B_lo + A_lo B_hi, which carries fp32-level
//      accuracy (the dropped A_lo B_lo term is ~2^-22 relative). B's split is precomputed (the
//      weights are constant). Four split warps write A_hi / A_lo of each stage into tensor
//      memory and the MMAs read A from there, so shared memory only feeds B. Tiles are
//      128 x 192: 192 columns for A_hi B_hi, 192 for the corrections and two 64-column A slots
//      fill the 512 tensor-memory columns (wider MMAs run faster per product: N = 256 took only
//      ~13% longer than N = 128 on B200).
//   3  fp16 pair: the same three products with 16-bit operands (kind::f16, twice the tf32
//      rate). fp16 has 11 significant bits but a narrow exponent range, so every operand is
//      first scaled by a power of two: A per (row, group) so that the row's largest magnitude
//      lies in [2^14, 2^15) (a one-pass kernel writes the scales to the caller's scratch), B per
//      output column (precomputed with the weights). x = hi + lo * 2^-11 with hi = fp16(x) and
//      lo = fp16((x - hi) * 2^11) keeps 22 significant bits of x relative to its row's (column's)
//      largest entry; lo is stored scaled so that it stays in fp16's normal range, and the
//      correction accumulator is scaled back by 2^-11 in the epilogue, where the row and column
//      scales are divided out again (all exact powers of two).
//
// Persistent CTAs (one per SM, 448 threads): warp 0 issues TMA loads, warp 1 allocates tensor
// memory and issues the MMAs (one elected lane), warps 2-9 run the epilogue (warp w reads
// tensor-memory lanes 32 * (w % 4) .. + 31, i.e. output rows of that quarter, and one column
// half of the tile), warps 10-13 split A (mode 2). K advances in 32-element (128-byte) stages
// through an S-deep mbarrier ring that runs on across tiles.
//
// Every wait is bounded: on expiry the CTA records an error code in g_tc_error, abandons the
// tile and still releases its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include <cstring>
#include <numeric>

#include "common.cuh"

// Pipeline depth (shared-memory stages) per precision mode; overridable at build time.
#ifndef ATOM_TC_STAGES_3X
#define ATOM_TC_STAGES_3X 3
#endif
#ifndef ATOM_TC_STAGES_1X
#define ATOM_TC_STAGES_1X 5
#endif
#ifndef ATOM_TC_BN128
#define ATOM_TC_BN128 1
#endif
#ifndef ATOM_TC_STAGES_F16
#define ATOM_TC_STAGES_F16 4
#endif

namespace atom {

__device__ int g_tc_error;

namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;                       // fp32 elements per stage along K (128 bytes)
constexpr uint32_t kTileA = BM * BK * 4;     // 16 KiB
constexpr long long kWaitCycles = 2000000000LL;  // bounded wait: ~1 s of SM clock

struct Groups {
    int ngroups;
    int a_col[8], K[8], c_col[8], N[8], t_col[8];
    const float* bias[8];
    const float* cinv[8];   // mode 3: per-column inverse scale of B (powers of two)
    int tile_start[9];
};

struct Args {
    long long M, ldc, ldt;
    float* C;
    float* Cpre;
    const float* T1;
    const float* T2;
    const int* idx1;
    const int* idx2;
    int act, accumulate;
    int bn;              // column-tile width of this launch (multiple of 32, <= the kernel's BN)
    int ksplit;          // K splits per tile (> 1: raw partial tiles go to the scratch rows)
    int mpad;            // rows per split in the partial buffer (a multiple of BM >= M)
    int tma_out;         // epilogue writes C (and Cpre) with TMA stores / reduce-adds
    int nacc;            // tensor-memory accumulators the K stages are spread over (1 or 4)
    const float* rscale; // mode 3: power-of-two scale of A per (group, row), rows rs_ld apart
    long long rs_ld;
    // gated A (modes 2, 3; gH > 0): A is the so2_1 output Y [M, ld = gld] laid out as
    // [gating rows 0, 1 | m-primed rows 0..8], gH channels each, and the A operand is the gate
    // applied on the fly: SiLU on row 0, row r >= 1 times sigmoid(gating row gate_row(r)),
    // the same expressions as the standalone gate kernel (tt_atom/activation.py:53-70)
    const float* gsrc;
    long long gld;
    int gH;
    Groups g;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false (and an error code) when the clock budget expires or another CTA of
// the grid has already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int code,
                                          long long budget = kWaitCycles) {
    const long long t0 = clock64();
    while (!mbar_try(b, parity)) {
        if (clock64() - t0 > budget) {
            atomicCAS(&g_tc_error, 0, code);
            return false;
        }
        if (*(volatile int*)&g_tc_error != 0) return false;
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// TMA store (or fp32 reduce-add) of one 32 x 32 box from shared memory, bulk-group completion.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y,
                                             bool add) {
    if (add)
        asm volatile(
            "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group"
            " [%0, {%1, %2}], [%3];" ::"l"(reinterpret_cast<uint64_t>(map)),
            "r"(x), "r"(y), "r"(smem_u32(src))
            : "memory");
    else
        asm volatile(
            "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                reinterpret_cast<uint64_t>(map)),
            "r"(x), "r"(y), "r"(smem_u32(src))
            : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                  // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset
    d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                  // 128-byte swizzle
    return d;
}

// Same for 16-bit K-major operands with 64-byte swizzle (32 fp16 per row, atoms 512 bytes apart).
__device__ __forceinline__ uint64_t sdesc64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(512 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;                  // 64-byte swizzle
    return d;
}

// Instruction descriptor (kind::f16): D fp32, A and B fp16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Instruction descriptor: D fp32, A and B tf32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
    return (1u << 4)                    // D: fp32
           | (2u << 7) | (2u << 10)     // A, B: tf32
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Warp roles: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-9 epilogue, 10-13 A split.
constexpr int kEpiWarps = 8;
constexpr int kSplitWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps + kSplitWarps);   // 448
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// Same, with A read from tensor memory (lane = row, one column per K element).
__device__ __forceinline__ void mma_tf32_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}
// kind::f16 with A (two fp16 per column, the even K element in the low half) from tensor memory.
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate));
}
// 16 consecutive tensor-memory columns of this thread's lane <- r[0..15].
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// 32 consecutive tensor-memory columns of this thread's lane <- r[0..31].
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Fast SiLU in the epilogue and 128-wide tiles for narrow launches: measured 17.48 -> 16.94 ms
// per config-2 step together (both on by default).
#ifndef ATOM_TC_FAST_SILU
#define ATOM_TC_FAST_SILU 1
#endif
// SiLU of the epilogue (act = 1)
__device__ __forceinline__ float epi_silu(float x) {
#if ATOM_TC_FAST_SILU
    return silu_gate(x);
#else
    return silu_f(x);
#endif
}

// The gate on four A elements of m-primed row grow: SiLU on row 0, otherwise times the
// sigmoid of the gating values g[0..3] (silu_gate / sigmoid_gate: the standalone gate kernel's
// expressions, so the gated operand is bit-identical to that kernel's output).
__device__ __forceinline__ float4 gate4(float4 x, int grow, const float* g) {
    if (grow == 0)
        return make_float4(silu_gate(x.x), silu_gate(x.y), silu_gate(x.z), silu_gate(x.w));
    return make_float4(x.x * sigmoid_gate(g[0]), x.y * sigmoid_gate(g[1]),
                       x.z * sigmoid_gate(g[2]), x.w * sigmoid_gate(g[3]));
}

__device__ __forceinline__ float4 ldg4(const float* q) {
    return *reinterpret_cast<const float4*>(q);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int MODE>
struct Cfg {
    // B is fp32 (modes 1, 2) or fp16 (mode 3) in shared memory; A always arrives as fp32
    static constexpr uint32_t kTileB = BN * BK * (MODE == 3 ? 2 : 4);
    // modes 2 and 3 keep no A_lo tile in shared memory: the split writes A_hi / A_lo to tensor
    // memory; they load B's lo part beside B
    static constexpr uint32_t kStage = kTileA + kTileB + (MODE >= 2 ? kTileB : 0);
    static constexpr uint32_t kLoadBytes = kTileA + kTileB * (MODE >= 2 ? 2 : 1);  // TMA bytes
    static constexpr int kStages =
        MODE == 3 ? ATOM_TC_STAGES_F16
                  : MODE == 2 ? (BN <= 128 ? ATOM_TC_STAGES_3X + 1 : ATOM_TC_STAGES_3X)
                              : ATOM_TC_STAGES_1X;
    // tensor-memory columns of one A slot (hi then lo): fp32 one K element per column, fp16 two
    static constexpr uint32_t kSlotCols = MODE == 3 ? BK : 2 * BK;
    static constexpr int kEpiCols = BN / 2;        // columns per epilogue warp
    // output staging: one 32 x 32 fp32 buffer (128-byte swizzled) per epilogue warp for the TMA
    // stores; the row-store path of gathered-table launches uses it as an XOR-swizzled tile
    static constexpr uint32_t kOutBuf = 32 * 32 * 4;
    static constexpr uint32_t kStageOut = kEpiWarps * kOutBuf;
    static constexpr uint32_t kSmem = kStages * kStage + kStageOut + 256 + 1024;
    static_assert(kSmem <= 232448, "shared memory per CTA");
    static_assert(kEpiCols % 32 == 0, "epilogue chunks");
    // mode 1: 4 accumulators of BN columns; modes 2, 3: main + corrections, then two A slots
    static_assert(MODE >= 2 ? 2 * BN + 2 * kSlotCols <= 512 : 4 * BN <= 512,
                  "tensor-memory columns");
};

// 1 / x for x = 2^s, |s| <= 126 (exact).
__device__ __forceinline__ float pow2_inv(float x) {
    return __uint_as_float((254u << 23) - (__float_as_uint(x) & 0x7F800000u));
}

// Power-of-two scale 2^(14 - e) for a row whose largest magnitude is mx in [2^e, 2^(e+1)), so
// that the scaled row's largest entry lies in [2^14, 2^15); shift clamped to [-126, 126]. Zero,
// infinite or NaN maxima get scale 1 (zeros stay zero, inf / NaN propagate).
__host__ __device__ inline float pow2_scale(float mx) {
    uint32_t u;
    memcpy(&u, &mx, 4);
    const int ex = (int)((u >> 23) & 0xFF);
    if (mx == 0.f || ex == 0xFF) return 1.f;
    int sh = 14 - (ex - 127);
    sh = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
    const uint32_t o = (uint32_t)(sh + 127) << 23;
    float f;
    memcpy(&f, &o, 4);
    return f;
}

// Mode-3 row scales: out[g * ld + m] = pow2_scale(max_k |A[m, a_col[g] + k]|), one warp per
// row, float4 loads (a_col and K multiples of 4).
__global__ void row_scale_kernel(const float* __restrict__ A, long long lda, long long M,
                                 Groups g, long long ld, float* __restrict__ out) {
    const long long m = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    const float* row = A + m * lda;
    for (int i = 0; i < g.ngroups; ++i) {
        const float* a = row + g.a_col[i];
        float mx = 0.f;
        for (int k = 4 * lane; k < g.K[i]; k += 128) {
            const float4 x = *reinterpret_cast<const float4*>(a + k);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) out[i * ld + m] = pow2_scale(mx);
    }
}

// Tensor maps of one launch: A, and per group the K-major weight (hi) and its lo part.
struct Maps {
    CUtensorMap a;
    CUtensorMap b[8];
    CUtensorMap l[8];
    CUtensorMap c[8];     // per group: C columns c_col .. c_col + N (TMA-store epilogue)
    CUtensorMap cp[8];    // per group: the same columns of Cpre
    CUtensorMap pm[8];    // per group: those columns of the split-K partial rows (ksplit x mpad)
};

// Tile t of the launch -> (group, first row, first column, K stages).
// Work item t = tile * ksplit + split: the split's K stages are [kt0, kt1).
struct TileInfo {
    int grp, n0, nk, kt0, kt1, ks;
    long long m0;
};
__device__ __forceinline__ TileInfo tile_info(const Args& p, int ntn, int t) {
    TileInfo ti;
    ti.ks = t % p.ksplit;
    t /= p.ksplit;
    int mt = t / ntn, tn = t - mt * ntn;
    int grp = 0;
    while (grp + 1 < p.g.ngroups && tn >= p.g.tile_start[grp + 1]) ++grp;
    ti.grp = grp;
    ti.n0 = (tn - p.g.tile_start[grp]) * p.bn;
    ti.m0 = (long long)mt * BM;
    const int nk = p.g.K[grp] / BK;
    ti.kt0 = ti.ks * nk / p.ksplit;
    ti.kt1 = (ti.ks + 1) * nk / p.ksplit;
    ti.nk = ti.kt1 - ti.kt0;
    return ti;
}

// Persistent kernel: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... (column
// tiles of one row block are adjacent, so concurrently running CTAs share A rows in L2).
// The epilogue drains the accumulators into registers and releases tensor memory before it
// computes and stores, so the next tile's MMAs overlap the previous tile's stores.
// TAB: the launch adds gathered table rows (T1 / T2) in the TMA-store epilogue; a separate
// instantiation so that launches without tables keep the lighter epilogue.
template <int BN, int MODE, bool TAB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Args p, int ntn,
                   int ntiles) {
    using CF = Cfg<BN, MODE>;
    constexpr int S = CF::kStages;
    constexpr int EC = CF::kEpiCols;
    constexpr uint32_t kSlot0 = 2 * BN;   // modes 2, 3: A slots after main and corrections
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* outbuf = smem + S * CF::kStage;                      // 1024-byte aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(outbuf + CF::kStageOut);
    uint64_t* conv = full + S;
    uint64_t* empty = conv + S;
    uint64_t* accf = empty + S;
    uint64_t* acce = accf + 1;
    uint64_t* afree = acce + 1;          // mode 2: tensor-memory A slot 0 / 1 free again
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(afree + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 32 * kSplitWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        mbar_init(acce, 32 * kEpiWarps);
        mbar_init(&afree[0], 1);
        mbar_init(&afree[1], 1);
        // a CTA that failed earlier in this grid (or an earlier launch) stops the rest here
        *abort_flag = *(volatile int*)&g_tc_error != 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (*(volatile int*)abort_flag) return;   // uniform over the CTA
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    auto stA = [&](int s) { return smem + s * CF::kStage; };
    auto stB = [&](int s) { return smem + s * CF::kStage + kTileA; };
    auto stBL = [&](int s) { return smem + s * CF::kStage + kTileA + CF::kTileB; };
    auto aborted = [&]() { return *(volatile int*)abort_flag != 0; };

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int t = blockIdx.x; t < ntiles && !aborted(); t += gridDim.x) {
                TileInfo ti = tile_info(p, ntn, t);
                const int a_x0 = p.g.a_col[ti.grp];
                for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++it) {
                    int s = it % S;
                    uint32_t ph = (it / S) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, 1) || aborted()) {
                        *(volatile int*)abort_flag = 1;
                        break;
                    }
                    mbar_expect_tx(&full[s], CF::kLoadBytes);
                    tma_load_2d(stA(s), &maps.a, a_x0 + kt * BK, (int)ti.m0, &full[s]);
                    tma_load_2d(stB(s), &maps.b[ti.grp], kt * BK, ti.n0, &full[s]);
                    if (MODE >= 2) tma_load_2d(stBL(s), &maps.l[ti.grp], kt * BK, ti.n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0, j = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
                TileInfo ti = tile_info(p, ntn, t);
                // a group's last tile multiplies only the columns that remain (N multiple of 16)
                const int rem = p.g.N[ti.grp] - ti.n0;
                const int nmma = rem >= p.bn ? p.bn : (rem + 15) & ~15;
                const uint32_t idesc = MODE == 3 ? idesc_f16(nmma) : idesc_tf32(nmma);
                bool ok = !aborted() && mbar_wait(acce, (j & 1u) ^ 1u, 5);
                if (ok) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int kt = ti.kt0; ok && kt < ti.kt1; ++kt, ++it) {
                    int s = it % S;
                    uint32_t ph = (it / S) & 1u;
                    if (!mbar_wait(MODE >= 2 ? &conv[s] : &full[s], ph, 2) || aborted()) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a = smem_u32(stA(s)), b = smem_u32(stB(s));
                    if constexpr (MODE == 2) {
                        // A_hi / A_lo from tensor-memory slot it % 2; A_hi B_hi into the main
                        // accumulator (columns 0 ..), both corrections into columns BN ..
                        const uint32_t slot = tmem + kSlot0 + (it & 1u) * 2 * BK;
                        const uint32_t bl = smem_u32(stBL(s));
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            const uint32_t acc = (kt > ti.kt0 || kk > 0) ? 1u : 0u;
                            mma_tf32_ta(tmem, slot + kk * 8, sdesc(b + kk * 32), idesc, acc);
                            mma_tf32_ta(tmem + BN, slot + kk * 8, sdesc(bl + kk * 32), idesc,
                                        acc);
                            mma_tf32_ta(tmem + BN, slot + BK + kk * 8, sdesc(b + kk * 32), idesc,
                                        1u);
                        }
                        mma_commit(&empty[s]);
                        mma_commit(&afree[it & 1u]);
                    } else if constexpr (MODE == 3) {
                        // fp16 pair: per 16-element k-step, A_hi (slot columns 0..15) B_hi into
                        // the main accumulator, A_hi B_lo and A_lo (columns 16..31) B_hi into the
                        // corrections (lo parts carry a factor 2^11)
                        const uint32_t slot = tmem + kSlot0 + (it & 1u) * CF::kSlotCols;
                        const uint32_t bl = smem_u32(stBL(s));
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t acc = (kt > ti.kt0 || kk > 0) ? 1u : 0u;
                            mma_f16_ta(tmem, slot + kk * 8, sdesc64(b + kk * 32), idesc, acc);
                            mma_f16_ta(tmem + BN, slot + kk * 8, sdesc64(bl + kk * 32), idesc,
                                       acc);
                            mma_f16_ta(tmem + BN, slot + BK / 2 + kk * 8, sdesc64(b + kk * 32),
                                       idesc, 1u);
                        }
                        mma_commit(&empty[s]);
                        mma_commit(&afree[it & 1u]);
                    } else {
                        // stage kt accumulates into accumulator kt % nacc (columns BN apart)
                        const uint32_t dacc = tmem + (uint32_t)(((kt - ti.kt0) % p.nacc) * BN);
                        const bool first = kt - ti.kt0 < p.nacc;
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            uint32_t acc = (!first || kk > 0) ? 1u : 0u;
                            mma_tf32(dacc, sdesc(a + kk * 32), sdesc(b + kk * 32), idesc, acc);
                        }
                        mma_commit(&empty[s]);
                    }
                }
                if (ok) {
                    mma_commit(accf);
                } else {
                    *(volatile int*)abort_flag = 1;
                    mbar_arrive(accf);
                    break;
                }
            }
        }
    } else if (warp >= 2 + kEpiWarps) {
        // ------------------------------------------------------ A split (modes 2 and 3)
        // Thread = tile row (warp w owns tensor-memory lanes 32 * (w % 4) ..): reads its row of
        // the swizzled A stage, writes A_hi and A_lo to tensor-memory slot it % 2, once the MMAs
        // that read that slot two stages earlier have completed. Mode 2: A_hi = A with the low
        // 13 mantissa bits cleared, A_lo = A - A_hi (fp32, 2 x BK columns). Mode 3: y = A times
        // the row's power-of-two scale, A_hi = fp16(y), A_lo = fp16((y - A_hi) * 2^11), packed
        // two per column (BK / 2 columns each).
        if (MODE >= 2) {
            const int quarter = warp & 3;
            const int r = quarter * 32 + lane;
            const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles && !aborted(); t += gridDim.x) {
                TileInfo ti = tile_info(p, ntn, t);
                float rs = 1.f;
                if (MODE == 3 && ti.m0 + r < p.M) rs = p.rscale[ti.grp * p.rs_ld + ti.m0 + r];
                const bool row_ok = ti.m0 + r < p.M;
                for (int kt = ti.kt0; kt < ti.kt1; ++kt, ++it) {
                    int s = it % S;
                    uint32_t ph = (it / S) & 1u;
                    // gated A: this stage's 32 K elements are channels gc .. gc + 31 of one
                    // m-primed row grow; its gating values are loaded before the TMA wait
                    int grow = -1;
                    float gv[BK];
                    if (p.gH > 0) {
                        const int x = p.g.a_col[ti.grp] + kt * BK;
                        grow = x / p.gH - 2;
                        const int gc = x - (grow + 2) * p.gH;
                        // the next stage's gating line into L1 while this one is processed
                        if (kt + 1 < ti.kt1 && row_ok) {
                            const int xn = x + BK, gn = xn / p.gH - 2;
                            if (gn > 0) {
                                const float* pn = p.gsrc + (ti.m0 + r) * p.gld +
                                                  gate_row(gn) * p.gH + (xn - (gn + 2) * p.gH);
                                asm volatile("prefetch.global.L1 [%0];" ::"l"(pn));
                            }
                        }
                        if (grow > 0 && !row_ok) {
#pragma unroll
                            for (int k = 0; k < BK; ++k) gv[k] = 0.f;
                        } else if (grow > 0) {
                            const float* gp =
                                p.gsrc + (ti.m0 + r) * p.gld + gate_row(grow) * p.gH + gc;
#pragma unroll
                            for (int c = 0; c < BK / 4; ++c) {
                                const float4 q = __ldg(reinterpret_cast<const float4*>(gp) + c);
                                gv[4 * c] = q.x;
                                gv[4 * c + 1] = q.y;
                                gv[4 * c + 2] = q.z;
                                gv[4 * c + 3] = q.w;
                            }
                        }
                    }
                    ok = mbar_wait(&full[s], ph, 3) &&
                         mbar_wait(&afree[it & 1u], ((it >> 1) & 1u) ^ 1u, 6) && !aborted();
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) {
                        *(volatile int*)abort_flag = 1;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint8_t* row = stA(s) + (r >> 3) * 1024 + (r & 7) * 128;
                    const uint32_t slot = lane_base + kSlot0 + (it & 1u) * CF::kSlotCols;
                    if constexpr (MODE == 3) {
                        uint32_t hi[BK / 2], lo[BK / 2];
#pragma unroll
                        for (int c = 0; c < BK / 4; ++c) {
                            float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) << 4));
                            if (grow >= 0) x = gate4(x, grow, gv + 4 * c);
                            const float y[4] = {x.x * rs, x.y * rs, x.z * rs, x.w * rs};
#pragma unroll
                            for (int k = 0; k < 2; ++k) {
                                const __half2 h = __floats2half2_rn(y[2 * k], y[2 * k + 1]);
                                const float2 hb = __half22float2(h);
                                const __half2 l = __floats2half2_rn((y[2 * k] - hb.x) * 2048.f,
                                                                    (y[2 * k + 1] - hb.y) * 2048.f);
                                hi[2 * c + k] = *reinterpret_cast<const uint32_t*>(&h);
                                lo[2 * c + k] = *reinterpret_cast<const uint32_t*>(&l);
                            }
                        }
                        tmem_st16(slot, hi);
                        tmem_st16(slot + BK / 2, lo);
                    } else {
                        uint32_t hi[BK], lo[BK];
#pragma unroll
                        for (int c = 0; c < BK / 4; ++c) {
                            float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) << 4));
                            if (grow >= 0) x = gate4(x, grow, gv + 4 * c);
                            const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint32_t h = __float_as_uint(xs[k]) & 0xFFFFE000u;
                                hi[4 * c + k] = h;
                                lo[4 * c + k] = __float_as_uint(xs[k] - __uint_as_float(h));
                            }
                        }
                        tmem_st32(slot, hi);
                        tmem_st32(slot + BK, lo);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    mbar_arrive(&conv[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        // warp w: output rows of lane quarter w % 4, columns half * EC .. + EC of the tile
        const int quarter = warp & 3;
        const int cbase = ((warp - 2) >> 2) * EC;
        uint8_t* mybuf = outbuf + (warp - 2) * CF::kOutBuf;
        uint32_t j = 0;
        bool pending = false;            // a TMA store from this warp's buffer may be reading it
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
            TileInfo ti = tile_info(p, ntn, t);
            bool ok = mbar_wait(accf, j & 1u, 4) && !aborted();
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int N = p.g.N[ti.grp];
            const bool active = ti.n0 + cbase < N && cbase < p.bn;
            // drain the accumulators into registers (partial sums added with round-to-nearest):
            // mode 1 the K-stage accumulators in use, modes 2, 3 main + corrections (mode 3: the
            // corrections carry 2^11, and the row and column scales are divided out)
            const int nused = MODE >= 2 ? 2 : (ti.nk < p.nacc ? ti.nk : p.nacc);
            float v[EC];
            const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)cbase;
            if (active) {
#pragma unroll
                for (int c0 = 0; c0 < EC; c0 += 16) tmem_ld16(lane_base + (uint32_t)c0, v + c0);
#pragma unroll 1
                for (int q = 1; q < nused; ++q) {
#pragma unroll
                    for (int c0 = 0; c0 < EC; c0 += 8) {
                        float w[8];
                        tmem_ld8(lane_base + (uint32_t)(q * BN + c0), w);
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            v[c0 + jj] += MODE == 3 ? w[jj] * (1.f / 2048.f) : w[jj];
                    }
                }
                if constexpr (MODE == 3) {
                    const long long row = ti.m0 + quarter * 32 + lane;
                    const float rinv =
                        row < p.M ? pow2_inv(p.rscale[ti.grp * p.rs_ld + row]) : 0.f;
                    const float* ci = p.g.cinv[ti.grp];
                    const int nb = ti.n0 + cbase;
#pragma unroll
                    for (int c = 0; c < EC; ++c)
                        v[c] *= rinv * (nb + c < N ? ci[nb + c] : 0.f);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(acce);                  // tensor memory may take the next tile now
            if (!active) continue;
            // split-K work items store the raw partial sums (bias, tables and SiLU are applied
            // when the partials are added)
            const bool split = p.ksplit > 1;
            const float* bias = split ? nullptr : p.g.bias[ti.grp];
            if (p.tma_out) {
                // each 32 x 32 block: bias (+ gathered table rows) (+ SiLU) applied in registers,
                // written 128-byte swizzled into this warp's buffer, stored by one lane with TMA
                // (reduce-add when accumulating); the tensor map clips rows >= M, cols >= N
                const int y0 = (int)(ti.m0 + quarter * 32);
                if (y0 >= p.M) continue;
                // this thread's output row and its rows of the gathered tables (one per lane)
                const long long row = (long long)y0 + lane;
                const float* t1row = nullptr;
                const float* t2row = nullptr;
                if (TAB && row < p.M) {
                    const int tc = p.g.t_col[ti.grp];
                    if (p.T1) t1row = p.T1 + (long long)p.idx1[row] * p.ldt + tc;
                    if (p.T2) t2row = p.T2 + (long long)p.idx2[row] * p.ldt + tc;
                }
#pragma unroll
                for (int c0 = 0; c0 < EC; c0 += 32) {
                    const int x0 = ti.n0 + cbase + c0;
                    if (x0 >= N || cbase + c0 >= p.bn) break;
                    // gathered-table launches: the block's pre-activation values (accumulator +
                    // bias + the two table rows) formed once, in place, before the staging
                    // buffer is waited for, so the gathered loads overlap the previous store;
                    // 16 columns at a time to bound the registers in flight
                    if (TAB) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            // the second half's loads are not hoisted above the first half's use
                            if (h) asm volatile("" ::: "memory");
#pragma unroll
                            for (int qq = 0; qq < 4; ++qq) {
                                const int q = 4 * h + qq;
                                // columns x0 + 4q .. + 3 are all inside or all outside the group
                                // (N is a multiple of 4 on this path)
                                const bool in = x0 + 4 * q < N;
                                float4 a1 = make_float4(0.f, 0.f, 0.f, 0.f), a2 = a1;
                                if (t1row && in) a1 = ldg4(t1row + x0 + 4 * q);
                                if (t2row && in) a2 = ldg4(t2row + x0 + 4 * q);
                                const float t1v[4] = {a1.x, a1.y, a1.z, a1.w};
                                const float t2v[4] = {a2.x, a2.y, a2.z, a2.w};
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int jj = 4 * q + k;
                                    const float b = (bias && in) ? bias[x0 + jj] : 0.f;
                                    v[c0 + jj] = (v[c0 + jj] + b + t1v[k]) + t2v[k];
                                }
                            }
                        }
                    }
#pragma unroll 1
                    for (int pass = 0; pass < 2; ++pass) {
                        // pass 0: pre-activation to Cpre (SiLU launches that keep it)
                        if (pass == 0 && (split || !(p.act == 1 && p.Cpre))) continue;
                        const bool silu = !split && pass == 1 && p.act == 1;
                        if (pending && lane == 0)
                            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                        __syncwarp();
                        float4* buf = reinterpret_cast<float4*>(mybuf);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float e[4];
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                // (TAB: bias and table rows already added above)
                                const int jj = 4 * q + k;
                                const float b =
                                    (!TAB && bias && x0 + jj < N) ? bias[x0 + jj] : 0.f;
                                const float y = TAB ? v[c0 + jj] : v[c0 + jj] + b;
                                e[k] = silu ? epi_silu(y) : y;
                            }
                            buf[lane * 8 + (q ^ (lane & 7))] = make_float4(e[0], e[1], e[2], e[3]);
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            if (split)
                                tma_store_2d(&maps.pm[ti.grp], buf, x0, ti.ks * p.mpad + y0, false);
                            else
                                tma_store_2d(pass == 0 ? &maps.cp[ti.grp] : &maps.c[ti.grp], buf,
                                             x0, y0, pass == 1 && p.accumulate);
                        }
                        pending = true;
                    }
                }
                continue;
            }
            // row stores (gathered-table launches): each 32 x 32 block goes through this warp's
            // XOR-swizzled shared tile, so that a warp writes 32 consecutive columns of one row
            // per instruction (and reads bias and table entries coalesced)
            const int ccol = p.g.c_col[ti.grp], tcol = p.g.t_col[ti.grp];
            float* st = reinterpret_cast<float*>(mybuf);
            const long long mrow0 = ti.m0 + quarter * 32;
#pragma unroll
            for (int c0 = 0; c0 < EC; c0 += 32) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) st[lane * 32 + (jj ^ lane)] = v[c0 + jj];
                __syncwarp();
                const int n = ti.n0 + cbase + c0 + lane;
                const bool nok = n < N && cbase + c0 + lane < p.bn;
                const float bn = (bias && nok) ? bias[n] : 0.f;
                for (int r = 0; r < 32; ++r) {
                    const long long m = mrow0 + r;
                    if (m >= p.M) break;
                    if (!nok) continue;
                    float x = st[r * 32 + (lane ^ r)] + bn;
                    if (p.T1) x += p.T1[(long long)p.idx1[m] * p.ldt + tcol + n];
                    if (p.T2) x += p.T2[(long long)p.idx2[m] * p.ldt + tcol + n];
                    const long long off = m * p.ldc + ccol + n;
                    if (p.act == 1) {
                        if (p.Cpre) p.Cpre[off] = x;
                        x = epi_silu(x);
                    }
                    p.C[off] = p.accumulate ? p.C[off] + x : x;
                }
                __syncwarp();
            }
        }
        // TMA stores issued by this warp must finish before the CTA (and its shared memory) ends
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int encoder() {
    if (g_encode) return ATOM_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return ATOM_ERR_CUDA;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return ATOM_OK;
}

// 2-D fp32 tensor map: `inner` contiguous columns, `outer` rows `ld` elements apart, box of
// 32 x box_rows with 128-byte swizzle; out-of-range reads are zero-filled.
static int make_map(CUtensorMap* m, const float* base, long long inner, long long outer,
                    long long ld, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d): inner %lld outer %lld ld %lld", (int)r,
                  inner, outer, ld);
        return ATOM_ERR_ARG;
    }
    return ATOM_OK;
}

// 2-D fp16 tensor map for mode 3's weights: `inner` contiguous K elements, `outer` rows `ld`
// elements apart, box of 32 x box_rows (64 bytes per row) with 64-byte swizzle.
static int make_map16(CUtensorMap* m, const void* base, long long inner, long long outer,
                      long long ld, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (fp16) failed (%d): inner %lld outer %lld ld %lld",
                  (int)r, inner, outer, ld);
        return ATOM_ERR_ARG;
    }
    return ATOM_OK;
}

// Accumulators per tile. The tensor core's fp32 accumulation rounds each k-step's sum toward
// zero, so its error grows with the number of steps in one accumulator; spreading the stages
// over 4 accumulators (summed in the epilogue with round-to-nearest) divides that by 4.
// Measured on B200 (K = 1024, all-positive operands, 3xTF32): mean relative bias -2.1e-5 with
// one accumulator (all three products in it), -5.3e-6 with four. TF32 uses four; 3xTF32
// keeps A_hi B_hi in one accumulator (K / 8 steps instead of 3 K / 8) and the two small
// correction products in another, whose rounding is negligible against the total.
constexpr int g_nacc = 4;

// Split-K: C[m, c_col + n] (+)= act((sum over splits in order of P[s, m, c_col + n]) + bias[n]),
// the pre-activation kept in Cpre when given; four columns per thread.
__global__ void splitk_reduce_kernel(const float* __restrict__ P, int S, long long mpad,
                                     long long ldc, long long M, int c_col, int N,
                                     const float* __restrict__ bias, int act, float* Cpre,
                                     int accumulate, float* C) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nq = N / 4;
    if (t >= M * nq) return;
    const long long m = t / nq;
    const int n = 4 * (int)(t - m * nq);
    const long long off = m * ldc + c_col + n;
    float4 acc = *reinterpret_cast<const float4*>(P + off);
    for (int k = 1; k < S; ++k) {
        const float4 q = *reinterpret_cast<const float4*>(P + k * mpad * ldc + off);
        acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
    }
    float x[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (bias) x[k] += bias[n + k];
        if (act == 1) {
            if (Cpre) Cpre[off + k] = x[k];
            x[k] = epi_silu(x[k]);
        }
        C[off + k] = accumulate ? C[off + k] + x[k] : x[k];
    }
}

template <int BN, int MODE>
static int launch(const float* A, long long lda, long long M, const atom_gemm_groups* g,
                  float* C, long long ldc, float* Cpre, const float* T1, const float* T2,
                  const int* idx1, const int* idx2, long long ldt, int act, int accumulate,
                  float* scratch, long long scratch_floats, cudaStream_t st, int gate_H = 0) {
    using CF = Cfg<BN, MODE>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, MODE, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)CF::kSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_tc_kernel<BN, MODE, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CF::kSmem);
        if (e != cudaSuccess) {
            set_error("gemm_tc: cannot reserve %u bytes of shared memory: %s", CF::kSmem,
                      cudaGetErrorString(e));
            return ATOM_ERR_CUDA;
        }
        attr_set = true;
    }
    Maps maps;
    memset(&maps, 0, sizeof(maps));
    if (int s = make_map(&maps.a, A, lda, M, lda, BM)) return s;
    Args p;
    p.M = M; p.ldc = ldc; p.ldt = ldt; p.C = C; p.Cpre = Cpre; p.T1 = T1; p.T2 = T2;
    p.idx1 = idx1; p.idx2 = idx2; p.act = act; p.accumulate = accumulate;
    p.nacc = MODE >= 2 ? 2 : g_nacc;
    p.g.ngroups = g->ngroups;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    // TMA-store epilogue: 16-byte aligned column blocks, rows and gathered-table rows. A
    // group's width must be a multiple of 4 columns too: the store clips at 16-byte granularity,
    // so a 130-column group would also get columns 130 and 131 written (measured on B200).
    bool tma_out = ldc % 4 == 0 && aligned16(C) && (!Cpre || aligned16(Cpre)) &&
                   ((!T1 && !T2) || ldt % 4 == 0) && (!T1 || aligned16(T1)) &&
                   (!T2 || aligned16(T2));
    for (int i = 0; i < g->ngroups; ++i)
        tma_out = tma_out && g->c_col[i] % 4 == 0 && g->N[i] % 4 == 0 && g->N[i] >= 32 &&
                  ((!T1 && !T2) || g->t_col[i] % 4 == 0);
    p.tma_out = tma_out ? 1 : 0;
    const long long mblocks = ceil_div(M, BM);
    auto count_tiles = [&](int w) {
        long long t = 0;
        for (int i = 0; i < g->ngroups; ++i) t += ceil_div(g->N[i], w);
        return t * mblocks;
    };
    // split-K (caller scratch given, TMA epilogue, no gathered tables): when full-width tiles
    // would leave at least half the SMs idle, each tile's K stages are split over up to 8 CTAs
    // (>= 4 K stages each, and only for K >= 512: short-K launches lose more to the partial
    // traffic than they gain); the raw partials are added in split order by a second kernel
    int ksplit = 1;
    const long long mpad = mblocks * BM;
    // mode 3 keeps its row scales (groups x mpad floats) at the start of the scratch; split-K
    // partials follow
    const long long rs_floats = MODE == 3 ? (g->ngroups * mpad + 63) / 64 * 64 : 0;
    if (MODE == 3 && (!scratch || scratch_floats < rs_floats)) {
        set_error("gemm_tc: precision 3 needs a scratch of %lld floats", rs_floats);
        return ATOM_ERR_ARG;
    }
    float* part = scratch ? scratch + rs_floats : nullptr;
    const long long part_floats = scratch ? scratch_floats - rs_floats : 0;
    if (part && tma_out && !T1 && !T2 && count_tiles(BN) * 2 <= nsm) {
        int min_nk = 1 << 30;
        for (int i = 0; i < g->ngroups; ++i) min_nk = min_nk < g->K[i] / BK ? min_nk : g->K[i] / BK;
        int sk = (int)(nsm / count_tiles(BN));
        sk = sk < 8 ? sk : 8;
        sk = min_nk < 16 ? 1 : (sk < min_nk / 4 ? sk : min_nk / 4);
        while (sk >= 2 && (long long)sk * mpad * ldc > part_floats) --sk;
        if (sk >= 2) ksplit = sk;
    }
    p.ksplit = ksplit;
    p.mpad = (int)mpad;
    // column-tile width: the full BN unless that leaves SMs without a tile (few rows, e.g.
    // node-level GEMMs without split-K); then the widest multiple of 32 (down to 64) that
    // gives every SM one
    int bn = BN;
    if (ksplit == 1 && count_tiles(BN) < nsm)
        for (int w = BN - 32; w >= 64; w -= 32) {
            bn = w;
            if (count_tiles(w) >= nsm) break;
        }
    p.bn = bn;
    int tiles = 0;
    for (int i = 0; i < g->ngroups; ++i) {
        p.g.a_col[i] = g->a_col[i];
        p.g.K[i] = g->K[i];
        p.g.c_col[i] = g->c_col[i];
        p.g.N[i] = g->N[i];
        p.g.t_col[i] = g->t_col[i];
        p.g.bias[i] = g->bias[i];
        p.g.cinv[i] = MODE == 3 ? g->Bh_inv[i] : nullptr;
        p.g.tile_start[i] = tiles;
        tiles += ceil_div(g->N[i], bn);
        if (MODE == 3) {
            if (int s = make_map16(&maps.b[i], g->Bh[i], g->K[i], g->N[i], g->K[i], BN)) return s;
            if (int s = make_map16(&maps.l[i], g->Bh_lo[i], g->K[i], g->N[i], g->K[i], BN))
                return s;
        } else {
            if (int s = make_map(&maps.b[i], g->Bt[i], g->K[i], g->N[i], g->K[i], BN)) return s;
            if (MODE == 2)
                if (int s = make_map(&maps.l[i], g->Bt_lo[i], g->K[i], g->N[i], g->K[i], BN))
                    return s;
        }
    }
    p.rscale = MODE == 3 ? scratch : nullptr;
    p.rs_ld = mpad;
    p.gsrc = gate_H > 0 ? A : nullptr;
    p.gld = lda;
    p.gH = gate_H;
    p.g.tile_start[g->ngroups] = tiles;
    if (tma_out) {
        for (int i = 0; i < g->ngroups; ++i) {
            if (int s = make_map(&maps.c[i], C + g->c_col[i], g->N[i], M, ldc, 32)) return s;
            if (act == 1 && Cpre)
                if (int s = make_map(&maps.cp[i], Cpre + g->c_col[i], g->N[i], M, ldc, 32))
                    return s;
            if (ksplit > 1)
                if (int s = make_map(&maps.pm[i], part + g->c_col[i], g->N[i],
                                     ksplit * mpad, ldc, 32))
                    return s;
        }
    }
    const long long ntiles = (long long)tiles * ceil_div(M, BM) * ksplit;
    if (ntiles >= (1LL << 31)) {
        set_error("gemm_tc: too many tiles");
        return ATOM_ERR_ARG;
    }
    // Persistent CTAs walk the work items `grid` apart. When grid shares a factor with the
    // items per row block (column tiles x K splits), a CTA meets the same column tiles in every
    // round, and a group's narrow last tile then makes some CTAs' share much lighter than
    // others' (e.g. N = 256 as 192 + 64 with 148 CTAs: the even CTAs get every wide tile). A
    // grid coprime with that period, a few CTAs short of one per SM at most, rotates each CTA
    // through the columns.
    int grid = (int)(ntiles < nsm ? ntiles : nsm);
    if (ntiles > nsm) {
        const int period = tiles * ksplit;
        for (int g = grid; g >= grid - 8 && g > 1; --g)
            if (std::gcd(g, period) == 1) {
                grid = g;
                break;
            }
    }
    if (MODE == 3) {
        row_scale_kernel<<<ceil_div(M * 32, 256), 256, 0, st>>>(A, lda, M, p.g, mpad, scratch);
        if (int s = check_launch("gemm_tc row scales")) return s;
    }
    if (tma_out && (T1 || T2))
        gemm_tc_kernel<BN, MODE, true><<<grid, kThreads, CF::kSmem, st>>>(maps, p, tiles,
                                                                         (int)ntiles);
    else
        gemm_tc_kernel<BN, MODE, false><<<grid, kThreads, CF::kSmem, st>>>(maps, p, tiles,
                                                                          (int)ntiles);
    if (int s = check_launch("gemm_tc")) return s;
    if (ksplit > 1) {
        for (int i = 0; i < g->ngroups; ++i) {
            const long long n4 = M * (g->N[i] / 4);
            splitk_reduce_kernel<<<ceil_div(n4, 256), 256, 0, st>>>(
                part, ksplit, mpad, ldc, M, g->c_col[i], g->N[i], g->bias[i], act, Cpre,
                accumulate, C);
            if (int s = check_launch("gemm_tc split-K reduce")) return s;
        }
    }
    return ATOM_OK;
}

}  // namespace tc

// True when the tensor-core path can run this problem: every K a multiple of 32, K-major weight
// copies present, TMA-compatible strides and alignment.
bool gemm_tc_supported(const float* A, long long lda, const atom_gemm_groups* g, int precision) {
    if (precision < 1 || precision > 3) return false;
    if (g->ngroups > 8 || lda % 4 != 0 || !aligned16(A)) return false;
    for (int i = 0; i < g->ngroups; ++i) {
        if (g->K[i] <= 0 || g->K[i] % tc::BK != 0 || g->a_col[i] % 4 != 0) return false;
        if (!g->Bt[i] || !aligned16(g->Bt[i])) return false;
        if (precision >= 2 && (!g->Bt_lo[i] || !aligned16(g->Bt_lo[i]))) return false;
    }
    return true;
}

// Mode 3 also needs the fp16 weight halves, their column scales and a scratch for the row
// scales; without them the launch runs as mode 2 (same accuracy class).
static bool f16_ready(long long M, const atom_gemm_groups* g, long long scratch_floats) {
    for (int i = 0; i < g->ngroups; ++i)
        if (!g->Bh[i] || !g->Bh_lo[i] || !g->Bh_inv[i] || !aligned16(g->Bh[i]) ||
            !aligned16(g->Bh_lo[i]))
            return false;
    return scratch_floats >= (g->ngroups * (ceil_div(M, tc::BM) * tc::BM) + 63) / 64 * 64;
}

int gemm_tc(const float* A, long long lda, long long M, const atom_gemm_groups* g, float* C,
            long long ldc, float* Cpre, const float* T1, const float* T2, const int* idx1,
            const int* idx2, long long ldt, int act, int accumulate, int precision,
            float* scratch, long long scratch_floats, cudaStream_t st) {
    if (int s = tc::encoder()) return s;
    if (precision == 3 && scratch && f16_ready(M, g, scratch_floats))
        return tc::launch<192, 3>(A, lda, M, g, C, ldc, Cpre, T1, T2, idx1, idx2, ldt, act,
                                  accumulate, scratch, scratch_floats, st);
#if ATOM_TC_BN128
    // launches whose groups are all at most 128 columns wide: 128-wide tiles (the epilogue
    // warps split 64 + 64 columns instead of 96 + 32)
    bool narrow = true;
    for (int i = 0; i < g->ngroups; ++i) narrow = narrow && g->N[i] <= 128;
    if (precision == 2 && narrow)
        return tc::launch<128, 2>(A, lda, M, g, C, ldc, Cpre, T1, T2, idx1, idx2, ldt, act,
                                  accumulate, scratch, scratch_floats, st);
#endif
    if (precision >= 2)
        return tc::launch<192, 2>(A, lda, M, g, C, ldc, Cpre, T1, T2, idx1, idx2, ldt, act,
                                  accumulate, scratch, scratch_floats, st);
    return tc::launch<128, 1>(A, lda, M, g, C, ldc, Cpre, T1, T2, idx1, idx2, ldt, act,
                              accumulate, scratch, scratch_floats, st);
}

// The so2_2 GEMM on the gated so2_1 output (see Args::gH): precision 2 or 3 only (the gate is
// applied where the split warps convert A); every group's A columns must lie in rows 0..8 of Y,
// stage-aligned (a_col and gH multiples of 32).
int gemm_tc_gated(const float* Y, long long ldy, long long M, const atom_gemm_groups* g, int H,
                  float* C, long long ldc, int precision, float* scratch,
                  long long scratch_floats, cudaStream_t st) {
    if (int s = tc::encoder()) return s;
    if (precision == 3 && scratch && f16_ready(M, g, scratch_floats))
        return tc::launch<192, 3>(Y, ldy, M, g, C, ldc, nullptr, nullptr, nullptr, nullptr,
                                  nullptr, 0, 0, 0, scratch, scratch_floats, st, H);
    return tc::launch<192, 2>(Y, ldy, M, g, C, ldc, nullptr, nullptr, nullptr, nullptr, nullptr,
                              0, 0, 0, scratch, scratch_floats, st, H);
}

}  // namespace atom

namespace atom {
namespace tc {
// One thread waits, with the GEMM's own bounded wait, on an mbarrier that nothing arrives on:
// the wait gives up after `budget` clocks and records `code` in g_tc_error, exactly as an
// expired wait inside the GEMM does.
__global__ void wait_selftest_kernel(long long budget, int code) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_wait(&bar, 0u, code, budget);
}
}  // namespace tc
}  // namespace atom

namespace atom {
namespace tc {
__global__ void take_error_kernel(int* dst) {
    *dst = *(volatile int*)&g_tc_error;
    g_tc_error = 0;
}
}  // namespace tc
}  // namespace atom

int* atom::device_error_word() {
    static int* addr[64] = {};      // per device of this process
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, atom::g_tc_error) == cudaSuccess)
            addr[dev] = static_cast<int*>(p);
    }
    return addr[dev];
}

extern "C" int atom_device_error_take(int* code_dev, void* stream) {
    ATOM_REQUIRE(code_dev, "atom_device_error_take: code_dev is NULL");
    atom::tc::take_error_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(code_dev);
    return atom::check_launch("atom_device_error_take");
}

extern "C" int atom_wait_selftest(int64_t budget_cycles, void* stream) {
    if (budget_cycles <= 0 || budget_cycles > atom::tc::kWaitCycles) {
        atom::set_error("atom_wait_selftest: budget_cycles must be in [1, %lld]",
                        atom::tc::kWaitCycles);
        return ATOM_ERR_ARG;
    }
    atom::tc::wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(budget_cycles,
                                                                        ATOM_WAIT_SELFTEST_CODE);
    return atom::check_launch("atom_wait_selftest");
}

extern "C" int atom_device_error(int* code_host, void* stream) {
    int h = 0;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&h, atom::g_tc_error, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && h != 0) {
        int zero = 0;
        e = cudaMemcpyToSymbolAsync(atom::g_tc_error, &zero, sizeof(int), 0,
                                    cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    if (e != cudaSuccess) {
        atom::set_error("atom_device_error: %s", cudaGetErrorString(e));
        return ATOM_ERR_CUDA;
    }
    if (code_host) *code_host = h;
    return ATOM_OK;
}
