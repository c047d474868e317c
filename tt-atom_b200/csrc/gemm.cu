// Grouped fp32 GEMM with fused epilogues (bias, per-row table gathers, SiLU, accumulate).
//
// One launch covers every group of a block-diagonal contraction, e.g. the three per-m blocks of
// an SO(2) convolution (tt_atom/so2.py:255-330: m = 0 dense linear with bias; each m > 0 one
// linear on [real | imag] with the block weight [[P, Q], [-Q, P]]) or the per-layer radial MLPs
// (tt_atom/so2.py:54-115). Group g reads columns [a_col, a_col + K) of A and writes columns
// [c_col, c_col + N) of C.
//
// precision 0: register-tiled FMA kernel (128 x 128 tile, 8 x 8 outputs per thread).
// precision 1 / 2 / 3: the tcgen05 tensor-core kernel of gemm_tc.cu (TF32 / 3xTF32 / fp16 pair)
// when the shape allows it (every K a multiple of 32, K-major weights given; mode 3 also needs
// its fp16 weight halves and a scratch, else it runs as mode 2); otherwise the FMA kernel,
// which is at least as accurate.
#include "common.cuh"

namespace atom {

bool gemm_tc_supported(const float* A, long long lda, const atom_gemm_groups* g, int precision);
int gemm_tc(const float* A, long long lda, long long M, const atom_gemm_groups* g, float* C,
            long long ldc, float* Cpre, const float* T1, const float* T2, const int* idx1,
            const int* idx2, long long ldt, int act, int accumulate, int precision,
            float* scratch, long long scratch_floats, cudaStream_t st);
int gemm_tc_gated(const float* Y, long long ldy, long long M, const atom_gemm_groups* g, int H,
                  float* C, long long ldc, int precision, float* scratch,
                  long long scratch_floats, cudaStream_t st);

struct GemmArgs {
    const float* A;
    long long lda, M;
    float* C;
    float* Cpre;
    long long ldc;
    const float* T1;
    const float* T2;
    const int* idx1;
    const int* idx2;
    long long ldt;
    int act, accumulate;
    atom_gemm_groups g;
    int tile_start[9];   // prefix of N tiles over groups
};

constexpr int BM = 128, BN = 128, BK = 16;

__device__ __forceinline__ void epilogue_store(const GemmArgs& p, int grp, long long m, int n,
                                               float v) {
    const float* bias = p.g.bias[grp];
    if (bias) v += bias[n];
    if (p.T1) v += p.T1[(long long)p.idx1[m] * p.ldt + p.g.t_col[grp] + n];
    if (p.T2) v += p.T2[(long long)p.idx2[m] * p.ldt + p.g.t_col[grp] + n];
    long long off = m * p.ldc + p.g.c_col[grp] + n;
    if (p.act == 1) {
        if (p.Cpre) p.Cpre[off] = v;
        v = silu_f(v);
    }
    p.C[off] = p.accumulate ? p.C[off] + v : v;
}

__global__ void __launch_bounds__(256) gemm_fma_kernel(GemmArgs p) {
    __shared__ float As[2][BK][BM + 4];
    __shared__ float Bs[2][BK][BN + 4];
    // locate the group of this N tile
    int tn = blockIdx.x, grp = 0;
    while (grp + 1 < p.g.ngroups && tn >= p.tile_start[grp + 1]) ++grp;
    const int n0 = (tn - p.tile_start[grp]) * BN;
    const long long m0 = (long long)blockIdx.y * BM;
    const int K = p.g.K[grp], N = p.g.N[grp], ldb = p.g.ldb[grp];
    const float* A = p.A + p.g.a_col[grp];
    const float* B = p.g.B[grp];
    const int tid = threadIdx.x;
    // loader mapping: A tile 128 x 16 -> row tid / 2, 8 columns from (tid & 1) * 8
    const int a_r = tid >> 1, a_k = (tid & 1) * 8;
    // B tile 16 x 128 -> row tid / 16, 8 columns from (tid & 15) * 8
    const int b_k = tid >> 4, b_n = (tid & 15) * 8;
    float ra[8], rb[8];
    auto load = [&](int k0) {
        long long m = m0 + a_r;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            int k = k0 + a_k + q;
            ra[q] = (m < p.M && k < K) ? __ldg(A + m * p.lda + k) : 0.f;
        }
        int k = k0 + b_k;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            int n = n0 + b_n + q;
            rb[q] = (k < K && n < N) ? __ldg(B + (long long)k * ldb + n) : 0.f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int q = 0; q < 8; ++q) As[buf][a_k + q][a_r] = ra[q];
#pragma unroll
        for (int q = 0; q < 8; ++q) Bs[buf][b_k][b_n + q] = rb[q];
    };
    // compute mapping: thread (ty, tx) owns rows {ty*4 + i, 64 + ty*4 + i}, cols likewise
    const int ty = tid >> 4, tx = tid & 15;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    const int nk = (K + BK - 1) / BK;
    load(0);
    stash(0);
    __syncthreads();
    for (int kt = 0; kt < nk; ++kt) {
        int buf = kt & 1;
        if (kt + 1 < nk) load((kt + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[8];
            float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < nk) stash(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        long long m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n < N) epilogue_store(p, grp, m, n, acc[i][j]);
        }
    }
}

}  // namespace atom

using namespace atom;

extern "C" int atom_gemm_ex(const float* A, int64_t lda, int64_t M,
                            const atom_gemm_groups* groups, float* Cout, int64_t ldc, float* C_pre,
                            const float* T1, const float* T2, const int* idx1, const int* idx2,
                            int64_t ldt, int act, int accumulate, int precision, float* scratch,
                            int64_t scratch_floats, void* stream) {
    ATOM_REQUIRE(groups && groups->ngroups >= 1 && groups->ngroups <= 8, "1..8 groups");
    ATOM_REQUIRE(act == 0 || act == 1, "act must be 0 or 1");
    ATOM_REQUIRE(!T1 || idx1, "T1 needs idx1");
    ATOM_REQUIRE(!T2 || idx2, "T2 needs idx2");
    ATOM_REQUIRE(precision >= 0 && precision <= 3, "precision mode %d not available", precision);
    GemmArgs p;
    p.A = A; p.lda = lda; p.M = M; p.C = Cout; p.Cpre = C_pre; p.ldc = ldc;
    p.T1 = T1; p.T2 = T2; p.idx1 = idx1; p.idx2 = idx2; p.ldt = ldt;
    p.act = act; p.accumulate = accumulate; p.g = *groups;
    int tiles = 0;
    for (int g = 0; g < groups->ngroups; ++g) {
        ATOM_REQUIRE(groups->K[g] >= 0 && groups->N[g] >= 0 && groups->B[g],
                     "group %d: bad K/N/B", g);
        p.tile_start[g] = tiles;
        tiles += ceil_div(groups->N[g], BN);
    }
    p.tile_start[groups->ngroups] = tiles;
    if (M == 0 || tiles == 0) return ATOM_OK;
    ATOM_REQUIRE(ceil_div(M, BM) < 65536, "M too large");
    if (gemm_tc_supported(A, lda, groups, precision))
        return gemm_tc(A, lda, M, groups, Cout, ldc, C_pre, T1, T2, idx1, idx2, ldt, act,
                       accumulate, precision, scratch, scratch_floats, (cudaStream_t)stream);
    dim3 grid(tiles, ceil_div(M, BM));
    gemm_fma_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(p);
    ATOM_CHECK_LAUNCH("gemm");
    return ATOM_OK;
}

extern "C" int atom_gemm_gated(const float* Y, int64_t ldy, int64_t M,
                               const atom_gemm_groups* groups, int H, float* Cout, int64_t ldc,
                               int precision, float* scratch, int64_t scratch_floats,
                               void* stream) {
    ATOM_REQUIRE(groups && groups->ngroups >= 1 && groups->ngroups <= 8, "1..8 groups");
    ATOM_REQUIRE(H > 0 && H % 32 == 0, "gemm_gated: H must be a positive multiple of 32");
    if (precision < 2) {
        set_error("gemm_gated: precision %d has no gated tensor-core path; apply "
                  "atom_gate_fwd and atom_gemm_ex instead", precision);
        return ATOM_ERR_UNSUPPORTED;
    }
    for (int g = 0; g < groups->ngroups; ++g)
        ATOM_REQUIRE(groups->a_col[g] >= 2 * H && groups->a_col[g] % 32 == 0 &&
                         groups->a_col[g] + groups->K[g] <= 11 * H && groups->K[g] % 32 == 0,
                     "gemm_gated: group %d must read 32-aligned columns of rows 0..8 of Y", g);
    ATOM_REQUIRE(ldy >= 11 * H, "gemm_gated: ldy < 11 H");
    if (M == 0) return ATOM_OK;
    if (!gemm_tc_supported(Y, ldy, groups, precision)) {
        set_error("gemm_gated: operands not usable by the tensor-core kernel (alignment)");
        return ATOM_ERR_UNSUPPORTED;
    }
    return gemm_tc_gated(Y, ldy, M, groups, H, Cout, ldc, precision, scratch, scratch_floats,
                         (cudaStream_t)stream);
}

extern "C" int atom_gemm(const float* A, int64_t lda, int64_t M, const atom_gemm_groups* groups,
                         float* Cout, int64_t ldc, float* C_pre, const float* T1, const float* T2,
                         const int* idx1, const int* idx2, int64_t ldt, int act, int accumulate,
                         int precision, void* stream) {
    return atom_gemm_ex(A, lda, M, groups, Cout, ldc, C_pre, T1, T2, idx1, idx2, ldt, act,
                        accumulate, precision, nullptr, 0, stream);
}
