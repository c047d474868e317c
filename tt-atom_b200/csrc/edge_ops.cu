// Edge-side fused ops of the eSCN-MD edgewise block and their VJPs.
//
// Reference: tt_atom/edgewise.py:39-87 (forward chain), tt_atom/rotation.py:211-260 (rotation and
// its adjoints), tt_atom/activation.py:53-70 (gate), tt_atom/forces.py:104-130,352-418 (VJPs),
// tt_atom/geometry.py:262-278 (edge-degree init).
//
// Layout: node features x [N, 9, C] (standard (l, m) order); per-edge rows [E, 9, W] in m-primed
// order; packed Wigner coefficients coef [E, 35] (see common.cuh). Each kernel maps one warp to
// one edge (or one node for the CSR reductions) and each lane to 4 consecutive channels
// (float4), so every row access is a coalesced 512-byte transaction at C = 128. There are no
// float atomics: per-node sums walk the receiver / sender CSR in a fixed order, per-edge sums
// are warp reductions.
#include "common.cuh"

#ifndef ATOM_RBB_ROWS
#define ATOM_RBB_ROWS 0
#endif
#ifndef ATOM_RBB_LEAN
#define ATOM_RBB_LEAN 1
#endif
#ifndef ATOM_RIBE_LEAN
#define ATOM_RIBE_LEAN 0
#endif
// rotate_back_reduce: four received edges' rows loaded per step instead of two (63.0 -> 62.0 us
// per launch at E = 60,000; bit-identical)
#ifndef ATOM_RBR_QUAD
#define ATOM_RBR_QUAD 1
#endif
// rotate-in VJP (edge part) at C = 128 through the shared-memory ring (see
// rotate_in_bwd_edge_bulk_kernel): on by default; warps per block and ring depth per warp
#ifndef ATOM_RIBE_BULK
#define ATOM_RIBE_BULK 1
#endif
#ifndef ATOM_RIBE_BULK_WARPS
#define ATOM_RIBE_BULK_WARPS 4
#endif
#ifndef ATOM_RIBE_BULK_STAGES
#define ATOM_RIBE_BULK_STAGES 2
#endif
// rotate_in at C = 128 through the same kind of ring
#ifndef ATOM_RIN_BULK
#define ATOM_RIN_BULK 1
#endif
#ifndef ATOM_RIN_BULK_WARPS
#define ATOM_RIN_BULK_WARPS 7
#endif
#ifndef ATOM_RIN_BULK_STAGES
#define ATOM_RIN_BULK_STAGES 2
#endif

namespace atom {

__device__ __forceinline__ float4 f4(float a) { return make_float4(a, a, a, a); }
__device__ __forceinline__ void fma4(float4& acc, float s, const float4& v) {
    acc.x = fmaf(s, v.x, acc.x);
    acc.y = fmaf(s, v.y, acc.y);
    acc.z = fmaf(s, v.z, acc.z);
    acc.w = fmaf(s, v.w, acc.w);
}
__device__ __forceinline__ float4 mul4(const float4& a, const float4& b) {
    return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}
// acc = fmaf(a, b, acc) per component
__device__ __forceinline__ void fma4v(float4& acc, const float4& a, const float4& b) {
    acc.x = fmaf(a.x, b.x, acc.x);
    acc.y = fmaf(a.y, b.y, acc.y);
    acc.z = fmaf(a.z, b.z, acc.z);
    acc.w = fmaf(a.w, b.w, acc.w);
}
__device__ __forceinline__ float dot4(const float4& a, const float4& b) {
    return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, const float4& v) { *reinterpret_cast<float4*>(p) = v; }

// Column offset (in units of the row width 2C) of the radial slice multiplying m-primed row r:
// rows 0..2 -> slices 0..2 (m = 0), rows 3,4 and 5,6 -> slices 3,4 (m = 1), rows 7,8 -> slice 5.
__host__ __device__ constexpr int rad_slice(int r) {
    return r < 3 ? r : (r < 5 ? r : (r < 7 ? r - 2 : 5));
}

// Wigner row r applied to a node row set v[9]: out = sum_jj W[r][jj] v[l^2 + jj].
template <int R>
__device__ __forceinline__ float4 wrow(const float* w, const float4* v) {
    constexpr int l = row_deg(R), o = row_off(R), c0 = deg_col0(l);
    float4 acc = f4(0.f);
#pragma unroll
    for (int jj = 0; jj < 2 * l + 1; ++jj) fma4(acc, w[o + jj], v[c0 + jj]);
    return acc;
}

// Reduce-scatter across a warp: on return, lane l's v[0] holds the warp-wide sum of v[l]
// (31 shuffles for 32 sums instead of 32 x 5). v[] is clobbered.
__device__ __forceinline__ float warp_reduce_scatter32(float* v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; ++i) {
            float send = upper ? v[i] : v[i + s];
            float keep = upper ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return v[0];
}

// Sums over the warp of pc[0..34] written by lane 0..34 mapping: lanes 0-31 own entries 0-31,
// entries 32..34 are reduced with plain butterflies; returns lane-owned total for entry `lane`
// (and fills tail[3] on every lane).
__device__ __forceinline__ float warp_sum35(float* pc, float* tail) {
    tail[0] = warp_sum(pc[32]);
    tail[1] = warp_sum(pc[33]);
    tail[2] = warp_sum(pc[34]);
    return warp_reduce_scatter32(pc);
}

// wrow<R> for a row index known only after unrolling
__device__ __forceinline__ float4 wrow_rt(const float* w, const float4* v, int r) {
    const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
    float4 acc = f4(0.f);
#pragma unroll
    for (int jj = 0; jj < 5; ++jj)
        if (jj < 2 * l + 1) fma4(acc, w[o + jj], v[c0 + jj]);
    return acc;
}

__device__ __forceinline__ void load_coef(const float* __restrict__ coef, long long e, float* w) {
#pragma unroll
    for (int k = 0; k < kNnz; ++k) w[k] = __ldg(coef + e * kNnz + k);
}

// The same row for a warp that owns edge e: one coalesced load per lane (lanes 0-2 also load
// the last three), then register broadcasts instead of 35 loads per lane.
__device__ __forceinline__ void load_coef_warp(const float* __restrict__ coef, long long e,
                                               int lane, float* w) {
    const float* row = coef + e * kNnz;
    const float a = __ldg(row + lane);
    const float b = lane < kNnz - 32 ? __ldg(row + 32 + lane) : 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) w[k] = __shfl_sync(0xffffffffu, a, k);
#pragma unroll
    for (int k = 32; k < kNnz; ++k) w[k] = __shfl_sync(0xffffffffu, b, k - 32);
}

// -------------------------------------------------------------------------- rotate-in (fwd)
__global__ void __launch_bounds__(256) rotate_in_kernel(
    const float* __restrict__ x, const int* __restrict__ src, const int* __restrict__ tgt,
    const float* __restrict__ coef, long long E, int C, const float* __restrict__ rad,
    long long ldr, int rad_col, float* __restrict__ rot, float* __restrict__ A) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float w[kNnz];
    load_coef_warp(coef, e, lane, w);
    const float* xs = x + (long long)__ldg(src + e) * kNsph * C;
    const float* xt = x + (long long)__ldg(tgt + e) * kNsph * C;
    const int W2 = 2 * C;
    float* rowA = A + e * kNsph * W2;
    float* rowR = rot ? rot + e * kNsph * W2 : nullptr;
    const float* rr = rad ? rad + e * ldr + rad_col : nullptr;
    // source-channel half, then target-channel half of every row
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
        const float* xh = half ? xt : xs;
        const int ho = half * C;
        for (int c = lane * 4; c < C; c += 128) {
            float4 v[kNsph];
#pragma unroll
            for (int j = 0; j < kNsph; ++j) v[j] = ld4(xh + j * C + c);
#pragma unroll
            for (int r = 0; r < kNsph; ++r) {
                float4 o = wrow_rt(w, v, r);
                if (rowR) st4(rowR + r * W2 + ho + c, o);
                if (rr) o = mul4(o, ld4(rr + rad_slice(r) * W2 + ho + c));
                st4(rowA + r * W2 + ho + c, o);
            }
        }
    }
}

// ------------------------------------------------------------------------------- gate

__global__ void gate_fwd_kernel(const float* __restrict__ Y, long long E, int H,
                                float* __restrict__ G) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * H) return;
    long long e = t / H;
    int c = (int)(t - e * H);
    const float* y = Y + e * 11LL * H;
    float* g = G + e * 9LL * H;
    float s0 = sigmoid_gate(y[c]), s1 = sigmoid_gate(y[H + c]);
    g[c] = silu_gate(y[2 * H + c]);
#pragma unroll
    for (int r = 1; r < kNsph; ++r) g[r * H + c] = y[(2 + r) * H + c] * (gate_row(r) ? s1 : s0);
}

__global__ void gate_bwd_kernel(const float* __restrict__ Y, const float* __restrict__ gG,
                                long long E, int H, float* __restrict__ gY) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * H) return;
    long long e = t / H;
    int c = (int)(t - e * H);
    const float* y = Y + e * 11LL * H;
    const float* gg = gG + e * 9LL * H;
    float* gy = gY + e * 11LL * H;
    float s0 = sigmoid_f(y[c]), s1 = sigmoid_f(y[H + c]);
    gy[2 * H + c] = gg[c] * dsilu_f(y[2 * H + c]);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int r = 1; r < kNsph; ++r) {
        float g = gg[r * H + c];
        float v = y[(2 + r) * H + c];
        if (gate_row(r)) {
            gy[(2 + r) * H + c] = g * s1;
            a1 = fmaf(g, v, a1);
        } else {
            gy[(2 + r) * H + c] = g * s0;
            a0 = fmaf(g, v, a0);
        }
    }
    gy[c] = a0 * s0 * (1.f - s0);
    gy[H + c] = a1 * s1 * (1.f - s1);
}

// The same two kernels on four channels per thread (H a multiple of 4, 16-byte aligned rows):
// float4 loads and stores, the per-element expressions unchanged (bit-identical results).
template <class F>
__device__ __forceinline__ float4 map4(const float4& a, F f) {
    return make_float4(f(a.x), f(a.y), f(a.z), f(a.w));
}
__global__ void gate_fwd4_kernel(const float* __restrict__ Y, long long E, int H,
                                 float* __restrict__ G) {
    const int H4 = H >> 2;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * H4) return;
    const long long e = t / H4;
    const int c = (int)(t - e * H4) * 4;
    const float* y = Y + e * 11LL * H + c;
    float* g = G + e * 9LL * H + c;
    float4 yr[kNsph + 2];
#pragma unroll
    for (int r = 0; r < kNsph + 2; ++r) yr[r] = ld4(y + (long long)r * H);
    const float4 s0 = map4(yr[0], [](float v) { return sigmoid_gate(v); });
    const float4 s1 = map4(yr[1], [](float v) { return sigmoid_gate(v); });
    st4(g, map4(yr[2], [](float v) { return silu_gate(v); }));
#pragma unroll
    for (int r = 1; r < kNsph; ++r) st4(g + (long long)r * H, mul4(yr[2 + r], gate_row(r) ? s1 : s0));
}

__global__ void gate_bwd4_kernel(const float* __restrict__ Y, const float* __restrict__ gG,
                                 long long E, int H, float* __restrict__ gY) {
    const int H4 = H >> 2;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * H4) return;
    const long long e = t / H4;
    const int c = (int)(t - e * H4) * 4;
    const float* y = Y + e * 11LL * H + c;
    const float* gg = gG + e * 9LL * H + c;
    float* gy = gY + e * 11LL * H + c;
    float4 yr[kNsph + 2], gr[kNsph];
#pragma unroll
    for (int r = 0; r < kNsph + 2; ++r) yr[r] = ld4(y + (long long)r * H);
#pragma unroll
    for (int r = 0; r < kNsph; ++r) gr[r] = ld4(gg + (long long)r * H);
    const float4 s0 = map4(yr[0], [](float v) { return sigmoid_f(v); });
    const float4 s1 = map4(yr[1], [](float v) { return sigmoid_f(v); });
    st4(gy + 2LL * H, mul4(gr[0], map4(yr[2], [](float v) { return dsilu_f(v); })));
    float4 a0 = f4(0.f), a1 = f4(0.f);
#pragma unroll
    for (int r = 1; r < kNsph; ++r) {
        if (gate_row(r)) {
            st4(gy + (long long)(2 + r) * H, mul4(gr[r], s1));
            fma4v(a1, gr[r], yr[2 + r]);
        } else {
            st4(gy + (long long)(2 + r) * H, mul4(gr[r], s0));
            fma4v(a0, gr[r], yr[2 + r]);
        }
    }
    st4(gy, make_float4(a0.x * s0.x * (1.f - s0.x), a0.y * s0.y * (1.f - s0.y),
                        a0.z * s0.z * (1.f - s0.z), a0.w * s0.w * (1.f - s0.w)));
    st4(gy + H, make_float4(a1.x * s1.x * (1.f - s1.x), a1.y * s1.y * (1.f - s1.y),
                            a1.z * s1.z * (1.f - s1.z), a1.w * s1.w * (1.f - s1.w)));
}

// --------------------------------------------------------- rotate-back + receiver reduction
// acc[j] += s * sum over rows r of degree l(j) of W[r][j - l^2] * y[r]
__device__ __forceinline__ void rotate_back_acc(const float* w, const float4* y, float s,
                                                float4* acc) {
    // l = 0: row 0
    fma4(acc[0], s * w[row_off(0)], y[0]);
    // l = 1: rows 1, 3, 5 -> columns 1..3
#pragma unroll
    for (int jj = 0; jj < 3; ++jj) {
        fma4(acc[1 + jj], s * w[row_off(1) + jj], y[1]);
        fma4(acc[1 + jj], s * w[row_off(3) + jj], y[3]);
        fma4(acc[1 + jj], s * w[row_off(5) + jj], y[5]);
    }
    // l = 2: rows 2, 4, 6, 7, 8 -> columns 4..8
#pragma unroll
    for (int jj = 0; jj < 5; ++jj) {
        fma4(acc[4 + jj], s * w[row_off(2) + jj], y[2]);
        fma4(acc[4 + jj], s * w[row_off(4) + jj], y[4]);
        fma4(acc[4 + jj], s * w[row_off(6) + jj], y[6]);
        fma4(acc[4 + jj], s * w[row_off(7) + jj], y[7]);
        fma4(acc[4 + jj], s * w[row_off(8) + jj], y[8]);
    }
}

// Channel-parallel receiver reduction: one block of kCP = 128 threads per node, one channel per
// thread (looping when C > 128). Each output keeps the fma order of the warp-per-node float4
// form (edges in CSR order), so results are identical, but four times as many warps stay in
// flight, which this gather-bound reduction over ~30 edges per node needs at a few thousand
// nodes.
#ifndef ATOM_RBR_CP
#define ATOM_RBR_CP 128
#endif
constexpr int kCP = ATOM_RBR_CP;

// acc[j] += s * sum over rows r of degree l(j) of W[r][j - l^2] * y[r], one channel
__device__ __forceinline__ void rotate_back_acc_s(const float* w, const float* y, float s,
                                                  float* acc) {
    acc[0] = fmaf(s * w[row_off(0)], y[0], acc[0]);
#pragma unroll
    for (int jj = 0; jj < 3; ++jj) {
        acc[1 + jj] = fmaf(s * w[row_off(1) + jj], y[1], acc[1 + jj]);
        acc[1 + jj] = fmaf(s * w[row_off(3) + jj], y[3], acc[1 + jj]);
        acc[1 + jj] = fmaf(s * w[row_off(5) + jj], y[5], acc[1 + jj]);
    }
#pragma unroll
    for (int jj = 0; jj < 5; ++jj) {
        acc[4 + jj] = fmaf(s * w[row_off(2) + jj], y[2], acc[4 + jj]);
        acc[4 + jj] = fmaf(s * w[row_off(4) + jj], y[4], acc[4 + jj]);
        acc[4 + jj] = fmaf(s * w[row_off(6) + jj], y[6], acc[4 + jj]);
        acc[4 + jj] = fmaf(s * w[row_off(7) + jj], y[7], acc[4 + jj]);
        acc[4 + jj] = fmaf(s * w[row_off(8) + jj], y[8], acc[4 + jj]);
    }
}

// out[n] = resid[n] + sum over edges e received by n (CSR order) of env[e] * Wig(e)^T Y[e]
// The coefficients and envelopes of 32 received edges at a time are staged in shared memory
// (coalesced loads by the whole block) instead of 35 broadcast loads per thread and edge; two
// edges' rows are loaded before either is accumulated. The fma order per output is unchanged.
constexpr int kRbChunk = 32;
__global__ void __launch_bounds__(kCP) rotate_back_reduce_kernel(
    const float* __restrict__ Y, const float* __restrict__ coef, const float* __restrict__ env,
    long long N, int C, const int* __restrict__ recv_ptr, const float* __restrict__ resid,
    float* __restrict__ out) {
    __shared__ float sw[kRbChunk][kNnz + 1];      // 35 coefficients + the envelope
    const long long n = blockIdx.x;
    const int e0 = recv_ptr[n], e1 = recv_ptr[n + 1];
    for (int cb = 0; cb < C; cb += kCP) {
        const int c = cb + threadIdx.x;
        const bool active = c < C;
        float acc[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j)
            acc[j] = (active && resid) ? resid[(n * kNsph + j) * C + c] : 0.f;
        for (int eb = e0; eb < e1; eb += kRbChunk) {
            const int ne = min(kRbChunk, e1 - eb);
            __syncthreads();                       // the previous chunk has been read
            for (int i = threadIdx.x; i < ne * (kNnz + 1); i += kCP) {
                const int k = i / (kNnz + 1), j = i - k * (kNnz + 1);
                sw[k][j] = j < kNnz ? coef[(long long)(eb + k) * kNnz + j] : env[eb + k];
            }
            __syncthreads();
            if (!active) continue;
            int k = 0;
#if ATOM_RBR_QUAD
            // four edges' rows in flight before any is accumulated (same fma order)
            for (; k + 3 < ne; k += 4) {
                float yq[4][kNsph];
                const float* pa = Y + (long long)(eb + k) * kNsph * C + c;
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int r = 0; r < kNsph; ++r) yq[u][r] = pa[((long long)u * kNsph + r) * C];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    rotate_back_acc_s(sw[k + u], yq[u], sw[k + u][kNnz], acc);
            }
#endif
            for (; k + 1 < ne; k += 2) {
                float ya[kNsph], yb[kNsph];
                const float* pa = Y + (long long)(eb + k) * kNsph * C + c;
                const float* pb = pa + (long long)kNsph * C;
#pragma unroll
                for (int r = 0; r < kNsph; ++r) {
                    ya[r] = pa[r * C];
                    yb[r] = pb[r * C];
                }
                rotate_back_acc_s(sw[k], ya, sw[k][kNnz], acc);
                rotate_back_acc_s(sw[k + 1], yb, sw[k + 1][kNnz], acc);
            }
            if (k < ne) {
                float ya[kNsph];
                const float* pa = Y + (long long)(eb + k) * kNsph * C + c;
#pragma unroll
                for (int r = 0; r < kNsph; ++r) ya[r] = pa[r * C];
                rotate_back_acc_s(sw[k], ya, sw[k][kNnz], acc);
            }
        }
        if (active) {
#pragma unroll
            for (int j = 0; j < kNsph; ++j) out[(n * kNsph + j) * C + c] = acc[j];
        }
    }
}

// -------------------------------------------------------------- rotate-back VJP (per edge)
// two blocks per SM (<= 128 registers): 16 warps in flight instead of 8 at its natural 179
// registers; measured 0.96 -> 0.68 ms per step despite ~100 bytes of spills
#ifndef ATOM_RBB_MINB
#define ATOM_RBB_MINB 2
#endif
__global__ void __launch_bounds__(256, ATOM_RBB_MINB) rotate_back_bwd_kernel(
    const float* __restrict__ gx, const int* __restrict__ tgt, const float* __restrict__ coef,
    const float* __restrict__ env, const float* __restrict__ Y, long long E, int C,
    float* __restrict__ gY, float* __restrict__ g_env, float* __restrict__ g_coef) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float w[kNnz];
    load_coef_warp(coef, e, lane, w);
    float s = env[e];
    const float* gt = gx + (long long)tgt[e] * kNsph * C;
    const float* ye = Y + e * kNsph * C;
    float* ge = gY + e * kNsph * C;
    float pc[kNnz];
#pragma unroll
    for (int k = 0; k < kNnz; ++k) pc[k] = 0.f;
    float penv = 0.f;
    for (int c = lane * 4; c < C; c += 128) {
#if ATOM_RBB_ROWS
        // row by row: one Y row and one rotated row live at a time (same sums, same order)
        float4 v[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j) v[j] = ld4(gt + j * C + c);
#pragma unroll
        for (int r = 0; r < kNsph; ++r) {
            const float4 yr = ld4(ye + r * C + c);
            const float4 R = wrow_rt(w, v, r);
            penv += dot4(R, yr);
            st4(ge + r * C + c, make_float4(s * R.x, s * R.y, s * R.z, s * R.w));
            const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
#pragma unroll
            for (int jj = 0; jj < 5; ++jj)
                if (jj < 2 * l + 1) pc[o + jj] += dot4(v[c0 + jj], yr);
        }
#else
        float4 v[kNsph], y[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j) {
            v[j] = ld4(gt + j * C + c);
            y[j] = ld4(ye + j * C + c);
        }
        float4 R[kNsph];
        R[0] = wrow<0>(w, v); R[1] = wrow<1>(w, v); R[2] = wrow<2>(w, v);
        R[3] = wrow<3>(w, v); R[4] = wrow<4>(w, v); R[5] = wrow<5>(w, v);
        R[6] = wrow<6>(w, v); R[7] = wrow<7>(w, v); R[8] = wrow<8>(w, v);
#pragma unroll
        for (int r = 0; r < kNsph; ++r) {
            penv += dot4(R[r], y[r]);
            st4(ge + r * C + c, make_float4(s * R[r].x, s * R[r].y, s * R[r].z, s * R[r].w));
        }
#pragma unroll
        for (int r = 0; r < kNsph; ++r) {
            const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
            for (int jj = 0; jj < 2 * l + 1; ++jj) pc[o + jj] += dot4(v[c0 + jj], y[r]);
        }
#endif
    }
    penv = warp_sum(penv);
    float tail[3];
    const float mine = warp_sum35(pc, tail);
    g_coef[e * kNnz + lane] += s * mine;
    if (lane < 3) g_coef[e * kNnz + 32 + lane] += s * tail[lane];
    if (lane == 0) g_env[e] += penv;
}

// Lean form for C = 128 (one float4 per lane covers the row): the coefficients stay in the
// lanes that loaded them and are broadcast by shuffles when used, and each coefficient adjoint
// is summed over the warp as soon as its per-lane dot product exists, so neither the 35
// coefficients nor 35 partial sums occupy registers per lane: 80 registers, 3 blocks of 256
// per SM. Measured at E = 60,000: 0.155 -> 0.131 ms per launch (0.57 -> 0.68 of measured HBM),
// results bit-identical (the warp sums pair lanes in the same xor order as the reduce-scatter
// of the general kernel). The same treatment of rotate_in_bwd_edge measured slower (0.41 ->
// 0.42-0.53 ms) and is not enabled (ATOM_RIBE_LEAN).
#ifndef ATOM_RBB_LEAN_MINB
#define ATOM_RBB_LEAN_MINB 3
#endif
__global__ void __launch_bounds__(256, ATOM_RBB_LEAN_MINB) rotate_back_bwd_lean_kernel(
    const float* __restrict__ gx, const int* __restrict__ tgt, const float* __restrict__ coef,
    const float* __restrict__ env, const float* __restrict__ Y, long long E,
    float* __restrict__ gY, float* __restrict__ g_env, float* __restrict__ g_coef) {
    constexpr int C = 128;
    const long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (e >= E) return;
    const float* cr = coef + e * kNnz;
    const float wa = __ldg(cr + lane);
    const float wb = lane < kNnz - 32 ? __ldg(cr + 32 + lane) : 0.f;
    const float s = env[e];
    const int c = lane * 4;
    const float* gt = gx + (long long)tgt[e] * kNsph * C + c;
    const float* ye = Y + e * kNsph * C + c;
    float* ge = gY + e * kNsph * C + c;
    float4 v[kNsph], y[kNsph];
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        v[j] = ld4(gt + j * C);
        y[j] = ld4(ye + j * C);
    }
    float penv = 0.f, mine = 0.f, tail = 0.f;
#pragma unroll
    for (int r = 0; r < kNsph; ++r) {
        const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
        float4 R = f4(0.f);
#pragma unroll
        for (int jj = 0; jj < 2 * l + 1; ++jj) {
            const int k = o + jj;
            const float wk = __shfl_sync(0xffffffffu, k < 32 ? wa : wb, k & 31);
            fma4(R, wk, v[c0 + jj]);
        }
        penv += dot4(R, y[r]);
        st4(ge + r * C, make_float4(s * R.x, s * R.y, s * R.z, s * R.w));
#pragma unroll
        for (int jj = 0; jj < 2 * l + 1; ++jj) {
            const int k = o + jj;
            const float d = warp_sum(dot4(v[c0 + jj], y[r]));
            if (k < 32) {
                if (lane == k) mine = d;
            } else if (lane == k - 32) {
                tail = d;
            }
        }
    }
    penv = warp_sum(penv);
    g_coef[e * kNnz + lane] += s * mine;
    if (lane < kNnz - 32) g_coef[e * kNnz + 32 + lane] += s * tail;
    if (lane == 0) g_env[e] += penv;
}

// ------------------------------------------------------------ rotate-in VJP (edge part)
// launched in 64-thread blocks (finer block retirement: 1.89 -> 1.77 ms per step at 255
// registers), capped at 204 registers for 5 blocks per SM (76 bytes of spills; 1.74 -> 1.57 ms;
// 6 blocks per SM measured slower, 8 about the same)
#ifndef ATOM_RIBE_MINB
#define ATOM_RIBE_MINB 5
#endif
#ifndef ATOM_RIBE_THREADS
#define ATOM_RIBE_THREADS 64
#endif
__global__ void __launch_bounds__(ATOM_RIBE_THREADS, ATOM_RIBE_MINB) rotate_in_bwd_edge_kernel(
    const float* __restrict__ gA, const float* __restrict__ rot, const float* __restrict__ rad,
    long long ldr, int rad_col, const float* __restrict__ x, const int* __restrict__ src,
    const int* __restrict__ tgt, const float* __restrict__ coef, long long E, int C,
    float* __restrict__ g_rot, float* __restrict__ g_rad, float* __restrict__ g_coef) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    const int W2 = 2 * C;
    float w[kNnz];
    load_coef_warp(coef, e, lane, w);
    const float* ga = gA + e * kNsph * W2;
    const float* rr = rad + e * ldr + rad_col;
    float* gr = g_rot + e * kNsph * W2;
    float* grd = g_rad + e * ldr + rad_col;
    const float* xs = x + (long long)src[e] * kNsph * C;
    const float* xt = x + (long long)tgt[e] * kNsph * C;
    float pc[kNnz];
#pragma unroll
    for (int k = 0; k < kNnz; ++k) pc[k] = 0.f;
    // the source-channel half and the target-channel half of every row, one after the other
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
        const float* xh = half ? xt : xs;
        const int ho = half * C;
        for (int c = lane * 4; c < C; c += 128) {
            float4 v[kNsph];
#pragma unroll
            for (int j = 0; j < kNsph; ++j) v[j] = ld4(xh + j * C + c);
            float4 gsl[6];   // radial-slice adjoints
#pragma unroll
            for (int q = 0; q < 6; ++q) gsl[q] = f4(0.f);
#pragma unroll
            for (int r = 0; r < kNsph; ++r) {
                const int q = rad_slice(r);
                float4 gav = ld4(ga + r * W2 + ho + c);
                float4 g = mul4(gav, ld4(rr + q * W2 + ho + c));
                st4(gr + r * W2 + ho + c, g);
                // the rotated input of this row (before the radial multiplier): stored, or
                // recomputed from the node rows already in registers
                float4 rv = rot ? ld4(rot + e * kNsph * W2 + r * W2 + ho + c) : wrow_rt(w, v, r);
                float4 p = mul4(gav, rv);
                gsl[q].x += p.x; gsl[q].y += p.y; gsl[q].z += p.z; gsl[q].w += p.w;
                const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
#pragma unroll
                for (int jj = 0; jj < 2 * l + 1; ++jj) pc[o + jj] += dot4(g, v[c0 + jj]);
            }
#pragma unroll
            for (int q = 0; q < 6; ++q) st4(grd + q * W2 + ho + c, gsl[q]);
        }
    }
    float tail[3];
    const float mine = warp_sum35(pc, tail);
    g_coef[e * kNnz + lane] += mine;
    if (lane < 3) g_coef[e * kNnz + 32 + lane] += tail[lane];
}

// Lean form for C = 128, as rotate_back_bwd_lean_kernel: coefficients broadcast by shuffles
// from the lanes that loaded them, each coefficient adjoint summed over the warp per channel
// half as soon as it exists (the two halves' sums then added), so the per-lane state is the
// node rows and the radial-slice adjoints only.
#ifndef ATOM_RIBE_LEAN_MINB
#define ATOM_RIBE_LEAN_MINB 3
#endif
__global__ void __launch_bounds__(256, ATOM_RIBE_LEAN_MINB) rotate_in_bwd_edge_lean_kernel(
    const float* __restrict__ gA, const float* __restrict__ rot, const float* __restrict__ rad,
    long long ldr, int rad_col, const float* __restrict__ x, const int* __restrict__ src,
    const int* __restrict__ tgt, const float* __restrict__ coef, long long E,
    float* __restrict__ g_rot, float* __restrict__ g_rad, float* __restrict__ g_coef) {
    constexpr int C = 128, W2 = 2 * C;
    const long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (e >= E) return;
    const float* cr = coef + e * kNnz;
    const float wa = __ldg(cr + lane);
    const float wb = lane < kNnz - 32 ? __ldg(cr + 32 + lane) : 0.f;
    const int c = lane * 4;
    const float* ga = gA + e * kNsph * W2 + c;
    const float* rr = rad + e * ldr + rad_col + c;
    float* gr = g_rot + e * kNsph * W2 + c;
    float* grd = g_rad + e * ldr + rad_col + c;
    const float* xs = x + (long long)src[e] * kNsph * C + c;
    const float* xt = x + (long long)tgt[e] * kNsph * C + c;
    float mine = 0.f, tail = 0.f;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
        const float* xh = half ? xt : xs;
        const int ho = half * C;
        float4 v[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j) v[j] = ld4(xh + j * C);
        float4 gsl[6];
#pragma unroll
        for (int q = 0; q < 6; ++q) gsl[q] = f4(0.f);
        float hm = 0.f, ht = 0.f;
#pragma unroll
        for (int r = 0; r < kNsph; ++r) {
            const int q = rad_slice(r), l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
            const float4 gav = ld4(ga + r * W2 + ho);
            const float4 g = mul4(gav, ld4(rr + q * W2 + ho));
            st4(gr + r * W2 + ho, g);
            float4 rv;
            if (rot) {
                rv = ld4(rot + e * kNsph * W2 + r * W2 + ho + c);
            } else {
                rv = f4(0.f);
#pragma unroll
                for (int jj = 0; jj < 2 * l + 1; ++jj) {
                    const int k = o + jj;
                    fma4(rv, __shfl_sync(0xffffffffu, k < 32 ? wa : wb, k & 31), v[c0 + jj]);
                }
            }
            const float4 p = mul4(gav, rv);
            gsl[q].x += p.x; gsl[q].y += p.y; gsl[q].z += p.z; gsl[q].w += p.w;
#pragma unroll
            for (int jj = 0; jj < 2 * l + 1; ++jj) {
                const int k = o + jj;
                const float d = warp_sum(dot4(g, v[c0 + jj]));
                if (k < 32) {
                    if (lane == k) hm = d;
                } else if (lane == k - 32) {
                    ht = d;
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 6; ++q) st4(grd + q * W2 + ho, gsl[q]);
        mine += hm;
        tail += ht;
    }
    g_coef[e * kNnz + lane] += mine;
    if (lane < kNnz - 32) g_coef[e * kNnz + 32 + lane] += tail;
}

// ------------------------------------------------ per-warp streaming of edge rows (C = 128)
// Persistent kernels in which every warp walks edges first, first + stride, ... (stride = warps
// in the grid) with a ring of S slots in shared memory: lane 0 fetches an edge's rows with
// cp.async.bulk (each row set contiguous in global memory) into a slot as soon as the warp has
// finished reading the edge that used it, so the next edges' loads are in flight while the
// warp computes. Outputs go straight to global memory with 512-byte coalesced stores.
// Every wait on a slot is bounded (kRingWaitCycles of SM clock): on expiry the kernel records
// ATOM_EDGE_WAIT_CODE in the library's error word, waits (bounded again) for the copies it still
// has in flight, and the warp returns.
constexpr int kRingC = 128;
constexpr uint32_t kRowsX = kNsph * kRingC * 4;          // 4608 bytes: one node's rows
constexpr uint32_t kRowsE2 = kNsph * 2 * kRingC * 4;     // 9216: an edge row of width 2C
constexpr uint32_t kRowsRad = 6 * 2 * kRingC * 4;        // 6144: six radial slices of width 2C
constexpr long long kRingWaitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t sm_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sm_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait; false when the budget ran out
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, long long budget) {
    const long long t0 = clock64();
    while (!bar_try(b, parity))
        if (clock64() - t0 > budget) return false;
    return true;
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_u32(b)),
                 "r"(bytes)
                 : "memory");
}
// global -> shared bulk copy (both 16-byte aligned, bytes a multiple of 16), completing on b
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(sm_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(sm_u32(b))
        : "memory");
}

// All lanes of a warp: bounded wait for a slot's barrier to complete phase `parity`; on expiry
// lane 0 records ATOM_EDGE_WAIT_CODE in *err and every lane returns false.
__device__ __forceinline__ bool ring_wait(uint64_t* b, uint32_t parity, long long budget,
                                          int* err) {
    if (__all_sync(0xffffffffu, bar_wait(b, parity, budget))) return true;
    if ((threadIdx.x & 31) == 0) atomicCAS(err, 0, ATOM_EDGE_WAIT_CODE);
    __syncwarp();
    return false;
}

// Test hook: one warp waits, with the ring's own ring_wait, on a barrier that expects 16 bytes
// no copy will bring, so the wait runs out after `budget` SM clocks and records its code.
__global__ void ring_wait_selftest_kernel(long long budget, int* err) {
    __shared__ uint64_t b;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&b)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        bar_expect(&b, 16);
    }
    __syncwarp();
    ring_wait(&b, 0, budget, err);
}

// The warp's edge loop. pre(e): all lanes, before the wait for edge e's slot (register loads
// whose latency the wait hides); fetch(e, slot, bar): lane 0, announces and issues edge e's
// copies; body(e, slot): all lanes, reads the slot; post(e): all lanes, after the slot has been
// handed to the next fetch (register-only work and stores). Returns false if a wait expired.
template <int S, class Pre, class Fetch, class Body, class Post>
__device__ __forceinline__ bool warp_stream(uint8_t* ring, uint64_t* bar, uint32_t slot_bytes,
                                            long long first, long long stride, long long E,
                                            int* err, Pre pre, Fetch fetch, Body body, Post post) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
        for (int s = 0; s < S; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_u32(&bar[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < S; ++k)
            if (first + k * stride < E) fetch(first + k * stride, ring + (size_t)k * slot_bytes, &bar[k]);
    }
    __syncwarp();
    int it = 0;
    for (long long e = first; e < E; e += stride, ++it) {
        const int s = it % S;
        uint8_t* slot = ring + (size_t)s * slot_bytes;
        pre(e);
        if (!ring_wait(&bar[s], (uint32_t)(it / S) & 1u, kRingWaitCycles, err)) {
            // give up: let the copies still in flight land before the warp's shared memory can
            // be reused
            if (lane == 0) {
                for (int k = 0; k < S; ++k) {
                    const int j = it + k;
                    if (e + (long long)k * stride < E)
                        bar_wait(&bar[j % S], (uint32_t)(j / S) & 1u, kRingWaitCycles);
                }
            }
            __syncwarp();
            return false;
        }
        body(e, reinterpret_cast<const float*>(slot));
        // every lane is done reading the slot: order those reads before the async-proxy
        // writes of the next fetch into it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        const long long nxt = e + (long long)S * stride;
        if (lane == 0 && nxt < E) fetch(nxt, slot, &bar[s]);
        post(e);
    }
    return true;
}

// Launch shape of a streamed kernel: W warps per block, S slots per warp, one block per SM.
template <int W, int S>
struct RingShape {
    static constexpr int kWarps = W, kStages = S;
};

// rotate-in VJP (edge part) at C = 128, streamed: the gA row, its six radial slices and the
// source and target node rows (24 KB per edge) per slot; the arithmetic of
// rotate_in_bwd_edge_kernel (recomputed rotated rows), so the results are bit-identical.
// The coefficient adjoints accumulated by earlier kernels are read with the coefficients,
// before the slot wait, so the final read-modify-write is a store. Measured at E = 60,000 (CUDA
// events): 0.390 -> 0.308 ms per launch (4.80 -> 6.05 TB/s) with 4 warps of two slots per SM
// (8 x 1: 0.332, 6 x 1: 0.320; before the adjoint prefetch 4 x 2 and 8 x 1 both ~0.332, 3 x 3
// 0.397, 2 x 4 0.536).
constexpr uint32_t kRibeSlot = kRowsE2 + kRowsRad + 2 * kRowsX;
template <int W, int S>
__global__ void __launch_bounds__(32 * W, 1) rotate_in_bwd_edge_bulk_kernel(
    const float* __restrict__ gA, const float* __restrict__ rad, long long ldr, int rad_col,
    const float* __restrict__ x, const int* __restrict__ src, const int* __restrict__ tgt,
    const float* __restrict__ coef, long long E, float* __restrict__ g_rot,
    float* __restrict__ g_rad, float* __restrict__ g_coef, int* err) {
    constexpr int C = kRingC, W2 = 2 * C;
    extern __shared__ __align__(128) uint8_t ring_smem[];
    __shared__ uint64_t bars[W][S];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, c = lane * 4;
    float wa = 0.f, wb = 0.f, ga0 = 0.f, gb0 = 0.f;
    float pc[kNnz];
    auto pre = [&](long long e) {
        // this edge's coefficients and the coefficient adjoints accumulated so far, loaded
        // while the slot's rows are still arriving
        wa = __ldg(coef + e * kNnz + lane);
        wb = lane < kNnz - 32 ? __ldg(coef + e * kNnz + 32 + lane) : 0.f;
        ga0 = g_coef[e * kNnz + lane];
        gb0 = lane < kNnz - 32 ? g_coef[e * kNnz + 32 + lane] : 0.f;
    };
    auto fetch = [&](long long e, uint8_t* slot, uint64_t* b) {
        const long long ns = __ldg(src + e), nt = __ldg(tgt + e);
        bar_expect(b, kRibeSlot);
        bulk_g2s(slot, gA + e * kNsph * W2, kRowsE2, b);
        bulk_g2s(slot + kRowsE2, rad + e * ldr + rad_col, kRowsRad, b);
        bulk_g2s(slot + kRowsE2 + kRowsRad, x + ns * kNsph * C, kRowsX, b);
        bulk_g2s(slot + kRowsE2 + kRowsRad + kRowsX, x + nt * kNsph * C, kRowsX, b);
    };
    auto body = [&](long long e, const float* sl) {
        float w[kNnz];
#pragma unroll
        for (int k = 0; k < 32; ++k) w[k] = __shfl_sync(0xffffffffu, wa, k);
#pragma unroll
        for (int k = 32; k < kNnz; ++k) w[k] = __shfl_sync(0xffffffffu, wb, k - 32);
        const float* ga = sl;
        const float* rr = sl + kNsph * W2;
        float* gr = g_rot + e * kNsph * W2 + c;
        float* grd = g_rad + e * ldr + rad_col + c;
#pragma unroll
        for (int k = 0; k < kNnz; ++k) pc[k] = 0.f;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            const float* xh = sl + kNsph * W2 + 6 * W2 + half * kNsph * C + c;
            const int ho = half * C + c;
            float4 v[kNsph];
#pragma unroll
            for (int j = 0; j < kNsph; ++j) v[j] = ld4(xh + j * C);
            float4 gsl[6];
#pragma unroll
            for (int q = 0; q < 6; ++q) gsl[q] = f4(0.f);
#pragma unroll
            for (int r = 0; r < kNsph; ++r) {
                const int q = rad_slice(r);
                const float4 gav = ld4(ga + r * W2 + ho);
                const float4 g = mul4(gav, ld4(rr + q * W2 + ho));
                st4(gr + r * W2 + half * C, g);
                const float4 p = mul4(gav, wrow_rt(w, v, r));
                gsl[q].x += p.x; gsl[q].y += p.y; gsl[q].z += p.z; gsl[q].w += p.w;
                const int l = row_deg(r), o = row_off(r), c0 = deg_col0(l);
#pragma unroll
                for (int jj = 0; jj < 2 * l + 1; ++jj) pc[o + jj] += dot4(g, v[c0 + jj]);
            }
#pragma unroll
            for (int q = 0; q < 6; ++q) st4(grd + q * W2 + half * C, gsl[q]);
        }
    };
    auto post = [&](long long e) {
        float tail[3];
        const float mine = warp_sum35(pc, tail);
        g_coef[e * kNnz + lane] = ga0 + mine;
        if (lane < kNnz - 32) g_coef[e * kNnz + 32 + lane] = gb0 + tail[lane];
    };
    warp_stream<S>(ring_smem + (size_t)wid * S * kRibeSlot, bars[wid], kRibeSlot,
                   (long long)blockIdx.x * W + wid, (long long)gridDim.x * W, E, err, pre, fetch,
                   body, post);
}

// rotate-in at C = 128, streamed: the source and target node rows and the six radial slices
// (15 KB per edge) per slot; the arithmetic of rotate_in_kernel with rad (bit-identical).
// Measured at E = 60,000: 0.171 -> 0.150 ms per launch (6.27 TB/s) with 7 warps x 2 slots
// (8 x 1: 0.160, 6 x 2: 0.158, 12 x 1: 0.167, 4 x 2: 0.196, 4 x 3: 0.197). The same ring for rotate_back_bwd (gx and Y rows, 9 KB per edge) measured
// slower than its lean kernel at 24 warps per SM (0.116 -> 0.126 ms at 12 x 1, 0.160 at 8 x 2)
// and is not built (reading the lean kernel's adjoints early, as the VJP above does, made it
// slower too: 0.117 -> 0.127 ms); nor is a producer-warp ring for rotate_back_reduce (a node's received rows
// in chunks of 4-8 edges, 1-3 blocks per SM: 0.068-0.118 ms against 0.063 ms for the
// block-per-node kernel, whose many resident blocks hide the latency better).
constexpr uint32_t kRinSlot = 2 * kRowsX + kRowsRad;
template <int W, int S>
__global__ void __launch_bounds__(32 * W, 1) rotate_in_bulk_kernel(
    const float* __restrict__ x, const int* __restrict__ src, const int* __restrict__ tgt,
    const float* __restrict__ coef, long long E, const float* __restrict__ rad, long long ldr,
    int rad_col, float* __restrict__ A, int* err) {
    constexpr int C = kRingC, W2 = 2 * C;
    extern __shared__ __align__(128) uint8_t ring_smem[];
    __shared__ uint64_t bars[W][S];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, c = lane * 4;
    float wa = 0.f, wb = 0.f;
    auto pre = [&](long long e) {
        wa = __ldg(coef + e * kNnz + lane);
        wb = lane < kNnz - 32 ? __ldg(coef + e * kNnz + 32 + lane) : 0.f;
    };
    auto fetch = [&](long long e, uint8_t* slot, uint64_t* b) {
        const long long ns = __ldg(src + e), nt = __ldg(tgt + e);
        bar_expect(b, kRinSlot);
        bulk_g2s(slot, x + ns * kNsph * C, kRowsX, b);
        bulk_g2s(slot + kRowsX, x + nt * kNsph * C, kRowsX, b);
        bulk_g2s(slot + 2 * kRowsX, rad + e * ldr + rad_col, kRowsRad, b);
    };
    auto body = [&](long long e, const float* sl) {
        float w[kNnz];
#pragma unroll
        for (int k = 0; k < 32; ++k) w[k] = __shfl_sync(0xffffffffu, wa, k);
#pragma unroll
        for (int k = 32; k < kNnz; ++k) w[k] = __shfl_sync(0xffffffffu, wb, k - 32);
        float* rowA = A + e * kNsph * W2 + c;
        const float* rr = sl + 2 * kNsph * C + c;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            const float* xh = sl + half * kNsph * C + c;
            float4 v[kNsph];
#pragma unroll
            for (int j = 0; j < kNsph; ++j) v[j] = ld4(xh + j * C);
#pragma unroll
            for (int r = 0; r < kNsph; ++r) {
                float4 o = wrow_rt(w, v, r);
                o = mul4(o, ld4(rr + rad_slice(r) * W2 + half * C));
                st4(rowA + r * W2 + half * C, o);
            }
        }
    };
    auto post = [](long long) {};
    warp_stream<S>(ring_smem + (size_t)wid * S * kRinSlot, bars[wid], kRinSlot,
                   (long long)blockIdx.x * W + wid, (long long)gridDim.x * W, E, err, pre, fetch,
                   body, post);
}

// Launch of a streamed kernel: one block of W warps per SM (fewer when there are fewer edges),
// W * S slots of `slot` bytes of dynamic shared memory (attribute set once per device).
template <class K, class... Args>
static int launch_streamed(K kernel, int W, int S, uint32_t slot, long long E, void* stream,
                           const char* what, bool* attr_set, Args... args) {
    int dev = 0;
    cudaGetDevice(&dev);
    ATOM_REQUIRE(dev >= 0 && dev < 64, "%s: device id %d", what, dev);
    static int sms[64] = {};
    if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = (size_t)W * S * slot;
    if (!attr_set[dev]) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr_set[dev] = true;
    }
    int* err = device_error_word();
    ATOM_REQUIRE(err, "%s: no device error word", what);
    const long long blocks = (E + W - 1) / W;
    kernel<<<(unsigned)(blocks < sms[dev] ? blocks : sms[dev]), 32 * W, smem,
             (cudaStream_t)stream>>>(args..., err);
    return check_launch(what);
}

// acc[j] += sum over rows r of degree l(j) of W[r][j - l^2] * g[r]   (Wig^T g)
__device__ __forceinline__ void wig_t_acc(const float* w, const float4* g, float4* acc) {
    rotate_back_acc(w, g, 1.f, acc);
}

// ------------------------------------------------------------ rotate-in VJP (node part)
constexpr int kNbChunk = 16;   // edges per staged coefficient chunk (even: pairs stay aligned)
// kSplit warps share one node: warp w walks part w of the node's (received, then sent) edge
// list; the partial sums are added in warp order through shared memory.
// Capped at 128 registers (8 blocks per SM): 0.55 -> 0.44 ms per step against the 140-register
// build; 12 and 16 blocks per SM spill and measured slower.
template <int kSplit>
__global__ void __launch_bounds__(32 * kSplit, 8) rotate_in_bwd_node_kernel(
    const float* __restrict__ g_rot, const float* __restrict__ coef, long long N, int C,
    const int* __restrict__ recv_ptr, const int* __restrict__ send_ptr,
    const int* __restrict__ send_eid, int accumulate, float* __restrict__ gx) {
    extern __shared__ float4 part[];    // [kSplit - 1][9][32] per 128-channel chunk
    __shared__ float swc[kSplit][kNbChunk][kNnz];
    const long long n = blockIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int W2 = 2 * C;
    const int r0 = recv_ptr[n], r1 = recv_ptr[n + 1];
    const int s0 = send_ptr[n], s1 = send_ptr[n + 1];
    const int nr = r1 - r0, total = nr + (s1 - s0);
    const int chunk = (total + kSplit - 1) / kSplit;
    const int k0 = wid * chunk, k1 = min(total, k0 + chunk);
    // every lane runs every channel pass (the staging below needs the whole warp); lanes past
    // C only help stage
    for (int cb = 0; cb < C; cb += 128) {
        const int c = cb + lane * 4;
        const bool act = c < C;
        float4 acc[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j)
            acc[j] = (act && accumulate && wid == 0) ? ld4(gx + (n * kNsph + j) * C + c)
                                                      : f4(0.f);
        // this warp's edges in chunks of kNbChunk: their coefficient rows are staged in shared
        // memory by the whole warp (instead of 35 broadcast loads per lane and edge); edges are
        // still taken in pairs from k0 in list order, so the sums are unchanged
        float(*sw)[kNnz] = swc[wid];
        for (int kb = k0; kb < k1; kb += kNbChunk) {
            const int ne = min(kNbChunk, k1 - kb);
            __syncwarp();
            for (int i = lane; i < ne * kNnz; i += 32) {
                const int q = i / kNnz, j = i - q * kNnz, kk = kb + q;
                const int e = kk < nr ? r0 + kk : send_eid[s0 + kk - nr];
                sw[q][j] = coef[(long long)e * kNnz + j];
            }
            __syncwarp();
            if (!act) continue;
            int q = 0;
            for (; q + 1 < ne; q += 2) {
                const int k = kb + q;
                const int ea = k < nr ? r0 + k : send_eid[s0 + k - nr];
                const int eb = k + 1 < nr ? r0 + k + 1 : send_eid[s0 + k + 1 - nr];
                const float* ga = g_rot + (long long)ea * kNsph * W2 + (k < nr ? C : 0);
                const float* gb = g_rot + (long long)eb * kNsph * W2 + (k + 1 < nr ? C : 0);
                float4 g1[kNsph], g2[kNsph];
#pragma unroll
                for (int r = 0; r < kNsph; ++r) {
                    g1[r] = ld4(ga + r * W2 + c);
                    g2[r] = ld4(gb + r * W2 + c);
                }
                wig_t_acc(sw[q], g1, acc);
                wig_t_acc(sw[q + 1], g2, acc);
            }
            if (q < ne) {
                const int k = kb + q;
                const int ea = k < nr ? r0 + k : send_eid[s0 + k - nr];
                const float* ga = g_rot + (long long)ea * kNsph * W2 + (k < nr ? C : 0);
                float4 g1[kNsph];
#pragma unroll
                for (int r = 0; r < kNsph; ++r) g1[r] = ld4(ga + r * W2 + c);
                wig_t_acc(sw[q], g1, acc);
            }
        }
        if (kSplit > 1) {
            if (wid > 0) {
#pragma unroll
                for (int j = 0; j < kNsph; ++j) part[((wid - 1) * kNsph + j) * 32 + lane] = acc[j];
            }
            __syncthreads();
            if (wid == 0) {
#pragma unroll
                for (int q = 0; q < kSplit - 1; ++q)
#pragma unroll
                    for (int j = 0; j < kNsph; ++j) {
                        const float4 p = part[(q * kNsph + j) * 32 + lane];
                        acc[j].x += p.x; acc[j].y += p.y; acc[j].z += p.z; acc[j].w += p.w;
                    }
            }
            __syncthreads();
        }
        if (wid == 0 && act) {
#pragma unroll
            for (int j = 0; j < kNsph; ++j) st4(gx + (n * kNsph + j) * C + c, acc[j]);
        }
    }
}

// ----------------------------------------------------------------- edge-degree node init
__global__ void __launch_bounds__(256) edge_degree_fwd_kernel(
    const float* __restrict__ rad, long long ldr, const float* __restrict__ coef,
    const float* __restrict__ env, const float* __restrict__ l0, long long N, int C,
    const int* __restrict__ recv_ptr, float inv_rescale, float* __restrict__ x) {
    long long n = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (n >= N) return;
    for (int c = lane * 4; c < C; c += 128) {
        float4 acc[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j) acc[j] = f4(0.f);
        for (int e = recv_ptr[n]; e < recv_ptr[n + 1]; ++e) {
            float w[kNnz];
            load_coef(coef, e, w);
            float s = env[e] * inv_rescale;
            const float* re = rad + (long long)e * ldr;
            float4 y[kNsph];
            y[0] = ld4(re + c);
            y[1] = ld4(re + C + c);
            y[2] = ld4(re + 2 * C + c);
#pragma unroll
            for (int r = 3; r < kNsph; ++r) y[r] = f4(0.f);
            // only rows 0..2 (the m = 0 rows) carry the radial output
            fma4(acc[0], s * w[row_off(0)], y[0]);
#pragma unroll
            for (int jj = 0; jj < 3; ++jj) fma4(acc[1 + jj], s * w[row_off(1) + jj], y[1]);
#pragma unroll
            for (int jj = 0; jj < 5; ++jj) fma4(acc[4 + jj], s * w[row_off(2) + jj], y[2]);
        }
        float4 z = ld4(l0 + n * C + c);
        acc[0].x += z.x; acc[0].y += z.y; acc[0].z += z.z; acc[0].w += z.w;
#pragma unroll
        for (int j = 0; j < kNsph; ++j) st4(x + (n * kNsph + j) * C + c, acc[j]);
    }
}

__global__ void __launch_bounds__(256) edge_degree_bwd_kernel(
    const float* __restrict__ gx, const int* __restrict__ tgt, const float* __restrict__ rad,
    long long ldr, const float* __restrict__ coef, const float* __restrict__ env, long long E,
    int C, float inv_rescale, float* __restrict__ g_rad, long long ldg,
    float* __restrict__ g_env, float* __restrict__ g_coef) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float w[kNnz];
    load_coef(coef, e, w);
    float s = env[e] * inv_rescale;
    const float* gt = gx + (long long)tgt[e] * kNsph * C;
    const float* re = rad + e * ldr;
    float* gr = g_rad + e * ldg;
    float pc[9];   // rows 0..2 hold 1 + 3 + 5 = 9 coefficients (packed offsets 0..8)
#pragma unroll
    for (int k = 0; k < 9; ++k) pc[k] = 0.f;
    float penv = 0.f;
    for (int c = lane * 4; c < C; c += 128) {
        float4 v[kNsph];
#pragma unroll
        for (int j = 0; j < kNsph; ++j) v[j] = ld4(gt + j * C + c);
        float4 R0 = wrow<0>(w, v), R1 = wrow<1>(w, v), R2 = wrow<2>(w, v);
        float4 y0 = ld4(re + c), y1 = ld4(re + C + c), y2 = ld4(re + 2 * C + c);
        penv += dot4(R0, y0) + dot4(R1, y1) + dot4(R2, y2);
        st4(gr + c, make_float4(s * R0.x, s * R0.y, s * R0.z, s * R0.w));
        st4(gr + C + c, make_float4(s * R1.x, s * R1.y, s * R1.z, s * R1.w));
        st4(gr + 2 * C + c, make_float4(s * R2.x, s * R2.y, s * R2.z, s * R2.w));
        pc[0] += dot4(v[0], y0);
#pragma unroll
        for (int jj = 0; jj < 3; ++jj) pc[1 + jj] += dot4(v[1 + jj], y1);
#pragma unroll
        for (int jj = 0; jj < 5; ++jj) pc[4 + jj] += dot4(v[4 + jj], y2);
    }
    penv = warp_sum(penv);
#pragma unroll
    for (int k = 0; k < 9; ++k) pc[k] = warp_sum(pc[k]);
    if (lane == 0) {
        g_env[e] += penv * inv_rescale;
#pragma unroll
        for (int k = 0; k < 9; ++k) g_coef[e * kNnz + k] += s * pc[k];
    }
}

static int check_c(int C) {
    ATOM_REQUIRE(C > 0 && C % 4 == 0, "channel count must be a positive multiple of 4 (got %d)", C);
    return ATOM_OK;
}

}  // namespace atom

using namespace atom;

#define WARP_GRID(n) ceil_div((long long)(n) * 32, 256), 256, 0, (cudaStream_t)stream
#define CP_GRID(n) (unsigned)(n), kCP, 0, (cudaStream_t)stream

extern "C" int atom_ring_wait_selftest(int64_t budget_cycles, void* stream) {
    ATOM_REQUIRE(budget_cycles > 0 && budget_cycles <= kRingWaitCycles,
                 "atom_ring_wait_selftest: budget_cycles must be in [1, %lld]", kRingWaitCycles);
    int* err = device_error_word();
    ATOM_REQUIRE(err, "atom_ring_wait_selftest: no device error word");
    ring_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(budget_cycles, err);
    ATOM_CHECK_LAUNCH("atom_ring_wait_selftest");
    return ATOM_OK;
}

extern "C" int atom_rotate_in(const float* x, const int* src, const int* tgt, const float* coef,
                              int64_t E, int C, const float* rad, int64_t ldr, int rad_col,
                              float* rot, float* A, void* stream) {
    if (int s = check_c(C)) return s;
    ATOM_REQUIRE(!rad || (ldr % 4 == 0 && rad_col % 4 == 0), "rad must be float4-aligned");
    if (E == 0) return ATOM_OK;
#if ATOM_RIN_BULK
    if (C == 128 && rad && !rot && aligned16(x) && aligned16(rad)) {
        constexpr int W = ATOM_RIN_BULK_WARPS, S = ATOM_RIN_BULK_STAGES;
        static bool attr[64] = {};
        return launch_streamed(rotate_in_bulk_kernel<W, S>, W, S, kRinSlot, E, stream,
                               "rotate_in", attr, x, src, tgt, coef, (long long)E, rad,
                               (long long)ldr, rad_col, A);
    }
#endif
    rotate_in_kernel<<<WARP_GRID(E)>>>(x, src, tgt, coef, E, C, rad, ldr, rad_col, rot, A);
    ATOM_CHECK_LAUNCH("rotate_in");
    return ATOM_OK;
}

extern "C" int atom_gate_fwd(const float* Y, int64_t E, int H, float* G, void* stream) {
    ATOM_REQUIRE(H > 0, "H must be positive");
    if (E == 0) return ATOM_OK;
    if (H % 4 == 0 && aligned16(Y) && aligned16(G))
        gate_fwd4_kernel<<<ceil_div(E * (H / 4), 256), 256, 0, (cudaStream_t)stream>>>(Y, E, H, G);
    else
        gate_fwd_kernel<<<ceil_div(E * H, 256), 256, 0, (cudaStream_t)stream>>>(Y, E, H, G);
    ATOM_CHECK_LAUNCH("gate_fwd");
    return ATOM_OK;
}

extern "C" int atom_gate_bwd(const float* Y, const float* gG, int64_t E, int H, float* gY,
                             void* stream) {
    ATOM_REQUIRE(H > 0, "H must be positive");
    if (E == 0) return ATOM_OK;
    if (H % 4 == 0 && aligned16(Y) && aligned16(gG) && aligned16(gY))
        gate_bwd4_kernel<<<ceil_div(E * (H / 4), 256), 256, 0, (cudaStream_t)stream>>>(Y, gG, E, H,
                                                                                    gY);
    else
        gate_bwd_kernel<<<ceil_div(E * H, 256), 256, 0, (cudaStream_t)stream>>>(Y, gG, E, H, gY);
    ATOM_CHECK_LAUNCH("gate_bwd");
    return ATOM_OK;
}

extern "C" int atom_rotate_back_reduce(const float* Y, const float* coef, const float* env,
                                       int64_t N, int C, const int* recv_ptr,
                                       const float* resid, float* out, void* stream) {
    if (int s = check_c(C)) return s;
    if (N == 0) return ATOM_OK;
    rotate_back_reduce_kernel<<<CP_GRID(N)>>>(Y, coef, env, N, C, recv_ptr, resid, out);
    ATOM_CHECK_LAUNCH("rotate_back_reduce");
    return ATOM_OK;
}

extern "C" int atom_rotate_back_bwd(const float* gx, const int* tgt, const float* coef,
                                    const float* env, const float* Y, int64_t E, int C,
                                    float* gY, float* g_env, float* g_coef, void* stream) {
    if (int s = check_c(C)) return s;
    if (E == 0) return ATOM_OK;
#if ATOM_RBB_LEAN
    if (C == 128)
        rotate_back_bwd_lean_kernel<<<WARP_GRID(E)>>>(gx, tgt, coef, env, Y, E, gY, g_env,
                                                      g_coef);
    else
#endif
        rotate_back_bwd_kernel<<<WARP_GRID(E)>>>(gx, tgt, coef, env, Y, E, C, gY, g_env, g_coef);
    ATOM_CHECK_LAUNCH("rotate_back_bwd");
    return ATOM_OK;
}

extern "C" int atom_rotate_in_bwd_edge(const float* gA, const float* rot, const float* rad,
                                       int64_t ldr, int rad_col, const float* x, const int* src,
                                       const int* tgt, const float* coef, int64_t E, int C,
                                       float* g_rot, float* g_rad, float* g_coef, void* stream) {
    if (int s = check_c(C)) return s;
    ATOM_REQUIRE(ldr % 4 == 0 && rad_col % 4 == 0, "rad must be float4-aligned");
    if (E == 0) return ATOM_OK;
#if ATOM_RIBE_BULK
    // the streamed kernel: C = 128, rows recomputed (rot NULL), every fetched row 16-byte aligned
    if (C == 128 && !rot && aligned16(gA) && aligned16(rad) && aligned16(x)) {
        constexpr int W = ATOM_RIBE_BULK_WARPS, S = ATOM_RIBE_BULK_STAGES;
        static bool attr[64] = {};
        return launch_streamed(rotate_in_bwd_edge_bulk_kernel<W, S>, W, S, kRibeSlot, E, stream,
                               "rotate_in_bwd_edge", attr, gA, rad, (long long)ldr, rad_col, x,
                               src, tgt, coef, (long long)E, g_rot, g_rad, g_coef);
    }
#endif
#if ATOM_RIBE_LEAN
    if (C == 128) {
        rotate_in_bwd_edge_lean_kernel<<<WARP_GRID(E)>>>(gA, rot, rad, ldr, rad_col, x, src, tgt,
                                                         coef, E, g_rot, g_rad, g_coef);
        ATOM_CHECK_LAUNCH("rotate_in_bwd_edge");
        return ATOM_OK;
    }
#endif
    rotate_in_bwd_edge_kernel<<<ceil_div((long long)E * 32, ATOM_RIBE_THREADS), ATOM_RIBE_THREADS,
                                0, (cudaStream_t)stream>>>(gA, rot, rad, ldr, rad_col, x, src, tgt, coef,
                                                E, C, g_rot, g_rad, g_coef);
    ATOM_CHECK_LAUNCH("rotate_in_bwd_edge");
    return ATOM_OK;
}

extern "C" int atom_rotate_in_bwd_node(const float* g_rot, const float* coef, int64_t N, int C,
                                       const int* recv_ptr, const int* send_ptr,
                                       const int* send_eid, int accumulate, float* gx,
                                       void* stream) {
    if (int s = check_c(C)) return s;
    if (N == 0) return ATOM_OK;
    // two warps per node: measured 0.82 -> 0.59 ms per step against one (four: 0.67)
    constexpr int kSplit = 2;
    rotate_in_bwd_node_kernel<kSplit><<<(unsigned)N, 32 * kSplit,
                                        (kSplit - 1) * kNsph * 32 * sizeof(float4),
                                        (cudaStream_t)stream>>>(g_rot, coef, N, C, recv_ptr,
                                                                send_ptr, send_eid, accumulate, gx);
    ATOM_CHECK_LAUNCH("rotate_in_bwd_node");
    return ATOM_OK;
}

extern "C" int atom_edge_degree_fwd(const float* rad, int64_t ldr, const float* coef,
                                    const float* env, const float* l0, int64_t N, int C,
                                    const int* recv_ptr, float rescale, float* x, void* stream) {
    if (int s = check_c(C)) return s;
    ATOM_REQUIRE(ldr % 4 == 0, "rad must be float4-aligned");
    if (N == 0) return ATOM_OK;
    edge_degree_fwd_kernel<<<WARP_GRID(N)>>>(rad, ldr, coef, env, l0, N, C, recv_ptr,
                                             1.0f / rescale, x);
    ATOM_CHECK_LAUNCH("edge_degree_fwd");
    return ATOM_OK;
}

extern "C" int atom_edge_degree_bwd(const float* gx, const int* tgt, const float* rad,
                                    int64_t ldr, const float* coef, const float* env, int64_t E,
                                    int C, float rescale, float* g_rad, int64_t ldg,
                                    float* g_env, float* g_coef, void* stream) {
    if (int s = check_c(C)) return s;
    ATOM_REQUIRE(ldr % 4 == 0 && ldg % 4 == 0, "rad/g_rad must be float4-aligned");
    if (E == 0) return ATOM_OK;
    edge_degree_bwd_kernel<<<WARP_GRID(E)>>>(gx, tgt, rad, ldr, coef, env, E, C, 1.0f / rescale,
                                             g_rad, ldg, g_env, g_coef);
    ATOM_CHECK_LAUNCH("edge_degree_bwd");
    return ATOM_OK;
}
