// Node-side ops: equivariant RMS norm (tt_atom/norm.py:24-111; VJP tt_atom/forces.py:73-98), the
// radial LayerNorm+SiLU and its VJP (tt_atom/so2.py:101-163), per-node sphere-grid projections
// (tt_atom/grid.py:63-76; VJP tt_atom/forces.py:230-252), SiLU VJP and deterministic sums.
#include "common.cuh"

namespace atom {

// Degree of standard-order coefficient j and its balance weight 1/(2l+1)/(lmax+1), lmax = 2.
__host__ __device__ constexpr int coef_deg(int j) { return j == 0 ? 0 : (j < 4 ? 1 : 2); }
__device__ __forceinline__ float bal_w(int j) {
    return coef_deg(j) == 0 ? (1.0f / 3.0f) : (coef_deg(j) == 1 ? (1.0f / 9.0f) : (1.0f / 15.0f));
}

// ---------------------------------------------------------------------- RMS norm SH (fwd)
// One warp per node; the node's 9 x C values are held in registers (C <= 256).
template <int CPL>  // channels per lane = C / 32 rounded up
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(
    const float* __restrict__ x, long long N, int C, const float* __restrict__ aw,
    const float* __restrict__ ab, const float* __restrict__ add0, float eps,
    float* __restrict__ out) {
    long long n = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (n >= N) return;
    const float* xn = x + n * kNsph * C;
    float v[kNsph][CPL];
    float s0 = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j)
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            int c = lane + 32 * q;
            v[j][q] = c < C ? xn[j * C + c] : 0.f;
        }
#pragma unroll
    for (int q = 0; q < CPL; ++q) s0 += v[0][q];
    float mean0 = warp_sum(s0) / C;
#pragma unroll
    for (int q = 0; q < CPL; ++q)
        if (lane + 32 * q < C) v[0][q] -= mean0;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < CPL; ++q) t = fmaf(v[j][q], v[j][q], t);
        ss = fmaf(bal_w(j), t, ss);
    }
    float fn = rsqrtf(warp_sum(ss) / C + eps);
    float* on = out + n * kNsph * C;
#pragma unroll
    for (int j = 0; j < kNsph; ++j)
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            int c = lane + 32 * q;
            if (c >= C) continue;
            float r = v[j][q] * (fn * aw[coef_deg(j) * C + c]);
            if (j == 0) {
                r += ab[c];
                if (add0) r += add0[n * C + c];
            }
            on[j * C + c] = r;
        }
}

// ---------------------------------------------------------------------- RMS norm SH (VJP)
// out_j = xc_j * fn * a_j (+ bias on j = 0); u_j = g_j * a_j;
// d/dxc_j = fn u_j - fn^3 bal_j xc_j S / C with S = sum_j sum_c u_j xc_j; the l = 0 centring
// subtracts the channel mean of the j = 0 adjoint.
template <int CPL>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const float* __restrict__ x, const float* __restrict__ g, long long N, int C,
    const float* __restrict__ aw, float eps, int accumulate, float* __restrict__ gx) {
    long long n = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (n >= N) return;
    const float* xn = x + n * kNsph * C;
    const float* gn = g + n * kNsph * C;
    // x, the adjoint and the affine weights are all loaded up front (one memory round trip)
    float v[kNsph][CPL], u[kNsph][CPL];
    float s0 = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j)
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            int c = lane + 32 * q;
            v[j][q] = c < C ? xn[j * C + c] : 0.f;
            u[j][q] = c < C ? gn[j * C + c] * aw[coef_deg(j) * C + c] : 0.f;
        }
#pragma unroll
    for (int q = 0; q < CPL; ++q) s0 += v[0][q];
    float mean0 = warp_sum(s0) / C;
#pragma unroll
    for (int q = 0; q < CPL; ++q)
        if (lane + 32 * q < C) v[0][q] -= mean0;
    float ss = 0.f, S = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            int c = lane + 32 * q;
            t = fmaf(v[j][q], v[j][q], t);
            if (c < C) S = fmaf(u[j][q], v[j][q], S);
        }
        ss = fmaf(bal_w(j), t, ss);
    }
    float fn = rsqrtf(warp_sum(ss) / C + eps);
    S = warp_sum(S);
    float k3 = fn * fn * fn * S / C;
    float* go = gx + n * kNsph * C;
    float gsum0 = 0.f;
    float gr0[CPL];
#pragma unroll
    for (int j = 0; j < kNsph; ++j)
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            int c = lane + 32 * q;
            if (c >= C) {
                if (j == 0) gr0[q] = 0.f;
                continue;
            }
            float r = fn * u[j][q] - k3 * bal_w(j) * v[j][q];
            if (j == 0) {
                gr0[q] = r;
                gsum0 += r;
            } else {
                go[j * C + c] = accumulate ? go[j * C + c] + r : r;
            }
        }
    float m = warp_sum(gsum0) / C;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
        int c = lane + 32 * q;
        if (c < C) go[c] = accumulate ? go[c] + (gr0[q] - m) : (gr0[q] - m);
    }
}

// -------------------------------------------------------------- LayerNorm + SiLU (fwd, VJP)
// One warp per (row, group).
__global__ void ln_silu_fwd_kernel(const float* __restrict__ X, long long rows, long long ld,
                                   int groups, int W, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float eps,
                                   float* __restrict__ Y) {
    long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= rows * groups) return;
    long long row = wid / groups;
    int g = (int)(wid - row * groups);
    const float* xr = X + row * ld + (long long)g * W;
    float* yr = Y + row * ld + (long long)g * W;
    const float* ga = gamma + g * W;
    const float* be = beta + g * W;
    float s = 0.f;
    for (int c = lane; c < W; c += 32) s += xr[c];
    float mean = warp_sum(s) / W;
    float v = 0.f;
    for (int c = lane; c < W; c += 32) {
        float d = xr[c] - mean;
        v = fmaf(d, d, v);
    }
    float rstd = rsqrtf(warp_sum(v) / W + eps);
    for (int c = lane; c < W; c += 32) yr[c] = silu_gate((xr[c] - mean) * rstd * ga[c] + be[c]);
}

// Register-resident forms for W = 128 * NV: each lane holds its 4 * NV elements of the row as
// float4s, so X, gY, gamma and beta are each read once (the loops above re-read the row per
// pass).
__device__ __forceinline__ float4 ldv4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float f4get(const float4& v, int k) {
    return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

template <int NV>
__global__ void ln_silu_fwd_v_kernel(const float* __restrict__ X, long long rows, long long ld,
                                     int groups, const float* __restrict__ gamma,
                                     const float* __restrict__ beta, float eps,
                                     float* __restrict__ Y) {
    constexpr int W = 128 * NV;
    long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= rows * groups) return;
    long long row = wid / groups;
    int g = (int)(wid - row * groups);
    const float* xr = X + row * ld + (long long)g * W;
    float* yr = Y + row * ld + (long long)g * W;
    float x[NV][4];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float4 t = ldv4(xr + 128 * i + 4 * lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) { x[i][k] = f4get(t, k); s += x[i][k]; }
    }
    const float mean = warp_sum(s) / W;
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) { const float d = x[i][k] - mean; v = fmaf(d, d, v); }
    const float rstd = rsqrtf(warp_sum(v) / W + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = 128 * i + 4 * lane;
        const float4 ga = ldv4(gamma + g * W + c), be = ldv4(beta + g * W + c);
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = silu_gate((x[i][k] - mean) * rstd * f4get(ga, k) + f4get(be, k));
        *reinterpret_cast<float4*>(yr + c) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// gY and dX may alias (in-place): all of a row is read before any of it is written
template <int NV>
__global__ void ln_silu_bwd_v_kernel(const float* __restrict__ X, const float* gY,
                                     long long rows, long long ld, int groups,
                                     const float* __restrict__ gamma,
                                     const float* __restrict__ beta, float eps, float* dX) {
    constexpr int W = 128 * NV;
    long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= rows * groups) return;
    long long row = wid / groups;
    int g = (int)(wid - row * groups);
    const float* xr = X + row * ld + (long long)g * W;
    const float* gr = gY + row * ld + (long long)g * W;
    float* dr = dX + row * ld + (long long)g * W;
    float x[NV][4], gy[NV][4];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = 128 * i + 4 * lane;
        const float4 t = ldv4(xr + c), u = ldv4(gr + c);
#pragma unroll
        for (int k = 0; k < 4; ++k) { x[i][k] = f4get(t, k); gy[i][k] = f4get(u, k); s += x[i][k]; }
    }
    const float mean = warp_sum(s) / W;
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) { const float d = x[i][k] - mean; v = fmaf(d, d, v); }
    const float rstd = rsqrtf(warp_sum(v) / W + eps);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c = 128 * i + 4 * lane;
        const float4 ga = ldv4(gamma + g * W + c), be = ldv4(beta + g * W + c);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            x[i][k] = (x[i][k] - mean) * rstd;                     // now x-hat
            const float gk = f4get(ga, k);
            gy[i][k] = gy[i][k] * dsilu_gate(x[i][k] * gk + f4get(be, k)) * gk;
            s1 += gy[i][k];
            s2 = fmaf(gy[i][k], x[i][k], s2);
        }
    }
    s1 = warp_sum(s1) / W;
    s2 = warp_sum(s2) / W;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = rstd * (gy[i][k] - s1 - x[i][k] * s2);
        *reinterpret_cast<float4*>(dr + 128 * i + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// gY and dX may alias (in-place)
__global__ void ln_silu_bwd_kernel(const float* __restrict__ X, const float* gY,
                                   long long rows, long long ld, int groups, int W,
                                   const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float eps, float* dX) {
    long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= rows * groups) return;
    long long row = wid / groups;
    int g = (int)(wid - row * groups);
    const float* xr = X + row * ld + (long long)g * W;
    const float* gr = gY + row * ld + (long long)g * W;
    float* dr = dX + row * ld + (long long)g * W;
    const float* ga = gamma + g * W;
    const float* be = beta + g * W;
    float s = 0.f;
    for (int c = lane; c < W; c += 32) s += xr[c];
    float mean = warp_sum(s) / W;
    float v = 0.f;
    for (int c = lane; c < W; c += 32) {
        float d = xr[c] - mean;
        v = fmaf(d, d, v);
    }
    float rstd = rsqrtf(warp_sum(v) / W + eps);
    float s1 = 0.f, s2 = 0.f;
    for (int c = lane; c < W; c += 32) {
        float xh = (xr[c] - mean) * rstd;
        float gy = gr[c] * dsilu_gate(xh * ga[c] + be[c]) * ga[c];
        s1 += gy;
        s2 = fmaf(gy, xh, s2);
    }
    s1 = warp_sum(s1) / W;
    s2 = warp_sum(s2) / W;
    for (int c = lane; c < W; c += 32) {
        float xh = (xr[c] - mean) * rstd;
        float gy = gr[c] * dsilu_gate(xh * ga[c] + be[c]) * ga[c];
        dr[c] = rstd * (gy - s1 - xh * s2);
    }
}

// ------------------------------------------------------------------- per-node projection
// out[n, q, c] (+)= sum_p M[q, p] in[n, p, c]; one thread per (n, c); M staged in shared memory.
// PT > 0: P known at compile time, so the P inputs of a thread stay in registers (PT = 0: any
// P <= 64, runtime loop).
template <int PT>
__global__ void node_project_kernel(const float* __restrict__ in, long long N, int Pr, int C,
                                    const float* __restrict__ M, int Q, int trans,
                                    int accumulate, float* __restrict__ out) {
    const int P = PT > 0 ? PT : Pr;
    extern __shared__ float sm[];   // [Q * P]
    for (int i = threadIdx.x; i < Q * P; i += blockDim.x) {
        int q = i / P, p = i - q * P;
        sm[i] = trans ? M[p * Q + q] : M[q * P + p];
    }
    __syncthreads();
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * C) return;
    long long n = t / C;
    int c = (int)(t - n * C);
    const float* xin = in + n * (long long)P * C + c;
    float* o = out + n * (long long)Q * C + c;
    float v[PT > 0 ? PT : 64];
#pragma unroll
    for (int p = 0; p < (PT > 0 ? PT : 64); ++p)
        if (PT > 0 || p < P) v[p] = xin[(long long)p * C];
    for (int q = 0; q < Q; ++q) {
        float acc = 0.f;
        const float* mr = sm + q * P;
#pragma unroll
        for (int p = 0; p < (PT > 0 ? PT : 64); ++p)
            if (PT > 0 || p < P) acc = fmaf(mr[p], v[p], acc);
        o[(long long)q * C] = accumulate ? o[(long long)q * C] + acc : acc;
    }
}

// The same on four channels per thread (C a multiple of 4, 16-byte aligned rows): one float4
// per input row, the outputs accumulated over p in the same order (bit-identical results).
// N = 2,000, C = 128 (CUDA events): 9 -> 42 rows 13.0 -> 11.1 us, 42 -> 9 rows (the kernel
// below) 12.5 -> 10.8 us.
template <int PT>
__global__ void node_project4_kernel(const float* __restrict__ in, long long N, int C,
                                     const float* __restrict__ M, int Q, int trans,
                                     int accumulate, float* __restrict__ out) {
    constexpr int P = PT;
    extern __shared__ float sm[];   // [Q * P]
    for (int i = threadIdx.x; i < Q * P; i += blockDim.x) {
        int q = i / P, p = i - q * P;
        sm[i] = trans ? M[p * Q + q] : M[q * P + p];
    }
    __syncthreads();
    const int C4 = C >> 2;
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * C4) return;
    long long n = t / C4;
    int c = (int)(t - n * C4) * 4;
    const float* xin = in + n * (long long)P * C + c;
    float* o = out + n * (long long)Q * C + c;
    float4 v[P];
#pragma unroll
    for (int p = 0; p < P; ++p) v[p] = *reinterpret_cast<const float4*>(xin + (long long)p * C);
    for (int q = 0; q < Q; ++q) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const float* mr = sm + q * P;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const float m = mr[p];
            acc.x = fmaf(m, v[p].x, acc.x);
            acc.y = fmaf(m, v[p].y, acc.y);
            acc.z = fmaf(m, v[p].z, acc.z);
            acc.w = fmaf(m, v[p].w, acc.w);
        }
        float4* op = reinterpret_cast<float4*>(o + (long long)q * C);
        if (accumulate) {
            const float4 b = *op;
            acc = make_float4(b.x + acc.x, b.y + acc.y, b.z + acc.z, b.w + acc.w);
        }
        *op = acc;
    }
}

// Many inputs, few outputs (P = 42 grid points -> Q = 9 coefficients): the loop over p is the
// outer one, with the Q float4 accumulators in registers, so no p row is held; each output
// still sums over p in ascending order (bit-identical to node_project_kernel).
template <int P, int Q>
__global__ void node_project4_pq_kernel(const float* __restrict__ in, long long N, int C,
                                        const float* __restrict__ M, int trans, int accumulate,
                                        float* __restrict__ out) {
    __shared__ float sm[Q * P];
    for (int i = threadIdx.x; i < Q * P; i += blockDim.x) {
        int q = i / P, p = i - q * P;
        sm[i] = trans ? M[p * Q + q] : M[q * P + p];
    }
    __syncthreads();
    const int C4 = C >> 2;
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * C4) return;
    long long n = t / C4;
    int c = (int)(t - n * C4) * 4;
    const float* xin = in + n * (long long)P * C + c;
    float* o = out + n * (long long)Q * C + c;
    float4 acc[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 6
    for (int p = 0; p < P; ++p) {
        const float4 v = *reinterpret_cast<const float4*>(xin + (long long)p * C);
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const float m = sm[q * P + p];
            acc[q].x = fmaf(m, v.x, acc[q].x);
            acc[q].y = fmaf(m, v.y, acc[q].y);
            acc[q].z = fmaf(m, v.z, acc[q].z);
            acc[q].w = fmaf(m, v.w, acc[q].w);
        }
    }
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        float4* op = reinterpret_cast<float4*>(o + (long long)q * C);
        float4 a = acc[q];
        if (accumulate) {
            const float4 b = *op;
            a = make_float4(b.x + a.x, b.y + a.y, b.z + a.z, b.w + a.w);
        }
        *op = a;
    }
}

// g and out may alias (in-place)
__global__ void silu_bwd_kernel(const float* g, const float* __restrict__ pre, long long n,
                                float* out) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = g[t] * dsilu_gate(pre[t]);
}

// four elements per thread (16-byte aligned arrays, n a multiple of 4); g and out may alias
__global__ void silu_bwd4_kernel(const float4* g, const float4* __restrict__ pre, long long n4,
                                 float4* out) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n4) return;
    const float4 a = g[t], b = pre[t];
    out[t] = make_float4(a.x * dsilu_gate(b.x), a.y * dsilu_gate(b.y), a.z * dsilu_gate(b.z),
                         a.w * dsilu_gate(b.w));
}

// Deterministic segmented sum: one 256-thread block per segment, strided partials then a
// fixed shared-memory tree.
__global__ void segment_sum_kernel(const float* __restrict__ v, long long n,
                                   const int* __restrict__ seg_ptr, float* __restrict__ out) {
    __shared__ float sh[256];
    long long b = seg_ptr ? seg_ptr[blockIdx.x] : 0;
    long long e = seg_ptr ? seg_ptr[blockIdx.x + 1] : n;
    float s = 0.f;
    for (long long i = b + threadIdx.x; i < e; i += 256) s += v[i];
    sh[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[blockIdx.x] = sh[0];
}

}  // namespace atom

namespace atom {
// ------------------------------------------------- RMS norm SH, channel-parallel (C = 128)
// One block of 128 threads per node, one channel per thread, the channel sums taken by a
// block reduction: four times the warps of the warp-per-node form, which a latency-bound pass
// over a few thousand nodes needs. Same arithmetic per element.
constexpr int kRC = 128;

// Sums of a and b over the block's 128 threads (all threads get both).
__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red) {
    a = warp_sum(a);
    b = warp_sum(b);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();                         // red may still be read from an earlier call
    if (lane == 0) red[w] = make_float2(a, b);
    __syncthreads();
    float2 t = red[0];
#pragma unroll
    for (int i = 1; i < kRC / 32; ++i) {
        t.x += red[i].x;
        t.y += red[i].y;
    }
    return t;
}

__global__ void __launch_bounds__(kRC) rmsnorm_fwd_c128_kernel(
    const float* __restrict__ x, const float* __restrict__ aw, const float* __restrict__ ab,
    const float* __restrict__ add0, float eps, float* __restrict__ out) {
    __shared__ float2 red[kRC / 32];
    constexpr int C = kRC;
    const long long n = blockIdx.x;
    const int c = threadIdx.x;
    const float* xn = x + n * kNsph * C + c;
    float v[kNsph];
#pragma unroll
    for (int j = 0; j < kNsph; ++j) v[j] = xn[j * C];
    const float mean0 = block_sum2(v[0], 0.f, red).x / C;
    v[0] -= mean0;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) ss = fmaf(bal_w(j), v[j] * v[j], ss);
    const float fn = rsqrtf(block_sum2(ss, 0.f, red).x / C + eps);
    float* on = out + n * kNsph * C + c;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        float r = v[j] * (fn * aw[coef_deg(j) * C + c]);
        if (j == 0) {
            r += ab[c];
            if (add0) r += add0[n * C + c];
        }
        on[j * C] = r;
    }
}

__global__ void __launch_bounds__(kRC) rmsnorm_bwd_c128_kernel(
    const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ aw,
    float eps, int accumulate, float* __restrict__ gx) {
    __shared__ float2 red[kRC / 32];
    constexpr int C = kRC;
    const long long n = blockIdx.x;
    const int c = threadIdx.x;
    const float* xn = x + n * kNsph * C + c;
    const float* gn = g + n * kNsph * C + c;
    float v[kNsph], u[kNsph];
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        v[j] = xn[j * C];
        u[j] = gn[j * C] * aw[coef_deg(j) * C + c];
    }
    const float mean0 = block_sum2(v[0], 0.f, red).x / C;
    v[0] -= mean0;
    float ss = 0.f, S = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        ss = fmaf(bal_w(j), v[j] * v[j], ss);
        S = fmaf(u[j], v[j], S);
    }
    const float2 t = block_sum2(ss, S, red);
    const float fn = rsqrtf(t.x / C + eps);
    const float k3 = fn * fn * fn * t.y / C;
    float* go = gx + n * kNsph * C + c;
    float r0 = 0.f;
#pragma unroll
    for (int j = 0; j < kNsph; ++j) {
        const float r = fn * u[j] - k3 * bal_w(j) * v[j];
        if (j == 0) {
            r0 = r;
        } else {
            go[j * C] = accumulate ? go[j * C] + r : r;
        }
    }
    const float m = block_sum2(r0, 0.f, red).x / C;
    go[0] = accumulate ? go[0] + (r0 - m) : (r0 - m);
}
}  // namespace atom

using namespace atom;

#define WARP_GRID(n) ceil_div((long long)(n) * 32, 256), 256, 0, (cudaStream_t)stream

extern "C" int atom_rmsnorm_sh_fwd(const float* x, int64_t N, int C, const float* aw,
                                   const float* ab, const float* add0, float eps, float* out,
                                   void* stream) {
    ATOM_REQUIRE(C > 0 && C <= 256, "rmsnorm: C must be in [1, 256] (got %d)", C);
    if (N == 0) return ATOM_OK;
    if (C == kRC)
        rmsnorm_fwd_c128_kernel<<<(unsigned)N, kRC, 0, (cudaStream_t)stream>>>(x, aw, ab, add0,
                                                                             eps, out);
    else if (C <= 32)
        rmsnorm_fwd_kernel<1><<<WARP_GRID(N)>>>(x, N, C, aw, ab, add0, eps, out);
    else if (C <= 64)
        rmsnorm_fwd_kernel<2><<<WARP_GRID(N)>>>(x, N, C, aw, ab, add0, eps, out);
    else if (C <= 128)
        rmsnorm_fwd_kernel<4><<<WARP_GRID(N)>>>(x, N, C, aw, ab, add0, eps, out);
    else
        rmsnorm_fwd_kernel<8><<<WARP_GRID(N)>>>(x, N, C, aw, ab, add0, eps, out);
    ATOM_CHECK_LAUNCH("rmsnorm_sh_fwd");
    return ATOM_OK;
}

extern "C" int atom_rmsnorm_sh_bwd(const float* x, const float* g, int64_t N, int C,
                                   const float* aw, float eps, int accumulate, float* gx,
                                   void* stream) {
    ATOM_REQUIRE(C > 0 && C <= 256, "rmsnorm: C must be in [1, 256] (got %d)", C);
    if (N == 0) return ATOM_OK;
    if (C == kRC)
        rmsnorm_bwd_c128_kernel<<<(unsigned)N, kRC, 0, (cudaStream_t)stream>>>(x, g, aw, eps,
                                                                             accumulate, gx);
    else if (C <= 32)
        rmsnorm_bwd_kernel<1><<<WARP_GRID(N)>>>(x, g, N, C, aw, eps, accumulate, gx);
    else if (C <= 64)
        rmsnorm_bwd_kernel<2><<<WARP_GRID(N)>>>(x, g, N, C, aw, eps, accumulate, gx);
    else if (C <= 128)
        rmsnorm_bwd_kernel<4><<<WARP_GRID(N)>>>(x, g, N, C, aw, eps, accumulate, gx);
    else
        rmsnorm_bwd_kernel<8><<<WARP_GRID(N)>>>(x, g, N, C, aw, eps, accumulate, gx);
    ATOM_CHECK_LAUNCH("rmsnorm_sh_bwd");
    return ATOM_OK;
}

extern "C" int atom_ln_silu_fwd(const float* X, int64_t rows, int64_t ld, int groups, int W,
                                const float* gamma, const float* beta, float eps, float* Y,
                                void* stream) {
    ATOM_REQUIRE(groups > 0 && W > 0 && ld >= (int64_t)groups * W, "ln_silu: bad shape");
    if (rows == 0) return ATOM_OK;
    const bool v4 = ld % 4 == 0 && aligned16(X) && aligned16(Y) && aligned16(gamma) &&
                    aligned16(beta);
    if (v4 && W == 128)
        ln_silu_fwd_v_kernel<1><<<WARP_GRID(rows * groups)>>>(X, rows, ld, groups, gamma, beta,
                                                              eps, Y);
    else if (v4 && W == 256)
        ln_silu_fwd_v_kernel<2><<<WARP_GRID(rows * groups)>>>(X, rows, ld, groups, gamma, beta,
                                                              eps, Y);
    else
        ln_silu_fwd_kernel<<<WARP_GRID(rows * groups)>>>(X, rows, ld, groups, W, gamma, beta,
                                                         eps, Y);
    ATOM_CHECK_LAUNCH("ln_silu_fwd");
    return ATOM_OK;
}

extern "C" int atom_ln_silu_bwd(const float* X, const float* gY, int64_t rows, int64_t ld,
                                int groups, int W, const float* gamma, const float* beta,
                                float eps, float* dX, void* stream) {
    ATOM_REQUIRE(groups > 0 && W > 0 && ld >= (int64_t)groups * W, "ln_silu: bad shape");
    if (rows == 0) return ATOM_OK;
    const bool v4 = ld % 4 == 0 && aligned16(X) && aligned16(gY) && aligned16(dX) &&
                    aligned16(gamma) && aligned16(beta);
    if (v4 && W == 128)
        ln_silu_bwd_v_kernel<1><<<WARP_GRID(rows * groups)>>>(X, gY, rows, ld, groups, gamma,
                                                              beta, eps, dX);
    else if (v4 && W == 256)
        ln_silu_bwd_v_kernel<2><<<WARP_GRID(rows * groups)>>>(X, gY, rows, ld, groups, gamma,
                                                              beta, eps, dX);
    else
        ln_silu_bwd_kernel<<<WARP_GRID(rows * groups)>>>(X, gY, rows, ld, groups, W, gamma,
                                                         beta, eps, dX);
    ATOM_CHECK_LAUNCH("ln_silu_bwd");
    return ATOM_OK;
}

extern "C" int atom_node_project(const float* in, int64_t N, int P, int C, const float* M,
                                 int Q, int trans, int accumulate, float* out, void* stream) {
    ATOM_REQUIRE(P > 0 && P <= 64 && Q > 0 && Q <= 64 && C > 0, "node_project: bad shape");
    if (N == 0) return ATOM_OK;
    const unsigned grid = ceil_div(N * C, 128);
    const size_t sh = Q * P * sizeof(float);
    cudaStream_t st = (cudaStream_t)stream;
    if (P == 9 && C % 4 == 0 && aligned16(in) && aligned16(out)) {
        node_project4_kernel<9><<<ceil_div(N * (C / 4), 128), 128, sh, st>>>(in, N, C, M, Q, trans,
                                                                           accumulate, out);
    } else if (P == 9)
        node_project_kernel<9><<<grid, 128, sh, st>>>(in, N, P, C, M, Q, trans, accumulate, out);
    else if (P == 42 && Q == 9 && C % 4 == 0 && aligned16(in) && aligned16(out))
        node_project4_pq_kernel<42, 9><<<ceil_div(N * (C / 4), 128), 128, 0, st>>>(
            in, N, C, M, trans, accumulate, out);
    else if (P == 42)
        node_project_kernel<42><<<grid, 128, sh, st>>>(in, N, P, C, M, Q, trans, accumulate, out);
    else
        node_project_kernel<0><<<grid, 128, sh, st>>>(in, N, P, C, M, Q, trans, accumulate, out);
    ATOM_CHECK_LAUNCH("node_project");
    return ATOM_OK;
}

extern "C" int atom_silu_bwd(const float* g, const float* pre, int64_t n, float* out,
                             void* stream) {
    if (n == 0) return ATOM_OK;
    if (n % 4 == 0 && aligned16(g) && aligned16(pre) && aligned16(out))
        silu_bwd4_kernel<<<ceil_div(n / 4, 256), 256, 0, (cudaStream_t)stream>>>(
            reinterpret_cast<const float4*>(g), reinterpret_cast<const float4*>(pre), n / 4,
            reinterpret_cast<float4*>(out));
    else
        silu_bwd_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(g, pre, n, out);
    ATOM_CHECK_LAUNCH("silu_bwd");
    return ATOM_OK;
}

extern "C" int atom_segment_sum(const float* v, int64_t n, const int* seg_ptr, int nseg,
                                float* out, void* stream) {
    ATOM_REQUIRE(nseg >= 1 && (seg_ptr || nseg == 1), "segment_sum: bad segments");
    segment_sum_kernel<<<nseg, 256, 0, (cudaStream_t)stream>>>(v, n, seg_ptr, out);
    ATOM_CHECK_LAUNCH("segment_sum");
    return ATOM_OK;
}

namespace atom {

__global__ void node_embed_kernel(const int* __restrict__ Z, const int* __restrict__ sys,
                                  const float* __restrict__ sphere,
                                  const float* __restrict__ sysemb, long long N, int C,
                                  float* __restrict__ out) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * C) return;
    long long n = t / C;
    int c = (int)(t - n * C);
    int s = sys ? sys[n] : 0;
    out[t] = sphere[(long long)Z[n] * C + c] + sysemb[(long long)s * C + c];
}

__global__ void edge_species_kernel(const int* __restrict__ Z, const int* __restrict__ src,
                                    const int* __restrict__ tgt, long long E,
                                    int* __restrict__ zs, int* __restrict__ zt) {
    long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    zs[e] = Z[src[e]];
    zt[e] = Z[tgt[e]];
}

}  // namespace atom

extern "C" int atom_node_embed(const int* Z, const int* sys_id, const float* sphere,
                               const float* sysemb, int64_t N, int C, float* out, void* stream) {
    if (N == 0) return ATOM_OK;
    node_embed_kernel<<<ceil_div(N * C, 256), 256, 0, (cudaStream_t)stream>>>(Z, sys_id, sphere,
                                                                            sysemb, N, C, out);
    ATOM_CHECK_LAUNCH("node_embed");
    return ATOM_OK;
}

extern "C" int atom_edge_species(const int* Z, const int* src, const int* tgt, int64_t E,
                                 int* zs, int* zt, void* stream) {
    if (E == 0) return ATOM_OK;
    edge_species_kernel<<<ceil_div(E, 256), 256, 0, (cudaStream_t)stream>>>(Z, src, tgt, E, zs, zt);
    ATOM_CHECK_LAUNCH("edge_species");
    return ATOM_OK;
}

// ------------------------------------------------------------ spectral feed-forward gate
// Natural (l, m) coefficient order, lmax = 2 (tt_atom/spectral.py:168-188):
//   out[n, 0] = silu(h[n, 0]);  out[n, j] = h[n, j] * sigmoid(gat[n, (l(j) - 1) H + c]), j >= 1,
// where gat is the post-SiLU scalar gating [N, 2H]. One thread per (n, c).
namespace atom {

__global__ void spectral_gate_fwd_kernel(const float* __restrict__ h,
                                         const float* __restrict__ gat, long long N, int H,
                                         float* __restrict__ out) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * H) return;
    long long n = t / H;
    int c = (int)(t - n * H);
    const float* hn = h + n * 9LL * H;
    float* on = out + n * 9LL * H;
    float s1 = sigmoid_f(gat[n * 2 * H + c]), s2 = sigmoid_f(gat[n * 2 * H + H + c]);
    on[c] = silu_f(hn[c]);
#pragma unroll
    for (int j = 1; j < 9; ++j) on[j * H + c] = hn[j * H + c] * (j < 4 ? s1 : s2);
}

// VJP: g_h [N, 9H] and g_gat [N, 2H] (adjoint of the post-SiLU gating) from g_out.
__global__ void spectral_gate_bwd_kernel(const float* __restrict__ h,
                                         const float* __restrict__ gat,
                                         const float* __restrict__ g_out, long long N, int H,
                                         float* __restrict__ g_h, float* __restrict__ g_gat) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * H) return;
    long long n = t / H;
    int c = (int)(t - n * H);
    const float* hn = h + n * 9LL * H;
    const float* gn = g_out + n * 9LL * H;
    float* ghn = g_h + n * 9LL * H;
    float s1 = sigmoid_f(gat[n * 2 * H + c]), s2 = sigmoid_f(gat[n * 2 * H + H + c]);
    ghn[c] = gn[c] * dsilu_f(hn[c]);
    float a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int j = 1; j < 9; ++j) {
        float g = gn[j * H + c];
        if (j < 4) {
            ghn[j * H + c] = g * s1;
            a1 = fmaf(g, hn[j * H + c], a1);
        } else {
            ghn[j * H + c] = g * s2;
            a2 = fmaf(g, hn[j * H + c], a2);
        }
    }
    g_gat[n * 2 * H + c] = a1 * s1 * (1.f - s1);
    g_gat[n * 2 * H + H + c] = a2 * s2 * (1.f - s2);
}

}  // namespace atom

extern "C" int atom_spectral_gate_fwd(const float* h, const float* gat, int64_t N, int H,
                                      float* out, void* stream) {
    if (N == 0) return ATOM_OK;
    spectral_gate_fwd_kernel<<<ceil_div(N * H, 256), 256, 0, (cudaStream_t)stream>>>(h, gat, N,
                                                                                   H, out);
    ATOM_CHECK_LAUNCH("spectral_gate_fwd");
    return ATOM_OK;
}

extern "C" int atom_spectral_gate_bwd(const float* h, const float* gat, const float* g_out,
                                      int64_t N, int H, float* g_h, float* g_gat, void* stream) {
    if (N == 0) return ATOM_OK;
    spectral_gate_bwd_kernel<<<ceil_div(N * H, 256), 256, 0, (cudaStream_t)stream>>>(
        h, gat, g_out, N, H, g_h, g_gat);
    ATOM_CHECK_LAUNCH("spectral_gate_bwd");
    return ATOM_OK;
}
