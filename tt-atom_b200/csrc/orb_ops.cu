// Orb-v3 (conservative) kernels: edge features and their VJP, row RMSNorm, sigmoid attention
// gates, CSR segment sums, the message-passing VJP, and node mean / broadcast.
//
// Reference: tt_atom/orb_geometry.py:29-139 (Bessel x real SH l <= 3 x cutoff, closed-form VJP),
// tt_atom/orb_model.py:69-82 (cutoff p = 4), :92-124 (RMSNorm eps 1e-6), :189-266 (attention
// interaction), :307-338 (energy head), tt_atom/orb_forces.py:67-148 (VJPs).
//
// Edge convention: the graph is stored UMA-style (src, tgt; receiver-major on tgt). Orb's
// senders are tgt and its receivers are src, so Orb's edge vector pos[receiver] - pos[sender]
// + shift equals the stored edge vector pos[src] - pos[tgt] + shift.
#include "common.cuh"

namespace atom {

constexpr float kSqrt3 = 1.7320508075688772f;
constexpr float kSqrt15 = 3.872983346207417f;

// Real spherical harmonics l = 0..3 of a unit vector, component normalisation (each degree
// scaled by sqrt(2l + 1)).
__device__ __forceinline__ void sh_l3(float x, float y, float z, float* s) {
    const float y2 = y * y, x2z2 = x * x + z * z;
    const float s20 = kSqrt3 * x * z, s21 = kSqrt3 * x * y, s22 = y2 - 0.5f * x2z2;
    const float s23 = kSqrt3 * y * z, s24 = 0.5f * kSqrt3 * (z * z - x * x);
    const float a = sqrtf(5.0f / 6.0f), c = sqrtf(3.0f / 8.0f), r5 = sqrtf(5.0f);
    const float m1 = kSqrt3, m2 = sqrtf(5.0f), m3 = sqrtf(7.0f);
    s[0] = 1.0f;
    s[1] = m1 * x; s[2] = m1 * y; s[3] = m1 * z;
    s[4] = m2 * s20; s[5] = m2 * s21; s[6] = m2 * s22; s[7] = m2 * s23; s[8] = m2 * s24;
    s[9] = m3 * a * (s20 * z + s24 * x);
    s[10] = m3 * r5 * s20 * y;
    s[11] = m3 * c * (4.0f * y2 - x2z2) * x;
    s[12] = m3 * 0.5f * y * (2.0f * y2 - 3.0f * x2z2);
    s[13] = m3 * c * z * (4.0f * y2 - x2z2);
    s[14] = m3 * r5 * s24 * y;
    s[15] = m3 * a * (s24 * z - s20 * x);
}

// Gradient of sum_m g[m] sh_m(x, y, z) with respect to (x, y, z), from the derivatives of the
// closed forms above.
__device__ __forceinline__ void sh_l3_vjp(float x, float y, float z, const float* g, float* out) {
    const float m1 = kSqrt3, m2 = sqrtf(5.0f), m3 = sqrtf(7.0f);
    const float b = sqrtf(5.0f / 6.0f) * kSqrt3 * 0.5f, c = sqrtf(3.0f / 8.0f);
    float q[16];
    q[0] = 0.f;
    for (int i = 1; i < 4; ++i) q[i] = g[i] * m1;
    for (int i = 4; i < 9; ++i) q[i] = g[i] * m2;
    for (int i = 9; i < 16; ++i) q[i] = g[i] * m3;
    float gx = q[1], gy = q[2], gz = q[3];
    gx += q[4] * kSqrt3 * z;                 gz += q[4] * kSqrt3 * x;
    gx += q[5] * kSqrt3 * y;                 gy += q[5] * kSqrt3 * x;
    gx -= q[6] * x; gy += q[6] * 2.0f * y;   gz -= q[6] * z;
    gy += q[7] * kSqrt3 * z;                 gz += q[7] * kSqrt3 * y;
    gx -= q[8] * kSqrt3 * x;                 gz += q[8] * kSqrt3 * z;
    gx += q[9] * b * (3.0f * z * z - 3.0f * x * x);
    gz += q[9] * b * 6.0f * x * z;
    gx += q[10] * kSqrt15 * y * z; gy += q[10] * kSqrt15 * x * z; gz += q[10] * kSqrt15 * x * y;
    gx += q[11] * c * (4.0f * y * y - 3.0f * x * x - z * z);
    gy += q[11] * c * 8.0f * x * y;
    gz -= q[11] * c * 2.0f * x * z;
    gx -= q[12] * 3.0f * x * y;
    gy += q[12] * (3.0f * y * y - 1.5f * (x * x + z * z));
    gz -= q[12] * 3.0f * y * z;
    gx -= q[13] * c * 2.0f * x * z;
    gy += q[13] * c * 8.0f * y * z;
    gz += q[13] * c * (4.0f * y * y - x * x - 3.0f * z * z);
    gx -= q[14] * kSqrt15 * x * y;
    gy += q[14] * 0.5f * kSqrt15 * (z * z - x * x);
    gz += q[14] * kSqrt15 * z * y;
    gx -= q[15] * b * 6.0f * x * z;
    gz += q[15] * b * (3.0f * z * z - 3.0f * x * x);
    out[0] = gx; out[1] = gy; out[2] = gz;
}

// Polynomial cutoff p = 4 and its derivative with respect to r.
__device__ __forceinline__ float orb_cutoff(float r, float rmax, float* d) {
    const float p = 4.f, A = (p + 1.f) * (p + 2.f) / 2.f, B = p * (p + 2.f),
                Cc = p * (p + 1.f) / 2.f;
    if (!(r < rmax)) {
        *d = 0.f;
        return 0.f;
    }
    float q = r / rmax, q2 = q * q, q3 = q2 * q, q4 = q2 * q2;
    *d = (-A * p * q3 + B * (p + 1.f) * q4 - Cc * (p + 2.f) * q4 * q) / rmax;
    return 1.f - A * q4 + B * q4 * q - Cc * q4 * q2;
}

__device__ __forceinline__ void edge_vector(const float* pos, int s, int t, const float* shifts,
                                            const int* img, long long e, float* v) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        float d = pos[s * 3 + k] - pos[t * 3 + k];
        v[k] = shifts ? d + shifts[(img ? img[e] : 0) * 3 + k] : d;
    }
}

// One warp per edge; every lane evaluates the (cheap) basis, lanes write 4 columns each.
__global__ void orb_feat_kernel(const float* __restrict__ pos, const int* __restrict__ src,
                                const int* __restrict__ tgt, const int* __restrict__ img,
                                const float* __restrict__ shifts, long long E, float rmax, int nb,
                                float* __restrict__ feat, float* __restrict__ cut,
                                float* __restrict__ ev) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float v[3];
    edge_vector(pos, src[e], tgt[e], shifts, img, e, v);
    float r = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    float inv = 1.f / fmaxf(r, 1e-12f);
    float sh[16];
    sh_l3(v[0] * inv, v[1] * inv, v[2] * inv, sh);
    float dc;
    float cv = orb_cutoff(r, rmax, &dc);
    const float pre = sqrtf(2.f / rmax);
    const int W = nb * 16;
    for (int k = lane; k < W; k += 32) {
        int n = k >> 4, m = k & 15;
        float w = 3.14159265358979323846f / rmax * (float)(n + 1);
        feat[e * W + k] = cv * (pre * sinf(w * r) / r) * sh[m];
    }
    if (lane == 0) {
        cut[e] = cv;
        if (ev) {
            ev[e * 3 + 0] = v[0];
            ev[e * 3 + 1] = v[1];
            ev[e * 3 + 2] = v[2];
        }
    }
}

__global__ void orb_feat_bwd_kernel(const float* __restrict__ pos, const int* __restrict__ src,
                                    const int* __restrict__ tgt, const int* __restrict__ img,
                                    const float* __restrict__ shifts, long long E, float rmax,
                                    int nb, const float* __restrict__ g_feat,
                                    const float* __restrict__ g_cut, float* __restrict__ g_ev) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float v[3];
    edge_vector(pos, src[e], tgt[e], shifts, img, e, v);
    float r = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    float inv = 1.f / fmaxf(r, 1e-12f);
    float u[3] = {v[0] * inv, v[1] * inv, v[2] * inv};
    float sh[16];
    sh_l3(u[0], u[1], u[2], sh);
    float dc;
    float cv = orb_cutoff(r, rmax, &dc);
    const float pre = sqrtf(2.f / rmax);
    const int W = nb * 16;
    float grbf[16], gang[16], gcut = 0.f;     // nb <= 16
    for (int n = 0; n < 16; ++n) grbf[n] = 0.f;
    for (int m = 0; m < 16; ++m) gang[m] = 0.f;
    for (int k = lane; k < W; k += 32) {
        int n = k >> 4, m = k & 15;
        float w = 3.14159265358979323846f / rmax * (float)(n + 1);
        float rb = pre * sinf(w * r) / r;
        float g = g_feat[e * W + k];
        grbf[n] += g * sh[m];       // times cutoff below
        gang[m] += g * rb;
        gcut += g * rb * sh[m];
    }
    for (int n = 0; n < nb; ++n) grbf[n] = warp_sum(grbf[n]);
    for (int m = 0; m < 16; ++m) gang[m] = warp_sum(gang[m]);
    gcut = warp_sum(gcut);
    if (lane != 0) return;
    gcut += g_cut[e];
    float gr = gcut * dc;
    for (int n = 0; n < nb; ++n) {
        float w = 3.14159265358979323846f / rmax * (float)(n + 1);
        float drb = pre * (w * cosf(w * r) * r - sinf(w * r)) / (r * r);
        gr += cv * grbf[n] * drb;
    }
    for (int m = 0; m < 16; ++m) gang[m] *= cv;
    float gu[3];
    sh_l3_vjp(u[0], u[1], u[2], gang, gu);
    float ug = u[0] * gu[0] + u[1] * gu[1] + u[2] * gu[2];
#pragma unroll
    for (int k = 0; k < 3; ++k) g_ev[e * 3 + k] = u[k] * gr + (gu[k] - u[k] * ug) * inv;
}

// ------------------------------------------------------------------------- row RMSNorm
// Y = X rsqrt(mean(X^2) + eps) w; with R_in, R_out: R_out = R_in + Y. One warp per row.
__global__ void rmsnorm_rows_kernel(const float* __restrict__ X, long long ldx, long long rows,
                                    int W, const float* __restrict__ w, float eps, float* Y,
                                    long long ldy, const float* R_in, long long ldr_in,
                                    float* R_out, long long ldr_out) {
    long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = X + row * ldx;
    float s = 0.f;
    for (int c = lane; c < W; c += 32) s = fmaf(x[c], x[c], s);
    float inv = rsqrtf(warp_sum(s) / W + eps);
    for (int c = lane; c < W; c += 32) {
        float y = x[c] * inv * w[c];
        if (Y) Y[row * ldy + c] = y;
        if (R_out) R_out[row * ldr_out + c] = R_in[row * ldr_in + c] + y;
    }
}

// The same for W = 32 NW with the row held in registers: each lane's NW loads are all issued
// before the reduction (lane l owns columns l, l + 32, ..., as above, so the sums and results
// are bit-identical). Orb-v3 shape (W = 256): the whole step 6.66 -> 6.61 ms.
template <int NW>
__global__ void rmsnorm_rows_r_kernel(const float* __restrict__ X, long long ldx, long long rows,
                                      const float* __restrict__ w, float eps, float* Y,
                                      long long ldy, const float* R_in, long long ldr_in,
                                      float* R_out, long long ldr_out) {
    constexpr int W = 32 * NW;
    long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = X + row * ldx;
    float xv[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) xv[i] = x[lane + 32 * i];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) s = fmaf(xv[i], xv[i], s);
    float inv = rsqrtf(warp_sum(s) / W + eps);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        float y = xv[i] * inv * w[c];
        if (Y) Y[row * ldy + c] = y;
        if (R_out) R_out[row * ldr_out + c] = R_in[row * ldr_in + c] + y;
    }
}

template <int NW>
__global__ void rmsnorm_rows_bwd_r_kernel(const float* __restrict__ X, const float* gY,
                                          long long rows, const float* __restrict__ w, float eps,
                                          float* dX) {
    constexpr int W = 32 * NW;
    long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = X + row * (long long)W;
    const float* g = gY + row * (long long)W;
    float xv[NW], gv[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        xv[i] = x[lane + 32 * i];
        gv[i] = g[lane + 32 * i];
    }
    float s = 0.f, t = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        s = fmaf(xv[i], xv[i], s);
        t = fmaf(gv[i] * w[c], xv[i], t);
    }
    float inv = rsqrtf(warp_sum(s) / W + eps);
    float k = inv * inv * inv * warp_sum(t) / W;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        dX[row * (long long)W + c] = inv * gv[i] * w[c] - k * xv[i];
    }
}

// dX = inv (u - xhat mean(u xhat)), u = gY w, xhat = X inv. dX may alias gY.
__global__ void rmsnorm_rows_bwd_kernel(const float* __restrict__ X, const float* gY,
                                        long long rows, int W, const float* __restrict__ w,
                                        float eps, float* dX) {
    long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = X + row * (long long)W;
    const float* g = gY + row * (long long)W;
    float s = 0.f, t = 0.f;
    for (int c = lane; c < W; c += 32) {
        s = fmaf(x[c], x[c], s);
        t = fmaf(g[c] * w[c], x[c], t);
    }
    float inv = rsqrtf(warp_sum(s) / W + eps);
    float k = inv * inv * inv * warp_sum(t) / W;
    for (int c = lane; c < W; c += 32) dX[row * (long long)W + c] = inv * g[c] * w[c] - k * x[c];
}

// ---------------------------------------------------------------------- attention gates
// lin[e] = (edges[e] . wr + br, edges[e] . ws + bs); att = sigmoid(lin) * cut. One warp per edge.
__global__ void orb_attention_kernel(const float* __restrict__ edges, long long E, int C,
                                     const float* __restrict__ wr, float br,
                                     const float* __restrict__ ws, float bs,
                                     const float* __restrict__ cut, float* __restrict__ lin,
                                     float* __restrict__ att) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float a = 0.f, b = 0.f;
    for (int c = lane; c < C; c += 32) {
        float x = edges[e * C + c];
        a = fmaf(x, wr[c], a);
        b = fmaf(x, ws[c], b);
    }
    a = warp_sum(a) + br;
    b = warp_sum(b) + bs;
    if (lane == 0) {
        lin[e * 2] = a;
        lin[e * 2 + 1] = b;
        att[e * 2] = sigmoid_f(a) * cut[e];
        att[e * 2 + 1] = sigmoid_f(b) * cut[e];
    }
}

// ------------------------------------------------------------------------ CSR sums
// out[n, :W] (+)= sum_{k in [ptr[n], ptr[n+1])} scale[e] X[e, :W], e = eid ? eid[k] : k.
// One block per node, one float4 of channels per thread: the loads of four edges are issued
// before their multiply-adds, which still run in CSR order (the same sums as one edge at a
// time).
__global__ void csr_sum_kernel(const float* __restrict__ X, long long ldx,
                               const float* __restrict__ scale, int sstride,
                               const int* __restrict__ ptr, const int* __restrict__ eid,
                               long long N, int W, float* __restrict__ out, long long ldo,
                               int accumulate) {
    const long long n = blockIdx.x;
    const int k0 = ptr[n], k1 = ptr[n + 1];
    for (int c = threadIdx.x * 4; c < W; c += blockDim.x * 4) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int k = k0;
        for (; k + 3 < k1; k += 4) {
            int e[4];
            float s[4];
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) e[u] = eid ? eid[k + u] : k + u;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                s[u] = scale ? scale[(long long)e[u] * sstride] : 1.f;
                v[u] = *reinterpret_cast<const float4*>(X + (long long)e[u] * ldx + c);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc.x = fmaf(s[u], v[u].x, acc.x);
                acc.y = fmaf(s[u], v[u].y, acc.y);
                acc.z = fmaf(s[u], v[u].z, acc.z);
                acc.w = fmaf(s[u], v[u].w, acc.w);
            }
        }
        for (; k < k1; ++k) {
            const int e = eid ? eid[k] : k;
            const float s = scale ? scale[(long long)e * sstride] : 1.f;
            const float4 v = *reinterpret_cast<const float4*>(X + (long long)e * ldx + c);
            acc.x = fmaf(s, v.x, acc.x);
            acc.y = fmaf(s, v.y, acc.y);
            acc.z = fmaf(s, v.z, acc.z);
            acc.w = fmaf(s, v.w, acc.w);
        }
        float4* o = reinterpret_cast<float4*>(out + n * ldo + c);
        if (accumulate) {
            float4 p = *o;
            acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
        }
        *o = acc;
    }
}

// ------------------------------------------------------------------- message-passing VJP
// Per edge (warp): with g_recv = g_agg[src, 0:C] (receiver aggregate adjoint) and
// g_sent = g_agg[tgt, C:2C] (sender aggregate adjoint):
//   g_ue = gE + att_s g_sent + att_r g_recv
//   g_att_r = <g_recv, ue>, g_att_s = <g_sent, ue>
//   gE += (g_att_r cut s_r (1 - s_r)) wr + (g_att_s cut s_s (1 - s_s)) ws
//   g_cut += g_att_r s_r + g_att_s s_s
__global__ void orb_messages_bwd_kernel(const float* __restrict__ g_agg, const float* gE_in,
                                        const float* __restrict__ ue,
                                        const float* __restrict__ lin,
                                        const float* __restrict__ att,
                                        const float* __restrict__ cut,
                                        const int* __restrict__ src,
                                        const int* __restrict__ tgt, long long E, int C,
                                        const float* __restrict__ wr,
                                        const float* __restrict__ ws,
                                        float* __restrict__ g_ue, float* gE_out,
                                        float* __restrict__ g_cut) {
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    const float* gr = g_agg + (long long)src[e] * 2 * C;
    const float* gs = g_agg + (long long)tgt[e] * 2 * C + C;
    const float ar = att[e * 2], as = att[e * 2 + 1];
    float pr = 0.f, ps = 0.f;
    for (int c = lane; c < C; c += 32) {
        float u = ue[e * C + c];
        pr = fmaf(gr[c], u, pr);
        ps = fmaf(gs[c], u, ps);
        g_ue[e * C + c] = gE_in[e * C + c] + as * gs[c] + ar * gr[c];
    }
    pr = warp_sum(pr);
    ps = warp_sum(ps);
    const float sr = sigmoid_f(lin[e * 2]), ss = sigmoid_f(lin[e * 2 + 1]);
    const float cv = cut[e];
    const float glr = pr * cv * sr * (1.f - sr), gls = ps * cv * ss * (1.f - ss);
    for (int c = lane; c < C; c += 32)
        gE_out[e * C + c] = gE_in[e * C + c] + glr * wr[c] + gls * ws[c];
    if (lane == 0) g_cut[e] += pr * sr + ps * ss;
}

// The two kernels above for C = 32 NW with each lane's loads issued before its multiply-adds
// (lane l owns columns l, l + 32, ... as above: the same sums in the same order, bit-identical).
// Orb-v3 shape (C = 256): the whole step 6.65 -> 6.54 ms.
template <int NW>
__global__ void orb_attention_r_kernel(const float* __restrict__ edges, long long E,
                                       const float* __restrict__ wr, float br,
                                       const float* __restrict__ ws, float bs,
                                       const float* __restrict__ cut, float* __restrict__ lin,
                                       float* __restrict__ att) {
    constexpr int C = 32 * NW;
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    float xv[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) xv[i] = edges[e * C + lane + 32 * i];
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        a = fmaf(xv[i], wr[c], a);
        b = fmaf(xv[i], ws[c], b);
    }
    a = warp_sum(a) + br;
    b = warp_sum(b) + bs;
    if (lane == 0) {
        lin[e * 2] = a;
        lin[e * 2 + 1] = b;
        att[e * 2] = sigmoid_f(a) * cut[e];
        att[e * 2 + 1] = sigmoid_f(b) * cut[e];
    }
}

template <int NW>
__global__ void orb_messages_bwd_r_kernel(const float* __restrict__ g_agg, const float* gE_in,
                                          const float* __restrict__ ue,
                                          const float* __restrict__ lin,
                                          const float* __restrict__ att,
                                          const float* __restrict__ cut,
                                          const int* __restrict__ src,
                                          const int* __restrict__ tgt, long long E,
                                          const float* __restrict__ wr,
                                          const float* __restrict__ ws,
                                          float* __restrict__ g_ue, float* gE_out,
                                          float* __restrict__ g_cut) {
    constexpr int C = 32 * NW;
    long long e = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (e >= E) return;
    const float* gr = g_agg + (long long)src[e] * 2 * C;
    const float* gs = g_agg + (long long)tgt[e] * 2 * C + C;
    const float ar = att[e * 2], as = att[e * 2 + 1];
    float uv[NW], rv[NW], sv[NW], iv[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        uv[i] = ue[e * C + c];
        rv[i] = gr[c];
        sv[i] = gs[c];
        iv[i] = gE_in[e * C + c];
    }
    float pr = 0.f, ps = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        pr = fmaf(rv[i], uv[i], pr);
        ps = fmaf(sv[i], uv[i], ps);
        g_ue[e * C + lane + 32 * i] = iv[i] + as * sv[i] + ar * rv[i];
    }
    pr = warp_sum(pr);
    ps = warp_sum(ps);
    const float sr = sigmoid_f(lin[e * 2]), ss = sigmoid_f(lin[e * 2 + 1]);
    const float cv = cut[e];
    const float glr = pr * cv * sr * (1.f - sr), gls = ps * cv * ss * (1.f - ss);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        gE_out[e * C + c] = iv[i] + glr * wr[c] + gls * ws[c];
    }
    if (lane == 0) g_cut[e] += pr * sr + ps * ss;
}

// --------------------------------------------------------------- node mean / broadcast
// out[c] = scale * sum_n X[n, c] in a fixed order (one thread per column, rows in order).
// 32 columns per block, 32 row groups (rows r, r + 32, ...) per column, then a fixed-order tree
// over the groups: deterministic, and the rows are read by 1,024 threads instead of 32.
__global__ void __launch_bounds__(1024) col_mean_kernel(const float* __restrict__ X, long long ld,
                                                        long long N, int C, float scale,
                                                        float* __restrict__ out) {
    __shared__ float part[32][33];
    const int cx = threadIdx.x, ry = threadIdx.y;
    const int c = blockIdx.x * 32 + cx;
    float s = 0.f;
    if (c < C)
        for (long long n = ry; n < N; n += 32) s += X[n * ld + c];
    part[ry][cx] = s;
    __syncthreads();
    for (int w = 16; w > 0; w >>= 1) {
        if (ry < w) part[ry][cx] += part[ry + w][cx];
        __syncthreads();
    }
    if (ry == 0 && c < C) out[c] = part[0][cx] * scale;
}

__global__ void row_broadcast_kernel(const float* __restrict__ v, long long N, int C,
                                     float scale, float* __restrict__ out, long long ld,
                                     int accumulate) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N * C) return;
    long long n = t / C;
    int c = (int)(t - n * C);
    float x = v[c] * scale;
    out[n * ld + c] = accumulate ? out[n * ld + c] + x : x;
}

// ------------------------------------------------------------- ZBL pair repulsion (fp64)
// Ziegler-Biersack-Littmark screened Coulomb repulsion of Orb's pair_repulsion.ZBLBasis as
// the reference evaluates it on the host (tt_atom/orb_model.py:491-537): per edge, with
// Zu / Zv the sender / receiver atomic numbers plus one (the upstream indexing convention),
//   a   = 0.4543 * 0.529 / (Zu^0.3 + Zv^0.3)
//   phi = sum_k c_k exp(-d_k x / a)          (c, d: the 4-term universal screening function)
//   v   = 0.5 * 14.3996 Zu Zv / x * phi * env(x / (r_cov[Zu] + r_cov[Zv])),
//   env(t) = 1 - (p+1)(p+2)/2 t^p + p(p+2) t^(p+1) - p(p+1)/2 t^(p+2) for t < 1, else 0 (p = 6)
// and the total is scale * sum_e v_e (scale = 1 / N for the per-node mean). Each thread also
// writes dE/d(edge vector) = scale dv/dx vec / x, from which the force / virial reduction
// follows; per-block partial energies (fixed grid, fixed tree) make the sum deterministic.
constexpr int kZblBlocks = 1024;

__global__ void __launch_bounds__(256) zbl_kernel(
    const float* __restrict__ ev, const int* __restrict__ Z, const int* __restrict__ src,
    const int* __restrict__ tgt, long long E, const double* __restrict__ rcov, int nrad,
    double scale, float* __restrict__ g_ev, double* __restrict__ part) {
    __shared__ double red[256];
    const double c[4] = {0.1818, 0.5099, 0.2802, 0.02817};
    const double d[4] = {3.2, 0.9423, 0.4028, 0.2016};
    const double p = 6.0;
    double acc = 0.0;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < E;
         e += (long long)gridDim.x * blockDim.x) {
        const double vx = ev[3 * e], vy = ev[3 * e + 1], vz = ev[3 * e + 2];
        const double x = sqrt(vx * vx + vy * vy + vz * vz);
        const int iu = Z[tgt[e]] + 1, iv = Z[src[e]] + 1;     // Orb: senders = tgt
        const double Zu = iu, Zv = iv;
        const double a = 0.4543 * 0.529 / (pow(Zu, 0.3) + pow(Zv, 0.3));
        double phi = 0.0, dphi = 0.0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const double t = c[k] * exp(-d[k] * x / a);
            phi += t;
            dphi -= t * d[k] / a;
        }
        const double q = 0.5 * 14.3996 * Zu * Zv;
        const double rmax = (iu < nrad ? rcov[iu] : 0.0) + (iv < nrad ? rcov[iv] : 0.0);
        double env = 0.0, denv = 0.0;
        if (x < rmax) {
            const double t = x / rmax;
            const double tp = pow(t, p - 1.0);
            env = 1.0 - (p + 1.0) * (p + 2.0) / 2.0 * tp * t + p * (p + 2.0) * tp * t * t -
                  p * (p + 1.0) / 2.0 * tp * t * t * t;
            denv = (-(p + 1.0) * (p + 2.0) / 2.0 * p * tp + p * (p + 2.0) * (p + 1.0) * tp * t -
                    p * (p + 1.0) / 2.0 * (p + 2.0) * tp * t * t) / rmax;
        }
        const double v = q / x * phi * env;
        const double dvdx = q * ((dphi * x - phi) / (x * x) * env + phi / x * denv);
        acc += v;
        const double gs = scale * dvdx / x;
        g_ev[3 * e] = (float)(gs * vx);
        g_ev[3 * e + 1] = (float)(gs * vy);
        g_ev[3 * e + 2] = (float)(gs * vz);
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

__global__ void zbl_total_kernel(const double* __restrict__ part, double scale,
                                 double* __restrict__ energy) {
    __shared__ double red[kZblBlocks];
    for (int i = threadIdx.x; i < kZblBlocks; i += blockDim.x) red[i] = part[i];
    __syncthreads();
    for (int w = kZblBlocks / 2; w > 0; w >>= 1) {
        for (int i = threadIdx.x; i < w; i += blockDim.x) red[i] += red[i + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) energy[0] = scale * red[0];
}

}  // namespace atom

using namespace atom;

#define WARPS(n) ceil_div((long long)(n) * 32, 256), 256, 0, (cudaStream_t)stream

extern "C" int atom_orb_edge_features(const float* pos, const int* src, const int* tgt,
                                      const int* img, const float* shifts, int64_t E, float rmax,
                                      int nb, float* feat, float* cut, float* ev, void* stream) {
    ATOM_REQUIRE(nb >= 1 && nb <= 16, "orb_edge_features: 1 <= num_bases <= 16");
    if (E == 0) return ATOM_OK;
    orb_feat_kernel<<<WARPS(E)>>>(pos, src, tgt, img, shifts, E, rmax, nb, feat, cut, ev);
    ATOM_CHECK_LAUNCH("orb_edge_features");
    return ATOM_OK;
}

extern "C" int atom_orb_edge_features_bwd(const float* pos, const int* src, const int* tgt,
                                          const int* img, const float* shifts, int64_t E,
                                          float rmax, int nb, const float* g_feat,
                                          const float* g_cut, float* g_ev, void* stream) {
    ATOM_REQUIRE(nb >= 1 && nb <= 16, "orb_edge_features_bwd: 1 <= num_bases <= 16");
    if (E == 0) return ATOM_OK;
    orb_feat_bwd_kernel<<<WARPS(E)>>>(pos, src, tgt, img, shifts, E, rmax, nb, g_feat, g_cut,
                                      g_ev);
    ATOM_CHECK_LAUNCH("orb_edge_features_bwd");
    return ATOM_OK;
}

extern "C" int atom_rmsnorm_rows(const float* X, int64_t ldx, int64_t rows, int W,
                                 const float* w, float eps, float* Y, int64_t ldy,
                                 const float* R_in, int64_t ldr_in, float* R_out,
                                 int64_t ldr_out, void* stream) {
    ATOM_REQUIRE(W > 0, "rmsnorm_rows: W must be positive");
    ATOM_REQUIRE(!R_out || R_in, "rmsnorm_rows: R_out needs R_in");
    if (rows == 0) return ATOM_OK;
    if (W == 256)
        rmsnorm_rows_r_kernel<8><<<WARPS(rows)>>>(X, ldx, rows, w, eps, Y, ldy, R_in, ldr_in,
                                                  R_out, ldr_out);
    else if (W == 128)
        rmsnorm_rows_r_kernel<4><<<WARPS(rows)>>>(X, ldx, rows, w, eps, Y, ldy, R_in, ldr_in,
                                                  R_out, ldr_out);
    else
        rmsnorm_rows_kernel<<<WARPS(rows)>>>(X, ldx, rows, W, w, eps, Y, ldy, R_in, ldr_in, R_out,
                                             ldr_out);
    ATOM_CHECK_LAUNCH("rmsnorm_rows");
    return ATOM_OK;
}

extern "C" int atom_rmsnorm_rows_bwd(const float* X, const float* gY, int64_t rows, int W,
                                     const float* w, float eps, float* dX, void* stream) {
    ATOM_REQUIRE(W > 0, "rmsnorm_rows_bwd: W must be positive");
    if (rows == 0) return ATOM_OK;
    if (W == 256)
        rmsnorm_rows_bwd_r_kernel<8><<<WARPS(rows)>>>(X, gY, rows, w, eps, dX);
    else if (W == 128)
        rmsnorm_rows_bwd_r_kernel<4><<<WARPS(rows)>>>(X, gY, rows, w, eps, dX);
    else
        rmsnorm_rows_bwd_kernel<<<WARPS(rows)>>>(X, gY, rows, W, w, eps, dX);
    ATOM_CHECK_LAUNCH("rmsnorm_rows_bwd");
    return ATOM_OK;
}

extern "C" int atom_orb_attention(const float* edges, int64_t E, int C, const float* wr,
                                  float br, const float* ws, float bs, const float* cut,
                                  float* lin, float* att, void* stream) {
    if (E == 0) return ATOM_OK;
    if (C == 256)
        orb_attention_r_kernel<8><<<WARPS(E)>>>(edges, E, wr, br, ws, bs, cut, lin, att);
    else
        orb_attention_kernel<<<WARPS(E)>>>(edges, E, C, wr, br, ws, bs, cut, lin, att);
    ATOM_CHECK_LAUNCH("orb_attention");
    return ATOM_OK;
}

extern "C" int atom_csr_sum(const float* X, int64_t ldx, const float* scale, int sstride,
                            const int* ptr, const int* eid, int64_t N, int W, float* out,
                            int64_t ldo, int accumulate, void* stream) {
    ATOM_REQUIRE(W % 4 == 0 && ldx % 4 == 0 && ldo % 4 == 0 && aligned16(X) && aligned16(out),
                 "csr_sum: W, ldx, ldo must be multiples of 4 and X, out 16-byte aligned");
    if (N == 0) return ATOM_OK;
    const int threads = W / 4 < 32 ? 32 : (W / 4 > 256 ? 256 : (W / 4 + 31) / 32 * 32);
    csr_sum_kernel<<<(unsigned)N, threads, 0, (cudaStream_t)stream>>>(X, ldx, scale, sstride,
                                                                      ptr, eid, N, W, out, ldo,
                                                                      accumulate);
    ATOM_CHECK_LAUNCH("csr_sum");
    return ATOM_OK;
}

extern "C" int atom_orb_messages_bwd(const float* g_agg, const float* gE_in, const float* ue,
                                     const float* lin, const float* att, const float* cut,
                                     const int* src, const int* tgt, int64_t E, int C,
                                     const float* wr, const float* ws, float* g_ue,
                                     float* gE_out, float* g_cut, void* stream) {
    if (E == 0) return ATOM_OK;
    if (C == 256)
        orb_messages_bwd_r_kernel<8><<<WARPS(E)>>>(g_agg, gE_in, ue, lin, att, cut, src, tgt, E,
                                                   wr, ws, g_ue, gE_out, g_cut);
    else
        orb_messages_bwd_kernel<<<WARPS(E)>>>(g_agg, gE_in, ue, lin, att, cut, src, tgt, E, C,
                                              wr, ws, g_ue, gE_out, g_cut);
    ATOM_CHECK_LAUNCH("orb_messages_bwd");
    return ATOM_OK;
}

extern "C" int atom_col_mean(const float* X, int64_t ld, int64_t N, int C, float scale,
                             float* out, void* stream) {
    col_mean_kernel<<<ceil_div(C, 32), dim3(32, 32), 0, (cudaStream_t)stream>>>(X, ld, N, C,
                                                                              scale, out);
    ATOM_CHECK_LAUNCH("col_mean");
    return ATOM_OK;
}

extern "C" int atom_row_broadcast(const float* v, int64_t N, int C, float scale, float* out,
                                  int64_t ld, int accumulate, void* stream) {
    if (N == 0) return ATOM_OK;
    row_broadcast_kernel<<<ceil_div(N * C, 256), 256, 0, (cudaStream_t)stream>>>(
        v, N, C, scale, out, ld, accumulate);
    ATOM_CHECK_LAUNCH("row_broadcast");
    return ATOM_OK;
}

extern "C" int atom_orb_zbl(const float* ev, const int* Z, const int* src, const int* tgt,
                            int64_t E, const double* rcov, int nrad, double scale, float* g_ev,
                            double* partials, double* energy, void* stream) {
    ATOM_REQUIRE(E >= 0 && nrad > 0, "orb_zbl: bad sizes");
    cudaStream_t st = (cudaStream_t)stream;
    zbl_kernel<<<kZblBlocks, 256, 0, st>>>(ev, Z, src, tgt, E, rcov, nrad, scale, g_ev,
                                          partials);
    ATOM_CHECK_LAUNCH("orb_zbl");
    zbl_total_kernel<<<1, 256, 0, st>>>(partials, scale, energy);
    ATOM_CHECK_LAUNCH("orb_zbl_total");
    return ATOM_OK;
}
