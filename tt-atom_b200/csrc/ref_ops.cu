// The four reference-op equivalents (fused_rotate, fused_rotate_gc, fused_gate, fused_ln_bw)
// plus the library's error plumbing.
//
// These keep the argument meaning of the reference's nanobind ops
// (custom_kernels/fused_rotate/fused_rotate_nanobind.cpp:17-96) so a caller of those ops can
// switch over; the model path uses the fused kernels of edge_ops.cu instead.
#include <stdarg.h>

#include "common.cuh"

namespace atom {

static thread_local char g_err[1024];

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

// ---------------------------------------------------------------------------- fused_rotate
// One thread per (edge, 4-column group); the nonzero pattern travels as a kernel parameter.
struct RotPattern {
    int n_out, nnz;
    unsigned char deg[32];
    unsigned char ks[128];
    unsigned char js[128];
};

__global__ void fused_rotate_kernel(const float* __restrict__ x, const float* __restrict__ coef,
                                    long long E, int n_in, int W, RotPattern p,
                                    float* __restrict__ out) {
    const int W4 = W >> 2;
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * W4) return;
    long long e = t / W4;
    int w4 = (int)(t - e * W4);
    const float4* xe = reinterpret_cast<const float4*>(x + e * (long long)n_in * W) + w4;
    const float* ce = coef + e * p.nnz;
    float4* oe = reinterpret_cast<float4*>(out + e * (long long)p.n_out * W) + w4;
    int k = 0;
    for (int i = 0; i < p.n_out; ++i) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int d = 0; d < p.deg[i]; ++d, ++k) {
            float c = __ldg(ce + p.ks[k]);
            float4 v = __ldg(xe + (long long)p.js[k] * W4);
            acc.x = fmaf(c, v.x, acc.x);
            acc.y = fmaf(c, v.y, acc.y);
            acc.z = fmaf(c, v.z, acc.z);
            acc.w = fmaf(c, v.w, acc.w);
        }
        oe[(long long)i * W4] = acc;
    }
}

// ------------------------------------------------------------------------- fused_rotate_gc
// One warp per (edge, nonzero): a W-long dot product reduced with shuffles.
__global__ void fused_rotate_gc_kernel(const float* __restrict__ gout,
                                       const float* __restrict__ xin, long long E, int n_out,
                                       int n_in, int W, RotPattern p, float* __restrict__ gc) {
    long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= E * p.nnz) return;
    long long e = wid / p.nnz;
    int k = (int)(wid - e * p.nnz);
    const float* g = gout + e * (long long)n_out * W + (long long)p.ks[k] * W;  // ks = is_
    const float* xv = xin + e * (long long)n_in * W + (long long)p.js[k] * W;
    float s = 0.f;
    for (int w = lane; w < W; w += 32) s = fmaf(__ldg(g + w), __ldg(xv + w), s);
    s = warp_sum(s);
    if (lane == 0) gc[e * p.nnz + k] = s;
}

// ------------------------------------------------------------------------------ fused_gate
__global__ void fused_gate_kernel(const float* __restrict__ a, const float* __restrict__ gate,
                                  const float* __restrict__ b, long long E, int H, int G,
                                  int mode, float* __restrict__ out) {
    const int Wc = H + G;
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * Wc) return;
    long long e = t / Wc;
    int c = (int)(t - e * Wc);
    float av = a[t];
    float r;
    if (c < H) {
        r = mode == 0 ? silu_f(av) : av * dsilu_f(b[t]);
    } else {
        r = av * gate[e * G + (c - H)];
    }
    out[t] = r;
}

// ------------------------------------------------------------------------------ fused_ln_bw
// One warp per row.
__global__ void fused_ln_bw_kernel(const float* __restrict__ g, const float* __restrict__ x,
                                   const float* __restrict__ n, const float* __restrict__ gamma,
                                   long long rows, int W, float eps, float* __restrict__ dx) {
    long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * W;
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
        float gy = g[row * W + c] * dsilu_f(n[row * W + c]) * gamma[c];
        float xh = (xr[c] - mean) * rstd;
        s1 += gy;
        s2 = fmaf(gy, xh, s2);
    }
    s1 = warp_sum(s1) / W;
    s2 = warp_sum(s2) / W;
    for (int c = lane; c < W; c += 32) {
        float gy = g[row * W + c] * dsilu_f(n[row * W + c]) * gamma[c];
        float xh = (xr[c] - mean) * rstd;
        dx[row * W + c] = rstd * (gy - s1 - xh * s2);
    }
}

static int make_pattern(RotPattern& p, int n_out, int nnz, const int* deg, const int* ks,
                        const int* js, int n_in, int ks_lim) {
    ATOM_REQUIRE(n_out > 0 && n_out <= 32 && n_in > 0 && n_in <= 32,
                 "n_in/n_out must be in [1, 32] (got %d, %d)", n_in, n_out);
    ATOM_REQUIRE(nnz > 0 && nnz <= 128, "nnz must be in [1, 128] (got %d)", nnz);
    p.n_out = n_out;
    p.nnz = nnz;
    int tot = 0;
    if (deg) {
        for (int i = 0; i < n_out; ++i) {
            ATOM_REQUIRE(deg[i] >= 0, "negative degree");
            p.deg[i] = (unsigned char)deg[i];
            tot += deg[i];
        }
        ATOM_REQUIRE(tot == nnz, "sum(deg) = %d != nnz = %d", tot, nnz);
    }
    for (int k = 0; k < nnz; ++k) {
        ATOM_REQUIRE(ks[k] >= 0 && ks[k] < ks_lim, "index %d out of range", ks[k]);
        ATOM_REQUIRE(js[k] >= 0 && js[k] < n_in, "input block %d out of range", js[k]);
        p.ks[k] = (unsigned char)ks[k];
        p.js[k] = (unsigned char)js[k];
    }
    return ATOM_OK;
}

}  // namespace atom

using namespace atom;

extern "C" int atom_last_error(char* buf, size_t n) {
    size_t len = strlen(g_err);
    if (buf && n) {
        size_t c = len < n - 1 ? len : n - 1;
        memcpy(buf, g_err, c);
        buf[c] = 0;
    }
    return (int)len;
}

extern "C" int atom_abi_version(void) { return 2; }

extern "C" int atom_launch_count(int64_t* n) {
    if (n) *n = atom::g_launches.load(std::memory_order_relaxed);
    return ATOM_OK;
}

extern "C" int atom_fused_rotate(const float* x, const float* coef, int64_t E, int n_in,
                                 int n_out, int W, int nnz, const int* deg, const int* ks,
                                 const int* js, float* out, void* stream) {
    ATOM_REQUIRE(E >= 0, "E < 0");
    ATOM_REQUIRE(W > 0 && W % 4 == 0, "W must be a positive multiple of 4 (got %d)", W);
    ATOM_REQUIRE(aligned16(x) && aligned16(out), "x/out must be 16-byte aligned");
    RotPattern p;
    int s = make_pattern(p, n_out, nnz, deg, ks, js, n_in, nnz);
    if (s) return s;
    if (E == 0) return ATOM_OK;
    long long T = E * (W / 4);
    fused_rotate_kernel<<<ceil_div(T, 256), 256, 0, (cudaStream_t)stream>>>(x, coef, E, n_in, W,
                                                                              p, out);
    ATOM_CHECK_LAUNCH("fused_rotate");
    return ATOM_OK;
}

extern "C" int atom_fused_rotate_gc(const float* gout, const float* xin, int64_t E, int n_out,
                                    int n_in, int W, int nnz, const int* is_, const int* js,
                                    float* gc, void* stream) {
    ATOM_REQUIRE(E >= 0 && W > 0, "bad shape");
    RotPattern p;
    // ks carries is_ (output-block index, < n_out)
    int s = make_pattern(p, n_out, nnz, nullptr, is_, js, n_in, n_out);
    if (s) return s;
    if (E == 0) return ATOM_OK;
    long long warps = E * nnz;
    fused_rotate_gc_kernel<<<ceil_div(warps * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        gout, xin, E, n_out, n_in, W, p, gc);
    ATOM_CHECK_LAUNCH("fused_rotate_gc");
    return ATOM_OK;
}

extern "C" int atom_fused_gate(const float* a, const float* gate, const float* b, int64_t E,
                               int H, int G, int mode, float* out, void* stream) {
    ATOM_REQUIRE(E >= 0 && H >= 0 && G >= 0, "bad shape");
    ATOM_REQUIRE(mode == 0 || mode == 1, "mode must be 0 or 1");
    ATOM_REQUIRE(mode == 0 || b != nullptr, "mode 1 needs b");
    long long T = E * (long long)(H + G);
    if (T == 0) return ATOM_OK;
    fused_gate_kernel<<<ceil_div(T, 256), 256, 0, (cudaStream_t)stream>>>(a, gate, b, E, H, G,
                                                                           mode, out);
    ATOM_CHECK_LAUNCH("fused_gate");
    return ATOM_OK;
}

extern "C" int atom_fused_ln_bw(const float* g, const float* x, const float* n,
                                const float* gamma, int64_t rows, int W, float eps, float* dx,
                                void* stream) {
    ATOM_REQUIRE(rows >= 0 && W > 0, "bad shape");
    if (rows == 0) return ATOM_OK;
    fused_ln_bw_kernel<<<ceil_div(rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        g, x, n, gamma, rows, W, eps, dx);
    ATOM_CHECK_LAUNCH("fused_ln_bw");
    return ATOM_OK;
}
