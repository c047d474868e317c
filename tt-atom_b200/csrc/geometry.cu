// Per-edge geometry (edge vector, distance, packed Wigner-D, Gaussian basis, envelope) and its
// VJP, plus the force / virial reduction.
//
// Reference: tt_atom/geometry.py:87-155 (safe acos/atan2, Euler angles with roll 0, e3nn
// Wigner-D D_l = Z(0) J Z(-beta) J Z(-alpha)), :209-224 (m-primed row permutation), :226-261
// (distance, Gaussian basis, polynomial envelope p = 5); tt_atom/forces.py:515-524,580-589 (the
// strain-leaf virial and the host autograd finish that these kernels replace).
#include "common.cuh"

namespace atom {

struct GeoConst {
    float jd1[9];
    float jd2[25];
    int perm[9];        // m-primed row -> standard coefficient index
    float cutoff, coeff;
};

// Z(theta) for degree L (dimension D = 2L + 1): cos(f theta) on the diagonal, sin(f theta) on
// the anti-diagonal, f = L - i; the centre element is cos(0) + sin(0) = 1.
template <int D>
__device__ __forceinline__ void zrot(float theta, float* Z) {
    constexpr int L = (D - 1) / 2;
#pragma unroll
    for (int i = 0; i < D * D; ++i) Z[i] = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float f = (float)(L - i);
        float s, c;
        sincosf(f * theta, &s, &c);
        Z[i * D + i] += c;
        Z[i * D + (D - 1 - i)] += s;
    }
}

// dZ/dtheta
template <int D>
__device__ __forceinline__ void dzrot(float theta, float* Z) {
    constexpr int L = (D - 1) / 2;
#pragma unroll
    for (int i = 0; i < D * D; ++i) Z[i] = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float f = (float)(L - i);
        float s, c;
        sincosf(f * theta, &s, &c);
        Z[i * D + i] += -f * s;
        Z[i * D + (D - 1 - i)] += f * c;
    }
}

template <int D>
__device__ __forceinline__ void mm(const float* A, const float* B, float* C) {
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int k = 0; k < D; ++k) {
            float s = 0.f;
#pragma unroll
            for (int m = 0; m < D; ++m) s = fmaf(A[i * D + m], B[m * D + k], s);
            C[i * D + k] = s;
        }
}

// D = J Zb J Za
template <int D>
__device__ __forceinline__ void wig_chain(const float* J, const float* Zb, const float* Za,
                                          float* out) {
    float t1[D * D], t2[D * D];
    mm<D>(J, Za, t1);
    mm<D>(Zb, t1, t2);
    mm<D>(J, t2, out);
}

// Euclidean norm as torch.linalg.norm evaluates it for 3-vectors on the CPU:
// sqrt(fma(z, z, fma(y, y, x * x))), correctly rounded.
__device__ __forceinline__ float norm3(float x, float y, float z) {
    return __fsqrt_rn(__fmaf_rn(z, z, __fmaf_rn(y, y, __fmul_rn(x, x))));
}

__device__ __forceinline__ void edge_vec(const float* __restrict__ pos, int s, int t,
                                         const float* __restrict__ shifts, int img, float* v) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        float d = __fsub_rn(pos[s * 3 + k], pos[t * 3 + k]);
        v[k] = shifts ? __fadd_rn(d, shifts[img * 3 + k]) : d;
    }
}

struct Angles {
    float x, y, z, nrm, alpha, beta;
};

__device__ __forceinline__ Angles angles(const float* v) {
    Angles a;
    a.nrm = norm3(v[0], v[1], v[2]);
    float d = fmaxf(a.nrm, 1e-12f);
    a.x = fminf(fmaxf(v[0] / d, -1.f), 1.f);
    a.y = fminf(fmaxf(v[1] / d, -1.f), 1.f);
    a.z = fminf(fmaxf(v[2] / d, -1.f), 1.f);
    a.beta = acosf(a.y);
    a.alpha = atan2f(a.x, a.z);
    return a;
}

__device__ __forceinline__ float envelope_val(float ds, float* dval) {
    const float p = 5.f, A = -(p + 1.f) * (p + 2.f) / 2.f, B = p * (p + 2.f),
                Cc = -p * (p + 1.f) / 2.f;
    if (!(ds < 1.f)) {
        *dval = 0.f;
        return 0.f;
    }
    float ds2 = ds * ds, ds4 = ds2 * ds2, ds5 = ds4 * ds;
    float poly = A + ds * (B + Cc * ds);
    *dval = 5.f * ds4 * poly + ds5 * (B + 2.f * Cc * ds);
    return 1.f + ds5 * poly;
}

__global__ void __launch_bounds__(128) geometry_fwd_kernel(
    const float* __restrict__ pos, const int* __restrict__ src, const int* __restrict__ tgt,
    const int* __restrict__ img, const float* __restrict__ shifts, long long E, GeoConst g,
    float* __restrict__ coef, float* __restrict__ env, float* __restrict__ ev_out,
    float* __restrict__ dist_out) {
    long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    float v[3];
    edge_vec(pos, src[e], tgt[e], shifts, img ? img[e] : 0, v);
    Angles a = angles(v);
    float D1[9], D2[25];
    {
        float Za[9], Zb[9];
        zrot<3>(-a.alpha, Za);
        zrot<3>(-a.beta, Zb);
        wig_chain<3>(g.jd1, Zb, Za, D1);
    }
    {
        float Za[25], Zb[25];
        zrot<5>(-a.alpha, Za);
        zrot<5>(-a.beta, Zb);
        wig_chain<5>(g.jd2, Zb, Za, D2);
    }
    float* ce = coef + e * kNnz;
#pragma unroll
    for (int r = 0; r < kNsph; ++r) {
        const int l = row_deg(r), o = row_off(r);
        int i = g.perm[r] - deg_col0(l);
        if (l == 0) ce[o] = 1.f;
        else if (l == 1) {
#pragma unroll
            for (int jj = 0; jj < 3; ++jj) ce[o + jj] = D1[i * 3 + jj];
        } else {
#pragma unroll
            for (int jj = 0; jj < 5; ++jj) ce[o + jj] = D2[i * 5 + jj];
        }
    }
    float dv;
    env[e] = envelope_val(a.nrm / g.cutoff, &dv);
    if (ev_out) {
        ev_out[e * 3 + 0] = v[0];
        ev_out[e * 3 + 1] = v[1];
        ev_out[e * 3 + 2] = v[2];
    }
    if (dist_out) dist_out[e] = a.nrm;
}

// gauss[e, k] = exp(coeff (dist_e - offset_k)^2), one thread per element.
__global__ void gauss_kernel(const float* __restrict__ pos, const int* __restrict__ src,
                             const int* __restrict__ tgt, const int* __restrict__ img,
                             const float* __restrict__ shifts, long long E,
                             const float* __restrict__ offset, int NB, float coeff,
                             float* __restrict__ gauss) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= E * NB) return;
    long long e = t / NB;
    int k = (int)(t - e * NB);
    float v[3];
    edge_vec(pos, src[e], tgt[e], shifts, img ? img[e] : 0, v);
    float d = norm3(v[0], v[1], v[2]) - offset[k];
    gauss[t] = expf(coeff * (d * d));
}

// The same, one block per edge (the edge vector computed once per block, not per element) and
// four Gaussians per thread with a 16-byte store (NB a multiple of 4, gauss 16-byte aligned).
__global__ void __launch_bounds__(128) gauss4_kernel(
    const float* __restrict__ pos, const int* __restrict__ src, const int* __restrict__ tgt,
    const int* __restrict__ img, const float* __restrict__ shifts, long long E,
    const float* __restrict__ offset, int NB, float coeff, float* __restrict__ gauss) {
    const long long e = blockIdx.x;
    float v[3];
    edge_vec(pos, src[e], tgt[e], shifts, img ? img[e] : 0, v);
    const float nrm = norm3(v[0], v[1], v[2]);
    for (int q = threadIdx.x; q < NB / 4; q += blockDim.x) {
        const float4 o = *reinterpret_cast<const float4*>(offset + 4 * q);
        const float d0 = nrm - o.x, d1 = nrm - o.y, d2 = nrm - o.z, d3 = nrm - o.w;
        *reinterpret_cast<float4*>(gauss + e * NB + 4 * q) =
            make_float4(expf(coeff * (d0 * d0)), expf(coeff * (d1 * d1)),
                        expf(coeff * (d2 * d2)), expf(coeff * (d3 * d3)));
    }
}

// <G, J Zb J Za> for given factor matrices
template <int D>
__device__ __forceinline__ float frob_chain(const float* G, const float* J, const float* Zb,
                                            const float* Za) {
    float M[D * D];
    wig_chain<D>(J, Zb, Za, M);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < D * D; ++i) s = fmaf(G[i], M[i], s);
    return s;
}

// One warp per edge: lanes reduce the Gaussian-basis adjoint, lane 0 runs the geometric chain.
__global__ void __launch_bounds__(128) geometry_bwd_kernel(
    const float* __restrict__ pos, const int* __restrict__ src, const int* __restrict__ tgt,
    const int* __restrict__ img, const float* __restrict__ shifts, long long E, GeoConst g,
    const float* __restrict__ offset, int NB, const float* __restrict__ g_coef,
    const float* __restrict__ gauss, const float* __restrict__ g_gauss,
    const float* __restrict__ g_env, float* __restrict__ g_ev) {
    // a warp owns 32 edges: the Gaussian-basis adjoint of each is a warp reduction over the NB
    // columns (one edge at a time, lane j keeps edge j's), then every lane runs the Wigner /
    // angle chain of its own edge
    const long long e0 = (((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32;
    const int lane = threadIdx.x & 31;
    if (e0 >= E) return;
    float gd = 0.f;   // dE/d dist of this lane's edge
    if (g_gauss) {
        const int nj = E - e0 < 32 ? (int)(E - e0) : 32;
        for (int j = 0; j < nj; ++j) {
            const long long ej = e0 + j;
            float vj[3];
            edge_vec(pos, src[ej], tgt[ej], shifts, img ? img[ej] : 0, vj);
            const float nrm = angles(vj).nrm;
            float t = 0.f;
            for (int k = lane; k < NB; k += 32) {
                float gk = gauss[ej * NB + k];
                t = fmaf(g_gauss[ej * NB + k] * gk, 2.f * g.coeff * (nrm - offset[k]), t);
            }
            t = warp_sum(t);
            if (lane == j) gd = t;
        }
    }
    const long long e = e0 + lane;
    if (e >= E) return;
    float v[3];
    edge_vec(pos, src[e], tgt[e], shifts, img ? img[e] : 0, v);
    Angles a = angles(v);
    float dv;
    envelope_val(a.nrm / g.cutoff, &dv);
    gd = fmaf(g_env[e], dv / g.cutoff, gd);

    // adjoint of the dense Wigner blocks from the packed coefficient adjoint
    const float* gc = g_coef + e * kNnz;
    float G1[9], G2[25];
#pragma unroll
    for (int i = 0; i < 9; ++i) G1[i] = 0.f;
#pragma unroll
    for (int i = 0; i < 25; ++i) G2[i] = 0.f;
#pragma unroll
    for (int r = 0; r < kNsph; ++r) {
        const int l = row_deg(r), o = row_off(r);
        int i = g.perm[r] - deg_col0(l);
        if (l == 1) {
#pragma unroll
            for (int jj = 0; jj < 3; ++jj) G1[i * 3 + jj] = gc[o + jj];
        } else if (l == 2) {
#pragma unroll
            for (int jj = 0; jj < 5; ++jj) G2[i * 5 + jj] = gc[o + jj];
        }
    }
    // dD/dbeta = -J Z'(-beta) J Z(-alpha);  dD/dalpha = -J Z(-beta) J Z'(-alpha)
    float g_beta = 0.f, g_alpha = 0.f;
    {
        float Za[9], Zb[9], dZa[9], dZb[9];
        zrot<3>(-a.alpha, Za);
        zrot<3>(-a.beta, Zb);
        dzrot<3>(-a.alpha, dZa);
        dzrot<3>(-a.beta, dZb);
        g_beta -= frob_chain<3>(G1, g.jd1, dZb, Za);
        g_alpha -= frob_chain<3>(G1, g.jd1, Zb, dZa);
    }
    {
        float Za[25], Zb[25], dZa[25], dZb[25];
        zrot<5>(-a.alpha, Za);
        zrot<5>(-a.beta, Zb);
        dzrot<5>(-a.alpha, dZa);
        dzrot<5>(-a.beta, dZb);
        g_beta -= frob_chain<5>(G2, g.jd2, dZb, Za);
        g_alpha -= frob_chain<5>(G2, g.jd2, Zb, dZa);
    }
    // beta = acos(y) with the guarded derivative; alpha = atan2(x, z) with a clamped denominator
    const float lo = (float)(-1.0 + 1e-7), hi = (float)(1.0 - 1e-7);
    float yc = fminf(fmaxf(a.y, lo), hi);
    float gy = -g_beta / fmaxf(sqrtf(1.f - yc * yc), 1e-7f);
    float den = fmaxf(a.z * a.z + a.x * a.x, 1e-7f);
    float gx = g_alpha * a.z / den;
    float gz = -g_alpha * a.x / den;
    // clamp(-1, 1) passes the gradient inside the interval
    float n = fmaxf(a.nrm, 1e-12f);
    float u[3] = {v[0] / n, v[1] / n, v[2] / n};
    float gu[3] = {(u[0] >= -1.f && u[0] <= 1.f) ? gx : 0.f,
                   (u[1] >= -1.f && u[1] <= 1.f) ? gy : 0.f,
                   (u[2] >= -1.f && u[2] <= 1.f) ? gz : 0.f};
    // normalize: g_v = (g_u - u (u . g_u)) / |v| (for |v| > 1e-12)
    float ug = u[0] * gu[0] + u[1] * gu[1] + u[2] * gu[2];
    float gv[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        gv[k] = a.nrm > 1e-12f ? (gu[k] - u[k] * ug) / a.nrm : gu[k] / 1e-12f;
        // distance: d |v| / dv = v / |v|
        if (a.nrm > 0.f) gv[k] = fmaf(gd, v[k] / a.nrm, gv[k]);
    }
    g_ev[e * 3 + 0] = gv[0];
    g_ev[e * 3 + 1] = gv[1];
    g_ev[e * 3 + 2] = gv[2];
}

// Forces, one thread per node, fixed CSR order.
__global__ void forces_kernel(const float* __restrict__ g_ev, long long N,
                              const int* __restrict__ recv_ptr, const int* __restrict__ send_ptr,
                              const int* __restrict__ send_eid, float* __restrict__ F) {
    long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float f0 = 0.f, f1 = 0.f, f2 = 0.f;
    for (int e = recv_ptr[n]; e < recv_ptr[n + 1]; ++e) {
        f0 += g_ev[e * 3 + 0];
        f1 += g_ev[e * 3 + 1];
        f2 += g_ev[e * 3 + 2];
    }
    for (int k = send_ptr[n]; k < send_ptr[n + 1]; ++k) {
        int e = send_eid[k];
        f0 -= g_ev[e * 3 + 0];
        f1 -= g_ev[e * 3 + 1];
        f2 -= g_ev[e * 3 + 2];
    }
    F[n * 3 + 0] = f0;
    F[n * 3 + 1] = f1;
    F[n * 3 + 2] = f2;
}

// Virial partials: a fixed 1024-block grid; block b sums edges b, b + 1024*256, ... per thread
// and reduces with a fixed tree.
constexpr int kVirBlocks = 1024;

__global__ void virial_partial_kernel(const float* __restrict__ g_ev,
                                      const float* __restrict__ ev, long long E,
                                      float* __restrict__ part) {
    __shared__ float sh[9][256];
    float acc[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) acc[k] = 0.f;
    for (long long e = (long long)blockIdx.x * 256 + threadIdx.x; e < E;
         e += (long long)kVirBlocks * 256) {
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int b = 0; b < 3; ++b) acc[a * 3 + b] = fmaf(ev[e * 3 + a], g_ev[e * 3 + b], acc[a * 3 + b]);
    }
#pragma unroll
    for (int k = 0; k < 9; ++k) sh[k][threadIdx.x] = acc[k];
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o)
#pragma unroll
            for (int k = 0; k < 9; ++k) sh[k][threadIdx.x] += sh[k][threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x < 9) part[blockIdx.x * 9 + threadIdx.x] = sh[threadIdx.x][0];
}

__global__ void virial_final_kernel(const float* __restrict__ part, float* __restrict__ vir) {
    __shared__ float sh[9][256];
    float acc[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) acc[k] = 0.f;
    for (int b = threadIdx.x; b < kVirBlocks; b += 256)
#pragma unroll
        for (int k = 0; k < 9; ++k) acc[k] += part[b * 9 + k];
#pragma unroll
    for (int k = 0; k < 9; ++k) sh[k][threadIdx.x] = acc[k];
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o)
#pragma unroll
            for (int k = 0; k < 9; ++k) sh[k][threadIdx.x] += sh[k][threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x < 9) {
        int a = threadIdx.x / 3, b = threadIdx.x % 3;
        vir[threadIdx.x] = 0.5f * (sh[a * 3 + b][0] + sh[b * 3 + a][0]);
    }
}

static int make_geo(GeoConst& g, const float* jd1, const float* jd2, const int* perm,
                    float cutoff, float coeff) {
    ATOM_REQUIRE(jd1 && jd2 && perm, "geometry: Jd tables and the permutation are required");
    for (int i = 0; i < 9; ++i) g.jd1[i] = jd1[i];
    for (int i = 0; i < 25; ++i) g.jd2[i] = jd2[i];
    for (int r = 0; r < 9; ++r) {
        int p = perm[r];
        ATOM_REQUIRE(p >= 0 && p < 9, "perm out of range");
        int l = p == 0 ? 0 : (p < 4 ? 1 : 2);
        if (l != row_deg(r)) {
            set_error("m-primed row %d maps to degree %d, expected %d (only the lmax = mmax = 2 "
                      "m-primed layout is implemented)", r, l, row_deg(r));
            return ATOM_ERR_UNSUPPORTED;
        }
        g.perm[r] = p;
    }
    g.cutoff = cutoff;
    g.coeff = coeff;
    return ATOM_OK;
}

}  // namespace atom

using namespace atom;

extern "C" int atom_edge_geometry(const float* pos, const int* src, const int* tgt,
                                  const int* img, const float* shifts, int64_t E,
                                  const float* jd1, const float* jd2, const int* perm9,
                                  const float* offset, int NB, float coeff, float cutoff,
                                  float* coef, float* gauss, float* env, float* ev_out,
                                  float* dist_out, void* stream) {
    GeoConst g;
    if (int s = make_geo(g, jd1, jd2, perm9, cutoff, coeff)) return s;
    if (E == 0) return ATOM_OK;
    cudaStream_t st = (cudaStream_t)stream;
    geometry_fwd_kernel<<<ceil_div(E, 128), 128, 0, st>>>(pos, src, tgt, img, shifts, E, g, coef,
                                                         env, ev_out, dist_out);
    ATOM_CHECK_LAUNCH("edge_geometry");
    if (gauss && NB > 0) {
        if (NB % 4 == 0 && aligned16(gauss) && aligned16(offset))
            gauss4_kernel<<<(unsigned)E, 128, 0, st>>>(pos, src, tgt, img, shifts, E, offset, NB,
                                                      coeff, gauss);
        else
            gauss_kernel<<<ceil_div(E * NB, 256), 256, 0, st>>>(pos, src, tgt, img, shifts, E,
                                                               offset, NB, coeff, gauss);
        ATOM_CHECK_LAUNCH("gauss");
    }
    return ATOM_OK;
}

extern "C" int atom_edge_geometry_bwd(const float* pos, const int* src, const int* tgt,
                                      const int* img, const float* shifts, int64_t E,
                                      const float* jd1, const float* jd2, const int* perm9,
                                      const float* offset, int NB, float coeff, float cutoff,
                                      const float* g_coef, const float* gauss,
                                      const float* g_gauss, const float* g_env, float* g_ev,
                                      void* stream) {
    GeoConst g;
    if (int s = make_geo(g, jd1, jd2, perm9, cutoff, coeff)) return s;
    ATOM_REQUIRE(!g_gauss || gauss, "g_gauss needs gauss");
    if (E == 0) return ATOM_OK;
    geometry_bwd_kernel<<<ceil_div(E, 128), 128, 0, (cudaStream_t)stream>>>(
        pos, src, tgt, img, shifts, E, g, offset, NB, g_coef, gauss, g_gauss, g_env, g_ev);
    ATOM_CHECK_LAUNCH("edge_geometry_bwd");
    return ATOM_OK;
}

extern "C" int atom_forces_virial(const float* g_ev, const float* ev, int64_t E, int64_t N,
                                  const int* recv_ptr, const int* send_ptr, const int* send_eid,
                                  float* forces, float* virial, float* scratch, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (N > 0) {
        forces_kernel<<<ceil_div(N, 128), 128, 0, st>>>(g_ev, N, recv_ptr, send_ptr, send_eid,
                                                        forces);
        ATOM_CHECK_LAUNCH("forces");
    }
    if (virial) {
        ATOM_REQUIRE(scratch && ev, "virial needs ev and scratch");
        virial_partial_kernel<<<kVirBlocks, 256, 0, st>>>(g_ev, ev, E, scratch);
        ATOM_CHECK_LAUNCH("virial_partial");
        virial_final_kernel<<<1, 256, 0, st>>>(scratch, virial);
        ATOM_CHECK_LAUNCH("virial_final");
    }
    return ATOM_OK;
}
