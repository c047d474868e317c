// Device neighbour list with the reference's fp32 predicate and edge order, plus the CSR
// helpers (prefix scan, sender CSR).
//
// Reference: tt_atom/geometry.py:48-81 (radius_graph). Aperiodic pairs are kept when
// ||pos[a] - pos[b]|| < cutoff (torch.linalg.norm, which on the CPU evaluates
// sqrt(fma(z, z, fma(y, y, x*x))) correctly rounded) and the edge list is ordered by
// (source a, target b). Periodic triples (i, j, c) are kept when
// |pos[i] - (pos[j] + shift[c])|^2 <= cutoff^2 and > 1e-8, with the square summed as
// (x*x + y*y) + z*z, no fused multiply-add, and ordered by (receiver i, source j, image c).
//
// This kernel emits receiver-major lists: receiver i, sources in (j, c) order. For periodic
// systems that IS the reference order. For aperiodic systems the distance is symmetric, so the
// per-receiver lists are the reference edge set transposed; the reference (source-major) order
// is recovered from the sender CSR (atom_sender_csr).
//
// Optional cap (not in the reference): keep per receiver the max_nbrs candidates with the
// smallest distance measure (aperiodic: distance, periodic: squared distance), ties broken by
// candidate order; survivors keep candidate order.
#include <climits>
#include "common.cuh"

namespace atom {

struct SysRange {
    // per-receiver candidate range [lo, hi) is the receiver's own system
    const long long* sys_ptr;
    int nsys;
};

__device__ __forceinline__ int find_sys(const long long* sp, int nsys, long long i) {
    int lo = 0, hi = nsys;   // sp[lo] <= i < sp[hi]
    while (hi - lo > 1) {
        int mid = (lo + hi) >> 1;
        if (sp[mid] <= i) lo = mid; else hi = mid;
    }
    return lo;
}

// The cap: rank each of a receiver's cnt candidates (in candidate order) by (key, position),
// drop those ranked >= max_nbrs and compact the survivors in place, in order. Whole warp.
__device__ int cap_candidates(int* ci, float* cd, int cnt, int max_nbrs, int lane) {
    for (int a = lane; a < cnt; a += 32) {
        float ka = cd[a];
        int rank = 0;
        for (int b = 0; b < cnt; ++b) {
            float kb = cd[b];
            rank += (kb < ka) || (kb == ka && b < a);
        }
        if (rank >= max_nbrs) ci[a] |= (int)0x80000000;
    }
    __syncwarp();
    int w = 0;
    for (int base = 0; base < cnt; base += 32) {
        int a = base + lane;
        int v = a < cnt ? ci[a] : (int)0x80000000;
        float d = a < cnt ? cd[a] : 0.f;
        bool s = v >= 0;
        unsigned m = __ballot_sync(0xffffffffu, s);
        __syncwarp();
        if (s) {
            int slot = w + __popc(m & ((1u << lane) - 1u));
            ci[slot] = v;
            cd[slot] = d;
        }
        __syncwarp();
        w += __popc(m);
    }
    return w;
}

// Pass 1: one warp per receiver, candidates in (j, c) order tested 32 at a time; the survivors
// are appended in order (ballot + popc) to the receiver's candidate slots.
// Images that cannot hold a neighbour of receiver i are skipped: image c is kept only if the
// bounding box of all positions, shifted by shift[c], comes within the cutoff of pos[i] (with
// a relative slack far above fp32 rounding, so no pair that passes the exact test is skipped).
// Candidates stay in (j, c) order.
struct BBox {
    float lo[3], hi[3];
};

__global__ void nl_collect_kernel(const float* __restrict__ pos, long long N,
                                  const long long* __restrict__ sys_ptr, int nsys,
                                  const float* __restrict__ shifts, int S, float cutoff,
                                  float cut2, int periodic, int max_nbrs, int max_cand,
                                  BBox box, const float* __restrict__ box_dev,
                                  int* __restrict__ cand_idx,
                                  float* __restrict__ cand_d, int* __restrict__ recv_cnt,
                                  int* __restrict__ need) {
    long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= N) return;
    long long lo = 0, hi = N;          // sys_ptr NULL: one system
    if (sys_ptr) {
        int k = find_sys(sys_ptr, nsys, i);
        lo = sys_ptr[k];
        hi = sys_ptr[k + 1];
    }
    if (box_dev) {                     // bounding box computed on the device
        for (int k = 0; k < 3; ++k) {
            box.lo[k] = box_dev[k];
            box.hi[k] = box_dev[3 + k];
        }
    }
    float pix = pos[i * 3 + 0], piy = pos[i * 3 + 1], piz = pos[i * 3 + 2];
    // surviving images for this receiver (all lanes compute the same list)
    unsigned char surv[256];
    int ns = 0;
    for (int c = 0; c < S; ++c) {
        if (!periodic) { surv[ns++] = (unsigned char)c; continue; }
        float d2 = 0.f;
        const float p[3] = {pix, piy, piz};
        for (int k = 0; k < 3; ++k) {
            float a = box.lo[k] + shifts[c * 3 + k], b = box.hi[k] + shifts[c * 3 + k];
            float d = p[k] < a ? a - p[k] : (p[k] > b ? p[k] - b : 0.f);
            d2 += d * d;
        }
        if (d2 <= cut2 * 1.0001f + 1e-3f) surv[ns++] = (unsigned char)c;
    }
    long long total = (hi - lo) * (long long)ns;
    int cnt = 0;
    int* ci = cand_idx + i * (long long)max_cand;
    float* cd = cand_d + i * (long long)max_cand;
    const float tiny = 1e-8f;
    for (long long base = 0; base < total; base += 32) {
        long long t = base + lane;
        bool keep = false;
        float key = 0.f;
        int tidx = 0;
        if (t < total) {
            long long j = lo + t / ns;
            int c = surv[t % ns];
            tidx = (int)((j - lo) * S + c);
            float pjx = pos[j * 3 + 0], pjy = pos[j * 3 + 1], pjz = pos[j * 3 + 2];
            if (periodic) {
                float qx = __fadd_rn(pjx, shifts[c * 3 + 0]);
                float qy = __fadd_rn(pjy, shifts[c * 3 + 1]);
                float qz = __fadd_rn(pjz, shifts[c * 3 + 2]);
                float dx = __fsub_rn(pix, qx), dy = __fsub_rn(piy, qy), dz = __fsub_rn(piz, qz);
                float d2 = __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)),
                                     __fmul_rn(dz, dz));
                keep = (d2 <= cut2) && (d2 > tiny);
                key = d2;
            } else {
                // the reference evaluates ||pos[a] - pos[b]|| with a = source j, b = receiver i
                float dx = __fsub_rn(pjx, pix), dy = __fsub_rn(pjy, piy), dz = __fsub_rn(pjz, piz);
                float d = __fsqrt_rn(__fmaf_rn(dz, dz, __fmaf_rn(dy, dy, __fmul_rn(dx, dx))));
                keep = (d < cutoff) && (d > 0.f);
                key = d;
            }
        }
        unsigned m = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            int slot = cnt + __popc(m & ((1u << lane) - 1u));
            if (slot < max_cand) {
                ci[slot] = tidx;
                cd[slot] = key;
            }
        }
        cnt += __popc(m);
    }
    if (cnt > max_cand) {
        if (lane == 0) atomicMax(need, cnt);
        if (lane == 0) recv_cnt[i] = 0;
        return;
    }
    int kept = cnt;
    __syncwarp();
    if (max_nbrs > 0 && cnt > max_nbrs) kept = cap_candidates(ci, cd, cnt, max_nbrs, lane);
    if (lane == 0) recv_cnt[i] = kept;
}

// ------------------------------------------------------------------------ cell list
// Periodic single systems: atoms are binned by their wrapped fractional coordinates
// w = f - floor(f), f = pos @ inv_cell (double), into nb[0] x nb[1] x nb[2] bins whose width
// along lattice direction k is at least the cutoff (plus slack) measured across the lattice
// planes. A receiver scans the bins within reach[k] of its own (27 for nb >= 3), each bin
// taken with the lattice translation L its extended index implies. Atom j seen in bin-extended
// position L stands for the image pos[j] + shift[c] with integer offset
// o = n_i + L - n_j (n = floor(f)); the candidate exists only when o lies in the shifts
// table's range [-r, r]^3, and it is then tested with exactly the brute-force expression on
// pos[j] and shifts[c]. Each (j, o) is met at most once, and every pair within the cutoff lies
// within reach, so the accepted set equals the brute force's. Candidates arrive in bin order;
// they are sorted back into (j, c) order before the cap is applied, so the result is the
// brute force's bit for bit.

__device__ __forceinline__ void frac_of(const float* __restrict__ pos, long long j,
                                       const atom_cell_grid& G, double f[3]) {
    const double p0 = pos[j * 3], p1 = pos[j * 3 + 1], p2 = pos[j * 3 + 2];
    for (int k = 0; k < 3; ++k)
        f[k] = p0 * G.inv_cell[0 * 3 + k] + p1 * G.inv_cell[1 * 3 + k] + p2 * G.inv_cell[2 * 3 + k];
}

__device__ __forceinline__ void wrap_bin(const double f[3], const int nb[3], int b[3], int n[3]) {
    for (int k = 0; k < 3; ++k) {
        const double fl = floor(f[k]);
        const double w = f[k] - fl;
        n[k] = (int)fl;
        int bk = (int)(w * nb[k]);
        b[k] = bk < 0 ? 0 : (bk >= nb[k] ? nb[k] - 1 : bk);
    }
}

__global__ void cl_bin_kernel(const float* __restrict__ pos, long long N, atom_cell_grid G) {
    long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= N) return;
    double f[3];
    int b[3], n[3];
    frac_of(pos, j, G, f);
    wrap_bin(f, G.nb, b, n);
    const int bin = (b[0] * G.nb[1] + b[1]) * G.nb[2] + b[2];
    G.atom_bin[j] = bin;
    for (int k = 0; k < 3; ++k) G.atom_off[j * 3 + k] = n[k];
    atomicAdd(G.bin_cnt + bin, 1);
}

__global__ void cl_fill_kernel(long long N, atom_cell_grid G) {
    long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= N) return;
    const int bin = G.atom_bin[j];
    const int slot = atomicAdd(G.bin_cnt + bin, 1);     // bin_cnt was cleared after the scan
    G.bin_atoms[G.bin_ptr[bin] + slot] = (int)j;
}

constexpr int kSortPerLane = 8;    // candidates a lane holds while sorting (max_cand <= 256)

__global__ void nl_collect_cells_kernel(const float* __restrict__ pos, long long N,
                                        const float* __restrict__ shifts, int S, float cut2,
                                        int max_nbrs, int max_cand, atom_cell_grid G,
                                        int* __restrict__ cand_idx, float* __restrict__ cand_d,
                                        int* __restrict__ recv_cnt, int* __restrict__ need) {
    long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= N) return;
    const float pix = pos[i * 3 + 0], piy = pos[i * 3 + 1], piz = pos[i * 3 + 2];
    double f[3];
    int bi[3], ni[3];
    frac_of(pos, i, G, f);
    wrap_bin(f, G.nb, bi, ni);
    const int w1 = 2 * G.img_r[1] + 1, w2 = 2 * G.img_r[2] + 1;
    int* ci = cand_idx + i * (long long)max_cand;
    float* cd = cand_d + i * (long long)max_cand;
    const float tiny = 1e-8f;
    int cnt = 0;
    for (int e0 = bi[0] - G.reach[0]; e0 <= bi[0] + G.reach[0]; ++e0)
        for (int e1 = bi[1] - G.reach[1]; e1 <= bi[1] + G.reach[1]; ++e1)
            for (int e2 = bi[2] - G.reach[2]; e2 <= bi[2] + G.reach[2]; ++e2) {
                const int e[3] = {e0, e1, e2};
                int bin = 0, L[3];
                for (int k = 0; k < 3; ++k) {
                    int q = e[k] % G.nb[k];
                    if (q < 0) q += G.nb[k];
                    L[k] = (e[k] - q) / G.nb[k];
                    bin = bin * G.nb[k] + q;
                }
                const int a0 = G.bin_ptr[bin], a1 = G.bin_ptr[bin + 1];
                for (int base = a0; base < a1; base += 32) {
                    const int t = base + lane;
                    bool keep = false;
                    int tidx = 0;
                    float key = 0.f;
                    if (t < a1) {
                        const int j = G.bin_atoms[t];
                        int o[3];
                        bool inr = true;
                        for (int k = 0; k < 3; ++k) {
                            o[k] = ni[k] + L[k] - G.atom_off[j * 3 + k];
                            inr = inr && o[k] >= -G.img_r[k] && o[k] <= G.img_r[k];
                        }
                        if (inr) {
                            const int c = ((o[0] + G.img_r[0]) * w1 + (o[1] + G.img_r[1])) * w2 +
                                          (o[2] + G.img_r[2]);
                            const float qx = __fadd_rn(pos[j * 3 + 0], shifts[c * 3 + 0]);
                            const float qy = __fadd_rn(pos[j * 3 + 1], shifts[c * 3 + 1]);
                            const float qz = __fadd_rn(pos[j * 3 + 2], shifts[c * 3 + 2]);
                            const float dx = __fsub_rn(pix, qx), dy = __fsub_rn(piy, qy),
                                        dz = __fsub_rn(piz, qz);
                            const float d2 = __fadd_rn(
                                __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
                            keep = (d2 <= cut2) && (d2 > tiny);
                            key = d2;
                            tidx = j * S + c;
                        }
                    }
                    const unsigned m = __ballot_sync(0xffffffffu, keep);
                    if (keep) {
                        const int slot = cnt + __popc(m & ((1u << lane) - 1u));
                        if (slot < max_cand) {
                            ci[slot] = tidx;
                            cd[slot] = key;
                        }
                    }
                    cnt += __popc(m);
                }
            }
    if (cnt > max_cand) {
        if (lane == 0) {
            atomicMax(need, cnt);
            recv_cnt[i] = 0;
        }
        return;
    }
    __syncwarp();
    // back into (j, c) order: rank of each candidate by its index, then scatter
    int vi[kSortPerLane], rk[kSortPerLane];
    float vd[kSortPerLane];
#pragma unroll
    for (int q = 0; q < kSortPerLane; ++q) {
        const int a = lane + 32 * q;
        vi[q] = a < cnt ? ci[a] : 0;
        vd[q] = a < cnt ? cd[a] : 0.f;
        int r = 0;
        if (a < cnt)
            for (int b = 0; b < cnt; ++b) r += ci[b] < vi[q];
        rk[q] = r;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < kSortPerLane; ++q) {
        if (lane + 32 * q < cnt) {
            ci[rk[q]] = vi[q];
            cd[rk[q]] = vd[q];
        }
    }
    __syncwarp();
    int kept = cnt;
    if (max_nbrs > 0 && cnt > max_nbrs) kept = cap_candidates(ci, cd, cnt, max_nbrs, lane);
    if (lane == 0) recv_cnt[i] = kept;
}

// Pass 2: copy each receiver's survivors to its CSR slots.
__global__ void nl_fill_kernel(long long N, const long long* __restrict__ sys_ptr, int nsys,
                               int S, int max_cand, const int* __restrict__ cand_idx,
                               const int* __restrict__ recv_cnt, const int* __restrict__ recv_ptr,
                               int* __restrict__ esrc, int* __restrict__ etgt,
                               int* __restrict__ eimg) {
    long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= N) return;
    int k = find_sys(sys_ptr, nsys, i);
    long long lo = sys_ptr[k];
    int n = recv_cnt[i], o = recv_ptr[i];
    const int* ci = cand_idx + i * (long long)max_cand;
    for (int a = lane; a < n; a += 32) {
        int t = ci[a];
        esrc[o + a] = (int)(lo + t / S);
        etgt[o + a] = (int)i;
        if (eimg) eimg[o + a] = t % S;
    }
}

// Exclusive scan, one 1024-thread block walking the array in chunks.
__global__ void scan_kernel(const int* __restrict__ cnt, long long n, int* __restrict__ ptr) {
    __shared__ int sh[1024];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (long long base = 0; base < n; base += 1024) {
        long long i = base + threadIdx.x;
        int v = i < n ? cnt[i] : 0;
        sh[threadIdx.x] = v;
        __syncthreads();
        for (int o = 1; o < 1024; o <<= 1) {
            int t = threadIdx.x >= o ? sh[threadIdx.x - o] : 0;
            __syncthreads();
            sh[threadIdx.x] += t;
            __syncthreads();
        }
        if (i < n) ptr[i] = carry + sh[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 1023) carry += sh[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) ptr[n] = carry;
}

__global__ void count_src_kernel(const int* __restrict__ src, long long E, int* __restrict__ cnt) {
    long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) atomicAdd(cnt + src[e], 1);
}

__global__ void zero_int_kernel(int* p, long long n) {
    long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) p[t] = 0;
}

__global__ void scatter_src_kernel(const int* __restrict__ src, long long E,
                                   const int* __restrict__ ptr, int* __restrict__ fill,
                                   int* __restrict__ eid) {
    long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) {
        int s = src[e];
        int slot = atomicAdd(fill + s, 1);
        eid[ptr[s] + slot] = (int)e;
    }
}

// Sort each sender's segment ascending (one warp per node; odd-even transposition over the
// segment, which is short).
__global__ void sort_segments_kernel(long long N, const int* __restrict__ ptr,
                                     int* __restrict__ eid) {
    long long n = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (n >= N) return;
    int b = ptr[n], len = ptr[n + 1] - b;
    int* s = eid + b;
    for (int phase = 0; phase < len; ++phase) {
        for (int a = 2 * lane + (phase & 1); a + 1 < len; a += 64) {
            int x = s[a], y = s[a + 1];
            if (x > y) {
                s[a] = y;
                s[a + 1] = x;
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------ device-resident refresh
// Bounding box of the positions (one block): lo[3], hi[3] into box.
__global__ void bbox_kernel(const float* __restrict__ pos, long long N, float* __restrict__ box) {
    __shared__ float red[6][32];
    float v[6] = {3.0e38f, 3.0e38f, 3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};
    for (long long i = threadIdx.x; i < N; i += blockDim.x) {
        for (int k = 0; k < 3; ++k) {
            float p = pos[i * 3 + k];
            v[k] = fminf(v[k], p);
            v[3 + k] = fmaxf(v[3 + k], p);
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int k = 0; k < 6; ++k) {
        for (int o = 16; o > 0; o >>= 1) {
            float w = __shfl_xor_sync(0xffffffffu, v[k], o);
            v[k] = k < 3 ? fminf(v[k], w) : fmaxf(v[k], w);
        }
        if (lane == 0) red[k][warp] = v[k];
    }
    __syncthreads();
    if (threadIdx.x < 6) {
        const int k = threadIdx.x, nw = blockDim.x >> 5;
        float r = red[k][0];
        for (int w = 1; w < nw; ++w) r = k < 3 ? fminf(r, red[k][w]) : fmaxf(r, red[k][w]);
        box[k] = r;
    }
}

// Commit the rebuilt list: when no receiver overflowed its candidate slots and the new edge
// count equals the caller's, write the edges (receiver-major) and the receiver CSR into the
// caller's arrays; otherwise leave them untouched and record why in status.
__global__ void nl_commit_kernel(long long N, int S, int max_cand,
                                 const int* __restrict__ cand_idx,
                                 const int* __restrict__ recv_cnt,
                                 const int* __restrict__ stage_ptr, long long E_expected,
                                 int* __restrict__ status, int* __restrict__ recv_ptr,
                                 int* __restrict__ esrc, int* __restrict__ etgt,
                                 int* __restrict__ eimg) {
    const long long total = stage_ptr[N];
    const int overflow = status[2];          // written by the collect pass (atomicMax)
    long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (overflow > 0 || total != E_expected) {
        if (gt == 0) {
            status[0] = overflow > 0 ? ATOM_REFRESH_OVERFLOW : ATOM_REFRESH_SIZE_CHANGED;
            status[1] = (int)total;
        }
        return;
    }
    if (gt == 0) {
        status[0] = ATOM_REFRESH_OK;
        status[1] = (int)total;
    }
    for (long long t = gt; t <= N; t += (long long)gridDim.x * blockDim.x) recv_ptr[t] = stage_ptr[t];
    long long i = gt >> 5;
    int lane = threadIdx.x & 31;
    if (i >= N) return;
    int n = recv_cnt[i], o = stage_ptr[i];
    const int* ci = cand_idx + i * (long long)max_cand;
    for (int a = lane; a < n; a += 32) {
        int t = ci[a];
        esrc[o + a] = t / S;
        etgt[o + a] = (int)i;
        eimg[o + a] = t % S;
    }
}

// Bins of the cell list (see nl_collect_cells_kernel); 5 launches, no host synchronisation.
static int build_bins(const float* pos, long long N, const atom_cell_grid& G, cudaStream_t st) {
    const long long nbins = (long long)G.nb[0] * G.nb[1] * G.nb[2];
    cudaError_t ce = cudaMemsetAsync(G.bin_cnt, 0, nbins * sizeof(int), st);
    if (ce == cudaSuccess) {
        cl_bin_kernel<<<ceil_div(N, 256), 256, 0, st>>>(pos, N, G);
        scan_kernel<<<1, 1024, 0, st>>>(G.bin_cnt, nbins, G.bin_ptr);
        ce = cudaMemsetAsync(G.bin_cnt, 0, nbins * sizeof(int), st);
    }
    if (ce == cudaSuccess) cl_fill_kernel<<<ceil_div(N, 256), 256, 0, st>>>(N, G);
    if (ce != cudaSuccess) {
        set_error("cell list: %s", cudaGetErrorString(ce));
        return ATOM_ERR_CUDA;
    }
    return check_launch("cell list bins", 3);
}

static int check_grid(const atom_cell_grid* g, int max_cand, int nshift) {
    if (!g) return ATOM_OK;
    ATOM_REQUIRE(max_cand <= 32 * kSortPerLane, "cell list: max_cand above %d",
                 32 * kSortPerLane);
    for (int k = 0; k < 3; ++k)
        ATOM_REQUIRE(g->nb[k] >= 1 && g->reach[k] >= 1 && g->img_r[k] >= 0,
                     "cell list: bad grid on axis %d", k);
    ATOM_REQUIRE((2 * g->img_r[0] + 1) * (2 * g->img_r[1] + 1) * (2 * g->img_r[2] + 1) == nshift,
                 "cell list: image ranges do not match nshift");
    ATOM_REQUIRE((long long)g->nb[0] * g->nb[1] * g->nb[2] <= (1LL << 24),
                 "cell list: too many bins");
    ATOM_REQUIRE(g->atom_bin && g->atom_off && g->bin_cnt && g->bin_ptr && g->bin_atoms,
                 "cell list: a scratch buffer is NULL");
    return ATOM_OK;
}

}  // namespace atom

using namespace atom;

extern "C" int atom_neighbor_refresh(const float* pos, int64_t N, const float* shifts,
                                     int nshift, float cutoff, int periodic, int max_nbrs,
                                     int max_cand, int* cand_idx, float* cand_d, int* recv_cnt,
                                     int* stage_ptr, float* box_scratch, int* status,
                                     int64_t E_expected, int* recv_ptr, int* edge_src,
                                     int* edge_tgt, int* edge_img,
                                     const atom_cell_grid* grid, void* stream) {
    ATOM_REQUIRE(N >= 1 && nshift >= 1 && nshift <= 255 && max_cand >= 1,
                 "neighbor_refresh: N, nshift (1..255) and max_cand must be positive");
    ATOM_REQUIRE(N * (long long)nshift < (1LL << 31), "N * nshift too large for this kernel");
    ATOM_REQUIRE(E_expected >= 0 && E_expected <= INT_MAX, "E_expected out of range");
    ATOM_REQUIRE(cand_idx && cand_d && recv_cnt && stage_ptr && status && recv_ptr && edge_src &&
                     edge_tgt && edge_img && (!periodic || box_scratch),
                 "neighbor_refresh: a required buffer is NULL");
    ATOM_REQUIRE(!grid || periodic, "the cell list takes a periodic system");
    if (int s = check_grid(grid, max_cand, nshift)) return s;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t ce = cudaMemsetAsync(status, 0, 4 * sizeof(int), st);
    if (ce != cudaSuccess) {
        set_error("neighbor_refresh: %s", cudaGetErrorString(ce));
        return ATOM_ERR_CUDA;
    }
    BBox box;
    for (int k = 0; k < 3; ++k) {
        box.lo[k] = -3.0e38f;
        box.hi[k] = 3.0e38f;
    }
    float cut2 = (float)((double)cutoff * (double)cutoff);
    if (grid) {
        if (int s2 = build_bins(pos, N, *grid, st)) return s2;
        nl_collect_cells_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(
            pos, N, shifts, nshift, cut2, max_nbrs, max_cand, *grid, cand_idx, cand_d, recv_cnt,
            status + 2);
    } else {
        if (periodic) bbox_kernel<<<1, 1024, 0, st>>>(pos, N, box_scratch);
        nl_collect_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(
            pos, N, nullptr, 1, shifts, nshift, cutoff, cut2, periodic, max_nbrs, max_cand, box,
            periodic ? box_scratch : nullptr, cand_idx, cand_d, recv_cnt, status + 2);
    }
    scan_kernel<<<1, 1024, 0, st>>>(recv_cnt, N, stage_ptr);
    nl_commit_kernel<<<ceil_div((N + 1) * 32, 256), 256, 0, st>>>(
        N, nshift, max_cand, cand_idx, recv_cnt, stage_ptr, E_expected, status, recv_ptr,
        edge_src, edge_tgt, edge_img);
    ATOM_CHECK_LAUNCHES("neighbor_refresh", (periodic && !grid) ? 4 : 3);
    return ATOM_OK;
}

extern "C" int atom_neighbor_list(const float* pos, int64_t N, const int64_t* sys_ptr_host,
                                  int nsys, const float* shifts, int nshift, float cutoff,
                                  int periodic, int max_nbrs, int max_cand, int* cand_idx,
                                  float* cand_d, int* recv_cnt, const int* recv_ptr,
                                  int* edge_src, int* edge_tgt, int* edge_img,
                                  const float* bbox_host, void* small_scratch, int* need_host,
                                  const atom_cell_grid* grid, void* stream) {
    ATOM_REQUIRE(nsys >= 1 && nsys <= 1 << 20, "nsys out of range");
    ATOM_REQUIRE(nshift >= 1 && max_cand >= 1, "nshift and max_cand must be positive");
    ATOM_REQUIRE(nshift <= 255, "at most 255 periodic images (cell too small for the cutoff)");
    ATOM_REQUIRE(sys_ptr_host[0] == 0 && sys_ptr_host[nsys] == N, "sys_ptr must span [0, N)");
    ATOM_REQUIRE(N * (long long)nshift < (1LL << 31), "N * nshift too large for this kernel");
    ATOM_REQUIRE(!grid || (nsys == 1 && periodic), "the cell list takes one periodic system");
    if (int s = check_grid(grid, max_cand, nshift)) return s;
    cudaStream_t st = (cudaStream_t)stream;
    if (N == 0) return ATOM_OK;
    ATOM_REQUIRE(small_scratch && (reinterpret_cast<uintptr_t>(small_scratch) & 7u) == 0,
                 "small_scratch must be 8-byte aligned");
    // system offsets and the capacity flag live in the caller's small scratch
    long long* sp = reinterpret_cast<long long*>(small_scratch);
    cudaError_t ce = cudaMemcpyAsync(sp, sys_ptr_host, (nsys + 1) * sizeof(long long),
                                     cudaMemcpyHostToDevice, st);
    if (ce != cudaSuccess) {
        set_error("neighbor_list: copy of system offsets failed: %s", cudaGetErrorString(ce));
        return ATOM_ERR_CUDA;
    }
    if (edge_src == nullptr) {
        int* dneed = reinterpret_cast<int*>(sp + nsys + 1);
        cudaMemsetAsync(dneed, 0, sizeof(int), st);
        float cut2 = (float)((double)cutoff * (double)cutoff);
        BBox box;
        for (int k = 0; k < 3; ++k) {
            box.lo[k] = bbox_host ? bbox_host[k] : -3.0e38f;
            box.hi[k] = bbox_host ? bbox_host[3 + k] : 3.0e38f;
        }
        if (grid) {
            if (int s2 = build_bins(pos, N, *grid, st)) return s2;
            nl_collect_cells_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(
                pos, N, shifts, nshift, cut2, max_nbrs, max_cand, *grid, cand_idx, cand_d,
                recv_cnt, dneed);
        } else {
            nl_collect_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(
                pos, N, sp, nsys, shifts, nshift, cutoff, cut2, periodic, max_nbrs, max_cand,
                box, nullptr, cand_idx, cand_d, recv_cnt, dneed);
        }
        ATOM_CHECK_LAUNCH("neighbor_list collect");
        int h = 0;
        ce = cudaMemcpyAsync(&h, dneed, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            set_error("neighbor_list: %s", cudaGetErrorString(ce));
            return ATOM_ERR_CUDA;
        }
        if (need_host) *need_host = h;
        if (h > 0) {
            set_error("neighbor_list: a receiver has %d candidates > max_cand %d", h, max_cand);
            return ATOM_ERR_CAPACITY;
        }
        return ATOM_OK;
    }
    ATOM_REQUIRE(recv_ptr && edge_tgt, "pass 2 needs recv_ptr and edge_tgt");
    nl_fill_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(N, sp, nsys, nshift, max_cand, cand_idx,
                                                        recv_cnt, recv_ptr, edge_src, edge_tgt,
                                                        edge_img);
    ATOM_CHECK_LAUNCH("neighbor_list fill");
    return ATOM_OK;
}

extern "C" int atom_exclusive_scan(const int* cnt, int64_t n, int* ptr, int* total_host,
                                   void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    scan_kernel<<<1, 1024, 0, st>>>(cnt, n, ptr);
    ATOM_CHECK_LAUNCH("exclusive_scan");
    if (total_host) {
        cudaError_t ce = cudaMemcpyAsync(total_host, ptr + n, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) {
            set_error("exclusive_scan: %s", cudaGetErrorString(ce));
            return ATOM_ERR_CUDA;
        }
    }
    return ATOM_OK;
}

extern "C" int atom_sender_csr(const int* edge_src, int64_t E, int64_t N, int* scratch,
                               int* send_ptr, int* send_eid, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    ATOM_REQUIRE(N >= 0 && E >= 0, "sender_csr: negative size");
    if (E > INT_MAX) {
        set_error("sender_csr: E = %lld exceeds the int32 edge ids of the CSR", (long long)E);
        return ATOM_ERR_CAPACITY;
    }
    if (N == 0) return ATOM_OK;
    zero_int_kernel<<<ceil_div(N, 256), 256, 0, st>>>(scratch, N);
    if (E > 0) count_src_kernel<<<ceil_div(E, 256), 256, 0, st>>>(edge_src, E, scratch);
    scan_kernel<<<1, 1024, 0, st>>>(scratch, N, send_ptr);
    zero_int_kernel<<<ceil_div(N, 256), 256, 0, st>>>(scratch, N);
    if (E > 0) {
        scatter_src_kernel<<<ceil_div(E, 256), 256, 0, st>>>(edge_src, E, send_ptr, scratch,
                                                              send_eid);
        sort_segments_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(N, send_ptr, send_eid);
    }
    ATOM_CHECK_LAUNCHES("sender_csr", E > 0 ? 6 : 3);
    return ATOM_OK;
}

// ------------------------------------------------------------------ scratch-free sender CSR
// A variant of atom_sender_csr for callers that cannot allocate device memory. Its per-node
// fill counters live in a file-scope device array instead of caller scratch. Each GPU that
// loads this library holds the array (ATOM_NOALLOC_MAX_NODES int32, 4 MiB) until the process
// exits. In host code the array's name is only a host-side stand-in, so its device address is
// looked up once per device with cudaGetSymbolAddress (on the first call made with that device
// current) and passed to the kernels.
#include <mutex>

static __device__ __align__(256) int g_noalloc_fill[ATOM_NOALLOC_MAX_NODES];

namespace atom {
constexpr int kMaxDevices = 64;
static std::mutex g_noalloc_mu;
static int* g_noalloc_addr[kMaxDevices];

static int noalloc_scratch(int** out) {
    int dev = -1;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) {
        set_error("sender_csr_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(ce));
        return ATOM_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("sender_csr_noalloc: device ordinal %d out of range", dev);
        return ATOM_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        ce = cudaGetSymbolAddress(&p, g_noalloc_fill);
        if (ce != cudaSuccess || !p) {
            set_error("sender_csr_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(ce));
            return ATOM_ERR_CUDA;
        }
        g_noalloc_addr[dev] = static_cast<int*>(p);
    }
    *out = g_noalloc_addr[dev];
    return ATOM_OK;
}
}  // namespace atom

extern "C" int atom_sender_csr_noalloc(const int* edge_src, int64_t E, int64_t N, int* send_ptr,
                                       int* send_eid, void* stream) {
    ATOM_REQUIRE(N >= 0 && E >= 0, "sender_csr_noalloc: negative size");
    if (E > INT_MAX) {
        set_error("sender_csr_noalloc: E = %lld exceeds the int32 edge ids of the CSR",
                  (long long)E);
        return ATOM_ERR_CAPACITY;
    }
    if (N > ATOM_NOALLOC_MAX_NODES) {
        set_error("sender_csr_noalloc: N = %lld exceeds the built-in scratch of %d nodes; use "
                  "atom_sender_csr with caller-provided scratch", (long long)N,
                  ATOM_NOALLOC_MAX_NODES);
        return ATOM_ERR_CAPACITY;
    }
    if (N == 0) return ATOM_OK;
    int* fill = nullptr;
    if (int s = noalloc_scratch(&fill)) return s;
    cudaStream_t st = (cudaStream_t)stream;
    // the counters keep the previous call's values: clear them before counting and again
    // before the fill pass
    zero_int_kernel<<<ceil_div(N, 256), 256, 0, st>>>(fill, N);
    if (E > 0) count_src_kernel<<<ceil_div(E, 256), 256, 0, st>>>(edge_src, E, fill);
    scan_kernel<<<1, 1024, 0, st>>>(fill, N, send_ptr);
    zero_int_kernel<<<ceil_div(N, 256), 256, 0, st>>>(fill, N);
    if (E > 0) {
        scatter_src_kernel<<<ceil_div(E, 256), 256, 0, st>>>(edge_src, E, send_ptr, fill,
                                                              send_eid);
        sort_segments_kernel<<<ceil_div(N * 32, 256), 256, 0, st>>>(N, send_ptr, send_eid);
    }
    ATOM_CHECK_LAUNCHES("sender_csr_noalloc", E > 0 ? 6 : 3);
    return ATOM_OK;
}
