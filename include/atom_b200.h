/*
 * atom_b200.h -- C ABI of the B200 (sm_100a) eSCN-MD energy/force/stress kernels.
 *
 * Conventions for every entry point:
 *  - Pointers are CUDA device pointers unless named *_host; sizes are element counts.
 *  - All floating-point buffers are fp32, row-major, densely packed unless a leading dimension
 *    (ld*) is given. Index buffers are int32.
 *  - Outputs are allocated by the caller. No entry point allocates device memory, except
 *    atom_neighbor_list, which uses caller-provided scratch (see its comment).
 *  - `stream` is a cudaStream_t passed as void*; work is stream-ordered and asynchronous.
 *  - Return value: ATOM_OK (0) or an error code; atom_last_error() gives the message of the
 *    last failing call on this host thread. No C++ exception crosses this boundary.
 *
 * Node features are [N, 9, C] in the standard (l, m) spherical-harmonic order (lmax = 2).
 * Per-edge Wigner matrices are passed packed: the 35 structural nonzeros of the m-primed
 * rotation, row-major by m-primed row (row degrees 0,1,2,1,2,1,2,2,2; each row holds the
 * 2l+1 columns of its degree block).
 * Edges are processed in receiver-major order with a receiver CSR (recv_ptr[N+1]) and a sender
 * CSR (send_ptr[N+1], send_eid[E]: edge ids grouped by source node, ascending within a group).
 */
#ifndef ATOM_B200_H
#define ATOM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ATOM_OK = 0,
    ATOM_ERR_ARG = 1,          /* invalid argument, shape or alignment */
    ATOM_ERR_CUDA = 2,         /* CUDA runtime / launch error */
    ATOM_ERR_CAPACITY = 3,     /* a device-side capacity was exceeded (retry with more room) */
    ATOM_ERR_UNSUPPORTED = 4   /* shape the kernels do not implement */
};

/* Copies the last error message of this host thread into buf (NUL-terminated); returns its
 * full length. */
int atom_last_error(char* buf, size_t n);
/* ABI version of this library. */
int atom_abi_version(void);
/* Number of kernels this library has launched since it was loaded (all threads). Launches
 * replayed from a captured CUDA graph are not counted again. No counterpart in the reference. */
int atom_launch_count(int64_t* n);

/* ------------------------------------------------------------------------------------------
 * Reference-op equivalents. These four replace the nanobind ops of the reference's custom
 * kernel library (custom_kernels/fused_rotate/fused_rotate_nanobind.cpp:17-96) with the same
 * argument meaning; the reference returns a new tensor, here the caller passes the output.
 * ---------------------------------------------------------------------------------------- */

/* fused_rotate (fused_rotate_nanobind.cpp:71-93; semantics custom_kernels/README.md "contract"):
 *   out[e, i*W + w] = sum over the deg[i] nonzeros k of block i: coef[e, ks[k]] * x[e, js[k]*W + w]
 * x [E, n_in*W], coef [E, nnz] (compact: the reference's tile-broadcast coef_exp is a ttnn layout
 * detail), out [E, n_out*W]. deg[n_out], ks[nnz], js[nnz] are HOST arrays grouped by output
 * block in order. Limits: n_in, n_out <= 32, nnz <= 128, W % 4 == 0. */
int atom_fused_rotate(const float* x, const float* coef, int64_t E, int n_in, int n_out, int W,
                      int nnz, const int* deg_host, const int* ks_host, const int* js_host,
                      float* out, void* stream);

/* fused_rotate_gc (fused_rotate_nanobind.cpp:52-70): coefficient adjoint
 *   gc[e, k] = sum_w gout[e, is_[k]*W + w] * xin[e, js[k]*W + w]
 * gout [E, n_out*W], xin [E, n_in*W], gc [E, nnz]; is_/js HOST arrays of length nnz.
 * The reference's column-selector operand `sel` is a Tensix matmul-reduce device and has no
 * counterpart here. */
int atom_fused_rotate_gc(const float* gout, const float* xin, int64_t E, int n_out, int n_in,
                         int W, int nnz, const int* is_host, const int* js_host, float* gc,
                         void* stream);

/* fused_gate (fused_rotate_nanobind.cpp:35-51; tt_atom/activation.py:53-70):
 *   mode 0: out = [silu(a[:, :H]) | a[:, H:] * gate]
 *   mode 1: out = [a[:, :H] * silu'(b[:, :H]) | a[:, H:] * gate]
 * a, b, out [E, H + G]; gate [E, G] (the gate already expanded per vector coefficient). The
 * reference passes H, G and H+G in 32-column tiles (Ht, Gt, Wt); here they are columns. */
int atom_fused_gate(const float* a, const float* gate, const float* b, int64_t E, int H, int G,
                    int mode, float* out, void* stream);

/* fused_ln_bw (fused_rotate_nanobind.cpp:18-34; tt_atom/so2.py:117-128): LayerNorm backward
 * with the SiLU backward and the affine scale folded in:
 *   gy = g * silu'(n) * gamma;  dx = rstd * (gy - mean(gy) - xhat * mean(gy * xhat))
 * g, x (the LN input), n (the LN output = SiLU input), dx [rows, W]; gamma [W]. */
int atom_fused_ln_bw(const float* g, const float* x, const float* n, const float* gamma,
                     int64_t rows, int W, float eps, float* dx, void* stream);

/* ------------------------------------------------------------------------------------------
 * Graph construction. Replaces tt_atom/geometry.py:48-81 (radius_graph) on the device, with
 * the same fp32 predicate and the same edge order, plus an optional per-receiver cap.
 * ---------------------------------------------------------------------------------------- */

/* Cell list of one fully periodic system (optional argument of atom_neighbor_list and
 * atom_neighbor_refresh; NULL: all-pairs candidates with bounding-box image pruning). Atoms are
 * binned by wrapped fractional coordinates (pos @ inv_cell, row-major, computed in double)
 * into nb[0] x nb[1] x nb[2] bins; a receiver scans reach[k] bins on either side along lattice
 * direction k. Every bin must be at least the cutoff wide across its lattice planes with
 * reach = 1, or reach = ceil(cutoff |b_k| nb_k) otherwise (b_k: reciprocal vector, column k of
 * inv_cell). img_r[k]: the image offsets -r..r of the shifts table (cartesian-product order,
 * first axis slowest). Device scratch: atom_bin [N], atom_off [3 N], bin_cnt [nbins],
 * bin_ptr [nbins + 1], bin_atoms [N] int32. The edge list is identical to the all-pairs one;
 * max_cand must not exceed 256. No counterpart in the reference (its radius_graph is
 * all-pairs, tt_atom/geometry.py:48-81). */
typedef struct {
    double inv_cell[9];
    int nb[3];
    int reach[3];
    int img_r[3];
    int* atom_bin;
    int* atom_off;
    int* bin_cnt;
    int* bin_ptr;
    int* bin_atoms;
} atom_cell_grid;

/* Neighbour list of `nsys` independent systems stored back to back (sys_ptr[nsys+1] atom
 * offsets, host array). Each system is periodic with `nshift` image shifts (shifts [nshift,3],
 * device; the zero shift alone for aperiodic systems) -- all systems share pbc and shifts.
 * Aperiodic: keep (a, b) with ||pos[a]-pos[b]|| < cutoff, a != b. Periodic: keep (i, j, c) with
 * |pos[i] - (pos[j] + shift[c])|^2 <= cutoff^2 and > 1e-8. Output per receiver, sources in
 * (source, image) order; with max_nbrs > 0 only the max_nbrs nearest (ties: that order) stay.
 *   recv_cnt [N]         edges per receiver (device, written)
 *   cand_idx, cand_d     scratch of N * max_cand int32 / fp32 each (device; pass 1 writes,
 *                        pass 2 reads)
 *   bbox_host            HOST [6] = (min xyz, max xyz) of all positions, or NULL: images
 *                        whose shifted box lies beyond the cutoff of a receiver are skipped
 *                        (exact; only speeds up large cells). At most 255 images.
 *   small_scratch        8 * (nsys + 2) bytes of device scratch, 8-byte aligned
 * Pass 1 (edges == NULL): fills recv_cnt, returns ATOM_ERR_CAPACITY (with the needed max_cand
 * in *need) if a receiver has more than max_cand candidates.
 * Pass 2 (edges != NULL, recv_ptr = exclusive scan of recv_cnt): writes edge_src[E],
 * edge_tgt[E], edge_img[E] (image index) in receiver-major order. */
int atom_neighbor_list(const float* pos, int64_t N, const int64_t* sys_ptr_host, int nsys,
                       const float* shifts, int nshift, float cutoff, int periodic, int max_nbrs,
                       int max_cand, int* cand_idx, float* cand_d, int* recv_cnt,
                       const int* recv_ptr, int* edge_src, int* edge_tgt, int* edge_img,
                       const float* bbox_host, void* small_scratch, int* need_host,
                       const atom_cell_grid* grid, void* stream);

/* Device-resident rebuild of one system's neighbour list into an existing edge set's arrays,
 * for a caller that replays a step on fixed-size buffers (relaxation, MD, repeated single
 * points): same predicate, order and cap as atom_neighbor_list, no host synchronisation and no
 * host round trip, so it can be captured in a CUDA graph together with the step.
 * Scratch: cand_idx / cand_d [N * max_cand], recv_cnt [N], stage_ptr [N + 1], box_scratch
 * [6] floats (periodic: the bounding box for image pruning is computed on the device),
 * status [4] int32. When no receiver has more than max_cand candidates and the new edge count
 * equals E_expected, the edges (receiver-major) and recv_ptr [N + 1] are written to the
 * caller's arrays and status[0] = ATOM_REFRESH_OK; otherwise those arrays are left unchanged,
 * status[0] = ATOM_REFRESH_OVERFLOW or ATOM_REFRESH_SIZE_CHANGED, status[1] = the new edge
 * count and status[2] = the largest candidate count when it overflowed. Read status after the
 * stream has run it and fall back to atom_neighbor_list when it is not OK. The sender CSR and
 * per-edge species are then refreshed with atom_sender_csr / atom_edge_species (also
 * capturable). Replaces the per-step host radius_graph of tt_atom/trace.py:83-215's callers
 * (tt_atom/calculator.py:256-277), which this path keeps on the device. */
#define ATOM_REFRESH_OK 0
#define ATOM_REFRESH_OVERFLOW 1
#define ATOM_REFRESH_SIZE_CHANGED 2
int atom_neighbor_refresh(const float* pos, int64_t N, const float* shifts, int nshift,
                          float cutoff, int periodic, int max_nbrs, int max_cand, int* cand_idx,
                          float* cand_d, int* recv_cnt, int* stage_ptr, float* box_scratch,
                          int* status, int64_t E_expected, int* recv_ptr, int* edge_src,
                          int* edge_tgt, int* edge_img, const atom_cell_grid* grid,
                          void* stream);

/* Exclusive prefix sum of n int32 counts: ptr[0] = 0, ptr[i+1] = ptr[i] + cnt[i]; also copies
 * the total to *total_host (synchronous on `stream`) when total_host is not NULL. */
int atom_exclusive_scan(const int* cnt, int64_t n, int* ptr, int* total_host, void* stream);

/* Sender CSR: send_ptr[N+1] and send_eid[E] (edge ids grouped by source, ascending), from
 * edge_src[E]. scratch: N int32. Every edge_src value must lie in [0, N) (not checked on the
 * device); E above INT_MAX returns ATOM_ERR_CAPACITY (edge ids are int32). */
int atom_sender_csr(const int* edge_src, int64_t E, int64_t N, int* scratch, int* send_ptr,
                    int* send_eid, void* stream);

/* Scratch-free variant of atom_sender_csr. It has no counterpart in the reference.
 * For callers that cannot allocate device memory -- e.g. a host MD engine or framework whose
 * own pool allocator owns the device memory and forbids allocations behind its back -- and so
 * cannot provide atom_sender_csr's N-int scratch. The per-node counters live in a static
 * device array of ATOM_NOALLOC_MAX_NODES int32 (4 MiB) that every GPU loading this library
 * holds until the process exits; N above that limit returns ATOM_ERR_CAPACITY. The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current, so make that first call before any stream capture. Calls share the array: calls
 * that overlap on the GPU (other streams, other host threads) race and must be serialised by
 * the caller. Allocates nothing (no cudaMalloc / cudaFree). Output equals atom_sender_csr's.
 * As there, every edge_src value must lie in [0, N) -- an id outside it would count into the
 * shared array past node N -- and E above INT_MAX returns ATOM_ERR_CAPACITY. */
#define ATOM_NOALLOC_MAX_NODES (1 << 20)
int atom_sender_csr_noalloc(const int* edge_src, int64_t E, int64_t N, int* send_ptr,
                            int* send_eid, void* stream);

/* ------------------------------------------------------------------------------------------
 * Geometry (tt_atom/geometry.py:112-280) and its VJP (replaces the host autograd finish of
 * tt_atom/forces.py:545-589).
 * ---------------------------------------------------------------------------------------- */

/* Per edge: ev = pos[src] - pos[tgt] + shift[img]; dist = |ev|; packed Wigner coef [E,35]
 * (Euler angles with roll 0, D_l = J Z(-beta) J Z(-alpha), rows permuted by perm9);
 * gauss [E, NB] = exp(coeff (dist - offset_k)^2); env [E]: polynomial envelope p = 5.
 * jd1 [9], jd2 [25] host arrays (e3nn J matrices); perm9 host [9]: m-primed row -> coefficient.
 * ev_out [E,3] and dist_out [E] may be NULL. */
int atom_edge_geometry(const float* pos, const int* src, const int* tgt, const int* img,
                       const float* shifts, int64_t E, const float* jd1_host,
                       const float* jd2_host, const int* perm9_host, const float* offset,
                       int NB, float coeff, float cutoff, float* coef, float* gauss,
                       float* env, float* ev_out, float* dist_out, void* stream);

/* VJP of atom_edge_geometry: from g_coef [E,35], g_gauss [E,NB] (may be NULL) and g_env [E]
 * accumulates dE/d(edge vector) into g_ev [E,3] (overwritten). */
int atom_edge_geometry_bwd(const float* pos, const int* src, const int* tgt, const int* img,
                           const float* shifts, int64_t E, const float* jd1_host,
                           const float* jd2_host, const int* perm9_host, const float* offset,
                           int NB, float coeff, float cutoff, const float* g_coef,
                           const float* gauss, const float* g_gauss, const float* g_env,
                           float* g_ev, void* stream);

/* Forces F[n] = sum_{e: tgt=n} g_ev[e] - sum_{e: src=n} g_ev[e] (F = -dE/dpos), in a fixed
 * order, and the virial dE/d(strain) = sym(sum_e ev[e] (x) g_ev[e]) [3,3] (may be NULL).
 * scratch: 9 * 1024 floats when virial != NULL. */
int atom_forces_virial(const float* g_ev, const float* ev, int64_t E, int64_t N,
                       const int* recv_ptr, const int* send_ptr, const int* send_eid,
                       float* forces, float* virial, float* scratch, void* stream);

/* ------------------------------------------------------------------------------------------
 * Dense contractions.
 * ---------------------------------------------------------------------------------------- */

/* Grouped fp32 GEMM (up to 8 groups, one launch): for each group g,
 *   C[m, c_col[g] + n] (+)= act( sum_k A[m, a_col[g] + k] * B_g[k * ldb[g] + n] + bias_g[n]
 *                                + T1[idx1[m] * ldt + t_col[g] + n] + T2[idx2[m] * ldt + t_col[g] + n] )
 * for m < M, n < N_g, k < K_g. bias/T1/T2 optional (NULL). act: 0 none, 1 SiLU (then
 * C_pre, when not NULL, receives the pre-activation). accumulate != 0 adds into C.
 * precision: 0 = fp32 FMA; 1 = TF32 tensor cores (tcgen05); 2 = 3xTF32 tensor cores (fp32-level
 * accuracy); 3 = fp16-pair tensor cores (fp32-level accuracy at twice mode 2's MMA rate).
 * Modes 1 and 2 read the K-major weight copies Bt[g] ([N_g, K_g] row-major, low 13
 * mantissa bits cleared) and, for mode 2, Bt_lo[g] = B^T - Bt; they need every K_g to be a
 * multiple of 32, lda % 4 == 0 and 16-byte aligned A / Bt, and otherwise run the fp32 kernel.
 * Mode 3 reads, per group, s_n = 2^(14 - floor(log2 max_k |B[k, n]|)) (1 for a zero column),
 * Bh[g] = fp16(B^T s) and Bh_lo[g] = fp16((B^T s - Bh) * 2^11) ([N_g, K_g] fp16 row-major) and
 * Bh_inv[g] = 1 / s (N_g floats); it needs a scratch (atom_gemm_ex) of at least
 * ceil(ngroups * ceil(M / 128) * 128 / 64) * 64 floats for its per-row scales of A, and runs
 * as mode 2 without one. */
typedef struct {
    int ngroups;
    int a_col[8], K[8], c_col[8], N[8], ldb[8], t_col[8];
    const float* B[8];
    const float* bias[8];
    const float* Bt[8];
    const float* Bt_lo[8];
    const void* Bh[8];
    const void* Bh_lo[8];
    const float* Bh_inv[8];
} atom_gemm_groups;

int atom_gemm(const float* A, int64_t lda, int64_t M, const atom_gemm_groups* groups,
              float* Cout, int64_t ldc, float* C_pre, const float* T1, const float* T2,
              const int* idx1, const int* idx2, int64_t ldt, int act, int accumulate,
              int precision, void* stream);

/* atom_gemm with caller scratch (scratch_floats floats, stream-ordered, caller-owned): when a
 * launch has too few output tiles to occupy the GPU (few rows, e.g. node-level layers), the
 * tensor-core path splits each tile's K range over several CTAs, writes raw partial tiles to
 * the scratch (splits x ceil(M / 128) * 128 rows of ldc floats) and adds them in split order
 * (deterministic) before the bias / SiLU / accumulate epilogue. scratch NULL: as atom_gemm.
 * No counterpart in the reference (its ttnn matmuls choose their own core split). */
int atom_gemm_ex(const float* A, int64_t lda, int64_t M, const atom_gemm_groups* groups,
                 float* C, int64_t ldc, float* Cpre, const float* T1, const float* T2,
                 const int* idx1, const int* idx2, int64_t ldt, int act, int accumulate,
                 int precision, float* scratch, int64_t scratch_floats, void* stream);

/* The so2_2 GEMM with the gate fused into its A operand (the reference's so2_conv_2 on
 * GateActivation's output, tt_atom/activation.py:53-70 then tt_atom/so2.py:255-296): Y is the
 * so2_1 output [M, ldy >= 11 H] = [gating rows 0, 1 | m-primed rows 0..8], H channels each; the
 * GEMM's A operand is row 0 -> SiLU(row 0), row r >= 1 -> row r * sigmoid(gating row
 * (r in {1, 3, 5} ? 0 : 1)), formed where the tensor-core kernel converts A, so the gated rows
 * are never written to memory; the result equals atom_gate_fwd followed by atom_gemm_ex bit for
 * bit. Groups address Y's columns (a_col >= 2 H, 32-aligned, within rows 0..8) and carry their
 * biases as in atom_gemm_ex; no activation or accumulation. precision 2 or 3 only
 * (ATOM_ERR_UNSUPPORTED otherwise, and when the operands do not suit the tensor-core kernel). */
int atom_gemm_gated(const float* Y, int64_t ldy, int64_t M, const atom_gemm_groups* groups,
                    int H, float* C, int64_t ldc, int precision, float* scratch,
                    int64_t scratch_floats, void* stream);

/* Reads and clears the device-side error code of the tensor-core kernels and the streamed edge
 * kernels (0 = none; a bounded wait expired otherwise: codes 1-6 tensor-core pipeline waits,
 * ATOM_WAIT_SELFTEST_CODE, ATOM_EDGE_WAIT_CODE). Synchronises `stream`. */
int atom_device_error(int* code_host, void* stream);

/* Stream-ordered form of atom_device_error: copies the device-side error code into the device
 * int *code_dev and clears it, without synchronising, so a caller can read it back together
 * with a step's results in one copy. No counterpart in the reference. */
int atom_device_error_take(int* code_dev, void* stream);

/* Test hook for the bounded waits: one thread runs the tensor-core kernels' own bounded
 * mbarrier wait on a barrier that nothing arrives on, for budget_cycles SM clocks (1 ..
 * 2e9), then gives up and records ATOM_WAIT_SELFTEST_CODE in the device-side error code,
 * exactly as an expired wait inside a GEMM does; atom_device_error then reports it. No
 * counterpart in the reference (its device waits are not bounded). */
#define ATOM_WAIT_SELFTEST_CODE 7
int atom_wait_selftest(int64_t budget_cycles, void* stream);

/* The same for the shared-memory rings of the streamed edge kernels (atom_rotate_in and
 * atom_rotate_in_bwd_edge at C = 128): one warp runs the rings' bounded wait on a barrier whose
 * bytes never arrive, for budget_cycles SM clocks (1 .. 2e9), then records
 * ATOM_EDGE_WAIT_CODE, exactly as an expired wait inside those kernels does (which then also
 * lets its copies in flight land before returning). No counterpart in the reference. */
#define ATOM_EDGE_WAIT_CODE 8
int atom_ring_wait_selftest(int64_t budget_cycles, void* stream);

/* ------------------------------------------------------------------------------------------
 * Edge-side fused ops of the edgewise block (tt_atom/edgewise.py:39-87, forces.py:352-418).
 * ---------------------------------------------------------------------------------------- */

/* Rotate-in with the radial multiplier: for each edge e and m-primed row r,
 *   rot[e, r, 0:C]  = sum_j Wig_e[r, j] x[src[e], j, :],  rot[e, r, C:2C] = same with tgt,
 *   A[e, r, :] = rot[e, r, :] * mult_e(r)  (rad [E, ldr] compact: rows 0-2 m=0, rows 3-4 and 5-6
 *   share the m=1 slices, rows 7-8 share the m=2 slice; each 2C wide, starting at rad_col).
 * rot may be NULL (not stored). rad may be NULL (no multiplier). */
int atom_rotate_in(const float* x, const int* src, const int* tgt, const float* coef, int64_t E,
                   int C, const float* rad, int64_t ldr, int rad_col, float* rot, float* A,
                   void* stream);

/* Gate (tt_atom/activation.py:53-70): Y [E, 2H + 9H] = [gating (2H) | rows 0..8 (9H)],
 * G [E, 9H] = [silu(row 0) | row r * sigmoid(gating[d(r)]) ], d = 0,1,0,1,0,1,1,1 for r=1..8. */
int atom_gate_fwd(const float* Y, int64_t E, int H, float* G, void* stream);
/* VJP of atom_gate_fwd: gY [E, 11H] from gG [E, 9H] and Y. */
int atom_gate_bwd(const float* Y, const float* gG, int64_t E, int H, float* gY, void* stream);

/* Rotate-back + envelope + receiver reduction + residual (one node per warp, CSR order):
 *   out[n, j, c] = resid[n, j, c] + sum_{e in recv(n)} env[e] sum_r Wig_e[r, j] Y[e, r, c].
 * resid may be NULL. Y [E, 9C]. */
int atom_rotate_back_reduce(const float* Y, const float* coef, const float* env, int64_t N,
                            int C, const int* recv_ptr, const float* resid, float* out,
                            void* stream);

/* VJP of atom_rotate_back_reduce through the edge messages: with gx [N,9,C] the adjoint of out,
 *   R[e] = Wig_e gx[tgt[e]],  gY[e] = env[e] R[e]   ([E, 9C])
 *   g_env[e] += sum R[e] . Y[e];  g_coef[e, (r,j)] += env[e] sum_c gx[tgt, j, c] Y[e, r, c]. */
int atom_rotate_back_bwd(const float* gx, const int* tgt, const float* coef, const float* env,
                         const float* Y, int64_t E, int C, float* gY, float* g_env,
                         float* g_coef, void* stream);

/* VJP of atom_rotate_in, edge part: with gA [E, 9*2C]:
 *   g_rot = gA * mult (written to g_rot [E, 9*2C]),
 *   g_rad[e, slice] = sum over rows sharing the slice of gA * rot  (overwrites [E, ldr] slice),
 *   g_coef[e, (r,j)] += sum_c g_rot[e,r,c] x[src,j,c] + g_rot[e,r,C+c] x[tgt,j,c]. */
int atom_rotate_in_bwd_edge(const float* gA, const float* rot, const float* rad, int64_t ldr,
                            int rad_col, const float* x, const int* src, const int* tgt,
                            const float* coef, int64_t E, int C, float* g_rot, float* g_rad,
                            float* g_coef, void* stream);

/* VJP of atom_rotate_in, node part (fixed order; receiver CSR then sender CSR):
 *   gx[n] (+)= sum_{e in recv(n)} Wig_e^T g_rot[e, :, C:2C] + sum_{e in send(n)} Wig_e^T g_rot[e, :, 0:C]. */
int atom_rotate_in_bwd_node(const float* g_rot, const float* coef, int64_t N, int C,
                            const int* recv_ptr, const int* send_ptr, const int* send_eid,
                            int accumulate, float* gx, void* stream);

/* Edge-degree node init (tt_atom/geometry.py:262-278):
 *   x[n, j, c] = l0[n, c] [j = 0] + sum_{e in recv(n)} env[e]/rescale sum_{m<3} Wig_e[m, j] rad[e, m*C + c]. */
int atom_edge_degree_fwd(const float* rad, int64_t ldr, const float* coef, const float* env,
                         const float* l0, int64_t N, int C, const int* recv_ptr, float rescale,
                         float* x, void* stream);

/* VJP of atom_edge_degree_fwd: g_rad[e, m*C+c] = env/rescale (Wig_e gx[tgt])[m, c];
 * g_env[e] += ...; g_coef[e] += .... */
int atom_edge_degree_bwd(const float* gx, const int* tgt, const float* rad, int64_t ldr,
                         const float* coef, const float* env, int64_t E, int C, float rescale,
                         float* g_rad, int64_t ldg, float* g_env, float* g_coef, void* stream);

/* ------------------------------------------------------------------------------------------
 * Node-side ops (tt_atom/norm.py, grid.py, model.py energy head; forces.py VJPs).
 * ---------------------------------------------------------------------------------------- */

/* Row-group LayerNorm + SiLU over `groups` consecutive W-wide column groups of X [rows, ld]:
 * Y = silu(LN_g(X)); gamma/beta [groups * W]. */
int atom_ln_silu_fwd(const float* X, int64_t rows, int64_t ld, int groups, int W,
                     const float* gamma, const float* beta, float eps, float* Y, void* stream);
/* VJP of atom_ln_silu_fwd (per group, the fused_ln_bw contraction): dX from gY and X. */
int atom_ln_silu_bwd(const float* X, const float* gY, int64_t rows, int64_t ld, int groups,
                     int W, const float* gamma, const float* beta, float eps, float* dX,
                     void* stream);

/* Equivariant RMS norm (tt_atom/norm.py:24-111): out = norm(x) * affine[l] (+ bias, + add0 on
 * l = 0); add0 [N, C] may be NULL. */
int atom_rmsnorm_sh_fwd(const float* x, int64_t N, int C, const float* affine_w,
                        const float* affine_b, const float* add0, float eps, float* out,
                        void* stream);
/* VJP: gx (+)= d norm / dx applied to gout. */
int atom_rmsnorm_sh_bwd(const float* x, const float* gout, int64_t N, int C,
                        const float* affine_w, float eps, int accumulate, float* gx,
                        void* stream);

/* Per-node coefficient projection: out[n, q, c] (+)= sum_p M[q, p] in[n, p, c]
 * (M [Q, P] row-major, or transposed when trans != 0). */
int atom_node_project(const float* in, int64_t N, int P, int C, const float* M, int Q,
                      int trans, int accumulate, float* out, void* stream);

/* Spectral feed-forward gate (tt_atom/spectral.py:168-188), natural (l, m) order, lmax = 2:
 * out[n, 0] = silu(h[n, 0]), out[n, j] = h[n, j] * sigmoid(gat[n, (l(j)-1) H : l(j) H]) for
 * j >= 1; h, out [N, 9, H], gat [N, 2H] the post-SiLU scalar gating. */
int atom_spectral_gate_fwd(const float* h, const float* gat, int64_t N, int H, float* out,
                           void* stream);
/* VJP (tt_atom/forces.py:307-346): g_h [N, 9, H] and g_gat [N, 2H] from g_out [N, 9, H]. */
int atom_spectral_gate_bwd(const float* h, const float* gat, const float* g_out, int64_t N,
                           int H, float* g_h, float* g_gat, void* stream);

/* Elementwise: out = g * silu'(pre) (n values). */
int atom_silu_bwd(const float* g, const float* pre, int64_t n, float* out, void* stream);

/* Deterministic sum of n floats -> out[0] (fixed reduction tree), optionally per segment:
 * seg_ptr [nseg+1] device offsets (NULL: one segment). */
int atom_segment_sum(const float* v, int64_t n, const int* seg_ptr, int nseg, float* out,
                     void* stream);

/* Node l = 0 init: out[n, c] = sphere[Z[n], c] + sysemb[sys_id[n], c] (sys_id NULL: system 0)
 * -- the pos-independent part of tt_atom/geometry.py:262-266. Z, sys_id int32. */
int atom_node_embed(const int* Z, const int* sys_id, const float* sphere, const float* sysemb,
                    int64_t N, int C, float* out, void* stream);

/* Per-edge species: zs[e] = Z[src[e]], zt[e] = Z[tgt[e]] (row indices of the radial tables). */
int atom_edge_species(const int* Z, const int* src, const int* tgt, int64_t E, int* zs, int* zt,
                      void* stream);

/* ------------------------------------------------------------------------------------------
 * Orb-v3 (conservative) path (tt_atom/orb_model.py, orb_geometry.py, orb_forces.py). The graph
 * is the UMA-style one above; Orb's senders are tgt and its receivers src, so Orb's edge vector
 * pos[receiver] - pos[sender] + shift is the stored pos[src] - pos[tgt] + shift.
 * ---------------------------------------------------------------------------------------- */

/* Edge features (tt_atom/orb_geometry.py:65-97): feat[e, n*16 + m] = cut(r) * bessel_n(r) *
 * sh_m(v / r) for nb Bessel bases and the 16 real SH of l <= 3 (component normalisation),
 * cut [E] the p = 4 polynomial envelope (orb_model.py:69-82); ev [E,3] (may be NULL). */
int atom_orb_edge_features(const float* pos, const int* src, const int* tgt, const int* img,
                           const float* shifts, int64_t E, float rmax, int nb, float* feat,
                           float* cut, float* ev, void* stream);
/* VJP (replaces the host finish of tt_atom/orb_geometry.py:100-139): g_ev [E,3] from
 * g_feat [E, 16 nb] and g_cut [E]. */
int atom_orb_edge_features_bwd(const float* pos, const int* src, const int* tgt, const int* img,
                               const float* shifts, int64_t E, float rmax, int nb,
                               const float* g_feat, const float* g_cut, float* g_ev,
                               void* stream);
/* Row RMSNorm (orb_model.py:92-112): Y = X rsqrt(mean(X^2) + eps) w (Y may be NULL); with
 * R_out: R_out = R_in + Y (the residual update). */
int atom_rmsnorm_rows(const float* X, int64_t ldx, int64_t rows, int W, const float* w,
                      float eps, float* Y, int64_t ldy, const float* R_in, int64_t ldr_in,
                      float* R_out, int64_t ldr_out, void* stream);
/* VJP of atom_rmsnorm_rows (orb_forces.py:67-79), X and gY dense [rows, W]; dX may alias gY. */
int atom_rmsnorm_rows_bwd(const float* X, const float* gY, int64_t rows, int W, const float* w,
                          float eps, float* dX, void* stream);
/* Attention gates (orb_model.py:245-250): lin[e] = (edges[e].wr + br, edges[e].ws + bs),
 * att[e] = sigmoid(lin[e]) * cut[e] ([E,2]: receive, send). */
int atom_orb_attention(const float* edges, int64_t E, int C, const float* wr, float br,
                       const float* ws, float bs, const float* cut, float* lin, float* att,
                       void* stream);
/* CSR segment sum: out[n] (+)= sum_{k in ptr[n]..ptr[n+1]} scale[e * sstride] X[e],
 * e = eid ? eid[k] : k (scale may be NULL). W, ldx, ldo multiples of 4. */
int atom_csr_sum(const float* X, int64_t ldx, const float* scale, int sstride, const int* ptr,
                 const int* eid, int64_t N, int W, float* out, int64_t ldo, int accumulate,
                 void* stream);
/* VJP of the two attention-weighted aggregations and the gates (orb_forces.py:94-148):
 * g_agg [N, 2C] = adjoint of [receiver aggregate | sender aggregate]; writes
 * g_ue = gE_in + att_s g_agg[tgt, C:] + att_r g_agg[src, :C], gE_out = gE_in + gate adjoints
 * (may alias gE_in), g_cut += cutoff adjoint. */
int atom_orb_messages_bwd(const float* g_agg, const float* gE_in, const float* ue,
                          const float* lin, const float* att, const float* cut, const int* src,
                          const int* tgt, int64_t E, int C, const float* wr, const float* ws,
                          float* g_ue, float* gE_out, float* g_cut, void* stream);
/* out[c] = scale * sum_n X[n, c] (fixed order; the energy head's node mean). */
int atom_col_mean(const float* X, int64_t ld, int64_t N, int C, float scale, float* out,
                  void* stream);
/* out[n, c] (+)= scale * v[c]. */
int atom_row_broadcast(const float* v, int64_t N, int C, float scale, float* out, int64_t ld,
                       int accumulate, void* stream);

/* ZBL pair repulsion of Orb (replaces the host closed form of tt_atom/orb_model.py:491-587:
 * host_zbl_energy / host_zbl_forces / host_zbl_stress), fp64 per edge. ev [E,3] edge vectors
 * (pos[src] - pos[tgt] + shift), Z [N] atomic numbers, src / tgt [E] (Orb senders = tgt),
 * rcov [nrad] covalent radii (A) indexed by Z + 1, scale = 1 / N (per-node mean) or 1 (sum).
 * Writes g_ev [E,3] = dE_zbl/d(ev) (feed atom_forces_virial for forces and virial),
 * partials [1024] (scratch) and energy [1] = scale * sum of pair terms. */
int atom_orb_zbl(const float* ev, const int* Z, const int* src, const int* tgt, int64_t E,
                 const double* rcov, int nrad, double scale, float* g_ev, double* partials,
                 double* energy, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ATOM_B200_H */
