// Shared helpers of the sm_100a kernels: status codes, the thread-local error message, launch
// checks and warp-level utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <stdio.h>
#include <string.h>

#include "../../include/atom_b200.h"

namespace atom {

// Thread-local last error message read back through atom_last_error().
void set_error(const char* fmt, ...);
// Device address of the library's error word (0 = no error; a kernel whose bounded wait ran out
// stores its code there with atomicCAS, and atom_device_error_take reads and clears it).
int* device_error_word();

// Kernels this library has launched (read through atom_launch_count): every launch site is
// followed by exactly one check_launch, told how many launches it covers.
inline std::atomic<long long> g_launches{0};

inline int check_launch(const char* what, int launches = 1) {
    g_launches.fetch_add(launches, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: CUDA launch error %s", what, cudaGetErrorString(e));
        return ATOM_ERR_CUDA;
    }
    return ATOM_OK;
}

#define ATOM_REQUIRE(cond, ...)            \
    do {                                   \
        if (!(cond)) {                     \
            ::atom::set_error(__VA_ARGS__);  \
            return ATOM_ERR_ARG;           \
        }                                  \
    } while (0)

#define ATOM_CHECK_LAUNCH(name)                   \
    do {                                          \
        int _s = ::atom::check_launch(name);      \
        if (_s != ATOM_OK) return _s;             \
    } while (0)
#define ATOM_CHECK_LAUNCHES(name, n)              \
    do {                                          \
        int _s = ::atom::check_launch(name, n);   \
        if (_s != ATOM_OK) return _s;             \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
// The gate's forward activations, from the fast exponential and the fast division intrinsics
// (a few ulp; used wherever the gated so2_2 operand is formed, so that the standalone gate
// kernel and the gate fused into the GEMM give the same bits).
__device__ __forceinline__ float sigmoid_gate(float x) {
    return __fdividef(1.0f, 1.0f + __expf(-x));
}
__device__ __forceinline__ float silu_gate(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
// Its derivative from the same sigmoid (radial LayerNorm + SiLU and the SiLU VJPs).
__device__ __forceinline__ float dsilu_gate(float x) {
    const float s = sigmoid_gate(x);
    return s * (1.0f + x * (1.0f - s));
}
// d/dx silu(x) = s (1 + x (1 - s)), s = sigmoid(x)
__device__ __forceinline__ float dsilu_f(float x) {
    float s = sigmoid_f(x);
    return s * (1.0f + x * (1.0f - s));
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// ------------------------------------------------------------------- lmax = 2 structure
// Node features are [N, 9, C] in the standard (l, m) coefficient order. The per-edge Wigner
// matrix in m-primed row order (rows permuted by to_m) has for row r the nonzero columns of the
// degree-l(r) block [l^2, (l+1)^2). The 35 nonzeros are packed row-major: row r starts at
// kRowOff[r] and has 2 l(r) + 1 entries.
//   m-primed rows: 0 l0m0 | 1 l1m0 | 2 l2m0 | 3 l1m1(re) | 4 l2m1(re) | 5 l1m1(im) | 6 l2m1(im)
//                  | 7 l2m2(re) | 8 l2m2(im)
constexpr int kNsph = 9;
constexpr int kNnz = 35;
__host__ __device__ constexpr int row_deg(int r) {
    return r == 0 ? 0 : ((r == 1 || r == 3 || r == 5) ? 1 : 2);
}
__host__ __device__ constexpr int row_off(int r) {
    // cumulative sizes [1,3,5,3,5,3,5,5,5]
    return r == 0 ? 0 : r == 1 ? 1 : r == 2 ? 4 : r == 3 ? 9 : r == 4 ? 12 : r == 5 ? 17
         : r == 6 ? 20 : r == 7 ? 25 : 30;
}
__host__ __device__ constexpr int deg_col0(int l) { return l * l; }
// Gating row (0 or 1) of vector row r = 1..8 in m-primed order (tt_atom/activation.py:19-26).
__host__ __device__ constexpr int gate_row(int r) {
    return (r == 1 || r == 3 || r == 5) ? 0 : 1;
}

}  // namespace atom
