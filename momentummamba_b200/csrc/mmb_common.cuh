// Shared device helpers for the sm_100a scan kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/momentum_scan_b200.h"

#define MMB_LOG2E 1.4426950408889634f
#define MMB_LN2 0.6931471805599453f

namespace mmb {

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// ---------------------------------------------------------------------------
// cp.async staging (global -> shared), with zero fill for out-of-range data.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(sdst)),
                 "l"(gsrc), "r"(n)
                 : "memory");
}

__device__ __forceinline__ void cp_async4(void* sdst, const void* gsrc, bool valid) {
    const int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(sdst)),
                 "l"(gsrc), "r"(n)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Stage a ROWS x COLS fp32 tile whose rows are `gstride` floats apart in global
// memory into shared memory with row pitch SPITCH floats.  Rows >= rvalid and
// columns >= cvalid are zero-filled.  `vec` selects 16-byte copies (caller
// guarantees 16-byte aligned rows and cvalid % 4 == 0 in that case).
template <int ROWS, int COLS, int SPITCH, int NTHREADS>
__device__ __forceinline__ void stage_tile(float* s, const float* g, int64_t gstride, int rvalid,
                                           int cvalid, bool vec, int tid) {
    if (vec) {
        constexpr int C4 = COLS / 4;
        constexpr int TOTAL = ROWS * C4;
#pragma unroll
        for (int i = tid; i < TOTAL; i += NTHREADS) {
            const int r = i / C4, c = (i % C4) * 4;
            const bool ok = (r < rvalid) && (c < cvalid);
            const float* src = ok ? g + (int64_t)r * gstride + c : g;
            cp_async16(s + r * SPITCH + c, src, ok);
        }
    } else {
        constexpr int TOTAL = ROWS * COLS;
#pragma unroll 4
        for (int i = tid; i < TOTAL; i += NTHREADS) {
            const int r = i / COLS, c = i % COLS;
            const bool ok = (r < rvalid) && (c < cvalid);
            const float* src = ok ? g + (int64_t)r * gstride + c : g;
            cp_async4(s + r * SPITCH + c, src, ok);
        }
    }
}

// ---------------------------------------------------------------------------
// math
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// torch.nn.functional.softplus with beta = 1, threshold = 20.
__device__ __forceinline__ float softplus_f(float r) { return r > 20.f ? r : log1pf(expf(r)); }

__device__ __forceinline__ float sigmoid_f(float r) { return 1.f / (1.f + expf(-r)); }

// ---------------------------------------------------------------------------
// warp reductions
// ---------------------------------------------------------------------------
// Sum `v` over the lanes that differ only in the bits of MASK_BITS (a
// contiguous range of lane bits [LO, LO+NB)).
template <int LO, int NB>
__device__ __forceinline__ float lane_sum(float v) {
#pragma unroll
    for (int b = 0; b < NB; ++b) v += __shfl_xor_sync(0xffffffffu, v, 1 << (LO + b));
    return v;
}

// Reduce-scatter of V values across the 2^NB lanes that differ in lane bits
// [LO, LO+NB).  On return the first max(V >> NB, 1) entries of `a` hold sums over
// all 2^NB lanes; entry i of this lane is original index
// rs_index<V, NB>(lane_bits, i).
template <int V, int LO, int NB>
__device__ __forceinline__ void reduce_scatter(float (&a)[V], int lane) {
    int cur = V;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const int mask = 1 << (LO + b);
        const bool hi = (lane & mask) != 0;
        if (cur > 1) {
            const int half = cur / 2;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < half) {
                    const float send = hi ? a[i] : a[i + half];
                    const float keep = hi ? a[i + half] : a[i];
                    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
                }
            }
            cur = half;
        } else {
            a[0] += __shfl_xor_sync(0xffffffffu, a[0], mask);
        }
    }
}

// Original index of entry i after reduce_scatter<V, LO, NB> on a lane whose
// bits [LO, LO+NB) equal `bits`.
template <int V, int NB>
__device__ __forceinline__ int rs_index(int bits, int i) {
    int base = 0, cur = V;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (cur > 1) {
            cur /= 2;
            if ((bits >> b) & 1) base += cur;
        }
    }
    return base + i;
}

// Vector reduction-add of 4 consecutive floats in global memory (sm_90+).
__device__ __forceinline__ void red_add_v4(float* gaddr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(gaddr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

}  // namespace mmb

// Host-side launch-status helper shared by the C-ABI wrappers.
static inline int mmb_launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MMB_OK : MMB_ERR_LAUNCH;
}

// Raise a kernel's dynamic shared-memory limit once per device (the attribute
// is per device; `done` has one slot per device ordinal).
#define MMB_MAX_DEVICES 64
template <typename Kernel>
static inline int mmb_smem_attr(Kernel kernel, size_t bytes, int* done) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MMB_MAX_DEVICES)
        return MMB_ERR_LAUNCH;
    if (!done[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)bytes) != cudaSuccess)
            return MMB_ERR_LAUNCH;
        done[dev] = 1;
    }
    return MMB_OK;
}
