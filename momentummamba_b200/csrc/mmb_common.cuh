// Shared device helpers for the sm_100a scan kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
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

__device__ __forceinline__ void cp_async8(void* sdst, const void* gsrc, bool valid) {
    const int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(smem_u32(sdst)),
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

// 16-bit elements (bf16 activations): stage a ROWS x COLS tile of 2-byte values
// with 16-byte copies; the caller guarantees COLS % 8 == 0, 16-byte aligned
// rows and cvalid % 8 == 0.  Out-of-range rows and columns are zero-filled.
template <int ROWS, int COLS, int SPITCH, int NTHREADS>
__device__ __forceinline__ void stage_tile_b16(uint16_t* s, const uint16_t* g, int64_t gstride,
                                               int rvalid, int cvalid, int tid) {
    constexpr int C8 = COLS / 8;
    constexpr int TOTAL = ROWS * C8;
#pragma unroll
    for (int i = tid; i < TOTAL; i += NTHREADS) {
        const int r = i / C8, c = (i % C8) * 8;
        const bool ok = (r < rvalid) && (c < cvalid);
        const uint16_t* src = ok ? g + (int64_t)r * gstride + c : g;
        cp_async16(s + r * SPITCH + c, src, ok);
    }
}

// bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Widen a staged ROWS x COLS bf16 tile (pitch SPIN) into an fp32 tile (pitch
// SPOUT, a multiple of 4).
template <int ROWS, int COLS, int SPIN, int SPOUT, int NTHREADS>
__device__ __forceinline__ void widen_tile(float* dst, const uint16_t* src, int tid) {
    constexpr int C8 = COLS / 8;
    constexpr int TOTAL = ROWS * C8;
#pragma unroll
    for (int i = tid; i < TOTAL; i += NTHREADS) {
        const int r = i / C8, c = (i % C8) * 8;
        const uint4 q = *reinterpret_cast<const uint4*>(src + r * SPIN + c);
        float4* o = reinterpret_cast<float4*>(dst + r * SPOUT + c);
        o[0] = make_float4(bf16_lo(q.x), bf16_hi(q.x), bf16_lo(q.y), bf16_hi(q.y));
        o[1] = make_float4(bf16_lo(q.z), bf16_hi(q.z), bf16_lo(q.w), bf16_hi(q.w));
    }
}

// fp32 -> bf16, round to nearest even (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// Element types of the activations: fp32 or bf16 (stored as raw 16-bit words).
struct ElemF32 {
    using T = float;
    static constexpr int BYTES = 4;
    __device__ static float load(const T* p, int64_t i) { return p[i]; }
    __device__ static void store(T* p, int64_t i, float v) { p[i] = v; }
};
struct ElemBF16 {
    using T = uint16_t;
    static constexpr int BYTES = 2;
    __device__ static float load(const T* p, int64_t i) { return bf16_lo(p[i]); }
    __device__ static void store(T* p, int64_t i, float v) { p[i] = f32_to_bf16(v); }
};

// ---------------------------------------------------------------------------
// TMA tile loads and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// make the barrier inits visible to the async (TMA) proxy
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n\tfence.proxy.async.shared::cta;" ::
                     : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of the barrier, giving up after `polls` polls (each
// poll itself suspends for a hardware-chosen while): false then.
__device__ __forceinline__ bool mbar_wait_polls(uint64_t* bar, uint32_t parity, int polls) {
    for (int i = 0; i < polls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// The tile pipelines' wait: at most 2^22 polls.
constexpr int MMB_WAIT_POLLS = 1 << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    return mbar_wait_polls(bar, parity, MMB_WAIT_POLLS);
}

// 3-D tiled TMA load of the box at (c0, c1, c2) into shared memory, completing
// on `bar` (no multicast).
__device__ __forceinline__ void tma_load_3d(void* sdst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(sdst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// math
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// torch.nn.functional.softplus (beta = 1): log(1 + e^r) = max(r, 0) + log1p(w),
// w = e^{-|r|} in (0, 1].  log1p(w) = 2 atanh(s) with s = w / (2 + w) in
// (0, 1/3]; the atanh series s + s^3/3 + ... + s^13/13 has a truncation error
// below 2e-8 relative there.  Inputs above 20 come out as r to fp32 precision,
// matching torch's threshold branch.  `wout` returns w for the derivative.
__device__ __forceinline__ float softplus_w(float r, float& wout) {
    const float w = ex2(-fabsf(r) * MMB_LOG2E);
    const float s = w * rcp_approx(2.f + w);
    const float s2 = s * s;
    float q = 1.f / 13.f;
    q = fmaf(q, s2, 1.f / 11.f);
    q = fmaf(q, s2, 1.f / 9.f);
    q = fmaf(q, s2, 1.f / 7.f);
    q = fmaf(q, s2, 1.f / 5.f);
    q = fmaf(q, s2, 1.f / 3.f);
    q = fmaf(q, s2, 1.f);
    wout = w;
    return fmaxf(r, 0.f) + 2.f * s * q;
}

__device__ __forceinline__ float softplus_f(float r) {
    float w;
    return softplus_w(r, w);
}

// d softplus / dr = sigmoid(r), from w = e^{-|r|}.
__device__ __forceinline__ float softplus_grad(float r) {
    const float w = ex2(-fabsf(r) * MMB_LOG2E);
    const float inv = rcp_approx(1.f + w);
    return r >= 0.f ? inv : w * inv;
}

// the same from w = e^{-|r|} as softplus_w returned it
__device__ __forceinline__ float softplus_grad_w(float r, float w) {
    const float inv = rcp_approx(1.f + w);
    return r >= 0.f ? inv : w * inv;
}

__device__ __forceinline__ float sigmoid_f(float r) {
    return rcp_approx(1.f + ex2(-r * MMB_LOG2E));
}

// ---------------------------------------------------------------------------
// packed fp32 pairs (sm_100 f32x2 pipes)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

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

// ---------------------------------------------------------------------------
// Affine maps x -> M x + w on complex 2-vectors (x1, x2), M a real 2x2 matrix
// type with members a, b, c, d ([[a, b], [c, d]]), and their composition
// across a warp's lanes: the chunk carries of the 2x2 scans, one chunk per lane.
// ---------------------------------------------------------------------------
template <class Mt>
struct Aff2 {
    Mt m;
    float x1r, x1i, x2r, x2i;
};
template <class Mt>
__device__ __forceinline__ Mt mat2_mul(const Mt& x, const Mt& y) {
    return {x.a * y.a + x.b * y.c, x.a * y.b + x.b * y.d, x.c * y.a + x.d * y.c,
            x.c * y.b + x.d * y.d};
}
// the map `later` after the map `earlier`
template <class Mt>
__device__ __forceinline__ Aff2<Mt> aff2_then(const Aff2<Mt>& later, const Aff2<Mt>& earlier) {
    const Mt& m = later.m;
    return {mat2_mul(m, earlier.m),
            m.a * earlier.x1r + m.b * earlier.x2r + later.x1r,
            m.a * earlier.x1i + m.b * earlier.x2i + later.x1i,
            m.c * earlier.x1r + m.d * earlier.x2r + later.x2r,
            m.c * earlier.x1i + m.d * earlier.x2i + later.x2i};
}
template <class Mt>
__device__ __forceinline__ Aff2<Mt> aff2_shfl_up(const Aff2<Mt>& v, int d) {
    const unsigned F = 0xffffffffu;
    return {{__shfl_up_sync(F, v.m.a, d), __shfl_up_sync(F, v.m.b, d),
             __shfl_up_sync(F, v.m.c, d), __shfl_up_sync(F, v.m.d, d)},
            __shfl_up_sync(F, v.x1r, d), __shfl_up_sync(F, v.x1i, d),
            __shfl_up_sync(F, v.x2r, d), __shfl_up_sync(F, v.x2i, d)};
}
template <class Mt>
__device__ __forceinline__ Aff2<Mt> aff2_shfl(const Aff2<Mt>& v, int src) {
    const unsigned F = 0xffffffffu;
    return {{__shfl_sync(F, v.m.a, src), __shfl_sync(F, v.m.b, src),
             __shfl_sync(F, v.m.c, src), __shfl_sync(F, v.m.d, src)},
            __shfl_sync(F, v.x1r, src), __shfl_sync(F, v.x1i, src),
            __shfl_sync(F, v.x2r, src), __shfl_sync(F, v.x2i, src)};
}
// Exclusive scan of the lanes' maps applied after `in` (a map: the product of
// the earlier chunks' matrices and the state they leave): lane l receives
// map_{l-1} o ... o map_0 o in; every lane gets map_31 o ... o map_0 o in back.
template <class Mt>
__device__ __forceinline__ Aff2<Mt> warp_aff2_exscan(Aff2<Mt> v, const Aff2<Mt>& in, int lane,
                                                     Aff2<Mt>& ex) {
#pragma unroll
    for (int k = 0; k < 5; ++k) {  // Hillis-Steele: v <- maps of lanes (l - 2^(k+1), l]
        const Aff2<Mt> o = aff2_shfl_up(v, 1 << k);
        if (lane >= (1 << k)) v = aff2_then(v, o);
    }
    const Aff2<Mt> prev = aff2_shfl_up(v, 1);  // maps of lanes 0 .. l-1
    ex = lane ? aff2_then(prev, in) : in;
    return aff2_then(aff2_shfl(v, 31), in);
}

// Vector reduction-add of 4 consecutive floats in global memory (sm_90+).
__device__ __forceinline__ void red_add_v4(float* gaddr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(gaddr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

}  // namespace mmb

// Last CUDA error seen by this library on the calling thread (see mmb_last_error).
void mmb_record_cuda_error(cudaError_t e);

// Device address of the error flag that bounded device waits set (current device).
int* mmb_device_error_flag();

// Encode a 3-D tiled tensor map over dims (dim0 innermost, unit stride; dim1 and
// dim2 with element strides stride1, stride2) for boxes of box0 x box1 x 1
// elements of elem_bytes (4: fp32, 2: bf16), swizzle span 0/32/64/128 bytes
// (16-byte chunks permuted within the span), or MMB_SWZ_128B_ATOM32 (32-byte
// chunks permuted within 128 bytes), out-of-range elements read as zero.
// false if the driver refuses.
constexpr int MMB_SWZ_128B_ATOM32 = 1128;
bool mmb_encode_tile_map(CUtensorMap* map, const void* base, int elem_bytes, int64_t dim0,
                         int64_t dim1, int64_t dim2, int64_t stride1, int64_t stride2,
                         int box0, int box1, int swizzle_bytes);

// NVTX range around one C-ABI call (named after the entry point), so that a
// profiler's timeline shows which library call launched which kernels.  NVTX3
// is header-only; without a tool attached a range costs a few nanoseconds.
struct MMBNvtxRange {
    explicit MMBNvtxRange(const char* name) { nvtxRangePushA(name); }
    ~MMBNvtxRange() { nvtxRangePop(); }
    MMBNvtxRange(const MMBNvtxRange&) = delete;
    MMBNvtxRange& operator=(const MMBNvtxRange&) = delete;
};
#define MMB_NVTX(name) MMBNvtxRange mmb_nvtx_range_(name)

// Host-side launch-status helper shared by the C-ABI wrappers.
static inline int mmb_launch_status() {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return MMB_OK;
    mmb_record_cuda_error(e);
    return MMB_ERR_LAUNCH;
}

// Raise a kernel's dynamic shared-memory limit once per device (the attribute
// is per device; `done` has one slot per device ordinal).
#define MMB_MAX_DEVICES 64
template <typename Kernel>
static inline int mmb_smem_attr(Kernel kernel, size_t bytes, int* done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= MMB_MAX_DEVICES) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    if (!done[dev]) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) {
            mmb_record_cuda_error(e);
            return MMB_ERR_LAUNCH;
        }
        done[dev] = 1;
    }
    return MMB_OK;
}
