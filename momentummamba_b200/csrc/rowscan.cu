// Diagonal scans on materialised (deltaA, u) tensors, sm_100a.
//
// Row layout (R, L), time unit-stride -- momentum_scan_cuda / warp_momentum_scan_cuda:
//   one CTA streams 128 rows through shared memory in 32-step chunks
//   (double-buffered cp.async, 16-byte copies along t), one thread per row runs
//   the recurrence reading 4 steps at a time as float4 from a padded tile
//   (pitch 36 floats: conflict-free quarter-warp phases), and the output tile
//   goes back to global memory with coalesced 16-byte stores.
//
// PScan layout (B, L, M), M unit-stride:
//   one thread per (b, m) column; a warp's loads of one time step are 128
//   contiguous bytes, so the kernel needs no staging: it keeps eight steps of
//   loads in flight per thread.
#include "mmb_common.cuh"

namespace mmb {

constexpr int RS_NT = 128;   // rows per CTA (one per thread)
constexpr int RS_T = 32;     // steps per chunk
constexpr int RS_P = 36;     // smem pitch (floats)
constexpr int RS_TILE = RS_NT * RS_P;

// Stage rows [r0, r0+128) x steps [t0, t0+32) of a (R, L) row-major tensor.
__device__ __forceinline__ void rs_stage(float* s, const float* g, int64_t R, int64_t L,
                                         int64_t r0, int64_t t0, bool vec, int tid) {
    const int rv = (int)min64(RS_NT, R - r0);
    const int cv = (int)min64(RS_T, L - t0);
    stage_tile<RS_NT, RS_T, RS_P, RS_NT>(s, g + r0 * L + t0, L, rv, cv, vec, tid);
}

// Copy a (128 x 32) output tile back to global memory.
__device__ __forceinline__ void rs_store(const float* s, float* g, int64_t R, int64_t L,
                                         int64_t r0, int64_t t0, bool vec, int tid) {
    const int rv = (int)min64(RS_NT, R - r0);
    const int cv = (int)min64(RS_T, L - t0);
    if (vec) {
        for (int i = tid; i < RS_NT * (RS_T / 4); i += RS_NT) {
            const int r = i / (RS_T / 4), c = (i % (RS_T / 4)) * 4;
            if (r < rv && c < cv)
                *reinterpret_cast<float4*>(g + (r0 + r) * L + t0 + c) =
                    *reinterpret_cast<const float4*>(s + r * RS_P + c);
        }
    } else {
        for (int i = tid; i < RS_NT * RS_T; i += RS_NT) {
            const int r = i / RS_T, c = i % RS_T;
            if (r < rv && c < cv) g[(r0 + r) * L + t0 + c] = s[r * RS_P + c];
        }
    }
}

__global__ void __launch_bounds__(RS_NT)
rows_fwd_kernel(int64_t R, int64_t L, const float* __restrict__ a, float beta,
                const float* __restrict__ u, float* __restrict__ h, float* __restrict__ vout,
                int vec) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    float* sh = smem + 4 * RS_TILE;
    float* sv = sh + RS_TILE;
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.x * RS_NT;
    const int nchunks = (int)((L + RS_T - 1) / RS_T);
    float hh = 0.f, vv = 0.f;

    rs_stage(smem, a, R, L, r0, 0, vec, tid);
    rs_stage(smem + RS_TILE, u, R, L, r0, 0, vec, tid);
    cp_async_commit();
    for (int c = 0; c < nchunks; ++c) {
        const int64_t t0 = (int64_t)c * RS_T;
        if (c + 1 < nchunks) {
            float* nx = smem + ((c + 1) & 1) * 2 * RS_TILE;
            rs_stage(nx, a, R, L, r0, t0 + RS_T, vec, tid);
            rs_stage(nx + RS_TILE, u, R, L, r0, t0 + RS_T, vec, tid);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* sa = smem + (c & 1) * 2 * RS_TILE;
        const float* su = sa + RS_TILE;
        // steps past L see a = u = 0 and are never stored
#pragma unroll
        for (int q = 0; q < RS_T / 4; ++q) {
            const float4 a4 = *reinterpret_cast<const float4*>(sa + tid * RS_P + 4 * q);
            const float4 u4 = *reinterpret_cast<const float4*>(su + tid * RS_P + 4 * q);
            float4 o, ov;
            vv = fmaf(beta, vv, u4.x); hh = fmaf(a4.x, hh, vv); o.x = hh; ov.x = vv;
            vv = fmaf(beta, vv, u4.y); hh = fmaf(a4.y, hh, vv); o.y = hh; ov.y = vv;
            vv = fmaf(beta, vv, u4.z); hh = fmaf(a4.z, hh, vv); o.z = hh; ov.z = vv;
            vv = fmaf(beta, vv, u4.w); hh = fmaf(a4.w, hh, vv); o.w = hh; ov.w = vv;
            *reinterpret_cast<float4*>(sh + tid * RS_P + 4 * q) = o;
            if (vout) *reinterpret_cast<float4*>(sv + tid * RS_P + 4 * q) = ov;
        }
        __syncthreads();
        rs_store(sh, h, R, L, r0, t0, vec, tid);
        if (vout) rs_store(sv, vout, R, L, r0, t0, vec, tid);
        __syncthreads();
    }
}

__global__ void __launch_bounds__(RS_NT)
rows_bwd_kernel(int64_t R, int64_t L, const float* __restrict__ g, const float* __restrict__ a,
                float beta, const float* __restrict__ h, float* __restrict__ da,
                float* __restrict__ du, int vec) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    // stage s: [g | a | h] tiles, plus a column with h_{t0-1} per row
    constexpr int STAGE = 3 * RS_TILE + RS_NT;
    float* sda = smem + 2 * STAGE;
    float* sdu = sda + RS_TILE;
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.x * RS_NT;
    const int64_t row = r0 + tid;
    const int nchunks = (int)((L + RS_T - 1) / RS_T);
    float gh = 0.f, gv = 0.f, anext = 0.f;

    auto stage = [&](int s, int c) {
        float* st = smem + s * STAGE;
        const int64_t t0 = (int64_t)c * RS_T;
        rs_stage(st, g, R, L, r0, t0, vec, tid);
        rs_stage(st + RS_TILE, a, R, L, r0, t0, vec, tid);
        rs_stage(st + 2 * RS_TILE, h, R, L, r0, t0, vec, tid);
        const bool ok = row < R && t0 > 0;
        cp_async4(st + 3 * RS_TILE + tid, ok ? h + row * L + t0 - 1 : h, ok);
    };

    stage(0, nchunks - 1);
    cp_async_commit();
    for (int it = 0; it < nchunks; ++it) {
        const int c = nchunks - 1 - it;
        const int64_t t0 = (int64_t)c * RS_T;
        if (c > 0) stage((it + 1) & 1, c - 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* st = smem + (it & 1) * STAGE;
        const float* sg = st;
        const float* sa = st + RS_TILE;
        const float* shh = st + 2 * RS_TILE;
        const float hprev0 = st[3 * RS_TILE + tid];
        // steps past L carry g = 0 so the adjoint stays zero there
#pragma unroll
        for (int q = RS_T / 4 - 1; q >= 0; --q) {
            const float4 g4 = *reinterpret_cast<const float4*>(sg + tid * RS_P + 4 * q);
            const float4 a4 = *reinterpret_cast<const float4*>(sa + tid * RS_P + 4 * q);
            const float4 h4 = *reinterpret_cast<const float4*>(shh + tid * RS_P + 4 * q);
            const float hp = q > 0 ? shh[tid * RS_P + 4 * q - 1] : hprev0;
            float4 oa, ou;
            gh = fmaf(anext, gh, g4.w); gv = fmaf(beta, gv, gh); ou.w = gv; oa.w = gh * h4.z; anext = a4.w;
            gh = fmaf(anext, gh, g4.z); gv = fmaf(beta, gv, gh); ou.z = gv; oa.z = gh * h4.y; anext = a4.z;
            gh = fmaf(anext, gh, g4.y); gv = fmaf(beta, gv, gh); ou.y = gv; oa.y = gh * h4.x; anext = a4.y;
            gh = fmaf(anext, gh, g4.x); gv = fmaf(beta, gv, gh); ou.x = gv; oa.x = gh * hp;   anext = a4.x;
            *reinterpret_cast<float4*>(sda + tid * RS_P + 4 * q) = oa;
            *reinterpret_cast<float4*>(sdu + tid * RS_P + 4 * q) = ou;
        }
        // da at t = 0 is zero by definition (no previous state)
        if (c == 0) sda[tid * RS_P] = 0.f;
        __syncthreads();
        if (da) rs_store(sda, da, R, L, r0, t0, vec, tid);
        if (du) rs_store(sdu, du, R, L, r0, t0, vec, tid);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// PScan layout (B, L, M)
// ---------------------------------------------------------------------------
constexpr int PS_NT = 256;
constexpr int PS_U = 8;  // steps of loads in flight

__global__ void __launch_bounds__(PS_NT)
pscan_fwd_kernel(int64_t Bsz, int64_t L, int64_t M, const float* __restrict__ A,
                 const float* __restrict__ X, float* __restrict__ H) {
    const int64_t col = (int64_t)blockIdx.x * PS_NT + threadIdx.x;
    if (col >= Bsz * M) return;
    const int64_t b = col / M, m = col % M;
    const int64_t base = b * L * M + m;
    float hv = 0.f;
    int64_t t = 0;
    for (; t + PS_U <= L; t += PS_U) {
        float av[PS_U], xv[PS_U];
#pragma unroll
        for (int k = 0; k < PS_U; ++k) {
            av[k] = __ldg(A + base + (t + k) * M);
            xv[k] = __ldg(X + base + (t + k) * M);
        }
#pragma unroll
        for (int k = 0; k < PS_U; ++k) {
            hv = fmaf(av[k], hv, xv[k]);
            H[base + (t + k) * M] = hv;
        }
    }
    for (; t < L; ++t) {
        hv = fmaf(A[base + t * M], hv, X[base + t * M]);
        H[base + t * M] = hv;
    }
}

__global__ void __launch_bounds__(PS_NT)
pscan_bwd_kernel(int64_t Bsz, int64_t L, int64_t M, const float* __restrict__ A,
                 const float* __restrict__ H, const float* __restrict__ G, float* __restrict__ dA,
                 float* __restrict__ dX) {
    const int64_t col = (int64_t)blockIdx.x * PS_NT + threadIdx.x;
    if (col >= Bsz * M) return;
    const int64_t b = col / M, m = col % M;
    const int64_t base = b * L * M + m;
    float gx = 0.f, anext = 0.f;
    int64_t t = L - 1;
    for (; t + 1 >= PS_U; t -= PS_U) {
        float gv[PS_U], av[PS_U], hp[PS_U];
#pragma unroll
        for (int k = 0; k < PS_U; ++k) {
            const int64_t tt = t - k;
            gv[k] = __ldg(G + base + tt * M);
            av[k] = __ldg(A + base + tt * M);
            hp[k] = tt > 0 ? __ldg(H + base + (tt - 1) * M) : 0.f;
        }
#pragma unroll
        for (int k = 0; k < PS_U; ++k) {
            const int64_t tt = t - k;
            gx = fmaf(anext, gx, gv[k]);
            if (dX) dX[base + tt * M] = gx;
            if (dA) dA[base + tt * M] = gx * hp[k];
            anext = av[k];
        }
    }
    for (; t >= 0; --t) {
        gx = fmaf(anext, gx, G[base + t * M]);
        if (dX) dX[base + t * M] = gx;
        if (dA) dA[base + t * M] = t > 0 ? gx * H[base + (t - 1) * M] : 0.f;
        anext = A[base + t * M];
    }
}

static bool al16(const void* p) { return p == nullptr || ((uintptr_t)p & 15) == 0; }

}  // namespace mmb

using namespace mmb;

extern "C" int mmb_rows_fwd(int64_t rows, int64_t L, const float* a, float beta, const float* u,
                            float* h, float* v_out, mmb_stream_t stream) {
    MMB_NVTX("mmb_rows_fwd");
    if (!a || !u || !h) return MMB_ERR_NULL;
    if (rows <= 0 || L <= 0) return MMB_ERR_SHAPE;
    const int vec = (L % 4 == 0) && al16(a) && al16(u) && al16(h) && al16(v_out);
    const size_t smem = sizeof(float) * 6 * RS_TILE;
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(rows_fwd_kernel, smem, attr_done);
    if (st != MMB_OK) return st;
    const int64_t nblk = (rows + RS_NT - 1) / RS_NT;
    if (nblk > 0x7fffffff) return MMB_ERR_SHAPE;
    rows_fwd_kernel<<<(unsigned)nblk, RS_NT, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
        rows, L, a, beta, u, h, v_out, vec);
    return mmb_launch_status();
}

extern "C" int mmb_rows_bwd(int64_t rows, int64_t L, const float* g, const float* a, float beta,
                            const float* h, float* da, float* du, mmb_stream_t stream) {
    MMB_NVTX("mmb_rows_bwd");
    if (!g || !a || !h) return MMB_ERR_NULL;
    if (rows <= 0 || L <= 0) return MMB_ERR_SHAPE;
    if (!da && !du) return MMB_OK;
    const int vec = (L % 4 == 0) && al16(g) && al16(a) && al16(h) && al16(da) && al16(du);
    const size_t smem = sizeof(float) * (2 * (3 * RS_TILE + RS_NT) + 2 * RS_TILE);
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(rows_bwd_kernel, smem, attr_done);
    if (st != MMB_OK) return st;
    const int64_t nblk = (rows + RS_NT - 1) / RS_NT;
    if (nblk > 0x7fffffff) return MMB_ERR_SHAPE;
    rows_bwd_kernel<<<(unsigned)nblk, RS_NT, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
        rows, L, g, a, beta, h, da, du, vec);
    return mmb_launch_status();
}

extern "C" int mmb_pscan_fwd(int64_t batch, int64_t L, int64_t M, const float* A, const float* X,
                             float* H, mmb_stream_t stream) {
    MMB_NVTX("mmb_pscan_fwd");
    if (!A || !X || !H) return MMB_ERR_NULL;
    if (batch <= 0 || L <= 0 || M <= 0) return MMB_ERR_SHAPE;
    const int64_t nblk = (batch * M + PS_NT - 1) / PS_NT;
    if (nblk > 0x7fffffff) return MMB_ERR_SHAPE;
    pscan_fwd_kernel<<<(unsigned)nblk, PS_NT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        batch, L, M, A, X, H);
    return mmb_launch_status();
}

extern "C" int mmb_pscan_bwd(int64_t batch, int64_t L, int64_t M, const float* A, const float* H,
                             const float* G, float* dA, float* dX, mmb_stream_t stream) {
    MMB_NVTX("mmb_pscan_bwd");
    if (!A || !H || !G) return MMB_ERR_NULL;
    if (batch <= 0 || L <= 0 || M <= 0) return MMB_ERR_SHAPE;
    if (!dA && !dX) return MMB_OK;
    const int64_t nblk = (batch * M + PS_NT - 1) / PS_NT;
    if (nblk > 0x7fffffff) return MMB_ERR_SHAPE;
    pscan_bwd_kernel<<<(unsigned)nblk, PS_NT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        batch, L, M, A, H, G, dA, dX);
    return mmb_launch_status();
}
