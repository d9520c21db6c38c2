// Fused momentum selective scan for sm_100a: forward and backward.
//
// Work decomposition: one CTA of 128 threads owns one sequence b and a tile of
// DT = 128 / (N/4) channels for the whole sequence; each thread owns one channel
// d and 4 of its N states (h, v in registers), so the N/4 lanes of a channel
// combine y = sum_n C h with two or three shuffles.  The sequence is streamed
// through shared memory in chunks of T = 32 steps with double-buffered
// cp.async (x, delta, z, B, C tiles; rows of the (B, L, D) tensors are
// coalesced 16-byte copies).  Per-(t, d) work (softplus, alpha*dt*x, SiLU(z),
// D*x) runs once per element of a tile in a pre-/post-pass, not once per state.
//
// The forward stores (h, v) every CK = 8 steps as checkpoints.  The backward
// walks the sequence in reverse, 8 steps at a time: it recomputes the 8-step
// window forward from its checkpoint into registers (a_t and h_t), then runs the
// adjoint recurrence backwards through the window:
//   gh_t = dy_t C_t + a_{t+1} gh_{t+1} ;  gv_t = gh_t + beta gv_{t+1}
// d-sums for dB, dC are reduce-scattered across the warp, summed across the
// CTA's warps in shared memory and added to global memory with vector
// reductions; dA, dD, d(delta_bias) accumulate in registers over the sequence.
#include "mmb_common.cuh"

namespace mmb {

constexpr int MM_NT = 128;  // threads per CTA
constexpr int MM_T = 32;    // steps per staged chunk
constexpr int MM_CK = 8;    // checkpoint interval = steps per register block
constexpr int MM_NPER = 4;  // states per thread
constexpr unsigned FULL = 0xffffffffu;

// How the backward sums the dB | dC contributions over channels:
//   0: reduce-scatter across the warp's channels with shuffles every step, warp
//      partials to shared memory, CTA sum + global vector reduction per chunk
//   1: shared window buffer for the CTA, summed after every 8-step window
//   2: per-warp window buffers, summed by each warp after every 8-step window
#ifndef MMB_BWD_DSUM
#define MMB_BWD_DSUM 2
#endif

template <int N>
struct MMCfg {
    static constexpr int G = N / MM_NPER;  // lanes per channel
    static constexpr int LOG2G = G == 2 ? 1 : G == 4 ? 2 : G == 8 ? 3 : G == 16 ? 4 : 0;
    static constexpr int LB = LOG2G < 3 ? LOG2G : 3;  // lane bits that split an 8-step block
    static constexpr int IPL = MM_CK >> LB;           // per-(t, d) items a lane owns per block
    static constexpr int DT = MM_NT / G;              // channels per CTA
    static constexpr int DPW = 32 / G;                // channels per warp
    static constexpr int LOG2DPW = 5 - LOG2G;
    // raw (T x DT) tile pitch: the 8/IPL rows x DPW channels a warp reads at once
    // fall in distinct banks
    static constexpr int RP = G == 16 ? DT + 4 : DT + DPW;
    static constexpr int TR = MM_T * RP;
    static constexpr int TN = MM_T * N;
    static_assert(N % MM_NPER == 0 && G >= 2 && G <= 16, "unsupported d_state");
};

// Lane (within its channel's group) that owns step s of an 8-step block: the
// inverse of the reduce-scatter placement rs_index<8, LB>.
template <int LB>
__host__ __device__ constexpr int block_owner(int s) {
    int ng = 0;
    for (int b = 0; b < LB; ++b)
        if ((s >> (2 - b)) & 1) ng |= 1 << b;
    return ng;
}

struct MMParams {
    int64_t Bsz, L, D;
    const float *x, *delta, *A, *Bm, *Cm, *Dskip, *z, *dbias;
    int64_t xs[2], ds[2], zs[2], bs[2], cs[2];
    float beta, alpha;
    int softplus;
    int vec;  // 16-byte staging allowed
    const float* ckpt_in;
    float* ckpt;
    float* out;
    // backward
    const float* dout;
    float *dx, *ddelta, *dA, *dB, *dC, *dD, *dz, *ddbias;
};

__device__ __forceinline__ int64_t ckpt_base(const MMParams& p, int64_t b, int64_t k, int64_t d,
                                             int N) {
    const int64_t K = (p.L + MM_CK - 1) / MM_CK;
    return ((b * K + k) * p.D + d) * (int64_t)(2 * N);
}

// ---------------------------------------------------------------------------
// forward
//
// Per 8-step block: each lane prepares its own IPL (t, d) items
// (dt = softplus(delta + bias), alpha*dt*x); the block's 8 per-step scalars are
// broadcast to the channel's lanes by shuffles and all 32 decay factors
// exp(dt*A) of the block are issued before the recurrence, which then runs as
// plain packed-FMA chains over the 8 steps.  The 8 partial sums of y are
// reduce-scattered so each lane ends with the full y of its own items, and the
// lane finishes those items (D skip, SiLU gate, store).  The next block's items
// are prepared while the current block's exponentials are in flight.
// ---------------------------------------------------------------------------
template <int N, bool SOFTPLUS, bool HAS_Z>
__global__ void __launch_bounds__(MM_NT) mmscan_fwd_kernel(const MMParams p) {
    using Cf = MMCfg<N>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T, RP = Cf::RP, IPL = Cf::IPL, LB = Cf::LB;
    constexpr int NBLK = T / MM_CK;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    constexpr int STAGE = 3 * Cf::TR + 2 * Cf::TN;  // x | delta | z (T x RP), B | C (T x N)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ng = lane & (G - 1);
    const int lane_base = lane & ~(G - 1);
    const int ibase = rs_index<MM_CK, LB>(ng & ((1 << LB) - 1), 0);
    const bool item_lane = (ng >> LB) == 0;  // G = 16: the upper 8 lanes duplicate
    const int dl = warp * Cf::DPW + (lane >> Cf::LOG2G);
    const int64_t b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * DT;
    const int64_t d = d0 + dl;
    const bool dvalid = d < p.D;
    const int dvalid_cols = (int)min64(DT, p.D - d0);

    float2 A2a = f2(0.f), A2b = f2(0.f);
    if (dvalid) {
        const float* Ar = p.A + d * N + ng * MM_NPER;
        A2a = make_float2(Ar[0] * MMB_LOG2E, Ar[1] * MMB_LOG2E);
        A2b = make_float2(Ar[2] * MMB_LOG2E, Ar[3] * MMB_LOG2E);
    }
    const float bias_d = (p.dbias && dvalid) ? p.dbias[d] : 0.f;
    const float Dv = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const float alpha = p.alpha;
    const float2 beta2 = f2(p.beta);
    float2 h01 = f2(0.f), h23 = f2(0.f), v01 = f2(0.f), v23 = f2(0.f);
    const int nchunks = (int)((p.L + T - 1) / T);

    auto stage = [&](int s, int c) {
        float* st = smem + s * STAGE;
        const int64_t t0 = (int64_t)c * T;
        const int rv = (int)min64(T, p.L - t0);
        stage_tile<T, DT, RP, MM_NT>(st, p.x + b * p.xs[0] + t0 * p.xs[1] + d0, p.xs[1], rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, DT, RP, MM_NT>(st + Cf::TR, p.delta + b * p.ds[0] + t0 * p.ds[1] + d0,
                                     p.ds[1], rv, dvalid_cols, p.vec, tid);
        if (HAS_Z)
            stage_tile<T, DT, RP, MM_NT>(st + 2 * Cf::TR, p.z + b * p.zs[0] + t0 * p.zs[1] + d0,
                                         p.zs[1], rv, dvalid_cols, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 3 * Cf::TR, p.Bm + b * p.bs[0] + t0 * p.bs[1], p.bs[1],
                                   rv, N, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 3 * Cf::TR + Cf::TN, p.Cm + b * p.cs[0] + t0 * p.cs[1],
                                   p.cs[1], rv, N, p.vec, tid);
    };
    // this lane's items of block k: x, dt, alpha*dt*x
    auto prep = [&](const float* sx, const float* sdl, int k, float (&xi)[IPL], float (&dti)[IPL],
                    float (&dtxi)[IPL]) {
#pragma unroll
        for (int i = 0; i < IPL; ++i) {
            const int row = (k * MM_CK + ibase + i) * RP + dl;
            xi[i] = sx[row];
            const float r = sdl[row] + bias_d;
            dti[i] = SOFTPLUS ? softplus_f(r) : r;
            dtxi[i] = alpha * dti[i] * xi[i];
        }
    };

    stage(0, 0);
    cp_async_commit();
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) stage((c + 1) & 1, c + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* st = smem + (c & 1) * STAGE;
        const float* sx = st;
        const float* sdl = st + Cf::TR;
        const float* sz = st + 2 * Cf::TR;
        const float* sB = st + 3 * Cf::TR;
        const float* sC = sB + Cf::TN;
        const int64_t t0 = (int64_t)c * T;

        float xi[IPL], dti[IPL], dtxi[IPL];
        prep(sx, sdl, 0, xi, dti, dtxi);
#pragma unroll
        for (int k = 0; k < NBLK; ++k) {
            // broadcast the block's per-step scalars, then all its decay factors
            float dts[MM_CK], dtxs[MM_CK];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int src = lane_base | block_owner<LB>(s - s % IPL);
                dts[s] = __shfl_sync(FULL, dti[s % IPL], src);
                dtxs[s] = __shfl_sync(FULL, dtxi[s % IPL], src);
            }
            float2 a[MM_CK][2];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const float2 e01 = fmul2(f2(dts[s]), A2a), e23 = fmul2(f2(dts[s]), A2b);
                a[s][0] = make_float2(ex2(e01.x), ex2(e01.y));
                a[s][1] = make_float2(ex2(e23.x), ex2(e23.y));
            }
            // next block's items while the exponentials are in flight
            float nxi[IPL], ndti[IPL], ndtxi[IPL];
            if (k + 1 < NBLK) prep(sx, sdl, k + 1, nxi, ndti, ndtxi);
            // checkpoint: state before the block's first step
            if (p.ckpt && dvalid && t0 + k * MM_CK < p.L) {
                const int64_t kk = (t0 + k * MM_CK) / MM_CK;
                float4* dst = reinterpret_cast<float4*>(p.ckpt + ckpt_base(p, b, kk, d, N) +
                                                        ng * 2 * MM_NPER);
                dst[0] = make_float4(h01.x, h01.y, h23.x, h23.y);
                dst[1] = make_float4(v01.x, v01.y, v23.x, v23.y);
            }
            float y[MM_CK];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int tt = k * MM_CK + s;
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
                const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
                v01 = ffma2(beta2, v01, fmul2(f2(dtxs[s]), make_float2(b4.x, b4.y)));
                v23 = ffma2(beta2, v23, fmul2(f2(dtxs[s]), make_float2(b4.z, b4.w)));
                h01 = ffma2(a[s][0], h01, v01);
                h23 = ffma2(a[s][1], h23, v23);
                float2 yy = fmul2(make_float2(c4.x, c4.y), h01);
                yy = ffma2(make_float2(c4.z, c4.w), h23, yy);
                y[s] = yy.x + yy.y;
            }
            reduce_scatter<MM_CK, 0, Cf::LOG2G>(y, lane);
            // finish this lane's items: D skip, gate, store
#pragma unroll
            for (int i = 0; i < IPL; ++i) {
                const int tt = k * MM_CK + ibase + i;
                const int64_t gt = t0 + tt;
                float o = fmaf(Dv, xi[i], y[i]);
                if (HAS_Z) {
                    const float zv = sz[tt * RP + dl];
                    o *= zv * sigmoid_f(zv);
                }
                if (item_lane && dvalid && gt < p.L) p.out[(b * p.L + gt) * p.D + d] = o;
            }
            if (k + 1 < NBLK) {
#pragma unroll
                for (int i = 0; i < IPL; ++i) {
                    xi[i] = nxi[i];
                    dti[i] = ndti[i];
                    dtxi[i] = ndtxi[i];
                }
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// backward
//
// Chunks of 32 steps in reverse; inside a chunk, 8-step windows in reverse.  A
// window replays the recurrence forward from its checkpoint keeping a_t and h_t
// in registers, then runs the adjoint backwards through it.  Per-(t, d) work is
// owned by one lane as in the forward, and the n-sums (dx, ddelta, the
// recomputed y) are reduce-scattered back to the owning lanes.  The d-sums of
// the dB | dC contributions go through a shared window buffer
// [8 steps][DT channels][2N] (float4 columns XOR-swizzled by channel parity so
// that each quarter-warp's stores hit distinct banks): after each window the
// CTA sums the buffer over its DT channels and adds the 8 x 2N results to
// global memory with vector reductions.
// ---------------------------------------------------------------------------
template <int N, bool SOFTPLUS, bool HAS_Z>
__global__ void __launch_bounds__(MM_NT) mmscan_bwd_kernel(const MMParams p) {
    using Cf = MMCfg<N>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T, RP = Cf::RP, IPL = Cf::IPL, LB = Cf::LB;
    constexpr int TR = Cf::TR;
    constexpr int WB = MM_CK * DT * 2 * N;  // window buffer floats
    constexpr int NQ = 2 * N / 4;           // float4 columns per buffer row
    constexpr int SWZ = NQ / 2;             // swizzle: odd channels swap the dB and dC halves
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    // stage s: [x | delta | z | dout] (T x RP), [B | C] (T x N)
    constexpr int STAGE = 4 * TR + 2 * Cf::TN;
    float* wbuf = smem + 2 * STAGE;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ng = lane & (G - 1);
    const int lane_base = lane & ~(G - 1);
    const int ibase = rs_index<MM_CK, LB>(ng & ((1 << LB) - 1), 0);
    const bool item_lane = (ng >> LB) == 0;
    const int dl = warp * Cf::DPW + (lane >> Cf::LOG2G);
    const int64_t b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * DT;
    const int64_t d = d0 + dl;
    const bool dvalid = d < p.D;
    const int dvalid_cols = (int)min64(DT, p.D - d0);
    const int swz = (dl & 1) ? SWZ : 0;

    float2 A2a = f2(0.f), A2b = f2(0.f);
    if (dvalid) {
        const float* Ar = p.A + d * N + ng * MM_NPER;
        A2a = make_float2(Ar[0] * MMB_LOG2E, Ar[1] * MMB_LOG2E);
        A2b = make_float2(Ar[2] * MMB_LOG2E, Ar[3] * MMB_LOG2E);
    }
    const float bias_d = (p.dbias && dvalid) ? p.dbias[d] : 0.f;
    const float Dv = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const float alpha = p.alpha;
    const float2 beta2 = f2(p.beta);
    float2 gh01 = f2(0.f), gh23 = f2(0.f), gv01 = f2(0.f), gv23 = f2(0.f);
    float2 an01 = f2(0.f), an23 = f2(0.f);  // a_{t+1}
    float2 dA01 = f2(0.f), dA23 = f2(0.f);
    float accD = 0.f, accBias = 0.f;
    const int nchunks = (int)((p.L + T - 1) / T);
    float4 nck_h = make_float4(0.f, 0.f, 0.f, 0.f), nck_v = nck_h;
    auto ck_load = [&](int64_t k, float4& hq, float4& vq) {
        if (dvalid) {
            const float4* src = reinterpret_cast<const float4*>(
                p.ckpt_in + ckpt_base(p, b, k, d, N) + ng * 2 * MM_NPER);
            hq = src[0];
            vq = src[1];
        }
    };

    auto stage = [&](int s, int c) {
        float* st = smem + s * STAGE;
        const int64_t t0 = (int64_t)c * T;
        const int rv = (int)min64(T, p.L - t0);
        stage_tile<T, DT, RP, MM_NT>(st, p.x + b * p.xs[0] + t0 * p.xs[1] + d0, p.xs[1], rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, DT, RP, MM_NT>(st + TR, p.delta + b * p.ds[0] + t0 * p.ds[1] + d0, p.ds[1],
                                     rv, dvalid_cols, p.vec, tid);
        if (HAS_Z)
            stage_tile<T, DT, RP, MM_NT>(st + 2 * TR, p.z + b * p.zs[0] + t0 * p.zs[1] + d0,
                                         p.zs[1], rv, dvalid_cols, p.vec, tid);
        stage_tile<T, DT, RP, MM_NT>(st + 3 * TR, p.dout + (b * p.L + t0) * p.D + d0, p.D, rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 4 * TR, p.Bm + b * p.bs[0] + t0 * p.bs[1], p.bs[1], rv, N,
                                   p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 4 * TR + Cf::TN, p.Cm + b * p.cs[0] + t0 * p.cs[1],
                                   p.cs[1], rv, N, p.vec, tid);
    };

    stage(0, nchunks - 1);
    cp_async_commit();
    for (int it = 0; it < nchunks; ++it) {
        const int c = nchunks - 1 - it;
        if (c > 0) stage((it + 1) & 1, c - 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const float* st = smem + (it & 1) * STAGE;
        const float* sx = st;
        const float* sdl = st + TR;
        const float* sz = st + 2 * TR;
        const float* sdo = st + 3 * TR;
        const float* sB = st + 4 * TR;
        const float* sC = sB + Cf::TN;
        const int64_t t0 = (int64_t)c * T;
        const int Lc = (int)min64(T, p.L - t0);

        for (int w = (Lc - 1) / MM_CK; w >= 0; --w) {
            const int w0 = w * MM_CK;
            // window checkpoint (loaded one window ahead)
            if (it == 0 && w == (Lc - 1) / MM_CK) ck_load((t0 + w0) / MM_CK, nck_h, nck_v);
            float2 h01 = make_float2(nck_h.x, nck_h.y), h23 = make_float2(nck_h.z, nck_h.w);
            float2 v01 = make_float2(nck_v.x, nck_v.y), v23 = make_float2(nck_v.z, nck_v.w);
            if (t0 + w0 > 0) ck_load((t0 + w0) / MM_CK - 1, nck_h, nck_v);
            // this lane's items: dt, alpha*dt*x, dy = dout*silu(z)
            float xi[IPL], ri[IPL], dti[IPL], dtxi[IPL], dyi[IPL];
#pragma unroll
            for (int i = 0; i < IPL; ++i) {
                const int row = (w0 + ibase + i) * RP + dl;
                xi[i] = sx[row];
                ri[i] = sdl[row] + bias_d;
                dti[i] = SOFTPLUS ? softplus_f(ri[i]) : ri[i];
                dtxi[i] = alpha * dti[i] * xi[i];
                float dy = sdo[row];
                if (HAS_Z) {
                    const float zv = sz[row];
                    dy *= zv * sigmoid_f(zv);
                }
                dyi[i] = dy;
            }
            float dts[MM_CK], dtxs[MM_CK];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int src = lane_base | block_owner<LB>(s - s % IPL);
                dts[s] = __shfl_sync(FULL, dti[s % IPL], src);
                dtxs[s] = __shfl_sync(FULL, dtxi[s % IPL], src);
            }
            float2 aa[MM_CK][2];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const float2 e01 = fmul2(f2(dts[s]), A2a), e23 = fmul2(f2(dts[s]), A2b);
                aa[s][0] = make_float2(ex2(e01.x), ex2(e01.y));
                aa[s][1] = make_float2(ex2(e23.x), ex2(e23.y));
            }
            // forward replay of the window
            float2 hh[MM_CK + 1][2];
            float yv[MM_CK];
            hh[0][0] = h01; hh[0][1] = h23;
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int tt = w0 + s;
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
                const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
                v01 = ffma2(beta2, v01, fmul2(f2(dtxs[s]), make_float2(b4.x, b4.y)));
                v23 = ffma2(beta2, v23, fmul2(f2(dtxs[s]), make_float2(b4.z, b4.w)));
                h01 = ffma2(aa[s][0], h01, v01);
                h23 = ffma2(aa[s][1], h23, v23);
                hh[s + 1][0] = h01; hh[s + 1][1] = h23;
                float2 yy = fmul2(make_float2(c4.x, c4.y), h01);
                yy = ffma2(make_float2(c4.z, c4.w), h23, yy);
                yv[s] = yy.x + yy.y;
            }
            reduce_scatter<MM_CK, 0, Cf::LOG2G>(yv, lane);
            float dys[MM_CK];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int src = lane_base | block_owner<LB>(s - s % IPL);
                dys[s] = __shfl_sync(FULL, dyi[s % IPL], src);
            }
            // adjoint sweep
            float sab[2 * MM_CK];
            float* wrow = wbuf + dl * 2 * N;
#pragma unroll
            for (int s = MM_CK - 1; s >= 0; --s) {
                const int tt = w0 + s;
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
                const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
                const float2 b01 = make_float2(b4.x, b4.y), b23 = make_float2(b4.z, b4.w);
                const float2 dy2 = f2(dys[s]);
                gh01 = ffma2(an01, gh01, fmul2(dy2, make_float2(c4.x, c4.y)));
                gh23 = ffma2(an23, gh23, fmul2(dy2, make_float2(c4.z, c4.w)));
                gv01 = ffma2(beta2, gv01, gh01);
                gv23 = ffma2(beta2, gv23, gh23);
                float2 sb = fmul2(gv01, b01);
                sb = ffma2(gv23, b23, sb);
                const float2 t01 = fmul2(fmul2(gh01, hh[s][0]), aa[s][0]);
                const float2 t23 = fmul2(fmul2(gh23, hh[s][1]), aa[s][1]);
                float2 sa = fmul2(t01, A2a);
                sa = ffma2(t23, A2b, sa);
                dA01 = ffma2(t01, f2(dts[s]), dA01);
                dA23 = ffma2(t23, f2(dts[s]), dA23);
                sab[2 * s] = sa.x + sa.y;
                sab[2 * s + 1] = sb.x + sb.y;
                const float2 pb01 = fmul2(gv01, f2(dtxs[s])), pb23 = fmul2(gv23, f2(dtxs[s]));
                const float2 pc01 = fmul2(dy2, hh[s + 1][0]), pc23 = fmul2(dy2, hh[s + 1][1]);
                an01 = aa[s][0];
                an23 = aa[s][1];
#if MMB_BWD_DSUM == 0
                {
                    // d-sum over this warp's channels by reduce-scatter
                    float vals[2 * MM_NPER] = {pb01.x, pb01.y, pb23.x, pb23.y,
                                               pc01.x, pc01.y, pc23.x, pc23.y};
                    reduce_scatter<2 * MM_NPER, Cf::LOG2G, Cf::LOG2DPW>(vals, lane);
                    constexpr int KEEP =
                        (2 * MM_NPER >> Cf::LOG2DPW) > 0 ? (2 * MM_NPER >> Cf::LOG2DPW) : 1;
                    constexpr int USED_BITS = Cf::LOG2DPW < 3 ? Cf::LOG2DPW : 3;
                    const int dbits = lane >> Cf::LOG2G;
                    if ((dbits >> USED_BITS) == 0) {
#pragma unroll
                        for (int i = 0; i < KEEP; ++i) {
                            const int idx = rs_index<2 * MM_NPER, Cf::LOG2DPW>(dbits, i);
                            const int kind = idx / MM_NPER, n = ng * MM_NPER + idx % MM_NPER;
                            wbuf[(warp * T + tt) * 2 * N + kind * N + n] = vals[i];
                        }
                    }
                }
#else
                // dB | dC contributions of (t, d, this lane's 4 states) into the window buffer
                float4* rowq = reinterpret_cast<float4*>(wrow + s * DT * 2 * N);
                rowq[(ng) ^ swz] = make_float4(pb01.x, pb01.y, pb23.x, pb23.y);
                rowq[(G + ng) ^ swz] = make_float4(pc01.x, pc01.y, pc23.x, pc23.y);
#endif
            }
            // n-sums back to the owning lanes: sab[2i], sab[2i + 1] = (SA, SB) of item i
            reduce_scatter<2 * MM_CK, 0, Cf::LOG2G>(sab, lane);
            if (G == 16) sab[1] = __shfl_xor_sync(FULL, sab[0], 8);
#pragma unroll
            for (int i = 0; i < IPL; ++i) {
                const int tt = w0 + ibase + i;
                const int64_t gt = t0 + tt;
                const int64_t gi = (b * p.L + gt) * p.D + d;
                const bool ok = item_lane && dvalid && gt < p.L;
                const float SA = sab[2 * i] * MMB_LN2;
                const float SB = sab[2 * i + 1];
                const float xv = xi[i];
                if (HAS_Z) {
                    const float zv = sz[tt * RP + dl];
                    const float sg = sigmoid_f(zv);
                    const float yfull = fmaf(Dv, xv, yv[i]);
                    const float gz = sdo[tt * RP + dl] * yfull * sg * (1.f + zv * (1.f - sg));
                    if (ok && p.dz) p.dz[gi] = gz;
                }
                float gdt = fmaf(alpha * xv, SB, SA);
                if (SOFTPLUS) gdt *= softplus_grad(ri[i]);
                if (ok) {
                    p.dx[gi] = fmaf(dyi[i], Dv, alpha * dti[i] * SB);
                    p.ddelta[gi] = gdt;
                    accD = fmaf(dyi[i], xv, accD);
                    accBias += gdt;
                }
            }
#if MMB_BWD_DSUM == 1
            __syncthreads();
            // d-sum of the window buffer: (step, float4 column) pairs spread over the CTA
            {
                constexpr int ITEMS = MM_CK * NQ;                       // (step, column) pairs
                constexpr int TPI = ITEMS >= MM_NT ? 1 : MM_NT / ITEMS;  // threads per pair
                constexpr int IPT = ITEMS >= MM_NT ? ITEMS / MM_NT : 1;  // pairs per thread
                constexpr int RPT = DT / TPI;                           // channel rows per thread
                static_assert((TPI & (TPI - 1)) == 0 && DT % TPI == 0, "window reduction layout");
#pragma unroll
                for (int j = 0; j < IPT; ++j) {
                    const int item = (tid / TPI) + j * (MM_NT / TPI), part = tid % TPI;
                    const int s = item / NQ, q = item % NQ;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
                    for (int r = 0; r < RPT; ++r) {
                        const int row = part * RPT + r;
                        const float4 v = reinterpret_cast<const float4*>(
                            wbuf + (s * DT + row) * 2 * N)[q ^ ((row & 1) ? SWZ : 0)];
                        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                    }
#pragma unroll
                    for (int m = 1; m < TPI; m <<= 1) {
                        acc.x += __shfl_xor_sync(FULL, acc.x, m);
                        acc.y += __shfl_xor_sync(FULL, acc.y, m);
                        acc.z += __shfl_xor_sync(FULL, acc.z, m);
                        acc.w += __shfl_xor_sync(FULL, acc.w, m);
                    }
                    const int64_t gt = t0 + w0 + s;
                    if (part == 0 && gt < p.L) {
                        const int col = q * 4;
                        float* dst = (col < N ? p.dB : p.dC) + (b * p.L + gt) * N + (col % N);
                        red_add_v4(dst, acc.x, acc.y, acc.z, acc.w);
                    }
                }
            }
            __syncthreads();
#elif MMB_BWD_DSUM == 2
            __syncwarp();
            // d-sum of this warp's part of the window buffer (its DPW channels)
            {
                constexpr int ITEMS = MM_CK * NQ;
                constexpr int IPT = ITEMS >= 32 ? ITEMS / 32 : 1;
                constexpr int TPI = ITEMS >= 32 ? 1 : 32 / ITEMS;
                constexpr int RPT = Cf::DPW / TPI;
#pragma unroll
                for (int j = 0; j < IPT; ++j) {
                    const int item = (lane / TPI) + j * (32 / TPI), part = lane % TPI;
                    const int s = item / NQ, q = item % NQ;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        const int row = warp * Cf::DPW + part * RPT + r;
                        const float4 v = reinterpret_cast<const float4*>(
                            wbuf + (s * DT + row) * 2 * N)[q ^ ((row & 1) ? SWZ : 0)];
                        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                    }
#pragma unroll
                    for (int m = 1; m < TPI; m <<= 1) {
                        acc.x += __shfl_xor_sync(FULL, acc.x, m);
                        acc.y += __shfl_xor_sync(FULL, acc.y, m);
                        acc.z += __shfl_xor_sync(FULL, acc.z, m);
                        acc.w += __shfl_xor_sync(FULL, acc.w, m);
                    }
                    const int64_t gt = t0 + w0 + s;
                    if (part == 0 && gt < p.L) {
                        const int col = q * 4;
                        float* dst = (col < N ? p.dB : p.dC) + (b * p.L + gt) * N + (col % N);
                        red_add_v4(dst, acc.x, acc.y, acc.z, acc.w);
                    }
                }
            }
            __syncwarp();
#endif
        }
        __syncthreads();
#if MMB_BWD_DSUM == 0
        // dB | dC of this chunk: sum the warps' partials, add to global
        for (int f = tid; f < T * 2 * N / 4; f += MM_NT) {
            const int tt = (f * 4) / (2 * N), q = (f * 4) % (2 * N);
            if (tt < Lc) {
                float4 acc = *reinterpret_cast<const float4*>(wbuf + tt * 2 * N + q);
#pragma unroll
                for (int w2 = 1; w2 < 4; ++w2) {
                    const float4 o =
                        *reinterpret_cast<const float4*>(wbuf + (w2 * T + tt) * 2 * N + q);
                    acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
                }
                float* dst = (q < N ? p.dB : p.dC) + (b * p.L + t0 + tt) * N + (q % N);
                red_add_v4(dst, acc.x, acc.y, acc.z, acc.w);
            }
        }
        __syncthreads();
#endif
    }

    // dA: this thread's 4 states of channel d, summed over its sequence
    if (dvalid) {
        float* dst = p.dA + d * N + ng * MM_NPER;
        atomicAdd(dst + 0, dA01.x);
        atomicAdd(dst + 1, dA01.y);
        atomicAdd(dst + 2, dA23.x);
        atomicAdd(dst + 3, dA23.y);
    }
    // dD, dbias: sum the channel's lanes
    accD = lane_sum<0, Cf::LOG2G>(accD);
    accBias = lane_sum<0, Cf::LOG2G>(accBias);
    if (ng == 0 && dvalid) {
        if (p.dD) atomicAdd(p.dD + d, accD);
        if (p.ddbias) atomicAdd(p.ddbias + d, accBias);
    }
}

template <int N>
size_t fwd_smem_bytes() {
    using Cf = MMCfg<N>;
    return sizeof(float) * (2 * (3 * Cf::TR + 2 * Cf::TN));
}

template <int N>
size_t bwd_smem_bytes() {
    using Cf = MMCfg<N>;
    const size_t dsum = MMB_BWD_DSUM == 0 ? 4 * MM_T * 2 * N : MM_CK * Cf::DT * 2 * N;
    return sizeof(float) * (2 * (4 * Cf::TR + 2 * Cf::TN) + dsum);
}

template <int N, bool SP, bool Z>
int launch_fwd_t(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N>;
    const size_t smem = fwd_smem_bytes<N>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_fwd_kernel<N, SP, Z>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_fwd_kernel<N, SP, Z><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
}

template <int N, bool SP, bool Z>
int launch_bwd_t(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N>;
    const size_t smem = bwd_smem_bytes<N>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_bwd_kernel<N, SP, Z>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_bwd_kernel<N, SP, Z><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
}

template <int N>
int launch_fwd(const MMParams& p, cudaStream_t stream) {
    const bool z = p.z != nullptr;
    if (p.softplus) return z ? launch_fwd_t<N, true, true>(p, stream) : launch_fwd_t<N, true, false>(p, stream);
    return z ? launch_fwd_t<N, false, true>(p, stream) : launch_fwd_t<N, false, false>(p, stream);
}

template <int N>
int launch_bwd(const MMParams& p, cudaStream_t stream) {
    const bool z = p.z != nullptr;
    if (p.softplus) return z ? launch_bwd_t<N, true, true>(p, stream) : launch_bwd_t<N, true, false>(p, stream);
    return z ? launch_bwd_t<N, false, true>(p, stream) : launch_bwd_t<N, false, false>(p, stream);
}

static bool aligned16(const void* ptr) { return ptr == nullptr || ((uintptr_t)ptr & 15) == 0; }

static int fill_params(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                       const float* A, const float* B, const float* C, const float* D,
                       const float* z, const float* dbias, MMParams& p) {
    if (!desc || !x || !delta || !A || !B || !C) return MMB_ERR_NULL;
    if (desc->batch <= 0 || desc->seqlen <= 0 || desc->dim <= 0) return MMB_ERR_SHAPE;
    if (desc->batch > 65535) return MMB_ERR_SHAPE;
    const int64_t N = desc->dstate;
    if (N != 8 && N != 16 && N != 32 && N != 64) return MMB_ERR_UNSUPPORTED;
    p = MMParams{};
    p.Bsz = desc->batch;
    p.L = desc->seqlen;
    p.D = desc->dim;
    p.x = x; p.delta = delta; p.A = A; p.Bm = B; p.Cm = C; p.Dskip = D; p.z = z; p.dbias = dbias;
    for (int i = 0; i < 2; ++i) {
        p.xs[i] = desc->x_stride[i];
        p.ds[i] = desc->delta_stride[i];
        p.zs[i] = desc->z_stride[i];
        p.bs[i] = desc->B_stride[i];
        p.cs[i] = desc->C_stride[i];
    }
    p.beta = desc->beta;
    p.alpha = desc->alpha;
    p.softplus = desc->delta_softplus != 0;
    bool vec = aligned16(x) && aligned16(delta) && aligned16(z) && aligned16(B) && aligned16(C) &&
               (p.D % 4 == 0);
    for (int i = 0; i < 2; ++i)
        vec = vec && (p.xs[i] % 4 == 0) && (p.ds[i] % 4 == 0) && (!z || p.zs[i] % 4 == 0) &&
              (p.bs[i] % 4 == 0) && (p.cs[i] % 4 == 0);
    p.vec = vec ? 1 : 0;
    return MMB_OK;
}

}  // namespace mmb

using namespace mmb;

extern "C" size_t mmb_mmscan_ckpt_floats(int64_t batch, int64_t seqlen, int64_t dim,
                                         int64_t dstate) {
    if (batch <= 0 || seqlen <= 0 || dim <= 0 || dstate <= 0) return 0;
    const int64_t K = (seqlen + MM_CK - 1) / MM_CK;
    return (size_t)(batch * K * dim * dstate * 2);
}

extern "C" int mmb_mmscan_fwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                              const float* A, const float* B, const float* C, const float* D,
                              const float* z, const float* delta_bias, float* out, float* ckpt,
                              mmb_stream_t stream) {
    MMParams p;
    int st = fill_params(desc, x, delta, A, B, C, D, z, delta_bias, p);
    if (st != MMB_OK) return st;
    if (!out) return MMB_ERR_NULL;
    if (!aligned16(ckpt)) return MMB_ERR_ALIGN;
    p.out = out;
    p.ckpt = ckpt;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (desc->dstate) {
        case 8: return launch_fwd<8>(p, s);
        case 16: return launch_fwd<16>(p, s);
        case 32: return launch_fwd<32>(p, s);
        default: return launch_fwd<64>(p, s);
    }
}

extern "C" int mmb_mmscan_bwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                              const float* A, const float* B, const float* C, const float* D,
                              const float* z, const float* delta_bias, const float* ckpt,
                              const float* dout, float* dx, float* ddelta, float* dA, float* dB,
                              float* dC, float* dD, float* dz, float* ddelta_bias,
                              mmb_stream_t stream) {
    MMParams p;
    int st = fill_params(desc, x, delta, A, B, C, D, z, delta_bias, p);
    if (st != MMB_OK) return st;
    if (!ckpt) return MMB_ERR_WORKSPACE;
    if (!dout || !dx || !ddelta || !dA || !dB || !dC) return MMB_ERR_NULL;
    if (!aligned16(ckpt) || !aligned16(dout) || !aligned16(dB) || !aligned16(dC))
        return MMB_ERR_ALIGN;
    p.ckpt_in = ckpt;
    p.dout = dout;
    p.dx = dx; p.ddelta = ddelta; p.dA = dA; p.dB = dB; p.dC = dC;
    p.dD = D ? dD : nullptr;
    p.dz = z ? dz : nullptr;
    p.ddbias = delta_bias ? ddelta_bias : nullptr;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t N = desc->dstate;
    const size_t bln = (size_t)(p.Bsz * p.L * N) * sizeof(float);
    if (cudaMemsetAsync(dB, 0, bln, s) != cudaSuccess) return MMB_ERR_LAUNCH;
    if (cudaMemsetAsync(dC, 0, bln, s) != cudaSuccess) return MMB_ERR_LAUNCH;
    if (cudaMemsetAsync(dA, 0, (size_t)(p.D * N) * sizeof(float), s) != cudaSuccess)
        return MMB_ERR_LAUNCH;
    if (p.dD && cudaMemsetAsync(p.dD, 0, (size_t)p.D * sizeof(float), s) != cudaSuccess)
        return MMB_ERR_LAUNCH;
    if (p.ddbias && cudaMemsetAsync(p.ddbias, 0, (size_t)p.D * sizeof(float), s) != cudaSuccess)
        return MMB_ERR_LAUNCH;
    switch (N) {
        case 8: return launch_bwd<8>(p, s);
        case 16: return launch_bwd<16>(p, s);
        case 32: return launch_bwd<32>(p, s);
        default: return launch_bwd<64>(p, s);
    }
}
