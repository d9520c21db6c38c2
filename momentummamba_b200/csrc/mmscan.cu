// Fused momentum selective scan for sm_100a: forward and backward.
//
// Work decomposition: one CTA of 128 threads owns one sequence b and a tile of
// DT = 128 / G channels for the whole sequence, G = N / NP lanes per channel; a
// thread owns one channel d and NP (2 or 4) of its N states, h and v in
// registers, updated with packed fp32 pairs (sm_100 f32x2 FMA).  NP is picked
// per call: 2 when the problem is so small that 4 states per thread would leave
// the SMs under two warps each, else 4 (fewer cross-lane sums; measured faster
// from B*D = 8192 channels up).  The sequence is streamed through shared memory in chunks of T = 32
// steps with double-buffered cp.async (x, delta, z, B, C tiles; rows of the
// (B, L, D) tensors are coalesced 16-byte copies).
//
// Per 8-step block, each lane owns 8/G (t, d) items of its channel (at least
// one): it computes softplus(delta + bias), alpha*dt*x and the SiLU(z) gate for
// them once, the per-step scalars are shuffled to the channel's lanes, the
// block's decay factors exp(dt*A) are issued before the recurrence, and the
// channel's partial sums of y = C h are reduce-scattered so each lane finishes
// its own items.
//
// The forward stores (h, v) every 8 steps as checkpoints.  The backward walks
// the sequence in reverse, 8 steps at a time: it recomputes the window forward
// from its checkpoint into registers (a_t and h_t), then runs the adjoint
// backwards through it:
//   gh_t = dy_t C_t + a_{t+1} gh_{t+1} ;  gv_t = gh_t + beta gv_{t+1}
// The n-sums (dx, ddelta, recomputed y) are reduce-scattered back to the
// owning lanes; the d-sums of the dB | dC contributions go through a per-warp
// shared window buffer and vector reductions to global memory; dA, dD and
// d(delta_bias) accumulate in registers over the sequence.
#include "mmb_common.cuh"

namespace mmb {

constexpr int MM_NT = 128;  // threads per CTA
constexpr int MM_T = 32;    // steps per staged chunk
constexpr int MM_CK = 8;    // checkpoint interval = steps per register block
constexpr unsigned FULL = 0xffffffffu;
// cp.async pipeline depth in chunks (3 and 4 stages measured no faster: the
// kernels are issue-latency bound, not load-latency bound)
constexpr int MM_NS = 2;

__host__ __device__ constexpr int ilog2c(int v) { return v <= 1 ? 0 : 1 + ilog2c(v / 2); }

template <int N, int NP>
struct MMCfg {
    static constexpr int NP2 = NP / 2;                // packed pairs per thread
    static constexpr int G = N / NP;                  // lanes per channel
    static constexpr int LOG2G = ilog2c(G);
    static constexpr int LB = LOG2G < 3 ? LOG2G : 3;  // lane bits that split an 8-step block
    static constexpr int IPL = MM_CK >> LB;           // (t, d) items a lane owns per block
    static constexpr int DT = MM_NT / G;              // channels per CTA
    static constexpr int DPW = 32 / G;                // channels per warp
    static constexpr int LOG2DPW = 5 - LOG2G;
    // raw (T x DT) tile pitch: the rows and channels a warp reads at once fall in
    // distinct banks
    static constexpr int RP = G >= 16 ? DT + 4 : DT + DPW;
    static constexpr int TR = MM_T * RP;
    static constexpr int TN = MM_T * N;
    static_assert((NP == 2 || NP == 4) && N % NP == 0 && G >= 2 && G <= 16, "unsupported shape");
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

// NP consecutive floats of shared memory as packed pairs.
template <int NP>
__device__ __forceinline__ void ld_pairs(const float* p, float2 (&o)[NP / 2]) {
    if constexpr (NP == 4) {
        const float4 q = *reinterpret_cast<const float4*>(p);
        o[0] = make_float2(q.x, q.y);
        o[1] = make_float2(q.z, q.w);
    } else {
        o[0] = *reinterpret_cast<const float2*>(p);
    }
}

// sum_j c_j h_j over this thread's NP states
template <int NP2>
__device__ __forceinline__ float dot_pairs(const float2 (&c)[NP2], const float2 (&h)[NP2]) {
    float2 acc = fmul2(c[0], h[0]);
#pragma unroll
    for (int j = 1; j < NP2; ++j) acc = ffma2(c[j], h[j], acc);
    return acc.x + acc.y;
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

// checkpoint record of (b, window k, channel d): 2N floats, lane ng's
// [h(NP) | v(NP)] at ng * 2 * NP
__device__ __forceinline__ int64_t ckpt_base(const MMParams& p, int64_t b, int64_t k, int64_t d,
                                             int N) {
    const int64_t K = (p.L + MM_CK - 1) / MM_CK;
    return ((b * K + k) * p.D + d) * (int64_t)(2 * N);
}

template <int NP>
__device__ __forceinline__ void ckpt_store(float* dst, const float2 (&h)[NP / 2],
                                           const float2 (&v)[NP / 2]) {
    if constexpr (NP == 4) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(h[0].x, h[0].y, h[1].x, h[1].y);
        reinterpret_cast<float4*>(dst)[1] = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
    } else {
        reinterpret_cast<float4*>(dst)[0] = make_float4(h[0].x, h[0].y, v[0].x, v[0].y);
    }
}

template <int NP>
__device__ __forceinline__ void ckpt_load(const float* src, float2 (&h)[NP / 2],
                                          float2 (&v)[NP / 2]) {
    if constexpr (NP == 4) {
        const float4 a = reinterpret_cast<const float4*>(src)[0];
        const float4 c = reinterpret_cast<const float4*>(src)[1];
        h[0] = make_float2(a.x, a.y); h[1] = make_float2(a.z, a.w);
        v[0] = make_float2(c.x, c.y); v[1] = make_float2(c.z, c.w);
    } else {
        const float4 a = reinterpret_cast<const float4*>(src)[0];
        h[0] = make_float2(a.x, a.y);
        v[0] = make_float2(a.z, a.w);
    }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <int N, int NP, bool SOFTPLUS, bool HAS_Z>
__global__ void __launch_bounds__(MM_NT) mmscan_fwd_kernel(const MMParams p) {
    using Cf = MMCfg<N, NP>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T, RP = Cf::RP, IPL = Cf::IPL, LB = Cf::LB;
    constexpr int NP2 = Cf::NP2, NBLK = T / MM_CK;
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

    float2 A2[NP2], h[NP2], v[NP2];
#pragma unroll
    for (int j = 0; j < NP2; ++j) {
        A2[j] = f2(0.f);
        h[j] = f2(0.f);
        v[j] = f2(0.f);
        if (dvalid) {
            const float* Ar = p.A + d * N + ng * NP + 2 * j;
            A2[j] = make_float2(Ar[0] * MMB_LOG2E, Ar[1] * MMB_LOG2E);
        }
    }
    const float bias_d = (p.dbias && dvalid) ? p.dbias[d] : 0.f;
    const float Dv = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const float alpha = p.alpha;
    const float2 beta2 = f2(p.beta);
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

#pragma unroll
    for (int c = 0; c < MM_NS - 1; ++c) {
        if (c < nchunks) stage(c, c);
        cp_async_commit();
    }
    for (int c = 0; c < nchunks; ++c) {
        if (c + MM_NS - 1 < nchunks) stage((c + MM_NS - 1) % MM_NS, c + MM_NS - 1);
        cp_async_commit();
        cp_async_wait<MM_NS - 1>();
        __syncthreads();
        const float* st = smem + (c % MM_NS) * STAGE;
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
            float2 a[MM_CK][NP2];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
#pragma unroll
                for (int j = 0; j < NP2; ++j) {
                    const float2 e = fmul2(f2(dts[s]), A2[j]);
                    a[s][j] = make_float2(ex2(e.x), ex2(e.y));
                }
            }
            // next block's items while the exponentials are in flight
            float nxi[IPL], ndti[IPL], ndtxi[IPL];
            if (k + 1 < NBLK) prep(sx, sdl, k + 1, nxi, ndti, ndtxi);
            // checkpoint: state before the block's first step
            if (p.ckpt && dvalid && t0 + k * MM_CK < p.L) {
                const int64_t kk = (t0 + k * MM_CK) / MM_CK;
                ckpt_store<NP>(p.ckpt + ckpt_base(p, b, kk, d, N) + ng * 2 * NP, h, v);
            }
            float y[MM_CK];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int tt = k * MM_CK + s;
                float2 bq[NP2], cq[NP2];
                ld_pairs<NP>(sB + tt * N + ng * NP, bq);
                ld_pairs<NP>(sC + tt * N + ng * NP, cq);
#pragma unroll
                for (int j = 0; j < NP2; ++j) {
                    v[j] = ffma2(beta2, v[j], fmul2(f2(dtxs[s]), bq[j]));
                    h[j] = ffma2(a[s][j], h[j], v[j]);
                }
                y[s] = dot_pairs(cq, h);
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
// Chunks of 32 steps in reverse; inside a chunk, 8-step windows in reverse.
// The d-sums of the dB | dC contributions go through a window buffer
// [8 steps][DT channels][2N]: each thread stores its NP dB and NP dC terms as
// units of NP floats (odd channels swap the dB and dC halves, so a warp's
// stores hit distinct banks); after the window each warp sums its own DPW
// channels' rows and adds the results to global memory with vector reductions.
// ---------------------------------------------------------------------------
template <int N, int NP, bool SOFTPLUS, bool HAS_Z>
__global__ void __launch_bounds__(MM_NT) mmscan_bwd_kernel(const MMParams p) {
    using Cf = MMCfg<N, NP>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T, RP = Cf::RP, IPL = Cf::IPL, LB = Cf::LB;
    constexpr int NP2 = Cf::NP2, TR = Cf::TR, DPW = Cf::DPW;
    constexpr int NQ = 2 * N / 4;  // float4 columns per window-buffer row
    constexpr int SWZ = NQ / 2;    // float4 swizzle of odd channels (= G units of NP floats)
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    // stage s: [x | delta | z | dout] (T x RP), [B | C] (T x N)
    constexpr int STAGE = 4 * TR + 2 * Cf::TN;
    float* wbuf = smem + MM_NS * STAGE;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ng = lane & (G - 1);
    const int lane_base = lane & ~(G - 1);
    const int ibase = rs_index<MM_CK, LB>(ng & ((1 << LB) - 1), 0);
    const bool item_lane = (ng >> LB) == 0;
    const int dl = warp * DPW + (lane >> Cf::LOG2G);
    const int64_t b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * DT;
    const int64_t d = d0 + dl;
    const bool dvalid = d < p.D;
    const int dvalid_cols = (int)min64(DT, p.D - d0);
    const int swz_units = (dl & 1) ? G : 0;

    float2 A2[NP2], gh[NP2], gv[NP2], an[NP2], dA[NP2];
#pragma unroll
    for (int j = 0; j < NP2; ++j) {
        A2[j] = gh[j] = gv[j] = an[j] = dA[j] = f2(0.f);
        if (dvalid) {
            const float* Ar = p.A + d * N + ng * NP + 2 * j;
            A2[j] = make_float2(Ar[0] * MMB_LOG2E, Ar[1] * MMB_LOG2E);
        }
    }
    const float bias_d = (p.dbias && dvalid) ? p.dbias[d] : 0.f;
    const float Dv = (p.Dskip && dvalid) ? p.Dskip[d] : 0.f;
    const float alpha = p.alpha;
    const float2 beta2 = f2(p.beta);
    float accD = 0.f, accBias = 0.f;
    const int nchunks = (int)((p.L + T - 1) / T);
    float2 nck_h[NP2], nck_v[NP2];  // checkpoint of the next window to process
#pragma unroll
    for (int j = 0; j < NP2; ++j) nck_h[j] = nck_v[j] = f2(0.f);
    auto ck_load = [&](int64_t k) {
        if (dvalid) ckpt_load<NP>(p.ckpt_in + ckpt_base(p, b, k, d, N) + ng * 2 * NP, nck_h, nck_v);
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

#pragma unroll
    for (int it = 0; it < MM_NS - 1; ++it) {
        if (it < nchunks) stage(it, nchunks - 1 - it);
        cp_async_commit();
    }
    for (int it = 0; it < nchunks; ++it) {
        const int c = nchunks - 1 - it;
        if (it + MM_NS - 1 < nchunks) stage((it + MM_NS - 1) % MM_NS, c - (MM_NS - 1));
        cp_async_commit();
        cp_async_wait<MM_NS - 1>();
        __syncthreads();
        const float* st = smem + (it % MM_NS) * STAGE;
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
            if (it == 0 && w == (Lc - 1) / MM_CK) ck_load((t0 + w0) / MM_CK);
            float2 h[NP2], v[NP2];
#pragma unroll
            for (int j = 0; j < NP2; ++j) {
                h[j] = nck_h[j];
                v[j] = nck_v[j];
            }
            if (t0 + w0 > 0) ck_load((t0 + w0) / MM_CK - 1);
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
            float2 aa[MM_CK][NP2];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
#pragma unroll
                for (int j = 0; j < NP2; ++j) {
                    const float2 e = fmul2(f2(dts[s]), A2[j]);
                    aa[s][j] = make_float2(ex2(e.x), ex2(e.y));
                }
            }
            // forward replay of the window
            float2 hh[MM_CK + 1][NP2];
            float yv[MM_CK];
#pragma unroll
            for (int j = 0; j < NP2; ++j) hh[0][j] = h[j];
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int tt = w0 + s;
                float2 bq[NP2], cq[NP2];
                ld_pairs<NP>(sB + tt * N + ng * NP, bq);
                ld_pairs<NP>(sC + tt * N + ng * NP, cq);
#pragma unroll
                for (int j = 0; j < NP2; ++j) {
                    v[j] = ffma2(beta2, v[j], fmul2(f2(dtxs[s]), bq[j]));
                    h[j] = ffma2(aa[s][j], h[j], v[j]);
                    hh[s + 1][j] = h[j];
                }
                yv[s] = dot_pairs(cq, h);
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
                float2 bq[NP2], cq[NP2];
                ld_pairs<NP>(sB + tt * N + ng * NP, bq);
                ld_pairs<NP>(sC + tt * N + ng * NP, cq);
                const float2 dy2 = f2(dys[s]);
                float2 sb = f2(0.f), sa = f2(0.f), pb[NP2], pc[NP2];
#pragma unroll
                for (int j = 0; j < NP2; ++j) {
                    gh[j] = ffma2(an[j], gh[j], fmul2(dy2, cq[j]));
                    gv[j] = ffma2(beta2, gv[j], gh[j]);
                    sb = ffma2(gv[j], bq[j], sb);
                    const float2 t2 = fmul2(fmul2(gh[j], hh[s][j]), aa[s][j]);
                    sa = ffma2(t2, A2[j], sa);
                    dA[j] = ffma2(t2, f2(dts[s]), dA[j]);
                    pb[j] = fmul2(gv[j], f2(dtxs[s]));
                    pc[j] = fmul2(dy2, hh[s + 1][j]);
                    an[j] = aa[s][j];
                }
                sab[2 * s] = sa.x + sa.y;
                sab[2 * s + 1] = sb.x + sb.y;
                // dB | dC terms of (t, d, this lane's states) into the window buffer
                float* rowp = wrow + s * DT * 2 * N;
                if constexpr (NP == 4) {
                    float4* r4 = reinterpret_cast<float4*>(rowp);
                    r4[ng ^ swz_units] = make_float4(pb[0].x, pb[0].y, pb[1].x, pb[1].y);
                    r4[(G + ng) ^ swz_units] = make_float4(pc[0].x, pc[0].y, pc[1].x, pc[1].y);
                } else {
                    float2* r2 = reinterpret_cast<float2*>(rowp);
                    r2[ng ^ swz_units] = pb[0];
                    r2[(G + ng) ^ swz_units] = pc[0];
                }
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
            __syncwarp();
            // d-sum of this warp's rows of the window buffer (its DPW channels)
            {
                constexpr int ITEMS = MM_CK * NQ;
                constexpr int IPT = ITEMS >= 32 ? ITEMS / 32 : 1;
                constexpr int TPI = ITEMS >= 32 ? 1 : 32 / ITEMS;
                constexpr int RPT = DPW / TPI > 0 ? DPW / TPI : 1;
#pragma unroll
                for (int j = 0; j < IPT; ++j) {
                    const int item = (lane / TPI) + j * (32 / TPI), part = lane % TPI;
                    const int s = item / NQ, q = item % NQ;
                    float2 acc01 = f2(0.f), acc23 = f2(0.f);
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        const int row = warp * DPW + part * RPT + r;
                        const float4 vv = reinterpret_cast<const float4*>(
                            wbuf + (s * DT + row) * 2 * N)[q ^ ((row & 1) ? SWZ : 0)];
                        acc01 = fadd2(acc01, make_float2(vv.x, vv.y));
                        acc23 = fadd2(acc23, make_float2(vv.z, vv.w));
                    }
#pragma unroll
                    for (int m = 1; m < TPI; m <<= 1) {
                        acc01.x += __shfl_xor_sync(FULL, acc01.x, m);
                        acc01.y += __shfl_xor_sync(FULL, acc01.y, m);
                        acc23.x += __shfl_xor_sync(FULL, acc23.x, m);
                        acc23.y += __shfl_xor_sync(FULL, acc23.y, m);
                    }
                    const int64_t gt = t0 + w0 + s;
                    if (part == 0 && gt < p.L) {
                        const int col = q * 4;
                        float* dst = (col < N ? p.dB : p.dC) + (b * p.L + gt) * N + (col % N);
                        red_add_v4(dst, acc01.x, acc01.y, acc23.x, acc23.y);
                    }
                }
            }
            __syncwarp();
        }
        __syncthreads();
    }

    // dA: this thread's states of channel d, summed over its sequence
    if (dvalid) {
        float* dst = p.dA + d * N + ng * NP;
#pragma unroll
        for (int j = 0; j < NP2; ++j) {
            atomicAdd(dst + 2 * j, dA[j].x);
            atomicAdd(dst + 2 * j + 1, dA[j].y);
        }
    }
    // dD, dbias: sum the channel's lanes
    accD = lane_sum<0, Cf::LOG2G>(accD);
    accBias = lane_sum<0, Cf::LOG2G>(accBias);
    if (ng == 0 && dvalid) {
        if (p.dD) atomicAdd(p.dD + d, accD);
        if (p.ddbias) atomicAdd(p.ddbias + d, accBias);
    }
}

template <int N, int NP>
size_t fwd_smem_bytes() {
    using Cf = MMCfg<N, NP>;
    return sizeof(float) * (MM_NS * (3 * Cf::TR + 2 * Cf::TN));
}

template <int N, int NP>
size_t bwd_smem_bytes() {
    using Cf = MMCfg<N, NP>;
    return sizeof(float) * (MM_NS * (4 * Cf::TR + 2 * Cf::TN) + MM_CK * Cf::DT * 2 * N);
}

template <int N, int NP, bool SP, bool Z>
int launch_fwd_t(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N, NP>;
    const size_t smem = fwd_smem_bytes<N, NP>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_fwd_kernel<N, NP, SP, Z>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_fwd_kernel<N, NP, SP, Z><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
}

template <int N, int NP, bool SP, bool Z>
int launch_bwd_t(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N, NP>;
    const size_t smem = bwd_smem_bytes<N, NP>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_bwd_kernel<N, NP, SP, Z>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_bwd_kernel<N, NP, SP, Z><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
}

template <int N, int NP>
int launch_fwd_np(const MMParams& p, cudaStream_t s) {
    const bool z = p.z != nullptr;
    if (p.softplus)
        return z ? launch_fwd_t<N, NP, true, true>(p, s) : launch_fwd_t<N, NP, true, false>(p, s);
    return z ? launch_fwd_t<N, NP, false, true>(p, s) : launch_fwd_t<N, NP, false, false>(p, s);
}

template <int N, int NP>
int launch_bwd_np(const MMParams& p, cudaStream_t s) {
    const bool z = p.z != nullptr;
    if (p.softplus)
        return z ? launch_bwd_t<N, NP, true, true>(p, s) : launch_bwd_t<N, NP, true, false>(p, s);
    return z ? launch_bwd_t<N, NP, false, true>(p, s) : launch_bwd_t<N, NP, false, false>(p, s);
}

// States per thread: 2 when 4 would leave the GPU with fewer than ~16 warps per
// SM (too few to hide the recurrence's latency), else 4.  The forward and the
// backward of one call must agree (the checkpoint layout depends on it), so
// this depends only on the shape.
#ifndef MMB_NP2_THRESHOLD_WARPS_PER_SM
#define MMB_NP2_THRESHOLD_WARPS_PER_SM 2
#endif
static int states_per_thread(const MMParams& p, int64_t N) {
    if (N == 64) return 4;
    const int64_t threads4 = p.Bsz * p.D * (N / 4);
    return threads4 < (int64_t)148 * MMB_NP2_THRESHOLD_WARPS_PER_SM * 32 ? 2 : 4;
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
    const bool two = states_per_thread(p, desc->dstate) == 2;
    switch (desc->dstate) {
        case 8: return two ? launch_fwd_np<8, 2>(p, s) : launch_fwd_np<8, 4>(p, s);
        case 16: return two ? launch_fwd_np<16, 2>(p, s) : launch_fwd_np<16, 4>(p, s);
        case 32: return two ? launch_fwd_np<32, 2>(p, s) : launch_fwd_np<32, 4>(p, s);
        default: return launch_fwd_np<64, 4>(p, s);
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
    const bool two = states_per_thread(p, N) == 2;
    switch (N) {
        case 8: return two ? launch_bwd_np<8, 2>(p, s) : launch_bwd_np<8, 4>(p, s);
        case 16: return two ? launch_bwd_np<16, 2>(p, s) : launch_bwd_np<16, 4>(p, s);
        case 32: return two ? launch_bwd_np<32, 2>(p, s) : launch_bwd_np<32, 4>(p, s);
        default: return launch_bwd_np<64, 4>(p, s);
    }
}
