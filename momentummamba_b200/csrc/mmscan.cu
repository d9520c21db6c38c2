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
constexpr int MM_CK = 8;    // checkpoint interval (steps)
constexpr int MM_NPER = 4;  // states per thread

template <int N>
struct MMCfg {
    static constexpr int G = N / MM_NPER;          // lanes per channel
    static constexpr int LOG2G = G == 2 ? 1 : G == 4 ? 2 : G == 8 ? 3 : G == 16 ? 4 : 0;
    static constexpr int DT = MM_NT / G;           // channels per CTA
    static constexpr int DPW = 32 / G;             // channels per warp
    static constexpr int TD = MM_T * DT;           // floats of a (T x DT) tile
    static constexpr int TN = MM_T * N;            // floats of a (T x N) tile
    static_assert(N % MM_NPER == 0 && G >= 2 && G <= 16, "unsupported d_state");
};

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
// ---------------------------------------------------------------------------
template <int N>
__global__ void __launch_bounds__(MM_NT) mmscan_fwd_kernel(const MMParams p) {
    using Cf = MMCfg<N>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    // stage s: [x | delta | z] (T x DT each), [B | C] (T x N each)
    constexpr int STAGE = 3 * Cf::TD + 2 * Cf::TN;
    float* sdtx = smem + 2 * STAGE;  // alpha*dt*x
    float* sy = sdtx + Cf::TD;       // sum_n C h

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ng = lane & (G - 1);
    const int dl = warp * Cf::DPW + lane / G;
    const int64_t b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * DT;
    const int64_t d = d0 + dl;
    const bool dvalid = d < p.D;
    const int dvalid_cols = (int)min64(DT, p.D - d0);

    float A2[MM_NPER], h[MM_NPER], v[MM_NPER];
#pragma unroll
    for (int j = 0; j < MM_NPER; ++j) {
        A2[j] = dvalid ? p.A[d * N + ng * MM_NPER + j] * MMB_LOG2E : 0.f;
        h[j] = 0.f;
        v[j] = 0.f;
    }
    const float beta = p.beta, alpha = p.alpha;
    const int nchunks = (int)((p.L + T - 1) / T);

    auto stage = [&](int s, int c) {
        float* st = smem + s * STAGE;
        const int64_t t0 = (int64_t)c * T;
        const int rv = (int)min64(T, p.L - t0);
        stage_tile<T, DT, DT, MM_NT>(st, p.x + b * p.xs[0] + t0 * p.xs[1] + d0, p.xs[1], rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, DT, DT, MM_NT>(st + Cf::TD, p.delta + b * p.ds[0] + t0 * p.ds[1] + d0,
                                     p.ds[1], rv, dvalid_cols, p.vec, tid);
        if (p.z)
            stage_tile<T, DT, DT, MM_NT>(st + 2 * Cf::TD, p.z + b * p.zs[0] + t0 * p.zs[1] + d0,
                                         p.zs[1], rv, dvalid_cols, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 3 * Cf::TD, p.Bm + b * p.bs[0] + t0 * p.bs[1], p.bs[1],
                                   rv, N, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 3 * Cf::TD + Cf::TN, p.Cm + b * p.cs[0] + t0 * p.cs[1],
                                   p.cs[1], rv, N, p.vec, tid);
    };

    stage(0, 0);
    cp_async_commit();
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) stage((c + 1) & 1, c + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        float* st = smem + (c & 1) * STAGE;
        float* sx = st;
        float* sdt = st + Cf::TD;  // delta, converted in place to dt
        const float* sz = st + 2 * Cf::TD;
        const float* sB = st + 3 * Cf::TD;
        const float* sC = sB + Cf::TN;
        const int64_t t0 = (int64_t)c * T;
        const int Lc = (int)min64(T, p.L - t0);

        // pre-pass: dt and alpha*dt*x per (t, d)
#pragma unroll
        for (int i = tid; i < Cf::TD; i += MM_NT) {
            const int dd = i % DT;
            float r = sdt[i];
            if (p.dbias && dd < dvalid_cols) r += p.dbias[d0 + dd];
            const float dt = p.softplus ? softplus_f(r) : r;
            sdt[i] = dt;
            sdtx[i] = alpha * dt * sx[i];
        }
        __syncthreads();

        // main recurrence
        auto step = [&](int tt) {
            const float dt = sdt[tt * DT + dl];
            const float dtx = sdtx[tt * DT + dl];
            const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
            const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
            const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
            float yp = 0.f;
#pragma unroll
            for (int j = 0; j < MM_NPER; ++j) {
                const float a = ex2(dt * A2[j]);
                v[j] = fmaf(beta, v[j], dtx * bb[j]);
                h[j] = fmaf(a, h[j], v[j]);
                yp = fmaf(cc[j], h[j], yp);
            }
            yp = lane_sum<0, Cf::LOG2G>(yp);
            if (ng == 0) sy[tt * DT + dl] = yp;
        };
        auto save_ckpt = [&](int tt) {
            if (p.ckpt && dvalid) {
                const int64_t k = (t0 + tt) / MM_CK;
                float4* dst = reinterpret_cast<float4*>(p.ckpt + ckpt_base(p, b, k, d, N) +
                                                        ng * 2 * MM_NPER);
                dst[0] = make_float4(h[0], h[1], h[2], h[3]);
                dst[1] = make_float4(v[0], v[1], v[2], v[3]);
            }
        };
        if (Lc == T) {
#pragma unroll
            for (int tt = 0; tt < T; ++tt) {
                if (tt % MM_CK == 0) save_ckpt(tt);
                step(tt);
            }
        } else {
            for (int tt = 0; tt < Lc; ++tt) {
                if (tt % MM_CK == 0) save_ckpt(tt);
                step(tt);
            }
        }
        __syncthreads();

        // post-pass: out = (y + D x) * silu(z)
#pragma unroll
        for (int i = tid; i < Cf::TD; i += MM_NT) {
            const int tt = i / DT, dd = i % DT;
            if (tt < Lc && dd < dvalid_cols) {
                float y = sy[i];
                if (p.Dskip) y = fmaf(p.Dskip[d0 + dd], sx[i], y);
                if (p.z) {
                    const float zv = sz[i];
                    y *= zv * sigmoid_f(zv);
                }
                p.out[(b * p.L + t0 + tt) * p.D + d0 + dd] = y;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
template <int N>
__global__ void __launch_bounds__(MM_NT) mmscan_bwd_kernel(const MMParams p) {
    using Cf = MMCfg<N>;
    constexpr int DT = Cf::DT, G = Cf::G, T = MM_T, TD = Cf::TD;
    constexpr int LOG2DPW = 5 - Cf::LOG2G;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    // stage s: [x | delta | z | dout] (T x DT), [B | C] (T x N)
    constexpr int STAGE = 4 * TD + 2 * Cf::TN;
    float* sdt = smem + 2 * STAGE;
    float* sdtx = sdt + TD;
    float* sdy = sdtx + TD;
    float* syp = sdy + TD;   // sum_n C h (recomputed)
    float* sSA = syp + TD;   // sum_n gh h_{t-1} a A log2(e)
    float* sSB = sSA + TD;   // sum_n gv B
    float* spart = sSB + TD; // [4 warps][T][2N] partial dB | dC
    float* sred = spart + 4 * T * 2 * N;  // [2][MM_NT] final dD / dbias reduction

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ng = lane & (G - 1);
    const int dbits = lane >> Cf::LOG2G;
    const int dl = warp * Cf::DPW + dbits;
    const int64_t b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * DT;
    const int64_t d = d0 + dl;
    const bool dvalid = d < p.D;
    const int dvalid_cols = (int)min64(DT, p.D - d0);

    float A2[MM_NPER], gh[MM_NPER], gv[MM_NPER], anext[MM_NPER], dAacc[MM_NPER];
#pragma unroll
    for (int j = 0; j < MM_NPER; ++j) {
        A2[j] = dvalid ? p.A[d * N + ng * MM_NPER + j] * MMB_LOG2E : 0.f;
        gh[j] = gv[j] = anext[j] = dAacc[j] = 0.f;
    }
    float accD = 0.f, accBias = 0.f;  // for channel d0 + tid % DT (post-pass ownership)
    const float beta = p.beta, alpha = p.alpha;
    const int nchunks = (int)((p.L + T - 1) / T);

    auto stage = [&](int s, int c) {
        float* st = smem + s * STAGE;
        const int64_t t0 = (int64_t)c * T;
        const int rv = (int)min64(T, p.L - t0);
        stage_tile<T, DT, DT, MM_NT>(st, p.x + b * p.xs[0] + t0 * p.xs[1] + d0, p.xs[1], rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, DT, DT, MM_NT>(st + TD, p.delta + b * p.ds[0] + t0 * p.ds[1] + d0, p.ds[1],
                                     rv, dvalid_cols, p.vec, tid);
        if (p.z)
            stage_tile<T, DT, DT, MM_NT>(st + 2 * TD, p.z + b * p.zs[0] + t0 * p.zs[1] + d0,
                                         p.zs[1], rv, dvalid_cols, p.vec, tid);
        stage_tile<T, DT, DT, MM_NT>(st + 3 * TD, p.dout + (b * p.L + t0) * p.D + d0, p.D, rv,
                                     dvalid_cols, p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 4 * TD, p.Bm + b * p.bs[0] + t0 * p.bs[1], p.bs[1], rv, N,
                                   p.vec, tid);
        stage_tile<T, N, N, MM_NT>(st + 4 * TD + Cf::TN, p.Cm + b * p.cs[0] + t0 * p.cs[1],
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
        const float* sdr = st + TD;
        const float* sz = st + 2 * TD;
        const float* sdo = st + 3 * TD;
        const float* sB = st + 4 * TD;
        const float* sC = sB + Cf::TN;
        const int64_t t0 = (int64_t)c * T;
        const int Lc = (int)min64(T, p.L - t0);

        // pre-pass: dt, alpha*dt*x, dy = dout * silu(z)
#pragma unroll
        for (int i = tid; i < TD; i += MM_NT) {
            const int dd = i % DT;
            float r = sdr[i];
            if (p.dbias && dd < dvalid_cols) r += p.dbias[d0 + dd];
            const float dt = p.softplus ? softplus_f(r) : r;
            sdt[i] = dt;
            sdtx[i] = alpha * dt * sx[i];
            float dy = sdo[i];
            if (p.z) {
                const float zv = sz[i];
                dy *= zv * sigmoid_f(zv);
            }
            sdy[i] = dy;
        }
        __syncthreads();

        // 8-step windows, last first
        for (int sub = (Lc - 1) / MM_CK; sub >= 0; --sub) {
            float h[MM_NPER], v[MM_NPER];
            {
                const int64_t k = (t0 + sub * MM_CK) / MM_CK;
                if (dvalid) {
                    const float4* src = reinterpret_cast<const float4*>(
                        p.ckpt_in + ckpt_base(p, b, k, d, N) + ng * 2 * MM_NPER);
                    const float4 h4 = src[0], v4 = src[1];
                    h[0] = h4.x; h[1] = h4.y; h[2] = h4.z; h[3] = h4.w;
                    v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
                } else {
#pragma unroll
                    for (int j = 0; j < MM_NPER; ++j) h[j] = v[j] = 0.f;
                }
            }
            float aa[MM_CK][MM_NPER], hh[MM_CK + 1][MM_NPER];
#pragma unroll
            for (int j = 0; j < MM_NPER; ++j) hh[0][j] = h[j];
            // forward replay of the window (steps past the end see zero input
            // and never reach an output)
#pragma unroll
            for (int s = 0; s < MM_CK; ++s) {
                const int tt = sub * MM_CK + s;
                const float dt = sdt[tt * DT + dl];
                const float dtx = sdtx[tt * DT + dl];
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
                const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
                const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
                float yp = 0.f;
#pragma unroll
                for (int j = 0; j < MM_NPER; ++j) {
                    const float a = ex2(dt * A2[j]);
                    v[j] = fmaf(beta, v[j], dtx * bb[j]);
                    h[j] = fmaf(a, h[j], v[j]);
                    aa[s][j] = a;
                    hh[s + 1][j] = h[j];
                    yp = fmaf(cc[j], h[j], yp);
                }
                yp = lane_sum<0, Cf::LOG2G>(yp);
                if (ng == 0) syp[tt * DT + dl] = yp;
            }
            // adjoint sweep of the window
#pragma unroll
            for (int s = MM_CK - 1; s >= 0; --s) {
                const int tt = sub * MM_CK + s;
                const float dy = sdy[tt * DT + dl];
                const float dt = sdt[tt * DT + dl];
                const float dtx = sdtx[tt * DT + dl];
                const float4 b4 = *reinterpret_cast<const float4*>(sB + tt * N + ng * MM_NPER);
                const float4 c4 = *reinterpret_cast<const float4*>(sC + tt * N + ng * MM_NPER);
                const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
                float SA = 0.f, SB = 0.f;
                float vals[2 * MM_NPER];
#pragma unroll
                for (int j = 0; j < MM_NPER; ++j) {
                    gh[j] = fmaf(anext[j], gh[j], dy * cc[j]);
                    gv[j] = fmaf(beta, gv[j], gh[j]);
                    SB = fmaf(gv[j], bb[j], SB);
                    const float t2 = gh[j] * hh[s][j] * aa[s][j];
                    SA = fmaf(t2, A2[j], SA);
                    dAacc[j] = fmaf(t2, dt, dAacc[j]);
                    vals[j] = gv[j] * dtx;
                    vals[MM_NPER + j] = dy * hh[s + 1][j];
                    anext[j] = aa[s][j];
                }
                // d-sum of the dB | dC contributions over this warp's channels
                reduce_scatter<2 * MM_NPER, Cf::LOG2G, LOG2DPW>(vals, lane);
                constexpr int KEEP = (2 * MM_NPER >> LOG2DPW) > 0 ? (2 * MM_NPER >> LOG2DPW) : 1;
                constexpr int USED_BITS = LOG2DPW < 3 ? LOG2DPW : 3;  // log2(2 * MM_NPER) = 3
                if ((dbits >> USED_BITS) == 0) {
#pragma unroll
                    for (int i = 0; i < KEEP; ++i) {
                        const int idx = rs_index<2 * MM_NPER, LOG2DPW>(dbits, i);
                        const int kind = idx / MM_NPER, n = ng * MM_NPER + idx % MM_NPER;
                        spart[(warp * T + tt) * 2 * N + kind * N + n] = vals[i];
                    }
                }
                // n-sums for dx and ddelta
                float s2[2] = {SA, SB};
                reduce_scatter<2, 0, Cf::LOG2G>(s2, lane);
                if (ng < 2) (ng == 0 ? sSA : sSB)[tt * DT + dl] = s2[0];
            }
        }
        __syncthreads();

        // post-pass per (t, d): dx, ddelta, dz; running dD / dbias
#pragma unroll
        for (int i = tid; i < TD; i += MM_NT) {
            const int tt = i / DT, dd = i % DT;
            if (tt < Lc && dd < dvalid_cols) {
                const int64_t gi = (b * p.L + t0 + tt) * p.D + d0 + dd;
                const float xv = sx[i];
                const float dt = sdt[i];
                const float SB = sSB[i];
                const float dy = sdy[i];
                float yp = syp[i];
                float gx = alpha * dt * SB;
                if (p.Dskip) {
                    const float Dv = p.Dskip[d0 + dd];
                    gx = fmaf(dy, Dv, gx);
                    yp = fmaf(Dv, xv, yp);
                }
                if (p.z) {
                    const float zv = sz[i];
                    const float sg = sigmoid_f(zv);
                    if (p.dz) p.dz[gi] = sdo[i] * yp * sg * (1.f + zv * (1.f - sg));
                }
                float gdt = fmaf(alpha * xv, SB, sSA[i] * MMB_LN2);
                if (p.softplus) {
                    const float r = sdr[i] + (p.dbias ? p.dbias[d0 + dd] : 0.f);
                    if (r <= 20.f) gdt *= sigmoid_f(r);
                }
                p.dx[gi] = gx;
                p.ddelta[gi] = gdt;
                accD = fmaf(dy, xv, accD);
                accBias += gdt;
            }
        }
        // dB | dC of this chunk: sum the warps' partials, add to global
        for (int f = tid; f < T * 2 * N / 4; f += MM_NT) {
            const int tt = (f * 4) / (2 * N), q = (f * 4) % (2 * N);
            if (tt < Lc) {
                float4 acc = *reinterpret_cast<const float4*>(spart + tt * 2 * N + q);
#pragma unroll
                for (int w = 1; w < 4; ++w) {
                    const float4 o = *reinterpret_cast<const float4*>(spart + (w * T + tt) * 2 * N + q);
                    acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w;
                }
                float* dst = (q < N ? p.dB : p.dC) + (b * p.L + t0 + tt) * N + (q % N);
                red_add_v4(dst, acc.x, acc.y, acc.z, acc.w);
            }
        }
        __syncthreads();
    }

    // dA: this thread's 4 states of channel d, summed over its sequence
    if (dvalid) {
#pragma unroll
        for (int j = 0; j < MM_NPER; ++j) atomicAdd(p.dA + d * N + ng * MM_NPER + j, dAacc[j]);
    }
    // dD, dbias: reduce the MM_NT/DT threads that own each channel
    sred[tid] = accD;
    sred[MM_NT + tid] = accBias;
    __syncthreads();
    if (tid < DT && tid < dvalid_cols) {
        float sD = 0.f, sb = 0.f;
        for (int r = tid; r < MM_NT; r += DT) {
            sD += sred[r];
            sb += sred[MM_NT + r];
        }
        if (p.dD) atomicAdd(p.dD + d0 + tid, sD);
        if (p.ddbias) atomicAdd(p.ddbias + d0 + tid, sb);
    }
}

template <int N>
size_t fwd_smem_bytes() {
    using Cf = MMCfg<N>;
    return sizeof(float) * (2 * (3 * Cf::TD + 2 * Cf::TN) + 2 * Cf::TD);
}

template <int N>
size_t bwd_smem_bytes() {
    using Cf = MMCfg<N>;
    return sizeof(float) *
           (2 * (4 * Cf::TD + 2 * Cf::TN) + 6 * Cf::TD + 4 * MM_T * 2 * N + 2 * MM_NT);
}

template <int N>
int launch_fwd(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N>;
    const size_t smem = fwd_smem_bytes<N>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_fwd_kernel<N>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_fwd_kernel<N><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
}

template <int N>
int launch_bwd(const MMParams& p, cudaStream_t stream) {
    using Cf = MMCfg<N>;
    const size_t smem = bwd_smem_bytes<N>();
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st = mmb_smem_attr(mmscan_bwd_kernel<N>, smem, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.D + Cf::DT - 1) / Cf::DT), (unsigned)p.Bsz);
    mmscan_bwd_kernel<N><<<grid, MM_NT, smem, stream>>>(p);
    return mmb_launch_status();
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
