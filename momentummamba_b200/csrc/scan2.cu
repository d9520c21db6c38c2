// 2x2 linear scans (LinOSS), sm_100a.
//
//   x_t = M_t x_{t-1} + F_t ,   x = (x1, x2) per (b, p) chain, x_{-1} = 0,
//
// with M_t a real 2x2 matrix and F_t real or complex.  Every chain has length L;
// to fill the GPU the sequence is cut into C chunks of T steps and scanned in
// three passes, none of which waits on another CTA:
//   1. chunk summaries   one thread per (b, chunk, p): the chunk's state from
//                        zero and its matrix product
//   2. carries           one thread per (b, p): compose the C summaries in order
//   3. final pass        one thread per (b, chunk, p): rerun the chunk from its
//                        carry and write the outputs
// The backward is the same structure run in reverse on the adjoint
//   lambda_t = gX_t + M_{t+1}^T lambda_{t+1},   dF_t = lambda_t,
//   dM_t = sum over channels of lambda_t (x) x_{t-1}.
// Threads of a warp take consecutive p, so for P >= 32 every load of a step is a
// coalesced row.
//
// Two entry families:
//   mmb_scan2_*    generic: M per (b, t, p) from memory, optional running product
//                  Mscan (the "A_scan" the reference returns) and its gradient.
//   mmb_linoss_*   LinOSS layer: M and F = (f1 Bu, f2 Bu) built in registers from
//                  A_diag, step (IM or IMEX) and Bu; the forward also keeps
//                  (x1, x2) every 8 steps so the backward can rebuild x_{t-1}.
#include <mutex>

#include "mmb_common.cuh"

namespace mmb {

constexpr int S2_NT = 256;
constexpr int S2_CK = 8;  // LinOSS checkpoint interval

struct Mat2 {
    float a, b, c, d;  // [[a, b], [c, d]]
};
__device__ __forceinline__ Mat2 mmul(const Mat2& x, const Mat2& y) {
    return {x.a * y.a + x.b * y.c, x.a * y.b + x.b * y.d, x.c * y.a + x.d * y.c,
            x.c * y.b + x.d * y.d};
}
__device__ __forceinline__ Mat2 mtrans(const Mat2& x) { return {x.a, x.c, x.b, x.d}; }
__device__ __forceinline__ Mat2 mident() { return {1.f, 0.f, 0.f, 1.f}; }
__device__ __forceinline__ void mvec(const Mat2& m, float& u, float& v) {
    const float nu = m.a * u + m.b * v;
    const float nv = m.c * u + m.d * v;
    u = nu;
    v = nv;
}

// Host-side chunking: MMB_S2_THREADS_PER_SM (b, chunk, p) threads per SM, chunks
// of at least 16 steps.  1024 rather than the 2048 an SM can hold: the LinOSS
// backward's final pass keeps 512 threads per SM resident, and with half as
// many, twice as long chunks it runs in two waves instead of four, each thread
// amortising its first window's load over 14 windows instead of 7 (B=16
// L=4096 P=256: backward 165 -> 140 us per call, forward unchanged; 512
// threads per SM made the forward passes slower).
#ifndef MMB_S2_THREADS_PER_SM
#define MMB_S2_THREADS_PER_SM 1024
#endif
static void s2_chunks(int64_t Bsz, int64_t L, int64_t P, int64_t& T, int64_t& C) {
    const int64_t target = 148 * MMB_S2_THREADS_PER_SM;
    int64_t chains = Bsz * P;
    int64_t want = (target + chains - 1) / chains;
    int64_t maxc = (L + 15) / 16;
    if (want < 1) want = 1;
    if (want > maxc) want = maxc;
    T = (L + want - 1) / want;
    C = (L + T - 1) / T;
}

// ---------------------------------------------------------------------------
// generic scan: layout helpers
// ---------------------------------------------------------------------------
struct S2Params {
    int64_t Bsz, L, P, T, C;
    int nc;  // components per F entry: 1 real, 2 complex
    const float *M, *F, *X, *gX, *Mscan_in, *gMs;
    float *Mscan, *Xo, *dM, *dF;
    float* work;
};

__device__ __forceinline__ int64_t m_off(const S2Params& p, int64_t b, int64_t t, int k, int64_t j) {
    return ((b * p.L + t) * 4 + k) * p.P + j;
}
__device__ __forceinline__ int64_t f_off(const S2Params& p, int64_t b, int64_t t, int row,
                                         int64_t j, int comp) {
    return (((b * p.L + t) * 2 + row) * p.P + j) * p.nc + comp;
}
__device__ __forceinline__ Mat2 load_m(const S2Params& p, int64_t b, int64_t t, int64_t j) {
    return {__ldg(p.M + m_off(p, b, t, 0, j)), __ldg(p.M + m_off(p, b, t, 1, j)),
            __ldg(p.M + m_off(p, b, t, 2, j)), __ldg(p.M + m_off(p, b, t, 3, j))};
}

// work layout (floats), per (b, chunk, p) record:
//   forward summary  : Mprod(4), x_loc(2*nc)
//   forward carry    : Mpre(4), x_in(2*nc)
constexpr int S2_REC = 8;  // floats per (b, chunk, p) record of each table (2*nc <= 4)

// ---------------------------------------------------------------------------
// generic forward
// ---------------------------------------------------------------------------
// The time loops work in windows of S2_W steps: a window's inputs are loaded
// before its dependent recurrence and stores (which would otherwise hold
// every later load behind them); the carry passes prefetch S2_W chunk records.
constexpr int S2_W = 4;

template <int NC, bool MSCAN>
__global__ void __launch_bounds__(S2_NT) s2_fwd_summary(const S2Params p) {
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= p.Bsz * p.C * p.P) return;
    const int64_t j = idx % p.P, bc = idx / p.P, c = bc % p.C, b = bc / p.C;
    const int64_t t0 = c * p.T, t1 = min64(p.L, t0 + p.T);
    float x1[NC], x2[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) x1[k] = x2[k] = 0.f;
    Mat2 mp = mident();
    for (int64_t t = t0; t < t1; ++t) {
        const Mat2 m = load_m(p, b, t, j);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const float f1 = __ldg(p.F + f_off(p, b, t, 0, j, k));
            const float f2 = __ldg(p.F + f_off(p, b, t, 1, j, k));
            const float n1 = m.a * x1[k] + m.b * x2[k] + f1;
            const float n2 = m.c * x1[k] + m.d * x2[k] + f2;
            x1[k] = n1;
            x2[k] = n2;
        }
        mp = mmul(m, mp);
    }
    float* rec = p.work + idx * S2_REC;
    rec[0] = mp.a; rec[1] = mp.b; rec[2] = mp.c; rec[3] = mp.d;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        rec[4 + 2 * k] = x1[k];
        rec[5 + 2 * k] = x2[k];
    }
}

// Per (b, p) chain: the state entering each chunk and (MSCAN) the product of
// the earlier chunks' matrices.  Chunk c's map is x -> Mprod_c x + x_loc_c; a
// warp composes 32 consecutive chunks' maps with a shuffle scan.
template <int NC, bool MSCAN>
__global__ void __launch_bounds__(S2_NT) s2_fwd_carry(const S2Params p) {
    const int64_t chain = (int64_t)blockIdx.x * (S2_NT / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (chain >= p.Bsz * p.P) return;  // whole warps
    const int64_t j = chain % p.P, b = chain / p.P;
    const float* __restrict__ summ = p.work;
    float* __restrict__ carry = p.work + p.Bsz * p.C * p.P * S2_REC;
    Aff2<Mat2> in = {mident(), 0.f, 0.f, 0.f, 0.f};
    for (int64_t c0 = 0; c0 < p.C; c0 += 32) {
        const int64_t c = c0 + lane;
        Aff2<Mat2> v = {mident(), 0.f, 0.f, 0.f, 0.f};
        const int64_t rec = ((b * p.C + c) * p.P + j) * S2_REC;
        if (c < p.C) {  // record: [Mprod | x1, x2 (real) | x1, x2 (imaginary)]
            const float4 sm = reinterpret_cast<const float4*>(summ + rec)[0];
            const float4 sx = reinterpret_cast<const float4*>(summ + rec)[1];
            v = {{sm.x, sm.y, sm.z, sm.w}, sx.x, NC > 1 ? sx.z : 0.f, sx.y, NC > 1 ? sx.w : 0.f};
        }
        Aff2<Mat2> ex;
        in = warp_aff2_exscan(v, in, lane, ex);
        if (c < p.C) {
            float4* out = reinterpret_cast<float4*>(carry + rec);
            out[0] = MSCAN ? make_float4(ex.m.a, ex.m.b, ex.m.c, ex.m.d)
                           : make_float4(1.f, 0.f, 0.f, 1.f);
            out[1] = make_float4(ex.x1r, ex.x2r, NC > 1 ? ex.x1i : 0.f, NC > 1 ? ex.x2i : 0.f);
        }
    }
}

template <int NC, bool MSCAN>
__global__ void __launch_bounds__(S2_NT) s2_fwd_final(const S2Params p) {
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= p.Bsz * p.C * p.P) return;
    const int64_t j = idx % p.P, bc = idx / p.P, c = bc % p.C, b = bc / p.C;
    const int64_t t0 = c * p.T, t1 = min64(p.L, t0 + p.T);
    const float* in = p.work + p.Bsz * p.C * p.P * S2_REC + idx * S2_REC;
    Mat2 mp = {in[0], in[1], in[2], in[3]};
    float x1[NC], x2[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        x1[k] = in[4 + 2 * k];
        x2[k] = in[5 + 2 * k];
    }
    for (int64_t t = t0; t < t1; ++t) {
        const Mat2 m = load_m(p, b, t, j);
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            const float f1 = __ldg(p.F + f_off(p, b, t, 0, j, k));
            const float f2 = __ldg(p.F + f_off(p, b, t, 1, j, k));
            const float n1 = m.a * x1[k] + m.b * x2[k] + f1;
            const float n2 = m.c * x1[k] + m.d * x2[k] + f2;
            x1[k] = n1;
            x2[k] = n2;
            p.Xo[f_off(p, b, t, 0, j, k)] = n1;
            p.Xo[f_off(p, b, t, 1, j, k)] = n2;
        }
        if (MSCAN) {
            mp = mmul(m, mp);
            p.Mscan[m_off(p, b, t, 0, j)] = mp.a;
            p.Mscan[m_off(p, b, t, 1, j)] = mp.b;
            p.Mscan[m_off(p, b, t, 2, j)] = mp.c;
            p.Mscan[m_off(p, b, t, 3, j)] = mp.d;
        }
    }
}

// ---------------------------------------------------------------------------
// generic backward.  Vector channels: NC for x (re, im) and, with GMS, the two
// columns of the adjoint of the running product.
// work layout per (b, chunk, p): summary [lam(2*NV), Q(4), M_t0(4)], then mu(2*NV)
// ---------------------------------------------------------------------------
template <int NC, bool GMS>
struct S2B {
    static constexpr int NV = NC + (GMS ? 2 : 0);
    static constexpr int SREC = 2 * NV + 8;
    static constexpr int MREC = 2 * NV;
};

template <int NC, bool GMS>
__device__ __forceinline__ void s2_gvec(const S2Params& p, int64_t b, int64_t t, int64_t j,
                                        float (&g1)[S2B<NC, GMS>::NV],
                                        float (&g2)[S2B<NC, GMS>::NV]) {
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        g1[k] = p.gX ? __ldg(p.gX + f_off(p, b, t, 0, j, k)) : 0.f;
        g2[k] = p.gX ? __ldg(p.gX + f_off(p, b, t, 1, j, k)) : 0.f;
    }
    if (GMS) {
        // column q of the running-product adjoint: (gMs[0][q], gMs[1][q])
        g1[NC] = __ldg(p.gMs + m_off(p, b, t, 0, j));
        g2[NC] = __ldg(p.gMs + m_off(p, b, t, 2, j));
        g1[NC + 1] = __ldg(p.gMs + m_off(p, b, t, 1, j));
        g2[NC + 1] = __ldg(p.gMs + m_off(p, b, t, 3, j));
    }
}

template <int NC, bool GMS>
__global__ void __launch_bounds__(S2_NT) s2_bwd_summary(const S2Params p) {
    using Q = S2B<NC, GMS>;
    constexpr int NV = Q::NV;
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= p.Bsz * p.C * p.P) return;
    const int64_t j = idx % p.P, bc = idx / p.P, c = bc % p.C, b = bc / p.C;
    const int64_t t0 = c * p.T, t1 = min64(p.L, t0 + p.T);
    float l1[NV], l2[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) l1[k] = l2[k] = 0.f;
    Mat2 q = mident();  // M_{t+1}^T ... M_{t1-1}^T
    Mat2 mn = {0.f, 0.f, 0.f, 0.f};  // M_{t+1}; none past the chunk end
    for (int64_t te = t1; te > t0; te -= S2_W) {  // window [te - S2_W, te)
        float g1[S2_W][NV], g2[S2_W][NV];
        Mat2 mw[S2_W];
#pragma unroll
        for (int s = 0; s < S2_W; ++s) {
            const int64_t t = te - 1 - s;
            if (t >= t0) {
                s2_gvec<NC, GMS>(p, b, t, j, g1[s], g2[s]);
                mw[s] = load_m(p, b, t, j);
            }
        }
#pragma unroll
        for (int s = 0; s < S2_W; ++s) {
            const int64_t t = te - 1 - s;
            if (t < t0) break;
            const Mat2 mt = mtrans(mn);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                float a = l1[k], bb = l2[k];
                mvec(mt, a, bb);
                l1[k] = a + g1[s][k];
                l2[k] = bb + g2[s][k];
            }
            if (t > t0) q = mmul(mtrans(mw[s]), q);
            mn = mw[s];
        }
    }
    float* rec = p.work + idx * Q::SREC;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        rec[2 * k] = l1[k];
        rec[2 * k + 1] = l2[k];
    }
    rec[2 * NV + 0] = q.a; rec[2 * NV + 1] = q.b; rec[2 * NV + 2] = q.c; rec[2 * NV + 3] = q.d;
    rec[2 * NV + 4] = mn.a; rec[2 * NV + 5] = mn.b; rec[2 * NV + 6] = mn.c; rec[2 * NV + 7] = mn.d;
}

template <int NC, bool GMS>
__global__ void __launch_bounds__(S2_NT) s2_bwd_carry(const S2Params p) {
    using Q = S2B<NC, GMS>;
    constexpr int NV = Q::NV;
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= p.Bsz * p.P) return;
    const int64_t j = idx % p.P, b = idx / p.P;
    float m1[NV], m2[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) m1[k] = m2[k] = 0.f;
    const float* __restrict__ summ = p.work;
    float* __restrict__ mu = p.work + p.Bsz * p.C * p.P * Q::SREC;
    for (int64_t c0 = p.C - 1; c0 >= 0; c0 -= S2_W) {
        float rs[S2_W][Q::SREC];
#pragma unroll
        for (int i = 0; i < S2_W; ++i) {  // records before the start: chunk 0 again (unused)
            const int64_t ci = c0 - i >= 0 ? c0 - i : 0;
            const float* s = summ + ((b * p.C + ci) * p.P + j) * Q::SREC;
#pragma unroll
            for (int e = 0; e < Q::SREC; ++e) rs[i][e] = s[e];
        }
#pragma unroll
        for (int i = 0; i < S2_W; ++i) {
            if (c0 - i < 0) break;
            float* out = mu + ((b * p.C + c0 - i) * p.P + j) * Q::MREC;
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                out[2 * k] = m1[k];
                out[2 * k + 1] = m2[k];
            }
            const float* s = rs[i];
            const Mat2 q = {s[2 * NV], s[2 * NV + 1], s[2 * NV + 2], s[2 * NV + 3]};
            const Mat2 mt0 = mtrans(Mat2{s[2 * NV + 4], s[2 * NV + 5], s[2 * NV + 6], s[2 * NV + 7]});
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                float a = m1[k], bb = m2[k];
                mvec(q, a, bb);
                a += s[2 * k];
                bb += s[2 * k + 1];
                mvec(mt0, a, bb);  // mu for the previous chunk
                m1[k] = a;
                m2[k] = bb;
            }
        }
    }
}

template <int NC, bool GMS>
__global__ void __launch_bounds__(S2_NT) s2_bwd_final(const S2Params p) {
    using Q = S2B<NC, GMS>;
    constexpr int NV = Q::NV;
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= p.Bsz * p.C * p.P) return;
    const int64_t j = idx % p.P, bc = idx / p.P, c = bc % p.C, b = bc / p.C;
    const int64_t t0 = c * p.T, t1 = min64(p.L, t0 + p.T);
    const float* mu = p.work + p.Bsz * p.C * p.P * Q::SREC + idx * Q::MREC;
    float l1[NV], l2[NV];  // holds M_{t+1}^T lambda_{t+1} before step t
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        l1[k] = mu[2 * k];
        l2[k] = mu[2 * k + 1];
    }
    for (int64_t te = t1; te > t0; te -= S2_W) {  // window [te - S2_W, te), backwards
        float g1[S2_W][NV], g2[S2_W][NV];
        float xp1[S2_W][NC], xp2[S2_W][NC];  // state before the step
        Mat2 mw[S2_W], pcw[S2_W];
#pragma unroll
        for (int s = 0; s < S2_W; ++s) {
            const int64_t t = te - 1 - s;
            if (t < t0) continue;
            s2_gvec<NC, GMS>(p, b, t, j, g1[s], g2[s]);
            mw[s] = load_m(p, b, t, j);
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                xp1[s][k] = t > 0 ? __ldg(p.X + f_off(p, b, t - 1, 0, j, k)) : 0.f;
                xp2[s][k] = t > 0 ? __ldg(p.X + f_off(p, b, t - 1, 1, j, k)) : 0.f;
            }
            if (GMS) {
                pcw[s] = mident();  // Mc_{t-1}; identity before the first step
                if (t > 0)
                    pcw[s] = {__ldg(p.Mscan_in + m_off(p, b, t - 1, 0, j)),
                              __ldg(p.Mscan_in + m_off(p, b, t - 1, 1, j)),
                              __ldg(p.Mscan_in + m_off(p, b, t - 1, 2, j)),
                              __ldg(p.Mscan_in + m_off(p, b, t - 1, 3, j))};
            }
        }
#pragma unroll
        for (int s = 0; s < S2_W; ++s) {
            const int64_t t = te - 1 - s;
            if (t < t0) break;
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                l1[k] += g1[s][k];
                l2[k] += g2[s][k];
            }
            // dF_t = lambda_t ; dM_t = sum over channels lambda_t (x) state_{t-1}
            float d11 = 0.f, d12 = 0.f, d21 = 0.f, d22 = 0.f;
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                p.dF[f_off(p, b, t, 0, j, k)] = l1[k];
                p.dF[f_off(p, b, t, 1, j, k)] = l2[k];
                d11 += l1[k] * xp1[s][k]; d12 += l1[k] * xp2[s][k];
                d21 += l2[k] * xp1[s][k]; d22 += l2[k] * xp2[s][k];
            }
            if (GMS) {
                const Mat2& pc = pcw[s];
                // column q of the adjoint pairs with column q of Mc_{t-1}
                d11 += l1[NC] * pc.a + l1[NC + 1] * pc.b;
                d12 += l1[NC] * pc.c + l1[NC + 1] * pc.d;
                d21 += l2[NC] * pc.a + l2[NC + 1] * pc.b;
                d22 += l2[NC] * pc.c + l2[NC + 1] * pc.d;
            }
            p.dM[m_off(p, b, t, 0, j)] = d11;
            p.dM[m_off(p, b, t, 1, j)] = d12;
            p.dM[m_off(p, b, t, 2, j)] = d21;
            p.dM[m_off(p, b, t, 3, j)] = d22;
            // carry M_t^T lambda_t to step t - 1
            const Mat2 mt = mtrans(mw[s]);
#pragma unroll
            for (int k = 0; k < NV; ++k) mvec(mt, l1[k], l2[k]);
        }
    }
}

// ---------------------------------------------------------------------------
// LinOSS layer: time-invariant M per oscillator, F = (f1 Bu, f2 Bu), Bu complex
// ---------------------------------------------------------------------------
struct LinParams {
    int64_t Bsz, L, P, T, C, K;  // K = checkpoints per chain (ceil(L / 8))
    int disc;                    // 0 IM, 1 IMEX
    const float *A, *step, *Bu, *dx2;
    float *x2, *dBu, *dA, *dstep;
    float* work;
};

struct LinCoef {
    Mat2 m;
    float f1, f2;
};

// IM:   S = 1/(1 + s^2 A); M = [[1 - s^2 A S, -s A S], [s S, S]]; f = (M11 s, M21 s)
// IMEX: M = [[1, -s A], [s, 1 - s^2 A]]; f = (s, s^2)
// (LinOSS_pytorch.py:164-178 and :209-222)
__device__ __forceinline__ LinCoef lin_coef(int disc, float A, float s) {
    LinCoef k;
    if (disc == 0) {
        const float S = 1.f / (1.f + s * s * A);
        k.m = {1.f - s * s * A * S, -s * A * S, s * S, S};
        k.f1 = k.m.a * s;
        k.f2 = k.m.c * s;
    } else {
        k.m = {1.f, -s * A, s, 1.f - s * s * A};
        k.f1 = s;
        k.f2 = s * s;
    }
    return k;
}

// work layout (floats):
//   ckpt  : Bsz * K * P * 4          (x1re, x1im, x2re, x2im every 8 steps)
//   summ  : Bsz * C * P * 4          (chunk state from zero / chunk adjoint from zero)
//   carry : Bsz * C * P * 4          (state entering / adjoint leaving each chunk)
//   grad  : P * 8                    (dM11, dM12, dM21, dM22, df1, df2 accumulators)
__device__ __forceinline__ float* lin_ckpt(const LinParams& q) { return q.work; }
__device__ __forceinline__ float* lin_summ(const LinParams& q) {
    return q.work + q.Bsz * q.K * q.P * 4;
}
__device__ __forceinline__ float* lin_carry(const LinParams& q) {
    return lin_summ(q) + q.Bsz * q.C * q.P * 4;
}
__device__ __forceinline__ float* lin_grad(const LinParams& q) {
    return lin_carry(q) + q.Bsz * q.C * q.P * 4;
}

__device__ __forceinline__ float2 ld_bu(const float* base, int64_t Bsz, int64_t L, int64_t P,
                                        int64_t b, int64_t t, int64_t j) {
    return __ldg(reinterpret_cast<const float2*>(base) + (b * L + t) * P + j);
}

// The time loops below work in 8-step windows: a window's inputs are loaded
// into registers before its dependent recurrence runs (the stores of a window
// would otherwise pin every later load behind them), and the carry passes
// prefetch 8 chunk records at a time.
__device__ __forceinline__ void lin_step(const LinCoef& k, float2 u, float& x1r, float& x1i,
                                         float& x2r, float& x2i) {
    const float n1r = k.m.a * x1r + k.m.b * x2r + k.f1 * u.x;
    const float n1i = k.m.a * x1i + k.m.b * x2i + k.f1 * u.y;
    const float n2r = k.m.c * x1r + k.m.d * x2r + k.f2 * u.x;
    const float n2i = k.m.c * x1i + k.m.d * x2i + k.f2 * u.y;
    x1r = n1r; x1i = n1i; x2r = n2r; x2i = n2i;
}

// the window [ws, ws + 8) of a chain's (B, L, P) complex sequence, zeros past t1
__device__ __forceinline__ void lin_load_window(const float* __restrict__ base, const LinParams& q,
                                                int64_t b, int64_t ws, int64_t t1, int64_t j,
                                                float2 (&u)[S2_CK]) {
    const float2* r = reinterpret_cast<const float2*>(base) + (b * q.L + ws) * q.P + j;
#pragma unroll
    for (int s = 0; s < S2_CK; ++s) {  // steps past t1 read step ws (in range) and drop it
        const float2 v = __ldg(r + (ws + s < t1 ? s : 0) * q.P);
        u[s] = ws + s < t1 ? v : make_float2(0.f, 0.f);
    }
}

__global__ void __launch_bounds__(S2_NT) lin_fwd_summary(const LinParams q) {
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.P) return;
    const int64_t j = idx % q.P, bc = idx / q.P, c = bc % q.C, b = bc / q.C;
    const int64_t t0 = c * q.T, t1 = min64(q.L, t0 + q.T);
    const LinCoef k = lin_coef(q.disc, q.A[j], q.step[j]);
    float x1r = 0.f, x1i = 0.f, x2r = 0.f, x2i = 0.f;
    // the next window's loads are issued before this window's recurrence
    float2 u[S2_CK], un[S2_CK];
    lin_load_window(q.Bu, q, b, t0, t1, j, u);
    for (int64_t ws = t0; ws < t1; ws += S2_CK) {
        if (ws + S2_CK < t1) lin_load_window(q.Bu, q, b, ws + S2_CK, t1, j, un);
#pragma unroll
        for (int s = 0; s < S2_CK; ++s)
            if (ws + s < t1) lin_step(k, u[s], x1r, x1i, x2r, x2i);
#pragma unroll
        for (int s = 0; s < S2_CK; ++s) u[s] = un[s];
    }
    reinterpret_cast<float4*>(lin_summ(q))[idx] = make_float4(x1r, x1i, x2r, x2i);
}

// ---------------------------------------------------------------------------
// Chunk carries of the LinOSS layer.  The transition is the same every step,
// so across chunks the carry follows x_{c+1} = K x_c + w_c with one constant K
// (a power of M); a warp takes 32 consecutive chunks of a chain and scans them
// with shuffles (Hillis-Steele, weights K^(2^k)), instead of one thread walking
// every chunk of its chain.
// ---------------------------------------------------------------------------
struct Cv2 {  // complex 2-vector (x1, x2)
    float x1r, x1i, x2r, x2i;
};
__device__ __forceinline__ void cv_mul(const Mat2& m, Cv2& v) {
    mvec(m, v.x1r, v.x2r);
    mvec(m, v.x1i, v.x2i);
}
__device__ __forceinline__ Cv2 cv_add(const Cv2& a, const Cv2& b) {
    return {a.x1r + b.x1r, a.x1i + b.x1i, a.x2r + b.x2r, a.x2i + b.x2i};
}
__device__ __forceinline__ Cv2 cv_shfl_up(const Cv2& v, int d) {
    return {__shfl_up_sync(0xffffffffu, v.x1r, d), __shfl_up_sync(0xffffffffu, v.x1i, d),
            __shfl_up_sync(0xffffffffu, v.x2r, d), __shfl_up_sync(0xffffffffu, v.x2i, d)};
}
__device__ __forceinline__ Cv2 cv_shfl(const Cv2& v, int src) {
    return {__shfl_sync(0xffffffffu, v.x1r, src), __shfl_sync(0xffffffffu, v.x1i, src),
            __shfl_sync(0xffffffffu, v.x2r, src), __shfl_sync(0xffffffffu, v.x2i, src)};
}
__device__ __forceinline__ Mat2 mpow(Mat2 m, int64_t e) {
    Mat2 r = mident();
    while (e > 0) {
        if (e & 1) r = mmul(m, r);
        m = mmul(m, m);
        e >>= 1;
    }
    return r;
}

// Exclusive scan over the warp's lanes of x_{l+1} = K x_l + w_l from x_0 = xin,
// with Kp[k] = K^(2^k) (k = 0..5) and Kl = K^lane: lane l receives x_l in
// `excl`; every lane gets x_32 back.
__device__ __forceinline__ Cv2 warp_carry_scan(const Mat2 (&Kp)[6], const Mat2& Kl, Cv2 w,
                                               const Cv2& xin, int lane, Cv2& excl) {
#pragma unroll
    for (int k = 0; k < 5; ++k) {  // w_l <- sum_{i <= l} K^(l - i) w_i
        Cv2 o = cv_shfl_up(w, 1 << k);
        cv_mul(Kp[k], o);
        if (lane >= (1 << k)) w = cv_add(w, o);
    }
    const Cv2 prev = cv_shfl_up(w, 1);
    Cv2 kx = xin;
    cv_mul(Kl, kx);
    excl = lane ? cv_add(kx, prev) : kx;
    Cv2 k32 = xin;
    cv_mul(Kp[5], k32);
    return cv_add(k32, cv_shfl(w, 31));
}

__device__ __forceinline__ void carry_powers(const Mat2& K, int lane, Mat2 (&Kp)[6], Mat2& Kl) {
    Kp[0] = K;
#pragma unroll
    for (int k = 1; k < 6; ++k) Kp[k] = mmul(Kp[k - 1], Kp[k - 1]);
    Kl = mident();
#pragma unroll
    for (int k = 0; k < 5; ++k)
        if ((lane >> k) & 1) Kl = mmul(Kp[k], Kl);
}

// forward: x entering chunk c, x_{c+1} = M^T x_c + summ_c (T steps per chunk)
__global__ void __launch_bounds__(S2_NT) lin_fwd_carry(const LinParams q) {
    const int64_t chain = (int64_t)blockIdx.x * (S2_NT / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (chain >= q.Bsz * q.P) return;  // whole warps
    const int64_t j = chain % q.P, b = chain / q.P;
    Mat2 Kp[6], Kl;
    carry_powers(mpow(lin_coef(q.disc, q.A[j], q.step[j]).m, q.T), lane, Kp, Kl);
    const float4* __restrict__ summ = reinterpret_cast<const float4*>(lin_summ(q));
    float4* __restrict__ carry = reinterpret_cast<float4*>(lin_carry(q));
    Cv2 x = {0.f, 0.f, 0.f, 0.f};
    for (int64_t c0 = 0; c0 < q.C; c0 += 32) {
        const int64_t c = c0 + lane;
        Cv2 w = {0.f, 0.f, 0.f, 0.f};
        if (c < q.C) {
            const float4 sv = summ[(b * q.C + c) * q.P + j];
            w = {sv.x, sv.y, sv.z, sv.w};
        }
        Cv2 ex;
        x = warp_carry_scan(Kp, Kl, w, x, lane, ex);
        if (c < q.C) carry[(b * q.C + c) * q.P + j] = make_float4(ex.x1r, ex.x1i, ex.x2r, ex.x2i);
    }
}

__global__ void __launch_bounds__(S2_NT) lin_fwd_final(const LinParams q) {
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.P) return;
    const int64_t j = idx % q.P, bc = idx / q.P, c = bc % q.C, b = bc / q.C;
    const int64_t t0 = c * q.T, t1 = min64(q.L, t0 + q.T);
    const LinCoef k = lin_coef(q.disc, q.A[j], q.step[j]);
    const float4 in = reinterpret_cast<const float4*>(lin_carry(q))[idx];
    float x1r = in.x, x1i = in.y, x2r = in.z, x2i = in.w;
    float4* __restrict__ ck = reinterpret_cast<float4*>(lin_ckpt(q));
    float2* __restrict__ xo = reinterpret_cast<float2*>(q.x2) + b * q.L * q.P + j;
    for (int64_t ws = t0; ws < t1; ws += S2_CK) {  // ws is a multiple of 8
        float2 u[S2_CK];
        lin_load_window(q.Bu, q, b, ws, t1, j, u);
        if (ck) ck[(b * q.K + ws / S2_CK) * q.P + j] = make_float4(x1r, x1i, x2r, x2i);
#pragma unroll
        for (int s = 0; s < S2_CK; ++s) {
            if (ws + s >= t1) break;
            lin_step(k, u[s], x1r, x1i, x2r, x2i);
            xo[(ws + s) * q.P] = make_float2(x2r, x2i);
        }
    }
}

// backward: gX_t = (0, dx2_t);  lambda_t = gX_t + M^T lambda_{t+1}
__global__ void __launch_bounds__(S2_NT) lin_bwd_summary(const LinParams q) {
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.P) return;
    const int64_t j = idx % q.P, bc = idx / q.P, c = bc % q.C, b = bc / q.C;
    const int64_t t0 = c * q.T, t1 = min64(q.L, t0 + q.T);
    const Mat2 mt = mtrans(lin_coef(q.disc, q.A[j], q.step[j]).m);
    float l1r = 0.f, l1i = 0.f, l2r = 0.f, l2i = 0.f;
    bool first = true;
    // the next (earlier) window's loads are issued before this window's recurrence
    const int64_t wlast = t0 + (t1 - 1 - t0) / S2_CK * S2_CK;
    float2 g[S2_CK], gn[S2_CK];
    lin_load_window(q.dx2, q, b, wlast, t1, j, g);
    for (int64_t ws = wlast; ws >= t0; ws -= S2_CK) {
        if (ws - S2_CK >= t0) lin_load_window(q.dx2, q, b, ws - S2_CK, t1, j, gn);
#pragma unroll
        for (int s = S2_CK - 1; s >= 0; --s) {
            if (ws + s >= t1) continue;
            if (!first) {
                mvec(mt, l1r, l2r);
                mvec(mt, l1i, l2i);
            }
            first = false;
            l2r += g[s].x;
            l2i += g[s].y;
        }
#pragma unroll
        for (int s = 0; s < S2_CK; ++s) g[s] = gn[s];
    }
    reinterpret_cast<float4*>(lin_summ(q))[idx] = make_float4(l1r, l1i, l2r, l2i);
}

// backward: mu_c = M^T lambda at the first step of chunk c + 1 (zero for the
// last chunk, the only one that may be shorter than T); lambda at chunk c's
// first step is lam_loc_c + (M^T)^(T-1) mu_c, so taking chunks from the last,
// mu_{c-1} = (M^T)^T mu_c + M^T lam_loc_c.
__global__ void __launch_bounds__(S2_NT) lin_bwd_carry(const LinParams q) {
    const int64_t chain = (int64_t)blockIdx.x * (S2_NT / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (chain >= q.Bsz * q.P) return;  // whole warps
    const int64_t j = chain % q.P, b = chain / q.P;
    const Mat2 mt = mtrans(lin_coef(q.disc, q.A[j], q.step[j]).m);
    Mat2 Kp[6], Kl;
    carry_powers(mpow(mt, q.T), lane, Kp, Kl);
    const float4* __restrict__ summ = reinterpret_cast<const float4*>(lin_summ(q));
    float4* __restrict__ carry = reinterpret_cast<float4*>(lin_carry(q));
    Cv2 m = {0.f, 0.f, 0.f, 0.f};
    for (int64_t r0 = 0; r0 < q.C; r0 += 32) {
        const int64_t c = q.C - 1 - (r0 + lane);  // lanes take chunks from the last
        Cv2 w = {0.f, 0.f, 0.f, 0.f};
        if (c >= 0) {
            const float4 sv = summ[(b * q.C + c) * q.P + j];
            w = {sv.x, sv.y, sv.z, sv.w};
            cv_mul(mt, w);
        }
        Cv2 ex;
        m = warp_carry_scan(Kp, Kl, w, m, lane, ex);
        if (c >= 0) carry[(b * q.C + c) * q.P + j] = make_float4(ex.x1r, ex.x1i, ex.x2r, ex.x2i);
    }
}

// Per chunk, 8-step windows in reverse: rebuild x_{t-1} from the forward
// checkpoint, then run the adjoint; dBu_t = f1 lambda1_t + f2 lambda2_t;
// dM += lambda_t x_{t-1}^T and (df1, df2) += (lambda1, lambda2) . Bu_t.
// Each thread copies its next window (Bu, dx2, checkpoint) into its own slots
// of shared memory with cp.async while it computes the current one, so a
// window's loads are in flight during the previous window's recurrences (a
// thread reads back only what it copied: no block barrier).
constexpr int LIN_BWD_SLOT = 2 * S2_CK * 2 + 4;  // floats per thread and buffer: Bu, dx2, ckpt
constexpr size_t LIN_BWD_SMEM = sizeof(float) * 2 * LIN_BWD_SLOT * S2_NT;
#ifndef MMB_LIN_BWD_MIN_CTAS
#define MMB_LIN_BWD_MIN_CTAS 2
#endif
__global__ void __launch_bounds__(S2_NT, MMB_LIN_BWD_MIN_CTAS) lin_bwd_final(const LinParams q) {
    extern __shared__ float4 lin_sm4[];
    const int tid = threadIdx.x;
    const int64_t idx = (int64_t)blockIdx.x * S2_NT + tid;
    const bool active = idx < q.Bsz * q.C * q.P;
    float g[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int64_t j = 0;
    if (active) {
        j = idx % q.P;
        const int64_t bc = idx / q.P, c = bc % q.C, b = bc / q.C;
        const int64_t t0 = c * q.T, t1 = min64(q.L, t0 + q.T);
        const LinCoef k = lin_coef(q.disc, q.A[j], q.step[j]);
        const Mat2 mt = mtrans(k.m);
        const float4 mu = reinterpret_cast<const float4*>(lin_carry(q))[idx];
        float l1r = mu.x, l1i = mu.y, l2r = mu.z, l2i = mu.w;  // M^T lambda_{t+1}
        const float4* __restrict__ ck = reinterpret_cast<const float4*>(lin_ckpt(q));
        float2* __restrict__ dbu = reinterpret_cast<float2*>(q.dBu) + b * q.L * q.P + j;
        const float2* __restrict__ bu = reinterpret_cast<const float2*>(q.Bu) + b * q.L * q.P + j;
        const float2* __restrict__ gx = reinterpret_cast<const float2*>(q.dx2) + b * q.L * q.P + j;
        // shared slots: [buffer][Bu(8) | dx2(8) | ckpt] float2/float4 units, thread-minor
        float2* sm2 = reinterpret_cast<float2*>(lin_sm4);
        float4* smck = lin_sm4 + 2 * 2 * S2_CK * S2_NT / 2;
        auto slot2 = [&](int buf, int arr, int s) -> float2* {
            return sm2 + ((buf * 2 + arr) * S2_CK + s) * S2_NT + tid;
        };
        // copy window [ws, ws + 8) (steps past t1 read step ws and are dropped)
        auto issue = [&](int buf, int64_t ws) {
#pragma unroll
            for (int s = 0; s < S2_CK; ++s) {
                const int64_t t = ws + s < t1 ? ws + s : ws;
                cp_async8(slot2(buf, 0, s), bu + t * q.P, true);
                cp_async8(slot2(buf, 1, s), gx + t * q.P, true);
            }
            cp_async16(smck + buf * S2_NT + tid, ck + (b * q.K + ws / S2_CK) * q.P + j, true);
            cp_async_commit();
        };
        // windows [ws, ws + 8) of the chunk (t0 and T are multiples of 8)
        int64_t ws = t0 + (t1 - 1 - t0) / S2_CK * S2_CK;
        int buf = 0;
        issue(0, ws);
        for (; ws >= t0; ws -= S2_CK, buf ^= 1) {
            if (ws - S2_CK >= t0)
                issue(buf ^ 1, ws - S2_CK);
            else
                cp_async_commit();  // an empty group keeps the wait count uniform
            cp_async_wait<1>();
            // Bu and dx2 are read from this thread's slots where each step uses
            // them (not held as register copies of the window: that pushed the
            // kernel past its 128-register cap into local-memory spills).
            // Steps past t1 replay with step ws's Bu; only the states they
            // produce use it, and the adjoint skips those steps.
            const float4 x0 = smck[buf * S2_NT + tid];
            float xs[S2_CK + 1][4];
            xs[0][0] = x0.x; xs[0][1] = x0.y; xs[0][2] = x0.z; xs[0][3] = x0.w;
#pragma unroll
            for (int s = 0; s < S2_CK; ++s) {
                xs[s + 1][0] = xs[s][0]; xs[s + 1][1] = xs[s][1];
                xs[s + 1][2] = xs[s][2]; xs[s + 1][3] = xs[s][3];
                lin_step(k, *slot2(buf, 0, s), xs[s + 1][0], xs[s + 1][1], xs[s + 1][2],
                         xs[s + 1][3]);
            }
#pragma unroll
            for (int s = S2_CK - 1; s >= 0; --s) {
                if (ws + s >= t1) continue;
                const float2 us = *slot2(buf, 0, s), gs = *slot2(buf, 1, s);
                const float a1r = l1r, a1i = l1i, a2r = l2r + gs.x, a2i = l2i + gs.y;
                dbu[(ws + s) * q.P] = make_float2(k.f1 * a1r + k.f2 * a2r, k.f1 * a1i + k.f2 * a2i);
                // state before step t (zero at t = 0: the checkpoint there is zero)
                g[0] += a1r * xs[s][0] + a1i * xs[s][1];
                g[1] += a1r * xs[s][2] + a1i * xs[s][3];
                g[2] += a2r * xs[s][0] + a2i * xs[s][1];
                g[3] += a2r * xs[s][2] + a2i * xs[s][3];
                g[4] += a1r * us.x + a1i * us.y;
                g[5] += a2r * us.x + a2i * us.y;
                l1r = a1r; l1i = a1i; l2r = a2r; l2i = a2i;
                mvec(mt, l1r, l2r);
                mvec(mt, l1i, l2i);
            }
        }
        cp_async_wait<0>();
    }
    // sum over (b, chunk) into per-oscillator accumulators; a warp spans
    // consecutive p, so each thread adds its own
    if (active) {
        float* acc = lin_grad(q) + j * 8;
#pragma unroll
        for (int i = 0; i < 6; ++i) atomicAdd(acc + i, g[i]);
    }
}

// chain rule from (dM, df1, df2) to (dA, dstep)
__global__ void lin_bwd_params(const LinParams q) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= q.P) return;
    const float* g = lin_grad(q) + j * 8;
    const float A = q.A[j], s = q.step[j];
    float dA, ds;
    if (q.disc == 0) {
        const float S = 1.f / (1.f + s * s * A);
        const float S2 = S * S;
        const float M11 = 1.f - s * s * A * S;
        // partial derivatives of (M11, M12, M21, M22, f1, f2) by A and by s
        const float pA[6] = {-s * s * S2, -s * S2, -s * s * s * S2, -s * s * S2, -s * s * s * S2,
                             -s * s * s * s * S2};
        const float pS[6] = {-2.f * s * A * S2, -A * S * (1.f - 2.f * s * s * A * S),
                             S * (1.f - 2.f * s * s * A * S), -2.f * s * A * S2,
                             M11 - 2.f * s * s * A * S2, 2.f * s * S - 2.f * s * s * s * A * S2};
        dA = ds = 0.f;
        for (int i = 0; i < 6; ++i) {
            dA += g[i] * pA[i];
            ds += g[i] * pS[i];
        }
    } else {
        dA = g[1] * (-s) + g[3] * (-s * s);
        ds = g[1] * (-A) + g[2] + g[3] * (-2.f * s * A) + g[4] + g[5] * 2.f * s;
    }
    if (q.dA) q.dA[j] = dA;
    if (q.dstep) q.dstep[j] = ds;
}

static bool al16(const void* ptr) { return ptr == nullptr || ((uintptr_t)ptr & 15) == 0; }

static unsigned s2_blocks(int64_t n) { return (unsigned)((n + S2_NT - 1) / S2_NT); }

template <int NC, bool MS>
static int s2_fwd_launch(const S2Params& p, cudaStream_t st) {
    s2_fwd_summary<NC, MS><<<s2_blocks(p.Bsz * p.C * p.P), S2_NT, 0, st>>>(p);
    s2_fwd_carry<NC, MS><<<s2_blocks(p.Bsz * p.P * 32), S2_NT, 0, st>>>(p);
    s2_fwd_final<NC, MS><<<s2_blocks(p.Bsz * p.C * p.P), S2_NT, 0, st>>>(p);
    return mmb_launch_status();
}

template <int NC, bool GMS>
static int s2_bwd_launch(const S2Params& p, cudaStream_t st) {
    s2_bwd_summary<NC, GMS><<<s2_blocks(p.Bsz * p.C * p.P), S2_NT, 0, st>>>(p);
    s2_bwd_carry<NC, GMS><<<s2_blocks(p.Bsz * p.P), S2_NT, 0, st>>>(p);
    s2_bwd_final<NC, GMS><<<s2_blocks(p.Bsz * p.C * p.P), S2_NT, 0, st>>>(p);
    return mmb_launch_status();
}

static size_t s2_work(int64_t Bsz, int64_t L, int64_t P, int nc) {
    int64_t T, C;
    s2_chunks(Bsz, L, P, T, C);
    const int64_t nv = nc + 2;
    const int64_t fwd = 2 * Bsz * C * P * S2_REC;
    const int64_t bwd = Bsz * C * P * (2 * nv + 8 + 2 * nv);
    return (size_t)(fwd > bwd ? fwd : bwd);
}

// Chunks of the LinOSS layer scan are whole 8-step windows, so chunk,
// window and checkpoint boundaries coincide.
static void lin_dims(int64_t Bsz, int64_t L, int64_t P, LinParams& q) {
    q.Bsz = Bsz;
    q.L = L;
    q.P = P;
    s2_chunks(Bsz, L, P, q.T, q.C);
    q.T = (q.T + S2_CK - 1) / S2_CK * S2_CK;
    q.C = (L + q.T - 1) / q.T;
    q.K = (L + S2_CK - 1) / S2_CK;
}

}  // namespace mmb

using namespace mmb;

extern "C" size_t mmb_scan2_work_floats(int64_t batch, int64_t L, int64_t P, int32_t complex_f) {
    if (batch <= 0 || L <= 0 || P <= 0) return 0;
    return s2_work(batch, L, P, complex_f ? 2 : 1);
}

extern "C" int mmb_scan2_fwd(int64_t batch, int64_t L, int64_t P, int32_t complex_f,
                             const float* M, const float* F, float* Mscan, float* X, float* work,
                             mmb_stream_t stream) {
    MMB_NVTX("mmb_scan2_fwd");
    if (!M || !F || !X) return MMB_ERR_NULL;
    if (!work) return MMB_ERR_WORKSPACE;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    S2Params p{};
    p.Bsz = batch; p.L = L; p.P = P; p.nc = complex_f ? 2 : 1;
    s2_chunks(batch, L, P, p.T, p.C);
    p.M = M; p.F = F; p.Mscan = Mscan; p.Xo = X; p.work = work;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (p.nc == 2) return Mscan ? s2_fwd_launch<2, true>(p, st) : s2_fwd_launch<2, false>(p, st);
    return Mscan ? s2_fwd_launch<1, true>(p, st) : s2_fwd_launch<1, false>(p, st);
}

extern "C" int mmb_scan2_bwd(int64_t batch, int64_t L, int64_t P, int32_t complex_f,
                             const float* M, const float* X, const float* gX, const float* Mscan,
                             const float* gMscan, float* dM, float* dF, float* work,
                             mmb_stream_t stream) {
    MMB_NVTX("mmb_scan2_bwd");
    if (!M || !X || !dM || !dF) return MMB_ERR_NULL;
    if (gMscan && !Mscan) return MMB_ERR_NULL;
    if (!work) return MMB_ERR_WORKSPACE;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    S2Params p{};
    p.Bsz = batch; p.L = L; p.P = P; p.nc = complex_f ? 2 : 1;
    s2_chunks(batch, L, P, p.T, p.C);
    p.M = M; p.X = X; p.gX = gX; p.Mscan_in = Mscan; p.gMs = gMscan;
    p.dM = dM; p.dF = dF; p.work = work;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (p.nc == 2) return gMscan ? s2_bwd_launch<2, true>(p, st) : s2_bwd_launch<2, false>(p, st);
    return gMscan ? s2_bwd_launch<1, true>(p, st) : s2_bwd_launch<1, false>(p, st);
}

extern "C" size_t mmb_linoss_work_floats(int64_t batch, int64_t L, int64_t P) {
    if (batch <= 0 || L <= 0 || P <= 0) return 0;
    LinParams q{};
    lin_dims(batch, L, P, q);
    return (size_t)(q.Bsz * q.K * q.P * 4 + 2 * q.Bsz * q.C * q.P * 4 + q.P * 8);
}

extern "C" int mmb_linoss_fwd(int32_t disc, int64_t batch, int64_t L, int64_t P,
                              const float* A_diag, const float* step, const float* Bu, float* x2,
                              float* work, mmb_stream_t stream) {
    MMB_NVTX("mmb_linoss_fwd");
    if (!A_diag || !step || !Bu || !x2) return MMB_ERR_NULL;
    if (!work) return MMB_ERR_WORKSPACE;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    if (disc != 0 && disc != 1) return MMB_ERR_UNSUPPORTED;
    if (((uintptr_t)Bu & 7) || ((uintptr_t)x2 & 7) || !al16(work)) return MMB_ERR_ALIGN;
    LinParams q{};
    lin_dims(batch, L, P, q);
    q.disc = disc; q.A = A_diag; q.step = step; q.Bu = Bu; q.x2 = x2; q.work = work;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    lin_fwd_summary<<<s2_blocks(q.Bsz * q.C * q.P), S2_NT, 0, st>>>(q);
    lin_fwd_carry<<<s2_blocks(q.Bsz * q.P * 32), S2_NT, 0, st>>>(q);
    lin_fwd_final<<<s2_blocks(q.Bsz * q.C * q.P), S2_NT, 0, st>>>(q);
    return mmb_launch_status();
}

extern "C" int mmb_linoss_bwd(int32_t disc, int64_t batch, int64_t L, int64_t P,
                              const float* A_diag, const float* step, const float* Bu,
                              const float* dx2, float* dBu, float* dA_diag, float* dstep,
                              float* work, mmb_stream_t stream) {
    MMB_NVTX("mmb_linoss_bwd");
    if (!A_diag || !step || !Bu || !dx2 || !dBu) return MMB_ERR_NULL;
    if (!work) return MMB_ERR_WORKSPACE;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    if (disc != 0 && disc != 1) return MMB_ERR_UNSUPPORTED;
    if (((uintptr_t)Bu & 7) || ((uintptr_t)dx2 & 7) || ((uintptr_t)dBu & 7) || !al16(work))
        return MMB_ERR_ALIGN;
    LinParams q{};
    lin_dims(batch, L, P, q);
    q.disc = disc; q.A = A_diag; q.step = step; q.Bu = Bu; q.dx2 = dx2; q.dBu = dBu;
    q.dA = dA_diag; q.dstep = dstep; q.work = work;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(work + (size_t)(q.Bsz * q.K * q.P * 4 + 2 * q.Bsz * q.C * q.P * 4), 0,
                        sizeof(float) * q.P * 8, st) != cudaSuccess)
        return MMB_ERR_LAUNCH;
    lin_bwd_summary<<<s2_blocks(q.Bsz * q.C * q.P), S2_NT, 0, st>>>(q);
    lin_bwd_carry<<<s2_blocks(q.Bsz * q.P * 32), S2_NT, 0, st>>>(q);
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int sa = mmb_smem_attr(lin_bwd_final, LIN_BWD_SMEM, attr_done);
    if (sa != MMB_OK) return sa;
    lin_bwd_final<<<s2_blocks(q.Bsz * q.C * q.P), S2_NT, LIN_BWD_SMEM, st>>>(q);
    lin_bwd_params<<<(unsigned)((P + 127) / 128), 128, 0, st>>>(q);
    return mmb_launch_status();
}

// ---------------------------------------------------------------------------
// No-allocation variant of mmb_scan2_fwd.  The chunk summaries and carries live
// in a fixed device array of this file instead of a caller workspace; the
// number of chunks is lowered until they fit.  Nothing in the array has to start
// at zero: each call writes every record before it reads it.  Host code must not
// pass the array's name to a kernel (on the host it only stands for the symbol);
// its device address comes from cudaGetSymbolAddress, once per device.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float s2_noalloc_scratch[MMB_SCAN2_NOALLOC_SCRATCH_FLOATS];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_scratch[MMB_MAX_DEVICES] = {};
}  // namespace

extern "C" int mmb_scan2_fwd_noalloc(int64_t batch, int64_t L, int64_t P, int32_t complex_f,
                                     const float* M, const float* F, float* Mscan, float* X,
                                     mmb_stream_t stream) {
    MMB_NVTX("mmb_scan2_fwd_noalloc");
    if (!M || !F || !X) return MMB_ERR_NULL;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    // one summary and one carry record of S2_REC floats per (b, chunk, p)
    const int64_t per_chunk = 2 * (int64_t)S2_REC * batch * P;
    const int64_t max_chunks = (int64_t)MMB_SCAN2_NOALLOC_SCRATCH_FLOATS / per_chunk;
    if (max_chunks < 1) return MMB_ERR_SHAPE;  // batch * P too large for the fixed scratch
    S2Params p{};
    p.Bsz = batch; p.L = L; p.P = P; p.nc = complex_f ? 2 : 1;
    s2_chunks(batch, L, P, p.T, p.C);
    if (p.C > max_chunks) {
        p.T = (L + max_chunks - 1) / max_chunks;
        p.C = (L + p.T - 1) / p.T;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= MMB_MAX_DEVICES) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_scratch[dev]) {
            float* ptr = nullptr;
            e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), s2_noalloc_scratch);
            if (e != cudaSuccess || ptr == nullptr) {
                mmb_record_cuda_error(e);
                return MMB_ERR_LAUNCH;
            }
            g_noalloc_scratch[dev] = ptr;
        }
        scratch = g_noalloc_scratch[dev];
    }
    p.M = M; p.F = F; p.Mscan = Mscan; p.Xo = X; p.work = scratch;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (p.nc == 2) return Mscan ? s2_fwd_launch<2, true>(p, st) : s2_fwd_launch<2, false>(p, st);
    return Mscan ? s2_fwd_launch<1, true>(p, st) : s2_fwd_launch<1, false>(p, st);
}
