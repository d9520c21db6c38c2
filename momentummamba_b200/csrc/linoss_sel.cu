// Selective LinOSS scan of the Mamba-LinOSS block (apply_linoss_vectorized,
// mamba_linoss.py:608-677), fused: the per-step transitions are built in
// registers from the step s = mean_D(delta)[b,t] and A_diag[p] instead of
// being materialised as (B, L, 4P) / (B, L, 2P) tensors, and the output
// contraction y[b,t] = Re sum_p C[b,t,p] x2[b,t,p] happens in the kernel.
//
//   IM   (:630-642): S = 1/(1 + s^2 A); M = [[S, -s A S], [s S, S]];
//                    F = (M11 B s, M21 B s)       (note 1 - s^2 A S = S)
//   IMEX (:646-657): M = [[1, -s A], [s, 1 - s^2 A]];  F = (B s, B s^2)
//   x_t = M_t x_{t-1} + F_t (x_{-1} = 0), complex entries, real M;
//   y_t = Re sum_p C_t x2_t                        (:668-675)
//
// Layout: B_re, B_im, C_re, C_im are (B, L, P) views with a shared (batch,
// seq) stride pair each (they are column slices of the x_proj output); s, y,
// dy, ds are (B, L); A, dA are (P).  One thread per (b, chunk, p); the p of a
// (b, chunk) fill whole warps (P rounded up to 32), so the sums over p are
// warp reduce-scatters followed by one atomic per warp and step.  Three
// passes each way (chunk summaries with the chunk's transition product,
// carries, final), chunks of whole 8-step windows; the forward keeps (x1, x2)
// every 8 steps and the backward replays each window from there.
#include "mmb_common.cuh"

namespace mmb {

constexpr int LS_NT = 256;
constexpr int LS_CK = 8;

struct LSParams {
    int64_t Bsz, L, P, PP, T, C, K;  // PP = P rounded up to 32; K = ceil(L / 8)
    int disc;                        // 0 IM, 1 IMEX
    const float *A, *s;
    const float *Bre, *Bim, *Cre, *Cim;
    int64_t bs[2], cs[2];
    float* y;
    float* work;
    const float* dy;
    float *dBre, *dBim, *dCre, *dCim, *dA, *ds;
};

struct LSMat {
    float a, b, c, d;  // [[a, b], [c, d]]
};

struct LSCoef {
    LSMat m;
    float f1, f2;  // F = (f1 B, f2 B)
};

__device__ __forceinline__ LSCoef ls_coef(int disc, float s, float A) {
    LSCoef k;
    if (disc == 0) {
        const float S = 1.f / fmaf(s * s, A, 1.f);
        k.m = {S, -s * A * S, s * S, S};
        k.f1 = s * S;
        k.f2 = s * s * S;
    } else {
        k.m = {1.f, -s * A, s, fmaf(-s * s, A, 1.f)};
        k.f1 = s;
        k.f2 = s * s;
    }
    return k;
}

// d/ds and d/dA of (m11, m12, m21, m22, f1, f2)
__device__ __forceinline__ void ls_dcoef(int disc, float s, float A, float (&ps)[6],
                                         float (&pa)[6]) {
    if (disc == 0) {
        const float S = 1.f / fmaf(s * s, A, 1.f);
        const float S2 = S * S;
        ps[0] = -2.f * s * A * S2;               pa[0] = -s * s * S2;
        ps[1] = -A * S + 2.f * s * s * A * A * S2; pa[1] = -s * S + s * s * s * A * S2;
        ps[2] = S - 2.f * s * s * A * S2;        pa[2] = -s * s * s * S2;
        ps[3] = -2.f * s * A * S2;               pa[3] = -s * s * S2;
        ps[4] = S - 2.f * s * s * A * S2;        pa[4] = -s * s * s * S2;
        ps[5] = 2.f * s * S - 2.f * s * s * s * A * S2; pa[5] = -s * s * s * s * S2;
    } else {
        ps[0] = 0.f;            pa[0] = 0.f;
        ps[1] = -A;             pa[1] = -s;
        ps[2] = 1.f;            pa[2] = 0.f;
        ps[3] = -2.f * s * A;   pa[3] = -s * s;
        ps[4] = 1.f;            pa[4] = 0.f;
        ps[5] = 2.f * s;        pa[5] = 0.f;
    }
}

__device__ __forceinline__ LSMat ls_mul(const LSMat& x, const LSMat& y) {
    return {x.a * y.a + x.b * y.c, x.a * y.b + x.b * y.d, x.c * y.a + x.d * y.c,
            x.c * y.b + x.d * y.d};
}

struct LSIdx {
    int64_t b, c, p, t0, t1;
    bool on;  // p < P
};

__device__ __forceinline__ LSIdx ls_idx(const LSParams& q, int64_t idx) {
    LSIdx r;
    r.p = idx % q.PP;
    const int64_t bc = idx / q.PP;
    r.c = bc % q.C;
    r.b = bc / q.C;
    r.t0 = r.c * q.T;
    r.t1 = min64(q.L, r.t0 + q.T);
    r.on = r.p < q.P;
    return r;
}

// the inputs of an 8-step window starting at ws (steps past t1 read step ws)
struct LSWin {
    float s[LS_CK], br[LS_CK], bi[LS_CK];
};

__device__ __forceinline__ void ls_load_win(const LSParams& q, const LSIdx& x, int64_t ws,
                                            LSWin& w) {
    const int64_t pp = x.on ? x.p : 0;
#pragma unroll
    for (int k = 0; k < LS_CK; ++k) {
        const int64_t t = ws + k < x.t1 ? ws + k : ws;
        w.s[k] = __ldg(q.s + x.b * q.L + t);
        const int64_t o = x.b * q.bs[0] + t * q.bs[1] + pp;
        w.br[k] = __ldg(q.Bre + o);
        w.bi[k] = __ldg(q.Bim + o);
    }
}

// work layout (floats):
//   ckpt : Bsz * K * P * 4               (x1re, x1im, x2re, x2im before every 8th step)
//   tab  : Bsz * C * PP * 16             forward: summary [Mprod(4) | x(4)] then carry [.. | x_in(4)]
//                                        backward: summary [lam(4) | Q(4) | M_t0(4)] then mu(4)
__device__ __forceinline__ float* ls_ckpt(const LSParams& q) { return q.work; }
__device__ __forceinline__ float* ls_tab(const LSParams& q) { return q.work + q.Bsz * q.K * q.P * 4; }

// ------------------------------- forward -----------------------------------
__global__ void __launch_bounds__(LS_NT) ls_fwd_summary(const LSParams q) {
    const int64_t idx = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.PP) return;
    const LSIdx x = ls_idx(q, idx);
    const float A = x.on ? q.A[x.p] : 0.f;
    float x1r = 0.f, x1i = 0.f, x2r = 0.f, x2i = 0.f;
    LSMat mp = {1.f, 0.f, 0.f, 1.f};
    for (int64_t ws = x.t0; ws < x.t1; ws += LS_CK) {
        LSWin w;
        ls_load_win(q, x, ws, w);
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            if (ws + k >= x.t1) break;
            const LSCoef c = ls_coef(q.disc, w.s[k], A);
            const float n1r = c.m.a * x1r + c.m.b * x2r + c.f1 * w.br[k];
            const float n1i = c.m.a * x1i + c.m.b * x2i + c.f1 * w.bi[k];
            const float n2r = c.m.c * x1r + c.m.d * x2r + c.f2 * w.br[k];
            const float n2i = c.m.c * x1i + c.m.d * x2i + c.f2 * w.bi[k];
            x1r = n1r; x1i = n1i; x2r = n2r; x2i = n2i;
            mp = ls_mul(c.m, mp);
        }
    }
    float4* rec = reinterpret_cast<float4*>(ls_tab(q) + idx * 8);
    rec[0] = make_float4(mp.a, mp.b, mp.c, mp.d);
    rec[1] = make_float4(x1r, x1i, x2r, x2i);
}

// Chunk carries.  Across chunks the state follows x_{c+1} = K_c x_c + w_c, an
// affine map per chunk (its transition product and its state from zero); a
// warp takes 32 consecutive chunks of a chain and composes the maps with a
// shuffle scan (Hillis-Steele) instead of one thread walking every chunk.
using LSAff = Aff2<LSMat>;
// Exclusive scan over the warp's lanes of x_{l+1} = map_l(x_l) from x_0 = xin:
// lane l gets x_l in `ex`; every lane gets x_32 back.
__device__ __forceinline__ float4 ls_warp_carry(const LSAff& v, const float4& xin, int lane,
                                                float4& ex) {
    const LSAff x0 = {{0.f, 0.f, 0.f, 0.f}, xin.x, xin.y, xin.z, xin.w};
    LSAff e;
    const LSAff n = warp_aff2_exscan(v, x0, lane, e);
    ex = make_float4(e.x1r, e.x1i, e.x2r, e.x2i);
    return make_float4(n.x1r, n.x1i, n.x2r, n.x2i);
}

// per (b, p): the state entering each chunk; overwrites the record's x with it
__global__ void __launch_bounds__(LS_NT) ls_fwd_carry(const LSParams q) {
    const int64_t chain = (int64_t)blockIdx.x * (LS_NT / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (chain >= q.Bsz * q.PP) return;  // whole warps
    const int64_t p = chain % q.PP, b = chain / q.PP;
    float4* tab = reinterpret_cast<float4*>(ls_tab(q));
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t c0 = 0; c0 < q.C; c0 += 32) {
        const int64_t c = c0 + lane;
        LSAff v = {{1.f, 0.f, 0.f, 1.f}, 0.f, 0.f, 0.f, 0.f};
        const int64_t r = (b * q.C + c) * q.PP + p;
        if (c < q.C) {
            const float4 mm = tab[r * 2], xs = tab[r * 2 + 1];
            v = {{mm.x, mm.y, mm.z, mm.w}, xs.x, xs.y, xs.z, xs.w};
        }
        float4 ex;
        x = ls_warp_carry(v, x, lane, ex);
        if (c < q.C) tab[r * 2 + 1] = ex;
    }
}

// Sum an 8-step vector over the warp's 32 lanes (consecutive p); lanes 0..7
// then hold the totals of steps rs_index<8, 5>(lane, 0) and add them to dst.
__device__ __forceinline__ void ls_warp_add8(float (&v)[LS_CK], float* dst_row, int64_t ws,
                                             int64_t t1, int lane) {
    reduce_scatter<LS_CK, 0, 5>(v, lane);
    if (lane < LS_CK) {
        const int k = rs_index<LS_CK, 5>(lane, 0);
        if (ws + k < t1) atomicAdd(dst_row + ws + k, v[0]);
    }
}

__global__ void __launch_bounds__(LS_NT) ls_fwd_final(const LSParams q) {
    const int64_t idx = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.PP) return;  // whole warps: PP % 32 == 0
    const int lane = threadIdx.x & 31;
    const LSIdx x = ls_idx(q, idx);
    const float A = x.on ? q.A[x.p] : 0.f;
    const float4 in = reinterpret_cast<const float4*>(ls_tab(q) + idx * 8)[1];
    float x1r = in.x, x1i = in.y, x2r = in.z, x2i = in.w;
    float4* ck = reinterpret_cast<float4*>(ls_ckpt(q));
    const int64_t pp = x.on ? x.p : 0;
    for (int64_t ws = x.t0; ws < x.t1; ws += LS_CK) {
        LSWin w;
        ls_load_win(q, x, ws, w);
        float cr[LS_CK], ci[LS_CK];
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            const int64_t t = ws + k < x.t1 ? ws + k : ws;
            const int64_t o = x.b * q.cs[0] + t * q.cs[1] + pp;
            cr[k] = __ldg(q.Cre + o);
            ci[k] = __ldg(q.Cim + o);
        }
        if (x.on) ck[(x.b * q.K + ws / LS_CK) * q.P + x.p] = make_float4(x1r, x1i, x2r, x2i);
        float yv[LS_CK];
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            yv[k] = 0.f;
            if (ws + k >= x.t1) continue;
            const LSCoef c = ls_coef(q.disc, w.s[k], A);
            const float n1r = c.m.a * x1r + c.m.b * x2r + c.f1 * w.br[k];
            const float n1i = c.m.a * x1i + c.m.b * x2i + c.f1 * w.bi[k];
            const float n2r = c.m.c * x1r + c.m.d * x2r + c.f2 * w.br[k];
            const float n2i = c.m.c * x1i + c.m.d * x2i + c.f2 * w.bi[k];
            x1r = n1r; x1i = n1i; x2r = n2r; x2i = n2i;
            yv[k] = x.on ? cr[k] * x2r - ci[k] * x2i : 0.f;
        }
        ls_warp_add8(yv, q.y + x.b * q.L, ws, x.t1, lane);
    }
}

// ------------------------------- backward ----------------------------------
// adjoint: lam_t = g_t + M_{t+1}^T lam_{t+1}, g_t = (0, dy_t (C_re, -C_im))
__global__ void __launch_bounds__(LS_NT) ls_bwd_summary(const LSParams q) {
    const int64_t idx = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.PP) return;
    const LSIdx x = ls_idx(q, idx);
    const float A = x.on ? q.A[x.p] : 0.f;
    const int64_t pp = x.on ? x.p : 0;
    float l1r = 0.f, l1i = 0.f, l2r = 0.f, l2i = 0.f;
    LSMat Q = {1.f, 0.f, 0.f, 1.f};   // M_{t0+1}^T ... M_{t1-1}^T
    LSMat mn = {0.f, 0.f, 0.f, 0.f};  // M_{t+1}; none past the chunk end
    for (int64_t ws = x.t0 + (x.t1 - 1 - x.t0) / LS_CK * LS_CK; ws >= x.t0; ws -= LS_CK) {
        float sv[LS_CK], gr[LS_CK], gi[LS_CK];
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            const int64_t t = ws + k < x.t1 ? ws + k : ws;
            sv[k] = __ldg(q.s + x.b * q.L + t);
            const float dy = __ldg(q.dy + x.b * q.L + t);
            const int64_t o = x.b * q.cs[0] + t * q.cs[1] + pp;
            gr[k] = dy * __ldg(q.Cre + o);
            gi[k] = -dy * __ldg(q.Cim + o);
        }
#pragma unroll
        for (int k = LS_CK - 1; k >= 0; --k) {
            if (ws + k >= x.t1) continue;
            // lam = g + mn^T lam
            const float a1r = mn.a * l1r + mn.c * l2r, a1i = mn.a * l1i + mn.c * l2i;
            const float a2r = mn.b * l1r + mn.d * l2r + gr[k], a2i = mn.b * l1i + mn.d * l2i + gi[k];
            l1r = a1r; l1i = a1i; l2r = a2r; l2i = a2i;
            const LSMat m = ls_coef(q.disc, sv[k], A).m;
            if (ws + k > x.t0) Q = ls_mul(LSMat{m.a, m.c, m.b, m.d}, Q);
            mn = m;
        }
    }
    float4* rec = reinterpret_cast<float4*>(ls_tab(q) + idx * 16);
    rec[0] = make_float4(l1r, l1i, l2r, l2i);
    rec[1] = make_float4(Q.a, Q.b, Q.c, Q.d);
    rec[2] = make_float4(mn.a, mn.b, mn.c, mn.d);
}

// per (b, p), chunks in reverse: mu_c = M_{t0(c+1)}^T lam_{t0(c+1)} entering chunk c
// from the right; written to the record's last float4.  With lam_{t0} = lam_loc
// + Q mu, mu_{c-1} = M_{t0}^T Q mu_c + M_{t0}^T lam_loc: an affine map per chunk,
// scanned by one warp per chain over 32 chunks at a time from the last.
__global__ void __launch_bounds__(LS_NT) ls_bwd_carry(const LSParams q) {
    const int64_t chain = (int64_t)blockIdx.x * (LS_NT / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (chain >= q.Bsz * q.PP) return;  // whole warps
    const int64_t p = chain % q.PP, b = chain / q.PP;
    float4* tab = reinterpret_cast<float4*>(ls_tab(q));
    float4 mu = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t r0 = 0; r0 < q.C; r0 += 32) {
        const int64_t c = q.C - 1 - (r0 + lane);  // lanes take chunks from the last
        LSAff v = {{1.f, 0.f, 0.f, 1.f}, 0.f, 0.f, 0.f, 0.f};
        const int64_t r = (b * q.C + c) * q.PP + p;
        if (c >= 0) {
            const float4 lam = tab[r * 4], Q = tab[r * 4 + 1], M = tab[r * 4 + 2];
            const LSMat mt = {M.x, M.z, M.y, M.w};  // M_{t0}^T
            v.m = ls_mul(mt, LSMat{Q.x, Q.y, Q.z, Q.w});
            v.x1r = mt.a * lam.x + mt.b * lam.z;
            v.x1i = mt.a * lam.y + mt.b * lam.w;
            v.x2r = mt.c * lam.x + mt.d * lam.z;
            v.x2i = mt.c * lam.y + mt.d * lam.w;
        }
        float4 ex;
        mu = ls_warp_carry(v, mu, lane, ex);
        if (c >= 0) tab[r * 4 + 3] = ex;
    }
}

__global__ void __launch_bounds__(LS_NT) ls_bwd_final(const LSParams q) {
    const int64_t idx = (int64_t)blockIdx.x * LS_NT + threadIdx.x;
    if (idx >= q.Bsz * q.C * q.PP) return;
    const int lane = threadIdx.x & 31;
    const LSIdx x = ls_idx(q, idx);
    const float A = x.on ? q.A[x.p] : 0.f;
    const int64_t pp = x.on ? x.p : 0;
    const float4 mu = reinterpret_cast<const float4*>(ls_tab(q) + idx * 16)[3];
    float c1r = mu.x, c1i = mu.y, c2r = mu.z, c2i = mu.w;  // M_{t+1}^T lam_{t+1}
    const float4* ck = reinterpret_cast<const float4*>(ls_ckpt(q));
    float dAacc = 0.f;
    for (int64_t ws = x.t0 + (x.t1 - 1 - x.t0) / LS_CK * LS_CK; ws >= x.t0; ws -= LS_CK) {
        LSWin w;
        ls_load_win(q, x, ws, w);
        float cr[LS_CK], ci[LS_CK], dyv[LS_CK];
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            const int64_t t = ws + k < x.t1 ? ws + k : ws;
            const int64_t o = x.b * q.cs[0] + t * q.cs[1] + pp;
            cr[k] = __ldg(q.Cre + o);
            ci[k] = __ldg(q.Cim + o);
            dyv[k] = __ldg(q.dy + x.b * q.L + t);
        }
        // replay the window: xs[k] = state before step ws + k
        const float4 x0 = x.on ? ck[(x.b * q.K + ws / LS_CK) * q.P + x.p]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        float xs[LS_CK + 1][4];
        xs[0][0] = x0.x; xs[0][1] = x0.y; xs[0][2] = x0.z; xs[0][3] = x0.w;
#pragma unroll
        for (int k = 0; k < LS_CK; ++k) {
            const LSCoef c = ls_coef(q.disc, w.s[k], A);
            xs[k + 1][0] = c.m.a * xs[k][0] + c.m.b * xs[k][2] + c.f1 * w.br[k];
            xs[k + 1][1] = c.m.a * xs[k][1] + c.m.b * xs[k][3] + c.f1 * w.bi[k];
            xs[k + 1][2] = c.m.c * xs[k][0] + c.m.d * xs[k][2] + c.f2 * w.br[k];
            xs[k + 1][3] = c.m.c * xs[k][1] + c.m.d * xs[k][3] + c.f2 * w.bi[k];
        }
        float dsv[LS_CK];
#pragma unroll
        for (int k = LS_CK - 1; k >= 0; --k) {
            dsv[k] = 0.f;
            if (ws + k >= x.t1) continue;
            const int64_t t = ws + k;
            const LSCoef c = ls_coef(q.disc, w.s[k], A);
            // lam_t
            const float l1r = c1r, l1i = c1i;
            const float l2r = c2r + dyv[k] * cr[k], l2i = c2i - dyv[k] * ci[k];
            // dM = lam x_{t-1}^T (over re, im), dF = lam; F = (f1 B, f2 B)
            const float dm11 = l1r * xs[k][0] + l1i * xs[k][1];
            const float dm12 = l1r * xs[k][2] + l1i * xs[k][3];
            const float dm21 = l2r * xs[k][0] + l2i * xs[k][1];
            const float dm22 = l2r * xs[k][2] + l2i * xs[k][3];
            const float df1 = l1r * w.br[k] + l1i * w.bi[k];
            const float df2 = l2r * w.br[k] + l2i * w.bi[k];
            float ps[6], pa[6];
            ls_dcoef(q.disc, w.s[k], A, ps, pa);
            const float g6[6] = {dm11, dm12, dm21, dm22, df1, df2};
            float gs = 0.f, ga = 0.f;
#pragma unroll
            for (int i = 0; i < 6; ++i) {
                gs = fmaf(g6[i], ps[i], gs);
                ga = fmaf(g6[i], pa[i], ga);
            }
            if (x.on) {
                const int64_t o = (x.b * q.L + t) * q.P + x.p;
                q.dBre[o] = c.f1 * l1r + c.f2 * l2r;
                q.dBim[o] = c.f1 * l1i + c.f2 * l2i;
                q.dCre[o] = dyv[k] * xs[k + 1][2];
                q.dCim[o] = -dyv[k] * xs[k + 1][3];
                dsv[k] = gs;
                dAacc += ga;
            }
            // carry M_t^T lam_t to step t - 1
            c1r = c.m.a * l1r + c.m.c * l2r; c1i = c.m.a * l1i + c.m.c * l2i;
            c2r = c.m.b * l1r + c.m.d * l2r; c2i = c.m.b * l1i + c.m.d * l2i;
        }
        ls_warp_add8(dsv, q.ds + x.b * q.L, ws, x.t1, lane);
    }
    if (x.on) atomicAdd(q.dA + x.p, dAacc);
}

static unsigned ls_blocks(int64_t n) { return (unsigned)((n + LS_NT - 1) / LS_NT); }

static void ls_dims(int64_t Bsz, int64_t L, int64_t P, LSParams& q) {
    q.Bsz = Bsz;
    q.L = L;
    q.P = P;
    q.PP = (P + 31) / 32 * 32;
    // chains x chunks to fill the GPU, chunks of whole 8-step windows (>= 16 steps)
    const int64_t target = 148 * 2048;
    int64_t want = (target + Bsz * q.PP - 1) / (Bsz * q.PP);
    const int64_t maxc = (L + 15) / 16;
    if (want < 1) want = 1;
    if (want > maxc) want = maxc;
    q.T = (L + want - 1) / want;
    q.T = (q.T + LS_CK - 1) / LS_CK * LS_CK;
    q.C = (L + q.T - 1) / q.T;
    q.K = (L + LS_CK - 1) / LS_CK;
}

static int ls_fill(int32_t disc, int64_t batch, int64_t L, int64_t P, const float* A_diag,
                   const float* s, const float* B_re, const float* B_im, const int64_t* B_stride,
                   const float* C_re, const float* C_im, const int64_t* C_stride, float* work,
                   LSParams& q) {
    if (!A_diag || !s || !B_re || !B_im || !B_stride || !C_re || !C_im || !C_stride)
        return MMB_ERR_NULL;
    if (!work) return MMB_ERR_WORKSPACE;
    if (batch <= 0 || L <= 0 || P <= 0) return MMB_ERR_SHAPE;
    if (disc != 0 && disc != 1) return MMB_ERR_UNSUPPORTED;
    if ((uintptr_t)work & 15) return MMB_ERR_ALIGN;
    q = LSParams{};
    ls_dims(batch, L, P, q);
    q.disc = disc;
    q.A = A_diag; q.s = s;
    q.Bre = B_re; q.Bim = B_im; q.Cre = C_re; q.Cim = C_im;
    q.bs[0] = B_stride[0]; q.bs[1] = B_stride[1];
    q.cs[0] = C_stride[0]; q.cs[1] = C_stride[1];
    q.work = work;
    return MMB_OK;
}

}  // namespace mmb

using namespace mmb;

extern "C" size_t mmb_linoss_sel_work_floats(int64_t batch, int64_t L, int64_t P) {
    if (batch <= 0 || L <= 0 || P <= 0) return 0;
    LSParams q{};
    ls_dims(batch, L, P, q);
    return (size_t)(q.Bsz * q.K * q.P * 4 + q.Bsz * q.C * q.PP * 16);
}

extern "C" int mmb_linoss_sel_fwd(int32_t disc, int64_t batch, int64_t L, int64_t P,
                                  const float* A_diag, const float* s, const float* B_re,
                                  const float* B_im, const int64_t* B_stride, const float* C_re,
                                  const float* C_im, const int64_t* C_stride, float* y,
                                  float* work, mmb_stream_t stream) {
    MMB_NVTX("mmb_linoss_sel_fwd");
    LSParams q;
    int st = ls_fill(disc, batch, L, P, A_diag, s, B_re, B_im, B_stride, C_re, C_im, C_stride,
                     work, q);
    if (st != MMB_OK) return st;
    if (!y) return MMB_ERR_NULL;
    q.y = y;
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    const cudaError_t e = cudaMemsetAsync(y, 0, (size_t)(batch * L) * sizeof(float), cs);
    if (e != cudaSuccess) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    ls_fwd_summary<<<ls_blocks(q.Bsz * q.C * q.PP), LS_NT, 0, cs>>>(q);
    ls_fwd_carry<<<ls_blocks(q.Bsz * q.PP * 32), LS_NT, 0, cs>>>(q);
    ls_fwd_final<<<ls_blocks(q.Bsz * q.C * q.PP), LS_NT, 0, cs>>>(q);
    return mmb_launch_status();
}

extern "C" int mmb_linoss_sel_bwd(int32_t disc, int64_t batch, int64_t L, int64_t P,
                                  const float* A_diag, const float* s, const float* B_re,
                                  const float* B_im, const int64_t* B_stride, const float* C_re,
                                  const float* C_im, const int64_t* C_stride, const float* dy,
                                  float* dB_re, float* dB_im, float* dC_re, float* dC_im,
                                  float* dA_diag, float* ds, float* work, mmb_stream_t stream) {
    MMB_NVTX("mmb_linoss_sel_bwd");
    LSParams q;
    int st = ls_fill(disc, batch, L, P, A_diag, s, B_re, B_im, B_stride, C_re, C_im, C_stride,
                     work, q);
    if (st != MMB_OK) return st;
    if (!dy || !dB_re || !dB_im || !dC_re || !dC_im || !dA_diag || !ds) return MMB_ERR_NULL;
    q.dy = dy;
    q.dBre = dB_re; q.dBim = dB_im; q.dCre = dC_re; q.dCim = dC_im;
    q.dA = dA_diag; q.ds = ds;
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(dA_diag, 0, (size_t)P * sizeof(float), cs);
    if (e == cudaSuccess) e = cudaMemsetAsync(ds, 0, (size_t)(batch * L) * sizeof(float), cs);
    if (e != cudaSuccess) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    ls_bwd_summary<<<ls_blocks(q.Bsz * q.C * q.PP), LS_NT, 0, cs>>>(q);
    ls_bwd_carry<<<ls_blocks(q.Bsz * q.PP * 32), LS_NT, 0, cs>>>(q);
    ls_bwd_final<<<ls_blocks(q.Bsz * q.C * q.PP), LS_NT, 0, cs>>>(q);
    return mmb_launch_status();
}
