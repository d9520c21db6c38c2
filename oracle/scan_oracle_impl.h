/*
 * Body of the CPU oracle, instantiated twice by scan_oracle.c (REAL = double
 * and REAL = float).  TEST INFRASTRUCTURE ONLY -- see scan_oracle.c.
 *
 * Layouts (all row-major, contiguous):
 *   x, delta, z, out, ypre, dx, ddelta, dz, dout : (Bsz, L, D)
 *   Bm, Cm, dB, dC                               : (Bsz, L, N)
 *   A, dA                                        : (D, N)
 *   Dskip, dbias, dD, ddbias                     : (D)
 *   rows scan                                    : (R, L)
 *   2x2 scan M                                   : (Bsz, L, 4P) = [M11 | M12 | M21 | M22]
 *   2x2 scan F, X                                : (Bsz, L, 2P) = [F1 | F2], complex
 *                                                  entries stored as (re, im) pairs
 */

static inline REAL SFX(softplus_)(REAL r) {
    /* torch.nn.functional.softplus, beta = 1, threshold = 20 */
    return r > (REAL)20 ? r : LOG1P(EXP(r));
}

static inline REAL SFX(sigmoid_)(REAL r) { return (REAL)1 / ((REAL)1 + EXP(-r)); }

/* ---------------------------------------------------------------------------
 * Momentum selective scan, forward.
 *   dt   = softplus(delta + bias) or delta              (mamba_momentum.py:247)
 *   a    = exp(dt * A[d,n]);  u = alpha*dt*B[n]*x      (mamba_momentum.py:291-296)
 *   v    = beta*v + u;  h = a*h + v                     (mamba_momentum.py:427-431)
 *   y    = sum_n C[n]*h + D*x                           (mamba_momentum.py:319-321)
 *   out  = y * silu(z)  when z is given                 (mamba_momentum.py:227-229)
 * ypre (nullable) receives y before the gate.
 * state_in / state_out (nullable, (Bsz, D, 2, N): h then v) are the state
 * before the first step (zeros when NULL) and after the last one; they carry
 * a sequence split into consecutive segments from one segment to the next.
 * ------------------------------------------------------------------------- */
void SFX(orc_mmscan_fwd)(i64 Bsz, i64 L, i64 D, i64 N,
                         const REAL* x, const REAL* delta, const REAL* A,
                         const REAL* Bm, const REAL* Cm, const REAL* Dskip,
                         const REAL* z, const REAL* dbias, int softplus,
                         double beta_d, double alpha_d, REAL* out, REAL* ypre,
                         const REAL* state_in, REAL* state_out) {
    const REAL beta = (REAL)beta_d, alpha = (REAL)alpha_d;
#pragma omp parallel for schedule(dynamic, 4)
    for (i64 bd = 0; bd < Bsz * D; ++bd) {
        const i64 b = bd / D, d = bd % D;
        REAL* h = (REAL*)calloc((size_t)(2 * N), sizeof(REAL));
        REAL* v = h + N;
        if (state_in)
            for (i64 n = 0; n < 2 * N; ++n) h[n] = state_in[bd * 2 * N + n];
        for (i64 t = 0; t < L; ++t) {
            const i64 io = (b * L + t) * D + d;
            const i64 bo = (b * L + t) * N;
            REAL dt = delta[io];
            if (dbias) dt += dbias[d];
            if (softplus) dt = SFX(softplus_)(dt);
            const REAL xv = x[io];
            REAL y = 0;
            for (i64 n = 0; n < N; ++n) {
                const REAL a = EXP(dt * A[d * N + n]);
                const REAL u = alpha * (dt * Bm[bo + n]) * xv;
                v[n] = beta * v[n] + u;
                h[n] = a * h[n] + v[n];
                y += Cm[bo + n] * h[n];
            }
            if (Dskip) y += Dskip[d] * xv;
            if (ypre) ypre[io] = y;
            if (z) {
                const REAL zv = z[io];
                y = y * zv * SFX(sigmoid_)(zv);
            }
            out[io] = y;
        }
        if (state_out)
            for (i64 n = 0; n < 2 * N; ++n) state_out[bd * 2 * N + n] = h[n];
        free(h);
    }
}

/* ---------------------------------------------------------------------------
 * Segment summary of the forward recurrence, for a sequence split into
 * consecutive segments.  Over one segment of T steps the state maps as
 *   h_T = P h_0 + beta Q' v_0 + h_T^0 ;  v_T = beta^T v_0 + v_T^0
 * with (h^0, v^0) the segment's result from a zero state, P = prod_t a_t and
 * Q' = sum_{t=1..T} beta^{t-1} prod_{s>t} a_s (Q'_t = a_t Q'_{t-1} + beta^{t-1}).
 * summary: (Bsz, D, 4, N) = [h^0 | v^0 | P | Q'].
 * ------------------------------------------------------------------------- */
void SFX(orc_mmscan_fwd_summary)(i64 Bsz, i64 L, i64 D, i64 N,
                                 const REAL* x, const REAL* delta, const REAL* A,
                                 const REAL* Bm, const REAL* dbias, int softplus,
                                 double beta_d, double alpha_d, REAL* summary) {
    const REAL beta = (REAL)beta_d, alpha = (REAL)alpha_d;
#pragma omp parallel for schedule(dynamic, 4)
    for (i64 bd = 0; bd < Bsz * D; ++bd) {
        const i64 b = bd / D, d = bd % D;
        REAL* h = summary + bd * 4 * N;
        REAL* v = h + N;
        REAL* P = h + 2 * N;
        REAL* Q = h + 3 * N;
        for (i64 n = 0; n < N; ++n) { h[n] = 0; v[n] = 0; P[n] = 1; Q[n] = 0; }
        REAL bp = 1; /* beta^(t-1) */
        for (i64 t = 0; t < L; ++t) {
            const i64 io = (b * L + t) * D + d;
            const i64 bo = (b * L + t) * N;
            REAL dt = delta[io];
            if (dbias) dt += dbias[d];
            if (softplus) dt = SFX(softplus_)(dt);
            const REAL xv = x[io];
            for (i64 n = 0; n < N; ++n) {
                const REAL a = EXP(dt * A[d * N + n]);
                const REAL u = alpha * (dt * Bm[bo + n]) * xv;
                v[n] = beta * v[n] + u;
                h[n] = a * h[n] + v[n];
                P[n] = a * P[n];
                Q[n] = a * Q[n] + bp;
            }
            bp *= beta;
        }
    }
}

/* ---------------------------------------------------------------------------
 * Momentum selective scan, backward: exact adjoint of the forward above.
 *   gh_t = dy_t*C_t + a_{t+1}*gh_{t+1};   gv_t = gh_t + beta*gv_{t+1}
 *   du_t = gv_t;   da_t = gh_t*h_{t-1} (zero at t = 0, as pscan.py:229-230 and
 *   momentum_scan_cuda.py:77 leave it)
 * Every output is overwritten.  dz / ddbias / dD may be NULL when the matching
 * input was absent.
 * Segments (all nullable, (Bsz, D, 2, N)): state_in is the forward's state_in;
 * gstate_in = (a_L gh_L, gv_L) arriving from the step after the segment (zeros
 * when NULL), gstate_out = (a_0 gh_0, gv_0) leaving it towards the step before.  Parallel over (b, block of 8 channels); the d-sums of dB
 * and dC and the (b,t)-sums of dA/dD/ddbias are reduced in a fixed order.
 * ------------------------------------------------------------------------- */
void SFX(orc_mmscan_bwd)(i64 Bsz, i64 L, i64 D, i64 N,
                         const REAL* x, const REAL* delta, const REAL* A,
                         const REAL* Bm, const REAL* Cm, const REAL* Dskip,
                         const REAL* z, const REAL* dbias, int softplus,
                         double beta_d, double alpha_d, const REAL* dout,
                         REAL* dx, REAL* ddelta, REAL* dA, REAL* dB, REAL* dC,
                         REAL* dD, REAL* dz, REAL* ddbias, const REAL* state_in,
                         const REAL* gstate_in, REAL* gstate_out) {
    const REAL beta = (REAL)beta_d, alpha = (REAL)alpha_d;
    const i64 DB = 8;
    const i64 nblk = (D + DB - 1) / DB;
    const i64 ntask = Bsz * nblk;
    /* per-task partials, reduced afterwards in task order */
    REAL* pB = (REAL*)calloc((size_t)(ntask * L * N), sizeof(REAL));
    REAL* pC = (REAL*)calloc((size_t)(ntask * L * N), sizeof(REAL));
    REAL* pA = (REAL*)calloc((size_t)(Bsz * D * N), sizeof(REAL));
    REAL* pD = (REAL*)calloc((size_t)(Bsz * D), sizeof(REAL));
    REAL* pbias = (REAL*)calloc((size_t)(Bsz * D), sizeof(REAL));

#pragma omp parallel for schedule(dynamic, 1)
    for (i64 task = 0; task < ntask; ++task) {
        const i64 b = task / nblk, blk = task % nblk;
        REAL* hs = (REAL*)malloc((size_t)((L + 1) * N) * sizeof(REAL));
        REAL* yp = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* dts = (REAL*)malloc((size_t)L * sizeof(REAL));
        REAL* gh = (REAL*)malloc((size_t)(2 * N) * sizeof(REAL));
        REAL* gv = gh + N;
        REAL* tB = pB + task * L * N;
        REAL* tC = pC + task * L * N;
        for (i64 d = blk * DB; d < D && d < (blk + 1) * DB; ++d) {
            /* forward replay; hs[t+1] holds h_t, hs[0] = 0 */
            REAL* v = gv; /* reuse as forward momentum state */
            const i64 so = (b * D + d) * 2 * N;
            for (i64 n = 0; n < N; ++n) {
                hs[n] = state_in ? state_in[so + n] : (REAL)0;
                v[n] = state_in ? state_in[so + N + n] : (REAL)0;
            }
            for (i64 t = 0; t < L; ++t) {
                const i64 io = (b * L + t) * D + d;
                const i64 bo = (b * L + t) * N;
                REAL dt = delta[io];
                if (dbias) dt += dbias[d];
                if (softplus) dt = SFX(softplus_)(dt);
                dts[t] = dt;
                const REAL xv = x[io];
                REAL y = 0;
                for (i64 n = 0; n < N; ++n) {
                    const REAL a = EXP(dt * A[d * N + n]);
                    const REAL u = alpha * (dt * Bm[bo + n]) * xv;
                    v[n] = beta * v[n] + u;
                    const REAL hn = a * hs[t * N + n] + v[n];
                    hs[(t + 1) * N + n] = hn;
                    y += Cm[bo + n] * hn;
                }
                if (Dskip) y += Dskip[d] * xv;
                yp[t] = y;
            }
            REAL accD = 0, accBias = 0;
            /* a_{t+1} factors carried from the previous (later) step; a carry
               arriving from the right enters as gh = a_L gh_L with a factor 1 */
            REAL* anext = (REAL*)calloc((size_t)N, sizeof(REAL));
            for (i64 n = 0; n < N; ++n) {
                gh[n] = gstate_in ? gstate_in[so + n] : (REAL)0;
                gv[n] = gstate_in ? gstate_in[so + N + n] : (REAL)0;
                anext[n] = gstate_in ? (REAL)1 : (REAL)0;
            }
            for (i64 t = L - 1; t >= 0; --t) {
                const i64 io = (b * L + t) * D + d;
                const i64 bo = (b * L + t) * N;
                const REAL dt = dts[t];
                const REAL xv = x[io];
                REAL dy = dout[io];
                if (z) {
                    const REAL zv = z[io];
                    const REAL sg = SFX(sigmoid_)(zv);
                    if (dz) dz[io] = dy * yp[t] * sg * ((REAL)1 + zv * ((REAL)1 - sg));
                    dy = dy * zv * sg;
                }
                accD += dy * xv;
                REAL gx = Dskip ? dy * Dskip[d] : (REAL)0;
                REAL gdt = 0;
                for (i64 n = 0; n < N; ++n) {
                    const REAL a = EXP(dt * A[d * N + n]);
                    const REAL hcur = hs[(t + 1) * N + n];
                    const REAL hprev = hs[t * N + n];
                    tC[t * N + n] += dy * hcur;
                    gh[n] = dy * Cm[bo + n] + anext[n] * gh[n];
                    gv[n] = gh[n] + beta * gv[n];
                    const REAL du = gv[n];
                    tB[t * N + n] += du * alpha * dt * xv;
                    gx += du * alpha * dt * Bm[bo + n];
                    gdt += du * alpha * Bm[bo + n] * xv;
                    const REAL da = gh[n] * hprev; /* hprev = state_in (0) at t = 0 */
                    gdt += da * a * A[d * N + n];
                    pA[(b * D + d) * N + n] += da * a * dt;
                    anext[n] = a;
                }
                dx[io] = gx;
                if (softplus) {
                    REAL r = delta[io] + (dbias ? dbias[d] : (REAL)0);
                    gdt = r > (REAL)20 ? gdt : gdt * SFX(sigmoid_)(r);
                }
                ddelta[io] = gdt;
                accBias += gdt;
            }
            if (gstate_out)
                for (i64 n = 0; n < N; ++n) {
                    gstate_out[so + n] = anext[n] * gh[n];
                    gstate_out[so + N + n] = gv[n];
                }
            free(anext);
            pD[b * D + d] = accD;
            pbias[b * D + d] = accBias;
        }
        free(hs); free(yp); free(dts); free(gh);
    }

    /* fixed-order reductions */
#pragma omp parallel for
    for (i64 bt = 0; bt < Bsz * L; ++bt) {
        const i64 b = bt / L, t = bt % L;
        for (i64 n = 0; n < N; ++n) {
            REAL sb = 0, sc = 0;
            for (i64 blk = 0; blk < nblk; ++blk) {
                const i64 task = b * nblk + blk;
                sb += pB[(task * L + t) * N + n];
                sc += pC[(task * L + t) * N + n];
            }
            dB[bt * N + n] = sb;
            dC[bt * N + n] = sc;
        }
    }
    for (i64 dn = 0; dn < D * N; ++dn) {
        REAL s = 0;
        for (i64 b = 0; b < Bsz; ++b) s += pA[b * D * N + dn];
        dA[dn] = s;
    }
    for (i64 d = 0; d < D; ++d) {
        REAL s = 0, sb = 0;
        for (i64 b = 0; b < Bsz; ++b) { s += pD[b * D + d]; sb += pbias[b * D + d]; }
        if (dD) dD[d] = s;
        if (ddbias) ddbias[d] = sb;
    }
    free(pB); free(pC); free(pA); free(pD); free(pbias);
}

/* ---------------------------------------------------------------------------
 * Row scan (momentum_scan_cuda semantics, momentum_scan_cuda.py:22-87):
 *   v_t = beta*v_{t-1} + u_t ;  h_t = a_t*h_{t-1} + v_t ;  rows of length L.
 * With beta = 0 this is the PScan recurrence H_t = A_t*H_{t-1} + X_t
 * (pscan.py:51) on rows.  vout may be NULL.
 * ------------------------------------------------------------------------- */
void SFX(orc_rows_fwd)(i64 R, i64 L, const REAL* a, double beta_d, const REAL* u,
                       REAL* h, REAL* vout) {
    const REAL beta = (REAL)beta_d;
#pragma omp parallel for schedule(static)
    for (i64 r = 0; r < R; ++r) {
        REAL hh = 0, vv = 0;
        const REAL* ar = a + r * L;
        const REAL* ur = u + r * L;
        for (i64 t = 0; t < L; ++t) {
            vv = beta * vv + ur[t];
            hh = ar[t] * hh + vv;
            h[r * L + t] = hh;
            if (vout) vout[r * L + t] = vv;
        }
    }
}

/* Adjoint of orc_rows_fwd.  g: dL/dh (R, L).  Writes da (zero at t = 0) and du;
 * either may be NULL. */
void SFX(orc_rows_bwd)(i64 R, i64 L, const REAL* g, const REAL* a, double beta_d,
                       const REAL* h, REAL* da, REAL* du) {
    const REAL beta = (REAL)beta_d;
#pragma omp parallel for schedule(static)
    for (i64 r = 0; r < R; ++r) {
        REAL gh = 0, gv = 0, anext = 0;
        for (i64 t = L - 1; t >= 0; --t) {
            const i64 i = r * L + t;
            gh = g[i] + anext * gh;
            gv = gh + beta * gv;
            if (du) du[i] = gv;
            if (da) da[i] = t > 0 ? gh * h[i - 1] : (REAL)0;
            anext = a[i];
        }
    }
}

/* ---------------------------------------------------------------------------
 * 2x2 scan  x_t = M_t x_{t-1} + F_t , x_{-1} = 0, per (b, p) chain; also the
 * running product Mc_t = M_t Mc_{t-1} (the scanned "A_elements" the reference
 * returns first, mamba_linoss.py:589-594).  cplx != 0: F and X hold complex
 * entries as (re, im) pairs; otherwise real.  Mscan may be NULL.
 * ------------------------------------------------------------------------- */
void SFX(orc_scan2_fwd)(i64 Bsz, i64 L, i64 P, const REAL* M, const REAL* F, int cplx,
                        REAL* Mscan, REAL* X) {
    const i64 nc = cplx ? 2 : 1;
#pragma omp parallel for schedule(static)
    for (i64 bp = 0; bp < Bsz * P; ++bp) {
        const i64 b = bp / P, p = bp % P;
        REAL c11 = 1, c12 = 0, c21 = 0, c22 = 1;
        REAL x1[2] = {0, 0}, x2[2] = {0, 0};
        for (i64 t = 0; t < L; ++t) {
            const REAL* m = M + (b * L + t) * 4 * P;
            const REAL m11 = m[p], m12 = m[P + p], m21 = m[2 * P + p], m22 = m[3 * P + p];
            const REAL* f = F + (b * L + t) * 2 * P * nc;
            REAL* xo = X + (b * L + t) * 2 * P * nc;
            for (i64 c = 0; c < nc; ++c) {
                const REAL n1 = m11 * x1[c] + m12 * x2[c] + f[p * nc + c];
                const REAL n2 = m21 * x1[c] + m22 * x2[c] + f[(P + p) * nc + c];
                x1[c] = n1; x2[c] = n2;
                xo[p * nc + c] = n1;
                xo[(P + p) * nc + c] = n2;
            }
            const REAL e11 = m11 * c11 + m12 * c21, e12 = m11 * c12 + m12 * c22;
            const REAL e21 = m21 * c11 + m22 * c21, e22 = m21 * c12 + m22 * c22;
            c11 = e11; c12 = e12; c21 = e21; c22 = e22;
            if (Mscan) {
                REAL* mo = Mscan + (b * L + t) * 4 * P;
                mo[p] = c11; mo[P + p] = c12; mo[2 * P + p] = c21; mo[3 * P + p] = c22;
            }
        }
    }
}

/* Adjoint of orc_scan2_fwd.  X: forward states; gX: dL/dX (may be NULL);
 * gMs: dL/dMscan (may be NULL, then Mscan is not needed).  Writes dM and dF. */
void SFX(orc_scan2_bwd)(i64 Bsz, i64 L, i64 P, const REAL* M, const REAL* X, int cplx,
                        const REAL* gX, const REAL* Mscan, const REAL* gMs,
                        REAL* dM, REAL* dF) {
    const i64 nc = cplx ? 2 : 1;
#pragma omp parallel for schedule(static)
    for (i64 bp = 0; bp < Bsz * P; ++bp) {
        const i64 b = bp / P, p = bp % P;
        REAL l1[2] = {0, 0}, l2[2] = {0, 0};
        REAL L11 = 0, L12 = 0, L21 = 0, L22 = 0;
        REAL n11 = 0, n12 = 0, n21 = 0, n22 = 0; /* M_{t+1}; zero past the end */
        for (i64 t = L - 1; t >= 0; --t) {
            const REAL* m = M + (b * L + t) * 4 * P;
            REAL* dm = dM + (b * L + t) * 4 * P;
            REAL g11 = 0, g12 = 0, g21 = 0, g22 = 0;
            for (i64 c = 0; c < nc; ++c) {
                const i64 o = (b * L + t) * 2 * P * nc;
                const REAL gx1 = gX ? gX[o + p * nc + c] : (REAL)0;
                const REAL gx2 = gX ? gX[o + (P + p) * nc + c] : (REAL)0;
                /* lambda_t = gX_t + M_{t+1}^T lambda_{t+1} */
                const REAL a1 = gx1 + n11 * l1[c] + n21 * l2[c];
                const REAL a2 = gx2 + n12 * l1[c] + n22 * l2[c];
                l1[c] = a1; l2[c] = a2;
                dF[o + p * nc + c] = a1;
                dF[o + (P + p) * nc + c] = a2;
                REAL p1 = 0, p2 = 0;
                if (t > 0) {
                    const i64 op = (b * L + t - 1) * 2 * P * nc;
                    p1 = X[op + p * nc + c];
                    p2 = X[op + (P + p) * nc + c];
                }
                g11 += a1 * p1; g12 += a1 * p2; g21 += a2 * p1; g22 += a2 * p2;
            }
            if (gMs) {
                const REAL* gm = gMs + (b * L + t) * 4 * P;
                /* Lambda_t = gMs_t + M_{t+1}^T Lambda_{t+1} */
                const REAL e11 = gm[p] + n11 * L11 + n21 * L21;
                const REAL e12 = gm[P + p] + n11 * L12 + n21 * L22;
                const REAL e21 = gm[2 * P + p] + n12 * L11 + n22 * L21;
                const REAL e22 = gm[3 * P + p] + n12 * L12 + n22 * L22;
                L11 = e11; L12 = e12; L21 = e21; L22 = e22;
                REAL q11 = 1, q12 = 0, q21 = 0, q22 = 1; /* Mc_{t-1}, identity at t = 0 */
                if (t > 0) {
                    const REAL* mc = Mscan + (b * L + t - 1) * 4 * P;
                    q11 = mc[p]; q12 = mc[P + p]; q21 = mc[2 * P + p]; q22 = mc[3 * P + p];
                }
                /* dM_t += Lambda_t Mc_{t-1}^T */
                g11 += L11 * q11 + L12 * q12;
                g12 += L11 * q21 + L12 * q22;
                g21 += L21 * q11 + L22 * q12;
                g22 += L21 * q21 + L22 * q22;
            }
            dm[p] = g11; dm[P + p] = g12; dm[2 * P + p] = g21; dm[3 * P + p] = g22;
            n11 = m[p]; n12 = m[P + p]; n21 = m[2 * P + p]; n22 = m[3 * P + p];
        }
    }
}
