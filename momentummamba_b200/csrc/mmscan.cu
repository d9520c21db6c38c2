// C ABI of the momentum selective scan: argument checks, states-per-thread
// choice, dispatch to the kernel families (mmscan_kernels.cuh), and the
// segment-carry folds.
#include "mmscan_kernels.cuh"

namespace mmb {

// States per thread: 2 when 4 would leave the GPU with under two warps per SM
// (too few to hide the recurrence's latency), else 4.  The forward and the
// backward of one call must agree (the checkpoint layout depends on it), so
// this depends only on the shape and element type.
#ifndef MMB_NP2_THRESHOLD_WARPS_PER_SM
#define MMB_NP2_THRESHOLD_WARPS_PER_SM 2
#endif
static int64_t time_chunks(const mmb_mmscan_desc* desc);

static int states_per_thread(const mmb_mmscan_desc* desc) {
    const int64_t N = desc->dstate;
    if (N == 64 || desc->dtype == MMB_BF16) return 4;
    const int64_t threads4 = desc->batch * desc->dim * (N / 4) * time_chunks(desc);
    return threads4 < (int64_t)148 * MMB_NP2_THRESHOLD_WARPS_PER_SM * 32 ? 2 : 4;
}

// ---------------------------------------------------------------------------
// Time chunks.  When the (sequence, channel) pairs of a call give the GPU too
// few warps, the sequence is cut into chunks of T_c steps that separate CTAs
// scan at once: a summary pass gives every chunk its affine map, a carry kernel
// folds the maps into each chunk's incoming state (forward) or adjoint pair
// (backward), and the full pass runs every chunk from its carry.
// ---------------------------------------------------------------------------
// Warps (one-warp backward CTAs of 128 / N channels) below which the library
// splits, and the warps it then aims for.  Measured per call (fwd / bwd, us,
// N = 16, D = 256): B=32 L=1024 (1024 warps) runs 122 / 226 unsplit and
// slower split (130-137 / 288-296); B=8 L=4096 (256 warps) 258 / 495 unsplit,
// 147 / 298 in chunks of 256; B=1 L=65536 (32 warps) 3874 / 7692 unsplit,
// 289 / 601 in chunks of 512.  More chunks than SMs can hold at once still
// pay: the summaries cost a fraction of the full pass.
constexpr int64_t MM_SPLIT_WARPS = 148 * 4;
constexpr int64_t MM_TARGET_WARPS = 148 * 16;
constexpr int64_t MM_MIN_AUTO_CHUNK = 256;  // shortest chunk the library picks

// Steps per time chunk of a call (a multiple of MM_T; >= seqlen: no split).
static int64_t time_chunk_len(const mmb_mmscan_desc* desc) {
    const int64_t L = desc->seqlen;
    int64_t tc;
    if (desc->time_chunk < 0) return L;
    if (desc->time_chunk > 0) {
        tc = desc->time_chunk;
    } else {
        const int64_t warps = desc->batch * ((desc->dim * desc->dstate + 127) / 128);
        if (warps >= MM_SPLIT_WARPS) return L;
        const int64_t want = (MM_TARGET_WARPS + warps - 1) / warps;
        tc = (L + want - 1) / want;
        if (tc < MM_MIN_AUTO_CHUNK) tc = MM_MIN_AUTO_CHUNK;
    }
    tc = (tc + MM_T - 1) / MM_T * MM_T;
    // grid z holds the chunks
    while ((L + tc - 1) / tc > 65535) tc *= 2;
    return tc >= L ? L : tc;
}

static int64_t time_chunks(const mmb_mmscan_desc* desc) {
    const int64_t tc = time_chunk_len(desc);
    return (desc->seqlen + tc - 1) / tc;
}

// Floats of the checkpoints: (h, v) every 8 steps.
static int64_t ckpt_floats(int64_t Bsz, int64_t L, int64_t D, int64_t N) {
    return Bsz * ((L + MM_CK - 1) / MM_CK) * D * N * 2;
}

// Floats after the checkpoints for the chunk carries: per chunk and (b, d) the
// summary [4N] and the carry [2N] (the forward's, then the backward's).
static int64_t chunk_floats(const mmb_mmscan_desc* desc) {
    const int64_t nch = time_chunks(desc);
    return nch > 1 ? nch * desc->batch * desc->dim * desc->dstate * 6 : 0;
}

static double pow_int(double base, int64_t e) {
    double r = 1.0;
    for (; e > 0; e >>= 1) {
        if (e & 1) r *= base;
        base *= base;
    }
    return r;
}

// Incoming (h, v) of every chunk: zeros for chunk 0, then the fold of the
// earlier chunks' summaries [h^0 | v^0 | P | Q'].  One thread per (b, d, n).
// Both folds read each chunk's summary independently of the carried pair, so a
// thread loads MM_CARRY_U chunks' summaries before folding them (one global
// round trip per MM_CARRY_U chunks instead of one per chunk: 17-18 -> 8.4 us
// per launch for 32 chunks at B=2 D=256 N=16).
constexpr int MM_CARRY_U = 8;

__global__ void chunk_carry_fwd_kernel(int64_t BD, int N, int nch, float beta, float betaTc,
                                       const float* __restrict__ summ,
                                       float* __restrict__ state_in) {
    const int64_t total = BD * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bd = e / N, n = e % N;
        float h = 0.f, v = 0.f;
        for (int c0 = 0; c0 < nch; c0 += MM_CARRY_U) {
            float h0[MM_CARRY_U], v0[MM_CARRY_U], P[MM_CARRY_U], Q[MM_CARRY_U];
#pragma unroll
            for (int u = 0; u < MM_CARRY_U; ++u) {
                const int c = c0 + u;
                h0[u] = v0[u] = P[u] = Q[u] = 0.f;
                if (c + 1 < nch) {  // the last chunk's summary is not needed
                    const float* sm = summ + ((int64_t)c * BD + bd) * 4 * N + n;
                    h0[u] = sm[0];
                    v0[u] = sm[N];
                    P[u] = sm[2 * N];
                    Q[u] = sm[3 * N];
                }
            }
#pragma unroll
            for (int u = 0; u < MM_CARRY_U; ++u) {
                const int c = c0 + u;
                if (c < nch) {
                    float* o = state_in + ((int64_t)c * BD + bd) * 2 * N;
                    o[n] = h;
                    o[N + n] = v;
                    const float hn = fmaf(P[u], h, fmaf(beta * Q[u], v, h0[u]));
                    v = fmaf(betaTc, v, v0[u]);
                    h = hn;
                }
            }
        }
    }
}

// Adjoint pair arriving at the end of every chunk: zeros for the last chunk,
// then the fold of the later chunks' summaries [lam^0 | mu^0 | P | Q'].
__global__ void chunk_carry_bwd_kernel(int64_t BD, int N, int nch, float betaTc,
                                       const float* __restrict__ gsumm,
                                       float* __restrict__ gstate_in) {
    const int64_t total = BD * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bd = e / N, n = e % N;
        float lam = 0.f, mu = 0.f;
        for (int c0 = nch - 1; c0 >= 0; c0 -= MM_CARRY_U) {
            float l0[MM_CARRY_U], m0[MM_CARRY_U], P[MM_CARRY_U], Q[MM_CARRY_U];
#pragma unroll
            for (int u = 0; u < MM_CARRY_U; ++u) {
                const int c = c0 - u;
                l0[u] = m0[u] = P[u] = Q[u] = 0.f;
                if (c > 0) {  // the first chunk's summary is not needed
                    const float* g = gsumm + ((int64_t)c * BD + bd) * 4 * N + n;
                    l0[u] = g[0];
                    m0[u] = g[N];
                    P[u] = g[2 * N];
                    Q[u] = g[3 * N];
                }
            }
#pragma unroll
            for (int u = 0; u < MM_CARRY_U; ++u) {
                const int c = c0 - u;
                if (c >= 0) {
                    float* o = gstate_in + ((int64_t)c * BD + bd) * 2 * N;
                    o[n] = lam;
                    o[N + n] = mu;
                    // nothing arrives after the last chunk: (lam, mu) are zero
                    // there, so the general fold gives (lam^0, mu^0)
                    mu = fmaf(Q[u], lam, fmaf(betaTc, mu, m0[u]));
                    lam = fmaf(P[u], lam, l0[u]);
                }
            }
        }
    }
}

static unsigned chunk_carry_blocks(int64_t BD, int64_t N) {
    const int64_t blocks = (BD * N + 255) / 256;
    return (unsigned)(blocks < 148 * 16 ? blocks : 148 * 16);
}

static bool aligned16(const void* ptr) { return ptr == nullptr || ((uintptr_t)ptr & 15) == 0; }

// Shape, pointer and stride checks shared by every entry point; fills the
// activation part of p.
static int fill_params(const mmb_mmscan_desc* desc, const void* x, const void* delta,
                       const float* A, const void* B, const void* C, const float* D,
                       const void* z, const float* dbias, MMParams& p) {
    if (!desc || !delta || !A) return MMB_ERR_NULL;
    if (desc->batch <= 0 || desc->seqlen <= 0 || desc->dim <= 0) return MMB_ERR_SHAPE;
    if (desc->batch > 65535) return MMB_ERR_SHAPE;
    const int64_t N = desc->dstate;
    if (N != 8 && N != 16 && N != 32 && N != 64) return MMB_ERR_UNSUPPORTED;
    if (desc->dtype != MMB_F32 && desc->dtype != MMB_BF16) return MMB_ERR_UNSUPPORTED;
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
    p.tchunk = p.L;  // one time chunk unless the call splits
    p.zoff = 0;
    p.nz = 1;
    // 16-byte staging: 4 fp32 or 8 bf16 elements per copy
    const int64_t q = desc->dtype == MMB_BF16 ? 8 : 4;
    bool vec = aligned16(x) && aligned16(delta) && aligned16(z) && aligned16(B) && aligned16(C) &&
               (p.D % q == 0);
    for (int i = 0; i < 2; ++i)
        vec = vec && (!x || p.xs[i] % q == 0) && (p.ds[i] % q == 0) && (!z || p.zs[i] % q == 0) &&
              (!B || p.bs[i] % q == 0) && (p.cs[i] % q == 0);
    p.vec = vec ? 1 : 0;
    if (desc->dtype == MMB_BF16 && !vec) return MMB_ERR_ALIGN;
    return MMB_OK;
}

static int launch(const mmb_mmscan_desc* desc, const MMParams& p, int kind, cudaStream_t s) {
    const int np = states_per_thread(desc);
    const bool fwd = kind == MM_FWD || kind == MM_FWD_SUMMARY;
    if (desc->dtype == MMB_BF16)
        return fwd ? mmscan_launch<ElemBF16, true>(p, desc->dstate, np, kind, s)
                   : mmscan_launch<ElemBF16, false>(p, desc->dstate, np, kind, s);
    return fwd ? mmscan_launch<ElemF32, true>(p, desc->dstate, np, kind, s)
               : mmscan_launch<ElemF32, false>(p, desc->dstate, np, kind, s);
}

static int forward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t, cudaStream_t s) {
    if (!t) return MMB_ERR_NULL;
    MMParams p;
    int st = fill_params(desc, t->x, t->delta, t->A, t->B, t->C, t->D, t->z, t->delta_bias, p);
    if (st != MMB_OK) return st;
    if (!t->x || !t->B || !t->C || !t->out) return MMB_ERR_NULL;
    if (!aligned16(t->ckpt) || !aligned16(t->state_in) || !aligned16(t->state_out))
        return MMB_ERR_ALIGN;
    p.out = t->out;
    p.ckpt = t->ckpt;
    p.state_in = t->state_in;
    p.state_out = t->state_out;
    const int64_t nch = time_chunks(desc);
    if (nch <= 1 || !t->ckpt || t->state_in || t->state_out) return launch(desc, p, MM_FWD, s);

    // split along time: chunk summaries, their fold, the full pass
    const int64_t tc = time_chunk_len(desc), BD = p.Bsz * p.D, N = desc->dstate;
    float* summ = t->ckpt + ckpt_floats(p.Bsz, p.L, p.D, N);
    float* sin = summ + nch * BD * 4 * N;
    MMParams ps = p;
    ps.z = nullptr;
    ps.Cm = nullptr;
    ps.ckpt = nullptr;
    ps.summary = summ;
    ps.tchunk = tc;
    ps.nz = (int)(nch - 1);
    st = launch(desc, ps, MM_FWD_SUMMARY, s);
    if (st != MMB_OK) return st;
    const float betaTc = (float)pow_int((double)desc->beta, tc);
    chunk_carry_fwd_kernel<<<chunk_carry_blocks(BD, N), 256, 0, s>>>(BD, (int)N, (int)nch,
                                                                      desc->beta, betaTc, summ, sin);
    st = mmb_launch_status();
    if (st != MMB_OK) return st;
    p.state_in = sin;
    p.tchunk = tc;
    p.nz = (int)nch;
    return launch(desc, p, MM_FWD, s);
}

// Zeroing of the backward's atomic sums.  dB and dC (16-byte aligned, length a
// multiple of 4) take float4 stores; dA, dD and d(delta_bias) scalar ones.
struct ZeroList {
    float* p[5];
    int64_t n[5];
};
__global__ void zero_sums_kernel(const ZeroList z) {
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int k = 0; k < 5; ++k) {
        if (!z.p[k]) continue;
        if (k < 2) {
            float4* q = reinterpret_cast<float4*>(z.p[k]);
            for (int64_t e = i0; e < z.n[k] / 4; e += step) q[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (int64_t e = i0; e < z.n[k]; e += step) z.p[k][e] = 0.f;
        }
    }
}

static int backward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t, cudaStream_t s) {
    if (!t) return MMB_ERR_NULL;
    MMParams p;
    int st = fill_params(desc, t->x, t->delta, t->A, t->B, t->C, t->D, t->z, t->delta_bias, p);
    if (st != MMB_OK) return st;
    if (!t->ckpt) return MMB_ERR_WORKSPACE;
    if (!t->x || !t->B || !t->C || !t->dout || !t->dx || !t->ddelta || !t->dA || !t->dB ||
        !t->dC)
        return MMB_ERR_NULL;
    if (!aligned16(t->ckpt) || !aligned16(t->dout) || !aligned16(t->dB) || !aligned16(t->dC) ||
        !aligned16(t->gstate_in) || !aligned16(t->gstate_out))
        return MMB_ERR_ALIGN;
    // the incoming adjoint pair enters at the last step of an 8-step window
    if (t->gstate_in && desc->seqlen % MM_CK != 0) return MMB_ERR_SHAPE;
    p.ckpt_in = t->ckpt;
    p.dout = t->dout;
    p.gstate_in = t->gstate_in;
    p.gstate_out = t->gstate_out;
    p.dx = t->dx; p.ddelta = t->ddelta; p.dA = t->dA; p.dB = t->dB; p.dC = t->dC;
    p.dD = t->D ? t->dD : nullptr;
    p.dz = t->z ? t->dz : nullptr;
    p.ddbias = t->delta_bias ? t->ddelta_bias : nullptr;
    const int64_t N = desc->dstate;
    const size_t bln = (size_t)(p.Bsz * p.L * N) * sizeof(float);
    const size_t dsz = (size_t)p.D * sizeof(float);
    // the sums are accumulated with atomics: clear them on the stream first,
    // all five in one launch
    ZeroList zl{};
    float* const sums[5] = {p.dB, p.dC, p.dA, p.dD, p.ddbias};
    const size_t bytes[5] = {bln, bln, (size_t)N * dsz, dsz, dsz};
    int64_t total = 0;
    for (int i = 0; i < 5; ++i) {
        zl.p[i] = sums[i];
        zl.n[i] = sums[i] ? (int64_t)(bytes[i] / sizeof(float)) : 0;
        total += zl.n[i];
    }
    const int64_t blocks = min64((total / 4 + 255) / 256 + 1, 148 * 4);
    zero_sums_kernel<<<(unsigned)blocks, 256, 0, s>>>(zl);
    const int zst = mmb_launch_status();
    if (zst != MMB_OK) return zst;
    const int64_t nch = time_chunks(desc);
    if (nch <= 1 || t->gstate_in || t->gstate_out) return launch(desc, p, MM_BWD, s);

    // split along time: summaries of chunks 1.. (adjoint pair from zero and
    // the chunk's P, Q'), their fold from the end, the full pass
    const int64_t tc = time_chunk_len(desc), BD = p.Bsz * p.D;
    float* gsumm = t->ckpt + ckpt_floats(p.Bsz, p.L, p.D, N);
    float* gin = gsumm + nch * BD * 4 * N;
    MMParams ps = p;
    ps.x = nullptr;
    ps.Bm = nullptr;
    ps.summary = gsumm;
    ps.bsum_pq = 1;
    ps.tchunk = tc;
    ps.zoff = 1;
    ps.nz = (int)(nch - 1);
    st = launch(desc, ps, MM_BWD_SUMMARY, s);
    if (st != MMB_OK) return st;
    const float betaTc = (float)pow_int((double)desc->beta, tc);
    chunk_carry_bwd_kernel<<<chunk_carry_blocks(BD, N), 256, 0, s>>>(BD, (int)N, (int)nch, betaTc,
                                                                      gsumm, gin);
    st = mmb_launch_status();
    if (st != MMB_OK) return st;
    p.gstate_in = gin;
    p.tchunk = tc;
    p.nz = (int)nch;
    return launch(desc, p, MM_BWD, s);
}

// ---------------------------------------------------------------------------
// segment-carry folds: one thread per (b, d, n)
// ---------------------------------------------------------------------------
struct CarryArgs {
    int nseg, seg;
    int64_t BD, N;
    float beta;
    float betaT[MMB_MAX_SEGMENTS];  // beta^(length of segment j)
};

__global__ void carry_fwd_kernel(const CarryArgs a, const float* __restrict__ summ,
                                 float* __restrict__ state_in) {
    const int64_t total = a.BD * a.N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bd = e / a.N, n = e % a.N;
        float h = 0.f, v = 0.f;
        for (int j = 0; j < a.seg; ++j) {
            const float* s = summ + ((int64_t)j * a.BD + bd) * 4 * a.N;
            const float hn = fmaf(s[2 * a.N + n], h, fmaf(a.beta * s[3 * a.N + n], v, s[n]));
            v = fmaf(a.betaT[j], v, s[a.N + n]);
            h = hn;
        }
        state_in[bd * 2 * a.N + n] = h;
        state_in[bd * 2 * a.N + a.N + n] = v;
    }
}

__global__ void carry_bwd_kernel(const CarryArgs a, const float* __restrict__ summ,
                                 const float* __restrict__ gsumm, float* __restrict__ gstate_in) {
    const int64_t total = a.BD * a.N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bd = e / a.N, n = e % a.N;
        float lam = 0.f, mu = 0.f;
        for (int j = a.nseg - 1; j > a.seg; --j) {
            const float* s = summ + ((int64_t)j * a.BD + bd) * 4 * a.N;
            const float* g = gsumm + ((int64_t)j * a.BD + bd) * 2 * a.N;
            const float P = s[2 * a.N + n], Q = s[3 * a.N + n];
            mu = fmaf(Q, lam, fmaf(a.betaT[j], mu, g[a.N + n]));
            lam = fmaf(P, lam, g[n]);
        }
        gstate_in[bd * 2 * a.N + n] = lam;
        gstate_in[bd * 2 * a.N + a.N + n] = mu;
    }
}

static int carry_args(int64_t nseg, int64_t seg, const int64_t* seg_len, int64_t batch,
                      int64_t dim, int64_t dstate, float beta, CarryArgs& a) {
    if (!seg_len) return MMB_ERR_NULL;
    if (nseg <= 0 || nseg > MMB_MAX_SEGMENTS || seg < 0 || seg >= nseg) return MMB_ERR_SHAPE;
    if (batch <= 0 || dim <= 0 || dstate <= 0) return MMB_ERR_SHAPE;
    a = CarryArgs{};
    a.nseg = (int)nseg;
    a.seg = (int)seg;
    a.BD = batch * dim;
    a.N = dstate;
    a.beta = beta;
    for (int64_t j = 0; j < nseg; ++j) {
        if (seg_len[j] <= 0) return MMB_ERR_SHAPE;
        // beta^T by squaring in double (T up to 2^63)
        double r = 1.0, base = (double)beta;
        for (int64_t e = seg_len[j]; e > 0; e >>= 1) {
            if (e & 1) r *= base;
            base *= base;
        }
        a.betaT[j] = (float)r;
    }
    return MMB_OK;
}

static dim3 carry_grid(const CarryArgs& a) {
    const int64_t blocks = (a.BD * a.N + 255) / 256;
    return dim3((unsigned)(blocks < 148 * 16 ? blocks : 148 * 16));
}

}  // namespace mmb

using namespace mmb;

extern "C" size_t mmb_mmscan_workspace_floats(const mmb_mmscan_desc* desc) {
    if (!desc || desc->batch <= 0 || desc->seqlen <= 0 || desc->dim <= 0 || desc->dstate <= 0)
        return 0;
    return (size_t)(ckpt_floats(desc->batch, desc->seqlen, desc->dim, desc->dstate) +
                    chunk_floats(desc));
}

extern "C" size_t mmb_mmscan_ckpt_floats(int64_t batch, int64_t seqlen, int64_t dim,
                                         int64_t dstate) {
    mmb_mmscan_desc d{};
    d.batch = batch;
    d.seqlen = seqlen;
    d.dim = dim;
    d.dstate = dstate;
    return mmb_mmscan_workspace_floats(&d);
}

extern "C" int mmb_mmscan_fwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                              const float* A, const float* B, const float* C, const float* D,
                              const float* z, const float* delta_bias, float* out, float* ckpt,
                              mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_fwd");
    if (desc && desc->dtype != MMB_F32) return MMB_ERR_UNSUPPORTED;
    mmb_mmscan_tensors t{};
    t.x = x; t.delta = delta; t.z = z; t.B = B; t.C = C; t.A = A; t.D = D; t.delta_bias = delta_bias;
    t.out = out;
    t.ckpt = ckpt;
    return forward(desc, &t, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_bwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                              const float* A, const float* B, const float* C, const float* D,
                              const float* z, const float* delta_bias, float* ckpt,
                              const float* dout, float* dx, float* ddelta, float* dA, float* dB,
                              float* dC, float* dD, float* dz, float* ddelta_bias,
                              mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_bwd");
    if (desc && desc->dtype != MMB_F32) return MMB_ERR_UNSUPPORTED;
    mmb_mmscan_tensors t{};
    t.x = x; t.delta = delta; t.z = z; t.B = B; t.C = C; t.A = A; t.D = D; t.delta_bias = delta_bias;
    t.ckpt = ckpt;
    t.dout = dout;
    t.dx = dx; t.ddelta = ddelta; t.dz = dz;
    t.dA = dA; t.dB = dB; t.dC = dC; t.dD = dD; t.ddelta_bias = ddelta_bias;
    return backward(desc, &t, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_forward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                                  mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_forward");
    return forward(desc, t, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_backward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                                   mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_backward");
    return backward(desc, t, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_fwd_summary(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                                      float* summary, mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_fwd_summary");
    if (!t) return MMB_ERR_NULL;
    MMParams p;
    // the summary reads x, delta, B, A, delta_bias only
    int st = fill_params(desc, t->x, t->delta, t->A, t->B, nullptr, nullptr, nullptr,
                         t->delta_bias, p);
    if (st != MMB_OK) return st;
    if (!t->x || !t->B || !summary) return MMB_ERR_NULL;
    if (!aligned16(summary)) return MMB_ERR_ALIGN;
    p.summary = summary;
    return launch(desc, p, MM_FWD_SUMMARY, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_bwd_summary(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                                      float* gsummary, mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_bwd_summary");
    if (!t) return MMB_ERR_NULL;
    MMParams p;
    // reads delta, z, dout, C, A, delta_bias
    int st = fill_params(desc, nullptr, t->delta, t->A, nullptr, t->C, nullptr, t->z,
                         t->delta_bias, p);
    if (st != MMB_OK) return st;
    if (!t->C || !t->dout || !gsummary) return MMB_ERR_NULL;
    if (!aligned16(t->dout) || !aligned16(gsummary)) return MMB_ERR_ALIGN;
    p.dout = t->dout;
    p.summary = gsummary;
    return launch(desc, p, MM_BWD_SUMMARY, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_mmscan_carry_fwd(int64_t nseg, int64_t seg, const int64_t* seg_len,
                                    int64_t batch, int64_t dim, int64_t dstate, float beta,
                                    const float* summaries, float* state_in,
                                    mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_carry_fwd");
    CarryArgs a;
    const int st = carry_args(nseg, seg, seg_len, batch, dim, dstate, beta, a);
    if (st != MMB_OK) return st;
    if (!summaries || !state_in) return MMB_ERR_NULL;
    carry_fwd_kernel<<<carry_grid(a), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        a, summaries, state_in);
    return mmb_launch_status();
}

extern "C" int mmb_mmscan_carry_bwd(int64_t nseg, int64_t seg, const int64_t* seg_len,
                                    int64_t batch, int64_t dim, int64_t dstate, float beta,
                                    const float* summaries, const float* gsummaries,
                                    float* gstate_in, mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_carry_bwd");
    CarryArgs a;
    const int st = carry_args(nseg, seg, seg_len, batch, dim, dstate, beta, a);
    if (st != MMB_OK) return st;
    if (!summaries || !gsummaries || !gstate_in) return MMB_ERR_NULL;
    carry_bwd_kernel<<<carry_grid(a), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        a, summaries, gsummaries, gstate_in);
    return mmb_launch_status();
}
