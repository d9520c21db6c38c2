// The momentum block's producer and its single-token decode, for sm_100a.
//
//  * causal depthwise conv1d + SiLU over (B, L, D) activations (the block's
//    x branch, mamba_momentum.py:217-223): out[b,t,d] = silu(bias[d] +
//    sum_k w[d,k] x[b, t-(W-1)+k, d]), inputs before t = 0 taken from an
//    optional conv state (zeros otherwise); forward and backward.
//  * decode: the conv-cache step (mamba_momentum.py:455-459, :466) and the
//    single-token momentum state update with the dt softplus and the SiLU(z)
//    gate fused (mamba_momentum.py:473-515 and :461-464).
//
// Layout: D is the unit-stride dimension everywhere, so a warp covers 32
// consecutive channels and every global access is a coalesced 128-byte row.
// A thread of the sequence kernels walks a chunk of time steps of one channel
// with the W-1 previous inputs in registers.
#include "mmb_common.cuh"

namespace mmb {

constexpr int CV_MAXW = 8;    // largest conv width compiled
constexpr int CV_TCHUNK = 64; // time steps per thread
constexpr int CV_NT = 128;

__device__ __forceinline__ float silu_f(float u) { return u * sigmoid_f(u); }
// d silu / du = s (1 + u (1 - s)), s = sigmoid(u)
__device__ __forceinline__ float silu_grad(float u) {
    const float s = sigmoid_f(u);
    return s * (1.f + u * (1.f - s));
}

struct ConvParams {
    int64_t Bsz, L, D;
    int W;
    const float* x;  // (B, L, D) with strides xs[0], xs[1]
    int64_t xs[2];
    const float* w;     // (D, W)
    const float* bias;  // (D) or null
    const float* state_in;  // (B, D, W-1) inputs before t = 0, or null
    float* state_out;       // (B, D, W-1) the last W-1 inputs, or null
    float* out;             // (B, L, D)
    // backward
    const float* dout;
    float* dx;     // (B, L, D)
    float* dw;     // (D, W) sums
    float* dbias;  // (D) sums or null
};

// input x[b, t, d], the conv state for t < 0, zero before that
__device__ __forceinline__ float conv_in(const ConvParams& p, int64_t b, int64_t t, int64_t d) {
    if (t >= 0) return t < p.L ? p.x[b * p.xs[0] + t * p.xs[1] + d] : 0.f;
    const int64_t k = (p.W - 1) + t;  // position in the state, 0 = oldest
    if (p.state_in && k >= 0) return p.state_in[(b * p.D + d) * (p.W - 1) + k];
    return 0.f;
}

template <int W>
__global__ void __launch_bounds__(CV_NT) conv_silu_fwd_kernel(const ConvParams p) {
    const int64_t d = (int64_t)blockIdx.x * CV_NT + threadIdx.x;
    const int64_t b = blockIdx.z;
    const int64_t t0 = (int64_t)blockIdx.y * CV_TCHUNK;
    if (d >= p.D) return;
    float w[W];
#pragma unroll
    for (int k = 0; k < W; ++k) w[k] = p.w[d * W + k];
    const float bs = p.bias ? p.bias[d] : 0.f;
    float win[W];  // win[W-1] = x[t], win[0] = x[t-W+1]
#pragma unroll
    for (int k = 0; k < W - 1; ++k) win[k] = conv_in(p, b, t0 - (W - 1) + k, d);
    const int64_t t1 = min64(t0 + CV_TCHUNK, p.L);
    const float* xp = p.x + b * p.xs[0] + d;
    float* op = p.out + b * p.L * p.D + d;
    for (int64_t t = t0; t < t1; ++t) {
        win[W - 1] = xp[t * p.xs[1]];
        float acc = bs;
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(w[k], win[k], acc);
        op[t * p.D] = silu_f(acc);
#pragma unroll
        for (int k = 0; k < W - 1; ++k) win[k] = win[k + 1];
    }
    // the last W-1 inputs (the decode cache), by the chunk holding the end
    if (p.state_out && t1 == p.L) {
#pragma unroll
        for (int k = 0; k < W - 1; ++k)
            p.state_out[(b * p.D + d) * (W - 1) + k] = conv_in(p, b, p.L - (W - 1) + k, d);
    }
}

// Backward: g[t] = dout[t] silu'(pre[t]); dx[t] = sum_k w[k] g[t + W-1-k];
// dw[k] = sum g[t] x[t-(W-1)+k]; dbias = sum g.  A thread walks its chunk
// backwards with the W-1 later g values and the W-1 earlier inputs in
// registers.
template <int W>
__global__ void __launch_bounds__(CV_NT) conv_silu_bwd_kernel(const ConvParams p) {
    const int64_t d = (int64_t)blockIdx.x * CV_NT + threadIdx.x;
    const int64_t b = blockIdx.z;
    const int64_t t0 = (int64_t)blockIdx.y * CV_TCHUNK;
    if (d >= p.D) return;
    float w[W];
#pragma unroll
    for (int k = 0; k < W; ++k) w[k] = p.w[d * W + k];
    const float bs = p.bias ? p.bias[d] : 0.f;
    const int64_t t1 = min64(t0 + CV_TCHUNK, p.L);
    const float* dop = p.dout + b * p.L * p.D + d;
    // g at t (computed from the input window ending at t)
    auto g_at = [&](int64_t t, const float (&win)[W]) {
        float acc = bs;
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(w[k], win[k], acc);
        return dop[t * p.D] * silu_grad(acc);
    };
    // inputs x[t1-W+1 .. t1-1 + (W-1)] and g[t1 .. t1+W-2] (the halo after the chunk)
    float gl[W];  // gl[j] = g[t + j] for j = 1..W-1 (gl[0] = g[t])
    float xw[2 * W];  // x[t-W+1 .. t+W-1]: xw[i] = x[t - (W-1) + i]
#pragma unroll
    for (int i = 0; i < 2 * W - 1; ++i) xw[i] = conv_in(p, b, t1 - 1 - (W - 1) + i, d);
    // g beyond the chunk: g[t1 + j - 1] for j = 1..W-1, each from its own window
#pragma unroll
    for (int j = 1; j < W; ++j) {
        const int64_t t = t1 - 1 + j;
        float g = 0.f;
        if (t < p.L) {
            float win[W];
#pragma unroll
            for (int k = 0; k < W; ++k) win[k] = xw[j + k];
            g = g_at(t, win);
        }
        gl[j] = g;
    }
    float dwacc[W], dbacc = 0.f;
#pragma unroll
    for (int k = 0; k < W; ++k) dwacc[k] = 0.f;
    float* dxp = p.dx + b * p.L * p.D + d;
    for (int64_t t = t1 - 1; t >= t0; --t) {
        // window for t: xw[0 .. W-1] = x[t-W+1 .. t]
        float win[W];
#pragma unroll
        for (int k = 0; k < W; ++k) win[k] = xw[k];
        const float g = g_at(t, win);
        gl[0] = g;
        dbacc += g;
#pragma unroll
        for (int k = 0; k < W; ++k) dwacc[k] = fmaf(g, win[k], dwacc[k]);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(w[k], gl[W - 1 - k], acc);
        dxp[t * p.D] = acc;
        // shift: the next (earlier) step
#pragma unroll
        for (int j = W - 1; j > 0; --j) gl[j] = gl[j - 1];
#pragma unroll
        for (int i = 2 * W - 2; i > 0; --i) xw[i] = xw[i - 1];
        xw[0] = conv_in(p, b, t - W, d);
    }
#pragma unroll
    for (int k = 0; k < W; ++k) atomicAdd(p.dw + d * W + k, dwacc[k]);
    if (p.dbias) atomicAdd(p.dbias + d, dbacc);
}

template <int W>
static int conv_launch(const ConvParams& p, bool fwd, cudaStream_t s) {
    dim3 grid((unsigned)((p.D + CV_NT - 1) / CV_NT), (unsigned)((p.L + CV_TCHUNK - 1) / CV_TCHUNK),
              (unsigned)p.Bsz);
    if (fwd)
        conv_silu_fwd_kernel<W><<<grid, CV_NT, 0, s>>>(p);
    else
        conv_silu_bwd_kernel<W><<<grid, CV_NT, 0, s>>>(p);
    return mmb_launch_status();
}

static int conv_dispatch(const ConvParams& p, bool fwd, cudaStream_t s) {
    switch (p.W) {
        case 2: return conv_launch<2>(p, fwd, s);
        case 3: return conv_launch<3>(p, fwd, s);
        case 4: return conv_launch<4>(p, fwd, s);
        case 5: return conv_launch<5>(p, fwd, s);
        case 6: return conv_launch<6>(p, fwd, s);
        case 7: return conv_launch<7>(p, fwd, s);
        case 8: return conv_launch<8>(p, fwd, s);
        default: return MMB_ERR_UNSUPPORTED;
    }
}

static int conv_fill(int64_t batch, int64_t seqlen, int64_t dim, int32_t width, const float* x,
                     const int64_t* x_stride, const float* weight, const float* bias,
                     ConvParams& p) {
    if (!x || !x_stride || !weight) return MMB_ERR_NULL;
    if (batch <= 0 || batch > 65535 || seqlen <= 0 || dim <= 0) return MMB_ERR_SHAPE;
    if (width < 2 || width > CV_MAXW) return MMB_ERR_UNSUPPORTED;
    if ((seqlen + CV_TCHUNK - 1) / CV_TCHUNK > 65535) return MMB_ERR_SHAPE;
    p = ConvParams{};
    p.Bsz = batch; p.L = seqlen; p.D = dim; p.W = width;
    p.x = x; p.xs[0] = x_stride[0]; p.xs[1] = x_stride[1];
    p.w = weight; p.bias = bias;
    return MMB_OK;
}

// ---------------------------------------------------------------------------
// decode: conv-cache step and momentum state step
// ---------------------------------------------------------------------------
__global__ void conv_step_kernel(int64_t Bsz, int64_t D, int W, const float* x, int64_t xs,
                                 const float* state_in, float* state_out, const float* w,
                                 const float* bias, float* out) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= Bsz * D) return;
    const int64_t b = e / D, d = e % D;
    const float* si = state_in + e * (W - 1);
    float* so = state_out + e * (W - 1);
    float win[CV_MAXW];
    for (int k = 0; k < W - 1; ++k) win[k] = si[k];  // all reads before any write (in place)
    const float xn = x[b * xs + d];
    win[W - 1] = xn;
    float acc = bias ? bias[d] : 0.f;
    for (int k = 0; k < W; ++k) acc = fmaf(w[d * W + k], win[k], acc);
    out[e] = silu_f(acc);
    for (int k = 0; k < W - 1; ++k) so[k] = win[k + 1];
}

struct StepParams {
    int64_t Bsz, D, N;
    const float *x, *delta, *z, *Bm, *Cm;  // rows of (B, ...) with the row strides below
    int64_t xs, ds, zs, bs, cs;
    const float *A, *Dskip, *dbias;
    const float *h_in, *v_in;  // element (b, d, n) at b*ss[0] + d*ss[1] + n
    float *h, *v;              // same layout; may equal h_in, v_in
    int64_t ss[2];
    float beta, alpha;
    int softplus;
    float* out;  // (B, D)
};

// One thread per (b, d); its N states in a loop (N <= 64).
__global__ void mmscan_step_kernel(const StepParams p) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= p.Bsz * p.D) return;
    const int64_t b = e / p.D, d = e % p.D;
    const float xv = p.x[b * p.xs + d];
    float dt = p.delta[b * p.ds + d] + (p.dbias ? p.dbias[d] : 0.f);
    if (p.softplus) dt = softplus_f(dt);
    const float dtx = p.alpha * dt * xv;
    const float* Br = p.Bm + b * p.bs;
    const float* Cr = p.Cm + b * p.cs;
    const float* Ar = p.A + d * p.N;
    const int64_t so = b * p.ss[0] + d * p.ss[1];
    const float* hi = p.h_in ? p.h_in + so : nullptr;  // null: zero state
    const float* vi = p.v_in ? p.v_in + so : nullptr;
    float* hr = p.h + so;
    float* vr = p.v + so;
    float y = 0.f;
    for (int64_t n = 0; n < p.N; ++n) {
        const float a = ex2(dt * Ar[n] * MMB_LOG2E);
        const float vn = fmaf(p.beta, vi ? vi[n] : 0.f, dtx * Br[n]);
        const float hn = fmaf(a, hi ? hi[n] : 0.f, vn);
        vr[n] = vn;
        hr[n] = hn;
        y = fmaf(Cr[n], hn, y);
    }
    if (p.Dskip) y = fmaf(p.Dskip[d], xv, y);
    if (p.z) {
        const float zv = p.z[b * p.zs + d];
        y *= silu_f(zv);
    }
    p.out[e] = y;
}

}  // namespace mmb

using namespace mmb;

extern "C" int mmb_conv1d_silu_fwd(int64_t batch, int64_t seqlen, int64_t dim, int32_t width,
                                   const float* x, const int64_t* x_stride, const float* weight,
                                   const float* bias, const float* state_in, float* state_out,
                                   float* out, mmb_stream_t stream) {
    MMB_NVTX("mmb_conv1d_silu_fwd");
    ConvParams p;
    int st = conv_fill(batch, seqlen, dim, width, x, x_stride, weight, bias, p);
    if (st != MMB_OK) return st;
    if (!out) return MMB_ERR_NULL;
    p.state_in = state_in;
    p.state_out = state_out;
    p.out = out;
    return conv_dispatch(p, true, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mmb_conv1d_silu_bwd(int64_t batch, int64_t seqlen, int64_t dim, int32_t width,
                                   const float* x, const int64_t* x_stride, const float* weight,
                                   const float* bias, const float* state_in, const float* dout,
                                   float* dx, float* dweight, float* dbias, mmb_stream_t stream) {
    MMB_NVTX("mmb_conv1d_silu_bwd");
    ConvParams p;
    int st = conv_fill(batch, seqlen, dim, width, x, x_stride, weight, bias, p);
    if (st != MMB_OK) return st;
    if (!dout || !dx || !dweight) return MMB_ERR_NULL;
    p.state_in = state_in;
    p.dout = dout;
    p.dx = dx;
    p.dw = dweight;
    p.dbias = bias ? dbias : nullptr;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(dweight, 0, (size_t)(dim * width) * sizeof(float), s);
    if (e == cudaSuccess && p.dbias) e = cudaMemsetAsync(p.dbias, 0, (size_t)dim * sizeof(float), s);
    if (e != cudaSuccess) {
        mmb_record_cuda_error(e);
        return MMB_ERR_LAUNCH;
    }
    return conv_dispatch(p, false, s);
}

extern "C" int mmb_conv1d_step(int64_t batch, int64_t dim, int32_t width, const float* x,
                               int64_t x_row_stride, const float* state_in, float* state_out,
                               const float* weight, const float* bias, float* out,
                               mmb_stream_t stream) {
    MMB_NVTX("mmb_conv1d_step");
    if (!x || !state_in || !state_out || !weight || !out) return MMB_ERR_NULL;
    if (batch <= 0 || dim <= 0) return MMB_ERR_SHAPE;
    if (width < 2 || width > CV_MAXW) return MMB_ERR_UNSUPPORTED;
    const int64_t n = batch * dim;
    conv_step_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        batch, dim, width, x, x_row_stride, state_in, state_out, weight, bias, out);
    return mmb_launch_status();
}

extern "C" int mmb_mmscan_step(const mmb_step_desc* desc, const float* x, const float* delta,
                               const float* A, const float* B, const float* C, const float* D,
                               const float* z, const float* delta_bias, const float* h_in,
                               const float* v_in, float* h, float* v, float* out,
                               mmb_stream_t stream) {
    MMB_NVTX("mmb_mmscan_step");
    if (!desc || !x || !delta || !A || !B || !C || !h || !v || !out) return MMB_ERR_NULL;
    if (desc->batch <= 0 || desc->dim <= 0 || desc->dstate <= 0 || desc->dstate > 256)
        return MMB_ERR_SHAPE;
    StepParams p{};
    p.Bsz = desc->batch; p.D = desc->dim; p.N = desc->dstate;
    p.x = x; p.delta = delta; p.z = z; p.Bm = B; p.Cm = C;
    p.xs = desc->x_row_stride; p.ds = desc->delta_row_stride; p.zs = desc->z_row_stride;
    p.bs = desc->B_row_stride; p.cs = desc->C_row_stride;
    p.A = A; p.Dskip = D; p.dbias = delta_bias;
    p.h_in = h_in; p.v_in = v_in; p.h = h; p.v = v;
    p.ss[0] = desc->state_stride[0]; p.ss[1] = desc->state_stride[1];
    p.beta = desc->beta; p.alpha = desc->alpha;
    p.softplus = desc->delta_softplus != 0;
    p.out = out;
    const int64_t n = p.Bsz * p.D;
    mmscan_step_kernel<<<(unsigned)((n + 127) / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
    return mmb_launch_status();
}
