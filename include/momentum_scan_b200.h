/*
 * momentum_scan_b200 -- C ABI of the B200 (sm_100a) momentum selective scan and
 * LinOSS 2x2 scan kernels.
 *
 * Conventions shared by every entry point:
 *   - all tensors are fp32 device pointers owned by the caller; the library never
 *     allocates device memory.  Workspaces (forward checkpoints, chunk carries)
 *     are caller-owned too; their size comes from the matching *_floats query.
 *   - strides are in elements; the innermost dimension is always unit-stride.
 *   - every call is asynchronous on `stream` (a cudaStream_t) and returns an
 *     mmb_status; nothing synchronises the device.
 *   - outputs are fully overwritten (gradient outputs that are sums over batch
 *     or channels are cleared on `stream` before they are accumulated).
 *   - nullable pointers are marked; a NULL there means "input absent" (for
 *     inputs) or "not wanted" (for outputs).
 */
#ifndef MOMENTUM_SCAN_B200_H
#define MOMENTUM_SCAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mmb_status {
    MMB_OK = 0,
    MMB_ERR_NULL = 1,        /* a required pointer is NULL */
    MMB_ERR_SHAPE = 2,       /* a size or stride is out of range */
    MMB_ERR_ALIGN = 3,       /* a pointer or stride breaks the stated alignment */
    MMB_ERR_UNSUPPORTED = 4, /* e.g. d_state outside the compiled set */
    MMB_ERR_WORKSPACE = 5,   /* workspace pointer missing */
    MMB_ERR_LAUNCH = 6,      /* the CUDA launch failed */
    MMB_ERR_TIMEOUT = 7      /* a bounded device-side wait gave up */
};

typedef struct CUstream_st* mmb_stream_t; /* identical to cudaStream_t */

/* Human-readable text for a status code (static storage). */
const char* mmb_status_string(int status);

/* ABI revision of this header; bumped on any incompatible change. */
int mmb_abi_version(void);

/* Text of the last CUDA runtime error behind an MMB_ERR_LAUNCH on the calling
 * thread (static storage), or "no CUDA error recorded". */
const char* mmb_last_error(void);

/* Synchronises `stream`, then reports whether a kernel of this library on the
 * current device gave up a bounded device-side wait since the last call
 * (MMB_ERR_TIMEOUT; the flag is cleared) -- the shared-memory tile pipelines
 * wait on transaction barriers with an iteration limit.  MMB_OK otherwise. */
int mmb_device_status(mmb_stream_t stream);

/* Self-test of that error path (no reference counterpart: the reference checks
 * no device-side error at all, momentum_scan_cuda.py:107,132 only synchronise).
 * Launches one CTA on `stream` that arms a transaction barrier for bytes that
 * never arrive (it issues no copy, so nothing asynchronous is left behind),
 * waits on it with at most `polls` polls (1..4096, else MMB_ERR_SHAPE), gives
 * up and sets the device flag: the next mmb_device_status then returns
 * MMB_ERR_TIMEOUT and clears it.  The GPU context stays usable. */
int mmb_selftest_device_wait(int32_t polls, mmb_stream_t stream);

/* =========================================================================
 * Momentum selective scan (fused discretisation, scan, C-contraction, D skip,
 * optional softplus(delta + bias) and optional SiLU(z) gate):
 *
 *   dt  = softplus(delta + delta_bias) if delta_softplus else delta
 *   a   = exp(dt * A[d,n]);   u = alpha * dt * B[b,t,n] * x[b,t,d]
 *   v_t = beta * v_{t-1} + u_t ;   h_t = a_t * h_{t-1} + v_t      (h, v start at 0)
 *   y   = sum_n C[b,t,n] * h_t[n] + D[d] * x ;   out = y * silu(z) if z else y
 *
 * Replaces MambaMomentumBlock.selective_scan_momentum (mamba_momentum.py:256-323)
 * -- and with it _cuda_momentum_scan_sequential / _specialized_momentum_pscan
 * (:325-413) -- plus the block's delta softplus (:247) and gate (:227-229).
 *
 * Shapes: x, delta, z, out, dout, dx, ddelta, dz (batch, seqlen, dim);
 *         A, dA (dim, dstate); B, C, dB, dC (batch, seqlen, dstate);
 *         D, delta_bias, dD, ddelta_bias (dim).
 * dstate must be 8, 16, 32 or 64 (callers pad other sizes with zero states).
 * out, dout, dx, ddelta, dz, dB, dC are contiguous.  16-byte aligned pointers
 * and strides that are multiples of 4 take the vector path; anything else works
 * with 4-byte copies.
 * ========================================================================= */

/* Element type of the activations x, delta, z, B, C, out, dout, dx, ddelta, dz
 * (desc.dtype).  A, D, delta_bias, dA, dB, dC, dD, ddelta_bias, states and
 * checkpoints are fp32 in every case; state and arithmetic are always fp32.
 * bf16 calls need 16-byte aligned activation pointers and dim and every stride
 * a multiple of 8 (MMB_ERR_ALIGN otherwise). */
enum mmb_dtype { MMB_F32 = 0, MMB_BF16 = 1 };

typedef struct mmb_mmscan_desc {
    int64_t batch, seqlen, dim, dstate;
    int64_t x_stride[2];     /* (batch, seq) strides of x     */
    int64_t delta_stride[2]; /* (batch, seq) strides of delta */
    int64_t z_stride[2];     /* (batch, seq) strides of z     */
    int64_t B_stride[2];     /* (batch, seq) strides of B     */
    int64_t C_stride[2];     /* (batch, seq) strides of C     */
    float beta, alpha;
    int32_t delta_softplus;
    int32_t dtype;           /* enum mmb_dtype (0 = fp32)     */
    int32_t time_chunk;      /* steps per time chunk: 0 = the library's choice,
                                < 0 = never split, > 0 = this many (rounded up
                                to a multiple of 32)                          */
    int32_t reserved;        /* 0 */
} mmb_mmscan_desc;

/* Time chunks.  When batch x dim gives the GPU few warps (short batches of
 * long sequences), mmb_mmscan_fwd / mmb_mmscan_bwd cut the sequence into
 * chunks that separate CTAs scan at once: a summary pass gives each chunk its
 * affine map (forward: end state from zero and the products P, Q'; backward:
 * the adjoint pair from zero and the same P, Q'), a small kernel folds the maps
 * into every chunk's incoming carry, and the full pass runs each chunk from it.
 * The library splits on its own when batch * ceil(dim * dstate / 128) < 592
 * (four one-warp backward CTAs per SM), aiming at sixteen per SM in chunks of
 * at least 256 steps; desc.time_chunk overrides that.  Calls that pass state_in, state_out,
 * gstate_in or gstate_out, and forwards without checkpoints, never split.
 * The forward and the backward split independently (the backward does not read
 * the forward's carries), so each may take its own path. */

/* Floats of workspace for a call: the checkpoints the forward writes for the
 * backward ((h, v) every 8 steps, batch * ceil(seqlen/8) * dim * dstate * 2)
 * followed, when the call splits along time, by scratch for the chunk carries
 * (chunks * batch * dim * dstate * 6) that the forward and the backward both
 * write. */
size_t mmb_mmscan_workspace_floats(const mmb_mmscan_desc* desc);

/* The same for a descriptor with these sizes and time_chunk = 0 (the
 * library's choice). */
size_t mmb_mmscan_ckpt_floats(int64_t batch, int64_t seqlen, int64_t dim, int64_t dstate);

/* Forward.  D, z, delta_bias nullable.  ckpt (mmb_mmscan_workspace_floats
 * floats) nullable (inference: no checkpoints, no time split); the backward
 * needs the checkpoints of the same call.
 * fp32 activations only (desc->dtype == MMB_F32); mmb_mmscan_forward takes
 * either type and the segment carries. */
int mmb_mmscan_fwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                   const float* A, const float* B, const float* C, const float* D,
                   const float* z, const float* delta_bias, float* out, float* ckpt,
                   mmb_stream_t stream);

/* Backward.  Inputs as in the forward plus ckpt (required: the workspace of
 * the forward, whose scratch past the checkpoints the backward also writes)
 * and dout.
 * Outputs dx, ddelta, dA, dB, dC are required; dD (when D given), dz (when z
 * given) and ddelta_bias (when delta_bias given) are nullable. */
int mmb_mmscan_bwd(const mmb_mmscan_desc* desc, const float* x, const float* delta,
                   const float* A, const float* B, const float* C, const float* D,
                   const float* z, const float* delta_bias, float* ckpt,
                   const float* dout, float* dx, float* ddelta, float* dA, float* dB,
                   float* dC, float* dD, float* dz, float* ddelta_bias,
                   mmb_stream_t stream);

/* -------------------------------------------------------------------------
 * The same scan with bf16 or fp32 activations and segment carries, for a
 * sequence split into consecutive segments (one per GPU when a long sequence
 * is sharded along time; each segment is one call with seqlen = its length).
 * The reference has no counterpart: its scan always covers the whole sequence.
 *
 * States are (batch, dim, 2, dstate) fp32: [h | v] for the forward state,
 * [lam | mu] = [a_t gh_t | gv_t] for the adjoint pair at a segment boundary.
 * Over a segment of T steps,
 *   forward   h_T = P h_0 + beta Q' v_0 + h^0 ,     v_T = beta^T v_0 + v^0
 *   adjoint   lam_0 = P lam_T + lam^0 ,             mu_0 = Q' lam_T + beta^T mu_T + mu^0
 * where P = prod a_t, Q' = sum_t beta^(t-1) prod_{s>t} a_s, (h^0, v^0) is the
 * end state from a zero start and (lam^0, mu^0) the pair leaving the first
 * step when none arrives.  The summaries below compute those coefficients so
 * every segment's incoming carry follows from one all-gather.
 * ------------------------------------------------------------------------- */
typedef struct mmb_mmscan_tensors {
    /* inputs (activations in desc->dtype; the rest fp32) */
    const void* x;
    const void* delta;
    const void* z;            /* nullable */
    const void* B;
    const void* C;
    const float* A;
    const float* D;           /* nullable */
    const float* delta_bias;  /* nullable */
    const float* state_in;    /* nullable: [h | v] before the first step (zeros) */
    const float* gstate_in;   /* nullable: [lam | mu] arriving from after the last
                                 step (zeros); needs seqlen % 8 == 0 */
    const void* dout;         /* backward */
    /* outputs */
    void* out;                /* forward, (batch, seqlen, dim) */
    float* state_out;         /* nullable: [h | v] after the last step */
    float* ckpt;              /* forward writes (nullable), backward reads */
    void* dx;                 /* backward, (batch, seqlen, dim) */
    void* ddelta;
    void* dz;                 /* nullable */
    float* dA;                /* backward, fp32 sums */
    float* dB;
    float* dC;
    float* dD;                /* nullable */
    float* ddelta_bias;       /* nullable */
    float* gstate_out;        /* nullable: [lam | mu] leaving the first step */
} mmb_mmscan_tensors;

/* Forward with either activation type and optional state_in / state_out.
 * Reads x, delta, z, B, C, A, D, delta_bias, state_in; writes out, ckpt,
 * state_out.  The backward of a segment reads the checkpoints its forward
 * wrote, which start from state_in. */
int mmb_mmscan_forward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                       mmb_stream_t stream);

/* Backward with either activation type and optional gstate_in / gstate_out.
 * Reads x, delta, z, B, C, A, D, delta_bias, ckpt, dout, gstate_in; writes dx,
 * ddelta, dz, dA, dB, dC, dD, ddelta_bias (dA, dB, dC, dD, ddelta_bias are
 * fp32 sums for either type) and gstate_out. */
int mmb_mmscan_backward(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                        mmb_stream_t stream);

/* Forward segment summary: summary (batch, dim, 4, dstate) = [h^0 | v^0 | P | Q'].
 * Reads x, delta, B, A, delta_bias. */
int mmb_mmscan_fwd_summary(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                           float* summary, mmb_stream_t stream);

/* Backward segment summary: gsummary (batch, dim, 2, dstate) = [lam^0 | mu^0].
 * Reads delta, z, dout, C, A, delta_bias. */
int mmb_mmscan_bwd_summary(const mmb_mmscan_desc* desc, const mmb_mmscan_tensors* t,
                           float* gsummary, mmb_stream_t stream);

#define MMB_MAX_SEGMENTS 64

/* Incoming forward state of segment `seg` of `nseg` (seg_len: host array of
 * the segments' lengths; summaries: (nseg, batch, dim, 4, dstate), segment j's
 * forward summary at j): folds segments 0..seg-1 into state_in (batch, dim, 2,
 * dstate).  nseg <= MMB_MAX_SEGMENTS. */
int mmb_mmscan_carry_fwd(int64_t nseg, int64_t seg, const int64_t* seg_len, int64_t batch,
                         int64_t dim, int64_t dstate, float beta, const float* summaries,
                         float* state_in, mmb_stream_t stream);

/* Incoming adjoint pair of segment `seg`: folds segments nseg-1 down to seg+1
 * (their forward summaries for P, Q' and gsummaries (nseg, batch, dim, 2,
 * dstate) for lam^0, mu^0) into gstate_in (batch, dim, 2, dstate). */
int mmb_mmscan_carry_bwd(int64_t nseg, int64_t seg, const int64_t* seg_len, int64_t batch,
                         int64_t dim, int64_t dstate, float beta, const float* summaries,
                         const float* gsummaries, float* gstate_in, mmb_stream_t stream);

/* =========================================================================
 * The block's producer: causal depthwise conv1d + SiLU over time,
 *   out[b,t,d] = silu(bias[d] + sum_k weight[d,k] x[b, t-(width-1)+k, d]),
 * inputs before t = 0 from state_in (batch, dim, width-1) or zeros.
 *   Replaces conv1d(x.transpose(1, 2))[:, :, :L] + silu of the block's x branch
 *   (mamba_momentum.py:217-223; weight (dim, 1, width) of nn.Conv1d with
 *   groups = dim, padding = width-1).
 * x: (batch, seqlen, dim) with strides x_stride[0..1] (dim unit-stride);
 * out, dout, dx: contiguous (batch, seqlen, dim); weight (dim, width); bias
 * (dim) nullable; width 2..8.  state_out (nullable) receives the last width-1
 * inputs (the decode cache).  The backward writes dx (no gradient reaches
 * state_in) and the sums dweight (dim, width) and dbias (when bias given).
 * ========================================================================= */
int mmb_conv1d_silu_fwd(int64_t batch, int64_t seqlen, int64_t dim, int32_t width,
                        const float* x, const int64_t* x_stride, const float* weight,
                        const float* bias, const float* state_in, float* state_out,
                        float* out, mmb_stream_t stream);

int mmb_conv1d_silu_bwd(int64_t batch, int64_t seqlen, int64_t dim, int32_t width,
                        const float* x, const int64_t* x_stride, const float* weight,
                        const float* bias, const float* state_in, const float* dout,
                        float* dx, float* dweight, float* dbias, mmb_stream_t stream);

/* =========================================================================
 * Decode (one token per call).
 *
 * mmb_conv1d_step: out = silu(bias + sum_k weight[:,k] [state_in | x][k]) and
 * state_out = state_in (batch, dim, width-1) shifted left with x appended
 * (mamba_momentum.py:455-459, :466); state_out may be state_in (in place).
 * x rows x_row_stride apart.
 *
 * mmb_mmscan_step: the single-token momentum update (mamba_momentum.py:473-515)
 * with the block's softplus and gate fused:
 *   dt = softplus(delta + delta_bias) or delta; a = exp(dt A)
 *   v = beta v + alpha dt B x ;  h = a h + v ;  out = (C.h + D x) * silu(z)
 * h_in, v_in (element (b, d, n) at b*state_stride[0] + d*state_stride[1] + n;
 * NULL = zero state, the reference's None cache) give the state before the
 * token and h, v (same layout; may be h_in, v_in) receive it after: the
 * reference's (batch, dim, dstate) caches, or the h and v halves of a
 * forward's state_out.  D, z, delta_bias nullable.
 * ========================================================================= */
typedef struct mmb_step_desc {
    int64_t batch, dim, dstate;
    int64_t x_row_stride, delta_row_stride, z_row_stride, B_row_stride, C_row_stride;
    int64_t state_stride[2];
    float beta, alpha;
    int32_t delta_softplus;
    int32_t reserved;
} mmb_step_desc;

int mmb_conv1d_step(int64_t batch, int64_t dim, int32_t width, const float* x,
                    int64_t x_row_stride, const float* state_in, float* state_out,
                    const float* weight, const float* bias, float* out, mmb_stream_t stream);

int mmb_mmscan_step(const mmb_step_desc* desc, const float* x, const float* delta,
                    const float* A, const float* B, const float* C, const float* D,
                    const float* z, const float* delta_bias, const float* h_in,
                    const float* v_in, float* h, float* v, float* out, mmb_stream_t stream);

/* =========================================================================
 * Row scan:  v_t = beta*v_{t-1} + u_t ;  h_t = a_t*h_{t-1} + v_t  over the rows
 * of contiguous (rows, L) tensors (t unit-stride).
 *   Replaces momentum_scan_kernel / launch_forward (momentum_scan_cuda.py:22-47,
 *   :89-108, :175-178) and warp_mat2_scan_kernel (warp_momentum_scan_cuda.py:34-126).
 * v_out nullable.
 * ========================================================================= */
int mmb_rows_fwd(int64_t rows, int64_t L, const float* a, float beta, const float* u,
                 float* h, float* v_out, mmb_stream_t stream);

/* Adjoint of mmb_rows_fwd given g = dL/dh:
 *   gh_t = g_t + a_{t+1} gh_{t+1};  gv_t = gh_t + beta gv_{t+1};
 *   du_t = gv_t;  da_t = gh_t h_{t-1} (0 at t = 0).
 *   Replaces momentum_scan_backward_kernel / launch_backward
 *   (momentum_scan_cuda.py:49-87, :110-133); the gradient of
 *   warp_mat2_scan_backward_kernel (warp_momentum_scan_cuda.py:130-230) is
 *   defined to be this one.  da, du nullable. */
int mmb_rows_bwd(int64_t rows, int64_t L, const float* g, const float* a, float beta,
                 const float* h, float* da, float* du, mmb_stream_t stream);

/* =========================================================================
 * Diagonal scan in the PScan layout: H_t = A_t H_{t-1} + X_t along dim 1 of
 * (batch, L, M) tensors (M = D*N flattened, unit stride).
 *   Replaces PScan.forward / PScan.pscan (pscan.py:45-100, :160-194).
 * ========================================================================= */
int mmb_pscan_fwd(int64_t batch, int64_t L, int64_t M, const float* A, const float* X,
                  float* H, mmb_stream_t stream);

/* Adjoint (pscan.py:197-232): gX_t = G_t + A_{t+1} gX_{t+1};
 * gA_t = H_{t-1} gX_t (0 at t = 0).  dA, dX nullable. */
int mmb_pscan_bwd(int64_t batch, int64_t L, int64_t M, const float* A, const float* H,
                  const float* G, float* dA, float* dX, mmb_stream_t stream);

/* =========================================================================
 * 2x2 scan  x_t = M_t x_{t-1} + F_t  per (b, p) chain, x_{-1} = 0, with the
 * running matrix product Mscan_t = M_t Mscan_{t-1} (Mscan_{-1} = I).
 *   M, Mscan, dM, gMscan : (batch, L, 4P) = [M11 | M12 | M21 | M22] blocks of P
 *   F, X, gX, dF         : (batch, L, 2P) = [F1 | F2] blocks of P; complex entries
 *                          are interleaved (re, im) float pairs when complex_f = 1
 * Replaces parallel_scan_batched_complex (mamba_linoss.py:336-415) with its
 * binary operator (:561-605) -- and the 'optimized' / 'vmap' scans of the same
 * signature (:418-558, :680-763) -- parallel_scan_batched (LinOSS_pytorch.py:53-132)
 * and pscan_matrix_ultra (pscan_optimized.py:42-158, P = 1).
 * Chunked three-pass scan; `work` is caller workspace of
 * mmb_scan2_work_floats(batch, L, P, complex_f) floats (scratch, any contents).
 * ========================================================================= */
size_t mmb_scan2_work_floats(int64_t batch, int64_t L, int64_t P, int32_t complex_f);

/* Forward.  Mscan nullable (not wanted). */
int mmb_scan2_fwd(int64_t batch, int64_t L, int64_t P, int32_t complex_f, const float* M,
                  const float* F, float* Mscan, float* X, float* work, mmb_stream_t stream);

/* Adjoint:  lambda_t = gX_t + M_{t+1}^T lambda_{t+1};  dF_t = lambda_t;
 * dM_t = sum over (re, im) of lambda_t x_{t-1}^T, plus Lambda_t Mscan_{t-1}^T for
 * the running product (Lambda_t = gMscan_t + M_{t+1}^T Lambda_{t+1}).
 * X is the forward output.  gX and gMscan nullable (absent gradients); Mscan
 * (the forward's) is required when gMscan is given.  dM, dF required. */
int mmb_scan2_bwd(int64_t batch, int64_t L, int64_t P, int32_t complex_f, const float* M,
                  const float* X, const float* gX, const float* Mscan, const float* gMscan,
                  float* dM, float* dF, float* work, mmb_stream_t stream);

/* -------------------------------------------------------------------------
 * mmb_scan2_fwd without a workspace argument; no counterpart in the reference.
 *
 * For callers that cannot hand the library device memory at call time: an
 * operator inside a host framework that owns all device memory and gives its
 * plugins no way to allocate, or a latency-critical caller for whom a
 * cudaMalloc (which can synchronise the whole device) is not acceptable.  The
 * call allocates nothing; the caller still provides M, F, X (and Mscan) as in
 * mmb_scan2_fwd, with the same meaning and layouts.
 *
 * The scratch is a fixed array of MMB_SCAN2_NOALLOC_SCRATCH_FLOATS floats
 * (4 MiB) inside the library, resident on every GPU that loads the library
 * until the process exits.  Limit: 16 * batch * P <= that size (at most 65536
 * chains); larger problems return MMB_ERR_SHAPE.  When the chunking that
 * mmb_scan2_fwd would use does not fit, fewer, longer chunks are used, so
 * results agree with mmb_scan2_fwd to rounding.
 * The first call on each device looks up the array's device address; make
 * that first call before any stream capture on that device.  The address is
 * kept until the process exits: calls after a cudaDeviceReset of that device
 * in the same process are not supported.  All calls on a
 * device share the one array and it keeps the last call's contents (nothing in
 * it needs to start at zero): calls that can overlap on the GPU race, so the
 * caller must order them, e.g. on one stream.
 * ------------------------------------------------------------------------- */
#define MMB_SCAN2_NOALLOC_SCRATCH_FLOATS (1 << 20)

int mmb_scan2_fwd_noalloc(int64_t batch, int64_t L, int64_t P, int32_t complex_f,
                          const float* M, const float* F, float* Mscan, float* X,
                          mmb_stream_t stream);

/* =========================================================================
 * fp32-accurate GEMM on the tensor cores (tcgen05, 3 x tf32 split), for the
 * dense contractions of the LinOSS layer -- complex_matmul_real_input and
 * complex_matmul_complex_state (LinOSS_pytorch.py:135-150), as real GEMMs on
 * interleaved complex data, and their gradients:
 *
 *   C[m, n] (= or +=) sum_k A(m, k) B(n, k)  [+ evec[n] * E[m, n]]
 *
 * A(m, k) = A[m * lda + k] (a_mn == 0, K-major) or A[k * lda + m] (a_mn != 0);
 * B(n, k) = B[n * ldb + k] (b_mn == 0) or B[k * ldb + n] (b_mn != 0);
 * C and E row-major with ldc, lde >= N.  A, B 16-byte aligned, lda and ldb
 * multiples of 4.  Each operand is split into a tf32 high part and an fp32
 * remainder; the three significant partial products are accumulated in fp32
 * (error within a few fp32 ulps of the products).  B_lo nullable: when given,
 * B holds the high parts and B_lo the remainders of a K-major B (as
 * mmb_split_tf32 makes them, e.g. once per call for weights), and only A is
 * split per tile.  accumulate != 0 adds into C with vector reductions (C
 * cleared by the caller); splits > 1 cuts K into that many slices, one CTA
 * per slice and tile (needs accumulate).  E, evec nullable (both or neither).
 * ========================================================================= */
int mmb_gemm_f32(int32_t a_mn, int32_t b_mn, int64_t M, int64_t N, int64_t K, const float* A,
                 int64_t lda, const float* B, const float* B_lo, int64_t ldb, float* C,
                 int64_t ldc, const float* E, int64_t lde, const float* evec,
                 int32_t accumulate, int32_t splits, mmb_stream_t stream);

/* hi = x with the low 13 mantissa bits cleared (exact in tf32), lo = x - hi,
 * n floats each. */
int mmb_split_tf32(const float* x, float* hi, float* lo, int64_t n, mmb_stream_t stream);

/* out[n] (= or +=) sum_m X[m * ldx + n] * Y[m * ldy + n] for n < N: the
 * feedthrough gradient d(D) = sum over (b, t) of dy * u of the LinOSS layer
 * (LinOSS_pytorch.py:306-312).  N, ldx, ldy multiples of 4, X and Y 16-byte
 * aligned. */
int mmb_col_dot_f32(int64_t M, int64_t N, const float* X, int64_t ldx, const float* Y,
                    int64_t ldy, float* out, int32_t accumulate, mmb_stream_t stream);

/* =========================================================================
 * LinOSS layer scan with a time-invariant transition per oscillator p -- the
 * scan inside apply_linoss_im_complex / apply_linoss_imex_complex
 * (LinOSS_pytorch.py:153-239), batched:
 *   IM   (disc 0): S = 1/(1 + s^2 A); M = [[1 - s^2 A S, -s A S], [s S, S]];
 *                  F_t = (M11 s Bu_t, M21 s Bu_t)
 *   IMEX (disc 1): M = [[1, -s A], [s, 1 - s^2 A]];  F_t = (s Bu_t, s^2 Bu_t)
 *   x_t = M x_{t-1} + F_t ;  output x2_t (the second state component).
 * A_diag, step, dA_diag, dstep : (P); s = step[p], A = A_diag[p].
 * Bu, x2, dx2, dBu : (batch, L, P) complex, interleaved (re, im), 8-byte aligned.
 * The GEMMs around it (Bu = B u, y = Re(C x2)) stay with cuBLAS.
 * `work`: mmb_linoss_work_floats(batch, L, P) floats, 16-byte aligned.  The
 * forward leaves (x1, x2) checkpoints there; the backward needs the work buffer
 * of its forward unchanged.
 * ========================================================================= */
size_t mmb_linoss_work_floats(int64_t batch, int64_t L, int64_t P);

int mmb_linoss_fwd(int32_t disc, int64_t batch, int64_t L, int64_t P, const float* A_diag,
                   const float* step, const float* Bu, float* x2, float* work,
                   mmb_stream_t stream);

/* Adjoint given dx2: writes dBu and, when non-NULL, dA_diag and dstep (the
 * sums over batch and time of the transition's and input scale's gradients). */
int mmb_linoss_bwd(int32_t disc, int64_t batch, int64_t L, int64_t P, const float* A_diag,
                   const float* step, const float* Bu, const float* dx2, float* dBu,
                   float* dA_diag, float* dstep, float* work, mmb_stream_t stream);

/* =========================================================================
 * Selective LinOSS scan of the Mamba-LinOSS block, fused
 * (apply_linoss_vectorized, mamba_linoss.py:608-677): per step the transition
 * and input scale are built from s[b,t] (= mean over channels of delta) and
 * A_diag[p], and the output contraction is done in the kernel:
 *   IM:   S = 1/(1 + s^2 A); M = [[S, -s A S], [s S, S]]; F = (s S B, s^2 S B)
 *   IMEX: M = [[1, -s A], [s, 1 - s^2 A]];               F = (s B, s^2 B)
 *   x_t = M_t x_{t-1} + F_t (complex, x_{-1} = 0);  y[b,t] = Re sum_p C x2
 * B_re, B_im, C_re, C_im: (batch, L, P) with (batch, seq) strides B_stride /
 * C_stride shared by each re/im pair, unit stride along P; s, y, dy, ds
 * (batch, L) contiguous; A_diag, dA_diag (P).  The backward writes dB_re,
 * dB_im, dC_re, dC_im ((batch, L, P) contiguous) and the sums dA_diag and ds.
 * `work`: mmb_linoss_sel_work_floats(batch, L, P) floats, 16-byte aligned; the
 * backward needs its forward's work buffer unchanged.
 * ========================================================================= */
size_t mmb_linoss_sel_work_floats(int64_t batch, int64_t L, int64_t P);

int mmb_linoss_sel_fwd(int32_t disc, int64_t batch, int64_t L, int64_t P, const float* A_diag,
                       const float* s, const float* B_re, const float* B_im,
                       const int64_t* B_stride, const float* C_re, const float* C_im,
                       const int64_t* C_stride, float* y, float* work, mmb_stream_t stream);

int mmb_linoss_sel_bwd(int32_t disc, int64_t batch, int64_t L, int64_t P, const float* A_diag,
                       const float* s, const float* B_re, const float* B_im,
                       const int64_t* B_stride, const float* C_re, const float* C_im,
                       const int64_t* C_stride, const float* dy, float* dB_re, float* dB_im,
                       float* dC_re, float* dC_im, float* dA_diag, float* ds, float* work,
                       mmb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOMENTUM_SCAN_B200_H */
