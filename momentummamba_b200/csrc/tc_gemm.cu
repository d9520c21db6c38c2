// fp32-accurate GEMM on the sm_100a tensor cores (tcgen05, TMEM accumulator)
// for the dense contractions around the LinOSS layer scan.
//
//   C[m, n] (= or +=) sum_k A(m, k) B(n, k)  [+ evec[n] * E[m, n]]
//
// A and B are fp32 in global memory, each either K-major (row m / n holds the
// K values contiguously) or MN-major (row k holds the M / N values
// contiguously).  Accuracy: every operand x is split in shared memory into
// x_hi = x with its low 13 mantissa bits cleared (exact in tf32) and
// x_lo = x - x_hi (exact in fp32); the tensor cores accumulate
// A_hi B_hi + A_hi B_lo + A_lo B_hi in fp32 (kind::tf32), which leaves an
// error of a few fp32 ulps of the products (the dropped A_lo B_lo term is
// 2^-22 relative) -- close to a plain fp32 GEMM, unlike one-pass tf32 (2^-11).
//
// Tile: 128 x BN (BN = 128 or 256) per CTA, K in steps of 16 (one 64-byte
// swizzle row of fp32 for K-major operands), two pipeline stages (48 KB each
// at BN = 256, 32 KB at BN = 128), so two CTAs share an SM and one's
// epilogue overlaps the other's loads (32-value K steps, one CTA per SM,
// measured 118 us for M=65536 N=512 K=128).  Thread 0 issues the TMA copies
// (raw fp32 tiles, 128-byte swizzle) and the MMAs; all 128 threads split the
// landed tiles into hi / lo in place and, at the end, read the accumulator out
// of TMEM (one row per thread) for the epilogue.  Split-K (grid z) adds its
// partial tile to C with vector reductions.
#include "mmb_common.cuh"

namespace mmb {

constexpr int TG_BM = 128;
constexpr int TG_BK = 16;
constexpr int TG_NT = 128;
// Pipeline stages of 128-column tiles (256-column tiles keep 2: three would
// leave one CTA per SM).  Three stages (the producer refills the stage of tile
// i - 2 while tile i - 1's MMAs still run) measured the same as two (85 us for
// M=65536 N=128 K=512): each tile's A still waits out a DRAM round trip, the
// prefetch being one tile deep either way.
// The warp-specialised persistent kernel (1) or the one-role-per-phase kernel
// with two CTAs per SM (0); SMs the persistent grid covers.
#ifndef MMB_TG_WS
#define MMB_TG_WS 1
#endif
#ifndef MMB_TG_SMS
#define MMB_TG_SMS 148
#endif
#ifndef MMB_TG_STAGES_N128
#define MMB_TG_STAGES_N128 2
#endif
#ifndef MMB_TG_BN_MAX
#define MMB_TG_BN_MAX 256
#endif
template <int BN>
__host__ __device__ constexpr int tg_stages() { return BN == 128 ? MMB_TG_STAGES_N128 : 2; }
constexpr uint32_t TG_MASK_HI = 0xffffe000u;  // fp32 bits kept by tf32

// ---------------------------------------------------------------------------
// tcgen05 / TMEM wrappers (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy writes to shared memory -> visible to the tensor cores
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32, issued by one thread
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on `bar` once every MMA this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
// 32 consecutive 32-bit columns of this thread's TMEM lane: the load, and the
// wait that makes them readable (the registers pass through the wait, so no
// use can be scheduled before it)
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld32_issue(taddr, r);
    tmem_wait32(r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (sm_100 layout: start address, leading and
// stride byte offsets in 16-byte units, version 1 at bit 46, swizzle mode at
// bits 61-63).
//   K-major (mode 4, 64-byte swizzle of 16-byte chunks): rows of 64 bytes
//   (16 K values), 8-row groups `sbo` apart; the leading offset is unused.
//   MN-major (mode 1, 128-byte swizzle of 32-byte chunks -- the only
//   MN-major layout tf32 operands take): K-rows of 128 bytes (32 M / N
//   values), 4-row groups `sbo` apart along K, 32-value M / N blocks `lbo`
//   apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t mode) {
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | ((uint64_t)mode << 61);
}

// Instruction descriptor of kind::tf32 with fp32 accumulation: M = 128, N = n;
// a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t tf32_idesc(int n, bool a_mn, bool b_mn) {
    return (1u << 4)                  // D fp32
           | (2u << 7) | (2u << 10)   // A, B tf32
           | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TG_BM >> 4) << 24);
}

struct TGParams {
    int64_t M, N, K, kchunk;  // kchunk: K per grid-z slice (multiple of TG_BK)
    float* C;
    int64_t ldc;
    const float* E;  // nullable epilogue term evec[n] * E[m, n]
    int64_t lde;
    const float* evec;
    int accumulate;  // 1: C += (vector reductions; split-K), 0: C =
    int tma_c;       // C goes out through 32 x 32 TMA boxes (aligned C)
    int e_vec;       // E and evec 16-byte aligned with lde % 4 == 0: vector loads
    int* err;
};
struct TGMaps {
    CUtensorMap a, b, c;  // c: 32 x 32 boxes of C, 128-byte swizzle (when p.tma_c)
    CUtensorMap blo;      // B's low parts when the caller split B (BLO)
};

// TMA store / reduce-add of one 32 x 32 box of C from shared memory (bulk group)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const float* src, int c0,
                                             int c1, bool add) {
    if (add)
        asm volatile(
            "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
            " [%0, {%1, %2, %3}], [%4];" ::"l"(reinterpret_cast<uint64_t>(map)),
            "r"(c0), "r"(c1), "r"(0), "r"(smem_u32(src))
            : "memory");
    else
        asm volatile(
            "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group"
            " [%0, {%1, %2, %3}], [%4];" ::"l"(reinterpret_cast<uint64_t>(map)),
            "r"(c0), "r"(c1), "r"(0), "r"(smem_u32(src))
            : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// wait until at most N bulk groups of this thread still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int BN>
struct TGSmem {
    static constexpr int A_FLOATS = TG_BM * TG_BK;  // 8 KB
    static constexpr int B_FLOATS = BN * TG_BK;
    // per stage: A_hi | A_lo | B_hi | B_lo (each 1024-byte aligned)
    static constexpr int STAGE = 2 * A_FLOATS + 2 * B_FLOATS;
    static constexpr size_t BYTES = (size_t)tg_stages<BN>() * STAGE * 4 + 1024;
};

// Load one 128 x 16 (A) or BN x 16 (B) fp32 tile.  K-major: one box of 16 (K)
// x rows, 64-byte swizzle.  MN-major: boxes of 32 (M / N) x 16 (K), one per
// 32-value block, each 2 KB, 32-byte-chunk swizzle.
template <int ROWS, bool MN>
__device__ __forceinline__ void tg_load(float* dst, const CUtensorMap* map, int64_t r0, int64_t k0,
                                        uint64_t* bar) {
    if constexpr (!MN) {
        tma_load_3d(dst, map, (int)k0, (int)r0, 0, bar);
    } else {
#pragma unroll
        for (int g = 0; g < ROWS / 32; ++g)
            tma_load_3d(dst + g * 32 * TG_BK, map, (int)(r0 + 32 * g), (int)k0, 0, bar);
    }
}

// Descriptor of K-step kk (8 values of K) of a tile at `base`.
template <int ROWS, bool MN>
__device__ __forceinline__ uint64_t tg_desc(const float* base, int kk) {
    const uint32_t s = smem_u32(base);
    if constexpr (!MN) return smem_desc(s + kk * 32, 16, 512, 4);
    else return smem_desc(s + kk * 1024, 32 * TG_BK * 4, 512, 1);
}

// Split the landed tile in place into hi, and lo into `lo` (same layout).
template <int FLOATS>
__device__ __forceinline__ void tg_split(float* hi, float* lo, int tid) {
#pragma unroll 4
    for (int i = tid; i < FLOATS / 4; i += TG_NT) {
        float4 x = reinterpret_cast<float4*>(hi)[i];
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(x.x) & TG_MASK_HI);
        h.y = __uint_as_float(__float_as_uint(x.y) & TG_MASK_HI);
        h.z = __uint_as_float(__float_as_uint(x.z) & TG_MASK_HI);
        h.w = __uint_as_float(__float_as_uint(x.w) & TG_MASK_HI);
        l.x = x.x - h.x; l.y = x.y - h.y; l.z = x.z - h.z; l.w = x.w - h.w;
        reinterpret_cast<float4*>(hi)[i] = h;
        reinterpret_cast<float4*>(lo)[i] = l;
    }
}

// BLO: B arrives split (B = its tf32 high parts, maps.blo its remainders), as
// weights split once per call are: only A is split per tile.
template <int BN, bool A_MN, bool B_MN, bool BLO>
__global__ void __launch_bounds__(TG_NT, 1)
    tc_gemm_kernel(const TGParams p, const __grid_constant__ TGMaps maps) {
    using Sm = TGSmem<BN>;
    extern __shared__ float4 tg_smem4[];
    constexpr int TG_STAGES = tg_stages<BN>();
    __shared__ uint64_t tma_bar[TG_STAGES], mma_bar[TG_STAGES];
    __shared__ uint32_t tmem_base_s;
    float* smem = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(tg_smem4) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t m0 = (int64_t)blockIdx.x * TG_BM;
    const int64_t n0 = (int64_t)blockIdx.y * BN;
    const int64_t kb = (int64_t)blockIdx.z * p.kchunk;
    const int64_t ke = min64(p.K, kb + p.kchunk);
    const int nk = (int)((ke - kb + TG_BK - 1) / TG_BK);
    constexpr uint32_t IDESC = tf32_idesc(BN, A_MN, B_MN);
    constexpr uint32_t TX = (uint32_t)(TG_BM + (BLO ? 2 : 1) * BN) * TG_BK * 4;

    if (tid == 0) {
        for (int s = 0; s < TG_STAGES; ++s) {
            mbar_init(&tma_bar[s], 1);
            mbar_init(&mma_bar[s], 1);
        }
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(&tmem_base_s, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    auto a_hi = [&](int s) { return smem + s * Sm::STAGE; };
    auto a_lo = [&](int s) { return smem + s * Sm::STAGE + Sm::A_FLOATS; };
    auto b_hi = [&](int s) { return smem + s * Sm::STAGE + 2 * Sm::A_FLOATS; };
    auto b_lo = [&](int s) { return smem + s * Sm::STAGE + 2 * Sm::A_FLOATS + Sm::B_FLOATS; };
    auto issue = [&](int i) {  // thread 0: TMA of K-tile i into stage i % 2
        const int s = i % TG_STAGES;
        const int64_t k0 = kb + (int64_t)i * TG_BK;
        mbar_expect_tx(&tma_bar[s], TX);
        tg_load<TG_BM, A_MN>(a_hi(s), &maps.a, m0, k0, &tma_bar[s]);
        tg_load<BN, B_MN>(b_hi(s), &maps.b, n0, k0, &tma_bar[s]);
        if constexpr (BLO) tg_load<BN, B_MN>(b_lo(s), &maps.blo, n0, k0, &tma_bar[s]);
    };

    bool ok = true;
    if (tid == 0 && nk > 0) issue(0);
    for (int i = 0; i < nk; ++i) {
        const int s = i % TG_STAGES;
        // thread 0: the next tile goes into its stage once the MMAs of the tile
        // that stage last held (i + 1 - STAGES) are done
        if (tid == 0 && i + 1 < nk) {
            const int prev = i + 1 - TG_STAGES;
            if (prev >= 0) ok = mbar_wait_bounded(&mma_bar[prev % TG_STAGES],
                                                  (uint32_t)((prev / TG_STAGES) & 1));
            if (ok) issue(i + 1);
        }
        if (ok) ok = mbar_wait_bounded(&tma_bar[s], (uint32_t)((i / TG_STAGES) & 1));
        if (__syncthreads_or(!ok)) break;
        tg_split<Sm::A_FLOATS>(a_hi(s), a_lo(s), tid);
        if constexpr (!BLO) tg_split<Sm::B_FLOATS>(b_hi(s), b_lo(s), tid);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < TG_BK / 8; ++kk) {
                const uint64_t ah = tg_desc<TG_BM, A_MN>(a_hi(s), kk);
                const uint64_t al = tg_desc<TG_BM, A_MN>(a_lo(s), kk);
                const uint64_t bh = tg_desc<BN, B_MN>(b_hi(s), kk);
                const uint64_t bl = tg_desc<BN, B_MN>(b_lo(s), kk);
                umma_tf32(tmem, ah, bh, IDESC, (i > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(tmem, ah, bl, IDESC, 1u);
                umma_tf32(tmem, al, bh, IDESC, 1u);
            }
            umma_commit(&mma_bar[s]);
        }
    }
    // the accumulator is complete once the last tile's MMAs are
    if (ok && nk > 0) {
        const int l = nk - 1;
        ok = mbar_wait_bounded(&mma_bar[l % TG_STAGES], (uint32_t)((l / TG_STAGES) & 1));
    }
    if (__syncthreads_or(!ok)) {
        // a bounded wait gave up: let this CTA's MMAs drain (bounded) before
        // the accumulator is freed, report, leave
        if (tid == 0) {
            if (p.err) atomicOr(p.err, 1);
            for (int s = 0; s < TG_STAGES && nk > 0; ++s) {
                const int last = (nk - 1 - s);
                if (last >= 0)
                    mbar_wait_polls(&mma_bar[last % TG_STAGES],
                                    (uint32_t)((last / TG_STAGES) & 1), 1 << 16);
            }
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tmem_dealloc(tmem, BN);
        }
        return;
    }
    tc_fence_after();

    // epilogue: warp w holds rows 32w..32w+31 (TMEM lanes), 32 columns at a time
    const int64_t m = m0 + warp * 32 + lane;
    const bool mok = m < p.M && nk > 0;
    if (p.tma_c) {
        // each warp stages its 32 x 32 boxes in two 4 KB buffers (in the first
        // stage's operand space, free once every MMA is done) with the 128-byte
        // swizzle, and lane 0 stores (or adds) them with TMA; out-of-range rows
        // and columns are clipped by the copy
        float* wb = smem + warp * 2 * 1024;
        // the next 32 columns leave TMEM while this box is staged and stored
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        uint32_t rr[2][32];
        tmem_ld32_issue(trow, rr[0]);
        tmem_wait32(rr[0]);
        // column boxes inside N (uniform across the CTA)
        const int64_t ncols = p.N - n0 < BN ? p.N - n0 : BN;
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
            const int cur = (c >> 5) & 1;
            if (c >= ncols) continue;
            if (c + 32 < ncols) tmem_ld32_issue(trow + (uint32_t)(c + 32), rr[cur ^ 1]);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rr[cur][j]);
            const int64_t nb = n0 + c;
            if (p.E && mok) {
                const float* er = p.E + m * p.lde;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (nb + j < p.N) v[j] = fmaf(p.evec[nb + j], er[nb + j], v[j]);
            }
            float* buf = wb + ((c >> 5) & 1) * 1024;
            if (lane == 0) bulk_wait_read<1>();  // the box this buffer held last has left
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j)
                reinterpret_cast<float4*>(buf + lane * 32)[j ^ (lane & 7)] =
                    make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&maps.c, buf, (int)nb, (int)(m0 + warp * 32), p.accumulate != 0);
                bulk_commit();
            }
            if (c + 32 < ncols) tmem_wait32(rr[cur ^ 1]);
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
    } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
        const int64_t nb = n0 + c;
        if (!mok || nb >= p.N) continue;
        if (p.E) {
            const float* er = p.E + m * p.lde;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (nb + j < p.N) v[j] = fmaf(p.evec[nb + j], er[nb + j], v[j]);
        }
        float* cr = p.C + m * p.ldc + nb;
        const bool vec = nb + 32 <= p.N && ((reinterpret_cast<uintptr_t>(cr) & 15) == 0);
        if (p.accumulate) {
            if (vec) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) red_add_v4(cr + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                for (int j = 0; j < 32 && nb + j < p.N; ++j) atomicAdd(cr + j, v[j]);
            }
        } else {
            if (vec) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(cr + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                for (int j = 0; j < 32 && nb + j < p.N; ++j) cr[j] = v[j];
            }
        }
    }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// ---------------------------------------------------------------------------
// Warp-specialised, persistent variant: one CTA per SM walks its tiles with
// the roles in separate warps, so loads, splits, MMAs and the epilogue of
// consecutive K-blocks and tiles overlap:
//   warp 0      TMA producer: raw tiles into a ring of WS_RING slots, up to
//               the ring's depth ahead (a slot is refilled once the MMAs that
//               read it have completed);
//   warp 1      TMEM owner and MMA issuer: two accumulators of BN columns, so
//               tile t + 1 accumulates while the epilogue drains tile t;
//   warps 2-5   split each landed tile in place into tf32 high parts and
//               remainders (A, and B unless it came split);
//   warps 6-9   epilogue: TMEM -> registers -> 32 x 32 boxes in shared memory
//               -> TMA store (or reduce-add for K slices).
// Every wait is bounded; a wait that gives up raises a CTA-wide abort flag
// that the other roles' waits see, the MMAs in flight are drained and TMEM is
// freed before the CTA leaves.
// ---------------------------------------------------------------------------
constexpr int WS_SPLIT_WARPS = 4;
constexpr int WS_SPLIT_THREADS = 32 * WS_SPLIT_WARPS;
constexpr int WS_NT = 32 * (2 + WS_SPLIT_WARPS + 4);
// Ring depth: the raw tiles in flight per SM are what hides the DRAM latency.
template <int BN>
__host__ __device__ constexpr int ws_ring() { return BN == 256 ? 3 : 6; }

template <int BN>
struct WSSmem {
    static constexpr int A_FLOATS = TG_BM * TG_BK;
    static constexpr int B_FLOATS = BN * TG_BK;
    static constexpr int SLOT = 2 * A_FLOATS + 2 * B_FLOATS;  // A_hi | A_lo | B_hi | B_lo
    static constexpr int EPI = 4 * 2 * 1024;                   // 2 staging boxes per epilogue warp
    static constexpr size_t BYTES = (size_t)(ws_ring<BN>() * SLOT + EPI) * 4 + 1024;
};

// Bounded wait on phase `parity` that also gives up when another role aborted.
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        int* err) {
    for (int i = 0; i < MMB_WAIT_POLLS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    if (err) atomicOr(err, 1);
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int BN, bool A_MN, bool B_MN, bool BLO>
__global__ void __launch_bounds__(WS_NT, 1)
    tc_gemm_ws_kernel(const TGParams p, const __grid_constant__ TGMaps maps) {
    using Sm = WSSmem<BN>;
    constexpr int R = ws_ring<BN>();
    constexpr uint32_t IDESC = tf32_idesc(BN, A_MN, B_MN);
    constexpr uint32_t TX = (uint32_t)(TG_BM + (BLO ? 2 : 1) * BN) * TG_BK * 4;
    extern __shared__ float4 ws_smem4[];
    __shared__ uint64_t full[R], split[R], empty[R], acc_full[2], acc_empty[2], drained;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    volatile int* abort = &abort_s;
    float* smem = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(ws_smem4) + 1023) & ~(uintptr_t)1023);
    float* epi = smem + R * Sm::SLOT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int64_t mt = (p.M + TG_BM - 1) / TG_BM, nt = (p.N + BN - 1) / BN;
    const int64_t nz = (p.K + p.kchunk - 1) / p.kchunk;
    const int64_t ntiles = mt * nt * nz;
    // tile t: m fastest (consecutive CTAs share the B panel in L2), then n, then K slice
    auto tile_of = [&](int64_t t, int64_t& m0, int64_t& n0, int64_t& kb, int& nk) {
        const int64_t z = t / (mt * nt), r = t % (mt * nt);
        m0 = (r % mt) * TG_BM;
        n0 = (r / mt) * BN;
        kb = z * p.kchunk;
        const int64_t ke = min64(p.K, kb + p.kchunk);
        nk = (int)((ke - kb + TG_BK - 1) / TG_BK);
    };
    auto slot_a = [&](int s) { return smem + s * Sm::SLOT; };
    auto slot_alo = [&](int s) { return smem + s * Sm::SLOT + Sm::A_FLOATS; };
    auto slot_b = [&](int s) { return smem + s * Sm::SLOT + 2 * Sm::A_FLOATS; };
    auto slot_blo = [&](int s) { return smem + s * Sm::SLOT + 2 * Sm::A_FLOATS + Sm::B_FLOATS; };

    if (tid == 0) {
        abort_s = 0;
        for (int s = 0; s < R; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&split[s], WS_SPLIT_THREADS);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 128);
        }
        mbar_init(&drained, 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base_s, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        // ---- producer ----
        if (lane == 0) {
            int64_t j = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                int64_t m0, n0, kb;
                int nk;
                tile_of(t, m0, n0, kb, nk);
                for (int k = 0; k < nk && ok; ++k, ++j) {
                    const int s = (int)(j % R);
                    if (j >= R) ok = ws_wait(&empty[s], (uint32_t)(((j / R) - 1) & 1), abort, p.err);
                    if (!ok) break;
                    const int64_t k0 = kb + (int64_t)k * TG_BK;
                    mbar_expect_tx(&full[s], TX);
                    tg_load<TG_BM, A_MN>(slot_a(s), &maps.a, m0, k0, &full[s]);
                    tg_load<BN, B_MN>(slot_b(s), &maps.b, n0, k0, &full[s]);
                    if constexpr (BLO) tg_load<BN, B_MN>(slot_blo(s), &maps.blo, n0, k0, &full[s]);
                }
            }
            // copies still in flight land before the CTA leaves
            for (int64_t q = j - R > 0 ? j - R : 0; q < j; ++q)
                mbar_wait_polls(&full[q % R], (uint32_t)((q / R) & 1), 1 << 16);
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            int64_t j = 0, lt = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
                int64_t m0, n0, kb;
                int nk;
                tile_of(t, m0, n0, kb, nk);
                const int a = (int)(lt & 1);
                if (lt >= 2) ok = ws_wait(&acc_empty[a], (uint32_t)(((lt / 2) - 1) & 1), abort, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(a * BN);
                for (int k = 0; k < nk && ok; ++k, ++j) {
                    const int s = (int)(j % R);
                    ok = ws_wait(&split[s], (uint32_t)((j / R) & 1), abort, p.err);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < TG_BK / 8; ++kk) {
                        const uint64_t ah = tg_desc<TG_BM, A_MN>(slot_a(s), kk);
                        const uint64_t al = tg_desc<TG_BM, A_MN>(slot_alo(s), kk);
                        const uint64_t bh = tg_desc<BN, B_MN>(slot_b(s), kk);
                        const uint64_t bl = tg_desc<BN, B_MN>(slot_blo(s), kk);
                        umma_tf32(acc, ah, bh, IDESC, (k > 0 || kk > 0) ? 1u : 0u);
                        umma_tf32(acc, ah, bl, IDESC, 1u);
                        umma_tf32(acc, al, bh, IDESC, 1u);
                    }
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[a]);
            }
            // every MMA this CTA issued has completed before TMEM is freed
            umma_commit(&drained);
            mbar_wait_polls(&drained, 0, 1 << 20);
        }
    } else if (warp < 2 + WS_SPLIT_WARPS) {
        // ---- splitters ----
        const int st = tid - 64;
        int64_t j = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            int64_t m0, n0, kb;
            int nk;
            tile_of(t, m0, n0, kb, nk);
            for (int k = 0; k < nk && ok; ++k, ++j) {
                const int s = (int)(j % R);
                ok = ws_wait(&full[s], (uint32_t)((j / R) & 1), abort, p.err);
                if (!ok) break;
#pragma unroll 4
                for (int i = st; i < Sm::A_FLOATS / 4; i += WS_SPLIT_THREADS) {
                    const float4 x = reinterpret_cast<float4*>(slot_a(s))[i];
                    float4 h, l;
                    h.x = __uint_as_float(__float_as_uint(x.x) & TG_MASK_HI);
                    h.y = __uint_as_float(__float_as_uint(x.y) & TG_MASK_HI);
                    h.z = __uint_as_float(__float_as_uint(x.z) & TG_MASK_HI);
                    h.w = __uint_as_float(__float_as_uint(x.w) & TG_MASK_HI);
                    l.x = x.x - h.x; l.y = x.y - h.y; l.z = x.z - h.z; l.w = x.w - h.w;
                    reinterpret_cast<float4*>(slot_a(s))[i] = h;
                    reinterpret_cast<float4*>(slot_alo(s))[i] = l;
                }
                if constexpr (!BLO) {
#pragma unroll 4
                    for (int i = st; i < Sm::B_FLOATS / 4; i += WS_SPLIT_THREADS) {
                        const float4 x = reinterpret_cast<float4*>(slot_b(s))[i];
                        float4 h, l;
                        h.x = __uint_as_float(__float_as_uint(x.x) & TG_MASK_HI);
                        h.y = __uint_as_float(__float_as_uint(x.y) & TG_MASK_HI);
                        h.z = __uint_as_float(__float_as_uint(x.z) & TG_MASK_HI);
                        h.w = __uint_as_float(__float_as_uint(x.w) & TG_MASK_HI);
                        l.x = x.x - h.x; l.y = x.y - h.y; l.z = x.z - h.z; l.w = x.w - h.w;
                        reinterpret_cast<float4*>(slot_b(s))[i] = h;
                        reinterpret_cast<float4*>(slot_blo(s))[i] = l;
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&split[s]);
            }
        }
    } else {
        // ---- epilogue: warp q = warp % 4 reads TMEM lanes 32q..32q+31 (the four
        // epilogue warps cover the four lane quarters) ----
        const int q = warp & 3;
        float* wb = epi + q * 2 * 1024;
        int64_t lt = 0;
        int nbox = 0;  // boxes this warp has stored (staging buffer parity)
        bool ok = true;
        for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
            int64_t m0, n0, kb;
            int nk;
            tile_of(t, m0, n0, kb, nk);
            const int a = (int)(lt & 1);
            ok = ws_wait(&acc_full[a], (uint32_t)((lt / 2) & 1), abort, p.err);
            if (!ok) break;
            tc_fence_after();
            const int64_t m = m0 + q * 32 + lane;
            const bool mok = m < p.M;
            const int64_t ncols = p.N - n0 < BN ? p.N - n0 : BN;
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN);
            uint32_t rr[2][32];
            tmem_ld32_issue(trow, rr[0]);
            tmem_wait32(rr[0]);
#pragma unroll
            for (int c = 0; c < BN; c += 32) {
                const int cur = (c >> 5) & 1;
                if (c >= ncols) continue;
                if (c + 32 < ncols) tmem_ld32_issue(trow + (uint32_t)(c + 32), rr[cur ^ 1]);
                float v[32];
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = __uint_as_float(rr[cur][jj]);
                const int64_t nb = n0 + c;
                if (p.E && mok) {
                    const float* er = p.E + m * p.lde + nb;
                    if (p.e_vec && nb + 32 <= p.N) {
                        // whole 32-column box of an aligned E: vector loads
#pragma unroll
                        for (int jj = 0; jj < 32; jj += 4) {
                            const float4 e4 = *reinterpret_cast<const float4*>(er + jj);
                            const float4 w4 = *reinterpret_cast<const float4*>(p.evec + nb + jj);
                            v[jj] = fmaf(w4.x, e4.x, v[jj]);
                            v[jj + 1] = fmaf(w4.y, e4.y, v[jj + 1]);
                            v[jj + 2] = fmaf(w4.z, e4.z, v[jj + 2]);
                            v[jj + 3] = fmaf(w4.w, e4.w, v[jj + 3]);
                        }
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj)
                            if (nb + jj < p.N) v[jj] = fmaf(p.evec[nb + jj], er[jj], v[jj]);
                    }
                }
                float* buf = wb + (nbox & 1) * 1024;
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    reinterpret_cast<float4*>(buf + lane * 32)[jj ^ (lane & 7)] =
                        make_float4(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&maps.c, buf, (int)nb, (int)(m0 + q * 32), p.accumulate != 0);
                    bulk_commit();
                }
                ++nbox;
                if (c + 32 < ncols) tmem_wait32(rr[cur ^ 1]);
            }
            // this warp's reads of the accumulator are done: it may be refilled
            tc_fence_before();
            mbar_arrive(&acc_empty[a]);
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

template <int BN, bool A_MN, bool B_MN, bool BLO>
static int tg_launch(const TGParams& p0, const float* A, int64_t lda, const float* B,
                     const float* Blo, int64_t ldb, int splits, cudaStream_t s) {
    TGParams p = p0;
    TGMaps maps;
    // K-major: dims (K, rows) with rows lda apart; MN-major: (rows, K) with K-rows lda apart
    const bool oka = A_MN ? mmb_encode_tile_map(&maps.a, A, 4, p.M, p.K, 1, lda, lda * p.K, 32,
                                                TG_BK, MMB_SWZ_128B_ATOM32)
                          : mmb_encode_tile_map(&maps.a, A, 4, p.K, p.M, 1, lda, lda * p.M, TG_BK,
                                                TG_BM, TG_BK * 4);
    const bool okb = B_MN ? mmb_encode_tile_map(&maps.b, B, 4, p.N, p.K, 1, ldb, ldb * p.K, 32,
                                                TG_BK, MMB_SWZ_128B_ATOM32)
                          : mmb_encode_tile_map(&maps.b, B, 4, p.K, p.N, 1, ldb, ldb * p.N, TG_BK,
                                                BN, TG_BK * 4);
    if (!oka || !okb) return MMB_ERR_ALIGN;
    if (BLO && !mmb_encode_tile_map(&maps.blo, Blo, 4, p.K, p.N, 1, ldb, ldb * p.N, TG_BK, BN,
                                    TG_BK * 4))
        return MMB_ERR_ALIGN;
    // C through TMA boxes when its base and row pitch are 16-byte aligned
    p.tma_c = (((uintptr_t)p.C & 15) == 0 && (p.ldc & 3) == 0 &&
               mmb_encode_tile_map(&maps.c, p.C, 4, p.N, p.M, 1, p.ldc, p.ldc * p.M, 32, 32, 128))
                  ? 1 : 0;
    p.err = mmb_device_error_flag();
    p.e_vec = p.E && ((uintptr_t)p.E & 15) == 0 && ((uintptr_t)p.evec & 15) == 0 &&
              (p.lde & 3) == 0;
    if (MMB_TG_WS && p.tma_c) {
        // persistent: one CTA per SM over all (m, n, K-slice) tiles
        static int attr_ws[MMB_MAX_DEVICES] = {};
        const int st =
            mmb_smem_attr(tc_gemm_ws_kernel<BN, A_MN, B_MN, BLO>, WSSmem<BN>::BYTES, attr_ws);
        if (st != MMB_OK) return st;
        const int64_t tiles = (p.M + TG_BM - 1) / TG_BM * ((p.N + BN - 1) / BN) * splits;
        const unsigned grid = (unsigned)(tiles < MMB_TG_SMS ? tiles : MMB_TG_SMS);
        tc_gemm_ws_kernel<BN, A_MN, B_MN, BLO><<<grid, WS_NT, WSSmem<BN>::BYTES, s>>>(p, maps);
        return mmb_launch_status();
    }
    static int attr_done[MMB_MAX_DEVICES] = {};
    const int st =
        mmb_smem_attr(tc_gemm_kernel<BN, A_MN, B_MN, BLO>, TGSmem<BN>::BYTES, attr_done);
    if (st != MMB_OK) return st;
    dim3 grid((unsigned)((p.M + TG_BM - 1) / TG_BM), (unsigned)((p.N + BN - 1) / BN),
              (unsigned)splits);
    tc_gemm_kernel<BN, A_MN, B_MN, BLO><<<grid, TG_NT, TGSmem<BN>::BYTES, s>>>(p, maps);
    return mmb_launch_status();
}

template <int BN>
static int tg_dispatch(bool a_mn, bool b_mn, const TGParams& p, const float* A, int64_t lda,
                       const float* B, const float* Blo, int64_t ldb, int splits,
                       cudaStream_t s) {
    if (Blo) return a_mn ? tg_launch<BN, true, false, true>(p, A, lda, B, Blo, ldb, splits, s)
                         : tg_launch<BN, false, false, true>(p, A, lda, B, Blo, ldb, splits, s);
    if (a_mn) return b_mn ? tg_launch<BN, true, true, false>(p, A, lda, B, Blo, ldb, splits, s)
                          : tg_launch<BN, true, false, false>(p, A, lda, B, Blo, ldb, splits, s);
    return b_mn ? tg_launch<BN, false, true, false>(p, A, lda, B, Blo, ldb, splits, s)
                : tg_launch<BN, false, false, false>(p, A, lda, B, Blo, ldb, splits, s);
}

// out[n] += sum_m X[m, n] Y[m, n] (the LinOSS layer's d(D) = sum over (b, t) of
// dy * u).  Each thread keeps 4 columns and walks a stride of rows four rows at
// a time (eight 16-byte loads in flight); the CTA's warps are summed in shared
// memory and each CTA adds its column sums to `out` once, as 4-wide vector
// reductions when `out` is 16-byte aligned.  The launcher keeps the grid at two
// CTAs per SM: with one CTA per 8 rows the reductions of ~1200 CTAs into the
// same 128 columns serialised in L2 (34.7 us for M = 65536, N = 128).
constexpr int CD_NT = 256;
constexpr int CD_ROWS = CD_NT / 32;  // rows a CTA covers per step of its walk
__global__ void __launch_bounds__(CD_NT)
    col_dot_kernel(int64_t M, int64_t N, const float* __restrict__ X, int64_t ldx,
                   const float* __restrict__ Y, int64_t ldy, float* __restrict__ out,
                   int vec_out) {
    __shared__ float4 part[CD_NT];
    const int64_t q = (int64_t)blockIdx.y * 32 + (threadIdx.x & 31);  // column quad
    const int64_t n0 = q * 4;
    const int rw = threadIdx.x >> 5;                                    // row lane (warp)
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n0 < N) {
        const int64_t stride = (int64_t)gridDim.x * CD_ROWS;
        int64_t m = (int64_t)blockIdx.x * CD_ROWS + rw;
        float4 acc1 = acc, acc2 = acc, acc3 = acc;
        for (; m + 3 * stride < M; m += 4 * stride) {
            float4 a[4], b[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                a[k] = *reinterpret_cast<const float4*>(X + (m + k * stride) * ldx + n0);
                b[k] = *reinterpret_cast<const float4*>(Y + (m + k * stride) * ldy + n0);
            }
            float4* accs[4] = {&acc, &acc1, &acc2, &acc3};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                accs[k]->x = fmaf(a[k].x, b[k].x, accs[k]->x);
                accs[k]->y = fmaf(a[k].y, b[k].y, accs[k]->y);
                accs[k]->z = fmaf(a[k].z, b[k].z, accs[k]->z);
                accs[k]->w = fmaf(a[k].w, b[k].w, accs[k]->w);
            }
        }
        for (; m < M; m += stride) {
            const float4 a = *reinterpret_cast<const float4*>(X + m * ldx + n0);
            const float4 b = *reinterpret_cast<const float4*>(Y + m * ldy + n0);
            acc.x = fmaf(a.x, b.x, acc.x);
            acc.y = fmaf(a.y, b.y, acc.y);
            acc.z = fmaf(a.z, b.z, acc.z);
            acc.w = fmaf(a.w, b.w, acc.w);
        }
        acc.x += acc1.x + (acc2.x + acc3.x);
        acc.y += acc1.y + (acc2.y + acc3.y);
        acc.z += acc1.z + (acc2.z + acc3.z);
        acc.w += acc1.w + (acc2.w + acc3.w);
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (rw == 0 && n0 < N) {
        float4 t = acc;
        for (int w = 1; w < CD_ROWS; ++w) {
            const float4 v = part[w * 32 + threadIdx.x];
            t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
        }
        if (vec_out) {
            red_add_v4(out + n0, t.x, t.y, t.z, t.w);
        } else {
            atomicAdd(out + n0, t.x);
            atomicAdd(out + n0 + 1, t.y);
            atomicAdd(out + n0 + 2, t.z);
            atomicAdd(out + n0 + 3, t.w);
        }
    }
}

// hi = x with the low 13 mantissa bits cleared, lo = x - hi
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const float h = __uint_as_float(__float_as_uint(v) & TG_MASK_HI);
        hi[i] = h;
        lo[i] = v - h;
    }
}

}  // namespace mmb

using namespace mmb;

extern "C" int mmb_gemm_f32(int32_t a_mn, int32_t b_mn, int64_t M, int64_t N, int64_t K,
                            const float* A, int64_t lda, const float* B, const float* B_lo,
                            int64_t ldb, float* C, int64_t ldc, const float* E, int64_t lde,
                            const float* evec, int32_t accumulate, int32_t splits,
                            mmb_stream_t stream) {
    MMB_NVTX("mmb_gemm_f32");
    if (!A || !B || !C || (E && !evec)) return MMB_ERR_NULL;
    if (B_lo && (b_mn || ((uintptr_t)B_lo & 15))) return B_lo && b_mn ? MMB_ERR_UNSUPPORTED
                                                                      : MMB_ERR_ALIGN;
    if (M <= 0 || N <= 0 || K <= 0 || splits < 1 || splits > 65535) return MMB_ERR_SHAPE;
    if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return MMB_ERR_SHAPE;
    if (ldc < N || (E && lde < N)) return MMB_ERR_SHAPE;
    if ((a_mn ? lda < M : lda < K) || (b_mn ? ldb < N : ldb < K)) return MMB_ERR_SHAPE;
    // TMA: 16-byte aligned bases and row pitches
    if (((uintptr_t)A & 15) || ((uintptr_t)B & 15) || (lda & 3) || (ldb & 3)) return MMB_ERR_ALIGN;
    if (splits > 1 && !accumulate) return MMB_ERR_SHAPE;
    TGParams p{};
    p.M = M; p.N = N; p.K = K;
    const int64_t per = (K + splits - 1) / splits;
    p.kchunk = (per + TG_BK - 1) / TG_BK * TG_BK;
    const int used = (int)((K + p.kchunk - 1) / p.kchunk);
    p.C = C; p.ldc = ldc; p.E = E; p.lde = lde; p.evec = evec;
    p.accumulate = accumulate ? 1 : 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // 256-column tiles when N fills them, else 128
    if (MMB_TG_BN_MAX > 128 && N > 128)
        return tg_dispatch<256>(a_mn != 0, b_mn != 0, p, A, lda, B, B_lo, ldb, used, s);
    return tg_dispatch<128>(a_mn != 0, b_mn != 0, p, A, lda, B, B_lo, ldb, used, s);
}

extern "C" int mmb_col_dot_f32(int64_t M, int64_t N, const float* X, int64_t ldx,
                               const float* Y, int64_t ldy, float* out, int32_t accumulate,
                               mmb_stream_t stream) {
    MMB_NVTX("mmb_col_dot_f32");
    if (!X || !Y || !out) return MMB_ERR_NULL;
    if (M <= 0 || N <= 0 || ldx < N || ldy < N) return MMB_ERR_SHAPE;
    if ((N & 3) || (ldx & 3) || (ldy & 3) || ((uintptr_t)X & 15) || ((uintptr_t)Y & 15))
        return MMB_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!accumulate && cudaMemsetAsync(out, 0, (size_t)N * sizeof(float), s) != cudaSuccess)
        return mmb_launch_status();
    // two CTAs per SM over the column quads (at least one CTA per quad group)
    const int64_t quads = (N / 4 + 31) / 32;
    const int64_t steps = (M + CD_ROWS - 1) / CD_ROWS;
    int64_t bx = (148 * 2 + quads - 1) / quads;
    if (bx > steps) bx = steps;
    if (bx < 1) bx = 1;
    col_dot_kernel<<<dim3((unsigned)bx, (unsigned)quads), CD_NT, 0, s>>>(
        M, N, X, ldx, Y, ldy, out, ((uintptr_t)out & 15) == 0 ? 1 : 0);
    return mmb_launch_status();
}

extern "C" int mmb_split_tf32(const float* x, float* hi, float* lo, int64_t n,
                              mmb_stream_t stream) {
    MMB_NVTX("mmb_split_tf32");
    if (!x || !hi || !lo) return MMB_ERR_NULL;
    if (n <= 0) return MMB_ERR_SHAPE;
    const int64_t blocks = (n + 255) / 256;
    split_tf32_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(x, hi, lo, n);
    return mmb_launch_status();
}
