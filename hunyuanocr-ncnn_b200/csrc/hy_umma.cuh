// Prompt-prefill projections on the 5th-generation tensor cores (tcgen05):
//   C[M x N] (=, +=, or SwiGLU of) A[M x K] . W[N x K]^T
// A = fp32 activation rows of the prompt, W = a decoder linear ([out x in],
// fp32 or bf16). This is the GEMM-shaped part of the prefill
// (export/text_decoder_kv.py:64-69, 93-95 run over the whole prompt by
// run_decoder_prefill, src/text_runtime.cpp:648-674).
//
// Arithmetic: tcgen05.mma kind::tf32 with fp32 accumulation in tensor memory,
// three-term split of the fp32 operands (x = hi + lo, hi = x with its low 13
// mantissa bits cleared): A.W ~ lo_A.hi_W + hi_A.lo_W + hi_A.hi_W; the
// dropped lo.lo term is below 2^-22 relative. bf16 weights are exact tf32
// values (lo_W = 0), so they take the first and last products only.
//
// Operands are laid out for the tensor core in HBM ("tiled"): a matrix of R
// rows (R a multiple of 8; activation rows padded to 128) and K columns is
// stored as blocks of 8 rows x 16 columns (512 bytes: four 8-row x 16-byte
// core matrices, the UMMA K-major no-swizzle canonical layout), block
// (row group g, column tile kt) at ((kt * R / 8) + g) * 512 bytes. The rows
// n0 .. n0 + BN of one 16-column tile are then one contiguous run of BN * 64
// bytes, fetched by a single cp.async.bulk. Weights are split into hi / lo
// tiles once, when they are loaded; activations are written split and tiled by
// the kernel that produces them (RMSNorm rows, attention output, SwiGLU).
//
// CTA = one 128 x BN output tile (BN = 128 or 64), 6 warps:
//   warp 4, one thread: per 16-column K step, 4 bulk copies (A hi / lo, W hi /
//     lo) into a 6-stage shared-memory ring, completing on the stage's `full`
//     mbarrier (expect-tx);
//   warp 5 allocates the tensor-memory accumulator (128 lanes x BN fp32
//     columns); one of its threads waits for each stage, issues its MMAs
//     (3 per 8 columns of K) and tcgen05.commit's the stage's `empty`
//     mbarrier, which hands the slot back to the copies; after the last stage
//     it commits `done`;
//   warps 0-3 (epilogue) read their 32 TMEM lanes (= tile rows) with
//     tcgen05.ld 32x32b and store, add to the residual, or apply SwiGLU and
//     write the result split and tiled for the next GEMM.
// Every mbarrier wait is bounded; a timeout sets an error bit and the CTA
// still waits for its copies and frees its tensor memory before it exits.
//
#pragma once

#include "hy_device.cuh"

namespace hy {

// ---------------------------------------------------------------------------
// tcgen05 wrappers (cta_group::1).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives (once) on `bar` when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive fp32 columns: thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Waits for this thread's tcgen05.ld; the registers are threaded through the
// asm so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// Bounded spin on phase `parity` of `bar` without the suspend hint: for the
// single MMA-issuing thread, which must react to a stage becoming ready at once.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err, int err_bit)
{
    const unsigned long long t0 = global_ns();
    for (unsigned it = 0;; ++it)
    {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((it & 255u) == 255u && global_ns() - t0 > kWaitLimitNs)
        {
            if (err) atomicOr(err, err_bit);
            return false;
        }
    }
}

// Shared-memory matrix descriptor, K-major, no swizzle: start address, the
// byte offset between core matrices adjacent in K (leading) and in M/N
// (stride), descriptor version 1 (bits 46-47).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor: fp32 accumulator (bits 4-5 = 1), A and B tf32
// (bits 7-9, 10-12 = 2), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int m, int n)
{
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Tiled operand layout.
// ---------------------------------------------------------------------------
// Float index of element (r, k) in a tiled matrix of `rows` rows.
__host__ __device__ __forceinline__ size_t tiled_index(int r, int k, int rows)
{
    return (static_cast<size_t>(k >> 4) * (rows >> 3) + (r >> 3)) * 128 + ((k >> 2) & 3) * 32 + (r & 7) * 4 + (k & 3);
}

__device__ __forceinline__ void split_hi_lo(float v, float& hi, float& lo)
{
    hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    lo = v - hi;
}

// Writes 4 consecutive columns k .. k + 3 (k % 4 == 0) of row r, split, into tiled hi / lo.
__device__ __forceinline__ void store_tiled4(float* hi, float* lo, int rows, int r, int k, float4 v)
{
    float4 h, l;
    split_hi_lo(v.x, h.x, l.x);
    split_hi_lo(v.y, h.y, l.y);
    split_hi_lo(v.z, h.z, l.z);
    split_hi_lo(v.w, h.w, l.w);
    const size_t i = tiled_index(r, k, rows);
    *reinterpret_cast<float4*>(hi + i) = h;
    *reinterpret_cast<float4*>(lo + i) = l;
}

// Weight [R x K] row-major (WT) -> tiled hi (and lo for fp32). One thread per 4 columns.
template <typename WT>
__global__ void tile_weight_kernel(const WT* __restrict__ src, int R, int K, float* __restrict__ hi, float* __restrict__ lo)
{
    const size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (q >= static_cast<size_t>(R) * (K / 4)) return;
    const int r = static_cast<int>(q / (K / 4)), k = static_cast<int>(q % (K / 4)) * 4;
    const float4 v = load4(src + static_cast<size_t>(r) * K + k);
    const size_t i = tiled_index(r, k, R);
    if (lo)
    {
        store_tiled4(hi, lo, R, r, k, v);
    }
    else
    {
        *reinterpret_cast<float4*>(hi + i) = v;   // bf16 values are exact in tf32
    }
}

// RMSNorm of row m (1024 wide: HunYuanDenseV1RMSNorm, w * (x * 1/sqrt(mean(x^2) + eps)))
// into tiled hi / lo of `rows_pad` rows. One CTA (256 threads) per row.
__global__ void rmsnorm_tiled_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                     int rows_pad, float* __restrict__ hi, float* __restrict__ lo)
{
    __shared__ float red[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float4 v = *reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * kHidden + tid * 4);
    const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    const float ri = 1.0f / sqrtf(t / static_cast<float>(kHidden) + eps);
    const float4 wv = *reinterpret_cast<const float4*>(w + tid * 4);
    store_tiled4(hi, lo, rows_pad, m, tid * 4,
                 make_float4(wv.x * (v.x * ri), wv.y * (v.y * ri), wv.z * (v.z * ri), wv.w * (v.w * ri)));
}

// Row m of x [rows x K] (K a multiple of 1024), split, into tiled hi / lo of
// `rows_pad` rows. One CTA (256 threads) per row.
__global__ void split_tiled_kernel(const float* __restrict__ x, int K, int rows_pad, float* __restrict__ hi,
                                   float* __restrict__ lo)
{
    const int m = blockIdx.x;
    for (int k = threadIdx.x * 4; k < K; k += 256 * 4)
        store_tiled4(hi, lo, rows_pad, m, k, *reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K + k));
}

// ---------------------------------------------------------------------------
// The prefill GEMM.
// ---------------------------------------------------------------------------
enum { UG_STORE = 0, UG_RESID = 1, UG_SWIGLU_TILED = 2 };

constexpr int kUmBM = 128, kUmBK = 16, kUmStages = 6;
constexpr int kUmEpiWarps = 4, kUmProducerWarp = 4, kUmMmaWarp = 5, kUmThreads = 6 * 32;
constexpr int kUmCoreBytes = 128;   // one core matrix: 8 rows x 16 bytes (LBO)
constexpr int kUmGroupBytes = 512;  // 8 rows x 16 columns (SBO)

template <int BN, bool B_SPLIT>
struct UmShape {
    static constexpr int A_TILE = kUmBM * kUmBK * 4;
    static constexpr int B_TILE = BN * kUmBK * 4;
    static constexpr int OFF_ALO = A_TILE;
    static constexpr int OFF_BHI = 2 * A_TILE;
    static constexpr int OFF_BLO = OFF_BHI + B_TILE;   // fp32 weights only
    static constexpr int STAGE = OFF_BHI + (B_SPLIT ? 2 : 1) * B_TILE;
    static constexpr int STAGE_BYTES = STAGE;            // bytes the copies of one stage deliver
    static constexpr int BAR_OFF = kUmStages * STAGE;
    static constexpr int SMEM = BAR_OFF + (2 * kUmStages + 2) * 8;
    static_assert(STAGE % 128 == 0, "stage alignment");
    static_assert(BN == 64 || BN == 128, "tile width (also the TMEM column count)");
};

struct UmmaGemmArgs {
    const float* a_hi;   // tiled [a_rows x K], a_rows = M rounded up to 128
    const float* a_lo;
    int a_rows;
    const float* w_hi;   // tiled [N x K]
    const float* w_lo;   // nullptr: bf16 weights (lo = 0)
    int M, N, K;         // N % BN == 0, K % 16 == 0 (checked by the host)
    float* C;            // STORE: C[m, n]; RESID: C[m, n] += (ldc)
    int ldc;
    float* act_hi;       // SWIGLU_TILED: act[m, n / 2] = silu(y[2j]) * y[2j + 1], tiled [a_rows x N / 2]
    float* act_lo;
    int* err;
};

template <int EPI, int BN, bool B_SPLIT>
__global__ void __launch_bounds__(kUmThreads, 1) umma_gemm_kernel(const UmmaGemmArgs a)
{
    using S = UmShape<BN, B_SPLIT>;
    constexpr int NS = kUmStages;
    constexpr uint32_t IDESC = umma_idesc_tf32(kUmBM, BN);
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
    uint64_t* empty = full + NS;
    uint64_t* done = empty + NS;
    __shared__ uint32_t s_tmem;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kUmBM;
    const int KT = a.K / kUmBK;

    if (warp == kUmMmaWarp)
    {
        tmem_alloc(&s_tmem, BN);
        tmem_relinquish();
    }
    if (tid == 0)
    {
        for (int s = 0; s < NS; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kUmProducerWarp)
    {
        // ---------------- bulk copies (one thread) ----------------
        if (lane == 0)
        {
            const size_t a_step = static_cast<size_t>(a.a_rows) * kUmBK;   // floats per 16-column tile of A
            const size_t w_step = static_cast<size_t>(a.N) * kUmBK;
            const float* ah = a.a_hi + static_cast<size_t>(m0) * kUmBK;
            const float* al = a.a_lo + static_cast<size_t>(m0) * kUmBK;
            const float* wh = a.w_hi + static_cast<size_t>(n0) * kUmBK;
            const float* wl = B_SPLIT ? a.w_lo + static_cast<size_t>(n0) * kUmBK : nullptr;
            int issued = 0;
            for (int kt = 0; kt < KT; ++kt)
            {
                const int s = kt % NS;
                if (kt >= NS && !mbar_wait(&empty[s], ((kt / NS) - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                unsigned char* st = smem + s * S::STAGE;
                mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
                bulk_g2s_plain(st, ah + kt * a_step, S::A_TILE, &full[s]);
                bulk_g2s_plain(st + S::OFF_ALO, al + kt * a_step, S::A_TILE, &full[s]);
                bulk_g2s_plain(st + S::OFF_BHI, wh + kt * w_step, S::B_TILE, &full[s]);
                if constexpr (B_SPLIT) bulk_g2s_plain(st + S::OFF_BLO, wl + kt * w_step, S::B_TILE, &full[s]);
                issued = kt + 1;
            }
            // Never leave the CTA with copies in flight: wait for the last stages to land.
            for (int kt = (issued > NS ? issued - NS : 0); kt < issued; ++kt)
                mbar_wait(&full[kt % NS], (kt / NS) & 1, a.err, kErrTimeoutFull);
        }
        __syncwarp();
    }
    else if (warp == kUmMmaWarp)
    {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0)
        {
            const uint32_t sbase = smem_u32(smem);
            for (int kt = 0; kt < KT; ++kt)
            {
                const int s = kt % NS;
                if (!mbar_wait_spin(&full[s], (kt / NS) & 1, a.err, kErrTimeoutFull)) break;
                tc_fence_after();
                const uint32_t st = sbase + s * S::STAGE;
#pragma unroll
                for (int ks = 0; ks < kUmBK / 8; ++ks)
                {
                    const uint32_t ko = ks * 2 * kUmCoreBytes;   // 8 tf32 of K = 2 core matrices
                    const uint64_t ahi = umma_desc(st + ko, kUmCoreBytes, kUmGroupBytes);
                    const uint64_t alo = umma_desc(st + S::OFF_ALO + ko, kUmCoreBytes, kUmGroupBytes);
                    const uint64_t bhi = umma_desc(st + S::OFF_BHI + ko, kUmCoreBytes, kUmGroupBytes);
                    umma_tf32(tmem, alo, bhi, IDESC, (kt | ks) ? 1u : 0u);
                    if constexpr (B_SPLIT)
                        umma_tf32(tmem, ahi, umma_desc(st + S::OFF_BLO + ko, kUmCoreBytes, kUmGroupBytes), IDESC, 1u);
                    umma_tf32(tmem, ahi, bhi, IDESC, 1u);
                }
                umma_commit(&empty[s]);   // the slot is free once these MMAs have read it
            }
            umma_commit(done);
        }
        __syncwarp();
    }
    else
    {
        // ---------------- epilogue (warps 0-3: TMEM lane quarter = warp) ----------------
        if (mbar_wait(done, 0, a.err, kErrTimeoutFull))
        {
            tc_fence_after();
            const int row = warp * 32 + lane;
            const int m = m0 + row;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16)
            {
                uint32_t r[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, r);
                tmem_ld_wait(r);
                if (m >= a.M) continue;
                if constexpr (EPI == UG_SWIGLU_TILED)
                {
                    // Rows 2j / 2j + 1 of the gate/up weight are gate_j / up_j; act columns
                    // (n0 + c0) / 2 .. + 7, split and tiled for the down projection.
                    float o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                    {
                        const float gt = __uint_as_float(r[2 * e]), up = __uint_as_float(r[2 * e + 1]);
                        o[e] = (gt / (1.0f + expf(-gt))) * up;
                    }
                    const int k = (n0 + c0) >> 1;
                    store_tiled4(a.act_hi, a.act_lo, a.a_rows, m, k, make_float4(o[0], o[1], o[2], o[3]));
                    store_tiled4(a.act_hi, a.act_lo, a.a_rows, m, k + 4, make_float4(o[4], o[5], o[6], o[7]));
                }
                else
                {
                    float* dst = a.C + static_cast<size_t>(m) * a.ldc + n0 + c0;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                    {
                        float4 v = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                               __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
                        if constexpr (EPI == UG_RESID)
                        {
                            const float4 o = *reinterpret_cast<const float4*>(dst + 4 * q);
                            v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
                        }
                        *reinterpret_cast<float4*>(dst + 4 * q) = v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kUmMmaWarp)
    {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

}  // namespace hy
