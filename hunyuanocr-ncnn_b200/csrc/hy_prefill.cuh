// Many-row projections for the prompt prefill:
//   C[M x N] (=, +=, or SwiGLU of) A[M x K] . W[N x K]^T
// with A the fp32 activation rows of the prompt and W a decoder linear
// ([out x in], fp32 or bf16), on the tensor cores.
//
// Replaces, for a prompt of M rows, the decoder's Gemm layers
// (export/text_decoder_kv.py:64-69, 93-95) that the reference runs once per
// prefill over the whole prompt (src/text_runtime.cpp:1387-1420). The 16-row
// step kernels stream every weight once per 16 prompt rows; here a weight tile
// is read once per 128 rows and the work is compute-bound.
//
// Arithmetic: mma.sync m16n8k8 tf32 with a three-term split of the fp32
// operands (x = hi + lo, hi = x with the low 13 mantissa bits cleared):
// x.w ~ lo_x.hi_w + hi_x.lo_w + hi_x.hi_w, with fp32 accumulation; the
// dropped lo.lo term is below 2^-22 relative. bf16 weights are exact tf32
// values (lo_w = 0), so they take two products.
//
// Tiling: CTA tile 128 rows (M) x 64 weight rows (N) x 32 (K), 8 warps as 4 x 2
// with a 32 x 32 warp tile (2 x 4 m16n8 tiles). A 4-stage cp.async ring holds
// the A and W tiles at padded pitches (row + 16 bytes), so each warp's fragment
// loads fall in 32 distinct banks. Two CTAs per SM.
#pragma once

#include "hy_device.cuh"
#include "hy_gemv.cuh"

namespace hy {

enum { PG_STORE = 0, PG_RESID = 1, PG_SWIGLU = 2 };

constexpr int kPgBM = 128, kPgBN = 64, kPgBK = 32, kPgStages = 4, kPgThreads = 256;
constexpr int kPgAPitch = kPgBK + 4;   // floats

template <typename WT>
struct PgShape {
    static constexpr int BPITCH = (sizeof(WT) == 4) ? kPgBK + 4 : kPgBK + 8;   // elements (16-byte rows + 16 bytes)
    static constexpr int A_BYTES = kPgBM * kPgAPitch * 4;
    static constexpr int B_BYTES = kPgBN * BPITCH * static_cast<int>(sizeof(WT));
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int SMEM = kPgStages * STAGE;
    static_assert(A_BYTES % 16 == 0 && B_BYTES % 16 == 0, "16-byte stage layout");
};

struct PrefillGemmArgs {
    const float* A;   // [M x lda], row m at A + m * lda
    int lda;
    const void* W;    // [N x ldw] of WT
    int ldw;
    int M, N, K;      // N % 64 == 0, K % 32 == 0 (checked by the host)
    float* C;         // STORE: C[m, n]; RESID: C[m, n] += ; SWIGLU: C[m, n / 2] = silu(y[2j]) * y[2j + 1]
    int ldc;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(pred ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename WT, int EPI>
__global__ void __launch_bounds__(kPgThreads, 2) prefill_gemm_kernel(const PrefillGemmArgs a)
{
    using S = PgShape<WT>;
    constexpr int BP = S::BPITCH;
    constexpr bool W_EXACT = sizeof(WT) == 2;
    constexpr int EPC = 16 / static_cast<int>(sizeof(WT));   // W elements per 16-byte chunk
    constexpr int CPR = kPgBK / EPC;                          // W chunks per tile row
    extern __shared__ __align__(128) unsigned char smem[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 1, wn = warp & 1;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * kPgBN, m0 = blockIdx.y * kPgBM;
    const WT* W = static_cast<const WT*>(a.W);
    const int KT = a.K / kPgBK;

    auto load_stage = [&](int slot, int kt) {
        float* As = reinterpret_cast<float*>(smem + slot * S::STAGE);
        WT* Bs = reinterpret_cast<WT*>(smem + slot * S::STAGE + S::A_BYTES);
        const int k0 = kt * kPgBK;
#pragma unroll
        for (int i = tid; i < kPgBM * 8; i += kPgThreads)
        {
            const int r = i >> 3, ch = i & 7;
            const bool ok = m0 + r < a.M;   // rows past M are zero-filled
            const float* src = a.A + static_cast<size_t>(ok ? m0 + r : 0) * a.lda + k0 + ch * 4;
            cp_async16(As + r * kPgAPitch + ch * 4, src, ok);
        }
#pragma unroll
        for (int i = tid; i < kPgBN * CPR; i += kPgThreads)
        {
            const int r = i / CPR, ch = i % CPR;
            cp_async16(Bs + r * BP + ch * EPC, W + static_cast<size_t>(n0 + r) * a.ldw + k0 + ch * EPC, true);
        }
    };

    float acc[2][4][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;

#pragma unroll
    for (int s = 0; s < kPgStages - 1; ++s)
    {
        if (s < KT) load_stage(s, s);
        cp_async_commit();
    }
    for (int kt = 0; kt < KT; ++kt)
    {
        cp_async_wait<kPgStages - 2>();
        __syncthreads();   // tile kt landed for every thread; slot (kt - 1) % S is free
        {
            const int nk = kt + kPgStages - 1;
            if (nk < KT) load_stage(nk % kPgStages, nk);
            cp_async_commit();
        }
        const float* As = reinterpret_cast<const float*>(smem + (kt % kPgStages) * S::STAGE);
        const WT* Bs = reinterpret_cast<const WT*>(smem + (kt % kPgStages) * S::STAGE + S::A_BYTES);
#pragma unroll
        for (int k8 = 0; k8 < kPgBK / 8; ++k8)
        {
            const int kc = k8 * 8 + t;
            unsigned ah[2][4], al[2][4];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
            {
                const float* ar = As + (wm * 32 + mi * 16 + g) * kPgAPitch + kc;
                const float x[4] = {ar[0], ar[8 * kPgAPitch], ar[4], ar[8 * kPgAPitch + 4]};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                {
                    ah[mi][e] = tf32_head(x[e]);
                    al[mi][e] = __float_as_uint(x[e] - __uint_as_float(ah[mi][e]));
                }
            }
            unsigned bh[4][2], bl[4][2];
#pragma unroll
            for (int ni = 0; ni < 4; ++ni)
            {
                const WT* br = Bs + (wn * 32 + ni * 8 + g) * BP + kc;
                const float w0 = to_f32<WT>(br[0]), w1 = to_f32<WT>(br[4]);
                bh[ni][0] = tf32_head(w0);
                bh[ni][1] = tf32_head(w1);
                bl[ni][0] = __float_as_uint(w0 - __uint_as_float(bh[ni][0]));
                bl[ni][1] = __float_as_uint(w1 - __uint_as_float(bh[ni][1]));
            }
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int ni = 0; ni < 4; ++ni)
                {
                    mma_tf32(acc[mi][ni], al[mi], bh[ni][0], bh[ni][1]);
                    if constexpr (!W_EXACT) mma_tf32(acc[mi][ni], ah[mi], bl[ni][0], bl[ni][1]);
                    mma_tf32(acc[mi][ni], ah[mi], bh[ni][0], bh[ni][1]);
                }
        }
    }
    cp_async_wait<0>();   // only empty groups remain; leave nothing in flight

    // Epilogue: tile element (r, c) of acc[mi][ni]: e0 (g, 2t), e1 (g, 2t + 1), e2 (g + 8, 2t), e3 (g + 8, 2t + 1).
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int h = 0; h < 2; ++h)
        {
            const int m = m0 + wm * 32 + mi * 16 + g + 8 * h;
            if (m >= a.M) continue;
#pragma unroll
            for (int ni = 0; ni < 4; ++ni)
            {
                const int n = n0 + wn * 32 + ni * 8 + 2 * t;
                const float v0 = acc[mi][ni][2 * h], v1 = acc[mi][ni][2 * h + 1];
                if constexpr (EPI == PG_SWIGLU)
                {
                    // Rows 2j / 2j + 1 of the gate/up weight are gate_j / up_j.
                    a.C[static_cast<size_t>(m) * a.ldc + (n >> 1)] = (v0 / (1.0f + expf(-v0))) * v1;
                }
                else
                {
                    float2* p = reinterpret_cast<float2*>(a.C + static_cast<size_t>(m) * a.ldc + n);
                    if constexpr (EPI == PG_RESID)
                    {
                        const float2 r = *p;
                        *p = make_float2(r.x + v0, r.y + v1);
                    }
                    else
                    {
                        *p = make_float2(v0, v1);
                    }
                }
            }
        }
}

}  // namespace hy
