// Many-row projections for the prompt prefill:
//   C[M x N] (=, +=, or SwiGLU of) A[M x K] . W[N x K]^T
// with A the fp32 activation rows of the prompt and W a decoder linear
// ([out x in], fp32 or bf16), on the tensor cores.
//
// Replaces, for a prompt of M rows, the decoder's Gemm layers
// (export/text_decoder_kv.py:64-69, 93-95) that the reference runs once per
// prefill over the whole prompt (run_decoder_prefill, src/text_runtime.cpp:648-674). The 16-row
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

#include "hy_attn.cuh"
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


// ---------------------------------------------------------------------------
// Prefill attention.
//
// RoPE + QK RMSNorm + KV append for every row of a prefill pass (the same
// per-head arithmetic as the decode/verify attention prologue): q heads are
// rewritten in place (times scale * log2 e), k heads and v heads go to the
// cache rows past .. past + rows - 1. One CTA per row, a warp per 4 heads.
// ---------------------------------------------------------------------------
struct PrefillRopeArgs {
    float* qkv;   // [rows x ldq]: q [0, 2048) rewritten, k [2048, 3072), v [3072, 4096)
    int ldq;
    const float* cos;   // [rows x 128]
    const float* sin;
    const float* qn_w;
    const float* kn_w;
    void* kc;     // this layer's cache [8][cap][128] of KT
    void* vc;
    int cap, past;
    float eps, scale_log2;
};

template <typename KT>
__global__ void __launch_bounds__(256) prefill_rope_kernel(const PrefillRopeArgs a)
{
    const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* row = a.qkv + static_cast<size_t>(m) * a.ldq;
    const float* c = a.cos + static_cast<size_t>(m) * kHeadDim;
    const float* s = a.sin + static_cast<size_t>(m) * kHeadDim;
    for (int j = warp; j < kNumQHeads + 2 * kNumKVHeads; j += 8)
    {
        if (j < kNumQHeads)
        {
            float* x = row + j * kHeadDim;
            float o[4];
            rope_norm_vec(x, c, s, a.qn_w, a.eps, lane, o);
#pragma unroll
            for (int i = 0; i < 4; ++i) x[lane + 32 * i] = o[i] * a.scale_log2;
        }
        else if (j < kNumQHeads + kNumKVHeads)
        {
            const int h = j - kNumQHeads;
            float o[4];
            rope_norm_vec(row + kQWidth + h * kHeadDim, c, s, a.kn_w, a.eps, lane, o);
            KT* dst = static_cast<KT*>(a.kc) + (static_cast<size_t>(h) * a.cap + a.past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = from_f32<KT>(o[i]);
        }
        else
        {
            const int h = j - kNumQHeads - kNumKVHeads;
            const float* x = row + kQWidth + kKVWidth + h * kHeadDim;
            KT* dst = static_cast<KT*>(a.vc) + (static_cast<size_t>(h) * a.cap + a.past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = from_f32<KT>(x[lane + 32 * i]);
        }
    }
}

// Causal attention of the rows of a prefill pass over the cache rows
// [0, past + row] (PreciseSDPA::forward, src/precise_sdpa.cpp:281-329, with the
// prefill mask of src/text_runtime.cpp:207-219), flash-attention style on the
// tensor cores: S = Q K^T and O += P V as mma.sync m16n8k8 tf32 with the
// three-term split, an online base-2 softmax in fp32 between them.
//
// CTA = 32 query rows x the 2 q heads of one KV head (64 query vectors, one
// m16 tile per warp), so each K/V tile in shared memory serves both heads.
// K/V stream in 32-key tiles through a 2-stage cp.async ring; the heaviest
// (last) row blocks are scheduled first.
// Within a 8-key step of P V the k order is permuted (logical k = t <-> key
// 2t, k = t + 4 <-> key 2t + 1), so the S accumulator fragments are the P
// operand fragments as they lie, with no shuffles.
// ---------------------------------------------------------------------------
constexpr int kPaRows = 32, kPaKeys = 32, kPaThreads = 128;

template <typename KT>
struct PaShape {
    static constexpr int KP = (sizeof(KT) == 4) ? kHeadDim + 4 : kHeadDim + 8;   // K/V tile pitch (elements)
    static constexpr int QP = kHeadDim + 4;                                      // Q tile pitch (floats)
    static constexpr int Q_BYTES = 2 * kPaRows * QP * 4;
    static constexpr int T_BYTES = kPaKeys * KP * static_cast<int>(sizeof(KT));
    static constexpr int STAGE = 2 * T_BYTES;
    static constexpr int SMEM = Q_BYTES + 2 * STAGE;
    static_assert(Q_BYTES % 16 == 0 && T_BYTES % 16 == 0, "16-byte tile layout");
};

struct PrefillAttnArgs {
    const float* q;   // [rows x ldq]: roped, normed q heads times scale * log2 e
    int ldq;
    const void* kc;   // this layer's cache [8][cap][128] of KT, rows [0, past + rows) written
    const void* vc;
    int cap, past, rows;
    float* out;       // [rows x 2048]
};

template <typename KT>
__global__ void __launch_bounds__(kPaThreads, 2) prefill_attn_kernel(const PrefillAttnArgs a)
{
    using S = PaShape<KT>;
    constexpr int KP = S::KP, QP = S::QP;
    constexpr bool KV_EXACT = sizeof(KT) == 2;
    constexpr int EPC = 16 / static_cast<int>(sizeof(KT));
    constexpr int CPR = kHeadDim / EPC;
    extern __shared__ __align__(128) unsigned char smem[];
    float* Qs = reinterpret_cast<float*>(smem);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nqb = (a.rows + kPaRows - 1) / kPaRows;
    const int qb = nqb - 1 - static_cast<int>(blockIdx.x);
    const int kvh = blockIdx.y;
    const int m0 = qb * kPaRows;
    const int nkeys = min(a.past + m0 + kPaRows, a.past + a.rows);
    const int nkb = (nkeys + kPaKeys - 1) / kPaKeys;
    const KT* kbase = static_cast<const KT*>(a.kc) + static_cast<size_t>(kvh) * a.cap * kHeadDim;
    const KT* vbase = static_cast<const KT*>(a.vc) + static_cast<size_t>(kvh) * a.cap * kHeadDim;

    auto load_kv = [&](int slot, int kb) {
        KT* Ks = reinterpret_cast<KT*>(smem + S::Q_BYTES + slot * S::STAGE);
        KT* Vs = Ks + kPaKeys * KP;
        for (int i = tid; i < kPaKeys * CPR; i += kPaThreads)
        {
            const int r = i / CPR, ch = i % CPR;
            const int key = kb * kPaKeys + r;
            const bool ok = key < nkeys;   // keys past the block's last row are zero-filled (and masked)
            const size_t off = static_cast<size_t>(ok ? key : 0) * kHeadDim + ch * EPC;
            cp_async16(Ks + r * KP + ch * EPC, kbase + off, ok);
            cp_async16(Vs + r * KP + ch * EPC, vbase + off, ok);
        }
    };

    // Query vector j = hl * 32 + r: row m0 + r, q head 2 kvh + hl.
    for (int i = tid; i < 2 * kPaRows * (kHeadDim / 4); i += kPaThreads)
    {
        const int j = i / (kHeadDim / 4), ch = i % (kHeadDim / 4);
        const int hl = j / kPaRows, r = j % kPaRows;
        const bool ok = m0 + r < a.rows;
        const float* src = a.q + static_cast<size_t>(ok ? m0 + r : 0) * a.ldq + (2 * kvh + hl) * kHeadDim + ch * 4;
        cp_async16(Qs + j * QP + ch * 4, src, ok);
    }
    load_kv(0, 0);
    cp_async_commit();

    const int hl = warp >> 1, r0 = (warp & 1) * 16;
    const float* Qw = Qs + (hl * kPaRows + r0) * QP;
    const int pq0 = a.past + m0 + r0 + g, pq1 = pq0 + 8;   // positions of rows g and g + 8
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
    float mrow0 = -INFINITY, mrow1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int kb = 0; kb < nkb; ++kb)
    {
        if (kb + 1 < nkb) load_kv((kb + 1) & 1, kb + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const KT* Ks = reinterpret_cast<const KT*>(smem + S::Q_BYTES + (kb & 1) * S::STAGE);
        const KT* Vs = Ks + kPaKeys * KP;

        // S = Q K^T for 16 rows x 32 keys.
        float s[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll 4
        for (int ks = 0; ks < kHeadDim / 8; ++ks)
        {
            const float* qa = Qw + g * QP + 8 * ks + t;
            const float x[4] = {qa[0], qa[8 * QP], qa[4], qa[8 * QP + 4]};
            unsigned ah[4], al[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                ah[e] = tf32_head(x[e]);
                al[e] = __float_as_uint(x[e] - __uint_as_float(ah[e]));
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
            {
                const KT* kr = Ks + (8 * nt + g) * KP + 8 * ks + t;
                const float k0 = to_f32<KT>(kr[0]), k1 = to_f32<KT>(kr[4]);
                const unsigned bh0 = tf32_head(k0), bh1 = tf32_head(k1);
                mma_tf32(s[nt], al, bh0, bh1);
                if constexpr (!KV_EXACT)
                    mma_tf32(s[nt], ah, __float_as_uint(k0 - __uint_as_float(bh0)),
                             __float_as_uint(k1 - __uint_as_float(bh1)));
                mma_tf32(s[nt], ah, bh0, bh1);
            }
        }

        // Causal mask, online softmax (scores are already in log2 units).
        float mx0 = mrow0, mx1 = mrow1;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
            {
                const int key = kb * kPaKeys + 8 * nt + 2 * t + e;
                if (key > pq0) s[nt][e] = -INFINITY;
                if (key > pq1) s[nt][2 + e] = -INFINITY;
                mx0 = fmaxf(mx0, s[nt][e]);
                mx1 = fmaxf(mx1, s[nt][2 + e]);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // Key 0 is visible to every row, so mx0 / mx1 are finite from the first tile on.
        const float c0 = exp2f(mrow0 - mx0), c1 = exp2f(mrow1 - mx1);
        mrow0 = mx0;
        mrow1 = mx1;
        float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
            {
                s[nt][e] = exp2f(s[nt][e] - mx0);
                s[nt][2 + e] = exp2f(s[nt][2 + e] - mx1);
                ls0 += s[nt][e];
                ls1 += s[nt][2 + e];
            }
        l0 = l0 * c0 + ls0;   // per-lane partial sums; the quad adds them at the end
        l1 = l1 * c1 + ls1;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
        {
            o[dt][0] *= c0;
            o[dt][1] *= c0;
            o[dt][2] *= c1;
            o[dt][3] *= c1;
        }

        // O += P V: 4 steps of 8 keys x 16 tiles of 8 dims.
#pragma unroll
        for (int j = 0; j < 4; ++j)
        {
            const float p[4] = {s[j][0], s[j][2], s[j][1], s[j][3]};
            unsigned ph[4], pl[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
            {
                ph[e] = tf32_head(p[e]);
                pl[e] = __float_as_uint(p[e] - __uint_as_float(ph[e]));
            }
            const KT* vr = Vs + (8 * j + 2 * t) * KP + g;
#pragma unroll
            for (int dt = 0; dt < 16; ++dt)
            {
                const float v0 = to_f32<KT>(vr[8 * dt]), v1 = to_f32<KT>(vr[KP + 8 * dt]);
                const unsigned bh0 = tf32_head(v0), bh1 = tf32_head(v1);
                mma_tf32(o[dt], pl, bh0, bh1);
                if constexpr (!KV_EXACT)
                    mma_tf32(o[dt], ph, __float_as_uint(v0 - __uint_as_float(bh0)),
                             __float_as_uint(v1 - __uint_as_float(bh1)));
                mma_tf32(o[dt], ph, bh0, bh1);
            }
        }
        __syncthreads();   // every warp is done with this slot before it is refilled
    }
    cp_async_wait<0>();

    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    const int h = 2 * kvh + hl;
    const int ma = m0 + r0 + g, mb = ma + 8;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
    {
        const int d = h * kHeadDim + 8 * dt + 2 * t;
        if (ma < a.rows)
            *reinterpret_cast<float2*>(a.out + static_cast<size_t>(ma) * kQWidth + d) =
                make_float2(o[dt][0] * inv0, o[dt][1] * inv0);
        if (mb < a.rows)
            *reinterpret_cast<float2*>(a.out + static_cast<size_t>(mb) * kQWidth + d) =
                make_float2(o[dt][2] * inv1, o[dt][3] * inv1);
    }
}

}  // namespace hy
