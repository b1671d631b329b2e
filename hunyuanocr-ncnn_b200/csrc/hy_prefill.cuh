// Attention of many-row steps on the tensor cores: RoPE + QK RMSNorm + KV
// append for every row of a step, and the causal attention of those rows over
// the KV cache - for prompt prefill passes (up to 1024 rows; the projections
// are in hy_umma.cuh) and for the steps of 2..16 rows (DFlash verify blocks,
// decoder steps).
#pragma once

#include "hy_attn.cuh"
#include "hy_device.cuh"
#include "hy_gemv.cuh"
#include "hy_umma.cuh"

namespace hy {

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

// ---------------------------------------------------------------------------
// Prefill attention.
//
// RoPE + QK RMSNorm + KV append for every row of a prefill pass (the same
// per-head arithmetic as the decode/verify attention prologue): q heads are
// rewritten in place (times scale * log2 e), k heads and v heads go to the
// cache rows past .. past + rows - 1. Grid (rows, 4): one warp per (row, head).
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
    const DecodeState* st;   // when set, past = st->kv_len (rows appended at the current length)
    int rope_state;          // rope row of row m: (rope_state ? past : 0) + m
    int* err;                // kErrBounds when a row would land past the capacity
    int norm_first;          // DFlash draft: RMSNorm before RoPE (the decoder ropes first)
    int kv_only;             // only k / v heads (grid y = 2): context rows of the draft cache
};

template <typename KT>
__global__ void __launch_bounds__(256) prefill_rope_kernel(const PrefillRopeArgs a)
{
    HY_STEP_TRACE_OPEN(0x200000000ull);
    pdl_wait();
    HY_STEP_TRACE_MARK(2);
    pdl_launch();
    const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int past = a.st ? a.st->kv_len : a.past;
    if (past + m >= a.cap)
    {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrBounds);
        return;
    }
    const int rr = (a.rope_state ? past : 0) + m;
    float* row = a.qkv + static_cast<size_t>(m) * a.ldq;
    const float* c = a.cos + static_cast<size_t>(rr) * kHeadDim;
    const float* s = a.sin + static_cast<size_t>(rr) * kHeadDim;
    {
        // 0..15 q heads, 16..23 k heads, 24..31 v heads
        const int j = (a.kv_only ? kNumQHeads : 0) + blockIdx.y * 8 + warp;
        if (j < kNumQHeads)
        {
            float* x = row + j * kHeadDim;
            float o[4];
            if (a.norm_first) norm_rope_vec(x, c, s, a.qn_w, a.eps, lane, o);
            else rope_norm_vec(x, c, s, a.qn_w, a.eps, lane, o);
#pragma unroll
            for (int i = 0; i < 4; ++i) x[lane + 32 * i] = o[i] * a.scale_log2;
        }
        else if (j < kNumQHeads + kNumKVHeads)
        {
            const int h = j - kNumQHeads;
            float o[4];
            if (a.norm_first) norm_rope_vec(row + kQWidth + h * kHeadDim, c, s, a.kn_w, a.eps, lane, o);
            else rope_norm_vec(row + kQWidth + h * kHeadDim, c, s, a.kn_w, a.eps, lane, o);
            KT* dst = static_cast<KT*>(a.kc) + (static_cast<size_t>(h) * a.cap + past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = from_f32<KT>(o[i]);
        }
        else
        {
            const int h = j - kNumQHeads - kNumKVHeads;
            const float* x = row + kQWidth + kKVWidth + h * kHeadDim;
            KT* dst = static_cast<KT*>(a.vc) + (static_cast<size_t>(h) * a.cap + past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = from_f32<KT>(x[lane + 32 * i]);
        }
    }
    HY_STEP_TRACE_MARK(4);
    HY_STEP_TRACE_EXIT();
}

// Causal attention of the rows of a prefill pass over the cache rows
// [0, past + row] (PreciseSDPA::forward, src/precise_sdpa.cpp:281-329, with the
// prefill mask of src/text_runtime.cpp:207-219), flash-attention style on the
// tensor cores: S = Q K^T and O += P V as mma.sync m16n8k8 tf32 with the
// three-term split, an online base-2 softmax in fp32 between them.
//
// CTA = QR query rows x the 2 q heads of one KV head (2 QR query vectors, one
// m16 tile per warp), so each K/V tile in shared memory serves both heads,
// over one chunk of the rows' keys: K/V stream in 32-key tiles through a
// 2-stage cp.async ring.
//   Prefill (QR = 32, host work list): a row block whose keys span several
//   chunks (the causal mask makes later blocks longer) leaves per-chunk
//   partials (running max, sum, unnormalised output) that
//   prefill_attn_merge_kernel combines; a single-chunk block writes its output
//   directly, split and tiled for the o_proj GEMM.
//   Verify / decoder steps of <= 16 rows (QR = 16, no work list): the keys
//   [0, kv_len + rows) are cut into gridDim.x equal chunks on the device (the
//   length is read from the decode state), every CTA leaves a partial and
//   attn_chunk_merge_kernel merges them into the row-major output.
// Within a 8-key step of P V the k order is permuted (logical k = t <-> key
// 2t, k = t + 4 <-> key 2t + 1), so the S accumulator fragments are the P
// operand fragments as they lie, with no shuffles.
// ---------------------------------------------------------------------------
constexpr int kPaRows = 32, kPaKeys = 32, kPaThreads = 128;   // prefill: QR = 32 rows, 4 warps
constexpr int kPaMaxChunks = 4;            // chunks per row block at most
constexpr int kPaMinChunkTiles = 8;        // 32-key tiles per chunk at least
constexpr int kPaPartStride = 132;         // (max, sum, -, -) + out[128]
constexpr float kPaMasked = -1.0e30f;      // masked score (finite: a fully masked chunk merges with weight 0)

template <typename KT, int QR>
struct PaShape {
    static constexpr int THREADS = 4 * QR;                                       // 2 heads x QR / 16 warps
    static constexpr int KP = (sizeof(KT) == 4) ? kHeadDim + 4 : kHeadDim + 8;   // K/V tile pitch (elements)
    static constexpr int QP = kHeadDim + 4;                                      // Q tile pitch (floats)
    static constexpr int Q_BYTES = 2 * QR * QP * 4;
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
    float* out_hi;    // output [rows x 2048], split and tiled (rows_pad rows) for the o_proj GEMM
    float* out_lo;
    int rows_pad;
    const int4* work; // per CTA (blockIdx.x): row block, first and end 32-key tile, partial slot (-1: direct);
                      // nullptr: device-side chunks (QR = 16)
    float* part;      // [slot][8 KV heads][2 QR query vectors][kPaPartStride]
    const DecodeState* st;   // device-side chunks: past = st->kv_len when set
    int* err;         // kErrBounds when past + rows exceeds the capacity (nothing is read then)
    int noncausal;    // every row sees all keys [0, past + rows) (the DFlash draft's all-zero
                      // mask, src/dflash_runtime.cpp:50-58); device-side chunks only
};

template <typename KT, int QR>
__global__ void __launch_bounds__(4 * QR, 2) prefill_attn_kernel(const PrefillAttnArgs a)
{
    using S = PaShape<KT, QR>;
    constexpr int KP = S::KP, QP = S::QP, NT = S::THREADS;
    constexpr int NQV = 2 * QR;   // query vectors per CTA
    constexpr bool KV_EXACT = sizeof(KT) == 2;
    constexpr int EPC = 16 / static_cast<int>(sizeof(KT));
    constexpr int CPR = kHeadDim / EPC;
    extern __shared__ __align__(128) unsigned char smem[];
    float* Qs = reinterpret_cast<float*>(smem);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kvh = blockIdx.y;
    HY_STEP_TRACE_OPEN(0x300000000ull | QR);
    pdl_wait();
    HY_STEP_TRACE_MARK(2);
    pdl_launch();
    const bool dev = (a.work == nullptr);
    const int past = (dev && a.st) ? a.st->kv_len : a.past;
    int qb = 0, kb0, kb1, slot;
    if (!dev)
    {
        const int4 wk = a.work[blockIdx.x];
        qb = wk.x;
        kb0 = wk.y;
        kb1 = wk.z;
        slot = wk.w;
    }
    else
    {
        const int nkb = (past + a.rows + kPaKeys - 1) / kPaKeys;
        kb0 = static_cast<int>(blockIdx.x) * nkb / static_cast<int>(gridDim.x);
        kb1 = (static_cast<int>(blockIdx.x) + 1) * nkb / static_cast<int>(gridDim.x);
        slot = blockIdx.x;
    }
    if (past + a.rows > a.cap)
    {
        if (tid == 0 && a.err) atomicOr(a.err, kErrBounds);
        return;
    }
    const int m0 = qb * QR;
    const int nkeys = a.noncausal ? past + a.rows : min(past + m0 + QR, past + a.rows);
    const KT* kbase = static_cast<const KT*>(a.kc) + static_cast<size_t>(kvh) * a.cap * kHeadDim;
    const KT* vbase = static_cast<const KT*>(a.vc) + static_cast<size_t>(kvh) * a.cap * kHeadDim;

    auto load_kv = [&](int slot, int kb) {
        KT* Ks = reinterpret_cast<KT*>(smem + S::Q_BYTES + slot * S::STAGE);
        KT* Vs = Ks + kPaKeys * KP;
        for (int i = tid; i < kPaKeys * CPR; i += NT)
        {
            const int r = i / CPR, ch = i % CPR;
            const int key = kb * kPaKeys + r;
            const bool ok = key < nkeys;   // keys past the block's last row are zero-filled (and masked)
            const size_t off = static_cast<size_t>(ok ? key : 0) * kHeadDim + ch * EPC;
            cp_async16(Ks + r * KP + ch * EPC, kbase + off, ok);
            cp_async16(Vs + r * KP + ch * EPC, vbase + off, ok);
        }
    };

    // Query vector j = hl * QR + r: row m0 + r, q head 2 kvh + hl.
    for (int i = tid; i < NQV * (kHeadDim / 4); i += NT)
    {
        const int j = i / (kHeadDim / 4), ch = i % (kHeadDim / 4);
        const int hl = j / QR, r = j % QR;
        const bool ok = m0 + r < a.rows;
        const float* src = a.q + static_cast<size_t>(ok ? m0 + r : 0) * a.ldq + (2 * kvh + hl) * kHeadDim + ch * 4;
        cp_async16(Qs + j * QP + ch * 4, src, ok);
    }
    load_kv(0, kb0);
    cp_async_commit();

    const int hl = warp / (QR / 16), r0 = (warp % (QR / 16)) * 16;
    const float* Qw = Qs + (hl * QR + r0) * QP;
    // Last visible key of rows g and g + 8: their own positions (causal), or the last key.
    const int pq0 = a.noncausal ? nkeys - 1 : past + m0 + r0 + g;
    const int pq1 = a.noncausal ? nkeys - 1 : pq0 + 8;
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
    float mrow0 = kPaMasked, mrow1 = kPaMasked, l0 = 0.f, l1 = 0.f;

    for (int kb = kb0; kb < kb1; ++kb)
    {
        const int it = kb - kb0;
        if (kb + 1 < kb1) load_kv((it + 1) & 1, kb + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const KT* Ks = reinterpret_cast<const KT*>(smem + S::Q_BYTES + (it & 1) * S::STAGE);
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
                if (key > pq0) s[nt][e] = kPaMasked;
                if (key > pq1) s[nt][2 + e] = kPaMasked;
                mx0 = fmaxf(mx0, s[nt][e]);
                mx1 = fmaxf(mx1, s[nt][2 + e]);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // Keys come in increasing order: a row's first tile with a visible key makes its
        // max a real score, after which masked scores weigh exp2(-1e30 - max) = 0. A row
        // with no visible key in this chunk keeps max = -1e30 and merges with weight 0.
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
    const int h = 2 * kvh + hl;
    const int ma = m0 + r0 + g, mb = ma + 8;
    if (slot >= 0)
    {
        // Partial of this chunk: (max, sum) per query vector, unnormalised output.
        float* pa = a.part + ((static_cast<size_t>(slot) * kNumKVHeads + kvh) * NQV + hl * QR + r0 + g) * kPaPartStride;
        float* pb = pa + 8 * kPaPartStride;
        if (t == 0)
        {
            pa[0] = mrow0;
            pa[1] = l0;
            pb[0] = mrow1;
            pb[1] = l1;
        }
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
        {
            *reinterpret_cast<float2*>(pa + 4 + 8 * dt + 2 * t) = make_float2(o[dt][0], o[dt][1]);
            *reinterpret_cast<float2*>(pb + 4 + 8 * dt + 2 * t) = make_float2(o[dt][2], o[dt][3]);
        }
        return;
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
    {
        const int d = h * kHeadDim + 8 * dt + 2 * t;
        float xh, xl, yh, yl;
        if (ma < a.rows)
        {
            split_hi_lo(o[dt][0] * inv0, xh, xl);
            split_hi_lo(o[dt][1] * inv0, yh, yl);
            const size_t i = tiled_index(ma, d, a.rows_pad);
            *reinterpret_cast<float2*>(a.out_hi + i) = make_float2(xh, yh);
            *reinterpret_cast<float2*>(a.out_lo + i) = make_float2(xl, yl);
        }
        if (mb < a.rows)
        {
            split_hi_lo(o[dt][2] * inv1, xh, xl);
            split_hi_lo(o[dt][3] * inv1, yh, yl);
            const size_t i = tiled_index(mb, d, a.rows_pad);
            *reinterpret_cast<float2*>(a.out_hi + i) = make_float2(xh, yh);
            *reinterpret_cast<float2*>(a.out_lo + i) = make_float2(xl, yl);
        }
    }
    HY_STEP_TRACE_MARK(4);
    HY_STEP_TRACE_EXIT();
}

// Combines the chunk partials of a row block (merge item: row block, first
// slot, chunk count): out = sum_c 2^(m_c - M) acc_c / sum_c 2^(m_c - M) l_c,
// M = max_c m_c, written split and tiled. CTA = one item x one KV head; thread
// = (query vector tid / 4, 32 dims).
__global__ void __launch_bounds__(256) prefill_attn_merge_kernel(const float* __restrict__ part, const int4* __restrict__ items,
                                                                 int rows, int rows_pad, float* out_hi, float* out_lo)
{
    const int4 it = items[blockIdx.x];
    const int qb = it.x, slot0 = it.y, nch = it.z;
    const int kvh = blockIdx.y, tid = threadIdx.x;
    const int qv = tid >> 2, d0 = (tid & 3) * 32;
    const int r = qv % kPaRows, hl = qv / kPaRows;
    const int m = qb * kPaRows + r;
    if (m >= rows) return;
    auto base = [&](int c) {
        return part + ((static_cast<size_t>(slot0 + c) * kNumKVHeads + kvh) * 64 + qv) * kPaPartStride;
    };
    float M = kPaMasked;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, base(c)[0]);
    float L = 0.f;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    for (int c = 0; c < nch; ++c)
    {
        const float* p = base(c);
        const float w = exp2f(p[0] - M);
        L += w * p[1];
#pragma unroll
        for (int i = 0; i < 32; i += 4)
        {
            const float4 v = *reinterpret_cast<const float4*>(p + 4 + d0 + i);
            acc[i] += w * v.x;
            acc[i + 1] += w * v.y;
            acc[i + 2] += w * v.z;
            acc[i + 3] += w * v.w;
        }
    }
    const float inv = 1.0f / L;
    const int col = (2 * kvh + hl) * kHeadDim + d0;
#pragma unroll
    for (int i = 0; i < 32; i += 4)
        store_tiled4(out_hi, out_lo, rows_pad, m, col + i,
                     make_float4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv, acc[i + 3] * inv));
}

// Merge of the device-side chunks of a <= 16-row step: CTA = (query vector, KV
// head), thread = output dimension; every chunk's (max, sum, value) is loaded at
// once. out[row][head * 128 + d] = sum_c 2^(m_c - M) acc_c[d] / sum_c 2^(m_c - M) l_c.
constexpr int kMaxVerifyChunks = 40;
struct ChunkMergeArgs {
    const float* part;   // [chunk][8 KV heads][32 query vectors][kPaPartStride]
    int nch, rows;
    float* out;          // [rows x 2048]
};

__global__ void __launch_bounds__(kHeadDim) attn_chunk_merge_kernel(const ChunkMergeArgs a)
{
    HY_STEP_TRACE_OPEN(0x400000000ull);
    pdl_wait();
    HY_STEP_TRACE_MARK(2);
    pdl_launch();
    const int qv = blockIdx.x, kvh = blockIdx.y, d = threadIdx.x;   // qv = hl * 16 + row
    const int row = qv % 16, hl = qv / 16;
    if (row >= a.rows) return;
    const size_t cstride = static_cast<size_t>(kNumKVHeads) * 32 * kPaPartStride;
    const float* p0 = a.part + (static_cast<size_t>(kvh) * 32 + qv) * kPaPartStride;
    float m[kMaxVerifyChunks], l[kMaxVerifyChunks], v[kMaxVerifyChunks];
#pragma unroll
    for (int c = 0; c < kMaxVerifyChunks; ++c)
    {
        m[c] = kPaMasked;
        l[c] = 0.f;
        v[c] = 0.f;
        if (c < a.nch)
        {
            const float* p = p0 + c * cstride;
            m[c] = __ldcg(p);
            l[c] = __ldcg(p + 1);
            v[c] = __ldcg(p + 4 + d);
        }
    }
    float M = kPaMasked;
#pragma unroll
    for (int c = 0; c < kMaxVerifyChunks; ++c) M = fmaxf(M, m[c]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxVerifyChunks; ++c)
    {
        const float w = exp2f(m[c] - M);
        L += w * l[c];
        acc += w * v[c];
    }
    a.out[static_cast<size_t>(row) * kQWidth + (2 * kvh + hl) * kHeadDim + d] = acc / L;
    HY_STEP_TRACE_MARK(4);
    HY_STEP_TRACE_EXIT();
}

}  // namespace hy
