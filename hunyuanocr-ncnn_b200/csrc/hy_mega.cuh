// Persistent AR decode kernel: whole tokens (embed -> 24 layers -> LM head ->
// penalised argmax -> commit) in one cooperative launch, one CTA per SM.
//
// The decode step of the reference (decode_from_embeddings' loop,
// src/text_runtime.cpp:1417-1508, executing the graph of
// export/text_decoder_kv.py:49-96 plus the LM head and select_next_token) is
// a chain of 121 dependent phases per token: for each layer q/k/v projection,
// attention, o projection, gate/up projection, down projection; then the LM
// head. Each phase reads a different slice of the weights, and no weight byte
// depends on an activation. So the kernel splits every CTA into
//   - a producer warp that walks the token's phase list and streams this CTA's
//     share of every phase (weight rows, or the K/V rows of its attention
//     split) through a 12-stage x 16 KB shared-memory ring with cp.async.bulk;
//     it only waits for free ring slots, never for the grid, so HBM stays busy
//     while the consumers cross a phase boundary;
//   - 8 consumer warps that, per phase, wait on a grid barrier (the phase's
//     input activations are complete), stage the activation vector in shared
//     memory (with the fused RMSNorm / SwiGLU / embedding gather), consume the
//     ring stages of that phase and write their outputs, then arrive on the
//     barrier.
// Attention splits each KV head's keys over 17 CTAs plus one CTA for the new
// row (RoPE + QK-norm + append); the last CTA of a head (atomic ticket) merges
// the partials. The LM head's last CTA merges the per-CTA argmax partials and
// commits the token (token log, state, penalty history).
//
// The grid barrier is a monotonic counter (zeroed before each launch): phase p
// may start when it reaches p * gridDim.x. All waits are bounded by wall clock;
// a wait that gives up sets the error word and the CTA winds down (the
// producer drains its in-flight copies first).
#pragma once

#include "hy_attn.cuh"
#include "hy_device.cuh"
#include "hy_gemv.cuh"

namespace hy {

constexpr int kMegaWarps = 8;
constexpr int kMegaThreads = (kMegaWarps + 1) * 32;
constexpr int kMegaStage = 16384;
constexpr int kMegaNst = 13;
constexpr int kMegaSplits = 9;    // per KV head: 8 splits of the past rows + the new-row split
constexpr int kMegaMaxK = 3584;

struct MegaArgs {
    const void* embed;
    const void* const* wqkv;  // device arrays of per-layer weight pointers
    const void* const* wo;
    const void* const* wgu;
    const void* const* wd;
    const float* norms;       // per layer: input[1024], post[1024], q_norm[128], k_norm[128]; final[1024] after
    void* kc;                 // [L][8][cap][128] of KT
    void* vc;
    int cap;
    const float* rope_cos;    // [cap][128]
    const float* rope_sin;
    float* x;                 // residual stream [1024]
    float* qkv;               // [4096]
    float* attn;              // [2048]
    float* gu;                // [2 * ffn]
    float* attn_part;         // [8][kMegaSplits][2][kPartStride]
    int* attn_cnt;            // [L][8]
    float4* lm_part;          // [gridDim.x]
    int* lm_cnt;
    unsigned* hist;
    DecodeState* st;
    int* log_tokens;
    int* log_raw;
    unsigned* bar;            // grid barrier counter, zero at launch
    int num_layers, vocab, ffn;
    float eps, scale_log2;
    int steps;                // tokens in this launch
    int* err;
    // Optional phase trace: for CTAs b < kTraceCtas and token trace_token,
    // %globaltimer at phase start, after the grid wait, after the prologue and at
    // the barrier arrive (consumer thread 0), then the producer's first and last
    // stage issue of the phase: trace[(b * phases + ph) * kTraceSlots + i].
    unsigned long long* trace;
    int trace_token;
    // Self-checks: the first failed bounds check stores (code, cta, phase, index)
    // in dbg[0..3] and the access is skipped. progress (host-mapped, nullable):
    // thread 0 of each CTA stores the number of phases it completed.
    int* dbg;
    volatile unsigned* progress;
};

__device__ __forceinline__ bool mega_check(bool ok, int* dbg, int code, int b, int ph, int idx)
{
    if (ok) return true;
    if (dbg && atomicCAS(dbg, 0, code) == 0)
    {
        dbg[1] = b;
        dbg[2] = ph;
        dbg[3] = idx;
    }
    return false;
}

constexpr int kTraceCtas = 4;
constexpr int kTraceSlots = 12;

struct MegaSmem {
    static constexpr int RING = 0;
    static constexpr int XS = RING + kMegaNst * kMegaStage;            // [3584] f32 activation vector
    // Attention phases do not use the activation vector; their buffers alias it.
    static constexpr int QS = XS;                                       // [2][128]
    static constexpr int NEWKV = QS + 2 * kHeadDim * 4;                 // k[128], v[128]
    static constexpr int ASCR = NEWKV + 2 * kHeadDim * 4;               // [8 warps][2][kPartStride]
    static_assert(ASCR + kMegaWarps * 2 * kPartStride * 4 <= XS + kMegaMaxK * 4, "attention scratch must fit");
    static constexpr int RED = XS + kMegaMaxK * 4;                      // 64 float4 + ints
    static constexpr int BARS = RED + 64 * 16 + 64 * 4;
    static constexpr int SIZE = BARS + 2 * kMegaNst * 8;
};

enum { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

// What this CTA streams in one phase.
struct MegaPlan {
    const unsigned char* src;   // gemv: first row of this CTA; attn: first K row
    const unsigned char* src2;  // attn: first V row
    int kind;
    int K;                      // gemv: row length (elements)
    int r0;                     // gemv: first row index
    int count;                  // gemv: rows; attn: key positions
    int unit_bytes;             // gemv: bytes per row; attn: bytes per K (or V) row
    int per_stage;              // rows / positions per ring stage
    int nstage;
    int g, split, p0;           // attn
};

template <typename WT, typename KT>
__device__ __forceinline__ MegaPlan mega_plan(const MegaArgs& a, int layer, int kind, int past, int b, int G)
{
    MegaPlan p;
    p.kind = kind;
    p.src = p.src2 = nullptr;
    p.g = p.split = p.p0 = 0;
    if (kind == PH_ATTN)
    {
        p.K = kHeadDim;
        p.r0 = 0;
        p.unit_bytes = kHeadDim * static_cast<int>(sizeof(KT));
        p.per_stage = kMegaStage / (2 * p.unit_bytes);
        p.count = 0;
        if (b < kNumKVHeads * kMegaSplits)
        {
            p.g = b / kMegaSplits;
            p.split = b % kMegaSplits;
            if (p.split < kMegaSplits - 1)
            {
                const int chunk = (past + kMegaSplits - 2) / (kMegaSplits - 1);
                const int p0 = min(past, p.split * chunk);
                const int p1 = min(past, p0 + chunk);
                p.p0 = p0;
                p.count = p1 - p0;
                const size_t off = ((static_cast<size_t>(layer) * kNumKVHeads + p.g) * a.cap + p0) * kHeadDim * sizeof(KT);
                p.src = static_cast<const unsigned char*>(a.kc) + off;
                p.src2 = static_cast<const unsigned char*>(a.vc) + off;
            }
        }
        p.nstage = (p.count + p.per_stage - 1) / p.per_stage;
        return p;
    }
    const void* W;
    int N;
    switch (kind)
    {
    case PH_QKV: W = a.wqkv[layer]; N = kQKVRows; p.K = kHidden; break;
    case PH_O: W = a.wo[layer]; N = kHidden; p.K = kQWidth; break;
    case PH_GU: W = a.wgu[layer]; N = 2 * a.ffn; p.K = kHidden; break;
    case PH_DOWN: W = a.wd[layer]; N = kHidden; p.K = a.ffn; break;
    default: W = a.embed; N = a.vocab; p.K = kHidden; break;
    }
    // gate/up rows are interleaved (2j = gate_j, 2j+1 = up_j): split that phase by pairs.
    const int unit = (kind == PH_GU) ? 2 : 1;
    p.r0 = unit * static_cast<int>(static_cast<long long>(N / unit) * b / G);
    const int r1 = unit * static_cast<int>(static_cast<long long>(N / unit) * (b + 1) / G);
    p.count = r1 - p.r0;
    p.unit_bytes = p.K * static_cast<int>(sizeof(WT));
    p.per_stage = max(1, kMegaStage / p.unit_bytes);
    p.nstage = (p.count + p.per_stage - 1) / p.per_stage;
    p.src = static_cast<const unsigned char*>(W) + static_cast<size_t>(p.r0) * p.unit_bytes;
    return p;
}

__device__ __forceinline__ void mega_phase_of(int ph, int num_layers, int& layer, int& kind)
{
    if (ph < 5 * num_layers)
    {
        layer = ph / 5;
        kind = ph % 5;
    }
    else
    {
        layer = num_layers;
        kind = PH_LM;
    }
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0 only: poll with acquire loads. Returns false on timeout.
// (Measured on B200 under streaming load: __threadfence + atomicAdd + acquire
// polling costs ~2.0 us per grid barrier; red.release or a trailing
// fence.acq_rel.gpu costs ~3.0 us.)
__device__ __forceinline__ bool grid_wait(const unsigned* bar, unsigned target, int* err)
{
    if (ld_acquire_u32(bar) >= target) return true;
    const unsigned long long t0 = global_ns();
    while (true)
    {
        for (int i = 0; i < 16; ++i)
        {
            if (ld_acquire_u32(bar) >= target) return true;
            __nanosleep(20);
        }
        if (global_ns() - t0 > kWaitLimitNs)
        {
            atomicOr(err, kErrTimeoutFull);
            return false;
        }
    }
}

// Thread 0 after a CTA barrier: make the CTA's writes visible, then count in.
__device__ __forceinline__ void grid_arrive(unsigned* bar)
{
    __threadfence();
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// <row0, xs> and <row1, xs> over K elements by one warp: lane-strided float4s,
// two accumulators per row to shorten the FMA chains, and one interleaved
// butterfly for both sums. `two` is warp-uniform; row1 is not read without it.
template <typename WT, int K>
__device__ __forceinline__ float2 row_dot2(const WT* row0, const WT* row1, const float* xs, int lane, bool two)
{
    static_assert(K % 128 == 0, "K must be a multiple of 128");
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int i = 0; i < K / 128; ++i)
    {
        const int c = lane + 32 * i;
        const float4 xv = *reinterpret_cast<const float4*>(xs + 4 * c);
        const float4 w0 = load4(row0 + 4 * c);
        if (i & 1) a1 += dot4(w0, xv);
        else a0 += dot4(w0, xv);
        if (two)
        {
            const float4 w1 = load4(row1 + 4 * c);
            if (i & 1) b1 += dot4(w1, xv);
            else b0 += dot4(w1, xv);
        }
    }
    float a = a0 + a1, b = b0 + b1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    return make_float2(a, b);
}

constexpr int kMegaHistWords = 64;   // LM rows per CTA <= 32 * 62

// RoPE + RMSNorm of one 128-vector (as rope_norm_vec) whose source was
// written by other CTAs of this launch: read through L2, never a stale L1 line.
__device__ __forceinline__ void rope_norm_vec_cg(const float* x, const float* c, const float* s, const float* w,
                                                 float eps, int lane, float out[4])
{
    const float x0 = __ldcg(x + lane), x1 = __ldcg(x + lane + 32), x2 = __ldcg(x + lane + 64), x3 = __ldcg(x + lane + 96);
    float y0 = x0 * c[lane] - x2 * s[lane];
    float y1 = x1 * c[lane + 32] - x3 * s[lane + 32];
    float y2 = x2 * c[lane + 64] + x0 * s[lane + 64];
    float y3 = x3 * c[lane + 96] + x1 * s[lane + 96];
    const float ss = warp_sum(y0 * y0 + y1 * y1 + y2 * y2 + y3 * y3);
    const float ri = 1.0f / sqrtf(ss / static_cast<float>(kHeadDim) + eps);
    out[0] = w[lane] * (y0 * ri);
    out[1] = w[lane + 32] * (y1 * ri);
    out[2] = w[lane + 64] * (y2 * ri);
    out[3] = w[lane + 96] * (y3 * ri);
}

// xs = w * x for a 1024-vector x written by other CTAs; returns 1/sqrt(mean(x^2)+eps)
// after one CTA barrier. The GEMV multiplies its dot products by it, i.e. the
// RMSNorm's per-row scale is applied after the projection.
__device__ __forceinline__ float mega_load_normed(float* xs, float4 v, const float* w, float eps, float* s_norm, int tid)
{
    const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    const float4 wv = *reinterpret_cast<const float4*>(w + tid * 4);
    float4 o;
    o.x = wv.x * v.x;
    o.y = wv.y * v.y;
    o.z = wv.z * v.z;
    o.w = wv.w * v.w;
    *reinterpret_cast<float4*>(xs + tid * 4) = o;
    if ((tid & 31) == 0) s_norm[tid >> 5] = ss;
    consumers_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kMegaWarps; ++i) t += s_norm[i];
    return 1.0f / sqrtf(t / static_cast<float>(kHidden) + eps);
}

template <typename WT, typename KT>
__global__ void __launch_bounds__(kMegaThreads, 1) mega_decode_kernel(const MegaArgs a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* ring = smem + MegaSmem::RING;
    float* xs = reinterpret_cast<float*>(smem + MegaSmem::XS);
    float* qs = reinterpret_cast<float*>(smem + MegaSmem::QS);
    float* knew = reinterpret_cast<float*>(smem + MegaSmem::NEWKV);
    float* vnew = knew + kHeadDim;
    float* ascr = reinterpret_cast<float*>(smem + MegaSmem::ASCR);
    float4* red4 = reinterpret_cast<float4*>(smem + MegaSmem::RED);
    int* redi = reinterpret_cast<int*>(red4 + 64);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + MegaSmem::BARS);
    uint64_t* empty = full + kMegaNst;
    __shared__ unsigned hist_s[kMegaHistWords];
    __shared__ float s_norm[kMegaWarps];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int L = a.num_layers;
    const int phases = 5 * L + 1;
    const int kv0 = a.st->kv_len;  // set by the host before the launch

    if (tid == 0)
    {
        for (int s = 0; s < kMegaNst; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMegaWarps);
        }
        fence_mbar_init();
        redi[0] = 0;  // abort flag
    }
    __syncthreads();

    if (warp == kMegaWarps)
    {
        // ======================= producer =======================
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first_policy();
        unsigned gs = 0;
        bool ok = true;
        for (int t = 0; t < a.steps && ok; ++t)
        {
            const int past = kv0 + t;
            for (int ph = 0; ph < phases && ok; ++ph)
            {
                int layer, kind;
                mega_phase_of(ph, L, layer, kind);
                const MegaPlan p = mega_plan<WT, KT>(a, layer, kind, past, b, G);
                if (kind == PH_ATTN && p.nstage > 0) asm volatile("fence.proxy.async.global;" ::: "memory");
                unsigned long long* ptr_ = (a.trace && t == a.trace_token && b < kTraceCtas)
                                               ? a.trace + (static_cast<size_t>(b) * phases + ph) * kTraceSlots
                                               : nullptr;
                for (int i = 0; i < p.nstage; ++i, ++gs)
                {
                    const int slot = gs % kMegaNst;
                    if (gs >= kMegaNst && !mbar_wait(&empty[slot], ((gs / kMegaNst) - 1) & 1, a.err, kErrTimeoutEmpty))
                    {
                        ok = false;
                        break;
                    }
                    if (ptr_)
                    {
                        if (i == 0) ptr_[4] = global_ns();
                        if (i == p.nstage - 1) ptr_[5] = global_ns();
                    }
                    const int n = min(p.per_stage, p.count - i * p.per_stage);
                    const uint32_t bytes = static_cast<uint32_t>(n * p.unit_bytes);
                    unsigned char* dst = ring + slot * kMegaStage;
                    const size_t off = static_cast<size_t>(i) * p.per_stage * p.unit_bytes;
                    if (kind == PH_ATTN)
                    {
                        mbar_arrive_expect_tx(&full[slot], 2 * bytes);
                        bulk_g2s(dst, p.src + off, bytes, &full[slot], pol);
                        bulk_g2s(dst + p.per_stage * p.unit_bytes, p.src2 + off, bytes, &full[slot], pol);
                    }
                    else
                    {
                        mbar_arrive_expect_tx(&full[slot], bytes);
                        bulk_g2s(dst, p.src + off, bytes, &full[slot], pol);
                    }
                }
            }
        }
        // Drain: the last kMegaNst stages issued (earlier ones completed before their slot was reused).
        const unsigned first = gs > kMegaNst ? gs - kMegaNst : 0;
        for (unsigned i = first; i < gs; ++i) mbar_wait(&full[i % kMegaNst], (i / kMegaNst) & 1, a.err, kErrTimeoutFull);
        return;
    }

    // ======================= consumers =======================
    unsigned gs = 0;
    unsigned phase_no = 0;
    float* xg = a.x;
    // A failed ring wait marks this warp bad; every warp still walks the same
    // sequence of CTA barriers, and the CTA leaves together after the phase.
    bool bad = false;
    // Per-warp argmax trackers for the LM phase.
    for (int t = 0; t < a.steps; ++t)
    {
        const int past = kv0 + t;
        for (int ph = 0; ph < phases; ++ph, ++phase_no)
        {
            int layer, kind;
            mega_phase_of(ph, L, layer, kind);
            const bool tracing = a.trace && t == a.trace_token && b < kTraceCtas && tid == 0;
            unsigned long long* tr = tracing ? a.trace + (static_cast<size_t>(b) * phases + ph) * kTraceSlots : nullptr;
            if (tracing) tr[0] = global_ns();
            if (phase_no > 0)
            {
                if (tid == 0 && !grid_wait(a.bar, phase_no * G, a.err)) redi[0] = 1;
                consumers_sync();
                if (redi[0]) return;
            }
            if (tracing) tr[1] = global_ns();
            const MegaPlan p = mega_plan<WT, KT>(a, layer, kind, past, b, G);
            const float* lnorm = a.norms + static_cast<size_t>(layer) * 2304;

            // ---------------- prologue: activation vector ----------------
            float rinv = 1.0f;   // RMSNorm scale applied to the dot products
            if (kind == PH_QKV)
            {
                float4 v;
                if (layer == 0)
                {
                    int id = __ldcg(&a.st->cur_token);
                    if (id < 0 || id >= a.vocab)
                    {
                        if (tid == 0) atomicOr(a.err, kErrBounds);
                        id = 0;
                    }
                    v = load4(static_cast<const WT*>(a.embed) + static_cast<size_t>(id) * kHidden + tid * 4);
                    // Publish this CTA's slice of the residual stream.
                    const int chunk = (kHidden + G - 1) / G;
                    const int i = b * chunk + tid;
                    if (tid < chunk && i < kHidden) xg[i] = to_f32<WT>(static_cast<const WT*>(a.embed)[static_cast<size_t>(id) * kHidden + i]);
                }
                else
                {
                    v = __ldcg(reinterpret_cast<const float4*>(xg) + tid);
                }
                rinv = mega_load_normed(xs, v, lnorm, a.eps, s_norm, tid);
            }
            else if (kind == PH_O)
            {
                // Merge the attention partials of every split (split-K flash-decode
                // combine): thread t handles q head t / 16, dims 8 * (t % 16) .. +8.
                // All loads are issued before any use, so this is one L2 round trip.
                const int h = tid >> 4, d0 = (tid & 15) * 8;
                const float* hp = a.attn_part + (static_cast<size_t>(h >> 1) * kMegaSplits * 2 + (h & 1)) * kPartStride;
                float ms[kMegaSplits], ls[kMegaSplits];
                float4 va[kMegaSplits], vb[kMegaSplits];
#pragma unroll
                for (int sp = 0; sp < kMegaSplits; ++sp)
                {
                    const float* ps = hp + static_cast<size_t>(sp) * 2 * kPartStride;
                    ms[sp] = __ldcg(ps);
                    ls[sp] = __ldcg(ps + 1);
                    va[sp] = __ldcg(reinterpret_cast<const float4*>(ps + 4 + d0));
                    vb[sp] = __ldcg(reinterpret_cast<const float4*>(ps + 8 + d0));
                }
                float M = -INFINITY;
#pragma unroll
                for (int sp = 0; sp < kMegaSplits; ++sp) M = fmaxf(M, ms[sp]);
                float Lsum = 0.f;
                float4 A0 = make_float4(0.f, 0.f, 0.f, 0.f), A1 = A0;
#pragma unroll
                for (int sp = 0; sp < kMegaSplits; ++sp)
                {
                    const float f = (ms[sp] == -INFINITY) ? 0.f : exp2f(ms[sp] - M);
                    Lsum += f * ls[sp];
                    A0.x += f * va[sp].x; A0.y += f * va[sp].y; A0.z += f * va[sp].z; A0.w += f * va[sp].w;
                    A1.x += f * vb[sp].x; A1.y += f * vb[sp].y; A1.z += f * vb[sp].z; A1.w += f * vb[sp].w;
                }
                const float inv = 1.0f / Lsum;
                A0.x *= inv; A0.y *= inv; A0.z *= inv; A0.w *= inv;
                A1.x *= inv; A1.y *= inv; A1.z *= inv; A1.w *= inv;
                *reinterpret_cast<float4*>(xs + h * kHeadDim + d0) = A0;
                *reinterpret_cast<float4*>(xs + h * kHeadDim + d0 + 4) = A1;
                consumers_sync();
            }
            else if (kind == PH_GU || kind == PH_LM)
            {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(xg) + tid);
                if (kind == PH_LM && p.count > 0)
                {
                    // Penalty-history words covering this CTA's vocab rows.
                    const int w0 = p.r0 >> 5, w1 = (p.r0 + p.count - 1) >> 5;
                    if (tid <= w1 - w0 && tid < kMegaHistWords) hist_s[tid] = __ldcg(a.hist + w0 + tid);
                }
                rinv = mega_load_normed(xs, v, kind == PH_GU ? lnorm + kHidden : a.norms + static_cast<size_t>(L) * 2304,
                                        a.eps, s_norm, tid);
            }
            else if (kind == PH_DOWN)
            {
                // The gate/up phase already wrote act = silu(gate) * up; all loads issue before use.
                constexpr int kPer = (kMegaMaxK / 4 + 255) / 256;
                float4 av[kPer];
#pragma unroll
                for (int u = 0; u < kPer; ++u)
                {
                    const int i = tid + 256 * u;
                    if (i < a.ffn / 4) av[u] = __ldcg(reinterpret_cast<const float4*>(a.gu) + i);
                }
#pragma unroll
                for (int u = 0; u < kPer; ++u)
                {
                    const int i = tid + 256 * u;
                    if (i < a.ffn / 4) reinterpret_cast<float4*>(xs)[i] = av[u];
                }
                consumers_sync();
            }

            if (tracing) tr[2] = global_ns();
            if (kind != PH_ATTN)
            {
                // ---------------- GEMV rows ----------------
                float best_rv = 0.f, best_pv = 0.f;
                int best_ri = -1, best_pi = -1;
                const float pen = a.st->penalty;
                const WT* ringw = reinterpret_cast<const WT*>(ring);
                // Units of up to two rows (a gate/up pair for PH_GU): unit o belongs to
                // warp o % 8 and its rows share one ring stage. Every warp observes
                // every stage of the phase in order and arrives once on it (the
                // owner after its dot products, the others at once): an mbarrier
                // parity wait is only meaningful one phase ahead, so no warp may skip
                // ahead of a stage that has not landed, nor let a slot be reused
                // before it has seen it.
                const int rpu = (p.per_stage >= 2) ? 2 : 1;
                const unsigned gs0 = gs;
                int o = warp;   // next unit this warp owns
                // Residual rows of this warp's first unit, fetched now so the
                // epilogue's read-modify-write does not wait on L2.
                float xpre0 = 0.f, xpre1 = 0.f;
                if ((kind == PH_O || kind == PH_DOWN) && lane == 0 && warp * rpu < p.count)
                {
                    xpre0 = __ldcg(xg + p.r0 + warp * rpu);
                    if (rpu == 2 && warp * rpu + 1 < p.count) xpre1 = __ldcg(xg + p.r0 + warp * rpu + 1);
                }
                unsigned long long t_wait = 0, t_dot = 0, n_units = 0;   // warp-0 trace accumulators
                for (int i = 0; i < p.nstage && !bad; ++i)
                {
                    const unsigned gsi = gs0 + i;
                    const int slot = gsi % kMegaNst;
                    const unsigned long long tw0 = tracing ? global_ns() : 0;
                    const bool okw = mbar_wait(&full[slot], (gsi / kMegaNst) & 1, a.err, kErrTimeoutFull);
                    if (tracing) t_wait += global_ns() - tw0;
                    if (!__all_sync(0xffffffffu, okw))
                    {
                        if (lane == 0) redi[0] = 1;
                        bad = true;
                        break;
                    }
                    if (tracing)
                    {
                        if (i == 0) tr[6] = global_ns();
                        if (i == p.nstage - 1) tr[7] = global_ns();
                    }
                    const int row_end = min(p.count, (i + 1) * p.per_stage);
                    const int q = o * rpu;
                    const bool mine = q < row_end;   // at most one unit per warp per stage
                    const bool two = mine && (rpu == 2) && (q + 1 < p.count);
                    float2 d = make_float2(0.f, 0.f);
                    const unsigned long long td0 = tracing ? global_ns() : 0;
                    if (mine)
                    {
                        const int j = q - i * p.per_stage;
                        const WT* row = ringw + (static_cast<size_t>(slot) * kMegaStage) / sizeof(WT) + static_cast<size_t>(j) * p.K;
                        if (mega_check(j >= 0 && (j + (two ? 2 : 1)) * p.K * static_cast<int>(sizeof(WT)) <= kMegaStage,
                                       a.dbg, 1, b, ph, j * 1000 + p.K))
                        {
                            if (p.K == kHidden) d = row_dot2<WT, kHidden>(row, row + kHidden, xs, lane, two);
                            else if (p.K == kQWidth) d = row_dot2<WT, kQWidth>(row, row + kQWidth, xs, lane, two);
                            else d = row_dot2<WT, kMegaMaxK>(row, row + kMegaMaxK, xs, lane, two);
                        }
                        o += kMegaWarps;
                    }
                    __syncwarp();
                    if (tracing && mine)
                    {
                        t_dot += global_ns() - td0;
                        ++n_units;
                    }
                    if (lane == 0) mbar_arrive(&empty[slot]);
                    if (mine && lane == 0)
                    {
                        const int nrow = p.r0 + q;
                        const float v0 = d.x * rinv, v1 = d.y * rinv;
                        const int nlimit = (kind == PH_QKV) ? kQKVRows : (kind == PH_GU) ? 2 * a.ffn
                                         : (kind == PH_LM) ? a.vocab : kHidden;
                        if (!mega_check(nrow >= 0 && nrow + (two ? 1 : 0) < nlimit, a.dbg, 2, b, ph, nrow)) continue;
                        if (kind == PH_QKV)
                        {
                            a.qkv[nrow] = v0;
                            if (two) a.qkv[nrow + 1] = v1;
                        }
                        else if (kind == PH_GU)
                        {
                            a.gu[nrow >> 1] = (v0 / (1.0f + expf(-v0))) * v1;   // act = silu(gate) * up
                        }
                        else if (kind == PH_O || kind == PH_DOWN)
                        {
                            const bool first = (q == warp * rpu);
                            const float x0 = first ? xpre0 : __ldcg(xg + nrow);
                            const float x1 = two ? (first ? xpre1 : __ldcg(xg + nrow + 1)) : 0.f;
                            xg[nrow] = x0 + v0;
                            if (two) xg[nrow + 1] = x1 + v1;
                        }
                        else
                        {
                            for (int r = 0; r < (two ? 2 : 1); ++r)
                            {
                                const float acc = r ? v1 : v0;
                                const int vr = nrow + r;
                                const int wi = (vr >> 5) - (p.r0 >> 5);
                                if (!mega_check(wi >= 0 && wi < kMegaHistWords, a.dbg, 3, b, ph, wi)) continue;
                                const bool hit = (hist_s[wi] >> (vr & 31)) & 1u;
                                const float ps = hit ? (acc < 0.0f ? acc * pen : acc / pen) : acc;
                                if (best_ri < 0 || acc > best_rv) { best_rv = acc; best_ri = vr; }
                                if (best_pi < 0 || ps > best_pv) { best_pv = ps; best_pi = vr; }
                            }
                        }
                    }
                }
                gs = gs0 + p.nstage;
                if (tracing)
                {
                    tr[8] = t_wait;
                    tr[9] = t_dot;
                    tr[10] = n_units;
                }
                if (kind == PH_LM)
                {
                    if (lane == 0) red4[warp] = make_float4(best_rv, __int_as_float(best_ri), best_pv, __int_as_float(best_pi));
                    consumers_sync();
                    if (tid == 0)
                    {
                        float rv = 0.f, pv = 0.f;
                        int ri = -1, pi = -1;
                        for (int w = 0; w < kMegaWarps; ++w)
                        {
                            const float4 v = red4[w];
                            if (__float_as_int(v.y) >= 0) best_update(rv, ri, v.x, __float_as_int(v.y));
                            if (__float_as_int(v.w) >= 0) best_update(pv, pi, v.z, __float_as_int(v.w));
                        }
                        a.lm_part[b] = make_float4(rv, __int_as_float(ri), pv, __int_as_float(pi));
                        __threadfence();
                        redi[1] = (atomicAdd(a.lm_cnt, 1) == G - 1) ? 1 : 0;
                    }
                    consumers_sync();
                    if (redi[1])
                    {
                        // Last CTA: merge the G partials (parallel loads, then a tree in shared memory).
                        __threadfence();
                        float rv = 0.f, pv = 0.f;
                        int ri = -1, pi = -1;
                        for (int c = tid; c < G; c += 256)
                        {
                            const float4 v = __ldcg(&a.lm_part[c]);
                            if (__float_as_int(v.y) >= 0) best_update(rv, ri, v.x, __float_as_int(v.y));
                            if (__float_as_int(v.w) >= 0) best_update(pv, pi, v.z, __float_as_int(v.w));
                        }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1)
                        {
                            const float orv = __shfl_xor_sync(0xffffffffu, rv, o);
                            const int ori = __shfl_xor_sync(0xffffffffu, ri, o);
                            const float opv = __shfl_xor_sync(0xffffffffu, pv, o);
                            const int opi = __shfl_xor_sync(0xffffffffu, pi, o);
                            if (ori >= 0) best_update(rv, ri, orv, ori);
                            if (opi >= 0) best_update(pv, pi, opv, opi);
                        }
                        if (lane == 0) red4[8 + warp] = make_float4(rv, __int_as_float(ri), pv, __int_as_float(pi));
                        consumers_sync();
                        if (tid == 0)
                        {
                            float frv = 0.f, fpv = 0.f;
                            int fri = -1, fpi = -1;
                            for (int w = 0; w < kMegaWarps; ++w)
                            {
                                const float4 v = red4[8 + w];
                                if (__float_as_int(v.y) >= 0) best_update(frv, fri, v.x, __float_as_int(v.y));
                                if (__float_as_int(v.w) >= 0) best_update(fpv, fpi, v.z, __float_as_int(v.w));
                            }
                            *a.lm_cnt = 0;
                            volatile DecodeState* st = a.st;
                            if (!mega_check(fpi >= 0 && fpi < a.vocab && fri >= 0 && fri < a.vocab, a.dbg, 4, b, phases - 1, fpi))
                            {
                                st->done = 1;
                            }
                            else if (!st->done)
                            {
                                const int n = st->n_gen;
                                if (n >= st->max_tokens) st->done = 1;
                                else
                                {
                                    a.log_tokens[n] = fpi;
                                    a.log_raw[n] = fri;
                                    st->n_gen = n + 1;
                                    st->cur_token = fpi;
                                    st->kv_len += 1;
                                    atomicOr(a.hist + (fpi >> 5), 1u << (fpi & 31));
                                    bool eos = false;
                                    for (int e = 0; e < st->n_eos && e < kMaxEos; ++e) eos |= (st->eos[e] == fpi);
                                    if (eos || n + 1 >= st->max_tokens) st->done = 1;
                                }
                            }
                            __threadfence();
                        }
                    }
                }
            }
            else if (b < kNumKVHeads * kMegaSplits)
            {
                // ---------------- attention ----------------
                const int g = p.g;
                const bool new_split = (p.split == kMegaSplits - 1);
                const float* qn_w = lnorm + 2048;
                const float* kn_w = lnorm + 2176;
                const float* c = a.rope_cos + static_cast<size_t>(past) * kHeadDim;
                const float* s = a.rope_sin + static_cast<size_t>(past) * kHeadDim;
                if (warp < 2)
                {
                    float o[4];
                    rope_norm_vec_cg(a.qkv + (2 * g + warp) * kHeadDim, c, s, qn_w, a.eps, lane, o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) qs[warp * kHeadDim + lane + 32 * i] = o[i] * a.scale_log2;
                }
                else if (new_split && warp == 2)
                {
                    float o[4];
                    rope_norm_vec_cg(a.qkv + kQWidth + g * kHeadDim, c, s, kn_w, a.eps, lane, o);
                    mega_check(past >= 0 && past < a.cap, a.dbg, 5, b, ph, past);
                    KT* krow = static_cast<KT*>(a.kc) +
                               ((static_cast<size_t>(layer) * kNumKVHeads + g) * a.cap + min(past, a.cap - 1)) * kHeadDim;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                    {
                        const KT q = from_f32<KT>(o[i]);
                        krow[lane + 32 * i] = q;
                        knew[lane + 32 * i] = to_f32<KT>(q);
                    }
                }
                else if (new_split && warp == 3)
                {
                    const float* vsrc = a.qkv + kQWidth + kKVWidth + g * kHeadDim;
                    KT* vrow = static_cast<KT*>(a.vc) +
                               ((static_cast<size_t>(layer) * kNumKVHeads + g) * a.cap + min(past, a.cap - 1)) * kHeadDim;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                    {
                        const KT q = from_f32<KT>(__ldcg(vsrc + lane + 32 * i));
                        vrow[lane + 32 * i] = q;
                        vnew[lane + 32 * i] = to_f32<KT>(q);
                    }
                }
                consumers_sync();

                // lane = (pg: 2, qq: 2, qr: 8); a lane owns dims 4*(qr + 8j) + e, j < 4.
                const int qr = lane & 7, qq = (lane >> 3) & 1, pg = lane >> 4;
                const int stream = warp * 2 + pg;  // 16 position streams
                float4 q4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) q4[j] = *reinterpret_cast<const float4*>(qs + qq * kHeadDim + 4 * (qr + 8 * j));
                float mx = -INFINITY, l = 0.f;
                float4 acc[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                auto visit = [&](const auto* krow, const auto* vrow, bool visible) {
                    float sc = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) sc += dot4(q4[j], load4(krow + 4 * (qr + 8 * j)));
                    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 2);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 4);
                    if (!visible) return;
                    const float mn = fmaxf(mx, sc);
                    const float corr = exp2f(mx - mn);
                    const float pe = exp2f(sc - mn);
                    l = l * corr + pe;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        const float4 vv = load4(vrow + 4 * (qr + 8 * j));
                        acc[j].x = acc[j].x * corr + pe * vv.x;
                        acc[j].y = acc[j].y * corr + pe * vv.y;
                        acc[j].z = acc[j].z * corr + pe * vv.z;
                        acc[j].w = acc[j].w * corr + pe * vv.w;
                    }
                    mx = mn;
                };
                const KT* ringk = reinterpret_cast<const KT*>(ring);
                for (int i = 0; i < p.nstage; ++i, ++gs)
                {
                    const int slot = gs % kMegaNst;
                    if (bad) continue;
                    const bool okw = mbar_wait(&full[slot], (gs / kMegaNst) & 1, a.err, kErrTimeoutFull);
                    if (!__all_sync(0xffffffffu, okw))
                    {
                        if (lane == 0) redi[0] = 1;
                        bad = true;
                        continue;
                    }
                    if (tracing)
                    {
                        if (i == 0) tr[6] = global_ns();
                        if (i == p.nstage - 1) tr[7] = global_ns();
                    }
                    const KT* kst = ringk + (static_cast<size_t>(slot) * kMegaStage) / sizeof(KT);
                    const KT* vst = kst + static_cast<size_t>(p.per_stage) * kHeadDim;
                    const int n = min(p.per_stage, p.count - i * p.per_stage);
                    for (int jb = 0; jb < n; jb += 16)
                    {
                        const int j = jb + stream;
                        const int jj = (j < n) ? j : 0;
                        visit(kst + static_cast<size_t>(jj) * kHeadDim, vst + static_cast<size_t>(jj) * kHeadDim, j < n);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                }
                if (new_split && warp == 0) visit(knew, vnew, pg == 0);
                // Merge the two position groups of the warp (lanes l and l^16).
                {
                    const float m2 = __shfl_xor_sync(0xffffffffu, mx, 16);
                    const float l2 = __shfl_xor_sync(0xffffffffu, l, 16);
                    const float M = fmaxf(mx, m2);
                    const float f1 = (mx == -INFINITY) ? 0.f : exp2f(mx - M);
                    const float f2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - M);
                    l = l * f1 + l2 * f2;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                    {
                        float4 o2;
                        o2.x = __shfl_xor_sync(0xffffffffu, acc[j].x, 16);
                        o2.y = __shfl_xor_sync(0xffffffffu, acc[j].y, 16);
                        o2.z = __shfl_xor_sync(0xffffffffu, acc[j].z, 16);
                        o2.w = __shfl_xor_sync(0xffffffffu, acc[j].w, 16);
                        acc[j].x = acc[j].x * f1 + o2.x * f2;
                        acc[j].y = acc[j].y * f1 + o2.y * f2;
                        acc[j].z = acc[j].z * f1 + o2.z * f2;
                        acc[j].w = acc[j].w * f1 + o2.w * f2;
                    }
                    mx = M;
                }
                if (pg == 0)
                {
                    float* w = ascr + (warp * 2 + qq) * kPartStride;
                    if (qr == 0)
                    {
                        w[0] = mx;
                        w[1] = l;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) *reinterpret_cast<float4*>(w + 4 + 4 * (qr + 8 * j)) = acc[j];
                }
                consumers_sync();
                // CTA partial per query (256 threads = 2 queries x 128 dims).
                {
                    const int q = tid >> 7, d = tid & 127;
                    float M = -INFINITY;
#pragma unroll
                    for (int w = 0; w < kMegaWarps; ++w) M = fmaxf(M, ascr[(w * 2 + q) * kPartStride]);
                    float Lsum = 0.f, A = 0.f;
                    if (M != -INFINITY)
                    {
#pragma unroll
                        for (int w = 0; w < kMegaWarps; ++w)
                        {
                            const float* sw = ascr + (w * 2 + q) * kPartStride;
                            if (sw[0] == -INFINITY) continue;
                            const float f = exp2f(sw[0] - M);
                            Lsum += f * sw[1];
                            A += f * sw[4 + d];
                        }
                    }
                    float* part = a.attn_part + ((static_cast<size_t>(g) * kMegaSplits + p.split) * 2 + q) * kPartStride;
                    if (d == 0)
                    {
                        part[0] = M;
                        part[1] = Lsum;
                    }
                    part[4 + d] = A;
                }
                // The o-projection phase merges the partials of all splits.
            }

            // ---------------- phase done: arrive on the grid barrier ----------------
            consumers_sync();
            if (redi[0]) return;
            if (tracing) tr[3] = global_ns();
            if (tid == 0)
            {
                grid_arrive(a.bar);
                if (a.progress) a.progress[b] = phase_no + 1;
            }
        }
    }
}

}  // namespace hy
