// GQA decode attention (one row) over the KV cache, split over the key axis
// (flash-decode), with the per-head RoPE, QK RMSNorm and KV append fused into
// the prologue; used by the per-phase AR path and the standalone attention
// entry point (steps of 2..16 rows: hy_prefill.cuh).
//
// Replaces, for the decode step:
//   - MultimodalRotaryEmbed (src/multimodal_rope.cpp:176-187): full-width
//     cos/sin, out[d] = x[d]c[d] - x[d+64]s[d], out[d+64] = x[d+64]c[d+64] + x[d]s[d+64];
//   - query_layernorm / key_layernorm applied after RoPE (export/text_decoder_kv.py:70-73);
//   - append_or_grow_kv_cache (src/kv_cache_capacity.cpp:232-280): rows are
//     written in place into a cache reserved up front;
//   - PreciseSDPA::forward (src/precise_sdpa.cpp:281-329): softmax(q k^T * scale + mask) v,
//     here with fp32 accumulation and an online (max-rescaled) softmax. The
//     mask is the one the reference builds: zeros for decode
//     (src/text_runtime.cpp:221-226) and causal inside a verify block
//     (src/dflash_runtime.cpp:60-76), i.e. row m sees keys <= past + m.
//
// The cache keeps the 8 unique KV heads, [8][capacity][128] per layer; q head
// h reads KV head h / 2, which is what the reference's repeat_kv expansion to
// 16 heads amounts to (export/text_decoder_kv.py:21-27).
//
// Grid (S, 8): split s < S-1 streams keys [s*chunk, ...) of the past rows
// through a shared-memory ring with cp.async.bulk; split S-1 computes the new
// rows (RoPE + norm), appends them and attends to them. Each CTA leaves a
// partial (max, sum, acc[128]) per query; the last CTA of a head (atomic
// ticket) merges the S partials into the output.
//
// Lane layout inside a warp: lane = (pg, qq, qr); qr = dim quarter (lowest two
// bits), qq = query, pg = position subgroup. A lane owns the 32 dims
// d = 4*(qr + 4j) + e (j < 8, e < 4), so the four quarters of a warp read
// distinct bank groups of a K/V row and a score needs only two shuffles.
#pragma once

#include "hy_device.cuh"

namespace hy {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = (kAttnWarps + 1) * 32;
constexpr int kAttnPos = 32;      // key positions per ring stage
constexpr int kAttnStages = 3;
constexpr int kPartStride = 132;  // (max, sum, -, -) + acc[128]

struct AttnArgs {
    const float* qkv;   // [rows x ldq]: q [0, 2048), k [2048, 3072), v [3072, 4096)
    int ldq;
    const float* qn_w;
    const float* kn_w;
    const float* cos;   // rope row = (rope_state ? kv_len : 0) + m, [.. x 128]
    const float* sin;
    int rope_state;
    void* kc;           // this layer's K cache [8][cap][128] of KT
    void* vc;
    int cap;
    const DecodeState* st;  // past = st->kv_len when st, else past_fixed
    int past_fixed;
    int rows;
    float scale_log2;   // attention scale * log2(e)
    float eps;
    float* part;        // [8][S][2*MT][kPartStride]
    int* counter;       // [8]
    float* out;         // [rows x 2048]
    int* err;
    // Batched decode (one row per sequence, grid z = row): row z attends to its own
    // slot's cache (kc / vc + z * slot_stride elements) at its own length; rows of
    // inactive slots do nothing. part / counter / out / qkv are offset by row.
    const SlotState* slots;
    size_t slot_stride;
};

template <int MT, typename KT>
struct AttnShape {
    static constexpr int NQ = 2 * MT;                              // queries per KV head
    static constexpr int ROWB = kHeadDim * static_cast<int>(sizeof(KT));
    static constexpr int STAGE = 2 * kAttnPos * ROWB;               // K block then V block
    static constexpr int QS_OFF = 0;                                // [NQ][128] f32
    static constexpr int NEW_OFF = QS_OFF + NQ * kHeadDim * 4;      // K new [MT][128], V new [MT][128] f32
    static constexpr int RING_OFF = NEW_OFF + 2 * MT * kHeadDim * 4;
    static constexpr int NSTREAM = (MT == 1) ? 32 : 4;
    // Per-stream softmax states reuse the ring once every stage has been consumed.
    static constexpr int SCR_OFF = RING_OFF;   // [NSTREAM][NQ] (m, l), [NSTREAM][NQ][128] acc
    static constexpr int SCR_BYTES = NSTREAM * NQ * 8 + NSTREAM * NQ * kHeadDim * 4;
    static constexpr int RING_REGION = (SCR_BYTES > kAttnStages * STAGE) ? SCR_BYTES : kAttnStages * STAGE;
    static constexpr int BAR_OFF = RING_OFF + RING_REGION;
    static constexpr int SMEM = BAR_OFF + 2 * kAttnStages * 8 + 16;
};

__device__ __forceinline__ void attn_consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// RoPE (full-width, non-interleaved) + RMSNorm of one 128-vector by one warp.
// Lane l owns dims l, l+32, l+64, l+96.
__device__ __forceinline__ void rope_norm_vec(const float* x, const float* c, const float* s, const float* w, float eps,
                                              int lane, float out[4])
{
    const float x0 = x[lane], x1 = x[lane + 32], x2 = x[lane + 64], x3 = x[lane + 96];
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

// RMSNorm, then RoPE, of one 128-vector by one warp: the DFlash draft's order
// (q_norm / k_norm before apply_external_rope, export/dflash_export.py:104-128).
__device__ __forceinline__ void norm_rope_vec(const float* x, const float* c, const float* s, const float* w, float eps,
                                              int lane, float out[4])
{
    const float x0 = x[lane], x1 = x[lane + 32], x2 = x[lane + 64], x3 = x[lane + 96];
    const float ss = warp_sum(x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3);
    const float ri = 1.0f / sqrtf(ss / static_cast<float>(kHeadDim) + eps);
    const float n0 = w[lane] * (x0 * ri), n1 = w[lane + 32] * (x1 * ri);
    const float n2 = w[lane + 64] * (x2 * ri), n3 = w[lane + 96] * (x3 * ri);
    out[0] = n0 * c[lane] - n2 * s[lane];
    out[1] = n1 * c[lane + 32] - n3 * s[lane + 32];
    out[2] = n2 * c[lane + 64] + n0 * s[lane + 64];
    out[3] = n3 * c[lane + 96] + n1 * s[lane + 96];
}

template <int MT, typename KT>
__global__ void __launch_bounds__(kAttnThreads, (MT == 1) ? 2 : 1) attn_kernel(const AttnArgs a)
{
    // Steps of 2..16 rows use the tensor-core kernels of hy_prefill.cuh (RoPE /
    // append kernel, key chunks, chunk merge).
    static_assert(MT == 1, "one-row decode attention");
    using S = AttnShape<MT, KT>;
    constexpr int NQ = S::NQ, NSTREAM = S::NSTREAM, ROWB = S::ROWB, STAGE = S::STAGE;
    extern __shared__ __align__(128) unsigned char smem[];
    float* qs = reinterpret_cast<float*>(smem + S::QS_OFF);
    float* knew = reinterpret_cast<float*>(smem + S::NEW_OFF);
    float* vnew = knew + MT * kHeadDim;
    unsigned char* ring = smem + S::RING_OFF;
    float* scr_ml = reinterpret_cast<float*>(smem + S::SCR_OFF);       // [NSTREAM][NQ][2]
    float* scr_acc = scr_ml + NSTREAM * NQ * 2;                        // [NSTREAM][NQ][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
    uint64_t* empty = full + kAttnStages;
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nsplit = gridDim.x, split = blockIdx.x, g = blockIdx.y, bz = blockIdx.z;
    HY_STEP_TRACE_OPEN(0x500000000ull | MT);
    const bool new_split = (split == nsplit - 1);
    // Rows [0, past) were written by earlier steps, so they (and past itself)
    // may be read before griddepcontrol.wait (the slot states too: the commit
    // that wrote them ran at least two kernels earlier).
    if (a.slots && !a.slots[bz].active)
    {
        pdl_wait();   // (every CTA waits, so the grid never ends before its predecessor)
        return;
    }
    const int past = a.slots ? a.slots[bz].kv_len : a.st ? a.st->kv_len : a.past_fixed;
    const int rows = a.rows;
    const size_t slot_off = a.slots ? static_cast<size_t>(bz) * a.slot_stride : 0;
    const float* qkv_base = a.qkv + static_cast<size_t>(bz) * a.ldq;
    float* out_base = a.out + static_cast<size_t>(bz) * kQWidth;
    int* counter = a.counter + bz * kNumKVHeads;
    int p0 = 0, p1 = 0;
    if (!new_split)
    {
        const int chunk = (past + nsplit - 2) / (nsplit - 1);
        p0 = min(past, split * chunk);
        p1 = min(past, p0 + chunk);
    }
    const int npos = p1 - p0;
    const int nstage = (npos + kAttnPos - 1) / kAttnPos;

    if (tid == 0)
    {
        for (int s = 0; s < kAttnStages; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAttnWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    const KT* kbase = static_cast<const KT*>(a.kc) + slot_off + static_cast<size_t>(g) * a.cap * kHeadDim;
    const KT* vbase = static_cast<const KT*>(a.vc) + slot_off + static_cast<size_t>(g) * a.cap * kHeadDim;

    if (warp == kAttnWarps)
    {
        // ---------------- producer: stream K/V rows [p0, p1) ----------------
        if (lane == 0 && nstage > 0)
        {
            const uint64_t pol = l2_evict_first_policy();
            int issued = 0;
            for (int i = 0; i < nstage; ++i)
            {
                const int slot = i % kAttnStages;
                if (i >= kAttnStages &&
                    !mbar_wait(&empty[slot], ((i / kAttnStages) - 1) & 1, a.err, kErrTimeoutEmpty))
                    break;
                const int q0 = p0 + i * kAttnPos;
                const int n = min(kAttnPos, p1 - q0);
                const uint32_t bytes = static_cast<uint32_t>(n * ROWB);
                mbar_arrive_expect_tx(&full[slot], 2 * bytes);
                unsigned char* dst = ring + slot * STAGE;
                bulk_g2s(dst, kbase + static_cast<size_t>(q0) * kHeadDim, bytes, &full[slot], pol);
                bulk_g2s(dst + kAttnPos * ROWB, vbase + static_cast<size_t>(q0) * kHeadDim, bytes, &full[slot], pol);
                issued = i + 1;
            }
            for (int i = (issued > kAttnStages ? issued - kAttnStages : 0); i < issued; ++i)
                mbar_wait(&full[i % kAttnStages], (i / kAttnStages) & 1, a.err, kErrTimeoutFull);
        }
        return;
    }

    // ---------------- consumers ----------------
    // Prologue: rotate + normalise the 2*MT queries (and, in the new-row split,
    // the MT keys; values are copied), append the new rows to the cache.
    const int nvec = new_split ? (NQ + 2 * MT) : NQ;
    // A warp's vectors are v = warp + 8 jv. The constants (RoPE cos / sin rows of
    // the rows' positions, known before the wait, and the QK-norm weights) are
    // loaded before griddepcontrol.wait; the rows themselves, written by the
    // previous kernel, after it, all in one L2 round trip.
    constexpr int kMaxVec = (4 * MT + kAttnWarps - 1) / kAttnWarps;
    float xv[kMaxVec][4], cv[kMaxVec][4], sv[kMaxVec][4], nv[kMaxVec][4];
#pragma unroll
    for (int jv = 0; jv < kMaxVec; ++jv)
    {
        const int v = warp + kAttnWarps * jv;
        int m, kind;
        if (v < NQ) { kind = 0; m = v % MT; }
        else if (v < NQ + MT) { kind = 1; m = v - NQ; }
        else { kind = 2; m = v - NQ - MT; }
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[jv][i] = cv[jv][i] = sv[jv][i] = nv[jv][i] = 0.f;
        if (v >= nvec || m >= rows || kind == 2) continue;
        const int prow = (a.rope_state ? past : 0) + m;
        const float* c = a.cos + static_cast<size_t>(prow) * kHeadDim;
        const float* sn = a.sin + static_cast<size_t>(prow) * kHeadDim;
        const float* nw = (kind == 0) ? a.qn_w : a.kn_w;
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            cv[jv][i] = __ldg(c + lane + 32 * i);
            sv[jv][i] = __ldg(sn + lane + 32 * i);
            nv[jv][i] = __ldg(nw + lane + 32 * i);
        }
    }
    pdl_wait();
    HY_STEP_TRACE_MARK(2);
    pdl_launch();
#pragma unroll
    for (int jv = 0; jv < kMaxVec; ++jv)
    {
        const int v = warp + kAttnWarps * jv;
        int m, kind, head;
        if (v < NQ) { kind = 0; head = v / MT; m = v % MT; }
        else if (v < NQ + MT) { kind = 1; head = 0; m = v - NQ; }
        else { kind = 2; head = 0; m = v - NQ - MT; }
        if (v >= nvec || m >= rows) continue;
        const float* src = qkv_base + static_cast<size_t>(m) * a.ldq +
                           ((kind == 0) ? (2 * g + head) * kHeadDim : (kind == 1) ? kQWidth + g * kHeadDim
                                                                                  : kQWidth + kKVWidth + g * kHeadDim);
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[jv][i] = src[lane + 32 * i];
    }
#pragma unroll
    for (int jv = 0; jv < kMaxVec; ++jv)
    {
        const int v = warp + kAttnWarps * jv;
        if (v >= nvec) break;
        int m, kind, head;
        if (v < NQ) { kind = 0; head = v / MT; m = v % MT; }
        else if (v < NQ + MT) { kind = 1; head = 0; m = v - NQ; }
        else { kind = 2; head = 0; m = v - NQ - MT; }
        (void)head;
        float* dst = (kind == 0) ? (qs + v * kHeadDim) : (kind == 1 ? knew + m * kHeadDim : vnew + m * kHeadDim);
        if (m >= rows)
        {
            for (int d = lane; d < kHeadDim; d += 32) dst[d] = 0.f;
            continue;
        }
        if (kind == 2)
        {
            KT* vrow = const_cast<KT*>(vbase) + static_cast<size_t>(past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                const KT q = from_f32<KT>(xv[jv][i]);
                vrow[lane + 32 * i] = q;
                dst[lane + 32 * i] = to_f32<KT>(q);
            }
            continue;
        }
        // RoPE (full-width, non-interleaved) + RMSNorm, lane l owning dims l + 32 i.
        const float y0 = xv[jv][0] * cv[jv][0] - xv[jv][2] * sv[jv][0];
        const float y1 = xv[jv][1] * cv[jv][1] - xv[jv][3] * sv[jv][1];
        const float y2 = xv[jv][2] * cv[jv][2] + xv[jv][0] * sv[jv][2];
        const float y3 = xv[jv][3] * cv[jv][3] + xv[jv][1] * sv[jv][3];
        const float ss = warp_sum(y0 * y0 + y1 * y1 + y2 * y2 + y3 * y3);
        const float ri = 1.0f / sqrtf(ss / static_cast<float>(kHeadDim) + a.eps);
        float o[4];
        o[0] = nv[jv][0] * (y0 * ri);
        o[1] = nv[jv][1] * (y1 * ri);
        o[2] = nv[jv][2] * (y2 * ri);
        o[3] = nv[jv][3] * (y3 * ri);
        if (kind == 0)
        {
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = o[i] * a.scale_log2;
        }
        else
        {
            KT* krow = const_cast<KT*>(kbase) + static_cast<size_t>(past + m) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 4; ++i)
            {
                const KT q = from_f32<KT>(o[i]);
                krow[lane + 32 * i] = q;
                dst[lane + 32 * i] = to_f32<KT>(q);
            }
        }
    }
    attn_consumers_sync();
    HY_STEP_TRACE_MARK(3);

    {
        // Lane roles.
        const int qr = lane & 3;
        int qi, stream;
        if (MT == 1)
        {
            qi = (lane >> 2) & 1;
            stream = warp * 4 + (lane >> 3);
        }
        else
        {
            qi = (warp & 3) * 8 + (lane >> 2);
            stream = warp >> 2;
        }
        const int qm = qi % MT;   // query row of this lane's query
        float4 q4[8];
    #pragma unroll
        for (int j = 0; j < 8; ++j) q4[j] = *reinterpret_cast<const float4*>(qs + qi * kHeadDim + 4 * (qr + 4 * j));
        float mx = -INFINITY, l = 0.f;
        float4 acc[8];
    #pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);

        // One key position for this lane's query; every lane of the warp calls it
        // the same number of times (the shuffles use the full mask).
        auto visit = [&](const auto* krow, const auto* vrow, bool visible) {
            float sc = 0.f;
    #pragma unroll
            for (int j = 0; j < 8; ++j) sc += dot4(q4[j], load4(krow + 4 * (qr + 4 * j)));
            sc += __shfl_xor_sync(0xffffffffu, sc, 1);
            sc += __shfl_xor_sync(0xffffffffu, sc, 2);
            if (!visible) return;
            const float mn = fmaxf(mx, sc);
            const float corr = exp2f(mx - mn);
            const float pe = exp2f(sc - mn);
            l = l * corr + pe;
    #pragma unroll
            for (int j = 0; j < 8; ++j)
            {
                const float4 vv = load4(vrow + 4 * (qr + 4 * j));
                acc[j].x = acc[j].x * corr + pe * vv.x;
                acc[j].y = acc[j].y * corr + pe * vv.y;
                acc[j].z = acc[j].z * corr + pe * vv.z;
                acc[j].w = acc[j].w * corr + pe * vv.w;
            }
            mx = mn;
        };

        // Past rows from the ring.
        for (int i = 0; i < nstage; ++i)
        {
            const int slot = i % kAttnStages;
            const bool ok = mbar_wait(&full[slot], (i / kAttnStages) & 1, a.err, kErrTimeoutFull);
            if (!__all_sync(0xffffffffu, ok)) break;
            const KT* kst = reinterpret_cast<const KT*>(ring + slot * STAGE);
            const KT* vst = reinterpret_cast<const KT*>(ring + slot * STAGE + kAttnPos * ROWB);
            const int n = min(kAttnPos, npos - i * kAttnPos);
            for (int jb = 0; jb < n; jb += NSTREAM)
            {
                const int j = jb + stream;
                const int jj = (j < n) ? j : 0;
                visit(kst + jj * kHeadDim, vst + jj * kHeadDim, j < n);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        // New rows (causal inside the block: row m sees new row j iff j <= m).
        if (new_split)
        {
            for (int jb = 0; jb < rows; jb += NSTREAM)
            {
                const int j = jb + stream;
                const int jj = (j < rows) ? j : 0;
                visit(knew + jj * kHeadDim, vnew + jj * kHeadDim, j < rows && j <= qm);
            }
        }

        // Per-stream states to shared memory (aliasing the drained ring).
        attn_consumers_sync();
        if (qr == 0)
        {
            scr_ml[(stream * NQ + qi) * 2 + 0] = mx;
            scr_ml[(stream * NQ + qi) * 2 + 1] = l;
        }
    #pragma unroll
        for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(scr_acc + (stream * NQ + qi) * kHeadDim + 4 * (qr + 4 * j)) = acc[j];
        attn_consumers_sync();
    }

    // CTA partial per query.
    float* const part_base = a.part + static_cast<size_t>(bz) * kNumKVHeads * nsplit * NQ * kPartStride;
    float* part = part_base + (static_cast<size_t>(g) * nsplit + split) * NQ * kPartStride;
    for (int e = tid; e < NQ * kHeadDim; e += 256)
    {
        const int q = e / kHeadDim, d = e % kHeadDim;
        float M = -INFINITY;
        for (int s = 0; s < NSTREAM; ++s) M = fmaxf(M, scr_ml[(s * NQ + q) * 2]);
        float L = 0.f, A = 0.f;
        if (M != -INFINITY)
        {
            for (int s = 0; s < NSTREAM; ++s)
            {
                const float ms = scr_ml[(s * NQ + q) * 2];
                if (ms == -INFINITY) continue;
                const float f = exp2f(ms - M);
                L += f * scr_ml[(s * NQ + q) * 2 + 1];
                A += f * scr_acc[(s * NQ + q) * kHeadDim + d];
            }
        }
        if (d == 0)
        {
            part[q * kPartStride + 0] = M;
            part[q * kPartStride + 1] = L;
        }
        part[q * kPartStride + 4 + d] = A;
    }
    __threadfence();
    attn_consumers_sync();
    if (tid == 0) s_last = (atomicAdd(&counter[g], 1) == nsplit - 1) ? 1 : 0;
    attn_consumers_sync();
    HY_STEP_TRACE_MARK(4);
    if (!s_last)
    {
        HY_STEP_TRACE_EXIT();
        return;
    }
    __threadfence();

    // Last CTA of this head: merge the S partials. First the (max, sum) of
    // every split and query, the merged max / sum and each split's weight (in
    // the drained ring), then the accumulators, every split's float4 of an
    // output in flight at once.
    const float* hp = part_base + static_cast<size_t>(g) * nsplit * NQ * kPartStride;
    float* mw = reinterpret_cast<float*>(ring);   // [nsplit][NQ] split max -> weight
    float* ls = mw + nsplit * NQ;                 // [nsplit][NQ] split sum
    float* inv_l = ls + nsplit * NQ;              // [NQ] 1 / merged sum
    for (int e = tid; e < nsplit * NQ; e += 256)
    {
        mw[e] = __ldcg(hp + e * kPartStride);
        ls[e] = __ldcg(hp + e * kPartStride + 1);
    }
    attn_consumers_sync();
    for (int q = tid; q < NQ; q += 256)
    {
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, mw[sp * NQ + q]);
        float L = 0.f;
        for (int sp = 0; sp < nsplit; ++sp)
        {
            const float ms = mw[sp * NQ + q];
            const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
            mw[sp * NQ + q] = f;
            L += f * ls[sp * NQ + q];
        }
        inv_l[q] = 1.0f / L;
    }
    attn_consumers_sync();
    constexpr int kMaxS = 20;
    for (int e = tid; e < NQ * (kHeadDim / 4); e += 256)
    {
        const int q = e / (kHeadDim / 4), d4 = e % (kHeadDim / 4);
        const int m = q % MT, head = q / MT;
        if (m >= rows) continue;
        float4 v[kMaxS];
#pragma unroll
        for (int sp = 0; sp < kMaxS; ++sp)
            if (sp < nsplit) v[sp] = __ldcg(reinterpret_cast<const float4*>(hp + (sp * NQ + q) * kPartStride + 4) + d4);
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < kMaxS; ++sp)
        {
            if (sp >= nsplit) break;
            const float f = mw[sp * NQ + q];
            A.x += f * v[sp].x; A.y += f * v[sp].y; A.z += f * v[sp].z; A.w += f * v[sp].w;
        }
        const float il = inv_l[q];
        A.x *= il; A.y *= il; A.z *= il; A.w *= il;
        *reinterpret_cast<float4*>(out_base + static_cast<size_t>(m) * kQWidth + (2 * g + head) * kHeadDim + 4 * d4) = A;
    }
    if (tid == 0) counter[g] = 0;
    HY_STEP_TRACE_EXIT();
}

}  // namespace hy
