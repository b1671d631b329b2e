// Persistent AR decode kernel: whole tokens (embed -> 24 layers -> LM head ->
// penalised argmax -> commit) in one cooperative launch, one CTA per SM.
//
// The decode step of the reference (decode_from_embeddings' loop,
// src/text_runtime.cpp:1417-1508, executing the graph of
// export/text_decoder_kv.py:49-96 plus the LM head and select_next_token) is
// a chain of 121 dependent phases per token: for each layer q/k/v projection,
// attention, o projection, gate/up projection, down projection; then the LM
// head. Every phase is split across the CTAs (rows of the weight matrix, or a
// range of cached positions for attention), and each CTA's share is cut into
// stages of at most 16 KB.
//
// Streaming: the CTA's stage sequence (over all phases and tokens of the
// launch) is dealt round-robin to its 7 consumer warps (stage g to warp g % 7)
// and into a ring of 12 shared-memory slots of 16 KB (stage g to slot g % 12).
// A producer warp streams the stages with cp.async.bulk (no multicast) across
// phase boundaries - no weight byte depends on an activation - keeping at most
// 2 stages in flight (6 in the LM head): more copies in flight delay the
// latency-critical exchange loads below. A consumer warp waits for its stage's
// slot to have been released by the slot's previous stage, then for the stage
// itself, so every mbarrier parity wait is at most one phase ahead. A stage's
// rows are reduced in one pass: the activation vector sits in registers (K =
// 1024) or shared memory, and a transposing butterfly leaves each row's sum in
// its own group of lanes, which run the epilogue in parallel.
//
// Exchange between CTAs, with no grid barrier: every activation a phase
// produces (q/k/v rows, the residual stream, SwiGLU outputs, attention split
// partials and merged head outputs) is one 64-bit word, float bits | phase epoch
// << 32, written with one relaxed store; the next phase polls the words it needs
// until they carry its epoch, then stages them in shared memory (fused RMSNorm,
// whose per-row scale is applied to the dot products; SwiGLU; embedding
// gather). The residual rows a CTA owns stay in its shared memory. Attention
// splits each KV head's cached positions over 17 CTAs plus one CTA for the new
// row (RoPE + QK-norm + KV append); the new-row CTA of each head pair merges
// the pair's split partials and publishes the merged head outputs for the o
// projection. The LM head's last CTA (atomic ticket) merges the per-CTA argmax
// partials, commits the token and publishes it with a release store; every CTA
// acquires it, which also orders the previous token's KV rows and state.
//
// All waits are bounded by wall clock (the launch's wait limit): a wait that
// gives up sets the error word, the consumers leave together at the end of the
// phase, and the producer drains its in-flight copies first.
#pragma once

#include "hy_attn.cuh"
#include "hy_device.cuh"
#include "hy_gemv.cuh"

namespace hy {

// Back-off (ns) between polling rounds of the epoch words. The exchanges are
// latency-bound, not contended: at config 0 a 1 ns back-off gave 1638 tokens/s,
// 32 ns 1610, 100 ns 1599, 250 ns 1579, 600 ns 1466 (device loop, KV 1024-1279).
#ifndef HY_POLL_NS
#define HY_POLL_NS 1
#endif

// Consumer warps. A CTA's share of the q/k/v, o and down phases is 4-7 stages
// (28 rows of 4 KB at 4 rows per stage; 7 rows of 8 KB at 2; 7 rows of 14 KB at
// 1): 7 warps take each of them in one round, 6 needed two.
#ifndef HY_MEGA_WARPS
#define HY_MEGA_WARPS 7
#endif
constexpr int kMegaWarps = HY_MEGA_WARPS;
constexpr int kMegaConsumers = kMegaWarps * 32;
constexpr int kMegaThreads = kMegaConsumers + 32;      // + the producer warp
constexpr int kMegaStage = 16384;        // bytes per slot
// Ring slots, shared by the consumer warps: global stage g lands in slot
// g % kMegaSlots (its use g / kMegaSlots) and is consumed by warp g % kMegaWarps.
constexpr int kMegaSlots = 12;
// Stages the producer keeps in flight (issued, not landed). More than the
// bandwidth-delay product only queues in the memory fabric, where the epoch-word
// polls of the exchanges wait behind it: with all 12 slots in flight a batch of
// polls took 1-2.5 us although the words were already published. Measured at the
// AR decode workload (tokens/s, device loop): 12 in flight 1674, 8 1694, 6 1712,
// 4 1806, 3 1879, 2 1917, 1 1402; with 2 for the layers, the LM head at 4 / 6 / 8:
// 1953 / 1955 / 1947.
#ifndef HY_MEGA_INFLIGHT
#define HY_MEGA_INFLIGHT 2
#endif
constexpr int kMegaInflight = HY_MEGA_INFLIGHT;
// The LM head streams the tied table with no exchange to wait for: it keeps more in flight.
#ifndef HY_MEGA_INFLIGHT_LM
#define HY_MEGA_INFLIGHT_LM 6
#endif
constexpr int kMegaInflightLm = HY_MEGA_INFLIGHT_LM;
// Attention streams cached K/V rows, which no exchange of the token waits for.
#ifndef HY_MEGA_INFLIGHT_ATTN
#define HY_MEGA_INFLIGHT_ATTN 2
#endif
constexpr int kMegaInflightAttn = HY_MEGA_INFLIGHT_ATTN;
static_assert(kMegaInflightAttn >= 1 && kMegaInflightAttn <= kMegaSlots, "in-flight stages must fit the ring");
static_assert(kMegaInflight >= 1 && kMegaInflight <= kMegaSlots, "in-flight stages must fit the ring");
static_assert(kMegaInflightLm >= 1 && kMegaInflightLm <= kMegaSlots, "in-flight stages must fit the ring");
#ifndef HY_MEGA_SPLITS
#define HY_MEGA_SPLITS 18
#endif
constexpr int kMegaSplits = HY_MEGA_SPLITS;   // per KV head: the past rows' splits + the new-row split (8 x 18 = 144 CTAs)
constexpr int kMegaMaxK = 3584;
constexpr int kMegaHistWords = 64;       // LM rows per CTA <= 32 * 62
constexpr int kMegaResRows = 32;         // o/down rows per CTA (1024 / gridDim.x)
constexpr int kMegaMaxLayers = 64;
constexpr unsigned kMegaEpochSpan = 32768;   // epochs per launch (>= 64 tokens x 321 phases)
constexpr int kAttnWords = 2 + 128;          // one split partial of one query: max, sum, acc[128]

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
    float* attn;              // unused here
    float* gu;                // act = silu(gate) * up, [ffn]
    float* attn_part;         // [8][kMegaSplits][2][kPartStride]
    int* attn_cnt;            // unused here
    float4* lm_part;          // [gridDim.x]
    int* lm_cnt;
    unsigned* hist;
    DecodeState* st;
    int* log_tokens;
    int* log_raw;
    int num_layers, vocab, ffn;
    float eps, scale_log2;
    int steps;                // tokens in this launch
    int* err;
    // Optional phase trace: for CTAs b < kTraceCtas and token trace_token,
    // trace[(b * phases + ph) * kTraceSlots + i] (thread 0; see hy_trace_persistent).
    unsigned long long* trace;
    int trace_token;
    // Self-checks: the first failed bounds check stores (code, cta, phase, index)
    // in dbg[0..3] and the access is skipped. progress (host-mapped, nullable):
    // thread 0 of each CTA stores the number of phases it completed.
    int* dbg;
    volatile unsigned* progress;
    // Activations passed between CTAs as 64-bit words: float bits | epoch << 32,
    // written and read with single-copy-atomic 64-bit accesses, so a reader that
    // sees the phase's epoch sees that phase's value (no barrier, no fence).
    // Epoch of phase ph of token t: epoch_base + t * phases + ph + 1.
    unsigned long long* x_ep;    // residual stream [1024] (o / down outputs)
    unsigned long long* qkv_ep;  // q/k/v projections [4096]
    unsigned long long* act_ep;  // silu(gate) * up [ffn]
    unsigned long long* tok_ep;  // committed token (int bits) [1], written with release
    unsigned long long* attn_ep;      // split partials [8 heads][8 past splits][2][kAttnWords]
    unsigned long long* attn_out_ep;  // merged attention output [2048]
    unsigned epoch_base;
    // Wait statistics (only in builds with HY_WAIT_STATS defined; nullptr otherwise):
    // per CTA and wait kind the waits longer than kWsLongNs (count, total ns, longest),
    // and per launch slot the first CTA start and last CTA exit (%globaltimer).
    unsigned long long* wstat;
    int launch_slot;
    unsigned long long wait_limit_ns;   // bound of every wait in the kernel (default 2 s)
};

// Kinds of wait counted by the HY_WAIT_STATS build.
enum {
    WS_SLOT_FREE = 0,   // consumer: the slot's previous stage released
    WS_SLOT_FULL,       // consumer: the stage's bytes landed
    WS_PROD_EMPTY,      // producer: the slot released for refill
    WS_PROD_TOKEN,      // producer: the consumers acquired the previous token
    WS_POLL_X,          // residual stream (q/k/v, gate/up and LM prologues)
    WS_POLL_ACT,        // SwiGLU outputs (down_proj prologue)
    WS_POLL_ATTN_OUT,   // merged attention outputs (o_proj prologue)
    WS_POLL_QKV,        // q/k/v rows (attention prologue)
    WS_POLL_PARTS,      // split partials (attention merge)
    WS_POLL_TOKEN,      // the previous token's commit
    WS_KINDS
};
constexpr int kWsCtas = 160;
constexpr int kWsLaunches = 64;
constexpr unsigned long long kWsLongNs = 20000;
// Layout of the statistics buffer (unsigned long long words).
constexpr int kWsLaunchBase = kWsCtas * WS_KINDS * 3;            // [kWsLaunches][2]: ~first start, last end
constexpr int kWsWords = kWsLaunchBase + kWsLaunches * 2;

__device__ __forceinline__ void ws_record(unsigned long long* ws, int b, int kind, unsigned long long ns)
{
#ifdef HY_WAIT_STATS
    if (ws && b < kWsCtas && ns > kWsLongNs)
    {
        unsigned long long* r = ws + (static_cast<size_t>(b) * WS_KINDS + kind) * 3;
        atomicAdd(r, 1ull);
        atomicAdd(r + 1, ns);
        atomicMax(r + 2, ns);
    }
#endif
}

#ifndef HY_TRACE_CTAS
#define HY_TRACE_CTAS 4
#endif
constexpr int kTraceCtas = HY_TRACE_CTAS;   // CTAs 0 .. kTraceCtas - 1 are traced
constexpr int kTraceSlots = 12;

struct MegaSmem {
    static constexpr int RING = 0;                                          // [slot] x 16 KB
    static constexpr int XS = RING + kMegaSlots * kMegaStage;               // [3584] f32 activation vector
    // Attention phases do not use the activation vector; their buffers alias it.
    static constexpr int QS = XS;                                           // [2][128]
    static constexpr int NEWKV = QS + 2 * kHeadDim * 4;                     // k[128], v[128]
    static constexpr int ASCR = NEWKV + 2 * kHeadDim * 4;                   // [warps][2][kPartStride]
    static constexpr int PBUF = ASCR + kMegaWarps * 2 * kPartStride * 4;    // [warps][32] softmax weights
    static constexpr int MINE = PBUF + kMegaWarps * 32 * 4;                 // [2][kPartStride] this CTA's partial
    static constexpr int PARTS = MINE + 2 * kPartStride * 4;                // [8 splits][2][130] polled partials
    static constexpr int XS_END = PARTS + (kMegaSplits - 1) * 2 * kAttnWords * 4;
    static constexpr int RED = (XS_END > XS + kMegaMaxK * 4 ? XS_END : XS + kMegaMaxK * 4);   // 64 float4 + 64 ints
    static constexpr int BARS = RED + 64 * 16 + 64 * 4;                     // full[slot], empty[slot]
    static constexpr int TOKBAR = BARS + 2 * kMegaSlots * 8;                // token-start mbarrier
    static constexpr int SIZE = TOKBAR + 8;
};
// Dynamic shared memory plus the kernel's static arrays (plan tables, history
// words, residual rows) must fit one SM's 227 KB, or the occupancy check
// turns the persistent path off.
static_assert(MegaSmem::SIZE + 4096 <= 227 * 1024, "persistent decode shared memory exceeds 227 KB");

enum { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

// What this CTA streams in one phase.
struct MegaPlan {
    const unsigned char* src;   // gemv: first row of this CTA; attn: first K row
    const unsigned char* src2;  // attn: first V row
    int kind;
    int K;                      // gemv: row length (elements)
    int r0;                     // gemv: first row index
    int count;                  // gemv: rows; attn: positions
    int unit_bytes;             // gemv: bytes per row; attn: bytes per K (or V) row
    int per_stage;              // rows / positions per stage
    int nstage;
    int g, split;               // attn
};

// This CTA's row split of one GEMV phase kind; the same for every layer and token.
struct KindPlan {
    int r0, count, per_stage, nstage, unit_bytes, K;
};

// Per-CTA plan tables in shared memory, built once per launch, so that the
// stage walk never waits on a global load or a 64-bit division.
struct MegaTables {
    KindPlan kp[6];                                  // by phase kind (PH_ATTN unused)
    const unsigned char* w[5][kMegaMaxLayers];       // weight base by kind and layer (PH_ATTN unused)
    const unsigned char* embed;                      // tied LM head
};

template <typename WT>
__device__ __forceinline__ void mega_init_tables(const MegaArgs& a, MegaTables& tb, int b, int G, int tid)
{
    if (tid < 6 && tid != PH_ATTN)
    {
        const int kind = tid;
        int N, K;
        switch (kind)
        {
        case PH_QKV: N = kQKVRows; K = kHidden; break;
        case PH_O: N = kHidden; K = kQWidth; break;
        case PH_GU: N = 2 * a.ffn; K = kHidden; break;
        case PH_DOWN: N = kHidden; K = a.ffn; break;
        default: N = a.vocab; K = kHidden; break;
        }
        // gate/up rows are interleaved (2j = gate_j, 2j+1 = up_j): that phase is
        // split by pairs, and a stage never splits a pair.
        const int unit = (kind == PH_GU) ? 2 : 1;
        KindPlan k;
        k.r0 = unit * static_cast<int>(static_cast<long long>(N / unit) * b / G);
        const int r1 = unit * static_cast<int>(static_cast<long long>(N / unit) * (b + 1) / G);
        k.count = r1 - k.r0;
        k.K = K;
        k.unit_bytes = K * static_cast<int>(sizeof(WT));
        k.per_stage = min(8, max(1, kMegaStage / k.unit_bytes));
        if (unit == 2) k.per_stage &= ~1;
        k.nstage = (k.count + k.per_stage - 1) / k.per_stage;
        tb.kp[kind] = k;
    }
    if (tid == 0) tb.embed = static_cast<const unsigned char*>(a.embed);
    for (int e = tid; e < 4 * a.num_layers; e += kMegaThreads)
    {
        const int j = e / a.num_layers, l = e - j * a.num_layers;
        const void* const* arr = (j == 0) ? a.wqkv : (j == 1) ? a.wo : (j == 2) ? a.wgu : a.wd;
        tb.w[(j == 0) ? PH_QKV : j + 1][l] = static_cast<const unsigned char*>(arr[l]);
    }
}

template <typename KT>
__device__ __forceinline__ MegaPlan mega_plan(const MegaArgs& a, const MegaTables& tb, int layer, int kind, int past,
                                              int b)
{
    MegaPlan p;
    p.kind = kind;
    p.src2 = nullptr;
    p.g = p.split = 0;
    if (kind == PH_ATTN)
    {
        p.src = nullptr;
        p.K = kHeadDim;
        p.r0 = 0;
        p.unit_bytes = kHeadDim * static_cast<int>(sizeof(KT));
        p.per_stage = kMegaStage / (2 * p.unit_bytes);
        p.count = 0;
        if (b < kNumKVHeads * kMegaSplits)
        {
            p.g = b / kMegaSplits;
            p.split = b - p.g * kMegaSplits;
            if (p.split < kMegaSplits - 1)
            {
                const int chunk = (past + kMegaSplits - 2) / (kMegaSplits - 1);
                const int p0 = min(past, p.split * chunk);
                const int p1 = min(past, p0 + chunk);
                p.count = p1 - p0;
                const size_t off = ((static_cast<size_t>(layer) * kNumKVHeads + p.g) * a.cap + p0) * kHeadDim * sizeof(KT);
                p.src = static_cast<const unsigned char*>(a.kc) + off;
                p.src2 = static_cast<const unsigned char*>(a.vc) + off;
            }
        }
        p.nstage = (p.count + p.per_stage - 1) / p.per_stage;
        return p;
    }
    const KindPlan& k = tb.kp[kind];
    p.K = k.K;
    p.r0 = k.r0;
    p.count = k.count;
    p.unit_bytes = k.unit_bytes;
    p.per_stage = k.per_stage;
    p.nstage = k.nstage;
    p.src = ((kind == PH_LM) ? tb.embed : tb.w[kind][layer]) + static_cast<size_t>(k.r0) * k.unit_bytes;
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

// ---- epoch words ----
__device__ __forceinline__ unsigned long long ep_word(float v, unsigned e)
{
    return (static_cast<unsigned long long>(e) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Poll the words src[first + stride * u] (u < PER, index < n) until each
// carries epoch e, and return their values in out[u] (0 past n). Every round
// has all of the thread's outstanding loads in flight at once. Returns false
// (and sets the timeout bit) when the wall-clock limit passes first.
template <int PER>
__device__ __forceinline__ bool poll_words(const unsigned long long* src, int n, int first, int stride, unsigned e,
                                           float (&out)[PER], int* err, unsigned long long limit_ns,
                                           unsigned long long* ws = nullptr, int b = 0, int kind = 0,
                                           int* rounds = nullptr)
{
    const unsigned long long done = static_cast<unsigned long long>(e) << 32;   // value 0, epoch e
    unsigned long long w[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u)
    {
        const int i = first + stride * u;
        w[u] = (i < n) ? ld_relaxed_u64(src + i) : done;
    }
    unsigned long long t0 = 0;
    bool ok = true;
    while (true)
    {
        bool all = true;
#pragma unroll
        for (int u = 0; u < PER; ++u) all &= static_cast<unsigned>(w[u] >> 32) == e;
        if (all) break;
        const unsigned long long now = global_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > limit_ns)
        {
            atomicOr(err, kErrTimeoutFull);
            ok = false;
            break;
        }
        __nanosleep(HY_POLL_NS);
        if (rounds) ++*rounds;
#pragma unroll
        for (int u = 0; u < PER; ++u)
            if (static_cast<unsigned>(w[u] >> 32) != e) w[u] = ld_relaxed_u64(src + first + stride * u);
    }
#ifdef HY_WAIT_STATS
    if (t0) ws_record(ws, b, kind, global_ns() - t0);
#endif
#pragma unroll
    for (int u = 0; u < PER; ++u) out[u] = __uint_as_float(static_cast<unsigned>(w[u]));
    return ok;
}

// mbar_wait that also counts long waits in the HY_WAIT_STATS build.
__device__ __forceinline__ bool mega_mbar_wait(uint64_t* bar, uint32_t parity, int* err, int err_bit,
                                               unsigned long long limit_ns, unsigned long long* ws, int b, int kind)
{
#ifdef HY_WAIT_STATS
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    const bool ok = mbar_wait(bar, parity, err, err_bit, limit_ns);
    ws_record(ws, b, kind, global_ns() - t0);
    return ok;
#else
    return mbar_wait(bar, parity, err, err_bit, limit_ns);
#endif
}

// Bounded-wait self-test: waits, with the library's own primitives, for
// something that nothing provides. kind 0: poll_words on an epoch word that
// never carries the awaited epoch; kind 1: mbar_wait on a shared-memory
// mbarrier phase that never completes. Each gives up after limit_ns and sets
// the timeout bit in *err; no copy is in flight, so the early return is clean.
__global__ void wait_probe_kernel(const unsigned long long* word, int kind, unsigned long long limit_ns, int* err)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0)
    {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (kind == 0)
    {
        float v[1];
        poll_words<1>(word, 1, 0, 1, 0xFFFFFFFFu, v, err, limit_ns);
    }
    else
    {
        mbar_wait(&bar, 0, err, kErrTimeoutFull, limit_ns);
    }
}

// Where a GEMV phase's epilogue publishes its outputs, and with which epoch.
struct EpOut {
    unsigned long long* qkv;
    unsigned long long* act;
    unsigned long long* x;
    unsigned e;
};

// Rows per stage of a K-element row of WT (at most 8; even for K = 1024, so a
// gate/up pair never straddles two stages).
template <typename WT, int K>
struct StageRows {
    static constexpr int v = (kMegaStage / (K * static_cast<int>(sizeof(WT)))) < 8
                                 ? (kMegaStage / (K * static_cast<int>(sizeof(WT))))
                                 : 8;
    static_assert(v >= 1, "a row must fit in a stage");
};

// Warp sum of R per-lane partials at once: halving exchanges (each lane keeps
// the half of the rows named by its lane bit and adds its partner's copy of
// them), then a plain butterfly. Lane l returns the sum of row l / (32 / R):
// R - 1 + log2(32 / R) shuffles instead of 5 R.
template <int R>
__device__ __forceinline__ float reduce_rows(float (&v)[R], int lane)
{
#pragma unroll
    for (int h = R / 2, o = 16; h >= 1; h >>= 1, o >>= 1)
    {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < h; ++j)
        {
            const float send = up ? v[j] : v[j + h];
            const float keep = up ? v[j + h] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float s = v[0];
#pragma unroll
    for (int o = 16 / R; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// Partial dot products of the R rows of one stage with x (lane-strided
// float4s), reduced with reduce_rows. x comes from registers (XREG, K = 1024:
// lane l holds float4 l + 32 i in xr[i]) or from shared memory.
template <typename WT, int K, int R, bool XREG>
__device__ __forceinline__ float stage_dot(const WT* rows, const float4 (&xr)[8], const float* xs, int lane)
{
    static_assert(K % 128 == 0, "K must be a multiple of 128");
    static_assert(!XREG || K == 1024, "register-resident x is 1024 wide");
    constexpr int A = (R >= 4) ? 1 : 2;   // accumulators per row (FMA chain length)
    float acc[R * A];
#pragma unroll
    for (int j = 0; j < R * A; ++j) acc[j] = 0.f;
#pragma unroll
    for (int i = 0; i < K / 128; ++i)
    {
        const int c = lane + 32 * i;
        float4 x;
        if constexpr (XREG) x = xr[i];
        else x = *reinterpret_cast<const float4*>(xs + 4 * c);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r * A + (i % A)] += dot4(load4(rows + r * K + 4 * c), x);
    }
    float v[R];
#pragma unroll
    for (int r = 0; r < R; ++r)
    {
        v[r] = acc[r * A];
#pragma unroll
        for (int j = 1; j < A; ++j) v[r] += acc[r * A + j];
    }
    return reduce_rows<R>(v, lane);
}

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

// Named barrier of the consumer warps (the producer warp never joins it).
__device__ __forceinline__ void mega_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kMegaConsumers) : "memory"); }

// xs = w * x for a 1024-vector x given as float4 i = tid + kMegaConsumers u in v[u];
// returns 1/sqrt(mean(x^2)+eps) after one CTA barrier. The GEMV multiplies its
// dot products by it, i.e. the RMSNorm's per-row scale is applied after the projection.
__device__ __forceinline__ float mega_load_normed(float* xs, const float4 v[2], const float* w, float eps,
                                                  float* s_norm, int tid)
{
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u)
    {
        const int i = tid + kMegaConsumers * u;
        if (i < kHidden / 4)
        {
            const float4 wv = *reinterpret_cast<const float4*>(w + 4 * i);
            ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
            float4 o;
            o.x = wv.x * v[u].x;
            o.y = wv.y * v[u].y;
            o.z = wv.z * v[u].z;
            o.w = wv.w * v[u].w;
            *reinterpret_cast<float4*>(xs + 4 * i) = o;
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) s_norm[tid >> 5] = ss;
    mega_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kMegaWarps; ++i) t += s_norm[i];
    return 1.0f / sqrtf(t / static_cast<float>(kHidden) + eps);
}

// xs = w * x for a 1024-vector x given as x[tid + kMegaConsumers u] in v[u] (u < kXPer);
// returns 1/sqrt(mean(x^2)+eps) after one consumer barrier (the GEMV applies
// the RMSNorm's per-row scale to its dot products).
constexpr int kXPer = (kHidden + kMegaConsumers - 1) / kMegaConsumers;

__device__ __forceinline__ float mega_load_normed_s(float* xs, const float (&v)[kXPer], const float (&w)[kXPer],
                                                    float eps, float* s_norm, int tid)
{
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < kXPer; ++u)
    {
        const int i = tid + kMegaConsumers * u;
        if (i < kHidden)
        {
            ss += v[u] * v[u];
            xs[i] = w[u] * v[u];
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) s_norm[tid >> 5] = ss;
    mega_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kMegaWarps; ++i) t += s_norm[i];
    return 1.0f / sqrtf(t / static_cast<float>(kHidden) + eps);
}

// The RoPE table entries and norm weights one lane needs for rope_norm_vals, loaded
// before the lane waits for the vector itself (they are constants of the phase).
struct RopeNormIn {
    float c[4], s[4], w[4];
};
__device__ __forceinline__ RopeNormIn rope_norm_in(const float* c, const float* s, const float* w, int lane)
{
    RopeNormIn r;
#pragma unroll
    for (int j = 0; j < 4; ++j)
    {
        r.c[j] = c[lane + 32 * j];
        r.s[j] = s[lane + 32 * j];
        r.w[j] = w[lane + 32 * j];
    }
    return r;
}

// RoPE + RMSNorm of one 128-vector given as x[lane + 32 j] in x[j] (as rope_norm_vec).
__device__ __forceinline__ void rope_norm_vals(const float (&x)[4], const RopeNormIn& in, float eps, float out[4])
{
    float y0 = x[0] * in.c[0] - x[2] * in.s[0];
    float y1 = x[1] * in.c[1] - x[3] * in.s[1];
    float y2 = x[2] * in.c[2] + x[0] * in.s[2];
    float y3 = x[3] * in.c[3] + x[1] * in.s[3];
    const float ss = warp_sum(y0 * y0 + y1 * y1 + y2 * y2 + y3 * y3);
    const float ri = 1.0f / sqrtf(ss / static_cast<float>(kHeadDim) + eps);
    out[0] = in.w[0] * (y0 * ri);
    out[1] = in.w[1] * (y1 * ri);
    out[2] = in.w[2] * (y2 * ri);
    out[3] = in.w[3] * (y3 * ri);
}

// One GEMV stage of a consumer warp: dot products of the stage's rows, slot
// release, and the epilogue run by one lane per row.
struct LmBest {
    float rv, pv;
    int ri, pi;
};

template <typename WT, int K, bool XREG>
__device__ __forceinline__ void gemv_stage(const MegaArgs& a, const MegaPlan& p, int kind, const WT* rows,
                                           const float4 (&xr)[8], const float* xs, int q0, float rinv, const EpOut& eo,
                                           float* xres_s, const unsigned* hist_s, float pen, LmBest& best,
                                           uint64_t* empty_bar, int lane, int b, int ph)
{
    constexpr int R = StageRows<WT, K>::v;
    const float val = stage_dot<WT, K, R, XREG>(rows, xr, xs, lane) * rinv;
    // Every lane's slot reads have returned (their values went through the
    // shuffles): hand the slot back to the producer.
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);

    const int n = min(R, p.count - q0);
    constexpr int LPR = 32 / R;   // lanes holding each row's sum
    const int r = lane / LPR;
    const int row = p.r0 + q0 + r;
    const int nrows = (kind == PH_QKV) ? kQKVRows : (kind == PH_GU) ? 2 * a.ffn : (kind == PH_LM) ? a.vocab : kHidden;
    const bool ok = mega_check(p.r0 + q0 + n <= nrows && ((kind != PH_O && kind != PH_DOWN) || q0 + n <= kMegaResRows),
                               a.dbg, 2, b, ph, p.r0 + q0);
    const bool lead = ok && (lane % LPR) == 0 && r < n;
    if (kind == PH_QKV)
    {
        if (lead) st_relaxed_u64(eo.qkv + row, ep_word(val, eo.e));
    }
    else if (kind == PH_GU)
    {
        // act = silu(gate) * up; gate = even row, up = the next row's lanes.
        const float up = __shfl_down_sync(0xffffffffu, val, LPR);
        if (lead && !(r & 1)) st_relaxed_u64(eo.act + (row >> 1), ep_word((val / (1.0f + expf(-val))) * up, eo.e));
    }
    else if (kind == PH_O || kind == PH_DOWN)
    {
        // The residual rows this CTA owns stay in shared memory across phases.
        if (lead)
        {
            const float xn = xres_s[q0 + r] + val;
            xres_s[q0 + r] = xn;
            st_relaxed_u64(eo.x + row, ep_word(xn, eo.e));
        }
    }
    else if (lead)
    {
        const int wi = (row >> 5) - (p.r0 >> 5);
        if (mega_check(wi >= 0 && wi < kMegaHistWords, a.dbg, 3, b, ph, wi))
        {
            const bool hit = (hist_s[wi] >> (row & 31)) & 1u;
            const float ps = hit ? (val < 0.0f ? val * pen : val / pen) : val;
            if (best.ri < 0 || val > best.rv) { best.rv = val; best.ri = row; }
            if (best.pi < 0 || ps > best.pv) { best.pv = ps; best.pi = row; }
        }
    }
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
    float* pbuf_all = reinterpret_cast<float*>(smem + MegaSmem::PBUF);
    float4* red4 = reinterpret_cast<float4*>(smem + MegaSmem::RED);
    int* redi = reinterpret_cast<int*>(red4 + 64);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + MegaSmem::BARS);   // [slot]
    uint64_t* empty = full + kMegaSlots;                                   // [slot]
    // Completes once per token t >= 1 when the consumers have acquired the
    // previous token's commit; the producer waits on it before streaming the
    // token's K/V rows, whose newest row the previous token wrote.
    uint64_t* tokbar = reinterpret_cast<uint64_t*>(smem + MegaSmem::TOKBAR);
    __shared__ unsigned hist_s[kMegaHistWords];
    __shared__ float xres_s[kMegaResRows];
    __shared__ float s_norm[kMegaWarps];
    __shared__ MegaTables tb;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int L = a.num_layers;
    const int phases = 5 * L + 1;
    const int kv0 = a.st->kv_len;  // set by the host before the launch

    if (tid == 0)
    {
        for (int s = 0; s < kMegaSlots; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tokbar, 1);
        fence_mbar_init();
        redi[0] = 0;  // abort flag
    }
    mega_init_tables<WT>(a, tb, b, G, tid);
#ifdef HY_WAIT_STATS
    if (tid == 0 && a.wstat)
        atomicMax(a.wstat + kWsLaunchBase + 2 * (a.launch_slot % kWsLaunches), ~global_ns());
#endif
    __syncthreads();

    if (warp == kMegaWarps)
    {
        // ======================= producer =======================
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first_policy();
        unsigned g = 0;   // global stage index: slot g % kMegaSlots, owner warp g % kMegaWarps
        bool ok = true;
        for (int t = 0; t < a.steps && ok; ++t)
        {
            for (int ph = 0; ph < phases && ok; ++ph)
            {
                int layer, kind;
                mega_phase_of(ph, L, layer, kind);
                const MegaPlan p = mega_plan<KT>(a, tb, layer, kind, kv0 + t, b);
                if (kind == PH_ATTN && layer == 0 && t > 0 && p.nstage > 0 &&
                    !mega_mbar_wait(tokbar, (t - 1) & 1, a.err, kErrTimeoutEmpty, a.wait_limit_ns, a.wstat, b, WS_PROD_TOKEN))
                {
                    ok = false;
                    break;
                }
                for (int i = 0; i < p.nstage; ++i, ++g)
                {
                    const int s = static_cast<int>(g % kMegaSlots);
                    const unsigned j = g / kMegaSlots;   // use of the slot
                    // The slot's previous stage (g - kMegaSlots) was released by its warp.
                    if (j >= 1 && !mega_mbar_wait(&empty[s], (j - 1) & 1, a.err, kErrTimeoutEmpty, a.wait_limit_ns, a.wstat, b, WS_PROD_EMPTY))
                    {
                        ok = false;
                        break;
                    }
                    // At most kMegaInflight stages in flight: stage g - kMegaInflight has
                    // landed (its slot's full phase; that slot is re-armed only by a later
                    // stage than g, so the parity wait is exact).
                    const int cap = (kind == PH_LM) ? kMegaInflightLm : (kind == PH_ATTN) ? kMegaInflightAttn : kMegaInflight;
                    if (cap < kMegaSlots && g >= static_cast<unsigned>(cap))
                    {
                        const unsigned gp = g - cap;
                        if (!mega_mbar_wait(&full[gp % kMegaSlots], (gp / kMegaSlots) & 1, a.err, kErrTimeoutFull,
                                            a.wait_limit_ns, a.wstat, b, WS_PROD_EMPTY))
                        {
                            ok = false;
                            break;
                        }
                    }
                    const int n = min(p.per_stage, p.count - i * p.per_stage);
                    const uint32_t bytes = static_cast<uint32_t>(n * p.unit_bytes);
                    unsigned char* dst = ring + static_cast<size_t>(s) * kMegaStage;
                    const size_t off = static_cast<size_t>(i) * p.per_stage * p.unit_bytes;
                    if (kind == PH_ATTN)
                    {
                        // (The K/V rows' writers fenced them for the async proxy.)
                        mbar_arrive_expect_tx(&full[s], 2 * bytes);
                        bulk_g2s(dst, p.src + off, bytes, &full[s], pol);
                        bulk_g2s(dst + p.per_stage * p.unit_bytes, p.src2 + off, bytes, &full[s], pol);
                    }
                    else
                    {
                        mbar_arrive_expect_tx(&full[s], bytes);
                        bulk_g2s(dst, p.src + off, bytes, &full[s], pol);
                    }
                }
            }
        }
        // Drain: the last kMegaSlots stages (earlier ones landed before their
        // slot was released).
        for (unsigned gg = (g > kMegaSlots ? g - kMegaSlots : 0); gg < g; ++gg)
            mbar_wait(&full[gg % kMegaSlots], (gg / kMegaSlots) & 1, a.err, kErrTimeoutFull);
        return;
    }

    // ======================= consumers =======================
    // Wait for global stage g (one of this warp's); its slot, or -1 on timeout.
    // A parity wait is exact only on the barrier's current phase or the one
    // just completed, and the slot's previous stage g - kMegaSlots belongs to
    // another warp, which may not have received (or released) it yet - copies
    // issued earlier can land later. So the warp first waits until that stage
    // was released (empty phase j - 1), then for stage g itself (full phase j).
    // Both waits start at most one phase early: if g - kMegaSlots is in this
    // phase, so is this warp's previous stage g - kMegaWarps, whose issue needed
    // g - kMegaSlots issued and so g - 2 kMegaSlots released; if it is in an
    // earlier phase, the phase-end barrier saw it released. A released stage
    // has landed, and no use after j can start before this warp releases g.
    auto wait_stage = [&](unsigned g) -> int {
        const int slot = static_cast<int>(g % kMegaSlots);
        const unsigned j = g / kMegaSlots;
        bool okw = (j == 0) || mega_mbar_wait(&empty[slot], (j - 1) & 1, a.err, kErrTimeoutEmpty, a.wait_limit_ns, a.wstat, b, WS_SLOT_FREE);
        okw = okw && mega_mbar_wait(&full[slot], j & 1, a.err, kErrTimeoutFull, a.wait_limit_ns, a.wstat, b, WS_SLOT_FULL);
        return __all_sync(0xffffffffu, okw) ? slot : -1;
    };

    unsigned gs = 0;          // global stage index of the current phase's first stage
    const MegaPlan po = mega_plan<KT>(a, tb, 0, PH_O, kv0, b);   // this CTA's residual rows (o and down)
    // A failed wait marks the warp bad and raises the CTA's abort flag; every
    // warp still takes the phase's CTA barriers, and the CTA leaves together.
    bool bad = false;
    for (int t = 0; t < a.steps && !bad; ++t)
    {
        const int past = kv0 + t;
        for (int ph = 0; ph < phases; ++ph)
        {
            int layer, kind;
            mega_phase_of(ph, L, layer, kind);
            // Epoch of the previous phase's outputs (for ph = 0: the previous token's commit).
            const unsigned e_in = a.epoch_base + static_cast<unsigned>(t * phases + ph);
            const EpOut eo{a.qkv_ep, a.act_ep, a.x_ep, e_in + 1};
            const bool tracing = a.trace && t == a.trace_token && b < kTraceCtas && tid == 0;
            unsigned long long* tr = tracing ? a.trace + (static_cast<size_t>(b) * phases + ph) * kTraceSlots : nullptr;
            if (tracing) tr[0] = global_ns();
            // Warp-0 trace: SM cycles waiting on slots / working, stages.
            const bool wtr = a.trace && t == a.trace_token && b < kTraceCtas && tid == 0;
            long long wwait = 0, wwork = 0, wn = 0;
            const MegaPlan p = mega_plan<KT>(a, tb, layer, kind, past, b);
            const float* lnorm = a.norms + static_cast<size_t>(layer) * 2304;
            // This warp's stages of the phase: first, first + kMegaWarps, ...
            const int first = static_cast<int>((warp - static_cast<int>(gs % kMegaWarps) + kMegaWarps) % kMegaWarps);

            // ---------------- prologue: wait for and stage the activation vector ----------------
            float rinv = 1.0f;   // RMSNorm scale applied to the dot products
            if (kind == PH_QKV || kind == PH_GU || kind == PH_LM)
            {
                // The RMSNorm weights are constants: their loads are in flight while the
                // activation words are polled.
                const float* nw = (kind == PH_QKV) ? lnorm
                                  : (kind == PH_GU) ? lnorm + kHidden
                                                    : a.norms + static_cast<size_t>(L) * 2304;
                float nwv[kXPer];
#pragma unroll
                for (int u = 0; u < kXPer; ++u)
                {
                    const int i = tid + kMegaConsumers * u;
                    nwv[u] = (i < kHidden) ? __ldg(nw + i) : 0.f;
                }
                float v[kXPer];
                if (kind == PH_QKV && layer == 0)
                {
                    // The token: set by the host for the launch's first token, then
                    // published by the previous token's commit (acquire: its history
                    // bits and state writes are visible after this).
                    int id;
                    if (t == 0)
                    {
                        id = __ldcg(&a.st->cur_token);
                    }
                    else
                    {
                        unsigned long long w = ld_acquire_u64(a.tok_ep);
                        const unsigned long long t0 = global_ns();
                        while (static_cast<unsigned>(w >> 32) != e_in)
                        {
                            if (global_ns() - t0 > a.wait_limit_ns)
                            {
                                atomicOr(a.err, kErrTimeoutFull);
                                redi[0] = 1;
                                break;
                            }
                            __nanosleep(HY_POLL_NS);
                            w = ld_acquire_u64(a.tok_ep);
                        }
#ifdef HY_WAIT_STATS
                        ws_record(a.wstat, b, WS_POLL_TOKEN, global_ns() - t0);
#endif
                        id = static_cast<int>(static_cast<unsigned>(w));
                        if (tid == 0) mbar_arrive(tokbar);   // after this thread's acquire
                    }
                    if (id < 0 || id >= a.vocab)
                    {
                        if (tid == 0) atomicOr(a.err, kErrBounds);
                        id = 0;
                    }
                    const WT* erow = static_cast<const WT*>(a.embed) + static_cast<size_t>(id) * kHidden;
#pragma unroll
                    for (int u = 0; u < kXPer; ++u)
                    {
                        const int i = tid + kMegaConsumers * u;
                        v[u] = (i < kHidden) ? to_f32<WT>(erow[i]) : 0.f;
                    }
                    // The residual rows this CTA owns start as the embedding.
                    if (tid < po.count && tid < kMegaResRows) xres_s[tid] = to_f32<WT>(erow[po.r0 + tid]);
                }
                else
                {
                    int rounds = 0;
                    const unsigned long long tp0 = tracing ? global_ns() : 0;
                    if (!poll_words<kXPer>(a.x_ep, kHidden, tid, kMegaConsumers, e_in, v, a.err, a.wait_limit_ns,
                                           a.wstat, b, WS_POLL_X, tracing ? &rounds : nullptr))
                        redi[0] = 1;
                    if (tracing)
                    {
                        tr[7] = rounds;
                        tr[8] = global_ns() - tp0;
                        tr[10] = tp0;
                    }
                }
                if (kind == PH_LM && p.count > 0)
                {
                    // Penalty-history words covering this CTA's vocab rows.
                    const int w0 = p.r0 >> 5, w1 = (p.r0 + p.count - 1) >> 5;
                    if (tid <= w1 - w0 && tid < kMegaHistWords) hist_s[tid] = __ldcg(a.hist + w0 + tid);
                }
                rinv = mega_load_normed_s(xs, v, nwv, a.eps, s_norm, tid);   // (one consumer barrier)
            }
            else if (kind == PH_DOWN)
            {
                // act = silu(gate) * up from the gate/up phase.
                constexpr int kPer = (kMegaMaxK + kMegaConsumers - 1) / kMegaConsumers;
                float v[kPer];
                int rounds = 0;
                const unsigned long long tp0 = tracing ? global_ns() : 0;
                if (!poll_words<kPer>(a.act_ep, a.ffn, tid, kMegaConsumers, e_in, v, a.err, a.wait_limit_ns, a.wstat, b,
                                      WS_POLL_ACT, tracing ? &rounds : nullptr))
                    redi[0] = 1;
                if (tracing)
                {
                    tr[7] = rounds;
                    tr[8] = global_ns() - tp0;
                    tr[10] = tp0;
                }
#pragma unroll
                for (int u = 0; u < kPer; ++u)
                {
                    const int i = tid + kMegaConsumers * u;
                    if (i < a.ffn) xs[i] = v[u];
                }
                mega_sync();
            }
            else if (kind == PH_O)
            {
                // The attention output of all 16 heads (merged by each head pair's new-row split).
                constexpr int kPer = (kQWidth + kMegaConsumers - 1) / kMegaConsumers;
                float v[kPer];
                int rounds = 0;
                const unsigned long long tp0 = tracing ? global_ns() : 0;
                if (!poll_words<kPer>(a.attn_out_ep, kQWidth, tid, kMegaConsumers, e_in, v, a.err, a.wait_limit_ns, a.wstat, b,
                                      WS_POLL_ATTN_OUT, tracing ? &rounds : nullptr))
                    redi[0] = 1;
                if (tracing)
                {
                    tr[7] = rounds;
                    tr[8] = global_ns() - tp0;
                    tr[10] = tp0;
                }
#pragma unroll
                for (int u = 0; u < kPer; ++u)
                {
                    const int i = tid + kMegaConsumers * u;
                    if (i < kQWidth) xs[i] = v[u];
                }
                mega_sync();
            }
            // (Attention polls its inputs below; every other kind has passed a
            // consumer barrier after its polls, so the flag is settled here.)
            if (kind != PH_ATTN && redi[0])
            {
                bad = true;
                break;
            }
            if (tracing) tr[1] = global_ns();
            if (tracing) tr[2] = global_ns();

            if (kind != PH_ATTN)
            {
                // ---------------- GEMV rows of this warp's stages ----------------
                LmBest best{0.f, 0.f, -1, -1};
                const float pen = a.st->penalty;
                // The normalised activation vector in registers for K = 1024.
                float4 xr[8];
                if (p.K == kHidden)
                {
#pragma unroll
                    for (int i = 0; i < 8; ++i) xr[i] = reinterpret_cast<const float4*>(xs)[lane + 32 * i];
                }
                for (int i = first; i < p.nstage && !bad; i += kMegaWarps)
                {
                    const long long c0 = wtr ? clock64() : 0;
                    const int slot = wait_stage(gs + static_cast<unsigned>(i));
                    const long long c1 = wtr ? clock64() : 0;
                    if (slot < 0)
                    {
                        if (lane == 0) redi[0] = 1;
                        bad = true;
                        break;
                    }
                    const WT* rows = reinterpret_cast<const WT*>(ring + slot * kMegaStage);
                    const int q0 = i * p.per_stage;
                    if (p.K == kHidden)
                        gemv_stage<WT, kHidden, true>(a, p, kind, rows, xr, xs, q0, rinv, eo, xres_s, hist_s, pen, best,
                                                      &empty[slot], lane, b, ph);
                    else if (p.K == kQWidth)
                        gemv_stage<WT, kQWidth, false>(a, p, kind, rows, xr, xs, q0, rinv, eo, xres_s, hist_s, pen, best,
                                                       &empty[slot], lane, b, ph);
                    else
                        gemv_stage<WT, kMegaMaxK, false>(a, p, kind, rows, xr, xs, q0, rinv, eo, xres_s, hist_s, pen,
                                                         best, &empty[slot], lane, b, ph);
                    if (wtr)
                    {
                        wwait += c1 - c0;
                        wwork += clock64() - c1;
                        ++wn;
                    }
                }
                if (kind == PH_LM)
                {
                    // This warp's best rows: merge the lanes, then the warps.
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
                    {
                        const float orv = __shfl_xor_sync(0xffffffffu, best.rv, o);
                        const int ori = __shfl_xor_sync(0xffffffffu, best.ri, o);
                        const float opv = __shfl_xor_sync(0xffffffffu, best.pv, o);
                        const int opi = __shfl_xor_sync(0xffffffffu, best.pi, o);
                        if (ori >= 0) best_update(best.rv, best.ri, orv, ori);
                        if (opi >= 0) best_update(best.pv, best.pi, opv, opi);
                    }
                    if (lane == 0) red4[warp] = make_float4(best.rv, __int_as_float(best.ri), best.pv, __int_as_float(best.pi));
                    mega_sync();
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
                    mega_sync();
                    if (redi[1])
                    {
                        // Last CTA: merge the G partials (parallel loads, then a tree).
                        __threadfence();
                        float rv = 0.f, pv = 0.f;
                        int ri = -1, pi = -1;
                        for (int c = tid; c < G; c += kMegaConsumers)
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
                        mega_sync();
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
                            if (!mega_check(fpi >= 0 && fpi < a.vocab && fri >= 0 && fri < a.vocab, a.dbg, 4, b, ph, fpi))
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
                            // Publish the next token (also after the stream ended: the
                            // remaining tokens of the launch still run, uncommitted).
                            // Release: the history bits, the state and the ticket reset
                            // above are visible to whoever acquires this word.
                            __threadfence();
                            st_release_u64(a.tok_ep, (static_cast<unsigned long long>(eo.e) << 32) |
                                                         static_cast<unsigned>(st->cur_token));
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
                // q/k/v of this KV head from the q/k/v phase (epoch words); the RoPE
                // entries and norm weights are loaded first, while the words are polled.
                if (warp < 2)
                {
                    const RopeNormIn rin = rope_norm_in(c, s, qn_w, lane);
                    float x[4], o[4];
                    if (!poll_words<4>(a.qkv_ep + (2 * g + warp) * kHeadDim, kHeadDim, lane, 32, e_in, x, a.err,
                                       a.wait_limit_ns, a.wstat, b, WS_POLL_QKV))
                        redi[0] = 1;
                    rope_norm_vals(x, rin, a.eps, o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) qs[warp * kHeadDim + lane + 32 * i] = o[i] * a.scale_log2;
                }
                else if (new_split && warp == 2)
                {
                    const RopeNormIn rin = rope_norm_in(c, s, kn_w, lane);
                    float x[4], o[4];
                    if (!poll_words<4>(a.qkv_ep + kQWidth + g * kHeadDim, kHeadDim, lane, 32, e_in, x, a.err, a.wait_limit_ns, a.wstat, b,
                                       WS_POLL_QKV))
                        redi[0] = 1;
                    rope_norm_vals(x, rin, a.eps, o);
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
                    // Later tokens read this row with bulk copies (async proxy).
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                else if (new_split && warp == 3)
                {
                    float x[4];
                    if (!poll_words<4>(a.qkv_ep + kQWidth + kKVWidth + g * kHeadDim, kHeadDim, lane, 32, e_in, x, a.err,
                                       a.wait_limit_ns, a.wstat, b, WS_POLL_QKV))
                        redi[0] = 1;
                    KT* vrow = static_cast<KT*>(a.vc) +
                               ((static_cast<size_t>(layer) * kNumKVHeads + g) * a.cap + min(past, a.cap - 1)) * kHeadDim;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                    {
                        const KT q = from_f32<KT>(x[i]);
                        vrow[lane + 32 * i] = q;
                        vnew[lane + 32 * i] = to_f32<KT>(q);
                    }
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                mega_sync();

                // Lane l owns dims 4l..4l+3 of both queries (o0, o1); the
                // running max / sum of each query (m0, l0, m1, l1) are kept
                // in every lane. Scores are in log2 units (q carries scale * log2 e).
                const float4 qv0 = reinterpret_cast<const float4*>(qs)[lane];
                const float4 qv1 = reinterpret_cast<const float4*>(qs + kHeadDim)[lane];
                float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
                float4 o0 = make_float4(0.f, 0.f, 0.f, 0.f), o1 = o0;
                float* pbuf = pbuf_all + warp * 32;
                // Rescale the running state to new maxima mn0 / mn1.
                auto rescale = [&](float mn0, float mn1) {
                    const float c0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mn0);
                    const float c1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mn1);
                    l0 *= c0;
                    l1 *= c1;
                    o0.x *= c0; o0.y *= c0; o0.z *= c0; o0.w *= c0;
                    o1.x *= c1; o1.y *= c1; o1.z *= c1; o1.w *= c1;
                    m0 = mn0;
                    m1 = mn1;
                };
                // 16 cached positions starting at row `base` of the stage, nv of them valid.
                auto block16 = [&](const KT* kst, const KT* vst, int nv) {
                    float v[32];   // v[q * 16 + j]: partial score of query q, position j
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                    {
                        const float4 k = load4(kst + static_cast<size_t>(j) * kHeadDim + 4 * lane);
                        v[j] = dot4(qv0, k);
                        v[16 + j] = dot4(qv1, k);
                    }
                    // Lane l: full score of query l >> 4, position l & 15.
                    float sc = reduce_rows<32>(v, lane);
                    const bool valid = (lane & 15) < nv;
                    sc = valid ? sc : -INFINITY;
                    float mx = sc;
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    const float mn0 = fmaxf(m0, __shfl_sync(0xffffffffu, mx, 0));
                    const float mn1 = fmaxf(m1, __shfl_sync(0xffffffffu, mx, 16));
                    const float pe = valid ? exp2f(sc - ((lane < 16) ? mn0 : mn1)) : 0.f;
                    float ps = pe;
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    rescale(mn0, mn1);
                    l0 += __shfl_sync(0xffffffffu, ps, 0);
                    l1 += __shfl_sync(0xffffffffu, ps, 16);
                    pbuf[lane] = pe;
                    __syncwarp();
                    auto accum = [&](int j, float p0, float p1) {
                        const float4 vv = load4(vst + static_cast<size_t>(j) * kHeadDim + 4 * lane);
                        o0.x += p0 * vv.x; o0.y += p0 * vv.y; o0.z += p0 * vv.z; o0.w += p0 * vv.w;
                        o1.x += p1 * vv.x; o1.y += p1 * vv.y; o1.z += p1 * vv.z; o1.w += p1 * vv.w;
                    };
                    if (nv == 16)
                    {
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4)
                        {
                            const float4 P0 = reinterpret_cast<const float4*>(pbuf)[j4];
                            const float4 P1 = reinterpret_cast<const float4*>(pbuf + 16)[j4];
                            accum(4 * j4 + 0, P0.x, P1.x);
                            accum(4 * j4 + 1, P0.y, P1.y);
                            accum(4 * j4 + 2, P0.z, P1.z);
                            accum(4 * j4 + 3, P0.w, P1.w);
                        }
                    }
                    else
                    {
                        // Warp-uniform bound: rows past nv hold stale data and are never read.
                        for (int j = 0; j < nv; ++j) accum(j, pbuf[j], pbuf[16 + j]);
                    }
                    __syncwarp();
                };
                // Trace: the warp that owns the split's first stage records its
                // slot-wait / work cycles and stages in slots 7..9, and the
                // time its stage loop ended in slot 10.
                const bool atr = a.trace && t == a.trace_token && b < kTraceCtas && lane == 0 && first == 0;
                long long await_ = 0, awork = 0, an = 0;
                for (int i = first; i < p.nstage && !bad; i += kMegaWarps)
                {
                    const long long c0 = atr ? clock64() : 0;
                    const int slot = wait_stage(gs + static_cast<unsigned>(i));
                    const long long c1 = atr ? clock64() : 0;
                    if (slot < 0)
                    {
                        if (lane == 0) redi[0] = 1;
                        bad = true;
                        break;
                    }
                    const KT* kst = reinterpret_cast<const KT*>(ring + slot * kMegaStage);
                    const KT* vst = kst + static_cast<size_t>(p.per_stage) * kHeadDim;
                    const int n = min(p.per_stage, p.count - i * p.per_stage);
                    for (int h = 0; h < n; h += 16)
                        block16(kst + static_cast<size_t>(h) * kHeadDim, vst + static_cast<size_t>(h) * kHeadDim,
                                min(16, n - h));
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                    if (atr)
                    {
                        await_ += c1 - c0;
                        awork += clock64() - c1;
                        ++an;
                    }
                }
                if (atr)
                {
                    unsigned long long* ta = a.trace + (static_cast<size_t>(b) * phases + ph) * kTraceSlots;
                    ta[7] = await_;
                    ta[8] = awork;
                    ta[9] = an;
                    ta[10] = global_ns();
                }
                if (new_split && warp == 0)
                {
                    // The new row (already rounded to the cache type).
                    const float4 k = reinterpret_cast<const float4*>(knew)[lane];
                    const float4 vv = reinterpret_cast<const float4*>(vnew)[lane];
                    float s0 = dot4(qv0, k), s1 = dot4(qv1, k);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
                    {
                        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
                    }
                    rescale(fmaxf(m0, s0), fmaxf(m1, s1));
                    const float p0 = exp2f(s0 - m0), p1 = exp2f(s1 - m1);
                    l0 += p0;
                    l1 += p1;
                    o0.x += p0 * vv.x; o0.y += p0 * vv.y; o0.z += p0 * vv.z; o0.w += p0 * vv.w;
                    o1.x += p1 * vv.x; o1.y += p1 * vv.y; o1.z += p1 * vv.z; o1.w += p1 * vv.w;
                }
                {
                    float* w0 = ascr + (warp * 2 + 0) * kPartStride;
                    float* w1 = ascr + (warp * 2 + 1) * kPartStride;
                    if (lane == 0)
                    {
                        w0[0] = m0;
                        w0[1] = l0;
                        w1[0] = m1;
                        w1[1] = l1;
                    }
                    reinterpret_cast<float4*>(w0 + 4)[lane] = o0;
                    reinterpret_cast<float4*>(w1 + 4)[lane] = o1;
                }
                mega_sync();
                // This CTA's partial per query: 2 queries x 128 dims. A past
                // split publishes it as epoch words; the new-row split keeps it.
                float* mine = reinterpret_cast<float*>(smem + MegaSmem::MINE);
                for (int e = tid; e < 2 * kHeadDim; e += kMegaConsumers)
                {
                    const int q = e >> 7, d = e & 127;
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
                    if (!new_split)
                    {
                        unsigned long long* part =
                            a.attn_ep + ((static_cast<size_t>(g) * (kMegaSplits - 1) + p.split) * 2 + q) * kAttnWords;
                        if (d == 0)
                        {
                            st_relaxed_u64(part, ep_word(M, eo.e));
                            st_relaxed_u64(part + 1, ep_word(Lsum, eo.e));
                        }
                        st_relaxed_u64(part + 2 + d, ep_word(A, eo.e));
                    }
                    else
                    {
                        if (d == 0)
                        {
                            mine[q * kPartStride] = M;
                            mine[q * kPartStride + 1] = Lsum;
                        }
                        mine[q * kPartStride + 4 + d] = A;
                    }
                }
                if (new_split)
                {
                    // Merge the head pair's split partials (split-K flash-decode
                    // combine, splits in order, this CTA's new-row split last) and
                    // publish the two heads' outputs for the o projection.
                    constexpr int kWords = (kMegaSplits - 1) * 2 * kAttnWords;
                    constexpr int kPer = (kWords + kMegaConsumers - 1) / kMegaConsumers;
                    float* parts = reinterpret_cast<float*>(smem + MegaSmem::PARTS);
                    float v[kPer];
                    if (!poll_words<kPer>(a.attn_ep + static_cast<size_t>(g) * kWords, kWords, tid, kMegaConsumers, eo.e,
                                          v, a.err, a.wait_limit_ns, a.wstat, b, WS_POLL_PARTS))
                        redi[0] = 1;
#pragma unroll
                    for (int u = 0; u < kPer; ++u)
                    {
                        const int i = tid + kMegaConsumers * u;
                        if (i < kWords) parts[i] = v[u];
                    }
                    mega_sync();
                    for (int e = tid; e < 2 * kHeadDim; e += kMegaConsumers)
                    {
                        const int q = e >> 7, d = e & 127;
                        const float mm = mine[q * kPartStride];
                        float M = mm;
#pragma unroll
                        for (int sp = 0; sp < kMegaSplits - 1; ++sp) M = fmaxf(M, parts[(sp * 2 + q) * kAttnWords]);
                        float Lsum = 0.f, A = 0.f;
#pragma unroll
                        for (int sp = 0; sp < kMegaSplits - 1; ++sp)
                        {
                            const float* ps = parts + (sp * 2 + q) * kAttnWords;
                            const float f = (ps[0] == -INFINITY) ? 0.f : exp2f(ps[0] - M);
                            Lsum += f * ps[1];
                            A += f * ps[2 + d];
                        }
                        {
                            const float f = (mm == -INFINITY) ? 0.f : exp2f(mm - M);
                            Lsum += f * mine[q * kPartStride + 1];
                            A += f * mine[q * kPartStride + 4 + d];
                        }
                        st_relaxed_u64(a.attn_out_ep + (2 * g + q) * kHeadDim + d, ep_word(A * (1.0f / Lsum), eo.e));
                    }
                }
            }

            gs += p.nstage;
            if (wtr)
            {
                tr[4] = wwait;
                tr[5] = wwork;
                tr[6] = wn;
            }
            // ---------------- phase done ----------------
            mega_sync();
            if (redi[0])
            {
                bad = true;
                break;
            }
            if (tracing) tr[3] = global_ns();
            if (tid == 0 && a.progress) a.progress[b] = static_cast<unsigned>(t * phases + ph + 1);
        }
    }
#ifdef HY_WAIT_STATS
    if (tid == 0 && a.wstat) atomicMax(a.wstat + kWsLaunchBase + 2 * (a.launch_slot % kWsLaunches) + 1, global_ns());
#endif
}

}  // namespace hy
