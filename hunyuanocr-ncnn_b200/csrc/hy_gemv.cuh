// Streaming row GEMV for the decode step: y[m, n] = <xs[m, :], W[n, k_off : k_off + KP]>
// for the `rows` (<= MT) activation rows of one decoder step.
//
// This replaces ncnn's Gemm layers of the exported decoder (pnnx Linear,
// export/text_decoder_kv.py:64-69, 93-95; the Vulkan M=1 -> GEMV dispatch of
// patches/ncnn/0004-vulkan-gemm-m1.patch:78-114) and the LM head
// (export/export_lm_head.py:16-24) with the host token selection
// (src/text_runtime.cpp:730-797) fused into its epilogue.
//
// Layout: one CTA per SM owns a contiguous block of weight rows. A producer
// warp streams that block (contiguous in HBM) through a ring of shared-memory
// stages with cp.async.bulk, hinting L2 to evict it first; 8 consumer warps
// each take groups of RPW rows and dot them with the activation rows held in
// shared memory. The producer starts before griddepcontrol.wait, so under
// programmatic dependent launch the weight stream overlaps the tail of the
// previous kernel.
//
// Prologues: plain copy, RMSNorm (HunYuanDenseV1RMSNorm: w * (x * 1/sqrt(mean(x^2)+eps))),
// SwiGLU (silu(gate) * up), and embedding gather from the tied table (AR token,
// explicit ids, or the synthetic drafter), which also writes the residual stream.
// Epilogues: store, residual add (+ optional aux copy), penalised argmax with
// a last-CTA reduction and the AR / DFlash commit.
#pragma once

#include "hy_device.cuh"

#include <cuda.h>   // CUtensorMap (the map is encoded on the host through the driver entry point)

namespace hy {

enum { PRO_PLAIN = 0, PRO_NORM = 1, PRO_SWIGLU = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_ARGMAX = 2, EPI_ACT = 3 };   // EPI_ACT: M = 16 only
// SRC_GATHER_BLOCK: the DFlash draft's noise block [st->cur_token, mask_token x 15]
// (build_dflash_block, src/dflash_runtime.cpp:20-25).
enum { SRC_X = 0, SRC_GATHER_STATE = 1, SRC_GATHER_IDS = 2, SRC_GATHER_DRAFT = 3, SRC_GATHER_BLOCK = 4 };
// LM_BATCH: row m is the next token of the sequence in slot m (batched decode):
// per-row history bitmaps, per-slot commit.
enum { LM_NONE = 0, LM_AR = 1, LM_VERIFY = 2, LM_BATCH = 3 };

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = (kGemvWarps + 1) * 32;
constexpr int kStageBytes = 16384;
constexpr int kRingBytes = 96 * 1024;
constexpr int kSmemBudget = 225 * 1024;   // dynamic shared memory per CTA we allow ourselves
constexpr int kPartUnits16 = 32;          // M = 16 K-mode tile slots (units of one launch at most)

struct GemvArgs {
    const void* W;   // [N x ldw] of WT; this launch reads columns [k_off, k_off + KP)
    int N, ldw, k_off;
    int rows;        // active activation rows (<= MT)
    int src;         // SRC_*
    const float* x;  // SRC_X: row m at x + m * ldx + k_off; SwiGLU: interleaved (gate_k, up_k) pairs at x + m * ldx + 2 * (k_off + k)
    int ldx;
    const float* norm_w;
    float eps;
    const void* table;    // gather: tied embedding table [vocab x 1024] of WT
    const int* ids;       // SRC_GATHER_IDS
    DecodeState* st;
    const int* greedy;    // SRC_GATHER_DRAFT
    int vocab;
    int mask_token;       // SRC_GATHER_BLOCK
    int* ids_out;         // gather: CTA 0 writes the gathered ids
    float* x_store;       // gather: fp32 rows written to the residual stream [rows x 1024]
    float* out;           // STORE / RESID target, out[m * ldo + n]
    int ldo;
    const float* extra;   // RESID: out = out + (extra + dot) (second half of a K split)
    float* aux;           // RESID: optional copy of the result, aux[m * ld_aux + n]
    int ld_aux;
    int lm_mode;          // LM_*
    unsigned* hist;       // penalty history bitmap (read; updated by the commit)
    const int* prefix;    // row m also counts prefix[0..m] as history (nullable)
    float* logits;        // optional dump [rows x ldl]
    int ldl;
    float4* part;         // [gridDim.x * MT] per-CTA (raw max, raw idx, pen max, pen idx)
    int* counter;
    int* tok_out;         // LM_NONE: [rows]
    int* raw_out;
    int* log_tokens;      // LM_AR / LM_VERIFY token log
    int* log_raw;
    int* accept_log;
    int* posterior_out;   // LM_VERIFY [16]
    float penalty;        // LM_NONE penalty (AR / verify read st->penalty)
    int* err;
    SlotState* slots;     // LM_BATCH: per-row sequence state
    int* slot_cur;        // LM_BATCH: each row's next token (the next step's gather ids)
    int hist_stride;      // LM_BATCH: words between the rows' history bitmaps
    int log_stride;       // LM_BATCH: token-log entries per row
    // M = 16 LM head: tensor map of the tied table (128-row x 128-byte boxes, 128-byte swizzle).
    CUtensorMap tmap;
};

template <typename WT, int KP, int MT>
struct GemvShape {
    static constexpr int RPW = (MT == 1) ? 1 : 2;
    static constexpr int SEG = KP * static_cast<int>(sizeof(WT));
    static constexpr int SPS0 = kStageBytes / SEG;
    static constexpr int SPS = (SPS0 < RPW) ? RPW : (SPS0 / RPW) * RPW;
    static constexpr int STAGE = SPS * SEG;
    static constexpr int GPS = SPS / RPW;
    static constexpr int XS_BYTES = MT * KP * 4;
    static constexpr int RED_BYTES = (kGemvWarps * MT + MT) * 16 + 16;
    static constexpr int NST_RING = kRingBytes / STAGE;
    static constexpr int NST_FIT = (kSmemBudget - XS_BYTES - RED_BYTES - 512) / STAGE;
    static constexpr int NST = NST_RING < NST_FIT ? NST_RING : NST_FIT;
    static constexpr int BAR_OFF = XS_BYTES + NST * STAGE;
    static constexpr int RED_OFF = BAR_OFF + 2 * NST * 8;
    static constexpr int SMEM = RED_OFF + RED_BYTES;
    static constexpr int XP = KP;   // activation row pitch (floats)
    static constexpr int KC16 = KP;  // (M = 16 only)
    static constexpr int TL_NST = 2, TL_TILE = 0, TL_KC = 8, TL_BAR_OFF = 0, TL_RED_OFF = 0, SMEM_TL = 0;   // (M = 16 only)
};

// M = 16 (DFlash verify blocks, prefill chunks) on the tensor cores (mma.sync
// m16n8k8, tf32 with a three-term split, see tf32_mma3_split): the CTA's weight rows
// are cut into units of 8 rows x KC columns; a unit is one stage, its rows at a
// padded pitch (row chunk + 16 bytes) and the 16 activation rows likewise
// (pitch KP + 4 floats), so the fragment loads of a warp fall in 32 different
// banks. The unit is the B operand (n = weight row), the activation rows the A
// operand (m = activation row), one 16 x 8 tile per unit.
//   K mode (at most 32 units: q/k/v, o, gate/up, down): stage u = unit u =
//     (group u / NKC, chunk u % NKC), owned by warp u % 8; the units' tiles go to
//     shared memory and are added in chunk order at the end.
//   G mode (many row groups: the LM head): warp w owns groups w, w + 8,
//     ... and takes all NKC chunks of a group in order, accumulating in its
//     fragments; the stages of a round of 8 groups are interleaved chunk-major.
template <typename WT, int KP>
struct GemvShape<WT, KP, 16> {
    static constexpr int KC = (KP == 1024) ? 256 : KP / 8;   // columns per unit
    static constexpr int NKC = KP / KC;
    static constexpr int ROWB = KC * static_cast<int>(sizeof(WT));
    static constexpr int PITCH = ROWB + 16;
    static constexpr int STAGE = 8 * PITCH;
    static constexpr int XP = KP + 4;
    static constexpr int XS_BYTES = 16 * XP * 4;
    static constexpr int PART_UNITS = kPartUnits16;              // K-mode tile slots
    static constexpr int PART_BYTES = PART_UNITS * 16 * 8 * 4;   // [unit][m][n]
    static constexpr int WSCR_BYTES = kGemvWarps * 16 * 8 * 4;   // G-mode per-warp [m][n]
    static constexpr int RED_BYTES = (kGemvWarps * 16 + 16) * 16 + 16;
    static constexpr int NST_FIT = (kSmemBudget - XS_BYTES - PART_BYTES - WSCR_BYTES - RED_BYTES - 512) / STAGE;
    static constexpr int NST = NST_FIT >= 16 ? 16 : 8;   // slots: 2 or 1 per consumer warp
    static_assert(NST_FIT >= 8, "one slot per consumer warp must fit");
    static constexpr int PART_OFF = XS_BYTES + NST * STAGE;
    static constexpr int WSCR_OFF = PART_OFF + PART_BYTES;
    static constexpr int BAR_OFF = WSCR_OFF + WSCR_BYTES;
    static constexpr int RED_OFF = BAR_OFF + 2 * NST * 8;
    static constexpr int SMEM = RED_OFF + RED_BYTES;
    // LM head (argmax epilogue): tiles of 128 rows x 128 bytes fetched by one TMA
    // copy each (tensor map with 128-byte swizzle), ring aligned to 1 KB at run time.
    static constexpr int TL_ROWS = 128;
    static constexpr int TL_KC = 128 / static_cast<int>(sizeof(WT));   // columns per tile
    static constexpr int TL_TILE = TL_ROWS * 128;
    static constexpr int TL_NST = 8;
    static constexpr int TL_WSCR_OFF = XS_BYTES + 1024 + TL_NST * TL_TILE;
    static constexpr int TL_BAR_OFF = TL_WSCR_OFF + WSCR_BYTES;
    static constexpr int TL_RED_OFF = TL_BAR_OFF + 2 * TL_NST * 8;
    static constexpr int SMEM_TL = TL_RED_OFF + RED_BYTES;
    static_assert(KP != 1024 || SMEM_TL <= 227 * 1024, "LM head tile ring (the LM head has K = 1024)");
    // Names the generic code refers to.
    static constexpr int RPW = 8, SEG = ROWB, SPS = 8, GPS = 1, KC16 = KC;
    static_assert(KP % KC == 0 && KC % 8 == 0 && ROWB % 16 == 0, "unit geometry");
};

struct Unit16 {
    int g, c, w, j;   // row group, column chunk, owner warp, index among the owner's units
};

__device__ __forceinline__ Unit16 unit16_of(int s, int ngroups, int nkc, bool kmode)
{
    if (kmode) return Unit16{s / nkc, s % nkc, s % kGemvWarps, s / kGemvWarps};
    const int per_round = nkc * kGemvWarps;
    const int r = s / per_round;   // every round before the last is full
    const int aw = min(kGemvWarps, ngroups - kGemvWarps * r);
    const int i = s - r * per_round;
    const int w = i % aw;
    return Unit16{kGemvWarps * r + w, i / aw, w, r * nkc + i / aw};
}

// d += A(x) * B(w) for one m16n8k8 tf32 tile with fp32-level accuracy: the
// operands are split into a tf32 head (mantissa truncated to 10 bits) and the
// fp32 remainder, and the three products head*head + lo*head + head*lo are
// accumulated (lo*lo, ~2^-22 relative, is dropped). With bf16 weights the
// weight head is exact and its remainder is zero (two products).
__device__ __forceinline__ unsigned tf32_head(float v) { return __float_as_uint(v) & 0xFFFFE000u; }

__device__ __forceinline__ void mma_tf32(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The three products go to three accumulators (lo.hi, hi.lo, hi.hi), so
// consecutive MMAs do not wait on each other; the caller adds them.
template <bool W_EXACT>
__device__ __forceinline__ void tf32_mma3_split(float (&d)[3][4], const float (&x)[4], float w0, float w1)
{
    unsigned ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        ah[i] = tf32_head(x[i]);
        al[i] = __float_as_uint(x[i] - __uint_as_float(ah[i]));
    }
    const unsigned bh0 = tf32_head(w0), bh1 = tf32_head(w1);
    mma_tf32(d[0], al, bh0, bh1);
    if constexpr (!W_EXACT)
    {
        const unsigned bl0 = __float_as_uint(w0 - __uint_as_float(bh0));
        const unsigned bl1 = __float_as_uint(w1 - __uint_as_float(bh1));
        mma_tf32(d[1], ah, bl0, bl1);
    }
    mma_tf32(d[2], ah, bh0, bh1);
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

struct ArgBest {
    float rv;
    int ri;
    float pv;
    int pi;
};

__device__ __forceinline__ void best_update(float& bv, int& bi, float v, int i)
{
    if (bi < 0 || v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__device__ __forceinline__ bool is_eos(const DecodeState* st, int tok)
{
    bool e = false;
    for (int i = 0; i < st->n_eos && i < kMaxEos; ++i) e |= (st->eos[i] == tok);
    return e;
}

// Synthetic drafter: slot i of the current block (see hy_decode.h).
__device__ __forceinline__ int draft_id(const DecodeState* st, const int* greedy, int vocab, int i)
{
    if (i == 0) return st->cur_token;
    const unsigned long long h = splitmix64(st->draft_base + 16ull * static_cast<unsigned long long>(st->block_count) + i);
    const float u = static_cast<float>(h >> 40) * 5.9604644775390625e-08f;  // 2^-24
    const int j = st->n_gen + i;
    if (u < st->draft_p && j < st->n_greedy) return greedy[j];
    return static_cast<int>((h & 0xFFFFFFFFull) % static_cast<unsigned long long>(vocab));
}

// The elements of a 16-byte chunk as floats (4 fp32 or 8 bf16, little-endian lanes).
template <typename WT>
__device__ __forceinline__ void unpack_chunk(const uint4& c, float* out)
{
    const unsigned w[4] = {c.x, c.y, c.z, c.w};
    if constexpr (sizeof(WT) == 4)
    {
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = __uint_as_float(w[i]);
    }
    else
    {
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
}

template <typename WT, int KP, int MT, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, (MT == 1) ? 2 : 1) gemv_kernel(const __grid_constant__ GemvArgs a)
{
    using S = GemvShape<WT, KP, MT>;
    constexpr int RPW = S::RPW, SEG = S::SEG, SPS = S::SPS, STAGE = S::STAGE, NST = S::NST;
    constexpr int XP = S::XP;   // activation row pitch in shared memory
    static_assert(NST >= 2, "ring too small");
    static_assert(S::GPS <= kGemvWarps, "a warp may own at most one row group per stage");
    static_assert(SEG % 16 == 0, "segments must be 16-byte multiples");
    static_assert(KP % 128 == 0, "K slice must be a multiple of 128");

    // M = 16 LM head: 64-row tiles by TMA (see GemvShape<WT, KP, 16>).
    constexpr bool TL = (MT == 16 && EPI == EPI_ARGMAX);
    constexpr int NS = TL ? S::TL_NST : NST;
    extern __shared__ __align__(128) unsigned char smem[];
    float* xs = reinterpret_cast<float*>(smem);
    unsigned char* ring = smem + S::XS_BYTES;
    if constexpr (TL) ring += (1024u - (smem_u32(ring) & 1023u)) & 1023u;   // 128-byte swizzle wants 1 KB alignment
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (TL ? S::TL_BAR_OFF : S::BAR_OFF));
    uint64_t* empty = full + NS;
    float4* red4 = reinterpret_cast<float4*>(smem + (TL ? S::TL_RED_OFF : S::RED_OFF));   // [8 warps][MT] trackers, [MT] merged
    int* redi = reinterpret_cast<int*>(red4 + kGemvWarps * MT + MT);  // last-CTA flag

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    HY_STEP_TRACE_OPEN(0x100000000ull | (static_cast<unsigned long long>(MT) << 24) | ((KP / 128) << 8) | (PRO << 4) | EPI);
    // EPI_ACT pairs rows (2j = gate_j, 2j+1 = up_j): split the rows by pairs.
    const int unit = (EPI == EPI_ACT) ? 2 : 1;
    const int r0 = unit * static_cast<int>(static_cast<long long>(a.N / unit) * b / G);
    const int r1 = unit * static_cast<int>(static_cast<long long>(a.N / unit) * (b + 1) / G);
    const int R = r1 - r0;
    // M = 16: row groups of 8, K mode when all units fit the tile slots.
    const int ngroups16 = (R + 7) / 8;
    const bool kmode16 = (MT == 16) && ngroups16 * (KP / S::KC16) <= kPartUnits16;
    const int nk_tl = KP / S::TL_KC;                    // TL: tiles per 64-row block
    const int nstage = TL ? ((R + 127) / 128) * nk_tl : (MT == 16) ? ngroups16 * (KP / S::KC16) : (R + SPS - 1) / SPS;

    __shared__ uint64_t s_xbar;   // M = 16: bulk copy of the activation rows
#ifdef HY_STEP_TRACE
    __shared__ unsigned long long* s_str;   // CTA 0's record, for every warp
    if (tid == 0) s_str = hy_str_;
#endif
    if (tid == 0)
    {
        for (int s = 0; s < NS; ++s)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], (MT == 16 && !TL) ? 1 : kGemvWarps);
        }
        mbar_init(&s_xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kGemvWarps)
    {
        // ---------------- producer ----------------
        if (lane == 0)
        {
            const uint64_t pol = l2_evict_first_policy();
            const WT* W = static_cast<const WT*>(a.W);
            int issued = 0;
            if constexpr (TL)
            {
                // One TMA copy per tile: rows r0 + 128 rb .., columns k_off + TL_KC kc ..
                // (rows past the table are zero-filled by the copy).
                for (int i = 0; i < nstage; ++i)
                {
                    const int slot = i % NS;
                    if (i >= NS && !mbar_wait(&empty[slot], ((i / NS) - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                    const int rb = i / nk_tl, kc = i % nk_tl;
                    mbar_arrive_expect_tx(&full[slot], S::TL_TILE);
                    tma_load_2d(ring + slot * S::TL_TILE, &a.tmap, a.k_off + kc * S::TL_KC, r0 + 128 * rb, &full[slot]);
                    issued = i + 1;
                }
                for (int i = (issued > NS ? issued - NS : 0); i < issued; ++i)
                    mbar_wait(&full[i % NS], (i / NS) & 1, a.err, kErrTimeoutFull);
                return;
            }
            int fills[(MT == 16) ? NST : 1] = {};   // M = 16: copies issued into each slot
            for (int i = 0; i < nstage; ++i)
            {
                const int slot = i % NST;
                if (MT != 16 && i >= NST && !mbar_wait(&empty[slot], ((i / NST) - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                unsigned char* dst = ring + slot * STAGE;
                if constexpr (MT == 16)
                {
                    // Unit (g, c): up to 8 row chunks of S::ROWB bytes at the padded pitch,
                    // into the next of its owner warp's slots.
                    const Unit16 u = unit16_of(i, ngroups16, S::NKC, kmode16);
                    constexpr int SPW = NST / kGemvWarps;
                    const int ws = u.w * SPW + u.j % SPW;
                    if (u.j >= SPW && !mbar_wait(&empty[ws], ((u.j / SPW) - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                    fills[ws] += 1;
                    dst = ring + ws * STAGE;
                    const int slot = ws;
                    const int gr0 = r0 + 8 * u.g;
                    const int nr = min(8, r1 - gr0);
                    mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nr * S::ROWB));
                    for (int j = 0; j < nr; ++j)
                        bulk_g2s(dst + j * S::PITCH, W + static_cast<size_t>(gr0 + j) * a.ldw + a.k_off + u.c * S::KC,
                                 S::ROWB, &full[slot], pol);
                    issued = i + 1;
                    continue;
                }
                const int sr0 = r0 + i * SPS;
                const int nseg = min(SPS, r1 - sr0);
                mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nseg * SEG));
                if (a.ldw == KP)
                {
                    bulk_g2s(dst, W + static_cast<size_t>(sr0) * KP, static_cast<uint32_t>(nseg * SEG), &full[slot], pol);
                }
                else
                {
                    for (int j = 0; j < nseg; ++j)
                        bulk_g2s(dst + j * SEG, W + static_cast<size_t>(sr0 + j) * a.ldw + a.k_off, SEG, &full[slot], pol);
                }
                issued = i + 1;
            }
            // Drain: never leave the CTA with copies in flight.
            if constexpr (MT == 16)
            {
                for (int ws = 0; ws < NST; ++ws)
                    if (fills[ws] > 0) mbar_wait(&full[ws], (fills[ws] - 1) & 1, a.err, kErrTimeoutFull);
            }
            else
            {
                for (int i = (issued > NST ? issued - NST : 0); i < issued; ++i)
                    mbar_wait(&full[i % NST], (i / NST) & 1, a.err, kErrTimeoutFull);
            }
        }
        return;
    }

    // ---------------- consumers (256 threads) ----------------
    // M = 16 RMSNorm: the norm weights of this lane's columns (k = 4 lane + 128 i;
    // constants) are loaded before the wait.
    float4 nwr[(MT == 16 && PRO == PRO_NORM) ? KP / 128 : 1];
    if constexpr (MT == 16 && PRO == PRO_NORM)
    {
#pragma unroll
        for (int i = 0; i < KP / 128; ++i)
            nwr[i] = __ldg(reinterpret_cast<const float4*>(a.norm_w + a.k_off + 4 * lane + 128 * i));
    }
    pdl_wait();
    HY_STEP_TRACE_MARK(2);

    __shared__ int s_ids[kMaxStepRows];
    __shared__ float s_rinv[kMaxStepRows];
    __shared__ int s_prefix[kMaxStepRows];
    const int rows = a.rows;

    // Source row ids for gathers.
    if (a.src != SRC_X)
    {
        if (tid < MT)
        {
            int id = 0;
            if (tid < rows)
            {
                if (a.src == SRC_GATHER_STATE) id = a.st->cur_token;
                else if (a.src == SRC_GATHER_IDS) id = a.ids[tid];
                else if (a.src == SRC_GATHER_BLOCK) id = (tid == 0) ? a.st->cur_token : a.mask_token;
                else id = draft_id(a.st, a.greedy, a.vocab, tid);
                if (id < 0 || id >= a.vocab)
                {
                    atomicOr(a.err, kErrBounds);
                    id = 0;
                }
                if (b == 0 && a.ids_out) a.ids_out[tid] = id;
            }
            s_ids[tid] = id;
        }
    }
    if (EPI == EPI_ARGMAX && tid < MT) s_prefix[tid] = (a.prefix && tid < rows) ? a.prefix[tid] : -1;
    // M = 16 argmax: the penalty-history words of this CTA's rows, read once.
    constexpr int kHistWords16 = 64;
    __shared__ unsigned s_hist[(MT == 16 && EPI == EPI_ARGMAX) ? kHistWords16 : 1];
    const bool hist_s_ok = (MT == 16 && EPI == EPI_ARGMAX) && a.hist_stride == 0 && R > 0 &&
                           ((r1 - 1) >> 5) - (r0 >> 5) < kHistWords16;
    if (hist_s_ok && tid <= ((r1 - 1) >> 5) - (r0 >> 5)) s_hist[tid] = a.hist[(r0 >> 5) + tid];
    consumers_sync();

    // Stage the activation rows (fp32) in shared memory.
    if constexpr (MT == 16)
    {
        // Batches of rows with every load of a batch in flight before its
        // stores (one L2 round trip per batch instead of per row).
        constexpr int KI = (KP + 1023) / 1024;            // float4 columns per thread and row
        constexpr int B = 8;                              // rows per batch
        const bool bulk = (a.src == SRC_X && PRO != PRO_SWIGLU);
        if (bulk)
        {
            // Plain / normed rows: one bulk copy per row, the padding rows zeroed.
            if (tid == 0)
            {
                mbar_arrive_expect_tx(&s_xbar, static_cast<uint32_t>(rows * KP * 4));
                for (int m = 0; m < rows; ++m)
                    bulk_g2s_plain(xs + m * XP, a.x + static_cast<size_t>(m) * a.ldx + a.k_off, KP * 4, &s_xbar);
            }
            for (int i = tid; i < (MT - rows) * (XP / 4); i += 256)
                reinterpret_cast<float4*>(xs + rows * XP)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            mbar_wait(&s_xbar, 0, a.err, kErrTimeoutFull);
        }
        for (int m0 = 0; m0 < MT && !bulk; m0 += B)
        {
            float4 p0[B][KI], p1[B][KI];
#pragma unroll
            for (int mm = 0; mm < B; ++mm)
#pragma unroll
                for (int i = 0; i < KI; ++i)
                {
                    const int m = m0 + mm, k = tid * 4 + 1024 * i;
                    p0[mm][i] = p1[mm][i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (m >= rows || k >= KP) continue;
                    if (a.src != SRC_X)
                        p0[mm][i] = load4(static_cast<const WT*>(a.table) + static_cast<size_t>(s_ids[m]) * kHidden + k);
                    else if (PRO == PRO_SWIGLU)
                    {
                        const float* gu = a.x + static_cast<size_t>(m) * a.ldx + 2 * a.k_off;
                        p0[mm][i] = *reinterpret_cast<const float4*>(gu + 2 * k);
                        p1[mm][i] = *reinterpret_cast<const float4*>(gu + 2 * k + 4);
                    }
                    else
                        p0[mm][i] = *reinterpret_cast<const float4*>(a.x + static_cast<size_t>(m) * a.ldx + a.k_off + k);
                }
#pragma unroll
            for (int mm = 0; mm < B; ++mm)
#pragma unroll
                for (int i = 0; i < KI; ++i)
                {
                    const int m = m0 + mm, k = tid * 4 + 1024 * i;
                    if (k >= KP) continue;
                    float4 r = p0[mm][i];
                    if (a.src == SRC_X && PRO == PRO_SWIGLU && m < rows)
                    {
                        // act_k = silu(gate_k) * up_k; the gate/up projection rows are interleaved.
                        const float4 q0 = p0[mm][i], q1 = p1[mm][i];
                        r.x = (q0.x / (1.0f + expf(-q0.x))) * q0.y;
                        r.y = (q0.z / (1.0f + expf(-q0.z))) * q0.w;
                        r.z = (q1.x / (1.0f + expf(-q1.x))) * q1.y;
                        r.w = (q1.z / (1.0f + expf(-q1.z))) * q1.w;
                    }
                    *reinterpret_cast<float4*>(xs + m * XP + k) = r;
                }
        }
    }
    else
    for (int m = 0; m < MT; ++m)
    {
        float* xr = xs + m * KP;
        if (m >= rows)
        {
            for (int k = tid * 4; k < KP; k += 256 * 4) *reinterpret_cast<float4*>(xr + k) = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        if (a.src != SRC_X)
        {
            const WT* trow = static_cast<const WT*>(a.table) + static_cast<size_t>(s_ids[m]) * kHidden;
            for (int k = tid * 4; k < KP; k += 256 * 4)
            {
                const float4 v = load4(trow + k);
                *reinterpret_cast<float4*>(xr + k) = v;
            }
        }
        else if (PRO == PRO_SWIGLU)
        {
            // act_k = silu(gate_k) * up_k; the gate/up projection rows are interleaved.
            const float* gu = a.x + static_cast<size_t>(m) * a.ldx + 2 * a.k_off;
            for (int k = tid * 4; k < KP; k += 256 * 4)
            {
                const float4 p0 = *reinterpret_cast<const float4*>(gu + 2 * k);
                const float4 p1 = *reinterpret_cast<const float4*>(gu + 2 * k + 4);
                float4 r;
                r.x = (p0.x / (1.0f + expf(-p0.x))) * p0.y;
                r.y = (p0.z / (1.0f + expf(-p0.z))) * p0.w;
                r.z = (p1.x / (1.0f + expf(-p1.x))) * p1.y;
                r.w = (p1.z / (1.0f + expf(-p1.z))) * p1.w;
                *reinterpret_cast<float4*>(xr + k) = r;
            }
        }
        else
        {
            const float* xp = a.x + static_cast<size_t>(m) * a.ldx + a.k_off;
            for (int k = tid * 4; k < KP; k += 256 * 4)
                *reinterpret_cast<float4*>(xr + k) = *reinterpret_cast<const float4*>(xp + k);
        }
    }
    consumers_sync();

    // Gather: publish the embedding rows as the residual stream (CTA slices).
    if (a.src != SRC_X && a.x_store)
    {
        const int total = rows * kHidden;
        const int per = (total + G - 1) / G;
        const int beg = b * per, end = min(total, beg + per);
        for (int i = beg + tid; i < end; i += 256) a.x_store[i] = xs[(i / kHidden) * XP + (i % kHidden)];
        // The RMSNorm below rewrites xs in place: every raw value is read first.
        if (PRO == PRO_NORM) consumers_sync();
    }

    if (PRO == PRO_NORM && MT == 16)
    {
        // One pass (warp w: rows w and w + 8): xs = w * x and the row's
        // 1/sqrt(mean(x^2) + eps), which the epilogue applies to the row's dot
        // products (group_epilogue): the RMSNorm's per-row scale commutes with the
        // projection, so the units need not wait for it.
        for (int m = warp; m < MT; m += kGemvWarps)
        {
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < KP / 128; ++i)
            {
                float4* p = reinterpret_cast<float4*>(xs + m * XP + 4 * lane + 128 * i);
                float4 v = *p;
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                v.x *= nwr[i].x;
                v.y *= nwr[i].y;
                v.z *= nwr[i].z;
                v.w *= nwr[i].w;
                *p = v;
            }
            ss = warp_sum(ss);
            if (lane == 0) s_rinv[m] = 1.0f / sqrtf(ss / static_cast<float>(KP) + a.eps);
        }
        consumers_sync();
    }
    else if (PRO == PRO_NORM)
    {
        // Per-row 1/sqrt(mean(x^2) + eps), then xs = w * (x * rinv).
        float* wsum = reinterpret_cast<float*>(red4);   // [8 warps][MT]
        for (int m = 0; m < MT; ++m)
        {
            float ss = 0.f;
            for (int k = tid * 4; k < KP; k += 256 * 4)
            {
                const float4 v = *reinterpret_cast<const float4*>(xs + m * KP + k);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) wsum[warp * MT + m] = ss;
        }
        consumers_sync();
        if (tid < MT)
        {
            float t = 0.f;
            for (int w = 0; w < kGemvWarps; ++w) t += wsum[w * MT + tid];
            s_rinv[tid] = 1.0f / sqrtf(t / static_cast<float>(KP) + a.eps);
        }
        consumers_sync();
        for (int m = 0; m < rows; ++m)
        {
            const float ri = s_rinv[m];
            for (int k = tid * 4; k < KP; k += 256 * 4)
            {
                float4 v = *reinterpret_cast<float4*>(xs + m * KP + k);
                const float4 w = *reinterpret_cast<const float4*>(a.norm_w + a.k_off + k);
                v.x = w.x * (v.x * ri);
                v.y = w.y * (v.y * ri);
                v.z = w.z * (v.z * ri);
                v.w = w.w * (v.w * ri);
                *reinterpret_cast<float4*>(xs + m * KP + k) = v;
            }
        }
        consumers_sync();
    }

    HY_STEP_TRACE_MARK(3);
    pdl_launch();

    // ---------------- main loop ----------------
    const float pen = (EPI == EPI_ARGMAX) ? ((a.lm_mode == LM_NONE) ? a.penalty : a.st->penalty) : 1.0f;
    ArgBest best;
    best.rv = 0.f; best.ri = -1; best.pv = 0.f; best.pi = -1;
    // M = 1: every consumer warp observes every stage in order and arrives once
    // on it; the warp owning a row group of the stage (group gi -> warp gi % 8)
    // computes it before arriving. (An mbarrier parity wait is only meaningful
    // one phase ahead, so no warp may skip past a stage that has not landed, nor
    // let a slot be reused before it has seen it.) M = 16: each warp has slots
    // of its own and waits only on those.
    if constexpr (MT == 16)
    {
        constexpr int NKC = S::NKC, KC = S::KC, PITCH = S::PITCH;
        constexpr bool W_EXACT = sizeof(WT) == 2;   // bf16 weights are exact tf32 heads
        float* part = reinterpret_cast<float*>(smem + S::PART_OFF);                 // [unit][m][n]
        float* wscr = reinterpret_cast<float*>(smem + (TL ? S::TL_WSCR_OFF : S::WSCR_OFF)) + warp * 128;   // [m][n]
        const int g8 = lane >> 2, t4 = lane & 3;
        float d[4];
        // Tile of the unit in `slot` (chunk c): d += x[0:16, chunk] * W[8 rows, chunk]^T.
        // Six accumulator chains (the three split products x even / odd k-steps),
        // added at the end, so consecutive MMAs of a unit do not wait on each other
        // (a warp's MMA time per unit fell by a quarter; the launch's time is set by
        // when its later weight units arrive).
        auto unit_mma = [&](int slot, int c) {
            const WT* wr = reinterpret_cast<const WT*>(ring + slot * STAGE + g8 * PITCH);
            const float* x0 = xs + g8 * XP + c * KC + t4;
            const float* x1 = x0 + 8 * XP;
            float acc[2][3][4];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int i = 0; i < 3; ++i) acc[h][i][0] = acc[h][i][1] = acc[h][i][2] = acc[h][i][3] = 0.f;
#pragma unroll 4
            for (int k8 = 0; k8 < KC / 8; ++k8)
            {
                const float xa[4] = {x0[8 * k8], x1[8 * k8], x0[8 * k8 + 4], x1[8 * k8 + 4]};
                const float w0 = to_f32<WT>(wr[8 * k8 + t4]), w1 = to_f32<WT>(wr[8 * k8 + t4 + 4]);
                tf32_mma3_split<W_EXACT>(acc[k8 & 1], xa, w0, w1);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e)
                d[e] += (acc[0][2][e] + acc[1][2][e]) + ((acc[0][0][e] + acc[1][0][e]) + (acc[0][1][e] + acc[1][1][e]));
        };
        // Store / residual / argmax epilogue of one output (row n of activation row m).
        // pm (argmax): bit j set when the block prefix's id j is n (see group_epilogue).
        auto emit = [&](int m, int n, float v, unsigned pm = 0u) {
            if (EPI == EPI_STORE || EPI == EPI_RESID)
            {
                const size_t o = static_cast<size_t>(m) * a.ldo + n;
                if (EPI == EPI_RESID)
                {
                    if (a.extra) v = a.extra[o] + v;
                    v = a.out[o] + v;
                    if (a.aux) a.aux[static_cast<size_t>(m) * a.ld_aux + n] = v;
                }
                a.out[o] = v;
            }
            else
            {
                if (a.logits) a.logits[static_cast<size_t>(m) * a.ldl + n] = v;
                const unsigned hw = a.hist_stride ? a.hist[static_cast<size_t>(m) * a.hist_stride + (n >> 5)]
                                    : hist_s_ok     ? s_hist[(n >> 5) - (r0 >> 5)]
                                                    : a.hist[n >> 5];
                // History of row m: the block's earlier rows plus its prefix ids 0..m.
                const bool hit = ((hw >> (n & 31)) & 1u) || (pm & ((2u << m) - 1u)) != 0u;
                const float ps = hit ? (v < 0.0f ? v * pen : v / pen) : v;
                if (best.ri < 0 || v > best.rv) { best.rv = v; best.ri = n; }
                if (best.pi < 0 || ps > best.pv) { best.pv = ps; best.pi = n; }
            }
        };
        // Epilogue of a finished 8-row group from its [m][n] tile (times the
        // activation row's RMSNorm scale when the prologue normalised).
        auto tval = [&](const float* tile, int m, int row) {
            const float v = tile[m * 8 + row];
            if constexpr (PRO == PRO_NORM) return v * s_rinv[m];
            else return v;
        };
        auto group_epilogue = [&](const float* tile, int g) {
            const int n0 = r0 + 8 * g;
            const int nr = min(8, R - 8 * g);
            if (EPI == EPI_ARGMAX)
            {
                // Lanes m and m + 16 take activation row m, the first for the group's
                // rows 0-3, the second for rows 4-7 (their trackers are merged before
                // the reduction); which prefix ids equal vocab row n is found once per
                // n by a ballot over the (at most 16) prefix entries.
                const int m = lane & 15, half = lane >> 4;
                const int pid = s_prefix[m];
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4)
                {
                    const unsigned pm0 = __ballot_sync(0xffffffffu, half == 0 && pid == n0 + r4);
                    const unsigned pm1 = __ballot_sync(0xffffffffu, half == 0 && pid == n0 + 4 + r4);
                    const int row = 4 * half + r4;
                    if (row < nr && m < rows) emit(m, n0 + row, tval(tile, m, row), half ? pm1 : pm0);
                }
            }
            else if (EPI == EPI_ACT)
            {
                // act[m][j] = silu(gate_j) * up_j for the row pairs (n0 is even).
                for (int p = lane; p < 16 * 4; p += 32)
                {
                    const int m = p >> 2, pr = p & 3;
                    if (2 * pr + 1 < nr && m < rows)
                    {
                        const float gt = tval(tile, m, 2 * pr), up = tval(tile, m, 2 * pr + 1);
                        a.out[static_cast<size_t>(m) * a.ldo + ((n0 >> 1) + pr)] = (gt / (1.0f + expf(-gt))) * up;
                    }
                }
            }
            else if (EPI == EPI_RESID)
            {
                // The lane's 4 outputs: every residual (and first-half) load is issued
                // before the first store, one L2 round trip instead of one per output.
                float old[4], ext[4];
#pragma unroll
                for (int it = 0; it < 4; ++it)
                {
                    const int p = lane + 32 * it, m = p >> 3, row = p & 7;
                    old[it] = ext[it] = 0.f;
                    if (row < nr && m < rows)
                    {
                        const size_t o = static_cast<size_t>(m) * a.ldo + n0 + row;
                        old[it] = a.out[o];
                        if (a.extra) ext[it] = a.extra[o];
                    }
                }
#pragma unroll
                for (int it = 0; it < 4; ++it)
                {
                    const int p = lane + 32 * it, m = p >> 3, row = p & 7;
                    if (row < nr && m < rows)
                    {
                        const size_t o = static_cast<size_t>(m) * a.ldo + n0 + row;
                        float v = tval(tile, m, row);
                        if (a.extra) v = ext[it] + v;
                        v = old[it] + v;
                        if (a.aux) a.aux[static_cast<size_t>(m) * a.ld_aux + n0 + row] = v;
                        a.out[o] = v;
                    }
                }
            }
            else
            {
                for (int p = lane; p < 16 * 8; p += 32)
                {
                    const int m = p >> 3, row = p & 7;
                    if (row < nr && m < rows) emit(m, n0 + row, tval(tile, m, row));
                }
            }
        };
        if constexpr (TL)
        {
            // Every warp reads every tile (rows 16 w .. 16 w + 15 of its 128: two 8-row MMA
            // tiles sharing each activation fragment) and arrives on it; a row block's tiles
            // come in column order, so the accumulators run across them.
            // Element k of tile row r sits in 16-byte chunk (k * size / 16) ^ (r & 7).
            // Three accumulators per 8-row tile (lo.hi, hi.lo, hi.hi products), added at readout.
            float acc3[2][3][4];
            for (int stage = 0; stage < nstage; ++stage)
            {
                const int slot = stage % NS;
                const bool ok = mbar_wait(&full[slot], (stage / NS) & 1, a.err, kErrTimeoutFull);
                if (!__all_sync(0xffffffffu, ok)) break;
                const int rb = stage / nk_tl, kc = stage % nk_tl;
                if (kc == 0)
                {
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int i = 0; i < 3; ++i) acc3[h][i][0] = acc3[h][i][1] = acc3[h][i][2] = acc3[h][i][3] = 0.f;
                }
                // The tile's k order is permuted so that each thread's operands are
                // contiguous: in k-step kk, logical k = t4 is column t4 * SPAN + 2 kk and
                // logical k = t4 + 4 is the column after it (A and B alike, so the sum
                // over k is unchanged). A thread then reads its SPAN activation columns of
                // rows g8 and g8 + 8 and its SPAN weights of each tile row with 16-byte loads
                // (the weights are two swizzled 16-byte chunks, 2 t4 and 2 t4 + 1).
                constexpr int NKK = S::TL_KC / 8;   // k-steps per tile
                constexpr int SPAN = 2 * NKK;       // columns per thread
                const float* x0 = xs + g8 * XP + kc * S::TL_KC + t4 * SPAN;
                const float* x1 = x0 + 8 * XP;
                float xv0[SPAN], xv1[SPAN];
#pragma unroll
                for (int i = 0; i < SPAN; i += 4)
                {
                    const float4 u0 = *reinterpret_cast<const float4*>(x0 + i);
                    const float4 u1 = *reinterpret_cast<const float4*>(x1 + i);
                    xv0[i] = u0.x; xv0[i + 1] = u0.y; xv0[i + 2] = u0.z; xv0[i + 3] = u0.w;
                    xv1[i] = u1.x; xv1[i + 1] = u1.y; xv1[i + 2] = u1.z; xv1[i + 3] = u1.w;
                }
                float wv[2][SPAN];
#pragma unroll
                for (int h = 0; h < 2; ++h)
                {
                    const int r = 16 * warp + 8 * h + g8;   // tile row; r & 7 == g8
                    const unsigned char* trow = ring + slot * S::TL_TILE + r * 128;
                    const uint4 c0 = *reinterpret_cast<const uint4*>(trow + (((2 * t4) ^ g8) << 4));
                    const uint4 c1 = *reinterpret_cast<const uint4*>(trow + (((2 * t4 + 1) ^ g8) << 4));
                    unpack_chunk<WT>(c0, wv[h]);
                    unpack_chunk<WT>(c1, wv[h] + SPAN / 2);
                }
#pragma unroll
                for (int kk = 0; kk < NKK; ++kk)
                {
                    const float xa[4] = {xv0[2 * kk], xv1[2 * kk], xv0[2 * kk + 1], xv1[2 * kk + 1]};
                    unsigned ah[4], al[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                    {
                        ah[i] = tf32_head(xa[i]);
                        al[i] = __float_as_uint(xa[i] - __uint_as_float(ah[i]));
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                    {
                        const float w0 = wv[h][2 * kk], w1 = wv[h][2 * kk + 1];
                        const unsigned bh0 = tf32_head(w0), bh1 = tf32_head(w1);
                        mma_tf32(acc3[h][0], al, bh0, bh1);
                        if constexpr (!W_EXACT)
                            mma_tf32(acc3[h][1], ah, __float_as_uint(w0 - __uint_as_float(bh0)),
                                     __float_as_uint(w1 - __uint_as_float(bh1)));
                        mma_tf32(acc3[h][2], ah, bh0, bh1);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                if (kc == nk_tl - 1)
                {
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                    {
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[e] = acc3[h][2][e] + (acc3[h][0][e] + acc3[h][1][e]);
                        wscr[g8 * 8 + 2 * t4] = d[0];
                        wscr[g8 * 8 + 2 * t4 + 1] = d[1];
                        wscr[(g8 + 8) * 8 + 2 * t4] = d[2];
                        wscr[(g8 + 8) * 8 + 2 * t4 + 1] = d[3];
                        __syncwarp();
                        group_epilogue(wscr, rb * 16 + 2 * warp + h);
                        __syncwarp();
                    }
                }
            }
        }
        else
        {
        // This warp's own units, in order, from its own slots (each refilled by the
        // producer once this warp released it, so every wait is one phase ahead).
        constexpr int SPW = NST / kGemvWarps;
        int jown = 0;
#ifdef HY_STEP_TRACE
        unsigned long long st_wait = 0, st_mma = 0;   // thread 0: ns waiting for its units / in their MMAs
#endif
        for (int stage = 0; stage < nstage; ++stage)
        {
            const Unit16 u = unit16_of(stage, ngroups16, NKC, kmode16);
            if (u.w != warp) continue;
            const int slot = warp * SPW + jown % SPW;
#ifdef HY_STEP_TRACE
            const unsigned long long sw0 = global_ns();
#endif
            const bool ok = mbar_wait(&full[slot], (jown / SPW) & 1, a.err, kErrTimeoutFull);
            ++jown;
            if (!__all_sync(0xffffffffu, ok)) break;
            if (kmode16 || u.c == 0) d[0] = d[1] = d[2] = d[3] = 0.f;
#ifdef HY_STEP_TRACE
            const unsigned long long sw1 = global_ns();
            st_wait += sw1 - sw0;
#endif
            unit_mma(slot, u.c);
#ifdef HY_STEP_TRACE
            __syncwarp();
            st_mma += global_ns() - sw1;
#endif
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            // Tile element (m, n): d0 (g8, 2 t4), d1 (g8, 2 t4 + 1), d2 (g8 + 8, 2 t4), d3 (g8 + 8, 2 t4 + 1).
            float* tile = kmode16 ? part + stage * 128 : wscr;
            if (kmode16 || u.c == NKC - 1)
            {
                tile[g8 * 8 + 2 * t4] = d[0];
                tile[g8 * 8 + 2 * t4 + 1] = d[1];
                tile[(g8 + 8) * 8 + 2 * t4] = d[2];
                tile[(g8 + 8) * 8 + 2 * t4 + 1] = d[3];
            }
            if (!kmode16 && u.c == NKC - 1)
            {
                __syncwarp();
                group_epilogue(wscr, u.g);
                __syncwarp();
            }
        }
#ifdef HY_STEP_TRACE
        if (hy_str_)
        {
            hy_str_[5] = st_wait;
            hy_str_[6] = st_mma;
            hy_str_[7] = global_ns();
        }
        if (s_str && lane == 0)
        {
            s_str[9 + warp] = global_ns();   // this warp's last unit done
            s_str[17 + warp] = st_wait;      // and its waits for units
        }
#endif
        if (kmode16)
        {
            // Add the units' tiles in chunk order and run the epilogue.
            consumers_sync();
            float* sum = reinterpret_cast<float*>(smem + S::PART_OFF);   // group g's sum overwrites unit g*NKC
            for (int e = tid; e < ngroups16 * 128; e += 256)
            {
                const int g = e >> 7, i = e & 127;
                float v = 0.f;
                for (int c = 0; c < NKC; ++c) v += part[(g * NKC + c) * 128 + i];
                sum[(g * NKC) * 128 + i] = v;
            }
            consumers_sync();
            for (int g = warp; g < ngroups16; g += kGemvWarps) group_epilogue(sum + (g * NKC) * 128, g);
        }
        }
    }
    else
    {
        const int ngroups = (R + RPW - 1) / RPW;
        int gi = warp;   // next group this warp owns
        for (int stage = 0; stage < nstage; ++stage)
        {
            const int slot = stage % NST;
            const bool ok = mbar_wait(&full[slot], (stage / NST) & 1, a.err, kErrTimeoutFull);
            if (!__all_sync(0xffffffffu, ok)) break;
            const int seg0 = gi * RPW;
            const bool mine = gi < ngroups && seg0 < (stage + 1) * SPS;   // at most one group per warp per stage
            const int nr = mine ? min(RPW, R - seg0) : 0;
            float acc[RPW][MT];
    #pragma unroll
            for (int r = 0; r < RPW; ++r)
    #pragma unroll
                for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
            if (mine)
            {
                const WT* wrow = reinterpret_cast<const WT*>(ring + slot * STAGE + (seg0 % SPS) * SEG);
    #pragma unroll 4
                for (int c = lane; c < KP / 4; c += 32)
                {
                    float4 w[RPW];
    #pragma unroll
                    for (int r = 0; r < RPW; ++r)
                        w[r] = (r < nr) ? load4(wrow + r * KP + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        const float4 xv = *reinterpret_cast<const float4*>(xs + m * KP + 4 * c);
    #pragma unroll
                        for (int r = 0; r < RPW; ++r) acc[r][m] += dot4(w[r], xv);
                    }
                }
    #pragma unroll
                for (int r = 0; r < RPW; ++r)
    #pragma unroll
                    for (int m = 0; m < MT; ++m) acc[r][m] = warp_sum(acc[r][m]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (!mine) continue;
            gi += kGemvWarps;

            const int n0 = r0 + seg0;
            if (EPI == EPI_STORE || EPI == EPI_RESID)
            {
    #pragma unroll
                for (int r = 0; r < RPW; ++r)
    #pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        if (lane == ((r * MT + m) & 31) && r < nr && m < rows)
                        {
                            const size_t o = static_cast<size_t>(m) * a.ldo + (n0 + r);
                            float v = acc[r][m];
                            if (EPI == EPI_RESID)
                            {
                                if (a.extra) v = a.extra[o] + v;
                                v = a.out[o] + v;
                                if (a.aux) a.aux[static_cast<size_t>(m) * a.ld_aux + (n0 + r)] = v;
                            }
                            a.out[o] = v;
                        }
                    }
            }
            else
            {
                // Penalised argmax: lane m tracks activation row m.
    #pragma unroll
                for (int r = 0; r < RPW; ++r)
                {
                    if (r >= nr) break;
                    const int v = n0 + r;
                    const bool in_hist = (a.hist[v >> 5] >> (v & 31)) & 1u;
    #pragma unroll
                    for (int m = 0; m < MT; ++m)
                    {
                        if (lane == m && m < rows)
                        {
                            const float s = acc[r][m];
                            if (a.logits) a.logits[static_cast<size_t>(m) * a.ldl + v] = s;
                            bool hit = in_hist;
                            for (int j = 0; j <= m; ++j) hit |= (s_prefix[j] == v);
                            const float ps = hit ? (s < 0.0f ? s * pen : s / pen) : s;
                            if (best.ri < 0 || s > best.rv) { best.rv = s; best.ri = v; }
                            if (best.pi < 0 || ps > best.pv) { best.pv = ps; best.pi = v; }
                        }
                    }
                }
            }
        }
    }

    if (EPI != EPI_ARGMAX)
    {
        HY_STEP_TRACE_MARK(4);
        HY_STEP_TRACE_EXIT();
        return;
    }

    // ---------------- argmax reduction ----------------
    if constexpr (MT == 16)
    {
        // Lane m + 16 tracked activation row m over the groups' rows 4-7: fold it into lane m
        // (larger value, then lower index: the first index of the maximum).
        const float orv = __shfl_down_sync(0xffffffffu, best.rv, 16);
        const int ori = __shfl_down_sync(0xffffffffu, best.ri, 16);
        const float opv = __shfl_down_sync(0xffffffffu, best.pv, 16);
        const int opi = __shfl_down_sync(0xffffffffu, best.pi, 16);
        if (lane < 16)
        {
            if (ori >= 0) best_update(best.rv, best.ri, orv, ori);
            if (opi >= 0) best_update(best.pv, best.pi, opv, opi);
        }
    }
    if (lane < MT)
        red4[warp * MT + lane] = make_float4(best.rv, __int_as_float(best.ri), best.pv, __int_as_float(best.pi));
    consumers_sync();
    if (tid < MT)
    {
        float rv = 0.f, pv = 0.f;
        int ri = -1, pi = -1;
        for (int w = 0; w < kGemvWarps; ++w)
        {
            const float4 t = red4[w * MT + tid];
            const int ti = __float_as_int(t.y), tp = __float_as_int(t.w);
            if (ti >= 0) best_update(rv, ri, t.x, ti);
            if (tp >= 0) best_update(pv, pi, t.z, tp);
        }
        a.part[b * MT + tid] = make_float4(rv, __int_as_float(ri), pv, __int_as_float(pi));
        __threadfence();
    }
    consumers_sync();
    if (tid == 0) redi[0] = (atomicAdd(a.counter, 1) == G - 1) ? 1 : 0;
    consumers_sync();
    HY_STEP_TRACE_MARK(4);
    HY_STEP_TRACE_EXIT();
    if (!redi[0]) return;
    __threadfence();

    float4* merged = red4 + kGemvWarps * MT;   // [MT]
    if (tid < MT)
    {
        float rv = 0.f, pv = 0.f;
        int ri = -1, pi = -1;
        for (int c = 0; c < G; ++c)
        {
            const float4 t = __ldcg(&a.part[c * MT + tid]);
            const int ti = __float_as_int(t.y), tp = __float_as_int(t.w);
            if (ti >= 0) best_update(rv, ri, t.x, ti);
            if (tp >= 0) best_update(pv, pi, t.z, tp);
        }
        merged[tid] = make_float4(rv, __int_as_float(ri), pv, __int_as_float(pi));
    }
    consumers_sync();
    if (tid != 0) return;
    *a.counter = 0;

    if (a.lm_mode == LM_NONE)
    {
        for (int m = 0; m < rows; ++m)
        {
            a.tok_out[m] = __float_as_int(merged[m].w);
            a.raw_out[m] = __float_as_int(merged[m].y);
        }
        return;
    }
    DecodeState* st = a.st;
    if (a.lm_mode == LM_BATCH)
    {
        // Per slot: log the token, extend the history and the KV length (this step
        // appended the row), stop at EOS or the slot's max_tokens.
        for (int m = 0; m < rows; ++m)
        {
            SlotState& ss = a.slots[m];
            if (!ss.active) continue;
            const int tok = __float_as_int(merged[m].w);
            const int n = ss.n_gen;
            a.log_tokens[static_cast<size_t>(m) * a.log_stride + n] = tok;
            a.log_raw[static_cast<size_t>(m) * a.log_stride + n] = __float_as_int(merged[m].y);
            ss.n_gen = n + 1;
            ss.kv_len += 1;
            a.slot_cur[m] = tok;
            a.hist[static_cast<size_t>(m) * a.hist_stride + (tok >> 5)] |= 1u << (tok & 31);
            if (is_eos(st, tok) || n + 1 >= ss.max_tokens) ss.active = 0;
        }
        return;
    }
    if (st->done) return;
    if (a.lm_mode == LM_AR)
    {
        const int tok = __float_as_int(merged[0].w);
        const int n = st->n_gen;
        if (n >= st->max_tokens)
        {
            st->done = 1;
            return;
        }
        a.log_tokens[n] = tok;
        a.log_raw[n] = __float_as_int(merged[0].y);
        st->n_gen = n + 1;
        st->cur_token = tok;
        st->kv_len += 1;
        a.hist[tok >> 5] |= 1u << (tok & 31);
        if (is_eos(st, tok) || n + 1 >= st->max_tokens) st->done = 1;
        return;
    }
    // LM_VERIFY: dflash_acceptance_length + commit + rollback (src/dflash_runtime.cpp:78-95,
    // src/text_runtime.cpp:1240-1296).
    int posterior[kBlock];
    for (int r = 0; r < kBlock; ++r)
    {
        posterior[r] = __float_as_int(merged[r].w);
        a.posterior_out[r] = posterior[r];
    }
    int accept = 0;
    for (int i = 1; i < kBlock; ++i)
    {
        if (s_prefix[i] != posterior[i - 1]) break;
        ++accept;
    }
    const int available = accept + 1;
    const int remaining = st->max_tokens - st->n_gen;
    int committed = min(available, remaining);
    int stop = 0;
    for (int i = 0; i < committed; ++i)
    {
        const int tok = s_prefix[i];
        a.log_tokens[st->n_gen + i] = tok;
        a.log_raw[st->n_gen + i] = -1;
        if (is_eos(st, tok))
        {
            committed = i + 1;
            stop = 1;
            break;
        }
    }
    for (int i = 0; i < committed; ++i)
    {
        const int tok = s_prefix[i];
        a.hist[tok >> 5] |= 1u << (tok & 31);
    }
    st->n_gen += committed;
    a.accept_log[st->block_count] = max(0, committed - 1);
    st->block_count += 1;
    st->kv_len += committed;
    st->cur_token = posterior[accept];
    st->accept = accept;
    st->committed = committed;
    st->stop = stop;
    if (committed < available || stop || st->n_gen >= st->max_tokens) st->done = 1;
}

}  // namespace hy
