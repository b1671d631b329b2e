// C ABI of the B200 text-decode library (include/hy_decode.h): device context,
// weight upload / synthetic generation, kernel launchers with programmatic
// dependent launch, CUDA-graph capture of the AR step and of the DFlash verify
// block, and the host loops that drive them.
#include "hy_attn.cuh"
#include "hy_device.cuh"
#include "hy_gemv.cuh"
#include "hy_mega.cuh"
#include "hy_prefill.cuh"
#include "hy_umma.cuh"
#include "hy_util.cuh"

#include "hy_decode.h"
#include "hy_debug.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <chrono>
#include <mutex>
#include <string>
#include <vector>

using namespace hy;

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& msg)
{
    g_error = msg;
    return code;
}

#define HY_CUDA(call)                                                                          \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(e_ == cudaErrorMemoryAllocation ? HY_ERR_OUT_OF_MEMORY : HY_ERR_CUDA,  \
                        std::string(#call) + ": " + cudaGetErrorString(e_));                   \
    } while (0)

constexpr int kFfn = 3584;                // kernels are specialised for the model's FFN width
// Splits per KV head of the M = 1 attention kernel: past splits + the new-row
// split. Measured per launch (7 / 10 / 13 / 19 splits): KV 1024 10.2 / 9.3 /
// 9.0 / 10.2 us, KV 8192 28.1 / 22.7 / 20.7 / 21.5 us - fewer splits shorten
// the last-CTA merge, more shorten each CTA's stream.
#ifndef HY_ATTN_SPLITS_AR
#define HY_ATTN_SPLITS_AR 13
#endif
constexpr int kAttnSplitsAR = HY_ATTN_SPLITS_AR;
// Key chunks per KV head of a <= 16-row step's attention (36: 288 CTAs, one wave at
// 2 per SM). In the verify graph at KV 2048, 18 / 24 / 36 / 40 chunks: attention
// 14.7 / 12.7 / 10.5 / 15.7 us + merge 2.8 / 3.1 / 3.8 / 4.1 us per layer.
#ifndef HY_VERIFY_CHUNKS
#define HY_VERIFY_CHUNKS 36
#endif
constexpr int kVerifyChunks = HY_VERIFY_CHUNKS;
constexpr int kMaxSplits = 20;
static_assert(kAttnSplitsAR >= 2 && kAttnSplitsAR <= kMaxSplits, "split count");
constexpr int kArStepsPerGraph = 4;
constexpr int kMegaChunk = 64;            // tokens per persistent-kernel launch
constexpr int kPrefillChunk = 1024;       // prompt rows per prefill pass (all layers)
constexpr unsigned long long kTidEmbed = 1, kTidFinalNorm = 2, kLayerTidBase = 100, kLayerTidStride = 16;
constexpr unsigned long long kTidDrafts = 9003;
enum { J_INPUT_NORM, J_Q, J_K, J_V, J_Q_NORM, J_K_NORM, J_O, J_POST_NORM, J_GATE, J_UP, J_DOWN };
constexpr int kAuxLayerIds[kAuxLayers] = {1, 8, 15, 22};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

float host_synth_mult(float std_dev) { return static_cast<float>(static_cast<double>(std_dev) * std::sqrt(3.0) / 65536.0); }

}  // namespace

namespace {
constexpr int kHistChunk = 4096;     // history ids per upload round
constexpr int kTimingEvents = 6;     // start, embedded, prefilled, first token, decode start, decode end
constexpr int kDflashGraphs = 4;     // DFlash blocks launched between host reads of the decode state
}  // namespace

struct hy_ctx {
    hy_config cfg{};
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    size_t device_bytes = 0;
    std::vector<void*> allocs;

    // weights
    void* embed = nullptr;                 // [V x 1024] WT
    std::vector<void*> wqkv, wo, wgu, wd;  // per layer
    float* norms = nullptr;                // per layer: input[1024], post[1024], qn[128], kn[128]; then final[1024]
    // KV cache [layers][8][cap][128] KT
    void* kc = nullptr;
    void* vc = nullptr;
    // rope (1-D) tables [max_context x 128]
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    float* pre_cos = nullptr;   // prefill / explicit-row tables [max(max_prefill,16) x 128]
    float* pre_sin = nullptr;
    int* pre_pos = nullptr;     // a prompt's position ids [4 x max(max_prefill,16)] (mRoPE gather)
    float* prompt = nullptr;    // [max_prefill x 1024]
    // step buffers
    float* x = nullptr;         // [16 x 1024] residual stream
    float* qkv = nullptr;       // [16 x 4096]
    float* attn = nullptr;      // [16 x 2048]
    float* gu = nullptr;        // [16 x 2 ffn]
    float* tmp = nullptr;       // [16 x 1024]
    float* act = nullptr;       // [16 x ffn] silu(gate) * up of 16-row steps
    float* hidden = nullptr;    // [16 x 1024]
    float* aux = nullptr;       // [4 x 16 x 1024]
    float* attn_part = nullptr;
    int* attn_cnt = nullptr;    // [layers][8]
    float4* lm_part = nullptr;  // [num_sms * 16]
    int* lm_cnt = nullptr;
    unsigned* hist = nullptr;   // [ceil(V/32)]
    DecodeState* st = nullptr;
    int* log_tokens = nullptr;
    int* log_raw = nullptr;
    int* accept_log = nullptr;
    int* proposed = nullptr;    // [16]
    int* posterior = nullptr;   // [16]
    int* tok_out = nullptr;     // [16]
    int* raw_out = nullptr;     // [16]
    int* prefix = nullptr;      // [16]
    int* greedy = nullptr;      // [max_tokens + 32]
    int* ids_buf = nullptr;     // [max_prefill]
    int* feat_idx = nullptr;    // [max_prefill]
    float* feats = nullptr;     // vision features [max_prefill x 1024]
    float* logits = nullptr;    // [16 x V] (lazily)
    // Prompt prefill in passes of up to pf_rows rows (the residual stream is ctx->prompt).
    // GEMM operands are split (hi / lo) and tiled for the tensor core (hy_umma.cuh);
    // activation buffers hold pf_pad = pf_rows rounded up to 128 rows.
    int pf_rows = 0, pf_pad = 0;
    float* pf_qkv = nullptr;                         // [pf_rows x 4096] row-major
    float* pf_a_hi = nullptr, *pf_a_lo = nullptr;    // normed rows, tiled [pf_pad x 1024]
    float* pf_at_hi = nullptr, *pf_at_lo = nullptr;  // attention output, tiled [pf_pad x 2048]
    float* pf_ac_hi = nullptr, *pf_ac_lo = nullptr;  // SwiGLU output, tiled [pf_pad x ffn]
    // Prefill attention work items (row block, key tiles, partial slot), merge items and partials.
    int4* pf_work = nullptr;
    int4* pf_merge = nullptr;
    float* pf_part = nullptr;
    float* va_part = nullptr;   // chunk partials of <= 16-row attention [kVerifyChunks][8][32][kPaPartStride]
    int pf_nwork = 0, pf_nmerge = 0;
    std::vector<int4> h_work, h_merge;
    // Per layer: q/k/v, o, gate/up, down weights, tiled hi (and lo for fp32 weights).
    std::vector<float*> tq_hi, tq_lo, to_hi, to_lo, tg_hi, tg_lo, td_hi, td_lo;
    int* err = nullptr;
    DecodeState* h_st = nullptr;  // pinned mirror
    int kv_len = 0;               // host mirror of the sequence length
    // Staging that keeps allocation and pageable copies off the call paths:
    // pinned host areas for the prompt uploads (ids, feature index, features,
    // cos, sin), history ids and small device reads; device buffers for history
    // ids and KV-row conversions. Every call that uses them has finished with
    // them (its stream synchronised) before it returns.
    unsigned char* h_stage = nullptr;
    size_t h_stage_bytes = 0;
    int* h_hist = nullptr;        // pinned [kHistChunk]
    int* h_small = nullptr;       // pinned [16]: first token, raw top-1, error words
    int* h_log = nullptr;         // pinned [2 x (max_tokens + 2 x 16)]: token logs read back at the end of a loop
    int* hist_ids = nullptr;      // device [kHistChunk]
    float* kv_stage = nullptr;    // device [max_context x 128]
    // Per-stage timing of the last AR / DFlash decode call (CUDA events on the stream).
    cudaEvent_t tev[kTimingEvents] = {};
    hy_decode_timing timing{};
    hy_dflash_timing dtiming{};

    // Persistent AR decode kernel (cooperative, one CTA per SM).
    const void** wptrs = nullptr;  // device arrays: wqkv[L], wo[L], wgu[L], wd[L]
    // Persistent kernel: activations exchanged between CTAs as 64-bit words
    // (value | epoch << 32), and the launch counter that makes epochs unique.
    unsigned long long* x_ep = nullptr;    // [1024]
    unsigned long long* qkv_ep = nullptr;  // [4096]
    unsigned long long* act_ep = nullptr;  // [ffn]
    unsigned long long* tok_ep = nullptr;  // [1]
    unsigned long long* attn_ep = nullptr;      // [8][8][2][130]
    unsigned long long* attn_out_ep = nullptr;  // [2048]
    unsigned mega_seq = 0;
    int* dbg = nullptr;            // persistent-kernel self-check record [4]
    unsigned* progress = nullptr;  // host-mapped per-CTA phase progress (HY_DEBUG_PROGRESS=1)
    unsigned long long* wstat = nullptr;  // wait statistics (builds with HY_WAIT_STATS only)
    unsigned long long wait_limit_ns = kWaitLimitNs;   // bound of the persistent kernel's waits
    unsigned long long* probe_word = nullptr;          // an epoch word nothing publishes (wait probe)
    int mega_launches = 0;                // persistent launches since the statistics were reset
    int ar_path = HY_AR_PATH_PERSISTENT;
    bool mega_ok = false;

    // Tensor map of the tied table for the 16-row LM head (128-row x 128-byte boxes, 128-byte swizzle).
    CUtensorMap lm_tmap;

    cudaGraphExec_t g_ar = nullptr;
    cudaGraphExec_t g_verify_draft = nullptr;
    cudaGraphExec_t g_verify_ids = nullptr;

    // DFlash draft network (hy_draft_load*): its weights (decoder-layer geometry),
    // its K/V cache of the context rows, its RoPE table (theta 10000) and buffers.
    // The draft context covers KV rows [0, d_len); every path that appends KV
    // rows while a draft is loaded appends their context rows too.
    int d_layers = 0;
    int d_mask = 0;                          // mask token of the noise block
    int d_len = 0;                           // host mirror: rows with draft context
    void* d_fc = nullptr;                    // [1024 x 4096] WT
    std::vector<void*> d_wqkv, d_wo, d_wgu, d_wd;
    float* d_norms = nullptr;                // per layer input, post, qn, kn (2304); then hidden_norm, norm
    void* d_kc = nullptr;                    // [d_layers][8][cap][128] KT
    void* d_vc = nullptr;
    float* d_cos = nullptr;                  // [max_context x 128], theta 10000
    float* d_sin = nullptr;
    float* d_x = nullptr;                    // [16 x 1024] draft residual stream
    float* d_aux = nullptr;                  // [16 x 4096] aux rows of a step (layers 1, 8, 15, 22 side by side)
    float* d_pf_aux = nullptr;               // [pf_rows x 4096] aux rows of a prefill pass
    float* d_pf_a_hi = nullptr;              // the same, split and tiled [pf_pad x 4096]
    float* d_pf_a_lo = nullptr;
    float* d_pf_fc = nullptr;                // [pf_rows x 1024] fc output
    float* d_tfc_hi = nullptr;               // fc tiled [1024 x 4096]
    float* d_tfc_lo = nullptr;
    std::vector<float*> d_tkv_hi, d_tkv_lo;  // k | v rows tiled [2048 x 1024] per draft layer
    std::vector<void*> d_allocs;
    size_t d_bytes = 0;
    // draft + verify + context append + commit: one graph per block of a group of
    // kDflashGraphs blocks between host reads, each recording its stage events
    // (block start, draft done, verify and context rows done).
    cudaGraphExec_t g_dflash[kDflashGraphs] = {};
    cudaEvent_t dflash_ev[kDflashGraphs][3] = {};
    cudaGraphExec_t g_verify_ids_ctx = nullptr;   // verify of given ids + context append + commit

    // Batched decode (hy_batch_decode): up to 16 sequences, sequence s in step row s,
    // each with its own KV cache [layer][8][cap][128] (slot-major), history bitmap
    // and token log; one CUDA graph = one decode step of every slot.
    int b_rows = 0;                          // rows (slots) of the captured step graph
    void* b_kc = nullptr;                    // [16][layers][8][cap][128] KT
    void* b_vc = nullptr;
    SlotState* b_state = nullptr;            // [16]
    SlotState* h_bstate = nullptr;           // pinned mirror
    int* b_cur = nullptr;                    // [16] next token per slot
    unsigned* b_hist = nullptr;              // [16][hist words]
    int* b_log = nullptr;                    // [16][max_tokens + 32]
    int* b_lograw = nullptr;
    int* b_cnt = nullptr;                    // [layers][16][8] attention tickets
    std::vector<void*> b_allocs;
    cudaGraphExec_t g_batch = nullptr;
    // Streaming: called with each committed token, in order, when the host reads
    // the decode state (every `cb_sync` AR tokens, every 4 DFlash blocks).
    hy_token_callback cb = nullptr;
    void* cb_user = nullptr;
    int cb_sync = 0;
    int cb_emitted = 0;     // tokens of the current generation already passed to cb
    int hist_words() const { return (cfg.vocab_size + 31) / 32; }
    int log_stride() const { return cfg.max_tokens + 2 * kBlock; }
    size_t slot_elems() const { return static_cast<size_t>(cfg.num_layers) * kNumKVHeads * cfg.max_context * kHeadDim; }

    size_t kv_elem() const { return cfg.kv_dtype == HY_DTYPE_BF16 ? 2 : 4; }
    size_t w_elem() const { return cfg.weight_dtype == HY_DTYPE_BF16 ? 2 : 4; }
    float* in_norm(int l) const { return norms + static_cast<size_t>(l) * 2304; }
    float* post_norm(int l) const { return norms + static_cast<size_t>(l) * 2304 + 1024; }
    float* qn(int l) const { return norms + static_cast<size_t>(l) * 2304 + 2048; }
    float* kn(int l) const { return norms + static_cast<size_t>(l) * 2304 + 2176; }
    float* final_norm() const { return norms + static_cast<size_t>(cfg.num_layers) * 2304; }
    void* kc_layer(int l) const
    {
        return static_cast<char*>(kc) + static_cast<size_t>(l) * kNumKVHeads * cfg.max_context * kHeadDim * kv_elem();
    }
    void* vc_layer(int l) const
    {
        return static_cast<char*>(vc) + static_cast<size_t>(l) * kNumKVHeads * cfg.max_context * kHeadDim * kv_elem();
    }
    float* d_in_norm(int l) const { return d_norms + static_cast<size_t>(l) * 2304; }
    float* d_post_norm(int l) const { return d_norms + static_cast<size_t>(l) * 2304 + 1024; }
    float* d_qn(int l) const { return d_norms + static_cast<size_t>(l) * 2304 + 2048; }
    float* d_kn(int l) const { return d_norms + static_cast<size_t>(l) * 2304 + 2176; }
    float* d_hidden_norm() const { return d_norms + static_cast<size_t>(d_layers) * 2304; }
    float* d_final_norm() const { return d_norms + static_cast<size_t>(d_layers) * 2304 + 1024; }
    void* d_kc_layer(int l) const
    {
        return static_cast<char*>(d_kc) + static_cast<size_t>(l) * kNumKVHeads * cfg.max_context * kHeadDim * kv_elem();
    }
    void* d_vc_layer(int l) const
    {
        return static_cast<char*>(d_vc) + static_cast<size_t>(l) * kNumKVHeads * cfg.max_context * kHeadDim * kv_elem();
    }
};

namespace {

template <typename T>
int dalloc(hy_ctx* c, T** p, size_t count)
{
    void* v = nullptr;
    const size_t bytes = align_up(std::max<size_t>(count * sizeof(T), 16), 256);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess)
        return fail(HY_ERR_OUT_OF_MEMORY, "cudaMalloc(" + std::to_string(bytes) + " bytes) failed: " + cudaGetErrorString(e));
    c->allocs.push_back(v);
    c->device_bytes += bytes;
    *p = static_cast<T*>(v);
    return HY_OK;
}

// ---------------------------------------------------------------------------
// Launch helpers.
// ---------------------------------------------------------------------------
// Every decode kernel is launched with programmatic stream serialization: its
// producer warp may start streaming weights while the previous kernel drains;
// its consumers wait with griddepcontrol.wait. `pdl` is false for a kernel
// that follows a copy in the stream.
thread_local bool t_next_plain = false;

template <typename Kern, typename Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Args& args)
{
    const bool pdl = !t_next_plain;
    t_next_plain = false;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

template <typename WT, int KP, int MT, int PRO, int EPI>
cudaError_t run_gemv(hy_ctx* c, const GemvArgs& a)
{
    using S = GemvShape<WT, KP, MT>;
    constexpr int smem = (MT == 16 && EPI == EPI_ARGMAX) ? S::SMEM_TL : S::SMEM;
    auto k = gemv_kernel<WT, KP, MT, PRO, EPI>;
    static unsigned long long configured = 0;  // per instantiation, one bit per device
    const unsigned long long bit = 1ull << (c->cfg.device & 63);
    if (!(configured & bit))
    {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    return launch_pdl(k, dim3(c->num_sms), dim3(kGemvThreads), smem, c->stream, a);
}

template <int MT, typename KT>
cudaError_t run_attn(hy_ctx* c, const AttnArgs& a, int splits)
{
    using S = AttnShape<MT, KT>;
    auto k = attn_kernel<MT, KT>;
    static unsigned long long configured = 0;
    const unsigned long long bit = 1ull << (c->cfg.device & 63);
    if (!(configured & bit))
    {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    return launch_pdl(k, dim3(splits, kNumKVHeads), dim3(kAttnThreads), S::SMEM, c->stream, a);
}

// Attention of a step of 2..16 rows (DFlash verify, decoder steps): RoPE + QK
// norm + KV append of the rows, then the tensor-core attention over the keys
// [0, past + rows) in kVerifyChunks chunks per KV head, then the chunk merge.
// The DFlash draft (draft = true) normalises q / k before RoPE and attends
// without a mask.
template <typename KT>
cudaError_t run_attn16(hy_ctx* c, const AttnArgs& at, bool draft = false)
{
    PrefillRopeArgs ra{const_cast<float*>(at.qkv), at.ldq, at.cos, at.sin, at.qn_w, at.kn_w, at.kc, at.vc, at.cap,
                       at.past_fixed, at.eps, at.scale_log2, at.st, at.rope_state, c->err, draft ? 1 : 0, 0};
    cudaError_t e = launch_pdl(prefill_rope_kernel<KT>, dim3(at.rows, 4), dim3(256), 0, c->stream, ra);
    if (e != cudaSuccess) return e;
    static_assert(kVerifyChunks <= kMaxVerifyChunks, "chunk merge capacity");
    using S = PaShape<KT, 16>;
    auto k = prefill_attn_kernel<KT, 16>;
    static unsigned long long configured = 0;
    const unsigned long long bit = 1ull << (c->cfg.device & 63);
    if (!(configured & bit))
    {
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM)) != cudaSuccess) return e;
        configured |= bit;
    }
    PrefillAttnArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.q = at.qkv;
    pa.ldq = at.ldq;
    pa.kc = at.kc;
    pa.vc = at.vc;
    pa.cap = at.cap;
    pa.past = at.past_fixed;
    pa.rows = at.rows;
    pa.part = c->va_part;
    pa.st = at.st;
    pa.err = c->err;
    pa.noncausal = draft ? 1 : 0;
    if ((e = launch_pdl(k, dim3(kVerifyChunks, kNumKVHeads), dim3(S::THREADS), S::SMEM, c->stream, pa)) != cudaSuccess)
        return e;
    const ChunkMergeArgs ma{c->va_part, kVerifyChunks, at.rows, at.out};
    return launch_pdl(attn_chunk_merge_kernel, dim3(32, kNumKVHeads), dim3(kHeadDim), 0, c->stream, ma);
}

// How the first layer's input rows are produced.
struct StepSource {
    int src;          // SRC_X (ctx->x already holds the rows) or a gather mode
    const int* ids;   // SRC_GATHER_IDS
};

struct StepPlan {
    int rows;          // active rows (1..16)
    StepSource source;
    const float* cos;  // rope tables and indexing
    const float* sin;
    int rope_state;
    bool past_from_state;
    int past_fixed;
    int lm_mode;       // -1: no LM head; else LM_* with PRO_NORM on x
    float** aux;       // optional [4] aux outputs, nullable
    int ld_aux;        // their row stride (0: 1024)
};

GemvArgs base_args(hy_ctx* c)
{
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.eps = c->cfg.rms_norm_eps;
    a.st = c->st;
    a.vocab = c->cfg.vocab_size;
    a.err = c->err;
    a.table = c->embed;
    a.hist = c->hist;
    a.part = c->lm_part;
    a.counter = c->lm_cnt;
    a.tmap = c->lm_tmap;
    return a;
}

template <typename WT, int MT>
cudaError_t enqueue_step_lm_t(hy_ctx* c, const StepPlan& p);

template <typename WT, typename KT, int MT>
cudaError_t enqueue_step_t(hy_ctx* c, const StepPlan& p)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < cfg.num_layers; ++l)
    {
        // q/k/v projections with the input RMSNorm (and, on layer 0, the embedding gather).
        GemvArgs q = base_args(c);
        q.W = c->wqkv[l];
        q.N = kQKVRows;
        q.ldw = kHidden;
        q.rows = p.rows;
        q.src = (l == 0) ? p.source.src : SRC_X;
        q.ids = p.source.ids;
        q.ids_out = (l == 0 && p.source.src == SRC_GATHER_DRAFT) ? c->proposed : nullptr;
        q.greedy = c->greedy;
        q.x_store = c->x;
        q.x = c->x;
        q.ldx = kHidden;
        q.norm_w = c->in_norm(l);
        q.out = c->qkv;
        q.ldo = kQKVRows;
        if ((e = run_gemv<WT, kHidden, MT, PRO_NORM, EPI_STORE>(c, q)) != cudaSuccess) return e;

        AttnArgs at;
        std::memset(&at, 0, sizeof(at));
        at.qkv = c->qkv;
        at.ldq = kQKVRows;
        at.qn_w = c->qn(l);
        at.kn_w = c->kn(l);
        at.cos = p.cos;
        at.sin = p.sin;
        at.rope_state = p.rope_state;
        at.kc = c->kc_layer(l);
        at.vc = c->vc_layer(l);
        at.cap = cfg.max_context;
        at.st = p.past_from_state ? c->st : nullptr;
        at.past_fixed = p.past_fixed;
        at.rows = p.rows;
        at.scale_log2 = cfg.attn_scale * 1.4426950408889634f;
        at.eps = cfg.rms_norm_eps;
        at.part = c->attn_part;
        at.counter = c->attn_cnt + l * kNumKVHeads;
        at.out = c->attn;
        at.err = c->err;
        if constexpr (MT == 1)
        {
            if ((e = run_attn<1, KT>(c, at, kAttnSplitsAR)) != cudaSuccess) return e;
        }
        else
        {
            if ((e = run_attn16<KT>(c, at)) != cudaSuccess) return e;
        }

        GemvArgs o = base_args(c);
        o.W = c->wo[l];
        o.N = kHidden;
        o.ldw = kQWidth;
        o.rows = p.rows;
        o.src = SRC_X;
        o.x = c->attn;
        o.ldx = kQWidth;
        o.out = c->x;
        o.ldo = kHidden;
        if ((e = run_gemv<WT, kQWidth, MT, PRO_PLAIN, EPI_RESID>(c, o)) != cudaSuccess) return e;

        GemvArgs gu = base_args(c);
        gu.W = c->wgu[l];
        gu.N = 2 * ffn;
        gu.ldw = kHidden;
        gu.rows = p.rows;
        gu.src = SRC_X;
        gu.x = c->x;
        gu.ldx = kHidden;
        gu.norm_w = c->post_norm(l);
        if constexpr (MT == 1)
        {
            gu.out = c->gu;
            gu.ldo = 2 * ffn;
            if ((e = run_gemv<WT, kHidden, MT, PRO_NORM, EPI_STORE>(c, gu)) != cudaSuccess) return e;
        }
        else
        {
            // 16 rows: the epilogue applies SwiGLU (act = silu(gate) * up).
            gu.out = c->act;
            gu.ldo = ffn;
            if ((e = run_gemv<WT, kHidden, MT, PRO_NORM, EPI_ACT>(c, gu)) != cudaSuccess) return e;
        }

        float* aux = nullptr;
        if (p.aux)
            for (int i = 0; i < kAuxLayers; ++i)
                if (kAuxLayerIds[i] == l) aux = p.aux[i];
        GemvArgs d = base_args(c);
        d.W = c->wd[l];
        d.N = kHidden;
        d.ldw = ffn;
        d.rows = p.rows;
        d.src = SRC_X;
        d.x = c->gu;
        d.ldx = 2 * ffn;
        if constexpr (MT == 1)
        {
            d.out = c->x;
            d.ldo = kHidden;
            d.aux = aux;
            d.ld_aux = p.ld_aux ? p.ld_aux : kHidden;
            if ((e = run_gemv<WT, kFfn, MT, PRO_SWIGLU, EPI_RESID>(c, d)) != cudaSuccess) return e;
        }
        else
        {
            // K split in two halves so the 16 activation rows fit in shared memory;
            // the inputs are the act rows of the gate/up step.
            d.x = c->act;
            d.ldx = ffn;
            GemvArgs d1 = d;
            d1.k_off = 0;
            d1.out = c->tmp;
            d1.ldo = kHidden;
            if ((e = run_gemv<WT, kFfn / 2, MT, PRO_PLAIN, EPI_STORE>(c, d1)) != cudaSuccess) return e;
            GemvArgs d2 = d;
            d2.k_off = kFfn / 2;
            d2.out = c->x;
            d2.ldo = kHidden;
            d2.extra = c->tmp;
            d2.aux = aux;
            d2.ld_aux = p.ld_aux ? p.ld_aux : kHidden;
            if ((e = run_gemv<WT, kFfn / 2, MT, PRO_PLAIN, EPI_RESID>(c, d2)) != cudaSuccess) return e;
        }
    }
    if (p.lm_mode >= 0) return enqueue_step_lm_t<WT, MT>(c, p);
    return cudaSuccess;
}

// Final norm + LM head + selection (and the AR / verify commit) of a step's rows in ctx->x.
template <typename WT, int MT>
cudaError_t enqueue_step_lm_t(hy_ctx* c, const StepPlan& p)
{
    const hy_config& cfg = c->cfg;
    cudaError_t e = cudaSuccess;
    {
        GemvArgs lm = base_args(c);
        lm.W = c->embed;
        lm.N = cfg.vocab_size;
        lm.ldw = kHidden;
        lm.rows = p.rows;
        lm.src = SRC_X;
        lm.x = c->x;
        lm.ldx = kHidden;
        lm.norm_w = c->final_norm();
        lm.lm_mode = p.lm_mode;
        lm.prefix = (p.lm_mode == LM_VERIFY) ? c->proposed : nullptr;
        lm.tok_out = c->tok_out;
        lm.raw_out = c->raw_out;
        lm.log_tokens = c->log_tokens;
        lm.log_raw = c->log_raw;
        lm.accept_log = c->accept_log;
        lm.posterior_out = c->posterior;
        if ((e = run_gemv<WT, kHidden, MT, PRO_NORM, EPI_ARGMAX>(c, lm)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t enqueue_step(hy_ctx* c, const StepPlan& p)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    const bool one = p.rows == 1;
    if (!wb && !kb) return one ? enqueue_step_t<float, float, 1>(c, p) : enqueue_step_t<float, float, 16>(c, p);
    if (!wb && kb)
        return one ? enqueue_step_t<float, __nv_bfloat16, 1>(c, p) : enqueue_step_t<float, __nv_bfloat16, 16>(c, p);
    if (wb && !kb)
        return one ? enqueue_step_t<__nv_bfloat16, float, 1>(c, p) : enqueue_step_t<__nv_bfloat16, float, 16>(c, p);
    return one ? enqueue_step_t<__nv_bfloat16, __nv_bfloat16, 1>(c, p)
               : enqueue_step_t<__nv_bfloat16, __nv_bfloat16, 16>(c, p);
}

// LM head + selection over rows of ctx->x that are already final-normed.
template <typename WT, int MT>
cudaError_t enqueue_lm_select_t(hy_ctx* c, int rows, const float* x, float penalty, bool with_prefix, float* logits)
{
    GemvArgs lm = base_args(c);
    lm.W = c->embed;
    lm.N = c->cfg.vocab_size;
    lm.ldw = kHidden;
    lm.rows = rows;
    lm.src = SRC_X;
    lm.x = x;
    lm.ldx = kHidden;
    lm.lm_mode = LM_NONE;
    lm.penalty = penalty;
    lm.prefix = with_prefix ? c->prefix : nullptr;
    lm.logits = logits;
    lm.ldl = c->cfg.vocab_size;
    lm.tok_out = c->tok_out;
    lm.raw_out = c->raw_out;
    return run_gemv<WT, kHidden, MT, PRO_PLAIN, EPI_ARGMAX>(c, lm);
}

cudaError_t enqueue_lm_select(hy_ctx* c, int rows, const float* x, float penalty, bool with_prefix, float* logits)
{
    if (c->cfg.weight_dtype == HY_DTYPE_BF16)
        return rows == 1 ? enqueue_lm_select_t<__nv_bfloat16, 1>(c, rows, x, penalty, with_prefix, logits)
                         : enqueue_lm_select_t<__nv_bfloat16, 16>(c, rows, x, penalty, with_prefix, logits);
    return rows == 1 ? enqueue_lm_select_t<float, 1>(c, rows, x, penalty, with_prefix, logits)
                     : enqueue_lm_select_t<float, 16>(c, rows, x, penalty, with_prefix, logits);
}

int check_device_error(hy_ctx* c)
{
    // Both words in one synchronisation, into pinned memory (h_small[8..12]).
    int* d = c->h_small + 8;
    if (c->dbg) HY_CUDA(cudaMemcpyAsync(d, c->dbg, 4 * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaMemcpyAsync(d + 4, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    if (c->dbg && d[0] != 0)
    {
        const std::string msg = "persistent kernel self-check " + std::to_string(d[0]) + " failed (cta " +
                                std::to_string(d[1]) + ", phase " + std::to_string(d[2]) + ", index " +
                                std::to_string(d[3]) + ")";
        HY_CUDA(cudaMemsetAsync(c->dbg, 0, 4 * sizeof(int), c->stream));
        return fail(HY_ERR_INVALID_ARGUMENT, msg);
    }
    const int h = d[4];
    if (h != 0)
    {
        HY_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
        HY_CUDA(cudaStreamSynchronize(c->stream));
        if (h & (kErrTimeoutFull | kErrTimeoutEmpty))
            return fail(HY_ERR_DEVICE_TIMEOUT, "a device-side bounded wait timed out (error bits " + std::to_string(h) + ")");
        return fail(HY_ERR_INVALID_ARGUMENT, "device-side bounds check failed (error bits " + std::to_string(h) + ")");
    }
    return HY_OK;
}

int sync_state_to_host(hy_ctx* c)
{
    HY_CUDA(cudaMemcpyAsync(c->h_st, c->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    c->kv_len = c->h_st->kv_len;
    return HY_OK;
}

int push_state(hy_ctx* c)
{
    HY_CUDA(cudaMemcpyAsync(c->st, c->h_st, sizeof(DecodeState), cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

int set_eos(hy_ctx* c, const int* eos_ids, int n_eos)
{
    if (n_eos < 0 || n_eos > kMaxEos || (n_eos > 0 && !eos_ids))
        return fail(HY_ERR_INVALID_ARGUMENT, "at most " + std::to_string(kMaxEos) + " EOS ids are supported");
    c->h_st->n_eos = n_eos;
    for (int i = 0; i < n_eos; ++i) c->h_st->eos[i] = eos_ids[i];
    return HY_OK;
}

int capture(hy_ctx* c, cudaGraphExec_t* out, const StepPlan& p, int repeats)
{
    cudaGraph_t graph = nullptr;
    HY_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < repeats && e == cudaSuccess; ++i) e = enqueue_step(c, p);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph capture end: ") + cudaGetErrorString(e2));
    e = cudaGraphInstantiate(out, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    return HY_OK;
}

thread_local unsigned long long* t_trace = nullptr;
thread_local int t_trace_token = 0;

template <typename WT, typename KT>
cudaError_t launch_mega_t(hy_ctx* c, int steps)
{
    auto k = mega_decode_kernel<WT, KT>;
    MegaArgs a;
    std::memset(&a, 0, sizeof(a));
    const int L = c->cfg.num_layers;
    a.embed = c->embed;
    a.wqkv = c->wptrs;
    a.wo = c->wptrs + L;
    a.wgu = c->wptrs + 2 * L;
    a.wd = c->wptrs + 3 * L;
    a.norms = c->norms;
    a.kc = c->kc;
    a.vc = c->vc;
    a.cap = c->cfg.max_context;
    a.rope_cos = c->rope_cos;
    a.rope_sin = c->rope_sin;
    a.x = c->x;
    a.qkv = c->qkv;
    a.attn = c->attn;
    a.gu = c->gu;
    a.attn_part = c->attn_part;
    a.attn_cnt = c->attn_cnt;
    a.lm_part = c->lm_part;
    a.lm_cnt = c->lm_cnt;
    a.hist = c->hist;
    a.st = c->st;
    a.log_tokens = c->log_tokens;
    a.log_raw = c->log_raw;
    a.num_layers = L;
    a.vocab = c->cfg.vocab_size;
    a.ffn = c->cfg.ffn_dim;
    a.eps = c->cfg.rms_norm_eps;
    a.scale_log2 = c->cfg.attn_scale * 1.4426950408889634f;
    a.steps = steps;
    a.err = c->err;
    a.trace = t_trace;
    a.trace_token = t_trace_token;
    a.dbg = c->dbg;
    a.wstat = c->wstat;
    a.launch_slot = c->mega_launches++;
    a.wait_limit_ns = c->wait_limit_ns;
    if (c->progress)
    {
        unsigned* dp = nullptr;
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&dp), c->progress, 0);
        a.progress = dp;
    }
    // Epochs of this launch: epoch_base + 1 .. epoch_base + steps * phases (< kMegaEpochSpan).
    // Epoch 0 never occurs, so zeroed words are never taken for data; on wrap-around
    // the words are cleared again.
    if (c->mega_seq == 0 || c->mega_seq >= 0xFFFFFFFFu / kMegaEpochSpan)
    {
        c->mega_seq = 0;
        cudaError_t z = cudaMemsetAsync(c->x_ep, 0, sizeof(unsigned long long) * kHidden, c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(c->qkv_ep, 0, sizeof(unsigned long long) * kQKVRows, c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(c->act_ep, 0, sizeof(unsigned long long) * c->cfg.ffn_dim, c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(c->tok_ep, 0, sizeof(unsigned long long), c->stream);
        if (z == cudaSuccess)
            z = cudaMemsetAsync(c->attn_ep, 0,
                                sizeof(unsigned long long) * kNumKVHeads * (kMegaSplits - 1) * 2 * kAttnWords, c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(c->attn_out_ep, 0, sizeof(unsigned long long) * kQWidth, c->stream);
        if (z != cudaSuccess) return z;
    }
    ++c->mega_seq;
    a.x_ep = c->x_ep;
    a.qkv_ep = c->qkv_ep;
    a.act_ep = c->act_ep;
    a.tok_ep = c->tok_ep;
    a.attn_ep = c->attn_ep;
    a.attn_out_ep = c->attn_out_ep;
    a.epoch_base = c->mega_seq * kMegaEpochSpan;
    void* params[] = {&a};
    return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(k), dim3(c->num_sms), dim3(kMegaThreads), params,
                                       MegaSmem::SIZE, c->stream);
}

cudaError_t launch_mega(hy_ctx* c, int steps)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    if (!wb && !kb) return launch_mega_t<float, float>(c, steps);
    if (!wb && kb) return launch_mega_t<float, __nv_bfloat16>(c, steps);
    if (wb && !kb) return launch_mega_t<__nv_bfloat16, float>(c, steps);
    return launch_mega_t<__nv_bfloat16, __nv_bfloat16>(c, steps);
}

template <typename WT, typename KT>
int setup_mega_t(hy_ctx* c)
{
    auto k = mega_decode_kernel<WT, KT>;
    HY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, MegaSmem::SIZE));
    int per_sm = 0;
    HY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kMegaThreads, MegaSmem::SIZE));
    int coop = 0;
    HY_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->cfg.device));
    // All attention splits (8 heads x 18) need a CTA each; one CTA per SM must fit.
    c->mega_ok = coop && per_sm >= 1 && c->num_sms >= kNumKVHeads * kMegaSplits &&
                 (c->cfg.vocab_size + c->num_sms - 1) / c->num_sms <= 32 * (kMegaHistWords - 2);
    if (!c->mega_ok) c->ar_path = HY_AR_PATH_GRAPH;
    return HY_OK;
}

int setup_mega(hy_ctx* c)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    if (!wb && !kb) return setup_mega_t<float, float>(c);
    if (!wb && kb) return setup_mega_t<float, __nv_bfloat16>(c);
    if (wb && !kb) return setup_mega_t<__nv_bfloat16, float>(c);
    return setup_mega_t<__nv_bfloat16, __nv_bfloat16>(c);
}

int ensure_graphs(hy_ctx* c)
{
    {
        int rc = setup_mega(c);
        if (rc) return rc;
    }
    if (!c->g_ar)
    {
        StepPlan p{};
        p.rows = 1;
        p.source.src = SRC_GATHER_STATE;
        p.cos = c->rope_cos;
        p.sin = c->rope_sin;
        p.rope_state = 1;
        p.past_from_state = true;
        p.lm_mode = LM_AR;
        int rc = capture(c, &c->g_ar, p, kArStepsPerGraph);
        if (rc) return rc;
    }
    if (!c->g_verify_draft)
    {
        StepPlan p{};
        p.rows = kBlock;
        p.source.src = SRC_GATHER_DRAFT;
        p.cos = c->rope_cos;
        p.sin = c->rope_sin;
        p.rope_state = 1;
        p.past_from_state = true;
        p.lm_mode = LM_VERIFY;
        int rc = capture(c, &c->g_verify_draft, p, 1);
        if (rc) return rc;
    }
    if (!c->g_verify_ids)
    {
        StepPlan p{};
        p.rows = kBlock;
        p.source.src = SRC_GATHER_IDS;
        p.source.ids = c->proposed;
        p.cos = c->rope_cos;
        p.sin = c->rope_sin;
        p.rope_state = 1;
        p.past_from_state = true;
        p.lm_mode = LM_VERIFY;
        int rc = capture(c, &c->g_verify_ids, p, 1);
        if (rc) return rc;
    }
    return HY_OK;
}

// rope_value (src/text_runtime.cpp:182-193), in the reference's float arithmetic.
float rope_value_host(int position, int dim, bool use_cos)
{
    const float base = static_cast<float>(10000.0 * std::pow(1000.0, 128.0 / 126.0));
    const int half_dim = dim % (kHeadDim / 2);
    const float exponent = static_cast<float>(2 * half_dim) / static_cast<float>(kHeadDim);
    const float inv_freq = 1.0f / std::pow(base, exponent);
    const float angle = static_cast<float>(position) * inv_freq;
    return use_cos ? std::cos(angle) : std::sin(angle);
}

int validate_config(const hy_config* cfg)
{
    if (!cfg) return fail(HY_ERR_INVALID_ARGUMENT, "config is null");
    if (cfg->num_layers <= 0 || cfg->num_layers > 64) return fail(HY_ERR_INVALID_ARGUMENT, "num_layers must be in 1..64");
    if (cfg->vocab_size < 16 || cfg->vocab_size > (1 << 24)) return fail(HY_ERR_INVALID_ARGUMENT, "vocab_size out of range");
    if (cfg->ffn_dim != kFfn) return fail(HY_ERR_UNSUPPORTED, "ffn_dim must be 3584 (kernels are specialised for it)");
    if (cfg->max_context < 32 || cfg->max_context > (1 << 20))
        return fail(HY_ERR_INVALID_ARGUMENT, "max_context out of range");
    if (cfg->max_prefill < 1 || cfg->max_prefill > cfg->max_context)
        return fail(HY_ERR_INVALID_ARGUMENT, "max_prefill must be in 1..max_context");
    if (cfg->max_tokens < 1) return fail(HY_ERR_INVALID_ARGUMENT, "max_tokens must be positive");
    if ((cfg->weight_dtype != HY_DTYPE_F32 && cfg->weight_dtype != HY_DTYPE_BF16) ||
        (cfg->kv_dtype != HY_DTYPE_F32 && cfg->kv_dtype != HY_DTYPE_BF16))
        return fail(HY_ERR_INVALID_ARGUMENT, "dtype must be HY_DTYPE_F32 or HY_DTYPE_BF16");
    if (!(cfg->rms_norm_eps > 0.f) || !(cfg->attn_scale > 0.f)) return fail(HY_ERR_INVALID_ARGUMENT, "eps/scale must be positive");
    return HY_OK;
}

// Pinned staging of one prompt upload: ids, feature index [rows] int, features
// [rows x 1024], cos, sin [rows x 128] float, each 256-byte aligned.
struct PromptStage {
    int* ids;
    int* feat_idx;
    float* feats;
    float* cos;
    float* sin;
};
size_t prompt_stage_bytes(int rows)
{
    const size_t r = static_cast<size_t>(std::max(rows, kMaxStepRows));
    return 2 * align_up(r * sizeof(int), 256) + align_up(r * kHidden * sizeof(float), 256) +
           2 * align_up(r * kHeadDim * sizeof(float), 256);
}
PromptStage prompt_stage(hy_ctx* c)
{
    const size_t r = static_cast<size_t>(std::max(c->cfg.max_prefill, kMaxStepRows));
    unsigned char* p = c->h_stage;
    PromptStage s;
    s.ids = reinterpret_cast<int*>(p);
    p += align_up(r * sizeof(int), 256);
    s.feat_idx = reinterpret_cast<int*>(p);
    p += align_up(r * sizeof(int), 256);
    s.feats = reinterpret_cast<float*>(p);
    p += align_up(r * kHidden * sizeof(float), 256);
    s.cos = reinterpret_cast<float*>(p);
    p += align_up(r * kHeadDim * sizeof(float), 256);
    s.sin = reinterpret_cast<float*>(p);
    return s;
}

int alloc_ctx(hy_ctx* c)
{
    const hy_config& cfg = c->cfg;
    HY_CUDA(cudaSetDevice(cfg.device));
    HY_CUDA(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, cfg.device));
    HY_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    const size_t we = c->w_elem();
    const int L = cfg.num_layers, ffn = cfg.ffn_dim;
    int rc;
    unsigned char* wbytes = nullptr;
    const size_t per_layer = align_up(static_cast<size_t>(kQKVRows) * kHidden * we, 256) +
                             align_up(static_cast<size_t>(kHidden) * kQWidth * we, 256) +
                             align_up(static_cast<size_t>(2 * ffn) * kHidden * we, 256) +
                             align_up(static_cast<size_t>(kHidden) * ffn * we, 256);
    const size_t embed_bytes = align_up(static_cast<size_t>(cfg.vocab_size) * kHidden * we, 256);
    if ((rc = dalloc(c, &wbytes, embed_bytes + per_layer * L))) return rc;
    c->embed = wbytes;
    unsigned char* p = wbytes + embed_bytes;
    for (int l = 0; l < L; ++l)
    {
        c->wqkv.push_back(p);
        p += align_up(static_cast<size_t>(kQKVRows) * kHidden * we, 256);
        c->wo.push_back(p);
        p += align_up(static_cast<size_t>(kHidden) * kQWidth * we, 256);
        c->wgu.push_back(p);
        p += align_up(static_cast<size_t>(2 * ffn) * kHidden * we, 256);
        c->wd.push_back(p);
        p += align_up(static_cast<size_t>(kHidden) * ffn * we, 256);
    }
    if ((rc = dalloc(c, &c->norms, static_cast<size_t>(L) * 2304 + kHidden))) return rc;
    const size_t kv_count = static_cast<size_t>(L) * kNumKVHeads * cfg.max_context * kHeadDim;
    unsigned char* kvb = nullptr;
    if ((rc = dalloc(c, &kvb, kv_count * c->kv_elem()))) return rc;
    c->kc = kvb;
    if ((rc = dalloc(c, &kvb, kv_count * c->kv_elem()))) return rc;
    c->vc = kvb;
    HY_CUDA(cudaMemsetAsync(c->kc, 0, kv_count * c->kv_elem(), c->stream));
    HY_CUDA(cudaMemsetAsync(c->vc, 0, kv_count * c->kv_elem(), c->stream));
    const size_t rope_rows = static_cast<size_t>(cfg.max_context);
    if ((rc = dalloc(c, &c->rope_cos, rope_rows * kHeadDim))) return rc;
    if ((rc = dalloc(c, &c->rope_sin, rope_rows * kHeadDim))) return rc;
    const size_t pre_rows = static_cast<size_t>(std::max(cfg.max_prefill, kMaxStepRows));
    if ((rc = dalloc(c, &c->pre_cos, pre_rows * kHeadDim))) return rc;
    if ((rc = dalloc(c, &c->pre_pos, 4 * pre_rows))) return rc;
    if ((rc = dalloc(c, &c->pre_sin, pre_rows * kHeadDim))) return rc;
    if ((rc = dalloc(c, &c->prompt, pre_rows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->feats, pre_rows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->ids_buf, pre_rows))) return rc;
    if ((rc = dalloc(c, &c->feat_idx, pre_rows))) return rc;
    c->pf_rows = std::min(cfg.max_prefill, kPrefillChunk);
    c->pf_pad = (c->pf_rows + kUmBM - 1) / kUmBM * kUmBM;
    {
        const size_t pad = static_cast<size_t>(c->pf_pad);
        if ((rc = dalloc(c, &c->pf_qkv, static_cast<size_t>(c->pf_rows) * kQKVRows))) return rc;
        float** bufs[6] = {&c->pf_a_hi, &c->pf_a_lo, &c->pf_at_hi, &c->pf_at_lo, &c->pf_ac_hi, &c->pf_ac_lo};
        const size_t cols[6] = {kHidden, kHidden, kQWidth, kQWidth, static_cast<size_t>(ffn), static_cast<size_t>(ffn)};
        for (int i = 0; i < 6; ++i)
            if ((rc = dalloc(c, bufs[i], pad * cols[i]))) return rc;
        const size_t nqb = pad / kPaRows;
        if ((rc = dalloc(c, &c->pf_work, nqb * kPaMaxChunks))) return rc;
        if ((rc = dalloc(c, &c->pf_merge, nqb))) return rc;
        if ((rc = dalloc(c, &c->pf_part, nqb * kPaMaxChunks * kNumKVHeads * 64 * kPaPartStride))) return rc;
        if ((rc = dalloc(c, &c->va_part, static_cast<size_t>(kVerifyChunks) * kNumKVHeads * 32 * kPaPartStride)))
            return rc;
    }
    {
        // Tiled prefill weights: hi for every weight, lo for fp32 weights.
        const size_t per_layer = static_cast<size_t>(kQKVRows) * kHidden + static_cast<size_t>(kHidden) * kQWidth +
                                 static_cast<size_t>(2 * ffn) * kHidden + static_cast<size_t>(kHidden) * ffn;
        const int planes = (cfg.weight_dtype == HY_DTYPE_BF16) ? 1 : 2;
        float* tw = nullptr;
        if ((rc = dalloc(c, &tw, per_layer * L * planes))) return rc;
        for (int pl = 0; pl < planes; ++pl)
            for (int l = 0; l < L; ++l)
            {
                float* p = tw + (static_cast<size_t>(pl) * L + l) * per_layer;
                (pl ? c->tq_lo : c->tq_hi).push_back(p);
                p += static_cast<size_t>(kQKVRows) * kHidden;
                (pl ? c->to_lo : c->to_hi).push_back(p);
                p += static_cast<size_t>(kHidden) * kQWidth;
                (pl ? c->tg_lo : c->tg_hi).push_back(p);
                p += static_cast<size_t>(2 * ffn) * kHidden;
                (pl ? c->td_lo : c->td_hi).push_back(p);
            }
        if (planes == 1)
        {
            c->tq_lo.assign(L, nullptr);
            c->to_lo.assign(L, nullptr);
            c->tg_lo.assign(L, nullptr);
            c->td_lo.assign(L, nullptr);
        }
    }
    if ((rc = dalloc(c, &c->x, kMaxStepRows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->qkv, kMaxStepRows * kQKVRows))) return rc;
    if ((rc = dalloc(c, &c->attn, kMaxStepRows * kQWidth))) return rc;
    if ((rc = dalloc(c, &c->gu, static_cast<size_t>(kMaxStepRows) * 2 * ffn))) return rc;
    if ((rc = dalloc(c, &c->tmp, kMaxStepRows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->act, static_cast<size_t>(kMaxStepRows) * cfg.ffn_dim))) return rc;
    if ((rc = dalloc(c, &c->hidden, kMaxStepRows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->aux, static_cast<size_t>(kAuxLayers) * kMaxStepRows * kHidden))) return rc;
    if ((rc = dalloc(c, &c->attn_part, static_cast<size_t>(kNumKVHeads) * kMaxSplits * 2 * kMaxStepRows * kPartStride)))
        return rc;
    if ((rc = dalloc(c, &c->attn_cnt, static_cast<size_t>(L) * kNumKVHeads))) return rc;
    if ((rc = dalloc(c, &c->lm_part, static_cast<size_t>(c->num_sms) * kMaxStepRows))) return rc;
    if ((rc = dalloc(c, &c->lm_cnt, 1))) return rc;
    if ((rc = dalloc(c, &c->hist, (static_cast<size_t>(cfg.vocab_size) + 31) / 32))) return rc;
    if ((rc = dalloc(c, &c->st, 1))) return rc;
    const size_t ntok = static_cast<size_t>(cfg.max_tokens) + 2 * kBlock;
    if ((rc = dalloc(c, &c->log_tokens, ntok))) return rc;
    if ((rc = dalloc(c, &c->log_raw, ntok))) return rc;
    if ((rc = dalloc(c, &c->accept_log, ntok))) return rc;
    if ((rc = dalloc(c, &c->greedy, ntok))) return rc;
    if ((rc = dalloc(c, &c->proposed, kBlock))) return rc;
    if ((rc = dalloc(c, &c->posterior, kBlock))) return rc;
    if ((rc = dalloc(c, &c->tok_out, kBlock))) return rc;
    if ((rc = dalloc(c, &c->raw_out, kBlock))) return rc;
    if ((rc = dalloc(c, &c->prefix, kBlock))) return rc;
    if ((rc = dalloc(c, &c->err, 1))) return rc;
    if ((rc = dalloc(c, &c->dbg, 4))) return rc;
    if ((rc = dalloc(c, &c->x_ep, kHidden))) return rc;
    if ((rc = dalloc(c, &c->qkv_ep, kQKVRows))) return rc;
    if ((rc = dalloc(c, &c->act_ep, cfg.ffn_dim))) return rc;
    if ((rc = dalloc(c, &c->tok_ep, 1))) return rc;
    if ((rc = dalloc(c, &c->attn_ep, static_cast<size_t>(kNumKVHeads) * (kMegaSplits - 1) * 2 * kAttnWords))) return rc;
    if ((rc = dalloc(c, &c->attn_out_ep, kQWidth))) return rc;
    HY_CUDA(cudaMemsetAsync(c->dbg, 0, 4 * sizeof(int), c->stream));
#ifdef HY_WAIT_STATS
    if ((rc = dalloc(c, &c->wstat, kWsWords))) return rc;
    HY_CUDA(cudaMemsetAsync(c->wstat, 0, kWsWords * sizeof(unsigned long long), c->stream));
#endif
    if (const char* e = std::getenv("HY_DEBUG_PROGRESS"); e && e[0] == '1')
    {
        HY_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&c->progress), 1024 * sizeof(unsigned), cudaHostAllocMapped));
        std::memset(c->progress, 0, 1024 * sizeof(unsigned));
    }
    if ((rc = dalloc(c, &c->wptrs, static_cast<size_t>(4) * L))) return rc;
    {
        std::vector<const void*> h(4 * static_cast<size_t>(L));
        for (int l = 0; l < L; ++l)
        {
            h[l] = c->wqkv[l];
            h[L + l] = c->wo[l];
            h[2 * L + l] = c->wgu[l];
            h[3 * L + l] = c->wd[l];
        }
        HY_CUDA(cudaMemcpy(c->wptrs, h.data(), h.size() * sizeof(void*), cudaMemcpyHostToDevice));
    }
    HY_CUDA(cudaMemsetAsync(c->attn_cnt, 0, sizeof(int) * L * kNumKVHeads, c->stream));
    HY_CUDA(cudaMemsetAsync(c->lm_cnt, 0, sizeof(int), c->stream));
    HY_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
    HY_CUDA(cudaMemsetAsync(c->hist, 0, sizeof(unsigned) * ((cfg.vocab_size + 31) / 32), c->stream));
    HY_CUDA(cudaMemsetAsync(c->proposed, 0, sizeof(int) * kBlock, c->stream));
    HY_CUDA(cudaMemsetAsync(c->prefix, 0xff, sizeof(int) * kBlock, c->stream));
    HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_st), sizeof(DecodeState)));
    std::memset(c->h_st, 0, sizeof(DecodeState));
    c->h_st->penalty = 1.08f;
    if ((rc = push_state(c))) return rc;
    // Staging (see hy_ctx): prompt uploads in one pinned area, history ids, small reads.
    c->h_stage_bytes = prompt_stage_bytes(cfg.max_prefill);
    HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_stage), c->h_stage_bytes));
    HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_hist), sizeof(int) * kHistChunk));
    HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_small), sizeof(int) * 16));
    HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_log), sizeof(int) * 2 * (cfg.max_tokens + 2 * kBlock)));
    std::memset(c->h_small, 0, sizeof(int) * 16);
    if ((rc = dalloc(c, &c->hist_ids, kHistChunk))) return rc;
    if ((rc = dalloc(c, &c->kv_stage, static_cast<size_t>(cfg.max_context) * kHeadDim))) return rc;
    if ((rc = dalloc(c, &c->probe_word, 2))) return rc;
    HY_CUDA(cudaMemsetAsync(c->probe_word, 0, 2 * sizeof(unsigned long long), c->stream));
    for (int i = 0; i < kTimingEvents; ++i) HY_CUDA(cudaEventCreate(&c->tev[i]));

    // 1-D RoPE table for decode / verify positions.
    std::vector<float> cs(rope_rows * kHeadDim), sn(rope_rows * kHeadDim);
    float inv[kHeadDim];
    {
        const float base = static_cast<float>(10000.0 * std::pow(1000.0, 128.0 / 126.0));
        for (int d = 0; d < kHeadDim; ++d)
            inv[d] = 1.0f / std::pow(base, static_cast<float>(2 * (d % (kHeadDim / 2))) / static_cast<float>(kHeadDim));
    }
    for (size_t pos = 0; pos < rope_rows; ++pos)
        for (int d = 0; d < kHeadDim; ++d)
        {
            const float angle = static_cast<float>(static_cast<int>(pos)) * inv[d];
            cs[pos * kHeadDim + d] = std::cos(angle);
            sn[pos * kHeadDim + d] = std::sin(angle);
        }
    HY_CUDA(cudaMemcpy(c->rope_cos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
    HY_CUDA(cudaMemcpy(c->rope_sin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
    return HY_OK;
}

template <typename WT>
void launch_synth(WT* out, size_t count, unsigned long long seed, unsigned long long tid, float std_dev, float offset,
                  cudaStream_t s)
{
    synth_fill_kernel<WT><<<1184, 256, 0, s>>>(out, count, synth_base(seed, tid), host_synth_mult(std_dev), offset);
}

int fill_synthetic(hy_ctx* c, unsigned long long seed, float std_dev, float norm_std)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    auto lin = [&](void* dst, size_t off_elems, unsigned long long tid, size_t count) {
        if (cfg.weight_dtype == HY_DTYPE_BF16)
            launch_synth(static_cast<__nv_bfloat16*>(dst) + off_elems, count, seed, tid, std_dev, 0.f, c->stream);
        else
            launch_synth(static_cast<float*>(dst) + off_elems, count, seed, tid, std_dev, 0.f, c->stream);
    };
    auto lin_rows = [&](void* dst, unsigned long long tid, int rows, int cols, int row_mult, int row_off) {
        const unsigned long long base = synth_base(seed, tid);
        const float mult = host_synth_mult(std_dev);
        if (cfg.weight_dtype == HY_DTYPE_BF16)
            synth_fill_rows_kernel<__nv_bfloat16><<<1184, 256, 0, c->stream>>>(static_cast<__nv_bfloat16*>(dst), rows, cols,
                                                                               row_mult, row_off, base, mult);
        else
            synth_fill_rows_kernel<float><<<1184, 256, 0, c->stream>>>(static_cast<float*>(dst), rows, cols, row_mult,
                                                                       row_off, base, mult);
    };
    lin(c->embed, 0, kTidEmbed, static_cast<size_t>(cfg.vocab_size) * kHidden);
    launch_synth(c->final_norm(), kHidden, seed, kTidFinalNorm, norm_std, 1.0f, c->stream);
    for (int l = 0; l < cfg.num_layers; ++l)
    {
        const unsigned long long b = kLayerTidBase + kLayerTidStride * l;
        launch_synth(c->in_norm(l), kHidden, seed, b + J_INPUT_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->post_norm(l), kHidden, seed, b + J_POST_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->qn(l), kHeadDim, seed, b + J_Q_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->kn(l), kHeadDim, seed, b + J_K_NORM, norm_std, 1.0f, c->stream);
        lin(c->wqkv[l], 0, b + J_Q, static_cast<size_t>(kQWidth) * kHidden);
        lin(c->wqkv[l], static_cast<size_t>(kQWidth) * kHidden, b + J_K, static_cast<size_t>(kKVWidth) * kHidden);
        lin(c->wqkv[l], static_cast<size_t>(kQWidth + kKVWidth) * kHidden, b + J_V,
            static_cast<size_t>(kKVWidth) * kHidden);
        lin(c->wo[l], 0, b + J_O, static_cast<size_t>(kHidden) * kQWidth);
        // gate_proj row j -> row 2j, up_proj row j -> row 2j + 1 (SwiGLU pairs stay together).
        lin_rows(c->wgu[l], b + J_GATE, ffn, kHidden, 2, 0);
        lin_rows(c->wgu[l], b + J_UP, ffn, kHidden, 2, 1);
        lin(c->wd[l], 0, b + J_DOWN, static_cast<size_t>(kHidden) * ffn);
    }
    HY_CUDA(cudaGetLastError());
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

int upload_weights(hy_ctx* c, const hy_weights* w)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    if (!w || !w->embed || !w->final_norm || !w->layers) return fail(HY_ERR_INVALID_ARGUMENT, "weights are incomplete");
    for (int l = 0; l < cfg.num_layers; ++l)
    {
        const hy_layer_weights& lw = w->layers[l];
        if (!lw.input_norm || !lw.q_proj || !lw.k_proj || !lw.v_proj || !lw.query_norm || !lw.key_norm || !lw.o_proj ||
            !lw.post_norm || !lw.gate_proj || !lw.up_proj || !lw.down_proj)
            return fail(HY_ERR_INVALID_ARGUMENT, "layer " + std::to_string(l) + " weights are incomplete");
    }
    float* staging = nullptr;
    const bool bf = cfg.weight_dtype == HY_DTYPE_BF16;
    if (bf)
    {
        void* s = nullptr;
        HY_CUDA(cudaMalloc(&s, static_cast<size_t>(std::max(cfg.vocab_size, 2 * ffn)) * kHidden * sizeof(float)));
        staging = static_cast<float*>(s);
    }
    auto put = [&](void* dst, size_t off_elems, const float* src, size_t count) -> cudaError_t {
        if (!bf)
            return cudaMemcpy(static_cast<float*>(dst) + off_elems, src, count * sizeof(float), cudaMemcpyHostToDevice);
        cudaError_t e = cudaMemcpy(staging, src, count * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        f32_to_bf16_kernel<<<1184, 256, 0, c->stream>>>(staging, static_cast<__nv_bfloat16*>(dst) + off_elems, count);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        return cudaStreamSynchronize(c->stream);
    };
    // rows r of src -> rows 2r + off of dst (gate/up interleave).
    auto put_rows = [&](void* dst, const float* src, int rows, int off) -> cudaError_t {
        const size_t es = bf ? 2 : 4;
        if (!bf)
            return cudaMemcpy2D(static_cast<char*>(dst) + static_cast<size_t>(off) * kHidden * es, 2 * kHidden * es, src,
                                kHidden * sizeof(float), kHidden * sizeof(float), rows, cudaMemcpyHostToDevice);
        cudaError_t e = cudaMemcpy(staging, src, static_cast<size_t>(rows) * kHidden * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        f32_to_bf16_rows_kernel<<<1184, 256, 0, c->stream>>>(staging, static_cast<__nv_bfloat16*>(dst), rows, kHidden, 2, off);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        return cudaStreamSynchronize(c->stream);
    };
    cudaError_t e = put(c->embed, 0, w->embed, static_cast<size_t>(cfg.vocab_size) * kHidden);
    for (int l = 0; l < cfg.num_layers && e == cudaSuccess; ++l)
    {
        const hy_layer_weights& lw = w->layers[l];
        e = put(c->wqkv[l], 0, lw.q_proj, static_cast<size_t>(kQWidth) * kHidden);
        if (e == cudaSuccess) e = put(c->wqkv[l], static_cast<size_t>(kQWidth) * kHidden, lw.k_proj, static_cast<size_t>(kKVWidth) * kHidden);
        if (e == cudaSuccess)
            e = put(c->wqkv[l], static_cast<size_t>(kQWidth + kKVWidth) * kHidden, lw.v_proj, static_cast<size_t>(kKVWidth) * kHidden);
        if (e == cudaSuccess) e = put(c->wo[l], 0, lw.o_proj, static_cast<size_t>(kHidden) * kQWidth);
        if (e == cudaSuccess) e = put_rows(c->wgu[l], lw.gate_proj, ffn, 0);
        if (e == cudaSuccess) e = put_rows(c->wgu[l], lw.up_proj, ffn, 1);
        if (e == cudaSuccess) e = put(c->wd[l], 0, lw.down_proj, static_cast<size_t>(kHidden) * ffn);
        if (e == cudaSuccess) e = cudaMemcpy(c->in_norm(l), lw.input_norm, kHidden * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->post_norm(l), lw.post_norm, kHidden * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->qn(l), lw.query_norm, kHeadDim * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->kn(l), lw.key_norm, kHeadDim * sizeof(float), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMemcpy(c->final_norm(), w->final_norm, kHidden * sizeof(float), cudaMemcpyHostToDevice);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
    return HY_OK;
}

void free_ctx(hy_ctx* c)
{
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->g_ar) cudaGraphExecDestroy(c->g_ar);
    if (c->g_verify_draft) cudaGraphExecDestroy(c->g_verify_draft);
    if (c->g_verify_ids) cudaGraphExecDestroy(c->g_verify_ids);
    for (int b = 0; b < kDflashGraphs; ++b)
    {
        if (c->g_dflash[b]) cudaGraphExecDestroy(c->g_dflash[b]);
        for (cudaEvent_t e : c->dflash_ev[b])
            if (e) cudaEventDestroy(e);
    }
    if (c->g_verify_ids_ctx) cudaGraphExecDestroy(c->g_verify_ids_ctx);
    if (c->g_batch) cudaGraphExecDestroy(c->g_batch);
    for (void* p : c->d_allocs) cudaFree(p);
    for (void* p : c->b_allocs) cudaFree(p);
    if (c->h_bstate) cudaFreeHost(c->h_bstate);
    for (void* p : c->allocs) cudaFree(p);
    if (c->logits) cudaFree(c->logits);
    if (c->h_st) cudaFreeHost(c->h_st);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->h_hist) cudaFreeHost(c->h_hist);
    if (c->h_small) cudaFreeHost(c->h_small);
    if (c->h_log) cudaFreeHost(c->h_log);
    for (cudaEvent_t e : c->tev)
        if (e) cudaEventDestroy(e);
    if (c->progress) cudaFreeHost(c->progress);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

// Splits and tiles every decoder weight for the prefill GEMMs (after the
// weights are loaded or synthesised).
template <typename WT>
int tile_weights_t(hy_ctx* c)
{
    const int L = c->cfg.num_layers, ffn = c->cfg.ffn_dim;
    for (int l = 0; l < L; ++l)
    {
        const void* src[4] = {c->wqkv[l], c->wo[l], c->wgu[l], c->wd[l]};
        float* hi[4] = {c->tq_hi[l], c->to_hi[l], c->tg_hi[l], c->td_hi[l]};
        float* lo[4] = {c->tq_lo[l], c->to_lo[l], c->tg_lo[l], c->td_lo[l]};
        const int R[4] = {kQKVRows, kHidden, 2 * ffn, kHidden}, K[4] = {kHidden, kQWidth, kHidden, ffn};
        for (int i = 0; i < 4; ++i)
        {
            const size_t n = static_cast<size_t>(R[i]) * (K[i] / 4);
            tile_weight_kernel<WT><<<static_cast<unsigned>((n + 255) / 256), 256, 0, c->stream>>>(
                static_cast<const WT*>(src[i]), R[i], K[i], hi[i], lo[i]);
            HY_CUDA(cudaGetLastError());
        }
    }
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

// Tensor map of the tied table [vocab x 1024] for the 16-row LM head: boxes of
// 128 bytes of a row x 128 rows, 128-byte swizzle (conflict-free fragment reads
// without padding), rows past the table zero-filled. cuTensorMapEncodeTiled is
// taken from the driver through the runtime's entry-point query.
int encode_lm_tmap(hy_ctx* c)
{
    using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    HY_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) return fail(HY_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const bool bf = c->cfg.weight_dtype == HY_DTYPE_BF16;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHidden), static_cast<cuuint64_t>(c->cfg.vocab_size)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHidden) * c->w_elem()};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / c->w_elem()), 128};
    const cuuint32_t estr[2] = {1, 1};
    std::memset(&c->lm_tmap, 0, sizeof(c->lm_tmap));
    const CUresult r = reinterpret_cast<EncodeFn>(fn)(
        &c->lm_tmap, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, c->embed, dims,
        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HY_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    return HY_OK;
}

int finish_create(hy_ctx* c, hy_ctx** out)
{
    int rc = (c->cfg.weight_dtype == HY_DTYPE_BF16) ? tile_weights_t<__nv_bfloat16>(c) : tile_weights_t<float>(c);
    if (!rc) rc = encode_lm_tmap(c);
    if (rc)
    {
        free_ctx(c);
        return rc;
    }
    rc = ensure_graphs(c);
    if (rc)
    {
        free_ctx(c);
        return rc;
    }
    *out = c;
    return HY_OK;
}

int set_device(hy_ctx* c)
{
    HY_CUDA(cudaSetDevice(c->cfg.device));
    return HY_OK;
}

// One step outside a graph (prefill chunks, hy_decoder_step): rows of ctx->x at
// explicit positions past..past+rows-1 with explicit rope rows.
int run_direct_step(hy_ctx* c, int rows, int past, const float* cos, const float* sin, float** aux, int ld_aux = 0)
{
    StepPlan p{};
    p.rows = rows;
    p.source.src = SRC_X;
    p.cos = cos;
    p.sin = sin;
    p.rope_state = 0;
    p.past_from_state = false;
    p.past_fixed = past;
    p.lm_mode = -1;
    p.aux = aux;
    p.ld_aux = ld_aux;
    t_next_plain = true;   // the rows were just copied into ctx->x
    cudaError_t e = enqueue_step(c, p);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("decoder step launch: ") + cudaGetErrorString(e));
    return HY_OK;
}

template <int EPI, int BN, bool B_SPLIT>
cudaError_t run_umma_gemm_bn(hy_ctx* c, const UmmaGemmArgs& a)
{
    using S = UmShape<BN, B_SPLIT>;
    auto k = umma_gemm_kernel<EPI, BN, B_SPLIT>;
    static unsigned long long configured = 0;
    const unsigned long long bit = 1ull << (c->cfg.device & 63);
    if (!(configured & bit))
    {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    k<<<dim3(a.N / BN, (a.M + kUmBM - 1) / kUmBM), kUmThreads, S::SMEM, c->stream>>>(a);
    return cudaGetLastError();
}

// C = A . W^T on the tcgen05 tensor cores from split, tiled operands; 128 x 128
// output tiles, or 128 x 64 when N is small (1024 rows: 2x the CTAs).
template <int EPI>
cudaError_t run_prefill_gemm(hy_ctx* c, UmmaGemmArgs a)
{
    if (a.M <= 0 || a.N % 64 != 0 || a.K % kUmBK != 0 || a.a_rows % kUmBM != 0 || a.a_rows < a.M)
        return cudaErrorInvalidValue;
    a.err = c->err;
    const bool split = a.w_lo != nullptr;
    if (a.N % 128 == 0 && a.N > 2048)
        return split ? run_umma_gemm_bn<EPI, 128, true>(c, a) : run_umma_gemm_bn<EPI, 128, false>(c, a);
    return split ? run_umma_gemm_bn<EPI, 64, true>(c, a) : run_umma_gemm_bn<EPI, 64, false>(c, a);
}

UmmaGemmArgs gemm_args(const float* a_hi, const float* a_lo, int a_rows, const float* w_hi, const float* w_lo, int M,
                       int N, int K)
{
    UmmaGemmArgs g;
    std::memset(&g, 0, sizeof(g));
    g.a_hi = a_hi;
    g.a_lo = a_lo;
    g.a_rows = a_rows;
    g.w_hi = w_hi;
    g.w_lo = w_lo;
    g.M = M;
    g.N = N;
    g.K = K;
    return g;
}

template <typename KT>
cudaError_t run_prefill_attn(hy_ctx* c, const float* q, int ldq, int layer, int past, int rows, int rows_pad)
{
    using S = PaShape<KT, kPaRows>;
    auto k = prefill_attn_kernel<KT, kPaRows>;
    static unsigned long long configured = 0;
    const unsigned long long bit = 1ull << (c->cfg.device & 63);
    if (!(configured & bit))
    {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
        if (e != cudaSuccess) return e;
        configured |= bit;
    }
    PrefillAttnArgs a{q, ldq, c->kc_layer(layer), c->vc_layer(layer), c->cfg.max_context, past, rows,
                      c->pf_at_hi, c->pf_at_lo, rows_pad, c->pf_work, c->pf_part, nullptr, c->err};
    k<<<dim3(c->pf_nwork, kNumKVHeads), S::THREADS, S::SMEM, c->stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || c->pf_nmerge == 0) return e;
    prefill_attn_merge_kernel<<<dim3(c->pf_nmerge, kNumKVHeads), 256, 0, c->stream>>>(c->pf_part, c->pf_merge, rows,
                                                                                     rows_pad, c->pf_at_hi, c->pf_at_lo);
    return cudaGetLastError();
}

// Work items of the prefill attention for one pass (rows at positions past ..):
// each 32-row block's keys [0, past + block end) in chunks of at least 8 tiles
// of 32 keys and at most kPaMaxChunks chunks per block, longest blocks first.
cudaError_t plan_prefill_attn(hy_ctx* c, int past, int rows)
{
    const int nqb = (rows + kPaRows - 1) / kPaRows;
    const int max_nkb = (past + rows + kPaKeys - 1) / kPaKeys;
    const int ckb = std::max(kPaMinChunkTiles, (max_nkb + kPaMaxChunks - 1) / kPaMaxChunks);
    c->h_work.clear();
    c->h_merge.clear();
    int slot = 0;
    for (int qb = nqb - 1; qb >= 0; --qb)
    {
        const int nkeys = std::min(past + qb * kPaRows + kPaRows, past + rows);
        const int nkb = (nkeys + kPaKeys - 1) / kPaKeys;
        const int nch = (nkb + ckb - 1) / ckb;
        if (nch == 1)
        {
            c->h_work.push_back(make_int4(qb, 0, nkb, -1));
            continue;
        }
        c->h_merge.push_back(make_int4(qb, slot, nch, 0));
        for (int ch = 0; ch < nch; ++ch)
            c->h_work.push_back(make_int4(qb, ch * ckb, std::min(nkb, (ch + 1) * ckb), slot++));
    }
    c->pf_nwork = static_cast<int>(c->h_work.size());
    c->pf_nmerge = static_cast<int>(c->h_merge.size());
    cudaError_t e = cudaMemcpyAsync(c->pf_work, c->h_work.data(), sizeof(int4) * c->h_work.size(),
                                    cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess || c->h_merge.empty()) return e;
    return cudaMemcpyAsync(c->pf_merge, c->h_merge.data(), sizeof(int4) * c->h_merge.size(), cudaMemcpyHostToDevice,
                           c->stream);
}

// Prompt prefill: the decoder over rows [0, seq) of ctx->prompt (the residual
// stream, updated in place), in passes of up to pf_rows rows through all
// layers; rope rows come from pre_cos / pre_sin. Per layer: RMSNorm (written
// split and tiled), the q/k/v GEMM, RoPE + QK norm + KV append of every row,
// causal attention of the pass's rows over the cache, then o_proj (residual
// add), RMSNorm, gate/up with SwiGLU (written split and tiled) and down_proj
// (residual add). Leaves the final-normed last row in ctx->hidden.
cudaError_t enqueue_draft_context_rows(hy_ctx* c, int rows, int past);

template <typename KT>
cudaError_t enqueue_prefill_t(hy_ctx* c, int seq)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    cudaError_t e = cudaSuccess;
    for (int p0 = 0; p0 < seq; p0 += c->pf_rows)
    {
        const int rows = std::min(c->pf_rows, seq - p0);
        const int pad = (rows + kUmBM - 1) / kUmBM * kUmBM;
        float* xr = c->prompt + static_cast<size_t>(p0) * kHidden;
        if ((e = plan_prefill_attn(c, p0, rows)) != cudaSuccess) return e;
        for (int l = 0; l < cfg.num_layers; ++l)
        {
            rmsnorm_tiled_kernel<<<rows, 256, 0, c->stream>>>(xr, c->in_norm(l), cfg.rms_norm_eps, pad, c->pf_a_hi,
                                                               c->pf_a_lo);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            UmmaGemmArgs q = gemm_args(c->pf_a_hi, c->pf_a_lo, pad, c->tq_hi[l], c->tq_lo[l], rows, kQKVRows, kHidden);
            q.C = c->pf_qkv;
            q.ldc = kQKVRows;
            if ((e = run_prefill_gemm<UG_STORE>(c, q)) != cudaSuccess) return e;
            PrefillRopeArgs ra{c->pf_qkv, kQKVRows,
                               c->pre_cos + static_cast<size_t>(p0) * kHeadDim,
                               c->pre_sin + static_cast<size_t>(p0) * kHeadDim,
                               c->qn(l), c->kn(l), c->kc_layer(l), c->vc_layer(l), cfg.max_context, p0,
                               cfg.rms_norm_eps, cfg.attn_scale * 1.4426950408889634f, nullptr, 0, c->err};
            prefill_rope_kernel<KT><<<dim3(rows, 4), 256, 0, c->stream>>>(ra);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            if ((e = run_prefill_attn<KT>(c, c->pf_qkv, kQKVRows, l, p0, rows, pad)) != cudaSuccess) return e;
            UmmaGemmArgs o = gemm_args(c->pf_at_hi, c->pf_at_lo, pad, c->to_hi[l], c->to_lo[l], rows, kHidden, kQWidth);
            o.C = xr;
            o.ldc = kHidden;
            if ((e = run_prefill_gemm<UG_RESID>(c, o)) != cudaSuccess) return e;
            rmsnorm_tiled_kernel<<<rows, 256, 0, c->stream>>>(xr, c->post_norm(l), cfg.rms_norm_eps, pad, c->pf_a_hi,
                                                               c->pf_a_lo);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            UmmaGemmArgs gu = gemm_args(c->pf_a_hi, c->pf_a_lo, pad, c->tg_hi[l], c->tg_lo[l], rows, 2 * ffn, kHidden);
            gu.act_hi = c->pf_ac_hi;
            gu.act_lo = c->pf_ac_lo;
            if ((e = run_prefill_gemm<UG_SWIGLU_TILED>(c, gu)) != cudaSuccess) return e;
            UmmaGemmArgs d = gemm_args(c->pf_ac_hi, c->pf_ac_lo, pad, c->td_hi[l], c->td_lo[l], rows, kHidden, ffn);
            d.C = xr;
            d.ldc = kHidden;
            if ((e = run_prefill_gemm<UG_RESID>(c, d)) != cudaSuccess) return e;
            // With a DFlash draft: this layer's output rows as draft context input.
            for (int i = 0; i < kAuxLayers && c->d_layers > 0; ++i)
                if (kAuxLayerIds[i] == l &&
                    (e = cudaMemcpy2DAsync(c->d_pf_aux + i * kHidden, sizeof(float) * kAuxLayers * kHidden, xr,
                                           sizeof(float) * kHidden, sizeof(float) * kHidden, rows,
                                           cudaMemcpyDeviceToDevice, c->stream)) != cudaSuccess)
                    return e;
        }
        if (c->d_layers > 0 && (e = enqueue_draft_context_rows(c, rows, p0)) != cudaSuccess) return e;
        if (p0 + rows == seq)
        {
            rmsnorm_rows_kernel<<<1, 256, 0, c->stream>>>(xr + static_cast<size_t>(rows - 1) * kHidden, c->final_norm(),
                                                         cfg.rms_norm_eps, c->hidden, kHidden);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
    }
    t_next_plain = true;
    return cudaSuccess;
}

int run_prefill(hy_ctx* c, int seq)
{
    const cudaError_t e = (c->cfg.kv_dtype == HY_DTYPE_BF16) ? enqueue_prefill_t<__nv_bfloat16>(c, seq)
                                                             : enqueue_prefill_t<float>(c, seq);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("prefill launch: ") + cudaGetErrorString(e));
    return HY_OK;
}

int set_length(hy_ctx* c, int rows)
{
    c->h_st->kv_len = rows;
    c->kv_len = rows;
    HY_CUDA(cudaMemcpyAsync(&c->st->kv_len, &c->h_st->kv_len, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

// ---------------------------------------------------------------------------
// DFlash draft network: the graph of export/dflash_export.py:88-177, run by
// DFlashDraftRuntime::run (src/dflash_runtime.cpp:213-290) from
// run_dflash_block (src/text_runtime.cpp:880-950).
//
// The reference hands the draft graph the aux hidden states of every context
// row on every block, and the graph recomputes fc / hidden_norm / k_proj /
// v_proj over all of them. A context row's draft keys and values depend only
// on that row and its position, so here they are computed once, when the row
// joins the sequence, and kept in a draft K/V cache beside the decoder's:
//   context rows: th = hidden_norm(fc(aux_1 | aux_8 | aux_15 | aux_22)); per
//     draft layer k = rope(k_norm(k_proj(th))), v = v_proj(th) at the row's
//     position (RoPE theta 10000, build_dflash_rope, src/dflash_runtime.cpp:27-48);
//   noise block (16 rows at positions len .. len + 15): per draft layer q / k /
//     v of RMSNorm(h), q_norm / k_norm then RoPE, the rows' k / v written after
//     the context, attention over keys [0, len + 16) with no mask and scale
//     1/sqrt(128), o_proj + residual, SwiGLU MLP + residual; final norm;
//   drafts: argmax of the tied LM head over rows 1 .. 15 (penalty 1, no history).
// A prompt's context rows go through the tcgen05 GEMMs (split, tiled operands);
// a step's (<= 16 rows, e.g. a verify block) through the 16-row projections.
// ---------------------------------------------------------------------------
constexpr unsigned long long kTidDraftFc = 19990, kTidDraftHiddenNorm = 19991, kTidDraftNorm = 19992;
constexpr unsigned long long kDraftTidBase = 20000, kDraftTidStride = 16;
constexpr int kMaxDraftLayers = 8;
constexpr int kAuxWidth = kAuxLayers * kHidden;   // 4096: the fc input row
const float kDraftScaleLog2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kHeadDim)));

bool draft_ready(const hy_ctx* c) { return c->d_layers > 0; }

// Context rows of a step: aux rows [rows x 4096] at `aux` (rows <= 16), KV
// positions past .. past + rows - 1 (past = st->kv_len when from_state).
template <typename WT, typename KT>
cudaError_t enqueue_draft_context16_t(hy_ctx* c, const float* aux, int rows, bool from_state, int past)
{
    cudaError_t e = cudaSuccess;
    // fc over the two column halves (the 16 activation rows of 2048 columns fit in
    // shared memory): tmp = aux[:, :2048] fc[:, :2048]^T, then tmp += aux[:, 2048:] fc[:, 2048:]^T.
    GemvArgs f = base_args(c);
    f.W = c->d_fc;
    f.N = kHidden;
    f.ldw = kAuxWidth;
    f.rows = rows;
    f.src = SRC_X;
    f.x = aux;
    f.ldx = kAuxWidth;
    f.out = c->tmp;
    f.ldo = kHidden;
    f.k_off = 0;
    if ((e = run_gemv<WT, kAuxWidth / 2, 16, PRO_PLAIN, EPI_STORE>(c, f)) != cudaSuccess) return e;
    f.k_off = kAuxWidth / 2;
    if ((e = run_gemv<WT, kAuxWidth / 2, 16, PRO_PLAIN, EPI_RESID>(c, f)) != cudaSuccess) return e;
    for (int l = 0; l < c->d_layers; ++l)
    {
        // k | v = hidden_norm(tmp) [k_proj; v_proj]^T into columns 2048.. of the qkv rows.
        GemvArgs kv = base_args(c);
        kv.W = static_cast<const WT*>(c->d_wqkv[l]) + static_cast<size_t>(kQWidth) * kHidden;
        kv.N = 2 * kKVWidth;
        kv.ldw = kHidden;
        kv.rows = rows;
        kv.src = SRC_X;
        kv.x = c->tmp;
        kv.ldx = kHidden;
        kv.norm_w = c->d_hidden_norm();
        kv.out = c->qkv + kQWidth;
        kv.ldo = kQKVRows;
        if ((e = run_gemv<WT, kHidden, 16, PRO_NORM, EPI_STORE>(c, kv)) != cudaSuccess) return e;
        PrefillRopeArgs ra{c->qkv, kQKVRows, c->d_cos, c->d_sin, c->d_qn(l), c->d_kn(l), c->d_kc_layer(l),
                           c->d_vc_layer(l), c->cfg.max_context, past, c->cfg.rms_norm_eps, kDraftScaleLog2,
                           from_state ? c->st : nullptr, 1, c->err, 1, 1};
        if ((e = launch_pdl(prefill_rope_kernel<KT>, dim3(rows, 2), dim3(256), 0, c->stream, ra)) != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

// The 16 noise rows through the draft layers. src: SRC_GATHER_BLOCK (embed
// [st->cur_token, mask x 15], ids written to ctx->proposed) or SRC_X (rows
// already in d_x). select: drafts into ctx->proposed[1..15]; else the
// final-normed rows into ctx->hidden.
template <typename WT, typename KT>
cudaError_t enqueue_draft_forward_t(hy_ctx* c, int src, bool from_state, int past, bool select)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < c->d_layers; ++l)
    {
        GemvArgs q = base_args(c);
        q.W = c->d_wqkv[l];
        q.N = kQKVRows;
        q.ldw = kHidden;
        q.rows = kBlock;
        q.src = (l == 0) ? src : SRC_X;
        q.mask_token = c->d_mask;
        q.ids_out = (l == 0 && src == SRC_GATHER_BLOCK) ? c->proposed : nullptr;
        q.x_store = c->d_x;
        q.x = c->d_x;
        q.ldx = kHidden;
        q.norm_w = c->d_in_norm(l);
        q.out = c->qkv;
        q.ldo = kQKVRows;
        if ((e = run_gemv<WT, kHidden, 16, PRO_NORM, EPI_STORE>(c, q)) != cudaSuccess) return e;

        AttnArgs at;
        std::memset(&at, 0, sizeof(at));
        at.qkv = c->qkv;
        at.ldq = kQKVRows;
        at.qn_w = c->d_qn(l);
        at.kn_w = c->d_kn(l);
        at.cos = c->d_cos;
        at.sin = c->d_sin;
        at.rope_state = 1;
        at.kc = c->d_kc_layer(l);
        at.vc = c->d_vc_layer(l);
        at.cap = cfg.max_context;
        at.st = from_state ? c->st : nullptr;
        at.past_fixed = past;
        at.rows = kBlock;
        at.scale_log2 = kDraftScaleLog2;
        at.eps = cfg.rms_norm_eps;
        at.out = c->attn;
        at.err = c->err;
        if ((e = run_attn16<KT>(c, at, true)) != cudaSuccess) return e;

        GemvArgs o = base_args(c);
        o.W = c->d_wo[l];
        o.N = kHidden;
        o.ldw = kQWidth;
        o.rows = kBlock;
        o.src = SRC_X;
        o.x = c->attn;
        o.ldx = kQWidth;
        o.out = c->d_x;
        o.ldo = kHidden;
        if ((e = run_gemv<WT, kQWidth, 16, PRO_PLAIN, EPI_RESID>(c, o)) != cudaSuccess) return e;

        GemvArgs gu = base_args(c);
        gu.W = c->d_wgu[l];
        gu.N = 2 * ffn;
        gu.ldw = kHidden;
        gu.rows = kBlock;
        gu.src = SRC_X;
        gu.x = c->d_x;
        gu.ldx = kHidden;
        gu.norm_w = c->d_post_norm(l);
        gu.out = c->act;
        gu.ldo = ffn;
        if ((e = run_gemv<WT, kHidden, 16, PRO_NORM, EPI_ACT>(c, gu)) != cudaSuccess) return e;

        GemvArgs d = base_args(c);
        d.W = c->d_wd[l];
        d.N = kHidden;
        d.ldw = ffn;
        d.rows = kBlock;
        d.src = SRC_X;
        d.x = c->act;
        d.ldx = ffn;
        GemvArgs d1 = d;
        d1.k_off = 0;
        d1.out = c->tmp;
        d1.ldo = kHidden;
        if ((e = run_gemv<WT, kFfn / 2, 16, PRO_PLAIN, EPI_STORE>(c, d1)) != cudaSuccess) return e;
        GemvArgs d2 = d;
        d2.k_off = kFfn / 2;
        d2.out = c->d_x;
        d2.ldo = kHidden;
        d2.extra = c->tmp;
        if ((e = run_gemv<WT, kFfn / 2, 16, PRO_PLAIN, EPI_RESID>(c, d2)) != cudaSuccess) return e;
    }
    if (!select)
    {
        rmsnorm_rows_kernel<<<kBlock, 256, 0, c->stream>>>(c->d_x, c->d_final_norm(), cfg.rms_norm_eps, c->hidden,
                                                          kHidden);
        t_next_plain = true;
        return cudaGetLastError();
    }
    // Drafts: final norm + tied LM head + argmax of rows 1..15 (run_dflash_block,
    // src/text_runtime.cpp:951-978: penalty 1, so the history bits change nothing).
    GemvArgs lm = base_args(c);
    lm.W = c->embed;
    lm.N = cfg.vocab_size;
    lm.ldw = kHidden;
    lm.rows = kBlock - 1;
    lm.src = SRC_X;
    lm.x = c->d_x + kHidden;
    lm.ldx = kHidden;
    lm.norm_w = c->d_final_norm();
    lm.lm_mode = LM_NONE;
    lm.penalty = 1.0f;
    lm.tok_out = c->proposed + 1;
    lm.raw_out = c->raw_out;
    return run_gemv<WT, kHidden, 16, PRO_NORM, EPI_ARGMAX>(c, lm);
}

// Context rows of a prefill pass: aux rows [rows x 4096] in d_pf_aux (rows <=
// pf_rows) at KV positions past .., through the tcgen05 GEMMs.
template <typename KT>
cudaError_t enqueue_draft_context_rows_t(hy_ctx* c, int rows, int past)
{
    const hy_config& cfg = c->cfg;
    const int pad = (rows + kUmBM - 1) / kUmBM * kUmBM;
    cudaError_t e = cudaSuccess;
    split_tiled_kernel<<<rows, 256, 0, c->stream>>>(c->d_pf_aux, kAuxWidth, pad, c->d_pf_a_hi, c->d_pf_a_lo);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    UmmaGemmArgs f = gemm_args(c->d_pf_a_hi, c->d_pf_a_lo, pad, c->d_tfc_hi, c->d_tfc_lo, rows, kHidden, kAuxWidth);
    f.C = c->d_pf_fc;
    f.ldc = kHidden;
    if ((e = run_prefill_gemm<UG_STORE>(c, f)) != cudaSuccess) return e;
    rmsnorm_tiled_kernel<<<rows, 256, 0, c->stream>>>(c->d_pf_fc, c->d_hidden_norm(), cfg.rms_norm_eps, pad, c->pf_a_hi,
                                                       c->pf_a_lo);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    for (int l = 0; l < c->d_layers; ++l)
    {
        UmmaGemmArgs kv = gemm_args(c->pf_a_hi, c->pf_a_lo, pad, c->d_tkv_hi[l], c->d_tkv_lo[l], rows, 2 * kKVWidth,
                                    kHidden);
        kv.C = c->pf_qkv + kQWidth;
        kv.ldc = kQKVRows;
        if ((e = run_prefill_gemm<UG_STORE>(c, kv)) != cudaSuccess) return e;
        PrefillRopeArgs ra{c->pf_qkv, kQKVRows, c->d_cos, c->d_sin, c->d_qn(l), c->d_kn(l), c->d_kc_layer(l),
                           c->d_vc_layer(l), cfg.max_context, past, cfg.rms_norm_eps, kDraftScaleLog2, nullptr, 1,
                           c->err, 1, 1};
        prefill_rope_kernel<KT><<<dim3(rows, 2), 256, 0, c->stream>>>(ra);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    t_next_plain = true;
    return cudaSuccess;
}

cudaError_t enqueue_draft_context_rows(hy_ctx* c, int rows, int past)
{
    return (c->cfg.kv_dtype == HY_DTYPE_BF16) ? enqueue_draft_context_rows_t<__nv_bfloat16>(c, rows, past)
                                              : enqueue_draft_context_rows_t<float>(c, rows, past);
}

cudaError_t enqueue_draft_context16(hy_ctx* c, const float* aux, int rows, bool from_state, int past)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    if (!wb && !kb) return enqueue_draft_context16_t<float, float>(c, aux, rows, from_state, past);
    if (!wb && kb) return enqueue_draft_context16_t<float, __nv_bfloat16>(c, aux, rows, from_state, past);
    if (wb && !kb) return enqueue_draft_context16_t<__nv_bfloat16, float>(c, aux, rows, from_state, past);
    return enqueue_draft_context16_t<__nv_bfloat16, __nv_bfloat16>(c, aux, rows, from_state, past);
}

cudaError_t enqueue_draft_forward(hy_ctx* c, int src, bool from_state, int past, bool select)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    if (!wb && !kb) return enqueue_draft_forward_t<float, float>(c, src, from_state, past, select);
    if (!wb && kb) return enqueue_draft_forward_t<float, __nv_bfloat16>(c, src, from_state, past, select);
    if (wb && !kb) return enqueue_draft_forward_t<__nv_bfloat16, float>(c, src, from_state, past, select);
    return enqueue_draft_forward_t<__nv_bfloat16, __nv_bfloat16>(c, src, from_state, past, select);
}

// One verify block at the state's length whose draft context rows are
// appended before the commit (the commit moves the length; the block's rows
// past the committed ones are rewritten by the next block before any read).
// With `draft`, the block's ids come from the draft network first.
// ev (nullable): stage events recorded inside the captured graph (block start,
// draft done, verify and context rows done).
cudaError_t enqueue_verify_with_context(hy_ctx* c, bool draft, cudaEvent_t* ev = nullptr)
{
    cudaError_t e = cudaSuccess;
    if (ev && (e = cudaEventRecordWithFlags(ev[0], c->stream, cudaEventRecordExternal)) != cudaSuccess) return e;
    if (draft && (e = enqueue_draft_forward(c, SRC_GATHER_BLOCK, true, 0, true)) != cudaSuccess) return e;
    if (ev && (e = cudaEventRecordWithFlags(ev[1], c->stream, cudaEventRecordExternal)) != cudaSuccess) return e;
    float* aux[kAuxLayers];
    for (int i = 0; i < kAuxLayers; ++i) aux[i] = c->d_aux + i * kHidden;
    StepPlan p{};
    p.rows = kBlock;
    p.source.src = SRC_GATHER_IDS;
    p.source.ids = c->proposed;
    p.cos = c->rope_cos;
    p.sin = c->rope_sin;
    p.rope_state = 1;
    p.past_from_state = true;
    p.lm_mode = -1;
    p.aux = aux;
    p.ld_aux = kAuxWidth;
    if ((e = enqueue_step(c, p)) != cudaSuccess) return e;
    if ((e = enqueue_draft_context16(c, c->d_aux, kBlock, true, 0)) != cudaSuccess) return e;
    if (ev && (e = cudaEventRecordWithFlags(ev[2], c->stream, cudaEventRecordExternal)) != cudaSuccess) return e;
    p.lm_mode = LM_VERIFY;
    return (c->cfg.weight_dtype == HY_DTYPE_BF16) ? enqueue_step_lm_t<__nv_bfloat16, 16>(c, p)
                                                  : enqueue_step_lm_t<float, 16>(c, p);
}

int capture_fn(hy_ctx* c, cudaGraphExec_t* out, bool draft, cudaEvent_t* ev = nullptr)
{
    cudaGraph_t graph = nullptr;
    HY_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const cudaError_t e = enqueue_verify_with_context(c, draft, ev);
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph capture end: ") + cudaGetErrorString(e2));
    const cudaError_t e3 = cudaGraphInstantiate(out, graph, 0);
    cudaGraphDestroy(graph);
    if (e3 != cudaSuccess) return fail(HY_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e3));
    return HY_OK;
}

void draft_free(hy_ctx* c)
{
    for (cudaGraphExec_t& g : c->g_dflash)
    {
        if (g) cudaGraphExecDestroy(g);
        g = nullptr;
    }
    if (c->g_verify_ids_ctx) cudaGraphExecDestroy(c->g_verify_ids_ctx);
    c->g_verify_ids_ctx = nullptr;
    for (void* p : c->d_allocs) cudaFree(p);
    c->d_allocs.clear();
    c->d_wqkv.clear();
    c->d_wo.clear();
    c->d_wgu.clear();
    c->d_wd.clear();
    c->d_tkv_hi.clear();
    c->d_tkv_lo.clear();
    c->d_layers = 0;
    c->d_len = 0;
    c->device_bytes -= c->d_bytes;
    c->d_bytes = 0;
}

template <typename T>
int draft_dalloc(hy_ctx* c, T** p, size_t count)
{
    void* v = nullptr;
    const size_t bytes = align_up(std::max<size_t>(count * sizeof(T), 16), 256);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess)
        return fail(HY_ERR_OUT_OF_MEMORY, "cudaMalloc(" + std::to_string(bytes) + " bytes) failed: " + cudaGetErrorString(e));
    c->d_allocs.push_back(v);
    c->d_bytes += bytes;
    c->device_bytes += bytes;
    *p = static_cast<T*>(v);
    return HY_OK;
}

// Device memory of a draft of `layers` layers: weights (the context's weight
// dtype), norms, the tiled fc / k|v operands, the draft K/V cache, the RoPE
// table (filled here) and the step and prefill-pass buffers.
int draft_alloc(hy_ctx* c, int layers, int mask_token)
{
    const hy_config& cfg = c->cfg;
    if (layers < 1 || layers > kMaxDraftLayers)
        return fail(HY_ERR_INVALID_ARGUMENT, "draft num_layers must be in 1.." + std::to_string(kMaxDraftLayers));
    if (mask_token < 0 || mask_token >= cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "draft mask_token out of range");
    draft_free(c);
    const size_t we = c->w_elem();
    const int ffn = cfg.ffn_dim;
    int rc;
    unsigned char* w = nullptr;
    const size_t sz[4] = {align_up(static_cast<size_t>(kQKVRows) * kHidden * we, 256),
                          align_up(static_cast<size_t>(kHidden) * kQWidth * we, 256),
                          align_up(static_cast<size_t>(2 * ffn) * kHidden * we, 256),
                          align_up(static_cast<size_t>(kHidden) * ffn * we, 256)};
    const size_t fc_bytes = align_up(static_cast<size_t>(kHidden) * kAuxWidth * we, 256);
    if ((rc = draft_dalloc(c, &w, fc_bytes + (sz[0] + sz[1] + sz[2] + sz[3]) * layers))) return rc;
    c->d_fc = w;
    w += fc_bytes;
    for (int l = 0; l < layers; ++l)
    {
        c->d_wqkv.push_back(w);
        c->d_wo.push_back(w += sz[0]);
        c->d_wgu.push_back(w += sz[1]);
        c->d_wd.push_back(w += sz[2]);
        w += sz[3];
    }
    c->d_layers = layers;
    c->d_mask = mask_token;
    if ((rc = draft_dalloc(c, &c->d_norms, static_cast<size_t>(layers) * 2304 + 2 * kHidden))) return rc;
    const int planes = (cfg.weight_dtype == HY_DTYPE_BF16) ? 1 : 2;
    float* tw = nullptr;
    const size_t tfc = static_cast<size_t>(kHidden) * kAuxWidth, tkv = static_cast<size_t>(2 * kKVWidth) * kHidden;
    if ((rc = draft_dalloc(c, &tw, (tfc + tkv * layers) * planes))) return rc;
    c->d_tfc_hi = tw;
    c->d_tfc_lo = (planes == 2) ? tw + tfc : nullptr;
    for (int l = 0; l < layers; ++l)
    {
        float* p = tw + tfc * planes + tkv * planes * l;
        c->d_tkv_hi.push_back(p);
        c->d_tkv_lo.push_back(planes == 2 ? p + tkv : nullptr);
    }
    const size_t kv_count = static_cast<size_t>(layers) * kNumKVHeads * cfg.max_context * kHeadDim;
    unsigned char* kvb = nullptr;
    if ((rc = draft_dalloc(c, &kvb, kv_count * c->kv_elem()))) return rc;
    c->d_kc = kvb;
    if ((rc = draft_dalloc(c, &kvb, kv_count * c->kv_elem()))) return rc;
    c->d_vc = kvb;
    HY_CUDA(cudaMemsetAsync(c->d_kc, 0, kv_count * c->kv_elem(), c->stream));
    HY_CUDA(cudaMemsetAsync(c->d_vc, 0, kv_count * c->kv_elem(), c->stream));
    const size_t rows = static_cast<size_t>(cfg.max_context);
    if ((rc = draft_dalloc(c, &c->d_cos, rows * kHeadDim))) return rc;
    if ((rc = draft_dalloc(c, &c->d_sin, rows * kHeadDim))) return rc;
    if ((rc = draft_dalloc(c, &c->d_x, static_cast<size_t>(kBlock) * kHidden))) return rc;
    if ((rc = draft_dalloc(c, &c->d_aux, static_cast<size_t>(kBlock) * kAuxWidth))) return rc;
    if ((rc = draft_dalloc(c, &c->d_pf_aux, static_cast<size_t>(c->pf_rows) * kAuxWidth))) return rc;
    if ((rc = draft_dalloc(c, &c->d_pf_a_hi, static_cast<size_t>(c->pf_pad) * kAuxWidth))) return rc;
    if ((rc = draft_dalloc(c, &c->d_pf_a_lo, static_cast<size_t>(c->pf_pad) * kAuxWidth))) return rc;
    if ((rc = draft_dalloc(c, &c->d_pf_fc, static_cast<size_t>(c->pf_rows) * kHidden))) return rc;
    // Aux columns of layers a shallow decoder does not have stay zero (finite drafts).
    HY_CUDA(cudaMemsetAsync(c->d_aux, 0, sizeof(float) * kBlock * kAuxWidth, c->stream));
    HY_CUDA(cudaMemsetAsync(c->d_pf_aux, 0, sizeof(float) * c->pf_rows * kAuxWidth, c->stream));
    // build_dflash_rope (src/dflash_runtime.cpp:27-48) in the reference's float arithmetic.
    std::vector<float> cs(rows * kHeadDim), sn(rows * kHeadDim);
    for (size_t pos = 0; pos < rows; ++pos)
        for (int d = 0; d < kHeadDim; ++d)
        {
            const float exponent = static_cast<float>(2 * (d % (kHeadDim / 2))) / kHeadDim;
            const float angle = static_cast<float>(static_cast<int>(pos)) / std::pow(10000.0f, exponent);
            cs[pos * kHeadDim + d] = std::cos(angle);
            sn[pos * kHeadDim + d] = std::sin(angle);
        }
    HY_CUDA(cudaMemcpy(c->d_cos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice));
    HY_CUDA(cudaMemcpy(c->d_sin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
    return HY_OK;
}

// After the draft weights are in place: tiled operands and the two graphs.
template <typename WT>
int draft_finish_t(hy_ctx* c)
{
    {
        const size_t n = static_cast<size_t>(kHidden) * (kAuxWidth / 4);
        tile_weight_kernel<WT><<<static_cast<unsigned>((n + 255) / 256), 256, 0, c->stream>>>(
            static_cast<const WT*>(c->d_fc), kHidden, kAuxWidth, c->d_tfc_hi, c->d_tfc_lo);
        HY_CUDA(cudaGetLastError());
    }
    for (int l = 0; l < c->d_layers; ++l)
    {
        const size_t n = static_cast<size_t>(2 * kKVWidth) * (kHidden / 4);
        tile_weight_kernel<WT><<<static_cast<unsigned>((n + 255) / 256), 256, 0, c->stream>>>(
            static_cast<const WT*>(c->d_wqkv[l]) + static_cast<size_t>(kQWidth) * kHidden, 2 * kKVWidth, kHidden,
            c->d_tkv_hi[l], c->d_tkv_lo[l]);
        HY_CUDA(cudaGetLastError());
    }
    HY_CUDA(cudaStreamSynchronize(c->stream));
    int rc = HY_OK;
    for (int b = 0; b < kDflashGraphs && !rc; ++b)
    {
        for (cudaEvent_t& ev : c->dflash_ev[b])
            if (!ev) HY_CUDA(cudaEventCreate(&ev));
        rc = capture_fn(c, &c->g_dflash[b], true, c->dflash_ev[b]);
    }
    if (!rc) rc = capture_fn(c, &c->g_verify_ids_ctx, false);
    if (!rc) c->d_len = 0;
    return rc;
}

int draft_finish(hy_ctx* c)
{
    const int rc = (c->cfg.weight_dtype == HY_DTYPE_BF16) ? draft_finish_t<__nv_bfloat16>(c) : draft_finish_t<float>(c);
    if (rc) draft_free(c);
    return rc;
}

// Seeded synthetic draft weights on the library's counter generator (tensor
// ids from kDraftTidBase; linears ~N(0, std), norms 1 + ~N(0, norm_std)).
int draft_fill_synthetic(hy_ctx* c, unsigned long long seed, float std_dev, float norm_std)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    const bool bf = cfg.weight_dtype == HY_DTYPE_BF16;
    auto lin = [&](void* dst, size_t off_elems, unsigned long long tid, size_t count) {
        if (bf)
            launch_synth(static_cast<__nv_bfloat16*>(dst) + off_elems, count, seed, tid, std_dev, 0.f, c->stream);
        else
            launch_synth(static_cast<float*>(dst) + off_elems, count, seed, tid, std_dev, 0.f, c->stream);
    };
    auto lin_rows = [&](void* dst, unsigned long long tid, int rows, int cols, int row_mult, int row_off) {
        const unsigned long long base = synth_base(seed, tid);
        const float mult = host_synth_mult(std_dev);
        if (bf)
            synth_fill_rows_kernel<__nv_bfloat16><<<1184, 256, 0, c->stream>>>(static_cast<__nv_bfloat16*>(dst), rows,
                                                                               cols, row_mult, row_off, base, mult);
        else
            synth_fill_rows_kernel<float><<<1184, 256, 0, c->stream>>>(static_cast<float*>(dst), rows, cols, row_mult,
                                                                       row_off, base, mult);
    };
    lin(c->d_fc, 0, kTidDraftFc, static_cast<size_t>(kHidden) * kAuxWidth);
    launch_synth(c->d_hidden_norm(), kHidden, seed, kTidDraftHiddenNorm, norm_std, 1.0f, c->stream);
    launch_synth(c->d_final_norm(), kHidden, seed, kTidDraftNorm, norm_std, 1.0f, c->stream);
    for (int l = 0; l < c->d_layers; ++l)
    {
        const unsigned long long b = kDraftTidBase + kDraftTidStride * l;
        launch_synth(c->d_in_norm(l), kHidden, seed, b + J_INPUT_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->d_post_norm(l), kHidden, seed, b + J_POST_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->d_qn(l), kHeadDim, seed, b + J_Q_NORM, norm_std, 1.0f, c->stream);
        launch_synth(c->d_kn(l), kHeadDim, seed, b + J_K_NORM, norm_std, 1.0f, c->stream);
        lin(c->d_wqkv[l], 0, b + J_Q, static_cast<size_t>(kQWidth) * kHidden);
        lin(c->d_wqkv[l], static_cast<size_t>(kQWidth) * kHidden, b + J_K, static_cast<size_t>(kKVWidth) * kHidden);
        lin(c->d_wqkv[l], static_cast<size_t>(kQWidth + kKVWidth) * kHidden, b + J_V,
            static_cast<size_t>(kKVWidth) * kHidden);
        lin(c->d_wo[l], 0, b + J_O, static_cast<size_t>(kHidden) * kQWidth);
        lin_rows(c->d_wgu[l], b + J_GATE, ffn, kHidden, 2, 0);
        lin_rows(c->d_wgu[l], b + J_UP, ffn, kHidden, 2, 1);
        lin(c->d_wd[l], 0, b + J_DOWN, static_cast<size_t>(kHidden) * ffn);
    }
    HY_CUDA(cudaGetLastError());
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

// Host fp32 draft weights -> device (bf16 contexts convert on the device).
int draft_upload(hy_ctx* c, const hy_draft_weights* w)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    const bool bf = cfg.weight_dtype == HY_DTYPE_BF16;
    float* staging = nullptr;
    if (bf)
    {
        void* s = nullptr;
        HY_CUDA(cudaMalloc(&s, static_cast<size_t>(std::max(kAuxWidth, 2 * ffn)) * kHidden * sizeof(float)));
        staging = static_cast<float*>(s);
    }
    auto put = [&](void* dst, size_t off_elems, const float* src, size_t count) -> cudaError_t {
        if (!bf)
            return cudaMemcpy(static_cast<float*>(dst) + off_elems, src, count * sizeof(float), cudaMemcpyHostToDevice);
        cudaError_t e = cudaMemcpy(staging, src, count * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        f32_to_bf16_kernel<<<1184, 256, 0, c->stream>>>(staging, static_cast<__nv_bfloat16*>(dst) + off_elems, count);
        e = cudaGetLastError();
        return e != cudaSuccess ? e : cudaStreamSynchronize(c->stream);
    };
    auto put_rows = [&](void* dst, const float* src, int rows, int off) -> cudaError_t {
        if (!bf)
            return cudaMemcpy2D(static_cast<float*>(dst) + static_cast<size_t>(off) * kHidden, 2 * kHidden * sizeof(float),
                                src, kHidden * sizeof(float), kHidden * sizeof(float), rows, cudaMemcpyHostToDevice);
        cudaError_t e = cudaMemcpy(staging, src, static_cast<size_t>(rows) * kHidden * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        f32_to_bf16_rows_kernel<<<1184, 256, 0, c->stream>>>(staging, static_cast<__nv_bfloat16*>(dst), rows, kHidden, 2, off);
        e = cudaGetLastError();
        return e != cudaSuccess ? e : cudaStreamSynchronize(c->stream);
    };
    auto vec = [&](float* dst, const float* src, size_t n) {
        return cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyHostToDevice);
    };
    cudaError_t e = put(c->d_fc, 0, w->fc, static_cast<size_t>(kHidden) * kAuxWidth);
    if (e == cudaSuccess) e = vec(c->d_hidden_norm(), w->hidden_norm, kHidden);
    if (e == cudaSuccess) e = vec(c->d_final_norm(), w->norm, kHidden);
    for (int l = 0; l < c->d_layers && e == cudaSuccess; ++l)
    {
        const hy_layer_weights& lw = w->layers[l];
        e = put(c->d_wqkv[l], 0, lw.q_proj, static_cast<size_t>(kQWidth) * kHidden);
        if (e == cudaSuccess)
            e = put(c->d_wqkv[l], static_cast<size_t>(kQWidth) * kHidden, lw.k_proj, static_cast<size_t>(kKVWidth) * kHidden);
        if (e == cudaSuccess)
            e = put(c->d_wqkv[l], static_cast<size_t>(kQWidth + kKVWidth) * kHidden, lw.v_proj,
                    static_cast<size_t>(kKVWidth) * kHidden);
        if (e == cudaSuccess) e = put(c->d_wo[l], 0, lw.o_proj, static_cast<size_t>(kHidden) * kQWidth);
        if (e == cudaSuccess) e = put_rows(c->d_wgu[l], lw.gate_proj, ffn, 0);
        if (e == cudaSuccess) e = put_rows(c->d_wgu[l], lw.up_proj, ffn, 1);
        if (e == cudaSuccess) e = put(c->d_wd[l], 0, lw.down_proj, static_cast<size_t>(kHidden) * ffn);
        if (e == cudaSuccess) e = vec(c->d_in_norm(l), lw.input_norm, kHidden);
        if (e == cudaSuccess) e = vec(c->d_post_norm(l), lw.post_norm, kHidden);
        if (e == cudaSuccess) e = vec(c->d_qn(l), lw.query_norm, kHeadDim);
        if (e == cudaSuccess) e = vec(c->d_kn(l), lw.key_norm, kHeadDim);
    }
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("draft weight upload: ") + cudaGetErrorString(e));
    return HY_OK;
}

// ---------------------------------------------------------------------------
// Batched decode: the reference's JSONL batch runs its records one after the
// other through one runtime (run_jsonl_batch, src/batch_jsonl.cpp:384-480;
// decode_from_embeddings per record). Here up to 16 records decode together:
// step row m carries the next token of the sequence in slot m, so one pass of
// the 16-row projections (weights streamed once) advances every sequence by a
// token. Per layer: q/k/v (16 rows, input RMSNorm), the one-row attention
// kernel with grid z = row (RoPE / QK norm / append and split-K attention over
// the row's own cache at its own length), o_proj, gate/up + SwiGLU, down_proj;
// then the LM head with per-row history bitmaps and a per-slot commit (token
// log, history, KV length, EOS / max_tokens). Prompts are prefilled into their
// slot's cache by the ordinary prefill when a slot frees up.
// ---------------------------------------------------------------------------
// Past-key splits + the new-row split per (record, KV head) of the batched attention.
// 16 records x 256 tokens at KV 1024..1280: 3 -> 2.19 ms per step, 4 -> 2.24, 6 -> 2.31, 9 -> 2.41.
#ifndef HY_BATCH_SPLITS
#define HY_BATCH_SPLITS 3
#endif
constexpr int kBatchSplits = HY_BATCH_SPLITS;

template <typename T>
int batch_dalloc(hy_ctx* c, T** p, size_t count)
{
    void* v = nullptr;
    const size_t bytes = align_up(std::max<size_t>(count * sizeof(T), 16), 256);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess)
        return fail(HY_ERR_OUT_OF_MEMORY, "cudaMalloc(" + std::to_string(bytes) + " bytes) failed: " + cudaGetErrorString(e));
    c->b_allocs.push_back(v);
    c->device_bytes += bytes;
    *p = static_cast<T*>(v);
    return HY_OK;
}

template <typename WT, typename KT>
cudaError_t enqueue_batch_step_t(hy_ctx* c, int rows)
{
    const hy_config& cfg = c->cfg;
    const int ffn = cfg.ffn_dim;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < cfg.num_layers; ++l)
    {
        GemvArgs q = base_args(c);
        q.W = c->wqkv[l];
        q.N = kQKVRows;
        q.ldw = kHidden;
        q.rows = rows;
        q.src = (l == 0) ? SRC_GATHER_IDS : SRC_X;
        q.ids = c->b_cur;
        q.x_store = c->x;
        q.x = c->x;
        q.ldx = kHidden;
        q.norm_w = c->in_norm(l);
        q.out = c->qkv;
        q.ldo = kQKVRows;
        if ((e = run_gemv<WT, kHidden, 16, PRO_NORM, EPI_STORE>(c, q)) != cudaSuccess) return e;

        AttnArgs at;
        std::memset(&at, 0, sizeof(at));
        at.qkv = c->qkv;
        at.ldq = kQKVRows;
        at.qn_w = c->qn(l);
        at.kn_w = c->kn(l);
        at.cos = c->rope_cos;
        at.sin = c->rope_sin;
        at.rope_state = 1;
        const size_t layer_off = static_cast<size_t>(l) * kNumKVHeads * cfg.max_context * kHeadDim * c->kv_elem();
        at.kc = static_cast<char*>(c->b_kc) + layer_off;
        at.vc = static_cast<char*>(c->b_vc) + layer_off;
        at.cap = cfg.max_context;
        at.rows = 1;
        at.scale_log2 = cfg.attn_scale * 1.4426950408889634f;
        at.eps = cfg.rms_norm_eps;
        at.part = c->attn_part;
        at.counter = c->b_cnt + static_cast<size_t>(l) * kMaxStepRows * kNumKVHeads;
        at.out = c->attn;
        at.err = c->err;
        at.slots = c->b_state;
        at.slot_stride = c->slot_elems();
        {
            using S = AttnShape<1, KT>;
            auto k = attn_kernel<1, KT>;
            static unsigned long long configured = 0;
            const unsigned long long bit = 1ull << (c->cfg.device & 63);
            if (!(configured & bit))
            {
                if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM)) != cudaSuccess)
                    return e;
                configured |= bit;
            }
            if ((e = launch_pdl(k, dim3(kBatchSplits, kNumKVHeads, rows), dim3(kAttnThreads), S::SMEM, c->stream, at)) !=
                cudaSuccess)
                return e;
        }

        GemvArgs o = base_args(c);
        o.W = c->wo[l];
        o.N = kHidden;
        o.ldw = kQWidth;
        o.rows = rows;
        o.src = SRC_X;
        o.x = c->attn;
        o.ldx = kQWidth;
        o.out = c->x;
        o.ldo = kHidden;
        if ((e = run_gemv<WT, kQWidth, 16, PRO_PLAIN, EPI_RESID>(c, o)) != cudaSuccess) return e;

        GemvArgs gu = base_args(c);
        gu.W = c->wgu[l];
        gu.N = 2 * ffn;
        gu.ldw = kHidden;
        gu.rows = rows;
        gu.src = SRC_X;
        gu.x = c->x;
        gu.ldx = kHidden;
        gu.norm_w = c->post_norm(l);
        gu.out = c->act;
        gu.ldo = ffn;
        if ((e = run_gemv<WT, kHidden, 16, PRO_NORM, EPI_ACT>(c, gu)) != cudaSuccess) return e;

        GemvArgs d = base_args(c);
        d.W = c->wd[l];
        d.N = kHidden;
        d.ldw = ffn;
        d.rows = rows;
        d.src = SRC_X;
        d.x = c->act;
        d.ldx = ffn;
        GemvArgs d1 = d;
        d1.k_off = 0;
        d1.out = c->tmp;
        d1.ldo = kHidden;
        if ((e = run_gemv<WT, kFfn / 2, 16, PRO_PLAIN, EPI_STORE>(c, d1)) != cudaSuccess) return e;
        GemvArgs d2 = d;
        d2.k_off = kFfn / 2;
        d2.out = c->x;
        d2.ldo = kHidden;
        d2.extra = c->tmp;
        if ((e = run_gemv<WT, kFfn / 2, 16, PRO_PLAIN, EPI_RESID>(c, d2)) != cudaSuccess) return e;
    }
    GemvArgs lm = base_args(c);
    lm.W = c->embed;
    lm.N = cfg.vocab_size;
    lm.ldw = kHidden;
    lm.rows = rows;
    lm.src = SRC_X;
    lm.x = c->x;
    lm.ldx = kHidden;
    lm.norm_w = c->final_norm();
    lm.lm_mode = LM_BATCH;
    lm.hist = c->b_hist;
    lm.hist_stride = c->hist_words();
    lm.slots = c->b_state;
    lm.slot_cur = c->b_cur;
    lm.log_tokens = c->b_log;
    lm.log_raw = c->b_lograw;
    lm.log_stride = c->log_stride();
    return run_gemv<WT, kHidden, 16, PRO_NORM, EPI_ARGMAX>(c, lm);
}

cudaError_t enqueue_batch_step(hy_ctx* c, int rows)
{
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16, kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    if (!wb && !kb) return enqueue_batch_step_t<float, float>(c, rows);
    if (!wb && kb) return enqueue_batch_step_t<float, __nv_bfloat16>(c, rows);
    if (wb && !kb) return enqueue_batch_step_t<__nv_bfloat16, float>(c, rows);
    return enqueue_batch_step_t<__nv_bfloat16, __nv_bfloat16>(c, rows);
}

// Slot buffers (first use) and the step graph for `rows` slots.
int batch_prepare(hy_ctx* c, int rows)
{
    int rc;
    if (!c->b_kc)
    {
        const size_t kv = static_cast<size_t>(kMaxStepRows) * c->slot_elems() * c->kv_elem();
        unsigned char* p = nullptr;
        if ((rc = batch_dalloc(c, &p, kv))) return rc;
        c->b_kc = p;
        if ((rc = batch_dalloc(c, &p, kv))) return rc;
        c->b_vc = p;
        if ((rc = batch_dalloc(c, &c->b_state, kMaxStepRows))) return rc;
        if ((rc = batch_dalloc(c, &c->b_cur, kMaxStepRows))) return rc;
        if ((rc = batch_dalloc(c, &c->b_hist, static_cast<size_t>(kMaxStepRows) * c->hist_words()))) return rc;
        if ((rc = batch_dalloc(c, &c->b_log, static_cast<size_t>(kMaxStepRows) * c->log_stride()))) return rc;
        if ((rc = batch_dalloc(c, &c->b_lograw, static_cast<size_t>(kMaxStepRows) * c->log_stride()))) return rc;
        if ((rc = batch_dalloc(c, &c->b_cnt, static_cast<size_t>(c->cfg.num_layers) * kMaxStepRows * kNumKVHeads)))
            return rc;
        HY_CUDA(cudaMemsetAsync(c->b_cnt, 0, sizeof(int) * c->cfg.num_layers * kMaxStepRows * kNumKVHeads, c->stream));
        HY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&c->h_bstate), sizeof(SlotState) * kMaxStepRows));
    }
    std::memset(c->h_bstate, 0, sizeof(SlotState) * kMaxStepRows);
    HY_CUDA(cudaMemcpyAsync(c->b_state, c->h_bstate, sizeof(SlotState) * kMaxStepRows, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemsetAsync(c->b_cur, 0, sizeof(int) * kMaxStepRows, c->stream));
    if (c->g_batch && c->b_rows == rows) return HY_OK;
    if (c->g_batch) cudaGraphExecDestroy(c->g_batch);
    c->g_batch = nullptr;
    cudaGraph_t graph = nullptr;
    HY_CUDA(cudaStreamSynchronize(c->stream));
    HY_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const cudaError_t e = enqueue_batch_step(c, rows);
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &graph);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("batch graph capture: ") + cudaGetErrorString(e));
    if (e2 != cudaSuccess) return fail(HY_ERR_CUDA, std::string("batch graph capture end: ") + cudaGetErrorString(e2));
    const cudaError_t e3 = cudaGraphInstantiate(&c->g_batch, graph, 0);
    cudaGraphDestroy(graph);
    if (e3 != cudaSuccess) return fail(HY_ERR_CUDA, std::string("batch graph instantiate: ") + cudaGetErrorString(e3));
    c->b_rows = rows;
    return HY_OK;
}

// ---------------------------------------------------------------------------
// LM-head select with device-global scratch, allocating nothing.
//
// For callers that cannot allocate device memory while they decode: a host
// runtime that reserves the device's memory up front for its own caching
// allocator (a cudaMalloc then fails or fragments that pool), or one that must
// not take the implicit device-wide synchronisation of cudaMalloc/cudaFree in
// the middle of a decode loop that shares the GPU with other streams. Inputs
// and outputs are device pointers; the argmax kernel's per-CTA partials and
// its completion ticket live in the file-scope array below instead of in
// context-owned buffers. The array is one per device and process, so calls
// that overlap in time on the same device (any context, stream or thread)
// race on it.
// ---------------------------------------------------------------------------
constexpr int kSelectScratchCtas = 256;      // partial slots per row (one launch: one CTA per SM)
constexpr size_t kSelectTicketBytes = 256;   // the completion ticket (one int), padded
constexpr size_t kSelectScratchBytes = kSelectTicketBytes + sizeof(float4) * kSelectScratchCtas * kMaxStepRows;  // 65,792 B
static __device__ __align__(256) unsigned char g_select_scratch[kSelectScratchBytes];

// Device address of g_select_scratch, resolved once per device with that device current.
int select_scratch_address(int device, unsigned char** out)
{
    static std::mutex m;
    static unsigned char* addr[64] = {};
    if (device < 0 || device >= 64) return fail(HY_ERR_INVALID_ARGUMENT, "device index out of range");
    std::lock_guard<std::mutex> lock(m);
    if (!addr[device])
    {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_select_scratch);
        if (e != cudaSuccess)
            return fail(HY_ERR_CUDA, std::string("cudaGetSymbolAddress(select scratch): ") + cudaGetErrorString(e));
        addr[device] = static_cast<unsigned char*>(p);
    }
    *out = addr[device];
    return HY_OK;
}

template <typename WT, int MT>
cudaError_t enqueue_lm_select_scratch_t(hy_ctx* c, int rows, const float* x, float penalty, unsigned char* scratch,
                                        int* tokens, int* raw_top1)
{
    GemvArgs lm = base_args(c);
    lm.part = reinterpret_cast<float4*>(scratch + kSelectTicketBytes);
    lm.counter = reinterpret_cast<int*>(scratch);
    lm.W = c->embed;
    lm.N = c->cfg.vocab_size;
    lm.ldw = kHidden;
    lm.rows = rows;
    lm.src = SRC_X;
    lm.x = x;
    lm.ldx = kHidden;
    lm.lm_mode = LM_NONE;
    lm.penalty = penalty;
    lm.prefix = nullptr;
    lm.logits = nullptr;
    lm.tok_out = tokens;
    lm.raw_out = raw_top1;
    return run_gemv<WT, kHidden, MT, PRO_PLAIN, EPI_ARGMAX>(c, lm);
}

// Pass the tokens committed since the last call, log entries [cb_emitted, n), to the callback.
int emit_tokens(hy_ctx* c, int n)
{
    if (!c->cb || n <= c->cb_emitted) return HY_OK;
    std::vector<int> t(static_cast<size_t>(n - c->cb_emitted));
    HY_CUDA(cudaMemcpy(t.data(), c->log_tokens + c->cb_emitted, sizeof(int) * t.size(), cudaMemcpyDeviceToHost));
    c->cb_emitted = n;
    for (int tok : t) c->cb(tok, c->cb_user);
    return HY_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* hy_version(void) { return "hy_decode 0.1 (sm_100a)"; }

const char* hy_last_error(void) { return g_error.c_str(); }

}  // extern "C"

// The message of a failure in the library's host code outside this file (the
// model-package reader), for hy_last_error.
namespace hy_internal {
void set_last_error(const std::string& msg) { g_error = msg; }
}  // namespace hy_internal

extern "C" {

int hy_config_init(hy_config* cfg)
{
    if (!cfg) return fail(HY_ERR_INVALID_ARGUMENT, "config is null");
    cfg->num_layers = 24;
    cfg->vocab_size = 120818;
    cfg->ffn_dim = kFfn;
    cfg->max_context = 8192 + 64;
    cfg->max_prefill = 2048;
    cfg->max_tokens = 2048;
    cfg->weight_dtype = HY_DTYPE_F32;
    cfg->kv_dtype = HY_DTYPE_F32;
    cfg->rms_norm_eps = 1e-5f;
    cfg->attn_scale = 0.0883883f;
    cfg->device = 0;
    return HY_OK;
}

int hy_ctx_create(const hy_config* cfg, const hy_weights* weights, hy_ctx** out)
{
    if (!out) return fail(HY_ERR_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    int rc = validate_config(cfg);
    if (rc) return rc;
    hy_ctx* c = new hy_ctx();
    c->cfg = *cfg;
    if ((rc = alloc_ctx(c)) || (rc = upload_weights(c, weights)))
    {
        free_ctx(c);
        return rc;
    }
    return finish_create(c, out);
}

int hy_ctx_create_synthetic(const hy_config* cfg, uint64_t seed, float std_dev, float norm_std, hy_ctx** out)
{
    if (!out) return fail(HY_ERR_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    int rc = validate_config(cfg);
    if (rc) return rc;
    hy_ctx* c = new hy_ctx();
    c->cfg = *cfg;
    if ((rc = alloc_ctx(c)) || (rc = fill_synthetic(c, seed, std_dev, norm_std)))
    {
        free_ctx(c);
        return rc;
    }
    return finish_create(c, out);
}

void hy_ctx_destroy(hy_ctx* ctx) { free_ctx(ctx); }

int hy_ctx_config(const hy_ctx* ctx, hy_config* cfg)
{
    if (!ctx || !cfg) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    *cfg = ctx->cfg;
    return HY_OK;
}

size_t hy_ctx_device_bytes(const hy_ctx* ctx) { return ctx ? ctx->device_bytes : 0; }

void* hy_ctx_stream(hy_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int hy_build_mrope(const int* position_ids, int seq_len, int use_cos, float* out)
{
    // detail::build_mrope (src/text_runtime.cpp:42-63).
    if (!position_ids || !out || seq_len <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "invalid mrope arguments");
    constexpr int section = kHeadDim / 4;
    const float base = static_cast<float>(10000.0 * std::pow(1000.0, 128.0 / 126.0));
    for (int dim = 0; dim < kHeadDim; ++dim)
    {
        const int axis = dim / section;
        const int fd = dim % (kHeadDim / 2);
        const float inv_freq = 1.0f / std::pow(base, static_cast<float>(2 * fd) / kHeadDim);
        for (int t = 0; t < seq_len; ++t)
        {
            const int position = position_ids[static_cast<size_t>(axis) * seq_len + t];
            const float angle = static_cast<float>(position) * inv_freq;
            out[static_cast<size_t>(t) * kHeadDim + dim] = use_cos ? std::cos(angle) : std::sin(angle);
        }
    }
    return HY_OK;
}

float hy_rope_value(int position, int dim, int use_cos) { return rope_value_host(position, dim, use_cos != 0); }

int hy_ctx_set_token_callback(hy_ctx* c, hy_token_callback cb, void* user, int tokens_per_sync)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    if (tokens_per_sync < 0 || tokens_per_sync > kMegaChunk)
        return fail(HY_ERR_INVALID_ARGUMENT, "tokens_per_sync must be in 0.." + std::to_string(kMegaChunk));
    c->cb = cb;
    c->cb_user = user;
    c->cb_sync = tokens_per_sync ? tokens_per_sync : kMegaChunk;
    return HY_OK;
}

int hy_ctx_set_ar_path(hy_ctx* c, int path)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    if (path != HY_AR_PATH_PERSISTENT && path != HY_AR_PATH_GRAPH) return fail(HY_ERR_INVALID_ARGUMENT, "unknown AR path");
    if (path == HY_AR_PATH_PERSISTENT && !c->mega_ok)
        return fail(HY_ERR_UNSUPPORTED, "the persistent decode kernel needs a cooperative launch of >= 144 co-resident CTAs");
    c->ar_path = path;
    return HY_OK;
}

int hy_ctx_ar_path(const hy_ctx* c) { return c ? c->ar_path : -1; }

int hy_debug_progress(const hy_ctx* c, unsigned* out, int n)
{
    if (!c || !out || n <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "invalid arguments");
    if (!c->progress) return fail(HY_ERR_NOT_READY, "start the process with HY_DEBUG_PROGRESS=1");
    for (int i = 0; i < n && i < 1024; ++i) out[i] = c->progress[i];
    return HY_OK;
}

int hy_ctx_set_wait_limit(hy_ctx* c, unsigned long long limit_ns)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (limit_ns < 1000000ull || limit_ns > 60000000000ull)
        return fail(HY_ERR_INVALID_ARGUMENT, "wait limit must be in 1 ms .. 60 s");
    c->wait_limit_ns = limit_ns;
    return HY_OK;
}

int hy_debug_wait_probe(hy_ctx* c, int kind, unsigned long long limit_ns)
{
    if (!c || (kind != 0 && kind != 1)) return fail(HY_ERR_INVALID_ARGUMENT, "kind must be 0 (epoch word) or 1 (mbarrier)");
    if (limit_ns < 1000ull || limit_ns > 10000000000ull)
        return fail(HY_ERR_INVALID_ARGUMENT, "probe limit must be in 1 us .. 10 s");
    int rc = set_device(c);
    if (rc) return rc;
    wait_probe_kernel<<<1, 32, 0, c->stream>>>(c->probe_word, kind, limit_ns, c->err);
    HY_CUDA(cudaGetLastError());
    return check_device_error(c);
}

int hy_debug_wait_stats(hy_ctx* c, unsigned long long* out, int n_words, int reset)
{
    if (!c || n_words < 0 || (n_words > 0 && !out)) return fail(HY_ERR_INVALID_ARGUMENT, "invalid arguments");
    if (!c->wstat) return fail(HY_ERR_UNSUPPORTED, "wait statistics need a library built with HY_WAIT_STATS");
    int rc = set_device(c);
    if (rc) return rc;
    if (n_words > 0)
    {
        HY_CUDA(cudaMemcpyAsync(out, c->wstat, sizeof(unsigned long long) * std::min(n_words, kWsWords),
                                cudaMemcpyDeviceToHost, c->stream));
    }
    if (reset)
    {
        HY_CUDA(cudaMemsetAsync(c->wstat, 0, kWsWords * sizeof(unsigned long long), c->stream));
        c->mega_launches = 0;
    }
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

int hy_debug_step_trace(hy_ctx* c, unsigned long long* out, int max_records, int* n_records, int reset)
{
    if (!c || max_records < 0 || (max_records > 0 && !out) || !n_records)
        return fail(HY_ERR_INVALID_ARGUMENT, "invalid arguments");
#ifdef HY_STEP_TRACE
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaStreamSynchronize(c->stream));
    unsigned n = 0;
    HY_CUDA(cudaMemcpyFromSymbol(&n, g_step_trace_n, sizeof(n)));
    n = std::min<unsigned>(n, static_cast<unsigned>(kStepTraceMax));
    const int k = std::min<int>(static_cast<int>(n), max_records);
    if (k > 0)
        HY_CUDA(cudaMemcpyFromSymbol(out, g_step_trace, sizeof(unsigned long long) * kStepTraceWords * k));
    *n_records = static_cast<int>(n);
    if (reset)
    {
        const unsigned zero = 0;
        HY_CUDA(cudaMemcpyToSymbol(g_step_trace_n, &zero, sizeof(zero)));
    }
    return HY_OK;
#else
    (void)reset;
    *n_records = 0;
    return fail(HY_ERR_UNSUPPORTED, "the step trace needs a library built with HY_STEP_TRACE");
#endif
}

int hy_trace_persistent(hy_ctx* c, int tokens, int trace_token, unsigned long long* out)
{
    if (!c || !out || tokens < 1 || trace_token < 0 || trace_token >= tokens || tokens > kMegaChunk)
        return fail(HY_ERR_INVALID_ARGUMENT, "invalid trace arguments");
    if (!c->mega_ok) return fail(HY_ERR_UNSUPPORTED, "the persistent decode kernel is not available");
    if (c->kv_len + tokens > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    int rc = set_device(c);
    if (rc) return rc;
    const int phases = 5 * c->cfg.num_layers + 1;
    const size_t n = static_cast<size_t>(kTraceCtas) * phases * kTraceSlots;
    unsigned long long* d = nullptr;
    HY_CUDA(cudaMalloc(reinterpret_cast<void**>(&d), n * sizeof(unsigned long long)));
    HY_CUDA(cudaMemsetAsync(d, 0, n * sizeof(unsigned long long), c->stream));
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.n_gen = 1;
    h.max_tokens = tokens + 1;
    h.done = 0;
    h.n_eos = 0;
    if ((rc = push_state(c)))
    {
        cudaFree(d);
        return rc;
    }
    t_trace = d;
    t_trace_token = trace_token;
    cudaError_t e = launch_mega(c, tokens);
    t_trace = nullptr;
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("trace launch: ") + cudaGetErrorString(e));
    if ((rc = check_device_error(c))) return rc;
    return set_length(c, c->kv_len);
}

int hy_seq_reset(hy_ctx* c)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemsetAsync(c->hist, 0, sizeof(unsigned) * ((c->cfg.vocab_size + 31) / 32), c->stream));
    c->d_len = 0;
    return set_length(c, 0);
}

int hy_seq_length(hy_ctx* c, int* rows)
{
    if (!c || !rows) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    *rows = c->kv_len;
    return HY_OK;
}

int hy_seq_truncate(hy_ctx* c, int rows)
{
    // view_dflash_rows (src/dflash_runtime.cpp:97-119) rejects rows <= 0 or > h.
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    if (rows <= 0 || rows > c->kv_len) return fail(HY_ERR_INVALID_ARGUMENT, "invalid DFlash row view");
    int rc = set_device(c);
    if (rc) return rc;
    c->d_len = std::min(c->d_len, rows);
    return set_length(c, rows);
}

int hy_seq_set_length(hy_ctx* c, int rows)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    if (rows < 0 || rows > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "length exceeds the KV capacity");
    int rc = set_device(c);
    if (rc) return rc;
    c->d_len = std::min(c->d_len, rows);
    return set_length(c, rows);
}

static int history_upload(hy_ctx* c, const int* ids, int n, bool clear)
{
    if (!c || n < 0 || (n > 0 && !ids)) return fail(HY_ERR_INVALID_ARGUMENT, "invalid history arguments");
    int rc = set_device(c);
    if (rc) return rc;
    if (clear) HY_CUDA(cudaMemsetAsync(c->hist, 0, sizeof(unsigned) * ((c->cfg.vocab_size + 31) / 32), c->stream));
    // Through the context's pinned and device id buffers, kHistChunk ids per round
    // (no allocation; each round's copy has finished before the next refills them).
    for (int done = 0; done < n; done += kHistChunk)
    {
        const int m = std::min(kHistChunk, n - done);
        if (done > 0) HY_CUDA(cudaStreamSynchronize(c->stream));
        std::memcpy(c->h_hist, ids + done, sizeof(int) * m);
        HY_CUDA(cudaMemcpyAsync(c->hist_ids, c->h_hist, sizeof(int) * m, cudaMemcpyHostToDevice, c->stream));
        hist_add_kernel<<<(m + 255) / 256, 256, 0, c->stream>>>(c->hist, c->hist_ids, m, c->cfg.vocab_size);
        HY_CUDA(cudaGetLastError());
    }
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

int hy_history_set(hy_ctx* c, const int* ids, int n) { return history_upload(c, ids, n, true); }
int hy_history_add(hy_ctx* c, const int* ids, int n) { return history_upload(c, ids, n, false); }

int hy_prefill(hy_ctx* c, const float* embeds, const float* cos, const float* sin, int seq, float* last_hidden,
               float* aux_hidden)
{
    if (!c || !embeds || !cos || !sin) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (seq <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "seq_len must be positive");
    if (seq > c->cfg.max_prefill || seq > c->cfg.max_context)
        return fail(HY_ERR_CAPACITY, "prompt of " + std::to_string(seq) + " rows exceeds max_prefill");
    if (aux_hidden) return fail(HY_ERR_UNSUPPORTED, "prefill aux hidden states are produced per step only");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemcpyAsync(c->prompt, embeds, sizeof(float) * seq * kHidden, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_cos, cos, sizeof(float) * seq * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_sin, sin, sizeof(float) * seq * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    if ((rc = run_prefill(c, seq))) return rc;
    if (last_hidden)
        HY_CUDA(cudaMemcpyAsync(last_hidden, c->hidden, sizeof(float) * kHidden, cudaMemcpyDeviceToHost, c->stream));
    if ((rc = check_device_error(c))) return rc;
    if (draft_ready(c)) c->d_len = seq;
    return set_length(c, seq);
}

int hy_decoder_step(hy_ctx* c, const float* embeds, int rows, const float* cos, const float* sin, float* hidden,
                    float* aux_hidden)
{
    if (!c || !embeds || !cos || !sin) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (rows < 1 || rows > kMaxStepRows) return fail(HY_ERR_INVALID_ARGUMENT, "rows must be in 1..16");
    if (c->kv_len + rows > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemcpyAsync(c->x, embeds, sizeof(float) * rows * kHidden, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_cos, cos, sizeof(float) * rows * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_sin, sin, sizeof(float) * rows * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    // With a DFlash draft whose context covers the sequence, the rows' aux states
    // also become draft context rows.
    const bool ctx_rows = draft_ready(c) && c->d_len == c->kv_len;
    float* aux[kAuxLayers];
    for (int i = 0; i < kAuxLayers; ++i)
        aux[i] = ctx_rows ? c->d_aux + i * kHidden : c->aux + static_cast<size_t>(i) * kMaxStepRows * kHidden;
    if ((rc = run_direct_step(c, rows, c->kv_len, c->pre_cos, c->pre_sin, (aux_hidden || ctx_rows) ? aux : nullptr,
                              ctx_rows ? kAuxWidth : kHidden)))
        return rc;
    if (ctx_rows)
    {
        const cudaError_t e = enqueue_draft_context16(c, c->d_aux, rows, false, c->kv_len);
        if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("draft context launch: ") + cudaGetErrorString(e));
    }
    if (hidden)
    {
        rmsnorm_rows_kernel<<<rows, 256, 0, c->stream>>>(c->x, c->final_norm(), c->cfg.rms_norm_eps, c->hidden, kHidden);
        HY_CUDA(cudaGetLastError());
        HY_CUDA(cudaMemcpyAsync(hidden, c->hidden, sizeof(float) * rows * kHidden, cudaMemcpyDeviceToHost, c->stream));
    }
    if (aux_hidden)
        for (int i = 0; i < kAuxLayers; ++i)
            HY_CUDA(cudaMemcpy2DAsync(aux_hidden + static_cast<size_t>(i) * rows * kHidden, sizeof(float) * kHidden, aux[i],
                                      sizeof(float) * (ctx_rows ? kAuxWidth : kHidden), sizeof(float) * kHidden, rows,
                                      cudaMemcpyDeviceToHost, c->stream));
    if ((rc = check_device_error(c))) return rc;
    if (ctx_rows) c->d_len = c->kv_len + rows;
    return set_length(c, c->kv_len + rows);
}

int hy_lm_head_select(hy_ctx* c, const float* hidden, int rows, const int* row_prefix, float penalty, int* tokens,
                      int* raw_top1, float* logits)
{
    if (!c || !hidden || !tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (rows < 1 || rows > kMaxStepRows) return fail(HY_ERR_INVALID_ARGUMENT, "rows must be in 1..16");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemcpyAsync(c->hidden, hidden, sizeof(float) * rows * kHidden, cudaMemcpyHostToDevice, c->stream));
    if (row_prefix) HY_CUDA(cudaMemcpyAsync(c->prefix, row_prefix, sizeof(int) * rows, cudaMemcpyHostToDevice, c->stream));
    if (logits && !c->logits)
        HY_CUDA(cudaMalloc(reinterpret_cast<void**>(&c->logits), sizeof(float) * kMaxStepRows * c->cfg.vocab_size));
    t_next_plain = true;
    cudaError_t e = enqueue_lm_select(c, rows, c->hidden, penalty, row_prefix != nullptr, logits ? c->logits : nullptr);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("LM head launch: ") + cudaGetErrorString(e));
    HY_CUDA(cudaMemcpyAsync(tokens, c->tok_out, sizeof(int) * rows, cudaMemcpyDeviceToHost, c->stream));
    if (raw_top1) HY_CUDA(cudaMemcpyAsync(raw_top1, c->raw_out, sizeof(int) * rows, cudaMemcpyDeviceToHost, c->stream));
    if (logits)
        HY_CUDA(cudaMemcpyAsync(logits, c->logits, sizeof(float) * rows * c->cfg.vocab_size, cudaMemcpyDeviceToHost,
                                c->stream));
    return check_device_error(c);
}

int hy_lm_head_select_noalloc(hy_ctx* c, const float* hidden_dev, int rows, float penalty, int* tokens_dev,
                              int* raw_top1_dev)
{
    if (!c || !hidden_dev || !tokens_dev || !raw_top1_dev) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (rows < 1 || rows > kMaxStepRows)
        return fail(HY_ERR_CAPACITY, "rows must be in 1..16 (the static select scratch holds partials for 16 rows)");
    if (c->num_sms > kSelectScratchCtas)
        return fail(HY_ERR_CAPACITY, "the static select scratch holds partials for at most " +
                                         std::to_string(kSelectScratchCtas) + " CTAs; this device launches " +
                                         std::to_string(c->num_sms));
    if (reinterpret_cast<uintptr_t>(hidden_dev) % 16 != 0)
        return fail(HY_ERR_INVALID_ARGUMENT, "hidden_dev must be 16-byte aligned");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    int rc = set_device(c);
    if (rc) return rc;
    unsigned char* scratch = nullptr;
    if ((rc = select_scratch_address(c->cfg.device, &scratch))) return rc;
    // The ticket must be zero when the launch starts (its last CTA re-zeroes
    // it; clearing it here also recovers from an aborted launch). The partials
    // need no clearing: every CTA writes its own slots before taking a ticket.
    HY_CUDA(cudaMemsetAsync(scratch, 0, sizeof(int), c->stream));
    t_next_plain = true;
    cudaError_t e;
    if (c->cfg.weight_dtype == HY_DTYPE_BF16)
        e = rows == 1 ? enqueue_lm_select_scratch_t<__nv_bfloat16, 1>(c, rows, hidden_dev, penalty, scratch, tokens_dev, raw_top1_dev)
                      : enqueue_lm_select_scratch_t<__nv_bfloat16, 16>(c, rows, hidden_dev, penalty, scratch, tokens_dev, raw_top1_dev);
    else
        e = rows == 1 ? enqueue_lm_select_scratch_t<float, 1>(c, rows, hidden_dev, penalty, scratch, tokens_dev, raw_top1_dev)
                      : enqueue_lm_select_scratch_t<float, 16>(c, rows, hidden_dev, penalty, scratch, tokens_dev, raw_top1_dev);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("LM head launch: ") + cudaGetErrorString(e));
    return check_device_error(c);
}

// Copy n ints of two device logs to the caller's (nullable) buffers through the
// pinned h_log area (one synchronisation).
static int read_logs(hy_ctx* c, const int* dev_a, int* out_a, const int* dev_b, int* out_b, int n_a, int n_b)
{
    const int cap = c->cfg.max_tokens + 2 * kBlock;
    if (n_a > cap || n_b > cap) return fail(HY_ERR_CAPACITY, "log longer than the context's token capacity");
    if (out_a && n_a > 0) HY_CUDA(cudaMemcpyAsync(c->h_log, dev_a, sizeof(int) * n_a, cudaMemcpyDeviceToHost, c->stream));
    if (out_b && n_b > 0)
        HY_CUDA(cudaMemcpyAsync(c->h_log + cap, dev_b, sizeof(int) * n_b, cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    if (out_a && n_a > 0) std::memcpy(out_a, c->h_log, sizeof(int) * n_a);
    if (out_b && n_b > 0) std::memcpy(out_b, c->h_log + cap, sizeof(int) * n_b);
    return HY_OK;
}

// The AR loop behind hy_generate and hy_run_vlm_decode_with_prompt; fills the
// decode stage of the context's timing (events around the launches).
static int generate_impl(hy_ctx* c, int first_token, int first_raw_top1, int max_tokens, float penalty,
                         const int* eos_ids, int n_eos, int* tokens, int* raw_top1, int* n_tokens)
{
    if (!n_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (max_tokens < 1 || max_tokens > c->cfg.max_tokens)
        return fail(HY_ERR_CAPACITY, "max_tokens must be in 1..config max_tokens");
    if (first_token < 0 || first_token >= c->cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "first_token out of range");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    if (c->kv_len + max_tokens > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = set_eos(c, eos_ids, n_eos))) return rc;
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.cur_token = first_token;
    h.n_gen = 1;
    h.max_tokens = max_tokens;
    h.penalty = penalty;
    bool first_eos = false;
    for (int i = 0; i < n_eos; ++i) first_eos |= (eos_ids[i] == first_token);
    h.done = (first_eos || max_tokens <= 1) ? 1 : 0;
    if ((rc = push_state(c))) return rc;
    c->h_small[2] = first_token;
    c->h_small[3] = first_raw_top1;
    HY_CUDA(cudaMemcpyAsync(c->log_tokens, c->h_small + 2, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->log_raw, c->h_small + 3, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    if ((rc = history_upload(c, &first_token, 1, false))) return rc;
    c->cb_emitted = 0;
    if ((rc = emit_tokens(c, 1))) return rc;
    const int chunk = c->cb ? c->cb_sync : kMegaChunk;
    int launched_steps = 0;
    HY_CUDA(cudaEventRecord(c->tev[4], c->stream));
    while (!h.done && launched_steps < max_tokens - 1)
    {
        if (c->ar_path == HY_AR_PATH_PERSISTENT)
        {
            const int n = std::min(chunk, max_tokens - 1 - launched_steps);
            cudaError_t e = launch_mega(c, n);
            if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("persistent decode launch: ") + cudaGetErrorString(e));
            launched_steps += n;
        }
        else
        {
            for (int i = 0; i < 4 && launched_steps < max_tokens - 1; ++i)
            {
                HY_CUDA(cudaGraphLaunch(c->g_ar, c->stream));
                launched_steps += kArStepsPerGraph;
            }
        }
        HY_CUDA(cudaEventRecord(c->tev[5], c->stream));
        if ((rc = sync_state_to_host(c))) return rc;
        if (h.kv_len + 0 > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
        if (c->cb && (rc = check_device_error(c)) == HY_OK) rc = emit_tokens(c, h.n_gen);
        if (rc) return rc;
    }
    if (launched_steps == 0) HY_CUDA(cudaEventRecord(c->tev[5], c->stream));
    if ((rc = check_device_error(c))) return rc;
    if ((rc = sync_state_to_host(c))) return rc;
    if ((rc = emit_tokens(c, h.n_gen))) return rc;
    float td = 0.f;
    HY_CUDA(cudaEventElapsedTime(&td, c->tev[4], c->tev[5]));
    c->timing.decode_ms = td;
    *n_tokens = h.n_gen;
    return read_logs(c, c->log_tokens, tokens, c->log_raw, raw_top1, h.n_gen, h.n_gen);
}

using TimingClock = std::chrono::steady_clock;

// Close the timing of an AR call: wall clock and the part not covered by device stages.
static int finish_timing(hy_ctx* c, TimingClock::time_point t0, int rc)
{
    hy_decode_timing& t = c->timing;
    t.total_ms = std::chrono::duration<double, std::milli>(TimingClock::now() - t0).count();
    t.host_overhead_ms = t.total_ms - (t.text_embed_ms + t.prefill_ms + t.lm_head_ms + t.decode_ms);
    return rc;
}

// Token and acceptance logs of a DFlash loop to the caller, and the counts of
// DFlashDecodeResult / DecoderStatistics into the context's DFlash timing.
static int dflash_results(hy_ctx* c, int* tokens, int* acceptance_lengths)
{
    const DecodeState& h = *c->h_st;
    const int cap = c->cfg.max_tokens + 2 * kBlock;
    if (h.n_gen > cap || h.block_count > cap) return fail(HY_ERR_CAPACITY, "log longer than the context's token capacity");
    int* acc = c->h_log + cap;
    if (tokens && h.n_gen > 0)
        HY_CUDA(cudaMemcpyAsync(c->h_log, c->log_tokens, sizeof(int) * h.n_gen, cudaMemcpyDeviceToHost, c->stream));
    if (h.block_count > 0)
        HY_CUDA(cudaMemcpyAsync(acc, c->accept_log, sizeof(int) * h.block_count, cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    if (tokens && h.n_gen > 0) std::memcpy(tokens, c->h_log, sizeof(int) * h.n_gen);
    long long accepted = 0;
    for (int b = 0; b < h.block_count; ++b) accepted += acc[b];
    if (acceptance_lengths) std::memcpy(acceptance_lengths, acc, sizeof(int) * h.block_count);
    c->dtiming.block_count = h.block_count;
    c->dtiming.drafted_token_count = h.block_count * (kBlock - 1);
    c->dtiming.accepted_draft_token_count = static_cast<int>(accepted);
    return HY_OK;
}

static int finish_dflash_timing(hy_ctx* c, TimingClock::time_point t0, int rc)
{
    hy_dflash_timing& t = c->dtiming;
    t.total_ms = std::chrono::duration<double, std::milli>(TimingClock::now() - t0).count();
    t.host_overhead_ms = t.total_ms - (t.prefill_ms + t.blocks_ms);
    return rc;
}

int hy_generate(hy_ctx* c, int first_token, int first_raw_top1, int max_tokens, float penalty, const int* eos_ids,
                int n_eos, int* tokens, int* raw_top1, int* n_tokens)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    const auto t0 = TimingClock::now();
    c->timing = hy_decode_timing{};
    return finish_timing(c, t0,
                         generate_impl(c, first_token, first_raw_top1, max_tokens, penalty, eos_ids, n_eos, tokens,
                                       raw_top1, n_tokens));
}

int hy_ctx_last_timing(const hy_ctx* c, hy_decode_timing* out)
{
    if (!c || !out) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    *out = c->timing;
    return HY_OK;
}

int hy_ctx_last_dflash_timing(const hy_ctx* c, hy_dflash_timing* out)
{
    if (!c || !out) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    *out = c->dtiming;
    return HY_OK;
}

int hy_verify_block(hy_ctx* c, const int* proposed, int max_commit, float penalty, const int* eos_ids, int n_eos,
                    int* posterior, int* acceptance_length, int* committed, int* stop)
{
    if (!c || !proposed) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (max_commit < 1 || max_commit > c->cfg.max_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "max_commit out of range");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    if (c->kv_len + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    for (int i = 0; i < kBlock; ++i)
        if (proposed[i] < 0 || proposed[i] >= c->cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "proposed id out of range");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = set_eos(c, eos_ids, n_eos))) return rc;
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.cur_token = proposed[0];
    h.n_gen = 0;
    h.max_tokens = max_commit;
    h.done = 0;
    h.penalty = penalty;
    h.block_count = 0;
    if ((rc = push_state(c))) return rc;
    HY_CUDA(cudaMemcpyAsync(c->proposed, proposed, sizeof(int) * kBlock, cudaMemcpyHostToDevice, c->stream));
    // With a DFlash draft whose context covers the sequence, the committed rows
    // also become draft context rows (append_dflash_rows, src/dflash_runtime.cpp:121-166).
    const bool ctx_rows = draft_ready(c) && c->d_len == c->kv_len;
    HY_CUDA(cudaGraphLaunch(ctx_rows ? c->g_verify_ids_ctx : c->g_verify_ids, c->stream));
    if ((rc = check_device_error(c))) return rc;
    if ((rc = sync_state_to_host(c))) return rc;
    if (ctx_rows) c->d_len = c->kv_len;
    if (posterior) HY_CUDA(cudaMemcpy(posterior, c->posterior, sizeof(int) * kBlock, cudaMemcpyDeviceToHost));
    if (acceptance_length) *acceptance_length = h.accept;
    if (committed) *committed = h.committed;
    if (stop) *stop = h.stop;
    return HY_OK;
}

int hy_dflash_generate_synthetic(hy_ctx* c, int first_token, int max_tokens, float penalty, const int* eos_ids,
                                 int n_eos, const int* greedy, int n_greedy, float p, uint64_t seed, int* tokens,
                                 int* n_tokens, int* acceptance_lengths, int* n_blocks)
{
    if (!c || !n_tokens || (n_greedy > 0 && !greedy)) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (max_tokens < 1 || max_tokens > c->cfg.max_tokens)
        return fail(HY_ERR_CAPACITY, "max_tokens must be in 1..config max_tokens");
    if (n_greedy < 0 || n_greedy > c->cfg.max_tokens + 2 * kBlock) return fail(HY_ERR_CAPACITY, "greedy sequence too long");
    if (first_token < 0 || first_token >= c->cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "first_token out of range");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    if (c->kv_len + max_tokens + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = set_eos(c, eos_ids, n_eos))) return rc;
    if (n_greedy > 0)
        HY_CUDA(cudaMemcpyAsync(c->greedy, greedy, sizeof(int) * n_greedy, cudaMemcpyHostToDevice, c->stream));
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.cur_token = first_token;
    h.n_gen = 0;
    h.max_tokens = max_tokens;
    h.done = 0;
    h.penalty = penalty;
    h.block_count = 0;
    h.n_greedy = n_greedy;
    h.draft_p = p;
    h.draft_base = synth_base(seed, kTidDrafts);
    if ((rc = push_state(c))) return rc;
    int launched = 0;
    c->cb_emitted = 0;
    const auto t0 = TimingClock::now();
    c->dtiming = hy_dflash_timing{};
    while (!h.done && launched < max_tokens)
    {
        HY_CUDA(cudaEventRecord(c->tev[4], c->stream));
        for (int i = 0; i < kDflashGraphs && launched < max_tokens; ++i, ++launched)
            HY_CUDA(cudaGraphLaunch(c->g_verify_draft, c->stream));
        HY_CUDA(cudaEventRecord(c->tev[5], c->stream));
        if ((rc = sync_state_to_host(c))) return rc;
        float ms = 0.f;
        HY_CUDA(cudaEventElapsedTime(&ms, c->tev[4], c->tev[5]));
        c->dtiming.blocks_ms += ms;
        if (c->cb && (rc = check_device_error(c)) == HY_OK) rc = emit_tokens(c, h.n_gen);
        if (rc) return rc;
    }
    if ((rc = check_device_error(c))) return rc;
    if ((rc = sync_state_to_host(c))) return rc;
    if ((rc = emit_tokens(c, h.n_gen))) return rc;
    *n_tokens = h.n_gen;
    if (n_blocks) *n_blocks = h.block_count;
    rc = dflash_results(c, tokens, acceptance_lengths);
    return finish_dflash_timing(c, t0, rc);
}

// The prompt half of run_vlm_decode_with_prompt (src/text_runtime.cpp:2053-2094,
// 1307-1416): prompt embedding with vision-feature injection, mRoPE tables,
// prefill (and the draft context when a draft is loaded), history = prompt ids,
// and the first token from the last row's logits.
static int prompt_prefill_first(hy_ctx* c, const int* input_ids, const int* position_ids, int seq_len,
                                int image_token_id, const float* vision_features, int vision_token_count,
                                float repetition_penalty, int* first, int* first_raw)
{
    // prepare_prompt_embeddings checks (src/text_runtime.cpp:506-568).
    if (!c || !input_ids || !position_ids) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (seq_len <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "prompt input_ids must not be empty");
    if (vision_token_count <= 0 || !vision_features) return fail(HY_ERR_INVALID_ARGUMENT, "vision feature size mismatch");
    if (!std::isfinite(repetition_penalty) || repetition_penalty <= 0.f)
        return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    if (seq_len > c->cfg.max_prefill) return fail(HY_ERR_CAPACITY, "prompt exceeds max_prefill");
    std::vector<int> feat_idx(seq_len, -1);
    int injected = 0;
    for (int t = 0; t < seq_len; ++t)
    {
        if (input_ids[t] != image_token_id) continue;
        if (injected >= vision_token_count) return fail(HY_ERR_INVALID_ARGUMENT, "more image tokens than vision features");
        feat_idx[t] = injected++;
    }
    if (injected != vision_token_count)
        return fail(HY_ERR_INVALID_ARGUMENT, "image token count mismatch: injected " + std::to_string(injected) +
                                                 ", expected " + std::to_string(vision_token_count));
    int rc = set_device(c);
    if (rc) return rc;
    // The prompt's host inputs and tables go through the context's pinned staging
    // area (filled on the host, then copied without a staging pass in the driver);
    // the previous call finished with it before returning.
    const PromptStage ps = prompt_stage(c);
    std::memcpy(ps.ids, input_ids, sizeof(int) * seq_len);
    std::memcpy(ps.feat_idx, feat_idx.data(), sizeof(int) * seq_len);
    std::memcpy(ps.feats, vision_features, sizeof(float) * vision_token_count * kHidden);
    // mRoPE tables: gathered on the device from the 1-D table when every position
    // lies inside it (mrope_gather_kernel), else built on the host.
    bool gather = true;
    for (int i = 0; i < 4 * seq_len && gather; ++i) gather = position_ids[i] >= 0 && position_ids[i] < c->cfg.max_context;
    int* ps_pos = reinterpret_cast<int*>(ps.cos);   // (the table staging holds 4 x seq ints)
    if (gather) std::memcpy(ps_pos, position_ids, sizeof(int) * 4 * seq_len);
    else if ((rc = hy_build_mrope(position_ids, seq_len, 1, ps.cos)) ||
             (rc = hy_build_mrope(position_ids, seq_len, 0, ps.sin)))
        return rc;
    HY_CUDA(cudaEventRecord(c->tev[0], c->stream));
    HY_CUDA(cudaMemcpyAsync(c->ids_buf, ps.ids, sizeof(int) * seq_len, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->feat_idx, ps.feat_idx, sizeof(int) * seq_len, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->feats, ps.feats, sizeof(float) * vision_token_count * kHidden, cudaMemcpyHostToDevice,
                            c->stream));
    if (gather)
    {
        HY_CUDA(cudaMemcpyAsync(c->pre_pos, ps_pos, sizeof(int) * 4 * seq_len, cudaMemcpyHostToDevice, c->stream));
        mrope_gather_kernel<<<seq_len, kHeadDim, 0, c->stream>>>(c->pre_pos, seq_len, c->rope_cos, c->rope_sin,
                                                                 c->cfg.max_context, c->pre_cos, c->pre_sin, c->err);
        HY_CUDA(cudaGetLastError());
    }
    else
    {
        HY_CUDA(cudaMemcpyAsync(c->pre_cos, ps.cos, sizeof(float) * seq_len * kHeadDim, cudaMemcpyHostToDevice, c->stream));
        HY_CUDA(cudaMemcpyAsync(c->pre_sin, ps.sin, sizeof(float) * seq_len * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    }
    if (c->cfg.weight_dtype == HY_DTYPE_BF16)
        embed_prompt_kernel<__nv_bfloat16><<<seq_len, 256, 0, c->stream>>>(
            c->ids_buf, c->feat_idx, c->feats, static_cast<const __nv_bfloat16*>(c->embed), c->cfg.vocab_size, c->prompt, c->err);
    else
        embed_prompt_kernel<float><<<seq_len, 256, 0, c->stream>>>(c->ids_buf, c->feat_idx, c->feats,
                                                                     static_cast<const float*>(c->embed),
                                                                     c->cfg.vocab_size, c->prompt, c->err);
    HY_CUDA(cudaGetLastError());
    // History = prompt ids (src/text_runtime.cpp:1393).
    HY_CUDA(cudaMemsetAsync(c->hist, 0, sizeof(unsigned) * ((c->cfg.vocab_size + 31) / 32), c->stream));
    hist_add_kernel<<<(seq_len + 255) / 256, 256, 0, c->stream>>>(c->hist, c->ids_buf, seq_len, c->cfg.vocab_size);
    HY_CUDA(cudaGetLastError());
    HY_CUDA(cudaEventRecord(c->tev[1], c->stream));
    if ((rc = run_prefill(c, seq_len))) return rc;
    HY_CUDA(cudaEventRecord(c->tev[2], c->stream));
    cudaError_t e = enqueue_lm_select(c, 1, c->hidden, repetition_penalty, false, nullptr);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("LM head launch: ") + cudaGetErrorString(e));
    HY_CUDA(cudaEventRecord(c->tev[3], c->stream));
    HY_CUDA(cudaMemcpyAsync(c->h_small, c->tok_out, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->h_small + 1, c->raw_out, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    if ((rc = check_device_error(c))) return rc;
    *first = c->h_small[0];
    *first_raw = c->h_small[1];
    if ((rc = set_length(c, seq_len))) return rc;
    if (c->d_layers > 0) c->d_len = seq_len;
    // Device time of the prompt stages (the events have completed).
    float te = 0.f, tp = 0.f, tl = 0.f;
    HY_CUDA(cudaEventElapsedTime(&te, c->tev[0], c->tev[1]));
    HY_CUDA(cudaEventElapsedTime(&tp, c->tev[1], c->tev[2]));
    HY_CUDA(cudaEventElapsedTime(&tl, c->tev[2], c->tev[3]));
    c->timing.text_embed_ms = te;
    c->timing.prefill_ms = tp;
    c->timing.lm_head_ms = tl;
    c->timing.token_select_ms = 0.0;
    return HY_OK;
}

int hy_run_vlm_decode_with_prompt(hy_ctx* c, const int* input_ids, const int* position_ids, int seq_len,
                                  int image_token_id, const float* vision_features, int vision_token_count,
                                  int max_tokens, float repetition_penalty, const int* eos_ids, int n_eos, int* tokens,
                                  int* raw_top1, int* n_tokens)
{
    if (!c || !n_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (max_tokens <= 0) max_tokens = 1024;   // src/text_runtime.cpp:1336-1341
    if (max_tokens > c->cfg.max_tokens) return fail(HY_ERR_CAPACITY, "max_tokens exceeds config max_tokens");
    const auto t0 = TimingClock::now();
    c->timing = hy_decode_timing{};
    int first = 0, first_raw = 0;
    int rc = prompt_prefill_first(c, input_ids, position_ids, seq_len, image_token_id, vision_features,
                                  vision_token_count, repetition_penalty, &first, &first_raw);
    if (rc) return finish_timing(c, t0, rc);
    return finish_timing(c, t0, generate_impl(c, first, first_raw, max_tokens, repetition_penalty, eos_ids, n_eos,
                                              tokens, raw_top1, n_tokens));
}

// ---- DFlash draft network --------------------------------------------------

static int draft_loaded_finish(hy_ctx* c, int rc)
{
    if (rc)
    {
        draft_free(c);
        return rc;
    }
    return draft_finish(c);
}

int hy_draft_load(hy_ctx* c, const hy_draft_weights* w)
{
    if (!c || !w || !w->fc || !w->hidden_norm || !w->norm || !w->layers)
        return fail(HY_ERR_INVALID_ARGUMENT, "DFlash draft weights are incomplete");
    for (int l = 0; l < w->num_layers; ++l)
    {
        const hy_layer_weights& lw = w->layers[l];
        if (!lw.input_norm || !lw.q_proj || !lw.k_proj || !lw.v_proj || !lw.query_norm || !lw.key_norm || !lw.o_proj ||
            !lw.post_norm || !lw.gate_proj || !lw.up_proj || !lw.down_proj)
            return fail(HY_ERR_INVALID_ARGUMENT, "DFlash draft layer " + std::to_string(l) + " weights are incomplete");
    }
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = draft_alloc(c, w->num_layers, w->mask_token))) return draft_loaded_finish(c, rc);
    return draft_loaded_finish(c, draft_upload(c, w));
}

int hy_draft_load_synthetic(hy_ctx* c, int num_layers, int mask_token, uint64_t seed, float std_dev, float norm_std)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "ctx is null");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = draft_alloc(c, num_layers, mask_token))) return draft_loaded_finish(c, rc);
    return draft_loaded_finish(c, draft_fill_synthetic(c, seed, std_dev, norm_std));
}

int hy_draft_context_length(const hy_ctx* c, int* rows)
{
    if (!c || !rows) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    *rows = c->d_len;
    return HY_OK;
}

int hy_draft_context_append(hy_ctx* c, const float* aux_hidden, int rows)
{
    if (!c || !aux_hidden) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (!draft_ready(c)) return fail(HY_ERR_NOT_READY, "DFlash draft runtime is not loaded");
    if (rows <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "DFlash target hidden shapes do not match");
    if (c->d_len + rows + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "draft context exceeds the KV capacity");
    int rc = set_device(c);
    if (rc) return rc;
    for (int p0 = 0; p0 < rows; p0 += c->pf_rows)
    {
        const int n = std::min(c->pf_rows, rows - p0);
        for (int i = 0; i < kAuxLayers; ++i)
            HY_CUDA(cudaMemcpy2DAsync(c->d_pf_aux + i * kHidden, sizeof(float) * kAuxWidth,
                                      aux_hidden + (static_cast<size_t>(i) * rows + p0) * kHidden, sizeof(float) * kHidden,
                                      sizeof(float) * kHidden, n, cudaMemcpyHostToDevice, c->stream));
        const cudaError_t e = enqueue_draft_context_rows(c, n, c->d_len + p0);
        if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("draft context launch: ") + cudaGetErrorString(e));
    }
    if ((rc = check_device_error(c))) return rc;
    c->d_len += rows;
    return HY_OK;
}

int hy_draft_run(hy_ctx* c, const float* noise, float* hidden)
{
    if (!c || !noise || !hidden) return fail(HY_ERR_INVALID_ARGUMENT, "DFlash output pointer is null");
    if (!draft_ready(c)) return fail(HY_ERR_NOT_READY, "DFlash draft runtime is not loaded");
    if (c->d_len <= 0) return fail(HY_ERR_INVALID_ARGUMENT, "invalid DFlash noise/context shape");
    if (c->d_len + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "draft block exceeds the KV capacity");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemcpyAsync(c->d_x, noise, sizeof(float) * kBlock * kHidden, cudaMemcpyHostToDevice, c->stream));
    t_next_plain = true;
    const cudaError_t e = enqueue_draft_forward(c, SRC_X, false, c->d_len, false);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("draft launch: ") + cudaGetErrorString(e));
    HY_CUDA(cudaMemcpyAsync(hidden, c->hidden, sizeof(float) * kBlock * kHidden, cudaMemcpyDeviceToHost, c->stream));
    return check_device_error(c);
}

static int draft_in_sync(hy_ctx* c)
{
    if (!draft_ready(c)) return fail(HY_ERR_NOT_READY, "DFlash draft runtime is not loaded");
    if (c->kv_len <= 0 || c->d_len != c->kv_len)
        return fail(HY_ERR_INVALID_ARGUMENT, "invalid DFlash block context: the draft context covers " +
                                                 std::to_string(c->d_len) + " of " + std::to_string(c->kv_len) + " rows");
    return HY_OK;
}

int hy_draft_propose(hy_ctx* c, int current_token, int* proposed)
{
    if (!c || !proposed) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    int rc = draft_in_sync(c);
    if (rc) return rc;
    if (current_token < 0 || current_token >= c->cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "invalid DFlash block context");
    if (c->kv_len + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    if ((rc = set_device(c))) return rc;
    c->h_st->kv_len = c->kv_len;
    c->h_st->cur_token = current_token;
    if ((rc = push_state(c))) return rc;
    t_next_plain = true;
    const cudaError_t e = enqueue_draft_forward(c, SRC_GATHER_BLOCK, true, 0, true);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("draft launch: ") + cudaGetErrorString(e));
    HY_CUDA(cudaMemcpyAsync(proposed, c->proposed, sizeof(int) * kBlock, cudaMemcpyDeviceToHost, c->stream));
    return check_device_error(c);
}

static int dflash_generate_impl(hy_ctx* c, int first_token, int max_tokens, float penalty, const int* eos_ids,
                                int n_eos, int* tokens, int* n_tokens, int* acceptance_lengths, int* n_blocks)
{
    if (!n_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    int rc = draft_in_sync(c);
    if (rc) return rc;
    if (max_tokens < 1 || max_tokens > c->cfg.max_tokens)
        return fail(HY_ERR_CAPACITY, "max_tokens must be in 1..config max_tokens");
    if (first_token < 0 || first_token >= c->cfg.vocab_size) return fail(HY_ERR_INVALID_ARGUMENT, "first_token out of range");
    if (!std::isfinite(penalty) || penalty <= 0.f) return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    if (c->kv_len + max_tokens + kBlock > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    if ((rc = set_device(c))) return rc;
    if ((rc = set_eos(c, eos_ids, n_eos))) return rc;
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.cur_token = first_token;
    h.n_gen = 0;
    h.max_tokens = max_tokens;
    h.done = 0;
    h.penalty = penalty;
    h.block_count = 0;
    if ((rc = push_state(c))) return rc;
    int launched = 0;
    c->cb_emitted = 0;
    hy_dflash_timing& t = c->dtiming;
    while (!h.done && launched < max_tokens)
    {
        int n = 0;
        for (; n < kDflashGraphs && launched < max_tokens; ++n, ++launched)
            HY_CUDA(cudaGraphLaunch(c->g_dflash[n], c->stream));
        HY_CUDA(cudaEventRecord(c->tev[5], c->stream));
        if ((rc = sync_state_to_host(c))) return rc;
        // Stage times of this group's blocks (each block ends where the next starts).
        for (int b = 0; b < n; ++b)
        {
            float a = 0.f, v = 0.f, m = 0.f;
            HY_CUDA(cudaEventElapsedTime(&a, c->dflash_ev[b][0], c->dflash_ev[b][1]));
            HY_CUDA(cudaEventElapsedTime(&v, c->dflash_ev[b][1], c->dflash_ev[b][2]));
            HY_CUDA(cudaEventElapsedTime(&m, c->dflash_ev[b][2], b + 1 < n ? c->dflash_ev[b + 1][0] : c->tev[5]));
            t.draft_ms += a;
            t.verify_ms += v;
            t.commit_ms += m;
        }
        if (c->cb && (rc = check_device_error(c)) == HY_OK) rc = emit_tokens(c, h.n_gen);
        if (rc) return rc;
    }
    t.blocks_ms = t.draft_ms + t.verify_ms + t.commit_ms;
    if ((rc = check_device_error(c))) return rc;
    if ((rc = sync_state_to_host(c))) return rc;
    if ((rc = emit_tokens(c, h.n_gen))) return rc;
    c->d_len = c->kv_len;
    *n_tokens = h.n_gen;
    if (n_blocks) *n_blocks = h.block_count;
    return dflash_results(c, tokens, acceptance_lengths);
}

int hy_dflash_generate(hy_ctx* c, int first_token, int max_tokens, float penalty, const int* eos_ids, int n_eos,
                       int* tokens, int* n_tokens, int* acceptance_lengths, int* n_blocks)
{
    if (!c) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    const auto t0 = TimingClock::now();
    c->dtiming = hy_dflash_timing{};
    return finish_dflash_timing(c, t0, dflash_generate_impl(c, first_token, max_tokens, penalty, eos_ids, n_eos, tokens,
                                                            n_tokens, acceptance_lengths, n_blocks));
}

int hy_run_vlm_dflash_with_prompt(hy_ctx* c, const int* input_ids, const int* position_ids, int seq_len,
                                  int image_token_id, const float* vision_features, int vision_token_count,
                                  int max_tokens, float repetition_penalty, const int* eos_ids, int n_eos, int* tokens,
                                  int* n_tokens, int* acceptance_lengths, int* n_blocks)
{
    if (!c || !n_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (!draft_ready(c)) return fail(HY_ERR_NOT_READY, "DFlash draft runtime is not loaded");
    if (max_tokens <= 0) max_tokens = 1024;   // src/text_runtime.cpp:1168-1171
    if (max_tokens > c->cfg.max_tokens) return fail(HY_ERR_CAPACITY, "max_tokens exceeds config max_tokens");
    const auto t0 = TimingClock::now();
    c->dtiming = hy_dflash_timing{};
    int first = 0, first_raw = 0;
    int rc = prompt_prefill_first(c, input_ids, position_ids, seq_len, image_token_id, vision_features,
                                  vision_token_count, repetition_penalty, &first, &first_raw);
    c->dtiming.prefill_ms = c->timing.text_embed_ms + c->timing.prefill_ms + c->timing.lm_head_ms;
    if (rc) return finish_dflash_timing(c, t0, rc);
    return finish_dflash_timing(c, t0, dflash_generate_impl(c, first, max_tokens, repetition_penalty, eos_ids, n_eos,
                                                            tokens, n_tokens, acceptance_lengths, n_blocks));
}

// ---- batched decode -----------------------------------------------------

// Prefill request r into slot `slot`'s cache and make the slot decode it: the
// context's own KV pointers are aimed at the slot for the prefill.
static int batch_admit(hy_ctx* c, int slot, const hy_request& r, int max_tokens, float penalty, const int* eos_ids,
                       int n_eos, bool* finished)
{
    if (r.seq_len <= 0 || r.seq_len > c->cfg.max_prefill || r.seq_len + max_tokens > c->cfg.max_context)
        return fail(HY_ERR_CAPACITY, "request of " + std::to_string(r.seq_len) + " prompt rows + " +
                                         std::to_string(max_tokens) + " tokens exceeds the context's capacity");
    void* const kc0 = c->kc;
    void* const vc0 = c->vc;
    const int d_layers = c->d_layers;
    const size_t off = static_cast<size_t>(slot) * c->slot_elems() * c->kv_elem();
    c->kc = static_cast<char*>(c->b_kc) + off;
    c->vc = static_cast<char*>(c->b_vc) + off;
    c->d_layers = 0;   // slots keep no draft context
    int first = 0, first_raw = 0;
    int rc = prompt_prefill_first(c, r.input_ids, r.position_ids, r.seq_len, r.image_token_id, r.vision_features,
                                  r.vision_token_count, penalty, &first, &first_raw);
    c->kc = kc0;
    c->vc = vc0;
    c->d_layers = d_layers;
    if (rc) return rc;
    const int hw = c->hist_words();
    unsigned* hist = c->b_hist + static_cast<size_t>(slot) * hw;
    HY_CUDA(cudaMemcpyAsync(hist, c->hist, sizeof(unsigned) * hw, cudaMemcpyDeviceToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->b_cur + slot, &first, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    hist_add_kernel<<<1, 256, 0, c->stream>>>(hist, c->b_cur + slot, 1, c->cfg.vocab_size);
    HY_CUDA(cudaGetLastError());
    const size_t lo = static_cast<size_t>(slot) * c->log_stride();
    HY_CUDA(cudaMemcpyAsync(c->b_log + lo, &first, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->b_lograw + lo, &first_raw, sizeof(int), cudaMemcpyHostToDevice, c->stream));
    bool first_eos = false;
    for (int i = 0; i < n_eos; ++i) first_eos |= (eos_ids[i] == first);
    SlotState& st = c->h_bstate[slot];
    st.kv_len = r.seq_len;
    st.n_gen = 1;
    st.max_tokens = max_tokens;
    st.active = (first_eos || max_tokens <= 1) ? 0 : 1;
    HY_CUDA(cudaMemcpyAsync(c->b_state + slot, &st, sizeof(SlotState), cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaStreamSynchronize(c->stream));
    *finished = !st.active;
    return HY_OK;
}

int hy_batch_decode(hy_ctx* c, const hy_request* requests, int n_requests, int slots, int max_tokens,
                    float repetition_penalty, const int* eos_ids, int n_eos, int* tokens, int* n_tokens, int* status)
{
    if (!c || (n_requests > 0 && (!requests || !tokens || !n_tokens))) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (n_requests < 0) return fail(HY_ERR_INVALID_ARGUMENT, "n_requests must not be negative");
    if (slots < 1 || slots > kMaxStepRows) return fail(HY_ERR_INVALID_ARGUMENT, "slots must be in 1..16");
    if (max_tokens < 1 || max_tokens > c->cfg.max_tokens)
        return fail(HY_ERR_CAPACITY, "max_tokens must be in 1..config max_tokens");
    if (!std::isfinite(repetition_penalty) || repetition_penalty <= 0.f)
        return fail(HY_ERR_INVALID_ARGUMENT, "repetition_penalty must be positive");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = set_eos(c, eos_ids, n_eos))) return rc;
    c->h_st->penalty = repetition_penalty;
    if ((rc = push_state(c))) return rc;
    if ((rc = batch_prepare(c, slots))) return rc;
    std::vector<int> owner(slots, -1);
    auto finish = [&](int s) -> int {
        const int r = owner[s];
        const int n = c->h_bstate[s].n_gen;
        HY_CUDA(cudaMemcpy(tokens + static_cast<size_t>(r) * max_tokens, c->b_log + static_cast<size_t>(s) * c->log_stride(),
                           sizeof(int) * n, cudaMemcpyDeviceToHost));
        n_tokens[r] = n;
        if (status) status[r] = HY_OK;
        owner[s] = -1;
        return HY_OK;
    };
    int next = 0;
    for (;;)
    {
        for (int s = 0; s < slots; ++s)
            while (owner[s] < 0 && next < n_requests)
            {
                const int r = next++;
                bool fin = false;
                n_tokens[r] = 0;
                rc = batch_admit(c, s, requests[r], max_tokens, repetition_penalty, eos_ids, n_eos, &fin);
                if (rc == HY_ERR_INVALID_ARGUMENT || rc == HY_ERR_CAPACITY)
                {
                    // A malformed record fails alone (run_jsonl_batch writes an error record and goes on).
                    if (status) status[r] = rc;
                    continue;
                }
                if (rc) return rc;
                owner[s] = r;
                if (fin && (rc = finish(s))) return rc;
            }
        bool any = false;
        for (int s = 0; s < slots; ++s) any |= owner[s] >= 0;
        if (!any) break;
        for (int i = 0; i < 4; ++i) HY_CUDA(cudaGraphLaunch(c->g_batch, c->stream));
        HY_CUDA(cudaMemcpyAsync(c->h_bstate, c->b_state, sizeof(SlotState) * kMaxStepRows, cudaMemcpyDeviceToHost,
                                c->stream));
        if ((rc = check_device_error(c))) return rc;
        for (int s = 0; s < slots; ++s)
            if (owner[s] >= 0 && !c->h_bstate[s].active && (rc = finish(s))) return rc;
    }
    // The context's own sequence was used for the prompts' first tokens: leave it empty.
    c->d_len = 0;
    HY_CUDA(cudaMemsetAsync(c->hist, 0, sizeof(unsigned) * c->hist_words(), c->stream));
    return set_length(c, 0);
}

// ---- regression fixtures (host only) -------------------------------------

// parse_vlm_fixture_meta (src/text_runtime.cpp:285-321): key=value lines.
static int fixture_meta(const std::string& dir, int* seq_len, int* expected, int* image_token, int* vision)
{
    const std::string path = dir + "/meta.txt";
    std::ifstream f(path);
    if (!f.is_open()) return fail(HY_ERR_INVALID_ARGUMENT, "failed to open fixture meta: " + path);
    int m[4] = {0, 0, -1, 0};
    const char* keys[4] = {"seq_len", "expected_token_count", "image_token_id", "vision_token_count"};
    std::string line;
    while (std::getline(f, line))
    {
        if (line.empty()) continue;
        const size_t eq = line.find('=');
        if (eq == std::string::npos) continue;
        const std::string key = line.substr(0, eq), value = line.substr(eq + 1);
        for (int i = 0; i < 4; ++i)
        {
            if (key != keys[i]) continue;
            char* end = nullptr;
            errno = 0;
            const long v = std::strtol(value.c_str(), &end, 10);
            if (end == value.c_str() || errno != 0 || v < -2147483647L || v > 2147483647L)
                return fail(HY_ERR_INVALID_ARGUMENT, "invalid fixture meta value: " + line);
            m[i] = static_cast<int>(v);
        }
    }
    if (m[0] <= 0 || m[1] <= 0 || m[2] < 0 || m[3] <= 0)
        return fail(HY_ERR_INVALID_ARGUMENT,
                    "vlm fixture meta must define positive seq_len, expected_token_count, image_token_id, and "
                    "vision_token_count");
    *seq_len = m[0];
    *expected = m[1];
    *image_token = m[2];
    *vision = m[3];
    return HY_OK;
}

// read_binary_vector (src/text_runtime.cpp:253-276): exactly `count` elements, no extra bytes.
static int fixture_vector(const std::string& path, size_t count, size_t elem, void* out)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) return fail(HY_ERR_INVALID_ARGUMENT, "failed to open: " + path);
    f.read(static_cast<char*>(out), static_cast<std::streamsize>(count * elem));
    if (f.gcount() != static_cast<std::streamsize>(count * elem)) return fail(HY_ERR_INVALID_ARGUMENT, "short read: " + path);
    char extra = 0;
    if (f.read(&extra, 1)) return fail(HY_ERR_INVALID_ARGUMENT, "unexpected extra bytes: " + path);
    return HY_OK;
}

int hy_fixture_meta(const char* fixture_dir, int* seq_len, int* expected_token_count, int* image_token_id,
                    int* vision_token_count)
{
    if (!fixture_dir || !seq_len || !expected_token_count || !image_token_id || !vision_token_count)
        return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    return fixture_meta(fixture_dir, seq_len, expected_token_count, image_token_id, vision_token_count);
}

int hy_fixture_load(const char* fixture_dir, int seq_capacity, int expected_capacity, int vision_capacity,
                    int* input_ids, int* position_ids, int* expected_tokens, float* vision_features)
{
    if (!fixture_dir || !input_ids || !position_ids || !expected_tokens) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    int seq = 0, expected = 0, image = 0, vision = 0;
    int rc = fixture_meta(fixture_dir, &seq, &expected, &image, &vision);
    if (rc) return rc;
    // meta.txt is read again here: the buffers were sized from an earlier read,
    // which the file may no longer match.
    if (seq > seq_capacity || expected > expected_capacity || (vision_features && vision > vision_capacity))
        return fail(HY_ERR_CAPACITY, "fixture meta asks for seq_len=" + std::to_string(seq) +
                                         ", expected_token_count=" + std::to_string(expected) +
                                         ", vision_token_count=" + std::to_string(vision) +
                                         " but the buffers hold " + std::to_string(seq_capacity) + ", " +
                                         std::to_string(expected_capacity) + ", " + std::to_string(vision_capacity));
    const std::string root(fixture_dir);
    if ((rc = fixture_vector(root + "/input_ids.i32", seq, sizeof(int), input_ids))) return rc;
    if ((rc = fixture_vector(root + "/position_ids.i32", static_cast<size_t>(seq) * 4, sizeof(int), position_ids)))
        return rc;
    if ((rc = fixture_vector(root + "/expected_tokens.i32", expected, sizeof(int), expected_tokens))) return rc;
    if (vision_features &&
        (rc = fixture_vector(root + "/vision_features.f32", static_cast<size_t>(vision) * kHidden, sizeof(float),
                             vision_features)))
        return rc;
    return HY_OK;
}

int hy_attention(hy_ctx* c, int layer, const float* qkv, int rows, const float* cos, const float* sin, float* out)
{
    if (!c || !qkv || !cos || !sin || !out) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    if (layer < 0 || layer >= c->cfg.num_layers) return fail(HY_ERR_INVALID_ARGUMENT, "layer out of range");
    if (rows < 1 || rows > kMaxStepRows) return fail(HY_ERR_INVALID_ARGUMENT, "rows must be in 1..16");
    if (c->kv_len + rows > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    int rc = set_device(c);
    if (rc) return rc;
    HY_CUDA(cudaMemcpyAsync(c->qkv, qkv, sizeof(float) * rows * kQKVRows, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_cos, cos, sizeof(float) * rows * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    HY_CUDA(cudaMemcpyAsync(c->pre_sin, sin, sizeof(float) * rows * kHeadDim, cudaMemcpyHostToDevice, c->stream));
    AttnArgs at;
    std::memset(&at, 0, sizeof(at));
    at.qkv = c->qkv;
    at.ldq = kQKVRows;
    at.qn_w = c->qn(layer);
    at.kn_w = c->kn(layer);
    at.cos = c->pre_cos;
    at.sin = c->pre_sin;
    at.kc = c->kc_layer(layer);
    at.vc = c->vc_layer(layer);
    at.cap = c->cfg.max_context;
    at.past_fixed = c->kv_len;
    at.rows = rows;
    at.scale_log2 = c->cfg.attn_scale * 1.4426950408889634f;
    at.eps = c->cfg.rms_norm_eps;
    at.part = c->attn_part;
    at.counter = c->attn_cnt + layer * kNumKVHeads;
    at.out = c->attn;
    at.err = c->err;
    const bool kb = c->cfg.kv_dtype == HY_DTYPE_BF16;
    cudaError_t e;
    t_next_plain = true;
    if (rows == 1)
        e = kb ? run_attn<1, __nv_bfloat16>(c, at, kAttnSplitsAR) : run_attn<1, float>(c, at, kAttnSplitsAR);
    else
        e = kb ? run_attn16<__nv_bfloat16>(c, at) : run_attn16<float>(c, at);
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
    HY_CUDA(cudaMemcpyAsync(out, c->attn, sizeof(float) * rows * kQWidth, cudaMemcpyDeviceToHost, c->stream));
    if ((rc = check_device_error(c))) return rc;
    return set_length(c, c->kv_len + rows);
}

static int kv_copy(hy_ctx* c, int layer, int start, int rows, const float* k, const float* v, float* ko, float* vo)
{
    if (!c || layer < 0 || layer >= c->cfg.num_layers || start < 0 || rows <= 0 ||
        start + rows > c->cfg.max_context)
        return fail(HY_ERR_INVALID_ARGUMENT, "invalid KV range");
    int rc = set_device(c);
    if (rc) return rc;
    const size_t es = c->kv_elem();
    const size_t n = static_cast<size_t>(rows) * kHeadDim;
    float* stage = c->kv_stage;   // [max_context x 128]: one head's rows at a time (reuse ordered by the stream)
    for (int which = 0; which < 2; ++which)
    {
        char* base = static_cast<char*>(which == 0 ? c->kc_layer(layer) : c->vc_layer(layer));
        for (int g = 0; g < kNumKVHeads; ++g)
        {
            char* dst = base + (static_cast<size_t>(g) * c->cfg.max_context + start) * kHeadDim * es;
            const float* hin = (which == 0 ? k : v);
            float* hout = (which == 0 ? ko : vo);
            if (hin)
            {
                if (es == 4)
                    HY_CUDA(cudaMemcpyAsync(dst, hin + g * n, n * 4, cudaMemcpyHostToDevice, c->stream));
                else
                {
                    HY_CUDA(cudaMemcpyAsync(stage, hin + g * n, n * 4, cudaMemcpyHostToDevice, c->stream));
                    f32_to_bf16_kernel<<<64, 256, 0, c->stream>>>(stage, reinterpret_cast<__nv_bfloat16*>(dst), n);
                }
            }
            if (hout)
            {
                if (es == 4)
                    HY_CUDA(cudaMemcpyAsync(hout + g * n, dst, n * 4, cudaMemcpyDeviceToHost, c->stream));
                else
                {
                    to_f32_kernel<__nv_bfloat16><<<64, 256, 0, c->stream>>>(reinterpret_cast<const __nv_bfloat16*>(dst),
                                                                             stage, n);
                    HY_CUDA(cudaMemcpyAsync(hout + g * n, stage, n * 4, cudaMemcpyDeviceToHost, c->stream));
                }
            }
        }
    }
    HY_CUDA(cudaStreamSynchronize(c->stream));
    return HY_OK;
}

int hy_kv_write(hy_ctx* c, int layer, int start, int rows, const float* k, const float* v)
{
    if (!k || !v) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    return kv_copy(c, layer, start, rows, k, v, nullptr, nullptr);
}

int hy_kv_read(hy_ctx* c, int layer, int start, int rows, float* k, float* v)
{
    if (!k || !v) return fail(HY_ERR_INVALID_ARGUMENT, "null argument");
    return kv_copy(c, layer, start, rows, nullptr, nullptr, k, v);
}

int hy_bench_ar_steps(hy_ctx* c, int count, float* ms)
{
    if (!c || !ms || count < 1) return fail(HY_ERR_INVALID_ARGUMENT, "invalid arguments");
    int rc = set_device(c);
    if (rc) return rc;
    DecodeState& h = *c->h_st;
    h.kv_len = c->kv_len;
    h.n_gen = 1;
    h.max_tokens = std::min(c->cfg.max_tokens, count * kArStepsPerGraph + 2);
    h.done = 0;
    h.n_eos = 0;
    if (c->kv_len + h.max_tokens > c->cfg.max_context) return fail(HY_ERR_CAPACITY, "KV capacity exceeded");
    if ((rc = push_state(c))) return rc;
    cudaEvent_t e0, e1;
    HY_CUDA(cudaEventCreate(&e0));
    HY_CUDA(cudaEventCreate(&e1));
    const int graphs = (count + kArStepsPerGraph - 1) / kArStepsPerGraph;
    HY_CUDA(cudaEventRecord(e0, c->stream));
    if (c->ar_path == HY_AR_PATH_PERSISTENT)
    {
        for (int done = 0; done < count; done += kMegaChunk)
        {
            cudaError_t e = launch_mega(c, std::min(kMegaChunk, count - done));
            if (e != cudaSuccess) return fail(HY_ERR_CUDA, std::string("persistent decode launch: ") + cudaGetErrorString(e));
        }
    }
    else
    {
        for (int i = 0; i < graphs; ++i) HY_CUDA(cudaGraphLaunch(c->g_ar, c->stream));
    }
    HY_CUDA(cudaEventRecord(e1, c->stream));
    HY_CUDA(cudaEventSynchronize(e1));
    float t = 0.f;
    HY_CUDA(cudaEventElapsedTime(&t, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms = t;
    if ((rc = check_device_error(c))) return rc;
    // Restore the sequence length the steps advanced.
    return set_length(c, c->kv_len);
}

int hy_bench_kernel(hy_ctx* c, int which, int count, float* ms)
{
    if (!c || !ms || count < 1) return fail(HY_ERR_INVALID_ARGUMENT, "invalid arguments");
    int rc = set_device(c);
    if (rc) return rc;
    cudaEvent_t e0, e1;
    HY_CUDA(cudaEventCreate(&e0));
    HY_CUDA(cudaEventCreate(&e1));
    const bool wb = c->cfg.weight_dtype == HY_DTYPE_BF16;
    auto once = [&]() -> cudaError_t {
        if (which == 0)
            return enqueue_lm_select(c, 1, c->hidden, 1.08f, false, nullptr);
        if (which == 1)
        {
            GemvArgs gu = base_args(c);
            gu.W = c->wgu[0];
            gu.N = 2 * c->cfg.ffn_dim;
            gu.ldw = kHidden;
            gu.rows = 1;
            gu.src = SRC_X;
            gu.x = c->x;
            gu.ldx = kHidden;
            gu.norm_w = c->post_norm(0);
            gu.out = c->gu;
            gu.ldo = 2 * c->cfg.ffn_dim;
            return wb ? run_gemv<__nv_bfloat16, kHidden, 1, PRO_NORM, EPI_STORE>(c, gu)
                      : run_gemv<float, kHidden, 1, PRO_NORM, EPI_STORE>(c, gu);
        }
        AttnArgs at;
        std::memset(&at, 0, sizeof(at));
        at.qkv = c->qkv;
        at.ldq = kQKVRows;
        at.qn_w = c->qn(0);
        at.kn_w = c->kn(0);
        at.cos = c->rope_cos;
        at.sin = c->rope_sin;
        at.rope_state = 0;
        at.kc = c->kc_layer(0);
        at.vc = c->vc_layer(0);
        at.cap = c->cfg.max_context;
        at.past_fixed = c->kv_len;
        at.rows = 1;
        at.scale_log2 = c->cfg.attn_scale * 1.4426950408889634f;
        at.eps = c->cfg.rms_norm_eps;
        at.part = c->attn_part;
        at.counter = c->attn_cnt;
        at.out = c->attn;
        at.err = c->err;
        return c->cfg.kv_dtype == HY_DTYPE_BF16 ? run_attn<1, __nv_bfloat16>(c, at, kAttnSplitsAR)
                                                : run_attn<1, float>(c, at, kAttnSplitsAR);
    };
    cudaError_t e = once();  // warm-up
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, cudaGetErrorString(e));
    HY_CUDA(cudaEventRecord(e0, c->stream));
    for (int i = 0; i < count && e == cudaSuccess; ++i) e = once();
    HY_CUDA(cudaEventRecord(e1, c->stream));
    if (e != cudaSuccess) return fail(HY_ERR_CUDA, cudaGetErrorString(e));
    HY_CUDA(cudaEventSynchronize(e1));
    float t = 0.f;
    HY_CUDA(cudaEventElapsedTime(&t, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms = t / count;
    return check_device_error(c);
}

}  // extern "C"
