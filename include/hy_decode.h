/*
 * hy_decode.h — C ABI of the B200 (sm_100a) text-decode library for
 * HunyuanOCR 1.5's 24-layer text decoder.
 *
 * The library replaces the text-decode hot path of HunyuanOCR-ncnn: the ncnn
 * decoder net driven by src/text_runtime.cpp, the PreciseSDPA and
 * MultimodalRotaryEmbed custom layers, the KV-cache append helpers, the tied
 * LM head and host token selection, and the DFlash verify/accept/rollback
 * logic. Every entry point below names the reference interface it replaces
 * (paths are relative to the HunyuanOCR-ncnn source tree).
 *
 * Conventions (mirroring the reference's `bool f(..., std::string* error)`):
 *   - every function returns an int status, HY_OK (0) on success;
 *   - on failure hy_last_error() returns a message for the calling thread;
 *   - all pointers are HOST pointers unless a name says otherwise, tensors
 *     are dense row-major fp32 (ids int32), sizes are element counts;
 *   - one context owns one device, one CUDA stream, the weights and one
 *     sequence's KV cache; calls on one context must not overlap (the
 *     reference runtime is sequential too, README_en.md:167).
 */
#ifndef HY_DECODE_H
#define HY_DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum hy_status {
    HY_OK = 0,
    HY_ERR_INVALID_ARGUMENT = 1,
    HY_ERR_CUDA = 2,
    HY_ERR_OUT_OF_MEMORY = 3,
    HY_ERR_CAPACITY = 4,       /* KV / prompt / token capacity exceeded */
    HY_ERR_DEVICE_TIMEOUT = 5, /* a bounded device wait gave up */
    HY_ERR_NOT_READY = 6,
    HY_ERR_UNSUPPORTED = 7
};

enum hy_dtype { HY_DTYPE_F32 = 0, HY_DTYPE_BF16 = 1 };

/* Fixed model geometry: src/text_decoder_step.h:19-24. */
#define HY_HIDDEN 1024
#define HY_HEAD_DIM 128
#define HY_NUM_Q_HEADS 16
#define HY_NUM_KV_HEADS 8
/* DFlash block (include/hunyuan_ocr/dflash_runtime.h:17-18). */
#define HY_DFLASH_BLOCK 16
#define HY_DFLASH_MASK_TOKEN 120817
/* Rows one decoder step accepts: 1 (AR) up to a DFlash block. */
#define HY_MAX_STEP_ROWS 16
/* Aux hidden states exported for the DFlash draft net
 * (export/text_decoder_kv.py:11, layers 1, 8, 15, 22). */
#define HY_NUM_AUX_LAYERS 4

typedef struct hy_config {
    int num_layers;     /* 24 */
    int vocab_size;     /* 120818 */
    int ffn_dim;        /* 3584; a multiple of 128 */
    int max_context;    /* KV rows reserved per layer (prompt + generated + one block) */
    int max_prefill;    /* longest prompt hy_prefill accepts */
    int max_tokens;     /* longest generation (device token log) */
    int weight_dtype;   /* HY_DTYPE_F32 (reference parity) or HY_DTYPE_BF16 */
    int kv_dtype;       /* HY_DTYPE_F32 or HY_DTYPE_BF16 */
    float rms_norm_eps; /* 1e-5 */
    float attn_scale;   /* 0.0883883: export/add_kvcache.py:26 prints 1/sqrt(128) with %g */
    int device;         /* CUDA device ordinal */
} hy_config;

/* nn.Linear layout [out x in]; norms are vectors (export/text_decoder_kv.py:49-96). */
typedef struct hy_layer_weights {
    const float* input_norm; /* [1024] */
    const float* q_proj;     /* [2048 x 1024] */
    const float* k_proj;     /* [1024 x 1024] */
    const float* v_proj;     /* [1024 x 1024] */
    const float* query_norm; /* [128] */
    const float* key_norm;   /* [128] */
    const float* o_proj;     /* [1024 x 2048] */
    const float* post_norm;  /* [1024] */
    const float* gate_proj;  /* [ffn x 1024] */
    const float* up_proj;    /* [ffn x 1024] */
    const float* down_proj;  /* [1024 x ffn] */
} hy_layer_weights;

typedef struct hy_weights {
    const float* embed;              /* [vocab x 1024]: text_embed and the tied LM head */
    const float* final_norm;         /* [1024] */
    const hy_layer_weights* layers;  /* [num_layers] */
} hy_weights;

typedef struct hy_ctx hy_ctx;

const char* hy_version(void);
const char* hy_last_error(void);

/* Defaults of the reference model (src/text_runtime.cpp:97-104). */
int hy_config_init(hy_config* cfg);

/* Replaces TextRuntime::load (src/text_runtime.cpp:1685-1749): uploads one
 * device copy of the weights (the tied table serves both embedding and LM
 * head, as SharedModelData does, src/mapped_model_file.h:50-67), reserves the
 * KV cache and the 1-D RoPE table, and captures the step graphs. */
int hy_ctx_create(const hy_config* cfg, const hy_weights* weights, hy_ctx** out);

/* Same, with the weights generated on the device by the library's seeded
 * counter generator (linears/embedding ~N(0, std), norms 1 + ~N(0, norm_std)).
 * Used for benchmarks on synthetic random-init weights. */
int hy_ctx_create_synthetic(const hy_config* cfg, uint64_t seed, float std, float norm_std, hy_ctx** out);

void hy_ctx_destroy(hy_ctx* ctx);

/* ---- model package (the reference's exported ncnn files) -------------- */
/* TextRuntime::load (src/text_runtime.cpp:1685-1749) from a model package
 * root (models/README.md): text_embed/text_embed.ncnn.{param,bin} - the tied
 * table, which the LM head's param also points at (1705-1745) - and
 * text_decoder/text_decoder_kv.ncnn.{param,bin}. The .bin files are
 * memory-mapped (src/mapped_model_file.cpp:156) and read in .param order by
 * ncnn's model-bin layout (fp32 or fp16 arrays); weights are found by the pnnx
 * layer names of the exported modules (layers.<i>.self_attn.q_proj, ...,
 * layers.<i>.mlp.down_proj, norm). num_layers, vocab_size and ffn_dim come
 * from the package; the other fields from cfg. One device copy of the weights,
 * the tied table shared by embedding and LM head. */
int hy_ctx_create_from_package(const hy_config* cfg, const char* model_root, hy_ctx** out);
/* DFlashDraftRuntime::load (src/dflash_runtime.cpp:175-201) from
 * <model_root>/dflash/dflash.ncnn.{param,bin} (fc, hidden_norm, layers.<i>.*,
 * norm), as hy_draft_load. */
int hy_draft_load_package(hy_ctx* ctx, const char* model_root, int mask_token);
/* Host-only checks of a package (no device work): its geometry, and one weight
 * as the reader sees it (field: embed, final_norm, or a hy_layer_weights field
 * name for `layer`; with draft != 0: fc, hidden_norm, norm or a draft layer's
 * field). draft_layers (nullable) is 0 without a dflash directory. */
int hy_package_inspect(const char* model_root, int* num_layers, int* vocab_size, int* ffn_dim, int* draft_layers);
int hy_package_read_tensor(const char* model_root, int draft, int layer, const char* field, float* out,
                           size_t capacity, size_t* count);

/* How hy_generate runs the AR loop. HY_AR_PATH_PERSISTENT (default): one
 * cooperative kernel per up to 64 tokens, one CTA per SM, all 24 layers and the
 * LM head of each token inside it; the CTAs exchange each phase's outputs as
 * epoch-tagged words that the next phase polls (no grid barrier).
 * HY_AR_PATH_GRAPH: one CUDA-graph replay of 121 kernels per token. Both compute
 * the same step (the reference's decode loop, src/text_runtime.cpp:1417-1508). */
enum hy_ar_path { HY_AR_PATH_PERSISTENT = 0, HY_AR_PATH_GRAPH = 1 };
int hy_ctx_set_ar_path(hy_ctx* ctx, int path);
int hy_ctx_ar_path(const hy_ctx* ctx);
/* Streaming (InferenceRequest::stream_callback, include/hunyuan_ocr/hunyuan_ocr.h:43-45,
 * and the TextTokenCallback of run_vlm_decode_with_prompt, text_runtime.h:21, 126-143):
 * callback(token, user) is called on the calling thread, in order, once for every
 * committed token of hy_generate, hy_dflash_generate(_synthetic) and the
 * hy_run_vlm_*_with_prompt calls (the first token included). The library calls it
 * when it reads the decode state: after every `tokens_per_sync` AR tokens (1..64,
 * 0 = 64; smaller values mean more launches of the persistent kernel) and after
 * every 4 DFlash blocks, so tokens arrive in small groups rather than one by one.
 * NULL removes the callback. */
typedef void (*hy_token_callback)(int token, void* user);
int hy_ctx_set_token_callback(hy_ctx* ctx, hy_token_callback callback, void* user, int tokens_per_sync);
int hy_ctx_config(const hy_ctx* ctx, hy_config* cfg);
size_t hy_ctx_device_bytes(const hy_ctx* ctx);   /* replaces mapped_weight_bytes() */

/* TextDecodeTiming (include/hunyuan_ocr/text_runtime.h:32-39, filled by host
 * clocks at src/text_runtime.cpp:1389-1511) of the last hy_generate /
 * hy_run_vlm_decode_with_prompt call on the context. Device stages are CUDA
 * events on the context's stream; total_ms is the host clock of the call. */
typedef struct hy_decode_timing {
    double text_embed_ms;     /* prompt upload, embedding with vision-feature injection, history */
    double prefill_ms;        /* prefill of all prompt rows */
    double decode_ms;         /* the decode loop: per token embed, all layers, LM head and selection
                                 (one fused kernel), launch gaps included */
    double lm_head_ms;        /* the first token's LM head and selection (later tokens': decode_ms) */
    double token_select_ms;   /* 0: selection is fused into the LM-head kernels */
    double total_ms;          /* host clock of the call */
    double host_overhead_ms;  /* total_ms minus the device stages: host work, copies, waits */
} hy_decode_timing;
int hy_ctx_last_timing(const hy_ctx* ctx, hy_decode_timing* out);

/* DFlashDecodeTiming (text_runtime.h:64-74, filled at src/text_runtime.cpp:
 * 913-1069, 1240-1302) with the counts of DFlashDecodeResult (76-83) and
 * DecoderStatistics (include/hunyuan_ocr/hunyuan_ocr.h:55-65) of the last
 * hy_dflash_generate / hy_run_vlm_dflash_with_prompt /
 * hy_dflash_generate_synthetic call. A block is one graph on the device; with
 * the draft network its stages are split by events inside every block's graph:
 * draft (draft_prepare + draft_infer + draft_postprocess of the reference),
 * verify (verify_prepare + verify_infer, with the block's draft context rows)
 * and commit (verify_postprocess + commit: LM head, posterior, acceptance,
 * commit and rollback). With the synthetic drafter only blocks_ms is split off. */
typedef struct hy_dflash_timing {
    double prefill_ms;        /* prompt upload, embedding, prefill and first token (device) */
    double draft_ms;
    double verify_ms;
    double commit_ms;
    double blocks_ms;         /* all blocks on the device */
    double total_ms;          /* host clock of the call */
    double host_overhead_ms;  /* total_ms minus prefill_ms and blocks_ms */
    int block_count;
    int drafted_token_count;          /* 15 per block */
    int accepted_draft_token_count;   /* sum of the acceptance lengths */
} hy_dflash_timing;
int hy_ctx_last_dflash_timing(const hy_ctx* ctx, hy_dflash_timing* out);

/* ---- host table builders (host code, no device work) ---------------- */
/* detail::build_mrope (src/text_runtime.cpp:42-63): position_ids [4 x seq]
 * axis-major, out [seq x 128]. */
int hy_build_mrope(const int* position_ids, int seq_len, int use_cos, float* out);
/* rope_value (src/text_runtime.cpp:182-193). */
float hy_rope_value(int position, int dim, int use_cos);

/* ---- sequence state --------------------------------------------------- */
/* Empty KV cache and penalty history. */
int hy_seq_reset(hy_ctx* ctx);
int hy_seq_length(hy_ctx* ctx, int* kv_rows);
/* view_dflash_rows (src/dflash_runtime.cpp:97-119): keep the first `rows` KV rows. */
int hy_seq_truncate(hy_ctx* ctx, int rows);
/* Penalty history = set(ids) (select_next_token's unordered_set,
 * src/text_runtime.cpp:744-750); hy_history_add inserts more ids. */
int hy_history_set(hy_ctx* ctx, const int* ids, int n);
int hy_history_add(hy_ctx* ctx, const int* ids, int n);

/* ---- decoder ---------------------------------------------------------- */
/* run_decoder_prefill (src/text_runtime.cpp:648-674) on an empty cache:
 * inputs_embeds [seq x 1024], cos/sin [seq x 128] (hy_build_mrope), causal mask
 * (make_prefill_mask, 207-219). Writes KV rows [0, seq). Outputs (nullable):
 * last_hidden [1024] = final-normed hidden of the last row; aux_hidden
 * [4 x seq x 1024] = un-normed hidden after layers 1, 8, 15, 22. */
int hy_prefill(hy_ctx* ctx, const float* inputs_embeds, const float* cos, const float* sin, int seq_len,
               float* last_hidden, float* aux_hidden);

/* detail::run_decoder_step (src/text_decoder_step.h:29-38): `rows` (1..16)
 * new embeddings at KV positions [len, len+rows) with row r attending to keys
 * <= len + r (make_decode_mask / build_dflash_verify_mask). cos/sin [rows x 128].
 * Appends the rows to the cache. hidden [rows x 1024] (final-normed, nullable),
 * aux_hidden [4 x rows x 1024] (nullable). */
int hy_decoder_step(hy_ctx* ctx, const float* embeds, int rows, const float* cos, const float* sin,
                    float* hidden, float* aux_hidden);

/* run_lm_head + select_logit_rows (src/text_runtime.cpp:430-439, 757-797) over
 * `rows` final-normed hidden rows [rows x 1024] with the context's penalty
 * history; row r also counts row_prefix[0..r] (nullable) as history.
 * tokens/raw_top1 [rows]; logits [rows x vocab] (nullable). */
int hy_lm_head_select(hy_ctx* ctx, const float* hidden, int rows, const int* row_prefix, float penalty,
                      int* tokens, int* raw_top1, float* logits);

/* No reference counterpart. hy_lm_head_select on DEVICE buffers that
 * allocates nothing: hidden_dev [rows x 1024] final-normed rows (16-byte
 * aligned), tokens_dev / raw_top1_dev [rows] written on the device, history
 * from the context, no row prefix, no logits. For callers that cannot
 * allocate device memory mid-decode (their memory is reserved by their own
 * caching allocator, or a cudaMalloc/cudaFree would synchronise a GPU shared
 * with other streams). The argmax kernel's scratch is a static device-global
 * array of 65,792 bytes (partials for at most 16 rows x 256 CTAs), one per
 * device and process: rows > 16 or a device launching more than 256 CTAs is
 * rejected with HY_ERR_CAPACITY, and calls that overlap in time on one device
 * race on the scratch. The first call on each device does a one-time set-up
 * (it resolves the array's device address with cudaGetSymbolAddress); make
 * that first call before any stream capture starts. Ordering: the call runs on
 * the context's stream (hy_ctx_stream), so hidden_dev must be complete before
 * it is made - synchronise the stream that wrote it, or record an event there
 * and make the context's stream wait on it. Every call blocks the calling
 * thread until the select has finished (it synchronises the context's stream
 * to read the device error word); tokens_dev / raw_top1_dev hold the result
 * on return. */
int hy_lm_head_select_noalloc(hy_ctx* ctx, const float* hidden_dev, int rows, float penalty, int* tokens_dev,
                              int* raw_top1_dev);

/* ---- on-device loops -------------------------------------------------- */
/* The AR loop of decode_from_embeddings (src/text_runtime.cpp:1417-1508):
 * starting from first_token (already selected from the prefill logits and
 * not yet in the history), runs up to max_tokens-1 decoder steps on the
 * device, each one CUDA-graph launch (embed -> 24 layers -> LM head ->
 * penalised argmax -> EOS check), with the token kept on the device.
 * tokens/raw_top1 (nullable) receive n_tokens ids including first_token;
 * raw_top1[0] is first_raw_top1. */
int hy_generate(hy_ctx* ctx, int first_token, int first_raw_top1, int max_tokens, float penalty,
                const int* eos_ids, int n_eos, int* tokens, int* raw_top1, int* n_tokens);

/* One DFlash block, the verify half of run_dflash_block plus the commit of
 * decode_dflash_from_embeddings (src/text_runtime.cpp:959-1070, 1240-1296):
 * verify forward over proposed[16] at the current length, posterior with the
 * per-row history, dflash_acceptance_length, commit of min(accept+1,
 * max_commit) tokens (cut at EOS) and KV rollback to length + committed.
 * posterior [16]; *stop is set when the commit hit EOS or was cut short. */
int hy_verify_block(hy_ctx* ctx, const int* proposed, int max_commit, float penalty, const int* eos_ids,
                    int n_eos, int* posterior, int* acceptance_length, int* committed, int* stop);

/* The DFlash loop (src/text_runtime.cpp:1206-1296) entirely on the device,
 * with a synthetic drafter standing in for the draft net: draft slot i of
 * block b is greedy[n_committed + i] with probability p, else a uniform id
 * (counter-generator stream `seed`). One graph launch per block. */
int hy_dflash_generate_synthetic(hy_ctx* ctx, int first_token, int max_tokens, float penalty,
                                 const int* eos_ids, int n_eos, const int* greedy, int n_greedy, float p,
                                 uint64_t seed, int* tokens, int* n_tokens, int* acceptance_lengths,
                                 int* n_blocks);

/* ---- DFlash draft network -------------------------------------------- */
/* Draft weights: the graph of export/dflash_export.py:40-177 (fc over the four
 * aux hidden states side by side, hidden_norm, draft layers, norm). Each draft
 * layer has the decoder layer's geometry and nn.Linear layout (q_norm /
 * k_norm in query_norm / key_norm; ffn = the context's ffn_dim). */
typedef struct hy_draft_weights {
    int num_layers;                 /* 1..8 */
    int mask_token;                 /* noise-block filler id: 120817
                                       (include/hunyuan_ocr/dflash_runtime.h:17-18) */
    const float* fc;                /* [1024 x 4096] */
    const float* hidden_norm;       /* [1024] */
    const float* norm;              /* [1024] */
    const hy_layer_weights* layers; /* [num_layers] */
} hy_draft_weights;

/* DFlashDraftRuntime::load (src/dflash_runtime.cpp:175-201): uploads the draft
 * (in the context's weight dtype) beside the decoder and reserves its K/V cache
 * of context rows. Replaces a draft loaded before. From then on every call that
 * appends KV rows (hy_prefill, hy_decoder_step, hy_verify_block,
 * hy_run_vlm_*_with_prompt) also appends the rows' draft context (k / v of
 * hidden_norm(fc(aux_1 | aux_8 | aux_15 | aux_22)) per draft layer) while the
 * draft context covers the sequence; hy_generate (AR) does not. */
int hy_draft_load(hy_ctx* ctx, const hy_draft_weights* weights);
/* Same with seeded synthetic draft weights (linears ~N(0, std), norms
 * 1 + ~N(0, norm_std)) from the library's counter generator. */
int hy_draft_load_synthetic(hy_ctx* ctx, int num_layers, int mask_token, uint64_t seed, float std, float norm_std);
/* Rows [0, rows) of the sequence that have draft context. */
int hy_draft_context_length(const hy_ctx* ctx, int* rows);
/* The target_hidden input of DFlashDraftRuntime::run for `rows` more context
 * rows (append_dflash_rows, src/dflash_runtime.cpp:121-166): aux_hidden
 * [4 x rows x 1024] (hy_decoder_step's layout), appended at positions
 * context_length .. context_length + rows - 1. */
int hy_draft_context_append(hy_ctx* ctx, const float* aux_hidden, int rows);
/* DFlashDraftRuntime::run (src/dflash_runtime.cpp:213-290): the draft graph for
 * noise [16 x 1024] at positions context_length .. + 15 over the draft context
 * (RoPE theta 10000, no mask); hidden [16 x 1024] = the final-normed rows. */
int hy_draft_run(hy_ctx* ctx, const float* noise, float* hidden);
/* The draft half of run_dflash_block (src/text_runtime.cpp:913-978) at the
 * sequence length: noise = embed([current_token, mask x 15]), draft, then
 * proposed[0] = current_token and proposed[1..15] = argmax of the tied LM head
 * over draft rows 1..15. Needs the draft context to cover the sequence. */
int hy_draft_propose(hy_ctx* ctx, int current_token, int* proposed);
/* decode_dflash_from_embeddings' block loop (src/text_runtime.cpp:1206-1296)
 * with the draft network, on the device: per block one CUDA-graph launch of
 * draft -> verify forward (M = 16) -> draft context of the block's rows ->
 * posterior, dflash_acceptance_length, commit of min(accept + 1, remaining)
 * tokens (cut at EOS) and rollback. first_token is not yet in the history.
 * tokens [n_tokens], acceptance_lengths [n_blocks] (nullable). */
int hy_dflash_generate(hy_ctx* ctx, int first_token, int max_tokens, float penalty, const int* eos_ids, int n_eos,
                       int* tokens, int* n_tokens, int* acceptance_lengths, int* n_blocks);
/* run_vlm_decode_with_prompt with the --dflash switch (src/hunyuan_ocr.cpp:166,
 * 357 -> decode_dflash_from_embeddings, src/text_runtime.cpp:1142-1305):
 * prompt embedding, prefill with the prompt's draft context, first token, then
 * hy_dflash_generate. */
int hy_run_vlm_dflash_with_prompt(hy_ctx* ctx, const int* input_ids, const int* position_ids, int seq_len,
                                  int image_token_id, const float* vision_features, int vision_token_count,
                                  int max_tokens, float repetition_penalty, const int* eos_ids, int n_eos, int* tokens,
                                  int* n_tokens, int* acceptance_lengths, int* n_blocks);

/* TextRuntime::run_vlm_decode_with_prompt (src/text_runtime.cpp:2053-2094):
 * prompt embedding with vision-feature injection (prepare_prompt_embeddings,
 * 506-568), mRoPE tables, prefill, first-token selection and the AR loop.
 * vision_features [vision_token_count x 1024]. */
int hy_run_vlm_decode_with_prompt(hy_ctx* ctx, const int* input_ids, const int* position_ids, int seq_len,
                                  int image_token_id, const float* vision_features, int vision_token_count,
                                  int max_tokens, float repetition_penalty, const int* eos_ids, int n_eos,
                                  int* tokens, int* raw_top1, int* n_tokens);

/* ---- batched decode (several requests on one GPU) --------------------- */
/* One prompt of a JSONL batch record (the arguments of run_vlm_decode_with_prompt). */
typedef struct hy_request {
    const int* input_ids;          /* [seq_len] */
    const int* position_ids;       /* [4 x seq_len], axis-major */
    int seq_len;
    int image_token_id;
    const float* vision_features;  /* [vision_token_count x 1024] */
    int vision_token_count;
} hy_request;

/* run_jsonl_batch's per-record decode (src/batch_jsonl.cpp:384-480: each record
 * through run_vlm_decode_with_prompt, one after the other) with up to `slots`
 * (1..16) records decoding together: each decode step advances every active
 * record by one AR greedy token (16-row projections stream the weights once for
 * all of them; attention, history, EOS and max_tokens are per record). A record
 * enters a slot when one frees up (its prompt is prefilled into the slot's own
 * KV cache). Each record's tokens equal hy_run_vlm_decode_with_prompt's for it.
 * tokens [n_requests x max_tokens] (record r's at r * max_tokens), n_tokens
 * [n_requests], status [n_requests] (nullable): a record whose prompt is
 * malformed or too long gets its error status and no tokens, the others go on
 * (run_jsonl_batch's error records). The context's own sequence is left empty. */
int hy_batch_decode(hy_ctx* ctx, const hy_request* requests, int n_requests, int slots, int max_tokens,
                    float repetition_penalty, const int* eos_ids, int n_eos, int* tokens, int* n_tokens, int* status);

/* ---- regression fixtures (host code, no device work) ------------------ */
/* parse_vlm_fixture_meta (src/text_runtime.cpp:285-321): `fixture_dir`/meta.txt
 * (key=value lines: seq_len, expected_token_count, image_token_id,
 * vision_token_count; all must be present and positive, image_token_id >= 0). */
int hy_fixture_meta(const char* fixture_dir, int* seq_len, int* expected_token_count, int* image_token_id,
                    int* vision_token_count);
/* load_vlm_fixture_with_features (src/text_runtime.cpp:334-381): input_ids.i32
 * [seq_len], position_ids.i32 [4 x seq_len], expected_tokens.i32
 * [expected_token_count] and vision_features.f32 [vision_token_count x 1024]
 * (skipped when vision_features is NULL), each exactly that size ("short read",
 * "unexpected extra bytes" otherwise). Sizes come from meta.txt, read again by
 * this call; the buffers hold seq_capacity ids (4 x seq_capacity position ids),
 * expected_capacity tokens and vision_capacity feature rows, and a meta.txt
 * asking for more fails with HY_ERR_CAPACITY before anything is written (the
 * reference reads into vectors it sizes itself). The fixture runs through
 * hy_run_vlm_decode_with_prompt / hy_run_vlm_dflash_with_prompt
 * (TextRuntime::run_vlm_fixture_decode / run_vlm_fixture_dflash_decode). */
int hy_fixture_load(const char* fixture_dir, int seq_capacity, int expected_capacity, int vision_capacity,
                    int* input_ids, int* position_ids, int* expected_tokens, float* vision_features);

/* ---- standalone kernels (benchmarks and parity tests) ----------------- */
/* Attention alone (PreciseSDPA decode/verify, src/precise_sdpa.cpp:281-329,
 * with the RoPE/QK-norm/append of export/text_decoder_kv.py:66-79): on layer
 * `layer` at the current length, rows (1..16) of raw projections
 * qkv [rows x 4096] (q 2048 | k 1024 | v 1024) are rotated with cos/sin
 * [rows x 128], QK-normed, appended, and attended; out [rows x 2048]. */
int hy_attention(hy_ctx* ctx, int layer, const float* qkv, int rows, const float* cos, const float* sin,
                 float* out);
/* Write/read KV rows [start, start+rows) of one layer; k, v [8 x rows x 128]. */
int hy_kv_write(hy_ctx* ctx, int layer, int start, int rows, const float* k, const float* v);
int hy_kv_read(hy_ctx* ctx, int layer, int start, int rows, float* k, float* v);
int hy_seq_set_length(hy_ctx* ctx, int rows);

/* Raw stream handle (cudaStream_t): the context's calls run on it; a caller
 * orders its own work before or after them with events on this stream. */
void* hy_ctx_stream(hy_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* HY_DECODE_H */
