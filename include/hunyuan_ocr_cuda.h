// hunyuan_ocr_cuda.h - C++17 drop-in for the text-decode half of HunyuanOCR-ncnn's
// C++ API, over the C ABI of libhy_decode.so (include/hy_decode.h).
//
// It mirrors, by name and meaning:
//   - hunyuan_ocr::TextRuntime (include/hunyuan_ocr/text_runtime.h:85-158): load,
//     load_dflash, ready, dflash_ready, mapped_weight_bytes,
//     run_vlm_decode_with_prompt, run_vlm_dflash_decode_with_prompt,
//     run_vlm_fixture_decode, run_vlm_fixture_dflash_decode; each returns bool and
//     fills std::string* error, as the reference's do;
//   - TextDecodeTiming / TextDecodeResult / DFlashDecodeTiming / DFlashDecodeResult
//     (text_runtime.h:32-83) and DecoderStatistics (include/hunyuan_ocr/hunyuan_ocr.h:55-65);
//   - RuntimeOptions (hunyuan_ocr.h:22-31) with the CUDA backend's own switch
//     (text_cuda, text_cuda_device) beside the untouched Vulkan fields;
//   - RuntimeError {stage, message} with the reference's stage names;
//   - detail::run_decoder_step (src/text_decoder_step.h:29-38), with the device
//     context standing in for the ncnn::Net and its caches.
// The vision encoder, tokenizer and prompt builder are not part of this path.
#pragma once

#include "hy_decode.h"

#include <array>
#include <cstdint>
#include <fstream>
#include <functional>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

namespace hunyuan_ocr {
namespace cuda {

struct RuntimeOptions {
    int num_threads = 0;          // host threads (the CUDA path's host work is small; unused)
    bool vision_vulkan = false;
    int vision_vulkan_device = 0;
    bool dflash = false;          // the --dflash switch (src/cli_options.cpp:173)
    float repetition_penalty = 1.08f;
    bool mmap_weights = false;    // the package is always mapped while it is uploaded
    bool text_vulkan = false;
    int text_vulkan_device = 0;
    bool text_cuda = true;        // the CUDA text decoder (this library)
    int text_cuda_device = 0;
    int max_context = 8192 + 64;  // KV rows reserved (prompt + generated + one block)
    int max_prefill = 2048;
    int max_tokens = 1024;
    bool bf16_weights = false;    // the bf16-weight variant (fp32 for reference parity)
};

struct RuntimeError {
    std::string stage;
    std::string message;
};

// The reference's option check (src/hunyuan_ocr.cpp:307-310 keeps text_vulkan and
// dflash apart); the CUDA backend supports DFlash, so only the backend pair conflicts.
inline bool validate_options(const RuntimeOptions& o, RuntimeError* error)
{
    if (o.text_cuda && o.text_vulkan)
    {
        if (error) *error = {"runtime_options", "text_cuda and text_vulkan select different text backends"};
        return false;
    }
    if (!(o.repetition_penalty > 0.f))
    {
        if (error) *error = {"runtime_options", "repetition_penalty must be positive"};
        return false;
    }
    return true;
}

struct TextDecodeTiming {
    double text_embed_ms = 0.0;
    double prefill_ms = 0.0;
    double decode_ms = 0.0;
    double lm_head_ms = 0.0;
    double token_select_ms = 0.0;
    double total_ms = 0.0;
};

struct TextDecodeResult {
    int seq_len = 0;
    int checked_tokens = 0;
    float repetition_penalty = 1.08f;
    TextDecodeTiming timing;
    std::vector<int> generated_tokens;
    std::vector<int> raw_top1_tokens;
    std::vector<int> expected_tokens;
    bool matches_expected() const { return generated_tokens == expected_tokens; }
};

struct DFlashDecodeTiming {
    double prefill_ms = 0.0;
    double draft_prepare_ms = 0.0;
    double draft_infer_ms = 0.0;
    double draft_postprocess_ms = 0.0;
    double verify_prepare_ms = 0.0;
    double verify_infer_ms = 0.0;
    double verify_postprocess_ms = 0.0;
    double commit_ms = 0.0;
    double total_ms = 0.0;
};

struct DFlashDecodeResult {
    TextDecodeResult decode;
    int block_count = 0;
    int drafted_token_count = 0;
    int accepted_draft_token_count = 0;
    std::vector<int> acceptance_lengths;
    DFlashDecodeTiming timing;
};

enum class DecoderMode { Autoregressive, DFlash };

struct DecoderStatistics {
    DecoderMode mode = DecoderMode::Autoregressive;
    int block_count = 0;
    int drafted_token_count = 0;
    int accepted_draft_token_count = 0;
};

using TextTokenCallback = std::function<void(int)>;

class TextRuntime {
public:
    explicit TextRuntime(const RuntimeOptions& options = RuntimeOptions()) : options_(options) {}
    ~TextRuntime() { release(); }
    TextRuntime(TextRuntime&& o) noexcept : options_(o.options_), ctx_(o.ctx_), eos_ids_(std::move(o.eos_ids_)),
                                            dflash_(o.dflash_)
    {
        o.ctx_ = nullptr;
    }
    TextRuntime& operator=(TextRuntime&& o) noexcept
    {
        if (this != &o)
        {
            release();
            options_ = o.options_;
            ctx_ = o.ctx_;
            eos_ids_ = std::move(o.eos_ids_);
            dflash_ = o.dflash_;
            o.ctx_ = nullptr;
        }
        return *this;
    }
    TextRuntime(const TextRuntime&) = delete;
    TextRuntime& operator=(const TextRuntime&) = delete;

    // TextRuntime::load: the package's text_embed and text_decoder networks, and the
    // EOS ids of tokenizer/eos_ids.json when the package has one.
    bool load(const std::string& model_root, std::string* error)
    {
        release();
        RuntimeError re;
        if (!validate_options(options_, &re)) return set(error, re.message);
        hy_config cfg = config();
        if (hy_ctx_create_from_package(&cfg, model_root.c_str(), &ctx_) != HY_OK) return fail(error);
        eos_ids_ = read_eos_ids(model_root + "/tokenizer/eos_ids.json");
        return true;
    }
    // Seeded synthetic weights (benchmarks and tests without a checkpoint).
    bool load_synthetic(uint64_t seed, int num_layers, int vocab_size, std::string* error, float std_dev = 0.02f,
                        float norm_std = 0.0f)
    {
        release();
        hy_config cfg = config();
        cfg.num_layers = num_layers;
        cfg.vocab_size = vocab_size;
        if (hy_ctx_create_synthetic(&cfg, seed, std_dev, norm_std, &ctx_) != HY_OK) return fail(error);
        return true;
    }
    bool load_dflash(const std::string& model_root, std::string* error, int mask_token = HY_DFLASH_MASK_TOKEN)
    {
        if (!ctx_) return set(error, "text runtime is not loaded");
        if (hy_draft_load_package(ctx_, model_root.c_str(), mask_token) != HY_OK) return fail(error);
        dflash_ = true;
        return true;
    }
    bool load_dflash_synthetic(int num_layers, int mask_token, uint64_t seed, std::string* error)
    {
        if (!ctx_) return set(error, "text runtime is not loaded");
        if (hy_draft_load_synthetic(ctx_, num_layers, mask_token, seed, 0.02f, 0.0f) != HY_OK) return fail(error);
        dflash_ = true;
        return true;
    }
    bool ready() const { return ctx_ != nullptr; }
    bool dflash_ready() const { return ctx_ != nullptr && dflash_; }
    size_t mapped_weight_bytes() const { return ctx_ ? hy_ctx_device_bytes(ctx_) : 0; }
    void set_eos_ids(std::vector<int> ids) { eos_ids_ = std::move(ids); }
    const std::vector<int>& eos_ids() const { return eos_ids_; }
    hy_ctx* context() const { return ctx_; }

    bool run_vlm_decode_with_prompt(const std::vector<int>& input_ids, const std::vector<int>& position_ids,
                                    int image_token_id, const std::vector<float>& vision_features,
                                    int vision_token_count, const std::vector<int>& expected_tokens, int max_tokens,
                                    float repetition_penalty, TextDecodeResult* result, std::string* error,
                                    const TextTokenCallback& token_callback = {}) const
    {
        if (!check_prompt(input_ids, position_ids, vision_features, vision_token_count, result, error)) return false;
        max_tokens = checked_max(max_tokens, expected_tokens);
        std::vector<int> tokens(static_cast<size_t>(max_tokens)), raw(static_cast<size_t>(max_tokens));
        int n = 0;
        CallbackScope cb(ctx_, token_callback);
        if (hy_run_vlm_decode_with_prompt(ctx_, input_ids.data(), position_ids.data(),
                                          static_cast<int>(input_ids.size()), image_token_id, vision_features.data(),
                                          vision_token_count, max_tokens, repetition_penalty, eos_ptr(), eos_count(),
                                          tokens.data(), raw.data(), &n) != HY_OK)
            return fail(error);
        TextDecodeResult r;
        r.seq_len = static_cast<int>(input_ids.size());
        r.repetition_penalty = repetition_penalty;
        r.generated_tokens.assign(tokens.begin(), tokens.begin() + n);
        r.raw_top1_tokens.assign(raw.begin(), raw.begin() + n);
        fill_expected(expected_tokens, max_tokens, &r);
        hy_decode_timing t{};
        hy_ctx_last_timing(ctx_, &t);
        r.timing = {t.text_embed_ms, t.prefill_ms, t.decode_ms, t.lm_head_ms, t.token_select_ms, t.total_ms};
        *result = std::move(r);
        return true;
    }

    bool run_vlm_dflash_decode_with_prompt(const std::vector<int>& input_ids, const std::vector<int>& position_ids,
                                           int image_token_id, const std::vector<float>& vision_features,
                                           int vision_token_count, const std::vector<int>& expected_tokens,
                                           int max_tokens, float repetition_penalty, DFlashDecodeResult* result,
                                           std::string* error, const TextTokenCallback& token_callback = {}) const
    {
        if (!dflash_ready()) return set(error, "DFlash draft runtime is not loaded");
        if (!check_prompt(input_ids, position_ids, vision_features, vision_token_count, result, error)) return false;
        max_tokens = checked_max(max_tokens, expected_tokens);
        std::vector<int> tokens(static_cast<size_t>(max_tokens)), acc(static_cast<size_t>(max_tokens) + HY_DFLASH_BLOCK);
        int n = 0, blocks = 0;
        CallbackScope cb(ctx_, token_callback);
        if (hy_run_vlm_dflash_with_prompt(ctx_, input_ids.data(), position_ids.data(),
                                          static_cast<int>(input_ids.size()), image_token_id, vision_features.data(),
                                          vision_token_count, max_tokens, repetition_penalty, eos_ptr(), eos_count(),
                                          tokens.data(), &n, acc.data(), &blocks) != HY_OK)
            return fail(error);
        DFlashDecodeResult r;
        r.decode.seq_len = static_cast<int>(input_ids.size());
        r.decode.repetition_penalty = repetition_penalty;
        r.decode.generated_tokens.assign(tokens.begin(), tokens.begin() + n);
        fill_expected(expected_tokens, max_tokens, &r.decode);
        r.acceptance_lengths.assign(acc.begin(), acc.begin() + blocks);
        hy_dflash_timing t{};
        hy_ctx_last_dflash_timing(ctx_, &t);
        r.block_count = t.block_count;
        r.drafted_token_count = t.drafted_token_count;
        r.accepted_draft_token_count = t.accepted_draft_token_count;
        // One graph per block on the device: draft (prepare + infer + postprocess),
        // verify (prepare + infer) and commit (postprocess + commit) stages.
        r.timing.prefill_ms = t.prefill_ms;
        r.timing.draft_infer_ms = t.draft_ms;
        r.timing.verify_infer_ms = t.verify_ms;
        r.timing.commit_ms = t.commit_ms;
        r.timing.total_ms = t.total_ms;
        *result = std::move(r);
        return true;
    }

    // run_vlm_fixture_decode (src/text_runtime.cpp:1793-1837): the fixture's prompt and
    // features, penalty 1.08, max_tokens <= 0 meaning every expected token.
    bool run_vlm_fixture_decode(const std::string& fixture_dir, int max_tokens, TextDecodeResult* result,
                                std::string* error) const
    {
        Fixture f;
        if (!read_fixture(fixture_dir, &f, error)) return false;
        return run_vlm_decode_with_prompt(f.ids, f.pos, f.image_token_id, f.features, f.vision_tokens, f.expected,
                                          max_tokens, 1.08f, result, error);
    }
    bool run_vlm_fixture_dflash_decode(const std::string& fixture_dir, int max_tokens, DFlashDecodeResult* result,
                                       std::string* error) const
    {
        Fixture f;
        if (!read_fixture(fixture_dir, &f, error)) return false;
        return run_vlm_dflash_decode_with_prompt(f.ids, f.pos, f.image_token_id, f.features, f.vision_tokens,
                                                 f.expected, max_tokens, 1.08f, result, error);
    }

    static DecoderStatistics statistics(const DFlashDecodeResult& r)
    {
        return {DecoderMode::DFlash, r.block_count, r.drafted_token_count, r.accepted_draft_token_count};
    }

private:
    struct Fixture {
        std::vector<int> ids, pos, expected;
        std::vector<float> features;
        int image_token_id = 0, vision_tokens = 0;
    };
    // The reference calls the stream callback synchronously per committed token; here it
    // is registered for the duration of one call.
    class CallbackScope {
    public:
        CallbackScope(hy_ctx* c, const TextTokenCallback& fn) : c_(fn ? c : nullptr), fn_(&fn)
        {
            if (c_) hy_ctx_set_token_callback(c_, &CallbackScope::trampoline, this, 0);
        }
        ~CallbackScope()
        {
            if (c_) hy_ctx_set_token_callback(c_, nullptr, nullptr, 0);
        }

    private:
        static void trampoline(int token, void* self) { (*static_cast<CallbackScope*>(self)->fn_)(token); }
        hy_ctx* c_;
        const TextTokenCallback* fn_;
    };

    hy_config config() const
    {
        hy_config cfg;
        hy_config_init(&cfg);
        cfg.device = options_.text_cuda_device;
        cfg.max_context = options_.max_context;
        cfg.max_prefill = options_.max_prefill;
        cfg.max_tokens = options_.max_tokens;
        cfg.weight_dtype = options_.bf16_weights ? HY_DTYPE_BF16 : HY_DTYPE_F32;
        cfg.kv_dtype = cfg.weight_dtype;
        return cfg;
    }
    void release()
    {
        if (ctx_) hy_ctx_destroy(ctx_);
        ctx_ = nullptr;
        dflash_ = false;
    }
    template <typename R>
    bool check_prompt(const std::vector<int>& ids, const std::vector<int>& pos, const std::vector<float>& features,
                      int vision_tokens, R* result, std::string* error) const
    {
        if (!ctx_) return set(error, "text runtime is not loaded");
        if (!result) return set(error, "result is null");
        if (pos.size() != 4 * ids.size()) return set(error, "position_ids must hold 4 x seq_len values");
        if (vision_tokens < 0 || features.size() != static_cast<size_t>(vision_tokens) * HY_HIDDEN)
            return set(error, "vision feature size mismatch");
        return true;
    }
    // decode_from_embeddings (src/text_runtime.cpp:1336-1350): with expected tokens,
    // max_tokens <= 0 or past their count means all of them; otherwise <= 0 means 1024.
    static int checked_max(int max_tokens, const std::vector<int>& expected)
    {
        const int n = static_cast<int>(expected.size());
        if (n > 0) return (max_tokens <= 0 || max_tokens > n) ? n : max_tokens;
        return max_tokens <= 0 ? 1024 : max_tokens;
    }
    static void fill_expected(const std::vector<int>& expected, int max_tokens, TextDecodeResult* r)
    {
        if (expected.empty()) return;
        r->checked_tokens = max_tokens;
        r->expected_tokens.assign(expected.begin(), expected.begin() + max_tokens);
    }
    const int* eos_ptr() const { return eos_ids_.empty() ? nullptr : eos_ids_.data(); }
    int eos_count() const { return static_cast<int>(eos_ids_.size()); }
    static bool set(std::string* error, const std::string& msg)
    {
        if (error) *error = msg;
        return false;
    }
    static bool fail(std::string* error) { return set(error, hy_last_error()); }
    static std::vector<int> read_eos_ids(const std::string& path)
    {
        // tokenizer/eos_ids.json: a JSON array of integers (or an object holding one).
        std::ifstream f(path);
        std::vector<int> ids;
        if (!f) return ids;
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string s = ss.str();
        for (size_t i = 0; i < s.size();)
        {
            if (s[i] >= '0' && s[i] <= '9')
            {
                int v = 0;
                while (i < s.size() && s[i] >= '0' && s[i] <= '9') v = v * 10 + (s[i++] - '0');
                ids.push_back(v);
            }
            else
                ++i;
        }
        return ids;
    }
    static bool read_fixture(const std::string& dir, Fixture* f, std::string* error)
    {
        int seq = 0, expected = 0;
        if (hy_fixture_meta(dir.c_str(), &seq, &expected, &f->image_token_id, &f->vision_tokens) != HY_OK)
            return fail(error);
        f->ids.resize(static_cast<size_t>(seq));
        f->pos.resize(static_cast<size_t>(seq) * 4);
        f->expected.resize(static_cast<size_t>(expected));
        f->features.resize(static_cast<size_t>(f->vision_tokens) * HY_HIDDEN);
        if (hy_fixture_load(dir.c_str(), seq, expected, f->vision_tokens, f->ids.data(), f->pos.data(),
                            f->expected.data(), f->features.data()) != HY_OK)
            return fail(error);
        return true;
    }

    RuntimeOptions options_;
    hy_ctx* ctx_ = nullptr;
    std::vector<int> eos_ids_;
    bool dflash_ = false;
};

namespace detail {

// run_decoder_step (src/text_decoder_step.h:29-38): `rows` new embeddings
// [rows x 1024] at the context's current length, cos / sin [rows x 128]; the rows
// are appended to the context's KV cache (the reference returns updated caches).
// hidden [rows x 1024] final-normed; target_hidden (nullable) the outputs of
// layers 1, 8, 15, 22 for the DFlash draft.
inline bool run_decoder_step(const TextRuntime& rt, const std::vector<float>& current_embed,
                             const std::vector<float>& cos, const std::vector<float>& sin,
                             std::vector<float>* hidden, std::array<std::vector<float>, 4>* target_hidden,
                             std::string* error)
{
    if (!rt.ready())
    {
        if (error) *error = "text runtime is not loaded";
        return false;
    }
    const int rows = static_cast<int>(current_embed.size() / HY_HIDDEN);
    if (rows < 1 || current_embed.size() != static_cast<size_t>(rows) * HY_HIDDEN ||
        cos.size() != static_cast<size_t>(rows) * HY_HEAD_DIM || sin.size() != cos.size())
    {
        if (error) *error = "decoder step inputs must be [rows x 1024] embeddings and [rows x 128] cos / sin";
        return false;
    }
    hidden->resize(current_embed.size());
    std::vector<float> aux(target_hidden ? static_cast<size_t>(HY_NUM_AUX_LAYERS) * current_embed.size() : 0);
    if (hy_decoder_step(rt.context(), current_embed.data(), rows, cos.data(), sin.data(), hidden->data(),
                        target_hidden ? aux.data() : nullptr) != HY_OK)
    {
        if (error) *error = hy_last_error();
        return false;
    }
    if (target_hidden)
        for (int i = 0; i < HY_NUM_AUX_LAYERS; ++i)
            (*target_hidden)[i].assign(aux.begin() + static_cast<long>(i) * current_embed.size(),
                                       aux.begin() + static_cast<long>(i + 1) * current_embed.size());
    return true;
}

}  // namespace detail
}  // namespace cuda
}  // namespace hunyuan_ocr
