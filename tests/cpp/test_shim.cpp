// Test program of the C++17 layer (include/hunyuan_ocr_cuda.h) over libhy_decode.so,
// run by tests/test_cpp_shim.py. Modes:
//   host                      checks that need no GPU: option validation with the
//                             reference's stage name, load errors, calls on an
//                             unloaded runtime, a known answer of the mRoPE builder
//                             (tests/text_rope_test.cpp:8-34 of the reference)
//   decode <package> <fixture> [dflash <mask>]
//                             loads a model package, decodes the fixture's prompt
//                             (AR with the stream callback, then DFlash when asked)
//                             and prints the tokens and the DFlash statistics
#include "hunyuan_ocr_cuda.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace hc = hunyuan_ocr::cuda;

static int check(bool ok, const char* what)
{
    if (!ok) std::printf("FAIL %s\n", what);
    return ok ? 0 : 1;
}

static int host_checks()
{
    int bad = 0;
    hc::RuntimeOptions o;
    o.text_vulkan = true;
    hc::RuntimeError re;
    bad += check(!hc::validate_options(o, &re) && re.stage == "runtime_options", "text_cuda + text_vulkan rejected");
    o.text_vulkan = false;
    o.dflash = true;
    bad += check(hc::validate_options(o, &re), "dflash accepted on the CUDA backend");
    o.repetition_penalty = 0.f;
    bad += check(!hc::validate_options(o, &re) && re.message == "repetition_penalty must be positive",
                 "non-positive penalty rejected");

    hc::TextRuntime rt;
    std::string err;
    bad += check(!rt.load("/nonexistent/model", &err) && err.find("failed to open model file") != std::string::npos,
                 "missing package reported");
    bad += check(!rt.ready() && !rt.dflash_ready() && rt.mapped_weight_bytes() == 0, "unloaded runtime");
    hc::TextDecodeResult res;
    err.clear();
    bad += check(!rt.run_vlm_decode_with_prompt({1, 2}, std::vector<int>(8, 0), 3, {}, 0, {}, 4, 1.08f, &res, &err) &&
                     err == "text runtime is not loaded",
                 "decode on an unloaded runtime");
    std::vector<float> hidden;
    bad += check(!hc::detail::run_decoder_step(rt, std::vector<float>(1024), std::vector<float>(128),
                                               std::vector<float>(128), &hidden, nullptr, &err),
                 "step on an unloaded runtime");

    // build_mrope known answer (position ids 978, 811, 621, 431).
    const int pos[4] = {978, 811, 621, 431};
    float cos[128];
    bad += check(hy_build_mrope(pos, 1, 1, cos) == HY_OK, "build_mrope");
    bad += check(std::fabs(cos[0] - (-0.569676042f)) <= 2e-7f && std::fabs(cos[64] - 0.510228872f) <= 2e-7f,
                 "mrope cos values");
    if (!bad) std::printf("host ok\n");
    return bad;
}

static bool load_fixture(const std::string& dir, std::vector<int>* ids, std::vector<int>* pos, std::vector<float>* feats,
                         int* image, int* vision)
{
    int seq = 0, expected = 0;
    if (hy_fixture_meta(dir.c_str(), &seq, &expected, image, vision) != HY_OK) return false;
    ids->resize(seq);
    pos->resize(4 * seq);
    feats->resize(static_cast<size_t>(*vision) * 1024);
    std::vector<int> exp(expected);
    return hy_fixture_load(dir.c_str(), seq, expected, *vision, ids->data(), pos->data(), exp.data(), feats->data()) ==
           HY_OK;
}

static void print_tokens(const char* tag, const std::vector<int>& t)
{
    std::printf("%s", tag);
    for (int v : t) std::printf(" %d", v);
    std::printf("\n");
}

static int decode(const std::string& pkg, const std::string& fixture, bool dflash, int mask)
{
    hc::RuntimeOptions o;
    o.max_context = 512;
    o.max_prefill = 256;
    o.max_tokens = 64;
    hc::TextRuntime rt(o);
    std::string err;
    if (!rt.load(pkg, &err)) return std::printf("FAIL load: %s\n", err.c_str()), 1;
    std::vector<int> ids, pos;
    std::vector<float> feats;
    int image = 0, vision = 0;
    if (!load_fixture(fixture, &ids, &pos, &feats, &image, &vision)) return std::printf("FAIL fixture: %s\n", hy_last_error()), 1;
    hc::TextDecodeResult r;
    std::vector<int> streamed;
    if (!rt.run_vlm_decode_with_prompt(ids, pos, image, feats, vision, {}, 24, 1.08f, &r, &err,
                                       [&](int t) { streamed.push_back(t); }))
        return std::printf("FAIL decode: %s\n", err.c_str()), 1;
    print_tokens("ar", r.generated_tokens);
    if (streamed != r.generated_tokens) return std::printf("FAIL streamed tokens differ\n"), 1;
    if (!(r.timing.prefill_ms > 0 && r.timing.decode_ms > 0 && r.timing.total_ms >= r.timing.decode_ms))
        return std::printf("FAIL timing\n"), 1;
    if (dflash)
    {
        if (!rt.load_dflash(pkg, &err, mask)) return std::printf("FAIL load_dflash: %s\n", err.c_str()), 1;
        hc::DFlashDecodeResult d;
        if (!rt.run_vlm_dflash_decode_with_prompt(ids, pos, image, feats, vision, {}, 24, 1.08f, &d, &err))
            return std::printf("FAIL dflash: %s\n", err.c_str()), 1;
        print_tokens("dflash", d.decode.generated_tokens);
        const hc::DecoderStatistics s = hc::TextRuntime::statistics(d);
        std::printf("blocks %d drafted %d accepted %d\n", s.block_count, s.drafted_token_count,
                    s.accepted_draft_token_count);
    }
    return 0;
}

int main(int argc, char** argv)
{
    const std::string mode = argc > 1 ? argv[1] : "host";
    if (mode == "host") return host_checks();
    if (mode == "decode" && argc >= 4)
        return decode(argv[2], argv[3], argc >= 5, argc >= 6 ? std::atoi(argv[5]) : HY_DFLASH_MASK_TOKEN);
    std::printf("usage: test_shim host | decode <package> <fixture> [dflash <mask>]\n");
    return 2;
}
