"""GPU parity of the bf16 variant (bf16 weights and bf16 KV cache, fp32 activations
and accumulation), reported separately from the fp32 path.

Stated tolerance: against the oracle run with the same roundings (linears and
embedding rounded to bf16, cached K/V rows rounded to bf16, both round-to-nearest-
even), token ids, raw top-1 ids and DFlash acceptance are bit-exact and logits are
within 2e-4 absolute / 1e-4 relative, the fp32 path's tolerance (the products are
exact in fp32; only the reduction order differs). Against the fp32 path itself no
token-level agreement is promised: the weight rounding moves the logits by about
1e-2 relative, which can flip near-ties.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BF16 = 1
SMALL = dict(num_layers=2, vocab_size=4096, max_context=2304, max_prefill=256, max_tokens=256,
             weight_dtype=BF16, kv_dtype=BF16)
SEED, NORM_STD = 11, 0.1
ATOL, RTOL = 2e-4, 1e-4


@pytest.fixture(scope="module")
def bf16(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=4096, kv_bf16=True)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD, bf16=True)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, **SMALL)
    yield cfg, w, rt
    rt.close()


@pytest.mark.parametrize("rows", [1, 16])
def test_bf16_lm_head_matches_rounded_oracle(bf16, oracle, rows):
    cfg, w, rt = bf16
    rng = np.random.default_rng(100 + rows)
    h = rng.standard_normal((rows, 1024)).astype(np.float32)
    hist = rng.integers(0, cfg.vocab, 200).tolist()
    rt.set_history(hist)
    tok, raw, logits = rt.select_logit_rows(h, 1.08, want_logits=True)
    ref = oracle.lm_head(w, h)
    np.testing.assert_allclose(logits, ref, rtol=RTOL, atol=ATOL)
    want = oracle.select_logit_rows(ref, hist, None, 1.08)
    assert list(tok) == list(want)
    assert list(raw) == [int(np.argmax(ref[r])) for r in range(rows)]


@pytest.mark.parametrize("path", ["persistent", "graph"])
def test_bf16_ar_decode_matches_rounded_oracle(pkg, bf16, oracle, path):
    cfg, w, rt = bf16
    prompt = oracle.synthetic_prompt(44, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    want = oracle.decode_ar(w, cfg, prompt, 96)
    rt.ar_path = pkg.AR_PATH_PERSISTENT if path == "persistent" else pkg.AR_PATH_GRAPH
    try:
        res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                            prompt.vision_features, max_tokens=96)
    finally:
        rt.ar_path = pkg.AR_PATH_PERSISTENT
    assert res.generated_tokens == want.tokens
    assert res.raw_top1_tokens == want.raw_top1


def test_bf16_dflash_is_lossless(bf16, oracle):
    cfg, w, rt = bf16
    prompt = oracle.synthetic_prompt(45, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    ar = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                       prompt.vision_features, max_tokens=80)
    first = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                          prompt.vision_features, max_tokens=1).generated_tokens[0]
    out = rt.dflash_generate_synthetic(first, 64, 1.08, ar.generated_tokens, 0.7, seed=5)
    assert out.generated_tokens == ar.generated_tokens[:len(out.generated_tokens)]
    assert len(out.generated_tokens) == 64


def test_bf16_batched_decode_matches_rounded_oracle(bf16, oracle):
    """hy_batch_decode on the bf16 variant: every record's tokens equal the rounded
    oracle's AR decode of that record alone."""
    cfg, w, rt = bf16
    prompts = [oracle.synthetic_prompt(300 + i, 2 + i % 3, 4, 10 + 7 * i, cfg.vocab, cfg.vocab - 3) for i in range(5)]
    toks, status = rt.batch_decode([(p.input_ids, p.position_ids, p.image_token_id, p.vision_features)
                                    for p in prompts], 24, slots=4)
    assert status == [0] * len(prompts)
    for p, got in zip(prompts, toks):
        assert got == oracle.decode_ar(w, cfg, p, 24).tokens


def test_bf16_draft_run_matches_rounded_oracle(pkg, oracle):
    """The DFlash draft network with bf16 draft weights and bf16 draft K/V against the
    oracle with the same roundings (weights rounded at load; the oracle's draft cache
    rounds its K/V rows to bf16 as the device cache stores them)."""
    dw = oracle.make_draft_weights(2, 19, 0.02, NORM_STD, bf16=True)
    rng = np.random.default_rng(9)
    aux = rng.standard_normal((4, 40, 1024)).astype(np.float32)
    noise = rng.standard_normal((16, 1024)).astype(np.float32)
    with pkg.TextRuntime.synthetic(seed=1, device=0, **dict(SMALL, max_context=256)) as rt:
        rt.load_draft_synthetic(2, 19, 0.02, NORM_STD, 4095)
        rt.draft_context_append(aux)
        got = rt.draft_run(noise)
    cache = oracle.DraftCache.empty(2, 56)
    oracle.draft_append_context(dw, cache, list(aux))
    for li in range(2):
        cache.k[li] = oracle.round_bf16(cache.k[li])
        cache.v[li] = oracle.round_bf16(cache.v[li])
    want = oracle.draft_forward(dw, noise, cache, kv_round=True)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
