"""Prompt prefill (run_decoder_prefill, src/text_runtime.cpp:648-674) through the
many-row tensor-core GEMMs, against the oracle: the final-normed last hidden row
and the K/V rows the prefill appends, for prompts that end inside a 128-row tile
and for one that takes two prefill passes (1024 rows, then the rest).

Tolerance: fp32 activations within 2e-4 absolute / 1e-4 relative, cached K/V
(values after the QK RMSNorm, so of order 1) within 1e-4; the GEMMs compute in
tf32 with a three-term split and fp32 accumulation, the oracle in fp32 BLAS.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED, NORM_STD = 11, 0.1
ATOL, RTOL = 2e-4, 1e-4
KV_TOL = 1e-4


@pytest.fixture(scope="module")
def long_rt(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=4096)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, num_layers=2,
                                   vocab_size=4096, max_context=2304, max_prefill=2048, max_tokens=64)
    yield cfg, w, rt
    rt.close()


@pytest.mark.parametrize("grid,n_text", [((4, 6), 113), ((16, 16), 1), ((24, 32), 340)])
def test_prefill_matches_oracle(long_rt, oracle, grid, n_text):
    cfg, w, rt = long_rt
    prompt = oracle.synthetic_prompt(5, grid[0], grid[1], n_text, cfg.vocab, cfg.vocab - 3)
    seq = prompt.input_ids.shape[0]   # 137, 257, 1108 rows
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    cos = oracle.build_mrope(prompt.position_ids, seq, True)
    sin = oracle.build_mrope(prompt.position_ids, seq, False)
    rt.reset()
    last = rt.prefill(emb, cos, sin)
    hidden, cache, _ = oracle.prefill(w, cfg, prompt, seq)
    np.testing.assert_allclose(last, hidden[-1], rtol=RTOL, atol=ATOL)
    assert rt.kv_length == seq
    starts = {0, 120, seq - 16}
    if seq > 1040:
        starts |= {1016, 1024}   # across the boundary of the two passes
    for layer in range(cfg.num_layers):
        for s in sorted(starts):
            k, v = rt.kv_read(layer, s, 16)
            np.testing.assert_allclose(k, cache.k[layer][:, s:s + 16], rtol=KV_TOL, atol=KV_TOL)
            np.testing.assert_allclose(v, cache.v[layer][:, s:s + 16], rtol=KV_TOL, atol=KV_TOL)


def test_prefill_then_decode_matches_oracle(pkg, long_rt, oracle):
    """A two-pass prompt, then greedy tokens through the reference-facing call."""
    cfg, w, rt = long_rt
    prompt = oracle.synthetic_prompt(8, 24, 32, 300, cfg.vocab, cfg.vocab - 3)
    want = oracle.decode_ar(w, cfg, prompt, 24)
    res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=24)
    assert res.generated_tokens == want.tokens
    assert res.raw_top1_tokens == want.raw_top1
