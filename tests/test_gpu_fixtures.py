"""Regression fixtures through the GPU path: TextRuntime::run_vlm_fixture_decode and
run_vlm_fixture_dflash_decode (src/text_runtime.cpp:1793-1920) on a fixture directory
in the reference's format whose expected tokens come from the oracle."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096


@pytest.fixture(scope="module")
def setup(pkg, oracle, tmp_path_factory):
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, 11, 0.02, 0.1)
    prompt = oracle.synthetic_prompt(77, 4, 6, 20, VOCAB, VOCAB - 3)
    want = oracle.decode_ar(w, cfg, prompt, 40).tokens
    d = str(tmp_path_factory.mktemp("fx") / "case0")
    pkg.write_vlm_fixture(d, prompt.input_ids, prompt.position_ids, prompt.image_token_id, prompt.vision_features,
                          want)
    rt = pkg.TextRuntime.synthetic(seed=11, std=0.02, norm_std=0.1, num_layers=2, vocab_size=VOCAB,
                                   max_context=512, max_prefill=256, max_tokens=128, device=0)
    yield d, want, rt
    rt.close()


def test_fixture_decode_matches_expected(setup):
    d, want, rt = setup
    res = rt.run_vlm_fixture_decode(d)            # max_tokens <= 0: all expected tokens
    assert res.checked_tokens == len(want) and res.matches_expected()
    res = rt.run_vlm_fixture_decode(d, max_tokens=10)
    assert res.generated_tokens == want[:10] and res.matches_expected()


def test_fixture_mismatch_is_reported(pkg, setup, tmp_path):
    d, want, rt = setup
    fx = pkg.read_vlm_fixture(d)
    bad = list(want)
    bad[5] = (bad[5] + 1) % VOCAB
    d2 = str(tmp_path / "bad")
    pkg.write_vlm_fixture(d2, fx.input_ids, fx.position_ids, fx.image_token_id, fx.vision_features, bad)
    res = rt.run_vlm_fixture_decode(d2)
    assert res.generated_tokens == want and not res.matches_expected()


def test_fixture_dflash_decode_is_lossless(setup):
    d, want, rt = setup
    rt.load_draft_synthetic(1, seed=5, std=0.02, mask_token=VOCAB - 1)
    res = rt.run_vlm_fixture_dflash_decode(d)
    assert res.matches_expected()
    assert sum(a + 1 for a in res.acceptance_lengths) == len(want)
