"""Streaming callback (InferenceRequest::stream_callback / TextTokenCallback,
include/hunyuan_ocr/hunyuan_ocr.h:43-45, text_runtime.h:21): every committed token
reaches the callback once, in order, on the AR paths and in DFlash."""

import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096


@pytest.fixture(scope="module")
def small(pkg, oracle):
    rt = pkg.TextRuntime.synthetic(seed=11, std=0.02, norm_std=0.1, num_layers=2, vocab_size=VOCAB,
                                   max_context=1024, max_prefill=256, max_tokens=256, device=0)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    yield rt, prompt
    rt.close()


@pytest.mark.parametrize("path,sync", [("persistent", 0), ("persistent", 5), ("graph", 0)])
def test_callback_sees_every_ar_token(pkg, small, path, sync):
    rt, p = small
    want = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                         max_tokens=70).generated_tokens
    got = []
    rt.ar_path = pkg.AR_PATH_PERSISTENT if path == "persistent" else pkg.AR_PATH_GRAPH
    rt.set_token_callback(got.append, tokens_per_sync=sync)
    try:
        res = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                            max_tokens=70)
    finally:
        rt.set_token_callback(None)
        rt.ar_path = pkg.AR_PATH_PERSISTENT
    assert res.generated_tokens == want
    assert got == want


def test_callback_in_dflash_and_removal(pkg, small):
    rt, p = small
    greedy = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                           max_tokens=60).generated_tokens
    got = []
    rt.set_token_callback(got.append)
    first = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                          max_tokens=1).generated_tokens[0]
    assert got == [first]
    got.clear()
    out = rt.dflash_generate_synthetic(first, 40, 1.08, greedy, 0.7, seed=3)
    assert out.generated_tokens == greedy[:40] and got == out.generated_tokens
    rt.set_token_callback(None)
    got.clear()
    rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features, max_tokens=5)
    assert got == []
    with pytest.raises(pkg.HyError):
        rt.set_token_callback(got.append, tokens_per_sync=65)
