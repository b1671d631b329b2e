"""Failure detection on the GPU without a GPU fault: every device wait of the
library is bounded by a wall-clock limit, after which the kernel sets the
context's error word and returns. A self-test kernel waits, with the library's
own primitives, for an epoch word that is never published and for an mbarrier
phase that never completes; the call must return HY_ERR_DEVICE_TIMEOUT after
about the limit, and the same context must then decode the oracle's tokens."""

import time

import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096


def test_bounded_waits_time_out_and_context_recovers(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, 11, 0.02, 0.1)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    want = oracle.decode_ar(w, cfg, prompt, 40)
    with pkg.TextRuntime.synthetic(seed=11, std=0.02, norm_std=0.1, num_layers=2, vocab_size=VOCAB,
                                   max_context=512, max_prefill=64, max_tokens=64, device=0) as rt:
        for kind in (0, 1):
            t0 = time.perf_counter()
            with pytest.raises(pkg.HyError) as e:
                rt.wait_probe(kind, 1_000_000)   # 1 ms
            assert e.value.status == pkg.HY_ERR_DEVICE_TIMEOUT, e.value.message
            assert "timed out" in e.value.message
            assert time.perf_counter() - t0 < 1.0
        # The error word was cleared: the context decodes the oracle's tokens.
        res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                            prompt.vision_features, max_tokens=40)
        assert res.generated_tokens == want.tokens
        with pytest.raises(pkg.HyError) as e:
            rt.wait_probe(2, 1_000_000)
        assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
        with pytest.raises(pkg.HyError):
            rt.set_wait_limit(10)   # below 1 ms
        rt.set_wait_limit(2_000_000_000)
