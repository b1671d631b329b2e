"""Per-stage timing and decode statistics of the result types: TextDecodeTiming
(include/hunyuan_ocr/text_runtime.h:32-39), DFlashDecodeTiming (64-74), the
drafted / accepted counts of DFlashDecodeResult (76-83) and DecoderStatistics
(include/hunyuan_ocr/hunyuan_ocr.h:55-65), filled by the library from CUDA
events on the context's stream and the host clock of the call."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096
MASK = VOCAB - 1


@pytest.fixture(scope="module")
def small(pkg, oracle):
    rt = pkg.TextRuntime.synthetic(seed=11, std=0.02, norm_std=0.1, num_layers=2, vocab_size=VOCAB,
                                   max_context=1024, max_prefill=256, max_tokens=256, device=0)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    yield rt, prompt
    rt.close()


def _device_sum(t):
    return t.text_embed_ms + t.prefill_ms + t.lm_head_ms + t.decode_ms


def test_ar_timing_stages(small):
    rt, p = small
    res = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                        max_tokens=80)
    t = res.timing
    assert len(res.generated_tokens) == 80
    assert t.text_embed_ms > 0 and t.prefill_ms > 0 and t.lm_head_ms > 0 and t.decode_ms > 0
    assert t.token_select_ms == 0.0   # fused into the LM-head kernels
    # The device stages are disjoint parts of the call (events vs the host clock: 50 us slack).
    assert t.total_ms + 0.05 >= _device_sum(t)
    assert abs(t.host_overhead_ms - (t.total_ms - _device_sum(t))) < 1e-6
    # hy_generate alone: no prompt stages.
    seq = p.input_ids.shape[0]
    rt.set_length(seq)
    rt.set_history(p.input_ids)
    toks, _ = rt.generate(res.generated_tokens[0], res.raw_top1_tokens[0], 80, 1.08)
    assert toks == res.generated_tokens
    g = rt.last_timing()
    assert g.text_embed_ms == 0 and g.prefill_ms == 0 and g.lm_head_ms == 0
    assert g.decode_ms > 0 and g.total_ms + 0.05 >= g.decode_ms


def test_dflash_timing_and_counts(pkg, small):
    rt, p = small
    greedy = rt.run_vlm_decode_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                           max_tokens=96).generated_tokens
    # Synthetic drafter: one device stage per block.
    seq = p.input_ids.shape[0]
    rt.set_length(seq)
    rt.set_history(p.input_ids)
    r = rt.dflash_generate_synthetic(greedy[0], 64, 1.08, greedy, 0.7, seed=5)
    assert r.generated_tokens == greedy[:64]
    t = r.timing
    assert r.block_count == len(r.acceptance_lengths) > 0
    assert r.drafted_token_count == 15 * r.block_count
    assert r.accepted_draft_token_count == sum(r.acceptance_lengths)
    assert t.blocks_ms > 0 and t.draft_ms == 0 and t.total_ms + 0.05 >= t.blocks_ms
    # With the draft network: draft / verify / commit split per block.
    rt.load_draft_synthetic(1, 3, 0.02, 0.0, MASK)
    try:
        d = rt.run_vlm_dflash_with_prompt(p.input_ids, p.position_ids, p.image_token_id, p.vision_features,
                                          max_tokens=48)
        assert d.generated_tokens == greedy[:48]   # lossless
        dt = d.timing
        assert d.block_count == len(d.acceptance_lengths) > 0
        assert d.drafted_token_count == 15 * d.block_count
        assert d.accepted_draft_token_count == sum(d.acceptance_lengths)
        assert dt.prefill_ms > 0 and dt.draft_ms > 0 and dt.verify_ms > 0 and dt.commit_ms > 0
        assert np.isclose(dt.blocks_ms, dt.draft_ms + dt.verify_ms + dt.commit_ms)
        assert dt.total_ms + 0.05 >= dt.prefill_ms + dt.blocks_ms
        assert abs(dt.host_overhead_ms - (dt.total_ms - dt.prefill_ms - dt.blocks_ms)) < 1e-6
    finally:
        rt.reset()
