"""Pins the CPU oracle: the reference's known-answer tests and the golden fixtures.

The golden fixtures (tests/golden/*.npz) come from tests/golden/make_golden.py,
which runs the reference's own decoder wrapper (export/text_decoder_kv.py) over
a transformers HunYuanDenseV1Model on CPU fp32.
"""

import math

import numpy as np
import pytest

from conftest import load_golden


def test_build_mrope_known_answer(oracle):
    # tests/text_rope_test.cpp:8-34
    pos = np.array([978, 811, 621, 431], np.int32).reshape(4, 1)
    cos = oracle.build_mrope(pos, 1, True)[0]
    dims = [0, 2, 31, 32, 63, 64, 95, 96, 127]
    want = [-0.569676042, -0.0682837293, 0.929675043, 0.970673621, 1.0, 0.510228872, 0.97144419, 0.991688073, 1.0]
    for d, w in zip(dims, want):
        assert abs(float(cos[d]) - w) <= 2e-7


def test_multimodal_rope_known_answer(oracle):
    # tests/multimodal_rope_test.cpp:17-48 (4-dim, non-interleaved, full-width cos/sin)
    x = np.array([[[1.0, 2.0, 3.0, 4.0]]], np.float32)
    c = np.array([[0.5, 0.25, 0.75, 0.125]], np.float32)
    s = np.array([[0.1, 0.2, 0.3, 0.4]], np.float32)
    out = oracle.apply_rope(x, c, s)[0, 0]
    want = [1 * 0.5 - 3 * 0.1, 2 * 0.25 - 4 * 0.2, 3 * 0.75 + 1 * 0.3, 4 * 0.125 + 2 * 0.4]
    assert np.allclose(out, want, atol=1e-6)


def test_precise_sdpa_closed_form(oracle):
    # tests/precise_sdpa_test.cpp:226-269
    q = np.array([[[1.0e8, 1.0, -1.0e8]]], np.float32)
    k = np.array([[[1.0, 1.0, 1.0], [0.0, 0.0, 0.0]]], np.float32)
    v = np.array([[[10.0], [20.0]]], np.float32)
    out = oracle.precise_sdpa(q, k, v, np.zeros((1, 2), np.float32), 1.0)
    p = math.exp(1.0) / (math.exp(1.0) + 1.0)
    assert abs(float(out[0, 0, 0]) - (p * 10 + (1 - p) * 20)) <= 1e-5


def _fill_channel_rows(shape, seed):
    c, h, w = shape
    return (seed + 0.01 * np.arange(c)[:, None, None] + 0.1 * np.arange(h)[None, :, None]
            + 0.001 * np.arange(w)[None, None, :]).astype(np.float32)


@pytest.mark.parametrize("query_len", [1, 16])
def test_precise_sdpa_gqa_matches_expanded_attention(oracle, query_len):
    # tests/precise_sdpa_test.cpp:557-629: 4 q heads / 2 kv heads, head_dim 4, past 7, scale 0.25.
    past = 7
    pk = _fill_channel_rows((2, past, 4), 0.2)
    pv = _fill_channel_rows((2, past, 4), 0.3)
    q = _fill_channel_rows((4, query_len, 4), 0.4)
    ck = _fill_channel_rows((2, query_len, 4), 0.5)
    cv = _fill_channel_rows((2, query_len, 4), 0.6)
    k = np.concatenate([pk, ck], axis=1)
    v = np.concatenate([pv, cv], axis=1)
    out = oracle.precise_sdpa(q, k, v, np.zeros((query_len, past + query_len), np.float32), 0.25)
    for h in range(4):
        kk, vv = k[h // 2].astype(np.float64), v[h // 2].astype(np.float64)
        s = q[h].astype(np.float64) @ kk.T * 0.25
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        assert np.allclose(out[h], p @ vv, atol=1e-5)


def test_dflash_helpers(oracle):
    # tests/dflash_runtime_test.cpp:9-63
    block = oracle.build_dflash_block(42)
    assert len(block) == 16 and block[0] == 42 and all(t == 120817 for t in block[1:])
    mask = oracle.build_dflash_verify_mask(3)
    assert mask.shape == (16, 19)
    for r in range(16):
        for c in range(19):
            visible = c <= 3 + r
            assert (mask[r, c] == 0.0) if visible else (mask[r, c] <= -1.0e30)
    assert oracle.dflash_acceptance_length([10, 11, 12, 13], [11, 12, 99, 100]) == 2
    assert oracle.dflash_acceptance_length([10, 11], [11]) == -1


def test_select_next_token_semantics(oracle):
    # src/text_runtime.cpp:730-755: raw top-1 is the first strict max; history ids are
    # penalised once (s<0 ? s*p : s/p); out-of-range ids are ignored; ties keep the first index.
    logits = np.array([1.0, 3.0, 3.0, -2.0, 2.9], np.float32)
    tok, raw = oracle.select_next_token(logits, [1, 1, 7, -1], 1.08)
    assert raw == 1 and tok == 2
    tok, raw = oracle.select_next_token(logits, [], 1.08)
    assert tok == 1 and raw == 1
    tok, _ = oracle.select_next_token(np.array([-1.0, -1.05], np.float32), [1], 1.08)
    assert tok == 0


def test_synth_generator_numpy_matches_c(oracle):
    a = oracle.synth_tensor(3, 17, 50000, 0.02)
    b = oracle.synth_tensor_fast(3, 17, 50000, 0.02)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert abs(float(a.std()) - 0.02) < 5e-4


def _run_case(oracle, g):
    layers, vocab = int(g["layers"]), int(g["vocab"])
    cfg = oracle.ModelConfig(num_layers=layers, vocab=vocab, attn_scale=float(g["attn_scale"]))
    w = oracle.make_weights(cfg, int(g["seed"]), std=0.02, norm_std=float(g["norm_std"]))
    prompt = oracle.synthetic_prompt(int(g["seed"]), int(g["grid_h"]), int(g["grid_w"]), int(g["n_text"]), vocab,
                                     int(g["image_token_id"]))
    assert np.array_equal(prompt.input_ids, g["input_ids"])
    assert np.array_equal(prompt.position_ids, g["position_ids"])
    assert abs(float(prompt.vision_features.astype(np.float64).sum()) - float(g["feature_checksum"])) < 1e-6
    return cfg, w, prompt


@pytest.mark.parametrize("case", ["small_2l", "full_24l"])
def test_oracle_matches_reference_wrapper(oracle, case):
    g = load_golden(case)
    cfg, w, prompt = _run_case(oracle, g)
    n = len(g["tokens"])
    seq = prompt.input_ids.shape[0]
    hidden, cache, _ = oracle.prefill(w, cfg, prompt, seq + n + 32)
    np.testing.assert_allclose(hidden[-1], g["prefill_last_hidden"], rtol=0, atol=2e-4)
    snapshot = (hidden.copy(), [k.copy() for k in cache.k], [v.copy() for v in cache.v], cache.length)
    tr = oracle.decode_ar(w, cfg, prompt, n, keep_logits=True, prefill_state=(hidden, cache))
    assert tr.tokens == g["tokens"].tolist()
    assert tr.raw_top1 == g["raw_top1"].tolist()
    for step in range(n):
        idx = g["top16_idx"][step]
        np.testing.assert_allclose(tr.logits[step][idx], g["top16_val"][step], rtol=0, atol=2e-4)
    if g["logits_first2"].size:
        np.testing.assert_allclose(np.stack(tr.logits[:2]), g["logits_first2"], rtol=0, atol=2e-4)
    # Cache rows after the AR run (16-head expanded in the reference: q head h <- kv head h//2).
    rows = g["cache_rows"]
    for which, (li, arr) in enumerate([(0, cache.k), (-1, cache.k), (-1, cache.v)]):
        mine = arr[li][:, rows, :]
        ref = g["cache_samples"][which]
        np.testing.assert_allclose(np.repeat(mine, 2, axis=0), ref, rtol=0, atol=2e-4)
    # Verify block from the prefill state.
    hidden0, k0, v0, l0 = snapshot
    cache2 = oracle.KVCache(k0, v0, l0)
    post, accept, vlogits, _ = oracle.verify_block(w, cfg, cache2, g["verify_proposed"].tolist(),
                                                   prompt.input_ids.tolist(), oracle.DEFAULT_PENALTY)
    assert post == g["verify_posterior"].tolist()
    assert accept == int(g["verify_accept"])
    np.testing.assert_allclose(np.take_along_axis(vlogits, g["verify_top8_idx"], 1), g["verify_top8_val"],
                               rtol=0, atol=2e-4)


def test_draft_network_matches_reference_wrapper(oracle):
    """The oracle's DFlash draft forward (context append + 2 draft layers) against the
    reference's own draft graph (export/dflash_export.py DFlashExportWrapper), run by
    tests/golden/make_dflash_draft_golden.py on the same synthetic draft weights."""
    g = load_golden("dflash_draft_2l")
    layers, ctx = int(g["layers"]), int(g["ctx"])
    dw = oracle.make_draft_weights(layers, int(g["seed"]), 0.02, float(g["norm_std"]))
    rng = np.random.default_rng(int(g["input_seed"]))
    noise = rng.standard_normal((oracle.DFLASH_BLOCK, oracle.HIDDEN)).astype(np.float32)
    aux = [rng.standard_normal((ctx, oracle.HIDDEN)).astype(np.float32) for _ in range(4)]
    assert math.isclose(noise.astype(np.float64).sum(), float(g["noise_sum"]), rel_tol=0, abs_tol=1e-9)
    assert math.isclose(sum(a.astype(np.float64).sum() for a in aux), float(g["aux_sum"]), rel_tol=0, abs_tol=1e-9)
    cache = oracle.DraftCache.empty(layers, ctx + oracle.DFLASH_BLOCK)
    oracle.draft_append_context(dw, cache, aux)
    out = oracle.draft_forward(dw, noise, cache)
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=2e-5)


def test_draft_rope_formula(oracle):
    """build_dflash_rope (src/dflash_runtime.cpp:27-48): position p, dim d uses
    p / 10000^(2 (d % 64) / 128); position 0 is cos 1, sin 0; dims d and d + 64 match."""
    c = oracle.build_dflash_rope(0, 5, True)
    s = oracle.build_dflash_rope(0, 5, False)
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)
    np.testing.assert_array_equal(c[:, :64], c[:, 64:])
    np.testing.assert_allclose(c[3, 1], math.cos(3.0 / 10000.0 ** (2.0 / 128.0)), rtol=1e-6)
    np.testing.assert_allclose(s[4, 0], math.sin(4.0), rtol=1e-6)
