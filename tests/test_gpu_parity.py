"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the
golden fixtures of the reference's own decoder wrapper.

Tolerances: integer outputs (token ids, raw top-1, acceptance lengths,
posterior ids) are bit-exact; fp32 activations and logits within 2e-4
absolute / 1e-4 relative of the oracle (fp32 GEMV reduction order and fp32
attention accumulation against the oracle's BLAS order and fp64 attention).
"""

import math

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu

SMALL = dict(num_layers=2, vocab_size=4096, max_context=2304, max_prefill=256, max_tokens=256)
SEED, NORM_STD = 11, 0.1
ATOL, RTOL = 2e-4, 1e-4


@pytest.fixture(scope="module")
def small(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=4096)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, **SMALL)
    yield cfg, w, rt
    rt.close()


def test_host_upload_equals_device_generator(pkg, small):
    cfg, w, rt = small
    rt2 = pkg.TextRuntime.from_weights(w, device=0, **SMALL)
    try:
        h = np.random.default_rng(0).standard_normal((1, 1024)).astype(np.float32)
        rt.set_history([])
        rt2.set_history([])
        _, _, l1 = rt.select_logit_rows(h, 1.0, want_logits=True)
        _, _, l2 = rt2.select_logit_rows(h, 1.0, want_logits=True)
        assert np.array_equal(l1, l2)
    finally:
        rt2.close()


@pytest.mark.parametrize("rows", [1, 16])
def test_lm_head_select_matches_oracle(small, oracle, rows):
    cfg, w, rt = small
    rng = np.random.default_rng(rows)
    h = rng.standard_normal((rows, 1024)).astype(np.float32)
    hist = rng.integers(0, cfg.vocab, 300).tolist()
    prefix = rng.integers(0, cfg.vocab, rows).tolist() if rows > 1 else None
    logits_ref = oracle.lm_head(w, h)
    # Make the history matter: put the best raw logits of each row in the history.
    hist += [int(np.argmax(logits_ref[r])) for r in range(rows)]
    rt.set_history(hist)
    tok, raw, logits = rt.select_logit_rows(h, 1.08, row_prefix=prefix, want_logits=True)
    np.testing.assert_allclose(logits, logits_ref, rtol=RTOL, atol=ATOL)
    want = oracle.select_logit_rows(logits_ref, hist, prefix, 1.08)
    assert tok.tolist() == want
    assert raw.tolist() == [int(np.argmax(logits_ref[r])) for r in range(rows)]


@pytest.mark.parametrize("rows", [1, 16])
@pytest.mark.parametrize("past", [0, 3, 100, 700, 2048])
def test_attention_matches_precise_sdpa(small, oracle, rows, past):
    cfg, w, rt = small
    rng = np.random.default_rng(1000 * rows + past)
    rt.reset()
    kpast = rng.standard_normal((8, past, 128)).astype(np.float32)
    vpast = rng.standard_normal((8, past, 128)).astype(np.float32)
    if past:
        rt.kv_write(0, 0, kpast, vpast)
    rt.set_length(past)
    qkv = rng.standard_normal((rows, 4096)).astype(np.float32)
    cos = oracle.rope_rows(past, rows, True)
    sin = oracle.rope_rows(past, rows, False)
    out = rt.attention(0, qkv, cos, sin)
    ref, knew, vnew = oracle.attention_rows(w.layers[0], qkv, cos, sin, kpast, vpast, cfg.attn_scale, cfg.rms_eps)
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    k, v = rt.kv_read(0, past, rows)
    np.testing.assert_allclose(k, knew, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(v, vnew)
    assert rt.kv_length == past + rows


def test_decoder_step_matches_oracle(small, oracle):
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(3, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    cos = oracle.build_mrope(prompt.position_ids, seq, True)
    sin = oracle.build_mrope(prompt.position_ids, seq, False)
    rt.reset()
    last = rt.prefill(emb, cos, sin)
    hidden, cache, _ = oracle.prefill(w, cfg, prompt, seq + 64)
    np.testing.assert_allclose(last, hidden[-1], rtol=RTOL, atol=ATOL)
    for rows in (1, 16):
        ids = np.arange(rows) * 7 + 5
        e = w.embed[ids]
        c = oracle.rope_rows(cache.length, rows, True)
        s = oracle.rope_rows(cache.length, rows, False)
        mask = np.where(np.arange(cache.length + rows)[None, :] > cache.length + np.arange(rows)[:, None],
                        np.float32(-1e38), np.float32(0)).astype(np.float32)
        ref, ref_aux = oracle.decoder_forward(w, cfg, e, mask, c, s, cache, aux=True)
        got, aux = rt.run_decoder_step(e, c, s, aux=True)
        np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(aux[0], ref_aux[0], rtol=RTOL, atol=ATOL)   # layer 1 (2-layer model)
    assert rt.kv_length == seq + 17


def _golden_runtime(pkg, g, **extra):
    return pkg.TextRuntime.synthetic(seed=int(g["seed"]), std=0.02, norm_std=float(g["norm_std"]),
                                     num_layers=int(g["layers"]), vocab_size=int(g["vocab"]),
                                     attn_scale=float(g["attn_scale"]), device=0, **extra)


def _golden_prompt(oracle, g):
    return oracle.synthetic_prompt(int(g["seed"]), int(g["grid_h"]), int(g["grid_w"]), int(g["n_text"]),
                                   int(g["vocab"]), int(g["image_token_id"]))


@pytest.mark.parametrize("case", ["small_2l", "full_24l"])
def test_ar_decode_matches_reference_golden(pkg, oracle, case):
    g = load_golden(case)
    prompt = _golden_prompt(oracle, g)
    n = len(g["tokens"])
    with _golden_runtime(pkg, g, max_context=2048, max_prefill=1024, max_tokens=64) as rt:
        res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                            prompt.vision_features, max_tokens=n)
        assert res.generated_tokens == g["tokens"].tolist()
        assert res.raw_top1_tokens == g["raw_top1"].tolist()


@pytest.mark.parametrize("case", ["small_2l", "full_24l"])
def test_verify_block_matches_reference_golden(pkg, oracle, case):
    g = load_golden(case)
    prompt = _golden_prompt(oracle, g)
    seq = prompt.input_ids.shape[0]
    # Only the embedding table is needed on the host (the prompt rows).
    emb_w = oracle.make_weights(oracle.ModelConfig(num_layers=0, vocab=int(g["vocab"])), int(g["seed"]))
    emb = oracle.prepare_prompt_embeddings(emb_w, prompt)
    with _golden_runtime(pkg, g, max_context=2048, max_prefill=1024, max_tokens=64) as rt:
        rt.reset()
        rt.prefill(emb, oracle.build_mrope(prompt.position_ids, seq, True),
                   oracle.build_mrope(prompt.position_ids, seq, False))
        rt.set_history(prompt.input_ids)
        post, accept, committed, stop = rt.dflash_verify_block(g["verify_proposed"], 16, 1.08)
        assert post == g["verify_posterior"].tolist()
        assert accept == int(g["verify_accept"])
        assert committed == accept + 1 and not stop
        assert rt.kv_length == seq + committed


def test_dflash_is_lossless_and_matches_oracle(small, oracle):
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    n = 48
    res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=n + 20)
    greedy = res.generated_tokens
    want_ar = oracle.decode_ar(w, cfg, prompt, n + 20)
    assert greedy == want_ar.tokens
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    cos = oracle.build_mrope(prompt.position_ids, seq, True)
    sin = oracle.build_mrope(prompt.position_ids, seq, False)
    for p in (0.3, 0.7, 0.9):
        rt.reset()
        rt.prefill(emb, cos, sin)
        rt.set_history(prompt.input_ids)
        out = rt.dflash_generate_synthetic(greedy[0], n, 1.08, greedy, p, seed=99)
        assert out.generated_tokens == greedy[:n], p
        ref = oracle.decode_dflash(w, cfg, prompt, n, oracle.synthetic_drafter(greedy, p, cfg.vocab, 99))
        assert ref.tokens == greedy[:n]
        assert out.acceptance_lengths == ref.acceptance_lengths, p
        assert out.block_count == ref.block_count


def test_dflash_lossless_repeated(small, oracle):
    """The verify path gives the same tokens on every run: 150 repetitions of the
    lossless check at p = 0.9 (a race between the layer-0 residual publication and the
    in-place RMSNorm once flipped one token in a few hundred runs)."""
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    n = 48
    greedy = oracle.decode_ar(w, cfg, prompt, n + 20).tokens
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    cos = oracle.build_mrope(prompt.position_ids, seq, True)
    sin = oracle.build_mrope(prompt.position_ids, seq, False)
    bad = []
    for rep in range(150):
        rt.reset()
        rt.prefill(emb, cos, sin)
        rt.set_history(prompt.input_ids)
        out = rt.dflash_generate_synthetic(greedy[0], n, 1.08, greedy, 0.9, seed=99)
        if out.generated_tokens != greedy[:n]:
            bad.append(rep)
    assert not bad, f"runs with different tokens: {bad}"


@pytest.mark.parametrize("penalty", [1.08, 1.0])
@pytest.mark.parametrize("path", ["persistent", "graph"])
def test_ar_paths_match_oracle(pkg, small, oracle, path, penalty):
    """Both AR paths, with the reference's default penalty and with none (config 0's two runs)."""
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(33, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    want = oracle.decode_ar(w, cfg, prompt, 150, penalty=penalty)
    rt.ar_path = pkg.AR_PATH_PERSISTENT if path == "persistent" else pkg.AR_PATH_GRAPH
    try:
        res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                            prompt.vision_features, max_tokens=150, repetition_penalty=penalty)
    finally:
        rt.ar_path = pkg.AR_PATH_PERSISTENT
    assert res.generated_tokens == want.tokens
    assert res.raw_top1_tokens == want.raw_top1
    assert rt.kv_length == prompt.input_ids.shape[0] + 149


def test_ar_paths_repeated(pkg, small, oracle):
    """Both AR paths give the oracle's tokens on every one of 40 runs each (the graph
    path's kernels read constants and the decode state before waiting on the kernel
    before them; a race there would show as a run that differs)."""
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(33, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    want = oracle.decode_ar(w, cfg, prompt, 100).tokens
    bad = []
    try:
        for path in (pkg.AR_PATH_GRAPH, pkg.AR_PATH_PERSISTENT):
            rt.ar_path = path
            for rep in range(40):
                res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                                    prompt.vision_features, max_tokens=100)
                if res.generated_tokens != want:
                    bad.append((path, rep))
    finally:
        rt.ar_path = pkg.AR_PATH_PERSISTENT
    assert not bad, f"runs with different tokens: {bad}"


def test_eos_stops_generation(small, oracle):
    cfg, w, rt = small
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, cfg.vocab, cfg.vocab - 3)
    res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=30)
    eos = res.generated_tokens[7]
    stop_at = res.generated_tokens.index(eos)
    res2 = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                         prompt.vision_features, max_tokens=30, eos_ids=[eos])
    assert res2.generated_tokens == res.generated_tokens[:stop_at + 1]


def test_capacity_and_argument_errors(pkg, small):
    cfg, w, rt = small
    with pytest.raises(pkg.HyError) as e:
        rt.truncate(10 ** 6)
    assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
    with pytest.raises(pkg.HyError) as e:
        rt.run_decoder_step(np.zeros((17, 1024), np.float32), np.zeros((17, 128), np.float32),
                            np.zeros((17, 128), np.float32))
    assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
    rt.set_length(SMALL["max_context"] - 1)
    with pytest.raises(pkg.HyError) as e:
        rt.dflash_verify_block(list(range(16)), 16, 1.08)
    assert e.value.status == pkg.HY_ERR_CAPACITY
    rt.reset()


def test_full_config_ar_tokens_match_oracle(pkg, oracle):
    """The AR decode workload in full (24 layers, vocab 120818, 768 image rows on 24x32 + 256 text
    ids, fp32, ncnn SDPA scale): all 256 greedy tokens with penalty 1.08 identical to the oracle."""
    cfg = oracle.ModelConfig()
    w = oracle.make_weights(cfg, 0)
    prompt = oracle.synthetic_prompt(0, 24, 32, 256, cfg.vocab)
    n = 256
    want = oracle.decode_ar(w, cfg, prompt, n)
    with pkg.TextRuntime.synthetic(seed=0, max_prefill=1024, max_tokens=256, max_context=2048, device=0) as rt:
        res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                            prompt.vision_features, max_tokens=n)
    mism = [i for i, (a, b) in enumerate(zip(res.generated_tokens, want.tokens)) if a != b]
    assert not mism, f"first mismatch at {mism[0]}, oracle top-2 margin {want.margins[mism[0]]:.3g}"


def test_lm_head_m1_full_vocab_logits(pkg, oracle):
    """The LM-head workload at M = 1: hidden N(0,1) against the full 120818 x 1024 tied table;
    logits within the fp32 tolerance, raw and penalised argmax bit-exact."""
    vocab = 120818
    w = oracle.make_weights(oracle.ModelConfig(num_layers=0, vocab=vocab), 3)
    rng = np.random.default_rng(120818)
    with pkg.TextRuntime.synthetic(seed=3, num_layers=2, vocab_size=vocab, max_prefill=64, max_tokens=32,
                                   max_context=256, device=0) as rt:
        for trial in range(3):
            h = rng.standard_normal((1, 1024)).astype(np.float32)
            ref = oracle.lm_head(w, h)
            hist = rng.integers(0, vocab, 500).tolist() + [int(np.argmax(ref[0]))]
            rt.set_history(hist)
            tok, raw, logits = rt.select_logit_rows(h, 1.08, want_logits=True)
            np.testing.assert_allclose(logits, ref, rtol=RTOL, atol=ATOL)
            assert raw.tolist() == [int(np.argmax(ref[0]))]
            assert tok.tolist() == oracle.select_logit_rows(ref, hist, None, 1.08)


def test_full_24l_golden_logits_within_tolerance(pkg, oracle):
    """The 24-layer golden of the reference's own decoder wrapper, step by step through the
    step interface (prefill, then run_decoder_step + LM head per token): every step's top-16
    logits within 1e-3 relative of the golden, tokens and raw top-1 exact."""
    g = load_golden("full_24l")
    prompt = _golden_prompt(oracle, g)
    seq = prompt.input_ids.shape[0]
    emb_w = oracle.make_weights(oracle.ModelConfig(num_layers=0, vocab=int(g["vocab"])), int(g["seed"]))
    emb = oracle.prepare_prompt_embeddings(emb_w, prompt)
    penalty = float(g["penalty"])
    with _golden_runtime(pkg, g, max_context=2048, max_prefill=1024, max_tokens=64) as rt:
        rt.reset()
        last = rt.prefill(emb, oracle.build_mrope(prompt.position_ids, seq, True),
                          oracle.build_mrope(prompt.position_ids, seq, False))
        # fp32 hidden state after 24 layers: 2e-4 absolute, the tolerance the oracle itself meets here.
        np.testing.assert_allclose(last, g["prefill_last_hidden"], rtol=1e-3, atol=2e-4)
        rt.set_history(prompt.input_ids)
        hidden = last[None, :]
        for i in range(len(g["tokens"])):
            tok, raw, logits = rt.select_logit_rows(hidden, penalty, want_logits=True)
            np.testing.assert_allclose(logits[0, g["top16_idx"][i]], g["top16_val"][i], rtol=1e-3, atol=1e-4)
            assert int(tok[0]) == int(g["tokens"][i]) and int(raw[0]) == int(g["raw_top1"][i])
            rt.add_history([int(tok[0])])
            pos = seq + i
            hidden, _ = rt.run_decoder_step(emb_w.embed[int(tok[0]):int(tok[0]) + 1], oracle.rope_rows(pos, 1, True),
                                            oracle.rope_rows(pos, 1, False))
