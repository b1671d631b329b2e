"""GPU parity of the DFlash draft network (export/dflash_export.py's graph, run by
DFlashDraftRuntime::run, src/dflash_runtime.cpp:213-290) and of the DFlash loop
that uses it (decode_dflash_from_embeddings, src/text_runtime.cpp:1142-1305),
through the C ABI.

Tolerances as in the other parity tests: draft hidden rows within 2e-4 absolute /
1e-4 relative of the reference wrapper's fixture and of the oracle; token ids,
acceptance lengths and block counts bit-exact. Draft proposals are compared
where the oracle's top-2 logit margin exceeds 1e-3 (a margin below the fp32
tolerance may flip either way; no such row decides an acceptance here).
"""

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-4, 1e-4
VOCAB = 4096
MASK = VOCAB - 1
SEED, NORM_STD = 7, 0.1
DRAFT_LAYERS, DRAFT_SEED = 2, 19


def _reference_inputs(g):
    rng = np.random.default_rng(int(g["input_seed"]))
    noise = rng.standard_normal((16, 1024)).astype(np.float32)
    aux = np.stack([rng.standard_normal((int(g["ctx"]), 1024)).astype(np.float32) for _ in range(4)])
    return noise, aux


@pytest.mark.parametrize("upload", [False, True])
def test_draft_run_matches_reference_wrapper(pkg, oracle, upload):
    """Context append + draft forward against the reference's DFlashExportWrapper
    output (tests/golden/make_dflash_draft_golden.py) on the same synthetic draft."""
    g = load_golden("dflash_draft_2l")
    layers, ctx = int(g["layers"]), int(g["ctx"])
    noise, aux = _reference_inputs(g)
    with pkg.TextRuntime.synthetic(seed=1, num_layers=2, vocab_size=VOCAB, max_context=256, max_prefill=64,
                                   max_tokens=64, device=0) as rt:
        if upload:
            rt.load_draft(oracle.make_draft_weights(layers, int(g["seed"]), 0.02, float(g["norm_std"])), MASK)
        else:
            rt.load_draft_synthetic(layers, int(g["seed"]), 0.02, float(g["norm_std"]), MASK)
        rt.draft_context_append(aux)
        assert rt.draft_context_length == ctx
        out = rt.draft_run(noise)
    np.testing.assert_allclose(out, g["out"], rtol=RTOL, atol=ATOL)


def test_draft_context_in_two_appends_and_steps(pkg, oracle):
    """Context rows appended in pieces (prompt path) and a draft run over them
    equal the oracle's one-shot append; a second run after more rows still matches."""
    dw = oracle.make_draft_weights(3, DRAFT_SEED, 0.02, NORM_STD)
    rng = np.random.default_rng(5)
    aux = rng.standard_normal((4, 300, 1024)).astype(np.float32)
    noise = rng.standard_normal((16, 1024)).astype(np.float32)
    with pkg.TextRuntime.synthetic(seed=1, num_layers=2, vocab_size=VOCAB, max_context=512, max_prefill=200,
                                   max_tokens=64, device=0) as rt:
        rt.load_draft_synthetic(3, DRAFT_SEED, 0.02, NORM_STD, MASK)
        rt.draft_context_append(aux[:, :37])
        rt.draft_context_append(aux[:, 37:250])   # two passes of the 200-row prefill buffers
        got1 = rt.draft_run(noise)
        rt.draft_context_append(aux[:, 250:])
        got2 = rt.draft_run(noise)
    for n, got in ((250, got1), (300, got2)):
        cache = oracle.DraftCache.empty(3, n + 16)
        oracle.draft_append_context(dw, cache, list(aux[:, :n]))
        want = oracle.draft_forward(dw, noise, cache)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.fixture(scope="module")
def deep(pkg, oracle):
    """24 decoder layers (the aux layers 1, 8, 15, 22 exist) with a 4096-id vocabulary."""
    cfg = oracle.ModelConfig(num_layers=24, vocab=VOCAB)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    dw = oracle.make_draft_weights(DRAFT_LAYERS, DRAFT_SEED, 0.02, NORM_STD)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, num_layers=24, vocab_size=VOCAB,
                                   max_context=512, max_prefill=128, max_tokens=128, device=0)
    rt.load_draft_synthetic(DRAFT_LAYERS, DRAFT_SEED, 0.02, NORM_STD, MASK)
    prompt = oracle.synthetic_prompt(23, 4, 6, 16, VOCAB, VOCAB - 3)
    yield cfg, w, dw, rt, prompt
    rt.close()


def test_draft_propose_matches_oracle(deep, oracle):
    cfg, w, dw, rt, prompt = deep
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    cos = oracle.build_mrope(prompt.position_ids, seq, True)
    sin = oracle.build_mrope(prompt.position_ids, seq, False)
    rt.reset()
    rt.prefill(emb, cos, sin)
    assert rt.draft_context_length == seq
    _, _, aux = oracle.prefill(w, cfg, prompt, seq + 32, aux=True)
    dcache = oracle.DraftCache.empty(DRAFT_LAYERS, seq + 32)
    oracle.draft_append_context(dw, dcache, aux, cfg.rms_eps)
    for current in (5, 1234):
        got = rt.draft_propose(current)
        want, hidden = oracle.draft_propose(w, dw, dcache, current, cfg.rms_eps, MASK)
        logits = oracle.lm_head(w, hidden[1:])
        top2 = np.sort(logits, axis=1)[:, -2:]
        sure = (top2[:, 1] - top2[:, 0]) > 1e-3
        assert got[0] == current
        assert [a for a, s in zip(got[1:], sure) if s] == [b for b, s in zip(want[1:], sure) if s]
        assert sure.sum() >= 12


def test_decoder_steps_extend_the_draft_context(deep, oracle):
    """Explicit decoder steps (1 row, then 5 rows) on a prefilled sequence also append
    their rows' draft context; the drafts then match the oracle's over the same context."""
    cfg, w, dw, rt, prompt = deep
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    rt.reset()
    rt.prefill(emb, oracle.build_mrope(prompt.position_ids, seq, True),
               oracle.build_mrope(prompt.position_ids, seq, False))
    _, cache, aux = oracle.prefill(w, cfg, prompt, seq + 64, aux=True)
    dcache = oracle.DraftCache.empty(DRAFT_LAYERS, seq + 64)
    oracle.draft_append_context(dw, dcache, aux, cfg.rms_eps)
    past = seq
    for ids in ([7], [8, 9, 10, 11, 12]):
        n = len(ids)
        x = w.embed[np.asarray(ids)]
        cos, sin = oracle.rope_rows(past, n, True), oracle.rope_rows(past, n, False)
        rt.run_decoder_step(x, cos, sin)
        col = np.arange(past + n)[None, :]
        mask = np.where(col > past + np.arange(n)[:, None], np.float32(-1e38), np.float32(0)).astype(np.float32)
        _, step_aux = oracle.decoder_forward(w, cfg, x, mask, cos, sin, cache, aux=True)
        oracle.draft_append_context(dw, dcache, step_aux, cfg.rms_eps)
        past += n
    assert rt.draft_context_length == rt.kv_length == past
    got = rt.draft_propose(33)
    want, hidden = oracle.draft_propose(w, dw, dcache, 33, cfg.rms_eps, MASK)
    top2 = np.sort(oracle.lm_head(w, hidden[1:]), axis=1)[:, -2:]
    sure = (top2[:, 1] - top2[:, 0]) > 1e-3
    assert [a for a, s_ in zip(got[1:], sure) if s_] == [b for b, s_ in zip(want[1:], sure) if s_]
    assert sure.sum() >= 12


def test_dflash_with_draft_is_lossless_and_matches_oracle(deep, oracle):
    """--dflash end to end on the device: tokens equal the AR greedy tokens (the
    lossless invariant, tests/hunyuan_ocr_runtime_integration_test.cpp:138-139),
    and the acceptance lengths equal the oracle's DFlash loop with its draft."""
    cfg, w, dw, rt, prompt = deep
    n = 40
    want_ar = oracle.decode_ar(w, cfg, prompt, n)
    want = oracle.decode_dflash_draft(w, cfg, dw, prompt, n, mask_token=MASK)
    assert want.tokens == want_ar.tokens
    res = rt.run_vlm_dflash_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=n)
    assert res.generated_tokens == want_ar.tokens
    assert res.acceptance_lengths == want.acceptance_lengths
    assert res.block_count == want.block_count
    # Every committed token went through a verify block, so the cache (and the draft
    # context) hold the prompt plus all generated tokens.
    seq = prompt.input_ids.shape[0]
    assert rt.kv_length == rt.draft_context_length == seq + n


def test_host_driven_draft_loop_matches_device_loop(deep, oracle):
    """The reference's block structure driven from the host (draft_propose ->
    verify block with the context append) gives the device loop's tokens."""
    cfg, w, dw, rt, prompt = deep
    n = 24
    res = rt.run_vlm_dflash_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=n)
    seq = prompt.input_ids.shape[0]
    emb = oracle.prepare_prompt_embeddings(w, prompt)
    rt.reset()
    rt.prefill(emb, oracle.build_mrope(prompt.position_ids, seq, True),
               oracle.build_mrope(prompt.position_ids, seq, False))
    rt.set_history(prompt.input_ids)
    tokens, accepts = [], []
    current = res.generated_tokens[0]
    while len(tokens) < n:
        proposed = rt.draft_propose(current)
        post, accept, committed, stop = rt.dflash_verify_block(proposed, n - len(tokens), 1.08)
        assert rt.draft_context_length == rt.kv_length
        tokens += proposed[:committed]
        accepts.append(max(0, committed - 1))
        current = post[accept]
        if stop or committed < accept + 1:
            break
    assert tokens == res.generated_tokens
    assert accepts == res.acceptance_lengths


def test_draft_errors(pkg, deep):
    cfg, w, dw, rt, prompt = deep
    with pkg.TextRuntime.synthetic(seed=1, num_layers=2, vocab_size=VOCAB, max_context=256, max_prefill=64,
                                   max_tokens=64, device=0) as rt2:
        with pytest.raises(pkg.HyError) as e:
            rt2.draft_propose(3)
        assert e.value.status == pkg.HY_ERR_NOT_READY
        with pytest.raises(pkg.HyError) as e:
            rt2.load_draft_synthetic(2, 1, mask_token=VOCAB)
        assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
        rt2.load_draft_synthetic(1, 1, mask_token=MASK)
        with pytest.raises(pkg.HyError) as e:
            rt2.draft_run(np.zeros((16, 1024), np.float32))   # empty context
        assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
    # AR generation does not extend the draft context: the DFlash loop then refuses to run.
    rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                  prompt.vision_features, max_tokens=4)
    assert rt.draft_context_length < rt.kv_length
    with pytest.raises(pkg.HyError) as e:
        rt.dflash_generate(5, 8, 1.08)
    assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
