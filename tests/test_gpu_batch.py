"""GPU parity of the batched decode (hy_batch_decode): several JSONL-style records
decoding together on one context, each record's tokens equal to the oracle's AR
greedy decode of that record alone (run_jsonl_batch runs the records one after the
other through run_vlm_decode_with_prompt, src/batch_jsonl.cpp:384-480). Token ids
are bit-exact; a malformed record fails alone.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 4096
SEED, NORM_STD = 11, 0.1
CFG = dict(num_layers=2, vocab_size=VOCAB, max_context=512, max_prefill=256, max_tokens=64)


@pytest.fixture(scope="module")
def model(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, **CFG)
    yield cfg, w, rt
    rt.close()


def _prompts(oracle, n):
    shapes = [(4, 6, 16), (2, 3, 40), (3, 5, 8), (6, 6, 30), (1, 4, 5), (5, 2, 60), (2, 2, 3)]
    out = []
    for i in range(n):
        gh, gw, nt = shapes[i % len(shapes)]
        out.append(oracle.synthetic_prompt(100 + i, gh, gw, nt, VOCAB, VOCAB - 3))
    return out


def _req(p):
    return (p.input_ids, p.position_ids, p.image_token_id, p.vision_features)


@pytest.mark.parametrize("slots", [3, 16])
def test_batch_tokens_match_oracle_per_record(model, oracle, slots):
    cfg, w, rt = model
    prompts = _prompts(oracle, 7)
    n = 40
    toks, status = rt.batch_decode([_req(p) for p in prompts], n, slots=slots)
    assert status == [0] * len(prompts)
    for p, got in zip(prompts, toks):
        assert got == oracle.decode_ar(w, cfg, p, n).tokens
    assert rt.kv_length == 0


def test_batch_repeated(model, oracle):
    """Ten batched runs of the same records give the same (oracle) tokens every time."""
    cfg, w, rt = model
    prompts = _prompts(oracle, 7)
    n = 40
    want = [oracle.decode_ar(w, cfg, p, n).tokens for p in prompts]
    for rep in range(10):
        toks, status = rt.batch_decode([_req(p) for p in prompts], n, slots=16)
        assert status == [0] * len(prompts)
        assert toks == want, rep


def test_batch_equals_single_record_calls_with_eos(model, oracle):
    cfg, w, rt = model
    prompts = _prompts(oracle, 5)
    n = 30
    single = [rt.run_vlm_decode_with_prompt(*_req(p), max_tokens=n).generated_tokens for p in prompts]
    eos = single[2][6]
    want = [s[:s.index(eos) + 1] if eos in s else s for s in single]
    toks, status = rt.batch_decode([_req(p) for p in prompts], n, slots=4, eos_ids=[eos])
    assert status == [0] * len(prompts)
    assert toks == want


def test_malformed_record_fails_alone(pkg, model, oracle):
    cfg, w, rt = model
    prompts = _prompts(oracle, 3)
    bad = prompts[1]
    reqs = [_req(prompts[0]), (bad.input_ids, bad.position_ids, bad.image_token_id, bad.vision_features[:-1]),
            _req(prompts[2])]
    toks, status = rt.batch_decode(reqs, 12, slots=2)
    assert status[1] == pkg.HY_ERR_INVALID_ARGUMENT and toks[1] == []
    assert status[0] == status[2] == 0
    assert toks[0] == oracle.decode_ar(w, cfg, prompts[0], 12).tokens
    assert toks[2] == oracle.decode_ar(w, cfg, prompts[2], 12).tokens


def test_batch_edge_cases(pkg, model, oracle):
    """No records; more slots than records; a record whose first token is EOS or whose
    max_tokens is 1 finishes at admission; bad arguments are rejected."""
    cfg, w, rt = model
    assert rt.batch_decode([], 8) == ([], [])
    prompts = _prompts(oracle, 2)
    want = [oracle.decode_ar(w, cfg, p, 6).tokens for p in prompts]
    toks, status = rt.batch_decode([_req(p) for p in prompts], 6, slots=16)
    assert status == [0, 0] and toks == want
    toks, _ = rt.batch_decode([_req(p) for p in prompts], 1, slots=2)
    assert toks == [t[:1] for t in want]
    toks, _ = rt.batch_decode([_req(p) for p in prompts], 6, slots=2, eos_ids=[want[0][0]])
    assert toks[0] == want[0][:1]
    with pytest.raises(pkg.HyError) as e:
        rt.batch_decode([_req(prompts[0])], 6, slots=17)
    assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT
    with pytest.raises(pkg.HyError) as e:
        rt.batch_decode([_req(prompts[0])], CFG["max_tokens"] + 1)
    assert e.value.status == pkg.HY_ERR_CAPACITY
