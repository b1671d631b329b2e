"""Decoding from a model package (hy_ctx_create_from_package, hy_draft_load_package): a
package written in the reference's exported layout (hunyuanocr-ncnn_b200/ncnn_package.py)
from the same seeded weights as TextRuntime.synthetic must decode the same tokens with the
same logits; an fp16-stored package must match a context created from the fp16-rounded
weights."""

import importlib.util
import os

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

VOCAB, SEED, NORM_STD = 4096, 11, 0.1
MASK = VOCAB - 1
CTX = dict(max_context=512, max_prefill=64, max_tokens=64, device=0)


def _writer():
    spec = importlib.util.spec_from_file_location("hy_ncnn_package",
                                                  os.path.join(REPO, "hunyuanocr-ncnn_b200", "ncnn_package.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _decode(rt, prompt, n=24):
    res = rt.run_vlm_decode_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                        prompt.vision_features, max_tokens=n)
    h = np.random.default_rng(5).standard_normal((2, 1024)).astype(np.float32)
    rt.set_history([])
    _, _, logits = rt.select_logit_rows(h, 1.0, want_logits=True)
    return res.generated_tokens, logits


def test_package_decodes_like_the_synthetic_context(pkg, oracle, tmp_path):
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    dw = oracle.make_draft_weights(1, 3, 0.02, 0.0)
    root = str(tmp_path / "pkg")
    _writer().write_package(root, w, draft=dw)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    with pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, num_layers=2, vocab_size=VOCAB,
                                   **CTX) as ref, pkg.TextRuntime.from_package(root, **CTX) as rt:
        assert (rt.cfg.num_layers, rt.cfg.vocab_size, rt.cfg.ffn_dim) == (2, VOCAB, 3584)
        t_ref, l_ref = _decode(ref, prompt)
        t_pkg, l_pkg = _decode(rt, prompt)
        assert t_pkg == t_ref
        assert np.array_equal(l_pkg, l_ref)
        # The draft from the package proposes what the synthetic draft proposes.
        ref.load_draft_synthetic(1, 3, 0.02, 0.0, MASK)
        rt.load_draft_package(root, MASK)
        a = ref.run_vlm_dflash_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                           prompt.vision_features, max_tokens=32)
        b = rt.run_vlm_dflash_with_prompt(prompt.input_ids, prompt.position_ids, prompt.image_token_id,
                                          prompt.vision_features, max_tokens=32)
        assert b.generated_tokens == a.generated_tokens and a.generated_tokens[:24] == t_ref   # lossless
        assert b.acceptance_lengths == a.acceptance_lengths


def test_fp16_package_matches_rounded_weights(pkg, oracle, tmp_path):
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    root = str(tmp_path / "pkg16")
    _writer().write_package(root, w, fp16=True)

    def r16(a):
        return a.astype(np.float16).astype(np.float32)

    for lw in w.layers:
        for k in ("q", "k", "v", "o", "gate", "up", "down"):
            setattr(lw, k, r16(getattr(lw, k)))
    w.embed = r16(w.embed)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    with pkg.TextRuntime.from_weights(w, num_layers=2, vocab_size=VOCAB, **CTX) as ref, \
            pkg.TextRuntime.from_package(root, **CTX) as rt:
        t_ref, l_ref = _decode(ref, prompt)
        t_pkg, l_pkg = _decode(rt, prompt)
    assert t_pkg == t_ref
    assert np.array_equal(l_pkg, l_ref)
