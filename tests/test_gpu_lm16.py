"""The 16-row LM head at the full vocabulary (120818 rows of the tied table,
read in 128-row TMA tiles; each CTA's share spans several tiles and the last
tiles run past the table, where the copy fills zeros) against the oracle:
run_lm_head + select_logit_rows (src/text_runtime.cpp:430-439, 757-797).

Tolerance: logits within 2e-4 absolute / 1e-4 relative (fp32 and the bf16
variant, where the oracle uses the bf16-rounded table); token ids and raw top-1
bit-exact.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-4, 1e-4
SEED, NORM_STD = 11, 0.1


@pytest.mark.parametrize("bf16", [False, True])
def test_full_vocab_lm_head_16_rows(pkg, oracle, bf16):
    cfg = oracle.ModelConfig(num_layers=1)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD, bf16=bf16)
    dt = 1 if bf16 else 0
    with pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, num_layers=1, max_prefill=32,
                                   max_tokens=32, max_context=256, weight_dtype=dt, kv_dtype=dt) as rt:
        rng = np.random.default_rng(7 + dt)
        for rows in (16, 5):
            h = rng.standard_normal((rows, 1024)).astype(np.float32)
            ref = oracle.lm_head(w, h)
            hist = rng.integers(0, cfg.vocab, 400).tolist() + [int(np.argmax(ref[r])) for r in range(rows)]
            prefix = rng.integers(0, cfg.vocab, rows).tolist()
            rt.set_history(hist)
            tok, raw, logits = rt.select_logit_rows(h, 1.08, row_prefix=prefix, want_logits=True)
            np.testing.assert_allclose(logits, ref, rtol=RTOL, atol=ATOL)
            assert tok.tolist() == oracle.select_logit_rows(ref, hist, prefix, 1.08)
            assert raw.tolist() == [int(np.argmax(ref[r])) for r in range(rows)]
