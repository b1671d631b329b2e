"""Long-context parity: the attention of every decode path at the KV lengths of
the attention-alone workload (1024 / 2048 / 4096 / 8192 cached rows, 1 and 16
query rows), against the oracle's PreciseSDPA (src/precise_sdpa.cpp:281-329).

The cache is preset with N(0,1) rows (hy_kv_write), as the attention-alone
workload fills it; the new rows are rotated with the 1-D RoPE at their
positions (rope_value, src/text_runtime.cpp:182-193). Cases:
  * hy_attention (the step path's attention kernels) at q = 1 and 16;
  * the persistent AR kernel (18 splits per KV head, partials merged by epoch
    words) decoding 20 tokens of a 2-layer model: tokens and raw top-1
    bit-exact, and the K/V rows it appends (layer 1's depend on layer 0's
    attention output) within the fp32 tolerance;
  * one DFlash verify block (16 rows): posterior and acceptance bit-exact.

Tolerances: ids exact; activations 2e-4 absolute / 1e-4 relative (fp32
accumulation against the oracle's fp64 attention and BLAS order).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED, NORM_STD = 11, 0.1
LONG = dict(num_layers=2, vocab_size=4096, max_context=8192 + 64, max_prefill=64, max_tokens=64)
ATOL, RTOL = 2e-4, 1e-4


@pytest.fixture(scope="module")
def long_rt(pkg, oracle):
    cfg = oracle.ModelConfig(num_layers=2, vocab=4096)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    rt = pkg.TextRuntime.synthetic(seed=SEED, std=0.02, norm_std=NORM_STD, device=0, **LONG)
    yield cfg, w, rt
    rt.close()


def _preset_cache(oracle, rt, past, rng, capacity):
    """Random N(0,1) K/V rows [0, past) in both layers, on the device and in an oracle cache."""
    rt.reset()
    cache = oracle.KVCache.empty(2, capacity)
    for li in range(2):
        k = rng.standard_normal((8, past, 128)).astype(np.float32)
        v = rng.standard_normal((8, past, 128)).astype(np.float32)
        rt.kv_write(li, 0, k, v)
        cache.k[li][:, :past] = k
        cache.v[li][:, :past] = v
    cache.length = past
    rt.set_length(past)
    return cache


@pytest.mark.parametrize("rows", [1, 16])
@pytest.mark.parametrize("past", [1024, 4096, 8192])
def test_attention_long_context(long_rt, oracle, rows, past):
    cfg, w, rt = long_rt
    rng = np.random.default_rng(7 * past + rows)
    rt.reset()
    kpast = rng.standard_normal((8, past, 128)).astype(np.float32)
    vpast = rng.standard_normal((8, past, 128)).astype(np.float32)
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


@pytest.mark.parametrize("past", [2048, 4096, 8192])
def test_persistent_ar_long_context(pkg, long_rt, oracle, past):
    cfg, w, rt = long_rt
    n = 20
    rng = np.random.default_rng(past)
    cache = _preset_cache(oracle, rt, past, rng, past + n + 16)
    history = rng.integers(0, cfg.vocab, 200).tolist()
    first = int(rng.integers(0, cfg.vocab))
    rt.set_history(history)
    assert rt.ar_path == pkg.AR_PATH_PERSISTENT
    toks, raw = rt.generate(first, first, n, 1.08)
    want = oracle.decode_from_cache(w, cfg, cache, first, n, history, 1.08)
    mism = [i for i, (a, b) in enumerate(zip(toks, want.tokens)) if a != b]
    assert not mism, f"first mismatch at token {mism[0]}, oracle top-2 margin {want.margins[mism[0] - 1]:.3g}"
    assert raw == want.raw_top1
    assert rt.kv_length == past + n - 1
    for li in range(2):
        k, v = rt.kv_read(li, past, n - 1)
        np.testing.assert_allclose(k, cache.k[li][:, past:past + n - 1], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(v, cache.v[li][:, past:past + n - 1], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("past", [2048, 8192])
def test_verify_block_long_context(long_rt, oracle, past):
    cfg, w, rt = long_rt
    rng = np.random.default_rng(past + 1)
    cache = _preset_cache(oracle, rt, past, rng, past + 32)
    history = rng.integers(0, cfg.vocab, 100).tolist()
    rt.set_history(history)
    # Proposals: the oracle's greedy continuation for the first rows, then noise,
    # so that the acceptance length is neither 0 nor 15.
    greedy = oracle.decode_from_cache(w, cfg, oracle.KVCache([k.copy() for k in cache.k], [v.copy() for v in cache.v],
                                                             past), int(rng.integers(0, cfg.vocab)), 6, history)
    proposed = greedy.tokens + rng.integers(0, cfg.vocab, 16 - len(greedy.tokens)).tolist()
    post_ref, acc_ref, _, _ = oracle.verify_block(w, cfg, cache, proposed, history, 1.08)
    post, acc, committed, stop = rt.dflash_verify_block(proposed, 16, 1.08)
    assert post == post_ref
    assert acc == acc_ref and acc >= 4
    assert committed == acc + 1 and not stop
    assert rt.kv_length == past + committed
    for li in range(2):
        k, v = rt.kv_read(li, past, committed)
        np.testing.assert_allclose(k, cache.k[li][:, past:past + committed], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(v, cache.v[li][:, past:past + committed], rtol=RTOL, atol=ATOL)
