"""The regression-fixture reader (CPU, host code of the library): the reference's
fixture directory format (src/text_runtime.cpp:253-381; written by
tools/prepare_regression_fixtures.py) and its error messages."""

import os

import numpy as np
import pytest


def _fixture(pkg, tmp_path, seq=7, vis=3, n_exp=5):
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 1000, seq).astype(np.int32)
    pos = rng.integers(0, 50, (4, seq)).astype(np.int32)
    feats = rng.standard_normal((vis, 1024)).astype(np.float32)
    exp = rng.integers(0, 1000, n_exp).astype(np.int32)
    d = str(tmp_path / "case")
    pkg.write_vlm_fixture(d, ids, pos, 999, feats, exp)
    return d, ids, pos, feats, exp


def test_fixture_round_trip(pkg, tmp_path):
    d, ids, pos, feats, exp = _fixture(pkg, tmp_path)
    with open(os.path.join(d, "meta.txt"), "a") as f:
        f.write("case=synthetic\nsafety_max_tokens=64\n")   # extra keys are ignored
    fx = pkg.read_vlm_fixture(d)
    assert (fx.seq_len, fx.image_token_id, fx.vision_token_count) == (7, 999, 3)
    assert np.array_equal(fx.input_ids, ids) and np.array_equal(fx.position_ids, pos)
    assert np.array_equal(fx.expected_tokens, exp) and np.array_equal(fx.vision_features, feats)
    os.remove(os.path.join(d, "vision_features.f32"))
    assert pkg.read_vlm_fixture(d, with_features=False).vision_features is None


@pytest.mark.parametrize("case", ["no_meta", "bad_value", "missing_key", "short", "extra", "no_features"])
def test_fixture_errors(pkg, tmp_path, case):
    d, ids, pos, feats, exp = _fixture(pkg, tmp_path)
    want = {"no_meta": "failed to open fixture meta", "bad_value": "invalid fixture meta value",
            "missing_key": "must define positive", "short": "short read", "extra": "unexpected extra bytes",
            "no_features": "failed to open"}[case]
    meta = os.path.join(d, "meta.txt")
    if case == "no_meta":
        os.remove(meta)
    elif case == "bad_value":
        with open(meta, "a") as f:
            f.write("seq_len=abc\n")
    elif case == "missing_key":
        with open(meta, "w") as f:
            f.write("seq_len=7\nexpected_token_count=5\nimage_token_id=999\n")
    elif case == "short":
        ids[:-1].tofile(os.path.join(d, "input_ids.i32"))
    elif case == "extra":
        np.concatenate([exp, exp[:1]]).tofile(os.path.join(d, "expected_tokens.i32"))
    else:
        os.remove(os.path.join(d, "vision_features.f32"))
    with pytest.raises(pkg.HyError) as e:
        pkg.read_vlm_fixture(d)
    assert e.value.status == pkg.HY_ERR_INVALID_ARGUMENT and want in e.value.message


def test_fixture_load_checks_buffer_capacity(pkg, tmp_path):
    """A meta.txt that asks for more than the caller's buffers hold fails before any write."""
    import ctypes
    d, ids, pos, feats, exp = _fixture(pkg, tmp_path)
    lib = pkg.load_library()
    seq = ids.size - 1                      # buffers sized one row short of meta.txt's seq_len
    b_ids = np.full(seq, -7, np.int32)
    b_pos = np.full((4, seq), -7, np.int32)
    b_exp = np.full(exp.size, -7, np.int32)
    b_feat = np.zeros((feats.shape[0], 1024), np.float32)
    rc = lib.hy_fixture_load(os.fsencode(d), seq, exp.size, feats.shape[0], b_ids.ctypes.data, b_pos.ctypes.data,
                             b_exp.ctypes.data, b_feat.ctypes.data)
    assert rc == pkg.HY_ERR_CAPACITY
    assert b"seq_len=7" in lib.hy_last_error()
    assert (b_ids == -7).all() and (b_pos == -7).all() and (b_exp == -7).all()
    rc = lib.hy_fixture_load(os.fsencode(d), ids.size, exp.size, feats.shape[0] - 1, b_ids.ctypes.data,
                             b_pos.ctypes.data, b_exp.ctypes.data, b_feat.ctypes.data)
    assert rc == pkg.HY_ERR_CAPACITY
    del ctypes
