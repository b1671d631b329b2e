"""The model-package reader (host code of the library, no device work): packages in the
layout of the reference's exported ncnn files (models/README.md), written by
hunyuanocr-ncnn_b200/ncnn_package.py from seeded weights, read back through
hy_package_inspect / hy_package_read_tensor - every weight as written, in each storage
variant an export may produce - and its error messages for damaged packages."""

import importlib.util
import os

import numpy as np
import pytest

from conftest import REPO

LAYERS, VOCAB, FFN = 2, 512, 256
FIELDS = {"input_norm": "input_norm", "q_proj": "q", "k_proj": "k", "v_proj": "v", "query_norm": "q_norm",
          "key_norm": "k_norm", "o_proj": "o", "post_norm": "post_norm", "gate_proj": "gate", "up_proj": "up",
          "down_proj": "down"}


def _writer():
    spec = importlib.util.spec_from_file_location("hy_ncnn_package",
                                                  os.path.join(REPO, "hunyuanocr-ncnn_b200", "ncnn_package.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def weights(oracle):
    cfg = oracle.ModelConfig(num_layers=LAYERS, vocab=VOCAB, ffn=FFN)
    return oracle.make_weights(cfg, 7, 0.02, 0.1), oracle.make_draft_weights(1, 9, 0.02, 0.1, ffn=FFN)


def _check_all(pkg, root, w, dw=None, rnd=lambda a: a):
    assert np.array_equal(pkg.package_tensor(root, "embed"), rnd(w.embed).reshape(-1))
    assert np.array_equal(pkg.package_tensor(root, "final_norm"), w.final_norm.reshape(-1))
    for li, lw in enumerate(w.layers):
        for field, attr in FIELDS.items():
            want = getattr(lw, attr)
            want = want if want.ndim == 1 else rnd(want)   # norms are stored as raw fp32
            assert np.array_equal(pkg.package_tensor(root, field, li), want.reshape(-1)), (li, field)
    if dw is not None:
        assert np.array_equal(pkg.package_tensor(root, "fc", draft=True), rnd(dw.fc).reshape(-1))
        assert np.array_equal(pkg.package_tensor(root, "hidden_norm", draft=True), dw.hidden_norm)
        assert np.array_equal(pkg.package_tensor(root, "norm", draft=True), dw.norm)
        for field, attr in FIELDS.items():
            want = getattr(dw.layers[0], attr)
            want = want if want.ndim == 1 else rnd(want)
            assert np.array_equal(pkg.package_tensor(root, field, 0, draft=True), want.reshape(-1)), field


@pytest.mark.parametrize("linear,norm", [("gemm", "rmsnorm"), ("innerproduct", "memorydata")])
def test_package_round_trip_fp32(pkg, weights, tmp_path, linear, norm):
    w, dw = weights
    root = str(tmp_path / "pkg")
    _writer().write_package(root, w, draft=dw, linear=linear, norm=norm)
    assert pkg.package_inspect(root) == {"num_layers": LAYERS, "vocab_size": VOCAB, "ffn_dim": FFN, "draft_layers": 1}
    _check_all(pkg, root, w, dw)
    # The embedding's table is stored once; the LM head's param points at it.
    assert os.path.exists(os.path.join(root, "lm_head", "lm_head.ncnn.param"))
    assert not os.path.exists(os.path.join(root, "lm_head", "lm_head.ncnn.bin"))


def test_package_fp16_storage(pkg, weights, tmp_path):
    w, dw = weights
    root = str(tmp_path / "pkg16")
    _writer().write_package(root, w, draft=dw, fp16=True)
    _check_all(pkg, root, w, dw, rnd=lambda a: a.astype(np.float16).astype(np.float32))


def _damage(root, what):
    dec = os.path.join(root, "text_decoder")
    param, binf = os.path.join(dec, "text_decoder_kv.ncnn.param"), os.path.join(dec, "text_decoder_kv.ncnn.bin")
    if what == "short":
        data = open(binf, "rb").read()
        open(binf, "wb").write(data[:-8])
    elif what == "extra":
        open(binf, "ab").write(b"\0" * 16)
    elif what == "magic":
        text = open(param).read()
        open(param, "w").write(text.replace("7767517", "7767518", 1))
    elif what == "missing":
        text = open(param).read()
        open(param, "w").write(text.replace("layers.1.self_attn.q_proj ", "layers.1.self_attn.qq_proj", 1))
    elif what == "shape":
        text = open(param).read()   # q_proj declared with N and K swapped: same byte count, wrong shape
        open(param, "w").write(text.replace("layers.0.self_attn.q_proj", "layers.0.self_attn.o_proj_x", 1)
                               .replace("layers.0.self_attn.o_proj ", "layers.0.self_attn.q_proj ", 1)
                               .replace("layers.0.self_attn.o_proj_x", "layers.0.self_attn.o_proj", 1))
    elif what == "tag":
        data = bytearray(open(binf, "rb").read())
        # The first tagged array follows the first RMSNorm gamma (1024 raw floats).
        data[4096:4100] = np.uint32(0x000D4B38).tobytes()
        open(binf, "wb").write(bytes(data))


@pytest.mark.parametrize("what,status,message", [
    ("short", 1, "shorter than its param file"), ("extra", 1, "bytes left after the last weight"),
    ("magic", 1, "not an ncnn param file"), ("missing", 1, "no weight for layers.1.q_proj"),
    ("shape", 1, "expected 2048 x 1024"), ("tag", 7, "storage tag 0x000D4B38")])
def test_package_errors(pkg, weights, tmp_path, what, status, message):
    w, _ = weights
    root = str(tmp_path / "bad")
    _writer().write_package(root, w)
    _damage(root, what)
    with pytest.raises(pkg.HyError) as e:
        pkg.package_inspect(root)
    assert e.value.status == status and message in e.value.message, e.value.message


def test_package_missing_directory(pkg, tmp_path):
    with pytest.raises(pkg.HyError) as e:
        pkg.package_inspect(str(tmp_path / "nothing"))
    assert "failed to open model file" in e.value.message
