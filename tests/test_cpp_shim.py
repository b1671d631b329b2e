"""The C++17 layer over the C ABI (include/hunyuan_ocr_cuda.h: hunyuan_ocr::cuda::TextRuntime,
RuntimeOptions, the result / timing types, detail::run_decoder_step), through its compiled test
program tests/cpp/test_shim.cpp (built by __graft_entry__.build())."""

import importlib.util
import os
import subprocess

import pytest

from conftest import REPO

BIN = os.path.join(REPO, "tests", "cpp", "test_shim")
VOCAB, SEED, NORM_STD = 4096, 11, 0.1
MASK = VOCAB - 1


@pytest.fixture(scope="module")
def shim(pkg):
    assert os.path.exists(BIN), "tests/cpp/test_shim was not built by build()"
    return BIN


def test_shim_host_checks(shim):
    out = subprocess.run([shim, "host"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "host ok" in out.stdout


@pytest.mark.gpu
def test_shim_decodes_a_package_like_the_python_path(pkg, oracle, shim, tmp_path):
    spec = importlib.util.spec_from_file_location("hy_ncnn_package",
                                                  os.path.join(REPO, "hunyuanocr-ncnn_b200", "ncnn_package.py"))
    writer = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(writer)
    cfg = oracle.ModelConfig(num_layers=2, vocab=VOCAB)
    w = oracle.make_weights(cfg, SEED, 0.02, NORM_STD)
    dw = oracle.make_draft_weights(1, 3, 0.02, 0.0)
    root, fx = str(tmp_path / "pkg"), str(tmp_path / "fixture")
    writer.write_package(root, w, draft=dw)
    prompt = oracle.synthetic_prompt(21, 4, 6, 16, VOCAB, VOCAB - 3)
    pkg.write_vlm_fixture(fx, prompt.input_ids, prompt.position_ids, prompt.image_token_id, prompt.vision_features,
                          [0])
    out = subprocess.run([shim, "decode", root, fx, "dflash", str(MASK)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = {ln.split()[0]: ln.split()[1:] for ln in out.stdout.splitlines() if ln.strip()}
    want = oracle.decode_ar(w, cfg, prompt, 24).tokens
    assert [int(t) for t in lines["ar"]] == want
    assert [int(t) for t in lines["dflash"]] == want   # lossless
    blocks, drafted, accepted = int(lines["blocks"][0]), int(lines["blocks"][2]), int(lines["blocks"][4])
    assert blocks > 0 and drafted == 15 * blocks and 0 <= accepted <= drafted
