"""CPU checks of the C ABI: the library loads, exports every declared symbol, and
its host-side table builders match the reference's known answers. No device
work runs here."""

import ctypes
import glob
import os
import re

import numpy as np

from conftest import REPO


def _declared_symbols():
    """Every function declared in the C headers include/hy_*.h (the reference-facing
    hy_decode.h and hy_debug.h; hunyuan_ocr_cuda.h is the C++ layer over them)."""
    names = set()
    for path in glob.glob(os.path.join(REPO, "include", "hy_*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
        names.update(re.findall(r"\b(hy_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(pkg.LIB_PATH)
    declared = _declared_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert set(pkg.EXPORTED_SYMBOLS) == set(declared)


def test_version_and_config_defaults(pkg):
    lib = pkg.load_library()
    assert b"sm_100a" in lib.hy_version()
    cfg = pkg.default_config()
    assert (cfg.num_layers, cfg.vocab_size, cfg.ffn_dim) == (24, 120818, 3584)
    assert abs(cfg.attn_scale - 0.0883883) < 1e-8 and abs(cfg.rms_norm_eps - 1e-5) < 1e-11


def test_host_build_mrope_known_answer(pkg):
    # tests/text_rope_test.cpp:8-34, through the library's host builder.
    cos = pkg.build_mrope(np.array([978, 811, 621, 431], np.int32), 1, True)[0]
    dims = [0, 2, 31, 32, 63, 64, 95, 96, 127]
    want = [-0.569676042, -0.0682837293, 0.929675043, 0.970673621, 1.0, 0.510228872, 0.97144419, 0.991688073, 1.0]
    for d, w in zip(dims, want):
        assert abs(float(cos[d]) - w) <= 2e-7


def test_host_tables_match_oracle(pkg, oracle):
    prompt = oracle.synthetic_prompt(1, 3, 5, 7, 4096, 4093)
    seq = prompt.input_ids.shape[0]
    for use_cos in (True, False):
        a = pkg.build_mrope(prompt.position_ids, seq, use_cos)
        b = oracle.build_mrope(prompt.position_ids, seq, use_cos)
        assert np.max(np.abs(a - b)) <= 2e-7
        r = pkg.rope_rows(1000, 3, use_cos)
        assert np.max(np.abs(r - oracle.rope_rows(1000, 3, use_cos))) <= 2e-7


def test_invalid_arguments_report_errors(pkg):
    lib = pkg.load_library()
    assert lib.hy_build_mrope(None, 1, 1, None) == pkg.HY_ERR_INVALID_ARGUMENT
    assert b"invalid" in lib.hy_last_error()
    assert lib.hy_config_init(None) == pkg.HY_ERR_INVALID_ARGUMENT
