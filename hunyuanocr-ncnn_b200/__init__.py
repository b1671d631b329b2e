"""Python host binding of the B200 text-decode library (ctypes over include/hy_decode.h).

The library itself is C++/CUDA (``csrc/``), built in-tree into
``libhy_decode.so``. This module only marshals numpy arrays across the C ABI
and mirrors the names of the reference's text runtime
(src/text_runtime.cpp, include/hunyuan_ocr/text_runtime.h) so that host code
and tests read like the reference's: ``TextRuntime.run_vlm_decode_with_prompt``,
``run_decoder_step``, ``select_logit_rows``, ``dflash_verify_block``.

Errors follow the reference's convention of a message per failing call: a
non-zero status raises ``HyError`` carrying ``hy_last_error()``. There is no
CPU fallback: importing this module without the built library raises.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhy_decode.so")

HY_OK = 0
HY_ERR_INVALID_ARGUMENT = 1
HY_ERR_CUDA = 2
HY_ERR_OUT_OF_MEMORY = 3
HY_ERR_CAPACITY = 4
HY_ERR_DEVICE_TIMEOUT = 5
HY_ERR_NOT_READY = 6
HY_ERR_UNSUPPORTED = 7
DTYPE_F32 = 0
DTYPE_BF16 = 1
HIDDEN = 1024
HEAD_DIM = 128
QKV_WIDTH = 4096
DFLASH_BLOCK = 16

EXPORTED_SYMBOLS = (
    "hy_version", "hy_last_error", "hy_config_init", "hy_ctx_create", "hy_ctx_create_synthetic",
    "hy_ctx_destroy", "hy_ctx_config", "hy_ctx_device_bytes", "hy_build_mrope", "hy_rope_value",
    "hy_seq_reset", "hy_seq_length", "hy_seq_truncate", "hy_history_set", "hy_history_add",
    "hy_prefill", "hy_decoder_step", "hy_lm_head_select", "hy_generate", "hy_verify_block",
    "hy_dflash_generate_synthetic", "hy_run_vlm_decode_with_prompt", "hy_attention", "hy_kv_write",
    "hy_kv_read", "hy_seq_set_length", "hy_bench_ar_steps", "hy_bench_kernel", "hy_ctx_stream",
    "hy_ctx_set_ar_path", "hy_ctx_ar_path", "hy_trace_persistent", "hy_debug_progress",
    "hy_lm_head_select_noalloc", "hy_draft_load", "hy_draft_load_synthetic", "hy_draft_context_length",
    "hy_draft_context_append", "hy_draft_run", "hy_draft_propose", "hy_dflash_generate",
    "hy_run_vlm_dflash_with_prompt", "hy_batch_decode", "hy_fixture_meta", "hy_fixture_load",
    "hy_ctx_set_token_callback", "hy_debug_wait_stats", "hy_ctx_last_timing", "hy_ctx_last_dflash_timing",
    "hy_ctx_set_wait_limit", "hy_debug_wait_probe", "hy_ctx_create_from_package", "hy_draft_load_package",
    "hy_package_inspect", "hy_package_read_tensor", "hy_debug_step_trace",
)
TOKEN_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_void_p)
DFLASH_MASK_TOKEN = 120817
AR_PATH_PERSISTENT = 0
AR_PATH_GRAPH = 1


class HyError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"hy status {status}: {message}")
        self.status = status
        self.message = message


class Config(ctypes.Structure):
    _fields_ = [
        ("num_layers", ctypes.c_int), ("vocab_size", ctypes.c_int), ("ffn_dim", ctypes.c_int),
        ("max_context", ctypes.c_int), ("max_prefill", ctypes.c_int), ("max_tokens", ctypes.c_int),
        ("weight_dtype", ctypes.c_int), ("kv_dtype", ctypes.c_int), ("rms_norm_eps", ctypes.c_float),
        ("attn_scale", ctypes.c_float), ("device", ctypes.c_int),
    ]


class _LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_norm", "q_proj", "k_proj", "v_proj", "query_norm", "key_norm", "o_proj", "post_norm",
        "gate_proj", "up_proj", "down_proj")]


class _DraftWeights(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int), ("mask_token", ctypes.c_int), ("fc", ctypes.c_void_p),
                ("hidden_norm", ctypes.c_void_p), ("norm", ctypes.c_void_p),
                ("layers", ctypes.POINTER(_LayerWeights))]


class _Request(ctypes.Structure):
    _fields_ = [("input_ids", ctypes.c_void_p), ("position_ids", ctypes.c_void_p), ("seq_len", ctypes.c_int),
                ("image_token_id", ctypes.c_int), ("vision_features", ctypes.c_void_p),
                ("vision_token_count", ctypes.c_int)]


class _DecodeTiming(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("text_embed_ms", "prefill_ms", "decode_ms", "lm_head_ms",
                                                "token_select_ms", "total_ms", "host_overhead_ms")]


class _DFlashTiming(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("prefill_ms", "draft_ms", "verify_ms", "commit_ms", "blocks_ms",
                                                "total_ms", "host_overhead_ms")] + [
        (n, ctypes.c_int) for n in ("block_count", "drafted_token_count", "accepted_draft_token_count")]


class _Weights(ctypes.Structure):
    _fields_ = [("embed", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("layers", ctypes.POINTER(_LayerWeights))]


_LIB = None
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libhy_decode.so (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing; build it with `python __graft_entry__.py build` "
                          "(there is no CPU fallback for the decode path)")
    lib = ctypes.CDLL(path)
    sig = {
        "hy_version": ([], ctypes.c_char_p),
        "hy_last_error": ([], ctypes.c_char_p),
        "hy_config_init": ([ctypes.POINTER(Config)], _I),
        "hy_ctx_create": ([ctypes.POINTER(Config), ctypes.POINTER(_Weights), ctypes.POINTER(_P)], _I),
        "hy_ctx_create_synthetic": ([ctypes.POINTER(Config), ctypes.c_uint64, _F, _F, ctypes.POINTER(_P)], _I),
        "hy_ctx_destroy": ([_P], None),
        "hy_ctx_config": ([_P, ctypes.POINTER(Config)], _I),
        "hy_ctx_device_bytes": ([_P], ctypes.c_size_t),
        "hy_ctx_stream": ([_P], _P),
        "hy_build_mrope": ([_P, _I, _I, _P], _I),
        "hy_rope_value": ([_I, _I, _I], _F),
        "hy_seq_reset": ([_P], _I),
        "hy_seq_length": ([_P, ctypes.POINTER(_I)], _I),
        "hy_seq_truncate": ([_P, _I], _I),
        "hy_seq_set_length": ([_P, _I], _I),
        "hy_history_set": ([_P, _P, _I], _I),
        "hy_history_add": ([_P, _P, _I], _I),
        "hy_prefill": ([_P, _P, _P, _P, _I, _P, _P], _I),
        "hy_decoder_step": ([_P, _P, _I, _P, _P, _P, _P], _I),
        "hy_lm_head_select": ([_P, _P, _I, _P, _F, _P, _P, _P], _I),
        "hy_lm_head_select_noalloc": ([_P, _P, _I, _F, _P, _P], _I),
        "hy_generate": ([_P, _I, _I, _I, _F, _P, _I, _P, _P, ctypes.POINTER(_I)], _I),
        "hy_verify_block": ([_P, _P, _I, _F, _P, _I, _P, ctypes.POINTER(_I), ctypes.POINTER(_I),
                             ctypes.POINTER(_I)], _I),
        "hy_dflash_generate_synthetic": ([_P, _I, _I, _F, _P, _I, _P, _I, _F, ctypes.c_uint64, _P,
                                          ctypes.POINTER(_I), _P, ctypes.POINTER(_I)], _I),
        "hy_run_vlm_decode_with_prompt": ([_P, _P, _P, _I, _I, _P, _I, _I, _F, _P, _I, _P, _P,
                                           ctypes.POINTER(_I)], _I),
        "hy_attention": ([_P, _I, _P, _I, _P, _P, _P], _I),
        "hy_kv_write": ([_P, _I, _I, _I, _P, _P], _I),
        "hy_kv_read": ([_P, _I, _I, _I, _P, _P], _I),
        "hy_bench_ar_steps": ([_P, _I, ctypes.POINTER(_F)], _I),
        "hy_bench_kernel": ([_P, _I, _I, ctypes.POINTER(_F)], _I),
        "hy_ctx_set_ar_path": ([_P, _I], _I),
        "hy_ctx_ar_path": ([_P], _I),
        "hy_trace_persistent": ([_P, _I, _I, _P], _I),
        "hy_draft_load": ([_P, ctypes.POINTER(_DraftWeights)], _I),
        "hy_batch_decode": ([_P, ctypes.POINTER(_Request), _I, _I, _I, _F, _P, _I, _P, _P, _P], _I),
        "hy_fixture_meta": ([ctypes.c_char_p, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                             ctypes.POINTER(_I)], _I),
        "hy_fixture_load": ([ctypes.c_char_p, _I, _I, _I, _P, _P, _P, _P], _I),
        "hy_ctx_set_token_callback": ([_P, TOKEN_CALLBACK, _P, _I], _I),
        "hy_draft_load_synthetic": ([_P, _I, _I, ctypes.c_uint64, _F, _F], _I),
        "hy_draft_context_length": ([_P, ctypes.POINTER(_I)], _I),
        "hy_draft_context_append": ([_P, _P, _I], _I),
        "hy_draft_run": ([_P, _P, _P], _I),
        "hy_draft_propose": ([_P, _I, _P], _I),
        "hy_dflash_generate": ([_P, _I, _I, _F, _P, _I, _P, ctypes.POINTER(_I), _P, ctypes.POINTER(_I)], _I),
        "hy_run_vlm_dflash_with_prompt": ([_P, _P, _P, _I, _I, _P, _I, _I, _F, _P, _I, _P, ctypes.POINTER(_I), _P,
                                           ctypes.POINTER(_I)], _I),
        "hy_debug_progress": ([_P, _P, _I], _I),
        "hy_debug_wait_stats": ([_P, _P, _I, _I], _I),
        "hy_debug_step_trace": ([_P, _P, _I, _P, _I], _I),
        "hy_ctx_create_from_package": ([ctypes.POINTER(Config), ctypes.c_char_p, ctypes.POINTER(_P)], _I),
        "hy_draft_load_package": ([_P, ctypes.c_char_p, _I], _I),
        "hy_package_inspect": ([ctypes.c_char_p, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                                ctypes.POINTER(_I)], _I),
        "hy_package_read_tensor": ([ctypes.c_char_p, _I, _I, ctypes.c_char_p, _P, ctypes.c_size_t,
                                    ctypes.POINTER(ctypes.c_size_t)], _I),
        "hy_ctx_set_wait_limit": ([_P, ctypes.c_uint64], _I),
        "hy_debug_wait_probe": ([_P, _I, ctypes.c_uint64], _I),
        "hy_ctx_last_timing": ([_P, ctypes.POINTER(_DecodeTiming)], _I),
        "hy_ctx_last_dflash_timing": ([_P, ctypes.POINTER(_DFlashTiming)], _I),
    }
    for name, (argtypes, restype) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _LIB = lib
    return lib


def _check(status: int) -> None:
    if status != HY_OK:
        raise HyError(status, _LIB.hy_last_error().decode(errors="replace"))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def default_config(**overrides) -> Config:
    lib = load_library()
    cfg = Config()
    _check(lib.hy_config_init(ctypes.byref(cfg)))
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def package_inspect(model_root: str) -> dict:
    """Geometry of a model package (the reference's exported ncnn files), read on the host."""
    lib = load_library()
    n, v, f, d = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _check(lib.hy_package_inspect(os.fsencode(model_root), ctypes.byref(n), ctypes.byref(v), ctypes.byref(f),
                                  ctypes.byref(d)))
    return {"num_layers": n.value, "vocab_size": v.value, "ffn_dim": f.value, "draft_layers": d.value}


def package_tensor(model_root: str, field: str, layer: int = -1, draft: bool = False) -> np.ndarray:
    """One weight of a package as the library's reader sees it (fp16 storage converted)."""
    lib = load_library()
    n = ctypes.c_size_t()
    root, f = os.fsencode(model_root), field.encode()
    _check(lib.hy_package_read_tensor(root, int(draft), layer, f, None, 0, ctypes.byref(n)))
    out = np.empty(n.value, np.float32)
    _check(lib.hy_package_read_tensor(root, int(draft), layer, f, _ptr(out), out.size, ctypes.byref(n)))
    return out


def build_mrope(position_ids: np.ndarray, seq_len: int, use_cos: bool) -> np.ndarray:
    """detail::build_mrope (src/text_runtime.cpp:42-63), evaluated by the library's host code."""
    lib = load_library()
    pos = _i32(position_ids).reshape(-1)
    out = np.empty((seq_len, HEAD_DIM), np.float32)
    _check(lib.hy_build_mrope(_ptr(pos), seq_len, int(use_cos), _ptr(out)))
    return out


def rope_rows(start: int, rows: int, use_cos: bool) -> np.ndarray:
    """build_decode_rope / build_verify_rope (src/text_runtime.cpp:228-251) via rope_value."""
    lib = load_library()
    out = np.empty((rows, HEAD_DIM), np.float32)
    for r in range(rows):
        for d in range(HEAD_DIM):
            out[r, d] = lib.hy_rope_value(start + r, d, int(use_cos))
    return out


@dataclass
class TextDecodeTiming:
    """include/hunyuan_ocr/text_runtime.h:32-39 (device stages from CUDA events; the LM head of
    every token after the first and all token selection are fused into decode_ms), plus
    host_overhead_ms = total_ms minus the device stages."""
    text_embed_ms: float = 0.0
    prefill_ms: float = 0.0
    decode_ms: float = 0.0
    lm_head_ms: float = 0.0
    token_select_ms: float = 0.0
    total_ms: float = 0.0
    host_overhead_ms: float = 0.0


@dataclass
class DFlashDecodeTiming:
    """include/hunyuan_ocr/text_runtime.h:64-74 in three device stages per block (draft =
    draft_prepare + draft_infer + draft_postprocess; verify = verify_prepare + verify_infer;
    commit = verify_postprocess + commit), plus blocks_ms and host_overhead_ms."""
    prefill_ms: float = 0.0
    draft_ms: float = 0.0
    verify_ms: float = 0.0
    commit_ms: float = 0.0
    blocks_ms: float = 0.0
    total_ms: float = 0.0
    host_overhead_ms: float = 0.0


@dataclass
class TextDecodeResult:
    """include/hunyuan_ocr/text_runtime.h:41-51 (the fields this path fills)."""
    seq_len: int
    repetition_penalty: float
    generated_tokens: list
    raw_top1_tokens: list
    checked_tokens: int = 0
    expected_tokens: list = field(default_factory=list)
    timing: TextDecodeTiming = field(default_factory=TextDecodeTiming)

    def matches_expected(self) -> bool:
        """TextDecodeResult::matches_expected (src/text_runtime.cpp:1788-1791)."""
        return self.generated_tokens == self.expected_tokens


@dataclass
class DFlashDecodeResult:
    """include/hunyuan_ocr/text_runtime.h:76-83 (counts as the library reports them)."""
    generated_tokens: list
    block_count: int
    drafted_token_count: int
    accepted_draft_token_count: int
    acceptance_lengths: list
    expected_tokens: list = field(default_factory=list)
    timing: DFlashDecodeTiming = field(default_factory=DFlashDecodeTiming)

    def matches_expected(self) -> bool:
        return self.generated_tokens == self.expected_tokens


@dataclass
class VlmFixture:
    """VlmFixtureInputs + vision features (src/text_runtime.cpp:278-381): one regression
    fixture directory (meta.txt, input_ids.i32, position_ids.i32, expected_tokens.i32,
    vision_features.f32)."""
    seq_len: int
    image_token_id: int
    vision_token_count: int
    input_ids: np.ndarray
    position_ids: np.ndarray
    expected_tokens: np.ndarray
    vision_features: np.ndarray | None


def read_vlm_fixture(fixture_dir: str, with_features: bool = True) -> VlmFixture:
    """load_vlm_fixture_with_features through the library's host reader (the reference's
    sizes, checks and messages: "failed to open", "short read", "unexpected extra bytes")."""
    lib = load_library()
    d = os.fsencode(fixture_dir)
    seq, exp, img, vis = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _check(lib.hy_fixture_meta(d, ctypes.byref(seq), ctypes.byref(exp), ctypes.byref(img), ctypes.byref(vis)))
    ids = np.empty(seq.value, np.int32)
    pos = np.empty((4, seq.value), np.int32)
    expected = np.empty(exp.value, np.int32)
    feats = np.empty((vis.value, HIDDEN), np.float32) if with_features else None
    _check(lib.hy_fixture_load(d, ids.size, expected.size, 0 if feats is None else feats.shape[0], _ptr(ids),
                               _ptr(pos), _ptr(expected), _ptr(feats)))
    return VlmFixture(seq.value, img.value, vis.value, ids, pos, expected, feats)


def write_vlm_fixture(fixture_dir: str, input_ids, position_ids, image_token_id: int, vision_features,
                      expected_tokens) -> None:
    """Writes a fixture directory in the reference's format (tools/prepare_regression_fixtures.py:
    little-endian int32 / float32 arrays and meta.txt with the four sizes)."""
    os.makedirs(fixture_dir, exist_ok=True)
    ids = _i32(input_ids).reshape(-1)
    feats = _f32(vision_features).reshape(-1, HIDDEN)
    exp = _i32(expected_tokens).reshape(-1)
    ids.astype("<i4").tofile(os.path.join(fixture_dir, "input_ids.i32"))
    _i32(position_ids).reshape(4, ids.size).astype("<i4").tofile(os.path.join(fixture_dir, "position_ids.i32"))
    exp.astype("<i4").tofile(os.path.join(fixture_dir, "expected_tokens.i32"))
    feats.astype("<f4").tofile(os.path.join(fixture_dir, "vision_features.f32"))
    with open(os.path.join(fixture_dir, "meta.txt"), "w") as f:
        f.write(f"seq_len={ids.size}\nexpected_token_count={exp.size}\nimage_token_id={int(image_token_id)}\n"
                f"vision_token_count={feats.shape[0]}\n")


class TextRuntime:
    """One device context: weights, KV cache and decode state on one GPU.

    Mirrors hunyuan_ocr::TextRuntime (include/hunyuan_ocr/text_runtime.h:85-158)
    for the text-decode path, over the C ABI in include/hy_decode.h.
    """

    def __init__(self, ctx, cfg: Config):
        self._ctx = ctx
        self.cfg = cfg

    # -- construction ------------------------------------------------------
    @classmethod
    def synthetic(cls, seed: int = 0, std: float = 0.02, norm_std: float = 0.0, **cfg_overrides) -> "TextRuntime":
        lib = load_library()
        cfg = default_config(**cfg_overrides)
        ctx = ctypes.c_void_p()
        _check(lib.hy_ctx_create_synthetic(ctypes.byref(cfg), seed, std, norm_std, ctypes.byref(ctx)))
        return cls(ctx, cfg)

    @classmethod
    def from_weights(cls, weights, **cfg_overrides) -> "TextRuntime":
        """weights: an object with .embed, .final_norm and .layers[i].{input_norm, q, k, v, q_norm,
        k_norm, o, post_norm, gate, up, down} numpy fp32 arrays (nn.Linear layout)."""
        lib = load_library()
        cfg = default_config(**cfg_overrides)
        keep = []

        def p(a):
            a = _f32(a)
            keep.append(a)
            return a.ctypes.data

        layers = (_LayerWeights * cfg.num_layers)()
        for i, lw in enumerate(weights.layers[:cfg.num_layers]):
            layers[i] = _LayerWeights(p(lw.input_norm), p(lw.q), p(lw.k), p(lw.v), p(lw.q_norm), p(lw.k_norm),
                                      p(lw.o), p(lw.post_norm), p(lw.gate), p(lw.up), p(lw.down))
        w = _Weights(p(weights.embed), p(weights.final_norm), layers)
        ctx = ctypes.c_void_p()
        _check(lib.hy_ctx_create(ctypes.byref(cfg), ctypes.byref(w), ctypes.byref(ctx)))
        return cls(ctx, cfg)

    @classmethod
    def from_package(cls, model_root: str, **cfg_overrides) -> "TextRuntime":
        """TextRuntime::load from a model package directory (hy_ctx_create_from_package):
        num_layers, vocab_size and ffn_dim come from the package."""
        lib = load_library()
        cfg = default_config(**cfg_overrides)
        ctx = ctypes.c_void_p()
        _check(lib.hy_ctx_create_from_package(ctypes.byref(cfg), os.fsencode(model_root), ctypes.byref(ctx)))
        out = Config()
        _check(lib.hy_ctx_config(ctx, ctypes.byref(out)))
        return cls(ctx, out)

    def close(self) -> None:
        if self._ctx:
            _LIB.hy_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_token_callback(self, fn, tokens_per_sync: int = 0) -> None:
        """stream_callback: fn(token) for every committed token, in order (None removes it)."""
        self._cb = TOKEN_CALLBACK(lambda tok, _user: fn(int(tok))) if fn is not None else TOKEN_CALLBACK()
        _check(_LIB.hy_ctx_set_token_callback(self._ctx, self._cb, None, tokens_per_sync))

    @property
    def ar_path(self) -> int:
        return int(_LIB.hy_ctx_ar_path(self._ctx))

    @ar_path.setter
    def ar_path(self, path: int) -> None:
        _check(_LIB.hy_ctx_set_ar_path(self._ctx, path))

    @property
    def device_bytes(self) -> int:
        return int(_LIB.hy_ctx_device_bytes(self._ctx))

    @property
    def stream(self) -> int:
        return int(_LIB.hy_ctx_stream(self._ctx) or 0)

    # -- sequence state ----------------------------------------------------
    def reset(self) -> None:
        _check(_LIB.hy_seq_reset(self._ctx))

    @property
    def kv_length(self) -> int:
        n = ctypes.c_int()
        _check(_LIB.hy_seq_length(self._ctx, ctypes.byref(n)))
        return n.value

    def truncate(self, rows: int) -> None:
        """view_dflash_rows (src/dflash_runtime.cpp:97-119)."""
        _check(_LIB.hy_seq_truncate(self._ctx, rows))

    def set_length(self, rows: int) -> None:
        _check(_LIB.hy_seq_set_length(self._ctx, rows))

    def set_history(self, ids) -> None:
        a = _i32(ids)
        _check(_LIB.hy_history_set(self._ctx, _ptr(a), a.size))

    def add_history(self, ids) -> None:
        a = _i32(ids)
        _check(_LIB.hy_history_add(self._ctx, _ptr(a), a.size))

    # -- decoder -----------------------------------------------------------
    def prefill(self, inputs_embeds: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
        """run_decoder_prefill (src/text_runtime.cpp:648-674); returns the final-normed last hidden row."""
        e, c, s = _f32(inputs_embeds), _f32(cos), _f32(sin)
        out = np.empty(HIDDEN, np.float32)
        _check(_LIB.hy_prefill(self._ctx, _ptr(e), _ptr(c), _ptr(s), e.shape[0], _ptr(out), None))
        return out

    def run_decoder_step(self, embeds: np.ndarray, cos: np.ndarray, sin: np.ndarray, aux: bool = False):
        """detail::run_decoder_step (src/text_decoder_step.h:29-38): returns (hidden, aux_hidden|None)."""
        e, c, s = _f32(embeds), _f32(cos), _f32(sin)
        rows = e.shape[0]
        hidden = np.empty((rows, HIDDEN), np.float32)
        auxh = np.empty((4, rows, HIDDEN), np.float32) if aux else None
        _check(_LIB.hy_decoder_step(self._ctx, _ptr(e), rows, _ptr(c), _ptr(s), _ptr(hidden), _ptr(auxh)))
        return hidden, auxh

    def select_logit_rows(self, hidden: np.ndarray, penalty: float, row_prefix=None, want_logits: bool = False):
        """run_lm_head + select_logit_rows (src/text_runtime.cpp:430-439, 757-797) with the current history."""
        h = _f32(hidden).reshape(-1, HIDDEN)
        rows = h.shape[0]
        tok = np.empty(rows, np.int32)
        raw = np.empty(rows, np.int32)
        pre = None if row_prefix is None else _i32(row_prefix)
        logits = np.empty((rows, self.cfg.vocab_size), np.float32) if want_logits else None
        _check(_LIB.hy_lm_head_select(self._ctx, _ptr(h), rows, _ptr(pre), penalty, _ptr(tok), _ptr(raw),
                                      _ptr(logits)))
        return tok, raw, logits

    def select_logit_rows_noalloc(self, hidden_dev: int, rows: int, penalty: float, tokens_dev: int,
                                  raw_top1_dev: int) -> None:
        """select_logit_rows on device pointers (ints), allocating nothing: the
        argmax scratch is a static device-global array (no reference counterpart)."""
        _check(_LIB.hy_lm_head_select_noalloc(self._ctx, ctypes.c_void_p(hidden_dev), rows, penalty,
                                              ctypes.c_void_p(tokens_dev), ctypes.c_void_p(raw_top1_dev)))

    def attention(self, layer: int, qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
        q, c, s = _f32(qkv), _f32(cos), _f32(sin)
        rows = q.shape[0]
        out = np.empty((rows, 2048), np.float32)
        _check(_LIB.hy_attention(self._ctx, layer, _ptr(q), rows, _ptr(c), _ptr(s), _ptr(out)))
        return out

    def kv_write(self, layer: int, start: int, k: np.ndarray, v: np.ndarray) -> None:
        k, v = _f32(k), _f32(v)
        _check(_LIB.hy_kv_write(self._ctx, layer, start, k.shape[1], _ptr(k), _ptr(v)))

    def kv_read(self, layer: int, start: int, rows: int):
        k = np.empty((8, rows, HEAD_DIM), np.float32)
        v = np.empty((8, rows, HEAD_DIM), np.float32)
        _check(_LIB.hy_kv_read(self._ctx, layer, start, rows, _ptr(k), _ptr(v)))
        return k, v

    # -- timing -------------------------------------------------------------
    def last_timing(self) -> TextDecodeTiming:
        """TextDecodeTiming of the last AR call (hy_ctx_last_timing)."""
        t = _DecodeTiming()
        _check(_LIB.hy_ctx_last_timing(self._ctx, ctypes.byref(t)))
        return TextDecodeTiming(*[getattr(t, n) for n, _ in _DecodeTiming._fields_])

    def _dflash_result(self, tokens, n, acc, nb) -> DFlashDecodeResult:
        t = _DFlashTiming()
        _check(_LIB.hy_ctx_last_dflash_timing(self._ctx, ctypes.byref(t)))
        timing = DFlashDecodeTiming(*[getattr(t, n) for n, _ in _DFlashTiming._fields_[:7]])
        return DFlashDecodeResult(tokens[:n.value].tolist(), t.block_count, t.drafted_token_count,
                                  t.accepted_draft_token_count, acc[:nb.value].tolist(), timing=timing)

    # -- loops -------------------------------------------------------------
    def generate(self, first_token: int, first_raw: int, max_tokens: int, penalty: float, eos_ids=()):
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        tokens = np.empty(max_tokens, np.int32)
        raw = np.empty(max_tokens, np.int32)
        n = ctypes.c_int()
        _check(_LIB.hy_generate(self._ctx, first_token, first_raw, max_tokens, penalty, _ptr(eos),
                                0 if eos is None else eos.size, _ptr(tokens), _ptr(raw), ctypes.byref(n)))
        return tokens[:n.value].tolist(), raw[:n.value].tolist()

    def dflash_verify_block(self, proposed, max_commit: int, penalty: float, eos_ids=()):
        p = _i32(proposed)
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        post = np.empty(DFLASH_BLOCK, np.int32)
        acc, com, stop = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _check(_LIB.hy_verify_block(self._ctx, _ptr(p), max_commit, penalty, _ptr(eos),
                                    0 if eos is None else eos.size, _ptr(post), ctypes.byref(acc),
                                    ctypes.byref(com), ctypes.byref(stop)))
        return post.tolist(), acc.value, com.value, bool(stop.value)

    def dflash_generate_synthetic(self, first_token: int, max_tokens: int, penalty: float, greedy, p: float,
                                  seed: int, eos_ids=()) -> DFlashDecodeResult:
        g = _i32(greedy)
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        tokens = np.empty(max_tokens, np.int32)
        acc = np.empty(max_tokens + DFLASH_BLOCK, np.int32)
        n, nb = ctypes.c_int(), ctypes.c_int()
        _check(_LIB.hy_dflash_generate_synthetic(self._ctx, first_token, max_tokens, penalty, _ptr(eos),
                                                 0 if eos is None else eos.size, _ptr(g), g.size, p, seed,
                                                 _ptr(tokens), ctypes.byref(n), _ptr(acc), ctypes.byref(nb)))
        return self._dflash_result(tokens, n, acc, nb)

    def run_vlm_decode_with_prompt(self, input_ids, position_ids, image_token_id: int, vision_features,
                                   max_tokens: int, repetition_penalty: float = 1.08,
                                   eos_ids=()) -> TextDecodeResult:
        """TextRuntime::run_vlm_decode_with_prompt (src/text_runtime.cpp:2053-2094)."""
        ids = _i32(input_ids)
        pos = _i32(position_ids).reshape(-1)
        feats = _f32(vision_features).reshape(-1, HIDDEN)
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        mt = max_tokens if max_tokens > 0 else 1024
        tokens = np.empty(mt, np.int32)
        raw = np.empty(mt, np.int32)
        n = ctypes.c_int()
        _check(_LIB.hy_run_vlm_decode_with_prompt(self._ctx, _ptr(ids), _ptr(pos), ids.size, image_token_id,
                                                  _ptr(feats), feats.shape[0], max_tokens, repetition_penalty,
                                                  _ptr(eos), 0 if eos is None else eos.size, _ptr(tokens),
                                                  _ptr(raw), ctypes.byref(n)))
        return TextDecodeResult(ids.size, repetition_penalty, tokens[:n.value].tolist(), raw[:n.value].tolist(),
                                timing=self.last_timing())

    def batch_decode(self, requests, max_tokens: int, slots: int = 16, repetition_penalty: float = 1.08,
                     eos_ids=()):
        """Records decoded together, up to `slots` at a time (hy_batch_decode).
        requests: (input_ids, position_ids, image_token_id, vision_features) tuples.
        Returns (tokens per record, status per record)."""
        keep = []
        reqs = (_Request * max(1, len(requests)))()
        for i, (ids, pos, img, feats) in enumerate(requests):
            ids, pos, feats = _i32(ids), _i32(pos).reshape(-1), _f32(feats).reshape(-1, HIDDEN)
            keep += [ids, pos, feats]
            reqs[i] = _Request(ids.ctypes.data, pos.ctypes.data, ids.size, img, feats.ctypes.data, feats.shape[0])
        n = len(requests)
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        tokens = np.zeros((max(1, n), max_tokens), np.int32)
        counts = np.zeros(max(1, n), np.int32)
        status = np.zeros(max(1, n), np.int32)
        _check(_LIB.hy_batch_decode(self._ctx, reqs, n, slots, max_tokens, repetition_penalty, _ptr(eos),
                                    0 if eos is None else eos.size, _ptr(tokens), _ptr(counts), _ptr(status)))
        return [tokens[i, :counts[i]].tolist() for i in range(n)], status[:n].tolist()

    # -- DFlash draft network -------------------------------------------------
    def load_draft(self, draft_weights, mask_token: int = DFLASH_MASK_TOKEN) -> None:
        """DFlashDraftRuntime::load (src/dflash_runtime.cpp:175-201). draft_weights: an object with
        .fc, .hidden_norm, .norm and .layers[i] as in from_weights (numpy fp32, nn.Linear layout)."""
        keep = []

        def p(a):
            a = _f32(a)
            keep.append(a)
            return a.ctypes.data

        n = len(draft_weights.layers)
        layers = (_LayerWeights * n)()
        for i, lw in enumerate(draft_weights.layers):
            layers[i] = _LayerWeights(p(lw.input_norm), p(lw.q), p(lw.k), p(lw.v), p(lw.q_norm), p(lw.k_norm),
                                      p(lw.o), p(lw.post_norm), p(lw.gate), p(lw.up), p(lw.down))
        w = _DraftWeights(n, mask_token, p(draft_weights.fc), p(draft_weights.hidden_norm), p(draft_weights.norm),
                          layers)
        _check(_LIB.hy_draft_load(self._ctx, ctypes.byref(w)))

    def load_draft_package(self, model_root: str, mask_token: int = DFLASH_MASK_TOKEN) -> None:
        """DFlashDraftRuntime::load from <model_root>/dflash (hy_draft_load_package)."""
        _check(_LIB.hy_draft_load_package(self._ctx, os.fsencode(model_root), mask_token))

    def load_draft_synthetic(self, num_layers: int, seed: int, std: float = 0.02, norm_std: float = 0.0,
                             mask_token: int = DFLASH_MASK_TOKEN) -> None:
        _check(_LIB.hy_draft_load_synthetic(self._ctx, num_layers, mask_token, seed, std, norm_std))

    @property
    def draft_context_length(self) -> int:
        n = ctypes.c_int()
        _check(_LIB.hy_draft_context_length(self._ctx, ctypes.byref(n)))
        return n.value

    def draft_context_append(self, aux_hidden) -> None:
        """append_dflash_rows (src/dflash_runtime.cpp:121-166): aux_hidden [4, rows, 1024]."""
        a = _f32(aux_hidden)
        _check(_LIB.hy_draft_context_append(self._ctx, _ptr(a), a.shape[1]))

    def draft_run(self, noise) -> np.ndarray:
        """DFlashDraftRuntime::run (src/dflash_runtime.cpp:213-290): final-normed draft rows [16, 1024]."""
        x = _f32(noise)
        out = np.empty((DFLASH_BLOCK, HIDDEN), np.float32)
        _check(_LIB.hy_draft_run(self._ctx, _ptr(x), _ptr(out)))
        return out

    def draft_propose(self, current_token: int) -> list:
        out = np.empty(DFLASH_BLOCK, np.int32)
        _check(_LIB.hy_draft_propose(self._ctx, current_token, _ptr(out)))
        return out.tolist()

    def dflash_generate(self, first_token: int, max_tokens: int, penalty: float, eos_ids=()) -> DFlashDecodeResult:
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        tokens = np.empty(max_tokens, np.int32)
        acc = np.empty(max_tokens + DFLASH_BLOCK, np.int32)
        n, nb = ctypes.c_int(), ctypes.c_int()
        _check(_LIB.hy_dflash_generate(self._ctx, first_token, max_tokens, penalty, _ptr(eos),
                                       0 if eos is None else eos.size, _ptr(tokens), ctypes.byref(n), _ptr(acc),
                                       ctypes.byref(nb)))
        return self._dflash_result(tokens, n, acc, nb)

    def run_vlm_dflash_with_prompt(self, input_ids, position_ids, image_token_id: int, vision_features,
                                   max_tokens: int, repetition_penalty: float = 1.08,
                                   eos_ids=()) -> DFlashDecodeResult:
        """run_vlm_decode_with_prompt with --dflash (src/text_runtime.cpp:1142-1305)."""
        ids = _i32(input_ids)
        pos = _i32(position_ids).reshape(-1)
        feats = _f32(vision_features).reshape(-1, HIDDEN)
        eos = _i32(list(eos_ids)) if len(eos_ids) else None
        mt = max_tokens if max_tokens > 0 else 1024
        tokens = np.empty(mt, np.int32)
        acc = np.empty(mt + DFLASH_BLOCK, np.int32)
        n, nb = ctypes.c_int(), ctypes.c_int()
        _check(_LIB.hy_run_vlm_dflash_with_prompt(self._ctx, _ptr(ids), _ptr(pos), ids.size, image_token_id,
                                                  _ptr(feats), feats.shape[0], max_tokens, repetition_penalty,
                                                  _ptr(eos), 0 if eos is None else eos.size, _ptr(tokens),
                                                  ctypes.byref(n), _ptr(acc), ctypes.byref(nb)))
        return self._dflash_result(tokens, n, acc, nb)

    # -- regression fixtures ---------------------------------------------------
    @staticmethod
    def _checked(max_tokens: int, expected) -> int:
        # decode_from_embeddings (src/text_runtime.cpp:1341-1350): with expected tokens,
        # max_tokens <= 0 or past their count means all of them.
        n = len(expected)
        return n if (max_tokens <= 0 or max_tokens > n) else max_tokens

    def run_vlm_fixture_decode(self, fixture_dir: str, max_tokens: int = 0, eos_ids=()) -> TextDecodeResult:
        """TextRuntime::run_vlm_fixture_decode (src/text_runtime.cpp:1793-1837), penalty 1.08."""
        fx = read_vlm_fixture(fixture_dir)
        n = self._checked(max_tokens, fx.expected_tokens)
        res = self.run_vlm_decode_with_prompt(fx.input_ids, fx.position_ids, fx.image_token_id, fx.vision_features,
                                              max_tokens=n, eos_ids=eos_ids)
        res.checked_tokens = n
        res.expected_tokens = fx.expected_tokens[:n].tolist()
        return res

    def run_vlm_fixture_dflash_decode(self, fixture_dir: str, max_tokens: int = 0, eos_ids=()) -> DFlashDecodeResult:
        """TextRuntime::run_vlm_fixture_dflash_decode (src/text_runtime.cpp:1886-1920), penalty 1.08."""
        fx = read_vlm_fixture(fixture_dir)
        n = self._checked(max_tokens, fx.expected_tokens)
        res = self.run_vlm_dflash_with_prompt(fx.input_ids, fx.position_ids, fx.image_token_id, fx.vision_features,
                                              max_tokens=n, eos_ids=eos_ids)
        res.expected_tokens = fx.expected_tokens[:n].tolist()
        return res

    # -- timing hooks --------------------------------------------------------
    def bench_ar_steps(self, count: int) -> float:
        ms = ctypes.c_float()
        _check(_LIB.hy_bench_ar_steps(self._ctx, count, ctypes.byref(ms)))
        return ms.value

    def trace_persistent(self, tokens: int, trace_token: int) -> np.ndarray:
        """Per-phase trace of one token of the persistent kernel, [4 CTAs, phases, 12] uint64:
        0 phase start, 1 inputs ready, 2 prologue done, 3 phase end (%globaltimer ns);
        4 / 5 / 6: warp 0's SM cycles waiting on its slots / working, and its stages;
        7 / 8 / 9 / 10 (attention): slot-wait cycles, work cycles, stages of the warp owning
        the split's first stage, and the time its stage loop ended (ns)."""
        phases = 5 * self.cfg.num_layers + 1
        out = np.zeros((4, phases, 12), np.uint64)
        _check(_LIB.hy_trace_persistent(self._ctx, tokens, trace_token, _ptr(out)))
        return out

    def step_trace(self, reset: bool = True, max_records: int = 16384):
        """Step trace of the per-phase kernels (library built with HY_STEP_TRACE): an
        [n, 5] array of {kernel id, CTA 0's %globaltimer ns at entry, after its
        griddepcontrol.wait, after its prologue, at its end; 16-row projections: ns its
        thread 0 waited for its weight units, ns in their MMAs, %globaltimer after its
        last unit; the latest exit of the CTAs of the kernels before it; 16-row
        projections: each warp's last-unit time and its ns waiting for units} per launch
        ([n, 25]), in launch order."""
        out = np.zeros(25 * max_records, np.uint64)
        n = ctypes.c_int(0)
        _check(_LIB.hy_debug_step_trace(self._ctx, _ptr(out), max_records, ctypes.byref(n), int(reset)))
        return out.reshape(max_records, 25)[:min(n.value, max_records)].copy()

    WAIT_KINDS = ("slot_free", "slot_full", "prod_slot", "prod_token", "poll_x", "poll_act", "poll_attn_out",
                  "poll_qkv", "poll_parts", "poll_token")

    def wait_stats(self, reset: bool = True):
        """Wait statistics of the persistent kernel (library built with HY_WAIT_STATS):
        (per-CTA [160, kinds, 3] = waits over 20 us, their ns, longest ns;
        per-launch [64, 2] = first CTA start, last CTA exit in %globaltimer ns, 0 if unused)."""
        n = 160 * len(self.WAIT_KINDS) * 3 + 64 * 2
        out = np.zeros(n, np.uint64)
        _check(_LIB.hy_debug_wait_stats(self._ctx, _ptr(out), n, int(reset)))
        per = out[:160 * len(self.WAIT_KINDS) * 3].reshape(160, len(self.WAIT_KINDS), 3)
        lw = out[160 * len(self.WAIT_KINDS) * 3:].reshape(64, 2).copy()
        used = lw[:, 1] != 0
        lw[used, 0] = ~lw[used, 0]
        lw[~used] = 0
        return per, lw

    def set_wait_limit(self, limit_ns: int) -> None:
        """Bound of the persistent kernel's waits (hy_ctx_set_wait_limit)."""
        _check(_LIB.hy_ctx_set_wait_limit(self._ctx, limit_ns))

    def wait_probe(self, kind: int, limit_ns: int) -> None:
        """Run the bounded-wait self-test (hy_debug_wait_probe); raises HyError
        (HY_ERR_DEVICE_TIMEOUT) when the wait ran out, as it should."""
        _check(_LIB.hy_debug_wait_probe(self._ctx, kind, limit_ns))

    def debug_progress(self, n: int = 148) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        _check(_LIB.hy_debug_progress(self._ctx, _ptr(out), n))
        return out

    def bench_kernel(self, which: int, count: int) -> float:
        ms = ctypes.c_float()
        _check(_LIB.hy_bench_kernel(self._ctx, which, count, ctypes.byref(ms)))
        return ms.value
