"""CPU oracle for the HunyuanOCR text-decode hot path (test infrastructure).

This module is the checker, not the product. Only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline leg may import it. The product
path (the CUDA library behind include/hy_decode.h) never calls into it.

It restates, in numpy, the reference's CPU fp32 decode path:
  * the decoder graph of export/text_decoder_kv.py (``_layer_forward`` 49-96,
    ``prefill`` 98-112, ``decode`` 168-183) that ncnn executes through
    ``run_decoder_step_impl`` (src/text_runtime.cpp:678-728);
  * PreciseSDPA's fp64-accumulated attention (src/precise_sdpa.cpp:281-329),
    with the ``%g``-printed scale literal 0.0883883 written into the ncnn param
    by export/add_kvcache.py:26,57-59;
  * the full-width RoPE of src/multimodal_rope.cpp:176-187;
  * the host logic of src/text_runtime.cpp (build_mrope 42-63, rope_value
    182-193, masks 207-251, select_next_token 730-755, select_logit_rows
    757-797, the AR loop 1307-1521, the DFlash block 880-1071 and loop
    1142-1305) and src/dflash_runtime.cpp (build_dflash_block 20-25,
    build_dflash_verify_mask 60-76, dflash_acceptance_length 78-95).

Pinning: tests/test_oracle_golden.py checks this module against
tests/golden/*.npz, produced by tests/golden/make_golden.py from the
reference's own TextDecoderExternalRopeKVWrapper (export/text_decoder_kv.py)
over a random-init transformers HunYuanDenseV1Model, and against the
known-answer values of the reference's C++ tests (tests/text_rope_test.cpp,
tests/multimodal_rope_test.cpp, tests/precise_sdpa_test.cpp,
tests/dflash_runtime_test.cpp).
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field

import numpy as np

# Model constants: src/text_decoder_step.h:19-24, src/text_runtime.cpp:97-104,
# include/hunyuan_ocr/dflash_runtime.h:17-18.
HIDDEN = 1024
HEAD_DIM = 128
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
Q_WIDTH = NUM_Q_HEADS * HEAD_DIM          # 2048
KV_WIDTH = NUM_KV_HEADS * HEAD_DIM        # 1024
FFN = 3584
VOCAB = 120818
NUM_LAYERS = 24
RMS_EPS = 1e-5
ROPE_THETA = 10000.0
ROPE_ALPHA = 1000.0
MASK_NEG_INF = np.float32(-1.0e38)
DEFAULT_PENALTY = 1.08
DFLASH_BLOCK = 16
DFLASH_MASK_TOKEN = 120817
IMAGE_TOKEN_ID = 120120                   # src/prompt_builder.cpp:8
EOS_ID = 120020                           # models/model.json.example
DFLASH_TARGET_LAYER_IDS = (1, 8, 15, 22)  # export/text_decoder_kv.py:11
# export/add_kvcache.py:26 writes f"{1/sqrt(128):g}" into the SDPA param.
NCNN_SDPA_SCALE = float(np.float32(float(f"{1.0 / math.sqrt(HEAD_DIM):g}")))
EXACT_SDPA_SCALE = 1.0 / math.sqrt(HEAD_DIM)


# ---------------------------------------------------------------------------
# Synthetic weights (same generator as oracle/synth.c and the CUDA library).
# ---------------------------------------------------------------------------
_M64 = (1 << 64) - 1
_GOLDEN = 0x9E3779B97F4A7C15
_TID = 0xD1B54A32D192ED03


def _splitmix64_scalar(z: int) -> int:
    z = (z + _GOLDEN) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def _splitmix64_np(z: np.ndarray) -> np.ndarray:
    z = z + np.uint64(_GOLDEN)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def synth_mult(std: float) -> np.float32:
    return np.float32(float(std) * math.sqrt(3.0) / 65536.0)


def synth_tensor(seed: int, tensor_id: int, count: int, std: float, offset: float = 0.0) -> np.ndarray:
    """Counter-based generator; see the header of oracle/synth.c for the definition."""
    base = _splitmix64_scalar((seed * _GOLDEN + tensor_id * _TID) & _M64)
    out = np.empty(count, dtype=np.float32)
    mult = synth_mult(std)
    off = np.float32(offset)
    chunk = 1 << 22
    with np.errstate(over="ignore"):
        for start in range(0, count, chunk):
            n = min(chunk, count - start)
            idx = np.arange(start, start + n, dtype=np.uint64) + np.uint64(base)
            h = _splitmix64_np(idx)
            s = ((h & np.uint64(0xFFFF)) + ((h >> np.uint64(16)) & np.uint64(0xFFFF))
                 + ((h >> np.uint64(32)) & np.uint64(0xFFFF)) + (h >> np.uint64(48)))
            c = (s.astype(np.int64) - 131070).astype(np.float32)
            out[start:start + n] = off + c * mult
    return out


_SYNTH_LIB = None


def _synth_lib():
    global _SYNTH_LIB
    if _SYNTH_LIB is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhy_synth.so")
        if not os.path.exists(path):
            return None
        lib = ctypes.CDLL(path)
        lib.hy_synth_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_void_p, ctypes.c_size_t]
        lib.hy_synth_fill.restype = None
        _SYNTH_LIB = lib
    return _SYNTH_LIB


def synth_tensor_fast(seed: int, tensor_id: int, count: int, std: float, offset: float = 0.0) -> np.ndarray:
    """Same values as synth_tensor, through oracle/libhy_synth.so when it is built."""
    lib = _synth_lib()
    if lib is None:
        return synth_tensor(seed, tensor_id, count, std, offset)
    out = np.empty(count, dtype=np.float32)
    lib.hy_synth_fill(seed, tensor_id, std, offset, out.ctypes.data, count)
    return out


# Tensor ids of the synthetic weight set (shared with the CUDA generator).
TID_EMBED = 1
TID_FINAL_NORM = 2
LAYER_TID_BASE = 100
LAYER_TID_STRIDE = 16
(J_INPUT_NORM, J_Q, J_K, J_V, J_Q_NORM, J_K_NORM, J_O, J_POST_NORM, J_GATE, J_UP, J_DOWN) = range(11)


@dataclass
class ModelConfig:
    num_layers: int = NUM_LAYERS
    vocab: int = VOCAB
    ffn: int = FFN
    rms_eps: float = RMS_EPS
    attn_scale: float = NCNN_SDPA_SCALE
    kv_bf16: bool = False   # bf16 variant: cached K/V rows rounded to bf16 (RNE)


@dataclass
class LayerWeights:
    input_norm: np.ndarray
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    o: np.ndarray
    post_norm: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray


@dataclass
class Weights:
    embed: np.ndarray
    final_norm: np.ndarray
    layers: list = field(default_factory=list)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


def make_weights(cfg: ModelConfig, seed: int, std: float = 0.02, norm_std: float = 0.0,
                 fast: bool = True, bf16: bool = False) -> Weights:
    """Seeded N(0, std)-like linears/embedding, norms = 1 + N(0, norm_std).
    bf16: the linears and the embedding rounded to bf16 (the library's bf16-weight
    variant rounds the same fp32 values); norms stay fp32."""
    gen = synth_tensor_fast if fast else synth_tensor

    def lin(tid, rows, cols):
        t = gen(seed, tid, rows * cols, std).reshape(rows, cols)
        return round_bf16(t) if bf16 else t

    def norm(tid, n):
        return gen(seed, tid, n, norm_std, 1.0)

    layers = []
    for li in range(cfg.num_layers):
        b = LAYER_TID_BASE + LAYER_TID_STRIDE * li
        layers.append(LayerWeights(
            input_norm=norm(b + J_INPUT_NORM, HIDDEN),
            q=lin(b + J_Q, Q_WIDTH, HIDDEN),
            k=lin(b + J_K, KV_WIDTH, HIDDEN),
            v=lin(b + J_V, KV_WIDTH, HIDDEN),
            q_norm=norm(b + J_Q_NORM, HEAD_DIM),
            k_norm=norm(b + J_K_NORM, HEAD_DIM),
            o=lin(b + J_O, HIDDEN, Q_WIDTH),
            post_norm=norm(b + J_POST_NORM, HIDDEN),
            gate=lin(b + J_GATE, cfg.ffn, HIDDEN),
            up=lin(b + J_UP, cfg.ffn, HIDDEN),
            down=lin(b + J_DOWN, HIDDEN, cfg.ffn),
        ))
    return Weights(embed=lin(TID_EMBED, cfg.vocab, HIDDEN),
                   final_norm=norm(TID_FINAL_NORM, HIDDEN), layers=layers)


# ---------------------------------------------------------------------------
# Host logic: RoPE tables and masks.
# ---------------------------------------------------------------------------
def _f32(x) -> np.float32:
    return np.float32(x)


def mrope_base() -> np.float32:
    # src/text_runtime.cpp:47 and 184-187: float(10000 * 1000^(128/126)) in double.
    return _f32(ROPE_THETA * math.pow(ROPE_ALPHA, HEAD_DIM / (HEAD_DIM - 2)))


def inv_freq_table() -> np.ndarray:
    """inv_freq[d] = 1.0f / powf(base, float(2*(d%64))/128) (src/text_runtime.cpp:53, 188-189)."""
    base = mrope_base()
    out = np.empty(HEAD_DIM, dtype=np.float32)
    for d in range(HEAD_DIM):
        fd = d % (HEAD_DIM // 2)
        expo = _f32(_f32(2 * fd) / _f32(HEAD_DIM))
        # powf is evaluated in double and rounded once (a correctly rounded powf).
        out[d] = _f32(1.0) / _f32(math.pow(float(base), float(expo)))
    return out


def _cos32(angle: np.ndarray) -> np.ndarray:
    """cosf of fp32 angles, evaluated in double and rounded once."""
    return np.cos(np.asarray(angle, dtype=np.float32).astype(np.float64)).astype(np.float32)


def _sin32(angle: np.ndarray) -> np.ndarray:
    return np.sin(np.asarray(angle, dtype=np.float32).astype(np.float64)).astype(np.float32)


def build_mrope(position_ids: np.ndarray, seq_len: int, use_cos: bool) -> np.ndarray:
    """src/text_runtime.cpp:42-63: dim d uses position axis d/32 and frequency index d%64."""
    pos = np.asarray(position_ids, dtype=np.int32).reshape(4, seq_len)
    inv = inv_freq_table()
    out = np.empty((seq_len, HEAD_DIM), dtype=np.float32)
    for d in range(HEAD_DIM):
        axis = d // (HEAD_DIM // 4)
        angle = pos[axis].astype(np.float32) * inv[d]
        out[:, d] = _cos32(angle) if use_cos else _sin32(angle)
    return out


def rope_rows(start: int, rows: int, use_cos: bool) -> np.ndarray:
    """build_decode_rope / build_verify_rope (src/text_runtime.cpp:228-251) via rope_value (182-193)."""
    inv = inv_freq_table()
    pos = np.arange(start, start + rows, dtype=np.int64).astype(np.float32)
    angle = (pos[:, None] * inv[None, :]).astype(np.float32)
    return _cos32(angle) if use_cos else _sin32(angle)


def make_prefill_mask(seq_len: int) -> np.ndarray:
    """src/text_runtime.cpp:207-219."""
    r = np.arange(seq_len)
    return np.where(r[None, :] > r[:, None], MASK_NEG_INF, np.float32(0.0)).astype(np.float32)


def make_decode_mask(past_len: int) -> np.ndarray:
    """src/text_runtime.cpp:221-226."""
    return np.zeros((1, past_len + 1), dtype=np.float32)


def build_dflash_verify_mask(past_len: int) -> np.ndarray:
    """src/dflash_runtime.cpp:60-76: row r sees columns <= past_len + r."""
    key_len = past_len + DFLASH_BLOCK
    col = np.arange(key_len)[None, :]
    row = np.arange(DFLASH_BLOCK)[:, None]
    return np.where(col > past_len + row, MASK_NEG_INF, np.float32(0.0)).astype(np.float32)


def build_dflash_block(first_token: int, mask_token: int = DFLASH_MASK_TOKEN) -> list:
    """src/dflash_runtime.cpp:20-25 (mask_token: kDFlashMaskTokenId = 120817; a
    smaller test vocabulary passes its own filler id)."""
    return [int(first_token)] + [int(mask_token)] * (DFLASH_BLOCK - 1)


def dflash_acceptance_length(proposed, posterior) -> int:
    """src/dflash_runtime.cpp:78-95."""
    if len(proposed) == 0 or len(proposed) != len(posterior):
        return -1
    accepted = 0
    for i in range(1, len(proposed)):
        if proposed[i] != posterior[i - 1]:
            break
        accepted += 1
    return accepted


# ---------------------------------------------------------------------------
# Decoder math.
# ---------------------------------------------------------------------------
def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """HunYuanDenseV1RMSNorm: x * rsqrt(mean(x^2) + eps), then weight * (.)."""
    x = x.astype(np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (w * (x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))))).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Full-width non-interleaved RoPE (src/multimodal_rope.cpp:176-187).

    x [..., rows, 128]; cos/sin [rows, 128].
    out[d] = x[d] c[d] - x[d+64] s[d];  out[d+64] = x[d+64] c[d+64] + x[d] s[d+64].
    """
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    out = np.empty_like(x, dtype=np.float32)
    out[..., :h] = x1 * cos[:, :h] - x2 * sin[:, :h]
    out[..., h:] = x2 * cos[:, h:] + x1 * sin[:, h:]
    return out


def precise_sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float) -> np.ndarray:
    """PreciseSDPA decode/verify (src/precise_sdpa.cpp:281-329), GQA without expansion.

    q [16, M, 128]; k, v [8, L, 128] (8 unique KV heads; q head h reads KV head
    h // 2, which is what repeat_kv_for_attention's expansion amounts to,
    export/text_decoder_kv.py:21-27); mask [M, L] additive. fp64 accumulation.
    """
    groups = q.shape[0] // k.shape[0]
    out = np.empty(q.shape, dtype=np.float32)
    m64 = mask.astype(np.float64)
    for kvh in range(k.shape[0]):
        k64 = k[kvh].astype(np.float64)
        v64 = v[kvh].astype(np.float64)
        for g in range(groups):
            h = kvh * groups + g
            s = (q[h].astype(np.float64) @ k64.T) * float(scale) + m64
            s = np.exp(s - s.max(axis=1, keepdims=True))
            s /= s.sum(axis=1, keepdims=True)
            out[h] = (s @ v64).astype(np.float32)
    return out


@dataclass
class KVCache:
    """Per layer K/V [8, capacity, 128] fp32 and the logical length (rows)."""
    k: list
    v: list
    length: int = 0

    @staticmethod
    def empty(num_layers: int, capacity: int) -> "KVCache":
        return KVCache([np.zeros((NUM_KV_HEADS, capacity, HEAD_DIM), np.float32) for _ in range(num_layers)],
                       [np.zeros((NUM_KV_HEADS, capacity, HEAD_DIM), np.float32) for _ in range(num_layers)], 0)


def layer_forward(lw: LayerWeights, x: np.ndarray, mask: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                  cache_k: np.ndarray, cache_v: np.ndarray, past: int, cfg: ModelConfig) -> np.ndarray:
    """One decoder layer (export/text_decoder_kv.py:49-96); appends M rows at `past`.

    x [M, 1024]. Keys are cached after RoPE and key_layernorm, as PreciseSDPA
    appends the post-norm keys (src/precise_sdpa.cpp:233-262).
    """
    m_rows = x.shape[0]
    h = rms_norm(x, lw.input_norm, cfg.rms_eps)
    q = (h @ lw.q.T).reshape(m_rows, NUM_Q_HEADS, HEAD_DIM).transpose(1, 0, 2)
    k = (h @ lw.k.T).reshape(m_rows, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
    v = (h @ lw.v.T).reshape(m_rows, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    q = rms_norm(q, lw.q_norm, cfg.rms_eps)
    k = rms_norm(k, lw.k_norm, cfg.rms_eps)
    if cfg.kv_bf16:
        k, v = round_bf16(k), round_bf16(v)
    cache_k[:, past:past + m_rows] = k
    cache_v[:, past:past + m_rows] = v
    L = past + m_rows
    attn = precise_sdpa(q, cache_k[:, :L], cache_v[:, :L], mask, cfg.attn_scale)
    attn = attn.transpose(1, 0, 2).reshape(m_rows, Q_WIDTH)
    x = (x + attn @ lw.o.T).astype(np.float32)
    m = rms_norm(x, lw.post_norm, cfg.rms_eps)
    g = m @ lw.gate.T
    u = m @ lw.up.T
    act = (g / (np.float32(1.0) + np.exp(-g))) * u
    return (x + act.astype(np.float32) @ lw.down.T).astype(np.float32)


def decoder_forward(w: Weights, cfg: ModelConfig, x: np.ndarray, mask: np.ndarray, cos: np.ndarray,
                    sin: np.ndarray, cache: KVCache, aux: bool = False):
    """Prefill/decode/verify over all layers, final norm applied (export/text_decoder_kv.py:98-183).

    Returns (normed hidden [M,1024], aux hidden list or None). Advances cache.length by M.
    """
    past = cache.length
    x = x.astype(np.float32)
    aux_out = [] if aux else None
    for li, lw in enumerate(w.layers):
        x = layer_forward(lw, x, mask, cos, sin, cache.k[li], cache.v[li], past, cfg)
        if aux and li in DFLASH_TARGET_LAYER_IDS:
            aux_out.append(x.copy())
    cache.length = past + x.shape[0]
    return rms_norm(x, w.final_norm, cfg.rms_eps), aux_out


def attention_rows(lw: LayerWeights, qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray, k_past: np.ndarray,
                   v_past: np.ndarray, scale: float, eps: float):
    """The attention block of one decoder layer for `rows` new rows over a cache
    (export/text_decoder_kv.py:66-79 RoPE, query/key layernorm, append; PreciseSDPA
    with the decode / verify mask, src/precise_sdpa.cpp:281-329 and
    src/text_runtime.cpp:221-226 / src/dflash_runtime.cpp:60-76: row r sees keys
    <= past + r).

    qkv [rows, 4096] raw projections (q 2048 | k 1024 | v 1024); k_past, v_past
    [8, past, 128]. Returns (attention output [rows, 2048], new k rows [8, rows, 128],
    new v rows [8, rows, 128]).
    """
    rows = qkv.shape[0]
    q = qkv[:, :Q_WIDTH].reshape(rows, NUM_Q_HEADS, HEAD_DIM).transpose(1, 0, 2)
    k = qkv[:, Q_WIDTH:Q_WIDTH + KV_WIDTH].reshape(rows, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
    v = qkv[:, Q_WIDTH + KV_WIDTH:].reshape(rows, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
    q = rms_norm(apply_rope(q, cos, sin), lw.q_norm, eps)
    k = rms_norm(apply_rope(k, cos, sin), lw.k_norm, eps)
    keys = np.concatenate([k_past, k], axis=1)
    vals = np.concatenate([v_past, v], axis=1)
    past = k_past.shape[1]
    col = np.arange(past + rows)[None, :]
    mask = np.where(col > past + np.arange(rows)[:, None], MASK_NEG_INF, np.float32(0)).astype(np.float32)
    out = precise_sdpa(q, keys, vals, mask, scale)
    return out.transpose(1, 0, 2).reshape(rows, Q_WIDTH), k, np.ascontiguousarray(v)


def decode_from_cache(w: Weights, cfg: ModelConfig, cache: KVCache, first_token: int, max_tokens: int,
                      history, penalty: float = DEFAULT_PENALTY) -> DecodeTrace:
    """The AR loop of decode_from_embeddings (src/text_runtime.cpp:1417-1508) from a
    cache that already holds cache.length rows: first_token is the first output
    (not yet in `history`), each step embeds the last token at position
    cache.length with the 1-D RoPE, runs the decoder and selects the next token."""
    hist = list(history) + [int(first_token)]
    tr = DecodeTrace([int(first_token)], [int(first_token)], [], [], [])
    tok = int(first_token)
    for _ in range(max_tokens - 1):
        pos = cache.length
        h, _ = decoder_forward(w, cfg, w.embed[tok:tok + 1], make_decode_mask(pos), rope_rows(pos, 1, True),
                               rope_rows(pos, 1, False), cache)
        logits = lm_head(w, h)[0]
        tok, raw = select_next_token(logits, hist, penalty)
        hist.append(tok)
        tr.tokens.append(tok)
        tr.raw_top1.append(raw)
        tr.margins.append(top2_margin(logits))
    return tr


def lm_head(w: Weights, hidden: np.ndarray) -> np.ndarray:
    """Tied LM head (export/export_lm_head.py:16-24): logits = h E^T."""
    return (hidden.astype(np.float32) @ w.embed.T).astype(np.float32)


def select_next_token(logits: np.ndarray, history, penalty: float):
    """src/text_runtime.cpp:730-755. Returns (token, raw_top1).

    raw top-1 is the first index of the strict maximum; then each unique history
    id in [0, V) is penalised (s<0 ? s*pen : s/pen) and the first index of the
    maximum is returned.
    """
    scores = np.array(logits, dtype=np.float32, copy=True)
    raw = int(np.argmax(scores))
    pen = np.float32(penalty)
    ids = np.unique(np.asarray(list(history), dtype=np.int64))
    ids = ids[(ids >= 0) & (ids < scores.shape[0])]
    s = scores[ids]
    scores[ids] = np.where(s < 0, s * pen, s / pen)
    return int(np.argmax(scores)), raw


def select_logit_rows(logits: np.ndarray, initial_history, row_prefix, penalty: float) -> list:
    """src/text_runtime.cpp:757-797: row r's history is initial + row_prefix[0..r]."""
    history = list(initial_history)
    out = []
    for r in range(logits.shape[0]):
        if row_prefix is not None:
            history.append(int(row_prefix[r]))
        out.append(select_next_token(logits[r], history, penalty)[0])
    return out


def top2_margin(logits: np.ndarray) -> float:
    part = np.partition(logits.astype(np.float64), -2)
    return float(part[-1] - part[-2])


# ---------------------------------------------------------------------------
# Prompt and loops.
# ---------------------------------------------------------------------------
@dataclass
class Prompt:
    input_ids: np.ndarray        # [seq] int32
    position_ids: np.ndarray     # [4, seq] int32, axis-major
    vision_features: np.ndarray  # [n_img, 1024] fp32
    image_token_id: int = IMAGE_TOKEN_ID


TID_PROMPT_FEATURES = 9001
TID_PROMPT_IDS = 9002


def synth_ids(seed: int, tensor_id: int, count: int, vocab: int) -> np.ndarray:
    """Uniform ids in [0, vocab): splitmix64 of the same counter stream, modulo vocab."""
    base = _splitmix64_scalar((seed * _GOLDEN + tensor_id * _TID) & _M64)
    with np.errstate(over="ignore"):
        h = _splitmix64_np(np.arange(count, dtype=np.uint64) + np.uint64(base))
    return (h % np.uint64(vocab)).astype(np.int64)


def synthetic_prompt(seed: int, grid_h: int, grid_w: int, n_text: int, vocab: int,
                     image_token_id: int = IMAGE_TOKEN_ID) -> Prompt:
    """Image rows first on a grid_h x grid_w mRoPE grid, then n_text text ids.

    Image slot i: axis0 = i, axis1 = i % grid_w, axis2 = i // grid_w, axis3 = 0
    (the spatial id layout of src/prompt_builder.cpp:94-120); text slots carry
    their sequence index on all four axes. Features are N(0,1)-like from the
    counter generator; text ids are uniform in [0, vocab) and never equal the
    image token id.
    """
    n_img = grid_h * grid_w
    seq = n_img + n_text
    text = synth_ids(seed, TID_PROMPT_IDS, n_text, vocab)
    text = np.where(text == image_token_id, (text + 1) % vocab, text)
    ids = np.concatenate([np.full(n_img, image_token_id, np.int64), text]).astype(np.int32)
    pos = np.tile(np.arange(seq, dtype=np.int32), (4, 1))
    i = np.arange(n_img)
    pos[1, :n_img] = i % grid_w
    pos[2, :n_img] = i // grid_w
    pos[3, :n_img] = 0
    feats = synth_tensor_fast(seed, TID_PROMPT_FEATURES, n_img * HIDDEN, 1.0).reshape(n_img, HIDDEN)
    return Prompt(ids, pos, feats, image_token_id)


def prepare_prompt_embeddings(w: Weights, prompt: Prompt) -> np.ndarray:
    """src/text_runtime.cpp:506-568: embed ids, then inject features at image slots in order."""
    ids = prompt.input_ids.astype(np.int64)
    emb = w.embed[np.clip(ids, 0, w.embed.shape[0] - 1)].copy()
    slots = np.nonzero(ids == prompt.image_token_id)[0]
    if len(slots) != prompt.vision_features.shape[0]:
        raise ValueError("image token count mismatch")
    emb[slots] = prompt.vision_features
    return emb.astype(np.float32)


@dataclass
class DecodeTrace:
    tokens: list
    raw_top1: list
    margins: list
    logits: list          # per generated token (optional, when keep_logits)
    hidden: list


def prefill(w: Weights, cfg: ModelConfig, prompt: Prompt, capacity: int, aux: bool = False):
    """run_decoder_prefill (src/text_runtime.cpp:648-674) with the 4-axis mRoPE tables."""
    seq = prompt.input_ids.shape[0]
    emb = prepare_prompt_embeddings(w, prompt)
    cos = build_mrope(prompt.position_ids, seq, True)
    sin = build_mrope(prompt.position_ids, seq, False)
    cache = KVCache.empty(cfg.num_layers, capacity)
    hidden, aux_h = decoder_forward(w, cfg, emb, make_prefill_mask(seq), cos, sin, cache, aux)
    return hidden, cache, aux_h


def decode_ar(w: Weights, cfg: ModelConfig, prompt: Prompt, max_tokens: int, penalty: float = DEFAULT_PENALTY,
              eos_ids=(), capacity: int | None = None, keep_logits: bool = False,
              prefill_state=None) -> DecodeTrace:
    """decode_from_embeddings (src/text_runtime.cpp:1307-1521)."""
    seq = prompt.input_ids.shape[0]
    if capacity is None:
        capacity = seq + max_tokens + DFLASH_BLOCK
    if prefill_state is None:
        hidden, cache, _ = prefill(w, cfg, prompt, capacity)
    else:
        hidden, cache = prefill_state
    logits = lm_head(w, hidden[seq - 1:seq])[0]
    history = [int(t) for t in prompt.input_ids]
    tok, raw = select_next_token(logits, history, penalty)
    tr = DecodeTrace([], [], [], [], [])
    tr.margins.append(top2_margin(logits))
    if keep_logits:
        tr.logits.append(logits)
        tr.hidden.append(hidden[seq - 1].copy())
    for out_index in range(max_tokens):
        tr.tokens.append(tok)
        tr.raw_top1.append(raw)
        history.append(tok)
        if tok in eos_ids or out_index + 1 >= max_tokens:
            break
        emb = w.embed[tok:tok + 1]
        position = seq + out_index
        cos = rope_rows(position, 1, True)
        sin = rope_rows(position, 1, False)
        h, _ = decoder_forward(w, cfg, emb, make_decode_mask(position), cos, sin, cache)
        logits = lm_head(w, h)[0]
        tok, raw = select_next_token(logits, history, penalty)
        tr.margins.append(top2_margin(logits))
        if keep_logits:
            tr.logits.append(logits)
            tr.hidden.append(h[0].copy())
    return tr


def verify_block(w: Weights, cfg: ModelConfig, cache: KVCache, proposed, history_before_block,
                 penalty: float, aux: bool = False):
    """The verify half of run_dflash_block (src/text_runtime.cpp:959-1070).

    Runs the M=16 verify forward at positions context_len..context_len+15 with
    the causal-in-block mask, then select_logit_rows with the growing history.
    Returns (posterior, acceptance_length, logits, hidden), or with aux the
    block's aux hidden states (layers 1, 8, 15, 22) in place of hidden; the
    cache keeps context_len + 16 rows (the caller rolls back).
    """
    ctx = cache.length
    emb = w.embed[np.asarray(proposed, dtype=np.int64)]
    mask = build_dflash_verify_mask(ctx)
    cos = rope_rows(ctx, DFLASH_BLOCK, True)
    sin = rope_rows(ctx, DFLASH_BLOCK, False)
    hidden, aux_h = decoder_forward(w, cfg, emb, mask, cos, sin, cache, aux)
    logits = lm_head(w, hidden)
    posterior = select_logit_rows(logits, history_before_block, proposed, penalty)
    return posterior, dflash_acceptance_length(proposed, posterior), logits, (aux_h if aux else hidden)


@dataclass
class DFlashTrace:
    tokens: list
    acceptance_lengths: list
    block_count: int = 0
    drafted: int = 0
    accepted: int = 0


def decode_dflash(w: Weights, cfg: ModelConfig, prompt: Prompt, max_tokens: int, draft_fn,
                  penalty: float = DEFAULT_PENALTY, eos_ids=(), capacity: int | None = None,
                  prefill_state=None) -> DFlashTrace:
    """decode_dflash_from_embeddings (src/text_runtime.cpp:1142-1305).

    draft_fn(block_index, n_committed, current_token) -> 15 draft ids stands in
    for the draft network (src/dflash_runtime.cpp:213-290).
    """
    seq = prompt.input_ids.shape[0]
    if capacity is None:
        capacity = seq + max_tokens + 2 * DFLASH_BLOCK
    if prefill_state is None:
        hidden, cache, _ = prefill(w, cfg, prompt, capacity)
    else:
        hidden, cache = prefill_state
    logits = lm_head(w, hidden[seq - 1:seq])[0]
    history = [int(t) for t in prompt.input_ids]
    current, _ = select_next_token(logits, history, penalty)
    tr = DFlashTrace([], [])
    stop = False
    block_index = 0
    while len(tr.tokens) < max_tokens and not stop:
        ctx = cache.length
        proposed = build_dflash_block(current)
        proposed[1:] = [int(t) for t in draft_fn(block_index, len(tr.tokens), current)]
        posterior, accept, _, _ = verify_block(w, cfg, cache, proposed, history, penalty)
        if accept < 0 or accept >= DFLASH_BLOCK:
            raise RuntimeError("invalid DFlash acceptance length")
        available = accept + 1
        remaining = max_tokens - len(tr.tokens)
        committed = min(available, remaining)
        for i in range(committed):
            tok = proposed[i]
            tr.tokens.append(tok)
            if tok in eos_ids:
                committed = i + 1
                stop = True
                break
        tr.block_count += 1
        tr.drafted += DFLASH_BLOCK - 1
        tr.accepted += max(0, committed - 1)
        tr.acceptance_lengths.append(max(0, committed - 1))
        block_index += 1
        if committed < available or stop or len(tr.tokens) >= max_tokens:
            break
        cache.length = ctx + committed            # view_dflash_rows rollback
        history.extend(proposed[:committed])
        current = posterior[accept]
    return tr


TID_DRAFTS = 9003


def synthetic_drafter(greedy: list, p: float, vocab: int, seed: int):
    """Config-3 drafts: draft i of a block equals the target's greedy token with probability p.

    For block b and draft slot i in 1..15: h = splitmix64(base + 16*b + i) on
    the counter stream of (seed, TID_DRAFTS); u = (h >> 40) * 2^-24; the draft
    is greedy[n_committed + i] when u < p (and that index exists), else
    (h & 0xFFFFFFFF) % vocab. The CUDA library's device drafter uses the same
    rule, so both sides see identical drafts.
    """
    base = _splitmix64_scalar((seed * _GOLDEN + TID_DRAFTS * _TID) & _M64)
    pf = np.float32(p)

    def fn(block_index: int, n_committed: int, current: int):
        out = []
        for i in range(1, DFLASH_BLOCK):
            h = _splitmix64_scalar((base + 16 * block_index + i) & _M64)
            u = np.float32(h >> 40) * np.float32(2.0 ** -24)
            j = n_committed + i
            if u < pf and j < len(greedy):
                out.append(int(greedy[j]))
            else:
                out.append(int((h & 0xFFFFFFFF) % vocab))
        return out
    return fn


# ---------------------------------------------------------------------------
# DFlash draft network (export/dflash_export.py:88-177, the graph that
# DFlashDraftRuntime::run executes, src/dflash_runtime.cpp:213-290; called by
# run_dflash_block, src/text_runtime.cpp:880-950).
#
# target_hidden = hidden_norm(fc(concat(aux_0..3))) over the context rows; per
# draft layer: q from the 16 noise rows, k/v from the context rows followed by
# the noise rows; q_norm / k_norm BEFORE RoPE (theta 10000, positions 0..ctx+15,
# src/dflash_runtime.cpp:27-48); SDPA with the all-zero mask
# (src/dflash_runtime.cpp:50-58) and scale 1/sqrt(128); o_proj + residual;
# SwiGLU MLP + residual; final RMSNorm. The block's drafts are the argmax of the
# tied LM head on rows 1..15 (penalty 1, no history).
# The draft's layers here have the decoder's geometry (16 q heads, 8 KV heads,
# head_dim 128, the FFN width of the config); the number of layers is a parameter.
# ---------------------------------------------------------------------------
DRAFT_ROPE_THETA = 10000.0
DRAFT_SCALE = 1.0 / math.sqrt(HEAD_DIM)
TID_DRAFT_FC = 19990
TID_DRAFT_HIDDEN_NORM = 19991
TID_DRAFT_NORM = 19992
DRAFT_TID_BASE = 20000
DRAFT_TID_STRIDE = 16


@dataclass
class DraftWeights:
    fc: np.ndarray            # [1024 x 4096] (aux layers 1, 8, 15, 22 concatenated)
    hidden_norm: np.ndarray   # [1024]
    norm: np.ndarray          # [1024]
    layers: list = field(default_factory=list)   # LayerWeights


def make_draft_weights(num_layers: int, seed: int, std: float = 0.02, norm_std: float = 0.0,
                       ffn: int = FFN, bf16: bool = False) -> DraftWeights:
    """Seeded draft weights on the same counter generator (tensor ids from DRAFT_TID_BASE)."""
    def lin(tid, rows, cols):
        t = synth_tensor_fast(seed, tid, rows * cols, std).reshape(rows, cols)
        return round_bf16(t) if bf16 else t

    def norm(tid, n):
        return synth_tensor_fast(seed, tid, n, norm_std, 1.0)

    layers = []
    for li in range(num_layers):
        b = DRAFT_TID_BASE + DRAFT_TID_STRIDE * li
        layers.append(LayerWeights(
            input_norm=norm(b + J_INPUT_NORM, HIDDEN), q=lin(b + J_Q, Q_WIDTH, HIDDEN),
            k=lin(b + J_K, KV_WIDTH, HIDDEN), v=lin(b + J_V, KV_WIDTH, HIDDEN),
            q_norm=norm(b + J_Q_NORM, HEAD_DIM), k_norm=norm(b + J_K_NORM, HEAD_DIM),
            o=lin(b + J_O, HIDDEN, Q_WIDTH), post_norm=norm(b + J_POST_NORM, HIDDEN),
            gate=lin(b + J_GATE, ffn, HIDDEN), up=lin(b + J_UP, ffn, HIDDEN), down=lin(b + J_DOWN, HIDDEN, ffn)))
    return DraftWeights(fc=lin(TID_DRAFT_FC, HIDDEN, 4 * HIDDEN), hidden_norm=norm(TID_DRAFT_HIDDEN_NORM, HIDDEN),
                        norm=norm(TID_DRAFT_NORM, HIDDEN), layers=layers)


def build_dflash_rope(start: int, rows: int, use_cos: bool) -> np.ndarray:
    """build_dflash_rope (src/dflash_runtime.cpp:27-48) rows start..start+rows-1:
    angle = float(position) / powf(10000, float(2 * (d % 64)) / 128), then cosf / sinf."""
    out = np.empty((rows, HEAD_DIM), dtype=np.float32)
    den = np.empty(HEAD_DIM, dtype=np.float32)
    for d in range(HEAD_DIM):
        expo = _f32(_f32(2 * (d % (HEAD_DIM // 2))) / _f32(HEAD_DIM))
        den[d] = _f32(math.pow(DRAFT_ROPE_THETA, float(expo)))
    pos = np.arange(start, start + rows, dtype=np.int64).astype(np.float32)
    angle = (pos[:, None] / den[None, :]).astype(np.float32)
    return _cos32(angle) if use_cos else _sin32(angle)


@dataclass
class DraftCache:
    """Per draft layer K (normed, roped) / V [8, capacity, 128] of the context rows."""
    k: list
    v: list
    length: int = 0

    @staticmethod
    def empty(num_layers: int, capacity: int) -> "DraftCache":
        return DraftCache([np.zeros((NUM_KV_HEADS, capacity, HEAD_DIM), np.float32) for _ in range(num_layers)],
                          [np.zeros((NUM_KV_HEADS, capacity, HEAD_DIM), np.float32) for _ in range(num_layers)], 0)


def draft_context_rows(dw: DraftWeights, aux: list, eps: float = RMS_EPS) -> np.ndarray:
    """target_hidden = hidden_norm(fc(concat(aux_0..3))) for rows [n, 1024] each."""
    cat = np.concatenate([np.asarray(a, np.float32) for a in aux], axis=-1)
    return rms_norm(cat @ dw.fc.T, dw.hidden_norm, eps)


def draft_append_context(dw: DraftWeights, cache: DraftCache, aux: list, eps: float = RMS_EPS) -> None:
    """Append context rows: each layer's k = rope(k_norm(k_proj(th))), v = v_proj(th) at their positions."""
    th = draft_context_rows(dw, aux, eps)
    n = th.shape[0]
    start = cache.length
    cos, sin = build_dflash_rope(start, n, True), build_dflash_rope(start, n, False)
    for li, lw in enumerate(dw.layers):
        k = (th @ lw.k.T).reshape(n, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        v = (th @ lw.v.T).reshape(n, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        k = apply_rope(rms_norm(k, lw.k_norm, eps), cos, sin)
        cache.k[li][:, start:start + n] = k
        cache.v[li][:, start:start + n] = v
    cache.length = start + n


def draft_forward(dw: DraftWeights, noise: np.ndarray, cache: DraftCache, eps: float = RMS_EPS,
                  kv_round: bool = False) -> np.ndarray:
    """The draft graph for the 16 noise rows over the cached context; returns the
    final-normed hidden rows [16, 1024]. kv_round: the noise rows' keys and values
    are rounded to bf16 as a bf16 draft cache stores them."""
    m = noise.shape[0]
    ctx = cache.length
    cos, sin = build_dflash_rope(ctx, m, True), build_dflash_rope(ctx, m, False)
    h = np.asarray(noise, np.float32)
    mask = np.zeros((m, ctx + m), np.float32)
    for li, lw in enumerate(dw.layers):
        a = rms_norm(h, lw.input_norm, eps)
        q = (a @ lw.q.T).reshape(m, NUM_Q_HEADS, HEAD_DIM).transpose(1, 0, 2)
        k = (a @ lw.k.T).reshape(m, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        v = (a @ lw.v.T).reshape(m, NUM_KV_HEADS, HEAD_DIM).transpose(1, 0, 2)
        q = apply_rope(rms_norm(q, lw.q_norm, eps), cos, sin)
        k = apply_rope(rms_norm(k, lw.k_norm, eps), cos, sin)
        if kv_round:
            k, v = round_bf16(k), round_bf16(v)
        K = np.concatenate([cache.k[li][:, :ctx], k], axis=1)
        V = np.concatenate([cache.v[li][:, :ctx], v], axis=1)
        att = precise_sdpa(q, K, V, mask, DRAFT_SCALE).transpose(1, 0, 2).reshape(m, Q_WIDTH)
        h = (h + att @ lw.o.T).astype(np.float32)
        p = rms_norm(h, lw.post_norm, eps)
        g = p @ lw.gate.T
        u = p @ lw.up.T
        h = (h + ((g / (np.float32(1.0) + np.exp(-g))) * u).astype(np.float32) @ lw.down.T).astype(np.float32)
    return rms_norm(h, dw.norm, eps)


def draft_propose(w: Weights, dw: DraftWeights, cache: DraftCache, current: int, eps: float = RMS_EPS,
                  mask_token: int = DFLASH_MASK_TOKEN):
    """run_dflash_block's draft half (src/text_runtime.cpp:913-978): noise = embed([current, MASK x 15]),
    drafts = argmax of the LM head on draft rows 1..15 (penalty 1, no history).
    Returns (proposed block [16], draft hidden [16, 1024])."""
    block = build_dflash_block(current, mask_token)
    hidden = draft_forward(dw, w.embed[np.asarray(block)], cache, eps)
    logits = lm_head(w, hidden[1:])
    block[1:] = select_logit_rows(logits, [], None, 1.0)
    return block, hidden


def decode_dflash_draft(w: Weights, cfg: ModelConfig, dw: DraftWeights, prompt: Prompt, max_tokens: int,
                        penalty: float = DEFAULT_PENALTY, eos_ids=(), mask_token: int = DFLASH_MASK_TOKEN,
                        proposals: list | None = None) -> DFlashTrace:
    """decode_dflash_from_embeddings with the draft network: the draft context starts
    as the prompt's aux hidden states (run_dflash_prefill) and grows by the aux
    rows of every block's committed tokens (append_dflash_rows)."""
    seq = prompt.input_ids.shape[0]
    capacity = seq + max_tokens + 2 * DFLASH_BLOCK
    hidden, cache, aux = prefill(w, cfg, prompt, capacity, aux=True)
    dcache = DraftCache.empty(len(dw.layers), capacity)
    draft_append_context(dw, dcache, aux, cfg.rms_eps)
    logits = lm_head(w, hidden[seq - 1:seq])[0]
    history = [int(t) for t in prompt.input_ids]
    current, _ = select_next_token(logits, history, penalty)
    tr = DFlashTrace([], [])
    while len(tr.tokens) < max_tokens:
        ctx = cache.length
        proposed, _ = draft_propose(w, dw, dcache, current, cfg.rms_eps, mask_token)
        if proposals is not None:
            proposals.append(list(proposed))
        posterior, accept, _, vaux = verify_block(w, cfg, cache, proposed, history, penalty, aux=True)
        available = accept + 1
        committed = min(available, max_tokens - len(tr.tokens))
        stop = False
        for i in range(committed):
            tr.tokens.append(proposed[i])
            if proposed[i] in eos_ids:
                committed = i + 1
                stop = True
                break
        tr.block_count += 1
        tr.acceptance_lengths.append(max(0, committed - 1))
        if committed < available or stop or len(tr.tokens) >= max_tokens:
            break
        cache.length = ctx + committed
        draft_append_context(dw, dcache, [a[:committed] for a in vaux], cfg.rms_eps)
        history.extend(proposed[:committed])
        current = posterior[accept]
    return tr
