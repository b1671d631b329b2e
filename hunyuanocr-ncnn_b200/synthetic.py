"""Synthetic prompts for benchmarks (no checkpoint or images are available).

Layout of the benchmark prompt: image-embedding rows first, on a grid_h x grid_w
mRoPE grid (slot i: axis0 = i, axis1 = i % grid_w, axis2 = i // grid_w,
axis3 = 0, the spatial id layout of src/prompt_builder.cpp:94-120), then
uniform text ids carrying their sequence index on all four axes. Values come
from the same splitmix64 counter streams as the device weight generator
(features ~N(0,1) by a 4-term Irwin-Hall sum, ids uniform modulo the vocab).
"""

from __future__ import annotations

import math

import numpy as np

IMAGE_TOKEN_ID = 120120   # src/prompt_builder.cpp:8
TID_PROMPT_FEATURES = 9001
TID_PROMPT_IDS = 9002
_M64 = (1 << 64) - 1


def _mix(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def _mix_np(z: np.ndarray) -> np.ndarray:
    z = z + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _stream(seed: int, tensor_id: int, count: int) -> np.ndarray:
    base = _mix((seed * 0x9E3779B97F4A7C15 + tensor_id * 0xD1B54A32D192ED03) & _M64)
    with np.errstate(over="ignore"):
        return _mix_np(np.arange(count, dtype=np.uint64) + np.uint64(base))


def normal_like(seed: int, tensor_id: int, count: int, std: float) -> np.ndarray:
    h = _stream(seed, tensor_id, count)
    s = ((h & np.uint64(0xFFFF)) + ((h >> np.uint64(16)) & np.uint64(0xFFFF))
         + ((h >> np.uint64(32)) & np.uint64(0xFFFF)) + (h >> np.uint64(48)))
    c = (s.astype(np.int64) - 131070).astype(np.float32)
    return c * np.float32(float(std) * math.sqrt(3.0) / 65536.0)


def synthetic_prompt(seed: int, grid_h: int, grid_w: int, n_text: int, vocab: int,
                     image_token_id: int = IMAGE_TOKEN_ID):
    """Returns (input_ids [seq] int32, position_ids [4, seq] int32, features [n_img, 1024] f32, image_token_id)."""
    n_img = grid_h * grid_w
    seq = n_img + n_text
    text = (_stream(seed, TID_PROMPT_IDS, n_text) % np.uint64(vocab)).astype(np.int64)
    text = np.where(text == image_token_id, (text + 1) % vocab, text)
    ids = np.concatenate([np.full(n_img, image_token_id, np.int64), text]).astype(np.int32)
    pos = np.tile(np.arange(seq, dtype=np.int32), (4, 1))
    i = np.arange(n_img)
    pos[1, :n_img] = i % grid_w
    pos[2, :n_img] = i // grid_w
    pos[3, :n_img] = 0
    feats = normal_like(seed, TID_PROMPT_FEATURES, n_img * 1024, 1.0).reshape(n_img, 1024)
    return ids, pos, feats, image_token_id
