#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own decoder definition,
``TextDecoderExternalRopeKVWrapper`` from export/text_decoder_kv.py, on CPU
fp32 over a random-init ``transformers`` HunYuanDenseV1Model whose weights are
the seeded synthetic set (oracle/hy_oracle.py::make_weights). The tied LM head
is ``h @ E^T`` as in export/export_lm_head.py:16-24. The host-side token
selection (src/text_runtime.cpp:730-755), verify mask
(src/dflash_runtime.cpp:60-76) and acceptance rule (src/dflash_runtime.cpp:78-95)
are restated here independently of the oracle, in plain Python loops.

This needs the reference checkout, so it runs only where it is mounted; the
outputs (small .npz files) are committed next to this script. The RoPE tables
come from the oracle's build_mrope, which tests/test_oracle_golden.py pins to
the reference's own known-answer values (tests/text_rope_test.cpp:8-34).

Usage: python tests/golden/make_golden.py [--reference /path/to/HunyuanOCR-ncnn]
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))
import hy_oracle as O  # noqa: E402

CASES = {
    # name: (layers, vocab, grid_h, grid_w, n_text, ar_tokens, norm_std, seed)
    "small_2l": (2, 4096, 4, 6, 16, 12, 0.1, 11),
    "full_24l": (24, O.VOCAB, 24, 32, 256, 8, 0.0, 0),
}


def ref_select_next_token(logits: np.ndarray, history, penalty: float):
    scores = [float(x) for x in np.asarray(logits, dtype=np.float32)]
    pen = np.float32(penalty)
    raw = 0
    for i in range(1, len(scores)):
        if scores[i] > scores[raw]:
            raw = i
    s32 = np.asarray(scores, dtype=np.float32)
    for tok in set(int(t) for t in history):
        if 0 <= tok < len(s32):
            v = s32[tok]
            s32[tok] = v * pen if v < 0 else v / pen
    best = 0
    for i in range(1, len(s32)):
        if s32[i] > s32[best]:
            best = i
    return best, raw


def ref_verify_mask(past: int, block: int) -> np.ndarray:
    key_len = past + block
    m = np.zeros((block, key_len), np.float32)
    for r in range(block):
        for c in range(past + r + 1, key_len):
            m[r, c] = -1.0e38
    return m


def ref_acceptance(proposed, posterior) -> int:
    if not proposed or len(proposed) != len(posterior):
        return -1
    a = 0
    for i in range(1, len(proposed)):
        if proposed[i] != posterior[i - 1]:
            break
        a += 1
    return a


def build_model(w: O.Weights, layers: int, vocab: int):
    from transformers.models.hunyuan_v1_dense import HunYuanDenseV1Config, HunYuanDenseV1Model
    cfg = HunYuanDenseV1Config(hidden_size=O.HIDDEN, intermediate_size=O.FFN, num_hidden_layers=layers,
                               num_attention_heads=O.NUM_Q_HEADS, num_key_value_heads=O.NUM_KV_HEADS,
                               head_dim=O.HEAD_DIM, vocab_size=vocab, rms_norm_eps=O.RMS_EPS,
                               hidden_act="silu", attention_bias=False, tie_word_embeddings=True)
    with torch.device("meta"):
        model = HunYuanDenseV1Model(cfg)
    sd = {"embed_tokens.weight": w.embed, "norm.weight": w.final_norm}
    for i, lw in enumerate(w.layers):
        p = f"layers.{i}."
        sd.update({
            p + "input_layernorm.weight": lw.input_norm,
            p + "self_attn.q_proj.weight": lw.q, p + "self_attn.k_proj.weight": lw.k,
            p + "self_attn.v_proj.weight": lw.v, p + "self_attn.o_proj.weight": lw.o,
            p + "self_attn.query_layernorm.weight": lw.q_norm,
            p + "self_attn.key_layernorm.weight": lw.k_norm,
            p + "post_attention_layernorm.weight": lw.post_norm,
            p + "mlp.gate_proj.weight": lw.gate, p + "mlp.up_proj.weight": lw.up,
            p + "mlp.down_proj.weight": lw.down,
        })
    model.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, strict=True, assign=True)
    return model.float().eval()


def t4(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x))[None, None]


def make_case(name: str, reference: Path, out_dir: Path) -> None:
    layers, vocab, gh, gw, n_text, ar_tokens, norm_std, seed = CASES[name]
    sys.path.insert(0, str(reference / "export"))
    from text_decoder_kv import TextDecoderExternalRopeKVWrapper

    cfg = O.ModelConfig(num_layers=layers, vocab=vocab)
    w = O.make_weights(cfg, seed, std=0.02, norm_std=norm_std)
    image_token = O.IMAGE_TOKEN_ID if vocab > O.IMAGE_TOKEN_ID else vocab - 3
    prompt = O.synthetic_prompt(seed, gh, gw, n_text, vocab, image_token)
    seq = int(prompt.input_ids.shape[0])
    wrapper = TextDecoderExternalRopeKVWrapper.from_decoder(build_model(w, layers, vocab))
    del w.layers

    emb = O.prepare_prompt_embeddings(w, prompt)
    cos = O.build_mrope(prompt.position_ids, seq, True)
    sin = O.build_mrope(prompt.position_ids, seq, False)
    mask = np.where(np.arange(seq)[None, :] > np.arange(seq)[:, None], np.float32(-1.0e38), np.float32(0.0))
    E = torch.from_numpy(w.embed)
    with torch.inference_mode():
        hidden, caches = wrapper.prefill(torch.from_numpy(emb)[None], t4(mask.astype(np.float32)), t4(cos), t4(sin))
        logits0 = (hidden[0, -1:] @ E.T)[0].numpy()
        history = [int(t) for t in prompt.input_ids]
        tok, raw = ref_select_next_token(logits0, history, O.DEFAULT_PENALTY)
        prefill_caches = [(k.clone(), v.clone()) for k, v in caches]
        tokens, raws, tops_i, tops_v, full_logits = [], [], [], [], [logits0]
        step_logits = logits0
        for out_index in range(ar_tokens):
            tokens.append(tok)
            raws.append(raw)
            top = np.argsort(-step_logits, kind="stable")[:16]
            tops_i.append(top)
            tops_v.append(step_logits[top])
            history.append(tok)
            if out_index + 1 >= ar_tokens:
                break
            pos = seq + out_index
            c1 = O.rope_rows(pos, 1, True)
            s1 = O.rope_rows(pos, 1, False)
            h, caches = wrapper.decode(E[tok:tok + 1][None], t4(np.zeros((1, pos + 1), np.float32)),
                                       t4(c1), t4(s1), caches)
            step_logits = (h[0] @ E.T)[0].numpy()
            if out_index == 0:
                full_logits.append(step_logits)
            tok, raw = ref_select_next_token(step_logits, history, O.DEFAULT_PENALTY)
        # Sample the layer-0 and last-layer caches after the AR run (16-head expanded layout).
        k0 = caches[0][0][0].numpy()
        kl = caches[-1][0][0].numpy()
        vl = caches[-1][1][0].numpy()
        L = k0.shape[1]
        rows = np.array([0, 1, seq - 1, L - 1])
        cache_samples = np.stack([k0[:, rows, :], kl[:, rows, :], vl[:, rows, :]])

        # DFlash verify block from the prefill state: proposed[0] = first token,
        # slots 1..5 follow the AR greedy continuation, the rest are drafted ids.
        proposed = [tokens[0]] + tokens[1:6] + [int(x) for x in O.synth_ids(seed, 77, 10, vocab)]
        proposed = proposed[:O.DFLASH_BLOCK]
        vmask = ref_verify_mask(seq, O.DFLASH_BLOCK)
        vc = O.rope_rows(seq, O.DFLASH_BLOCK, True)
        vs = O.rope_rows(seq, O.DFLASH_BLOCK, False)
        vh, _ = wrapper.decode(E[torch.tensor(proposed)][None], t4(vmask), t4(vc), t4(vs), prefill_caches)
        vlogits = (vh[0] @ E.T).numpy()
        vhist = [int(t) for t in prompt.input_ids]
        posterior = []
        for r in range(O.DFLASH_BLOCK):
            vhist.append(proposed[r])
            posterior.append(ref_select_next_token(vlogits[r], vhist, O.DEFAULT_PENALTY)[0])
        accept = ref_acceptance(proposed, posterior)
        vtop_i = np.argsort(-vlogits, axis=1, kind="stable")[:, :8]
        vtop_v = np.take_along_axis(vlogits, vtop_i, axis=1)

    np.savez_compressed(
        out_dir / f"{name}.npz",
        layers=layers, vocab=vocab, grid_h=gh, grid_w=gw, n_text=n_text, seed=seed, norm_std=norm_std,
        image_token_id=image_token, attn_scale=1.0 / math.sqrt(O.HEAD_DIM), penalty=O.DEFAULT_PENALTY,
        input_ids=prompt.input_ids, position_ids=prompt.position_ids,
        feature_checksum=np.float64(prompt.vision_features.astype(np.float64).sum()),
        prefill_last_hidden=hidden[0, -1].numpy(),
        tokens=np.array(tokens, np.int32), raw_top1=np.array(raws, np.int32),
        top16_idx=np.array(tops_i, np.int32), top16_val=np.array(tops_v, np.float32),
        logits_first2=np.stack(full_logits[:2]).astype(np.float32) if vocab <= 8192 else np.zeros(0, np.float32),
        cache_rows=rows, cache_samples=cache_samples.astype(np.float32),
        verify_proposed=np.array(proposed, np.int32), verify_posterior=np.array(posterior, np.int32),
        verify_accept=np.int32(accept), verify_top8_idx=vtop_i.astype(np.int32),
        verify_top8_val=vtop_v.astype(np.float32),
    )
    print(f"{name}: tokens={tokens} accept={accept} posterior={posterior}")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="root of the HunyuanOCR-ncnn source tree (its export/ directory is imported)")
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    args = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for name in args.cases:
        make_case(name, args.reference, HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
