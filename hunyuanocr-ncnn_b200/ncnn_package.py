"""Model-package writer: decoder, tied-table and DFlash draft weights in the layout of the
reference's exported ncnn files (models/README.md; export/export_text_embed.py,
export/export_text_decoder_kv.py with export/add_kvcache.py, export/export_lm_head.py and
export/dflash_export.py, run through pnnx with fp16=0, export/_common.py:80-98).

The library reads such a package with hy_ctx_create_from_package / hy_draft_load_package
(csrc/hy_package.cpp). This writer serialises weights that are already in memory (the
seeded synthetic weights of the tests, or a converted checkpoint) into that layout:

* `<root>/text_embed/text_embed.ncnn.{param,bin}`: an Embed layer over the tied table
  [vocab x 1024] (a tagged array);
* `<root>/lm_head/lm_head.ncnn.param`: the LM head's Gemm, whose constant B the reference
  reads from text_embed.ncnn.bin (the tied table is stored once);
* `<root>/text_decoder/text_decoder_kv.ncnn.{param,bin}`: per decoder layer, in the order the
  exported graph computes them, the input RMSNorm, the q/k/v Gemms, the query / key
  RMSNorms, the SDPA with the KV-cache inputs add_kvcache.py adds, o_proj, the post-attention
  RMSNorm and the gate / up / down Gemms; then the final norm. Weightless layers (Input,
  Split, RotaryEmbed, SDPA, BinaryOp, Swish) sit between them as in an export;
* `<root>/dflash/dflash.ncnn.{param,bin}` (optional): fc, hidden_norm, the draft layers (k
  and v projections appear twice, for the context rows and the noise rows, as the traced
  draft graph calls them twice) and norm.

ncnn's model-bin layout: the weighted layers' arrays follow each other in .param order; a
Gemm's constant B, an InnerProduct's and an Embed's weight start with a 4-byte storage tag
(0: fp32 follows, 0x01306B47: fp16 follows, padded to 4 bytes); RMSNorm gammas and
MemoryData constants are raw fp32. Options select the variants an export may produce:
`fp16` (tagged arrays stored as fp16), `linear` ("gemm" or "innerproduct") and `norm`
("rmsnorm", or "memorydata": the norm weight folded into a constant named
<module>.weight).
"""

from __future__ import annotations

import os

import numpy as np

MAGIC = 7767517
TAG_FP32 = 0
TAG_FP16 = 0x01306B47


class _Net:
    """One .param / .bin pair being written."""

    def __init__(self, fp16: bool, linear: str, norm: str):
        self.lines: list[str] = []
        self.blob_count = 0
        self.bin = bytearray()
        self.fp16, self.linear, self.norm = fp16, linear, norm
        self._n = 0

    def blob(self) -> str:
        self._n += 1
        return f"b{self._n}"

    def layer(self, type_: str, name: str, inputs, outputs, params: dict | None = None) -> None:
        p = " ".join(f"{k}={v}" for k, v in (params or {}).items())
        self.lines.append(f"{type_:<24} {name:<40} {len(inputs)} {len(outputs)} {' '.join(list(inputs) + list(outputs))}"
                          + (f" {p}" if p else ""))
        self.blob_count += len(outputs)

    def tagged(self, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
        if self.fp16:
            self.bin += np.uint32(TAG_FP16).tobytes()
            h = a.astype(np.float16).tobytes()
            self.bin += h + b"\0" * ((-len(h)) % 4)
        else:
            self.bin += np.uint32(TAG_FP32).tobytes()
            self.bin += a.tobytes()

    def raw(self, a: np.ndarray) -> None:
        self.bin += np.ascontiguousarray(a, dtype=np.float32).reshape(-1).tobytes()

    def linear_layer(self, name: str, x: str, w: np.ndarray) -> str:
        out = self.blob()
        n, k = w.shape
        if self.linear == "gemm":
            self.layer("Gemm", name, [x], [out], {10: -1, 2: 0, 3: 1, 4: 0, 5: 1, 6: 0, 7: 0, 8: n, 9: k})
        else:
            self.layer("InnerProduct", name, [x], [out], {0: n, 1: 0, 2: n * k})
        self.tagged(w)
        return out

    def rms_norm(self, name: str, x: str, w: np.ndarray, eps: float = 1e-5) -> str:
        out = self.blob()
        if self.norm == "rmsnorm":
            self.layer("RMSNorm", name, [x], [out], {0: w.size, 1: f"{eps:e}", 2: 1})
            self.raw(w)
        else:
            c = self.blob()
            self.layer("MemoryData", f"{name}.weight", [], [c], {0: w.size})
            self.raw(w)
            self.layer("RMSNorm", name, [x, c], [out], {0: w.size, 1: f"{eps:e}", 2: 0})
        return out

    def write(self, directory: str, stem: str, with_bin: bool = True) -> None:
        os.makedirs(directory, exist_ok=True)
        with open(os.path.join(directory, f"{stem}.ncnn.param"), "w") as f:
            f.write(f"{MAGIC}\n{len(self.lines)} {self.blob_count}\n" + "\n".join(self.lines) + "\n")
        if with_bin:
            with open(os.path.join(directory, f"{stem}.ncnn.bin"), "wb") as f:
                f.write(bytes(self.bin))


def _layer(net: _Net, i: int, lw, x: str, prefix: str, mask: str, ck: str, cv: str, kv_twice: str | None = None,
           qk_norms: tuple = ("query_layernorm", "key_layernorm")) -> str:
    """One decoder (or draft) layer in the order of the exported graph; returns the output blob."""
    a, res = net.blob(), net.blob()
    net.layer("Split", f"splitncnn_{prefix}{i}_0", [x], [a, res])
    h = net.rms_norm(f"{prefix}layers.{i}.input_layernorm", a, lw.input_norm)
    h1, h2, h3 = net.blob(), net.blob(), net.blob()
    net.layer("Split", f"splitncnn_{prefix}{i}_1", [h], [h1, h2, h3])
    q = net.linear_layer(f"{prefix}layers.{i}.self_attn.q_proj", h1, lw.q)
    k = net.linear_layer(f"{prefix}layers.{i}.self_attn.k_proj", h2, lw.k)
    v = net.linear_layer(f"{prefix}layers.{i}.self_attn.v_proj", h3, lw.v)
    if kv_twice is not None:   # the draft graph projects the context rows with the same modules
        net.linear_layer(f"{prefix}layers.{i}.self_attn.k_proj_1", kv_twice, lw.k)
        net.linear_layer(f"{prefix}layers.{i}.self_attn.v_proj_1", kv_twice, lw.v)
    qr, kr = net.blob(), net.blob()
    net.layer("RotaryEmbed", f"rope_{prefix}{i}", [q, k], [qr, kr])
    qn = net.rms_norm(f"{prefix}layers.{i}.self_attn.{qk_norms[0]}", qr, lw.q_norm)
    kn = net.rms_norm(f"{prefix}layers.{i}.self_attn.{qk_norms[1]}", kr, lw.k_norm)
    att, ok_, ov_ = net.blob(), net.blob(), net.blob()
    net.layer("SDPA", f"sdpa_{prefix}{i}", [qn, kn, v, mask, ck, cv], [att, ok_, ov_],
              {5: 1, 6: "0.0883883", 7: 1})
    o = net.linear_layer(f"{prefix}layers.{i}.self_attn.o_proj", att, lw.o)
    x2 = net.blob()
    net.layer("BinaryOp", f"add_{prefix}{i}_0", [res, o], [x2], {0: 0})
    b, res2 = net.blob(), net.blob()
    net.layer("Split", f"splitncnn_{prefix}{i}_2", [x2], [b, res2])
    m = net.rms_norm(f"{prefix}layers.{i}.post_attention_layernorm", b, lw.post_norm)
    m1, m2 = net.blob(), net.blob()
    net.layer("Split", f"splitncnn_{prefix}{i}_3", [m], [m1, m2])
    g = net.linear_layer(f"{prefix}layers.{i}.mlp.gate_proj", m1, lw.gate)
    u = net.linear_layer(f"{prefix}layers.{i}.mlp.up_proj", m2, lw.up)
    sg, act = net.blob(), net.blob()
    net.layer("Swish", f"silu_{prefix}{i}", [g], [sg])
    net.layer("BinaryOp", f"mul_{prefix}{i}", [sg, u], [act], {0: 2})
    d = net.linear_layer(f"{prefix}layers.{i}.mlp.down_proj", act, lw.down)
    out = net.blob()
    net.layer("BinaryOp", f"add_{prefix}{i}_1", [res2, d], [out], {0: 0})
    return out


def write_package(root: str, weights, draft=None, fp16: bool = False, linear: str = "gemm",
                  norm: str = "rmsnorm") -> None:
    """weights: .embed [vocab x 1024], .final_norm, .layers[i].{input_norm, q, k, v, q_norm,
    k_norm, o, post_norm, gate, up, down} (nn.Linear layout); draft (optional): .fc
    [1024 x 4096], .hidden_norm, .norm, .layers like the decoder's."""
    if linear not in ("gemm", "innerproduct") or norm not in ("rmsnorm", "memorydata"):
        raise ValueError("linear must be gemm or innerproduct, norm rmsnorm or memorydata")
    vocab, hidden = weights.embed.shape

    emb = _Net(fp16, linear, norm)
    ids, e = emb.blob(), emb.blob()
    emb.layer("Input", "in0", [], [ids])
    emb.layer("Embed", "embed_tokens", [ids], [e], {0: hidden, 1: vocab, 2: 0, 3: vocab * hidden})
    emb.tagged(weights.embed)
    emb.write(os.path.join(root, "text_embed"), "text_embed")

    lm = _Net(fp16, linear, norm)   # constant B read from text_embed.ncnn.bin
    hs, logits = lm.blob(), lm.blob()
    lm.layer("Input", "in0", [], [hs])
    lm.layer("Gemm", "lm_head", [hs], [logits], {10: -1, 2: 0, 3: 1, 4: 0, 5: 1, 6: 0, 7: 0, 8: vocab, 9: hidden})
    lm.write(os.path.join(root, "lm_head"), "lm_head", with_bin=False)

    dec = _Net(fp16, linear, norm)
    x, mask, c0, s0, c1, s1 = (dec.blob() for _ in range(6))
    for n, b in zip(("in0", "in1", "in2", "in3", "in4", "in5"), (x, mask, c0, s0, c1, s1)):
        dec.layer("Input", n, [], [b])
    caches = [dec.blob() for _ in range(2 * len(weights.layers))]
    dec.layer("Input", "kv_cache", [], caches)
    for i, lw in enumerate(weights.layers):
        x = _layer(dec, i, lw, x, "", mask, caches[2 * i], caches[2 * i + 1])
    dec.rms_norm("norm", x, weights.final_norm)
    dec.write(os.path.join(root, "text_decoder"), "text_decoder_kv")

    if draft is not None:
        dr = _Net(fp16, linear, norm)
        noise, t1, t2, t3, t4, cos, sin, dmask = (dr.blob() for _ in range(8))
        for n, b in zip(("in0", "in1", "in2", "in3", "in4", "in5", "in6", "in7"),
                        (noise, t1, t2, t3, t4, cos, sin, dmask)):
            dr.layer("Input", n, [], [b])
        cat = dr.blob()
        dr.layer("Concat", "cat_target", [t1, t2, t3, t4], [cat], {0: -1})
        th = dr.rms_norm("hidden_norm", dr.linear_layer("fc", cat, draft.fc), draft.hidden_norm)
        y = noise
        for i, lw in enumerate(draft.layers):
            ck, cv = dr.blob(), dr.blob()
            dr.layer("MemoryData", f"empty_cache_{i}", [], [ck], {0: 0})
            dr.raw(np.zeros(1, np.float32))
            dr.layer("MemoryData", f"empty_cache_v_{i}", [], [cv], {0: 0})
            dr.raw(np.zeros(1, np.float32))
            y = _layer(dr, i, lw, y, "", dmask, ck, cv, kv_twice=th, qk_norms=("q_norm", "k_norm"))
        dr.rms_norm("norm", y, draft.norm)
        dr.write(os.path.join(root, "dflash"), "dflash")
