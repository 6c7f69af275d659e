"""Seeded random-init GPT-2 artifacts: weight file, config and tensor inventory.

The three files are exactly what ``model_load`` consumes (``include/model.h``):

* ``model.safetensors`` -- an 8-byte little-endian header length, a compact JSON
  header (``__metadata__`` plus one member per tensor with dtype, shape and
  data_offsets relative to the data segment), then the raw little-endian F32
  bytes with no padding.  This is the layout the reference reader parses
  (reference ``src/safetensors.h:13-33``).  The ``h.*.attn.bias`` causal-mask
  buffers of a real GPT-2 checkpoint are not written: the forward pass does not
  read them (reference ``src/model.c:6-15``).
* ``config.json`` -- the keys the loader requires (reference
  ``src/model.c:354-372``): n_layer, n_head, n_embd, n_ctx, n_positions,
  vocab_size, layer_norm_epsilon, activation_function.
* ``inventory.json`` -- one tensor object per line carrying name, dtype, shape,
  begin, end, file_offset, nbytes and orientation, plus the
  ``config_values_used`` object.  The loader finds a tensor by the line prefix
  ``{"name": "<name>",`` and cross-checks it against the weight file (reference
  ``src/model.c:166-203, 287-317, 377-389``), so the line format is kept as the
  reference's inventory tool writes it (``src/safetensors.c:539-814``).

Values: every matrix, embedding table and bias is N(0, 0.02) in float32; the
LayerNorm gains are 1 and the shifts 0 unless ``ln_affine="random"`` (used by the
tests so the affine path is exercised: gain 1 + N(0, 0.1), shift N(0, 0.1)).
Each tensor draws from its own ``numpy.random.default_rng([seed, index])`` stream,
so a file can be regenerated bit-for-bit on any machine with the same numpy.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import numpy as np

__all__ = ["GPT2Shape", "SHAPES", "tensor_specs", "write_model", "prompt_ids",
           "ensure_model", "default_cache_dir"]


@dataclass(frozen=True)
class GPT2Shape:
    name: str
    n_layer: int
    n_head: int
    n_embd: int
    n_ctx: int
    vocab_size: int
    layer_norm_epsilon: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


SHAPES = {
    # test-sized models (head_dim 64, like every GPT-2 size)
    "tiny":   GPT2Shape("tiny", 2, 2, 128, 64, 500),
    "mini":   GPT2Shape("mini", 3, 4, 256, 256, 2003),
    # the GPT-2 family
    "small":  GPT2Shape("small", 12, 12, 768, 1024, 50257),
    "medium": GPT2Shape("medium", 24, 16, 1024, 1024, 50257),
    "xl":     GPT2Shape("xl", 48, 25, 1600, 1024, 50257),
}


def tensor_specs(s: GPT2Shape):
    """(name, shape, kind) in the canonical order; kind selects the init."""
    E = s.n_embd
    out = [("wte.weight", (s.vocab_size, E), "normal"),
           ("wpe.weight", (s.n_ctx, E), "normal"),
           ("ln_f.weight", (E,), "ln_gain"),
           ("ln_f.bias", (E,), "ln_shift")]
    for l in range(s.n_layer):
        p = f"h.{l}."
        out += [(p + "ln_1.weight", (E,), "ln_gain"),
                (p + "ln_1.bias", (E,), "ln_shift"),
                (p + "attn.c_attn.weight", (E, 3 * E), "normal"),
                (p + "attn.c_attn.bias", (3 * E,), "normal"),
                (p + "attn.c_proj.weight", (E, E), "normal"),
                (p + "attn.c_proj.bias", (E,), "normal"),
                (p + "ln_2.weight", (E,), "ln_gain"),
                (p + "ln_2.bias", (E,), "ln_shift"),
                (p + "mlp.c_fc.weight", (E, 4 * E), "normal"),
                (p + "mlp.c_fc.bias", (4 * E,), "normal"),
                (p + "mlp.c_proj.weight", (4 * E, E), "normal"),
                (p + "mlp.c_proj.bias", (E,), "normal")]
    return out


def _draw(kind: str, shape, seed: int, index: int, ln_affine: str) -> np.ndarray:
    n = int(np.prod(shape))
    if kind in ("ln_gain", "ln_shift") and ln_affine == "unit":
        return np.full(n, 1.0 if kind == "ln_gain" else 0.0, dtype=np.float32)
    rng = np.random.default_rng([seed, index])
    z = rng.standard_normal(n, dtype=np.float32)
    if kind == "normal":
        return z * np.float32(0.02)
    if kind == "ln_gain":
        return np.float32(1.0) + z * np.float32(0.1)
    return z * np.float32(0.1)


def _orientation(name: str, shape, s: GPT2Shape):
    """The inventory's orientation fields for one tensor (same vocabulary as
    the reference inventory tool, src/safetensors.c:720-790)."""
    if len(shape) != 2:
        return "not_applicable", "not a 2-D weight", None
    if shape[0] == shape[1]:
        return ("unresolved_by_shape", "axes_equal",
                f"Both extents are {shape[0]}; the sibling bias matches either axis, so "
                f"shape cannot pin the reading.")
    if name.endswith(".weight") and name.startswith("h."):
        return ("axis0_input_axis1_output", "pinned_by_bias_length",
                f"The sibling bias has length {shape[1]}, equal to extent 1 only, so axis 1 "
                f"is the output axis.")
    return ("axis0_index_axis1_feature", "pinned_by_shape_arithmetic_against_config",
            f"Extent 0 is {shape[0]} ({'vocab_size' if shape[0] == s.vocab_size else 'n_ctx'}) "
            f"and extent 1 is n_embd = {shape[1]}: one row per index.")


def bf16_round(w: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, for finite values."""
    u = np.ascontiguousarray(w, dtype=np.float32).view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)


def int8_dequant(w: np.ndarray, axis: int) -> np.ndarray:
    """Per-channel symmetric absmax int8 of w, reduced along `axis` (the input
    axis), back to fp32: scale = absmax / 127, q = rint(w / scale) clamped to
    +-127 (0 for an all-zero channel), weight = q * scale -- all in fp32."""
    w = np.asarray(w, dtype=np.float32)
    scale = (np.max(np.abs(w), axis=axis, keepdims=True) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(scale > 0, np.rint(w / scale), np.float32(0)).astype(np.float32)
    q = np.clip(q, -127, 127).astype(np.float32)
    return (q * scale).astype(np.float32)


def reduce_matrix(name: str, w: np.ndarray, fmt: str) -> np.ndarray:
    """The weight a reduced format stands for, for one tensor as stored in the
    file: the five matrix kinds are reduced (wte per row; the layers' [input,
    output] matrices per output column), everything else is left as is."""
    if fmt == "f32":
        return w
    is_matrix = name == "wte.weight" or (name.startswith("h.") and name.endswith(".weight") and w.ndim == 2)
    if not is_matrix:
        return w
    if fmt == "bf16":
        return bf16_round(w)
    if fmt == "int8":
        return int8_dequant(w, axis=1 if name == "wte.weight" else 0)
    raise ValueError(fmt)


def write_model(out_dir: str, s: GPT2Shape, seed: int = 1234, ln_affine: str = "unit", fmt: str = "f32"):
    """Writes model.safetensors, config.json and inventory.json into out_dir.
    With fmt "bf16" or "int8" the matrices are the fp32 weights that reduced
    format stands for (reduce_matrix). Returns the three paths (weights,
    inventory, config)."""
    os.makedirs(out_dir, exist_ok=True)
    specs = tensor_specs(s)
    offsets, header = [], {"__metadata__": {"format": "pt"}}
    pos = 0
    for name, shape, _ in specs:
        nbytes = 4 * int(np.prod(shape))
        header[name] = {"dtype": "F32", "shape": list(shape),
                        "data_offsets": [pos, pos + nbytes]}
        offsets.append((pos, nbytes))
        pos += nbytes
    hdr = json.dumps(header, separators=(",", ":")).encode("ascii")
    data_offset = 8 + len(hdr)

    wpath = os.path.join(out_dir, "model.safetensors")
    tmp = wpath + ".partial"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for idx, (name, shape, kind) in enumerate(specs):
            w = _draw(kind, shape, seed, idx, ln_affine).reshape(shape)
            f.write(reduce_matrix(name, w, fmt).astype("<f4").tobytes())
    os.replace(tmp, wpath)

    cpath = os.path.join(out_dir, "config.json")
    cfg = {"activation_function": "gelu_new", "model_type": "gpt2",
           "n_layer": s.n_layer, "n_head": s.n_head, "n_embd": s.n_embd,
           "n_ctx": s.n_ctx, "n_positions": s.n_ctx, "vocab_size": s.vocab_size,
           "layer_norm_epsilon": s.layer_norm_epsilon,
           "init": {"seed": seed, "ln_affine": ln_affine, "std": 0.02}}
    with open(cpath, "w") as f:
        json.dump(cfg, f, indent=2)

    ipath = os.path.join(out_dir, "inventory.json")
    file_size = data_offset + pos
    lines = ["{",
             '  "note": "Tensor inventory of a seeded random-init GPT-2 weight file. '
             "'begin'/'end' are relative to the data segment; 'file_offset' is absolute.\",",
             f'  "weight_file": "{wpath}",',
             f'  "config_file": "{cpath}",',
             f'  "file_size_bytes": {file_size},',
             f'  "header_length_bytes": {len(hdr)},',
             f'  "data_segment_offset": {data_offset},',
             '  "header_metadata_present": true,',
             '  "header_metadata_format": "pt",',
             f'  "config_values_used": {{"n_embd": {s.n_embd}, "n_head": {s.n_head}, '
             f'"n_layer": {s.n_layer}, "n_ctx": {s.n_ctx}, "n_positions": {s.n_ctx}, '
             f'"vocab_size": {s.vocab_size}}},',
             f'  "tensor_count": {len(specs)},',
             '  "tensors": [']
    for i, ((name, shape, _), (begin, nbytes)) in enumerate(zip(specs, offsets)):
        orient, evidence, detail = _orientation(name, shape, s)
        rec = (f'    {{"name": "{name}", "dtype": "F32", "shape": [{", ".join(map(str, shape))}], '
               f'"begin": {begin}, "end": {begin + nbytes}, "file_offset": {data_offset + begin}, '
               f'"nbytes": {nbytes}, "orientation": "{orient}", "orientation_evidence": "{evidence}"')
        if detail:
            rec += f', "orientation_detail": "{detail}"'
        rec += "}" + ("," if i + 1 < len(specs) else "")
        lines.append(rec)
    lines += ["  ]", "}"]
    with open(ipath, "w") as f:
        f.write("\n".join(lines) + "\n")
    return wpath, ipath, cpath


def default_cache_dir() -> str:
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(os.path.dirname(here))
    return os.environ.get("TIE_CACHE_DIR", os.path.join(root, "_cache"))


def ensure_model(shape: str, seed: int = 1234, ln_affine: str = "unit", cache_dir: str | None = None,
                 fmt: str = "f32"):
    """Returns (weights, inventory, config) for a named shape, writing them once
    into the cache directory (keyed by shape, seed, LayerNorm init and, for a
    reduced-format stand-in, the format)."""
    s = SHAPES[shape]
    tag = "" if fmt == "f32" else f"_{fmt}"
    d = os.path.join(cache_dir or default_cache_dir(), f"{shape}_s{seed}_{ln_affine}{tag}")
    paths = (os.path.join(d, "model.safetensors"), os.path.join(d, "inventory.json"),
             os.path.join(d, "config.json"))
    if all(os.path.exists(p) for p in paths):
        return paths
    return write_model(d, s, seed=seed, ln_affine=ln_affine, fmt=fmt)


def prompt_ids(vocab_size: int, n_seq: int, n_tokens: int, seed: int) -> np.ndarray:
    """Seeded uniform token ids in [0, vocab_size), shape [n_seq, n_tokens], int32.
    Sequence i is the same whatever n_seq is asked for beyond it, so a shard of
    a batch can regenerate exactly its own rows."""
    out = np.empty((n_seq, n_tokens), dtype=np.int32)
    for i in range(n_seq):
        rng = np.random.default_rng([seed, i])
        out[i] = rng.integers(0, vocab_size, size=n_tokens, dtype=np.int64).astype(np.int32)
    return out
