"""MLX-affine export of quantized linears and the safetensors checkpoint layout (host side).

Mirrors src/gsq_rco/gsq/export.py of the reference (same names, arguments and errors):

    native   codes uint8 [out, in] (index into quant.get_grid(bits)), scales [out, in / g]
             W[o, i] = scales[o, i // g] * grid[codes[o, i]]
    affine   W[o, i] = scale[o, i // g] * q[o, i] + bias[o, i // g], q in [0, 2^b),
             q packed least-significant-bit first into little-endian uint32 words along the
             input dimension (value j of a row at stream bits [j b, (j + 1) b))

For b >= 2, grid[c] = c - 2^(b-1), so q = c, scale = s, bias = -2^(b-1) s (export.py:13-19);
ternary is stored as 2-bit with q = c + 1. Scales and biases are stored in bf16 by default;
bias is a power-of-two multiple of the scale, so bf16(bias) = -2^(b-1) bf16(s).

The packed words are what the GPU eval reads (qgemm_packed / qdequant_packed in the CUDA
library); the reference writes them for mlx-lm's QuantizedLinear. No MLX is needed here: the
scale rounding uses torch's round-to-nearest-even casts, the safetensors file is written and read
with this module's own header code.
"""
from __future__ import annotations

import json
import math
import os
import shutil
import struct
from collections import Counter

import numpy as np
import torch

from .quant import get_grid

MLX_BITS = (2, 3, 4, 5, 6, 8)
GROUP_SIZES = (32, 64, 128)
SCALE_DTYPES = {  # name -> (torch dtype, safetensors dtype, bits per element)
    "bfloat16": (torch.bfloat16, "BF16", 16),
    "float16": (torch.float16, "F16", 16),
    "float32": (torch.float32, "F32", 32),
}
SCALE_DTYPE_CODE = {"BF16": 0, "F16": 1, "F32": 2}  # the C ABI's scale_dtype
_ITEMSIZE = {"BF16": 2, "F16": 2, "F32": 4, "U32": 4, "U8": 1, "I32": 4}
_TORCH_OF = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32,
             "I32": torch.int32, "U8": torch.uint8}
TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "vocab.json",
                   "merges.txt", "generation_config.json")

# decoder tensor names of an mlx-lm / HF Qwen2 checkpoint (reference gsq/e2e.py:26-35)
WKEY = {"q_proj": "self_attn.q_proj.weight",
        "k_proj": "self_attn.k_proj.weight",
        "v_proj": "self_attn.v_proj.weight",
        "o_proj": "self_attn.o_proj.weight",
        "gate_proj": "mlp.gate_proj.weight",
        "up_proj": "mlp.up_proj.weight",
        "down_proj": "mlp.down_proj.weight"}
BKEY = {"q_bias": "self_attn.q_proj.bias",
        "k_bias": "self_attn.k_proj.bias",
        "v_bias": "self_attn.v_proj.bias"}
NKEY = {"in_norm": "input_layernorm.weight",
        "post_norm": "post_attention_layernorm.weight"}


def mlx_bits(bits: int) -> int:
    """MLX storage width for a native bit-width (ternary is stored as 2-bit), export.py:52-58."""
    if bits == 1:
        return 2
    if bits in MLX_BITS:
        return bits
    raise ValueError(f"no MLX affine format for {bits} bits")


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """uint8 codes [out, in] (< 2^bits) -> uint32 [out, in * bits / 32] (export.py:61-73).

    Every 32 values of a row fill exactly `bits` words, so the row is cut into 32-value blocks
    and value j of a block is added at bit j * bits of the block's words (bit fields of distinct
    values do not overlap, so the sum is the bitwise OR); a field crossing a word boundary puts
    its high part at the start of the next word."""
    codes = np.asarray(codes)
    if codes.ndim != 2:
        raise ValueError("codes must be 2-D [out, in]")
    out_f, in_f = codes.shape
    if (in_f * bits) % 32:
        raise ValueError(f"{in_f} inputs x {bits} bits is not a whole number of words")
    if in_f % 32:
        # a whole number of words but ragged 32-value blocks (e.g. 8 bits x 4 inputs):
        # pad to whole blocks, then keep the words the real inputs fill
        pad = np.zeros((out_f, (in_f + 31) // 32 * 32), dtype=np.uint8)
        pad[:, :in_f] = codes
        return pack_codes(pad, bits)[:, : in_f * bits // 32]
    v = codes.astype(np.uint64).reshape(out_f, in_f // 32, 32)
    words = np.zeros((out_f, in_f // 32, bits), dtype=np.uint64)
    mask = np.uint64(0xFFFFFFFF)
    for j in range(32):
        bit = j * bits
        wi, sh = bit >> 5, bit & 31
        words[:, :, wi] += (v[:, :, j] << np.uint64(sh)) & mask
        if sh + bits > 32:
            words[:, :, wi + 1] += v[:, :, j] >> np.uint64(32 - sh)
    return np.ascontiguousarray(words.reshape(out_f, in_f // 32 * bits).astype("<u4"))


def unpack_codes(words: np.ndarray, bits: int, in_f: int) -> np.ndarray:
    """Inverse of pack_codes: uint32 [out, in * bits / 32] -> uint8 [out, in]."""
    w = np.asarray(words, dtype=np.uint32).astype(np.uint64)
    out_f = w.shape[0]
    n_pad = (in_f + 31) // 32 * 32
    if w.shape[1] * 32 < in_f * bits:
        raise ValueError("too few words for the row")
    full = np.zeros((out_f, n_pad // 32 * bits), dtype=np.uint64)
    full[:, : w.shape[1]] = w
    blk = full.reshape(out_f, n_pad // 32, bits)
    out = np.empty((out_f, n_pad // 32, 32), dtype=np.uint64)
    m = np.uint64((1 << bits) - 1)
    for j in range(32):
        bit = j * bits
        wi, sh = bit >> 5, bit & 31
        x = blk[:, :, wi] >> np.uint64(sh)
        if sh + bits > 32:
            x = x | (blk[:, :, wi + 1] << np.uint64(32 - sh))
        out[:, :, j] = x & m
    return out.reshape(out_f, n_pad)[:, :in_f].astype(np.uint8)


def to_mlx_affine(codes, scales, bits, group_size=64, scale_dtype="bfloat16"):
    """Native (codes, scales) -> (packed uint32 weight, scales, biases) in MLX affine form
    (export.py:76-91). Scales and biases are CPU torch tensors of the scale dtype."""
    codes = np.asarray(codes)
    out_f, in_f = codes.shape
    if codes.dtype != np.uint8 or codes.max(initial=0) >= len(get_grid(bits)):
        raise ValueError(f"codes must be uint8 indices below {len(get_grid(bits))} levels")
    if group_size not in GROUP_SIZES or in_f % group_size:
        raise ValueError(f"group_size {group_size} must be in {GROUP_SIZES} and divide {in_f}")
    if np.shape(scales) != (out_f, in_f // group_size):
        raise ValueError(f"scales shape {np.shape(scales)} != {(out_f, in_f // group_size)}")
    mb = mlx_bits(bits)
    q = codes + np.uint8(1) if bits == 1 else codes
    s32 = np.asarray(scales, dtype=np.float32)
    dtype = SCALE_DTYPES[scale_dtype][0]
    packed = pack_codes(q, mb)
    sc = torch.from_numpy(s32.copy()).to(dtype)
    bi = torch.from_numpy((np.float32(-(1 << (mb - 1))) * s32).astype(np.float32)).to(dtype)
    return packed, sc, bi


# ------------------------------------------------------------------- safetensors ---

class SafetensorsFile:
    """Header parser with per-tensor byte reads, so no full-file load is needed
    (export.py:94-134)."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
        self.metadata = header.pop("__metadata__", None)
        self.header = header
        self._data_start = 8 + n

    def __contains__(self, name: str) -> bool:
        return name in self.header

    def names(self) -> list:
        """Tensor names in file order."""
        return sorted(self.header, key=lambda k: self.header[k]["data_offsets"][0])

    def dtype(self, name: str) -> str:
        return self.header[name]["dtype"]

    def shape(self, name: str) -> list:
        return list(self.header[name]["shape"])

    def read_bytes(self, name: str) -> bytes:
        begin, end = self.header[name]["data_offsets"]
        with open(self.path, "rb") as f:
            f.seek(self._data_start + begin)
            return f.read(end - begin)

    def tensor_f32(self, name: str) -> np.ndarray:
        """A BF16 tensor widened exactly to float32."""
        if self.dtype(name) != "BF16":
            raise TypeError(f"{name} is {self.dtype(name)}, expected BF16")
        u = np.frombuffer(self.read_bytes(name), dtype="<u2").astype(np.uint32) << 16
        return u.view(np.float32).reshape(self.shape(name))

    def tensor(self, name: str) -> torch.Tensor:
        """A CPU torch tensor of the stored dtype (U32 words come back as int32 bit patterns)."""
        dt = self.dtype(name)
        raw = bytearray(self.read_bytes(name))
        if dt == "U32":
            return torch.frombuffer(raw, dtype=torch.int32).reshape(self.shape(name))
        return torch.frombuffer(raw, dtype=_TORCH_OF[dt]).reshape(self.shape(name))


def _tensor_bytes(t) -> tuple:
    """(safetensors dtype, bytes) of a torch tensor or numpy array."""
    if isinstance(t, np.ndarray):
        if t.dtype == np.uint32:
            return "U32", np.ascontiguousarray(t).astype("<u4").tobytes()
        if t.dtype == np.uint8:
            return "U8", t.tobytes()
        if t.dtype == np.float32:
            return "F32", np.ascontiguousarray(t).astype("<f4").tobytes()
        raise TypeError(f"unsupported array dtype {t.dtype}")
    t = t.detach().cpu().contiguous()
    name = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32",
            torch.int32: "I32", torch.uint8: "U8"}[t.dtype]
    if t.dtype == torch.bfloat16:
        return name, t.view(torch.int16).numpy().astype("<i2").tobytes()
    return name, t.numpy().tobytes()


def write_safetensors(path: str, tensors: dict, metadata: dict = None):
    """Write {name: torch tensor | numpy array} in the given order."""
    plan, blobs = [], []
    for name, t in tensors.items():
        dt, b = _tensor_bytes(t)
        plan.append((name, dt, list(t.shape), len(b)))
        blobs.append(b)
    _write_plan(path, plan, iter(blobs), metadata)


def _write_plan(path, plan, chunks, metadata):
    header = {"__metadata__": metadata} if metadata else {}
    off = 0
    for name, dtype, shape, n in plan:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + n]}
        off += n
    head = json.dumps(header, separators=(",", ":")).encode()
    head += b" " * (-len(head) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for (name, _, _, n), data in zip(plan, chunks):
            if len(data) != n:
                raise RuntimeError(f"{name}: wrote {len(data)} bytes, header says {n}")
            f.write(data)


def export_mlx_lm(out_dir, quantized, base_model_dir, scale_dtype="bfloat16"):
    """Write an mlx-lm checkpoint: model.safetensors, config.json, tokenizer files
    (export.py:137-215).

    quantized: {module path: dict(codes, scales, bits, group_size)} with the path being the
    weight name without ".weight" (e.g. "model.layers.3.mlp.down_proj"). Every other base tensor
    is copied byte for byte. Tensors are streamed one at a time."""
    if not quantized:
        raise ValueError("no quantized linears to export")
    base = SafetensorsFile(os.path.join(base_model_dir, "model.safetensors"))
    for path, q in quantized.items():
        if path + ".weight" not in base or base.shape(path + ".weight") != list(q["codes"].shape):
            raise ValueError(f"{path}: not a base linear of shape {q['codes'].shape}")
    st_dtype = SCALE_DTYPES[scale_dtype][1]

    plan = []  # (name, safetensors dtype, shape, bytes) in file order
    for name in base.names():
        path = name[: -len(".weight")] if name.endswith(".weight") else None
        if path is not None and path in quantized:
            q = quantized[path]
            out_f, in_f = q["codes"].shape
            gshape = [out_f, in_f // q["group_size"]]
            ng = gshape[0] * gshape[1] * _ITEMSIZE[st_dtype]
            plan += [(name, "U32", [out_f, in_f * mlx_bits(q["bits"]) // 32],
                      out_f * in_f * mlx_bits(q["bits"]) // 8),
                     (path + ".scales", st_dtype, gshape, ng),
                     (path + ".biases", st_dtype, gshape, ng)]
        else:
            shape = base.shape(name)
            plan.append((name, base.dtype(name), shape,
                         math.prod(shape) * _ITEMSIZE[base.dtype(name)]))

    def chunks():
        for name in base.names():
            path = name[: -len(".weight")] if name.endswith(".weight") else None
            if path is None or path not in quantized:
                yield base.read_bytes(name)
                continue
            q = quantized[path]
            packed, sc, bi = to_mlx_affine(q["codes"], q["scales"], q["bits"],
                                           q["group_size"], scale_dtype)
            yield packed.astype("<u4").tobytes()
            yield _tensor_bytes(sc)[1]
            yield _tensor_bytes(bi)[1]

    os.makedirs(out_dir, exist_ok=True)
    out_path = os.path.join(out_dir, "model.safetensors")
    _write_plan(out_path, plan, chunks(), {"format": "mlx"})

    with open(os.path.join(base_model_dir, "config.json")) as f:
        config = json.load(f)
    per_module = {p: {"group_size": q["group_size"], "bits": mlx_bits(q["bits"])}
                  for p, q in quantized.items()}
    default = {
        "group_size": Counter(v["group_size"] for v in per_module.values()).most_common(1)[0][0],
        "bits": Counter(v["bits"] for v in per_module.values()).most_common(1)[0][0],
    }
    config["quantization"] = {**default, **per_module}
    config["quantization_config"] = config["quantization"]
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(config, f, indent=2)
    for fn in TOKENIZER_FILES:
        src = os.path.join(base_model_dir, fn)
        if os.path.exists(src):
            shutil.copy2(src, out_dir)
    return out_path


def bits_report(quantized, n_quantized_params, native_scale_bits=16, export_scale_bits=16):
    """Bits per quantized weight under four accountings (export.py:218-250): code_bpp
    log2(#grid levels), native_bpp + native scale bits per group, mlx_bpp MLX bits + scale and
    bias bits per group, shard_bpp uint8 codes + fp16 scales. Raises if n_quantized_params is not
    the sum of the codes' sizes."""
    n = groups = 0
    code_bits = stored_bits = 0.0
    for q in quantized.values():
        cnt = q["codes"].size
        n += cnt
        groups += q["scales"].size
        code_bits += cnt * math.log2(len(get_grid(q["bits"])))
        stored_bits += cnt * mlx_bits(q["bits"])
    if n != n_quantized_params:
        raise ValueError(f"codes hold {n} weights, caller says {n_quantized_params}")
    native_total = code_bits + native_scale_bits * groups
    mlx_total = stored_bits + 2 * export_scale_bits * groups
    return {
        "n_params": n,
        "code_bpp": code_bits / n,
        "native_bpp": native_total / n,
        "mlx_bpp": mlx_total / n,
        "shard_bpp": (8 * n + 16 * groups) / n,
        "native_bytes": native_total / 8,
        "mlx_bytes": mlx_total / 8,
        "shard_bytes": n + 2 * groups,
    }


def module_path(layer: int, short: str) -> str:
    """The weight name without ".weight" of a block linear (export.py:256-259)."""
    if short not in WKEY:
        raise ValueError(f"unknown linear {short!r}")
    return f"model.layers.{layer}." + WKEY[short][: -len(".weight")]


def qwen2_config(cfg, n_layers: int, vocab: int) -> dict:
    """config.json of a Qwen2 checkpoint with the block shape cfg (gsq.e2e.BlockConfig)."""
    return dict(model_type="qwen2", architectures=["Qwen2ForCausalLM"], hidden_size=cfg.hidden,
                num_hidden_layers=n_layers, intermediate_size=cfg.inter,
                num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv,
                rms_norm_eps=cfg.eps, vocab_size=vocab, max_position_embeddings=32768,
                rope_theta=cfg.theta, tie_word_embeddings=True, torch_dtype="bfloat16")


def save_base_checkpoint(model, out_dir) -> str:
    """Write a bf16 Qwen2 checkpoint (model.safetensors + config.json, mlx-lm tensor names) of a
    QwenModel held on the GPU: the base that export_mlx_lm copies from."""
    os.makedirs(out_dir, exist_ok=True)
    tensors = {"model.embed_tokens.weight": model.embed}
    for L, W in enumerate(model.layers):
        p = f"model.layers.{L}."
        for k, name in NKEY.items():
            tensors[p + name] = W[k]
        for k, name in WKEY.items():
            tensors[p + name] = W[k]
        for k, name in BKEY.items():
            tensors[p + name] = W[k]
    tensors["model.norm.weight"] = model.norm
    # file order: sorted names, as mx.save_safetensors writes them
    tensors = {k: tensors[k] for k in sorted(tensors)}
    path = os.path.join(out_dir, "model.safetensors")
    write_safetensors(path, tensors, {"format": "mlx"})
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(qwen2_config(model.cfg, len(model.layers), model.embed.shape[0]), f, indent=2)
    return path
