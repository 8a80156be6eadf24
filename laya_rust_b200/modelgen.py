"""Seeded random-init Laya GGUF at the reference's hyper-parameters.

The real checkpoint is not available, so every run uses a synthetic model
written in exactly the container format the reference's converter produces
(laya-rust ``src/convert.rs:33-273``):

* metadata: every ``laya.*`` key ``ModelMeta::from_header`` checks
  (weights.rs:175-202), ``general.architecture = "laya"``, ``file_type = 1``,
  calibration temperatures 1.0 and ``temperature_by_options = "{}"``;
* 207 tensors in ``arch.weight_names()`` order with the stored shapes the
  loader pins (weights.rs:353-395), written with reversed (GGUF) dims;
* linear and embedding weights ``N(0, std)`` drawn from
  ``numpy.random.default_rng(seed)`` in that order, rounded to f16
  round-to-nearest-even; biases 0; layer-norm gammas 1 and betas 0;
* ``rope.freq_full`` / ``rope.freq_sliding`` stored as F32,
  ``1 / theta^(2j/64)`` evaluated with libm ``powf`` in f32 (convert.rs:16-21),
  theta 160000 and 10000.

``std`` defaults to 0.02 (the configuration the benchmark names).
"""
from __future__ import annotations

import ctypes
import ctypes.util
import hashlib
import os

import numpy as np

from . import arch
from . import gguf
from . import tokgen

THETA_FULL = 160000.0
THETA_SLIDING = 10000.0

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]


def rope_table(theta: float, half: int = arch.HD // 2) -> np.ndarray:
    """convert.rs:16-21: ``1.0f32 / theta.powf((2*j) as f32 / d)`` in f32."""
    d = np.float32(2 * half)
    out = np.empty(half, dtype=np.float32)
    for j in range(half):
        e = np.float32(np.float32(2 * j) / d)
        out[j] = np.float32(1.0) / np.float32(_libm.powf(np.float32(theta), e))
    return out


def _is_bias_or_norm(name: str) -> tuple[bool, float]:
    """Returns (constant?, value) for biases (0) and layer-norm gammas (1)."""
    if name.endswith(".bias") or name.endswith("in_proj_bias"):
        return True, 0.0
    if "norm" in name or name == arch.SCORER_W:
        return True, 1.0
    return False, 0.0


def write_model(path: str, seed: int = 0, std: float = 0.02) -> str:
    """Writes the random-init model to ``path``; returns the path."""
    rng = np.random.default_rng(seed)
    shapes = arch.stored_shapes()
    w = gguf.Writer()
    V = gguf.Value
    w.add_kv("general.architecture", V(gguf.STR, "laya"))
    w.add_kv("general.name", V(gguf.STR, f"Laya random-init seed {seed}"))
    w.add_kv("general.file_type", V(gguf.U32, gguf.FT_MOSTLY_F16))
    w.add_kv("general.alignment", V(gguf.U32, gguf.ALIGNMENT))
    w.add_kv("laya.weight_layout", V(gguf.STR, "ggml-canonical"))
    for key, val in [("hidden_size", arch.H), ("num_layers", arch.NLAYER),
                     ("num_heads", arch.NH), ("head_dim", arch.HD),
                     ("intermediate_size", arch.INTER), ("vocab_size", arch.NVOCAB)]:
        w.add_kv(f"laya.{key}", V(gguf.U32, val))
    w.add_kv("laya.attention_scale", V(gguf.F32, float(np.float32(arch.SCALE))))
    w.add_kv("laya.layer_norm_epsilon", V(gguf.F32, float(np.float32(arch.EPS))))
    for key, val in [("sliding_window", arch.WINDOW), ("global_layer_every", arch.GLOBAL_EVERY),
                     ("head_layers", arch.HEAD_LAYERS), ("head_intermediate_size", arch.HEAD_INTER),
                     ("act_hidden_size", arch.ACT_HIDDEN), ("act_input_features", arch.ACT_INPUT),
                     ("question_types", arch.QTYPES), ("max_len", 512), ("head_max_len", 192),
                     ("max_prefixes", 6)]:
        w.add_kv(f"laya.{key}", V(gguf.U32, val))
    w.add_kv("laya.rope_theta.full", V(gguf.F32, THETA_FULL))
    w.add_kv("laya.rope_theta.sliding", V(gguf.F32, THETA_SLIDING))
    for i in range(3):
        w.add_kv(f"laya.temperature.{i}", V(gguf.F32, 1.0))
    w.add_kv("laya.temperature_by_options", V(gguf.STR, "{}"))
    # the tokenizer travels inside the model file, as the reference's
    # converter embeds it (convert.rs:188-223; read back by lib.rs:47-57)
    w.add_kv("tokenizer.ggml.model", V(gguf.STR, "gpt2"))
    for key, name in (("bos", "[CLS]"), ("eos", "[SEP]"), ("cls", "[CLS]"), ("mask", "[MASK]"),
                      ("unknown", "[UNK]"), ("padding", "[PAD]")):
        w.add_kv(f"tokenizer.ggml.{key}_token_id", V(gguf.U32, dict((c, i) for c, i, _ in tokgen.SPECIALS)[name]))
    w.add_kv("tokenizer.huggingface.json", V(gguf.STR, tokgen.tokenizer_json(seed)))
    for name in arch.weight_names():
        shape = shapes[name]
        gdims = list(reversed(shape))
        if name in (arch.ROPE_FREQ_FULL, arch.ROPE_FREQ_SLIDING):
            theta = THETA_FULL if name == arch.ROPE_FREQ_FULL else THETA_SLIDING
            w.add_tensor(name, gdims, gguf.T_F32, gguf.f32_bytes(rope_table(theta)))
            continue
        const, val = _is_bias_or_norm(name)
        n = int(np.prod(shape))
        if const:
            data = np.full(n, val, dtype=np.float32)
        else:
            data = rng.standard_normal(n, dtype=np.float32) * np.float32(std)
        w.add_tensor(name, gdims, gguf.T_F16, gguf.f16_bytes(data))
    tmp = f"{path}.tmp{os.getpid()}"
    w.write(tmp)
    os.replace(tmp, path)
    return path


def cached_model(seed: int = 0, std: float = 0.02, directory: str | None = None) -> str:
    """Path of the seeded model, writing it once per (seed, std) into ``directory``
    (default: ``$LAYA_MODEL_CACHE`` or ``/tmp/laya-b200-models``)."""
    directory = directory or os.environ.get("LAYA_MODEL_CACHE", "/tmp/laya-b200-models")
    os.makedirs(directory, exist_ok=True)
    tag = hashlib.sha1(f"v3:{seed}:{std}".encode()).hexdigest()[:10]
    path = os.path.join(directory, f"laya-rand-s{seed}-{tag}.gguf")
    if not os.path.exists(path):
        write_model(path, seed=seed, std=std)
    return path
