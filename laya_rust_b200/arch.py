"""Laya model constants and weight roles (laya-rust ``src/arch.rs``).

The constants are pinned the same way the reference pins them: the GGUF
metadata must match them exactly (weights.rs:138-222).
"""
H = 1024
NH = 16
HD = 64
NLAYER = 28
INTER = 2624
NVOCAB = 50368
SCALE = 0.3535533845424652
EPS = 1e-5
WINDOW = 64
HEAD_LAYERS = 2
HEAD_INTER = 4096
ACT_HIDDEN = 256
ACT_INPUT = H + 4
QTYPES = 3
GLOBAL_EVERY = 3
MAX_LEN = 512          # systemone.rs:4
HEAD_MAX_LEN = 192     # systemone.rs:5

CLS_ID, SEP_ID, MASK_ID, PAD_ID = 50281, 50282, 50284, 0   # tests/fixtures/*.json layout

TOK_EMB = "encoder.embeddings.tok_embeddings.weight"
TYPE_EMB = "type_emb.weight"
FINAL_NORM = "encoder.final_norm.weight"
ROPE_FREQ_FULL = "rope.freq_full"
ROPE_FREQ_SLIDING = "rope.freq_sliding"
SCORER_W, SCORER_B = "scorer.0.weight", "scorer.0.bias"
SCORER_HID, SCORER_HID_B = "scorer.1.weight", "scorer.1.bias"
SCORER_OUT, SCORER_OUT_B = "scorer.3.weight", "scorer.3.bias"
ACT_W1, ACT_B1, ACT_W2, ACT_B2 = ("act_head.0.weight", "act_head.0.bias",
                                  "act_head.2.weight", "act_head.2.bias")


def attn_norm(i):
    """arch.rs ATTN_NORM: layer 0 uses the embedding norm."""
    return "encoder.embeddings.norm.weight" if i == 0 else f"encoder.layers.{i}.attn_norm.weight"


def mlp_norm(i):
    return f"encoder.layers.{i}.mlp_norm.weight"


def wqkv(i):
    return f"encoder.layers.{i}.attn.Wqkv.weight"


def wo_attn(i):
    return f"encoder.layers.{i}.attn.Wo.weight"


def wi(i):
    return f"encoder.layers.{i}.mlp.Wi.weight"


def wo_mlp(i):
    return f"encoder.layers.{i}.mlp.Wo.weight"


HEAD_SUFFIXES = ["norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias",
                 "self_attn.in_proj_weight", "self_attn.in_proj_bias",
                 "self_attn.out_proj.weight", "self_attn.out_proj.bias",
                 "linear1.weight", "linear1.bias", "linear2.weight", "linear2.bias"]


def head(i, suffix):
    return f"head.layers.{i}.{suffix}"


def weight_names():
    """arch.rs:263-304, in load order (207 names)."""
    names = [TOK_EMB, TYPE_EMB, FINAL_NORM, ROPE_FREQ_FULL, ROPE_FREQ_SLIDING,
             SCORER_W, SCORER_B, SCORER_HID, SCORER_HID_B, SCORER_OUT, SCORER_OUT_B,
             ACT_W1, ACT_B1, ACT_W2, ACT_B2]
    for i in range(NLAYER):
        names += [attn_norm(i), mlp_norm(i), wqkv(i), wo_attn(i), wi(i), wo_mlp(i)]
    for i in range(HEAD_LAYERS):
        names += [head(i, s) for s in HEAD_SUFFIXES]
    return names


def transpose_names():
    """arch.rs:306-322: the 120 role-driven transposes for ``matmul`` weights."""
    names = []
    for i in range(NLAYER):
        names += [wqkv(i), wo_attn(i), wi(i), wo_mlp(i)]
    for i in range(HEAD_LAYERS):
        names += [head(i, "self_attn.in_proj_weight"), head(i, "linear1.weight"),
                  head(i, "linear2.weight")]
    names += [SCORER_HID, SCORER_OUT]
    return names


def is_global_layer(layer):
    return layer % GLOBAL_EVERY == 0


def stored_shapes():
    """Stored ([out, in]) shapes the loader pins (weights.rs:353-395)."""
    s = {TOK_EMB: [NVOCAB, H], TYPE_EMB: [QTYPES, H], FINAL_NORM: [H],
         ROPE_FREQ_FULL: [HD // 2], ROPE_FREQ_SLIDING: [HD // 2],
         SCORER_W: [H], SCORER_B: [H], SCORER_HID: [H, H], SCORER_HID_B: [H],
         SCORER_OUT: [1, H], SCORER_OUT_B: [1],
         ACT_W1: [ACT_HIDDEN, ACT_INPUT], ACT_B1: [ACT_HIDDEN], ACT_W2: [2, ACT_HIDDEN], ACT_B2: [2]}
    for i in range(NLAYER):
        s[attn_norm(i)] = [H]
        s[mlp_norm(i)] = [H]
        s[wqkv(i)] = [3 * H, H]
        s[wo_attn(i)] = [H, H]
        s[wi(i)] = [2 * INTER, H]
        s[wo_mlp(i)] = [H, INTER]
    for i in range(HEAD_LAYERS):
        s[head(i, "norm1.weight")] = [H]
        s[head(i, "norm1.bias")] = [H]
        s[head(i, "norm2.weight")] = [H]
        s[head(i, "norm2.bias")] = [H]
        s[head(i, "self_attn.in_proj_weight")] = [3 * H, H]
        s[head(i, "self_attn.in_proj_bias")] = [3 * H]
        s[head(i, "self_attn.out_proj.weight")] = [H, H]
        s[head(i, "self_attn.out_proj.bias")] = [H]
        s[head(i, "linear1.weight")] = [HEAD_INTER, H]
        s[head(i, "linear1.bias")] = [HEAD_INTER]
        s[head(i, "linear2.weight")] = [H, HEAD_INTER]
        s[head(i, "linear2.bias")] = [H]
    return s
