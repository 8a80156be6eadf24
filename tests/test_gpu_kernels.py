"""Single-kernel numerics on the B200 against plain PyTorch fp32 references.

The tcgen05 GEMM must equal an fp32 matmul of the same f16 operands up to
summation order; the ragged attention kernel must equal an fp32
softmax(QK^T + mask)V per (sequence, head) up to its f16 output rounding.
"""
import numpy as np
import pytest
import torch

from laya_rust_b200 import engine as E

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,tile_n", [(1, 256, 64, 256), (200, 256, 64, 256), (129, 3072, 1024, 256),
                                          (1000, 512, 1024, 256), (300, 1024, 2624, 256), (2048, 1024, 4096, 256),
                                          (1, 128, 64, 128), (9872, 1024, 1024, 128), (777, 1024, 2624, 128)])
def test_gemm_matches_torch_fp32(m, n, k, tile_n):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float16)
    got = E.selftest_gemm(a, w, tile_n=tile_n)
    ref = (torch.from_numpy(a).float() @ torch.from_numpy(w).float().T).numpy()
    err = np.abs(got - ref).max()
    scale = np.abs(ref).max()
    # f32 accumulation of exact f16 products: only the summation order differs
    assert err <= 2e-5 * k ** 0.5 * max(scale, 1.0), (err, scale)


def attention_ref(qkv, lens, window):
    q = torch.from_numpy(qkv[:, :1024].astype(np.float32))
    k = torch.from_numpy(qkv[:, 1024:2048].astype(np.float32))
    v = torch.from_numpy(qkv[:, 2048:].astype(np.float32))
    out = torch.zeros(qkv.shape[0], 1024)
    s0 = 0
    for ln in lens:
        for h in range(16):
            sl = slice(h * 64, h * 64 + 64)
            qs, ks, vs = q[s0:s0 + ln, sl], k[s0:s0 + ln, sl], v[s0:s0 + ln, sl]
            sc = qs @ ks.T
            if window >= 0:
                i = torch.arange(ln)
                sc = sc.masked_fill((i[:, None] - i[None, :]).abs() > window, float("-inf"))
            out[s0:s0 + ln, sl] = torch.softmax(sc, dim=-1) @ vs
        s0 += ln
    return out.numpy()


@pytest.mark.parametrize("window", [-1, 64])
def test_attention_matches_torch_fp32(window):
    rng = np.random.default_rng(5 + window)
    lens = [1, 17, 64, 65, 128, 129, 200, 256, 300, 512]
    R = sum(lens)
    qkv = (rng.standard_normal((R, 3072)) * 0.7).astype(np.float16)
    got = E.selftest_attention(qkv, lens, window)
    ref = attention_ref(qkv, lens, window)
    err = np.abs(got - ref).max()
    # P and the output are rounded to f16 (rel 2^-11); values are O(1)
    assert err <= 4e-3, err
