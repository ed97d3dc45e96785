"""Seeded inputs of the decoder-layer parity fixtures (BASELINE config 3 and
the FFN half of config 4), shared by tests/golden/make_layer_golden.py and
the tests that read tests/golden/layer_golden.npz.

Config 3: qkv = q|k|v of 16 + 16 + 48 heads x 128, a rolling conv state
[3][10240] and depthwise conv weights [10240][4]; beta = sigmoid(b) with b ~
N(0,1); the decay g = exp(-softplus(a) * 0.1), i.e. the reference's gate
softplus(a + dt_bias) * A with dt_bias = 0 and A = -0.1; GDN state
[48][128][128] ~ N(0, 0.02); z ~ N(0,1) and the gated-norm weight [128].
FFN: the residual [5120], the post-attention norm weight and the gate/up
projections [17408].
"""
from __future__ import annotations

import hashlib

import numpy as np

QK_HEADS, VALUE_HEADS, HEAD_DIM = 16, 48, 128
KEY_DIM, VALUE_DIM = QK_HEADS * HEAD_DIM, VALUE_HEADS * HEAD_DIM
QKV_ROWS = 2 * KEY_DIM + VALUE_DIM
HIDDEN, FFN_DIM = 5120, 17408
EPS = np.float32(1e-6)
SEED = 20260302


def _g(seed: int, n: int, scale: float = 1.0, offset: float = 0.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(n) * scale + offset).astype(np.float32)


def layer_inputs() -> dict[str, np.ndarray]:
    return {
        "qkv": _g(SEED + 1, QKV_ROWS),
        "conv_state_in": _g(SEED + 2, 3 * QKV_ROWS),
        "conv_weight": _g(SEED + 3, 4 * QKV_ROWS, 0.5),
        "beta_raw": _g(SEED + 4, VALUE_HEADS),
        "alpha_raw": _g(SEED + 5, VALUE_HEADS),
        "dt_bias": np.zeros(VALUE_HEADS, np.float32),
        "ssm_a": np.full(VALUE_HEADS, -0.1, np.float32),
        "gdn_state_in": _g(SEED + 6, VALUE_HEADS * HEAD_DIM * HEAD_DIM, 0.02),
        "z": _g(SEED + 7, VALUE_DIM),
        "ssm_norm_weight": _g(SEED + 8, HEAD_DIM, 0.1, 1.0),
    }


def ffn_inputs() -> dict[str, np.ndarray]:
    return {
        "residual": _g(SEED + 11, HIDDEN),
        "post_norm_weight": _g(SEED + 12, HIDDEN, 0.1, 1.0),
        "ffn_gate": _g(SEED + 13, FFN_DIM),
        "ffn_up": _g(SEED + 14, FFN_DIM),
    }


def digest(a: np.ndarray) -> str:
    """sha256 of an array's float32 bytes: pins arrays too large to store."""
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def sample_index(n: int, count: int = 4096, seed: int = 5) -> np.ndarray:
    return np.sort(np.random.default_rng(seed).choice(n, size=min(n, count), replace=False)).astype(np.int64)
