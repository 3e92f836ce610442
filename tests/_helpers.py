"""Shared helpers for the parity tests: seeded synthetic inputs with the benchmark configs' shapes and
value distributions, and the tolerance checks of the bf16 path (max-abs <= 2e-2 and per-head cosine
>= 0.9999 against the fp32 reference)."""

from __future__ import annotations

import numpy as np

from oracle import attention_oracle as O

BF16_MAX_ABS = 2e-2
BF16_MIN_COS = 0.9999


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    # uint32 arithmetic cannot overflow for finite values or infinities (the largest pattern,
    # 0xFF800000, plus 0x8000 stays below 2^32)
    a = np.array(x, dtype=np.float32, copy=True).view(np.uint32)
    a += np.uint32(0x7FFF) + ((a >> np.uint32(16)) & np.uint32(1))
    a &= np.uint32(0xFFFF0000)
    return a.view(np.float32).reshape(np.shape(x))


def per_head_cosine(a: np.ndarray, b: np.ndarray, D: int) -> np.ndarray:
    """Cosine similarity per head: a, b [..., H*D] -> [H]."""
    a = np.asarray(a, np.float64).reshape(-1, a.shape[-1] // D, D).transpose(1, 0, 2).reshape(a.shape[-1] // D, -1)
    b = np.asarray(b, np.float64).reshape(-1, b.shape[-1] // D, D).transpose(1, 0, 2).reshape(b.shape[-1] // D, -1)
    num = np.sum(a * b, axis=1)
    den = np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1)
    return np.where(den > 0, num / np.maximum(den, 1e-300), 1.0)


def assert_close_bf16(got: np.ndarray, want: np.ndarray, D: int, max_abs: float = BF16_MAX_ABS,
                      min_cos: float = BF16_MIN_COS, what: str = "") -> None:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = float(np.max(np.abs(got - want))) if got.size else 0.0
    cos = per_head_cosine(got, want, D)
    assert err <= max_abs, f"{what}: max-abs error {err:.3e} > {max_abs}"
    assert float(cos.min()) >= min_cos, f"{what}: min per-head cosine {cos.min():.6f} < {min_cos}"


def joint_inputs(seed: int, B: int, h: int, w: int, Lt: int, lv_range, C: int = 1536, bf16: bool = True):
    """Seeded synthetic DiT joint-attention inputs: packed qkv
    [B, L + Lt, 3C] ~ N(0,1) (bf16-rounded when ``bf16``), norm weights, valid text lengths drawn
    uniformly from ``lv_range``, and log prompt-weight biases with w in {0.7, 1.0, 1.3}."""
    rng = np.random.default_rng(seed)
    L = h * w
    qkv = rng.standard_normal((B, L + Lt, 3 * C), dtype=np.float32)
    qkv[:, L:, :C] = 0.0   # text rows carry no queries
    if bf16:
        qkv = bf16_round(qkv)
    q_w = (1.0 + 0.2 * rng.standard_normal(96)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(96)).astype(np.float32)
    lv = rng.integers(lv_range[0], lv_range[1] + 1, size=B).astype(np.int32)
    weights = rng.choice(np.array([0.7, 1.0, 1.3], np.float32), size=(B, Lt))
    bias = np.log(weights).astype(np.float32)
    return qkv, q_w, k_w, lv, bias


def gemma_inputs(seed: int, B: int, L: int, bf16: bool = True):
    """Seeded Gemma3 layer inputs: qkv [B, L, 1536] ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    qkv = rng.standard_normal((B, L, 1536), dtype=np.float32)
    if bf16:
        qkv = bf16_round(qkv)
    q_w = (1.0 + 0.2 * rng.standard_normal(256)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(256)).astype(np.float32)
    return qkv, q_w, k_w


def lora_oracle(xr, q_or_w, scale, b, entries, N, alpha=1.0):
    """The oracle's linear (oracle.linear / linear_int8) plus LoRA side paths, with the bf16 roundings
    of the packed side path (nsa_lora_pack, the T factor) emulated.  Returns the
    result and a bound on what one bf16 step of each T element (whose rounding the GPU takes after its
    own fp32 summation order) can move it: sum_j |T[m][j]| 2^-8 |B_eff[n][j]|."""
    a_cat = np.concatenate([bf16_round(e["A"]) for e in entries])
    T = bf16_round((np.asarray(xr, np.float64) @ a_cat.astype(np.float64).T).astype(np.float32)).astype(np.float64)
    y = (O.linear_int8(xr, q_or_w, scale, acc=np.float64) if scale is not None
         else O.linear(xr, q_or_w, acc=np.float64)) * alpha
    bound = np.zeros_like(y)
    r0 = 0
    for e in entries:
        r = e["A"].shape[0]
        off = int(e.get("off", 0))
        den = alpha * (scale[off:off + e["B"].shape[0], None].astype(np.float64) if scale is not None else 1.0)
        bq = bf16_round((e["scale"] * e["B"].astype(np.float64) / den).astype(np.float32)).astype(np.float64) * den
        y[:, off:off + bq.shape[0]] += T[:, r0:r0 + r] @ bq.T
        bound[:, off:off + bq.shape[0]] += (np.abs(T[:, r0:r0 + r]) * 2 ** -8) @ np.abs(bq).T
        r0 += r
    return (y + b if b is not None else y), bound
