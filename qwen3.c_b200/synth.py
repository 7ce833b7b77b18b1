"""Seeded synthetic inputs shared by the tests, the CPU oracle runs and bench.py.

A counter-based generator (splitmix64 -> uniform -> Box-Muller) keyed by
(config, tensor name, request index), so the CPU oracle and the CUDA kernels
consume bit-identical inputs on any machine and numpy version. Shapes and
value distributions follow the benchmark configurations of the qwen3.c
token-mixing path (gated GQA decode/prefill, GatedDeltaNet decode/prefill);
no public dataset is involved.
"""
import numpy as np

_GOLD = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _fnv1a(text: str) -> int:
    h = 0xCBF29CE484222325
    for ch in text.encode():
        h ^= ch
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def seed_of(config: str, name: str, req: int = 0) -> int:
    """Stable 64-bit seed for one tensor of one request of one config."""
    return _fnv1a(f"{config}/{name}/{req}")


def _splitmix(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        idx = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed) + idx * _GOLD
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, shape, lo=0.0, hi=1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u = (_splitmix(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def normal(seed: int, shape, std=1.0, mean=0.0) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = _splitmix(seed, 2 * m)
    u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    u1 = np.maximum(u[0::2], 1e-300)
    u2 = u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(2.0 * np.pi * u2)
    out[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (mean + std * out[:n]).astype(np.float32).reshape(shape)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (b >> np.uint32(16)) & np.uint32(1)
    r = (b + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
